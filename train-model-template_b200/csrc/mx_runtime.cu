// Host runtime shared by all entry points: error strings, status plumbing, device queries and
// the TMA tensor-map encoder (driver entry point fetched through the runtime, no -lcuda).
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "mx_common.cuh"
#include "mx_runtime.h"

__device__ int g_mx_dev_error = 0;

static thread_local char t_err[512] = "";

void mx_set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
}

int mx_cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MXM_OK;
  mx_set_last_error("%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
  return MXM_ERR_CUDA;
}

int mx_launch_status(const char* what) { return mx_cuda_status(cudaGetLastError(), what); }

int* mx_dev_error_ptr() {
  static int* cache[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!cache[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_mx_dev_error) == cudaSuccess) cache[dev] = static_cast<int*>(p);
  }
  return cache[dev];
}

static std::atomic<unsigned long long> g_launches{0};

void mx_note_launch(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }

extern "C" unsigned long long mxm_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" int mxm_version(void) { return MXM_ABI_VERSION; }

extern "C" const char* mxm_last_error(void) { return t_err; }

extern "C" int mxm_device_error(int* code, int clear) {
  if (!code) {
    mx_set_last_error("mxm_device_error: null output pointer");
    return MXM_ERR_ARG;
  }
  int v = 0;
  int st = mx_cuda_status(cudaMemcpyFromSymbol(&v, g_mx_dev_error, sizeof(int)), "read device error flag");
  if (st) return st;
  *code = v;
  if (clear && v) {
    const int zero = 0;
    st = mx_cuda_status(cudaMemcpyToSymbol(g_mx_dev_error, &zero, sizeof(int)), "clear device error flag");
    if (st) return st;
  }
  if (v) {
    static const char* what[] = {"", "producer", "MMA issue", "epilogue", "MMA accumulator hand-back"};
    mx_set_last_error("a kernel gave up a bounded wait (device error code %d: %s)", v,
                      v == MX_DEV_TIMEOUT_SELFTEST ? "self-test wait" : (v > 0 && v < 5 ? what[v] : "unknown"));
    return MXM_ERR_DEVICE;
  }
  return MXM_OK;
}

// One CTA waits on an mbarrier that nothing arrives on, with a bounded wait of limit_ns: the wait runs
// out, records MX_DEV_TIMEOUT_SELFTEST in the device error flag and the kernel returns.
__global__ void k_selftest_wait(uint64_t limit_ns, int* err) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  mbar_wait_ns(&bar, 0, err, MX_DEV_TIMEOUT_SELFTEST, limit_ns);
}

extern "C" int mxm_selftest_wait(int64_t limit_ns, void* stream) {
  MX_CHECK_ARG(limit_ns > 0 && limit_ns <= 100000000, "mxm_selftest_wait: limit_ns must be in (0, 1e8] (got %lld)",
               (long long)limit_ns);
  int* err = mx_dev_error_ptr();
  if (!err) {
    mx_set_last_error("mxm_selftest_wait: no device error flag on the current device");
    return MXM_ERR_CUDA;
  }
  k_selftest_wait<<<1, 32, 0, (cudaStream_t)stream>>>((uint64_t)limit_ns, err);
  mx_note_launch();
  return mx_launch_status("mxm_selftest_wait");
}

cudaError_t mx_smem_attr(const void* fn, size_t bytes) {
  struct Entry {
    const void* fn;
    int dev;
    size_t bytes;
  };
  static std::mutex mu;
  static Entry tab[256];
  static int n = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < n; ++i)
      if (tab[i].fn == fn && tab[i].dev == dev && tab[i].bytes >= bytes) return cudaSuccess;
  }
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess) {
    std::lock_guard<std::mutex> lock(mu);
    if (n < 256) tab[n++] = Entry{fn, dev, bytes};
  }
  return e;
}

extern "C" int mxm_num_sms(void) {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encoder() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Tiled tensor map of rank 2 or 3: dims / box innermost first, strides (bytes) of dims 1 .. rank-1.
static int make_tmap(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, int rank, const uint64_t* dims,
                     const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn enc = get_encoder();
  if (!enc) {
    mx_set_last_error("cuTensorMapEncodeTiled unavailable from the driver");
    return MXM_ERR_CUDA;
  }
  bool aligned = ((uintptr_t)base & 15) == 0;
  for (int i = 0; i + 1 < rank; ++i) aligned = aligned && (strides[i] & 15) == 0;
  if (!aligned) {
    mx_set_last_error("TMA operand not 16-byte aligned (base %p, stride %llu bytes)", base,
                      (unsigned long long)strides[0]);
    return MXM_ERR_ARG;
  }
  // The encoder is a driver call and needs a current context; the runtime binds the primary context to
  // a thread only at that thread's first runtime call that needs it, and a fresh thread (autograd's
  // device thread runs the backward) may reach this first.  cudaSetDevice binds it (no synchronization).
  static thread_local bool bound = false;
  if (!bound) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaSetDevice(dev);
    if (e != cudaSuccess) return mx_cuda_status(e, "bind the device context for cuTensorMapEncodeTiled");
    bound = true;
  }
  cuuint64_t d[3], st[2];
  cuuint32_t b[3], estr[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    if (i + 1 < rank) st[i] = strides[i];
  }
  CUresult r = enc(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), d, st, b, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    mx_set_last_error("cuTensorMapEncodeTiled failed (%d) for a rank-%d map, dims [%llu x %llu], box [%u x %u]",
                      (int)r, rank, (unsigned long long)dims[rank - 1], (unsigned long long)dims[0], box[rank - 1],
                      box[0]);
    return MXM_ERR_CUDA;
  }
  return MXM_OK;
}

int mx_make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t elem_bytes, const void* base,
                    uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                    uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  (void)elem_bytes;
  const uint64_t dims[2] = {inner, outer}, strides[1] = {row_stride_bytes};
  const uint32_t box[2] = {box_inner, box_outer};
  return make_tmap(map, dtype, base, 2, dims, strides, box, swizzle);
}

int mx_make_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t (&dims)[3],
                    const uint64_t (&strides_bytes)[2], const uint32_t (&box)[3], CUtensorMapSwizzle swizzle) {
  return make_tmap(map, dtype, base, 3, dims, strides_bytes, box, swizzle);
}
