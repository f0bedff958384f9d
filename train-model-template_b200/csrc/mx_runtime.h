// Host-side helpers shared by the .cu translation units (not part of the public ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mxmlp.h"

void mx_set_last_error(const char* fmt, ...);
int mx_cuda_status(cudaError_t e, const char* what);
int mx_launch_status(const char* what);

// Counts kernel launches made by this library (host side), read with mxm_launch_count().
void mx_note_launch(int n = 1);

// cudaFuncSetAttribute(fn, MaxDynamicSharedMemorySize, bytes) once per (kernel, device): later calls with
// no larger size return at once (the attribute is a per-context property of the kernel).
cudaError_t mx_smem_attr(const void* fn, size_t bytes);

// Device address of the device-side error flag on the current device (nullptr if unavailable).
int* mx_dev_error_ptr();

// 2-D tiled tensor map over a row-major [outer, inner] matrix.
int mx_make_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t elem_bytes, const void* base,
                    uint64_t inner, uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner,
                    uint32_t box_outer, CUtensorMapSwizzle swizzle);

// 3-D tiled tensor map: dims and box innermost first, strides (bytes) of dims 1 and 2.
int mx_make_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, const uint64_t (&dims)[3],
                    const uint64_t (&strides_bytes)[2], const uint32_t (&box)[3], CUtensorMapSwizzle swizzle);

#define MX_CHECK_ARG(cond, ...)        \
  do {                                 \
    if (!(cond)) {                     \
      mx_set_last_error(__VA_ARGS__);  \
      return MXM_ERR_ARG;              \
    }                                  \
  } while (0)

static inline bool mx_aligned(const void* p, uintptr_t a) { return ((uintptr_t)p % a) == 0; }
