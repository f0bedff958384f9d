"""Generates tests/golden/scale_rule_b200.npz ON A B200: the E8M0 scale code the reference's quantizer
arithmetic produces on the GPU for every non-negative bf16 block abs-max.

The reference computes a block's scale in Triton as ``descale = amax / 448.0`` (fp32 division as Triton
lowers it for the GPU) followed by the PTX ``cvt.rp.satfinite.ue8m0x2.f32`` (scripts/mxfp8.py:61-63).
The CPU golden fixtures (make_golden.py) ran that code under Triton's interpreter, where the division is
numpy's IEEE division; whether the GPU lowering gives the same quotient where it matters -- amax = 7 * 2^k,
whose quotient 2^(k-6) is exact, so a result one ulp high would round the scale up a power of two -- is a
property of the compiled GPU code.  This script restates those two operations in a small Triton kernel
(test infrastructure only; the library has no Triton) and runs it on all 32,768 non-negative bf16 values
(plus +inf and NaN) as block maxima, recording the quotient's bits and the scale code.  The reference
sources themselves are not needed: only the two operations above are.

    python tests/golden/make_scale_rule_b200.py      # on a GPU box; writes the .npz next to this file
"""
import os
import sys

import numpy as np
import torch
import triton
import triton.language as tl

HERE = os.path.dirname(os.path.abspath(__file__))


@triton.jit
def _scale_kernel(a_ptr, d_ptr, e_ptr, n, BLOCK: tl.constexpr):
    i = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
    m = i < n
    amax = tl.load(a_ptr + i, mask=m, other=0.0)
    descale = amax / 448.0
    e = tl.inline_asm_elementwise(asm="cvt.rp.satfinite.ue8m0x2.f32 $0, 0.0, $1;", constraints="=h,r",
                                  args=[descale], dtype=tl.uint16, is_pure=True, pack=1).to(tl.uint8)
    tl.store(d_ptr + i, descale, mask=m)
    tl.store(e_ptr + i, e, mask=m)


def main():
    assert torch.cuda.is_available(), "run this on a GPU box"
    bits = np.arange(0, 0x8000, dtype=np.uint32)                 # every non-negative bf16 pattern
    amax = (bits << np.uint32(16)).view(np.float32)
    a = torch.from_numpy(amax.copy()).cuda()
    d = torch.empty_like(a)
    e = torch.empty(a.shape, dtype=torch.uint8, device="cuda")
    _scale_kernel[(triton.cdiv(a.numel(), 1024),)](a, d, e, a.numel(), BLOCK=1024)
    torch.cuda.synchronize()
    out = os.path.join(HERE, "scale_rule_b200.npz")
    np.savez_compressed(out, amax_bits=bits.astype(np.uint16), descale_bits=d.cpu().numpy().view(np.uint32),
                        e=e.cpu().numpy(), device=np.array(torch.cuda.get_device_name()),
                        triton=np.array(triton.__version__), torch=np.array(torch.__version__))
    with np.errstate(invalid="ignore"):
        ieee = (amax / np.float32(448.0)).astype(np.float32).view(np.uint32)
    diff = np.flatnonzero(d.cpu().numpy().view(np.uint32) != ieee)
    print(f"wrote {out}: {len(diff)} quotients differ from IEEE division", file=sys.stderr)


if __name__ == "__main__":
    main()
