"""CPU oracle of the dense FP8 linear -- TEST INFRASTRUCTURE ONLY.

numpy restatement of the reference's ``linear`` on a float8_e4m3fn weight
(vendor/deepseek_v4_ref/inference/model.py:114-124), paths relative to the
reference project root:

* act_quant per 1x128 (vendor/deepseek_v4_ref/inference/kernel.py:40-125,
  engines/deepseek_v4/v4_kernels_cpu.py:68-104): ``scale_fmt`` None -> scale
  amax/448 (``oracle.dsv3.act_quant``), "ue8m0" -> 2^ceil(log2(amax/448))
  (``oracle.v4.act_quant``), amax floored at 1e-4, values saturated to e4m3.
* fp8_gemm_kernel's per-element chain (kernel.py:203-255): for each 128-wide K
  block kb in ascending order, D_kb = the block's dot product of e4m3 values,
  Scale_C = s_x[m, kb] * s_w[n // 128, kb] in fp32, and
  ``C_local_accum += C_local * Scale_C`` -- one fp32 fused multiply-add; bf16 at
  the end.

Here D_kb is exact (products of e4m3 values have 8 significant bits and a
128-term sum spans fewer than 53 bits, so the float64 sum is exact in any order)
and rounded once to fp32; the multiply-add is evaluated in float64 (the product
of two fp32 values is exact there) and rounded to fp32, which matches a true fma
except for double rounding when the sum needs more than 53 bits.  A tensor core
may round D_kb differently from the exact partial: GPU parity carries that as
its tolerance.
"""
import numpy as np

from . import dsv3, v4
from .dsv3 import e4m3_values
from .fp import round_bf16

F32 = np.float32


def act_quant(x, scale_fmt=None):
    """float32 [n, K] -> (e4m3 values float32 [n, K], scales float32 [n, K/128])."""
    return v4.act_quant(x) if scale_fmt == "ue8m0" else dsv3.act_quant(x)


def weight_scales(w_scale):
    """fp32 [N/128, K/128], or e8m0 bytes (uint8) -> their fp32 powers of two."""
    s = np.asarray(w_scale)
    return v4.e8m0(s) if s.dtype == np.uint8 else s.astype(F32)


def fp8_gemm_chain(qa, sa, w_bits, w_scale):
    """The reference chain: qa e4m3 values [n, K], sa fp32 [n, K/128], w_bits uint8
    e4m3 [N, K], w_scale [N/128, K/128] -> bf16 values (float32) [n, N]."""
    qa = np.asarray(qa, F32)
    n, K = qa.shape
    wv = e4m3_values(w_bits).astype(np.float64)
    N = wv.shape[0]
    sw = np.repeat(weight_scales(w_scale), 128, axis=0)[:N]
    qa64 = qa.astype(np.float64)
    acc = np.zeros((n, N), F32)
    for kb in range(K // 128):
        blk = slice(kb * 128, (kb + 1) * 128)
        d = (qa64[:, blk] @ wv[:, blk].T).astype(F32)
        sc = (np.asarray(sa, F32)[:, kb][:, None] * sw[:, kb][None, :]).astype(F32)
        acc = (d.astype(np.float64) * sc.astype(np.float64) + acc.astype(np.float64)).astype(F32)
    return round_bf16(acc)


def linear(x, w_bits, w_scale, scale_fmt=None):
    """linear(x, W): x float32 [n, K] (bf16 values) -> bf16 values (float32) [n, N]."""
    qa, sa = act_quant(np.asarray(x, F32), scale_fmt)
    return fp8_gemm_chain(qa, sa, w_bits, w_scale)


def weight_bytes(N, K, e8m0=False):
    """Algorithmic bytes a call reads for the weight: e4m3 values + block scales."""
    return N * K + (N // 128) * (K // 128) * (1 if e8m0 else 4)
