"""CPU oracle of the Kimi-K3 routed experts -- TEST INFRASTRUCTURE ONLY.

numpy restatement of ``KimiSparseMoeBlock.moe_infer`` (vendor/kimi_k3_ref/
modeling_kimi_linear.py:841-875) on experts whose weights are the checkpoint's
MXFP4 tensors (``mxfp4-pack-quantized``: e2m1 nibbles, low nibble first, one e8m0
scale per 32 along K; engines/kimi_k3/k3_moe_mxfp4.py:326-340), paths relative to
the reference project root:

* each expert is ``KimiBlockSparseMLP.forward`` (:242-268) with ``hidden_act``
  "situ": ``w1(x)`` and ``w3(x)`` as bf16 Linear outputs (fp32 products summed in
  fp32, rounded once to bf16), ``SituAndMul`` (:64-80) in fp32 --
  beta*tanh(g/beta)*sigmoid(g) times linear_beta*tanh(u/linear_beta) (or u when
  linear_beta is None) -- to bf16, then ``w2`` the same way;
* the fold: every (token, slot) row in bf16, cast to fp32, times the slot's
  routing weight, summed over the k slots in slot order, to bf16.

The dequantised MXFP4 weights are exact in bf16 and fp32; matrix products run
through numpy's BLAS, whose summation order is not torch's, so results agree
with the reference to fp32 rounding (the committed fixtures pin it).
"""
import numpy as np

from .fp import round_bf16
from .v4 import dequant_fp4

F32 = np.float32


def situ(g, u, beta, linear_beta):
    """SituAndMul on fp32 gate / up values -> bf16 values (float32)."""
    g = np.asarray(g, F32)
    u = np.asarray(u, F32)
    b = F32(beta)
    a = ((b * np.tanh((g / b).astype(F32))).astype(F32) *
         (F32(1.0) / (F32(1.0) + np.exp(-g).astype(F32))).astype(F32)).astype(F32)
    if linear_beta is not None:
        lb = F32(linear_beta)
        u = (lb * np.tanh((u / lb).astype(F32))).astype(F32)
    return round_bf16((a * u).astype(F32))


def expert_forward(x, w1, s1, w3, s3, w2, s2, beta, linear_beta):
    """One expert on its token rows: x float32 [n, H] (bf16 values) -> bf16 values [n, H]."""
    x = np.asarray(x, F32)
    g = round_bf16((x @ dequant_fp4(w1, s1).T).astype(F32))
    u = round_bf16((x @ dequant_fp4(w3, s3).T).astype(F32))
    h = situ(g, u, beta, linear_beta)
    return round_bf16((h @ dequant_fp4(w2, s2).T).astype(F32))


def moe_infer(x, topk_ids, topk_weight, expert, beta, linear_beta):
    """x float32 [M, H]; topk_ids int [M, k]; topk_weight float32 [M, k]; expert(e) ->
    (w1, s1, w3, s3, w2, s2) as numpy uint8 -> y bf16 values (float32) [M, H]."""
    x = np.asarray(x, F32)
    ids = np.asarray(topk_ids)
    w = np.asarray(topk_weight, F32)
    M, k = ids.shape
    rows = np.zeros((M, k, x.shape[1]), F32)
    for e in sorted(set(int(v) for v in ids.ravel())):
        t, s = np.nonzero(ids == e)
        rows[t, s] = expert_forward(x[t], *expert(e), beta, linear_beta)
    acc = (rows[:, 0] * w[:, 0:1]).astype(F32)
    for s in range(1, k):
        acc = (acc + (rows[:, s] * w[:, s:s + 1]).astype(F32)).astype(F32)
    return round_bf16(acc)


def expert_bytes(hidden, inter):
    """MXFP4 bytes of one expert (w1, w3, w2 with their e8m0 scales)."""
    return 3 * hidden * inter // 2 + 3 * hidden * inter // 32
