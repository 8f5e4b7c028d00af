"""CPU oracle of the DeepSeek-V4 W4A8 MoE layer -- TEST INFRASTRUCTURE ONLY.

numpy restatement of the reference's arithmetic for this layer (paths relative
to the reference project root):

* gate -- ``Gate.forward`` (vendor/deepseek_v4_ref/inference/model.py:569-589):
  fp32 logits ``linear(x.float(), W.float())``, ``sqrt(softplus(.))`` scores
  (torch's softplus: x above 20 passes through), ``+ bias`` for the choice only,
  ``topk`` (sorted, torch's CPU order via ``oracle.topk``) or, on a hash-routed
  layer, ``tid2eid[input_ids]``; the unbiased scores gathered, divided by their
  sum, times ``route_scale``.
* experts -- ``Expert.forward`` (model.py:592-611) whose w1/w3/w2 are fp4
  ``Linear``s (model.py:114-121): ``act_quant`` per 1x128 with the power-of-two
  scale ``2^ceil(log2(amax/448))`` (``scale_fmt`` "ue8m0", amax floored at 1e-4;
  engines/deepseek_v4/v4_kernels_cpu.py:68-100), ``fp4_gemm`` = dequantised e4m3
  activations times e2m1 weights with one e8m0 scale per 32 along K, fp32
  products summed in fp32, output bf16 (v4_kernels_cpu.py:166-172); gate/up to
  fp32, ``up`` clamped to +-swiglu_limit and ``gate`` to <= swiglu_limit,
  ``silu(gate) * up``, times the routing weight, to bf16, then w2 the same way.
* shared expert -- the same Expert with fp8 ``Linear``s (e4m3 weights, one e8m0
  scale per 128x128 block; ``fp8_gemm``, v4_kernels_cpu.py:158-164), no weight.
* combine -- ``MoE.forward`` (model.py:634-649): fp32 ``y``, routed experts in
  ascending id, ``y[idx] += expert(...)``: an expert named by several slots of
  one token (possible only with ``tid2eid``) contributes only its LAST slot --
  advanced-index ``+=`` writes every duplicate back and the last write wins
  (engines/deepseek_v4/v4_moe_grouped.py:623-631 restates the same rule); then
  the shared expert; ``y`` to bf16.

fp32 matrix products here run through numpy's BLAS, whose summation order is
not torch's: results agree with the reference to fp32 rounding, not bit for bit
(the committed fixtures pin the tolerance).
"""
import numpy as np

from .dsv3 import e4m3_values
from .fp import E2M1_VALUES, f32_to_e4m3_bits, round_bf16
from .topk import topk_row

F32 = np.float32
INV448 = F32(1.0 / 448.0)


def sqrtsoftplus(v):
    """torch.nn.functional.softplus(v).sqrt() in fp32 (beta 1, threshold 20)."""
    v = np.asarray(v, F32)
    sp = np.where(v > F32(20.0), v, np.log1p(np.exp(np.minimum(v, F32(20.0)))).astype(F32)).astype(F32)
    return np.sqrt(sp).astype(F32)


def gate(x, router_w, bias, top_k, route_scale, tid2eid=None, input_ids=None):
    """x float32 [M, H] (bf16 values), router_w float32 [E, H] (bf16 values), bias
    float32 [E] -> (ids int64 [M, k], weights float32 [M, k], logits float32 [M, E])."""
    logits = (np.asarray(x, F32) @ np.asarray(router_w, F32).T).astype(F32)
    scores = sqrtsoftplus(logits)
    M = scores.shape[0]
    if tid2eid is not None:
        ids = np.asarray(tid2eid, np.int64)[np.asarray(input_ids, np.int64)].reshape(M, top_k)
    else:
        choice = (scores + np.asarray(bias, F32)).astype(F32)
        ids = np.array([topk_row(row, top_k, sorted=True) for row in choice], dtype=np.int64)
        ids = ids.reshape(M, top_k)
    wts = np.zeros((M, top_k), dtype=F32)
    for t in range(M):
        w = scores[t, ids[t]].astype(F32)
        s = F32(0.0)
        for v in w:
            s = F32(s + v)
        wts[t] = ((w / s).astype(F32) * F32(route_scale)).astype(F32)
    return ids, wts, logits


def round_scale_ue8m0(amax):
    """2^ceil(log2(amax * (1/448))), exact at powers of two (frexp)."""
    v = (np.asarray(amax, F32) * INV448).astype(F32)
    mant, ex = np.frexp(v)
    return np.ldexp(F32(1.0), np.where(mant == 0.5, ex - 1, ex)).astype(F32)


def act_quant(x):
    """act_quant(x, 128, "ue8m0"): float32 [n, K] -> (e4m3 values as float32 [n, K],
    power-of-two scales float32 [n, K/128])."""
    x = np.asarray(x, F32)
    n, K = x.shape
    z = x.reshape(n, K // 128, 128)
    amax = np.maximum(np.abs(z).max(-1), F32(1e-4)).astype(F32)
    s = round_scale_ue8m0(amax)
    q = np.clip((z / s[..., None]).astype(F32), -448.0, 448.0)
    return e4m3_values(f32_to_e4m3_bits(q)).reshape(n, K), s


def e8m0(bits):
    """e8m0 bytes -> float32 powers of two."""
    return np.ldexp(F32(1.0), np.asarray(bits, np.int32) - 127).astype(F32)


def dequant_fp4(packed, scales):
    """uint8 [N, K/2] packed e2m1 (low nibble = even K) + e8m0 [N, K/32] -> float32 [N, K]."""
    b = np.asarray(packed, np.uint8)
    N = b.shape[0]
    v = np.stack([E2M1_VALUES[b & 0x0F], E2M1_VALUES[b >> 4]], axis=-1).reshape(N, -1)
    return (v * np.repeat(e8m0(scales), 32, axis=1)).astype(F32)


def fp4_gemm(qa, sa, w_packed, w_scales):
    """dequant(A) [n, K] @ dequant(W fp4)^T -> bf16 values (float32) [n, N]."""
    n, K = qa.shape
    da = (qa.reshape(n, K // 128, 128) * sa[..., None]).astype(F32).reshape(n, K)
    return round_bf16((da @ dequant_fp4(w_packed, w_scales).T).astype(F32))


def fp8_gemm(qa, sa, w_bits, w_scales_e8m0):
    """dequant(A) [n, K] @ dequant(W e4m3, 128x128 e8m0 blocks)^T -> bf16 values [n, N]."""
    n, K = qa.shape
    da = (qa.reshape(n, K // 128, 128) * sa[..., None]).astype(F32).reshape(n, K)
    wv = e4m3_values(w_bits)
    N = wv.shape[0]
    sw = np.repeat(np.repeat(e8m0(w_scales_e8m0), 128, axis=0)[:N], 128, axis=1)[:, :K]
    return round_bf16((da @ (wv * sw).astype(F32).T).astype(F32))


def _swiglu(gate_v, up_v, weights, limit):
    if limit > 0:
        up_v = np.clip(up_v, -limit, limit).astype(F32)
        gate_v = np.minimum(gate_v, F32(limit)).astype(F32)
    h = ((gate_v / (F32(1.0) + np.exp(-gate_v))).astype(F32) * up_v).astype(F32)
    if weights is not None:
        h = (np.asarray(weights, F32)[:, None] * h).astype(F32)
    return round_bf16(h)


def expert_forward(x, w13, s13, w2, s2, weights, limit):
    """A routed fp4 Expert on its token rows: w13 uint8 [2I, H/2] ([w1; w3]), s13
    e8m0 [2I, H/32], w2 uint8 [H, I/2], s2 e8m0 [H, I/32]."""
    I = np.asarray(w2).shape[1] * 2
    qa, sa = act_quant(x)
    gate_v = fp4_gemm(qa, sa, w13[:I], s13[:I])
    up_v = fp4_gemm(qa, sa, w13[I:], s13[I:])
    h = _swiglu(gate_v, up_v, weights, limit)
    qh, sh = act_quant(h)
    return fp4_gemm(qh, sh, w2, s2)


def shared_forward(x, w13, s13, w2, s2, limit):
    """The fp8 shared Expert: w13 e4m3 bytes [2I, H], s13 e8m0 [2I/128, H/128]."""
    I = np.asarray(w2).shape[1]
    qa, sa = act_quant(x)
    w13 = np.asarray(w13, np.uint8)
    gate_v = fp8_gemm(qa, sa, w13[:I], s13[: I // 128])
    up_v = fp8_gemm(qa, sa, w13[I:], s13[I // 128:])
    h = _swiglu(gate_v, up_v, None, limit)
    qh, sh = act_quant(h)
    return fp8_gemm(qh, sh, np.asarray(w2, np.uint8), s2)


def keep_last_of_each(ids_row):
    """Slots of one token that survive the duplicate-index ``y[idx] +=``: a slot is
    dropped when a later slot names the same expert."""
    ids_row = list(ids_row)
    return [all(ids_row[j] != ids_row[i] for j in range(i + 1, len(ids_row)))
            for i in range(len(ids_row))]


def moe_forward(x, ids, wts, expert, shared, limit):
    """MoE.forward: ``expert(e)`` -> (w13, s13, w2, s2) numpy, ``shared()`` likewise.
    Returns bf16 values (float32) [M, H]."""
    x = np.asarray(x, F32)
    ids = np.asarray(ids)
    y = np.zeros_like(x, dtype=F32)
    for e in sorted(set(int(v) for v in ids.ravel())):
        rows, slots = np.nonzero(ids == e)            # torch.where: row-major (token, slot)
        out = expert_forward(x[rows], *expert(e), np.asarray(wts)[rows, slots], limit)
        base = y[rows].copy()                         # y[idx] += v reads every row first,
        for i, r in enumerate(rows):                  # then writes back: the last write wins
            y[r] = (base[i] + out[i]).astype(F32)
    if shared is not None:
        y = (y + shared_forward(x, *shared(), limit)).astype(F32)
    return round_bf16(y)


def expert_bytes(hidden, inter):
    """HBM bytes of one routed fp4 expert: packed w1, w3, w2 and their e8m0 scales."""
    w = 3 * hidden * inter
    return w // 2 + w // 32


def shared_bytes(hidden, inter):
    """HBM bytes of the fp8 shared expert: e4m3 weights and their block scales (as
    the kernel bank holds them: one fp32 per 128x128 block)."""
    w = 3 * hidden * inter
    return w + 4 * (w // (128 * 128))


def touched_bytes(ids, num_tokens, hidden, inter, num_experts):
    """Algorithmic HBM bytes of one layer call: distinct routed experts, the shared
    expert, router (bf16 [E, H] + fp32 bias), x and y (bf16)."""
    distinct = len(set(int(v) for v in np.asarray(ids).ravel()))
    return (distinct * expert_bytes(hidden, inter) + shared_bytes(hidden, inter) +
            num_experts * hidden * 2 + num_experts * 4 + 2 * num_tokens * hidden * 2)
