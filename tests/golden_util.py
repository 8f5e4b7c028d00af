"""Shared fixture loading for the oracle and GPU parity tests.

Inputs of each fixture are regenerated with ``flyai_b200.synth`` from the stored
seed (the small cases also carry their inputs verbatim) and verified against the
fixture's SHA-256 digest before use.
"""
import hashlib

import numpy as np
import torch

from flyai_b200 import synth
from oracle import gpt_oss as og
from oracle.fp import bf16_bits_to_f32, f32_to_bf16_bits


def _tie_heavy_router(layer, seed):
    g = torch.Generator().manual_seed(seed + 77)
    E, H = layer.router_w.shape
    layer.router_w = (torch.randint(-2, 3, (E, H), generator=g).float() * 2.0 ** -6).bfloat16()
    layer.router_b = torch.zeros(E).bfloat16()
    return layer


def _digest(layer, x):
    h = hashlib.sha256()
    for t in (layer.router_w, layer.router_b, layer.w13_blocks, layer.w13_scales, layer.w13_bias,
              layer.w2_blocks, layer.w2_scales, layer.w2_bias, x):
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def load_case(path):
    f = dict(np.load(path))
    shape = dict(num_experts=int(f["num_experts"]), top_k=int(f["top_k"]),
                 hidden=int(f["hidden"]), inter=int(f["inter"]))
    seed, M = int(f["seed"]), int(f["tokens"])
    layer = synth.make_gpt_oss_layer(**shape, seed=seed)
    if int(f["ties"]):
        layer = _tie_heavy_router(layer, seed)
    x = synth.make_tokens(M, shape["hidden"], seed=seed)
    if int(f["ties"]):
        x = torch.round(x.float() * 2).bfloat16()
    return dict(fixture=f, layer=layer, x=x, tokens=M, shape=shape,
                digest_ok=_digest(layer, x) == str(f["digest"]))


def oracle_weights(layer):
    f = lambda t: t.float().numpy()
    return og.GptOssWeights(f(layer.router_w), f(layer.router_b), layer.w13_blocks.numpy(),
                            layer.w13_scales.numpy(), f(layer.w13_bias), layer.w2_blocks.numpy(),
                            layer.w2_scales.numpy(), f(layer.w2_bias), layer.limit)


def oracle_for_case(case, expert_range=None):
    layer, x = case["layer"], case["x"]
    out = og.moe_forward(x.float().numpy(), oracle_weights(layer), layer.top_k, expert_range)
    out["y_bits"] = f32_to_bf16_bits(out["y"])
    out["logits_bits"] = f32_to_bf16_bits(out["logits"])
    out["weights_bits"] = f32_to_bf16_bits(out["weights"])
    return out


def bf16_tensor_to_f32(t):
    return bf16_bits_to_f32(t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16))


def parity_metrics(y, y_ref):
    """Return dict(max_abs, max_ref, rms_ref, rel_l2, exact_frac) for bf16-valued arrays."""
    y = np.asarray(y, dtype=np.float64)
    y_ref = np.asarray(y_ref, dtype=np.float64)
    d = np.abs(y - y_ref)
    rms = float(np.sqrt((y_ref ** 2).mean())) if y_ref.size else 0.0
    nrm = float(np.linalg.norm(y_ref))
    return dict(max_abs=float(d.max()) if d.size else 0.0, rms_ref=rms,
                max_ref=float(np.abs(y_ref).max()) if y_ref.size else 0.0,
                rel_l2=float(np.linalg.norm(y - y_ref) / nrm) if nrm > 0 else float(np.linalg.norm(y - y_ref)),
                exact_frac=float((d == 0).mean()) if d.size else 1.0)


# Tolerances (bf16 outputs): rel-L2 <= 5e-3 and max-abs <= 2e-2 on the output
# scaled to unit peak (max|y_ref| when that exceeds 1).  The synthetic MXFP4
# weights give outputs with RMS ~1e2 and peaks ~5e2, where one bf16 ulp is 2.0:
# an unscaled 2e-2 would demand bit-exactness of every element.
REL_L2_TOL = 5e-3
MAX_ABS_TOL = 2e-2


def bf16_peak_ulp(y_ref):
    """One bf16 ulp at the largest |y_ref| (the spacing of bf16 values there)."""
    peak = float(np.abs(np.asarray(y_ref, np.float64)).max()) if np.size(y_ref) else 0.0
    return float(np.exp2(np.floor(np.log2(peak)) - 7)) if peak > 0 else 0.0


def assert_within_tolerance(y, y_ref, ulp_frac1=0.999, peak_ulps=1.0):
    """The layer tolerance plus element-wise bounds in bf16 steps: at least
    ulp_frac1 of the elements within one step of the reference (bf16_steps), and
    every element within peak_ulps bf16 ulps at the output's peak, i.e. an
    absolute error no larger than one rounding of the largest outputs.  (A step
    bound on every element cannot hold: the reference folds the experts' rows with
    a bf16 rounding after every add, so an output that cancels to a small value
    carries the rounding of partial sums near the peak.)  The metrics returned
    carry the unscaled max-abs and the step statistics either way."""
    m = parity_metrics(y, y_ref)
    m.update(ulp_stats(y, y_ref))
    m["peak_ulp"] = bf16_peak_ulp(y_ref)
    assert m["rel_l2"] <= REL_L2_TOL, m
    assert m["max_abs"] <= MAX_ABS_TOL * max(m["max_ref"], 1.0), m
    if ulp_frac1 is not None:
        assert m["ulp_le1"] >= ulp_frac1, m
    if peak_ulps is not None:
        assert m["max_abs"] <= peak_ulps * m["peak_ulp"], m
    return m


def bf16_steps(y, y_ref, floor_div=16.0):
    """Element-wise |y - y_ref| in bf16 steps (ulps) of the reference value, where
    values smaller than RMS(y_ref)/floor_div count as that size: an output that
    cancels to near zero is a sum of terms of the output's scale, and fp32
    summation order moves it by a fraction of their ulp, not of its own."""
    y = np.asarray(y, np.float64)
    y_ref = np.asarray(y_ref, np.float64)
    if y_ref.size == 0:
        return np.zeros(0)
    rms = float(np.sqrt(np.mean(y_ref ** 2)))
    a = np.maximum(np.maximum(np.abs(y_ref), rms / floor_div), np.finfo(np.float32).tiny)
    return np.abs(y - y_ref) / np.exp2(np.floor(np.log2(a)) - 7)


def ulp_stats(y, y_ref):
    d = bf16_steps(y, y_ref)
    if d.size == 0:
        return dict(ulp_max=0.0, ulp_le1=1.0, ulp_exact=1.0)
    return dict(ulp_max=float(d.max()), ulp_le1=float((d <= 1).mean()), ulp_exact=float((d == 0).mean()))
