"""Shared helpers of the MiniMax-M2.5 NVFP4 tests: fixture loading with the input
digest that guards the seeded generator, and the oracle on a fixture's layer."""
import hashlib

import numpy as np
import torch

from flyai_b200 import synth
from oracle import m25
from oracle.fp import bf16_bits_to_f32

SHAPE_KEYS = ("num_experts", "top_k", "hidden", "inter")


def load_case(path):
    f = dict(np.load(path))
    shape = {k: int(f[k]) for k in SHAPE_KEYS}
    seed = int(f["seed"])
    layer = synth.make_m25_layer(**shape, seed=seed, global_scale=float(f["global_scale"]))
    x = synth.make_tokens(int(f["M"]), layer.hidden, seed=seed)
    return dict(fixture=f, shape=shape, layer=layer, x=x, seed=seed, path=path)


def dequant_expert(layer, e, device=None, bf16=False):
    """Expert e's [w1; w3] and w2 dequantised (exact NVFP4 values, or bf16-rounded)."""
    w13, s13, g13, w2, s2, g2 = layer.expert(e, device=device)
    I = layer.inter
    s13b, s2b = s13.view(torch.uint8).cpu().numpy(), s2.view(torch.uint8).cpu().numpy()
    w13, w2 = w13.cpu().numpy(), w2.cpu().numpy()
    top = m25.dequant_nvfp4(w13[:I], s13b[:I], float(g13[0]), bf16)
    bot = m25.dequant_nvfp4(w13[I:], s13b[I:], float(g13[1]), bf16)
    return np.concatenate([top, bot]), m25.dequant_nvfp4(w2, s2b, float(g2[0]), bf16)


def digest_ok(case):
    layer, f = case["layer"], case["fixture"]
    inner = hashlib.sha256()
    for e in sorted(set(int(v) for v in f["ids"].ravel())):
        for t in layer.expert(e):
            inner.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    h = hashlib.sha256()
    for t in (layer.router_w, layer.bias, case["x"]):
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    h.update(inner.hexdigest().encode())
    return h.hexdigest() == str(f["digest"])


def oracle_case(case, bf16_weights=False):
    layer = case["layer"]
    x = case["x"].float().numpy()
    ids, wts, logits = m25.router(x, layer.router_w.float().numpy(), layer.bias.numpy(), layer.top_k,
                                  layer.route_scale)
    y = m25.moe_forward(x, ids, wts, lambda e: dequant_expert(layer, e, bf16=bf16_weights))
    return dict(ids=ids, wts=wts, logits=logits, y=y)


def exact_in_bf16(case):
    """True when the case's global scale is a power of two: its NVFP4 weights are
    then exactly bf16 values and the HF module sees the exact weights."""
    g = float(case["fixture"]["global_scale"])
    return g > 0 and np.frexp(g)[0] == 0.5


def fixture_y(case):
    return bf16_bits_to_f32(case["fixture"]["y"])


def is_f32_fixture(case):
    """The fixture holds HF's MiniMaxM2Experts.forward run in fp32 on the exact NVFP4
    weights ("y_f32"), not the bf16 module's output."""
    return "y_f32" in case["fixture"]


def bf16_module_distance(case):
    """rel-L2 of HF's bf16 module (the fixture of the same layer and tokens held in
    bf16) from the fp32 exact-weight evaluation of an _f32 fixture: the reference
    CPU arithmetic's own distance to the exact-weight layer."""
    import os
    from tests.dsv3_util import metrics
    path = case["path"].replace("_f32.npz", ".npz")
    bf = np.load(path)
    assert int(bf["seed"]) == case["seed"] and str(bf["digest"]) == str(case["fixture"]["digest"])
    return metrics(bf16_bits_to_f32(bf["y"]), case["fixture"]["y_f32"])["rel_l2"]


def metrics_of(got, ref):
    from tests.dsv3_util import metrics
    return metrics(got, ref)
