"""Shared helpers of the DeepSeek-V4 W4A8 tests: fixture loading with the input
digest that guards the seeded generator, and the oracle on a fixture's layer."""
import hashlib

import numpy as np
import torch

from flyai_b200 import synth
from oracle import v4

SHAPE_KEYS = ("num_experts", "top_k", "hidden", "inter")


def load_case(path):
    f = dict(np.load(path))
    shape = {k: int(f[k]) for k in SHAPE_KEYS}
    shape["route_scale"] = float(f["route_scale"])
    shape["swiglu_limit"] = float(f["swiglu_limit"])
    seed, vocab = int(f["seed"]), int(f["hash_vocab"])
    layer = synth.make_v4_layer(**shape, seed=seed, hash_vocab=vocab)
    x = synth.make_tokens(int(f["M"]), layer.hidden, seed=seed)
    return dict(fixture=f, shape=shape, layer=layer, x=x, seed=seed,
                input_ids=torch.from_numpy(f["input_ids"].astype(np.int64)))


def expert_np(layer):
    cache = {}

    def get(e):
        if e not in cache:
            cache[e] = tuple(t.cpu().numpy() for t in layer.expert(e))
        return cache[e]
    return get


def shared_np(layer):
    w13, s13, w2, s2 = layer.shared()
    t = (w13.view(torch.uint8).cpu().numpy(), s13.cpu().numpy(), w2.view(torch.uint8).cpu().numpy(),
         s2.cpu().numpy())
    return lambda: t


def digest_ok(case):
    layer, f = case["layer"], case["fixture"]
    inner = hashlib.sha256()
    for e in sorted(set(int(v) for v in f["ids"].ravel())):
        for t in layer.expert(e):
            inner.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    for t in layer.shared():
        inner.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    h = hashlib.sha256()
    extra = (layer.tid2eid,) if layer.tid2eid is not None else ()
    for t in (layer.router_w, layer.bias, case["x"], case["input_ids"]) + extra:
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    h.update(inner.hexdigest().encode())
    return h.hexdigest() == str(f["digest"])


def oracle_case(case, rows=None):
    layer = case["layer"]
    x = case["x"].float().numpy()
    tid = layer.tid2eid.cpu().numpy() if layer.tid2eid is not None else None
    ids, wts, logits = v4.gate(x, layer.router_w.float().cpu().numpy(), layer.bias.cpu().numpy(),
                               layer.top_k, layer.route_scale, tid, case["input_ids"].numpy())
    sel = slice(None) if rows is None else rows
    y = v4.moe_forward(x[sel], ids[sel], wts[sel], expert_np(layer), shared_np(layer),
                       layer.swiglu_limit)
    return dict(ids=ids, wts=wts, logits=logits, y=y)
