"""Shared helpers of the Kimi-K3 tests: fixture loading with the input digest
that guards the seeded generator, and the oracle on a fixture's layer."""
import hashlib

import numpy as np
import torch

from flyai_b200 import synth
from oracle import k3


def load_case(path):
    f = dict(np.load(path))
    E, k, H, I, M, seed = (int(f[n]) for n in ("E", "k", "H", "I", "M", "seed"))
    lb = float(f["linear_beta"])
    lb = None if lb < 0 else lb
    layer = synth.make_k3_layer(E, k, H, I, beta=float(f["beta"]), linear_beta=lb, seed=seed)
    x = synth.make_tokens(M, H, seed=seed)
    ids, wts = layer.routing(M, seed=seed)
    h = hashlib.sha256()
    for t in (x, ids, wts):
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    for e in sorted(set(int(v) for v in ids.ravel())):
        for t in layer.expert(e):
            h.update(t.contiguous().numpy().tobytes())
    assert h.hexdigest() == str(f["digest"]), "synth generator drifted from the fixture's inputs"
    return dict(fixture=f, layer=layer, x=x, ids=ids, wts=wts)


def oracle_case(case):
    layer = case["layer"]
    cache = {}

    def get(e):
        if e not in cache:
            cache[e] = tuple(t.numpy() for t in layer.expert(e))
        return cache[e]
    return k3.moe_infer(case["x"].float().numpy(), case["ids"].numpy(), case["wts"].numpy(), get,
                        layer.beta, layer.linear_beta)
