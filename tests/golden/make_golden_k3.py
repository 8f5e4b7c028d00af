"""Generate the Kimi-K3 routed-expert fixtures by running the reference itself.

    python tests/golden/make_golden_k3.py --reference <FlyAI checkout>

The reference code that runs (nothing of it is copied into this repository):
``KimiSparseMoeBlock.moe_infer`` and ``KimiBlockSparseMLP`` / ``SituAndMul`` of
vendor/kimi_k3_ref/modeling_kimi_linear.py (:64-80, 242-268, 841-875), with
``hidden_act`` "situ" and the case's beta / linear_beta, the experts' nn.Linear
weights set to the dequantised MXFP4 tensors (e2m1 x 2^(e8m0 - 127), exact in
bf16), run in bf16 on the CPU with the caller's ids and weights.  The module
imports names this image's transformers no longer has (``OutputRecorder``,
``check_model_inputs``); stand-ins are installed for them first -- they are
used only by the model classes, never on this path.

Inputs come from ``flyai_b200.synth.make_k3_layer`` (seeded; one seed per
expert); each fixture keeps a SHA-256 of the tokens, the routing and the touched
experts' tensors.
"""
import argparse
import hashlib
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from flyai_b200 import synth  # noqa: E402
from oracle.v4 import dequant_fp4  # noqa: E402

CASES = [
    # name, (E, k, H, I), tokens, seed, beta, linear_beta
    ("k3_small_m5", (16, 4, 256, 128), 5, 0, 4.0, 25.0),
    ("k3_small_m33", (32, 8, 512, 256), 33, 1, 4.0, 25.0),
    ("k3_nolinear_m8", (24, 6, 256, 192), 8, 2, 1.0, None),
    ("k3_top16_m12", (64, 16, 1024, 512), 12, 3, 4.0, 25.0),
]


def load_reference(root):
    import transformers.utils.generic as g
    if not hasattr(g, "OutputRecorder"):
        g.OutputRecorder = type("OutputRecorder", (), {"__init__": lambda self, *a, **k: None})
    if not hasattr(g, "check_model_inputs"):
        g.check_model_inputs = lambda *a, **k: (a[0] if a and callable(a[0]) else (lambda f: f))
    sys.path.insert(0, os.path.join(root, "vendor"))
    import kimi_k3_ref.configuration_kimi_k3 as c
    import kimi_k3_ref.modeling_kimi_linear as m
    return c, m


def digest_of(layer, x, ids, wts):
    h = hashlib.sha256()
    for t in (x, ids, wts):
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    for e in sorted(set(int(v) for v in ids.ravel())):
        for t in layer.expert(e):
            h.update(t.contiguous().numpy().tobytes())
    return h.hexdigest()


def run_reference(conf, mod, layer, x, ids, wts, beta, linear_beta):
    cfg = conf.KimiLinearConfig(hidden_size=layer.hidden, moe_intermediate_size=layer.inter,
                                num_experts=layer.num_experts, num_experts_per_token=layer.top_k,
                                hidden_act="situ", activation_situ_beta=beta,
                                activation_situ_linear_beta=linear_beta)
    experts = torch.nn.ModuleList()
    for e in range(layer.num_experts):
        mlp = mod.KimiBlockSparseMLP(cfg, hidden_size=layer.hidden, intermediate_size=layer.inter)
        if e in set(int(v) for v in ids.ravel()):
            w1, s1, w3, s3, w2, s2 = (t.numpy() for t in layer.expert(e))
            mlp.w1.weight.data = torch.from_numpy(dequant_fp4(w1, s1)).bfloat16()
            mlp.w3.weight.data = torch.from_numpy(dequant_fp4(w3, s3)).bfloat16()
            mlp.w2.weight.data = torch.from_numpy(dequant_fp4(w2, s2)).bfloat16()
        experts.append(mlp.bfloat16())
    block = types.SimpleNamespace(experts=experts, ep_rank=0, experts_per_rank=layer.num_experts)
    with torch.no_grad():
        return mod.KimiSparseMoeBlock.moe_infer(block, x, ids, wts)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of a FlyAI checkout")
    a = ap.parse_args()
    conf, mod = load_reference(a.reference)
    for name, (E, k, H, I), M, seed, beta, lb in CASES:
        layer = synth.make_k3_layer(E, k, H, I, beta=beta, linear_beta=lb, seed=seed)
        x = synth.make_tokens(M, H, seed=seed)
        ids, wts = layer.routing(M, seed=seed)
        y = run_reference(conf, mod, layer, x, ids, wts, beta, lb)
        assert y.dtype == torch.bfloat16 and tuple(y.shape) == (M, H)
        np.savez_compressed(os.path.join(HERE, name + ".npz"),
                            y=y.contiguous().view(torch.int16).numpy().view(np.uint16),
                            E=E, k=k, H=H, I=I, M=M, seed=seed, beta=beta,
                            linear_beta=-1.0 if lb is None else lb,
                            digest=digest_of(layer, x, ids, wts))
        print(name, "tokens", M, "experts touched", len(set(ids.ravel().tolist())))


if __name__ == "__main__":
    main()
