"""Generate the golden fixtures by running the reference implementation itself.

Run in a container that has the reference's Python dependencies (transformers
5.5.0 is what this repository was checked against):

    python tests/golden/make_golden.py [--only name,name]

Every shape is a multiple of 64 in hidden and inter: the tcgen05 kernels (the
only expert path) take K-tiles of 64.

GPT-OSS fixtures come from HuggingFace transformers' own CPU modules -- the code
the reference loads for GPT-OSS (phase0/pipeline.py:126-182):
``GptOssTopKRouter`` (transformers/models/gpt_oss/modeling_gpt_oss.py:117-131),
``GptOssExperts`` eager forward (:69-114) on weights dequantised by
``_convert_moe_packed_tensors`` (transformers/integrations/mxfp4.py:279-330).
Inputs come from ``flyai_b200.synth`` with the stored seeds; each fixture keeps a
SHA-256 of those inputs so a drifting generator is caught instead of silently
producing a different layer.
"""
import hashlib
import os
import sys
from types import SimpleNamespace

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from flyai_b200 import synth  # noqa: E402


def layer_digest(layer, x):
    h = hashlib.sha256()
    for t in (layer.router_w, layer.router_b, layer.w13_blocks, layer.w13_scales, layer.w13_bias,
              layer.w2_blocks, layer.w2_scales, layer.w2_bias, x):
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def reference_gpt_oss(layer, x):
    from transformers.integrations.mxfp4 import _convert_moe_packed_tensors
    from transformers.models.gpt_oss.modeling_gpt_oss import GptOssExperts, GptOssTopKRouter
    E, H, I, k = layer.num_experts, layer.hidden, layer.inter, layer.top_k
    cfg = SimpleNamespace(num_experts_per_tok=k, num_local_experts=E, hidden_size=H,
                          intermediate_size=I, _experts_implementation="eager")
    router = GptOssTopKRouter(cfg)
    router.weight.data = layer.router_w.clone()
    router.bias.data = layer.router_b.clone()
    experts = GptOssExperts(cfg)
    with torch.no_grad():
        logits, scores, idx = router(x)
        hit = sorted(set(idx.flatten().tolist()))
        gu = torch.zeros(E, H, 2 * I, dtype=torch.bfloat16)
        dn = torch.zeros(E, I, H, dtype=torch.bfloat16)
        if hit:
            gu[hit] = _convert_moe_packed_tensors(layer.w13_blocks[hit], layer.w13_scales[hit])
            dn[hit] = _convert_moe_packed_tensors(layer.w2_blocks[hit], layer.w2_scales[hit])
        experts.gate_up_proj.data = gu
        experts.down_proj.data = dn
        experts.gate_up_proj_bias.data = layer.w13_bias.clone()
        experts.down_proj_bias.data = layer.w2_bias.clone()
        experts.to(torch.bfloat16)
        experts.limit = layer.limit
        experts.alpha = layer.alpha
        y = experts(x, idx, scores) if x.shape[0] else torch.zeros_like(x)
    return logits, idx, scores, y


def tie_heavy_router(layer, seed):
    """Router weights on a coarse grid so many bf16 logits tie exactly."""
    g = torch.Generator().manual_seed(seed + 77)
    E, H = layer.router_w.shape
    layer.router_w = (torch.randint(-2, 3, (E, H), generator=g).float() * 2.0 ** -6).bfloat16()
    layer.router_b = torch.zeros(E).bfloat16()
    return layer


CASES = [
    # name, shape, tokens, seed, options
    ("gptoss_cfg0_seed0", synth.GPT_OSS_20B, 5, 0, {}),
    ("gptoss_small_seed0", dict(num_experts=8, top_k=4, hidden=256, inter=128), 7, 0, {}),
    ("gptoss_small_seed1", dict(num_experts=16, top_k=4, hidden=128, inter=128), 33, 1, {}),
    ("gptoss_small_m1", dict(num_experts=8, top_k=2, hidden=64, inter=64), 1, 2, {}),
    ("gptoss_small_ties", dict(num_experts=32, top_k=4, hidden=64, inter=64), 64, 3, {"ties": True}),
    ("gptoss_small_e128", dict(num_experts=128, top_k=4, hidden=128, inter=64), 16, 4, {"ties": True}),
]


def main(only=None):
    os.makedirs(HERE, exist_ok=True)
    for name, shape, M, seed, opt in CASES:
        if only and name not in only:
            continue
        layer = synth.make_gpt_oss_layer(**shape, seed=seed)
        if opt.get("ties"):
            layer = tie_heavy_router(layer, seed)
        x = synth.make_tokens(M, shape["hidden"], seed=seed)
        if opt.get("ties"):
            x = torch.round(x.float() * 2).bfloat16()
        logits, idx, scores, y = reference_gpt_oss(layer, x)
        out = dict(num_experts=shape["num_experts"], top_k=shape["top_k"], hidden=shape["hidden"],
                   inter=shape["inter"], tokens=M, seed=seed, ties=int(bool(opt.get("ties"))),
                   digest=layer_digest(layer, x), logits=bits(logits), ids=idx.numpy().astype(np.int32),
                   weights=bits(scores), y=bits(y))
        small = shape["hidden"] <= 256
        if small:   # small cases also store their inputs verbatim
            out.update(x=bits(x), router_w=bits(layer.router_w), router_b=bits(layer.router_b))
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **out)
        ties = int((logits.float().unsqueeze(-1) == logits.float().unsqueeze(-2)).sum() - logits.numel())
        print(f"{name}: M={M} E={shape['num_experts']} hit={len(set(idx.flatten().tolist()))} "
              f"tie_pairs={ties} |y|rms={y.float().pow(2).mean().sqrt():.3f}")


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=None, help="comma-separated case names")
    a = ap.parse_args()
    main(a.only.split(",") if a.only else None)
