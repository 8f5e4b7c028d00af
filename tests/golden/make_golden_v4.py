"""Generate the DeepSeek-V4 W4A8 MoE fixtures by running the reference itself.

    python tests/golden/make_golden_v4.py --reference <FlyAI checkout> [--only name,name]

The reference code that runs (nothing of it is copied into this repository):
``engines/deepseek_v4/v4_ref_cpu.load_ref()`` -- the vendored DeepSeek-V4 model
(vendor/deepseek_v4_ref/inference/model.py) with the reference's own CPU kernels
(engines/deepseek_v4/v4_kernels_cpu.py: act_quant, fp4_gemm, fp8_gemm).  Its
``MoE`` (model.py:615-649) is built as a V4-Flash checkpoint configures it
(config.json: expert_dtype "fp4", dtype "fp8", scale_fmt "ue8m0", scale_dtype
"fp8", score_func "sqrtsoftplus"): routed experts are fp4 ``Linear``s, the
shared expert an fp8 one, the module globals set as Transformer.__init__ sets
them (model.py:881-886), run under default dtype bf16 (model.py:950).  The
reference's MoE.forward levers (v4_moe_decode, v4_moe_grouped) are switched off
(V4_MOE_DECODE=0, V4_MOE_GROUPED=0), so the untouched reference forward runs.
A hash-routed case builds the layer with layer_id < n_hash_layers, so the gate
reads ``tid2eid[input_ids]`` (model.py:581-582) and repeated experts exercise
the duplicate-index rule of ``y[idx] +=``.

Inputs come from ``flyai_b200.synth`` (seeded; every expert has its own seed);
each fixture keeps a SHA-256 of the router, the tokens, the touched experts and
the shared expert.
"""
import argparse
import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from flyai_b200 import synth  # noqa: E402

SMALL = dict(num_experts=32, top_k=6, hidden=256, inter=256)
CASES = [
    # name, layer shape, tokens, seed, hash vocabulary (0 = score-routed)
    ("v4_small_seed0", SMALL, 5, 0, 0),
    ("v4_small_m1", dict(num_experts=64, top_k=6, hidden=512, inter=256), 1, 1, 0),
    ("v4_small_m33", SMALL, 33, 2, 0),
    ("v4_small_hash", SMALL, 16, 3, 8),          # 8 token ids, repeats inside tid2eid rows
    ("v4_full_m1", synth.V4, 1, 0, 0),
    ("v4_full_m6", synth.V4, 6, 1, 0),
    ("v4_full_hash_m4", synth.V4, 4, 2, 64),
]


def input_ids_for(M, vocab, seed):
    g = torch.Generator().manual_seed(seed + 4242)
    return torch.randint(0, vocab, (M,), generator=g) if vocab else torch.zeros(M, dtype=torch.long)


def load_reference(root):
    os.environ["V4_MOE_DECODE"] = "0"
    os.environ["V4_MOE_GROUPED"] = "0"
    sys.path.insert(0, os.path.join(root, "engines", "deepseek_v4"))
    import v4_ref_cpu
    return v4_ref_cpu.load_ref()


def run_reference(ref, layer, x, input_ids):
    E, H, I, k = layer.num_experts, layer.hidden, layer.inter, layer.top_k
    hashed = layer.tid2eid is not None
    args = ref.ModelArgs(dim=H, moe_inter_dim=I, n_routed_experts=E, n_activated_experts=k,
                         n_shared_experts=1, n_hash_layers=1 if hashed else 0,
                         score_func="sqrtsoftplus", route_scale=layer.route_scale,
                         swiglu_limit=layer.swiglu_limit, expert_dtype="fp4", dtype="fp8",
                         scale_fmt="ue8m0", scale_dtype="fp8",
                         vocab_size=layer.tid2eid.shape[0] if hashed else 1024)
    saved = (ref.default_dtype, ref.scale_fmt, ref.scale_dtype)
    ref.default_dtype = torch.float8_e4m3fn
    ref.scale_fmt = "ue8m0"
    ref.scale_dtype = torch.float8_e8m0fnu
    digest = hashlib.sha256()
    try:
        with ref.set_dtype(torch.bfloat16):
            moe = ref.MoE(0, args).eval()
        moe.gate.weight.data = layer.router_w.clone()
        if hashed:
            moe.gate.tid2eid.data = layer.tid2eid.clone()
            touched = sorted(set(layer.tid2eid[input_ids].flatten().tolist()))
        else:
            moe.gate.bias.data = layer.bias.clone()
            with torch.no_grad(), ref.set_dtype(torch.bfloat16):
                _, idx = moe.gate(x, input_ids)
            touched = sorted(set(idx.flatten().tolist()))
        for e in touched:
            w13, s13, w2, s2 = layer.expert(e)
            for t in (w13, s13, w2, s2):
                digest.update(t.contiguous().view(torch.uint8).numpy().tobytes())
            ex = moe.experts[e]
            for lin, w, s in ((ex.w1, w13[:I], s13[:I]), (ex.w3, w13[I:], s13[I:]), (ex.w2, w2, s2)):
                lin.weight.data = w.clone().view(torch.float4_e2m1fn_x2)
                lin.weight.scale = s.clone().view(torch.float8_e8m0fnu)
        w13, s13, w2, s2 = layer.shared()
        for t in (w13, s13, w2, s2):
            digest.update(t.contiguous().view(torch.uint8).numpy().tobytes())
        sh = moe.shared_experts
        for lin, w, s in ((sh.w1, w13[:I], s13[: I // 128]), (sh.w3, w13[I:], s13[I // 128:]),
                          (sh.w2, w2, s2)):
            lin.weight.data = w.clone()
            lin.weight.scale = s.clone().view(torch.float8_e8m0fnu)
        with torch.no_grad(), ref.set_dtype(torch.bfloat16):
            wts, ids = moe.gate(x, input_ids)
            logits = torch.nn.functional.linear(x.float(), moe.gate.weight.float())
            y = moe(x.view(1, -1, H), input_ids.view(1, -1)).view(-1, H)
    finally:
        ref.default_dtype, ref.scale_fmt, ref.scale_dtype = saved
    return ids, wts, logits, y, digest.hexdigest()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of a FlyAI checkout")
    ap.add_argument("--only", default=None, help="comma-separated case names")
    a = ap.parse_args()
    ref = load_reference(a.reference)
    only = set(a.only.split(",")) if a.only else None
    for name, shape, M, seed, vocab in CASES:
        if only and name not in only:
            continue
        layer = synth.make_v4_layer(**shape, seed=seed, hash_vocab=vocab)
        x = synth.make_tokens(M, layer.hidden, seed=seed)
        input_ids = input_ids_for(M, vocab, seed)
        ids, wts, logits, y, exp_digest = run_reference(ref, layer, x, input_ids)
        h = hashlib.sha256()
        for t in (layer.router_w, layer.bias, x, input_ids) + ((layer.tid2eid,) if vocab else ()):
            h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
        h.update(exp_digest.encode())
        np.savez_compressed(
            os.path.join(HERE, name + ".npz"),
            ids=ids.numpy().astype(np.int32), wts=wts.float().numpy(), logits=logits.numpy(),
            y=y.contiguous().view(torch.int16).numpy().view(np.uint16),
            input_ids=input_ids.numpy().astype(np.int32),
            M=M, seed=seed, digest=h.hexdigest(), num_experts=layer.num_experts,
            top_k=layer.top_k, hidden=layer.hidden, inter=layer.inter, hash_vocab=vocab,
            route_scale=layer.route_scale, swiglu_limit=layer.swiglu_limit)
        dup = int(sum(len(r) - len(set(r)) for r in ids.tolist()))
        print(name, "tokens", M, "experts touched", len(set(ids.flatten().tolist())),
              "repeated slots", dup)


if __name__ == "__main__":
    main()
