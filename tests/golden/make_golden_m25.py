"""Generate the MiniMax-M2.5 NVFP4 MoE fixtures by running the reference's CPU
arithmetic itself: HF transformers' MiniMaxM2SparseMoeBlock (installed:
transformers/models/minimax_m2/modeling_minimax_m2.py; the reference's M2.5
stage configures its vLLM FusedMoE to the same gating, engines/minimax_m25/
m25_stage.py:288-311) on expert weights dequantised from NVFP4 (e2m1 x e4m3
block-16 scale x fp32 global scale, to bf16).

    python tests/golden/make_golden_m25.py [--only name,name]

Inputs come from ``flyai_b200.synth`` (seeded, per-expert seeds; only the
experts the tokens touch are dequantised, the others stay zero and unused);
each fixture keeps a SHA-256 of the router, the tokens and the touched experts.
The routed_scaling_factor of these cases is 1.0 (the HF module has none).
"""
import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from flyai_b200 import synth  # noqa: E402

# Global scale 2^-7 makes every NVFP4 weight an exact bf16 value, so the HF
# module computes with the exact weights; the config's own 1e-2 does not, and
# its fixture also records how far bf16-held weights move the layer output.
# The "_f32" case pins the config's own scale against exact weights: the
# reference's M2.5 stage runs vLLM's NVFP4 FusedMoE, whose cutlass fp4 GEMMs
# take the e2m1 x e4m3 block values as they are and apply each expert's global
# scale to the fp32 accumulator as alpha (vllm/model_executor/layers/fused_moe/
# experts/cutlass_moe.py:481-643, run_cutlass_moe_fp4: w1_alphas / w2_alphas).
# HF's MiniMaxM2Experts.forward is run in fp32 on fp32 weights holding the exact
# NVFP4 values (one fp32 rounding of e2m1 x e4m3 x global), routed by the bf16
# gate as in the other cases; the fixture stores that fp32 output.
CASES = [
    # name, layer shape, tokens, seed, global scale
    ("m25_small_seed0", dict(num_experts=32, top_k=4, hidden=256, inter=128), 5, 0, 2.0 ** -7),
    ("m25_small_m1", dict(num_experts=64, top_k=8, hidden=128, inter=256), 1, 1, 2.0 ** -7),
    ("m25_small_m37", dict(num_experts=32, top_k=8, hidden=256, inter=256), 37, 2, 2.0 ** -7),
    ("m25_full_m5_pow2", synth.M25, 5, 0, 2.0 ** -7),
    ("m25_full_m5", synth.M25, 5, 0, 1e-2),
    ("m25_full_m5_f32", synth.M25, 5, 0, 1e-2),
]


def dequant(blocks, scales, g):
    lut = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                        -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])
    v = torch.stack([lut[(blocks & 0x0F).long()], lut[(blocks >> 4).long()]], -1).flatten(-2)
    s = scales.float().repeat_interleave(16, -1)
    return (v * s * g).bfloat16()


def run_reference(layer, x):
    from transformers.models.minimax_m2.configuration_minimax_m2 import MiniMaxM2Config
    from transformers.models.minimax_m2.modeling_minimax_m2 import MiniMaxM2SparseMoeBlock
    E, H, I, k = layer.num_experts, layer.hidden, layer.inter, layer.top_k
    cfg = MiniMaxM2Config(num_local_experts=E, num_experts_per_tok=k, hidden_size=H,
                          intermediate_size=I, hidden_act="silu", router_jitter_noise=0.0)
    cfg._experts_implementation = "eager"
    blk = MiniMaxM2SparseMoeBlock(cfg).eval()
    with torch.no_grad():
        blk.gate.weight.data = layer.router_w.clone()
        blk.e_score_correction_bias.copy_(layer.bias)
        _, _, idx = blk.gate(x, blk.e_score_correction_bias)
        touched = sorted(set(idx.flatten().tolist()))
        gu = torch.zeros(E, 2 * I, H, dtype=torch.bfloat16)
        dn = torch.zeros(E, H, I, dtype=torch.bfloat16)
        digest = hashlib.sha256()
        for e in touched:
            w13, s13, g13, w2, s2, g2 = layer.expert(e)
            for t in (w13, s13, g13, w2, s2, g2):
                digest.update(t.contiguous().view(torch.uint8).numpy().tobytes())
            gu[e, :I] = dequant(w13[:I], s13[:I], g13[0])
            gu[e, I:] = dequant(w13[I:], s13[I:], g13[1])
            dn[e] = dequant(w2, s2, g2[0])
        blk.experts.gate_up_proj.data = gu
        blk.experts.down_proj.data = dn
        blk.to(torch.bfloat16)
        blk.e_score_correction_bias.copy_(layer.bias)   # keep the fp32 buffer's values
        logits, scores, idx = blk.gate(x, blk.e_score_correction_bias.float())
        y = blk(x.view(1, -1, H)).view(-1, H)
    return logits, idx, scores, y, digest.hexdigest()


def dequant_f32(blocks, scales, g):
    """Exact NVFP4 values rounded once to fp32 (the product is formed in float64)."""
    lut = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                        -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=torch.float64)
    v = torch.stack([lut[(blocks & 0x0F).long()], lut[(blocks >> 4).long()]], -1).flatten(-2)
    s = scales.double().repeat_interleave(16, -1)
    return (v * s * float(g)).float()


def run_reference_f32(layer, x):
    """bf16 gate (as the bf16 module), then HF's MiniMaxM2Experts.forward in fp32 on
    the exact NVFP4 weights."""
    from transformers.models.minimax_m2.configuration_minimax_m2 import MiniMaxM2Config
    from transformers.models.minimax_m2.modeling_minimax_m2 import MiniMaxM2SparseMoeBlock
    E, H, I, k = layer.num_experts, layer.hidden, layer.inter, layer.top_k
    cfg = MiniMaxM2Config(num_local_experts=E, num_experts_per_tok=k, hidden_size=H,
                          intermediate_size=I, hidden_act="silu", router_jitter_noise=0.0)
    cfg._experts_implementation = "eager"
    blk = MiniMaxM2SparseMoeBlock(cfg).eval()
    with torch.no_grad():
        blk.gate.weight.data = layer.router_w.clone()          # bf16: bf16 F.linear logits
        logits, scores, idx = blk.gate(x, layer.bias.float())
        touched = sorted(set(idx.flatten().tolist()))
        gu = torch.zeros(E, 2 * I, H, dtype=torch.float32)
        dn = torch.zeros(E, H, I, dtype=torch.float32)
        digest = hashlib.sha256()
        for e in touched:
            w13, s13, g13, w2, s2, g2 = layer.expert(e)
            for t in (w13, s13, g13, w2, s2, g2):
                digest.update(t.contiguous().view(torch.uint8).numpy().tobytes())
            gu[e, :I] = dequant_f32(w13[:I], s13[:I], g13[0])
            gu[e, I:] = dequant_f32(w13[I:], s13[I:], g13[1])
            dn[e] = dequant_f32(w2, s2, g2[0])
        blk.experts.gate_up_proj.data = gu
        blk.experts.down_proj.data = dn
        y = blk.experts(x.float(), idx, scores.float())
    return logits, idx, scores, y, digest.hexdigest()


def main(only=None):
    for name, shape, M, seed, gscale in CASES:
        if only and name not in only:
            continue
        layer = synth.make_m25_layer(**shape, seed=seed, global_scale=gscale)
        x = synth.make_tokens(M, layer.hidden, seed=seed)
        f32 = name.endswith("_f32")
        logits, ids, wts, y, exp_digest = (run_reference_f32 if f32 else run_reference)(layer, x)
        h = hashlib.sha256()
        for t in (layer.router_w, layer.bias, x):
            h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
        h.update(exp_digest.encode())
        np.savez_compressed(
            os.path.join(HERE, name + ".npz"),
            ids=ids.numpy().astype(np.int32), wts=wts.float().numpy(),
            logits=logits.contiguous().view(torch.int16).numpy().view(np.uint16),
            **(dict(y_f32=y.numpy().astype(np.float32)) if f32 else
               dict(y=y.contiguous().view(torch.int16).numpy().view(np.uint16))),
            M=M, seed=seed, digest=h.hexdigest(), num_experts=layer.num_experts,
            top_k=layer.top_k, hidden=layer.hidden, inter=layer.inter, global_scale=gscale)
        print(name, "tokens", M, "experts touched", len(set(ids.flatten().tolist())))


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=None, help="comma-separated case names")
    a = ap.parse_args()
    main(a.only.split(",") if a.only else None)
