"""The drop-in levers at the reference's seams, on the GPU:

* GPT-OSS -- a real transformers ``GptOssMLP`` whose forward ``gpt_oss.install``
  rebinds: (out, router_scores) against the module's own CPU forward, declines
  counted by ``coverage()``;
* DeepSeek -- ``deepseek.install`` on a module whose MoE / Gate / Expert / Linear
  classes carry the vendored reference's attributes (vendor/deepseek_v4_ref/
  inference/model.py:114-649; the reference tree does not travel to this box):
  a V4 layer (fp4 experts, score- and hash-routed) and a DeepSeek-V3-style layer
  (fp8 experts, grouped gate) against the oracles, declined shapes reaching the
  previous forward, ``coverage()`` per layer;
* MiniMax-M2.5 -- the stage's ``self.moe(h, router_logits)`` call with logits the
  caller computed on the GPU."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from flyai_b200 import deepseek, gpt_oss, synth
from oracle import dsv3 as od3
from oracle import m25 as om25
from oracle import v4 as ov4
from oracle.topk import topk_row
from tests.dsv3_util import M25_ULP_FRAC1, assert_close, expert_cache
from tests.golden_util import assert_within_tolerance, bf16_tensor_to_f32
from tests.m25_util import dequant_expert
from tests.v4_util import expert_np, shared_np

pytestmark = pytest.mark.gpu


# ---------------------------------------------------------------- GPT-OSS
def test_gpt_oss_mlp_install_against_the_module_forward(monkeypatch):
    from transformers.integrations.mxfp4 import _convert_moe_packed_tensors
    from transformers.models.gpt_oss.modeling_gpt_oss import GptOssMLP
    monkeypatch.setattr(gpt_oss, "ENABLED", True)
    gpt_oss.reset_coverage()
    layer = synth.make_gpt_oss_layer(num_experts=16, top_k=4, hidden=256, inter=256, seed=8)
    cfg = SimpleNamespace(num_experts_per_tok=4, num_local_experts=16, hidden_size=256,
                          intermediate_size=256, _experts_implementation="eager")
    mlp = GptOssMLP(cfg)
    with torch.no_grad():
        mlp.router.weight.data = layer.router_w.clone()
        mlp.router.bias.data = layer.router_b.clone()
        mlp.experts.gate_up_proj.data = _convert_moe_packed_tensors(layer.w13_blocks, layer.w13_scales)
        mlp.experts.down_proj.data = _convert_moe_packed_tensors(layer.w2_blocks, layer.w2_scales)
        mlp.experts.gate_up_proj_bias.data = layer.w13_bias.clone()
        mlp.experts.down_proj_bias.data = layer.w2_bias.clone()
    mlp = mlp.to(torch.bfloat16)
    x = synth.make_tokens(6, 256, seed=9).view(1, 6, 256)
    with torch.no_grad():
        ref_out, ref_scores = mlp(x)                      # the module's own forward, CPU
    mlp = mlp.cuda()
    holder = SimpleNamespace(mlp=mlp)
    bank = dict(router_weight=layer.router_w, router_bias=layer.router_b,
                gate_up_blocks=layer.w13_blocks, gate_up_scales=layer.w13_scales,
                gate_up_bias=layer.w13_bias, down_blocks=layer.w2_blocks, down_scales=layer.w2_scales,
                down_bias=layer.w2_bias, top_k=4)
    installed = gpt_oss.install([holder], [bank], max_tokens=8)
    assert len(installed) == 1 and gpt_oss.installed_count() == 1
    out, scores = mlp(x.cuda())
    torch.cuda.synchronize()
    assert out.shape == (1, 6, 256) and scores.shape == (6, 4)
    d = np.abs(bf16_tensor_to_f32(scores).astype(np.float64) - bf16_tensor_to_f32(ref_scores))
    assert d.max() <= 2.0 ** -8
    assert_within_tolerance(bf16_tensor_to_f32(out.view(6, 256)), bf16_tensor_to_f32(ref_out.view(6, 256)))
    big = synth.make_tokens(9, 256, seed=10).view(1, 9, 256).cuda()   # 9 > max_tokens: declined
    out9, _ = mlp(big)
    torch.cuda.synchronize()
    assert out9.shape == (1, 9, 256)
    assert gpt_oss.coverage() == {"claimed": 1, "declined:tokens>max_tokens": 1}
    assert gpt_oss.install([holder], [bank])[0] is installed[0]       # no second wrapper


# ---------------------------------------------------------------- DeepSeek
class _Linear(torch.nn.Module):
    def __init__(self, weight, scale):
        super().__init__()
        self.weight = torch.nn.Parameter(weight, requires_grad=False)
        self.weight.scale = self.scale = torch.nn.Parameter(scale, requires_grad=False)


class _Expert(torch.nn.Module):
    def __init__(self, w13, s13, w2, s2, I, sI, swiglu_limit):
        super().__init__()
        self.w1 = _Linear(w13[:I], s13[:sI])
        self.w3 = _Linear(w13[I:], s13[sI:])
        self.w2 = _Linear(w2, s2)
        self.swiglu_limit = swiglu_limit


def _reference_module():
    """A module with the reference's MoE class layout; its forward stands for the
    previous (reference) forward and marks the calls it receives."""
    calls = []

    class MoE(torch.nn.Module):
        def forward(self, x, input_ids):
            calls.append(x.shape)
            return torch.full_like(x, 7.0)
    return SimpleNamespace(MoE=MoE, world_size=1), calls


def _v4_block(mod, layer, layer_id):
    f4, e8 = torch.float4_e2m1fn_x2, torch.float8_e8m0fnu
    moe = mod.MoE()
    E, H, I = layer.num_experts, layer.hidden, layer.inter
    moe.dim, moe.n_routed_experts, moe.layer_id = H, E, layer_id
    moe.experts_start_idx, moe.experts_end_idx = 0, E
    gate = torch.nn.Module()
    gate.weight = torch.nn.Parameter(layer.router_w.cuda(), requires_grad=False)
    gate.hash = layer.tid2eid is not None
    gate.bias = None if gate.hash else torch.nn.Parameter(layer.bias.cuda(), requires_grad=False)
    gate.tid2eid = layer.tid2eid.cuda() if gate.hash else None
    gate.topk, gate.score_func, gate.route_scale = layer.top_k, "sqrtsoftplus", layer.route_scale
    moe.gate = gate
    experts = []
    for e in range(E):
        w13, s13, w2, s2 = (t.cuda() for t in layer.expert(e))
        experts.append(_Expert(w13.view(f4), s13.view(e8), w2.view(f4), s2.view(e8), I, I,
                               layer.swiglu_limit))
    moe.experts = torch.nn.ModuleList(experts)
    w13, s13, w2, s2 = (t.cuda() for t in layer.shared())
    moe.shared_experts = _Expert(w13, s13.view(e8), w2, s2.view(e8), I, I // 128, layer.swiglu_limit)
    return moe


def test_deepseek_v4_lever_claims_decode_and_declines_prefill(monkeypatch):
    monkeypatch.setattr(deepseek, "ENABLED", True)
    mod, calls = _reference_module()
    assert deepseek.install(mod)
    assert not deepseek.install(mod)                       # idempotent
    layer = synth.make_v4_layer(num_experts=32, top_k=6, hidden=256, inter=256, seed=51)
    hashed = synth.make_v4_layer(num_experts=32, top_k=6, hidden=256, inter=256, seed=52, hash_vocab=8)
    blocks = [_v4_block(mod, layer, 3), _v4_block(mod, hashed, 0)]
    model = torch.nn.ModuleList(blocks)
    for blk, lyr in zip(blocks, (layer, hashed)):
        for M in (1, 6):
            x = synth.make_tokens(M, 256, seed=60 + M, device="cuda")
            ii = torch.randint(0, 8, (1, M), device="cuda")
            y = blk(x.view(1, M, 256), ii)
            torch.cuda.synchronize()
            xc = x.float().cpu().numpy()
            tid = lyr.tid2eid.numpy() if lyr.tid2eid is not None else None
            ids, wts, _ = ov4.gate(xc, lyr.router_w.float().numpy(), lyr.bias.numpy(), 6,
                                   lyr.route_scale, tid, ii.view(-1).cpu().numpy())
            y_ref = ov4.moe_forward(xc, ids, wts, expert_np(lyr), shared_np(lyr), lyr.swiglu_limit)
            assert_close(y.view(M, 256).float().cpu().numpy(), y_ref)
    assert not calls
    y = blocks[0](synth.make_tokens(65, 256, seed=1, device="cuda").view(1, 65, 256),
                  torch.zeros(1, 65, dtype=torch.long, device="cuda"))     # prefill: declined
    y_cpu = blocks[0](synth.make_tokens(2, 256, seed=2).view(1, 2, 256), torch.zeros(1, 2, dtype=torch.long))
    assert calls == [(1, 65, 256), (1, 2, 256)] and float(y.flatten()[0]) == 7.0
    cov = deepseek.coverage(model)
    assert cov[3] == (2, {"s>64": 1, "device": 1}) and cov[0] == (2, {})
    deepseek.uninstall(mod)
    assert not getattr(mod.MoE.forward, "_flyai_b200", False)


def test_deepseek_drafter_lever_binds_instances(monkeypatch):
    """install_drafter: the drafter's MoE instances (a T-row block: T x k pairs)
    run on the kernels while other instances of the class keep the reference's
    forward; the result equals the oracle, the class is untouched."""
    monkeypatch.setattr(deepseek, "ENABLED", True)
    mod, calls = _reference_module()
    layer = synth.make_v4_layer(num_experts=32, top_k=6, hidden=256, inter=256, seed=53)
    drafter, main = _v4_block(mod, layer, 0), _v4_block(mod, layer, 1)
    assert deepseek.install_drafter([drafter]) == 1
    assert deepseek.install_drafter([drafter]) == 0            # idempotent
    assert not getattr(mod.MoE.forward, "_flyai_b200", False)  # the class is not rebound
    T = 5                                                       # a drafter block: 5 rows x 6 experts
    x = synth.make_tokens(T, 256, seed=70, device="cuda")
    ii = torch.zeros(1, T, dtype=torch.long, device="cuda")
    y = drafter(x.view(1, T, 256), ii)
    torch.cuda.synchronize()
    xc = x.float().cpu().numpy()
    ids, wts, _ = ov4.gate(xc, layer.router_w.float().numpy(), layer.bias.numpy(), 6, layer.route_scale)
    y_ref = ov4.moe_forward(xc, ids, wts, expert_np(layer), shared_np(layer), layer.swiglu_limit)
    assert_close(y.view(T, 256).float().cpu().numpy(), y_ref)
    main(x.view(1, T, 256), ii)                                 # the reference's forward
    assert calls == [(1, T, 256)]
    assert deepseek.coverage(drafter)[0] == (1, {})
    assert drafter in deepseek.installed()
    deepseek.uninstall_drafter([drafter])
    assert drafter not in deepseek.installed()
    drafter(x.view(1, T, 256), ii)
    assert len(calls) == 2


def test_deepseek_v3_lever_on_fp8_block_with_grouped_gate(monkeypatch):
    monkeypatch.setattr(deepseek, "ENABLED", True)
    mod, calls = _reference_module()
    assert deepseek.install(mod)
    layer = synth.make_dsv3_layer(num_experts=32, top_k=4, hidden=256, inter=256, n_group=4,
                                  topk_group=2, seed=53)
    moe = mod.MoE()
    E, H, I = 32, 256, 256
    moe.dim, moe.n_routed_experts, moe.layer_id = H, E, 1
    moe.experts_start_idx, moe.experts_end_idx = 0, E
    gate = torch.nn.Module()
    gate.weight = torch.nn.Parameter(layer.router_w.cuda(), requires_grad=False)
    gate.e_score_correction_bias = torch.nn.Parameter(layer.bias.cuda(), requires_grad=False)
    gate.num_expert_group, gate.topk_group, gate.top_k = 4, 2, 4
    gate.routed_scaling_factor, gate.moe_router_activation_func = layer.route_scale, "sigmoid"
    moe.gate = gate
    ex = []
    for e in range(E + 1):
        w13, s13, w2, s2 = (t.cuda() for t in layer.expert(e))
        ex.append(_Expert(w13, s13, w2, s2, I, I // 128, 0.0))
    moe.experts = torch.nn.ModuleList(ex[:E])
    moe.shared_experts = ex[E]
    x = synth.make_tokens(5, 256, seed=54, device="cuda")
    y = moe(x.view(1, 5, 256), torch.zeros(1, 5, dtype=torch.long, device="cuda"))
    torch.cuda.synchronize()
    xc = x.float().cpu().numpy()
    ids, wts, _ = od3.gate(xc, layer.router_w.float().numpy(), layer.bias.numpy(), 4, 4, 2, layer.route_scale)
    assert_close(y.view(5, 256).float().cpu().numpy(), od3.moe_forward(xc, ids, wts, expert_cache(layer), E))
    assert not calls
    assert deepseek.coverage(moe) == {1: (1, {})}
    deepseek.uninstall(mod)


# ---------------------------------------------------------------- MiniMax-M2.5
def test_m25_stage_moe_call_routes_from_passed_logits():
    """The stage computes rl = F.linear(h, gate) on the GPU and calls moe(h, rl)."""
    from flyai_b200.m25 import Nvfp4MoE
    layer = synth.make_m25_layer(num_experts=64, top_k=8, hidden=256, inter=256, seed=55)
    moe = Nvfp4MoE.from_layer(layer, max_tokens=64, device="cuda")
    for M in (5, 64):
        h = synth.make_tokens(M, 256, seed=56 + M, device="cuda")
        rl = torch.nn.functional.linear(h, layer.router_w.cuda())          # cuBLAS bf16 logits
        y = moe(h, rl)
        torch.cuda.synchronize()
        assert moe.read_error()[0] == 0
        lg = rl.float().cpu().numpy()
        scores = (1.0 / (1.0 + np.exp(-lg.astype(np.float32)))).astype(np.float32)
        choice = (scores + layer.bias.numpy()).astype(np.float32)
        ids = np.array([topk_row(r, 8, sorted=False) for r in choice], dtype=np.int64)
        wts = np.zeros((M, 8), np.float32)
        for t in range(M):                    # unbiased scores / their sum in slot order
            w = scores[t, ids[t]]
            s = np.float32(0.0)
            for v in w:
                s = np.float32(s + v)
            wts[t] = (w / s).astype(np.float32)
        y_ref = om25.moe_forward(h.float().cpu().numpy(), ids, wts, lambda e: dequant_expert(layer, e))
        assert_close(y.float().cpu().numpy(), y_ref, ulp_frac1=M25_ULP_FRAC1)
        y_own = moe(h)                                                      # the layer's own router
        torch.cuda.synchronize()
        assert y_own.shape == y.shape
