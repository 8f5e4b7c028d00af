"""GPU parity of the DeepSeek-V4 W4A8 layer (C ABI; tcgen05 kind::mxf8f6f4 with the
fp4 weights expanded to e4m3 in shared memory) against the fixtures the reference
produced and the CPU oracle.  Routing: the reference's ids slot for slot
(torch.topk sorted, or tid2eid on a hash-routed layer) and weights within fp32
rounding; output: the layer tolerance plus bf16-step bounds."""
import glob
import os

import numpy as np
import pytest
import torch

from flyai_b200 import synth
from flyai_b200.moe import launch_count
from flyai_b200.v4 import W4A8MoE
from oracle import v4 as ov4
from oracle.fp import bf16_bits_to_f32
from tests.dsv3_util import assert_close, assert_same_routing, stable_plan
from tests.v4_util import expert_np, load_case, oracle_case, shared_np

pytestmark = pytest.mark.gpu
GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "v4_*.npz")))
# fraction of outputs within one bf16 step of the reference (the layer re-quantises
# its SwiGLU rows to e4m3, like DeepSeek-V3; measured on the full-size fixtures)
V4_ULP_FRAC1 = 0.98


def f32(t):
    return t.detach().float().cpu().numpy()


def run(moe, x, input_ids=None):
    M = x.shape[0]
    logits, ids_r, wts_r = moe.route(x, input_ids)
    ids = torch.empty(M, moe.top_k, dtype=torch.int32, device=x.device)
    wts = torch.empty(M, moe.top_k, dtype=torch.float32, device=x.device)
    y = moe.forward(x, input_ids, ids=ids, wts=wts)
    torch.cuda.synchronize()
    return dict(logits=f32(logits), ids_route=ids_r.cpu().numpy(), wts_route=f32(wts_r),
                ids=ids.cpu().numpy(), wts=f32(wts), y=f32(y))


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_v4_layer_matches_reference_fixture(path):
    case = load_case(path)
    f = case["fixture"]
    M = case["x"].shape[0]
    touched = sorted(set(int(v) for v in f["ids"].ravel()))
    moe = W4A8MoE.from_layer(case["layer"], max_tokens=max(M, 1), device="cuda", experts=touched)
    n0 = launch_count()
    ii = case["input_ids"].cuda() if int(f["hash_vocab"]) else None
    out = run(moe, case["x"].cuda(), ii)
    assert launch_count() > n0
    assert moe.read_error()[0] == 0
    for ids, wts in ((out["ids"], out["wts"]), (out["ids_route"], out["wts_route"])):
        assert_same_routing(ids, wts, f["ids"], f["wts"])
    np.testing.assert_allclose(out["logits"], f["logits"], rtol=1e-4, atol=1e-4)
    m = assert_close(out["y"], bf16_bits_to_f32(f["y"]), ulp_frac1=V4_ULP_FRAC1)
    print(os.path.basename(path), m)


@pytest.fixture(scope="module")
def full_layer():
    """The V4-Flash MoE shape (256 fp4 routed experts + the fp8 shared expert, H 4096,
    I 2048), every expert generated on the GPU and packed (3.3 GB of banks)."""
    layer = synth.make_v4_layer(**synth.V4, seed=7, device="cuda")
    moe = W4A8MoE.from_layer(layer, max_tokens=64, device="cuda")
    torch.cuda.synchronize()
    yield layer, moe
    del moe
    torch.cuda.empty_cache()


@pytest.mark.parametrize("M", [1, 6, 32, 64])
def test_full_size_layer_matches_oracle(full_layer, M):
    layer, moe = full_layer
    x = synth.make_tokens(M, layer.hidden, seed=500 + M, device="cuda")
    out = run(moe, x)
    assert moe.read_error()[0] == 0
    xc = x.float().cpu().numpy()
    ids, wts, logits = ov4.gate(xc, layer.router_w.float().cpu().numpy(), layer.bias.cpu().numpy(),
                                layer.top_k, layer.route_scale)
    assert_same_routing(out["ids"], out["wts"], ids, wts)
    sub = sorted(set([0, M // 2, M - 1]))
    y_ref = ov4.moe_forward(xc[sub], ids[sub], wts[sub], expert_np(layer), shared_np(layer),
                            layer.swiglu_limit)
    m = assert_close(out["y"][sub], y_ref, ulp_frac1=V4_ULP_FRAC1)
    print("M", M, m)


def test_hash_routed_layer_with_repeated_experts():
    """tid2eid names the same expert twice for some tokens: the fold keeps only the
    last slot of a repeated expert, as the reference's y[idx] += does."""
    layer = synth.make_v4_layer(num_experts=32, top_k=6, hidden=256, inter=256, seed=17,
                                hash_vocab=16)
    g = torch.Generator().manual_seed(5)
    ii = torch.randint(0, 16, (40,), generator=g)
    moe = W4A8MoE.from_layer(layer, max_tokens=64, device="cuda")
    x = synth.make_tokens(40, 256, seed=18, device="cuda")
    out = run(moe, x, ii.cuda())
    assert moe.read_error()[0] == 0
    xc = x.float().cpu().numpy()
    ids, wts, _ = ov4.gate(xc, layer.router_w.float().numpy(), layer.bias.numpy(), 6, layer.route_scale,
                           layer.tid2eid.numpy(), ii.numpy())
    assert any(len(set(r)) < len(r) for r in ids.tolist())
    assert_same_routing(out["ids"], out["wts"], ids, wts)
    y_ref = ov4.moe_forward(xc, ids, wts, expert_np(layer), shared_np(layer), layer.swiglu_limit)
    assert_close(out["y"], y_ref, ulp_frac1=V4_ULP_FRAC1)


def test_hash_input_id_out_of_range_is_reported():
    layer = synth.make_v4_layer(num_experts=32, top_k=6, hidden=256, inter=256, seed=19,
                                hash_vocab=8)
    moe = W4A8MoE.from_layer(layer, max_tokens=8, device="cuda")
    x = synth.make_tokens(3, 256, seed=20, device="cuda")
    ii = torch.tensor([1, 99, 2], dtype=torch.int32, device="cuda")   # 99 >= vocab
    y = moe.forward(x, ii)
    torch.cuda.synchronize()
    assert moe.read_error()[0] & 2
    assert torch.isfinite(y.float()).all()
    moe.forward(x, torch.tensor([1, 3, 2], dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    assert moe.read_error()[0] == 0


@pytest.mark.parametrize("M,expert_range", [(1, None), (6, None), (64, None), (33, (8, 40))])
def test_plan_is_stable_argsort_of_routing(M, expert_range):
    layer = synth.make_v4_layer(num_experts=64, top_k=6, hidden=256, inter=256, seed=23)
    moe = W4A8MoE.from_layer(layer, max_tokens=64, device="cuda", expert_range=expert_range)
    x = synth.make_tokens(M, 256, seed=1300 + M, device="cuda")
    _, ids, _ = moe.route(x, logits=False)
    counts, offsets, perm = moe.read_plan(M)
    torch.cuda.synchronize()
    ref_ids, _, _ = ov4.gate(x.float().cpu().numpy(), layer.router_w.float().numpy(),
                             layer.bias.numpy(), 6, layer.route_scale)
    np.testing.assert_array_equal(ids.cpu().numpy(), ref_ids)
    lo, hi = expert_range or (0, layer.num_experts)
    ref_counts, ref_offsets, ref_perm = stable_plan(ref_ids, lo, hi)
    np.testing.assert_array_equal(counts.cpu().numpy(), ref_counts)
    np.testing.assert_array_equal(offsets.cpu().numpy(), ref_offsets)
    np.testing.assert_array_equal(perm.cpu().numpy()[:len(ref_perm)], ref_perm)
    assert moe.read_error()[0] == 0


def test_repeated_calls_and_shards_sum_to_full_layer():
    layer = synth.make_v4_layer(num_experts=64, top_k=6, hidden=256, inter=256, seed=29)
    full = W4A8MoE.from_layer(layer, max_tokens=64, device="cuda")
    xs = [synth.make_tokens(M, 256, seed=600 + M, device="cuda") for M in (3, 64, 1, 17)]
    first = [full.forward(x).clone() for x in xs]
    again = [full.forward(x).clone() for x in reversed(xs)][::-1]
    torch.cuda.synchronize()
    for a, b in zip(first, again):
        assert torch.equal(a, b)
    shards = [W4A8MoE.from_layer(layer, max_tokens=64, device="cuda", expert_range=r)
              for r in ((0, 16), (16, 64))]
    for x, y_full in zip(xs, first):
        M = x.shape[0]
        rows = None
        for sh in shards:
            sh.route(x, logits=False)
            r = sh.experts_pairs(x)
            r = torch.cat([r, torch.zeros(full.pair_rows(M) - r.shape[0], 256, dtype=r.dtype,
                                          device=r.device)]) if r.shape[0] < full.pair_rows(M) else r
            rows = r.float() if rows is None else rows + r.float()
        y = shards[0].combine(rows.bfloat16(), M)
        torch.cuda.synchronize()
        assert torch.equal(y, y_full), M
    for m in shards + [full]:
        assert m.read_error()[0] == 0


def test_cuda_graph_replay_matches_eager():
    layer = synth.make_v4_layer(num_experts=64, top_k=6, hidden=256, inter=256, seed=31)
    moe = W4A8MoE.from_layer(layer, max_tokens=8, device="cuda")
    x = synth.make_tokens(5, 256, seed=32, device="cuda")
    y_eager = moe.forward(x).clone()
    static_y = torch.empty_like(y_eager)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        moe.forward(x, out=static_y)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        moe.forward(x, out=static_y)
    static_y.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(static_y, y_eager)
    assert moe.read_error()[0] == 0
