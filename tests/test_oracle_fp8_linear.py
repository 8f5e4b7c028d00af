"""Pin the dense FP8 linear oracle (oracle/fp8_linear.py) against fixtures
produced by the reference itself (tests/golden/make_golden_fp8_linear.py runs the
vendored ``linear`` with the reference's CPU kernels), plus known answers."""
import glob
import hashlib
import os

import numpy as np
import pytest
import torch

from flyai_b200 import synth
from oracle import dsv3, v4
from oracle import fp8_linear as ol
from oracle.fp import bf16_bits_to_f32

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "lin_*.npz")))


def load_case(path):
    f = dict(np.load(path))
    N, K, M, seed, e8m0 = (int(f[k]) for k in ("N", "K", "M", "seed", "e8m0"))
    w, s = synth.make_fp8_linear(N, K, seed=seed, e8m0=bool(e8m0))
    x = synth.make_tokens(M, K, seed=seed)
    h = hashlib.sha256()
    for t in (w, s, x):
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    assert h.hexdigest() == str(f["digest"]), "synth generator drifted from the fixture's inputs"
    return f, w, s, x, bool(e8m0)


def test_fixtures_present():
    assert len(GOLDEN) >= 6


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_oracle_matches_reference_fixture(path):
    f, w, s, x, e8m0 = load_case(path)
    y = ol.linear(x.float().numpy(), w.view(torch.uint8).numpy(), s.numpy(), "ue8m0" if e8m0 else None)
    y_ref = bf16_bits_to_f32(f["y"])
    # the reference's CPU kernels dequantise and multiply (one fp32 sum over K);
    # the oracle keeps fp8_gemm_kernel's per-128-block chain: the same values to
    # fp32 rounding, within one bf16 ulp at the output's peak
    d = np.abs(y - y_ref)
    peak = np.abs(y_ref).max()
    assert d.max() <= np.exp2(np.floor(np.log2(peak)) - 7), (d.max(), peak)
    assert (d == 0).mean() > 0.97, (d == 0).mean()


@pytest.mark.parametrize("e8m0", [True, False])
def test_chain_agrees_with_dense_dequant_product(e8m0):
    w, s = synth.make_fp8_linear(256, 1024, seed=7, e8m0=e8m0)
    x = synth.make_tokens(9, 1024, seed=7).float().numpy()
    wb = w.view(torch.uint8).numpy()
    if e8m0:
        qa, sa = v4.act_quant(x)
        dense = v4.fp8_gemm(qa, sa, wb, s.numpy())
    else:
        qa, sa = dsv3.act_quant(x)
        dense = dsv3.fp8_gemm(qa, sa, wb, s.numpy())
    chain = ol.fp8_gemm_chain(qa, sa, wb, s.numpy())
    d = np.abs(chain - dense)
    assert d.max() <= np.exp2(np.floor(np.log2(np.abs(dense).max())) - 7)
    assert (d == 0).mean() > 0.97


def test_one_hot_row_reads_one_weight_column():
    """ue8m0: x = e_k gives scale 2^-8, q = 256 at k, so y[n] = W[n, k] * s_w exactly."""
    N, K, k = 256, 512, 300
    w, s = synth.make_fp8_linear(N, K, seed=3, e8m0=True)
    x = np.zeros((1, K), np.float32)
    x[0, k] = 1.0
    y = ol.linear(x, w.view(torch.uint8).numpy(), s.numpy(), "ue8m0")
    col = w.float().numpy()[:, k] * np.repeat(v4.e8m0(s.numpy()), 128, axis=0)[:, k // 128]
    np.testing.assert_array_equal(y[0], col)


def test_blocks_accumulate_in_ascending_k():
    """The fold, step by step: block 0 (weight scale 1) gives acc = D_0 * Scale_C0,
    block 1 (weight scale 2^30) one fused multiply-add onto it, then bf16."""
    K = 256
    w = torch.zeros(128, K, dtype=torch.float8_e4m3fn)
    w[:, 0] = 1.0
    w[:, 128] = 1.0
    s = torch.tensor([[1.0, 2.0 ** 30]], dtype=torch.float32)
    x = np.zeros((1, K), np.float32)
    x[0, 0] = 1.0
    x[0, 128] = 1.0
    y = ol.linear(x, w.view(torch.uint8).numpy(), s.numpy(), None)
    # per block: D = 448 * 1, Scale_C = (1/448 rounded) * s_w; block 0 first
    inv = np.float32(1.0 / 448.0)
    a = np.float32(np.float32(448.0) * np.float32(inv * np.float32(1.0)))
    b = np.float32(np.float64(448.0) * np.float64(np.float32(inv * np.float32(2.0 ** 30))) + np.float64(a))
    assert y[0, 0] == np.float32(torch.tensor(b).bfloat16().float().item())
