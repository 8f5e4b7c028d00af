"""Dense FP8 linear on the B200 (flyai_fp8_linear) against the CPU oracle of the
reference's ``linear`` on an fp8 weight (oracle/fp8_linear.py).

Tolerance: every element within one bf16 ulp of its own magnitude or one ulp at
the output's peak, and at least 99 % bit-identical.  The oracle's per-block dot
products are exact and rounded once, and its fp32 chain runs over all of K; the
kernel's dot products come from the tensor core, and it adds the chains of
512-element pieces of K, so a few elements may sit one bf16 step away.
"""
import numpy as np
import pytest
import torch

from flyai_b200 import synth
from flyai_b200.linear import Fp8Linear
from oracle import fp8_linear as ol
from tests.dsv3_util import bf16_ulp
from tests.golden_util import bf16_peak_ulp

pytestmark = pytest.mark.gpu


def _oracle(x, w, s, scale_fmt):
    return ol.linear(x.float().numpy(), w.view(torch.uint8).numpy(), s.numpy(), scale_fmt)


def assert_linear_close(y, ref, exact_frac=0.99):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    bound = np.maximum(bf16_ulp(ref), bf16_peak_ulp(ref))
    d = np.abs(y - ref)
    assert np.isfinite(y).all()
    assert (d <= bound).all(), (float(d.max()), int((d > bound).sum()))
    frac = float((y == ref).mean())
    assert frac >= exact_frac, frac
    return frac


@pytest.mark.parametrize("M", [1, 2, 5, 16, 17, 33, 64])
@pytest.mark.parametrize("e8m0,scale_fmt", [(True, "ue8m0"), (False, None)])
def test_small_shapes_match_oracle(M, e8m0, scale_fmt):
    N, K = 384, 1024
    w, s = synth.make_fp8_linear(N, K, seed=M, e8m0=e8m0)
    x = synth.make_tokens(M, K, seed=M)
    lin = Fp8Linear(w, s, scale_fmt=scale_fmt, max_tokens=M)
    y = lin(x.cuda())
    torch.cuda.synchronize()
    assert lin.read_error() == 0
    assert_linear_close(y.float().cpu().numpy(), _oracle(x, w, s, scale_fmt))


@pytest.mark.parametrize("name", ["wq_a", "wkv", "shared_w2", "idx_wq_b", "wo_b"])
def test_v4_decode_shapes_match_oracle(name):
    """The V4 layer's single-row GEMMs at M=1 and a verify batch of 4."""
    N, K = synth.V4_LINEARS[name]
    w, s = synth.make_fp8_linear(N, K, seed=3, e8m0=True)
    lin = Fp8Linear(w, s, scale_fmt="ue8m0", max_tokens=4)
    for M in (1, 4):
        x = synth.make_tokens(M, K, seed=10 + M)
        y = lin(x.cuda())
        assert_linear_close(y.float().cpu().numpy(), _oracle(x, w, s, "ue8m0"))
    assert lin.read_error() == 0


def test_wide_bank_matches_oracle_on_sampled_rows():
    """wq_b [32768, 1024]: every row block whole in one CTA's share."""
    N, K = synth.V4_LINEARS["wq_b"]
    w, s = synth.make_fp8_linear(N, K, seed=5, e8m0=True)
    lin = Fp8Linear(w, s, scale_fmt="ue8m0", max_tokens=2)
    x = synth.make_tokens(2, K, seed=5)
    y = lin(x.cuda()).float().cpu().numpy()
    rows = np.r_[0:256, 16384:16640, N - 256:N]
    ref = ol.linear(x.float().numpy(), w.view(torch.uint8).numpy()[rows],
                    np.repeat(s.numpy(), 128, axis=0)[rows][::128], "ue8m0")
    assert_linear_close(y[:, rows], ref)


def test_long_k_matches_oracle_on_sampled_rows():
    """K = 32768 (256 K blocks, 64 pieces per row block) at 16 tokens."""
    N, K = 4096, 32768
    w, s = synth.make_fp8_linear(N, K, seed=13, e8m0=False, device="cuda")
    lin = Fp8Linear(w, s, scale_fmt=None, max_tokens=16)
    x = synth.make_tokens(16, K, seed=13)
    y = lin(x.cuda()).float().cpu().numpy()
    rows = np.r_[0:128, 2048:2176, N - 128:N]
    wr = w.view(torch.uint8)[torch.as_tensor(rows, device="cuda")].cpu().numpy()
    sr = s.cpu().numpy()[rows[::128] // 128]
    assert_linear_close(y[:, rows], ol.linear(x.float().numpy(), wr, sr, None))
    assert lin.read_error() == 0


def test_stacked_bank_is_the_concatenation():
    """[w1; w3] as one bank = the two linears side by side, bit for bit: the
    arithmetic of an output depends on K only, not on which CTA computed it."""
    K = 4096
    w1, s1 = synth.make_fp8_linear(2048, K, seed=1)
    w3, s3 = synth.make_fp8_linear(2048, K, seed=2)
    x = synth.make_tokens(3, K, seed=4)
    fused = Fp8Linear([w1, w3], [s1, s3], scale_fmt="ue8m0", max_tokens=3)
    y = fused(x.cuda())
    assert y.shape == (3, 4096)
    g, u = fused.split(y)
    for part, w, s in ((g, w1, s1), (u, w3, s3)):
        alone = Fp8Linear(w, s, scale_fmt="ue8m0", max_tokens=3)(x.cuda())
        assert torch.equal(part, alone)
        assert_linear_close(part.float().cpu().numpy(), _oracle(x, w, s, "ue8m0"))


def test_small_workspace_runs_in_token_slices():
    """A workspace sized for 4 tokens serves 11 in launches of 4, the same bits."""
    N, K = 512, 2048
    w, s = synth.make_fp8_linear(N, K, seed=12)
    x = synth.make_tokens(11, K, seed=12).cuda()
    big = Fp8Linear(w, s, scale_fmt="ue8m0", max_tokens=16)
    small = Fp8Linear(w, s, scale_fmt="ue8m0", max_tokens=4)
    assert small.workspace.numel() < big.workspace.numel()
    assert torch.equal(small(x), big(x))


def test_repeat_calls_are_deterministic_and_slices_cover_large_batches():
    N, K = 1024, 4096
    w, s = synth.make_fp8_linear(N, K, seed=9, e8m0=False)
    lin = Fp8Linear(w, s, scale_fmt=None, max_tokens=130)
    x = synth.make_tokens(130, K, seed=9).cuda()
    a = lin(x)
    b = lin(x)
    assert torch.equal(a, b)
    # rows past 64 run in later launches; each slice equals its own call
    assert torch.equal(a[64:128], lin(x[64:128].contiguous()))
    assert torch.equal(a[128:], lin(x[128:].contiguous()))
    ref = _oracle(x[:8].cpu(), w, s, None)
    assert_linear_close(a[:8].float().cpu().numpy(), ref)
    empty = lin(x[:0])
    assert empty.shape == (0, N)
    assert lin.read_error() == 0


def test_out_argument_and_leading_dims():
    N, K = 256, 512
    w, s = synth.make_fp8_linear(N, K, seed=11)
    lin = Fp8Linear(w, s, scale_fmt="ue8m0", max_tokens=6)
    x = synth.make_tokens(6, K, seed=11).cuda().view(2, 3, K)
    out = torch.empty(2, 3, N, dtype=torch.bfloat16, device="cuda")
    y = lin(x, out=out)
    assert y.data_ptr() == out.data_ptr()
    assert torch.equal(y.view(6, N), lin(x.view(6, K)))
