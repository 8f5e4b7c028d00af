"""Pin the DeepSeek-V4 W4A8 oracle (oracle/v4.py) against fixtures produced by the
reference itself (tests/golden/make_golden_v4.py runs the vendored MoE with the
reference's CPU kernels), at small shapes and at the V4-Flash shape, score- and
hash-routed; plus known answers for the pieces."""
import glob
import os

import numpy as np
import pytest

from oracle import v4
from oracle.fp import bf16_bits_to_f32
from tests.v4_util import digest_ok, load_case, oracle_case

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "v4_*.npz")))


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_v4_oracle_matches_reference_fixture(path):
    case = load_case(path)
    assert digest_ok(case), "synth generator drifted from the fixture's inputs"
    f = case["fixture"]
    out = oracle_case(case)
    np.testing.assert_array_equal(out["ids"], f["ids"])          # torch's sorted order, ties too
    np.testing.assert_allclose(out["wts"], f["wts"], rtol=2e-6, atol=1e-9)
    np.testing.assert_allclose(out["logits"], f["logits"], rtol=1e-5, atol=1e-5)
    y_ref = bf16_bits_to_f32(f["y"])
    d = np.abs(out["y"] - y_ref)
    peak = np.abs(y_ref).max()
    # same arithmetic in another fp32 summation order: bit-identical on the small
    # cases, within one bf16 ulp at the output's peak on the full-size ones
    assert d.max() <= np.exp2(np.floor(np.log2(peak)) - 7), (d.max(), peak)
    assert (d == 0).mean() > 0.95
    if os.path.basename(path) == "v4_small_hash.npz":   # 8 token ids: repeats inside tid2eid rows
        assert any(len(set(r)) < len(r) for r in f["ids"].tolist()), "no repeated expert exercised"


def test_act_quant_ue8m0_known_answers():
    # power-of-two scale 2^ceil(log2(amax/448)), exact at powers of two
    x = np.zeros((3, 128), np.float32)
    x[0, 0] = 448.0                    # amax/448 = 1 -> scale 1
    x[1, 0] = 449.0                    # just above -> scale 2
    x[2, :] = 1e-6                     # amax floored at 1e-4
    q, s = v4.act_quant(x)
    assert s[0, 0] == 1.0 and s[1, 0] == 2.0
    assert s[2, 0] == 2.0 ** np.ceil(np.log2(np.float32(1e-4) * np.float32(1 / 448)))
    assert q[0, 0] == 448.0 and q[1, 0] == 224.0


def test_fp4_dequant_and_gemm_known_answers():
    # low nibble = even K; e8m0 per 32; one-hot activation picks one weight
    w = np.zeros((2, 64), np.uint8)    # N = 2, K = 128 (packed 64 bytes)
    w[0, 0] = 0x21                     # K0 = 0.5, K1 = 1.0
    w[1, 63] = 0xF7                    # K126 = 6.0, K127 = -6.0
    s = np.full((2, 4), 127, np.uint8)
    s[1, 3] = 128                      # last 32-block of row 1 scaled by 2
    d = v4.dequant_fp4(w, s)
    assert d[0, 0] == 0.5 and d[0, 1] == 1.0 and d[1, 126] == 12.0 and d[1, 127] == -12.0
    a = np.zeros((1, 128), np.float32)
    a[0, 127] = 1.0
    qa, sa = v4.act_quant(a)
    out = v4.fp4_gemm(qa, sa, w, s)
    assert out[0, 0] == 0.0 and out[0, 1] == -12.0


def test_duplicate_slots_keep_only_the_last():
    assert v4.keep_last_of_each([3, 5, 3, 7, 5, 5]) == [False, False, True, True, False, True]
    assert v4.keep_last_of_each([1, 2, 3]) == [True, True, True]


def test_sqrtsoftplus_threshold():
    v = np.array([-30.0, 0.0, 19.5, 20.0, 20.5, 50.0], np.float32)
    got = v4.sqrtsoftplus(v)
    ref = np.sqrt(np.where(v > 20, v, np.log1p(np.exp(v.astype(np.float64))))).astype(np.float32)
    np.testing.assert_allclose(got, ref, rtol=2e-7)
