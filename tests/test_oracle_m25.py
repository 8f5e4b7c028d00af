"""Pin the MiniMax-M2.5 NVFP4 oracle (oracle/m25.py) against fixtures produced by
the reference arithmetic itself (tests/golden/make_golden_m25.py runs HF
transformers' MiniMaxM2SparseMoeBlock on NVFP4-dequantised weights), one of them
at the full M2.5 shape."""
import glob
import os

import numpy as np
import pytest

from oracle import m25
from oracle.fp import bf16_bits_to_f32
from tests.dsv3_util import M25_ULP_FRAC1, assert_close
from tests.m25_util import (bf16_module_distance, digest_ok, exact_in_bf16, fixture_y, is_f32_fixture,
                            load_case, metrics_of, oracle_case)

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "m25_*.npz")))


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_m25_oracle_matches_reference_fixture(path):
    case = load_case(path)
    assert digest_ok(case), "synth generator drifted from the fixture's inputs"
    f = case["fixture"]
    if is_f32_fixture(case):
        # HF's experts in fp32 on the exact NVFP4 weights at the config's own 1e-2 global
        # scale: the oracle's exact-weight bf16 chain is at least as close to it as
        # HF's own bf16 module (bf16-held weights) is
        out = oracle_case(case)
        np.testing.assert_array_equal(out["ids"], f["ids"])
        np.testing.assert_array_equal(out["logits"], bf16_bits_to_f32(f["logits"]))
        m = metrics_of(out["y"], f["y_f32"])
        ref = bf16_module_distance(case)
        assert m["rel_l2"] <= ref, (m, ref)
        print("oracle vs HF fp32 exact", m, "HF bf16 module", ref)
        return
    # bf16-held weights: the HF module's own arithmetic, pinned closely
    out = oracle_case(case, bf16_weights=True)
    np.testing.assert_array_equal(out["ids"], f["ids"])   # torch's unsorted order too
    np.testing.assert_array_equal(out["logits"], bf16_bits_to_f32(f["logits"]))
    np.testing.assert_allclose(out["wts"], f["wts"], rtol=2e-6, atol=1e-9)
    m = assert_close(out["y"], fixture_y(case), rel_l2=2e-3, ulp_frac1=M25_ULP_FRAC1)
    assert m["exact_frac"] > 0.98, m
    # exact NVFP4 weights (what the tensor-core path computes with): identical when
    # the global scale is a power of two, else off by the bf16 weight rounding
    exact = oracle_case(case)["y"]
    if exact_in_bf16(case):
        np.testing.assert_array_equal(exact, out["y"])
    else:
        me = metrics_of(exact, fixture_y(case))
        assert me["rel_l2"] < 1e-2, me


def test_nvfp4_dequant_known_answers():
    # nibble order (low = even K), e4m3 block-16 scale, global scale, bf16 rounding
    blocks = np.array([[0x21] + [0] * 7 + [0xF7] + [0] * 7], dtype=np.uint8)   # K = 32
    scales = np.array([[0x38, 0x40]], dtype=np.uint8)   # e4m3 1.0 and 2.0
    w = m25.dequant_nvfp4(blocks, scales, 0.5)
    assert w[0, 0] == 0.25 and w[0, 1] == 0.5          # 0.5*1*0.5, 1.0*1*0.5
    assert w[0, 16] == 6.0 and w[0, 17] == -6.0        # 6*2*0.5, -6*2*0.5
    assert not w[0, 2:16].any()
