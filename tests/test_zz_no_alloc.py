"""flyai_moe_forward_noalloc: the layer for callers that cannot supply device memory.

Some hosts of this library have no way to hand it a workspace -- a program that
reaches it over an FFI (cgo, JNI, N-API) with no CUDA allocator of its own, or a
serving loop whose device-memory budget is fixed at start-up.  The no-allocation
entry point keeps its intermediate data in a static device array inside the
library.  These tests call it through the C ABI, twice in a row on different
batches (the array keeps the previous call's contents), and check each result
against the regular workspace entry point within the parity tolerance; they also
check that a descriptor too large for the array is refused.

This file is collected last so that, in a run that stops at the first failure,
every other test has already run.
"""
import ctypes

import numpy as np
import pytest
import torch

from flyai_b200 import _lib, synth
from flyai_b200.moe import Mxfp4MoE
from tests.golden_util import assert_within_tolerance, bf16_tensor_to_f32

pytestmark = pytest.mark.gpu


def _noalloc(moe, x):
    M = x.shape[0]
    y = torch.empty(M, moe.hidden, dtype=torch.bfloat16, device=moe.device)
    ids = torch.empty(M, moe.top_k, dtype=torch.int32, device=moe.device)
    wts = torch.empty(M, moe.top_k, dtype=torch.bfloat16, device=moe.device)
    st = _lib.load().flyai_moe_forward_noalloc(
        ctypes.byref(moe.desc), M, ctypes.c_void_p(x.data_ptr()), ctypes.byref(moe.weights),
        ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(ids.data_ptr()),
        ctypes.c_void_p(wts.data_ptr()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _lib.OK, _lib.load().flyai_moe_strerror(st).decode()
    return y, ids, wts


def test_noalloc_matches_workspace_entry_point_twice():
    layer = synth.make_gpt_oss_layer(**synth.GPT_OSS_120B, seed=5, device="cuda")
    moe = Mxfp4MoE.from_layer(layer, max_tokens=64, device="cuda")
    n = ctypes.c_size_t()
    _lib.call("flyai_moe_workspace_bytes", ctypes.byref(moe.desc), ctypes.byref(n))
    assert n.value <= 8 << 20
    for M, seed in ((64, 1), (5, 2)):              # two calls in a row, different batches
        x = synth.make_tokens(M, 2880, seed=seed, device="cuda")
        y_ref, ids_ref, w_ref = moe.forward(x)
        y, ids, wts = _noalloc(moe, x)
        torch.cuda.synchronize()
        assert torch.equal(ids, ids_ref)
        assert torch.equal(wts, w_ref)
        assert_within_tolerance(bf16_tensor_to_f32(y), bf16_tensor_to_f32(y_ref))


def test_noalloc_refuses_descriptor_beyond_its_array():
    layer = synth.make_gpt_oss_layer(num_experts=8, top_k=4, hidden=256, inter=128, seed=1,
                                     device="cuda")
    moe = Mxfp4MoE.from_layer(layer, max_tokens=16, device="cuda")
    big = _lib.Desc.from_buffer_copy(moe.desc)
    big.max_tokens = 8192                           # workspace far beyond 8 MiB
    x = synth.make_tokens(4, 256, seed=0, device="cuda")
    y = torch.empty(4, 256, dtype=torch.bfloat16, device="cuda")
    st = _lib.load().flyai_moe_forward_noalloc(
        ctypes.byref(big), 4, ctypes.c_void_p(x.data_ptr()), ctypes.byref(moe.weights),
        ctypes.c_void_p(y.data_ptr()), None, None,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _lib.ERR_WORKSPACE
    y1, ids1, _ = _noalloc(moe, x)                  # a valid call still works afterwards
    y0, ids0, _ = moe.forward(x)
    torch.cuda.synchronize()
    assert torch.equal(ids1, ids0)
    np.testing.assert_array_equal(bf16_tensor_to_f32(y1), bf16_tensor_to_f32(y0))


def _noalloc_fp(moe, x):
    """The no-allocation call for an FP8 or NVFP4 layer (fp32 routing weights)."""
    M = x.shape[0]
    y = torch.empty(M, moe.hidden, dtype=torch.bfloat16, device=x.device)
    ids = torch.empty(M, moe.top_k, dtype=torch.int32, device=x.device)
    wts = torch.empty(M, moe.top_k, dtype=torch.float32, device=x.device)
    st = _lib.load().flyai_moe_forward_noalloc(
        ctypes.byref(moe.desc), M, ctypes.c_void_p(x.data_ptr()), ctypes.byref(moe.weights),
        ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(ids.data_ptr()),
        ctypes.c_void_p(wts.data_ptr()), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _lib.OK, _lib.load().flyai_moe_strerror(st).decode()
    return y, ids, wts


def test_noalloc_array_shared_across_weight_formats():
    """One array serves every descriptor: calls alternate between an MXFP4, an NVFP4
    and an FP8 layer (whose intermediate data sit at different offsets of the array)
    and each result equals the workspace entry point's for the same layer."""
    from flyai_b200.dsv3 import Fp8MoE
    from flyai_b200.m25 import Nvfp4MoE
    mx = Mxfp4MoE.from_layer(synth.make_gpt_oss_layer(num_experts=32, top_k=4, hidden=256,
                                                      inter=192, seed=3), max_tokens=16, device="cuda")
    nv = Nvfp4MoE.from_layer(synth.make_m25_layer(num_experts=64, top_k=8, hidden=256, inter=256,
                                                  seed=4), max_tokens=16, device="cuda")
    f8 = Fp8MoE.from_layer(synth.make_dsv3_layer(num_experts=32, top_k=4, hidden=256, inter=128,
                                                 n_group=4, topk_group=2, seed=5),
                           max_tokens=16, device="cuda")
    for rnd in range(2):
        for name, moe in (("mxfp4", mx), ("nvfp4", nv), ("fp8", f8)):
            x = synth.make_tokens(5 + 4 * rnd, 256, seed=50 + rnd, device="cuda")
            if name == "mxfp4":
                y_ref, ids_ref, _ = moe.forward(x)
                y, ids, _ = _noalloc(moe, x)
            else:
                ids_ref = torch.empty(x.shape[0], moe.top_k, dtype=torch.int32, device="cuda")
                wts_ref = torch.empty(x.shape[0], moe.top_k, dtype=torch.float32, device="cuda")
                y_ref = moe.forward(x, ids=ids_ref, wts=wts_ref)
                y, ids, _ = _noalloc_fp(moe, x)
            torch.cuda.synchronize()
            assert torch.equal(ids, ids_ref), (name, rnd)
            assert torch.equal(y, y_ref), (name, rnd)
