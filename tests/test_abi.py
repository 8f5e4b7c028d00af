"""The C-ABI library loads on a CPU-only machine, exports every symbol the header
declares, and validates descriptors without touching a GPU."""
import ctypes
import os
import re

import pytest

from flyai_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            names |= set(re.findall(r"FLYAI_API\s+[\w\s\*]+?\b(flyai_\w+)\s*\(", text))
    return names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    declared = header_symbols()
    assert declared, "no declarations parsed from include/*.h"
    assert declared == set(_lib.EXPORTS), (declared ^ set(_lib.EXPORTS))
    for name in declared:
        assert hasattr(lib, name), name


def good_desc(**kw):
    d = dict(abi_version=_lib.ABI_VERSION, format=_lib.FMT_MXFP4, gating=_lib.GATE_SOFTMAX_TOPK,
             activation=_lib.ACT_GPTOSS_SWIGLU, num_experts=128, top_k=4, hidden=2880,
             inter=2880, expert_begin=0, expert_end=128, max_tokens=64, swiglu_limit=7.0,
             swiglu_alpha=1.702)
    d.update(kw)
    return _lib.Desc(**d)


def test_desc_validation():
    lib = _lib.load()
    assert lib.flyai_moe_check_desc(ctypes.byref(good_desc())) == _lib.OK
    assert lib.flyai_moe_check_desc(None) == _lib.ERR_INVALID_ARG
    assert lib.flyai_moe_check_desc(ctypes.byref(good_desc(abi_version=99))) == _lib.ERR_ABI
    assert lib.flyai_moe_check_desc(ctypes.byref(good_desc(format=7))) == _lib.ERR_UNSUPPORTED
    assert lib.flyai_moe_check_desc(ctypes.byref(good_desc(top_k=9))) == _lib.ERR_INVALID_ARG
    assert lib.flyai_moe_check_desc(ctypes.byref(good_desc(hidden=2880 + 16))) == _lib.ERR_ALIGNMENT
    # one expert path (tcgen05): K-tiles of 64, at most 3072 per projection
    assert lib.flyai_moe_check_desc(ctypes.byref(good_desc(hidden=96))) == _lib.ERR_ALIGNMENT
    assert lib.flyai_moe_check_desc(ctypes.byref(good_desc(inter=2880 + 32))) == _lib.ERR_ALIGNMENT
    assert lib.flyai_moe_check_desc(ctypes.byref(good_desc(hidden=3136))) == _lib.ERR_UNSUPPORTED
    assert lib.flyai_moe_check_desc(ctypes.byref(good_desc(expert_end=129))) == _lib.ERR_INVALID_ARG
    d = good_desc()
    d.reserved[3] = 1
    assert lib.flyai_moe_check_desc(ctypes.byref(d)) == _lib.ERR_INVALID_ARG


def test_sizes_and_errors_without_gpu():
    lib = _lib.load()
    n = ctypes.c_size_t()
    assert lib.flyai_moe_packed_bytes(ctypes.byref(good_desc()), _lib.PROJ_W13, ctypes.byref(n)) == 0
    # the reference's storage plus the tile layout's padded scale chunks (< 0.5 %)
    ref = 128 * 2 * 2880 * (2880 // 2 + 2880 // 32)
    assert ref <= n.value <= ref * 1.005
    assert lib.flyai_moe_packed_bytes(ctypes.byref(good_desc(expert_begin=32, expert_end=64)),
                                      _lib.PROJ_W2, ctypes.byref(n)) == 0
    ref = 32 * 2880 * (2880 // 2 + 2880 // 32)
    assert ref <= n.value <= ref * 1.005
    assert lib.flyai_moe_workspace_bytes(ctypes.byref(good_desc()), ctypes.byref(n)) == 0
    assert n.value > 64 * 4 * 2880 * 4
    # calls that would launch refuse bad inputs before touching the device
    w = _lib.Weights()
    st = lib.flyai_moe_forward(ctypes.byref(good_desc()), 5, None, ctypes.byref(w), None, None, None,
                               None, 0, None)
    assert st == _lib.ERR_WORKSPACE
    st = lib.flyai_moe_forward(ctypes.byref(good_desc()), 65, None, ctypes.byref(w), None, None, None,
                               None, 0, None)
    assert st == _lib.ERR_INVALID_ARG
    assert lib.flyai_moe_strerror(_lib.ERR_WORKSPACE).decode().startswith("workspace")


def nvfp4_desc(**kw):
    d = dict(abi_version=_lib.ABI_VERSION, format=_lib.FMT_NVFP4, gating=_lib.GATE_SIGMOID_BF16,
             activation=_lib.ACT_SILU_BF16, num_experts=256, top_k=8, hidden=3072, inter=1536,
             expert_begin=0, expert_end=256, max_tokens=64, n_group=1, topk_group=1, route_scale=1.0)
    d.update(kw)
    return _lib.Desc(**d)


def test_nvfp4_prefill_workspace_limits():
    """NVFP4 descriptors accept up to 8192 tokens (calls above 64 take the prefill
    kernels, whose chunk buffers the workspace then holds); FP8 stays at 64."""
    lib = _lib.load()
    small, big = ctypes.c_size_t(), ctypes.c_size_t()
    assert lib.flyai_moe_workspace_bytes(ctypes.byref(nvfp4_desc()), ctypes.byref(small)) == _lib.OK
    assert lib.flyai_moe_workspace_bytes(ctypes.byref(nvfp4_desc(max_tokens=4096)), ctypes.byref(big)) == _lib.OK
    # at least the f16 token rows and bf16 SwiGLU rows of every pair, plus the pair rows
    P = 4096 * 8
    assert big.value > P * (3072 + 1536) * 2 + P * 3072 * 2 > small.value
    assert lib.flyai_moe_check_desc(ctypes.byref(nvfp4_desc(max_tokens=8192))) == _lib.OK
    assert lib.flyai_moe_check_desc(ctypes.byref(nvfp4_desc(max_tokens=8193))) == _lib.ERR_UNSUPPORTED
    fp8 = nvfp4_desc(format=_lib.FMT_FP8_BLOCK, gating=_lib.GATE_SIGMOID_GROUP,
                     activation=_lib.ACT_SILU, hidden=7168, inter=2048, n_group=8, topk_group=4,
                     route_scale=2.5, n_shared=1, max_tokens=65)
    assert lib.flyai_moe_check_desc(ctypes.byref(fp8)) == _lib.ERR_UNSUPPORTED


def test_v4_descriptor_validation():
    lib = _lib.load()
    ok = good_desc(format=_lib.FMT_FP4_W4A8, gating=_lib.GATE_SQRTSOFTPLUS, activation=_lib.ACT_SILU,
                   num_experts=256, top_k=6, hidden=4096, inter=2048, expert_end=256,
                   swiglu_limit=10.0, swiglu_alpha=0.0, n_group=1, topk_group=1, route_scale=1.5,
                   n_shared=1)
    assert lib.flyai_moe_check_desc(ctypes.byref(ok)) == _lib.OK
    for kw, st in ((dict(gating=_lib.GATE_SIGMOID_GROUP), _lib.ERR_UNSUPPORTED),
                   (dict(hidden=4096 + 64), _lib.ERR_ALIGNMENT),
                   (dict(max_tokens=65), _lib.ERR_UNSUPPORTED),
                   (dict(n_group=8), _lib.ERR_INVALID_ARG)):
        d = _lib.Desc.from_buffer_copy(ok)
        for k, v in kw.items():
            setattr(d, k, v)
        assert lib.flyai_moe_check_desc(ctypes.byref(d)) == st, kw
    # bank: routed fp4 experts (0.5 B + 1/32 B per weight) then the fp8 shared expert
    n = ctypes.c_size_t()
    assert lib.flyai_moe_packed_bytes(ctypes.byref(ok), _lib.PROJ_W13, ctypes.byref(n)) == _lib.OK
    routed = 256 * 2 * 2048 * 4096 * (0.5 + 1 / 32)
    shared = 2 * 2048 * 4096 * (1 + 1 / 32)
    assert n.value == int(routed + shared)


def test_python_layer_refuses_cpu_device():
    import torch
    with pytest.raises((ValueError, RuntimeError)):
        from flyai_b200.moe import Mxfp4MoE
        z = torch.zeros
        Mxfp4MoE(z(4, 64, dtype=torch.bfloat16), z(4, dtype=torch.bfloat16),
                 z(4, 128, 2, 16, dtype=torch.uint8), z(4, 128, 2, dtype=torch.uint8), z(4, 128),
                 z(4, 64, 2, 16, dtype=torch.uint8), z(4, 64, 2, dtype=torch.uint8), z(4, 64), 2,
                 device="cpu")


def test_caller_routed_and_situ_descriptors():
    """Kimi-K3 (FLYAI_GATE_EXTERNAL + FLYAI_ACT_SITU) and the token-sharded pair
    executor (FLYAI_GATE_EXTERNAL + GPT-OSS SwiGLU) validate on the host; the
    entry points that route themselves refuse caller-routed descriptors before any
    device work."""
    lib = _lib.load()
    k3 = good_desc(gating=_lib.GATE_EXTERNAL, activation=_lib.ACT_SITU, num_experts=896,
                   expert_end=896, top_k=16, hidden=2048, inter=1024, swiglu_alpha=4.0,
                   swiglu_limit=25.0)
    assert lib.flyai_moe_check_desc(ctypes.byref(k3)) == _lib.OK
    for kw, st in ((dict(top_k=17), _lib.ERR_INVALID_ARG),            # 16 slots at most
                   (dict(swiglu_alpha=0.0), _lib.ERR_INVALID_ARG),    # beta > 0
                   (dict(swiglu_limit=-1.0), _lib.ERR_INVALID_ARG),   # linear_beta >= 0 (0 = None)
                   (dict(swiglu_limit=0.0), _lib.OK),
                   (dict(max_tokens=65), _lib.ERR_UNSUPPORTED),       # verify kernels only
                   (dict(activation=_lib.ACT_SILU), _lib.ERR_UNSUPPORTED)):
        d = _lib.Desc.from_buffer_copy(k3)
        for k, v in kw.items():
            setattr(d, k, v)
        assert lib.flyai_moe_check_desc(ctypes.byref(d)) == st, kw
    # situ needs caller routing; 16 slots need caller routing
    assert lib.flyai_moe_check_desc(ctypes.byref(good_desc(activation=_lib.ACT_SITU))) == _lib.ERR_UNSUPPORTED
    assert lib.flyai_moe_check_desc(ctypes.byref(good_desc(top_k=16))) == _lib.ERR_INVALID_ARG
    pairs = good_desc(gating=_lib.GATE_EXTERNAL, top_k=1, max_tokens=4096, expert_end=64)
    assert lib.flyai_moe_check_desc(ctypes.byref(pairs)) == _lib.OK
    # routing entry points: each takes its own kind of descriptor only
    assert lib.flyai_moe_forward(ctypes.byref(k3), 1, None, None, None, None, None, None, 0,
                                 None) == _lib.ERR_UNSUPPORTED
    assert lib.flyai_moe_route(ctypes.byref(k3), 1, None, None, None, None, None, None, 0,
                               None) == _lib.ERR_UNSUPPORTED
    assert lib.flyai_moe_route_ids(ctypes.byref(good_desc()), 1, None, None, None, 0,
                                   None) == _lib.ERR_UNSUPPORTED
    assert lib.flyai_moe_route_ids(ctypes.byref(k3), 1, None, None, None, 0,
                                   None) == _lib.ERR_WORKSPACE
    # the slot-table experts entry is the V4 layer's
    assert lib.flyai_moe_experts_slots(ctypes.byref(k3), 1, None, None, None, 4, None, None, 0,
                                       None) == _lib.ERR_UNSUPPORTED


def test_fp8_linear_sizes_and_argument_checks():
    lib = _lib.load()
    n = ctypes.c_size_t()
    # bank: per 128x128 block a 16-byte scale header + the 16 KB tile
    assert lib.flyai_fp8_linear_bank_bytes(512, 4096, ctypes.byref(n)) == _lib.OK
    assert n.value == 4 * 32 * (16 + 128 * 128)
    assert lib.flyai_fp8_linear_bank_bytes(500, 4096, ctypes.byref(n)) == _lib.ERR_ALIGNMENT
    assert lib.flyai_fp8_linear_bank_bytes(0, 4096, ctypes.byref(n)) == _lib.ERR_INVALID_ARG
    w1 = ctypes.c_size_t()
    w64 = ctypes.c_size_t()
    assert lib.flyai_fp8_linear_workspace_bytes(1, 4096, 8192, ctypes.byref(w1)) == _lib.OK
    assert lib.flyai_fp8_linear_workspace_bytes(64, 4096, 8192, ctypes.byref(w64)) == _lib.OK
    assert 0 < w1.value < w64.value
    big = ctypes.c_size_t()
    assert lib.flyai_fp8_linear_workspace_bytes(1000, 4096, 8192, ctypes.byref(big)) == _lib.OK
    assert big.value == w64.value            # one launch holds 64 rows at most
    assert lib.flyai_fp8_linear_pack(512, 4096, None, None, 0, None, None) == _lib.ERR_INVALID_ARG
    assert lib.flyai_fp8_linear_pack(512, 4096, None, None, 7, None, None) == _lib.ERR_INVALID_ARG
    assert lib.flyai_fp8_linear(1, 512, 4096, None, None, 5, None, None, 0, None) == _lib.ERR_INVALID_ARG
    assert lib.flyai_fp8_linear(0, 512, 4096, None, None, 1, None, None, 0, None) == _lib.OK
    assert lib.flyai_fp8_linear(1, 512, 4096, ctypes.c_void_p(256), ctypes.c_void_p(256), 1,
                                ctypes.c_void_p(256), None, 0, None) == _lib.ERR_WORKSPACE
    assert lib.flyai_fp8_linear(1, 512, 4096, ctypes.c_void_p(256), ctypes.c_void_p(256), 1,
                                ctypes.c_void_p(256), ctypes.c_void_p(256), 16,
                                None) == _lib.ERR_WORKSPACE
