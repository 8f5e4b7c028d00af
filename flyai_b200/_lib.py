"""ctypes binding of ``libflyai_moe.so`` (the C ABI declared in include/flyai_moe.h).

There is no fallback: if the library is missing or fails to load, every call
raises.  Build it with ``python -m flyai_b200.build``.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libflyai_moe.so")

ABI_VERSION = 1
OK = 0
ERR_INVALID_ARG = -1
ERR_UNSUPPORTED = -2
ERR_ALIGNMENT = -3
ERR_WORKSPACE = -4
ERR_CUDA = -5
ERR_ABI = -6

FMT_MXFP4 = 1
FMT_FP8_BLOCK = 2
FMT_NVFP4 = 3
FMT_FP4_W4A8 = 4
GATE_SOFTMAX_TOPK = 1
GATE_SIGMOID_GROUP = 2
GATE_SIGMOID_BF16 = 3
GATE_SQRTSOFTPLUS = 4
GATE_EXTERNAL = 5
ACT_GPTOSS_SWIGLU = 1
ACT_SILU = 2
ACT_SILU_BF16 = 3
ACT_SITU = 4
PROJ_W13 = 0
PROJ_W2 = 1
LIN_SCALE_F32 = 0
LIN_SCALE_E8M0 = 1
LIN_FMT_AMAX = 0
LIN_FMT_UE8M0 = 1

EXPORTS = (
    "flyai_moe_abi_version", "flyai_moe_strerror", "flyai_moe_check_desc",
    "flyai_moe_packed_bytes", "flyai_moe_pack_mxfp4", "flyai_moe_workspace_bytes",
    "flyai_moe_route", "flyai_moe_experts", "flyai_moe_experts_pairs", "flyai_moe_combine",
    "flyai_moe_forward", "flyai_moe_launch_count", "flyai_moe_read_plan",
    "flyai_moe_set_profile_events", "flyai_moe_ep_mailbox_bytes", "flyai_moe_ep_alloc",
    "flyai_moe_ep_free", "flyai_moe_ipc_get_handle", "flyai_moe_ipc_open", "flyai_moe_ipc_close",
    "flyai_moe_experts_ep", "flyai_moe_combine_ep", "flyai_moe_forward_ep",
    "flyai_moe_forward_noalloc", "flyai_moe_read_error", "flyai_moe_pack_fp8",
    "flyai_moe_pack_nvfp4", "flyai_moe_pack_nvfp4_swizzled", "flyai_moe_pack_fp4", "flyai_moe_pack_shared_fp8",
    "flyai_moe_route_hash", "flyai_moe_route_logits", "flyai_moe_route_ids", "flyai_moe_experts_slots",
    "flyai_fp8_linear_bank_bytes", "flyai_fp8_linear_pack", "flyai_fp8_linear_workspace_bytes",
    "flyai_fp8_linear",
)


class Desc(ctypes.Structure):
    _fields_ = [
        ("abi_version", ctypes.c_int32), ("format", ctypes.c_int32),
        ("gating", ctypes.c_int32), ("activation", ctypes.c_int32),
        ("num_experts", ctypes.c_int32), ("top_k", ctypes.c_int32),
        ("hidden", ctypes.c_int32), ("inter", ctypes.c_int32),
        ("expert_begin", ctypes.c_int32), ("expert_end", ctypes.c_int32),
        ("max_tokens", ctypes.c_int32),
        ("swiglu_limit", ctypes.c_float), ("swiglu_alpha", ctypes.c_float),
        ("n_group", ctypes.c_int32), ("topk_group", ctypes.c_int32),
        ("route_scale", ctypes.c_float), ("n_shared", ctypes.c_int32),
        ("reserved", ctypes.c_int32 * 4),
    ]


class Weights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in
                ("router_w", "router_b", "w13", "w13_bias", "w2", "w2_bias")]


EP_MAX_RANKS = 8


class EpPeers(ctypes.Structure):
    """flyai_moe_ep_peers: ranks, this rank, call epoch, mailbox of every rank as mapped here."""
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("epoch", ctypes.c_uint32),
                ("reserved", ctypes.c_int32), ("mailbox", ctypes.c_void_p * EP_MAX_RANKS)]


class FlyaiError(RuntimeError):
    def __init__(self, fn, status, msg):
        super().__init__(f"{fn} failed: {msg} (status {status})")
        self.status = status


class FlyaiDeviceError(RuntimeError):
    """A kernel of a call gave up on a bounded wait and set the workspace's
    error word: that call's output is not valid (it is zero, or partial)."""


# FLYAI_MOE_CHECK=1: every layer call reads the workspace error word back and
# raises FlyaiDeviceError when it is set.  The read synchronises the host with
# the stream, so it is off by default and skipped while a CUDA graph is captured.
CHECK = os.environ.get("FLYAI_MOE_CHECK", "0") not in ("", "0")


def checking():
    """FLYAI_MOE_CHECK is on and the current stream is not capturing."""
    import torch
    if not CHECK:
        return False
    return not (torch.cuda.is_available() and torch.cuda.is_current_stream_capturing())


def raise_on_error_bits(bits, where):
    if bits:
        raise FlyaiDeviceError(f"{where}: a kernel gave up on a bounded wait (error bits {bits:#x}); "
                               "the output of this call is not valid")


_lib = None


def load():
    """Load the library once; raise (never fall back) if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m flyai_b200.build`")
    lib = ctypes.CDLL(LIB_PATH)
    vp, i32, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_size_t
    pd, pw = ctypes.POINTER(Desc), ctypes.POINTER(Weights)
    sigs = {
        "flyai_moe_abi_version": ([], ctypes.c_int),
        "flyai_moe_strerror": ([ctypes.c_int], ctypes.c_char_p),
        "flyai_moe_check_desc": ([pd], ctypes.c_int),
        "flyai_moe_packed_bytes": ([pd, i32, ctypes.POINTER(sz)], ctypes.c_int),
        "flyai_moe_pack_mxfp4": ([pd, i32, vp, vp, vp, vp], ctypes.c_int),
        "flyai_moe_pack_fp8": ([pd, i32, vp, vp, vp, vp], ctypes.c_int),
        "flyai_moe_pack_nvfp4": ([pd, i32, vp, vp, vp, vp, vp], ctypes.c_int),
        "flyai_moe_pack_nvfp4_swizzled": ([pd, i32, vp, vp, vp, vp, vp], ctypes.c_int),
        "flyai_moe_pack_fp4": ([pd, i32, vp, vp, vp, vp], ctypes.c_int),
        "flyai_moe_pack_shared_fp8": ([pd, i32, vp, vp, vp, vp], ctypes.c_int),
        "flyai_moe_route_hash": ([pd, i32, vp, vp, vp, i32, pw, vp, vp, vp, vp, sz, vp], ctypes.c_int),
        "flyai_moe_route_logits": ([pd, i32, vp, vp, pw, vp, vp, vp, sz, vp], ctypes.c_int),
        "flyai_moe_route_ids": ([pd, i32, vp, vp, vp, sz, vp], ctypes.c_int),
        "flyai_moe_experts_slots": ([pd, i32, vp, pw, vp, i32, vp, vp, sz, vp], ctypes.c_int),
        "flyai_moe_workspace_bytes": ([pd, ctypes.POINTER(sz)], ctypes.c_int),
        "flyai_moe_route": ([pd, i32, vp, pw, vp, vp, vp, vp, sz, vp], ctypes.c_int),
        "flyai_moe_experts": ([pd, i32, vp, pw, vp, vp, sz, vp], ctypes.c_int),
        "flyai_moe_experts_pairs": ([pd, i32, vp, pw, vp, vp, sz, vp], ctypes.c_int),
        "flyai_moe_combine": ([pd, i32, vp, vp, vp, sz, vp], ctypes.c_int),
        "flyai_moe_forward": ([pd, i32, vp, pw, vp, vp, vp, vp, sz, vp], ctypes.c_int),
        "flyai_moe_launch_count": ([], ctypes.c_int64),
        "flyai_moe_set_profile_events": ([vp, vp], ctypes.c_int),
        "flyai_moe_ep_mailbox_bytes": ([pd, ctypes.POINTER(sz)], ctypes.c_int),
        "flyai_moe_ep_alloc": ([sz, ctypes.POINTER(vp)], ctypes.c_int),
        "flyai_moe_ep_free": ([vp], ctypes.c_int),
        "flyai_moe_ipc_get_handle": ([vp, vp], ctypes.c_int),
        "flyai_moe_ipc_open": ([vp, ctypes.POINTER(vp)], ctypes.c_int),
        "flyai_moe_ipc_close": ([vp], ctypes.c_int),
        "flyai_moe_experts_ep": ([pd, i32, vp, pw, ctypes.POINTER(EpPeers), vp, sz, vp], ctypes.c_int),
        "flyai_moe_forward_ep": ([pd, i32, vp, pw, ctypes.POINTER(EpPeers), vp, vp, vp, sz, vp], ctypes.c_int),
        "flyai_moe_combine_ep": ([pd, i32, ctypes.POINTER(EpPeers), vp, vp, sz, vp], ctypes.c_int),
        "flyai_moe_read_plan": ([pd, i32, vp, sz, vp, vp, vp, vp], ctypes.c_int),
        "flyai_moe_forward_noalloc": ([pd, i32, vp, pw, vp, vp, vp, vp], ctypes.c_int),
        "flyai_moe_read_error": ([pd, vp, sz, vp, i32, vp], ctypes.c_int),
        "flyai_fp8_linear_bank_bytes": ([i32, i32, ctypes.POINTER(sz)], ctypes.c_int),
        "flyai_fp8_linear_pack": ([i32, i32, vp, vp, i32, vp, vp], ctypes.c_int),
        "flyai_fp8_linear_workspace_bytes": ([i32, i32, i32, ctypes.POINTER(sz)], ctypes.c_int),
        "flyai_fp8_linear": ([i32, i32, i32, vp, vp, i32, vp, vp, sz, vp], ctypes.c_int),
    }
    for name, (args, res) in sigs.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    if lib.flyai_moe_abi_version() != ABI_VERSION:
        raise RuntimeError("libflyai_moe.so ABI version mismatch; rebuild it")
    _lib = lib
    return lib


def check(fn_name, status):
    if status != OK:
        msg = load().flyai_moe_strerror(status).decode()
        raise FlyaiError(fn_name, status, msg)
    return status


def call(fn_name, *args):
    return check(fn_name, getattr(load(), fn_name)(*args))
