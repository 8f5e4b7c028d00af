"""Kimi-K3 routed experts (MXFP4 weights, the `situ` activation) behind the
reference's ``moe_infer`` seam.

The K3 stage keeps its own router (``KimiMoEGate``), latent projections, norm and
shared experts, and hands only the routed experts to a backend through
``KimiSparseMoeBlock.moe_infer(x, topk_ids, topk_weight)``
(vendor/kimi_k3_ref/modeling_kimi_linear.py:841-875); the reference's backend is
vLLM's Marlin MXFP4 kernels with `situ` injected (engines/kimi_k3/
k3_moe_mxfp4.py:258-412).  ``K3MoE`` is that backend on the sm_100a tcgen05
kernels: ``flyai_moe_route_ids`` takes the caller's ids and weights, then
``flyai_moe_experts`` runs gate/up with `situ`, down, and the reference's fold
(bf16 rows times fp32 weights, summed in slot order, to bf16).

``install(block, moe)`` binds one block's ``moe_infer`` to it, keeping the
block's own ``moe_infer`` as the fallback for what it declines (tensors not on
the layer's device, non-bf16 input); ``coverage(module)`` counts claimed and
declined calls per block.  Enabled by ``FLYAI_MOE_K3`` (default on; "0" makes
``install`` a no-op), read at import.
"""
import ctypes
import os
import threading

import torch

from . import _lib
from .moe import _ptr, _stream

ENABLED = os.environ.get("FLYAI_MOE_K3", "1") not in ("", "0")
MAX_TOKENS = 64   # rows per kernel call (larger batches run in slices)

_LOCK = threading.Lock()
_INSTALLED = []
_ATTEMPTS = [0]


class K3MoE:
    """The routed experts of one Kimi-K3 MoE layer: ``num_experts`` MXFP4 experts
    (w1, w3: [inter, hidden], w2: [hidden, inter]; e2m1 + e8m0 per 32), `situ`
    with ``beta`` and ``linear_beta`` (None: up passes through)."""

    def __init__(self, expert, num_experts, hidden, inter, top_k, beta=1.0, linear_beta=None,
                 max_tokens=MAX_TOKENS, device=None, experts=None):
        """``expert(e)`` -> (w1 uint8 [I, H/2], s1 uint8 [I, H/32], w3, s3, w2 uint8
        [H, I/2], s2 uint8 [H, I/32]) -- each Linear's ``weight_packed`` and
        ``weight_scale``.  ``experts`` limits which experts are packed (the rest of
        the bank stays zero)."""
        _lib.load()
        device = torch.device(device or "cuda")
        if device.type != "cuda":
            raise ValueError("K3MoE runs on a CUDA device")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        if not 1 <= max_tokens <= MAX_TOKENS:
            raise ValueError(f"max_tokens must be in [1, {MAX_TOKENS}]")
        self.device = device
        self.num_experts, self.hidden, self.inter, self.top_k = num_experts, hidden, inter, top_k
        self.beta, self.linear_beta = float(beta), linear_beta
        self.max_tokens = max_tokens
        self.desc = _lib.Desc(
            abi_version=_lib.ABI_VERSION, format=_lib.FMT_MXFP4, gating=_lib.GATE_EXTERNAL,
            activation=_lib.ACT_SITU, num_experts=num_experts, top_k=top_k, hidden=hidden,
            inter=inter, expert_begin=0, expert_end=num_experts, max_tokens=max_tokens,
            swiglu_limit=float(linear_beta or 0.0), swiglu_alpha=float(beta))
        _lib.call("flyai_moe_check_desc", ctypes.byref(self.desc))
        self.w13 = self._bank(_lib.PROJ_W13, full=experts is None)
        self.w2 = self._bank(_lib.PROJ_W2, full=experts is None)
        todo = range(num_experts) if experts is None else sorted(set(int(e) for e in experts))
        for e in todo:
            w1, s1, w3, s3, w2, s2 = expert(e)
            self._pack(e, _lib.PROJ_W13, self.w13, torch.cat([_u8(w1), _u8(w3)]),
                       torch.cat([_u8(s1), _u8(s3)]))
            self._pack(e, _lib.PROJ_W2, self.w2, _u8(w2), _u8(s2))
        self.weights = _lib.Weights(router_w=None, router_b=None, w13=self.w13.data_ptr(),
                                    w13_bias=None, w2=self.w2.data_ptr(), w2_bias=None)
        nbytes = ctypes.c_size_t()
        _lib.call("flyai_moe_workspace_bytes", ctypes.byref(self.desc), ctypes.byref(nbytes))
        self.workspace = torch.zeros(nbytes.value, dtype=torch.uint8, device=device)

    @classmethod
    def from_layer(cls, layer, max_tokens=MAX_TOKENS, device=None, experts=None):
        """Build from a ``flyai_b200.synth.K3Layer``."""
        return cls(layer.expert, layer.num_experts, layer.hidden, layer.inter, layer.top_k,
                   beta=layer.beta, linear_beta=layer.linear_beta, max_tokens=max_tokens,
                   device=device, experts=experts)

    @classmethod
    def from_checkpoint(cls, get_tensor, prefix, cfg, device=None):
        """Build from a K3 checkpoint: ``get_tensor(name)`` returns the tensors of
        ``{prefix}.experts.{e}.{w1,w3,w2}.{weight_packed,weight_scale}``, the names
        the reference's loader reads (engines/kimi_k3/k3_moe_mxfp4.py:326-340);
        ``cfg`` is the model config (``num_experts``, ``num_experts_per_token``,
        ``moe_intermediate_size``, ``routed_expert_hidden_size`` or ``hidden_size``,
        ``activation_situ_beta``, ``activation_situ_linear_beta``)."""
        def expert(e):
            b = f"{prefix}.experts.{e}"
            return tuple(get_tensor(f"{b}.{w}.{t}") for w in ("w1", "w3", "w2")
                         for t in ("weight_packed", "weight_scale"))
        hidden = getattr(cfg, "routed_expert_hidden_size", None) or cfg.hidden_size
        return cls(expert, cfg.num_experts, hidden, cfg.moe_intermediate_size,
                   cfg.num_experts_per_token, beta=getattr(cfg, "activation_situ_beta", None) or 1.0,
                   linear_beta=getattr(cfg, "activation_situ_linear_beta", None), device=device)

    def _bank(self, proj, full):
        nbytes = ctypes.c_size_t()
        _lib.call("flyai_moe_packed_bytes", ctypes.byref(self.desc), proj, ctypes.byref(nbytes))
        alloc = torch.empty if full else torch.zeros
        return alloc(nbytes.value, dtype=torch.uint8, device=self.device)

    def _pack(self, e, proj, bank, blocks, scales):
        d = _lib.Desc.from_buffer_copy(self.desc)
        d.expert_begin, d.expert_end = e, e + 1
        per = ctypes.c_size_t()
        _lib.call("flyai_moe_packed_bytes", ctypes.byref(d), proj, ctypes.byref(per))
        b = blocks.to(self.device).contiguous()
        s = scales.to(self.device).contiguous()
        with torch.cuda.device(self.device):
            _lib.call("flyai_moe_pack_mxfp4", ctypes.byref(d), proj, _ptr(b), _ptr(s),
                      ctypes.c_void_p(bank.data_ptr() + e * per.value), _stream())
            torch.cuda.current_stream().synchronize()   # load time only: b and s are temporaries

    def moe_infer(self, x, topk_ids, topk_weight, out=None):
        """y = moe_infer(x, topk_ids, topk_weight): x bf16 [T, hidden], topk_ids
        [T, k] (any integer dtype), topk_weight [T, k] (any float dtype; taken as
        fp32) -> bf16 [T, hidden].  Batches above max_tokens run in slices."""
        if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != self.hidden:
            raise ValueError(f"x must be bf16 [T, {self.hidden}]")
        if x.device != self.device:
            raise ValueError("x must be on the layer's device")
        T = x.shape[0]
        if tuple(topk_ids.shape) != (T, self.top_k) or tuple(topk_weight.shape) != (T, self.top_k):
            raise ValueError(f"topk_ids / topk_weight must be [{T}, {self.top_k}]")
        x = x.contiguous()
        ids = topk_ids.to(device=self.device, dtype=torch.int32).contiguous()
        wts = topk_weight.to(device=self.device, dtype=torch.float32).contiguous()
        y = out if out is not None else torch.empty(T, self.hidden, dtype=torch.bfloat16,
                                                    device=self.device)
        ws = self.workspace
        with torch.cuda.device(self.device):
            for t0 in range(0, T, self.max_tokens):
                m = min(self.max_tokens, T - t0)
                _lib.call("flyai_moe_route_ids", ctypes.byref(self.desc), m, _ptr(ids[t0:t0 + m]),
                          _ptr(wts[t0:t0 + m]), _ptr(ws), ws.numel(), _stream())
                _lib.call("flyai_moe_experts", ctypes.byref(self.desc), m, _ptr(x[t0:t0 + m]),
                          ctypes.byref(self.weights), _ptr(y[t0:t0 + m]), _ptr(ws), ws.numel(),
                          _stream())
        if _lib.checking():
            self.raise_on_error()
        return y

    __call__ = moe_infer

    def read_error(self, clear=True):
        out = torch.zeros(9, dtype=torch.int32, device=self.device)
        with torch.cuda.device(self.device):
            _lib.call("flyai_moe_read_error", ctypes.byref(self.desc), _ptr(self.workspace),
                      self.workspace.numel(), _ptr(out), 1 if clear else 0, _stream())
        return out.cpu().tolist()

    def raise_on_error(self, where="K3MoE"):
        """Raise FlyaiDeviceError if a kernel left the error word set (bit 1: a
        bounded wait gave up; bit 2: an expert id outside [0, E))."""
        bits = self.read_error(clear=True)[0]
        if bits & 2:
            raise _lib.FlyaiDeviceError(f"{where}: an expert id outside [0, {self.num_experts}) "
                                        "was read as expert 0; the output of this call is not valid")
        _lib.raise_on_error_bits(bits, where)


def _u8(t):
    return t.detach().contiguous().view(torch.uint8)


def _decline(block, why, prev, x, topk_ids, topk_weight):
    with _LOCK:
        tally = block.__dict__.setdefault("_flyai_declined", {})
        tally[why] = tally.get(why, 0) + 1
    return prev(x, topk_ids, topk_weight)


def install(block, moe):
    """Bind ``block.moe_infer`` (a ``KimiSparseMoeBlock`` or anything with that
    method) to ``moe`` (a ``K3MoE`` holding the block's routed experts), keeping
    the block's own ``moe_infer`` as the fallback.  Returns True if it took;
    idempotent; a no-op with FLYAI_MOE_K3=0 or without CUDA."""
    _ATTEMPTS[0] += 1
    if not ENABLED or not torch.cuda.is_available():
        return False
    if getattr(block.__dict__.get("moe_infer"), "_flyai_b200", False):
        return False
    prev = block.moe_infer

    def moe_infer(x, topk_ids, topk_weight):
        if not x.is_cuda or x.device != moe.device:
            return _decline(block, "not on the layer's device", prev, x, topk_ids, topk_weight)
        if x.dtype != torch.bfloat16:
            return _decline(block, f"dtype {x.dtype}", prev, x, topk_ids, topk_weight)
        y = moe.moe_infer(x.view(-1, moe.hidden), topk_ids.view(-1, moe.top_k),
                          topk_weight.view(-1, moe.top_k))
        with _LOCK:
            block.__dict__["_flyai_steps"] = block.__dict__.get("_flyai_steps", 0) + 1
        return y

    moe_infer._flyai_b200 = True
    moe_infer._flyai_prev = prev
    block.moe_infer = moe_infer
    with _LOCK:
        _INSTALLED.append(block)
    return True


def uninstall(block):
    """Drop the ``moe_infer`` that ``install`` bound."""
    if getattr(block.__dict__.get("moe_infer"), "_flyai_b200", False):
        del block.moe_infer
    with _LOCK:
        if block in _INSTALLED:
            _INSTALLED.remove(block)


def attempts():
    return _ATTEMPTS[0]


def installed():
    with _LOCK:
        return [b for b in _INSTALLED if getattr(b.__dict__.get("moe_infer"), "_flyai_b200", False)]


def coverage(module):
    """{block index: (claimed calls, {reason: declines})} for every block under
    ``module`` whose moe_infer this lever bound."""
    out = {}
    mods = module.modules() if hasattr(module, "modules") else [module]
    for m in mods:
        if getattr(m.__dict__.get("moe_infer"), "_flyai_b200", False) if hasattr(m, "__dict__") else False:
            out[len(out)] = (m.__dict__.get("_flyai_steps", 0), dict(m.__dict__.get("_flyai_declined", {})))
    return out
