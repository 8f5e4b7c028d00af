"""Host-side API of the DeepSeek-V3-style FP8 MoE layer over the C ABI.

``Fp8MoE`` owns the packed fp8 expert banks (routed experts then the shared
one), the router and a workspace on one device, and exposes the reference's
operator surface:

* ``gate(x)``    -> (topk_idx, topk_weight) -- KimiMoEGate.forward
  (vendor/kimi_k3_ref/modeling_kimi_linear.py:703-759; ids int64 in the order
  torch.topk(sorted=False) returns them on CPU, weights fp32)
* ``route(x)``   -> (logits fp32, topk_idx, topk_weight)
* ``forward(x)`` -> y bf16 -- MoE.forward with fp8 experts and the shared expert
  (vendor/deepseek_v4_ref/inference/model.py:634-649)

All work is stream-ordered on torch's current CUDA stream, with no host
synchronisation and no allocation after construction.
"""
import ctypes

import torch

from . import _lib
from .moe import _ptr, _stream


class Fp8MoE:
    """A DeepSeek-V3-style layer: grouped sigmoid gate, fp8 (e4m3 + 128x128 fp32
    block scales) routed experts and one shared expert, SiLU-gated."""

    def __init__(self, router_w, bias, expert, num_experts, hidden, inter, top_k, n_group,
                 topk_group, route_scale, n_shared=1, swiglu_limit=0.0, max_tokens=64,
                 device=None, experts=None, expert_range=None):
        """router_w bf16 [E, H]; bias fp32 [E] (e_score_correction_bias);
        ``expert(e)`` -> (w13 e4m3 [2I, H] = [w1; w3], s13 fp32 [2I/128, H/128],
        w2 e4m3 [H, I], s2 fp32 [H/128, I/128]) for e in [0, E) and e = E for the
        shared expert -- the reference's Linear.weight / Linear.scale pairs
        (model.py:143-147) with fp32 scales.  ``experts`` limits which routed
        experts are packed (the rest of the bank is zero); default all.
        ``expert_range`` = (lo, hi): an expert-parallel shard holding experts
        [lo, hi) (and the shared expert, computed by the shard with lo == 0);
        such a shard serves ``route`` / ``experts_pairs`` / ``combine``."""
        _lib.load()
        device = torch.device(device or router_w.device)
        if device.type != "cuda":
            raise ValueError("Fp8MoE runs on a CUDA device")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        E, H, I = num_experts, hidden, inter
        lo, hi = expert_range if expert_range is not None else (0, E)
        self.device = device
        self.num_experts, self.hidden, self.inter, self.top_k = E, H, I, top_k
        self.n_shared = n_shared
        self.expert_range = (lo, hi)
        self.desc = _lib.Desc(
            abi_version=_lib.ABI_VERSION, format=_lib.FMT_FP8_BLOCK,
            gating=_lib.GATE_SIGMOID_GROUP, activation=_lib.ACT_SILU, num_experts=E, top_k=top_k,
            hidden=H, inter=I, expert_begin=lo, expert_end=hi, max_tokens=max_tokens,
            swiglu_limit=swiglu_limit, swiglu_alpha=0.0, n_group=n_group, topk_group=topk_group,
            route_scale=route_scale, n_shared=n_shared)
        _lib.call("flyai_moe_check_desc", ctypes.byref(self.desc))
        self.router_w = router_w.to(device=device, dtype=torch.bfloat16).contiguous()
        self.bias = bias.to(device=device, dtype=torch.float32).contiguous()
        todo = [e for e in (range(E) if experts is None else sorted(set(int(e) for e in experts)))
                if lo <= e < hi]
        if n_shared:
            todo.append(E)
        self.w13 = self._bank(_lib.PROJ_W13, full=experts is None)
        self.w2 = self._bank(_lib.PROJ_W2, full=experts is None)
        for e in todo:
            w13, s13, w2, s2 = expert(e)
            self._pack_one(e, _lib.PROJ_W13, self.w13, w13, s13)
            self._pack_one(e, _lib.PROJ_W2, self.w2, w2, s2)
        self.weights = _lib.Weights(router_w=self.router_w.data_ptr(), router_b=self.bias.data_ptr(),
                                    w13=self.w13.data_ptr(), w13_bias=None,
                                    w2=self.w2.data_ptr(), w2_bias=None)
        nbytes = ctypes.c_size_t()
        _lib.call("flyai_moe_workspace_bytes", ctypes.byref(self.desc), ctypes.byref(nbytes))
        self.workspace = torch.zeros(nbytes.value, dtype=torch.uint8, device=device)
        self.max_tokens = max_tokens

    @classmethod
    def from_layer(cls, layer, max_tokens=64, device=None, experts=None, expert_range=None):
        """Build from a ``flyai_b200.synth.Dsv3Layer`` (experts generated on the
        layer's device, one at a time)."""
        return cls(layer.router_w, layer.bias, layer.expert, layer.num_experts, layer.hidden,
                   layer.inter, layer.top_k, layer.n_group, layer.topk_group, layer.route_scale,
                   n_shared=layer.n_shared, max_tokens=max_tokens, device=device, experts=experts,
                   expert_range=expert_range)

    def _bank(self, proj, full):
        nbytes = ctypes.c_size_t()
        _lib.call("flyai_moe_packed_bytes", ctypes.byref(self.desc), proj, ctypes.byref(nbytes))
        alloc = torch.empty if full else torch.zeros
        return alloc(nbytes.value, dtype=torch.uint8, device=self.device)

    def _one_desc(self, e):
        d = _lib.Desc.from_buffer_copy(self.desc)
        if e < self.num_experts:
            d.expert_begin, d.expert_end, d.n_shared = e, e + 1, 0
        else:
            d.expert_begin, d.expert_end, d.n_shared = 0, 0, 1
        return d

    def _slot(self, e):
        """Bank slot of expert e: this shard's experts first, then the shared one."""
        lo, hi = self.expert_range
        return e - lo if e < self.num_experts else hi - lo

    def _pack_one(self, e, proj, bank, w, s):
        d = self._one_desc(e)
        per = ctypes.c_size_t()
        _lib.call("flyai_moe_packed_bytes", ctypes.byref(d), proj, ctypes.byref(per))
        w = w.to(self.device).contiguous().view(torch.uint8)
        s = s.to(device=self.device, dtype=torch.float32).contiguous()
        dst = ctypes.c_void_p(bank.data_ptr() + self._slot(e) * per.value)
        with torch.cuda.device(self.device):
            _lib.call("flyai_moe_pack_fp8", ctypes.byref(d), proj, _ptr(w), _ptr(s), dst, _stream())

    def _check_x(self, x):
        if x.dtype != torch.bfloat16 or not x.is_contiguous() or x.device != self.device:
            raise ValueError("x must be contiguous bf16 on the layer's device")
        if x.dim() != 2 or x.shape[1] != self.hidden:
            raise ValueError(f"x must be [M, {self.hidden}]")
        if x.shape[0] > self.max_tokens:
            raise ValueError(f"at most {self.max_tokens} tokens per call")

    def pair_rows(self, num_tokens):
        """Rows of the expert-parallel pair-row buffer: M*k pairs, then the shared expert's."""
        return num_tokens * (self.top_k + self.n_shared)

    def route(self, x, logits=True):
        self._check_x(x)
        M = x.shape[0]
        logits = (torch.empty(M, self.num_experts, dtype=torch.float32, device=self.device)
                  if logits else None)
        ids = torch.empty(M, self.top_k, dtype=torch.int32, device=self.device)
        wts = torch.empty(M, self.top_k, dtype=torch.float32, device=self.device)
        with torch.cuda.device(self.device):
            _lib.call("flyai_moe_route", ctypes.byref(self.desc), M, _ptr(x),
                      ctypes.byref(self.weights), _ptr(logits), _ptr(ids), _ptr(wts),
                      _ptr(self.workspace), self.workspace.numel(), _stream())
        return logits, ids.long(), wts

    def read_plan(self, num_tokens):
        """(counts [El], offsets [El+1], perm [M*k]) int32 left by the last ``route()``:
        this shard's pairs by ascending expert, ascending flat pair index inside one."""
        El = self.expert_range[1] - self.expert_range[0]
        counts = torch.empty(El, dtype=torch.int32, device=self.device)
        offsets = torch.empty(El + 1, dtype=torch.int32, device=self.device)
        perm = torch.empty(max(num_tokens * self.top_k, 1), dtype=torch.int32, device=self.device)
        with torch.cuda.device(self.device):
            _lib.call("flyai_moe_read_plan", ctypes.byref(self.desc), num_tokens, _ptr(self.workspace),
                      self.workspace.numel(), _ptr(counts), _ptr(offsets), _ptr(perm), _stream())
        return counts, offsets, perm

    def experts_pairs(self, x, pair_out=None):
        """This shard's expert rows (flyai_moe_experts_pairs) on the routing of the last
        ``route(x)``: bf16 [pair_rows(M), H], rows of other shards' experts zero."""
        self._check_x(x)
        M = x.shape[0]
        if pair_out is None:
            pair_out = torch.empty(self.pair_rows(M), self.hidden, dtype=torch.bfloat16,
                                   device=self.device)
        with torch.cuda.device(self.device):
            _lib.call("flyai_moe_experts_pairs", ctypes.byref(self.desc), M, _ptr(x),
                      ctypes.byref(self.weights), _ptr(pair_out), _ptr(self.workspace),
                      self.workspace.numel(), _stream())
        return pair_out

    def combine(self, pair_out, num_tokens, out=None):
        """Fold every shard's rows (summed over ranks) into y bf16 [M, H]."""
        y = out if out is not None else torch.empty(num_tokens, self.hidden, dtype=torch.bfloat16,
                                                    device=self.device)
        with torch.cuda.device(self.device):
            _lib.call("flyai_moe_combine", ctypes.byref(self.desc), num_tokens, _ptr(pair_out),
                      _ptr(y), _ptr(self.workspace), self.workspace.numel(), _stream())
        return y

    def gate(self, x):
        _, ids, wts = self.route(x)
        return ids, wts

    def forward(self, x, out=None, ids=None, wts=None):
        """y = MoE.forward(x); ``ids``/``wts`` (int32 / fp32 [M, k]) receive the routing."""
        self._check_x(x)
        M = x.shape[0]
        y = out if out is not None else torch.empty_like(x)
        with torch.cuda.device(self.device):
            _lib.call("flyai_moe_forward", ctypes.byref(self.desc), M, _ptr(x),
                      ctypes.byref(self.weights), _ptr(y), _ptr(ids), _ptr(wts),
                      _ptr(self.workspace), self.workspace.numel(), _stream())
        if _lib.checking():
            self.raise_on_error(type(self).__name__ + ".forward")
        return y

    __call__ = forward

    def raise_on_error(self, where=None):
        """Raise FlyaiDeviceError if a kernel left the error word set (reads and
        clears it; synchronises the host with the stream)."""
        _lib.raise_on_error_bits(self.read_error(clear=True)[0], where or type(self).__name__)

    def read_error(self, clear=True):
        out = torch.zeros(9, dtype=torch.int32, device=self.device)
        with torch.cuda.device(self.device):
            _lib.call("flyai_moe_read_error", ctypes.byref(self.desc), _ptr(self.workspace),
                      self.workspace.numel(), _ptr(out), 1 if clear else 0, _stream())
        return out.cpu().tolist()
