"""Host-side API of the DeepSeek-V4 W4A8 MoE layer over the C ABI.

``W4A8MoE`` owns the packed expert bank (fp4 routed experts, then the fp8 shared
expert), the router and a workspace on one device, and exposes the reference's
operator surface (vendor/deepseek_v4_ref/inference/model.py):

* ``gate(x, input_ids)``    -> (weights fp32, indices int64) -- Gate.forward
  (:569-589): sqrt(softplus) scores, torch.topk (sorted) or, on a hash-routed
  layer, tid2eid[input_ids]
* ``forward(x, input_ids)`` -> y bf16 -- MoE.forward (:634-649): fp4 routed experts
  (W4A8, swiglu_limit clamp), the shared expert, fp32 fold in ascending id with
  a repeated expert counted once (its last slot)

All work is stream-ordered on torch's current CUDA stream, with no host
synchronisation and no allocation after construction.
"""
import ctypes

import torch

from . import _lib
from .moe import _ptr, _stream


class W4A8MoE:
    """A DeepSeek-V4 MoE layer: sqrt(softplus) gate (score- or hash-routed), fp4
    routed experts (e2m1 + e8m0 per 32), one fp8 shared expert (e4m3 + e8m0 per
    128x128), SiLU-gated with the swiglu_limit clamp."""

    def __init__(self, router_w, bias, expert, shared, num_experts, hidden, inter, top_k,
                 route_scale, swiglu_limit, tid2eid=None, max_tokens=64, device=None,
                 experts=None, expert_range=None):
        """router_w bf16 [E, H]; bias fp32 [E]; ``expert(e)`` -> (w13 uint8 [2I, H/2]
        packed e2m1 of [w1; w3], s13 uint8 [2I, H/32] e8m0, w2 uint8 [H, I/2], s2
        uint8 [H, I/32]) -- the fp4 Linear weight / scale pairs (model.py:133-139);
        ``shared()`` -> (w13 e4m3 [2I, H], s13 uint8 [2I/128, H/128] e8m0, w2 e4m3
        [H, I], s2 uint8 [H/128, I/128]) or None; ``tid2eid`` int32 [vocab, k] makes
        the layer hash-routed.  ``experts`` limits which routed experts are packed
        (the rest of the bank stays zero); ``expert_range`` = (lo, hi): an
        expert-parallel shard (the shared expert lives on the shard with lo == 0)."""
        _lib.load()
        device = torch.device(device or router_w.device)
        if device.type != "cuda":
            raise ValueError("W4A8MoE runs on a CUDA device")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        E, H, I = num_experts, hidden, inter
        lo, hi = expert_range if expert_range is not None else (0, E)
        n_shared = 1 if (shared is not None and lo == 0) else 0
        self.device = device
        self.num_experts, self.hidden, self.inter, self.top_k = E, H, I, top_k
        self.n_shared = n_shared
        self.expert_range = (lo, hi)
        self.desc = _lib.Desc(
            abi_version=_lib.ABI_VERSION, format=_lib.FMT_FP4_W4A8, gating=_lib.GATE_SQRTSOFTPLUS,
            activation=_lib.ACT_SILU, num_experts=E, top_k=top_k, hidden=H, inter=I,
            expert_begin=lo, expert_end=hi, max_tokens=max_tokens, swiglu_limit=swiglu_limit,
            swiglu_alpha=0.0, n_group=1, topk_group=1, route_scale=route_scale, n_shared=n_shared)
        _lib.call("flyai_moe_check_desc", ctypes.byref(self.desc))
        self.router_w = router_w.to(device=device, dtype=torch.bfloat16).contiguous()
        self.bias = bias.to(device=device, dtype=torch.float32).contiguous()
        self.tid2eid = (tid2eid.to(device=device, dtype=torch.int32).contiguous()
                        if tid2eid is not None else None)
        self.w13 = self._bank(_lib.PROJ_W13, full=experts is None)
        self.w2 = self._bank(_lib.PROJ_W2, full=experts is None)
        todo = [e for e in (range(E) if experts is None else sorted(set(int(e) for e in experts)))
                if lo <= e < hi]
        for e in todo:
            w13, s13, w2, s2 = expert(e)
            self._pack_routed(e, _lib.PROJ_W13, self.w13, w13, s13)
            self._pack_routed(e, _lib.PROJ_W2, self.w2, w2, s2)
        if n_shared:
            w13, s13, w2, s2 = shared()
            self._pack_shared(_lib.PROJ_W13, self.w13, w13, s13)
            self._pack_shared(_lib.PROJ_W2, self.w2, w2, s2)
        self.weights = _lib.Weights(router_w=self.router_w.data_ptr(), router_b=self.bias.data_ptr(),
                                    w13=self.w13.data_ptr(), w13_bias=None,
                                    w2=self.w2.data_ptr(), w2_bias=None)
        nbytes = ctypes.c_size_t()
        _lib.call("flyai_moe_workspace_bytes", ctypes.byref(self.desc), ctypes.byref(nbytes))
        self.workspace = torch.zeros(nbytes.value, dtype=torch.uint8, device=device)
        self.max_tokens = max_tokens

    @classmethod
    def from_layer(cls, layer, max_tokens=64, device=None, experts=None, expert_range=None,
                   shared=True):
        """Build from a ``flyai_b200.synth.V4Layer`` (experts generated on the layer's
        device, one at a time)."""
        return cls(layer.router_w, layer.bias, layer.expert, layer.shared if shared else None,
                   layer.num_experts, layer.hidden, layer.inter, layer.top_k, layer.route_scale,
                   layer.swiglu_limit, tid2eid=layer.tid2eid, max_tokens=max_tokens, device=device,
                   experts=experts, expert_range=expert_range)

    def _bank(self, proj, full):
        nbytes = ctypes.c_size_t()
        _lib.call("flyai_moe_packed_bytes", ctypes.byref(self.desc), proj, ctypes.byref(nbytes))
        alloc = torch.empty if full else torch.zeros
        return alloc(nbytes.value, dtype=torch.uint8, device=self.device)

    def _pack_routed(self, e, proj, bank, w, s):
        d = _lib.Desc.from_buffer_copy(self.desc)
        d.expert_begin, d.expert_end, d.n_shared = e, e + 1, 0
        per = ctypes.c_size_t()
        _lib.call("flyai_moe_packed_bytes", ctypes.byref(d), proj, ctypes.byref(per))
        w = w.to(self.device).contiguous().view(torch.uint8)
        s = s.to(self.device).contiguous().view(torch.uint8)
        dst = ctypes.c_void_p(bank.data_ptr() + (e - self.expert_range[0]) * per.value)
        with torch.cuda.device(self.device):
            _lib.call("flyai_moe_pack_fp4", ctypes.byref(d), proj, _ptr(w), _ptr(s), dst, _stream())

    def _pack_shared(self, proj, bank, w, s):
        w = w.to(self.device).contiguous().view(torch.uint8)
        s = s.to(self.device).contiguous().view(torch.uint8)
        with torch.cuda.device(self.device):
            _lib.call("flyai_moe_pack_shared_fp8", ctypes.byref(self.desc), proj, _ptr(w), _ptr(s),
                      _ptr(bank), _stream())

    def _check_x(self, x, input_ids):
        if x.dtype != torch.bfloat16 or not x.is_contiguous() or x.device != self.device:
            raise ValueError("x must be contiguous bf16 on the layer's device")
        if x.dim() != 2 or x.shape[1] != self.hidden:
            raise ValueError(f"x must be [M, {self.hidden}]")
        if x.shape[0] > self.max_tokens:
            raise ValueError(f"at most {self.max_tokens} tokens per call")
        if self.tid2eid is not None:
            if input_ids is None or input_ids.numel() != x.shape[0]:
                raise ValueError("a hash-routed layer needs one input id per token")
            return input_ids.to(device=self.device, dtype=torch.int32).contiguous().view(-1)
        return None

    def pair_rows(self, num_tokens):
        return num_tokens * (self.top_k + self.n_shared)

    def route(self, x, input_ids=None, logits=True):
        ids32 = self._check_x(x, input_ids)
        M = x.shape[0]
        lg = torch.empty(M, self.num_experts, dtype=torch.float32, device=self.device) if logits else None
        ids = torch.empty(M, self.top_k, dtype=torch.int32, device=self.device)
        wts = torch.empty(M, self.top_k, dtype=torch.float32, device=self.device)
        with torch.cuda.device(self.device):
            if ids32 is None:
                _lib.call("flyai_moe_route", ctypes.byref(self.desc), M, _ptr(x),
                          ctypes.byref(self.weights), _ptr(lg), _ptr(ids), _ptr(wts),
                          _ptr(self.workspace), self.workspace.numel(), _stream())
            else:
                _lib.call("flyai_moe_route_hash", ctypes.byref(self.desc), M, _ptr(x), _ptr(ids32),
                          _ptr(self.tid2eid), self.tid2eid.shape[0], ctypes.byref(self.weights),
                          _ptr(lg), _ptr(ids), _ptr(wts), _ptr(self.workspace),
                          self.workspace.numel(), _stream())
        return lg, ids.long(), wts

    def gate(self, x, input_ids=None):
        _, ids, wts = self.route(x, input_ids, logits=False)
        return wts, ids

    def read_plan(self, num_tokens):
        El = self.expert_range[1] - self.expert_range[0]
        counts = torch.empty(El, dtype=torch.int32, device=self.device)
        offsets = torch.empty(El + 1, dtype=torch.int32, device=self.device)
        perm = torch.empty(max(num_tokens * self.top_k, 1), dtype=torch.int32, device=self.device)
        with torch.cuda.device(self.device):
            _lib.call("flyai_moe_read_plan", ctypes.byref(self.desc), num_tokens, _ptr(self.workspace),
                      self.workspace.numel(), _ptr(counts), _ptr(offsets), _ptr(perm), _stream())
        return counts, offsets, perm

    def experts(self, x, out=None):
        """y on the routing of the last ``route()`` (flyai_moe_experts)."""
        M = x.shape[0]
        y = out if out is not None else torch.empty_like(x)
        with torch.cuda.device(self.device):
            _lib.call("flyai_moe_experts", ctypes.byref(self.desc), M, _ptr(x),
                      ctypes.byref(self.weights), _ptr(y), _ptr(self.workspace),
                      self.workspace.numel(), _stream())
        return y

    def experts_pairs(self, x, pair_out=None):
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
        y = out if out is not None else torch.empty(num_tokens, self.hidden, dtype=torch.bfloat16,
                                                    device=self.device)
        with torch.cuda.device(self.device):
            _lib.call("flyai_moe_combine", ctypes.byref(self.desc), num_tokens, _ptr(pair_out),
                      _ptr(y), _ptr(self.workspace), self.workspace.numel(), _stream())
        return y

    def forward(self, x, input_ids=None, out=None, ids=None, wts=None):
        """y = MoE.forward(x, input_ids); ``ids``/``wts`` (int32 / fp32 [M, k]) receive
        the routing."""
        ids32 = self._check_x(x, input_ids)
        M = x.shape[0]
        y = out if out is not None else torch.empty_like(x)
        with torch.cuda.device(self.device):
            if ids32 is None:
                _lib.call("flyai_moe_forward", ctypes.byref(self.desc), M, _ptr(x),
                          ctypes.byref(self.weights), _ptr(y), _ptr(ids), _ptr(wts),
                          _ptr(self.workspace), self.workspace.numel(), _stream())
            else:
                _lib.call("flyai_moe_route_hash", ctypes.byref(self.desc), M, _ptr(x), _ptr(ids32),
                          _ptr(self.tid2eid), self.tid2eid.shape[0], ctypes.byref(self.weights),
                          None, _ptr(ids), _ptr(wts), _ptr(self.workspace), self.workspace.numel(),
                          _stream())
                _lib.call("flyai_moe_experts", ctypes.byref(self.desc), M, _ptr(x),
                          ctypes.byref(self.weights), _ptr(y), _ptr(self.workspace),
                          self.workspace.numel(), _stream())
        if _lib.checking():
            self.raise_on_error("W4A8MoE.forward")
        return y

    __call__ = forward

    def raise_on_error(self, where="W4A8MoE"):
        """Raise FlyaiDeviceError if a kernel left the error word set (reads and
        clears it; synchronises the host with the stream)."""
        _lib.raise_on_error_bits(self.read_error(clear=True)[0], where)

    def read_error(self, clear=True):
        out = torch.zeros(9, dtype=torch.int32, device=self.device)
        with torch.cuda.device(self.device):
            _lib.call("flyai_moe_read_error", ctypes.byref(self.desc), _ptr(self.workspace),
                      self.workspace.numel(), _ptr(out), 1 if clear else 0, _stream())
        return out.cpu().tolist()
