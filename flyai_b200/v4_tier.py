"""DeepSeek-V4 MoE layer with its routed experts in host memory (an expert tier).

The reference keeps a local RAM pool of routed experts and a fixed set of GPU
slots, loads the experts a step routes to into slots, and runs the step's experts
from the slots (engines/deepseek_v4/v4_hybrid.py:113-160, the cache of
v4_expert_cache.py).  ``TieredW4A8MoE`` does the same around the sm_100a kernels:

* the routed experts are packed once into the kernel's bank layout and kept in
  pinned host memory; the device holds ``slots`` expert slots plus the fp8 shared
  expert;
* per call the gate runs on the GPU (``flyai_moe_route`` / ``_route_hash``), its
  ids come back to the host (one synchronisation, as the reference's host-side
  slot map needs), missing experts are copied into free or least-recently-used
  slots (one ``cudaMemcpyAsync`` per expert and projection, from pinned memory),
  the slot table goes to the device, and ``flyai_moe_experts_slots`` runs the
  experts from the slots;
* a batch whose experts do not fit in the slots at once runs in token groups that
  do; tokens are independent, so the output is the single-call output.

The output is bit-identical to ``W4A8MoE`` on the full bank.
"""
import ctypes
from collections import OrderedDict

import numpy as np
import torch

from . import _lib
from .moe import _ptr, _stream


def token_groups(ids_rows, slots):
    """Consecutive token groups whose union of experts fits in ``slots``: a list of
    (start, stop).  ``ids_rows``: per token its expert ids."""
    groups, start, union = [], 0, set()
    for t, row in enumerate(ids_rows):
        need = set(int(e) for e in row)
        if len(need) > slots:
            raise ValueError(f"token {t} routes to {len(need)} experts, more than {slots} slots")
        if len(union | need) > slots:
            groups.append((start, t))
            start, union = t, set()
        union |= need
    if start < len(ids_rows):
        groups.append((start, len(ids_rows)))
    return groups


class SlotCache:
    """Least-recently-used assignment of experts to ``slots`` device slots."""

    def __init__(self, slots):
        self.slots = slots
        self.lru = OrderedDict()          # expert -> slot, least recent first
        self.free = list(range(slots - 1, -1, -1))
        self.loads = 0
        self.hits = 0

    def assign(self, experts):
        """Slots for ``experts`` (at most ``slots`` of them): returns (slot of each,
        [(expert, slot) to load]).  Experts of this call are never evicted by it."""
        experts = list(dict.fromkeys(int(e) for e in experts))
        if len(experts) > self.slots:
            raise ValueError(f"{len(experts)} experts for {self.slots} slots")
        want = set(experts)
        loads = []
        for e in experts:
            if e in self.lru:
                self.lru.move_to_end(e)
                self.hits += 1
        for e in experts:
            if e in self.lru:
                continue
            if self.free:
                s = self.free.pop()
            else:
                victim = next(v for v in self.lru if v not in want)
                s = self.lru.pop(victim)
            self.lru[e] = s
            loads.append((e, s))
            self.loads += 1
        return {e: self.lru[e] for e in experts}, loads

    def table(self, num_experts):
        t = np.full(num_experts, -1, np.int32)
        for e, s in self.lru.items():
            t[e] = s
        return t


class TieredW4A8MoE:
    """``W4A8MoE`` with the routed experts in pinned host memory and ``slots``
    device slots (same constructor arguments, plus ``slots``)."""

    def __init__(self, router_w, bias, expert, shared, num_experts, hidden, inter, top_k,
                 route_scale, swiglu_limit, slots, tid2eid=None, max_tokens=64, device=None):
        _lib.load()
        device = torch.device(device or router_w.device)
        if device.type != "cuda":
            raise ValueError("TieredW4A8MoE runs on a CUDA device")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        E = num_experts
        if not 1 <= slots <= E:
            raise ValueError(f"slots must be in [1, {E}]")
        self.device, self.num_experts, self.hidden, self.top_k = device, E, hidden, top_k
        self.slots, self.max_tokens = slots, max_tokens
        n_shared = 1 if shared is not None else 0
        self.desc = _lib.Desc(
            abi_version=_lib.ABI_VERSION, format=_lib.FMT_FP4_W4A8, gating=_lib.GATE_SQRTSOFTPLUS,
            activation=_lib.ACT_SILU, num_experts=E, top_k=top_k, hidden=hidden, inter=inter,
            expert_begin=0, expert_end=E, max_tokens=max_tokens, swiglu_limit=swiglu_limit,
            swiglu_alpha=0.0, n_group=1, topk_group=1, route_scale=route_scale, n_shared=n_shared)
        _lib.call("flyai_moe_check_desc", ctypes.byref(self.desc))
        # the cache bank: the bank of a descriptor holding `slots` routed experts
        self.cdesc = _lib.Desc.from_buffer_copy(self.desc)
        self.cdesc.expert_end = slots
        one = _lib.Desc.from_buffer_copy(self.desc)
        one.expert_end, one.n_shared = 1, 0
        self.per = {p: self._bytes(one, p) for p in (_lib.PROJ_W13, _lib.PROJ_W2)}
        self.host = {p: torch.empty(E * self.per[p], dtype=torch.uint8, pin_memory=True)
                     for p in self.per}
        self.cache = {p: torch.zeros(self._bytes(self.cdesc, p), dtype=torch.uint8, device=device)
                      for p in self.per}
        stage = {p: torch.empty(self.per[p], dtype=torch.uint8, device=device) for p in self.per}
        with torch.cuda.device(device):
            for e in range(E):
                w13, s13, w2, s2 = expert(e)
                for p, w, s in ((_lib.PROJ_W13, w13, s13), (_lib.PROJ_W2, w2, s2)):
                    d = _lib.Desc.from_buffer_copy(one)
                    d.expert_begin, d.expert_end = e, e + 1
                    wd = w.to(device).contiguous().view(torch.uint8)
                    sd = s.to(device).contiguous().view(torch.uint8)
                    _lib.call("flyai_moe_pack_fp4", ctypes.byref(d), p, _ptr(wd), _ptr(sd),
                              _ptr(stage[p]), _stream())
                    self.host[p][e * self.per[p]:(e + 1) * self.per[p]].copy_(stage[p])
            if n_shared:
                w13, s13, w2, s2 = shared()
                for p, w, s in ((_lib.PROJ_W13, w13, s13), (_lib.PROJ_W2, w2, s2)):
                    wd = w.to(device).contiguous().view(torch.uint8)
                    sd = s.to(device).contiguous().view(torch.uint8)
                    _lib.call("flyai_moe_pack_shared_fp8", ctypes.byref(self.cdesc), p, _ptr(wd),
                              _ptr(sd), _ptr(self.cache[p]), _stream())
            torch.cuda.current_stream().synchronize()
        self.router_w = router_w.to(device=device, dtype=torch.bfloat16).contiguous()
        self.bias = bias.to(device=device, dtype=torch.float32).contiguous()
        self.tid2eid = (tid2eid.to(device=device, dtype=torch.int32).contiguous()
                        if tid2eid is not None else None)
        self.weights = _lib.Weights(router_w=self.router_w.data_ptr(), router_b=self.bias.data_ptr(),
                                    w13=self.cache[_lib.PROJ_W13].data_ptr(), w13_bias=None,
                                    w2=self.cache[_lib.PROJ_W2].data_ptr(), w2_bias=None)
        nbytes = ctypes.c_size_t()
        _lib.call("flyai_moe_workspace_bytes", ctypes.byref(self.desc), ctypes.byref(nbytes))
        self.workspace = torch.zeros(nbytes.value, dtype=torch.uint8, device=device)
        self.slot_cache = SlotCache(slots)
        self.table_host = torch.full((E,), -1, dtype=torch.int32).pin_memory()
        self.table = torch.full((E,), -1, dtype=torch.int32, device=device)

    @classmethod
    def from_layer(cls, layer, slots, max_tokens=64, device=None, shared=True):
        """Build from a ``flyai_b200.synth.V4Layer``."""
        return cls(layer.router_w, layer.bias, layer.expert, layer.shared if shared else None,
                   layer.num_experts, layer.hidden, layer.inter, layer.top_k, layer.route_scale,
                   layer.swiglu_limit, slots, tid2eid=layer.tid2eid, max_tokens=max_tokens,
                   device=device)

    def _bytes(self, d, proj):
        n = ctypes.c_size_t()
        _lib.call("flyai_moe_packed_bytes", ctypes.byref(d), proj, ctypes.byref(n))
        return n.value

    def _route(self, x, ids32):
        M = x.shape[0]
        ids = torch.empty(M, self.top_k, dtype=torch.int32, device=self.device)
        if ids32 is None:
            _lib.call("flyai_moe_route", ctypes.byref(self.desc), M, _ptr(x), ctypes.byref(self.weights),
                      None, _ptr(ids), None, _ptr(self.workspace), self.workspace.numel(), _stream())
        else:
            _lib.call("flyai_moe_route_hash", ctypes.byref(self.desc), M, _ptr(x), _ptr(ids32),
                      _ptr(self.tid2eid), self.tid2eid.shape[0], ctypes.byref(self.weights), None,
                      _ptr(ids), None, _ptr(self.workspace), self.workspace.numel(), _stream())
        return ids

    def _run(self, x, ids32, ids_host, y, routed):
        _, loads = self.slot_cache.assign(ids_host.ravel())
        for e, s in loads:
            for p in self.per:
                n = self.per[p]
                self.cache[p][s * n:(s + 1) * n].copy_(self.host[p][e * n:(e + 1) * n], non_blocking=True)
        self.table_host.copy_(torch.from_numpy(self.slot_cache.table(self.num_experts)))
        self.table.copy_(self.table_host, non_blocking=True)
        if not routed:
            self._route(x, ids32)    # the plan of exactly these tokens in the workspace
        _lib.call("flyai_moe_experts_slots", ctypes.byref(self.desc), x.shape[0], _ptr(x),
                  ctypes.byref(self.weights), _ptr(self.table), self.slots, _ptr(y),
                  _ptr(self.workspace), self.workspace.numel(), _stream())

    def forward(self, x, input_ids=None, out=None):
        """y = MoE.forward(x, input_ids), the routed experts served from the slots."""
        if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != self.hidden or x.device != self.device:
            raise ValueError(f"x must be bf16 [M, {self.hidden}] on the layer's device")
        if x.shape[0] > self.max_tokens:
            raise ValueError(f"at most {self.max_tokens} tokens per call")
        x = x.contiguous()
        ids32 = None
        if self.tid2eid is not None:
            if input_ids is None or input_ids.numel() != x.shape[0]:
                raise ValueError("a hash-routed layer needs one input id per token")
            ids32 = input_ids.to(device=self.device, dtype=torch.int32).contiguous().view(-1)
        y = out if out is not None else torch.empty_like(x)
        M = x.shape[0]
        if M == 0:
            return y
        with torch.cuda.device(self.device):
            ids_host = self._route(x, ids32).cpu().numpy()      # the one host synchronisation
            groups = token_groups(ids_host, self.slots)
            for a, b in groups:
                # one group: the workspace already holds its plan
                self._run(x[a:b], None if ids32 is None else ids32[a:b], ids_host[a:b], y[a:b],
                          routed=len(groups) == 1)
        if _lib.checking():
            self.raise_on_error("TieredW4A8MoE.forward")
        return y

    __call__ = forward

    def stats(self):
        return {"slots": self.slots, "loads": self.slot_cache.loads, "hits": self.slot_cache.hits,
                "resident": len(self.slot_cache.lru)}

    def read_error(self, clear=True):
        out = torch.zeros(9, dtype=torch.int32, device=self.device)
        with torch.cuda.device(self.device):
            _lib.call("flyai_moe_read_error", ctypes.byref(self.desc), _ptr(self.workspace),
                      self.workspace.numel(), _ptr(out), 1 if clear else 0, _stream())
        return out.cpu().tolist()

    def raise_on_error(self, where="TieredW4A8MoE"):
        bits = self.read_error(clear=True)[0]
        if bits & 2:
            raise _lib.FlyaiDeviceError(f"{where}: a routed expert was not in a slot")
        _lib.raise_on_error_bits(bits, where)
