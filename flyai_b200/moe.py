"""Host-side API over the C ABI: one quantized MoE layer resident on a B200.

``Mxfp4MoE`` owns the packed expert banks, the router weights and a workspace
on one device, and exposes the reference's operator surface:

* ``route(x)``   -> (logits, topk_ids, topk_weights)  -- GptOssTopKRouter.forward
  (transformers/models/gpt_oss/modeling_gpt_oss.py:125-131; logits bf16,
  ids int64 like torch.topk, weights bf16)
* ``forward(x)`` -> (y, topk_ids, topk_weights)       -- GptOssMLP.forward's
  expert output and router scores (modeling_gpt_oss.py:140-146)
* ``experts_pairs(x)`` / ``combine(pairs)``           -- the expert-parallel halves

All work is stream-ordered on torch's current CUDA stream; nothing synchronises
the host and nothing allocates after construction, so a forward can be captured
in a CUDA graph.  Inputs must be bf16, contiguous, on the layer's device.
"""
import ctypes

import torch

from . import _lib


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


class Mxfp4MoE:
    """A GPT-OSS-style MXFP4 MoE layer (softmax-over-top-k router, clamped SwiGLU)."""

    def __init__(self, router_w, router_b, w13_blocks, w13_scales, w13_bias, w2_blocks,
                 w2_scales, w2_bias, top_k, limit=7.0, alpha=1.702, expert_range=None,
                 max_tokens=64, device=None):
        """Weights in the reference's native MXFP4 layout (Mxfp4GptOssExperts,
        transformers/integrations/mxfp4.py:357-386):
        router_w bf16 [E, H], router_b bf16 [E]; w13_blocks uint8 [El, 2I, H/32, 16],
        w13_scales uint8 [El, 2I, H/32], w13_bias [El, 2I]; w2_blocks uint8
        [El, H, I/32, 16], w2_scales uint8 [El, H, I/32], w2_bias [El, H], where
        El = experts of ``expert_range`` (default: all)."""
        lib = _lib.load()
        device = torch.device(device or router_w.device)
        if device.type != "cuda":
            raise ValueError("Mxfp4MoE runs on a CUDA device")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        E, H = router_w.shape
        I = w2_blocks.shape[2] * 32
        lo, hi = expert_range if expert_range is not None else (0, E)
        El = hi - lo
        if w13_blocks.shape[0] != El or w2_blocks.shape[0] != El:
            raise ValueError("expert banks must hold exactly the experts of expert_range")
        self.device = device
        self.num_experts, self.hidden, self.inter, self.top_k = E, H, I, top_k
        self.expert_range = (lo, hi)
        self.desc = _lib.Desc(
            abi_version=_lib.ABI_VERSION, format=_lib.FMT_MXFP4, gating=_lib.GATE_SOFTMAX_TOPK,
            activation=_lib.ACT_GPTOSS_SWIGLU, num_experts=E, top_k=top_k, hidden=H, inter=I,
            expert_begin=lo, expert_end=hi, max_tokens=max_tokens, swiglu_limit=limit,
            swiglu_alpha=alpha)
        _lib.call("flyai_moe_check_desc", ctypes.byref(self.desc))
        dev = dict(device=device)
        self.router_w = router_w.to(**dev, dtype=torch.bfloat16).contiguous()
        self.router_b = (router_b.to(**dev, dtype=torch.bfloat16).contiguous()
                         if router_b is not None else None)
        self.w13_bias = (w13_bias.to(**dev, dtype=torch.float32).contiguous()
                         if w13_bias is not None else None)
        self.w2_bias = (w2_bias.to(**dev, dtype=torch.float32).contiguous()
                        if w2_bias is not None else None)
        self.w13 = self._pack(_lib.PROJ_W13, w13_blocks, w13_scales)
        self.w2 = self._pack(_lib.PROJ_W2, w2_blocks, w2_scales)
        self.weights = _lib.Weights(
            router_w=self.router_w.data_ptr(),
            router_b=self.router_b.data_ptr() if self.router_b is not None else None,
            w13=self.w13.data_ptr(),
            w13_bias=self.w13_bias.data_ptr() if self.w13_bias is not None else None,
            w2=self.w2.data_ptr(),
            w2_bias=self.w2_bias.data_ptr() if self.w2_bias is not None else None)
        nbytes = ctypes.c_size_t()
        _lib.call("flyai_moe_workspace_bytes", ctypes.byref(self.desc), ctypes.byref(nbytes))
        self.workspace = torch.zeros(max(nbytes.value, 256), dtype=torch.uint8, **dev)
        self.max_tokens = max_tokens

    @classmethod
    def from_layer(cls, layer, expert_range=None, max_tokens=64, device="cuda"):
        """Build from a ``flyai_b200.synth.GptOssLayer`` (or anything with its fields)."""
        lo, hi = expert_range if expert_range is not None else (0, layer.router_w.shape[0])
        sl = slice(lo, hi)
        return cls(layer.router_w, layer.router_b, layer.w13_blocks[sl], layer.w13_scales[sl],
                   layer.w13_bias[sl], layer.w2_blocks[sl], layer.w2_scales[sl],
                   layer.w2_bias[sl], layer.top_k, layer.limit, layer.alpha,
                   expert_range=(lo, hi), max_tokens=max_tokens, device=device)

    def _pack(self, proj, blocks, scales):
        nbytes = ctypes.c_size_t()
        _lib.call("flyai_moe_packed_bytes", ctypes.byref(self.desc), proj, ctypes.byref(nbytes))
        out = torch.empty(max(nbytes.value, 16), dtype=torch.uint8, device=self.device)
        if nbytes.value == 0:
            return out
        b = blocks.to(self.device, dtype=torch.uint8).contiguous()
        s = scales.to(self.device, dtype=torch.uint8).contiguous()
        _lib.call("flyai_moe_pack_mxfp4", ctypes.byref(self.desc), proj, _ptr(b), _ptr(s),
                  _ptr(out), _stream())
        torch.cuda.current_stream().synchronize()   # load time only: b/s are temporaries
        return out

    # ---- checks shared by the entry points ----
    def _check_x(self, x):
        if x.device != self.device or x.dtype != torch.bfloat16 or x.dim() != 2:
            raise ValueError("x must be a 2-D bf16 tensor on the layer's device")
        if x.shape[1] != self.hidden:
            raise ValueError(f"x has {x.shape[1]} features, layer expects {self.hidden}")
        if x.shape[0] > self.max_tokens:
            raise ValueError(f"{x.shape[0]} tokens exceed max_tokens={self.max_tokens}")
        return x.contiguous()

    def route(self, x, logits=True):
        x = self._check_x(x)
        M = x.shape[0]
        lg = torch.empty(M, self.num_experts, dtype=torch.bfloat16, device=self.device) if logits else None
        ids = torch.empty(M, self.top_k, dtype=torch.int32, device=self.device)
        wts = torch.empty(M, self.top_k, dtype=torch.bfloat16, device=self.device)
        _lib.call("flyai_moe_route", ctypes.byref(self.desc), M, _ptr(x), ctypes.byref(self.weights),
                  _ptr(lg), _ptr(ids), _ptr(wts), _ptr(self.workspace),
                  self.workspace.numel(), _stream())
        return lg, ids, wts

    def read_plan(self, num_tokens):
        """(counts [El], offsets [El+1], perm [M*k]) int32 left by the last route()."""
        El = self.expert_range[1] - self.expert_range[0]
        counts = torch.empty(El, dtype=torch.int32, device=self.device)
        offsets = torch.empty(El + 1, dtype=torch.int32, device=self.device)
        perm = torch.empty(num_tokens * self.top_k, dtype=torch.int32, device=self.device)
        _lib.call("flyai_moe_read_plan", ctypes.byref(self.desc), num_tokens, _ptr(self.workspace),
                  self.workspace.numel(), _ptr(counts), _ptr(offsets), _ptr(perm), _stream())
        return counts, offsets, perm

    def read_error(self, clear=True):
        """(error bits, detail words) kernels left in the workspace; see flyai_moe_read_error."""
        out = torch.zeros(9, dtype=torch.int32, device=self.device)
        _lib.call("flyai_moe_read_error", ctypes.byref(self.desc), _ptr(self.workspace),
                  self.workspace.numel(), _ptr(out), int(clear), _stream())
        host = out.cpu().tolist()
        return host[0], host[1:]

    def forward(self, x, out=None):
        """Whole layer on one GPU: y bf16 [M, H], topk ids int32 [M, k], weights bf16 [M, k]."""
        x = self._check_x(x)
        M = x.shape[0]
        y = out if out is not None else torch.empty(M, self.hidden, dtype=torch.bfloat16, device=self.device)
        ids = torch.empty(M, self.top_k, dtype=torch.int32, device=self.device)
        wts = torch.empty(M, self.top_k, dtype=torch.bfloat16, device=self.device)
        _lib.call("flyai_moe_forward", ctypes.byref(self.desc), M, _ptr(x), ctypes.byref(self.weights),
                  _ptr(y), _ptr(ids), _ptr(wts), _ptr(self.workspace),
                  self.workspace.numel(), _stream())
        if _lib.checking():
            self.raise_on_error("Mxfp4MoE.forward")
        return y, ids, wts

    def raise_on_error(self, where="Mxfp4MoE"):
        """Raise FlyaiDeviceError if a kernel left the error word set (reads and
        clears it; synchronises the host with the stream)."""
        _lib.raise_on_error_bits(self.read_error(clear=True)[0], where)

    def experts(self, x, out=None):
        """Experts + combine on the routing of the last ``route(x)`` (same stream)."""
        x = self._check_x(x)
        M = x.shape[0]
        y = out if out is not None else torch.empty(M, self.hidden, dtype=torch.bfloat16, device=self.device)
        _lib.call("flyai_moe_experts", ctypes.byref(self.desc), M, _ptr(x), ctypes.byref(self.weights),
                  _ptr(y), _ptr(self.workspace), self.workspace.numel(), _stream())
        return y

    def experts_pairs(self, x, pair_out=None):
        """This shard's weighted per-(token, slot) rows, bf16 [M*k, H]; other rows zero.
        Requires ``route(x)`` on the same stream first."""
        x = self._check_x(x)
        M = x.shape[0]
        if pair_out is None:
            pair_out = torch.empty(M * self.top_k, self.hidden, dtype=torch.bfloat16, device=self.device)
        _lib.call("flyai_moe_experts_pairs", ctypes.byref(self.desc), M, _ptr(x),
                  ctypes.byref(self.weights), _ptr(pair_out), _ptr(self.workspace),
                  self.workspace.numel(), _stream())
        return pair_out

    def experts_ep(self, x, peers):
        """Expert parallel over peer memory (flyai_moe_experts_ep): this rank's
        weighted pair rows into every rank's mailbox, then its flag raised.
        Requires ``route(x)`` on the same stream first.  Returns the status code
        (``_lib.ERR_UNSUPPORTED`` when the shape has no peer-memory path)."""
        x = self._check_x(x)
        st = _lib.load().flyai_moe_experts_ep(ctypes.byref(self.desc), x.shape[0], _ptr(x),
                                              ctypes.byref(self.weights), ctypes.byref(peers),
                                              _ptr(self.workspace), self.workspace.numel(),
                                              _stream())
        if st not in (_lib.OK, _lib.ERR_UNSUPPORTED):
            _lib.check("flyai_moe_experts_ep", st)
        return st

    def forward_ep(self, x, peers, ids=None, wts=None):
        """Expert parallel at verify size in one launch per rank (flyai_moe_forward_ep):
        route every token over all experts, run this shard's experts, store their pair
        rows into every rank's mailbox, raise this rank's flag.  x replicated on every
        rank.  Optional outputs: ids int32 [M, k], wts bf16 [M, k].  Returns the status
        code (``_lib.ERR_UNSUPPORTED`` for shapes without this path)."""
        x = self._check_x(x)
        st = _lib.load().flyai_moe_forward_ep(ctypes.byref(self.desc), x.shape[0], _ptr(x),
                                              ctypes.byref(self.weights), ctypes.byref(peers),
                                              _ptr(ids), _ptr(wts), _ptr(self.workspace),
                                              self.workspace.numel(), _stream())
        if st not in (_lib.OK, _lib.ERR_UNSUPPORTED):
            _lib.check("flyai_moe_forward_ep", st)
        return st

    def combine_ep(self, num_tokens, peers, out=None):
        """Wait for every rank's rows (bounded) and fold them: y bf16 [M, H]."""
        y = out if out is not None else torch.empty(num_tokens, self.hidden, dtype=torch.bfloat16, device=self.device)
        _lib.call("flyai_moe_combine_ep", ctypes.byref(self.desc), num_tokens, ctypes.byref(peers),
                  _ptr(y), _ptr(self.workspace), self.workspace.numel(), _stream())
        if _lib.checking():
            self.raise_on_error("Mxfp4MoE.combine_ep")
        return y

    def combine(self, pair_out, num_tokens, out=None):
        y = out if out is not None else torch.empty(num_tokens, self.hidden, dtype=torch.bfloat16, device=self.device)
        _lib.call("flyai_moe_combine", ctypes.byref(self.desc), num_tokens, _ptr(pair_out), _ptr(y),
                  _ptr(self.workspace), self.workspace.numel(), _stream())
        return y


def set_profile_events(start=None, stop=None):
    """Record torch.cuda.Event `start`/`stop` around every later expert-kernel
    launch (both None switches it off); for timing that kernel alone."""
    def h(e):
        if e is None:
            return None
        if not e.cuda_event:   # torch creates the CUDA event on its first record
            e.record()
        return ctypes.c_void_p(e.cuda_event)
    _lib.call("flyai_moe_set_profile_events", h(start), h(stop))


def launch_count():
    """Kernels this process launched through the library so far."""
    return int(_lib.load().flyai_moe_launch_count())
