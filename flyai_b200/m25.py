"""Host-side API of the MiniMax-M2.5-style NVFP4 MoE layer over the C ABI.

``Nvfp4MoE`` owns the packed NVFP4 expert banks, the router and a workspace on
one device, with the reference's operator surface:

* ``route(x)``   -> (logits fp32 holding bf16 values, topk_idx, topk_weight) --
  MiniMaxM2TopKRouter.forward (transformers/models/minimax_m2/modeling_minimax_m2.py;
  ids in torch.topk(sorted=False)'s CPU order)
* ``forward(x)`` -> y bf16 -- MiniMaxM2SparseMoeBlock.forward
* ``self(h, router_logits)`` -> y bf16 -- the FusedMoE call of the M2.5 stage,
  ``self.moe(h, rl)`` with rl = F.linear(h, gate) computed by the caller
  (engines/minimax_m25/m25_stage.py:412-416): routes from the passed logits

Stream-ordered on torch's current CUDA stream, no host synchronisation and no
allocation after construction.
"""
import ctypes
import os

import torch

from . import _lib
from .dsv3 import Fp8MoE
from .moe import _ptr, _stream


class Nvfp4MoE(Fp8MoE):
    """NVFP4 experts (e2m1 + e4m3 block-16 scales + fp32 global scale per tensor),
    sigmoid top-k gate over bf16 logits with a correction bias, bf16 SiLU-gated
    experts, bf16 fold in ascending expert id."""

    def __init__(self, router_w, bias, expert, num_experts, hidden, inter, top_k,
                 route_scale=1.0, max_tokens=64, device=None, experts=None, expert_range=None,
                 scales_swizzled=False):
        """``expert(e)`` -> (w13 uint8 [2I, H/2] = [w1; w3] packed nibbles, s13 e4m3
        [2I, H/16], g13 fp32 [2] (w1's, w3's weight_scale_2), w2 uint8 [H, I/2], s2 e4m3
        [H, I/16], g2 fp32 [1]) -- the ModelOpt NVFP4 tensors of one expert; with
        ``scales_swizzled`` s13 / s2 come in the block-scale layout vLLM swizzles a
        loaded layer's scales into (flyai_moe_pack_nvfp4_swizzled), as they are read
        from a FusedMoE layer after loading.
        ``expert_range`` = (lo, hi) makes an expert-parallel shard (see Fp8MoE)."""
        _lib.load()
        device = torch.device(device or router_w.device)
        if device.type != "cuda":
            raise ValueError("Nvfp4MoE runs on a CUDA device")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        E, H, I = num_experts, hidden, inter
        lo, hi = expert_range if expert_range is not None else (0, E)
        self.device = device
        self.num_experts, self.hidden, self.inter, self.top_k = E, H, I, top_k
        self.n_shared = 0
        self.expert_range = (lo, hi)
        self.scales_swizzled = scales_swizzled
        self.desc = _lib.Desc(
            abi_version=_lib.ABI_VERSION, format=_lib.FMT_NVFP4, gating=_lib.GATE_SIGMOID_BF16,
            activation=_lib.ACT_SILU_BF16, num_experts=E, top_k=top_k, hidden=H, inter=I,
            expert_begin=lo, expert_end=hi, max_tokens=max_tokens, swiglu_limit=0.0,
            swiglu_alpha=0.0, n_group=1, topk_group=1, route_scale=route_scale, n_shared=0)
        _lib.call("flyai_moe_check_desc", ctypes.byref(self.desc))
        self.router_w = router_w.to(device=device, dtype=torch.bfloat16).contiguous()
        self.bias = bias.to(device=device, dtype=torch.float32).contiguous()
        todo = [e for e in (range(E) if experts is None else sorted(set(int(e) for e in experts)))
                if lo <= e < hi]
        self.w13 = self._bank(_lib.PROJ_W13, full=experts is None)
        self.w2 = self._bank(_lib.PROJ_W2, full=experts is None)
        for e in todo:
            w13, s13, g13, w2, s2, g2 = expert(e)
            self._pack_nv(e, _lib.PROJ_W13, self.w13, w13, s13, g13)
            self._pack_nv(e, _lib.PROJ_W2, self.w2, w2, s2, g2)
        self.weights = _lib.Weights(router_w=self.router_w.data_ptr(), router_b=self.bias.data_ptr(),
                                    w13=self.w13.data_ptr(), w13_bias=None,
                                    w2=self.w2.data_ptr(), w2_bias=None)
        nbytes = ctypes.c_size_t()
        _lib.call("flyai_moe_workspace_bytes", ctypes.byref(self.desc), ctypes.byref(nbytes))
        self.workspace = torch.zeros(nbytes.value, dtype=torch.uint8, device=device)
        self.max_tokens = max_tokens

    @classmethod
    def from_layer(cls, layer, max_tokens=64, device=None, experts=None, expert_range=None):
        """Build from a ``flyai_b200.synth.M25Layer``."""
        return cls(layer.router_w, layer.bias, layer.expert, layer.num_experts, layer.hidden,
                   layer.inter, layer.top_k, route_scale=layer.route_scale,
                   max_tokens=max_tokens, device=device, experts=experts, expert_range=expert_range)

    def _pack_nv(self, e, proj, bank, blocks, scales, gscale):
        """Pack expert e alone: its tiles go to e's slot of the bank, its global
        scale(s) to e's entry of the table after the tiles."""
        d = self._one_desc(e)
        per = ctypes.c_size_t()
        _lib.call("flyai_moe_packed_bytes", ctypes.byref(d), proj, ctypes.byref(per))
        blocks = blocks.to(self.device).contiguous().view(torch.uint8)
        scales = scales.to(self.device).contiguous().view(torch.uint8)
        g = gscale.to(device=self.device, dtype=torch.float32).contiguous()
        stage = torch.empty(per.value, dtype=torch.uint8, device=self.device)
        with torch.cuda.device(self.device):
            _lib.call("flyai_moe_pack_nvfp4_swizzled" if self.scales_swizzled else "flyai_moe_pack_nvfp4",
                      ctypes.byref(d), proj, _ptr(blocks), _ptr(scales), _ptr(g), _ptr(stage), _stream())
        ng = 2 if proj == _lib.PROJ_W13 else 1
        expert_bytes = self._expert_bytes(proj)
        if per.value != (expert_bytes + ng * 4 + 255) // 256 * 256:
            raise RuntimeError("NVFP4 bank layout of the library and of this module disagree")
        slot = self._slot(e)
        bank[slot * expert_bytes:(slot + 1) * expert_bytes].copy_(stage[:expert_bytes])
        lo, hi = self.expert_range
        goff = (hi - lo) * expert_bytes
        bank[goff + slot * ng * 4: goff + (slot + 1) * ng * 4].copy_(stage[expert_bytes:expert_bytes + ng * 4])

    def _expert_bytes(self, proj):
        """Tile bytes of one expert (nv4.cuh: 128 rows x 128 K of nibbles + two 512-byte
        scale chunks per tile; W13 blocks hold the w1 and the w3 tile)."""
        H, I = self.hidden, self.inter
        tiles = 2 if proj == _lib.PROJ_W13 else 1
        rb = (I if proj == _lib.PROJ_W13 else H) // 128
        kb = (H if proj == _lib.PROJ_W13 else I) // 128
        return tiles * (128 * 64 + 2 * 512) * rb * kb

    def fused_moe(self, hidden_states, router_logits=None, out=None):
        """The M2.5 stage's ``self.moe(h, router_logits)``: routed from the caller's bf16
        logits [M, E] (flyai_moe_route_logits), or from the layer's own router when
        they are None."""
        if router_logits is None:
            return Fp8MoE.forward(self, hidden_states, out=out)
        self._check_x(hidden_states)
        M = hidden_states.shape[0]
        rl = router_logits.to(device=self.device, dtype=torch.bfloat16).contiguous()
        if rl.shape != (M, self.num_experts):
            raise ValueError(f"router_logits must be [M, {self.num_experts}]")
        y = out if out is not None else torch.empty_like(hidden_states)
        with torch.cuda.device(self.device):
            _lib.call("flyai_moe_route_logits", ctypes.byref(self.desc), M, _ptr(hidden_states), _ptr(rl),
                      ctypes.byref(self.weights), None, None, _ptr(self.workspace),
                      self.workspace.numel(), _stream())
            _lib.call("flyai_moe_experts", ctypes.byref(self.desc), M, _ptr(hidden_states),
                      ctypes.byref(self.weights), _ptr(y), _ptr(self.workspace),
                      self.workspace.numel(), _stream())
        return y

    __call__ = fused_moe


# ---- the M2.5 stage lever ---------------------------------------------------
ENABLED = os.environ.get("FLYAI_MOE_M25", "1") not in ("", "0")
_INSTALLED = []
_ATTEMPTS = [0]


def install(layers, build):
    """Replace each M2.5 stage layer's FusedMoE -- ``layer.moe``, which the stage
    calls as ``self.moe(h, router_logits)`` (engines/minimax_m25/m25_stage.py:
    412-416) -- by the ``Nvfp4MoE`` that ``build(layer)`` returns (built from the
    layer's ModelOpt NVFP4 tensors).  The replaced module stays reachable as
    ``layer._flyai_prev_moe``.  A no-op with FLYAI_MOE_M25=0.  Returns the number
    of layers replaced."""
    _ATTEMPTS[0] += 1
    if not ENABLED:
        return 0
    n = 0
    for layer in layers:
        if isinstance(layer.moe, Nvfp4MoE):
            continue
        layer._flyai_prev_moe = layer.moe
        layer.moe = build(layer)
        _INSTALLED.append(layer)
        n += 1
    return n


def attempts():
    return _ATTEMPTS[0]


def installed():
    """Stage layers whose ``moe`` is this lever's module right now."""
    return [layer for layer in _INSTALLED if isinstance(layer.moe, Nvfp4MoE)]
