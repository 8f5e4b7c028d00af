"""Drop-in lever for the DeepSeek MoE blocks the reference stages run.

The reference's DeepSeek engines run the vendored model (vendor/deepseek_v4_ref/
inference/model.py) whose MoE block is ``MoE.forward(x, input_ids) -> y`` (:634-649),
called by ``Block.forward`` as ``self.ffn(x, input_ids)`` (:705).  Its own levers
(engines/deepseek_v4/v4_moe_decode.py:71-90, v4_moe_grouped.py:747-766) rebind
``mod.MoE.forward`` after model.py is executed, keep the previously bound forward as
the fallback, claim some shapes, decline the others with a recorded reason, and
report ``coverage()`` per layer.  ``install(mod)`` does the same with the sm_100a
kernels underneath:

* DeepSeek-V4 layers -- fp4 routed experts (``float4_e2m1fn_x2`` weights with
  ``float8_e8m0fnu`` scales), an fp8 shared expert, the sqrt(softplus) gate, score-
  or hash-routed -- run on ``flyai_b200.v4.W4A8MoE``;
* DeepSeek-V3-style layers -- fp8 experts with 128x128 block scales and a grouped
  sigmoid gate (``KimiMoEGate``, vendor/kimi_k3_ref/modeling_kimi_linear.py:
  666-759) -- run on ``flyai_b200.dsv3.Fp8MoE``.

Each MoE instance packs its bank once, on its first claimed call (the module's
parameters stay as they are).  Declined: tensors not on a CUDA device, non-bf16
input, more than 64 tokens, world_size > 1 (the reference all-reduces the routed
sum across ranks before the shared expert), and expert or gate formats neither
layer takes.  Enabled by ``FLYAI_MOE_DEEPSEEK`` (default on; "0" turns ``install``
into a no-op), read at import like the reference's ``V4_MOE_*`` flags.
"""
import os
import threading

import torch

ENABLED = os.environ.get("FLYAI_MOE_DEEPSEEK", "1") not in ("", "0")
MAX_TOKENS = 64

_LOCK = threading.Lock()
_INSTALLED = []   # modules whose MoE.forward this lever rebound
_INSTALLED_DRAFTERS = []   # MoE instances bound by install_drafter
_ATTEMPTS = [0]   # install() calls


def _decline(moe, why, prev, x, input_ids):
    with _LOCK:
        tally = moe.__dict__.setdefault("_flyai_declined", {})
        tally[why] = tally.get(why, 0) + 1
    return prev(moe, x, input_ids)


def _float4_dtype():
    return getattr(torch, "float4_e2m1fn_x2", None)


def _u8(t):
    return t.detach().contiguous().view(torch.uint8)


def _build_v4(moe):
    from .v4 import W4A8MoE
    gate = moe.gate
    E, H = moe.n_routed_experts, moe.dim
    lo, hi = moe.experts_start_idx, moe.experts_end_idx
    ex0 = moe.experts[lo]
    I = ex0.w1.weight.shape[0]

    def expert(e):
        ex = moe.experts[e]
        return (torch.cat([_u8(ex.w1.weight), _u8(ex.w3.weight)]),
                torch.cat([_u8(ex.w1.scale), _u8(ex.w3.scale)]), _u8(ex.w2.weight), _u8(ex.w2.scale))

    sh = moe.shared_experts

    def shared():
        return (torch.cat([sh.w1.weight.detach(), sh.w3.weight.detach()]),
                torch.cat([_u8(sh.w1.scale), _u8(sh.w3.scale)]), sh.w2.weight.detach(), _u8(sh.w2.scale))

    bias = gate.bias.detach() if gate.bias is not None else torch.zeros(E, device=gate.weight.device)
    tid2eid = gate.tid2eid.detach() if gate.hash else None
    return W4A8MoE(gate.weight.detach(), bias, expert, shared, E, H, I, gate.topk, float(gate.route_scale),
                   float(ex0.swiglu_limit), tid2eid=tid2eid, max_tokens=MAX_TOKENS,
                   device=gate.weight.device, expert_range=(lo, hi) if (lo, hi) != (0, E) else None)


def _build_fp8(moe):
    from .dsv3 import Fp8MoE
    gate = moe.gate
    E, H = moe.n_routed_experts, moe.dim
    ex0 = moe.experts[moe.experts_start_idx]
    I = ex0.w1.weight.shape[0]

    def expert(e):
        ex = moe.experts[e] if e < E else moe.shared_experts
        return (torch.cat([ex.w1.weight.detach(), ex.w3.weight.detach()]),
                torch.cat([ex.w1.scale.detach().float(), ex.w3.scale.detach().float()]),
                ex.w2.weight.detach(), ex.w2.scale.detach().float())

    return Fp8MoE(gate.weight.detach(), gate.e_score_correction_bias.detach(), expert, E, H, I,
                  gate.top_k, gate.num_expert_group, gate.topk_group, float(gate.routed_scaling_factor),
                  n_shared=1, swiglu_limit=float(getattr(ex0, "swiglu_limit", 0.0)), max_tokens=MAX_TOKENS,
                  device=gate.weight.device)


def _layer_kind(moe):
    """'v4', 'fp8' or the reason the block is not claimed."""
    ex0 = moe.experts[moe.experts_start_idx]
    wdt = ex0.w1.weight.dtype
    gate = moe.gate
    if _float4_dtype() is not None and wdt == _float4_dtype():
        if getattr(gate, "score_func", None) != "sqrtsoftplus":
            return "gate"
        if moe.shared_experts.w1.weight.dtype != torch.float8_e4m3fn:
            return "shared-expert-format"
        return "v4"
    if wdt == torch.float8_e4m3fn:
        if not (hasattr(gate, "num_expert_group") and hasattr(gate, "e_score_correction_bias")):
            return "gate"
        if getattr(gate, "moe_router_activation_func", "sigmoid") != "sigmoid":
            return "gate"
        return "fp8"
    return "expert-format"


def _claimed_forward(moe, x, input_ids, prev, world):
    shape = x.shape
    xv = x.reshape(-1, moe.dim)
    if world > 1:
        return _decline(moe, "world_size>1", prev, x, input_ids)
    if xv.device.type != "cuda":
        return _decline(moe, "device", prev, x, input_ids)
    if xv.dtype != torch.bfloat16:
        return _decline(moe, "dtype", prev, x, input_ids)
    if xv.shape[0] > MAX_TOKENS:
        return _decline(moe, "s>64", prev, x, input_ids)
    lever = moe.__dict__.get("_flyai_lever")
    if lever is None:
        kind = moe.__dict__.get("_flyai_kind") or _layer_kind(moe)
        moe.__dict__["_flyai_kind"] = kind
        if kind not in ("v4", "fp8"):
            return _decline(moe, kind, prev, x, input_ids)
        lever = _build_v4(moe) if kind == "v4" else _build_fp8(moe)
        moe.__dict__["_flyai_lever"] = lever
    xv = xv.contiguous()
    if moe.__dict__["_flyai_kind"] == "v4":
        ids = input_ids.reshape(-1) if getattr(lever, "tid2eid", None) is not None else None
        y = lever.forward(xv, ids)
    else:
        y = lever.forward(xv)
    with _LOCK:
        moe.__dict__["_flyai_steps"] = moe.__dict__.get("_flyai_steps", 0) + 1
    return y.view(shape)


def install(mod):
    """Rebind ``mod.MoE.forward`` to the sm_100a path.  Returns True if it took.

    Run after model.py is executed (and after the reference's own levers, whose
    forward then becomes this lever's fallback).  Idempotent; a no-op with
    FLYAI_MOE_DEEPSEEK=0 or without CUDA."""
    _ATTEMPTS[0] += 1
    if not ENABLED or not torch.cuda.is_available():
        return False
    if getattr(mod.MoE.forward, "_flyai_b200", False):
        return False
    prev = mod.MoE.forward
    world = int(getattr(mod, "world_size", 1) or 1)

    def forward(self, x, input_ids):
        return _claimed_forward(self, x, input_ids, prev, world)

    forward._flyai_b200 = True
    forward._flyai_prev = prev
    mod.MoE.forward = forward
    with _LOCK:
        _INSTALLED.append(mod)
    return True


def install_drafter(moes):
    """Per-instance lever for the drafter's MoE blocks (the MTP blocks' ``MoE``
    instances), as the reference binds its drafter lever after MTP construction
    (engines/deepseek_v4/v4_dspark_moe.py:231-305, ``draft_forward``).  Each
    instance's ``forward`` becomes the claimed path with the class's current
    forward (the reference's, or ``install``'s) as its fallback; a drafter block
    of T rows runs as one T-token layer call -- T x k (row, expert) pairs in one
    launch chain, no host sync, routing and fold in the reference's order.
    Unlike the reference's drafter lever it also claims T == 1 and hash-routed
    blocks (one kernel path serves every T <= 64).  Returns how many instances
    it bound; idempotent; a no-op with FLYAI_MOE_DEEPSEEK=0 or without CUDA."""
    _ATTEMPTS[0] += 1
    if not ENABLED or not torch.cuda.is_available():
        return 0
    bound = 0
    for moe in moes:
        if getattr(moe.__dict__.get("forward"), "_flyai_b200", False):
            continue
        prev = type(moe).forward
        world = int(moe.__dict__.get("world_size", 1) or 1)

        def forward(x, input_ids, _moe=moe, _prev=prev, _world=world):
            return _claimed_forward(_moe, x, input_ids, _prev, _world)

        forward._flyai_b200 = True
        moe.forward = forward
        bound += 1
        with _LOCK:
            _INSTALLED_DRAFTERS.append(moe)
    return bound


def uninstall_drafter(moes):
    """Drop the per-instance forwards ``install_drafter`` bound."""
    for moe in moes:
        if getattr(moe.__dict__.get("forward"), "_flyai_b200", False):
            del moe.forward
        with _LOCK:
            if moe in _INSTALLED_DRAFTERS:
                _INSTALLED_DRAFTERS.remove(moe)


def uninstall(mod):
    """Restore the forward that ``install`` replaced."""
    fwd = mod.MoE.forward
    if getattr(fwd, "_flyai_b200", False):
        mod.MoE.forward = fwd._flyai_prev
    with _LOCK:
        if mod in _INSTALLED:
            _INSTALLED.remove(mod)


def attempts():
    return _ATTEMPTS[0]


def installed():
    """Modules whose MoE.forward is this lever right now, and drafter MoE
    instances whose own forward is."""
    with _LOCK:
        return ([m for m in _INSTALLED if getattr(m.MoE.forward, "_flyai_b200", False)] +
                [m for m in _INSTALLED_DRAFTERS if getattr(m.__dict__.get("forward"), "_flyai_b200", False)])


def coverage(module):
    """{layer_id: (claimed steps, {reason: declines})} for every MoE block under
    ``module`` (a model, a stage, or one block) -- "did the lever fire on every
    layer", as engines/deepseek_v4/v4_moe_grouped.py:677-697 reports it.  Under a
    CUDA graph the counters move only while capturing."""
    out = {}
    mods = module.modules() if hasattr(module, "modules") else [module]
    for m in mods:
        if hasattr(m, "experts") and hasattr(m, "experts_start_idx"):
            out[getattr(m, "layer_id", len(out))] = (m.__dict__.get("_flyai_steps", 0),
                                                     dict(m.__dict__.get("_flyai_declined", {})))
    return out
