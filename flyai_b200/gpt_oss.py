"""Drop-in replacement for the GPT-OSS MoE block the reference stages run.

The reference runs GPT-OSS decoder layers from HuggingFace transformers
(phase0/pipeline.py:51-88 ``run_block`` calls each layer; phase0/fastverify.py
replays them in a CUDA graph), whose MoE block is ``GptOssMLP``
(transformers/models/gpt_oss/modeling_gpt_oss.py:134-146):

    forward(hidden_states [B, S, H]) -> (out [B, S, H], router_scores [B*S, k])

or, with native MXFP4 loaded, the hub ``mlp_forward``
(transformers/integrations/mxfp4.py:493-511) returning (out, router_logits).
``B200GptOssMLP`` keeps both signatures.  ``install`` rebinds the forward of the
given layers' ``mlp`` modules in place -- the same plugin mechanism as the
reference's V4 levers (engines/deepseek_v4/v4_moe_grouped.py:747-766): the
previously bound forward is kept, shapes the kernel does not claim (input not
on the layer's GPU, more tokens than the workspace holds) are declined to it
with the reason recorded, and ``coverage()`` reports claimed vs declined.
Enabled per process with ``FLYAI_MOE_B200=1`` (read at import, like the
reference's ``V4_MOE_*`` flags).
"""
import os
import threading
from collections import Counter

import torch

from .moe import Mxfp4MoE

ENABLED = os.environ.get("FLYAI_MOE_B200", "0") == "1"

_LOCK = threading.Lock()
_COVERAGE = Counter()
_INSTALLED = []   # mlp modules whose forward this lever rebound
_ATTEMPTS = [0]   # install() calls


def coverage():
    """{'claimed': n, 'declined:<reason>': n} since import (or the last reset)."""
    with _LOCK:
        return dict(_COVERAGE)


def reset_coverage():
    with _LOCK:
        _COVERAGE.clear()


def _note(key):
    with _LOCK:
        _COVERAGE[key] += 1


class B200GptOssMLP(torch.nn.Module):
    """GptOssMLP with the experts running on the sm_100a kernels."""

    def __init__(self, moe: Mxfp4MoE, fallback=None, return_logits=False):
        super().__init__()
        self.moe = moe
        self.fallback = fallback
        self.return_logits = return_logits

    @classmethod
    def from_checkpoint(cls, router_weight, router_bias, gate_up_blocks, gate_up_scales,
                        gate_up_bias, down_blocks, down_scales, down_bias, top_k,
                        swiglu_limit=7.0, alpha=1.702, max_tokens=64, device="cuda", **kw):
        """Tensors as stored in a GPT-OSS MXFP4 checkpoint
        (``mlp.router.{weight,bias}``, ``mlp.experts.gate_up_proj_{blocks,scales,bias}``,
        ``mlp.experts.down_proj_{blocks,scales,bias}``)."""
        moe = Mxfp4MoE(router_weight, router_bias, gate_up_blocks, gate_up_scales, gate_up_bias,
                       down_blocks, down_scales, down_bias, top_k, swiglu_limit, alpha,
                       max_tokens=max_tokens, device=device)
        return cls(moe, **kw)

    def _decline(self, reason, hidden_states):
        _note("declined:" + reason)
        if self.fallback is None:
            raise RuntimeError(f"B200GptOssMLP cannot run this call ({reason}) and has no fallback")
        return self.fallback(hidden_states)

    def forward(self, hidden_states):
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1])
        if x.device != self.moe.device:
            return self._decline("device", hidden_states)
        if x.shape[0] > self.moe.max_tokens:
            return self._decline("tokens>max_tokens", hidden_states)
        if x.dtype != torch.bfloat16:
            return self._decline("dtype", hidden_states)
        _note("claimed")
        if self.return_logits:
            logits, _, _ = self.moe.route(x, logits=True)
            y = self.moe.experts(x)
            return y.reshape(shape), logits
        y, _, wts = self.moe.forward(x)
        return y.reshape(shape), wts


def install(layers, banks, max_tokens=64, return_logits=False):
    """Rebind ``layer.mlp.forward`` for each decoder layer in ``layers``.

    ``banks[i]`` is the dict of checkpoint tensors of layer i (keys as
    ``B200GptOssMLP.from_checkpoint`` arguments).  Returns the installed
    modules.  The previous forward of each mlp stays reachable as the fallback.
    Stage code calls this when FLYAI_MOE_B200=1 (``ENABLED``); the lever registry
    (flyai_b200.levers) reports a call made with the flag off."""
    _ATTEMPTS[0] += 1
    installed = []
    for layer, bank in zip(layers, banks):
        mlp = layer.mlp
        prev = mlp.forward
        if getattr(prev, "_flyai_b200", False):     # already installed: no cycles
            installed.append(prev.__self__)
            continue
        mod = B200GptOssMLP.from_checkpoint(**bank, max_tokens=max_tokens, fallback=prev,
                                            return_logits=return_logits)
        fwd = mod.forward
        fwd.__func__._flyai_b200 = True
        mlp.forward = fwd
        installed.append(mod)
        with _LOCK:
            _INSTALLED.append(mlp)
    return installed


def attempts():
    return _ATTEMPTS[0]


def installed_count():
    """mlp modules whose forward is this lever right now."""
    with _LOCK:
        return sum(1 for m in _INSTALLED if getattr(m.forward, "_flyai_b200", False))
