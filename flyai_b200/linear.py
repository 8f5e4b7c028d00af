"""Host-side API of the dense FP8 linear over the C ABI.

``Fp8Linear`` is the reference's ``linear(x, weight)`` on a float8_e4m3fn weight
with one scale per 128x128 block (vendor/deepseek_v4_ref/inference/model.py:114-124):
act_quant of x per 1x128 -- scale amax/448 for ``scale_fmt=None``, the power of
two 2^ceil(log2(amax/448)) for ``scale_fmt="ue8m0"`` (kernel.py:40-125) --, then
fp8_gemm (kernel.py:203-274), bf16 out.  These are the seven single-row GEMMs of
a V4 decode layer (attention wq_a / wq_b / wkv / wo_b, the indexer's wq_b, the
shared expert's w1 / w3 / w2) that engines/deepseek_v4/v4_fp8_gemv.py re-tiles.

The weight is packed into the kernel's bank at construction.  Several weights
that read the same x share one bank (``Fp8Linear([w1, w3], [s1, s3])``: the
reference's fused shared-expert w1/w3 bank, v4_fp8_gemv.py:280-441); ``split``
cuts the output back into the parts.

All work is stream-ordered on torch's current CUDA stream, with no host
synchronisation; a call allocates only its output (or writes ``out``).
"""
import ctypes

import torch

from . import _lib
from .moe import _ptr, _stream

MAX_TOKENS = 32   # rows per launch the workspace is sized for (more run in slices)


def _scale_dtype(scale):
    if scale.dtype == torch.float32:
        return _lib.LIN_SCALE_F32
    if scale.dtype in (torch.uint8, getattr(torch, "float8_e8m0fnu", torch.uint8)):
        return _lib.LIN_SCALE_E8M0
    raise TypeError(f"weight scale dtype {scale.dtype}: expected float32 or float8_e8m0fnu")


class Fp8Linear:
    """y = linear(x, W) for e4m3 W [N, K] (or several weights stacked along N)
    with 128x128 block scales; x bf16 [..., K] -> y bf16 [..., N]."""

    def __init__(self, weight, scale, scale_fmt=None, max_tokens=MAX_TOKENS, device="cuda"):
        weights = list(weight) if isinstance(weight, (list, tuple)) else [weight]
        scales = list(scale) if isinstance(scale, (list, tuple)) else [scale]
        if len(weights) != len(scales) or not weights:
            raise ValueError("one scale tensor per weight")
        if scale_fmt not in (None, "ue8m0"):
            raise ValueError(f"scale_fmt {scale_fmt!r}: expected None or 'ue8m0'")
        self.device = torch.device(device)
        self.scale_fmt = scale_fmt
        self.K = int(weights[0].shape[1])
        self.parts = [int(w.shape[0]) for w in weights]
        self.N = sum(self.parts)
        self.max_tokens = int(max_tokens)
        lib = _lib.load()
        sizes = []
        for n in self.parts:
            b = ctypes.c_size_t()
            _lib.check("flyai_fp8_linear_bank_bytes", lib.flyai_fp8_linear_bank_bytes(n, self.K, ctypes.byref(b)))
            sizes.append(b.value)
        self.bank = torch.empty(sum(sizes), dtype=torch.uint8, device=self.device)
        wsb = ctypes.c_size_t()
        _lib.check("flyai_fp8_linear_workspace_bytes",
                   lib.flyai_fp8_linear_workspace_bytes(self.max_tokens, self.N, self.K, ctypes.byref(wsb)))
        self.workspace = torch.zeros(wsb.value, dtype=torch.uint8, device=self.device)
        with torch.cuda.device(self.device):
            off = 0
            for w, s, nbytes in zip(weights, scales, sizes):
                if w.shape[1] != self.K:
                    raise ValueError("stacked weights must share K")
                if w.dtype != torch.float8_e4m3fn:
                    raise TypeError(f"weight dtype {w.dtype}: expected float8_e4m3fn")
                wd = w.to(self.device).contiguous().view(torch.uint8)
                sd = s.to(self.device).contiguous()
                fmt = _scale_dtype(sd)
                if fmt == _lib.LIN_SCALE_E8M0:
                    sd = sd.view(torch.uint8)
                if tuple(sd.shape) != (w.shape[0] // 128, self.K // 128):
                    raise ValueError(f"scale shape {tuple(sd.shape)} for weight {tuple(w.shape)}")
                _lib.call("flyai_fp8_linear_pack", int(w.shape[0]), self.K, _ptr(wd), _ptr(sd), fmt,
                          _ptr(self.bank[off:off + nbytes]), _stream())
                off += nbytes

    def forward(self, x, out=None):
        if x.dtype != torch.bfloat16 or x.shape[-1] != self.K:
            raise ValueError(f"x must be bf16 [..., {self.K}]")
        x = x.contiguous()
        M = x.numel() // self.K
        y = out if out is not None else torch.empty(*x.shape[:-1], self.N, dtype=torch.bfloat16,
                                                    device=self.device)
        fmt = _lib.LIN_FMT_UE8M0 if self.scale_fmt == "ue8m0" else _lib.LIN_FMT_AMAX
        with torch.cuda.device(self.device):
            _lib.call("flyai_fp8_linear", M, self.N, self.K, _ptr(x), _ptr(self.bank), fmt, _ptr(y),
                      _ptr(self.workspace), self.workspace.numel(), _stream())
        if _lib.checking():
            self.raise_on_error()
        return y

    __call__ = forward

    def split(self, y):
        """The parts of a stacked bank's output (views along the last dim)."""
        return torch.split(y, self.parts, dim=-1)

    def read_error(self):
        """The workspace's error word (bit 1: a bounded wait gave up); synchronises."""
        return int(self.workspace[:4].view(torch.int32).item())

    def raise_on_error(self, where="Fp8Linear"):
        """Raise FlyaiDeviceError if a kernel left the error word set (reads and
        clears it; synchronises the host with the stream)."""
        bits = self.read_error()
        if bits:
            self.workspace[:4].zero_()
        _lib.raise_on_error_bits(bits, where)
