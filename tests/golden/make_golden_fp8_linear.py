"""Generate the dense FP8 linear fixtures by running the reference itself.

    python tests/golden/make_golden_fp8_linear.py --reference <FlyAI checkout>

The reference code that runs (nothing of it is copied into this repository):
``engines/deepseek_v4/v4_ref_cpu.load_ref()`` -- the vendored DeepSeek-V4 model
module with the reference's own CPU kernels installed (act_quant and fp8_gemm of
engines/deepseek_v4/v4_kernels_cpu.py) -- and its module-level ``linear``
(vendor/deepseek_v4_ref/inference/model.py:114-124) on a float8_e4m3fn weight
carrying ``.scale``, under default dtype bf16.  The module globals ``scale_fmt``
and ``scale_dtype`` are set per case as a checkpoint configures them: "ue8m0" +
float8_e8m0fnu (V4, e8m0 block scales) or None + float32 (fp32 block scales).

Inputs come from ``flyai_b200.synth`` (seeded); each fixture keeps a SHA-256 of
the weight, its scale and the tokens.
"""
import argparse
import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from flyai_b200 import synth  # noqa: E402

CASES = [
    # name, N, K, tokens, seed, e8m0 weight scales + ue8m0 activation scales
    ("lin_small_ue8m0_m5", 384, 1024, 5, 0, True),
    ("lin_small_f32_m33", 256, 512, 33, 1, False),
    ("lin_v4_wkv_m1", 512, 4096, 1, 2, True),
    ("lin_v4_wq_a_m4", 1024, 4096, 4, 3, True),
    ("lin_v4_w2_m1", 4096, 2048, 1, 4, True),
    ("lin_f32_k7168_m8", 1024, 7168, 8, 5, False),
]


def load_reference(root):
    sys.path.insert(0, os.path.join(root, "engines", "deepseek_v4"))
    import v4_ref_cpu
    return v4_ref_cpu.load_ref()


def digest_of(w, s, x):
    h = hashlib.sha256()
    for t in (w, s, x):
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def run_reference(ref, w, s, x, e8m0):
    saved = (ref.scale_fmt, ref.scale_dtype)
    ref.scale_fmt = "ue8m0" if e8m0 else None
    ref.scale_dtype = torch.float8_e8m0fnu if e8m0 else torch.float32
    try:
        weight = torch.nn.Parameter(w.clone(), requires_grad=False)
        weight.scale = s.clone().view(torch.float8_e8m0fnu) if e8m0 else s.clone()
        with torch.no_grad(), ref.set_dtype(torch.bfloat16):
            y = ref.linear(x.clone(), weight)
    finally:
        ref.scale_fmt, ref.scale_dtype = saved
    assert y.dtype == torch.bfloat16 and tuple(y.shape) == (x.shape[0], w.shape[0])
    return y


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of a FlyAI checkout")
    a = ap.parse_args()
    ref = load_reference(a.reference)
    for name, N, K, M, seed, e8m0 in CASES:
        w, s = synth.make_fp8_linear(N, K, seed=seed, e8m0=e8m0)
        x = synth.make_tokens(M, K, seed=seed)
        y = run_reference(ref, w, s, x, e8m0)
        np.savez_compressed(os.path.join(HERE, name + ".npz"),
                            y=y.contiguous().view(torch.int16).numpy().view(np.uint16),
                            N=N, K=K, M=M, seed=seed, e8m0=int(e8m0), digest=digest_of(w, s, x))
        print(name, "N", N, "K", K, "tokens", M)


if __name__ == "__main__":
    main()
