"""Build the sm_100a shared library ``flyai_b200/_lib/libflyai_moe.so`` with nvcc.

Run ``python -m flyai_b200.build`` (or ``__graft_entry__.build()``).  The build
is in-tree so the library travels with the repository snapshot; nvcc
cross-compiles without a GPU.
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_lib")
LIB = os.path.join(OUT_DIR, "libflyai_moe.so")
SOURCES = ["abi.cu", "route.cu", "combine.cu", "tc_experts.cu", "tc_prefill.cu", "fp8_moe.cu", "nv4_moe.cu", "nv4_prefill.cu", "v4_moe.cu",
           "fp8_linear.cu",
           "noalloc.cu"]
HEADERS = ["act_quant.cuh", "common.cuh", "route.cuh", "route_dev.cuh", "torch_topk.cuh", "tcgen05.cuh", "terms.cuh", "tc_bank.cuh", "fp8_moe.cuh", "nv4.cuh", "v4.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path():
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else (shutil.which("nvcc") or cand)


def _stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(HERE, "..", "include", "flyai_moe.h"))
    deps.append(os.path.abspath(__file__))
    return any(os.path.getmtime(p) > t for p in deps if os.path.exists(p))


def build(force=False, verbose=False):
    if not force and not _stale():
        return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    tmp = LIB + ".tmp"
    cmd = [nvcc_path(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "--shared",
           "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
           "-Xptxas", "-v" if verbose else "-O3",
           "-I", os.path.join(HERE, "..", "include"),
           "-o", tmp] + [os.path.join(CSRC, f) for f in SOURCES] + ["-cudart", "static"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libflyai_moe.so")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
