"""Build recipe for the checker side of the repository (TEST INFRASTRUCTURE).

Two outputs, both git-ignored and both carried to the GPU box with the tree:

* ``oracle/_build/liboracle.so`` -- the CPU restatement in ``oracle.cpp``
  (g++, OpenMP).  Always built.
* ``oracle/_ref/*.so`` -- the reference's own sources compiled where they lie
  under the reference checkout (never copied): its CPU loops (run anywhere),
  its CUDA kernels and its whole decode engine for sm_100a (run on the GPU box),
  and a CPU decode composed from its CPU loops.  Built only when the reference
  checkout is present; the GPU box uses the prebuilt files.

Flags follow the reference Makefile (Makefile:137: ``--use_fast_math -O3
-std=c++17``) with the architecture fixed to sm_100a.

Usage: ``python oracle/build_oracle.py [--reference DIR] [--force]``.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "_build")
REF_OUT = os.path.join(HERE, "_ref")
SHIMS = os.path.join(HERE, "ref_shims")
# The reference checkout: $GPT2B_REFERENCE_DIR, else a directory named "reference"
# beside this repository's root (absent on hosts that only run prebuilt files).
DEFAULT_REFERENCE = (os.environ.get("GPT2B_REFERENCE_DIR")
                     or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

# (output name, shim source, extra defines): the reference CPU loops.
CPU_SHIMS = [
    ("libref_cpu_gemv.so", "ref_cpu_gemv.cu", []),
    ("libref_cpu_attention.so", "ref_cpu_attention.cu", []),
    ("libref_cpu_fused.so", "ref_cpu_fused.cu", []),
    ("libref_cpu_gelu.so", "ref_cpu_gelu.cu", []),
    ("libref_cpu_encoder.so", "ref_cpu_encoder.cu", []),
]
# The reference CUDA kernels / engine, one library per precision flag set
# (Makefile:78-105).
GPU_SHIMS = [
    ("libref_ops_f32.so", "ref_gpu_ops.cu", ["-DENABLE_FP32"]),
    ("libref_ops_bf16.so", "ref_gpu_ops.cu", ["-DENABLE_BF16"]),
    ("libref_w8_int8.so", "ref_gpu_w8.cu", ["-DENABLE_BF16", "-DUSE_W8", "-DUSE_INT8", "-DUSE_KV_W8"]),
    ("libref_w8_fp8.so", "ref_gpu_w8.cu", ["-DENABLE_BF16", "-DUSE_W8", "-DUSE_FP8", "-DUSE_KV_W8"]),
    ("libref_quant.so", "ref_gpu_quant.cu", []),
    ("libref_engine_f32.so", "ref_gpu_engine.cu", ["-DENABLE_FP32"]),
    ("libref_engine_bf16.so", "ref_gpu_engine.cu", ["-DENABLE_BF16"]),
    ("libref_engine_int8.so", "ref_gpu_engine.cu", ["-DENABLE_BF16", "-DUSE_W8", "-DUSE_INT8"]),
    ("libref_engine_int8kv8.so", "ref_gpu_engine.cu", ["-DENABLE_BF16", "-DUSE_W8", "-DUSE_INT8", "-DUSE_KV_W8"]),
    ("libref_engine_fp8kv8.so", "ref_gpu_engine.cu", ["-DENABLE_BF16", "-DUSE_W8", "-DUSE_FP8", "-DUSE_KV_W8"]),
]


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        raise RuntimeError("build step failed:\n" + " ".join(cmd) + "\n" + proc.stdout[-4000:])


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build_oracle(force: bool = False) -> str:
    """Compile oracle.cpp into oracle/_build/liboracle.so and return its path."""
    os.makedirs(BUILD, exist_ok=True)
    out = os.path.join(BUILD, "liboracle.so")
    src = os.path.join(HERE, "oracle.cpp")
    if force or _stale(out, [src, os.path.join(HERE, "oracle.h"), __file__]):
        _run(["g++", "-O2", "-std=c++17", "-fopenmp", "-fPIC", "-shared", f"-I{CUDA_HOME}/include",
              src, "-o", out])
    return out


def _nvcc_shim(reference: str, name: str, src: str, defs: list[str]) -> str:
    out = os.path.join(REF_OUT, name)
    cmd = [NVCC, *ARCH, "-O3", "--use_fast_math", "-std=c++17", "-shared",
           "-Xcompiler", "-fPIC,-fopenmp,-fvisibility=hidden", f"-I{reference}", f"-I{SHIMS}", *defs,
           os.path.join(SHIMS, src), "-o", out, "-lcublas", "-lcublasLt", "-lgomp"]
    _run(cmd)
    return out


def build_reference(reference: str = DEFAULT_REFERENCE, force: bool = False, jobs: int = 8,
                    gpu: bool = True) -> list[str]:
    """Compile the reference sources in place into oracle/_ref/.  Returns the
    list of libraries built (empty when the reference checkout is absent)."""
    if not os.path.isdir(reference):
        return []
    os.makedirs(REF_OUT, exist_ok=True)
    todo = list(CPU_SHIMS) + (list(GPU_SHIMS) if gpu else [])
    work = [(n, s, d) for (n, s, d) in todo
            if force or _stale(os.path.join(REF_OUT, n), [os.path.join(SHIMS, s), os.path.join(SHIMS, "ref_api.h"), os.path.join(SHIMS, "fp8_compat.h")])]
    built = []
    with cf.ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        futs = {ex.submit(_nvcc_shim, reference, n, s, d): n for (n, s, d) in work}
        for f in cf.as_completed(futs):
            built.append(f.result())
    # the composed CPU decode links the CPU-loop shims
    out = os.path.join(REF_OUT, "libref_cpu_decode.so")
    src = os.path.join(SHIMS, "ref_cpu_decode.cpp")
    if force or _stale(out, [src] + [os.path.join(REF_OUT, n) for (n, _, _) in CPU_SHIMS]):
        libs = [f"-l:{n}" for (n, _, _) in CPU_SHIMS]
        _run(["g++", "-O3", "-std=c++17", "-fopenmp", "-fPIC", "-shared", "-fvisibility=hidden", src,
              f"-L{REF_OUT}", *libs, "-Wl,-rpath,$ORIGIN", "-o", out])
        built.append(out)
    return built


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=DEFAULT_REFERENCE)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--cpu-only", action="store_true", help="skip the reference CUDA libraries")
    ap.add_argument("--jobs", type=int, default=os.cpu_count() or 4)
    a = ap.parse_args()
    print(build_oracle(a.force))
    for p in build_reference(a.reference, a.force, a.jobs, gpu=not a.cpu_only):
        print(p)
    return 0


if __name__ == "__main__":
    sys.exit(main())
