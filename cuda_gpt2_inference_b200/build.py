"""Build recipe for the CUDA library (in-tree, sm_100a).

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` (``-gencode
arch=compute_100a,code=sm_100a -lineinfo -O3 --use_fast_math``) into
``cuda_gpt2_inference_b200/libgpt2b.so``.  ``--use_fast_math`` matches the
reference build (Makefile:137) so fast-math divisions in the quantisers give
the reference's bytes.  Objects go to ``cuda_gpt2_inference_b200/_build/``.

Usage: ``python -m cuda_gpt2_inference_b200.build [--force] [--verbose] [--trace]``.
``--trace`` builds ``libgpt2b_trace.so`` instead (objects in ``_build_trace/``): the
persistent kernel stamps ``%globaltimer`` at its phase boundaries
(``GPT2B_PERSIST_TRACE``; ``bench.py --profile-case trace`` reads them).  Load it with
``GPT2B_LIB=<path>``.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libgpt2b.so")
OBJ_TRACE = os.path.join(HERE, "_build_trace")
LIB_TRACE = os.path.join(HERE, "libgpt2b_trace.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "--use_fast_math", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=default",
              f"-I{INCLUDE}", f"-I{CSRC}"]


def _nccl_paths():
    """Include and library directories of the NCCL shipped with torch's wheels."""
    try:
        import nvidia.nccl  # type: ignore
        base = os.path.dirname(nvidia.nccl.__file__) if nvidia.nccl.__file__ else list(nvidia.nccl.__path__)[0]
    except Exception:  # pragma: no cover - probed at build time
        return None, None
    inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
    if os.path.exists(os.path.join(inc, "nccl.h")) and os.path.exists(os.path.join(lib, "libnccl.so.2")):
        return inc, lib
    return None, None


def _run(cmd, verbose=False):
    if verbose:
        print(" ".join(cmd))
    p = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if p.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + p.stdout[-6000:])
    return p.stdout


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def build(force: bool = False, verbose: bool = False, jobs: int | None = None, ptxas_info: bool = False,
          trace: bool = False) -> str:
    """Compile csrc/*.cu into libgpt2b.so (or the trace build) incrementally and return its path."""
    obj_dir, lib = (OBJ_TRACE, LIB_TRACE) if trace else (OBJ, LIB)
    os.makedirs(obj_dir, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdr_t = max((os.path.getmtime(h) for h in _headers()), default=0.0)
    nccl_inc, nccl_lib = _nccl_paths()
    extra = [f"-I{nccl_inc}", "-DGPT2B_HAVE_NCCL=1"] if nccl_inc else []
    if trace:
        extra.append("-DGPT2B_PERSIST_TRACE=1")
    objs, work = [], []
    for s in srcs:
        o = os.path.join(obj_dir, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr_t,
                                                                         os.path.getmtime(__file__)):
            cmd = [NVCC, *ARCH, *NVCC_FLAGS, *extra, "-c", s, "-o", o]
            if ptxas_info:
                cmd.insert(1, "-Xptxas=-v")
            work.append(cmd)
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        outs = list(ex.map(lambda c: _run(c, verbose), work))
    if ptxas_info:
        for o in outs:
            print(o)
    if work or force or not os.path.exists(lib):
        link = [NVCC, *ARCH, "-shared", "-o", lib, *objs, "-lcudart"]
        if nccl_lib:
            link += [f"-L{nccl_lib}", "-l:libnccl.so.2", f"-Xlinker=-rpath,{nccl_lib}"]
        _run(link, verbose)
    return lib


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v register/spill/smem usage")
    ap.add_argument("--trace", action="store_true", help="build libgpt2b_trace.so (persistent-kernel phase stamps)")
    a = ap.parse_args()
    print(build(a.force, a.verbose, ptxas_info=a.ptxas_info, trace=a.trace))
    return 0


if __name__ == "__main__":
    sys.exit(main())
