"""Build libsunshape_b200.so in-tree with nvcc for sm_100a.

    python -m sunshape_b200.build [--verbose]

The library is a plain C-ABI shared object (no torch headers), compiled with
``-gencode arch=compute_100a,code=sm_100a`` and the CUDA runtime linked
statically, so it loads in any process on a B200 host.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB_NAME = "libsunshape_b200.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)
SOURCES = ["capi.cu", "decode_f32.cu", "decode_bf16.cu", "decode_f16.cu", "decode_scores.cu", "decode_mma_bf16.cu",
           "decode_mma_f16.cu", "noalloc.cu", "peer.cu", "encode_tc.cu", "exchange.cu", "packed.cu"]
DEPS = SOURCES + ["common.cuh", "decode.cuh", "decode_mma.cuh", "encode.cuh", "encode_params.cuh"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the sunshape_b200 CUDA library cannot be built")


def is_stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    lib_m = os.path.getmtime(LIB_PATH)
    deps = [os.path.join(CSRC, d) for d in DEPS] + [os.path.join(ROOT, "include", "sunshape_b200.h")]
    return any(os.path.getmtime(d) > lib_m for d in deps if os.path.exists(d))


def build(verbose: bool = False, force: bool = False, out: str | None = None,
          defines: tuple[str, ...] = ()) -> str:
    """Compile the library (to ``out``, default in-tree) with optional -D defines."""
    lib_path = out or LIB_PATH
    if not force and not defines and out is None and not is_stale():
        return LIB_PATH
    from concurrent.futures import ThreadPoolExecutor

    obj_dir = os.path.join(ROOT, "_build", "-".join(defines) or "default")
    os.makedirs(obj_dir, exist_ok=True)
    common = [nvcc(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
              "-I", os.path.join(ROOT, "include"), *[f"-D{d}" for d in defines]]
    if verbose:
        common.append("-Xptxas=-v")

    def compile_one(src: str) -> str:
        obj = os.path.join(obj_dir, src.replace(".cu", ".o"))
        cmd = [*common, "-c", os.path.join(CSRC, src), "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        sys.stderr.write(r.stdout + r.stderr if verbose or r.returncode else "")
        if r.returncode:
            raise RuntimeError(f"nvcc failed on {src}")
        return obj

    with ThreadPoolExecutor(max_workers=min(len(SOURCES), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(compile_one, SOURCES))
    link = [nvcc(), *ARCH_FLAGS, "--shared", "-cudart", "static", *objs, "-o", lib_path + ".tmp"]
    subprocess.run(link, check=True)
    os.replace(lib_path + ".tmp", lib_path)
    return lib_path


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--out", default=None, help="output path (default: in-tree library)")
    ap.add_argument("--define", action="append", default=[], help="extra -D define (e.g. SUNSHAPE_TRACE)")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force, out=a.out, defines=tuple(a.define)))
