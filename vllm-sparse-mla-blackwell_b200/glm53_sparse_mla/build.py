"""In-tree build of the sm_100a extension.

Produces, next to this file:
  libglm53_sparse_mla.so  the CUDA kernels behind the plain C ABI
                          (include/glm53_sparse_mla.h); no torch dependency.
  _C.so                   the TORCH_LIBRARY registration of
                          torch.ops.glm53_sparse_mla.*, linked against the
                          library above through an $ORIGIN rpath.

Target is sm_100a only (B200 class), with -lineinfo and without
--use_fast_math: the softmax calls exp2f / log2f, never their fast variants.
The reference's JIT helper (glm53_sparse_mla/build.py:14-41) instead built for
the device it found; this build is explicit and cross-compiles without a GPU.
"""

from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
PROJECT_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PROJECT_DIR, "csrc")


def _find_include_dir() -> str:
    # repository layout: <repo>/include next to <repo>/vllm-sparse-mla-blackwell_b200
    cands = [os.path.join(PROJECT_DIR, "include"),
             os.path.join(os.path.dirname(PROJECT_DIR), "include")]
    for c in cands:
        if os.path.exists(os.path.join(c, "glm53_sparse_mla.h")):
            return c
    raise FileNotFoundError("glm53_sparse_mla.h not found in " + ", ".join(cands))


CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
              "-Xcompiler", "-fPIC", "-Xptxas", "--warn-on-spills"]

LIB_NAME = "libglm53_sparse_mla.so"
# attention kernel + host launcher; latent KV-cache writer; indexer scores and top-k
KERNEL_SOURCES = ["sparse_mla_sm100.cu", "kv_cache_writer_sm100.cu", "indexer_logits_sm100.cu",
                  "topk_sm100.cu"]
OP_NAME = "_C.so"


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"build step failed ({res.returncode}): {cmd[0]}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, flush=True)


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build_kernel_lib(force: bool = False, verbose: bool = False) -> str:
    inc = _find_include_dir()
    srcs = [os.path.join(CSRC, f) for f in KERNEL_SOURCES]
    deps = srcs + [os.path.join(CSRC, "sm100_ptx.cuh"), os.path.join(inc, "glm53_sparse_mla.h")]
    out = os.path.join(PKG_DIR, LIB_NAME)
    if force or _newer(out, deps):
        tmp = out + ".tmp"
        _run([NVCC, *GENCODE, *NVCC_FLAGS, "-I", inc, "-I", CSRC, "-shared", *srcs, "-o", tmp],
             verbose)
        os.replace(tmp, out)
    return out


def build_torch_op(force: bool = False, verbose: bool = False) -> str:
    import torch
    from torch.utils import cpp_extension

    inc = _find_include_dir()
    src = os.path.join(CSRC, "torch_binding.cpp")
    lib = os.path.join(PKG_DIR, LIB_NAME)
    out = os.path.join(PKG_DIR, OP_NAME)
    if not (force or _newer(out, [src, lib, os.path.join(inc, "glm53_sparse_mla.h")])):
        return out
    torch_inc = cpp_extension.include_paths()
    torch_lib = cpp_extension.library_paths()
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-I", inc, "-I", os.path.join(CUDA_HOME, "include"),
           "-I", sysconfig.get_paths()["include"]]
    for d in torch_inc:
        cmd += ["-I", d]
    cmd += [src, "-o", out + ".tmp", "-L", PKG_DIR, "-l:" + LIB_NAME]
    for d in torch_lib:
        cmd += ["-L", d]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
            "-Wl,-rpath,$ORIGIN"]
    _run(cmd, verbose)
    os.replace(out + ".tmp", out)
    return out


def build(force: bool = False, verbose: bool = False) -> list[str]:
    """Build both shared objects in place; returns their paths."""
    return [build_kernel_lib(force, verbose), build_torch_op(force, verbose)]


if __name__ == "__main__":
    for p in build(force="--force" in sys.argv, verbose=True):
        print(p)
