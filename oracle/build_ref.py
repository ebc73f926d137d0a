"""Compile the reference's own CUDA op from its source, for sm_100a, into
oracle/_ref/ -- TEST/BENCH INFRASTRUCTURE ONLY (a comparator, never shipped).

The reference kernel (csrc/sparse_mla.cu of jsmcconn/vllm-sparse-mla-blackwell)
is a single source file over libtorch; its own JIT helper builds it for the
current device (glm53_sparse_mla/build.py:27-41), so on a B200 it becomes an
sm_100a mma.sync kernel. This recipe does the same build ahead of time with
nvcc, reading the file where it lies (nothing is copied into this repository).
The library registers torch.ops.glm53_sparse_mla.sparse_fwd exactly like this
repository's op, so it must be loaded in a separate process
(oracle/ref_gpu_bench.py). Output: oracle/_ref/ref_sparse_mla_sm100.so.
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
OUT = os.path.join(OUT_DIR, "ref_sparse_mla_sm100.so")


def build_reference(ref_root: str = "/root/reference", force: bool = False) -> str | None:
    src = os.path.join(ref_root, "csrc", "sparse_mla.cu")
    if not os.path.exists(src):
        return None
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= os.path.getmtime(src):
        return OUT
    import torch
    from torch.utils import cpp_extension

    os.makedirs(OUT_DIR, exist_ok=True)
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cmd = [os.path.join(cuda, "bin", "nvcc"), "-gencode", "arch=compute_100a,code=sm_100a",
           # the reference's own nvcc flags (setup.py:31-43), minus its gencode
           "-O3", "-std=c++17", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
           "-U__CUDA_NO_BFLOAT162_OPERATORS__", "--expt-relaxed-constexpr",
           "--expt-extended-lambda", "-lineinfo", "-DNDEBUG",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           "-Xcompiler", "-fPIC", "-shared"]
    for d in cpp_extension.include_paths():
        cmd += ["-I", d]
    cmd += [src, "-o", OUT + ".tmp"]
    for d in cpp_extension.library_paths():
        cmd += ["-L", d]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("building the reference kernel failed")
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build_reference(sys.argv[1] if len(sys.argv) > 1 else "/root/reference", force=True))
