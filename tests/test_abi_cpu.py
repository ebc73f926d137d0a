"""C ABI and torch-op host logic, without a GPU.

* libglm53_sparse_mla.so loads and exports every function include/*.h declares
* argument validation returns the documented status codes before any CUDA call
  (the reference host op's TORCH_CHECKs, csrc/sparse_mla.cu:457-470, 488-496)
* the torch op keeps the reference schema byte-for-byte and has fake kernels
"""

from __future__ import annotations

import ctypes
import glob
import os
import re

import pytest
import torch

from conftest import REPO

import glm53_sparse_mla as G  # noqa: E402

OK, E_RANK, E_DIM, E_HEADS, E_TOPK, E_DTYPE, E_ALIGN, E_SPLITS = range(8)


def _declared_functions():
    names = set()
    for h in glob.glob(os.path.join(REPO, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(glm53_\w+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    lib = ctypes.CDLL(G.library_path())
    lib.glm53_sparse_mla_check.argtypes = [ctypes.c_int64] * 6 + [ctypes.c_int, ctypes.c_int]
    lib.glm53_sparse_mla_auto_splits.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int]
    lib.glm53_sparse_mla_strerror.restype = ctypes.c_char_p
    lib.glm53_sparse_mla_fwd.argtypes = [
        ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
        ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_int,
        ctypes.c_void_p]
    return lib


def test_every_declared_symbol_is_exported(lib):
    names = _declared_functions()
    assert "glm53_sparse_mla_fwd" in names and len(names) >= 7
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/ but not exported"


def test_validation_codes(lib):
    chk = lib.glm53_sparse_mla_check
    assert chk(4, 64, 512, 4096, 512, 2048, 0, 0) == OK
    assert chk(4, 8, 512, 4096, 512, 2048, 1, 4) == OK
    assert chk(4, 12, 512, 4096, 512, 2048, 0, 0) == E_HEADS
    assert chk(4, 128, 512, 4096, 512, 2048, 0, 0) == E_HEADS
    assert chk(4, 64, 576, 4096, 576, 2048, 0, 0) == E_DIM
    assert chk(4, 64, 512, 4096, 512, 2040, 0, 0) == E_TOPK
    assert chk(4, 64, 512, 4096, 512, 32768, 0, 0) == E_TOPK
    assert chk(4, 64, 512, 4096, 512, 8192, 0, 2) == E_TOPK      # 4096 per CTA > 2048
    assert chk(4, 64, 512, 4096, 512, 2048, 2, 0) == E_DTYPE
    assert chk(4, 64, 512, 4096, 512, 2048, 0, 3) == E_SPLITS
    assert chk(-1, 64, 512, 4096, 512, 2048, 0, 0) == E_RANK


def test_fwd_rejects_before_touching_cuda(lib):
    f = lib.glm53_sparse_mla_fwd
    # invalid head count: error code, no CUDA call (there is no GPU here)
    assert f(None, None, None, None, None, 4, 12, 512, 64, 512, 64, 0, 0.1, 1.0, 0, None) == E_HEADS
    # T == 0 is a no-op, as in the reference (csrc/sparse_mla.cu:472)
    assert f(None, None, None, None, None, 0, 64, 512, 64, 512, 64, 0, 0.1, 1.0, 0, None) == OK
    # null / misaligned pointers
    assert f(None, None, None, None, None, 4, 64, 512, 64, 512, 64, 0, 0.1, 1.0, 0, None) == E_ALIGN
    assert f(16, 32, 48, 65, None, 4, 64, 512, 64, 512, 64, 0, 0.1, 1.0, 0, None) == E_ALIGN
    for code in range(12):
        assert lib.glm53_sparse_mla_strerror(code)


def test_workspace_entry_points_validate_before_cuda(lib):
    import ctypes
    nb = ctypes.c_uint64(7)
    wsb = lib.glm53_sparse_mla_workspace_bytes
    wsb.argtypes = [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                    ctypes.POINTER(ctypes.c_uint64)]
    assert wsb(4, 12, 2048, 0, ctypes.byref(nb)) == E_HEADS
    assert wsb(0, 64, 2048, 0, ctypes.byref(nb)) == OK and nb.value == 0
    f = lib.glm53_sparse_mla_fwd_ws
    f.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int64] * 6 + [
        ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_void_p,
        ctypes.c_uint64, ctypes.c_void_p]
    assert f(None, None, None, None, None, 4, 12, 512, 64, 512, 64, 0, 0.1, 1.0, 0, None, 0,
             None) == E_HEADS
    assert f(None, None, None, None, None, 0, 64, 512, 64, 512, 64, 0, 0.1, 1.0, 0, None, 0,
             None) == OK


def test_auto_splits(lib):
    s = lib.glm53_sparse_mla_auto_splits
    assert s(32, 2048, 148) == 4      # C2 decode: 128 CTAs in one wave
    assert s(64, 2048, 148) == 2      # C4
    assert s(512, 2048, 148) == 1     # C5
    assert s(4127, 2048, 148) == 1    # C3
    assert s(1, 2048, 148) == 8
    assert s(1, 128, 148) == 1        # short lists are not split
    assert s(4096, 16384, 148) == 8   # 2048 indices per CTA at most


def test_op_schema_is_the_reference_schema():
    want = ("glm53_sparse_mla::sparse_fwd(Tensor q, Tensor kv, Tensor indices, float sm_scale, "
            "float kv_scale, Tensor(a!) out) -> ()")
    assert str(torch.ops.glm53_sparse_mla.sparse_fwd.default._schema) == want
    lse = str(torch.ops.glm53_sparse_mla.sparse_fwd_lse.default._schema)
    assert "Tensor(a!) out, Tensor(b!) lse" in lse


def test_constants():
    assert G.KV_LORA_RANK == 512
    assert G.SUPPORTED_HEADS_PER_RANK == (8, 16, 32, 64)


def test_cpu_tensors_have_no_kernel():
    q = torch.zeros(2, 16, 512, dtype=torch.bfloat16)
    kv = torch.zeros(64, 512, dtype=torch.bfloat16)
    idx = torch.zeros(2, 64, dtype=torch.int32)
    with pytest.raises(NotImplementedError):
        G.sparse_fwd(q, kv, idx, 0.1)


def test_fake_kernels_trace():
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        q = torch.empty(4, 64, 512, dtype=torch.bfloat16, device="cuda")
        kv = torch.empty(1024, 512, dtype=torch.bfloat16, device="cuda")
        idx = torch.empty(4, 2048, dtype=torch.int32, device="cuda")
        out = G.sparse_fwd(q, kv, idx, 0.04)
        assert out.shape == q.shape
        o2, lse = G.sparse_fwd_with_lse(q, kv, idx, 0.04)
        assert lse.shape == (4, 64) and lse.dtype == torch.float32


PAGED_ARGS = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
              ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
              ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p] + [ctypes.c_int64] * 6 + [
              ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_void_p,
              ctypes.c_uint64, ctypes.c_void_p]


def test_paged_entry_validates_before_cuda(lib):
    f = lib.glm53_sparse_mla_fwd_paged
    f.argtypes = PAGED_ARGS

    def call(T=4, H=64, topk=64, row_stride=64, bt_stride=8, max_blocks=8, bs=64, bstride=64,
             kv_rows=4096):
        return f(None, None, None, row_stride, None, None, bt_stride, max_blocks, bs, bstride,
                 None, None, T, H, 512, kv_rows, 512, topk, 0, 0.1, 1.0, 0, None, 0, None)

    assert call(H=12) == E_HEADS
    assert call(row_stride=32) == E_RANK          # positions rows narrower than topk
    assert call(bt_stride=4) == E_RANK            # block-table rows narrower than max_blocks
    assert call(bs=0) == E_RANK
    assert call(bstride=32) == E_RANK             # blocks closer than a block apart
    assert call(kv_rows=1 << 31) == E_RANK        # slots must fit int32
    assert call(T=0) == OK                        # nothing to do
    assert call() == E_ALIGN                      # null pointers, still no CUDA call


GATHER_ARGS = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
               ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p] + [ctypes.c_int64] * 6 + [
               ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_void_p,
               ctypes.c_uint64, ctypes.c_void_p]


def test_heads_gather_entry_validates_before_cuda(lib):
    """The fused head gather refuses a bad output set before any CUDA call
    (fake, aligned, never dereferenced addresses stand in for device ones)."""
    f = lib.glm53_sparse_mla_fwd_heads_gather
    f.argtypes = GATHER_ARGS
    f.restype = ctypes.c_int
    fake = 0x10000

    def call(n_outs=2, head_offset=0, heads_total=64, H=32, ptrs=(fake, fake + 4096)):
        arr = (ctypes.c_void_p * 8)(*ptrs)
        return f(fake, fake, fake, arr, n_outs, head_offset, heads_total, None, 4, H, 512, 4096,
                 512, 64, 0, 0.1, 1.0, 0, None, 0, None)

    assert call(n_outs=0) == 1                        # GLM53_ERR_RANK
    assert call(n_outs=9) == 1
    assert call(head_offset=40) == 1                  # 40 + 32 heads > 64
    assert call(heads_total=16, H=32) == 1
    assert call(ptrs=(fake, 0)) == 6                  # null output: GLM53_ERR_ALIGN
    assert call(ptrs=(fake, fake + 8)) == 6           # misaligned output
    assert call(H=12) == 3                            # heads per launch not served


def test_fake_gather_heads_traces():
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        q = torch.empty(4, 16, 512, dtype=torch.bfloat16, device="cuda")
        kv = torch.empty(1024, 512, dtype=torch.bfloat16, device="cuda")
        idx = torch.empty(4, 2048, dtype=torch.int32, device="cuda")
        out = torch.empty(4, 64, 512, dtype=torch.bfloat16, device="cuda")
        torch.ops.glm53_sparse_mla.sparse_fwd_gather_heads(q, kv, idx, 0.04, 1.0, [1024], 0, 16,
                                                           out)
