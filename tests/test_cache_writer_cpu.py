"""The latent KV-cache writer without a GPU.

* the oracle's float -> e4m3 encoder: every finite code round-trips, exact
  midpoints round to the even code, |x| > 448 and +-inf saturate, the sign of
  zero is kept; and it agrees with torch's own float8_e4m3fn cast in range;
* the oracle against vLLM's own concat_and_cache_mla, through the golden
  vectors tests/golden/make_cache_golden.py recorded on a GPU;
* glm53_concat_and_cache validates its arguments before any CUDA call;
* the torch op carries vLLM's concat_and_cache_mla schema and a fake kernel.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest
import torch

from conftest import REPO
from oracle import cache_writer_oracle as CW
from oracle import sparse_mla_oracle as O

import glm53_sparse_mla as G  # noqa: E402

GOLDEN = os.path.join(REPO, "tests", "golden", "cache_writer_golden.npz")
OK, E_RANK, E_DTYPE, E_ALIGN = 0, 1, 5, 6


def test_e4m3_codes_round_trip():
    codes = np.arange(256, dtype=np.uint8)
    finite = (codes & 0x7F) != 0x7F
    vals = O.e4m3_to_f32(codes)
    assert np.array_equal(CW.f32_to_e4m3_satfinite(vals[finite]), codes[finite])
    assert np.all(CW.f32_to_e4m3_satfinite(np.array([np.nan], np.float32)) == 0x7F)


def test_e4m3_ties_saturation_and_zero():
    pos = O.e4m3_to_f32(np.arange(0x7F, dtype=np.uint8)).astype(np.float64)
    mids = ((pos[:-1] + pos[1:]) / 2).astype(np.float32)
    got = CW.f32_to_e4m3_satfinite(mids).astype(int)
    lo = np.arange(0x7E)
    assert np.array_equal(got, np.where(lo % 2 == 0, lo, lo + 1))      # ties to even
    sat = CW.f32_to_e4m3_satfinite(np.array([448, 449, 464, 480, 1e30, np.inf], np.float32))
    assert np.all(sat == 0x7E)
    assert np.all(CW.f32_to_e4m3_satfinite(-np.array([500, np.inf], np.float32)) == 0xFE)
    assert list(CW.f32_to_e4m3_satfinite(np.array([0.0, -0.0, 1e-30, -1e-30], np.float32))) == \
        [0x00, 0x80, 0x00, 0x80]


def test_e4m3_agrees_with_torch_cast_in_range():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(50000) * s for s in (1e-3, 0.1, 1, 30, 200)])
    x = x[np.abs(x) <= 448].astype(np.float32)
    want = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(CW.f32_to_e4m3_satfinite(x), want)


def test_oracle_matches_vllm_golden():
    """Byte-exact against vLLM's compiled concat_and_cache_mla, run on a B200
    by tests/golden/make_cache_golden.py."""
    g = np.load(GOLDEN)
    kv_c, slots = g["kv_c"], g["slots"]
    assert kv_c.shape[0] > slots.shape[0] and (slots < 0).any()
    got = CW.concat_and_cache_mla(kv_c, g["init_bf16"], slots, "auto")
    assert np.array_equal(got, g["out_auto"])
    for k, s in enumerate(g["scales"]):
        got = CW.concat_and_cache_mla(kv_c, g["init_fp8"], slots, "fp8", float(s))
        assert np.array_equal(got, g[f"out_fp8_{k}"]), f"scale {s}"
    # the tie and saturation rows took part
    assert slots[0] >= 0 and slots[1] >= 0


def test_oracle_rejects_other_cache_dtypes():
    with pytest.raises(ValueError):
        CW.concat_and_cache_mla(np.zeros((1, 512), np.uint16), np.zeros((1, 4, 512), np.uint8),
                                np.zeros(1, np.int64), "fp8_e5m2")


@pytest.fixture(scope="module")
def lib():
    lib = ctypes.CDLL(G.library_path())
    lib.glm53_concat_and_cache.argtypes = [
        ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int,
        ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
        ctypes.c_void_p, ctypes.c_void_p]
    return lib


def test_c_abi_validates_before_cuda(lib):
    f = lib.glm53_concat_and_cache
    A, S = 0x10000, 0x20000                     # aligned dummies; never dereferenced
    # (kv_c, kv_c_stride, T, cache, dtype, num_blocks, block_size, block_stride,
    #  entry_stride, slots, scale, stream)
    assert f(A, 512, 0, A, 1, 4, 64, 64 * 512, 512, S, A, None) == OK        # T == 0
    assert f(A, 512, -1, A, 1, 4, 64, 64 * 512, 512, S, A, None) == E_RANK
    assert f(A, 500, 4, A, 1, 4, 64, 64 * 512, 512, S, A, None) == E_RANK   # row stride < 512
    assert f(A, 512, 4, A, 1, 4, 0, 0, 512, S, A, None) == E_RANK           # block_size 0
    assert f(A, 512, 4, A, 1, 4, 64, 63 * 512, 512, S, A, None) == E_RANK   # overlapping pages
    assert f(A, 512, 4, A, 2, 4, 64, 64 * 512, 512, S, A, None) == E_DTYPE
    assert f(A, 512, 4, None, 1, 4, 64, 64 * 512, 512, S, A, None) == E_ALIGN
    assert f(A, 512, 4, A, 1, 4, 64, 64 * 512, 512, S, None, None) == E_ALIGN   # fp8 needs scale
    assert f(A + 8, 512, 4, A, 1, 4, 64, 64 * 512, 512, S, A, None) == E_ALIGN
    assert f(A, 516, 4, A, 0, 4, 64, 64 * 516, 516, S, A, None) == E_ALIGN    # bf16 stride 1032 B


def test_op_schema_and_fake():
    schema = str(torch.ops.glm53_sparse_mla.concat_and_cache_mla.default._schema)
    assert schema == ("glm53_sparse_mla::concat_and_cache_mla(Tensor kv_c, Tensor k_pe, "
                      "Tensor(a!) kv_cache, Tensor slot_mapping, str kv_cache_dtype, "
                      "Tensor scale) -> ()")
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        kv_c = torch.empty((4, 512), dtype=torch.bfloat16)
        cache = torch.empty((2, 16, 512), dtype=torch.uint8)
        torch.ops.glm53_sparse_mla.concat_and_cache_mla(
            kv_c, kv_c[:, :0], cache, torch.empty(4, dtype=torch.int64), "fp8", torch.ones(1))
