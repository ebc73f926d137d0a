"""Bounded pipeline waits and the gather-roof probe, on a B200.

* A wait limit far below a launch's runtime makes the attention kernel's
  waits run out on purpose (no GPU fault: the waits give up by design). The
  launch must return, raise GLM53_DEV_TIMEOUT in the device status word, and
  leave the device usable: with the default limit restored, the next launch
  of every merge path matches the oracle, which also shows that the aborted
  CTAs released their tensor memory.
* glm53_gather_roof: the per-CTA checksum of the rows it gathered equals the
  host's, for one CTA per token and for a machine-wide cut of the index list.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from test_parity_gpu import _abi, _check, _oracle, abi_fwd

pytestmark = pytest.mark.gpu

import glm53_sparse_mla as G  # noqa: E402
from glm53_sparse_mla import workloads as W  # noqa: E402


def _lib():
    lib = ctypes.CDLL(G.library_path())
    lib.glm53_sparse_mla_set_wait_timeout_ns.restype = ctypes.c_int
    lib.glm53_sparse_mla_set_wait_timeout_ns.argtypes = [ctypes.c_uint64]
    lib.glm53_sparse_mla_device_status.restype = ctypes.c_int
    lib.glm53_sparse_mla_device_status.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int]
    lib.glm53_gather_roof.restype = ctypes.c_int
    lib.glm53_gather_roof.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                      ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                      ctypes.c_void_p, ctypes.c_void_p]
    return lib


def _status(lib) -> int:
    st = ctypes.c_uint32(0)
    assert lib.glm53_sparse_mla_device_status(ctypes.byref(st), 1) == 0
    return st.value


@pytest.mark.parametrize("path", ["torch_op_ws", "split1", "split2", "split4", "split8"])
def test_wait_timeout_raises_status_and_device_recovers(path):
    lib = _lib()
    abi = _abi()
    w = W.config_c2(device="cuda")
    splits = {"torch_op_ws": 0, "split1": 1, "split2": 2, "split4": 4, "split8": 8}[path]

    def run():
        if path == "torch_op_ws":
            return G.sparse_fwd(w.q, w.kv, w.indices, w.sm_scale)
        return abi_fwd(abi, w, splits)

    torch.cuda.synchronize()
    _status(lib)                                   # clear
    try:
        # 1 ns: every wait that is not already satisfied gives up at its first
        # timer check; a C2 launch has many such waits
        assert lib.glm53_sparse_mla_set_wait_timeout_ns(1) == 0
        run()
        torch.cuda.synchronize()
    finally:
        assert lib.glm53_sparse_mla_set_wait_timeout_ns(0) == 0
    assert _status(lib) & 1, "no wait gave up under a 1 ns limit"
    # default limit again: the same launch is correct and records no timeout
    ref, _ = _oracle(w)
    for _ in range(2):
        out = run()
        torch.cuda.synchronize()
        _check(f"c2/after-timeout/{path}", out, ref, w.indices)
    assert _status(lib) & 1 == 0


def _xor_rows(words: np.ndarray, idx: np.ndarray, R: int) -> int:
    ok = (idx >= 0) & (idx < R)
    x = np.uint32(0)
    for v in words[idx[ok]]:
        x ^= v
    return int(x)


@pytest.mark.parametrize("ctas", [0, 7, 148])
def test_gather_roof_checksum(ctas):
    lib = _lib()
    rng = np.random.default_rng(11)
    R, T, K = 4096, 5, 256
    kv = torch.randn(R, 512, device="cuda").to(torch.bfloat16)
    words = kv.view(torch.int16).cpu().numpy()[:, :2].copy().view(np.uint32)[:, 0]
    idx = rng.integers(0, R, size=(T, K)).astype(np.int32)
    idx[1, ::3] = -1
    idx[2, 5] = R + 9                      # out of range: skipped
    idx[4, :] = -1                         # a token with no row
    idx_d = torch.from_numpy(idx).cuda()
    total = T * K
    grid = T if ctas == 0 else min(ctas, total)
    per = -(-total // grid)
    sink = torch.full((grid,), -1, dtype=torch.int32, device="cuda")
    rc = lib.glm53_gather_roof(kv.data_ptr(), idx_d.data_ptr(), T, K, R, ctas, sink.data_ptr(),
                               torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    got = sink.cpu().numpy().view(np.uint32)
    flat = idx.reshape(-1)
    for c in range(grid):
        want = _xor_rows(words, flat[c * per:min(total, (c + 1) * per)], R)
        assert int(got[c]) == want, (c, int(got[c]), want)
