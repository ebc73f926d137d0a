"""Pin the CPU oracle against vectors made by the reference's own fp32 ground
truth (tests/reference.py of the reference), see tests/golden/make_golden.py."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from golden.make_golden import golden_cases, input_digest
from oracle import sparse_mla_oracle as O

CASES = golden_cases()


@pytest.mark.parametrize("case", CASES, ids=[c.name for c in CASES])
def test_oracle_matches_reference(case, golden):
    key = case.name
    assert np.array_equal(input_digest(case), golden[f"{key}/input_sha256"]), \
        "input generator drifted from the one the golden vectors were made with"
    q = case.q.float().numpy()
    kv = case.kv.float().numpy()
    out, lse = O.sparse_mla_fp32(q, kv, case.indices.numpy(), case.sm_scale)
    ref_out = golden[f"{key}/out"]
    ref_lse = golden[f"{key}/lse"]
    # Summation order differs from torch.einsum; with q x 100 the scores reach
    # ~1e3 and exp() amplifies last-bit differences, hence a scale-relative atol.
    np.testing.assert_allclose(out, ref_out, rtol=1e-4, atol=1e-5 * max(np.abs(ref_out).max(), 1))
    assert np.array_equal(np.isneginf(lse), np.isneginf(ref_lse))
    fin = np.isfinite(ref_lse)
    np.testing.assert_allclose(lse[fin], ref_lse[fin], rtol=1e-5, atol=1e-5)
    # fully masked tokens: exact zeros
    dead = (case.indices.numpy() < 0).all(axis=1)
    assert (out[dead] == 0).all()


def test_lse_log2_is_log_sum_exp():
    rng = np.random.default_rng(0)
    q = O.bf16_round(rng.standard_normal((3, 4, 512)).astype(np.float32))
    kv = O.bf16_round(rng.standard_normal((256, 512)).astype(np.float32))
    idx = rng.integers(-1, 256, size=(3, 64)).astype(np.int32)
    idx[1] = -1
    sm = 512 ** -0.5
    _, m, s = O.sparse_mla_stats(q, kv, idx, sm)
    lse = O.lse_log2(m, s)
    for t in range(3):
        for h in range(4):
            v = idx[t] >= 0
            if not v.any():
                assert np.isneginf(lse[t, h])
                continue
            sc = (kv[idx[t][v]].astype(np.float64) @ q[t, h].astype(np.float64)) * sm
            want = np.log2(np.exp(sc - sc.max()).sum()) + sc.max() / np.log(2)
            assert abs(lse[t, h] - want) < 1e-4
    # the reference's formula agrees with the log-sum-exp only at sm_scale == 1
    _, m1, s1 = O.sparse_mla_stats(q, kv, idx, 1.0)
    fin = s1 > 0
    np.testing.assert_allclose(O.lse_reference(m1, s1, 1.0)[fin], O.lse_log2(m1, s1)[fin],
                               rtol=1e-6, atol=1e-5)


def test_fp8_dequant_helper_matches_torch():
    x = torch.randn(4096) * 20
    q8 = x.clamp(-448, 448).to(torch.float8_e4m3fn)
    want = (q8.float() * 0.05).to(torch.bfloat16).float().numpy()
    got = O.dequant_fp8(q8.view(torch.uint8).numpy(), 0.05)
    assert np.array_equal(got, want)


def test_bf16_rounding_matches_torch():
    x = (torch.randn(10000) * 3).float()
    assert np.array_equal(O.bf16_round(x.numpy()), x.to(torch.bfloat16).float().numpy())


def test_converter_restatement_known_answers():
    """Request-local positions -> slots, hand-checked: position p of request r
    is block_table[r][p // 64] * 64 + p % 64, -1 for p < 0 or a block past
    the table (vLLM 0.22.0 sparse_utils.py:11-84 semantics)."""
    bt = np.array([[5, 2, 7], [1, 0, 3]], np.int32)
    req = np.array([1, 0], np.int32)
    ti = np.array([[0, 63, 64, 130, -1, 192], [0, 65, 191, 192, -5, 1]], np.int32)
    want = np.array([[64, 127, 0, 194, -1, -1], [320, 129, 511, -1, -1, 321]], np.int32)
    assert np.array_equal(O.convert_req_index_to_global(req, bt, ti, 64), want)
    # a non-contiguous page layout: consecutive blocks 100 rows apart
    got = O.convert_req_index_to_global(req, bt, ti, 64, block_stride_rows=100)
    assert got[0, 3] == 3 * 100 + 2 and got[1, 0] == 5 * 100
