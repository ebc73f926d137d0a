"""The paged index form on a B200: vLLM's request-local top-k positions,
converted to slots inside the kernel (glm53_sparse_mla.sparse_fwd_paged),
and the vLLM backend's forward_mqa built on it.

* The oracle's restatement of vLLM's index converter is pinned against the
  converter itself (vLLM 0.22.0, triton_convert_req_index_to_global_index).
* The fused op must give bit-identical output and LSE to the plain op fed
  the converted slots: the kernel compacts the same valid slots in the same
  order, so the arithmetic is the same.
* forward_mqa (hand-built metadata, a stand-in layer) matches the oracle, and
  with decode context parallelism returns the natural-log LSE.
"""

from __future__ import annotations

import math
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from conftest import COS_TOL, REL_TOL, parity_metrics
from oracle import sparse_mla_oracle as O

pytestmark = pytest.mark.gpu

import glm53_sparse_mla as G  # noqa: E402
from glm53_sparse_mla import workloads as W  # noqa: E402

BLOCK = 64


def _paged_batch(T, heads, topk, width, n_req, ctx, n_blocks, kv_dtype="bf16", seed=0):
    """A decode-like batch in vLLM's form: per-request block tables over a
    shared pool, request-local positions (some -1, some past the request's
    table) in a buffer wider than topk whose extra columns hold garbage."""
    rng = np.random.default_rng(seed)
    max_blocks = ctx // BLOCK
    bt = np.stack([rng.choice(n_blocks, max_blocks, replace=False) for _ in range(n_req)]).astype(np.int32)
    req = rng.integers(0, n_req, T).astype(np.int32)
    pos = np.full((T, width), 7777, np.int32)            # garbage past topk
    for t in range(T):
        pos[t, :topk] = rng.choice(ctx, topk, replace=False)
    pos[:, :topk][rng.random((T, topk)) < 0.05] = -1
    pos[:, :topk][rng.random((T, topk)) < 0.01] = ctx + 5   # block past the table: masked
    dev = torch.device("cuda")
    q = W.bf16_tensor_from_f32(rng.standard_normal((T, heads, 512), dtype=np.float32), dev)
    kv = W.device_pool(n_blocks * BLOCK, seed, dev, kv_dtype, 0.05)
    return (q, kv, torch.from_numpy(pos).to(dev), torch.from_numpy(req).to(dev),
            torch.from_numpy(bt).to(dev))


def test_converter_restatement_matches_vllm():
    conv = pytest.importorskip("vllm.v1.attention.backends.mla.sparse_utils")
    q, kv, pos, req, bt = _paged_batch(T=40, heads=16, topk=256, width=256, n_req=7, ctx=2048,
                                       n_blocks=512, seed=3)
    got = conv.triton_convert_req_index_to_global_index(req, bt, pos, BLOCK_SIZE=BLOCK,
                                                        NUM_TOPK_TOKENS=256)
    want = O.convert_req_index_to_global(req.cpu().numpy(), bt.cpu().numpy(), pos.cpu().numpy(),
                                         BLOCK)
    assert np.array_equal(got.cpu().numpy(), want)


@pytest.mark.parametrize("kv_dtype", ["bf16", "fp8"])
@pytest.mark.parametrize("heads,T", [(64, 32), (32, 40), (16, 64), (8, 8), (64, 160)])
def test_fused_equals_unfused(heads, T, kv_dtype):
    topk, width = 2048, 2176
    q, kv, pos, req, bt = _paged_batch(T, heads, topk, width, n_req=max(1, T // 4), ctx=8192,
                                       n_blocks=4096, kv_dtype=kv_dtype, seed=heads + T)
    scale = 0.05 if kv_dtype == "fp8" else 1.0
    slots = torch.from_numpy(O.convert_req_index_to_global(
        req.cpu().numpy(), bt.cpu().numpy(), pos[:, :topk].cpu().numpy(), BLOCK)).cuda()
    ref_out, ref_lse = G.sparse_fwd_with_lse(q, kv, slots, 512 ** -0.5, scale)
    lse = torch.empty(T, heads, device="cuda")
    out = G.sparse_fwd_paged(q, kv, pos, req, bt, BLOCK, 512 ** -0.5, scale, topk=topk, lse=lse)
    torch.cuda.synchronize()
    assert torch.equal(out, ref_out)
    assert torch.equal(lse, ref_lse)


def test_fused_matches_oracle():
    q, kv, pos, req, bt = _paged_batch(T=8, heads=32, topk=512, width=640, n_req=3, ctx=4096,
                                       n_blocks=1024, seed=11)
    out = G.sparse_fwd_paged(q, kv, pos, req, bt, BLOCK, 512 ** -0.5, topk=512)
    torch.cuda.synchronize()
    slots = O.convert_req_index_to_global(req.cpu().numpy(), bt.cpu().numpy(),
                                          pos[:, :512].cpu().numpy(), BLOCK)
    uniq, inv = np.unique(np.maximum(slots, 0), return_inverse=True)
    local = np.where(slots >= 0, inv.reshape(slots.shape), -1)
    ref, _, _ = O.sparse_mla_stats(q.float().cpu().numpy(), kv[torch.from_numpy(uniq).cuda()].float().cpu().numpy(),
                                   local, 512 ** -0.5)
    rel, cmin, finite = parity_metrics(out.float().cpu().numpy(), ref)
    assert finite and rel <= REL_TOL and cmin >= COS_TOL, (rel, cmin)


def _backend_impl(heads, buf):
    B = pytest.importorskip("glm53_sparse_mla.backend")
    return B.Glm53SparseMLAImpl(
        num_heads=heads, head_size=512, scale=512 ** -0.5, num_kv_heads=1, alibi_slopes=None,
        sliding_window=None, kv_cache_dtype="auto", logits_soft_cap=None, attn_type="decoder",
        kv_sharing_target_layer_name=None, topk_indices_buffer=buf, kv_lora_rank=512)


@pytest.mark.parametrize("dcp", [1, 2])
def test_backend_forward_mqa(dcp):
    heads, T, topk = 32, 12, 2048
    q, kv, pos, req, bt = _paged_batch(T, heads, topk, 2176, n_req=3, ctx=8192, n_blocks=2048,
                                       seed=5 + dcp)
    impl = _backend_impl(heads, pos)
    impl.dcp_world_size = dcp
    meta = SimpleNamespace(topk_tokens=topk, block_size=BLOCK, req_id_per_token=req,
                           block_table=bt)
    cache = kv.view(-1, BLOCK, 512)                       # vLLM's [blocks, 64, 512] cache
    out, lse = impl.forward_mqa(q, cache, meta, SimpleNamespace())
    torch.cuda.synchronize()
    slots = torch.from_numpy(O.convert_req_index_to_global(
        req.cpu().numpy(), bt.cpu().numpy(), pos[:, :topk].cpu().numpy(), BLOCK)).cuda()
    ref_out, ref_lse = G.sparse_fwd_with_lse(q, kv, slots, 512 ** -0.5)
    assert torch.equal(out, ref_out)
    if dcp == 1:
        assert lse is None
    else:
        fin = torch.isfinite(ref_lse)
        assert torch.equal(torch.isfinite(lse), fin)
        assert torch.allclose(lse[fin], ref_lse[fin] * math.log(2.0), rtol=1e-6, atol=1e-6)
