"""The indexer's paged fp8 MQA logits on a B200
(glm53_sparse_mla.fp8_paged_mqa_logits, C ABI glm53_indexer_logits).

* against the oracle (oracle/indexer_logits_oracle.py) on seeded inputs:
  H 32 and 64, next_n 1, 2 and 4, per-request and per-token lengths, block
  sizes 64 and 16, padded block strides, lengths from 1 to max_model_len
  (not a multiple of the 512-position chunk), with and without clean_logits
  (without it, positions a row does not see keep their old values);
  tolerance: the -inf pattern exactly, and per row
  max |got - want| <= 1e-3 * max |want| (fp32 sums of exact e4m3 products in
  another order);
* a block id past the cache reads nothing and raises the status bit;
* indexer -> top-k -> attention: logits to positions to sparse_fwd_paged.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import indexer_logits_oracle as IL
from oracle import topk_oracle as TK

pytestmark = pytest.mark.gpu

import glm53_sparse_mla as G  # noqa: E402

DEV = torch.device("cuda")


def _case(seed, B, next_n, H, bs, max_blocks, pad_bytes=0, scale_lo=0.25):
    rng = np.random.default_rng(seed)
    nb = B * max_blocks + 3
    q = torch.from_numpy(rng.standard_normal((B, next_n, H, 128)).astype(np.float32)) \
        .to(torch.float8_e4m3fn)
    vals = torch.from_numpy(rng.standard_normal((nb, bs * 128)).astype(np.float32)) \
        .to(torch.float8_e4m3fn).view(torch.uint8)
    sc = torch.from_numpy(rng.uniform(scale_lo, 2.0, (nb, bs)).astype(np.float32)).view(torch.uint8)
    pad = torch.zeros((nb, pad_bytes), dtype=torch.uint8)
    flat = torch.cat([vals, sc, pad], 1).contiguous()              # block stride bs*132 + pad
    w = torch.from_numpy(rng.standard_normal((B * next_n, H)).astype(np.float32))
    bt = torch.from_numpy(np.stack([rng.permutation(nb)[:max_blocks] for _ in range(B)])
                          .astype(np.int32))
    return rng, q, flat, w, bt


def _kv_view(flat, bs):
    """[num_blocks, block_size, 1, 132] view over blocks that may carry padding."""
    nb, stride = flat.shape
    return torch.as_strided(flat, (nb, bs, 1, 132), (stride, 132, 132, 1))


def _check(got, want):
    g, w = got.cpu().numpy(), want
    fin = np.isfinite(w)
    assert np.array_equal(fin, np.isfinite(g)), "visible-position pattern differs"
    for r in range(w.shape[0]):
        f = fin[r]
        if f.any():
            err = np.abs(g[r, f] - w[r, f]).max()
            assert err <= 1e-3 * max(np.abs(w[r, f]).max(), 1e-30), (r, err)


@pytest.mark.parametrize("H,next_n", [(64, 1), (32, 1), (64, 2), (32, 4), (64, 4)])
@pytest.mark.parametrize("bs,pad", [(64, 0), (16, 48)])
def test_matches_oracle(H, next_n, bs, pad):
    B, max_blocks = 6, 40
    max_len = max_blocks * bs - 5
    rng, q, flat, w, bt = _case(H * 10 + next_n + bs, B, next_n, H, bs, max_blocks, pad)
    ctx = rng.integers(next_n, max_len + 1, B).astype(np.int32)
    ctx[0] = next_n                 # the first token sees a single position
    ctx[1] = max_len
    logits = G.fp8_paged_mqa_logits(q.to(DEV), _kv_view(flat.to(DEV), bs), w.to(DEV),
                                    torch.from_numpy(ctx).to(DEV), bt.to(DEV), max_len)
    torch.cuda.synchronize()
    want = IL.paged_mqa_logits(q.view(torch.uint8).numpy(), flat.numpy()[:, :bs * 132],
                               w.numpy(), ctx, bt.numpy(), max_len)
    _check(logits, want)


def test_per_token_lengths_and_unclean():
    B, next_n, H, bs, max_blocks = 5, 2, 64, 64, 20
    max_len = max_blocks * bs
    rng, q, flat, w, bt = _case(99, B, next_n, H, bs, max_blocks)
    lens = np.sort(rng.integers(1, max_len, (B, next_n)), axis=1).astype(np.int32)
    out = torch.full((B * next_n, max_len + 7), 12345.0, device=DEV)
    G.fp8_paged_mqa_logits(q.to(DEV), _kv_view(flat.to(DEV), bs), w.to(DEV),
                           torch.from_numpy(lens).to(DEV), bt.to(DEV), max_len,
                           clean_logits=False, logits=out)
    torch.cuda.synchronize()
    o = out.cpu().numpy()
    L = lens.reshape(-1)
    for r in range(B * next_n):
        i, j = divmod(r, next_n)
        want = IL.paged_mqa_logits(q.view(torch.uint8).numpy()[i:i + 1, j:j + 1], flat.numpy(),
                                   w.numpy()[r:r + 1], np.array([L[r]]), bt.numpy()[i:i + 1],
                                   max_len)[0]
        seen = slice(0, L[r])
        assert np.abs(o[r, seen] - want[seen]).max() <= 1e-3 * np.abs(want[seen]).max()
        assert np.all(o[r, L[r]:] == 12345.0)      # unseen positions and padding untouched


def test_block_past_cache_is_skipped_and_reported():
    lib = ctypes.CDLL(G.library_path())
    lib.glm53_indexer_status.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int]
    st = ctypes.c_uint32(0)
    assert lib.glm53_indexer_status(ctypes.byref(st), 1) == 0
    B, H, bs, max_blocks = 2, 64, 64, 4
    rng, q, flat, w, bt = _case(5, B, 1, H, bs, max_blocks)
    bt[1, 2] = flat.shape[0] + 100                  # past the cache
    ctx = torch.tensor([4 * bs, 4 * bs], dtype=torch.int32)
    logits = G.fp8_paged_mqa_logits(q.to(DEV), _kv_view(flat.to(DEV), bs), w.to(DEV), ctx.to(DEV),
                                    bt.to(DEV), 4 * bs)
    torch.cuda.synchronize()
    assert lib.glm53_indexer_status(ctypes.byref(st), 1) == 0
    assert st.value & 2
    # the skipped block reads as zero rows with zero scale: logits 0 there
    assert torch.all(logits[1, 2 * bs:3 * bs] == 0)
    ok_bt = bt.clone()
    ok_bt[1, 2] = 0
    want = IL.paged_mqa_logits(q.view(torch.uint8).numpy(), flat.numpy(), w.numpy(), ctx.numpy(),
                               ok_bt.numpy(), 4 * bs)
    _check(logits[:1], want[:1])


def test_indexer_topk_attention_chain():
    """A decode step's sparse path: indexer logits -> per-row top-2048 ->
    sparse_fwd_paged, each stage fed the previous one's output on the GPU."""
    B, H, bs, ctx_len, heads = 8, 64, 64, 6000, 64
    max_blocks = (ctx_len + bs - 1) // bs
    rng, q, flat, w, bt = _case(123, B, 1, H, bs, max_blocks)
    ctx = torch.full((B,), ctx_len, dtype=torch.int32, device=DEV)
    logits = G.fp8_paged_mqa_logits(q.to(DEV), _kv_view(flat.to(DEV), bs), w.to(DEV), ctx,
                                    bt.to(DEV), 8192)
    pos = torch.empty((B, 2048), dtype=torch.int32, device=DEV)
    G.top_k_per_row_decode(logits, 1, ctx, pos, B, logits.stride(0), 1, 2048)
    torch.cuda.synchronize()
    lg = logits.cpu().numpy()
    for r in range(B):
        assert TK.check_row(pos[r].cpu().numpy(), lg[r], 0, ctx_len, 2048) is None
    # the attention's latent cache shares the block table with the indexer cache
    kv = torch.randn((flat.shape[0] * bs, 512), device=DEV).to(torch.bfloat16)
    qa = torch.randn((B, heads, 512), device=DEV).to(torch.bfloat16)
    req = torch.arange(B, dtype=torch.int32, device=DEV)
    out = G.sparse_fwd_paged(qa, kv, pos, req, bt.to(DEV), bs, 512 ** -0.5)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
