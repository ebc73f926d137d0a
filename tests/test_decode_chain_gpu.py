"""A sparse decode step's four kernels chained on one stream, several steps in
a row with no host synchronisation between them, in the order vLLM's decode
runs them: the latent KV-cache writer, the indexer's fp8 logits, its per-row
top-k, and the paged sparse-MLA attention.

Each kernel may begin launching while the previous one drains, and waits for
it before its first global access. So each step's attention must read the
row that its own writer stored three launches earlier, never the previous
step's row. Every step writes a different row at the newest position. The
row is aligned with every head's query, so it carries a large share of the
softmax weight. Each step's output is checked against the fp32 oracle
computed with that step's rows, within the parity tolerance. The test also
checks that reading the previous step's row would miss by far more than the
tolerance.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import COS_TOL, REL_TOL, parity_metrics
from oracle import sparse_mla_oracle as O

pytestmark = pytest.mark.gpu

import glm53_sparse_mla as G  # noqa: E402

DEV = torch.device("cuda")


def test_chained_decode_steps_see_their_own_writes():
    g = torch.Generator().manual_seed(7)
    R, ctx, bs, H, topk, steps = 4, 1024, 64, 64, 2048, 4
    bpr = ctx // bs
    nb = R * bpr + 3
    scale = 512 ** -0.5
    bt = torch.stack([torch.randperm(nb, generator=g)[:bpr] for _ in range(R)]).to(torch.int32)
    lat0 = (torch.randn((nb, bs, 512), generator=g) * 0.5).to(torch.bfloat16)
    u = torch.randn(512, generator=g)
    q = (u + 0.5 * torch.randn((R, H, 512), generator=g)).to(torch.bfloat16)
    kv_new = torch.stack([0.3 * (s + 1) * u.expand(R, 512) + 0.1 * torch.randn((R, 512), generator=g)
                          for s in range(steps)]).to(torch.bfloat16)          # [steps, R, 512]
    # the indexer's inputs (ctx <= topk, so the top-k keeps every position)
    vals = torch.randn((nb, bs * 128), generator=g).to(torch.float8_e4m3fn).view(torch.uint8)
    sc = (torch.rand((nb, bs), generator=g) + 0.5).view(torch.uint8)
    icache = torch.cat([vals, sc], 1).contiguous().view(nb, bs, 1, 132)
    qi = torch.randn((R, 1, 64, 128), generator=g).to(torch.float8_e4m3fn)
    w = torch.randn((R, 64), generator=g)

    last = ctx - 1
    slots = bt[:, last // bs].to(torch.int64) * bs + last % bs
    lat = lat0.to(DEV)
    bt_d, slots_d, kvn_d = bt.to(DEV), slots.to(DEV), kv_new.to(DEV)
    q_d, icache_d, qi_d, w_d = q.to(DEV), icache.to(DEV), qi.to(DEV), w.to(DEV)
    ctx_t = torch.full((R,), ctx, dtype=torch.int32, device=DEV)
    req = torch.arange(R, dtype=torch.int32, device=DEV)
    logits = torch.empty((R, ctx), dtype=torch.float32, device=DEV)
    pos = torch.empty((R, topk), dtype=torch.int32, device=DEV)
    one = torch.ones(1, dtype=torch.float32, device=DEV)
    outs = [torch.empty((R, H, 512), dtype=torch.bfloat16, device=DEV) for _ in range(steps)]
    for s in range(steps):
        G.concat_and_cache_mla(kvn_d[s], kvn_d[s][:, :0], lat, slots_d, "auto", one)
        G.fp8_paged_mqa_logits(qi_d, icache_d, w_d, ctx_t, bt_d, ctx, logits=logits)
        G.top_k_per_row_decode(logits, 1, ctx_t, pos, R, ctx, 1, topk)
        G.sparse_fwd_paged(q_d, lat.view(-1, 512), pos, req, bt_d, bs, scale, out=outs[s])
    torch.cuda.synchronize()

    p = np.arange(topk)
    idx = np.where(p[None, :] < ctx,
                   bt.numpy()[:, np.minimum(p, ctx - 1) // bs].astype(np.int64) * bs + p % bs, -1)
    assert np.array_equal(pos.cpu().numpy(), np.where(p < ctx, p, -1)[None, :].repeat(R, 0))

    def oracle(rows):
        kv = lat0.clone().view(-1, 512)
        kv[slots] = rows
        ref, _, _ = O.sparse_mla_stats(q.float().numpy(), kv.float().numpy(), idx, scale)
        return ref

    refs = [oracle(kv_new[s]) for s in range(steps)]
    for s in range(steps):
        rel, cmin, finite = parity_metrics(outs[s].float().cpu().numpy(), refs[s])
        assert finite, s
        assert rel <= REL_TOL and cmin >= COS_TOL, f"step {s}: rel={rel:.3e} cos={cmin:.7f}"
        if s > 0:   # the previous step's row would be caught
            stale_rel, _, _ = parity_metrics(refs[s - 1], refs[s])
            assert stale_rel > 10 * REL_TOL, (s, stale_rel)
