"""The latent KV-cache writer on a B200 (glm53_sparse_mla.concat_and_cache_mla,
C ABI glm53_concat_and_cache), checked byte for byte.

* against the oracle (oracle/cache_writer_oracle.py) on seeded inputs: bf16
  ``auto`` and fp8 at several scales, padded tokens (slot -1), strided kv_c
  rows, padded pages (block stride > block_size * 512), magnitudes from e4m3
  subnormals through saturation, T = 0, 1 and a prefill-sized batch;
* against vLLM's own concat_and_cache_mla on the same inputs, when vLLM's
  compiled ops load;
* a slot past the cache is skipped, raises the writer's status bit and leaves
  the memory past the cache untouched;
* write -> attend: the fp8 cache it writes, read by sparse_fwd_paged, matches
  the attention oracle on the exactly dequantised cache;
* the backend's do_kv_cache_update goes through it.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from conftest import COS_TOL, REL_TOL, parity_metrics
from oracle import cache_writer_oracle as CW
from oracle import sparse_mla_oracle as O

pytestmark = pytest.mark.gpu

import glm53_sparse_mla as G  # noqa: E402

DEV = torch.device("cuda")


def _inputs(T, N, blocks, bs, seed, kv_stride=512):
    rng = np.random.default_rng(seed)
    mag = 10.0 ** rng.uniform(-6, 4, size=(N, 1))
    x = (rng.standard_normal((N, 512)) * mag).astype(np.float32)
    base = torch.from_numpy(
        np.concatenate([x, rng.standard_normal((N, kv_stride - 512)).astype(np.float32)], 1)
    ).to(torch.bfloat16).to(DEV)
    kv_c = base[:, :512]                                  # rows kv_stride apart
    slots = rng.permutation(blocks * bs)[:T].astype(np.int64)
    slots[rng.random(T) < 0.1] = -1
    return kv_c, torch.from_numpy(slots).to(DEV)


def _cache(blocks, bs, dtype, page_pad, seed):
    """A paged cache view [blocks, bs, 512] over a buffer with page_pad extra
    entries per block, plus the buffer (to check the padding stays as it was)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    if dtype == "auto":
        buf = torch.randn((blocks, bs + page_pad, 512), generator=g).to(torch.bfloat16).to(DEV)
    else:
        buf = torch.randint(0, 256, (blocks, bs + page_pad, 512), generator=g,
                            dtype=torch.uint8).to(DEV)
    return buf[:, :bs], buf


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.cpu()
    return (t.view(torch.uint16) if t.dtype == torch.bfloat16 else t.view(torch.uint8)).numpy()


@pytest.mark.parametrize("dtype,scale", [("auto", 1.0), ("fp8", 1.0), ("fp8", 0.05),
                                         ("fp8_e4m3", 3.7)])
@pytest.mark.parametrize("T,kv_stride,page_pad", [(1, 512, 0), (61, 576, 0), (200, 512, 3),
                                                  (5000, 512, 0)])
def test_matches_oracle(dtype, scale, T, kv_stride, page_pad):
    bs = 64
    blocks = max(4, (T + bs - 1) // bs + 2)
    kv_c, slots = _inputs(T, T + 5, blocks, bs, seed=T + kv_stride, kv_stride=kv_stride)
    cache, buf = _cache(blocks, bs, dtype, page_pad, seed=T)
    want_buf = _bits(buf).copy()
    s = torch.tensor([scale], dtype=torch.float32, device=DEV)
    G.concat_and_cache_mla(kv_c, kv_c[:, :0], cache, slots, dtype, s)
    torch.cuda.synchronize()
    want = CW.concat_and_cache_mla(_bits(kv_c.contiguous()), want_buf[:, :bs], slots.cpu().numpy(),
                                   dtype, scale)
    got = _bits(buf)
    assert np.array_equal(got[:, :bs], want)
    assert np.array_equal(got[:, bs:], want_buf[:, bs:])   # page padding untouched


SCALES = [1.0, 0.05, 3.7, 1.0 / 3.0, 2.0 ** -7, 448.0 / 65504.0, 1e-3, 123.456, 0.999, 1.001,
          -0.5] + list(np.exp(np.random.default_rng(5).uniform(np.log(1e-4), np.log(1e4), 30)))


def _all_bf16():
    """Every bf16 bit pattern once: 128 rows x 512."""
    return torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16) \
        .reshape(128, 512).to(DEV)


def test_fp8_every_bf16_value_every_scale():
    """The division by the scale (reciprocal + FMA correction) and the e4m3
    conversion, over all 65536 bf16 inputs at each scale: bytes equal the
    oracle's IEEE-division result; NaN inputs give an e4m3 NaN."""
    kv_c = _all_bf16()
    bits = _bits(kv_c)
    nan = np.isnan(O.bf16_to_f32(bits))
    slots = torch.arange(128, dtype=torch.int64, device=DEV)
    for scale in SCALES:
        cache = torch.zeros((2, 64, 512), dtype=torch.uint8, device=DEV)
        G.concat_and_cache_mla(kv_c, kv_c[:, :0], cache, slots, "fp8",
                               torch.tensor([scale], dtype=torch.float32, device=DEV))
        got = _bits(cache).reshape(128, 512)
        want = CW.concat_and_cache_mla(bits, np.zeros((2, 64, 512), np.uint8),
                                       np.arange(128), "fp8", float(np.float32(scale)))
        want = want.reshape(128, 512)
        bad = (got != want) & ~nan
        assert not bad.any(), (scale, int(bad.sum()), bits[bad][:8], got[bad][:8], want[bad][:8])
        assert np.all((got[nan] & 0x7F) == 0x7F)


def test_empty_batch_is_a_no_op():
    cache, buf = _cache(2, 16, "fp8", 0, seed=1)
    before = _bits(buf).copy()
    G.concat_and_cache_mla(torch.empty((0, 512), dtype=torch.bfloat16, device=DEV),
                           torch.empty((0, 0), dtype=torch.bfloat16, device=DEV), cache,
                           torch.empty((0,), dtype=torch.int64, device=DEV), "fp8",
                           torch.ones(1, device=DEV))
    torch.cuda.synchronize()
    assert np.array_equal(_bits(buf), before)


def test_matches_vllm_op():
    try:
        from vllm import _custom_ops as ops
        ops_fn = torch.ops._C_cache_ops.concat_and_cache_mla
    except Exception as exc:   # vLLM's compiled ops are library code, optional here
        pytest.skip(f"vLLM cache ops unavailable: {exc}")
    del ops_fn
    T, bs, blocks = 300, 64, 8
    kv_c, slots = _inputs(T, T, blocks, bs, seed=7)
    k_pe = torch.empty((T, 0), dtype=torch.bfloat16, device=DEV)
    for dtype, scale in [("auto", 1.0), ("fp8", 1.0), ("fp8", 0.05), ("fp8", 3.7)]:
        ours, _ = _cache(blocks, bs, dtype, 0, seed=3)
        theirs = ours.clone()
        s = torch.tensor([scale], dtype=torch.float32, device=DEV)
        G.concat_and_cache_mla(kv_c, k_pe, ours, slots, dtype, s)
        ops.concat_and_cache_mla(kv_c, k_pe, theirs, slots, dtype, s)
        torch.cuda.synchronize()
        assert torch.equal(ours.view(torch.uint8), theirs.view(torch.uint8)), (dtype, scale)
    # every bf16 value (NaN and inf included) at every test scale
    allv = _all_bf16()
    slots = torch.arange(128, dtype=torch.int64, device=DEV)
    pe = torch.empty((128, 0), dtype=torch.bfloat16, device=DEV)
    for scale in SCALES:
        ours = torch.zeros((2, 64, 512), dtype=torch.uint8, device=DEV)
        theirs = ours.clone()
        s = torch.tensor([scale], dtype=torch.float32, device=DEV)
        G.concat_and_cache_mla(allv, pe, ours, slots, "fp8", s)
        ops.concat_and_cache_mla(allv, pe, theirs, slots, "fp8", s)
        torch.cuda.synchronize()
        assert torch.equal(ours, theirs), scale


def test_slot_past_cache_is_skipped_and_reported():
    lib = ctypes.CDLL(G.library_path())
    lib.glm53_concat_and_cache_status.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_int]
    st = ctypes.c_uint32(0)
    assert lib.glm53_concat_and_cache_status(ctypes.byref(st), 1) == 0
    blocks, bs = 4, 16
    buf = torch.zeros((blocks + 1, bs, 512), dtype=torch.uint8, device=DEV)
    cache = buf[:blocks]                       # the last block is a guard
    kv_c = torch.ones((3, 512), dtype=torch.bfloat16, device=DEV)
    slots = torch.tensor([5, blocks * bs, blocks * bs + 7], dtype=torch.int64, device=DEV)
    G.concat_and_cache_mla(kv_c, kv_c[:, :0], cache, slots, "fp8", torch.ones(1, device=DEV))
    torch.cuda.synchronize()
    assert lib.glm53_concat_and_cache_status(ctypes.byref(st), 1) == 0
    assert st.value & 4                         # GLM53_DEV_BAD_SLOT
    assert int(buf[blocks].count_nonzero()) == 0
    assert int(cache.view(-1, 512)[5].count_nonzero()) == 512   # the valid slot was written


def test_rejects_other_layouts():
    cache = torch.zeros((2, 16, 512), dtype=torch.uint8, device=DEV)
    kv_c = torch.zeros((4, 512), dtype=torch.bfloat16, device=DEV)
    slots = torch.zeros(4, dtype=torch.int64, device=DEV)
    one = torch.ones(1, device=DEV)
    with pytest.raises(RuntimeError, match="pe_dim"):
        G.concat_and_cache_mla(kv_c, torch.zeros((4, 64), dtype=torch.bfloat16, device=DEV),
                               cache, slots, "fp8", one)
    with pytest.raises(RuntimeError, match="kv_cache_dtype"):
        G.concat_and_cache_mla(kv_c, kv_c[:, :0], cache, slots, "fp8_e5m2", one)
    with pytest.raises(RuntimeError, match="auto"):
        G.concat_and_cache_mla(kv_c, kv_c[:, :0], cache, slots, "auto", one)
    with pytest.raises(RuntimeError, match="int64"):
        G.concat_and_cache_mla(kv_c, kv_c[:, :0], cache, slots.int(), "fp8", one)


def test_write_then_attend_fp8():
    """Decode step: the writer fills an fp8 cache from bf16 latents, the
    paged op attends over it; compared with the attention oracle on the
    cache dequantised exactly (e4m3 * scale in fp32)."""
    T, H, topk, bs, n_req, ctx = 8, 32, 512, 64, 2, 2048
    rng = np.random.default_rng(21)
    blocks = n_req * ctx // bs
    bt = rng.permutation(blocks).reshape(n_req, ctx // bs).astype(np.int32)
    # every position of every request is written once
    pos = np.arange(ctx)
    slots = np.concatenate([bt[r][pos // bs] * bs + pos % bs for r in range(n_req)]).astype(np.int64)
    lat = torch.from_numpy(rng.standard_normal((n_req * ctx, 512)).astype(np.float32)).to(
        torch.bfloat16).to(DEV)
    cache = torch.zeros((blocks, bs, 512), dtype=torch.uint8, device=DEV)
    scale = 0.05
    G.concat_and_cache_mla(lat, lat[:, :0], cache, torch.from_numpy(slots).to(DEV), "fp8",
                           torch.tensor([scale], device=DEV))
    req = rng.integers(0, n_req, T).astype(np.int32)
    tp = np.stack([rng.choice(ctx, topk, replace=False) for _ in range(T)]).astype(np.int32)
    q = torch.from_numpy(rng.standard_normal((T, H, 512)).astype(np.float32)).to(torch.bfloat16).to(DEV)
    kv8 = cache.view(torch.float8_e4m3fn).view(-1, 512)
    out = G.sparse_fwd_paged(q, kv8, torch.from_numpy(tp).to(DEV), torch.from_numpy(req).to(DEV),
                             torch.from_numpy(bt).to(DEV), bs, 512 ** -0.5, scale)
    torch.cuda.synchronize()
    gslots = O.convert_req_index_to_global(req, bt, tp, bs)
    kv_deq = O.e4m3_to_f32(cache.view(-1, 512).cpu().numpy()) * np.float32(scale)
    uniq, inv = np.unique(gslots, return_inverse=True)
    ref, _, _ = O.sparse_mla_stats(q.float().cpu().numpy(), kv_deq[uniq], inv.reshape(gslots.shape),
                                   512 ** -0.5)
    rel, cmin, finite = parity_metrics(out.float().cpu().numpy(), ref)
    assert finite and rel <= REL_TOL and cmin >= COS_TOL, (rel, cmin)
    # and the cache bytes are the oracle's
    want = CW.concat_and_cache_mla(_bits(lat), np.zeros((blocks, bs, 512), np.uint8), slots, "fp8",
                                   scale)
    assert np.array_equal(_bits(cache), want)


def test_backend_do_kv_cache_update():
    B = pytest.importorskip("glm53_sparse_mla.backend")
    impl = B.Glm53SparseMLAImpl(
        num_heads=64, head_size=512, scale=512 ** -0.5, num_kv_heads=1, alibi_slopes=None,
        sliding_window=None, kv_cache_dtype="fp8", logits_soft_cap=None, attn_type="decoder",
        kv_sharing_target_layer_name=None, topk_indices_buffer=None, kv_lora_rank=512)
    T, bs, blocks = 40, 64, 4
    kv_c, slots = _inputs(T, T, blocks, bs, seed=9)
    ours = torch.zeros((blocks, bs, 512), dtype=torch.uint8, device=DEV)
    k_pe = torch.empty((T, 1, 0), dtype=torch.bfloat16, device=DEV)   # MLA layer's NoPE k_pe
    impl.do_kv_cache_update(kv_c, k_pe, ours, slots.view(-1, 1), "fp8",
                            torch.tensor([0.05], device=DEV))
    torch.cuda.synchronize()
    want = CW.concat_and_cache_mla(_bits(kv_c.contiguous()), np.zeros((blocks, bs, 512), np.uint8),
                                   slots.cpu().numpy(), "fp8", 0.05)
    assert np.array_equal(_bits(ours), want)
