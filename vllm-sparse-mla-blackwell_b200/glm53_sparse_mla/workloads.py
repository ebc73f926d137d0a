"""Seeded synthetic inputs for the sparse-MLA path.

Two families:

* ``case_matrix`` -- the mask/shape cases the reference gates its kernel on
  (tests/cases.py:26-71 of the reference): all valid, 10% and 50% scattered
  -1, one 64-wide tile masked, one token fully masked, duplicate indices,
  index 0 repeated, extreme logits (q x 100), token-count tails. Indices are
  drawn uniformly with replacement from [0, rows).
* ``baseline_config`` -- the five configurations the benchmark is quoted on:
  C1 CPU plumbing, C2 decode bf16 @ 64 heads, C3 mixed prefill + decode,
  C4 fp8 long-context decode, C5 MTP head-sharding sweep. Paged KV with
  block size 64 and random / shuffled block tables; indices are the physical
  slot ids ``block_table[pos // 64] * 64 + pos % 64``.

Small tensors (q, indices, the C1 / case-matrix pools) are generated with
numpy's PCG64 from a fixed seed, so their bits are identical on every machine
and device. Large KV pools are generated in chunks on the target device with a
seeded torch generator; parity tests read back only the rows they check.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

D = 512
BLOCK = 64
FP8_MAX = 448.0


@dataclass
class Workload:
    name: str
    q: torch.Tensor            # [T, H, 512] bf16
    kv: torch.Tensor           # [R, 512] bf16 or float8_e4m3fn
    indices: torch.Tensor      # [T, topk] int32
    sm_scale: float
    kv_scale: float = 1.0
    meta: dict = field(default_factory=dict)

    @property
    def T(self) -> int:
        return int(self.q.shape[0])

    @property
    def H(self) -> int:
        return int(self.q.shape[1])

    @property
    def topk(self) -> int:
        return int(self.indices.shape[1])

    def n_valid(self) -> int:
        return int((self.indices >= 0).sum().item())

    def algorithmic_bytes(self, with_lse: bool = False) -> int:
        """Unique bytes the op must move: gathered KV rows (counted per valid
        index), q in, out, indices (and lse)."""
        e_kv = 1 if self.kv.dtype == torch.float8_e4m3fn else 2
        b = self.n_valid() * D * e_kv + 2 * self.T * self.H * D * 2 + self.T * self.topk * 4
        if with_lse:
            b += self.T * self.H * 4
        return b

    def flops(self) -> int:
        """QK^T plus PV over the valid indices: 4 * N_valid * H * 512."""
        return 4 * self.n_valid() * self.H * D


# ---------------------------------------------------------------------------
# value helpers
# ---------------------------------------------------------------------------
def _bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(
        np.uint16)


def bf16_tensor_from_f32(x: np.ndarray, device="cpu") -> torch.Tensor:
    bits = _bf16_bits(x)
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(device)


def quantize_fp8(x: torch.Tensor, scale: float) -> torch.Tensor:
    """e4m3(clamp(x / scale, +-448)), as vLLM's per-tensor cache writer does."""
    return (x.float() / scale).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)


def dequantize_fp8(kv8: torch.Tensor, scale: float, exact: bool = False) -> torch.Tensor:
    """The fp8 cache's values: float(e4m3) * scale in fp32 (``exact``, what
    this repository's kernel computes with: e4m3 exactly in f16 operands,
    the scale applied in fp32), or rounded to bf16 as the reference kernel
    and its fp8 test do (tests/run_fp8.py:36 of the reference)."""
    v = kv8.float() * scale
    return v if exact else v.to(torch.bfloat16)


def _normal_bf16(rng: np.random.Generator, shape, device) -> torch.Tensor:
    return bf16_tensor_from_f32(rng.standard_normal(shape, dtype=np.float32), device)


def device_pool(rows: int, seed: int, device, kv_dtype: str = "bf16", fp8_scale: float = 0.05,
                chunk_rows: int = 1 << 18) -> torch.Tensor:
    """[rows, 512] KV pool ~N(0,1), generated on `device` in chunks.

    kv_dtype "fp8": values N(0,1) / fp8_scale clipped to +-448 and cast to
    e4m3 (so the dequantised values are ~N(0,1) again with scale fp8_scale).
    """
    dt = torch.float8_e4m3fn if kv_dtype == "fp8" else torch.bfloat16
    out = torch.empty(rows, D, dtype=dt, device=device)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    for r0 in range(0, rows, chunk_rows):
        r1 = min(rows, r0 + chunk_rows)
        x = torch.randn(r1 - r0, D, generator=g, device=device, dtype=torch.float32)
        if kv_dtype == "fp8":
            out[r0:r1] = quantize_fp8(x, fp8_scale)
        else:
            out[r0:r1] = x.to(torch.bfloat16)
    return out


# ---------------------------------------------------------------------------
# the reference's mask / shape case matrix
# ---------------------------------------------------------------------------
def case_matrix(heads: int = 32, topk: int = 2048, rows: int = 8192, device="cpu",
                kv_dtype: str = "bf16", seed: int = 0):
    """Yields Workloads covering the reference's case list (see module doc)."""

    def base(T, s):
        rng = np.random.default_rng(1000 * seed + s)
        q = _normal_bf16(rng, (T, heads, D), device)
        kv32 = rng.standard_normal((rows, D), dtype=np.float32)
        if kv_dtype == "fp8":
            scale = float(np.abs(bf16_tensor_from_f32(kv32).float().numpy()).max() / FP8_MAX)
            kv = quantize_fp8(bf16_tensor_from_f32(kv32).float(), scale).to(device)
        else:
            scale = 1.0
            kv = bf16_tensor_from_f32(kv32, device)
        return rng, q, kv, scale

    def idx(rng, T, k):
        return rng.integers(0, rows, size=(T, k), dtype=np.int64).astype(np.int32)

    def W(name, q, kv, ind, scale):
        return Workload(name, q, kv, torch.from_numpy(np.ascontiguousarray(ind)).to(device),
                        D ** -0.5, scale)

    rng, q, kv, sc = base(8, 1)
    yield W("all_valid", q, kv, idx(rng, 8, topk), sc)
    for frac, name in ((0.1, "mask_10pct"), (0.5, "mask_50pct")):
        rng, q, kv, sc = base(8, 2)
        ind = idx(rng, 8, topk)
        ind[rng.random(ind.shape) < frac] = -1
        yield W(name, q, kv, ind, sc)
    rng, q, kv, sc = base(4, 3)
    ind = idx(rng, 4, topk)
    ind[:, 64:128] = -1
    yield W("one_tile_masked", q, kv, ind, sc)
    rng, q, kv, sc = base(4, 4)
    ind = idx(rng, 4, topk)
    ind[2, :] = -1
    yield W("row_fully_masked", q, kv, ind, sc)
    rng, q, kv, sc = base(4, 5)
    yield W("duplicate_indices", q, kv, np.tile(idx(rng, 4, max(topk // 8, 1)), (1, 8))[:, :topk], sc)
    rng, q, kv, sc = base(2, 6)
    yield W("index0_repeated", q, kv, np.zeros((2, topk), np.int32), sc)
    rng, q, kv, sc = base(4, 7)
    q100 = (q.float() * 100).to(torch.bfloat16)
    yield W("extreme_logits", q100, kv, idx(rng, 4, topk), sc)
    for T in (1, 7, 128):
        rng, q, kv, sc = base(T, 100 + T)
        yield W(f"tokens_{T}", q, kv, idx(rng, T, topk), sc)


def edge_cases(heads: int = 16, topk: int = 512, rows: int = 4096, device="cpu", seed: int = 7):
    """Shapes aimed at this kernel's compaction and split logic: valid counts
    around the 64-row tile size, a chunk with no valid entry, front-packed
    (prefill-like) rows, a single valid index, and ids >= rows (masked)."""
    rng = np.random.default_rng(seed)
    T = 12
    q = _normal_bf16(rng, (T, heads, D), device)
    kv = _normal_bf16(rng, (rows, D), device)
    ind = rng.integers(0, rows, size=(T, topk), dtype=np.int64).astype(np.int32)
    counts = [63, 64, 65, 1, 127, 128, 129, topk // 4, 0, topk - 1]
    for t, c in enumerate(counts):
        ind[t, c:] = -1                       # valid entries packed at the front
    ind[10, :] = -1
    ind[10, topk - 1] = int(rng.integers(0, rows))   # one valid index at the very end
    ind[11, ::3] = rows + 5                   # out of range -> treated as masked
    return Workload("edge_cases", q, kv, torch.from_numpy(ind).to(device), D ** -0.5, 1.0,
                    meta={"bad_index_row": 11})


# ---------------------------------------------------------------------------
# the benchmark configurations
# ---------------------------------------------------------------------------
def _paged_slots(rng, block_table: np.ndarray, pos: np.ndarray) -> np.ndarray:
    return (block_table[pos // BLOCK] * BLOCK + pos % BLOCK).astype(np.int32)


def config_c1(device="cpu", seed: int = 1) -> Workload:
    """CPU plumbing: 4 tokens, 16 heads, topk 128, pool 4096 bf16; indices
    uniform without replacement, ~10% -1, token 3 fully masked."""
    rng = np.random.default_rng(seed)
    T, H, K, R = 4, 16, 128, 4096
    q = _normal_bf16(rng, (T, H, D), device)
    kv = _normal_bf16(rng, (R, D), device)
    ind = np.stack([rng.choice(R, K, replace=False) for _ in range(T)]).astype(np.int32)
    ind[rng.random(ind.shape) < 0.1] = -1
    ind[3, :] = -1
    return Workload("c1_cpu_plumbing", q, kv, torch.from_numpy(ind).to(device), D ** -0.5)


def config_c2(device="cuda", seed: int = 2, heads: int = 64) -> Workload:
    """Decode, bf16 KV: 32 sequences x 1 token, 64 heads, topk 2048; pool of
    131072 slots (2048 blocks of 64); each sequence owns a random 128-block
    table (context 8192) and picks 2048 distinct positions of its context."""
    rng = np.random.default_rng(seed)
    n_seq, ctx, n_blocks, K = 32, 8192, 2048, 2048
    ind = np.empty((n_seq, K), np.int32)
    for s in range(n_seq):
        bt = rng.choice(n_blocks, ctx // BLOCK, replace=False)
        ind[s] = _paged_slots(rng, bt, rng.choice(ctx, K, replace=False))
    q = _normal_bf16(rng, (n_seq, heads, D), device)
    kv = device_pool(n_blocks * BLOCK, seed, device)
    return Workload("c2_decode_bf16_h%d" % heads, q, kv, torch.from_numpy(ind).to(device),
                    D ** -0.5, meta={"n_seq": n_seq, "context": ctx})


def config_c3(device="cuda", seed: int = 3, heads: int = 32) -> Workload:
    """Mixed prefill + decode in one launch: one 4096-token prefill plus 31
    decode tokens at context 16384, 32 heads, topk 2048, shuffled blocks.
    Prefill token i picks min(i+1, 2048) causal positions <= i, tail -1."""
    rng = np.random.default_rng(seed)
    K, pre, n_dec, ctx_dec = 2048, 4096, 31, 16384
    blocks_pre, blocks_dec = pre // BLOCK, ctx_dec // BLOCK
    n_blocks = blocks_pre + n_dec * blocks_dec
    perm = rng.permutation(n_blocks)
    bt_pre = perm[:blocks_pre]
    ind = np.full((pre + n_dec, K), -1, np.int32)
    for i in range(pre):
        n = min(i + 1, K)
        pos = rng.permutation(i + 1)[:n] if i + 1 > K else rng.permutation(i + 1)
        ind[i, :n] = _paged_slots(rng, bt_pre, pos)
    for j in range(n_dec):
        bt = perm[blocks_pre + j * blocks_dec: blocks_pre + (j + 1) * blocks_dec]
        ind[pre + j] = _paged_slots(rng, bt, rng.choice(ctx_dec, K, replace=False))
    q = _normal_bf16(rng, (pre + n_dec, heads, D), device)
    kv = device_pool(n_blocks * BLOCK, seed, device)
    return Workload("c3_mixed_prefill_decode", q, kv, torch.from_numpy(ind).to(device), D ** -0.5,
                    meta={"prefill_tokens": pre, "decode_tokens": n_dec})


def config_c4(device="cuda", seed: int = 4, heads: int = 16, kv_dtype: str = "fp8") -> Workload:
    """fp8_e4m3 decode at long context: 64 sequences x 1 token, 16 heads, topk
    2048, context 65536, pool of 524288 fp8 slots with per-tensor scale 0.05,
    ~2% -1 sentinels. ``kv_dtype="bf16"`` gives the same shape with a bf16
    pool (the fp8-vs-bf16 comparison at this shape)."""
    rng = np.random.default_rng(seed)
    n_seq, ctx, n_blocks, K, scale = 64, 65536, 8192, 2048, 0.05
    ind = np.empty((n_seq, K), np.int32)
    for s in range(n_seq):
        bt = rng.choice(n_blocks, ctx // BLOCK, replace=False)
        ind[s] = _paged_slots(rng, bt, rng.choice(ctx, K, replace=False))
    ind[rng.random(ind.shape) < 0.02] = -1
    q = _normal_bf16(rng, (n_seq, heads, D), device)
    kv = device_pool(n_blocks * BLOCK, seed, device, kv_dtype, scale)
    name = "c4_decode_fp8_long" if kv_dtype == "fp8" else "c4_decode_bf16_long"
    return Workload(name, q, kv, torch.from_numpy(ind).to(device), D ** -0.5,
                    kv_scale=scale if kv_dtype == "fp8" else 1.0, meta={"n_seq": n_seq, "context": ctx})


def config_c5(device="cuda", seed: int = 5, heads: int = 64, kv_dtype: str = "bf16",
              head_offset: int = 0) -> Workload:
    """MTP head-sharding shape: 128 sequences x 4 query tokens (uniform batch),
    context 32768, pool 4,194,304 slots (disjoint shuffled block tables), topk
    2048 causal picks per token. `heads` / `head_offset` select this rank's
    slice of the 64 query heads (q is generated for all 64 and sliced)."""
    rng = np.random.default_rng(seed)
    n_seq, mtp, ctx, K = 128, 4, 32768, 2048
    blocks = ctx // BLOCK
    perm = rng.permutation(n_seq * blocks)
    ind = np.full((n_seq * mtp, K), -1, np.int32)
    for s in range(n_seq):
        bt = perm[s * blocks:(s + 1) * blocks]
        for j in range(mtp):
            p = ctx - mtp + j
            n = min(p + 1, K)
            ind[s * mtp + j, :n] = _paged_slots(rng, bt, rng.choice(p + 1, n, replace=False))
    q_all = _normal_bf16(rng, (n_seq * mtp, 64, D), device)
    q = q_all[:, head_offset:head_offset + heads].contiguous()
    kv = device_pool(n_seq * blocks * BLOCK, seed, device, kv_dtype, 0.05)
    return Workload(f"c5_mtp_{kv_dtype}_h{heads}", q, kv, torch.from_numpy(ind).to(device),
                    D ** -0.5, kv_scale=0.05 if kv_dtype == "fp8" else 1.0,
                    meta={"n_seq": n_seq, "mtp": mtp, "context": ctx})
