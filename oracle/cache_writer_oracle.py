"""CPU oracle for the latent KV-cache writer -- TEST INFRASTRUCTURE ONLY.

Only tests/ and bench.py's CPU legs may import this module, and only as the
checker (or as the timed CPU reference in bench.py). The product path never
calls it.

The reference's backend keeps vLLM's plain ``fp8`` cache layout for this NoPE
model (glm53_sparse_mla/backend.py:398-428 of jsmcconn/vllm-sparse-mla-
blackwell) and leaves the write itself to vLLM: MLAAttentionImpl's default
``do_kv_cache_update`` (vllm 0.22.0, vllm/v1/attention/backend.py:990-1010)
calls ``concat_and_cache_mla`` (vllm/_custom_ops.py:2613-2623), a compiled
vLLM op. vLLM is a dependency of the reference, not part of it; this module
restates the op's published rule for the path's geometry
(kv_lora_rank = 512, pe_dim = 0):

  * tokens: ``slot_mapping.shape[0]`` of them (kv_c may hold more rows,
    padding for CUDA graphs); a slot < 0 is a padded token and writes nothing;
  * slot s lands in block ``s // block_size`` at offset ``s % block_size``;
  * ``kv_cache_dtype == "auto"``: the cache entry is the bf16 row as it is;
  * ``"fp8"`` / ``"fp8_e4m3"``: each element becomes
    e4m3(float(x) / scale), fp32 division rounded to nearest even, then the
    float -> e4m3 conversion with round-to-nearest-even and saturation to
    +-448 (``__NV_SATFINITE``).

Parity pin: tests/golden/make_cache_golden.py runs vLLM's own op on a GPU and
stores its inputs and outputs (tests/golden/cache_writer_golden.npz);
tests/test_cache_writer_cpu.py checks this restatement against them byte for
byte.
"""

from __future__ import annotations

import numpy as np

from .sparse_mla_oracle import bf16_to_f32, e4m3_to_f32

KV_WIDTH = 512
E4M3_MAX = 448.0

# the 127 non-negative finite e4m3 values, code i <-> value _E4M3_POS[i]
_E4M3_POS = e4m3_to_f32(np.arange(0x7F, dtype=np.uint8)).astype(np.float64)


def f32_to_e4m3_satfinite(x: np.ndarray) -> np.ndarray:
    """float32 -> float8_e4m3fn bit patterns: nearest value, ties to the even
    code, |x| beyond 448 saturated to 448, the sign kept (also on zero); NaN
    maps to 0x7F."""
    x = np.asarray(x, dtype=np.float32)
    mag = np.minimum(np.abs(x).astype(np.float64), E4M3_MAX)
    hi = np.searchsorted(_E4M3_POS, mag, side="left")          # first value >= mag
    hi = np.minimum(hi, len(_E4M3_POS) - 1)
    lo = np.maximum(hi - 1, 0)
    d_lo = mag - _E4M3_POS[lo]
    d_hi = _E4M3_POS[hi] - mag
    pick_hi = (d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0))
    code = np.where(pick_hi, hi, lo).astype(np.uint8)
    code = np.where(np.signbit(x), code | np.uint8(0x80), code).astype(np.uint8)
    return np.where(np.isnan(x), np.uint8(0x7F), code).astype(np.uint8)


def quantize_row_e4m3(row_bf16_bits: np.ndarray, scale: float) -> np.ndarray:
    """Cache entries of the fp8 path: e4m3(float(x) / scale) per element."""
    v = bf16_to_f32(row_bf16_bits)
    q = (v / np.float32(scale)).astype(np.float32)              # IEEE fp32 division
    return f32_to_e4m3_satfinite(q)


def concat_and_cache_mla(kv_c_bits: np.ndarray, cache: np.ndarray, slot_mapping: np.ndarray,
                         kv_cache_dtype: str, scale: float = 1.0,
                         inplace: bool = False) -> np.ndarray:
    """Returns the cache after the write (a new array unless ``inplace``).

    kv_c_bits: uint16 bf16 bit patterns [N >= T, 512]; cache: uint16 (auto) or
    uint8 (fp8) [num_blocks, block_size, 512]; slot_mapping: int [T].
    """
    if not inplace:
        cache = np.array(cache, copy=True)
    nb, bs, width = cache.shape
    assert width == KV_WIDTH and kv_c_bits.shape[1] == KV_WIDTH
    slots = np.asarray(slot_mapping, dtype=np.int64)
    assert kv_c_bits.shape[0] >= slots.shape[0]
    fp8 = kv_cache_dtype in ("fp8", "fp8_e4m3")
    if not fp8 and kv_cache_dtype != "auto":
        raise ValueError(f"kv_cache_dtype {kv_cache_dtype!r} is not written by this path")
    t = np.nonzero(slots >= 0)[0]              # padded tokens write nothing
    blk, off = np.divmod(slots[t], bs)
    rows = kv_c_bits[t]
    cache[blk, off] = quantize_row_e4m3(rows, scale) if fp8 else rows
    return cache
