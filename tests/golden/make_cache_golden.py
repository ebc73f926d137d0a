"""Generate the golden vectors that pin oracle/cache_writer_oracle.py.

Run on a GPU machine with vLLM installed (it is NOT needed at test time):

    python tests/golden/make_cache_golden.py

It runs vLLM's own latent-cache write, ``vllm._custom_ops.concat_and_cache_mla``
(vllm 0.22.0, vllm/_custom_ops.py:2613-2623: the op MLAAttentionImpl's default
``do_kv_cache_update`` calls and the reference leaves vLLM to run), on seeded
inputs in this path's geometry (kv_lora_rank 512, pe_dim 0) and stores inputs
and outputs in tests/golden/cache_writer_golden.npz:

  kv_c           uint16 [N, 512]  bf16 bit patterns (N >= T: padded rows)
  slots          int64  [T]       slot mapping (-1 = padded token)
  init_bf16      uint16 [B, S, 512] cache before the write ("auto" case)
  init_fp8       uint8  [B, S, 512] cache before the write ("fp8" cases)
  out_auto       uint16 [B, S, 512] cache after the "auto" write
  out_fp8_<k>    uint8  [B, S, 512] cache after the "fp8" write, scale k
  scales         float32 [K]       the fp8 scales used (k indexes them)

The rows mix magnitudes from 1e-6 to 1e4, so the fp8 cases cover e4m3
subnormals, rounding ties and saturation at +-448.
"""

from __future__ import annotations

import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "cache_writer_golden.npz")

BLOCKS, BLOCK_SIZE, WIDTH = 6, 16, 512
T, N = 72, 80
SCALES = np.array([1.0, 0.05, 3.7], np.float32)


def make_inputs(seed: int = 1234):
    rng = np.random.default_rng(seed)
    mag = 10.0 ** rng.uniform(-6, 4, size=(N, 1))
    x = (rng.standard_normal((N, WIDTH)) * mag).astype(np.float32)
    # the exact midpoints between neighbouring e4m3 values (exact in bf16 as
    # well) exercise ties-to-even at scale 1
    codes = np.arange(0x7F)
    e4m3 = np.where(codes >> 3 == 0, (codes & 7) / 8.0 * 2.0 ** -6,
                    (1 + (codes & 7) / 8.0) * 2.0 ** ((codes >> 3) - 7.0))
    mids = ((e4m3[:-1] + e4m3[1:]) / 2).astype(np.float32)
    x[0, :mids.size] = mids
    x[0, mids.size:2 * mids.size] = -mids
    x[1, :8] = [448.0, 464.0, 480.0, -500.0, 1e30, -1e30, 2.0 ** -10, -(2.0 ** -10)]
    kv_c = torch.from_numpy(x).to(torch.bfloat16)
    slots = rng.permutation(BLOCKS * BLOCK_SIZE)[:T].astype(np.int64)
    slots[rng.random(T) < 0.1] = -1
    assert slots[0] >= 0 and slots[1] >= 0   # the tie and saturation rows are written
    init_bf16 = torch.from_numpy(
        rng.standard_normal((BLOCKS, BLOCK_SIZE, WIDTH)).astype(np.float32)).to(torch.bfloat16)
    init_fp8 = torch.from_numpy(rng.integers(0, 256, (BLOCKS, BLOCK_SIZE, WIDTH), dtype=np.uint8))
    return kv_c, slots, init_bf16, init_fp8


def main() -> None:
    from vllm import _custom_ops as ops

    dev = torch.device("cuda")
    kv_c, slots, init_bf16, init_fp8 = make_inputs()
    kv_c_d = kv_c.to(dev)
    k_pe = torch.empty((N, 0), dtype=torch.bfloat16, device=dev)
    slots_d = torch.from_numpy(slots).to(dev)
    res = {
        "kv_c": kv_c.view(torch.uint16).numpy(),
        "slots": slots,
        "init_bf16": init_bf16.view(torch.uint16).numpy(),
        "init_fp8": init_fp8.numpy(),
        "scales": SCALES,
    }
    cache = init_bf16.to(dev)
    one = torch.ones(1, dtype=torch.float32, device=dev)
    ops.concat_and_cache_mla(kv_c_d, k_pe, cache, slots_d, "auto", one)
    res["out_auto"] = cache.cpu().view(torch.uint16).numpy()
    for k, s in enumerate(SCALES):
        cache8 = init_fp8.to(dev)
        scale = torch.tensor([float(s)], dtype=torch.float32, device=dev)
        ops.concat_and_cache_mla(kv_c_d, k_pe, cache8, slots_d, "fp8", scale)
        res[f"out_fp8_{k}"] = cache8.cpu().numpy()
    torch.cuda.synchronize()
    np.savez_compressed(OUT, **res)
    print("wrote", OUT, {k: v.shape for k, v in res.items()})


if __name__ == "__main__":
    main()
