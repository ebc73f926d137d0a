// Sparse MLA (NoPE: head size = kv_lora_rank = 512, no rope tail) for B200,
// sm_100a only. One launch serves prefill and decode tokens alike: each query
// token attends to the rows of a flat latent KV pool named by its top-k index
// list; an index < 0 is the only mask (causality belongs to the indexer).
//
// Work decomposition
//   grid.x = T * splits. The `splits` CTAs of one token form a thread-block
//   cluster and each takes a contiguous chunk of the token's index list; their
//   partial results are merged at the end of the same launch, either through a
//   global workspace that stays in L2 (glm53_sparse_mla_fwd_ws, the torch op,
//   the no-allocation entry point; at 32 and 64 heads the partials cross it as
//   f16 of each CTA's normalised output) or through distributed shared memory
//   (glm53_sparse_mla_fwd, no global scratch).
//   Before its grid-dependency wait a CTA prefetches its q rows and index
//   chunk into L2, so those loads overlap the previous grid's tail.
//
// Per CTA (384 threads, one CTA per SM, ~222 KB shared memory)
//   warps 0-3   softmax, GEMM2 issue, epilogue (warp w owns TMEM lanes 32w..)
//   warps 4-10  gather: bf16 KV by 16-byte cp.async, fp8 KV by register loads
//               + dequantisation, into a 2-stage ring (seven warps: a 64 KB
//               tile is issued in about half the time three warps need)
//   warp  11    TMEM allocator + GEMM1 issuer (one lane)
//   all warps gather the first two tiles; warps 0-7 run the split merge
//
// Index handling: the CTA first compacts its chunk of the index list to the
// valid entries (order preserved), so masked indices cost neither bandwidth
// nor tensor work, a fully masked chunk costs nothing, and out-of-range rows
// are never addressed. Tiles are 64 compacted rows; the last tile's tail is
// zero-filled in shared memory and masked in the softmax.
//
// Math per 64-row tile (bf16 operands, fp32 accumulation):
//   GEMM1  S[h, i]  = Q[h, :] . KV[i, :]        M=64 (heads, zero-padded),
//          N=64 (rows), K=512; A=Q and B=KV both K-major in smem; S in TMEM.
//   softmax in the log2 domain on S * (sm_scale * log2 e); P -> smem (bf16).
//   GEMM2  O^T[d, h] += KV^T[d, i] . P^T[i, h]   M=128 (d, four chunks),
//          N=NH (heads), K=64; A=KV read MN-major from the same smem tile,
//          B=P K-major; O^T accumulates in TMEM across all tiles. The four
//          d-chunks are issued interleaved so consecutive UMMAs are independent.
// UMMAs are issued in short straight-line bursts by five threads: lane 0 of
// warp 11 issues GEMM1(t) as soon as tile t's rows have landed; once P(t) is written,
// each softmax warp issues the 4 K-steps of one d-chunk of GEMM2(t). The
// tensor pipe interleaves the streams, so the GEMM2 that frees a stage never
// waits for a whole GEMM1 burst.
// The running max only moves when a head's tile max exceeds it by more than
// 2^8; then the O^T columns of the moved heads are rescaled in TMEM.
//
// Shared-memory operands use the canonical 128-byte-swizzle layout: a tile is
// stored as 64-element (128 B) column blocks; inside a block, row r sits at
// r * 128 and its 16-byte chunk c at ((c ^ (r % 8)) * 16). The KV tile serves
// GEMM1 as a K-major operand and GEMM2 as an MN-major one without re-layout.
// (A TMA tile::gather4 of the same layout was measured at ~90 cycles per
// 512-byte instruction issue on this part, well below the gather rate needed,
// so the gather uses cp.async.)
//
// Every pipeline wait is bounded in wall time; on expiry the CTA raises a
// device status bit, finishes without further waiting and releases its TMEM.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <cstdint>
#include <cstdlib>
#include <mutex>
#include <type_traits>

#include <nvtx3/nvToolsExt.h>

#include "glm53_sparse_mla.h"
#include "sm100_ptx.cuh"

namespace glm53 {

constexpr int kDim = 512;           // latent width = head size
constexpr int kRows = 64;           // KV rows per pipeline tile
constexpr int kMaxChunk = 2048;     // indices one CTA can hold after compaction
constexpr int kThreads = 384;       // 12 warps
constexpr int kProducerWarp0 = 4;   // warps 4-10 gather
constexpr int kProducerWarps = 7;
constexpr int kProducerThreads = 32 * kProducerWarps;
constexpr int kMmaWarp = 11;
constexpr int kMaxOutputs = 8;      // ranks of a head-sharded group written by one launch
constexpr int kTmemCols = 512;
constexpr uint32_t kTmemS = 256;    // S double buffer at columns 256 and 320
constexpr float kRescaleThreshold = 8.0f;   // log2 units: rescale when max grows > 256x

constexpr uint32_t kStageBytes = 65536;   // one KV tile: 64 rows x 512 bf16 (or f16)

// Shared-memory map (byte offsets from a 1024-aligned base), per padded head
// count. Q is GEMM1's M = 64 A operand, stored in 64-element column blocks
// (kQRows x 128 B each). At 32 and 64 heads it keeps all 64 rows (rows >= H
// zero). At 16 heads only its 16 rows are stored: the UMMA's rows 16-63 then
// read whatever follows (the next column blocks, the first 6 KB of KV stage
// 0), which only produces S rows of heads that do not exist and that nothing
// reads. The 48 KB this saves, with 2 KB P buffers, hold a third KV stage.
template <int NH>
struct Lay {
  static constexpr int kStages = NH == 16 ? 3 : 2;
  static constexpr uint32_t kQRows = NH == 16 ? 16 : 64;
  static constexpr uint32_t kQBlock = kQRows * 128;                // one column block of Q
  static constexpr uint32_t kSmQ = 0;
  static constexpr uint32_t kSmKV = 8 * kQBlock;                   // stages; reused by the merge
  static constexpr uint32_t kPBytes = NH == 16 ? 2048 : 8192;       // NH (<= 64) rows x 128 B
  static constexpr uint32_t kSmP = kSmKV + kStages * kStageBytes;  // 2 P buffers
  static constexpr uint32_t kSmIdx = kSmP + 2 * kPBytes;           // int32[kMaxChunk]
  static constexpr uint32_t kSmHead = kSmIdx + 4 * kMaxChunk;      // m[64] l[64] alpha[64] f[64]
  static constexpr uint32_t kSmBar = kSmHead + 4 * 64 * 4;         // mbarriers
  static constexpr uint32_t kSmMisc = kSmBar + 24 * 8;             // tmem base, counts, abort flag
  static constexpr uint32_t kSmMlRecv = kSmMisc + 64;              // m[8][64], l[8][64] of the peers
  static constexpr uint32_t kSmFlags = kSmMlRecv + 2 * 8 * 64 * 4;    // f16-overflow flag per peer
  static constexpr uint32_t kSmUsed = kSmFlags + 8 * 4;
  static constexpr uint32_t kSmemBytes = kSmUsed + 1024;           // + slack to align the base
  static_assert(kSmemBytes <= 232448, "shared memory per block");
  static_assert(kSmKV % 1024 == 0 && kSmP % 1024 == 0, "swizzle atoms need 1024-byte bases");
};

// mbarrier slots
enum : int {
  kBarKvFull = 0,    // [stages] producers -> GEMM1 issuer: stage of tile >= 2 loaded
  kBarKvEmpty = 3,   // [stages] GEMM2 (4 commits) -> producers: stage consumed
  kBarSFull = 6,     // [2] GEMM1 (commit) -> softmax: S ready
  kBarSEmpty = 8,    // [2] softmax -> GEMM1 issuer: S buffer read
  kBarODone = 10,    // GEMM2 (4 commits) -> softmax: a GEMM2 finished
  kBarDrain = 11,    // GEMM1 issuer's UMMAs all retired
  kBarQFull = 12,    // Q landed (bf16: TMA transaction count; fp8: all threads) -> GEMM1 issuer
  kBarKvFirst = 13,  // [2] all threads -> GEMM1 issuer: tile 0 / 1 loaded
  kBarG2Drain = 15,  // [4] GEMM2 issuer of softmax warp w: its UMMAs all retired
  kNumBars = 19
};

// Bound of the waits that drain this CTA's own UMMAs before TMEM is released.
// UMMAs wait on nothing once issued, so these complete in microseconds; the
// bound is fixed (not the configurable pipeline-wait limit) so that a short
// pipeline limit can never release TMEM under a UMMA still in flight.
constexpr unsigned long long kDrainTimeoutNs = 1000000000ull;

// misc words
enum : int { kMiscTmem = 0, kMiscWarpCount = 2, kMiscAbort = 10 };

struct Params {
  const __nv_bfloat16* q;   // [T, H, 512]
  const void* kv;           // [R, 512] bf16 or fp8_e4m3
  const int32_t* idx;       // [T, idx_stride], the first topk columns used
  // Paged form (block_table != nullptr): idx holds request-local token
  // positions, converted here to slots as block_table[req][pos / block_size]
  // * block_stride + pos % block_size (-1 when pos < 0 or the block is past
  // max_blocks), the conversion vLLM's index converter performs.
  const int32_t* req_id;    // [T]
  const int32_t* block_table;   // [requests, bt_stride]
  long long idx_stride;
  long long bt_stride;
  int max_blocks, block_size, block_stride;
  // Outputs: n_out buffers (1 for the plain forward; one per rank of a
  // head-sharded group, possibly on other GPUs, for the fused head gather).
  // Output i of token t, head h (h < H), element d is
  // outs[i][t * out_tok_stride + h * 512 + d]; the head offset of this rank's
  // shard is folded into the base pointers.
  __nv_bfloat16* outs[kMaxOutputs];
  int n_out;
  long long out_tok_stride;
  float* lse;               // [T, H] or nullptr
  float* ws;                // split-merge workspace (see the merge), or nullptr
  long long kv_rows;
  int T, H, topk, splits, chunk;
  float c;                  // sm_scale * log2(e)
  float kv_scale;
  unsigned long long timeout_ns;
};

__device__ unsigned int g_device_status = 0;

template <uint32_t kBlock = 8192>
__device__ __forceinline__ uint32_t swz(uint32_t row, uint32_t chunk) {
  // byte offset of 16-byte chunk `chunk` (0..63) of row `row` in a tile of
  // 64-element column blocks, each block (rows x 128 B) kBlock bytes apart
  return (chunk >> 3) * kBlock + row * 128u + (((chunk & 7u) ^ (row & 7u)) << 4);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&b);
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// fp8 KV runs the tensor-core datapath in f16: two e4m3 values (low byte
// first) -> two f16, exactly (every e4m3 value is an f16 value). kv_scale is
// applied in fp32 instead: to the softmax scale and to the output.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two) {
  const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two),
                                                    __NV_E4M3);
  return static_cast<uint32_t>(hr.x) | (static_cast<uint32_t>(hr.y) << 16);
}

// Eight e4m3 values -> one 16-byte chunk of f16.
__device__ __forceinline__ uint4 dequant8(const uint2 w) {
  return make_uint4(e4m3x2_to_f16x2(w.x & 0xFFFFu), e4m3x2_to_f16x2(w.x >> 16),
                    e4m3x2_to_f16x2(w.y & 0xFFFFu), e4m3x2_to_f16x2(w.y >> 16));
}

// Write one bf16x2 (elements d_even, d_even + 1 of head hw of token `token`)
// to every output buffer: plain stores, to peer GPUs' memory for the outputs
// of a head-sharded group.
// kMulti is a separate kernel instantiation, so the single-output kernel
// carries none of the multi-output code.
// o_tok is output 0's base for this token.
template <bool kMulti>
__device__ __forceinline__ void store_out_pair(const Params& p, __nv_bfloat16* o_tok, int token, int hw,
                                               int d_even, uint32_t pair) {
  if constexpr (!kMulti) {
    *reinterpret_cast<uint32_t*>(o_tok + static_cast<size_t>(hw) * kDim + d_even) = pair;
    return;
  }
  const size_t off = static_cast<size_t>(token) * p.out_tok_stride + static_cast<size_t>(hw) * kDim + d_even;
#pragma unroll
  for (int i = 0; i < kMaxOutputs; ++i)   // constant indices: read straight from the parameters
    if (i < p.n_out) *reinterpret_cast<uint32_t*>(p.outs[i] + off) = pair;
}

// bf16 store of out[h0 + j][d] for j < N: neighbouring lanes (d, d ^ 1) swap
// one value per head pair so each lane writes a bf16x2 of two adjacent d.
template <int N, bool kMulti>
__device__ __forceinline__ void store_pairs_n(const Params& p, __nv_bfloat16* o_tok, int token, int d, int h0,
                                              const float (&o)[N]) {
  const bool odd = threadIdx.x & 1;
  const int d_even = d & ~1;
#pragma unroll
  for (int j = 0; j < N; j += 2) {
    const float recv = __shfl_xor_sync(0xFFFFFFFFu, odd ? o[j] : o[j + 1], 1);
    const int hw = h0 + (odd ? j + 1 : j);
    const uint32_t pair = odd ? pack_bf16x2(recv, o[j + 1]) : pack_bf16x2(o[j], recv);
    if (hw < p.H) store_out_pair<kMulti>(p, o_tok, token, hw, d_even, pair);
  }
}

template <int NH, bool kFp8, bool kMulti>
__global__ void __launch_bounds__(kThreads, 1) sparse_mla_fwd_kernel(const __grid_constant__ Params p,
                                                                 const __grid_constant__ CUtensorMap q_map) {
  static_assert(NH == 16 || NH == 32 || NH == 64, "padded head count");
  using L = Lay<NH>;
  constexpr int kStages = L::kStages;
  constexpr uint32_t kSmQ = L::kSmQ, kSmKV = L::kSmKV, kSmP = L::kSmP, kPBytes = L::kPBytes;
  constexpr uint32_t kSmIdx = L::kSmIdx, kSmHead = L::kSmHead, kSmBar = L::kSmBar;
  constexpr uint32_t kSmMisc = L::kSmMisc, kSmMlRecv = L::kSmMlRecv, kSmFlags = L::kSmFlags;
  constexpr uint32_t kQRows = L::kQRows, kQBlock = L::kQBlock;
  // KV ring slot of tile t (S and P stay double-buffered: t & 1)
  auto stage_of = [](int t) -> int { return kStages == 2 ? (t & 1) : t % kStages; };
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sb = (raw + 1023u) & ~1023u;
  uint8_t* const gb = smem_raw + (sb - raw);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int split = static_cast<int>(blockIdx.x) % p.splits;
  const int token = static_cast<int>(blockIdx.x) / p.splits;
  const int nranks = p.splits;

  float* const m_sm = reinterpret_cast<float*>(gb + kSmHead);
  float* const l_sm = m_sm + 64;
  float* const alpha_sm = m_sm + 128;
  float* const f_sm = m_sm + 192;
  int32_t* const idx_sm = reinterpret_cast<int32_t*>(gb + kSmIdx);
  uint32_t* const misc = reinterpret_cast<uint32_t*>(gb + kSmMisc);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(misc + kMiscAbort);
  auto bar = [sb](int i) -> uint32_t { return sb + kSmBar + 8u * static_cast<uint32_t>(i); };

  // ------------------------------------------------------------------ setup
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(kBarKvFull + s), kProducerThreads);
      mbar_init(bar(kBarKvEmpty + s), 4);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(kBarSFull + s), 1);
      mbar_init(bar(kBarSEmpty + s), 128);
    }
    mbar_init(bar(kBarODone), 4);
    mbar_init(bar(kBarDrain), 1);
    mbar_init(bar(kBarQFull), kFp8 ? kThreads : 1);
    mbar_init(bar(kBarKvFirst), kThreads);
    mbar_init(bar(kBarKvFirst + 1), kThreads);
    for (int w = 0; w < 4; ++w) mbar_init(bar(kBarG2Drain + w), 1);
    misc[kMiscAbort] = 0;
    fence_mbarrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(sb + kSmMisc + 4 * kMiscTmem, kTmemCols);
    tmem_relinquish();
  }
  if (warp == kMmaWarp - 1 && lane == 0) {
    // L2 prefetch (a hint: it returns nothing, so it may precede the grid
    // dependency wait) of this CTA's share of q and of its index chunk
    const uint32_t qb = static_cast<uint32_t>(p.H) * kDim * 2u;
    const uint32_t qs = qb / static_cast<uint32_t>(p.splits);
    prefetch_l2_bulk(reinterpret_cast<const uint8_t*>(p.q) + static_cast<size_t>(token) * qb +
                         static_cast<size_t>(split) * qs, qs);
    const int k0p = split * p.chunk;
    const int lenp = max(0, min(p.chunk, p.topk - k0p));
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(p.idx + static_cast<size_t>(token) * p.idx_stride + k0p);
    const uintptr_t lo = (a0 + 15u) & ~uintptr_t(15), hi = (a0 + 4u * lenp) & ~uintptr_t(15);
    if (hi > lo) prefetch_l2_bulk(reinterpret_cast<const void*>(lo), static_cast<uint32_t>(hi - lo));
  }
  __syncthreads();   // barriers initialised before anyone arrives on them
  // With programmatic dependent launch the set-up above overlaps the previous
  // grid's tail; nothing global is read or written before this point.
  griddep_wait();
  // bf16: Q by TMA, 8 boxes of kQRows x 64 elements (128-byte swizzle, the
  // operand layout), rows past H zero-filled by the tensor map's bounds
  if constexpr (!kFp8) {
    if (tid == 0) {
      mbar_arrive_expect_tx(bar(kBarQFull), 8u * kQRows * 128u);
#pragma unroll
      for (int cb = 0; cb < 8; ++cb)
        asm volatile(
            "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
            "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(sb + kSmQ + cb * kQBlock),
            "l"(reinterpret_cast<uint64_t>(&q_map)), "r"(cb * 64), "r"(0), "r"(token), "r"(bar(kBarQFull))
            : "memory");
    }
  }

  // Index compaction, pass 1: warps 0-7 each take a contiguous sub-range of
  // this CTA's chunk, keep it in registers and count the valid entries.
  const int k0 = split * p.chunk;
  const int len = max(0, min(p.chunk, p.topk - k0));
  const int per_warp = ((len + 255) / 256) * 32;   // multiple of 32, <= 256
  int32_t vals[8];
  uint32_t masks[8];
  if (warp < 8) {
    const int32_t* irow = p.idx + static_cast<size_t>(token) * p.idx_stride + k0;
    const int32_t* btrow =
        p.block_table != nullptr ? p.block_table + static_cast<size_t>(p.req_id[token]) * p.bt_stride
                                 : nullptr;
    int cnt = 0;
    bool bad = false;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k = warp * per_warp + j * 32 + lane;
      int32_t v = -1;
      if (j * 32 < per_warp && k < len) v = irow[k];
      if (btrow != nullptr && v >= 0) {
        const int blk = v / p.block_size;
        long long slot = -1;
        if (blk < p.max_blocks)
          slot = static_cast<long long>(btrow[blk]) * p.block_stride + (v - blk * p.block_size);
        // a slot past the pool (kv_rows < 2^31 here) is reported below like
        // any bad index
        v = slot < 0 ? -1 : static_cast<int32_t>(slot < p.kv_rows ? slot : 0x7FFFFFFFll);
      }
      const bool valid = v >= 0 && static_cast<long long>(v) < p.kv_rows;
      bad |= (v >= 0) && !valid;
      vals[j] = v;
      masks[j] = __ballot_sync(0xFFFFFFFFu, valid);
      cnt += __popc(masks[j]);
    }
    if (lane == 0) misc[kMiscWarpCount + warp] = static_cast<uint32_t>(cnt);
    if (bad) atomicOr(&g_device_status, static_cast<unsigned>(GLM53_DEV_BAD_INDEX));
  }
  // fp8 KV (f16 datapath): Q (the kQRows stored rows of the M=64 operand; rows
  // >= H are zero) through registers, converted to f16 with one power-of-two
  // scale s_q per token that puts max |q * s_q| in [2^13, 2^14): exact for
  // every bf16 value in range, never overflowing; 1 / s_q is folded into the
  // softmax scale. Issued after the index loads so those are not queued
  // behind it.
  constexpr int kQPer = (kQRows * 64 + kThreads - 1) / kThreads;
  uint4 qv[kFp8 ? kQPer : 1];
  float s_q = 1.f;
  if constexpr (kFp8) {
    const __nv_bfloat16* qtok = p.q + static_cast<size_t>(token) * p.H * kDim;
    float qmax = 0.f;
#pragma unroll
    for (int i = 0; i < kQPer; ++i) {
      const int u = tid + i * kThreads;
      const int h = u >> 6, c = u & 63;
      qv[i] = (u < kQRows * 64 && h < p.H) ? ldg_nc_v4(qtok + h * kDim + c * 8) : make_uint4(0u, 0u, 0u, 0u);
      const uint32_t w4[4] = {qv[i].x, qv[i].y, qv[i].z, qv[i].w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w4[k]));
        qmax = fmaxf(qmax, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
#pragma unroll
    for (int k = 16; k >= 1; k >>= 1) qmax = fmaxf(qmax, __shfl_xor_sync(0xFFFFFFFFu, qmax, k));
    if (lane == 0) alpha_sm[warp] = qmax;   // alpha_sm is free until the softmax
  }
  __syncthreads();
  if constexpr (kFp8) {
    float qmax = 0.f;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) qmax = fmaxf(qmax, alpha_sm[w]);
    int ex = 0;
    frexpf(qmax, &ex);
    s_q = qmax > 0.f ? ldexpf(1.f, 14 - min(max(ex, -100), 100)) : 1.f;
#pragma unroll
    for (int i = 0; i < kQPer; ++i) {
      const int u = tid + i * kThreads;
      if (u < kQRows * 64) {
        const uint32_t w4[4] = {qv[i].x, qv[i].y, qv[i].z, qv[i].w};
        uint32_t o4[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w4[k]));
          o4[k] = pack_f16x2(f.x * s_q, f.y * s_q);
        }
        sts_v4(sb + kSmQ + swz<kQBlock>(u >> 6, u & 63), make_uint4(o4[0], o4[1], o4[2], o4[3]));
      }
    }
    fence_proxy_async_smem();
    mbar_arrive(bar(kBarQFull));
  }
  // fp8 KV: the tensor cores see e4m3 values and q * s_q; the softmax scale
  // and the final normalisation take kv_scale and 1 / s_q back.
  const float kvs = kFp8 ? p.kv_scale : 1.f;
  const float c_soft = p.c * kvs / s_q;

  // pass 2: scatter the valid entries to their compacted positions
  int n_valid = 0, base = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const int c = static_cast<int>(misc[kMiscWarpCount + w]);
    if (w < warp) base += c;
    n_valid += c;
  }
  if (warp < 8) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t m = masks[j];
      if (m & (1u << lane)) idx_sm[base + __popc(m & ((1u << lane) - 1u))] = vals[j];
      base += __popc(m);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[kMiscTmem];
  const int n_tiles = (n_valid + kRows - 1) / kRows;

  // UMMA steps. GEMM1 of tile t is 32 K-steps into S[t & 1]; GEMM2 of tile t
  // is 4 K-steps x 4 d-chunks into O^T, chunks innermost so consecutive UMMAs
  // are independent.
  constexpr uint32_t kIdesc1 = kFp8 ? idesc_f16_f32(64, 64, false, false)
                                    : idesc_bf16_f32(64, 64, false, false);
  constexpr uint32_t kIdesc2 = kFp8 ? idesc_f16_f32(128, NH, true, false)
                                    : idesc_bf16_f32(128, NH, true, false);
  constexpr int kSteps1 = kDim / 16;          // 32
  auto gemm1_step = [=](int t, int kk) {
    const uint32_t stage = sb + kSmKV + stage_of(t) * kStageBytes;
    const uint32_t off = (kk >> 2) * 8192u + (kk & 3) * 32u;
    const uint32_t qoff = (kk >> 2) * kQBlock + (kk & 3) * 32u;
    umma_bf16(tmem + kTmemS + 64u * (t & 1), sdesc_sw128(sb + kSmQ + qoff, 16, 1024),
              sdesc_sw128(stage + off, 16, 1024), kIdesc1, kk > 0 ? 1u : 0u);
  };
  auto gemm2_step = [=](int t, int i) {
    const int kk = i >> 2, m = i & 3;
    const uint32_t stage = sb + kSmKV + stage_of(t) * kStageBytes;
    const uint32_t pbuf = sb + kSmP + (t & 1) * kPBytes;
    umma_bf16(tmem + static_cast<uint32_t>(m * NH),
              sdesc_sw128(stage + m * 16384u + kk * 2048u, 8192, 1024),
              sdesc_sw128(pbuf + kk * 32u, 16, 1024), kIdesc2, (t > 0 || kk > 0) ? 1u : 0u);
  };

  // Gather rows r = r0, r0 + step, ... of tile t into its stage: bf16 rows by
  // 16-byte cp.async per lane (half a row per warp instruction; the last
  // tile's missing rows are zero-filled through src-size 0), fp8 rows by
  // 8-byte register loads, e4m3 -> f16 in registers and swizzled 16-byte
  // shared stores. Then arrive on `full`: bf16 through the
  // deferred cp.async arrive (fires once this thread's copies have landed),
  // fp8 after a proxy fence.
  auto gather_rows = [&](int t, int r0, auto step_c, uint32_t full) {
    constexpr int kStep = decltype(step_c)::value;
    const uint32_t stage = sb + kSmKV + stage_of(t) * kStageBytes;
    const int rows = min(kRows, n_valid - kRows * t);
    if constexpr (!kFp8) {
      const uint8_t* kvb = static_cast<const uint8_t*>(p.kv);
#pragma unroll 4
      for (int r = r0; r < kRows; r += kStep) {
        const bool valid = r < rows;
        const long long row = valid ? idx_sm[kRows * t + r] : 0;
        const uint8_t* src = kvb + row * (kDim * 2);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int c = lane + 32 * hh;
          cp_async_16(stage + swz(r, c), src + c * 16, valid ? 16u : 0u);
        }
      }
      cp_async_mbar_arrive_noinc(full);
    } else {
      // lane l owns bf16 chunks l and l + 32 of each row (fp8 bytes 8l and
      // 256 + 8l): a warp's loads cover 256 contiguous bytes and a
      // quarter-warp's swizzled 16-byte stores hit 8 distinct bank groups
      const uint8_t* kv8 = static_cast<const uint8_t*>(p.kv);
      constexpr int kPer = (kRows + kStep - 1) / kStep;
      uint2 buf[kPer][2];
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int r = r0 + kStep * j;
        if (r < rows) {
          const uint8_t* src = kv8 + static_cast<long long>(idx_sm[kRows * t + r]) * kDim + lane * 8;
          buf[j][0] = ldg_nc_v2(src);
          buf[j][1] = ldg_nc_v2(src + 256);
        } else {
          buf[j][0] = buf[j][1] = make_uint2(0u, 0u);
        }
      }
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int r = r0 + kStep * j;
        if (r < kRows) {
          sts_v4(stage + swz(r, lane), dequant8(buf[j][0]));
          sts_v4(stage + swz(r, lane + 32), dequant8(buf[j][1]));
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(full);
    }
  };

  // Both stages are empty at the start: every warp gathers tiles 0 and 1
  // (each warp a row in 8), which brings the first GEMM1 forward.
  for (int t = 0; t < min(2, n_tiles); ++t)
    gather_rows(t, warp, std::integral_constant<int, kThreads / 32>{}, bar(kBarKvFirst + t));

  // ------------------------------------------------------------------ roles
  if (warp >= kProducerWarp0 && warp < kMmaWarp) {
    // ================= gather (tiles 2, 3, ...) =================
    // bf16: cp.async into the stage once it is free (gather_rows); its writes
    // land spread out as the data arrives.
    // fp8: register-staged with one tile of prefetch: the rows of tile t + 1
    // are loaded right after tile t is stored, so their DRAM latency runs
    // while the stage they go to is still being consumed, and converted to
    // f16 at store time. (Staging bf16 the same way measured slower:
    // its 64 KB burst of shared stores stalls the tensor core's operand reads.)
    // Lane l owns the 16-byte chunks l and l + 32 of each of its rows: a
    // warp's loads cover 256 contiguous bytes and a quarter-warp's swizzled
    // stores hit 8 distinct bank groups.
    const int pw = warp - kProducerWarp0;
    constexpr int kPer = (kRows + kProducerWarps - 1) / kProducerWarps;
    using Chunk = typename std::conditional<kFp8, uint2, uint4>::type;
    Chunk buf[kPer][2];   // only the fp8 path uses it
    auto load_tile = [&](int t) {
      const int rows = min(kRows, n_valid - kRows * t);
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int r = pw + kProducerWarps * j;
        if (r < rows) {
          const long long row = idx_sm[kRows * t + r];
          if constexpr (kFp8) {
            const uint8_t* src = static_cast<const uint8_t*>(p.kv) + row * kDim + lane * 8;
            buf[j][0] = ldg_nc_v2(src);
            buf[j][1] = ldg_nc_v2(src + 256);
          } else {
            const uint8_t* src = static_cast<const uint8_t*>(p.kv) + row * (2 * kDim) + lane * 16;
            buf[j][0] = ldg_nc_v4(src);
            buf[j][1] = ldg_nc_v4(src + 512);
          }
        } else {
          if constexpr (kFp8) {
            buf[j][0] = buf[j][1] = make_uint2(0u, 0u);
          } else {
            buf[j][0] = buf[j][1] = make_uint4(0u, 0u, 0u, 0u);
          }
        }
      }
    };
    auto store_tile = [&](int t) {
      const uint32_t stage = sb + kSmKV + stage_of(t) * kStageBytes;
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int r = pw + kProducerWarps * j;
        if (r < kRows) {
          if constexpr (kFp8) {
            sts_v4(stage + swz(r, lane), dequant8(buf[j][0]));
            sts_v4(stage + swz(r, lane + 32), dequant8(buf[j][1]));
          } else {
            sts_v4(stage + swz(r, lane), buf[j][0]);
            sts_v4(stage + swz(r, lane + 32), buf[j][1]);
          }
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(bar(kBarKvFull + stage_of(t)));
    };
    if constexpr (kFp8) {
      if (n_tiles > 2) load_tile(2);
      for (int t = 2; t < n_tiles; ++t) {
        // a stage's first tile (t < kStages) needs no wait
        if (t >= kStages && !mbar_wait_bounded(bar(kBarKvEmpty + stage_of(t)), ((t / kStages) - 1) & 1,
                                               abort_flag, p.timeout_ns))
          break;
        store_tile(t);
        if (t + 1 < n_tiles) load_tile(t + 1);
      }
    } else {
      // The rows of tile t + 1 are prefetched into L2 (one 1 KB bulk prefetch
      // per row) as soon as tile t is issued, so when their stage frees the
      // cp.async is served from L2 instead of waiting out DRAM latency.
      const uint8_t* kvb = static_cast<const uint8_t*>(p.kv);
      const int pt = tid - 32 * kProducerWarp0;   // 0 .. kProducerThreads - 1
      auto prefetch_tile = [&](int t) {
        const int rows = min(kRows, n_valid - kRows * t);
        if (pt < rows) prefetch_l2_bulk(kvb + static_cast<long long>(idx_sm[kRows * t + pt]) * (2 * kDim), 2 * kDim);
      };
      if (n_tiles > 2) prefetch_tile(2);
      for (int t = 2; t < n_tiles; ++t) {
        if (t >= kStages && !mbar_wait_bounded(bar(kBarKvEmpty + stage_of(t)), ((t / kStages) - 1) & 1,
                                               abort_flag, p.timeout_ns))
          break;
        gather_rows(t, pw, std::integral_constant<int, kProducerWarps>{}, bar(kBarKvFull + stage_of(t)));
        if (t + 1 < n_tiles) prefetch_tile(t + 1);
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ================= GEMM1 issue =================
    // One straight-line burst of 32 UMMAs per tile. Waits sit only between
    // bursts: a data-dependent branch inside a burst stalls the issuing
    // thread for hundreds of cycles per UMMA.
    if (lane == 0) {
      bool ok = n_tiles == 0 || mbar_wait_bounded(bar(kBarQFull), 0, abort_flag, p.timeout_ns);
      for (int g1 = 0; ok && g1 < n_tiles; ++g1) {
        // tiles 0 and 1 arrive on kBarKvFirst, so KvFull of stages 0 and 1
        // completes first for tile kStages and kStages + 1
        const int use = g1 / kStages - (stage_of(g1) < 2 ? 1 : 0);
        ok = (g1 < 2 ? mbar_wait_bounded(bar(kBarKvFirst + g1), 0, abort_flag, p.timeout_ns)
                     : mbar_wait_bounded(bar(kBarKvFull + stage_of(g1)), use & 1, abort_flag,
                                         p.timeout_ns)) &&
             (g1 < 2 ||
              mbar_wait_bounded(bar(kBarSEmpty + (g1 & 1)), ((g1 >> 1) - 1) & 1, abort_flag, p.timeout_ns));
        if (!ok) break;
        fence_proxy_async_smem();   // generic-proxy / cp.async smem writes -> tensor-core reads
        tc_fence_after();
#pragma unroll
        for (int i = 0; i < kSteps1; ++i) gemm1_step(g1, i);
        umma_commit(bar(kBarSFull + (g1 & 1)));
      }
      // Drain: never release TMEM while a UMMA may still write it.
      umma_commit(bar(kBarDrain));
      int no_abort = 0;
      mbar_wait_bounded(bar(kBarDrain), 0, &no_abort, kDrainTimeoutNs);
    }
    __syncwarp();
  } else if (warp < 4) {
    // ================= softmax (warps 0-3) =================
    const int q4 = warp;                       // TMEM lane quadrant
    const int h = 16 * q4 + (lane & 15);       // head owned (M=64 layout)
    const int half = lane >> 4;                // which 32 of the 64 tile rows
    const bool has_head = (16 * q4) < NH;      // warp-uniform
    const uint32_t lane_base = static_cast<uint32_t>(32 * q4) << 16;
    float m_used = -INFINITY;   // running max, log2 units (score * c)
    float l_part = 0.f;         // this thread's share of the running sum

    for (int t = 0; t < n_tiles; ++t) {
      const int b = t & 1;
      // A failed wait leaves the loop running on garbage with every barrier
      // still taken, so no thread of the group can strand the others.
      mbar_wait_bounded(bar(kBarSFull + b), (t >> 1) & 1, abort_flag, p.timeout_ns);
      tc_fence_after();
      float v[32];
      if (has_head) {
        tmem_ld_16x32bx2_x32(tmem + lane_base + kTmemS + 64u * b, v);
        tmem_wait_ld();
      }
      tc_fence_before();
      mbar_arrive(bar(kBarSEmpty + b));

      const int rows = min(kRows, n_valid - kRows * t);
      float mx = -INFINITY;
      if (has_head) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const bool valid = 32 * half + j < rows;
          v[j] = valid ? v[j] * c_soft : -INFINITY;
          mx = fmaxf(mx, v[j]);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, 16));
      const bool need = has_head && (mx > m_used + kRescaleThreshold);
      const float new_m = need ? mx : m_used;
      const float alpha = need ? exp2f(m_used - new_m) : 1.f;

      __syncwarp();
      if (named_bar_or(1, 128, need && t > 0)) {
        if (has_head && half == 0) alpha_sm[h] = alpha;
        named_bar_sync(1, 128);
        // O^T must hold GEMM2(t-1) in full before it is rescaled.
        mbar_wait_bounded(bar(kBarODone), (t - 1) & 1, abort_flag, p.timeout_ns);
        tc_fence_after();
        // 16 columns at a time: the S values of this tile stay live here
#pragma unroll 1
        for (int m = 0; m < 4; ++m) {
#pragma unroll
          for (int cc = 0; cc < NH / 16; ++cc) {
            float o[16];
            const uint32_t ta = tmem + lane_base + static_cast<uint32_t>(m * NH + 16 * cc);
            tmem_ld_32x32b_x16(ta, o);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) o[j] *= alpha_sm[16 * cc + j];
            tmem_st_32x32b_x16(ta, o);
          }
        }
        tmem_wait_st();
      }
      l_part *= alpha;
      m_used = new_m;

      if (has_head) {
        uint32_t packed[16];
        float ps = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float p0 = exp2f(v[2 * j] - m_used);
          const float p1 = exp2f(v[2 * j + 1] - m_used);
          ps += p0 + p1;
          packed[j] = kFp8 ? pack_f16x2(p0, p1) : pack_bf16x2(p0, p1);
        }
        l_part += ps;
        const uint32_t prow = sb + kSmP + b * kPBytes + static_cast<uint32_t>(h) * 128u;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const uint32_t c = static_cast<uint32_t>(4 * half + k);
          sts_v4(prow + ((c ^ (static_cast<uint32_t>(h) & 7u)) << 4),
                 make_uint4(packed[4 * k], packed[4 * k + 1], packed[4 * k + 2], packed[4 * k + 3]));
        }
        fence_proxy_async_smem();
      }
      // GEMM2(t) right away: once every P row is written (and O rescaled),
      // lane 0 of each softmax warp issues the 4 K-steps of d-chunk `warp`.
      tc_fence_before();
      named_bar_sync(2, 128);
      if (lane == 0) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) gemm2_step(t, 4 * kk + warp);
        umma_commit(bar(kBarKvEmpty + stage_of(t)));
        umma_commit(bar(kBarODone));
      }
      __syncwarp();
    }

    // Each GEMM2 issuer retires its own UMMAs before anything may release
    // TMEM. The merge's waits on kBarODone cover this when no wait timed out;
    // after a timeout they return at once, and this drain is what keeps TMEM
    // allocated until the last GEMM2 has written it.
    if (lane == 0 && n_tiles > 0) {
      umma_commit(bar(kBarG2Drain + warp));
      int no_abort = 0;
      mbar_wait_bounded(bar(kBarG2Drain + warp), 0, &no_abort, kDrainTimeoutNs);
    }
    // publish this CTA's per-head max and sum for the merge
    __syncwarp();
    const float l_tot = l_part + __shfl_xor_sync(0xFFFFFFFFu, l_part, 16);
    if (has_head && half == 0) {
      m_sm[h] = n_tiles > 0 ? m_used : -INFINITY;
      l_sm[h] = n_tiles > 0 ? l_tot : 0.f;
      f_sm[h] = (n_tiles > 0 && l_tot > 0.f) ? 1.f / l_tot : 0.f;   // the f16 split-merge partials' scale
    }
  }

  // ------------------------------------------------------------------ merge
  // Every CTA of this grid is resident by now, so the next grid in the stream
  // may start launching (its CTAs wait in griddep_wait for this one to end).
  griddep_launch_dependents();
  __nv_bfloat16* const o_tok = p.outs[0] + static_cast<size_t>(token) * p.out_tok_stride;
  const uint32_t lane_base = static_cast<uint32_t>(32 * (warp & 3)) << 16;
  const bool odd = lane & 1;

  // O^T[d][0..NH) of TMEM lane d of chunk m (all loads issued, one wait)
  auto load_o = [=](int m, float (&o)[NH]) {
    if constexpr (NH == 16) {
      tmem_ld_32x32b_x16(tmem + lane_base + static_cast<uint32_t>(m * NH), o);
      tmem_wait_ld();
    } else {
#pragma unroll
      for (int cc = 0; cc < NH / 32; ++cc) {
        float o32[32];
        tmem_ld_32x32b_x32(tmem + lane_base + static_cast<uint32_t>(m * NH + 32 * cc), o32);
#pragma unroll
        for (int j = 0; j < 32; ++j) o[32 * cc + j] = o32[j];
      }
      tmem_wait_ld();
    }
  };
  // bf16 store of out[h][d] for all heads of this lane's d: neighbouring lanes
  // swap one value per head pair so each lane writes a bf16x2 of two d
  auto store_pairs = [=](int d, const float (&o)[NH]) {
    const int d_even = d & ~1;
#pragma unroll
    for (int j = 0; j < NH; j += 2) {
      const float recv = __shfl_xor_sync(0xFFFFFFFFu, odd ? o[j] : o[j + 1], 1);
      const int hw = odd ? j + 1 : j;
      const uint32_t pair = odd ? pack_bf16x2(recv, o[j + 1]) : pack_bf16x2(o[j], recv);
      if (hw < p.H) store_out_pair<kMulti>(p, o_tok, token, hw, d_even, pair);
    }
  };

  if (nranks > 1 && p.ws != nullptr) {
    // ---- split across 2, 4 or 8 CTAs, merged through a global workspace
    // (it stays in L2). Each CTA owns a d-slice of the output. All 8 warps
    // work: warp w reads TMEM lane quadrant w & 3 and head half w >> 2 (at
    // NH = 16, warps 0-3 take all heads). Per-head (max, sum) pairs go to
    // every peer's shared memory (a few hundred bytes); the partials go to
    // the workspace, per (token, CTA) one slice per destination CTA. Every
    // slice is written before a cluster barrier and read after it, so the
    // workspace needs no initialisation.
    //
    // At 32 and 64 heads a partial is sent as f16 of this CTA's own
    // normalised output O / l (laid out [NH / 8][dspan][8], a warp's 16-byte
    // stores and loads cover 512 contiguous bytes): half the bytes of fp32,
    // and O / l is a convex combination of the gathered rows, so it fits
    // f16's range unless the cache itself holds values beyond it. A CTA that
    // meets such a value (or a non-finite one) raises a flag beside its
    // (max, sum); if any CTA of the cluster did, all of them resend their
    // unnormalised fp32 partials ([NH / 4][dspan][4] floats) behind a second
    // barrier. At 16 heads (a quarter of the bytes) the partials are always
    // fp32: there the flag's extra block barrier costs more than it saves.
    constexpr bool kF16Part = NH >= 32;
    constexpr int kHalf = NH >= 32 ? NH / 2 : NH;
    constexpr int kV = kHalf / 4;                   // float4 per (d, peer)
    const int dspan = kDim / nranks;
    const size_t blk = static_cast<size_t>(NH) * kDim;   // floats per (token, CTA)
    float* const ws_tok = p.ws + static_cast<size_t>(token) * nranks * blk;
    const int qd = warp & 3;
    const bool active = warp < (NH >= 32 ? 8 : 4);
    const int h0 = NH >= 32 ? (warp >> 2) * kHalf : 0;
    const uint32_t tcol = static_cast<uint32_t>(32 * qd) << 16;
    float* const scal = reinterpret_cast<float*>(gb + kSmIdx);   // e[8][NH], 1/L[NH]
    const float* const ml = reinterpret_cast<const float*>(gb + kSmMlRecv);   // m[8][64], l[8][64]
    const float* const flags = reinterpret_cast<const float*>(gb + kSmFlags);   // [8]
    auto load_half = [=](int m, float (&o)[kHalf]) {
      const uint32_t ta = tmem + tcol + static_cast<uint32_t>(m * NH + h0);
      if constexpr (kHalf == 32) {
        tmem_ld_32x32b_x32(ta, o);
      } else {
        tmem_ld_32x32b_x16(ta, o);
      }
      tmem_wait_ld();
    };
    // This CTA's partials for every other CTA's d-slice: f16 of O / l (returns
    // whether a value left f16's finite range) or fp32 O.
    auto send_partials = [&](auto f16_c) -> bool {
      constexpr bool kF16 = decltype(f16_c)::value;
      bool ovf = false;
      if (!active) return ovf;
#pragma unroll 1
      for (int m = 0; m < 4; ++m) {
        const int d = 128 * m + 32 * qd + lane;
        const int owner = d / dspan;               // warp-uniform (dspan >= 64)
        if (owner == split) continue;
        float o[kHalf];
        load_half(m, o);
        if (n_tiles == 0) {
#pragma unroll
          for (int j = 0; j < kHalf; ++j) o[j] = 0.f;
        }
        const int dl = d - owner * dspan;
        if constexpr (kF16) {
          __half* const dst = reinterpret_cast<__half*>(ws_tok + static_cast<size_t>(split) * blk) +
                              static_cast<size_t>(owner) * NH * dspan;
#pragma unroll
          for (int c = 0; c < kHalf / 8; ++c) {
            uint32_t w[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float a = o[8 * c + 2 * k] * f_sm[h0 + 8 * c + 2 * k];
              const float b = o[8 * c + 2 * k + 1] * f_sm[h0 + 8 * c + 2 * k + 1];
              ovf |= !(fabsf(a) <= 65504.f) || !(fabsf(b) <= 65504.f);
              w[k] = pack_f16x2(a, b);
            }
            stg_cg_v4u(dst + (static_cast<size_t>(h0 / 8 + c) * dspan + dl) * 8, make_uint4(w[0], w[1], w[2], w[3]));
          }
        } else {
          float* const dst = ws_tok + static_cast<size_t>(split) * blk + static_cast<size_t>(owner) * NH * dspan;
#pragma unroll
          for (int c = 0; c < kV; ++c)
            stg_cg_f4(dst + (static_cast<size_t>(h0 / 4 + c) * dspan + dl) * 4,
                      make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]));
        }
      }
      return ovf;
    };

    if (n_tiles > 0) mbar_wait_bounded(bar(kBarODone), (n_tiles - 1) & 1, abort_flag, p.timeout_ns);
    __syncthreads();   // every role past its main loop; m_sm / l_sm written
    tc_fence_after();
    if (tid < NH) {
      const float mv = m_sm[tid], lv = l_sm[tid];
      for (int q = 0; q < nranks; ++q) {
        const uint32_t a = sb + kSmMlRecv + 4u * static_cast<uint32_t>(split * 64 + tid);
        st_dsmem_f32(mapa_shared(a, q), mv);
        st_dsmem_f32(mapa_shared(a + 4u * 8u * 64u, q), lv);
      }
    }
    bool wide = !kF16Part;   // fp32 partials; cluster-uniform
    if constexpr (kF16Part) {
      const bool ovf = __syncthreads_or(send_partials(std::true_type{}));
      if (tid < nranks)
        st_dsmem_f32(mapa_shared(sb + kSmFlags + 4u * static_cast<uint32_t>(split), tid), ovf ? 1.f : 0.f);
      __threadfence();
      cluster_sync_all();   // every CTA's (max, sum), flag and f16 partials visible
      for (int r = 0; r < nranks; ++r) wide |= flags[r] != 0.f;   // every CTA reads the same flags
    }
    if (wide) {
      send_partials(std::false_type{});
      __threadfence();
      cluster_sync_all();   // every CTA's (max, sum) and fp32 partials visible
    }
    if (tid < NH) {
      // every rank's (max, sum) loaded at once (unrolled over the largest
      // cluster), then combined
      float mr[8], lr[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        mr[r] = r < nranks ? ml[r * 64 + tid] : 0.f;
        lr[r] = r < nranks ? ml[512 + r * 64 + tid] : 0.f;
      }
      float M = -INFINITY;
#pragma unroll
      for (int r = 0; r < 8; ++r)
        if (lr[r] > 0.f) M = fmaxf(M, mr[r]);
      float L = 0.f;
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const float e = lr[r] > 0.f ? exp2f(mr[r] - M) : 0.f;
        // a peer's f16 partial is O / l, its fp32 partial and this CTA's TMEM are O
        if (r < nranks) scal[r * NH + tid] = (!wide && r != split) ? e * lr[r] : e;
        L += lr[r] * e;
      }
      scal[8 * NH + tid] = L > 0.f ? kvs / L : 0.f;
      if (split == 0 && p.lse != nullptr && tid < p.H)
        p.lse[static_cast<size_t>(token) * p.H + tid] = L > 0.f ? log2f(L) + M : -INFINITY;
    }
    __syncthreads();
    if (active) {
#pragma unroll 1
      for (int m = 0; m < 4; ++m) {
        const int d = 128 * m + 32 * qd + lane;
        if (d / dspan != split) continue;          // warp-uniform
        const int dl = d - split * dspan;
        // 16 heads per pass keeps a pass's peer loads in registers
#pragma unroll 1
        for (int hp = 0; hp < kHalf; hp += 16) {
          const int hb = h0 + hp;
          float o[16];
          tmem_ld_32x32b_x16(tmem + tcol + static_cast<uint32_t>(m * NH + hb), o);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] = n_tiles > 0 ? o[j] * scal[split * NH + hb + j] : 0.f;
          if (!wide) {
            const __half* const src0 = reinterpret_cast<const __half*>(ws_tok) + static_cast<size_t>(split) * NH * dspan +
                                       static_cast<size_t>(hb / 8) * dspan * 8 + dl * 8;
            // peers in batches of three, each batch's loads issued together
#pragma unroll 1
            for (int i0 = 0; i0 < nranks - 1; i0 += 3) {
              uint4 v[3][2];
#pragma unroll
              for (int i = 0; i < 3; ++i) {
                const int r = i0 + i < split ? i0 + i : i0 + i + 1;
                if (i0 + i < nranks - 1) {
#pragma unroll
                  for (int c = 0; c < 2; ++c)
                    v[i][c] = ldg_cg_v4u(src0 + static_cast<size_t>(r) * blk * 2 + static_cast<size_t>(c) * dspan * 8);
                }
              }
#pragma unroll
              for (int i = 0; i < 3; ++i) {
                const int r = i0 + i < split ? i0 + i : i0 + i + 1;
                if (i0 + i < nranks - 1) {
                  const float* e = scal + r * NH + hb;
#pragma unroll
                  for (int c = 0; c < 2; ++c) {
                    const uint32_t w[4] = {v[i][c].x, v[i][c].y, v[i][c].z, v[i][c].w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
                      o[8 * c + 2 * k] += f.x * e[8 * c + 2 * k];
                      o[8 * c + 2 * k + 1] += f.y * e[8 * c + 2 * k + 1];
                    }
                  }
                }
              }
            }
          } else {
            const float* const src0 = ws_tok + static_cast<size_t>(split) * NH * dspan +
                                      static_cast<size_t>(hb / 4) * dspan * 4 + dl * 4;
#pragma unroll 1
            for (int i0 = 0; i0 < nranks - 1; i0 += 3) {
              float4 v[3][4];
#pragma unroll
              for (int i = 0; i < 3; ++i) {
                const int r = i0 + i < split ? i0 + i : i0 + i + 1;
                if (i0 + i < nranks - 1) {
#pragma unroll
                  for (int c = 0; c < 4; ++c)
                    v[i][c] = ldg_cg_f4(src0 + static_cast<size_t>(r) * blk + static_cast<size_t>(c) * dspan * 4);
                }
              }
#pragma unroll
              for (int i = 0; i < 3; ++i) {
                const int r = i0 + i < split ? i0 + i : i0 + i + 1;
                if (i0 + i < nranks - 1) {
                  const float* e = scal + r * NH + hb;
#pragma unroll
                  for (int c = 0; c < 4; ++c) {
                    o[4 * c] += v[i][c].x * e[4 * c];
                    o[4 * c + 1] += v[i][c].y * e[4 * c + 1];
                    o[4 * c + 2] += v[i][c].z * e[4 * c + 2];
                    o[4 * c + 3] += v[i][c].w * e[4 * c + 3];
                  }
                }
              }
            }
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] *= scal[8 * NH + hb + j];
          store_pairs_n<16, kMulti>(p, o_tok, token, d, hb, o);
        }
      }
    }
    tc_fence_before();
    __syncthreads();
  } else if (nranks == 1) {
    // ---- single CTA per token: normalise and store straight from TMEM
    __syncthreads();
    if (warp < 4) {
      if (tid < NH) {
        const float L = l_sm[tid];
        f_sm[tid] = L > 0.f ? kvs / L : 0.f;
        if (p.lse != nullptr && tid < p.H)
          p.lse[static_cast<size_t>(token) * p.H + tid] = L > 0.f ? log2f(L) + m_sm[tid] : -INFINITY;
      }
      named_bar_sync(1, 128);
      if (n_tiles > 0)
        mbar_wait_bounded(bar(kBarODone), (n_tiles - 1) & 1, abort_flag, p.timeout_ns);
      tc_fence_after();
#pragma unroll 1
      for (int m = 0; m < 4; ++m) {
        float o[NH];
        load_o(m, o);
#pragma unroll
        for (int j = 0; j < NH; ++j) o[j] = n_tiles > 0 ? o[j] * f_sm[j] : 0.f;
        store_pairs(128 * m + 32 * warp + lane, o);
      }
      tc_fence_before();
    }
    __syncthreads();
  } else if (nranks <= 4) {
    // ---- split across 2 or 4 CTAs: each CTA owns a d-slice of the output.
    // After a cluster barrier (every CTA past its main loop, so receive
    // buffers are free), each CTA stores, into every peer's receive slot, its
    // per-head (max, sum) and its unscaled partial for that peer's slice; a
    // second barrier publishes the stores and each owner combines them with
    // its own partial, read straight from TMEM. Slot layout: m[NH], l[NH],
    // then one row of NH floats per d of the slice, its 16-byte chunks XOR-
    // swizzled by the row index (within groups of up to 8 chunks) so a warp
    // reading 32 consecutive rows spreads over all banks.
    const int dspan = kDim / nranks;                                 // 256 or 128
    const uint32_t slot_bytes = 4u * (2u * NH + static_cast<uint32_t>(NH * dspan));
    const uint32_t recv_base = sb;                                   // (nranks-1) slots
    float* const scal = reinterpret_cast<float*>(gb + kSmIdx);       // e[4][NH], 1/L[NH]
    constexpr int kSw = NH / 4 < 8 ? NH / 4 : 8;   // chunks per swizzle group (row = NH/4 chunks)
    auto row_chunk = [](int row, int c) { return (c & ~(kSw - 1)) | ((c ^ row) & (kSw - 1)); };
    // The receive slots overlay Q and the first KV stage, which this CTA's
    // last GEMM2 may still be reading: retire it before peers may write.
    if (warp < 4 && n_tiles > 0)
      mbar_wait_bounded(bar(kBarODone), (n_tiles - 1) & 1, abort_flag, p.timeout_ns);
    cluster_sync_all();   // every CTA is past its main loop, its UMMAs retired
    if (warp < 4) {
      tc_fence_after();
      if (tid < NH) {
        for (int q = 0; q < nranks; ++q) {
          if (q == split) continue;
          const uint32_t rslot = recv_base + (split < q ? split : split - 1) * slot_bytes;
          st_dsmem_f32(mapa_shared(rslot + 4u * tid, q), m_sm[tid]);
          st_dsmem_f32(mapa_shared(rslot + 4u * (NH + tid), q), l_sm[tid]);
        }
      }
#pragma unroll 1
      for (int m = 0; m < 4; ++m) {
        const int d = 128 * m + 32 * warp + lane;
        const int owner = d / dspan;
        if (owner == split) continue;            // own slice stays in TMEM
        float o[NH];
        if (n_tiles > 0) {
          load_o(m, o);
        } else {
#pragma unroll
          for (int j = 0; j < NH; ++j) o[j] = 0.f;
        }
        const int dl = d - owner * dspan;
        const uint32_t row = mapa_shared(recv_base + (split < owner ? split : split - 1) * slot_bytes +
                                             4u * (2 * NH + dl * NH), owner);
#pragma unroll
        for (int c = 0; c < NH / 4; ++c)
          st_dsmem_v4(row + 16u * row_chunk(dl, c),
                      make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]));
      }
      tc_fence_before();
    }
    cluster_sync_all();   // every peer's stores into this CTA are visible
    if (warp < 4) {
      if (tid < NH) {
        // ranks in order; own (max, sum) from local smem, others from slots
        float mr[4], lr[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          if (r < nranks) {
            if (r == split) {
              mr[r] = m_sm[tid];
              lr[r] = l_sm[tid];
            } else {
              const float* slot = reinterpret_cast<const float*>(gb + (r < split ? r : r - 1) * slot_bytes);
              mr[r] = slot[tid];
              lr[r] = slot[NH + tid];
            }
          }
        }
        float M = -INFINITY;
#pragma unroll
        for (int r = 0; r < 4; ++r)
          if (r < nranks && lr[r] > 0.f) M = fmaxf(M, mr[r]);
        float L = 0.f, e[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          e[r] = (r < nranks && lr[r] > 0.f) ? exp2f(mr[r] - M) : 0.f;
          if (r < nranks) L += lr[r] * e[r];
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) scal[r * NH + tid] = e[r];
        scal[4 * NH + tid] = L > 0.f ? kvs / L : 0.f;
        if (split == 0 && p.lse != nullptr && tid < p.H)
          p.lse[static_cast<size_t>(token) * p.H + tid] = L > 0.f ? log2f(L) + M : -INFINITY;
      }
      named_bar_sync(1, 128);
#pragma unroll 1
      for (int mm = 0; mm < 4 / nranks; ++mm) {
        const int m = split * (4 / nranks) + mm;
        const int d = 128 * m + 32 * warp + lane;
        const int dl = d - split * dspan;
#pragma unroll 1
        for (int hb = 0; hb < NH; hb += 16) {   // 16 heads at a time
          float o[16];
          if (n_tiles > 0) {
            tmem_ld_32x32b_x16(tmem + lane_base + static_cast<uint32_t>(m * NH + hb), o);
            tmem_wait_ld();
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) o[j] = 0.f;
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] *= scal[split * NH + hb + j];
          for (int r = 0; r < nranks; ++r) {
            if (r == split) continue;
            const float4* row = reinterpret_cast<const float4*>(
                gb + (r < split ? r : r - 1) * slot_bytes + 4u * (2 * NH + dl * NH));
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              const float4 v = row[row_chunk(dl, hb / 4 + c)];
              const float* e = scal + r * NH + hb + 4 * c;
              o[4 * c] += v.x * e[0];
              o[4 * c + 1] += v.y * e[1];
              o[4 * c + 2] += v.z * e[2];
              o[4 * c + 3] += v.w * e[3];
            }
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) o[j] *= scal[4 * NH + hb + j];
          store_pairs_n<16, kMulti>(p, o_tok, token, d, hb, o);
        }
      }
      tc_fence_before();
    }
    __syncthreads();
  } else {
    // ---- split across 8 CTAs (tiny batches): merge through distributed
    // shared memory reads
    cluster_sync_all();   // (A) every CTA's m / l visible cluster-wide
    if (warp < 4) {
      if (tid < NH) {
        const int hh = tid;
        const uint32_t m_addr = sb + kSmHead + 4u * hh;
        const uint32_t l_addr = m_addr + 256u;
        float M = -INFINITY, L = 0.f;
        for (int r = 0; r < nranks; ++r) {
          const float lr = ld_dsmem_f32(mapa_shared(l_addr, r));
          if (lr > 0.f) M = fmaxf(M, ld_dsmem_f32(mapa_shared(m_addr, r)));
        }
        for (int r = 0; r < nranks; ++r) {
          const float lr = ld_dsmem_f32(mapa_shared(l_addr, r));
          if (lr > 0.f) L += lr * exp2f(ld_dsmem_f32(mapa_shared(m_addr, r)) - M);
        }
        const float l_own = l_sm[hh];
        f_sm[hh] = (L > 0.f && l_own > 0.f) ? kvs * exp2f(m_sm[hh] - M) / L : 0.f;
        if (split == 0 && p.lse != nullptr && hh < p.H)
          p.lse[static_cast<size_t>(token) * p.H + hh] = L > 0.f ? log2f(L) + M : -INFINITY;
      }
      named_bar_sync(1, 128);
      if (n_tiles > 0)
        mbar_wait_bounded(bar(kBarODone), (n_tiles - 1) & 1, abort_flag, p.timeout_ns);
      tc_fence_after();
      // scaled partial -> fp32 [h][512] in the (now idle) KV stage region
      float* const part = reinterpret_cast<float*>(gb + kSmKV);
#pragma unroll 1
      for (int m = 0; m < 4; ++m) {
        const int d = 128 * m + 32 * warp + lane;
        float o[NH];
        load_o(m, o);
#pragma unroll
        for (int j = 0; j < NH; ++j) part[j * kDim + d] = n_tiles > 0 ? o[j] * f_sm[j] : 0.f;
      }
      tc_fence_before();
    }
    cluster_sync_all();   // (B) every CTA's scaled partial visible cluster-wide
    const int dspan = kDim / nranks;
    const int units_per_head = dspan / 8;
    const int units = p.H * units_per_head;
    for (int u = tid; u < units; u += kThreads) {
      const int hh = u / units_per_head;
      const int d = split * dspan + (u % units_per_head) * 8;
      const uint32_t off = sb + kSmKV + static_cast<uint32_t>(hh * kDim + d) * 4u;
      float4 x[8], y[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const uint32_t a = mapa_shared(off, r);
        x[r] = ld_dsmem_v4(a);
        y[r] = ld_dsmem_v4(a + 16);
      }
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        acc[0] += x[r].x; acc[1] += x[r].y; acc[2] += x[r].z; acc[3] += x[r].w;
        acc[4] += y[r].x; acc[5] += y[r].y; acc[6] += y[r].z; acc[7] += y[r].w;
      }
      const uint4 v = make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                                 pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
      if constexpr (!kMulti) {
        stg_v4(o_tok + static_cast<size_t>(hh) * kDim + d, v);
      } else {
        const size_t o_off = static_cast<size_t>(token) * p.out_tok_stride + static_cast<size_t>(hh) * kDim + d;
#pragma unroll
        for (int i = 0; i < kMaxOutputs; ++i)
          if (i < p.n_out) stg_v4(p.outs[i] + o_off, v);
      }
    }
    cluster_sync_all();   // (C) no CTA leaves while a peer still reads its smem
  }

  cp_async_wait_all();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  if (tid == 0 && *abort_flag) atomicOr(&g_device_status, static_cast<unsigned>(GLM53_DEV_TIMEOUT));
}

// ---------------------------------------------------------------------------
// gather-only probe: the attention's gather (16-byte cp.async per lane into
// the same swizzled 64-row tiles) with no math, over a 3-stage ring
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_2() { asm volatile("cp.async.wait_group 2;" ::: "memory"); }

constexpr int kRoofStages = 3;
constexpr int kRoofThreads = 256;

// CTA c gathers entries [c * per_cta, min(total, (c + 1) * per_cta)) of the
// flattened [T, topk] index list; entries outside [0, kv_rows) are skipped.
// sink[c] = XOR of the first 32-bit word of every row it gathered, so the
// copies cannot be elided and the result can be checked on the host.
__global__ void __launch_bounds__(kRoofThreads, 1) gather_roof_kernel(const uint8_t* __restrict__ kv,
                                                                      const int32_t* __restrict__ idx,
                                                                      long long total, long long per_cta,
                                                                      long long kv_rows,
                                                                      uint32_t* __restrict__ sink) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t sb = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* const gb = smem_raw + (sb - smem_u32(smem_raw));
  __shared__ uint32_t red[kRoofThreads / 32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long k0 = static_cast<long long>(blockIdx.x) * per_cta;
  const long long n = max(0ll, min(per_cta, total - k0));
  const int ntiles = static_cast<int>((n + kRows - 1) / kRows);
  uint32_t x = 0;
  // thread r < 64 folds in row r of a tile that has landed
  auto check = [&](int t) {
    if (threadIdx.x < kRows) {
      const long long k = static_cast<long long>(kRows) * t + threadIdx.x;
      const int32_t v = k < n ? idx[k0 + k] : -1;
      if (v >= 0 && v < kv_rows)
        x ^= *reinterpret_cast<const uint32_t*>(gb + (t % kRoofStages) * kStageBytes + swz(threadIdx.x, 0));
    }
  };
  for (int t = 0; t < ntiles; ++t) {
    // stage t % 3 was last read by check(t - 3), before the barrier of the
    // previous iteration; this barrier orders that read before the overwrite
    if (t >= kRoofStages) __syncthreads();
    const uint32_t stage = sb + (t % kRoofStages) * kStageBytes;
    for (int r = warp; r < kRows; r += kRoofThreads / 32) {
      const long long k = static_cast<long long>(kRows) * t + r;
      const int32_t v = k < n ? idx[k0 + k] : -1;
      const bool valid = v >= 0 && v < kv_rows;
      const uint8_t* src = kv + (valid ? static_cast<long long>(v) : 0) * (kDim * 2);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int c = lane + 32 * hh;
        cp_async_16(stage + swz(r, c), src + c * 16, valid ? 16u : 0u);
      }
    }
    cp_async_commit();
    if (t >= kRoofStages - 1) {
      cp_async_wait_2();     // tile t - 2 landed (this thread's part)
      __syncthreads();       // ... and every thread's
      check(t - (kRoofStages - 1));
    }
  }
  cp_async_wait_all();
  __syncthreads();
  for (int t = max(0, ntiles - (kRoofStages - 1)); t < ntiles; ++t) check(t);
#pragma unroll
  for (int k = 16; k >= 1; k >>= 1) x ^= __shfl_xor_sync(0xFFFFFFFFu, x, k);
  if (lane == 0) red[warp] = x;
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t y = 0;
    for (int w = 0; w < kRoofThreads / 32; ++w) y ^= red[w];
    if (sink != nullptr) sink[blockIdx.x] = y;
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
constexpr int kMaxDevices = 64;
std::mutex g_mutex;
bool g_prepared[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};
int g_cc_major[kMaxDevices] = {};
// Pipeline-wait limit passed to every launch (0: not yet resolved). Set from
// GLM53_WAIT_TIMEOUT_MS (default 1000 ms) on first use, or by
// glm53_sparse_mla_set_wait_timeout_ns.
std::atomic<unsigned long long> g_timeout_ns{0};

unsigned long long default_timeout_ns() {
  const char* env = std::getenv("GLM53_WAIT_TIMEOUT_MS");
  const long long ms = env ? std::atoll(env) : 0;
  return static_cast<unsigned long long>(ms > 0 ? ms : 1000) * 1000000ull;
}
int g_env_splits = -1;   // GLM53_SPLITS: forced split count for splits == 0 (-1: unread)

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's tensor-map encoder, fetched once through the runtime (the
// library links only the CUDA runtime).
EncodeTiledFn q_encoder() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// Tensor map of q [T, H, 512] bf16 viewed as the 3-D tensor {512, H, T}, boxes
// of {64 elements, rows heads, 1 token} with the 128-byte swizzle: one box is
// one 64-element column block of GEMM1's A operand. Heads past H read as zero
// (the box leaves the tensor), which pads Q to the kernel's head count.
bool make_q_map(CUtensorMap* map, const void* q, int64_t T, int64_t H, int rows) {
  EncodeTiledFn enc = q_encoder();
  if (enc == nullptr) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kDim), static_cast<cuuint64_t>(H),
                              static_cast<cuuint64_t>(T)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kDim * 2), static_cast<cuuint64_t>(H * kDim * 2)};
  const cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(rows), 1u};
  const cuuint32_t elem[3] = {1u, 1u, 1u};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box, elem,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NH, bool FP8, bool MULTI>
cudaError_t launch_fwd(const Params& p, int splits, cudaStream_t stream) {
  CUtensorMap q_map;
  std::memset(&q_map, 0, sizeof(q_map));
  if (!FP8 && !make_q_map(&q_map, p.q, p.T, p.H, static_cast<int>(Lay<NH>::kQRows)))
    return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.T) * static_cast<unsigned>(splits), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = Lay<NH>::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = static_cast<unsigned>(splits);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = splits > 1 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, sparse_mla_fwd_kernel<NH, FP8, MULTI>, p, q_map);
}

template <int NH, bool FP8, bool MULTI = false>
cudaError_t set_smem_attr() {
  return cudaFuncSetAttribute(sparse_mla_fwd_kernel<NH, FP8, MULTI>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(Lay<NH>::kSmemBytes));
}

int prepare_current_device(int* dev_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GLM53_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return GLM53_ERR_CUDA;
  if (dev_out) *dev_out = dev;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_prepared[dev]) return GLM53_OK;
  if (g_env_splits < 0) {
    const char* env = std::getenv("GLM53_SPLITS");
    const int v = env ? std::atoi(env) : 0;
    g_env_splits = (v == 1 || v == 2 || v == 4 || v == 8) ? v : 0;
  }
  if (g_timeout_ns.load() == 0) g_timeout_ns.store(default_timeout_ns());
  int major = 0, sms = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return GLM53_ERR_CUDA;
  g_cc_major[dev] = major;
  g_sm_count[dev] = sms;
  if (major != 10) return GLM53_ERR_DEVICE;
  cudaError_t e = cudaSuccess;
  if (e == cudaSuccess) e = set_smem_attr<16, false>();
  if (e == cudaSuccess) e = set_smem_attr<32, false>();
  if (e == cudaSuccess) e = set_smem_attr<64, false>();
  if (e == cudaSuccess) e = set_smem_attr<16, true>();
  if (e == cudaSuccess) e = set_smem_attr<32, true>();
  if (e == cudaSuccess) e = set_smem_attr<64, true>();
  if (e == cudaSuccess) e = set_smem_attr<16, false, true>();
  if (e == cudaSuccess) e = set_smem_attr<32, false, true>();
  if (e == cudaSuccess) e = set_smem_attr<64, false, true>();
  if (e == cudaSuccess) e = set_smem_attr<16, true, true>();
  if (e == cudaSuccess) e = set_smem_attr<32, true, true>();
  if (e == cudaSuccess) e = set_smem_attr<64, true, true>();
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gather_roof_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kRoofStages * kStageBytes + 1024));
  if (e != cudaSuccess) return GLM53_ERR_CUDA;
  g_prepared[dev] = true;
  return GLM53_OK;
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace glm53

using namespace glm53;

extern "C" int glm53_sparse_mla_check(int64_t T, int64_t H, int64_t head_dim, int64_t kv_rows,
                                      int64_t kv_width, int64_t topk, int kv_dtype, int splits) {
  if (T < 0 || kv_rows < 0 || topk < 0) return GLM53_ERR_RANK;
  if (head_dim != kDim || kv_width != kDim) return GLM53_ERR_HEAD_DIM;
  if (kv_dtype != GLM53_KV_BF16 && kv_dtype != GLM53_KV_FP8_E4M3) return GLM53_ERR_DTYPE;
  if (H != 8 && H != 16 && H != 32 && H != 64) return GLM53_ERR_HEADS;
  if (topk % 32 != 0 || topk > 8 * kMaxChunk) return GLM53_ERR_TOPK;
  if (splits != 0 && splits != 1 && splits != 2 && splits != 4 && splits != 8)
    return GLM53_ERR_SPLITS;
  if (splits != 0 && (topk + splits - 1) / splits > kMaxChunk) return GLM53_ERR_TOPK;
  if (T > (int64_t{1} << 28) || kv_rows > (int64_t{1} << 31)) return GLM53_ERR_RANK;
  return GLM53_OK;
}

extern "C" int glm53_sparse_mla_auto_splits(int64_t T, int64_t topk, int sm_count) {
  if (T <= 0) return 1;
  int s = 1;
  // widen while the grid still fits in one wave and each CTA keeps >= 4 tiles
  while (s < 8 && T * (2 * s) <= sm_count && topk / (2 * s) >= 4 * kRows) s *= 2;
  while ((topk + s - 1) / s > kMaxChunk && s < 8) s *= 2;
  return s;
}

extern "C" int glm53_sparse_mla_prepare(void) { return prepare_current_device(nullptr); }

namespace glm53 {

int padded_heads(int64_t H) { return H <= 16 ? 16 : static_cast<int>(H); }

// Split count the launcher uses for this shape on device `dev`.
int resolve_splits(int64_t T, int64_t topk, int splits, int dev) {
  if (splits != 0) return splits;
  return g_env_splits > 0 ? g_env_splits : glm53_sparse_mla_auto_splits(T, topk, g_sm_count[dev]);
}

// Launch plan: tokens [0, t_main) with s_main CTAs each, then tokens
// [t_main, T) with s_tail CTAs each. Automatic splitting of a batch too large
// to split (more tokens than SMs) keeps whole waves unsplit and splits the
// tokens of the last, partial wave so they fill the machine instead of
// running on a few SMs at the end.
struct Plan {
  int64_t t_main;
  int s_main;
  int64_t t_tail;
  int s_tail;
};

Plan make_plan(int64_t T, int64_t topk, int splits, int dev) {
  Plan pl{T, resolve_splits(T, topk, splits, dev), 0, 1};
  if (splits == 0 && g_env_splits <= 0 && pl.s_main == 1) {
    const int64_t sms = g_sm_count[dev];
    const int64_t full = (T / sms) * sms, rem = T - full;
    if (full > 0 && rem > 0) {
      int ts = 1;
      while (ts < 8 && rem * (2 * ts) <= sms && topk / (2 * ts) >= 4 * kRows) ts *= 2;
      if (ts > 1) pl = Plan{full, 1, rem, ts};
    }
  }
  return pl;
}

uint64_t workspace_floats(int64_t T, int64_t H, int splits) {
  if (splits <= 1) return 0;
  const uint64_t nh = static_cast<uint64_t>(padded_heads(H));
  return static_cast<uint64_t>(T) * static_cast<uint64_t>(splits) * nh * kDim;
}

uint64_t workspace_floats(const Plan& pl, int64_t H) {
  return workspace_floats(pl.t_main, H, pl.s_main) + workspace_floats(pl.t_tail, H, pl.s_tail);
}

// Paged index form (glm53_sparse_mla_fwd_paged): request-local positions
// converted in the kernel.
struct Paged {
  const int32_t* req_id;
  const int32_t* block_table;
  int64_t idx_stride, bt_stride, max_blocks, block_size, block_stride;
};

// Output set of the fused head gather: n buffers [T, heads_total, 512], this
// launch's H heads written at heads [head_offset, head_offset + H) of each.
struct OutSet {
  void* const* outs;
  int n;
  int64_t heads_total, head_offset;
};

// Shared body of the forward entry points. `ws == nullptr` selects the
// distributed-shared-memory split merge; otherwise `ws` (at least
// `ws_bytes`) is the global workspace of the L2 split merge. `pg` selects the
// paged index form, `os` the outputs of a head-sharded group (else `out`).
int launch_forward(const void* q, const void* kv, const int32_t* indices, void* out, float* lse,
                   int64_t T, int64_t H, int64_t head_dim, int64_t kv_rows, int64_t kv_width,
                   int64_t topk, int kv_dtype, float sm_scale, float kv_scale, int splits,
                   bool use_ws, void* ws, uint64_t ws_bytes, void* stream,
                   const Paged* pg = nullptr, const OutSet* os = nullptr) {
  // A named host range for profilers and tracers (a no-op without one).
  struct NvtxRange {
    NvtxRange() { nvtxRangePushA("glm53_sparse_mla_fwd"); }
    ~NvtxRange() { nvtxRangePop(); }
  } nvtx_range;
  int rc = glm53_sparse_mla_check(T, H, head_dim, kv_rows, kv_width, topk, kv_dtype, splits);
  if (rc != GLM53_OK) return rc;
  if (T == 0) return GLM53_OK;
  // the paged form reads indices with 4-byte loads at any row stride
  const bool idx_ok = pg != nullptr ? (reinterpret_cast<uintptr_t>(indices) & 3u) == 0 : aligned16(indices);
  if (!aligned16(q) || !aligned16(kv) || !idx_ok || !aligned16(out) ||
      q == nullptr || kv == nullptr || indices == nullptr || out == nullptr)
    return GLM53_ERR_ALIGN;
  if (lse != nullptr && (reinterpret_cast<uintptr_t>(lse) & 3u) != 0) return GLM53_ERR_ALIGN;
  void* const single[1] = {out};
  const OutSet one{single, 1, H, 0};
  if (os == nullptr) os = &one;
  if (os->n < 1 || os->n > kMaxOutputs || os->outs == nullptr || os->head_offset < 0 ||
      os->head_offset + H > os->heads_total || os->heads_total > 64 * kMaxOutputs)
    return GLM53_ERR_RANK;
  for (int i = 0; i < os->n; ++i)
    if (os->outs[i] == nullptr || !aligned16(os->outs[i])) return GLM53_ERR_ALIGN;
  int dev = 0;
  rc = prepare_current_device(&dev);
  if (rc != GLM53_OK) return rc;
  const Plan pl = make_plan(T, topk, splits, dev);
  if ((topk + pl.s_main - 1) / pl.s_main > kMaxChunk) return GLM53_ERR_TOPK;
  const uint64_t need = 4 * workspace_floats(pl, H);
  if (use_ws && need > 0 && (ws == nullptr || !aligned16(ws) || ws_bytes < need))
    return GLM53_ERR_WORKSPACE;

  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool fp8 = kv_dtype == GLM53_KV_FP8_E4M3;
  const bool multi = os->n > 1;
  const size_t q_tok = static_cast<size_t>(H) * kDim;   // bf16 elements per token of q / out
  float* ws_next = use_ws ? static_cast<float*>(ws) : nullptr;
  for (int part = 0; part < 2; ++part) {
    const int64_t t0 = part == 0 ? 0 : pl.t_main;
    const int64_t n = part == 0 ? pl.t_main : pl.t_tail;
    const int s = part == 0 ? pl.s_main : pl.s_tail;
    if (n == 0) continue;
    Params p;
    p.q = static_cast<const __nv_bfloat16*>(q) + t0 * q_tok;
    p.kv = kv;
    const int64_t istride = pg != nullptr ? pg->idx_stride : topk;
    p.idx = indices + t0 * istride;
    p.idx_stride = istride;
    p.req_id = pg != nullptr ? pg->req_id + t0 : nullptr;
    p.block_table = pg != nullptr ? pg->block_table : nullptr;
    p.bt_stride = pg != nullptr ? pg->bt_stride : 0;
    p.max_blocks = pg != nullptr ? static_cast<int>(pg->max_blocks) : 0;
    p.block_size = pg != nullptr ? static_cast<int>(pg->block_size) : 1;
    p.block_stride = pg != nullptr ? static_cast<int>(pg->block_stride) : 1;
    for (int i = 0; i < kMaxOutputs; ++i)
      p.outs[i] = i < os->n ? static_cast<__nv_bfloat16*>(os->outs[i]) +
                                  (t0 * os->heads_total + os->head_offset) * kDim
                            : nullptr;
    p.n_out = os->n;
    p.out_tok_stride = os->heads_total * kDim;
    p.lse = lse != nullptr ? lse + t0 * H : nullptr;
    p.ws = (use_ws && s > 1) ? ws_next : nullptr;
    if (p.ws != nullptr) ws_next += workspace_floats(n, H, s);
    p.kv_rows = kv_rows;
    p.T = static_cast<int>(n);
    p.H = static_cast<int>(H);
    p.topk = static_cast<int>(topk);
    p.splits = s;
    p.chunk = static_cast<int>((topk + s - 1) / s);
    p.c = sm_scale * 1.4426950408889634f;
    p.kv_scale = kv_dtype == GLM53_KV_BF16 ? 1.0f : kv_scale;
    p.timeout_ns = g_timeout_ns.load();
    cudaError_t e;
    if (H <= 16)
      e = multi ? (fp8 ? launch_fwd<16, true, true>(p, s, st) : launch_fwd<16, false, true>(p, s, st))
                : (fp8 ? launch_fwd<16, true, false>(p, s, st) : launch_fwd<16, false, false>(p, s, st));
    else if (H == 32)
      e = multi ? (fp8 ? launch_fwd<32, true, true>(p, s, st) : launch_fwd<32, false, true>(p, s, st))
                : (fp8 ? launch_fwd<32, true, false>(p, s, st) : launch_fwd<32, false, false>(p, s, st));
    else
      e = multi ? (fp8 ? launch_fwd<64, true, true>(p, s, st) : launch_fwd<64, false, true>(p, s, st))
                : (fp8 ? launch_fwd<64, true, false>(p, s, st) : launch_fwd<64, false, false>(p, s, st));
    if (e != cudaSuccess) return GLM53_ERR_CUDA;
  }
  return GLM53_OK;
}

}  // namespace glm53

extern "C" int glm53_sparse_mla_fwd(const void* q, const void* kv, const int32_t* indices,
                                    void* out, float* lse, int64_t T, int64_t H, int64_t head_dim,
                                    int64_t kv_rows, int64_t kv_width, int64_t topk, int kv_dtype,
                                    float sm_scale, float kv_scale, int splits, void* stream) {
  return launch_forward(q, kv, indices, out, lse, T, H, head_dim, kv_rows, kv_width, topk,
                        kv_dtype, sm_scale, kv_scale, splits, false, nullptr, 0, stream);
}

extern "C" int glm53_sparse_mla_workspace_bytes(int64_t T, int64_t H, int64_t topk, int splits,
                                                uint64_t* bytes) {
  if (bytes == nullptr) return GLM53_ERR_ALIGN;
  *bytes = 0;
  const int rc0 = glm53_sparse_mla_check(T, H, kDim, 0, kDim, topk, GLM53_KV_BF16, splits);
  if (rc0 != GLM53_OK) return rc0;
  if (T == 0) return GLM53_OK;
  int dev = 0;
  const int rc = prepare_current_device(&dev);
  if (rc != GLM53_OK) return rc;
  *bytes = 4 * workspace_floats(make_plan(T, topk, splits, dev), H);
  return GLM53_OK;
}

extern "C" int glm53_sparse_mla_fwd_paged(
    const void* q, const void* kv, const int32_t* topk_positions, int64_t positions_row_stride,
    const int32_t* req_id_per_token, const int32_t* block_table, int64_t block_table_row_stride,
    int64_t max_blocks_per_req, int64_t block_size, int64_t block_stride_rows, void* out, float* lse,
    int64_t T, int64_t H, int64_t head_dim, int64_t kv_rows, int64_t kv_width, int64_t topk,
    int kv_dtype, float sm_scale, float kv_scale, int splits, void* workspace,
    uint64_t workspace_bytes, void* stream) {
  int rc = glm53_sparse_mla_check(T, H, head_dim, kv_rows, kv_width, topk, kv_dtype, splits);
  if (rc != GLM53_OK) return rc;
  if (positions_row_stride < topk || block_size <= 0 || block_size > (int64_t{1} << 20) ||
      max_blocks_per_req <= 0 || max_blocks_per_req > (int64_t{1} << 30) ||
      block_table_row_stride < max_blocks_per_req || block_stride_rows < block_size ||
      block_stride_rows > (int64_t{1} << 24) || kv_rows > 0x7FFFFFFFll)
    return GLM53_ERR_RANK;
  if (T == 0) return GLM53_OK;
  if (req_id_per_token == nullptr || block_table == nullptr ||
      (reinterpret_cast<uintptr_t>(req_id_per_token) & 3u) != 0 ||
      (reinterpret_cast<uintptr_t>(block_table) & 3u) != 0)
    return GLM53_ERR_ALIGN;
  const Paged pg{req_id_per_token, block_table, positions_row_stride, block_table_row_stride,
                 max_blocks_per_req, block_size, block_stride_rows};
  return launch_forward(q, kv, topk_positions, out, lse, T, H, head_dim, kv_rows, kv_width, topk,
                        kv_dtype, sm_scale, kv_scale, splits, true, workspace, workspace_bytes,
                        stream, &pg);
}

extern "C" int glm53_sparse_mla_fwd_ws(const void* q, const void* kv, const int32_t* indices,
                                       void* out, float* lse, int64_t T, int64_t H,
                                       int64_t head_dim, int64_t kv_rows, int64_t kv_width,
                                       int64_t topk, int kv_dtype, float sm_scale, float kv_scale,
                                       int splits, void* workspace, uint64_t workspace_bytes,
                                       void* stream) {
  return launch_forward(q, kv, indices, out, lse, T, H, head_dim, kv_rows, kv_width, topk,
                        kv_dtype, sm_scale, kv_scale, splits, true, workspace, workspace_bytes,
                        stream);
}

extern "C" int glm53_sparse_mla_fwd_heads_gather(
    const void* q, const void* kv, const int32_t* indices, void* const* outs, int n_outs,
    int64_t head_offset, int64_t heads_total, float* lse, int64_t T, int64_t H, int64_t head_dim,
    int64_t kv_rows, int64_t kv_width, int64_t topk, int kv_dtype, float sm_scale, float kv_scale,
    int splits, void* workspace, uint64_t workspace_bytes, void* stream) {
  if (outs == nullptr || n_outs < 1 || n_outs > kMaxOutputs) return GLM53_ERR_RANK;
  const OutSet os{outs, n_outs, heads_total, head_offset};
  return launch_forward(q, kv, indices, outs[0], lse, T, H, head_dim, kv_rows, kv_width, topk,
                        kv_dtype, sm_scale, kv_scale, splits, true, workspace, workspace_bytes,
                        stream, nullptr, &os);
}

extern "C" int glm53_copy_head_slices(void* const* dsts, int n_dsts, const void* src,
                                      int64_t tokens, int64_t heads_total, int64_t head_offset,
                                      int64_t heads, void* stream) {
  if (dsts == nullptr || n_dsts < 0 || n_dsts > kMaxOutputs || src == nullptr || tokens < 0 ||
      heads_total <= 0 || head_offset < 0 || heads <= 0 || head_offset + heads > heads_total)
    return GLM53_ERR_RANK;
  if (tokens == 0) return GLM53_OK;
  const size_t row = static_cast<size_t>(kDim) * 2;                      // bytes per (token, head)
  const size_t pitch = static_cast<size_t>(heads_total) * row;           // bytes per token
  const size_t off = static_cast<size_t>(head_offset) * row;
  for (int i = 0; i < n_dsts; ++i) {
    if (dsts[i] == nullptr) return GLM53_ERR_ALIGN;
    if (dsts[i] == src) continue;
    if (cudaMemcpy2DAsync(static_cast<uint8_t*>(dsts[i]) + off, pitch,
                          static_cast<const uint8_t*>(src) + off, pitch,
                          static_cast<size_t>(heads) * row, static_cast<size_t>(tokens),
                          cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream)) != cudaSuccess)
      return GLM53_ERR_CUDA;
  }
  return GLM53_OK;
}

// ---------------------------------------------------------------------------
// No-allocation entry point
// ---------------------------------------------------------------------------
// Some callers cannot allocate device memory at call time: code running
// under a custom or fixed-size memory pool, embedders whose allocator is not
// reachable from the attention call site, runtimes that forbid cudaMalloc once
// serving has started. For them the split-merge workspace is a file-scope
// device array of a fixed size. Every device that loads this library keeps it
// (kNoAllocScratchBytes) until the process exits.
namespace glm53 {
constexpr uint64_t kNoAllocScratchBytes = 32ull << 20;   // 32 MiB
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / 4];
void* g_noalloc_addr[kMaxDevices] = {};
}  // namespace glm53

extern "C" int glm53_sparse_mla_fwd_noalloc(const void* q, const void* kv, const int32_t* indices,
                                            void* out, float* lse, int64_t T, int64_t H,
                                            int64_t head_dim, int64_t kv_rows, int64_t kv_width,
                                            int64_t topk, int kv_dtype, float sm_scale,
                                            float kv_scale, int splits, void* stream) {
  int rc = glm53_sparse_mla_check(T, H, head_dim, kv_rows, kv_width, topk, kv_dtype, splits);
  if (rc != GLM53_OK) return rc;
  if (T == 0) return GLM53_OK;
  int dev = 0;
  rc = prepare_current_device(&dev);
  if (rc != GLM53_OK) return rc;
  void* scratch = nullptr;
  {
    // The array's host-side name is only a stand-in; its device address is
    // looked up once per device, with that device current.
    std::lock_guard<std::mutex> lock(g_mutex);
    if (g_noalloc_addr[dev] == nullptr) {
      void* ptr = nullptr;
      if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr)
        return GLM53_ERR_CUDA;
      g_noalloc_addr[dev] = ptr;
    }
    scratch = g_noalloc_addr[dev];
  }
  if (4 * workspace_floats(make_plan(T, topk, splits, dev), H) > kNoAllocScratchBytes)
    return GLM53_ERR_SCRATCH_LIMIT;
  return launch_forward(q, kv, indices, out, lse, T, H, head_dim, kv_rows, kv_width, topk,
                        kv_dtype, sm_scale, kv_scale, splits, true, scratch, kNoAllocScratchBytes,
                        stream);
}

extern "C" int glm53_sparse_mla_set_wait_timeout_ns(uint64_t ns) {
  g_timeout_ns.store(ns > 0 ? static_cast<unsigned long long>(ns) : default_timeout_ns());
  return GLM53_OK;
}

extern "C" int glm53_sparse_mla_device_status(uint32_t* status, int clear) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_status, sizeof(v)) != cudaSuccess) return GLM53_ERR_CUDA;
  if (status) *status = v;
  if (clear) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(g_device_status, &zero, sizeof(zero)) != cudaSuccess)
      return GLM53_ERR_CUDA;
  }
  return GLM53_OK;
}

extern "C" int glm53_gather_roof(const void* kv, const int32_t* indices, int64_t T, int64_t topk,
                                 int64_t kv_rows, int ctas, uint32_t* sink, void* stream) {
  if (T < 0 || topk < 0 || kv_rows < 0 || ctas < 0) return GLM53_ERR_RANK;
  if (T == 0 || topk == 0) return GLM53_OK;
  if (kv == nullptr || indices == nullptr || !aligned16(kv)) return GLM53_ERR_ALIGN;
  const int rc = prepare_current_device(nullptr);
  if (rc != GLM53_OK) return rc;
  const long long total = T * topk;
  const long long grid = ctas == 0 ? T : std::min<long long>(ctas, total);
  const long long per_cta = (total + grid - 1) / grid;
  gather_roof_kernel<<<static_cast<unsigned>(grid), kRoofThreads, kRoofStages * kStageBytes + 1024,
                       static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(kv), indices, total, per_cta, kv_rows, sink);
  return cudaGetLastError() == cudaSuccess ? GLM53_OK : GLM53_ERR_CUDA;
}

extern "C" const char* glm53_sparse_mla_strerror(int code) {
  switch (code) {
    case GLM53_OK: return "ok";
    case GLM53_ERR_RANK: return "expected q [T, H, 512], kv [R, 512], indices [T, topk], out shaped like q";
    case GLM53_ERR_HEAD_DIM: return "expected kv_lora_rank 512 with qk_rope_head_dim 0 (NoPE)";
    case GLM53_ERR_HEADS: return "unsupported heads-per-rank; built for 8, 16, 32 or 64 (TP=8/4/2/1 on a 64-head model)";
    case GLM53_ERR_TOPK: return "topk must be a multiple of 32 and at most 16384";
    case GLM53_ERR_DTYPE: return "kv must be bfloat16 or float8_e4m3fn";
    case GLM53_ERR_ALIGN: return "a tensor pointer is null or not 16-byte aligned";
    case GLM53_ERR_SPLITS: return "splits must be 0 (auto), 1, 2, 4 or 8";
    case GLM53_ERR_CUDA: return "CUDA runtime error while launching the sparse-MLA kernel";
    case GLM53_ERR_DEVICE: return "the current device is not an sm_100 (B200-class) GPU";
    case GLM53_ERR_WORKSPACE: return "workspace missing, not 16-byte aligned or smaller than glm53_sparse_mla_workspace_bytes";
    case GLM53_ERR_SCRATCH_LIMIT: return "shape needs more split-merge scratch than the 32 MiB built into glm53_sparse_mla_fwd_noalloc; use glm53_sparse_mla_fwd_ws";
    default: return "unknown glm53_sparse_mla status";
  }
}
