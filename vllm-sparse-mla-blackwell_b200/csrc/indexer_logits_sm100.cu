// Sparse-attention indexer scores over a paged fp8 cache, sm_100a: the logits
// the indexer's per-row top-k (topk_sm100.cu) selects from. Same contract as
// DeepGEMM's fp8 paged MQA logits as vLLM 0.22.0 calls it
// (vllm/utils/deep_gemm.py:407-456, from
// vllm/model_executor/layers/sparse_attn_indexer.py:324-333), with vLLM's
// torch restatement (vllm/v1/attention/ops/rocm_aiter_mla_sparse.py:256-356)
// as the arithmetic:
//
//   query token j of request i (row i * next_n + j) sees cache positions
//   p < context_lens[i] - next_n + j + 1 (or p < context_lens[i][j] when the
//   lengths are given per token), and
//     logits[row, p] = scale[p] * sum_h relu(q[i, j, h, :] . k[p, :]) * w[row, h]
//   with q, k e4m3 (head dim 128) and per-position fp32 scales; the cache is
//   paged, each block holding block_size rows of 128 e4m3 values followed by
//   block_size fp32 scales. With `clean`, every other position up to
//   max_model_len is written as -inf; without it, they are left untouched.
//
// Design: one CTA per (request, 1024 cache positions; 512 or 256 when a
// small batch would leave SMs idle), 256 threads.
//   warps 5-7  gather: the request's queries (N = H * next_n rows of 128 B)
//              and the block ids of the CTA's positions (into shared memory)
//              once; then, for each 128-position tile, one lane of warp
//              5 + t % 3 issues a TMA load per cache block in it (a block's
//              rows are one contiguous run; the tensor map's 128-byte
//              swizzle lands them in the K-major layout the tensor core
//              reads) and a bulk copy of the block's scales, into a 4- to
//              6-stage ring. Three issuing warps keep several tiles' issues
//              in flight; a box with nothing to read is zero-filled instead.
//   warp 4     TMEM allocation; one lane issues per tile four e4m3 UMMAs
//              (M = 128 positions, N = H * next_n, K = 32 each) into one of
//              two TMEM accumulators S^T[position][head];
//   warps 0-3  epilogue: thread t owns position t of the tile (TMEM lane t),
//              reads its row of S^T, applies relu, weights and sums over each
//              token's heads in registers, multiplies by the scale and
//              writes the logits (coalesced across the warp).
// The reduction over heads is a row sum in TMEM order, so no shuffle or
// shared-memory pass is needed. Positions outside the block table, or blocks
// past the cache, read nothing and raise a status bit; every wait is bounded.
// (Measured on B200 at 32 x 8192 positions: per-chunk cp.async addressing
// 39 -> 17 us once block ids were staged in shared memory, a single TMA
// issuer 12.5 us, three issuers 11.5 us, cp.async per block 14.0 us, half
// TMA and half cp.async 12.2 us. The TMA loads are bound by the per-SM copy
// engine's rate on this HBM stream, about 12 B/clk.)

#include <cuda.h>   // CUtensorMap and its enums (the encoder is fetched at run time)
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <atomic>
#include <mutex>
#include <utility>

#include "glm53_sparse_mla.h"
#include "sm100_ptx.cuh"

namespace glm53 {
namespace indexer {

constexpr int kD = 128;                 // index head dim = bytes per fp8 row
constexpr int kTile = 128;              // cache positions per UMMA tile (M)
constexpr int kMaxTilesPerCta = 8;      // up to 1024 positions per CTA
constexpr int kMaxCols = kTile * kMaxTilesPerCta / 16 + 1;   // block-table entries a CTA touches (block >= 16)
constexpr int kThreads = 256;
constexpr int kMmaWarp = 4;
constexpr int kGatherWarp0 = 5;
constexpr int kGatherThreads = 96;
constexpr uint32_t kStageBytes = kTile * kD;     // 16 KB
constexpr uint32_t kScaleBytes = kTile * 4;      // 512 B

constexpr unsigned kStatusTimeout = 1u;
constexpr unsigned kStatusBadBlock = 2u;

__device__ unsigned int g_indexer_status = 0;

struct Params {
  const uint8_t* q;            // [B, next_n, H, 128] e4m3
  const uint8_t* kv;           // num_blocks blocks of block_bytes
  const float* weights;        // [B * next_n, H]
  const int32_t* ctx_lens;     // [B] per request, or [B * next_n] per token (per_row_lens)
  int per_row_lens;
  const int32_t* block_table;  // [B, bt_stride]
  long long bt_stride;
  long long block_bytes;
  long long num_blocks;
  float* logits;               // [B * next_n, logits_stride]
  long long logits_stride;
  int block_size;
  int log2_block;              // block_size is a power of two, 16 .. 1024
  int box_rows;                // rows per TMA box: min(block_size, 128)
  int max_blocks;
  int max_model_len;
  int clean;
  int tiles_per_cta;           // 128-position tiles per CTA: 8, or 4 / 2 for small batches
  unsigned long long timeout_ns;
};

// Shared memory map (offsets from a 1024-aligned base) for N = H * next_n
// query rows: the queries, then as many 16.5 KB cache stages as keep two
// CTAs on an SM (more bytes in flight per SM is what the gather needs).
template <int N>
struct Layout {
  static constexpr uint32_t kQ = 0;                                  // N rows x 128 B
  static constexpr uint32_t kQBytes = (N * 128 + 1023) / 1024 * 1024;
  static constexpr int kStages = N <= 64 ? 6 : (N <= 128 ? 5 : 4);
  static constexpr uint32_t kStage = kQBytes;                        // kStages x 16 KB
  static constexpr uint32_t kScale = kStage + kStages * kStageBytes;
  static constexpr uint32_t kW = kScale + kStages * kScaleBytes;     // N floats
  static constexpr uint32_t kBar = kW + N * 4;
  static constexpr uint32_t kMisc = kBar + 24 * 8;                   // tmem base, abort flag
  static constexpr uint32_t kBt = kMisc + 64;                        // [kMaxCols] block ids
  static constexpr uint32_t kBytes = kBt + 4 * kMaxCols + 1024;      // + slack to align the base
  static_assert(kBytes <= 113 * 1024, "two CTAs per SM");
};

// mbarrier slots: full[s] = s, empty[s] = 8 + s (s < 8), then
enum : int {
  kBarFull = 0,     // [kStages] gather -> MMA: tile landed
  kBarEmpty = 8,    // [kStages] MMA commit + 4 epilogue warps -> gather: stage free
  kBarSFull = 16,   // [2] MMA commit -> epilogue: S ready
  kBarSEmpty = 18,  // [2] epilogue (128 threads) -> MMA: S read
  kBarQ = 20,       // gather -> MMA: queries landed
  kBarDrain = 21    // MMA commit -> issuer: every UMMA retired
};

__device__ __forceinline__ uint32_t swz128(uint32_t row, uint32_t chunk) {
  return row * 128u + (((chunk ^ row) & 7u) << 4);
}

// One TMA box: box_rows cache rows (128 e4m3 values each) of one block into
// 128-byte-swizzled shared memory, counted on `bar`.
__device__ __forceinline__ void tma_load_rows(uint32_t dst, const CUtensorMap* map, int row, int blk,
                                              uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(row), "r"(blk), "r"(bar)
      : "memory");
}

template <int H, int NEXT_N>
__global__ void __launch_bounds__(kThreads, 1) indexer_logits_kernel(const __grid_constant__ Params p,
                                                                     const __grid_constant__ CUtensorMap kv_map) {
  constexpr int N = H * NEXT_N;
  using L = Layout<N>;
  constexpr int kStages = L::kStages;
  constexpr uint32_t kSmQ = L::kQ, kSmStage = L::kStage, kSmScale = L::kScale, kSmW = L::kW,
                     kSmBar = L::kBar, kSmMisc = L::kMisc, kSmBt = L::kBt;
  constexpr uint32_t kTmemCols = 2 * N <= 64 ? 64u : (2 * N <= 128 ? 128u : (2 * N <= 256 ? 256u : 512u));
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t sb = (raw + 1023u) & ~1023u;
  uint8_t* const gb = smem_raw + (sb - raw);
  float* const w_sm = reinterpret_cast<float*>(gb + kSmW);
  const float* const scale_sm = reinterpret_cast<const float*>(gb + kSmScale);
  uint32_t* const misc = reinterpret_cast<uint32_t*>(gb + kSmMisc);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(misc + 1);
  auto bar = [sb](int i) -> uint32_t { return sb + kSmBar + 8u * static_cast<uint32_t>(i); };

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int b = blockIdx.y;
  const long long span = static_cast<long long>(kTile) * p.tiles_per_cta;
  const long long p0 = static_cast<long long>(blockIdx.x) * span;
  const long long chunk_end = p0 + span < p.max_model_len
                                  ? p0 + span
                                  : static_cast<long long>(p.max_model_len);
  const long long row0 = static_cast<long long>(b) * NEXT_N;
  // Programmatic dependent launch: the logits and the inputs may come from
  // the previous kernel in the stream. Dependents may launch at once: they
  // wait in turn for this grid to finish.
  griddep_wait();
  griddep_launch_dependents();
  // visible length of each of the request's tokens, and the longest
  long long lens[NEXT_N];
  long long ctx = 0;
#pragma unroll
  for (int j = 0; j < NEXT_N; ++j) {
    lens[j] = p.per_row_lens ? static_cast<long long>(p.ctx_lens[row0 + j])
                             : static_cast<long long>(p.ctx_lens[b]) - NEXT_N + j + 1;
    if (lens[j] > ctx) ctx = lens[j];
  }
  const long long seen_end = ctx < chunk_end ? ctx : chunk_end;
  const int n_tiles = seen_end > p0 ? static_cast<int>((seen_end - p0 + kTile - 1) / kTile) : 0;

  // positions [first, chunk_end) of token j that it does not see -> -inf
  auto clean_tail = [&](long long first) {
    if (!p.clean) return;
    for (int j = 0; j < NEXT_N; ++j) {
      const long long lj = lens[j];
      long long s = lj > first ? lj : first;
      if (s < p0) s = p0;
      float* const out = p.logits + (row0 + j) * p.logits_stride;
      for (long long q = s + tid; q < chunk_end; q += kThreads) out[q] = -INFINITY;
    }
  };
  if (n_tiles == 0) {
    clean_tail(p0);
    return;
  }

  // ------------------------------------------------------------------ setup
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(kBarFull + s), 1);
      mbar_init(bar(kBarEmpty + s), 1 + 4);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(kBarSFull + s), 1);
      mbar_init(bar(kBarSEmpty + s), 128);
    }
    mbar_init(bar(kBarQ), kGatherThreads);
    mbar_init(bar(kBarDrain), 1);
    misc[1] = 0;
    fence_mbarrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(sb + kSmMisc, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc[0];

  if (warp >= kGatherWarp0) {
    // ================= gather =================
    const int gt = tid - 32 * kGatherWarp0;
    for (int u = gt; u < N * 8; u += kGatherThreads) {
      const int n = u >> 3, c = u & 7;
      const int j = n / H, h = n % H;
      const uint8_t* src = p.q + ((row0 + j) * H + h) * kD + c * 16;
      cp_async_16(sb + kSmQ + swz128(n, c), src, 16u);
    }
    cp_async_mbar_arrive_noinc(bar(kBarQ));
    // the block ids of every column this CTA reads, once: -1 for a column
    // past the table or a block past the cache (nothing is read there)
    int32_t* const bt_sm = reinterpret_cast<int32_t*>(gb + kSmBt);
    const long long col0 = p0 >> p.log2_block;
    const int ncols = static_cast<int>(((seen_end - 1) >> p.log2_block) - col0 + 1);
    const int32_t* bt = p.block_table + static_cast<long long>(b) * p.bt_stride;
    bool bad = false;
    for (int c = gt; c < ncols; c += kGatherThreads) {
      const long long col = col0 + c;
      long long blk = col < p.max_blocks ? bt[col] : -1;
      if (blk < 0 || blk >= p.num_blocks) {
        bad = true;
        blk = -1;
      }
      bt_sm[c] = static_cast<int32_t>(blk);
    }
    if (bad) atomicOr(&g_indexer_status, kStatusBadBlock);
    named_bar_sync(2, kGatherThreads);
    const long long bmask = (1ll << p.log2_block) - 1;
    const int nbox = kTile / p.box_rows;
    const uint32_t box_bytes = static_cast<uint32_t>(p.box_rows) * kD;
    // block id of the box starting at position P (-1: nothing to read)
    auto box_block = [&](long long P) -> int32_t {
      return P >= ctx ? -1 : bt_sm[(P >> p.log2_block) - col0];
    };
    // tile t is issued by gather warp t % 3, so up to three tiles' loads are
    // being issued at once (a TMA issue holds its thread for a while)
    const int gw = gt >> 5;
    for (int t = gw; t < n_tiles; t += kGatherThreads / 32) {
      const int s = t % kStages;
      if (t >= kStages &&
          !mbar_wait_bounded(bar(kBarEmpty + s), ((t / kStages) - 1) & 1, abort_flag, p.timeout_ns))
        break;
      const uint32_t stage = sb + kSmStage + s * kStageBytes;
      const uint32_t scales = sb + kSmScale + s * kScaleBytes;
      const long long pt = p0 + static_cast<long long>(t) * kTile;
      // boxes with nothing to read (past the context, or a bad block) are
      // zero-filled here, so stale rows never reach the tensor core
      bool any_zero = false;
      for (int k = 0; k < nbox; ++k) {
        if (box_block(pt + static_cast<long long>(k) * p.box_rows) >= 0) continue;
        any_zero = true;
        for (uint32_t o = 16u * lane; o < box_bytes; o += 16u * 32u)
          sts_v4(stage + k * box_bytes + o, make_uint4(0u, 0u, 0u, 0u));
        for (uint32_t o = 16u * lane; o < 4u * p.box_rows; o += 16u * 32u)
          sts_v4(scales + 4u * k * p.box_rows + o, make_uint4(0u, 0u, 0u, 0u));
      }
      if (any_zero) fence_proxy_async_smem();   // these stores -> the tensor core's reads
      __syncwarp();
      if (lane == 0) {
        uint32_t bytes = 0;
        for (int k = 0; k < nbox; ++k)
          if (box_block(pt + static_cast<long long>(k) * p.box_rows) >= 0) bytes += box_bytes + 4u * p.box_rows;
        mbar_arrive_expect_tx(bar(kBarFull + s), bytes);
        for (int k = 0; k < nbox; ++k) {
          const long long P = pt + static_cast<long long>(k) * p.box_rows;
          const int32_t blk = box_block(P);
          if (blk < 0) continue;
          const int row = static_cast<int>(P & bmask);
          tma_load_rows(stage + k * box_bytes, &kv_map, row, blk, bar(kBarFull + s));
          bulk_load_g2s(scales + 4u * k * p.box_rows,
                        p.kv + static_cast<long long>(blk) * p.block_bytes +
                            static_cast<long long>(p.block_size) * kD + row * 4,
                        4u * p.box_rows, bar(kBarFull + s));
        }
      }
      __syncwarp();
    }
  } else if (warp == kMmaWarp) {
    // ================= UMMA issue (one lane) =================
    if (lane == 0) {
      constexpr uint32_t kIdesc = idesc_e4m3_f32(kTile, N);
      bool ok = mbar_wait_bounded(bar(kBarQ), 0, abort_flag, p.timeout_ns);
      for (int t = 0; ok && t < n_tiles; ++t) {
        const int s = t % kStages;
        if (!mbar_wait_bounded(bar(kBarFull + s), (t / kStages) & 1, abort_flag, p.timeout_ns)) break;
        if (t >= 2 &&
            !mbar_wait_bounded(bar(kBarSEmpty + (t & 1)), ((t >> 1) - 1) & 1, abort_flag, p.timeout_ns))
          break;
        fence_proxy_async_smem();   // cp.async writes -> tensor-core reads
        tc_fence_after();
        const uint32_t stage = sb + kSmStage + s * kStageBytes;
#pragma unroll
        for (int kk = 0; kk < kD / 32; ++kk)
          umma_e4m3(tmem + static_cast<uint32_t>((t & 1) * N), sdesc_sw128(stage + kk * 32u, 16, 1024),
                    sdesc_sw128(sb + kSmQ + kk * 32u, 16, 1024), kIdesc, kk > 0 ? 1u : 0u);
        umma_commit(bar(kBarSFull + (t & 1)));
        umma_commit(bar(kBarEmpty + s));
      }
      umma_commit(bar(kBarDrain));
      volatile int own = 0;
      mbar_wait_bounded(bar(kBarDrain), 0, &own, p.timeout_ns);
    }
    __syncwarp();
  } else {
    // ================= epilogue (warps 0-3, thread = position) =================
    for (int i = tid; i < N; i += 128) w_sm[i] = p.weights[row0 * H + i];
    named_bar_sync(1, 128);
    const uint32_t lane_base = static_cast<uint32_t>(32 * warp) << 16;
    for (int t = 0; t < n_tiles; ++t) {
      if (!mbar_wait_bounded(bar(kBarSFull + (t & 1)), (t >> 1) & 1, abort_flag, p.timeout_ns)) break;
      tc_fence_after();
      const int s = t % kStages;
      const float sc = scale_sm[s * kTile + tid];
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kBarEmpty + s));   // this warp has read its scales
      const long long P = p0 + static_cast<long long>(t) * kTile + tid;
#pragma unroll
      for (int j = 0; j < NEXT_N; ++j) {
        float acc = 0.f;
#pragma unroll
        for (int c0 = 0; c0 < H; c0 += 32) {
          float v[32];
          tmem_ld_32x32b_x32(tmem + lane_base + static_cast<uint32_t>((t & 1) * N + j * H + c0), v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) acc = fmaf(fmaxf(v[i], 0.f), w_sm[j * H + c0 + i], acc);
        }
        const long long lj = lens[j];
        float* const out = p.logits + (row0 + j) * p.logits_stride;
        if (P < lj) out[P] = acc * sc;
        else if (p.clean && P < chunk_end) out[P] = -INFINITY;
      }
      tc_fence_before();
      mbar_arrive(bar(kBarSEmpty + (t & 1)));
    }
  }

  // positions past the last tile this CTA computed
  clean_tail(p0 + static_cast<long long>(n_tiles) * kTile);
  cp_async_wait_all();
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  if (tid == 0 && *abort_flag) atomicOr(&g_indexer_status, kStatusTimeout);
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's tensor-map encoder, fetched once through the runtime (the
// library links only the CUDA runtime).
EncodeTiledFn encoder() {
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

// 3-D view of the cache values: 128 bytes x block_size rows x num_blocks,
// boxes of min(block_size, 128) rows of one block, 128-byte swizzle (the
// layout the UMMA descriptors read).
// Launch with programmatic stream serialization, so this grid may begin
// launching while the previous kernel in the stream drains; the kernel's
// griddepcontrol.wait, before its first global access, keeps the order.
template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

bool make_kv_map(CUtensorMap* map, const Params& p) {
  EncodeTiledFn enc = encoder();
  if (enc == nullptr) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(p.block_size),
                              static_cast<cuuint64_t>(p.num_blocks)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(p.block_bytes)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(kD), static_cast<cuuint32_t>(p.box_rows), 1u};
  const cuuint32_t elem[3] = {1u, 1u, 1u};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t*>(p.kv), dims, strides, box,
             elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int H, int NEXT_N>
cudaError_t launch(const Params& p, const CUtensorMap& map, int B, cudaStream_t stream) {
  // once per device and instantiation, under a lock (first calls may come
  // from several host threads)
  static std::atomic<bool> attr_set[64] = {};
  static std::mutex attr_mutex;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64 && !attr_set[dev].load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(attr_mutex);
    if (!attr_set[dev].load(std::memory_order_relaxed)) {
      e = cudaFuncSetAttribute(indexer_logits_kernel<H, NEXT_N>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(Layout<H * NEXT_N>::kBytes));
      if (e != cudaSuccess) return e;
      attr_set[dev].store(true, std::memory_order_release);
    }
  }
  const int span = kTile * p.tiles_per_cta;
  const dim3 grid(static_cast<unsigned>((p.max_model_len + span - 1) / span),
                  static_cast<unsigned>(B));
  return launch_pdl(indexer_logits_kernel<H, NEXT_N>, grid, dim3(kThreads), Layout<H * NEXT_N>::kBytes,
                    stream, p, map);
}

bool aligned(const void* ptr, uintptr_t a) { return (reinterpret_cast<uintptr_t>(ptr) & (a - 1)) == 0; }

}  // namespace indexer
}  // namespace glm53

using namespace glm53::indexer;

extern "C" int glm53_indexer_logits(const void* q, const void* kv_cache, const float* weights,
                                    const int32_t* context_lens, int per_token_lens,
                                    const int32_t* block_table,
                                    int64_t B, int next_n, int64_t H, int64_t head_dim,
                                    int64_t num_blocks, int64_t block_size, int64_t block_bytes,
                                    int64_t bt_stride, int64_t max_blocks, float* logits,
                                    int64_t logits_stride, int64_t max_model_len, int clean,
                                    void* stream) {
  if (B < 0 || B > 65535 || num_blocks < 0 || max_blocks < 0 || max_model_len < 0 ||
      max_model_len > 0x7FFFFFFF || logits_stride < max_model_len || bt_stride < max_blocks)
    return GLM53_ERR_RANK;
  if (head_dim != kD) return GLM53_ERR_HEAD_DIM;
  if ((H != 32 && H != 64) || (next_n != 1 && next_n != 2 && next_n != 4)) return GLM53_ERR_HEADS;
  if (block_size < 16 || block_size > 1024 || (block_size & (block_size - 1)) ||
      block_bytes < block_size * (kD + 4) || block_bytes % 16)
    return GLM53_ERR_RANK;
  if (B == 0 || max_model_len == 0) return GLM53_OK;
  if (q == nullptr || kv_cache == nullptr || weights == nullptr || context_lens == nullptr ||
      block_table == nullptr || logits == nullptr)
    return GLM53_ERR_ALIGN;
  if (!aligned(q, 16) || !aligned(kv_cache, 16) || !aligned(weights, 4) || !aligned(logits, 4) ||
      !aligned(context_lens, 4) || !aligned(block_table, 4))
    return GLM53_ERR_ALIGN;
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return GLM53_ERR_CUDA;
  if (major != 10) return GLM53_ERR_DEVICE;
  Params p;
  p.q = static_cast<const uint8_t*>(q);
  p.kv = static_cast<const uint8_t*>(kv_cache);
  p.weights = weights;
  p.ctx_lens = context_lens;
  p.per_row_lens = per_token_lens ? 1 : 0;
  p.block_table = block_table;
  p.bt_stride = bt_stride;
  p.block_bytes = block_bytes;
  p.num_blocks = num_blocks;
  p.logits = logits;
  p.logits_stride = logits_stride;
  p.block_size = static_cast<int>(block_size);
  p.log2_block = 0;
  while ((1ll << p.log2_block) < block_size) ++p.log2_block;
  p.box_rows = block_size < kTile ? static_cast<int>(block_size) : kTile;
  p.max_blocks = static_cast<int>(max_blocks);
  p.max_model_len = static_cast<int>(max_model_len);
  p.clean = clean ? 1 : 0;
  // 1024 positions per CTA, halved (down to 256) while the launch would have
  // fewer CTAs than SMs: a small batch then spreads over more SMs (16
  // requests x 8192 positions: 10.5 -> 9.0 us)
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return GLM53_ERR_CUDA;
  p.tiles_per_cta = kMaxTilesPerCta;
  while (p.tiles_per_cta > 2 &&
         B * ((max_model_len + kTile * p.tiles_per_cta - 1) / (kTile * p.tiles_per_cta)) < sms)
    p.tiles_per_cta /= 2;
  p.timeout_ns = 1000000000ull;
  if (num_blocks == 0 || num_blocks > 0xFFFFFFFFll) return GLM53_ERR_RANK;
  alignas(64) CUtensorMap map;
  if (!make_kv_map(&map, p)) return GLM53_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int b = static_cast<int>(B);
  cudaError_t e;
  if (H == 32) {
    e = next_n == 1 ? launch<32, 1>(p, map, b, s)
                    : (next_n == 2 ? launch<32, 2>(p, map, b, s) : launch<32, 4>(p, map, b, s));
  } else {
    e = next_n == 1 ? launch<64, 1>(p, map, b, s)
                    : (next_n == 2 ? launch<64, 2>(p, map, b, s) : launch<64, 4>(p, map, b, s));
  }
  return e == cudaSuccess ? GLM53_OK : GLM53_ERR_CUDA;
}

extern "C" int glm53_indexer_status(uint32_t* status, int clear) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_indexer_status, sizeof(v)) != cudaSuccess) return GLM53_ERR_CUDA;
  if (status) *status = v;
  if (clear) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(g_indexer_status, &zero, sizeof(zero)) != cudaSuccess) return GLM53_ERR_CUDA;
  }
  return GLM53_OK;
}
