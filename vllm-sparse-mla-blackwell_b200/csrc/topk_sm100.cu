// Per-row top-k of the indexer's logits, sm_100a: the step that turns the
// sparse-attention indexer's scores into the request-local top-k positions the
// attention consumes (vLLM's topk_indices_buffer). Same contract as vLLM
// 0.22.0's top_k_per_row_decode / top_k_per_row_prefill (vllm/_custom_ops.py:
// 2799-2840, called from vllm/model_executor/layers/sparse_attn_indexer.py:
// 247-256 and 351-360):
//
//   row r covers logits[r, start, end):
//     decode:  start = 0, end = seq_lens[r / next_n] - next_n + r % next_n + 1
//     prefill: start = row_starts[r], end = row_ends[r]
//   len = end - start <= k: out[r] = 0, 1, ..., len - 1, then -1 up to k;
//   otherwise out[r] = the positions (relative to start) of the k largest
//   values, in no particular order; among values equal to the k-th largest,
//   which ones are taken is unspecified. Values compare by IEEE order with
//   +NaN above +inf.
//
// Design: one CTA of 512 threads per row, radix selection on order-preserving
// 32-bit keys. The row goes through shared memory in chunks of up to 32K
// values, each brought in by one bulk copy (plus plain loads for its ragged
// ends); a row that fits in one chunk is loaded once.
//   1. Histogram of the top 11 key bits over the row (four copies, so shared
//      atomics collide across four warps at most); a block-wide suffix scan
//      finds the bin d0 holding the k-th largest key. The row passes read
//      shared memory in 16-byte vectors: in each sweep of 8192 values, warp w
//      reads the 512 values from 512 w, lane l the words 4 l + 128 q + (0..3)
//      for q = 0..3, so each warp load covers 512 contiguous bytes and a
//      thread has its 16 values in flight at once.
//   2. One pass over the row writes every position whose top bits are above
//      d0 and gathers the keys in bin d0 (typically a few percent of the row)
//      with their positions as candidates; each thread counts its share, and
//      a block scan of the counts places every write without atomics or
//      per-element warp votes.
//   3. The remaining 21 bits are resolved on the candidates alone (10- and
//      11-bit digits, stopping as soon as a whole bin is taken), and the
//      candidates above the threshold plus the first of those equal to it
//      are written.
// A row whose bin d0 holds more than kCand keys (heavy ties) resolves the
// remaining bits with passes over the whole row instead.
//
// Small batches of long rows (12K values and more, up to 4 rows per 4 SMs)
// share each row over a cluster of 2 or 4 CTAs instead (topk_cluster_kernel,
// below): the same steps, each CTA on its slice of the row.

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <mutex>
#include <utility>

#include "glm53_sparse_mla.h"

namespace glm53 {
namespace topk {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kBins0 = 2048;              // first digit: key bits 31..21
constexpr int kBins = 256;                // candidate digits: 8 bits
constexpr int kHists = 4;                 // warp w adds into first-digit histogram w % kHists
constexpr int kChunk = 32 * 1024;         // keys held in shared memory at a time (4 sweeps)
constexpr int kCand = 4096;               // candidates (keys in the threshold bin) kept
constexpr int kMaxTopk = 16384;
constexpr long long kSpecMax = 16 * 1024;  // decode rows this wide are loaded before their length is known
constexpr unsigned kStatusTimeout = 1u;

__device__ unsigned int g_topk_status = 0;

struct Params {
  const float* logits;
  long long stride0;                // elements between rows
  long long num_rows;
  const int32_t* seq_lens;          // decode (with next_n), or nullptr
  int next_n;
  const int32_t* row_starts;        // prefill, or nullptr
  const int32_t* row_ends;
  int32_t* out;
  long long out_stride;
  int k;
  unsigned long long timeout_ns;
};

// shared memory (32-bit words): keys (+4 alignment pad), kHists first-digit
// histograms, the merged histogram, candidate keys and positions, per-warp
// counts, control words, one mbarrier
constexpr size_t kSmemWords = kChunk + 4 + kHists * kBins0 + kBins0 + 2 * kCand + 4 * kWarps + 16;
constexpr size_t kSmemBytes = sizeof(uint32_t) * kSmemWords + 16;

__device__ __forceinline__ uint32_t order_key(const float x) {
  const uint32_t b = __float_as_uint(x);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Block-wide search over `nb` bins (a multiple of kThreads, or kBins with
// threads >= kBins idle): finds the digit d with count(> d) < need <=
// count(>= d) and leaves d, count(> d) and count(d) in ctl[0..2].
__device__ __forceinline__ void find_digit(const uint32_t* hist, int nb, uint32_t need,
                                           uint32_t* wsum, uint32_t* ctl) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int bpt = nb >= kThreads ? nb / kThreads : 1;
  const bool owns = tid * bpt < nb;
  uint32_t s = 0;
  if (owns)
    for (int j = 0; j < bpt; ++j) s += hist[bpt * tid + j];
  uint32_t incl = s;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t v = __shfl_down_sync(0xFFFFFFFFu, incl, off);
    if (lane + off < 32) incl += v;
  }
  if (lane == 0) wsum[warp] = incl;
  __syncthreads();
  for (int w = warp + 1; w < kWarps; ++w) incl += wsum[w];
  uint32_t above = incl - s;
  if (owns && above < need && need <= incl) {
    for (int j = bpt - 1; j >= 0; --j) {
      const uint32_t c = hist[bpt * tid + j];
      if (above + c >= need) {
        ctl[0] = static_cast<uint32_t>(bpt * tid + j);
        ctl[1] = above;
        ctl[2] = c;
        break;
      }
      above += c;
    }
  }
  __syncthreads();
}

// find_digit over the first digit, reading the kHists per-warp histogram
// copies directly: thread t sums bins 4t..4t+3 of every copy (one 16-byte
// load per copy), which saves a merge pass and its barrier.
template <int NC = kHists>
__device__ __forceinline__ void find_digit0(const uint32_t* whist, uint32_t need, uint32_t* wsum,
                                            uint32_t* ctl) {
  static_assert(kBins0 == 4 * kThreads, "four first-digit bins per thread");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t c[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int w = 0; w < NC; ++w) {
    const uint4 v = *reinterpret_cast<const uint4*>(whist + w * kBins0 + 4 * tid);
    c[0] += v.x;
    c[1] += v.y;
    c[2] += v.z;
    c[3] += v.w;
  }
  const uint32_t s = c[0] + c[1] + c[2] + c[3];
  uint32_t incl = s;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t v = __shfl_down_sync(0xFFFFFFFFu, incl, off);
    if (lane + off < 32) incl += v;
  }
  if (lane == 0) wsum[warp] = incl;
  __syncthreads();
  for (int w = warp + 1; w < kWarps; ++w) incl += wsum[w];
  uint32_t above = incl - s;
  if (above < need && need <= incl) {
#pragma unroll
    for (int j = 3; j >= 0; --j) {
      if (above + c[j] >= need) {
        ctl[0] = static_cast<uint32_t>(4 * tid + j);
        ctl[1] = above;
        ctl[2] = c[j];
        break;
      }
      above += c[j];
    }
  }
  __syncthreads();
}

// Block-wide exclusive prefix sums of two per-thread counts (thread order):
// returns this thread's offsets and the block totals. Uses scratch[2 * kWarps].
__device__ __forceinline__ void block_scan2(uint32_t a, uint32_t b, uint32_t* scratch,
                                            uint32_t& ea, uint32_t& eb, uint32_t& ta,
                                            uint32_t& tb) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t sa = a, sb = b;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t xa = __shfl_up_sync(0xFFFFFFFFu, sa, off);
    const uint32_t xb = __shfl_up_sync(0xFFFFFFFFu, sb, off);
    if (lane >= off) {
      sa += xa;
      sb += xb;
    }
  }
  if (lane == 31) {
    scratch[warp] = sa;
    scratch[kWarps + warp] = sb;
  }
  __syncthreads();
  uint32_t pa = 0, pb = 0;
  ta = tb = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const uint32_t wa = scratch[w], wb = scratch[kWarps + w];
    if (w < warp) {
      pa += wa;
      pb += wb;
    }
    ta += wa;
    tb += wb;
  }
  ea = pa + sa - a;
  eb = pb + sb - b;
  __syncthreads();   // scratch may be reused right after
}

// The k_rem largest of the threshold bin's keys (bits 20..0 still open),
// from the n candidates (keys and positions) held in shared memory, written
// to out_c[0, k_rem) (n_above of them strictly above the final prefix first,
// then the first k_rem - n_above equal to it). Every thread of the block
// calls it; hist and whist are free scratch (2048 words each).
__device__ __forceinline__ void finish_candidates(const uint32_t* cand_key, const uint32_t* cand_pos,
                                                  uint32_t c0_count, uint32_t d0, int k, uint32_t n_gt0,
                                                  uint32_t k_rem, int32_t* out_c, uint32_t* hist,
                                                  uint32_t* whist, uint32_t* wsum, uint32_t* wcnt,
                                                  uint32_t* ctl) {
  const int tid = threadIdx.x;
  // two digits over bits 20..0 (bits 20..11 in 1024 bins, then 10..0 in
  // 2048), each with its own histogram, zeroed together up front. ctl and
  // wsum are rewritten only after the next pass's first barrier, which every
  // thread reaches after reading them, so a pass needs no closing barrier.
  uint32_t prefix = d0 << 21, mask = 0xFFE00000u;
  bool settled = c0_count == k_rem;
  const int n = static_cast<int>(c0_count);
  if (!settled) {
    for (int i = tid; i < kBins0; i += kThreads) {
      hist[i] = 0;
      whist[i] = 0;
    }
    __syncthreads();
  }
#pragma unroll 1
  for (int pss = 0; pss < 2 && !settled; ++pss) {
    const int shift = pss == 0 ? 11 : 0;
    const uint32_t width = pss == 0 ? 0x3FFu : 0x7FFu;
    uint32_t* const h = pss == 0 ? hist : whist;
    for (int i = tid; i < n; i += kThreads) {
      const uint32_t u = cand_key[i];
      if ((u & mask) == prefix) atomicAdd(&h[(u >> shift) & width], 1u);
    }
    __syncthreads();
    find_digit(h, static_cast<int>(width) + 1, k_rem, wsum, ctl);
    prefix |= ctl[0] << shift;
    mask |= width << shift;
    k_rem -= ctl[1];
    settled = ctl[2] == k_rem;
  }
  // candidates above the prefix, then the first k_rem equal to it: per-thread
  // counts over a strided share of the candidates and a block scan
  const uint32_t n_above = static_cast<uint32_t>(k) - n_gt0 - k_rem;
  uint32_t ng = 0, ne = 0;
  for (int i = tid; i < n; i += kThreads) {
    const uint32_t u = cand_key[i] & mask;
    ng += u > prefix;
    ne += u == prefix;
  }
  uint32_t og, oe, tg, te;
  block_scan2(ng, ne, wcnt, og, oe, tg, te);
  for (int i = tid; i < n; i += kThreads) {
    const uint32_t u = cand_key[i] & mask;
    if (u > prefix) {
      out_c[og++] = static_cast<int32_t>(cand_pos[i]);
    } else if (u == prefix) {
      if (oe < k_rem) out_c[n_above + oe] = static_cast<int32_t>(cand_pos[i]);
      ++oe;
    }
  }
}

// One row by one CTA (every thread of the block), shared memory `smem` of
// kSmemBytes: the whole algorithm, rows of any length.
__device__ __forceinline__ void topk_row_single(const Params& p, long long row, uint32_t* smem) {
  uint32_t* const keys_raw = smem;                               // [kChunk + 4]
  uint32_t* const whist = smem + kChunk + 4;                     // [kHists][kBins0]
  uint32_t* const hist = whist + kHists * kBins0;                // [kBins0]
  uint32_t* const cand_key = hist + kBins0;                      // [kCand]
  uint32_t* const cand_pos = cand_key + kCand;                   // [kCand]
  uint32_t* const wcnt = cand_pos + kCand;                       // [4][kWarps]
  uint32_t* const wsum = wcnt + 2 * kWarps;                      // [kWarps] (scan scratch)
  uint32_t* const ctl = wcnt + 4 * kWarps;                       // [8]
  const uint32_t bar = static_cast<uint32_t>(__cvta_generic_to_shared(ctl + 8));

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  // The row goes through shared memory in chunks of kChunk values (a row
  // that fits is loaded once): each chunk's 16-byte aligned interior by one
  // bulk copy, its ragged ends (< 4 values each) by plain loads. kChunk is a
  // multiple of 4, so every chunk starts at the same offset within 16 bytes,
  // and `pad` puts its interior on a 16-byte boundary: keys[i] holds value
  // c0 + i, converted to its key in place.
  // A decode row starts at position 0, so when the logits rows are at most
  // kSpecMax values wide the whole row is requested before its length is
  // read: the length load and the row load overlap (one dependent L2 round
  // trip fewer). Wider rows are not, since a row shorter than k would still
  // have to wait for its copy to land before the CTA may exit.
  const bool decode = p.seq_lens != nullptr;
  const long long spec = decode && p.stride0 <= kSpecMax ? p.stride0 : 0;
  auto head_of = [](const float* a) {
    return static_cast<uint32_t>(((16u - (reinterpret_cast<uintptr_t>(a) & 15u)) & 15u) >> 2);
  };
  auto issue_copy = [&](const float* from, long long clen, uint32_t h0, uint32_t* to) {
    // thread 0: the aligned interior of [from, from + clen) into to[h, ...)
    const long long h = h0 < clen ? h0 : clen;
    const uint32_t bytes = static_cast<uint32_t>(((clen - h) / 4) * 4 * 4);
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
    if (bytes > 0)
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
              static_cast<uint32_t>(__cvta_generic_to_shared(to + h))),
          "l"(from + h), "r"(bytes), "r"(bar)
          : "memory");
  };
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (spec > 0) {
      const float* const r0 = p.logits + row * p.stride0;
      issue_copy(r0, spec, head_of(r0), keys_raw + ((4u - head_of(r0)) & 3u));
    }
  }
  long long start, end;
  if (decode) {
    start = 0;
    end = static_cast<long long>(p.seq_lens[row / p.next_n]) - p.next_n + row % p.next_n + 1;
  } else {
    start = p.row_starts[row];
    end = p.row_ends[row];
  }
  const long long len = end > start ? end - start : 0;
  int32_t* const out = p.out + row * p.out_stride;
  const int k = p.k;
  auto wait_copy = [&](uint32_t parity) {
    uint32_t done = 0;
    const uint64_t t0 = now_ns();
    while (true) {
      asm volatile(
          "{\n\t.reg .pred q;\n\tmbarrier.try_wait.parity.acquire.cta.shared::cta.b64 q, [%1], %2;\n\t"
          "selp.u32 %0, 1, 0, q;\n\t}"
          : "=r"(done)
          : "r"(bar), "r"(parity)
          : "memory");
      if (done) break;
      if (now_ns() - t0 > p.timeout_ns) {
        if (tid == 0) atomicOr(&g_topk_status, kStatusTimeout);
        break;
      }
    }
  };
  if (len <= k) {
    for (int i = tid; i < k; i += kThreads) out[i] = i < len ? i : -1;
    if (tid == 0 && spec > 0) wait_copy(0);   // no copy may still target this CTA's shared memory
    return;
  }
  const float* const src = p.logits + row * p.stride0 + start;
  const bool one_chunk = len <= kChunk;
  const uint32_t head = head_of(src);
  uint32_t* const keys = keys_raw + ((4u - head) & 3u);
  __syncthreads();
  uint32_t phase = 0;
  bool spec_left = spec > 0;   // the requested first chunk is consumed once (later passes reload)
  auto load_chunk = [&](long long c0, long long clen) {
    if (c0 == 0 && spec_left) {
      spec_left = false;
      // the decode row's first chunk, requested above for `spec` values:
      // its ragged ends, then (an invalid row longer than stride0 only)
      // whatever lies past it
      const long long h = head < spec ? head : spec;
      const long long tail0 = h + ((spec - h) / 4) * 4;
      if (tid < h) keys[tid] = __float_as_uint(src[tid]);
      if (tid < spec - tail0) keys[tail0 + tid] = __float_as_uint(src[tail0 + tid]);
      for (long long i = spec + tid; i < clen; i += kThreads) keys[i] = __float_as_uint(src[i]);
      wait_copy(phase);
      phase ^= 1u;
      __syncthreads();
      return;
    }
    const long long h = head < clen ? head : clen;
    const long long tail0 = h + ((clen - h) / 4) * 4;
    if (tid == 0) issue_copy(src + c0, clen, head, keys);
    if (tid < h) keys[tid] = __float_as_uint(src[c0 + tid]);
    if (tid < clen - tail0) keys[tail0 + tid] = __float_as_uint(src[c0 + tail0 + tid]);
    wait_copy(phase);
    phase ^= 1u;
    __syncthreads();
  };

  // ---- first digit (11 bits) over the whole row; keys are formed in place
  uint32_t* const my_hist = whist + (warp % kHists) * kBins0;
  for (int i = tid; i < kHists * kBins0; i += kThreads) whist[i] = 0;
  __syncthreads();
  // keys[i] is word off + i of the 16-byte aligned keys_raw; a chunk spans
  // words [off, off + clen)
  const int off = static_cast<int>((4u - head) & 3u);
  const int lane = tid & 31;
#pragma unroll 1
  for (long long c0 = 0; c0 < len; c0 += kChunk) {
    const long long clen = len - c0 < kChunk ? len - c0 : kChunk;
    load_chunk(c0, clen);
    const int W = off + static_cast<int>(clen);
#pragma unroll 1
    for (int s0 = 0; s0 < W; s0 += 16 * kThreads) {
      const int base = s0 + 512 * warp + 4 * lane;
      uint4 v[4] = {};
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (base + 128 * q < W) v[q] = *reinterpret_cast<const uint4*>(keys_raw + base + 128 * q);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int a = base + 128 * q;
        if (a < W) {
          uint32_t w[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            w[c] = order_key(__uint_as_float(w[c]));
            if (a + c >= off && a + c < W) atomicAdd(&my_hist[w[c] >> 21], 1u);
          }
          if (a >= off && a + 4 <= W) {
            *reinterpret_cast<uint4*>(keys_raw + a) = make_uint4(w[0], w[1], w[2], w[3]);
          } else {
#pragma unroll
            for (int c = 0; c < 4; ++c)
              if (a + c >= off && a + c < W) keys_raw[a + c] = w[c];
          }
        }
      }
    }
    __syncthreads();
  }
  find_digit0(whist, static_cast<uint32_t>(k), wsum, ctl);
  const uint32_t d0 = ctl[0];
  uint32_t k_rem = static_cast<uint32_t>(k) - ctl[1];
  const uint32_t c0_count = ctl[2];
  const uint32_t n_gt0 = ctl[1];
  __syncthreads();

  // ---- one pass over the row: positions with a first digit above d0 go out
  // (slots [0, n_gt0)); those equal to d0 are the candidates. Thread t takes
  // positions t, t + kThreads, ... of each chunk (conflict-free shared reads),
  // counts its two classes, and a block scan of the counts gives it the
  // slots it writes, in order; no atomics. The output order is thread-major,
  // which the contract leaves open.
  const bool keep = c0_count <= static_cast<uint32_t>(kCand);
  uint32_t gt_base = 0, eq_base = 0;
#pragma unroll 1
  for (long long c0 = 0; c0 < len; c0 += kChunk) {
    const long long clen = len - c0 < kChunk ? len - c0 : kChunk;
    if (!one_chunk) {
      load_chunk(c0, clen);
      for (long long i = tid; i < clen; i += kThreads) keys[i] = order_key(__uint_as_float(keys[i]));
      __syncthreads();
    }
    const int W = off + static_cast<int>(clen);
    uint32_t ng = 0, ne = 0;
#pragma unroll 1
    for (int s0 = 0; s0 < W; s0 += 16 * kThreads) {
      const int base = s0 + 512 * warp + 4 * lane;
      uint4 v[4] = {};
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (base + 128 * q < W) v[q] = *reinterpret_cast<const uint4*>(keys_raw + base + 128 * q);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int a = base + 128 * q;
        const uint32_t w[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const bool ok = a + c >= off && a + c < W;
          const uint32_t dg = w[c] >> 21;
          ng += ok && dg > d0;
          ne += ok && dg == d0;
        }
      }
    }
    uint32_t og, oe, tg, te;
    block_scan2(ng, ne, wcnt, og, oe, tg, te);
    og += gt_base;
    oe += eq_base;
#pragma unroll 1
    for (int s0 = 0; s0 < W; s0 += 16 * kThreads) {
      const int base = s0 + 512 * warp + 4 * lane;
      uint4 v[4] = {};
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (base + 128 * q < W) v[q] = *reinterpret_cast<const uint4*>(keys_raw + base + 128 * q);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int a = base + 128 * q;
        const uint32_t w[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (a + c < off || a + c >= W) continue;
          const uint32_t u = w[c];
          const uint32_t dg = u >> 21;
          const long long i = a + c - off;
          if (dg > d0) {
            out[og++] = static_cast<int32_t>(c0 + i);
          } else if (dg == d0) {
            if (keep) {
              cand_key[oe] = u;
              cand_pos[oe] = static_cast<uint32_t>(c0 + i);
            } else if (c0_count == k_rem) {
              out[n_gt0 + oe] = static_cast<int32_t>(c0 + i);   // the whole bin is taken
            }
            ++oe;
          }
        }
      }
    }
    gt_base += tg;
    eq_base += te;
    __syncthreads();
  }
  if (c0_count == k_rem && !keep) return;   // the whole threshold bin went out above

  // ---- the k_rem largest of the threshold bin's keys (bits 20..0 still open)
  int32_t* const out_c = out + n_gt0;
  if (keep) {
    finish_candidates(cand_key, cand_pos, c0_count, d0, k, n_gt0, k_rem, out_c, hist, whist, wsum, wcnt, ctl);
    return;
  }

  // ---- too many candidates to keep: 8-bit digit passes over the whole row
  // for bits 20..0, then one output pass for the bin (rare: a row where more
  // than kCand values share the top 11 key bits with the k-th largest)
  uint32_t prefix = d0 << 21, mask = 0xFFE00000u;
  const int shifts[3] = {13, 5, 0};
  const uint32_t widths[3] = {0xFFu, 0xFFu, 0x1Fu};
  bool settled = false;
#pragma unroll 1
  for (int pss = 0; pss < 3 && !settled; ++pss) {
    for (int i = tid; i < kBins; i += kThreads) hist[i] = 0;
    __syncthreads();
#pragma unroll 1
    for (long long c0 = 0; c0 < len; c0 += kChunk) {
      const long long clen = len - c0 < kChunk ? len - c0 : kChunk;
      if (!one_chunk) {
        load_chunk(c0, clen);
        for (long long i = tid; i < clen; i += kThreads) keys[i] = order_key(__uint_as_float(keys[i]));
        __syncthreads();
      }
      for (long long i = tid; i < clen; i += kThreads) {
        const uint32_t u = keys[i];
        if ((u & mask) == prefix) atomicAdd(&hist[(u >> shifts[pss]) & widths[pss]], 1u);
      }
      __syncthreads();
    }
    find_digit(hist, kBins, k_rem, wsum, ctl);
    prefix |= ctl[0] << shifts[pss];
    mask |= widths[pss] << shifts[pss];
    k_rem -= ctl[1];
    settled = ctl[2] == k_rem;
    __syncthreads();
  }
  const uint32_t n_above = static_cast<uint32_t>(k) - n_gt0 - k_rem;
  uint32_t g_base = 0, e_base = 0;
#pragma unroll 1
  for (long long c0 = 0; c0 < len; c0 += kChunk) {
    const long long clen = len - c0 < kChunk ? len - c0 : kChunk;
    if (!one_chunk) {
      load_chunk(c0, clen);
      for (long long i = tid; i < clen; i += kThreads) keys[i] = order_key(__uint_as_float(keys[i]));
      __syncthreads();
    }
    uint32_t ng = 0, ne = 0;
    for (long long i = tid; i < clen; i += kThreads) {
      const uint32_t u = keys[i];
      const bool in_bin = (u & 0xFFE00000u) == (d0 << 21);
      ng += in_bin && (u & mask) > prefix;
      ne += in_bin && (u & mask) == prefix;
    }
    uint32_t og, oe, tg, te;
    block_scan2(ng, ne, wcnt, og, oe, tg, te);
    og += g_base;
    oe += e_base;
    for (long long i = tid; i < clen; i += kThreads) {
      const uint32_t u = keys[i];
      if ((u & 0xFFE00000u) != (d0 << 21)) continue;
      if ((u & mask) > prefix) {
        out_c[og++] = static_cast<int32_t>(c0 + i);
      } else if ((u & mask) == prefix) {
        if (oe < k_rem) out_c[n_above + oe] = static_cast<int32_t>(c0 + i);
        ++oe;
      }
    }
    g_base += tg;
    e_base += te;
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kThreads, 1) topk_per_row_kernel(const Params p) {
  // Programmatic dependent launch: the logits come from the previous kernel
  // in the stream, so wait for it before any global access; dependents may
  // launch at once (they wait in turn for this grid to finish).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ __align__(16) uint32_t smem[];
  topk_row_single(p, blockIdx.x, smem);
}

// ---------------------------------------------------------------------------
// Small batches: one row over a cluster of C CTAs
// ---------------------------------------------------------------------------
// A decode batch has few rows (32 at a 32-sequence decode step), so one CTA
// per row leaves most SMs idle while each row's load, histogram and
// compaction run on one SM. Here C CTAs (a thread-block cluster) share a row:
// CTA c loads, keys, histograms and compacts slice c of it (len / C values),
// and the cluster exchanges the few words it must through distributed shared
// memory:
//   1. CTA 0 reads every CTA's 11-bit histogram, finds the threshold bin d0
//      and sends (d0, count above, count in d0) back;
//   2. every CTA counts its positions above d0 and in d0 and sends the two
//      counts to all; each writes its positions above d0 at its offset,
//      stages its candidates (keys in d0 with positions) and then sends them
//      to CTA 0 in one burst;
//   3. CTA 0 resolves the candidates alone (finish_candidates).
// A row longer than C slices, or whose threshold bin holds more than kCand
// keys (heavy ties), is done by CTA 0 alone with the one-CTA algorithm.
constexpr int kSlice = 32 * 1024;   // values per CTA slice
// shared memory of the cluster kernel (words, as laid out there): it also
// holds the one-CTA layout (kSmemBytes) for the rows CTA 0 does alone
template <int C>
constexpr size_t cluster_smem_bytes() {
  return sizeof(uint32_t) * (kSlice + 4 + kHists * kBins0 + kBins0 + 2 * kCand + 4 * kWarps + 8 + 16 + 2) + 16;
}
static_assert(cluster_smem_bytes<4>() <= 232448, "cluster top-k shared memory");
static_assert(cluster_smem_bytes<2>() >= kSmemBytes, "room for the one-CTA layout");

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
               : "=r"(r)
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))), "r"(rank));
  return r;
}

__device__ __forceinline__ void st_cluster_u32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ uint4 ld_cluster_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared::cluster.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

template <int C>
__global__ void __launch_bounds__(kThreads, 1) topk_cluster_kernel(const Params p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ __align__(16) uint32_t smem[];
  const long long row = blockIdx.x / C;
  const uint32_t rank = blockIdx.x % C;   // clusters are C consecutive CTAs: the cluster rank
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  long long start, end;
  if (p.seq_lens != nullptr) {
    start = 0;
    end = static_cast<long long>(p.seq_lens[row / p.next_n]) - p.next_n + row % p.next_n + 1;
  } else {
    start = p.row_starts[row];
    end = p.row_ends[row];
  }
  const long long len = end > start ? end - start : 0;
  int32_t* const out = p.out + row * p.out_stride;
  const int k = p.k;
  // (every CTA of the cluster takes the same branch: the same row)
  if (len <= k) {
    if (rank == 0)
      for (int i = tid; i < k; i += kThreads) out[i] = i < len ? i : -1;
    return;
  }
  if (len > static_cast<long long>(C) * kSlice) {
    if (rank == 0) topk_row_single(p, row, smem);
    return;
  }

  uint32_t* const keys_raw = smem;                       // [kSlice + 4]
  uint32_t* const whist = keys_raw + kSlice + 4;         // [kHists][kBins0]
  uint32_t* const rhist = whist + kHists * kBins0;       // [kBins0]: this slice's histogram (CTA 0: the row's)
  uint32_t* const cand_key = rhist + kBins0;             // [kCand]: this slice's candidates (CTA 0: the row's)
  uint32_t* const cand_pos = cand_key + kCand;           // [kCand]
  uint32_t* const wcnt = cand_pos + kCand;               // [4][kWarps]
  uint32_t* const wsum = wcnt + 2 * kWarps;              // [kWarps] (scan scratch)
  uint32_t* const ctl = wcnt + 4 * kWarps;               // [8]: d0, count above d0, count in d0 (from CTA 0)
  uint32_t* const cnt = ctl + 8;                         // [2][8]: each CTA's counts above / in d0
  const uint32_t bar = static_cast<uint32_t>(__cvta_generic_to_shared(cnt + 16));

  const long long per = (len + C - 1) / C;
  const long long s0 = static_cast<long long>(rank) * per;
  const long long slen = s0 < len ? (len - s0 < per ? len - s0 : per) : 0;
  const float* const src = p.logits + row * p.stride0 + start + s0;
  const uint32_t head = static_cast<uint32_t>(((16u - (reinterpret_cast<uintptr_t>(src) & 15u)) & 15u) >> 2);
  const int off = static_cast<int>((4u - head) & 3u);
  uint32_t* const keys = keys_raw + off;

  uint32_t* const my_hist = whist + (warp % kHists) * kBins0;
  for (int i = tid; i < kHists * kBins0; i += kThreads) whist[i] = 0;
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // the slice: its 16-byte aligned interior by one bulk copy, its ragged
  // ends (< 4 values each) by plain loads
  if (slen > 0) {
    const long long h = head < slen ? head : slen;
    const long long body = ((slen - h) / 4) * 4;
    if (tid == 0) {
      const uint32_t bytes = static_cast<uint32_t>(body * 4);
      asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                   : "memory");
      if (bytes > 0)
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                static_cast<uint32_t>(__cvta_generic_to_shared(keys + h))),
            "l"(src + h), "r"(bytes), "r"(bar)
            : "memory");
    }
    if (tid < h) keys[tid] = __float_as_uint(src[tid]);
    const long long tail0 = h + body;
    if (tid < slen - tail0) keys[tail0 + tid] = __float_as_uint(src[tail0 + tid]);
    uint32_t done = 0;
    const uint64_t t0 = now_ns();
    while (true) {
      asm volatile(
          "{\n\t.reg .pred q;\n\tmbarrier.try_wait.parity.acquire.cta.shared::cta.b64 q, [%1], 0;\n\t"
          "selp.u32 %0, 1, 0, q;\n\t}"
          : "=r"(done)
          : "r"(bar)
          : "memory");
      if (done) break;
      if (now_ns() - t0 > p.timeout_ns) {
        if (tid == 0) atomicOr(&g_topk_status, kStatusTimeout);
        break;
      }
    }
  }
  __syncthreads();
  // keys in place and this slice's first-digit histogram (16-byte sweeps as
  // in the one-CTA algorithm; keys_raw words [off, off + slen) hold the slice)
  const int W = off + static_cast<int>(slen);
#pragma unroll 1
  for (int s = 0; s < W; s += 16 * kThreads) {
    const int base = s + 512 * warp + 4 * lane;
    uint4 v[4] = {};
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (base + 128 * q < W) v[q] = *reinterpret_cast<const uint4*>(keys_raw + base + 128 * q);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int a = base + 128 * q;
      if (a < W) {
        uint32_t w[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          w[c] = order_key(__uint_as_float(w[c]));
          if (a + c >= off && a + c < W) atomicAdd(&my_hist[w[c] >> 21], 1u);
        }
        if (a >= off && a + 4 <= W) {
          *reinterpret_cast<uint4*>(keys_raw + a) = make_uint4(w[0], w[1], w[2], w[3]);
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c)
            if (a + c >= off && a + c < W) keys_raw[a + c] = w[c];
        }
      }
    }
  }
  __syncthreads();
  // 1. this slice's histogram (its kHists copies summed) into its own rhist;
  // after the barrier CTA 0 pulls every slice's histogram (each thread its
  // four bins from every CTA, summed)
  {
    uint4 h4 = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int w = 0; w < kHists; ++w) {
      const uint4 v = *reinterpret_cast<const uint4*>(whist + w * kBins0 + 4 * tid);
      h4.x += v.x;
      h4.y += v.y;
      h4.z += v.z;
      h4.w += v.w;
    }
    *reinterpret_cast<uint4*>(rhist + 4 * tid) = h4;
  }
  cluster_sync_all();
  if (rank == 0) {
    uint4 v[C];
#pragma unroll
    for (int r = 0; r < C; ++r) v[r] = ld_cluster_v4(cluster_addr(rhist + 4 * tid, r));
    uint4 h4 = v[0];
#pragma unroll
    for (int r = 1; r < C; ++r) {
      h4.x += v[r].x;
      h4.y += v[r].y;
      h4.z += v[r].z;
      h4.w += v[r].w;
    }
    *reinterpret_cast<uint4*>(rhist + 4 * tid) = h4;   // this thread's bins only: no barrier needed
    find_digit0<1>(rhist, static_cast<uint32_t>(k), wsum, ctl);
    if (tid < C)
      for (int j = 0; j < 3; ++j) st_cluster_u32(cluster_addr(ctl + j, tid), ctl[j]);
  }
  cluster_sync_all();
  const uint32_t d0 = ctl[0];
  const uint32_t n_gt0 = ctl[1];
  const uint32_t c0_count = ctl[2];
  const uint32_t k_rem = static_cast<uint32_t>(k) - n_gt0;
  const bool keep = c0_count <= static_cast<uint32_t>(kCand);
  if (!keep && c0_count != k_rem) {
    // heavy ties in the threshold bin: the whole row by CTA 0 (no further
    // access to another CTA's shared memory by anyone)
    if (rank == 0) topk_row_single(p, row, smem);
    return;
  }
  // 2. positions above d0 and in d0: per-thread counts over this slice, a
  // block scan, the block totals to every CTA
  uint32_t ng = 0, ne = 0;
#pragma unroll 1
  for (int s = 0; s < W; s += 16 * kThreads) {
    const int base = s + 512 * warp + 4 * lane;
    uint4 v[4] = {};
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (base + 128 * q < W) v[q] = *reinterpret_cast<const uint4*>(keys_raw + base + 128 * q);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int a = base + 128 * q;
      const uint32_t w[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const bool ok = a + c >= off && a + c < W;
        const uint32_t dg = w[c] >> 21;
        ng += ok && dg > d0;
        ne += ok && dg == d0;
      }
    }
  }
  uint32_t og, oe, tg, te;
  block_scan2(ng, ne, wcnt, og, oe, tg, te);
  if (tid < C) {
    st_cluster_u32(cluster_addr(cnt + rank, tid), tg);
    st_cluster_u32(cluster_addr(cnt + 8 + rank, tid), te);
  }
  cluster_sync_all();
  uint32_t eq_base = 0;
  for (uint32_t r = 0; r < rank; ++r) {
    og += cnt[r];
    eq_base += cnt[8 + r];
  }
#pragma unroll 1
  for (int s = 0; s < W; s += 16 * kThreads) {
    const int base = s + 512 * warp + 4 * lane;
    uint4 v[4] = {};
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (base + 128 * q < W) v[q] = *reinterpret_cast<const uint4*>(keys_raw + base + 128 * q);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int a = base + 128 * q;
      const uint32_t w[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (a + c < off || a + c >= W) continue;
        const uint32_t u = w[c];
        const uint32_t dg = u >> 21;
        const int32_t pos = static_cast<int32_t>(s0 + (a + c - off));
        if (dg > d0) {
          out[og++] = pos;
        } else if (dg == d0) {
          if (keep) {
            cand_key[oe] = u;        // staged here, sent to CTA 0 after the pass
            cand_pos[oe] = static_cast<uint32_t>(pos);
          } else {
            out[n_gt0 + eq_base + oe] = pos;   // the whole bin is taken
          }
          ++oe;
        }
      }
    }
  }
  if (keep && rank != 0) {
    // this slice's candidates to CTA 0 in one burst (CTA 0's own are in place)
    __syncthreads();
    for (uint32_t i = tid; i < te; i += kThreads) {
      st_cluster_u32(cluster_addr(cand_key + eq_base + i, 0), cand_key[i]);
      st_cluster_u32(cluster_addr(cand_pos + eq_base + i, 0), cand_pos[i]);
    }
  }
  cluster_sync_all();   // every candidate in CTA 0; no shared-memory access across CTAs after this
  // 3. the candidates, by CTA 0 (rhist and whist are free scratch now)
  if (rank == 0 && keep)
    finish_candidates(cand_key, cand_pos, c0_count, d0, k, n_gt0, k_rem, out + n_gt0, rhist, whist, wsum, wcnt,
                      ctl);
}

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

// per-device set-up, done once under g_init_mutex (first calls may come
// from several host threads)
std::mutex g_init_mutex;
std::atomic<bool> g_attr_set[64] = {};
int g_sm_count[64] = {};

// Cluster size for a batch: C CTAs per row while the batch then still fits
// on the SMs at once and every row fits in C slices, else one CTA per row.
// The cluster's synchronisation costs about 2 us per launch, which rows
// shorter than about 12K values do not earn back (measured on a B200: at 32
// rows, 8.8 vs 11.0 us at 8192 values, 11.4 vs 11.0 us at 12288, 17.1 vs
// 11.8 us at 32768), so they keep one CTA per row.
constexpr long long kClusterMinWidth = 12 * 1024;
int cluster_ctas(long long num_rows, long long row_width, int sms) {
  if (row_width < kClusterMinWidth) return 1;
  if (num_rows * 4 <= sms && row_width <= 4ll * kSlice) return 4;
  if (num_rows * 2 <= sms && row_width <= 2ll * kSlice) return 2;
  return 1;
}

template <int C>
cudaError_t launch_cluster(const Params& p, long long num_rows, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(num_rows * C));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = cluster_smem_bytes<C>();
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = C;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, topk_cluster_kernel<C>, p);
}

}  // namespace topk
}  // namespace glm53

using namespace glm53::topk;

extern "C" int glm53_topk_per_row(const float* logits, int64_t num_rows, int64_t stride0,
                                  int64_t stride1, const int32_t* seq_lens, int next_n,
                                  const int32_t* row_starts, const int32_t* row_ends,
                                  int32_t* out, int64_t out_stride, int topk, void* stream) {
  if (num_rows < 0 || stride0 < 0 || out_stride < topk) return GLM53_ERR_RANK;
  if (topk <= 0 || topk > kMaxTopk) return GLM53_ERR_TOPK;
  if (stride1 != 1) return GLM53_ERR_RANK;           // rows must be contiguous
  const bool decode = seq_lens != nullptr;
  if (decode == (row_starts != nullptr || row_ends != nullptr)) return GLM53_ERR_RANK;
  if (!decode && (row_starts == nullptr || row_ends == nullptr)) return GLM53_ERR_RANK;
  if (decode && next_n <= 0) return GLM53_ERR_RANK;
  if (num_rows == 0) return GLM53_OK;
  if (logits == nullptr || out == nullptr) return GLM53_ERR_ALIGN;
  if ((reinterpret_cast<uintptr_t>(logits) & 3u) || (reinterpret_cast<uintptr_t>(out) & 3u))
    return GLM53_ERR_ALIGN;
  if (num_rows > 0x7FFFFFFFll) return GLM53_ERR_RANK;
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return GLM53_ERR_CUDA;
  if (major != 10) return GLM53_ERR_DEVICE;
  if (dev < 0 || dev >= 64) return GLM53_ERR_DEVICE;
  // Opt in to the large dynamic shared-memory size once per device, before
  // any capture (the host call itself is not capturable).
  if (!g_attr_set[dev].load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(g_init_mutex);
    if (!g_attr_set[dev].load(std::memory_order_relaxed)) {
      if (cudaFuncSetAttribute(topk_per_row_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(kSmemBytes)) != cudaSuccess ||
          cudaFuncSetAttribute(topk_cluster_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(cluster_smem_bytes<2>())) != cudaSuccess ||
          cudaFuncSetAttribute(topk_cluster_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(cluster_smem_bytes<4>())) != cudaSuccess ||
          cudaDeviceGetAttribute(&g_sm_count[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return GLM53_ERR_CUDA;
      g_attr_set[dev].store(true, std::memory_order_release);
    }
  }
  Params p;
  p.logits = logits;
  p.stride0 = stride0;
  p.num_rows = num_rows;
  p.seq_lens = seq_lens;
  p.next_n = next_n;
  p.row_starts = row_starts;
  p.row_ends = row_ends;
  p.out = out;
  p.out_stride = out_stride;
  p.k = topk;
  p.timeout_ns = 1000000000ull;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int c = cluster_ctas(num_rows, stride0, g_sm_count[dev]);
  cudaError_t e;
  if (c == 4)
    e = launch_cluster<4>(p, num_rows, st);
  else if (c == 2)
    e = launch_cluster<2>(p, num_rows, st);
  else
    e = launch_pdl(topk_per_row_kernel, dim3(static_cast<unsigned>(num_rows)), dim3(kThreads), kSmemBytes, st, p);
  return e == cudaSuccess ? GLM53_OK : GLM53_ERR_CUDA;
}

extern "C" int glm53_topk_status(uint32_t* status, int clear) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_topk_status, sizeof(v)) != cudaSuccess) return GLM53_ERR_CUDA;
  if (status) *status = v;
  if (clear) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(g_topk_status, &zero, sizeof(zero)) != cudaSuccess) return GLM53_ERR_CUDA;
  }
  return GLM53_OK;
}
