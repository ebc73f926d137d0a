// Latent KV-cache writer for the sparse-MLA path, sm_100a only.
//
// Writes each new token's 512-wide latent row (kv_c, bf16) into its slot of the
// paged cache [num_blocks, block_size, 512] the attention kernel gathers from:
// bf16 as it is (kv_cache_dtype "auto"), or plain fp8_e4m3 with one per-tensor
// scale, element = e4m3(float(x) / scale) with round-to-nearest-even and
// saturation to +-448. It is the write vLLM 0.22.0 performs for this NoPE
// geometry (pe_dim 0) in concat_and_cache_mla, called from
// MLAAttentionImpl.do_kv_cache_update (vllm/v1/attention/backend.py:990-1010);
// the reference keeps that layout (glm53_sparse_mla/backend.py:398-428) and
// leaves the write to vLLM.
//
// Design: pure HBM streaming (1024 B read, 512 or 1024 B written per token),
// one warp per token. Lane l moves elements [8l, 8l + 8) and [256 + 8l,
// 256 + 8l + 8): every warp-wide load covers 512 contiguous bytes and every
// fp8 store 256, so each token's traffic is a handful of full 128-byte lines.
// The scale is read on the device (no host synchronisation), a slot < 0 (a
// padded token) writes nothing, and a slot past the cache is skipped and
// reported through this writer's device status word instead of written out of
// bounds.

#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "glm53_sparse_mla.h"

namespace glm53 {
namespace cache_writer {

constexpr int kWidth = 512;
constexpr int kWarpsPerBlock = 8;

__device__ unsigned int g_writer_status = 0;

struct Params {
  const __nv_bfloat16* kv_c;   // [>= T, kv_c_stride]
  long long kv_c_stride;       // elements
  uint8_t* cache;              // element (b, o, i) at b * block_stride + o * entry_stride + i
  long long block_stride;      // elements of the cache type
  long long entry_stride;
  const int64_t* slots;        // [T]
  long long T;
  long long capacity;          // num_blocks * block_size
  long long block_size;
  const float* scale;          // fp8 only: device scalar
};

__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// x / s rounded to nearest fp32, from r = RN(1 / s) with one FMA correction:
// q = RN(x * r), rem = x - s * q (exact through the FMA), RN(q + rem * r) is
// the correctly rounded quotient when nothing overflows or underflows
// (Markstein's theorem on FMA division: P. Markstein, IBM J. Res. Dev. 34(1),
// 1990; also in Muller et al., Handbook of Floating-Point Arithmetic).
// Outside that range the e4m3 result does not depend on the last bit:
// |q| >= 512 saturates to 448 either way (the correction is skipped there, so
// an x / s beyond fp32 range cannot become inf - inf), and quotients far below
// the smallest e4m3 subnormal round to 0. A zero result keeps q's sign, as
// the division would. The caller falls back to the division itself when r is
// not finite (s zero, subnormal or not finite).
__device__ __forceinline__ float div_by_scale(const float x, const float s, const float r) {
  const float q = x * r;
  if (!(fabsf(q) < 512.f)) return q;
  const float c = fmaf(fmaf(-s, q, x), r, q);
  return c == 0.f ? q : c;
}

// Eight bf16 -> eight e4m3 (byte j = element j): fp32 division by the scale,
// then the hardware float -> e4m3 conversion with saturation.
__device__ __forceinline__ uint2 quantize8(const uint4 w, const float s, const float r) {
  const uint32_t in[4] = {w.x, w.y, w.z, w.w};
  uint32_t out[2] = {0u, 0u};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&in[k]));
    if (isfinite(r)) {
      f.x = div_by_scale(f.x, s, r);
      f.y = div_by_scale(f.y, s, r);
    } else {
      f.x = __fdiv_rn(f.x, s);
      f.y = __fdiv_rn(f.y, s);
    }
    const uint32_t q = __nv_cvt_float2_to_fp8x2(f, __NV_SATFINITE, __NV_E4M3);
    out[k >> 1] |= (q & 0xFFFFu) << (16 * (k & 1));
  }
  return make_uint2(out[0], out[1]);
}

template <bool kFp8>
__global__ void __launch_bounds__(32 * kWarpsPerBlock) concat_and_cache_kernel(const Params p) {
  // Programmatic dependent launch: the new rows come from the previous
  // kernel in the stream, so wait for it before any global access;
  // dependents may launch at once (they wait in turn for this grid).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const long long t = static_cast<long long>(blockIdx.x) * kWarpsPerBlock + (threadIdx.x >> 5);
  if (t >= p.T) return;
  const int lane = threadIdx.x & 31;
  const __nv_bfloat16* src = p.kv_c + t * p.kv_c_stride;
  // bf16: the row does not depend on the slot, so its loads go out with the
  // slot's and the warp waits out one memory latency, not two. (Measured
  // slower for fp8, which keeps the slot-first order.)
  uint4 a = make_uint4(0u, 0u, 0u, 0u), b = a;
  if constexpr (!kFp8) {
    a = ldg_stream_v4(src + 8 * lane);
    b = ldg_stream_v4(src + 256 + 8 * lane);
  }
  const long long slot = p.slots[t];
  if (slot < 0) return;   // padded token
  if (slot >= p.capacity) {
    if (lane == 0) atomicOr(&g_writer_status, static_cast<unsigned>(GLM53_DEV_BAD_SLOT));
    return;
  }
  const long long blk = slot / p.block_size;
  const long long entry = blk * p.block_stride + (slot - blk * p.block_size) * p.entry_stride;
  if constexpr (kFp8) {
    a = ldg_stream_v4(src + 8 * lane);
    b = ldg_stream_v4(src + 256 + 8 * lane);
    const float s = *p.scale;
    const float r = __frcp_rn(s);
    uint8_t* dst = p.cache + entry;
    *reinterpret_cast<uint2*>(dst + 8 * lane) = quantize8(a, s, r);
    *reinterpret_cast<uint2*>(dst + 256 + 8 * lane) = quantize8(b, s, r);
  } else {
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.cache) + entry;
    *reinterpret_cast<uint4*>(dst + 8 * lane) = a;
    *reinterpret_cast<uint4*>(dst + 256 + 8 * lane) = b;
  }
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace cache_writer
}  // namespace glm53

using namespace glm53::cache_writer;

extern "C" int glm53_concat_and_cache(const void* kv_c, int64_t kv_c_stride, int64_t T,
                                      void* kv_cache, int cache_dtype, int64_t num_blocks,
                                      int64_t block_size, int64_t block_stride,
                                      int64_t entry_stride, const int64_t* slot_mapping,
                                      const float* scale, void* stream) {
  if (T < 0 || num_blocks < 0 || block_size <= 0) return GLM53_ERR_RANK;
  if (kv_c_stride < kWidth || entry_stride < kWidth || block_stride < block_size * entry_stride)
    return GLM53_ERR_RANK;
  if (cache_dtype != GLM53_KV_BF16 && cache_dtype != GLM53_KV_FP8_E4M3) return GLM53_ERR_DTYPE;
  if (T == 0) return GLM53_OK;
  const bool fp8 = cache_dtype == GLM53_KV_FP8_E4M3;
  const int64_t elem = fp8 ? 1 : 2;
  if (kv_c == nullptr || kv_cache == nullptr || slot_mapping == nullptr || (fp8 && scale == nullptr))
    return GLM53_ERR_ALIGN;
  if (!aligned16(kv_c) || !aligned16(kv_cache) || (reinterpret_cast<uintptr_t>(slot_mapping) & 7u) ||
      (fp8 && (reinterpret_cast<uintptr_t>(scale) & 3u)) || (kv_c_stride * 2) % 16 ||
      (entry_stride * elem) % 16 || (block_stride * elem) % 16)
    return GLM53_ERR_ALIGN;
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return GLM53_ERR_CUDA;
  if (major != 10) return GLM53_ERR_DEVICE;

  Params p;
  p.kv_c = static_cast<const __nv_bfloat16*>(kv_c);
  p.kv_c_stride = kv_c_stride;
  p.cache = static_cast<uint8_t*>(kv_cache);
  p.block_stride = block_stride;
  p.entry_stride = entry_stride;
  p.slots = slot_mapping;
  p.T = T;
  p.capacity = num_blocks * block_size;
  p.block_size = block_size;
  p.scale = scale;
  const long long blocks = (T + kWarpsPerBlock - 1) / kWarpsPerBlock;
  if (blocks > 0x7FFFFFFFll) return GLM53_ERR_RANK;
  // launched with programmatic stream serialization, so the grid may begin
  // launching while the previous kernel in the stream drains
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks));
  cfg.blockDim = dim3(32 * kWarpsPerBlock);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = fp8 ? cudaLaunchKernelEx(&cfg, concat_and_cache_kernel<true>, p)
                            : cudaLaunchKernelEx(&cfg, concat_and_cache_kernel<false>, p);
  return e == cudaSuccess ? GLM53_OK : GLM53_ERR_CUDA;
}

extern "C" int glm53_concat_and_cache_status(uint32_t* status, int clear) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_writer_status, sizeof(v)) != cudaSuccess) return GLM53_ERR_CUDA;
  if (status) *status = v;
  if (clear) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(g_writer_status, &zero, sizeof(zero)) != cudaSuccess)
      return GLM53_ERR_CUDA;
  }
  return GLM53_OK;
}
