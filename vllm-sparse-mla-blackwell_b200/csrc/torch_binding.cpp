// PyTorch operator binding for the sparse-MLA C ABI.
//
// Registers `torch.ops.glm53_sparse_mla.sparse_fwd` with the exact schema of
// the reference extension (csrc/sparse_mla.cu:500-505) so that existing
// callers (the vLLM backend, tests, benches) bind unchanged, plus
// `sparse_fwd_lse`, which also returns the per-(token, head) log2-space LSE.
// Argument checks mirror the reference host op (csrc/sparse_mla.cu:455-498):
// same conditions, same order (T == 0 returns before the dtype / head-count
// dispatch), raised as RuntimeError through TORCH_CHECK. The launch itself goes
// through glm53_sparse_mla_fwd_ws on the caller's current CUDA stream.
// `sparse_fwd_paged` takes vLLM's request-local positions directly, and
// `concat_and_cache_mla` is the latent KV-cache write that feeds the op, with
// the schema of vLLM's cache op of that name; `top_k_per_row_decode` /
// `top_k_per_row_prefill` produce the top-k positions from the indexer's
// logits with the schemas of vLLM's ops of those names, and
// `fp8_paged_mqa_logits` computes those logits over the paged fp8 indexer
// cache (DeepGEMM's contract as vLLM calls it).

#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/all.h>

#include <string>

#include "glm53_sparse_mla.h"

namespace {

constexpr int64_t kDim = 512;

void run_sparse_fwd(const torch::Tensor& q, const torch::Tensor& kv, const torch::Tensor& indices,
                    double sm_scale, double kv_scale, torch::Tensor& out, float* lse) {
  TORCH_CHECK(q.is_cuda() && kv.is_cuda() && indices.is_cuda() && out.is_cuda(),
              "glm53_sparse_mla: q, kv, indices and out must be CUDA tensors");
  TORCH_CHECK(q.dim() == 3 && kv.dim() == 2 && indices.dim() == 2,
              "glm53_sparse_mla: expected q [T, H, 512], kv [R, 512], indices [T, topk]");
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16, "glm53_sparse_mla: q must be bfloat16");
  TORCH_CHECK(indices.scalar_type() == torch::kInt, "glm53_sparse_mla: indices must be int32");
  TORCH_CHECK(q.is_contiguous() && kv.is_contiguous() && indices.is_contiguous(),
              "glm53_sparse_mla: q, kv and indices must be contiguous");
  TORCH_CHECK(q.size(2) == kDim && kv.size(1) == kDim, "expected kv_lora_rank ", kDim,
              " with qk_rope_head_dim 0 (NoPE)");
  const int64_t T = q.size(0);
  const int64_t topk = indices.size(1);
  TORCH_CHECK(topk % 32 == 0, "glm53_sparse_mla: topk must be a multiple of 32, got ", topk);
  TORCH_CHECK(indices.size(0) == T && out.sizes() == q.sizes(),
              "glm53_sparse_mla: indices must have T rows and out the shape of q");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.is_contiguous(),
              "glm53_sparse_mla: out must be a contiguous bfloat16 tensor");
  TORCH_CHECK(kv.get_device() == q.get_device() && indices.get_device() == q.get_device() &&
                  out.get_device() == q.get_device(),
              "glm53_sparse_mla: all tensors must be on the same device");

  if (T == 0) return;

  int kv_dtype = -1;
  if (kv.scalar_type() == torch::kBFloat16) kv_dtype = GLM53_KV_BF16;
  else if (kv.scalar_type() == torch::kFloat8_e4m3fn) kv_dtype = GLM53_KV_FP8_E4M3;
  TORCH_CHECK(kv_dtype >= 0, "kv must be bfloat16 or float8_e4m3fn, got ", kv.scalar_type());
  const int64_t H = q.size(1);
  TORCH_CHECK(H == 8 || H == 16 || H == 32 || H == 64, "unsupported heads-per-rank ", H,
              "; built for 8, 16, 32 or 64 (TP=8/4/2/1 on a 64-head model)");

  const c10::cuda::CUDAGuard guard(q.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(q.get_device()).stream();
  // Split-merge workspace from the caching allocator (stream-ordered, so it
  // is also valid inside a CUDA graph capture); empty when no token is split.
  uint64_t ws_bytes = 0;
  int rc = glm53_sparse_mla_workspace_bytes(T, H, topk, /*splits=*/0, &ws_bytes);
  TORCH_CHECK(rc == GLM53_OK, "glm53_sparse_mla: ", glm53_sparse_mla_strerror(rc));
  torch::Tensor ws;
  if (ws_bytes > 0)
    ws = torch::empty({static_cast<int64_t>(ws_bytes)},
                      torch::TensorOptions().dtype(torch::kUInt8).device(q.device()));
  rc = glm53_sparse_mla_fwd_ws(q.data_ptr(), kv.data_ptr(), indices.data_ptr<int32_t>(),
                               out.data_ptr(), lse, T, H, q.size(2), kv.size(0), kv.size(1), topk,
                               kv_dtype, static_cast<float>(sm_scale),
                               static_cast<float>(kv_scale), /*splits=*/0,
                               ws_bytes > 0 ? ws.data_ptr() : nullptr, ws_bytes,
                               static_cast<void*>(stream));
  TORCH_CHECK(rc == GLM53_OK, "glm53_sparse_mla: ", glm53_sparse_mla_strerror(rc));
}

}  // namespace

void sparse_fwd(torch::Tensor q, torch::Tensor kv, torch::Tensor indices, double sm_scale,
                double kv_scale, torch::Tensor out) {
  run_sparse_fwd(q, kv, indices, sm_scale, kv_scale, out, nullptr);
}

void sparse_fwd_lse(torch::Tensor q, torch::Tensor kv, torch::Tensor indices, double sm_scale,
                    double kv_scale, torch::Tensor out, torch::Tensor lse) {
  TORCH_CHECK(lse.is_cuda() && lse.scalar_type() == torch::kFloat && lse.is_contiguous() &&
                  lse.dim() == 2 && q.dim() == 3 && lse.size(0) == q.size(0) &&
                  lse.size(1) == q.size(1) && lse.get_device() == q.get_device(),
              "glm53_sparse_mla: lse must be a contiguous float32 CUDA tensor of shape [T, H]");
  run_sparse_fwd(q, kv, indices, sm_scale, kv_scale, out, lse.data_ptr<float>());
}

// Paged form: vLLM's request-local top-k positions plus req_id_per_token and
// the block table; the kernel converts them to slots (no separate converter
// launch, no narrowing copy: only the first `topk` columns of each row of
// topk_positions are read, at its row stride).
void sparse_fwd_paged(torch::Tensor q, torch::Tensor kv, torch::Tensor topk_positions,
                      torch::Tensor req_id_per_token, torch::Tensor block_table,
                      int64_t block_size, int64_t topk, double sm_scale, double kv_scale,
                      torch::Tensor out, const std::optional<torch::Tensor>& lse,
                      int64_t block_stride_rows) {
  TORCH_CHECK(q.is_cuda() && kv.is_cuda() && topk_positions.is_cuda() && out.is_cuda() &&
                  req_id_per_token.is_cuda() && block_table.is_cuda(),
              "glm53_sparse_mla: all tensors must be CUDA tensors");
  TORCH_CHECK(q.dim() == 3 && kv.dim() == 2 && topk_positions.dim() == 2,
              "glm53_sparse_mla: expected q [T, H, 512], kv [R, 512], topk_positions [T, >= topk]");
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16, "glm53_sparse_mla: q must be bfloat16");
  TORCH_CHECK(topk_positions.scalar_type() == torch::kInt && req_id_per_token.scalar_type() == torch::kInt &&
                  block_table.scalar_type() == torch::kInt,
              "glm53_sparse_mla: topk_positions, req_id_per_token and block_table must be int32");
  TORCH_CHECK(q.is_contiguous() && kv.is_contiguous() && req_id_per_token.is_contiguous(),
              "glm53_sparse_mla: q, kv and req_id_per_token must be contiguous");
  TORCH_CHECK(topk_positions.stride(1) == 1 && block_table.dim() == 2 && block_table.stride(1) == 1,
              "glm53_sparse_mla: topk_positions and block_table rows must be contiguous");
  TORCH_CHECK(q.size(2) == kDim && kv.size(1) == kDim, "expected kv_lora_rank ", kDim,
              " with qk_rope_head_dim 0 (NoPE)");
  const int64_t T = q.size(0);
  TORCH_CHECK(topk % 32 == 0 && topk > 0 && topk <= topk_positions.size(1),
              "glm53_sparse_mla: topk must be a positive multiple of 32, at most the position columns");
  TORCH_CHECK(topk_positions.size(0) >= T && req_id_per_token.size(0) >= T && out.sizes() == q.sizes(),
              "glm53_sparse_mla: topk_positions and req_id_per_token need T rows, out the shape of q");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.is_contiguous(),
              "glm53_sparse_mla: out must be a contiguous bfloat16 tensor");
  float* lse_ptr = nullptr;
  if (lse.has_value() && lse->defined()) {
    TORCH_CHECK(lse->is_cuda() && lse->scalar_type() == torch::kFloat && lse->is_contiguous() &&
                    lse->dim() == 2 && lse->size(0) == T && lse->size(1) == q.size(1),
                "glm53_sparse_mla: lse must be a contiguous float32 CUDA tensor of shape [T, H]");
    lse_ptr = lse->data_ptr<float>();
  }
  if (T == 0) return;
  int kv_dtype = -1;
  if (kv.scalar_type() == torch::kBFloat16) kv_dtype = GLM53_KV_BF16;
  else if (kv.scalar_type() == torch::kFloat8_e4m3fn) kv_dtype = GLM53_KV_FP8_E4M3;
  TORCH_CHECK(kv_dtype >= 0, "kv must be bfloat16 or float8_e4m3fn, got ", kv.scalar_type());
  const int64_t H = q.size(1);
  const c10::cuda::CUDAGuard guard(q.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(q.get_device()).stream();
  uint64_t ws_bytes = 0;
  int rc = glm53_sparse_mla_workspace_bytes(T, H, topk, /*splits=*/0, &ws_bytes);
  TORCH_CHECK(rc == GLM53_OK, "glm53_sparse_mla: ", glm53_sparse_mla_strerror(rc));
  torch::Tensor ws;
  if (ws_bytes > 0)
    ws = torch::empty({static_cast<int64_t>(ws_bytes)},
                      torch::TensorOptions().dtype(torch::kUInt8).device(q.device()));
  rc = glm53_sparse_mla_fwd_paged(
      q.data_ptr(), kv.data_ptr(), topk_positions.data_ptr<int32_t>(), topk_positions.stride(0),
      req_id_per_token.data_ptr<int32_t>(), block_table.data_ptr<int32_t>(), block_table.stride(0),
      block_table.size(1), block_size, block_stride_rows > 0 ? block_stride_rows : block_size,
      out.data_ptr(), lse_ptr, T, H, q.size(2), kv.size(0), kv.size(1), topk, kv_dtype,
      static_cast<float>(sm_scale), static_cast<float>(kv_scale), /*splits=*/0,
      ws_bytes > 0 ? ws.data_ptr() : nullptr, ws_bytes, static_cast<void*>(stream));
  TORCH_CHECK(rc == GLM53_OK, "glm53_sparse_mla: ", glm53_sparse_mla_strerror(rc));
}

// One rank of a head-sharded group writing its heads straight into every
// rank's full output. `out` is this rank's own [T, heads_total, 512] buffer
// (its pointer must be the entry of out_ptrs at index `rank`); out_ptrs are
// the device pointers of all ranks' buffers as this GPU addresses them
// (symmetric memory). The caller synchronises the ranks afterwards.
void sparse_fwd_gather_heads(torch::Tensor q, torch::Tensor kv, torch::Tensor indices,
                             double sm_scale, double kv_scale, std::vector<int64_t> out_ptrs,
                             int64_t rank, int64_t head_offset, torch::Tensor out) {
  TORCH_CHECK(q.is_cuda() && kv.is_cuda() && indices.is_cuda() && out.is_cuda(),
              "glm53_sparse_mla: q, kv, indices and out must be CUDA tensors");
  TORCH_CHECK(q.dim() == 3 && kv.dim() == 2 && indices.dim() == 2 && out.dim() == 3,
              "glm53_sparse_mla: expected q [T, H, 512], kv [R, 512], indices [T, topk], "
              "out [T, heads_total, 512]");
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16 && indices.scalar_type() == torch::kInt,
              "glm53_sparse_mla: q must be bfloat16 and indices int32");
  TORCH_CHECK(q.is_contiguous() && kv.is_contiguous() && indices.is_contiguous() &&
                  out.is_contiguous() && out.scalar_type() == torch::kBFloat16,
              "glm53_sparse_mla: q, kv, indices and out must be contiguous, out bfloat16");
  TORCH_CHECK(q.size(2) == kDim && kv.size(1) == kDim && out.size(2) == kDim,
              "expected kv_lora_rank ", kDim, " with qk_rope_head_dim 0 (NoPE)");
  const int64_t T = q.size(0), H = q.size(1), topk = indices.size(1);
  TORCH_CHECK(indices.size(0) == T && out.size(0) == T, "glm53_sparse_mla: T rows everywhere");
  TORCH_CHECK(!out_ptrs.empty() && out_ptrs.size() <= 8 && rank >= 0 &&
                  rank < static_cast<int64_t>(out_ptrs.size()) &&
                  out_ptrs[rank] == reinterpret_cast<int64_t>(out.data_ptr()),
              "glm53_sparse_mla: out_ptrs must list 1 to 8 buffers, out at index rank");
  TORCH_CHECK(head_offset >= 0 && head_offset + H <= out.size(1),
              "glm53_sparse_mla: heads [head_offset, head_offset + H) must lie in out");
  if (T == 0) return;
  int kv_dtype = -1;
  if (kv.scalar_type() == torch::kBFloat16) kv_dtype = GLM53_KV_BF16;
  else if (kv.scalar_type() == torch::kFloat8_e4m3fn) kv_dtype = GLM53_KV_FP8_E4M3;
  TORCH_CHECK(kv_dtype >= 0, "kv must be bfloat16 or float8_e4m3fn, got ", kv.scalar_type());
  const c10::cuda::CUDAGuard guard(q.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(q.get_device()).stream();
  uint64_t ws_bytes = 0;
  int rc = glm53_sparse_mla_workspace_bytes(T, H, topk, /*splits=*/0, &ws_bytes);
  TORCH_CHECK(rc == GLM53_OK, "glm53_sparse_mla: ", glm53_sparse_mla_strerror(rc));
  torch::Tensor ws;
  if (ws_bytes > 0)
    ws = torch::empty({static_cast<int64_t>(ws_bytes)},
                      torch::TensorOptions().dtype(torch::kUInt8).device(q.device()));
  void* ptrs[8];
  for (size_t i = 0; i < out_ptrs.size(); ++i) ptrs[i] = reinterpret_cast<void*>(out_ptrs[i]);
  rc = glm53_sparse_mla_fwd_heads_gather(
      q.data_ptr(), kv.data_ptr(), indices.data_ptr<int32_t>(), ptrs,
      static_cast<int>(out_ptrs.size()), head_offset, out.size(1), nullptr, T, H, q.size(2),
      kv.size(0), kv.size(1), topk, kv_dtype, static_cast<float>(sm_scale),
      static_cast<float>(kv_scale), /*splits=*/0, ws_bytes > 0 ? ws.data_ptr() : nullptr, ws_bytes,
      static_cast<void*>(stream));
  TORCH_CHECK(rc == GLM53_OK, "glm53_sparse_mla: ", glm53_sparse_mla_strerror(rc));
}

// Latent KV-cache write with the schema and argument meaning of vLLM's
// _C_cache_ops::concat_and_cache_mla (vllm 0.22.0 vllm/_custom_ops.py:2613-2623)
// for this path's geometry: kv_lora_rank 512, pe_dim 0. The token count is
// slot_mapping's length (kv_c may hold more rows: padding for CUDA graphs).
void concat_and_cache_mla(const torch::Tensor& kv_c, const torch::Tensor& k_pe,
                          torch::Tensor& kv_cache, const torch::Tensor& slot_mapping,
                          const std::string& kv_cache_dtype, const torch::Tensor& scale) {
  TORCH_CHECK(kv_c.is_cuda() && kv_cache.is_cuda() && slot_mapping.is_cuda(),
              "glm53_sparse_mla: kv_c, kv_cache and slot_mapping must be CUDA tensors");
  TORCH_CHECK(kv_c.dim() == 2 && kv_c.size(1) == kDim && kv_c.stride(1) == 1 &&
                  kv_c.scalar_type() == torch::kBFloat16,
              "glm53_sparse_mla: kv_c must be bfloat16 [num_tokens, 512] with contiguous rows");
  TORCH_CHECK(k_pe.numel() == 0, "glm53_sparse_mla: this path writes NoPE caches (pe_dim 0); got k_pe ",
              k_pe.sizes());
  TORCH_CHECK(kv_cache.dim() == 3 && kv_cache.size(2) == kDim && kv_cache.stride(2) == 1,
              "glm53_sparse_mla: kv_cache must be [num_blocks, block_size, 512] (kv_lora_rank + pe_dim)");
  TORCH_CHECK(slot_mapping.dim() == 1 && slot_mapping.scalar_type() == torch::kLong &&
                  slot_mapping.is_contiguous(),
              "glm53_sparse_mla: slot_mapping must be a contiguous int64 vector");
  const int64_t T = slot_mapping.size(0);
  TORCH_CHECK(kv_c.size(0) >= T, "glm53_sparse_mla: kv_c has fewer rows than slot_mapping");
  TORCH_CHECK(kv_c.get_device() == kv_cache.get_device() &&
                  slot_mapping.get_device() == kv_cache.get_device(),
              "glm53_sparse_mla: all tensors must be on the same device");
  int cache_dtype = -1;
  if (kv_cache_dtype == "auto") {
    TORCH_CHECK(kv_cache.scalar_type() == torch::kBFloat16,
                "glm53_sparse_mla: kv_cache_dtype 'auto' needs a bfloat16 cache like kv_c");
    cache_dtype = GLM53_KV_BF16;
  } else if (kv_cache_dtype == "fp8" || kv_cache_dtype == "fp8_e4m3") {
    TORCH_CHECK(kv_cache.scalar_type() == torch::kUInt8 || kv_cache.scalar_type() == torch::kFloat8_e4m3fn,
                "glm53_sparse_mla: an fp8 cache must be uint8 or float8_e4m3fn");
    TORCH_CHECK(scale.is_cuda() && scale.scalar_type() == torch::kFloat && scale.numel() >= 1 &&
                    scale.get_device() == kv_cache.get_device(),
                "glm53_sparse_mla: scale must be a float32 CUDA tensor on the cache's device");
    cache_dtype = GLM53_KV_FP8_E4M3;
  } else {
    TORCH_CHECK(false, "glm53_sparse_mla: unsupported kv_cache_dtype '", kv_cache_dtype,
                "' (this path writes 'auto' bf16 or 'fp8' / 'fp8_e4m3')");
  }
  if (T == 0) return;
  const c10::cuda::CUDAGuard guard(kv_cache.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(kv_cache.get_device()).stream();
  const int rc = glm53_concat_and_cache(
      kv_c.data_ptr(), kv_c.stride(0), T, kv_cache.data_ptr(), cache_dtype, kv_cache.size(0),
      kv_cache.size(1), kv_cache.stride(0), kv_cache.stride(1), slot_mapping.data_ptr<int64_t>(),
      cache_dtype == GLM53_KV_FP8_E4M3 ? scale.data_ptr<float>() : nullptr,
      static_cast<void*>(stream));
  TORCH_CHECK(rc == GLM53_OK, "glm53_sparse_mla: ", glm53_sparse_mla_strerror(rc));
}

// Indexer top-k with the schemas of vLLM's top_k_per_row_decode /
// top_k_per_row_prefill (vllm 0.22.0 vllm/_custom_ops.py:2799-2840). seq_lens
// may be 1-D [B] (row r ends at seq_lens[r / next_n] - next_n + r % next_n + 1)
// or 2-D [B, next_n] (row r ends at the r-th entry: per-token context lengths).
void run_topk(const torch::Tensor& logits, const int32_t* seq_lens, int64_t next_n,
              const int32_t* starts, const int32_t* ends, torch::Tensor& out, int64_t num_rows,
              int64_t stride0, int64_t stride1, int64_t topk) {
  TORCH_CHECK(logits.is_cuda() && out.is_cuda(), "glm53_sparse_mla: logits and indices must be CUDA tensors");
  TORCH_CHECK(logits.scalar_type() == torch::kFloat, "glm53_sparse_mla: logits must be float32");
  TORCH_CHECK(out.scalar_type() == torch::kInt && out.dim() == 2 && out.stride(1) == 1,
              "glm53_sparse_mla: raw_topk_indices must be int32 [rows, >= topk] with contiguous rows");
  TORCH_CHECK(num_rows <= out.size(0) && topk <= out.size(1),
              "glm53_sparse_mla: raw_topk_indices is smaller than [num_rows, topk_tokens]");
  TORCH_CHECK(num_rows <= 0 || (num_rows - 1) * stride0 < logits.numel(),
              "glm53_sparse_mla: num_rows * stride0 exceeds logits");
  if (num_rows == 0) return;
  const c10::cuda::CUDAGuard guard(logits.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(logits.get_device()).stream();
  const int rc = glm53_topk_per_row(logits.data_ptr<float>(), num_rows, stride0, stride1, seq_lens,
                                    static_cast<int>(next_n), starts, ends, out.data_ptr<int32_t>(),
                                    out.stride(0), static_cast<int>(topk), static_cast<void*>(stream));
  TORCH_CHECK(rc == GLM53_OK, "glm53_sparse_mla: ", glm53_sparse_mla_strerror(rc));
}

void top_k_per_row_decode(const torch::Tensor& logits, int64_t next_n, const torch::Tensor& seq_lens,
                          torch::Tensor& raw_topk_indices, int64_t num_rows, int64_t stride0,
                          int64_t stride1, int64_t topk_tokens) {
  TORCH_CHECK(seq_lens.is_cuda() && seq_lens.scalar_type() == torch::kInt && seq_lens.is_contiguous(),
              "glm53_sparse_mla: seq_lens must be a contiguous int32 CUDA tensor");
  TORCH_CHECK(next_n >= 1, "glm53_sparse_mla: next_n must be >= 1");
  int64_t nn = next_n;
  if (seq_lens.dim() == 2 && seq_lens.size(1) > 1) {
    TORCH_CHECK(seq_lens.size(1) == next_n && seq_lens.numel() >= num_rows,
                "glm53_sparse_mla: 2-D seq_lens must be [B, next_n] covering num_rows");
    nn = 1;   // per-row context lengths
  } else {
    TORCH_CHECK(seq_lens.dim() >= 1 && seq_lens.numel() * next_n >= num_rows,
                "glm53_sparse_mla: seq_lens must hold ceil(num_rows / next_n) lengths");
  }
  run_topk(logits, seq_lens.data_ptr<int32_t>(), nn, nullptr, nullptr, raw_topk_indices, num_rows,
           stride0, stride1, topk_tokens);
}

void top_k_per_row_prefill(const torch::Tensor& logits, const torch::Tensor& cu_seqlen_ks,
                           const torch::Tensor& cu_seqlen_ke, torch::Tensor& raw_topk_indices,
                           int64_t num_rows, int64_t stride0, int64_t stride1, int64_t topk_tokens) {
  TORCH_CHECK(cu_seqlen_ks.is_cuda() && cu_seqlen_ke.is_cuda() &&
                  cu_seqlen_ks.scalar_type() == torch::kInt && cu_seqlen_ke.scalar_type() == torch::kInt &&
                  cu_seqlen_ks.is_contiguous() && cu_seqlen_ke.is_contiguous() &&
                  cu_seqlen_ks.numel() >= num_rows && cu_seqlen_ke.numel() >= num_rows,
              "glm53_sparse_mla: cu_seqlen_ks / cu_seqlen_ke must be contiguous int32 CUDA tensors "
              "with num_rows entries");
  run_topk(logits, nullptr, 1, cu_seqlen_ks.data_ptr<int32_t>(), cu_seqlen_ke.data_ptr<int32_t>(),
           raw_topk_indices, num_rows, stride0, stride1, topk_tokens);
}

// Indexer scores with the contract of DeepGEMM's fp8 paged MQA logits as
// vLLM 0.22.0 calls it (vllm/utils/deep_gemm.py:407-456): q [B, next_n, H, 128]
// fp8_e4m3, kv_cache [num_blocks, block_size, (1,) 132] uint8 (128 e4m3
// values per row, then the block's fp32 scales), weights [B * next_n, H] fp32,
// context_lens [B] or [B, next_n] int32 (the latter per token), block_tables
// [B, max_blocks] int32; writes logits [B * next_n, >= max_model_len] fp32.
void fp8_paged_mqa_logits(const torch::Tensor& q, const torch::Tensor& kv_cache,
                          const torch::Tensor& weights, const torch::Tensor& context_lens,
                          const torch::Tensor& block_tables, int64_t max_model_len,
                          bool clean_logits, torch::Tensor& logits) {
  TORCH_CHECK(q.is_cuda() && kv_cache.is_cuda() && weights.is_cuda() && context_lens.is_cuda() &&
                  block_tables.is_cuda() && logits.is_cuda(),
              "glm53_sparse_mla: indexer tensors must be CUDA tensors");
  TORCH_CHECK(q.dim() == 4 && q.is_contiguous() &&
                  (q.scalar_type() == torch::kFloat8_e4m3fn || q.scalar_type() == torch::kUInt8),
              "glm53_sparse_mla: q must be a contiguous fp8_e4m3 tensor [B, next_n, H, 128]");
  const int64_t B = q.size(0), next_n = q.size(1), H = q.size(2);
  TORCH_CHECK(q.size(3) == 128, "glm53_sparse_mla: the indexer head dim must be 128");
  TORCH_CHECK(kv_cache.scalar_type() == torch::kUInt8 && (kv_cache.dim() == 3 || kv_cache.dim() == 4) &&
                  kv_cache.size(-1) == 132 && kv_cache.stride(-1) == 1 &&
                  kv_cache.stride(1) == (kv_cache.dim() == 4 ? kv_cache.size(2) * 132 : 132),
              "glm53_sparse_mla: kv_cache must be uint8 [num_blocks, block_size, (1,) 132] with "
              "contiguous blocks");
  TORCH_CHECK(weights.scalar_type() == torch::kFloat && weights.is_contiguous() &&
                  weights.dim() == 2 && weights.size(0) == B * next_n && weights.size(1) == H,
              "glm53_sparse_mla: weights must be contiguous float32 [B * next_n, H]");
  TORCH_CHECK(context_lens.scalar_type() == torch::kInt && context_lens.is_contiguous() &&
                  context_lens.size(0) == B && (context_lens.dim() == 1 ||
                  (context_lens.dim() == 2 && (context_lens.size(1) == 1 || context_lens.size(1) == next_n))),
              "glm53_sparse_mla: context_lens must be int32 [B] or [B, next_n]");
  TORCH_CHECK(block_tables.scalar_type() == torch::kInt && block_tables.dim() == 2 &&
                  block_tables.size(0) >= B && block_tables.stride(1) == 1,
              "glm53_sparse_mla: block_tables must be int32 [B, max_blocks] with contiguous rows");
  TORCH_CHECK(logits.scalar_type() == torch::kFloat && logits.dim() == 2 &&
                  logits.size(0) >= B * next_n && logits.size(1) >= max_model_len && logits.stride(1) == 1,
              "glm53_sparse_mla: logits must be float32 [B * next_n, >= max_model_len]");
  const bool per_token = context_lens.dim() == 2 && context_lens.size(1) == next_n && next_n > 1;
  if (B == 0 || max_model_len == 0) return;
  const c10::cuda::CUDAGuard guard(q.device());
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(q.get_device()).stream();
  const int rc = glm53_indexer_logits(
      q.data_ptr(), kv_cache.data_ptr(), weights.data_ptr<float>(), context_lens.data_ptr<int32_t>(),
      per_token ? 1 : 0, block_tables.data_ptr<int32_t>(), B, static_cast<int>(next_n), H, 128,
      kv_cache.size(0), kv_cache.size(1), kv_cache.stride(0), block_tables.stride(0),
      block_tables.size(1), logits.data_ptr<float>(), logits.stride(0), max_model_len,
      clean_logits ? 1 : 0, static_cast<void*>(stream));
  TORCH_CHECK(rc == GLM53_OK, "glm53_sparse_mla: ", glm53_sparse_mla_strerror(rc));
}

TORCH_LIBRARY(glm53_sparse_mla, m) {
  m.def("sparse_fwd(Tensor q, Tensor kv, Tensor indices, float sm_scale, float kv_scale, Tensor(a!) out) -> ()");
  m.def("sparse_fwd_lse(Tensor q, Tensor kv, Tensor indices, float sm_scale, float kv_scale, Tensor(a!) out, Tensor(b!) lse) -> ()");
  m.def("sparse_fwd_paged(Tensor q, Tensor kv, Tensor topk_positions, Tensor req_id_per_token, Tensor block_table, int block_size, int topk, float sm_scale, float kv_scale, Tensor(a!) out, Tensor(b!)? lse=None, int block_stride_rows=0) -> ()");
  m.def("sparse_fwd_gather_heads(Tensor q, Tensor kv, Tensor indices, float sm_scale, float kv_scale, int[] out_ptrs, int rank, int head_offset, Tensor(a!) out) -> ()");
  m.def("concat_and_cache_mla(Tensor kv_c, Tensor k_pe, Tensor(a!) kv_cache, Tensor slot_mapping, str kv_cache_dtype, Tensor scale) -> ()");
  m.def("top_k_per_row_decode(Tensor logits, int next_n, Tensor seq_lens, Tensor(a!) raw_topk_indices, int num_rows, int stride0, int stride1, int topk_tokens) -> ()");
  m.def("top_k_per_row_prefill(Tensor logits, Tensor cu_seqlen_ks, Tensor cu_seqlen_ke, Tensor(a!) raw_topk_indices, int num_rows, int stride0, int stride1, int topk_tokens) -> ()");
  m.def("fp8_paged_mqa_logits(Tensor q, Tensor kv_cache, Tensor weights, Tensor context_lens, Tensor block_tables, int max_model_len, bool clean_logits, Tensor(a!) logits) -> ()");
}

TORCH_LIBRARY_IMPL(glm53_sparse_mla, CUDA, m) {
  m.impl("sparse_fwd", &sparse_fwd);
  m.impl("sparse_fwd_lse", &sparse_fwd_lse);
  m.impl("sparse_fwd_paged", &sparse_fwd_paged);
  m.impl("sparse_fwd_gather_heads", &sparse_fwd_gather_heads);
  m.impl("concat_and_cache_mla", &concat_and_cache_mla);
  m.impl("top_k_per_row_decode", &top_k_per_row_decode);
  m.impl("top_k_per_row_prefill", &top_k_per_row_prefill);
  m.impl("fp8_paged_mqa_logits", &fp8_paged_mqa_logits);
}
