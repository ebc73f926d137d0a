/*
 * C ABI of the B200 (sm_100a) sparse-MLA attention library.
 *
 * Sparse MLA in the NoPE geometry (qk_rope_head_dim = 0, head size =
 * kv_lora_rank = 512): every query token attends only to the top-k rows of a
 * flat latent KV pool named by its index list, and an index < 0 is the only
 * mask. The same row serves as key and value (absorbed MLA).
 *
 * Plain pointers, sizes and scalars only; no framework types cross this
 * boundary. All device pointers must be 16-byte aligned and the tensors
 * row-major contiguous. The stream argument is a cudaStream_t passed as void*.
 *
 * Build: libglm53_sparse_mla.so (nvcc, -gencode arch=compute_100a,code=sm_100a).
 */
#ifndef GLM53_SPARSE_MLA_H_
#define GLM53_SPARSE_MLA_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes returned by every entry point. */
enum glm53_status {
  GLM53_OK = 0,
  GLM53_ERR_RANK = 1,          /* wrong tensor rank / shape mismatch            */
  GLM53_ERR_HEAD_DIM = 2,      /* head size or kv width is not 512              */
  GLM53_ERR_HEADS = 3,         /* heads per launch not in {8, 16, 32, 64}        */
  GLM53_ERR_TOPK = 4,          /* top-k not a multiple of 32, or too large       */
  GLM53_ERR_DTYPE = 5,         /* kv dtype is neither bf16 nor fp8_e4m3          */
  GLM53_ERR_ALIGN = 6,         /* a pointer is null or not 16-byte aligned       */
  GLM53_ERR_SPLITS = 7,        /* explicit split count not in {0, 1, 2, 4, 8}    */
  GLM53_ERR_CUDA = 8,          /* a CUDA runtime call failed                     */
  GLM53_ERR_DEVICE = 9,        /* current device is not sm_100                   */
  GLM53_ERR_WORKSPACE = 10,    /* workspace missing, misaligned or too small     */
  GLM53_ERR_SCRATCH_LIMIT = 11 /* shape needs more than the no-alloc scratch     */
};

/* KV pool element type. */
enum glm53_kv_dtype {
  GLM53_KV_BF16 = 0,
  GLM53_KV_FP8_E4M3 = 1
};

/* Bits of the device-side status word (see glm53_sparse_mla_device_status). */
enum glm53_device_status_bits {
  GLM53_DEV_TIMEOUT = 1u,      /* a pipeline wait gave up after its time limit   */
  GLM53_DEV_BAD_INDEX = 2u,    /* an index >= kv_rows was seen and masked out    */
  GLM53_DEV_BAD_SLOT = 4u      /* cache writer: a slot past the cache was skipped */
};

/*
 * Sparse-MLA forward.
 *
 *   q        [T, H, 512]  bf16
 *   kv       [R, 512]     bf16 or fp8_e4m3 (per-tensor scale kv_scale)
 *   indices  [T, topk]    int32 physical row ids into kv, < 0 = masked
 *   out      [T, H, 512]  bf16, written in place (caller-owned)
 *   lse      [T, H]       fp32, or NULL: log2(sum_i exp(sm_scale * q . kv_i))
 *                         over the valid indices. A fully masked (token, head)
 *                         gets -inf and an all-zero output row.
 *
 * sm_scale is the natural-log softmax scale (the kernel multiplies by log2 e).
 * kv_scale multiplies dequantised fp8 values; it is ignored for bf16.
 * splits: 0 = automatic (or the GLM53_SPLITS environment variable, read once):
 * small batches split every token; a batch with more tokens than SMs runs its
 * whole waves unsplit and splits the tokens of the last, partial wave (two
 * launches). 1, 2, 4 or 8 = split each token's top-k list across that many
 * CTAs of one thread-block cluster.
 * H must be 8, 16, 32 or 64; head_dim and the kv width must be 512; topk must
 * be a multiple of 32 and at most 16384. T == 0 is a no-op.
 *
 * Replaces the host launcher `sparse_fwd(q, kv, indices, sm_scale, kv_scale,
 * out)` of the reference (csrc/sparse_mla.cu:455-498) and its launch helper
 * (csrc/sparse_mla.cu:434-453). The lse output has no counterpart in the
 * reference op; its fp32 oracle returns a log2 LSE (tests/reference.py:71-73)
 * whose max term carries sm_scale twice, so the two agree at sm_scale == 1.
 * Launch is asynchronous on `stream`; no host synchronisation, no allocation.
 */
int glm53_sparse_mla_fwd(const void* q, const void* kv, const int32_t* indices, void* out,
                         float* lse, int64_t T, int64_t H, int64_t head_dim, int64_t kv_rows,
                         int64_t kv_width, int64_t topk, int kv_dtype, float sm_scale,
                         float kv_scale, int splits, void* stream);

/*
 * Bytes of global workspace glm53_sparse_mla_fwd_ws needs for this shape on
 * the current device (0 when each token runs on a single CTA). Resolves
 * splits == 0 exactly as the forward does. The size is
 * (split tokens) * splits * Hp * 512 * 4 bytes, Hp = max(H, 16): 16 MiB for a
 * 32-token, 64-head decode batch split 4 ways. With splits == 0 and more
 * tokens than SMs, only the tokens of the last, partial wave are split.
 * No counterpart in the reference, whose kernel never splits a token.
 */
int glm53_sparse_mla_workspace_bytes(int64_t T, int64_t H, int64_t topk, int splits,
                                     uint64_t* bytes);

/*
 * As glm53_sparse_mla_fwd, with the per-token split partials merged through
 * `workspace` (global memory, 16-byte aligned, at least
 * glm53_sparse_mla_workspace_bytes; unused when no token is split) instead of
 * distributed shared memory. All 8 warps of a CTA take part and the traffic
 * stays in L2, which makes the merge of small decode batches several times
 * cheaper. Every byte the kernel reads from the workspace it first writes in
 * the same launch, so it needs no initialisation, but two launches that may
 * run concurrently must not share one workspace.
 * Replaces the same host launcher as glm53_sparse_mla_fwd
 * (csrc/sparse_mla.cu:434-498); this is what the torch op calls, with the
 * workspace taken from the PyTorch caching allocator.
 */
int glm53_sparse_mla_fwd_ws(const void* q, const void* kv, const int32_t* indices, void* out,
                            float* lse, int64_t T, int64_t H, int64_t head_dim, int64_t kv_rows,
                            int64_t kv_width, int64_t topk, int kv_dtype, float sm_scale,
                            float kv_scale, int splits, void* workspace,
                            uint64_t workspace_bytes, void* stream);

/*
 * As glm53_sparse_mla_fwd_ws, for one rank of a head-sharded group (vLLM
 * tensor parallelism: each rank serves H of heads_total heads of every
 * token): the kernel writes its output directly into every rank's full
 * output. outs is a HOST array of n_outs (1..8) device pointers, each to a
 * bf16 [T, heads_total, 512] buffer (16-byte aligned) that this GPU can
 * store to: its own, and the other ranks' buffers mapped into this process
 * (CUDA IPC or symmetric memory, peer access over NVLink). This launch's H
 * heads land at heads [head_offset, head_offset + H) of each buffer, with
 * plain stores from the epilogue, so the output exchange overlaps the rest of
 * the kernel and no all-gather or reorder copy follows. The caller
 * synchronises the ranks after the launch (a barrier on the same stream)
 * before reading the gathered buffers. Requires head_offset + H <=
 * heads_total <= 512.
 * Replaces the output all-gather a tensor-parallel caller would run after the
 * reference op (csrc/sparse_mla.cu:455-505 serves one rank's heads and
 * returns them in a [T, H, 512] tensor of its own).
 */
int glm53_sparse_mla_fwd_heads_gather(const void* q, const void* kv, const int32_t* indices,
                                      void* const* outs, int n_outs, int64_t head_offset,
                                      int64_t heads_total, float* lse, int64_t T, int64_t H,
                                      int64_t head_dim, int64_t kv_rows, int64_t kv_width,
                                      int64_t topk, int kv_dtype, float sm_scale, float kv_scale,
                                      int splits, void* workspace, uint64_t workspace_bytes,
                                      void* stream);

/*
 * Copy this rank's heads [head_offset, head_offset + heads) of `tokens`
 * tokens from src, a bf16 [tokens, heads_total, 512] buffer, into the same
 * place of each buffer in dsts (n_dsts device pointers, 0..8; an entry equal
 * to src is skipped). One cudaMemcpy2DAsync per destination on `stream`, so
 * the copy engines move the data (over NVLink for peer buffers) without SMs.
 * It reads only src, which is local, and writes the destinations.
 * This is the exchange step of the chunked head gather (glm53_sparse_mla.
 * sharding.HeadShardGather, mode "copy"): each wave's attention output is
 * pushed to the peers while the next wave computes.
 * Replaces, like glm53_sparse_mla_fwd_heads_gather, the output all-gather a
 * tensor-parallel caller would run after the reference op.
 */
int glm53_copy_head_slices(void* const* dsts, int n_dsts, const void* src, int64_t tokens,
                           int64_t heads_total, int64_t head_offset, int64_t heads,
                           void* stream);

/*
 * As glm53_sparse_mla_fwd_ws, with the index list in vLLM's request-local
 * form: topk_positions[t][k] (row stride positions_row_stride >= topk, only
 * the first topk columns read) is a token position within request
 * req_id_per_token[t], converted in the kernel's index compaction to the slot
 *   block_table[req][pos / block_size] * block_stride_rows + pos % block_size
 * (block_table row stride block_table_row_stride, max_blocks_per_req valid
 * blocks per row; block_stride_rows = block_size for contiguous pages). A
 * negative position, or a block past max_blocks_per_req, is masked; a slot
 * outside [0, kv_rows) is masked and raises GLM53_DEV_BAD_INDEX. kv_rows must
 * be below 2^31. Pointers to the three int32 arrays need 4-byte alignment.
 * Replaces the reference backend's converter call and its narrowing copy
 * before the op (glm53_sparse_mla/backend.py:341-348, 371-378), i.e. vLLM
 * 0.22's triton_convert_req_index_to_global_index without a prefill
 * workspace (v1/attention/backends/mla/sparse_utils.py:11-84 there): one
 * launch and one [T, topk] int32 round trip through memory fewer.
 */
int glm53_sparse_mla_fwd_paged(const void* q, const void* kv, const int32_t* topk_positions,
                               int64_t positions_row_stride, const int32_t* req_id_per_token,
                               const int32_t* block_table, int64_t block_table_row_stride,
                               int64_t max_blocks_per_req, int64_t block_size,
                               int64_t block_stride_rows, void* out, float* lse, int64_t T,
                               int64_t H, int64_t head_dim, int64_t kv_rows, int64_t kv_width,
                               int64_t topk, int kv_dtype, float sm_scale, float kv_scale,
                               int splits, void* workspace, uint64_t workspace_bytes,
                               void* stream);

/*
 * As glm53_sparse_mla_fwd_ws, for callers that cannot allocate device memory
 * when they call attention (a fixed-size memory pool, an allocator that the
 * call site cannot reach, a runtime that forbids cudaMalloc after start-up):
 * the split-merge workspace is a 32 MiB array built into the library, which
 * every device that loads the library holds until the process exits. This
 * call allocates nothing. A shape whose workspace
 * (glm53_sparse_mla_workspace_bytes) exceeds 32 MiB is rejected with
 * GLM53_ERR_SCRATCH_LIMIT before any launch. With automatic splitting a
 * launch that splits its tokens has at most one CTA per SM (148 on B200),
 * which needs at most 18.5 MiB.
 * The first call on each device looks up the array's device address (and
 * sets the kernels' shared-memory limit); make that first call before any
 * stream capture. All calls share the one array and it keeps the previous
 * call's contents; the kernel writes every scratch byte it reads within the
 * same launch, so nothing needs clearing, but calls that can overlap on the
 * GPU (different streams, or several host threads) race on it.
 * No counterpart in the reference, which has no split merge and no scratch.
 */
int glm53_sparse_mla_fwd_noalloc(const void* q, const void* kv, const int32_t* indices, void* out,
                                 float* lse, int64_t T, int64_t H, int64_t head_dim,
                                 int64_t kv_rows, int64_t kv_width, int64_t topk, int kv_dtype,
                                 float sm_scale, float kv_scale, int splits, void* stream);

/*
 * Argument validation alone, with no CUDA call: returns the status that
 * glm53_sparse_mla_fwd would return before launching. Mirrors the TORCH_CHECKs
 * of the reference host op (csrc/sparse_mla.cu:457-470, 488-496).
 */
int glm53_sparse_mla_check(int64_t T, int64_t H, int64_t head_dim, int64_t kv_rows,
                           int64_t kv_width, int64_t topk, int kv_dtype, int splits);

/* Split count the launcher would use for this shape on the current device. */
int glm53_sparse_mla_auto_splits(int64_t T, int64_t topk, int sm_count);

/*
 * Raise the kernels' dynamic shared-memory limit on the current device. Called
 * implicitly by the first glm53_sparse_mla_fwd on each device; call it
 * explicitly before a CUDA graph capture if the first launch would otherwise
 * happen inside the capture. Replaces the function-local static of
 * csrc/sparse_mla.cu:440-444.
 */
int glm53_sparse_mla_prepare(void);

/*
 * Read (and optionally clear) the device status word of the current device:
 * the OR of glm53_device_status_bits raised by kernels since the last clear.
 * Synchronises the device. Not part of the hot path.
 */
int glm53_sparse_mla_device_status(uint32_t* status, int clear);

/*
 * Set the wall-time limit of every pipeline wait inside the attention kernel
 * for launches made from now on (a CUDA graph keeps the limit it was
 * captured with). ns == 0 restores the default: GLM53_WAIT_TIMEOUT_MS
 * milliseconds if that environment variable is set, else 1 s. When a wait
 * runs out, its CTA stops waiting, retires its own tensor-core work, releases
 * its tensor memory and raises GLM53_DEV_TIMEOUT; the output of that launch
 * is undefined. Process-wide; safe to call from any thread.
 * No counterpart in the reference, whose waits are __syncthreads and a
 * launch check (csrc/sparse_mla.cu:440-452); the bound is how a pipeline
 * fault becomes an error status here instead of a hung GPU.
 */
int glm53_sparse_mla_set_wait_timeout_ns(uint64_t ns);

/* Human-readable text for a glm53_status code. */
const char* glm53_sparse_mla_strerror(int code);

/*
 * Gather-only bandwidth probe: the attention kernel's gather (16-byte
 * cp.async per lane into 64-row swizzled shared-memory tiles, 1 KiB bf16
 * rows) with no math, over a 3-stage ring of 64 KiB tiles. The flattened
 * [T, topk] index list is cut into `ctas` equal contiguous ranges, one per
 * CTA (ctas == 0: one CTA per token, the reference probe's grid); entries
 * outside [0, kv_rows) are skipped. sink (NULL, or one uint32 per CTA)
 * receives the XOR of the first 32-bit word of every row the CTA gathered.
 * The time of one call bounds how fast any kernel can gather the same rows
 * with this load scheme: the attention's gather roof.
 * Replaces the bench-only probe gather_only / gather_roof of the reference
 * (bench/gather_roof.cu:13-55, driven by bench/gather_roof.py:12-23).
 */
int glm53_gather_roof(const void* kv, const int32_t* indices, int64_t T, int64_t topk,
                      int64_t kv_rows, int ctas, uint32_t* sink, void* stream);

/*
 * Latent KV-cache writer (the write that feeds the attention above).
 *
 *   kv_c          [>= T, kv_c_stride] bf16, row t = token t's 512-wide latent
 *                 (kv_c_stride >= 512 elements; rows past T, padding for CUDA
 *                 graphs, are ignored)
 *   kv_cache      paged cache [num_blocks, block_size, 512] of cache_dtype,
 *                 element (b, o, i) at b * block_stride + o * entry_stride + i
 *                 (strides in elements; entries must not overlap)
 *   slot_mapping  [T] int64: token t goes to block slot / block_size at offset
 *                 slot % block_size; slot < 0 (a padded token) writes nothing;
 *                 a slot >= num_blocks * block_size is skipped and raises
 *                 GLM53_DEV_BAD_SLOT in glm53_concat_and_cache_status.
 *   cache_dtype   GLM53_KV_BF16: the row is copied ("auto");
 *                 GLM53_KV_FP8_E4M3: element = e4m3(float(x) / *scale), round
 *                 to nearest even, saturated to +-448 ("fp8" / "fp8_e4m3").
 *   scale         device pointer to the fp32 per-tensor scale (fp8 only; read
 *                 on the device, so no host synchronisation).
 *
 * Replaces, for this path's geometry (kv_lora_rank 512, pe_dim 0), vLLM's
 * concat_and_cache_mla (vllm 0.22.0 vllm/_custom_ops.py:2613-2623), which the
 * reference leaves vLLM to call (its backend keeps the plain fp8 layout,
 * glm53_sparse_mla/backend.py:398-428) through MLAAttentionImpl's
 * do_kv_cache_update (vllm/v1/attention/backend.py:990-1010).
 * Asynchronous on `stream`; no allocation. T == 0 is a no-op.
 */
int glm53_concat_and_cache(const void* kv_c, int64_t kv_c_stride, int64_t T, void* kv_cache,
                           int cache_dtype, int64_t num_blocks, int64_t block_size,
                           int64_t block_stride, int64_t entry_stride,
                           const int64_t* slot_mapping, const float* scale, void* stream);

/* Read (and optionally clear) the cache writer's device status word
 * (GLM53_DEV_BAD_SLOT). Synchronises the device. Not part of the hot path. */
int glm53_concat_and_cache_status(uint32_t* status, int clear);

/*
 * Per-row top-k of the sparse-attention indexer's logits: fills the
 * request-local top-k positions the attention consumes.
 *
 *   logits      [num_rows, stride0] fp32 (stride1 must be 1)
 *   row r covers logits[r, start, end):
 *     decode  (seq_lens != NULL, row_starts = row_ends = NULL):
 *             start = 0, end = seq_lens[r / next_n] - next_n + r % next_n + 1
 *     prefill (seq_lens == NULL): start = row_starts[r], end = row_ends[r]
 *   out         [num_rows, out_stride] int32, the first topk columns written:
 *               len = end - start <= topk: 0, 1, ..., len - 1, then -1;
 *               otherwise the positions (relative to start) of the topk
 *               largest values in no particular order (IEEE order, +NaN above
 *               +inf; which of several values equal to the k-th largest are
 *               taken is unspecified).
 *
 * Replaces vLLM's top_k_per_row_decode / top_k_per_row_prefill (vllm 0.22.0
 * vllm/_custom_ops.py:2799-2840), which vLLM's sparse-attention indexer calls
 * to fill the topk_indices_buffer the reference's backend reads
 * (glm53_sparse_mla/backend.py:310-314 of the reference). 1 <= topk <= 16384.
 * A small batch of rows at least 12K values wide (stride0) runs each row on a
 * cluster of 2 or 4 CTAs, otherwise each row on one CTA; the choice depends
 * only on num_rows, stride0 and the device's SM count, so a captured launch
 * stays valid for every replay of the same shapes.
 * The first call on a device sets the kernels' shared-memory sizes; make it
 * before any stream capture. Asynchronous on `stream`; no allocation.
 */
int glm53_topk_per_row(const float* logits, int64_t num_rows, int64_t stride0, int64_t stride1,
                       const int32_t* seq_lens, int next_n, const int32_t* row_starts,
                       const int32_t* row_ends, int32_t* out, int64_t out_stride, int topk,
                       void* stream);

/* Read (and optionally clear) the top-k kernel's device status word
 * (GLM53_DEV_TIMEOUT: a row load gave up after its time limit).
 * Synchronises the device. Not part of the hot path. */
int glm53_topk_status(uint32_t* status, int clear);

/*
 * Sparse-attention indexer scores over a paged fp8 cache: the logits the
 * top-k above selects from.
 *
 *   q              [B, next_n, H, 128] fp8_e4m3 (H = 32 or 64, next_n = 1, 2
 *                  or 4)
 *   kv_cache       num_blocks blocks, block_bytes apart (a multiple of 16,
 *                  >= block_size * 132; block_size a power of two, 16 to
 *                  1024): block_size rows of 128 e4m3 values, then
 *                  block_size fp32 scales
 *   weights        [B * next_n, H] fp32
 *   context_lens   [B] (token j of request i sees positions
 *                  < context_lens[i] - next_n + j + 1), or with
 *                  per_token_lens, [B * next_n] (token j sees
 *                  < context_lens[i * next_n + j])
 *   block_table    [B, bt_stride] int32, the first max_blocks columns used
 *   logits         [B * next_n, logits_stride] fp32:
 *                  logits[row, p] = scale[p] * sum_h relu(q[h] . k[p]) * w[row, h]
 *                  on visible positions; with `clean`, -inf elsewhere up to
 *                  max_model_len, otherwise untouched.
 *
 * Replaces DeepGEMM's fp8 paged MQA logits as vLLM's sparse-attention
 * indexer calls it (vllm 0.22.0 vllm/utils/deep_gemm.py:407-456, from
 * vllm/model_executor/layers/sparse_attn_indexer.py:324-333); the indexer's
 * top-k then fills the topk_indices_buffer the reference's backend reads
 * (glm53_sparse_mla/backend.py:310-314 of the reference). Positions whose
 * block is past the table or the cache read nothing and raise a bit in
 * glm53_indexer_status. Asynchronous on `stream`; no allocation.
 */
int glm53_indexer_logits(const void* q, const void* kv_cache, const float* weights,
                         const int32_t* context_lens, int per_token_lens,
                         const int32_t* block_table, int64_t B, int next_n, int64_t H,
                         int64_t head_dim, int64_t num_blocks, int64_t block_size,
                         int64_t block_bytes, int64_t bt_stride, int64_t max_blocks,
                         float* logits, int64_t logits_stride, int64_t max_model_len, int clean,
                         void* stream);

/* Read (and optionally clear) the indexer-logits status word (1: a wait gave
 * up after its time limit; 2: a block past the table or the cache was
 * skipped). Synchronises the device. Not part of the hot path. */
int glm53_indexer_status(uint32_t* status, int clear);

#ifdef __cplusplus
}
#endif

#endif /* GLM53_SPARSE_MLA_H_ */
