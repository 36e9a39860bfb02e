/*
 * lean_attn.h — C ABI of the B200 (sm_100a) paged-attention backend for the
 * lean-infer Qwen3 engine.
 *
 * Every entry point takes plain device pointers, element strides and sizes, and
 * the CUDA stream to launch on; none allocates device memory, synchronises the
 * host or calls exit/abort. Each returns LA_OK or an la_status code; argument
 * errors are reported before anything is launched. Conditions that can only be
 * seen on the device (a block id outside the pool, a sequence longer than its
 * block table, a bounded wait that ran out) are recorded in the caller's
 * optional device error word (`dev_error`, one int32 in device memory; the
 * first non-zero code wins) and the offending access is skipped.
 *
 * Layout contract (reference: leaninfer/engine/cache_manager.py:53-60, 63-76):
 *   k_cache / v_cache : [num_blocks, block_size, num_kv_heads, head_dim] bf16,
 *                       head_dim contiguous; the block/token/head strides are
 *                       passed explicitly so a layer slice of the engine's
 *                       [L, NB, BS, Hkv, D] pool can be used in place.
 *   block_table       : [batch, max_blocks_per_seq] int32, logical block ->
 *                       physical block id. Block 0 is the engine's trash block.
 *   cache_seqlens     : [batch] int32, number of valid keys per sequence.
 *
 * Graph capture: all launches are asynchronous on `stream`, use a grid that
 * does not depend on device data, and take their scratch from the caller, so
 * a sequence of calls can be captured in a CUDA graph. Call la_init() for the
 * device once before the first capture.
 */
#ifndef LEAN_ATTN_H_
#define LEAN_ATTN_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LA_VERSION 1

typedef enum {
  LA_OK = 0,
  LA_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad size, inconsistent shapes */
  LA_ERR_UNSUPPORTED = 2,      /* a shape the kernels are not built for (e.g. head_dim != 128) */
  LA_ERR_ALIGNMENT = 3,        /* pointer or stride not aligned as TMA / vector loads need */
  LA_ERR_WORKSPACE = 4,        /* workspace missing or smaller than la_*_workspace_size() */
  LA_ERR_CUDA = 5,             /* a CUDA runtime/driver call failed (see la_last_cuda_error) */
  LA_ERR_TENSOR_MAP = 6        /* cuTensorMapEncodeTiled rejected a descriptor */
} la_status;

/* Codes written to the device error word. */
#define LA_DEVERR_WAIT_TIMEOUT 1   /* a bounded mbarrier wait ran out; kernel returned early */
#define LA_DEVERR_BLOCK_ID 2       /* block_table entry outside [0, num_blocks) */
#define LA_DEVERR_SEQLEN 3         /* a sequence needs more blocks than max_blocks_per_seq */
#define LA_DEVERR_ROPE_POS 4       /* a position is outside the rope table */
#define LA_DEVERR_SMEM_ALIGN 5     /* dynamic shared memory base not 1024-byte aligned (kernel returned) */

int la_version(void);
const char* la_status_string(int status);
/* The last CUDA error code seen by the library on this thread (0 if none). */
int la_last_cuda_error(void);

/* Per-device one-time setup: shared-memory opt-in of every kernel and module
 * load. Call before capturing any call into a CUDA graph. Idempotent. */
int la_init(int device);

/* ------------------------------------------------------------------------
 * (a) Fused pre-attention: per-head QK RMSNorm, NeoX RoPE and paged KV write.
 *
 * Replaces, for one layer, the op sequence of leaninfer/qwen3/model.py:50-55:
 *   q = q_norm(q_proj(x)); k = k_norm(k_proj(x))          (model.py:50-51)
 *   q = apply_rope(q, cos, sin); k = apply_rope(k, ...)    (model.py:53-54,
 *                                                           layers.py:18-23)
 *   cache.write(layer, block_tables, pos, k, v)            (model.py:55,
 *                                                           cache_manager.py:63-76)
 * with the rounding order of the reference: RMSNorm in fp32 (weight multiply
 * included) rounded once to bf16; x*cos, rotate_half(x)*sin and their sum each
 * rounded to bf16. rope_cos / rope_sin are [rope_max_pos, head_dim/2] bf16
 * tables indexed by absolute position (the first half of build_rope's
 * cat(angles, angles), layers.py:7-15).
 *
 * Tokens: if cu_seqlens is NULL, num_tokens = num_seqs * q_len and token i is
 * position seq_start_pos[i / q_len] + i % q_len of sequence i / q_len
 * (decode: q_len = 1). Otherwise token i belongs to the sequence s with
 * cu_seqlens[s] <= i < cu_seqlens[s+1] (packed varlen prefill).
 * q / k / v: [num_tokens, heads, head_dim] with the given element strides.
 * q_out receives the normed, rotated q; k (normed, rotated) and v are written
 * to k_cache / v_cache at block_table[s][col / block_size], col % block_size.
 * k_out (nullable) also receives the normed, rotated k as [num_tokens, Hkv, D]
 * (the fresh keys a prefill attends to, model.py:56-57).
 * A sequence whose seq_start_pos is negative is idle: nothing is written to
 * the cache, its rows of q_out (and k_out) are zeros and no error is raised.
 * With cache_seqlens 0 for such a row, la_paged_decode returns zeros for it,
 * so idle batch rows need no trash block (the reference points them at block
 * 0 with position 0 and context 1, llm_engine.py:67-69, which also works).
 * ------------------------------------------------------------------------ */
int la_qk_norm_rope_paged_write(
    const void* q, int64_t q_token_stride, int64_t q_head_stride,
    const void* k, int64_t k_token_stride, int64_t k_head_stride,
    const void* v, int64_t v_token_stride, int64_t v_head_stride,
    const void* q_norm_weight, const void* k_norm_weight, float eps,
    const void* rope_cos, const void* rope_sin, int64_t rope_max_pos,
    const int64_t* seq_start_pos, const int32_t* cu_seqlens,
    int num_seqs, int q_len, int64_t num_tokens,
    const int32_t* block_table, int64_t bt_seq_stride, int max_blocks_per_seq,
    void* k_cache, void* v_cache,
    int64_t kv_block_stride, int64_t kv_token_stride, int64_t kv_head_stride,
    int64_t num_blocks, int block_size,
    void* q_out, int64_t qo_token_stride, int64_t qo_head_stride,
    void* k_out, int64_t ko_token_stride, int64_t ko_head_stride,
    int num_q_heads, int num_kv_heads, int head_dim,
    int* dev_error, cudaStream_t stream);

/* Plain paged KV write (no norm, no rope): the scatter of BlockCache.write
 * (leaninfer/engine/cache_manager.py:63-76). k / v: [num_tokens, Hkv, D]. */
int la_paged_kv_write(
    const void* k, int64_t k_token_stride, int64_t k_head_stride,
    const void* v, int64_t v_token_stride, int64_t v_head_stride,
    const int64_t* seq_start_pos, const int32_t* cu_seqlens,
    int num_seqs, int q_len, int64_t num_tokens,
    const int32_t* block_table, int64_t bt_seq_stride, int max_blocks_per_seq,
    void* k_cache, void* v_cache,
    int64_t kv_block_stride, int64_t kv_token_stride, int64_t kv_head_stride,
    int64_t num_blocks, int block_size,
    int num_kv_heads, int head_dim,
    int* dev_error, cudaStream_t stream);

/* ------------------------------------------------------------------------
 * (b) Paged GQA decode attention, split-KV with a combine pass.
 *
 * Replaces flash_attn.flash_attn_with_kvcache(q, k_cache, v_cache,
 * cache_seqlens=, block_table=, causal=True, num_splits=1) as called at
 * leaninfer/qwen3/model.py:60-67 (one query token per sequence).
 * q: [batch, 1, num_q_heads, head_dim] bf16; out: same shape. Query head h
 * attends to kv head h / (num_q_heads / num_kv_heads) over keys
 * 0 .. cache_seqlens[b]-1. softmax_lse (nullable): [batch, num_q_heads] fp32,
 * natural log. A sequence with cache_seqlens[b] <= 0 gets a zero output and
 * lse = -inf. block_size must be a multiple of 16; head_dim must be 128;
 * num_kv_heads must divide 8 and num_q_heads / num_kv_heads must be <= 8.
 * workspace: device memory of at least la_paged_decode_workspace_size() bytes
 * (partial results of sequences split across CTAs), 256-byte aligned.
 * ------------------------------------------------------------------------ */
int la_paged_decode_workspace_size(int device, int num_q_heads, int num_kv_heads, int head_dim,
                                   size_t* bytes);

int la_paged_decode(
    const void* q, int64_t q_batch_stride, int64_t q_head_stride,
    const void* k_cache, const void* v_cache,
    int64_t kv_block_stride, int64_t kv_token_stride, int64_t kv_head_stride,
    int64_t num_blocks, int block_size,
    const int32_t* block_table, int64_t bt_seq_stride, int max_blocks_per_seq,
    const int32_t* cache_seqlens,
    int batch, int num_q_heads, int num_kv_heads, int head_dim,
    float softmax_scale,
    void* out, int64_t out_batch_stride, int64_t out_head_stride,
    float* softmax_lse,
    void* workspace, size_t workspace_bytes,
    int* dev_error, cudaStream_t stream);

/* ------------------------------------------------------------------------
 * KV-head-sharded decode with the all-gather fused in (NVLink peer stores).
 *
 * For P ranks (one process per GPU) each holding kv heads
 * [r*Hkv/P, (r+1)*Hkv/P) of every request: rank r runs la_paged_decode on
 * its heads (num_q_heads / num_kv_heads = this rank's counts) and stores
 * each output row into every rank's gather buffer [batch, P*num_q_heads, D]
 * at heads [r*num_q_heads, (r+1)*num_q_heads), over NVLink; every combine
 * CTA that stored fences once at system scope. la_p2p_barrier, next on the same
 * stream, completes the exchange: after it the gather buffer holds all
 * heads. Replaces the NCCL all-gather of the attention outputs before
 * o_proj (leaninfer/qwen3/model.py:68-69) for the KV-head-sharded variant;
 * the reference itself is single-GPU.
 * gather_bufs: host array of `world` device pointers in rank order (own
 * buffer included; peers' mapped with la_p2p_open). A gather buffer is
 * written by every rank, so a caller double-buffers it across consecutive
 * calls (the barrier of call n+1 orders call n+2's stores after call n's
 * reads on every rank).
 * ------------------------------------------------------------------------ */
int la_paged_decode_allgather(
    const void* q, int64_t q_batch_stride, int64_t q_head_stride,
    const void* k_cache, const void* v_cache,
    int64_t kv_block_stride, int64_t kv_token_stride, int64_t kv_head_stride,
    int64_t num_blocks, int block_size,
    const int32_t* block_table, int64_t bt_seq_stride, int max_blocks_per_seq,
    const int32_t* cache_seqlens,
    int batch, int num_q_heads, int num_kv_heads, int head_dim,
    float softmax_scale,
    void* const* gather_bufs, int64_t out_batch_stride, int64_t out_head_stride,
    int rank, int world,
    void* workspace, size_t workspace_bytes,
    int* dev_error, cudaStream_t stream);

/* Device-side barrier of `world` ranks on `stream` (one 32-thread launch):
 * publishes this rank's next epoch into word [rank] of every rank's signal
 * words (store-release, system scope), then waits until every peer's epoch in
 * this rank's words has reached it (bounded: LA_DEVERR_WAIT_TIMEOUT after 2 s,
 * then returns). Peer stores made earlier on each rank's stream with a
 * system-scope fence are visible after it. signals: host array of `world`
 * device pointers to each rank's signal words (world + 1 uint32, zeroed once
 * by la_p2p_alloc), rank order. */
int la_p2p_barrier(unsigned int* const* signals, int world, int rank, int* dev_error, cudaStream_t stream);

/* The publishing half of la_p2p_barrier alone: this rank's next epoch goes to
 * every rank's word [rank]; nothing waits. For a consumer that waits for each
 * peer's epoch itself, as la_o_proj_gathered does. */
int la_p2p_publish(unsigned int* const* signals, int world, int rank, int* dev_error, cudaStream_t stream);

/* o_proj of the KV-head-sharded partition, fused with its all-gather:
 *   out[m, n] = sum_k gathered[m, k] * weight[n, k]   (bf16 in, fp32
 * accumulation on tcgen05, bf16 out), the o_proj Linear of
 * leaninfer/qwen3/model.py:68-69 applied to this rank's gather buffer
 * [m, k = P*num_q_heads*D] right after la_paged_decode_allgather and
 * la_p2p_publish on the same stream. Columns [q*k/P, (q+1)*k/P) belong to
 * rank q: the kernel reads them only after rank q's epoch in `signals` (this
 * rank's signal words: [q] rank q's epoch, [world] this rank's own) has
 * reached this rank's own, waiting for each peer separately (bounded:
 * LA_DEVERR_WAIT_TIMEOUT after 2 s, the output is then invalid), so the
 * peers' transfers overlap the GEMM and no barrier is needed. The columns are
 * summed in one fixed order on every rank (all ranks get the same bits). With
 * world = 1 it is a plain GEMM. k a multiple of 64 * world, n of 32; rows
 * 16-byte aligned. No counterpart in the single-GPU reference beyond the
 * Linear itself. */
int la_o_proj_gathered(const void* gathered, int64_t gathered_row_stride,
                       const void* weight, int64_t weight_row_stride,
                       void* out, int64_t out_row_stride,
                       int m, int n, int k,
                       const unsigned int* signals, int world, int rank,
                       int* dev_error, cudaStream_t stream);

/* Peer-memory setup (host-side, outside the hot path; these allocate):
 * la_p2p_alloc: cudaMalloc + zero + CUDA IPC handle (64 bytes) to share;
 * la_p2p_open: map a peer's handle; la_p2p_close / la_p2p_free undo them. */
int la_p2p_alloc(size_t bytes, void** ptr, void* ipc_handle);
int la_p2p_open(const void* ipc_handle, void** peer_ptr);
int la_p2p_close(void* peer_ptr);
int la_p2p_free(void* ptr);

/* Allocation-free form of la_paged_decode, for callers that cannot allocate
 * device memory where they run decode: a host framework that owns every
 * device allocation (a plugin may not call cudaMalloc behind its back), a
 * runtime that hands out device memory only from a fixed arena reserved at
 * start-up, or a latency-bound loop where an allocation would synchronise
 * the device. It has no counterpart in the
 * reference (flash-attn allocates its own split buffers).
 * Same arguments and results as la_paged_decode without the workspace: the
 * split-KV partials live in a fixed LA_NOALLOC_SCRATCH_BYTES array inside
 * this library, held on every GPU that loads it until the process exits.
 * Calls whose partials need more (2 * #SMs * num_q_heads * (head_dim + 1)
 * fp32, e.g. more than 27 query heads on a 148-SM B200) return
 * LA_ERR_WORKSPACE. No call allocates. All calls share the array, so calls
 * that overlap on the GPU (other streams or threads) race; nothing in it must
 * start at zero. The first call on each device resolves the array's device
 * address (and loads the module there): make that first call before any
 * stream capture. The address is resolved again whenever the current CUDA
 * context differs from the one it was resolved in (after a device reset, or
 * under a caller's own non-primary context). */
#define LA_NOALLOC_SCRATCH_BYTES (4u << 20)

int la_paged_decode_noalloc(
    const void* q, int64_t q_batch_stride, int64_t q_head_stride,
    const void* k_cache, const void* v_cache,
    int64_t kv_block_stride, int64_t kv_token_stride, int64_t kv_head_stride,
    int64_t num_blocks, int block_size,
    const int32_t* block_table, int64_t bt_seq_stride, int max_blocks_per_seq,
    const int32_t* cache_seqlens,
    int batch, int num_q_heads, int num_kv_heads, int head_dim,
    float softmax_scale,
    void* out, int64_t out_batch_stride, int64_t out_head_stride,
    float* softmax_lse,
    int* dev_error, cudaStream_t stream);

/* ------------------------------------------------------------------------
 * (c) Causal varlen prefill attention on tcgen05 / TMEM.
 *
 * Replaces F.scaled_dot_product_attention(q, k, v, is_causal=True,
 * enable_gqa=True) at leaninfer/qwen3/model.py:56-57 (one prompt, B=1) with
 * the flash-attn varlen contract: q [total_tokens, Hq, D], k / v
 * [total_tokens, Hkv, D] bf16 holding num_seqs packed sequences, sequence s
 * being tokens cu_seqlens[s] .. cu_seqlens[s+1]-1 (int32, on the device);
 * max_seqlen >= every length (a shorter value is reported as
 * LA_DEVERR_SEQLEN). causal != 0 masks key j > query i within a sequence.
 * out: [total_tokens, Hq, D] bf16 (strides and base 16-byte aligned).
 * softmax_lse (nullable): [Hq, total_tokens] fp32, natural log.
 * head_dim must be 128 and Hq / Hkv one of 1, 2, 4, 8. No workspace.
 * ------------------------------------------------------------------------ */
int la_prefill_varlen(
    const void* q, int64_t q_token_stride, int64_t q_head_stride,
    const void* k, int64_t k_token_stride, int64_t k_head_stride,
    const void* v, int64_t v_token_stride, int64_t v_head_stride,
    const int32_t* cu_seqlens, int num_seqs, int max_seqlen, int64_t total_tokens,
    int num_q_heads, int num_kv_heads, int head_dim,
    float softmax_scale, int causal,
    void* out, int64_t out_token_stride, int64_t out_head_stride,
    float* softmax_lse,
    int* dev_error, cudaStream_t stream);

/* ------------------------------------------------------------------------
 * Chunked prefill over the paged cache (kernel (c) with paged keys).
 * Replaces flash_attn_with_kvcache with q_len > 1 at its call site
 * (leaninfer/qwen3/model.py:60-67; the chunked prefill of README.md:112-124)
 * and flash-attn's varlen call with a block_table.
 *
 * Sequence s has queries at packed rows [cu_seqlens_q[s], cu_seqlens_q[s+1])
 * of q [total_q, Hq, D] — or, with cu_seqlens_q == NULL, q_len queries at rows
 * [s*q_len, (s+1)*q_len) (total_q = num_seqs*q_len; max_seqlen_q ignored) —
 * and cache_seqlens[s] keys in the pool [num_blocks, block_size, Hkv, D]
 * through block_table row s (the chunk's own keys already written there, e.g.
 * by la_qk_norm_rope_paged_write). Causal masking is bottom-right aligned:
 * query i of n sees key j iff j <= i + cache_seqlens[s] - n; a row that sees
 * no key is written as zeros (lse -inf). block_size: a multiple of 128, or
 * 16, 32 or 64. Pool slots past a sequence's last key are never used (they may hold
 * anything, NaN included). out [total_q, Hq, D]; softmax_lse (nullable)
 * [Hq, total_q], natural log. Block ids outside [0, num_blocks) and keys past
 * the block table are reported on dev_error and read as zeros.
 * ------------------------------------------------------------------------ */
int la_prefill_paged(
    const void* q, int64_t q_token_stride, int64_t q_head_stride,
    const void* k_cache, const void* v_cache,
    int64_t kv_block_stride, int64_t kv_token_stride, int64_t kv_head_stride,
    int64_t num_blocks, int block_size,
    const int32_t* block_table, int64_t bt_seq_stride, int max_blocks_per_seq,
    const int32_t* cache_seqlens,
    const int32_t* cu_seqlens_q, int q_len, int num_seqs, int max_seqlen_q, int64_t total_q,
    int num_q_heads, int num_kv_heads, int head_dim,
    float softmax_scale, int causal,
    void* out, int64_t out_token_stride, int64_t out_head_stride,
    float* softmax_lse,
    int* dev_error, cudaStream_t stream);

/* ------------------------------------------------------------------------
 * Decode-step glue (one launch each; no counterpart in the attention path).
 * la_add_rms_norm: h' = bf16(h + a) (a nullable: h' = h), written to h_out
 * (nullable; may alias h), and x_out = bf16(h' * rsqrt(mean(h'^2) + eps) * w)
 * computed in fp32 — the residual add closing a sub-layer and the nn.RMSNorm
 * opening the next (leaninfer/qwen3/model.py:80-83, 75-76, 92). bf16 rows of
 * n elements (n a multiple of 8, at most 4096), 16-byte aligned rows.
 * la_silu_mul: out = bf16(SiLU(gate) * up) from gate_up [rows, 2n] = gate |
 * up (Qwen3MLP with a fused gate/up projection, model.py:32-33).
 * ------------------------------------------------------------------------ */
int la_add_rms_norm(const void* h, int64_t h_row_stride, const void* a, int64_t a_row_stride,
                    void* h_out, int64_t h_out_row_stride, void* x_out, int64_t x_out_row_stride,
                    const void* weight, int64_t rows, int n, float eps, cudaStream_t stream);
int la_silu_mul(const void* gate_up, int64_t gate_up_row_stride, void* out, int64_t out_row_stride,
                int64_t rows, int n, cudaStream_t stream);

/* la_argmax_rows: out[r] = index of the maximum of row r of a bf16 matrix
 * [rows, cols] (row stride in elements), int64 — the greedy next token,
 * logits[:, -1].argmax(-1) (leaninfer/engine/llm_engine.py:86, 111, 135),
 * with torch.argmax's rules: the first index holding the maximum (+0 and -0
 * equal), and a NaN counts as larger than every number. cols >= 1; rows whose
 * starts are 16-byte aligned are read with 16-byte loads. */
int la_argmax_rows(const void* x, int64_t row_stride, int64_t rows, int64_t cols, int64_t* out,
                   cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* LEAN_ATTN_H_ */
