/*
 * lightserve_b200 — C ABI of the B200 (sm_100a) attention hot path.
 *
 * Each entry point replaces one operator of lightserve's Python/Triton hot
 * path (citations are file:line inside the lightserve project). The ABI takes
 * only plain pointers, sizes, element strides (in elements, not bytes), a
 * dtype code and a cudaStream_t passed as void*. It never allocates device
 * memory and never synchronises: callers own every buffer, including the
 * scratch ("workspace") buffers whose sizes the *_workspace_size helpers
 * report. All launches are recorded on `stream` and can be captured into a
 * CUDA graph.
 *
 * Return value: LSB_OK (0) on success, otherwise an LSB_ERR_* code; the
 * reason is available from lsb_last_error() on the calling thread.
 */
#ifndef LIGHTSERVE_B200_H_
#define LIGHTSERVE_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define LSB_API __attribute__((visibility("default")))
#else
#define LSB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ----------------------------------------------------------------- codes -- */
#define LSB_OK 0
#define LSB_ERR_INVALID 1     /* bad shape, stride, pointer or size        */
#define LSB_ERR_UNSUPPORTED 2 /* valid request this build cannot serve     */
#define LSB_ERR_CUDA 3        /* a CUDA runtime call or launch failed      */

/* lsb_device_error(): the device error words could not be read. */
#define LSB_DEVICE_ERR_QUERY 0xCDA

#define LSB_DTYPE_F32 0
#define LSB_DTYPE_BF16 1
#define LSB_DTYPE_F16 2

/* Attention forward implementation selector (lsb_attn_fwd `impl`). */
#define LSB_IMPL_AUTO 0    /* tcgen05 kernel when eligible, else SIMT kernel */
#define LSB_IMPL_SIMT 1    /* CUDA-core kernel, any dtype / head dim <= 256  */
#define LSB_IMPL_TCGEN05 2 /* tcgen05 + TMEM + TMA kernel; error if ineligible */

/* Message describing the last failure on this thread ("" if none). */
LSB_API const char* lsb_last_error(void);

/* Nonzero if a kernel of this library gave up on a bounded on-chip wait (an
 * mbarrier that never completed); the value names the wait. Reading it
 * synchronises the device. 0 when no kernel ever timed out.
 * LSB_DEVICE_ERR_QUERY when the error words could not be read at all (the
 * CUDA context holds an error; lsb_last_error() names it). */
LSB_API int lsb_device_error(void);

/* Returns lsb_device_error() and clears every error word. No counterpart in
 * the reference (its Triton kernels have no bounded waits). */
LSB_API int lsb_device_error_reset(void);

/* Self-test of the bounded-wait failure path: launches one thread that waits
 * on an mbarrier nothing arrives on; after about one second the wait gives
 * up, the kernel writes *status = 0 (device int) and lsb_device_error()
 * returns 0xE01. The GPU context stays usable. No counterpart in the
 * reference. */
LSB_API int lsb_selftest_bounded_wait(int* status, void* stream);

/* Process-wide switch for programmatic dependent launch (default on): the
 * norm, SwiGLU, RoPE/KV-write, paged-decode, greedy-sampling and linear
 * kernels are launched so that each may start while the previous kernel of
 * its stream finishes, and each waits (griddepcontrol.wait) for that kernel's
 * completion before it touches memory -- this hides launch gaps inside a
 * decode step. Results do not depend on it. Returns the previous setting.
 * No counterpart in the reference. */
LSB_API int lsb_set_programmatic_launch(int enable);

/* Library version string. */
LSB_API const char* lsb_version(void);

/*
 * Fused residual-add + RMSNorm.
 * Replaces fused_add_rmsnorm / _fused_add_rmsnorm_kernel
 * (kernels/fused_rmsnorm_residual.py:73-117, :31-70):
 *   h   = x + residual                       (stored in the input dtype)
 *   out = (float(h) * rsqrt(mean(float(h)^2) + eps) * float(w)) -> dtype
 * x, residual, out, h are [M, N] row-major with row strides ld_*; w is [N].
 */
LSB_API int lsb_rmsnorm_residual(const void* x, const void* residual, const void* weight,
                         void* out, void* h_out, int64_t M, int64_t N,
                         int64_t ld_x, int64_t ld_r, int64_t ld_out, int64_t ld_h,
                         float eps, int dtype, void* stream);

/*
 * FlashAttention forward, O = softmax(Q K^T * scale [+ causal mask]) V.
 * Replaces flash_attention_forward / _flash_attn_fwd_kernel
 * (kernels/flash_attention.py:182-222, :84-179) and, when lse != NULL,
 * _flash_attention_forward_lse / _flash_attn_fwd_lse_kernel
 * (kernels/flash_attention_backward.py:172-199, :88-169).
 * q, k, v, o: [B, H, N, D] with element strides s*[4] = {b, h, n, d}.
 * lse (optional): fp32 [B, H, N] contiguous, lse = rowmax + ln(rowsum(exp)).
 */
LSB_API int lsb_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse,
                 int64_t B, int64_t H, int64_t N, int64_t D,
                 const int64_t* sq, const int64_t* sk, const int64_t* sv,
                 const int64_t* so, float scale, int causal, int dtype, int impl,
                 void* stream);

/*
 * Variable-length FlashAttention forward over sequences packed along the
 * token axis (the prefill shape of a paged-KV server). lightserve's forward
 * takes one [B, H, N, D] batch with Nq == Nkv (kernels/flash_attention.py:
 * 192-199); its block manager admits prompts of different lengths
 * (engine/request.py:86-93, engine/block_manager.py:47-157), which this
 * entry point serves without padding. Sequence s holds tokens
 * [cu_seqlens[s], cu_seqlens[s+1]) of q, k, v, o ([total_tokens, H, D],
 * element strides {token, head, 1}); cu_seqlens is int32 [num_seqs + 1] in
 * device memory, non-decreasing from 0 to total_tokens; max_seqlen bounds
 * the longest sequence. Attention (causal within a sequence when causal != 0)
 * never crosses sequences. lse (optional): fp32 [H, total_tokens].
 * bf16 / fp16 with D in {64, 128} (tcgen05 kernel only).
 */
LSB_API int lsb_attn_fwd_varlen(const void* q, const void* k, const void* v, void* o, float* lse,
                        const int32_t* cu_seqlens, int64_t num_seqs, int64_t max_seqlen,
                        int64_t total_tokens, int64_t H, int64_t D,
                        const int64_t* sq, const int64_t* sk, const int64_t* sv,
                        const int64_t* so, float scale, int causal, int dtype, void* stream);

/* Bytes of fp32 scratch lsb_attn_bwd needs: Dsum [B,H,N] + dQ accumulator
 * [B,H,N,D] (each region 256-byte aligned). */
LSB_API int64_t lsb_attn_bwd_workspace_size(int64_t B, int64_t H, int64_t N, int64_t D);

/*
 * FlashAttention backward (recomputation strategy).
 * Replaces _flash_attention_backward and its two kernels
 * (kernels/flash_attention_backward.py:333-382, :202-229, :232-330):
 *   Dsum = rowsum(dO * O); P = exp(S - lse); dV = P^T dO; dP = dO V^T;
 *   dS = P * (dP - Dsum); dK = dS^T Q * scale; dQ = dS K * scale.
 * Strides are element strides {b, h, n, d} for q,k,v,o,do,dq,dk,dv.
 * workspace: >= lsb_attn_bwd_workspace_size bytes, 256-byte aligned.
 */
LSB_API int lsb_attn_bwd(const void* q, const void* k, const void* v, const void* o,
                 const void* dout, const float* lse, void* dq, void* dk, void* dv,
                 int64_t B, int64_t H, int64_t N, int64_t D,
                 const int64_t* sq, const int64_t* sk, const int64_t* sv,
                 const int64_t* so, const int64_t* sdo, const int64_t* sdq,
                 const int64_t* sdk, const int64_t* sdv, float scale, int causal,
                 int dtype, int impl, void* workspace, int64_t workspace_bytes,
                 void* stream);

/*
 * Write new K/V rows into the paged KV cache.
 * No counterpart kernel exists in lightserve (engine/README.md:142-155 says
 * the decode path is missing); the slot arithmetic follows the block-table
 * convention of engine/block_manager.py:58-61 (block i of a request holds
 * tokens [i*block_size, (i+1)*block_size)).
 * k, v: [T, H, D] (strides {t, h} in elements, d contiguous).
 * k_cache, v_cache: [num_blocks, H, block_size, D] contiguous.
 * slot_mapping: int64 [T], slot = block_id * block_size + offset; a negative
 * slot skips that row.
 */
LSB_API int lsb_kv_cache_write(const void* k, const void* v, void* k_cache, void* v_cache,
                       const int64_t* slot_mapping, int64_t T, int64_t H, int64_t D,
                       int64_t num_blocks, int64_t block_size,
                       int64_t sk_t, int64_t sk_h, int64_t sv_t, int64_t sv_h,
                       int dtype, void* stream);

/* Bytes of fp32 scratch lsb_paged_decode needs for split-context partials. */
LSB_API int64_t lsb_paged_decode_workspace_size(int64_t S, int64_t H, int64_t D,
                                        int64_t max_blocks_per_seq,
                                        int64_t block_size);

/*
 * Paged-KV decode attention (one query token per sequence).
 * New operator: lightserve has no decode-shaped attention kernel
 * (engine/README.md:142-147, engine/request.py:86-93); its oracle is the
 * full-recompute decode of model/cuda_graph_decode.py:108-149 over
 * model/minimal_llama.py:253-293.
 * q, o: [S, H, D] (strides {s, h}, d contiguous).
 * k_cache, v_cache: [num_blocks, H, block_size, D] contiguous.
 * block_tables: int32 [S, max_blocks_per_seq] row-major; context_lens: int32 [S].
 * o[s,h] = softmax(q[s,h] . K[s,h,:L]^T * scale) V[s,h,:L], L = context_lens[s].
 * workspace: >= lsb_paged_decode_workspace_size bytes (may be NULL when that
 * size is 0).
 */
LSB_API int lsb_paged_decode(const void* q, const void* k_cache, const void* v_cache,
                     const int32_t* block_tables, const int32_t* context_lens,
                     void* o, int64_t S, int64_t H, int64_t D,
                     int64_t max_blocks_per_seq, int64_t block_size,
                     int64_t num_blocks, int64_t sq_s, int64_t sq_h,
                     int64_t so_s, int64_t so_h, float scale, int dtype,
                     void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Fused RoPE + paged KV-cache write for one decode step (one token per
 * sequence). Replaces the decode-time use of lightserve's apply_rope
 * (model/minimal_llama.py:167-182: q*cos + rotate_half(q)*sin with each
 * product and the sum rounded to the model dtype) plus the cache write and
 * slot lookup through the block table (engine/block_manager.py:58-61).
 * qkv: [S, 3, H, D] with strides {s_s, s_part, s_h} (d contiguous);
 * cos/sin tables: [max_pos, D] with row stride s_pos; positions: int64 [S];
 * block_tables: int32 [S, max_blocks_per_seq]. Writes rotated q to q_out
 * [S, H, D] contiguous, rotated k and raw v into the caches at slot
 * (block_tables[s][pos / block_size], pos % block_size), and
 * context_lens[s] = pos + 1 when context_lens != NULL.
 */
LSB_API int lsb_rope_kv_write(const void* qkv, int64_t s_s, int64_t s_part, int64_t s_h,
                              const void* cos_table, const void* sin_table, int64_t s_pos,
                              const int64_t* positions, const int32_t* block_tables,
                              int64_t max_blocks_per_seq, void* q_out, void* k_cache,
                              void* v_cache, int32_t* context_lens, int64_t S, int64_t H,
                              int64_t D, int64_t num_blocks, int64_t block_size, int dtype,
                              void* stream);

/*
 * Fused RoPE + paged KV-cache write for a packed prefill: lsb_rope_kv_write
 * for T tokens of any sequences, each with its own position and cache slot
 * (slot_mapping: int64 [T], block * block_size + offset as produced from
 * engine/block_manager.py:58-61's tables; < 0 skips the cache write).
 * Writes rotated q to q_out and (when k_out != NULL) rotated k to k_out,
 * both [T, H, D] contiguous, for lsb_attn_fwd_varlen.
 */
LSB_API int lsb_rope_kv_write_slots(const void* qkv, int64_t s_s, int64_t s_part, int64_t s_h,
                                    const void* cos_table, const void* sin_table, int64_t s_pos,
                                    const int64_t* positions, const int64_t* slot_mapping,
                                    void* q_out, void* k_out, void* k_cache, void* v_cache,
                                    int64_t T, int64_t H, int64_t D, int64_t num_blocks,
                                    int64_t block_size, int dtype, void* stream);

/*
 * Fused SwiGLU of the Llama MLP: out = silu(gate) * up with
 * gate = gu[:, :I], up = gu[:, I:] (gu = [S, 2I], the fused gate|up GEMM
 * output, row stride ld_gu; out = [S, I], row stride ld_out). Replaces
 * F.silu(gate_proj(h)) * up_proj(h) (model/minimal_llama.py:231-233) with the
 * same roundings: silu in fp32 rounded to dtype, then the dtype product.
 */
LSB_API int lsb_swiglu(const void* gu, void* out, int64_t S, int64_t I, int64_t ld_gu,
                       int64_t ld_out, int dtype, void* stream);

/*
 * Greedy next token of every decode row: tokens[s] = argmax(logits[s, :V])
 * (torch.argmax order: the first index of the maximum; NaN counts as the
 * maximum), and positions[s] += 1 when positions is not NULL. logits is
 * [S, V] with row stride ld (f32 / bf16 / fp16); tokens and positions are
 * int64 [S]. Replaces `logits[:, -1].argmax(-1)` and the write of the next
 * id in lightserve's decode loop (model/cuda_graph_decode.py:114-118).
 */
LSB_API int lsb_greedy_next(const void* logits, int64_t S, int64_t V, int64_t ld, int dtype,
                            int64_t* tokens, int64_t* positions, void* stream);

/*
 * Weight-streaming linear layer for decode batches: y[S, N] = x[S, K] @ W[K, N]
 * with fp32 accumulation and one rounding to dtype (bf16 or fp16).
 * Replaces the projections of lightserve's decode step, `h @ w` in
 * model/minimal_llama.py:216-234 (q/k/v, o, gate/up, down) and :249
 * (lm_head), which lightserve runs through torch.matmul / its Triton
 * kernels/tiled_matmul.py:55-151.
 * The weight is packed once with lsb_linear_pack from W^T ([N, K], row
 * stride ldw, K contiguous) into lsb_linear_packed_bytes(N, K) bytes of
 * 16 KiB tiles (128 features x 64 of K, 128-byte swizzled, zero-padded).
 * x is [S, K] (row stride ldx), y is [S, N] (row stride ldy).
 * Limits: 1 <= S <= 128; K a multiple of 8; x and the packed weight 16-byte
 * aligned, ldx a multiple of 8. Needs no scratch memory; the result does not
 * depend on timing (fixed summation order).
 * pdl != 0 launches with programmatic stream serialisation: the weight
 * stream may start while the previous kernel of the stream finishes (x is
 * read only after that kernel has completed).
 */
LSB_API int64_t lsb_linear_packed_bytes(int64_t N, int64_t K);
LSB_API int lsb_linear_pack(const void* w_t, int64_t ldw, int64_t N, int64_t K, int dtype,
                            void* packed, int64_t packed_bytes, void* stream);
LSB_API int lsb_linear(const void* x, int64_t ldx, const void* w_packed, void* y, int64_t ldy,
                       int64_t S, int64_t N, int64_t K, int dtype, int pdl, void* stream);

/*
 * Allocation-free paged decode. No counterpart exists in lightserve: this is
 * lsb_paged_decode for callers that cannot allocate device memory (runtimes
 * whose own pool owns the GPU's memory, FFI bindings without access to the
 * host framework's allocator). The split-context scratch comes from a fixed
 * 8 MiB array inside the library (lsb_paged_decode_static_scratch_capacity());
 * sizes whose lsb_paged_decode_workspace_size exceeds it are rejected with
 * LSB_ERR_INVALID. The first call on each device looks up the array's device
 * address and should come before any stream capture. Calls share the array:
 * calls that overlap on the GPU race and must be serialised by the caller.
 * Arguments are those of lsb_paged_decode without the workspace.
 */
LSB_API int64_t lsb_paged_decode_static_scratch_capacity(void);
LSB_API int lsb_paged_decode_static_scratch(
    const void* q, const void* k_cache, const void* v_cache, const int32_t* block_tables,
    const int32_t* context_lens, void* o, int64_t S, int64_t H, int64_t D,
    int64_t max_blocks_per_seq, int64_t block_size, int64_t num_blocks, int64_t sq_s,
    int64_t sq_h, int64_t so_s, int64_t so_h, float scale, int dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LIGHTSERVE_B200_H_ */
