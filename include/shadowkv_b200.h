/*
 * shadowkv_b200 -- C ABI of the B200 (sm_100a) kernels for ShadowKV's sparse
 * decode-attention step.
 *
 * Conventions
 *  - Every entry point returns an int status (skv_status).  On failure the
 *    message of the calling thread's last error is available from
 *    skv_last_error().  Nothing in the library exits the process.
 *  - Pointers are plain device pointers, except the `values` argument of the
 *    V-gather functions, which must be page-locked host memory mapped into
 *    the device address space (cudaHostAlloc / cudaHostRegister with
 *    cudaHostRegisterMapped, or torch pin_memory).  That pointer is checked
 *    with cudaPointerGetAttributes before launch; pageable memory is
 *    rejected with SKV_ERR_NOT_PINNED.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *    stream).  Every launch goes to that stream; no call synchronizes.
 *  - bf16 arrays are passed as void* (2-byte elements); ids are int64_t or
 *    int32_t exactly as in the reference binding.
 *  - Index errors that can only be seen on the device (a chunk id beyond the
 *    host buffer, a slot beyond the budget) are counted by the kernels into
 *    a per-device error word and the access is skipped;
 *    skv_device_errors() reads and clears it.
 *
 * The first twelve functions are the reference's Python bindings
 * (kernels/main.cu:24-37, C++ signatures kernels/functions.h:23-121) with
 * the same argument order and meaning; the torch::Tensor arguments become
 * raw pointers.  The skv_decode_* functions are the fused decode path of
 * this library (no reference counterpart as single calls; they implement
 * models/kvcache/shadow.py:547-597 and models/attention/shadow.py:22-48).
 */
#ifndef SHADOWKV_B200_H
#define SHADOWKV_B200_H

#include <stdint.h>
#include <stddef.h>

#if defined(__GNUC__)
#define SKV_API __attribute__((visibility("default")))
#else
#define SKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    SKV_OK = 0,
    SKV_ERR_INVALID_ARGUMENT = 1, /* bad size / null pointer / misaligned pointer */
    SKV_ERR_UNSUPPORTED = 2,      /* shape outside what the kernels implement */
    SKV_ERR_CUDA = 3,             /* a CUDA runtime call or launch failed */
    SKV_ERR_NOT_PINNED = 4,       /* host pointer is not device-accessible */
} skv_status;

/* Message of the calling thread's last failing call ("" if none). */
SKV_API const char *skv_last_error(void);

/* Library version (major*10000 + minor*100 + patch). */
SKV_API int skv_version(void);

/* Read (and clear) the device-side error counter of the current device.
 * *count = number of skipped out-of-range accesses since the last call,
 * *first_code = kind of the first one (1 host chunk id, 2 slot, 3 row). */
SKV_API int skv_device_errors(uint32_t *count, uint32_t *first_code);

/* ---------------------------------------------------------------------
 * Reuse cache (reference kernels/gather_copy.cu, copy.cuh, map.cuh)
 * ------------------------------------------------------------------- */

/* Replaces gather_copy (kernels/functions.h:23-25; gather_copy.cu:47-109).
 * For block bid = b*heads+h and slot i < map_size: the 2048-byte chunk
 * position_ids[bid*map_size+i] of host region bid*cpu_v_length (bf16
 * elements) is copied to device region bid*gpu_v_length, slot i. */
SKV_API int skv_gather_copy(const void *values, void *v_cache_buffer, const int64_t *position_ids,
                    int batch_size, int heads, int cpu_v_length, int gpu_v_length, int map_size,
                    void *stream);

/* Replaces gather_copy_d2d_with_offsets (kernels/functions.h:27-35;
 * gather_copy.cu:112-185).  In-place compaction of cache hits in the K
 * buffer: slot i < cnts[bid] of region bid*gpu_k_stride + gpu_k_offset gets
 * the old slot offsets[bid*map_size+i].  gpu_k_length is accepted for
 * signature parity (it sized the reference's temp buffer). */
SKV_API int skv_gather_copy_d2d_with_offsets(void *keys, const int32_t *offsets, const int32_t *cnts,
                                     int batch_size, int heads, int gpu_k_length, int gpu_k_offset,
                                     int gpu_k_stride, int map_size, void *stream);

/* Replaces reorder_keys_and_compute_offsets (kernels/functions.h:37-42;
 * gather_copy.cu:189-235; map.cuh:475-516).  cached_pos_ids is in/out:
 * on entry the cached chunk ids (slot order), on exit the new ids reordered
 * as hits (sorted by old slot) then misses (sorted by id).  offsets: hit ->
 * old slot, miss -> chunk id.  cnts: hits per block.  map_size 1..1024. */
SKV_API int skv_reorder_keys_and_compute_offsets(int64_t *cached_pos_ids, const int64_t *cur_pos_ids,
                                         int32_t *offsets, int32_t *cnts, int batch_size,
                                         int heads, int map_size, void *stream);

/* Replaces gather_copy_with_offsets (kernels/functions.h:44-51;
 * gather_copy.cu:239-324; copy.cuh:438-498).  Slot i < cnts[bid] of region
 * bid*gpu_v_stride+gpu_v_offset gets old slot offsets[i] (in place);
 * slot i >= cnts[bid] gets host chunk offsets[i] of region
 * bid*cpu_v_length.  temp and signals are accepted for signature parity and
 * are not touched (no inter-CTA signalling is used). */
SKV_API int skv_gather_copy_with_offsets(const void *values, void *v_cache_buffer, void *temp,
                                 const int32_t *offsets, const int32_t *cnts, int32_t *signals,
                                 int batch_size, int heads, int cpu_v_length, int gpu_v_length,
                                 int gpu_v_offset, int gpu_v_stride, int map_size, void *stream);

/* ---------------------------------------------------------------------
 * RoPE (reference kernels/rope.cu, rope_new.cu)
 * All strides are in elements.  Arithmetic is bf16 op by op: each multiply
 * and add is rounded to bf16, as __hmul/__hadd in the reference.
 * ------------------------------------------------------------------- */

/* Replaces apply_rotary_pos_emb (kernels/functions.h:53-59; rope.cu:26-87):
 * separate cos and sin tables of width 2*half_dim. */
SKV_API int skv_apply_rotary_pos_emb(const void *x, const void *cos, const void *sin,
                             const int64_t *position_ids, void *output, int batch_size, int heads,
                             int seq_len, int embed_dim, int stride_xb, int stride_xh,
                             int stride_xs, int stride_xe, int stride_cos, int stride_sin,
                             int stride_pid_b, int stride_pid_h, int stride_pid_s, int half_dim,
                             void *stream);

/* Replaces apply_rotary_pos_emb_new (kernels/functions.h:61-67;
 * rope_new.cu:26-84): cos_sin row = cos[0:half] | sin[0:half], token
 * positions int64. */
SKV_API int skv_apply_rotary_pos_emb_new(const void *x, const void *cos_sin, const int64_t *position_ids,
                                 void *output, int batch_size, int heads, int seq_len,
                                 int embed_dim, int stride_xb, int stride_xh, int stride_xs,
                                 int stride_xe, int stride_cos_sin, int stride_pid_b,
                                 int stride_pid_h, int stride_pid_s, int half_dim, void *stream);

/* Replaces apply_rotary_pos_emb_new_v2 (kernels/functions.h:69-75;
 * rope_new.cu:86-144): int32 chunk ids, position = id*chunk + s%chunk. */
SKV_API int skv_apply_rotary_pos_emb_new_v2(const void *x, const void *cos_sin,
                                    const int32_t *position_ids, void *output, int batch_size,
                                    int heads, int seq_len, int embed_dim, int stride_xb,
                                    int stride_xh, int stride_xs, int stride_xe,
                                    int stride_cos_sin, int stride_pid_b, int stride_pid_h,
                                    int stride_pid_s, int half_dim, int chunk_size, void *stream);

/* Replaces apply_rotary_pos_emb_push_cache (kernels/functions.h:77-86;
 * rope_new.cu:146-222) and apply_rotary_pos_emb_push_cache_opt
 * (functions.h:88-97; rope_new.cu:224-302), which compute the same values:
 * rows s with s/chunk >= cnts[b*heads+h] and offset_output_s_start+s <
 * offset_output_s_end are rotated and written to output row
 * offset_output_s_start+s. */
SKV_API int skv_apply_rotary_pos_emb_push_cache(const void *x, const void *cos_sin,
                                        const int32_t *position_ids, void *output,
                                        const int32_t *cnts, int batch_size, int heads,
                                        int seq_len, int embed_dim, int stride_xb, int stride_xh,
                                        int stride_xs, int stride_xe, int stride_cos_sin,
                                        int stride_pid_b, int stride_pid_h, int stride_pid_s,
                                        int stride_output_b, int stride_output_h,
                                        int stride_output_s, int offset_output_s_start,
                                        int offset_output_s_end, int half_dim, int chunk_size,
                                        void *stream);
SKV_API int skv_apply_rotary_pos_emb_push_cache_opt(
    const void *x, const void *cos_sin, const int32_t *position_ids, void *output,
    const int32_t *cnts, int batch_size, int heads, int seq_len, int embed_dim, int stride_xb,
    int stride_xh, int stride_xs, int stride_xe, int stride_cos_sin, int stride_pid_b,
    int stride_pid_h, int stride_pid_s, int stride_output_b, int stride_output_h,
    int stride_output_s, int offset_output_s_start, int offset_output_s_end, int half_dim,
    int chunk_size, void *stream);

/* Replaces apply_rotary_pos_emb_push_cache_opt_glm (kernels/functions.h:
 * 99-108; rope_new.cu:305-404): GLM partial interleaved rotary on dims
 * 0..63 (pairs 2t,2t+1; cos = cs[t], sin = cs[t+32]); dims 64..127 copied. */
SKV_API int skv_apply_rotary_pos_emb_push_cache_opt_glm(
    const void *x, const void *cos_sin, const int32_t *position_ids, void *output,
    const int32_t *cnts, int batch_size, int heads, int seq_len, int embed_dim, int stride_xb,
    int stride_xh, int stride_xs, int stride_xe, int stride_cos_sin, int stride_pid_b,
    int stride_pid_h, int stride_pid_s, int stride_output_b, int stride_output_h,
    int stride_output_s, int offset_output_s_start, int offset_output_s_end, int half_dim,
    int chunk_size, void *stream);

/* ---------------------------------------------------------------------
 * Low-rank key reconstruction (reference kernels/batch_gather_gemm.cu)
 * ------------------------------------------------------------------- */

/* Replaces batch_gather_gemm (kernels/functions.h:110-116;
 * batch_gather_gemm.cu:136-213).  a = U [batch][seq_len][rank] bf16,
 * b = SV^T [batch][heads][embed_dim][rank] bf16, position_ids int32
 * [batch][heads][sparse_budget/chunk_size] chunk ids, output bf16
 * [batch][heads][sparse_budget][embed_dim].  Row r of head (b,h) with
 * r/chunk >= offset_array[b*heads+h] gets
 *   bf16( sum_k a[b][id*chunk + r%chunk][k] * b[b][h][n][k] ).
 * Rows of cache hits are not written.  cos/sin are accepted for signature
 * parity (the reference's RoPE epilogue is disabled).  embed_dim must be
 * 128, rank a multiple of 16 and <= 256, chunk_size 8. */
SKV_API int skv_batch_gather_gemm(const void *a, const void *b, const void *cos, const void *sin,
                          const int32_t *position_ids, void *output, int batch_size, int heads,
                          int seq_len, int embed_dim, int rank, int sparse_budget,
                          int max_seq_len, int chunk_size, const int32_t *offset_array,
                          void *stream);

/* ---------------------------------------------------------------------
 * Landmark scoring (reference kernels/batch_gemm_softmax.cu)
 * ------------------------------------------------------------------- */

/* Replaces batch_gemm_softmax (kernels/functions.h:118-121;
 * batch_gemm_softmax.cu:143-196).  A [batch][m][k] bf16, B [batch][n][k]
 * bf16 (the column-major k x n operand), D and Softmax [batch][m][n] bf16,
 * Norm and Sum [batch][ceil(n/256)][m] fp32.  D = bf16(alpha*A.B^T);
 * Norm/Sum hold per-256-column partial max / sum-exp of the fp32 values and
 * block 0 is overwritten with the row max and 1/row-sum;
 * Softmax = bf16(exp(float(D) - max) * (1/sum)).  beta is ignored (the
 * reference passes no C operand).  k must be 128, m <= 64. */
SKV_API int skv_batch_gemm_softmax(const void *A, const void *B, void *D, float *Norm, float *Sum,
                           void *Softmax, int batch_count, int m, int n, int k, float alpha,
                           float beta, void *stream);

/* ---------------------------------------------------------------------
 * Fused decode path (this library)
 * ------------------------------------------------------------------- */

/* Geometry of one layer of the decode state. */
typedef struct {
    int batch;          /* sequences */
    int kv_heads;       /* key/value heads */
    int q_heads;        /* query heads (multiple of kv_heads, group <= 16) */
    int head_dim;       /* must be 128 */
    int rank;           /* low-rank width of U / SV (multiple of 16, <= 256) */
    int chunk_size;     /* tokens per chunk, must be 8 */
    int select_sets;    /* chunks selected per head (budget / chunk_size), <= 1024 */
    int num_landmarks;  /* landmarks per head */
    int num_chunks;     /* chunk ids are in [0, num_chunks) */
    int ctx_len;        /* rows of U per sequence */
    int buf_len;        /* rows of each K/V buffer per head */
    int sparse_start;   /* first buffer row of the selected chunks */
    int rope_mode;      /* 0: rotate-half (cos_sin width 128), 1: GLM (width 64) */
    int cos_sin_stride; /* elements per cos_sin row */
    int cos_sin_rows;   /* rows of the cos_sin table */
    float scale;        /* softmax scale for scoring and attention, usually 1/sqrt(128) */
} skv_decode_geom;

/* New-token step (replaces the vllm rotary_embedding call of
 * models/attention/shadow.py:26 / models/llama.py:149-154 and
 * ShadowKVCache_CPU.update_kv_cache, models/kvcache/shadow.py:621-633):
 * q [batch][q_heads][128] and k_new, v_new [batch][kv][128] bf16 of the
 * generated token, positions [batch] int64.  Writes RoPE(q) to q_out, RoPE(k)
 * to k_buf row `row` and v to v_buf row `row` of every head.  bf16 op-by-op
 * RoPE arithmetic; rope_mode / cos_sin as in the geometry. */
SKV_API int skv_decode_append(const skv_decode_geom *g, const void *q, const void *k_new,
                              const void *v_new, const int64_t *positions, const void *cos_sin,
                              void *q_out, void *k_buf, void *v_buf, int row, void *stream);

/* Bytes of caller-provided scratch the selection needs. */
SKV_API size_t skv_decode_select_workspace(const skv_decode_geom *g);

/* Kernels one skv_decode_select / skv_decode_append_select launches: 2
 * (scoring, selection), or 3 for more than 32768 landmarks per head, where a
 * keys kernel between them computes the selection keys on the whole GPU
 * (0 for a rejected geometry). */
SKV_API int skv_decode_select_kernels(const skv_decode_geom *g);

/* Landmark scoring + top-k + slot-stable reuse-cache diff for one layer.
 * q [batch][q_heads][128] bf16 (post-RoPE), landmarks [batch][kv][L][128]
 * bf16, landmark_idx [batch][kv][L] int64 chunk ids, slots
 * [batch][kv][select_sets] int32 in/out: slot s holds the chunk id cached
 * in buffer rows sparse_start + 8s .. +8.  Hits keep their slot; the slots
 * of chunks that dropped out are refilled (ascending slot) with the missed
 * ids (ascending id).  miss_slot/miss_chunk [batch][kv][select_sets] int32
 * and miss_count [batch][kv] int32 list the refilled slots. */
SKV_API int skv_decode_select(const skv_decode_geom *g, const void *q, const void *landmarks,
                      const int64_t *landmark_idx, int32_t *slots, int32_t *miss_slot,
                      int32_t *miss_chunk, int32_t *miss_count, void *workspace,
                      size_t workspace_bytes, void *stream);

/* skv_decode_append followed by skv_decode_select in one scoring pass: the
 * scoring kernel rotates the query rows of each GQA group itself and its
 * first split per head writes q_out and the new key/value rows.  q is the
 * pre-RoPE query; the selection uses the rotated query.  Same results as
 * the two calls in sequence. */
SKV_API int skv_decode_append_select(const skv_decode_geom *g, const void *q, const void *k_new,
                                     const void *v_new, const int64_t *positions,
                                     const void *cos_sin, void *q_out, void *k_buf, void *v_buf,
                                     int row, const void *landmarks, const int64_t *landmark_idx,
                                     int32_t *slots, int32_t *miss_slot, int32_t *miss_chunk,
                                     int32_t *miss_count, void *workspace, size_t workspace_bytes,
                                     void *stream);

/* Allocation-free skv_decode_select (no counterpart in the reference).
 * For callers that cannot provide a scratch buffer: an FFI host that owns no
 * CUDA allocator (it only receives the model-state tensors), or a runtime that
 * plans all device memory at start-up and forbids allocation on the token
 * path.  The scratch is a fixed 32 MiB array in the library's device memory,
 * held on every GPU that loads the library until exit; geometries needing
 * more (skv_decode_select_workspace) are rejected with SKV_ERR_UNSUPPORTED.
 * All calls on a device share the array: calls that overlap on the GPU race.
 * Nothing in it needs clearing (each call writes what it reads).  The first
 * call on a device looks up the array's address; make it before any stream
 * capture.  Same outputs as skv_decode_select. */
SKV_API int skv_decode_select_noalloc(const skv_decode_geom *g, const void *q, const void *landmarks,
                                      const int64_t *landmark_idx, int32_t *slots,
                                      int32_t *miss_slot, int32_t *miss_chunk,
                                      int32_t *miss_count, void *stream);

/* Zero-copy fetch of the missed value chunks from page-locked host memory:
 * v_host [batch][kv][num_chunks][8*128] bf16 -> v_buf rows
 * sparse_start + 8*slot of [batch][kv][buf_len][128]. */
SKV_API int skv_decode_gather_values(const skv_decode_geom *g, const void *v_host, void *v_buf,
                             const int32_t *miss_slot, const int32_t *miss_chunk,
                             const int32_t *miss_count, void *stream);

/* Reconstruction of the missed keys: U [batch][ctx_len][rank] bf16 times
 * SV^T [batch][kv][128][rank] bf16 on tensor cores with fp32 accumulation,
 * RoPE at the original positions (rope_mode, cos_sin) applied to the fp32
 * accumulator, one rounding to bf16, written to k_buf rows
 * sparse_start + 8*slot.  (The reference's two-kernel path rounds the GEMM
 * output and every RoPE term to bf16; skv_batch_gather_gemm +
 * skv_apply_rotary_pos_emb_push_cache_opt keep that arithmetic.) */
SKV_API int skv_decode_reconstruct_keys(const skv_decode_geom *g, const void *U, const void *SVt,
                                const void *cos_sin, void *k_buf, const int32_t *miss_slot,
                                const int32_t *miss_chunk, const int32_t *miss_count,
                                void *stream);

/* Bytes of caller-provided scratch the attention needs for seq_len rows.
 * Returns 0: the split partials are merged through distributed shared memory
 * inside one thread-block cluster per head (the function is kept so callers
 * can size a workspace generically). */
SKV_API size_t skv_decode_attention_workspace(const skv_decode_geom *g, int seq_len);

/* Split-K GQA decode attention over buffer rows [0, seq_len):
 * q [batch][q_heads][128] bf16, k_buf/v_buf [batch][kv][buf_len][128] bf16
 * -> out [batch][q_heads][128] bf16.  One 8-CTA cluster per (b, kv head);
 * workspace may be NULL. */
SKV_API int skv_decode_attention(const skv_decode_geom *g, const void *q, const void *k_buf,
                         const void *v_buf, int seq_len, void *out, void *workspace,
                         size_t workspace_bytes, void *stream);

/* Bytes of caller-provided scratch skv_decode_sparse_attention needs for
 * seq_len rows: per-CTA partials plus one ticket per (b, kv head).  The
 * scratch must be zero-filled before its first use (the kernel leaves the
 * tickets at zero when it completes); it must not be shared by launches that
 * can run at the same time. */
SKV_API size_t skv_decode_sparse_attention_workspace(const skv_decode_geom *g, int seq_len);

/* One launch for value fetch + key reconstruction + attention of a decode
 * step, after skv_decode_select / skv_decode_append_select:
 *   - the missed chunks of the miss lists are fetched from page-locked
 *     v_host into v_buf (as skv_decode_gather_values),
 *   - their keys are reconstructed from U and SV^T with RoPE into k_buf (as
 *     skv_decode_reconstruct_keys),
 *   - out = GQA attention of q over buffer rows [0, seq_len) (as
 *     skv_decode_attention; per-CTA partials merged by the last CTA).
 * seq_len must cover the selected rows (>= sparse_start + 8*select_sets).
 * out may be device memory or page-locked host memory: the last CTA of each
 * head then writes its rows over the host link, with no separate
 * device-to-host copy after the launch.
 * No counterpart in the reference, which runs these as separate kernels
 * (kernels/gather_copy.cu, kernels/batch_gather_gemm.cu + kernels/rope_new.cu,
 * flash_attn_with_kvcache in models/attention/shadow.py:48). */
SKV_API int skv_decode_sparse_attention(const skv_decode_geom *g, const void *q, const void *U,
                                        const void *SVt, const void *cos_sin, const void *v_host,
                                        void *k_buf, void *v_buf, const int32_t *miss_slot,
                                        const int32_t *miss_chunk, const int32_t *miss_count,
                                        int seq_len, void *out, void *workspace,
                                        size_t workspace_bytes, void *stream);

/* Bytes of scratch skv_decode_step needs for any seq_len up to buf_len (0 if
 * the geometry or head_groups is rejected).  Zero-fill it before its first
 * use; calls leave it ready for the next call; launches that can run at the
 * same time must not share it. */
SKV_API size_t skv_decode_step_workspace(const skv_decode_geom *g, int head_groups);

/* One decode step of one layer: skv_decode_append_select (new token's RoPE +
 * append at buffer row `row`, scoring, top-k, reuse diff) followed by
 * skv_decode_sparse_attention (value fetch, key reconstruction, attention),
 * with the same results.  The selection's miss lists live in the workspace;
 * miss_count, if not null, receives the number of missed chunks of every
 * (sequence, kv head) [batch * kv_heads] int32 (the reference's cnts are the
 * hits: select_sets - miss_count).
 * head_groups > 1 (batch 1, dividing kv_heads, at most 8) pipelines the step
 * over groups of kv heads: each group's chain runs on a library stream, the
 * groups' scoring passes one after the other, so the first group's value
 * fetch starts after a fraction of the landmark scan and the other groups'
 * scoring and selection overlap it.  The fork and join are event waits on
 * `stream`, so stream capture records the whole step.  The library streams
 * and events of a device are created by its first call with head_groups > 1:
 * make that call outside stream capture.
 * q, k_new, v_new and positions may lie in device memory or in page-locked
 * host memory mapped for the device (8-byte aligned): inputs in host memory
 * are read over the host link into the workspace by a small staging kernel
 * at the head of each kv-head group's chain (the step then needs no separate
 * host-to-device copy of its inputs).
 * row_dev (optional, device int32): the append row read on the device at run
 * time -- the attention then covers rows [0, *row_dev + 1) -- so a captured
 * step can be replayed at later positions (advance *row_dev between
 * replays); `row` and `seq_len` are then the largest row and row count the
 * position may reach (they size the launches).  A position outside them is
 * counted in skv_device_errors (code 3) and the launch's own values are used.
 * Early fetch (off by default, skv_decode_step_early_fetch): where the selection's shared memory allows it
 * (8-CTA selection clusters: at most 32768 landmarks per head), the
 * selection kernel itself requests the value chunks of the misses that are
 * certain once its score histogram has located the k-th score, before the
 * selection is complete, reconstructs the missed keys and stores keys and
 * values into their slots; the attention kernel then reads every selected row
 * from the buffers.  The state (buffers, slots, miss lists) is the same bits
 * as without it; the output differs only in fp32 summation order (the rows
 * are split into partials differently).
 * Replaces, per step, shadowkv.batch_gemm_softmax + torch.topk +
 * reorder_keys_and_compute_offsets + gather_copy_with_offsets +
 * gather_copy_d2d_with_offsets + batch_gather_gemm + the push-cache RoPE and
 * flash_attn_with_kvcache (models/kvcache/shadow.py:547-633,
 * models/attention/shadow.py:22-48). */
SKV_API int skv_decode_step(const skv_decode_geom *g, const void *q, const void *k_new, const void *v_new,
                            const int64_t *positions, const void *cos_sin, void *q_out, void *k_buf,
                            void *v_buf, int row, const int32_t *row_dev, const void *landmarks,
                            const int64_t *landmark_idx,
                            int32_t *slots, const void *U, const void *SVt, const void *v_host,
                            int seq_len, void *out, int32_t *miss_count, int head_groups,
                            void *workspace, size_t workspace_bytes, void *stream);

/* Turn the early fetch of skv_decode_step on (enable != 0) or off (the
 * default) for the whole process; returns the previous setting.  Calls enqueued
 * afterwards use the new setting (a captured graph keeps the path it was
 * captured with).  For comparisons and diagnosis: both paths leave the same
 * state, and outputs equal up to fp32 summation order. */
SKV_API int skv_decode_step_early_fetch(int enable);

/* Kernel timing of skv_decode_step, off by default, for the whole process;
 * returns the previous setting.  The kernels of a step enqueued with it on
 * (scoring, selection and attention of each kv-head group) stamp the GPU's
 * global timer: thread 0 of every CTA at its start, after its wait for the
 * kernel before it, and at its end, into a (earliest start, latest end) pair
 * per kernel kept on the device.  The launches are those of an untimed step;
 * a graph captured from a timed step stamps on every replay.  Results are
 * unchanged. */
SKV_API int skv_decode_step_timing(int enable);

/* The spans of the last timed step (or replay of a graph captured from one)
 * on the current device: waits for the device, then for groups
 * i < min(*groups, max_groups) and kernels k (0 scoring, 1 selection,
 * 2 attention) us[6 i + 2 k] = start, us[6 i + 2 k + 1] = end, in microseconds
 * after the earliest start of any kernel of the step; -1 for a kernel that
 * did not run (the attention of an early-fetch step runs in its selection
 * kernel).  Clears the spans for the next step.  *groups = the step's head
 * groups.  Returns an error if no step was enqueued with timing on, or if
 * none of its kernels has run since the last read. */
SKV_API int skv_decode_step_kernel_times(double *us, int max_groups, int *groups);

/* ---- prefill state builder (ShadowKVCache_CPU.prefill_kv_cache,
 * models/kvcache/shadow.py:463-544) for one layer of `batch` sequences. */
typedef struct {
    int batch, kv_heads, q_heads;
    int tokens;         /* prompt length T */
    int chunks;         /* landmark candidates per head: T/8 - local_chunk (rounded down
                           to a multiple of 8 for the CPU-class geometry); the last
                           T - 8*chunks tokens are the local window */
    int outlier_chunk;  /* chunks of lowest key similarity kept in the buffer (<= 256) */
    int select_sets;    /* chunks of the first selection */
    int buf_len;        /* rows of each K/V buffer per head */
    int host_chunks;    /* chunk slots per head of the host value store (>= T/8) */
} skv_prefill_geom;

SKV_API size_t skv_prefill_workspace(const skv_prefill_geom *p);

/* The prompt's values v [batch][kv][T][128] bf16 into the page-locked host
 * store v_host [batch][kv][host_chunks][8*128], chunks 0 .. T/8-1 (one
 * strided device-to-host copy; give it a stream of its own to overlap
 * skv_prefill_build). */
SKV_API int skv_prefill_store_values(const skv_prefill_geom *p, const void *v, void *v_host, void *stream);

/* k_roped, v [batch][kv][T][128] bf16 (post-RoPE keys, values), q_last
 * [batch][q_heads][128] bf16 (post-RoPE last prompt query).  Writes
 *   k_buf, v_buf [batch][kv][buf_len][128] rows 0 .. sparse_end-1: local
 *     window, the outlier chunks (ascending minimum similarity, ties to the
 *     lower chunk id), the selected chunks in slot order;
 *   landmarks [batch][kv][chunks-outlier_chunk][128] bf16 and landmark_idx
 *     (int64): means of the non-outlier chunks in chunk order;
 *   slots (int32) and position_ids (int64) [batch][kv][select_sets]: the
 *     first selection (scores of q_last against the landmarks; ascending
 *     chunk id in slot order).
 * Mean and cosine similarity are computed op by op in bf16 like the torch
 * ops they replace; the selection uses fp32 scores (the reference rounds
 * them to bf16 and leaves ties to torch.topk). */
SKV_API int skv_prefill_build(const skv_prefill_geom *p, const void *k_roped, const void *v, const void *q_last,
                              void *k_buf, void *v_buf, void *landmarks, int64_t *landmark_idx, int32_t *slots,
                              int64_t *position_ids, void *workspace, size_t workspace_bytes, void *stream);

/* skv_decode_sparse_attention on at most max_ctas CTAs (one per SM), each
 * taking (kv head, 128-row block) work items in strides.  With many sequences
 * the host link stays saturated by far fewer SMs than the GPU has; the SMs
 * left free run the next batch slice's scoring and selection meanwhile (on
 * another, higher-priority stream). */
SKV_API int skv_decode_sparse_attention_ctas(const skv_decode_geom *g, const void *q, const void *U,
                                             const void *SVt, const void *cos_sin, const void *v_host,
                                             void *k_buf, void *v_buf, const int32_t *miss_slot,
                                             const int32_t *miss_chunk, const int32_t *miss_count,
                                             int seq_len, void *out, int max_ctas, void *workspace,
                                             size_t workspace_bytes, void *stream);

/* ---- rank-r factorisation of the prompt's keys (ShadowKVCache_CPU.get_svd,
 * models/kvcache/shadow.py:411-444: torch.svd of K [T, H*128], leading
 * `rank` triplets).  The library forms the Gram matrix K^T K on the tensor
 * cores; its leading eigenvectors are K's right singular vectors (the
 * eigensolve of the D x D matrix and U = K V / s are left to the caller). */

/* Bytes of scratch skv_gram needs for `tokens` rows of `dim` columns (0 if
 * dim is not a multiple of 128 in 128..8192). */
SKV_API size_t skv_gram_workspace(int tokens, int dim);

/* gram [dim][dim] float64 = K^T K for K [tokens][ld] bf16 (the first `dim`
 * columns of each row; ld >= dim, a multiple of 8).  bf16 products with fp32
 * accumulation over slices of the rows, the slices summed in float64. */
SKV_API int skv_gram(const void *k, int tokens, int dim, int ld, double *gram, void *workspace,
                     size_t workspace_bytes, void *stream);

/* ---- attention output gathered over peer memory (kv heads split over ranks)
 *
 * With the kv heads of a sequence split over `world` GPUs (one process per
 * GPU), o_proj needs every rank's attention rows.  The reference would
 * all-gather them after the attention (NCCL, one collective per layer);
 * here the attention kernel's merge writes its rows straight into every
 * rank's landing buffer over NVLink and bumps every rank's arrival counter,
 * and skv_peer_gather_finish waits for the counter and copies the full
 * output out of the landing buffer.  Each rank owns one peer block
 * (skv_peer_block_bytes): [arrival counter | status | epoch | landing buffer
 * [2][batch][q_heads_total][128] bf16]; the landing half used by a step is
 * epoch & 1, so a rank one step ahead never writes the half a slower rank
 * still reads.  Blocks are shared through CUDA IPC handles (64 bytes).
 * A finish whose wait runs out sets the block's status (sticky) and neither
 * copies nor advances the epoch; every later finish on that block does
 * nothing.  Read it with skv_peer_status; after a non-zero status every rank
 * must re-create its peer blocks (the step counts of the ranks disagree). */
#define SKV_MAX_PEERS 8
typedef struct {
    int world;            /* ranks sharing the output, 1..SKV_MAX_PEERS */
    int rank;             /* this rank */
    int q_head0;          /* first query head of this rank in the full output */
    int q_heads_total;    /* query heads of the full output */
    int merges_per_step;  /* (sequence, kv head) units of one step summed over all ranks:
                             batch * q_heads_total / (q heads per kv head) */
    int batch;            /* sequences of a step: the landing buffers hold this many */
    void *block[SKV_MAX_PEERS];  /* every rank's peer block, as addressed from this GPU */
} skv_peer_gather;

SKV_API size_t skv_peer_block_bytes(int batch, int q_heads_total);
/* cudaMalloc'd, zero-filled block of `bytes`. */
SKV_API int skv_peer_alloc(size_t bytes, void **block);
SKV_API int skv_peer_free(void *block);
/* CUDA IPC handle (64 bytes) of a block, and its mapping in another process
 * (peer access enabled on first use); skv_peer_close unmaps it. */
SKV_API int skv_peer_export(const void *block, void *handle64);
SKV_API int skv_peer_import(const void *handle64, void **block);
SKV_API int skv_peer_close(void *block);

/* skv_decode_sparse_attention with the output written to every rank's
 * landing buffer (rows q_head0 .. q_head0 + q_heads of the full output).
 * g->batch must equal pg->batch and pg->merges_per_step must equal
 * g->batch * pg->q_heads_total / (g->q_heads / g->kv_heads). */
SKV_API int skv_decode_sparse_attention_gather(const skv_decode_geom *g, const void *q, const void *U,
                                               const void *SVt, const void *cos_sin, const void *v_host,
                                               void *k_buf, void *v_buf, const int32_t *miss_slot,
                                               const int32_t *miss_chunk, const int32_t *miss_count,
                                               int seq_len, const skv_peer_gather *pg, void *workspace,
                                               size_t workspace_bytes, void *stream);

/* Waits (bounded, about one second) until every rank's rows of this step
 * have arrived, copies the full output [batch][q_heads_total][128] into `out`
 * (device memory) and advances the epoch.  A wait that runs out sets the
 * block's status to 4 (also counted in skv_device_errors) and copies nothing.
 * batch must equal pg->batch.  One call per step, after
 * skv_decode_sparse_attention_gather, on the same stream. */
SKV_API int skv_peer_gather_finish(const skv_peer_gather *pg, int batch, void *out, void *stream);

/* The status word of this rank's peer block (0: fine; 4: a finish timed out).
 * Synchronous: waits for the work of the current device (a device-to-host
 * copy of 4 bytes); call it between steps. */
SKV_API int skv_peer_status(const skv_peer_gather *pg, uint32_t *status);

#ifdef __cplusplus
}
#endif

#endif /* SHADOWKV_B200_H */
