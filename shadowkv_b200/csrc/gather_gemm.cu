// Entry points of the gathered low-rank key reconstruction: the drop-in
// batch_gather_gemm binding and the fused path's reconstruct_keys.
//
// Reference: kernels/batch_gather_gemm.cu:136-213 (CUTLASS 2.x gather GEMM,
// 128x128x32 tiles, tiles of cache hits skipped) and the RoPE push-cache
// kernels kernels/rope_new.cu:224-374 (applied as a second pass there).
// Both run gather_gemm_tc_kernel (gather_gemm_tc.cu): tcgen05 tensor-core
// MMAs with the accumulator in tensor memory.
#include "gather_gemm.cuh"

namespace skv {

int launch_gather_gemm(const GatherGemmArgs &a, int rope, int nbh, cudaStream_t stream)
{
    return launch_gather_gemm_tc(a, rope, nbh, stream);
}

}  // namespace skv

using namespace skv;

extern "C" {

int skv_batch_gather_gemm(const void *a, const void *b, const void *cos, const void *sin,
                          const int32_t *position_ids, void *output, int batch_size, int heads,
                          int seq_len, int embed_dim, int rank, int sparse_budget,
                          int max_seq_len, int chunk_size, const int32_t *offset_array,
                          void *stream)
{
    (void)cos;
    (void)sin;
    (void)max_seq_len;
    SKV_CHECK_ARG(a && b && position_ids && output && offset_array, "null pointer argument");
    SKV_CHECK_ARG(batch_size > 0 && heads > 0 && seq_len > 0, "sizes must be positive");
    SKV_CHECK_SUPPORTED(embed_dim == 128, "embed_dim must be 128");
    SKV_CHECK_SUPPORTED(chunk_size == 8, "chunk_size must be 8");
    SKV_CHECK_SUPPORTED(rank % 16 == 0 && rank >= 16 && rank <= 256, "rank must be a multiple of 16 in 16..256");
    SKV_CHECK_ARG(sparse_budget > 0 && sparse_budget % chunk_size == 0, "sparse_budget must be a multiple of chunk_size");
    SKV_CHECK_ARG(aligned(a, 16) && aligned(b, 16) && aligned(output, 16), "operands must be 16-byte aligned");
    GatherGemmArgs g = {};
    g.U = (const __nv_bfloat16 *)a;
    g.SVt = (const __nv_bfloat16 *)b;
    g.out = (__nv_bfloat16 *)output;
    g.ids = position_ids;
    g.slots = nullptr;
    g.lo = offset_array;
    g.hi = nullptr;
    g.H = heads;
    g.M = sparse_budget / chunk_size;
    g.rank = rank;
    g.ctx = seq_len;
    g.out_bh_stride = (int64_t)sparse_budget * 128;
    g.out_row0 = 0;
    return launch_gather_gemm(g, 0, batch_size * heads, (cudaStream_t)stream);
}

int skv_decode_reconstruct_keys(const skv_decode_geom *gm, const void *U, const void *SVt,
                                const void *cos_sin, void *k_buf, const int32_t *miss_slot,
                                const int32_t *miss_chunk, const int32_t *miss_count,
                                void *stream)
{
    SKV_CHECK_ARG(gm && U && SVt && cos_sin && k_buf && miss_slot && miss_chunk && miss_count,
                  "null pointer argument");
    SKV_CHECK_SUPPORTED(gm->head_dim == 128 && gm->chunk_size == 8, "head_dim 128 and chunk 8 only");
    SKV_CHECK_SUPPORTED(gm->rank % 16 == 0 && gm->rank >= 16 && gm->rank <= 256,
                        "rank must be a multiple of 16 in 16..256");
    SKV_CHECK_SUPPORTED(gm->rope_mode == 0 || gm->rope_mode == 1, "rope_mode must be 0 or 1");
    SKV_CHECK_ARG(gm->cos_sin_stride >= (gm->rope_mode == 0 ? 128 : 64), "cos_sin_stride too small");
    SKV_CHECK_ARG(gm->sparse_start >= 0 && gm->sparse_start + 8 * (int64_t)gm->select_sets <= gm->buf_len,
                  "selected rows exceed buf_len");
    SKV_CHECK_ARG(aligned(U, 16) && aligned(SVt, 16) && aligned(k_buf, 16) && aligned(cos_sin, 16) &&
                      gm->cos_sin_stride % 8 == 0,
                  "operands and cos/sin rows must be 16-byte aligned");
    GatherGemmArgs g = {};
    g.U = (const __nv_bfloat16 *)U;
    g.SVt = (const __nv_bfloat16 *)SVt;
    g.cos_sin = (const __nv_bfloat16 *)cos_sin;
    g.out = (__nv_bfloat16 *)k_buf;
    g.ids = miss_chunk;
    g.slots = miss_slot;
    g.lo = nullptr;
    g.hi = miss_count;
    g.H = gm->kv_heads;
    g.M = gm->select_sets;
    g.rank = gm->rank;
    g.ctx = gm->ctx_len;
    g.out_bh_stride = (int64_t)gm->buf_len * 128;
    g.out_row0 = gm->sparse_start;
    g.cs_stride = gm->cos_sin_stride;
    g.cs_rows = gm->cos_sin_rows;
    return launch_gather_gemm(g, gm->rope_mode == 0 ? 1 : 2, gm->batch * gm->kv_heads,
                              (cudaStream_t)stream);
}

}  // extern "C"
