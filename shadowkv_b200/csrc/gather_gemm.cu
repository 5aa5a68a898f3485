// Gathered low-rank key reconstruction: rows of U selected by chunk id times
// the per-head SV^T, bf16 in / fp32 accumulate / bf16 out, with an optional
// RoPE epilogue at the original token positions.
//
// Reference: kernels/batch_gather_gemm.cu:136-213 (CUTLASS 2.x gather GEMM,
// 128x128x32 tiles, tiles of cache hits skipped) and the RoPE push-cache
// kernels kernels/rope_new.cu:224-374 (applied as a second pass there).
//
// One CTA computes 8 chunks (64 rows) x 128 output dims over the full rank.
// U rows of one chunk are one contiguous 8*rank*2-byte run, staged with
// cp.async; SV^T of the head is staged once per CTA.  The epilogue applies
// RoPE to the fp32 accumulators in registers (the (t, t+64) pair of a row
// lives in the same thread of the mma accumulator layout), rounds once to
// bf16, stages the tile in shared memory and writes 256-byte rows.
#include "common.cuh"

namespace skv {

constexpr int GG_CHUNKS = 8;           // chunks per CTA
constexpr int GG_ROWS = GG_CHUNKS * 8; // 64 rows
constexpr int GG_N = 128;              // head_dim
constexpr int GG_THREADS = 128;        // 4 warps x 16 rows

struct GatherGemmArgs {
    const __nv_bfloat16 *U;     // [B][ctx][rank]
    const __nv_bfloat16 *SVt;   // [B][H][128][rank]
    const __nv_bfloat16 *cos_sin;
    __nv_bfloat16 *out;
    const int32_t *ids;         // [B*H][M] chunk ids (entry j)
    const int32_t *slots;       // [B*H][M] destination slot of entry j (fused) or null
    const int32_t *lo;          // per-(b,h) first valid entry (drop-in: cnts) or null
    const int32_t *hi;          // per-(b,h) end of valid entries (fused: miss_count) or null
    int H, M, rank, ctx;
    int64_t out_bh_stride;      // elements between (b,h) blocks of out
    int out_row0;               // first destination row (sparse_start) in the fused path
    int cs_stride, cs_rows;
};

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem)
{
    uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_wait_all()
{
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void ldmatrix_x4(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3,
                                            const void *p)
{
    uint32_t s = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(s));
}

// ROPE: 0 none, 1 rotate-half (cos_sin width 128), 2 GLM interleaved (width 64)
template <int ROPE>
__global__ void __launch_bounds__(GG_THREADS) gather_gemm_kernel(GatherGemmArgs a)
{
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int bh = blockIdx.y;
    const int b = bh / a.H;
    const int j0 = blockIdx.x * GG_CHUNKS;
    const int lo = a.lo ? a.lo[bh] : 0;
    const int hi = a.hi ? a.hi[bh] : a.M;
    if (j0 + GG_CHUNKS <= lo || j0 >= hi) return;

    const int KP = a.rank + 8;  // padded row pitch (elements), conflict-free ldmatrix
    __nv_bfloat16 *sA = reinterpret_cast<__nv_bfloat16 *>(smem_raw);
    __nv_bfloat16 *sB = sA + GG_ROWS * KP;
    __shared__ int s_chunk[GG_CHUNKS];
    __shared__ int s_dst[GG_CHUNKS];

    if (threadIdx.x < GG_CHUNKS) {
        const int j = j0 + threadIdx.x;
        int c = -1, d = -1;
        if (j >= lo && j < hi && j < a.M) {
            c = a.ids[(int64_t)bh * a.M + j];
            const int slot = a.slots ? a.slots[(int64_t)bh * a.M + j] : j;
            if (c < 0 || (int64_t)c * 8 + 8 > a.ctx) {
                report_dev_error(DEV_ERR_ROW);
                c = -1;
            } else if (slot < 0 || slot >= a.M) {
                report_dev_error(DEV_ERR_SLOT);
                c = -1;
            } else {
                d = slot;
            }
        }
        s_chunk[threadIdx.x] = c;
        s_dst[threadIdx.x] = d;
    }
    __syncthreads();

    // ---- stage A (gathered U rows) and B (SV^T of the head) ----
    const int ppr = a.rank / 8;  // 16-byte pieces per row
    {
        const __nv_bfloat16 *Ub = a.U + (int64_t)b * a.ctx * a.rank;
        for (int p = threadIdx.x; p < GG_ROWS * ppr; p += GG_THREADS) {
            const int r = p / ppr, q = p % ppr;
            const int c = s_chunk[r >> 3];
            if (c >= 0)
                cp_async16(sA + r * KP + q * 8, Ub + ((int64_t)c * 8 + (r & 7)) * a.rank + q * 8);
        }
        const __nv_bfloat16 *Bb = a.SVt + (int64_t)bh * GG_N * a.rank;
        for (int p = threadIdx.x; p < GG_N * ppr; p += GG_THREADS) {
            const int r = p / ppr, q = p % ppr;
            cp_async16(sB + r * KP + q * 8, Bb + (int64_t)r * a.rank + q * 8);
        }
        cp_async_wait_all();
        __syncthreads();
    }

    // ---- tensor-core main loop ----
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float acc[16][4];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;

    const __nv_bfloat16 *aRow = sA + (warp * 16 + (lane & 15)) * KP + (lane >> 4) * 8;
    const int bRowOff = (lane & 7) + ((lane >> 4) << 3);
    const int bColOff = ((lane >> 3) & 1) * 8;
    for (int k0 = 0; k0 < a.rank; k0 += 16) {
        uint32_t a0, a1, a2, a3;
        ldmatrix_x4(a0, a1, a2, a3, aRow + k0);
#pragma unroll
        for (int np = 0; np < 8; ++np) {
            uint32_t b0, b1, b2, b3;
            ldmatrix_x4(b0, b1, b2, b3, sB + (np * 16 + bRowOff) * KP + k0 + bColOff);
            mma_bf16_16816(acc[2 * np], a0, a1, a2, a3, b0, b1);
            mma_bf16_16816(acc[2 * np + 1], a0, a1, a2, a3, b2, b3);
        }
    }

    // ---- epilogue: bf16 rounding, RoPE, staged 256-byte row stores ----
    const int g = lane >> 2, t4 = lane & 3;
    __syncthreads();  // sA is reused as the output staging tile
    const int OP = GG_N + 8;
    __nv_bfloat16 *sO = sA;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const int r = warp * 16 + g + half * 8;  // row in the CTA tile
        const int e = r >> 3;                    // chunk entry
        const int c = s_chunk[e];
        const int64_t pos = (int64_t)(c < 0 ? 0 : c) * 8 + (r & 7);
        // Without RoPE the product is rounded to bf16 (batch_gather_gemm output).
        // With RoPE the rotation is applied to the fp32 accumulator and the
        // result is rounded once: the fused path does not round the GEMM
        // output and each RoPE term to bf16 as the two-kernel reference does.
        float v[16][2];
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
            v[nt][0] = acc[nt][half * 2 + 0];
            v[nt][1] = acc[nt][half * 2 + 1];
        }
        if (ROPE != 0 && c >= 0) {
            if (pos >= a.cs_rows) {
                if (t4 == 0) report_dev_error(DEV_ERR_ROW);
            } else {
                const __nv_bfloat16 *cs = a.cos_sin + pos * a.cs_stride;
                if (ROPE == 1) {
#pragma unroll
                    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            const int t = nt * 8 + t4 * 2 + u;
                            const float cc = bf2f(cs[t]), ss = bf2f(cs[t + 64]);
                            const float x1 = v[nt][u], x2 = v[nt + 8][u];
                            v[nt][u] = x1 * cc - x2 * ss;
                            v[nt + 8][u] = x2 * cc + x1 * ss;
                        }
                    }
                } else {
#pragma unroll
                    for (int nt = 0; nt < 8; ++nt) {
                        const int tp = (nt * 8 + t4 * 2) >> 1;  // pair index < 32
                        const float cc = bf2f(cs[tp]), ss = bf2f(cs[tp + 32]);
                        const float xe = v[nt][0], xo = v[nt][1];
                        v[nt][0] = xe * cc - xo * ss;
                        v[nt][1] = xo * cc + xe * ss;
                    }
                }
            }
        }
#pragma unroll
        for (int nt = 0; nt < 16; ++nt)
            *reinterpret_cast<uint32_t *>(sO + r * OP + nt * 8 + t4 * 2) = pack_bf2(v[nt][0], v[nt][1]);
    }
    __syncwarp();
    // each warp writes its own 16 rows: 16 rows x 16 pieces of 16 bytes
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int p = lane + 32 * i;
        const int r = warp * 16 + (p >> 4);
        const int q = p & 15;
        const int e = r >> 3;
        const int d = s_dst[e];
        if (d < 0) continue;
        const int64_t row = (int64_t)a.out_row0 + (int64_t)d * 8 + (r & 7);
        const uint4 val = *reinterpret_cast<const uint4 *>(sO + r * OP + q * 8);
        st_v4(a.out + (int64_t)bh * a.out_bh_stride + row * GG_N + q * 8, val);
    }
}

static size_t gg_smem_bytes(int rank)
{
    const size_t operands = (size_t)(GG_ROWS + GG_N) * (rank + 8) * 2;
    const size_t staging = (size_t)GG_ROWS * (GG_N + 8) * 2;  // epilogue tile reuses the operand space
    return operands > staging ? operands : staging;
}

int launch_gather_gemm(const GatherGemmArgs &a, int rope, int nbh, cudaStream_t stream)
{
    const int smem = (int)gg_smem_bytes(a.rank);
    dim3 grid(ceil_div(a.M, GG_CHUNKS), nbh);
    const void *fn = rope == 0 ? (const void *)gather_gemm_kernel<0>
                   : rope == 1 ? (const void *)gather_gemm_kernel<1> : (const void *)gather_gemm_kernel<2>;
    int st = ensure_smem_attr(fn, smem, "gather_gemm_kernel");
    if (st) return st;
    if (rope == 0) gather_gemm_kernel<0><<<grid, GG_THREADS, smem, stream>>>(a);
    else if (rope == 1) gather_gemm_kernel<1><<<grid, GG_THREADS, smem, stream>>>(a);
    else gather_gemm_kernel<2><<<grid, GG_THREADS, smem, stream>>>(a);
    return check_launch("gather_gemm_kernel");
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
    SKV_CHECK_SUPPORTED(embed_dim == GG_N, "embed_dim must be 128");
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
    g.out_bh_stride = (int64_t)sparse_budget * GG_N;
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
    SKV_CHECK_SUPPORTED(gm->head_dim == GG_N && gm->chunk_size == 8, "head_dim 128 and chunk 8 only");
    SKV_CHECK_SUPPORTED(gm->rank % 16 == 0 && gm->rank >= 16 && gm->rank <= 256,
                        "rank must be a multiple of 16 in 16..256");
    SKV_CHECK_SUPPORTED(gm->rope_mode == 0 || gm->rope_mode == 1, "rope_mode must be 0 or 1");
    SKV_CHECK_ARG(gm->cos_sin_stride >= (gm->rope_mode == 0 ? 128 : 64), "cos_sin_stride too small");
    SKV_CHECK_ARG(gm->sparse_start >= 0 && gm->sparse_start + 8 * (int64_t)gm->select_sets <= gm->buf_len,
                  "selected rows exceed buf_len");
    SKV_CHECK_ARG(aligned(U, 16) && aligned(SVt, 16) && aligned(k_buf, 16), "operands must be 16-byte aligned");
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
    g.out_bh_stride = (int64_t)gm->buf_len * GG_N;
    g.out_row0 = gm->sparse_start;
    g.cs_stride = gm->cos_sin_stride;
    g.cs_rows = gm->cos_sin_rows;
    return launch_gather_gemm(g, gm->rope_mode == 0 ? 1 : 2, gm->batch * gm->kv_heads,
                              (cudaStream_t)stream);
}

}  // extern "C"
