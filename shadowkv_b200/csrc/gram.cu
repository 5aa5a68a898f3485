// Gram matrix K^T K of the prompt's pre-RoPE keys on the 5th-generation tensor
// cores -- the contraction of the rank-r factorisation of the prefill.
//
// Reference: ShadowKVCache_CPU.get_svd (models/kvcache/shadow.py:411-444) runs
// torch.svd on K [T, H*128] (fp32) and keeps the leading `rank` singular
// triplets.  The library computes the same leading subspace from the Gram
// matrix: K^T K = V S^2 V^T, its `rank` leading eigenvectors are the right
// singular vectors, and U = K V / s.  The T x D x D contraction (D = H*128,
// T up to 1M) is the heavy part; the D x D eigensolve stays a library call.
//
// One CTA per (256 x 256 output block of the upper triangle -- four 128 x 128
// tiles, the lower one left out on the diagonal --, slice of the T rows):
//   * one thread streams 64-row slices of the block's two 256-column operands
//     of K through a 3-stage ring of tensor-map (TMA) copies, two boxes of 64
//     columns x 64 rows per 128 columns, in the 128-byte-swizzled MN-major layout
//     the tensor cores read (a 64-column half is 64 rows of 128 bytes, the
//     16-byte pieces of row r permuted by r % 8; halves LBO = 8 KB apart,
//     8-row groups SBO = 1 KB apart), so K needs no transposition.  Rows past
//     the end of K are zero-filled by the copy.  (16-byte cp.async loads by
//     all threads into the no-swizzle layout held the kernel to the load
//     path's rate, long-scoreboard stalls, ~0.13 of the tensor peak);
//   * the same thread issues 4 tcgen05.mma (kind::f16, bf16 -> fp32,
//     M = N = 128, K = 16, both operands MN-major) per tile and slice once the
//     slice's copies have landed (the stage's mbarrier), committed to the
//     slice's MMA mbarrier, which frees the stage for the slice three ahead
//     (bounded waits).  A 256 x 256 block takes two operand bytes per 256
//     flops where a single 128 x 128 tile took one per 64: the operand feed
//     into the SM, not the tensor cores, bounded the 128 x 128 version;
//   * the four fp32 accumulators (all 512 tensor-memory columns) are read
//     back with tcgen05.ld and stored as the slice's partial tiles.
// gram_reduce_kernel then sums the partials of every tile in float64 and
// writes both triangles of the D x D result.
#include "common.cuh"

namespace skv {

constexpr int GR_THREADS = 256;
constexpr int GR_ROWS = 64;                        // K rows (the contraction dim) per stage
constexpr int GR_STAGES = 3;
constexpr int GR_BLOCK_BYTES = GR_ROWS * 128 * 2;  // one 128-column operand block of a stage: 16 KB
constexpr int GR_OPER_BYTES = 2 * GR_BLOCK_BYTES;  // one 256-column operand of a stage: 32 KB
constexpr int GR_STAGE_BYTES = 2 * GR_OPER_BYTES;
// stages, and the slack of the 1024-byte alignment of the swizzled tiles
constexpr int GR_SMEM = GR_STAGES * GR_STAGE_BYTES + 1024;
constexpr uint32_t GR_LBO = 8192;  // between the 64-column halves of a 128-column block (MN direction)
constexpr uint32_t GR_SBO = 1024;  // between 8-row groups (K direction): 8 rows x 128 B
constexpr uint32_t GR_TMEM_COLS = 512;  // four 128 x 128 fp32 accumulators
// kind::f16: D fp32, A and B bf16, A and B MN-major (bits 15, 16), N/8 at 17, M/16 at 24
constexpr uint32_t GR_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (1u << 16) | ((128u >> 3) << 17) |
                              ((128u >> 4) << 24);

__device__ __forceinline__ uint64_t gr_sdesc(uint32_t saddr)
{
    // version 1 (bit 46), layout 128-byte swizzle (2 at bits 61-63)
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((GR_LBO >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((GR_SBO >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Tensor-map copy of the 64 x 64 box at (column x, row y) of K, completion on bar
__device__ __forceinline__ void gr_tma(void *smem, const CUtensorMap *map, int x, int y, uint64_t *bar)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(smem_u32(smem)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)) : "memory");
}

struct GramArgs {
    float *part;  // [splits][pairs][128][128], pairs of 128-column blocks
    int T, D;
    int nb, pairs;    // 128-column blocks and their upper-triangle pairs
    int nb2;          // 256-column blocks (the CTAs' column blocks)
    int splits, rows_per_split;
};

// p enumerates the upper-triangle block pairs (bi <= bj) of n blocks row by row
__device__ __forceinline__ void gr_pair(int p, int n, int *bi, int *bj)
{
    int i = 0;
    while (p >= n - i) {
        p -= n - i;
        ++i;
    }
    *bi = i;
    *bj = i + p;
}

// tmK: K as [T rows][D columns] (row stride ld), box 64 x 64, 128-byte swizzle.
// CTA (pair of 256-column blocks BI <= BJ, split): the 128 x 128 tiles (2 BI + ti,
// 2 BJ + tj) of the upper triangle, ti, tj in {0, 1}, accumulated in tensor-memory
// columns 128 (2 ti + tj) over the split's rows.
__global__ void __launch_bounds__(GR_THREADS, 1) gram_tc_kernel(GramArgs a, const __grid_constant__ CUtensorMap tmK)
{
    extern __shared__ __align__(128) unsigned char smem_raw[];
    unsigned char *smem = reinterpret_cast<unsigned char *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    __shared__ uint32_t s_tmem;
    __shared__ __align__(8) uint64_t s_full[GR_STAGES];  // the copies of the slice in the stage have landed
    __shared__ __align__(8) uint64_t s_mma[GR_STAGES];   // MMAs of the slice in the stage are done
    __shared__ __align__(8) uint64_t s_fin;

    const int pair = blockIdx.x, split = blockIdx.y;
    int BI, BJ;
    gr_pair(pair, a.nb2, &BI, &BJ);
    const bool diag = BI == BJ;
    const int t0 = split * a.rows_per_split, t1 = min(a.T, t0 + a.rows_per_split);
    const int nk = t1 > t0 ? (t1 - t0 + GR_ROWS - 1) / GR_ROWS : 0;
    const int tid = threadIdx.x, warp = tid >> 5;
    // 128-column blocks inside K: the second block of the last 256-column block
    // is past the end when D is an odd number of 128-column blocks
    const int nti = min(2, a.nb - 2 * BI), ntj = min(2, a.nb - 2 * BJ);
    // the tile (ti, tj) is computed when it is inside K and in the upper triangle
    auto live = [&](int ti, int tj) { return ti < nti && tj < ntj && (!diag || ti <= tj); };

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&s_tmem)), "r"(GR_TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int s = 0; s < GR_STAGES; ++s) {
            mbar_init(&s_full[s], 1);
            mbar_init(&s_mma[s], 1);
        }
        mbar_init(&s_fin, 1);
        mbar_fence_init();
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = s_tmem;

    // slice it of the CTA's rows into stage it % GR_STAGES (thread 0): operand A =
    // columns 256 BI .. +255, B = columns 256 BJ .. (not loaded on the diagonal),
    // the 128-column blocks inside K only; rows past the end of K land as zeros.
    // The split's rows are a multiple of 64, so a slice never reaches into the
    // next split's rows.
    auto load = [&](int it) {
        const int s = it % GR_STAGES;
        unsigned char *st = smem + (size_t)s * GR_STAGE_BYTES;
        const int r0 = t0 + it * GR_ROWS;
        mbar_arrive_expect_tx(&s_full[s], (unsigned)((nti + (diag ? 0 : ntj)) * GR_BLOCK_BYTES));
        for (int c = 0; c < 2; ++c) {
            for (int h = 0; h < 2; ++h) {
                if (c < nti)
                    gr_tma(st + c * GR_BLOCK_BYTES + h * GR_LBO, &tmK, (2 * BI + c) * 128 + h * 64, r0, &s_full[s]);
                if (!diag && c < ntj)
                    gr_tma(st + GR_OPER_BYTES + c * GR_BLOCK_BYTES + h * GR_LBO, &tmK, (2 * BJ + c) * 128 + h * 64,
                           r0, &s_full[s]);
            }
        }
    };

    if (tid == 0) {
        for (int it = 0; it < min(GR_STAGES, nk); ++it) load(it);
        for (int it = 0; it < nk; ++it) {
            const int s = it % GR_STAGES;
            // bounded waits: a copy or an MMA that never completes is reported, it does not hang the GPU
            if (!mbar_wait(&s_full[s], (it / GR_STAGES) & 1)) {
                report_dev_error(DEV_ERR_WAIT);
                mbar_wait(&s_full[s], (it / GR_STAGES) & 1);
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t sa = smem_u32(smem + (size_t)s * GR_STAGE_BYTES);
            const uint32_t sb = diag ? sa : sa + GR_OPER_BYTES;
            for (int ti = 0; ti < 2; ++ti) {
                for (int tj = 0; tj < 2; ++tj) {
                    if (!live(ti, tj)) continue;
                    const uint32_t d = tmem + (uint32_t)(2 * ti + tj) * 128u;
#pragma unroll
                    for (int ks = 0; ks < GR_ROWS / 16; ++ks) {
                        // 16 rows = two 8-row groups per MMA
                        const uint64_t ad = gr_sdesc(sa + (uint32_t)(ti * GR_BLOCK_BYTES) + (uint32_t)ks * 2u * GR_SBO);
                        const uint64_t bd = gr_sdesc(sb + (uint32_t)(tj * GR_BLOCK_BYTES) + (uint32_t)ks * 2u * GR_SBO);
                        const uint32_t acc = (it > 0 || ks > 0) ? 1u : 0u;
                        asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                                     "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
                                     ::"r"(d), "l"(ad), "l"(bd), "r"(GR_IDESC), "r"(acc), "r"(0u) : "memory");
                    }
                }
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                         ::"r"(smem_u32(&s_mma[s])) : "memory");
            // the stage of slice it - 1 takes slice it - 1 + GR_STAGES once that slice's MMAs are done
            const int nxt = it - 1 + GR_STAGES;
            if (it >= 1 && nxt < nk) {
                const int ps = (it - 1) % GR_STAGES;
                if (!mbar_wait(&s_mma[ps], ((it - 1) / GR_STAGES) & 1)) {
                    report_dev_error(DEV_ERR_WAIT);
                    mbar_wait(&s_mma[ps], ((it - 1) / GR_STAGES) & 1);
                }
                load(nxt);
            }
        }
    }
    // every MMA issued so far is complete once the last commit arrives
    if (tid == 0) {
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                     ::"r"(smem_u32(&s_fin)) : "memory");
    }
    __syncwarp();
    if (!mbar_wait(&s_fin, 0)) {
        if ((tid & 31) == 0) report_dev_error(DEV_ERR_WAIT);
        mbar_wait(&s_fin, 0);  // the MMAs must be done before the tensor memory is read or released
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

    // epilogue: per live tile, warp w reads tensor-memory lanes 32 (w % 4) .. +31
    // (one output row per thread), warps 0-3 columns 0..63, warps 4-7 columns
    // 64..127, into the partial of its 128-column block pair
    for (int ti = 0; ti < 2; ++ti) {
        for (int tj = 0; tj < 2; ++tj) {
            if (!live(ti, tj)) continue;
            const int bi = 2 * BI + ti, bj = 2 * BJ + tj;
            const int p128 = bi * a.nb - bi * (bi - 1) / 2 + (bj - bi);  // row-major upper-triangle index
            const int q = warp & 3, half = warp >> 2;
            const int r = q * 32 + (tid & 31);
            float *dst = a.part + (((int64_t)split * a.pairs + p128) * 128 + r) * 128 + half * 64;
            const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((2 * ti + tj) * 128 + half * 64);
#pragma unroll
            for (int c = 0; c < 64; c += 16) {
                uint32_t v[16];
                asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                             "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                             : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                               "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
                               "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                             : "r"(trow + (uint32_t)c));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int i = 0; i < 16; i += 4)
                    *reinterpret_cast<uint4 *>(dst + c + i) = make_uint4(v[i], v[i + 1], v[i + 2], v[i + 3]);
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(GR_TMEM_COLS) : "memory");
    }
}

// gram[D][D] (float64) = the sum over the splits of each tile's partials;
// grid (pairs, 128): block (p, r) writes row r of tile p and, off the
// diagonal, the mirrored column.
__global__ void __launch_bounds__(128) gram_reduce_kernel(const float *part, double *gram, int D, int nb, int pairs,
                                                         int splits)
{
    const int pair = blockIdx.x, r = blockIdx.y, c = threadIdx.x;
    int bi, bj;
    gr_pair(pair, nb, &bi, &bj);
    double s = 0.0;
    for (int k = 0; k < splits; ++k) s += (double)part[(((int64_t)k * pairs + pair) * 128 + r) * 128 + c];
    const int i = bi * 128 + r, j = bj * 128 + c;
    gram[(int64_t)i * D + j] = s;
    if (bi != bj) gram[(int64_t)j * D + i] = s;
}

struct GramPlan {
    int nb, pairs, nb2, pairs2, splits, rows_per_split;
    size_t part_bytes;
};

static GramPlan plan_gram(int T, int D)
{
    GramPlan p;
    p.nb = D / 128;
    p.pairs = p.nb * (p.nb + 1) / 2;
    p.nb2 = (p.nb + 1) / 2;
    p.pairs2 = p.nb2 * (p.nb2 + 1) / 2;
    const int sms = device_sm_count();
    int s = max(1, sms / p.pairs2);  // one CTA per SM
    s = min(s, ceil_div(T, GR_ROWS));
    p.rows_per_split = ceil_div(ceil_div(T, s), GR_ROWS) * GR_ROWS;
    p.splits = ceil_div(T, p.rows_per_split);
    p.part_bytes = (size_t)p.splits * p.pairs * 128 * 128 * 4;
    return p;
}

}  // namespace skv

using namespace skv;

extern "C" {

size_t skv_gram_workspace(int tokens, int dim)
{
    if (tokens <= 0 || dim <= 0 || dim % 128 != 0 || dim > 8192) return 0;
    return plan_gram(tokens, dim).part_bytes;
}

int skv_gram(const void *k, int tokens, int dim, int ld, double *gram, void *workspace, size_t workspace_bytes,
             void *stream)
{
    SKV_CHECK_ARG(k && gram && workspace, "null pointer argument");
    SKV_CHECK_SUPPORTED(tokens > 0 && dim > 0 && dim % 128 == 0 && dim <= 8192,
                        "dim must be a multiple of 128 in 128..8192 (tokens > 0)");
    SKV_CHECK_ARG(ld >= dim && ld % 8 == 0, "ld must be >= dim and a multiple of 8 (16-byte rows)");
    SKV_CHECK_ARG(aligned(k, 16) && aligned(workspace, 16) && aligned(gram, 8), "k, workspace (16 B) or gram unaligned");
    const GramPlan p = plan_gram(tokens, dim);
    SKV_CHECK_ARG(workspace_bytes >= p.part_bytes, "workspace of %zu bytes needed, %zu given", p.part_bytes,
                  workspace_bytes);
    int st = ensure_smem_attr((const void *)gram_tc_kernel, GR_SMEM, "gram_tc_kernel");
    if (st) return st;
    CUtensorMap tmK;
    {
        const cuuint64_t dims[2] = {(cuuint64_t)dim, (cuuint64_t)tokens};
        const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
        const cuuint32_t box[2] = {64, (cuuint32_t)GR_ROWS};
        st = encode_tensor_map_bf16(&tmK, k, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "K");
        if (st) return st;
    }
    GramArgs a;
    a.part = (float *)workspace;
    a.T = tokens;
    a.D = dim;
    a.nb = p.nb;
    a.pairs = p.pairs;
    a.nb2 = p.nb2;
    a.splits = p.splits;
    a.rows_per_split = p.rows_per_split;
    cudaStream_t s = (cudaStream_t)stream;
    gram_tc_kernel<<<dim3(p.pairs2, p.splits), GR_THREADS, GR_SMEM, s>>>(a, tmK);
    st = check_launch("gram_tc_kernel");
    if (st) return st;
    gram_reduce_kernel<<<dim3(p.pairs, 128), 128, 0, s>>>(a.part, gram, dim, p.nb, p.pairs, p.splits);
    return check_launch("gram_reduce_kernel");
}

}  // extern "C"
