// Gathered low-rank key reconstruction on the 5th-generation tensor cores
// (tcgen05.mma, accumulator in tensor memory).
//
// Same operation as gather_gemm.cu (reference: kernels/batch_gather_gemm.cu:
// 136-213 and the RoPE epilogue of kernels/rope_new.cu:224-374): rows of U
// selected by chunk id times the per-head SV^T, bf16 in, fp32 accumulate, an
// optional RoPE at the original token positions applied to the fp32
// accumulator, one rounding to bf16.
//
// One CTA computes 16 chunks (M = 128 rows) x 128 output dims over the full
// rank K:
//   * the operands come in through tensor-map (TMA) copies that write the
//     tensor cores' shared-memory layout directly, with no relayout pass and
//     without the SM's load/store path (16-byte cp.async loads through it held
//     a CTA's 112 KB of operands to about 25 GB/s per SM).  SV^T of the head
//     is requested before the chunk ids are known.
//       - rank >= 64: the 128-byte-swizzled K-major layout.  A copy of a box of
//         64 k x 8 rows (one chunk of U) or 64 k x 128 rows (SV^T of the head)
//         per 64-element k-block writes 8-row x 128-byte atoms, 8-row groups
//         1 KB apart; k past the rank is zero-filled.  Every request moves a
//         whole 128-byte row.
//       - smaller ranks: the no-swizzle K-major core-matrix layout (8-row x
//         16-byte core matrices).  The maps view a row as rank/8 pieces of 16
//         bytes with the piece index as the outermost box dimension, so one
//         copy of box {8 elements, rows, rank/8} lands piece-major: SV^T rows
//         16 bytes apart and pieces 2 KiB apart, a chunk's pieces 128 bytes
//         apart and chunks rank*16 bytes apart.
//     The cos/sin rows of the epilogue come in by cp.async (padded rows);
//   * one thread issues K/16 tcgen05.mma (kind::f16, bf16 x bf16 -> fp32,
//     M=128, N=128) into 128 columns of tensor memory and commits them to an
//     mbarrier (bounded wait);
//   * warps w and w+4 read rows 32w..32w+31 back with tcgen05.ld (thread =
//     row, half of the columns each), so the rotate-half pairs (t, t+64) and
//     the GLM pairs (2i, 2i+1) of a row are in one thread; RoPE on the fp32
//     values (cos/sin rows staged in shared memory), one rounding, rows
//     staged in shared memory and written as coalesced 256-byte rows.
#include "gather_gemm.cuh"

namespace skv {

constexpr int TC_CHUNKS = 16;               // chunks per CTA
constexpr int TC_ROWS = TC_CHUNKS * 8;      // M = 128
constexpr int TC_N = 128;                   // N = head_dim
constexpr int TC_THREADS = 256;             // warps w and w+4 read tensor-memory lanes 32w .. 32w+31
constexpr int TC_PITCH = 136;               // row pitch (bf16) of the cos/sin and output staging tiles
constexpr uint32_t TC_TMEM_COLS = 128;      // fp32 accumulator: one column per output dim
// SV^T operand: byte distance between its 16-byte k-pieces (N/8 core matrices)
// and between its 8-row groups
constexpr uint32_t TC_LBO = (TC_N / 8) * 128;
constexpr uint32_t TC_SBO = 128;

// Instruction descriptor, kind::f16: D fp32 (bits 4-5 = 1), A bf16 (bits 7-9 = 1),
// B bf16 (bits 10-12 = 1), A and B K-major (bits 15, 16 = 0), N/8 at bits 17-22,
// M/16 at bits 24-28.
constexpr uint32_t TC_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TC_N >> 3) << 17) |
                              ((uint32_t)(TC_ROWS >> 4) << 24);

// Shared-memory matrix descriptor: start address, leading (k-chunk) and stride
// (8-row group) byte offsets in 16-byte units, version 1, no swizzle.
__device__ __forceinline__ uint64_t tc_sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo)
{
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Tensor-map copy of one box into shared memory, completion (transaction
// bytes) on the mbarrier; the innermost coordinate is always 0 (aligned).
__device__ __forceinline__ void tc_tma3(void *smem, const CUtensorMap *map, int y, int z, uint64_t *bar)
{
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3, %4}], [%5];"
                 ::"r"(smem_u32(smem)), "l"(map), "r"(0), "r"(y), "r"(z), "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tc_tma2(void *smem, const CUtensorMap *map, int x, int y, uint64_t *bar)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(smem_u32(smem)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)) : "memory");
}
// K-major operand in the 128-byte-swizzled layout: 64-element k-blocks of 8-row
// atoms (8 rows x 128 bytes, the 16-byte pieces of row r permuted by r % 8),
// 8-row groups 1 KB apart; the start steps 32 bytes per 16 k inside a block
__device__ __forceinline__ uint64_t tc_sdesc_sw(uint32_t saddr)
{
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(1024u >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}
__device__ __forceinline__ void tc_tma4(void *smem, const CUtensorMap *map, int w, uint64_t *bar)
{
    asm volatile("cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3, %4, %5}], [%6];"
                 ::"r"(smem_u32(smem)), "l"(map), "r"(0), "r"(0), "r"(0), "r"(w), "r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tc_cp16(void *smem, const void *gmem)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem));
}

__device__ __forceinline__ void tc_ld16(uint32_t taddr, float *v)
{
    uint32_t r[16];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                   "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
                   "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Operand bytes of U (A) or SV^T (B) in shared memory: 128 rows of rank
// elements, padded to whole 64-element k-blocks in the swizzled layout.
__host__ __device__ __forceinline__ int tc_oper_bytes(int rank, bool sw)
{
    return sw ? ((rank + 63) / 64) * 16384 : 128 * rank * 2;
}

// ROPE: 0 none, 1 rotate-half (cos_sin width 128), 2 GLM interleaved (width 64).
// SW (rank >= 64): the operands in the 128-byte-swizzled K-major layout,
//   tmU: U as [rows = B*ctx][rank], box {64, 8} (one chunk, one k-block),
//   tmB: SV^T as [B*H*128][rank], box {64, 128} (one head, one k-block);
//   a copy moves whole 128-byte rows (768 row requests per CTA at rank 160).
// Otherwise the no-swizzle layout of 16-byte pieces,
//   tmU: U as [rows = B*ctx][rank/8 pieces][8], box {8, 8, rank/8} (one chunk),
//   tmB: SV^T as [B*H][128][rank/8 pieces][8], box {8, 128, rank/8, 1} (one head).
template <int ROPE, bool SW>
__global__ void __launch_bounds__(TC_THREADS) gather_gemm_tc_kernel(GatherGemmArgs a, const __grid_constant__ CUtensorMap tmU,
                                                                    const __grid_constant__ CUtensorMap tmB)
{
    extern __shared__ __align__(128) unsigned char smem_raw[];
    // operand tiles start on a 1024-byte boundary (the tensor copies need 128;
    // the MMA descriptors of U step through it in 256-byte pieces of K)
    unsigned char *smem = reinterpret_cast<unsigned char *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    // U rows: SW [k-block][16 chunks][8 rows x 128 B], else [16 chunks][K/8][8][8];
    // SV^T: SW [k-block][128 rows x 128 B], else [K/8][128][8]
    const int opb = tc_oper_bytes(a.rank, SW);
    __nv_bfloat16 *sA = reinterpret_cast<__nv_bfloat16 *>(smem);
    __nv_bfloat16 *sB = sA + opb / 2;
    __nv_bfloat16 *sCS = sB + opb / 2;                                 // cos/sin rows [128][TC_PITCH]
    // output rows [128][TC_PITCH]: in the operand tiles once the MMAs have
    // consumed them, past the cos/sin rows when the tiles are smaller (low rank)
    const bool o_in_ops = opb >= TC_ROWS * TC_PITCH * 2;
    __nv_bfloat16 *sO = o_in_ops ? sA : sCS + TC_ROWS * TC_PITCH;
    __shared__ uint32_t s_tmem;
    __shared__ __align__(8) uint64_t s_bar;    // the MMAs are complete
    __shared__ __align__(8) uint64_t s_bar_a;  // the U rows have landed
    __shared__ __align__(8) uint64_t s_bar_b;  // SV^T has landed
    __shared__ int s_chunk[TC_CHUNKS], s_dst[TC_CHUNKS];

    const int bh = blockIdx.y;
    const int b = bh / a.H;
    const int j0 = blockIdx.x * TC_CHUNKS;
    const int lo = a.lo ? a.lo[bh] : 0;
    const int hi = a.hi ? a.hi[bh] : a.M;
    if (j0 + TC_CHUNKS <= lo || j0 >= hi) return;  // uniform: before any tensor-memory use
    const int tid = threadIdx.x, warp = tid >> 5;
    const int kc = a.rank / 8;
    const unsigned chunk_bytes = (unsigned)kc * 128u;  // 8 rows x rank, bf16
    const int nkb = (a.rank + 63) / 64;                // 64-element k-blocks (SW)

    if (tid == 0) {
        mbar_init(&s_bar, 1);
        mbar_init(&s_bar_a, 1);
        mbar_init(&s_bar_b, 1);
        mbar_fence_init();
        // SV^T of the head does not depend on the chunk ids: requested first
        if (SW) {
            mbar_arrive_expect_tx(&s_bar_b, (unsigned)nkb * 16384u);  // whole boxes, k past rank zero-filled
            for (int kb = 0; kb < nkb; ++kb) tc_tma2(sB + kb * 8192, &tmB, kb * 64, bh * TC_N, &s_bar_b);
        } else {
            mbar_arrive_expect_tx(&s_bar_b, 16u * chunk_bytes);
            tc_tma4(sB, &tmB, bh, &s_bar_b);
        }
    }
    if (tid < TC_CHUNKS) {
        const int j = j0 + tid;
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
        s_chunk[tid] = c;
        s_dst[tid] = d;
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&s_tmem)), "r"(TC_TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    __syncthreads();

    // ---- U rows of the chunks: one tensor copy per chunk, straight into the
    //      core-matrix layout; the rows of missing chunks are zero
    if (tid == 0) {
        unsigned n = 0;
        for (int e = 0; e < TC_CHUNKS; ++e) n += s_chunk[e] >= 0 ? 1u : 0u;
        mbar_arrive_expect_tx(&s_bar_a, n * (SW ? (unsigned)nkb * 1024u : chunk_bytes));
    }
    __syncwarp();
    if (tid < TC_CHUNKS && s_chunk[tid] >= 0) {
        if (SW) {
            for (int kb = 0; kb < nkb; ++kb)
                tc_tma2(sA + kb * 8192 + tid * 512, &tmU, kb * 64, b * a.ctx + s_chunk[tid] * 8, &s_bar_a);
        } else {
            tc_tma3(sA + tid * kc * 64, &tmU, b * a.ctx + s_chunk[tid] * 8, 0, &s_bar_a);
        }
    }
    // rows of missing chunks are zero (16-byte pieces: SW 64 per chunk and k-block)
    for (int p = tid; p < (SW ? nkb * TC_CHUNKS * 64 : TC_CHUNKS * kc * 8); p += TC_THREADS) {
        const int e = SW ? (p >> 6) & (TC_CHUNKS - 1) : p / (kc * 8);
        if (s_chunk[e] < 0) st_v4(sA + p * 8, make_uint4(0, 0, 0, 0));
    }
    {
        if (ROPE != 0) {
            // cos/sin rows of the output rows' positions, for the epilogue
            const int csp = ROPE == 1 ? 16 : 8;  // 16-byte pieces per row
            for (int p = tid; p < TC_ROWS * csp; p += TC_THREADS) {
                const int r = p / csp, c = p % csp;
                const int ch = s_chunk[r >> 3];
                const int64_t pos = (int64_t)(ch < 0 ? 0 : ch) * 8 + (r & 7);
                if (ch >= 0 && pos < a.cs_rows) tc_cp16(sCS + r * TC_PITCH + c * 8, a.cos_sin + pos * a.cs_stride + c * 8);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        // generic-proxy writes of shared memory (zero rows) become visible to the tensor core
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    // bounded waits: a copy that never lands is reported, it does not hang the GPU
    if (!mbar_wait(&s_bar_b, 0) || !mbar_wait(&s_bar_a, 0)) {
        if ((tid & 31) == 0) report_dev_error(DEV_ERR_WAIT);
        mbar_wait(&s_bar_b, 0);  // the copies must land before the memory is reused
        mbar_wait(&s_bar_a, 0);
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = s_tmem;

    // ---- K/16 MMAs by one thread, completion to the mbarrier
    if (tid == 0) {
        const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
        for (int ks = 0; ks < a.rank / 16; ++ks) {
            uint64_t ad, bd;
            if (SW) {
                // k-block ks / 4, 32 bytes per 16 k inside it
                const uint32_t off = (uint32_t)(ks >> 2) * 16384u + (uint32_t)(ks & 3) * 32u;
                ad = tc_sdesc_sw(a0 + off);
                bd = tc_sdesc_sw(b0 + off);
            } else {
                // A: pieces 128 bytes apart, 8-row groups (chunks) rank*16 bytes apart
                ad = tc_sdesc(a0 + (uint32_t)ks * 256u, 128u, chunk_bytes);
                bd = tc_sdesc(b0 + (uint32_t)ks * 2u * TC_LBO, TC_LBO, TC_SBO);
            }
            const uint32_t acc = ks > 0 ? 1u : 0u;
            asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                         "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
                         ::"r"(tmem), "l"(ad), "l"(bd), "r"(TC_IDESC), "r"(acc), "r"(0u) : "memory");
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                     ::"r"(smem_u32(&s_bar)) : "memory");
    }
    __syncwarp();
    if (!mbar_wait(&s_bar, 0)) {
        if ((tid & 31) == 0) report_dev_error(DEV_ERR_WAIT);
        mbar_wait(&s_bar, 0);  // the MMAs must be done before the memory is released
    }
    // the cos/sin rows of the epilogue (every thread's cp.async) have landed
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");

    // ---- epilogue: warp w (and w+4) reads rows 32(w%4) .. +31, one row per
    //      thread; warps 0-3 take column blocks {0,16,64,80}, warps 4-7
    //      {32,48,96,112}, so the rotate-half pair (t, t+64) stays in a thread.
    //      Rows go through shared memory for coalesced 256-byte stores.
    {
        const int q = warp & 3, half = warp >> 2;
        const int r = q * 32 + (tid & 31);
        const int e = r >> 3;
        const int c = s_chunk[e];
        const int64_t pos = (int64_t)(c < 0 ? 0 : c) * 8 + (r & 7);
        const bool rope_ok = ROPE == 0 || (c >= 0 && pos < a.cs_rows);
        if (ROPE != 0 && c >= 0 && pos >= a.cs_rows && half == 0) report_dev_error(DEV_ERR_ROW);
        const __nv_bfloat16 *cs = sCS + r * TC_PITCH;
        const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int h = half * 2 + hh;
            float x[16], y[16];  // columns 16h .. 16h+15 and 64+16h .. 64+16h+15
            tc_ld16(trow + 16 * h, x);
            tc_ld16(trow + 64 + 16 * h, y);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (ROPE == 1 && rope_ok) {
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int t = 16 * h + i;
                    const float cc = bf2f(cs[t]), ss = bf2f(cs[t + 64]);
                    const float x1 = x[i], x2 = y[i];
                    x[i] = x1 * cc - x2 * ss;
                    y[i] = x2 * cc + x1 * ss;
                }
            } else if (ROPE == 2 && rope_ok) {
#pragma unroll
                for (int i = 0; i < 16; i += 2) {
                    const int tp = (16 * h + i) >> 1;  // pair index < 32
                    const float cc = bf2f(cs[tp]), ss = bf2f(cs[tp + 32]);
                    const float xe = x[i], xo = x[i + 1];
                    x[i] = xe * cc - xo * ss;
                    x[i + 1] = xo * cc + xe * ss;
                }
            }
            __nv_bfloat16 *orow = sO + r * TC_PITCH;
            st_v4(orow + 16 * h, make_uint4(pack_bf2(x[0], x[1]), pack_bf2(x[2], x[3]), pack_bf2(x[4], x[5]), pack_bf2(x[6], x[7])));
            st_v4(orow + 16 * h + 8, make_uint4(pack_bf2(x[8], x[9]), pack_bf2(x[10], x[11]), pack_bf2(x[12], x[13]), pack_bf2(x[14], x[15])));
            st_v4(orow + 64 + 16 * h, make_uint4(pack_bf2(y[0], y[1]), pack_bf2(y[2], y[3]), pack_bf2(y[4], y[5]), pack_bf2(y[6], y[7])));
            st_v4(orow + 64 + 16 * h + 8, make_uint4(pack_bf2(y[8], y[9]), pack_bf2(y[10], y[11]), pack_bf2(y[12], y[13]), pack_bf2(y[14], y[15])));
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    // coalesced row stores: 16 threads per 256-byte row
    for (int p = tid; p < TC_ROWS * 16; p += TC_THREADS) {
        const int r = p >> 4, c = (p & 15) * 8;
        const int d = s_dst[r >> 3];
        if (d < 0) continue;
        st_v4(a.out + (int64_t)bh * a.out_bh_stride + ((int64_t)a.out_row0 + (int64_t)d * 8 + (r & 7)) * TC_N + c,
              ld_v4(sO + r * TC_PITCH + c));
    }

    // ---- release the tensor memory (every lane's loads completed before the barrier above)
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS) : "memory");
    }
}

static bool tc_swizzled(int rank) { return rank >= 64; }

size_t gg_tc_smem_bytes(int rank)
{
    // operands, cos/sin rows, output rows (in the operand tiles when they fit), alignment slack
    const size_t opb = (size_t)tc_oper_bytes(rank, tc_swizzled(rank)), tile = (size_t)TC_ROWS * TC_PITCH * 2;
    return 2 * opb + tile + (opb >= tile ? 0 : tile) + 1024;
}

// Tensor map of a bf16 matrix whose rows are rank/8 pieces of 16 bytes, viewed
// as [outer][rows][pieces][8] with the pieces as the outer box dimension
// (dims innermost first: 8 elements, rows, pieces, outer).
static int tc_tensor_map(CUtensorMap *m, const void *base, uint64_t rows, uint64_t outer, bool four_d, int rank,
                         uint32_t box_rows, const char *name)
{
    const uint64_t row_bytes = (uint64_t)rank * 2;
    const cuuint64_t dims[4] = {8, rows, (cuuint64_t)(rank / 8), outer};
    const cuuint64_t strides[3] = {row_bytes, 16, row_bytes * rows};  // of dims 1..3, bytes
    const cuuint32_t box[4] = {8, box_rows, (cuuint32_t)(rank / 8), 1};
    return encode_tensor_map_bf16(m, base, four_d ? 4u : 3u, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE, name);
}

int launch_gather_gemm_tc(const GatherGemmArgs &a, int rope, int nbh, cudaStream_t stream)
{
    SKV_CHECK_ARG(aligned(a.U, 16) && aligned(a.SVt, 16), "U and SV^T must be 16-byte aligned");
    SKV_CHECK_ARG(nbh % a.H == 0, "batch x heads must be a multiple of heads");
    const int smem = (int)gg_tc_smem_bytes(a.rank);
    dim3 grid(ceil_div(a.M, TC_CHUNKS), nbh);
    int st = SKV_OK;
    CUtensorMap tmU, tmB;
    const bool sw = tc_swizzled(a.rank);
    const uint64_t urows = (uint64_t)(nbh / a.H) * (uint64_t)a.ctx;  // every sequence's rows of U
    if (sw) {
        const cuuint64_t ustr[1] = {(cuuint64_t)a.rank * 2};
        const cuuint64_t udims[2] = {(cuuint64_t)a.rank, urows}, bdims[2] = {(cuuint64_t)a.rank, (cuuint64_t)nbh * TC_N};
        const cuuint32_t ubox[2] = {64, 8}, bbox[2] = {64, (cuuint32_t)TC_N};
        st = encode_tensor_map_bf16(&tmU, a.U, 2, udims, ustr, ubox, CU_TENSOR_MAP_SWIZZLE_128B, "U");
        if (st) return st;
        st = encode_tensor_map_bf16(&tmB, a.SVt, 2, bdims, ustr, bbox, CU_TENSOR_MAP_SWIZZLE_128B, "SV^T");
        if (st) return st;
    } else {
        // U: one chunk of 8 rows per box; SV^T: 128 rows per (sequence, head), one head per box
        st = tc_tensor_map(&tmU, a.U, urows, 1, false, a.rank, 8, "U");
        if (st) return st;
        st = tc_tensor_map(&tmB, a.SVt, TC_N, (uint64_t)nbh, true, a.rank, TC_N, "SV^T");
        if (st) return st;
    }
    const void *fn = sw ? (rope == 0 ? (const void *)gather_gemm_tc_kernel<0, true>
                           : rope == 1 ? (const void *)gather_gemm_tc_kernel<1, true>
                                       : (const void *)gather_gemm_tc_kernel<2, true>)
                        : (rope == 0 ? (const void *)gather_gemm_tc_kernel<0, false>
                           : rope == 1 ? (const void *)gather_gemm_tc_kernel<1, false>
                                       : (const void *)gather_gemm_tc_kernel<2, false>);
    st = ensure_smem_attr(fn, smem, "gather_gemm_tc_kernel");
    if (st) return st;
    void *args[] = {const_cast<GatherGemmArgs *>(&a), &tmU, &tmB};
    SKV_CUDA(cudaLaunchKernel(fn, grid, dim3(TC_THREADS), args, (size_t)smem, stream));
    return check_launch("gather_gemm_tc_kernel");
}

}  // namespace skv
