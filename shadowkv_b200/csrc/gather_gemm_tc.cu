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
//   * 256 threads gather the U rows of the chunks and SV^T of the head into
//     shared memory with 16-byte cp.async, in the no-swizzle K-major layout of
//     the tensor-core descriptors: 8-row x 16-byte core matrices of 128
//     contiguous bytes, 8-row groups 128 bytes apart, 16-byte k-chunks
//     (M/8)*128 bytes apart;
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
// byte distance between the 16-byte k-chunks of one operand (M/8 core matrices)
constexpr uint32_t TC_LBO = (TC_ROWS / 8) * 128;
constexpr uint32_t TC_SBO = 128;            // between 8-row groups

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

// Element offset of (row r, k) in the K-major core-matrix layout of an operand with TC_ROWS rows.
__device__ __forceinline__ int tc_off(int r, int k)
{
    return ((k >> 3) * (TC_ROWS / 8) + (r >> 3)) * 64 + (r & 7) * 8 + (k & 7);
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

// ROPE: 0 none, 1 rotate-half (cos_sin width 128), 2 GLM interleaved (width 64)
template <int ROPE>
__global__ void __launch_bounds__(TC_THREADS) gather_gemm_tc_kernel(GatherGemmArgs a)
{
    extern __shared__ __align__(128) unsigned char smem_raw[];
    // operand tiles start on a 1024-byte boundary: the descriptors address a
    // matrix from an aligned base (an unaligned start shifted the rows read)
    unsigned char *smem = reinterpret_cast<unsigned char *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    __nv_bfloat16 *sA = reinterpret_cast<__nv_bfloat16 *>(smem);       // U rows  [K/8][16][8][8]
    __nv_bfloat16 *sB = sA + TC_ROWS * a.rank;                         // SV^T    [K/8][16][8][8]
    __nv_bfloat16 *sCS = sB + TC_N * a.rank;                           // cos/sin rows [128][TC_PITCH]
    // output rows [128][TC_PITCH]: in the operand tiles once the MMAs have
    // consumed them, past the cos/sin rows when the tiles are smaller (low rank)
    const bool o_in_ops = 2 * a.rank >= TC_PITCH;
    __nv_bfloat16 *sO = o_in_ops ? sA : sCS + TC_ROWS * TC_PITCH;
    __shared__ uint32_t s_tmem;
    __shared__ __align__(8) uint64_t s_bar;
    __shared__ int s_chunk[TC_CHUNKS], s_dst[TC_CHUNKS];

    const int bh = blockIdx.y;
    const int b = bh / a.H;
    const int j0 = blockIdx.x * TC_CHUNKS;
    const int lo = a.lo ? a.lo[bh] : 0;
    const int hi = a.hi ? a.hi[bh] : a.M;
    if (j0 + TC_CHUNKS <= lo || j0 >= hi) return;  // uniform: before any tensor-memory use
    const int tid = threadIdx.x, warp = tid >> 5;

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
    if (tid == 0) {
        mbar_init(&s_bar, 1);
        mbar_fence_init();
    }
    __syncthreads();

    // ---- operands into the core-matrix layout (rows of missing chunks are zero)
    const int kc = a.rank / 8;
    {
        const __nv_bfloat16 *Ub = a.U + (int64_t)b * a.ctx * a.rank;
        for (int p = tid; p < TC_ROWS * kc; p += TC_THREADS) {
            const int r = p / kc, c = p % kc;
            const int ch = s_chunk[r >> 3];
            __nv_bfloat16 *dst = sA + tc_off(r, c * 8);
            if (ch >= 0) tc_cp16(dst, Ub + ((int64_t)ch * 8 + (r & 7)) * a.rank + c * 8);
            else st_v4(dst, make_uint4(0, 0, 0, 0));
        }
        const __nv_bfloat16 *Bb = a.SVt + (int64_t)bh * TC_N * a.rank;
        for (int p = tid; p < TC_N * kc; p += TC_THREADS) {
            const int n = p / kc, c = p % kc;
            tc_cp16(sB + tc_off(n, c * 8), Bb + (int64_t)n * a.rank + c * 8);
        }
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
        asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
        // generic-proxy writes of shared memory become visible to the tensor core
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = s_tmem;

    // ---- K/16 MMAs by one thread, completion to the mbarrier
    if (tid == 0) {
        const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
        for (int ks = 0; ks < a.rank / 16; ++ks) {
            const uint64_t ad = tc_sdesc(a0 + (uint32_t)ks * 2u * TC_LBO, TC_LBO, TC_SBO);
            const uint64_t bd = tc_sdesc(b0 + (uint32_t)ks * 2u * TC_LBO, TC_LBO, TC_SBO);
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

size_t gg_tc_smem_bytes(int rank)
{
    // operands, cos/sin rows, output rows (in the operand tiles when they fit), alignment slack
    const size_t ops = (size_t)(TC_ROWS + TC_N) * rank * 2, tile = (size_t)TC_ROWS * TC_PITCH * 2;
    return ops + tile + (2 * rank >= TC_PITCH ? 0 : tile) + 1024;
}

int launch_gather_gemm_tc(const GatherGemmArgs &a, int rope, int nbh, cudaStream_t stream)
{
    const int smem = (int)gg_tc_smem_bytes(a.rank);
    dim3 grid(ceil_div(a.M, TC_CHUNKS), nbh);
    const void *fn = rope == 0 ? (const void *)gather_gemm_tc_kernel<0>
                   : rope == 1 ? (const void *)gather_gemm_tc_kernel<1> : (const void *)gather_gemm_tc_kernel<2>;
    int st = ensure_smem_attr(fn, smem, "gather_gemm_tc_kernel");
    if (st) return st;
    if (rope == 0) gather_gemm_tc_kernel<0><<<grid, TC_THREADS, smem, stream>>>(a);
    else if (rope == 1) gather_gemm_tc_kernel<1><<<grid, TC_THREADS, smem, stream>>>(a);
    else gather_gemm_tc_kernel<2><<<grid, TC_THREADS, smem, stream>>>(a);
    return check_launch("gather_gemm_tc_kernel");
}

}  // namespace skv
