// Landmark scoring and chunk selection.
//
// Reference: kernels/batch_gemm_softmax.cu:143-196 with
// kernels/batch_gemm_softmax.h:66-523 (CUTLASS 2.x GEMM + epilogue visitor +
// final reduction + softmax apply, three launches), then torch.max /
// torch.topk / gather in models/kvcache/shadow.py:547-576, then the reuse
// diff of kernels/map.cuh:475-516.
//
// The scoring GEMM has M = landmarks (thousands) and N = query heads of one
// GQA group (4 for Llama, 16 for GLM), K = 128.  It is bound by the landmark
// read.  Each warp multiplies 16 landmark rows with mma.sync m16n8k16; the K
// (head_dim) axis is permuted identically for A and B so that each thread
// feeds its fragments from four 16-byte loads per row straight from global
// memory -- no shared-memory staging and fully coalesced 256-byte rows.
#include "select.cuh"

namespace skv {

constexpr int SC_THREADS = 256;   // 8 warps
constexpr int SC_ROWS_PER_PASS = 16 * (SC_THREADS / 32);

// q fragments for one n-tile of 8 query rows: thread (g = lane>>2, j = lane&3)
// holds row nt*8+g, elements (i*4+j)*8 .. +8 for i = 0..3.
__device__ __forceinline__ void load_q_frag(uint4 (&qf)[4], const __nv_bfloat16 *qrows, int nrows,
                                            int nt, int lane)
{
    const int n = nt * 8 + (lane >> 2), j = lane & 3;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if (n < nrows) qf[i] = ld_nc_v4(qrows + (int64_t)n * 128 + (i * 4 + j) * 8);
        else qf[i] = make_uint4(0, 0, 0, 0);
    }
}

__device__ __forceinline__ uint32_t wsel(const uint4 &v, int w)
{
    return w == 0 ? v.x : (w == 1 ? v.y : (w == 2 ? v.z : v.w));
}

// 16 rows x (8*NT) logits.  ra/rb: rows g and g+8 (4 x uint4 each).
template <int NT>
__device__ __forceinline__ void tile_mma(float (&acc)[NT][4], const uint4 (&ra)[4],
                                         const uint4 (&rb)[4], const uint4 (&qf)[NT][4])
{
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
        const int i = s >> 1, w = (s & 1) * 2;
        const uint32_t a0 = wsel(ra[i], w), a2 = wsel(ra[i], w + 1);
        const uint32_t a1 = wsel(rb[i], w), a3 = wsel(rb[i], w + 1);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
            mma_bf16_16816(acc[nt], a0, a1, a2, a3, wsel(qf[nt][i], w), wsel(qf[nt][i], w + 1));
    }
}

__device__ __forceinline__ void online_update(float &m, float &s, float x)
{
    if (x > m) {
        s = s * __expf(m - x) + 1.f;
        m = x;
    } else {
        s += __expf(x - m);
    }
}

__device__ __forceinline__ void merge_stats(float &m, float &s, float m2, float s2)
{
    const float mm = fmaxf(m, m2);
    if (mm == -INFINITY) return;
    s = s * __expf(m - mm) + s2 * __expf(m2 - mm);
    m = mm;
}

// ---------------------------------------------------------------------------
// Fused path, kernel 1: logits[bh][c][g] = scale * q_g . LM_c and per-split
// online (max, sum-exp) per query head.
//
// grid = (nsplit, B*Hkv); 8 consumer warps + 1 producer warp, two CTAs per
// SM.  The producer streams the CTA's landmark rows through a 3-stage ring of
// 128-row (32 KB) shared-memory tiles with bulk (TMA) copies completed on
// mbarriers; each consumer warp multiplies 16 rows of a tile per stage on the
// tensor cores.  The three stages are requested before anything else the CTA
// does, so the landmark stream is in flight during the launch's prologue.
// The host sizes the grid from the device's SM count (the rows of a head split
// evenly over its CTAs), leaving a few SMs to the selection kernel that follows.
// With APPEND the kernel also performs the new-token step: it rotates the
// query rows of its GQA group itself, and the split-0 CTA of each head writes
// the rotated query, the rotated key and the value of the new token.
// ---------------------------------------------------------------------------
constexpr int ST_STAGES = 3;  // 3 x 32 KB tiles: two CTAs per SM
constexpr int ST_ROWS = 128;
constexpr int ST_CONSUMERS = 8;
constexpr int ST_THREADS = (ST_CONSUMERS + 1) * 32;
constexpr int ST_STAGE_BYTES = ST_ROWS * 256;
constexpr int ST_SMEM = ST_STAGES * ST_STAGE_BYTES + 16 * 128 * 2 + 1024;  // tiles, q rows, alignment slack

struct ScoreArgs {
    const __nv_bfloat16 *q;      // [B][Hq][128]: rotated (plain) or pre-RoPE (APPEND)
    const __nv_bfloat16 *lm;     // [BH][L][128]
    float *logits;               // [BH][L][G]
    float2 *part;                // [BH][G][nsplit]
    int Hkv, G, L, rows_per_split;
    float scale;
    // new-token step (APPEND)
    const __nv_bfloat16 *k_new, *v_new, *cos_sin;
    const int64_t *positions;
    __nv_bfloat16 *q_out, *k_buf, *v_buf;
    int buf_len, row, rope_mode, cs_stride, cs_rows;
    const int32_t *row_dev;  // if set: the append row, read on the device (graph replays of later steps)
    unsigned long long *span;  // optional: kernel span pair of a timed step (span_begin)
};

template <int NT, bool APPEND>
__global__ void __launch_bounds__(ST_THREADS, 2) score_tma_kernel(ScoreArgs a)
{
    extern __shared__ unsigned char smem_dyn[];
    unsigned char *smem = reinterpret_cast<unsigned char *>(((uintptr_t)smem_dyn + 1023) & ~(uintptr_t)1023);
    __nv_bfloat16 *sT = reinterpret_cast<__nv_bfloat16 *>(smem);                       // [STAGES][128][128]
    __nv_bfloat16 *sQ = reinterpret_cast<__nv_bfloat16 *>(smem + ST_STAGES * ST_STAGE_BYTES);  // [16][128]
    __shared__ __align__(8) uint64_t full[ST_STAGES], empty[ST_STAGES];
    __shared__ float2 s_part[ST_CONSUMERS][16];
    __shared__ int s_abort;

    const int bh = blockIdx.y, split = blockIdx.x, nsplit = gridDim.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, j = lane & 3;
    const int G = a.G, L = a.L;
    const int b = bh / a.Hkv, h = bh % a.Hkv;
    const int r_begin = split * a.rows_per_split;
    const int r_end = min(L, r_begin + a.rows_per_split);
    const int nst = r_end > r_begin ? (r_end - r_begin + ST_ROWS - 1) / ST_ROWS : 0;
    const __nv_bfloat16 *lmh = a.lm + (int64_t)bh * L * 128;

    pdl_launch_dependents();  // the selection kernel may be scheduled early (it waits for this grid)
    span_begin(a.span);
    SKV_TRACE_CTA(TR_SCORE_START);
    // trace builds: a record per CTA (thread 0, a consumer): 0 = bh | split << 16,
    // 1 = 0x5C0, 2 = start, 3 = first tile in, 4 = ns spent waiting for tiles,
    // 5 = loop end, 6 = tiles, 7 = end
    SKV_TRACE_REC_DECL;
    SKV_TRACE_REC_OPEN();
    SKV_TRACE_REC(0, (unsigned long long)bh | ((unsigned long long)split << 16));
    SKV_TRACE_REC(1, 0x5C0ull);
    SKV_TRACE_REC_NOW(2);
    SKV_TRACE_REC(6, (unsigned long long)nst);
#ifdef SKV_TRACE
    unsigned long long tr_wait = 0;
#endif
    const bool producer = warp == ST_CONSUMERS && lane == 0;
    if (producer) {
        for (int s = 0; s < ST_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], ST_CONSUMERS);
        }
        s_abort = 0;
        mbar_fence_init();
        // every stage of the ring is requested before the query prologue
        // below: the landmark stream is the bound of the kernel
        for (int i = 0; i < min(nst, ST_STAGES); ++i) {
            const int r0 = r_begin + i * ST_ROWS;
            const int nr = min(ST_ROWS, r_end - r0);
            mbar_arrive_expect_tx(&full[i], (unsigned)nr * 256u);
            bulk_g2s(sT + (size_t)i * ST_ROWS * 128, lmh + (int64_t)r0 * 128, (unsigned)nr * 256u, &full[i]);
        }
    }
    // Everything above reads only the landmarks.  A launch that follows the
    // step's input staging kernel as its programmatic dependent waits here for
    // the staged inputs (a no-op for an ordinary launch).
    pdl_wait();
    // query rows of the group in shared memory (rows >= G are zero).  The raw
    // rows (and the cos/sin row) are loaded in one parallel round first, so the
    // prologue costs one memory latency, not one per loop trip.
    const __nv_bfloat16 *qrows = a.q + ((int64_t)b * a.Hkv * G + (int64_t)h * G) * 128;
    __shared__ __align__(16) __nv_bfloat16 s_raw[18 * 128];  // q rows, then k row, then cos/sin row
    int64_t pos = 0;
    bool pos_ok = true;
    if (APPEND) {
        pos = a.positions[b];
        pos_ok = pos >= 0 && pos < a.cs_rows;
        if (!pos_ok && tid == 0 && split == 0) report_dev_error(DEV_ERR_ROW);
    }
    const int nrows = APPEND ? 18 : 16;  // q rows (16) [+ new key row, cos/sin row]
    for (int it = tid; it < nrows * 16; it += ST_THREADS) {
        const int r = it >> 4, c = (it & 15) * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < G) v = ld_nc_v4(qrows + (int64_t)r * 128 + c);
        else if (APPEND && r == 16) v = ld_nc_v4(a.k_new + (int64_t)bh * 128 + c);
        else if (APPEND && r == 17 && pos_ok && c < a.cs_stride) v = ld_nc_v4(a.cos_sin + pos * a.cs_stride + c);
        st_v4((APPEND ? s_raw : sQ) + r * 128 + c, v);
    }
    uint4 vnew = make_uint4(0, 0, 0, 0);
    if (APPEND && split == 0 && tid >= 64 && tid < 80) vnew = ld_nc_v4(a.v_new + (int64_t)bh * 128 + (tid - 64) * 8);
    __syncthreads();
    if (APPEND) {
        const __nv_bfloat16 *cs = s_raw + 17 * 128;
        for (int it = tid; it < 16 * 64; it += ST_THREADS) {
            const int r = it >> 6, t = it & 63;
            if (r < G && pos_ok) rope_pair_bf16(s_raw + r * 128, sQ + r * 128, cs, t, a.rope_mode);
            else if (r >= G) { sQ[r * 128 + t] = f2bf(0.f); sQ[r * 128 + t + 64] = f2bf(0.f); }
        }
        const int row = a.row_dev ? *a.row_dev : a.row;
        const bool row_ok = row >= 0 && row < a.buf_len;
        if (!row_ok && tid == 0 && split == 0) report_dev_error(DEV_ERR_ROW);
        if (split == 0 && pos_ok && row_ok) {
            // new token: rotated key and value of head h at buffer row `row`
            const int64_t brow = ((int64_t)bh * a.buf_len + row) * 128;
            if (tid < 64) rope_pair_bf16(s_raw + 16 * 128, a.k_buf + brow, cs, tid, a.rope_mode);
            else if (tid < 80) st_v4(a.v_buf + brow + (tid - 64) * 8, vnew);
        }
    }
    __syncthreads();
    if (APPEND && split == 0) {
        // rotated query rows of the group for the attention
        for (int it = tid; it < G * 16; it += ST_THREADS) {
            const int r = it >> 4, c = (it & 15) * 8;
            st_v4(a.q_out + ((int64_t)b * a.Hkv * G + (int64_t)h * G + r) * 128 + c, ld_v4(sQ + r * 128 + c));
        }
    }
    float m[NT][2], sm[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) m[nt][0] = m[nt][1] = -INFINITY, sm[nt][0] = sm[nt][1] = 0.f;

    if (warp == ST_CONSUMERS) {
        // ---- producer: one elected lane streams the row tiles
        if (lane == 0) {
            for (int i = ST_STAGES; i < nst; ++i) {
                const int s = i % ST_STAGES;
                if (i >= ST_STAGES && !mbar_wait(&empty[s], ((i / ST_STAGES) - 1) & 1)) {
                    report_dev_error(DEV_ERR_WAIT);
                    atomicExch(&s_abort, 1);
                    break;
                }
                const int r0 = r_begin + i * ST_ROWS;
                const int nr = min(ST_ROWS, r_end - r0);
                mbar_arrive_expect_tx(&full[s], (unsigned)nr * 256u);
                bulk_g2s(sT + (size_t)s * ST_ROWS * 128, lmh + (int64_t)r0 * 128, (unsigned)nr * 256u, &full[s]);
            }
        }
    } else {
        // ---- consumers
        uint4 qf[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int n = nt * 8 + g;
#pragma unroll
            for (int i = 0; i < 4; ++i) qf[nt][i] = ld_v4(sQ + n * 128 + (i * 4 + j) * 8);
        }
        float *lg = a.logits + (int64_t)bh * L * G;
        for (int i = 0; i < nst; ++i) {
            const int s = i % ST_STAGES;
#ifdef SKV_TRACE
            const unsigned long long tw0 = ::skv::trace_now();
#endif
            if (!mbar_wait(&full[s], (i / ST_STAGES) & 1)) {
                report_dev_error(DEV_ERR_WAIT);
                atomicExch(&s_abort, 1);
                break;
            }
#ifdef SKV_TRACE
            tr_wait += ::skv::trace_now() - tw0;
            if (i == 0) SKV_TRACE_REC_NOW(3);
#endif
            if (i == 0) SKV_TRACE_CTA(TR_SCORE_TILE0);
            const __nv_bfloat16 *tile = sT + (size_t)s * ST_ROWS * 128;
            const int lr = warp * 16 + g;  // local rows lr and lr+8
            uint4 ra[4], rb[4];
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
                ra[q4] = ld_v4(tile + lr * 128 + (q4 * 4 + j) * 8);
                rb[q4] = ld_v4(tile + (lr + 8) * 128 + (q4 * 4 + j) * 8);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);  // the tile's rows are in registers
            float acc[NT][4];
            tile_mma<NT>(acc, ra, rb, qf);
            const int r0 = r_begin + i * ST_ROWS;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int n0 = nt * 8 + 2 * j;
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int row = r0 + lr + 8 * u;
                    const float x0 = acc[nt][2 * u] * a.scale, x1 = acc[nt][2 * u + 1] * a.scale;
                    if (row < r_end) {
                        if (n0 + 1 < G && (G & 1) == 0) {
                            *reinterpret_cast<float2 *>(lg + (int64_t)row * G + n0) = make_float2(x0, x1);
                            online_update(m[nt][0], sm[nt][0], x0);
                            online_update(m[nt][1], sm[nt][1], x1);
                        } else if (n0 + 1 < G) {
                            lg[(int64_t)row * G + n0] = x0;
                            lg[(int64_t)row * G + n0 + 1] = x1;
                            online_update(m[nt][0], sm[nt][0], x0);
                            online_update(m[nt][1], sm[nt][1], x1);
                        } else if (n0 < G) {
                            lg[(int64_t)row * G + n0] = x0;
                            online_update(m[nt][0], sm[nt][0], x0);
                        }
                    }
                }
            }
        }
        SKV_TRACE_REC(4, tr_wait);
        SKV_TRACE_REC_NOW(5);
        // reduce over the 8 lanes sharing j
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                float mm = m[nt][u], ss = sm[nt][u];
#pragma unroll
                for (int o = 4; o < 32; o <<= 1) {
                    const float m2 = __shfl_xor_sync(0xffffffffu, mm, o);
                    const float s2 = __shfl_xor_sync(0xffffffffu, ss, o);
                    merge_stats(mm, ss, m2, s2);
                }
                const int n = nt * 8 + 2 * j + u;
                if (g == 0 && n < 16) s_part[warp][n] = make_float2(mm, ss);
            }
        }
    }
    __syncthreads();
    if (s_abort && warp == ST_CONSUMERS && lane == 0) {
        // do not leave bulk copies in flight into this CTA's shared memory
        for (int s = 0; s < ST_STAGES; ++s) mbar_wait(&full[s], 0, 1u << 16), mbar_wait(&full[s], 1, 1u << 16);
    }
    if (tid < G) {
        float mm = -INFINITY, ss = 0.f;
        for (int w = 0; w < ST_CONSUMERS; ++w) merge_stats(mm, ss, s_part[w][tid].x, s_part[w][tid].y);
        a.part[((int64_t)bh * G + tid) * nsplit + split] = make_float2(mm, ss);  // [BH][G][nsplit]
    }
    SKV_TRACE_CTA(TR_SCORE_END);
    SKV_TRACE_REC_NOW(7);
    span_finish(a.span);
}

// ---------------------------------------------------------------------------
// Drop-in batch_gemm_softmax, kernel 1: D, per-256-column partial stats.
// grid = (ceil(n/256), batch), 256 threads; warp w covers rows 32w..32w+31.
// ---------------------------------------------------------------------------
template <int NT>
__global__ void __launch_bounds__(SC_THREADS) bgs_gemm_kernel(
    const __nv_bfloat16 *__restrict__ A, const __nv_bfloat16 *__restrict__ Bm,
    __nv_bfloat16 *__restrict__ D, float *__restrict__ Norm, float *__restrict__ Sum, int m, int n,
    float alpha)
{
    const int bt = blockIdx.y, blk = blockIdx.x, nblk = gridDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, j = lane & 3;
    const __nv_bfloat16 *qrows = A + (int64_t)bt * m * 128;
    const __nv_bfloat16 *lmh = Bm + (int64_t)bt * n * 128;
    __nv_bfloat16 *Db = D + (int64_t)bt * m * n;

    uint4 qf[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) load_q_frag(qf[nt], qrows, m, nt, lane);
    float mx[NT][2], sm[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) mx[nt][0] = mx[nt][1] = -INFINITY, sm[nt][0] = sm[nt][1] = 0.f;

    for (int t = 0; t < 2; ++t) {
        const int r0 = blk * 256 + warp * 32 + t * 16;
        const int rowa = r0 + g, rowb = r0 + g + 8;
        uint4 ra[4], rb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            ra[i] = rowa < n ? ld_nc_v4(lmh + (int64_t)rowa * 128 + (i * 4 + j) * 8) : make_uint4(0, 0, 0, 0);
            rb[i] = rowb < n ? ld_nc_v4(lmh + (int64_t)rowb * 128 + (i * 4 + j) * 8) : make_uint4(0, 0, 0, 0);
        }
        float acc[NT][4];
        tile_mma<NT>(acc, ra, rb, qf);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int row = u ? rowb : rowa;
                if (row >= n) continue;
#pragma unroll
                for (int v = 0; v < 2; ++v) {
                    const int mr = nt * 8 + 2 * j + v;
                    if (mr >= m) continue;
                    const float x = alpha * acc[nt][2 * u + v];
                    Db[(int64_t)mr * n + row] = f2bf(x);
                    online_update(mx[nt][v], sm[nt][v], x);
                }
            }
        }
    }
    __shared__ float2 s_part[SC_THREADS / 32][32];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int v = 0; v < 2; ++v) {
            float mm = mx[nt][v], ss = sm[nt][v];
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                const float m2 = __shfl_xor_sync(0xffffffffu, mm, o);
                const float s2 = __shfl_xor_sync(0xffffffffu, ss, o);
                merge_stats(mm, ss, m2, s2);
            }
            const int mr = nt * 8 + 2 * j + v;
            if (g == 0 && mr < 32) s_part[warp][mr] = make_float2(mm, ss);
        }
    }
    __syncthreads();
    if (threadIdx.x < m) {
        float mm = -INFINITY, ss = 0.f;
        for (int w = 0; w < SC_THREADS / 32; ++w) merge_stats(mm, ss, s_part[w][threadIdx.x].x, s_part[w][threadIdx.x].y);
        Norm[((int64_t)bt * nblk + blk) * m + threadIdx.x] = mm;
        Sum[((int64_t)bt * nblk + blk) * m + threadIdx.x] = ss;
    }
}

// kernel 2: final reduction into block 0 and the softmax of the bf16 D.
// grid = (m, batch), 256 threads.
__global__ void __launch_bounds__(256) bgs_softmax_kernel(const __nv_bfloat16 *__restrict__ D,
                                                          float *Norm, float *Sum,
                                                          __nv_bfloat16 *__restrict__ Soft, int m,
                                                          int n, int nblk)
{
    const int mr = blockIdx.x, bt = blockIdx.y;
    __shared__ float s_max, s_inv;
    if (threadIdx.x < 32) {
        float mm = -INFINITY, ss = 0.f;
        for (int i = threadIdx.x; i < nblk; i += 32)
            merge_stats(mm, ss, Norm[((int64_t)bt * nblk + i) * m + mr], Sum[((int64_t)bt * nblk + i) * m + mr]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float m2 = __shfl_xor_sync(0xffffffffu, mm, o);
            const float s2 = __shfl_xor_sync(0xffffffffu, ss, o);
            merge_stats(mm, ss, m2, s2);
        }
        if (threadIdx.x == 0) {
            s_max = mm;
            s_inv = 1.f / ss;
        }
    }
    __syncthreads();
    const float M = s_max, inv = s_inv;
    if (threadIdx.x == 0) {
        Norm[(int64_t)bt * nblk * m + mr] = M;
        Sum[(int64_t)bt * nblk * m + mr] = inv;
    }
    const __nv_bfloat16 *Dr = D + ((int64_t)bt * m + mr) * n;
    __nv_bfloat16 *Sr = Soft + ((int64_t)bt * m + mr) * n;
    for (int c = threadIdx.x; c < n; c += 256) Sr[c] = f2bf(__expf(bf2f(Dr[c]) - M) * inv);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct SelectPlan {
    int nsplit, rows_per_split;
    size_t off_logits, off_part, off_keys, off_kin, total;
    bool keys_global;
    bool keys_pre;  // long contexts: keys_kernel computes the keys on the whole GPU first
    int keys_rows;  // landmarks per keys_kernel CTA
    int cl;         // CTAs per selection cluster
    size_t sel_smem;
};

static SelectPlan plan_select(const skv_decode_geom *g)
{
    SelectPlan p = {};
    const int G = g->q_heads / g->kv_heads;
    const int BH = g->batch * g->kv_heads;
    const int sms_all = device_sm_count();
    const int tiles = ceil_div(g->num_landmarks, ST_ROWS);  // 128-row tiles per head
    // SMs left to the selection kernel that follows (programmatic dependent
    // launch): its CTAs become resident there while the scan runs and do the
    // work that does not need the scores (landmark ids, bitmaps, slots) early.
    // Two selection CTAs fit an SM; the scan keeps at least 3/4 of the SMs.
    // With the keys pass between them (very long contexts, below) the selection
    // cannot start during the scan, and the scan takes every SM.
    const bool keys_between = g->num_landmarks > 8 * 4096;
    const int sel_ctas = BH * (keys_between ? 16 : 8);
    const int reserve = keys_between ? 0 : min(ceil_div(sel_ctas, 2), sms_all / 4);
    const int sms = sms_all - reserve;
    // Scoring grid: two CTAs per SM on the SMs not reserved, the rows of a head
    // split evenly over nsplit of them (every SM reads about the same bytes).
    {
        const int ns = max(1, min(tiles, 2 * sms / BH));
        p.rows_per_split = ceil_div(g->num_landmarks, ns);
        p.nsplit = ceil_div(g->num_landmarks, p.rows_per_split);
    }
    // very long contexts (more than 4096 landmarks per CTA at 8): the keys are
    // computed by keys_kernel on the whole GPU (the selection's clusters would
    // spend long reading the logits) and the selection uses 16-CTA clusters
    const int L = g->num_landmarks;
    p.keys_pre = L > 8 * 4096;
    const int64_t kr = ((int64_t)L * BH + 2 * sms_all - 1) / (2 * sms_all);  // about two CTAs per SM
    p.keys_rows = kr < 512 ? 512 : (int)kr;
    p.cl = 8;
    if (p.keys_pre) {
        const bool kg16 = select_smem_bytes(L, g->num_chunks, G, false, 16, true) > SEL_SMEM_CAP;
        const size_t s16 = select_smem_bytes(L, g->num_chunks, G, kg16, 16, true);
        if (s16 <= SEL_SMEM_CAP && select_cluster16_ok(s16)) p.cl = 16;
    }
    p.keys_global = select_smem_bytes(L, g->num_chunks, G, false, p.cl, p.keys_pre) > SEL_SMEM_CAP;
    p.sel_smem = select_smem_bytes(L, g->num_chunks, G, p.keys_global, p.cl, p.keys_pre);
    auto align = [](size_t x) { return (x + 255) & ~(size_t)255; };
    p.off_logits = 0;
    p.off_part = align((size_t)BH * L * G * 4);
    p.off_keys = p.off_part + align((size_t)BH * p.nsplit * G * 8);
    // sized for the 8-CTA plan, whose key scratch is the larger: the size does
    // not depend on which cluster size the device allows
    const bool keys_global8 = select_smem_bytes(L, g->num_chunks, G, false, 8, p.keys_pre) > SEL_SMEM_CAP;
    p.off_kin = p.off_keys + (keys_global8 ? align((size_t)BH * L * 4) : 0);
    p.total = p.off_kin + (p.keys_pre ? align((size_t)BH * L * 4) : 0);
    return p;
}

static int check_geom(const skv_decode_geom *g)
{
    SKV_CHECK_ARG(g != nullptr, "null geometry");
    SKV_CHECK_ARG(g->batch > 0 && g->kv_heads > 0 && g->q_heads > 0, "sizes must be positive");
    SKV_CHECK_SUPPORTED(g->head_dim == 128 && g->chunk_size == 8, "head_dim 128 and chunk 8 only");
    SKV_CHECK_ARG(g->q_heads % g->kv_heads == 0, "q_heads must be a multiple of kv_heads");
    SKV_CHECK_SUPPORTED(g->q_heads / g->kv_heads <= 16, "GQA group larger than 16");
    SKV_CHECK_SUPPORTED(g->select_sets >= 1 && g->select_sets <= 1024, "select_sets outside 1..1024");
    SKV_CHECK_ARG(g->num_landmarks >= g->select_sets, "fewer landmarks than selected chunks");
    SKV_CHECK_ARG(g->num_chunks > 0 && g->num_chunks <= (1 << 21), "num_chunks outside 1..2M");
    return SKV_OK;
}

static int run_select(const skv_decode_geom *g, const ScoreArgs &sa_in, const int64_t *landmark_idx,
                      int32_t *slots, int32_t *miss_slot, int32_t *miss_chunk, int32_t *miss_count,
                      void *workspace, size_t workspace_bytes, bool append, cudaStream_t s,
                      const SelectArgs *fetch = nullptr, bool *fetched = nullptr, bool after_stage = false)
{
    if (fetched) *fetched = false;
    const SelectPlan p = plan_select(g);
    SKV_CHECK_ARG(workspace != nullptr && workspace_bytes >= p.total,
                  "workspace of %zu bytes needed, %zu given", p.total, workspace_bytes);
    SKV_CHECK_ARG(aligned(workspace, 256), "workspace must be 256-byte aligned");
    const int G = g->q_heads / g->kv_heads;
    const int BH = g->batch * g->kv_heads;
    unsigned char *ws = reinterpret_cast<unsigned char *>(workspace);
    ScoreArgs sa = sa_in;
    sa.logits = reinterpret_cast<float *>(ws + p.off_logits);
    sa.part = reinterpret_cast<float2 *>(ws + p.off_part);
    sa.Hkv = g->kv_heads;
    sa.G = G;
    sa.L = g->num_landmarks;
    sa.rows_per_split = p.rows_per_split;
    sa.scale = g->scale;
    sa.span = launch_spans().score;
    const void *fn = G <= 8 ? (append ? (const void *)score_tma_kernel<1, true> : (const void *)score_tma_kernel<1, false>)
                            : (append ? (const void *)score_tma_kernel<2, true> : (const void *)score_tma_kernel<2, false>);
    const int smem = ST_SMEM;
    int st = ensure_smem_attr(fn, smem, "score_tma_kernel");
    if (st) return st;
    void *kargs[] = {&sa};
    if (after_stage) {
        // programmatic dependent of the staging kernel: the landmark tiles are
        // requested before the kernel waits for the staged inputs (pdl_wait)
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(p.nsplit, BH, 1);
        cfg.blockDim = dim3(ST_THREADS, 1, 1);
        cfg.dynamicSmemBytes = (size_t)smem;
        cfg.stream = s;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        SKV_CUDA(cudaLaunchKernelExC(&cfg, fn, kargs));
    } else {
        SKV_CUDA(cudaLaunchKernel(fn, dim3(p.nsplit, BH), dim3(ST_THREADS), kargs, (size_t)smem, s));
    }
    st = check_launch("score_tma_kernel");
    if (st) return st;
    SelectArgs a = {};
    a.logits = sa.logits;
    a.part = sa.part;
    a.gkeys = p.keys_global ? reinterpret_cast<uint32_t *>(ws + p.off_keys) : nullptr;
    a.landmark_idx = landmark_idx;
    a.slots = slots;
    a.miss_slot = miss_slot;
    a.miss_chunk = miss_chunk;
    a.miss_count = miss_count;
    a.G = G, a.L = g->num_landmarks, a.K = g->select_sets, a.nsplit = p.nsplit;
    a.num_chunks = g->num_chunks;
    a.span = launch_spans().select;
    if (p.keys_pre) {
        KeysArgs k;
        k.logits = sa.logits;
        k.part = sa.part;
        k.keys = reinterpret_cast<uint32_t *>(ws + p.off_kin);
        k.G = G, k.L = g->num_landmarks, k.nsplit = p.nsplit, k.rows = p.keys_rows;
        st = launch_keys(k, BH, s);
        if (st) return st;
        a.keys_in = k.keys;
    }
    if (fetch && p.cl == SEL_CL && !p.keys_pre && !p.keys_global) {
        const FetchLayout f = fetch_layout(g->num_landmarks, g->num_chunks, G, g->select_sets, g->rank, g->buf_len);
        if (f.bytes) {
            a.v_host = fetch->v_host;
            a.U = fetch->U;
            a.SVt = fetch->SVt;
            a.cos_sin = fetch->cos_sin;
            a.k_buf = fetch->k_buf;
            a.v_buf = fetch->v_buf;
            a.Hkv = g->kv_heads;
            a.rank = g->rank;
            a.ctx = g->ctx_len;
            a.buf_len = g->buf_len;
            a.sparse_start = g->sparse_start;
            a.rope_mode = g->rope_mode;
            a.cs_stride = g->cos_sin_stride;
            a.cs_rows = g->cos_sin_rows;
            a.cap = f.cap;
            a.stage_off = f.stage_off;
            a.list_off = f.list_off;
            a.msg_off = f.msg_off;
            a.bmc_off = f.bmc_off;
            a.recon_off = f.recon_off;
            a.att_off = f.att_off;
            a.q_rot = fetch->q_rot;
            a.out = fetch->out;
            a.row_dev = fetch->row_dev;
            a.seq_len = fetch->seq_len;
            a.scale = g->scale;
            st = launch_select_fetch(a, BH, f.bytes, s);
            if (st == SKV_OK && fetched) *fetched = true;
            return st;
        }
    }
    return launch_select(a, BH, p.sel_smem, p.cl, s);
}

}  // namespace skv

using namespace skv;

extern "C" {

size_t skv_decode_select_workspace(const skv_decode_geom *g)
{
    if (check_geom(g) != SKV_OK) return 0;
    return plan_select(g).total;
}

int skv_decode_select_kernels(const skv_decode_geom *g)
{
    if (check_geom(g) != SKV_OK) return 0;
    return plan_select(g).keys_pre ? 3 : 2;
}

int skv_decode_select(const skv_decode_geom *g, const void *q, const void *landmarks,
                      const int64_t *landmark_idx, int32_t *slots, int32_t *miss_slot,
                      int32_t *miss_chunk, int32_t *miss_count, void *workspace,
                      size_t workspace_bytes, void *stream)
{
    int st = check_geom(g);
    if (st) return st;
    SKV_CHECK_ARG(q && landmarks && landmark_idx && slots && miss_slot && miss_chunk && miss_count,
                  "null pointer argument");
    SKV_CHECK_ARG(aligned(q, 16) && aligned(landmarks, 16), "q and landmarks must be 16-byte aligned");
    ScoreArgs sa = {};
    sa.q = (const __nv_bfloat16 *)q;
    sa.lm = (const __nv_bfloat16 *)landmarks;
    return run_select(g, sa, landmark_idx, slots, miss_slot, miss_chunk, miss_count, workspace, workspace_bytes,
                      false, (cudaStream_t)stream);
}

int skv_decode_append_select(const skv_decode_geom *g, const void *q, const void *k_new, const void *v_new,
                             const int64_t *positions, const void *cos_sin, void *q_out, void *k_buf,
                             void *v_buf, int row, const void *landmarks, const int64_t *landmark_idx,
                             int32_t *slots, int32_t *miss_slot, int32_t *miss_chunk, int32_t *miss_count,
                             void *workspace, size_t workspace_bytes, void *stream)
{
    return skv::append_select_launch(g, q, k_new, v_new, positions, cos_sin, q_out, k_buf, v_buf, row, landmarks,
                                     landmark_idx, slots, miss_slot, miss_chunk, miss_count, workspace,
                                     workspace_bytes, (cudaStream_t)stream, nullptr);
}

}  // extern "C"

namespace skv {

int append_select_launch(const skv_decode_geom *g, const void *q, const void *k_new, const void *v_new,
                         const int64_t *positions, const void *cos_sin, void *q_out, void *k_buf, void *v_buf,
                         int row, const void *landmarks, const int64_t *landmark_idx, int32_t *slots,
                         int32_t *miss_slot, int32_t *miss_chunk, int32_t *miss_count, void *workspace,
                         size_t workspace_bytes, cudaStream_t stream, const int32_t *row_dev,
                         const SelectArgs *fetch, bool *fetched, bool after_stage)
{
    int st = check_geom(g);
    if (st) return st;
    SKV_CHECK_ARG(q && k_new && v_new && positions && cos_sin && q_out && k_buf && v_buf && landmarks &&
                      landmark_idx && slots && miss_slot && miss_chunk && miss_count,
                  "null pointer argument");
    SKV_CHECK_SUPPORTED(g->rope_mode == 0 || g->rope_mode == 1, "rope_mode must be 0 or 1");
    SKV_CHECK_ARG(g->cos_sin_stride >= (g->rope_mode == 0 ? 128 : 64), "cos_sin_stride too small");
    SKV_CHECK_ARG(row >= 0 && row < g->buf_len, "append row %d outside the buffer", row);
    SKV_CHECK_ARG(aligned(q, 16) && aligned(landmarks, 16) && aligned(q_out, 16) && aligned(v_new, 16) &&
                      aligned(v_buf, 16) && aligned(k_new, 16) && aligned(cos_sin, 16) && g->cos_sin_stride % 8 == 0,
                  "q, q_out, k_new, v_new, v_buf, landmarks and cos_sin rows must be 16-byte aligned");
    ScoreArgs sa = {};
    sa.q = (const __nv_bfloat16 *)q;
    sa.lm = (const __nv_bfloat16 *)landmarks;
    sa.k_new = (const __nv_bfloat16 *)k_new;
    sa.v_new = (const __nv_bfloat16 *)v_new;
    sa.cos_sin = (const __nv_bfloat16 *)cos_sin;
    sa.positions = positions;
    sa.q_out = (__nv_bfloat16 *)q_out;
    sa.k_buf = (__nv_bfloat16 *)k_buf;
    sa.v_buf = (__nv_bfloat16 *)v_buf;
    sa.buf_len = g->buf_len;
    sa.row = row;
    sa.row_dev = row_dev;
    sa.rope_mode = g->rope_mode;
    sa.cs_stride = g->cos_sin_stride;
    sa.cs_rows = g->cos_sin_rows;
    return run_select(g, sa, landmark_idx, slots, miss_slot, miss_chunk, miss_count, workspace, workspace_bytes,
                      true, stream, fetch, fetched, after_stage);
}

}  // namespace skv

extern "C" {

int skv_batch_gemm_softmax(const void *A, const void *B, void *D, float *Norm, float *Sum,
                           void *Softmax, int batch_count, int m, int n, int k, float alpha,
                           float beta, void *stream)
{
    (void)beta;
    SKV_CHECK_ARG(A && B && D && Norm && Sum && Softmax, "null pointer argument");
    SKV_CHECK_ARG(batch_count > 0 && m > 0 && n > 0, "sizes must be positive");
    SKV_CHECK_SUPPORTED(k == 128, "k must be 128");
    SKV_CHECK_SUPPORTED(m <= 32, "m must be <= 32");
    SKV_CHECK_ARG(aligned(A, 16) && aligned(B, 16), "A and B must be 16-byte aligned");
    cudaStream_t s = (cudaStream_t)stream;
    const int nblk = ceil_div(n, 256);
    dim3 grid(nblk, batch_count);
    const int NT = ceil_div(m, 8);
    const __nv_bfloat16 *a = (const __nv_bfloat16 *)A, *b = (const __nv_bfloat16 *)B;
    __nv_bfloat16 *d = (__nv_bfloat16 *)D;
    if (NT == 1) bgs_gemm_kernel<1><<<grid, SC_THREADS, 0, s>>>(a, b, d, Norm, Sum, m, n, alpha);
    else if (NT == 2) bgs_gemm_kernel<2><<<grid, SC_THREADS, 0, s>>>(a, b, d, Norm, Sum, m, n, alpha);
    else bgs_gemm_kernel<4><<<grid, SC_THREADS, 0, s>>>(a, b, d, Norm, Sum, m, n, alpha);
    int st = check_launch("bgs_gemm_kernel");
    if (st) return st;
    bgs_softmax_kernel<<<dim3(m, batch_count), 256, 0, s>>>(d, Norm, Sum, (__nv_bfloat16 *)Softmax, m, n, nblk);
    return check_launch("bgs_softmax_kernel");
}

}  // extern "C"
