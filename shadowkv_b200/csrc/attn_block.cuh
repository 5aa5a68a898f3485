// One 128-row block of GQA decode attention, and the merge of a head's block
// partials.  Shared by the fused attention kernel and the early-fetch
// selection (which attends over the buffers once its values are in), so that
// both produce the same bits for a step.
//
// Reference: the attention of models/attention/shadow.py:48
// (flash_attn_with_kvcache over the K/V buffers, q_len = 1): out = softmax(q
// K^T * scale) V per query head; here per 128-row block the scores, the
// block's max m_j and weights P = exp(s - m_j) rounded to bf16, l_j = sum P and
// O_j = P V (fp32 accumulation), merged as sum_j e^{m_j - M} O_j / sum_j
// e^{m_j - M} l_j.
#pragma once

#include "recon.cuh"

namespace skv {

constexpr int AB_ROWS = 128;   // rows of a block
constexpr int AB_PITCH = 136;  // bf16 row pitch of the K / V / q / P tiles

// S = K q^T * scale of one block: warp w (of 8) scores keys 16w .. 16w+15
// against the 16 query rows of sQ (rows >= G zero); rows >= nrows get -inf.
// sK rows have pitch KT; sS is [128][16].  NT: n-tiles of query heads (1: G
// <= 8, 2: G <= 16).
template <int NT>
__device__ __forceinline__ void ab_scores(const __nv_bfloat16 *sK, int KT, const __nv_bfloat16 *sQ, float *sS,
                                          int nrows, float scale, int warp, int lane)
{
    float sc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
    const __nv_bfloat16 *aRow = sK + (warp * 16 + (lane & 15)) * KT + (lane >> 4) * 8;
    const int bRow = (lane & 7) + ((lane >> 4) << 3);
    const int bCol = ((lane >> 3) & 1) * 8;
#pragma unroll
    for (int kk = 0; kk < 128; kk += 16) {
        uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
        sa_ldsm(a0, a1, a2, a3, aRow + kk);
        sa_ldsm(b0, b1, b2, b3, sQ + bRow * AB_PITCH + kk + bCol);
        mma_bf16_16816(sc[0], a0, a1, a2, a3, b0, b1);
        if (NT == 2) mma_bf16_16816(sc[NT - 1], a0, a1, a2, a3, b2, b3);
    }
    const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int r0 = warp * 16 + g, r1 = r0 + 8;
        const int n0 = nt * 8 + 2 * t4;
        sS[r0 * 16 + n0] = r0 < nrows ? sc[nt][0] * scale : -INFINITY;
        sS[r0 * 16 + n0 + 1] = r0 < nrows ? sc[nt][1] * scale : -INFINITY;
        sS[r1 * 16 + n0] = r1 < nrows ? sc[nt][2] * scale : -INFINITY;
        sS[r1 * 16 + n0 + 1] = r1 < nrows ? sc[nt][3] * scale : -INFINITY;
    }
}

// Softmax of the block: warp w (of 8) handles heads w and w+8 (128 keys, 4 per
// lane); writes P (bf16) to sP [16][AB_PITCH], the block max to s_m and the
// sum of the rounded weights to s_l.  nrows >= 1.
__device__ __forceinline__ void ab_softmax(const float *sS, __nv_bfloat16 *sP, float *s_m, float *s_l, int G,
                                           int warp, int lane)
{
    for (int gg = warp; gg < 16; gg += 8) {
        if (gg < G) {
            float x[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) x[u] = sS[(lane + 32 * u) * 16 + gg];
            const float m = warp_max(fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3])));  // finite: nrows >= 1
            float psum = 0.f;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float p = x[u] == -INFINITY ? 0.f : __expf(x[u] - m);
                const __nv_bfloat16 pb = f2bf(p);
                sP[gg * AB_PITCH + lane + 32 * u] = pb;
                psum += bf2f(pb);  // the sum uses the same rounded weights as P V
            }
            psum = warp_sum(psum);
            if (lane == 0) {
                s_m[gg] = m;
                s_l[gg] = psum;
            }
        } else {
#pragma unroll
            for (int u = 0; u < 4; ++u) sP[gg * AB_PITCH + lane + 32 * u] = f2bf(0.f);
        }
    }
}

// O = P V of the block: warp w (of 8) computes dims 16w .. 16w+15 of the 16
// head rows; o[i] is n-tile i of the warp (rows g / g+8, columns 2 t4, +1).
__device__ __forceinline__ void ab_pv(const __nv_bfloat16 *sP, const __nv_bfloat16 *sV, float o[2][4], int warp,
                                      int lane)
{
#pragma unroll
    for (int i = 0; i < 2; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    const __nv_bfloat16 *aRow = sP + (lane & 15) * AB_PITCH + (lane >> 4) * 8;
    const int vRow = (lane & 7) + ((lane >> 3) & 1) * 8;
    const int vCol = warp * 16 + (lane >> 4) * 8;
#pragma unroll
    for (int kk = 0; kk < AB_ROWS; kk += 16) {
        uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
        sa_ldsm(a0, a1, a2, a3, aRow + kk);
        sa_ldsm_t(b0, b1, b2, b3, sV + (kk + vRow) * AB_PITCH + vCol);
        mma_bf16_16816(o[0], a0, a1, a2, a3, b0, b1);
        mma_bf16_16816(o[1], a0, a1, a2, a3, b2, b3);
    }
}

// The block's partial: O rows into po [G][128], (max, sum) of head g into pml[g]
// (pml written by threads tid < G of the block's 256).
__device__ __forceinline__ void ab_partial(const float o[2][4], float *po, float2 *pml, const float *s_m,
                                           const float *s_l, int G, int warp, int lane, int tid)
{
    const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int d = warp * 16 + i * 8 + 2 * t4;
        if (g < G) *reinterpret_cast<float2 *>(po + g * 128 + d) = make_float2(o[i][0], o[i][1]);
        if (g + 8 < G) *reinterpret_cast<float2 *>(po + (g + 8) * 128 + d) = make_float2(o[i][2], o[i][3]);
    }
    if (tid < G) pml[tid] = make_float2(s_m[tid], s_l[tid]);
}

// Merge of a head's nblk partials (po_head [nblk][G][128], ml [nblk][G]) by
// `nthreads` threads: each of the first G * 32 threads sums 4 columns of one
// query row over the partials, in partial order.  The (m, l) pairs are loaded
// and warp w turns those of heads w, w + nwarps, ... into weights
// w_j = exp(m_j - M) / L.  scratch: 2 nblk G floats of shared memory.
// stage (optional, 16-byte aligned shared memory of nblk G 512 bytes, free of
// other readers and writers): the partials are brought in by bulk copies on
// `bar` (an mbarrier of count 1 whose phase of parity `parity` is the next to
// complete), issued before the weights are computed, so that the sums wait
// for one transfer instead of a chain of loads.  The merge runs once per head
// and step, always from a cold instruction cache: its loops are kept rolled
// (fewer instructions to fetch).  emit(gg, d, pk) stores the 4 bf16 outputs
// (packed) of row gg, columns d .. d+3.
constexpr unsigned AB_STAGE_CHUNK = 32768;  // bytes per staging bulk copy
template <typename Emit>
__device__ __forceinline__ void ab_merge(const float *po_head, const float2 *ml, int nblk, int G, void *scratch,
                                         float *stage, uint64_t *bar, unsigned parity, int tid, int nthreads,
                                         Emit emit)
{
    const int lane = tid & 31, warp = tid >> 5, nwarps = nthreads / 32;
    const int nml = nblk * G;
    float2 *s_ml = reinterpret_cast<float2 *>(scratch);  // [nblk][G]
    float *s_w = reinterpret_cast<float *>(s_ml + nml);  // [nblk][G]
    if (stage && tid == 0) {
        const unsigned bytes = (unsigned)nml * 512u;
        fence_proxy_async_all();  // the generic accesses to this shared memory and the acquired partials come first
        mbar_arrive_expect_tx(bar, bytes);
#pragma unroll 1
        for (unsigned o = 0; o < bytes; o += AB_STAGE_CHUNK)
            bulk_g2s(reinterpret_cast<unsigned char *>(stage) + o, reinterpret_cast<const unsigned char *>(po_head) + o,
                     min(AB_STAGE_CHUNK, bytes - o), bar);
    }
#pragma unroll 1
    for (int t = tid; t < nml; t += nthreads) s_ml[t] = __ldcg(&ml[t]);
    __syncthreads();
#pragma unroll 1
    for (int gg = warp; gg < G; gg += nwarps) {
        float M = -INFINITY, L = 0.f;
#pragma unroll 1
        for (int j = lane; j < nblk; j += 32) M = fmaxf(M, s_ml[j * G + gg].x);
        M = warp_max(M);
#pragma unroll 1
        for (int j = lane; j < nblk; j += 32) L += s_ml[j * G + gg].y * __expf(s_ml[j * G + gg].x - M);
        L = warp_sum(L);
        const float inv = 1.f / L;
#pragma unroll 1
        for (int j = lane; j < nblk; j += 32) s_w[j * G + gg] = __expf(s_ml[j * G + gg].x - M) * inv;
    }
    if (stage && !mbar_wait(bar, parity)) {
        // a transfer that did not land in time is reported; the bytes in flight
        // must still land before the shared memory is read or reused
        if (tid == 0) report_dev_error(DEV_ERR_WAIT);
        mbar_wait(bar, parity);
    }
    __syncthreads();
#pragma unroll 1
    for (int p = tid; p < G * 32; p += nthreads) {
        const int gg = p >> 5, d = (p & 31) * 4;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        if (stage) {
            const float *po = stage + gg * 128 + d;
#pragma unroll 1
            for (int j = 0; j < nblk; ++j) {
                const float4 v = *reinterpret_cast<const float4 *>(po + j * G * 128);
                const float w = s_w[j * G + gg];
                acc.x = fmaf(v.x, w, acc.x), acc.y = fmaf(v.y, w, acc.y);
                acc.z = fmaf(v.z, w, acc.z), acc.w = fmaf(v.w, w, acc.w);
            }
        } else {
            const float *po = po_head + gg * 128 + d;
#pragma unroll 1
            for (int j = 0; j < nblk; ++j) {
                const float4 v = __ldcg(reinterpret_cast<const float4 *>(po + (int64_t)j * G * 128));
                const float w = s_w[j * G + gg];
                acc.x = fmaf(v.x, w, acc.x), acc.y = fmaf(v.y, w, acc.y);
                acc.z = fmaf(v.z, w, acc.z), acc.w = fmaf(v.w, w, acc.w);
            }
        }
        __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t *>(&lo);
        pk.y = *reinterpret_cast<uint32_t *>(&hi);
        emit(gg, d, pk);
    }
}

}  // namespace skv
