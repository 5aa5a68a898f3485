// Low-rank key reconstruction of 16 rows by one warp: U rows x SV^T on
// mma.sync, RoPE on the fp32 accumulators, one rounding to bf16.  Shared by the
// fused attention kernel and the early-fetch selection, so that both write the
// same key bits for a chunk.
//
// Reference: kernels/batch_gather_gemm.cu:136-213 (the gathered GEMM) and
// kernels/rope_new.cu:224-374 (the RoPE of its output); the reference rounds
// the GEMM to bf16 and rotates in bf16 op by op, this rotates the fp32
// accumulators and rounds once.
#pragma once

#include "common.cuh"

namespace skv {

__device__ __forceinline__ void sa_ldsm(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, const void *p)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void sa_ldsm_t(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, const void *p)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(smem_u32(p)));
}

// acc[i] = n-tile (i < 4 ? 4 half + i : 8 + 4 half + i - 4) of the product of
// the warp's 16 U rows (aRow: this lane's ldmatrix row pointer, k = 0) with
// SV^T (sB: 128 rows of pitch KP).  The n-tiles {4h .. 4h+3} and
// {8+4h .. 8+4h+3} keep the rotate-half pairs (t, t+64) of a row in one thread.
__device__ __forceinline__ void recon_half(float acc[8][4], const __nv_bfloat16 *aRow, const __nv_bfloat16 *sB,
                                           int KP, int rank, int half, int lane)
{
    const int bColOff = ((lane >> 3) & 1) * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    for (int k0 = 0; k0 < rank; k0 += 16) {
        uint32_t a0, a1, a2, a3;
        sa_ldsm(a0, a1, a2, a3, aRow + k0);
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {
            // one x4 ldmatrix: SV^T rows of n-tile (4h + pr) for lanes 0-15 and of
            // n-tile (8 + 4h + pr) for lanes 16-31, k halves by lane bit 3
            const int ntA = 4 * half + pr, ntB = 8 + 4 * half + pr;
            const int rsel = (lane & 7) + ((lane >> 4) ? ntB * 8 : ntA * 8);
            uint32_t b0, b1, b2, b3;
            sa_ldsm(b0, b1, b2, b3, sB + rsel * KP + k0 + bColOff);
            mma_bf16_16816(acc[pr], a0, a1, a2, a3, b0, b1);
            mma_bf16_16816(acc[4 + pr], a0, a1, a2, a3, b2, b3);
        }
    }
}

// RoPE of one row's values of one half (v[i][u]: n-tile as in recon_half,
// column 2 t4 + u) with that row's cos/sin (cs: 64 cos then 64 sin, or the GLM
// table's 32 cos then 32 sin).
__device__ __forceinline__ void recon_rope(float v[8][2], const __nv_bfloat16 *cs, int rope_mode, int half, int t4)
{
    if (rope_mode == 0) {
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int t = (4 * half + pr) * 8 + t4 * 2 + u;  // < 64
                const float cc = bf2f(cs[t]), ss = bf2f(cs[t + 64]);
                const float x1 = v[pr][u], x2 = v[4 + pr][u];
                v[pr][u] = x1 * cc - x2 * ss;
                v[4 + pr][u] = x2 * cc + x1 * ss;
            }
        }
    } else {
        // GLM: pairs (2i, 2i+1) of the first 64 dims, both in one thread
#pragma unroll
        for (int pr = 0; pr < 4; ++pr) {
            const int tp = ((4 * half + pr) * 8 + t4 * 2) >> 1;  // pair index < 32
            const float cc = bf2f(cs[tp]), ss = bf2f(cs[tp + 32]);
            const float xe = v[pr][0], xo = v[pr][1];
            v[pr][0] = xe * cc - xo * ss;
            v[pr][1] = xo * cc + xe * ss;
        }
    }
}

// Column of packed pair i of a row (n-tile order of recon_half).
__device__ __forceinline__ int recon_col(int half, int i, int t4)
{
    const int nt = i < 4 ? 4 * half + i : 8 + 4 * half + (i - 4);
    return nt * 8 + t4 * 2;
}

}  // namespace skv
