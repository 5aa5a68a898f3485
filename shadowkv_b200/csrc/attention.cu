// Split-K GQA decode attention over the K/V buffers of the selected budget.
//
// Replaces flash_attn_with_kvcache(q, k, v, causal=True) of
// models/attention/shadow.py:48 (flash-attn 2.7.4, q_len = 1, so causal has
// no effect) with repeat_kv GQA mapping (models/tensor_op.py:125-130):
// query head i attends with kv head i / G.
//
// One launch, one 8-CTA thread-block cluster per (b, kv head).  The CTAs of
// a cluster split the keys.  Each CTA walks its keys in tiles of up to 128:
// the K and V rows of the next tile are in flight (cp.async, double
// buffered) while the current tile is computed.  Both products run on the
// tensor cores: S = K q^T with the keys as the M dimension, then
// O += P V with the (padded to 16) query heads of the group as M, P in bf16
// as flash-attention does.  An online softmax keeps the running max / sum
// per head.  The partials stay in shared memory; after a cluster barrier
// rank 0 merges them through distributed shared memory.  No global scratch.
#include "common.cuh"

namespace skv {

constexpr int AT_THREADS = 256;            // 8 warps
constexpr int AT_CL = 8;                   // CTAs per (b, kv head)
constexpr int AT_TILE = 128;               // keys per tile: 16 per warp in QK^T
constexpr int AT_PITCH = 136;              // padded row pitch (bf16) of K, V, q, P tiles
constexpr int AT_SMEM = (2 * 2 * AT_TILE * AT_PITCH + 16 * AT_PITCH + 16 * AT_PITCH) * 2  // K,V x2, q, P
                        + AT_TILE * 16 * 4;                                                // fp32 logits

__device__ __forceinline__ void cp_async16_at(void *smem, const void *gmem)
{
    uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void ldsm_x4(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, const void *p)
{
    uint32_t s = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(s));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3, const void *p)
{
    uint32_t s = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(s));
}
__device__ __forceinline__ void cluster_sync_all()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n"
                 "barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ float ld_dsmem_f32(const float *local, unsigned rank)
{
    uint32_t a = (uint32_t)__cvta_generic_to_shared(local), r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(r) : "memory");
    return v;
}

// NT = n-tiles of query heads in S = K q^T (1: G <= 8, 2: G <= 16)
template <int NT>
__global__ void __launch_bounds__(AT_THREADS) attn_kernel(
    const __nv_bfloat16 *__restrict__ q, const __nv_bfloat16 *__restrict__ kb,
    const __nv_bfloat16 *__restrict__ vb, __nv_bfloat16 *__restrict__ out, int Hkv, int G, int buf_len,
    int S, int keys_per_cta, float scale)
{
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __nv_bfloat16 *sK = reinterpret_cast<__nv_bfloat16 *>(smem_raw);  // [2][AT_TILE][AT_PITCH]
    __nv_bfloat16 *sV = sK + 2 * AT_TILE * AT_PITCH;                    // [2][AT_TILE][AT_PITCH]
    __nv_bfloat16 *sQ = sV + 2 * AT_TILE * AT_PITCH;                    // [16][AT_PITCH]
    __nv_bfloat16 *sPb = sQ + 16 * AT_PITCH;                            // [16 heads][AT_PITCH] probabilities
    float *sS = reinterpret_cast<float *>(sPb + 16 * AT_PITCH);        // [AT_TILE][16] logits
    __shared__ float s_alpha[16], s_m[16], s_l[16];
    __shared__ __align__(16) float s_acc[16 * 128];                   // per-head partial output (DSMEM-read)

    const unsigned rank = blockIdx.x;
    const int bh = blockIdx.y;
    const int b = bh / Hkv, h = bh % Hkv;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gq = lane >> 2, t4 = lane & 3;
    const int kbeg = (int)rank * keys_per_cta;
    const int kend = min(S, kbeg + keys_per_cta);
    const int ntiles = kend > kbeg ? (kend - kbeg + AT_TILE - 1) / AT_TILE : 0;
    const __nv_bfloat16 *kbase = kb + ((int64_t)bh * buf_len) * 128;
    const __nv_bfloat16 *vbase = vb + ((int64_t)bh * buf_len) * 128;

    auto stage = [&](int t) {
        const int k0 = kbeg + t * AT_TILE;
        const int nk = min(kend - k0, AT_TILE);
        __nv_bfloat16 *dk = sK + (t & 1) * AT_TILE * AT_PITCH;
        __nv_bfloat16 *dv = sV + (t & 1) * AT_TILE * AT_PITCH;
        for (int p = tid; p < nk * 16; p += AT_THREADS) {
            const int r = p >> 4, c = (p & 15) * 8;
            cp_async16_at(dk + r * AT_PITCH + c, kbase + (int64_t)(k0 + r) * 128 + c);
            cp_async16_at(dv + r * AT_PITCH + c, vbase + (int64_t)(k0 + r) * 128 + c);
        }
        // rows past the end of the keys are zero so the tensor-core tiles stay finite
        for (int p = tid; p < (AT_TILE - nk) * 16; p += AT_THREADS) {
            const int r = nk + (p >> 4), c = (p & 15) * 8;
            *reinterpret_cast<uint4 *>(dk + r * AT_PITCH + c) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4 *>(dv + r * AT_PITCH + c) = make_uint4(0, 0, 0, 0);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    if (ntiles > 0) stage(0);
    // q of the group (rows >= G are zero) and the running statistics
    {
        const __nv_bfloat16 *qrows = q + ((int64_t)b * Hkv * G + (int64_t)h * G) * 128;
        for (int p = tid; p < 16 * 16; p += AT_THREADS) {
            const int r = p >> 4, c = (p & 15) * 8;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (r < G) v = ld_nc_v4(qrows + (int64_t)r * 128 + c);
            *reinterpret_cast<uint4 *>(sQ + r * AT_PITCH + c) = v;
        }
        if (tid < 16) {
            s_m[tid] = -INFINITY;
            s_l[tid] = 0.f;
        }
    }
    // output accumulator: warp w owns dims 16w .. 16w+15 (two n-tiles), rows = heads
    float oacc[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.f;

    for (int t = 0; t < ntiles; ++t) {
        const int k0 = kbeg + t * AT_TILE;
        const int nk = min(kend - k0, AT_TILE);
        if (t + 1 < ntiles) {
            stage(t + 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const __nv_bfloat16 *tk = sK + (t & 1) * AT_TILE * AT_PITCH;
        const __nv_bfloat16 *tv = sV + (t & 1) * AT_TILE * AT_PITCH;

        // ---- S = K q^T: warp w scores keys 16w .. 16w+15
        {
            float sc[NT][4];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
            const __nv_bfloat16 *aRow = tk + (warp * 16 + (lane & 15)) * AT_PITCH + (lane >> 4) * 8;
            const int bRow = (lane & 7) + ((lane >> 4) << 3);
            const int bCol = ((lane >> 3) & 1) * 8;
#pragma unroll
            for (int kk = 0; kk < 128; kk += 16) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4(a0, a1, a2, a3, aRow + kk);
                if (NT == 1) {
                    uint32_t b0, b1, b2, b3;  // heads 0..7 (b0,b1) and 8..15 (b2,b3) -- only 0..7 used
                    ldsm_x4(b0, b1, b2, b3, sQ + bRow * AT_PITCH + kk + bCol);
                    mma_bf16_16816(sc[0], a0, a1, a2, a3, b0, b1);
                } else {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(b0, b1, b2, b3, sQ + bRow * AT_PITCH + kk + bCol);
                    mma_bf16_16816(sc[0], a0, a1, a2, a3, b0, b1);
                    mma_bf16_16816(sc[NT - 1], a0, a1, a2, a3, b2, b3);
                }
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int r0 = warp * 16 + gq, r1 = r0 + 8;
                const int n0 = nt * 8 + 2 * t4;
                sS[r0 * 16 + n0] = r0 < nk ? sc[nt][0] * scale : -INFINITY;
                sS[r0 * 16 + n0 + 1] = r0 < nk ? sc[nt][1] * scale : -INFINITY;
                sS[r1 * 16 + n0] = r1 < nk ? sc[nt][2] * scale : -INFINITY;
                sS[r1 * 16 + n0 + 1] = r1 < nk ? sc[nt][3] * scale : -INFINITY;
            }
        }
        __syncthreads();
        // ---- online softmax: warp w updates heads w and w+8 (128 keys, 4 per lane)
        for (int gg = warp; gg < 16; gg += 8) {
            if (gg < G) {
                float x[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) x[u] = sS[(lane + 32 * u) * 16 + gg];
                const float m_old = s_m[gg];
                const float m_new = fmaxf(m_old, warp_max(fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]))));
                float psum = 0.f;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float p = x[u] == -INFINITY ? 0.f : __expf(x[u] - m_new);
                    const __nv_bfloat16 pb = f2bf(p);
                    sPb[gg * AT_PITCH + lane + 32 * u] = pb;
                    psum += bf2f(pb);  // the sum uses the same rounded weights as P.V
                }
                psum = warp_sum(psum);
                __syncwarp();
                if (lane == 0) {
                    const float alpha = m_old == -INFINITY ? 0.f : __expf(m_old - m_new);
                    s_alpha[gg] = alpha;
                    s_m[gg] = m_new;
                    s_l[gg] = s_l[gg] * alpha + psum;
                }
            } else {
                // padded head rows of P stay zero
#pragma unroll
                for (int u = 0; u < 4; ++u) sPb[gg * AT_PITCH + lane + 32 * u] = f2bf(0.f);
                if (lane == 0) s_alpha[gg] = 0.f;
            }
        }
        __syncthreads();
        // ---- O = alpha * O + P V: warp w computes dims 16w .. 16w+15 for all 16 head rows
        {
            const float al0 = s_alpha[gq], al1 = s_alpha[gq + 8];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                oacc[i][0] *= al0;
                oacc[i][1] *= al0;
                oacc[i][2] *= al1;
                oacc[i][3] *= al1;
            }
            const __nv_bfloat16 *aRow = sPb + (lane & 15) * AT_PITCH + (lane >> 4) * 8;
            const int vRow = (lane & 7) + ((lane >> 3) & 1) * 8;
            const int vCol = warp * 16 + (lane >> 4) * 8;
#pragma unroll
            for (int kk = 0; kk < AT_TILE; kk += 16) {
                uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
                ldsm_x4(a0, a1, a2, a3, aRow + kk);
                ldsm_x4_t(b0, b1, b2, b3, tv + (kk + vRow) * AT_PITCH + vCol);
                mma_bf16_16816(oacc[0], a0, a1, a2, a3, b0, b1);
                mma_bf16_16816(oacc[1], a0, a1, a2, a3, b2, b3);
            }
        }
        __syncthreads();  // tile buffers and P are rewritten by the next iteration
    }

    // ---- publish this CTA's partial output, then rank 0 merges the cluster
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int dcol = warp * 16 + i * 8 + 2 * t4;
        s_acc[gq * 128 + dcol] = oacc[i][0];
        s_acc[gq * 128 + dcol + 1] = oacc[i][1];
        s_acc[(gq + 8) * 128 + dcol] = oacc[i][2];
        s_acc[(gq + 8) * 128 + dcol + 1] = oacc[i][3];
    }
    cluster_sync_all();
    if (rank == 0) {
        for (int p = tid; p < G * 128; p += AT_THREADS) {
            const int gg = p >> 7, d = p & 127;
            float mr[AT_CL], lr[AT_CL], ar[AT_CL];
            float M = -INFINITY;
#pragma unroll
            for (unsigned r = 0; r < AT_CL; ++r) {
                mr[r] = ld_dsmem_f32(&s_m[gg], r);
                lr[r] = ld_dsmem_f32(&s_l[gg], r);
                ar[r] = ld_dsmem_f32(&s_acc[gg * 128 + d], r);
                M = fmaxf(M, mr[r]);
            }
            float L = 0.f, o = 0.f;
#pragma unroll
            for (unsigned r = 0; r < AT_CL; ++r) {
                const float w = mr[r] == -INFINITY ? 0.f : __expf(mr[r] - M);
                L += lr[r] * w;
                o += ar[r] * w;
            }
            out[((int64_t)bh * G + gg) * 128 + d] = f2bf(o / L);
        }
    }
    cluster_sync_all();  // keep every CTA's shared memory alive until rank 0 is done
}

}  // namespace skv

using namespace skv;

extern "C" {

size_t skv_decode_attention_workspace(const skv_decode_geom *g, int seq_len)
{
    (void)g;
    (void)seq_len;
    return 0;  // partials live in shared memory
}

int skv_decode_attention(const skv_decode_geom *g, const void *q, const void *k_buf,
                         const void *v_buf, int seq_len, void *out, void *workspace,
                         size_t workspace_bytes, void *stream)
{
    (void)workspace;
    (void)workspace_bytes;
    SKV_CHECK_ARG(g && q && k_buf && v_buf && out, "null pointer argument");
    SKV_CHECK_ARG(g->batch > 0 && g->kv_heads > 0 && g->q_heads % g->kv_heads == 0, "bad head counts");
    SKV_CHECK_SUPPORTED(g->head_dim == 128, "head_dim must be 128");
    const int G = g->q_heads / g->kv_heads;
    SKV_CHECK_SUPPORTED(G <= 16, "GQA group larger than 16");
    SKV_CHECK_ARG(seq_len > 0 && seq_len <= g->buf_len, "seq_len %d outside 1..buf_len", seq_len);
    SKV_CHECK_ARG(aligned(q, 16) && aligned(k_buf, 16) && aligned(v_buf, 16), "operands must be 16-byte aligned");
    const int keys_per_cta = 16 * ceil_div(ceil_div(seq_len, AT_CL), 16);
    const void *fn = G <= 8 ? (const void *)attn_kernel<1> : (const void *)attn_kernel<2>;
    int st = ensure_smem_attr(fn, AT_SMEM, "attn_kernel");
    if (st) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(AT_CL, g->batch * g->kv_heads, 1);
    cfg.blockDim = dim3(AT_THREADS, 1, 1);
    cfg.dynamicSmemBytes = AT_SMEM;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = AT_CL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const __nv_bfloat16 *qq = (const __nv_bfloat16 *)q, *kk = (const __nv_bfloat16 *)k_buf,
                        *vv = (const __nv_bfloat16 *)v_buf;
    __nv_bfloat16 *oo = (__nv_bfloat16 *)out;
    cudaError_t e;
    if (G <= 8)
        e = cudaLaunchKernelEx(&cfg, attn_kernel<1>, qq, kk, vv, oo, g->kv_heads, G, g->buf_len, seq_len,
                               keys_per_cta, g->scale);
    else
        e = cudaLaunchKernelEx(&cfg, attn_kernel<2>, qq, kk, vv, oo, g->kv_heads, G, g->buf_len, seq_len,
                               keys_per_cta, g->scale);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("launch of attn_kernel failed: %s", cudaGetErrorString(e));
        return SKV_ERR_CUDA;
    }
    return SKV_OK;
}

}  // extern "C"
