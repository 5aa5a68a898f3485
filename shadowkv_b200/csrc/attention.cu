// Split-K GQA decode attention over the K/V buffers of the selected budget.
//
// Replaces flash_attn_with_kvcache(q, k, v, causal=True) of
// models/attention/shadow.py:48 (flash-attn 2.7.4, q_len = 1, so causal has
// no effect) with repeat_kv GQA mapping (models/tensor_op.py:125-130):
// query head i attends with kv head i / G.
//
// One launch.  Each CTA takes 64 keys of one (b, kv head): V of the split is
// prefetched with cp.async, K rows are read straight into mma.sync fragments
// (the permuted-K trick of scoring.cu), the fp32 softmax partials and the
// P.V partial (fp32 FMAs against the shared-memory V tile) are written to the
// workspace.  The last CTA of a head to finish (atomic counter) merges the
// splits of that head and writes the bf16 output, then re-arms the counter.
#include "common.cuh"

namespace skv {

constexpr int AT_THREADS = 128;  // 4 warps
constexpr int AT_KPS = 64;       // keys per split (one 16-key mma tile per warp)

__device__ __forceinline__ uint32_t wsel_a(const uint4 &v, int w)
{
    return w == 0 ? v.x : (w == 1 ? v.y : (w == 2 ? v.z : v.w));
}

__device__ __forceinline__ void cp_async16_at(void *smem, const void *gmem)
{
    uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem));
}

template <int NT>
__global__ void __launch_bounds__(AT_THREADS) attn_kernel(
    const __nv_bfloat16 *__restrict__ q, const __nv_bfloat16 *__restrict__ kb,
    const __nv_bfloat16 *__restrict__ vb, float *__restrict__ part_o, float2 *__restrict__ part_ml,
    unsigned int *__restrict__ counters, __nv_bfloat16 *__restrict__ out, int Hkv, int G, int buf_len,
    int S, float scale)
{
    __shared__ __align__(16) __nv_bfloat16 sV[AT_KPS * 128];
    __shared__ __align__(16) float sP[AT_KPS * 16];
    __shared__ float s_m[16], s_l[16];
    __shared__ float s_w[1024];
    __shared__ bool s_last;

    const int split = blockIdx.x, nsplit = gridDim.x, bh = blockIdx.y;
    const int b = bh / Hkv, h = bh % Hkv;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, j = lane & 3;
    const int k0 = split * AT_KPS;
    const int nk = min(S - k0, AT_KPS);

    const __nv_bfloat16 *krows = kb + ((int64_t)bh * buf_len + k0) * 128;
    const __nv_bfloat16 *vrows = vb + ((int64_t)bh * buf_len + k0) * 128;

    for (int p = threadIdx.x; p < nk * 16; p += AT_THREADS)
        cp_async16_at(sV + (size_t)p * 8, vrows + (size_t)p * 8);
    asm volatile("cp.async.commit_group;" ::: "memory");

    // QK^T: warp w scores keys 16w .. 16w+15 for the G heads of the group
    {
        const __nv_bfloat16 *qrows = q + ((int64_t)b * Hkv * G + (int64_t)h * G) * 128;
        const int ra_i = warp * 16 + gq, rb_i = ra_i + 8;
        uint4 ra[4], rbv[4], qf[NT][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            ra[i] = ra_i < nk ? ld_nc_v4(krows + (int64_t)ra_i * 128 + (i * 4 + j) * 8) : make_uint4(0, 0, 0, 0);
            rbv[i] = rb_i < nk ? ld_nc_v4(krows + (int64_t)rb_i * 128 + (i * 4 + j) * 8) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int n = nt * 8 + gq;
#pragma unroll
            for (int i = 0; i < 4; ++i)
                qf[nt][i] = n < G ? ld_nc_v4(qrows + (int64_t)n * 128 + (i * 4 + j) * 8) : make_uint4(0, 0, 0, 0);
        }
        float acc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const int i = s >> 1, w = (s & 1) * 2;
            const uint32_t a0 = wsel_a(ra[i], w), a2 = wsel_a(ra[i], w + 1);
            const uint32_t a1 = wsel_a(rbv[i], w), a3 = wsel_a(rbv[i], w + 1);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
                mma_bf16_16816(acc[nt], a0, a1, a2, a3, wsel_a(qf[nt][i], w), wsel_a(qf[nt][i], w + 1));
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int n0 = nt * 8 + 2 * j;
            if (n0 < G) {
                sP[ra_i * 16 + n0] = ra_i < nk ? acc[nt][0] * scale : -INFINITY;
                sP[rb_i * 16 + n0] = rb_i < nk ? acc[nt][2] * scale : -INFINITY;
            }
            if (n0 + 1 < G) {
                sP[ra_i * 16 + n0 + 1] = ra_i < nk ? acc[nt][1] * scale : -INFINITY;
                sP[rb_i * 16 + n0 + 1] = rb_i < nk ? acc[nt][3] * scale : -INFINITY;
            }
        }
    }
    __syncthreads();

    // softmax partial per query head over the 64 keys (2 per lane)
    for (int gg = warp; gg < G; gg += 4) {
        const float x0 = sP[lane * 16 + gg], x1 = sP[(lane + 32) * 16 + gg];
        const float m = warp_max(fmaxf(x0, x1));
        const float p0 = x0 == -INFINITY ? 0.f : __expf(x0 - m);
        const float p1 = x1 == -INFINITY ? 0.f : __expf(x1 - m);
        sP[lane * 16 + gg] = p0;
        sP[(lane + 32) * 16 + gg] = p1;
        const float l = warp_sum(p0 + p1);
        if (lane == 0) {
            s_m[gg] = m;
            s_l[gg] = l;
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();

    // P.V: thread d owns output dim d for every head of the group
    const int d = threadIdx.x;
    float acc[16];
#pragma unroll
    for (int gg = 0; gg < 16; ++gg) acc[gg] = 0.f;
    for (int kk = 0; kk < nk; ++kk) {
        const float v = bf2f(sV[kk * 128 + d]);
        const float4 *pr = reinterpret_cast<const float4 *>(sP + kk * 16);
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
            if (q4 * 4 < G) {
                const float4 p = pr[q4];
                acc[q4 * 4 + 0] = fmaf(p.x, v, acc[q4 * 4 + 0]);
                acc[q4 * 4 + 1] = fmaf(p.y, v, acc[q4 * 4 + 1]);
                acc[q4 * 4 + 2] = fmaf(p.z, v, acc[q4 * 4 + 2]);
                acc[q4 * 4 + 3] = fmaf(p.w, v, acc[q4 * 4 + 3]);
            }
        }
    }
    float *po = part_o + (((int64_t)bh * nsplit + split) * G) * 128;
#pragma unroll
    for (int gg = 0; gg < 16; ++gg)
        if (gg < G) __stcg(po + (int64_t)gg * 128 + d, acc[gg]);
    if (threadIdx.x < G)
        __stcg(part_ml + ((int64_t)bh * nsplit + split) * G + threadIdx.x, make_float2(s_m[threadIdx.x], s_l[threadIdx.x]));

    // the last split of this head to arrive merges all splits
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&counters[bh], 1u) == (unsigned)(nsplit - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int gg = 0; gg < G; ++gg) {
        if (warp == 0) {
            float M = -INFINITY;
            for (int i = lane; i < nsplit; i += 32) M = fmaxf(M, __ldcg(&part_ml[((int64_t)bh * nsplit + i) * G + gg].x));
            M = warp_max(M);
            float Ls = 0.f;
            for (int i = lane; i < nsplit; i += 32) {
                const float2 ml = __ldcg(&part_ml[((int64_t)bh * nsplit + i) * G + gg]);
                const float w = ml.x == -INFINITY ? 0.f : __expf(ml.x - M);
                s_w[i] = w;
                Ls += ml.y * w;
            }
            Ls = warp_sum(Ls);
            if (lane == 0) s_l[gg] = 1.f / Ls;
        }
        __syncthreads();
        float o = 0.f;
        for (int i = 0; i < nsplit; ++i)
            o = fmaf(__ldcg(part_o + (((int64_t)bh * nsplit + i) * G + gg) * 128 + d), s_w[i], o);
        out[((int64_t)bh * G + gg) * 128 + d] = f2bf(o * s_l[gg]);
        __syncthreads();
    }
    if (threadIdx.x == 0) counters[bh] = 0;  // re-arm for the next call
}

struct AttnPlan {
    int nsplit;
    size_t off_o, off_ml, off_cnt, total;
};

static AttnPlan plan_attn(const skv_decode_geom *g, int S)
{
    AttnPlan p = {};
    const int BH = g->batch * g->kv_heads;
    const int G = g->q_heads / g->kv_heads;
    p.nsplit = ceil_div(S, AT_KPS);
    auto align = [](size_t x) { return (x + 255) & ~(size_t)255; };
    p.off_cnt = 0;
    p.off_o = align((size_t)BH * 4);
    p.off_ml = p.off_o + align((size_t)BH * p.nsplit * G * 128 * 4);
    p.total = p.off_ml + align((size_t)BH * p.nsplit * G * 8);
    return p;
}

}  // namespace skv

using namespace skv;

extern "C" {

size_t skv_decode_attention_workspace(const skv_decode_geom *g, int seq_len)
{
    if (!g || seq_len <= 0 || g->kv_heads <= 0 || g->batch <= 0) return 0;
    if (seq_len > 1024 * AT_KPS) return 0;
    return plan_attn(g, seq_len).total;
}

int skv_decode_attention(const skv_decode_geom *g, const void *q, const void *k_buf,
                         const void *v_buf, int seq_len, void *out, void *workspace,
                         size_t workspace_bytes, void *stream)
{
    SKV_CHECK_ARG(g && q && k_buf && v_buf && out, "null pointer argument");
    SKV_CHECK_ARG(g->batch > 0 && g->kv_heads > 0 && g->q_heads % g->kv_heads == 0, "bad head counts");
    SKV_CHECK_SUPPORTED(g->head_dim == 128, "head_dim must be 128");
    const int G = g->q_heads / g->kv_heads;
    SKV_CHECK_SUPPORTED(G <= 16, "GQA group larger than 16");
    SKV_CHECK_ARG(seq_len > 0 && seq_len <= g->buf_len, "seq_len %d outside 1..buf_len", seq_len);
    SKV_CHECK_SUPPORTED(seq_len <= 1024 * AT_KPS, "seq_len above %d", 1024 * AT_KPS);
    SKV_CHECK_ARG(aligned(q, 16) && aligned(k_buf, 16) && aligned(v_buf, 16), "operands must be 16-byte aligned");
    const AttnPlan p = plan_attn(g, seq_len);
    SKV_CHECK_ARG(workspace && workspace_bytes >= p.total, "workspace of %zu bytes needed, %zu given",
                  p.total, workspace_bytes);
    SKV_CHECK_ARG(aligned(workspace, 256), "workspace must be 256-byte aligned");
    cudaStream_t s = (cudaStream_t)stream;
    unsigned char *ws = reinterpret_cast<unsigned char *>(workspace);
    unsigned int *cnt = reinterpret_cast<unsigned int *>(ws + p.off_cnt);
    float *po = reinterpret_cast<float *>(ws + p.off_o);
    float2 *pml = reinterpret_cast<float2 *>(ws + p.off_ml);
    const int BH = g->batch * g->kv_heads;
    dim3 grid(p.nsplit, BH);
    if (G <= 8)
        attn_kernel<1><<<grid, AT_THREADS, 0, s>>>((const __nv_bfloat16 *)q, (const __nv_bfloat16 *)k_buf,
                                                   (const __nv_bfloat16 *)v_buf, po, pml, cnt,
                                                   (__nv_bfloat16 *)out, g->kv_heads, G, g->buf_len, seq_len,
                                                   g->scale);
    else
        attn_kernel<2><<<grid, AT_THREADS, 0, s>>>((const __nv_bfloat16 *)q, (const __nv_bfloat16 *)k_buf,
                                                   (const __nv_bfloat16 *)v_buf, po, pml, cnt,
                                                   (__nv_bfloat16 *)out, g->kv_heads, G, g->buf_len, seq_len,
                                                   g->scale);
    return check_launch("attn_kernel");
}

}  // extern "C"
