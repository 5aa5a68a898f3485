// Split-K GQA decode attention over the K/V buffers of the selected budget.
//
// Replaces flash_attn_with_kvcache(q, k, v, causal=True) of
// models/attention/shadow.py:48 (flash-attn 2.7.4, q_len = 1, so causal has
// no effect) with repeat_kv GQA mapping (models/tensor_op.py:125-130):
// query head i attends with kv head i / G.
//
// Kernel 1: one CTA per (split of keys, b, kv head).  QK^T on mma.sync with
// the permuted-K fragment loads of scoring.cu (K rows read straight from
// global memory), exact fp32 softmax partials, P.V with fp32 FMAs against a
// V tile staged by cp.async.  Kernel 2 merges the splits.
#include "common.cuh"

namespace skv {

constexpr int AT_THREADS = 128;  // 4 warps

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
__global__ void __launch_bounds__(AT_THREADS) attn_split_kernel(
    const __nv_bfloat16 *__restrict__ q, const __nv_bfloat16 *__restrict__ kb,
    const __nv_bfloat16 *__restrict__ vb, float *__restrict__ part_o, float2 *__restrict__ part_ml,
    int Hkv, int G, int buf_len, int S, int kps, float scale)
{
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int split = blockIdx.x, nsplit = gridDim.x, bh = blockIdx.y;
    const int b = bh / Hkv, h = bh % Hkv;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, j = lane & 3;
    const int k0 = split * kps;
    const int k1 = min(S, k0 + kps);
    const int nk = k1 - k0;

    __nv_bfloat16 *sV = reinterpret_cast<__nv_bfloat16 *>(smem_raw);   // [kps][128]
    float *sP = reinterpret_cast<float *>(sV + (size_t)kps * 128);     // [kps][G]
    __shared__ float s_m[16], s_l[16];

    const __nv_bfloat16 *krows = kb + ((int64_t)bh * buf_len + k0) * 128;
    const __nv_bfloat16 *vrows = vb + ((int64_t)bh * buf_len + k0) * 128;

    // stage V of the split (overlaps with QK^T)
    for (int p = threadIdx.x; p < nk * 16; p += AT_THREADS)
        cp_async16_at(sV + (size_t)p * 8, vrows + (size_t)p * 8);
    asm volatile("cp.async.commit_group;" ::: "memory");

    // q fragments of the group
    const __nv_bfloat16 *qrows = q + ((int64_t)b * Hkv * G + (int64_t)h * G) * 128;
    uint4 qf[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int n = nt * 8 + gq;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            qf[nt][i] = n < G ? ld_nc_v4(qrows + (int64_t)n * 128 + (i * 4 + j) * 8) : make_uint4(0, 0, 0, 0);
    }

    // logits of 16-key tiles
    for (int r0 = warp * 16; r0 < nk; r0 += 64) {
        const int ra_i = r0 + gq, rb_i = r0 + gq + 8;
        uint4 ra[4], rbv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            ra[i] = ra_i < nk ? ld_nc_v4(krows + (int64_t)ra_i * 128 + (i * 4 + j) * 8) : make_uint4(0, 0, 0, 0);
            rbv[i] = rb_i < nk ? ld_nc_v4(krows + (int64_t)rb_i * 128 + (i * 4 + j) * 8) : make_uint4(0, 0, 0, 0);
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
            if (ra_i < nk) {
                if (n0 < G) sP[ra_i * G + n0] = acc[nt][0] * scale;
                if (n0 + 1 < G) sP[ra_i * G + n0 + 1] = acc[nt][1] * scale;
            }
            if (rb_i < nk) {
                if (n0 < G) sP[rb_i * G + n0] = acc[nt][2] * scale;
                if (n0 + 1 < G) sP[rb_i * G + n0 + 1] = acc[nt][3] * scale;
            }
        }
    }
    __syncthreads();

    // softmax partials per query head (warp w handles heads w, w+4, ...)
    for (int gg = warp; gg < G; gg += 4) {
        float m = -INFINITY;
        for (int kk = lane; kk < nk; kk += 32) m = fmaxf(m, sP[kk * G + gg]);
        m = warp_max(m);
        float l = 0.f;
        for (int kk = lane; kk < nk; kk += 32) {
            const float p = __expf(sP[kk * G + gg] - m);
            sP[kk * G + gg] = p;
            l += p;
        }
        l = warp_sum(l);
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
        const float v = bf2f(sV[(size_t)kk * 128 + d]);
        const float *pr = sP + kk * G;
#pragma unroll
        for (int gg = 0; gg < 16; ++gg)
            if (gg < G) acc[gg] = fmaf(pr[gg], v, acc[gg]);
    }
    float *po = part_o + (((int64_t)bh * nsplit + split) * G) * 128;
    for (int gg = 0; gg < G; ++gg) po[(int64_t)gg * 128 + d] = acc[gg];
    if (threadIdx.x < G)
        part_ml[((int64_t)bh * nsplit + split) * G + threadIdx.x] = make_float2(s_m[threadIdx.x], s_l[threadIdx.x]);
}

// grid = B*Hq, 128 threads: merge the splits of one query head.
__global__ void __launch_bounds__(AT_THREADS) attn_combine_kernel(
    const float *__restrict__ part_o, const float2 *__restrict__ part_ml,
    __nv_bfloat16 *__restrict__ out, int G, int nsplit)
{
    const int hq_global = blockIdx.x;  // b*Hq + hq
    const int bh = hq_global / G, gg = hq_global % G;
    __shared__ float s_w[1024];
    __shared__ float s_inv;
    if (threadIdx.x < 32) {
        float M = -INFINITY;
        for (int i = threadIdx.x; i < nsplit; i += 32) M = fmaxf(M, part_ml[((int64_t)bh * nsplit + i) * G + gg].x);
        M = warp_max(M);
        float Lsum = 0.f;
        for (int i = threadIdx.x; i < nsplit; i += 32) {
            const float2 ml = part_ml[((int64_t)bh * nsplit + i) * G + gg];
            const float w = __expf(ml.x - M);
            s_w[i] = w;
            Lsum += ml.y * w;
        }
        Lsum = warp_sum(Lsum);
        if (threadIdx.x == 0) s_inv = 1.f / Lsum;
    }
    __syncthreads();
    const int d = threadIdx.x;
    float o = 0.f;
    for (int i = 0; i < nsplit; ++i) o = fmaf(part_o[(((int64_t)bh * nsplit + i) * G + gg) * 128 + d], s_w[i], o);
    out[(int64_t)hq_global * 128 + d] = f2bf(o * s_inv);
}

struct AttnPlan {
    int kps, nsplit;
    size_t off_o, off_ml, total, smem;
};

static AttnPlan plan_attn(const skv_decode_geom *g, int S)
{
    AttnPlan p = {};
    const int BH = g->batch * g->kv_heads;
    const int G = g->q_heads / g->kv_heads;
    const int target = 2 * 148;
    int kps = 64 * ceil_div(ceil_div(S * BH, target), 64);
    if (kps < 64) kps = 64;
    if (kps > 512) kps = 512;
    p.kps = kps;
    p.nsplit = ceil_div(S, kps);
    if (p.nsplit > 1024) {
        p.nsplit = 1024;
        p.kps = 64 * ceil_div(ceil_div(S, 1024), 64);
        p.nsplit = ceil_div(S, p.kps);
    }
    auto align = [](size_t x) { return (x + 255) & ~(size_t)255; };
    p.off_o = 0;
    p.off_ml = align((size_t)BH * p.nsplit * G * 128 * 4);
    p.total = p.off_ml + align((size_t)BH * p.nsplit * G * 8);
    p.smem = (size_t)p.kps * 128 * 2 + (size_t)p.kps * G * 4;
    return p;
}

}  // namespace skv

using namespace skv;

extern "C" {

size_t skv_decode_attention_workspace(const skv_decode_geom *g, int seq_len)
{
    if (!g || seq_len <= 0 || g->kv_heads <= 0 || g->batch <= 0) return 0;
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
    SKV_CHECK_ARG(aligned(q, 16) && aligned(k_buf, 16) && aligned(v_buf, 16), "operands must be 16-byte aligned");
    const AttnPlan p = plan_attn(g, seq_len);
    SKV_CHECK_ARG(workspace && workspace_bytes >= p.total, "workspace of %zu bytes needed, %zu given",
                  p.total, workspace_bytes);
    SKV_CHECK_ARG(aligned(workspace, 256), "workspace must be 256-byte aligned");
    cudaStream_t s = (cudaStream_t)stream;
    unsigned char *ws = reinterpret_cast<unsigned char *>(workspace);
    float *po = reinterpret_cast<float *>(ws + p.off_o);
    float2 *pml = reinterpret_cast<float2 *>(ws + p.off_ml);
    const int BH = g->batch * g->kv_heads;
    dim3 grid(p.nsplit, BH);
    cudaError_t e;
    if (G <= 8) {
        e = cudaFuncSetAttribute(attn_split_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
        if (e == cudaSuccess)
            attn_split_kernel<1><<<grid, AT_THREADS, p.smem, s>>>(
                (const __nv_bfloat16 *)q, (const __nv_bfloat16 *)k_buf, (const __nv_bfloat16 *)v_buf, po, pml,
                g->kv_heads, G, g->buf_len, seq_len, p.kps, g->scale);
    } else {
        e = cudaFuncSetAttribute(attn_split_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
        if (e == cudaSuccess)
            attn_split_kernel<2><<<grid, AT_THREADS, p.smem, s>>>(
                (const __nv_bfloat16 *)q, (const __nv_bfloat16 *)k_buf, (const __nv_bfloat16 *)v_buf, po, pml,
                g->kv_heads, G, g->buf_len, seq_len, p.kps, g->scale);
    }
    if (e != cudaSuccess) {
        set_error("cudaFuncSetAttribute(attn_split_kernel) failed: %s", cudaGetErrorString(e));
        return SKV_ERR_CUDA;
    }
    int st = check_launch("attn_split_kernel");
    if (st) return st;
    attn_combine_kernel<<<g->batch * g->q_heads, AT_THREADS, 0, s>>>(po, pml, (__nv_bfloat16 *)out, G, p.nsplit);
    return check_launch("attn_combine_kernel");
}

}  // extern "C"
