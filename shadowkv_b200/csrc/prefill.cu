// Prefill state builder: landmarks, outlier chunks, host value store and the
// first selection of one layer, as GPU kernels.
//
// Restates ShadowKVCache_CPU.prefill_kv_cache (models/kvcache/shadow.py:463-544):
//   * the values of the whole prompt go to the page-locked chunk store
//     (shadow.py:471-474): one strided device-to-host copy, the chunk layout
//     [chunk][8 rows][128] being the prompt's own row order
//     (skv_prefill_store_values, for a stream of its own: it overlaps the rest);
//   * landmark candidates = mean of each chunk's 8 post-RoPE keys, and the
//     chunk's minimum cosine similarity between the mean and its rows
//     (shadow.py:484-488) -- prefill_landmark_kernel, bf16 op by op like the
//     torch ops it replaces (fp32 sums, one bf16 rounding per op);
//   * the outlier_chunk chunks of smallest minimum similarity
//     (shadow.py:491, topk(largest=False)) -- prefill_outlier_kernel, exact
//     radix select on the bf16 values, ties to the lower chunk id, listed by
//     (value, chunk id) ascending like the sorted topk;
//   * the landmarks of the other chunks in chunk order with their ids
//     (shadow.py:508-515) -- prefill_compact_kernel;
//   * the first selection with the last prompt query (shadow.py:518-524): the
//     decode selection (fp32 scores; the reference rounds the scores to bf16
//     first and leaves ties to torch.topk) into slots initialised to -1;
//   * the buffer rows (shadow.py:479-481, 503-505, 527-531): local window,
//     outlier chunks, selected chunks, copied from the prompt's own K/V rows --
//     prefill_rows_kernel.
#include <string.h>

#include "common.cuh"

namespace skv {

namespace {

constexpr int PF_OUT_T = 1024;  // threads of the outlier selection (one CTA per head)
constexpr int PF_MAX_OUTLIERS = 256;

struct PrefillDims {
    int B, H, T, chunks, nout, K, buf_len, host_chunks, local;
};

// Ascending order of float bits as unsigned integers.
__device__ __forceinline__ uint32_t asc_key(float v)
{
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float warp_sum_f(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One warp per chunk: lane l owns dims 4l..4l+3 of the 8 rows.
//   mean_d  = bf16(sum_i x_id / 8)                      (Tensor.mean, fp32 sum)
//   |v|     = bf16(sqrt(sum_d v_d^2)), clamped at bf16(1e-8)   (vector_norm)
//   cos_i   = bf16(sum_d bf16(bf16(mean_d/|mean|) * bf16(x_id/|x_i|)))
//   min_i cos_i -> minsim (as F.cosine_similarity(...).min(dim=-1))
__global__ void __launch_bounds__(256) prefill_landmark_kernel(const __nv_bfloat16 *__restrict__ k, PrefillDims d,
                                                               __nv_bfloat16 *__restrict__ cand,
                                                               float *__restrict__ minsim)
{
    const int bh = blockIdx.y, lane = threadIdx.x & 31;
    const int c = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (c >= d.chunks) return;
    const __nv_bfloat16 *rows = k + ((int64_t)bh * d.T + (int64_t)c * 8) * 128 + lane * 4;
    float x[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const uint2 raw = *reinterpret_cast<const uint2 *>(rows + i * 128);
        const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162 *>(&raw.x);
        const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162 *>(&raw.y);
        x[i][0] = __low2float(lo), x[i][1] = __high2float(lo), x[i][2] = __low2float(hi), x[i][3] = __high2float(hi);
    }
    const float eps = bf2f(f2bf(1e-8f));
    float m[4], nm = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) s = __fadd_rn(s, x[i][j]);
        m[j] = bf2f(f2bf(__fdiv_rn(s, 8.f)));
        nm = __fmaf_rn(m[j], m[j], nm);
    }
    {
        __nv_bfloat162 lo = __floats2bfloat162_rn(m[0], m[1]), hi = __floats2bfloat162_rn(m[2], m[3]);
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t *>(&lo);
        pk.y = *reinterpret_cast<uint32_t *>(&hi);
        *reinterpret_cast<uint2 *>(cand + ((int64_t)bh * d.chunks + c) * 128 + lane * 4) = pk;
    }
    const float norm_m = fmaxf(bf2f(f2bf(__fsqrt_rn(warp_sum_f(nm)))), eps);
    float a[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) a[j] = bf2f(f2bf(__fdiv_rn(m[j], norm_m)));
    float mn = INFINITY;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float nx = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) nx = __fmaf_rn(x[i][j], x[i][j], nx);
        const float norm_x = fmaxf(bf2f(f2bf(__fsqrt_rn(warp_sum_f(nx)))), eps);
        float dot = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) dot = __fadd_rn(dot, bmul(a[j], bf2f(f2bf(__fdiv_rn(x[i][j], norm_x)))));
        mn = fminf(mn, bf2f(f2bf(warp_sum_f(dot))));
    }
    if (lane == 0) minsim[(int64_t)bh * d.chunks + c] = mn;
}

// One CTA per head: the nout chunks of smallest minsim (exact; two 8-bit
// radix passes over the top 16 bits, which hold the whole bf16 value), ties
// to the lower chunk id; out[bh][r] = chunk of rank r by (value, chunk id).
__global__ void __launch_bounds__(PF_OUT_T) prefill_outlier_kernel(const float *__restrict__ minsim, PrefillDims d,
                                                                  int32_t *__restrict__ out)
{
    __shared__ unsigned s_hist[256];
    __shared__ int s_bin, s_need;
    __shared__ unsigned s_nsel;
    __shared__ uint32_t s_key[PF_MAX_OUTLIERS];
    __shared__ int s_idx[PF_MAX_OUTLIERS];
    __shared__ int s_wcnt[PF_OUT_T / 32];
    const int bh = blockIdx.x, tid = threadIdx.x;
    const float *ms = minsim + (int64_t)bh * d.chunks;
    uint32_t prefix = 0;  // the boundary's top bits found so far
    int need = d.nout;
    for (int pass = 0; pass < 2; ++pass) {
        for (int i = tid; i < 256; i += PF_OUT_T) s_hist[i] = 0;
        __syncthreads();
        const int shift = pass == 0 ? 24 : 16;
        for (int c = tid; c < d.chunks; c += PF_OUT_T) {
            const uint32_t kk = asc_key(ms[c]);
            if (pass == 0 || (kk >> 24) == prefix) atomicAdd(&s_hist[(kk >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            int acc = 0, b = 0;
            for (; b < 256; ++b) {
                if (acc + (int)s_hist[b] >= need) break;
                acc += (int)s_hist[b];
            }
            s_bin = b;
            s_need = need - acc;
        }
        __syncthreads();
        prefix = (prefix << 8) | (uint32_t)s_bin;
        need = s_need;
        __syncthreads();
    }
    // keys below the boundary value are in; of the keys equal to it, the
    // `need` lowest chunk ids (scanned in chunk order, one CTA-wide round at a time)
    if (tid == 0) s_nsel = 0;
    __syncthreads();
    int taken_eq = 0;
    for (int base = 0; base < d.chunks; base += PF_OUT_T) {
        const int c = base + tid;
        uint32_t kk = 0xffffffffu;
        if (c < d.chunks) kk = asc_key(ms[c]);
        const uint32_t top = kk >> 16;
        const bool below = c < d.chunks && top < prefix;
        const bool equal = c < d.chunks && top == prefix;
        if (below) {
            const unsigned pos = atomicAdd(&s_nsel, 1u);
            if (pos < PF_MAX_OUTLIERS) s_key[pos] = kk, s_idx[pos] = c;
        }
        // rank of this equal key among this round's equal keys (chunk order)
        const unsigned bal = __ballot_sync(0xffffffffu, equal);
        if ((tid & 31) == 0) s_wcnt[tid >> 5] = __popc(bal);
        __syncthreads();
        int before = 0, total = 0;
        for (int w = 0; w < PF_OUT_T / 32; ++w) {
            if (w < (tid >> 5)) before += s_wcnt[w];
            total += s_wcnt[w];
        }
        before += __popc(bal & ((1u << (tid & 31)) - 1u));
        if (equal && taken_eq + before < need) {
            const unsigned pos = atomicAdd(&s_nsel, 1u);
            if (pos < PF_MAX_OUTLIERS) s_key[pos] = kk, s_idx[pos] = c;
        }
        taken_eq += total;
        __syncthreads();
    }
    __syncthreads();
    const int n = min((int)s_nsel, d.nout);
    if (tid < n) {
        const uint32_t ki = s_key[tid];
        const int ci = s_idx[tid];
        int r = 0;
        for (int j = 0; j < n; ++j) r += (s_key[j] < ki || (s_key[j] == ki && s_idx[j] < ci)) ? 1 : 0;
        out[(int64_t)bh * d.nout + r] = ci;
    }
    if (tid == 0 && (int)s_nsel != d.nout) report_dev_error(DEV_ERR_SLOT);
}

// Landmarks of the non-outlier chunks in chunk order: one warp per chunk;
// the chunk's destination is its id minus the outliers below it.
__global__ void __launch_bounds__(256) prefill_compact_kernel(const __nv_bfloat16 *__restrict__ cand,
                                                              const int32_t *__restrict__ outl, PrefillDims d,
                                                              __nv_bfloat16 *__restrict__ lm, int64_t *__restrict__ lm_idx)
{
    __shared__ int s_out[PF_MAX_OUTLIERS];
    const int bh = blockIdx.y, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < d.nout; i += blockDim.x) s_out[i] = outl[(int64_t)bh * d.nout + i];
    __syncthreads();
    const int c = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (c >= d.chunks) return;
    int below = 0, is_out = 0;
    for (int i = lane; i < d.nout; i += 32) {
        below += s_out[i] < c ? 1 : 0;
        is_out |= s_out[i] == c ? 1 : 0;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        below += __shfl_xor_sync(0xffffffffu, below, o);
        is_out |= __shfl_xor_sync(0xffffffffu, is_out, o);
    }
    if (is_out) return;
    const int dst = c - below;
    const int L = d.chunks - d.nout;
    const uint2 v = *reinterpret_cast<const uint2 *>(cand + ((int64_t)bh * d.chunks + c) * 128 + lane * 4);
    *reinterpret_cast<uint2 *>(lm + ((int64_t)bh * L + dst) * 128 + lane * 4) = v;
    if (lane == 0) lm_idx[(int64_t)bh * L + dst] = c;
}

// Buffer rows [0, sparse_end) of every head from the prompt's own K/V rows:
// local window, outlier chunks (in the outlier list's order), selected chunks
// (slot order); one warp per row, K and V.  Also position_ids = slots (int64).
__global__ void __launch_bounds__(256) prefill_rows_kernel(const __nv_bfloat16 *__restrict__ k,
                                                           const __nv_bfloat16 *__restrict__ v,
                                                           const int32_t *__restrict__ outl,
                                                           const int32_t *__restrict__ slots, PrefillDims d,
                                                           __nv_bfloat16 *__restrict__ k_buf,
                                                           __nv_bfloat16 *__restrict__ v_buf,
                                                           int64_t *__restrict__ position_ids)
{
    const int bh = blockIdx.y, lane = threadIdx.x & 31;
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int sparse_start = d.local + 8 * d.nout, sparse_end = sparse_start + 8 * d.K;
    if (r >= sparse_end) return;
    int64_t src;
    if (r < d.local) {
        src = (int64_t)d.T - d.local + r;
    } else if (r < sparse_start) {
        const int o = (r - d.local) >> 3;
        src = (int64_t)outl[(int64_t)bh * d.nout + o] * 8 + ((r - d.local) & 7);
    } else {
        const int j = (r - sparse_start) >> 3;
        const int cid = slots[(int64_t)bh * d.K + j];
        if (((r - sparse_start) & 7) == 0 && lane == 0) position_ids[(int64_t)bh * d.K + j] = cid;
        if (cid < 0 || cid >= d.chunks) {
            if (lane == 0) report_dev_error(DEV_ERR_HOST_CHUNK);
            return;
        }
        src = (int64_t)cid * 8 + ((r - sparse_start) & 7);
    }
    const int64_t so = ((int64_t)bh * d.T + src) * 128 + lane * 4, dof = ((int64_t)bh * d.buf_len + r) * 128 + lane * 4;
    *reinterpret_cast<uint2 *>(k_buf + dof) = *reinterpret_cast<const uint2 *>(k + so);
    *reinterpret_cast<uint2 *>(v_buf + dof) = *reinterpret_cast<const uint2 *>(v + so);
}

struct PrefillPlan {
    size_t off_cand, off_min, off_out, off_miss, off_sel, total;
};

PrefillPlan plan_prefill(const skv_prefill_geom *p, const skv_decode_geom &g)
{
    auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
    const size_t BH = (size_t)p->batch * p->kv_heads;
    PrefillPlan q;
    q.off_cand = 0;
    q.off_min = q.off_cand + al(BH * p->chunks * 128 * 2);
    q.off_out = q.off_min + al(BH * p->chunks * 4);
    q.off_miss = q.off_out + al(BH * p->outlier_chunk * 4);
    q.off_sel = q.off_miss + al(BH * (2 * (size_t)p->select_sets + 1) * 4);
    q.total = q.off_sel + al(skv_decode_select_workspace(&g));
    return q;
}

skv_decode_geom select_geom(const skv_prefill_geom *p)
{
    skv_decode_geom g = {};
    g.batch = p->batch;
    g.kv_heads = p->kv_heads;
    g.q_heads = p->q_heads;
    g.head_dim = 128;
    g.rank = 16;  // unused by the selection
    g.chunk_size = 8;
    g.select_sets = p->select_sets;
    g.num_landmarks = p->chunks - p->outlier_chunk;
    g.num_chunks = p->chunks;
    g.ctx_len = p->tokens;
    g.buf_len = p->buf_len;
    g.sparse_start = (p->tokens - 8 * p->chunks) + 8 * p->outlier_chunk;
    g.rope_mode = 0;
    g.cos_sin_stride = 128;
    g.cos_sin_rows = 1;
    g.scale = 0.08838834764831845f;  // 1 / sqrt(128)
    return g;
}

int check_prefill(const skv_prefill_geom *p)
{
    SKV_CHECK_ARG(p != nullptr, "null geometry");
    SKV_CHECK_ARG(p->batch > 0 && p->kv_heads > 0 && p->q_heads > 0 && p->q_heads % p->kv_heads == 0,
                  "bad head counts");
    SKV_CHECK_SUPPORTED(p->q_heads / p->kv_heads <= 16, "GQA group larger than 16");
    SKV_CHECK_ARG(p->tokens > 0 && p->chunks > 0 && 8 * (int64_t)p->chunks <= p->tokens, "chunks exceed the prompt");
    SKV_CHECK_SUPPORTED(p->outlier_chunk >= 1 && p->outlier_chunk <= PF_MAX_OUTLIERS,
                        "outlier_chunk outside 1..%d", PF_MAX_OUTLIERS);
    SKV_CHECK_ARG(p->chunks - p->outlier_chunk >= p->select_sets && p->select_sets >= 1,
                  "fewer landmarks than selected chunks");
    const int local = p->tokens - 8 * p->chunks;
    SKV_CHECK_ARG(local + 8 * (int64_t)(p->outlier_chunk + p->select_sets) <= p->buf_len,
                  "buffer too small for the prefill rows");
    SKV_CHECK_ARG(p->host_chunks >= p->tokens / 8, "host store holds fewer chunks than the prompt");
    return SKV_OK;
}

}  // namespace

}  // namespace skv

using namespace skv;

extern "C" {

size_t skv_prefill_workspace(const skv_prefill_geom *p)
{
    if (check_prefill(p) != SKV_OK) return 0;
    const skv_decode_geom g = select_geom(p);
    return plan_prefill(p, g).total;
}

int skv_prefill_store_values(const skv_prefill_geom *p, const void *v, void *v_host, void *stream)
{
    int st = check_prefill(p);
    if (st) return st;
    SKV_CHECK_ARG(v && v_host, "null pointer argument");
    // [B*H][T] rows -> [B*H][host_chunks][8 rows]: the chunk layout is the prompt's row order
    const void *hdev = nullptr;
    st = host_to_device_ptr(v_host, &hdev, "v_host");
    if (st) return st;
    const size_t row_bytes = 128 * 2, width = (size_t)(p->tokens / 8) * 8 * row_bytes;
    cudaError_t e = cudaMemcpy2DAsync(v_host, (size_t)p->host_chunks * 8 * row_bytes, v, (size_t)p->tokens * row_bytes,
                                      width, (size_t)p->batch * p->kv_heads, cudaMemcpyDeviceToHost,
                                      (cudaStream_t)stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("copy of the values to the host store failed: %s", cudaGetErrorString(e));
        return SKV_ERR_CUDA;
    }
    return SKV_OK;
}

int skv_prefill_build(const skv_prefill_geom *p, const void *k_roped, const void *v, const void *q_last,
                      void *k_buf, void *v_buf, void *landmarks, int64_t *landmark_idx, int32_t *slots,
                      int64_t *position_ids, void *workspace, size_t workspace_bytes, void *stream)
{
    int st = check_prefill(p);
    if (st) return st;
    SKV_CHECK_ARG(k_roped && v && q_last && k_buf && v_buf && landmarks && landmark_idx && slots && position_ids &&
                      workspace,
                  "null pointer argument");
    SKV_CHECK_ARG(aligned(k_roped, 16) && aligned(v, 16) && aligned(k_buf, 16) && aligned(v_buf, 16) &&
                      aligned(landmarks, 16) && aligned(workspace, 256),
                  "operands must be 16-byte aligned (workspace 256)");
    const skv_decode_geom g = select_geom(p);
    const PrefillPlan plan = plan_prefill(p, g);
    SKV_CHECK_ARG(workspace_bytes >= plan.total, "workspace of %zu bytes needed, %zu given", plan.total,
                  workspace_bytes);
    cudaStream_t s = (cudaStream_t)stream;
    const int BH = p->batch * p->kv_heads;
    PrefillDims d;
    d.B = p->batch, d.H = p->kv_heads, d.T = p->tokens, d.chunks = p->chunks, d.nout = p->outlier_chunk;
    d.K = p->select_sets, d.buf_len = p->buf_len, d.host_chunks = p->host_chunks, d.local = p->tokens - 8 * p->chunks;
    unsigned char *ws = static_cast<unsigned char *>(workspace);
    __nv_bfloat16 *cand = reinterpret_cast<__nv_bfloat16 *>(ws + plan.off_cand);
    float *minsim = reinterpret_cast<float *>(ws + plan.off_min);
    int32_t *outl = reinterpret_cast<int32_t *>(ws + plan.off_out);
    int32_t *miss = reinterpret_cast<int32_t *>(ws + plan.off_miss);

    const dim3 cgrid((p->chunks + 7) / 8, BH);
    prefill_landmark_kernel<<<cgrid, 256, 0, s>>>((const __nv_bfloat16 *)k_roped, d, cand, minsim);
    st = check_launch("prefill_landmark_kernel");
    if (st) return st;
    prefill_outlier_kernel<<<BH, PF_OUT_T, 0, s>>>(minsim, d, outl);
    st = check_launch("prefill_outlier_kernel");
    if (st) return st;
    prefill_compact_kernel<<<cgrid, 256, 0, s>>>(cand, outl, d, (__nv_bfloat16 *)landmarks, landmark_idx);
    st = check_launch("prefill_compact_kernel");
    if (st) return st;
    // first selection: every slot starts empty, so every selected chunk is a miss
    cudaError_t e = cudaMemsetAsync(slots, 0xff, (size_t)BH * p->select_sets * 4, s);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("cudaMemsetAsync of the slots failed: %s", cudaGetErrorString(e));
        return SKV_ERR_CUDA;
    }
    st = skv_decode_select(&g, q_last, landmarks, landmark_idx, slots, miss, miss + (size_t)BH * p->select_sets,
                           miss + (size_t)2 * BH * p->select_sets, ws + plan.off_sel,
                           plan.total - plan.off_sel, stream);
    if (st) return st;
    const int rows = d.local + 8 * (d.nout + d.K);
    prefill_rows_kernel<<<dim3((rows + 7) / 8, BH), 256, 0, s>>>((const __nv_bfloat16 *)k_roped,
                                                                 (const __nv_bfloat16 *)v, outl, slots, d,
                                                                 (__nv_bfloat16 *)k_buf, (__nv_bfloat16 *)v_buf,
                                                                 position_ids);
    return check_launch("prefill_rows_kernel");
}

}  // extern "C"
