// RoPE bindings of the reference (kernels/rope.cu, kernels/rope_new.cu).
//
// Every variant rotates one (t, t+half) pair (or one GLM interleaved pair)
// per thread with bf16 op-by-op arithmetic: o1 = x1*cos + (-x2)*sin,
// o2 = x2*cos + x1*sin, each multiply and add rounded to bf16 exactly as the
// reference's __hmul/__hadd chain (rope_new.cu:49-57, 262-270).
// Launch: a flat grid-stride loop over (row, pair) instead of one CTA per
// row, so that short rows do not leave most of the 148 SMs idle.
#include "common.cuh"

namespace skv {

enum RopeMode {
    ROPE_SEPARATE = 0,   // rope.cu: separate cos and sin tables, int64 token ids
    ROPE_NEW = 1,        // rope_new.cu:26-58: cos_sin table, int64 token ids
    ROPE_NEW_V2 = 2,     // rope_new.cu:86-118: int32 chunk ids
    ROPE_PUSH = 3,       // rope_new.cu:146-190 / 224-272: chunk ids, skip hits, write cache rows
    ROPE_PUSH_GLM = 4,   // rope_new.cu:305-374
};

struct RopeArgs {
    const __nv_bfloat16 *x;
    const __nv_bfloat16 *cos;  // or cos_sin
    const __nv_bfloat16 *sin;
    const void *pid;
    __nv_bfloat16 *out;
    const int32_t *cnts;
    int B, H, S, half;
    int sxb, sxh, sxs;
    int scos, ssin;
    int spb, sph, sps;
    int sob, soh, sos;
    int s_start, s_end;
    int chunk;
};

template <int MODE>
__global__ void __launch_bounds__(256) rope_kernel(RopeArgs a)
{
    const int pairs = (MODE == ROPE_PUSH_GLM) ? 64 : a.half;
    const int64_t total = (int64_t)a.B * a.H * a.S * pairs;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(idx % pairs);
        int64_t r = idx / pairs;
        const int s = (int)(r % a.S);
        r /= a.S;
        const int h = (int)(r % a.H);
        const int b = (int)(r / a.H);

        int64_t pos;
        if (MODE == ROPE_SEPARATE || MODE == ROPE_NEW) {
            const int64_t *p = reinterpret_cast<const int64_t *>(a.pid);
            pos = (int)p[(int64_t)b * a.spb + (int64_t)h * a.sph + (int64_t)s * a.sps];
        } else {
            if (MODE == ROPE_PUSH || MODE == ROPE_PUSH_GLM) {
                if (s / a.chunk < a.cnts[b * a.H + h]) continue;
                if (a.s_start + s >= a.s_end) continue;
            }
            const int32_t *p = reinterpret_cast<const int32_t *>(a.pid);
            const int id = p[(int64_t)b * a.spb + (int64_t)h * a.sph + (int64_t)(s / a.chunk) * a.sps];
            pos = (int64_t)id * a.chunk + s % a.chunk;
        }
        const __nv_bfloat16 *xr = a.x + (int64_t)b * a.sxb + (int64_t)h * a.sxh + (int64_t)s * a.sxs;
        __nv_bfloat16 *orow;
        if (MODE == ROPE_PUSH || MODE == ROPE_PUSH_GLM)
            orow = a.out + (int64_t)b * a.sob + (int64_t)h * a.soh + (int64_t)(a.s_start + s) * a.sos;
        else  // the reference writes the output with the strides of x
            orow = a.out + (int64_t)b * a.sxb + (int64_t)h * a.sxh + (int64_t)s * a.sxs;

        if (MODE == ROPE_PUSH_GLM) {
            const __nv_bfloat16 *cs = a.cos + pos * a.scos;
            if (t < 32) {
                const float xe = bf2f(xr[2 * t]), xo = bf2f(xr[2 * t + 1]);
                const float c = bf2f(cs[t]), sn = bf2f(cs[t + 32]);
                orow[2 * t] = f2bf(badd(bmul(xe, c), bmul(-xo, sn)));
                orow[2 * t + 1] = f2bf(badd(bmul(xo, c), bmul(xe, sn)));
            } else {
                orow[t + 32] = xr[t + 32];
                orow[t + 64] = xr[t + 64];
            }
        } else {
            const float x1 = bf2f(xr[t]), x2 = bf2f(xr[t + a.half]);
            float c1, s1, c2, s2;
            if (MODE == ROPE_SEPARATE) {
                const __nv_bfloat16 *cr = a.cos + pos * a.scos;
                const __nv_bfloat16 *sr = a.sin + pos * a.ssin;
                c1 = bf2f(cr[t]);
                c2 = bf2f(cr[t + a.half]);
                s1 = bf2f(sr[t]);
                s2 = bf2f(sr[t + a.half]);
            } else {
                const __nv_bfloat16 *cs = a.cos + pos * a.scos;
                c1 = c2 = bf2f(cs[t]);
                s1 = s2 = bf2f(cs[t + a.half]);
            }
            orow[t] = f2bf(badd(bmul(x1, c1), bmul(-x2, s1)));
            orow[t + a.half] = f2bf(badd(bmul(x2, c2), bmul(x1, s2)));
        }
    }
}

template <int MODE>
static int launch_rope(const RopeArgs &a, cudaStream_t stream, const char *name)
{
    const int pairs = (MODE == ROPE_PUSH_GLM) ? 64 : a.half;
    const int64_t total = (int64_t)a.B * a.H * a.S * pairs;
    if (total == 0) return SKV_OK;
    int64_t blocks = (total + 255) / 256;
    if (blocks > 148 * 16) blocks = 148 * 16;
    rope_kernel<MODE><<<(unsigned)blocks, 256, 0, stream>>>(a);
    return check_launch(name);
}

static int check_common(const void *x, const void *cs, const void *pid, const void *out, int B,
                        int H, int S, int D, int half)
{
    SKV_CHECK_ARG(x && cs && pid && out, "null pointer argument");
    SKV_CHECK_ARG(B >= 0 && H >= 0 && S >= 0, "negative size");
    SKV_CHECK_ARG(half > 0 && 2 * half <= D, "half_dim must satisfy 0 < 2*half_dim <= embed_dim");
    return SKV_OK;
}

}  // namespace skv

using namespace skv;

extern "C" {

int skv_apply_rotary_pos_emb(const void *x, const void *cos, const void *sin,
                             const int64_t *position_ids, void *output, int batch_size, int heads,
                             int seq_len, int embed_dim, int stride_xb, int stride_xh,
                             int stride_xs, int stride_xe, int stride_cos, int stride_sin,
                             int stride_pid_b, int stride_pid_h, int stride_pid_s, int half_dim,
                             void *stream)
{
    (void)stride_xe;
    SKV_CHECK_ARG(sin != nullptr, "null pointer argument");
    int st = check_common(x, cos, position_ids, output, batch_size, heads, seq_len, embed_dim, half_dim);
    if (st) return st;
    RopeArgs a = {};
    a.x = (const __nv_bfloat16 *)x;
    a.cos = (const __nv_bfloat16 *)cos;
    a.sin = (const __nv_bfloat16 *)sin;
    a.pid = position_ids;
    a.out = (__nv_bfloat16 *)output;
    a.B = batch_size, a.H = heads, a.S = seq_len, a.half = half_dim;
    a.sxb = stride_xb, a.sxh = stride_xh, a.sxs = stride_xs;
    a.scos = stride_cos, a.ssin = stride_sin;
    a.spb = stride_pid_b, a.sph = stride_pid_h, a.sps = stride_pid_s;
    return launch_rope<ROPE_SEPARATE>(a, (cudaStream_t)stream, "rope(separate)");
}

int skv_apply_rotary_pos_emb_new(const void *x, const void *cos_sin, const int64_t *position_ids,
                                 void *output, int batch_size, int heads, int seq_len,
                                 int embed_dim, int stride_xb, int stride_xh, int stride_xs,
                                 int stride_xe, int stride_cos_sin, int stride_pid_b,
                                 int stride_pid_h, int stride_pid_s, int half_dim, void *stream)
{
    (void)stride_xe;
    int st = check_common(x, cos_sin, position_ids, output, batch_size, heads, seq_len, embed_dim, half_dim);
    if (st) return st;
    RopeArgs a = {};
    a.x = (const __nv_bfloat16 *)x;
    a.cos = (const __nv_bfloat16 *)cos_sin;
    a.pid = position_ids;
    a.out = (__nv_bfloat16 *)output;
    a.B = batch_size, a.H = heads, a.S = seq_len, a.half = half_dim;
    a.sxb = stride_xb, a.sxh = stride_xh, a.sxs = stride_xs;
    a.scos = stride_cos_sin;
    a.spb = stride_pid_b, a.sph = stride_pid_h, a.sps = stride_pid_s;
    return launch_rope<ROPE_NEW>(a, (cudaStream_t)stream, "rope(new)");
}

int skv_apply_rotary_pos_emb_new_v2(const void *x, const void *cos_sin,
                                    const int32_t *position_ids, void *output, int batch_size,
                                    int heads, int seq_len, int embed_dim, int stride_xb,
                                    int stride_xh, int stride_xs, int stride_xe,
                                    int stride_cos_sin, int stride_pid_b, int stride_pid_h,
                                    int stride_pid_s, int half_dim, int chunk_size, void *stream)
{
    (void)stride_xe;
    int st = check_common(x, cos_sin, position_ids, output, batch_size, heads, seq_len, embed_dim, half_dim);
    if (st) return st;
    SKV_CHECK_ARG(chunk_size > 0, "chunk_size must be positive");
    RopeArgs a = {};
    a.x = (const __nv_bfloat16 *)x;
    a.cos = (const __nv_bfloat16 *)cos_sin;
    a.pid = position_ids;
    a.out = (__nv_bfloat16 *)output;
    a.B = batch_size, a.H = heads, a.S = seq_len, a.half = half_dim;
    a.sxb = stride_xb, a.sxh = stride_xh, a.sxs = stride_xs;
    a.scos = stride_cos_sin;
    a.spb = stride_pid_b, a.sph = stride_pid_h, a.sps = stride_pid_s;
    a.chunk = chunk_size;
    return launch_rope<ROPE_NEW_V2>(a, (cudaStream_t)stream, "rope(new_v2)");
}

static int push_cache_impl(const void *x, const void *cos_sin, const int32_t *position_ids,
                           void *output, const int32_t *cnts, int batch_size, int heads,
                           int seq_len, int embed_dim, int stride_xb, int stride_xh,
                           int stride_xs, int stride_cos_sin, int stride_pid_b, int stride_pid_h,
                           int stride_pid_s, int stride_output_b, int stride_output_h,
                           int stride_output_s, int offset_output_s_start,
                           int offset_output_s_end, int half_dim, int chunk_size, bool glm,
                           cudaStream_t stream)
{
    int st = check_common(x, cos_sin, position_ids, output, batch_size, heads, seq_len, embed_dim, half_dim);
    if (st) return st;
    SKV_CHECK_ARG(cnts != nullptr, "null pointer argument");
    SKV_CHECK_ARG(chunk_size > 0, "chunk_size must be positive");
    SKV_CHECK_ARG(offset_output_s_start >= 0, "offset_output_s_start must be >= 0");
    if (glm) SKV_CHECK_SUPPORTED(half_dim == 64 && embed_dim == 128,
                                 "the GLM rotary is defined for embed_dim 128 / half_dim 64");
    RopeArgs a = {};
    a.x = (const __nv_bfloat16 *)x;
    a.cos = (const __nv_bfloat16 *)cos_sin;
    a.pid = position_ids;
    a.out = (__nv_bfloat16 *)output;
    a.cnts = cnts;
    a.B = batch_size, a.H = heads, a.S = seq_len, a.half = half_dim;
    a.sxb = stride_xb, a.sxh = stride_xh, a.sxs = stride_xs;
    a.scos = stride_cos_sin;
    a.spb = stride_pid_b, a.sph = stride_pid_h, a.sps = stride_pid_s;
    a.sob = stride_output_b, a.soh = stride_output_h, a.sos = stride_output_s;
    a.s_start = offset_output_s_start, a.s_end = offset_output_s_end;
    a.chunk = chunk_size;
    if (glm) return launch_rope<ROPE_PUSH_GLM>(a, stream, "rope(push_cache_glm)");
    return launch_rope<ROPE_PUSH>(a, stream, "rope(push_cache)");
}

int skv_apply_rotary_pos_emb_push_cache(const void *x, const void *cos_sin,
                                        const int32_t *position_ids, void *output,
                                        const int32_t *cnts, int batch_size, int heads,
                                        int seq_len, int embed_dim, int stride_xb, int stride_xh,
                                        int stride_xs, int stride_xe, int stride_cos_sin,
                                        int stride_pid_b, int stride_pid_h, int stride_pid_s,
                                        int stride_output_b, int stride_output_h,
                                        int stride_output_s, int offset_output_s_start,
                                        int offset_output_s_end, int half_dim, int chunk_size,
                                        void *stream)
{
    (void)stride_xe;
    return push_cache_impl(x, cos_sin, position_ids, output, cnts, batch_size, heads, seq_len,
                           embed_dim, stride_xb, stride_xh, stride_xs, stride_cos_sin, stride_pid_b,
                           stride_pid_h, stride_pid_s, stride_output_b, stride_output_h,
                           stride_output_s, offset_output_s_start, offset_output_s_end, half_dim,
                           chunk_size, false, (cudaStream_t)stream);
}

int skv_apply_rotary_pos_emb_push_cache_opt(
    const void *x, const void *cos_sin, const int32_t *position_ids, void *output,
    const int32_t *cnts, int batch_size, int heads, int seq_len, int embed_dim, int stride_xb,
    int stride_xh, int stride_xs, int stride_xe, int stride_cos_sin, int stride_pid_b,
    int stride_pid_h, int stride_pid_s, int stride_output_b, int stride_output_h,
    int stride_output_s, int offset_output_s_start, int offset_output_s_end, int half_dim,
    int chunk_size, void *stream)
{
    (void)stride_xe;
    return push_cache_impl(x, cos_sin, position_ids, output, cnts, batch_size, heads, seq_len,
                           embed_dim, stride_xb, stride_xh, stride_xs, stride_cos_sin, stride_pid_b,
                           stride_pid_h, stride_pid_s, stride_output_b, stride_output_h,
                           stride_output_s, offset_output_s_start, offset_output_s_end, half_dim,
                           chunk_size, false, (cudaStream_t)stream);
}

int skv_apply_rotary_pos_emb_push_cache_opt_glm(
    const void *x, const void *cos_sin, const int32_t *position_ids, void *output,
    const int32_t *cnts, int batch_size, int heads, int seq_len, int embed_dim, int stride_xb,
    int stride_xh, int stride_xs, int stride_xe, int stride_cos_sin, int stride_pid_b,
    int stride_pid_h, int stride_pid_s, int stride_output_b, int stride_output_h,
    int stride_output_s, int offset_output_s_start, int offset_output_s_end, int half_dim,
    int chunk_size, void *stream)
{
    (void)stride_xe;
    return push_cache_impl(x, cos_sin, position_ids, output, cnts, batch_size, heads, seq_len,
                           embed_dim, stride_xb, stride_xh, stride_xs, stride_cos_sin, stride_pid_b,
                           stride_pid_h, stride_pid_s, stride_output_b, stride_output_h,
                           stride_output_s, offset_output_s_start, offset_output_s_end, half_dim,
                           chunk_size, true, (cudaStream_t)stream);
}

}  // extern "C"
