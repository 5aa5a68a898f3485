// New-token step of the decode: RoPE of the query and key of the generated
// token and the append of key and value to the K/V buffers, in one launch.
//
// Reference: ShadowAttention.decode rotates q/k with vllm's rotary_embedding
// custom op (models/attention/shadow.py:26 -> models/llama.py:149-154,
// models/glm.py:200-205) and appends with two tensor copies in
// ShadowKVCache_CPU.update_kv_cache (models/kvcache/shadow.py:621-633).
// The rotation uses bf16 op-by-op arithmetic (each product and sum rounded
// to bf16), rotate-half for rope_mode 0, GLM interleaved pairs on dims 0..63
// for rope_mode 1.
#include "common.cuh"

namespace skv {

// grid = (ceil(items/256), batch), 256 threads, one item per thread:
// items = (q heads + kv heads) * 64 pairs + kv heads * 16 pieces of v
__global__ void __launch_bounds__(256) append_kernel(
    const __nv_bfloat16 *__restrict__ q, const __nv_bfloat16 *__restrict__ k_new,
    const __nv_bfloat16 *__restrict__ v_new, const int64_t *__restrict__ positions,
    const __nv_bfloat16 *__restrict__ cos_sin, __nv_bfloat16 *__restrict__ q_out,
    __nv_bfloat16 *__restrict__ k_buf, __nv_bfloat16 *__restrict__ v_buf, int Hq, int Hkv, int buf_len,
    int row, int rope_mode, int cs_stride, int cs_rows)
{
    const int b = blockIdx.y;
    const int64_t pos = positions[b];
    const bool pos_ok = pos >= 0 && pos < cs_rows;
    if (!pos_ok && threadIdx.x == 0 && blockIdx.x == 0) report_dev_error(DEV_ERR_ROW);
    const __nv_bfloat16 *cs = cos_sin + (pos_ok ? pos : 0) * cs_stride;
    const int rot_items = (Hq + Hkv) * 64;
    const int total = rot_items + Hkv * 16;
    for (int it = blockIdx.x * blockDim.x + threadIdx.x; it < total; it += gridDim.x * blockDim.x) {
        if (it < rot_items) {
            const int head = it / 64, t = it % 64;
            const __nv_bfloat16 *x;
            __nv_bfloat16 *o;
            if (head < Hq) {
                x = q + ((int64_t)b * Hq + head) * 128;
                o = q_out + ((int64_t)b * Hq + head) * 128;
            } else {
                const int h = head - Hq;
                x = k_new + ((int64_t)b * Hkv + h) * 128;
                o = k_buf + (((int64_t)b * Hkv + h) * buf_len + row) * 128;
            }
            if (!pos_ok) continue;
            if (rope_mode == 0) {
                const float x1 = bf2f(x[t]), x2 = bf2f(x[t + 64]);
                const float c = bf2f(cs[t]), s = bf2f(cs[t + 64]);
                o[t] = f2bf(badd(bmul(x1, c), bmul(-x2, s)));
                o[t + 64] = f2bf(badd(bmul(x2, c), bmul(x1, s)));
            } else if (t < 32) {
                const float xe = bf2f(x[2 * t]), xo = bf2f(x[2 * t + 1]);
                const float c = bf2f(cs[t]), s = bf2f(cs[t + 32]);
                o[2 * t] = f2bf(badd(bmul(xe, c), bmul(-xo, s)));
                o[2 * t + 1] = f2bf(badd(bmul(xo, c), bmul(xe, s)));
            } else {
                o[t + 32] = x[t + 32];
                o[t + 64] = x[t + 64];
            }
        } else {
            const int p = it - rot_items;
            const int h = p / 16, piece = p % 16;
            const uint4 v = ld_nc_v4(v_new + ((int64_t)b * Hkv + h) * 128 + piece * 8);
            st_v4(v_buf + (((int64_t)b * Hkv + h) * buf_len + row) * 128 + piece * 8, v);
        }
    }
}

}  // namespace skv

using namespace skv;

extern "C" {

int skv_decode_append(const skv_decode_geom *g, const void *q, const void *k_new, const void *v_new,
                      const int64_t *positions, const void *cos_sin, void *q_out, void *k_buf,
                      void *v_buf, int row, void *stream)
{
    SKV_CHECK_ARG(g && q && k_new && v_new && positions && cos_sin && q_out && k_buf && v_buf,
                  "null pointer argument");
    SKV_CHECK_SUPPORTED(g->head_dim == 128, "head_dim must be 128");
    SKV_CHECK_ARG(g->batch > 0 && g->kv_heads > 0 && g->q_heads > 0, "sizes must be positive");
    SKV_CHECK_SUPPORTED(g->rope_mode == 0 || g->rope_mode == 1, "rope_mode must be 0 or 1");
    SKV_CHECK_ARG(g->cos_sin_stride >= (g->rope_mode == 0 ? 128 : 64), "cos_sin_stride too small");
    SKV_CHECK_ARG(row >= 0 && row < g->buf_len, "append row %d outside the buffer", row);
    SKV_CHECK_ARG(aligned(v_new, 16) && aligned(v_buf, 16), "v_new and v_buf must be 16-byte aligned");
    const int items = (g->q_heads + g->kv_heads) * 64 + g->kv_heads * 16;
    append_kernel<<<dim3(ceil_div(items, 256), g->batch), 256, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16 *)q, (const __nv_bfloat16 *)k_new, (const __nv_bfloat16 *)v_new, positions,
        (const __nv_bfloat16 *)cos_sin, (__nv_bfloat16 *)q_out, (__nv_bfloat16 *)k_buf, (__nv_bfloat16 *)v_buf,
        g->q_heads, g->kv_heads, g->buf_len, row, g->rope_mode, g->cos_sin_stride, g->cos_sin_rows);
    return check_launch("append_kernel");
}

}  // extern "C"
