// Shared helpers of the shadowkv_b200 CUDA library (sm_100a).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <stdarg.h>

#include "../../include/shadowkv_b200.h"

namespace skv {

// ---------------------------------------------------------------------------
// Host-side error reporting (thread-local last message, status codes)
// ---------------------------------------------------------------------------
void set_error(const char *fmt, ...);
void clear_error();

#define SKV_CHECK_ARG(cond, ...)                     \
    do {                                             \
        if (!(cond)) {                               \
            ::skv::set_error(__VA_ARGS__);           \
            return SKV_ERR_INVALID_ARGUMENT;         \
        }                                            \
    } while (0)

#define SKV_CHECK_SUPPORTED(cond, ...)               \
    do {                                             \
        if (!(cond)) {                               \
            ::skv::set_error(__VA_ARGS__);           \
            return SKV_ERR_UNSUPPORTED;              \
        }                                            \
    } while (0)

// A failed runtime call is also kept as the thread's last CUDA error; it is
// taken off here, so that the next launch check does not report it again.
#define SKV_CUDA(call)                                                              \
    do {                                                                            \
        cudaError_t e_ = (call);                                                    \
        if (e_ != cudaSuccess) {                                                    \
            (void)cudaGetLastError();                                               \
            ::skv::set_error("%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), \
                             __FILE__, __LINE__);                                   \
            return SKV_ERR_CUDA;                                                    \
        }                                                                           \
    } while (0)

// Check the launch that was just issued.
int check_launch(const char *what);

// Raise the dynamic shared-memory limit of `func` to `bytes` on the current
// device.  Done once per (function, device); later calls only compare, so a
// launch path makes no CUDA API call beyond the launch itself (safe inside
// stream capture after the first call).
int ensure_smem_attr(const void *func, int bytes, const char *name);

// Verify that `p` is page-locked host memory mapped for the current device;
// on success *dev holds the device-side address of p.
int host_to_device_ptr(const void *p, const void **dev, const char *name);
// Device address of an output that is device memory or page-locked host
// memory (the kernel then writes it over the host link).
int out_to_device_ptr(void *p, void **dev, const char *name);
// The same for an input; *host tells which of the two it is.
int in_to_device_ptr(const void *p, const void **dev, bool *host, const char *name);

inline bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Streaming multiprocessors of the current device (queried once per device;
// 148 on a B200).  Grids are sized from it, not from a constant.
int device_sm_count();

// Tiled tensor map of a bf16 tensor for the bulk tensor copies
// (cuTensorMapEncodeTiled, reached through the runtime's driver entry points:
// the library does not link libcuda itself).  dims, strides (bytes, of dims
// 1.. rank-1) and box as the driver takes them, element strides 1, no
// interleave, 256-byte L2 promotion, zero fill out of bounds.
int encode_tensor_map_bf16(CUtensorMap *m, const void *base, unsigned rank, const cuuint64_t *dims,
                           const cuuint64_t *strides, const cuuint32_t *box, CUtensorMapSwizzle swizzle,
                           const char *name);

// Span pairs (see span_begin) of the kernels this host thread launches next;
// null: no stamps.  Set by skv_decode_step while it enqueues a timed group.
struct LaunchSpans {
    unsigned long long *score = nullptr, *select = nullptr, *attend = nullptr;
};
LaunchSpans launch_spans();

// ---------------------------------------------------------------------------
// Device-side error counter: a kernel that finds an index out of range skips
// the access and records it here (read back by skv_device_errors()).
// ---------------------------------------------------------------------------
enum DevErr : uint32_t { DEV_ERR_HOST_CHUNK = 1, DEV_ERR_SLOT = 2, DEV_ERR_ROW = 3, DEV_ERR_WAIT = 4 };

extern __device__ unsigned int g_dev_err_count;
extern __device__ unsigned int g_dev_err_first;

__device__ __forceinline__ void report_dev_error(uint32_t code)
{
    unsigned int prev = atomicAdd(&g_dev_err_count, 1u);
    if (prev == 0) atomicExch(&g_dev_err_first, code);
}

// Global timer of the GPU (nanoseconds).
__device__ __forceinline__ unsigned long long globaltimer_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Kernel spans of a timed decode step (skv_decode_step_timing): thread 0 of
// every CTA stamps its start (after its dependency wait) and its end into the
// kernel's pair; span[0] keeps the complement of the earliest start (an
// atomic max of ~t, so that a zeroed pair is empty), span[1] the latest end.
// A null pair stamps nothing.
__device__ __forceinline__ void span_begin(unsigned long long *span)
{
    if (span && threadIdx.x == 0) atomicMax(span, ~globaltimer_ns());
}
__device__ __forceinline__ void span_finish(unsigned long long *span)
{
    if (span && threadIdx.x == 0) atomicMax(span + 1, globaltimer_ns());
}

// ---------------------------------------------------------------------------
// Phase tracing (builds with -DSKV_TRACE only): thread 0 of a CTA stamps the
// global timer into event e; slot 2e keeps the earliest stamp of any CTA,
// slot 2e+1 the latest.  skv_trace_read() (exported by trace builds only)
// copies the slots out and resets them.  Without SKV_TRACE the stamps
// compile to nothing.
// ---------------------------------------------------------------------------
constexpr int SKV_TRACE_EVENTS = 32;
#ifdef SKV_TRACE
extern __device__ unsigned long long g_trace[2 * SKV_TRACE_EVENTS];
__device__ __forceinline__ void trace_stamp(int e)
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    atomicMin(&g_trace[2 * e], t);
    atomicMax(&g_trace[2 * e + 1], t);
}
#define SKV_TRACE_CTA(e)                                    \
    do {                                                    \
        if (threadIdx.x == 0) ::skv::trace_stamp(e);        \
    } while (0)
// Per-CTA records (trace builds only): a record of SKV_TRACE_FIELDS words per
// opened slot; skv_trace_records() copies them out and resets the count.
constexpr int SKV_TRACE_RECS = 4096, SKV_TRACE_FIELDS = 8;
extern __device__ unsigned long long g_trace_rec[SKV_TRACE_RECS * SKV_TRACE_FIELDS];
extern __device__ unsigned int g_trace_nrec;
__device__ __forceinline__ unsigned long long trace_now() { return globaltimer_ns(); }
__device__ __forceinline__ unsigned trace_smid()
{
    unsigned s;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(s));
    return s;
}
__device__ __forceinline__ int trace_rec_open()
{
    const unsigned i = atomicAdd(&g_trace_nrec, 1u);
    return i < (unsigned)SKV_TRACE_RECS ? (int)i : -1;
}
#define SKV_TRACE_REC_DECL int skv_trace_slot = -1
#define SKV_TRACE_REC_OPEN()                                                  \
    do {                                                                      \
        if (threadIdx.x == 0) skv_trace_slot = ::skv::trace_rec_open();       \
    } while (0)
#define SKV_TRACE_REC(f, v)                                                   \
    do {                                                                      \
        if (threadIdx.x == 0 && skv_trace_slot >= 0)                          \
            ::skv::g_trace_rec[skv_trace_slot * ::skv::SKV_TRACE_FIELDS + (f)] = (v); \
    } while (0)
#define SKV_TRACE_REC_NOW(f) SKV_TRACE_REC(f, ::skv::trace_now())
#else
#define SKV_TRACE_CTA(e) ((void)0)
#define SKV_TRACE_REC_DECL ((void)0)
#define SKV_TRACE_REC_OPEN() ((void)0)
#define SKV_TRACE_REC(f, v) ((void)0)
#define SKV_TRACE_REC_NOW(f) ((void)0)
#endif
// trace events of the fused decode step
enum TraceEvent : int {
    TR_SCORE_START = 0, TR_SCORE_TILE0 = 1, TR_SCORE_END = 2,
    TR_SEL_START = 3, TR_SEL_WAITED = 4, TR_SEL_KEYS = 5, TR_SEL_CAND = 6, TR_SEL_END = 7,
    TR_SA_START = 8, TR_SA_WAITED = 9, TR_SA_ISSUED = 10, TR_SA_KEYS = 11, TR_SA_VALUES = 12,
    TR_SA_TICKET = 13, TR_SA_MERGED = 14, TR_MARK_BEFORE = 15, TR_MARK_AFTER = 16,
    TR_SEL_C = 17, TR_SEL_TILE = 18, TR_SEL_HIST = 19, TR_SEL_SYNC1 = 20, TR_SEL_SCAN = 21, TR_SEL_MARKED = 22,
    TR_SEL_RANKED = 23, TR_SEL_DIFF = 24, TR_SA_LISTS = 25,
    TR_FX_TAIL = 26, TR_FX_KEYS = 27, TR_FX_VALUES = 28, TR_FX_END = 29,
};

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 ld_nc_v4(const void *p)
{
    uint4 r;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// Streaming 128-bit load that does not allocate in L1 (host / one-touch data).
__device__ __forceinline__ uint4 ld_stream_v4(const void *p)
{
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint4 ld_v4(const void *p)
{
    return *reinterpret_cast<const uint4 *>(p);
}

__device__ __forceinline__ void st_v4(void *p, uint4 v)
{
    *reinterpret_cast<uint4 *>(p) = v;
}

__device__ __forceinline__ float bf2f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ __nv_bfloat16 f2bf(float v) { return __float2bfloat16_rn(v); }

// bf16 multiply / add with a single rounding.  The product of two bf16
// values is exact in fp32 and fp32 has more than 2*8+2 significand bits, so
// fp32 arithmetic followed by one round-to-nearest-even to bf16 gives the
// correctly rounded bf16 result.  __fmul_rn/__fadd_rn keep the compiler from
// contracting the pair into an FMA.
__device__ __forceinline__ float bmul(float a, float b) { return bf2f(f2bf(__fmul_rn(a, b))); }
__device__ __forceinline__ float badd(float a, float b) { return bf2f(f2bf(__fadd_rn(a, b))); }

__device__ __forceinline__ float bf_lo(uint32_t w)
{
    return __uint_as_float(w << 16);
}
__device__ __forceinline__ float bf_hi(uint32_t w)
{
    return __uint_as_float(w & 0xffff0000u);
}
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi)
{
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

// mma.sync m16n8k16, bf16 inputs, fp32 accumulators (D = A*B + C in place).
__device__ __forceinline__ void mma_bf16_16816(float *c, uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__host__ __device__ __forceinline__ int ceil_div(int a, int b) { return (a + b - 1) / b; }

// RoPE of pair t of one 128-dim bf16 row in bf16 op-by-op arithmetic.
// mode 0: rotate-half, pair (t, t+64), cos = cs[t], sin = cs[t+64], t < 64.
// mode 1: GLM, pair (2t, 2t+1) with cos = cs[t], sin = cs[t+32] for t < 32;
//         for 32 <= t < 64 the pass-through dims t+32 and t+64 are copied.
__device__ __forceinline__ void rope_pair_bf16(const __nv_bfloat16 *x, __nv_bfloat16 *o,
                                               const __nv_bfloat16 *cs, int t, int mode)
{
    if (mode == 0) {
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
}

// ---- mbarrier / bulk-copy helpers (sm_90+ PTX) ----
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, unsigned bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Raise the transaction count of the current phase without arriving (the
// copies that complete it may be issued by several threads; one arrival,
// after all of them, closes the phase).
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, unsigned bytes)
{
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// Programmatic dependent launch (sm_90+).  A kernel launched with the
// programmatic-serialization attribute may start while the previous kernel of
// its stream still runs; pdl_wait() blocks until that kernel has completed and
// its memory is visible (a no-op for an ordinary launch).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Orders this thread's earlier generic accesses to shared memory before the
// bulk (async-proxy) copies it issues next into the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// The same for every state space: also orders global data this thread has
// acquired from other CTAs before the bulk copies it issues next from it.
__device__ __forceinline__ void fence_proxy_async_all() { asm volatile("fence.proxy.async;" ::: "memory"); }

// Bounded wait for the phase with the given parity; false if it did not complete.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, unsigned parity, unsigned max_iter = 1u << 22)
{
    const uint32_t a = smem_u32(bar);
    for (unsigned it = 0; it < max_iter; ++it) {
        uint32_t done;
        asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                     : "=r"(done) : "r"(a), "r"(parity) : "memory");
        if (done) return true;
    }
    return false;
}
// Bulk (TMA) copy of `bytes` from this GPU's global memory into this CTA's shared memory only.
__device__ __forceinline__ void bulk_g2s(void *smem_dst, const void *gmem_src, unsigned bytes, uint64_t *bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(smem_dst)), "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

}  // namespace skv
