// One whole decode step of one layer, pipelined over groups of kv heads.
//
// Replaces, for a step, the reference's sequence (models/attention/shadow.py:
// 22-48 with models/kvcache/shadow.py:547-633): new-token RoPE + append,
// landmark scoring and top-k, value gather with the reuse cache, key
// reconstruction and attention -- the work of skv_decode_append_select
// followed by skv_decode_sparse_attention.
//
// The step is bound by the host link (the missed value chunks), and no byte
// of it can be requested before the selection of its head is done.  With all
// kv heads in one launch chain the link waits for every head's scoring and
// selection.  Here the heads are split into `head_groups` groups, each with
// its own launch chain on a library stream, forked from and joined back to the
// caller's stream:
//
//   caller stream:  fork ---------------------------------------------- join
//   group 0:        score0 > select0 > fetch/reconstruct/attend0 --------+
//   group 1:        score1 ...> select1 > fetch/reconstruct/attend1 -----+
//   group 2:        score2 ......> select2 > ...                         +
//
// The GPU hands out the CTAs of the groups' scoring kernels in launch order,
// so group 0's landmark scan gets the SMs first and its selection and value
// fetch start after a fraction of the whole scan; the later groups' scans and
// selections overlap the host-link transfer of the earlier ones.  (Making
// each scan wait for the previous one was measured slower: the groups'
// attention CTAs, one per SM while they wait on the link, then starve the
// later scans.)  The results are the same bits as one
// skv_decode_append_select + skv_decode_sparse_attention over all heads
// (the heads are independent).
//
// Early fetch (off by default: at the config1 decode step it measures slower
// than the attention kernel's own fetch; skv_decode_step_early_fetch(1) turns
// it on where the selection's shared memory allows it):
// the selection kernel of each group requests the value chunks of the
// certain misses from the host as soon as its histogram has located the
// boundary score, reconstructs the missed keys, writes keys and values into
// their slots and computes the head's attention itself, each CTA over the
// rows it fetched plus a share of the rows already in the buffers, merged
// through distributed shared memory: the step is then two kernels per group.
// The state is the same bits either way; the output differs only by fp32
// summation order (a different split of the rows into partials).
//
// Kernel timing (skv_decode_step_timing, off by default): the kernels of a
// timed step stamp the global timer into a span pair per (group, kernel) --
// thread 0 of every CTA, at its start (after its dependency wait) and at its
// end -- read with skv_decode_step_kernel_times.  The launches are those of an
// untimed step (programmatic dependent launch included); a captured graph
// stamps on every replay.
//
// Library streams and events are created per device on the first call that
// needs them (make that call before any stream capture); the fork and join are
// event waits, so a capture of the caller's stream captures the whole DAG.
// Calls from several host threads are serialised on a per-device lock while
// they enqueue work.
#include <atomic>
#include <mutex>

#include "select.cuh"

namespace skv {

constexpr int STEP_MAX_GROUPS = 8;
constexpr int STEP_MAX_DEVICES = 64;

struct StepStreams {
    bool ready = false;
    cudaStream_t s[STEP_MAX_GROUPS] = {};
    cudaEvent_t fork = nullptr, done[STEP_MAX_GROUPS] = {};
    std::mutex mu;
};
static StepStreams g_step[STEP_MAX_DEVICES];
static std::atomic<int> g_early_fetch{0};
static std::atomic<int> g_step_timing{0};
// kernel spans of timed steps: [group][scoring, selection, attention][begin, end]
// (span_begin); zero = empty, cleared by skv_decode_step_kernel_times
constexpr int STEP_SPAN_WORDS = STEP_MAX_GROUPS * 6;
__device__ unsigned long long g_step_span[STEP_SPAN_WORDS];
static std::atomic<int> g_timed_groups[STEP_MAX_DEVICES];  // groups of the last timed step
static thread_local LaunchSpans t_spans;

bool step_early_fetch() { return g_early_fetch.load(std::memory_order_relaxed) != 0; }
LaunchSpans launch_spans() { return t_spans; }

// Sets the span pairs of this host thread's next launches, restored on every return.
struct SpanScope {
    LaunchSpans prev;
    explicit SpanScope(const LaunchSpans &sp) : prev(t_spans) { t_spans = sp; }
    ~SpanScope() { t_spans = prev; }
};

static int step_streams(int dev, StepStreams **out)
{
    SKV_CHECK_SUPPORTED(dev >= 0 && dev < STEP_MAX_DEVICES, "device index %d above %d", dev, STEP_MAX_DEVICES - 1);
    StepStreams &st = g_step[dev];
    // called with st.mu held
    if (!st.ready) {
        int lo = 0, hi = 0;
        SKV_CUDA(cudaDeviceGetStreamPriorityRange(&lo, &hi));
        for (int i = 0; i < STEP_MAX_GROUPS; ++i) {
            SKV_CUDA(cudaStreamCreateWithPriority(&st.s[i], cudaStreamNonBlocking, hi));
            SKV_CUDA(cudaEventCreateWithFlags(&st.done[i], cudaEventDisableTiming));
        }
        SKV_CUDA(cudaEventCreateWithFlags(&st.fork, cudaEventDisableTiming));
        st.ready = true;
    }
    *out = &st;
    return SKV_OK;
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

// Per-group workspace: attention partials, miss slots, miss chunk ids, miss
// counts, selection scratch, staged inputs (each 256-byte aligned).
struct StepLayout {
    size_t miss_slot, miss_chunk, miss_count, sel, sel_bytes, att, att_bytes, stage, group_bytes;
};

// Inputs of the step (q, k_new, v_new, positions) that lie in page-locked
// host memory are copied into the group's staging area by one small kernel at
// the head of the group's chain (the groups' chains keep no common dependency
// but the fork): one 16-byte (or 8-byte) piece per thread, so every load over
// the host link is in flight at once.  Sizes are those of one group.
constexpr int STAGE_INPUTS = 4;
static void stage_input_bytes(const skv_decode_geom *g, size_t bytes[STAGE_INPUTS])
{
    const size_t B = (size_t)g->batch;
    bytes[0] = B * g->q_heads * 256;   // q [B][Hq][128] bf16
    bytes[1] = B * g->kv_heads * 256;  // k_new [B][Hkv][128] bf16
    bytes[2] = B * g->kv_heads * 256;  // v_new
    bytes[3] = B * 8;                  // positions [B] int64
}
static size_t stage_bytes(const skv_decode_geom *g)
{
    size_t b[STAGE_INPUTS], t = 0;
    stage_input_bytes(g, b);
    for (int j = 0; j < STAGE_INPUTS; ++j) t += align256(b[j]);
    return t;
}

struct StageArgs {
    const unsigned char *src[STAGE_INPUTS];
    unsigned char *dst[STAGE_INPUTS];
    int pieces[STAGE_INPUTS];  // pieces of input j (0: not staged)
    int wide[STAGE_INPUTS];    // 1: 16-byte pieces, 0: 8-byte pieces
};

__global__ void __launch_bounds__(256) stage_inputs_kernel(StageArgs a)
{
    // the scoring kernel after it may start (its landmark tiles) at once; it
    // waits for this grid before reading the staged inputs
    pdl_launch_dependents();
    int p = blockIdx.x * blockDim.x + threadIdx.x;  // piece over the staged inputs, in order
#pragma unroll
    for (int j = 0; j < STAGE_INPUTS; ++j) {
        if (p < a.pieces[j]) {
            if (a.wide[j])
                reinterpret_cast<uint4 *>(a.dst[j])[p] = ld_stream_v4(a.src[j] + 16 * (size_t)p);
            else
                reinterpret_cast<uint2 *>(a.dst[j])[p] = __ldg(reinterpret_cast<const uint2 *>(a.src[j]) + p);
            return;
        }
        p -= a.pieces[j];
    }
}

// The layout depends on the geometry only (the attention part is sized for
// buf_len rows, the longest step): the tickets of every group stay at fixed
// offsets from one call to the next.
static bool step_layout(const skv_decode_geom *gp, StepLayout *L)
{
    const size_t bh = (size_t)gp->batch * gp->kv_heads, K = (size_t)gp->select_sets;
    L->sel_bytes = skv_decode_select_workspace(gp);
    L->att_bytes = skv_decode_sparse_attention_workspace(gp, gp->buf_len);
    if (L->sel_bytes == 0 || L->att_bytes == 0) return false;
    L->att = 0;  // attention partials first: their tickets must be zero on the first call
    L->miss_slot = align256(L->att_bytes);
    L->miss_chunk = L->miss_slot + align256(bh * K * 4);
    L->miss_count = L->miss_chunk + align256(bh * K * 4);
    L->sel = L->miss_count + align256(bh * 4);
    L->stage = L->sel + align256(L->sel_bytes);
    L->group_bytes = L->stage + stage_bytes(gp);
    return true;
}

static skv_decode_geom group_geom(const skv_decode_geom *g, int groups)
{
    skv_decode_geom gp = *g;
    gp.kv_heads = g->kv_heads / groups;
    gp.q_heads = g->q_heads / groups;
    return gp;
}

}  // namespace skv

using namespace skv;

extern "C" {

int skv_decode_step_early_fetch(int enable)
{
    return g_early_fetch.exchange(enable ? 1 : 0);
}

size_t skv_decode_step_workspace(const skv_decode_geom *g, int head_groups)
{
    if (!g || head_groups < 1 || head_groups > STEP_MAX_GROUPS || g->kv_heads <= 0 ||
        g->kv_heads % head_groups != 0 || (head_groups > 1 && g->batch != 1))
        return 0;
    const skv_decode_geom gp = group_geom(g, head_groups);
    StepLayout L;
    if (!step_layout(&gp, &L)) return 0;
    return L.group_bytes * head_groups;
}

int skv_decode_step(const skv_decode_geom *g, const void *q, const void *k_new, const void *v_new,
                    const int64_t *positions, const void *cos_sin, void *q_out, void *k_buf, void *v_buf,
                    int row, const int32_t *row_dev, const void *landmarks, const int64_t *landmark_idx,
                    int32_t *slots, const void *U,
                    const void *SVt, const void *v_host, int seq_len, void *out, int32_t *miss_count,
                    int head_groups, void *workspace, size_t workspace_bytes, void *stream)
{
    SKV_CHECK_ARG(g != nullptr, "null geometry");
    SKV_CHECK_ARG(q && k_new && v_new && positions && cos_sin && q_out && k_buf && v_buf && landmarks &&
                      landmark_idx && slots && U && SVt && v_host && out && workspace,
                  "null pointer argument");
    SKV_CHECK_ARG(head_groups >= 1 && head_groups <= STEP_MAX_GROUPS && g->kv_heads > 0 &&
                      g->kv_heads % head_groups == 0,
                  "head_groups must divide kv_heads and be in 1..%d", STEP_MAX_GROUPS);
    SKV_CHECK_SUPPORTED(head_groups == 1 || g->batch == 1,
                        "head groups need batch 1 (a head group of a batch is not one contiguous block)");
    SKV_CHECK_ARG(aligned(workspace, 256), "workspace must be 256-byte aligned");
    const skv_decode_geom gp = group_geom(g, head_groups);
    StepLayout L;
    SKV_CHECK_ARG(step_layout(&gp, &L), "geometry rejected (see skv_decode_select_workspace)");
    SKV_CHECK_ARG(workspace_bytes >= L.group_bytes * head_groups, "workspace of %zu bytes needed, %zu given",
                  L.group_bytes * head_groups, workspace_bytes);
    const int G = g->q_heads / g->kv_heads, hg = gp.kv_heads;
    unsigned char *ws = static_cast<unsigned char *>(workspace);
    const cudaStream_t caller = (cudaStream_t)stream;

    // operands of the early fetch, checked before anything is launched
    const bool early = step_early_fetch();
    const void *hdev = nullptr;
    void *dout = nullptr;
    if (early) {
        SKV_CHECK_ARG(seq_len >= g->sparse_start + 8 * g->select_sets && seq_len <= g->buf_len,
                      "seq_len %d must cover the selected rows and fit in buf_len", seq_len);
        int so = out_to_device_ptr(out, &dout, "out");
        if (so != SKV_OK) return so;
        SKV_CHECK_ARG(aligned(dout, 8), "out must be 8-byte aligned");
        SKV_CHECK_SUPPORTED(g->rank % 16 == 0 && g->rank >= 16 && g->rank <= 256,
                            "rank must be a multiple of 16 in 16..256");
        SKV_CHECK_ARG(g->sparse_start >= 0 && g->sparse_start % 8 == 0 &&
                          g->sparse_start + 8 * (int64_t)g->select_sets <= g->buf_len,
                      "selected rows exceed buf_len (or sparse_start not a multiple of 8)");
        SKV_CHECK_ARG(aligned(U, 16) && aligned(SVt, 16) && aligned(k_buf, 16) && aligned(v_buf, 16) &&
                          aligned(cos_sin, 16) && g->cos_sin_stride % 8 == 0,
                      "U, SVt, k_buf, v_buf and cos_sin rows must be 16-byte aligned");
        int st = host_to_device_ptr(v_host, &hdev, "v_host");
        if (st != SKV_OK) return st;
        SKV_CHECK_ARG(aligned(hdev, 16), "v_host must be 16-byte aligned");
    }

    // inputs: device memory, or page-locked host memory staged by each group
    const void *in_dev[STAGE_INPUTS] = {q, k_new, v_new, positions};
    bool in_host[STAGE_INPUTS] = {};
    bool any_host = false;
    {
        static const char *const names[STAGE_INPUTS] = {"q", "k_new", "v_new", "positions"};
        for (int j = 0; j < STAGE_INPUTS; ++j) {
            int st = in_to_device_ptr(in_dev[j], &in_dev[j], &in_host[j], names[j]);
            if (st) return st;
            SKV_CHECK_ARG(!in_host[j] || aligned(in_dev[j], 8), "%s in host memory must be 8-byte aligned",
                          names[j]);
            any_host = any_host || in_host[j];
        }
    }

    // kernel timing: the span pairs of the device's g_step_span
    const bool timing = g_step_timing.load(std::memory_order_relaxed) != 0;
    unsigned long long *span = nullptr;
    int dev = 0;
    if (timing) {
        SKV_CUDA(cudaGetDevice(&dev));
        SKV_CHECK_SUPPORTED(dev >= 0 && dev < STEP_MAX_DEVICES, "device index %d above %d", dev,
                            STEP_MAX_DEVICES - 1);
        SKV_CUDA(cudaGetSymbolAddress(reinterpret_cast<void **>(&span), g_step_span));
        g_timed_groups[dev].store(0);  // set again once the whole timed step is enqueued
    }

    auto group = [&](int i, cudaStream_t s) -> int {
        const SpanScope spans(timing ? LaunchSpans{span + 6 * i, span + 6 * i + 2, span + 6 * i + 4} : LaunchSpans{});
        const int64_t h0 = (int64_t)i * hg;  // first kv head of the group (batch 1 when groups > 1)
        unsigned char *w = ws + L.group_bytes * i;
        int32_t *ms = reinterpret_cast<int32_t *>(w + L.miss_slot);
        int32_t *mc = reinterpret_cast<int32_t *>(w + L.miss_chunk);
        int32_t *mn = miss_count ? miss_count + h0 : reinterpret_cast<int32_t *>(w + L.miss_count);
        // the group's inputs (batch 1 when groups > 1: the group's heads are contiguous)
        const void *gin[STAGE_INPUTS] = {static_cast<const unsigned char *>(in_dev[0]) + h0 * G * 256,
                                         static_cast<const unsigned char *>(in_dev[1]) + h0 * 256,
                                         static_cast<const unsigned char *>(in_dev[2]) + h0 * 256, in_dev[3]};
        if (any_host) {
            size_t bytes[STAGE_INPUTS];
            stage_input_bytes(&gp, bytes);
            StageArgs sa = {};
            int64_t pieces = 0;
            size_t off = L.stage;
            for (int j = 0; j < STAGE_INPUTS; ++j) {
                if (in_host[j]) {
                    const bool wide = aligned(gin[j], 16) && bytes[j] % 16 == 0;
                    sa.src[j] = static_cast<const unsigned char *>(gin[j]);
                    sa.dst[j] = w + off;
                    sa.pieces[j] = (int)(bytes[j] / (wide ? 16 : 8));
                    sa.wide[j] = wide ? 1 : 0;
                    pieces += sa.pieces[j];
                    gin[j] = w + off;
                }
                off += align256(bytes[j]);
            }
            stage_inputs_kernel<<<(unsigned)((pieces + 255) / 256), 256, 0, s>>>(sa);
            int st = check_launch("stage_inputs_kernel");
            if (st) return st;
        }
        const __nv_bfloat16 *qb = static_cast<const __nv_bfloat16 *>(gin[0]);
        __nv_bfloat16 *qo = (__nv_bfloat16 *)q_out + h0 * G * 128;
        __nv_bfloat16 *kb = (__nv_bfloat16 *)k_buf + h0 * g->buf_len * 128;
        __nv_bfloat16 *vb = (__nv_bfloat16 *)v_buf + h0 * g->buf_len * 128;
        const __nv_bfloat16 *svt = (const __nv_bfloat16 *)SVt + h0 * 128 * g->rank;
        SelectArgs fx = {};
        if (early) {
            fx.v_host = (const uint4 *)hdev + h0 * (int64_t)g->num_chunks * 128;
            fx.U = (const __nv_bfloat16 *)U;
            fx.SVt = svt;
            fx.cos_sin = (const __nv_bfloat16 *)cos_sin;
            fx.k_buf = kb;
            fx.v_buf = vb;
            fx.q_rot = qo;
            fx.out = (__nv_bfloat16 *)dout + h0 * G * 128;
            fx.row_dev = row_dev;
            fx.seq_len = seq_len;
        }
        bool fetched = false;
        int st = append_select_launch(&gp, qb, static_cast<const __nv_bfloat16 *>(gin[1]),
                                      static_cast<const __nv_bfloat16 *>(gin[2]), static_cast<const int64_t *>(gin[3]),
                                      cos_sin, qo, kb, vb, row,
                                      (const __nv_bfloat16 *)landmarks + h0 * g->num_landmarks * 128,
                                      landmark_idx + h0 * g->num_landmarks, slots + h0 * g->select_sets, ms, mc, mn,
                                      w + L.sel, L.sel_bytes, s, row_dev, early ? &fx : nullptr, &fetched, any_host);
        if (st) return st;
        if (fetched) return SKV_OK;  // the selection kernel computed the attention too
        return sparse_attention_launch(&gp, qo, U, svt, cos_sin,
                                       (const __nv_bfloat16 *)v_host + h0 * (int64_t)g->num_chunks * 1024, kb, vb,
                                       ms, mc, mn, seq_len, (__nv_bfloat16 *)out + h0 * G * 128, w + L.att,
                                       L.att_bytes, s, row_dev);
    };

    if (head_groups == 1) {
        int st = group(0, caller);
        if (st == SKV_OK && timing) g_timed_groups[dev].store(1);
        return st;
    }

    SKV_CUDA(cudaGetDevice(&dev));
    SKV_CHECK_SUPPORTED(dev >= 0 && dev < STEP_MAX_DEVICES, "device index %d above %d", dev, STEP_MAX_DEVICES - 1);
    std::lock_guard<std::mutex> lock(g_step[dev].mu);
    StepStreams *ss = nullptr;
    int st = step_streams(dev, &ss);
    if (st) return st;
    SKV_CUDA(cudaEventRecord(ss->fork, caller));
    for (int i = 0; i < head_groups; ++i) {
        // group i's scoring after group i-1's (its whole bandwidth), after the fork
        SKV_CUDA(cudaStreamWaitEvent(ss->s[i], ss->fork, 0));
        st = group(i, ss->s[i]);
        if (st) {
            // join what was enqueued so far, so the caller's stream is not left forked
            for (int j = 0; j <= i; ++j) {
                cudaEventRecord(ss->done[j], ss->s[j]);
                cudaStreamWaitEvent(caller, ss->done[j], 0);
            }
            return st;
        }
        SKV_CUDA(cudaEventRecord(ss->done[i], ss->s[i]));
    }
    for (int i = 0; i < head_groups; ++i) SKV_CUDA(cudaStreamWaitEvent(caller, ss->done[i], 0));
    if (timing) g_timed_groups[dev].store(head_groups);
    return SKV_OK;
}

int skv_decode_step_timing(int enable)
{
    return g_step_timing.exchange(enable ? 1 : 0);
}

int skv_decode_step_kernel_times(double *us, int max_groups, int *groups)
{
    SKV_CHECK_ARG(us != nullptr && groups != nullptr && max_groups >= 1, "null output or max_groups < 1");
    int dev = 0;
    SKV_CUDA(cudaGetDevice(&dev));
    SKV_CHECK_SUPPORTED(dev >= 0 && dev < STEP_MAX_DEVICES, "device index %d above %d", dev, STEP_MAX_DEVICES - 1);
    const int ng = g_timed_groups[dev].load();
    SKV_CHECK_ARG(ng > 0, "no skv_decode_step has been enqueued with kernel timing on this device");
    SKV_CUDA(cudaDeviceSynchronize());
    unsigned long long h[STEP_SPAN_WORDS];
    SKV_CUDA(cudaMemcpyFromSymbol(h, g_step_span, sizeof(h)));
    static const unsigned long long zero[STEP_SPAN_WORDS] = {};
    SKV_CUDA(cudaMemcpyToSymbol(g_step_span, zero, sizeof(zero)));
    unsigned long long t0 = ~0ull;  // the earliest start of any kernel of the step
    for (int j = 0; j < ng * 3; ++j)
        if (h[2 * j] && ~h[2 * j] < t0) t0 = ~h[2 * j];
    SKV_CHECK_ARG(t0 != ~0ull, "no kernel of a timed step has run since the last read");
    const int n = ng < max_groups ? ng : max_groups;
    for (int j = 0; j < n * 3; ++j) {
        const bool ran = h[2 * j] != 0 && h[2 * j + 1] != 0;
        us[2 * j] = ran ? (double)(~h[2 * j] - t0) * 1e-3 : -1.0;
        us[2 * j + 1] = ran ? (double)(h[2 * j + 1] - t0) * 1e-3 : -1.0;
    }
    *groups = ng;
    return SKV_OK;
}

}  // extern "C"
