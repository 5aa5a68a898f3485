// Top-k chunk selection and slot-stable reuse diff of the fused decode path.
//
// Reference: the selection of models/kvcache/shadow.py:567-573 (torch.max over
// the GQA group, torch.topk of select_sets chunks, gather through
// k_landmark_idx) and the reuse-cache diff of kernels/map.cuh:475-516.
//
// One 8-CTA thread-block cluster per (b, kv head).  Every CTA turns its
// eighth of the landmarks into order-preserving keys (max over the group of
// the softmax-normalised score) and builds a 256-bin histogram of their top
// bits (exponent and three mantissa bits).  After one cluster barrier every CTA sums the eight histograms through
// distributed shared memory and finds the bin that holds the K-th largest key.
// Keys above that bin are selected outright: their chunk ids are set in rank
// 0's bitmap of the new set with cluster-scope shared-memory atomics.  Keys in
// the bin (a few dozen for softmax scores) are appended to rank 0's candidate
// list, which rank 0 ranks exactly -- key descending, landmark index
// ascending, so that when the K-th score is tied the lowest landmark indices
// win.  Should more than SEL_REGION keys share the bin, the cluster falls back
// to an exact 4-pass radix select (8 bits per pass) with the same tie rule.
// Rank 0 then computes the slot-stable diff from the two bitmaps.
#include "attn_block.cuh"
#include "select.cuh"

#include <atomic>

namespace skv {

__device__ __forceinline__ uint32_t dsmem_addr(const void *local, unsigned rank)
{
    uint32_t a = (uint32_t)__cvta_generic_to_shared(local), r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    return r;
}
__device__ __forceinline__ uint32_t ld_dsmem_u32(uint32_t addr)
{
    uint32_t v;
    asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ void st_dsmem_u32(uint32_t addr, uint32_t v)
{
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void cluster_sync()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n"
                 "barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

// Split cluster barrier: arrive (releasing this thread's earlier memory
// accesses to the cluster) and, later, wait (acquiring the others').  A
// thread that requests bulk copies from host memory arrives before it issues
// them: a release issued while such copies are in flight waits for them.
__device__ __forceinline__ void cluster_arrive_release()
{
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire()
{
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// 16 bytes into CTA-of-the-cluster shared memory (remote_addr), completing as
// transaction bytes on that CTA's mbarrier (remote_bar): data and signal in
// one, no fence.
__device__ __forceinline__ void st_async_v4(uint32_t remote_addr, uint4 v, uint32_t remote_bar)
{
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];"
                 ::"r"(remote_addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w), "r"(remote_bar) : "memory");
}
// 16-byte asynchronous copy global -> shared through the load path (these do
// not queue behind bulk copies from host memory, which wait on the host link).
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gmem_src)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all()
{
    asm volatile("cp.async.commit_group;\n"
                 "cp.async.wait_group 0;\n" ::: "memory");
}

__device__ __forceinline__ void merge_ms(float &m, float &s, float m2, float s2)
{
    const float mm = fmaxf(m, m2);
    if (mm == -INFINITY) return;
    s = s * __expf(m - mm) + s2 * __expf(m2 - mm);
    m = mm;
}

__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }

// Exclusive prefix sum over the CTA (SEL_T threads).
__device__ int cta_excl_scan(int v, int *total, int *s_warp)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int NW = SEL_T / 32;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        const int w = lane < NW ? s_warp[lane] : 0;
        int wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += y;
        }
        if (lane < NW) s_warp[lane] = wi - w;
        if (lane == NW - 1) s_warp[32] = wi;
    }
    __syncthreads();
    const int r = s_warp[warp] + x - v;
    *total = s_warp[32];
    __syncthreads();
    return r;
}

__device__ __forceinline__ void atom_or_dsmem_u32(uint32_t addr, uint32_t v)
{
    asm volatile("red.shared::cluster.or.b32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void red_add_dsmem_u32(uint32_t addr, uint32_t v)
{
    asm volatile("red.shared::cluster.add.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint4 ld_dsmem_v4(uint32_t addr)
{
    uint4 v;
    asm volatile("ld.shared::cluster.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr) : "memory");
    return v;
}

// Exact cluster-wide radix select (4 passes of 8 bits) of the K largest keys,
// for the rare case of more boundary-bin candidates than a CTA's region holds
// (e.g. many equal scores); ties at the K-th key go to the lowest landmark
// indices (ranks in index order).  Sets the chunks in rank 0's bitmap (bmA0).
// Kept out of line so that the common path stays compact in the instruction cache.
// C_g = M_g + ln Z_g of query head gg from the scoring splits' (max, sum-exp)
// partials of head bh; one warp, the result in every lane.  The selection and
// keys_kernel both use it, so their keys are the same bits.
__device__ __forceinline__ float merge_partials(const float2 *part, int bh, int nsplit, int G, int gg, int lane)
{
    float mm = -INFINITY, ss = 0.f;
    // part is [BH][G][nsplit]: a warp's loads are contiguous; eight in flight
    // per lane before they are merged (long contexts have a hundred or more
    // splits per head)
    const float2 *ph = part + ((int64_t)bh * G + gg) * nsplit;
    for (int i0 = lane; i0 < nsplit; i0 += 8 * 32) {
        float2 p[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int i = i0 + 32 * u;
            p[u] = i < nsplit ? ph[i] : make_float2(-INFINITY, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) merge_ms(mm, ss, p[u].x, p[u].y);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, mm, o);
        const float s2 = __shfl_xor_sync(0xffffffffu, ss, o);
        merge_ms(mm, ss, m2, s2);
    }
    return mm + logf(ss);
}

// Keys of the landmarks of one logits tile in shared memory (cnt landmarks,
// rows of G = 4Q floats; the first is landmark k0 of the CTA) and their
// first-pass histogram.  The key of landmark c is
//     max_g softmax_g(c) = exp(max_g (logit_g(c) - C_g)),  C_g = M_g + ln Z_g,
// one exponential per landmark (exp is increasing, so the max moves inside).
// A warp takes 32 landmarks in Q reads of 32 consecutive 16-byte words (no
// bank conflicts): lane l holds heads 4(l%Q)..4(l%Q)+3 of one landmark, the Q
// lanes of a landmark reduce their maxima by shuffles, and the maximum moves
// to the landmark's lane.  The Q reads are independent (unrolled) chains.
template <int Q>
__device__ __forceinline__ void ring_tile_keys(const float4 *tile, int k0, int cnt, const float *s_C,
                                               uint32_t *keys, unsigned *s_hw)
{
    constexpr int LPL = 32 / Q;  // landmarks per read
    const int lane = threadIdx.x & 31, g0 = (lane & (Q - 1)) * 4;
    const float4 Cg = make_float4(s_C[g0], s_C[g0 + 1], s_C[g0 + 2], s_C[g0 + 3]);
    for (int base = threadIdx.x & ~31; base < cnt; base += SEL_T) {
        float m[Q];
#pragma unroll
        for (int j = 0; j < Q; ++j) {
            m[j] = -INFINITY;
            if (base + j * LPL + lane / Q < cnt) {
                const float4 v = tile[(base + j * LPL) * Q + lane];
                m[j] = fmaxf(fmaxf(m[j], v.x - Cg.x), v.y - Cg.y);
                m[j] = fmaxf(fmaxf(m[j], v.z - Cg.z), v.w - Cg.w);
            }
        }
#pragma unroll
        for (int o = 1; o < Q; o <<= 1)
#pragma unroll
            for (int j = 0; j < Q; ++j) m[j] = fmaxf(m[j], __shfl_xor_sync(0xffffffffu, m[j], o));
        float d = -INFINITY;
#pragma unroll
        for (int j = 0; j < Q; ++j) {
            const float v2 = __shfl_sync(0xffffffffu, m[j], (lane % LPL) * Q);
            if (lane / LPL == j) d = v2;
        }
        const float sc = __expf(d);
        const bool valid = base + lane < cnt;
        if (valid) keys[k0 + base + lane] = __float_as_uint(sc);
        if (valid) atomicAdd(&s_hw[sel_key_bin(__float_as_uint(sc))], 1u);
    }
}

template <int CL>
__device__ __noinline__ void select_radix_fallback(const uint32_t *keys, int n, int K, int c0, unsigned rank,
                                                   const int *lidx_s, const int64_t *lidx, int num_chunks,
                                                   uint32_t bmA0, unsigned (*s_hist)[256], unsigned *s_tot,
                                                   int *s_warp, unsigned *s_eq_rank)
{
    __shared__ int s_digit, s_above;
    const int tid = threadIdx.x, lane = tid & 31;
    auto chunk_of = [&](int c) -> int {
        if (lidx_s) return lidx_s[c];
        const int64_t v = lidx[c];
        return (v >= 0 && v < num_chunks) ? (int)v : -1;
    };
    auto mark = [&](int cid) {
        if (cid >= 0) atom_or_dsmem_u32(bmA0 + 4u * (uint32_t)(cid >> 5), 1u << (cid & 31));
        else report_dev_error(DEV_ERR_HOST_CHUNK);
    };
    (void)c0;
    uint32_t prefix = 0, pmask = 0;
    int remaining = K, n_equal = 0;
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        unsigned *h = s_hist[pass & 1];
        if (tid < 256) h[tid] = 0;
        __syncthreads();
        for (int base = (tid & ~31); base < n; base += SEL_T) {
            const int c = base + lane;
            const uint32_t k = c < n ? keys[c] : 0u;
            const bool part = c < n && (k & pmask) == prefix;
            const int bin = part ? (int)((k >> shift) & 255) : 256 + lane;
            const unsigned peers = __match_any_sync(0xffffffffu, bin);
            if (part && lane == __ffs(peers) - 1) atomicAdd(&h[bin], (unsigned)__popc(peers));
        }
        cluster_sync();  // every CTA's histogram of this pass is complete
        if (tid < 256) {
            unsigned t = 0;
            for (unsigned r = 0; r < CL; ++r) t += ld_dsmem_u32(dsmem_addr(&h[tid], r));
            s_tot[tid] = t;
        }
        __syncthreads();
        if (tid < 32) {
            // lane l owns digits 255-8l .. 248-8l (descending)
            int cnt[8], tot = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                cnt[i] = (int)s_tot[255 - 8 * tid - i];
                tot += cnt[i];
            }
            int incl = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (tid >= o) incl += y;
            }
            int above = incl - tot;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                if (above < remaining && above + cnt[i] >= remaining) {
                    s_digit = 255 - 8 * tid - i;
                    s_above = above;
                }
                above += cnt[i];
            }
        }
        __syncthreads();
        const int d = s_digit;
        remaining -= s_above;
        prefix |= (uint32_t)d << shift;
        pmask |= 255u << shift;
        if (pass == 3) {
            n_equal = (int)s_tot[d];
            if (tid < CL) s_eq_rank[tid] = ld_dsmem_u32(dsmem_addr(&h[d], tid));
        }
        __syncthreads();
    }
    const uint32_t T = prefix;  // the K-th largest key
    const bool take_all_equal = n_equal == remaining;
    for (int base = (tid & ~31); base < n; base += SEL_T) {
        const int c = base + lane;
        if (c < n) {
            const uint32_t k = keys[c];
            if (k > T || (take_all_equal && k == T)) mark(chunk_of(c));
        }
    }
    if (!take_all_equal) {
        // ties at the threshold: lowest landmark index first, ranks in index order
        int before = 0;
        for (unsigned r = 0; r < rank; ++r) before += (int)s_eq_rank[r];
        const int quota = max(0, min(remaining - before, (int)s_eq_rank[rank]));
        int taken = 0;
        for (int base = 0; base < n && taken < quota; base += SEL_T) {
            const int c = base + tid;
            const int f = (c < n && keys[c] == T) ? 1 : 0;
            int tot;
            const int r = cta_excl_scan(f, &tot, s_warp);
            if (f && taken + r < quota) mark(chunk_of(c));
            taken += tot;
        }
    }
}

// ---- the FETCH tail: value fetch, key reconstruction and attention ----------

// Value chunks a CTA requests right after the scan: its certain misses, up to
// the staging area, at most 16 for rank 0.  Rank 0 still has to send its
// message with asynchronous shared-memory stores, which can queue behind the
// bulk copies of its SM when many are in flight; the rest of its chunks are
// requested after the message is out.
__host__ __device__ __forceinline__ int fx_early_count(int nC, int K, int cap, unsigned rank)
{
    const int n = nC < K ? nC : K;
    const int m = n < cap ? n : cap;
    return rank == 0 && m > 16 ? 16 : m;
}

// Scores S = K q^T * scale of a 32-row tile (warps 0 and 1, 16 rows each)
// against the G query rows of sQ (row G of sQ is zero); rows >= nrows get
// -inf.  sK rows have pitch KT; sS is [32][16].
template <int NT>
__device__ __forceinline__ void fx_scores(const __nv_bfloat16 *sK, int KT, const __nv_bfloat16 *sQ, int G, float *sS,
                                          int nrows, float scale, int warp, int lane)
{
    float sc[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
    const __nv_bfloat16 *aRow = sK + (warp * 16 + (lane & 15)) * KT + (lane >> 4) * 8;
    const int bRow = (lane & 7) + ((lane >> 4) << 3);
    const __nv_bfloat16 *qRow = sQ + (bRow < G ? bRow : G) * AB_PITCH + ((lane >> 3) & 1) * 8;
#pragma unroll
    for (int kk = 0; kk < 128; kk += 16) {
        uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
        sa_ldsm(a0, a1, a2, a3, aRow + kk);
        sa_ldsm(b0, b1, b2, b3, qRow + kk);
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

// Softmax of a 32-row tile (warp gg for query row gg < G): weights P =
// bf16(exp(s - m)) into P [G][FX_PPITCH], (m, sum of the rounded weights)
// into ml[gg].  A tile has at least one row, so m is finite.
__device__ __forceinline__ void fx_softmax(const float *sS, __nv_bfloat16 *P, float2 *ml, int G, int warp, int lane)
{
    for (int gg = warp; gg < G; gg += SEL_T / 32) {
        const float x = sS[lane * 16 + gg];
        const float m = warp_max(x);  // -inf only when every row of the tile is invalid
        const float p = x == -INFINITY ? 0.f : __expf(x - m);
        const __nv_bfloat16 pb = f2bf(p);
        P[gg * FX_PPITCH + lane] = pb;
        const float l = warp_sum(bf2f(pb));
        if (lane == 0) ml[gg] = make_float2(m, l);
    }
}

// O_t = P V of a 32-row tile (warps 0-7, dims 16w .. 16w+15; V rows of pitch
// AB_PITCH) merged into the running (M, L, O) of the CTA:
// M' = max(M, m_t), O = O e^{M - M'} + O_t e^{m_t - M'}, L likewise.
__device__ __forceinline__ void fx_pv_merge(const __nv_bfloat16 *P, const __nv_bfloat16 *zp, const __nv_bfloat16 *sV,
                                            const float2 *ml, float *sO, float *sM, float *sL, int G, int warp,
                                            int lane, int tid)
{
    if (warp < 8) {
        float o[2][4];
#pragma unroll
        for (int i = 0; i < 2; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
        const int row = lane & 15;
        const __nv_bfloat16 *aRow = (row < G ? P + row * FX_PPITCH : zp) + (lane >> 4) * 8;
        const int vRow = (lane & 7) + ((lane >> 3) & 1) * 8;
        const int vCol = warp * 16 + (lane >> 4) * 8;
#pragma unroll
        for (int kk = 0; kk < FETCH_ROWS; kk += 16) {
            uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
            sa_ldsm(a0, a1, a2, a3, aRow + kk);
            sa_ldsm_t(b0, b1, b2, b3, sV + (kk + vRow) * AB_PITCH + vCol);
            mma_bf16_16816(o[0], a0, a1, a2, a3, b0, b1);
            mma_bf16_16816(o[1], a0, a1, a2, a3, b2, b3);
        }
        const int g = lane >> 2, t4 = lane & 3;
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
            const int r = g + 8 * hr;
            if (r >= G) continue;
            const float Mo = sM[r], mt = ml[r].x, Mn = fmaxf(Mo, mt);
            const float ao = Mo == -INFINITY ? 0.f : __expf(Mo - Mn), at = mt == -INFINITY ? 0.f : __expf(mt - Mn);
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                float2 *po = reinterpret_cast<float2 *>(sO + r * 128 + warp * 16 + i * 8 + 2 * t4);
                float2 v = *po;
                v.x = v.x * ao + o[i][2 * hr] * at;
                v.y = v.y * ao + o[i][2 * hr + 1] * at;
                *po = v;
            }
        }
    }
    __syncthreads();  // every O row is rescaled with the old M
    if (tid < G) {
        const float Mo = sM[tid], mt = ml[tid].x, Mn = fmaxf(Mo, mt);
        const float ao = Mo == -INFINITY ? 0.f : __expf(Mo - Mn), at = mt == -INFINITY ? 0.f : __expf(mt - Mn);
        sM[tid] = Mn;
        sL[tid] = sL[tid] * ao + ml[tid].y * at;
    }
    __syncthreads();
}

// FETCH tail of the selection kernel.  Rank 0's message (every miss of the
// head, ascending chunk id, with its slot and whether the exact ranking
// decided it) arrives on this CTA's mbarrier.  This CTA's misses are the
// certain ones it found at the scan (values already requested) and the
// ranking-decided misses r with r % cl == rank; its buffer rows (prefix,
// cached slots that stay, generated rows) are every cl-th 32-row tile of them.
// The CTA attends over exactly those rows, keeping a running (max, sum, O):
//   - buffer-row tiles first (their keys and values are in the buffers);
//   - then its misses, `cap` at a time: the values not requested yet are
//     requested, the keys are reconstructed 32 rows at a time (U, cos/sin and
//     SV^T rows through the load path, which bulk copies waiting on the host
//     link do not hold up; the same arithmetic as the fused attention), stored
//     into their slots of k_buf and scored at once (softmax per tile); when
//     the round's values are in, each tile's P V is added and the values are
//     stored into their slots of v_buf.
// Finally the cluster merges the CTAs' (max, sum, O) through distributed
// shared memory: CTA r writes output columns 16r .. 16r+15.  No bulk copy is
// in flight by then, so the cluster barriers cost their usual round trip.
// Invalid chunk ids or slots are counted as device errors and skipped.
__device__ __forceinline__ void fetch_tail(const SelectArgs &a, int bh, unsigned rank, unsigned cl,
                                           unsigned char *smem_raw, uint64_t *vbar, uint64_t *mbar, unsigned nC_raw,
                                           unsigned *s_nB, int *s_ngrp)
{
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = a.K, G = a.G;
    const int KP = a.rank + 8, KT = fetch_kt(a.rank);
    const int b = bh / a.Hkv;
    unsigned char *stage = smem_raw + a.stage_off;
    const int *lC = reinterpret_cast<const int *>(smem_raw + a.list_off);
    int *lB = reinterpret_cast<int *>(smem_raw + a.list_off) + K;
    int *lS = lB + K;  // [2K] slot of work entry i
    const int2 *msg = reinterpret_cast<const int2 *>(smem_raw + a.msg_off);  // [0]: count; [1 + r]: miss r
    __nv_bfloat16 *sU = reinterpret_cast<__nv_bfloat16 *>(smem_raw + a.recon_off);  // [32][KT] U rows, then keys
    __nv_bfloat16 *sB = sU + FETCH_ROWS * KT;                                          // [128][KP] SV^T of the head
    __nv_bfloat16 *sCS = sB + 128 * KP;                                                // [32][136] cos/sin, or V
    const FxAttLayout L = fx_att_layout(G, a.cap, a.buf_len, K);
    unsigned char *att = smem_raw + a.att_off;
    __nv_bfloat16 *sQ = reinterpret_cast<__nv_bfloat16 *>(att + L.q);
    float *sO = reinterpret_cast<float *>(att + L.o), *sM = reinterpret_cast<float *>(att + L.m);
    float *sL = reinterpret_cast<float *>(att + L.l), *sS = reinterpret_cast<float *>(att + L.s);
    __nv_bfloat16 *zp = reinterpret_cast<__nv_bfloat16 *>(att + L.zp);
    __nv_bfloat16 *pt = reinterpret_cast<__nv_bfloat16 *>(att + L.pt);
    __nv_bfloat16 *pTiles = reinterpret_cast<__nv_bfloat16 *>(att + L.p);
    float2 *tml = reinterpret_cast<float2 *>(att + L.tml);  // [ntiles + 1][16]; the last for buffer-row tiles
    int *grp = reinterpret_cast<int *>(att + L.grp);
    uint32_t *msb = reinterpret_cast<uint32_t *>(att + L.msb);
    const uint4 *vh = a.v_host + (int64_t)bh * a.num_chunks * 128;
    const int ppr = a.rank / 8, csp = a.rope_mode == 0 ? 16 : 8;  // 16-byte pieces per U / cos-sin row
    const __nv_bfloat16 *kb = a.k_buf + (int64_t)bh * a.buf_len * 128, *vb = a.v_buf + (int64_t)bh * a.buf_len * 128;

    if (!mbar_wait(mbar, 0)) {
        if (tid == 0) report_dev_error(DEV_ERR_WAIT);
        mbar_wait(mbar, 0);  // the message must be complete before it is read
    }
    SKV_TRACE_CTA(TR_FX_TAIL);
#ifdef SKV_TRACE
    __shared__ int s_trec3;
    if (tid == 0) {
        s_trec3 = ::skv::trace_rec_open();
        if (s_trec3 >= 0) {
            ::skv::g_trace_rec[s_trec3 * 8 + 0] = (unsigned long long)rank | ((unsigned long long)bh << 8);
            ::skv::g_trace_rec[s_trec3 * 8 + 1] = 0xF1F1ull;
            ::skv::g_trace_rec[s_trec3 * 8 + 2] = ::skv::trace_now();
        }
    }
#define SKV_TRACE_R3(f) do { if (tid == 0 && s_trec3 >= 0) ::skv::g_trace_rec[s_trec3 * 8 + (f)] = ::skv::trace_now(); } while (0)
#else
#define SKV_TRACE_R3(f) ((void)0)
#endif
    const int count = min(max(msg[0].x, 0), K);
    // rows of this step: seq_len of the launch, or the device-side position
    int seq_len = a.seq_len;
    if (a.row_dev) {
        const int r1 = *a.row_dev + 1;
        if (r1 >= a.sparse_start + 8 * K && r1 <= a.seq_len) seq_len = r1;
        else if (tid == 0 && rank == 0) report_dev_error(DEV_ERR_ROW);
    }
    const int sparse_end = a.sparse_start + 8 * K;
    // the slots refilled by misses; the query rows; the running state
    for (int w = tid; w < (K + 31) / 32; w += SEL_T) msb[w] = 0;
    for (int i = tid; i < FX_PPITCH; i += SEL_T) zp[i] = f2bf(0.f);
    for (int p = tid; p < (G + 1) * 16; p += SEL_T) {
        const int r = p >> 4, c = (p & 15) * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < G) v = ld_nc_v4(a.q_rot + ((int64_t)bh * G + r) * 128 + c);
        st_v4(sQ + r * AB_PITCH + c, v);
    }
    for (int i = tid; i < G * 128; i += SEL_T) sO[i] = 0.f;
    if (tid < 16) {
        sM[tid] = -INFINITY;
        sL[tid] = 0.f;
    }
    __syncthreads();
    SKV_TRACE_R3(3);
    for (int r = tid; r < count; r += SEL_T) {
        const int sl = msg[1 + r].y & 0x7fffffff;
        if (sl < K) atomicOr(&msb[sl >> 5], 1u << (sl & 31));
    }
    // the ranking-decided misses of this CTA
    if (warp == 0) {
        int nb = 0;
        for (int r0 = 0; r0 < count; r0 += 32) {
            const int r = r0 + lane;
            const bool mine = r < count && (msg[1 + r].y < 0) && (unsigned)r % cl == rank;
            const unsigned ball = __ballot_sync(0xffffffffu, mine);
            if (mine) lB[nb + __popc(ball & ((1u << lane) - 1u))] = msg[1 + r].x;
            nb += __popc(ball);
        }
        if (lane == 0) *s_nB = (unsigned)nb;
    }
    __syncthreads();
    SKV_TRACE_R3(4);
    // the 8-row groups of buffer rows, in row order: prefix, cached slots that
    // stay, generated rows (row0 | count << 24)
    if (warp == 0) {
        const int npre = a.sparse_start / 8;
        for (int q = lane; q < npre; q += 32) grp[q] = (q * 8) | (8 << 24);
        int n = npre;
        for (int s0 = 0; s0 < K; s0 += 32) {
            const int sl = s0 + lane;
            const bool hit = sl < K && !((msb[sl >> 5] >> (sl & 31)) & 1u);
            const unsigned ball = __ballot_sync(0xffffffffu, hit);
            if (hit) grp[n + __popc(ball & ((1u << lane) - 1u))] = (a.sparse_start + 8 * sl) | (8 << 24);
            n += __popc(ball);
        }
        for (int r0 = sparse_end + 8 * lane; r0 < seq_len; r0 += 256) grp[n + (r0 - sparse_end) / 8] = r0 | (min(8, seq_len - r0) << 24);
        n += (max(seq_len - sparse_end, 0) + 7) / 8;
        if (lane == 0) *s_ngrp = n;
    }
    const int nC = (int)min(nC_raw, (unsigned)K);
    __syncthreads();
    SKV_TRACE_R3(5);
    const int nB = (int)min(*s_nB, (unsigned)K), ngrp = *s_ngrp;
    const int nW = nC + nB, cap = a.cap, nEarly = fx_early_count((int)nC_raw, K, cap, rank);
    auto entry = [&](int i) -> int { return i < nC ? lC[i] : lB[i - nC]; };
    auto valid = [&](int cid) -> bool { return cid >= 0 && cid < a.num_chunks && (int64_t)cid * 8 + 8 <= a.ctx; };
    // the slot of every work entry (binary search of the message, ascending chunk ids)
    for (int i = tid; i < nW; i += SEL_T) {
        const int cid = entry(i);
        int lo = 0, hi = count;
        while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (msg[1 + mid].x < cid) lo = mid + 1;
            else hi = mid;
        }
        int sl = -1;
        if (lo < count && msg[1 + lo].x == cid) sl = msg[1 + lo].y & 0x7fffffff;
        if (sl >= K || !valid(cid)) sl = -1;
        if (sl < 0) report_dev_error(DEV_ERR_SLOT);
        lS[i] = sl;
    }
    SKV_TRACE_R3(6);
    SKV_TRACE_REC_DECL;
    SKV_TRACE_REC_OPEN();
    SKV_TRACE_REC(0, (unsigned long long)rank | ((unsigned long long)bh << 8) | ((unsigned long long)nC << 24) |
                         ((unsigned long long)nB << 40));
    SKV_TRACE_REC(1, (unsigned long long)(uintptr_t)a.k_buf);
    SKV_TRACE_REC_NOW(2);
    SKV_TRACE_REC(7, 0xF0F0ull);  // marks a record of this tail
    __syncthreads();

    auto score_tile = [&](int nrows, __nv_bfloat16 *P, float2 *ml) {
        if (warp < 2) {
            if (G <= 8) fx_scores<1>(sU, KT, sQ, G, sS, nrows, a.scale, warp, lane);
            else fx_scores<2>(sU, KT, sQ, G, sS, nrows, a.scale, warp, lane);
        }
        __syncthreads();
        fx_softmax(sS, P, ml, G, warp, lane);
        __syncthreads();
    };

    // buffer-row tiles: every cl-th group of four 8-row groups
    float2 *bml = tml + L.ntiles * 16;
    for (int t = (int)rank; 4 * t < ngrp; t += (int)cl) {
        int nrows = 0;
        for (int q = 0; q < 4 && 4 * t + q < ngrp; ++q) nrows += grp[4 * t + q] >> 24;
        for (int p = tid; p < FETCH_ROWS * 32; p += SEL_T) {
            const int r = (p >> 4) & (FETCH_ROWS - 1), c = (p & 15) * 8, q = r >> 3;
            const bool isv = p >= FETCH_ROWS * 16;
            __nv_bfloat16 *dst = isv ? sCS + r * AB_PITCH + c : sU + r * KT + c;
            const int gq = 4 * t + q < ngrp ? grp[4 * t + q] : 0;
            if (4 * t + q < ngrp && (r & 7) < (gq >> 24)) {
                const int64_t row = (gq & 0xffffff) + (r & 7);
                cp_async16(dst, (isv ? vb : kb) + row * 128 + c);
            } else {
                st_v4(dst, make_uint4(0, 0, 0, 0));
            }
        }
        cp_async_wait_all();
        __syncthreads();
        score_tile(nrows, pt, bml);
        fx_pv_merge(pt, zp, sCS, bml, sO, sM, sL, G, warp, lane, tid);
    }

    bool svt = false;
    for (int r0 = 0, round = 0; r0 < nW; r0 += cap, ++round) {
        const int rn = min(cap, nW - r0);
        // the round's value chunks that were not requested at the scan (later
        // rounds reuse the staging area: every copy of the last round is in)
        if (round > 0) fence_proxy_async_smem();
        {
            // copy j by warp j % 16, lane j / 16 (the issue is spread over every warp; rn <= 64)
            const int j = (tid & 31) * (SEL_T / 32) + (tid >> 5);
            const int i = r0 + j;
            const int cid = j < rn && i >= nEarly ? entry(i) : -1;  // below nEarly: requested at the scan
            if (cid >= 0 && cid < a.num_chunks) {
                uint64_t *tb = &vbar[j / (FETCH_ROWS / 8)];
                mbar_expect_tx(tb, 2048u);
                bulk_g2s(stage + (size_t)j * 2048, vh + (int64_t)cid * 128, 2048u, tb);
            }
        }
        __syncthreads();
        // one arrival per tile of the round closes its phase: it completes when its chunks are in
        const int ntr = (rn + FETCH_ROWS / 8 - 1) / (FETCH_ROWS / 8);
        if (tid < ntr) mbar_arrive(&vbar[tid]);
        // keys of the round's chunks, 4 chunks per pass: reconstructed, stored, scored
        for (int p0 = 0; p0 < rn; p0 += FETCH_ROWS / 8) {
            const int pn = min(FETCH_ROWS / 8, rn - p0);
            const int nu = pn * 8 * ppr, ncs = pn * 8 * csp, nsv = svt ? 0 : 128 * ppr;
            for (int p = tid; p < nu + ncs + nsv; p += SEL_T) {
                if (p < nu) {
                    const int r = p / ppr, c = p % ppr;
                    const int cid = entry(r0 + p0 + (r >> 3));
                    if (valid(cid))
                        cp_async16(sU + r * KT + c * 8, a.U + ((int64_t)b * a.ctx + (int64_t)cid * 8 + (r & 7)) * a.rank + c * 8);
                } else if (p < nu + ncs) {
                    const int q = p - nu, r = q / csp, c = q % csp;
                    const int cid = entry(r0 + p0 + (r >> 3));
                    const int64_t pos = (int64_t)cid * 8 + (r & 7);
                    if (valid(cid) && pos < a.cs_rows)
                        cp_async16(sCS + r * FETCH_PITCH + c * 8, a.cos_sin + pos * a.cs_stride + c * 8);
                } else {
                    const int q = p - nu - ncs, r = q / ppr, c = q % ppr;
                    cp_async16(sB + r * KP + c * 8, a.SVt + ((int64_t)bh * 128 + r) * a.rank + c * 8);
                }
            }
            cp_async_wait_all();
            __syncthreads();
            svt = true;
            // warp w < 4: rows 16 (w & 1) .. +15, output half (w >> 1)
            const int rg = warp & 1, half = (warp >> 1) & 1, g = lane >> 2, t4 = lane & 3;
            const bool mine = warp < 4 && 2 * rg < pn;
            uint32_t kres[16];
            if (mine) {
                float acc[8][4];
                recon_half(acc, sU + (rg * 16 + (lane & 15)) * KT + (lane >> 4) * 8, sB, KP, a.rank, half, lane);
#pragma unroll
                for (int hr = 0; hr < 2; ++hr) {
                    const int r = rg * 16 + g + 8 * hr, q = r >> 3;
                    float v[8][2];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        v[i][0] = acc[i][2 * hr];
                        v[i][1] = acc[i][2 * hr + 1];
                    }
                    const int cid = q < pn ? entry(r0 + p0 + q) : -1;
                    if (valid(cid)) {
                        if ((int64_t)cid * 8 + (r & 7) < a.cs_rows)
                            recon_rope(v, sCS + r * FETCH_PITCH, a.rope_mode, half, t4);
                        else if (t4 == 0)
                            report_dev_error(DEV_ERR_ROW);
                    }
#pragma unroll
                    for (int i = 0; i < 8; ++i) kres[hr * 8 + i] = pack_bf2(v[i][0], v[i][1]);
                }
            }
            __syncthreads();  // every warp is done reading the U rows
            if (mine) {
#pragma unroll
                for (int hr = 0; hr < 2; ++hr) {
                    const int r = rg * 16 + g + 8 * hr;
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        *reinterpret_cast<uint32_t *>(sU + r * KT + recon_col(half, i, t4)) = kres[hr * 8 + i];
                }
            }
            // rows of invalid entries are zero keys (their weights are zero below)
            for (int p = tid; p < FETCH_ROWS * 16; p += SEL_T) {
                const int r = p >> 4, c = (p & 15) * 8, q = r >> 3;
                if (q >= pn || lS[r0 + p0 + q] < 0) st_v4(sU + r * KT + c, make_uint4(0, 0, 0, 0));
            }
            __syncthreads();
            // the keys into their slots of k_buf
            for (int p = tid; p < pn * 8 * 16; p += SEL_T) {
                const int r = p >> 4, c = (p & 15) * 8;
                const int sl = lS[r0 + p0 + (r >> 3)];
                if (sl < 0) continue;
                st_v4(a.k_buf + ((int64_t)bh * a.buf_len + a.sparse_start + 8 * sl + (r & 7)) * 128 + c,
                      ld_v4(sU + r * KT + c));
            }
            // scores and weights of the pass's rows (an invalid entry's rows count as -inf)
            const int tp = p0 / (FETCH_ROWS / 8);
            __nv_bfloat16 *Pt = pTiles + (size_t)tp * G * FX_PPITCH;
            int nrows = pn * 8;
            if (warp < 2) {
                if (G <= 8) fx_scores<1>(sU, KT, sQ, G, sS, nrows, a.scale, warp, lane);
                else fx_scores<2>(sU, KT, sQ, G, sS, nrows, a.scale, warp, lane);
            }
            __syncthreads();
            for (int p = tid; p < FETCH_ROWS * 16; p += SEL_T) {
                const int r = p >> 4, q = r >> 3;
                if (q < pn && lS[r0 + p0 + q] < 0) sS[p] = -INFINITY;
            }
            __syncthreads();
            fx_softmax(sS, Pt, tml + tp * 16, G, warp, lane);
            __syncthreads();  // the tile is free for the next pass
        }
        if (round == 0) {
            SKV_TRACE_CTA(TR_FX_KEYS);
            SKV_TRACE_REC_NOW(3);
        }
        // per tile, in order, once its values are in: the values into the V
        // tile and their slots of v_buf, then P V
        for (int p0 = 0; p0 < rn; p0 += FETCH_ROWS / 8) {
            const int pn = min(FETCH_ROWS / 8, rn - p0), tp = p0 / (FETCH_ROWS / 8);
            if (!mbar_wait(&vbar[tp], (unsigned)round & 1u)) {
                if (tid == 0) report_dev_error(DEV_ERR_WAIT);
                mbar_wait(&vbar[tp], (unsigned)round & 1u);  // the copies must land before the area is read
            }
            if (round == 0 && p0 + FETCH_ROWS / 8 >= rn) {
                SKV_TRACE_CTA(TR_FX_VALUES);
                SKV_TRACE_REC_NOW(4);
            }
            for (int p = tid; p < FETCH_ROWS * 16; p += SEL_T) {
                const int r = p >> 4, c = (p & 15) * 8, q = r >> 3;
                uint4 v = make_uint4(0, 0, 0, 0);
                if (q < pn) {
                    const int sl = lS[r0 + p0 + q];
                    if (sl >= 0) {
                        v = ld_v4(stage + (size_t)(p0 + q) * 2048 + ((r & 7) * 16 + (p & 15)) * 16);
                        st_v4(a.v_buf + ((int64_t)bh * a.buf_len + a.sparse_start + 8 * sl + (r & 7)) * 128 + c, v);
                    }
                }
                st_v4(sCS + r * AB_PITCH + c, v);
            }
            __syncthreads();
            fx_pv_merge(pTiles + (size_t)tp * G * FX_PPITCH, zp, sCS, tml + tp * 16, sO, sM, sL, G, warp, lane, tid);
        }
    }
    SKV_TRACE_CTA(TR_FX_END);
    SKV_TRACE_REC_NOW(5);

    // the head's output: the cl partials merged through distributed shared memory
    cluster_sync();  // every CTA's (M, L, O) is final
    {
        const int dpc = 128 / (int)cl;  // output columns per CTA
        if (tid < G * dpc) {
            const int g = tid / dpc, d = (int)rank * dpc + tid % dpc;
            float Mj[16], Lj[16], Oj[16];
            float M = -INFINITY;
            for (unsigned j = 0; j < cl; ++j) {
                Mj[j] = __uint_as_float(ld_dsmem_u32(dsmem_addr(sM + g, j)));
                Lj[j] = __uint_as_float(ld_dsmem_u32(dsmem_addr(sL + g, j)));
                Oj[j] = __uint_as_float(ld_dsmem_u32(dsmem_addr(sO + g * 128 + d, j)));
                M = fmaxf(M, Mj[j]);
            }
            float Ls = 0.f, Os = 0.f;
            for (unsigned j = 0; j < cl; ++j) {
                if (Mj[j] == -INFINITY) continue;
                const float w = __expf(Mj[j] - M);
                Ls += Lj[j] * w;
                Os += Oj[j] * w;
            }
            a.out[((int64_t)bh * G + g) * 128 + d] = f2bf(Ls > 0.f ? Os / Ls : 0.f);
        }
    }
    cluster_sync();  // no CTA leaves while another may still read its shared memory
}

// FETCH (the decode step): the kernel also fetches the values of the missed
// chunks and writes their keys and values into their slots.  Every CTA loads
// the cached slots; right after the boundary bin is known, the chunks above it
// that are not cached -- certain misses -- are requested from the host value
// store with bulk copies into this CTA's shared memory (bulk copies do not
// hold up the SM's other memory requests while they wait on the host link;
// loads through the load/store unit would), rank 0 hands the misses decided
// later (boundary bin, or the exact fallback) to the CTAs round-robin, and
// after the slot diff every CTA reconstructs the keys of its chunks, waits
// for their values and stores both into the chunks' slots.  The host transfer
// thus starts several microseconds before the selection is complete.
template <int CL, bool FETCH>
__global__ void __launch_bounds__(SEL_T) select_cluster_kernel(SelectArgs a)
{
    constexpr int REGION = SEL_CAND / CL;  // candidates a CTA may push on the fast path
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ float s_C[16];  // M_g + ln Z_g of each query head of the group
    __shared__ __align__(16) unsigned s_h1[SEL_BINS];  // first-pass histogram (DSMEM-read)
    __shared__ unsigned s_hist[2][256];                // exact fallback: 8-bit pass histograms
    __shared__ unsigned s_tot[256];
    __shared__ int s_warp[33];
    __shared__ uint32_t s_ckey[SEL_CAND];              // rank 0: boundary-bin candidates (key,
    __shared__ int s_clm[SEL_CAND], s_cchunk[SEL_CAND]; //   landmark index, chunk id), region r from CTA r
    __shared__ unsigned s_ccnt[CL];                // rank 0: candidates pushed by CTA r
    __shared__ int s_pre[CL + 1];                  // rank 0: their exclusive prefix
    __shared__ int s_misssorted[1024];                 // rank 0: missed chunk ids, ascending
    __shared__ unsigned s_nloc;                        // candidates this CTA pushed so far
    // rank 0: the candidates, compacted; order word = key << 32 | ~landmark
    // (larger word = earlier in the selection order)
    __shared__ uint64_t s_lord[SEL_REGION];
    __shared__ int s_lchunk[SEL_REGION];
    __shared__ int s_bin, s_bin_above, s_bin_cnt;
    __shared__ unsigned s_eq_rank[CL];
    // FETCH: value copies issued at the scan ([0]) and later ([1], one phase per
    // round); reconstruction operands; chunks of this CTA (certain misses found
    // here, misses handed over by rank 0); rank 0: misses handed to each CTA
    // FETCH: completion of the value chunks of each 4-chunk tile of the staging
    // area (one phase per round); s_mbar: rank 0's message of the misses
    __shared__ __align__(8) uint64_t s_vbar[FX_MAX_TILES], s_mbar;
    __shared__ unsigned s_nC, s_nB;
    __shared__ int s_ngrp;                              // FETCH: groups of buffer rows attended here

    const unsigned rank = blockIdx.x;
    const int bh = blockIdx.y, tid = threadIdx.x, lane = tid & 31;
    const int G = a.G, L = a.L, K = a.K;
    const int slice = (L + CL - 1) / CL;
    const int c0 = (int)rank * slice;
    const int n = max(0, min(L, c0 + slice) - c0);
    const int nbw = (a.num_chunks + 31) >> 5;
    uint32_t *dyn = reinterpret_cast<uint32_t *>(smem_raw);
    uint32_t *keys = a.gkeys ? a.gkeys + (int64_t)bh * L + c0 : dyn;
    int *lidx_s = a.gkeys ? nullptr : reinterpret_cast<int *>(dyn + slice);
    uint32_t *bmA = a.gkeys ? dyn : dyn + 2 * slice;
    uint32_t *bmB = bmA + nbw;
    // per-warp first-pass histograms and the ring of logits tiles, after the
    // keys, chunk ids and bitmaps (128-byte aligned)
    unsigned (*s_hw)[SEL_BINS] = reinterpret_cast<unsigned (*)[SEL_BINS]>(
        smem_raw + ((select_base_bytes(L, a.num_chunks, a.gkeys != nullptr, CL) + 127) & ~(size_t)127));
    float *ring = reinterpret_cast<float *>(&s_hw[SEL_T / 32][0]);
    __shared__ __align__(8) uint64_t s_full[SEL_RING];
    const int64_t *lidx = a.landmark_idx + (int64_t)bh * L + c0;
    int32_t *slots = a.slots + (int64_t)bh * K;

    // The fused attention that follows (one CTA per SM) may become resident on
    // the SMs this grid leaves free; it waits for this grid before reading.
    // (FETCH: this grid runs until the values are in; the attention launches
    // as the grid ends rather than hold SMs that long.)
    if constexpr (!FETCH) pdl_launch_dependents();
    SKV_TRACE_CTA(TR_SEL_START);
    SKV_TRACE_REC_DECL;
#ifdef SKV_TRACE
    __shared__ int s_trec2;  // a second record of this CTA, written by any thread
#define SKV_TRACE_R2(f) do { if (s_trec2 >= 0) ::skv::g_trace_rec[s_trec2 * ::skv::SKV_TRACE_FIELDS + (f)] = ::skv::trace_now(); } while (0)
#else
#define SKV_TRACE_R2(f) ((void)0)
#endif
    if constexpr (FETCH) {
        SKV_TRACE_REC_OPEN();
        SKV_TRACE_REC(0, (unsigned long long)rank | ((unsigned long long)bh << 8));
        SKV_TRACE_REC(1, 0x5E1ull);  // marks a record of the selection phases
        SKV_TRACE_REC_NOW(2);
#ifdef SKV_TRACE
        if (tid == 0) {
            s_trec2 = ::skv::trace_rec_open();
            if (s_trec2 >= 0) {
                ::skv::g_trace_rec[s_trec2 * 8 + 0] = (unsigned long long)rank | ((unsigned long long)bh << 8);
                ::skv::g_trace_rec[s_trec2 * 8 + 1] = 0x5E2ull;
            }
        }
#endif
    }
#ifdef SKV_TRACE
    else if (tid == 0) {
        s_trec2 = -1;  // no second record: shared memory starts undefined
    }
#endif

    // 0) loads that do not depend on the scores: the cached slots (rank 0,
    //    thread t owns slots 2t, 2t+1) and the chunk ids of this slice
    int old[2] = {-1, -1};
    if (rank == 0 || FETCH) {
        for (int w = tid; w < 2 * nbw; w += SEL_T) bmA[w] = 0;  // bmA and bmB are contiguous
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int sl = 2 * tid + u;
            if (sl < K) old[u] = slots[sl];
        }
    }
    if (lidx_s) {
        for (int cb = tid; cb < n; cb += 4 * SEL_T) {
            int64_t v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = cb + u * SEL_T < n ? __ldg(lidx + cb + u * SEL_T) : -1;
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (cb + u * SEL_T < n) lidx_s[cb + u * SEL_T] = (v[u] >= 0 && v[u] < a.num_chunks) ? (int)v[u] : -1;
        }
    }
    for (int i = tid; i < SEL_BINS; i += SEL_T) s_h1[i] = 0;
    for (int i = tid; i < (SEL_T / 32) * SEL_BINS; i += SEL_T) (&s_hw[0][0])[i] = 0;
    if (tid == 0) s_nloc = 0;
    if (tid < CL) s_ccnt[tid] = 0;
    if constexpr (FETCH) {
        if (tid == 0) {
            s_nC = 0;
            s_nB = 0;
            for (int t = 0; t < FX_MAX_TILES; ++t) mbar_init(&s_vbar[t], 1);
            mbar_init(&s_mbar, 1);
            mbar_fence_init();
            // rank 0's message comes as transaction bytes on s_mbar: expected before
            // the first cluster barrier, which precedes its sending
            mbar_arrive_expect_tx(&s_mbar, fetch_msg_bytes(K));
        }
        if (rank == 0) {
            uint32_t *bmC = reinterpret_cast<uint32_t *>(smem_raw + a.bmc_off);
            for (int w = tid; w < nbw; w += SEL_T) bmC[w] = 0;
        }
    }

    pdl_wait();  // the scoring kernel's logits and partials are complete from here on
    span_begin(a.span);
    SKV_TRACE_CTA(TR_SEL_WAITED);

    // the logits of this CTA's landmarks come in through bulk (TMA) copies,
    // SEL_RING tiles in flight, issued before the split partials are merged;
    // for G = 4, 8 or 16 (a landmark row of 1, 2 or 4 16-byte words);
    // other group sizes read them directly
    const float *lg = a.logits + ((int64_t)bh * L + c0) * G;
    const bool use_ring = !a.keys_in && (G == 4 || G == 8 || G == 16);
    const int kps = use_ring ? (SEL_RSTAGE / (G * 4)) & ~31 : 0;  // landmarks per tile
    const int ntile = use_ring ? (n + kps - 1) / kps : 0;
    auto issue_tile = [&](int i) {
        const int cnt = min(kps, n - i * kps);
        const unsigned bytes = (unsigned)cnt * (unsigned)G * 4u;
        mbar_arrive_expect_tx(&s_full[i % SEL_RING], bytes);
        bulk_g2s(ring + (size_t)(i % SEL_RING) * (SEL_RSTAGE / 4), lg + (int64_t)i * kps * G, bytes, &s_full[i % SEL_RING]);
    };
    if (use_ring && tid == 0) {
        for (int i = 0; i < SEL_RING; ++i) mbar_init(&s_full[i], 1);
        mbar_fence_init();
        for (int i = 0; i < min(ntile, SEL_RING); ++i) issue_tile(i);
    }

    // 1) softmax normalisers of each query head of the group: warp w merges the
    //    split partials of head w (lanes load in parallel, then a shuffle merge)
    if (!a.keys_in && warp_id() < G) {
        const float C = merge_partials(a.part, bh, a.nsplit, G, warp_id(), lane);
        if (lane == 0) s_C[warp_id()] = C;
    }
    __syncthreads();
    SKV_TRACE_CTA(TR_SEL_C);
    bool hit[2] = {false, false};
    if (rank == 0 || FETCH) {
#pragma unroll
        for (int u = 0; u < 2; ++u)
            if (old[u] >= 0 && old[u] < a.num_chunks) atomicOr(&bmB[old[u] >> 5], 1u << (old[u] & 31));
    }

    // 2) keys of this CTA's landmarks -- the bits of max_g softmax_g =
    //    exp(max_g (logit_g - C_g)), which is >= 0, so the unsigned order of
    //    the bits is the order of the scores -- and their first-pass
    //    histogram.  Warp-uniform loops (compact code: it runs once per step, cold).
    auto key_of = [&](const float *row) -> float {
        float d = -INFINITY;
        for (int gg = 0; gg < G; ++gg) d = fmaxf(d, row[gg] - s_C[gg]);
        return __expf(d);
    };
    auto add_key = [&](int c, bool valid, float sc) {
        if (valid) keys[c] = __float_as_uint(sc);
        if (valid) atomicAdd(&s_hw[warp_id()][sel_key_bin(__float_as_uint(sc))], 1u);
    };
    if (a.keys_in) {
        // keys computed by keys_kernel: copied into this CTA's slice, eight
        // loads in flight per thread, and counted
        const uint32_t *kin = a.keys_in + (int64_t)bh * L + c0;
        for (int cb = tid; cb < n; cb += 8 * SEL_T) {
            uint32_t kk[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) kk[u] = cb + u * SEL_T < n ? __ldg(kin + cb + u * SEL_T) : 0u;
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (cb + u * SEL_T < n) {
                    keys[cb + u * SEL_T] = kk[u];
                    atomicAdd(&s_hw[warp_id()][sel_key_bin(kk[u])], 1u);
                }
        }
    } else if (use_ring) {
        for (int i = 0; i < ntile; ++i) {
            if (!mbar_wait(&s_full[i % SEL_RING], (i / SEL_RING) & 1)) {
                if (tid == 0) report_dev_error(DEV_ERR_WAIT);
                mbar_wait(&s_full[i % SEL_RING], (i / SEL_RING) & 1);  // the tile must land before it is reused
            }
            if (i == 0) SKV_TRACE_CTA(TR_SEL_TILE);
            const float4 *tile = reinterpret_cast<const float4 *>(ring + (size_t)(i % SEL_RING) * (SEL_RSTAGE / 4));
            const int k0 = i * kps, cnt = min(kps, n - k0);
            switch (G) {
            case 4: ring_tile_keys<1>(tile, k0, cnt, s_C, keys, s_hw[warp_id()]); break;
            case 8: ring_tile_keys<2>(tile, k0, cnt, s_C, keys, s_hw[warp_id()]); break;
            default: ring_tile_keys<4>(tile, k0, cnt, s_C, keys, s_hw[warp_id()]); break;
            }
            __syncthreads();  // every thread is done with this tile: its slot takes the next one
            if (tid == 0 && i + SEL_RING < ntile) issue_tile(i + SEL_RING);
        }
    } else {
        for (int base = (tid & ~31); base < n; base += SEL_T) {
            const int c = base + lane;
            const float sc = c < n ? key_of(lg + (int64_t)c * G) : 0.f;
            add_key(c, c < n, sc);
        }
    }
    __syncthreads();
    SKV_TRACE_CTA(TR_SEL_HIST);
    for (int t = tid; t < SEL_BINS; t += SEL_T) {
        unsigned h = 0;
#pragma unroll
        for (int w = 0; w < SEL_T / 32; ++w) h += s_hw[w][t];
        s_h1[t] = h;
    }
    SKV_TRACE_CTA(TR_SEL_KEYS);
    cluster_sync();  // every CTA's first-pass histogram is complete; rank 0's bitmaps are zero
    SKV_TRACE_CTA(TR_SEL_SYNC1);

    // 3) every CTA sums the CL histograms and finds the bin holding the K-th
    //    largest key.  Warp r copies CTA r's histogram into row r of this
    //    CTA's (now free) per-warp histograms, all CL remote reads at once;
    //    then warp 0, lane l summing bins 255-8l .. 248-8l, scans.
    if (warp_id() < CL) {
        const uint32_t ra = dsmem_addr(&s_h1[lane * 8], (unsigned)warp_id());
        const uint4 x = ld_dsmem_v4(ra), y = ld_dsmem_v4(ra + 16u);
        st_v4(&s_hw[warp_id()][lane * 8], x);
        st_v4(&s_hw[warp_id()][lane * 8 + 4], y);
    }
    __syncthreads();
    if (warp_id() == 0) {
        const int b0 = SEL_BINS - 8 - 8 * lane;
        uint4 lo[CL], hi[CL];
#pragma unroll
        for (unsigned r = 0; r < CL; ++r) {
            lo[r] = ld_v4(&s_hw[r][b0]);
            hi[r] = ld_v4(&s_hw[r][b0 + 4]);
        }
        int cnt[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // cnt[i]: bin b0 + 7 - i
#pragma unroll
        for (unsigned r = 0; r < CL; ++r) {
            cnt[0] += (int)hi[r].w;
            cnt[1] += (int)hi[r].z;
            cnt[2] += (int)hi[r].y;
            cnt[3] += (int)hi[r].x;
            cnt[4] += (int)lo[r].w;
            cnt[5] += (int)lo[r].z;
            cnt[6] += (int)lo[r].y;
            cnt[7] += (int)lo[r].x;
        }
        int tot = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) tot += cnt[i];
        int incl = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        int above = incl - tot;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (above < K && above + cnt[i] >= K) {
                s_bin = b0 + 7 - i;
                s_bin_above = above;
                s_bin_cnt = cnt[i];
            }
            above += cnt[i];
        }
    }
    __syncthreads();
    SKV_TRACE_CTA(TR_SEL_SCAN);
    SKV_TRACE_REC_NOW(3);
    const int bstar = s_bin, bin_above = s_bin_above, bin_cnt = s_bin_cnt;
    const uint32_t bmA0 = dsmem_addr(bmA, 0);
    auto chunk_of = [&](int c) -> int {
        if (lidx_s) return lidx_s[c];
        const int64_t v = lidx[c];
        return (v >= 0 && v < a.num_chunks) ? (int)v : -1;
    };
    auto mark = [&](int cid) {  // set the chunk in rank 0's bitmap of the new set
        if (cid >= 0) atom_or_dsmem_u32(bmA0 + 4u * (uint32_t)(cid >> 5), 1u << (cid & 31));
        else report_dev_error(DEV_ERR_HOST_CHUNK);
    };

    if (bin_cnt <= REGION) {
        // 4) keys above the boundary bin are selected; the keys inside it are
        //    the candidates.  CTA r pushes its candidates into region r of rank
        //    0's store and adds their count to rank 0's s_ccnt[r]: only
        //    fire-and-forget remote writes, no round trip.
        const uint32_t reg0 = (uint32_t)rank * REGION;
        const uint32_t ckey0 = dsmem_addr(s_ckey, 0), clm0 = dsmem_addr(s_clm, 0), cch0 = dsmem_addr(s_cchunk, 0);
        const uint32_t ccnt0 = dsmem_addr(&s_ccnt[rank], 0);
        int *lC = nullptr;
        unsigned char *stage = nullptr;
        if constexpr (FETCH) {
            lC = reinterpret_cast<int *>(smem_raw + a.list_off);
            stage = smem_raw + a.stage_off;  // the histograms and the logits ring are no longer read
            fence_proxy_async_smem();
        }
        for (int base = (tid & ~31); base < n; base += SEL_T) {
            const int c = base + lane;
            const uint32_t k = c < n ? keys[c] : 0u;
            const int bin = sel_key_bin(k);
            if (c < n && bin > bstar) {
                const int cid = chunk_of(c);
                mark(cid);
                if constexpr (FETCH) {
                    // a certain miss: listed here, its value requested after the barrier below
                    if (cid >= 0 && !((bmB[cid >> 5] >> (cid & 31)) & 1u)) {
                        const unsigned pos = atomicAdd(&s_nC, 1u);
                        if (pos < (unsigned)K) lC[pos] = cid;
                    }
                }
            }
            const bool cand = c < n && bin == bstar;
            const unsigned ballot = __ballot_sync(0xffffffffu, cand);
            if (ballot) {
                unsigned pos0 = 0;
                if (lane == 0) {
                    pos0 = atomicAdd(&s_nloc, (unsigned)__popc(ballot));
                    red_add_dsmem_u32(ccnt0, (unsigned)__popc(ballot));
                }
                pos0 = __shfl_sync(0xffffffffu, pos0, 0);
                if (cand) {
                    const uint32_t off = 4u * (reg0 + pos0 + __popc(ballot & ((1u << lane) - 1u)));
                    st_dsmem_u32(ckey0 + off, k);
                    st_dsmem_u32(clm0 + off, (uint32_t)(c0 + c));
                    st_dsmem_u32(cch0 + off, (uint32_t)chunk_of(c));
                }
            }
        }
        SKV_TRACE_CTA(TR_SEL_MARKED);
        if constexpr (FETCH) {
            // rank 0 holds the candidates and the bits of the keys above them once
            // every thread has arrived; the last warp requests the certain misses'
            // values between its arrival and its wait (a release issued while they
            // are in flight would wait for the host link)
            __syncthreads();  // the list of certain misses is complete
            {
                // ascending chunk ids (the order of the list decides the attention's
                // summation order: the same every run)
                const int nCk = min((int)s_nC, K);
                int *tmp = lC + 2 * K;
                for (int t = tid; t < nCk; t += SEL_T) {
                    const int v = lC[t];
                    int r = 0;
                    for (int j = 0; j < nCk; ++j) r += lC[j] < v ? 1 : 0;
                    tmp[r] = v;
                }
                __syncthreads();
                for (int t = tid; t < nCk; t += SEL_T) lC[t] = tmp[t];
                __syncthreads();
            }
            cluster_arrive_release();
            {
                // copy j is issued by warp j % 16, lane j / 16: the issue, which costs
                // each issuing thread a while per copy, is spread over every warp
                if (tid == 0) SKV_TRACE_R2(2);
                const int ne = fx_early_count((int)s_nC, K, a.cap, rank);
                const int j = (tid & 31) * (SEL_T / 32) + (tid >> 5);
                if (j < ne) {
                    uint64_t *tb = &s_vbar[j / (FETCH_ROWS / 8)];
                    mbar_expect_tx(tb, 2048u);
                    bulk_g2s(stage + (size_t)j * 2048, a.v_host + ((int64_t)bh * a.num_chunks + lC[j]) * 128, 2048u, tb);
                }
                if (tid == 0) SKV_TRACE_R2(3);
            }
            SKV_TRACE_REC_NOW(4);
            cluster_wait_acquire();
            SKV_TRACE_REC_NOW(5);
        } else {
            cluster_sync();  // rank 0 holds the candidates and the bits of the keys above them
            if (rank != 0) return;
        }
    }
    if (rank == 0 && bin_cnt <= REGION) {
        SKV_TRACE_CTA(TR_SEL_CAND);
        // the regions, compacted
        if (tid == 0) {
            int acc = 0;
            for (int r = 0; r < CL; ++r) {
                s_pre[r] = acc;
                acc += (int)s_ccnt[r];
            }
            s_pre[CL] = acc;
        }
        __syncthreads();
        for (int t = tid; t < SEL_CAND; t += SEL_T) {
            const int r = t / REGION, o = t % REGION;
            if (o < (int)s_ccnt[r]) {
                s_lord[s_pre[r] + o] = ((uint64_t)s_ckey[t] << 32) | (uint32_t)~s_clm[t];
                s_lchunk[s_pre[r] + o] = s_cchunk[t];
            }
        }
        __syncthreads();
        if (tid == 0) SKV_TRACE_R2(4);
        // 5) exact order among the candidates (key descending, landmark index
        //    ascending); the first K - bin_above of them are selected.  Two
        //    threads per candidate (nc <= REGION <= SEL_T / 2) count the
        //    order words above its own, each over half of the candidates.
        const int nc = s_pre[CL], need = K - bin_above;
        {
            const int i = tid >> 1;
            unsigned before = 0;
            if (i < nc) {
                const uint64_t oi = s_lord[i];
                for (int j = tid & 1; j < nc; j += 2) before += s_lord[j] > oi ? 1u : 0u;
            }
            before += __shfl_xor_sync(0xffffffffu, before, 1);
            if (i < nc && (tid & 1) == 0 && (int)before < need) {
                const int cid = s_lchunk[i];
                if (cid >= 0) {
                    atomicOr(&bmA[cid >> 5], 1u << (cid & 31));
                    // FETCH: a miss decided by the ranking (no CTA requested it at the scan)
                    if (FETCH && !((bmB[cid >> 5] >> (cid & 31)) & 1u))
                        atomicOr(reinterpret_cast<uint32_t *>(smem_raw + a.bmc_off) + (cid >> 5), 1u << (cid & 31));
                } else {
                    report_dev_error(DEV_ERR_HOST_CHUNK);
                }
            }
        }
    }
    if (bin_cnt > REGION) {
        // 4') more than REGION keys share the boundary bin (e.g. many equal
        //     scores): exact cluster-wide radix select, out of line
        select_radix_fallback<CL>(keys, n, K, c0, rank, lidx_s, lidx, a.num_chunks, bmA0, s_hist, s_tot, s_warp,
                                  s_eq_rank);
        cluster_sync();  // rank 0's bitmap holds the complete selection
        if constexpr (FETCH) {
        } else {
            if (rank != 0) return;
        }
    }
    if (rank == 0) {
    if (tid == 0) SKV_TRACE_R2(5);
    __syncthreads();
    SKV_TRACE_CTA(TR_SEL_RANKED);
    SKV_TRACE_REC_NOW(6);

    // 6) classify the cached slots against the new set; count the missed ids
    //    (in A, not in B) of this thread's bitmap words; one scan gives both
    //    the miss ranks (high half) and the free-slot ranks (low half)
#pragma unroll
    for (int u = 0; u < 2; ++u)
        if (old[u] >= 0 && old[u] < a.num_chunks) hit[u] = (bmA[old[u] >> 5] >> (old[u] & 31)) & 1;
    const int wpt = (nbw + SEL_T - 1) / SEL_T;
    const int w0 = tid * wpt;
    int local = 0;
    for (int w = w0; w < min(nbw, w0 + wpt); ++w) local += __popc(bmA[w] & ~bmB[w]);
    const int f0 = (2 * tid < K && !hit[0]) ? 1 : 0;
    const int f1 = (2 * tid + 1 < K && !hit[1]) ? 1 : 0;
    int tot;
    const int packed = cta_excl_scan((local << 16) | (f0 + f1), &tot, s_warp);
    const int nmiss = tot >> 16, nfree = tot & 0xffff;
    int rk = packed >> 16;
    const int r0 = packed & 0xffff;
    for (int w = w0; w < min(nbw, w0 + wpt); ++w) {
        uint32_t bits = bmA[w] & ~bmB[w];
        while (bits) {
            const int bit = __ffs(bits) - 1;
            bits &= bits - 1;
            if (rk < 1024) s_misssorted[rk] = w * 32 + bit;
            ++rk;
        }
    }
    __syncthreads();
    SKV_TRACE_CTA(TR_SEL_DIFF);

    // 7) refill the free slots (ascending) with the misses (ascending)
    const int nassign = min(nfree, nmiss);
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int f = u == 0 ? f0 : f1;
        const int r = u == 0 ? r0 : r0 + f0;
        const int sl = 2 * tid + u;
        if (f && r < nassign) {
            const int id = s_misssorted[r];
            slots[sl] = id;
            a.miss_slot[(int64_t)bh * K + r] = sl;
            a.miss_chunk[(int64_t)bh * K + r] = id;
            if constexpr (FETCH) reinterpret_cast<int *>(smem_raw + a.list_off)[K + r] = sl;  // slot of miss r
        }
    }
    if (tid == 0) {
        a.miss_count[bh] = nassign;
        if (nfree != nmiss) report_dev_error(DEV_ERR_SLOT);
    }
    if constexpr (FETCH) {
        if (tid == 0) SKV_TRACE_R2(6);
        // the message to every CTA: [count, 0], then (chunk id, slot) of miss r in
        // ascending id order, the slot negated-bit marked (bit 31) when the miss was
        // decided by the ranking or the exact fallback (no CTA requested it early)
        __syncthreads();
        const uint32_t *bmC = reinterpret_cast<const uint32_t *>(smem_raw + a.bmc_off);
        const int *slot_r = reinterpret_cast<const int *>(smem_raw + a.list_off) + K;
        const bool all_late = bin_cnt > REGION;
        auto pair = [&](int p) -> int2 {
            if (p == 0) return make_int2(nassign, 0);
            const int r = p - 1;
            if (r >= nassign) return make_int2(-1, -1);
            const int id = s_misssorted[r];
            const bool late = all_late || ((bmC[id >> 5] >> (id & 31)) & 1u);
            return make_int2(id, late ? (int)(0x80000000u | (unsigned)slot_r[r]) : slot_r[r]);
        };
        const int nw = (int)(fetch_msg_bytes(K) / 16);  // 16-byte words per message
        for (int w = tid; w < nw * CL; w += SEL_T) {
            const unsigned t = (unsigned)(w / nw);
            const int wi = w % nw;
            const int2 x = pair(2 * wi), y = pair(2 * wi + 1);
            st_async_v4(dsmem_addr(smem_raw + a.msg_off + (size_t)wi * 16, t),
                        make_uint4((unsigned)x.x, (unsigned)x.y, (unsigned)y.x, (unsigned)y.y), dsmem_addr(&s_mbar, t));
        }
    }
    SKV_TRACE_CTA(TR_SEL_END);
    SKV_TRACE_REC_NOW(7);
    }  // rank 0
    if constexpr (FETCH) fetch_tail(a, bh, rank, CL, smem_raw, &s_vbar[0], &s_mbar, s_nC, &s_nB, &s_ngrp);
    span_finish(a.span);  // (ranks other than 0 of a plain selection returned earlier)
}

size_t select_smem_bytes(int L, int num_chunks, int G, bool keys_global, int cl, bool keys_pre)
{
    // keys + chunk ids of the slice and bitmaps, then (128-byte aligned) the
    // per-warp histograms and the logits ring (none when the keys come ready)
    return ((select_base_bytes(L, num_chunks, keys_global, cl) + 127) & ~(size_t)127) +
           (size_t)(SEL_T / 32) * SEL_BINS * 4 + (keys_pre ? 0 : select_ring_bytes(L, G, cl));
}

// Keys of landmarks [r0, r1) of head bh, one thread per landmark, G = 4Q logits per row.
template <int Q>
__device__ __forceinline__ void keys_rows(const KeysArgs &k, int bh, int r0, int r1, const float *s_C)
{
    for (int c = r0 + (int)threadIdx.x; c < r1; c += KEYS_T) {
        const float4 *row = reinterpret_cast<const float4 *>(k.logits + ((int64_t)bh * k.L + c) * (4 * Q));
        float4 v[Q];
#pragma unroll
        for (int q = 0; q < Q; ++q) v[q] = row[q];
        float d = -INFINITY;
#pragma unroll
        for (int q = 0; q < Q; ++q) {
            d = fmaxf(fmaxf(d, v[q].x - s_C[4 * q]), v[q].y - s_C[4 * q + 1]);
            d = fmaxf(fmaxf(d, v[q].z - s_C[4 * q + 2]), v[q].w - s_C[4 * q + 3]);
        }
        k.keys[(int64_t)bh * k.L + c] = __float_as_uint(__expf(d));
    }
}

__global__ void __launch_bounds__(KEYS_T) keys_kernel(KeysArgs k)
{
    __shared__ float s_C[16];
    const int bh = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = k.G, L = k.L;
    pdl_launch_dependents();  // the selection may become resident; it waits for this grid
    pdl_wait();               // the scoring kernel's logits and partials are complete
    for (int gg = warp; gg < G; gg += KEYS_T / 32) {
        const float C = merge_partials(k.part, bh, k.nsplit, G, gg, lane);
        if (lane == 0) s_C[gg] = C;
    }
    __syncthreads();
    const int r0 = blockIdx.x * k.rows, r1 = min(L, r0 + k.rows);
    switch (G) {  // a row's 16-byte words all in flight at once
    case 4: keys_rows<1>(k, bh, r0, r1, s_C); break;
    case 8: keys_rows<2>(k, bh, r0, r1, s_C); break;
    case 16: keys_rows<4>(k, bh, r0, r1, s_C); break;
    default:
        for (int c = r0 + tid; c < r1; c += KEYS_T) {
            const float *row = k.logits + ((int64_t)bh * L + c) * G;
            float d = -INFINITY;
            for (int gg = 0; gg < G; ++gg) d = fmaxf(d, row[gg] - s_C[gg]);
            k.keys[(int64_t)bh * L + c] = __float_as_uint(__expf(d));
        }
    }
}

int launch_keys(const KeysArgs &k, int BH, cudaStream_t stream)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((k.L + k.rows - 1) / k.rows, BH, 1);
    cfg.blockDim = dim3(KEYS_T, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, keys_kernel, k);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("launch of keys_kernel failed: %s", cudaGetErrorString(e));
        return SKV_ERR_CUDA;
    }
    return SKV_OK;
}

// Whether this device can schedule 16-CTA clusters of the selection kernel
// (a non-portable cluster size) with `smem` bytes of dynamic shared memory per
// CTA.  Decided once per device, probed at SEL_SMEM_CAP -- the largest size
// plan_select asks for -- so a yes holds for every smaller plan.
bool select_cluster16_ok(size_t smem)
{
    if (smem > SEL_SMEM_CAP) return false;
    static std::atomic<int> cached[64];  // 0: not probed yet, 1: yes, -1: no (host threads may race here)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return false;
    }
    const int known = cached[dev].load(std::memory_order_relaxed);
    if (known) return known > 0;
    int ok = -1;
    const void *fn = (const void *)select_cluster_kernel<16, false>;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess &&
        ensure_smem_attr(fn, (int)SEL_SMEM_CAP, "select_cluster_kernel<16>") == SKV_OK) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(16, 1, 1);
        cfg.blockDim = dim3(SEL_T, 1, 1);
        cfg.dynamicSmemBytes = SEL_SMEM_CAP;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 16;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) == cudaSuccess && n >= 1) ok = 1;
    }
    cudaGetLastError();
    cached[dev].store(ok, std::memory_order_relaxed);
    return ok > 0;
}

FetchLayout fetch_layout(int L, int num_chunks, int G, int K, int rank, int buf_len)
{
    FetchLayout f = {};
    auto a128 = [](size_t x) { return (x + 127) & ~(size_t)127; };
    const size_t base = a128(select_base_bytes(L, num_chunks, false, SEL_CL));
    const size_t hist_ring = (size_t)(SEL_T / 32) * SEL_BINS * 4 + select_ring_bytes(L, G, SEL_CL);
    const size_t list = a128((size_t)4 * K * 4), msg = a128(fetch_msg_bytes(K));
    const size_t bmc = a128((size_t)((num_chunks + 31) / 32) * 4);
    const size_t recon = a128((size_t)FETCH_ROWS * fetch_kt(rank) * 2 + (size_t)128 * (rank + 8) * 2 +
                              (size_t)FETCH_ROWS * FETCH_PITCH * 2);
    // the largest staging area that fits; the attention region reuses the
    // selection's keys, ids and bitmaps when it fits there (they are no longer
    // read once rank 0's message is out), else it comes on top
    for (int cap = 64; cap >= 16; --cap) {
        const FxAttLayout at = fx_att_layout(G, cap, buf_len, K);
        const size_t att = at.bytes <= base ? 0 : a128(at.bytes);
        const size_t stage = a128((size_t)cap * 2048) > a128(hist_ring) ? a128((size_t)cap * 2048) : a128(hist_ring);
        const size_t bytes = base + stage + list + msg + bmc + recon + att;
        if (bytes > FETCH_SMEM_CAP) continue;
        f.cap = cap;
        f.stage_off = (unsigned)base;
        f.list_off = (unsigned)(base + stage);
        f.msg_off = (unsigned)(f.list_off + list);
        f.bmc_off = (unsigned)(f.msg_off + msg);
        f.recon_off = (unsigned)(f.bmc_off + bmc);
        f.att_off = att ? (unsigned)(f.recon_off + recon) : 0u;
        f.bytes = (unsigned)bytes;
        return f;
    }
    return f;  // fewer than 16 chunks staged at once: not used
}

int launch_select_fetch(const SelectArgs &a, int BH, size_t smem, cudaStream_t stream)
{
    const void *fn = (const void *)select_cluster_kernel<SEL_CL, true>;
    int st = ensure_smem_attr(fn, (int)smem, "select_cluster_kernel<fetch>");
    if (st) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(SEL_CL, BH, 1);
    cfg.blockDim = dim3(SEL_T, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = SEL_CL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaError_t e = cudaLaunchKernelEx(&cfg, select_cluster_kernel<SEL_CL, true>, a);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("launch of select_cluster_kernel<fetch> failed: %s", cudaGetErrorString(e));
        return SKV_ERR_CUDA;
    }
    return SKV_OK;
}

int launch_select(const SelectArgs &a, int BH, size_t smem, int cl, cudaStream_t stream)
{
    const void *fn = cl == 16 ? (const void *)select_cluster_kernel<16, false> : (const void *)select_cluster_kernel<8, false>;
    int st = ensure_smem_attr(fn, (int)smem, "select_cluster_kernel");
    if (st) return st;
    if (cl == 16 && cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
        cudaGetLastError();
        set_error("16-CTA clusters not available for select_cluster_kernel");
        return SKV_ERR_CUDA;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(cl, BH, 1);
    cfg.blockDim = dim3(SEL_T, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    // may start while the scoring kernel drains; it reads the scores only after pdl_wait()
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaError_t e = cl == 16 ? cudaLaunchKernelEx(&cfg, select_cluster_kernel<16, false>, a)
                             : cudaLaunchKernelEx(&cfg, select_cluster_kernel<8, false>, a);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("launch of select_cluster_kernel failed: %s", cudaGetErrorString(e));
        return SKV_ERR_CUDA;
    }
    return SKV_OK;
}

}  // namespace skv
