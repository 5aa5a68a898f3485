// Top-k chunk selection and slot-stable reuse diff of the fused decode path.
//
// Reference: the selection of models/kvcache/shadow.py:567-573 (torch.max over
// the GQA group, torch.topk of select_sets chunks, gather through
// k_landmark_idx) and the reuse-cache diff of kernels/map.cuh:475-516.
//
// One 8-CTA thread-block cluster per (b, kv head).  Every CTA turns its
// eighth of the landmarks into order-preserving keys (max over the group of
// the softmax-normalised score), then the cluster runs a 4-pass radix select
// (8 bits per pass): each CTA builds a private histogram, the cluster barrier
// publishes it, and every CTA sums the eight histograms through distributed
// shared memory.  Selected landmarks are appended to rank 0's list with
// cluster-scope shared-memory atomics (one per warp); when the k-th score is
// tied the lowest landmark indices win.  Rank 0 then maps landmarks to chunk
// ids and computes the slot-stable diff with two shared-memory bitmaps.
#include "select.cuh"

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
__device__ __forceinline__ uint32_t atom_add_dsmem_u32(uint32_t addr, uint32_t v)
{
    uint32_t old;
    asm volatile("atom.shared::cluster.add.u32 %0, [%1], %2;" : "=r"(old) : "r"(addr), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void cluster_sync()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n"
                 "barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
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

__global__ void __launch_bounds__(SEL_T) select_cluster_kernel(SelectArgs a)
{
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ float s_M[16], s_invZ[16];
    __shared__ unsigned s_hist[2][256];
    __shared__ unsigned s_tot[256];
    __shared__ int s_warp[33];
    __shared__ int s_sel[1024];        // rank 0: selected landmark index, then chunk id
    __shared__ int s_misssorted[1024]; // rank 0: missed chunk ids, ascending
    __shared__ unsigned s_cnt;         // rank 0: append position of the selected list
    __shared__ int s_digit, s_above;
    __shared__ unsigned s_eq_rank[SEL_CL];

    const unsigned rank = blockIdx.x;
    const int bh = blockIdx.y, tid = threadIdx.x, lane = tid & 31;
    const int G = a.G, L = a.L, K = a.K;
    const int slice = (L + SEL_CL - 1) / SEL_CL;
    const int c0 = (int)rank * slice;
    const int n = max(0, min(L, c0 + slice) - c0);
    const int nbw = (a.num_chunks + 31) >> 5;
    uint32_t *dyn = reinterpret_cast<uint32_t *>(smem_raw);
    uint32_t *keys = a.gkeys ? a.gkeys + (int64_t)bh * L + c0 : dyn;
    uint32_t *bmA = a.gkeys ? dyn : dyn + slice;
    uint32_t *bmB = bmA + nbw;

    if (tid == 0) s_cnt = 0;

    // 1) softmax normalisers of each query head of the group: warp w merges the
    //    split partials of head w (lanes load in parallel, then a shuffle merge)
    if (warp_id() < G) {
        const int gg = warp_id();
        float mm = -INFINITY, ss = 0.f;
        for (int i = lane; i < a.nsplit; i += 32) {
            const float2 p = a.part[((int64_t)bh * a.nsplit + i) * G + gg];
            merge_ms(mm, ss, p.x, p.y);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float m2 = __shfl_xor_sync(0xffffffffu, mm, o);
            const float s2 = __shfl_xor_sync(0xffffffffu, ss, o);
            merge_ms(mm, ss, m2, s2);
        }
        if (lane == 0) {
            s_M[gg] = mm;
            s_invZ[gg] = 1.f / ss;
        }
    }
    __syncthreads();

    // 2) keys of this CTA's landmarks: bits of max_g softmax_g (>= 0, so the
    //    unsigned order of the bits is the order of the scores)
    const float *lg = a.logits + ((int64_t)bh * L + c0) * G;
    if ((G & 3) == 0) {
        constexpr int U = 4;
        const int G4 = G >> 2;
        for (int base = tid; base < n; base += U * SEL_T) {
            float4 v[U][4];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = base + u * SEL_T;
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4)
                    if (q4 < G4 && c < n) v[u][q4] = __ldcg(reinterpret_cast<const float4 *>(lg + (int64_t)c * G) + q4);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int c = base + u * SEL_T;
                if (c >= n) continue;
                float sc = 0.f;
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    if (q4 < G4) {
                        sc = fmaxf(sc, __expf(v[u][q4].x - s_M[4 * q4 + 0]) * s_invZ[4 * q4 + 0]);
                        sc = fmaxf(sc, __expf(v[u][q4].y - s_M[4 * q4 + 1]) * s_invZ[4 * q4 + 1]);
                        sc = fmaxf(sc, __expf(v[u][q4].z - s_M[4 * q4 + 2]) * s_invZ[4 * q4 + 2]);
                        sc = fmaxf(sc, __expf(v[u][q4].w - s_M[4 * q4 + 3]) * s_invZ[4 * q4 + 3]);
                    }
                }
                keys[c] = __float_as_uint(sc);
            }
        }
    } else {
        for (int c = tid; c < n; c += SEL_T) {
            float sc = 0.f;
            for (int gg = 0; gg < G; ++gg) sc = fmaxf(sc, __expf(lg[(int64_t)c * G + gg] - s_M[gg]) * s_invZ[gg]);
            keys[c] = __float_as_uint(sc);
        }
    }

    // 3) cluster-wide radix select of the K-th largest key
    uint32_t prefix = 0, pmask = 0;
    int remaining = K, n_equal = 0;
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        unsigned *h = s_hist[pass & 1];
        if (tid < 256) h[tid] = 0;
        __syncthreads();
        for (int base = 0; base < n; base += SEL_T) {
            const int c = base + tid;
            const uint32_t k = c < n ? keys[c] : 0u;
            const bool part = c < n && (k & pmask) == prefix;
            const int bin = part ? (int)((k >> shift) & 255) : 256 + lane;
            const unsigned peers = __match_any_sync(0xffffffffu, bin);
            if (part && lane == __ffs(peers) - 1) atomicAdd(&h[bin], (unsigned)__popc(peers));
        }
        cluster_sync();  // every CTA's histogram of this pass is complete
        if (tid < 256) {
            unsigned t = 0;
#pragma unroll
            for (unsigned r = 0; r < SEL_CL; ++r) t += ld_dsmem_u32(dsmem_addr(&h[tid], r));
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
            if (tid < SEL_CL) s_eq_rank[tid] = ld_dsmem_u32(dsmem_addr(&h[d], tid));
        }
        __syncthreads();
    }
    const uint32_t T = prefix;     // the K-th largest key
    const int ngt = K - remaining;  // keys strictly above T

    // 4) append the selected landmarks to rank 0's list
    const bool take_all_equal = n_equal == remaining;
    const uint32_t cnt_addr = dsmem_addr(&s_cnt, 0);
    const uint32_t sel_addr = dsmem_addr(&s_sel[0], 0);
    for (int base = 0; base < n; base += SEL_T) {
        const int c = base + tid;
        const uint32_t k = c < n ? keys[c] : 0u;
        const bool take = c < n && (k > T || (take_all_equal && k == T));
        const unsigned ballot = __ballot_sync(0xffffffffu, take);
        if (ballot) {
            unsigned pos0 = 0;
            if (lane == 0) pos0 = atom_add_dsmem_u32(cnt_addr, (unsigned)__popc(ballot));
            pos0 = __shfl_sync(0xffffffffu, pos0, 0);
            if (take) st_dsmem_u32(sel_addr + 4u * (pos0 + __popc(ballot & ((1u << lane) - 1u))), (uint32_t)(c0 + c));
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
            if (f && taken + r < quota) st_dsmem_u32(sel_addr + 4u * (ngt + before + taken + r), (uint32_t)(c0 + c));
            taken += tot;
        }
    }
    cluster_sync();  // rank 0 holds the complete selection
    if (rank != 0) return;

    // 5) landmark -> chunk id; bitmap A of the new set
    for (int w = tid; w < 2 * nbw; w += SEL_T) bmA[w] = 0;  // bmA and bmB are contiguous
    __syncthreads();
    const int64_t *lidx = a.landmark_idx + (int64_t)bh * L;
    for (int jj = tid; jj < K; jj += SEL_T) {
        const int lm = s_sel[jj];
        const int64_t cid = (lm >= 0 && lm < L) ? lidx[lm] : -1;
        int v = -1;
        if (cid >= 0 && cid < a.num_chunks) {
            v = (int)cid;
            atomicOr(&bmA[v >> 5], 1u << (v & 31));
        } else {
            report_dev_error(DEV_ERR_HOST_CHUNK);
        }
        s_sel[jj] = v;
    }
    __syncthreads();

    // 6) classify the cached slots (thread t owns slots 2t, 2t+1); bitmap B of the cached set
    int32_t *slots = a.slots + (int64_t)bh * K;
    int hit[2] = {0, 0};
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int s = 2 * tid + u;
        if (s < K) {
            const int old = slots[s];
            if (old >= 0 && old < a.num_chunks) {
                hit[u] = (bmA[old >> 5] >> (old & 31)) & 1;
                atomicOr(&bmB[old >> 5], 1u << (old & 31));
            }
        }
    }
    __syncthreads();

    // 7) missed ids (in A, not in B) in ascending order
    const int wpt = (nbw + SEL_T - 1) / SEL_T;
    const int w0 = tid * wpt;
    int local = 0;
    for (int w = w0; w < min(nbw, w0 + wpt); ++w) local += __popc(bmA[w] & ~bmB[w]);
    int nmiss;
    int rk = cta_excl_scan(local, &nmiss, s_warp);
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

    // 8) refill the free slots (ascending) with the misses (ascending)
    const int f0 = (2 * tid < K && !hit[0]) ? 1 : 0;
    const int f1 = (2 * tid + 1 < K && !hit[1]) ? 1 : 0;
    int nfree;
    const int r0 = cta_excl_scan(f0 + f1, &nfree, s_warp);
    const int nassign = min(nfree, nmiss);
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int f = u == 0 ? f0 : f1;
        const int r = u == 0 ? r0 : r0 + f0;
        const int s = 2 * tid + u;
        if (f && r < nassign) {
            const int id = s_misssorted[r];
            slots[s] = id;
            a.miss_slot[(int64_t)bh * K + r] = s;
            a.miss_chunk[(int64_t)bh * K + r] = id;
        }
    }
    if (tid == 0) {
        a.miss_count[bh] = nassign;
        if (nfree != nmiss) report_dev_error(DEV_ERR_SLOT);
    }
}

size_t select_smem_bytes(int L, int num_chunks, bool keys_global)
{
    const size_t slice = (size_t)((L + SEL_CL - 1) / SEL_CL);
    const size_t nbw = (size_t)((num_chunks + 31) / 32);
    return (keys_global ? 0 : slice * 4) + 2 * nbw * 4;
}

int launch_select(const SelectArgs &a, int BH, size_t smem, cudaStream_t stream)
{
    int st = ensure_smem_attr((const void *)select_cluster_kernel, (int)smem, "select_cluster_kernel");
    if (st) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(SEL_CL, BH, 1);
    cfg.blockDim = dim3(SEL_T, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = SEL_CL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, select_cluster_kernel, a);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("launch of select_cluster_kernel failed: %s", cudaGetErrorString(e));
        return SKV_ERR_CUDA;
    }
    return SKV_OK;
}

}  // namespace skv
