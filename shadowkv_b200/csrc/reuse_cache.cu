// Reuse cache of selected chunks: reorder/diff, in-place compaction of hits,
// zero-copy fetch of misses from page-locked host memory.
//
// Reference (WilliamBy/ShadowKV): kernels/map.cuh (hash diff + sorts),
// kernels/copy.cuh (gather/copy kernels), kernels/gather_copy.cu (launchers).
//
// Design for sm_100a:
//  * reorder: one CTA per (b,h); the cached ids are sorted in shared memory
//    (bitonic, key|slot composite) and each new id is located by binary
//    search -- deterministic for any map size 1..1024 (the reference hash
//    handles 128/256/512/1024 only).
//  * compaction + miss fetch: one 8-CTA thread-block cluster per (b,h).
//    Every thread first loads its share of all source chunks (old device
//    slot for hits, host chunk for misses) into registers, the cluster
//    barrier orders all reads of the head before any write, then every
//    thread stores.  This replaces the reference's two-CTA scheme with a
//    temp buffer and an unbounded inter-CTA spin (copy.cuh:86-113,
//    489-497): no spin-wait, no temp round trip, 8x the parallelism.
//  * slot-stable miss fetch (fused decode path): hits never move; only the
//    missed chunks are read from host memory, by many CTAs.
#include "common.cuh"

namespace skv {

constexpr int CHUNK_BYTES = 2048;            // 8 tokens x 128 dims x bf16
constexpr int CHUNK_V4 = CHUNK_BYTES / 16;   // 128 16-byte pieces
constexpr int CHUNK_ELEMS = 1024;            // bf16 elements per chunk
constexpr int REUSE_CLUSTER = 8;

// ---------------------------------------------------------------------------
// block-wide helpers (blockDim.x threads, <= 1024)
// ---------------------------------------------------------------------------

// Exclusive prefix sum of `v` over the block; *total gets the sum.
__device__ int block_exclusive_scan(int v, int *total, int *s_warp)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nwarps = (blockDim.x + 31) >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int w = lane < nwarps ? s_warp[lane] : 0;
        int wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += y;
        }
        if (lane < nwarps) s_warp[lane] = wi - w;  // exclusive warp offsets
        if (lane == nwarps - 1) s_warp[32] = wi;
    }
    __syncthreads();
    int r = s_warp[warp] + x - v;
    *total = s_warp[32];
    __syncthreads();
    return r;
}

template <typename T>
__device__ void block_bitonic_sort(T *s, int n /* power of two == blockDim.x */)
{
    const int tid = threadIdx.x;
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            __syncthreads();
            int ixj = tid ^ j;
            if (ixj > tid) {
                bool up = (tid & k) == 0;
                T a = s[tid], b = s[ixj];
                if ((a > b) == up) {
                    s[tid] = b;
                    s[ixj] = a;
                }
            }
        }
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------
// reorder_keys_and_compute_offsets (map.cuh:475-516 semantics)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) reorder_kernel(int64_t *cached, const int64_t *cur,
                                                       int32_t *offsets, int32_t *cnts, int M)
{
    __shared__ unsigned long long s_old[1024];
    __shared__ int s_hitkey[1024];
    __shared__ int s_miss[1024];
    __shared__ int s_warp[33];
    const int P = blockDim.x;
    const int tid = threadIdx.x;
    const int64_t base = (int64_t)blockIdx.x * M;
    const int HIT_NONE = INT32_MIN;

    int newkey = 0;
    if (tid < M) {
        int ok = (int)cached[base + tid];  // ids are truncated to int32 like the reference
        newkey = (int)cur[base + tid];
        s_old[tid] = ((unsigned long long)((uint32_t)ok ^ 0x80000000u) << 32) | (uint32_t)tid;
    } else {
        s_old[tid] = ~0ull;
    }
    s_hitkey[tid] = HIT_NONE;
    block_bitonic_sort(s_old, P);

    // locate the new id among the cached ids (lowest slot for repeated ids)
    int hit_slot = -1;
    if (tid < M) {
        const uint32_t kb = (uint32_t)newkey ^ 0x80000000u;
        int lo = 0, hi = P;
        while (lo < hi) {
            int mid = (lo + hi) >> 1;
            if ((uint32_t)(s_old[mid] >> 32) < kb) lo = mid + 1;
            else hi = mid;
        }
        if (lo < P && (uint32_t)(s_old[lo] >> 32) == kb) {
            int slot = (int)(uint32_t)(s_old[lo] & 0xffffffffu);
            if (slot < M) hit_slot = slot;
        }
        if (hit_slot >= 0) s_hitkey[hit_slot] = newkey;
    }
    s_miss[tid] = (tid < M && hit_slot < 0) ? newkey : INT32_MAX;
    block_bitonic_sort(s_miss, P);  // misses ascending; ends with __syncthreads

    // hits in old-slot order
    const int is_hit = (tid < M && s_hitkey[tid] != HIT_NONE) ? 1 : 0;
    int nhit = 0;
    const int pos = block_exclusive_scan(is_hit, &nhit, s_warp);
    if (is_hit) {
        cached[base + pos] = (int64_t)s_hitkey[tid];
        offsets[base + pos] = tid;
    }
    if (tid < M - nhit) {
        int key = s_miss[tid];
        cached[base + nhit + tid] = (int64_t)key;
        offsets[base + nhit + tid] = key;
    }
    if (tid == 0) cnts[blockIdx.x] = nhit;
}

// ---------------------------------------------------------------------------
// In-place hit compaction (+ optional host miss fetch) with a cluster barrier.
// grid = (REUSE_CLUSTER, nblocks), cluster = (REUSE_CLUSTER, 1, 1), 256 threads.
// Slots are processed in rounds of 256 (32 per CTA, 16 pieces per thread).
// Within a round every read happens before the cluster barrier and every
// write after it.  Across rounds no barrier is needed: a hit of slot j reads
// old slot offsets[j] >= j (offsets of hits ascend), so a round never reads a
// slot that an earlier round wrote, and a round's writes wait for every CTA
// to finish that round's reads, which follow all of its earlier reads.
// ---------------------------------------------------------------------------
constexpr int MOVE_THREADS = 256;
constexpr int MOVE_SLOTS_PER_CTA = 32;
constexpr int MOVE_ITEMS = MOVE_SLOTS_PER_CTA * CHUNK_V4 / MOVE_THREADS;  // 16
constexpr int MOVE_ROUND = MOVE_SLOTS_PER_CTA * REUSE_CLUSTER;            // 256

template <bool FETCH_MISSES>
__global__ void __launch_bounds__(MOVE_THREADS) reuse_move_kernel(
    const uint4 *__restrict__ host, uint4 *buf, const int32_t *__restrict__ offsets,
    const int32_t *__restrict__ cnts, int M, int64_t host_stride_v4, int64_t host_chunks,
    int64_t buf_stride_v4, int64_t buf_offset_v4)
{
    const int bid = blockIdx.y;
    const int cnt = cnts[bid];
    const int32_t *off = offsets + (int64_t)bid * M;
    uint4 *region = buf + (int64_t)bid * buf_stride_v4 + buf_offset_v4;
    const uint4 *hregion = host + (int64_t)bid * host_stride_v4;
    const int rounds = (M + MOVE_ROUND - 1) / MOVE_ROUND;

    for (int rd = 0; rd < rounds; ++rd) {
        const int slot0 = rd * MOVE_ROUND + blockIdx.x * MOVE_SLOTS_PER_CTA;
        uint4 data[MOVE_ITEMS];
        bool act[MOVE_ITEMS];
#pragma unroll
        for (int t = 0; t < MOVE_ITEMS; ++t) {
            const int u = threadIdx.x + t * MOVE_THREADS;
            const int slot = slot0 + u / CHUNK_V4;
            const int piece = u % CHUNK_V4;
            act[t] = false;
            if (slot < M) {
                const int o = off[slot];
                if (slot < cnt) {
                    if (o != slot) {
                        if (o >= slot && o < M) {
                            data[t] = __ldcg(region + (int64_t)o * CHUNK_V4 + piece);
                            act[t] = true;
                        } else if (piece == 0) {
                            report_dev_error(DEV_ERR_SLOT);
                        }
                    }
                } else if (FETCH_MISSES) {
                    if (o >= 0 && o < host_chunks) {
                        data[t] = ld_stream_v4(hregion + (int64_t)o * CHUNK_V4 + piece);
                        act[t] = true;
                    } else if (piece == 0) {
                        report_dev_error(DEV_ERR_HOST_CHUNK);
                    }
                }
            }
        }
        // every read of this round of the (b,h) block happens before any write of it
        asm volatile("barrier.cluster.arrive.release.aligned;\n"
                     "barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
#pragma unroll
        for (int t = 0; t < MOVE_ITEMS; ++t) {
            if (act[t]) {
                const int u = threadIdx.x + t * MOVE_THREADS;
                const int slot = slot0 + u / CHUNK_V4;
                const int piece = u % CHUNK_V4;
                __stcg(region + (int64_t)slot * CHUNK_V4 + piece, data[t]);
            }
        }
    }
}

template <bool FETCH>
static int launch_reuse_move(const void *host_dev, void *buf, const int32_t *offsets,
                             const int32_t *cnts, int nblocks, int M, int64_t host_stride_elems,
                             int64_t host_chunks, int64_t buf_stride_elems,
                             int64_t buf_offset_elems, cudaStream_t stream)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(REUSE_CLUSTER, nblocks, 1);
    cfg.blockDim = dim3(MOVE_THREADS, 1, 1);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = REUSE_CLUSTER;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const uint4 *h = reinterpret_cast<const uint4 *>(host_dev);
    uint4 *b = reinterpret_cast<uint4 *>(buf);
    const int64_t hs = host_stride_elems / 8, bs = buf_stride_elems / 8, bo = buf_offset_elems / 8;
    cudaError_t e = cudaLaunchKernelEx(&cfg, reuse_move_kernel<FETCH>, h, b, offsets, cnts, M, hs,
                                       host_chunks, bs, bo);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("launch of reuse_move_kernel failed: %s", cudaGetErrorString(e));
        return SKV_ERR_CUDA;
    }
    return SKV_OK;
}

// ---------------------------------------------------------------------------
// gather_copy: every slot from host (copy.cuh:248-274 semantics)
// grid = (ceil(M/16), nblocks), 256 threads, 8 pieces per thread.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) gather_copy_kernel(const uint4 *__restrict__ host,
                                                          uint4 *__restrict__ buf,
                                                          const int64_t *__restrict__ ids, int M,
                                                          int64_t host_stride_v4,
                                                          int64_t host_chunks,
                                                          int64_t buf_stride_v4)
{
    const int bid = blockIdx.y;
    const int slot0 = blockIdx.x * 16;
    uint4 data[8];
    int64_t src[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        const int u = threadIdx.x + t * 256;
        const int slot = slot0 + u / CHUNK_V4;
        src[t] = -1;
        if (slot < M) {
            const int64_t id = (int64_t)(int32_t)ids[(int64_t)bid * M + slot];
            if (id >= 0 && id < host_chunks)
                src[t] = (int64_t)bid * host_stride_v4 + id * CHUNK_V4 + (u % CHUNK_V4);
            else if ((u % CHUNK_V4) == 0)
                report_dev_error(DEV_ERR_HOST_CHUNK);
        }
    }
#pragma unroll
    for (int t = 0; t < 8; ++t)
        if (src[t] >= 0) data[t] = ld_stream_v4(host + src[t]);
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        if (src[t] >= 0) {
            const int u = threadIdx.x + t * 256;
            const int slot = slot0 + u / CHUNK_V4;
            __stcg(buf + (int64_t)bid * buf_stride_v4 + (int64_t)slot * CHUNK_V4 + (u % CHUNK_V4),
                   data[t]);
        }
    }
}

// ---------------------------------------------------------------------------
// Fused decode path: fetch the missed chunks only (slot-stable cache).
// grid = (ceil(M/16), B*H), 256 threads; entry j = blockIdx.x*16 + u/128.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) fetch_misses_kernel(
    const uint4 *__restrict__ host, uint4 *__restrict__ buf, const int32_t *__restrict__ miss_slot,
    const int32_t *__restrict__ miss_chunk, const int32_t *__restrict__ miss_count, int M,
    int num_chunks, int buf_len, int sparse_start)
{
    const int bh = blockIdx.y;
    const int j0 = blockIdx.x * 16;
    const int nmiss = miss_count[bh];
    if (j0 >= nmiss) return;
    uint4 data[8];
    int64_t dst[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) {
        const int u = threadIdx.x + t * 256;
        const int j = j0 + u / CHUNK_V4;
        const int piece = u % CHUNK_V4;
        dst[t] = -1;
        if (j < nmiss) {
            const int chunk = miss_chunk[(int64_t)bh * M + j];
            const int slot = miss_slot[(int64_t)bh * M + j];
            if (chunk >= 0 && chunk < num_chunks && slot >= 0 && slot < M) {
                data[t] = ld_stream_v4(host + ((int64_t)bh * num_chunks + chunk) * CHUNK_V4 + piece);
                dst[t] = ((int64_t)bh * buf_len + sparse_start + (int64_t)slot * 8) * 16 + piece;
            } else if (piece == 0) {
                report_dev_error(chunk < 0 || chunk >= num_chunks ? DEV_ERR_HOST_CHUNK : DEV_ERR_SLOT);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < 8; ++t)
        if (dst[t] >= 0) __stcg(buf + dst[t], data[t]);
}

int launch_fetch_misses(const skv_decode_geom *g, const void *v_host_dev, void *v_buf,
                        const int32_t *miss_slot, const int32_t *miss_chunk,
                        const int32_t *miss_count, cudaStream_t stream)
{
    dim3 grid(ceil_div(g->select_sets, 16), g->batch * g->kv_heads);
    fetch_misses_kernel<<<grid, 256, 0, stream>>>(
        reinterpret_cast<const uint4 *>(v_host_dev), reinterpret_cast<uint4 *>(v_buf), miss_slot,
        miss_chunk, miss_count, g->select_sets, g->num_chunks, g->buf_len, g->sparse_start);
    return check_launch("fetch_misses_kernel");
}

}  // namespace skv

using namespace skv;

extern "C" {

int skv_reorder_keys_and_compute_offsets(int64_t *cached_pos_ids, const int64_t *cur_pos_ids,
                                         int32_t *offsets, int32_t *cnts, int batch_size,
                                         int heads, int map_size, void *stream)
{
    SKV_CHECK_ARG(cached_pos_ids && cur_pos_ids && offsets && cnts, "null pointer argument");
    SKV_CHECK_ARG(batch_size > 0 && heads > 0, "batch_size and heads must be positive");
    SKV_CHECK_SUPPORTED(map_size >= 1 && map_size <= 1024, "map_size %d outside 1..1024", map_size);
    int P = 32;
    while (P < map_size) P <<= 1;
    reorder_kernel<<<batch_size * heads, P, 0, (cudaStream_t)stream>>>(cached_pos_ids, cur_pos_ids,
                                                                      offsets, cnts, map_size);
    return check_launch("reorder_kernel");
}

int skv_gather_copy_with_offsets(const void *values, void *v_cache_buffer, void *temp,
                                 const int32_t *offsets, const int32_t *cnts, int32_t *signals,
                                 int batch_size, int heads, int cpu_v_length, int gpu_v_length,
                                 int gpu_v_offset, int gpu_v_stride, int map_size, void *stream)
{
    (void)temp;
    (void)signals;
    (void)gpu_v_length;
    SKV_CHECK_ARG(v_cache_buffer && offsets && cnts, "null pointer argument");
    SKV_CHECK_ARG(batch_size > 0 && heads > 0, "batch_size and heads must be positive");
    SKV_CHECK_SUPPORTED(map_size >= 1 && map_size <= 1024, "map_size %d outside 1..1024", map_size);
    SKV_CHECK_ARG(cpu_v_length > 0 && cpu_v_length % CHUNK_ELEMS == 0,
                  "cpu_v_length must be a positive multiple of 1024");
    SKV_CHECK_ARG(gpu_v_offset >= 0 && gpu_v_offset % 8 == 0 && gpu_v_stride % 8 == 0,
                  "gpu_v_offset/gpu_v_stride must be multiples of 8 elements");
    SKV_CHECK_ARG((int64_t)gpu_v_offset + (int64_t)map_size * CHUNK_ELEMS <= gpu_v_stride ||
                      batch_size * heads == 1,
                  "gpu_v_offset + map_size*1024 exceeds gpu_v_stride");
    SKV_CHECK_ARG(aligned(v_cache_buffer, 16), "v_cache_buffer must be 16-byte aligned");
    const void *hdev = nullptr;
    int st = host_to_device_ptr(values, &hdev, "values");
    if (st != SKV_OK) return st;
    SKV_CHECK_ARG(aligned(hdev, 16), "values must be 16-byte aligned");
    return launch_reuse_move<true>(hdev, v_cache_buffer, offsets, cnts, batch_size * heads,
                                   map_size, cpu_v_length, cpu_v_length / CHUNK_ELEMS,
                                   gpu_v_stride, gpu_v_offset, (cudaStream_t)stream);
}

int skv_gather_copy_d2d_with_offsets(void *keys, const int32_t *offsets, const int32_t *cnts,
                                     int batch_size, int heads, int gpu_k_length, int gpu_k_offset,
                                     int gpu_k_stride, int map_size, void *stream)
{
    (void)gpu_k_length;
    SKV_CHECK_ARG(keys && offsets && cnts, "null pointer argument");
    SKV_CHECK_ARG(batch_size > 0 && heads > 0, "batch_size and heads must be positive");
    SKV_CHECK_SUPPORTED(map_size >= 1 && map_size <= 1024, "map_size %d outside 1..1024", map_size);
    SKV_CHECK_ARG(gpu_k_offset >= 0 && gpu_k_offset % 8 == 0 && gpu_k_stride % 8 == 0,
                  "gpu_k_offset/gpu_k_stride must be multiples of 8 elements");
    SKV_CHECK_ARG((int64_t)gpu_k_offset + (int64_t)map_size * CHUNK_ELEMS <= gpu_k_stride ||
                      batch_size * heads == 1,
                  "gpu_k_offset + map_size*1024 exceeds gpu_k_stride");
    SKV_CHECK_ARG(aligned(keys, 16), "keys must be 16-byte aligned");
    return launch_reuse_move<false>(nullptr, keys, offsets, cnts, batch_size * heads, map_size, 0, 0,
                                    gpu_k_stride, gpu_k_offset, (cudaStream_t)stream);
}

int skv_gather_copy(const void *values, void *v_cache_buffer, const int64_t *position_ids,
                    int batch_size, int heads, int cpu_v_length, int gpu_v_length, int map_size,
                    void *stream)
{
    SKV_CHECK_ARG(v_cache_buffer && position_ids, "null pointer argument");
    SKV_CHECK_ARG(batch_size > 0 && heads > 0, "batch_size and heads must be positive");
    SKV_CHECK_SUPPORTED(map_size >= 1 && map_size <= 1024, "map_size %d outside 1..1024", map_size);
    SKV_CHECK_ARG(cpu_v_length > 0 && cpu_v_length % CHUNK_ELEMS == 0,
                  "cpu_v_length must be a positive multiple of 1024");
    SKV_CHECK_ARG(gpu_v_length % 8 == 0 && (int64_t)map_size * CHUNK_ELEMS <= gpu_v_length,
                  "gpu_v_length must hold map_size chunks");
    SKV_CHECK_ARG(aligned(v_cache_buffer, 16), "v_cache_buffer must be 16-byte aligned");
    const void *hdev = nullptr;
    int st = host_to_device_ptr(values, &hdev, "values");
    if (st != SKV_OK) return st;
    SKV_CHECK_ARG(aligned(hdev, 16), "values must be 16-byte aligned");
    dim3 grid(ceil_div(map_size, 16), batch_size * heads);
    gather_copy_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(
        reinterpret_cast<const uint4 *>(hdev), reinterpret_cast<uint4 *>(v_cache_buffer),
        position_ids, map_size, cpu_v_length / 8, cpu_v_length / CHUNK_ELEMS, gpu_v_length / 8);
    return check_launch("gather_copy_kernel");
}

int skv_decode_gather_values(const skv_decode_geom *g, const void *v_host, void *v_buf,
                             const int32_t *miss_slot, const int32_t *miss_chunk,
                             const int32_t *miss_count, void *stream)
{
    SKV_CHECK_ARG(g && v_buf && miss_slot && miss_chunk && miss_count, "null pointer argument");
    SKV_CHECK_SUPPORTED(g->head_dim == 128 && g->chunk_size == 8, "head_dim 128 and chunk 8 only");
    SKV_CHECK_ARG(g->sparse_start >= 0 &&
                      g->sparse_start + 8 * (int64_t)g->select_sets <= g->buf_len,
                  "selected rows exceed buf_len");
    SKV_CHECK_ARG(aligned(v_buf, 16), "v_buf must be 16-byte aligned");
    const void *hdev = nullptr;
    int st = host_to_device_ptr(v_host, &hdev, "v_host");
    if (st != SKV_OK) return st;
    SKV_CHECK_ARG(aligned(hdev, 16), "v_host must be 16-byte aligned");
    return launch_fetch_misses(g, hdev, v_buf, miss_slot, miss_chunk, miss_count,
                               (cudaStream_t)stream);
}

}  // extern "C"
