// Fused value fetch + key reconstruction + decode attention of the fused
// decode path (one launch after the selection).
//
// Replaces, for one step, the three launches
//   gather of the missed value chunks from pinned host memory
//     (kernels/gather_copy.cu:193-253, gather_copy_with_offsets),
//   low-rank reconstruction of the missed keys with RoPE
//     (kernels/batch_gather_gemm.cu:136-213 + kernels/rope_new.cu:224-374),
//   GQA decode attention over the budget
//     (models/attention/shadow.py:48, flash_attn_with_kvcache, q_len = 1),
// and leaves the same state behind: the missed rows of k_buf / v_buf hold the
// reconstructed keys and the fetched values, as the separate kernels write them.
//
// Grid: ceil(seq_len / 128) * B * Hkv CTAs; CTA (b, h, j) owns buffer rows
// [128 j, 128 j + 128): sixteen 8-row groups, each either a group of buffer
// rows (prefix, cached slot, generated token) or a missed slot.  A CTA
//   1. waits for the selection (programmatic dependent launch: the CTA may
//      be resident before the selection kernel ends),
//   2. reads the miss list, issues the zero-copy loads of its missed value
//      chunks into registers, then bulk-copies SV^T, the U and cos/sin rows
//      of those chunks and the buffer rows of the other groups,
//   3. reconstructs the missed keys on the tensor cores (RoPE on the fp32
//      accumulators, one rounding) while the values cross the host link --
//      device-memory rows come in through bulk copies, which do not queue
//      behind the zero-copy loads, and global stores wait until the values
//      are in,
//   4. computes S = K q^T and the softmax of its 128 keys for the G query
//      heads of the group, then, once the values are in, O = P V,
//   5. writes its partial (max, sum, O) and takes a ticket; the last CTA of
//      the head merges the partials into the output.
// The host link is the bound of the step; everything but the final P V and
// the merge overlaps the value transfer.
#include <string.h>

#include "attn_block.cuh"
#include "select.cuh"

namespace skv {

constexpr int SA_THREADS = 256;  // 8 warps
constexpr int SA_ROWS = 128;     // rows per CTA
constexpr int SA_GROUPS = SA_ROWS / 8;
constexpr int SA_PITCH = 136;    // K / V tile row pitch (bf16)

struct SparseAttendArgs {
    const __nv_bfloat16 *q;        // [B][Hq][128] rotated queries
    const __nv_bfloat16 *U;        // [B][ctx][rank]
    const __nv_bfloat16 *SVt;      // [B][Hkv][128][rank]
    const __nv_bfloat16 *cos_sin;  // [cs_rows][cs_stride]
    const uint4 *v_host;           // device view of the pinned values [B*Hkv][num_chunks][8 rows][128]
    __nv_bfloat16 *k_buf, *v_buf;  // [B*Hkv][buf_len][128]
    const int32_t *miss_slot, *miss_chunk, *miss_count;  // [BH][K], [BH][K], [BH]
    float *part_o;                 // [BH][nblk][G][128]
    float2 *part_ml;               // [BH][nblk][G] (max, sum)
    unsigned *ticket;              // [BH], zero between launches
    __nv_bfloat16 *out;            // [B][Hq][128] (world == 0)
    int Hkv, G, K, rank, ctx, num_chunks, buf_len, sparse_start, seq_len, nblk;
    int total;                     // work items: nblk * B * Hkv
    int rope_mode, cs_stride, cs_rows;
    float scale;
    // world > 0: the output rows go to every rank's landing buffer
    // [2][B][q_heads_total][128] (half epoch & 1) over peer memory, then one
    // system-scope increment of every rank's arrival counter per (b, kv head)
    int world, q_head0, q_heads_total;
    __nv_bfloat16 *landing[SKV_MAX_PEERS];
    unsigned *counter[SKV_MAX_PEERS];
    const unsigned *epoch;
    // if set: the row this step appended at, read on the device; the attention
    // then covers [0, *row_dev + 1) (at most seq_len rows, which sized the grid)
    const int32_t *row_dev;
    unsigned long long *span;  // optional: kernel span pair of a timed step (span_begin)
    int smem_bytes;            // dynamic shared memory of a CTA (the merge stages partials in it)
};

// NT: n-tiles of query heads in S = K q^T (1: G <= 8, 2: G <= 16)
template <int NT>
__global__ void __launch_bounds__(SA_THREADS, 1) sparse_attend_kernel(SparseAttendArgs a)
{
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int KP = a.rank + 8;         // row pitch of SV^T (conflict-free ldmatrix)
    const int KT = max(KP, SA_PITCH);  // row pitch of the U rows (rank wide) / keys (128 wide)
    __nv_bfloat16 *sK = reinterpret_cast<__nv_bfloat16 *>(smem_raw);  // [128][KT]: U rows, then keys
    __nv_bfloat16 *sB = sK + SA_ROWS * KT;                              // [128][KP]: SV^T of the head
    __nv_bfloat16 *sV = sB + 128 * KP;                                  // [128][SA_PITCH]: values
    __nv_bfloat16 *sQ = sV + SA_ROWS * SA_PITCH;                        // [16][SA_PITCH]
    __nv_bfloat16 *sP = sQ + 16 * SA_PITCH;                             // [16][SA_PITCH] probabilities
    float *sS = reinterpret_cast<float *>(sP + 16 * SA_PITCH);         // [128][16] logits
    __nv_bfloat16 *sCS = reinterpret_cast<__nv_bfloat16 *>(sS + SA_ROWS * 16);  // [128][SA_PITCH] cos/sin rows
    __shared__ int s_kind[SA_GROUPS];   // 0: buffer rows, 1: missed slot
    __shared__ int s_chunk[SA_GROUPS];  // chunk id of a missed slot
    __shared__ int s_any_miss;
    __shared__ float s_m[16], s_l[16];
    __shared__ unsigned s_last;
    __shared__ __align__(8) uint64_t s_bar;  // completion of the bulk copies of the device-memory rows
    __shared__ __align__(8) uint64_t s_mbar;  // completion of the staging copies of a merge

    if (threadIdx.x == 0) {
        mbar_init(&s_bar, 1);
        mbar_init(&s_mbar, 1);
        mbar_fence_init();
    }
    SKV_TRACE_CTA(TR_SA_START);
    pdl_wait();  // the selection (and the scoring before it) are complete from here on
    span_begin(a.span);
    SKV_TRACE_CTA(TR_SA_WAITED);

    // Work items: (kv head, 128-row block), the blocks that hold selected slots
    // first -- with more items than CTAs the ones left for later are the light
    // ones (prefix and generated rows only), not ones that wait on the host
    // link.  One item per CTA for a full grid; a grid of fewer CTAs (leaving
    // SMs to other work while the link is busy) walks the items in strides.
    unsigned iter = 0;
    unsigned nmerge = 0;  // staged merges done by this CTA: the phase of s_mbar
    for (int item = blockIdx.x; item < a.total; item += gridDim.x) {
    // the previous item's (generic) shared-memory accesses are ordered before
    // this item's bulk copies into the same bytes, and are complete
    fence_proxy_async_smem();
    __syncthreads();
    int blk, bh;
    {
        const int blo = a.sparse_start / SA_ROWS;
        const int nheavy = min(a.nblk, ceil_div(a.sparse_start + 8 * a.K, SA_ROWS)) - blo;
        const int nlight = a.nblk - nheavy;
        const int L = item;
        const int BHn = a.total / a.nblk;
        if (L < BHn * nheavy) {
            bh = L / nheavy;
            blk = blo + L % nheavy;
        } else {
            const int L2 = L - BHn * nheavy;
            bh = L2 / nlight;
            const int j = L2 % nlight;
            blk = j < blo ? j : j + nheavy;
        }
    }
    // rows of this step: seq_len from the launch, or the device-side position
    int seq_len = a.seq_len;
    if (a.row_dev) {
        const int r1 = *a.row_dev + 1;
        if (r1 >= a.sparse_start + 8 * a.K && r1 <= a.seq_len) seq_len = r1;
        else if (threadIdx.x == 0 && blk == 0) report_dev_error(DEV_ERR_ROW);
    }
    const int nblk = ceil_div(seq_len, SA_ROWS);  // blocks of this step (a.nblk: of the grid and the partials' stride)
    if (blk >= nblk) continue;                    // past this step's rows: no work, no ticket
    SKV_TRACE_REC_DECL;
    SKV_TRACE_REC_OPEN();
    SKV_TRACE_REC(0, (unsigned long long)::skv::trace_smid() | ((unsigned long long)bh << 8) | ((unsigned long long)blk << 20));
    SKV_TRACE_REC(1, (unsigned long long)(uintptr_t)a.k_buf);
    SKV_TRACE_REC_NOW(2);
    const int b = bh / a.Hkv;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = a.G;
    const int row0 = blk * SA_ROWS;
    const int nrows = min(SA_ROWS, seq_len - row0);
    const int sparse_end = a.sparse_start + 8 * a.K;
    const bool has_slots = row0 < sparse_end && row0 + SA_ROWS > a.sparse_start;
    const int ppr = a.rank / 8;  // 16-byte pieces per U / SV^T row

    if (tid < SA_GROUPS) {
        s_kind[tid] = 0;
        s_chunk[tid] = -1;
    }
    if (tid == 0) s_any_miss = 0;
    __syncthreads();

    // 2) query rows of the group (rows >= G are zero) and the missed slots of
    //    this CTA; every load of this phase is issued in one round: the miss
    //    count, slots and chunk ids are read together (K <= 4 * SA_THREADS)
    {
        const __nv_bfloat16 *qrows = a.q + (int64_t)bh * G * 128;
        for (int p = tid; p < 16 * 16; p += SA_THREADS) {
            const int r = p >> 4, c = (p & 15) * 8;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (r < G) v = ld_nc_v4(qrows + (int64_t)r * 128 + c);
            st_v4(sQ + r * SA_PITCH + c, v);
        }
    }
    if (has_slots) {
        const int32_t *msl = a.miss_slot + (int64_t)bh * a.K, *mch = a.miss_chunk + (int64_t)bh * a.K;
        const int nm_raw = a.miss_count[bh];
        int sv[4], cv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int t = tid + SA_THREADS * u;
            sv[u] = t < a.K ? msl[t] : -1;
            cv[u] = t < a.K ? mch[t] : -1;
        }
        const int nmiss = min(max(nm_raw, 0), a.K);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int t = tid + SA_THREADS * u;
            const int s = sv[u];
            if (t >= nmiss || s < 0 || s >= a.K || a.sparse_start + 8 * s < row0) continue;
            const int gi = (a.sparse_start + 8 * s - row0) >> 3;
            if (gi >= SA_GROUPS) continue;
            const int c = cv[u];
            if (c >= 0 && c < a.num_chunks && (int64_t)c * 8 + 8 <= a.ctx) {
                s_chunk[gi] = c;
                s_kind[gi] = 1;
                s_any_miss = 1;
            } else {
                report_dev_error(DEV_ERR_HOST_CHUNK);
            }
        }
    }
    __syncthreads();
    SKV_TRACE_CTA(TR_SA_LISTS);
    const bool any_miss = s_any_miss != 0;

    // 3) zero-copy loads of the missed value chunks (2 KiB each), issued
    //    first -- the host link is the bound of the step -- and kept in
    //    registers until the end: element p = tid + 256 u is piece p & 127 of group p >> 7
    uint4 vreg[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
        const int p = tid + SA_THREADS * u;
        const int gi = p >> 7;
        vreg[u] = make_uint4(0, 0, 0, 0);
        if (s_kind[gi] == 1)
            vreg[u] = ld_stream_v4(a.v_host + ((int64_t)bh * a.num_chunks + s_chunk[gi]) * 128 + (p & 127));
    }
    if (any_miss) SKV_TRACE_CTA(TR_SA_ISSUED);
    SKV_TRACE_REC_NOW(3);

    // 4) device-memory rows as bulk (TMA) copies: SV^T of the head, U and
    //    cos/sin rows of the missed groups, K and V rows of the buffer groups.
    //    They do not go through the load path the zero-copy loads above
    //    occupy, so they land while the values are still crossing the link.
    //    Rows past seq_len are zero.
    const unsigned ub = (unsigned)a.rank * 2u, csb = a.rope_mode == 0 ? 256u : 128u;
    if (tid == 0) {
        unsigned total = has_slots && any_miss ? 128u * ub : 0u;
        for (int gi = 0; gi < SA_GROUPS; ++gi) {
            const int k = s_kind[gi];
            for (int i = 0; i < 8; ++i) {
                const int r = gi * 8 + i;
                if (k == 1) {
                    total += ub;
                    if ((int64_t)s_chunk[gi] * 8 + i < a.cs_rows) total += csb;
                } else if (r < nrows) {
                    total += 512u;
                }
            }
        }
        mbar_arrive_expect_tx(&s_bar, total);
    }
    __syncthreads();
    {
        if (has_slots && any_miss && tid < 128) {
            const __nv_bfloat16 *Bb = a.SVt + (int64_t)bh * 128 * a.rank;
            bulk_g2s(sB + tid * KP, Bb + (int64_t)tid * a.rank, ub, &s_bar);
        }
        const __nv_bfloat16 *Ub = a.U + (int64_t)b * a.ctx * a.rank;
        const __nv_bfloat16 *kb = a.k_buf + ((int64_t)bh * a.buf_len + row0) * 128;
        const __nv_bfloat16 *vb = a.v_buf + ((int64_t)bh * a.buf_len + row0) * 128;
        const int r = tid & (SA_ROWS - 1);
        const int gi = r >> 3;
        if (tid < SA_ROWS) {
            if (s_kind[gi] == 1) {
                bulk_g2s(sK + r * KT, Ub + ((int64_t)s_chunk[gi] * 8 + (r & 7)) * a.rank, ub, &s_bar);
            } else if (r < nrows) {
                bulk_g2s(sK + r * KT, kb + (int64_t)r * 128, 256u, &s_bar);
            }
        } else {
            if (s_kind[gi] == 1) {
                const int64_t pos = (int64_t)s_chunk[gi] * 8 + (r & 7);
                if (pos < a.cs_rows) bulk_g2s(sCS + r * SA_PITCH, a.cos_sin + pos * a.cs_stride, csb, &s_bar);
            } else if (r < nrows) {
                bulk_g2s(sV + r * SA_PITCH, vb + (int64_t)r * 128, 256u, &s_bar);
            }
        }
    }
    for (int p = tid; p < SA_ROWS * 16; p += SA_THREADS) {
        const int r = p >> 4, c = (p & 15) * 8;
        if (r >= nrows && s_kind[r >> 3] == 0) {
            st_v4(sK + r * KT + c, make_uint4(0, 0, 0, 0));
            st_v4(sV + r * SA_PITCH + c, make_uint4(0, 0, 0, 0));
        }
    }
    // bounded waits: a copy that never lands is reported, it does not hang the GPU
    if (!mbar_wait(&s_bar, iter & 1u)) {
        if (lane == 0) report_dev_error(DEV_ERR_WAIT);
    }
    __syncthreads();

    // 5) key reconstruction of the missed groups: U rows x SV^T, RoPE at the
    //    original positions on the fp32 accumulators, one rounding to bf16.
    //    Warp w owns rows 16w .. 16w+15: it reads only its own U rows, so it
    //    overwrites them with its keys once both column halves are done.
    if (any_miss && (s_kind[2 * warp] == 1 || s_kind[2 * warp + 1] == 1)) {
        const int g = lane >> 2, t4 = lane & 3;
        const __nv_bfloat16 *aRow = sK + (warp * 16 + (lane & 15)) * KT + (lane >> 4) * 8;
        uint32_t kres[2][16];  // packed bf16 keys: [half][row g / g+8][8 n-tiles]
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            float acc[8][4];
            recon_half(acc, aRow, sB, KP, a.rank, half, lane);
            // epilogue of this half: acc[pr] is n-tile 4h + pr, acc[4 + pr] is 8 + 4h + pr
#pragma unroll
            for (int hr = 0; hr < 2; ++hr) {
                const int r = warp * 16 + g + 8 * hr;
                const int gi = r >> 3;
                float v[8][2];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    v[i][0] = acc[i][2 * hr];
                    v[i][1] = acc[i][2 * hr + 1];
                }
                if (s_kind[gi] == 1) {
                    const int64_t pos = (int64_t)s_chunk[gi] * 8 + (r & 7);
                    if (pos >= a.cs_rows) {
                        if (t4 == 0) report_dev_error(DEV_ERR_ROW);
                    } else {
                        recon_rope(v, sCS + r * SA_PITCH, a.rope_mode, half, t4);
                    }
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) kres[half][hr * 8 + i] = pack_bf2(v[i][0], v[i][1]);
            }
        }
        __syncwarp();  // every lane is done reading this warp's U rows
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
            for (int hr = 0; hr < 2; ++hr) {
                const int r = warp * 16 + g + 8 * hr;
                if (s_kind[r >> 3] != 1) continue;
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    *reinterpret_cast<uint32_t *>(sK + r * KT + recon_col(half, i, t4)) = kres[half][hr * 8 + i];
            }
        }
    }
    __syncthreads();
    if (any_miss) SKV_TRACE_CTA(TR_SA_KEYS);
    SKV_TRACE_REC_NOW(4);

    // 6) S = K q^T: warp w scores keys 16w .. 16w+15, then the softmax of the tile
    ab_scores<NT>(sK, KT, sQ, sS, nrows, a.scale, warp, lane);
    __syncthreads();
    ab_softmax(sS, sP, s_m, s_l, G, warp, lane);

    // 7) the fetched values: into the V tile and back to the slot in v_buf.
    //    Global stores come only now: issued earlier, they would queue behind
    //    the zero-copy loads.  The reconstructed keys go back to k_buf here too
    //    (the slot keeps them for later hits).
    if (any_miss) {
        __nv_bfloat16 *kdst = a.k_buf + ((int64_t)bh * a.buf_len + row0) * 128;
        for (int p = tid; p < SA_ROWS * 16; p += SA_THREADS) {
            const int r = p >> 4, c = (p & 15) * 8;
            if (s_kind[r >> 3] == 1) st_v4(kdst + (int64_t)r * 128 + c, ld_v4(sK + r * KT + c));
        }
        __nv_bfloat16 *vdst = a.v_buf + ((int64_t)bh * a.buf_len + row0) * 128;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int p = tid + SA_THREADS * u;
            const int gi = p >> 7;
            if (s_kind[gi] == 1) {
                const int r = gi * 8 + ((p & 127) >> 4), c = (p & 15) * 8;
                st_v4(sV + r * SA_PITCH + c, vreg[u]);
                __stcg(reinterpret_cast<uint4 *>(vdst + (int64_t)r * 128 + c), vreg[u]);
            }
        }
    }
    __syncthreads();
    if (any_miss) SKV_TRACE_CTA(TR_SA_VALUES);
    SKV_TRACE_REC_NOW(5);

    // 8) O = P V: warp w computes dims 16w .. 16w+15 for the 16 head rows
    float o[2][4];
    ab_pv(sP, sV, o, warp, lane);

    // 9) partial of this CTA, then the last CTA of the head merges
    ab_partial(o, a.part_o + ((int64_t)bh * a.nblk + blk) * G * 128, a.part_ml + ((int64_t)bh * a.nblk + blk) * G, s_m,
               s_l, G, warp, lane, tid);
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&a.ticket[bh], 1u) == (unsigned)(nblk - 1) ? 1u : 0u;
    SKV_TRACE_CTA(TR_SA_TICKET);
    SKV_TRACE_REC_NOW(6);
    __syncthreads();
    if (s_last) {
    __threadfence();
    // merge of the head's nblk partial outputs (the tiles' shared memory is free)
    // the partials come into the (free) tile memory after the merge scratch when they fit
    const size_t scratch = ((size_t)nblk * G * 12 + 15) & ~(size_t)15;
    float *stage = scratch + (size_t)nblk * G * 512 <= (size_t)a.smem_bytes
                       ? reinterpret_cast<float *>(smem_raw + scratch) : nullptr;
    ab_merge(a.part_o + (int64_t)bh * a.nblk * G * 128, a.part_ml + (int64_t)bh * a.nblk * G, nblk, G, smem_raw,
             stage, &s_mbar, nmerge & 1u, tid, SA_THREADS, [&](int gg, int d, uint2 pk) {
                 if (a.world == 0) {
                     *reinterpret_cast<uint2 *>(a.out + ((int64_t)bh * G + gg) * 128 + d) = pk;
                 } else {
                     const int b = bh / a.Hkv, h = bh % a.Hkv;
                     const int64_t o = (((int64_t)(*a.epoch & 1u) * (a.total / a.nblk / a.Hkv) + b) * a.q_heads_total +
                                        a.q_head0 + h * G + gg) * 128 + d;
                     for (int r = 0; r < a.world; ++r) *reinterpret_cast<uint2 *>(a.landing[r] + o) = pk;
                 }
             });
    if (stage) ++nmerge;
    if (a.world > 0) {
        // the rows are in every rank's memory before any counter moves
        __threadfence_system();
        __syncthreads();
        if (tid == 0)
            for (int r = 0; r < a.world; ++r) atomicAdd_system(a.counter[r], 1u);
    }
    if (tid == 0) a.ticket[bh] = 0;  // ready for the next launch
    SKV_TRACE_CTA(TR_SA_MERGED);
    SKV_TRACE_REC_NOW(7);
    }  // the head's last block
    ++iter;  // items that did work: the phase of the copy barrier
    }  // work items
    span_finish(a.span);
}

// Peer block layout: arrival counter, status, this rank's epoch, landing buffer.
constexpr size_t PEER_COUNTER_OFF = 0, PEER_STATUS_OFF = 64, PEER_EPOCH_OFF = 128, PEER_LANDING_OFF = 256;

struct PeerFinishArgs {
    const unsigned *counter;  // arrivals of (sequence, kv head) rows from every rank
    unsigned *status;         // sticky: DEV_ERR_WAIT once a wait ran out
    unsigned *epoch;          // steps completed by this rank
    const uint4 *landing;     // [2][n16] 16-byte words
    uint4 *out;               // [n16]
    int64_t n16;
    unsigned merges;          // arrivals per step
};

// One CTA: a bounded wait until every rank's rows of this step have arrived
// (counter >= (epoch + 1) * merges), the copy of the landing half epoch & 1,
// and the epoch advance.  A wait that runs out sets the sticky status (and
// counts a device error) instead: no copy, no epoch advance -- a late arrival
// must not count toward the next step -- and every later finish on the block
// returns at once.
__global__ void __launch_bounds__(256) peer_gather_finish_kernel(PeerFinishArgs f)
{
    __shared__ unsigned s_e, s_ok;
    if (threadIdx.x == 0) {
        const unsigned e = *f.epoch;
        const unsigned target = (e + 1u) * f.merges;
        bool ok = *f.status == 0u;  // a block that timed out before stays stopped
        if (ok) {
            ok = false;
            for (unsigned it = 0; it < (1u << 22); ++it) {
                unsigned v;
                asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f.counter) : "memory");
                if ((int)(v - target) >= 0) {
                    ok = true;
                    break;
                }
                __nanosleep(64);
            }
            if (!ok) {
                *f.status = DEV_ERR_WAIT;
                report_dev_error(DEV_ERR_WAIT);
            }
        }
        s_e = e;
        s_ok = ok ? 1u : 0u;
    }
    __syncthreads();
    if (!s_ok) return;
    const uint4 *src = f.landing + (int64_t)(s_e & 1u) * f.n16;
    for (int64_t i = threadIdx.x; i < f.n16; i += blockDim.x) f.out[i] = __ldcg(src + i);
    __syncthreads();
    if (threadIdx.x == 0) *f.epoch = s_e + 1u;
}

static size_t sa_smem_bytes(int rank)
{
    const size_t KP = (size_t)rank + 8, KT = KP > (size_t)SA_PITCH ? KP : (size_t)SA_PITCH;
    return (SA_ROWS * KT + 128 * KP + 2 * SA_ROWS * SA_PITCH + 2 * 16 * SA_PITCH) * 2 + SA_ROWS * 16 * 4;
}

}  // namespace skv

using namespace skv;

extern "C" {

size_t skv_decode_sparse_attention_workspace(const skv_decode_geom *g, int seq_len)
{
    if (!g || g->batch <= 0 || g->kv_heads <= 0 || g->q_heads % g->kv_heads != 0 || seq_len <= 0) return 0;
    const size_t BH = (size_t)g->batch * g->kv_heads, G = (size_t)(g->q_heads / g->kv_heads);
    const size_t nblk = (size_t)ceil_div(seq_len, SA_ROWS);
    const size_t o = BH * nblk * G * 128 * 4, ml = BH * nblk * G * 8, tk = BH * 4;
    return ((o + 255) & ~(size_t)255) + ((ml + 255) & ~(size_t)255) + ((tk + 255) & ~(size_t)255);
}

}  // extern "C"

static int launch_sparse_attention(const skv_decode_geom *g, const void *q, const void *U, const void *SVt,
                                   const void *cos_sin, const void *v_host, void *k_buf, void *v_buf,
                                   const int32_t *miss_slot, const int32_t *miss_chunk,
                                   const int32_t *miss_count, int seq_len, void *out,
                                   const skv_peer_gather *pg, void *workspace, size_t workspace_bytes,
                                   void *stream, int max_ctas = 0, const int32_t *row_dev = nullptr)
{
    SKV_CHECK_ARG(g && q && U && SVt && cos_sin && k_buf && v_buf && miss_slot && miss_chunk && miss_count &&
                      (out || pg) && workspace,
                  "null pointer argument");
    SKV_CHECK_ARG(g->batch > 0 && g->kv_heads > 0 && g->q_heads % g->kv_heads == 0, "bad head counts");
    SKV_CHECK_SUPPORTED(g->head_dim == 128 && g->chunk_size == 8, "head_dim 128 and chunk 8 only");
    const int G = g->q_heads / g->kv_heads;
    SKV_CHECK_SUPPORTED(G <= 16, "GQA group larger than 16");
    SKV_CHECK_SUPPORTED(g->rank % 16 == 0 && g->rank >= 16 && g->rank <= 256, "rank must be a multiple of 16 in 16..256");
    SKV_CHECK_SUPPORTED(g->rope_mode == 0 || g->rope_mode == 1, "rope_mode must be 0 or 1");
    SKV_CHECK_ARG(g->cos_sin_stride >= (g->rope_mode == 0 ? 128 : 64), "cos_sin_stride too small");
    SKV_CHECK_SUPPORTED(g->select_sets <= 4 * SA_THREADS, "select_sets above %d", 4 * SA_THREADS);
    SKV_CHECK_ARG(g->select_sets >= 1 && g->sparse_start >= 0 && g->sparse_start % 8 == 0 &&
                      g->sparse_start + 8 * (int64_t)g->select_sets <= g->buf_len,
                  "selected rows exceed buf_len (or sparse_start not a multiple of 8)");
    SKV_CHECK_ARG(seq_len >= g->sparse_start + 8 * g->select_sets && seq_len <= g->buf_len,
                  "seq_len %d must cover the selected rows and fit in buf_len", seq_len);
    SKV_CHECK_ARG(aligned(q, 16) && aligned(U, 16) && aligned(SVt, 16) && aligned(cos_sin, 16) && aligned(k_buf, 16) &&
                      aligned(v_buf, 16) && aligned(workspace, 256),
                  "operands must be 16-byte aligned (workspace 256)");
    SKV_CHECK_ARG(g->cos_sin_stride % 8 == 0, "cos_sin_stride must be a multiple of 8 (16-byte rows)");
    const size_t need = skv_decode_sparse_attention_workspace(g, seq_len);
    SKV_CHECK_ARG(workspace_bytes >= need, "workspace too small: %zu < %zu bytes", workspace_bytes, need);
    const void *hdev = nullptr;
    int st = host_to_device_ptr(v_host, &hdev, "v_host");
    if (st != SKV_OK) return st;
    SKV_CHECK_ARG(aligned(hdev, 16), "v_host must be 16-byte aligned");
    void *dout = nullptr;
    if (!pg) {
        st = out_to_device_ptr(out, &dout, "out");
        if (st != SKV_OK) return st;
        SKV_CHECK_ARG(aligned(dout, 8), "out must be 8-byte aligned");
    } else {
        SKV_CHECK_ARG(pg->world >= 1 && pg->world <= SKV_MAX_PEERS && pg->rank >= 0 && pg->rank < pg->world,
                      "peer gather: world must be 1..%d and rank in [0, world)", SKV_MAX_PEERS);
        SKV_CHECK_ARG(pg->q_head0 >= 0 && pg->q_head0 + g->q_heads <= pg->q_heads_total,
                      "peer gather: query heads [%d, %d) outside the %d of the full output", pg->q_head0,
                      pg->q_head0 + g->q_heads, pg->q_heads_total);
        SKV_CHECK_ARG(pg->batch == g->batch, "peer gather: the blocks hold batch %d, the step has %d", pg->batch,
                      g->batch);
        SKV_CHECK_ARG(pg->q_heads_total % G == 0 &&
                          (int64_t)pg->merges_per_step == (int64_t)g->batch * (pg->q_heads_total / G),
                      "peer gather: merges_per_step must be batch * q_heads_total / %d = %lld", G,
                      (long long)g->batch * (pg->q_heads_total / (G > 0 ? G : 1)));
        for (int r = 0; r < pg->world; ++r)
            SKV_CHECK_ARG(pg->block[r] && aligned(pg->block[r], 256), "peer gather: block %d null or unaligned", r);
    }

    const int BH = g->batch * g->kv_heads;
    const int nblk = ceil_div(seq_len, SA_ROWS);
    const size_t o_bytes = (size_t)BH * nblk * G * 128 * 4, ml_bytes = (size_t)BH * nblk * G * 8;
    unsigned char *ws = static_cast<unsigned char *>(workspace);
    SparseAttendArgs a = {};
    a.q = (const __nv_bfloat16 *)q;
    a.U = (const __nv_bfloat16 *)U;
    a.SVt = (const __nv_bfloat16 *)SVt;
    a.cos_sin = (const __nv_bfloat16 *)cos_sin;
    a.v_host = (const uint4 *)hdev;
    a.k_buf = (__nv_bfloat16 *)k_buf;
    a.v_buf = (__nv_bfloat16 *)v_buf;
    a.miss_slot = miss_slot;
    a.miss_chunk = miss_chunk;
    a.miss_count = miss_count;
    // tickets first: their offset must not depend on seq_len (they stay zero between launches)
    const size_t tk_bytes = ((size_t)BH * 4 + 255) & ~(size_t)255;
    a.ticket = reinterpret_cast<unsigned *>(ws);
    a.part_ml = reinterpret_cast<float2 *>(ws + tk_bytes);
    a.part_o = reinterpret_cast<float *>(ws + tk_bytes + ((ml_bytes + 255) & ~(size_t)255));
    (void)o_bytes;
    a.out = (__nv_bfloat16 *)dout;
    if (pg) {
        a.world = pg->world;
        a.q_head0 = pg->q_head0;
        a.q_heads_total = pg->q_heads_total;
        for (int r = 0; r < pg->world; ++r) {
            unsigned char *blk = static_cast<unsigned char *>(pg->block[r]);
            a.counter[r] = reinterpret_cast<unsigned *>(blk + PEER_COUNTER_OFF);
            a.landing[r] = reinterpret_cast<__nv_bfloat16 *>(blk + PEER_LANDING_OFF);
        }
        a.epoch = reinterpret_cast<const unsigned *>(static_cast<unsigned char *>(pg->block[pg->rank]) + PEER_EPOCH_OFF);
    }
    a.Hkv = g->kv_heads;
    a.G = G;
    a.K = g->select_sets;
    a.rank = g->rank;
    a.ctx = g->ctx_len;
    a.num_chunks = g->num_chunks;
    a.buf_len = g->buf_len;
    a.sparse_start = g->sparse_start;
    a.seq_len = seq_len;
    a.row_dev = row_dev;
    a.nblk = nblk;
    a.total = nblk * BH;
    a.rope_mode = g->rope_mode;
    a.cs_stride = g->cos_sin_stride;
    a.cs_rows = g->cos_sin_rows;
    a.scale = g->scale;
    a.span = launch_spans().attend;

    const int smem = (int)sa_smem_bytes(g->rank);
    a.smem_bytes = smem;
    SKV_CHECK_SUPPORTED((size_t)nblk * G * 12 <= (size_t)smem, "seq_len %d too long for the merge of the partials", seq_len);
    const void *fn = G <= 8 ? (const void *)sparse_attend_kernel<1> : (const void *)sparse_attend_kernel<2>;
    st = ensure_smem_attr(fn, smem, "sparse_attend_kernel");
    if (st) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(max_ctas > 0 && max_ctas < nblk * BH ? max_ctas : nblk * BH, 1, 1);
    cfg.blockDim = dim3(SA_THREADS, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    // may start while the selection drains: only SV^T is read before pdl_wait()
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = G <= 8 ? cudaLaunchKernelEx(&cfg, sparse_attend_kernel<1>, a)
                           : cudaLaunchKernelEx(&cfg, sparse_attend_kernel<2>, a);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("launch of sparse_attend_kernel failed: %s", cudaGetErrorString(e));
        return SKV_ERR_CUDA;
    }
    return SKV_OK;
}

int skv::sparse_attention_launch(const skv_decode_geom *g, const void *q, const void *U, const void *SVt,
                                 const void *cos_sin, const void *v_host, void *k_buf, void *v_buf,
                                 const int32_t *miss_slot, const int32_t *miss_chunk, const int32_t *miss_count,
                                 int seq_len, void *out, void *workspace, size_t workspace_bytes, cudaStream_t stream,
                                 const int32_t *row_dev)
{
    SKV_CHECK_ARG(out != nullptr, "null pointer argument");
    return launch_sparse_attention(g, q, U, SVt, cos_sin, v_host, k_buf, v_buf, miss_slot, miss_chunk, miss_count,
                                   seq_len, out, nullptr, workspace, workspace_bytes, stream, 0, row_dev);
}

extern "C" {

int skv_decode_sparse_attention(const skv_decode_geom *g, const void *q, const void *U, const void *SVt,
                                const void *cos_sin, const void *v_host, void *k_buf, void *v_buf,
                                const int32_t *miss_slot, const int32_t *miss_chunk,
                                const int32_t *miss_count, int seq_len, void *out, void *workspace,
                                size_t workspace_bytes, void *stream)
{
    SKV_CHECK_ARG(out != nullptr, "null pointer argument");
    return launch_sparse_attention(g, q, U, SVt, cos_sin, v_host, k_buf, v_buf, miss_slot, miss_chunk, miss_count,
                                   seq_len, out, nullptr, workspace, workspace_bytes, stream);
}

int skv_decode_sparse_attention_ctas(const skv_decode_geom *g, const void *q, const void *U, const void *SVt,
                                     const void *cos_sin, const void *v_host, void *k_buf, void *v_buf,
                                     const int32_t *miss_slot, const int32_t *miss_chunk,
                                     const int32_t *miss_count, int seq_len, void *out, int max_ctas,
                                     void *workspace, size_t workspace_bytes, void *stream)
{
    SKV_CHECK_ARG(out != nullptr && max_ctas >= 1, "null output or max_ctas < 1");
    return launch_sparse_attention(g, q, U, SVt, cos_sin, v_host, k_buf, v_buf, miss_slot, miss_chunk, miss_count,
                                   seq_len, out, nullptr, workspace, workspace_bytes, stream, max_ctas);
}

int skv_decode_sparse_attention_gather(const skv_decode_geom *g, const void *q, const void *U, const void *SVt,
                                       const void *cos_sin, const void *v_host, void *k_buf, void *v_buf,
                                       const int32_t *miss_slot, const int32_t *miss_chunk,
                                       const int32_t *miss_count, int seq_len, const skv_peer_gather *pg,
                                       void *workspace, size_t workspace_bytes, void *stream)
{
    SKV_CHECK_ARG(pg != nullptr, "null pointer argument");
    return launch_sparse_attention(g, q, U, SVt, cos_sin, v_host, k_buf, v_buf, miss_slot, miss_chunk, miss_count,
                                   seq_len, nullptr, pg, workspace, workspace_bytes, stream);
}

size_t skv_peer_block_bytes(int batch, int q_heads_total)
{
    if (batch <= 0 || q_heads_total <= 0) return 0;
    return PEER_LANDING_OFF + (size_t)2 * batch * q_heads_total * 128 * 2;
}

int skv_peer_alloc(size_t bytes, void **block)
{
    SKV_CHECK_ARG(block != nullptr && bytes >= PEER_LANDING_OFF, "bad peer block request");
    *block = nullptr;
    cudaError_t e = cudaMalloc(block, bytes);
    if (e == cudaSuccess) e = cudaMemset(*block, 0, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        if (*block) cudaFree(*block);
        *block = nullptr;
        set_error("peer block of %zu bytes: %s", bytes, cudaGetErrorString(e));
        return SKV_ERR_CUDA;
    }
    return SKV_OK;
}

int skv_peer_free(void *block)
{
    if (!block) return SKV_OK;
    cudaError_t e = cudaFree(block);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("cudaFree of a peer block: %s", cudaGetErrorString(e));
        return SKV_ERR_CUDA;
    }
    return SKV_OK;
}

int skv_peer_export(const void *block, void *handle64)
{
    SKV_CHECK_ARG(block && handle64, "null pointer argument");
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void *>(block));
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
        return SKV_ERR_CUDA;
    }
    memcpy(handle64, &h, sizeof(h));
    return SKV_OK;
}

int skv_peer_import(const void *handle64, void **block)
{
    SKV_CHECK_ARG(handle64 && block, "null pointer argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(block, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
        return SKV_ERR_CUDA;
    }
    return SKV_OK;
}

int skv_peer_close(void *block)
{
    SKV_CHECK_ARG(block != nullptr, "null pointer argument");
    cudaError_t e = cudaIpcCloseMemHandle(block);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
        return SKV_ERR_CUDA;
    }
    return SKV_OK;
}

int skv_peer_gather_finish(const skv_peer_gather *pg, int batch, void *out, void *stream)
{
    SKV_CHECK_ARG(pg && out && batch > 0, "null pointer argument or batch <= 0");
    SKV_CHECK_ARG(pg->world >= 1 && pg->world <= SKV_MAX_PEERS && pg->rank >= 0 && pg->rank < pg->world &&
                      pg->q_heads_total > 0 && pg->merges_per_step > 0 &&
                      (int64_t)pg->merges_per_step <= (int64_t)pg->batch * pg->q_heads_total,
                  "bad peer gather description");
    SKV_CHECK_ARG(batch == pg->batch, "peer gather: the blocks hold batch %d, finish asked for %d", pg->batch, batch);
    SKV_CHECK_ARG(pg->block[pg->rank] && aligned(pg->block[pg->rank], 256) && aligned(out, 16),
                  "peer block or output unaligned");
    unsigned char *blk = static_cast<unsigned char *>(pg->block[pg->rank]);
    PeerFinishArgs f;
    f.counter = reinterpret_cast<const unsigned *>(blk + PEER_COUNTER_OFF);
    f.status = reinterpret_cast<unsigned *>(blk + PEER_STATUS_OFF);
    f.epoch = reinterpret_cast<unsigned *>(blk + PEER_EPOCH_OFF);
    f.landing = reinterpret_cast<const uint4 *>(blk + PEER_LANDING_OFF);
    f.out = static_cast<uint4 *>(out);
    f.n16 = (int64_t)batch * pg->q_heads_total * 128 * 2 / 16;
    f.merges = (unsigned)pg->merges_per_step;
    peer_gather_finish_kernel<<<1, 256, 0, (cudaStream_t)stream>>>(f);
    return check_launch("peer_gather_finish_kernel");
}

int skv_peer_status(const skv_peer_gather *pg, uint32_t *status)
{
    SKV_CHECK_ARG(pg && status && pg->rank >= 0 && pg->rank < SKV_MAX_PEERS && pg->block[pg->rank],
                  "null pointer argument or bad rank");
    const unsigned char *blk = static_cast<const unsigned char *>(pg->block[pg->rank]);
    SKV_CUDA(cudaMemcpy(status, blk + PEER_STATUS_OFF, sizeof(uint32_t), cudaMemcpyDeviceToHost));
    return SKV_OK;
}

}  // extern "C"
