// Chunk selection of the fused decode path (shared between scoring.cu and select.cu).
#pragma once

#include "common.cuh"

namespace skv {

constexpr int SEL_CL = 8;    // CTAs per (b, kv head): one thread-block cluster (16 for very long contexts)
constexpr int SEL_T = 512;   // threads per CTA
// First pass: a 256-bin histogram of key bits 30..20 (exponent and 3
// mantissa bits).  Keys are probabilities in [0, 1] (bits 30..20 <= 1016);
// bins 1..255 hold bits 769..1023, bin 0 every key below 2^-31.
constexpr int SEL_BIN_LO = 768;
constexpr int SEL_BINS = 256;
constexpr int SEL_CAND = 2048;                 // rank 0's candidate store: one region per CTA
constexpr int SEL_REGION = SEL_CAND / SEL_CL;  // largest per-CTA candidate region (8-CTA clusters)

__device__ __forceinline__ int sel_key_bin(uint32_t k)
{
    // finite softmax keys are <= 1.0 (bits 30..20 <= 1016); a non-finite key
    // (inf or nan scores from non-finite inputs) is clamped into the last bin
    const int t = (int)(k >> 20);
    return t > SEL_BIN_LO ? min(t - SEL_BIN_LO, SEL_BINS - 1) : 0;
}

struct SelectArgs {
    const float *logits;          // [BH][L][G] scaled logits
    const float2 *part;           // [BH][G][nsplit] (max, sum-exp) of the scoring splits
    uint32_t *gkeys;              // [BH][L] key scratch when a slice does not fit in shared memory, else null
    const int64_t *landmark_idx;  // [BH][L] chunk id of every landmark
    int32_t *slots;               // [BH][K] in/out slot table
    int32_t *miss_slot, *miss_chunk, *miss_count;
    int G, L, K, nsplit, num_chunks;
    // [BH][L] keys already computed by keys_kernel (long contexts), or null:
    // the selection then computes them from the logits itself
    const uint32_t *keys_in;
    // Early fetch (the FETCH variant only): value chunks, keys and slots of
    // the misses, written by the selection kernel itself.
    const uint4 *v_host;              // device view of the page-locked values [BH][num_chunks][128 x 16 B]
    const __nv_bfloat16 *U;           // [B][ctx][rank]
    const __nv_bfloat16 *SVt;         // [BH][128][rank]
    const __nv_bfloat16 *cos_sin;     // [cs_rows][cs_stride]
    __nv_bfloat16 *k_buf, *v_buf;     // [BH][buf_len][128]
    int Hkv, rank, ctx, buf_len, sparse_start, rope_mode, cs_stride, cs_rows;
    int cap;                          // value chunks staged in shared memory at once
    unsigned stage_off, list_off, msg_off, bmc_off, recon_off, att_off;  // byte offsets in dynamic shared memory
    // ... and the step's attention, by the cluster of each head
    const __nv_bfloat16 *q_rot;       // [BH][G][128] rotated queries (written by the scoring kernel)
    __nv_bfloat16 *out;               // [BH][G][128]
    const int32_t *row_dev;           // optional: the append row, read on the device
    int seq_len;
    float scale;
    unsigned long long *span;         // optional: kernel span pair of a timed step (span_begin)
};

// Early-fetch variant of the selection (decode step): shared-memory layout of
// one CTA for rank `rank` and `cap` staged chunks; 0 when it does not fit.
constexpr int FETCH_ROWS = 32;            // rows of one key-reconstruction pass / attention tile
constexpr int FETCH_PITCH = 136;          // bf16 row pitch of the cos/sin rows
constexpr size_t FETCH_SMEM_CAP = 190 * 1024;  // dynamic shared memory of a FETCH CTA (static ~37 KB)
struct FetchLayout {
    unsigned stage_off, list_off, msg_off, bmc_off, recon_off, att_off, bytes;
    int cap;
};
constexpr int FX_PPITCH = 40;  // bf16 row pitch of a tile's attention weights (32 rows + 8)
constexpr int FX_MAX_TILES = 16;  // 4-chunk tiles of the staging area (at most 64 chunks)
// The attention region of a FETCH CTA (offsets from att_off): the G rotated
// query rows and a zero row, the running output O [G][128] and its row (max,
// sum), the scores of one 32-row tile, a zero weight row, the weights of a
// buffer-row tile, the weights and (max, sum) of the round's miss tiles, the
// 8-row groups of buffer rows attended by the CTA and the bitmap of the slots
// refilled by misses.
struct FxAttLayout {
    unsigned q, o, m, l, s, zp, pt, p, tml, grp, msb, bytes;
    int ntiles;
};
__host__ __device__ inline FxAttLayout fx_att_layout(int G, int cap, int buf_len, int K)
{
    FxAttLayout f = {};
    unsigned off = 0;
    auto take = [&off](unsigned bytes) {
        const unsigned o = off;
        off = (off + bytes + 15u) & ~15u;
        return o;
    };
    f.ntiles = (cap + FETCH_ROWS / 8 - 1) / (FETCH_ROWS / 8);
    f.q = take((unsigned)(G + 1) * 136u * 2u);
    f.o = take((unsigned)G * 128u * 4u);
    f.m = take(16u * 4u);
    f.l = take(16u * 4u);
    f.s = take((unsigned)FETCH_ROWS * 16u * 4u);
    f.zp = take((unsigned)FX_PPITCH * 2u);
    f.pt = take((unsigned)G * FX_PPITCH * 2u);
    f.p = take((unsigned)f.ntiles * G * FX_PPITCH * 2u);
    f.tml = take((unsigned)(f.ntiles + 1) * 16u * 8u);
    f.grp = take((unsigned)((buf_len + 7) / 8 + 1) * 4u);
    f.msb = take((unsigned)((K + 31) / 32) * 4u);
    f.bytes = off;
    return f;
}
// Rank 0's message to every CTA of the cluster: a (count, 0) pair and K
// (chunk id, slot) pairs, padded to 16 bytes.
__host__ __device__ inline unsigned fetch_msg_bytes(int K) { return (unsigned)(((K + 2) & ~1) * 8); }
__host__ __device__ inline int fetch_kt(int rank) { return rank + 8 > FETCH_PITCH ? rank + 8 : FETCH_PITCH; }
FetchLayout fetch_layout(int L, int num_chunks, int G, int K, int rank, int buf_len);

// keys_kernel: the selection keys of every landmark from the scoring
// kernel's logits and split partials, spread over the whole GPU (long
// contexts, where the selection's clusters alone would take long to read the
// logits).  grid = (ceil(L / rows), BH), KEYS_T threads.
constexpr int KEYS_T = 512;  // 16 warps: one per query head of a group when the partials are merged
struct KeysArgs {
    const float *logits;   // [BH][L][G]
    const float2 *part;    // [BH][G][nsplit]
    uint32_t *keys;        // [BH][L]
    int G, L, nsplit, rows;
};
int launch_keys(const KeysArgs &k, int BH, cudaStream_t stream);

constexpr int SEL_RING = 2;              // logits tiles in flight per CTA
constexpr size_t SEL_SMEM_CAP = 188 * 1024;  // dynamic shared memory of a selection CTA (static ~37 KB)
constexpr int SEL_RSTAGE = 32 * 1024;    // bytes per logits tile

// Keys + chunk ids of a CTA's slice and the two bitmaps (bytes).
__host__ __device__ inline size_t select_base_bytes(int L, int num_chunks, bool keys_global, int cl)
{
    const size_t slice = (size_t)((L + cl - 1) / cl);
    const size_t nbw = (size_t)((num_chunks + 31) / 32);
    return (keys_global ? 0 : slice * 8) + 2 * nbw * 4;
}

// Logits ring of one selection CTA (bytes): one tile when the slice fits in
// one, else SEL_RING full tiles; none for group sizes read directly.
__host__ __device__ inline size_t select_ring_bytes(int L, int G, int cl)
{
    if (!(G == 4 || G == 8 || G == 16)) return 0;
    const size_t slice_bytes = (size_t)((L + cl - 1) / cl) * G * 4;
    const size_t kps_bytes = (size_t)((SEL_RSTAGE / (G * 4)) & ~31) * G * 4;
    if (slice_bytes <= kps_bytes) return (slice_bytes + 127) & ~(size_t)127;
    const size_t ntile = (slice_bytes + kps_bytes - 1) / kps_bytes;
    return (size_t)(ntile < SEL_RING ? ntile : SEL_RING) * SEL_RSTAGE;
}

// Dynamic shared memory of one CTA of the selection kernel (cl CTAs per cluster).
size_t select_smem_bytes(int L, int num_chunks, int G, bool keys_global, int cl, bool keys_pre = false);

// Whether 16-CTA clusters of the selection kernel can be scheduled on this device.
bool select_cluster16_ok(size_t smem);

int launch_select(const SelectArgs &a, int BH, size_t smem, int cl, cudaStream_t stream);
int launch_select_fetch(const SelectArgs &a, int BH, size_t smem, cudaStream_t stream);

// Whether skv_decode_step uses the early-fetch selection (process-wide; off by default).
bool step_early_fetch();

// skv_decode_append_select on a cudaStream_t (for the library's own callers);
// row_dev (optional): the append row read on the device instead of `row`
int append_select_launch(const skv_decode_geom *g, const void *q, const void *k_new, const void *v_new,
                         const int64_t *positions, const void *cos_sin, void *q_out, void *k_buf, void *v_buf,
                         int row, const void *landmarks, const int64_t *landmark_idx, int32_t *slots,
                         int32_t *miss_slot, int32_t *miss_chunk, int32_t *miss_count, void *workspace,
                         size_t workspace_bytes, cudaStream_t stream, const int32_t *row_dev,
                         const SelectArgs *fetch = nullptr, bool *fetched = nullptr, bool after_stage = false);
// fetch (optional): the early-fetch fields of SelectArgs (v_host .. v_buf and
// q_rot .. seq_len, pstride; already validated); when the geometry allows it
// the selection runs as the FETCH variant, which leaves the missed rows' keys
// and values in k_buf / v_buf and writes the step's attention output, and
// *fetched is set.
// after_stage: the kernel before this call on the stream is the step's input
// staging kernel; the scoring kernel is then launched as its programmatic
// dependent and streams its first landmark tiles while the staged inputs are
// still crossing the host link.

// skv_decode_sparse_attention with a device-side position: row_dev (optional)
// holds the row the step appended at; the attention covers [0, *row_dev + 1),
// at most seq_len rows (which sizes the grid and the workspace)
int sparse_attention_launch(const skv_decode_geom *g, const void *q, const void *U, const void *SVt,
                            const void *cos_sin, const void *v_host, void *k_buf, void *v_buf,
                            const int32_t *miss_slot, const int32_t *miss_chunk, const int32_t *miss_count,
                            int seq_len, void *out, void *workspace, size_t workspace_bytes, cudaStream_t stream,
                            const int32_t *row_dev);

}  // namespace skv
