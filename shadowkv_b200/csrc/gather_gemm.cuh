// Argument block shared by the gathered-GEMM kernels (gather_gemm.cu, gather_gemm_tc.cu).
#pragma once

#include "common.cuh"

namespace skv {

struct GatherGemmArgs {
    const __nv_bfloat16 *U;     // [B][ctx][rank]
    const __nv_bfloat16 *SVt;   // [B][H][128][rank]
    const __nv_bfloat16 *cos_sin;
    __nv_bfloat16 *out;
    const int32_t *ids;         // [B*H][M] chunk ids (entry j)
    const int32_t *slots;       // [B*H][M] destination slot of entry j (fused) or null
    const int32_t *lo;          // per-(b,h) first valid entry (drop-in: cnts) or null
    const int32_t *hi;          // per-(b,h) end of valid entries (fused: miss_count) or null
    int H, M, rank, ctx;
    int64_t out_bh_stride;      // elements between (b,h) blocks of out
    int out_row0;               // first destination row (sparse_start) in the fused path
    int cs_stride, cs_rows;
};

// tcgen05 (tensor-memory accumulator) version, 16 chunks per CTA.
int launch_gather_gemm_tc(const GatherGemmArgs &a, int rope, int nbh, cudaStream_t stream);

}  // namespace skv
