// Allocation-free variant of skv_decode_select.
//
// Some callers cannot hand the library a scratch buffer: a serving process
// that drives the library through a foreign-function interface and owns no
// CUDA allocator of its own (it only receives the device tensors of the
// model state), or a runtime that plans every byte of device memory at
// start-up and does not allow an allocation on the token path.  For them the
// selection's scratch (per-landmark logits and per-split softmax partials)
// lives in a fixed array in the library's own device memory.
//
// Properties a caller must know:
//  * the array is 32 MiB on every GPU that loads the library and stays
//    allocated until the process exits;
//  * geometries that need more scratch are rejected with SKV_ERR_UNSUPPORTED;
//  * every call on a device shares the one array: calls whose execution
//    overlaps on the GPU (different streams, no ordering between them) race
//    on it and produce wrong selections;
//  * nothing in the array has to start at zero: each call writes every byte
//    it later reads, so the contents left by the previous call do not matter;
//  * the first call on a device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current; make that first call
//    before any stream capture.
#include "common.cuh"

#include <mutex>

namespace skv {

constexpr size_t NOALLOC_SCRATCH_BYTES = 32u << 20;
constexpr int NOALLOC_MAX_DEVICES = 64;

static __device__ __align__(256) unsigned char g_noalloc_select_scratch[NOALLOC_SCRATCH_BYTES];

static void *s_scratch_ptr[NOALLOC_MAX_DEVICES];
static std::mutex s_scratch_mu;

// Device address of the scratch array on the current device (looked up once per device).
static int noalloc_scratch(void **out)
{
    int dev = 0;
    SKV_CUDA(cudaGetDevice(&dev));
    SKV_CHECK_SUPPORTED(dev >= 0 && dev < NOALLOC_MAX_DEVICES, "device index %d above %d", dev,
                        NOALLOC_MAX_DEVICES - 1);
    std::lock_guard<std::mutex> lock(s_scratch_mu);
    if (s_scratch_ptr[dev] == nullptr) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_select_scratch);
        if (e != cudaSuccess || p == nullptr) {
            cudaGetLastError();
            set_error("cudaGetSymbolAddress of the selection scratch failed on device %d: %s", dev,
                      cudaGetErrorString(e));
            return SKV_ERR_CUDA;
        }
        s_scratch_ptr[dev] = p;
    }
    *out = s_scratch_ptr[dev];
    return SKV_OK;
}

}  // namespace skv

using namespace skv;

extern "C" {

int skv_decode_select_noalloc(const skv_decode_geom *g, const void *q, const void *landmarks,
                              const int64_t *landmark_idx, int32_t *slots, int32_t *miss_slot,
                              int32_t *miss_chunk, int32_t *miss_count, void *stream)
{
    SKV_CHECK_ARG(g != nullptr, "null geometry");
    const size_t need = skv_decode_select_workspace(g);
    SKV_CHECK_ARG(need > 0, "geometry rejected by skv_decode_select_workspace");
    SKV_CHECK_SUPPORTED(need <= NOALLOC_SCRATCH_BYTES,
                        "this geometry needs %zu bytes of selection scratch; the allocation-free entry "
                        "point holds %zu bytes (use skv_decode_select with a caller workspace)",
                        need, (size_t)NOALLOC_SCRATCH_BYTES);
    void *scratch = nullptr;
    int st = noalloc_scratch(&scratch);
    if (st) return st;
    return skv_decode_select(g, q, landmarks, landmark_idx, slots, miss_slot, miss_chunk, miss_count,
                             scratch, NOALLOC_SCRATCH_BYTES, stream);
}

}  // extern "C"
