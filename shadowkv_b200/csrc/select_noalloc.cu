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
//    before any stream capture;
//  * the address is cached per CUDA context: after cudaDeviceReset (or any
//    other way the device's primary context is destroyed and created again)
//    the next call looks it up again in the new context, so that call, too,
//    must come before any stream capture.
#include "common.cuh"

#include <cuda.h>
#include <mutex>
#include <utility>

namespace skv {

constexpr size_t NOALLOC_SCRATCH_BYTES = 32u << 20;
constexpr int NOALLOC_MAX_DEVICES = 64;

static __device__ __align__(256) unsigned char g_noalloc_select_scratch[NOALLOC_SCRATCH_BYTES];

static void *s_scratch_ptr[NOALLOC_MAX_DEVICES];
static unsigned long long s_scratch_ctx[NOALLOC_MAX_DEVICES];  // id of the context of the cached address
static std::mutex s_scratch_mu;

// Unique id of the calling thread's current driver context (cuCtxGetCurrent +
// cuCtxGetId, reached through the runtime's driver entry points: the library
// does not link libcuda itself); 0 when there is none or it cannot be read.
// Ids are never reused within a process, so a context created after a
// cudaDeviceReset has a new one.
static unsigned long long current_context_id()
{
    typedef CUresult (*CtxGetCurrent)(CUcontext *);
    typedef CUresult (*CtxGetId)(CUcontext, unsigned long long *);
    static const std::pair<CtxGetCurrent, CtxGetId> fns = []() {
        void *p = nullptr, *q = nullptr;
        cudaDriverEntryPointQueryResult r1, r2;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &r1) != cudaSuccess ||
            r1 != cudaDriverEntryPointSuccess ||
            cudaGetDriverEntryPoint("cuCtxGetId", &q, cudaEnableDefault, &r2) != cudaSuccess ||
            r2 != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return std::pair<CtxGetCurrent, CtxGetId>(nullptr, nullptr);
        }
        return std::pair<CtxGetCurrent, CtxGetId>(reinterpret_cast<CtxGetCurrent>(p), reinterpret_cast<CtxGetId>(q));
    }();
    CUcontext c = nullptr;
    unsigned long long id = 0;
    if (fns.first == nullptr || fns.first(&c) != CUDA_SUCCESS || c == nullptr) return 0;
    if (fns.second(c, &id) != CUDA_SUCCESS) return 0;
    return id;
}

// Device address of the scratch array in the current context: looked up once
// per device and context, and on every call when the context cannot be
// identified.
static int noalloc_scratch(void **out)
{
    int dev = 0;
    SKV_CUDA(cudaGetDevice(&dev));
    SKV_CHECK_SUPPORTED(dev >= 0 && dev < NOALLOC_MAX_DEVICES, "device index %d above %d", dev,
                        NOALLOC_MAX_DEVICES - 1);
    const unsigned long long ctx = current_context_id();
    std::lock_guard<std::mutex> lock(s_scratch_mu);
    if (s_scratch_ptr[dev] != nullptr && ctx != 0 && s_scratch_ctx[dev] == ctx) {
        *out = s_scratch_ptr[dev];
        return SKV_OK;
    }
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_select_scratch);
    if (e != cudaSuccess || p == nullptr) {
        cudaGetLastError();
        set_error("cudaGetSymbolAddress of the selection scratch failed on device %d: %s", dev,
                  cudaGetErrorString(e));
        return SKV_ERR_CUDA;
    }
    s_scratch_ptr[dev] = p;
    s_scratch_ctx[dev] = current_context_id();  // the lookup made the device's context current
    *out = p;
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
