// Error plumbing shared by all entry points of the C ABI.
#include "common.cuh"

#include <string.h>
#include <atomic>
#include <mutex>

namespace skv {

static thread_local char t_last_error[512] = "";

void set_error(const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
    va_end(ap);
}

void clear_error() { t_last_error[0] = '\0'; }

int check_launch(const char *what)
{
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error("launch of %s failed: %s", what, cudaGetErrorString(e));
        return SKV_ERR_CUDA;
    }
    return SKV_OK;
}

int ensure_smem_attr(const void *func, int bytes, const char *name)
{
    struct Entry {
        const void *func;
        int device;
        int bytes;
    };
    static Entry table[256];
    static int used = 0;
    static std::mutex mu;
    int dev = 0;
    SKV_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < used; ++i)
        if (table[i].func == func && table[i].device == dev) {
            if (table[i].bytes >= bytes) return SKV_OK;
            cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
            if (e != cudaSuccess) {
                set_error("cudaFuncSetAttribute(%s, %d bytes) failed: %s", name, bytes, cudaGetErrorString(e));
                return SKV_ERR_CUDA;
            }
            table[i].bytes = bytes;
            return SKV_OK;
        }
    cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) {
        set_error("cudaFuncSetAttribute(%s, %d bytes) failed: %s", name, bytes, cudaGetErrorString(e));
        return SKV_ERR_CUDA;
    }
    if (used < 256) table[used++] = Entry{func, dev, bytes};
    return SKV_OK;
}

int host_to_device_ptr(const void *p, const void **dev, const char *name)
{
    if (p == nullptr) {
        set_error("%s is null", name);
        return SKV_ERR_INVALID_ARGUMENT;
    }
    cudaPointerAttributes attr;
    cudaError_t e = cudaPointerGetAttributes(&attr, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("%s: cudaPointerGetAttributes failed: %s", name, cudaGetErrorString(e));
        return SKV_ERR_NOT_PINNED;
    }
    if (attr.type != cudaMemoryTypeHost) {
        set_error("%s must be page-locked host memory mapped into the device address space "
                  "(pointer type %d)", name, (int)attr.type);
        return SKV_ERR_NOT_PINNED;
    }
    if (attr.devicePointer == nullptr) {
        set_error("%s is page-locked but not mapped for the device", name);
        return SKV_ERR_NOT_PINNED;
    }
    // the device pointer of the start of the allocation plus p's offset
    *dev = attr.devicePointer;
    return SKV_OK;
}

int out_to_device_ptr(void *p, void **dev, const char *name)
{
    if (p == nullptr) {
        set_error("%s is null", name);
        return SKV_ERR_INVALID_ARGUMENT;
    }
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        attr.type = cudaMemoryTypeUnregistered;
    }
    if (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged) {
        *dev = p;
        return SKV_OK;
    }
    if (attr.type == cudaMemoryTypeHost && attr.devicePointer != nullptr) {
        *dev = attr.devicePointer;
        return SKV_OK;
    }
    set_error("%s must be device memory or page-locked host memory mapped for the device", name);
    return SKV_ERR_INVALID_ARGUMENT;
}

int in_to_device_ptr(const void *p, const void **dev, bool *host, const char *name)
{
    if (p == nullptr) {
        set_error("%s is null", name);
        return SKV_ERR_INVALID_ARGUMENT;
    }
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        attr.type = cudaMemoryTypeUnregistered;
    }
    if (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged) {
        *dev = p;
        *host = false;
        return SKV_OK;
    }
    if (attr.type == cudaMemoryTypeHost && attr.devicePointer != nullptr) {
        *dev = attr.devicePointer;
        *host = true;
        return SKV_OK;
    }
    set_error("%s must be device memory or page-locked host memory mapped for the device", name);
    return SKV_ERR_INVALID_ARGUMENT;
}

typedef CUresult (*TensorMapEncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                         const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                         CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                         CUtensorMapFloatOOBfill);

int encode_tensor_map_bf16(CUtensorMap *m, const void *base, unsigned rank, const cuuint64_t *dims,
                           const cuuint64_t *strides, const cuuint32_t *box, CUtensorMapSwizzle swizzle,
                           const char *name)
{
    static const TensorMapEncodeTiled enc = []() -> TensorMapEncodeTiled {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        return reinterpret_cast<TensorMapEncodeTiled>(p);
    }();
    SKV_CHECK_SUPPORTED(enc != nullptr, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void *>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed for %s (CUresult %d)", name, (int)r);
        return SKV_ERR_CUDA;
    }
    return SKV_OK;
}

int device_sm_count()
{
    static std::atomic<int> cached[64];  // 0: not queried yet (host threads may race here)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return 148;
    }
    int n = cached[dev].load(std::memory_order_relaxed);
    if (n > 0) return n;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        return 148;
    }
    cached[dev].store(n, std::memory_order_relaxed);
    return n;
}

__device__ unsigned int g_dev_err_count = 0;
__device__ unsigned int g_dev_err_first = 0;
#ifdef SKV_TRACE
__device__ unsigned long long g_trace[2 * SKV_TRACE_EVENTS];
__device__ unsigned long long g_trace_rec[SKV_TRACE_RECS * SKV_TRACE_FIELDS];
__device__ unsigned int g_trace_nrec = 0;
#endif

}  // namespace skv

extern "C" {

const char *skv_last_error(void) { return skv::t_last_error; }

int skv_version(void) { return 1 * 10000 + 0 * 100 + 0; }

int skv_device_errors(uint32_t *count, uint32_t *first_code)
{
    unsigned int c = 0, f = 0, zero = 0;
    SKV_CUDA(cudaMemcpyFromSymbol(&c, skv::g_dev_err_count, sizeof(c)));
    SKV_CUDA(cudaMemcpyFromSymbol(&f, skv::g_dev_err_first, sizeof(f)));
    SKV_CUDA(cudaMemcpyToSymbol(skv::g_dev_err_count, &zero, sizeof(zero)));
    SKV_CUDA(cudaMemcpyToSymbol(skv::g_dev_err_first, &zero, sizeof(zero)));
    if (count) *count = c;
    if (first_code) *first_code = f;
    return SKV_OK;
}

#ifdef SKV_TRACE
__global__ void trace_mark_kernel(int e) { skv::trace_stamp(e); }
// Trace builds only: one thread stamps event e on the stream.
SKV_API int skv_trace_mark(int e, void *stream)
{
    trace_mark_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(e);
    return skv::check_launch("trace_mark_kernel");
}
// Trace builds only (not part of the public header): copy the 2 * n trace
// slots into out (earliest / latest stamp of each event, ns of the global
// timer) and reset them.
SKV_API int skv_trace_read(unsigned long long *out, int n)
{
    unsigned long long h[2 * skv::SKV_TRACE_EVENTS];
    SKV_CUDA(cudaMemcpyFromSymbol(h, skv::g_trace, sizeof(h)));
    if (out) memcpy(out, h, sizeof(unsigned long long) * 2 * (n < skv::SKV_TRACE_EVENTS ? n : skv::SKV_TRACE_EVENTS));
    for (int e = 0; e < skv::SKV_TRACE_EVENTS; ++e) {
        h[2 * e] = ~0ull;
        h[2 * e + 1] = 0ull;
    }
    SKV_CUDA(cudaMemcpyToSymbol(skv::g_trace, h, sizeof(h)));
    return SKV_OK;
}
// Trace builds only: copy up to max per-CTA records (SKV_TRACE_FIELDS words
// each) into out, reset them; returns the number of records opened.
SKV_API int skv_trace_records(unsigned long long *out, int max)
{
    unsigned int n = 0, zero = 0;
    SKV_CUDA(cudaMemcpyFromSymbol(&n, skv::g_trace_nrec, sizeof(n)));
    const int m = (int)(n < (unsigned)max ? n : (unsigned)max);
    const int k = m < skv::SKV_TRACE_RECS ? m : skv::SKV_TRACE_RECS;
    if (out && k > 0)
        SKV_CUDA(cudaMemcpyFromSymbol(out, skv::g_trace_rec, sizeof(unsigned long long) * skv::SKV_TRACE_FIELDS * k));
    SKV_CUDA(cudaMemcpyToSymbol(skv::g_trace_nrec, &zero, sizeof(zero)));
    return (int)n;
}
#endif

}  // extern "C"
