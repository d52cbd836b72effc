// rwq_noalloc.cu -- a decoder-shaped matmul that allocates no memory.
//
// Some callers cannot let this library call cudaMalloc: a live-microphone
// decode loop on a latency-critical thread, where cudaMalloc/cudaFree can
// stall on an implicit device synchronization; or an embedder whose GPU
// memory is owned by another allocator (a framework's caching pool, a
// fixed per-process budget) so the library may not reserve memory behind
// its back.  rwq_matmul_t_q_noalloc serves them for the decoder's shapes
// (m <= 8 rows, k <= 8192) with the int8 activation quantizer and the GEMV
// family of rwq_matmul_t_q_dev (launch_gemv_i8: by default the integer-MMA
// kernel, or whichever GEMV kind rwq_set_gemv_kernel chose on this host
// thread), so its results are bit-identical to rwq_matmul_t_q_dev called
// on the same thread.  Their scratch (the quantized activations) is held
// in the file-scope array below instead of a workspace.
#include <cuda_runtime.h>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include "../../include/rwq.h"
#include "rwq_common.cuh"
#include "rwq_internal.h"

namespace {

constexpr int NOALLOC_MAX_M = 8;
constexpr int NOALLOC_MAX_K = 8192;
constexpr size_t align256(size_t x) { return (x + 255) / 256 * 256; }
// Quantized activations for the largest call: int8 codes [8][8192] and
// d_a, sum(q_a), d_a*sum(q_a) [8][256] each.
constexpr size_t Q8_BYTES = align256(size_t(NOALLOC_MAX_M) * NOALLOC_MAX_K);
constexpr size_t ROW_BYTES = align256(size_t(NOALLOC_MAX_M) * (NOALLOC_MAX_K / rwq::QK) * 4);
constexpr size_t SCRATCH_BYTES = Q8_BYTES + 3 * ROW_BYTES;  // 90112 bytes (88 KiB)

// Every GPU that loads the library holds this array until the process
// exits.  In host code `g_noalloc_scratch` is only a host-side stand-in
// for the symbol, never a device address: the device address comes from
// cudaGetSymbolAddress below, once per device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_mu;
void* g_dev_ptr[MAX_DEVICES] = {};

int fail(int code, const char* fmt, ...) {
    char buf[256];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    rwq::set_last_error(buf);
    return code;
}

// Device address of the scratch array on the current device; resolved on
// the first call per device and kept.  A cudaDeviceReset while the library
// is loaded is not supported: the module would be reloaded elsewhere and
// the kept address would be stale.
int scratch_address(int dev, unsigned char** out) {
    if (dev < 0 || dev >= MAX_DEVICES) return fail(RWQ_ERR_ARG, "device %d out of range", dev);
    std::lock_guard<std::mutex> g(g_mu);
    if (!g_dev_ptr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return fail(RWQ_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
        g_dev_ptr[dev] = p;
    }
    *out = static_cast<unsigned char*>(g_dev_ptr[dev]);
    return RWQ_OK;
}

}  // namespace

extern "C" int rwq_matmul_t_q_noalloc(const float* a, int64_t m, int64_t k, const rwq_qtensor* b, const float* bias,
                                      float* out, void* stream) {
    if (!b) return fail(RWQ_ERR_ARG, "weight is null");
    const rwq::Weight& w = rwq::weight_of(b);
    if (m < 0 || m > NOALLOC_MAX_M)
        return fail(RWQ_ERR_ARG, "rwq_matmul_t_q_noalloc: m=%lld, this entry point takes 0..%d rows", (long long)m,
                    NOALLOC_MAX_M);
    if (k <= 0 || k % rwq::QK || k > NOALLOC_MAX_K)
        return fail(RWQ_ERR_ARG, "rwq_matmul_t_q_noalloc: k=%lld, needs a multiple of 32 up to %d", (long long)k,
                    NOALLOC_MAX_K);
    if (k != w.k) return fail(RWQ_ERR_SHAPE, "matmul_t_q inner dims: %lld vs %d", (long long)k, w.k);
    if (m == 0 || w.n == 0) return RWQ_OK;
    if (!a || !out) return fail(RWQ_ERR_ARG, "null activation or output pointer");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(RWQ_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev != w.device) return fail(RWQ_ERR_ARG, "weight lives on device %d, current device is %d", w.device, dev);
    unsigned char* base = nullptr;
    int rc = scratch_address(dev, &base);
    if (rc) return rc;

    // The quantizer writes every byte of the scratch the GEMV then reads
    // for these m rows, so nothing needs clearing between calls.
    rwq::ActsView v;
    v.m = int(m);
    v.k = int(k);
    v.nb = int(k / rwq::QK);
    v.m_pad = v.m;
    v.q8 = reinterpret_cast<int8_t*>(base);
    v.d = reinterpret_cast<float*>(base + Q8_BYTES);
    v.sum = reinterpret_cast<int32_t*>(base + Q8_BYTES + ROW_BYTES);
    v.u = reinterpret_cast<float*>(base + Q8_BYTES + 2 * ROW_BYTES);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if ((e = rwq::launch_quantize_acts(a, v, false, s)) != cudaSuccess)
        return fail(RWQ_ERR_CUDA, "quantize launch: %s", cudaGetErrorString(e));
    if ((e = rwq::launch_gemv_i8(v, w, bias, out, s)) != cudaSuccess)
        return fail(RWQ_ERR_CUDA, "gemv launch: %s", cudaGetErrorString(e));
    return RWQ_OK;
}
