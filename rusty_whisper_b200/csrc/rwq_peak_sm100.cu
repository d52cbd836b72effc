// rwq_peak_sm100.cu -- dense tensor-core rate of this GPU, measured with
// the instructions the GEMMs use: back-to-back `tcgen05.mma` (M = 128,
// N = 256) from shared-memory operands into one TMEM accumulator, one CTA
// per SM, kind::i8 (K = 32, s8 x s8 -> s32) or kind::f16 (K = 16, f16 x
// f16 -> f32).  The operands are a fixed pseudo-random byte pattern (not
// zeros, which would understate the power draw).  The roofline
// denominators of the int8 and f16 tensor paths come from here; the bf16
// denominator stays cuBLAS's measured rate.
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdio>
#include "../../include/rwq.h"
#include "rwq_internal.h"
#include "rwq_sm100.cuh"

namespace rwq {
namespace {

using namespace tc;

constexpr int PK_N = 256;
constexpr int PK_TILE = 128 * 128;           // A: 128 rows x 128 bytes, 128-byte swizzle
// Shared memory beyond the operands' 48 KiB so that one CTA occupies an SM.
constexpr int PK_SMEM = 120 * 1024;
static_assert(PK_TILE + PK_N * 128 + 1024 + 64 <= PK_SMEM, "operands fit");

template <int KIND>   // 0 = i8, 1 = f16
__global__ void __launch_bounds__(128, 1) k_mma_peak(long long iters, int* err_flag) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint64_t* done = reinterpret_cast<uint64_t*>(base + PK_TILE + PK_N * 128);
    uint32_t* tbase = reinterpret_cast<uint32_t*>(done + 1);
    __shared__ int abort_flag;
    // Fill both operands: small signed bytes / f16 values of magnitude < 2.
    for (int i = threadIdx.x; i < (PK_TILE + PK_N * 128) / 4; i += blockDim.x) {
        uint32_t h = uint32_t(i) * 2654435761u + blockIdx.x * 97u;
        h ^= h >> 15;
        uint32_t v = KIND == 0 ? (h & 0x3F3F3F3Fu) : ((h & 0x03FF03FFu) | 0x3C003C00u);
        reinterpret_cast<uint32_t*>(base)[i] = v;
    }
    if (threadIdx.x == 0) {
        mbar_init(done, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (threadIdx.x < 32) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tbase)),
                     "r"(PK_N)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tbase;
    if (threadIdx.x == 0) {
        const uint32_t a0 = smem_u32(base), b0 = a0 + PK_TILE;
        // i8: D s32, A/B signed 8-bit; f16: D f32, A/B f16.  K-major both.
        constexpr uint32_t IDESC = KIND == 0 ? ((2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(PK_N >> 3) << 17) |
                                                (uint32_t(128 >> 4) << 24))
                                             : ((1u << 4) | (uint32_t(PK_N >> 3) << 17) | (uint32_t(128 >> 4) << 24));
        for (long long i = 0; i < iters; ++i) {
            const uint32_t off = uint32_t(i & 3) * 32u;
            const uint64_t ad = sw128_desc(a0 + off), bd = sw128_desc(b0 + off);
            const uint32_t acc = i != 0;
            if (KIND == 0)
                asm volatile(
                    "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p; }" ::"r"(
                        tmem),
                    "l"(ad), "l"(bd), "r"(IDESC), "r"(acc)
                    : "memory");
            else
                mma_f16_id(tmem, ad, bd, IDESC, acc);
        }
        mma_commit(done);
        mbar_wait(done, 0, &abort_flag, err_flag, 21);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x < 32)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PK_N) : "memory");
}

}  // namespace
}  // namespace rwq

extern "C" int rwq_mma_peak(int kind, long long iters, int ctas, double* tops, double* ms) {
    if ((kind != 0 && kind != 1) || iters <= 0 || !tops) {
        rwq::set_last_error("rwq_mma_peak: kind must be 0 (i8) or 1 (f16), iters > 0, tops non-null");
        return RWQ_ERR_ARG;
    }
    int dev = 0;
    cudaGetDevice(&dev);
    if (ctas <= 0) cudaDeviceGetAttribute(&ctas, cudaDevAttrMultiProcessorCount, dev);
    auto kern = kind == 0 ? rwq::k_mma_peak<0> : rwq::k_mma_peak<1>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, rwq::PK_SMEM);
    int* err = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (e == cudaSuccess) e = cudaMalloc(&err, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(err, 0, sizeof(int));
    if (e == cudaSuccess) e = cudaEventCreate(&e0);
    if (e == cudaSuccess) e = cudaEventCreate(&e1);
    float t = 0.f;
    int code = 0;
    if (e == cudaSuccess) {
        kern<<<ctas, 128, rwq::PK_SMEM>>>(iters / 8 + 1, err);   // warm-up
        cudaEventRecord(e0);
        kern<<<ctas, 128, rwq::PK_SMEM>>>(iters, err);
        cudaEventRecord(e1);
        e = cudaEventSynchronize(e1);
        if (e == cudaSuccess) e = cudaEventElapsedTime(&t, e0, e1);
        if (e == cudaSuccess) e = cudaMemcpy(&code, err, sizeof(int), cudaMemcpyDeviceToHost);
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (err) cudaFree(err);
    if (e != cudaSuccess) {
        char buf[256];
        snprintf(buf, sizeof buf, "rwq_mma_peak: %s", cudaGetErrorString(e));
        rwq::set_last_error(buf);
        return RWQ_ERR_CUDA;
    }
    if (code) {
        rwq::set_last_error("rwq_mma_peak: bounded wait expired");
        return RWQ_ERR_DEVICE;
    }
    const double k = kind == 0 ? 32.0 : 16.0;
    *tops = double(ctas) * double(iters) * 2.0 * 128.0 * rwq::PK_N * k / (double(t) * 1e-3) / 1e12;
    if (ms) *ms = t;
    return RWQ_OK;
}
