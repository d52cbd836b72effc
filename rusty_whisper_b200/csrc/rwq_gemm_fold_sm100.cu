// rwq_gemm_fold_sm100.cu -- encoder GEMM with the weight scales folded into
// the tensor-core operand (the default kernel for m > 8).
//
// rusty_whisper's int8 path computes (quant.rs:10, 349-354, 452-454)
//     y[i,j] = sum_kb d_a[i,kb] * ( sum_{l<32} q_a[i,32kb+l] * x[j,32kb+l] )
// where x = d_b*q_b + m_b is the dequantized weight (the reference's
// d_a*d_b*S + m_b*d_a*sum(q_a) is the same sum).  Only d_a has to be applied
// per block on the CUDA cores; x goes into the B operand.  Each weight row
// is scaled by a power of two 2^e_j (exact) so its largest |x| lies in
// [2^10, 2^11), then split into f16 hi + lo (x*2^e = hi + lo to 22 bits;
// exact for the _0 formats, whose d*q has at most 19 significant bits).
// The activation codes q_a (|q| <= 127) are exact in f16.  Per 32-wide
// block, four `tcgen05.mma.kind::f16` (two K halves x {hi, lo}) leave
//     T[i,j,kb] = sum_l q_a * (hi + lo)
// in an f32 TMEM buffer; the epilogue does acc <- fma(d_a, T, acc) with
// packed f32x2 math, and finally y = acc * 2^-e_j (+ bias).
//
// Roles (320 threads, one CTA per 128 x BN output tile, BN = 128 or 256):
//   warp 0     TMA producer: A (q_a f16, two blocks = 64 K per stage),
//              B (hi|lo rows, 64 f16 per block), both 128-byte swizzled,
//              and a 1-D bulk copy of the block's d_a row into a shared
//              ring; allocates / frees the 512 TMEM columns.
//   warp 1     MMA issuer (one thread), NBUF = 512/BN accumulator buffers.
//   warps 2-9  epilogue: warp w reads TMEM lanes 32*(w%4).., columns
//              (w-2)/4 * BN/2 .. + BN/2, 64 per round trip; at the end it
//              scales, adds the bias, stages its 32-row block in shared
//              memory (the drained B ring) and writes it with TMA stores,
//              which clip the ragged M and N edges.
// Every wait is bounded (see rwq_sm100.cuh).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cstdio>
#include <cstring>
#include <mutex>
#include "rwq_common.cuh"
#include "rwq_internal.h"
#include "rwq_sm100.cuh"

namespace rwq {
namespace {

using namespace tc;

constexpr int BM = 128;
constexpr int SA = 3;                      // A stages, two 32-wide blocks each (128-byte swizzle)
constexpr int SB = 4;                      // B stages, one block each
constexpr int EPI_WARPS = 8;
constexpr int THREADS = (2 + EPI_WARPS) * 32;
constexpr int A_STAGE = BM * 64 * 2;       // 16 KiB: 128 rows x 64 f16
constexpr int SC_SLOTS = 8;                // d_a rows, 128 floats each
constexpr int TMEM_COLS = 512;

template <int BN>
struct Cfg {
    static constexpr int B_STAGE = BN * 64 * 2;      // BN rows x (32 hi + 32 lo) f16
    static constexpr int NBUF = TMEM_COLS / BN;
    static constexpr int CPW = BN / 2;               // output columns per epilogue warp
    static constexpr int SMEM = SB * B_STAGE + SA * A_STAGE + SC_SLOTS * 512 + 1024 + 512;
    // kind::f16, D f32, A/B f16, K-major, N>>3 at bit 17, M>>4 at bit 24.
    static constexpr uint32_t IDESC = (1u << 4) | (uint32_t(BN >> 3) << 17) | (uint32_t(BM >> 4) << 24);
    // The output staging (one 32 x CPW f32 block per epilogue warp) reuses the B ring.
    static_assert(EPI_WARPS * 32 * CPW * 4 <= SB * B_STAGE, "staging must fit in the B ring");
};

struct Bars {
    uint64_t fullA[SA], emptyA[SA], fullB[SB], emptyB[SB], acc_full[4], acc_empty[4], sc_full[SC_SLOTS],
        sc_empty[SC_SLOTS];
    uint32_t tmem_base;
    int abort;
};

template <int BN>
__global__ void __launch_bounds__(THREADS, 1)
    k_gemm_fold(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmY, int use_tma_store, const float* __restrict__ daT,
                const float* __restrict__ colscale, const float* __restrict__ bias, float* __restrict__ Y, int M,
                int N, int nb, int m_pad, int* __restrict__ err_flag) {
    using C = Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sB = base;                                   // all stages 1024-aligned (128-byte swizzle)
    uint8_t* sA = base + SB * C::B_STAGE;
    float* ring = reinterpret_cast<float*>(sA + SA * A_STAGE);
    Bars* bar = reinterpret_cast<Bars*>(reinterpret_cast<uint8_t*>(ring) + SC_SLOTS * 512);
    volatile int* abort = &bar->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;

    if (threadIdx.x == 0) {
        for (int s = 0; s < SA; ++s) {
            mbar_init(&bar->fullA[s], 1);
            mbar_init(&bar->emptyA[s], 1);
        }
        for (int s = 0; s < SB; ++s) {
            mbar_init(&bar->fullB[s], 1);
            mbar_init(&bar->emptyB[s], 1);
        }
        for (int b = 0; b < C::NBUF; ++b) {
            mbar_init(&bar->acc_full[b], 1);
            mbar_init(&bar->acc_empty[b], EPI_WARPS);
        }
        for (int c = 0; c < SC_SLOTS; ++c) {
            mbar_init(&bar->sc_full[c], 1);
            mbar_init(&bar->sc_empty[c], EPI_WARPS);
        }
        bar->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&bar->tmem_base)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bar->tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
            for (int kb = 0; kb < nb; ++kb) {
                if ((kb & 1) == 0) {
                    const int t = kb >> 1, s = t % SA;
                    if (!mbar_wait(&bar->emptyA[s], ((t / SA) & 1) ^ 1, abort, err_flag, 1)) break;
                    mbar_expect_tx(&bar->fullA[s], A_STAGE);
                    tma_load_2d(sA + s * A_STAGE, &tmA, kb * 32, m0, &bar->fullA[s]);
                }
                const int s = kb % SB;
                if (!mbar_wait(&bar->emptyB[s], ((kb / SB) & 1) ^ 1, abort, err_flag, 1)) break;
                mbar_expect_tx(&bar->fullB[s], C::B_STAGE);
                tma_load_2d(sB + s * C::B_STAGE, &tmB, kb * 64, n0, &bar->fullB[s]);
                const int c = kb % SC_SLOTS;
                if (!mbar_wait(&bar->sc_empty[c], ((kb / SC_SLOTS) & 1) ^ 1, abort, err_flag, 5)) break;
                mbar_expect_tx(&bar->sc_full[c], 512);
                bulk_load(ring + c * 128, daT + size_t(kb) * m_pad + m0, 512, &bar->sc_full[c]);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (int kb = 0; kb < nb; ++kb) {
                const int t = kb >> 1, sa = t % SA, sb = kb % SB;
                if ((kb & 1) == 0 && !mbar_wait(&bar->fullA[sa], (t / SA) & 1, abort, err_flag, 2)) break;
                if (!mbar_wait(&bar->fullB[sb], (kb / SB) & 1, abort, err_flag, 2)) break;
                const int buf = kb % C::NBUF;
                if (!mbar_wait(&bar->acc_empty[buf], ((kb / C::NBUF) & 1) ^ 1, abort, err_flag, 3)) break;
                tc_fence_after();
                const uint32_t a0 = smem_u32(sA + sa * A_STAGE) + uint32_t((kb & 1) * 64);
                const uint32_t b0 = smem_u32(sB + sb * C::B_STAGE);
                const uint32_t d = tmem + uint32_t(buf * BN);
                // K half 0: A bytes +0..31, B hi +0..31, lo +64..95;
                // K half 1: A bytes +32..63, B hi +32..63, lo +96..127.
                mma_f16_id(d, sw128_desc(a0), sw128_desc(b0), C::IDESC, 0);
                mma_f16_id(d, sw128_desc(a0), sw128_desc(b0 + 64), C::IDESC, 1);
                mma_f16_id(d, sw128_desc(a0 + 32), sw128_desc(b0 + 32), C::IDESC, 1);
                mma_f16_id(d, sw128_desc(a0 + 32), sw128_desc(b0 + 96), C::IDESC, 1);
                mma_commit(&bar->acc_full[buf]);
                mma_commit(&bar->emptyB[sb]);
                if ((kb & 1) == 1 || kb == nb - 1) mma_commit(&bar->emptyA[sa]);
            }
        }
    } else {
        const int q = warp & 3;
        const int h = (warp - 2) >> 2;
        constexpr int CPW = C::CPW;
        float2 acc[CPW / 2];
#pragma unroll
        for (int c = 0; c < CPW / 2; ++c) acc[c] = make_float2(0.f, 0.f);
        for (int kb = 0; kb < nb; ++kb) {
            const int buf = kb % C::NBUF;
            const int c = kb % SC_SLOTS;
            const bool got = mbar_wait(&bar->sc_full[c], (kb / SC_SLOTS) & 1, abort, err_flag, 6) &&
                             mbar_wait(&bar->acc_full[buf], (kb / C::NBUF) & 1, abort, err_flag, 4);
            if (!__all_sync(0xffffffffu, got)) break;
            tc_fence_after();
            const float da = ring[c * 128 + q * 32 + lane];
            const float2 da2 = make_float2(da, da);
            const uint32_t taddr = tmem + (uint32_t(q * 32) << 16) + uint32_t(buf * BN + h * CPW);
            // 64 columns per TMEM round trip.
#pragma unroll
            for (int ch = 0; ch < CPW / 64; ++ch) {
                uint32_t r[64];
                tmem_ld32(taddr + ch * 64, r);
                tmem_ld32(taddr + ch * 64 + 32, r + 32);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    acc[ch * 32 + i] =
                        __ffma2_rn(da2, make_float2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])),
                                   acc[ch * 32 + i]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bar->acc_empty[buf]);
                mbar_arrive(&bar->sc_empty[c]);
            }
        }
        // y = acc * 2^-e_j (+ bias), written through shared memory.
        const int col0 = n0 + h * CPW;
        const bool bias_vec = (reinterpret_cast<uintptr_t>(bias) & 15) == 0;
        const int row = m0 + q * 32 + lane;
        if (!*abort) {
            if (use_tma_store) {
                // Staging for this warp: CPW/32 boxes of 32 rows x 128 bytes,
                // 128-byte swizzle (16-byte chunk c of row r at c ^ (r & 7)).
                uint8_t* stg = sB + (warp - 2) * (32 * CPW * 4);
#pragma unroll
                for (int b = 0; b < CPW / 32; ++b) {
                    uint8_t* box = stg + b * 4096 + lane * 128;
#pragma unroll
                    for (int c4 = 0; c4 < 8; ++c4) {
                        const int col = col0 + b * 32 + c4 * 4;   // < n0 + BN <= padded width
                        const float4 cs = __ldg(reinterpret_cast<const float4*>(colscale + col));
                        const float2 a01 = acc[b * 16 + c4 * 2], a23 = acc[b * 16 + c4 * 2 + 1];
                        float4 v = make_float4(__fmul_rn(a01.x, cs.x), __fmul_rn(a01.y, cs.y),
                                               __fmul_rn(a23.x, cs.z), __fmul_rn(a23.y, cs.w));
                        if (bias && col < N) {  // N % 4 == 0 on this path
                            const float4 bb = bias_vec ? __ldg(reinterpret_cast<const float4*>(bias + col))
                                                       : make_float4(__ldg(bias + col), __ldg(bias + col + 1),
                                                                     __ldg(bias + col + 2), __ldg(bias + col + 3));
                            v.x = __fadd_rn(v.x, bb.x); v.y = __fadd_rn(v.y, bb.y);
                            v.z = __fadd_rn(v.z, bb.z); v.w = __fadd_rn(v.w, bb.w);
                        }
                        *reinterpret_cast<float4*>(box + ((c4 ^ (lane & 7)) << 4)) = v;
                    }
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) {
#pragma unroll
                    for (int b = 0; b < CPW / 32; ++b)
                        if (col0 + b * 32 < N && m0 + q * 32 < M)
                            tma_store_2d(&tmY, col0 + b * 32, m0 + q * 32, stg + b * 4096);
                    bulk_commit();
                    bulk_wait_read_all();
                }
                __syncwarp();
            } else if (row < M) {
                float* yr = Y + size_t(row) * N;
#pragma unroll
                for (int cc = 0; cc < CPW / 2; ++cc) {
                    const int col = col0 + 2 * cc;
                    if (col < N) {
                        const float v = __fmul_rn(acc[cc].x, __ldg(colscale + col));
                        yr[col] = bias ? __fadd_rn(v, __ldg(bias + col)) : v;
                    }
                    if (col + 1 < N) {
                        const float v = __fmul_rn(acc[cc].y, __ldg(colscale + col + 1));
                        yr[col + 1] = bias ? __fadd_rn(v, __ldg(bias + col + 1)) : v;
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

// ------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_once;

bool encode_map(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* ptr, uint64_t inner, uint64_t rows,
                uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw, char* why, size_t why_len) {
    std::call_once(g_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!g_encode) {
        snprintf(why, why_len, "cuTensorMapEncodeTiled entry point unavailable");
        return false;
    }
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {inner * uint64_t(esize)};
    cuuint32_t box[2] = {box_inner, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        snprintf(why, why_len, "cuTensorMapEncodeTiled failed (%d)", int(r));
        return false;
    }
    return true;
}

template <int BN>
cudaError_t launch_bn(const ActsView& v, const Weight& w, const float* bias, float* y, int* err_flag,
                      cudaStream_t s, char* why, size_t why_len) {
    CUtensorMap ma, mb, my;
    if (!encode_map(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, v.q16, uint64_t(v.k), uint64_t(v.m), 64, BM,
                    CU_TENSOR_MAP_SWIZZLE_128B, why, why_len))
        return cudaErrorInvalidValue;
    if (!encode_map(&mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, w.bhl, uint64_t(w.nb) * 64, uint64_t(w.n), 64, BN,
                    CU_TENSOR_MAP_SWIZZLE_128B, why, why_len))
        return cudaErrorInvalidValue;
    // Output through TMA stores when the row pitch is 16-byte aligned.
    int use_tma_store = (w.n % 4 == 0) && (reinterpret_cast<uintptr_t>(y) % 16 == 0);
    if (use_tma_store && !encode_map(&my, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, y, uint64_t(w.n), uint64_t(v.m), 32, 32,
                                     CU_TENSOR_MAP_SWIZZLE_128B, why, why_len))
        use_tma_store = 0;
    if (!use_tma_store) memset(&my, 0, sizeof my);
    auto kern = k_gemm_fold<BN>;
    static int attr_dev_mask = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_dev_mask & (1 << dev))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<BN>::SMEM);
        if (e != cudaSuccess) return e;
        attr_dev_mask |= 1 << dev;
    }
    dim3 grid((w.n + BN - 1) / BN, (v.m + BM - 1) / BM);
    kern<<<grid, THREADS, Cfg<BN>::SMEM, s>>>(ma, mb, my, use_tma_store, v.dT, w.colscale, bias, y, v.m, w.n, w.nb,
                                              v.m_pad, err_flag);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm_fold(const ActsView& v, const Weight& w, const float* bias, float* y, int* err_flag,
                             cudaStream_t s, char* why, size_t why_len) {
    if (v.m <= 0 || w.n <= 0) return cudaSuccess;
    // 256-wide tiles for wide outputs.  The choice depends on N only, so a
    // row's result never depends on M.
    if (w.n >= 2304) return launch_bn<256>(v, w, bias, y, err_flag, s, why, why_len);
    return launch_bn<128>(v, w, bias, y, err_flag, s, why, why_len);
}

}  // namespace rwq
