// rwq_gemm_sm100.cu -- encoder GEMM on the 5th-generation tensor cores.
//
//   Y[M,N] = sum_kb  d_a[i,kb]*d_b[j,kb] * S[i,j,kb]  (+ d_a*sum(q_a) * m_b)
//   S[i,j,kb] = sum_{l<32} q_a[i,32kb+l] * q_b[j,32kb+l]
//
// rusty_whisper scales every 32-wide K block on BOTH sides (quant.rs:10,
// 349-351, 452-454), so the integer dot of every block has to be read out
// and scaled separately.  The codes (|q| <= 128) are exact in f16, their
// products (< 2^14) and 32-term sums (< 2^20) are exact in the f32
// accumulator, so one block's S comes out of a pair of K=16
// `tcgen05.mma.kind::f16` instructions as an exact integer in f32: no
// int->float conversion is needed in the epilogue.
//
// Roles (320 threads, one CTA per 128x128 output tile):
//   warp 0     TMA producer: A = q_a (f16 codes) and B = q_b tiles, 64 K
//              elements (two quant blocks) per stage, 128-byte swizzle;
//              also allocates / frees tensor memory.
//   warp 1     MMA issuer (one thread): per quant block kb, two MMAs into
//              TMEM accumulator buffer kb % 4 (4 x 128 columns), then a
//              commit to acc_full[buf]; a commit per stage frees the stage.
//   warps 2-9  epilogue: warp w reads TMEM lanes 32*(w%4).. (its hardware
//              sub-partition), columns 64*((w-2)/4)..+63, releases the
//              buffer, then acc <- fma(d_a*d_b, S, acc) (and the min term)
//              with packed f32x2 math, in kb order.
// Every wait is bounded: on timeout the kernel records an error code,
// stops all roles, frees its tensor memory and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cstdio>
#include <cstring>
#include <mutex>
#include "rwq_common.cuh"
#include "rwq_internal.h"
#include "rwq_sm100.cuh"

namespace rwq {
namespace {

using namespace tc;

constexpr int BM = 128, BN = 128, BK = 64;  // BK f16 elements = 128 bytes per row per stage
constexpr int STAGES = 4, NBUF = 4;
constexpr int EPI_WARPS = 8;
constexpr int THREADS = (2 + EPI_WARPS) * 32;
constexpr int A_STAGE_BYTES = BM * BK * 2;   // 16 KiB
constexpr int B_STAGE_BYTES = BN * BK * 2;   // 16 KiB
constexpr int TMEM_COLS = NBUF * BN;         // 512
// Per-quant-block scale rows staged by the producer: d_a[128 rows],
// d_b[128 cols], u_a = d_a*sum(q_a) [128 rows], m_b[128 cols].
constexpr int SC_SLOTS = 8;
constexpr int SC_FLOATS = 4 * 128;
constexpr int SC_BYTES = SC_SLOTS * SC_FLOATS * 4;  // 16 KiB
constexpr int SMEM_BYTES = STAGES * (A_STAGE_BYTES + B_STAGE_BYTES) + SC_BYTES + 1024 /*align*/ + 512 /*barriers*/;

// Instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A/B f16
// (bits 7-12 = 0), both K-major, N>>3 at bits 17-22, M>>4 at bits 24-28.
constexpr uint32_t IDESC = (1u << 4) | (uint32_t(BN >> 3) << 17) | (uint32_t(BM >> 4) << 24);

struct Smem {
    uint64_t full[STAGES], empty[STAGES], acc_full[NBUF], acc_empty[NBUF], sc_full[SC_SLOTS], sc_empty[SC_SLOTS];
    uint32_t tmem_base;
    int abort;
};

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(
            d_tmem),
        "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(accumulate)
        : "memory");
}

template <bool HAS_MIN, bool DUMP>
__global__ void __launch_bounds__(THREADS, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const float* __restrict__ daT, const float* __restrict__ uaT, const float* __restrict__ dbT,
              const float* __restrict__ mbT, const float* __restrict__ bias, float* __restrict__ Y, int M, int N,
              int nb, int m_pad, int n_pad, int32_t* __restrict__ S_dump, int* __restrict__ err_flag) {
    extern __shared__ uint8_t smem_raw[];
    // 128-byte swizzle atoms need 1024-byte aligned shared addresses.
    uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sA = base;
    uint8_t* sB = base + STAGES * A_STAGE_BYTES;
    float* sc_ring = reinterpret_cast<float*>(sB + STAGES * B_STAGE_BYTES);
    Smem* sm = reinterpret_cast<Smem*>(sB + STAGES * B_STAGE_BYTES + SC_BYTES);
    volatile int* abort = &sm->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int k_tiles = (nb + 1) / 2;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&sm->full[s], 1);
            mbar_init(&sm->empty[s], 1);
        }
        for (int b = 0; b < NBUF; ++b) {
            mbar_init(&sm->acc_full[b], 1);
            mbar_init(&sm->acc_empty[b], EPI_WARPS);
        }
        for (int c = 0; c < SC_SLOTS; ++c) {
            mbar_init(&sm->sc_full[c], 1);
            mbar_init(&sm->sc_empty[c], EPI_WARPS);
        }
        sm->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm->tmem_base)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = sm->tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
            for (int kt = 0; kt < k_tiles; ++kt) {
                const int s = kt % STAGES;
                const uint32_t ph = (kt / STAGES) & 1;
                if (!mbar_wait(&sm->empty[s], ph ^ 1, abort, err_flag, 1)) break;
                mbar_expect_tx(&sm->full[s], A_STAGE_BYTES + B_STAGE_BYTES);
                tma_load_2d(sA + s * A_STAGE_BYTES, &tmA, kt * BK, m0, &sm->full[s]);
                tma_load_2d(sB + s * B_STAGE_BYTES, &tmB, kt * BK, n0, &sm->full[s]);
                bool ok = true;
                for (int j = 0; j < 2 && ok; ++j) {
                    const int kb = 2 * kt + j;
                    if (kb >= nb) break;
                    const int c = kb % SC_SLOTS;
                    const uint32_t cu = kb / SC_SLOTS;
                    if (!mbar_wait(&sm->sc_empty[c], (cu & 1) ^ 1, abort, err_flag, 5)) {
                        ok = false;
                        break;
                    }
                    float* slot = sc_ring + c * SC_FLOATS;
                    mbar_expect_tx(&sm->sc_full[c], HAS_MIN ? 2048u : 1024u);
                    bulk_load(slot, daT + size_t(kb) * m_pad + m0, 512, &sm->sc_full[c]);
                    bulk_load(slot + 128, dbT + size_t(kb) * n_pad + n0, 512, &sm->sc_full[c]);
                    if (HAS_MIN) {
                        bulk_load(slot + 256, uaT + size_t(kb) * m_pad + m0, 512, &sm->sc_full[c]);
                        bulk_load(slot + 384, mbT + size_t(kb) * n_pad + n0, 512, &sm->sc_full[c]);
                    }
                }
                if (!ok) break;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (int kt = 0; kt < k_tiles; ++kt) {
                const int s = kt % STAGES;
                const uint32_t ph = (kt / STAGES) & 1;
                if (!mbar_wait(&sm->full[s], ph, abort, err_flag, 2)) break;
                tc_fence_after();
                const uint32_t a0 = smem_u32(sA + s * A_STAGE_BYTES);
                const uint32_t b0 = smem_u32(sB + s * B_STAGE_BYTES);
                bool ok = true;
                for (int j = 0; j < 2; ++j) {
                    const int kb = 2 * kt + j;
                    if (kb >= nb) break;
                    const int buf = kb % NBUF;
                    const uint32_t use = kb / NBUF;
                    if (!mbar_wait(&sm->acc_empty[buf], (use & 1) ^ 1, abort, err_flag, 3)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem + uint32_t(buf * BN);
#pragma unroll
                    for (int kk = 0; kk < 2; ++kk) {
                        const uint32_t koff = uint32_t(j * 64 + kk * 32);  // bytes inside the 128-byte row
                        mma_f16(d_tmem, sw128_desc(a0 + koff), sw128_desc(b0 + koff), kk);
                    }
                    mma_commit(&sm->acc_full[buf]);
                }
                if (!ok) break;
                mma_commit(&sm->empty[s]);
            }
        }
    } else {
        const int q = warp & 3;               // TMEM lane quarter of this warp
        const int h = (warp - 2) >> 2;        // column half
        const int row = m0 + q * 32 + lane;   // < m_pad
        const int col0 = n0 + h * 64;
        float2 acc[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) acc[c] = make_float2(0.f, 0.f);
        for (int kb = 0; kb < nb; ++kb) {
            const int buf = kb % NBUF;
            const uint32_t use = kb / NBUF;
            const int c = kb % SC_SLOTS;
            const uint32_t cu = kb / SC_SLOTS;
            const bool got = mbar_wait(&sm->sc_full[c], cu & 1, abort, err_flag, 6) &&
                             mbar_wait(&sm->acc_full[buf], use & 1, abort, err_flag, 4);
            if (!__all_sync(0xffffffffu, got)) break;  // keep the warp converged for tcgen05.ld
            tc_fence_after();
            uint32_t r[64];
            const uint32_t taddr = tmem + (uint32_t(q * 32) << 16) + uint32_t(buf * BN + h * 64);
            tmem_ld32(taddr, r);
            tmem_ld32(taddr + 32, r + 32);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm->acc_empty[buf]);

            const float* slot = sc_ring + c * SC_FLOATS;
            const float da = slot[q * 32 + lane];
            const float2 da2 = make_float2(da, da);
            const float4* db4 = reinterpret_cast<const float4*>(slot + 128 + h * 64);
            const float ua = HAS_MIN ? slot[256 + q * 32 + lane] : 0.f;
            const float4* mb4 = reinterpret_cast<const float4*>(slot + 384 + h * 64);
            const float2 ua2 = make_float2(ua, ua);
#pragma unroll
            for (int c4 = 0; c4 < 16; ++c4) {
                const float4 db = db4[c4];
                const uint32_t* rr = &r[c4 * 4];
                const float2 s01 = __fmul2_rn(da2, make_float2(db.x, db.y));
                const float2 s23 = __fmul2_rn(da2, make_float2(db.z, db.w));
                acc[2 * c4] = __ffma2_rn(s01, make_float2(__uint_as_float(rr[0]), __uint_as_float(rr[1])), acc[2 * c4]);
                acc[2 * c4 + 1] =
                    __ffma2_rn(s23, make_float2(__uint_as_float(rr[2]), __uint_as_float(rr[3])), acc[2 * c4 + 1]);
                if (HAS_MIN) {
                    const float4 mb = mb4[c4];
                    acc[2 * c4] = __ffma2_rn(ua2, make_float2(mb.x, mb.y), acc[2 * c4]);
                    acc[2 * c4 + 1] = __ffma2_rn(ua2, make_float2(mb.z, mb.w), acc[2 * c4 + 1]);
                }
                if (DUMP && row < M) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int col = col0 + c4 * 4 + e;
                        if (col < N) S_dump[(size_t(row) * N + col) * nb + kb] = int(__uint_as_float(rr[e]));
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm->sc_empty[c]);
        }
        if (row < M && !*abort) {
            float* yr = Y + size_t(row) * N;
            const bool vec = (N % 4 == 0) && (col0 + 64 <= N) && (reinterpret_cast<uintptr_t>(Y) & 15) == 0 &&
                             (reinterpret_cast<uintptr_t>(bias) & 15) == 0;
            if (vec) {
#pragma unroll
                for (int c4 = 0; c4 < 16; ++c4) {
                    float4 v = make_float4(acc[2 * c4].x, acc[2 * c4].y, acc[2 * c4 + 1].x, acc[2 * c4 + 1].y);
                    if (bias) {
                        const float4 b = __ldg(reinterpret_cast<const float4*>(bias + col0) + c4);
                        v.x = __fadd_rn(v.x, b.x); v.y = __fadd_rn(v.y, b.y);
                        v.z = __fadd_rn(v.z, b.z); v.w = __fadd_rn(v.w, b.w);
                    }
                    *reinterpret_cast<float4*>(yr + col0 + 4 * c4) = v;
                }
            } else {
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const int col = col0 + 2 * c;
                    if (col < N) yr[col] = bias ? __fadd_rn(acc[c].x, __ldg(bias + col)) : acc[c].x;
                    if (col + 1 < N) yr[col + 1] = bias ? __fadd_rn(acc[c].y, __ldg(bias + col + 1)) : acc[c].y;
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
std::once_flag g_encode_once;

bool get_encode(char* why, size_t why_len) {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!g_encode) snprintf(why, why_len, "cuTensorMapEncodeTiled entry point unavailable");
    return g_encode != nullptr;
}

// 2-D f16 tensor [rows][k] (k contiguous), box 64 x 128, 128-byte swizzle.
bool make_map(CUtensorMap* map, const void* ptr, int rows, int k, char* why, size_t why_len) {
    cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(rows)};
    cuuint64_t strides[1] = {cuuint64_t(k) * 2};
    cuuint32_t box[2] = {BK, 128};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        snprintf(why, why_len, "cuTensorMapEncodeTiled failed (%d) rows=%d k=%d", int(r), rows, k);
        return false;
    }
    return true;
}

template <bool HAS_MIN, bool DUMP>
cudaError_t launch_variant(const CUtensorMap& a, const CUtensorMap& b, const ActsView& v, const Weight& w,
                           const float* bias, float* y, int32_t* S_dump, int* err_flag, cudaStream_t s) {
    auto kern = k_gemm_tc<HAS_MIN, DUMP>;
    static int attr_dev_mask = 0;  // one bit per device that has the smem attribute set
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_dev_mask & (1 << dev))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e != cudaSuccess) return e;
        attr_dev_mask |= 1 << dev;
    }
    dim3 grid((w.n + BN - 1) / BN, (v.m + BM - 1) / BM);
    kern<<<grid, THREADS, SMEM_BYTES, s>>>(a, b, v.dT, v.uT, w.dT, w.mT, bias, y, v.m, w.n, w.nb, v.m_pad, w.n_pad,
                                           S_dump, err_flag);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm_tc(const ActsView& v, const Weight& w, const float* bias, float* y, int32_t* S_dump,
                           int* err_flag, cudaStream_t s, char* why, size_t why_len) {
    if (!get_encode(why, why_len)) return cudaErrorNotSupported;
    if (v.m <= 0 || w.n <= 0) return cudaSuccess;
    CUtensorMap ma, mb;
    if (!make_map(&ma, v.q16, v.m, v.k, why, why_len)) return cudaErrorInvalidValue;
    if (!make_map(&mb, w.q16, w.n, w.k, why, why_len)) return cudaErrorInvalidValue;
    const bool mn = has_min(w.dtype);
    if (S_dump) {
        return mn ? launch_variant<true, true>(ma, mb, v, w, bias, y, S_dump, err_flag, s)
                  : launch_variant<false, true>(ma, mb, v, w, bias, y, S_dump, err_flag, s);
    }
    return mn ? launch_variant<true, false>(ma, mb, v, w, bias, y, nullptr, err_flag, s)
              : launch_variant<false, false>(ma, mb, v, w, bias, y, nullptr, err_flag, s);
}

}  // namespace rwq
