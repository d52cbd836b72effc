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
// Roles (352 threads, one CTA per 128 x 128 output tile):
//   warp 0     TMA producer: per pair of blocks one stage with A (q_a
//              f16, 128 x 64) and B (two 128-row hi|lo tiles), 128-byte
//              swizzled, plus 1-D bulk copies of the pair's d_a rows into a
//              shared ring; allocates / frees the 512 TMEM columns.
//   warps 1-2  MMA issuers (one thread each; even / odd pairs): 8 MMAs per
//              pair into a pair of TMEM buffers, then one commit to the
//              pair's accumulator barrier and one to the stage's empty
//              barrier.
//   warps 3-10 epilogue: warp w reads TMEM lanes 32*(w%4).., columns
//              (w-3)/4 * 64 .. + 64 of each block; at the end it
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
constexpr int BN = 128;
// The MMA-issuing thread is the critical resource: the tensor pipe only
// queues about one MMA ahead, so every barrier wait or commit between
// MMAs idles it.  Work is therefore handled in pairs of 32-wide blocks:
// one stage (A: 128 rows x 64 f16, B: two 128-row hi|lo tiles) per pair,
// one full/empty barrier per stage, and TMEM buffers used in pairs, so an
// iteration is 2 waits + 8 MMAs + 2 commits.
constexpr int STAGES = 4;                  // 8 blocks in flight
constexpr int EPI_WARPS = 8;
constexpr int EPI0 = 3;                    // first epilogue warp (warps 1, 2 issue MMAs)
constexpr int THREADS = (EPI0 + EPI_WARPS) * 32;
constexpr int A_BYTES = BM * 64 * 2;       // 16 KiB
constexpr int B_BYTES = BN * 64 * 2;       // 16 KiB per block (32 hi + 32 lo f16 per row)
constexpr int STAGE_BYTES = A_BYTES + 2 * B_BYTES;
constexpr int SC_SLOTS = 8;                // d_a rows for a pair of blocks: 2 x 128 floats
constexpr int NPAIR = 2;                   // TMEM: 2 pairs x 2 blocks x 128 columns = 512
constexpr int TMEM_COLS = 512;
constexpr int CPW = BN / 2;                // output columns per epilogue warp
// kind::f16, D f32, A/B f16, K-major, N>>3 at bit 17, M>>4 at bit 24.
constexpr uint32_t IDESC = (1u << 4) | (uint32_t(BN >> 3) << 17) | (uint32_t(BM >> 4) << 24);

struct Bars {
    uint64_t full[STAGES], empty[STAGES], acc_full[NPAIR], acc_empty[NPAIR], sc_full[SC_SLOTS], sc_empty[SC_SLOTS];
    uint32_t tmem_base;
    int abort;
};
constexpr int SMEM = STAGES * STAGE_BYTES + SC_SLOTS * 1024 + int(sizeof(Bars)) + 1024;
static_assert(SMEM <= 227 * 1024, "shared memory budget");
static_assert(EPI_WARPS * 32 * CPW * 4 <= STAGES * STAGE_BYTES, "output staging must fit in the stages");

__global__ void __launch_bounds__(THREADS, 1)
    k_gemm_fold(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmY, int use_tma_store, const float* __restrict__ daT,
                const float* __restrict__ colscale, const float* __restrict__ bias, float* __restrict__ Y, int M,
                int N, int nb, int m_pad, int* __restrict__ err_flag) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    float* ring = reinterpret_cast<float*>(base + STAGES * STAGE_BYTES);
    Bars* bar = reinterpret_cast<Bars*>(reinterpret_cast<uint8_t*>(ring) + SC_SLOTS * 1024);
    volatile int* abort = &bar->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int npairs = (nb + 1) / 2;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&bar->full[s], 1);
            mbar_init(&bar->empty[s], 1);
        }
        for (int b = 0; b < NPAIR; ++b) {
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
    if (threadIdx.x == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bar->tmem_base;
    // Setup above overlaps the previous kernel; global memory only below.
    pdl_trigger();
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            for (int pr = 0; pr < npairs; ++pr) {
                const int s = pr % STAGES;
                if (!mbar_wait(&bar->empty[s], ((pr / STAGES) & 1) ^ 1, abort, err_flag, 1)) break;
                uint8_t* st = base + s * STAGE_BYTES;
                mbar_expect_tx(&bar->full[s], STAGE_BYTES);
                tma_load_2d(st, &tmA, pr * 64, m0, &bar->full[s]);                        // blocks 2pr, 2pr+1
                tma_load_2d(st + A_BYTES, &tmB, pr * 128, n0, &bar->full[s]);             // block 2pr
                tma_load_2d(st + A_BYTES + B_BYTES, &tmB, pr * 128 + 64, n0, &bar->full[s]);  // block 2pr+1
                const int c = pr % SC_SLOTS;
                if (!mbar_wait(&bar->sc_empty[c], ((pr / SC_SLOTS) & 1) ^ 1, abort, err_flag, 5)) break;
                const int two = (2 * pr + 1 < nb) ? 2 : 1;
                mbar_expect_tx(&bar->sc_full[c], 512u * two);
                for (int j = 0; j < two; ++j)
                    bulk_load(ring + c * 256 + j * 128, daT + size_t(2 * pr + j) * m_pad + m0, 512, &bar->sc_full[c]);
            }
        }
    } else if (warp == 1 || warp == 2) {
        // Two issuing threads: warp 1 takes the even pairs (TMEM pair 0),
        // warp 2 the odd ones (pair 1).  Each commit tracks the issuing
        // thread's own MMAs, and the two accumulators are independent, so
        // one thread's MMAs keep the tensor pipe busy while the other waits
        // on its barriers or commits.
        if (lane == 0) {
            for (int pr = warp - 1; pr < npairs; pr += 2) {
                const int s = pr % STAGES, p = pr % NPAIR;
                if (!mbar_wait(&bar->full[s], (pr / STAGES) & 1, abort, err_flag, 2)) break;
                if (!mbar_wait(&bar->acc_empty[p], ((pr / NPAIR) & 1) ^ 1, abort, err_flag, 3)) break;
                tc_fence_after();
                const uint32_t a0 = smem_u32(base + s * STAGE_BYTES);
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    if (2 * pr + j >= nb) break;
                    const uint32_t a = a0 + uint32_t(j * 64);
                    const uint32_t b = a0 + uint32_t(A_BYTES + j * B_BYTES);
                    const uint32_t d = tmem + uint32_t(p * 2 * BN + j * BN);
                    // K half 0: A bytes +0..31, B hi +0..31, lo +64..95;
                    // K half 1: A bytes +32..63, B hi +32..63, lo +96..127.
                    mma_f16_id(d, sw128_desc(a), sw128_desc(b), IDESC, 0);
                    mma_f16_id(d, sw128_desc(a), sw128_desc(b + 64), IDESC, 1);
                    mma_f16_id(d, sw128_desc(a + 32), sw128_desc(b + 32), IDESC, 1);
                    mma_f16_id(d, sw128_desc(a + 32), sw128_desc(b + 96), IDESC, 1);
                }
                mma_commit(&bar->acc_full[p]);
                mma_commit(&bar->empty[s]);
            }
        }
    } else {
        const int q = warp & 3;
        const int h = (warp - EPI0) >> 2;
        float2 acc[CPW / 2];
#pragma unroll
        for (int c = 0; c < CPW / 2; ++c) acc[c] = make_float2(0.f, 0.f);
        for (int pr = 0; pr < npairs; ++pr) {
            const int p = pr % NPAIR, c = pr % SC_SLOTS;
            const bool got = mbar_wait(&bar->sc_full[c], (pr / SC_SLOTS) & 1, abort, err_flag, 6) &&
                             mbar_wait(&bar->acc_full[p], (pr / NPAIR) & 1, abort, err_flag, 4);
            if (!__all_sync(0xffffffffu, got)) break;
            tc_fence_after();
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                if (2 * pr + j >= nb) break;
                const float da = ring[c * 256 + j * 128 + q * 32 + lane];
                const float2 da2 = make_float2(da, da);
                const uint32_t taddr = tmem + (uint32_t(q * 32) << 16) + uint32_t(p * 2 * BN + j * BN + h * CPW);
                uint32_t r[64];
                tmem_ld32(taddr, r);
                tmem_ld32(taddr + 32, r + 32);
                tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    acc[i] = __ffma2_rn(da2, make_float2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])),
                                        acc[i]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bar->acc_empty[p]);
                mbar_arrive(&bar->sc_empty[c]);
            }
        }
        // y = acc * 2^-e_j (+ bias), written through shared memory.
        const int col0 = n0 + h * CPW;
        const int row = m0 + q * 32 + lane;
        const bool bias_vec = (reinterpret_cast<uintptr_t>(bias) & 15) == 0;
        if (!*abort) {
            if (use_tma_store) {
                // Staging for this warp (in the drained stage ring): CPW/32
                // boxes of 32 rows x 128 bytes, 128-byte swizzle (16-byte
                // chunk c of row r at c ^ (r & 7)).
                uint8_t* stg = base + (warp - EPI0) * (32 * CPW * 4);
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

cudaError_t launch_fold(const ActsView& v, const Weight& w, const float* bias, float* y, int* err_flag,
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
    static int attr_dev_mask = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_dev_mask & (1 << dev))) {
        cudaError_t e = cudaFuncSetAttribute(k_gemm_fold, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
        if (e != cudaSuccess) return e;
        attr_dev_mask |= 1 << dev;
    }
    dim3 grid((w.n + BN - 1) / BN, (v.m + BM - 1) / BM);
    return launch_pdl(k_gemm_fold, grid, dim3(THREADS), SMEM, s, ma, mb, my, use_tma_store, v.dT, w.colscale, bias, y,
                      v.m, w.n, w.nb, v.m_pad, err_flag);
}

}  // namespace

cudaError_t launch_gemm_fold(const ActsView& v, const Weight& w, const float* bias, float* y, int* err_flag,
                             cudaStream_t s, char* why, size_t why_len) {
    if (v.m <= 0 || w.n <= 0) return cudaSuccess;
    return launch_fold(v, w, bias, y, err_flag, s, why, why_len);
}

}  // namespace rwq
