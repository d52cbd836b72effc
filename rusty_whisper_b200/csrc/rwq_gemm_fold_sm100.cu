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
//              swizzled; per 16 blocks one 2-D load of their d_a rows
//              (16 x 128 floats) into a 3-slot ring; allocates / frees the
//              512 TMEM columns.
//   warps 1-2  MMA issuers (one thread each; even / odd pairs): per block
//              4 MMAs into one of four 128-column TMEM buffers and a commit
//              to that buffer's barrier, then a commit to the stage's empty
//              barrier.
//   warps 3-10 epilogue: warp w reads TMEM lanes 32*(w%4).., columns
//              (w-3)/4 * 64 .. + 64 of each block; at the end it
//              scales, adds the bias, stages its 32-row block in shared
//              memory (the drained B ring) and writes it with TMA stores,
//              which clip the ragged M and N edges.
// Every wait is bounded (see rwq_sm100.cuh).
#include <cuda.h>
#include <cuda_fp16.h>
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
// The MMA-issuing thread is the critical resource: the tensor pipe only
// queues about one MMA ahead, so every barrier wait or commit between
// MMAs idles it.  Work is therefore handled in pairs of 32-wide blocks:
// one stage (A: 128 rows x 64 f16, B: two BN-row hi|lo tiles) per pair and
// one full/empty barrier per stage.
//
// Tile width BN is 128 or 64.  At 128 the MMAs are most efficient; 64 is
// used when 128-wide tiles would leave half the SMs idle (the N = 768
// encoder shapes at M = 1500 give 72 tiles for 148 SMs): its MMAs are a
// third less efficient per flop, but twice the SMs run, and each block's
// accumulator is half as many TMEM bytes for the epilogue to read.
constexpr int EPI_WARPS = 8;
constexpr int EPI0 = 3;                    // first epilogue warp (warps 1, 2 issue MMAs)
constexpr int THREADS = (EPI0 + EPI_WARPS) * 32;
constexpr int A_BYTES = BM * 64 * 2;       // 16 KiB
// d_a arrives 16 blocks at a time (one 8 KiB TMA load instead of 16
// small copies: each copy is a TMA operation, and at two per block pair
// they slowed the operand stream by a seventh).
constexpr int DA_GROUP = 16;
constexpr int DA_SLOTS = 3;
constexpr int DA_BYTES = DA_GROUP * BM * 4;
constexpr int TMEM_COLS = 512;

template <int BN>
struct Fold {
    static constexpr int B_BYTES = BN * 64 * 2;   // per block: BN rows x (32 hi + 32 lo f16)
    static constexpr int STAGE_BYTES = A_BYTES + 2 * B_BYTES;
    static constexpr int STAGES = BN == 128 ? 4 : 6;   // 192 KiB of stages either way
    // TMEM: single-block accumulators of BN columns.  A block's buffer is
    // handed back as soon as the epilogue has read it, so the MMAs can run
    // up to NBUF - 1 blocks ahead of the epilogue.
    static constexpr int NBUF = TMEM_COLS / BN;
    static constexpr int CPW = BN / 2;            // output columns per epilogue warp
    // kind::f16, D f32, A/B f16, K-major, N>>3 at bit 17, M>>4 at bit 24.
    static constexpr uint32_t IDESC = (1u << 4) | (uint32_t(BN >> 3) << 17) | (uint32_t(BM >> 4) << 24);
    struct Bars {
        alignas(16) float cs[BN];   // the tile's column scales and bias, read once early
        alignas(16) float bs[BN];
        uint64_t full[STAGES], empty[STAGES], acc_full[NBUF], acc_empty[NBUF], da_full[DA_SLOTS], da_empty[DA_SLOTS];
        uint32_t tmem_base;
        int abort;
    };
    static constexpr int SMEM = STAGES * STAGE_BYTES + DA_SLOTS * DA_BYTES + int(sizeof(Bars)) + 1024;
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
    static_assert(EPI_WARPS * 32 * CPW * 4 <= STAGES * STAGE_BYTES, "output staging must fit in the stages");
};

template <int BN>
__global__ void __launch_bounds__(THREADS, 1)
    k_gemm_fold(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmD, int use_tma_store,
                const float* __restrict__ colscale, const float* __restrict__ bias, float* __restrict__ Y, int M,
                int N, int nb, int* __restrict__ err_flag) {
    using F = Fold<BN>;
    constexpr int STAGES = F::STAGES, STAGE_BYTES = F::STAGE_BYTES, B_BYTES = F::B_BYTES, NBUF = F::NBUF;
    constexpr int CPW = F::CPW;
    constexpr uint32_t IDESC = F::IDESC;
    using Bars = typename F::Bars;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    float* ring = reinterpret_cast<float*>(base + STAGES * STAGE_BYTES);
    Bars* bar = reinterpret_cast<Bars*>(reinterpret_cast<uint8_t*>(ring) + DA_SLOTS * DA_BYTES);
    volatile int* abort = &bar->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int npairs = (nb + 1) / 2;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&bar->full[s], 1);
            mbar_init(&bar->empty[s], 1);
        }
        for (int b = 0; b < NBUF; ++b) {
            mbar_init(&bar->acc_full[b], 1);
            mbar_init(&bar->acc_empty[b], EPI_WARPS);
        }
        for (int c = 0; c < DA_SLOTS; ++c) {
            mbar_init(&bar->da_full[c], 1);
            mbar_init(&bar->da_empty[c], EPI_WARPS);
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
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmD)) : "memory");
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
                if ((2 * pr) % DA_GROUP == 0) {
                    // d_a rows of blocks 2pr .. 2pr+15 (rows past nb read as 0).
                    const int g = 2 * pr / DA_GROUP, c = g % DA_SLOTS;
                    if (!mbar_wait(&bar->da_empty[c], ((g / DA_SLOTS) & 1) ^ 1, abort, err_flag, 5)) break;
                    mbar_expect_tx(&bar->da_full[c], DA_BYTES);
                    tma_load_2d(ring + c * (DA_BYTES / 4), &tmD, m0, g * DA_GROUP, &bar->da_full[c]);
                }
                if (!mbar_wait(&bar->empty[s], ((pr / STAGES) & 1) ^ 1, abort, err_flag, 1)) break;
                uint8_t* st = base + s * STAGE_BYTES;
                mbar_expect_tx(&bar->full[s], STAGE_BYTES);
                tma_load_2d(st, &tmA, pr * 64, m0, &bar->full[s]);                        // blocks 2pr, 2pr+1
                tma_load_2d(st + A_BYTES, &tmB, pr * 128, n0, &bar->full[s]);             // block 2pr
                tma_load_2d(st + A_BYTES + B_BYTES, &tmB, pr * 128 + 64, n0, &bar->full[s]);  // block 2pr+1
            }
        }
    } else if (warp == 1 || warp == 2) {
        // Two issuing threads: warp 1 takes the even pairs (TMEM buffers 0
        // and 1), warp 2 the odd ones (buffers 2 and 3).  Each commit tracks
        // the issuing thread's own MMAs and the buffers are independent, so
        // one thread's MMAs keep the tensor pipe busy while the other waits
        // on its barriers or commits.
        if (lane == 0) {
            bool ok = true;
            for (int pr = warp - 1; pr < npairs && ok; pr += 2) {
                const int s = pr % STAGES;
                if (!mbar_wait(&bar->full[s], (pr / STAGES) & 1, abort, err_flag, 2)) break;
                const uint32_t a0 = smem_u32(base + s * STAGE_BYTES);
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int blk = 2 * pr + j;
                    if (blk >= nb) break;
                    const int u = blk % NBUF;
                    if (!mbar_wait(&bar->acc_empty[u], ((blk / NBUF) & 1) ^ 1, abort, err_flag, 3)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a = a0 + uint32_t(j * 64);
                    const uint32_t b = a0 + uint32_t(A_BYTES + j * B_BYTES);
                    const uint32_t d = tmem + uint32_t(u * BN);
                    // K half 0: A bytes +0..31, B hi +0..31, lo +64..95;
                    // K half 1: A bytes +32..63, B hi +32..63, lo +96..127.
                    mma_f16_id(d, sw128_desc(a), sw128_desc(b), IDESC, 0);
                    mma_f16_id(d, sw128_desc(a), sw128_desc(b + 64), IDESC, 1);
                    mma_f16_id(d, sw128_desc(a + 32), sw128_desc(b + 32), IDESC, 1);
                    mma_f16_id(d, sw128_desc(a + 32), sw128_desc(b + 96), IDESC, 1);
                    mma_commit(&bar->acc_full[u]);
                }
                mma_commit(&bar->empty[s]);
            }
        }
    } else {
        const int q = warp & 3;
        const int h = (warp - EPI0) >> 2;
        float2 acc[CPW / 2];
#pragma unroll
        for (int c = 0; c < CPW / 2; ++c) acc[c] = make_float2(0.f, 0.f);
        // The tile's column scales and bias into shared memory now, so the
        // final scaling does not wait on their loads.
        for (int c = int(threadIdx.x) - EPI0 * 32; c < BN; c += EPI_WARPS * 32) {
            bar->cs[c] = __ldg(colscale + n0 + c);   // padded width
            bar->bs[c] = bias && n0 + c < N ? __ldg(bias + n0 + c) : 0.f;
        }
        for (int blk = 0; blk < nb; ++blk) {
            const int u = blk % NBUF, g = blk / DA_GROUP, c = g % DA_SLOTS;
            const bool got = (blk % DA_GROUP != 0 || mbar_wait(&bar->da_full[c], (g / DA_SLOTS) & 1, abort, err_flag, 6)) &&
                             mbar_wait(&bar->acc_full[u], (blk / NBUF) & 1, abort, err_flag, 4);
            if (!__all_sync(0xffffffffu, got)) break;
            tc_fence_after();
            const float da = ring[c * (DA_BYTES / 4) + (blk % DA_GROUP) * BM + q * 32 + lane];
            const float2 da2 = make_float2(da, da);
            const uint32_t taddr = tmem + (uint32_t(q * 32) << 16) + uint32_t(u * BN + h * CPW);
            uint32_t r[CPW];
            tmem_ld32(taddr, r);
            if constexpr (CPW == 64) tmem_ld32(taddr + 32, r + 32);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bar->acc_empty[u]);
                if (blk % DA_GROUP == DA_GROUP - 1 || blk == nb - 1) mbar_arrive(&bar->da_empty[c]);
            }
#pragma unroll
            for (int i = 0; i < CPW / 2; ++i)
                acc[i] = __ffma2_rn(da2, make_float2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1])), acc[i]);
        }
        // y = acc * 2^-e_j (+ bias), written through shared memory.
        const int col0 = n0 + h * CPW;
        const int row = m0 + q * 32 + lane;
        asm volatile("bar.sync 1, %0;" ::"r"(EPI_WARPS * 32) : "memory");   // scales and bias in place
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
                        const float4 cs = *reinterpret_cast<const float4*>(bar->cs + (col - n0));
                        const float2 a01 = acc[b * 16 + c4 * 2], a23 = acc[b * 16 + c4 * 2 + 1];
                        float4 v = make_float4(__fmul_rn(a01.x, cs.x), __fmul_rn(a01.y, cs.y),
                                               __fmul_rn(a23.x, cs.z), __fmul_rn(a23.y, cs.w));
                        if (bias && col < N) {  // N % 4 == 0 on this path
                            const float4 bb = *reinterpret_cast<const float4*>(bar->bs + (col - n0));
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

// ------------------------------------------------------------- wide tiles
// k_gemm_fold_w: the same arithmetic on 128 x 256 output tiles.
//
// Measured on the 128 x 128 kernel above: a block takes ~0.35 us against
// 0.14 us of MMA, and neither the operand stream (3 and 4 stages run
// alike), nor the tensor-memory read rate (16 epilogue warps run like 8)
// sets that.  What a wider tile changes: an N = 256 MMA reads its A and B
// operands from shared memory at 96 B/clock instead of the 128 B/clock
// (the whole shared-memory read rate) of an N = 128 one, so the
// epilogue's tensor-memory loads and the TMA writes no longer contend
// with the MMAs for it; each A tile feeds twice the columns; and a
// whisper-small N = 3072 GEMM at M = 1500 is 144 tiles, one wave, where
// 128-wide tiles needed two.
//
// Roles (608 threads): warp 0 the TMA producer (one 40 KiB stage per
// block: A 128 x 32 f16 with the 64-byte swizzle, B 256 rows x 64 f16 hi|lo
// with the 128-byte swizzle; d_a 16 blocks at a time); warps 1-2 issue the
// MMAs of even / odd blocks (four N = 256 MMAs per block into one of two
// 256-column TMEM buffers); warps 3-18 the epilogue, four warps per TMEM
// lane quarter, each 64 columns (acc <- fma(d_a, T, acc) in registers,
// 16 columns per tensor-memory load).
//
// A K split over a cluster of CTAs (partial tiles added through distributed
// shared memory) was measured and dropped: moving a 128 x 256 f32 partial
// between CTAs ran at ~25-30 GB/s per SM, by per-thread remote stores and
// by bulk shared::cluster copies alike, so the reduction cost more than the
// split saved on the N = 768 shapes, which stay on the 64-column kernel.
namespace wide {
constexpr int BN = 256;
constexpr int EW = 16;                                   // epilogue warps
constexpr int THREADS = (EPI0 + EW) * 32;                // 608
constexpr int CPW = BN / 4;                              // columns per epilogue warp
constexpr int A_BYTES = BM * 32 * 2;                     // 8 KiB, 64-byte rows
constexpr int B_BYTES = BN * 64 * 2;                     // 32 KiB, 128-byte rows
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;           // 40 KiB
constexpr int STAGES = 5;
constexpr int NBUF = 2;                                  // 2 x 256 TMEM columns
constexpr int DA_SLOTS = 2;
constexpr uint32_t IDESC = (1u << 4) | (uint32_t(BN >> 3) << 17) | (uint32_t(BM >> 4) << 24);
struct Bars {
    alignas(16) float cs[BN];   // the tile's column scales and bias, read once early
    alignas(16) float bs[BN];
    uint64_t full[STAGES], empty[STAGES], acc_full[NBUF], acc_empty[NBUF], da_full[DA_SLOTS], da_empty[DA_SLOTS];
    uint32_t tmem_base;
    int abort;
};
constexpr int SMEM = STAGES * STAGE_BYTES + DA_SLOTS * DA_BYTES + int(sizeof(Bars)) + 1024;
static_assert(SMEM <= 227 * 1024, "shared memory budget");
static_assert(EW * 32 * CPW * 4 <= STAGES * STAGE_BYTES, "output staging must fit in the stages");
static_assert(STAGE_BYTES % 1024 == 0, "stages keep the 1024-byte swizzle alignment");
}  // namespace wide

// Shared-memory matrix descriptor: K-major, 64-byte swizzle (8-row groups
// 512 bytes apart), layout type 4 = SWIZZLE_64B.
__device__ __forceinline__ uint64_t sw64_desc(uint32_t saddr) {
    uint64_t d = uint64_t((saddr & 0x3FFFFu) >> 4);
    d |= uint64_t(16 >> 4) << 16;
    d |= uint64_t(512 >> 4) << 32;
    d |= uint64_t(1) << 46;
    d |= uint64_t(4) << 61;
    return d;
}

// tcgen05.wait::ld with the 16 loaded registers as operands, so no use of
// them can be scheduled before the wait.
__device__ __forceinline__ void tmem_wait_ld16(uint32_t* r) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15])
                 :
                 : "memory");
}

__global__ void __launch_bounds__(wide::THREADS, 1)
    k_gemm_fold_w(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmD, int use_tma_store,
                  const float* __restrict__ colscale, const float* __restrict__ bias, float* __restrict__ Y, int M,
                  int N, int nb, int* __restrict__ err_flag, const __grid_constant__ CUtensorMap tmQ,
                  float* __restrict__ qdT, float* __restrict__ quT, int q_m_pad, __half* __restrict__ hdst,
                  int hT, int hH, float hscale) {
    constexpr int BN = wide::BN, EW = wide::EW, CPW = wide::CPW;
    constexpr int A_BYTES = wide::A_BYTES, STAGE_BYTES = wide::STAGE_BYTES, STAGES = wide::STAGES;
    constexpr int NBUF = wide::NBUF, DA_SLOTS = wide::DA_SLOTS;
    constexpr uint32_t IDESC = wide::IDESC;
    using Bars = wide::Bars;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    float* ring = reinterpret_cast<float*>(base + STAGES * STAGE_BYTES);
    Bars* bar = reinterpret_cast<Bars*>(reinterpret_cast<uint8_t*>(ring) + DA_SLOTS * DA_BYTES);
    volatile int* abort = &bar->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = int(blockIdx.x) * BN, m0 = int(blockIdx.y) * BM;
    const int nblk = nb;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&bar->full[s], 1);
            mbar_init(&bar->empty[s], 1);
        }
        for (int b = 0; b < NBUF; ++b) {
            mbar_init(&bar->acc_full[b], 1);
            mbar_init(&bar->acc_empty[b], EW);
        }
        for (int c = 0; c < DA_SLOTS; ++c) {
            mbar_init(&bar->da_full[c], 1);
            mbar_init(&bar->da_empty[c], EW);
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
    if (threadIdx.x == 32) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmD)) : "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bar->tmem_base;
    // Set-up above overlaps the previous kernel; global memory only below.
    pdl_trigger();
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            for (int i = 0; i < nblk; ++i) {
                const int s = i % STAGES;
                if (i % DA_GROUP == 0) {
                    // d_a rows of blocks i .. i+15 (rows past nb read as 0).
                    const int g = i / DA_GROUP, c = g % DA_SLOTS;
                    if (!mbar_wait(&bar->da_empty[c], ((g / DA_SLOTS) & 1) ^ 1, abort, err_flag, 5)) break;
                    mbar_expect_tx(&bar->da_full[c], DA_BYTES);
                    tma_load_2d(ring + c * (DA_BYTES / 4), &tmD, m0, i, &bar->da_full[c]);
                }
                if (!mbar_wait(&bar->empty[s], ((i / STAGES) & 1) ^ 1, abort, err_flag, 1)) break;
                uint8_t* st = base + s * STAGE_BYTES;
                mbar_expect_tx(&bar->full[s], STAGE_BYTES);
                tma_load_2d(st, &tmA, i * 32, m0, &bar->full[s]);
                tma_load_2d(st + A_BYTES, &tmB, i * 64, n0, &bar->full[s]);
            }
        }
    } else if (warp == 1 || warp == 2) {
        // Warp 1 issues the even blocks (TMEM buffer 0), warp 2 the odd ones
        // (buffer 1); each commit tracks the issuing thread's own MMAs.
        if (lane == 0) {
            const int u = warp - 1;
            const uint32_t d = tmem + uint32_t(u * BN);
            for (int i = u; i < nblk; i += 2) {
                const int s = i % STAGES;
                if (!mbar_spin(&bar->full[s], (i / STAGES) & 1, abort, err_flag, 2)) break;
                if (!mbar_spin(&bar->acc_empty[u], ((i / NBUF) & 1) ^ 1, abort, err_flag, 3)) break;
                tc_fence_after();
                const uint32_t a = smem_u32(base + s * STAGE_BYTES);
                const uint32_t b = a + uint32_t(A_BYTES);
                // K half 0: A bytes +0..31, B hi +0..31, lo +64..95;
                // K half 1: A bytes +32..63, B hi +32..63, lo +96..127.
                mma_f16_id(d, sw64_desc(a), sw128_desc(b), IDESC, 0);
                mma_f16_id(d, sw64_desc(a), sw128_desc(b + 64), IDESC, 1);
                mma_f16_id(d, sw64_desc(a + 32), sw128_desc(b + 32), IDESC, 1);
                mma_f16_id(d, sw64_desc(a + 32), sw128_desc(b + 96), IDESC, 1);
                mma_commit(&bar->acc_full[u]);
                mma_commit(&bar->empty[s]);
            }
        }
    } else {
        const int q = warp & 3, h = (warp - EPI0) >> 2;   // TMEM lane quarter, column quarter
        float2 acc[CPW / 2];
#pragma unroll
        for (int c = 0; c < CPW / 2; ++c) acc[c] = make_float2(0.f, 0.f);
        // The tile's column scales and bias into shared memory now, so the
        // final scaling does not wait on their loads.
        for (int c = int(threadIdx.x) - EPI0 * 32; c < BN; c += EW * 32) {
            bar->cs[c] = __ldg(colscale + n0 + c);   // padded width
            bar->bs[c] = bias && n0 + c < N ? __ldg(bias + n0 + c) : 0.f;
        }
        const uint32_t lane_off = uint32_t(q * 32) << 16;
        for (int i = 0; i < nblk; ++i) {
            const int u = i % NBUF, g = i / DA_GROUP, c = g % DA_SLOTS;
            const bool got = (i % DA_GROUP != 0 || mbar_wait(&bar->da_full[c], (g / DA_SLOTS) & 1, abort, err_flag, 6)) &&
                             mbar_spin(&bar->acc_full[u], (i / NBUF) & 1, abort, err_flag, 4);
            if (!__all_sync(0xffffffffu, got)) break;
            tc_fence_after();
            const float da = ring[c * (DA_BYTES / 4) + (i % DA_GROUP) * BM + q * 32 + lane];
            const float2 da2 = make_float2(da, da);
            const uint32_t taddr = tmem + lane_off + uint32_t(u * BN + h * CPW);
#pragma unroll
            for (int cc = 0; cc < CPW / 16; ++cc) {
                uint32_t r[16];
                tmem_ld16(taddr + uint32_t(cc * 16), r);
                tmem_wait_ld16(r);
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    acc[cc * 8 + e] = __ffma2_rn(da2, make_float2(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1])),
                                                 acc[cc * 8 + e]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bar->acc_empty[u]);
                if (i % DA_GROUP == DA_GROUP - 1 || i == nblk - 1) mbar_arrive(&bar->da_empty[c]);
            }
        }
        const int col0 = n0 + h * CPW;
        const int row = m0 + q * 32 + lane;
        asm volatile("bar.sync 1, %0;" ::"r"(EW * 32) : "memory");   // scales and bias in place
        if (!*abort && q_m_pad > 0) {
            // GELU, then the reference's int8 quantizer per 32-column block,
            // straight into the next GEMM's operand: f16 codes through the
            // staging boxes (tmQ, 64 f16 x 32 rows, 128-byte swizzle), d_a and
            // d_a*sum(q_a) transposed [block][m_pad].  Each thread holds one
            // row's whole blocks, so the values and their order are those of
            // a GEMM writing y and the GELU row kernel quantizing it.
            uint8_t* box = base + (warp - EPI0) * 4096 + lane * 128;
#pragma unroll
            for (int j = 0; j < CPW / 32; ++j) {
                float amax = 0.f;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int col = col0 + j * 32 + 2 * i;   // < n0 + BN <= N on this path
                    float2 v = make_float2(__fmul_rn(acc[j * 16 + i].x, bar->cs[col - n0]),
                                           __fmul_rn(acc[j * 16 + i].y, bar->cs[col - n0 + 1]));
                    if (bias) {
                        v.x = __fadd_rn(v.x, bar->bs[col - n0]);
                        v.y = __fadd_rn(v.y, bar->bs[col - n0 + 1]);
                    }
                    v = make_float2(gelu_ref(v.x), gelu_ref(v.y));
                    acc[j * 16 + i] = v;
                    const float ax = fabsf(v.x), ay = fabsf(v.y);
                    amax = fmaxf(amax, fmaxf(isnan(ax) ? 0.f : ax, isnan(ay) ? 0.f : ay));
                }
                const float d = __fdiv_rn(amax, 127.0f);
                const float inv = d > 0.f ? __fdiv_rn(1.0f, d) : 0.f;
                auto code = [inv](float v) {
                    const float r = roundf(__fmul_rn(v, inv));
                    return isnan(r) ? 0 : int(fminf(127.f, fmaxf(-127.f, r)));
                };
                int sum = 0;
#pragma unroll
                for (int ch = 0; ch < 4; ++ch) {   // 8 codes = one 16-byte chunk of the row
                    uint32_t w[4];
#pragma unroll
                    for (int p2 = 0; p2 < 4; ++p2) {
                        const float2 v = acc[j * 16 + ch * 4 + p2];
                        const int c0 = code(v.x), c1 = code(v.y);
                        sum += c0 + c1;
                        w[p2] = uint32_t(__half_as_ushort(__int2half_rn(c0))) |
                                (uint32_t(__half_as_ushort(__int2half_rn(c1))) << 16);
                    }
                    const int chunk = j * 4 + ch;
                    *reinterpret_cast<uint4*>(box + ((chunk ^ (lane & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
                }
                if (row < q_m_pad) {
                    const size_t bl = size_t((col0 + j * 32) / QK);
                    qdT[bl * q_m_pad + row] = row < M ? d : 0.f;
                    quT[bl * q_m_pad + row] = row < M ? __fmul_rn(d, float(sum)) : 0.f;
                }
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                if (m0 + q * 32 < M) tma_store_2d(&tmQ, col0, m0 + q * 32, base + (warp - EPI0) * 4096);
                bulk_commit();
                bulk_wait_read_all();
            }
            __syncwarp();
        } else if (!*abort && hdst) {
            // Attention heads: f16(y * hscale) of row (window w, frame t) and
            // head c/64 at hdst[((w*H + c/64)*T + t)*64 + c%64] -- a warp's
            // 64 columns are one head.  Rows of one window go out as one
            // 32 x 64 f16 TMA box (tmQ over [W*H*T][64]); a warp whose rows
            // cross a window boundary stores its rows itself.
            uint8_t* box = base + (warp - EPI0) * 4096 + lane * 128;
#pragma unroll
            for (int ch = 0; ch < 8; ++ch) {
                uint32_t wv[4];
#pragma unroll
                for (int p2 = 0; p2 < 4; ++p2) {
                    const int i = ch * 4 + p2, col = col0 + 2 * i;
                    float2 v = make_float2(__fmul_rn(acc[i].x, bar->cs[col - n0]),
                                           __fmul_rn(acc[i].y, bar->cs[col - n0 + 1]));
                    if (bias) {
                        v.x = __fadd_rn(v.x, bar->bs[col - n0]);
                        v.y = __fadd_rn(v.y, bar->bs[col - n0 + 1]);
                    }
                    const __half2 hv = __floats2half2_rn(__fmul_rn(v.x, hscale), __fmul_rn(v.y, hscale));
                    wv[p2] = *reinterpret_cast<const uint32_t*>(&hv);
                }
                *reinterpret_cast<uint4*>(box + ((ch ^ (lane & 7)) << 4)) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
            }
            fence_async_smem();
            __syncwarp();
            const int r0 = m0 + q * 32, hd = col0 / 64;
            const int w0 = r0 / hT, t0 = r0 - w0 * hT;
            if (t0 + 32 <= hT) {
                if (lane == 0) {
                    if (r0 < M) tma_store_2d(&tmQ, 0, (w0 * hH + hd) * hT + t0, base + (warp - EPI0) * 4096);
                    bulk_commit();
                    bulk_wait_read_all();
                }
            } else if (row < M) {
                const int w = row / hT, t = row - w * hT;
                uint4* dst = reinterpret_cast<uint4*>(hdst + ((size_t(w) * hH + hd) * hT + t) * 64);
#pragma unroll
                for (int ch = 0; ch < 8; ++ch) dst[ch] = *reinterpret_cast<const uint4*>(box + ((ch ^ (lane & 7)) << 4));
            }
            __syncwarp();
        } else if (!*abort) {
            if (use_tma_store) {
                // Staging for this warp: CPW/32 boxes of 32 rows x 128 bytes,
                // 128-byte swizzle (16-byte chunk c of row r at c ^ (r & 7)).
                uint8_t* stg = base + (warp - EPI0) * (32 * CPW * 4);
#pragma unroll
                for (int b = 0; b < CPW / 32; ++b) {
                    uint8_t* box = stg + b * 4096 + lane * 128;
#pragma unroll
                    for (int c4 = 0; c4 < 8; ++c4) {
                        const int col = col0 + b * 32 + c4 * 4;   // < n0 + BN <= padded width
                        const float4 cs = *reinterpret_cast<const float4*>(bar->cs + (col - n0));
                        const float2 a01 = acc[b * 16 + c4 * 2], a23 = acc[b * 16 + c4 * 2 + 1];
                        float4 v = make_float4(__fmul_rn(a01.x, cs.x), __fmul_rn(a01.y, cs.y),
                                               __fmul_rn(a23.x, cs.z), __fmul_rn(a23.y, cs.w));
                        if (bias && col < N) {  // N % 4 == 0 on this path
                            const float4 bb = *reinterpret_cast<const float4*>(bar->bs + (col - n0));
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
cudaError_t launch_fold_bn(const ActsView& v, const Weight& w, const float* bias, float* y, int* err_flag,
                        cudaStream_t s, char* why, size_t why_len) {
    CUtensorMap ma, mb, my, md;
    if (!encode_map(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, v.q16, uint64_t(v.k), uint64_t(v.m), 64, BM,
                    CU_TENSOR_MAP_SWIZZLE_128B, why, why_len))
        return cudaErrorInvalidValue;
    if (!encode_map(&mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, w.bhl, uint64_t(w.nb) * 64, uint64_t(w.n), 64, BN,
                    CU_TENSOR_MAP_SWIZZLE_128B, why, why_len))
        return cudaErrorInvalidValue;
    // d_a rows, transposed [nb][m_pad]: a box is 16 blocks x 128 rows.
    if (!encode_map(&md, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, v.dT, uint64_t(v.m_pad), uint64_t(w.nb), BM, DA_GROUP,
                    CU_TENSOR_MAP_SWIZZLE_NONE, why, why_len))
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
        cudaError_t e = cudaFuncSetAttribute(k_gemm_fold<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             Fold<BN>::SMEM);
        if (e != cudaSuccess) return e;
        attr_dev_mask |= 1 << dev;
    }
    dim3 grid((w.n + BN - 1) / BN, (v.m + BM - 1) / BM);
    return launch_pdl(k_gemm_fold<BN>, grid, dim3(THREADS), Fold<BN>::SMEM, s, ma, mb, my, md, use_tma_store, w.colscale, bias, y,
                      v.m, w.n, w.nb, err_flag);
}

std::mutex g_dev_mu;
int g_sms[64];
int g_wide_attr[64];

int cur_dev() {
    int dev = 0;
    cudaGetDevice(&dev);
    return dev < 64 ? dev : 63;
}

int sms_of(int dev) {
    std::lock_guard<std::mutex> g(g_dev_mu);
    if (g_sms[dev] == 0 && cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        g_sms[dev] = 148;
    return g_sms[dev];
}

cudaError_t wide_smem_attr(int dev) {
    std::lock_guard<std::mutex> g(g_dev_mu);
    if (g_wide_attr[dev]) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(k_gemm_fold_w, cudaFuncAttributeMaxDynamicSharedMemorySize, wide::SMEM);
    if (e == cudaSuccess) g_wide_attr[dev] = 1;
    return e;
}

// Tile width.  Per-CTA time is modelled from measured per-block costs
// (128 x 64: 0.24 us, 128 x 128: 0.35 us, 128 x 256: 0.5 us) plus fixed
// costs (prologue and output write: ~3.5 us, ~5.5 us for the 128 x 256
// tile's 128 KiB), times the waves of CTAs.  Returns true for 256.
thread_local int t_fold_override = 0;

bool fold_wide(int dev, int m, int n, int nb) {
    const int sms = sms_of(dev);
    const long mt = (m + BM - 1) / BM;
    const long tiles128 = long((n + 127) / 128) * mt;
    const bool bn64 = 2 * tiles128 <= sms;
    const long narrow_tiles = bn64 ? 2 * tiles128 : tiles128;
    const double narrow = double((narrow_tiles + sms - 1) / sms) * (3.5 + nb * (bn64 ? 0.24 : 0.35));
    const long wide_tiles = long((n + wide::BN - 1) / wide::BN) * mt;
    const double wide_t = double((wide_tiles + sms - 1) / sms) * (5.5 + nb * 0.5);
    return wide_t < narrow;
}

// qout (optional): instead of y, GELU of the output quantized into this
// GEMM-layout operand (q16, dT, uT, m_pad; k = w.n).
// heads (optional): instead of y, f16 attention heads [n_win][H][T][64] of
// y * scale (v.m == n_win * T, w.n == H * 64).
struct HeadsOut {
    __half* dst;
    int n_win, T, H;
    float scale;
};
cudaError_t launch_fold_wide(const ActsView& v, const Weight& w, const float* bias, float* y, int* err_flag,
                             cudaStream_t s, char* why, size_t why_len, const ActsView* qout = nullptr,
                             const HeadsOut* heads = nullptr) {
    const int dev = cur_dev();
    cudaError_t e = wide_smem_attr(dev);
    if (e != cudaSuccess) return e;
    CUtensorMap ma, mb, my, md;
    if (!encode_map(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, v.q16, uint64_t(v.k), uint64_t(v.m), 32, BM,
                    CU_TENSOR_MAP_SWIZZLE_64B, why, why_len))
        return cudaErrorInvalidValue;
    if (!encode_map(&mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, w.bhl, uint64_t(w.nb) * 64, uint64_t(w.n), 64, wide::BN,
                    CU_TENSOR_MAP_SWIZZLE_128B, why, why_len))
        return cudaErrorInvalidValue;
    if (!encode_map(&md, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, v.dT, uint64_t(v.m_pad), uint64_t(w.nb), BM, DA_GROUP,
                    CU_TENSOR_MAP_SWIZZLE_NONE, why, why_len))
        return cudaErrorInvalidValue;
    int use_tma_store = !qout && !heads && (w.n % 4 == 0) && (reinterpret_cast<uintptr_t>(y) % 16 == 0);
    if (use_tma_store && !encode_map(&my, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, y, uint64_t(w.n), uint64_t(v.m), 32, 32,
                                     CU_TENSOR_MAP_SWIZZLE_128B, why, why_len))
        use_tma_store = 0;
    if (!use_tma_store) memset(&my, 0, sizeof my);
    CUtensorMap mq;
    memset(&mq, 0, sizeof mq);
    if (qout && !encode_map(&mq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, qout->q16, uint64_t(w.n), uint64_t(v.m), 64, 32,
                            CU_TENSOR_MAP_SWIZZLE_128B, why, why_len))
        return cudaErrorInvalidValue;
    if (heads && !encode_map(&mq, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, heads->dst, 64,
                             uint64_t(heads->n_win) * heads->H * heads->T, 64, 32, CU_TENSOR_MAP_SWIZZLE_128B, why,
                             why_len))
        return cudaErrorInvalidValue;
    const int nt = (w.n + wide::BN - 1) / wide::BN, mt = (v.m + BM - 1) / BM;
    const dim3 grid(static_cast<unsigned>(nt), static_cast<unsigned>(mt));
    return launch_pdl(k_gemm_fold_w, grid, dim3(wide::THREADS), wide::SMEM, s, ma, mb, my, md, use_tma_store,
                      w.colscale, bias, y, v.m, w.n, w.nb, err_flag, mq, qout ? qout->dT : nullptr,
                      qout ? qout->uT : nullptr, qout ? qout->m_pad : 0, heads ? heads->dst : nullptr,
                      heads ? heads->T : 1, heads ? heads->H : 1, heads ? heads->scale : 1.0f);
}

cudaError_t launch_fold(const ActsView& v, const Weight& w, const float* bias, float* y, int* err_flag,
                        cudaStream_t s, char* why, size_t why_len) {
    const int dev = cur_dev();
    const bool wide_tiles = t_fold_override ? t_fold_override == 2 : fold_wide(dev, v.m, w.n, w.nb);
    if (wide_tiles) return launch_fold_wide(v, w, bias, y, err_flag, s, why, why_len);
    const long tiles128 = long((w.n + 127) / 128) * ((v.m + BM - 1) / BM);
    // 64-wide tiles when they still fit in one wave and 128-wide ones
    // would leave at least half the SMs idle.
    if (2 * tiles128 <= sms_of(dev)) return launch_fold_bn<64>(v, w, bias, y, err_flag, s, why, why_len);
    return launch_fold_bn<128>(v, w, bias, y, err_flag, s, why, why_len);
}

}  // namespace

cudaError_t launch_gemm_fold(const ActsView& v, const Weight& w, const float* bias, float* y, int* err_flag,
                             cudaStream_t s, char* why, size_t why_len) {
    if (v.m <= 0 || w.n <= 0) return cudaSuccess;
    return launch_fold(v, w, bias, y, err_flag, s, why, why_len);
}

bool gemm_fold_gelu_fits(const ActsView& v, const Weight& w, const ActsView& out) {
    auto al = [](const void* p, uintptr_t a) { return p && (reinterpret_cast<uintptr_t>(p) % a) == 0; };
    return v.m > 0 && w.n % wide::BN == 0 && out.k == w.n && out.m_pad >= v.m && al(out.q16, 16) && al(out.dT, 4) &&
           al(out.uT, 4);
}

cudaError_t launch_gemm_fold_gelu(const ActsView& v, const Weight& w, const float* bias, const ActsView& out,
                                  int* err_flag, cudaStream_t s, char* why, size_t why_len) {
    if (!gemm_fold_gelu_fits(v, w, out)) return cudaErrorInvalidValue;
    return launch_fold_wide(v, w, bias, nullptr, err_flag, s, why, why_len, &out);
}

bool gemm_fold_heads_fits(const ActsView& v, const Weight& w, int n_win, int T, int H, const __half* dst) {
    return v.m > 0 && v.m == n_win * T && T >= 32 && w.n == H * 64 && w.n % wide::BN == 0 && dst &&
           (reinterpret_cast<uintptr_t>(dst) % 16) == 0;
}

cudaError_t launch_gemm_fold_heads(const ActsView& v, const Weight& w, const float* bias, __half* dst, int n_win,
                                   int T, int H, float scale, int* err_flag, cudaStream_t s, char* why,
                                   size_t why_len) {
    if (!gemm_fold_heads_fits(v, w, n_win, T, H, dst)) return cudaErrorInvalidValue;
    const HeadsOut ho{dst, n_win, T, H, scale};
    return launch_fold_wide(v, w, bias, nullptr, err_flag, s, why, why_len, nullptr, &ho);
}

int gemm_fold_config(int m, int n, int nb) { return fold_wide(cur_dev(), m, n, nb) ? 2 : 1; }

void set_gemm_fold_config(int code) { t_fold_override = (code == 1 || code == 2) ? code : 0; }

}  // namespace rwq
