// rwq_gemm_hl_sm100.cu -- tensor-core GEMM with both operands split into
// f16 hi + lo and the whole K accumulated in tensor memory.
//
// rusty_whisper's int8 tier computes (quant.rs:10, 349-354, 452-454)
//     y[i,j] = sum_kb d_a[i,kb] * sum_{l<32} q_a[i,32kb+l] * x[j,32kb+l]
// with x = d_b*q_b + m_b the dequantized weight; that is the plain dot
// product of the dequantized activation a'[i,l] = d_a*q_a (one f32 product,
// __fmul_rn) with x.  Its f32 fallback (quant.rs:995-1018) and
// `matmul_t(a, to_dense)` (quant.rs:1194) are the same dot with a' = a.  So
// both tiers are one dense GEMM  y = A' X^T  whose operands need about 22
// significant bits each (the 1e-3 rule of quant.rs:1365 holds for outputs
// near zero only if the operands' rounding stays below ~2^-16 of the row's
// scale).  Each row of A' and X is scaled by a power of two (exact) so its
// largest magnitude lies in [2^10, 2^11) and split into f16 hi + lo
// (hi = f16(v), lo = f16(v - hi)); per 16-wide K step three
// `tcgen05.mma.kind::f16` form hi*hi + hi*lo + lo*hi (the lo*lo term is
// below 2^-22 of the product).  The tensor core adds each MMA into its f32
// accumulator without rounding to nearest (the dropped bits always move
// the sum toward zero), so a long K run into one accumulator drifts by up
// to ~0.5 ulp of the running sum per MMA: at k = 5120 that reached 1e-3 of
// the outputs near zero.  Hence two accumulators: D1 takes the small
// hi*lo + lo*hi terms over the whole K (2^-11 of the sum, so its drift is
// negligible), D0 takes hi*hi and is drained every DRAIN K blocks into f32
// registers of the epilogue warps (round to nearest), so each D0 run is
// 2*DRAIN MMAs of partial sums of 32*DRAIN terms.  y = sum of the D0 runs
// + D1, then times the two scales' inverses (exact), plus the bias.
//
// Operand layout, A and B alike: per row and 32-wide K block, 32 f16 "hi"
// then 32 f16 "lo" (128 bytes); rows are nb * 128 bytes.  B is the weight's
// folded operand cache (Weight::bhl / colscale, k_build_fold_cache) or,
// for dense f32 weights, the same layout built by rwq_hl_build_dense.
//
// Roles (320 threads, one CTA per 128 x BN output tile and K slice):
//   warp 0     TMA producer: per K block one stage (A: 128 x 64 f16, B: BN
//              x 64 f16, 128-byte swizzle); allocates / frees TMEM;
//   warp 1     MMA issuer (one thread): per block 4 MMAs into D1 and 2 into
//              D0 (after waiting for D0's drain at a run start), a commit
//              per stage and one per D0 run;
//   warps 2-9  epilogue: warp w owns TMEM lanes 32*(w%4).. and half of the
//              columns; it adds every D0 run into registers, then D1,
//              scales, adds the bias and writes 32 x 32 boxes into the
//              drained stage ring for TMA stores.  With the K range split
//              over a cluster of S CTAs, each leaves its unscaled tile in
//              shared memory and adds a row slice of all S tiles in slice
//              order (distributed shared memory).
// Every wait is bounded (rwq_sm100.cuh); no load uses cluster multicast.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include "rwq_common.cuh"
#include "rwq_internal.h"
#include "rwq_sm100.cuh"

namespace rwq {
namespace {

using namespace tc;

constexpr int HL_BM = 128;
constexpr int HL_A_BYTES = HL_BM * 128;     // one K block: 128 rows x (32 hi + 32 lo) f16
constexpr int HL_EPI0 = 2;                  // first epilogue warp
constexpr int HL_EPI_WARPS = 8;
constexpr int HL_THREADS = (HL_EPI0 + HL_EPI_WARPS) * 32;
constexpr int HL_DRAIN = 8;                 // K blocks per D0 run
// How an unsplit tile reaches Y: TMA stores of 32 x 32 boxes (N % 4 == 0
// and Y 16-byte aligned), float4 stores, or element stores.
enum { HL_STORE_TMA = 0, HL_STORE_VEC = 1, HL_STORE_SCALAR = 2 };

template <int BN>
struct Hl {
    static constexpr int B_BYTES = BN * 128;
    static constexpr int STAGE_BYTES = HL_A_BYTES + B_BYTES;
    static constexpr int STAGES = BN == 256 ? 4 : BN == 128 ? 6 : 8;   // 192 KiB of stages
    // K-split partial tiles in the drained stages: rows of BN + 4 floats, so
    // the eight rows a quarter-warp writes at once fall in distinct banks.
    static constexpr int PITCH = BN + 4;
    static constexpr int TMEM_COLS = 2 * BN;              // D0 at column 0, D1 at column BN
    static constexpr int CPW = BN / 2;                    // columns per epilogue warp
    // kind::f16, D f32, A/B f16, both K-major, N>>3 at bit 17, M>>4 at bit 24.
    static constexpr uint32_t IDESC = (1u << 4) | (uint32_t(BN >> 3) << 17) | (uint32_t(HL_BM >> 4) << 24);
    struct Bars {
        uint64_t full[STAGES], empty[STAGES], d0_full, d0_empty;
        uint32_t tmem_base;
        int abort;
        // the tile's row scales, column scales and bias, loaded during the
        // mainloop so the copy-out reads them from shared memory
        alignas(16) float rs[HL_BM];
        alignas(16) float cs[BN];
        alignas(16) float bs[BN];
    };
    static constexpr int SMEM = STAGES * STAGE_BYTES + int(sizeof(Bars)) + 1024;
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
    static_assert(HL_BM * PITCH * 4 <= STAGES * STAGE_BYTES, "the output tile must fit in the drained stages");
    static_assert(BN == 64 || BN == 128 || BN == 256, "tile width");
};

__device__ __forceinline__ uint32_t hl_mapa(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ float4 hl_ld_cluster4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}
__device__ __forceinline__ void hl_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// grid: x = n_tiles * S (K slice = blockIdx.x % S), y = m_tiles.  Slice r
// covers K blocks [r*kps, min(nb, (r+1)*kps)), never empty (the host picks
// S so).  S > 1: the S CTAs of a cluster (along x) each leave their
// unscaled tile in shared memory and add row slices of all S tiles.
template <int BN>
__global__ void __launch_bounds__(HL_THREADS, 1)
    k_gemm_hl(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const __grid_constant__ CUtensorMap tmY, const float* __restrict__ rowscale,
              const float* __restrict__ colscale, const float* __restrict__ bias, float* __restrict__ Y, int M, int N,
              int nb, int kps, int S, int store_mode, int* __restrict__ err_flag, int gelu,
              const float* __restrict__ epos, int epos_period) {
    using F = Hl<BN>;
    constexpr int STAGES = F::STAGES, STAGE_BYTES = F::STAGE_BYTES, PITCH = F::PITCH, CPW = F::CPW;
    constexpr uint32_t IDESC = F::IDESC;
    using Bars = typename F::Bars;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    Bars* bar = reinterpret_cast<Bars*>(base + STAGES * STAGE_BYTES);
    volatile int* abort = &bar->abort;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int split = int(blockIdx.x) % S;
    const int n0 = (int(blockIdx.x) / S) * BN, m0 = int(blockIdx.y) * HL_BM;
    const int kb0 = split * kps, kb1 = min(nb, kb0 + kps);
    const int nblk = kb1 - kb0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&bar->full[s], 1);
            mbar_init(&bar->empty[s], 1);
        }
        mbar_init(&bar->d0_full, 1);
        mbar_init(&bar->d0_empty, HL_EPI_WARPS);
        bar->abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&bar->tmem_base)),
                     "r"(F::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (threadIdx.x == 32) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
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
                if (!mbar_wait(&bar->empty[s], ((i / STAGES) & 1) ^ 1, abort, err_flag, 11)) break;
                uint8_t* st = base + s * STAGE_BYTES;
                mbar_expect_tx(&bar->full[s], STAGE_BYTES);
                tma_load_2d(st, &tmA, (kb0 + i) * 64, m0, &bar->full[s]);
                tma_load_2d(st + HL_A_BYTES, &tmB, (kb0 + i) * 64, n0, &bar->full[s]);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t d0 = tmem, d1 = tmem + uint32_t(BN);
            for (int i = 0; i < nblk; ++i) {
                const int s = i % STAGES;
                if (!mbar_wait(&bar->full[s], (i / STAGES) & 1, abort, err_flag, 12)) break;
                tc_fence_after();
                const uint32_t a0 = smem_u32(base + s * STAGE_BYTES);
                const uint32_t b0 = a0 + uint32_t(HL_A_BYTES);
                // K step ks of the block: hi at bytes 32ks.., lo at 64 + 32ks..
#pragma unroll
                for (int ks = 0; ks < 2; ++ks) {
                    const uint32_t ah = a0 + 32u * ks, bh = b0 + 32u * ks;
                    mma_f16_id(d1, sw128_desc(ah), sw128_desc(bh + 64u), IDESC, (i | ks) != 0);
                    mma_f16_id(d1, sw128_desc(ah + 64u), sw128_desc(bh), IDESC, 1);
                }
                const int run = i / HL_DRAIN, pos = i % HL_DRAIN;
                // A new D0 run starts once the epilogue has drained the last.
                if (pos == 0 && run > 0 && !mbar_wait(&bar->d0_empty, (run - 1) & 1, abort, err_flag, 14)) break;
                tc_fence_after();
#pragma unroll
                for (int ks = 0; ks < 2; ++ks)
                    mma_f16_id(d0, sw128_desc(a0 + 32u * ks), sw128_desc(b0 + 32u * ks), IDESC, (pos | ks) != 0);
                mma_commit(&bar->empty[s]);
                if (pos == HL_DRAIN - 1 || i == nblk - 1) mma_commit(&bar->d0_full);   // the last one covers D1
            }
        }
        __syncwarp();
    } else {
        {   // scales and bias of the tile, zero past the edges
            const int t = int(threadIdx.x) - HL_EPI0 * 32;   // 0 .. 255
            if (t < HL_BM) bar->rs[t] = m0 + t < M ? __ldg(rowscale + m0 + t) : 0.f;
            for (int c = t; c < BN; c += HL_EPI_WARPS * 32) {
                bar->cs[c] = __ldg(colscale + n0 + c);   // padded to a multiple of 256 columns
                bar->bs[c] = (bias && n0 + c < N) ? __ldg(bias + n0 + c) : 0.f;
            }
        }
        // Epilogue: warp w owns TMEM lanes 32*(w%4).. (tile rows) and
        // columns h*CPW .. h*CPW + CPW of D0 and D1.
        const int q = warp & 3, h = (warp - HL_EPI0) >> 2;
        const uint32_t lane_off = uint32_t(q * 32) << 16;
        float acc[CPW];
#pragma unroll
        for (int c = 0; c < CPW; ++c) acc[c] = 0.f;
        const int runs = (nblk + HL_DRAIN - 1) / HL_DRAIN;
        bool ok = true;
        for (int r = 0; r < runs && ok; ++r) {
            ok = __all_sync(0xffffffffu, mbar_wait(&bar->d0_full, r & 1, abort, err_flag, 13));
            if (!ok) break;
            tc_fence_after();
            // 16 columns per load: the 10 warps' registers share four
            // 16K-register sub-partitions (3 warps on two of them), so a
            // thread has 168 registers, CPW of them the run sums.
#pragma unroll
            for (int c = 0; c < CPW; c += 16) {
                uint32_t v[16];
                tmem_ld16(tmem + lane_off + uint32_t(h * CPW + c), v);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 16; ++e) acc[c + e] = __fadd_rn(acc[c + e], __uint_as_float(v[e]));
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar->d0_empty);
        }
        if (ok) {
            // The last D0 commit came after every MMA, D1's included.  One
            // 32-column box at a time: sums = D0 runs + D1, then (S == 1)
            // y = sum * 2^-e_j * 2^-e_i (+ bias) into a 32 x 32 box of the
            // drained stage ring for a TMA store (128-byte swizzle: 16-byte
            // chunk k of row r at k ^ (r & 7); box (q, column box cb) at
            // (q * BN/32 + cb) * 4 KiB), or straight to Y; (S > 1) the
            // unscaled sums into the drained ring as rows of PITCH floats.
            const int row = q * 32 + lane;
            const float rs = bar->rs[row];
#pragma unroll
            for (int bx = 0; bx < CPW / 32; ++bx) {
                const int c0 = bx * 32, cb = h * (CPW / 32) + bx;
                float v[32];
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint32_t d1[16];
                    tmem_ld16(tmem + lane_off + uint32_t(BN + h * CPW + c0 + 16 * half), d1);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 16; ++e) v[16 * half + e] = __fadd_rn(acc[c0 + 16 * half + e], __uint_as_float(d1[e]));
                }
                if (S == 1) {
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        const int cc = cb * 32 + e;
                        float t = __fmul_rn(__fmul_rn(v[e], bar->cs[cc]), rs);
                        v[e] = bias ? __fadd_rn(t, bar->bs[cc]) : t;
                    }
                    if (gelu) {
#pragma unroll
                        for (int e = 0; e < 32; ++e) v[e] = gelu_ref(v[e]);
                    }
                    if (epos && m0 + row < M && n0 + cb * 32 + 32 <= N) {   // rows of N floats, N % 4 == 0
                        const float4* pr = reinterpret_cast<const float4*>(
                            epos + size_t((m0 + row) % epos_period) * N + n0 + cb * 32);
#pragma unroll
                        for (int k4 = 0; k4 < 8; ++k4) {
                            const float4 pv = __ldg(pr + k4);
                            v[4 * k4] = __fadd_rn(v[4 * k4], pv.x);
                            v[4 * k4 + 1] = __fadd_rn(v[4 * k4 + 1], pv.y);
                            v[4 * k4 + 2] = __fadd_rn(v[4 * k4 + 2], pv.z);
                            v[4 * k4 + 3] = __fadd_rn(v[4 * k4 + 3], pv.w);
                        }
                    } else if (epos && m0 + row < M) {
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            if (n0 + cb * 32 + e < N)
                                v[e] = __fadd_rn(v[e], epos[size_t((m0 + row) % epos_period) * N + n0 + cb * 32 + e]);
                    }
                    if (store_mode == HL_STORE_TMA) {
                        uint8_t* box = base + (q * (BN / 32) + cb) * 4096 + lane * 128;
#pragma unroll
                        for (int k4 = 0; k4 < 8; ++k4)
                            *reinterpret_cast<float4*>(box + ((k4 ^ (lane & 7)) << 4)) =
                                make_float4(v[4 * k4], v[4 * k4 + 1], v[4 * k4 + 2], v[4 * k4 + 3]);
                    } else if (m0 + row < M) {
                        float* yr = Y + size_t(m0 + row) * N + n0 + cb * 32;
#pragma unroll
                        for (int e = 0; e < 32; ++e)
                            if (n0 + cb * 32 + e < N) yr[e] = v[e];
                    }
                } else {
                    float* pr = reinterpret_cast<float*>(base) + size_t(row) * PITCH + cb * 32;
#pragma unroll
                    for (int e = 0; e < 32; e += 4)
                        *reinterpret_cast<float4*>(pr + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
                }
            }
            if (S == 1 && store_mode == HL_STORE_TMA) {
                fence_async_smem();
                __syncwarp();
                if (lane == 0) {
#pragma unroll
                    for (int bx = 0; bx < CPW / 32; ++bx) {
                        const int cb = h * (CPW / 32) + bx;
                        if (n0 + cb * 32 < N && m0 + q * 32 < M)
                            tma_store_2d(&tmY, n0 + cb * 32, m0 + q * 32, base + (q * (BN / 32) + cb) * 4096);
                    }
                    bulk_commit();
                    bulk_wait_read_all();
                }
                __syncwarp();
            }
        }
    }

    // Every thread of every CTA of the cluster reaches both barriers, also
    // after an expired wait, so the cluster never waits on a CTA that left.
    tc_fence_before();
    if (S > 1) hl_cluster_sync();
    else __syncthreads();
    if (S > 1 && !*abort) {
        // Slice `split` adds rows [r0, r1) of the S partial tiles in slice
        // order (distributed shared memory), scales, adds the bias and
        // stores; four float4 per thread per round, loads before stores.
        const int r0 = split * HL_BM / S, r1 = (split + 1) * HL_BM / S;
        const uint32_t part_s = smem_u32(base);
        constexpr int C4 = BN / 4, U = 4;
        const int total = (r1 - r0) * C4;
        for (int i0 = threadIdx.x; i0 < total; i0 += U * HL_THREADS) {
            float4 acc[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int idx = min(i0 + u * HL_THREADS, total - 1);
                const int rr = r0 + idx / C4, c = (idx % C4) * 4;
                const uint32_t off = part_s + uint32_t((rr * PITCH + c) * 4);
                acc[u] = hl_ld_cluster4(hl_mapa(off, 0));
                for (int s2 = 1; s2 < S; ++s2) {
                    const float4 t = hl_ld_cluster4(hl_mapa(off, uint32_t(s2)));
                    acc[u].x = __fadd_rn(acc[u].x, t.x);
                    acc[u].y = __fadd_rn(acc[u].y, t.y);
                    acc[u].z = __fadd_rn(acc[u].z, t.z);
                    acc[u].w = __fadd_rn(acc[u].w, t.w);
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int idx = i0 + u * HL_THREADS;
                if (idx >= total) break;
                const int rr = r0 + idx / C4, c = (idx % C4) * 4;
                const int gi = m0 + rr, gj = n0 + c;
                if (gi >= M || gj >= N) continue;
                const float rs = bar->rs[rr];
                const float4 cs = *reinterpret_cast<const float4*>(bar->cs + c);
                const float4 bs = *reinterpret_cast<const float4*>(bar->bs + c);
                float4 v = make_float4(__fmul_rn(__fmul_rn(acc[u].x, cs.x), rs), __fmul_rn(__fmul_rn(acc[u].y, cs.y), rs),
                                       __fmul_rn(__fmul_rn(acc[u].z, cs.z), rs), __fmul_rn(__fmul_rn(acc[u].w, cs.w), rs));
                if (bias) {
                    v.x = __fadd_rn(v.x, bs.x);
                    v.y = __fadd_rn(v.y, bs.y);
                    v.z = __fadd_rn(v.z, bs.z);
                    v.w = __fadd_rn(v.w, bs.w);
                }
                if (gelu) v = make_float4(gelu_ref(v.x), gelu_ref(v.y), gelu_ref(v.z), gelu_ref(v.w));
                if (epos) {
                    const float* pr = epos + size_t(gi % epos_period) * N + gj;
                    v.x = __fadd_rn(v.x, pr[0]);
                    if (gj + 1 < N) v.y = __fadd_rn(v.y, pr[1]);
                    if (gj + 2 < N) v.z = __fadd_rn(v.z, pr[2]);
                    if (gj + 3 < N) v.w = __fadd_rn(v.w, pr[3]);
                }
                float* yr = Y + size_t(gi) * N + gj;
                if (store_mode != HL_STORE_SCALAR) {   // N % 4 == 0 and Y 16-byte aligned: gj + 3 < N
                    *reinterpret_cast<float4*>(yr) = v;
                } else {
                    const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        if (gj + e < N) yr[e] = vv[e];
                }
            }
        }
    }
    // No CTA leaves (or frees its TMEM) while a peer still reads its tile.
    if (S > 1) hl_cluster_sync();
    else __syncthreads();
    tc_fence_after();
    if (warp == 0) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(F::TMEM_COLS)
                     : "memory");
    }
}

// ------------------------------------------------ activation operand
// One CTA of 128 threads per row.  QUANT: the reference's int8 quantizer
// (quant.rs:690-716, as k_quantize: d = amax/127, inv = 1/d or 0, q =
// round(x*inv) half away from zero, clamped, NaN -> 0), then the
// dequantized value a' = d*q; otherwise a' = x.  Pass 1 finds the row's
// largest |a'| (NaN ignored), pass 2 writes a'*2^e = hi + lo.  Eight lanes
// share a 32-element block (4 elements each).
template <bool QUANT, bool VEC>
__device__ __forceinline__ float4 hl_act_values(const float* __restrict__ xr, int e) {
    const float4 x = VEC ? *reinterpret_cast<const float4*>(xr + e) : make_float4(xr[e], xr[e + 1], xr[e + 2], xr[e + 3]);
    if (!QUANT) return x;
    auto absnn = [](float v) { const float w = fabsf(v); return isnan(w) ? 0.f : w; };
    float amax = fmaxf(fmaxf(absnn(x.x), absnn(x.y)), fmaxf(absnn(x.z), absnn(x.w)));
    const unsigned grp = 0xFFu << (threadIdx.x & 24);
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(grp, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    const float inv = d > 0.f ? __fdiv_rn(1.0f, d) : 0.f;
    auto deq = [d, inv](float v) {
        const float r = roundf(__fmul_rn(v, inv));
        const int c = isnan(r) ? 0 : int(fminf(127.f, fmaxf(-127.f, r)));
        return __fmul_rn(d, float(c));
    };
    return make_float4(deq(x.x), deq(x.y), deq(x.z), deq(x.w));
}

__device__ __forceinline__ uint2 hl_pack_hi(float4 v, float4& rest) {
    const __half h0 = __float2half_rn(v.x), h1 = __float2half_rn(v.y), h2 = __float2half_rn(v.z),
                 h3 = __float2half_rn(v.w);
    rest = make_float4(__fsub_rn(v.x, __half2float(h0)), __fsub_rn(v.y, __half2float(h1)),
                       __fsub_rn(v.z, __half2float(h2)), __fsub_rn(v.w, __half2float(h3)));
    return make_uint2(uint32_t(__half_as_ushort(h0)) | (uint32_t(__half_as_ushort(h1)) << 16),
                      uint32_t(__half_as_ushort(h2)) | (uint32_t(__half_as_ushort(h3)) << 16));
}

// Power-of-two exponent putting a row's largest magnitude in [2^10, 2^11)
// (0 for an all-zero or non-finite row), as k_build_fold_cache does for
// weight rows.
__device__ __forceinline__ int hl_row_exp(float mx) {
    if (!(mx > 0.f) || !isfinite(mx)) return 0;
    int E;
    frexpf(mx, &E);
    return max(-120, min(120, 11 - E));
}

template <bool QUANT, bool VEC>
__global__ void __launch_bounds__(128) k_split_rows(const float* __restrict__ a, int m, int k, int lda,
                                                    uint16_t* __restrict__ ahl, float* __restrict__ rowscale) {
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.x;
    if (row >= m) return;
    const float* xr = a + size_t(row) * lda;
    const int nb = k / QK;
    // 128 threads = 16 blocks per pass; thread t: block t/8, elements 4(t%8)..
    const int bsub = threadIdx.x >> 3, esub = (threadIdx.x & 7) * 4;
    float mx = 0.f;
    for (int b0 = 0; b0 < nb; b0 += 16) {
        const int b = b0 + bsub;
        if (b < nb) {   // the 8 lanes of a block take part together
            const float4 v = hl_act_values<QUANT, VEC>(xr, b * QK + esub);
            auto absnn = [](float t) { const float w = fabsf(t); return isnan(w) ? 0.f : w; };
            mx = fmaxf(mx, fmaxf(fmaxf(absnn(v.x), absnn(v.y)), fmaxf(absnn(v.z), absnn(v.w))));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    __shared__ float s_mx[4];
    if ((threadIdx.x & 31) == 0) s_mx[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(s_mx[0], s_mx[1]), fmaxf(s_mx[2], s_mx[3]));
    const int ex = hl_row_exp(mx);
    const float up = ldexpf(1.0f, ex);
    for (int b0 = 0; b0 < nb; b0 += 16) {
        const int b = b0 + bsub;
        if (b < nb) {
            float4 v = hl_act_values<QUANT, VEC>(xr, b * QK + esub);
            v = make_float4(__fmul_rn(v.x, up), __fmul_rn(v.y, up), __fmul_rn(v.z, up), __fmul_rn(v.w, up));
            float4 rest;
            const uint2 hi = hl_pack_hi(v, rest);
            float4 dummy;
            const uint2 lo = hl_pack_hi(rest, dummy);
            uint16_t* o = ahl + (size_t(row) * nb + b) * 64;
            *reinterpret_cast<uint2*>(o + esub) = hi;
            *reinterpret_cast<uint2*>(o + 32 + esub) = lo;
        }
    }
    if (threadIdx.x == 0) rowscale[row] = ldexpf(1.0f, -ex);
}

// The im2col rows of a kernel-3, padding-1 conv1d (tensor.rs:335-370),
// straight into the hi|lo operand: output row r = (window w, time t) has
// column j = c*3 + kk (j < 3*c_in) = in[w, c, t*stride + kk - 1] (0 outside
// [0, t_in)), columns 3*c_in .. kp-1 zero; element (w, c, t) of the input
// sits at in[w*sw + c*sc + t*st].  One CTA of 128 threads per row: pass 1
// finds the row's largest |value|, pass 2 writes value*2^e = hi + lo.
__device__ __forceinline__ float im2col_at(const float* __restrict__ in, int w, int t, int j, int c_in, int t_in,
                                           int stride, size_t sw, size_t sc, size_t st) {
    if (j >= 3 * c_in) return 0.f;
    const int c = j / 3, ti = t * stride + (j - 3 * c) - 1;
    return (ti >= 0 && ti < t_in) ? __ldg(in + size_t(w) * sw + size_t(c) * sc + size_t(ti) * st) : 0.f;
}

__global__ void __launch_bounds__(128) k_im2col_split(const float* __restrict__ in, int c_in, int t_in, int t_out,
                                                      int stride, size_t sw, size_t sc, size_t st, int kp,
                                                      uint16_t* __restrict__ ahl, float* __restrict__ rowscale) {
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.x;
    const int w = row / t_out, t = row % t_out;
    const int nb = kp / QK;
    const int bsub = threadIdx.x >> 3, esub = (threadIdx.x & 7) * 4;
    float mx = 0.f;
    for (int b = bsub; b < nb; b += 16)
#pragma unroll
        for (int e = 0; e < 4; ++e)
            mx = fmaxf(mx, fabsf(im2col_at(in, w, t, b * QK + esub + e, c_in, t_in, stride, sw, sc, st)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    __shared__ float s_mx[4];
    if ((threadIdx.x & 31) == 0) s_mx[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = fmaxf(fmaxf(s_mx[0], s_mx[1]), fmaxf(s_mx[2], s_mx[3]));
    const int ex = hl_row_exp(mx);
    const float up = ldexpf(1.0f, ex);
    for (int b = bsub; b < nb; b += 16) {
        float4 v;
        v.x = __fmul_rn(im2col_at(in, w, t, b * QK + esub, c_in, t_in, stride, sw, sc, st), up);
        v.y = __fmul_rn(im2col_at(in, w, t, b * QK + esub + 1, c_in, t_in, stride, sw, sc, st), up);
        v.z = __fmul_rn(im2col_at(in, w, t, b * QK + esub + 2, c_in, t_in, stride, sw, sc, st), up);
        v.w = __fmul_rn(im2col_at(in, w, t, b * QK + esub + 3, c_in, t_in, stride, sw, sc, st), up);
        float4 rest, dummy;
        const uint2 hi = hl_pack_hi(v, rest);
        const uint2 lo = hl_pack_hi(rest, dummy);
        uint16_t* o = ahl + (size_t(row) * nb + b) * 64;
        *reinterpret_cast<uint2*>(o + esub) = hi;
        *reinterpret_cast<uint2*>(o + 32 + esub) = lo;
    }
    if (threadIdx.x == 0) rowscale[row] = ldexpf(1.0f, -ex);
}

// Dense f32 weight rows [n][ldw] (first kv columns used, zeros up to k,
// k % 32 == 0) into the hi|lo operand layout with per-row scales; rows
// n..n_pad-1 get colscale 0.  One warp per row.
__global__ void k_split_dense(const float* __restrict__ w, int n, int k, int kv, int ldw, int n_pad,
                              uint16_t* __restrict__ bhl, float* __restrict__ colscale) {
    const int lane = threadIdx.x & 31;
    const int j = int((size_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
    if (j >= n_pad) return;
    if (j >= n) {
        if (lane == 0) colscale[j] = 0.f;
        return;
    }
    const float* wr = w + size_t(j) * ldw;
    float mx = 0.f;
    for (int e = lane; e < kv; e += 32) mx = fmaxf(mx, fabsf(wr[e]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const int ex = hl_row_exp(mx);
    const float up = ldexpf(1.0f, ex);
    const int nb = k / QK;
    for (int b = 0; b < nb; ++b) {
        const int e = b * QK + lane;
        const float v = e < kv ? __fmul_rn(wr[e], up) : 0.f;
        const __half h = __float2half_rn(v);
        const __half l = __float2half_rn(__fsub_rn(v, __half2float(h)));
        uint16_t* o = bhl + (size_t(j) * nb + b) * 64;
        o[lane] = __half_as_ushort(h);
        o[32 + lane] = __half_as_ushort(l);
    }
    if (lane == 0) colscale[j] = ldexpf(1.0f, -ex);
}

// ------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_once;

bool encode_map(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t rows, uint32_t box_rows, char* why,
                size_t why_len) {
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
    cuuint64_t strides[1] = {inner * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        snprintf(why, why_len, "cuTensorMapEncodeTiled failed (%d)", int(r));
        return false;
    }
    return true;
}

// Y as a 2-D f32 tensor [rows][inner] for 32 x 32 TMA store boxes,
// 128-byte swizzle (inner * 4 must be a multiple of 16).
bool encode_map_f32(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t rows, char* why, size_t why_len) {
    if (!g_encode) return false;
    cuuint64_t dims[2] = {inner, rows};
    cuuint64_t strides[1] = {inner * 4};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        snprintf(why, why_len, "cuTensorMapEncodeTiled (output) failed (%d)", int(r));
        return false;
    }
    return true;
}

struct DevInfo {
    int sms = 0;
    bool attr[3] = {};
};
DevInfo g_dev[64];
std::mutex g_dev_mu;

template <int BN>
constexpr int bn_index() {
    return BN == 64 ? 0 : BN == 128 ? 1 : 2;
}

// Active clusters of S CTAs that fit at once (cached per device, BN, S).
int g_max_clusters[64][3][5];

template <int BN>
int max_active_clusters(int dev, int S) {
    std::lock_guard<std::mutex> g(g_dev_mu);
    int& slot = g_max_clusters[dev][bn_index<BN>()][S];
    if (slot == 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(unsigned(S) * 60, 1);
        cfg.blockDim = dim3(HL_THREADS);
        cfg.dynamicSmemBytes = Hl<BN>::SMEM;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = unsigned(S);
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, k_gemm_hl<BN>, &cfg) != cudaSuccess || n < 1) {
            cudaGetLastError();
            n = -1;
        }
        slot = n;
    }
    return slot;
}

thread_local int t_ksplit_override = 0;

int cur_dev() {
    int dev = 0;
    cudaGetDevice(&dev);
    return dev < 64 ? dev : 63;
}


int sms_of(int dev) {
    std::lock_guard<std::mutex> g(g_dev_mu);
    if (g_dev[dev].sms == 0) cudaDeviceGetAttribute(&g_dev[dev].sms, cudaDevAttrMultiProcessorCount, dev);
    return g_dev[dev].sms > 0 ? g_dev[dev].sms : 148;
}

template <int BN>
cudaError_t ensure_smem_attr(int dev) {
    std::lock_guard<std::mutex> g(g_dev_mu);
    if (!g_dev[dev].attr[bn_index<BN>()]) {
        cudaError_t e = cudaFuncSetAttribute(k_gemm_hl<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, Hl<BN>::SMEM);
        if (e != cudaSuccess) return e;
        g_dev[dev].attr[bn_index<BN>()] = true;
    }
    return cudaSuccess;
}

// Tile width BN and K slices S of an m x n GEMM with nb blocks, from a
// cost estimate in units of one 128 x 256 K block of MMAs: per CTA
// ceil(nb/S) blocks at a BN-dependent cost (narrower MMAs do less work per
// cycle but are bound by shared-memory bandwidth, not proportionally
// cheaper) plus fixed costs (prologue, TMEM drain and copy-out; each
// extra slice adds a partial tile to read through distributed shared
// memory), times the waves of CTAs.  K-split clusters must all be resident
// at once.  A row's sums depend on m only through S.
struct HlCfg {
    int bn = 256, S = 1;
};

// Cost in units of one K block of a 128 x 256 tile (~0.47 us measured;
// a 128 x 128 tile's block takes ~0.45 us: narrow MMAs are not cheaper,
// so narrow tiles only pay where wide ones leave SMs idle).  Fixed per
// CTA: prologue (~1.2 us) and writing its output (~4 us for a 128 x 256
// f32 tile, in proportion); a K split adds the partial tile's round trip
// through shared memory and a share of the distributed reduction.
template <int BN>
constexpr double hl_block_cost() {
    return BN == 256 ? 1.0 : BN == 128 ? 0.95 : 0.9;
}

template <int BN>
void hl_consider(int dev, int m, int n, int nb, int sms, HlCfg* best, double* best_t) {
    if (ensure_smem_attr<BN>(dev) != cudaSuccess) return;
    const long tiles = long((m + HL_BM - 1) / HL_BM) * ((n + BN - 1) / BN);
    for (int S = 1; S <= 4; ++S) {
        if (S > 1) {
            if (nb / S < 4 || tiles * S > sms) break;
            const int mc = max_active_clusters<BN>(dev, S);
            if (mc < 0 || tiles > mc) continue;
        }
        const long ctas = tiles * S, waves = (ctas + sms - 1) / sms;
        const double store = 8.5 * BN / 256.0;
        const double fixed = 2.5 + (S == 1 ? store : 3.0 + store / S);
        const double t = double(waves) * (double((nb + S - 1) / S) * hl_block_cost<BN>() + fixed);
        if (t < *best_t - 1e-9) {
            *best_t = t;
            best->bn = BN;
            best->S = S;
        }
    }
}

HlCfg hl_choose(int dev, int m, int n, int nb) {
    const int sms = sms_of(dev);
    HlCfg best;
    double t = 1e300;
    if (n > 128) hl_consider<256>(dev, m, n, nb, sms, &best, &t);
    if (n > 64) hl_consider<128>(dev, m, n, nb, sms, &best, &t);
    hl_consider<64>(dev, m, n, nb, sms, &best, &t);
    return best;
}


template <int BN>
cudaError_t launch_hl_bn(const uint16_t* ahl, const float* rowscale, int m, const uint16_t* bhl,
                         const float* colscale, int n, int nb, const float* bias, float* y, int* err_flag, int S,
                         cudaStream_t s, char* why, size_t why_len, const HlEpilogue& epi) {
    const int dev = cur_dev();
    cudaError_t e = ensure_smem_attr<BN>(dev);
    if (e != cudaSuccess) return e;
    const int mt = (m + HL_BM - 1) / HL_BM, nt = (n + BN - 1) / BN;
    // Never an empty slice.
    while (S > 1 && (S - 1) * ((nb + S - 1) / S) >= nb) --S;
    const int kps = (nb + S - 1) / S;
    CUtensorMap ma, mb, my;
    if (!encode_map(&ma, ahl, uint64_t(nb) * 64, uint64_t(m), HL_BM, why, why_len)) return cudaErrorInvalidValue;
    if (!encode_map(&mb, bhl, uint64_t(nb) * 64, uint64_t(n), BN, why, why_len)) return cudaErrorInvalidValue;
    const bool vec = (n % 4 == 0) && (reinterpret_cast<uintptr_t>(y) % 16 == 0);
    int mode = vec ? HL_STORE_VEC : HL_STORE_SCALAR;
    memset(&my, 0, sizeof my);
    if (S == 1 && vec && encode_map_f32(&my, y, uint64_t(n), uint64_t(m), why, why_len)) mode = HL_STORE_TMA;
    dim3 grid(unsigned(nt * S), unsigned(mt));
    if (S == 1)
        return launch_pdl(k_gemm_hl<BN>, grid, dim3(HL_THREADS), Hl<BN>::SMEM, s, ma, mb, my, rowscale, colscale, bias,
                          y, m, n, nb, kps, S, mode, err_flag, int(epi.gelu), epi.pos, epi.pos_period);
    return launch_pdl_cluster(k_gemm_hl<BN>, grid, dim3(HL_THREADS), Hl<BN>::SMEM, S, s, ma, mb, my, rowscale, colscale,
                              bias, y, m, n, nb, kps, S, mode, err_flag, int(epi.gelu), epi.pos, epi.pos_period);
}

}  // namespace

cudaError_t launch_split_rows(const float* a, int m, int k, int lda, bool quantize, uint16_t* ahl, float* rowscale,
                              cudaStream_t s) {
    if (m <= 0) return cudaSuccess;
    const bool vec = (reinterpret_cast<uintptr_t>(a) & 15) == 0 && lda % 4 == 0;
    auto kern = quantize ? (vec ? k_split_rows<true, true> : k_split_rows<true, false>)
                         : (vec ? k_split_rows<false, true> : k_split_rows<false, false>);
    return launch_pdl(kern, dim3(unsigned(m)), dim3(128), 0, s, a, m, k, lda, ahl, rowscale);
}

cudaError_t launch_split_dense(const float* w, int n, int k, int kv, int ldw, int n_pad, uint16_t* bhl,
                               float* colscale, cudaStream_t s) {
    if (n_pad <= 0) return cudaSuccess;
    const size_t threads = size_t(n_pad) * 32;
    k_split_dense<<<unsigned((threads + 255) / 256), 256, 0, s>>>(w, n, k, kv, ldw, n_pad, bhl, colscale);
    return cudaGetLastError();
}

cudaError_t launch_im2col_split(const float* in, int n_win, int c_in, int t_in, int t_out, int stride, size_t sw,
                                size_t sc, size_t st, int kp, uint16_t* ahl, float* rowscale, cudaStream_t s) {
    const long rows = long(n_win) * t_out;
    if (rows <= 0) return cudaSuccess;
    return launch_pdl(k_im2col_split, dim3(unsigned(rows)), dim3(128), 0, s, in, c_in, t_in, t_out, stride, sw, sc,
                      st, kp, ahl, rowscale);
}

int gemm_hl_ksplit(int m, int n, int nb) { return hl_choose(cur_dev(), m, n, nb).S; }

void set_gemm_hl_ksplit(int S) { t_ksplit_override = (S >= 1 && S <= 4) ? S : 0; }

cudaError_t launch_gemm_hl(const uint16_t* ahl, const float* rowscale, int m, const uint16_t* bhl,
                           const float* colscale, int n, int nb, const float* bias, float* y, int* err_flag,
                           cudaStream_t s, char* why, size_t why_len, const HlEpilogue* epi) {
    if (m <= 0 || n <= 0) return cudaSuccess;
    const HlEpilogue none;
    const HlEpilogue& ep = epi ? *epi : none;
    if (ep.pos && ep.pos_period <= 0) return cudaErrorInvalidValue;
    HlCfg c = hl_choose(cur_dev(), m, n, nb);
    if (t_ksplit_override > 0) c.S = t_ksplit_override;
    switch (c.bn) {
        case 256: return launch_hl_bn<256>(ahl, rowscale, m, bhl, colscale, n, nb, bias, y, err_flag, c.S, s, why, why_len, ep);
        case 128: return launch_hl_bn<128>(ahl, rowscale, m, bhl, colscale, n, nb, bias, y, err_flag, c.S, s, why, why_len, ep);
        default: return launch_hl_bn<64>(ahl, rowscale, m, bhl, colscale, n, nb, bias, y, err_flag, c.S, s, why, why_len, ep);
    }
}

}  // namespace rwq
