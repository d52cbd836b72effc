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
//              columns; it adds every D0 run into registers, then D1, and
//              writes the tile to shared memory (the drained stage ring);
//              then all 320 threads add the K slices' tiles
//              (clusters of S CTAs, read through distributed shared memory
//              in slice order), scale, add the bias and store coalesced.
// Every wait is bounded (rwq_sm100.cuh); no load uses cluster multicast.
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

constexpr int HL_BM = 128;
constexpr int HL_A_BYTES = HL_BM * 128;     // one K block: 128 rows x (32 hi + 32 lo) f16
constexpr int HL_EPI0 = 2;                  // first epilogue warp
constexpr int HL_EPI_WARPS = 8;
constexpr int HL_THREADS = (HL_EPI0 + HL_EPI_WARPS) * 32;
constexpr int HL_DRAIN = 8;                 // K blocks per D0 run

template <int BN>
struct Hl {
    static constexpr int B_BYTES = BN * 128;
    static constexpr int STAGE_BYTES = HL_A_BYTES + B_BYTES;
    static constexpr int STAGES = BN == 256 ? 4 : BN == 128 ? 6 : 8;   // 192 KiB of stages
    // The f32 tile in shared memory: rows of BN + 4 floats, so the eight
    // rows a quarter-warp writes at once fall in distinct 16-byte banks.
    static constexpr int PITCH = BN + 4;
    static constexpr int PART_BYTES = HL_BM * PITCH * 4;
    static constexpr int TMEM_COLS = 2 * BN;              // D0 at column 0, D1 at column BN
    static constexpr int CPW = BN / 2;                    // columns per epilogue warp
    // kind::f16, D f32, A/B f16, both K-major, N>>3 at bit 17, M>>4 at bit 24.
    static constexpr uint32_t IDESC = (1u << 4) | (uint32_t(BN >> 3) << 17) | (uint32_t(HL_BM >> 4) << 24);
    struct Bars {
        uint64_t full[STAGES], empty[STAGES], d0_full, d0_empty;
        uint32_t tmem_base;
        int abort;
    };
    static constexpr int SMEM = STAGES * STAGE_BYTES + int(sizeof(Bars)) + 1024;
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
    static_assert(PART_BYTES <= STAGES * STAGE_BYTES, "the f32 tile must fit in the drained stages");
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

// grid: x = n_tiles * S (K slice = blockIdx.x % S, clusters of S CTAs along
// x when S > 1), y = m_tiles.  Slice r covers K blocks [r*kps, min(nb,
// (r+1)*kps)), never empty (the host picks S so).
template <int BN>
__global__ void __launch_bounds__(HL_THREADS, 1)
    k_gemm_hl(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const float* __restrict__ rowscale, const float* __restrict__ colscale, const float* __restrict__ bias,
              float* __restrict__ Y, int M, int N, int nb, int kps, int S, int vec_store, int* __restrict__ err_flag) {
    using F = Hl<BN>;
    constexpr int STAGES = F::STAGES, STAGE_BYTES = F::STAGE_BYTES, PITCH = F::PITCH, CPW = F::CPW;
    constexpr uint32_t IDESC = F::IDESC;
    using Bars = typename F::Bars;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    Bars* bar = reinterpret_cast<Bars*>(base + STAGES * STAGE_BYTES);
    volatile int* abort = &bar->abort;
    float* part = reinterpret_cast<float*>(base);   // the f32 tile, after the last MMA

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
            // The last D0 commit came after every MMA, D1's included.
            const int row = q * 32 + lane;
            float* prow = part + size_t(row) * PITCH;
#pragma unroll
            for (int c = 0; c < CPW; c += 16) {
                uint32_t v[16];
                tmem_ld16(tmem + lane_off + uint32_t(BN + h * CPW + c), v);
                tmem_wait_ld();
#pragma unroll
                for (int e = 0; e < 16; e += 4)
                    *reinterpret_cast<float4*>(prow + h * CPW + c + e) = make_float4(
                        __fadd_rn(acc[c + e], __uint_as_float(v[e])), __fadd_rn(acc[c + e + 1], __uint_as_float(v[e + 1])),
                        __fadd_rn(acc[c + e + 2], __uint_as_float(v[e + 2])),
                        __fadd_rn(acc[c + e + 3], __uint_as_float(v[e + 3])));
            }
        }
    }

    // Every thread of every CTA of the cluster reaches both barriers, also
    // after an expired wait, so the cluster never waits on a CTA that left.
    tc_fence_before();
    if (S > 1) hl_cluster_sync();
    else __syncthreads();

    // Slice `split` adds rows [split*RS, +RS) of the S partial tiles in
    // slice order, then y = acc * 2^-e_i * 2^-e_j (+ bias).
    const int RS = HL_BM / S;
    const int r0 = split * RS;
    if (!*abort) {
        const uint32_t part_s = smem_u32(part);
        constexpr int C4 = BN / 4;
        for (int idx = threadIdx.x; idx < RS * C4; idx += HL_THREADS) {
            const int rr = r0 + idx / C4, c = (idx % C4) * 4;
            const int gi = m0 + rr, gj = n0 + c;
            if (gi >= M || gj >= N) continue;
            const uint32_t off = uint32_t((rr * PITCH + c) * 4);
            float4 acc;
            if (S == 1) {
                acc = *reinterpret_cast<const float4*>(part + rr * PITCH + c);
            } else {
                acc = hl_ld_cluster4(hl_mapa(part_s + off, 0));
                for (int s2 = 1; s2 < S; ++s2) {
                    const float4 t = hl_ld_cluster4(hl_mapa(part_s + off, uint32_t(s2)));
                    acc.x = __fadd_rn(acc.x, t.x);
                    acc.y = __fadd_rn(acc.y, t.y);
                    acc.z = __fadd_rn(acc.z, t.z);
                    acc.w = __fadd_rn(acc.w, t.w);
                }
            }
            const float rs = __ldg(rowscale + gi);
            const float4 cs = __ldg(reinterpret_cast<const float4*>(colscale + gj));   // padded, 16-byte aligned
            float4 v = make_float4(__fmul_rn(__fmul_rn(acc.x, cs.x), rs), __fmul_rn(__fmul_rn(acc.y, cs.y), rs),
                                   __fmul_rn(__fmul_rn(acc.z, cs.z), rs), __fmul_rn(__fmul_rn(acc.w, cs.w), rs));
            float* yr = Y + size_t(gi) * N + gj;
            if (vec_store) {   // N % 4 == 0 and Y 16-byte aligned: gj + 3 < N
                if (bias) {
                    v.x = __fadd_rn(v.x, __ldg(bias + gj));
                    v.y = __fadd_rn(v.y, __ldg(bias + gj + 1));
                    v.z = __fadd_rn(v.z, __ldg(bias + gj + 2));
                    v.w = __fadd_rn(v.w, __ldg(bias + gj + 3));
                }
                *reinterpret_cast<float4*>(yr) = v;
            } else {
                const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    if (gj + e < N) yr[e] = bias ? __fadd_rn(vv[e], __ldg(bias + gj + e)) : vv[e];
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

struct DevInfo {
    int sms = 0;
    int max_clusters[3][3] = {};   // [BN index][S index: 2, 4] (0 = not queried)
    bool attr[3] = {};
};
DevInfo g_dev[64];
std::mutex g_dev_mu;

template <int BN>
constexpr int bn_index() {
    return BN == 64 ? 0 : BN == 128 ? 1 : 2;
}

template <int BN>
int max_active_clusters(int dev, int S) {
    std::lock_guard<std::mutex> g(g_dev_mu);
    DevInfo& di = g_dev[dev];
    int& slot = di.max_clusters[bn_index<BN>()][S == 2 ? 0 : 1];
    if (slot == 0) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(unsigned(S) * 64, 1);
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

// K slices of an m x n GEMM with nb blocks: double while the CTAs still fit
// in one wave, every slice keeps at least 4 blocks, and all clusters can be
// resident at once.  A row's sums depend on m only through this choice.
template <int BN>
int ksplit_bn(int dev, int m, int n, int nb) {
    if (ensure_smem_attr<BN>(dev) != cudaSuccess) return 1;
    const int sms = sms_of(dev);
    const long tiles = long((m + HL_BM - 1) / HL_BM) * ((n + BN - 1) / BN);
    int S = 1;
    while (S < 4 && tiles * S * 2 <= sms && nb / (S * 2) >= 4) {
        const int mc = max_active_clusters<BN>(dev, S * 2);
        if (mc < 0 || tiles > mc) break;
        S *= 2;
    }
    return S;
}

int cur_dev() {
    int dev = 0;
    cudaGetDevice(&dev);
    return dev < 64 ? dev : 63;
}

template <int BN>
cudaError_t launch_hl_bn(const uint16_t* ahl, const float* rowscale, int m, const uint16_t* bhl,
                         const float* colscale, int n, int nb, const float* bias, float* y, int* err_flag,
                         cudaStream_t s, char* why, size_t why_len) {
    const int dev = cur_dev();
    cudaError_t e = ensure_smem_attr<BN>(dev);
    if (e != cudaSuccess) return e;
    const int mt = (m + HL_BM - 1) / HL_BM, nt = (n + BN - 1) / BN;
    int S = t_ksplit_override > 0 ? t_ksplit_override : ksplit_bn<BN>(dev, m, n, nb);
    // Never an empty slice.
    while (S > 1 && (S - 1) * ((nb + S - 1) / S) >= nb) S /= 2;
    const int kps = (nb + S - 1) / S;
    CUtensorMap ma, mb;
    if (!encode_map(&ma, ahl, uint64_t(nb) * 64, uint64_t(m), HL_BM, why, why_len)) return cudaErrorInvalidValue;
    if (!encode_map(&mb, bhl, uint64_t(nb) * 64, uint64_t(n), BN, why, why_len)) return cudaErrorInvalidValue;
    const int vec = (n % 4 == 0) && (reinterpret_cast<uintptr_t>(y) % 16 == 0);
    dim3 grid(unsigned(nt * S), unsigned(mt));
    if (S == 1)
        return launch_pdl(k_gemm_hl<BN>, grid, dim3(HL_THREADS), Hl<BN>::SMEM, s, ma, mb, rowscale, colscale, bias, y,
                          m, n, nb, kps, S, vec, err_flag);
    return launch_pdl_cluster(k_gemm_hl<BN>, grid, dim3(HL_THREADS), Hl<BN>::SMEM, S, s, ma, mb, rowscale, colscale,
                              bias, y, m, n, nb, kps, S, vec, err_flag);
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

int gemm_hl_ksplit(int m, int n, int nb) {
    const int dev = cur_dev();
    if (n > 128) return ksplit_bn<256>(dev, m, n, nb);
    if (n > 64) return ksplit_bn<128>(dev, m, n, nb);
    return ksplit_bn<64>(dev, m, n, nb);
}

void set_gemm_hl_ksplit(int S) { t_ksplit_override = (S == 1 || S == 2 || S == 4) ? S : 0; }

cudaError_t launch_gemm_hl(const uint16_t* ahl, const float* rowscale, int m, const uint16_t* bhl,
                           const float* colscale, int n, int nb, const float* bias, float* y, int* err_flag,
                           cudaStream_t s, char* why, size_t why_len) {
    if (m <= 0 || n <= 0) return cudaSuccess;
    if (n > 128) return launch_hl_bn<256>(ahl, rowscale, m, bhl, colscale, n, nb, bias, y, err_flag, s, why, why_len);
    if (n > 64) return launch_hl_bn<128>(ahl, rowscale, m, bhl, colscale, n, nb, bias, y, err_flag, s, why, why_len);
    return launch_hl_bn<64>(ahl, rowscale, m, bhl, colscale, n, nb, bias, y, err_flag, s, why, why_len);
}

}  // namespace rwq
