// rwq_decoder_kernels.cu -- device kernels of the KV-cached decoder step
// (reference decoder.rs:102-206) besides the quantized linears:
//   * k_kv_append: a step's new self-attention K/V rows into the per-stream
//     f16 caches (decoder.rs:159-163);
//   * k_attn_dec: attention of one new query per stream over cached keys
//     (self: the stream's own cache, causal by construction; cross: the
//     window's encoder K/V, shared by all streams decoding that window, so
//     a CTA reads each window's K/V once for all of them);
//   * k_argmax: greedy choice over the logits (decoder.rs:339-367).
#include <cuda_fp16.h>
#include <cstdint>
#include "rwq_common.cuh"
#include "rwq_decoder.h"

namespace rwq {

namespace {

constexpr int HD = 64;   // head dim (every Whisper size)

// k_new, v_new [S][D] f32 -> cache [S][H][ctx][64] f16 at position *dpos.
__global__ void k_kv_append(const float* __restrict__ k_new, const float* __restrict__ v_new, int S, int H, int ctx,
                            const int* __restrict__ dpos, __half* __restrict__ kc, __half* __restrict__ vc) {
    pdl_trigger();
    pdl_wait();
    const int pos = *dpos;
    const int D = H * HD;
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= size_t(S) * D) return;
    const int s = int(i / D), c = int(i % D), h = c / HD, e = c % HD;
    const size_t o = ((size_t(s) * H + h) * ctx + pos) * HD + e;
    kc[o] = __float2half_rn(k_new[i]);
    vc[o] = __float2half_rn(v_new[i]);
}

// One CTA per (head, group).  Group g reads the keys/values at
// kc/vc + (grp_kv[g]*H + h)*kv_stride (f16 [L][64]) for its streams
// grp_streams[grp_off[g] .. grp_off[g+1]) (at most DEC_MAX_G).  Scores stay in shared memory; q is scaled by 1/8
// (1/sqrt(64), exact) as the reference scales the scores (encoder.rs:58).
constexpr int DEC_THREADS = 256;

__global__ void __launch_bounds__(DEC_THREADS) k_attn_dec(const float* __restrict__ q, const __half* __restrict__ kc,
                                                         const __half* __restrict__ vc, size_t kv_stride, int L,
                                                         const int* __restrict__ dpos, int H,
                                                         const int* __restrict__ grp_kv, const int* __restrict__ grp_off,
                                                         const int* __restrict__ grp_streams, float* __restrict__ out) {
    pdl_trigger();
    extern __shared__ __align__(16) float sm[];
    const int h = blockIdx.x, g = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int D = H * HD;
    pdl_wait();
    if (dpos) L = min(*dpos + 1, L);   // self-attention: keys 0..pos (L is the cache capacity)
    const int s0 = grp_off[g], G = grp_off[g + 1] - s0;
    if (G <= 0) return;
    constexpr int PH = DEC_THREADS / 32;          // key phases of the output pass (one per warp)
    float* sq = sm;                               // [G][64] scaled queries
    float* part = sq + DEC_MAX_G * HD;            // [PH][G][64] partial outputs
    float* sums = part + PH * DEC_MAX_G * HD;     // [G] softmax denominators
    float* sc = sums + DEC_MAX_G;                 // [G][L] scores, then probabilities
    for (int i = tid; i < G * HD; i += DEC_THREADS) {
        const int gi = i / HD, e = i % HD;
        sq[i] = __fmul_rn(q[size_t(grp_streams[s0 + gi]) * D + h * HD + e], 0.125f);
    }
    __syncthreads();
    const __half* K = kc + (size_t(grp_kv[g]) * H + h) * kv_stride;
    const __half* V = vc + (size_t(grp_kv[g]) * H + h) * kv_stride;
    // scores: 8 lanes per key (16 bytes = 8 dims each), so a warp
    // instruction reads four whole 128-byte key rows; warp w takes keys
    // 4w + 32t .. 4w + 32t + 3, two rounds in flight.
    {
        const int kq = lane >> 3, e8 = (lane & 7) * 8;
        float qv[DEC_MAX_G][8];
#pragma unroll
        for (int gi = 0; gi < DEC_MAX_G; ++gi)
#pragma unroll
            for (int t = 0; t < 8; ++t) qv[gi][t] = gi < G ? sq[gi * HD + e8 + t] : 0.f;
#pragma unroll 2
        for (int j0 = warp * 4; j0 < L; j0 += 4 * (DEC_THREADS / 32)) {
            const int j = j0 + kq;
            float kf[8];
            if (j < L) {
                const uint4 u = __ldg(reinterpret_cast<const uint4*>(K + size_t(j) * HD + e8));
                const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&wv[t]));
                    kf[2 * t] = f.x;
                    kf[2 * t + 1] = f.y;
                }
            } else {
#pragma unroll
                for (int t = 0; t < 8; ++t) kf[t] = 0.f;
            }
#pragma unroll
            for (int gi = 0; gi < DEC_MAX_G; ++gi) {
                if (gi < G) {
                    float a = 0.f;
#pragma unroll
                    for (int t = 0; t < 8; ++t) a = fmaf(qv[gi][t], kf[t], a);
                    a += __shfl_xor_sync(0xffffffffu, a, 1);
                    a += __shfl_xor_sync(0xffffffffu, a, 2);
                    a += __shfl_xor_sync(0xffffffffu, a, 4);
                    if ((lane & 7) == 0 && j < L) sc[size_t(gi) * L + j] = a;
                }
            }
        }
    }
    __syncthreads();
    // softmax per query: one warp each
    for (int gi = warp; gi < G; gi += DEC_THREADS / 32) {
        float* row = sc + size_t(gi) * L;
        float mx = -INFINITY;
        for (int j = lane; j < L; j += 32) mx = fmaxf(mx, row[j]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.f;
        for (int j = lane; j < L; j += 32) {
            const float p = expf(row[j] - mx);
            row[j] = p;
            sum += p;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) sums[gi] = sum;
    }
    __syncthreads();
    // out[g][e] = sum_j p[g][j] v[j][e]: a warp instruction reads four
    // whole 128-byte rows (lane: key j0 + lane/8, dims 8*(lane%8)..+7);
    // warp w takes keys 4w + 32t .. 4w + 32t + 3.
    const int kq = lane >> 3, e8 = (lane & 7) * 8;
    float acc[DEC_MAX_G][8];
#pragma unroll
    for (int gi = 0; gi < DEC_MAX_G; ++gi)
#pragma unroll
        for (int t = 0; t < 8; ++t) acc[gi][t] = 0.f;
#pragma unroll 4
    for (int j0 = warp * 4; j0 < L; j0 += 4 * PH) {
        const int j = j0 + kq;
        if (j < L) {
            const uint4 u = __ldg(reinterpret_cast<const uint4*>(V + size_t(j) * HD + e8));
            const uint32_t wv[4] = {u.x, u.y, u.z, u.w};
            float v[8];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&wv[t]));
                v[2 * t] = f.x;
                v[2 * t + 1] = f.y;
            }
#pragma unroll
            for (int gi = 0; gi < DEC_MAX_G; ++gi)
                if (gi < G) {
                    const float p = sc[size_t(gi) * L + j];
#pragma unroll
                    for (int t = 0; t < 8; ++t) acc[gi][t] = fmaf(p, v[t], acc[gi][t]);
                }
        }
    }
    // lanes with the same dims (4 keys) then warps (phases) are summed
#pragma unroll
    for (int gi = 0; gi < DEC_MAX_G; ++gi)
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            acc[gi][t] += __shfl_xor_sync(0xffffffffu, acc[gi][t], 8);
            acc[gi][t] += __shfl_xor_sync(0xffffffffu, acc[gi][t], 16);
        }
    if (kq == 0) {
#pragma unroll
        for (int gi = 0; gi < DEC_MAX_G; ++gi)
            if (gi < G) {
                float* dst = part + (size_t(warp) * G + gi) * HD + e8;
                *reinterpret_cast<float4*>(dst) = make_float4(acc[gi][0], acc[gi][1], acc[gi][2], acc[gi][3]);
                *reinterpret_cast<float4*>(dst + 4) = make_float4(acc[gi][4], acc[gi][5], acc[gi][6], acc[gi][7]);
            }
    }
    __syncthreads();
    for (int i = tid; i < G * HD; i += DEC_THREADS) {
        const int gi = i / HD, ee = i % HD;
        float a = 0.f;
        for (int p = 0; p < PH; ++p) a += part[(size_t(p) * G + gi) * HD + ee];
        out[size_t(grp_streams[s0 + gi]) * D + h * HD + ee] = a / sums[gi];
    }
}

// Greedy choice (decoder.rs:345-365): the first maximum over ids
// [0, limit), taken only if it is strictly above logits[limit]; else limit.
// limit < 0: the first maximum over the whole row.
__global__ void __launch_bounds__(256) k_argmax(const float* __restrict__ logits, int V, int limit,
                                                int32_t* __restrict__ best) {
    pdl_trigger();
    pdl_wait();
    const float* row = logits + size_t(blockIdx.x) * V;
    const int n = limit >= 0 ? limit : V;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
        const float v = row[j];
        if (v > bv || (v == bv && j < bi)) {
            bv = v;
            bi = j;
        }
    }
    __shared__ float sv[8];
    __shared__ int si[8];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = bv;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < int(blockDim.x >> 5); ++w)
            if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) {
                bv = sv[w];
                bi = si[w];
            }
        if (limit >= 0 && limit < V) best[blockIdx.x] = (bi < n && bv > row[limit]) ? bi : limit;
        else best[blockIdx.x] = bi < n ? bi : 0;
    }
}

}  // namespace

size_t attn_dec_smem(int L) {
    return (size_t(DEC_MAX_G) * HD * (1 + DEC_THREADS / 32) + DEC_MAX_G + size_t(DEC_MAX_G) * L) * 4;
}

cudaError_t launch_kv_append(const float* k_new, const float* v_new, int S, int H, int ctx, const int* dpos,
                             __half* kc, __half* vc, cudaStream_t s) {
    const size_t total = size_t(S) * H * HD;
    if (!total) return cudaSuccess;
    return launch_pdl(k_kv_append, dim3(unsigned((total + 255) / 256)), dim3(256), 0, s, k_new, v_new, S, H, ctx, dpos,
                      kc, vc);
}

// *dpos += 1 (the decode position, advanced on the device so that a step
// can be replayed from a CUDA graph).
__global__ void k_pos_advance(int* dpos) {
    pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) *dpos += 1;
}

cudaError_t launch_pos_advance(int* dpos, cudaStream_t s) {
    return launch_pdl(k_pos_advance, dim3(1), dim3(32), 0, s, dpos);
}

cudaError_t launch_attn_dec(const float* q, const __half* kc, const __half* vc, size_t kv_stride, int L,
                            const int* dpos, int H, int n_groups, const int* grp_kv, const int* grp_off,
                            const int* grp_streams, float* out, cudaStream_t s) {
    if (!n_groups || !L) return cudaSuccess;
    const size_t smem = attn_dec_smem(L);
    static unsigned attr_dev_mask = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (smem > 48 * 1024 && !(attr_dev_mask & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(k_attn_dec, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        attr_dev_mask |= 1u << dev;
    }
    return launch_pdl(k_attn_dec, dim3(unsigned(H), unsigned(n_groups)), dim3(DEC_THREADS), smem, s, q, kc, vc,
                      kv_stride, L, dpos, H, grp_kv, grp_off, grp_streams, out);
}

cudaError_t launch_argmax(const float* logits, int rows, int V, int limit, int32_t* best, cudaStream_t s) {
    if (!rows) return cudaSuccess;
    return launch_pdl(k_argmax, dim3(unsigned(rows)), dim3(256), 0, s, logits, V, limit, best);
}

}  // namespace rwq
