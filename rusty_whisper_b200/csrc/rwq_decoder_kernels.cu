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
// grp_streams[grp_off[g] .. grp_off[g+1]) (at most DEC_MAX_G).  One pass
// over K and V with an online softmax (flash decoding): warp w streams keys
// 4w + 32t .. 4w + 32t + 3, 8 lanes per key with 16-byte loads of the K and
// V rows, keeping a running max, sum and 8-dim partial output per query;
// the 8 warps combine through shared memory at the end.  q is scaled by
// 1/8 (1/sqrt(64), exact) as the reference scales the scores
// (encoder.rs:58); exponentials are base 2 on log2(e)-scaled scores.
constexpr int DEC_THREADS = 256;
constexpr int DEC_WARPS = DEC_THREADS / 32;

__device__ __forceinline__ void h8_to_f(const uint4 u, float (&f)[8]) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&w[t]));
        f[2 * t] = x.x;
        f[2 * t + 1] = x.y;
    }
}

template <int GM>
__global__ void __launch_bounds__(DEC_THREADS) k_attn_dec(const float* __restrict__ q, const __half* __restrict__ kc,
                                                         const __half* __restrict__ vc, size_t kv_stride, int L,
                                                         const int* __restrict__ dpos, int H,
                                                         const int* __restrict__ grp_kv, const int* __restrict__ grp_off,
                                                         const int* __restrict__ grp_streams, float* __restrict__ out) {
    pdl_trigger();
    __shared__ float s_acc[DEC_WARPS][GM][HD];
    __shared__ float s_ml[DEC_WARPS][GM][2];
    const int h = blockIdx.x, g = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int D = H * HD;
    pdl_wait();
    if (dpos) L = min(*dpos + 1, L);   // self-attention: keys 0..pos (L is the cache capacity)
    const int s0 = grp_off[g], G = grp_off[g + 1] - s0;
    if (G <= 0) return;
    const float L2E = 1.4426950408889634f;
    const int kq = lane >> 3, e8 = (lane & 7) * 8;
    // this lane's 8 query dims, scaled by 1/8 and log2(e)
    float qv[GM][8];
#pragma unroll
    for (int gi = 0; gi < GM; ++gi) {
        if (gi < G) {
            const float4* qp = reinterpret_cast<const float4*>(q + size_t(grp_streams[s0 + gi]) * D + h * HD + e8);
            const float4 a = __ldg(qp), b = __ldg(qp + 1);
            const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int t = 0; t < 8; ++t) qv[gi][t] = __fmul_rn(v[t], 0.125f) * L2E;
        } else {
#pragma unroll
            for (int t = 0; t < 8; ++t) qv[gi][t] = 0.f;
        }
    }
    const __half* K = kc + (size_t(grp_kv[g]) * H + h) * kv_stride;
    const __half* V = vc + (size_t(grp_kv[g]) * H + h) * kv_stride;
    float m[GM], l[GM], acc[GM][8];
#pragma unroll
    for (int gi = 0; gi < GM; ++gi) {
        m[gi] = -INFINITY;
        l[gi] = 0.f;
#pragma unroll
        for (int t = 0; t < 8; ++t) acc[gi][t] = 0.f;
    }
#pragma unroll 2
    for (int j0 = warp * 4; j0 < L; j0 += 4 * DEC_WARPS) {
        const int j = j0 + kq;
        float kf[8], vf[8];
        if (j < L) {
            h8_to_f(__ldg(reinterpret_cast<const uint4*>(K + size_t(j) * HD + e8)), kf);
            h8_to_f(__ldg(reinterpret_cast<const uint4*>(V + size_t(j) * HD + e8)), vf);
        } else {
#pragma unroll
            for (int t = 0; t < 8; ++t) kf[t] = vf[t] = 0.f;
        }
#pragma unroll
        for (int gi = 0; gi < GM; ++gi) {
            if (gi < G) {
                float sc = 0.f;
#pragma unroll
                for (int t = 0; t < 8; ++t) sc = fmaf(qv[gi][t], kf[t], sc);
                sc += __shfl_xor_sync(0xffffffffu, sc, 1);
                sc += __shfl_xor_sync(0xffffffffu, sc, 2);
                sc += __shfl_xor_sync(0xffffffffu, sc, 4);
                if (j >= L) sc = -INFINITY;
                // the four keys of this round
                float mr = fmaxf(sc, __shfl_xor_sync(0xffffffffu, sc, 8));
                mr = fmaxf(mr, __shfl_xor_sync(0xffffffffu, mr, 16));
                const float mn = fmaxf(m[gi], mr);
                const float scale = exp2f(m[gi] - mn);   // 0 on the first round (m = -inf)
                const float p = exp2f(sc - mn);
                float ps = p + __shfl_xor_sync(0xffffffffu, p, 8);
                ps += __shfl_xor_sync(0xffffffffu, ps, 16);
                l[gi] = fmaf(l[gi], scale, ps);
#pragma unroll
                for (int t = 0; t < 8; ++t) acc[gi][t] = fmaf(acc[gi][t], scale, p * vf[t]);
                m[gi] = mn;
            }
        }
    }
    // lanes with the same dims (the four key slots) share m: sum their parts
#pragma unroll
    for (int gi = 0; gi < GM; ++gi)
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            acc[gi][t] += __shfl_xor_sync(0xffffffffu, acc[gi][t], 8);
            acc[gi][t] += __shfl_xor_sync(0xffffffffu, acc[gi][t], 16);
        }
    if (kq == 0) {
#pragma unroll
        for (int gi = 0; gi < GM; ++gi)
            if (gi < G) {
#pragma unroll
                for (int t = 0; t < 8; ++t) s_acc[warp][gi][e8 + t] = acc[gi][t];
                if (lane == 0) {
                    s_ml[warp][gi][0] = m[gi];
                    s_ml[warp][gi][1] = l[gi];
                }
            }
    }
    __syncthreads();
    for (int i = tid; i < G * HD; i += DEC_THREADS) {
        const int gi = i / HD, e = i % HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < DEC_WARPS; ++w) M = fmaxf(M, s_ml[w][gi][0]);
        float num = 0.f, den = 0.f;
#pragma unroll
        for (int w = 0; w < DEC_WARPS; ++w) {
            const float f = s_ml[w][gi][0] == -INFINITY ? 0.f : exp2f(s_ml[w][gi][0] - M);
            num = fmaf(s_acc[w][gi][e], f, num);
            den = fmaf(s_ml[w][gi][1], f, den);
        }
        out[size_t(grp_streams[s0 + gi]) * D + h * HD + e] = num / den;
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
                            const int* dpos, int H, int n_groups, int max_group, const int* grp_kv, const int* grp_off,
                            const int* grp_streams, float* out, cudaStream_t s) {
    if (!n_groups || !L) return cudaSuccess;
    const dim3 grid = dim3(unsigned(H), unsigned(n_groups));
    // registers scale with the queries a group may hold
    if (max_group <= 1)
        return launch_pdl(k_attn_dec<1>, grid, dim3(DEC_THREADS), 0, s, q, kc, vc, kv_stride, L, dpos, H, grp_kv,
                          grp_off, grp_streams, out);
    if (max_group <= 2)
        return launch_pdl(k_attn_dec<2>, grid, dim3(DEC_THREADS), 0, s, q, kc, vc, kv_stride, L, dpos, H, grp_kv,
                          grp_off, grp_streams, out);
    if (max_group <= 4)
        return launch_pdl(k_attn_dec<4>, grid, dim3(DEC_THREADS), 0, s, q, kc, vc, kv_stride, L, dpos, H, grp_kv,
                          grp_off, grp_streams, out);
    return launch_pdl(k_attn_dec<DEC_MAX_G>, grid, dim3(DEC_THREADS), 0, s, q, kc, vc, kv_stride, L, dpos, H, grp_kv,
                      grp_off, grp_streams, out);
}

cudaError_t launch_argmax(const float* logits, int rows, int V, int limit, int32_t* best, cudaStream_t s) {
    if (!rows) return cudaSuccess;
    return launch_pdl(k_argmax, dim3(unsigned(rows)), dim3(256), 0, s, logits, V, limit, best);
}

}  // namespace rwq
