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
#include <cstdlib>
#include "rwq_common.cuh"
#include "rwq_decoder.h"

namespace rwq {

namespace {

constexpr int HD = 64;   // head dim (every Whisper size)

// k_new, v_new [S][D] f32 (row stride ld) -> cache [S][H][ctx][64] f16 at
// position *dpos.
__global__ void k_kv_append(const float* __restrict__ k_new, const float* __restrict__ v_new, int ld, int S, int H,
                            int ctx, const int* __restrict__ dpos, __half* __restrict__ kc, __half* __restrict__ vc) {
    pdl_trigger();
    pdl_wait();
    const int pos = *dpos;
    const int D = H * HD;
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= size_t(S) * D) return;
    const int s = int(i / D), c = int(i % D), h = c / HD, e = c % HD;
    const size_t o = ((size_t(s) * H + h) * ctx + pos) * HD + e;
    kc[o] = __float2half_rn(k_new[size_t(s) * ld + c]);
    vc[o] = __float2half_rn(v_new[size_t(s) * ld + c]);
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
                                                         const int* __restrict__ grp_streams, float* __restrict__ out,
                                                         int ldq) {
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
            const float4* qp = reinterpret_cast<const float4*>(q + size_t(grp_streams[s0 + gi]) * ldq + h * HD + e8);
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

// ------------------------------------------------- decode attention, MMA
// Decode attention on the f16 tensor cores (mma.sync m16n8k16, f32
// accumulate) for groups of up to 8 streams that share K/V (the beams of
// one window read it once; one stream per group for greedy decoding and
// the self-attention, with dpos as in k_attn_dec).  The 16 rows of the A operand
// hold each query twice: rows 0..7 its f16 high part, rows 8..15 the low
// part (q - hi), so S[g] + S[g+8] is the score with q to 22 bits, as with
// the f32 queries of k_attn_dec; P is split the same way for O = P V, and
// O[g] + O[g+8] is the output row.  K and V stay f16 as cached.
// CTA (head, group, split): 4 warps, each streaming its own 32-key K/V
// tiles (warp w: tiles w, w+4, ...) through a two-stage cp.async buffer
// (128-byte rows, 16-byte chunks swizzled by chunk ^ (row & 7) so ldmatrix
// is conflict-free), with an online softmax per query in the log2 domain;
// the warps are combined through shared memory at the end.
// Split keys (gridDim.z = splits > 1, when the (head, group) grid alone
// would leave the GPU idle): CTA z takes keys [z*L/splits, (z+1)*L/splits)
// and leaves its per-query running max, sum and 64-dim numerator in
// `part`; the CTA that finishes a (head, group) last (counter `cnt`, reset
// after use) adds the splits in split order, so the result does not depend
// on which CTA finishes when.
constexpr int TC_WARPS = 4, TC_KEYS = 32;
constexpr int TC_TILE = TC_KEYS * 128;                  // bytes of one K (or V) tile
constexpr int TC_SMEM = TC_WARPS * 2 * 2 * TC_TILE;     // warps x stages x {K, V}

__device__ __forceinline__ uint32_t tc_swz(int row, int chunk) {
    return uint32_t(row * 128 + ((chunk ^ (row & 7)) << 4));
}
__device__ __forceinline__ void tc_cp16(uint32_t dst, const void* src, bool ok) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(ok ? 16 : 0) : "memory");
}
__device__ __forceinline__ void tc_ldm4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void tc_ldm4t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void tc_mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// f16 pair of (x0, x1) and the pair of the remainders.
__device__ __forceinline__ void tc_split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(x0 - hf.x, x1 - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

// The GEMV-layout int8 quantizer of the activation row kernels
// (quant.rs:690-716) on one 32-element block held one element per lane:
// d = amax/127, inv = 1/d or 0, q = round(x*inv) half away from zero,
// clamped to +-127, NaN -> 0; sum(q) and d*sum(q).  Max and integer sums
// do not depend on the order, so the bits equal k_rows_quant's.
__device__ __forceinline__ void tc_quant32(float x, int lane, int8_t* q, float* d_out, int32_t* s_out, float* u_out) {
    float a = fabsf(x);
    a = isnan(a) ? 0.f : a;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    const float d = __fdiv_rn(a, 127.0f);
    const float inv = d > 0.f ? __fdiv_rn(1.0f, d) : 0.f;
    const float r = roundf(__fmul_rn(x, inv));
    const int c = isnan(r) ? 0 : int(fminf(127.f, fmaxf(-127.f, r)));
    q[lane] = int8_t(c);
    int sm = c;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
    if (lane == 0) {
        *d_out = d;
        *s_out = sm;
        *u_out = __fmul_rn(d, float(sm));
    }
}

__global__ void __launch_bounds__(TC_WARPS * 32) k_attn_dec_tc(const float* __restrict__ q, const __half* __restrict__ kc,
                                                              const __half* __restrict__ vc, size_t kv_stride, int L,
                                                              const int* __restrict__ dpos, int H,
                                                              const int* __restrict__ grp_kv,
                                                              const int* __restrict__ grp_off,
                                                              const int* __restrict__ grp_streams,
                                                              float* __restrict__ out, float* __restrict__ part,
                                                              unsigned* __restrict__ cnt, int ldq, AttnQuantOut qo) {
    pdl_trigger();
    extern __shared__ __align__(128) uint8_t tc_smem[];
    __shared__ float s_acc[TC_WARPS][DEC_MAX_G][HD];
    __shared__ float s_ml[TC_WARPS][DEC_MAX_G][2];
    __shared__ float s_o[DEC_MAX_G][HD];   // quantized output: the rows before quantizing
    __shared__ int s_last;
    const int h = blockIdx.x, gr = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, c = lane & 3;
    // Output element (query gi, dim e) of this head: f32, or kept for the
    // quantizer below.
    auto emit = [&](int gi, int e, float v) {
        if (qo.q8) s_o[gi][e] = v;
        else out[size_t(grp_streams[grp_off[gr] + gi]) * (H * HD) + h * HD + e] = v;
    };
    // Blocks 2h, 2h+1 of each query's row, one warp per block.
    auto quantize = [&]() {
        if (!qo.q8) return;
        __syncthreads();
        const int s0q = grp_off[gr], Gq = grp_off[gr + 1] - s0q, nbq = H * HD / QK;
        for (int i = warp; i < 2 * Gq; i += TC_WARPS) {
            const int gi = i >> 1, half = i & 1, st = grp_streams[s0q + gi], kb = 2 * h + half;
            tc_quant32(s_o[gi][half * 32 + lane], lane, qo.q8 + size_t(st) * (H * HD) + kb * QK,
                       qo.d + size_t(st) * nbq + kb, qo.sum + size_t(st) * nbq + kb, qo.u + size_t(st) * nbq + kb);
        }
    };
    const int splits = int(gridDim.z), sp = int(blockIdx.z);
    // Cross-attention (no position): its K/V and group maps are written once
    // when the decode begins, so its first K/V tile is requested before the
    // wait for the predecessor (which produces the queries).
    const bool early = dpos == nullptr;
    if (!early) {
        pdl_wait();
        L = min(*dpos + 1, L);   // self-attention: keys 0..pos (L is the cache capacity)
    }
    const int s0 = grp_off[gr], G = grp_off[gr + 1] - s0;
    if (G <= 0) return;
    const int k_lo = int(int64_t(sp) * L / splits), k_hi = int(int64_t(sp + 1) * L / splits);
    const __half* K = kc + (size_t(grp_kv[gr]) * H + h) * kv_stride;
    const __half* V = vc + (size_t(grp_kv[gr]) * H + h) * kv_stride;
    const uint32_t sb = uint32_t(__cvta_generic_to_shared(tc_smem)) + uint32_t(warp * 4 * TC_TILE);
    // stage st: K tile at sb + st*2*TC_TILE, the V tile after it
    auto load = [&](int t, int st) {
        const int r0 = k_lo + t * TC_KEYS;
        const uint32_t dk = sb + uint32_t(st * 2 * TC_TILE), dv = dk + TC_TILE;
#pragma unroll
        for (int i = 0; i < TC_KEYS * 8 / 32; ++i) {
            const int idx = lane + 32 * i, row = idx >> 3, ch = idx & 7;
            const bool ok = r0 + row < k_hi;
            const size_t o = size_t(ok ? r0 + row : 0) * HD + ch * 8;
            tc_cp16(dk + tc_swz(row, ch), K + o, ok);
            tc_cp16(dv + tc_swz(row, ch), V + o, ok);
        }
    };
    const int ntiles = (k_hi - k_lo + TC_KEYS - 1) / TC_KEYS;
    if (early) {
        if (warp < ntiles) load(warp, 0);
        asm volatile("cp.async.commit_group;" ::: "memory");
        pdl_wait();
    }
    // A fragments of the queries (scaled by log2(e)/8): row g = hi, g+8 = lo.
    const float L2E = 1.4426950408889634f;
    uint32_t qa[4][4];
    {
        const bool live = g < G;
        const float* qp = q + size_t(live ? grp_streams[s0 + g] : 0) * ldq + h * HD;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const float2 v = live ? __ldg(reinterpret_cast<const float2*>(qp + kk * 16 + u * 8 + 2 * c))
                                      : make_float2(0.f, 0.f);
                tc_split2(__fmul_rn(v.x, 0.125f) * L2E, __fmul_rn(v.y, 0.125f) * L2E, qa[kk][2 * u], qa[kk][2 * u + 1]);
            }
    }
    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m = -INFINITY, l = 0.f;   // query g (the four lanes of one g agree on m)
    if (!early) {
        if (warp < ntiles) load(warp, 0);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int t = warp, it = 0; t < ntiles; t += TC_WARPS, ++it) {
        const int st = it & 1;
        if (t + TC_WARPS < ntiles) load(t + TC_WARPS, st ^ 1);
        asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        __syncwarp();
        const uint32_t sk = sb + uint32_t(st * 2 * TC_TILE), sv = sk + TC_TILE;
        // S = Q K^T over 32 keys: s[nt] keys nt*8 + 2c, +1; [0,1] hi row, [2,3] lo row
        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
            for (int np = 0; np < 2; ++np) {
                uint32_t b[4];
                const int mi = lane >> 3, key = np * 16 + (lane & 7) + (mi >> 1) * 8, ch = kk * 2 + (mi & 1);
                tc_ldm4(sk + tc_swz(key, ch), b);
                tc_mma(s[2 * np], qa[kk], b[0], b[1]);
                tc_mma(s[2 * np + 1], qa[kk], b[2], b[3]);
            }
        const int kb = k_lo + t * TC_KEYS;
        float sc[4][2], mx = m;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int key = kb + nt * 8 + 2 * c + e;
                sc[nt][e] = key < k_hi ? s[nt][e] + s[nt][2 + e] : -INFINITY;
                mx = fmaxf(mx, sc[nt][e]);
            }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float alpha = exp2f(m - mx);   // 0 on the first tile (m = -inf)
        m = mx;
        l *= alpha;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) o[nt][e] *= alpha;
        // O += P V with P split hi (row g) / lo (row g+8)
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            float p[2][2];
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    p[hh][e] = exp2f(sc[2 * kk + hh][e] - mx);
                    l += p[hh][e];
                }
            uint32_t a[4];
            tc_split2(p[0][0], p[0][1], a[0], a[1]);
            tc_split2(p[1][0], p[1][1], a[2], a[3]);
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                uint32_t b[4];
                const int mi = lane >> 3, key = kk * 16 + (lane & 7) + (mi & 1) * 8, ch = np * 2 + (mi >> 1);
                tc_ldm4t(sv + tc_swz(key, ch), b);
                tc_mma(o[2 * np], a, b[0], b[1]);
                tc_mma(o[2 * np + 1], a, b[2], b[3]);
            }
        }
        __syncwarp();
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    if (g < G) {
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            s_acc[warp][g][nt * 8 + 2 * c] = o[nt][0] + o[nt][2];
            s_acc[warp][g][nt * 8 + 2 * c + 1] = o[nt][1] + o[nt][3];
        }
        if (c == 0) {
            s_ml[warp][g][0] = m;
            s_ml[warp][g][1] = l;
        }
    }
    __syncthreads();
    constexpr int REC = HD + 2;   // part record: {max, sum, numerator[64]}
    auto rec = [&](int z, int gi) {
        return part + ((size_t(gr) * splits + z) * H + h) * size_t(DEC_MAX_G * REC) + size_t(gi) * REC;
    };
    for (int i = tid; i < G * HD; i += TC_WARPS * 32) {
        const int gi = i / HD, e = i % HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < TC_WARPS; ++w) M = fmaxf(M, s_ml[w][gi][0]);
        float num = 0.f, den = 0.f;
#pragma unroll
        for (int w = 0; w < TC_WARPS; ++w) {
            const float f = s_ml[w][gi][0] == -INFINITY ? 0.f : exp2f(s_ml[w][gi][0] - M);
            num = fmaf(s_acc[w][gi][e], f, num);
            den = fmaf(s_ml[w][gi][1], f, den);
        }
        if (splits == 1) {
            emit(gi, e, num / den);
        } else {
            float* r = rec(sp, gi);
            r[2 + e] = num;
            if (e == 0) {
                r[0] = M;
                r[1] = den;
            }
        }
    }
    if (splits == 1) {
        quantize();
        return;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(cnt + size_t(gr) * H + h, 1u) == unsigned(splits - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int i = tid; i < G * HD; i += TC_WARPS * 32) {
        const int gi = i / HD, e = i % HD;
        float M = -INFINITY;
        for (int z = 0; z < splits; ++z) M = fmaxf(M, __ldcg(rec(z, gi)));
        float num = 0.f, den = 0.f;
        for (int z = 0; z < splits; ++z) {
            const float* r = rec(z, gi);
            const float mz = __ldcg(r);
            const float f = mz == -INFINITY ? 0.f : exp2f(mz - M);
            num = fmaf(__ldcg(r + 2 + e), f, num);
            den = fmaf(__ldcg(r + 1), f, den);
        }
        emit(gi, e, num / den);
    }
    if (tid == 0) cnt[size_t(gr) * H + h] = 0u;   // ready for the next launch
    quantize();
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

cudaError_t launch_kv_append(const float* k_new, const float* v_new, int ld, int S, int H, int ctx, const int* dpos,
                             __half* kc, __half* vc, cudaStream_t s) {
    const size_t total = size_t(S) * H * HD;
    if (!total) return cudaSuccess;
    return launch_pdl(k_kv_append, dim3(unsigned((total + 255) / 256)), dim3(256), 0, s, k_new, v_new, ld, S, H, ctx,
                      dpos, kc, vc);
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
                            const int* grp_streams, float* out, int splits, float* part, unsigned* cnt, int ldq,
                            const AttnQuantOut* qout, cudaStream_t s) {
    if (!n_groups || !L) return cudaSuccess;
    if (max_group > DEC_MAX_G || splits < 1 || splits > 8 || (splits > 1 && (!part || !cnt || max_group <= 1)))
        return cudaErrorInvalidValue;
    const dim3 grid = dim3(unsigned(H), unsigned(n_groups), unsigned(splits));
    // The tensor-core kernel for every group (config 5's single-stream
    // cross-attention: 15.4 instead of 17.9 ms per decode step);
    // RWQ_ATTN_TC=0 keeps single-stream groups on the CUDA-core kernel
    // (measurements).
    static int use_tc = -1;
    if (use_tc < 0) {
        const char* e = getenv("RWQ_ATTN_TC");
        use_tc = (e && e[0] == '0') ? 0 : 1;
    }
    if (max_group > 1 || use_tc) {
        static unsigned attr_mask = 0;
        int dev = 0;
        cudaGetDevice(&dev);
        if (!(attr_mask & (1u << (dev & 31)))) {
            const cudaError_t e =
                cudaFuncSetAttribute(k_attn_dec_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
            if (e != cudaSuccess) return e;
            attr_mask |= 1u << (dev & 31);
        }
        return launch_pdl(k_attn_dec_tc, grid, dim3(TC_WARPS * 32), size_t(TC_SMEM), s, q, kc, vc, kv_stride, L, dpos,
                          H, grp_kv, grp_off, grp_streams, out, part, cnt, ldq, qout ? *qout : AttnQuantOut{});
    }
    if (qout) return cudaErrorNotSupported;   // the CUDA-core kernel writes f32 only
    return launch_pdl(k_attn_dec<1>, grid, dim3(DEC_THREADS), 0, s, q, kc, vc, kv_stride, L, dpos, H, grp_kv, grp_off,
                      grp_streams, out, ldq);
}

bool attn_dec_quantizes(int max_group) {
    (void)max_group;
    static int use_tc = -1;
    if (use_tc < 0) {
        const char* e = getenv("RWQ_ATTN_TC");
        use_tc = (e && e[0] == '0') ? 0 : 1;
    }
    return max_group > 1 || use_tc;
}

int attn_dec_splits(int H, int n_groups, int max_group, int L, int sms) {
    if (max_group <= 1) return 1;
    if (const char* e = getenv("RWQ_ATTN_SPLITS")) {   // fixed split count (sweeps)
        const int z = atoi(e);
        if (z >= 1 && z <= 8) return z;
    }
    // Split only when the (head, group) grid alone leaves SMs without a
    // CTA (measured on config 4, 256 CTAs: no split 2.84 ms per step, 2-6
    // splits 3.06-3.15 ms).
    const long ctas = long(H) * n_groups;
    int z = int((long(sms) + ctas - 1) / ctas);
    z = z < 1 ? 1 : (z > 8 ? 8 : z);
    while (z > 1 && L / z < 128) --z;
    return z;
}

cudaError_t launch_argmax(const float* logits, int rows, int V, int limit, int32_t* best, cudaStream_t s) {
    if (!rows) return cudaSuccess;
    return launch_pdl(k_argmax, dim3(unsigned(rows)), dim3(256), 0, s, logits, V, limit, best);
}

}  // namespace rwq
