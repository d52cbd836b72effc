// rwq_encoder_kernels.cu -- the device kernels of the encoder forward
// (reference encoder.rs:123-234) around the quantized GEMM:
//   * k_rows_quant: per row, optional residual add, LayerNorm
//     (tensor.rs:274-289) or tanh-GELU (tensor.rs:291-306), then the int8
//     activation quantizer (quant.rs:690-716) writing the tensor-core
//     GEMM's operand directly (f16 codes + transposed block scales);
//   * k_to_heads + k_attn: non-causal multi-head attention
//     (encoder.rs:48-80) as a flash-style kernel on f16 tensor-core MMAs
//     with f32 accumulation and an online softmax, so the [T, T] score
//     matrix never leaves the SM.
#include <cuda_fp16.h>
#include <atomic>
#include <cstdint>
#include "rwq_common.cuh"
#include "rwq_encoder.h"

namespace rwq {

namespace {

// One 32-element block held as 4 values by each of 8 consecutive lanes
// (lane & 7 = position): the reference quantizer (quant.rs:690-716), as
// k_quantize does it -- d = amax/127, inv = 1/d or 0, q = round(x*inv)
// half away from zero, clamped to +-127, NaN -> 0.
constexpr int RQ_WPR = 4;     // warps per row in the LayerNorm modes

struct QOut {
    uint16_t* q16;   // GEMM layout: f16 codes [m][k], d_a and d_a*sum transposed [nb][m_pad]
    float* dT;
    float* uT;
    int m_pad;
    int8_t* q8;      // GEMV layout: int8 codes [m][k], d_a, sum, d_a*sum [m][nb]
    float* d;
    int32_t* sum;
    float* u;
};

__device__ __forceinline__ void quant_block4(float4 x, int row, int k, int e, const QOut& o) {
    auto absnn = [](float v) { const float w = fabsf(v); return isnan(w) ? 0.f : w; };
    float amax = fmaxf(fmaxf(absnn(x.x), absnn(x.y)), fmaxf(absnn(x.z), absnn(x.w)));
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    const float inv = d > 0.f ? __fdiv_rn(1.0f, d) : 0.f;
    auto code = [inv](float v) {
        const float r = roundf(__fmul_rn(v, inv));
        return isnan(r) ? 0 : int(fminf(127.f, fmaxf(-127.f, r)));
    };
    const int c0 = code(x.x), c1 = code(x.y), c2 = code(x.z), c3 = code(x.w);
    int s = c0 + c1 + c2 + c3;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const int bl = e / QK, nb = k / QK;
    const float u = __fmul_rn(d, float(s));
    if (o.q16) {
        const uint32_t h01 =
            uint32_t(__half_as_ushort(__int2half_rn(c0))) | (uint32_t(__half_as_ushort(__int2half_rn(c1))) << 16);
        const uint32_t h23 =
            uint32_t(__half_as_ushort(__int2half_rn(c2))) | (uint32_t(__half_as_ushort(__int2half_rn(c3))) << 16);
        *reinterpret_cast<uint2*>(o.q16 + size_t(row) * k + e) = make_uint2(h01, h23);
        if ((threadIdx.x & 7) == 0) {
            o.dT[size_t(bl) * o.m_pad + row] = d;
            o.uT[size_t(bl) * o.m_pad + row] = u;
        }
    }
    if (o.q8) {
        *reinterpret_cast<uint32_t*>(o.q8 + size_t(row) * k + e) = uint32_t(uint8_t(c0)) | (uint32_t(uint8_t(c1)) << 8) |
                                                                 (uint32_t(uint8_t(c2)) << 16) |
                                                                 (uint32_t(uint8_t(c3)) << 24);
        if ((threadIdx.x & 7) == 0) {
            o.d[size_t(row) * nb + bl] = d;
            o.sum[size_t(row) * nb + bl] = s;
            o.u[size_t(row) * nb + bl] = u;
        }
    }
}

// Rows of k elements (k % 128 == 0) in 128-element chunks; lane l covers
// elements 4l..4l+3 of a chunk, so 8 lanes share a quant block.
// MODE: RQ_PLAIN quantize x; RQ_GELU quantize gelu(x); RQ_LN quantize
// LayerNorm(x); RQ_ADD_LN x += add (written back to xout), then as RQ_LN.
// PLAIN / GELU: each warp takes `slice` consecutive chunks of a row.
// LayerNorm: RQ_WPR warps per row (chunks c = w, w + RQ_WPR, ...; at most
// NV each, held in registers); the row statistics add each lane's chunks
// in order, then the lanes (xor tree), then the warps in order, so a row's
// result depends on k only.
// The codes go to the GEMM layout (q16/dT/uT), the GEMV layout (q8/d/sum/
// u), or both; with yout the transformed row is also written as f32 (e.g.
// ln_post).  GEMM-layout rows m..m_pad-1 get zero block scales.  x and xout may
// alias: the residual stream is updated in place.
template <int MODE, int NV>
__global__ void __launch_bounds__(256) k_rows_quant(const float* x, const float* __restrict__ add, float* xout,
                                                    const float* __restrict__ lw, const float* __restrict__ lb,
                                                    int m, int k, QOut o, float* __restrict__ yout, int slice_len) {
    constexpr bool LN = MODE == RQ_LN || MODE == RQ_ADD_LN;
    const int lane = threadIdx.x & 31;
    const int nb = k / QK, nch = k / 128;
    const int wpr = LN ? RQ_WPR : (nch + slice_len - 1) / slice_len;   // warps per row
    const size_t wg = (size_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int row = int(wg / wpr), wr = int(wg % wpr);
    // The LayerNorm's weight and bias are never written by a kernel that
    // runs as a programmatic dependent: read them before the wait, while
    // the predecessor finishes.
    float4 lwv[LN ? NV : 1], lbv[LN ? NV : 1];
    if constexpr (LN) {
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int c = wr + RQ_WPR * j;
            if (c < nch) {
                lwv[j] = __ldg(reinterpret_cast<const float4*>(lw + c * 128 + lane * 4));
                lbv[j] = __ldg(reinterpret_cast<const float4*>(lb + c * 128 + lane * 4));
            }
        }
    }
    pdl_trigger();
    pdl_wait();
    const int rows = o.q16 ? o.m_pad : m;
    const bool live = row < m;
    if (!LN && !live) {
        if (row >= rows || wr) return;
        for (int bl = lane; bl < nb; bl += 32) {
            o.dT[size_t(bl) * o.m_pad + row] = 0.f;
            o.uT[size_t(bl) * o.m_pad + row] = 0.f;
        }
        return;
    }
    const float4* xr = reinterpret_cast<const float4*>(x + size_t(row) * k);
    const bool quant = o.q16 || o.q8;
    auto emit = [&](int c, float4 v) {
        const int e = c * 128 + lane * 4;
        if (quant) quant_block4(v, row, k, e, o);
        if (yout) *reinterpret_cast<float4*>(yout + size_t(row) * k + e) = v;
    };
    if constexpr (!LN) {
        const int c1 = min(nch, (wr + 1) * slice_len);
        for (int c = wr * slice_len; c < c1; ++c) {
            float4 v = __ldg(xr + c * 32 + lane);
            if (MODE == RQ_GELU) v = make_float4(gelu_ref(v.x), gelu_ref(v.y), gelu_ref(v.z), gelu_ref(v.w));
            emit(c, v);
        }
        return;
    } else {
        // Every warp of the CTA reaches both barriers (rows past m too).
        __shared__ float s_red[256 / 32];
        const int wi = int(threadIdx.x >> 5), w0 = wi - wr;   // this row's first warp in the CTA
        float4 v[NV];
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int c = wr + RQ_WPR * j;
            if (live && c < nch) {
                v[j] = xr[c * 32 + lane];
                if (MODE == RQ_ADD_LN) {
                    const float4 a = __ldg(reinterpret_cast<const float4*>(add + size_t(row) * k) + c * 32 + lane);
                    v[j] = make_float4(__fadd_rn(v[j].x, a.x), __fadd_rn(v[j].y, a.y), __fadd_rn(v[j].z, a.z),
                                       __fadd_rn(v[j].w, a.w));
                    reinterpret_cast<float4*>(xout + size_t(row) * k)[c * 32 + lane] = v[j];
                }
                s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
            }
        }
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o2);
        if (lane == 0) s_red[wi] = s;
        __syncthreads();
        float tot = s_red[w0];
#pragma unroll
        for (int w = 1; w < RQ_WPR; ++w) tot = __fadd_rn(tot, s_red[w0 + w]);
        const float mean = __fdiv_rn(tot, float(k));
        float q = 0.f;
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int c = wr + RQ_WPR * j;
            if (live && c < nch) {
                const float a = __fsub_rn(v[j].x, mean), b = __fsub_rn(v[j].y, mean), cc = __fsub_rn(v[j].z, mean),
                            dd = __fsub_rn(v[j].w, mean);
                q += (__fmul_rn(a, a) + __fmul_rn(b, b)) + (__fmul_rn(cc, cc) + __fmul_rn(dd, dd));
            }
        }
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o2);
        __syncthreads();
        if (lane == 0) s_red[wi] = q;
        __syncthreads();
        float qt = s_red[w0];
#pragma unroll
        for (int w = 1; w < RQ_WPR; ++w) qt = __fadd_rn(qt, s_red[w0 + w]);
        if (!live) {
            if (row < rows && wr == 0)
                for (int bl = lane; bl < nb; bl += 32) {
                    o.dT[size_t(bl) * o.m_pad + row] = 0.f;
                    o.uT[size_t(bl) * o.m_pad + row] = 0.f;
                }
            return;
        }
        const float var = __fdiv_rn(qt, float(k));
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int c = wr + RQ_WPR * j;
            if (c < nch) {
                const float4 w = lwv[j], b = lbv[j];
                auto f = [&](float xv, float wv, float bv) {
                    return __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xv, mean), inv), wv), bv);
                };
                emit(c, make_float4(f(v[j].x, w.x, b.x), f(v[j].y, w.y, b.y), f(v[j].z, w.z, b.z),
                                    f(v[j].w, w.w, b.w)));
            }
        }
    }
}

// The LayerNorm modes of k_rows_quant with one warp per row, for encoder-
// sized batches: each lane holds all the row's chunks (c = 0 .. nch-1, at
// most NV), so a warp has NV loads in flight and needs no CTA barrier.  The
// statistics are added in exactly k_rows_quant's order -- per lane the
// chunks c = w, w + RQ_WPR, ... for each of the RQ_WPR chunk classes w, one
// xor tree per class, then the classes in order -- so both kernels give the
// same bits and the choice between them depends on the row count only.
template <int MODE, int NV>
__global__ void __launch_bounds__(128) k_ln_rows_warp(const float* x, const float* __restrict__ add, float* xout,
                                                      const float* __restrict__ lw, const float* __restrict__ lb,
                                                      int m, int k, QOut o, float* __restrict__ yout) {
    static_assert(MODE == RQ_LN || MODE == RQ_ADD_LN, "LayerNorm modes only");
    const int lane = threadIdx.x & 31;
    const int nb = k / QK, nch = k / 128;
    const int row = int((size_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
    pdl_trigger();
    pdl_wait();
    const int rows = o.q16 ? o.m_pad : m;
    if (row >= rows) return;
    if (row >= m) {
        for (int bl = lane; bl < nb; bl += 32) {
            o.dT[size_t(bl) * o.m_pad + row] = 0.f;
            o.uT[size_t(bl) * o.m_pad + row] = 0.f;
        }
        return;
    }
    const float4* xr = reinterpret_cast<const float4*>(x + size_t(row) * k);
    float4 v[NV];
#pragma unroll
    for (int c = 0; c < NV; ++c)
        if (c < nch) v[c] = xr[c * 32 + lane];
    if (MODE == RQ_ADD_LN) {
        const float4* ar = reinterpret_cast<const float4*>(add + size_t(row) * k);
        float4* xo = reinterpret_cast<float4*>(xout + size_t(row) * k);
#pragma unroll
        for (int c = 0; c < NV; ++c)
            if (c < nch) {
                const float4 a = __ldg(ar + c * 32 + lane);
                v[c] = make_float4(__fadd_rn(v[c].x, a.x), __fadd_rn(v[c].y, a.y), __fadd_rn(v[c].z, a.z),
                                   __fadd_rn(v[c].w, a.w));
                xo[c * 32 + lane] = v[c];
            }
    }
    // Sum of one chunk class w over this lane, then over the warp.
    auto class_sum = [&](int w, auto term) {
        float s = 0.f;
#pragma unroll
        for (int c = 0; c < NV; ++c)
            if (c % RQ_WPR == w && c < nch) s += term(v[c]);
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o2);
        return s;
    };
    auto plain = [](float4 a) { return (a.x + a.y) + (a.z + a.w); };
    float tot = class_sum(0, plain);
#pragma unroll
    for (int w = 1; w < RQ_WPR; ++w) tot = __fadd_rn(tot, class_sum(w, plain));
    const float mean = __fdiv_rn(tot, float(k));
    auto sq = [mean](float4 a) {
        const float p = __fsub_rn(a.x, mean), q = __fsub_rn(a.y, mean), r = __fsub_rn(a.z, mean),
                    t = __fsub_rn(a.w, mean);
        return (__fmul_rn(p, p) + __fmul_rn(q, q)) + (__fmul_rn(r, r) + __fmul_rn(t, t));
    };
    float qt = class_sum(0, sq);
#pragma unroll
    for (int w = 1; w < RQ_WPR; ++w) qt = __fadd_rn(qt, class_sum(w, sq));
    const float var = __fdiv_rn(qt, float(k));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, 1e-5f)));
#pragma unroll
    for (int c = 0; c < NV; ++c)
        if (c < nch) {
            // LayerNorm weights read here (L1 hits after the first rows):
            // holding them across the wait cost 30 registers and a third of
            // the resident warps
            const float4 w = __ldg(reinterpret_cast<const float4*>(lw + c * 128 + lane * 4));
            const float4 b = __ldg(reinterpret_cast<const float4*>(lb + c * 128 + lane * 4));
            auto f = [&](float xv, float wv, float bv) {
                return __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xv, mean), inv), wv), bv);
            };
            const float4 y = make_float4(f(v[c].x, w.x, b.x), f(v[c].y, w.y, b.y), f(v[c].z, w.z, b.z),
                                         f(v[c].w, w.w, b.w));
            const int e = c * 128 + lane * 4;
            if (o.q16 || o.q8) quant_block4(y, row, k, e, o);
            if (yout) *reinterpret_cast<float4*>(yout + size_t(row) * k + e) = y;
        }
}

// im2col for a kernel-3, pad-1 conv over windows: out row (w, t) holds
// in(w, ic, t*stride + j - 1) at column ic*3 + j (zero outside [0, t_in)).
// in(w, ic, t) = in[w*sw + ic*sc + t*st].
// f32 [n_win*T][ld] (head h = columns col0 + h*64 ..) -> f16 [n_win][H][T][64],
// multiplied by `scale` (a power of two: exact).
__global__ void k_to_heads(const float* __restrict__ src, int ld, int col0, int n_win, int T, int H, float scale,
                           __half* __restrict__ dst) {
    const size_t total = size_t(n_win) * H * T * 16;   // float4 groups
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
        const int c4 = int(i & 15);
        const size_t r = i >> 4;                         // (w, h, t)
        const int t = int(r % T), h = int((r / T) % H), w = int(r / (size_t(T) * H));
        const float4 v = __ldg(reinterpret_cast<const float4*>(src + (size_t(w) * T + t) * ld + col0 + h * 64) + c4);
        const __half2 a = __floats2half2_rn(__fmul_rn(v.x, scale), __fmul_rn(v.y, scale));
        const __half2 b = __floats2half2_rn(__fmul_rn(v.z, scale), __fmul_rn(v.w, scale));
        uint2 o;
        o.x = *reinterpret_cast<const uint32_t*>(&a);
        o.y = *reinterpret_cast<const uint32_t*>(&b);
        reinterpret_cast<uint2*>(dst + r * 64)[c4] = o;
    }
}

// ------------------------------------------------------------ attention
// Flash-style attention, head dim 64.  CTA: 4 warps x 16 query rows; K/V
// tiles of 64 keys in a three-stage cp.async ring in shared memory; f16
// m16n8k16 MMAs with f32 accumulators; 128-byte rows swizzled by 16-byte
// chunk (chunk ^ (row & 7)) so ldmatrix is conflict-free.
constexpr int AT_Q = 64, AT_K = 64, AT_D = 64, AT_THREADS = 128, AT_STAGES = 3;
constexpr int AT_SMEM = AT_Q * 128 + AT_STAGES * 2 * AT_K * 128;   // 56 KB: four CTAs per SM

__device__ __forceinline__ uint32_t swz(int row, int chunk) { return uint32_t(row * 128 + ((chunk ^ (row & 7)) << 4)); }

__device__ __forceinline__ void cpa16(uint32_t dst, const void* src, bool ok) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(ok ? 16 : 0) : "memory");
}

__device__ __forceinline__ void ldm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// 2^x by the MUFU.EX2 unit (PTX ex2.approx.ftz.f32: relative error about
// 2^-22, below the f16 rounding of the probabilities that use it; 2^-inf = 0).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// QOUT: the output rows quantized straight into the GEMM-layout operand of
// the next linear (o.q16, o.dT, o.uT), as the quantizer row kernel would
// write them, instead of f32 rows into `out`.
template <bool QOUT>
__global__ void __launch_bounds__(AT_THREADS, 4) k_attn(const __half* __restrict__ Qh, const __half* __restrict__ Kh,
                                                     const __half* __restrict__ Vh, int T, int H,
                                                     float* __restrict__ out, QOut qo) {
    pdl_trigger();
    extern __shared__ __align__(128) uint8_t at_smem[];   // Q tile, then AT_STAGES x (K tile, V tile)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, tig = lane & 3;
    const int w = blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * AT_Q;
    const size_t head = (size_t(w) * H + h) * size_t(T) * AT_D;
    const __half* Qb = Qh + head;
    const __half* Kb = Kh + head;
    const __half* Vb = Vh + head;
    const uint32_t sQa = uint32_t(__cvta_generic_to_shared(at_smem));
    auto sKa = [sQa](int st) { return sQa + uint32_t(AT_Q * 128 + st * 2 * AT_K * 128); };
    auto sVa = [sQa](int st) { return sQa + uint32_t(AT_Q * 128 + st * 2 * AT_K * 128 + AT_K * 128); };

    auto load_tile = [&](const __half* base, int r0, uint32_t dst) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int idx = tid + i * AT_THREADS, row = idx >> 3, ch = idx & 7;
            const bool ok = r0 + row < T;
            cpa16(dst + swz(row, ch), base + size_t(ok ? r0 + row : 0) * AT_D + ch * 8, ok);
        }
    };
    pdl_wait();
    const int nkv = (T + AT_K - 1) / AT_K;
    // cp.async group g holds K/V tile g (group 0 the Q tile too); tiles
    // 0 .. AT_STAGES-2 are in flight before the loop.
    load_tile(Qb, q0, sQa);
#pragma unroll
    for (int t = 0; t < AT_STAGES - 1; ++t) {
        if (t < nkv) {
            load_tile(Kb, t * AT_K, sKa(t));
            load_tile(Vb, t * AT_K, sVa(t));
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    }

    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
    uint32_t qf[4][4];
    const float L2E = 1.4426950408889634f;

    for (int j = 0; j < nkv; ++j) {
        // Tile j has landed (at most AT_STAGES-2 younger groups pending);
        // after the barrier every warp is done with tile j-1, whose stage
        // the load of tile j + AT_STAGES - 1 reuses: one barrier per tile.
        const int st = j % AT_STAGES;
        asm volatile("cp.async.wait_group %0;" ::"n"(AT_STAGES - 2) : "memory");
        __syncthreads();
        {
            const int jn = j + AT_STAGES - 1;
            if (jn < nkv) {
                load_tile(Kb, jn * AT_K, sKa(jn % AT_STAGES));
                load_tile(Vb, jn * AT_K, sVa(jn % AT_STAGES));
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
        }
        if (j == 0) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const int mi = lane >> 3, row = warp * 16 + (lane & 7) + (mi & 1) * 8, ch = kk * 2 + (mi >> 1);
                ldm_x4(sQa + swz(row, ch), qf[kk]);
            }
        }
        // S = Q K^T for this warp's 16 rows x 64 keys
        float s[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                uint32_t b[4];
                const int mi = lane >> 3, key = np * 16 + (lane & 7) + (mi >> 1) * 8, ch = kk * 2 + (mi & 1);
                ldm_x4(sKa(st) + swz(key, ch), b);
                mma16816(s[2 * np], qf[kk], b[0], b[1]);
                mma16816(s[2 * np + 1], qf[kk], b[2], b[3]);
            }
        }
        // mask keys past T (last tile only), then the online softmax:
        // p = 2^(s*log2e - m*log2e), one FFMA and one MUFU.EX2 per score
        const int kbase = j * AT_K;
        if (kbase + AT_K > T) {
#pragma unroll
            for (int nt = 0; nt < 8; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    if (kbase + nt * 8 + tig * 2 + (e & 1) >= T) s[nt][e] = -INFINITY;
        }
        // row maxima and sums as trees (short dependency chains)
        float mx[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            float t[8];
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) t[nt] = fmaxf(s[nt][2 * r], s[nt][2 * r + 1]);
#pragma unroll
            for (int w2 = 4; w2 > 0; w2 >>= 1)
#pragma unroll
                for (int i = 0; i < w2; ++i) t[i] = fmaxf(t[i], t[i + w2]);
            mx[r] = fmaxf(mrow[r], t[0]);
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
        }
        float alpha[2], nmx[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            alpha[r] = ex2_approx(__fmul_rn(__fsub_rn(mrow[r], mx[r]), L2E));
            nmx[r] = -__fmul_rn(mx[r], L2E);
            mrow[r] = mx[r];
            lrow[r] *= alpha[r];
        }
        // Once the row maxima settle alpha is 1 and the rescale a no-op.
        if (__any_sync(0xffffffffu, alpha[0] != 1.f || alpha[1] != 1.f)) {
#pragma unroll
            for (int nt = 0; nt < 8; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) o[nt][e] *= alpha[e >> 1];
        }
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) s[nt][e] = ex2_approx(fmaf(s[nt][e], L2E, nmx[e >> 1]));
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            float t[8];
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) t[nt] = s[nt][2 * r] + s[nt][2 * r + 1];
#pragma unroll
            for (int w2 = 4; w2 > 0; w2 >>= 1)
#pragma unroll
                for (int i = 0; i < w2; ++i) t[i] += t[i + w2];
            lrow[r] += t[0];
        }
        // O += P V
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t a[4];
            a[0] = pack_h2(s[2 * kk][0], s[2 * kk][1]);
            a[1] = pack_h2(s[2 * kk][2], s[2 * kk][3]);
            a[2] = pack_h2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
            a[3] = pack_h2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                uint32_t b[4];
                const int mi = lane >> 3, key = kk * 16 + (lane & 7) + (mi & 1) * 8, ch = np * 2 + (mi >> 1);
                ldm_x4_t(sVa(st) + swz(key, ch), b);
                mma16816(o[2 * np], a, b[0], b[1]);
                mma16816(o[2 * np + 1], a, b[2], b[3]);
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 1);
        lrow[r] += __shfl_xor_sync(0xffffffffu, lrow[r], 2);
    }
    const int D = H * AT_D;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int t = q0 + warp * 16 + g + r * 8;
        const float inv = 1.0f / lrow[r];
        if constexpr (QOUT) {
            // Two 32-column blocks per row of this head (columns 0-31: n-tiles
            // 0-3, 32-63: 4-7), spread over the quad's four lanes: the
            // reference quantizer with the block's amax and code sum over the
            // quad (every lane runs the shuffles; rows past T write nothing).
            const size_t row = size_t(w) * T + t;
#pragma unroll
            for (int hb = 0; hb < 2; ++hb) {
                float v[8], amax = 0.f;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    v[2 * j] = o[hb * 4 + j][2 * r] * inv;
                    v[2 * j + 1] = o[hb * 4 + j][2 * r + 1] * inv;
                    const float a0 = fabsf(v[2 * j]), a1 = fabsf(v[2 * j + 1]);
                    amax = fmaxf(amax, fmaxf(isnan(a0) ? 0.f : a0, isnan(a1) ? 0.f : a1));
                }
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
                const float d = __fdiv_rn(amax, 127.0f);
                const float qinv = d > 0.f ? __fdiv_rn(1.0f, d) : 0.f;
                int c[8], sum = 0;
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float rr = roundf(__fmul_rn(v[e], qinv));
                    c[e] = isnan(rr) ? 0 : int(fminf(127.f, fmaxf(-127.f, rr)));
                    sum += c[e];
                }
                sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                sum += __shfl_xor_sync(0xffffffffu, sum, 2);
                if (t < T) {
                    uint16_t* dst = qo.q16 + row * D + h * AT_D + hb * 32;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        *reinterpret_cast<uint32_t*>(dst + j * 8 + tig * 2) =
                            uint32_t(__half_as_ushort(__int2half_rn(c[2 * j]))) |
                            (uint32_t(__half_as_ushort(__int2half_rn(c[2 * j + 1]))) << 16);
                    if (tig == 0) {
                        const size_t bl = size_t(h) * 2 + hb;
                        qo.dT[bl * qo.m_pad + row] = d;
                        qo.uT[bl * qo.m_pad + row] = __fmul_rn(d, float(sum));
                    }
                }
            }
        } else {
            if (t >= T) continue;
            float* dst = out + (size_t(w) * T + t) * D + h * AT_D;
#pragma unroll
            for (int nt = 0; nt < 8; ++nt)
                *reinterpret_cast<float2*>(dst + nt * 8 + tig * 2) =
                    make_float2(o[nt][2 * r] * inv, o[nt][2 * r + 1] * inv);
        }
    }
}

unsigned grid_stride(size_t total, int tpb) {
    size_t g = (total + tpb - 1) / tpb;
    return unsigned(g > 148 * 16 ? 148 * 16 : (g ? g : 1));
}

template <int MODE>
cudaError_t rows_quant_mode(const float* x, const float* add, float* xout, const float* lw, const float* lb, int m,
                            int k, const QOut& o, float* yout, cudaStream_t s) {
    const int rows = o.q16 ? o.m_pad : m;
    const int nch = k / 128;
    if constexpr (MODE == RQ_PLAIN || MODE == RQ_GELU) {
        // One chunk per warp for decoder-sized batches (latency), four for
        // encoder-sized ones; the result does not depend on the split.
        const int slice = size_t(rows) * nch >= size_t(1) << 16 ? 4 : 1;
        const int wpr = (nch + slice - 1) / slice;
        const unsigned grid = unsigned((size_t(rows) * wpr * 32 + 255) / 256);
        return launch_pdl(k_rows_quant<MODE, 1>, dim3(grid), dim3(256), 0, s, x, add, xout, lw, lb, m, k, o, yout,
                          slice);
    } else {
        // Encoder-sized batches: one warp per row (k_ln_rows_warp); the result
        // is the same bits as the RQ_WPR-warp kernel's.
        if (rows >= 2048 && nch <= 16) {
            const unsigned grid = unsigned((size_t(rows) * 32 + 127) / 128);
            if (nch <= 4)
                return launch_pdl(k_ln_rows_warp<MODE, 4>, dim3(grid), dim3(128), 0, s, x, add, xout, lw, lb, m, k, o,
                                  yout);
            if (nch <= 8)
                return launch_pdl(k_ln_rows_warp<MODE, 8>, dim3(grid), dim3(128), 0, s, x, add, xout, lw, lb, m, k, o,
                                  yout);
            if (nch <= 12)
                return launch_pdl(k_ln_rows_warp<MODE, 12>, dim3(grid), dim3(128), 0, s, x, add, xout, lw, lb, m, k, o,
                                  yout);
            return launch_pdl(k_ln_rows_warp<MODE, 16>, dim3(grid), dim3(128), 0, s, x, add, xout, lw, lb, m, k, o, yout);
        }
        // Decoder-sized batches: one row (RQ_WPR warps) per CTA, to spread
        // the few rows over the SMs.
        const int tpb = RQ_WPR * 32;
        const unsigned grid = unsigned((size_t(rows) * RQ_WPR * 32 + tpb - 1) / tpb);
        if (nch <= RQ_WPR * 2)
            return launch_pdl(k_rows_quant<MODE, 2>, dim3(grid), dim3(tpb), 0, s, x, add, xout, lw, lb, m, k, o, yout, 1);
        if (nch <= RQ_WPR * 4)
            return launch_pdl(k_rows_quant<MODE, 4>, dim3(grid), dim3(tpb), 0, s, x, add, xout, lw, lb, m, k, o, yout, 1);
        return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t launch_rows_quant(int mode, const float* x, const float* add, float* xout, const float* lw,
                              const float* lb, int m, int k, int m_pad, uint16_t* q16, float* dT, float* uT,
                              float* yout, cudaStream_t s) {
    ActsView v;
    v.m_pad = m_pad;
    v.q16 = q16;
    v.dT = dT;
    v.uT = uT;
    return launch_rows_quant_v(mode, x, add, xout, lw, lb, m, k, q16 ? &v : nullptr, nullptr, yout, s);
}

cudaError_t launch_rows_quant_v(int mode, const float* x, const float* add, float* xout, const float* lw,
                                const float* lb, int m, int k, const ActsView* gemm, const ActsView* gemv,
                                float* yout, cudaStream_t s) {
    if (k % 128) return cudaErrorInvalidValue;
    if (m <= 0) return cudaSuccess;
    QOut o = {};
    if (gemm) {
        o.q16 = gemm->q16;
        o.dT = gemm->dT;
        o.uT = gemm->uT;
        o.m_pad = gemm->m_pad;
    }
    if (gemv) {
        o.q8 = gemv->q8;
        o.d = gemv->d;
        o.sum = gemv->sum;
        o.u = gemv->u;
    }
    switch (mode) {
        case RQ_PLAIN: return rows_quant_mode<RQ_PLAIN>(x, add, xout, lw, lb, m, k, o, yout, s);
        case RQ_GELU: return rows_quant_mode<RQ_GELU>(x, add, xout, lw, lb, m, k, o, yout, s);
        case RQ_LN: return rows_quant_mode<RQ_LN>(x, add, xout, lw, lb, m, k, o, yout, s);
        case RQ_ADD_LN: return rows_quant_mode<RQ_ADD_LN>(x, add, xout, lw, lb, m, k, o, yout, s);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_to_heads(const float* src, int ld, int col0, int n_win, int T, int H, float scale, __half* dst,
                            cudaStream_t s) {
    const size_t total = size_t(n_win) * H * T * 16;
    if (!total) return cudaSuccess;
    k_to_heads<<<grid_stride(total, 256), 256, 0, s>>>(src, ld, col0, n_win, T, H, scale, dst);
    return cudaGetLastError();
}

// The dynamic shared-memory limit of k_attn<QOUT> (variant v), raised once
// per device, with the whole carveout as shared memory (four 57 KB CTAs).
cudaError_t attn_smem_attr(void (*kern)(const __half*, const __half*, const __half*, int, int, float*, QOut), int v) {
    static std::atomic<uint64_t> done{0};
    int dev = 0;
    if (const cudaError_t e = cudaGetDevice(&dev)) return e;
    const uint64_t bit = uint64_t(1) << ((dev & 31) * 2 + v);
    if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
    if (const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM))
        return e;
    if (const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                                   int(cudaSharedmemCarveoutMaxShared)))
        return e;
    done.fetch_or(bit, std::memory_order_acq_rel);
    return cudaSuccess;
}

cudaError_t launch_attention(const __half* Qh, const __half* Kh, const __half* Vh, int n_win, int T, int H,
                             float* out, cudaStream_t s, uint16_t* q16, float* dT, float* uT, int m_pad) {
    if (!n_win || !T || !H) return cudaSuccess;
    dim3 grid((T + AT_Q - 1) / AT_Q, H, n_win);
    QOut qo{};
    if (q16) {
        qo.q16 = q16;
        qo.dT = dT;
        qo.uT = uT;
        qo.m_pad = m_pad;
        if (const cudaError_t e = attn_smem_attr(k_attn<true>, 0)) return e;
        return launch_pdl(k_attn<true>, grid, dim3(AT_THREADS), size_t(AT_SMEM), s, Qh, Kh, Vh, T, H, out, qo);
    }
    if (const cudaError_t e = attn_smem_attr(k_attn<false>, 1)) return e;
    return launch_pdl(k_attn<false>, grid, dim3(AT_THREADS), size_t(AT_SMEM), s, Qh, Kh, Vh, T, H, out, qo);
}

}  // namespace rwq
