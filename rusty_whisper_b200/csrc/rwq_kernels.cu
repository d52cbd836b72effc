// rwq_kernels.cu -- CUDA-core kernels of the quantized-matmul path:
// weight repack, activation int8 quantizer, bit-exact dequant gather,
// per-block integer dots (debug/parity), the decoder GEMVs (int8 and
// dequant-then-f32), and the builder of the tensor-core operand cache.
#include <cuda_fp16.h>
#include <cstdio>
#include <cstdlib>
#include "rwq_common.cuh"
#include "rwq_internal.h"
#include "rwq_decoder.h"

namespace rwq {

namespace {

constexpr int TPB = 256;

// Current device and its SM count, cached per device (launch paths run per
// call; the attribute query is not free).
inline void dev_sms(int* dev, int* sms) {
    static int cache[64] = {};
    cudaGetDevice(dev);
    if (*dev < 0 || *dev >= 64) {
        cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, *dev);
        return;
    }
    if (!cache[*dev]) cudaDeviceGetAttribute(&cache[*dev], cudaDevAttrMultiProcessorCount, *dev);
    *sms = cache[*dev];
}

inline unsigned grid_for(size_t work, int per_block) {
    size_t g = (work + per_block - 1) / per_block;
    return unsigned(g ? g : 1);
}

// ---------------------------------------------------------------- repack
// raw ggml records [n*nb][bb] -> planes (layout in rwq_common.cuh).  One
// thread per block; the raw records are not 16-byte aligned, so they are
// read bytewise, once.  Pad blocks (kb >= nb) keep the zeros the planes
// were cleared to.
template <int DT>
__global__ void k_repack(const uint8_t* __restrict__ raw, uint8_t* __restrict__ qs, uint32_t* __restrict__ qh,
                         uint16_t* __restrict__ d, uint16_t* __restrict__ m, size_t nblk, int nb, int nb4) {
    size_t b = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (b >= nblk) return;
    constexpr int BB = block_bytes(DT), QSB = qs_bytes(DT), QO = raw_qs_off(DT);
    const size_t j = b / size_t(nb);
    const int kb = int(b % size_t(nb));
    const size_t pb = j * size_t(nb4) + kb;
    const uint8_t* p = raw + b * BB;
    d[pb] = uint16_t(p[0] | (p[1] << 8));
    if (has_min(DT)) m[pb] = uint16_t(p[2] | (p[3] << 8));
    if (has_qh(DT)) {
        const uint8_t* h = p + raw_qh_off(DT);
        qh[pb] = qh_plane_bits(uint32_t(h[0]) | (uint32_t(h[1]) << 8) | (uint32_t(h[2]) << 16) |
                               (uint32_t(h[3]) << 24));
    }
    uint8_t* grp = qs + qs_group_off<DT>(j, kb, nb4);
#pragma unroll
    for (int i = 0; i < QSB / 4; ++i) {
        const uint32_t word = uint32_t(p[QO + 4 * i]) | (uint32_t(p[QO + 4 * i + 1]) << 8) |
                              (uint32_t(p[QO + 4 * i + 2]) << 16) | (uint32_t(p[QO + 4 * i + 3]) << 24);
        *reinterpret_cast<uint32_t*>(grp + qs_word_off<DT>(i, kb & 3)) = word;
    }
}

// ------------------------------------------------------------ quantizer
// quantize_acts_i8 (quant.rs:690-716): per 32-element block d = amax/127
// (IEEE division), inv = 1/d or 0, q = round(x*inv) half away from zero,
// clamped to [-127,127]; NaN codes become 0 as Rust's `as i32` makes them.
// Eight lanes share a block (4 elements each, one 16-byte load), so a warp
// quantizes four blocks; amax and sum(q) are xor-reduced over the 8 lanes.
// Rows m..m_pad-1 of the transposed scale planes are written as zeros.
template <bool VEC>
__global__ void k_quantize(const float* __restrict__ a, int m, int k, int nb, int m_pad, int8_t* __restrict__ q8,
                           float* __restrict__ dd, int32_t* __restrict__ sum, float* __restrict__ uu,
                           uint16_t* __restrict__ q16, float* __restrict__ dT, float* __restrict__ uT) {
    pdl_trigger();
    pdl_wait();
    const size_t t = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    const size_t blk = t >> 3;
    const int sub = int(t & 7);
    if (blk >= size_t(m_pad) * nb) return;  // whole groups of 8 lanes leave together
    const int i = int(blk / nb), bl = int(blk % nb);
    if (i >= m) {
        if (sub == 0 && dT) {
            dT[size_t(bl) * m_pad + i] = 0.f;
            uT[size_t(bl) * m_pad + i] = 0.f;
        }
        return;
    }
    const size_t off = size_t(i) * k + size_t(bl) * QK + sub * 4;
    const float4 x = VEC ? *reinterpret_cast<const float4*>(a + off)
                         : make_float4(a[off], a[off + 1], a[off + 2], a[off + 3]);
    auto absnn = [](float v) { const float w = fabsf(v); return isnan(w) ? 0.f : w; };  // f32::max skips NaN
    float amax = fmaxf(fmaxf(absnn(x.x), absnn(x.y)), fmaxf(absnn(x.z), absnn(x.w)));
    const unsigned grp = 0xFFu << (threadIdx.x & 24);
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(grp, amax, o));
    const float d = __fdiv_rn(amax, 127.0f);
    const float inv = d > 0.f ? __fdiv_rn(1.0f, d) : 0.f;
    auto code = [inv](float v) {
        const float r = roundf(__fmul_rn(v, inv));
        return isnan(r) ? 0 : int(fminf(127.f, fmaxf(-127.f, r)));
    };
    const int c0 = code(x.x), c1 = code(x.y), c2 = code(x.z), c3 = code(x.w);
    int s = c0 + c1 + c2 + c3;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) s += __shfl_xor_sync(grp, s, o);
    if (q8)
        *reinterpret_cast<uint32_t*>(q8 + off) =
            uint32_t(uint8_t(c0)) | (uint32_t(uint8_t(c1)) << 8) | (uint32_t(uint8_t(c2)) << 16) | (uint32_t(uint8_t(c3)) << 24);
    if (q16) {
        const uint32_t h01 = uint32_t(__half_as_ushort(__int2half_rn(c0))) | (uint32_t(__half_as_ushort(__int2half_rn(c1))) << 16);
        const uint32_t h23 = uint32_t(__half_as_ushort(__int2half_rn(c2))) | (uint32_t(__half_as_ushort(__int2half_rn(c3))) << 16);
        *reinterpret_cast<uint2*>(q16 + off) = make_uint2(h01, h23);
    }
    if (sub == 0) {
        const size_t o = size_t(i) * nb + bl;
        const float u = __fmul_rn(d, float(s));
        dd[o] = d;
        sum[o] = s;
        uu[o] = u;
        if (dT) {
            dT[size_t(bl) * m_pad + i] = d;
            uT[size_t(bl) * m_pad + i] = u;
        }
    }
}

// ------------------------------------------------------ block decoding
// Load one block's code bytes and scales from the planes.
template <int DT>
struct BlockCodes {
    uint32_t w[8];   // u8x4 codes (4/5-bit formats) or s8x4 codes (Q8_0)
    float d, m;
};

// The code words of block kb of row j (gathered from the interleaved
// group: four 4-byte loads, or four 8-byte loads for Q8_0).
template <int DT>
__device__ __forceinline__ void load_words(const uint8_t* __restrict__ qs, size_t j, int kb, int nb4, uint32_t (&w)[8]) {
    const uint8_t* g = qs + qs_group_off<DT>(j, kb, nb4);
    const int b = kb & 3;
    if (DT == Q8_0) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint2 v = __ldg(reinterpret_cast<const uint2*>(g + qs_word_off<DT>(c, b)));
            w[c] = v.x;
            w[4 + c] = v.y;
        }
    } else {
#pragma unroll
        for (int c = 0; c < 4; ++c) w[c] = __ldg(reinterpret_cast<const uint32_t*>(g + qs_word_off<DT>(c, b)));
    }
}

template <int DT>
__device__ __forceinline__ void load_block(const uint8_t* __restrict__ qs, const uint32_t* __restrict__ qh,
                                           const uint16_t* __restrict__ dp, const uint16_t* __restrict__ mp,
                                           size_t j, int kb, int nb4, BlockCodes<DT>& bc) {
    const size_t b = j * size_t(nb4) + kb;
    if (DT == Q8_0) {
        load_words<DT>(qs, j, kb, nb4, bc.w);
    } else {
        uint32_t v[8];
        load_words<DT>(qs, j, kb, nb4, v);
        uint32_t h = has_qh(DT) ? __ldg(qh + b) : 0u;
        codes_u8x4<DT>(make_uint4(v[0], v[1], v[2], v[3]), h, bc.w);
    }
    bc.d = h2f(__ldg(dp + b));
    bc.m = has_min(DT) ? h2f(__ldg(mp + b)) : 0.f;
}

// Integer block dot S = sum(q_a * q_b) with q_b centred, exact.
template <int DT>
__device__ __forceinline__ int block_dot(const uint32_t (&w)[8], const int4 a0, const int4 a1, int suma) {
    const uint32_t a[8] = {uint32_t(a0.x), uint32_t(a0.y), uint32_t(a0.z), uint32_t(a0.w),
                           uint32_t(a1.x), uint32_t(a1.y), uint32_t(a1.z), uint32_t(a1.w)};
    int s = 0;
    if (DT == Q8_0) {
#pragma unroll
        for (int t = 0; t < 8; ++t) s = dp4a_ss(a[t], w[t], s);
    } else {
#pragma unroll
        for (int t = 0; t < 8; ++t) s = dp4a_su(a[t], w[t], s);
        if (code_offset(DT)) s -= code_offset(DT) * suma;
    }
    return s;
}

// Centred code of element e (0..31) from the u8x4 / s8x4 words.
template <int DT>
__device__ __forceinline__ int code_at(const uint32_t (&w)[8], int e) {
    const int word = (e < 16) ? (e >> 2) : 4 + ((e - 16) >> 2);
    const int byte = e & 3;
    const uint32_t v = (w[word] >> (8 * byte)) & 0xFFu;
    if (DT == Q8_0) return int(int8_t(v));
    return int(v) - code_offset(DT);
}

// ------------------------------------------------------------- dequant
// QTensor::row_f32 / to_dense (quant.rs:528-537, 566-576): x = d*q + m with
// a separate rounded multiply and add, bit-identical to the reference.
template <int DT>
__global__ void k_dequant_rows(const uint8_t* __restrict__ qs, const uint32_t* __restrict__ qh,
                               const uint16_t* __restrict__ dp, const uint16_t* __restrict__ mp,
                               const int32_t* __restrict__ rows, int nrows, int n, int nb, float* __restrict__ out) {
    size_t t = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= size_t(nrows) * nb) return;
    const int r = int(t / nb), bl = int(t % nb);
    const int j = rows ? rows[r] : r;
    if (j < 0 || j >= n) return;  // host validated; guard anyway
    BlockCodes<DT> bc;
    load_block<DT>(qs, qh, dp, mp, size_t(j), bl, round4(nb), bc);
    float* o = out + size_t(r) * nb * QK + size_t(bl) * QK;
#pragma unroll
    for (int e = 0; e < QK; e += 4) {
        float4 v;
        v.x = __fadd_rn(__fmul_rn(bc.d, float(code_at<DT>(bc.w, e + 0))), bc.m);
        v.y = __fadd_rn(__fmul_rn(bc.d, float(code_at<DT>(bc.w, e + 1))), bc.m);
        v.z = __fadd_rn(__fmul_rn(bc.d, float(code_at<DT>(bc.w, e + 2))), bc.m);
        v.w = __fadd_rn(__fmul_rn(bc.d, float(code_at<DT>(bc.w, e + 3))), bc.m);
        *reinterpret_cast<float4*>(o + e) = v;
    }
}

// Token embedding gather for the decoder (decoder.rs:125-136): row
// tokens[r] dequantized exactly like QTensor::row_f32, plus the learned
// position row *dpos of `pos` (x = dequant + pos, one rounding).
template <int DT>
__global__ void k_embed(const uint8_t* __restrict__ qs, const uint32_t* __restrict__ qh,
                        const uint16_t* __restrict__ dp, const uint16_t* __restrict__ mp,
                        const int32_t* __restrict__ tokens, int nrows, int n, int nb, const float* __restrict__ pos,
                        const int* __restrict__ dpos, float* __restrict__ x) {
    pdl_trigger();
    pdl_wait();
    pos += size_t(*dpos) * nb * QK;
    size_t t = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= size_t(nrows) * nb) return;
    const int r = int(t / nb), bl = int(t % nb);
    int j = tokens[r];
    j = j < 0 ? 0 : (j >= n ? n - 1 : j);   // the host validates ids; keep the access in bounds regardless
    BlockCodes<DT> bc;
    load_block<DT>(qs, qh, dp, mp, size_t(j), bl, round4(nb), bc);
    float* o = x + size_t(r) * nb * QK + size_t(bl) * QK;
    const float* p = pos + size_t(bl) * QK;
#pragma unroll
    for (int e = 0; e < QK; e += 4) {
        float4 v;
        v.x = __fadd_rn(__fadd_rn(__fmul_rn(bc.d, float(code_at<DT>(bc.w, e + 0))), bc.m), p[e + 0]);
        v.y = __fadd_rn(__fadd_rn(__fmul_rn(bc.d, float(code_at<DT>(bc.w, e + 1))), bc.m), p[e + 1]);
        v.z = __fadd_rn(__fadd_rn(__fmul_rn(bc.d, float(code_at<DT>(bc.w, e + 2))), bc.m), p[e + 2]);
        v.w = __fadd_rn(__fadd_rn(__fmul_rn(bc.d, float(code_at<DT>(bc.w, e + 3))), bc.m), p[e + 3]);
        *reinterpret_cast<float4*>(o + e) = v;
    }
}

// ---------------------------------------------------------- block dots
// S[i][j][kb] for parity tests of the integer core (quant.rs:1352-1360).
template <int DT>
__global__ void k_block_dots(const uint8_t* __restrict__ qs, const uint32_t* __restrict__ qh,
                             const uint16_t* __restrict__ dp, const uint16_t* __restrict__ mp,
                             const int8_t* __restrict__ q8, const int32_t* __restrict__ suma, int m, int n, int nb,
                             int32_t* __restrict__ S) {
    size_t t = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= size_t(m) * n * nb) return;
    const int bl = int(t % nb);
    const int j = int((t / nb) % n);
    const int i = int(t / (size_t(nb) * n));
    BlockCodes<DT> bc;
    load_block<DT>(qs, qh, dp, mp, size_t(j), bl, round4(nb), bc);
    const int4* a = reinterpret_cast<const int4*>(q8 + size_t(i) * nb * QK + size_t(bl) * QK);
    S[t] = block_dot<DT>(bc.w, a[0], a[1], suma[size_t(i) * nb + bl]);
}

// -------------------------------------------------------------- GEMV i8
// Undecoded block bytes, loaded one row group ahead of their use.
template <int DT>
struct RawBlock {
    uint4 v0, v1;   // code bytes (v1: Q8_0 only)
    uint32_t qh;
    uint16_t d, m;
};

template <int DT>
__device__ __forceinline__ void load_raw(const uint8_t* __restrict__ qs, const uint32_t* __restrict__ qh,
                                         const uint16_t* __restrict__ dp, const uint16_t* __restrict__ mp, size_t j,
                                         int kb, int nb4, RawBlock<DT>& rb) {
    uint32_t w[8];
    load_words<DT>(qs, j, kb, nb4, w);
    rb.v0 = make_uint4(w[0], w[1], w[2], w[3]);
    if (DT == Q8_0) rb.v1 = make_uint4(w[4], w[5], w[6], w[7]);
    const size_t b = j * size_t(nb4) + kb;
    if (has_qh(DT)) rb.qh = __ldg(qh + b);
    rb.d = __ldg(dp + b);
    if (has_min(DT)) rb.m = __ldg(mp + b);
}

template <int DT>
__device__ __forceinline__ void decode(const RawBlock<DT>& rb, BlockCodes<DT>& bc) {
    if (DT == Q8_0) {
        bc.w[0] = rb.v0.x; bc.w[1] = rb.v0.y; bc.w[2] = rb.v0.z; bc.w[3] = rb.v0.w;
        bc.w[4] = rb.v1.x; bc.w[5] = rb.v1.y; bc.w[6] = rb.v1.z; bc.w[7] = rb.v1.w;
    } else {
        codes_u8x4<DT>(rb.v0, has_qh(DT) ? rb.qh : 0u, bc.w);
    }
    bc.d = h2f(rb.d);
    bc.m = has_min(DT) ? h2f(rb.m) : 0.f;
}

// Decoder GEMV, M <= 8 activation rows.  Each warp owns 32/L weight rows
// (a "row group"), L lanes per row; lane `sub` takes blocks kb = sub +
// L*t, t < BPL.  Because a lane always visits the same blocks, its
// activation codes and scales for those blocks are loaded into registers
// once.  Weight blocks are read with 128-bit loads of the code plane, PF
// row groups ahead of use; nibbles and high bits are unpacked in
// registers.  The dp4a chain starts from the bits of 1.5*2^23 (minus the
// Q4_0/Q5_0 code offset times sum(q_a)), so for |S| < 2^22 its result is
// the f32 1.5*2^23 + S exactly and S = bits - 1.5*2^23 is one FADD.  Per
// block, in kb order,
//     acc <- fma(d_a*d_b, S, acc);  acc <- fma(d_a*sum(q_a), m_b, acc)
// then an xor butterfly over the L lanes.  L and BPL depend on K only, so
// every output row is bit-identical whatever M (quant.rs:1372-1384).

template <int DT, int L, int BPL, int MR, int PF, bool REGA>
__global__ void __launch_bounds__(TPB) k_gemv_i8(const uint8_t* __restrict__ qs, const uint32_t* __restrict__ qh,
                                                 const uint16_t* __restrict__ dp, const uint16_t* __restrict__ mp,
                                                 const int8_t* __restrict__ q8, const float* __restrict__ da,
                                                 const int32_t* __restrict__ sa, const float* __restrict__ ua, int M,
                                                 int N, int K, const float* __restrict__ bias, float* __restrict__ y) {
    pdl_trigger();
    const int nb = K / QK, nb4 = round4(nb);
    constexpr int RPW = 32 / L;
    const int lane = threadIdx.x & 31, sub = lane % L, slot = lane / L;
    const int warps_per_cta = blockDim.x >> 5;
    const int nw = gridDim.x * warps_per_cta;
    const int groups = (N + RPW - 1) / RPW;
    const int g0 = blockIdx.x * warps_per_cta + (threadIdx.x >> 5);

    RawBlock<DT> ring[PF][BPL];
    auto fetch = [&](int grp, RawBlock<DT>(&dst)[BPL]) {
        const int j = grp * RPW + slot;
#pragma unroll
        for (int t = 0; t < BPL; ++t) {
            const int kb = sub + L * t;
            if (grp < groups && j < N && kb < nb) load_raw<DT>(qs, qh, dp, mp, size_t(j), kb, nb4, dst[t]);
        }
    };
    // The weights are not written by the previous kernel in the stream, so
    // their first loads go out before waiting for it; the activations and
    // the output are, so everything else waits.
#pragma unroll
    for (int u = 0; u < PF; ++u) fetch(g0 + u * nw, ring[u]);
    pdl_wait();

    // This lane's activation blocks, for every row: in registers when they
    // are few (REGA), else staged once per CTA in shared memory.
    constexpr int TB = REGA ? BPL : 1, TR = REGA ? MR : 1;
    int4 a0[TB][TR], a1[TB][TR];
    float ad[TB][TR], au[TB][TR];
    uint32_t init[TB][TR];
    extern __shared__ __align__(16) uint8_t smem[];
    int8_t* s_q = reinterpret_cast<int8_t*>(smem);
    float* s_d = reinterpret_cast<float*>(smem + size_t(M) * K);
    float* s_u = s_d + M * nb;
    int32_t* s_s = reinterpret_cast<int32_t*>(s_u + M * nb);
    if (!REGA) {
        const int4* src = reinterpret_cast<const int4*>(q8);
        int4* dst = reinterpret_cast<int4*>(s_q);
        for (int i = threadIdx.x; i < M * K / 16; i += blockDim.x) dst[i] = __ldg(src + i);
        for (int i = threadIdx.x; i < M * nb; i += blockDim.x) {
            s_d[i] = __ldg(da + i);
            s_u[i] = __ldg(ua + i);
            s_s[i] = __ldg(sa + i);
        }
        __syncthreads();
    }
#pragma unroll
    for (int t = 0; t < TB; ++t) {
        const int kb = sub + L * t;
#pragma unroll
        for (int r = 0; r < TR; ++r) {
            if (REGA && r < M && kb < nb) {
                const int4* a = reinterpret_cast<const int4*>(q8 + size_t(r) * K + size_t(kb) * QK);
                a0[t][r] = __ldg(a);
                a1[t][r] = __ldg(a + 1);
                ad[t][r] = __ldg(da + r * nb + kb);
                au[t][r] = has_min(DT) ? __ldg(ua + r * nb + kb) : 0.f;
                init[t][r] = MAGIC_BITS - uint32_t(code_offset(DT) * __ldg(sa + r * nb + kb));
            } else {
                a0[t][r] = a1[t][r] = make_int4(0, 0, 0, 0);
                ad[t][r] = au[t][r] = 0.f;
                init[t][r] = MAGIC_BITS;
            }
        }
    }

    for (int gb = g0; gb < groups; gb += PF * nw) {
#pragma unroll
        for (int u = 0; u < PF; ++u) {
            const int g = gb + u * nw;
            const int j = g * RPW + slot;
            float acc[MR];
#pragma unroll
            for (int r = 0; r < MR; ++r) acc[r] = 0.f;
#pragma unroll
            for (int t = 0; t < BPL; ++t) {
                const int kb = sub + L * t;
                if (g < groups && j < N && kb < nb) {
                    BlockCodes<DT> bc;
                    decode<DT>(ring[u][t], bc);
#pragma unroll
                    for (int r = 0; r < MR; ++r) {
                        if (r < M) {
                            int4 x0, x1;
                            float xd, xu;
                            uint32_t xi;
                            if (REGA) {
                                x0 = a0[REGA ? t : 0][REGA ? r : 0];
                                x1 = a1[REGA ? t : 0][REGA ? r : 0];
                                xd = ad[REGA ? t : 0][REGA ? r : 0];
                                xu = au[REGA ? t : 0][REGA ? r : 0];
                                xi = init[REGA ? t : 0][REGA ? r : 0];
                            } else {
                                const int4* ap = reinterpret_cast<const int4*>(s_q + size_t(r) * K + kb * QK);
                                x0 = ap[0];
                                x1 = ap[1];
                                xd = s_d[r * nb + kb];
                                xu = has_min(DT) ? s_u[r * nb + kb] : 0.f;
                                xi = MAGIC_BITS - uint32_t(code_offset(DT) * s_s[r * nb + kb]);
                            }
                            const uint32_t av[8] = {uint32_t(x0.x), uint32_t(x0.y), uint32_t(x0.z), uint32_t(x0.w),
                                                    uint32_t(x1.x), uint32_t(x1.y), uint32_t(x1.z), uint32_t(x1.w)};
                            int sbits = int(xi);
#pragma unroll
                            for (int w = 0; w < 8; ++w)
                                sbits = DT == Q8_0 ? dp4a_ss(av[w], bc.w[w], sbits) : dp4a_su(av[w], bc.w[w], sbits);
                            const float S = __fsub_rn(__int_as_float(sbits), MAGIC_F);
                            acc[r] = __fmaf_rn(__fmul_rn(xd, bc.d), S, acc[r]);
                            if (has_min(DT)) acc[r] = __fmaf_rn(xu, bc.m, acc[r]);
                        }
                    }
                }
            }
            // refill this ring slot PF groups ahead
            fetch(g + PF * nw, ring[u]);
#pragma unroll
            for (int r = 0; r < MR; ++r) {
                if (r < M) {   // M is the same for the whole warp
#pragma unroll
                    for (int o = L / 2; o > 0; o >>= 1)
                        acc[r] = __fadd_rn(acc[r], __shfl_xor_sync(0xffffffffu, acc[r], o));
                }
            }
            if (g < groups && j < N && sub == 0) {
                const float b = bias ? __ldg(bias + j) : 0.f;
#pragma unroll
                for (int r = 0; r < MR; ++r)
                    if (r < M) y[size_t(r) * N + j] = bias ? __fadd_rn(acc[r], b) : acc[r];
            }
        }
    }
}

// ------------------------------------------------------------ GEMV mma
// Decoder GEMV on the integer MMA (mma.sync m16n8k32, s32 accumulate),
// M <= 8 activation rows.  A warp owns a tile of 16 weight rows and walks
// its K range one 4-block group at a time; quad lane c (lane = 4g + c)
// loads word c of the group's four blocks for rows g and g+8 with one
// 16-byte load per row (32 for Q8_0) -- the interleaved code plane makes
// that exactly its A fragment: low nibbles are elements 4c..4c+3, high
// nibbles elements 16+4c..16+4c+3, fifth bits from the permuted qh word
// with one shift and mask.  The activation codes (B fragments) and their
// per-block scales are staged once per CTA in shared memory in fragment
// order.  Each block is one MMA whose accumulator starts at the bits of
// 1.5*2^23 minus the code offset times sum(q_a), so S = D - 1.5*2^23 is
// the exact centred integer block dot, then per output (row j, act row i)
//     acc <- fma(d_a*d_b, S, acc);  acc <- fma(d_a*sum(q_a), m_b, acc)
// in kb order (the formula of quant.rs:349-351 / :452-454).  With KS > 1
// the K range is split over KS warps of a CTA and their partial sums are
// added in slice order.  KS depends on N and K only, so a row's result
// does not depend on M (quant.rs:1372-1384).
constexpr int GM_THREADS = 256;

// 4-byte cp.async global -> shared; `ok` false writes zeros and reads nothing.
__device__ __forceinline__ void cp_async4(void* dst, const void* src, bool ok) {
    const uint32_t d = uint32_t(__cvta_generic_to_shared(dst));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(d), "l"(src), "r"(ok ? 4 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <int DT>
struct MmaGroup {
    uint32_t q[2][qs_bytes(DT) / 4];    // [row g, g+8][word c (and 4+c) of blocks 0..3]
    uint32_t h[2][has_qh(DT) ? 4 : 1];  // qh words of blocks 0..3
    uint2 d[2], m[2];                   // f16 d (m) of blocks 0..3
};

// Two f16 (low half first) to f32, exactly.
__device__ __forceinline__ float2 h2f2(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

template <bool SA>
__device__ __forceinline__ void mma_i8(const uint32_t (&a)[4], uint2 b, int2 ci, int (&d)[4]) {
    if (SA)
        asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                     "{%10,%11,%12,%13};"
                     : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y), "r"(ci.x), "r"(ci.y),
                       "r"(ci.x), "r"(ci.y));
    else
        asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                     "{%10,%11,%12,%13};"
                     : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y), "r"(ci.x), "r"(ci.y),
                       "r"(ci.x), "r"(ci.y));
}

// Shared-memory staging of the activations, per block kb and n-tile nt
// (8 activation rows each): 32 B-fragment pairs (lane order); per quad
// lane c the seeds and d_a of act rows 2c and 2c+1 as one 16-byte record
// {seed, seed, d_a, d_a}; d_a*sum(q_a) of the tile's 8 rows.
struct MmaActs {
    const uint2* frag;   // [nb4][NT][32]
    const int4* sc;      // [nb4][NT][4]
    const float* ua;     // [nb4][NT][8]
};

template <int DT, int NT>
__device__ __forceinline__ void mma_compute(const MmaGroup<DT>& r, const MmaActs& A, int G, int lane, float2 (&a01)[NT],
                                            float2 (&a23)[NT]) {
    const int c = lane & 3;
    const float2 dr0[2] = {h2f2(r.d[0].x), h2f2(r.d[0].y)}, dr1[2] = {h2f2(r.d[1].x), h2f2(r.d[1].y)};
    float2 mr0[2], mr1[2];
    if (has_min(DT)) {
        mr0[0] = h2f2(r.m[0].x); mr0[1] = h2f2(r.m[0].y);
        mr1[0] = h2f2(r.m[1].x); mr1[1] = h2f2(r.m[1].y);
    }
    const float2 nmag = make_float2(-MAGIC_F, -MAGIC_F);
    // Pad blocks (kb >= nb) need no test: their weight codes and scales
    // are zero and their activation records are staged as zero scales with
    // seed 1.5*2^23, so they add exactly 0.
#pragma unroll
    for (int b = 0; b < 4; ++b) {
        const int kb = 4 * G + b;
        uint32_t a[4];
        if (DT == Q8_0) {
            a[0] = r.q[0][(2 * b) % (qs_bytes(DT) / 4)];
            a[1] = r.q[1][(2 * b) % (qs_bytes(DT) / 4)];
            a[2] = r.q[0][(2 * b + 1) % (qs_bytes(DT) / 4)];
            a[3] = r.q[1][(2 * b + 1) % (qs_bytes(DT) / 4)];
        } else {
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                const uint32_t w = r.q[rr][b % (qs_bytes(DT) / 4)];
                uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
                if (has_qh(DT)) {
                    const uint32_t h = r.h[rr][b % (has_qh(DT) ? 4 : 1)];
                    lo |= (h << (4 - c)) & 0x10101010u;
                    hi |= (h >> c) & 0x10101010u;
                }
                a[rr] = lo;
                a[2 + rr] = hi;
            }
        }
        const float db0 = (b & 1) ? dr0[b >> 1].y : dr0[b >> 1].x;
        const float db1 = (b & 1) ? dr1[b >> 1].y : dr1[b >> 1].x;
        float mb0 = 0.f, mb1 = 0.f;
        if (has_min(DT)) {
            mb0 = (b & 1) ? mr0[b >> 1].y : mr0[b >> 1].x;
            mb1 = (b & 1) ? mr1[b >> 1].y : mr1[b >> 1].x;
        }
        // One MMA per 8 activation rows, all on the same decoded A fragment.
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const uint2 bf = A.frag[(kb * NT + nt) * 32 + lane];
            const int4 sc = A.sc[(kb * NT + nt) * 4 + c];
            int dd[4];
            mma_i8<DT == Q8_0>(a, bf, make_int2(sc.x, sc.y), dd);
            const float2 da = make_float2(__int_as_float(sc.z), __int_as_float(sc.w));
            // S exactly (integer < 2^22 below 1.5*2^23); acc += (d_a*d_b)*S
            const float2 s01 = __fadd2_rn(make_float2(__int_as_float(dd[0]), __int_as_float(dd[1])), nmag);
            const float2 s23 = __fadd2_rn(make_float2(__int_as_float(dd[2]), __int_as_float(dd[3])), nmag);
            a01[nt] = __ffma2_rn(__fmul2_rn(da, make_float2(db0, db0)), s01, a01[nt]);
            a23[nt] = __ffma2_rn(__fmul2_rn(da, make_float2(db1, db1)), s23, a23[nt]);
            if (has_min(DT)) {
                const float2 ua = *reinterpret_cast<const float2*>(A.ua + (kb * NT + nt) * 8 + 2 * c);
                a01[nt] = __ffma2_rn(ua, make_float2(mb0, mb0), a01[nt]);
                a23[nt] = __ffma2_rn(ua, make_float2(mb1, mb1), a23[nt]);
            }
        }
    }
}

template <int NT>
__device__ __forceinline__ void mma_store(const float2 (&a01)[NT], const float2 (&a23)[NT], int T, int lane, int M,
                                          int N, const float* __restrict__ bias, float* __restrict__ y) {
    const int g = lane >> 2, c = lane & 3;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const float v[4] = {a01[nt].x, a01[nt].y, a23[nt].x, a23[nt].y};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int row = T * 16 + g + ((i & 2) ? 8 : 0), col = nt * 8 + 2 * c + (i & 1);
            if (row < N && col < M) y[size_t(col) * N + row] = bias ? __fadd_rn(v[i], __ldg(bias + row)) : v[i];
        }
    }
}

// Per-warp shared-memory ring of weight groups, filled with cp.async so
// that the data in flight costs no registers.  Slot layout (one 4-block
// group of the warp's 16 rows): codes [16 rows][4 lanes][QSB] (the 16- or
// 32-byte share of quad lane c), then qh [16][16 B], d [16][8 B],
// m [16][8 B].
template <int DT>
struct Slot {
    static constexpr int Q = 16 * 4 * qs_bytes(DT);
    static constexpr int QH = Q, D = Q + 256, M = Q + 384, BYTES = Q + 512;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

// Request group G of tile T into the slot at shared address `slot`.
template <int DT>
__device__ __forceinline__ void ring_issue(const uint8_t* __restrict__ qs, const uint32_t* __restrict__ qh,
                                           const uint16_t* __restrict__ dp, const uint16_t* __restrict__ mp, int N,
                                           int nb4, int T, int G, int lane, uint32_t slot) {
    // Rows past N re-read row N-1 (their sums are never stored).  Offsets
    // fit 32 bits: the host checks n * nb4 * qs_bytes < 2^32.
    const int g = lane >> 2, c = lane & 3;
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        const int r = g + 8 * rr, row = min(T * 16 + r, N - 1);
        const uint32_t pb = uint32_t(row) * uint32_t(nb4) + uint32_t(4 * G);
        const uint8_t* src = qs + (pb * qs_bytes(DT) + uint32_t(c * qs_bytes(DT)));
        const uint32_t dst = slot + uint32_t((r * 4 + c) * qs_bytes(DT));
        cp_async16(dst, src);
        if (DT == Q8_0) cp_async16(dst + 16, src + 16);
    }
    const int r = lane & 15, row = min(T * 16 + r, N - 1);
    const uint32_t pb = uint32_t(row) * uint32_t(nb4) + uint32_t(4 * G);
    if (lane < 16) {
        if (has_qh(DT)) cp_async16(slot + Slot<DT>::QH + r * 16, qh + pb);
        if (has_min(DT)) cp_async8(slot + Slot<DT>::M + r * 8, mp + pb);
    } else {
        cp_async8(slot + Slot<DT>::D + r * 8, dp + pb);
    }
}

// This lane's share of a landed slot, into registers.
template <int DT>
__device__ __forceinline__ void ring_read(const uint8_t* slot, int lane, MmaGroup<DT>& r) {
    const int g = lane >> 2, c = lane & 3;
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
        const int row = g + 8 * rr;
        const uint4 v = *reinterpret_cast<const uint4*>(slot + (row * 4 + c) * qs_bytes(DT));
        r.q[rr][0] = v.x; r.q[rr][1] = v.y; r.q[rr][2] = v.z; r.q[rr][3] = v.w;
        if (DT == Q8_0) {
            const uint4 v2 = *reinterpret_cast<const uint4*>(slot + (row * 4 + c) * qs_bytes(DT) + 16);
            r.q[rr][4 % (qs_bytes(DT) / 4)] = v2.x; r.q[rr][5 % (qs_bytes(DT) / 4)] = v2.y;
            r.q[rr][6 % (qs_bytes(DT) / 4)] = v2.z; r.q[rr][7 % (qs_bytes(DT) / 4)] = v2.w;
        }
        if (has_qh(DT)) {
            const uint4 h = *reinterpret_cast<const uint4*>(slot + Slot<DT>::QH + row * 16);
            r.h[rr][0] = h.x; r.h[rr][1 % 4] = h.y; r.h[rr][2 % 4] = h.z; r.h[rr][3 % 4] = h.w;
        }
        r.d[rr] = *reinterpret_cast<const uint2*>(slot + Slot<DT>::D + row * 8);
        if (has_min(DT)) r.m[rr] = *reinterpret_cast<const uint2*>(slot + Slot<DT>::M + row * 8);
    }
}

// Shared memory of k_gemv_mma for NT n-tiles: per block and n-tile the B
// fragments (256 B), seed/d_a records (64 B) and d_a*sum(q_a) (32 B); the
// partial-sum buffer (4 KB per n-tile); then each warp's weight ring.
__host__ __device__ constexpr size_t gemv_mma_act_smem(int nb, int nt) {
    return size_t(round4(nb)) * size_t(nt) * 352 + size_t(nt) * 4096;
}

// PF groups in flight per warp; NT n-tiles of 8 activation rows per CTA:
// CTA row blockIdx.y takes activation rows [8*NT*y, 8*NT*(y+1)) of the M
// (the CTAs of different rows share the weights through L2).
template <int DT, int KS, int PF, int NT>
__global__ void __launch_bounds__(GM_THREADS, 1)
    k_gemv_mma(const uint8_t* __restrict__ qs, const uint32_t* __restrict__ qh, const uint16_t* __restrict__ dp,
               const uint16_t* __restrict__ mp, const int8_t* __restrict__ q8, const float* __restrict__ da,
               const int32_t* __restrict__ sa, const float* __restrict__ ua, int M, int N, int K,
               const float* __restrict__ bias, float* __restrict__ y) {
    constexpr int pf = PF;
    pdl_trigger();
    constexpr int WARPS = GM_THREADS / 32;
    const int nb = K / QK, nb4 = round4(nb), ng = nb4 / 4;
    {
        const int row0 = int(blockIdx.y) * 8 * NT;
        M = min(M - row0, 8 * NT);
        q8 += size_t(row0) * K;
        da += size_t(row0) * nb;
        sa += size_t(row0) * nb;
        ua += size_t(row0) * nb;
        y += size_t(row0) * N;
    }
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int tiles = (N + 15) / 16;

    extern __shared__ __align__(16) uint8_t smem[];
    uint2* s_frag = reinterpret_cast<uint2*>(smem);                          // [nb4][NT][32]
    int* s_sc = reinterpret_cast<int*>(smem + size_t(nb4) * NT * 256);        // [nb4][NT][4 lanes][seed, seed, d_a, d_a]
    float* s_ua = reinterpret_cast<float*>(s_sc + nb4 * NT * 16);             // [nb4][NT][8]
    float* s_red = s_ua + nb4 * NT * 8;                                       // [8 warps][32 lanes][NT][4]
    uint8_t* ring = reinterpret_cast<uint8_t*>(s_red + WARPS * 32 * 4 * NT) + size_t(warp) * pf * Slot<DT>::BYTES;
    const uint32_t ring_s = uint32_t(__cvta_generic_to_shared(ring));
    const MmaActs A{s_frag, reinterpret_cast<const int4*>(s_sc), s_ua};

    auto stage = [&]() {
        pdl_wait();
        // Only entries of existing rows and blocks are copied: the other
        // columns' sums are never stored.
        for (int i = tid; i < nb * M * 4; i += GM_THREADS) {
            const int cc = i & 3, row = (i >> 2) % M, kb = (i >> 2) / M;
            const int8_t* p = q8 + size_t(row) * K + kb * QK + 4 * cc;
            uint2* dst = s_frag + (kb * NT + (row >> 3)) * 32 + (row & 7) * 4 + cc;
            cp_async4(&dst->x, p, true);
            cp_async4(&dst->y, p + 16, true);
        }
        // record of (kb, act row col): {0,1} seed, {2,3} d_a of rows 2c, 2c+1
        auto sc_at = [&](int kb, int col, int f) {
            return s_sc + ((kb * NT + (col >> 3)) * 4 + ((col & 7) >> 1)) * 4 + 2 * f + (col & 1);
        };
        for (int i = tid; i < nb * M; i += GM_THREADS) {
            const int col = i % M, kb = i / M;
            const size_t o = size_t(col) * nb + kb;
            if (code_offset(DT)) cp_async4(sc_at(kb, col, 0), sa + o, true);
            cp_async4(sc_at(kb, col, 1), da + o, true);
            if (has_min(DT)) cp_async4(s_ua + (kb * NT + (col >> 3)) * 8 + (col & 7), ua + o, true);
        }
        // Pad blocks: zero codes, zero scales, seed 1.5*2^23 -> add 0.
        for (int i = tid; i < (nb4 - nb) * NT * 32; i += GM_THREADS) {
            const int kb = nb + i / (NT * 32), nt = (i / 32) % NT, l = i & 31;
            s_frag[(kb * NT + nt) * 32 + l] = make_uint2(0u, 0u);
            if (l < 8) {
                *sc_at(kb, nt * 8 + l, 0) = int(MAGIC_BITS);
                *reinterpret_cast<float*>(sc_at(kb, nt * 8 + l, 1)) = 0.f;
                s_ua[(kb * NT + nt) * 8 + l] = 0.f;
            }
        }
        cp_async_wait_all();
        __syncthreads();
        for (int i = tid; i < nb * M; i += GM_THREADS) {
            int* p = sc_at(i / M, i % M, 0);
            *p = code_offset(DT) ? int(MAGIC_BITS - uint32_t(code_offset(DT) * *p)) : int(MAGIC_BITS);
        }
        __syncthreads();
    };

    // One item: wait for its slot, read it, refill the slot with the item
    // pf places ahead (or commit an empty group, so the pending count stays
    // pf - 1), then run the block MMAs.
    MmaGroup<DT> cur;
    float2 a01[NT], a23[NT];
    auto zero = [&]() {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) a01[nt] = a23[nt] = make_float2(0.f, 0.f);
    };
    auto consume = [&](int u, int G, bool refill, int nT, int nG) {
        asm volatile("cp.async.wait_group %0;" ::"n"(PF - 1) : "memory");
        __syncwarp();
        ring_read<DT>(ring + u * Slot<DT>::BYTES, lane, cur);
        __syncwarp();
        if (refill) ring_issue<DT>(qs, qh, dp, mp, N, nb4, nT, nG, lane, ring_s + u * Slot<DT>::BYTES);
        cp_async_commit();
        mma_compute<DT, NT>(cur, A, G, lane, a01, a23);
    };
    float4* red_me = reinterpret_cast<float4*>(s_red) + (warp * 32 + lane) * NT;
    auto park = [&](float4* dst) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) dst[nt] = make_float4(a01[nt].x, a01[nt].y, a23[nt].x, a23[nt].y);
    };
    auto add_parked = [&](const float4* src) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const float4 t = src[nt];
            a01[nt] = __fadd2_rn(a01[nt], make_float2(t.x, t.y));
            a23[nt] = __fadd2_rn(a23[nt], make_float2(t.z, t.w));
        }
    };

    if (KS == 1) {
        // The CTA owns the contiguous tiles [t_lo, t_hi); its warps split
        // the (tile, group) items evenly into contiguous ranges.  With at
        // least 8 tiles per CTA every range holds a full tile's groups, so
        // a tile is shared by at most two neighbouring warps: the first
        // ends with its head (groups 0..x-1), the next starts with its
        // tail (x..); the tail is passed through shared memory and the
        // head's owner stores head + tail.  Fewer tiles: whole tiles.
        const int t_lo = int(int64_t(blockIdx.x) * tiles / gridDim.x);
        const int t_hi = int(int64_t(blockIdx.x + 1) * tiles / gridDim.x);
        const int nt_ = t_hi - t_lo, items = nt_ * ng;
        int i_lo, i_hi;
        if (nt_ >= WARPS) {
            i_lo = warp * items / WARPS;
            i_hi = (warp + 1) * items / WARPS;
        } else {
            i_lo = min(warp, nt_) * ng;
            i_hi = min(warp + 1, nt_) * ng;
        }
        const int n_items = i_hi - i_lo;
        int lt = t_lo + i_lo / ng, lG = i_lo % ng;
        int ct = lt, cG = lG;
        const int shared_first = lG != 0 ? lt : -1;   // tile whose head the previous warp holds
        for (int u = 0; u < pf; ++u) {
            if (u < n_items) {
                ring_issue<DT>(qs, qh, dp, mp, N, nb4, lt, lG, lane, ring_s + u * Slot<DT>::BYTES);
                if (++lG == ng) { lG = 0; ++lt; }
            }
            cp_async_commit();
        }
        stage();
        zero();
        for (int i0 = 0; i0 < n_items; i0 += PF) {
#pragma unroll
            for (int u = 0; u < PF; ++u) {
                const int i = i0 + u;
                if (i >= n_items) break;
                const bool refill = i + pf < n_items;
                consume(u, cG, refill, lt, lG);
                if (refill && ++lG == ng) { lG = 0; ++lt; }
                if (++cG == ng) {
                    if (ct == shared_first) park(red_me);
                    else mma_store<NT>(a01, a23, ct, lane, M, N, bias, y);
                    zero();
                    cG = 0;
                    ++ct;
                }
            }
        }
        __syncthreads();
        if (n_items > 0 && cG != 0) {   // this warp holds the head of tile ct; warp + 1 its tail
            add_parked(reinterpret_cast<const float4*>(s_red) + ((warp + 1) * 32 + lane) * NT);
            mma_store<NT>(a01, a23, ct, lane, M, N, bias, y);
        }
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        return;
    }

    // KS > 1: the CTA's warps form (8/KS) tiles x KS K-slices; each CTA
    // iteration ends with a slice-ordered reduction in shared memory.
    constexpr int TPC = WARPS / KS;
    const int ks = warp % KS, tw = warp / KS;
    const int g0 = ks * ng / KS, gn = (ks + 1) * ng / KS - g0;
    int base = blockIdx.x * TPC;
    for (bool first = true; base < tiles; base += gridDim.x * TPC, first = false) {
        const int T = base + tw;
        for (int u = 0; u < pf; ++u) {
            if (u < gn) ring_issue<DT>(qs, qh, dp, mp, N, nb4, T, g0 + u, lane, ring_s + u * Slot<DT>::BYTES);
            cp_async_commit();
        }
        if (first) stage();
        zero();
        for (int i0 = 0; i0 < gn; i0 += PF) {
#pragma unroll
            for (int u = 0; u < PF; ++u) {
                const int i = i0 + u;
                if (i >= gn) break;
                consume(u, g0 + i, i + pf < gn, T, g0 + i + pf);
            }
        }
        park(red_me);
        __syncthreads();
        if (ks == 0) {
#pragma unroll
            for (int s2 = 1; s2 < KS; ++s2) add_parked(reinterpret_cast<const float4*>(s_red) + ((warp + s2) * 32 + lane) * NT);
            mma_store<NT>(a01, a23, T, lane, M, N, bias, y);
        }
        __syncthreads();
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// ------------------------------------------------------------ GEMV tiles
// The GEMV family at many activation rows (one decoder step over many
// streams): the integer-MMA arithmetic of k_gemv_mma, tiled like a GEMM so
// that each decoded weight fragment serves 8*NT activation rows and each
// staged activation fragment 16*WN weight rows.  A CTA of 2 x 2 warps owns
// BN = 32*WN weight rows x BM = 16*NT activation rows and walks K one
// 4-block group at a time through a cp.async ring of GT_STAGES groups
// (weight codes/qh/d/m as in the planes; activation codes row-major with a
// 144-byte row pitch, so the B-fragment words of 8 rows x 4 quad lanes
// fall in 32 distinct banks; sum(q_a), d_a, d_a*sum(q_a) as [row][4]).
//
// Every output accumulates its blocks in kb order with exactly the
// operations of k_gemv_mma, and the K ranges that k_gemv_mma gives to
// different warps are accumulated separately here and added in the same
// order: for KS > 1 each of its K slices is one CTA of a cluster of KS
// CTAs, whose partial tiles are added in slice order through distributed
// shared memory (each CTA adds and stores 1/KS of the tile); for KS == 1
// the head/tail split of a tile shared by two of its warps is reproduced
// inside the CTA.  The results are therefore bit-identical to k_gemv_mma's
// for every m, and a row's result stays independent of m across the whole
// GEMV family (quant.rs:1372-1384).
constexpr int GT_THREADS = 128;
constexpr int GT_STAGES = 4;
constexpr int GT_APITCH = 144;   // activation code bytes per row in shared memory

template <int DT, int WN, int NT>
struct TileSmem {
    static constexpr int BN = 32 * WN, BM = 16 * NT;
    static constexpr int QROW = 4 * qs_bytes(DT) + (DT == Q8_0 ? 16 : 0);   // padded for Q8_0 (bank spread)
    static constexpr int WQ = 0;
    static constexpr int WH = WQ + BN * QROW;
    static constexpr int WD = WH + (has_qh(DT) ? BN * 16 : 0);
    static constexpr int WM = WD + BN * 8;
    static constexpr int AQ = WM + (has_min(DT) ? BN * 8 : 0);
    static constexpr int AS = AQ + BM * GT_APITCH;                       // sum(q_a)  [BM][4] int
    static constexpr int AD = AS + (code_offset(DT) ? BM * 16 : 0);      // d_a       [BM][4] f32
    static constexpr int AU = AD + BM * 16;                              // d_a*sum   [BM][4] f32
    static constexpr int STAGE = AU + (has_min(DT) ? BM * 16 : 0);
    static constexpr int BYTES = GT_STAGES * STAGE;
};

__device__ __forceinline__ void gt_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Exit guard only (no memory ordering needed: the peers' reads of this
// CTA's shared memory have returned their values before they arrive).
__device__ __forceinline__ void gt_cluster_sync_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}
// Shared::cluster address of shared byte offset `off` in cluster CTA `rank`.
__device__ __forceinline__ uint32_t gt_mapa(uint32_t off, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(off), "r"(rank));
    return r;
}
// (No memory clobber: the loads of one output's slices are issued back to
// back; the cluster barriers order them against the partials' writes.)
__device__ __forceinline__ float4 gt_ld_cluster4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

__device__ __forceinline__ void cp_async16z(uint32_t dst, const void* src, bool ok) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(ok ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async4z(uint32_t dst, const void* src, bool ok) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(ok ? 4 : 0) : "memory");
}

template <int DT, int WN, int NT, bool CL>
__global__ void __launch_bounds__(GT_THREADS, 3)
    k_gemv_tile(const uint8_t* __restrict__ qs, const uint32_t* __restrict__ qh, const uint16_t* __restrict__ dp,
                const uint16_t* __restrict__ mp, const int8_t* __restrict__ q8, const float* __restrict__ da,
                const int32_t* __restrict__ sa, const float* __restrict__ ua, int M, int N, int K,
                const float* __restrict__ bias, float* __restrict__ y, int ks, int gx, int vec16) {
    using L = TileSmem<DT, WN, NT>;
    constexpr int QSB = qs_bytes(DT), WCH = 4 * QSB / 16;   // 16-byte chunks of one row's group codes
    pdl_trigger();
    const int nb = K / QK, nb4 = round4(nb), ng = nb4 / 4, tiles = (N + 15) / 16;
    // ks > 1: the launch has clusters of ks CTAs along x, CTA `rank` of a
    // cluster takes K slice `rank`; ks == 1: one CTA takes all of K.
    const int cs = CL ? ks : 1, rank = int(blockIdx.x) % cs;
    const int g_lo = rank * ng / cs, g_hi = (rank + 1) * ng / cs;
    const int n0 = int(blockIdx.x) / cs * L::BN, m0 = int(blockIdx.y) * L::BM;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, wn = warp & 1, wm = warp >> 1;
    const int g = lane >> 2, c = lane & 3;

    extern __shared__ __align__(16) uint8_t smem[];
    const uint32_t sbase = uint32_t(__cvta_generic_to_shared(smem));

    auto issue_w = [&](int G, int slot) {
        const uint32_t st = sbase + uint32_t(slot * L::STAGE);
        for (int i = tid; i < L::BN * WCH; i += GT_THREADS) {
            const int r = i / WCH, ch = i % WCH, row = min(n0 + r, N - 1);
            const uint8_t* src = qs + ((size_t(row) * nb4 + size_t(4 * G)) * QSB + ch * 16);
            cp_async16(st + L::WQ + r * L::QROW + ch * 16, src);
        }
        for (int r = tid; r < L::BN; r += GT_THREADS) {
            const size_t pb = size_t(min(n0 + r, N - 1)) * nb4 + size_t(4 * G);
            if (has_qh(DT)) cp_async16(st + L::WH + r * 16, qh + pb);
            cp_async8(st + L::WD + r * 8, dp + pb);
            if (has_min(DT)) cp_async8(st + L::WM + r * 8, mp + pb);
        }
    };
    auto issue_a = [&](int G, int slot) {
        const uint32_t st = sbase + uint32_t(slot * L::STAGE);
        for (int i = tid; i < L::BM * 8; i += GT_THREADS) {
            const int r = i >> 3, ch = i & 7, row = m0 + r;
            const bool ok = row < M && 4 * G + (ch >> 1) < nb;
            const int8_t* src = ok ? q8 + (size_t(row) * K + size_t(128 * G) + ch * 16) : q8;
            cp_async16z(st + L::AQ + r * GT_APITCH + ch * 16, src, ok);
        }
        if (vec16) {   // nb % 4 == 0: every group is whole
            for (int r = tid; r < L::BM; r += GT_THREADS) {
                const bool ok = m0 + r < M;
                const size_t o = ok ? size_t(m0 + r) * nb + size_t(4 * G) : 0;
                if (code_offset(DT)) cp_async16z(st + L::AS + r * 16, sa + o, ok);
                cp_async16z(st + L::AD + r * 16, da + o, ok);
                if (has_min(DT)) cp_async16z(st + L::AU + r * 16, ua + o, ok);
            }
        } else {       // pad blocks (kb >= nb) read as zeros: seed 1.5*2^23, scales 0
            for (int i = tid; i < L::BM * 4; i += GT_THREADS) {
                const int r = i >> 2, b = i & 3;
                const bool ok = m0 + r < M && 4 * G + b < nb;
                const size_t o = ok ? size_t(m0 + r) * nb + size_t(4 * G + b) : 0;
                if (code_offset(DT)) cp_async4z(st + L::AS + i * 4, sa + o, ok);
                cp_async4z(st + L::AD + i * 4, da + o, ok);
                if (has_min(DT)) cp_async4z(st + L::AU + i * 4, ua + o, ok);
            }
        }
    };

    // CL (clusters): the CTA's K range is one slice, its sum is a partial.
    // Otherwise `tot` holds the finished slices of a tile and `part` (q02,
    // q13) the running one.  Accumulator pairs: q02 = (row g, row g+8) at
    // column 2c, q13 = the same rows at column 2c+1.
    float2 q02[WN][NT], q13[WN][NT];
    float2 t02[CL ? 1 : WN][CL ? 1 : NT], t13[CL ? 1 : WN][CL ? 1 : NT];
    int nsl[WN], nxt[WN];
#pragma unroll
    for (int mt = 0; mt < WN; ++mt) {
        nsl[mt] = 0;
        nxt[mt] = CL ? (1 << 30) : gemv_slice_start((n0 >> 4) + wn * WN + mt, 1, ks, ng, gx, tiles);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) q02[mt][nt] = q13[mt][nt] = make_float2(0.f, 0.f);
    }
    auto close_slice = [&](int mt) {
        if constexpr (!CL) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                if (nsl[mt] == 0) {
                    t02[mt][nt] = q02[mt][nt];
                    t13[mt][nt] = q13[mt][nt];
                } else {
                    t02[mt][nt] = __fadd2_rn(t02[mt][nt], q02[mt][nt]);
                    t13[mt][nt] = __fadd2_rn(t13[mt][nt], q13[mt][nt]);
                }
                q02[mt][nt] = q13[mt][nt] = make_float2(0.f, 0.f);
            }
            ++nsl[mt];
            nxt[mt] = gemv_slice_start((n0 >> 4) + wn * WN + mt, nsl[mt] + 1, ks, ng, gx, tiles);
        }
    };

    const int n_g = g_hi - g_lo;
    for (int u = 0; u < GT_STAGES - 1; ++u)
        if (u < n_g) issue_w(g_lo + u, u);
    pdl_wait();
    for (int u = 0; u < GT_STAGES - 1; ++u) {
        if (u < n_g) issue_a(g_lo + u, u);
        cp_async_commit();
    }

    const float2 nmag = make_float2(-MAGIC_F, -MAGIC_F);
    for (int i = 0; i < n_g; ++i) {
        const int G = g_lo + i;
        asm volatile("cp.async.wait_group %0;" ::"n"(GT_STAGES - 2) : "memory");
        __syncthreads();
        {
            const int in = i + GT_STAGES - 1;
            if (in < n_g) {
                issue_w(g_lo + in, in % GT_STAGES);
                issue_a(g_lo + in, in % GT_STAGES);
            }
            cp_async_commit();
        }
        if constexpr (!CL) {
#pragma unroll
            for (int mt = 0; mt < WN; ++mt)
                while (G == nxt[mt]) close_slice(mt);
        }

        const uint8_t* st = smem + (i % GT_STAGES) * L::STAGE;
        // Weight fragments of this warp's m-tiles, decoded for all 4 blocks;
        // d_b (m_b) of rows g and g+8 as pairs.
        uint32_t a[WN][4][4];
        float2 dbp[WN][4], mbp[WN][4];
#pragma unroll
        for (int mt = 0; mt < WN; ++mt) {
            MmaGroup<DT> r;
            float dbv[2][4], mbv[2][4];
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                const int row = (wn * WN + mt) * 16 + g + 8 * rr;
                const uint8_t* q = st + L::WQ + row * L::QROW + c * QSB;
                const uint4 v = *reinterpret_cast<const uint4*>(q);
                r.q[rr][0] = v.x; r.q[rr][1] = v.y; r.q[rr][2] = v.z; r.q[rr][3] = v.w;
                if (DT == Q8_0) {
                    const uint4 v2 = *reinterpret_cast<const uint4*>(q + 16);
                    r.q[rr][4 % (QSB / 4)] = v2.x; r.q[rr][5 % (QSB / 4)] = v2.y;
                    r.q[rr][6 % (QSB / 4)] = v2.z; r.q[rr][7 % (QSB / 4)] = v2.w;
                }
                if (has_qh(DT)) {
                    const uint4 h = *reinterpret_cast<const uint4*>(st + L::WH + row * 16);
                    r.h[rr][0] = h.x; r.h[rr][1 % 4] = h.y; r.h[rr][2 % 4] = h.z; r.h[rr][3 % 4] = h.w;
                }
                const uint2 dw = *reinterpret_cast<const uint2*>(st + L::WD + row * 8);
                const float2 d01 = h2f2(dw.x), d23 = h2f2(dw.y);
                dbv[rr][0] = d01.x; dbv[rr][1] = d01.y; dbv[rr][2] = d23.x; dbv[rr][3] = d23.y;
                if (has_min(DT)) {
                    const uint2 mw = *reinterpret_cast<const uint2*>(st + L::WM + row * 8);
                    const float2 m01 = h2f2(mw.x), m23 = h2f2(mw.y);
                    mbv[rr][0] = m01.x; mbv[rr][1] = m01.y; mbv[rr][2] = m23.x; mbv[rr][3] = m23.y;
                }
            }
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                dbp[mt][b] = make_float2(dbv[0][b], dbv[1][b]);
                if (has_min(DT)) mbp[mt][b] = make_float2(mbv[0][b], mbv[1][b]);
                if (DT == Q8_0) {
                    a[mt][b][0] = r.q[0][(2 * b) % (QSB / 4)];
                    a[mt][b][1] = r.q[1][(2 * b) % (QSB / 4)];
                    a[mt][b][2] = r.q[0][(2 * b + 1) % (QSB / 4)];
                    a[mt][b][3] = r.q[1][(2 * b + 1) % (QSB / 4)];
                } else {
#pragma unroll
                    for (int rr = 0; rr < 2; ++rr) {
                        const uint32_t w = r.q[rr][b % (QSB / 4)];
                        uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
                        if (has_qh(DT)) {
                            const uint32_t h = r.h[rr][b % (has_qh(DT) ? 4 : 1)];
                            lo |= (h << (4 - c)) & 0x10101010u;
                            hi |= (h >> c) & 0x10101010u;
                        }
                        a[mt][b][rr] = lo;
                        a[mt][b][2 + rr] = hi;
                    }
                }
            }
        }
        // Activation n-tiles: B fragments (row g of the n-tile, words c and
        // 4+c of each block) and the scales of columns 2c, 2c+1.  The MMAs
        // of all blocks and m-tiles issue first; the f32 updates follow, in
        // kb order for every output.
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int col = (wm * NT + nt) * 8;
            const uint8_t* aq = st + L::AQ + (col + g) * GT_APITCH + 4 * c;
            const int r0 = col + 2 * c;
            int4 s0 = make_int4(0, 0, 0, 0), s1 = make_int4(0, 0, 0, 0);
            if (code_offset(DT)) {
                s0 = *reinterpret_cast<const int4*>(st + L::AS + r0 * 16);
                s1 = *reinterpret_cast<const int4*>(st + L::AS + (r0 + 1) * 16);
            }
            const int sx[4] = {s0.x, s0.y, s0.z, s0.w}, sy[4] = {s1.x, s1.y, s1.z, s1.w};
            const float4 d0 = *reinterpret_cast<const float4*>(st + L::AD + r0 * 16);
            const float4 d1 = *reinterpret_cast<const float4*>(st + L::AD + (r0 + 1) * 16);
            float4 u0 = make_float4(0.f, 0.f, 0.f, 0.f), u1 = u0;
            if (has_min(DT)) {
                u0 = *reinterpret_cast<const float4*>(st + L::AU + r0 * 16);
                u1 = *reinterpret_cast<const float4*>(st + L::AU + (r0 + 1) * 16);
            }
            const float dx[4] = {d0.x, d0.y, d0.z, d0.w}, dy[4] = {d1.x, d1.y, d1.z, d1.w};
            const float ux[4] = {u0.x, u0.y, u0.z, u0.w}, uy[4] = {u1.x, u1.y, u1.z, u1.w};
            // Blocks in batches of MB: MB * WN MMAs in flight before their
            // f32 updates (fewer where the slice totals hold registers).
            constexpr int MB = (CL || WN * NT <= 4) ? 4 : 2;
#pragma unroll
            for (int b0 = 0; b0 < 4; b0 += MB) {
                int dd[MB][WN][4];
#pragma unroll
                for (int bb = 0; bb < MB; ++bb) {
                    const int b = b0 + bb;
                    const uint2 bf = make_uint2(*reinterpret_cast<const uint32_t*>(aq + b * 32),
                                                *reinterpret_cast<const uint32_t*>(aq + b * 32 + 16));
                    const int2 ci = code_offset(DT)
                                        ? make_int2(int(MAGIC_BITS - uint32_t(code_offset(DT) * sx[b])),
                                                    int(MAGIC_BITS - uint32_t(code_offset(DT) * sy[b])))
                                        : make_int2(int(MAGIC_BITS), int(MAGIC_BITS));
#pragma unroll
                    for (int mt = 0; mt < WN; ++mt) mma_i8<DT == Q8_0>(a[mt][b], bf, ci, dd[bb][mt]);
                }
#pragma unroll
                for (int bb = 0; bb < MB; ++bb) {
                    const int b = b0 + bb;
                    const float2 da0 = make_float2(dx[b], dx[b]), da1 = make_float2(dy[b], dy[b]);
#pragma unroll
                    for (int mt = 0; mt < WN; ++mt) {
                        // S exactly, then acc <- fma(d_a*d_b, S, acc) (+ fma(d_a*sum, m_b, acc))
                        const float2 s02 = __fadd2_rn(
                            make_float2(__int_as_float(dd[bb][mt][0]), __int_as_float(dd[bb][mt][2])), nmag);
                        const float2 s13 = __fadd2_rn(
                            make_float2(__int_as_float(dd[bb][mt][1]), __int_as_float(dd[bb][mt][3])), nmag);
                        q02[mt][nt] = __ffma2_rn(__fmul2_rn(dbp[mt][b], da0), s02, q02[mt][nt]);
                        q13[mt][nt] = __ffma2_rn(__fmul2_rn(dbp[mt][b], da1), s13, q13[mt][nt]);
                        if (has_min(DT)) {
                            q02[mt][nt] = __ffma2_rn(mbp[mt][b], make_float2(ux[b], ux[b]), q02[mt][nt]);
                            q13[mt][nt] = __ffma2_rn(mbp[mt][b], make_float2(uy[b], uy[b]), q13[mt][nt]);
                        }
                    }
                }
            }
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    if constexpr (CL) {
        // This CTA's slice partial -> own shared memory [BM][BN]; after the
        // cluster barrier CTA `rank` adds the slices of its share of the
        // tile in slice order (k_gemv_mma's order) and stores it.
        __syncthreads();
        float* part = reinterpret_cast<float*>(smem);
#pragma unroll
        for (int mt = 0; mt < WN; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int rl = (wn * WN + mt) * 16 + g, cl = (wm * NT + nt) * 8 + 2 * c;
                part[cl * L::BN + rl] = q02[mt][nt].x;
                part[cl * L::BN + rl + 8] = q02[mt][nt].y;
                part[(cl + 1) * L::BN + rl] = q13[mt][nt].x;
                part[(cl + 1) * L::BN + rl + 8] = q13[mt][nt].y;
            }
        gt_cluster_sync();
        constexpr int Q4 = L::BN * L::BM / 4;
        const int q_lo = rank * Q4 / cs, q_hi = (rank + 1) * Q4 / cs;
        for (int q = q_lo + tid; q < q_hi; q += GT_THREADS) {
            const uint32_t off = sbase + uint32_t(q * 16);
            float4 t[8];
#pragma unroll
            for (int s2 = 0; s2 < 8; ++s2)
                if (s2 < cs) t[s2] = gt_ld_cluster4(gt_mapa(off, uint32_t(s2)));
            float4 v = t[0];
#pragma unroll
            for (int s2 = 1; s2 < 8; ++s2)
                if (s2 < cs) {
                    v.x = __fadd_rn(v.x, t[s2].x); v.y = __fadd_rn(v.y, t[s2].y);
                    v.z = __fadd_rn(v.z, t[s2].z); v.w = __fadd_rn(v.w, t[s2].w);
                }
            const int col = m0 + 4 * q / L::BN, row = n0 + 4 * q % L::BN;
            const float vv[4] = {v.x, v.y, v.z, v.w};
            if (col < M) {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (row + j < N) y[size_t(col) * N + row + j] = bias ? __fadd_rn(vv[j], __ldg(bias + row + j)) : vv[j];
            }
        }
        gt_cluster_sync_relaxed();   // no CTA leaves while its partial is being read
    } else {
#pragma unroll
        for (int mt = 0; mt < WN; ++mt) {
            close_slice(mt);
            const int T = (n0 >> 4) + wn * WN + mt;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                // (row g, col 2c), (row g+8, col 2c), (row g, col 2c+1), (row g+8, col 2c+1)
                const float v[4] = {t02[mt][nt].x, t02[mt][nt].y, t13[mt][nt].x, t13[mt][nt].y};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int row = T * 16 + g + ((i & 1) ? 8 : 0);
                    const int col = m0 + (wm * NT + nt) * 8 + 2 * c + (i >> 1);
                    if (row < N && col < M) y[size_t(col) * N + row] = bias ? __fadd_rn(v[i], __ldg(bias + row)) : v[i];
                }
            }
        }
    }
}

// ------------------------------------------------------------- GEMV f32
// Dequant-then-fp path (the f32 tier, quant.rs:995-1018): weights
// dequantized bit-exactly, dotted with unquantized f32 activations.
template <int DT, int L, int MR>
__global__ void __launch_bounds__(TPB) k_gemv_f32(const uint8_t* __restrict__ qs, const uint32_t* __restrict__ qh,
                                                  const uint16_t* __restrict__ dp, const uint16_t* __restrict__ mp,
                                                  const float* __restrict__ a, int M, int N, int K,
                                                  const float* __restrict__ bias, float* __restrict__ y) {
    const int nb = K / QK;
    const int lane = threadIdx.x & 31, sub = lane % L, slot = lane / L;
    constexpr int RPW = 32 / L;
    const int warps_per_cta = blockDim.x >> 5;
    const int gw = blockIdx.x * warps_per_cta + (threadIdx.x >> 5);
    const int nw = gridDim.x * warps_per_cta;
    for (int row0 = gw * RPW; row0 < N; row0 += nw * RPW) {
        const int j = row0 + slot;
        float acc[MR];
#pragma unroll
        for (int r = 0; r < MR; ++r) acc[r] = 0.f;
        if (j < N) {
            for (int kb = sub; kb < nb; kb += L) {
                BlockCodes<DT> bc;
                load_block<DT>(qs, qh, dp, mp, size_t(j), kb, round4(nb), bc);
                float w[QK];
#pragma unroll
                for (int e = 0; e < QK; ++e) w[e] = __fadd_rn(__fmul_rn(bc.d, float(code_at<DT>(bc.w, e))), bc.m);
#pragma unroll
                for (int r = 0; r < MR; ++r) {
                    if (r < M) {
                        const float4* ar = reinterpret_cast<const float4*>(a + size_t(r) * K + size_t(kb) * QK);
#pragma unroll
                        for (int e4 = 0; e4 < QK / 4; ++e4) {
                            const float4 v = __ldg(ar + e4);
                            acc[r] = __fmaf_rn(v.x, w[4 * e4 + 0], acc[r]);
                            acc[r] = __fmaf_rn(v.y, w[4 * e4 + 1], acc[r]);
                            acc[r] = __fmaf_rn(v.z, w[4 * e4 + 2], acc[r]);
                            acc[r] = __fmaf_rn(v.w, w[4 * e4 + 3], acc[r]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int r = 0; r < MR; ++r) {
#pragma unroll
            for (int o = L / 2; o > 0; o >>= 1) acc[r] = __fadd_rn(acc[r], __shfl_xor_sync(0xffffffffu, acc[r], o));
        }
        if (j < N && sub == 0) {
            const float b = bias ? __ldg(bias + j) : 0.f;
#pragma unroll
            for (int r = 0; r < MR; ++r)
                if (r < M) y[size_t(r) * N + j] = bias ? __fadd_rn(acc[r], b) : acc[r];
        }
    }
}

// ----------------------------------------------------- GEMM operand cache
// Planes -> f16 centred codes [n][k] + transposed f32 scales [nb][n_pad]
// (the tensor-core GEMM's B operand; the GPU counterpart of the
// reference's cached int8 unpack, quant.rs:589-639).  Padding columns of
// the scale planes are zeroed.
template <int DT>
__global__ void k_build_gemm_cache(const uint8_t* __restrict__ qs, const uint32_t* __restrict__ qh,
                                   const uint16_t* __restrict__ dp, const uint16_t* __restrict__ mp, int n, int nb,
                                   int n_pad, uint16_t* __restrict__ q16, float* __restrict__ dT,
                                   float* __restrict__ mT) {
    size_t t = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= size_t(n_pad) * nb) return;
    const int j = int(t / nb), bl = int(t % nb);
    if (j >= n) {
        dT[size_t(bl) * n_pad + j] = 0.f;
        if (mT) mT[size_t(bl) * n_pad + j] = 0.f;
        return;
    }
    BlockCodes<DT> bc;
    load_block<DT>(qs, qh, dp, mp, size_t(j), bl, round4(nb), bc);
    uint4* o = reinterpret_cast<uint4*>(q16 + size_t(j) * nb * QK + size_t(bl) * QK);
#pragma unroll
    for (int e8 = 0; e8 < QK / 8; ++e8) {
        uint32_t h[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            const int e = 8 * e8 + 2 * p;
            const uint32_t lo = __half_as_ushort(__int2half_rn(code_at<DT>(bc.w, e)));
            const uint32_t hi = __half_as_ushort(__int2half_rn(code_at<DT>(bc.w, e + 1)));
            h[p] = lo | (hi << 16);
        }
        o[e8] = make_uint4(h[0], h[1], h[2], h[3]);
    }
    dT[size_t(bl) * n_pad + j] = bc.d;
    if (mT) mT[size_t(bl) * n_pad + j] = bc.m;
}

// ------------------------------------------------- folded-scale operand
// One warp per weight row j: x = d*q + m for every element (the
// reference's dequant, bit-exact), e_j so that max|x|*2^e_j lies in
// [2^10, 2^11), then x*2^e_j (exact) = hi + lo in f16.  Rows n..n_pad-1
// get colscale 0.
template <int DT>
__global__ void k_build_fold_cache(const uint8_t* __restrict__ qs, const uint32_t* __restrict__ qh,
                                   const uint16_t* __restrict__ dp, const uint16_t* __restrict__ mp, int n, int nb,
                                   int n_pad, uint16_t* __restrict__ bhl, float* __restrict__ colscale) {
    const int lane = threadIdx.x & 31;
    const int j = int((size_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5);
    if (j >= n_pad) return;
    if (j >= n) {
        if (lane == 0) colscale[j] = 0.f;
        return;
    }
    float mx = 0.f;
    for (int kb = lane; kb < nb; kb += 32) {
        BlockCodes<DT> bc;
        load_block<DT>(qs, qh, dp, mp, size_t(j), kb, round4(nb), bc);
#pragma unroll
        for (int e = 0; e < QK; ++e) {
            const float x = __fadd_rn(__fmul_rn(bc.d, float(code_at<DT>(bc.w, e))), bc.m);
            mx = fmaxf(mx, fabsf(x));
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    int ex = 0;
    if (mx > 0.f && isfinite(mx)) {
        int E;
        frexpf(mx, &E);          // mx = f * 2^E, f in [0.5, 1)
        ex = 11 - E;             // mx * 2^ex in [2^10, 2^11)
        ex = max(-120, min(120, ex));
    }
    const float up = ldexpf(1.0f, ex);
    for (int kb = lane; kb < nb; kb += 32) {
        BlockCodes<DT> bc;
        load_block<DT>(qs, qh, dp, mp, size_t(j), kb, round4(nb), bc);
        uint32_t hi2[16], lo2[16];
#pragma unroll
        for (int e = 0; e < QK; e += 2) {
            const float x0 = __fmul_rn(__fadd_rn(__fmul_rn(bc.d, float(code_at<DT>(bc.w, e))), bc.m), up);
            const float x1 = __fmul_rn(__fadd_rn(__fmul_rn(bc.d, float(code_at<DT>(bc.w, e + 1))), bc.m), up);
            const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
            const __half l0 = __float2half_rn(__fsub_rn(x0, __half2float(h0)));
            const __half l1 = __float2half_rn(__fsub_rn(x1, __half2float(h1)));
            hi2[e / 2] = uint32_t(__half_as_ushort(h0)) | (uint32_t(__half_as_ushort(h1)) << 16);
            lo2[e / 2] = uint32_t(__half_as_ushort(l0)) | (uint32_t(__half_as_ushort(l1)) << 16);
        }
        uint4* o = reinterpret_cast<uint4*>(bhl + (size_t(j) * nb + kb) * 64);
#pragma unroll
        for (int i = 0; i < 4; ++i) o[i] = make_uint4(hi2[4 * i], hi2[4 * i + 1], hi2[4 * i + 2], hi2[4 * i + 3]);
#pragma unroll
        for (int i = 0; i < 4; ++i) o[4 + i] = make_uint4(lo2[4 * i], lo2[4 * i + 1], lo2[4 * i + 2], lo2[4 * i + 3]);
    }
    if (lane == 0) colscale[j] = ldexpf(1.0f, -ex);
}

// ------------------------------------------------------------ dispatch
template <template <int> class F, typename... Args>
cudaError_t by_dtype(int dt, Args&&... args) {
    switch (dt) {
        case Q4_0: return F<Q4_0>::run(args...);
        case Q4_1: return F<Q4_1>::run(args...);
        case Q5_0: return F<Q5_0>::run(args...);
        case Q5_1: return F<Q5_1>::run(args...);
        case Q8_0: return F<Q8_0>::run(args...);
        default: return cudaErrorInvalidValue;
    }
}

template <int DT>
struct RepackF {
    static cudaError_t run(const uint8_t* raw, Weight& w, cudaStream_t s) {
        size_t nblk = size_t(w.n) * w.nb;
        if (!nblk) return cudaSuccess;
        k_repack<DT><<<grid_for(nblk, TPB), TPB, 0, s>>>(raw, w.qs, w.qh, w.d, w.m, nblk, w.nb, round4(w.nb));
        return cudaGetLastError();
    }
};

template <int DT>
struct DequantF {
    static cudaError_t run(const Weight& w, const int32_t* rows, int nrows, float* out, cudaStream_t s) {
        size_t work = size_t(nrows) * w.nb;
        if (!work) return cudaSuccess;
        k_dequant_rows<DT><<<grid_for(work, TPB), TPB, 0, s>>>(w.qs, w.qh, w.d, w.m, rows, nrows, w.n, w.nb, out);
        return cudaGetLastError();
    }
};

template <int DT>
struct EmbedF {
    static cudaError_t run(const Weight& w, const int32_t* tokens, int nrows, const float* pos, const int* dpos,
                           float* x, cudaStream_t s) {
        size_t work = size_t(nrows) * w.nb;
        if (!work) return cudaSuccess;
        return launch_pdl(k_embed<DT>, dim3(grid_for(work, TPB)), dim3(TPB), 0, s, w.qs, w.qh, w.d, w.m, tokens,
                          nrows, w.n, w.nb, pos, dpos, x);
    }
};

template <int DT>
struct BlockDotsF {
    static cudaError_t run(const ActsView& v, const Weight& w, int32_t* S, cudaStream_t s) {
        size_t work = size_t(v.m) * w.n * w.nb;
        if (!work) return cudaSuccess;
        k_block_dots<DT><<<grid_for(work, TPB), TPB, 0, s>>>(w.qs, w.qh, w.d, w.m, v.q8, v.sum, v.m, w.n, w.nb, S);
        return cudaGetLastError();
    }
};

template <int DT>
struct FoldCacheF {
    static cudaError_t run(Weight& w, cudaStream_t s) {
        const int np = (w.n + 255) / 256 * 256;  // colscale is allocated to this length
        const size_t threads = size_t(np) * 32;
        k_build_fold_cache<DT><<<grid_for(threads, TPB), TPB, 0, s>>>(w.qs, w.qh, w.d, w.m, w.n, w.nb, np, w.bhl,
                                                                      w.colscale);
        return cudaGetLastError();
    }
};

template <int DT>
struct GemmCacheF {
    static cudaError_t run(Weight& w, cudaStream_t s) {
        size_t work = size_t(w.n_pad) * w.nb;
        k_build_gemm_cache<DT><<<grid_for(work, TPB), TPB, 0, s>>>(w.qs, w.qh, w.d, w.m, w.n, w.nb, w.n_pad, w.q16,
                                                                   w.dT, w.mT);
        return cudaGetLastError();
    }
};

// Lanes per weight row for a row of nb blocks: the widest of 32/16/8 that
// divides nb (all lanes busy), else 8.
inline int lanes_for(int nb) {
    if (nb % 32 == 0 && nb >= 64) return 32;
    if (nb % 16 == 0) return 16;
    if (nb % 8 == 0) return 8;
    return nb >= 32 ? 32 : 8;
}

// Grid for a grid-stride GEMV kernel: one CTA per row group of the
// output, but never more than fit on the GPU at once (a second, partial
// wave would redo a full wave's per-warp work).
template <typename Kern>
unsigned gemv_grid(Kern kern, int n, int L, size_t smem) {
    const int rows_per_cta = (TPB / 32) * (32 / L);
    unsigned g = unsigned((n + rows_per_cta - 1) / rows_per_cta);
    int dev = 0, sms = 148, per_sm = 1;
    dev_sms(&dev, &sms);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, TPB, smem) != cudaSuccess || per_sm < 1)
        per_sm = 1;
    const unsigned cap = unsigned(sms) * unsigned(per_sm);
    return g < 1 ? 1 : (g > cap ? cap : g);
}

template <int DT, int L, int BPL, int MR>
cudaError_t gemv_i8_launch(const ActsView& v, const Weight& w, const float* bias, float* y, cudaStream_t s) {
    constexpr int PF = BPL == 1 ? 3 : (BPL == 2 ? 2 : 1);
    constexpr bool REGA = BPL * MR <= 8;
    size_t smem = 0;
    if (!REGA) {
        smem = size_t(v.m) * v.k + size_t(v.m) * w.nb * 12;
        static int attr_dev_mask = 0;  // one bit per device with the attribute set
        int dev = 0;
        cudaGetDevice(&dev);
        if (!(attr_dev_mask & (1 << dev))) {
            cudaError_t e = cudaFuncSetAttribute(k_gemv_i8<DT, L, BPL, MR, PF, REGA>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
            if (e != cudaSuccess) return e;
            attr_dev_mask |= 1 << dev;
        }
    }
    auto kern = k_gemv_i8<DT, L, BPL, MR, PF, REGA>;
    return launch_pdl(kern, dim3(gemv_grid(kern, w.n, L, smem)), dim3(TPB), smem, s, w.qs, w.qh, w.d, w.m, v.q8, v.d,
                      v.sum, v.u, v.m, w.n, w.k, bias, y);
}

template <int DT, int L, int BPL>
cudaError_t gemv_i8_mr(const ActsView& v, const Weight& w, const float* bias, float* y, cudaStream_t s) {
    if (v.m <= 1) return gemv_i8_launch<DT, L, BPL, 1>(v, w, bias, y, s);
    if (v.m <= 4) return gemv_i8_launch<DT, L, BPL, 4>(v, w, bias, y, s);
    return gemv_i8_launch<DT, L, BPL, 8>(v, w, bias, y, s);
}

template <int DT>
struct GemvI8F {
    static cudaError_t run(const ActsView& v, const Weight& w, const float* bias, float* y, cudaStream_t s) {
        // Lanes per row (L) and blocks per lane (BPL) depend on K only, so
        // results do not depend on M.  Several blocks per lane keep the
        // xor reduction (log2 L steps per row) small next to the block work.
        const int nb = w.nb;
        if (nb <= 8) return gemv_i8_mr<DT, 8, 1>(v, w, bias, y, s);
        if (nb <= 16) return gemv_i8_mr<DT, 8, 2>(v, w, bias, y, s);
        if (nb <= 32) return gemv_i8_mr<DT, 8, 4>(v, w, bias, y, s);
        if (nb <= 64) return gemv_i8_mr<DT, 16, 4>(v, w, bias, y, s);
        if (nb <= 128) return gemv_i8_mr<DT, 32, 4>(v, w, bias, y, s);
        if (nb <= 256) return gemv_i8_mr<DT, 32, 8>(v, w, bias, y, s);
        return cudaErrorInvalidValue;
    }
};

// Ring depth, n-tiles and grid.  The grid does not depend on NT or on the
// occupancy (two CTAs per SM are assumed for the cap), so a row's result
// is the same for every M: the K-split and the KS == 1 tile ranges depend
// on N, K and the SM count only.
template <int DT, int KS, int PF, int NT>
cudaError_t gemv_mma_go(const ActsView& v, const Weight& w, const float* bias, float* y, cudaStream_t s) {
    auto kern = k_gemv_mma<DT, KS, PF, NT>;
    const size_t smem = gemv_mma_act_smem(w.nb, NT) + size_t(PF) * Slot<DT>::BYTES * (GM_THREADS / 32);
    int dev = 0, sms = 148;
    dev_sms(&dev, &sms);
    static unsigned attr_dev_mask = 0;  // one bit per device with the attribute set
    if (!(attr_dev_mask & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 224 * 1024);
        if (e != cudaSuccess) return e;
        attr_dev_mask |= 1u << dev;
    }
    const int tiles = (w.n + 15) / 16, tpc = (GM_THREADS / 32) / KS;
    // KS == 1: one contiguous range of at least 8 tiles per CTA (see the
    // kernel); KS > 1: grid-stride over groups of tpc tiles.
    unsigned grid = KS == 1 ? unsigned(tiles / (GM_THREADS / 32)) : unsigned((tiles + tpc - 1) / tpc);
    const unsigned cap = unsigned(sms) * 2u;
    grid = grid < 1 ? 1 : (grid > cap ? cap : grid);
    const unsigned rows = unsigned((v.m + 8 * NT - 1) / (8 * NT));
    return launch_pdl(kern, dim3(grid, rows), dim3(GM_THREADS), smem, s, w.qs, w.qh, w.d, w.m, v.q8, v.d, v.sum, v.u,
                      v.m, w.n, w.k, bias, y);
}

constexpr size_t GEMV_SMEM_MAX = 224 * 1024;

template <int DT>
size_t gemv_slot8() { return size_t(Slot<DT>::BYTES) * (GM_THREADS / 32); }

// The most n-tiles (of 1, 2, 4, 8) whose staging fits with a 4-deep ring.
template <int DT>
int gemv_mma_nt_max(int nb) {
    for (int nt = 8; nt > 1; nt >>= 1)
        if (gemv_mma_act_smem(nb, nt) + 4 * gemv_slot8<DT>() <= GEMV_SMEM_MAX) return nt;
    return 1;
}

// n-tiles per CTA: as many as the rows need (up to what fits) when the
// weight gives the grid enough CTAs on its own; otherwise two (16 rows),
// so that more CTAs share the rows.
template <int DT, int KS>
cudaError_t gemv_mma_launch(const ActsView& v, const Weight& w, const float* bias, float* y, cudaStream_t s) {
    const int need = (v.m + 7) / 8;
    int nt = need <= 1 ? 1 : need <= 2 ? 2 : need <= 4 ? 4 : 8;
    const int nt_max = gemv_mma_nt_max<DT>(w.nb);
    int dev = 0, sms = 148;
    dev_sms(&dev, &sms);
    const int tiles = (w.n + 15) / 16;
    if (nt > 2 && tiles * KS < 2 * sms * (GM_THREADS / 32)) nt = 2;
    if (nt > nt_max) nt = nt_max;
    switch (nt) {
        case 1:
            if (gemv_mma_act_smem(w.nb, 1) + 8 * gemv_slot8<DT>() <= GEMV_SMEM_MAX / 2)
                return gemv_mma_go<DT, KS, 8, 1>(v, w, bias, y, s);
            return gemv_mma_go<DT, KS, 4, 1>(v, w, bias, y, s);
        case 2: return gemv_mma_go<DT, KS, 4, 2>(v, w, bias, y, s);
        case 4: return gemv_mma_go<DT, KS, 4, 4>(v, w, bias, y, s);
        default: return gemv_mma_go<DT, KS, 4, 8>(v, w, bias, y, s);
    }
}

// K-split of k_gemv_mma: keep splitting while the GPU would hold fewer
// than 8 warps per SM and every slice keeps at least two block groups.
// Depends on N and K only (results stay independent of M).
inline int gemv_mma_ks(int n, int nb) {
    int dev = 0, sms = 148;
    dev_sms(&dev, &sms);
    const int tiles = (n + 15) / 16, ng = round4(nb) / 4;
    int ks = 1;
    while (ks < 8 && ng >= 2 * ks && tiles * ks < sms * 8) ks *= 2;
    return ks;
}

template <int DT>
struct GemvMmaF {
    static cudaError_t run(const ActsView& v, const Weight& w, const float* bias, float* y, cudaStream_t s) {
        switch (gemv_mma_ks(w.n, w.nb)) {
            case 1: return gemv_mma_launch<DT, 1>(v, w, bias, y, s);
            case 2: return gemv_mma_launch<DT, 2>(v, w, bias, y, s);
            case 4: return gemv_mma_launch<DT, 4>(v, w, bias, y, s);
            default: return gemv_mma_launch<DT, 8>(v, w, bias, y, s);
        }
    }
};

// Tile configuration of k_gemv_tile (every configuration gives the same
// bits; chosen from a B200 sweep over the whisper decoder shapes):
//   * K-split weights (ks > 1) with short K (<= 16 groups) and enough
//     32 x 32 tiles for 1.5 CTAs per SM: one CTA walks all K slices of a
//     32 x 32 tile (WN = 1, NT = 2, no cluster) -- the pipeline then hides
//     the loads, and the tiles fill the GPU on their own;
//   * other K-split weights: clusters of ks CTAs, one per slice, on 64 x
//     32 tiles (up to 80 rows) or 64 x 64 tiles;
//   * unsplit (wide) weights: 64 x 32 or 64 x 64 tiles, no cluster.
// RWQ_GEMV_TILE="WN,NT" and RWQ_GEMV_TILE_CL=0|1 override (sweeps).
inline void gemv_tile_cfg(int m, int n, int nb, int ks, int sms, int* wn, int* nt, bool* cl) {
    static int env_wn = -1, env_nt = -1, env_cl = -1;
    if (env_wn < 0) {
        env_wn = env_nt = 0;
        if (const char* e = getenv("RWQ_GEMV_TILE")) {
            int a = 0, b = 0;
            if (sscanf(e, "%d,%d", &a, &b) == 2 && (a == 1 || a == 2) && (b == 2 || b == 4)) env_wn = a, env_nt = b;
        }
        const char* c = getenv("RWQ_GEMV_TILE_CL");
        env_cl = (c && (c[0] == '0' || c[0] == '1')) ? c[0] - '0' : 2;
    }
    const long small_tiles = long((n + 31) / 32) * long((m + 31) / 32);
    const bool walk = ks > 1 && round4(nb) / 4 <= 16 && small_tiles * 2 >= long(sms) * 3;
    *cl = ks > 1 && !walk;
    *wn = walk ? 1 : 2;
    *nt = walk ? 2 : (m > 80 ? 4 : 2);
    if (env_wn) { *wn = env_wn; *nt = env_nt; }
    if (env_cl != 2) *cl = ks > 1 && env_cl == 1;
}

template <int DT, int WN, int NT, bool CL>
cudaError_t gemv_tile_launch(const ActsView& v, const Weight& w, const float* bias, float* y, int ks, int gx,
                             int vec16, cudaStream_t s) {
    using L = TileSmem<DT, WN, NT>;
    auto kern = k_gemv_tile<DT, WN, NT, CL>;
    int dev = 0, sms = 148;
    dev_sms(&dev, &sms);
    static unsigned attr_dev_mask = 0;
    if (!(attr_dev_mask & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES);
        if (e != cudaSuccess) return e;
        // Three CTAs per SM need more shared memory than the default split.
        e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        if (e != cudaSuccess) return e;
        attr_dev_mask |= 1u << dev;
    }
    const int cs = CL ? ks : 1;
    const dim3 grid(unsigned((w.n + L::BN - 1) / L::BN * cs), unsigned((v.m + L::BM - 1) / L::BM));
    if (!CL)
        return launch_pdl(kern, grid, dim3(GT_THREADS), size_t(L::BYTES), s, w.qs, w.qh, w.d, w.m, v.q8, v.d,
                          v.sum, v.u, v.m, w.n, w.k, bias, y, ks, gx, vec16);
    return launch_pdl_cluster(kern, grid, dim3(GT_THREADS), size_t(L::BYTES), cs, s, w.qs, w.qh, w.d, w.m, v.q8,
                              v.d, v.sum, v.u, v.m, w.n, w.k, bias, y, ks, gx, vec16);
}

// cl: K slices as clusters (one CTA per slice); otherwise one CTA walks
// all slices, keeping their order with the slice totals.
template <int DT, int WN, int NT>
cudaError_t gemv_tile_go(const ActsView& v, const Weight& w, const float* bias, float* y, int ks, int gx,
                         int vec16, bool cl, cudaStream_t s) {
    return cl ? gemv_tile_launch<DT, WN, NT, true>(v, w, bias, y, ks, gx, vec16, s)
              : gemv_tile_launch<DT, WN, NT, false>(v, w, bias, y, ks, gx, vec16, s);
}

template <int DT>
struct GemvTileF {
    static cudaError_t run(const ActsView& v, const Weight& w, const float* bias, float* y, cudaStream_t s) {
        int dev = 0, sms = 148;
        dev_sms(&dev, &sms);
        // k_gemv_mma's K-split and (KS == 1) grid, whose summation order
        // k_gemv_tile reproduces.
        const int ks = gemv_mma_ks(w.n, w.nb), tiles = (w.n + 15) / 16;
        int gx = 0;
        if (ks == 1) {
            gx = tiles / (GM_THREADS / 32);
            gx = gx < 1 ? 1 : (gx > 2 * sms ? 2 * sms : gx);
        }
        const int vec16 = (v.nb % 4 == 0 && (reinterpret_cast<uintptr_t>(v.d) & 15) == 0 &&
                           (reinterpret_cast<uintptr_t>(v.sum) & 15) == 0 &&
                           (reinterpret_cast<uintptr_t>(v.u) & 15) == 0) ? 1 : 0;
        int wn = 1, nt = 2;
        bool cl = false;
        gemv_tile_cfg(v.m, w.n, w.nb, ks, sms, &wn, &nt, &cl);
        if (wn == 1) return nt == 2 ? gemv_tile_go<DT, 1, 2>(v, w, bias, y, ks, gx, vec16, cl, s)
                                    : gemv_tile_go<DT, 1, 4>(v, w, bias, y, ks, gx, vec16, cl, s);
        return nt == 2 ? gemv_tile_go<DT, 2, 2>(v, w, bias, y, ks, gx, vec16, cl, s)
                       : gemv_tile_go<DT, 2, 4>(v, w, bias, y, ks, gx, vec16, cl, s);
    }
};

template <int DT>
struct GemvRowsF {
    static cudaError_t run(int nb, int* out) {
        *out = 8 * gemv_mma_nt_max<DT>(nb);
        return cudaSuccess;
    }
};

thread_local int t_gemv_kind = 0;

// Rows from which the automatic choice takes k_gemv_tile (measured on the
// whisper decoder shapes): 32 when k_gemv_mma splits K (its CTAs then
// re-stage the activations per 16 weight rows), 80 for the wide weights
// it runs without a split (the logits), where both are close below that.
int gemv_tile_min_m(int n, int nb) { return gemv_mma_ks(n, nb) > 1 ? 32 : 80; }

template <int DT, int L, int MR>
cudaError_t gemv_f32_launch(const float* a, int m, const Weight& w, const float* bias, float* y, cudaStream_t s) {
    k_gemv_f32<DT, L, MR><<<gemv_grid(k_gemv_f32<DT, L, MR>, w.n, L, 0), TPB, 0, s>>>(w.qs, w.qh, w.d, w.m, a, m, w.n,
                                                                                      w.k, bias, y);
    return cudaGetLastError();
}

template <int DT, int L>
cudaError_t gemv_f32_mr(const float* a, int m, const Weight& w, const float* bias, float* y, cudaStream_t s) {
    if (m <= 1) return gemv_f32_launch<DT, L, 1>(a, m, w, bias, y, s);
    if (m <= 2) return gemv_f32_launch<DT, L, 2>(a, m, w, bias, y, s);
    if (m <= 4) return gemv_f32_launch<DT, L, 4>(a, m, w, bias, y, s);
    return gemv_f32_launch<DT, L, 8>(a, m, w, bias, y, s);
}

template <int DT>
struct GemvF32F {
    static cudaError_t run(const float* a, int m, const Weight& w, const float* bias, float* y, cudaStream_t s) {
        switch (lanes_for(w.nb)) {
            case 32: return gemv_f32_mr<DT, 32>(a, m, w, bias, y, s);
            case 16: return gemv_f32_mr<DT, 16>(a, m, w, bias, y, s);
            default: return gemv_f32_mr<DT, 8>(a, m, w, bias, y, s);
        }
    }
};

}  // namespace

cudaError_t launch_repack(const uint8_t* raw, Weight& w, cudaStream_t s) { return by_dtype<RepackF>(w.dtype, raw, w, s); }

cudaError_t launch_build_gemm_cache(Weight& w, cudaStream_t s) { return by_dtype<GemmCacheF>(w.dtype, w, s); }

cudaError_t launch_build_fold_cache(Weight& w, cudaStream_t s) { return by_dtype<FoldCacheF>(w.dtype, w, s); }

cudaError_t launch_quantize_acts(const float* a, const ActsView& v, bool want_gemm, cudaStream_t s) {
    const int m_pad = want_gemm ? v.m_pad : v.m;
    const size_t blocks = size_t(m_pad) * v.nb;
    if (!blocks) return cudaSuccess;
    auto kern = (reinterpret_cast<uintptr_t>(a) & 15) ? k_quantize<false> : k_quantize<true>;
    return launch_pdl(kern, dim3(grid_for(blocks * 8, TPB)), dim3(TPB), 0, s, a, v.m, v.k, v.nb, m_pad,
                      want_gemm ? nullptr : v.q8, v.d, v.sum, v.u, want_gemm ? v.q16 : nullptr,
                      want_gemm ? v.dT : nullptr, want_gemm ? v.uT : nullptr);
}

cudaError_t launch_dequant_rows(const Weight& w, const int32_t* rows, int nrows, float* out, cudaStream_t s) {
    return by_dtype<DequantF>(w.dtype, w, rows, nrows, out, s);
}

cudaError_t launch_embed(const Weight& w, const int32_t* tokens, int n, const float* pos, const int* dpos, float* x,
                         cudaStream_t s) {
    return by_dtype<EmbedF>(w.dtype, w, tokens, n, pos, dpos, x, s);
}

cudaError_t launch_block_dots(const ActsView& v, const Weight& w, int32_t* S, cudaStream_t s) {
    return by_dtype<BlockDotsF>(w.dtype, v, w, S, s);
}

void set_gemv_kind(int kind) { t_gemv_kind = kind; }

int gemv_rows_per_launch(int dtype, int k) {
    int r = 8;
    by_dtype<GemvRowsF>(dtype, k / QK, &r);
    return r;
}

// Kernel of one launch of the GEMV family for activations `c` (c.m <= 256):
// 4 row-per-lane (one or two rows on a weight k_gemv_mma runs without a K
// split: the wide ones), 3 tiled integer MMA (many rows; needs 16-byte
// aligned activation codes), 2 integer MMA, 1 dp4a.  2, 3 and 4 give the
// same bits, so the choice is a speed choice; the MMA kernels address the
// planes with 32-bit offsets.
int gemv_choice(const ActsView& c, const Weight& w) {
    const int forced = t_gemv_kind;
    if (forced == 1) return 1;
    if ((forced == 0 || forced == 4) && c.m <= GEMV_ROWS_MAX_M && gemv_mma_ks(w.n, w.nb) == 1 && gemv_rows_fits(c, w))
        return 4;
    if (uint64_t(w.n) * uint64_t(round4(w.nb)) * uint64_t(qs_bytes(w.dtype)) >= (uint64_t(1) << 32)) return 1;
    const bool tile_ok = (reinterpret_cast<uintptr_t>(c.q8) & 15) == 0;
    if (forced == 3) return tile_ok ? 3 : 2;
    if (forced == 2) return 2;
    return tile_ok && c.m >= gemv_tile_min_m(w.n, w.nb) ? 3 : 2;
}

cudaError_t launch_gemv_i8(const ActsView& v, const Weight& w, const float* bias, float* y, cudaStream_t s,
                           int* err_flag) {
    if (v.m <= 0 || w.n <= 0) return cudaSuccess;
    // The MMA kernels take up to 256 rows per launch (CTA rows of up to 64
    // activation rows share the weights through L2); dp4a launches 8 rows.
    const int per = gemv_choice(v, w) == 1 ? GEMV_MAX_M : GEMV_FAMILY_MAX_M;
    for (int m0 = 0; m0 < v.m; m0 += per) {
        ActsView c = v;
        c.m = v.m - m0 < per ? v.m - m0 : per;
        c.q8 = v.q8 + size_t(m0) * v.k;
        c.d = v.d + size_t(m0) * v.nb;
        c.sum = v.sum + size_t(m0) * v.nb;
        c.u = v.u + size_t(m0) * v.nb;
        float* yc = y + size_t(m0) * w.n;
        cudaError_t e;
        switch (gemv_choice(c, w)) {
            case 4: {
                int dev = 0, sms = 148;
                dev_sms(&dev, &sms);
                // k_gemv_mma's grid at KS == 1, whose tile split k_gemv_rows reproduces.
                int gx = ((w.n + 15) / 16) / (GM_THREADS / 32);
                gx = gx < 1 ? 1 : (gx > 2 * sms ? 2 * sms : gx);
                e = launch_gemv_rows(c, w, bias, yc, gx, err_flag, s);
                break;
            }
            case 3: e = by_dtype<GemvTileF>(w.dtype, c, w, bias, yc, s); break;
            case 2: e = by_dtype<GemvMmaF>(w.dtype, c, w, bias, yc, s); break;
            default: e = by_dtype<GemvI8F>(w.dtype, c, w, bias, yc, s); break;
        }
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

int gemv_kernel_for(const Weight& w, int m) {
    ActsView c;
    c.m = m;
    c.k = w.k;
    c.nb = w.nb;
    c.q8 = reinterpret_cast<int8_t*>(uintptr_t(256));   // library-allocated codes are 256-byte aligned
    return gemv_choice(c, w);
}

cudaError_t launch_gemv_f32(const float* a, int m, const Weight& w, const float* bias, float* y, cudaStream_t s) {
    if (m <= 0 || w.n <= 0) return cudaSuccess;
    return by_dtype<GemvF32F>(w.dtype, a, m, w, bias, y, s);
}

}  // namespace rwq
