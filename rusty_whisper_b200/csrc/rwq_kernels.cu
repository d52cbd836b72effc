// rwq_kernels.cu -- CUDA-core kernels of the quantized-matmul path:
// weight repack, activation int8 quantizer, bit-exact dequant gather,
// per-block integer dots (debug/parity), the decoder GEMVs (int8 and
// dequant-then-f32), and the builder of the tensor-core operand cache.
#include <cuda_fp16.h>
#include "rwq_common.cuh"
#include "rwq_internal.h"

namespace rwq {

namespace {

constexpr int TPB = 256;

inline unsigned grid_for(size_t work, int per_block) {
    size_t g = (work + per_block - 1) / per_block;
    return unsigned(g ? g : 1);
}

// ---------------------------------------------------------------- repack
// raw ggml records [n*nb][bb] -> planes.  One thread per block; the raw
// records are not 16-byte aligned, so they are read bytewise, once.
template <int DT>
__global__ void k_repack(const uint8_t* __restrict__ raw, uint8_t* __restrict__ qs, uint32_t* __restrict__ qh,
                         uint16_t* __restrict__ d, uint16_t* __restrict__ m, size_t nblk) {
    size_t b = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (b >= nblk) return;
    constexpr int BB = block_bytes(DT), QSB = qs_bytes(DT), QO = raw_qs_off(DT);
    const uint8_t* p = raw + b * BB;
    d[b] = uint16_t(p[0] | (p[1] << 8));
    if (has_min(DT)) m[b] = uint16_t(p[2] | (p[3] << 8));
    if (has_qh(DT)) {
        const uint8_t* h = p + raw_qh_off(DT);
        qh[b] = qh_plane_bits(uint32_t(h[0]) | (uint32_t(h[1]) << 8) | (uint32_t(h[2]) << 16) |
                              (uint32_t(h[3]) << 24));
    }
    uint32_t words[QSB / 4];
#pragma unroll
    for (int i = 0; i < QSB / 4; ++i)
        words[i] = uint32_t(p[QO + 4 * i]) | (uint32_t(p[QO + 4 * i + 1]) << 8) |
                   (uint32_t(p[QO + 4 * i + 2]) << 16) | (uint32_t(p[QO + 4 * i + 3]) << 24);
    uint4* dst = reinterpret_cast<uint4*>(qs + b * QSB);
#pragma unroll
    for (int i = 0; i < QSB / 16; ++i) dst[i] = make_uint4(words[4 * i], words[4 * i + 1], words[4 * i + 2], words[4 * i + 3]);
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

template <int DT>
__device__ __forceinline__ void load_block(const uint8_t* __restrict__ qs, const uint32_t* __restrict__ qh,
                                           const uint16_t* __restrict__ dp, const uint16_t* __restrict__ mp,
                                           size_t b, BlockCodes<DT>& bc) {
    if (DT == Q8_0) {
        const uint4* p = reinterpret_cast<const uint4*>(qs + b * 32);
        uint4 v0 = __ldg(p), v1 = __ldg(p + 1);
        bc.w[0] = v0.x; bc.w[1] = v0.y; bc.w[2] = v0.z; bc.w[3] = v0.w;
        bc.w[4] = v1.x; bc.w[5] = v1.y; bc.w[6] = v1.z; bc.w[7] = v1.w;
    } else {
        uint4 v = __ldg(reinterpret_cast<const uint4*>(qs + b * 16));
        uint32_t h = has_qh(DT) ? __ldg(qh + b) : 0u;
        codes_u8x4<DT>(v, h, bc.w);
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
    load_block<DT>(qs, qh, dp, mp, size_t(j) * nb + bl, bc);
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
    load_block<DT>(qs, qh, dp, mp, size_t(j) * nb + bl, bc);
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
                                         const uint16_t* __restrict__ dp, const uint16_t* __restrict__ mp, size_t b,
                                         RawBlock<DT>& rb) {
    if (DT == Q8_0) {
        const uint4* p = reinterpret_cast<const uint4*>(qs + b * 32);
        rb.v0 = __ldg(p);
        rb.v1 = __ldg(p + 1);
    } else {
        rb.v0 = __ldg(reinterpret_cast<const uint4*>(qs + b * 16));
    }
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
constexpr uint32_t MAGIC_BITS = 0x4B400000u;  // 12582912.0f
constexpr float MAGIC_F = 12582912.0f;

template <int DT, int L, int BPL, int MR, int PF, bool REGA>
__global__ void __launch_bounds__(TPB) k_gemv_i8(const uint8_t* __restrict__ qs, const uint32_t* __restrict__ qh,
                                                 const uint16_t* __restrict__ dp, const uint16_t* __restrict__ mp,
                                                 const int8_t* __restrict__ q8, const float* __restrict__ da,
                                                 const int32_t* __restrict__ sa, const float* __restrict__ ua, int M,
                                                 int N, int K, const float* __restrict__ bias, float* __restrict__ y) {
    pdl_trigger();
    const int nb = K / QK;
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
            if (grp < groups && j < N && kb < nb) load_raw<DT>(qs, qh, dp, mp, size_t(j) * nb + kb, dst[t]);
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
                load_block<DT>(qs, qh, dp, mp, size_t(j) * nb + kb, bc);
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
    load_block<DT>(qs, qh, dp, mp, size_t(j) * nb + bl, bc);
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
        load_block<DT>(qs, qh, dp, mp, size_t(j) * nb + kb, bc);
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
        load_block<DT>(qs, qh, dp, mp, size_t(j) * nb + kb, bc);
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
        k_repack<DT><<<grid_for(nblk, TPB), TPB, 0, s>>>(raw, w.qs, w.qh, w.d, w.m, nblk);
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
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
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

cudaError_t launch_block_dots(const ActsView& v, const Weight& w, int32_t* S, cudaStream_t s) {
    return by_dtype<BlockDotsF>(w.dtype, v, w, S, s);
}

cudaError_t launch_gemv_i8(const ActsView& v, const Weight& w, const float* bias, float* y, cudaStream_t s) {
    if (v.m <= 0 || w.n <= 0) return cudaSuccess;
    return by_dtype<GemvI8F>(w.dtype, v, w, bias, y, s);
}

cudaError_t launch_gemv_f32(const float* a, int m, const Weight& w, const float* bias, float* y, cudaStream_t s) {
    if (m <= 0 || w.n <= 0) return cudaSuccess;
    return by_dtype<GemvF32F>(w.dtype, a, m, w, bias, y, s);
}

}  // namespace rwq
