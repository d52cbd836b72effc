// rwq_oracle.cpp -- CPU restatement of rusty_whisper's quantized-matmul path.
//
// TEST INFRASTRUCTURE ONLY.  This file is the parity checker and the timed
// CPU baseline; it is never part of the shipped GPU path.  Only tests/,
// __graft_entry__.smoke() and bench.py (cpu_baseline leg and the
// `--impl reference` arm) may load the library built from it.
//
// What it restates (reference = baileyrd/rusty_whisper, Rust, src/ paths):
//   * f16 <-> f32                      model.rs:68-86, model.rs:90-115
//   * ggml block sizes / unpack        quant.rs:43-52, quant.rs:57-131
//   * scalar dequant                   quant.rs:528-537
//   * AVX2 dequant (mul+add, no FMA)   quant.rs:193-238
//   * int8 activation quantizer        quant.rs:690-716
//   * AVX2 / AVX-512 VNNI int8 dots    quant.rs:330-490
//   * matmul_t_q tiering, N_BLOCK/M_BLOCK blocking, N-chunk threads,
//     cold (scratch) and packed (cached) weight paths
//                                      quant.rs:754-1051
//   * f32 fallback (dequant + dot4)    quant.rs:995-1018, tensor.rs:104-158
//   * dense matmul_t                   tensor.rs:165-258
//   * log-mel front end: periodic Hann window, 400-point FFT (radix-2
//     recursion down to odd-length DFTs), power spectrum, Slaney mel
//     filterbank, log10 + dynamic-range clamp  audio.rs:10-198
//   * encoder graph: conv stem, pre-LN attention / MLP blocks, ln_post,
//     with layernorm, tanh-GELU, softmax, conv1d and matmul
//                                      encoder.rs:48-234, tensor.rs:75-100, 274-370
//   * KV-cached decoder: cross K/V, causal self-attention, cross-attention,
//     MLP, final LN, tied logits          decoder.rs:36-321
//   * test helpers: LCG test_matrix, rand_byte, quantize_q8_0, quantize_q5_1
//                                      quant.rs:1071-1123, quant.rs:1131-1135
//
// Parity pin: the reference is Rust and no Rust toolchain exists here, so
// it cannot be built or run.  This restatement is pinned against every
// known-answer and bit-identity test the reference carries for the path
// (quant.rs:1125-1174, quant.rs:1336-1384, model.rs:282-291, 348-390);
// tests/test_oracle_pins.py runs them.
//
// Build: oracle/build.sh (g++ -O2 -ffp-contract=off, no fast-math; the
// reference never fuses d*q+m, and neither may this file).
#include <immintrin.h>
#include <cstdlib>
#include <string>
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

constexpr int QK = 32;
constexpr int N_BLOCK = 8;    // quant.rs:25
constexpr int M_BLOCK = 64;   // quant.rs:36
constexpr size_t PAR_THRESHOLD = size_t(1) << 20;  // tensor.rs:44

// ---------------------------------------------------------------- f16
// model.rs:68-86: exact f16 -> f32, subnormals via the msb position.
float f16_to_f32(uint16_t h) {
    uint32_t sign = h >> 15, exp = (h >> 10) & 0x1f, frac = h & 0x3ff, bits;
    if (exp == 0 && frac == 0) {
        bits = sign << 31;
    } else if (exp == 0) {
        uint32_t p = 31 - __builtin_clz(frac);
        uint32_t mant = (frac << (10 - p)) & 0x3ff;
        bits = (sign << 31) | ((p + 103) << 23) | (mant << 13);
    } else if (exp == 0x1f && frac == 0) {
        bits = (sign << 31) | 0x7f800000u;
    } else if (exp == 0x1f) {
        bits = (sign << 31) | 0x7f800000u | (frac << 13);
    } else {
        bits = (sign << 31) | ((exp + 127 - 15) << 23) | (frac << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// model.rs:90-115: f32 -> f16 rounding half-up on the first dropped bit
// (not round-to-nearest-even), which is how every test scale was made.
uint16_t f32_to_f16(float x) {
    uint32_t bits;
    std::memcpy(&bits, &x, 4);
    uint16_t sign = (bits >> 16) & 0x8000;
    int32_t exp = (bits >> 23) & 0xff;
    uint32_t frac = bits & 0x007fffff;
    if (exp == 0xff) return sign | 0x7c00 | (frac != 0 ? 0x200 : 0);
    int32_t e = exp - 127 + 15;
    if (e >= 0x1f) return sign | 0x7c00;
    if (e <= 0) {
        if (e < -10) return sign;
        uint32_t f = frac | 0x00800000;
        uint32_t shift = uint32_t(14 - e);
        uint16_t half = uint16_t(f >> shift);
        uint16_t round = uint16_t((f >> (shift - 1)) & 1);
        return sign | uint16_t(half + round);
    }
    uint16_t half = uint16_t((uint32_t(e) << 10) | (frac >> 13));
    uint16_t round = uint16_t((frac >> 12) & 1);
    return sign | uint16_t(half + round);
}

inline float half_at(const uint8_t* p) { return f16_to_f32(uint16_t(p[0] | (p[1] << 8))); }
inline uint32_t u32_at(const uint8_t* p) {
    return uint32_t(p[0]) | (uint32_t(p[1]) << 8) | (uint32_t(p[2]) << 16) | (uint32_t(p[3]) << 24);
}

// quant.rs:43-52
int block_bytes(int dtype) {
    switch (dtype) {
        case 2: return 18;  // Q4_0
        case 3: return 20;  // Q4_1
        case 6: return 22;  // Q5_0
        case 7: return 24;  // Q5_1
        case 8: return 34;  // Q8_0
        default: return -1;
    }
}

// quant.rs:57-63: element j<16 = low nibble of byte j, j>=16 = high nibble
// of byte j-16, minus `offset`.
void unpack_nibbles(const uint8_t* packed, int8_t* q, int offset) {
    for (int j = 0; j < QK / 2; ++j) {
        q[j] = int8_t(int(packed[j] & 0x0F) - offset);
        q[j + QK / 2] = int8_t(int(packed[j] >> 4) - offset);
    }
}

// quant.rs:84-94: bit j of qh adds 16 to element j (the HI_BITS table is a
// lookup of exactly this; the table is a CPU speed device only).
void apply_high_bits(uint32_t qh, int8_t* q) {
    for (int j = 0; j < QK; ++j) q[j] = int8_t(q[j] + (((qh >> j) & 1) << 4));
}

// quant.rs:98-131: centred int8 quants + (d, m) with x = d*q + m.
// Returns false for an unsupported dtype (the reference panics).
bool unpack_block(int dtype, const uint8_t* b, int8_t* q, float* d, float* m) {
    switch (dtype) {
        case 2: unpack_nibbles(b + 2, q, 8); *d = half_at(b); *m = 0.f; return true;
        case 3: unpack_nibbles(b + 4, q, 0); *d = half_at(b); *m = half_at(b + 2); return true;
        case 6:
            unpack_nibbles(b + 6, q, 0);
            apply_high_bits(u32_at(b + 2), q);
            for (int j = 0; j < QK; ++j) q[j] = int8_t(q[j] - 16);
            *d = half_at(b); *m = 0.f; return true;
        case 7:
            unpack_nibbles(b + 8, q, 0);
            apply_high_bits(u32_at(b + 4), q);
            *d = half_at(b); *m = half_at(b + 2); return true;
        case 8:
            for (int j = 0; j < QK; ++j) q[j] = int8_t(b[2 + j]);
            *d = half_at(b); *m = 0.f; return true;
        default: return false;
    }
}

// quant.rs:528-537: o = d*q + m, unfused (compiled with -ffp-contract=off).
void dequant_row_scalar(int dtype, const uint8_t* raw, size_t nblocks, float* out) {
    int bb = block_bytes(dtype);
    int8_t q[QK];
    for (size_t bl = 0; bl < nblocks; ++bl) {
        float d, m;
        unpack_block(dtype, raw + bl * bb, q, &d, &m);
        for (int l = 0; l < QK; ++l) out[bl * QK + l] = d * float(q[l]) + m;
    }
}

// ------------------------------------------------------------ AVX2 tier
// quant.rs:147-155
__attribute__((target("avx2,fma"))) inline void nibbles(const uint8_t* p, __m128i* lo, __m128i* hi) {
    __m128i qs = _mm_loadu_si128((const __m128i*)p);
    __m128i mask = _mm_set1_epi8(0x0F);
    *lo = _mm_and_si128(qs, mask);
    *hi = _mm_and_si128(_mm_srli_epi16(qs, 4), mask);
}

// quant.rs:158-170: bits base..base+16 of qh -> per-byte 0x10 flags.
__attribute__((target("avx2,fma"))) inline __m128i high_bits(uint32_t qh, int base) {
    __m128i bytes = _mm_set1_epi32(int(qh));
    __m128i shuf = base == 0 ? _mm_setr_epi8(0, 0, 0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1, 1, 1, 1)
                             : _mm_setr_epi8(2, 2, 2, 2, 2, 2, 2, 2, 3, 3, 3, 3, 3, 3, 3, 3);
    __m128i bits = _mm_setr_epi8(1, 2, 4, 8, 16, 32, 64, -128, 1, 2, 4, 8, 16, 32, 64, -128);
    __m128i picked = _mm_and_si128(_mm_shuffle_epi8(bytes, shuf), bits);
    return _mm_and_si128(_mm_cmpeq_epi8(picked, bits), _mm_set1_epi8(0x10));
}

// quant.rs:175-188: out = d*q + m with separate mul and add.
__attribute__((target("avx2,fma"))) inline void store32(__m128i q0, __m128i q1, float d, float m, float* out) {
    __m256 dv = _mm256_set1_ps(d), mv = _mm256_set1_ps(m);
    __m128i qs[2] = {q0, q1};
    for (int h = 0; h < 2; ++h) {
        __m256i lo = _mm256_cvtepi8_epi32(qs[h]);
        __m256i hi = _mm256_cvtepi8_epi32(_mm_srli_si128(qs[h], 8));
        __m256i ints[2] = {lo, hi};
        for (int g = 0; g < 2; ++g) {
            __m256 f = _mm256_cvtepi32_ps(ints[g]);
            __m256 r = _mm256_add_ps(_mm256_mul_ps(f, dv), mv);
            _mm256_storeu_ps(out + h * 16 + g * 8, r);
        }
    }
}

// quant.rs:193-238
__attribute__((target("avx2,fma"))) void dequant_row_avx2(int dtype, const uint8_t* raw, size_t nblocks, float* out) {
    int bb = block_bytes(dtype);
    for (size_t bi = 0; bi < nblocks; ++bi) {
        float* o = out + bi * QK;
        const uint8_t* p = raw + bi * bb;
        __m128i q0, q1, lo, hi;
        switch (dtype) {
            case 2: {
                float d = half_at(p);
                nibbles(p + 2, &q0, &q1);
                store32(q0, q1, d, -8.0f * d, o);
                break;
            }
            case 3:
                nibbles(p + 4, &q0, &q1);
                store32(q0, q1, half_at(p), half_at(p + 2), o);
                break;
            case 6: {
                float d = half_at(p);
                uint32_t qh = u32_at(p + 2);
                nibbles(p + 6, &lo, &hi);
                store32(_mm_or_si128(lo, high_bits(qh, 0)), _mm_or_si128(hi, high_bits(qh, 16)), d, -16.0f * d, o);
                break;
            }
            case 7: {
                uint32_t qh = u32_at(p + 4);
                nibbles(p + 8, &lo, &hi);
                store32(_mm_or_si128(lo, high_bits(qh, 0)), _mm_or_si128(hi, high_bits(qh, 16)), half_at(p),
                        half_at(p + 2), o);
                break;
            }
            case 8:
                store32(_mm_loadu_si128((const __m128i*)(p + 2)), _mm_loadu_si128((const __m128i*)(p + 18)),
                        half_at(p), 0.0f, o);
                break;
        }
    }
}

// quant.rs:241-247: ((v0+v4)+(v1+v5)) + ((v2+v6)+(v3+v7)) via two hadds.
__attribute__((target("avx2,fma"))) inline float hsum256_ps(__m256 v) {
    __m128 s = _mm_add_ps(_mm256_castps256_ps128(v), _mm256_extractf128_ps(v, 1));
    s = _mm_hadd_ps(s, s);
    s = _mm_hadd_ps(s, s);
    return _mm_cvtss_f32(s);
}

// quant.rs:256-320: weight row -> int8 quants + per-block d, m.
__attribute__((target("avx2,fma"))) void unpack_row_i8_avx2(int dtype, const uint8_t* raw, int8_t* qb, float* db,
                                                        float* mb, int nb) {
    int bb = block_bytes(dtype);
    for (int bl = 0; bl < nb; ++bl) {
        const uint8_t* p = raw + size_t(bl) * bb;
        int8_t* o = qb + size_t(bl) * QK;
        __m128i lo, hi;
        switch (dtype) {
            case 8:
                _mm256_storeu_si256((__m256i*)o, _mm256_loadu_si256((const __m256i*)(p + 2)));
                db[bl] = half_at(p); mb[bl] = 0.f;
                break;
            case 2: {
                nibbles(p + 2, &lo, &hi);
                __m128i e = _mm_set1_epi8(8);
                _mm_storeu_si128((__m128i*)o, _mm_sub_epi8(lo, e));
                _mm_storeu_si128((__m128i*)(o + 16), _mm_sub_epi8(hi, e));
                db[bl] = half_at(p); mb[bl] = 0.f;
                break;
            }
            case 3:
                nibbles(p + 4, &lo, &hi);
                _mm_storeu_si128((__m128i*)o, lo);
                _mm_storeu_si128((__m128i*)(o + 16), hi);
                db[bl] = half_at(p); mb[bl] = half_at(p + 2);
                break;
            case 6: {
                uint32_t qh = u32_at(p + 2);
                nibbles(p + 6, &lo, &hi);
                __m128i e = _mm_set1_epi8(16);
                _mm_storeu_si128((__m128i*)o, _mm_sub_epi8(_mm_or_si128(lo, high_bits(qh, 0)), e));
                _mm_storeu_si128((__m128i*)(o + 16), _mm_sub_epi8(_mm_or_si128(hi, high_bits(qh, 16)), e));
                db[bl] = half_at(p); mb[bl] = 0.f;
                break;
            }
            case 7: {
                uint32_t qh = u32_at(p + 4);
                nibbles(p + 8, &lo, &hi);
                _mm_storeu_si128((__m128i*)o, _mm_or_si128(lo, high_bits(qh, 0)));
                _mm_storeu_si128((__m128i*)(o + 16), _mm_or_si128(hi, high_bits(qh, 16)));
                db[bl] = half_at(p); mb[bl] = half_at(p + 2);
                break;
            }
        }
    }
}

// quant.rs:403-418: per-block sum of the weight quants (VNNI correction).
__attribute__((target("avx2,fma"))) void weight_block_sums_avx2(const int8_t* qb, int32_t* sumb, int nb) {
    __m256i ones = _mm256_set1_epi16(1);
    for (int bl = 0; bl < nb; ++bl) {
        __m256i b = _mm256_loadu_si256((const __m256i*)(qb + size_t(bl) * QK));
        __m256i lo = _mm256_cvtepi8_epi16(_mm256_castsi256_si128(b));
        __m256i hi = _mm256_cvtepi8_epi16(_mm256_extracti128_si256(b, 1));
        __m256i s = _mm256_add_epi32(_mm256_madd_epi16(lo, ones), _mm256_madd_epi16(hi, ones));
        __m128i s128 = _mm_add_epi32(_mm256_castsi256_si128(s), _mm256_extracti128_si256(s, 1));
        __m128i s64 = _mm_add_epi32(s128, _mm_shuffle_epi32(s128, 0x4E));
        __m128i s32 = _mm_add_epi32(s64, _mm_shuffle_epi32(s64, 0x01));
        sumb[bl] = _mm_cvtsi128_si32(s32);
    }
}

struct RowRef {
    const int8_t* q;
    const float* d;
    const int32_t* s;
};

// quant.rs:366-395: four activation rows against one weight row, maddubs
// sign trick; corr = m_b*d_a*sum(q_a) accumulated in scalar f32.
__attribute__((target("avx2,fma"))) void dot_i8_avx2_x4(const RowRef* a, const int8_t* qb, const float* db,
                                                    const float* mb, int nb, float* out) {
    __m256i ones = _mm256_set1_epi16(1);
    __m256 acc[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps()};
    float corr[4] = {0.f, 0.f, 0.f, 0.f};
    for (int bl = 0; bl < nb; ++bl) {
        __m256i b = _mm256_loadu_si256((const __m256i*)(qb + size_t(bl) * QK));
        __m256i absb = _mm256_sign_epi8(b, b);
        float dbl = db[bl];
        for (int r = 0; r < 4; ++r) {
            __m256i av = _mm256_loadu_si256((const __m256i*)(a[r].q + size_t(bl) * QK));
            __m256i prod = _mm256_maddubs_epi16(absb, _mm256_sign_epi8(av, b));
            __m256i p32 = _mm256_madd_epi16(prod, ones);
            __m256 scale = _mm256_set1_ps(a[r].d[bl] * dbl);
            acc[r] = _mm256_fmadd_ps(scale, _mm256_cvtepi32_ps(p32), acc[r]);
            corr[r] += mb[bl] * a[r].d[bl] * float(a[r].s[bl]);
        }
    }
    for (int r = 0; r < 4; ++r) out[r] = hsum256_ps(acc[r]) + corr[r];
}

// quant.rs:331-354
__attribute__((target("avx2,fma"))) float dot_i8_avx2(RowRef a, const int8_t* qb, const float* db, const float* mb,
                                                 int nb) {
    __m256i ones = _mm256_set1_epi16(1);
    __m256 acc = _mm256_setzero_ps();
    float corr = 0.f;
    for (int bl = 0; bl < nb; ++bl) {
        __m256i av = _mm256_loadu_si256((const __m256i*)(a.q + size_t(bl) * QK));
        __m256i b = _mm256_loadu_si256((const __m256i*)(qb + size_t(bl) * QK));
        __m256i prod = _mm256_maddubs_epi16(_mm256_sign_epi8(b, b), _mm256_sign_epi8(av, b));
        __m256i p32 = _mm256_madd_epi16(prod, ones);
        __m256 scale = _mm256_set1_ps(a.d[bl] * db[bl]);
        acc = _mm256_fmadd_ps(scale, _mm256_cvtepi32_ps(p32), acc);
        corr += mb[bl] * a.d[bl] * float(a.s[bl]);
    }
    return hsum256_ps(acc) + corr;
}

// quant.rs:431-460: dpbusd on (q_a + 128) x q_b; the -128*sum(q_b) offset
// rides in the scalar correction.
__attribute__((target("avx2,fma,avx512vl,avx512vnni"))) void dot_i8_vnni_x4(const RowRef* a, const int8_t* qb,
                                                                        const float* db, const float* mb,
                                                                        const int32_t* sumb, int nb, float* out) {
    __m256i off = _mm256_set1_epi8(char(0x80));
    __m256 acc[4] = {_mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps(), _mm256_setzero_ps()};
    float corr[4] = {0.f, 0.f, 0.f, 0.f};
    for (int bl = 0; bl < nb; ++bl) {
        __m256i b = _mm256_loadu_si256((const __m256i*)(qb + size_t(bl) * QK));
        float dbl = db[bl], mbl = mb[bl], sbl = float(sumb[bl]);
        for (int r = 0; r < 4; ++r) {
            __m256i av = _mm256_loadu_si256((const __m256i*)(a[r].q + size_t(bl) * QK));
            __m256i au = _mm256_xor_si256(av, off);
            __m256i dp = _mm256_dpbusd_epi32(_mm256_setzero_si256(), au, b);
            float s = a[r].d[bl] * dbl;
            acc[r] = _mm256_fmadd_ps(_mm256_set1_ps(s), _mm256_cvtepi32_ps(dp), acc[r]);
            corr[r] += s * (-128.0f) * sbl + mbl * a[r].d[bl] * float(a[r].s[bl]);
        }
    }
    for (int r = 0; r < 4; ++r) out[r] = hsum256_ps(acc[r]) + corr[r];
}

// quant.rs:468-490
__attribute__((target("avx2,fma,avx512vl,avx512vnni"))) float dot_i8_vnni(RowRef a, const int8_t* qb, const float* db,
                                                                     const float* mb, const int32_t* sumb, int nb) {
    __m256i off = _mm256_set1_epi8(char(0x80));
    __m256 acc = _mm256_setzero_ps();
    float corr = 0.f;
    for (int bl = 0; bl < nb; ++bl) {
        __m256i b = _mm256_loadu_si256((const __m256i*)(qb + size_t(bl) * QK));
        __m256i av = _mm256_loadu_si256((const __m256i*)(a.q + size_t(bl) * QK));
        __m256i dp = _mm256_dpbusd_epi32(_mm256_setzero_si256(), _mm256_xor_si256(av, off), b);
        float s = a.d[bl] * db[bl];
        acc = _mm256_fmadd_ps(_mm256_set1_ps(s), _mm256_cvtepi32_ps(dp), acc);
        corr += s * (-128.0f) * float(sumb[bl]) + mb[bl] * a.d[bl] * float(a.s[bl]);
    }
    return hsum256_ps(acc) + corr;
}

// quant.rs:690-716: per 32-block d = amax/127, inv = 1/d (0 if d == 0),
// q = round(x*inv) (half away from zero) clamped to [-127, 127].
void quantize_acts_i8(const float* a, int m, int k, int8_t* q, float* d, int32_t* sum) {
    int nb = k / QK;
    for (int i = 0; i < m; ++i) {
        for (int bl = 0; bl < nb; ++bl) {
            const float* x = a + size_t(i) * k + size_t(bl) * QK;
            float amax = 0.f;
            // Rust f32::max returns the non-NaN operand.
            for (int l = 0; l < QK; ++l) {
                float v = std::fabs(x[l]);
                if (!(v <= amax) && !std::isnan(v)) amax = v;
            }
            float dd = amax / 127.0f;
            float inv = dd > 0.f ? 1.0f / dd : 0.f;
            int32_t s = 0;
            for (int l = 0; l < QK; ++l) {
                float r = std::round(x[l] * inv);
                int32_t qi;
                if (std::isnan(r)) qi = 0;  // Rust `NaN as i32` == 0
                else qi = int32_t(std::min(127.f, std::max(-127.f, r)));
                q[size_t(i) * k + size_t(bl) * QK + l] = int8_t(qi);
                s += qi;
            }
            d[size_t(i) * nb + bl] = dd;
            sum[size_t(i) * nb + bl] = s;
        }
    }
}

// ------------------------------------------------------- f32 dot kernels
constexpr int LANES = 8;

// tensor.rs:109-128: per-lane accumulators, sequential lane sum, tail.
// Rust's float `Sum` folds from -0.0.
float dot(const float* a, const float* b, int k) {
    float acc[LANES] = {0, 0, 0, 0, 0, 0, 0, 0};
    int k8 = k / LANES * LANES;
    for (int p = 0; p < k8; p += LANES)
        for (int l = 0; l < LANES; ++l) acc[l] += a[p + l] * b[p + l];
    float tail = -0.0f;
    for (int p = k8; p < k; ++p) tail += a[p] * b[p];
    float s = -0.0f;
    for (int l = 0; l < LANES; ++l) s += acc[l];
    return s + tail;
}

// tensor.rs:132-158: identical per-row arithmetic to dot(), 4 rows share b.
void dot4(const float* a0, const float* a1, const float* a2, const float* a3, const float* b, int k, float* out) {
    const float* as[4] = {a0, a1, a2, a3};
    float acc[4][LANES] = {};
    int k8 = k / LANES * LANES;
    for (int p = 0; p < k8; p += LANES)
        for (int l = 0; l < LANES; ++l)
            for (int r = 0; r < 4; ++r) acc[r][l] += as[r][p + l] * b[p + l];
    for (int r = 0; r < 4; ++r) {
        float tail = -0.0f;
        for (int p = k8; p < k; ++p) tail += as[r][p] * b[p];
        float s = -0.0f;
        for (int l = 0; l < LANES; ++l) s += acc[r][l];
        out[r] = s + tail;
    }
}

int n_threads_default() {
    unsigned t = std::thread::hardware_concurrency();
    return t ? int(t) : 1;
}

bool cpu_has_avx2() { return __builtin_cpu_supports("avx2"); }
bool cpu_has_vnni() { return __builtin_cpu_supports("avx512vnni") && __builtin_cpu_supports("avx512vl"); }

// Cached int8 unpack of a whole weight (quant.rs:515-524, 590-639).
struct Packed {
    std::vector<int8_t> q;
    std::vector<float> d, m;
    std::vector<int32_t> sum;
};

void build_packed(int dtype, const uint8_t* raw, int n, int k, Packed* pk) {
    int nb = k / QK, bb = block_bytes(dtype);
    pk->q.assign(size_t(n) * k, 0);
    pk->d.assign(size_t(n) * nb, 0.f);
    pk->m.assign(size_t(n) * nb, 0.f);
    pk->sum.assign(size_t(n) * nb, 0);
    for (int r = 0; r < n; ++r) {
        unpack_row_i8_avx2(dtype, raw + size_t(r) * nb * bb, &pk->q[size_t(r) * k], &pk->d[size_t(r) * nb],
                           &pk->m[size_t(r) * nb], nb);
        weight_block_sums_avx2(&pk->q[size_t(r) * k], &pk->sum[size_t(r) * nb], nb);
    }
}

struct QActs {
    std::vector<int8_t> q;
    std::vector<float> d;
    std::vector<int32_t> sum;
};

// One worker's share of quant.rs:790-1019: columns [j0, j0+cols) of every
// output row into block_out[m, cols].
void cols_block(int tier, const float* a, int m, int k, int dtype, const uint8_t* raw, const QActs* qa,
                const Packed* packed, int j0, int cols, float* block_out) {
    int nb = k / QK, bb = block_bytes(dtype);
    auto arow = [&](int i) { return RowRef{&qa->q[size_t(i) * k], &qa->d[size_t(i) * nb], &qa->sum[size_t(i) * nb]}; };
    bool vnni = tier == 1;
    if (tier == 1 || tier == 2) {
        std::vector<int8_t> qbs;
        std::vector<float> dbs, mbs;
        std::vector<int32_t> sbs;
        if (!packed) {
            qbs.assign(size_t(N_BLOCK) * k, 0);
            dbs.assign(size_t(N_BLOCK) * nb, 0.f);
            mbs.assign(size_t(N_BLOCK) * nb, 0.f);
            sbs.assign(size_t(N_BLOCK) * nb, 0);
        }
        for (int m0 = 0; m0 < m; m0 += M_BLOCK) {
            int m1 = std::min(m0 + M_BLOCK, m);
            for (int j = j0; j < j0 + cols; j += N_BLOCK) {
                int jn = std::min(N_BLOCK, j0 + cols - j);
                const int8_t* qb[N_BLOCK];
                const float *db[N_BLOCK], *mb[N_BLOCK];
                const int32_t* sb[N_BLOCK];
                for (int r = 0; r < jn; ++r) {
                    if (packed) {
                        qb[r] = &packed->q[size_t(j + r) * k];
                        db[r] = &packed->d[size_t(j + r) * nb];
                        mb[r] = &packed->m[size_t(j + r) * nb];
                        sb[r] = &packed->sum[size_t(j + r) * nb];
                    } else {
                        // cold path: unpack into scratch (quant.rs:900-918)
                        unpack_row_i8_avx2(dtype, raw + size_t(j + r) * nb * bb, &qbs[size_t(r) * k],
                                           &dbs[size_t(r) * nb], &mbs[size_t(r) * nb], nb);
                        if (vnni) weight_block_sums_avx2(&qbs[size_t(r) * k], &sbs[size_t(r) * nb], nb);
                        qb[r] = &qbs[size_t(r) * k];
                        db[r] = &dbs[size_t(r) * nb];
                        mb[r] = &mbs[size_t(r) * nb];
                        sb[r] = &sbs[size_t(r) * nb];
                    }
                }
                int i = m0;
                for (; i + 4 <= m1; i += 4) {
                    RowRef rows[4] = {arow(i), arow(i + 1), arow(i + 2), arow(i + 3)};
                    for (int r = 0; r < jn; ++r) {
                        float o[4];
                        if (vnni) dot_i8_vnni_x4(rows, qb[r], db[r], mb[r], sb[r], nb, o);
                        else dot_i8_avx2_x4(rows, qb[r], db[r], mb[r], nb, o);
                        for (int rr = 0; rr < 4; ++rr) block_out[size_t(i + rr) * cols + (j + r - j0)] = o[rr];
                    }
                }
                for (; i < m1; ++i)
                    for (int r = 0; r < jn; ++r)
                        block_out[size_t(i) * cols + (j + r - j0)] =
                            vnni ? dot_i8_vnni(arow(i), qb[r], db[r], mb[r], sb[r], nb)
                                 : dot_i8_avx2(arow(i), qb[r], db[r], mb[r], nb);
            }
        }
        return;
    }
    // f32 fallback (quant.rs:995-1018)
    std::vector<float> fb(k);
    for (int j = j0; j < j0 + cols; ++j) {
        dequant_row_avx2(dtype, raw + size_t(j) * nb * bb, nb, fb.data());
        int i = 0;
        for (; i + 4 <= m; i += 4) {
            float s[4];
            dot4(a + size_t(i) * k, a + size_t(i + 1) * k, a + size_t(i + 2) * k, a + size_t(i + 3) * k, fb.data(), k,
                 s);
            for (int r = 0; r < 4; ++r) block_out[size_t(i + r) * cols + (j - j0)] = s[r];
        }
        for (; i < m; ++i) block_out[size_t(i) * cols + (j - j0)] = dot(a + size_t(i) * k, fb.data(), k);
    }
}

}  // namespace

extern "C" {

float orc_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
uint16_t orc_f32_to_f16(float x) { return f32_to_f16(x); }
int orc_block_bytes(int dtype) { return block_bytes(dtype); }
int orc_has_avx2(void) { return cpu_has_avx2() ? 1 : 0; }
int orc_has_vnni(void) { return cpu_has_vnni() ? 1 : 0; }
int orc_default_threads(void) { return n_threads_default(); }

// Tier the reference dispatches to on this host: 1 VNNI, 2 AVX2, 3 f32.
int orc_dispatch_tier(void) { return cpu_has_vnni() ? 1 : (cpu_has_avx2() ? 2 : 3); }

int orc_unpack_block(int dtype, const uint8_t* block, int8_t* q, float* d, float* m) {
    return unpack_block(dtype, block, q, d, m) ? 0 : -1;
}

int orc_dequant_row_scalar(int dtype, const uint8_t* raw, size_t nblocks, float* out) {
    if (block_bytes(dtype) < 0) return -1;
    dequant_row_scalar(dtype, raw, nblocks, out);
    return 0;
}

int orc_dequant_row_avx2(int dtype, const uint8_t* raw, size_t nblocks, float* out) {
    if (block_bytes(dtype) < 0 || !cpu_has_avx2()) return -1;
    dequant_row_avx2(dtype, raw, nblocks, out);
    return 0;
}

int orc_quantize_acts_i8(const float* a, int m, int k, int8_t* q, float* d, int32_t* sum) {
    if (k % QK) return -1;
    quantize_acts_i8(a, m, k, q, d, sum);
    return 0;
}

// Per-block integer dots S[i][j][kb] = sum_l q_a[i,kb*32+l] * q_b[j,kb*32+l]
// with q_b the centred quants of unpack_block (the integer core of
// quant.rs:1352-1360).
int orc_block_dots(const int8_t* qa, int m, int k, int dtype, const uint8_t* raw, int n, int32_t* S) {
    int bb = block_bytes(dtype);
    if (bb < 0 || k % QK) return -1;
    int nb = k / QK;
    std::vector<int8_t> qb(size_t(n) * k);
    std::vector<float> tmp(2);
    for (int j = 0; j < n; ++j)
        for (int bl = 0; bl < nb; ++bl)
            unpack_block(dtype, raw + (size_t(j) * nb + bl) * bb, &qb[size_t(j) * k + size_t(bl) * QK], &tmp[0],
                         &tmp[1]);
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j)
            for (int bl = 0; bl < nb; ++bl) {
                int32_t s = 0;
                for (int l = 0; l < QK; ++l)
                    s += int32_t(qa[size_t(i) * k + size_t(bl) * QK + l]) * int32_t(qb[size_t(j) * k + size_t(bl) * QK + l]);
                S[(size_t(i) * n + j) * nb + bl] = s;
            }
    return 0;
}

// The scalar int8 reference of quant.rs:1346-1362, extended with the
// asymmetric term: acc += d_a*d_b*s + m_b*d_a*sum(q_a), per block in order.
int orc_int8_scalar_matmul(const float* a, int m, int k, int dtype, const uint8_t* raw, int n, float* out) {
    int bb = block_bytes(dtype);
    if (bb < 0 || k % QK) return -1;
    int nb = k / QK;
    std::vector<int8_t> q(size_t(m) * k);
    std::vector<float> d(size_t(m) * nb);
    std::vector<int32_t> sum(size_t(m) * nb);
    quantize_acts_i8(a, m, k, q.data(), d.data(), sum.data());
    int8_t qb[QK];
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) {
            float acc = 0.f;
            for (int bl = 0; bl < nb; ++bl) {
                float db, mb;
                unpack_block(dtype, raw + (size_t(j) * nb + bl) * bb, qb, &db, &mb);
                int32_t s = 0;
                for (int l = 0; l < QK; ++l) s += int32_t(q[size_t(i) * k + size_t(bl) * QK + l]) * int32_t(qb[l]);
                acc += d[size_t(i) * nb + bl] * db * float(s);
                acc += mb * d[size_t(i) * nb + bl] * float(sum[size_t(i) * nb + bl]);
            }
            out[size_t(i) * n + j] = acc;
        }
    return 0;
}

// quant.rs:754-1051.  tier: 0 = what the reference dispatches here,
// 1 = VNNI, 2 = AVX2, 3 = f32 fallback.  threads: 0 = all cores
// (available_parallelism).  packed: 0 = cold path (first call on a
// weight), 1 = cached int8 unpack (second call on; quant.rs:778-786).
int orc_matmul_t_q(const float* a, int m, int k, int dtype, const uint8_t* raw, int n, float* out, int tier,
                   int threads, int packed) {
    if (block_bytes(dtype) < 0 || k % QK || m < 0 || n < 0) return -1;
    if (tier == 0) tier = orc_dispatch_tier();
    if (tier == 1 && !cpu_has_vnni()) return -2;
    if ((tier == 1 || tier == 2 || tier == 3) && !cpu_has_avx2()) return -2;  // restated kernels need avx2
    if (threads <= 0) threads = n_threads_default();
    if (m == 0 || n == 0) return 0;
    QActs qa;
    if (tier != 3) {
        int nb = k / QK;
        qa.q.resize(size_t(m) * k);
        qa.d.resize(size_t(m) * nb);
        qa.sum.resize(size_t(m) * nb);
        quantize_acts_i8(a, m, k, qa.q.data(), qa.d.data(), qa.sum.data());
    }
    Packed pk;
    const Packed* pkp = nullptr;
    if (packed && tier != 3) {
        build_packed(dtype, raw, n, k, &pk);
        pkp = &pk;
    }
    if (threads > 1 && size_t(m) * n * k > PAR_THRESHOLD) {
        int chunk = (n + threads - 1) / threads;
        int nchunks = (n + chunk - 1) / chunk;
        std::vector<std::vector<float>> bufs(nchunks);
        std::vector<std::thread> ths;
        for (int c = 0; c < nchunks; ++c) {
            ths.emplace_back([&, c] {
                int j0 = c * chunk, cols = std::min(chunk, n - j0);
                bufs[c].assign(size_t(m) * cols, 0.f);
                cols_block(tier, a, m, k, dtype, raw, &qa, pkp, j0, cols, bufs[c].data());
            });
        }
        for (auto& t : ths) t.join();
        for (int c = 0; c < nchunks; ++c) {
            int j0 = c * chunk, cols = std::min(chunk, n - j0);
            for (int i = 0; i < m; ++i)
                std::memcpy(out + size_t(i) * n + j0, &bufs[c][size_t(i) * cols], sizeof(float) * cols);
        }
    } else {
        cols_block(tier, a, m, k, dtype, raw, &qa, pkp, 0, n, out);
    }
    return 0;
}

// A weight that persists across calls, like QTensor with its call-count
// gated cache (quant.rs:495-513, 778-786): call 1 takes the cold path,
// call 2 builds the packed int8 unpack (row-parallel, quant.rs:601-635),
// calls 2+ read it.  Used to time the reference's steady state.
struct OrcQTensor {
    int dtype, n, k;
    std::vector<uint8_t> raw;
    Packed packed;
    bool have_packed = false;
    size_t calls = 0;
};

void* orc_qtensor_new(int dtype, const uint8_t* raw, int n, int k) {
    if (block_bytes(dtype) < 0 || k % QK || n < 0) return nullptr;
    auto* t = new OrcQTensor{dtype, n, k, {}, {}, false, 0};
    t->raw.assign(raw, raw + size_t(n) * (k / QK) * block_bytes(dtype));
    return t;
}

void orc_qtensor_free(void* h) { delete static_cast<OrcQTensor*>(h); }

int orc_qtensor_matmul(void* h, const float* a, int m, float* out, int tier, int threads) {
    auto* t = static_cast<OrcQTensor*>(h);
    if (!t) return -1;
    int n = t->n, k = t->k, dtype = t->dtype, nb = k / QK, bb = block_bytes(dtype);
    if (tier == 0) tier = orc_dispatch_tier();
    if (tier == 1 && !cpu_has_vnni()) return -2;
    if (!cpu_has_avx2()) return -2;
    if (threads <= 0) threads = n_threads_default();
    size_t prior = t->calls++;
    if (m == 0 || n == 0) return 0;
    QActs qa;
    if (tier != 3) {
        qa.q.resize(size_t(m) * k);
        qa.d.resize(size_t(m) * nb);
        qa.sum.resize(size_t(m) * nb);
        quantize_acts_i8(a, m, k, qa.q.data(), qa.d.data(), qa.sum.data());
    }
    const Packed* pkp = nullptr;
    if (tier != 3 && prior >= 1) {
        if (!t->have_packed) {
            Packed& pk = t->packed;
            pk.q.assign(size_t(n) * k, 0);
            pk.d.assign(size_t(n) * nb, 0.f);
            pk.m.assign(size_t(n) * nb, 0.f);
            pk.sum.assign(size_t(n) * nb, 0);
            auto pack_rows = [&](int r0, int r1) {
                for (int r = r0; r < r1; ++r) {
                    unpack_row_i8_avx2(dtype, t->raw.data() + size_t(r) * nb * bb, &pk.q[size_t(r) * k],
                                       &pk.d[size_t(r) * nb], &pk.m[size_t(r) * nb], nb);
                    weight_block_sums_avx2(&pk.q[size_t(r) * k], &pk.sum[size_t(r) * nb], nb);
                }
            };
            if (threads > 1 && n > threads) {
                int chunk = (n + threads - 1) / threads;
                std::vector<std::thread> ths;
                for (int r0 = 0; r0 < n; r0 += chunk) ths.emplace_back(pack_rows, r0, std::min(n, r0 + chunk));
                for (auto& th : ths) th.join();
            } else {
                pack_rows(0, n);
            }
            t->have_packed = true;
        }
        pkp = &t->packed;
    }
    const uint8_t* raw = t->raw.data();
    if (threads > 1 && size_t(m) * n * k > PAR_THRESHOLD) {
        int chunk = (n + threads - 1) / threads;
        int nchunks = (n + chunk - 1) / chunk;
        std::vector<std::vector<float>> bufs(nchunks);
        std::vector<std::thread> ths;
        for (int c = 0; c < nchunks; ++c) {
            ths.emplace_back([&, c] {
                int j0 = c * chunk, cols = std::min(chunk, n - j0);
                bufs[c].assign(size_t(m) * cols, 0.f);
                cols_block(tier, a, m, k, dtype, raw, &qa, pkp, j0, cols, bufs[c].data());
            });
        }
        for (auto& th : ths) th.join();
        for (int c = 0; c < nchunks; ++c) {
            int j0 = c * chunk, cols = std::min(chunk, n - j0);
            for (int i = 0; i < m; ++i)
                std::memcpy(out + size_t(i) * n + j0, &bufs[c][size_t(i) * cols], sizeof(float) * cols);
        }
    } else {
        cols_block(tier, a, m, k, dtype, raw, &qa, pkp, 0, n, out);
    }
    return 0;
}

// Dense C = A[m,k] * B[n,k]^T with the reference's dot/dot4 arithmetic
// (tensor.rs:165-258).  Per-output results do not depend on the thread
// split, so this runs a plain row-parallel loop.
int orc_matmul_t(const float* a, int m, int k, const float* b, int n, float* out, int threads) {
    if (threads <= 0) threads = n_threads_default();
    auto rows = [&](int i0, int i1) {
        int i = i0;
        for (; i + 4 <= i1; i += 4)
            for (int j = 0; j < n; ++j) {
                float s[4];
                dot4(a + size_t(i) * k, a + size_t(i + 1) * k, a + size_t(i + 2) * k, a + size_t(i + 3) * k,
                     b + size_t(j) * k, k, s);
                for (int r = 0; r < 4; ++r) out[size_t(i + r) * n + j] = s[r];
            }
        for (; i < i1; ++i)
            for (int j = 0; j < n; ++j) out[size_t(i) * n + j] = dot(a + size_t(i) * k, b + size_t(j) * k, k);
    };
    if (threads > 1 && m >= threads) {
        int chunk = (m + threads - 1) / threads;
        std::vector<std::thread> ths;
        for (int i0 = 0; i0 < m; i0 += chunk) ths.emplace_back(rows, i0, std::min(m, i0 + chunk));
        for (auto& t : ths) t.join();
    } else {
        rows(0, m);
    }
    return 0;
}

// Whole-tensor dequant (QTensor::to_dense, quant.rs:572-576).
int orc_to_dense(int dtype, const uint8_t* raw, int n, int k, float* out) {
    if (block_bytes(dtype) < 0 || k % QK) return -1;
    size_t nblocks = size_t(n) * (k / QK);
    if (cpu_has_avx2()) dequant_row_avx2(dtype, raw, nblocks, out);
    else dequant_row_scalar(dtype, raw, nblocks, out);
    return 0;
}

// ---------------------------------------------------- reference test data
// quant.rs:1115-1123: LCG, value (state>>8)/2^24*2-1.
void orc_test_matrix(int n, int k, uint32_t seed, float* out) {
    uint32_t state = seed;
    for (size_t i = 0; i < size_t(n) * k; ++i) {
        state = state * 1664525u + 1013904223u;
        out[i] = float(state >> 8) / float(1u << 24) * 2.0f - 1.0f;
    }
}

// quant.rs:1131-1135: LCG bytes (state>>16) as u8.
void orc_rand_bytes(uint32_t seed, size_t count, uint8_t* out) {
    uint32_t state = seed;
    for (size_t i = 0; i < count; ++i) {
        state = state * 1664525u + 1013904223u;
        out[i] = uint8_t(state >> 16);
    }
}

// quant.rs:1071-1083
void orc_quantize_q8_0(const float* x, size_t count, uint8_t* raw) {
    for (size_t b0 = 0; b0 < count; b0 += QK) {
        float amax = 0.f;
        for (int l = 0; l < QK; ++l) amax = std::max(amax, std::fabs(x[b0 + l]));
        float d = amax / 127.0f;
        float id = d > 0.f ? 1.0f / d : 0.f;
        uint16_t h = f32_to_f16(d);
        *raw++ = uint8_t(h);
        *raw++ = uint8_t(h >> 8);
        for (int l = 0; l < QK; ++l) {
            float r = std::min(127.f, std::max(-127.f, std::round(x[b0 + l] * id)));
            *raw++ = uint8_t(int8_t(int(r)));
        }
    }
}

// quant.rs:1088-1113
void orc_quantize_q5_1(const float* x, size_t count, uint8_t* raw) {
    for (size_t b0 = 0; b0 < count; b0 += QK) {
        float mn = 3.402823466e+38f, mx = -3.402823466e+38f;
        for (int l = 0; l < QK; ++l) {
            mn = std::min(mn, x[b0 + l]);
            mx = std::max(mx, x[b0 + l]);
        }
        float d = (mx - mn) / 31.0f;
        float id = d > 0.f ? 1.0f / d : 0.f;
        uint8_t qs[QK];
        for (int l = 0; l < QK; ++l)
            qs[l] = uint8_t(int(std::min(31.f, std::max(0.f, std::round((x[b0 + l] - mn) * id)))));
        uint16_t hd = f32_to_f16(d), hm = f32_to_f16(mn);
        *raw++ = uint8_t(hd); *raw++ = uint8_t(hd >> 8);
        *raw++ = uint8_t(hm); *raw++ = uint8_t(hm >> 8);
        uint32_t qh = 0;
        for (int e = 0; e < QK; ++e)
            if (qs[e] & 0x10) qh |= 1u << e;
        for (int b = 0; b < 4; ++b) *raw++ = uint8_t(qh >> (8 * b));
        for (int e = 0; e < 16; ++e) *raw++ = uint8_t((qs[e] & 0xF) | ((qs[e + 16] & 0xF) << 4));
    }
}

// ------------------------------------------------------------- log-mel
// audio.rs:10-198, operation for operation in f32 (libm sinf/cosf/logf/
// expf/log10f are what Rust's f32 methods call on this platform).

}  // extern "C"

namespace {

constexpr int A_N_FFT = 400, A_HOP = 160, A_N_FREQS = A_N_FFT / 2 + 1;
constexpr float A_PI = 3.14159265358979323846f;   // std::f32::consts::PI

// audio.rs:55-72
void dft_ref(const std::vector<float>& re, const std::vector<float>& im, std::vector<float>& ore,
             std::vector<float>& oim) {
    const size_t n = re.size();
    ore.assign(n, 0.f);
    oim.assign(n, 0.f);
    for (size_t k = 0; k < n; ++k) {
        float sr = 0.f, si = 0.f;
        for (size_t t = 0; t < n; ++t) {
            const float theta = -2.0f * A_PI * float(k * t) / float(n);
            const float s = std::sin(theta), c = std::cos(theta);
            sr += re[t] * c - im[t] * s;
            si += re[t] * s + im[t] * c;
        }
        ore[k] = sr;
        oim[k] = si;
    }
}

// audio.rs:20-53: even n splits into even/odd halves, odd n is a DFT.
void fft_ref(const std::vector<float>& re, const std::vector<float>& im, std::vector<float>& ore,
             std::vector<float>& oim) {
    const size_t n = re.size();
    if (n == 1) {
        ore = re;
        oim = im;
        return;
    }
    if (n % 2 == 1) {
        dft_ref(re, im, ore, oim);
        return;
    }
    const size_t half = n / 2;
    std::vector<float> er(half), ei(half), odr(half), odi(half);
    for (size_t i = 0; i < half; ++i) {
        er[i] = re[2 * i];
        ei[i] = im[2 * i];
        odr[i] = re[2 * i + 1];
        odi[i] = im[2 * i + 1];
    }
    std::vector<float> Er, Ei, Or, Oi;
    fft_ref(er, ei, Er, Ei);
    fft_ref(odr, odi, Or, Oi);
    ore.assign(n, 0.f);
    oim.assign(n, 0.f);
    for (size_t k = 0; k < half; ++k) {
        const float theta = -2.0f * A_PI * float(k) / float(n);
        const float s = std::sin(theta), c = std::cos(theta);
        const float tr = c * Or[k] - s * Oi[k];
        const float ti = c * Oi[k] + s * Or[k];
        ore[k] = Er[k] + tr;
        oim[k] = Ei[k] + ti;
        ore[k + half] = Er[k] - tr;
        oim[k + half] = Ei[k] - ti;
    }
}

// audio.rs:81-102 (Slaney scale)
float hz_to_mel(float hz) {
    const float F_SP = 200.0f / 3.0f, MIN_LOG_HZ = 1000.0f, MIN_LOG_MEL = MIN_LOG_HZ / F_SP;
    if (hz < MIN_LOG_HZ) return hz / F_SP;
    return MIN_LOG_MEL + std::log(hz / MIN_LOG_HZ) / (std::log(6.4f) / 27.0f);
}
float mel_to_hz(float mel) {
    const float F_SP = 200.0f / 3.0f, MIN_LOG_HZ = 1000.0f, MIN_LOG_MEL = MIN_LOG_HZ / F_SP;
    if (mel < MIN_LOG_MEL) return mel * F_SP;
    return MIN_LOG_HZ * std::exp((mel - MIN_LOG_MEL) * (std::log(6.4f) / 27.0f));
}

}  // namespace

extern "C" {

// audio.rs:74-79
void orc_hann_window(int n, float* out) {
    for (int i = 0; i < n; ++i) out[i] = 0.5f * (1.0f - std::cos(2.0f * A_PI * float(i) / float(n)));
}

int orc_fft(const float* re, const float* im, int n, float* ore, float* oim, int naive) {
    std::vector<float> r(re, re + n), m(im, im + n), a, b;
    if (naive) dft_ref(r, m, a, b);
    else fft_ref(r, m, a, b);
    std::memcpy(ore, a.data(), sizeof(float) * n);
    std::memcpy(oim, b.data(), sizeof(float) * n);
    return 0;
}

// audio.rs:107-130
void orc_mel_filterbank(int n_mels, int n_fft, int sample_rate, float* out) {
    const int n_freqs = n_fft / 2 + 1;
    const float fmax = float(sample_rate) / 2.0f;
    const float mel_max = hz_to_mel(fmax);
    std::vector<float> edges(size_t(n_mels) + 2);
    for (int i = 0; i < n_mels + 2; ++i) edges[size_t(i)] = mel_to_hz(mel_max * float(i) / float(n_mels + 1));
    std::fill(out, out + size_t(n_mels) * n_freqs, 0.f);
    for (int m = 0; m < n_mels; ++m) {
        const float f_lo = edges[size_t(m)], f_center = edges[size_t(m) + 1], f_hi = edges[size_t(m) + 2];
        const float norm = 2.0f / (f_hi - f_lo);
        for (int k = 0; k < n_freqs; ++k) {
            const float f = float(k) * float(sample_rate) / float(n_fft);
            const float w = std::fmin((f - f_lo) / (f_center - f_lo), (f_hi - f) / (f_hi - f_center));
            if (w > 0.0f) out[size_t(m) * n_freqs + k] = w * norm;
        }
    }
}

// audio.rs:147-198: `out` is n_mels x n_frames, n_frames = n / 160.
int orc_log_mel(const float* samples, int n, const float* filters, int n_mels, float* out, int* n_frames_out,
                int threads) {
    if (n < A_N_FFT / 2 + 1) return -1;
    std::vector<float> window(A_N_FFT);
    orc_hann_window(A_N_FFT, window.data());
    const int pad = A_N_FFT / 2;
    std::vector<float> padded(size_t(n) + 2 * pad);
    for (long i = 0; i < long(n) + 2 * pad; ++i) {
        long j = i - pad;
        if (j < 0) j = -j;
        else if (j >= n) j = 2L * (n - 1) - j;
        padded[size_t(i)] = samples[std::min<long>(j, n - 1)];
    }
    const int n_frames = n / A_HOP;
    std::vector<float> power(size_t(n_frames) * A_N_FREQS);
    auto frames = [&](int t0, int t1) {
        std::vector<float> re(A_N_FFT), im(A_N_FFT, 0.f), fr, fi;
        for (int t = t0; t < t1; ++t) {
            for (int i = 0; i < A_N_FFT; ++i) re[size_t(i)] = padded[size_t(t) * A_HOP + i] * window[size_t(i)];
            std::fill(im.begin(), im.end(), 0.f);
            fft_ref(re, im, fr, fi);
            for (int k = 0; k < A_N_FREQS; ++k)
                power[size_t(t) * A_N_FREQS + k] = fr[size_t(k)] * fr[size_t(k)] + fi[size_t(k)] * fi[size_t(k)];
        }
    };
    if (threads <= 0) threads = n_threads_default();
    if (threads > 1 && n_frames >= threads) {
        const int chunk = (n_frames + threads - 1) / threads;
        std::vector<std::thread> ths;
        for (int t0 = 0; t0 < n_frames; t0 += chunk) ths.emplace_back(frames, t0, std::min(n_frames, t0 + chunk));
        for (auto& th : ths) th.join();
    } else {
        frames(0, n_frames);
    }
    orc_matmul_t(filters, n_mels, A_N_FREQS, power.data(), n_frames, out, threads);
    const size_t total = size_t(n_mels) * n_frames;
    for (size_t i = 0; i < total; ++i) out[i] = std::log10(std::fmax(out[i], 1e-10f));
    float mmax = -3.40282347e+38f;   // f32::MIN
    for (size_t i = 0; i < total; ++i) mmax = std::fmax(mmax, out[i]);
    for (size_t i = 0; i < total; ++i) out[i] = (std::fmax(out[i], mmax - 8.0f) + 4.0f) / 4.0f;
    if (n_frames_out) *n_frames_out = n_frames;
    return 0;
}

}  // extern "C"

// ================================================================ encoder
// Restatement of the reference's encoder graph (encoder.rs:1-234) and the
// dense tensor ops it uses (tensor.rs:75-100 matmul, :274-370 layernorm,
// gelu, softmax, conv1d), with every quantized linear going through the
// persistent-weight matmul_t_q above (quant.rs:1054-1063 linear_w).
namespace {

// tensor.rs:274-289 (eps as ggml: 1e-5)
void ln_rows(float* x, size_t rows, int cols, const float* w, const float* b) {
    for (size_t r = 0; r < rows; ++r) {
        float* row = x + r * cols;
        float s = 0.f;
        for (int i = 0; i < cols; ++i) s += row[i];
        const float mean = s / float(cols);
        float v = 0.f;
        for (int i = 0; i < cols; ++i) v += (row[i] - mean) * (row[i] - mean);
        const float var = v / float(cols);
        const float inv = 1.0f / std::sqrt(var + 1e-5f);
        for (int i = 0; i < cols; ++i) row[i] = (row[i] - mean) * inv * w[i] + b[i];
    }
}

// tensor.rs:291-306 (tanh approximation)
void gelu_n(float* x, size_t n) {
    const float C = 0.7978846f;
    for (size_t i = 0; i < n; ++i) {
        const float t = x[i];
        x[i] = 0.5f * t * (1.0f + std::tanh(C * (t + 0.044715f * t * t * t)));
    }
}

// tensor.rs:309-331
void softmax_rows(float* x, size_t rows, int cols) {
    for (size_t r = 0; r < rows; ++r) {
        float* row = x + r * cols;
        float mx = -3.40282347e+38f;  // f32::MIN, folded with f32::max
        for (int i = 0; i < cols; ++i) mx = std::fmax(mx, row[i]);
        float sum = 0.f;
        for (int i = 0; i < cols; ++i) {
            row[i] = std::exp(row[i] - mx);
            sum += row[i];
        }
        for (int i = 0; i < cols; ++i) row[i] /= sum;
    }
}

// tensor.rs:335-370: input [in_ch][t], weight [out][in][kernel], pad kernel/2.
void conv1d_ref(const float* in, int in_ch, int t, const float* w, int out_ch, int kernel, const float* bias,
                int stride, float* out, int threads) {
    const int pad = kernel / 2, t_out = (t + 2 * pad - kernel) / stride + 1;
    auto chans = [&](int o0, int o1) {
        for (int oc = o0; oc < o1; ++oc)
            for (int ot = 0; ot < t_out; ++ot) {
                float sum = bias[oc];
                for (int ic = 0; ic < in_ch; ++ic) {
                    const float* wr = w + (size_t(oc) * in_ch + ic) * kernel;
                    const float* ir = in + size_t(ic) * t;
                    for (int k = 0; k < kernel; ++k) {
                        const long it = long(ot) * stride + k - pad;
                        if (it >= 0 && it < t) sum += wr[k] * ir[it];
                    }
                }
                out[size_t(oc) * t_out + ot] = sum;
            }
    };
    if (threads > 1 && out_ch >= threads) {
        const int chunk = (out_ch + threads - 1) / threads;
        std::vector<std::thread> ths;
        for (int o0 = 0; o0 < out_ch; o0 += chunk) ths.emplace_back(chans, o0, std::min(out_ch, o0 + chunk));
        for (auto& th : ths) th.join();
    } else {
        chans(0, out_ch);
    }
}

// tensor.rs:75-100: C = A[m,k] x B[k,n], zero A entries skipped.
void matmul_ref(const float* a, int m, int k, const float* b, int n, float* out) {
    std::fill(out, out + size_t(m) * n, 0.f);
    for (int i = 0; i < m; ++i) {
        float* o = out + size_t(i) * n;
        for (int p = 0; p < k; ++p) {
            const float av = a[size_t(i) * k + p];
            if (av == 0.0f) continue;
            const float* br = b + size_t(p) * n;
            for (int j = 0; j < n; ++j) o[j] += av * br[j];
        }
    }
}

// Test switches of the model restatements (not reference behaviour):
//   g_model_tier  0 = the dispatched tier for every quantized linear of the
//                 encoder/decoder restatements, 1 = VNNI, 2 = AVX2: the
//                 reference's two x86 tiers differ only in f32 rounding, so
//                 running both measures how far two valid runs of the
//                 reference drift apart through requantized layers;
//   g_attn_f16    1 = attention operands rounded to f16 (q, k, v and the
//                 unnormalised softmax weights exp(s - max), to nearest
//                 even), the narrowing the GPU attention kernels apply,
//                 so its effect on the outputs can be measured on the CPU.
int g_model_tier = 0;
int g_attn_f16 = 0;

// f32 -> f16 -> f32, round to nearest even (IEEE 754 binary16), written
// from the format's definition: 10 stored fraction bits, exponent range
// [-14, 15], subnormals down to 2^-24, overflow to infinity.
float round_f16(float x) {
    if (!std::isfinite(x)) return x;
    const float a = std::fabs(x);
    if (a >= 65520.0f) return std::copysign(INFINITY, x);   // rounds past the largest f16 (65504)
    int e;
    std::frexp(a, &e);                       // a = f * 2^e, f in [0.5, 1)
    const int q = std::max(e - 11, -24);     // quantum: 2^(e-11) (11 significant bits), 2^-24 floor
    const float u = std::ldexp(1.0f, q);
    const float r = std::nearbyint(a / u) * u;   // a / u is exact (power of two); nearbyint rounds half to even
    return std::copysign(r, x);
}

// encoder.rs:48-80 (mha_split_kv over already-projected q, k, v [t, n_state]).
void mha_ref(const float* q, int tq, const float* k, const float* v, int tkv, int n_state, int n_head, bool causal,
             float* out, int threads) {
    const int dh = n_state / n_head;
    const float scale = 1.0f / std::sqrt(float(dh));
    auto heads = [&](int h0, int h1) {
        std::vector<float> qh(size_t(tq) * dh), kh(size_t(tkv) * dh), vh(size_t(tkv) * dh), sc(size_t(tq) * tkv),
            oh(size_t(tq) * dh);
        for (int h = h0; h < h1; ++h) {
            for (int r = 0; r < tq; ++r)
                std::memcpy(&qh[size_t(r) * dh], q + size_t(r) * n_state + h * dh, sizeof(float) * dh);
            for (int r = 0; r < tkv; ++r) {
                std::memcpy(&kh[size_t(r) * dh], k + size_t(r) * n_state + h * dh, sizeof(float) * dh);
                std::memcpy(&vh[size_t(r) * dh], v + size_t(r) * n_state + h * dh, sizeof(float) * dh);
            }
            if (g_attn_f16) {
                for (auto* vec : {&qh, &kh, &vh})
                    for (auto& x : *vec) x = round_f16(x);
            }
            orc_matmul_t(qh.data(), tq, dh, kh.data(), tkv, sc.data(), 1);
            for (auto& s : sc) s *= scale;
            if (causal) {
                const int off = tkv - tq;
                for (int i = 0; i < tq; ++i)
                    for (int j = off + i + 1; j < tkv; ++j) sc[size_t(i) * tkv + j] = -INFINITY;
            }
            if (g_attn_f16) {
                // softmax with the weights exp(s - max) rounded to f16 before
                // P.V and the normaliser summed from the unrounded weights
                for (int i = 0; i < tq; ++i) {
                    float* row = &sc[size_t(i) * tkv];
                    float mx = -3.40282347e+38f;
                    for (int j = 0; j < tkv; ++j) mx = std::fmax(mx, row[j]);
                    float sum = 0.f;
                    for (int j = 0; j < tkv; ++j) {
                        const float e = std::exp(row[j] - mx);
                        sum += e;
                        row[j] = round_f16(e);
                    }
                    for (int j = 0; j < tkv; ++j) row[j] /= sum;
                }
            } else {
                softmax_rows(sc.data(), size_t(tq), tkv);
            }
            matmul_ref(sc.data(), tq, tkv, vh.data(), dh, oh.data());
            for (int r = 0; r < tq; ++r)
                std::memcpy(out + size_t(r) * n_state + h * dh, &oh[size_t(r) * dh], sizeof(float) * dh);
        }
    };
    if (threads > 1 && n_head > 1) {
        std::vector<std::thread> ths;
        const int per = (n_head + threads - 1) / threads;
        for (int h0 = 0; h0 < n_head; h0 += per) ths.emplace_back(heads, h0, std::min(n_head, h0 + per));
        for (auto& th : ths) th.join();
    } else {
        heads(0, n_head);
    }
}

struct OrcLayer {
    std::vector<float> attn_ln_w, attn_ln_b, q_b, v_b, o_b, mlp_ln_w, mlp_ln_b, fc1_b, fc2_b;
    OrcQTensor *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr, *fc1 = nullptr, *fc2 = nullptr;
};

struct OrcEncoder {
    int n_mels, n_ctx, n_state, n_head, n_layer;
    std::vector<float> conv1_w, conv1_b, conv2_w, conv2_b, pos, ln_post_w, ln_post_b;
    std::vector<OrcLayer> layers;
    ~OrcEncoder() {
        for (auto& l : layers)
            for (OrcQTensor* t : {l.q, l.k, l.v, l.o, l.fc1, l.fc2}) delete t;
    }
};

// quant.rs:1054-1063: y = x W^T (+ b) through the weight's own matmul_t_q.
void linear_q(OrcQTensor* w, const float* x, int m, const float* bias, float* y, int threads) {
    orc_qtensor_matmul(w, x, m, y, g_model_tier, threads);
    if (bias)
        for (int i = 0; i < m; ++i)
            for (int j = 0; j < w->n; ++j) y[size_t(i) * w->n + j] += bias[j];
}

}  // namespace

extern "C" {

void* orc_encoder_new(int n_mels, int n_ctx, int n_state, int n_head, int n_layer) {
    if (n_mels <= 0 || n_ctx <= 0 || n_state <= 0 || n_head <= 0 || n_state % n_head || n_layer < 0) return nullptr;
    auto* e = new OrcEncoder{n_mels, n_ctx, n_state, n_head, n_layer, {}, {}, {}, {}, {}, {}, {}, {}};
    e->layers.resize(size_t(n_layer));
    return e;
}

void orc_encoder_free(void* h) { delete static_cast<OrcEncoder*>(h); }

// Tensors by their whisper.cpp names (encoder.rs:130-234).  Dense ones are
// f32 arrays; the six linears per block are raw ggml blocks.
int orc_encoder_set(void* h, const char* name, const float* dense, size_t count, int dtype, const uint8_t* raw,
                    int n, int k) {
    auto* e = static_cast<OrcEncoder*>(h);
    std::string s(name);
    auto vec = [&](std::vector<float>& dst) {
        if (!dense) return -1;
        dst.assign(dense, dense + count);
        return 0;
    };
    if (s == "encoder.conv1.weight") return vec(e->conv1_w);
    if (s == "encoder.conv1.bias") return vec(e->conv1_b);
    if (s == "encoder.conv2.weight") return vec(e->conv2_w);
    if (s == "encoder.conv2.bias") return vec(e->conv2_b);
    if (s == "encoder.positional_embedding") return vec(e->pos);
    if (s == "encoder.ln_post.weight") return vec(e->ln_post_w);
    if (s == "encoder.ln_post.bias") return vec(e->ln_post_b);
    const std::string pre = "encoder.blocks.";
    if (s.compare(0, pre.size(), pre) != 0) return -1;
    size_t dot = s.find('.', pre.size());
    if (dot == std::string::npos) return -1;
    const int l = std::atoi(s.substr(pre.size(), dot - pre.size()).c_str());
    if (l < 0 || l >= e->n_layer) return -1;
    OrcLayer& L = e->layers[size_t(l)];
    const std::string f = s.substr(dot + 1);
    auto quant = [&](OrcQTensor*& dst) {
        if (!raw) return -1;
        delete dst;
        dst = static_cast<OrcQTensor*>(orc_qtensor_new(dtype, raw, n, k));
        return dst ? 0 : -1;
    };
    if (f == "attn_ln.weight") return vec(L.attn_ln_w);
    if (f == "attn_ln.bias") return vec(L.attn_ln_b);
    if (f == "attn.query.weight") return quant(L.q);
    if (f == "attn.query.bias") return vec(L.q_b);
    if (f == "attn.key.weight") return quant(L.k);
    if (f == "attn.value.weight") return quant(L.v);
    if (f == "attn.value.bias") return vec(L.v_b);
    if (f == "attn.out.weight") return quant(L.o);
    if (f == "attn.out.bias") return vec(L.o_b);
    if (f == "mlp_ln.weight") return vec(L.mlp_ln_w);
    if (f == "mlp_ln.bias") return vec(L.mlp_ln_b);
    if (f == "mlp.0.weight") return quant(L.fc1);
    if (f == "mlp.0.bias") return vec(L.fc1_b);
    if (f == "mlp.2.weight") return quant(L.fc2);
    if (f == "mlp.2.bias") return vec(L.fc2_b);
    return -1;
}

// encoder.rs:180-234 for one window: mel [n_mels][2*n_ctx] -> out [n_ctx][n_state].
int orc_encode(void* h, const float* mel, float* out, int threads) {
    auto* e = static_cast<OrcEncoder*>(h);
    if (!e) return -1;
    if (threads <= 0) threads = n_threads_default();
    const int T = e->n_ctx, D = e->n_state, F = 2 * T;
    for (auto& L : e->layers)
        if (!L.q || !L.k || !L.v || !L.o || !L.fc1 || !L.fc2) return -2;
    std::vector<float> c1(size_t(D) * F), c2(size_t(D) * T);
    conv1d_ref(mel, e->n_mels, F, e->conv1_w.data(), D, 3, e->conv1_b.data(), 1, c1.data(), threads);
    gelu_n(c1.data(), c1.size());
    conv1d_ref(c1.data(), D, F, e->conv2_w.data(), D, 3, e->conv2_b.data(), 2, c2.data(), threads);
    gelu_n(c2.data(), c2.size());
    std::vector<float> x(size_t(T) * D);
    for (int i = 0; i < D; ++i)
        for (int t = 0; t < T; ++t) x[size_t(t) * D + i] = c2[size_t(i) * T + t];
    for (size_t i = 0; i < x.size(); ++i) x[i] += e->pos[i];
    const int F4 = e->layers.empty() ? 0 : e->layers[0].fc1->n;
    std::vector<float> cur(x.size()), q(x.size()), k(x.size()), v(x.size()), att(x.size()), proj(x.size()),
        hbuf(size_t(T) * std::max(F4, 1));
    for (auto& L : e->layers) {
        cur = x;
        ln_rows(cur.data(), size_t(T), D, L.attn_ln_w.data(), L.attn_ln_b.data());
        linear_q(L.q, cur.data(), T, L.q_b.data(), q.data(), threads);
        linear_q(L.k, cur.data(), T, nullptr, k.data(), threads);
        linear_q(L.v, cur.data(), T, L.v_b.data(), v.data(), threads);
        mha_ref(q.data(), T, k.data(), v.data(), T, D, e->n_head, false, att.data(), threads);
        linear_q(L.o, att.data(), T, L.o_b.data(), proj.data(), threads);
        for (size_t i = 0; i < x.size(); ++i) x[i] += proj[i];
        cur = x;
        ln_rows(cur.data(), size_t(T), D, L.mlp_ln_w.data(), L.mlp_ln_b.data());
        linear_q(L.fc1, cur.data(), T, L.fc1_b.data(), hbuf.data(), threads);
        gelu_n(hbuf.data(), hbuf.size());
        linear_q(L.fc2, hbuf.data(), T, L.fc2_b.data(), proj.data(), threads);
        for (size_t i = 0; i < x.size(); ++i) x[i] += proj[i];
    }
    ln_rows(x.data(), size_t(T), D, e->ln_post_w.data(), e->ln_post_b.data());
    std::memcpy(out, x.data(), sizeof(float) * x.size());
    return 0;
}

// Pieces, for the kernels' own parity tests.
void orc_layernorm(float* x, size_t rows, int cols, const float* w, const float* b) { ln_rows(x, rows, cols, w, b); }
void orc_set_model_tier(int tier) { g_model_tier = (tier >= 0 && tier <= 2) ? tier : 0; }
void orc_set_attn_f16(int on) { g_attn_f16 = on ? 1 : 0; }
float orc_round_f16(float x) { return round_f16(x); }
void orc_gelu(float* x, size_t n) { gelu_n(x, n); }
int orc_mha(const float* q, int tq, const float* k, const float* v, int tkv, int n_state, int n_head, int causal,
            float* out, int threads) {
    if (n_head <= 0 || n_state % n_head) return -1;
    mha_ref(q, tq, k, v, tkv, n_state, n_head, causal != 0, out, threads <= 0 ? n_threads_default() : threads);
    return 0;
}
int orc_conv1d(const float* in, int in_ch, int t, const float* w, int out_ch, int kernel, const float* bias,
               int stride, float* out, int threads) {
    conv1d_ref(in, in_ch, t, w, out_ch, kernel, bias, stride, out, threads <= 0 ? n_threads_default() : threads);
    return 0;
}

}  // extern "C"

// ================================================================ decoder
// Restatement of the reference's KV-cached decoder (decoder.rs:36-321):
// cross K/V projected once per window, per step token + learned position,
// n_text_layer x {causal self-attention over the cache, cross-attention,
// MLP}, final LN, tied logits through the token-embedding matrix.
namespace {

struct OrcDecLayer {
    std::vector<float> attn_ln_w, attn_ln_b, q_b, v_b, o_b, x_ln_w, x_ln_b, xq_b, xv_b, xo_b, mlp_ln_w, mlp_ln_b,
        fc1_b, fc2_b;
    OrcQTensor *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr, *xq = nullptr, *xk = nullptr, *xv = nullptr,
               *xo = nullptr, *fc1 = nullptr, *fc2 = nullptr;
};

struct OrcDecoder {
    int n_vocab, n_ctx, n_state, n_head, n_layer;
    std::vector<float> pos, ln_w, ln_b;
    OrcQTensor* emb = nullptr;
    std::vector<OrcDecLayer> layers;
    // state
    int n_audio = 0;
    std::vector<std::vector<float>> cross_k, cross_v, self_k, self_v;
    int n_past = 0;
    bool owns = true;
    ~OrcDecoder() {
        if (!owns) return;
        delete emb;
        for (auto& l : layers)
            for (OrcQTensor* t : {l.q, l.k, l.v, l.o, l.xq, l.xk, l.xv, l.xo, l.fc1, l.fc2}) delete t;
    }
};

}  // namespace

extern "C" {

void* orc_decoder_new(int n_vocab, int n_ctx, int n_state, int n_head, int n_layer) {
    if (n_vocab <= 0 || n_ctx <= 0 || n_state <= 0 || n_head <= 0 || n_state % n_head || n_layer < 0) return nullptr;
    auto* d = new OrcDecoder{n_vocab, n_ctx, n_state, n_head, n_layer, {}, {}, {}, nullptr, {}, 0, {}, {}, {}, {}, 0,
                             true};
    d->layers.resize(size_t(n_layer));
    d->self_k.resize(size_t(n_layer));
    d->self_v.resize(size_t(n_layer));
    return d;
}

void orc_decoder_free(void* h) { delete static_cast<OrcDecoder*>(h); }

int orc_decoder_set(void* h, const char* name, const float* dense, size_t count, int dtype, const uint8_t* raw, int n,
                    int k) {
    auto* d = static_cast<OrcDecoder*>(h);
    std::string s(name);
    auto vec = [&](std::vector<float>& dst) {
        if (!dense) return -1;
        dst.assign(dense, dense + count);
        return 0;
    };
    auto quant = [&](OrcQTensor*& dst) {
        if (!raw) return -1;
        delete dst;
        dst = static_cast<OrcQTensor*>(orc_qtensor_new(dtype, raw, n, k));
        return dst ? 0 : -1;
    };
    if (s == "decoder.positional_embedding") return vec(d->pos);
    if (s == "decoder.ln.weight") return vec(d->ln_w);
    if (s == "decoder.ln.bias") return vec(d->ln_b);
    if (s == "decoder.token_embedding.weight") return quant(d->emb);
    const std::string pre = "decoder.blocks.";
    if (s.compare(0, pre.size(), pre) != 0) return -1;
    const size_t dot = s.find('.', pre.size());
    if (dot == std::string::npos) return -1;
    const int l = std::atoi(s.substr(pre.size(), dot - pre.size()).c_str());
    if (l < 0 || l >= d->n_layer) return -1;
    OrcDecLayer& L = d->layers[size_t(l)];
    const std::string f = s.substr(dot + 1);
    if (f == "attn_ln.weight") return vec(L.attn_ln_w);
    if (f == "attn_ln.bias") return vec(L.attn_ln_b);
    if (f == "attn.query.weight") return quant(L.q);
    if (f == "attn.query.bias") return vec(L.q_b);
    if (f == "attn.key.weight") return quant(L.k);
    if (f == "attn.value.weight") return quant(L.v);
    if (f == "attn.value.bias") return vec(L.v_b);
    if (f == "attn.out.weight") return quant(L.o);
    if (f == "attn.out.bias") return vec(L.o_b);
    if (f == "cross_attn_ln.weight") return vec(L.x_ln_w);
    if (f == "cross_attn_ln.bias") return vec(L.x_ln_b);
    if (f == "cross_attn.query.weight") return quant(L.xq);
    if (f == "cross_attn.query.bias") return vec(L.xq_b);
    if (f == "cross_attn.key.weight") return quant(L.xk);
    if (f == "cross_attn.value.weight") return quant(L.xv);
    if (f == "cross_attn.value.bias") return vec(L.xv_b);
    if (f == "cross_attn.out.weight") return quant(L.xo);
    if (f == "cross_attn.out.bias") return vec(L.xo_b);
    if (f == "mlp_ln.weight") return vec(L.mlp_ln_w);
    if (f == "mlp_ln.bias") return vec(L.mlp_ln_b);
    if (f == "mlp.0.weight") return quant(L.fc1);
    if (f == "mlp.0.bias") return vec(L.fc1_b);
    if (f == "mlp.2.weight") return quant(L.fc2);
    if (f == "mlp.2.bias") return vec(L.fc2_b);
    return -1;
}

// Decoder::new (decoder.rs:36-69): cross K (no bias) and V per layer from
// the window's encoder output [n_audio][n_state]; clears the self cache.
int orc_decoder_begin(void* h, const float* enc_out, int n_audio, int threads) {
    auto* d = static_cast<OrcDecoder*>(h);
    if (!d || n_audio <= 0) return -1;
    if (threads <= 0) threads = n_threads_default();
    d->n_audio = n_audio;
    d->cross_k.assign(size_t(d->n_layer), {});
    d->cross_v.assign(size_t(d->n_layer), {});
    for (int l = 0; l < d->n_layer; ++l) {
        OrcDecLayer& L = d->layers[size_t(l)];
        if (!L.xk || !L.xv) return -2;
        d->cross_k[size_t(l)].assign(size_t(n_audio) * d->n_state, 0.f);
        d->cross_v[size_t(l)].assign(size_t(n_audio) * d->n_state, 0.f);
        linear_q(L.xk, enc_out, n_audio, nullptr, d->cross_k[size_t(l)].data(), threads);
        linear_q(L.xv, enc_out, n_audio, L.xv_b.data(), d->cross_v[size_t(l)].data(), threads);
    }
    for (auto& v : d->self_k) v.clear();
    for (auto& v : d->self_v) v.clear();
    d->n_past = 0;
    return 0;
}

// Decoder::forward (decoder.rs:102-206, 315-321): logits [n_tok][n_vocab].
int orc_decoder_forward(void* h, const int32_t* tokens, int n_tok, float* logits, int threads) {
    auto* d = static_cast<OrcDecoder*>(h);
    if (!d || n_tok <= 0 || !d->emb) return -1;
    if (d->n_past + n_tok > d->n_ctx) return -3;   // context overflow (decoder.rs:115-120)
    if (threads <= 0) threads = n_threads_default();
    const int D = d->n_state, H = d->n_head;
    std::vector<float> x(size_t(n_tok) * D), cur, q(x.size()), kn(x.size()), vn(x.size()), att(x.size()),
        proj(x.size());
    const int nbe = D / QK, bb = block_bytes(d->emb->dtype);
    for (int i = 0; i < n_tok; ++i) {
        if (tokens[i] < 0 || tokens[i] >= d->n_vocab) return -4;
        dequant_row_scalar(d->emb->dtype, d->emb->raw.data() + size_t(tokens[i]) * nbe * bb, size_t(nbe),
                           &x[size_t(i) * D]);
        for (int c = 0; c < D; ++c) x[size_t(i) * D + c] += d->pos[size_t(d->n_past + i) * D + c];
    }
    for (int l = 0; l < d->n_layer; ++l) {
        OrcDecLayer& L = d->layers[size_t(l)];
        cur = x;
        ln_rows(cur.data(), size_t(n_tok), D, L.attn_ln_w.data(), L.attn_ln_b.data());
        linear_q(L.q, cur.data(), n_tok, L.q_b.data(), q.data(), threads);
        linear_q(L.k, cur.data(), n_tok, nullptr, kn.data(), threads);
        linear_q(L.v, cur.data(), n_tok, L.v_b.data(), vn.data(), threads);
        d->self_k[size_t(l)].insert(d->self_k[size_t(l)].end(), kn.begin(), kn.end());
        d->self_v[size_t(l)].insert(d->self_v[size_t(l)].end(), vn.begin(), vn.end());
        const int t_kv = d->n_past + n_tok;
        mha_ref(q.data(), n_tok, d->self_k[size_t(l)].data(), d->self_v[size_t(l)].data(), t_kv, D, H, true,
                att.data(), 1);
        linear_q(L.o, att.data(), n_tok, L.o_b.data(), proj.data(), threads);
        for (size_t i = 0; i < x.size(); ++i) x[i] += proj[i];
        cur = x;
        ln_rows(cur.data(), size_t(n_tok), D, L.x_ln_w.data(), L.x_ln_b.data());
        linear_q(L.xq, cur.data(), n_tok, L.xq_b.data(), q.data(), threads);
        mha_ref(q.data(), n_tok, d->cross_k[size_t(l)].data(), d->cross_v[size_t(l)].data(), d->n_audio, D, H, false,
                att.data(), 1);
        linear_q(L.xo, att.data(), n_tok, L.xo_b.data(), proj.data(), threads);
        for (size_t i = 0; i < x.size(); ++i) x[i] += proj[i];
        cur = x;
        ln_rows(cur.data(), size_t(n_tok), D, L.mlp_ln_w.data(), L.mlp_ln_b.data());
        std::vector<float> hb(size_t(n_tok) * L.fc1->n);
        linear_q(L.fc1, cur.data(), n_tok, L.fc1_b.data(), hb.data(), threads);
        gelu_n(hb.data(), hb.size());
        linear_q(L.fc2, hb.data(), n_tok, L.fc2_b.data(), proj.data(), threads);
        for (size_t i = 0; i < x.size(); ++i) x[i] += proj[i];
    }
    d->n_past += n_tok;
    ln_rows(x.data(), size_t(n_tok), D, d->ln_w.data(), d->ln_b.data());
    linear_q(d->emb, x.data(), n_tok, nullptr, logits, threads);
    return 0;
}

void orc_decoder_reset(void* h) {
    auto* d = static_cast<OrcDecoder*>(h);
    for (auto& v : d->self_k) v.clear();
    for (auto& v : d->self_v) v.clear();
    d->n_past = 0;
}

int orc_decoder_n_past(void* h) { return static_cast<OrcDecoder*>(h)->n_past; }

}  // extern "C"
