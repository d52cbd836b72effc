// rwq_mel.cu -- the log-mel front end on the GPU (reference audio.rs:10-198,
// `log_mel_spectrogram`), batched over independent windows.
//
// Per window of n samples (16 kHz): reflect-pad 200 samples on both sides,
// n/160 frames of 400 samples times the periodic Hann window, the power of
// the 201 one-sided DFT bins, the mel filterbank, log10(max(v, 1e-10)),
// then, with the window's maximum M, (max(v, M - 8) + 4) / 4.  Output is
// [n_mels][n_frames] per window (whisper.cpp's layout).
//
// Kernels:
//   k_log_mel    one CTA per 32 frames of one window, one warp per frame:
//                the frame's 400 real samples packed as 200 complex values
//                (even + i*odd), a 200-point Stockham FFT in shared memory
//                (radix 2, 4, 5, 5), the real spectrum unpacked, power,
//                the filterbank over each band's nonzero bins, log10; the
//                32 x n_mels tile leaves coalesced; the CTA's maximum goes
//                to the window's slot with an order-preserving atomicMax.
//   k_mel_norm   the clamp and affine normalisation, elementwise.
// Twiddles come from a double-precision table rounded to f32; the FFT's
// rounding therefore differs from the reference's f32 recursion, which the
// parity tests bound (not bit-exact).
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>
#include <cuda_runtime.h>
#include "rwq.h"
#include "rwq_common.cuh"
#include "rwq_internal.h"

namespace {

constexpr int N_FFT = 400, HOP = 160, PAD = N_FFT / 2, N_FREQS = N_FFT / 2 + 1, NC = N_FFT / 2;   // NC: complex points
constexpr int FT = 32;                       // frames per CTA
constexpr int WARPS = 8;
constexpr int THREADS = WARPS * 32;
constexpr int SEG = FT * HOP + N_FFT - HOP;  // samples a CTA needs

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    rwq::set_last_error(buf);
    return code;
}

// Monotone map f32 -> u32 (so unsigned max is float max, NaN aside).
__device__ __forceinline__ unsigned order_f32(float f) {
    const unsigned u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float unorder_f32(unsigned u) {
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u);
}

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
    return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }

// One Stockham pass of radix R over NC points: butterfly j reads
// in[j + r*NC/R], applies W_{Ns*R}^{(j % Ns) r}, does a size-R DFT and
// writes out[(j / Ns) * Ns * R + j % Ns + r * Ns].  `tw` is W_NC^i, i < NC.
template <int R>
__device__ __forceinline__ void stockham_pass(const float2* in, float2* out, int Ns, const float2* tw, int lane) {
    constexpr int B = NC / R;
    for (int j = lane; j < B; j += 32) {
        float2 v[R];
        const int jm = j % Ns;
        const int step = (NC / (Ns * R)) * jm;   // twiddle index stride for this butterfly
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const float2 x = in[j + r * B];
            v[r] = r == 0 ? x : cmul(x, tw[(step * r) % NC]);
        }
        float2 y[R];
        if (R == 2) {
            y[0] = cadd(v[0], v[1]);
            y[1] = csub(v[0], v[1]);
        } else if (R == 4) {
            const float2 a = cadd(v[0], v[2]), b = csub(v[0], v[2]);
            const float2 c = cadd(v[1], v[3]), d = csub(v[1], v[3]);
            y[0] = cadd(a, c);
            y[2] = csub(a, c);
            y[1] = make_float2(b.x + d.y, b.y - d.x);   // b - i d
            y[3] = make_float2(b.x - d.y, b.y + d.x);   // b + i d
        } else {   // R == 5: direct, W_5^q = W_NC^(q * NC/5)
#pragma unroll
            for (int q = 0; q < R; ++q) {
                float2 acc = v[0];
#pragma unroll
                for (int r = 1; r < R; ++r) acc = cadd(acc, cmul(v[r], tw[((q * r) % R) * (NC / R)]));
                y[q] = acc;
            }
        }
        const int base = (j / Ns) * Ns * R + jm;
#pragma unroll
        for (int r = 0; r < R; ++r) out[base + r * Ns] = y[r];
    }
}

// Shared-memory layout of k_log_mel (byte offsets, each 16-byte aligned).
struct MelSmem {
    size_t tw, tw400, hann, seg, blo, blen, boff, bval, tile, wbuf, total;
};
constexpr int WBUF_F2 = 2 * NC + (N_FREQS + 1) / 2 + 1;   // per warp: two complex buffers + power
__host__ __device__ inline MelSmem mel_layout(int n_mels, int nnz) {
    MelSmem L;
    size_t o = 0;
    auto take = [&](size_t bytes) {
        const size_t at = o;
        o = (o + bytes + 15) / 16 * 16;
        return at;
    };
    L.tw = take(sizeof(float2) * NC);
    L.tw400 = take(sizeof(float2) * (N_FREQS + 1));
    L.hann = take(sizeof(float) * N_FFT);
    L.seg = take(sizeof(float) * SEG);
    L.blo = take(sizeof(int) * size_t(n_mels));
    L.blen = take(sizeof(int) * size_t(n_mels));
    L.boff = take(sizeof(int) * size_t(n_mels));
    L.bval = take(sizeof(float) * size_t(nnz));
    L.tile = take(sizeof(float) * size_t(n_mels) * FT);
    L.wbuf = take(sizeof(float2) * size_t(WARPS) * WBUF_F2);
    L.total = o;
    return L;
}

struct Bands {
    const int* lo;       // [n_mels] first nonzero bin
    const int* len;      // [n_mels] number of bins
    const int* off;      // [n_mels] offset into vals
    const float* vals;   // packed filter values
    int nnz;
};

__global__ void __launch_bounds__(THREADS) k_log_mel(const float* __restrict__ samples, int n_samples, int n_frames,
                                                     Bands bands, int n_mels, const float2* __restrict__ tw_g,
                                                     const float2* __restrict__ tw400_g,
                                                     const float* __restrict__ hann_g, float* __restrict__ out,
                                                     unsigned* __restrict__ wmax) {
    extern __shared__ __align__(16) uint8_t smem[];
    const MelSmem L = mel_layout(n_mels, bands.nnz);
    float2* tw = reinterpret_cast<float2*>(smem + L.tw);          // W_200^i, i < 200
    float2* tw400 = reinterpret_cast<float2*>(smem + L.tw400);    // W_400^k, k <= 201
    float* hann = reinterpret_cast<float*>(smem + L.hann);        // 400
    float* seg = reinterpret_cast<float*>(smem + L.seg);          // SEG samples
    int* blo = reinterpret_cast<int*>(smem + L.blo);
    int* blen = reinterpret_cast<int*>(smem + L.blen);
    int* boff = reinterpret_cast<int*>(smem + L.boff);
    float* bval = reinterpret_cast<float*>(smem + L.bval);
    float* tile = reinterpret_cast<float*>(smem + L.tile);        // [n_mels][FT]
    float2* wbuf = reinterpret_cast<float2*>(smem + L.wbuf);      // per warp: 2 x NC complex + power
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float2* z0 = wbuf + warp * WBUF_F2;
    float2* z1 = z0 + NC;
    float* pw = reinterpret_cast<float*>(z1 + NC);

    const int w = blockIdx.y, t0 = blockIdx.x * FT;
    const float* x = samples + size_t(w) * n_samples;
    for (int i = threadIdx.x; i < NC; i += THREADS) tw[i] = tw_g[i];
    for (int i = threadIdx.x; i <= N_FREQS; i += THREADS) tw400[i] = tw400_g[i];
    for (int i = threadIdx.x; i < N_FFT; i += THREADS) hann[i] = hann_g[i];
    for (int i = threadIdx.x; i < n_mels; i += THREADS) {
        blo[i] = bands.lo[i];
        blen[i] = bands.len[i];
        boff[i] = bands.off[i];
    }
    for (int i = threadIdx.x; i < bands.nnz; i += THREADS) bval[i] = bands.vals[i];
    // Frames t0..t0+FT-1 read padded samples [t0*HOP, t0*HOP + SEG); padded
    // index p is sample p - PAD reflected at both ends (torch.stft center).
    const int p0 = t0 * HOP;
    for (int i = threadIdx.x; i < SEG; i += THREADS) {
        int j = p0 + i - PAD;
        if (j < 0) j = -j;
        else if (j >= n_samples) j = 2 * (n_samples - 1) - j;
        j = j < 0 ? 0 : (j > n_samples - 1 ? n_samples - 1 : j);
        seg[i] = (p0 + i < n_samples + 2 * PAD) ? __ldg(x + j) : 0.f;
    }
    __syncthreads();

    float lmax = -3.40282347e+38f;
    for (int f = warp; f < FT; f += WARPS) {
        const int t = t0 + f;
        if (t >= n_frames) break;
        const float* fr = seg + f * HOP;
        // z[n] = x[2n] + i x[2n+1] (windowed)
        for (int n = lane; n < NC; n += 32)
            z0[n] = make_float2(fr[2 * n] * hann[2 * n], fr[2 * n + 1] * hann[2 * n + 1]);
        __syncwarp();
        stockham_pass<2>(z0, z1, 1, tw, lane);
        __syncwarp();
        stockham_pass<4>(z1, z0, 2, tw, lane);
        __syncwarp();
        stockham_pass<5>(z0, z1, 8, tw, lane);
        __syncwarp();
        stockham_pass<5>(z1, z0, 40, tw, lane);
        __syncwarp();
        // Real spectrum from Z = FFT(z): with E = (Z[k] + conj Z[-k]) / 2 and
        // O = (Z[k] - conj Z[-k]) / 2i, X[k] = E + W_400^k O, k = 0..200.
        for (int k = lane; k < N_FREQS; k += 32) {
            const float2 a = z0[k % NC], b = z0[(NC - k) % NC];
            const float2 e = make_float2(0.5f * (a.x + b.x), 0.5f * (a.y - b.y));
            const float2 o = make_float2(0.5f * (a.y + b.y), -0.5f * (a.x - b.x));
            const float2 X = cadd(e, cmul(tw400[k], o));
            pw[k] = X.x * X.x + X.y * X.y;
        }
        __syncwarp();
        for (int m = lane; m < n_mels; m += 32) {
            const int lo = blo[m], ln = blen[m], of = boff[m];
            float acc = 0.f;
            for (int q = 0; q < ln; ++q) acc = fmaf(bval[of + q], pw[lo + q], acc);
            const float v = log10f(fmaxf(acc, 1e-10f));
            tile[m * FT + f] = v;
            lmax = fmaxf(lmax, v);
        }
        __syncwarp();
    }
    // Warp, then CTA maximum -> the window's slot.
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
    __syncthreads();
    if (lane == 0) atomicMax(wmax + w, order_f32(lmax));
    const int nf = (n_frames - t0) < FT ? (n_frames - t0) : FT;
    float* o = out + size_t(w) * n_mels * n_frames;
    for (int i = threadIdx.x; i < n_mels * FT; i += THREADS) {
        const int m = i / FT, f = i % FT;
        if (f < nf) o[size_t(m) * n_frames + t0 + f] = tile[m * FT + f];
    }
}

__global__ void k_mel_norm(float* __restrict__ out, size_t per_window, int n_windows, const unsigned* __restrict__ wmax) {
    const size_t total = per_window * size_t(n_windows);
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
        const float mx = unorder_f32(wmax[i / per_window]);
        out[i] = (fmaxf(out[i], mx - 8.0f) + 4.0f) / 4.0f;
    }
}

__global__ void k_fill_u32(unsigned* p, int n, unsigned v) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}

}  // namespace

// A filterbank prepared for the GPU: each band's nonzero bins (a run of
// consecutive bins; zeros inside the run are kept), the FFT tables, and a
// per-window maximum slot array that grows with the batch.
struct rwq_mel {
    int n_mels = 0, nnz = 0, device = 0;
    int* lo = nullptr;
    int* len = nullptr;
    int* off = nullptr;
    float* vals = nullptr;
    float2* tw = nullptr;      // W_200^i
    float2* tw400 = nullptr;   // W_400^k, k <= 201
    float* hann = nullptr;
    unsigned* wmax = nullptr;
    int wcap = 0;
    std::mutex mu;
    ~rwq_mel() {
        cudaFree(lo);
        cudaFree(len);
        cudaFree(off);
        cudaFree(vals);
        cudaFree(tw);
        cudaFree(tw400);
        cudaFree(hann);
        cudaFree(wmax);
    }
};

namespace {

size_t smem_bytes(int n_mels, int nnz) { return mel_layout(n_mels, nnz).total; }

}  // namespace

extern "C" {

int rwq_mel_filterbank(int n_mels, int n_fft, int sample_rate, float* out) {
    // audio.rs:81-130: Slaney mel scale, band edges uniform in mel,
    // triangular filters with constant energy per band.
    if (n_mels <= 0 || n_fft <= 0 || sample_rate <= 0 || !out) return fail(RWQ_ERR_ARG, "bad filterbank arguments");
    auto hz_to_mel = [](float hz) {
        const float F_SP = 200.0f / 3.0f, MIN_LOG_HZ = 1000.0f, MIN_LOG_MEL = MIN_LOG_HZ / F_SP;
        if (hz < MIN_LOG_HZ) return hz / F_SP;
        return MIN_LOG_MEL + std::log(hz / MIN_LOG_HZ) / (std::log(6.4f) / 27.0f);
    };
    auto mel_to_hz = [](float mel) {
        const float F_SP = 200.0f / 3.0f, MIN_LOG_HZ = 1000.0f, MIN_LOG_MEL = MIN_LOG_HZ / F_SP;
        if (mel < MIN_LOG_MEL) return mel * F_SP;
        return MIN_LOG_HZ * std::exp((mel - MIN_LOG_MEL) * (std::log(6.4f) / 27.0f));
    };
    const int n_freqs = n_fft / 2 + 1;
    const float mel_max = hz_to_mel(float(sample_rate) / 2.0f);
    std::vector<float> edges(size_t(n_mels) + 2);
    for (int i = 0; i < n_mels + 2; ++i) edges[size_t(i)] = mel_to_hz(mel_max * float(i) / float(n_mels + 1));
    std::memset(out, 0, sizeof(float) * size_t(n_mels) * size_t(n_freqs));
    for (int m = 0; m < n_mels; ++m) {
        const float f_lo = edges[size_t(m)], f_c = edges[size_t(m) + 1], f_hi = edges[size_t(m) + 2];
        const float norm = 2.0f / (f_hi - f_lo);
        for (int k = 0; k < n_freqs; ++k) {
            const float f = float(k) * float(sample_rate) / float(n_fft);
            const float wv = std::fmin((f - f_lo) / (f_c - f_lo), (f_hi - f) / (f_hi - f_c));
            if (wv > 0.0f) out[size_t(m) * n_freqs + k] = wv * norm;
        }
    }
    return RWQ_OK;
}

int rwq_mel_new(const float* filters, int n_mels, rwq_mel** out) {
    if (!out) return fail(RWQ_ERR_ARG, "out is null");
    *out = nullptr;
    if (!filters || n_mels <= 0 || n_mels > 512) return fail(RWQ_ERR_ARG, "bad filterbank (n_mels %d)", n_mels);
    std::vector<int> lo(static_cast<size_t>(n_mels)), len(static_cast<size_t>(n_mels)), off(static_cast<size_t>(n_mels));
    std::vector<float> vals;
    for (int m = 0; m < n_mels; ++m) {
        const float* row = filters + size_t(m) * N_FREQS;
        int a = 0, b = N_FREQS;
        while (a < N_FREQS && row[a] == 0.0f) ++a;
        while (b > a && row[b - 1] == 0.0f) --b;
        lo[size_t(m)] = a;
        len[size_t(m)] = b - a;
        off[size_t(m)] = int(vals.size());
        vals.insert(vals.end(), row + a, row + b);
    }
    // Tables in double precision, rounded to f32.
    std::vector<float2> tw(NC), tw400(N_FREQS + 1);
    const double PI = 3.14159265358979323846;
    for (int i = 0; i < NC; ++i) tw[size_t(i)] = make_float2(float(std::cos(-2.0 * PI * i / NC)), float(std::sin(-2.0 * PI * i / NC)));
    for (int k = 0; k <= N_FREQS; ++k)
        tw400[size_t(k)] = make_float2(float(std::cos(-2.0 * PI * k / N_FFT)), float(std::sin(-2.0 * PI * k / N_FFT)));
    // The reference's periodic Hann window, f32 (audio.rs:74-79).
    std::vector<float> hann(N_FFT);
    for (int i = 0; i < N_FFT; ++i)
        hann[size_t(i)] = 0.5f * (1.0f - std::cos(2.0f * 3.14159265358979323846f * float(i) / float(N_FFT)));

    auto* p = new rwq_mel;
    p->n_mels = n_mels;
    p->nnz = int(vals.size());
    cudaGetDevice(&p->device);
    cudaError_t e = cudaSuccess;
    auto up = [&](void** dst, const void* src, size_t bytes) {
        if (e != cudaSuccess) return;
        if ((e = cudaMalloc(dst, bytes ? bytes : 16)) == cudaSuccess && bytes)
            e = cudaMemcpy(*dst, src, bytes, cudaMemcpyHostToDevice);
    };
    up(reinterpret_cast<void**>(&p->lo), lo.data(), sizeof(int) * lo.size());
    up(reinterpret_cast<void**>(&p->len), len.data(), sizeof(int) * len.size());
    up(reinterpret_cast<void**>(&p->off), off.data(), sizeof(int) * off.size());
    up(reinterpret_cast<void**>(&p->vals), vals.data(), sizeof(float) * vals.size());
    up(reinterpret_cast<void**>(&p->tw), tw.data(), sizeof(float2) * tw.size());
    up(reinterpret_cast<void**>(&p->tw400), tw400.data(), sizeof(float2) * tw400.size());
    up(reinterpret_cast<void**>(&p->hann), hann.data(), sizeof(float) * hann.size());
    if (e != cudaSuccess) {
        delete p;
        return fail(e == cudaErrorMemoryAllocation ? RWQ_ERR_NOMEM : RWQ_ERR_CUDA, "mel plan: %s",
                    cudaGetErrorString(e));
    }
    if (smem_bytes(n_mels, p->nnz) > 227 * 1024) {
        delete p;
        return fail(RWQ_ERR_ARG, "filterbank too large (%d mels, %d nonzeros)", n_mels, int(vals.size()));
    }
    *out = p;
    return RWQ_OK;
}

int rwq_mel_free(rwq_mel* p) {
    delete p;
    return RWQ_OK;
}

// Windows [n_windows][n_samples] -> [n_windows][n_mels][n_samples / 160],
// all on the device, asynchronous on `stream`.  One plan serves one stream
// at a time (its per-window maximum slots are reused).
int rwq_log_mel_dev(rwq_mel* p, const float* samples, int64_t n_windows, int64_t n_samples, float* out,
                    void* stream) {
    if (!p) return fail(RWQ_ERR_ARG, "plan is null");
    if (n_windows < 0 || n_windows > 65535) return fail(RWQ_ERR_ARG, "n_windows %lld out of range", (long long)n_windows);
    if (n_samples < PAD + 1 || n_samples > (int64_t(1) << 30))
        return fail(RWQ_ERR_ARG, "n_samples %lld: need at least %d", (long long)n_samples, PAD + 1);
    if (n_windows == 0) return RWQ_OK;
    if (!samples || !out) return fail(RWQ_ERR_ARG, "null samples or output");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    std::lock_guard<std::mutex> g(p->mu);
    cudaError_t e;
    if (n_windows > p->wcap) {
        cudaStreamSynchronize(s);
        cudaFree(p->wmax);
        p->wmax = nullptr;
        p->wcap = 0;
        if ((e = cudaMalloc(&p->wmax, sizeof(unsigned) * size_t(n_windows))) != cudaSuccess)
            return fail(RWQ_ERR_NOMEM, "mel scratch: %s", cudaGetErrorString(e));
        p->wcap = int(n_windows);
    }
    const int n_frames = int(n_samples / HOP);
    k_fill_u32<<<unsigned((n_windows + 255) / 256), 256, 0, s>>>(p->wmax, int(n_windows), 0u);
    const size_t smem = smem_bytes(p->n_mels, p->nnz);
    static int attr_dev_mask = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_dev_mask & (1 << dev))) {
        if ((e = cudaFuncSetAttribute(k_log_mel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024)) !=
            cudaSuccess)
            return fail(RWQ_ERR_CUDA, "mel kernel attribute: %s", cudaGetErrorString(e));
        attr_dev_mask |= 1 << dev;
    }
    Bands b{p->lo, p->len, p->off, p->vals, p->nnz};
    dim3 grid(unsigned((n_frames + FT - 1) / FT), unsigned(n_windows));
    if (n_frames > 0)
        k_log_mel<<<grid, THREADS, smem, s>>>(samples, int(n_samples), n_frames, b, p->n_mels, p->tw, p->tw400,
                                              p->hann, out, p->wmax);
    const size_t per = size_t(p->n_mels) * size_t(n_frames);
    if (per)
        k_mel_norm<<<unsigned(std::min<size_t>((per * n_windows + 255) / 256, 148 * 16)), 256, 0, s>>>(
            out, per, int(n_windows), p->wmax);
    if ((e = cudaGetLastError()) != cudaSuccess) return fail(RWQ_ERR_CUDA, "mel launch: %s", cudaGetErrorString(e));
    return RWQ_OK;
}

// One window, host buffers: out is [n_mels][n_samples / 160].
int rwq_log_mel(rwq_mel* p, const float* samples, int64_t n_samples, float* out) {
    if (!p) return fail(RWQ_ERR_ARG, "plan is null");
    if (!samples || !out) return fail(RWQ_ERR_ARG, "null samples or output");
    if (n_samples < PAD + 1 || n_samples > (int64_t(1) << 30))
        return fail(RWQ_ERR_ARG, "n_samples %lld: need at least %d", (long long)n_samples, PAD + 1);
    const size_t nout = size_t(p->n_mels) * size_t(n_samples / HOP);
    float *ds = nullptr, *dout = nullptr;
    cudaError_t e = cudaMalloc(&ds, sizeof(float) * size_t(n_samples));
    if (e == cudaSuccess) e = cudaMalloc(&dout, sizeof(float) * (nout ? nout : 1));
    if (e == cudaSuccess) e = cudaMemcpy(ds, samples, sizeof(float) * size_t(n_samples), cudaMemcpyHostToDevice);
    int rc = RWQ_OK;
    if (e == cudaSuccess) rc = rwq_log_mel_dev(p, ds, 1, n_samples, dout, nullptr);
    if (e == cudaSuccess && !rc) e = cudaMemcpy(out, dout, sizeof(float) * nout, cudaMemcpyDeviceToHost);
    cudaFree(ds);
    cudaFree(dout);
    if (rc) return rc;
    if (e != cudaSuccess) return fail(RWQ_ERR_CUDA, "log_mel: %s", cudaGetErrorString(e));
    return RWQ_OK;
}

}  // extern "C"
