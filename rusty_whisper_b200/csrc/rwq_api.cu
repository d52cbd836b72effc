// rwq_api.cu -- the C ABI (include/rwq.h): weight objects, per-stream
// scratch workspaces, argument checking and kernel dispatch.
//
// Dispatch of a matmul (quant.rs:754-1051 restated for the GPU):
//   mode INT8 (the reference's tier on every x86 host):
//     m <= 256 -> quantize (one launch), GEMV family (decoder shapes,
//                 HBM-bound): the integer-MMA kernels
//     m >  256 -> quantize (one launch), tcgen05 GEMM k_gemm_fold with the
//                 weight scales folded into the operand (encoder shapes);
//                 path 4 forces k_gemm_hl on the split dequantized
//                 activations
//   mode F32 (the reference's f32 fallback, dequant-then-f32):
//     m <= 256 -> dequant-then-f32 GEMV kernel over row chunks of 8
//     m >  256 -> split the f32 activations into f16 hi|lo, k_gemm_hl.
#include <cuda_runtime.h>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <functional>
#include <algorithm>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <utility>
#include "../../include/rwq.h"
#include "rwq_common.cuh"
#include "rwq_internal.h"
#include "rwq_encoder.h"

struct rwq_qtensor {
    rwq::Weight w;
    std::mutex mu;
};

// Quantized activations that outlive one call (rwq_qacts_*).
struct rwq_qacts {
    int device = 0;
    int max_m = 0, k = 0;
    void* buf = nullptr;
    rwq::ActsView v;       // valid rows: v.m
    int layout = rwq::LAYOUT_GEMV;   // the operand layout the last quantize produced
};

const rwq::Weight& rwq::weight_of(const rwq_qtensor* t) { return t->w; }

namespace {

thread_local std::string t_err;
thread_local int t_gemm_path = 0;

}  // namespace

void rwq::set_last_error(const char* msg) { t_err = msg; }

namespace {

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    t_err = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(e == cudaErrorMemoryAllocation ? RWQ_ERR_NOMEM : RWQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define RWQ_CUDA(call, what)                       \
    do {                                           \
        cudaError_t e_ = (call);                   \
        if (e_ != cudaSuccess) return cuda_fail(e_, what); \
    } while (0)

bool valid_dtype(int dt) { return rwq::block_bytes(dt) > 0; }

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Scratch arena for one (device, stream): grown on demand, never shrunk.
struct Workspace {
    std::mutex mu;
    void* buf = nullptr;
    size_t cap = 0;
    int* err = nullptr;  // device-side fault code written by kernels
};

// What an arena serves on its (device, stream): the device-pointer
// matmuls, the host-buffer entry points' copies of A/bias/C, and the
// block-dot dumps' scratch output.  Part of the key, so no stream handle
// value (cudaStreamLegacy, cudaStreamPerThread, ...) can alias another
// purpose's arena.
enum WsPurpose : int { WS_MATMUL = 0, WS_HOST_COPY = 1, WS_DOT_DUMP = 2 };

std::mutex g_ws_mu;
std::map<std::tuple<int, cudaStream_t, int>, Workspace*> g_ws;

int get_workspace(cudaStream_t s, Workspace** out, int purpose = WS_MATMUL) {
    int dev = 0;
    RWQ_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
    std::lock_guard<std::mutex> g(g_ws_mu);
    auto& w = g_ws[std::make_tuple(dev, s, purpose)];
    if (!w) {
        auto* nw = new Workspace;
        cudaError_t e = cudaMalloc(&nw->err, sizeof(int));
        if (e != cudaSuccess) {
            delete nw;
            return cuda_fail(e, "cudaMalloc(error flag)");
        }
        e = cudaMemset(nw->err, 0, sizeof(int));
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(error flag)");
        w = nw;
    }
    *out = w;
    return RWQ_OK;
}

int ensure_cap(Workspace* ws, size_t bytes) {
    if (ws->cap >= bytes) return RWQ_OK;
    if (ws->buf) {
        RWQ_CUDA(cudaFree(ws->buf), "cudaFree(workspace)");  // implicit device sync
        ws->buf = nullptr;
        ws->cap = 0;
    }
    const size_t want = align_up(bytes + bytes / 4, 1 << 20);
    RWQ_CUDA(cudaMalloc(&ws->buf, want), "cudaMalloc(workspace)");
    ws->cap = want;
    return RWQ_OK;
}

// Carve an activation view in `layout` out of the arena starting at
// `base` (nullptr: only measure).  Returns the bytes used.
size_t acts_layout(int m, int k, int layout, rwq::ActsView* v, uint8_t* base) {
    const int nb = k / rwq::QK;
    const int m_pad = (m + 255) / 256 * 256;   // the fold GEMM's CTA pairs cover 256 rows
    size_t off = 0;
    auto take = [&](size_t bytes) {
        uint8_t* p = base ? base + off : nullptr;
        off = align_up(off + bytes, 256);
        return p;
    };
    *v = rwq::ActsView();
    v->m = m;
    v->k = k;
    v->nb = nb;
    v->m_pad = m_pad;
    if (layout == rwq::LAYOUT_HL) {
        v->ahl = reinterpret_cast<uint16_t*>(take(size_t(m) * k * 4));
        v->rowscale = reinterpret_cast<float*>(take(size_t(m) * 4));
        return off;
    }
    v->q8 = reinterpret_cast<int8_t*>(take(size_t(m) * k));
    v->d = reinterpret_cast<float*>(take(size_t(m) * nb * 4));
    v->sum = reinterpret_cast<int32_t*>(take(size_t(m) * nb * 4));
    v->u = reinterpret_cast<float*>(take(size_t(m) * nb * 4));
    if (layout == rwq::LAYOUT_FOLD) {
        v->q16 = reinterpret_cast<uint16_t*>(take(size_t(m) * k * 2));
        v->dT = reinterpret_cast<float*>(take(size_t(nb) * m_pad * 4));
        v->uT = reinterpret_cast<float*>(take(size_t(nb) * m_pad * 4));
    }
    return off;
}

size_t acts_bytes_max(int m, int k) {
    rwq::ActsView v;
    size_t b = 0;
    for (int l : {rwq::LAYOUT_GEMV, rwq::LAYOUT_FOLD, rwq::LAYOUT_HL}) b = std::max(b, acts_layout(m, k, l, &v, nullptr));
    return b;
}

// Fill `v` (already carved in `layout`) from f32 activations `a`.
cudaError_t prepare_acts(const float* a, const rwq::ActsView& v, int layout, bool quantize, cudaStream_t s) {
    if (layout == rwq::LAYOUT_HL) return rwq::launch_split_rows(a, v.m, v.k, v.k, quantize, v.ahl, v.rowscale, s);
    return rwq::launch_quantize_acts(a, v, layout == rwq::LAYOUT_FOLD, s);
}

// Activation layout of a kernel path (1 GEMV family, 2 fold GEMM, 3 exact
// GEMM, 4 hi|lo GEMM).
int layout_of_path(int path) {
    return path == 1 ? rwq::LAYOUT_GEMV : path == 4 ? rwq::LAYOUT_HL : rwq::LAYOUT_FOLD;
}

int weight_gemm_cache(rwq_qtensor* t, cudaStream_t s) {
    std::lock_guard<std::mutex> g(t->mu);
    rwq::Weight& w = t->w;
    if (w.gemm_ready) return RWQ_OK;
    w.n_pad = (w.n + 127) / 128 * 128;
    RWQ_CUDA(cudaMalloc(&w.q16, size_t(w.n) * w.k * 2 + 16), "cudaMalloc(q16)");
    RWQ_CUDA(cudaMalloc(&w.dT, size_t(w.nb) * w.n_pad * 4), "cudaMalloc(dT)");
    if (rwq::has_min(w.dtype)) RWQ_CUDA(cudaMalloc(&w.mT, size_t(w.nb) * w.n_pad * 4), "cudaMalloc(mT)");
    RWQ_CUDA(rwq::launch_build_gemm_cache(w, s), "build gemm cache");
    // Other streams may use the cache next: finish building it here.
    RWQ_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize(gemm cache)");
    w.gemm_ready = true;
    return RWQ_OK;
}

int weight_fold_cache(rwq_qtensor* t, cudaStream_t s) {
    std::lock_guard<std::mutex> g(t->mu);
    rwq::Weight& w = t->w;
    if (w.fold_ready) return RWQ_OK;
    RWQ_CUDA(cudaMalloc(&w.bhl, size_t(w.n) * w.nb * 64 * 2 + 16), "cudaMalloc(bhl)");
    RWQ_CUDA(cudaMalloc(&w.colscale, size_t((w.n + 255) / 256 * 256) * 4), "cudaMalloc(colscale)");
    RWQ_CUDA(rwq::launch_build_fold_cache(w, s), "build fold cache");
    RWQ_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize(fold cache)");
    w.fold_ready = true;
    return RWQ_OK;
}

int check_matmul_args(const float* a, int64_t m, int64_t k, const rwq_qtensor* b, const float* out, int mode) {
    if (!b) return fail(RWQ_ERR_ARG, "weight is null");
    if (m < 0 || k <= 0) return fail(RWQ_ERR_ARG, "bad shape m=%lld k=%lld", (long long)m, (long long)k);
    if (k != b->w.k) return fail(RWQ_ERR_SHAPE, "matmul_t_q inner dims: %lld vs %d", (long long)k, b->w.k);
    if (k % rwq::QK) return fail(RWQ_ERR_ARG, "k must be a multiple of 32 (k=%lld)", (long long)k);
    if (m > (int64_t(1) << 31) / 2) return fail(RWQ_ERR_ARG, "m too large (%lld)", (long long)m);
    if (mode != RWQ_MODE_INT8 && mode != RWQ_MODE_F32) return fail(RWQ_ERR_ARG, "unknown mode %d", mode);
    if (m > 0 && (!a || (!out && b->w.n > 0))) return fail(RWQ_ERR_ARG, "null activation or output pointer");
    return RWQ_OK;
}

int read_device_error(Workspace* ws, cudaStream_t s) {
    int code = 0;
    RWQ_CUDA(cudaMemcpyAsync(&code, ws->err, sizeof(int), cudaMemcpyDeviceToHost, s), "read error flag");
    RWQ_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    if (code) {
        cudaMemsetAsync(ws->err, 0, sizeof(int), s);
        return fail(RWQ_ERR_DEVICE, "GEMM kernel stopped: bounded wait expired (role %d)", code);
    }
    return RWQ_OK;
}

// Second half of a matmul: activations `v` prepared in `layout` against
// weight `b`.  FOLD runs k_gemm_fold, or k_gemm_tc when block dots are
// dumped or path 3 is forced.
int run_quantized(const rwq::ActsView& v, int layout, rwq_qtensor* b, const float* bias, float* out, cudaStream_t s,
                  int32_t* S_dump, int* err_flag) {
    const rwq::Weight& w = b->w;
    const int64_t k = v.k;
    if (layout == rwq::LAYOUT_GEMV) {
        if (k > 8192) return fail(RWQ_ERR_ARG, "k=%lld too large for the GEMV kernels (max 8192)", (long long)k);
        RWQ_CUDA(rwq::launch_gemv_i8(v, w, bias, out, s, err_flag), "gemv launch");
        return RWQ_OK;
    }
    int rc;
    char why[256] = {0};
    if (layout == rwq::LAYOUT_HL) {
        if ((rc = weight_fold_cache(b, s))) return rc;
        cudaError_t e = rwq::launch_gemm_hl(v.ahl, v.rowscale, v.m, w.bhl, w.colscale, w.n, w.nb, bias, out, err_flag,
                                            s, why, sizeof why);
        if (e != cudaSuccess) return fail(RWQ_ERR_CUDA, "gemm launch: %s %s", cudaGetErrorString(e), why);
        return RWQ_OK;
    }
    if (!S_dump && t_gemm_path != 3) {
        if ((rc = weight_fold_cache(b, s))) return rc;
        cudaError_t e = rwq::launch_gemm_fold(v, w, bias, out, err_flag, s, why, sizeof why);
        if (e != cudaSuccess) return fail(RWQ_ERR_CUDA, "gemm launch: %s %s", cudaGetErrorString(e), why);
        return RWQ_OK;
    }
    if ((rc = weight_gemm_cache(b, s))) return rc;
    cudaError_t e = rwq::launch_gemm_tc(v, w, bias, out, S_dump, err_flag, s, why, sizeof why);
    if (e != cudaSuccess) return fail(RWQ_ERR_CUDA, "gemm launch: %s %s", cudaGetErrorString(e), why);
    return RWQ_OK;
}

// The kernel path of an m-row matmul: forced, this thread's setting, or
// automatic: the GEMV family up to 256 rows; above, the folded-scale GEMM
// for the int8 tier (faster than the hi|lo GEMM on the encoder's shapes:
// both move the same operand bytes per flop, and the hi|lo kernel's K
// splits cost more than they save at M = 1500) and the hi|lo GEMM for the
// f32 tier.
int pick_path(int64_t m, int force_path, int mode = RWQ_MODE_INT8) {
    int path = force_path ? force_path : t_gemm_path;
    if (path == 0) path = (m <= rwq::GEMV_FAMILY_MAX_M) ? 1 : (mode == RWQ_MODE_F32 ? 4 : 2);
    return path;
}

// The core device-pointer matmul.  `S_dump` (tests) routes through the
// exact GEMM and makes it write the per-block integer dots.
int matmul_dev_impl(const float* a, int64_t m, int64_t k, rwq_qtensor* b, const float* bias, float* out, int mode,
                    cudaStream_t s, int32_t* S_dump, int force_path) {
    int rc = check_matmul_args(a, m, k, b, out, mode);
    if (rc) return rc;
    if (m == 0 || b->w.n == 0) return RWQ_OK;
    const rwq::Weight& w = b->w;
    int path = pick_path(m, force_path, mode);
    if (mode == RWQ_MODE_F32) {
        // The f32 tier has two kernels: the CUDA-core GEMV (rows in chunks
        // of 8) and, from 257 rows (or path 4 forced), the hi|lo GEMM.
        if (path != 4) {
            if (reinterpret_cast<uintptr_t>(a) & 15)
                return fail(RWQ_ERR_ARG, "f32 mode needs 16-byte aligned device activations");
            for (int64_t m0 = 0; m0 < m; m0 += rwq::GEMV_MAX_M) {
                const int mc = int(m - m0 < rwq::GEMV_MAX_M ? m - m0 : rwq::GEMV_MAX_M);
                RWQ_CUDA(rwq::launch_gemv_f32(a + m0 * k, mc, w, bias, out + m0 * w.n, s), "gemv_f32 launch");
            }
            return RWQ_OK;
        }
    }
    if (S_dump) path = 3;
    const int layout = layout_of_path(path);
    if (layout == rwq::LAYOUT_FOLD && (k * 2) % 16)
        return fail(RWQ_ERR_ARG, "k*2 bytes must be a multiple of 16 for the GEMM");
    Workspace* ws = nullptr;
    if ((rc = get_workspace(s, &ws))) return rc;
    std::lock_guard<std::mutex> g(ws->mu);
    rwq::ActsView v;
    const size_t need = acts_layout(int(m), int(k), layout, &v, nullptr);
    if ((rc = ensure_cap(ws, need))) return rc;
    acts_layout(int(m), int(k), layout, &v, static_cast<uint8_t*>(ws->buf));
    RWQ_CUDA(prepare_acts(a, v, layout, mode == RWQ_MODE_INT8, s), "activation operand launch");
    return run_quantized(v, layout, b, bias, out, s, S_dump, ws->err);
}

cudaStream_t thread_stream() {
    // One non-blocking stream per (host thread, device) for the
    // host-buffer entry points.
    thread_local std::map<int, cudaStream_t> streams;
    int dev = 0;
    cudaGetDevice(&dev);
    auto it = streams.find(dev);
    if (it != streams.end()) return it->second;
    cudaStream_t s = nullptr;
    cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    streams[dev] = s;
    return s;
}


// Copy streams of the chunked host-buffer matmul, per (host thread, device).
struct CopyPipe {
    cudaStream_t up = nullptr, down = nullptr;
    cudaEvent_t ev_up[6] = {}, ev_mm[6] = {}, ev_in = nullptr, ev_out = nullptr;
};

int copy_pipe(CopyPipe** out) {
    thread_local std::map<int, CopyPipe> pipes;
    int dev = 0;
    cudaGetDevice(&dev);
    auto it = pipes.find(dev);
    if (it != pipes.end()) {
        *out = &it->second;
        return RWQ_OK;
    }
    CopyPipe p;
    RWQ_CUDA(cudaStreamCreateWithFlags(&p.up, cudaStreamNonBlocking), "cudaStreamCreate");
    RWQ_CUDA(cudaStreamCreateWithFlags(&p.down, cudaStreamNonBlocking), "cudaStreamCreate");
    for (int i = 0; i < 6; ++i) {
        RWQ_CUDA(cudaEventCreateWithFlags(&p.ev_up[i], cudaEventDisableTiming), "cudaEventCreate");
        RWQ_CUDA(cudaEventCreateWithFlags(&p.ev_mm[i], cudaEventDisableTiming), "cudaEventCreate");
    }
    RWQ_CUDA(cudaEventCreateWithFlags(&p.ev_in, cudaEventDisableTiming), "cudaEventCreate");
    RWQ_CUDA(cudaEventCreateWithFlags(&p.ev_out, cudaEventDisableTiming), "cudaEventCreate");
    *out = &(pipes[dev] = p);
    return RWQ_OK;
}

}  // namespace

int rwq::gemm_quantized(const ActsView& v, rwq_qtensor* w, const float* bias, float* out, cudaStream_t s) {
    Workspace* ws = nullptr;
    int rc = get_workspace(s, &ws);
    if (rc) return rc;
    if (v.k != w->w.k) return fail(RWQ_ERR_SHAPE, "gemm inner dims: %d vs %d", v.k, w->w.k);
    return run_quantized(v, v.ahl ? LAYOUT_HL : LAYOUT_FOLD, w, bias, out, s, nullptr, ws->err);
}

bool rwq::gemm_gelu_quantized_fits(const ActsView& v, rwq_qtensor* w, const ActsView& out) {
    return w && t_gemm_path != 3 && !v.ahl && v.k == w->w.k && rwq::gemm_fold_gelu_fits(v, w->w, out);
}

int rwq::gemm_gelu_quantized(const ActsView& v, rwq_qtensor* w, const float* bias, const ActsView& out,
                             cudaStream_t s) {
    if (!gemm_gelu_quantized_fits(v, w, out)) return fail(RWQ_ERR_ARG, "fused GELU GEMM does not apply here");
    Workspace* ws = nullptr;
    int rc = get_workspace(s, &ws);
    if (rc) return rc;
    if ((rc = weight_fold_cache(w, s))) return rc;
    char why[256] = {0};
    cudaError_t e = rwq::launch_gemm_fold_gelu(v, w->w, bias, out, ws->err, s, why, sizeof why);
    if (e != cudaSuccess) return fail(RWQ_ERR_CUDA, "gemm launch: %s %s", cudaGetErrorString(e), why);
    return RWQ_OK;
}

bool rwq::gemm_heads_fits(const ActsView& v, rwq_qtensor* w, int n_win, int T, int H, const __half* dst) {
    return w && t_gemm_path != 3 && !v.ahl && v.k == w->w.k && rwq::gemm_fold_heads_fits(v, w->w, n_win, T, H, dst);
}

int rwq::gemm_heads(const ActsView& v, rwq_qtensor* w, const float* bias, __half* dst, int n_win, int T, int H,
                    float scale, cudaStream_t s) {
    if (!gemm_heads_fits(v, w, n_win, T, H, dst)) return fail(RWQ_ERR_ARG, "fused heads GEMM does not apply here");
    Workspace* ws = nullptr;
    int rc = get_workspace(s, &ws);
    if (rc) return rc;
    if ((rc = weight_fold_cache(w, s))) return rc;
    char why[256] = {0};
    cudaError_t e = rwq::launch_gemm_fold_heads(v, w->w, bias, dst, n_win, T, H, scale, ws->err, s, why, sizeof why);
    if (e != cudaSuccess) return fail(RWQ_ERR_CUDA, "gemm launch: %s %s", cudaGetErrorString(e), why);
    return RWQ_OK;
}

int rwq::linear_acts(const ActsView& v, bool gemm, rwq_qtensor* w, const float* bias, float* out, cudaStream_t s) {
    Workspace* ws = nullptr;
    int rc = get_workspace(s, &ws);
    if (rc) return rc;
    if (v.k != w->w.k) return fail(RWQ_ERR_SHAPE, "linear inner dims: %d vs %d", v.k, w->w.k);
    return run_quantized(v, !gemm ? LAYOUT_GEMV : v.ahl ? LAYOUT_HL : LAYOUT_FOLD, w, bias, out, s, nullptr, ws->err);
}

int rwq::gemm_path() { return pick_path(GEMV_FAMILY_MAX_M + 1, 0); }

int rwq::gemm_hl(const uint16_t* ahl, const float* rowscale, int m, const uint16_t* bhl, const float* colscale, int n,
                 int nb, const float* bias, float* out, cudaStream_t s, const HlEpilogue* epi) {
    Workspace* ws = nullptr;
    int rc = get_workspace(s, &ws);
    if (rc) return rc;
    char why[256] = {0};
    cudaError_t e = launch_gemm_hl(ahl, rowscale, m, bhl, colscale, n, nb, bias, out, ws->err, s, why, sizeof why, epi);
    if (e != cudaSuccess) return fail(RWQ_ERR_CUDA, "gemm launch: %s %s", cudaGetErrorString(e), why);
    return RWQ_OK;
}

int rwq::with_stream_scratch(cudaStream_t s, size_t bytes, const std::function<int(void*)>& fn) {
    Workspace* ws = nullptr;
    int rc = get_workspace(s, &ws);
    if (rc) return rc;
    std::lock_guard<std::mutex> g(ws->mu);
    if ((rc = ensure_cap(ws, bytes))) return rc;
    return fn(ws->buf);
}

namespace rwq {
// A weight whose rows are those of `parts` one after another (same dtype
// and k, same device): each plane is row-major, so the planes are copied
// end to end.  Used by the decoder to run the Q, K and V projections of a
// layer as one GEMV.
int qtensor_concat_rows(rwq_qtensor* const* parts, int np, cudaStream_t s, rwq_qtensor** out) {
    *out = nullptr;
    if (np <= 0) return fail(RWQ_ERR_ARG, "no parts");
    const Weight& w0 = parts[0]->w;
    int64_t n = 0;
    for (int i = 0; i < np; ++i) {
        const Weight& wi = parts[i]->w;
        if (wi.dtype != w0.dtype || wi.k != w0.k || wi.device != w0.device)
            return fail(RWQ_ERR_ARG, "parts differ in dtype, k or device");
        n += wi.n;
    }
    if (n > INT32_MAX) return fail(RWQ_ERR_ARG, "weight too large");
    auto* t = new rwq_qtensor;
    Weight& w = t->w;
    w.dtype = w0.dtype;
    w.n = int(n);
    w.k = w0.k;
    w.nb = w0.nb;
    w.device = w0.device;
    const size_t nb4 = size_t(round4(w.nb)), rows = size_t(n) * nb4;
    cudaError_t e;
    auto cleanup = [&](int rc) {
        rwq_qtensor_free(t);
        return rc;
    };
    if ((e = cudaMalloc(&w.qs, rows * qs_bytes(w.dtype))) != cudaSuccess) return cleanup(cuda_fail(e, "cudaMalloc(qs)"));
    if ((e = cudaMalloc(&w.d, rows * 2)) != cudaSuccess) return cleanup(cuda_fail(e, "cudaMalloc(d)"));
    if (has_min(w.dtype) && (e = cudaMalloc(&w.m, rows * 2)) != cudaSuccess) return cleanup(cuda_fail(e, "cudaMalloc(m)"));
    if (has_qh(w.dtype) && (e = cudaMalloc(&w.qh, rows * 4)) != cudaSuccess) return cleanup(cuda_fail(e, "cudaMalloc(qh)"));
    size_t r0 = 0;
    for (int i = 0; i < np; ++i) {
        const Weight& wi = parts[i]->w;
        const size_t ri = size_t(wi.n) * nb4;
        e = cudaMemcpyAsync(w.qs + r0 * qs_bytes(w.dtype), wi.qs, ri * qs_bytes(w.dtype), cudaMemcpyDeviceToDevice, s);
        if (e == cudaSuccess) e = cudaMemcpyAsync(w.d + r0, wi.d, ri * 2, cudaMemcpyDeviceToDevice, s);
        if (e == cudaSuccess && w.m) e = cudaMemcpyAsync(w.m + r0, wi.m, ri * 2, cudaMemcpyDeviceToDevice, s);
        if (e == cudaSuccess && w.qh) e = cudaMemcpyAsync(w.qh + r0, wi.qh, ri * 4, cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) return cleanup(cuda_fail(e, "copy weight planes"));
        r0 += ri;
    }
    prepare_gemv_rows(w);
    *out = t;
    return RWQ_OK;
}
}  // namespace rwq

extern "C" {

int rwq_block_bytes(int dtype) {
    const int bb = rwq::block_bytes(dtype);
    return bb > 0 ? bb : fail(RWQ_ERR_DTYPE, "unsupported quantized dtype %d", dtype);
}

const char* rwq_last_error(void) { return t_err.c_str(); }

int rwq_init(int device) {
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) return fail(RWQ_ERR_NOGPU, "no CUDA device");
    if (device < 0 || device >= count) return fail(RWQ_ERR_ARG, "device %d out of range (%d devices)", device, count);
    RWQ_CUDA(cudaSetDevice(device), "cudaSetDevice");
    cudaDeviceProp p;
    RWQ_CUDA(cudaGetDeviceProperties(&p, device), "cudaGetDeviceProperties");
    if (p.major != 10) return fail(RWQ_ERR_NOGPU, "device %d is sm_%d%d, this build targets sm_100a", device, p.major, p.minor);
    return RWQ_OK;
}

static int qtensor_new_impl(const void* raw, bool raw_on_device, size_t raw_len, int dtype, int64_t n, int64_t k,
                            cudaStream_t s, rwq_qtensor** out) {
    if (!out) return fail(RWQ_ERR_ARG, "out is null");
    *out = nullptr;
    if (!valid_dtype(dtype)) return fail(RWQ_ERR_DTYPE, "unsupported quantized dtype %d", dtype);
    if (n < 0 || k <= 0 || k % rwq::QK) return fail(RWQ_ERR_ARG, "bad weight shape [%lld, %lld] (k %% 32 must be 0)",
                                                   (long long)n, (long long)k);
    if (n > INT32_MAX || k > INT32_MAX) return fail(RWQ_ERR_ARG, "weight too large");
    const size_t nb = size_t(k) / rwq::QK, nblk = size_t(n) * nb;
    const size_t want = nblk * size_t(rwq::block_bytes(dtype));
    if (raw_len != want) return fail(RWQ_ERR_ARG, "raw length %zu != %zu for [%lld, %lld] dtype %d", raw_len, want,
                                     (long long)n, (long long)k, dtype);
    if (nblk && !raw) return fail(RWQ_ERR_ARG, "raw is null");
    auto* t = new rwq_qtensor;
    rwq::Weight& w = t->w;
    w.dtype = dtype;
    w.n = int(n);
    w.k = int(k);
    w.nb = int(nb);
    cudaGetDevice(&w.device);
    auto cleanup = [&](int rc) {
        rwq_qtensor_free(t);
        return rc;
    };
    cudaError_t e;
    // Planes hold nb4 = round4(nb) blocks per row; pad blocks stay zero.
    const size_t nalloc = nblk ? size_t(n) * size_t(rwq::round4(int(nb))) : 1;
    if ((e = cudaMalloc(&w.qs, nalloc * rwq::qs_bytes(dtype))) != cudaSuccess) return cleanup(cuda_fail(e, "cudaMalloc(qs)"));
    if ((e = cudaMalloc(&w.d, nalloc * 2)) != cudaSuccess) return cleanup(cuda_fail(e, "cudaMalloc(d)"));
    if (rwq::has_min(dtype) && (e = cudaMalloc(&w.m, nalloc * 2)) != cudaSuccess)
        return cleanup(cuda_fail(e, "cudaMalloc(m)"));
    if (rwq::has_qh(dtype) && (e = cudaMalloc(&w.qh, nalloc * 4)) != cudaSuccess)
        return cleanup(cuda_fail(e, "cudaMalloc(qh)"));
    if (nblk && nalloc != nblk) {
        cudaMemsetAsync(w.qs, 0, nalloc * rwq::qs_bytes(dtype), s);
        cudaMemsetAsync(w.d, 0, nalloc * 2, s);
        if (w.m) cudaMemsetAsync(w.m, 0, nalloc * 2, s);
        if (w.qh) cudaMemsetAsync(w.qh, 0, nalloc * 4, s);
    }
    if (nblk) {
        const uint8_t* src = static_cast<const uint8_t*>(raw);
        uint8_t* tmp = nullptr;
        if (!raw_on_device) {
            if ((e = cudaMalloc(&tmp, raw_len)) != cudaSuccess) return cleanup(cuda_fail(e, "cudaMalloc(raw)"));
            if ((e = cudaMemcpyAsync(tmp, raw, raw_len, cudaMemcpyHostToDevice, s)) != cudaSuccess) {
                cudaFree(tmp);
                return cleanup(cuda_fail(e, "copy raw blocks"));
            }
            src = tmp;
        }
        e = rwq::launch_repack(src, w, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (tmp) cudaFree(tmp);
        if (e != cudaSuccess) return cleanup(cuda_fail(e, "repack"));
    }
    rwq::prepare_gemv_rows(w);
    *out = t;
    return RWQ_OK;
}

int rwq_qtensor_new(const uint8_t* raw, size_t raw_len, int dtype, int64_t n, int64_t k, rwq_qtensor** out) {
    return qtensor_new_impl(raw, false, raw_len, dtype, n, k, thread_stream(), out);
}

int rwq_qtensor_new_device(const void* raw_dev, size_t raw_len, int dtype, int64_t n, int64_t k, void* stream,
                           rwq_qtensor** out) {
    return qtensor_new_impl(raw_dev, true, raw_len, dtype, n, k, static_cast<cudaStream_t>(stream), out);
}

int rwq_qtensor_free(rwq_qtensor* t) {
    if (!t) return RWQ_OK;
    rwq::Weight& w = t->w;
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != w.device) cudaSetDevice(w.device);
    cudaFree(w.qs);
    cudaFree(w.qh);
    cudaFree(w.d);
    cudaFree(w.m);
    cudaFree(w.q16);
    cudaFree(w.dT);
    cudaFree(w.mT);
    cudaFree(w.bhl);
    cudaFree(w.colscale);
    if (prev != w.device) cudaSetDevice(prev);
    delete t;
    return RWQ_OK;
}

int rwq_qtensor_shape(const rwq_qtensor* t, int* dtype, int64_t* n, int64_t* k) {
    if (!t) return fail(RWQ_ERR_ARG, "weight is null");
    if (dtype) *dtype = t->w.dtype;
    if (n) *n = t->w.n;
    if (k) *k = t->w.k;
    return RWQ_OK;
}

int rwq_qtensor_prepare_gemm(rwq_qtensor* t, void* stream) {
    if (!t) return fail(RWQ_ERR_ARG, "weight is null");
    return weight_gemm_cache(t, static_cast<cudaStream_t>(stream));
}

int rwq_matmul_t_q_dev(const float* a, int64_t m, int64_t k, const rwq_qtensor* b, const float* bias, float* out,
                       int mode, void* stream) {
    return matmul_dev_impl(a, m, k, const_cast<rwq_qtensor*>(b), bias, out, mode, static_cast<cudaStream_t>(stream),
                           nullptr, 0);
}

int rwq_matmul_t_q(const float* a, int64_t m, int64_t k, const rwq_qtensor* b, const float* bias, float* out,
                   int mode) {
    int rc = check_matmul_args(a, m, k, b, out, mode);
    if (rc) return rc;
    const int64_t n = b->w.n;
    if (m == 0 || n == 0) return RWQ_OK;
    cudaStream_t s = thread_stream();
    // Host-buffer compat path: device copies of A, bias and C live in a
    // second arena keyed on this thread's stream.
    Workspace* ws = nullptr;
    if ((rc = get_workspace(s, &ws, WS_HOST_COPY))) return rc;
    std::lock_guard<std::mutex> g(ws->mu);
    const size_t a_b = align_up(size_t(m) * k * 4, 256), o_b = align_up(size_t(m) * n * 4, 256),
                 b_b = align_up(size_t(n) * 4, 256);
    if ((rc = ensure_cap(ws, a_b + o_b + b_b))) return rc;
    float* da = static_cast<float*>(ws->buf);
    float* dout = reinterpret_cast<float*>(static_cast<uint8_t*>(ws->buf) + a_b);
    float* dbias = bias ? reinterpret_cast<float*>(static_cast<uint8_t*>(ws->buf) + a_b + o_b) : nullptr;
    if (bias) RWQ_CUDA(cudaMemcpyAsync(dbias, bias, size_t(n) * 4, cudaMemcpyHostToDevice, s), "copy bias");
    // GEMM-family calls (m > 256 and no forced path) run in row chunks of
    // more than 256 rows, so every chunk stays in the family and the results
    // are those of one call (each output row's sum does not depend on which
    // other rows share the GEMM as long as the kernel and its K split are
    // the same; both are picked from the tile count): the upload of chunk c+1, the matmul of chunk c
    // and the download of chunk c-1 overlap (PCIe is full duplex).  With
    // pageable host buffers the copies still work, without the overlap.
    const int chunks = (t_gemm_path == 0) ? int(std::min<int64_t>(6, m / 257)) : 1;
    if (chunks < 2) {
        RWQ_CUDA(cudaMemcpyAsync(da, a, size_t(m) * k * 4, cudaMemcpyHostToDevice, s), "copy A to device");
        if ((rc = matmul_dev_impl(da, m, k, const_cast<rwq_qtensor*>(b), dbias, dout, mode, s, nullptr, 0)))
            return rc;
        RWQ_CUDA(cudaMemcpyAsync(out, dout, size_t(m) * n * 4, cudaMemcpyDeviceToHost, s), "copy C to host");
    } else {
        CopyPipe* cp = nullptr;
        if ((rc = copy_pipe(&cp))) return rc;
        // Every chunk runs with the kernel and K split of the whole call,
        // so the chunks give the bits of one device call.
        struct KsplitGuard {
            KsplitGuard(int S, int fold) {
                rwq::set_gemm_hl_ksplit(S);
                rwq::set_gemm_fold_config(fold);
            }
            ~KsplitGuard() {
                rwq::set_gemm_hl_ksplit(0);
                rwq::set_gemm_fold_config(0);
            }
        } ks_guard(rwq::gemm_hl_ksplit(int(m), int(n), int(k / rwq::QK)),
                   rwq::gemm_fold_config(int(m), int(n), int(k / rwq::QK)));
        RWQ_CUDA(cudaEventRecord(cp->ev_in, s), "event");
        RWQ_CUDA(cudaStreamWaitEvent(cp->up, cp->ev_in, 0), "event wait");
        RWQ_CUDA(cudaStreamWaitEvent(cp->down, cp->ev_in, 0), "event wait");
        for (int c = 0; c < chunks && !rc; ++c) {
            const int64_t r0 = c * m / chunks, rows = (c + 1) * m / chunks - r0;   // > 256 each
            RWQ_CUDA(cudaMemcpyAsync(da + r0 * k, a + r0 * k, size_t(rows) * k * 4, cudaMemcpyHostToDevice, cp->up),
                     "copy A to device");
            RWQ_CUDA(cudaEventRecord(cp->ev_up[c], cp->up), "event");
            RWQ_CUDA(cudaStreamWaitEvent(s, cp->ev_up[c], 0), "event wait");
            rc = matmul_dev_impl(da + r0 * k, rows, k, const_cast<rwq_qtensor*>(b), dbias, dout + r0 * n, mode, s,
                                 nullptr, 0);
            if (rc) break;
            RWQ_CUDA(cudaEventRecord(cp->ev_mm[c], s), "event");
            RWQ_CUDA(cudaStreamWaitEvent(cp->down, cp->ev_mm[c], 0), "event wait");
            RWQ_CUDA(cudaMemcpyAsync(out + r0 * n, dout + r0 * n, size_t(rows) * n * 4, cudaMemcpyDeviceToHost,
                                     cp->down),
                     "copy C to host");
        }
        // The caller's buffers and this workspace are free again only when
        // both copy streams are done.
        cudaEventRecord(cp->ev_out, cp->down);
        cudaStreamWaitEvent(s, cp->ev_out, 0);
        cudaEventRecord(cp->ev_in, cp->up);
        cudaStreamWaitEvent(s, cp->ev_in, 0);
        if (rc) {
            cudaStreamSynchronize(s);
            return rc;
        }
    }
    Workspace* mws = nullptr;
    if ((rc = get_workspace(s, &mws))) return rc;
    return read_device_error(mws, s);
}

int rwq_dequant_rows_dev(const rwq_qtensor* t, const int32_t* rows, int64_t nrows, float* out, void* stream) {
    if (!t) return fail(RWQ_ERR_ARG, "weight is null");
    if (nrows < 0 || (nrows > 0 && !out)) return fail(RWQ_ERR_ARG, "bad output");
    if (!rows && nrows > t->w.n) return fail(RWQ_ERR_ARG, "nrows %lld > n %d", (long long)nrows, t->w.n);
    if (reinterpret_cast<uintptr_t>(out) & 15) return fail(RWQ_ERR_ARG, "dequant output must be 16-byte aligned");
    RWQ_CUDA(rwq::launch_dequant_rows(t->w, rows, int(nrows), out, static_cast<cudaStream_t>(stream)), "dequant launch");
    return RWQ_OK;
}

int rwq_row_f32(const rwq_qtensor* t, int64_t row, float* out) {
    if (!t) return fail(RWQ_ERR_ARG, "weight is null");
    if (row < 0 || row >= t->w.n) return fail(RWQ_ERR_ARG, "row %lld out of range [0, %d)", (long long)row, t->w.n);
    if (!out) return fail(RWQ_ERR_ARG, "out is null");
    cudaStream_t s = thread_stream();
    Workspace* ws = nullptr;
    int rc;
    if ((rc = get_workspace(s, &ws, WS_HOST_COPY))) return rc;
    std::lock_guard<std::mutex> g(ws->mu);
    if ((rc = ensure_cap(ws, size_t(t->w.k) * 4 + 256))) return rc;
    int32_t* drow = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(ws->buf) + size_t(t->w.k) * 4);
    const int32_t r32 = int32_t(row);
    RWQ_CUDA(cudaMemcpyAsync(drow, &r32, 4, cudaMemcpyHostToDevice, s), "copy row index");
    RWQ_CUDA(rwq::launch_dequant_rows(t->w, drow, 1, static_cast<float*>(ws->buf), s), "dequant launch");
    RWQ_CUDA(cudaMemcpyAsync(out, ws->buf, size_t(t->w.k) * 4, cudaMemcpyDeviceToHost, s), "copy row");
    RWQ_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    return RWQ_OK;
}

int rwq_quantize_acts_dev(const float* a, int64_t m, int64_t k, int8_t* q, float* d, int32_t* sum, void* stream) {
    if (m < 0 || k <= 0 || k % rwq::QK) return fail(RWQ_ERR_ARG, "bad shape (k %% 32 must be 0)");
    if (m == 0) return RWQ_OK;
    if (!a || !q || !d || !sum) return fail(RWQ_ERR_ARG, "null pointer");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    Workspace* ws = nullptr;
    int rc;
    if ((rc = get_workspace(s, &ws))) return rc;
    std::lock_guard<std::mutex> g(ws->mu);
    const size_t ub = align_up(size_t(m) * (k / 32) * 4, 256);
    if ((rc = ensure_cap(ws, ub))) return rc;
    rwq::ActsView v;
    v.m = int(m);
    v.k = int(k);
    v.nb = int(k / 32);
    v.m_pad = v.m;
    v.q8 = q;
    v.d = d;
    v.sum = sum;
    v.u = static_cast<float*>(ws->buf);
    RWQ_CUDA(rwq::launch_quantize_acts(a, v, false, s), "quantize launch");
    return RWQ_OK;
}

int rwq_block_dots_dev(const float* a, int64_t m, int64_t k, const rwq_qtensor* b, int32_t* S, int path,
                       void* stream) {
    int rc = check_matmul_args(a, m, k, b, S ? reinterpret_cast<float*>(S) : nullptr, RWQ_MODE_INT8);
    if (rc) return rc;
    if (m == 0 || b->w.n == 0) return RWQ_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (path == 1) {
        // The GEMM writes S while computing C; C goes to scratch.
        Workspace* ws = nullptr;
        if ((rc = get_workspace(s, &ws, WS_DOT_DUMP))) return rc;
        std::lock_guard<std::mutex> g(ws->mu);
        if ((rc = ensure_cap(ws, size_t(m) * b->w.n * 4 + 256))) return rc;
        return matmul_dev_impl(a, m, k, const_cast<rwq_qtensor*>(b), nullptr, static_cast<float*>(ws->buf),
                               RWQ_MODE_INT8, s, S, 2);
    }
    if (path != 0) return fail(RWQ_ERR_ARG, "unknown block-dot path %d", path);
    Workspace* ws = nullptr;
    if ((rc = get_workspace(s, &ws))) return rc;
    std::lock_guard<std::mutex> g(ws->mu);
    rwq::ActsView v;
    const size_t need = acts_layout(int(m), int(k), rwq::LAYOUT_GEMV, &v, nullptr);
    if ((rc = ensure_cap(ws, need))) return rc;
    acts_layout(int(m), int(k), rwq::LAYOUT_GEMV, &v, static_cast<uint8_t*>(ws->buf));
    RWQ_CUDA(rwq::launch_quantize_acts(a, v, false, s), "quantize launch");
    RWQ_CUDA(rwq::launch_block_dots(v, b->w, S, s), "block dots launch");
    return RWQ_OK;
}

int rwq_set_gemm_path(int path) {
    if (path < 0 || path > 4) return fail(RWQ_ERR_ARG, "path must be 0, 1, 2, 3 or 4");
    t_gemm_path = path;
    return RWQ_OK;
}

int rwq_set_gemv_kernel(int kind) {
    if (kind < 0 || kind > 4) return fail(RWQ_ERR_ARG, "kind must be 0, 1, 2, 3 or 4");
    rwq::set_gemv_kind(kind);
    return RWQ_OK;
}

int rwq_gemv_kernel_for(const rwq_qtensor* w, int64_t m) {
    if (!w) return fail(RWQ_ERR_ARG, "weight is null");
    if (m < 1 || m > rwq::GEMV_FAMILY_MAX_M) return fail(RWQ_ERR_ARG, "m=%lld outside [1, 256]", (long long)m);
    return rwq::gemv_kernel_for(w->w, int(m));
}

int rwq_stream_check(void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    RWQ_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    RWQ_CUDA(cudaGetLastError(), "pending CUDA error");
    Workspace* ws = nullptr;
    int rc;
    if ((rc = get_workspace(s, &ws))) return rc;
    return read_device_error(ws, s);
}

int rwq_qacts_new(int64_t max_m, int64_t k, rwq_qacts** out) {
    if (!out) return fail(RWQ_ERR_ARG, "out is null");
    *out = nullptr;
    if (max_m < 0 || max_m > (int64_t(1) << 30) || k <= 0 || k % rwq::QK || k > INT32_MAX)
        return fail(RWQ_ERR_ARG, "bad qacts shape [%lld, %lld] (k %% 32 must be 0)", (long long)max_m, (long long)k);
    auto* q = new rwq_qacts;
    cudaGetDevice(&q->device);
    q->max_m = int(max_m);
    q->k = int(k);
    const size_t bytes = acts_bytes_max(q->max_m, q->k);
    cudaError_t e = cudaMalloc(&q->buf, bytes ? bytes : 256);
    if (e != cudaSuccess) {
        delete q;
        return cuda_fail(e, "cudaMalloc(qacts)");
    }
    q->v.m = 0;
    *out = q;
    return RWQ_OK;
}

int rwq_qacts_free(rwq_qacts* q) {
    if (!q) return RWQ_OK;
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != q->device) cudaSetDevice(q->device);
    cudaFree(q->buf);
    if (prev != q->device) cudaSetDevice(prev);
    delete q;
    return RWQ_OK;
}

int rwq_qacts_quantize(rwq_qacts* q, const float* a, int64_t m, void* stream) {
    if (!q) return fail(RWQ_ERR_ARG, "qacts is null");
    if (m < 0 || m > q->max_m) return fail(RWQ_ERR_ARG, "m=%lld outside [0, %d]", (long long)m, q->max_m);
    if (m > 0 && !a) return fail(RWQ_ERR_ARG, "activations are null");
    q->layout = layout_of_path(pick_path(m, 0));
    // Carve for the current m (row strides depend on m); the arena was
    // sized for max_m in the largest layout.
    acts_layout(int(m), q->k, q->layout, &q->v, static_cast<uint8_t*>(q->buf));
    if (m == 0) return RWQ_OK;
    RWQ_CUDA(prepare_acts(a, q->v, q->layout, true, static_cast<cudaStream_t>(stream)), "quantize launch");
    return RWQ_OK;
}

int rwq_matmul_t_q_qacts(const rwq_qacts* q, const rwq_qtensor* b, const float* bias, float* out, void* stream) {
    if (!q || !b) return fail(RWQ_ERR_ARG, "null qacts or weight");
    if (q->k != b->w.k) return fail(RWQ_ERR_SHAPE, "matmul_t_q inner dims: %d vs %d", q->k, b->w.k);
    if (q->v.m == 0 || b->w.n == 0) return RWQ_OK;
    if (!out) return fail(RWQ_ERR_ARG, "out is null");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    Workspace* ws = nullptr;
    int rc;
    if ((rc = get_workspace(s, &ws))) return rc;
    return run_quantized(q->v, q->layout, const_cast<rwq_qtensor*>(b), bias, out, s, nullptr, ws->err);
}

}  // extern "C"
