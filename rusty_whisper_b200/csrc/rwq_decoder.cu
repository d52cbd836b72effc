// rwq_decoder.cu -- the device-resident KV-cached decoder behind the C ABI
// (rwq_decoder_* in include/rwq.h): the reference's Decoder
// (decoder.rs:36-321) for S decode streams in lockstep.  A stream decodes
// one window; several streams may share a window (beams), and then share
// its cross-attention K/V (the reference shares them through an Arc,
// decoder.rs:18-24, 71-79).
//
//   begin   cross K (no bias) and V of every layer from the windows'
//           encoder outputs: one quantization, two GEMMs per layer, f16
//           heads [win][H][n_audio][64] kept in HBM for the whole decode;
//   step    token + position -> per layer {[residual +] LN + quantize ->
//           Q, K, V linears -> KV-cache append -> self-attention ->
//           quantize -> out linear -> residual + LN + quantize -> cross Q
//           -> cross-attention (per window: K/V read once for all its
//           streams) -> quantize -> cross out -> residual + LN + quantize
//           -> fc1 -> GELU + quantize -> fc2} -> residual + final LN +
//           quantize -> tied logits -> greedy argmax.
// Linears take the integer-MMA GEMV (weights streamed from HBM once per
// step for up to 64 streams per launch) for up to 256 streams and the
// tensor-core GEMM above that; everything stays on the device between steps.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>
#include "../../include/rwq.h"
#include "rwq_common.cuh"
#include "rwq_decoder.h"
#include "rwq_encoder.h"
#include "rwq_internal.h"

namespace {

int dfail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    rwq::set_last_error(buf);
    return code;
}

#define DEC_CUDA(call, what)                                                                               \
    do {                                                                                                   \
        cudaError_t e_ = (call);                                                                           \
        if (e_ != cudaSuccess)                                                                             \
            return dfail(e_ == cudaErrorMemoryAllocation ? RWQ_ERR_NOMEM : RWQ_ERR_CUDA, "%s: %s", what,   \
                         cudaGetErrorString(e_));                                                          \
    } while (0)

#define DEC_RC(call)             \
    do {                         \
        int rc_ = (call);        \
        if (rc_) return rc_;     \
    } while (0)

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct DLayer {
    rwq_qtensor *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr;
    rwq_qtensor *xq = nullptr, *xk = nullptr, *xv = nullptr, *xo = nullptr;
    rwq_qtensor *fc1 = nullptr, *fc2 = nullptr;
    // Q, K, V as one weight [3D][D] (built at begin) and its bias
    // [q_b, 0, v_b]: one GEMV per layer instead of three.
    rwq_qtensor* qkv = nullptr;
    float* qkv_b = nullptr;
    // device pointers of the dense tensors, resolved once per begin
    const float *attn_ln_w = nullptr, *attn_ln_b = nullptr, *q_b = nullptr, *v_b = nullptr, *o_b = nullptr;
    const float *x_ln_w = nullptr, *x_ln_b = nullptr, *xq_b = nullptr, *xo_b = nullptr;
    const float *mlp_ln_w = nullptr, *mlp_ln_b = nullptr, *fc1_b = nullptr, *fc2_b = nullptr;
};

const char* const kDenseLayer[] = {"attn_ln.weight", "attn_ln.bias", "attn.query.bias", "attn.value.bias",
                                   "attn.out.bias", "cross_attn_ln.weight", "cross_attn_ln.bias",
                                   "cross_attn.query.bias", "cross_attn.value.bias", "cross_attn.out.bias",
                                   "mlp_ln.weight", "mlp_ln.bias", "mlp.2.bias"};

}  // namespace

struct rwq_decoder {
    int device = 0;
    int n_vocab = 0, n_ctx = 0, n_state = 0, n_head = 0, n_layer = 0, n_ff = 0;
    std::map<std::string, float*> dense;
    std::map<std::string, size_t> dense_len;
    std::vector<DLayer> layers;
    rwq_qtensor* emb = nullptr;
    // decode state (begin)
    int n_streams = 0, n_windows = 0, n_audio = 0, n_past = 0, n_cross_groups = 0, max_group = 1;
    void* state = nullptr;        // caches, group tables and step buffers
    size_t state_bytes = 0;
    __half *cross_k = nullptr, *cross_v = nullptr, *self_k = nullptr, *self_v = nullptr;
    int *cross_kv = nullptr, *cross_off = nullptr, *cross_streams = nullptr;
    int *self_kv = nullptr, *self_off = nullptr;   // identity tables for self-attention
    int cross_splits = 1;          // key splits of the cross-attention (multi-stream groups)
    float* attn_part = nullptr;    // per-split partial results of the cross-attention
    unsigned* attn_cnt = nullptr;  // per (group, head) split counters, zero between launches
    float *x = nullptr, *tmp = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr, *h = nullptr,
          *logits = nullptr, *qkv = nullptr;
    float* hid = nullptr;          // final-layernormed states of the last hidden step [S][D]
    int32_t* win_dev = nullptr;    // stream -> window, on the device (fork checks)
    int32_t* best = nullptr;
    int* dpos = nullptr;           // the decode position, on the device
    int32_t* tok_in = nullptr;     // this step's tokens (graph input)
    rwq::ActsView gemv, gemm;
    // One captured step per (output mode, limit); a mode runs eagerly once
    // (first-use set-up happens there) before it is captured.
    std::map<std::pair<int, int>, cudaGraphExec_t> graphs;
    std::map<std::pair<int, int>, int> eager_runs;
    // Steps run on this decoder's own stream (graphs cannot be captured on
    // the legacy default stream), ordered after and before the caller's
    // stream by two events.
    cudaStream_t gs = nullptr;
    cudaEvent_t ev_in = nullptr, ev_out = nullptr;
    std::mutex mu;
};

namespace {

std::string lname(int l, const char* f) { return "decoder.blocks." + std::to_string(l) + "." + f; }

rwq_qtensor** quant_slot(rwq_decoder* d, const std::string& name, int64_t* wn, int64_t* wk) {
    const int64_t D = d->n_state, F = d->n_ff;
    *wn = D;
    *wk = D;
    if (name == "decoder.token_embedding.weight") {
        *wn = d->n_vocab;
        return &d->emb;
    }
    const std::string pre = "decoder.blocks.";
    if (name.compare(0, pre.size(), pre) != 0) return nullptr;
    const size_t dot = name.find('.', pre.size());
    if (dot == std::string::npos) return nullptr;
    const std::string idx = name.substr(pre.size(), dot - pre.size());
    if (idx.empty() || idx.find_first_not_of("0123456789") != std::string::npos) return nullptr;
    const int l = std::atoi(idx.c_str());
    if (l < 0 || l >= d->n_layer) return nullptr;
    DLayer& L = d->layers[size_t(l)];
    const std::string f = name.substr(dot + 1);
    if (f == "attn.query.weight") return &L.q;
    if (f == "attn.key.weight") return &L.k;
    if (f == "attn.value.weight") return &L.v;
    if (f == "attn.out.weight") return &L.o;
    if (f == "cross_attn.query.weight") return &L.xq;
    if (f == "cross_attn.key.weight") return &L.xk;
    if (f == "cross_attn.value.weight") return &L.xv;
    if (f == "cross_attn.out.weight") return &L.xo;
    if (f == "mlp.0.weight") { *wn = F; return &L.fc1; }
    if (f == "mlp.2.weight") { *wk = F; return &L.fc2; }
    return nullptr;
}

int check_ready(rwq_decoder* d) {
    for (auto& kv : d->dense_len)
        if (!d->dense.count(kv.first)) return dfail(RWQ_ERR_ARG, "decoder tensor '%s' was not set", kv.first.c_str());
    if (!d->emb) return dfail(RWQ_ERR_ARG, "decoder.token_embedding.weight was not set");
    for (int l = 0; l < d->n_layer; ++l) {
        const DLayer& L = d->layers[size_t(l)];
        for (rwq_qtensor* t : {L.q, L.k, L.v, L.o, L.xq, L.xk, L.xv, L.xo, L.fc1, L.fc2})
            if (!t) return dfail(RWQ_ERR_ARG, "decoder block %d: a linear weight was not set", l);
    }
    return RWQ_OK;
}

// Lay out (base == nullptr: size) the decode state for S streams, W windows.
size_t layout_state(rwq_decoder* d, int S, int W, int n_audio, int n_groups, int splits, uint8_t* base) {
    const size_t D = size_t(d->n_state), F = size_t(d->n_ff), H = size_t(d->n_head), L = size_t(d->n_layer);
    const size_t kmax = std::max(D, F), m_pad = align_up(size_t(S), 256);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        uint8_t* p = base ? base + off : nullptr;
        off = align_up(off + bytes, 256);
        return p;
    };
    d->cross_k = reinterpret_cast<__half*>(take(L * W * H * n_audio * 64 * 2));
    d->cross_v = reinterpret_cast<__half*>(take(L * W * H * n_audio * 64 * 2));
    d->self_k = reinterpret_cast<__half*>(take(L * S * H * d->n_ctx * 64 * 2));
    d->self_v = reinterpret_cast<__half*>(take(L * S * H * d->n_ctx * 64 * 2));
    d->cross_kv = reinterpret_cast<int*>(take(size_t(n_groups) * 4));
    d->cross_off = reinterpret_cast<int*>(take(size_t(n_groups + 1) * 4));
    d->cross_streams = reinterpret_cast<int*>(take(size_t(S) * 4));
    d->self_kv = reinterpret_cast<int*>(take(size_t(S) * 4));
    d->self_off = reinterpret_cast<int*>(take(size_t(S + 1) * 4));
    d->attn_part = splits > 1 ? reinterpret_cast<float*>(take(size_t(n_groups) * splits * H * rwq::DEC_MAX_G * 66 * 4))
                              : nullptr;
    d->attn_cnt = splits > 1 ? reinterpret_cast<unsigned*>(take(size_t(n_groups) * H * 4)) : nullptr;
    d->x = reinterpret_cast<float*>(take(S * D * 4));
    d->tmp = reinterpret_cast<float*>(take(S * D * 4));
    d->q = reinterpret_cast<float*>(take(S * D * 4));
    d->k = reinterpret_cast<float*>(take(S * D * 4));
    d->v = reinterpret_cast<float*>(take(S * D * 4));
    d->att = reinterpret_cast<float*>(take(S * D * 4));
    d->qkv = reinterpret_cast<float*>(take(S * 3 * D * 4));
    d->h = reinterpret_cast<float*>(take(S * F * 4));
    d->logits = reinterpret_cast<float*>(take(S * size_t(d->n_vocab) * 4));
    d->hid = reinterpret_cast<float*>(take(S * D * 4));
    d->win_dev = reinterpret_cast<int32_t*>(take(size_t(S) * 4));
    d->best = reinterpret_cast<int32_t*>(take(size_t(S) * 4));
    d->dpos = reinterpret_cast<int*>(take(4));
    d->tok_in = reinterpret_cast<int32_t*>(take(size_t(S) * 4));
    rwq::ActsView& g = d->gemv;
    g = rwq::ActsView();
    g.m = S;
    g.q8 = reinterpret_cast<int8_t*>(take(S * kmax));
    g.d = reinterpret_cast<float*>(take(S * (kmax / 32) * 4));
    g.sum = reinterpret_cast<int32_t*>(take(S * (kmax / 32) * 4));
    g.u = reinterpret_cast<float*>(take(S * (kmax / 32) * 4));
    rwq::ActsView& m = d->gemm;
    m = rwq::ActsView();
    m.m = S;
    m.m_pad = int(m_pad);
    m.q16 = reinterpret_cast<uint16_t*>(take(S * kmax * 2));
    m.dT = reinterpret_cast<float*>(take((kmax / 32) * m_pad * 4));
    m.uT = reinterpret_cast<float*>(take((kmax / 32) * m_pad * 4));
    return off;
}

rwq::ActsView with_k(rwq::ActsView v, int k) {
    v.k = k;
    v.nb = k / rwq::QK;
    return v;
}

// Row transform + quantize into the layout the linears of this step read
// (quantize false: only the transformed rows into yout).
int rows(rwq_decoder* d, int mode, const float* x, const float* add, float* xout, const float* w, const float* b, int k,
         cudaStream_t s, float* yout = nullptr, bool quantize = true) {
    const int S = d->n_streams;
    const bool gemm = S > rwq::GEMV_FAMILY_MAX_M;
    const rwq::ActsView a = with_k(gemm ? d->gemm : d->gemv, k);
    const rwq::ActsView* ga = quantize && gemm ? &a : nullptr;
    const rwq::ActsView* va = quantize && !gemm ? &a : nullptr;
    DEC_CUDA(rwq::launch_rows_quant_v(mode, x, add, xout, w, b, S, k, ga, va, yout, s), "decoder row transform");
    return RWQ_OK;
}

int linear(rwq_decoder* d, rwq_qtensor* w, const float* bias, float* out, cudaStream_t s) {
    const bool gemm = d->n_streams > rwq::GEMV_FAMILY_MAX_M;
    const rwq::ActsView a = with_k(gemm ? d->gemm : d->gemv, rwq::weight_of(w).k);
    return rwq::linear_acts(a, gemm, w, bias, out, s);
}

void drop_graphs(rwq_decoder* d) {
    for (auto& kv : d->graphs) cudaGraphExecDestroy(kv.second);
    d->graphs.clear();
    d->eager_runs.clear();
}

bool graphs_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("RWQ_DECODER_GRAPHS");
        return !(v && v[0] == '0');
    }();
    return on;
}

// The kernels of one decode position (decoder.rs:102-206), reading the
// tokens from d->tok_in and the position from d->dpos; mode bit 0: tied
// logits into d->logits, bit 1: greedy choice into d->best, bit 2: the
// final-layernormed states into d->hid (forward_hidden, decoder.rs:110).
int issue_step(rwq_decoder* d, int mode, int32_t limit, cudaStream_t s) {
    const int S = d->n_streams, D = d->n_state, H = d->n_head, F = d->n_ff;
    DEC_CUDA(rwq::launch_embed(rwq::weight_of(d->emb), d->tok_in, S, d->dense["decoder.positional_embedding"], d->dpos,
                               d->x, s),
             "embed");
    const size_t self_layer = size_t(S) * H * d->n_ctx * 64, cross_layer = size_t(d->n_windows) * H * d->n_audio * 64;
    // GEMV-family steps: the attention kernels quantize their output rows
    // themselves (the layout k_rows_quant would write), one launch less
    // per attention.
    const bool gemv = S <= rwq::GEMV_FAMILY_MAX_M;
    rwq::AttnQuantOut qo;
    {
        const rwq::ActsView a = with_k(d->gemv, D);
        qo.q8 = a.q8;
        qo.d = a.d;
        qo.sum = a.sum;
        qo.u = a.u;
    }
    const rwq::AttnQuantOut* q_self = gemv && rwq::attn_dec_quantizes(1) ? &qo : nullptr;
    const rwq::AttnQuantOut* q_cross = gemv && rwq::attn_dec_quantizes(d->max_group) ? &qo : nullptr;
    for (int l = 0; l < d->n_layer; ++l) {
        const DLayer& L = d->layers[size_t(l)];
        // causal self-attention over the cache (decoder.rs:140-171)
        DEC_RC(rows(d, l ? rwq::RQ_ADD_LN : rwq::RQ_LN, d->x, d->tmp, d->x, L.attn_ln_w, L.attn_ln_b, D, s));
        const float *qp = d->q, *kp = d->k, *vp = d->v;
        int ld = D;
        if (L.qkv) {   // rows [q | k | v]
            DEC_RC(linear(d, L.qkv, L.qkv_b, d->qkv, s));
            qp = d->qkv;
            kp = d->qkv + D;
            vp = d->qkv + 2 * D;
            ld = 3 * D;
        } else {
            DEC_RC(linear(d, L.q, L.q_b, d->q, s));
            DEC_RC(linear(d, L.k, nullptr, d->k, s));
            DEC_RC(linear(d, L.v, L.v_b, d->v, s));
        }
        __half* kc = d->self_k + size_t(l) * self_layer;
        __half* vc = d->self_v + size_t(l) * self_layer;
        DEC_CUDA(rwq::launch_kv_append(kp, vp, ld, S, H, d->n_ctx, d->dpos, kc, vc, s), "kv append");
        DEC_CUDA(rwq::launch_attn_dec(qp, kc, vc, size_t(d->n_ctx) * 64, d->n_ctx, d->dpos, H, S, 1, d->self_kv,
                                      d->self_off, d->self_kv, d->att, 1, nullptr, nullptr, ld, q_self, s),
                 "self attention");
        if (!q_self) DEC_RC(rows(d, rwq::RQ_PLAIN, d->att, nullptr, nullptr, nullptr, nullptr, D, s));
        DEC_RC(linear(d, L.o, L.o_b, d->tmp, s));
        // cross-attention to the window's K/V (decoder.rs:173-188)
        DEC_RC(rows(d, rwq::RQ_ADD_LN, d->x, d->tmp, d->x, L.x_ln_w, L.x_ln_b, D, s));
        DEC_RC(linear(d, L.xq, L.xq_b, d->q, s));
        DEC_CUDA(rwq::launch_attn_dec(d->q, d->cross_k + size_t(l) * cross_layer, d->cross_v + size_t(l) * cross_layer,
                                      size_t(d->n_audio) * 64, d->n_audio, nullptr, H, d->n_cross_groups, d->max_group,
                                      d->cross_kv, d->cross_off, d->cross_streams, d->att, d->cross_splits,
                                      d->attn_part, d->attn_cnt, D, q_cross, s),
                 "cross attention");
        if (!q_cross) DEC_RC(rows(d, rwq::RQ_PLAIN, d->att, nullptr, nullptr, nullptr, nullptr, D, s));
        DEC_RC(linear(d, L.xo, L.xo_b, d->tmp, s));
        // MLP (encoder.rs:154-172)
        DEC_RC(rows(d, rwq::RQ_ADD_LN, d->x, d->tmp, d->x, L.mlp_ln_w, L.mlp_ln_b, D, s));
        DEC_RC(linear(d, L.fc1, L.fc1_b, d->h, s));
        DEC_RC(rows(d, rwq::RQ_GELU, d->h, nullptr, nullptr, nullptr, nullptr, F, s));
        DEC_RC(linear(d, L.fc2, L.fc2_b, d->tmp, s));
    }
    if (mode) {
        // final LN (decoder.rs:200-204), tied logits (decoder.rs:315-321)
        const bool proj = (mode & 3) != 0;
        DEC_RC(rows(d, d->n_layer ? rwq::RQ_ADD_LN : rwq::RQ_LN, d->x, d->tmp, d->x, d->dense["decoder.ln.weight"],
                    d->dense["decoder.ln.bias"], D, s, (mode & 4) ? d->hid : nullptr, proj));
        if (proj) DEC_RC(linear(d, d->emb, nullptr, d->logits, s));
        if (mode & 2) DEC_CUDA(rwq::launch_argmax(d->logits, S, d->n_vocab, limit, d->best, s), "argmax");
    }
    DEC_CUDA(rwq::launch_pos_advance(d->dpos, s), "position advance");
    return RWQ_OK;
}

// Run one position: replay its graph, capture it (second run of a mode),
// or issue it eagerly.
int run_step(rwq_decoder* d, int mode, int32_t limit, cudaStream_t s) {
    const std::pair<int, int> key(mode, (mode & 2) ? limit : 0);
    auto it = d->graphs.find(key);
    if (it != d->graphs.end()) {
        DEC_CUDA(cudaGraphLaunch(it->second, s), "cudaGraphLaunch(decoder step)");
        return RWQ_OK;
    }
    if (!graphs_enabled() || d->eager_runs[key] == 0) {
        ++d->eager_runs[key];
        return issue_step(d, mode, limit, s);
    }
    cudaGraph_t g = nullptr;
    DEC_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeRelaxed), "cudaStreamBeginCapture");
    const int rc = issue_step(d, mode, limit, s);
    const cudaError_t ec = cudaStreamEndCapture(s, &g);
    if (rc || ec != cudaSuccess || !g) {
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        if (rc) return rc;
        ++d->eager_runs[key];
        return issue_step(d, mode, limit, s);   // not capturable here: stay eager
    }
    cudaGraphExec_t ex = nullptr;
    const cudaError_t ei = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    if (ei != cudaSuccess) {
        cudaGetLastError();
        ++d->eager_runs[key];
        return issue_step(d, mode, limit, s);
    }
    d->graphs[key] = ex;
    DEC_CUDA(cudaGraphLaunch(ex, s), "cudaGraphLaunch(decoder step)");
    return RWQ_OK;
}

}  // namespace

extern "C" {

int rwq_decoder_new(int n_vocab, int n_ctx, int n_state, int n_head, int n_layer, rwq_decoder** out) {
    if (!out) return dfail(RWQ_ERR_ARG, "out is null");
    *out = nullptr;
    if (n_vocab <= 0 || n_ctx <= 0 || n_state <= 0 || n_head <= 0 || n_layer < 0)
        return dfail(RWQ_ERR_ARG, "bad decoder shape");
    if (n_state % n_head || n_state / n_head != 64)
        return dfail(RWQ_ERR_ARG, "head dim must be 64 (n_state %d, n_head %d)", n_state, n_head);
    if (n_state % 128) return dfail(RWQ_ERR_ARG, "n_state must be a multiple of 128 (got %d)", n_state);
    auto* d = new rwq_decoder;
    cudaGetDevice(&d->device);
    d->n_vocab = n_vocab;
    d->n_ctx = n_ctx;
    d->n_state = n_state;
    d->n_head = n_head;
    d->n_layer = n_layer;
    d->n_ff = 4 * n_state;
    d->layers.resize(size_t(n_layer));
    if (cudaStreamCreateWithFlags(&d->gs, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&d->ev_in, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&d->ev_out, cudaEventDisableTiming) != cudaSuccess) {
        rwq_decoder_free(d);
        return dfail(RWQ_ERR_CUDA, "decoder stream/event creation failed");
    }
    d->dense_len["decoder.positional_embedding"] = size_t(n_ctx) * n_state;
    d->dense_len["decoder.ln.weight"] = size_t(n_state);
    d->dense_len["decoder.ln.bias"] = size_t(n_state);
    for (int l = 0; l < n_layer; ++l) {
        for (const char* f : kDenseLayer) d->dense_len[lname(l, f)] = size_t(n_state);
        d->dense_len[lname(l, "mlp.0.bias")] = size_t(d->n_ff);
    }
    *out = d;
    return RWQ_OK;
}

int rwq_decoder_free(rwq_decoder* d) {
    if (!d) return RWQ_OK;
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != d->device) cudaSetDevice(d->device);
    for (auto& kv : d->dense) cudaFree(kv.second);
    for (auto& L : d->layers) {
        for (rwq_qtensor* t : {L.q, L.k, L.v, L.o, L.xq, L.xk, L.xv, L.xo, L.fc1, L.fc2, L.qkv}) rwq_qtensor_free(t);
        cudaFree(L.qkv_b);
    }
    rwq_qtensor_free(d->emb);
    if (d->gs) cudaStreamSynchronize(d->gs);
    drop_graphs(d);
    cudaFree(d->state);
    if (d->ev_in) cudaEventDestroy(d->ev_in);
    if (d->ev_out) cudaEventDestroy(d->ev_out);
    if (d->gs) cudaStreamDestroy(d->gs);
    if (prev != d->device) cudaSetDevice(prev);
    delete d;
    return RWQ_OK;
}

int rwq_decoder_set_dense(rwq_decoder* d, const char* name, const float* data, int64_t count) {
    if (!d || !name || !data) return dfail(RWQ_ERR_ARG, "null argument");
    std::lock_guard<std::mutex> g(d->mu);
    auto it = d->dense_len.find(name);
    if (it == d->dense_len.end()) return dfail(RWQ_ERR_ARG, "'%s' is not a dense decoder tensor", name);
    if (count < 0 || size_t(count) != it->second)
        return dfail(RWQ_ERR_SHAPE, "'%s': %lld elements, expected %zu", name, (long long)count, it->second);
    float*& dst = d->dense[name];
    if (!dst) DEC_CUDA(cudaMalloc(&dst, it->second * 4), "cudaMalloc(dense tensor)");
    DEC_CUDA(cudaMemcpy(dst, data, it->second * 4, cudaMemcpyHostToDevice), "copy dense tensor");
    return RWQ_OK;
}

int rwq_decoder_set_quant(rwq_decoder* d, const char* name, int dtype, const uint8_t* raw, size_t raw_len, int64_t n,
                          int64_t k) {
    if (!d || !name) return dfail(RWQ_ERR_ARG, "null argument");
    std::lock_guard<std::mutex> g(d->mu);
    int64_t wn = 0, wk = 0;
    rwq_qtensor** slot = quant_slot(d, name, &wn, &wk);
    if (!slot) return dfail(RWQ_ERR_ARG, "'%s' is not a quantized decoder matrix", name);
    if (n != wn || k != wk)
        return dfail(RWQ_ERR_SHAPE, "'%s': [%lld, %lld], expected [%lld, %lld]", name, (long long)n, (long long)k,
                     (long long)wn, (long long)wk);
    rwq_qtensor* t = nullptr;
    DEC_RC(rwq_qtensor_new(raw, raw_len, dtype, n, k, &t));
    rwq_qtensor_free(*slot);
    *slot = t;
    for (auto& L : d->layers)   // rebuilt from the new matrices at the next begin
        if (slot == &L.q || slot == &L.k || slot == &L.v) {
            rwq_qtensor_free(L.qkv);
            L.qkv = nullptr;
        }
    return RWQ_OK;
}

int rwq_decoder_begin(rwq_decoder* d, const float* enc_out, int64_t n_windows, int64_t n_audio,
                      const int32_t* stream_window, int64_t n_streams, void* stream) {
    if (!d) return dfail(RWQ_ERR_ARG, "decoder is null");
    if (n_windows <= 0 || n_audio <= 0 || n_streams <= 0) return dfail(RWQ_ERR_ARG, "bad begin shape");
    if (!enc_out || (reinterpret_cast<uintptr_t>(enc_out) & 15))
        return dfail(RWQ_ERR_ARG, "encoder output must be a 16-byte aligned device pointer");
    if (n_windows > (1 << 20) || n_streams > (1 << 20) || n_audio > 8192) return dfail(RWQ_ERR_ARG, "begin too large");
    std::lock_guard<std::mutex> g(d->mu);
    DEC_RC(check_ready(d));
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev != d->device) return dfail(RWQ_ERR_ARG, "decoder lives on device %d, current device is %d", d->device, dev);
    for (int l = 0; l < d->n_layer; ++l) {
        DLayer& L = d->layers[size_t(l)];
        auto P = [&](const char* f) { return static_cast<const float*>(d->dense[lname(l, f)]); };
        L.attn_ln_w = P("attn_ln.weight");
        L.attn_ln_b = P("attn_ln.bias");
        L.q_b = P("attn.query.bias");
        L.v_b = P("attn.value.bias");
        L.o_b = P("attn.out.bias");
        L.x_ln_w = P("cross_attn_ln.weight");
        L.x_ln_b = P("cross_attn_ln.bias");
        L.xq_b = P("cross_attn.query.bias");
        L.xo_b = P("cross_attn.out.bias");
        L.mlp_ln_w = P("mlp_ln.weight");
        L.mlp_ln_b = P("mlp_ln.bias");
        L.fc1_b = P("mlp.0.bias");
        L.fc2_b = P("mlp.2.bias");
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int S = int(n_streams), W = int(n_windows), T = int(n_audio), D = d->n_state, H = d->n_head;
    // Q, K and V of each layer as one weight (same bits as three GEMVs:
    // the GEMV family's summation order depends on N only through its K
    // split, the same at D and 3D rows for whisper's sizes; the GEMM
    // family's does not depend on N), bias [q_b, 0, v_b].
    for (int l = 0; l < d->n_layer; ++l) {
        DLayer& L = d->layers[size_t(l)];
        if (!L.q || !L.k || !L.v) continue;
        if (!L.qkv) {
            rwq_qtensor* parts[3] = {L.q, L.k, L.v};
            if (rwq::qtensor_concat_rows(parts, 3, s, &L.qkv) != RWQ_OK) L.qkv = nullptr;   // three GEMVs then
        }
        if (L.qkv && !L.qkv_b) DEC_CUDA(cudaMalloc(&L.qkv_b, size_t(3) * D * 4), "cudaMalloc(qkv bias)");
        if (L.qkv) {
            DEC_CUDA(cudaMemsetAsync(L.qkv_b, 0, size_t(3) * D * 4, s), "qkv bias");
            if (L.q_b) DEC_CUDA(cudaMemcpyAsync(L.qkv_b, L.q_b, size_t(D) * 4, cudaMemcpyDeviceToDevice, s), "qkv bias");
            if (L.v_b)
                DEC_CUDA(cudaMemcpyAsync(L.qkv_b + 2 * D, L.v_b, size_t(D) * 4, cudaMemcpyDeviceToDevice, s), "qkv bias");
        }
    }
    // stream -> window map and the cross-attention groups (<= DEC_MAX_G
    // streams of one window each)
    std::vector<int> win(static_cast<size_t>(S));
    for (int i = 0; i < S; ++i) {
        win[size_t(i)] = stream_window ? stream_window[i] : (W == S ? i : -1);
        if (win[size_t(i)] < 0 || win[size_t(i)] >= W)
            return dfail(RWQ_ERR_ARG, "stream %d maps to window %d of %d", i, win[size_t(i)], W);
    }
    // Cross-attention groups: the streams of one window (beams) share a
    // group of up to DEC_MAX_G, which reads the window's K/V once on the
    // tensor-core kernel, with the keys split over several CTAs per (head,
    // group) to fill the GPU.  One stream per window: one group each,
    // ordered by window, on the CUDA-core kernel.
    std::vector<int> gkv, goff(1, 0), gst;
    for (int w = 0; w < W; ++w) {
        int in_group = 0;
        for (int i = 0; i < S; ++i) {
            if (win[size_t(i)] != w) continue;
            if (in_group == rwq::DEC_MAX_G) {
                goff.push_back(int(gst.size()));
                in_group = 0;
            }
            if (in_group == 0) gkv.push_back(w);
            gst.push_back(i);
            ++in_group;
        }
        if (in_group) goff.push_back(int(gst.size()));
    }
    const int NG = int(gkv.size());
    int max_group = 1;
    for (int i = 0; i < NG; ++i) max_group = std::max(max_group, goff[size_t(i) + 1] - goff[size_t(i)]);
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d->device);
    const int splits = rwq::attn_dec_splits(H, NG, max_group, T, sms);
    DEC_CUDA(cudaStreamSynchronize(d->gs), "cudaStreamSynchronize(decoder)");
    drop_graphs(d);
    const size_t need = layout_state(d, S, W, T, NG, splits, nullptr);
    if (d->state_bytes < need) {
        DEC_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
        cudaFree(d->state);
        d->state = nullptr;
        d->state_bytes = 0;
        DEC_CUDA(cudaMalloc(&d->state, need), "cudaMalloc(decoder state)");
        d->state_bytes = need;
    }
    layout_state(d, S, W, T, NG, splits, static_cast<uint8_t*>(d->state));
    d->n_streams = S;
    d->n_windows = W;
    d->n_audio = T;
    d->n_cross_groups = NG;
    d->max_group = max_group;
    d->cross_splits = splits;
    if (d->attn_cnt) DEC_CUDA(cudaMemsetAsync(d->attn_cnt, 0, size_t(NG) * H * 4, s), "zero split counters");
    d->n_past = 0;
    std::vector<int> sid(static_cast<size_t>(S)), soff(static_cast<size_t>(S) + 1);
    for (int i = 0; i <= S; ++i) {
        if (i < S) sid[size_t(i)] = i;
        soff[size_t(i)] = i;
    }
    DEC_CUDA(cudaMemsetAsync(d->dpos, 0, sizeof(int), s), "reset position");
    DEC_CUDA(cudaMemcpyAsync(d->cross_kv, gkv.data(), gkv.size() * 4, cudaMemcpyHostToDevice, s), "copy groups");
    DEC_CUDA(cudaMemcpyAsync(d->cross_off, goff.data(), goff.size() * 4, cudaMemcpyHostToDevice, s), "copy groups");
    DEC_CUDA(cudaMemcpyAsync(d->cross_streams, gst.data(), gst.size() * 4, cudaMemcpyHostToDevice, s), "copy groups");
    DEC_CUDA(cudaMemcpyAsync(d->self_kv, sid.data(), sid.size() * 4, cudaMemcpyHostToDevice, s), "copy groups");
    DEC_CUDA(cudaMemcpyAsync(d->self_off, soff.data(), soff.size() * 4, cudaMemcpyHostToDevice, s), "copy groups");
    DEC_CUDA(cudaMemcpyAsync(d->win_dev, win.data(), win.size() * 4, cudaMemcpyHostToDevice, s), "copy windows");
    // cross K/V (decoder.rs:41-56): quantize the encoder output once, then
    // two GEMMs per layer, windows in chunks to bound the scratch.
    const int per = std::max(1, int((size_t(1) << 30) / (size_t(T) * D * 14)));
    for (int w0 = 0; w0 < W; w0 += per) {
        const int nw = std::min(per, W - w0);
        const int M = nw * T;
        const size_t m_pad = align_up(size_t(M), 256);
        const size_t kv_b = align_up(size_t(M) * D * 4, 256), q_b = align_up(size_t(M) * D * 2, 256),
                     sc_b = align_up(size_t(D / 32) * m_pad * 4, 256);
        int rc = rwq::with_stream_scratch(s, 2 * kv_b + q_b + 2 * sc_b, [&](void* buf) {
            uint8_t* p = static_cast<uint8_t*>(buf);
            float* kt = reinterpret_cast<float*>(p);
            float* vt = reinterpret_cast<float*>(p + kv_b);
            rwq::ActsView a;
            a.m = M;
            a.k = D;
            a.nb = D / 32;
            a.m_pad = int(m_pad);
            a.q16 = reinterpret_cast<uint16_t*>(p + 2 * kv_b);
            a.dT = reinterpret_cast<float*>(p + 2 * kv_b + q_b);
            a.uT = reinterpret_cast<float*>(p + 2 * kv_b + q_b + sc_b);
            DEC_CUDA(rwq::launch_rows_quant_v(rwq::RQ_PLAIN, enc_out + size_t(w0) * T * D, nullptr, nullptr, nullptr,
                                              nullptr, M, D, &a, nullptr, nullptr, s),
                     "quantize encoder output");
            for (int l = 0; l < d->n_layer; ++l) {
                const DLayer& L = d->layers[size_t(l)];
                const size_t lo = (size_t(l) * W + w0) * H * size_t(T) * 64;
                const float* vb = d->dense[lname(l, "cross_attn.value.bias")];
                if (rwq::gemm_heads_fits(a, L.xk, nw, T, H, d->cross_k + lo) &&
                    rwq::gemm_heads_fits(a, L.xv, nw, T, H, d->cross_v + lo)) {
                    // the projections write their f16 heads themselves
                    DEC_RC(rwq::gemm_heads(a, L.xk, nullptr, d->cross_k + lo, nw, T, H, 1.0f, s));
                    DEC_RC(rwq::gemm_heads(a, L.xv, vb, d->cross_v + lo, nw, T, H, 1.0f, s));
                } else {
                    DEC_RC(rwq::gemm_quantized(a, L.xk, nullptr, kt, s));
                    DEC_RC(rwq::gemm_quantized(a, L.xv, vb, vt, s));
                    DEC_CUDA(rwq::launch_to_heads(kt, D, 0, nw, T, H, 1.0f, d->cross_k + lo, s), "cross k heads");
                    DEC_CUDA(rwq::launch_to_heads(vt, D, 0, nw, T, H, 1.0f, d->cross_v + lo, s), "cross v heads");
                }
            }
            return int(RWQ_OK);
        });
        if (rc) return rc;
    }
    return RWQ_OK;
}

namespace {
int step_impl(rwq_decoder* d, const int32_t* tokens, float* logits, int32_t* best, int32_t limit, float* hidden,
              void* stream);
}

int rwq_decoder_step(rwq_decoder* d, const int32_t* tokens, float* logits, int32_t* best, int32_t limit,
                     void* stream) {
    return step_impl(d, tokens, logits, best, limit, nullptr, stream);
}

int rwq_decoder_step_hidden(rwq_decoder* d, const int32_t* tokens, float* hidden, void* stream) {
    if (!hidden) return dfail(RWQ_ERR_ARG, "hidden is null");
    return step_impl(d, tokens, nullptr, nullptr, -1, hidden, stream);
}

int rwq_decoder_project(rwq_decoder* d, const float* hidden, int64_t rows_n, float* logits, void* stream) {
    if (!d) return dfail(RWQ_ERR_ARG, "decoder is null");
    std::lock_guard<std::mutex> g(d->mu);
    if (!d->n_streams) return dfail(RWQ_ERR_ARG, "rwq_decoder_begin was not called");
    if (rows_n < 0 || rows_n > d->n_streams)
        return dfail(RWQ_ERR_ARG, "project: %lld rows, at most the %d streams", (long long)rows_n, d->n_streams);
    if (rows_n == 0) return RWQ_OK;
    if (!hidden || !logits) return dfail(RWQ_ERR_ARG, "null hidden or logits");
    if (reinterpret_cast<uintptr_t>(hidden) & 15) return dfail(RWQ_ERR_ARG, "hidden must be 16-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int R = int(rows_n), D = d->n_state;
    // The step's own row kernel and linear, on R rows: the same bits as the
    // projection inside rwq_decoder_step (the GEMV family's results do not
    // depend on the row count).
    const bool gemm = d->n_streams > rwq::GEMV_FAMILY_MAX_M;
    rwq::ActsView a = with_k(gemm ? d->gemm : d->gemv, D);
    a.m = R;
    DEC_CUDA(rwq::launch_rows_quant_v(rwq::RQ_PLAIN, hidden, nullptr, nullptr, nullptr, nullptr, R, D,
                                      gemm ? &a : nullptr, gemm ? nullptr : &a, nullptr, s),
             "quantize hidden rows");
    return rwq::linear_acts(a, gemm, d->emb, nullptr, logits, s);
}

int rwq_decoder_fork(rwq_decoder* d, const int32_t* src, void* stream) {
    if (!d) return dfail(RWQ_ERR_ARG, "decoder is null");
    if (!src) return dfail(RWQ_ERR_ARG, "src is null");
    std::lock_guard<std::mutex> g(d->mu);
    if (!d->n_streams) return dfail(RWQ_ERR_ARG, "rwq_decoder_begin was not called");
    DEC_CUDA(rwq::launch_self_fork(src, d->win_dev, d->n_streams, d->n_head, d->n_ctx, d->n_layer, d->dpos,
                                   d->self_k, d->self_v, static_cast<cudaStream_t>(stream)),
             "fork");
    return RWQ_OK;
}

namespace {
int step_impl(rwq_decoder* d, const int32_t* tokens, float* logits, int32_t* best, int32_t limit, float* hidden,
              void* stream) {
    if (!d) return dfail(RWQ_ERR_ARG, "decoder is null");
    if (!tokens) return dfail(RWQ_ERR_ARG, "tokens is null");
    std::lock_guard<std::mutex> g(d->mu);
    if (!d->n_streams) return dfail(RWQ_ERR_ARG, "rwq_decoder_begin was not called");
    if (d->n_past >= d->n_ctx)
        return dfail(RWQ_ERR_ARG, "decoder context overflow: %d + 1 > %d", d->n_past, d->n_ctx);   // decoder.rs:115-120
    if (limit >= d->n_vocab) return dfail(RWQ_ERR_ARG, "limit %d >= n_vocab %d", limit, d->n_vocab);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int S = d->n_streams;
    if (tokens != d->tok_in)
        DEC_CUDA(cudaMemcpyAsync(d->tok_in, tokens, size_t(S) * 4, cudaMemcpyDeviceToDevice, s), "copy tokens");
    const int mode = (logits ? 1 : 0) | (best ? 2 : 0) | (hidden ? 4 : 0);
    DEC_CUDA(cudaEventRecord(d->ev_in, s), "cudaEventRecord");
    DEC_CUDA(cudaStreamWaitEvent(d->gs, d->ev_in, 0), "cudaStreamWaitEvent");
    DEC_RC(run_step(d, mode, limit, d->gs));
    DEC_CUDA(cudaEventRecord(d->ev_out, d->gs), "cudaEventRecord");
    DEC_CUDA(cudaStreamWaitEvent(s, d->ev_out, 0), "cudaStreamWaitEvent");
    d->n_past += 1;
    if (logits)
        DEC_CUDA(cudaMemcpyAsync(logits, d->logits, size_t(S) * d->n_vocab * 4, cudaMemcpyDeviceToDevice, s),
                 "copy logits");
    if (best) DEC_CUDA(cudaMemcpyAsync(best, d->best, size_t(S) * 4, cudaMemcpyDeviceToDevice, s), "copy ids");
    if (hidden && hidden != d->hid)
        DEC_CUDA(cudaMemcpyAsync(hidden, d->hid, size_t(S) * d->n_state * 4, cudaMemcpyDeviceToDevice, s),
                 "copy hidden");
    return RWQ_OK;
}
}  // namespace

int rwq_decoder_reset(rwq_decoder* d) {
    if (!d) return dfail(RWQ_ERR_ARG, "decoder is null");
    std::lock_guard<std::mutex> g(d->mu);
    d->n_past = 0;   // the self-attention cache is overwritten from position 0
    if (d->dpos) {
        DEC_CUDA(cudaDeviceSynchronize(), "cudaDeviceSynchronize");   // no step of this decoder in flight
        DEC_CUDA(cudaMemset(d->dpos, 0, sizeof(int)), "reset position");
    }
    return RWQ_OK;
}

int rwq_decoder_n_past(const rwq_decoder* d, int64_t* n_past) {
    if (!d || !n_past) return dfail(RWQ_ERR_ARG, "null argument");
    *n_past = d->n_past;
    return RWQ_OK;
}

}  // extern "C"
