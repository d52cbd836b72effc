// rwq_encoder.cu -- the device-resident Whisper encoder forward behind the
// C ABI (rwq_encoder_* in include/rwq.h): the reference's encoder::encode
// (encoder.rs:180-234) for a batch of 30 s windows at once, every 2-D
// linear on the quantized tensor-core GEMM.
//
// Per batch of W windows (T = n_ctx frames each, M = W*T rows):
//   conv stem   the conv weights stay dense f32, as the reference keeps
//               them (model.rs:231-257); each conv1d (tensor.rs:335-370)
//               is an im2col GEMM on the tensor cores with both operands
//               split into f16 hi + lo (k_im2col_split, k_gemm_hl: about
//               22 significant bits per operand, the accuracy of f32 for
//               these sums), bias/GELU (+ positions) in the GEMM epilogue;
//   per block   [residual add +] LayerNorm + int8 quantize (one kernel)
//               -> Q, K, V GEMMs sharing the quantized activations
//               -> f16 heads -> flash attention -> quantize -> out GEMM
//               -> residual add + LayerNorm + quantize -> fc1 GEMM
//               -> GELU + quantize -> fc2 GEMM;
//   ln_post     fused with the last residual add.
// The activations stay in HBM between kernels; nothing returns to the host.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>
#include "../../include/rwq.h"
#include "rwq_common.cuh"
#include "rwq_encoder.h"
#include "rwq_internal.h"

namespace {

int efail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    rwq::set_last_error(buf);
    return code;
}

#define ENC_CUDA(call, what)                                                                               \
    do {                                                                                                   \
        cudaError_t e_ = (call);                                                                           \
        if (e_ != cudaSuccess)                                                                             \
            return efail(e_ == cudaErrorMemoryAllocation ? RWQ_ERR_NOMEM : RWQ_ERR_CUDA, "%s: %s", what,   \
                         cudaGetErrorString(e_));                                                          \
    } while (0)

#define ENC_RC(call)              \
    do {                          \
        int rc_ = (call);         \
        if (rc_) return rc_;      \
    } while (0)

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct Layer {
    rwq_qtensor *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr, *fc1 = nullptr, *fc2 = nullptr;
};

}  // namespace

struct rwq_encoder {
    int device = 0;
    int n_mels = 0, n_ctx = 0, n_state = 0, n_head = 0, n_layer = 0, n_ff = 0;
    std::map<std::string, float*> dense;       // device copies, by whisper.cpp name
    std::map<std::string, size_t> dense_len;   // expected element counts
    std::vector<Layer> layers;
    // conv weights as hi|lo GEMM operands [D][kp/32][64] + column scales,
    // built from the dense tensors at the first encode after they are set
    uint16_t *conv1_hl = nullptr, *conv2_hl = nullptr;
    float *conv1_cs = nullptr, *conv2_cs = nullptr;
    bool stem_ready = false;
    void* ws = nullptr;                        // batch workspace (grown on demand)
    size_t ws_bytes = 0;
    std::mutex mu;
};

namespace {

std::string lname(int l, const char* f) { return "encoder.blocks." + std::to_string(l) + "." + f; }

// The dense tensors the encoder needs, with their element counts.
void expected_dense(rwq_encoder* e) {
    const size_t D = size_t(e->n_state);
    auto& m = e->dense_len;
    m["encoder.conv1.weight"] = D * e->n_mels * 3;
    m["encoder.conv1.bias"] = D;
    m["encoder.conv2.weight"] = D * D * 3;
    m["encoder.conv2.bias"] = D;
    m["encoder.positional_embedding"] = size_t(e->n_ctx) * D;
    m["encoder.ln_post.weight"] = D;
    m["encoder.ln_post.bias"] = D;
    for (int l = 0; l < e->n_layer; ++l) {
        for (const char* f : {"attn_ln.weight", "attn_ln.bias", "attn.query.bias", "attn.value.bias", "attn.out.bias",
                              "mlp_ln.weight", "mlp_ln.bias", "mlp.2.bias"})
            m[lname(l, f)] = D;
        m[lname(l, "mlp.0.bias")] = size_t(e->n_ff);
    }
}

rwq_qtensor** quant_slot(rwq_encoder* e, const std::string& name, int64_t* want_n, int64_t* want_k) {
    const std::string pre = "encoder.blocks.";
    if (name.compare(0, pre.size(), pre) != 0) return nullptr;
    const size_t dot = name.find('.', pre.size());
    if (dot == std::string::npos) return nullptr;
    const std::string idx = name.substr(pre.size(), dot - pre.size());
    if (idx.empty() || idx.find_first_not_of("0123456789") != std::string::npos) return nullptr;
    const int l = std::atoi(idx.c_str());
    if (l < 0 || l >= e->n_layer) return nullptr;
    const std::string f = name.substr(dot + 1);
    Layer& L = e->layers[size_t(l)];
    const int64_t D = e->n_state, F = e->n_ff;
    *want_n = D;
    *want_k = D;
    if (f == "attn.query.weight") return &L.q;
    if (f == "attn.key.weight") return &L.k;
    if (f == "attn.value.weight") return &L.v;
    if (f == "attn.out.weight") return &L.o;
    if (f == "mlp.0.weight") { *want_n = F; return &L.fc1; }
    if (f == "mlp.2.weight") { *want_k = F; return &L.fc2; }
    return nullptr;
}

struct Bufs {
    float *x, *tmp, *q, *k, *v, *h, *att, *c1;
    uint16_t *a1, *a2;    // conv1 / conv2 im2col rows as hi|lo operands
    float *rs1, *rs2;     // their row scales
    __half *qh, *kh, *vh;
    rwq::ActsView acts;   // GEMM layout, k up to n_ff
};

// Columns of conv1's im2col rows: 3 * n_mels rounded up to a 32-block.
int conv1_kp(const rwq_encoder* e) { return (3 * e->n_mels + 31) / 32 * 32; }

size_t carve(const rwq_encoder* e, int nwin, uint8_t* base, Bufs* b) {
    const size_t T = size_t(e->n_ctx), D = size_t(e->n_state), F = size_t(e->n_ff), M = size_t(nwin) * T;
    const size_t m_pad = align_up(M, 256), kmax = std::max(D, F);
    size_t off = 0;
    auto take = [&](size_t bytes) {
        uint8_t* p = base ? base + off : nullptr;
        off = align_up(off + bytes, 256);
        return p;
    };
    Bufs z;
    z.x = reinterpret_cast<float*>(take(M * D * 4));
    z.tmp = reinterpret_cast<float*>(take(M * D * 4));
    z.q = reinterpret_cast<float*>(take(M * D * 4));
    z.k = reinterpret_cast<float*>(take(M * D * 4));
    z.v = reinterpret_cast<float*>(take(M * D * 4));
    z.h = reinterpret_cast<float*>(take(M * F * 4));
    z.att = reinterpret_cast<float*>(take(M * D * 4));
    z.a1 = reinterpret_cast<uint16_t*>(take(2 * M * size_t(conv1_kp(e)) * 4));
    z.rs1 = reinterpret_cast<float*>(take(2 * M * 4));
    z.c1 = reinterpret_cast<float*>(take(2 * M * D * 4));
    z.a2 = reinterpret_cast<uint16_t*>(take(M * D * 3 * 4));
    z.rs2 = reinterpret_cast<float*>(take(M * 4));
    z.qh = reinterpret_cast<__half*>(take(M * D * 2));
    z.kh = reinterpret_cast<__half*>(take(M * D * 2));
    z.vh = reinterpret_cast<__half*>(take(M * D * 2));
    z.acts.m = int(M);
    z.acts.m_pad = int(m_pad);
    z.acts.q16 = reinterpret_cast<uint16_t*>(take(M * kmax * 2));
    z.acts.dT = reinterpret_cast<float*>(take(kmax / 32 * m_pad * 4));
    z.acts.uT = reinterpret_cast<float*>(take(kmax / 32 * m_pad * 4));
    if (b) *b = z;
    return off;
}

int check_ready(rwq_encoder* e) {
    for (auto& kv : e->dense_len)
        if (!e->dense.count(kv.first)) return efail(RWQ_ERR_ARG, "encoder tensor '%s' was not set", kv.first.c_str());
    for (int l = 0; l < e->n_layer; ++l) {
        const Layer& L = e->layers[size_t(l)];
        if (!L.q || !L.k || !L.v || !L.o || !L.fc1 || !L.fc2)
            return efail(RWQ_ERR_ARG, "encoder block %d: a linear weight was not set", l);
    }
    return RWQ_OK;
}

rwq::ActsView acts_for(const Bufs& b, int k) {
    rwq::ActsView v = b.acts;
    v.k = k;
    v.nb = k / rwq::QK;
    return v;
}

// The conv weights as hi|lo GEMM operands (once per set of weights).
int ensure_stem(rwq_encoder* e, cudaStream_t s) {
    if (e->stem_ready) return RWQ_OK;
    const int D = e->n_state, NM = e->n_mels, k1 = conv1_kp(e);
    const int n_pad = (D + 255) / 256 * 256;
    if (!e->conv1_hl) {
        ENC_CUDA(cudaMalloc(&e->conv1_hl, size_t(D) * k1 * 4), "cudaMalloc(conv1 operand)");
        ENC_CUDA(cudaMalloc(&e->conv2_hl, size_t(D) * 3 * D * 4), "cudaMalloc(conv2 operand)");
        ENC_CUDA(cudaMalloc(&e->conv1_cs, size_t(n_pad) * 4), "cudaMalloc(conv1 scales)");
        ENC_CUDA(cudaMalloc(&e->conv2_cs, size_t(n_pad) * 4), "cudaMalloc(conv2 scales)");
    }
    // weight [D][in][3]: row j's column c*3 + kk is the im2col column order
    ENC_CUDA(rwq::launch_split_dense(e->dense["encoder.conv1.weight"], D, k1, 3 * NM, 3 * NM, n_pad, e->conv1_hl,
                                     e->conv1_cs, s),
             "split conv1 weights");
    ENC_CUDA(rwq::launch_split_dense(e->dense["encoder.conv2.weight"], D, 3 * D, 3 * D, 3 * D, n_pad, e->conv2_hl,
                                     e->conv2_cs, s),
             "split conv2 weights");
    e->stem_ready = true;
    return RWQ_OK;
}

// The forward for `nwin` windows (mel [nwin][n_mels][2*n_ctx] on the device).
int encode_batch(rwq_encoder* e, const Bufs& b, const float* mel, int nwin, float* out, cudaStream_t s) {
    const int T = e->n_ctx, D = e->n_state, F = e->n_ff, H = e->n_head, NM = e->n_mels;
    const int M = nwin * T, M2 = 2 * M, m_pad = b.acts.m_pad, k1 = conv1_kp(e);
    auto W = [&](const std::string& n) { return e->dense[n]; };
    ENC_RC(ensure_stem(e, s));
    // conv1 (stride 1) + bias + GELU in the GEMM's epilogue:
    // [2T][n_mels*3] x [D][n_mels*3]^T per window
    ENC_CUDA(rwq::launch_im2col_split(mel, nwin, NM, 2 * T, 2 * T, 1, size_t(NM) * 2 * T, size_t(2 * T), 1, k1, b.a1,
                                      b.rs1, s),
             "im2col conv1");
    rwq::HlEpilogue epi;
    epi.gelu = true;
    ENC_RC(rwq::gemm_hl(b.a1, b.rs1, M2, e->conv1_hl, e->conv1_cs, D, k1 / rwq::QK, W("encoder.conv1.bias"), b.c1, s,
                        &epi));
    // conv2 (stride 2) + bias + GELU + positions, written time-major: x [M][D]
    ENC_CUDA(rwq::launch_im2col_split(b.c1, nwin, D, 2 * T, T, 2, size_t(2 * T) * D, 1, size_t(D), 3 * D, b.a2, b.rs2,
                                      s),
             "im2col conv2");
    epi.pos = W("encoder.positional_embedding");
    epi.pos_period = T;
    ENC_RC(rwq::gemm_hl(b.a2, b.rs2, M, e->conv2_hl, e->conv2_cs, D, 3 * D / rwq::QK, W("encoder.conv2.bias"), b.x, s,
                        &epi));
    const rwq::ActsView aD = acts_for(b, D), aF = acts_for(b, F);
    // fc2's operand in b.h's memory (f16 codes [M][F], then d_a and
    // d_a*sum(q_a) [F/32][m_pad]): the fused fc1 writes it while its own
    // operand (b.acts) is still being read.
    rwq::ActsView aH = aF;
    aH.q16 = reinterpret_cast<uint16_t*>(b.h);
    aH.dT = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(b.h) + align_up(size_t(M) * F * 2, 256));
    aH.uT = aH.dT + size_t(F / rwq::QK) * m_pad;
    aH.q8 = nullptr;
    aH.d = nullptr;
    aH.sum = nullptr;
    aH.u = nullptr;
    const float qscale = 1.0f / std::sqrt(float(D / H));   // 1/8 for head dim 64: exact
    for (int l = 0; l < e->n_layer; ++l) {
        const Layer& L = e->layers[size_t(l)];
        // [x += mlp out of the previous block;] LayerNorm -> quantize
        ENC_CUDA(rwq::launch_rows_quant(l ? rwq::RQ_ADD_LN : rwq::RQ_LN, b.x, b.tmp, b.x, W(lname(l, "attn_ln.weight")),
                                        W(lname(l, "attn_ln.bias")), M, D, m_pad, aD.q16, aD.dT, aD.uT, nullptr, s),
                 "attn_ln");
        if (rwq::gemm_heads_fits(aD, L.q, nwin, T, H, b.qh) && rwq::gemm_heads_fits(aD, L.k, nwin, T, H, b.kh) &&
            rwq::gemm_heads_fits(aD, L.v, nwin, T, H, b.vh)) {
            // the projections write their f16 heads themselves
            ENC_RC(rwq::gemm_heads(aD, L.q, W(lname(l, "attn.query.bias")), b.qh, nwin, T, H, qscale, s));
            ENC_RC(rwq::gemm_heads(aD, L.k, nullptr, b.kh, nwin, T, H, 1.0f, s));   // no key bias in whisper
            ENC_RC(rwq::gemm_heads(aD, L.v, W(lname(l, "attn.value.bias")), b.vh, nwin, T, H, 1.0f, s));
        } else {
            ENC_RC(rwq::gemm_quantized(aD, L.q, W(lname(l, "attn.query.bias")), b.q, s));
            ENC_RC(rwq::gemm_quantized(aD, L.k, nullptr, b.k, s));   // whisper's key projection has no bias
            ENC_RC(rwq::gemm_quantized(aD, L.v, W(lname(l, "attn.value.bias")), b.v, s));
            ENC_CUDA(rwq::launch_to_heads(b.q, D, 0, nwin, T, H, qscale, b.qh, s), "q heads");
            ENC_CUDA(rwq::launch_to_heads(b.k, D, 0, nwin, T, H, 1.0f, b.kh, s), "k heads");
            ENC_CUDA(rwq::launch_to_heads(b.v, D, 0, nwin, T, H, 1.0f, b.vh, s), "v heads");
        }
        // attention output rows quantized by the attention kernel itself
        ENC_CUDA(rwq::launch_attention(b.qh, b.kh, b.vh, nwin, T, H, b.att, s, aD.q16, aD.dT, aD.uT, m_pad),
                 "attention");
        ENC_RC(rwq::gemm_quantized(aD, L.o, W(lname(l, "attn.out.bias")), b.tmp, s));
        ENC_CUDA(rwq::launch_rows_quant(rwq::RQ_ADD_LN, b.x, b.tmp, b.x, W(lname(l, "mlp_ln.weight")),
                                        W(lname(l, "mlp_ln.bias")), M, D, m_pad, aD.q16, aD.dT, aD.uT, nullptr, s),
                 "mlp_ln");
        if (rwq::gemm_gelu_quantized_fits(aD, L.fc1, aH)) {
            // fc1 with GELU and the quantizer in its epilogue, into fc2's
            // operand (carved from b.h, which the f32 output would use)
            ENC_RC(rwq::gemm_gelu_quantized(aD, L.fc1, W(lname(l, "mlp.0.bias")), aH, s));
            ENC_RC(rwq::gemm_quantized(aH, L.fc2, W(lname(l, "mlp.2.bias")), b.tmp, s));
        } else {
            ENC_RC(rwq::gemm_quantized(aD, L.fc1, W(lname(l, "mlp.0.bias")), b.h, s));
            ENC_CUDA(rwq::launch_rows_quant(rwq::RQ_GELU, b.h, nullptr, nullptr, nullptr, nullptr, M, F, m_pad,
                                            aF.q16, aF.dT, aF.uT, nullptr, s),
                     "gelu quantize");
            ENC_RC(rwq::gemm_quantized(aF, L.fc2, W(lname(l, "mlp.2.bias")), b.tmp, s));
        }
    }
    // [x += last mlp out;] ln_post -> out
    ENC_CUDA(rwq::launch_rows_quant(e->n_layer ? rwq::RQ_ADD_LN : rwq::RQ_LN, b.x, b.tmp, b.x,
                                    W("encoder.ln_post.weight"), W("encoder.ln_post.bias"), M, D, m_pad, nullptr,
                                    nullptr, nullptr, out, s),
             "ln_post");
    return RWQ_OK;
}

// Windows per pass through the workspace: bounded so that one pass stays
// within a few GB.
int max_windows_per_pass(const rwq_encoder* e) {
    const size_t per = carve(e, 1, nullptr, nullptr);
    size_t n = (size_t(6) << 30) / (per ? per : 1);
    return int(n < 1 ? 1 : (n > 64 ? 64 : n));
}

}  // namespace

extern "C" {

int rwq_encoder_new(int n_mels, int n_ctx, int n_state, int n_head, int n_layer, rwq_encoder** out) {
    if (!out) return efail(RWQ_ERR_ARG, "out is null");
    *out = nullptr;
    if (n_mels <= 0 || n_ctx <= 0 || n_state <= 0 || n_head <= 0 || n_layer < 0)
        return efail(RWQ_ERR_ARG, "bad encoder shape");
    if (n_state % n_head || n_state / n_head != 64)
        return efail(RWQ_ERR_ARG, "head dim must be 64 (n_state %d, n_head %d)", n_state, n_head);
    if (n_state % 128) return efail(RWQ_ERR_ARG, "n_state must be a multiple of 128 (got %d)", n_state);
    auto* e = new rwq_encoder;
    cudaGetDevice(&e->device);
    e->n_mels = n_mels;
    e->n_ctx = n_ctx;
    e->n_state = n_state;
    e->n_head = n_head;
    e->n_layer = n_layer;
    e->n_ff = 4 * n_state;
    e->layers.resize(size_t(n_layer));
    expected_dense(e);
    *out = e;
    return RWQ_OK;
}

int rwq_encoder_free(rwq_encoder* e) {
    if (!e) return RWQ_OK;
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != e->device) cudaSetDevice(e->device);
    for (auto& kv : e->dense) cudaFree(kv.second);
    for (auto& L : e->layers)
        for (rwq_qtensor* t : {L.q, L.k, L.v, L.o, L.fc1, L.fc2}) rwq_qtensor_free(t);
    cudaFree(e->ws);
    for (void* p : {static_cast<void*>(e->conv1_hl), static_cast<void*>(e->conv2_hl), static_cast<void*>(e->conv1_cs),
                    static_cast<void*>(e->conv2_cs)})
        cudaFree(p);
    if (prev != e->device) cudaSetDevice(prev);
    delete e;
    return RWQ_OK;
}

int rwq_encoder_set_dense(rwq_encoder* e, const char* name, const float* data, int64_t count) {
    if (!e || !name || !data) return efail(RWQ_ERR_ARG, "null argument");
    std::lock_guard<std::mutex> g(e->mu);
    auto it = e->dense_len.find(name);
    if (it == e->dense_len.end()) return efail(RWQ_ERR_ARG, "'%s' is not a dense encoder tensor", name);
    if (count < 0 || size_t(count) != it->second)
        return efail(RWQ_ERR_SHAPE, "'%s': %lld elements, expected %zu", name, (long long)count, it->second);
    float*& dst = e->dense[name];
    if (!dst) ENC_CUDA(cudaMalloc(&dst, it->second * 4), "cudaMalloc(dense tensor)");
    ENC_CUDA(cudaMemcpy(dst, data, it->second * 4, cudaMemcpyHostToDevice), "copy dense tensor");
    if (std::strncmp(name, "encoder.conv", 12) == 0) e->stem_ready = false;   // re-split at the next encode
    return RWQ_OK;
}

int rwq_conv1d_dev(const float* x, int64_t n_win, int64_t in_ch, int64_t t_in, const float* w, int64_t out_ch,
                   const float* bias, int stride, float* out, void* stream) {
    if (n_win < 0 || in_ch <= 0 || t_in <= 0 || out_ch <= 0 || (stride != 1 && stride != 2))
        return efail(RWQ_ERR_ARG, "conv1d: bad shape (windows %lld, in %lld, t %lld, out %lld, stride %d)",
                     (long long)n_win, (long long)in_ch, (long long)t_in, (long long)out_ch, stride);
    if (in_ch > (1 << 20) || out_ch > (1 << 20) || t_in > (1 << 24)) return efail(RWQ_ERR_ARG, "conv1d: too large");
    if (n_win == 0) return RWQ_OK;
    if (!x || !w || !out) return efail(RWQ_ERR_ARG, "conv1d: null pointer");
    const int64_t t_out = (t_in - 1) / stride + 1, rows = n_win * t_out;
    if (rows > INT32_MAX) return efail(RWQ_ERR_ARG, "conv1d: too many output rows");
    const int kp = int((3 * in_ch + 31) / 32 * 32), n_pad = int((out_ch + 255) / 256 * 256);
    const size_t a_b = align_up(size_t(rows) * kp * 4, 256), r_b = align_up(size_t(rows) * 4, 256),
                 b_b = align_up(size_t(out_ch) * kp * 4, 256), c_b = align_up(size_t(n_pad) * 4, 256);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return rwq::with_stream_scratch(s, a_b + r_b + b_b + c_b, [&](void* buf) {
        uint8_t* p = static_cast<uint8_t*>(buf);
        uint16_t* ahl = reinterpret_cast<uint16_t*>(p);
        float* rs = reinterpret_cast<float*>(p + a_b);
        uint16_t* bhl = reinterpret_cast<uint16_t*>(p + a_b + r_b);
        float* cs = reinterpret_cast<float*>(p + a_b + r_b + b_b);
        ENC_CUDA(rwq::launch_split_dense(w, int(out_ch), kp, int(3 * in_ch), int(3 * in_ch), n_pad, bhl, cs, s),
                 "split conv weights");
        ENC_CUDA(rwq::launch_im2col_split(x, int(n_win), int(in_ch), int(t_in), int(t_out), stride,
                                          size_t(in_ch) * t_in, size_t(t_in), 1, kp, ahl, rs, s),
                 "im2col");
        return rwq::gemm_hl(ahl, rs, int(rows), bhl, cs, int(out_ch), kp / rwq::QK, bias, out, s);
    });
}

int rwq_encoder_set_quant(rwq_encoder* e, const char* name, int dtype, const uint8_t* raw, size_t raw_len, int64_t n,
                          int64_t k) {
    if (!e || !name) return efail(RWQ_ERR_ARG, "null argument");
    std::lock_guard<std::mutex> g(e->mu);
    int64_t wn = 0, wk = 0;
    rwq_qtensor** slot = quant_slot(e, name, &wn, &wk);
    if (!slot) return efail(RWQ_ERR_ARG, "'%s' is not a quantized encoder linear", name);
    if (n != wn || k != wk)
        return efail(RWQ_ERR_SHAPE, "'%s': [%lld, %lld], expected [%lld, %lld]", name, (long long)n, (long long)k,
                     (long long)wn, (long long)wk);
    rwq_qtensor* t = nullptr;
    ENC_RC(rwq_qtensor_new(raw, raw_len, dtype, n, k, &t));
    rwq_qtensor_free(*slot);
    *slot = t;
    return RWQ_OK;
}

int rwq_encoder_encode_dev(rwq_encoder* e, const float* mel, int64_t n_windows, float* out, void* stream) {
    if (!e) return efail(RWQ_ERR_ARG, "encoder is null");
    if (n_windows < 0) return efail(RWQ_ERR_ARG, "negative window count");
    if (n_windows == 0) return RWQ_OK;
    if (!mel || !out) return efail(RWQ_ERR_ARG, "null mel or output pointer");
    if ((reinterpret_cast<uintptr_t>(mel) | reinterpret_cast<uintptr_t>(out)) & 15)
        return efail(RWQ_ERR_ARG, "mel and output must be 16-byte aligned");
    std::lock_guard<std::mutex> g(e->mu);
    ENC_RC(check_ready(e));
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev != e->device) return efail(RWQ_ERR_ARG, "encoder lives on device %d, current device is %d", e->device, dev);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int per = max_windows_per_pass(e);
    const int first = int(n_windows < per ? n_windows : per);
    const size_t need = carve(e, first, nullptr, nullptr);
    if (e->ws_bytes < need) {
        ENC_CUDA(cudaStreamSynchronize(s), "cudaStreamSynchronize");
        cudaFree(e->ws);
        e->ws = nullptr;
        e->ws_bytes = 0;
        ENC_CUDA(cudaMalloc(&e->ws, need), "cudaMalloc(encoder workspace)");
        e->ws_bytes = need;
    }
    const size_t in_per = size_t(e->n_mels) * 2 * e->n_ctx, out_per = size_t(e->n_ctx) * e->n_state;
    for (int64_t w0 = 0; w0 < n_windows; w0 += per) {
        const int nw = int(n_windows - w0 < per ? n_windows - w0 : per);
        Bufs b;
        carve(e, nw, static_cast<uint8_t*>(e->ws), &b);
        ENC_RC(encode_batch(e, b, mel + size_t(w0) * in_per, nw, out + size_t(w0) * out_per, s));
    }
    return RWQ_OK;
}

int rwq_encoder_encode(rwq_encoder* e, const float* mel, int64_t n_windows, float* out) {
    if (!e) return efail(RWQ_ERR_ARG, "encoder is null");
    if (n_windows <= 0) return n_windows == 0 ? RWQ_OK : efail(RWQ_ERR_ARG, "negative window count");
    if (!mel || !out) return efail(RWQ_ERR_ARG, "null mel or output pointer");
    const size_t in_b = size_t(n_windows) * e->n_mels * 2 * e->n_ctx * 4;
    const size_t out_b = size_t(n_windows) * e->n_ctx * e->n_state * 4;
    float *dm = nullptr, *dout = nullptr;
    cudaStream_t s = nullptr;
    ENC_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
    int rc = RWQ_OK;
    auto done = [&](int code) {
        cudaFree(dm);
        cudaFree(dout);
        cudaStreamDestroy(s);
        return code;
    };
    cudaError_t ce = cudaMalloc(&dm, in_b);
    if (ce == cudaSuccess) ce = cudaMalloc(&dout, out_b);
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(dm, mel, in_b, cudaMemcpyHostToDevice, s);
    if (ce != cudaSuccess) return done(efail(RWQ_ERR_CUDA, "encoder host copies: %s", cudaGetErrorString(ce)));
    if ((rc = rwq_encoder_encode_dev(e, dm, n_windows, dout, s))) return done(rc);
    ce = cudaMemcpyAsync(out, dout, out_b, cudaMemcpyDeviceToHost, s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
    if (ce != cudaSuccess) return done(efail(RWQ_ERR_CUDA, "encoder: %s", cudaGetErrorString(ce)));
    if ((rc = rwq_stream_check(s))) return done(rc);
    return done(RWQ_OK);
}

int rwq_attention_dev(const float* q, const float* k, const float* v, int64_t n_windows, int64_t t, int64_t n_state,
                      int64_t n_head, float* out, void* stream) {
    if (n_windows < 0 || t < 0 || n_head <= 0 || n_state <= 0) return efail(RWQ_ERR_ARG, "bad attention shape");
    if (n_state % n_head || n_state / n_head != 64) return efail(RWQ_ERR_ARG, "head dim must be 64");
    if (n_windows == 0 || t == 0) return RWQ_OK;
    if (!q || !k || !v || !out) return efail(RWQ_ERR_ARG, "null pointer");
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v) |
         reinterpret_cast<uintptr_t>(out)) & 15)
        return efail(RWQ_ERR_ARG, "attention operands must be 16-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t per = align_up(size_t(n_windows) * t * n_state * 2, 256);
    const int W = int(n_windows), T = int(t), D = int(n_state), H = int(n_head);
    return rwq::with_stream_scratch(s, 3 * per, [&](void* buf) {
        __half* qh = static_cast<__half*>(buf);
        __half* kh = reinterpret_cast<__half*>(static_cast<uint8_t*>(buf) + per);
        __half* vh = reinterpret_cast<__half*>(static_cast<uint8_t*>(buf) + 2 * per);
        ENC_CUDA(rwq::launch_to_heads(q, D, 0, W, T, H, 1.0f / std::sqrt(64.0f), qh, s), "q heads");
        ENC_CUDA(rwq::launch_to_heads(k, D, 0, W, T, H, 1.0f, kh, s), "k heads");
        ENC_CUDA(rwq::launch_to_heads(v, D, 0, W, T, H, 1.0f, vh, s), "v heads");
        ENC_CUDA(rwq::launch_attention(qh, kh, vh, W, T, H, out, s), "attention");
        return int(RWQ_OK);
    });
}

int rwq_layer_norm_dev(const float* x, const float* add, float* x_out, const float* weight, const float* bias,
                       int64_t m, int64_t k, float* y, int8_t* q, float* d, int32_t* sum, void* stream) {
    if (m < 0 || k <= 0 || k % 128 || k > 2048) return efail(RWQ_ERR_ARG, "bad shape (k %% 128 == 0, k <= 2048)");
    if (m > INT32_MAX / k) return efail(RWQ_ERR_ARG, "too many rows");
    if (m == 0) return RWQ_OK;
    if (!x || !weight || !bias || (add && !x_out)) return efail(RWQ_ERR_ARG, "null pointer");
    if (!y && !q) return efail(RWQ_ERR_ARG, "no output (y and q both NULL)");
    if (q && (!d || !sum)) return efail(RWQ_ERR_ARG, "q, d and sum go together");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(add) | reinterpret_cast<uintptr_t>(x_out) |
         reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(weight) | reinterpret_cast<uintptr_t>(bias)) &
        15)
        return efail(RWQ_ERR_ARG, "layer_norm operands must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(q) & 3) return efail(RWQ_ERR_ARG, "q must be 4-byte aligned");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int mode = add ? rwq::RQ_ADD_LN : rwq::RQ_LN;
    const int M = int(m), K = int(k);
    if (!q) {
        ENC_CUDA(rwq::launch_rows_quant_v(mode, x, add, x_out, weight, bias, M, K, nullptr, nullptr, y, s),
                 "layer_norm");
        return RWQ_OK;
    }
    return rwq::with_stream_scratch(s, size_t(m) * (k / 32) * 4, [&](void* buf) {
        rwq::ActsView v;
        v.m = M;
        v.k = K;
        v.nb = K / 32;
        v.m_pad = M;
        v.q8 = q;
        v.d = d;
        v.sum = sum;
        v.u = static_cast<float*>(buf);
        ENC_CUDA(rwq::launch_rows_quant_v(mode, x, add, x_out, weight, bias, M, K, nullptr, &v, y, s), "layer_norm");
        return int(RWQ_OK);
    });
}

}  // extern "C"
