// rwq_encoder.h -- internal declarations of the encoder forward's kernels
// (rwq_encoder_kernels.cu) and the quantized-GEMM hook the encoder uses
// (rwq_api.cu).  Not part of the public C ABI (include/rwq.h).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include <functional>
#include "rwq_internal.h"

struct rwq_qtensor;

namespace rwq {

// Row transforms in front of the int8 quantizer (k_rows_quant).
enum RowQuantMode : int { RQ_PLAIN = 0, RQ_GELU = 1, RQ_LN = 2, RQ_ADD_LN = 3 };

cudaError_t launch_rows_quant(int mode, const float* x, const float* add, float* xout, const float* lw,
                              const float* lb, int m, int k, int m_pad, uint16_t* q16, float* dT, float* uT,
                              float* yout, cudaStream_t s);
// Same with the codes going to the GEMM layout (`gemm`: q16, dT, uT,
// m_pad), the GEMV layout (`gemv`: q8, d, sum, u), or both.
cudaError_t launch_rows_quant_v(int mode, const float* x, const float* add, float* xout, const float* lw,
                                const float* lb, int m, int k, const ActsView* gemm, const ActsView* gemv,
                                float* yout, cudaStream_t s);
cudaError_t launch_to_heads(const float* src, int ld, int col0, int n_win, int T, int H, float scale, __half* dst,
                            cudaStream_t s);
// With q16 set, the output rows go quantized into that GEMM-layout operand
// (q16 [n_win*T][H*64], dT and uT [H*2][m_pad]) instead of f32 into `out`.
cudaError_t launch_attention(const __half* Qh, const __half* Kh, const __half* Vh, int n_win, int T, int H,
                             float* out, cudaStream_t s, uint16_t* q16 = nullptr, float* dT = nullptr,
                             float* uT = nullptr, int m_pad = 0);

// The tensor-core GEMM on activations already quantized into `v` (GEMM
// layout): out = A W^T (+ bias).  Builds the weight's operand cache on
// first use.  Returns an RWQ_* status (error text set).
int gemm_quantized(const ActsView& v, rwq_qtensor* w, const float* bias, float* out, cudaStream_t s);

// Same GEMM with GELU and the int8 quantizer fused into its epilogue: the
// output goes straight into `out`'s GEMM-layout operand (q16, dT, uT) for
// the next GEMM (the encoder's fc1 -> fc2).  `out` must not share memory
// with `v`.  gemm_gelu_quantized_fits says whether this call can run
// fused (w.n a multiple of 256, the default tensor-core path); otherwise
// the caller runs gemm_quantized and the GELU row kernel.
bool gemm_gelu_quantized_fits(const ActsView& v, rwq_qtensor* w, const ActsView& out);
// Same GEMM writing f16 attention heads [n_win][H][T][64] of (A W^T + bias)
// * scale directly (the encoder's Q, K and V: no f32 output, no
// launch_to_heads); the _fits predicate as above (w.n == H * 64, a multiple
// of 256).
bool gemm_heads_fits(const ActsView& v, rwq_qtensor* w, int n_win, int T, int H, const __half* dst);
int gemm_heads(const ActsView& v, rwq_qtensor* w, const float* bias, __half* dst, int n_win, int T, int H, float scale,
               cudaStream_t s);
int gemm_gelu_quantized(const ActsView& v, rwq_qtensor* w, const float* bias, const ActsView& out, cudaStream_t s);

// Same on either layout: `gemm` false reads the GEMV layout (q8, d, sum, u;
// integer-MMA GEMV in chunks of 8 rows), true the GEMM layout.
int linear_acts(const ActsView& v, bool gemm, rwq_qtensor* w, const float* bias, float* out, cudaStream_t s);

// k_gemm_hl on prepared hi|lo operands (launch_split_rows /
// launch_im2col_split for A, launch_split_dense for a dense B), with this
// stream's fault flag.  Returns an RWQ_* status.
int gemm_hl(const uint16_t* ahl, const float* rowscale, int m, const uint16_t* bhl, const float* colscale, int n,
            int nb, const float* bias, float* out, cudaStream_t s, const HlEpilogue* epi = nullptr);

// The GEMM kernel path that GEMM-sized matmuls take on this host thread
// (2 folded-scale, 3 exact-integer, 4 hi|lo; rwq_set_gemm_path), which
// decides the activation layout (LAYOUT_FOLD or LAYOUT_HL) callers prepare.
int gemm_path();

// Run `fn` with this stream's scratch arena (at least `bytes`), holding
// its lock.  Returns fn's status (or an RWQ_* error).
int with_stream_scratch(cudaStream_t s, size_t bytes, const std::function<int(void*)>& fn);

}  // namespace rwq
