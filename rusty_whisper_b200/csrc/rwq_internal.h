// rwq_internal.h -- declarations shared by the library's translation units.
// Not part of the public C ABI (that is include/rwq.h).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace rwq {

// Device-resident weight: the "planes" layout of rwq_common.cuh plus the
// lazily built tensor-core operand cache.
struct Weight {
    int dtype = 0, n = 0, k = 0, nb = 0, device = 0;
    uint8_t* qs = nullptr;     // [n][nb4/4][4*qs_bytes], word-interleaved groups (rwq_common.cuh)
    uint32_t* qh = nullptr;    // [n][nb4]         (Q5_0 / Q5_1)
    uint16_t* d = nullptr;     // [n][nb4] f16 bits
    uint16_t* m = nullptr;     // [n][nb4] f16 bits (Q4_1 / Q5_1)
    // tensor-core operand cache (built on first GEMM-sized call)
    uint16_t* q16 = nullptr;   // [n][k] centred codes as f16
    float* dT = nullptr;       // [nb][n_pad] d as f32, transposed
    float* mT = nullptr;       // [nb][n_pad] m as f32, transposed (min formats)
    int n_pad = 0;
    bool gemm_ready = false;
    // folded-scale tensor-core operand (built on first use): per row and
    // block, 32 f16 "hi" then 32 f16 "lo" of x*2^e_j (x = d*q + m), and
    // colscale[j] = 2^-e_j ([n_pad], zero padded).
    uint16_t* bhl = nullptr;   // [n][nb][64]
    float* colscale = nullptr;
    bool fold_ready = false;
    // TMA descriptors (CUtensorMap, 128 bytes each) of the qs, qh, d and m
    // planes for k_gemv_rows, encoded when the weight is created;
    // rows_ready is false where the plane layout does not allow them.
    alignas(64) unsigned char row_maps[4][128] = {};
    bool rows_ready = false;
};

// Scratch for one activation quantization (quantize_acts_i8 output).
struct ActsView {
    int m = 0, k = 0, nb = 0, m_pad = 0;
    int8_t* q8 = nullptr;      // [m][k]        GEMV operand
    float* d = nullptr;        // [m][nb]       d_a
    int32_t* sum = nullptr;    // [m][nb]       sum(q_a)
    float* u = nullptr;        // [m][nb]       d_a * sum(q_a)
    uint16_t* q16 = nullptr;   // [m][k] f16    GEMM operand (optional)
    float* dT = nullptr;       // [nb][m_pad]   (optional)
    float* uT = nullptr;       // [nb][m_pad]   (optional)
    // hi|lo operand of k_gemm_hl (optional): per row and block 32 f16 hi
    // then 32 f16 lo of a'*2^e_i (a' = d_a*q_a, or the f32 activation in
    // f32 mode), rowscale[i] = 2^-e_i.
    uint16_t* ahl = nullptr;   // [m][nb][64]
    float* rowscale = nullptr; // [m]
};

// Operand layouts of a quantized activation matrix.
enum ActsLayout : int {
    LAYOUT_GEMV = 0,   // q8, d, sum, u
    LAYOUT_FOLD = 1,   // d, sum, u, q16, dT, uT (k_gemm_fold, k_gemm_tc)
    LAYOUT_HL = 2      // ahl, rowscale (k_gemm_hl)
};

// ---- launchers (return a cudaError_t of the launch) ----
cudaError_t launch_repack(const uint8_t* raw, Weight& w, cudaStream_t s);
cudaError_t launch_build_gemm_cache(Weight& w, cudaStream_t s);
cudaError_t launch_build_fold_cache(Weight& w, cudaStream_t s);
cudaError_t launch_quantize_acts(const float* a, const ActsView& v, bool want_gemm, cudaStream_t s);
cudaError_t launch_dequant_rows(const Weight& w, const int32_t* rows, int nrows, float* out, cudaStream_t s);
cudaError_t launch_block_dots(const ActsView& v, const Weight& w, int32_t* S, cudaStream_t s);
// err_flag (may be null) receives a code if a bounded wait of k_gemv_rows
// expires.
cudaError_t launch_gemv_i8(const ActsView& v, const Weight& w, const float* bias, float* y, cudaStream_t s,
                           int* err_flag = nullptr);
// GEMV kernel choice for the calling host thread: 0 auto, 1 dp4a, 2
// integer MMA, 3 tiled integer MMA, 4 row-per-lane TMA kernel.
void set_gemv_kind(int kind);
// The kernel (1-4) launch_gemv_i8 runs for m rows on w with aligned codes.
int gemv_kernel_for(const Weight& w, int m);
// The row-per-lane GEMV (k_gemv_rows, one or two activation rows, weights
// that k_gemv_mma runs without a K split): encode the plane descriptors
// at weight creation; whether it can run these activations; the launch
// (gx = k_gemv_mma's grid, whose tile split it reproduces).
void prepare_gemv_rows(Weight& w);
constexpr int GEMV_ROWS_MAX_M = 2;
bool gemv_rows_fits(const ActsView& v, const Weight& w);
cudaError_t launch_gemv_rows(const ActsView& v, const Weight& w, const float* bias, float* y, int gx,
                             int* err_flag, cudaStream_t s);
cudaError_t launch_gemv_f32(const float* a, int m, const Weight& w, const float* bias, float* y, cudaStream_t s);
// tcgen05 GEMM.  S_dump (optional, small shapes) receives the per-block
// integer dots read back from tensor memory.
cudaError_t launch_gemm_tc(const ActsView& v, const Weight& w, const float* bias, float* y, int32_t* S_dump,
                           int* err_flag, cudaStream_t s, char* why, size_t why_len);

// tcgen05 GEMM with the weight scales folded into the B operand.
cudaError_t launch_gemm_fold(const ActsView& v, const Weight& w, const float* bias, float* y, int* err_flag,
                             cudaStream_t s, char* why, size_t why_len);
// k_gemm_fold on 128 x 256 tiles whose epilogue applies GELU to y (with
// bias) and quantizes it, per 32-column block as the reference's int8
// quantizer does, straight into `out`'s GEMM-layout operand (q16, dT, uT;
// out.k == w.n, a multiple of 256): the encoder's fc1 without its f32
// output and the row kernel that would read it back.
bool gemm_fold_gelu_fits(const ActsView& v, const Weight& w, const ActsView& out);
cudaError_t launch_gemm_fold_gelu(const ActsView& v, const Weight& w, const float* bias, const ActsView& out,
                                  int* err_flag, cudaStream_t s, char* why, size_t why_len);
// k_gemm_fold on 128 x 256 tiles writing f16 attention heads
// [n_win][H][T][64] of y * scale (v.m == n_win * T, w.n == H * 64, a
// multiple of 256): the encoder's Q, K and V projections without their f32
// outputs and the conversion kernel that would read them back.
bool gemm_fold_heads_fits(const ActsView& v, const Weight& w, int n_win, int T, int H, const __half* dst);
cudaError_t launch_gemm_fold_heads(const ActsView& v, const Weight& w, const float* bias, __half* dst, int n_win,
                                   int T, int H, float scale, int* err_flag, cudaStream_t s, char* why,
                                   size_t why_len);
// The tile width k_gemm_fold picks for an m x n GEMM of nb blocks on the
// current device: 1 = 128- or 64-column tiles, 2 = 128 x 256 tiles.
int gemm_fold_config(int m, int n, int nb);
// Force that choice for this host thread (1 or 2; anything else:
// automatic).  The host-buffer entry point runs row chunks with the choice
// of the whole call.
void set_gemm_fold_config(int code);

// Rows of activations a[m][lda] (first k columns) into the hi|lo operand
// of k_gemm_hl: with `quantize` the reference's int8 quantizer runs first
// and the dequantized values d_a*q_a are split, else the f32 values.
cudaError_t launch_split_rows(const float* a, int m, int k, int lda, bool quantize, uint16_t* ahl, float* rowscale,
                              cudaStream_t s);
// Dense f32 weight rows w[n][ldw] (first kv columns, zeros up to k) into
// the hi|lo operand layout [n][k/32][64] with colscale[n_pad] (n_pad >=
// round4(n)).
cudaError_t launch_split_dense(const float* w, int n, int k, int kv, int ldw, int n_pad, uint16_t* bhl,
                               float* colscale, cudaStream_t s);
// im2col rows of a kernel-3, padding-1 conv1d straight into the hi|lo
// operand: n_win * t_out rows of kp columns (3*c_in used, then zeros),
// input element (w, c, t) at in[w*sw + c*sc + t*st].
cudaError_t launch_im2col_split(const float* in, int n_win, int c_in, int t_in, int t_out, int stride, size_t sw,
                                size_t sc, size_t st, int kp, uint16_t* ahl, float* rowscale, cudaStream_t s);
// Optional element-wise tail of k_gemm_hl's epilogue, after the bias:
// y = gelu(y) (tanh form) and then y += pos[(row % pos_period)][col] (pos
// has n columns) -- the conv stem's bias/GELU/position step.
struct HlEpilogue {
    bool gelu = false;
    const float* pos = nullptr;
    int pos_period = 1;
};
// y[m][n] = (A'*2^e_i)(B*2^e_j)^T * 2^-e_i * 2^-e_j (+ bias) on tcgen05 with
// both operands split into f16 hi + lo, the whole K accumulated in TMEM.
cudaError_t launch_gemm_hl(const uint16_t* ahl, const float* rowscale, int m, const uint16_t* bhl,
                           const float* colscale, int n, int nb, const float* bias, float* y, int* err_flag,
                           cudaStream_t s, char* why, size_t why_len, const HlEpilogue* epi = nullptr);
// The K split (1, 2 or 4 CTAs per output tile) k_gemm_hl picks for an
// m x n GEMM of nb blocks on the current device.
int gemm_hl_ksplit(int m, int n, int nb);
// Force the K split of this host thread's k_gemm_hl launches (1, 2 or 4;
// anything else: automatic).  The host-buffer entry point runs row chunks
// with the split of the whole call so that chunks give its bits.
void set_gemm_hl_ksplit(int S);

// The dp4a GEMV takes at most 8 activation rows per launch.
constexpr int GEMV_MAX_M = 8;
// Matmuls of up to this many rows take the GEMV family (the integer-MMA
// kernel, several launches of up to 64 rows that re-read the weights from
// L2); more rows take the tensor-core GEMM.
constexpr int GEMV_FAMILY_MAX_M = 256;
// Activation rows one integer-MMA GEMV launch takes for a weight of this
// dtype and k (64 unless the staging of 64 rows would not fit).
int gemv_rows_per_launch(int dtype, int k);

}  // namespace rwq

struct rwq_qtensor;
namespace rwq {
// The device weight behind a C-ABI handle (defined in rwq_api.cu).
const Weight& weight_of(const rwq_qtensor* t);
// A new weight holding the rows of `parts` in order (same dtype, k and
// device); status code as the C ABI.
int qtensor_concat_rows(rwq_qtensor* const* parts, int np, cudaStream_t s, rwq_qtensor** out);
// Set the text rwq_last_error() returns on this host thread.
void set_last_error(const char* msg);
}  // namespace rwq
