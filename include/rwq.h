/*
 * rwq.h -- C ABI of the B200 (sm_100a) quantized-matmul path that replaces
 * rusty_whisper's `quant::matmul_t_q` / `quant::linear_w`.
 *
 * Conventions (mirroring the crate's only C-ABI precedent, src/wasm.rs:25-111):
 *   - every entry point returns an int status: RWQ_OK (0) or a negative code;
 *   - the text of the last error is kept per host thread (rwq_last_error);
 *   - nothing aborts: bad shapes, bad dtypes and CUDA failures are statuses.
 * Matrices are row-major f32; a weight is ggml blocks, row-major [n][k/32]
 * (quant.rs:493-498), passed as the raw bytes a ggml/gguf loader holds.
 * `stream` is a cudaStream_t (NULL = the legacy default stream).  Calls on
 * one weight from several host threads are safe; calls that share a stream
 * are ordered by it.
 */
#ifndef RWQ_H
#define RWQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    RWQ_OK = 0,
    RWQ_ERR_ARG = -1,     /* null pointer, negative size, k % 32 != 0, ... */
    RWQ_ERR_DTYPE = -2,   /* not one of Q4_0/Q4_1/Q5_0/Q5_1/Q8_0 */
    RWQ_ERR_SHAPE = -3,   /* inner dimensions disagree */
    RWQ_ERR_CUDA = -4,    /* a CUDA call failed; see rwq_last_error() */
    RWQ_ERR_NOMEM = -5,   /* device or pinned allocation failed */
    RWQ_ERR_DEVICE = -6,  /* kernel reported a fault (bounded wait expired) */
    RWQ_ERR_NOGPU = -7    /* no usable sm_100 device */
};

/* ggml type codes (quant.rs:43-52). */
enum { RWQ_Q4_0 = 2, RWQ_Q4_1 = 3, RWQ_Q5_0 = 6, RWQ_Q5_1 = 7, RWQ_Q8_0 = 8 };

/* Arithmetic of a matmul:
 *   RWQ_MODE_INT8: activations quantized per 32-block to int8 and integer
 *     block dots, the tier rusty_whisper runs on every AVX2/VNNI host
 *     (quant.rs:763-994).
 *   RWQ_MODE_F32: weights dequantized, f32 dot with unquantized
 *     activations, the reference's f32 fallback (quant.rs:995-1018). */
enum { RWQ_MODE_INT8 = 0, RWQ_MODE_F32 = 1 };

typedef struct rwq_qtensor rwq_qtensor;

/* Bytes per 32-element block, or RWQ_ERR_DTYPE.  Replaces
 * `quant::block_bytes` (quant.rs:43). */
int rwq_block_bytes(int dtype);

/* Text of the last failure on this host thread ("" if none).  Mirrors the
 * thread-local error text of wasm.rs:18-21. */
const char* rwq_last_error(void);

/* Select the CUDA device for this host thread and check it is sm_100. */
int rwq_init(int device);

/* Upload an [n, k] ggml weight to the current device.  `raw` holds
 * n * (k/32) * rwq_block_bytes(dtype) bytes (host memory).  Replaces
 * `QTensor::new(shape, dtype, raw)` (quant.rs:553). */
int rwq_qtensor_new(const uint8_t* raw, size_t raw_len, int dtype, int64_t n, int64_t k, rwq_qtensor** out);

/* Same, from device memory already holding the raw blocks (e.g. a loader
 * that copied the file to the GPU). */
int rwq_qtensor_new_device(const void* raw_dev, size_t raw_len, int dtype, int64_t n, int64_t k, void* stream,
                           rwq_qtensor** out);

int rwq_qtensor_free(rwq_qtensor* t);
int rwq_qtensor_shape(const rwq_qtensor* t, int* dtype, int64_t* n, int64_t* k);

/* Build the tensor-core operand cache now rather than on the first
 * GEMM-sized call (the reference builds its int8 cache on the second call,
 * quant.rs:778-786). */
int rwq_qtensor_prepare_gemm(rwq_qtensor* t, void* stream);

/* C[m, n] = A[m, k] * dequant(B)^T (+ bias), host buffers: copies in,
 * computes, copies out, synchronizes.  Keeps the signature and ownership
 * of `matmul_t_q(a: &Tensor, b: &QTensor) -> Tensor` (quant.rs:754) and,
 * with `bias`, of `linear_w` (quant.rs:1054).  `bias` may be NULL. */
int rwq_matmul_t_q(const float* a, int64_t m, int64_t k, const rwq_qtensor* b, const float* bias, float* out,
                   int mode);

/* Device-pointer variant, asynchronous on `stream`: the perf path.
 * `a`, `bias`, `out` are device pointers (RWQ_MODE_F32 needs `a` 16-byte
 * aligned).  Scratch comes from a per-(device, stream) workspace owned by
 * the library. */
int rwq_matmul_t_q_dev(const float* a, int64_t m, int64_t k, const rwq_qtensor* b, const float* bias, float* out,
                       int mode, void* stream);

/* Activations quantized once and reused against several weights: the
 * reference quantizes inside every matmul_t_q call (quant.rs:766); a
 * caller that feeds one layernormed input to the Q, K and V projections
 * (encoder.rs:130-141) can quantize it once.  Results are identical to
 * rwq_matmul_t_q_dev on the same activations. */
typedef struct rwq_qacts rwq_qacts;
/* Device buffers for up to max_m rows of width k on the current device. */
int rwq_qacts_new(int64_t max_m, int64_t k, rwq_qacts** out);
int rwq_qacts_free(rwq_qacts* q);
/* Quantize a[m, k] (device f32) into q; m <= max_m. */
int rwq_qacts_quantize(rwq_qacts* q, const float* a, int64_t m, void* stream);
/* out[m, n] = (quantized a) * dequant(b)^T (+ bias), device pointers. */
int rwq_matmul_t_q_qacts(const rwq_qacts* q, const rwq_qtensor* b, const float* bias, float* out, void* stream);

/* Dequantize rows `rows[0..nrows)` (device int32 indices; NULL = rows
 * 0..nrows-1) into out[nrows, k] (device, 16-byte aligned), bit-identical to the
 * reference's scalar dequant.  Replaces `QTensor::row_f32` (quant.rs:566)
 * and, with rows = NULL and nrows = n, `to_dense` (quant.rs:572). */
int rwq_dequant_rows_dev(const rwq_qtensor* t, const int32_t* rows, int64_t nrows, float* out, void* stream);

/* Host-buffer gather of one row, `QTensor::row_f32` (quant.rs:566). */
int rwq_row_f32(const rwq_qtensor* t, int64_t row, float* out);

/* The int8 activation quantizer, `quantize_acts_i8` (quant.rs:690-716):
 * q[m, k] int8, d[m, k/32] f32, sum[m, k/32] int32; device pointers. */
int rwq_quantize_acts_dev(const float* a, int64_t m, int64_t k, int8_t* q, float* d, int32_t* sum, void* stream);

/* Per-block integer dots S[m][n][k/32] = sum q_a * q_b (centred weight
 * codes) of f32 activations a[m, k] (device pointers).  `path`
 * 0 = the CUDA-core dp4a core used by the GEMV, 1 = the tensor-core GEMM
 * (values read back from tensor memory).  For bit-exact tests of the
 * integer core; no reference counterpart beyond quant.rs:1352-1360. */
int rwq_block_dots_dev(const float* a, int64_t m, int64_t k, const rwq_qtensor* b, int32_t* S, int path,
                       void* stream);

/* Decoder-shaped int8 matmul that allocates no memory: out[m, n] =
 * A[m, k] * dequant(b)^T (+ bias) with m <= 8 and k <= 8192, device
 * pointers, asynchronous on `stream`.  It runs the quantizer and GEMV
 * kernels of rwq_matmul_t_q_dev (the same GEMV kind on the same host
 * thread), so the results are bit-identical to that entry point's.
 * No counterpart in the reference.  For callers that may not allocate GPU
 * memory: a live-microphone decode loop on a latency-critical thread
 * (cudaMalloc/cudaFree can stall on an implicit device synchronization),
 * or an embedder whose GPU memory belongs to another allocator.  Its
 * scratch (the quantized activations, 88 KiB) is a fixed array that every
 * GPU loading this library holds until exit.  The first call on a device
 * looks up that array's device address, which may make the driver load the
 * library's module on that device (a driver-side allocation that can
 * synchronize): make one warm-up call at initialisation, outside the
 * latency-critical loop and before any stream capture.  The address is
 * kept, so a cudaDeviceReset while the library is loaded is not supported.
 * All calls share the one array: calls that overlap on the GPU (other
 * streams, other host threads) race and must be ordered by the caller,
 * e.g. on one stream.  Larger m or k returns RWQ_ERR_ARG. */
int rwq_matmul_t_q_noalloc(const float* a, int64_t m, int64_t k, const rwq_qtensor* b, const float* bias,
                           float* out, void* stream);

/* Force the kernel family (testing and benchmarking): 0 = automatic
 * (GEMV family for m <= 256; above, path 2 for RWQ_MODE_INT8 and path 4
 * for RWQ_MODE_F32), 1 = GEMV family in row
 * chunks, 2 = tensor-core GEMM with the weight scales folded into the
 * operand and each block's partial sum scaled by d_a on the CUDA cores,
 * 3 = tensor-core GEMM that forms each block's integer dot exactly and
 * scales it on the CUDA cores, 4 = tensor-core GEMM with both operands
 * (dequantized activations d_a*q_a, or the f32 activations in
 * RWQ_MODE_F32, and the dequantized weights) split into f16 hi + lo and
 * the whole K accumulated in tensor memory (the f32 tier's kernel from
 * 257 rows).  Applies to this host thread. */
int rwq_set_gemm_path(int path);

/* Force the kernel of the GEMV family (m <= 256, or path 1 above) for
 * testing and benchmarking: 0 = automatic (kernels 4, 2 and 3 by m and
 * shape; they give identical bits, so a row's result does not depend on
 * m), 1 = dp4a kernel (one warp lane per block, lanes per row from k,
 * launches of 8 rows), 2 = integer-MMA kernel (mma.sync m16n8k32: one
 * instruction per block for 16 weight rows x 8 activation rows, up to 64
 * rows per launch sharing each decoded weight fragment), 3 = tiled
 * integer-MMA kernel (the same arithmetic tiled like a GEMM: 32-64 weight
 * rows x 32-64 activation rows per CTA, K streamed through shared memory;
 * automatic from 32 rows on), 4 = row-per-lane kernel (one weight row per
 * warp lane, dp4a block dots, the weight planes staged by TMA; automatic
 * at 1-2 rows on weights the integer-MMA kernel runs without a K split,
 * i.e. wide ones such as the logits projection; elsewhere kind 4 runs the
 * automatic choice).  All compute the reference's per-block formula
 * (quant.rs:349-351, :452-454) with exact integer block dots; 1 differs
 * from the others only in f32 summation order, 0, 2, 3 and 4 give
 * identical bits.  Applies to this host thread. */
int rwq_set_gemv_kernel(int kind);

/* The GEMV kernel (1-4 as above) this host thread's setting runs for an
 * m-row call on weight `w` (m <= 256), or a negative status. */
int rwq_gemv_kernel_for(const rwq_qtensor* w, int64_t m);

/* Synchronize `stream` and report any fault a kernel recorded on it. */
int rwq_stream_check(void* stream);

/* Dense tensor-core rate of the current device with the instructions the
 * GEMMs issue: `iters` back-to-back tcgen05 MMAs of 128 x 256 (K = 32 for
 * kind 0 = int8, K = 16 for kind 1 = f16) per CTA from shared memory into
 * tensor memory, `ctas` CTAs (<= 0: one per SM), timed with CUDA events on
 * the legacy stream after one shorter warm-up launch.  *tops = 2*M*N*K*
 * iters*ctas / time in 1e12 ops/s; *ms (may be NULL) = the timed launch.
 * A measurement aid for roofline denominators; no reference counterpart. */
int rwq_mma_peak(int kind, long long iters, int ctas, double* tops, double* ms);

/* ---- Model files ---------------------------------------------------------
 * Replace `model::load_model` (reference src/model.rs:145-275, legacy ggml
 * container) and `gguf::load` (src/gguf.rs:156-300, GGUF v2/v3), chosen by
 * the file's magic.  Parsing touches no GPU: hyper-parameters, the mel
 * filterbank, the vocabulary (padded with "[_extra_token_<i>]" to n_vocab)
 * and the tensors (f32; f16 widened to f32; quantized blocks kept verbatim).
 * A 2-D quantized tensor becomes a device weight the first time
 * rwq_model_qtensor asks for it (raw blocks uploaded unchanged, on the
 * current device); the model owns it.  Tensor shapes are row-major (the
 * reverse of ggml's ne[]), shape3 padded with 1s. */
typedef struct rwq_model rwq_model;

int rwq_model_load(const char* path, rwq_model** out);
int rwq_model_load_memory(const uint8_t* data, size_t len, rwq_model** out);
int rwq_model_free(rwq_model* m);
/* n_vocab, n_audio_ctx, n_audio_state, n_audio_head, n_audio_layer,
 * n_text_ctx, n_text_state, n_text_head, n_text_layer, n_mels, ftype
 * (the reference's HParams field order). */
int rwq_model_hparams(const rwq_model* m, int32_t* out11);
int rwq_model_mel_filters(const rwq_model* m, const float** data, int64_t* n_mel, int64_t* n_fft_bins);
int rwq_model_vocab_size(const rwq_model* m, int64_t* n);
int rwq_model_token(const rwq_model* m, int64_t id, const char** bytes, int64_t* len);
int rwq_model_n_tensors(const rwq_model* m, int64_t* n);
int rwq_model_find(const rwq_model* m, const char* name, int64_t* index);
int rwq_model_tensor(const rwq_model* m, int64_t i, const char** name, int* dtype, int* ndims, int64_t* shape3);
/* The raw ggml blocks of a quantized tensor (host memory owned by m). */
int rwq_model_tensor_raw(const rwq_model* m, int64_t i, const uint8_t** data, size_t* len);
/* Device weight of a 2-D quantized tensor (owned by m; do not free). */
int rwq_model_qtensor(rwq_model* m, int64_t i, rwq_qtensor** out);
/* Host f32 values of a dense tensor (f32/f16), or of a quantized tensor
 * of rank 1 or 3 (dequantized bit-exactly on the GPU on first call, like
 * the reference's load-time `to_dense`). */
int rwq_model_dense(rwq_model* m, int64_t i, const float** data, int64_t* n);

/* ---- Log-mel front end -----------------------------------------------
 * Replaces `audio::log_mel_spectrogram` (reference src/audio.rs:147-198):
 * periodic Hann window, 400-point FFT with hop 160 over the reflect-padded
 * signal, power, the mel filterbank, log10, then per window the clamp to
 * (max - 8) and (x + 4) / 4.  A plan holds a filterbank ([n_mels][201]
 * f32, host memory, e.g. from rwq_model_mel_filters or
 * rwq_mel_filterbank) prepared for the GPU. */
typedef struct rwq_mel rwq_mel;

/* `audio::mel_filterbank` (src/audio.rs:107-130) into out[n_mels][n_fft/2+1]. */
int rwq_mel_filterbank(int n_mels, int n_fft, int sample_rate, float* out);
int rwq_mel_new(const float* filters, int n_mels, rwq_mel** out);
int rwq_mel_free(rwq_mel* p);
/* Device buffers: samples [n_windows][n_samples] -> out
 * [n_windows][n_mels][n_samples / 160], each window normalised on its own
 * maximum; asynchronous on `stream`.  One plan serves one stream at a
 * time.  n_samples >= 201. */
int rwq_log_mel_dev(rwq_mel* p, const float* samples, int64_t n_windows, int64_t n_samples, float* out,
                    void* stream);
/* One window, host buffers (copies inside, synchronous). */
int rwq_log_mel(rwq_mel* p, const float* samples, int64_t n_samples, float* out);

/* ---- Encoder forward -----------------------------------------------------
 * Replaces `encoder::encode` (reference src/encoder.rs:180-234) for a batch
 * of 30 s windows, on the device: conv stem (k3 s1 then k3 s2, GELU),
 * positions, n_layer pre-LN blocks {attention, MLP}, ln_post, with every
 * block linear (`linear_w`, src/quant.rs:1054) on the quantized tensor-core
 * GEMM with int8 activation semantics.  Tensors are set by their
 * whisper.cpp names (those `encoder.rs` looks up), dense ones as f32
 * (conv weights [n_state][in][3], biases, LayerNorm, positions
 * [n_ctx][n_state]) and the six linears of each block as raw ggml blocks.
 * Head dim 64 and n_state % 128 == 0 (every Whisper size).  An encoder
 * serves one call at a time (its workspace is shared). */
typedef struct rwq_encoder rwq_encoder;

int rwq_encoder_new(int n_mels, int n_ctx, int n_state, int n_head, int n_layer, rwq_encoder** out);
int rwq_encoder_free(rwq_encoder* e);
int rwq_encoder_set_dense(rwq_encoder* e, const char* name, const float* data, int64_t count);
int rwq_encoder_set_quant(rwq_encoder* e, const char* name, int dtype, const uint8_t* raw, size_t raw_len, int64_t n,
                          int64_t k);
/* Device buffers: mel [n_windows][n_mels][2*n_ctx] -> out
 * [n_windows][n_ctx][n_state]; asynchronous on `stream`. */
int rwq_encoder_encode_dev(rwq_encoder* e, const float* mel, int64_t n_windows, float* out, void* stream);
/* Host buffers (copies inside, synchronous). */
int rwq_encoder_encode(rwq_encoder* e, const float* mel, int64_t n_windows, float* out);

/* `conv1d` with kernel 3 and padding 1 (tensor.rs:335-370, the encoder's
 * stem, encoder.rs:196-210) on the tensor cores: x [n_win][in_ch][t_in]
 * (each window channel-major, as the reference's input), w
 * [out_ch][in_ch][3], bias [out_ch] (may be NULL), stride 1 or 2; out
 * [n_win][t_out][out_ch], t_out = (t_in - 1) / stride + 1, is the
 * reference's [out_ch][t_out] result transposed to time-major (the layout
 * the encoder continues in, encoder.rs:215-220).  Both operands are split
 * into f16 hi + lo (about 22 significant bits each), so the sums match an
 * f32 conv to ~1e-6 of their scale.  Device buffers; scratch from this
 * stream's workspace. */
int rwq_conv1d_dev(const float* x, int64_t n_win, int64_t in_ch, int64_t t_in, const float* w, int64_t out_ch,
                   const float* bias, int stride, float* out, void* stream);

/* Non-causal multi-head attention over projected q, k, v
 * [n_windows][t][n_state] (`multi_head_attention`, src/encoder.rs:107-121,
 * with `mha_split_kv` :48-80): softmax(q k^T / 8) v per head of 64, on f16
 * tensor-core MMAs with f32 accumulation.  Device buffers, 16-byte aligned. */
int rwq_attention_dev(const float* q, const float* k, const float* v, int64_t n_windows, int64_t t, int64_t n_state,
                      int64_t n_head, float* out, void* stream);

/* The encoder's and decoder's row transform: with `add` non-NULL first
 * x_out = x + add (x_out may be x: the residual stream in place), then the
 * LayerNorm of each of the m rows of k (`layer_norm`, src/tensor.rs:274-289,
 * eps 1e-5) into y[m, k] and/or, quantized by `quantize_acts_i8`
 * (quant.rs:690-716), into q[m, k] int8, d[m, k/32] f32, sum[m, k/32]
 * int32 -- the operand the next quantized linear reads.  y or q may be
 * NULL (not both); q, d and sum go together.  k % 128 == 0; x, add, x_out,
 * y, weight and bias 16-byte aligned; device pointers.  A row's result is
 * the same bits whatever m is. */
int rwq_layer_norm_dev(const float* x, const float* add, float* x_out, const float* weight, const float* bias,
                       int64_t m, int64_t k, float* y, int8_t* q, float* d, int32_t* sum, void* stream);

/* ---- Decoder ---------------------------------------------------------------
 * Replaces the KV-cached `decoder::Decoder` (reference src/decoder.rs:36-321)
 * for S decode streams stepping in lockstep on the device.  A stream decodes
 * one window; streams of the same window (beams) share its cross K/V.
 * Tensors are set by their whisper.cpp names: dense f32 (LayerNorms,
 * biases, positional_embedding [n_text_ctx][n_state]) and raw ggml blocks
 * for the token embedding (also the tied logits matrix) and the ten
 * linears of each block.  Head dim 64, n_state % 128 == 0.  A decoder
 * serves one call at a time. */
typedef struct rwq_decoder rwq_decoder;

int rwq_decoder_new(int n_vocab, int n_text_ctx, int n_state, int n_head, int n_layer, rwq_decoder** out);
int rwq_decoder_free(rwq_decoder* d);
int rwq_decoder_set_dense(rwq_decoder* d, const char* name, const float* data, int64_t count);
int rwq_decoder_set_quant(rwq_decoder* d, const char* name, int dtype, const uint8_t* raw, size_t raw_len, int64_t n,
                          int64_t k);
/* `Decoder::new` for every stream (decoder.rs:36-69): cross K/V from the
 * windows' encoder outputs enc_out [n_windows][n_audio][n_state] (device),
 * stream i decoding window stream_window[i] (host array; NULL: stream i ->
 * window i), self caches cleared.  Asynchronous on `stream`. */
int rwq_decoder_begin(rwq_decoder* d, const float* enc_out, int64_t n_windows, int64_t n_audio,
                      const int32_t* stream_window, int64_t n_streams, void* stream);
/* One position for every stream (`forward(&[token])`, decoder.rs:102-206):
 * tokens [S] (device).  logits [S][n_vocab] (device, may be NULL) gets the
 * tied projection; best [S] (device, may be NULL) the greedy choice: the
 * first maximum over ids < limit if it beats logits[limit], else limit
 * (decoder.rs:345-365); limit < 0: the first maximum of the whole row.
 * With both NULL the projection is skipped (prompt positions).  A full
 * context (n_text_ctx positions) returns RWQ_ERR_ARG (decoder.rs:115-120). */
int rwq_decoder_step(rwq_decoder* d, const int32_t* tokens, float* logits, int32_t* best, int32_t limit, void* stream);
/* ---- Beam search on the device --------------------------------------
 * The pieces of one step of the reference's beam search (decode_window_beam,
 * transcribe.rs:835-1011), so a beam decode stays on the device between
 * steps: the beams of a window are its streams, stored contiguously
 * (stream w*B + b is beam b of window w: stream_window = [0]*B + [1]*B + ...
 * at rwq_decoder_begin).  The host policy around them (timestamp rules,
 * finished hypotheses, the final ranking) stays with the caller. */

/* `forward_hidden` (decoder.rs:110-206) for every stream: one position,
 * then the final layernorm; hidden [S][n_state] (device) receives the
 * states, no projection. */
int rwq_decoder_step_hidden(rwq_decoder* d, const int32_t* tokens, float* hidden, void* stream);

/* `project_logits` (decoder.rs:315-321): logits[rows][n_vocab] =
 * hidden[rows][n_state] . token_embedding^T as one stacked projection, as
 * the reference projects all beams at once (transcribe.rs:970-977).
 * rows <= the decoder's streams; device pointers, hidden 16-byte aligned.
 * The same bits as the projection inside rwq_decoder_step. */
int rwq_decoder_project(rwq_decoder* d, const float* hidden, int64_t rows, float* logits, void* stream);

/* `Decoder::fork` for a whole beam step (decoder.rs:71-79): stream i's
 * self-attention cache becomes stream src[i]'s (device array [S]).  Only
 * entries with src[i] != i, src[i] in i's window and src[src[i]] ==
 * src[i] (the source keeps its own history) are copied, in place; the
 * others are ignored.  rwq_beam_select's src always qualifies. */
int rwq_decoder_fork(rwq_decoder* d, const int32_t* src, void* stream);

/* log_softmax (transcribe.rs:482-486) and top_k (:672-685) of each row of
 * logits[rows][n_vocab] (device): ids >= limit are excluded like
 * suppressed tokens (limit < 0: none), -inf logits are never chosen; lp
 * [rows][k] descending with id [rows][k] (-1 / -inf past the choosable
 * ids); 1 <= k <= 8, rows <= 65535.  Ties in value are ordered by id. */
int rwq_beam_topk(const float* logits, int64_t rows, int64_t n_vocab, int32_t limit, int k, float* lp, int32_t* id,
                  void* stream);

/* The candidate ranking of one beam step for each of n_windows windows of
 * `beams` streams (transcribe.rs:890-925): the live beams (rank[s] <
 * n_live; rank NULL: slot order, used with n_live = 1 after the prompt)
 * each offer their k candidates (lp, id from rwq_beam_topk) scored
 * sum_lp[s] + max(lp, -30) (sum_lp NULL: 0); a stable sort by score in
 * the reference's beam order keeps the best `beams`.  Per slot s of the
 * window: src[s] the stream whose history it continues (for
 * rwq_decoder_fork), token[s], sum_out[s], step_lp[s] = max(lp, -30),
 * rank_out[s] its place in the ranking.  A survivor stays in its parent's
 * slot if it is that parent's first survivor, so only the others are
 * copied by rwq_decoder_fork.  All arrays device, [n_windows * beams]. */
int rwq_beam_select(const float* lp, const int32_t* id, int k, const float* sum_lp, const int32_t* rank,
                    int64_t n_windows, int beams, int n_live, int32_t* src, int32_t* token, float* sum_out,
                    float* step_lp, int32_t* rank_out, void* stream);

/* `Decoder::reset` (decoder.rs:83-91): positions restart at 0, cross K/V kept. */
int rwq_decoder_reset(rwq_decoder* d);
int rwq_decoder_n_past(const rwq_decoder* d, int64_t* n_past);

#ifdef __cplusplus
}
#endif
#endif /* RWQ_H */
