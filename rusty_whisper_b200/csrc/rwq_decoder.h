// rwq_decoder.h -- internal declarations of the decoder step's kernels
// (rwq_decoder_kernels.cu, rwq_kernels.cu).  Not part of the public C ABI.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include "rwq_internal.h"

namespace rwq {

constexpr int DEC_MAX_G = 8;   // streams sharing one key group in k_attn_dec

// The decode position lives on the device (*dpos), so a step replays from
// a CUDA graph.
// k_new / v_new rows are ld floats apart.
cudaError_t launch_kv_append(const float* k_new, const float* v_new, int ld, int S, int H, int ctx, const int* dpos,
                             __half* kc, __half* vc, cudaStream_t s);
cudaError_t launch_pos_advance(int* dpos, cudaStream_t s);
// Attention of one query per stream (q [S][H*64] f32) over n_groups
// groups: group g's keys/values are kc/vc + (grp_kv[g]*H + h)*kv_stride,
// f16 [L][64]; its streams are grp_streams[grp_off[g] .. grp_off[g+1])
// (<= max_group <= DEC_MAX_G).  Device arrays.  With dpos the keys are 0..*dpos
// (self-attention over the cache; L is then the capacity).
// With qout the output rows go straight to the int8 GEMV layout (codes
// [S][D], d / sum / d*sum [S][D/32], as k_rows_quant writes them; out is
// then unused).
struct AttnQuantOut {
    int8_t* q8 = nullptr;
    float* d = nullptr;
    int32_t* sum = nullptr;
    float* u = nullptr;
};
// Runs on the tensor cores (k_attn_dec_tc; RWQ_ATTN_TC=0 keeps
// single-stream groups on the CUDA-core k_attn_dec); splits > 1
// (those groups only) divides the keys over that many CTAs per (head,
// group): part then holds n_groups * splits * H * DEC_MAX_G * 66 floats
// and cnt n_groups * H zeroed counters (left zeroed).
cudaError_t launch_attn_dec(const float* q, const __half* kc, const __half* vc, size_t kv_stride, int L,
                            const int* dpos, int H, int n_groups, int max_group, const int* grp_kv, const int* grp_off,
                            const int* grp_streams, float* out, int splits, float* part, unsigned* cnt, int ldq,
                            const AttnQuantOut* qout, cudaStream_t s);
// Whether launch_attn_dec takes qout for groups of this size (the
// tensor-core kernel; not the CUDA-core one that RWQ_ATTN_TC=0 selects).
bool attn_dec_quantizes(int max_group);
// Key splits for a grid of H x n_groups CTAs: 1 for single-stream groups,
// else enough for one CTA per SM, at most 8 splits of at least 128 keys.
int attn_dec_splits(int H, int n_groups, int max_group, int L, int sms);
cudaError_t launch_argmax(const float* logits, int rows, int V, int limit, int32_t* best, cudaStream_t s);
// Decoder::fork for a beam step (rwq_beam.cu): stream i's self-attention
// cache [layer][S][H][ctx][64] (both K and V, positions 0 .. *dpos) takes
// stream src[i]'s, for src[i] != i in the same window (win[]) whose own
// src is itself; other entries are left alone.  Device arrays.
cudaError_t launch_self_fork(const int32_t* src, const int32_t* win, int S, int H, int ctx, int n_layer,
                             const int* dpos, __half* kc, __half* vc, cudaStream_t s);
// x[i] = dequant(w row tokens[i]) + pos[*dpos] (bit-exact dequant,
// quant.rs:528-537); pos is [ctx][k].
cudaError_t launch_embed(const Weight& w, const int32_t* tokens, int n, const float* pos, const int* dpos, float* x,
                         cudaStream_t s);

}  // namespace rwq
