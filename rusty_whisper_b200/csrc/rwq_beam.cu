// rwq_beam.cu -- the per-step pieces of beam search on the device
// (reference decode_window_beam, transcribe.rs:835-1011), so a beam decode
// never returns to the host between steps:
//   * k_beam_topk: per stream, log_softmax of the logits (transcribe.rs:
//     482-486) and its top k (transcribe.rs:672-685);
//   * k_beam_select: per window, every live beam's k candidates scored
//     sum_lp + max(lp, -30), a stable sort by score, the best `beams`
//     kept (transcribe.rs:890-925), and each survivor given a stream slot;
//   * k_self_fork: `Decoder::fork` (decoder.rs:71-79) for the survivors,
//     copying self-attention caches between the slots.
// The reference clones a parent's whole self-attention cache for every
// surviving candidate.  Here a survivor whose parent has no other child
// already assigned stays in its parent's slot (its cache is already the
// right one), and only the others are copied, into slots that no
// survivor descends from, so the copies can run in place.
#include <cuda_runtime.h>
#include <cstdarg>
#include <cstdio>
#include "../../include/rwq.h"
#include "rwq_common.cuh"
#include "rwq_decoder.h"
#include "rwq_internal.h"

namespace rwq {
namespace {

constexpr int BEAM_MAX = 8;     // beams per window and candidates per beam
constexpr int TOPK_THREADS = 256;

// (v, i) ranks before (bv, bi): larger value first, then smaller id.
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

// One CTA per row.  Ids >= n are excluded (suppressed); -inf logits are
// never chosen (the reference skips lp == -inf); rows with fewer than k
// choosable ids get id -1 and lp -inf in the remaining places.
__global__ void __launch_bounds__(TOPK_THREADS) k_beam_topk(const float* __restrict__ logits, int V, int n, int k,
                                                          float* __restrict__ lp_out, int32_t* __restrict__ id_out) {
    pdl_trigger();
    pdl_wait();
    const float* row = logits + size_t(blockIdx.x) * V;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    __shared__ float s_red[TOPK_THREADS / 32];
    __shared__ float s_v[TOPK_THREADS * BEAM_MAX];
    __shared__ int s_i[TOPK_THREADS * BEAM_MAX];
    // max (NaN ignored, as f32::max folding from -inf)
    float mx = -INFINITY;
    for (int j = t; j < n; j += TOPK_THREADS) mx = fmaxf(mx, row[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) s_red[warp] = mx;
    __syncthreads();
    mx = s_red[0];
#pragma unroll
    for (int w = 1; w < TOPK_THREADS / 32; ++w) mx = fmaxf(mx, s_red[w]);
    __syncthreads();
    // sum of exp(v - max), then lse = max + ln(sum) (transcribe.rs:484)
    float sum = 0.f;
    for (int j = t; j < n; j += TOPK_THREADS) sum += expf(__fsub_rn(row[j], mx));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) s_red[warp] = sum;
    __syncthreads();
    sum = 0.f;
#pragma unroll
    for (int w = 0; w < TOPK_THREADS / 32; ++w) sum += s_red[w];
    const float lse = __fadd_rn(mx, logf(sum));
    // this thread's best k, sorted
    float tv[BEAM_MAX];
    int ti[BEAM_MAX];
#pragma unroll
    for (int c = 0; c < BEAM_MAX; ++c) {
        tv[c] = -INFINITY;
        ti[c] = 0x7fffffff;
    }
    for (int j = t; j < n; j += TOPK_THREADS) {
        const float v = row[j];
        if (!(v > -INFINITY)) continue;   // -inf and NaN are never chosen
        if (!better(v, j, tv[k - 1], ti[k - 1])) continue;
        int c = k - 1;
        while (c > 0 && better(v, j, tv[c - 1], ti[c - 1])) {
            tv[c] = tv[c - 1];
            ti[c] = ti[c - 1];
            --c;
        }
        tv[c] = v;
        ti[c] = j;
    }
    for (int c = 0; c < BEAM_MAX; ++c) {
        s_v[t * BEAM_MAX + c] = c < k ? tv[c] : -INFINITY;
        s_i[t * BEAM_MAX + c] = c < k ? ti[c] : 0x7fffffff;
    }
    __syncthreads();
    // warp 0 merges: k rounds of a (value, id) arg-max over all lists
    if (warp == 0) {
        for (int r = 0; r < k; ++r) {
            float bv = -INFINITY;
            int bi = 0x7fffffff, bslot = -1;
            for (int e = lane; e < TOPK_THREADS * BEAM_MAX; e += 32) {
                const float v = s_v[e];
                const int i = s_i[e];
                if (i != 0x7fffffff && better(v, i, bv, bi)) {
                    bv = v;
                    bi = i;
                    bslot = e;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                const int os = __shfl_xor_sync(0xffffffffu, bslot, o);
                if ((oi != 0x7fffffff && bi == 0x7fffffff) || (oi != 0x7fffffff && better(ov, oi, bv, bi))) {
                    bv = ov;
                    bi = oi;
                    bslot = os;
                }
            }
            if (lane == 0) {
                const size_t o = size_t(blockIdx.x) * k + r;
                if (bslot >= 0) {
                    lp_out[o] = __fsub_rn(bv, lse);
                    id_out[o] = bi;
                    s_i[bslot] = 0x7fffffff;   // taken
                } else {
                    lp_out[o] = -INFINITY;
                    id_out[o] = -1;
                }
            }
            __syncwarp();
        }
    }
}

// One thread per window (<= 64 candidates).  Streams of window w are
// w*B .. w*B + B - 1; the live beams are the slots whose rank is below
// n_live, visited in rank order (the reference's beam order), each with
// its k candidates in top-k order; a stable sort by score keeps that
// order among equal scores (Rust's sort_by, transcribe.rs:924).
__global__ void k_beam_select(const float* __restrict__ lp, const int32_t* __restrict__ id, int k,
                              const float* __restrict__ sum_in, const int32_t* __restrict__ rank_in, int W, int B,
                              int n_live, int32_t* __restrict__ src, int32_t* __restrict__ tok,
                              float* __restrict__ sum_out, float* __restrict__ step_out,
                              int32_t* __restrict__ rank_out) {
    pdl_trigger();
    pdl_wait();
    const int w = blockIdx.x * blockDim.x + threadIdx.x;
    if (w >= W) return;
    const int s0 = w * B;
    int order[BEAM_MAX];
    int nb = 0;
    for (int r = 0; r < n_live; ++r)
        for (int b = 0; b < B; ++b)
            if ((rank_in ? rank_in[s0 + b] : b) == r) {
                order[nb++] = b;
                break;
            }
    float score[BEAM_MAX * BEAM_MAX], slp[BEAM_MAX * BEAM_MAX];
    int par[BEAM_MAX * BEAM_MAX], cid[BEAM_MAX * BEAM_MAX];
    int nc = 0;
    for (int q = 0; q < nb; ++q) {
        const int b = order[q];
        for (int j = 0; j < k; ++j) {
            const int i = id[size_t(s0 + b) * k + j];
            if (i < 0) continue;
            const float st = fmaxf(lp[size_t(s0 + b) * k + j], -30.0f);
            const float sc = __fadd_rn(sum_in ? sum_in[s0 + b] : 0.f, st);
            int c = nc++;
            while (c > 0 && score[c - 1] < sc) {   // stable: equal scores keep their order
                score[c] = score[c - 1];
                slp[c] = slp[c - 1];
                par[c] = par[c - 1];
                cid[c] = cid[c - 1];
                --c;
            }
            score[c] = sc;
            slp[c] = st;
            par[c] = b;
            cid[c] = i;
        }
    }
    const int nsel = nc < B ? nc : B;
    // Slots: the first survivor of each parent stays in the parent's slot;
    // the others take the slots no survivor descends from.
    int slot_of[BEAM_MAX];
    bool used[BEAM_MAX], parent[BEAM_MAX];
    for (int b = 0; b < B; ++b) used[b] = parent[b] = false;
    for (int c = 0; c < nsel; ++c) parent[par[c]] = true;
    for (int c = 0; c < nsel; ++c) {
        slot_of[c] = -1;
        if (!used[par[c]]) {
            slot_of[c] = par[c];
            used[par[c]] = true;
        }
    }
    int next_free = 0;
    for (int c = 0; c < nsel; ++c) {
        if (slot_of[c] >= 0) continue;
        while (next_free < B && (used[next_free] || parent[next_free])) ++next_free;
        slot_of[c] = next_free;
        used[next_free] = true;
    }
    for (int c = 0; c < nsel; ++c) {
        const int s = s0 + slot_of[c];
        src[s] = s0 + par[c];
        tok[s] = cid[c];
        sum_out[s] = score[c];
        step_out[s] = slp[c];
        rank_out[s] = c;
    }
    // Fewer candidates than beams (a row with fewer than k choosable ids):
    // the remaining slots repeat the best survivor, ranked last.
    int extra = nsel;
    for (int b = 0; b < B; ++b) {
        if (used[b]) continue;
        const int s = s0 + b;
        if (nsel == 0) {
            src[s] = s;
            tok[s] = 0;
            sum_out[s] = -INFINITY;
            step_out[s] = -INFINITY;
        } else {
            src[s] = s0 + par[0];
            tok[s] = cid[0];
            sum_out[s] = score[0];
            step_out[s] = slp[0];
        }
        rank_out[s] = extra++;
    }
}

// Stream i's self-attention cache (every layer, positions 0 .. *dpos)
// becomes stream src[i]'s.  Sources outside [0, S), in another window, or
// themselves copied this step are ignored (the stream keeps its own
// history).  Grid (S, n_layer); cache [layer][S][H][ctx][64] f16.
__global__ void k_self_fork(const int32_t* __restrict__ src, const int32_t* __restrict__ win, int S, int H, int ctx,
                            const int* __restrict__ dpos, __half* __restrict__ kc, __half* __restrict__ vc) {
    pdl_trigger();
    pdl_wait();
    const int i = blockIdx.x, l = blockIdx.y;
    const int j = src[i];
    if (j == i || j < 0 || j >= S || win[j] != win[i] || src[j] != j) return;
    const int n = min(*dpos, ctx);
    const size_t layer = size_t(l) * S * H * ctx * 64;
    const int per_head = n * 8;   // 16-byte vectors of the first n rows
    for (int e = threadIdx.x; e < H * per_head; e += blockDim.x) {
        const int h = e / per_head, r = e % per_head;
        const size_t di = layer + (size_t(i) * H + h) * ctx * 64, si = layer + (size_t(j) * H + h) * ctx * 64;
        reinterpret_cast<uint4*>(kc + di)[r] = reinterpret_cast<const uint4*>(kc + si)[r];
        reinterpret_cast<uint4*>(vc + di)[r] = reinterpret_cast<const uint4*>(vc + si)[r];
    }
}

int bfail(int code, const char* fmt, ...) {
    char buf[256];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    set_last_error(buf);
    return code;
}

}  // namespace

cudaError_t launch_self_fork(const int32_t* src, const int32_t* win, int S, int H, int ctx, int n_layer,
                             const int* dpos, __half* kc, __half* vc, cudaStream_t s) {
    if (S <= 0 || n_layer <= 0) return cudaSuccess;
    return launch_pdl(k_self_fork, dim3(unsigned(S), unsigned(n_layer)), dim3(256), 0, s, src, win, S, H, ctx, dpos,
                      kc, vc);
}

}  // namespace rwq

extern "C" {

int rwq_beam_topk(const float* logits, int64_t rows, int64_t n_vocab, int32_t limit, int k, float* lp, int32_t* id,
                  void* stream) {
    if (rows < 0 || n_vocab <= 0 || n_vocab > INT32_MAX || k < 1 || k > rwq::BEAM_MAX)
        return rwq::bfail(RWQ_ERR_ARG, "rwq_beam_topk: rows %lld, n_vocab %lld, k %d (1..%d)", (long long)rows,
                          (long long)n_vocab, k, rwq::BEAM_MAX);
    if (rows == 0) return RWQ_OK;
    if (!logits || !lp || !id) return rwq::bfail(RWQ_ERR_ARG, "rwq_beam_topk: null pointer");
    if (rows > (1 << 24)) return rwq::bfail(RWQ_ERR_ARG, "rwq_beam_topk: too many rows");
    const int n = (limit >= 0 && limit < n_vocab) ? int(limit) : int(n_vocab);
    cudaError_t e = rwq::launch_pdl(rwq::k_beam_topk, dim3(unsigned(rows)), dim3(rwq::TOPK_THREADS), 0,
                                    static_cast<cudaStream_t>(stream), logits, int(n_vocab), n, k, lp, id);
    if (e != cudaSuccess) return rwq::bfail(RWQ_ERR_CUDA, "rwq_beam_topk: %s", cudaGetErrorString(e));
    return RWQ_OK;
}

int rwq_beam_select(const float* lp, const int32_t* id, int k, const float* sum_lp, const int32_t* rank,
                    int64_t n_windows, int beams, int n_live, int32_t* src, int32_t* token, float* sum_out,
                    float* step_lp, int32_t* rank_out, void* stream) {
    if (n_windows < 0 || n_windows > (1 << 24) || beams < 1 || beams > rwq::BEAM_MAX || k < 1 ||
        k > rwq::BEAM_MAX || n_live < 1 || n_live > beams)
        return rwq::bfail(RWQ_ERR_ARG, "rwq_beam_select: windows %lld, beams %d (1..%d), k %d, n_live %d",
                          (long long)n_windows, beams, rwq::BEAM_MAX, k, n_live);
    if (n_windows == 0) return RWQ_OK;
    if (!lp || !id || !src || !token || !sum_out || !step_lp || !rank_out)
        return rwq::bfail(RWQ_ERR_ARG, "rwq_beam_select: null pointer");
    const unsigned blocks = unsigned((n_windows + 63) / 64);
    cudaError_t e = rwq::launch_pdl(rwq::k_beam_select, dim3(blocks), dim3(64), 0, static_cast<cudaStream_t>(stream),
                                    lp, id, k, sum_lp, rank, int(n_windows), beams, n_live, src, token, sum_out,
                                    step_lp, rank_out);
    if (e != cudaSuccess) return rwq::bfail(RWQ_ERR_CUDA, "rwq_beam_select: %s", cudaGetErrorString(e));
    return RWQ_OK;
}

}  // extern "C"
