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

// Rows are split over a cluster of TOPK_CHUNKS CTAs (one chunk of the
// first n ids each): every CTA finds its chunk's max m_c, s_c = sum of
// exp(v - m_c) and top k; CTA 0 of the cluster reads the partials through
// distributed shared memory, forms lse = M + ln(sum_c s_c exp(m_c - M))
// (M = max m_c; transcribe.rs:482-486 with the sum split by chunk) and
// merges the top k.  Ids >= n are excluded (suppressed); -inf and NaN
// logits are never chosen (the reference skips lp == -inf); rows with
// fewer than k choosable ids get id -1 and lp -inf in the remaining places.
constexpr int TOPK_CHUNKS = 8;
constexpr int NOID = 0x7fffffff;

struct TopkPart {
    float m, s;
    float v[BEAM_MAX];
    int i[BEAM_MAX];
};

// Pop the best of the lanes' sorted lists (heads tv[0], ti[0]) k times:
// the result, best first, in every lane's ov/oi.  Ids are distinct, so the
// butterfly agrees on one winner, whose lane shifts its list.
template <int K>
__device__ __forceinline__ void warp_topk(float (&tv)[K], int (&ti)[K], float (&ov)[K], int (&oi)[K]) {
#pragma unroll
    for (int r = 0; r < K; ++r) {
        float bv = tv[0];
        int bi = ti[0];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float v = __shfl_xor_sync(0xffffffffu, bv, o);
            const int i = __shfl_xor_sync(0xffffffffu, bi, o);
            if (i != NOID && (bi == NOID || better(v, i, bv, bi))) {
                bv = v;
                bi = i;
            }
        }
        ov[r] = bv;
        oi[r] = bi;
        if (bi != NOID && ti[0] == bi) {
#pragma unroll
            for (int c = 0; c + 1 < K; ++c) {
                tv[c] = tv[c + 1];
                ti[c] = ti[c + 1];
            }
            tv[K - 1] = -INFINITY;
            ti[K - 1] = NOID;
        }
    }
}

__device__ __forceinline__ uint32_t bk_mapa(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(uint32_t(__cvta_generic_to_shared(p))), "r"(rank));
    return r;
}
__device__ __forceinline__ float bk_ld_f(uint32_t a) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ int bk_ld_i(uint32_t a) {
    int v;
    asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
    return v;
}
__device__ __forceinline__ void bk_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

template <int K>
__global__ void __launch_bounds__(TOPK_THREADS) k_beam_topk(const float* __restrict__ logits, int V, int n,
                                                          float* __restrict__ lp_out, int32_t* __restrict__ id_out) {
    pdl_trigger();
    pdl_wait();
    const int c = int(blockIdx.x), r_row = int(blockIdx.y);
    const float* row = logits + size_t(r_row) * V;
    const int j0 = int(int64_t(c) * n / TOPK_CHUNKS), j1 = int(int64_t(c + 1) * n / TOPK_CHUNKS);
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    constexpr int NW = TOPK_THREADS / 32;
    __shared__ float s_red[NW];
    __shared__ float s_wv[NW][BEAM_MAX];
    __shared__ int s_wi[NW][BEAM_MAX];
    __shared__ TopkPart part;
    // max (NaN ignored, as f32::max folding from -inf)
    float mx = -INFINITY;
    for (int j = j0 + t; j < j1; j += TOPK_THREADS) mx = fmaxf(mx, row[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) s_red[warp] = mx;
    __syncthreads();
    mx = s_red[0];
#pragma unroll
    for (int w = 1; w < NW; ++w) mx = fmaxf(mx, s_red[w]);
    __syncthreads();
    // sum of exp(v - m_c) over the chunk (0 for a chunk without a finite max)
    float sum = 0.f;
    if (mx > -INFINITY)
        for (int j = j0 + t; j < j1; j += TOPK_THREADS) sum += expf(__fsub_rn(row[j], mx));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) s_red[warp] = sum;
    __syncthreads();
    sum = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) sum += s_red[w];
    // this thread's best k, sorted, then the warp's, then the CTA's
    float tv[K], ov[K];
    int ti[K], oi[K];
#pragma unroll
    for (int q = 0; q < K; ++q) {
        tv[q] = -INFINITY;
        ti[q] = NOID;
    }
    auto offer = [&](float v, int j) {
        if (!(v > -INFINITY)) return;   // -inf and NaN are never chosen
        if (ti[K - 1] != NOID && !better(v, j, tv[K - 1], ti[K - 1])) return;
        // insert, keeping tv[0..K) sorted (registers: fixed-index moves)
        bool placed = false;
#pragma unroll
        for (int q = K - 1; q >= 0; --q) {
            if (placed) continue;
            const bool above = q > 0 && (ti[q - 1] == NOID || better(v, j, tv[q - 1], ti[q - 1]));
            if (above) {
                tv[q] = tv[q - 1];
                ti[q] = ti[q - 1];
            } else {
                tv[q] = v;
                ti[q] = j;
                placed = true;
            }
        }
    };
    for (int j = j0 + t; j < j1; j += TOPK_THREADS) offer(row[j], j);
    warp_topk<K>(tv, ti, ov, oi);
    if (lane == 0)
#pragma unroll
        for (int q = 0; q < K; ++q) {
            s_wv[warp][q] = ov[q];
            s_wi[warp][q] = oi[q];
        }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int q = 0; q < K; ++q) {
            tv[q] = lane < NW ? s_wv[lane][q] : -INFINITY;
            ti[q] = lane < NW ? s_wi[lane][q] : NOID;
        }
        warp_topk<K>(tv, ti, ov, oi);
        if (lane == 0) {
            part.m = mx;
            part.s = sum;
#pragma unroll
            for (int q = 0; q < K; ++q) {
                part.v[q] = ov[q];
                part.i[q] = oi[q];
            }
        }
    }
    bk_cluster_sync();
    if (c == 0 && warp == 0) {
        // lane q < TOPK_CHUNKS reads chunk q's partial
        float m_c = -INFINITY, s_c = 0.f;
#pragma unroll
        for (int q = 0; q < K; ++q) {
            tv[q] = -INFINITY;
            ti[q] = NOID;
        }
        if (lane < TOPK_CHUNKS) {
            m_c = bk_ld_f(bk_mapa(&part.m, lane));
            s_c = bk_ld_f(bk_mapa(&part.s, lane));
#pragma unroll
            for (int q = 0; q < K; ++q) {
                tv[q] = bk_ld_f(bk_mapa(&part.v[q], lane));
                ti[q] = bk_ld_i(bk_mapa(&part.i[q], lane));
            }
        }
        float M = m_c;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        // sum in chunk order
        float S = 0.f;
#pragma unroll
        for (int q = 0; q < TOPK_CHUNKS; ++q) {
            const float mq = __shfl_sync(0xffffffffu, m_c, q), sq = __shfl_sync(0xffffffffu, s_c, q);
            if (sq > 0.f) S = __fadd_rn(S, __fmul_rn(sq, expf(__fsub_rn(mq, M))));
        }
        const float lse = __fadd_rn(M, logf(S));
        warp_topk<K>(tv, ti, ov, oi);
        if (lane == 0) {
#pragma unroll
            for (int q = 0; q < K; ++q) {
                const size_t o = size_t(r_row) * K + q;
                if (oi[q] != NOID) {
                    lp_out[o] = __fsub_rn(ov[q], lse);
                    id_out[o] = oi[q];
                } else {
                    lp_out[o] = -INFINITY;
                    id_out[o] = -1;
                }
            }
        }
    }
    bk_cluster_sync();   // the partials stay readable until CTA 0 is done
}

// One warp per window (<= 64 candidates: beams x k <= 8 x 8, two per
// lane).  Streams of window w are w*B .. w*B + B - 1; the live beams are
// the slots whose rank is below n_live, visited in rank order (the
// reference's beam order), each with its k candidates in top-k order;
// candidate e = (beam order q)*k + j.  A candidate's place in the stable
// sort by score (Rust's sort_by, transcribe.rs:924) is the number of valid
// candidates with a higher score or an equal score and a smaller e.
// Survivors take stream slots: the best survivor of each parent stays in
// the parent's slot; the others take, in survivor order, the slots no
// survivor descends from, in slot order.
__global__ void k_beam_select(const float* __restrict__ lp, const int32_t* __restrict__ id, int k,
                              const float* __restrict__ sum_in, const int32_t* __restrict__ rank_in, int W, int B,
                              int n_live, int32_t* __restrict__ src, int32_t* __restrict__ tok,
                              float* __restrict__ sum_out, float* __restrict__ step_out,
                              int32_t* __restrict__ rank_out) {
    pdl_trigger();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int w = int(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (w >= W) return;   // whole warps leave together
    const int s0 = w * B;
    // slot of beam-order position q (lanes q < n_live), broadcast below
    int slot_q = -1;
    if (lane < n_live)
        for (int b = 0; b < B; ++b)
            if ((rank_in ? rank_in[s0 + b] : b) == lane) {
                slot_q = b;
                break;
            }
    // two candidates per lane: e = lane and e = lane + 32
    float sc[2], st[2];
    int par[2], cid[2];
    bool ok[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int e = lane + 32 * h, q = e / k, jj = e % k;
        const int b = __shfl_sync(0xffffffffu, slot_q, q < 32 ? q : 0);
        ok[h] = e < n_live * k && q < n_live && b >= 0;
        sc[h] = st[h] = 0.f;
        par[h] = cid[h] = 0;
        if (ok[h]) {
            const int i = id[size_t(s0 + b) * k + jj];
            ok[h] = i >= 0;
            st[h] = fmaxf(lp[size_t(s0 + b) * k + jj], -30.0f);
            sc[h] = __fadd_rn(sum_in ? sum_in[s0 + b] : 0.f, st[h]);
            par[h] = b;
            cid[h] = i;
        }
    }
    // stable rank among the valid candidates
    int rk[2] = {0, 0};
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
        for (int l2 = 0; l2 < 32; ++l2) {
            const float o_sc = __shfl_sync(0xffffffffu, sc[h2], l2);
            const bool o_ok = __shfl_sync(0xffffffffu, ok[h2] ? 1 : 0, l2) != 0;
            const int oe = l2 + 32 * h2;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int e = lane + 32 * h;
                if (o_ok && (o_sc > sc[h] || (o_sc == sc[h] && oe < e))) ++rk[h];
            }
        }
    }
    const int nvalid = __popc(__ballot_sync(0xffffffffu, ok[0])) + __popc(__ballot_sync(0xffffffffu, ok[1]));
    const int nsel = nvalid < B ? nvalid : B;
    // survivors' parents; keepers: no better survivor of the same parent
    unsigned parent_mask = 0;
    bool surv[2], keep[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) surv[h] = ok[h] && rk[h] < nsel;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        unsigned m = __ballot_sync(0xffffffffu, surv[h]);
        for (unsigned mm = m; mm; mm &= mm - 1) parent_mask |= 1u << __shfl_sync(0xffffffffu, par[h], __ffs(mm) - 1);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) keep[h] = surv[h];
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2)
        for (int l2 = 0; l2 < 32; ++l2) {
            const bool o_s = __shfl_sync(0xffffffffu, surv[h2] ? 1 : 0, l2) != 0;
            const int o_p = __shfl_sync(0xffffffffu, par[h2], l2), o_r = __shfl_sync(0xffffffffu, rk[h2], l2);
#pragma unroll
            for (int h = 0; h < 2; ++h)
                if (o_s && o_p == par[h] && o_r < rk[h]) keep[h] = false;
        }
    const unsigned all = (1u << B) - 1u;
    const unsigned free_mask = all & ~parent_mask;
    // keepers stay in their parent's slot; the m-th non-keeper (by rank)
    // takes the m-th free slot
    int slot[2] = {-1, -1}, m_nk[2] = {0, 0};
    unsigned used = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        if (keep[h]) slot[h] = par[h];
        const unsigned km = __ballot_sync(0xffffffffu, keep[h]);
        for (unsigned mm = km; mm; mm &= mm - 1) used |= 1u << __shfl_sync(0xffffffffu, par[h], __ffs(mm) - 1);
    }
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2)
        for (int l2 = 0; l2 < 32; ++l2) {
            const bool o_nk = __shfl_sync(0xffffffffu, (surv[h2] && !keep[h2]) ? 1 : 0, l2) != 0;
            const int o_r = __shfl_sync(0xffffffffu, rk[h2], l2);
#pragma unroll
            for (int h = 0; h < 2; ++h)
                if (o_nk && o_r < rk[h]) ++m_nk[h];
        }
#pragma unroll
    for (int h = 0; h < 2; ++h)
        if (surv[h] && !keep[h]) {
            unsigned fm = free_mask;
            for (int q = 0; q < m_nk[h]; ++q) fm &= fm - 1;
            slot[h] = __ffs(fm) - 1;
        }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const unsigned nm = __ballot_sync(0xffffffffu, surv[h] && !keep[h]);
        for (unsigned mm = nm; mm; mm &= mm - 1) used |= 1u << __shfl_sync(0xffffffffu, slot[h], __ffs(mm) - 1);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h)
        if (surv[h]) {
            const int sI = s0 + slot[h];
            src[sI] = s0 + par[h];
            tok[sI] = cid[h];
            sum_out[sI] = sc[h];
            step_out[sI] = st[h];
            rank_out[sI] = rk[h];
        }
    // Fewer candidates than beams (a row with fewer than k choosable ids):
    // the remaining slots repeat the best survivor, ranked last.
    if (nsel < B) {
        int best_lane = -1, best_h = 0;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const unsigned bm = __ballot_sync(0xffffffffu, surv[h] && rk[h] == 0);
            if (bm) {
                best_lane = __ffs(bm) - 1;
                best_h = h;
            }
        }
        float b_sc = -INFINITY, b_st = -INFINITY;
        int b_par = 0, b_cid = 0;
        if (best_lane >= 0) {
            b_sc = __shfl_sync(0xffffffffu, best_h ? sc[1] : sc[0], best_lane);
            b_st = __shfl_sync(0xffffffffu, best_h ? st[1] : st[0], best_lane);
            b_par = __shfl_sync(0xffffffffu, best_h ? par[1] : par[0], best_lane);
            b_cid = __shfl_sync(0xffffffffu, best_h ? cid[1] : cid[0], best_lane);
        }
        if (lane == 0) {
            int extra = nsel;
            for (int b = 0; b < B; ++b) {
                if (used & (1u << b)) continue;
                const int sI = s0 + b;
                if (nsel == 0) {
                    src[sI] = sI;
                    tok[sI] = 0;
                    sum_out[sI] = -INFINITY;
                    step_out[sI] = -INFINITY;
                } else {
                    src[sI] = s0 + b_par;
                    tok[sI] = b_cid;
                    sum_out[sI] = b_sc;
                    step_out[sI] = b_st;
                }
                rank_out[sI] = extra++;
            }
        }
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
    const int n = (limit >= 0 && limit < n_vocab) ? int(limit) : int(n_vocab);
    if (rows > 65535) return rwq::bfail(RWQ_ERR_ARG, "rwq_beam_topk: too many rows");
    auto go = [&](auto kern) {
        return rwq::launch_pdl_cluster(kern, dim3(rwq::TOPK_CHUNKS, unsigned(rows)), dim3(rwq::TOPK_THREADS), 0,
                                       rwq::TOPK_CHUNKS, static_cast<cudaStream_t>(stream), logits, int(n_vocab), n,
                                       lp, id);
    };
    cudaError_t e;
    switch (k) {
        case 1: e = go(rwq::k_beam_topk<1>); break;
        case 2: e = go(rwq::k_beam_topk<2>); break;
        case 3: e = go(rwq::k_beam_topk<3>); break;
        case 4: e = go(rwq::k_beam_topk<4>); break;
        case 5: e = go(rwq::k_beam_topk<5>); break;
        case 6: e = go(rwq::k_beam_topk<6>); break;
        case 7: e = go(rwq::k_beam_topk<7>); break;
        default: e = go(rwq::k_beam_topk<8>); break;
    }
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
    const unsigned blocks = unsigned((n_windows + 3) / 4);   // a warp per window
    cudaError_t e = rwq::launch_pdl(rwq::k_beam_select, dim3(blocks), dim3(128), 0, static_cast<cudaStream_t>(stream),
                                    lp, id, k, sum_lp, rank, int(n_windows), beams, n_live, src, token, sum_out,
                                    step_lp, rank_out);
    if (e != cudaSuccess) return rwq::bfail(RWQ_ERR_CUDA, "rwq_beam_select: %s", cudaGetErrorString(e));
    return RWQ_OK;
}

}  // extern "C"
