// rwq_gemv_rows_sm100.cu -- the decoder GEMV at one or two activation rows
// on wide weights (the tied logits projection of a single-stream decode):
// one weight row per lane, the weight planes staged by TMA.
//
// k_gemv_mma gives each 16-row tile to one warp and decodes the codes into
// mma.sync fragments; at one activation row 7/8 of every MMA is idle and
// the per-block fragment work (~3.5 warp instructions per row-block) holds
// it near half of the HBM rate.  Here lane l of a warp owns weight row
// 32*slab + l: it decodes each of its blocks once (nibbles, fifth bits)
// and takes the integer block dot with dp4a against the activation codes,
// which every lane reads from the same shared-memory address (a broadcast)
// -- about 1.4 warp instructions per row-block at one activation row.
//
// Feed: a warp's 32 rows x 8 blocks are one stage of three or four TMA
// boxes in a per-warp ring of GR_RING stages: codes [32 rows][128 B] with
// the 128-byte swizzle and fifth bits [32][32 B] with the 32-byte swizzle
// (a lane's 16-byte reads of its own row then fall in distinct banks for
// every 8 consecutive lanes), f16 scales and mins [32][16 B] unswizzled.
// The loads are issued by lane 0 of the warp and complete on the stage's
// mbarrier; no registers hold data in flight.  A warp reads a landed stage
// into registers and hands the slot back before it does the stage's math,
// so the weight stream never waits for the arithmetic.  One CTA per SM
// whose warps (up to 11) cover the SM's share of the 32-row slabs, so
// nearly the whole weight is requested at once.
//
// Results are bit-identical to k_gemv_mma's (and so to k_gemv_tile's):
// every output adds its blocks in kb order with the same f32 operations,
//     acc <- fma(d_a*d_b, S, acc);  acc <- fma(d_a*sum(q_a), m_b, acc)
// (S the exact integer block dot), and where k_gemv_mma's warp ranges split
// a 16-row tile -- head and tail summed separately, then added -- the lane
// does the same (gemv_slice_start).  Only weights that k_gemv_mma runs
// without a K split come here (the host checks), so that one lane can walk
// all of K in order.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cstdio>
#include <mutex>
#include "rwq_common.cuh"
#include "rwq_internal.h"
#include "rwq_sm100.cuh"

namespace rwq {
namespace {

using tc::mbar_expect_tx;
using tc::mbar_init;
using tc::mbar_wait;
using tc::smem_u32;
using tc::tma_load_2d;

constexpr int GR_RING = 2;         // stages in flight per warp
constexpr int GR_MAX_WARPS = 11;
constexpr int GR_ERR_WAIT = 41;    // error code: a stage never arrived
constexpr size_t GR_SMEM_CTA = 227 * 1024;

// One stage: 32 weight rows x 2 groups of 4 blocks.  The code boxes of all
// stages form one array (4 KB boxes, 1024-byte aligned for the 128-byte
// swizzle), the small planes another (offsets multiples of 256 bytes for
// the 32-byte swizzle).
template <int DT>
struct GrStage {
    static constexpr int QBOXES = 8 * qs_bytes(DT) / 128;   // [32][128 B] code boxes: 1, or 2 for Q8_0
    static constexpr int QBYTES = QBOXES * 4096;
    static constexpr int H = 0;                             // fifth bits [32][32 B]
    static constexpr int D = H + (has_qh(DT) ? 1024 : 0);   // d [32][16 B]
    static constexpr int MN = D + 512;                      // m [32][16 B]
    static constexpr int SMALL = MN + (has_min(DT) ? 512 : 0);
    static constexpr uint32_t TX = QBYTES + SMALL;          // bytes the boxes deliver
    static constexpr int BYTES = QBYTES + SMALL;
};

__host__ __device__ constexpr size_t gr_act_bytes(int m, int nb4) { return size_t(m) * nb4 * 48; }

__host__ __device__ constexpr size_t gr_smem(int warps, int stage_bytes, int m, int nb4) {
    return 1024 + size_t(warps) * GR_RING * stage_bytes + gr_act_bytes(m, nb4) + size_t(warps) * GR_RING * 8 + 16;
}

template <int DT>
__device__ __forceinline__ int gr_dot(uint32_t act, uint32_t code, int c) {
    return DT == Q8_0 ? dp4a_ss(act, code, c) : dp4a_su(act, code, c);
}

template <int DT, int M>
__global__ void __launch_bounds__(GR_MAX_WARPS * 32, 1)
    k_gemv_rows(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap th,
                const __grid_constant__ CUtensorMap td, const __grid_constant__ CUtensorMap tm,
                const int8_t* __restrict__ q8, const float* __restrict__ da, const int32_t* __restrict__ sa,
                const float* __restrict__ ua, int N, int K, const float* __restrict__ bias, float* __restrict__ y,
                int gx, int* __restrict__ err_flag) {
    using L = GrStage<DT>;
    constexpr int NONE = 1 << 30;
    const int nb = K / QK, nb4 = round4(nb), ng = nb4 / 4, ns = ng / 2;   // ng is even (host)
    const int tiles = (N + 15) / 16, slabs = (N + 31) / 32;
    const int W = int(blockDim.x) >> 5;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* ring = base + size_t(warp) * GR_RING * L::QBYTES;                        // code boxes
    uint8_t* small = base + size_t(W) * GR_RING * L::QBYTES + size_t(warp) * GR_RING * L::SMALL;
    uint8_t* acts = base + size_t(W) * GR_RING * L::BYTES;                   // [M][nb4][32] codes
    int4* recs = reinterpret_cast<int4*>(acts + size_t(M) * nb4 * 32);       // [M][nb4] {seed, d_a, d_a*sum, 0}
    uint64_t* full = reinterpret_cast<uint64_t*>(recs + M * nb4) + warp * GR_RING;
    volatile int* abort = reinterpret_cast<volatile int*>(reinterpret_cast<uint64_t*>(recs + M * nb4) + W * GR_RING);

    // This CTA's slabs [s_lo, s_hi); warp w takes s_lo + w, s_lo + w + W, ...
    const int s_lo = int(int64_t(blockIdx.x) * slabs / gridDim.x);
    const int s_hi = int(int64_t(blockIdx.x + 1) * slabs / gridDim.x);
    const int mine = s_hi - s_lo > warp ? (s_hi - s_lo - warp + W - 1) / W : 0;
    const int items = mine * ns;

    if (lane == 0) {
        for (int s = 0; s < GR_RING; ++s) mbar_init(full + s, 1);
        if (warp == 0) *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncwarp();
    // Stage `it` of this warp into its ring slot, issued by the warp's own
    // lane 0.  The planes are never written by a kernel launched as a
    // programmatic dependent, so they are read before griddepcontrol.wait
    // (overlapping the predecessor's tail).
    auto issue = [&](int it) {
        const int sl = s_lo + warp + (it / ns) * W, st = it % ns;
        uint8_t* dst = ring + (it % GR_RING) * L::QBYTES;
        uint8_t* dsm = small + (it % GR_RING) * L::SMALL;
        uint64_t* bar = full + it % GR_RING;
        mbar_expect_tx(bar, L::TX);
#pragma unroll
        for (int q = 0; q < L::QBOXES; ++q) tma_load_2d(dst + q * 4096, &tq, (st * L::QBOXES + q) * 128, sl * 32, bar);
        if (has_qh(DT)) tma_load_2d(dsm + L::H, &th, st * 32, sl * 32, bar);
        tma_load_2d(dsm + L::D, &td, st * 16, sl * 32, bar);
        if (has_min(DT)) tma_load_2d(dsm + L::MN, &tm, st * 16, sl * 32, bar);
    };
    if (lane == 0)
        for (int it = 0; it < GR_RING && it < items; ++it) issue(it);

    pdl_trigger();
    pdl_wait();
    // Activations: codes of rows [0, M) with zero pad blocks; per block the
    // dot's seed, d_a and d_a*sum(q_a) (pad blocks: seed 1.5*2^23, zero
    // scales, so they add exactly 0 as in k_gemv_mma).
    for (int i = tid; i < M * nb4 * 8; i += blockDim.x) {
        const int r = i / (nb4 * 8), wd = i % (nb4 * 8);
        reinterpret_cast<uint32_t*>(acts)[i] =
            wd < nb * 8 ? __ldg(reinterpret_cast<const uint32_t*>(q8 + size_t(r) * K) + wd) : 0u;
    }
    for (int i = tid; i < M * nb4; i += blockDim.x) {
        const int r = i / nb4, kb = i % nb4;
        int4 rec = make_int4(int(MAGIC_BITS), 0, 0, 0);
        if (kb < nb) {
            const size_t o = size_t(r) * nb + kb;
            if (code_offset(DT)) rec.x = int(MAGIC_BITS - uint32_t(code_offset(DT) * __ldg(sa + o)));
            rec.y = __float_as_int(__ldg(da + o));
            if (has_min(DT)) rec.z = __float_as_int(__ldg(ua + o));
        }
        recs[i] = rec;
    }
    __syncthreads();

    float acc[M], head[M];
    int cut = NONE, row = 0;
    for (int it = 0; it < items; ++it) {
        const int st = it % ns;
        if (st == 0) {
            row = (s_lo + warp + (it / ns) * W) * 32 + lane;
            cut = gemv_slice_start(min(row, N - 1) >> 4, 1, 1, ng, gx, tiles);
#pragma unroll
            for (int i = 0; i < M; ++i) acc[i] = head[i] = 0.f;
        }
        if (!mbar_wait(full + it % GR_RING, uint32_t(it / GR_RING) & 1u, abort, err_flag, GR_ERR_WAIT)) return;
        // The whole stage into registers, then the slot goes back to the
        // TMA at once: the next loads do not wait for this stage's math.
        constexpr int CW = qs_bytes(DT) / 4;   // 16-byte chunks per row and group
        const uint8_t* stg = ring + (it % GR_RING) * L::QBYTES;
        const uint8_t* sms = small + (it % GR_RING) * L::SMALL;
        uint4 cq[2][CW], hq[2];
#pragma unroll
        for (int gi = 0; gi < 2; ++gi) {
            // Q4/Q5: the group's 4 chunks follow each other in the row's 128
            // bytes; Q8_0: a group is a whole 128-byte box row.
            const uint8_t* rowp = stg + (DT == Q8_0 ? gi * 4096 : 0) + lane * 128;
#pragma unroll
            for (int w = 0; w < CW; ++w) {
                const int ch = DT == Q8_0 ? w : gi * 4 + w;
                cq[gi][w] = *reinterpret_cast<const uint4*>(rowp + ((ch ^ (lane & 7)) << 4));
            }
            hq[gi] = has_qh(DT) ? *reinterpret_cast<const uint4*>(sms + L::H + lane * 32 + ((gi ^ ((lane >> 2) & 1)) << 4))
                                : make_uint4(0u, 0u, 0u, 0u);
        }
        const uint4 dv = *reinterpret_cast<const uint4*>(sms + L::D + lane * 16);
        const uint4 mv = has_min(DT) ? *reinterpret_cast<const uint4*>(sms + L::MN + lane * 16) : make_uint4(0u, 0u, 0u, 0u);
        __syncwarp();
        if (lane == 0 && it + GR_RING < items) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the reads above before the refill
            issue(it + GR_RING);
        }
        const uint32_t dw[4] = {dv.x, dv.y, dv.z, dv.w}, mw[4] = {mv.x, mv.y, mv.z, mv.w};

        // One block: codes cw[8] (word j = elements of activation word j).
        auto block = [&](int kb, const uint32_t (&cw)[8], int j) {
            const float db = __half2float(__ushort_as_half(uint16_t(dw[j >> 1] >> (16 * (j & 1)))));
            const float mb = has_min(DT) ? __half2float(__ushort_as_half(uint16_t(mw[j >> 1] >> (16 * (j & 1))))) : 0.f;
#pragma unroll
            for (int i = 0; i < M; ++i) {
                const uint8_t* ap = acts + (size_t(i) * nb4 + kb) * 32;
                const uint4 a0 = *reinterpret_cast<const uint4*>(ap);
                const uint4 a1 = *reinterpret_cast<const uint4*>(ap + 16);
                const int4 rc = recs[i * nb4 + kb];
                // Two chains (exact integers, any order), then their sum.
                int D0 = rc.x, D1 = 0;
                D0 = gr_dot<DT>(a0.x, cw[0], D0);
                D1 = gr_dot<DT>(a1.x, cw[4], D1);
                D0 = gr_dot<DT>(a0.y, cw[1], D0);
                D1 = gr_dot<DT>(a1.y, cw[5], D1);
                D0 = gr_dot<DT>(a0.z, cw[2], D0);
                D1 = gr_dot<DT>(a1.z, cw[6], D1);
                D0 = gr_dot<DT>(a0.w, cw[3], D0);
                D1 = gr_dot<DT>(a1.w, cw[7], D1);
                const float s = __fadd_rn(__int_as_float(D0 + D1), -MAGIC_F);
                acc[i] = __fmaf_rn(__fmul_rn(__int_as_float(rc.y), db), s, acc[i]);
                if (has_min(DT)) acc[i] = __fmaf_rn(__int_as_float(rc.z), mb, acc[i]);
            }
        };

#pragma unroll
        for (int gi = 0; gi < 2; ++gi) {
            const int g = st * 2 + gi;
            if (g == cut) {   // k_gemv_mma's next warp starts this tile's tail here
#pragma unroll
                for (int i = 0; i < M; ++i) {
                    head[i] = acc[i];
                    acc[i] = 0.f;
                }
            }
            const uint32_t hw[4] = {hq[gi].x, hq[gi].y, hq[gi].z, hq[gi].w};
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                uint32_t cw[8];
                if (DT != Q8_0) {
                    // Chunk w of the group holds word w of its blocks 0..3.
                    auto comp = [b](const uint4& v) { return b == 0 ? v.x : b == 1 ? v.y : b == 2 ? v.z : v.w; };
                    codes_u8x4<DT>(make_uint4(comp(cq[gi][0]), comp(cq[gi][1 % CW]), comp(cq[gi][2 % CW]),
                                              comp(cq[gi][3 % CW])), hw[b], cw);
                } else {
                    // Word w of block b sits at (w%4)*32 + b*8 + (w/4)*4 of
                    // the group: chunk (w%4)*2 + b/2, component (b%2)*2 + w/4.
#pragma unroll
                    for (int w = 0; w < 8; ++w) {
                        const uint4 v = cq[gi][((w & 3) * 2 + (b >> 1)) % CW];
                        const int c = (b & 1) * 2 + (w >> 2);
                        cw[w] = c == 0 ? v.x : c == 1 ? v.y : c == 2 ? v.z : v.w;
                    }
                }
                block(g * 4 + b, cw, gi * 4 + b);
            }
        }
        if (st == ns - 1 && row < N) {
            const float bb = bias ? __ldg(bias + row) : 0.f;
#pragma unroll
            for (int i = 0; i < M; ++i) {
                float v = cut < ng ? __fadd_rn(head[i], acc[i]) : acc[i];
                if (bias) v = __fadd_rn(v, bb);
                y[size_t(i) * N + row] = v;
            }
        }
    }
}

// ------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 g_encode_rows = nullptr;
std::once_flag g_encode_rows_once;

bool encode_plane(void* map, const void* ptr, uint64_t row_bytes, uint64_t rows, uint32_t box_bytes,
                  CUtensorMapSwizzle sw) {
    std::call_once(g_encode_rows_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode_rows = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!g_encode_rows) return false;
    cuuint64_t dims[2] = {row_bytes, rows};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_bytes, 32};
    cuuint32_t estr[2] = {1, 1};
    return g_encode_rows(static_cast<CUtensorMap*>(map), CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr),
                         dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sms_here(int* dev) {
    static int cache[64] = {};
    cudaGetDevice(dev);
    int sms = 0;
    if (*dev >= 0 && *dev < 64) {
        if (!cache[*dev]) cudaDeviceGetAttribute(&cache[*dev], cudaDevAttrMultiProcessorCount, *dev);
        return cache[*dev];
    }
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, *dev);
    return sms;
}

template <int DT, int M>
cudaError_t gemv_rows_go(const ActsView& v, const Weight& w, const float* bias, float* y, int gx, int* err_flag,
                         cudaStream_t s) {
    using L = GrStage<DT>;
    auto kern = k_gemv_rows<DT, M>;
    int dev = 0;
    const int sms = sms_here(&dev);
    static unsigned attr_dev_mask = 0;   // one bit per device with the attribute set
    if (dev >= 0 && dev < 32 && !(attr_dev_mask & (1u << dev))) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(GR_SMEM_CTA));
        if (e != cudaSuccess) return e;
        attr_dev_mask |= 1u << dev;
    }
    const int nb4 = round4(w.nb), slabs = (w.n + 31) / 32;
    int W = (slabs + sms - 1) / sms;
    W = W < 1 ? 1 : (W > GR_MAX_WARPS ? GR_MAX_WARPS : W);
    while (W > 1 && gr_smem(W, L::BYTES, M, nb4) > GR_SMEM_CTA) --W;
    const size_t smem = gr_smem(W, L::BYTES, M, nb4);
    if (smem > GR_SMEM_CTA) return cudaErrorInvalidValue;
    int grid = (slabs + W - 1) / W;
    grid = grid > sms ? sms : grid;
    const CUtensorMap* mp = reinterpret_cast<const CUtensorMap*>(w.row_maps);
    return launch_pdl(kern, dim3(unsigned(grid)), dim3(unsigned(W * 32)), smem, s, mp[0], mp[1], mp[2], mp[3], v.q8,
                      v.d, v.sum, v.u, w.n, w.k, bias, y, gx, err_flag);
}

template <int DT>
cudaError_t gemv_rows_dt(const ActsView& v, const Weight& w, const float* bias, float* y, int gx, int* err_flag,
                         cudaStream_t s) {
    return v.m <= 1 ? gemv_rows_go<DT, 1>(v, w, bias, y, gx, err_flag, s)
                    : gemv_rows_go<DT, 2>(v, w, bias, y, gx, err_flag, s);
}

template <int DT>
constexpr int gr_stage_bytes() { return GrStage<DT>::BYTES; }

int stage_bytes_of(int dt) {
    switch (dt) {
        case Q4_0: return gr_stage_bytes<Q4_0>();
        case Q4_1: return gr_stage_bytes<Q4_1>();
        case Q5_0: return gr_stage_bytes<Q5_0>();
        case Q5_1: return gr_stage_bytes<Q5_1>();
        case Q8_0: return gr_stage_bytes<Q8_0>();
        default: return -1;
    }
}

}  // namespace

void prepare_gemv_rows(Weight& w) {
    w.rows_ready = false;
    const int nb4 = round4(w.nb);
    // The d/m planes' rows (2*nb4 bytes) must be multiples of 16 bytes for
    // a TMA descriptor, and a stage spans two whole groups.
    if (w.n <= 0 || nb4 == 0 || nb4 % 8 != 0 || stage_bytes_of(w.dtype) < 0) return;
    auto aligned = [](const void* p) { return p && (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!aligned(w.qs) || !aligned(w.d) || (has_qh(w.dtype) && !aligned(w.qh)) || (has_min(w.dtype) && !aligned(w.m)))
        return;
    const uint64_t n = uint64_t(w.n);
    bool ok = encode_plane(w.row_maps[0], w.qs, uint64_t(nb4) * qs_bytes(w.dtype), n, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    ok = ok && encode_plane(w.row_maps[2], w.d, uint64_t(nb4) * 2, n, 16, CU_TENSOR_MAP_SWIZZLE_NONE);
    // Formats without the plane pass the d descriptor as a placeholder.
    ok = ok && encode_plane(w.row_maps[1], has_qh(w.dtype) ? static_cast<const void*>(w.qh) : w.d,
                            has_qh(w.dtype) ? uint64_t(nb4) * 4 : uint64_t(nb4) * 2, n, has_qh(w.dtype) ? 32 : 16,
                            has_qh(w.dtype) ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_NONE);
    ok = ok && encode_plane(w.row_maps[3], has_min(w.dtype) ? w.m : w.d, uint64_t(nb4) * 2, n, 16,
                            CU_TENSOR_MAP_SWIZZLE_NONE);
    w.rows_ready = ok;
}

bool gemv_rows_fits(const ActsView& v, const Weight& w) {
    if (!w.rows_ready || v.m < 1 || v.m > GEMV_ROWS_MAX_M) return false;
    if (reinterpret_cast<uintptr_t>(v.q8) & 3) return false;
    const int sb = stage_bytes_of(w.dtype);
    return sb > 0 && gr_smem(1, sb, v.m, round4(w.nb)) <= GR_SMEM_CTA;
}

cudaError_t launch_gemv_rows(const ActsView& v, const Weight& w, const float* bias, float* y, int gx,
                             int* err_flag, cudaStream_t s) {
    if (!gemv_rows_fits(v, w)) return cudaErrorInvalidValue;
    switch (w.dtype) {
        case Q4_0: return gemv_rows_dt<Q4_0>(v, w, bias, y, gx, err_flag, s);
        case Q4_1: return gemv_rows_dt<Q4_1>(v, w, bias, y, gx, err_flag, s);
        case Q5_0: return gemv_rows_dt<Q5_0>(v, w, bias, y, gx, err_flag, s);
        case Q5_1: return gemv_rows_dt<Q5_1>(v, w, bias, y, gx, err_flag, s);
        case Q8_0: return gemv_rows_dt<Q8_0>(v, w, bias, y, gx, err_flag, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace rwq
