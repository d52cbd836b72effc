// rwq_common.cuh -- shared device helpers for the quantized-matmul kernels.
//
// Block formats (ggml, 32 elements per block; quant.rs:43-131):
//   Q4_0 (2): d f16 | qs[16]             q = nib - 8
//   Q4_1 (3): d f16 | m f16 | qs[16]     q = nib,           x = d*q + m
//   Q5_0 (6): d f16 | qh u32 | qs[16]    q = (nib|h<<4) - 16
//   Q5_1 (7): d f16 | m f16 | qh u32 | qs[16]   q = nib|h<<4, x = d*q + m
//   Q8_0 (8): d f16 | q[32] i8
// Element j<16 is the low nibble of qs[j], j>=16 the high nibble of
// qs[j-16]; bit j of qh is element j's fifth bit.
//
// On the device a weight lives as "planes" (same bytes per block as the
// ggml record, split so that code bytes are 16-byte aligned).  Each row is
// padded to nb4 = nb rounded up to a multiple of 4 blocks (pad blocks are
// zero):
//             qs [n][nb4/4][4*QSB]  (QSB = 16, or 32 for Q8_0), see below,
//             qh [n][nb4] u32 (Q5 only, bits permuted: see qh_plane_bits),
//             d [n][nb4] f16 bits, m [n][nb4] f16 bits (Q4_1/Q5_1 only).
// The code plane interleaves each group of four blocks by 4-byte word:
// word w of block b (b = kb % 4) sits at w*16 + b*4 of the group (Q8_0:
// (w%4)*32 + b*8 + (w/4)*4), so one 16-byte load (32 for Q8_0) at c*16
// (c*32) returns word c (and 4+c) of all four blocks -- exactly the
// operand fragment lane c of a quad feeds to an m16n8k32 integer MMA.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <utility>

namespace rwq {

constexpr int QK = 32;

// GELU as tensor.rs:291-306 computes it, same operation order:
//   0.5 * t * (1 + tanh(C * (t + 0.044715 * t * t * t)))
__device__ __forceinline__ float gelu_ref(float t) {
    const float C = 0.7978846f;
    const float cube = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, t), t), t);
    return __fmul_rn(__fmul_rn(0.5f, t), __fadd_rn(1.0f, tanhf(__fmul_rn(C, __fadd_rn(t, cube)))));
}

enum Dtype : int { Q4_0 = 2, Q4_1 = 3, Q5_0 = 6, Q5_1 = 7, Q8_0 = 8 };

__host__ __device__ constexpr int block_bytes(int dt) {
    return dt == Q4_0 ? 18 : dt == Q4_1 ? 20 : dt == Q5_0 ? 22 : dt == Q5_1 ? 24 : dt == Q8_0 ? 34 : -1;
}
__host__ __device__ constexpr bool has_min(int dt) { return dt == Q4_1 || dt == Q5_1; }
__host__ __device__ constexpr bool has_qh(int dt) { return dt == Q5_0 || dt == Q5_1; }
__host__ __device__ constexpr int qs_bytes(int dt) { return dt == Q8_0 ? 32 : 16; }
// Unsigned code offset removed after the integer dot (Q4_0: 8, Q5_0: 16).
__host__ __device__ constexpr int code_offset(int dt) { return dt == Q4_0 ? 8 : dt == Q5_0 ? 16 : 0; }

// Byte offsets of the fields inside a raw ggml block.
__host__ __device__ constexpr int raw_m_off(int) { return 2; }
__host__ __device__ constexpr int raw_qh_off(int dt) { return dt == Q5_0 ? 2 : 4; }
__host__ __device__ constexpr int raw_qs_off(int dt) {
    return dt == Q4_0 ? 2 : dt == Q4_1 ? 4 : dt == Q5_0 ? 6 : dt == Q5_1 ? 8 : 2;
}

// Plane addressing (see the layout above).
__host__ __device__ constexpr int round4(int nb) { return (nb + 3) & ~3; }
// Byte offset of code word w of block b (0..3) inside its 4-block group.
template <int DT>
__host__ __device__ constexpr int qs_word_off(int w, int b) {
    return DT == Q8_0 ? ((w & 3) * 32 + b * 8 + (w >> 2) * 4) : (w * 16 + b * 4);
}
// First byte of the 4-block group holding block kb of row j.
template <int DT>
__host__ __device__ inline size_t qs_group_off(size_t j, int kb, int nb4) {
    return (j * size_t(nb4) + size_t(kb & ~3)) * size_t(qs_bytes(DT));
}

// Exact f16 -> f32 (model.rs:68-86 semantics; the hardware conversion is
// exact for every f16 including subnormals, inf and NaN payloads).
__device__ __forceinline__ float h2f(uint16_t h) {
    float f;
    asm("{ .reg .f16 t; mov.b16 t, %1; cvt.f32.f16 %0, t; }" : "=f"(f) : "h"(h));
    return f;
}

// The Q5 high-bit plane stores ggml's qh with its bits permuted so that a
// code word's four fifth bits come out with one shift and one mask: bit
// 4t+i (element 4t+i, i < 4) moves to bit 8i+t and bit 16+4t+i to bit
// 8i+4+t.  Then for word t (elements 4t..4t+3) the fifth bits are
// (p << (4-t)) & 0x10101010 and for word 4+t (elements 16+4t..) they are
// (p >> t) & 0x10101010; no other bit lands on bit 4 of a byte.  Applied
// once when a weight is uploaded (k_repack).
__host__ __device__ inline uint32_t qh_plane_bits(uint32_t h) {
    uint32_t p = 0;
    for (int e = 0; e < 32; ++e) {
        const int upper = e >> 4, t = (e & 15) >> 2, i = e & 3;
        p |= ((h >> e) & 1u) << (8 * i + 4 * upper + t);
    }
    return p;
}

// Unsigned 5-/4-bit code words for one block: word t < 4 holds elements
// 4t..4t+3, word 4+t holds elements 16+4t..16+4t+3, one code per byte.
// `qh` is the permuted plane word (qh_plane_bits).
template <int DT>
__device__ __forceinline__ void codes_u8x4(const uint4 qs, uint32_t qh, uint32_t (&w)[8]) {
    const uint32_t v[4] = {qs.x, qs.y, qs.z, qs.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        uint32_t lo = v[t] & 0x0F0F0F0Fu;
        uint32_t hi = (v[t] >> 4) & 0x0F0F0F0Fu;
        if (has_qh(DT)) {
            lo |= (qh << (4 - t)) & 0x10101010u;
            hi |= (qh >> t) & 0x10101010u;
        }
        w[t] = lo;
        w[4 + t] = hi;
    }
}

__device__ __forceinline__ int dp4a_su(uint32_t a_s8, uint32_t b_u8, int c) {
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_s8), "r"(b_u8), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a_s8, uint32_t b_s8, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_s8), "r"(b_s8), "r"(c));
    return d;
}

// The integer dots of the GEMV kernels start from the bits of 1.5*2^23
// (minus the Q4_0/Q5_0 code offset times sum(q_a)), so for |S| < 2^22 the
// chain's result read as f32 is 1.5*2^23 + S exactly and S is one FADD.
constexpr uint32_t MAGIC_BITS = 0x4B400000u;  // 12582912.0f
constexpr float MAGIC_F = 12582912.0f;

// Start of the s-th K slice (s >= 1) that k_gemv_mma uses for weight tile
// T, or a value past every group if there is none.  KS > 1: slice s of the
// group range starts at s*ng/KS.  KS == 1: k_gemv_mma's CTA c owns tiles
// [c*tiles/gx, (c+1)*tiles/gx) and its 8 warps split the (tile, group)
// items evenly; a warp range that starts inside tile T splits it there.
__device__ inline int gemv_slice_start(int T, int s, int ks, int ng, int gx, int tiles) {
    constexpr int NONE = 1 << 30;
    if (ks > 1) return s < ks ? s * ng / ks : NONE;
    if (s != 1 || gx <= 0) return NONE;
    int c = int(int64_t(T) * gx / tiles);
    while (c > 0 && int(int64_t(c) * tiles / gx) > T) --c;
    while (c + 1 < gx && int(int64_t(c + 1) * tiles / gx) <= T) ++c;
    const int t_lo = int(int64_t(c) * tiles / gx), t_hi = int(int64_t(c + 1) * tiles / gx);
    const int nt = t_hi - t_lo;
    if (nt < 8) return NONE;   // whole tiles per warp
    const int items = nt * ng, local = (T - t_lo) * ng;
    for (int w = 1; w < 8; ++w) {
        const int i = w * items / 8;
        if (i > local && i < local + ng) return i - local;
    }
    return NONE;
}

// Programmatic dependent launch: a kernel launched with
// launch_pdl() may start while its predecessor on the stream is finishing.
// It must call pdl_wait() before its first global-memory access (read or
// write): that waits until the predecessor grid has completed and its
// memory is visible.  pdl_trigger() lets the successor launch early.  Both
// are no-ops for a normal launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// launch_pdl() with thread-block clusters of `cluster_x` CTAs along x.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, int cluster_x,
                                      cudaStream_t s, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = unsigned(cluster_x);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace rwq
