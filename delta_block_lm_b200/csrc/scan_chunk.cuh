// Pieces shared by the chunked GDN-2 scan (scan_chunk.cu) and its backward (scan_chunk_bwd.cu):
// the chunk length, the per-chunk map block layout, cp.async staging and small shared-memory
// matrix tiles.
#pragma once

#include "common.cuh"

namespace dbl {
namespace chunk {

constexpr int CC = 16;      // tokens per chunk
constexpr int CVMAX = 128;  // value width limit of the chunked path
constexpr int CTH = 256;

// Per-chunk block of the workspace, in floats.  The part every column group reads (Qe, B', G with
// rows padded to KP = K rounded up to 4, plus 4, so that two rows read by one warp fall in different
// banks; |k_t|) comes first, then the column-sliced part (O0, U0, H as rows of V).
// With `extra` (the backward's use) the block also keeps Q' = q (.) P, Wd, P (rows of KP) and M, Ti.
struct ChunkBlock {
    int kp, qe, bp, g, kn, sh, o0, u0, hh, qp, wd, pp, mm, ti, total;
};
__host__ __device__ inline ChunkBlock chunk_block(int K, int V, bool extra = false) {
    ChunkBlock L{};
    L.kp = ((K + 3) & ~3) + 4;
    int o = 0;
    L.qe = o; o += CC * L.kp;
    L.bp = o; o += CC * L.kp;
    L.g = o; o += K * L.kp;
    L.kn = o; o += CC;
    L.sh = o;
    L.o0 = o; o += CC * V;
    L.u0 = o; o += CC * V;
    L.hh = o; o += K * V;
    o = (o + 3) & ~3;
    if (extra) {
        L.qp = o; o += CC * L.kp;
        L.wd = o; o += CC * L.kp;
        L.pp = o; o += CC * L.kp;
        L.mm = o; o += CC * CC;
        L.ti = o; o += CC * CC;
    }
    L.total = (o + 3) & ~3;  // 16-byte aligned blocks
    return L;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
// waits until at most `pending` (0..2) of this thread's most recent cp.async groups are in flight
__device__ __forceinline__ void cp_async_wait_pending(int pending) {
    if (pending <= 0) asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    else if (pending == 1) asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    else asm volatile("cp.async.wait_group 2;\n" ::: "memory");
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    return x;
}

__device__ __forceinline__ float4 lds4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// acc[r][c] += sum_{s < CC} A[(r0 + r) lda + s] Bm[s ldb + n0 + c] for a 2 x 4 tile: A rows are
// contiguous in s, Bm rows contiguous in n; every operand is read four at a time (16-byte aligned).
__device__ __forceinline__ void tile_mm(float (&acc)[2][4], const float* A, int lda, int r0, const float* Bm,
                                        int ldb, int n0) {
#pragma unroll
    for (int s = 0; s < CC; s += 4) {
        const float4 b0 = lds4(Bm + (s + 0) * ldb + n0), b1 = lds4(Bm + (s + 1) * ldb + n0);
        const float4 b2 = lds4(Bm + (s + 2) * ldb + n0), b3 = lds4(Bm + (s + 3) * ldb + n0);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const float4 a = lds4(A + (r0 + r) * lda + s);
            acc[r][0] = fmaf(a.x, b0.x, fmaf(a.y, b1.x, fmaf(a.z, b2.x, fmaf(a.w, b3.x, acc[r][0]))));
            acc[r][1] = fmaf(a.x, b0.y, fmaf(a.y, b1.y, fmaf(a.z, b2.y, fmaf(a.w, b3.y, acc[r][1]))));
            acc[r][2] = fmaf(a.x, b0.z, fmaf(a.y, b1.z, fmaf(a.z, b2.z, fmaf(a.w, b3.z, acc[r][2]))));
            acc[r][3] = fmaf(a.x, b0.w, fmaf(a.y, b1.w, fmaf(a.z, b2.w, fmaf(a.w, b3.w, acc[r][3]))));
        }
    }
}


}  // namespace chunk
}  // namespace dbl
