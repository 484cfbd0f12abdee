// Reference-layout relay attention, forward: every query attends, in one softmax, to the keys of
// its own document within 128 tokens of it and to the 16 relay slots of its document.
//
// Replaces relay_forward_kernel (reuse/crates/dre-attention/src/relay_attention_kernel.rs:38-130;
// launcher relay_forward_cube :214-229; entry run_relay_windowed_attention :311-340) with the same
// contract: q, k, v [B,H,T,64] and relay_k, relay_v [Ndoc,H,16,64] in F (f32 or bf16); doc_id,
// doc_start, doc_end [B,T] (inclusive limits, doc_end < doc_start marks padding); scale 1/8;
// outputs o [B,H,T,64] in F and normalization [B,H,T,2] f32 = (row maximum, sum of exp(score -
// maximum)); a padding row writes o = 0 and (0, 1).
//
// bf16 runs on the tensor cores, one CTA per (b, h, 128 queries):
//   * TMA brings Q [128 x 64] and the key band K, V [384 x 64] (tokens q0 - 128 .. q0 + 255, the
//     union of the tile's windows) into shared memory, 128-byte swizzled; rows outside [0, T) are
//     zero-filled by the copy, and the K / V rows of padding tokens are zeroed before use (the
//     reference never reads them, and a NaN there must not reach 0 * NaN in the P V product);
//   * S = Q K^T (M 128, N 3 x 128, K 64) accumulates in TMEM columns [0, 384);
//   * thread i owns query row i (TMEM lane i): it reads its row's 257 window columns twice (the
//     exact row maximum, then p = exp(s - max) and the sum), adds its 16 relay scores (computed on
//     the CUDA cores while the copies land: a row's relay slots depend on its own document, so
//     the tile has no common relay operand), and writes P [128 x 384] as bf16 in the swizzled
//     K-major layout, zero outside the window;
//   * O = P V (M 128, N 64, K 384, V read MN-major) accumulates in TMEM columns [384, 448);
//   * the epilogue adds the relay values sum_s p_s rv_s, divides by the sum and stores.
// f32 runs on the CUDA cores with the reference's online-softmax order: four lanes per query,
// 16 channels each, scores reduced by two shuffles.
#include <cuda_bf16.h>

#include "common.cuh"
#include "tc_ptx.cuh"

namespace dbl {
namespace {

constexpr int D = 64, RADIUS = 128, SLOTS = 16;
constexpr float SCALE = 0.125f;

// ------------------------------------------------------------------------------ tensor cores
constexpr int TQ = 128;                 // queries per CTA = TMEM lanes
constexpr int KB = TQ + 2 * RADIUS;     // 384 band keys
constexpr int NTH = 128;
constexpr uint32_t OFF_Q = 0;           // [128][128 B]
constexpr uint32_t OFF_K = 16384;       // 3 x [128][128 B]
constexpr uint32_t OFF_V = OFF_K + 49152;
constexpr uint32_t OFF_P = OFF_V + 49152;  // 6 x [128 rows][128 B]: keys 64 a .. 64 a + 63
constexpr uint32_t OFF_BAR = OFF_P + 98304;
constexpr uint32_t SMEM_TC = OFF_BAR + 64 + 1024;  // + alignment slack
constexpr uint32_t TM_O = 384;
constexpr uint32_t IDESC_S = umma_idesc_bf16(128, 128, false);
constexpr uint32_t IDESC_O = umma_idesc_bf16(128, 64, true);
constexpr int kRelayDocError = 101;  // a live row's doc_id outside [0, documents)

struct RelayParams {
    int B, H, T, ndoc;
    const void *q, *k, *v, *rk, *rv;
    const int32_t *doc_id, *doc_start, *doc_end;
    void* o;
    float* norm;
    int* err;
};

__device__ __forceinline__ uint64_t kdesc(uint32_t saddr) { return umma_sdesc_sw128(saddr, 16, 1024); }

__global__ void __launch_bounds__(NTH, 1)
    relay_attn_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const RelayParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bar_ld = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
    uint64_t* bar_s = bar_ld + 1;
    uint64_t* bar_o = bar_ld + 2;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bar_ld + 3);
    int* serr = reinterpret_cast<int*>(tslot + 1);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int T = p.T, tiles = (T + TQ - 1) / TQ;
    const int tile = blockIdx.x % tiles, bh = blockIdx.x / tiles, b = bh / p.H, h = bh % p.H;
    const int q0 = tile * TQ, kb0 = q0 - RADIUS;

    if (tid == 0) {
        prefetch_tmap(&tm_q);
        prefetch_tmap(&tm_k);
        prefetch_tmap(&tm_v);
        mbar_init(bar_ld, 1);
        mbar_init(bar_s, 1);
        mbar_init(bar_o, 1);
        *serr = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tmem_alloc(tslot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    if (tid == 0) {
        mbar_arrive_expect_tx(bar_ld, 16384 + 2 * 49152);
        tma_load_4d(sm + OFF_Q, &tm_q, bar_ld, 0, q0, h, b);
#pragma unroll
        for (int j = 0; j < 3; ++j) {
            tma_load_4d(sm + OFF_K + 16384 * j, &tm_k, bar_ld, 0, kb0 + 128 * j, h, b);
            tma_load_4d(sm + OFF_V + 16384 * j, &tm_v, bar_ld, 0, kb0 + 128 * j, h, b);
        }
    }

    // the row: query t = q0 + tid
    const int t = q0 + tid;
    const bool in_t = t < T;
    int st = 0, en = -1, doc = 0;
    if (in_t) {
        st = p.doc_start[(size_t)b * T + t];
        en = p.doc_end[(size_t)b * T + t];
        doc = p.doc_id[(size_t)b * T + t];
    }
    const bool live = in_t && en >= st;
    const bool relay_ok = live && doc >= 0 && doc < p.ndoc;
    if (live && !relay_ok) atomicExch(p.err, kRelayDocError);
    // window columns (band index = key - kb0), inclusive
    const int lo = max(max(t - RADIUS, st), 0), hi = min(min(t + RADIUS, en), T - 1);
    const int clo = live ? lo - kb0 : 1, chi = live ? hi - kb0 : 0;

    // relay scores on the CUDA cores while the copies land
    float rs[SLOTS];
    const size_t rbase = ((size_t)doc * p.H + h) * SLOTS * D;
    {
        uint4 qv[8];
        const uint4* qg = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.q) +
                                                         (((size_t)b * p.H + h) * T + (in_t ? t : 0)) * D);
#pragma unroll
        for (int i = 0; i < 8; ++i) qv[i] = in_t ? qg[i] : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int s = 0; s < SLOTS; ++s) {
            float acc = 0.f;
            if (relay_ok) {
                const uint4* kg = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.rk) + rbase + s * D);
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const uint4 kv = __ldg(kg + i);
                    acc = fmaf(bf16_lo(qv[i].x), bf16_lo(kv.x), acc);
                    acc = fmaf(bf16_hi(qv[i].x), bf16_hi(kv.x), acc);
                    acc = fmaf(bf16_lo(qv[i].y), bf16_lo(kv.y), acc);
                    acc = fmaf(bf16_hi(qv[i].y), bf16_hi(kv.y), acc);
                    acc = fmaf(bf16_lo(qv[i].z), bf16_lo(kv.z), acc);
                    acc = fmaf(bf16_hi(qv[i].z), bf16_hi(kv.z), acc);
                    acc = fmaf(bf16_lo(qv[i].w), bf16_lo(kv.w), acc);
                    acc = fmaf(bf16_hi(qv[i].w), bf16_hi(kv.w), acc);
                }
            }
            rs[s] = acc * SCALE;
        }
    }

    // padding keys: zero their K and V rows once they have landed
    mbar_wait(bar_ld, 0, serr, 1);
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        const int r = tid + 128 * j, key = kb0 + r;
        if (key >= 0 && key < T && p.doc_end[(size_t)b * T + key] < p.doc_start[(size_t)b * T + key]) {
            uint4* kr = reinterpret_cast<uint4*>(sm + OFF_K + r * 128);
            uint4* vr = reinterpret_cast<uint4*>(sm + OFF_V + r * 128);
#pragma unroll
            for (int i = 0; i < 8; ++i) kr[i] = vr[i] = make_uint4(0u, 0u, 0u, 0u);
        }
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
        tc_fence_after();
        const uint32_t qa = smem_u32addr(sm + OFF_Q), ka = smem_u32addr(sm + OFF_K);
#pragma unroll
        for (int j = 0; j < 3; ++j)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                umma_ss(tmem + 128 * j, kdesc(qa + 32 * kk), kdesc(ka + 16384 * j + 32 * kk), IDESC_S, kk > 0 ? 1u : 0u);
        umma_commit(bar_s);
    }

    // softmax over the row: the warp's rows need band columns [32 w, 32 w + 288)
    mbar_wait(bar_s, 0, serr, 2);
    tc_fence_after();
    const uint32_t trow = tmem + ((uint32_t)(32 * warp) << 16);
    const int cb = 32 * warp;
    float m = -INFINITY;
#pragma unroll 1
    for (int c = 0; c < 18; ++c) {
        uint32_t r[16];
        tmem_ld16(trow + cb + 16 * c, r);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            const int col = cb + 16 * c + e;
            if (col >= clo && col <= chi) m = fmaxf(m, __uint_as_float(r[e]) * SCALE);
        }
    }
    if (relay_ok) {
#pragma unroll
        for (int s = 0; s < SLOTS; ++s) m = fmaxf(m, rs[s]);
    }
    float total = 0.f;
    uint8_t* P = sm + OFF_P;
    const int prow = tid * 128, sw = tid & 7;
#pragma unroll 1
    for (int c = 0; c < 18; ++c) {
        uint32_t r[16];
        tmem_ld16(trow + cb + 16 * c, r);
        tmem_ld_wait();
        uint32_t pk[8];
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
            const int col = cb + 16 * c + e;
            const float p0 = (col >= clo && col <= chi) ? __expf(__uint_as_float(r[e]) * SCALE - m) : 0.f;
            const float p1 = (col + 1 >= clo && col + 1 <= chi) ? __expf(__uint_as_float(r[e + 1]) * SCALE - m) : 0.f;
            total += p0 + p1;
            pk[e / 2] = pack_bf16x2(p0, p1);
        }
        // columns cb + 16 c .. + 15: atom a, 16-byte chunks cc and cc + 1
        const int kc = cb + 16 * c, a = kc >> 6, cc = (kc & 63) >> 3;
        uint8_t* base = P + a * 16384 + prow;
        *reinterpret_cast<uint4*>(base + ((cc ^ sw) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        *reinterpret_cast<uint4*>(base + (((cc + 1) ^ sw) << 4)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
    }
    // the columns outside the warp's range hold zeros
    for (int kc = 0; kc < KB; kc += 8) {
        if (kc >= cb && kc < cb + 288) continue;
        *reinterpret_cast<uint4*>(P + (kc >> 6) * 16384 + prow + ((((kc & 63) >> 3) ^ sw) << 4)) =
            make_uint4(0u, 0u, 0u, 0u);
    }
    float pr[SLOTS];
#pragma unroll
    for (int s = 0; s < SLOTS; ++s) {
        pr[s] = relay_ok ? __expf(rs[s] - m) : 0.f;
        total += pr[s];
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        tc_fence_after();
        const uint32_t pa = smem_u32addr(P), va = smem_u32addr(sm + OFF_V);
#pragma unroll
        for (int kk = 0; kk < KB / 16; ++kk)
            umma_ss(tmem + TM_O, kdesc(pa + 16384 * (kk >> 2) + 32 * (kk & 3)), umma_sdesc_sw128(va + 2048 * kk, 16384, 1024),
                    IDESC_O, kk > 0 ? 1u : 0u);
        umma_commit(bar_o);
    }
    mbar_wait(bar_o, 0, serr, 3);
    tc_fence_after();
    float o[D];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        uint32_t r[16];
        tmem_ld16(trow + TM_O + 16 * c, r);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e) o[16 * c + e] = __uint_as_float(r[e]);
    }
    if (relay_ok) {
#pragma unroll 1
        for (int s = 0; s < SLOTS; ++s) {
            const uint4* vg = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.rv) + rbase + s * D);
            const float w = pr[s];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint4 vv = __ldg(vg + i);
                o[8 * i + 0] = fmaf(w, bf16_lo(vv.x), o[8 * i + 0]);
                o[8 * i + 1] = fmaf(w, bf16_hi(vv.x), o[8 * i + 1]);
                o[8 * i + 2] = fmaf(w, bf16_lo(vv.y), o[8 * i + 2]);
                o[8 * i + 3] = fmaf(w, bf16_hi(vv.y), o[8 * i + 3]);
                o[8 * i + 4] = fmaf(w, bf16_lo(vv.z), o[8 * i + 4]);
                o[8 * i + 5] = fmaf(w, bf16_hi(vv.z), o[8 * i + 5]);
                o[8 * i + 6] = fmaf(w, bf16_lo(vv.w), o[8 * i + 6]);
                o[8 * i + 7] = fmaf(w, bf16_hi(vv.w), o[8 * i + 7]);
            }
        }
    }
    if (in_t) {
        const size_t row = ((size_t)b * p.H + h) * T + t;
        uint4* og = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.o) + row * D);
        const float inv = live ? 1.f / total : 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i)
            og[i] = make_uint4(pack_bf16x2(o[8 * i] * inv, o[8 * i + 1] * inv), pack_bf16x2(o[8 * i + 2] * inv, o[8 * i + 3] * inv),
                               pack_bf16x2(o[8 * i + 4] * inv, o[8 * i + 5] * inv), pack_bf16x2(o[8 * i + 6] * inv, o[8 * i + 7] * inv));
        reinterpret_cast<float2*>(p.norm)[row] = live ? make_float2(m, total) : make_float2(0.f, 1.f);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
    if (tid == 0 && *serr != 0) atomicExch(p.err, *serr);
}

// ------------------------------------------------------------------------------ CUDA cores (f32)
// Four lanes per query (16 channels each), eight queries per warp, 32 per CTA.  Each query walks
// its window keys in order, then its relay slots, with the reference's online update:
// next = first or score > max ? score : max; alpha = first ? 0 : exp(max - next);
// p = exp(score - next); total = total alpha + p; acc = acc alpha + p v.
constexpr int QPB = 32;
__global__ void __launch_bounds__(128) relay_attn_f32_kernel(const RelayParams p) {
    const int T = p.T, tiles = (T + QPB - 1) / QPB;
    const int tile = blockIdx.x % tiles, bh = blockIdx.x / tiles, b = bh / p.H, h = bh % p.H;
    const int lane = threadIdx.x & 31, sub = lane & 3;
    const int t = tile * QPB + (threadIdx.x >> 2);
    const bool in_t = t < T;
    int st = 0, en = -1, doc = 0;
    if (in_t) {
        st = p.doc_start[(size_t)b * T + t];
        en = p.doc_end[(size_t)b * T + t];
        doc = p.doc_id[(size_t)b * T + t];
    }
    const bool live = in_t && en >= st;
    const bool relay_ok = live && doc >= 0 && doc < p.ndoc;
    if (live && !relay_ok && sub == 0) atomicExch(p.err, kRelayDocError);
    const float* hq = static_cast<const float*>(p.q) + ((size_t)b * p.H + h) * T * D;
    const float* hk = static_cast<const float*>(p.k) + ((size_t)b * p.H + h) * T * D;
    const float* hv = static_cast<const float*>(p.v) + ((size_t)b * p.H + h) * T * D;
    float4 qv[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
        qv[i] = in_t ? reinterpret_cast<const float4*>(hq + (size_t)t * D + 16 * sub)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    const int lo = live ? max(max(t - RADIUS, st), 0) : 1, hi = live ? min(min(t + RADIUS, en), T - 1) : 0;
    // the warp walks the union of its queries' ranges so that the shuffles stay converged
    int wlo = live ? lo : 0x7fffffff, whi = live ? hi : -1;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        wlo = min(wlo, __shfl_xor_sync(0xffffffffu, wlo, o));
        whi = max(whi, __shfl_xor_sync(0xffffffffu, whi, o));
    }
    float acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.f;
    float mx = 0.f, total = 0.f;
    auto visit = [&](const float* krow, const float* vrow, bool take) {
        float d = 0.f;
        if (take) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 kv = reinterpret_cast<const float4*>(krow + 16 * sub)[i];
                d = fmaf(qv[i].x, kv.x, d);
                d = fmaf(qv[i].y, kv.y, d);
                d = fmaf(qv[i].z, kv.z, d);
                d = fmaf(qv[i].w, kv.w, d);
            }
        }
        d += __shfl_xor_sync(0xffffffffu, d, 1);
        d += __shfl_xor_sync(0xffffffffu, d, 2);
        if (!take) return;
        const float score = d * SCALE;
        const bool first = total == 0.f;
        const float next = (first || score > mx) ? score : mx;
        const float alpha = first ? 0.f : expf(mx - next);
        const float pw = expf(score - next);
        total = total * alpha + pw;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float4 vv = reinterpret_cast<const float4*>(vrow + 16 * sub)[i];
            acc[4 * i + 0] = acc[4 * i + 0] * alpha + pw * vv.x;
            acc[4 * i + 1] = acc[4 * i + 1] * alpha + pw * vv.y;
            acc[4 * i + 2] = acc[4 * i + 2] * alpha + pw * vv.z;
            acc[4 * i + 3] = acc[4 * i + 3] * alpha + pw * vv.w;
        }
        mx = next;
    };
    for (int key = wlo; key <= whi; ++key) {
        const bool take = key >= lo && key <= hi;
        const int kk = take ? key : lo;  // any in-range row for lanes that skip
        visit(hk + (size_t)kk * D, hv + (size_t)kk * D, take);
    }
    const float* rk = static_cast<const float*>(p.rk) + ((size_t)(relay_ok ? doc : 0) * p.H + h) * SLOTS * D;
    const float* rv = static_cast<const float*>(p.rv) + ((size_t)(relay_ok ? doc : 0) * p.H + h) * SLOTS * D;
    for (int s = 0; s < SLOTS; ++s) visit(rk + s * D, rv + s * D, relay_ok);
    if (in_t) {
        const size_t row = ((size_t)b * p.H + h) * T + t;
        float4* og = reinterpret_cast<float4*>(static_cast<float*>(p.o) + row * D + 16 * sub);
#pragma unroll
        for (int i = 0; i < 4; ++i)
            og[i] = live ? make_float4(acc[4 * i] / total, acc[4 * i + 1] / total, acc[4 * i + 2] / total,
                                       acc[4 * i + 3] / total)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
        if (sub == 0) reinterpret_cast<float2*>(p.norm)[row] = live ? make_float2(mx, total) : make_float2(0.f, 1.f);
    }
}

// ------------------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// 4-D bf16 map over a contiguous [B][H][T][64] array; box {64, 128, 1, 1}, 128-byte swizzle
int make_band_map(CUtensorMap* m, const void* base, int64_t B, int64_t H, int64_t T) {
    static EncodeTiledFn enc = nullptr;
    if (!enc) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult qr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qr) == cudaSuccess &&
            qr == cudaDriverEntryPointSuccess)
            enc = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    if (!enc) return fail(DBL_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)T, (cuuint64_t)H, (cuuint64_t)B};
    cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)(T * D * 2), (cuuint64_t)(H * T * D * 2)};
    cuuint32_t box[4] = {(cuuint32_t)D, 128, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(DBL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return DBL_OK;
}

}  // namespace
}  // namespace dbl

extern "C" int dbl_relay_attention_forward(const dbl_relay_attention_args* a, dbl_stream_t stream) {
    using namespace dbl;
    if (!a) return fail(DBL_ERR_INVALID_ARGUMENT, "relay_attention_forward: null args");
    if (a->batch <= 0 || a->heads <= 0 || a->time <= 0 || a->documents <= 0)
        return fail(DBL_ERR_INVALID_ARGUMENT, "relay_attention_forward: batch, heads, tokens and documents must be positive");
    if (a->head_dim != D)
        return fail(DBL_ERR_UNSUPPORTED, "relay_attention_forward: head width must be 64 (relay_attention_kernel.rs asserts it)");
    if (a->dtype != DBL_F32 && a->dtype != DBL_BF16)
        return fail(DBL_ERR_INVALID_ARGUMENT, "relay_attention_forward: dtype must be f32 or bf16");
    if (!a->q || !a->k || !a->v || !a->relay_k || !a->relay_v || !a->doc_id || !a->doc_start || !a->doc_end || !a->o ||
        !a->normalization)
        return fail(DBL_ERR_INVALID_ARGUMENT, "relay_attention_forward: every pointer is required");
    if (!aligned(a->q, 16) || !aligned(a->k, 16) || !aligned(a->v, 16) || !aligned(a->relay_k, 16) ||
        !aligned(a->relay_v, 16) || !aligned(a->o, 16) || !aligned(a->normalization, 8))
        return fail(DBL_ERR_INVALID_ARGUMENT, "relay_attention_forward: arrays must be 16-byte aligned");
    if (a->time > 0x7fffffffLL || a->heads > 0x7fffffffLL || a->documents > 0x7fffffffLL ||
        a->batch * a->heads * ((a->time + 31) / 32) > 0x7fffffffLL)
        return fail(DBL_ERR_UNSUPPORTED, "relay_attention_forward: axis exceeds 32-bit limits");
    RelayParams p{};
    p.B = (int)a->batch;
    p.H = (int)a->heads;
    p.T = (int)a->time;
    p.ndoc = (int)a->documents;
    p.q = a->q;
    p.k = a->k;
    p.v = a->v;
    p.rk = a->relay_k;
    p.rv = a->relay_v;
    p.doc_id = a->doc_id;
    p.doc_start = a->doc_start;
    p.doc_end = a->doc_end;
    p.o = a->o;
    p.norm = a->normalization;
    int rc = device_error_record(&p.err);
    if (rc != DBL_OK) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (a->dtype == DBL_F32) {
        const size_t tiles = (size_t)(p.T + QPB - 1) / QPB;
        relay_attn_f32_kernel<<<(unsigned)(tiles * p.B * p.H), 128, 0, st>>>(p);
        return launch_status("relay_attn_f32_kernel");
    }
    CUtensorMap mq, mk, mv;
    rc = make_band_map(&mq, a->q, a->batch, a->heads, a->time);
    if (rc == DBL_OK) rc = make_band_map(&mk, a->k, a->batch, a->heads, a->time);
    if (rc == DBL_OK) rc = make_band_map(&mv, a->v, a->batch, a->heads, a->time);
    if (rc != DBL_OK) return rc;
    static bool attr_set = false;
    if (!attr_set) {
        const cudaError_t e =
            cudaFuncSetAttribute(relay_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_TC);
        if (e != cudaSuccess) return cuda_status(e, "relay_attention_forward: cudaFuncSetAttribute");
        attr_set = true;
    }
    const size_t tiles = (size_t)(p.T + TQ - 1) / TQ;
    relay_attn_tc_kernel<<<(unsigned)(tiles * p.B * p.H), NTH, SMEM_TC, st>>>(mq, mk, mv, p);
    return launch_status("relay_attn_tc_kernel");
}
