// Chunked GDN-2 prefill on tcgen05 tensor cores: bf16 q/k/v, K = V = 128, chunk C = 64,
// f32 gates, f32 state (BASELINE configs 1 and 4).
//
// Algorithm (the chunkwise solver of crates/mixers/src/chunk.rs:129-250, with scalar gates and
// the decay products formed in log space instead of the reference's direct products; chunk 64
// instead of its <= 16 because the triangular system is solved by substitution, not by the
// nilpotent series).  For a chunk with start state S (key-major, K x V) and rows r = 0..63:
//   g_r = sum_{u<=r} log2 alpha_u, gamma_r = 2^g_r, Gamma[r][s] = 2^(g_r - g_s) (s <= r);
//   a zero alpha (a reset, or alpha = 0) zeroes every product that spans it.
//   A  = strict_lower(beta_r Gamma[r][s] k_r.k_s)      T = (I + A)^-1
//   R  = beta V - diag(beta gamma) K S                  Delta = T R        (the edits)
//   O  = diag(gamma) (scale Q) S + (scale Gamma o Q K^T, s <= r) Delta
//   S' = gamma_63 S + (diag(Gamma[63][r]) K)^T Delta
// Padding tokens get beta = 0 and alpha = 1 (their edit is exactly zero) and output 0.
//
// B200 mapping.  One CTA per (b, h), 512 threads, one CTA per SM (all 512 TMEM columns); the
// block launches at 128 registers per thread and setmaxnreg moves them to the chain warps.
//   * prep warps 0-7: TMA loads of the chunk tiles (K and Q 128-byte swizzled, V plain), the gate
//     scan, UMMA [K;Q] K^T -> TMEM, decay masks, the 64x64 unit-lower inverse by block doubling
//     (8x8 diagonal blocks by substitution, then 8 -> 16 -> 32 -> 64 joins, the last two on
//     mma.sync tf32 tiles), T and P written as bf16 UMMA operands.  Prep runs one chunk ahead of
//     the chain.  Shared-memory stages: K/Q tiles x 3 (the chain leader loads chunk c + 3 as soon
//     as the MMAs of chunk c are done), gates x 3, V x 2 (loaded two chunks ahead), T / P x 2
//     (handed back to the prep warps through an mbarrier; the prep warps wait for it only when they
//     start writing T and P, after the first half of the inverse), and one output staging tile.
//   * chain warps 8-15: the state-dependent chain, transposed so that the value column j of the
//     state is TMEM lane j and every activation stays in TMEM (A operands of the TS form):
//       MMA1  D1[j][r]  = sum_i S^T[j][i] K[r][i]          (A = S^T bf16 in TMEM; issued as one
//             N = 128 product with DQ[j][r] = sum_i S^T[j][i] Q[r][i] over the [K;Q] rows)
//       E1    R^T[j][r] = beta_r V[r][j] - beta_r gamma_r D1[j][r]   -> TMEM (fp16)
//       MMA2  D2[j][r'] = sum_r R^T[j][r] T[r'][r]          (Delta^T; T in fp16)
//       E2    Delta^T scaled by Gamma[63][r'] (bf16, for MMA3) and plain (fp16, for MMA4) -> TMEM
//       MMA3  D3[j][i]  = sum_r' (Gamma Delta)^T[j][r'] K[r'][i]   (B = K tile read MN-major)
//       MMA4  DP[j][r]  = sum_r' Delta^T[j][r'] P[r][r'],  P = (scale Gamma o Q K^T, s <= r) in fp16
//     Operand formats: MMAs whose B operand is an input tile (K, Q) stay bf16; the ones whose
//     operands are produced inside the kernel (R, T, Delta, P) run in fp16, whose 11-bit mantissa
//     keeps the output error below the bf16-pair scheme's with half the MMAs (tests/chunk_model.py).
//     Magnitudes: T has entries of at most 1 for unit keys and beta <= 1; R, Delta and P are of the
//     order of V and scale; a value beyond fp16 range is reported through dbl_device_error.
//       E3    S[i][j] = gamma_63 S + D3 (f32 master state in registers, 64 per thread),
//             S^T -> TMEM bf16; then MMA1 of the next chunk is issued.  The output
//             O[r][j] = scale gamma_r DQ[j][r] + DP[j][r] -> the chunk's V stage -> TMA store is
//             written while MMA2 of the next chunk runs.
// Roofline: HBM (intensity ~172 FLOP/B at the algorithmic minimum of 1032 B per token-head).
#include <cuda.h>

#include "common.cuh"
#include "tc_ptx.cuh"

namespace dbl {

__device__ int g_tc_error = 0;  // set by a bounded wait that gave up (code = site id) or a range check
constexpr int kTcRangeError = 100;

namespace {

constexpr int C = 64;
constexpr int DK = 128;
constexpr int NTHREADS = 512;
constexpr int NPREP = 256;   // warps 0-7, 112 registers each after setmaxnreg
constexpr int NCHAIN = 256;  // warps 8-15, 144 registers each (the f32 state lives in registers)
constexpr int PREP_REGS = 112, CHAIN_REGS = 144;
static_assert(NPREP * PREP_REGS + NCHAIN * CHAIN_REGS <= 65536, "register split exceeds the launch budget");
constexpr int BAR_PREP = 1, BAR_CHAIN = 2, BAR_SCAN = 3;  // BAR_SCAN: the gate-scan warps 0-1

// TMEM column map (512 columns, f32 accumulators unless noted).  Two 128-column regions alternate
// by chunk parity p = c & 1: region p holds [D1 | DO] of chunk c (K S, then the output accumulator
// that starts as Q S), and region 1 - p holds D3 of chunk c, the state increment.  D3 of chunk c
// lands on [D1 | DO] of chunk c - 1 only after that chunk's output has been read, and [D1 | DO] of
// chunk c + 1 lands on D3 of chunk c only after E3 has read it.
constexpr uint32_t TM_S = 0;      // S^T bf16 A operand: 64 cols (128 keys, 2 per column)
constexpr uint32_t TM_KK = 64;    // prep: [K;Q] K^T, 64 cols
constexpr uint32_t TM_D2 = 128;   // Delta^T (64 cols) -> scaled / plain bf16 in place
constexpr uint32_t TM_R0 = 192;   // regions 0 and 1, 128 cols each (192..447)

// Shared memory (offsets from a 1024-aligned base).  The K/Q tiles and the gates have three stages,
// so the loads of chunk c + 3 go out as soon as the chain is done with chunk c; V, T and P have
// two (V of chunk c + 2 loads as soon as E1 of chunk c has read its stage).
constexpr int NXS = 3;
constexpr uint32_t X_BYTES = 2 * 128 * 128;  // 2 key blocks x 128 rows ([K;Q]) x 128 B, swizzled
constexpr uint32_t V_BYTES = C * 128 * 2;    // [64][128] bf16 plain
constexpr uint32_t T_BYTES = C * 128;        // [64][64] bf16 swizzled
constexpr uint32_t P_BYTES = C * 128;         // [64][64] fp16 swizzled
constexpr uint32_t G_BYTES = 2048;           // gates
constexpr uint32_t OFF_X = 0;
constexpr uint32_t OFF_V = OFF_X + NXS * X_BYTES;
constexpr uint32_t OFF_T = OFF_V + 2 * V_BYTES;
constexpr uint32_t OFF_P = OFF_T + 2 * T_BYTES;
constexpr uint32_t OFF_G = OFF_P + 2 * P_BYTES;
constexpr uint32_t OFF_O = OFF_G + NXS * G_BYTES;  // output staging tile [64][128] bf16
constexpr uint32_t O_BYTES = C * 128 * 2;
constexpr uint32_t OFF_SA = OFF_O + O_BYTES;
constexpr int LDA = 68;   // A rows (16-byte aligned: a lane writes its row with 16-byte stores)
constexpr int LDT = 68;   // T rows (read as float4: 16-byte aligned stride)
constexpr uint32_t OFF_ST = OFF_SA + C * LDA * 4;
constexpr uint32_t OFF_SX = OFF_ST + C * LDT * 4;
constexpr int XLD = 40;   // inverse scratch rows (B-fragment reads hit 32 distinct banks)
constexpr uint32_t OFF_SG = OFF_SX + 1280 * 4;
constexpr uint32_t OFF_SEM = OFF_SG + 64 * 4;   // 2^-g_s (fast decay path), 16-byte aligned
constexpr uint32_t OFF_SCNT = OFF_SEM + 64 * 4;
constexpr uint32_t OFF_SWT = OFF_SCNT + 64 * 4;
constexpr uint32_t OFF_SGT = OFF_SWT + 64;        // gate staging [2][valid, reset, alpha, beta, write][64]
constexpr uint32_t OFF_SDD = OFF_SGT + 2 * 5 * 64 * 4;  // edit-norm partials [4][64] (scores)
constexpr uint32_t OFF_BAR = (OFF_SDD + 4 * 64 * 4 + 7) / 8 * 8;
constexpr uint32_t NBARS = 19;
constexpr uint32_t OFF_TSLOT = OFF_BAR + NBARS * 8;
constexpr uint32_t SMEM_BYTES = OFF_TSLOT + 16 + 1024;  // + alignment slack
static_assert(SMEM_BYTES <= 232448, "shared memory beyond the 227 KB a block can have");
static_assert(OFF_T % 1024 == 0 && OFF_P % 1024 == 0 && T_BYTES % 1024 == 0, "swizzled tiles need 1024-B alignment");
// gate arrays inside a stage's G region (floats)
constexpr int G_CB = 0, G_CG = 64, G_CD = 128, G_OM = 192, G_VAL = 256, G_GC = 320, G_CE = 384, G_KK = 448;
constexpr float kF16Max = 65504.f;

constexpr uint32_t IDESC_M128_N64 = umma_idesc_bf16(128, 64, false);        // [K;Q] K^T on the raw bf16 tiles
constexpr uint32_t IDESC_F16_M128_N128_BMN = umma_idesc_f16(128, 128, true);  // MMA3: B = K (fp16) MN-major
constexpr uint32_t IDESC_F16_M128_N128 = umma_idesc_f16(128, 128, false);     // MMA1: B = [K; Q~] (fp16)
constexpr uint32_t IDESC_F16_M128_N64 = umma_idesc_f16(128, 64, false);

struct TcParams {
    int B, T, H, nchunks;
    float scale;
    const float *alpha, *beta;  // beta: the erase gate (and the write gate unless `write` is set)
    int64_t as[3], bs[3];
    const float* write;         // optional separate write gate (strides ws)
    int64_t ws[3];
    float* out_f32;             // f32 output written directly (instead of the bf16 TMA store), strides os
    int64_t os[3];
    float* scores;              // optional [B,T,H]: |k_t| |edit_t| (0 for padding)
    const int* route;           // optional per-(b,h) flags: the CTA runs only where (route != 0) == route_want
    int route_want;
    const float *valid, *reset;
    const float* initial;
    int init_mode;  // 0 zeros, 1 initial pointer, 2 identity
    int v_zero;     // values treated as zero (span transition)
    int write_out;
    float* final_state;
    int* err;
};

__device__ __forceinline__ uint64_t kdesc(const uint8_t* p) {  // K-major, 128-B swizzle
    return umma_sdesc_sw128(smem_u32addr(p), 16, 1024);
}

// c (16 x 8) += A[16 x 8 ks] B[8 ks x 8] over the k-steps [ks0, ks1) on mma.sync tf32; A and B are
// row-major f32 in shared memory (leading dimensions lda, ldb); g = lane / 4, t4 = lane % 4.
__device__ __forceinline__ void tile_mma_tf32(float (&c)[4], const float* A, int lda, const float* Bm, int ldb,
                                              int ks0, int ks1, int g, int t4) {
    for (int ks = ks0; ks < ks1; ++ks) {
        const float* Ar = A + g * lda + 8 * ks + t4;
        const float* Bc = Bm + (8 * ks + t4) * ldb + g;
        mma_tf32_16x8x8(c, to_tf32(Ar[0]), to_tf32(Ar[8 * lda]), to_tf32(Ar[4]), to_tf32(Ar[8 * lda + 4]),
                        to_tf32(Bc[0]), to_tf32(Bc[4 * ldb]));
    }
}

// Writes sgn * c (a 16 x 8 accumulator fragment) to the row-major f32 tile D.
__device__ __forceinline__ void store_tile(float* D, int ld, const float (&c)[4], int g, int t4, float sgn) {
    *reinterpret_cast<float2*>(D + g * ld + 2 * t4) = make_float2(sgn * c[0], sgn * c[1]);
    *reinterpret_cast<float2*>(D + (g + 8) * ld + 2 * t4) = make_float2(sgn * c[2], sgn * c[3]);
}

// Writes sgn * c as fp16 into a K-major operand tile of 64 columns (128-byte rows, 128-byte swizzle):
// rows row0 + g and row0 + g + 8 (row0 a multiple of 8), 16-byte chunk `chunk` (columns 8 chunk ..).
__device__ __forceinline__ void store_tile_f16(uint8_t* Tt, int row0, int chunk, const float (&c)[4], int g, int t4,
                                               float sgn) {
    const int sw = (chunk ^ g) << 4;
    *reinterpret_cast<uint32_t*>(Tt + (row0 + g) * 128 + sw + 4 * t4) = pack_f16x2(sgn * c[0], sgn * c[1]);
    *reinterpret_cast<uint32_t*>(Tt + (row0 + g + 8) * 128 + sw + 4 * t4) = pack_f16x2(sgn * c[2], sgn * c[3]);
}

__device__ __forceinline__ void zero_tile_16(uint8_t* Tt, int row0, int chunk, int g, int t4) {
    const int sw = (chunk ^ g) << 4;
    *reinterpret_cast<uint32_t*>(Tt + (row0 + g) * 128 + sw + 4 * t4) = 0u;
    *reinterpret_cast<uint32_t*>(Tt + (row0 + g + 8) * 128 + sw + 4 * t4) = 0u;
}

// TRAIN: the training-scan instance (separate write gate, f32 output, scores, route flags); the
// prefill instance compiles without those paths.
template <bool TRAIN>
__global__ void __launch_bounds__(NTHREADS, 1)
    gdn2_prefill_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                           const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                           const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    // routed launches: this (b, h) is served by the other kernel of the call
    if (TRAIN && p.route && ((p.route[blockIdx.x] != 0) != (p.route_want != 0))) return;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* bar_x = bars + 0;      // [3] K/Q tiles landed
    uint64_t* bar_v = bars + 3;      // [2] V tile landed
    uint64_t* bar_prep = bars + 5;   // [2] prep done with the chunk (T, P, gates ready)
    uint64_t* bar_tfree = bars + 7;  // [2] the chain is done with a T / P stage
    uint64_t* bar_kk = bars + 9;
    uint64_t* bar_m1 = bars + 10;
    uint64_t* bar_m2 = bars + 11;
    uint64_t* bar_m3 = bars + 12;
    uint64_t* bar_kkx = bars + 13;  // [3] the [K;Q] K^T MMA of the stage's chunk is complete (its tiles are free)
    uint64_t* bar_gt = bars + 16;   // [3] the stage's gate arrays are written
    uint32_t* tslot = reinterpret_cast<uint32_t*>(smem + OFF_TSLOT);
    int* serr = reinterpret_cast<int*>(smem + OFF_TSLOT + 8);  // the block's wait-error word
    float* sA = reinterpret_cast<float*>(smem + OFF_SA);
    float* sT = reinterpret_cast<float*>(smem + OFF_ST);
    float* sXs = reinterpret_cast<float*>(smem + OFF_SX);
    float* sg = reinterpret_cast<float*>(smem + OFF_SG);
    float* sem = reinterpret_cast<float*>(smem + OFF_SEM);
    int* scnt = reinterpret_cast<int*>(smem + OFF_SCNT);
    float* swt = reinterpret_cast<float*>(smem + OFF_SWT);
    int* swc = reinterpret_cast<int*>(smem + OFF_SWT + 32);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int bh = blockIdx.x;
    const int b = bh / p.H, h = bh - b * p.H;
    const int nchunks = p.nchunks;

    auto stX = [&](int xs) { return smem + OFF_X + xs * X_BYTES; };
    auto stV = [&](int s) { return smem + OFF_V + s * V_BYTES; };
    auto stT = [&](int s) { return smem + OFF_T + s * T_BYTES; };
    auto stP = [&](int s) { return smem + OFF_P + s * P_BYTES; };
    auto stG = [&](int xs) { return reinterpret_cast<float*>(smem + OFF_G + xs * G_BYTES); };

    if (tid == 0) {
        *serr = 0;
        for (int i = 0; i < (int)NBARS; ++i) mbar_init(bars + i, i == 12 ? 2 : 1);  // bar_m3: two issuers
        fence_mbar_init();
        prefetch_tmap(&tm_q);
        prefetch_tmap(&tm_k);
        prefetch_tmap(&tm_v);
        prefetch_tmap(&tm_o);
    }
    if (warp == 0) {
        tmem_alloc(tslot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    // Register split: launched at 512 x 128; prep warpgroups give up 32 each, chain warpgroups take 32.
    if (warp < 8) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(PREP_REGS));
    else asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(CHAIN_REGS));

    auto load_x = [&](int c) {  // K and Q tiles of chunk c into stage c % 3
        const int xs = c % NXS;
        uint8_t* X = stX(xs);
        mbar_arrive_expect_tx(&bar_x[xs], X_BYTES);
#pragma unroll
        for (int ib = 0; ib < 2; ++ib) {
            tma_load_4d(X + ib * 16384, &tm_k, &bar_x[xs], ib * 64, c * C, h, b);
            tma_load_4d(X + ib * 16384 + 8192, &tm_q, &bar_x[xs], ib * 64, c * C, h, b);
        }
    };
    auto load_v = [&](int c) {  // V tile of chunk c into stage c & 1
        if (p.v_zero) return;
        const int s = c & 1;
        mbar_arrive_expect_tx(&bar_v[s], V_BYTES);
        tma_load_4d(stV(s), &tm_v, &bar_v[s], 0, c * C, h, b);
    };

    if (warp < 8) {
        // =================================================================== prep warps
        const int q = warp & 3, half = warp >> 2;
        if (tid == 0) {
            for (int c = 0; c < NXS && c < nchunks; ++c) load_x(c);
            load_v(0);
            if (nchunks > 1) load_v(1);
        }
        // gates of the next chunk are fetched one iteration ahead by asynchronous copies into shared
        // memory, issued by warp 3 (idle during the gate scan; two tokens per lane) and waited for by it
        // before the barrier that ends the iteration, so no scanning warp stalls on them
        float* sgt = reinterpret_cast<float*>(smem + OFF_SGT);
        auto fetch_gates = [&](int c) {
            if (warp != 3) return;
            float* st = sgt + (c & 1) * 320;
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int r = lane + 32 * u, t = c * C + r;
                if (t < p.T) {
                    if (p.valid) cpa_4(st + r, p.valid + (size_t)b * p.T + t);
                    else st[r] = 1.f;
                    if (p.reset) cpa_4(st + 64 + r, p.reset + (size_t)b * p.T + t);
                    else st[64 + r] = 0.f;
                    cpa_4(st + 128 + r, p.alpha + (size_t)b * p.as[0] + (size_t)t * p.as[1] + (size_t)h * p.as[2]);
                    cpa_4(st + 192 + r, p.beta + (size_t)b * p.bs[0] + (size_t)t * p.bs[1] + (size_t)h * p.bs[2]);
                    if (TRAIN && p.write)
                        cpa_4(st + 256 + r, p.write + (size_t)b * p.ws[0] + (size_t)t * p.ws[1] + (size_t)h * p.ws[2]);
                } else {
                    st[r] = 0.f;  // past the end: padding
                }
            }
            cpa_commit();
        };
        fetch_gates(0);
        if (warp == 3) cpa_wait_all();
        named_bar_sync(BAR_PREP, NPREP);
        // P = (scale Gamma o Q K^T, s <= r) in fp16 into stage s, from the Q rows of [K;Q] K^T in TMEM
        // (lanes 64..127, so warps with q = 2, 3): row r = 32 (q - 2) + lane, columns [32 half, 32 half
        // + 32).  Fast path: P[r][s] = (scale 2^g_r) 2^-g_s (q_r . k_s), every factor finite in f32.
        auto write_p = [&](int s, bool fast, const float* G) {
            const int r = 32 * (q - 2) + lane;
            const float vr = G[G_VAL + r];  // a padding row's P row is zero (its output is zero)
            const float gr = sg[r];
            const int cr = scnt[r];
            const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + TM_KK + 32 * half;
            uint32_t gl[32];
            tmem_ld16(ta, *reinterpret_cast<uint32_t(*)[16]>(&gl[0]));
            tmem_ld16(ta + 16, *reinterpret_cast<uint32_t(*)[16]>(&gl[16]));
            tmem_ld_wait();
            const float4* sem4 = reinterpret_cast<const float4*>(sem + 32 * half);
            const int s0 = 32 * half;
            float big = 0.f;
            if (fast) {
                const float er = vr * p.scale * exp2f(gr);
#pragma unroll
                for (int e4 = 0; e4 < 8; ++e4) {
                    const float4 m = sem4[e4];
                    const int e = s0 + 4 * e4;
                    gl[4 * e4] = __float_as_uint(e <= r ? er * m.x * __uint_as_float(gl[4 * e4]) : 0.f);
                    gl[4 * e4 + 1] = __float_as_uint(e + 1 <= r ? er * m.y * __uint_as_float(gl[4 * e4 + 1]) : 0.f);
                    gl[4 * e4 + 2] = __float_as_uint(e + 2 <= r ? er * m.z * __uint_as_float(gl[4 * e4 + 2]) : 0.f);
                    gl[4 * e4 + 3] = __float_as_uint(e + 3 <= r ? er * m.w * __uint_as_float(gl[4 * e4 + 3]) : 0.f);
                }
            } else {
#pragma unroll
                for (int e = 0; e < 32; ++e)
                    gl[e] = __float_as_uint((s0 + e <= r && scnt[s0 + e] == cr) ? vr * p.scale * exp2f(gr - sg[s0 + e]) * __uint_as_float(gl[e]) : 0.f);
            }
            uint8_t* P = stP(s);
#pragma unroll
            for (int x = 0; x < 4; ++x) {
                uint32_t ph[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float v0 = __uint_as_float(gl[8 * x + 2 * u]), v1 = __uint_as_float(gl[8 * x + 2 * u + 1]);
                    big = fmaxf(big, fmaxf(fabsf(v0), fabsf(v1)));
                    ph[u] = pack_f16x2(v0, v1);
                }
                const int cc = 4 * half + x;
                *reinterpret_cast<uint4*>(P + r * 128 + ((cc ^ (r & 7)) << 4)) = make_uint4(ph[0], ph[1], ph[2], ph[3]);
            }
            if (!(big <= kF16Max)) atomicExch(p.err, kTcRangeError);
        };
        for (int c = 0; c < nchunks; ++c) {
            const int s = c & 1, xs = c % NXS;
            const uint32_t xpar = (uint32_t)(c / NXS) & 1u;
            // ---- gates: threads 0..63, token r = tid
            // this chunk's gates (padding: alpha 1, beta 0; a reset zeroes alpha)
            float a = 1.f, be = 0.f, wr = 0.f, vf = 0.f;
            if (tid < C) {
                const float* st = sgt + (c & 1) * 320;
                if (st[tid] != 0.f) {
                    vf = 1.f;
                    a = st[64 + tid] != 0.f ? 0.f : st[128 + tid];
                    be = st[192 + tid];
                    wr = (TRAIN && p.write) ? st[256 + tid] : be;
                }
            }
            if (c + 1 < nchunks) fetch_gates(c + 1);
            if (warp == 2) {
                // [K;Q] K^T on the tensor cores needs only the TMA tiles: warp 2 (outside the gate scan)
                // issues it as soon as they land, so it runs while warps 0-1 scan the gates
                mbar_wait(&bar_x[xs], xpar, serr, 1);
                if (lane == 0) {
                    tc_fence_after();
                    const uint8_t* X = stX(xs);
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint8_t* xa = X + (kk >> 2) * 16384 + (kk & 3) * 32;
                        umma_ss(tmem + TM_KK, kdesc(xa), kdesc(xa), IDESC_M128_N64, kk > 0 ? 1u : 0u);
                    }
                    umma_commit(bar_kk);
                    umma_commit(&bar_kkx[xs]);
                }
                __syncwarp();
            }
            // ---- gates: warps 0-1, token r = tid.  They synchronise among themselves only, so warp 2's
            //      MMA issue above and the idle warps do not hold up the scan.
            float lg = 0.f;
            int z = 0;
            float* G = stG(xs);
            if (tid < C) {
                z = a <= 0.f;
                lg = z ? 0.f : __log2f(a);  // log2 domain: every decay product is one exp2
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const float y = __shfl_up_sync(0xffffffffu, lg, off);
                    const int yc = __shfl_up_sync(0xffffffffu, z, off);
                    if (lane >= off) {
                        lg += y;
                        z += yc;
                    }
                }
                if (lane == 31) {
                    swt[warp] = lg;
                    swc[warp] = z;
                }
                named_bar_sync(BAR_SCAN, C);
                if (tid >= 32) {
                    lg += swt[0];
                    z += swc[0];
                }
                // the chunk's K/Q tiles have landed.  The gate stage c % 3 was last read by the chain
                // in chunk c - 3, which finished before the chain reloaded the stage for chunk c.
                mbar_wait(&bar_x[xs], xpar, serr, 1);
                sg[tid] = lg;
                scnt[tid] = z;
                sem[tid] = exp2f(-lg);
                named_bar_sync(BAR_SCAN, C);
                const float gC = sg[C - 1];
                const int cC = scnt[C - 1];
                const float gamma = (z == 0) ? exp2f(lg) : 0.f;
                G[G_CB + tid] = wr;                // write gate: R = write V - ...
                if (TRAIN) G[G_CE + tid] = be;     // erase gate: rows of A (the prefill's is beta)
                G[G_CG + tid] = be * gamma;
                G[G_CD + tid] = (cC == z) ? exp2f(gC - lg) : 0.f;
                // output: O_r = om_r (Q S)_r + (P Delta)_r with om_r = scale gamma_r
                G[G_OM + tid] = gamma * p.scale;
                G[G_VAL + tid] = vf;
                if (tid == C - 1) G[G_GC] = gamma;
            }
            named_bar_sync(BAR_PREP, NPREP);
            if (tid == 0) mbar_arrive(&bar_gt[xs]);
            mbar_wait(bar_kk, c & 1, serr, 2);
            tc_fence_after();
            // Fast path: no zero decay in the chunk and a bounded total decay, so
            // Gamma[r][s] = 2^g_r 2^-g_s is a rank-1 product (no exponential per element).
            const bool fast = scnt[C - 1] == 0 && sg[C - 1] > -100.f;
            if (q < 2) {
                // A = strict_lower(beta_r Gamma[r][s] k_r.k_s): row r = 32q + lane of [K;Q] K^T,
                // columns s in [32 half, 32 half + 32)
                const int r = 32 * q + lane;
                const float gr = sg[r];
                const int cr = scnt[r];
                const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + TM_KK + 32 * half;
                uint32_t gl[32];
                tmem_ld16(ta, *reinterpret_cast<uint32_t(*)[16]>(&gl[0]));
                tmem_ld16(ta + 16, *reinterpret_cast<uint32_t(*)[16]>(&gl[16]));
                tmem_ld_wait();
                const float4* sem4 = reinterpret_cast<const float4*>(sem + 32 * half);
                const int s0 = 32 * half;
                const float br = TRAIN ? G[G_CE + r] : G[G_CB + r];
                if (TRAIN && p.scores && (r >> 5) == half) {
                    float kk = 0.f;
#pragma unroll
                    for (int e = 0; e < 32; ++e)
                        if (e == (r & 31)) kk = __uint_as_float(gl[e]);
                    G[G_KK + r] = kk;
                }
                if (fast) {
                    const float brer = br * exp2f(gr);
                    float4* Arow = reinterpret_cast<float4*>(sA + r * LDA + s0);
#pragma unroll
                    for (int e4 = 0; e4 < 8; ++e4) {
                        const float4 m = sem4[e4];
                        const int e = s0 + 4 * e4;
                        float4 v;
                        v.x = e < r ? brer * __uint_as_float(gl[4 * e4]) * m.x : 0.f;
                        v.y = e + 1 < r ? brer * __uint_as_float(gl[4 * e4 + 1]) * m.y : 0.f;
                        v.z = e + 2 < r ? brer * __uint_as_float(gl[4 * e4 + 2]) * m.z : 0.f;
                        v.w = e + 3 < r ? brer * __uint_as_float(gl[4 * e4 + 3]) * m.w : 0.f;
                        Arow[e4] = v;
                    }
                } else {
                    float* Af = sA + r * LDA + s0;
#pragma unroll
                    for (int e = 0; e < 32; ++e)
                        Af[e] = (s0 + e < r && scnt[s0 + e] == cr) ? br * exp2f(gr - sg[s0 + e]) * __uint_as_float(gl[e]) : 0.f;
                }
            }
            tc_fence_before();
            named_bar_sync(BAR_PREP, NPREP);
            // ---- T = (I + A)^-1 by block doubling.  Level 0 inverts the eight 8 x 8 diagonal blocks by
            //      substitution; every later level joins pairs of inverted n x n diagonal blocks into
            //      2n x 2n ones through the lower-left block of a unit-lower block inverse,
            //          T10 = -T11 (A10 T00),
            //      and writes zeros to the upper-right block.  8 -> 16 runs in f32 FMAs (one element per
            //      thread), 16 -> 32 and 32 -> 64 on mma.sync tf32 tiles (4 and 8 warps).  Depth: one
            //      8-step substitution and three two-product levels.
            if (tid < C) {
                const int blk = tid >> 3, c0 = tid & 7;
                const float* Ab = sA + (8 * blk) * LDA + 8 * blk;
                // column c0 of the block inverse: x_s = [s == c0] - sum_{s' < s} A[s][s'] x_s'
                float x[8], acc[8];
#pragma unroll
                for (int r = 0; r < 8; ++r) acc[r] = 0.f;
#pragma unroll
                for (int s2 = 0; s2 < 8; ++s2) {
                    x[s2] = (s2 < c0) ? 0.f : (s2 == c0 ? 1.f : -acc[s2]);
#pragma unroll
                    for (int r = s2 + 1; r < 8; ++r) acc[r] = fmaf(Ab[r * LDA + s2], x[s2], acc[r]);
                }
#pragma unroll
                for (int r = 0; r < 8; ++r) sT[(8 * blk + r) * LDT + 8 * blk + c0] = x[r];
            }
            named_bar_sync(BAR_PREP, NPREP);
            {
                // 8 -> 16: pair pr joins the diagonal blocks at a0 = 16 pr and a0 + 8; thread = (pr, i, jj)
                const int pr = tid >> 6, i = (tid >> 3) & 7, jj = tid & 7, a0 = 16 * pr;
                float x = 0.f;
#pragma unroll
                for (int k = 0; k < 8; ++k) x = fmaf(sA[(a0 + 8 + i) * LDA + a0 + k], sT[(a0 + k) * LDT + a0 + jj], x);
                sXs[tid] = x;  // X[pr][i][jj]
                named_bar_sync(BAR_PREP, NPREP);
                float t = 0.f;
#pragma unroll
                for (int k = 0; k < 8; ++k) t = fmaf(sT[(a0 + 8 + i) * LDT + a0 + 8 + k], sXs[64 * pr + 8 * k + jj], t);
                sT[(a0 + 8 + i) * LDT + a0 + jj] = -t;
                sT[(a0 + i) * LDT + a0 + 8 + jj] = 0.f;
            }
            named_bar_sync(BAR_PREP, NPREP);
            // T and P go to stage s: the chain must be done with it (chunk c - 2)
            if (c >= 2) mbar_wait(&bar_tfree[s], (uint32_t)((c - 2) >> 1) & 1u, serr, 3);
            {
                // T goes to the stage as the fp16 K-major UMMA operand (rows r', 64 columns r, 128-byte
                // swizzle) block by block, as soon as each block is final
                const int g = lane >> 2, t4 = lane & 3;
                uint8_t* Tt = stT(s);
                if (q < 2) {
                    // warps 0, 1, 4, 5 -> lw = 0..3.  16 -> 32: lw = (pair pr, column tile nt); X and T10
                    // tiles are 16 x 8 and the second product only needs this warp's own X columns
                    const int lw = (warp & 1) | ((warp >> 2) << 1);
                    const int pr = lw >> 1, nt = lw & 1, a0 = 32 * pr;
                    float* Xp = sXs + pr * (16 * XLD);
                    float c4[4] = {0.f, 0.f, 0.f, 0.f};
                    // T00 is lower triangular: k-steps below 8 nt contribute nothing
                    tile_mma_tf32(c4, sA + (a0 + 16) * LDA + a0, LDA, sT + a0 * LDT + a0 + 8 * nt, LDT, nt, 2, g, t4);
                    store_tile(Xp + 8 * nt, XLD, c4, g, t4, 1.f);
                    __syncwarp();
                    float d[4] = {0.f, 0.f, 0.f, 0.f};
                    tile_mma_tf32(d, sT + (a0 + 16) * LDT + a0 + 16, LDT, Xp + 8 * nt, XLD, 0, 2, g, t4);
                    store_tile(sT + (a0 + 16) * LDT + a0 + 8 * nt, LDT, d, g, t4, -1.f);  // read by 32 -> 64
                    store_tile_f16(Tt, a0 + 16, (a0 >> 3) + nt, d, g, t4, -1.f);
                    zero_tile_16(Tt, a0, ((a0 + 16) >> 3) + nt, g, t4);
                    // then one 16-byte chunk each of the four 16 x 16 diagonal blocks (final since 8 -> 16)
                    const int e = 32 * lw + lane, row = e >> 1, cc = 2 * (row >> 4) + (e & 1);
                    const float4 u = *reinterpret_cast<const float4*>(sT + row * LDT + cc * 8);
                    const float4 w = *reinterpret_cast<const float4*>(sT + row * LDT + cc * 8 + 4);
                    *reinterpret_cast<uint4*>(Tt + row * 128 + ((cc ^ (row & 7)) << 4)) =
                        make_uint4(pack_f16x2(u.x, u.y), pack_f16x2(u.z, u.w), pack_f16x2(w.x, w.y),
                                   pack_f16x2(w.z, w.w));
                } else if (p.write_out) {
                    // warps 2, 3, 6, 7 meanwhile: P from the Q rows of [K;Q] K^T (only the output
                    // reads P: a launch without outputs, the span maps, skips it and MMA4)
                    write_p(s, fast, G);
                    tc_fence_before();  // these TMEM reads precede the next chunk's [K;Q] K^T
                }
                named_bar_sync(BAR_PREP, NPREP);
                // 32 -> 64: warp = (row tile mt, column tile nt) of the 32 x 32 lower-left block
                const int mt = warp >> 2, nt = warp & 3;
                float c4[4] = {0.f, 0.f, 0.f, 0.f};
                tile_mma_tf32(c4, sA + (32 + 16 * mt) * LDA, LDA, sT + 8 * nt, LDT, nt, 4, g, t4);
                store_tile(sXs + 16 * mt * XLD + 8 * nt, XLD, c4, g, t4, 1.f);
                named_bar_sync(BAR_PREP, NPREP);
                float d[4] = {0.f, 0.f, 0.f, 0.f};
                // T11 is lower triangular: rows 16 mt .. 16 mt + 15 need k-steps below 2 mt + 2
                tile_mma_tf32(d, sT + (32 + 16 * mt) * LDT + 32, LDT, sXs + 8 * nt, XLD, 0, 2 * mt + 2, g, t4);
                store_tile_f16(Tt, 32 + 16 * mt, nt, d, g, t4, -1.f);
                zero_tile_16(Tt, 16 * mt, 4 + nt, g, t4);
            }
            fence_proxy_async_smem();
            if (warp == 3) cpa_wait_all();  // the next chunk's gates are in shared memory
            named_bar_sync(BAR_PREP, NPREP);
            if (tid == 0) mbar_arrive(&bar_prep[s]);
        }
    } else {
        // =================================================================== chain warps
        const int ct = tid - NPREP;
        const int q = warp & 3, hh = (warp - 8) >> 2;
        const int j = 32 * q + lane;  // state value column == TMEM lane
        const uint32_t tl = tmem + ((uint32_t)(32 * q) << 16);
        float S[64];  // S[i][j], i = 64 hh + e
        const size_t sbase = (size_t)bh * DK * DK;
#pragma unroll
        for (int e = 0; e < 64; ++e) {
            const int i = 64 * hh + e;
            float x = 0.f;
            if (p.init_mode == 1) x = p.initial[sbase + (size_t)i * DK + j];
            else if (p.init_mode == 2) x = (i == j) ? 1.f : 0.f;
            S[e] = x;
        }
        // S^T as the fp16 A operand of MMA1 (an S beyond fp16 range makes Delta non-finite, which E2
        // reports)
        // The K and Q tiles of chunk cn to fp16 in place, Q rows scaled by their output multiplier
        // om_r = scale gamma_r (0 for padding), so that MMA1 gives om o (Q S) and MMA4 adds P Delta onto
        // it.  Runs once the [K;Q] K^T MMA that read the tiles as bf16 is complete and the chunk's gate
        // arrays are written.  Four 8 KB blocks (K and Q of the two key blocks); thread ct converts the
        // 16-byte chunks ct and ct + 256 of each, rows ct / 8 and ct / 8 + 32.  An fp16 overflow here
        // (inputs far outside unit norm) makes Delta or the output non-finite, which is reported.
        auto convert_x = [&](int cn) {
            const int xn = cn % NXS;
            const uint32_t pn = (uint32_t)(cn / NXS) & 1u;
            mbar_wait(&bar_kkx[xn], pn, serr, 9);
            mbar_wait(&bar_gt[xn], pn, serr, 10);
            const float* Gn = stG(xn);
            uint8_t* X = stX(xn);
            float f[2];
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const int row = (ct >> 3) + 32 * i;
                f[i] = Gn[G_VAL + row] != 0.f ? Gn[G_OM + row] : 0.f;
            }
#pragma unroll
            for (int blk = 0; blk < 4; ++blk) {
                // the Q blocks (odd) feed only the Q S half of MMA1, which only the output reads: a
                // launch without outputs leaves them as they are (that half then holds values nothing
                // reads; each MMA1 column depends on its own row of [K;Q] only)
                if ((blk & 1) && !p.write_out) continue;
                uint4* base = reinterpret_cast<uint4*>(X + blk * 8192) + ct;
                uint4 u[2];
#pragma unroll
                for (int i = 0; i < 2; ++i) u[i] = base[256 * i];
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    uint32_t w[4] = {u[i].x, u[i].y, u[i].z, u[i].w};
#pragma unroll
                    for (int k2 = 0; k2 < 4; ++k2)
                        w[k2] = (blk & 1) ? pack_f16x2(f[i] * bf16_lo(w[k2]), f[i] * bf16_hi(w[k2]))
                                          : pack_f16x2(bf16_lo(w[k2]), bf16_hi(w[k2]));
                    base[256 * i] = make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
            fence_proxy_async_smem();  // the converted tiles are read by MMA1 and MMA3 (async proxy)
        };
        auto store_state_op = [&]() {
#pragma unroll
            for (int pc = 0; pc < 4; ++pc) {
                uint32_t pk[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) pk[u] = pack_f16x2(S[16 * pc + 2 * u], S[16 * pc + 2 * u + 1]);
                tmem_st8(tl + TM_S + 32 * hh + 8 * pc, pk);
            }
        };
        // MMA1 of chunk c (issued by the chain leader): one N = 128 product over the 128 rows [K;Q] of
        // each key block, D[j][r] = sum_i S^T[j][i] K[r][i] into D1 and D[j][64 + r] = sum_i S^T[j][i]
        // Q[r][i] into DO (the Q S half of the output, which only needs the chunk-start state)
        auto issue_mma1 = [&](int c) {
            mbar_wait(&bar_prep[c & 1], (c >> 1) & 1, serr, 4);
            tc_fence_after();
            const uint8_t* X = stX(c % NXS);
            const uint32_t tr = TM_R0 + 128 * (c & 1);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk)
                umma_ts(tmem + tr, tmem + TM_S + 8 * kk, kdesc(X + (kk >> 2) * 16384 + (kk & 3) * 32),
                        IDESC_F16_M128_N128, kk > 0 ? 1u : 0u);
            umma_commit(bar_m1);
        };
        // Output of chunk cc: O[r][j] = scale gamma_r DQ[j][r] + DP[j][r] (0 for padding rows) into the
        // staging tile, as bf16 for the TMA store.  DQ sits in the upper half
        // of region cc & 1; MMA3 of chunk cc + 1 overwrites it and MMA4 of chunk cc + 1 overwrites DP,
        // so this runs in chunk cc + 1 between MMA2 and the barrier that precedes those MMAs.
        // Output of chunk cc: O[r][j] = om_r (Q S)[r][j] + (P Delta)[r][j], accumulated in the upper half of
        // region cc & 1 by MMA1 (Q rows pre-scaled by om_r, zero for padding) and MMA4 (P rows of
        // padding zero), into the staging tile as bf16 for the TMA store (f32 straight to global memory
        // in the training-scan instance).  MMA3 of chunk cc + 1 overwrites the region, so this runs in
        // chunk cc + 1 between MMA2 and the barrier that precedes MMA3.
        auto write_output = [&](int cc) {
            const uint32_t tdq = TM_R0 + 128 * (cc & 1) + 64;
            uint32_t o[32];
            tmem_ld16(tl + tdq + 32 * hh, *reinterpret_cast<uint32_t(*)[16]>(&o[0]));
            tmem_ld16(tl + tdq + 32 * hh + 16, *reinterpret_cast<uint32_t(*)[16]>(&o[16]));
            tmem_ld_wait();
            float big = 0.f;
#pragma unroll
            for (int e = 0; e < 32; ++e) big = fmaxf(big, fabsf(__uint_as_float(o[e])));
            if (!(big <= 3.0e38f)) atomicExch(p.err, kTcRangeError);  // inf or NaN: an fp16 operand overflowed
            if (TRAIN) {
                // f32 rows straight to global memory: a warp writes 32 consecutive values per row
                // (the row pointer and stride are formed once: per-element 64-bit index products cost
                // about a fifth of the call; the tail chunk keeps static indices into o)
                const int t0 = cc * C + 32 * hh;
                const int64_t rs = p.os[1];
                float* orow = p.out_f32 + (size_t)b * p.os[0] + (size_t)h * p.os[2] + j + (size_t)t0 * rs;
                if (t0 + 32 <= p.T) {
#pragma unroll
                    for (int e = 0; e < 32; ++e) orow[e * rs] = __uint_as_float(o[e]);
                } else {
#pragma unroll
                    for (int e = 0; e < 32; ++e)
                        if (e < p.T - t0) orow[e * rs] = __uint_as_float(o[e]);
                }
                return;
            }
            __nv_bfloat16* Os = reinterpret_cast<__nv_bfloat16*>(smem + OFF_O);
#pragma unroll
            for (int e = 0; e < 32; ++e) Os[(32 * hh + e) * 128 + j] = __float2bfloat16_rn(__uint_as_float(o[e]));
            fence_proxy_async_smem();
        };
        convert_x(0);
        store_state_op();
        tmem_st_wait();
        tc_fence_before();
        named_bar_sync(BAR_CHAIN, NCHAIN);
        if (ct == 0) issue_mma1(0);

        for (int c = 0; c < nchunks; ++c) {
            const int s = c & 1, xs = c % NXS;
            const uint32_t par = c & 1;
            const uint32_t TM_D1 = TM_R0 + 128 * (c & 1);        // K S -> R^T (bf16 hi/lo) in place
            const uint32_t TM_D3 = TM_R0 + 128 * ((c & 1) ^ 1);  // (Gamma Delta)^T K, 128 cols
            mbar_wait(&bar_prep[s], (c >> 1) & 1, serr, 4);
            const float* G = stG(xs);
            const float gC = G[G_GC];
            mbar_wait(bar_m1, par, serr, 5);
            if (!p.v_zero) mbar_wait(&bar_v[s], (uint32_t)(c >> 1) & 1u, serr, 8);
            tc_fence_after();
            // ---- E1: R^T[j][r] = beta_r V[r][j] - beta_r gamma_r (K S)[r][j],  r in [32 hh, 32 hh + 32),
            //      written in place as fp16 pairs (r, r + 1) to columns [32 hh, 32 hh + 16)
            {
                const __nv_bfloat16* Vs = reinterpret_cast<const __nv_bfloat16*>(stV(s));
                uint32_t a[32];
                tmem_ld16(tl + TM_D1 + 32 * hh, *reinterpret_cast<uint32_t(*)[16]>(&a[0]));
                tmem_ld16(tl + TM_D1 + 32 * hh + 16, *reinterpret_cast<uint32_t(*)[16]>(&a[16]));
                tmem_ld_wait();
                const float2* cb2 = reinterpret_cast<const float2*>(G + G_CB + 32 * hh);
                const float2* cg2 = reinterpret_cast<const float2*>(G + G_CG + 32 * hh);
#pragma unroll
                for (int pc = 0; pc < 2; ++pc) {
                    uint32_t pk[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const float2 cb = cb2[8 * pc + u], cg = cg2[8 * pc + u];
                        float x[2];
#pragma unroll
                        for (int w = 0; w < 2; ++w) {
                            const int e = 16 * pc + 2 * u + w;
                            const int r = 32 * hh + e;
                            const float vv = p.v_zero ? 0.f : __bfloat162float(Vs[r * 128 + j]);
                            x[w] = (w ? cb.y : cb.x) * vv - (w ? cg.y : cg.x) * __uint_as_float(a[e]);
                        }
                        pk[u] = pack_f16x2(x[0], x[1]);
                    }
                    tmem_st8(tl + TM_D1 + 32 * hh + 8 * pc, pk);
                }
                tmem_st_wait();
            }
            tc_fence_before();
            named_bar_sync(BAR_CHAIN, NCHAIN);
            // ---- MMA2: D2[j][r'] = sum_r R^T[j][r] T[r'][r]   (fp16; rows r = 16 kk .. 16 kk + 15 of R^T are
            //      TMEM columns 32 (kk / 2) + 8 (kk % 2) ..); then V stage s, read by E1, takes V of chunk c + 2
            if (ct == 0) {
                tc_fence_after();
                const uint8_t* Tt = stT(s);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_ts(tmem + TM_D2, tmem + TM_D1 + 32 * (kk >> 1) + 8 * (kk & 1), kdesc(Tt + kk * 32),
                            IDESC_F16_M128_N64, kk > 0 ? 1u : 0u);
                umma_commit(bar_m2);
                if (c + 2 < nchunks) load_v(c + 2);
            }
            // while MMA2 runs: the output of chunk c - 1
            if (p.write_out && c >= 1) write_output(c - 1);
            mbar_wait(bar_m2, par, serr, 6);
            tc_fence_after();
            // ---- E2: Delta^T for r' in [32 hh, 32 hh + 32), in place: for the 16 rows of columns
            //      [16k, 16k + 16), the Gamma[63][r']-scaled copy (bf16, MMA3) goes to [16k, +8) and the
            //      plain copy (fp16, MMA4) to [16k + 8, +8)
            {
                uint32_t d[32];
                tmem_ld16(tl + TM_D2 + 32 * hh, *reinterpret_cast<uint32_t(*)[16]>(&d[0]));
                tmem_ld16(tl + TM_D2 + 32 * hh + 16, *reinterpret_cast<uint32_t(*)[16]>(&d[16]));
                tmem_ld_wait();
                float big = 0.f;
#pragma unroll
                for (int pc = 0; pc < 2; ++pc) {
                    const uint32_t col = TM_D2 + 32 * hh + 16 * pc;
                    uint32_t ps[8], pp[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const int e = 16 * pc + 2 * u;
                        const int r = 32 * hh + e;
                        const float x0 = __uint_as_float(d[e]), x1 = __uint_as_float(d[e + 1]);
                        big = fmaxf(big, fmaxf(fabsf(x0), fabsf(x1)));
                        ps[u] = pack_f16x2(x0 * G[G_CD + r], x1 * G[G_CD + r + 1]);
                        pp[u] = pack_f16x2(x0, x1);
                    }
                    tmem_st8(tl + col, ps);
                    tmem_st8(tl + col + 8, pp);
                }
                // an fp16 operand overflowed (R or T, so Delta is not finite) or Delta itself is out of
                // fp16 range: report it (the NaN test is the negated comparison)
                if (!(big <= kF16Max)) atomicExch(p.err, kTcRangeError);
                if (TRAIN && p.scores) {
                    // |edit_r|^2 = sum_j Delta[r][j]^2: a reduce-scatter over the warp's 32 columns
                    // (lane l ends with row 32 hh + l), then the four warps of a row half in shared memory
                    float v[32];
#pragma unroll
                    for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(d[e]) * __uint_as_float(d[e]);
                    const bool up16 = lane & 16, up8 = lane & 8, up4 = lane & 4, up2 = lane & 2, up1 = lane & 1;
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const float keep = up16 ? v[e + 16] : v[e], send = up16 ? v[e] : v[e + 16];
                        v[e] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
                    }
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const float keep = up8 ? v[e + 8] : v[e], send = up8 ? v[e] : v[e + 8];
                        v[e] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
                    }
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float keep = up4 ? v[e + 4] : v[e], send = up4 ? v[e] : v[e + 4];
                        v[e] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
                    }
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const float keep = up2 ? v[e + 2] : v[e], send = up2 ? v[e] : v[e + 2];
                        v[e] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
                    }
                    {
                        const float keep = up1 ? v[1] : v[0], send = up1 ? v[0] : v[1];
                        v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 1);
                    }
                    reinterpret_cast<float*>(smem + OFF_SDD)[q * 64 + 32 * hh + lane] = v[0];
                }
                tmem_st_wait();
            }
            tc_fence_before();
            named_bar_sync(BAR_CHAIN, NCHAIN);
            if (TRAIN && p.scores && ct < C) {
                // score_r = |k_r| |edit_r| (0 for padding, whose edit is exactly zero)
                const float* sdd = reinterpret_cast<const float*>(smem + OFF_SDD);
                const float dd = sdd[ct] + sdd[64 + ct] + sdd[128 + ct] + sdd[192 + ct];
                const int t = c * C + ct;
                if (t < p.T) p.scores[((size_t)b * p.T + t) * p.H + h] = G[G_VAL + ct] != 0.f ? sqrtf(G[G_KK + ct] * dd) : 0.f;
            }
            // ---- MMA3: D3 = (Gamma Delta)^T K (state increment) issued by thread 0 of the chain, MMA4:
            //      DP = Delta^T P^T (output) by thread 32 (independent accumulators; bar_m3 counts both commits)
            if (ct == 0) {
                if (!TRAIN && p.write_out && c >= 1) {
                    tma_store_4d(&tm_o, smem + OFF_O, 0, (c - 1) * C, h, b);
                    tma_store_commit();
                }
                tc_fence_after();
                const uint8_t* X = stX(xs);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    umma_ts(tmem + TM_D3, tmem + TM_D2 + 16 * kk,
                            umma_sdesc_sw128(smem_u32addr(X + kk * 2048), 16384, 1024), IDESC_F16_M128_N128_BMN,
                            kk > 0 ? 1u : 0u);
                umma_commit(bar_m3);
            } else if (ct == 32) {
                tc_fence_after();
                if (p.write_out) {
                    const uint8_t* P = stP(s);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        umma_ts(tmem + TM_R0 + 128 * (c & 1) + 64, tmem + TM_D2 + 16 * kk + 8, kdesc(P + kk * 32),
                                IDESC_F16_M128_N64, 1u);  // onto om o (Q S): the output
                }
                umma_commit(bar_m3);
            }
            // while MMA3 / MMA4 run: the next chunk's tiles to fp16 (read by its MMA1 after E3)
            if (c + 1 < nchunks) convert_x(c + 1);
            mbar_wait(bar_m3, par, serr, 7);
            tc_fence_after();
            // every MMA of chunk c is done: its K/Q stage takes chunk c + 3, and its T / P stage goes
            // back to the prep warps
            if (ct == 0) {
                if (c + NXS < nchunks) load_x(c + NXS);
                mbar_arrive(&bar_tfree[s]);
                // the staging tile is written again in chunk c + 1 (after the barrier that ends E3)
                tma_store_wait_read0();
            }
            // ---- E3: state update (f32 master copy) and its bf16 image for the next MMA1
            {
#pragma unroll
                for (int pc = 0; pc < 2; ++pc) {
                    uint32_t d[32];
                    tmem_ld16(tl + TM_D3 + 64 * hh + 32 * pc, *reinterpret_cast<uint32_t(*)[16]>(&d[0]));
                    tmem_ld16(tl + TM_D3 + 64 * hh + 32 * pc + 16, *reinterpret_cast<uint32_t(*)[16]>(&d[16]));
                    tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 32; ++e) S[32 * pc + e] = fmaf(gC, S[32 * pc + e], __uint_as_float(d[e]));
                }
                store_state_op();
                tmem_st_wait();
            }
            tc_fence_before();
            named_bar_sync(BAR_CHAIN, NCHAIN);
            // the recurrence moves on (the output of chunk c is written during MMA2 of chunk c + 1)
            if (ct == 0 && c + 1 < nchunks) issue_mma1(c + 1);
            // ---- end of chunk c
        }
        if (p.write_out && nchunks > 0) {
            // the last chunk's output (its MMAs completed before its E3)
            write_output(nchunks - 1);
            tc_fence_before();
            named_bar_sync(BAR_CHAIN, NCHAIN);
            if (ct == 0 && !TRAIN) {
                tma_store_4d(&tm_o, smem + OFF_O, 0, (nchunks - 1) * C, h, b);
                tma_store_commit();
            }
        }
        if (p.final_state) {
#pragma unroll
            for (int e = 0; e < 64; ++e) p.final_state[sbase + (size_t)(64 * hh + e) * DK + j] = S[e];
        }
        if (ct == 0) tma_store_wait_all0();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
    if (tid == 0 && *serr != 0) atomicExch(p.err, *serr);  // reported by dbl_device_error
}

// ------------------------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult qr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qr) == cudaSuccess &&
            qr == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    return fn;
}

// 4-D bf16 map over [B][T][H][128] with element strides `st` (st[3] == 1); box {box0, 64, 1, 1}.
int make_map(CUtensorMap* m, const void* base, int64_t B, int64_t T, int64_t H, const int64_t* st, uint32_t box0,
             bool swizzle) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(DBL_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[4] = {128, (cuuint64_t)T, (cuuint64_t)H, (cuuint64_t)B};
    cuuint64_t strides[3] = {(cuuint64_t)st[1] * 2, (cuuint64_t)st[2] * 2, (cuuint64_t)st[0] * 2};
    cuuint32_t box[4] = {box0, (cuuint32_t)C, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(DBL_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return DBL_OK;
}

bool tma_strides_ok(const void* base, const int64_t* st) {
    if (!base || !aligned(base, 16) || st[3] != 1) return false;
    for (int d = 0; d < 3; ++d)
        if (st[d] <= 0 || (st[d] * 2) % 16 != 0 || st[d] * 2 >= (int64_t(1) << 40)) return false;
    return true;
}

}  // namespace

int tc_prefill_supported(const dbl_prefill_args* a, const int64_t* qs, const int64_t* ks, const int64_t* vs,
                         const int64_t* os) {
    if (a->dtype != DBL_BF16 || a->key_dim != 128 || a->value_dim != 128) return 0;
    if (a->chunk_size != 0 && a->chunk_size != 64) return 0;
    if (!tma_strides_ok(a->q, qs) || !tma_strides_ok(a->k, ks)) return 0;
    if (a->v && !tma_strides_ok(a->v, vs)) return 0;
    if (a->out && !tma_strides_ok(a->out, os)) return 0;
    if (a->batch * a->heads > 0x7fffffffLL) return 0;
    return 1;
}

int tc_prefill_launch(const dbl_prefill_args* a, const int64_t* qs, const int64_t* ks, const int64_t* vs,
                      const int64_t* as, const int64_t* bs, const int64_t* os, int mode, float* transition,
                      cudaStream_t st) {
    CUtensorMap mq, mk, mv, mo;
    int rc = make_map(&mq, mode == 1 ? a->k : a->q, a->batch, a->time, a->heads, mode == 1 ? ks : qs, 64, true);
    if (rc == DBL_OK) rc = make_map(&mk, a->k, a->batch, a->time, a->heads, ks, 64, true);
    if (rc == DBL_OK) {
        const bool hv = mode == 0 && a->v;
        rc = make_map(&mv, hv ? a->v : a->k, a->batch, a->time, a->heads, hv ? vs : ks, 128, false);
    }
    const bool write_out = mode == 0 && a->out != nullptr;
    if (rc == DBL_OK) rc = make_map(&mo, write_out ? a->out : a->k, a->batch, a->time, a->heads, write_out ? os : ks, 128, false);
    if (rc != DBL_OK) return rc;
    TcParams p{};
    p.B = (int)a->batch;
    p.T = (int)a->time;
    p.H = (int)a->heads;
    p.nchunks = (int)((a->time + C - 1) / C);
    p.scale = a->scale;
    p.alpha = a->alpha;
    p.beta = a->beta;
    for (int d = 0; d < 3; ++d) {
        p.as[d] = as[d];
        p.bs[d] = bs[d];
    }
    p.valid = a->valid;
    p.reset = a->reset;
    if (mode == 1) {
        p.init_mode = 2;
        p.v_zero = 1;
        p.write_out = 0;
        p.final_state = transition;
    } else {
        p.init_mode = a->initial_state ? 1 : 0;
        p.initial = a->initial_state;
        p.v_zero = 0;
        p.write_out = write_out ? 1 : 0;
        p.final_state = a->final_state;
    }
    int* err = nullptr;
    cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_tc_error);
    if (e != cudaSuccess) return cuda_status(e, "prefill_tc: error record");
    p.err = err;
    static std::atomic<uint64_t> attr_done{0};
    rc = once_per_device(attr_done, [] {
        return cuda_status(cudaFuncSetAttribute(gdn2_prefill_tc_kernel<false>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES),
                           "prefill_tc: cudaFuncSetAttribute");
    });
    if (rc != DBL_OK) return rc;
    gdn2_prefill_tc_kernel<false><<<(unsigned)(a->batch * a->heads), NTHREADS, SMEM_BYTES, st>>>(mq, mk, mv, mo, p);
    return launch_status("gdn2_prefill_tc_kernel");
}

// The reference's stateful training scan (dbl_gdn_training_scan) on this kernel: bf16 q/k/v
// [B,T,H,128] contiguous, gates read at channel 0 of the channel-wise [B,T,H,K|V] arrays (the caller
// has checked, per (b, h), that they are constant across channels: `route`), separate erase and
// write gates, valid / reset masks, optional initial and final states, f32 output and scores.  CTAs
// whose route flag differs from `route_want` return at once.
bool tc_training_scan_supported(const dbl_training_scan_args* a) {
    if (a->dtype != DBL_BF16 || a->key_dim != 128 || a->value_dim != 128) return false;
    if (a->batch * a->heads > 0x7fffffffLL) return false;
    for (const void* ptr : {a->q, a->k, a->v})
        if (!aligned(ptr, 16)) return false;
    return aligned(a->output, 16);
}

int tc_training_scan_launch(const dbl_training_scan_args* a, const int* route, int route_want, cudaStream_t st) {
    const int64_t T = a->time, H = a->heads;
    const int64_t st4[4] = {T * H * 128, H * 128, 128, 1};
    CUtensorMap mq, mk, mv, mo;
    int rc = make_map(&mq, a->q, a->batch, T, H, st4, 64, true);
    if (rc == DBL_OK) rc = make_map(&mk, a->k, a->batch, T, H, st4, 64, true);
    if (rc == DBL_OK) rc = make_map(&mv, a->v, a->batch, T, H, st4, 128, false);
    if (rc == DBL_OK) rc = make_map(&mo, a->k, a->batch, T, H, st4, 128, false);  // unused: f32 output path
    if (rc != DBL_OK) return rc;
    TcParams p{};
    p.B = (int)a->batch;
    p.T = (int)T;
    p.H = (int)H;
    p.nchunks = (int)((T + C - 1) / C);
    p.scale = 1.f;  // the training scan takes q as it is
    p.alpha = a->alpha;
    p.beta = a->erase;
    p.write = a->write;
    const int64_t gk[3] = {T * H * a->key_dim, H * a->key_dim, a->key_dim};
    const int64_t gv[3] = {T * H * a->value_dim, H * a->value_dim, a->value_dim};
    for (int d = 0; d < 3; ++d) {
        p.as[d] = gk[d];
        p.bs[d] = gk[d];
        p.ws[d] = gv[d];
        p.os[d] = gv[d];
    }
    p.valid = a->valid;
    p.reset = a->reset;
    p.init_mode = a->initial_state ? 1 : 0;
    p.initial = a->initial_state;
    p.v_zero = 0;
    p.write_out = 1;
    p.out_f32 = a->output;
    p.scores = a->scores;
    p.final_state = a->final_state;
    p.route = route;
    p.route_want = route_want;
    int* err = nullptr;
    cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&err), g_tc_error);
    if (e != cudaSuccess) return cuda_status(e, "prefill_tc: error record");
    p.err = err;
    static std::atomic<uint64_t> attr_done{0};
    rc = once_per_device(attr_done, [] {
        return cuda_status(cudaFuncSetAttribute(gdn2_prefill_tc_kernel<true>,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES),
                           "prefill_tc: cudaFuncSetAttribute");
    });
    if (rc != DBL_OK) return rc;
    gdn2_prefill_tc_kernel<true><<<(unsigned)(a->batch * a->heads), NTHREADS, SMEM_BYTES, st>>>(mq, mk, mv, mo, p);
    return launch_status("gdn2_prefill_tc_kernel (training scan)");
}

int device_error_record(int** out) {
    const cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(out), g_tc_error);
    return e == cudaSuccess ? DBL_OK : cuda_status(e, "device error record");
}

}  // namespace dbl

extern "C" int dbl_device_error(int* code) {
    int host = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&host, dbl::g_tc_error, sizeof(int));
    if (e != cudaSuccess) return dbl::cuda_status(e, "dbl_device_error");
    if (host != 0) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(dbl::g_tc_error, &zero, sizeof(int));
        if (e != cudaSuccess) return dbl::cuda_status(e, "dbl_device_error");
    }
    if (code) *code = host;
    if (host == dbl::kTcRangeError)
        return dbl::fail(DBL_ERR_UNSUPPORTED,
                         "tensor-core prefill: an fp16 MMA operand left fp16 range (inputs far outside unit-norm keys "
                         "and beta in [0, 1]); its outputs are not valid");
    if (host == 101)
        return dbl::fail(DBL_ERR_INVALID_ARGUMENT,
                         "relay attention: a live row's document id lies outside [0, documents); its relay slots "
                         "were skipped");
    return host ? dbl::fail(DBL_ERR_TIMEOUT, "a kernel gave up a bounded wait (site %d)", host) : DBL_OK;
}
