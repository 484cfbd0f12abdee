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
//   * the relay slots of the tile's documents (up to 8 distinct documents, gathered by TMA) give
//     S_relay = Q RK^T (N = 16 per document) in TMEM columns [384, 384 + 16 J);
//   * the four warps that share TMEM lane quarter qd (rows 32 qd ..) split the 288 band columns
//     their rows can reach into chunks of 16 and take the exact row maximum and then p = exp(s -
//     max) and the sum in two passes, exchanging per-row partials through shared memory; column
//     group 0 adds the row's own document's relay scores;
//   * after a barrier that closes every read of S, P (bf16 pairs, zero outside the window and
//     outside the row's document group) overwrites S in TMEM, and O = P V + P_relay RV (A from
//     TMEM, V read MN-major) accumulates in TMEM columns [192, 256);
//   * the epilogue divides by the sum and stores, each column group 16 output channels.
// A tile with more than 8 documents computes its relay scores and values on the CUDA cores.
// f32 runs on the CUDA cores with the reference's online-softmax order: four lanes per query,
// 16 channels each, scores reduced by two shuffles.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "tc_ptx.cuh"

namespace dbl {
namespace {

constexpr int D = 64, RADIUS = 128, SLOTS = 16;
constexpr float SCALE = 0.125f;

// ------------------------------------------------------------------------------ tensor cores
constexpr int TQ = 128;                 // queries per tile = TMEM lanes
constexpr int KB = TQ + 2 * RADIUS;     // 384 band keys: blocks t - 1, t, t + 1 of 128 keys
constexpr int NTH = 512;                // 16 warps: lane quarter = warp % 4, column group = warp / 4
constexpr int JMAX = 4;                 // relay documents per tile on the tensor cores
constexpr int EMPTY_DOC = -1;
// shared memory: Q double-buffered, key and value blocks in rings of 4 (block j in slot j % 4), the
// relay slots double-buffered, then the per-tile bookkeeping (double-buffered where tile u + 1 is
// prepared while tile u runs)
constexpr uint32_t OFF_Q = 0;                 // 2 x [128][128 B]
constexpr uint32_t OFF_K = 32768;             // 4 x [128][128 B]
constexpr uint32_t OFF_V = OFF_K + 65536;     // 4 x [128][128 B]
constexpr uint32_t OFF_RK = OFF_V + 65536;    // 2 x JMAX x [16][128 B]
constexpr uint32_t OFF_RV = OFF_RK + 16384;   // 2 x JMAX x [16][128 B]
constexpr uint32_t OFF_RED = OFF_RV + 16384;  // f32 [2][4][128]: per-group row maxima and sums
constexpr uint32_t OFF_ROW = OFF_RED + 4096;  // int4 [2][128]: window columns, relay group, document
constexpr uint32_t OFF_PR = OFF_ROW + 4096;   // f32 [128][16]: relay weights (CUDA-core relay)
constexpr uint32_t OFF_DOC = OFF_PR + 8192;   // int [2][8]: JMAX documents, overflow flag
constexpr uint32_t OFF_PAD = OFF_DOC + 64;    // u32 [2][12]: padding bits of the band keys to load
constexpr uint32_t OFF_META = OFF_PAD + 128;  // int [3][128] rows (start, end, id), [2][384] keys (start, end)
constexpr uint32_t OFF_BAR = OFF_META + 4608;
constexpr uint32_t SMEM_TC = OFF_BAR + 128 + 1024;  // + alignment slack
// TMEM columns: S of the band [0, 384) and of the relay slots [384, 384 + 16 J); once the softmax
// has read them, P of the band (bf16 pairs) [0, 192), O in two partial sums [192, 256) and
// [320, 384), P of the relay slots [256, 256 + 8 J)
constexpr uint32_t TM_SR = 384, TM_O = 192, TM_PR = 256, TM_O2 = 320;
constexpr uint32_t IDESC_S = umma_idesc_bf16(128, 128, false);
constexpr uint32_t IDESC_S256 = umma_idesc_bf16(128, 256, false);
constexpr uint32_t IDESC_O = umma_idesc_bf16(128, 64, true);
constexpr int ISSUER2 = 128;  // the second MMA-issuing thread (warp 4): the product chains are split in two
constexpr int LOADER = 256;   // the thread (warp 8) that issues the next tile's copies
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
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }
__device__ __forceinline__ uint64_t mndesc(uint32_t saddr) { return umma_sdesc_sw128(saddr, 16384, 1024); }

// dot of a bf16 row of 64 (eight 16-byte words already in registers) with a bf16 row in memory
__device__ __forceinline__ float dot64(const uint4 (&qv)[8], const __nv_bfloat16* row) {
    const uint4* kg = reinterpret_cast<const uint4*>(row);
    float acc = 0.f;
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
    return acc;
}

// The persistent kernel: CTA c takes the tiles [c NT / G, (c + 1) NT / G) of the (b, h)-major tile
// order, NT = B H ceil(T / 128), G = gridDim.x.  Consecutive tiles of one (b, h) share two of their
// three key blocks, so a tile loads Q and one new key / value block, issued while the previous tile
// computes; a change of (b, h) loads all three blocks once the previous tile's products are done.
__global__ void __launch_bounds__(NTH, 1)
    relay_attn_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_rk,
                         const __grid_constant__ CUtensorMap tm_rv, const RelayParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* smax = reinterpret_cast<float*>(sm + OFF_RED);  // [4][128]
    float* ssum = smax + 512;                              // [4][128]
    int4* srow = reinterpret_cast<int4*>(sm + OFF_ROW);    // [2][128]
    float* spr = reinterpret_cast<float*>(sm + OFF_PR);
    int* sdoc = reinterpret_cast<int*>(sm + OFF_DOC);      // [2][8]: [0, JMAX) documents, [JMAX] overflow
    uint32_t* spad = reinterpret_cast<uint32_t*>(sm + OFF_PAD);  // [2][12]
    uint64_t* bar_ld = reinterpret_cast<uint64_t*>(sm + OFF_BAR);  // [2]
    uint64_t* bar_rl = bar_ld + 2;                                 // [2]
    uint64_t* bar_s = bar_ld + 4;
    uint64_t* bar_o = bar_ld + 5;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bar_ld + 6);
    int* serr = reinterpret_cast<int*>(tslot + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int qd = warp & 3, g = warp >> 2;     // TMEM lane quarter, column group
    const int r = 32 * qd + lane;               // the row (query of the tile) this thread works on
    const int T = p.T, tps = (T + TQ - 1) / TQ;
    const int64_t NT = (int64_t)p.B * p.H * tps;
    const int64_t ubeg = NT * blockIdx.x / gridDim.x, uend = NT * (blockIdx.x + 1) / gridDim.x;
    if (ubeg >= uend) return;

    if (tid == 0) {
        prefetch_tmap(&tm_q);
        prefetch_tmap(&tm_k);
        prefetch_tmap(&tm_v);
        prefetch_tmap(&tm_rk);
        prefetch_tmap(&tm_rv);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bar_ld[i], 1);
            mbar_init(&bar_rl[i], 1);
        }
        mbar_init(bar_s, 2);
        mbar_init(bar_o, 2);
        *serr = 0;
        fence_mbar_init();
    }
    if (tid < 16) sdoc[tid] = (tid & 7) < JMAX ? EMPTY_DOC : 0;
    if (tid < 24) spad[tid] = 0u;
    if (warp == 0) {
        tmem_alloc(tslot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint32_t trow = tmem + ((uint32_t)(32 * qd) << 16);

    // ---- per-tile preparation, run by column group 0 (thread = row r): the row's window columns and
    // relay group into srow[buf], its document into sdoc[buf] (deduplicated), and the padding bits of
    // the band keys this tile loads into spad[buf] (all three blocks, or only the third).  The
    // metadata arrives by cp.async into shared memory (no register waits on it), each thread
    // copying and later reading only its own row and keys.
    int* mrow = reinterpret_cast<int*>(sm + OFF_META);  // [3][128]
    int* mkey = mrow + 384;                             // [2][384]
    auto fetch_meta = [&](int bh, int t, bool full) {
        const int b = bh / p.H, q0 = t * TQ, kb0 = q0 - RADIUS;
        if (q0 + r < T) {
            cp_async4(&mrow[r], p.doc_start + (size_t)b * T + q0 + r);
            cp_async4(&mrow[128 + r], p.doc_end + (size_t)b * T + q0 + r);
            cp_async4(&mrow[256 + r], p.doc_id + (size_t)b * T + q0 + r);
        } else {
            mrow[r] = 0;
            mrow[128 + r] = -1;
            mrow[256 + r] = 0;
        }
#pragma unroll
        for (int jb = 0; jb < 3; ++jb) {
            const int key = kb0 + 128 * jb + r, kk = 128 * jb + r;
            if ((full || jb == 2) && key >= 0 && key < T) {
                cp_async4(&mkey[kk], p.doc_start + (size_t)b * T + key);
                cp_async4(&mkey[384 + kk], p.doc_end + (size_t)b * T + key);
            } else {
                mkey[kk] = 0;
                mkey[384 + kk] = 0;
            }
        }
    };
    auto prepare = [&](int t, int buf) {
        cp_async_wait_all();
        const int st = mrow[r], en = mrow[128 + r], doc = mrow[256 + r];
        const int q0 = t * TQ, kb0 = q0 - RADIUS, tq = q0 + r;
        const bool live = tq < T && en >= st;
        const bool relay_ok = live && doc >= 0 && doc < p.ndoc;
        if (live && !relay_ok) atomicExch(p.err, kRelayDocError);
        // deduplicate within the warp first: one leader per distinct document takes a slot
        const unsigned peers = __match_any_sync(0xffffffffu, relay_ok ? doc : -2 - lane);
        const int leader = __ffs(peers) - 1;
        int jr = -1;
        if (relay_ok && lane == leader) {
            for (int k = 0; k < JMAX; ++k) {
                const int prev = atomicCAS(&sdoc[buf * 8 + k], EMPTY_DOC, doc);
                if (prev == EMPTY_DOC || prev == doc) {
                    jr = k;
                    break;
                }
            }
            if (jr < 0) atomicOr(&sdoc[buf * 8 + JMAX], 1);
        }
        jr = __shfl_sync(0xffffffffu, jr, leader);
        if (!relay_ok) jr = -1;
        const int lo = max(max(tq - RADIUS, st), 0), hi = min(min(tq + RADIUS, en), T - 1);
        srow[buf * 128 + r] = make_int4(live ? lo - kb0 : 1, live ? hi - kb0 : 0, jr, live ? (relay_ok ? doc : -2) : -1);
        unsigned bits[3];
#pragma unroll
        for (int jb = 0; jb < 3; ++jb) bits[jb] = __ballot_sync(0xffffffffu, mkey[384 + 128 * jb + r] < mkey[128 * jb + r]);
        if (lane == 0) {
#pragma unroll
            for (int jb = 0; jb < 3; ++jb) spad[buf * 12 + 4 * jb + qd] = bits[jb];
        }
    };
    // TMA of tile (bh, t)'s Q and its new key / value blocks
    auto load_tile = [&](int bh, int t, int buf, bool full) {
        const int b = bh / p.H, h = bh % p.H;
        mbar_arrive_expect_tx(&bar_ld[buf], 16384u + (full ? 3u : 1u) * 32768u);
        tma_load_4d(sm + OFF_Q + 16384 * buf, &tm_q, &bar_ld[buf], 0, t * TQ, h, b);
        for (int jb = full ? 0 : 2; jb < 3; ++jb) {
            const int blk = t - 1 + jb, slot = blk & 3;
            tma_load_4d(sm + OFF_K + 16384 * slot, &tm_k, &bar_ld[buf], 0, 128 * blk, h, b);
            tma_load_4d(sm + OFF_V + 16384 * slot, &tm_v, &bar_ld[buf], 0, 128 * blk, h, b);
        }
    };
    // TMA of tile (bh, t)'s relay slots; armed with zero bytes when the tile has none, so that every
    // tile completes one phase of bar_rl[buf]
    auto load_relay = [&](int bh, int buf) {
        const int h = bh % p.H;
        int J = 0;
        for (int k = 0; k < JMAX; ++k) J += sdoc[buf * 8 + k] != EMPTY_DOC;
        const bool tc = sdoc[buf * 8 + JMAX] == 0;
        mbar_arrive_expect_tx(&bar_rl[buf], tc ? 4096u * (uint32_t)J : 0u);
        if (tc)
            for (int j = 0; j < J; ++j) {
                tma_load_4d(sm + OFF_RK + 8192 * buf + 2048 * j, &tm_rk, &bar_rl[buf], 0, 0, h, sdoc[buf * 8 + j]);
                tma_load_4d(sm + OFF_RV + 8192 * buf + 2048 * j, &tm_rv, &bar_rl[buf], 0, 0, h, sdoc[buf * 8 + j]);
            }
    };

    int cur_bh = (int)(ubeg / tps), cur_t = (int)(ubeg % tps);
    if (g == 0) {
        fetch_meta(cur_bh, cur_t, true);
        prepare(cur_t, 0);
    }
    __syncthreads();
    if (tid == 0) {
        load_tile(cur_bh, cur_t, 0, true);
        load_relay(cur_bh, 0);
    }

    const int ntile = (int)(uend - ubeg);
    for (int i = 0; i < ntile; ++i) {
        const int buf = i & 1;
        const uint32_t ph2 = (uint32_t)(i >> 1) & 1u, ph1 = (uint32_t)i & 1u;
        const int bh = cur_bh, t = cur_t, b = bh / p.H, h = bh % p.H;
        const int q0 = t * TQ;
        const bool has_next = i + 1 < ntile, next_same = has_next && t + 1 < tps;
        const int nbh = next_same ? bh : bh + 1, nt = next_same ? t + 1 : 0;
        int J = 0;
#pragma unroll
        for (int k = 0; k < JMAX; ++k) J += sdoc[buf * 8 + k] != EMPTY_DOC;
        const bool tc_relay = sdoc[buf * 8 + JMAX] == 0;
        const int4 ri = srow[buf * 128 + r];
        const int clo = ri.x, chi = ri.y, jr = ri.z, rdoc = ri.w;
        const size_t rbase = ((size_t)(rdoc >= 0 ? rdoc : 0) * p.H + h) * SLOTS * D;
        // the next tile's metadata copies go out now; they are used while this tile's O products run
        if (g == 0 && has_next) fetch_meta(nbh, nt, !next_same);

        // the tile's copies have landed: zero the rows of padding keys among the new blocks
        mbar_wait(&bar_ld[buf], ph2, serr, 1);
        if (tid < KB && (spad[buf * 12 + tid / 32] >> (tid & 31) & 1u)) {
            const int slot = (t - 1 + tid / 128) & 3;
            uint4* kr = reinterpret_cast<uint4*>(sm + OFF_K + 16384 * slot + (tid & 127) * 128);
            uint4* vr = reinterpret_cast<uint4*>(sm + OFF_V + 16384 * slot + (tid & 127) * 128);
#pragma unroll
            for (int e = 0; e < 8; ++e) kr[e] = vr[e] = make_uint4(0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        // the other buffer's bookkeeping is free (tile u - 1 is complete): clear it for tile u + 1
        if (tid < 8) sdoc[(buf ^ 1) * 8 + tid] = tid < JMAX ? EMPTY_DOC : 0;
        if (tid >= 32 && tid < 44) spad[(buf ^ 1) * 12 + tid - 32] = 0u;
        if (tid == 0 || tid == ISSUER2) {
            // two chains over the three band blocks: the two blocks that sit in adjacent ring slots
            // go as one N = 256 product (blocks t - 1, t unless block t - 1 is in the last slot)
            const uint32_t qa = smem_u32addr(sm + OFF_Q + 16384 * buf), ka = smem_u32addr(sm + OFF_K);
            const bool lead_pair = ((t - 1) & 3) != 3;
            const bool mine_wide = (tid == 0) == lead_pair;  // this issuer takes the N = 256 chain
            const int jb0 = tid == 0 ? 0 : (lead_pair ? 2 : 1);
            const uint32_t idesc = mine_wide ? IDESC_S256 : IDESC_S;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                umma_ss(tmem + 128 * jb0, kdesc(qa + 32 * kk), kdesc(ka + 16384 * ((t - 1 + jb0) & 3) + 32 * kk), idesc,
                        kk > 0 ? 1u : 0u);
            if (tid == ISSUER2) {
                mbar_wait(&bar_rl[buf], ph2, serr, 2);
                if (tc_relay && J > 0) {
                    tc_fence_after();
                    const uint32_t ra = smem_u32addr(sm + OFF_RK + 8192 * buf), idesc = umma_idesc_bf16(128, 16 * J, false);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        umma_ss(tmem + TM_SR, kdesc(qa + 32 * kk), kdesc(ra + 32 * kk), idesc, kk > 0 ? 1u : 0u);
                }
            }
            umma_commit(bar_s);
        }
        // the next tile of this (b, h) needs Q and one new block, whose slots tile u - 1 has released
        if (tid == LOADER && next_same) load_tile(nbh, nt, buf ^ 1, false);
        // more documents than the tensor-core relay holds: relay scores on the CUDA cores
        float rs[SLOTS];
#pragma unroll
        for (int s = 0; s < SLOTS; ++s) rs[s] = 0.f;
        if (!tc_relay && g == 0 && rdoc >= 0) {
            uint4 qv[8];
            const uint4* qg = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(p.q) +
                                                             (((size_t)b * p.H + h) * T + q0 + r) * D);
#pragma unroll
            for (int e = 0; e < 8; ++e) qv[e] = qg[e];
#pragma unroll
            for (int s = 0; s < SLOTS; ++s)
                rs[s] = dot64(qv, static_cast<const __nv_bfloat16*>(p.rk) + rbase + s * D) * SCALE;
        }

        // ---- softmax: this warp reads columns [cb + 16 c0, cb + 16 c1) of its lane quarter's band span
        mbar_wait(bar_s, ph1, serr, 3);
        tc_fence_after();
        const int cb = 32 * qd, c0 = (18 * g) / 4, c1 = (18 * (g + 1)) / 4;
        // raw scores: max(s) / 8 is max(s / 8) exactly.  A chunk inside every lane's window (most of
        // them) takes the unmasked loop; one outside every window is skipped.
        float mraw = -INFINITY;
        auto max_chunk = [&](const uint32_t (&v)[16], int cs) {
            if (__all_sync(0xffffffffu, cs >= clo && cs + 15 <= chi)) {
#pragma unroll
                for (int e = 0; e < 16; ++e) mraw = fmaxf(mraw, __uint_as_float(v[e]));
            } else if (!__all_sync(0xffffffffu, cs > chi || cs + 15 < clo)) {
#pragma unroll
                for (int e = 0; e < 16; ++e)
                    if (cs + e >= clo && cs + e <= chi) mraw = fmaxf(mraw, __uint_as_float(v[e]));
            }
        };
        // the warp's 4 or 5 chunks stay in registers for both passes: one TMEM wait
        uint32_t sv[80];
        tmem_ld32(trow + cb + 16 * c0, &sv[0]);
        tmem_ld32(trow + cb + 16 * (c0 + 2), &sv[32]);
        if (c0 + 4 < c1) tmem_ld16(trow + cb + 16 * (c0 + 4), *reinterpret_cast<uint32_t(*)[16]>(&sv[64]));
        tmem_ld_wait();
#pragma unroll
        for (int k = 0; k < 5; ++k)
            if (c0 + k < c1) max_chunk(*reinterpret_cast<const uint32_t(*)[16]>(&sv[16 * k]), cb + 16 * (c0 + k));
        float m = mraw * SCALE;
        // relay scores (column group 0): this row's document group of the relay columns
        if (g == 0) {
            if (tc_relay) {
                for (int j = 0; j < J; ++j) {
                    uint32_t v[16];
                    tmem_ld16(trow + TM_SR + 16 * j, v);
                    tmem_ld_wait();
                    if (j == jr) {
#pragma unroll
                        for (int s = 0; s < SLOTS; ++s) rs[s] = __uint_as_float(v[s]) * SCALE;
                    }
                }
            }
            if (rdoc >= 0) {
#pragma unroll
                for (int s = 0; s < SLOTS; ++s) m = fmaxf(m, rs[s]);
            }
        }
        smax[g * 128 + r] = m;
        __syncthreads();
        m = fmaxf(fmaxf(smax[r], smax[128 + r]), fmaxf(smax[256 + r], smax[384 + r]));
        float total = 0.f;
        // p = exp(s / 8 - m) packed to bf16 pairs; s / 8 - m is formed exactly before the
        // exponential (scores far below zero stay exact).  The pairs of a chunk overwrite the
        // first half of its registers (pair e / 2 is written after scores e, e + 1 are read).
        auto exp_chunk = [&](uint32_t (&v)[16], int cs) {
            uint32_t (&out)[16] = v;
            if (__all_sync(0xffffffffu, cs >= clo && cs + 15 <= chi)) {
#pragma unroll
                for (int e = 0; e < 16; e += 2) {
                    const float p0 = __expf(fmaf(__uint_as_float(v[e]), SCALE, -m));
                    const float p1 = __expf(fmaf(__uint_as_float(v[e + 1]), SCALE, -m));
                    total += p0 + p1;
                    out[e / 2] = pack_bf16x2(p0, p1);
                }
            } else if (__all_sync(0xffffffffu, cs > chi || cs + 15 < clo)) {
#pragma unroll
                for (int e = 0; e < 8; ++e) out[e] = 0u;
            } else {
#pragma unroll
                for (int e = 0; e < 16; e += 2) {
                    const int col = cs + e;
                    const float p0 = (col >= clo && col <= chi) ? __expf(fmaf(__uint_as_float(v[e]), SCALE, -m)) : 0.f;
                    const float p1 =
                        (col + 1 >= clo && col + 1 <= chi) ? __expf(fmaf(__uint_as_float(v[e + 1]), SCALE, -m)) : 0.f;
                    total += p0 + p1;
                    out[e / 2] = pack_bf16x2(p0, p1);
                }
            }
        };
#pragma unroll
        for (int k = 0; k < 5; ++k)
            if (c0 + k < c1) exp_chunk(*reinterpret_cast<uint32_t(*)[16]>(&sv[16 * k]), cb + 16 * (c0 + k));
        uint32_t prk[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
        if (g == 0 && rdoc >= 0) {
            float pr[SLOTS];
#pragma unroll
            for (int s = 0; s < SLOTS; ++s) {
                pr[s] = __expf(rs[s] - m);
                total += pr[s];
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) prk[e] = pack_bf16x2(pr[2 * e], pr[2 * e + 1]);
            if (!tc_relay) {
#pragma unroll
                for (int s = 0; s < SLOTS; ++s) spr[r * SLOTS + s] = pr[s];
            }
        }
        ssum[g * 128 + r] = total;
        tc_fence_before();
        __syncthreads();  // every read of S is complete: P may now overwrite it
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 5; ++k)
            if (c0 + k < c1)
                tmem_st8(trow + (uint32_t)(16 * qd + 8 * (c0 + k)), *reinterpret_cast<const uint32_t(*)[8]>(&sv[16 * k]));
        {
            // P columns outside the lane quarter's span [16 qd, 16 qd + 144) are zero: six groups of 8
            const uint32_t zero[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
            for (int zc = g; zc < 6; zc += 4) {
                const int col = zc < 2 * qd ? 8 * zc : 16 * qd + 144 + 8 * (zc - 2 * qd);
                tmem_st8(trow + (uint32_t)col, zero);
            }
            if (g == 0 && tc_relay) {
                // one warp-wide store per document group; each lane supplies its row's values
                for (int j = 0; j < J; ++j) {
                    uint32_t val[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) val[e] = j == jr ? prk[e] : 0u;
                    tmem_st8(trow + TM_PR + 8 * j, val);
                }
            }
        }
        tmem_st_wait();
        tc_fence_before();
        __syncthreads();
        if (tid == 0 || tid == ISSUER2) {
            // two partial sums: band keys [0, 192) and the relay slots into [192, 256), keys
            // [192, 384) into [320, 384)
            tc_fence_after();
            const uint32_t va = smem_u32addr(sm + OFF_V), rva = smem_u32addr(sm + OFF_RV + 8192 * buf);
            const int k0 = tid == 0 ? 0 : KB / 32;
            const uint32_t dst = tmem + (tid == 0 ? TM_O : TM_O2);
#pragma unroll
            for (int k = 0; k < KB / 32; ++k) {
                const int kk = k0 + k;  // 16 band keys: block kk / 8, rows 16 (kk % 8) ..
                umma_ts(dst, tmem + 8 * kk, mndesc(va + 16384 * ((t - 1 + kk / 8) & 3) + 2048 * (kk & 7)), IDESC_O,
                        k > 0 ? 1u : 0u);
            }
            if (tid == 0 && tc_relay)
                for (int j = 0; j < J; ++j) umma_ts(dst, tmem + TM_PR + 8 * j, mndesc(rva + 2048 * j), IDESC_O, 1u);
            umma_commit(bar_o);
        }
        // while the products run: the next tile's preparation, then its relay copies
        if (g == 0 && has_next) prepare(nt, buf ^ 1);
        __syncthreads();
        if (tid == LOADER && has_next) load_relay(nbh, buf ^ 1);
        mbar_wait(bar_o, ph1, serr, 4);
        tc_fence_after();
        // epilogue: column group g stores output channels 16 g .. 16 g + 15 of its row
        uint32_t v[16], v2[16];
        tmem_ld16(trow + TM_O + 16 * g, v);
        tmem_ld16(trow + TM_O2 + 16 * g, v2);
        tmem_ld_wait();
        // a new (b, h): every ring slot is free now that this tile's products are done
        if (tid == 0 && has_next && !next_same) load_tile(nbh, nt, buf ^ 1, true);
        const int tq = q0 + r;
        if (tq < T) {
            const bool live = rdoc != -1;
            const float tot = ssum[r] + ssum[128 + r] + ssum[256 + r] + ssum[384 + r];
            float o[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) o[e] = __uint_as_float(v[e]) + __uint_as_float(v2[e]);
            if (!tc_relay && rdoc >= 0) {
                const __nv_bfloat16* rv = static_cast<const __nv_bfloat16*>(p.rv) + rbase + 16 * g;
#pragma unroll 4
                for (int s = 0; s < SLOTS; ++s) {
                    const float w = spr[r * SLOTS + s];
                    const uint4* vg = reinterpret_cast<const uint4*>(rv + s * D);
                    const uint4 a = __ldg(vg), c = __ldg(vg + 1);
                    o[0] = fmaf(w, bf16_lo(a.x), o[0]);   o[1] = fmaf(w, bf16_hi(a.x), o[1]);
                    o[2] = fmaf(w, bf16_lo(a.y), o[2]);   o[3] = fmaf(w, bf16_hi(a.y), o[3]);
                    o[4] = fmaf(w, bf16_lo(a.z), o[4]);   o[5] = fmaf(w, bf16_hi(a.z), o[5]);
                    o[6] = fmaf(w, bf16_lo(a.w), o[6]);   o[7] = fmaf(w, bf16_hi(a.w), o[7]);
                    o[8] = fmaf(w, bf16_lo(c.x), o[8]);   o[9] = fmaf(w, bf16_hi(c.x), o[9]);
                    o[10] = fmaf(w, bf16_lo(c.y), o[10]); o[11] = fmaf(w, bf16_hi(c.y), o[11]);
                    o[12] = fmaf(w, bf16_lo(c.z), o[12]); o[13] = fmaf(w, bf16_hi(c.z), o[13]);
                    o[14] = fmaf(w, bf16_lo(c.w), o[14]); o[15] = fmaf(w, bf16_hi(c.w), o[15]);
                }
            }
            const size_t row = ((size_t)b * p.H + h) * T + tq;
            const float inv = live ? 1.f / tot : 0.f;
            uint4* og = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.o) + row * D + 16 * g);
            og[0] = make_uint4(pack_bf16x2(o[0] * inv, o[1] * inv), pack_bf16x2(o[2] * inv, o[3] * inv),
                               pack_bf16x2(o[4] * inv, o[5] * inv), pack_bf16x2(o[6] * inv, o[7] * inv));
            og[1] = make_uint4(pack_bf16x2(o[8] * inv, o[9] * inv), pack_bf16x2(o[10] * inv, o[11] * inv),
                               pack_bf16x2(o[12] * inv, o[13] * inv), pack_bf16x2(o[14] * inv, o[15] * inv));
            if (g == 0) reinterpret_cast<float2*>(p.norm)[row] = live ? make_float2(m, tot) : make_float2(0.f, 1.f);
        }
        tc_fence_before();
        cur_bh = nbh;
        cur_t = nt;
    }
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

// 4-D bf16 map over a contiguous [outer][H][rows][64] array; box {64, box_rows, 1, 1}, 128-byte swizzle
int make_map64(CUtensorMap* m, const void* base, int64_t outer, int64_t H, int64_t rows, uint32_t box_rows) {
    static EncodeTiledFn enc = nullptr;
    if (!enc) {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult qr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qr) == cudaSuccess &&
            qr == cudaDriverEntryPointSuccess)
            enc = reinterpret_cast<EncodeTiledFn>(ptr);
    }
    if (!enc) return fail(DBL_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)rows, (cuuint64_t)H, (cuuint64_t)outer};
    cuuint64_t strides[3] = {(cuuint64_t)D * 2, (cuuint64_t)(rows * D * 2), (cuuint64_t)(H * rows * D * 2)};
    cuuint32_t box[4] = {(cuuint32_t)D, box_rows, 1, 1};
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
    if (a->batch <= 0 || a->heads <= 0 || a->time <= 0 || a->documents < 0)
        return fail(DBL_ERR_INVALID_ARGUMENT,
                    "relay_attention_forward: batch, heads and tokens must be positive, documents non-negative");
    if (a->head_dim != D)
        return fail(DBL_ERR_UNSUPPORTED, "relay_attention_forward: head width must be 64 (relay_attention_kernel.rs asserts it)");
    if (a->dtype != DBL_F32 && a->dtype != DBL_BF16)
        return fail(DBL_ERR_INVALID_ARGUMENT, "relay_attention_forward: dtype must be f32 or bf16");
    // with no documents (a batch of padding) the relay slots are empty and may be null
    const bool has_docs = a->documents > 0;
    if (!a->q || !a->k || !a->v || (has_docs && (!a->relay_k || !a->relay_v)) || !a->doc_id || !a->doc_start ||
        !a->doc_end || !a->o || !a->normalization)
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
    CUtensorMap mq, mk, mv, mrk, mrv;
    rc = make_map64(&mq, a->q, a->batch, a->heads, a->time, 128);
    if (rc == DBL_OK) rc = make_map64(&mk, a->k, a->batch, a->heads, a->time, 128);
    if (rc == DBL_OK) rc = make_map64(&mv, a->v, a->batch, a->heads, a->time, 128);
    // no documents: no row can reach a relay slot (its document id is out of range), so the relay
    // maps only need to be valid descriptors; they cover q
    if (rc == DBL_OK)
        rc = has_docs ? make_map64(&mrk, a->relay_k, a->documents, a->heads, SLOTS, SLOTS)
                      : make_map64(&mrk, a->q, a->batch, a->heads, a->time, SLOTS);
    if (rc == DBL_OK)
        rc = has_docs ? make_map64(&mrv, a->relay_v, a->documents, a->heads, SLOTS, SLOTS)
                      : make_map64(&mrv, a->q, a->batch, a->heads, a->time, SLOTS);
    if (rc != DBL_OK) return rc;
    static std::atomic<uint64_t> attr_done{0};
    rc = once_per_device(attr_done, [] {
        return cuda_status(
            cudaFuncSetAttribute(relay_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_TC),
            "relay_attention_forward: cudaFuncSetAttribute");
    });
    if (rc != DBL_OK) return rc;
    // persistent: one CTA per SM (or per tile when there are fewer tiles)
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_status(e, "relay_attention_forward: device query");
    const int64_t ntiles = (int64_t)p.B * p.H * ((p.T + TQ - 1) / TQ);
    const unsigned grid = (unsigned)std::min<int64_t>(ntiles, (int64_t)sms);
    relay_attn_tc_kernel<<<grid, NTH, SMEM_TC, st>>>(mq, mk, mv, mrk, mrv, p);
    return launch_status("relay_attn_tc_kernel");
}
