// Parameters of the token-sequential GDN-2 scan kernel (scan_seq.cu), shared with the
// prefill dispatcher (prefill.cu).
#pragma once

#include "common.cuh"

namespace dbl {

struct SeqParams {
    int B, T, H, K, V;
    const void *q, *k, *v;
    int64_t qs[4], ks[4], vs[4];
    // gate_mode 0: channel-wise alpha/erase [B,T,H,K], write [B,T,H,V] (strides as/es/ws).
    // gate_mode 1: scalar alpha [B,T,H] (as[0..2]) and beta = erase pointer (es[0..2]).
    int gate_mode;
    const float *alpha, *erase, *write;
    int64_t as[4], es[4], ws[4];
    float scale;
    int mask_mode;  // 0 none, 1 valid/reset [B,T] f32, 2 doc_start/doc_end [B,T] int32
    const float *valid, *reset;
    const int32_t *doc_start, *doc_end;
    int init_mode;  // 0 zeros, 1 initial pointer [B,H,K,V], 2 identity (transition matrices)
    const float* initial;
    int v_zero;     // 1: values are treated as zero (span transition)
    void* out;      // optional
    int out_dtype;  // DBL_F32 / DBL_BF16
    int64_t os[4];
    float* final_state;  // optional, [B,H,K,V]
    float* scores;       // optional, [B,T,H]
    float* chunk_states; // optional, chunked form only: the state at every 16-token chunk start,
                         // [B*H][ceil(T/16)][K][V]
    float* edits;        // optional, chunked form only: every token's edit, [B,T,H,V] f32
    const int* route;    // optional per-(b,h) flags: a CTA runs only where (route != 0) == route_want
    int route_want;
};

// The library's stream-ordered memory pool of the current device (scan_chunk.cu).
int scratch_pool(cudaMemPool_t* out);

// Checks the arguments of the training-scan forward (dbl_gdn_training_scan) and fills `out`.
int training_scan_params(const dbl_training_scan_args* a, SeqParams* out);

// Validates the shape limits of the sequential kernel and launches it on `st`.
int launch_seq_scan(const SeqParams& p, int in_dtype, cudaStream_t st);

// The chunked form of the same scan (scan_chunk.cu): whether it takes `p`, its workspace and its
// launcher (maps in `ext_ws` when given, else in the library's pool; `extra` keeps the maps the
// chunked backward reads).
bool chunk_scan_supported(const SeqParams& p);
size_t chunk_scan_workspace_floats(const SeqParams& p, bool extra);
int launch_chunk_scan(const SeqParams& p, int in_dtype, cudaStream_t st, float* ext_ws = nullptr, bool extra = false);

// The chunked backward of the training scan for 16-token checkpoints (scan_chunk_bwd.cu): the
// forward parameters it runs (f32 [B,T,H,W] inputs, valid/reset masks, no outputs), its workspace
// and its launcher (`ws` 16-byte aligned).
SeqParams chunk_backward_forward_params(int B, int T, int H, int K, int V, const float* q, const float* k,
                                        const float* v, const float* alpha, const float* erase, const float* write,
                                        const float* valid, const float* reset, const float* initial);
size_t chunk_backward_workspace_floats(const SeqParams& sp);
bool chunk_backward_supported(const SeqParams& sp);
int launch_chunk_backward(const SeqParams& sp, const float* g_out, const float* g_fin, const float* g_score,
                          float* dq, float* dk, float* dv, float* dalpha, float* derase, float* dwrite,
                          float* dinitial, float* ws, cudaStream_t st);

// The saved forward context of the chunked backward (chunk-start states, chunk maps, every token's
// edit): its size for the shapes of `sp`, the forward that writes it beside the outputs (`ctx`
// 16-byte aligned), and the backward that reads it instead of recomputing the forward (`ws` as for
// launch_chunk_backward).
size_t chunk_context_floats(const SeqParams& sp);
int launch_chunk_forward_saved(const SeqParams& sp, int in_dtype, float* ctx, cudaStream_t st);
int launch_chunk_backward_saved(const SeqParams& sp, const float* g_out, const float* g_fin, const float* g_score,
                                float* dq, float* dk, float* dv, float* dalpha, float* derase, float* dwrite,
                                float* dinitial, const float* ctx, float* ws, cudaStream_t st);

}  // namespace dbl
