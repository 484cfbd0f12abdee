/*
 * dbl_gdn2.h -- C ABI of the B200 (sm_100a) GDN-2 hot path.
 *
 * GDN-2 is the gated delta rule.  Per (batch row b, head h) the key-major state S [K,V] evolves,
 * for every valid token t (crates/mixers/src/reference.rs:57-111):
 *     if reset[t]:  S = 0
 *     S      = diag(alpha_t) S
 *     edit_j = write_j v_j - sum_i erase_i k_i S_ij
 *     S     += k edit^T
 *     o_j    = sum_i q_i S_ij            (padding: o = 0, S unchanged)
 * The scalar-gate form used by the prefill / decode entry points sets alpha[i] = alpha_t,
 * erase[i] = write[j] = beta_t and pre-scales q by `scale` (1/sqrt(K) in the reference model).
 *
 * Conventions shared by every entry point:
 *   - All pointers are DEVICE pointers on the current CUDA device, owned by the caller.
 *     No entry point allocates device memory except where a function says so.
 *   - Strides are in ELEMENTS.  A stride array of all zeros means "contiguous".
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Calls are asynchronous and
 *     return after enqueueing; errors in arguments are reported before anything is enqueued.
 *   - Every function returns a dbl_status; it never aborts the process.  A human-readable
 *     reason for the last failure on the calling thread is returned by dbl_last_error().
 *   - Layout: inputs [B,T,H,C] (C = channel), states [B,H,K,V] f32 key-major, as the
 *     reference's tensors (crates/mixers/src/chunk.rs:126).
 */
#ifndef DBL_GDN2_H
#define DBL_GDN2_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *dbl_stream_t; /* == cudaStream_t */

typedef enum {
    DBL_OK = 0,
    DBL_ERR_INVALID_ARGUMENT = 1, /* bad shape, null required pointer, bad stride or alignment */
    DBL_ERR_UNSUPPORTED = 2,      /* valid request outside what the kernels implement         */
    DBL_ERR_CUDA = 3,             /* a CUDA runtime/driver call failed                         */
    DBL_ERR_WORKSPACE = 4,        /* workspace missing or smaller than *_workspace_bytes()     */
    DBL_ERR_TIMEOUT = 5           /* a bounded wait gave up (multi-GPU hand-off)               */
} dbl_status;

typedef enum { DBL_F32 = 0, DBL_BF16 = 1 } dbl_dtype;

/* Human-readable name of a status code (static storage). */
const char *dbl_status_string(int status);
/* Reason for the last non-OK status returned on this thread (thread-local, static storage). */
const char *dbl_last_error(void);
/* ABI version: major * 10000 + minor * 100 + patch. */
int dbl_abi_version(void);
/* Every wait inside the library's kernels (the tensor-core prefill and relay attention, the relay
 * merge's copy ring) is bounded; one that gives up records a site code on the current device and
 * lets the kernel run to completion (its outputs are then undefined).  The
 * tensor-core prefill also records code 100 when one of its fp16 MMA operands left fp16 range
 * (inputs far outside unit-norm keys and beta in [0, 1]; its outputs are then not valid), and
 * relay attention records code 101 when a live row's document id lies outside [0, documents).
 * This call synchronises with the device, stores the code in *code (0 = none; code may be NULL),
 * clears the record and returns DBL_OK, DBL_ERR_UNSUPPORTED (code 100), DBL_ERR_INVALID_ARGUMENT
 * (code 101) or DBL_ERR_TIMEOUT.  No counterpart in the reference, whose kernels have no bounded
 * waits or range checks. */
int dbl_device_error(int *code);

/* =============================================================================================
 * 1. Chunked prefill scan, scalar gates (the BASELINE prefill: configs 0, 1 and 4).
 *
 * Replaces, for scalar gates, the forward of delta_kernels::gdn_training_scan
 * (crates/kernels/src/gdn_training_ops.rs:288-333) as reached from
 * chunk::scan_selected(ScanBackend::FusedGdn2, ...) (crates/mixers/src/chunk.rs:40-67), and the
 * CPU tensor solver chunk::scan (chunk.rs:129-250) it must agree with.  Unlike the reference
 * (chunk <= 16, K32/V64, f32 only) this runs chunk 64 at K,V in {64,128}, f32 or bf16 inputs,
 * f32 gates, f32 state.  bf16 inputs at K = V = 128 run on the tcgen05 tensor-core kernel.
 * ========================================================================================== */
typedef struct {
    int64_t batch, time, heads, key_dim, value_dim; /* B, T, H, K, V                         */
    int32_t dtype;            /* dbl_dtype of q, k, v and out                                 */
    int32_t chunk_size;       /* 0 or 64                                                      */
    float scale;              /* q multiplier (1/sqrt(K) in the reference model)              */
    const void *q;            /* [B,T,H,K]                                                    */
    const void *k;            /* [B,T,H,K]                                                    */
    const void *v;            /* [B,T,H,V]                                                    */
    int64_t q_stride[4], k_stride[4], v_stride[4]; /* innermost stride must be 1            */
    const float *alpha;       /* [B,T,H] decay in (0,1]; 0 behaves as a reset                 */
    const float *beta;        /* [B,T,H] erase = write strength                               */
    int64_t alpha_stride[3], beta_stride[3];
    const float *valid;       /* optional [B,T] contiguous, nonzero = token present           */
    const float *reset;       /* optional [B,T] contiguous, nonzero = zero state first        */
    const float *initial_state; /* optional [B,H,K,V] contiguous f32 (NULL = zeros)           */
    void *out;                /* optional [B,T,H,V] (dtype); NULL skips the output            */
    int64_t out_stride[4];
    float *final_state;       /* optional [B,H,K,V] contiguous f32; may equal initial_state   */
} dbl_prefill_args;

int dbl_gdn2_prefill(const dbl_prefill_args *args, dbl_stream_t stream);

/* Span transition for time sharding (config 4).  For the token span described by `args`
 * (q, v, out, initial_state and final_state are ignored) writes, per (b,h), the K x K matrix
 * A with  S_end = A S_start + B_span  (B_span = dbl_gdn2_prefill from a zero state).
 * transition: [B,H,K,K] contiguous f32.  No counterpart in the reference, which has no time
 * sharding; it is the hand-off object of the long-context prefill. */
int dbl_gdn2_span_transition(const dbl_prefill_args *args, float *transition,
                             dbl_stream_t stream);

/* Fold of span maps (the time-sharding hand-off).  For s = 0 .. segments-1,
 *     X_{s+1} = transition[s] X_s + offset[s],   X_0 = start (NULL = zeros),
 * per head, in f32.  transition [S,H,K,K] and offset [S,H,K,V] are the maps of consecutive token
 * spans (dbl_gdn2_span_transition and dbl_gdn2_prefill from a zero state); starts [S,H,K,V]
 * (optional) receives X_0 .. X_{S-1}, the start state of every span, end [H,K,V] (optional) X_S,
 * and composed_transition [H,K,K] (optional) transition[S-1] ... transition[0], the transition of
 * the whole run of spans.  K a multiple of 16 up to 128, V a multiple of 16; arrays contiguous and
 * 16-byte aligned.  f32 accuracy: tensor-core products of operands split into two tf32 parts.
 * No counterpart in the reference, which has no time sharding. */
int dbl_gdn2_span_fold(const float *transition, const float *offset, int64_t segments, int64_t heads,
                       int64_t key_dim, int64_t value_dim, const float *start, float *starts, float *end,
                       float *composed_transition, dbl_stream_t stream);

/* Prefill of ONE long sequence (batch 1, config 4) on one device by time segments that run side
 * by side.  segments > 0: `segments` equal segments -- pass 1 the segment maps, a fold of their
 * start states from initial_state, pass 2 every segment rescanned from its start.  segments = 0:
 * when T is a multiple of 64 and m = floor(SMs / heads) >= 2, a lead segment and m equal segments
 * of ceil(T / 64 / (m + 1.8)) chunks: the lead segment is scanned from initial_state on a side stream
 * (one per device, created on first use) while the maps of segments 1 .. m-1 run on `stream`, then
 * a fold and one rescan of segments 1 .. m; otherwise the largest power of two with segments x
 * heads <= the SM count and whole 64-token chunks per segment.  Same arguments and results as
 * dbl_gdn2_prefill (out, final_state); the result agrees with the one-pass scan to the rounding of
 * the maps.  workspace: device memory of dbl_gdn2_prefill_segmented_workspace_bytes() bytes (same
 * `segments`), 256-byte aligned.  Replaces, for one long sequence, the chunk-boundary carry of
 * chunk::scan (crates/mixers/src/chunk.rs:147-244), whose chunk loop runs the whole sequence in
 * order. */
size_t dbl_gdn2_prefill_segmented_workspace_bytes(const dbl_prefill_args *args, int64_t segments);
int dbl_gdn2_prefill_segmented(const dbl_prefill_args *args, int64_t segments, void *workspace,
                               size_t workspace_bytes, dbl_stream_t stream);

/* Prefill of ONE long sequence sharded along time over n_gpus devices, driven from one host thread
 * (config 4 for a host that owns several GPUs in one process).  spans[g] describes the g-th
 * consecutive time span (batch 1; device pointers on devices[g]; same heads, widths and dtype);
 * spans[0].initial_state is the sequence's initial state (the other spans' initial_state is
 * ignored) and the last span's final_state receives the sequence's final state.  Each device scans
 * its span's segment maps (as dbl_gdn2_prefill_segmented); device g then pulls the span maps of
 * devices 0 .. g-1 -- 2 x H x K x (K + V) x 4 bytes each, one cudaMemcpyPeerAsync per array on
 * streams[g] after an event of the producing device -- folds them into its start state and
 * rescans its span.  Peer memory is only read by those copies.  Work is enqueued on streams[g];
 * the call returns without waiting.  workspaces[g]: device memory on devices[g] of
 * dbl_gdn2_prefill_time_sharded_workspace_bytes(&spans[g], n_gpus, segments) bytes (the segment
 * count 0 = automatic follows the SM count of the device current at the query).  The calling
 * thread's current device is restored on return.  No counterpart in the reference, which runs on
 * one device; its sequence-scaling contract is the chunk-boundary carry of chunk.rs:147-244. */
size_t dbl_gdn2_prefill_time_sharded_workspace_bytes(const dbl_prefill_args *span, int n_gpus,
                                                     int64_t segments);
int dbl_gdn2_prefill_time_sharded(const dbl_prefill_args *spans, int n_gpus, const int *devices,
                                  dbl_stream_t const *streams, int64_t segments, void *const *workspaces,
                                  const size_t *workspace_bytes);

/* =============================================================================================
 * 2. Single-token recurrent decode step, state updated IN PLACE (config 2).
 *
 * Replaces the reference decode, which is chunk::scan_selected with T = 1 and `initial` set
 * (crates/mixers/src/lib.rs:544-556 -> gdn_training_scan, out of place) and the one-step oracle
 * gdn2_reference::step (crates/mixers/src/gdn2_reference.rs:52-83).  K, V in {64, 128}.
 * ========================================================================================== */
typedef struct {
    int64_t batch, heads, key_dim, value_dim; /* N sequences, H, K, V                          */
    int32_t dtype;            /* dtype of q, k, v, out                                         */
    float scale;              /* q multiplier                                                  */
    const void *q, *k;        /* [N,H,K]                                                       */
    const void *v;            /* [N,H,V]                                                       */
    int64_t q_stride[3], k_stride[3], v_stride[3];
    const float *alpha, *beta; /* [N,H] contiguous                                             */
    float *state;             /* [N,H,K,V] contiguous f32, read and written in place          */
    void *out;                /* [N,H,V] (dtype)                                               */
    int64_t out_stride[3];
} dbl_decode_args;

int dbl_gdn2_decode_step(const dbl_decode_args *args, dbl_stream_t stream);

/* =============================================================================================
 * 3. Reference contract, channel-wise gates: the stateful fused scan.
 *
 * Mirrors delta_kernels::gdn_training_scan(q, k, v, alpha, erase, write, valid, reset, initial,
 * chunk_size) -> GdnTrainingOutput { output, final_state, scores }
 * (crates/kernels/src/gdn_training_ops.rs:288-333; kernel gdn_training.rs:12-115).
 * Shapes: q,k,alpha,erase [B,T,H,K]; v,write [B,T,H,V]; valid,reset [B,T] f32 {0,1};
 * initial [B,H,K,V].  chunk_size must be 1..=16 as in the reference (gdn_training.rs:370-373);
 * it only bounds the reference's backward checkpoints, which this forward-only build does not
 * produce.  Generalised to K <= 128, V <= 256 and bf16 q/k/v (the reference: K32/V64 f32).
 * Outputs f32: output [B,T,H,V], final_state [B,H,K,V], scores [B,T,H] = |k| |edit|.
 * All arrays contiguous.  initial may be NULL (zeros); scores may be NULL.
 * ========================================================================================== */
typedef struct {
    int64_t batch, time, heads, key_dim, value_dim;
    int32_t dtype;            /* dtype of q, k, v (gates and masks are always f32)            */
    int32_t chunk_size;
    const void *q, *k, *v;
    const float *alpha, *erase, *write;
    const float *valid, *reset;     /* required, [B,T]                                       */
    const float *initial_state;     /* optional                                              */
    float *output;                  /* required                                              */
    float *final_state;             /* optional                                              */
    float *scores;                  /* optional                                              */
} dbl_training_scan_args;

int dbl_gdn_training_scan(const dbl_training_scan_args *args, dbl_stream_t stream);

/* Backward (vector-Jacobian product) of dbl_gdn_training_scan for the loss
 *     L = sum grad_output . output + sum grad_final_state . final_state + sum grad_scores . scores.
 * Replaces delta_kernels' gdn_training_backward (crates/kernels/src/gdn_training_ops.rs:95-127,
 * kernel gdn_training.rs:117-284), whose upstream tensor packs the three gradients; here they are
 * separate pointers.  The reference reads the checkpoints and per-token edits its forward saved;
 * this call recomputes them into `workspace` (dbl_gdn_training_scan_backward_workspace_bytes()
 * bytes), so it needs only the forward's inputs.  f32 throughout, as the reference; K <= 64,
 * V <= 256; chunk_size (1..=16) is the checkpoint spacing.  All arrays contiguous.
 * Outputs: dq, dk, dalpha, derase [B,T,H,K]; dv, dwrite [B,T,H,V]; dinitial [B,H,K,V] (optional).
 * grad_final_state, grad_scores and initial_state may be NULL (zeros). */
typedef struct {
    int64_t batch, time, heads, key_dim, value_dim;
    int32_t chunk_size;
    const float *q, *k, *v;
    const float *alpha, *erase, *write;
    const float *valid, *reset;       /* required, [B,T]                                        */
    const float *initial_state;       /* optional [B,H,K,V]                                     */
    const float *grad_output;         /* required [B,T,H,V]                                     */
    const float *grad_final_state;    /* optional [B,H,K,V]                                     */
    const float *grad_scores;         /* optional [B,T,H]                                       */
    float *dq, *dk, *dv, *dalpha, *derase, *dwrite;
    float *dinitial;                  /* optional                                               */
} dbl_training_scan_backward_args;

size_t dbl_gdn_training_scan_backward_workspace_bytes(int64_t batch, int64_t time, int64_t heads,
                                                      int64_t key_dim, int64_t value_dim,
                                                      int32_t chunk_size);
int dbl_gdn_training_scan_backward(const dbl_training_scan_backward_args *args, void *workspace,
                                   size_t workspace_bytes, dbl_stream_t stream);

/* The forward -> backward hand-off of the reference: its gdn_training_scan returns checkpoint and
 * auxiliary tensors beside the packed outputs and its gdn_training_backward consumes them
 * (crates/kernels/src/gdn_training_ops.rs:201-224 and :87-112).  At the shapes of the chunked
 * backward (chunk_size 16, key width <= 64, value width <= 128, T >= 32) the saved context holds the chunk-start states, the chunk maps and every token's edit,
 * and the backward skips the forward it would otherwise rerun; elsewhere the context is empty
 * (0 bytes) and these calls are dbl_gdn_training_scan and dbl_gdn_training_scan_backward.
 * The context must be 16-byte aligned and hold dbl_gdn_training_scan_context_bytes() bytes; the
 * backward takes the same inputs as the forward that wrote it and a workspace of
 * dbl_gdn_training_scan_backward_workspace_bytes() bytes (16-byte aligned). */
size_t dbl_gdn_training_scan_context_bytes(int64_t batch, int64_t time, int64_t heads, int64_t key_dim,
                                           int64_t value_dim, int32_t chunk_size);
int dbl_gdn_training_scan_save(const dbl_training_scan_args *args, void *context, size_t context_bytes,
                               dbl_stream_t stream);
int dbl_gdn_training_scan_backward_saved(const dbl_training_scan_backward_args *args, const void *context,
                                         size_t context_bytes, void *workspace, size_t workspace_bytes,
                                         dbl_stream_t stream);

/* Backward of dbl_gdn2_scan: replaces Gdn2Ops::gdn2_backward(q, k, v, alpha, erase, write,
 * output_grad, checkpoint, doc_start, doc_end) -> (dq, dk, dv, dalpha, derase, dwrite)
 * (crates/kernels/src/ops.rs:106-160; kernels gdn2.rs:285-519).  Layouts as dbl_gdn2_scan; q, k,
 * v, grad_output and dq, dk, dv in dtype (f32 or bf16), the gates and their gradients f32.  The
 * forward's checkpoint tensor is not taken: the chunk states are recomputed in the workspace
 * (dbl_gdn2_scan_backward_workspace_bytes).  K <= 64, V <= 256. */
typedef struct {
    int64_t batch, time, heads, key_dim, value_dim;
    int32_t dtype;
    const void *q, *k, *v;
    const float *alpha, *erase, *write;
    const int32_t *doc_start, *doc_end;
    const void *grad_output;
    void *dq, *dk, *dv;
    float *dalpha, *derase, *dwrite;
} dbl_gdn2_scan_backward_args;

size_t dbl_gdn2_scan_backward_workspace_bytes(int64_t batch, int64_t time, int64_t heads, int64_t key_dim,
                                              int64_t value_dim, int32_t dtype);
int dbl_gdn2_scan_backward(const dbl_gdn2_scan_backward_args *args, void *workspace, size_t workspace_bytes,
                           dbl_stream_t stream);

/* GDN-2 mixer prologue: what Mixer::forward_inner computes between the projections and the scan
 * (crates/mixers/src/lib.rs:446-528, MixerKind::Gdn2), fused into one memory-bound pass:
 *   q, k = l2(silu(conv(proj_q|proj_k))),  v = silu(conv(proj_v)),
 *   alpha = exp(-softplus(proj_decay + decay_bias[h,k]) exp(decay_scale[h])),
 *   erase = sigmoid(proj_erase),  write = sigmoid(proj_write).
 * conv is the depthwise causal convolution kept inside one document (conv.rs:7-45; documents =
 * cumsum(reset * valid) over time), l2 is x / sqrt(sum x^2 + 1e-6) per head row (norm.rs mode 0),
 * softplus switches to x above 20 (decay.rs:13-20).  Projections [B,T,H*K] (q, k, decay, erase)
 * and [B,T,H*V] (v, write) in in_dtype; conv weights [W,H*K] / [W,H*V] f32 (W <= 8);
 * decay_bias [H*K], decay_scale [H], valid / reset [B,T] f32.  Outputs q, k [B,T,H,K] and
 * v [B,T,H,V] in out_dtype; alpha, erase [B,T,H,K] and write [B,T,H,V] f32.  K, V <= 256; all
 * arrays contiguous. */
typedef struct {
    int64_t batch, time, heads, key_dim, value_dim, conv_width;
    int32_t in_dtype, out_dtype;
    const void *proj_q, *proj_k, *proj_v;
    const void *proj_decay, *proj_erase, *proj_write;
    const float *conv_q, *conv_k, *conv_v;
    const float *decay_bias, *decay_scale;
    const float *valid, *reset;
    void *q, *k, *v;
    float *alpha, *erase, *write;
} dbl_gdn2_prologue_args;

int dbl_gdn2_prologue(const dbl_gdn2_prologue_args *args, dbl_stream_t stream);

/* Mirrors delta_kernels::gdn2_scan(q, k, v, alpha, erase, write, doc_start, doc_end) -> output
 * (crates/kernels/src/ops.rs:251-276, kernels gdn2.rs:23-283; oracle gdn2_reference.rs:87-105):
 * inclusive int32 document limits [B,T]; `end < start` marks padding (output 0, state kept),
 * `start == t` resets.  Zero initial state.  Output [B,T,H,V] in the q dtype.  Contiguous. */
typedef struct {
    int64_t batch, time, heads, key_dim, value_dim;
    int32_t dtype;
    const void *q, *k, *v;
    const float *alpha, *erase, *write;
    const int32_t *doc_start, *doc_end;
    void *output;
} dbl_gdn2_scan_args;

int dbl_gdn2_scan(const dbl_gdn2_scan_args *args, dbl_stream_t stream);

/* =============================================================================================
 * 4. Relay attention, decode case (config 3): one query per (sequence, head) attends to a
 * shared prefix KV (stored once, read once per head for all sequences) and to the sequence's
 * own KV; the two softmax parts are merged by log-sum-exp inside one kernel.
 *
 * Replaces, for the split prefix/own layout, the forward of
 * RelayAttentionKernelOps::relay_attention_forward (reuse/crates/dre-attention/src/
 * relay_attention_kernel.rs:14-20, kernel :38-130, host run_relay_windowed_attention :311-340):
 * same online-softmax arithmetic, same [max, sum] statistics and the same empty-row convention
 * (o = 0, max = 0, sum = 1).  head_dim 128 (64 supported too), bf16 or f32.
 * Layouts (contiguous): q [N,H,D]; prefix_k, prefix_v [H,Lp,D]; own_k, own_v [N,H,Lo,D];
 * own_len optional int32 [N] (0..Lo, ragged own segments); out [N,H,D] (dtype);
 * row_max, row_sum optional f32 [N,H].
 * The kernel needs scratch for the split partials: pass a device buffer of at least
 * dbl_relay_merge_workspace_bytes(...) bytes (16-byte aligned).  It is reusable across calls on
 * the same stream; calls that overlap on the GPU must use distinct workspaces.
 * ========================================================================================== */
typedef struct {
    int64_t n_seq, heads, head_dim, prefix_len, own_cap;
    int32_t dtype;
    float scale;                      /* softmax scale (1/sqrt(D))                            */
    const void *q;
    const void *prefix_k, *prefix_v;
    const void *own_k, *own_v;
    const int32_t *own_len;           /* optional                                             */
    void *out;
    float *row_max, *row_sum;         /* optional                                             */
} dbl_relay_merge_args;

size_t dbl_relay_merge_workspace_bytes(int64_t n_seq, int64_t heads, int64_t head_dim,
                                       int64_t prefix_len, int64_t own_cap);
/* Scratch bytes of one call's own layout (its dtype's): at most dbl_relay_merge_workspace_bytes,
 * which bounds both dtypes.  0 for an invalid shape.  Host-only; needs no device. */
size_t dbl_relay_merge_call_workspace_bytes(const dbl_relay_merge_args *args);
int dbl_relay_merge_decode(const dbl_relay_merge_args *args, void *workspace,
                           size_t workspace_bytes, dbl_stream_t stream);

/* Relay merge for callers that cannot allocate device memory at the call site -- a host whose
 * device memory belongs to its own pooling allocator, or a serving loop that must not call
 * cudaMalloc/cudaFree while it runs.  No counterpart in the reference.  Same arguments and results
 * as dbl_relay_merge_decode; the split-softmax partials go to a fixed array of
 * DBL_RELAY_NOALLOC_SCRATCH_BYTES that the library keeps in device memory (reserved on every
 * device that loads the library, until the process exits), so the call allocates nothing.
 *   - The limit is checked against the scratch of the call's own dtype, which
 *     dbl_relay_merge_call_workspace_bytes(args) returns: a call needing more than the array
 *     returns DBL_ERR_WORKSPACE and launches nothing.
 *   - The first call in a CUDA context looks up the array's device address in that context
 *     (cudaGetSymbolAddress) and keeps it for later calls in the same context; a call from another
 *     context of the device (a driver-API host, or after cudaDeviceReset) looks it up again.
 *     Make the first call of each context before any stream capture.
 *   - Every call on a device shares the one array and the array keeps the last call's partials
 *     (the arrival counters are cleared at the start of each call): calls that overlap on the GPU,
 *     e.g. on two streams, race on it. */
#define DBL_RELAY_NOALLOC_SCRATCH_BYTES (16u << 20)
int dbl_relay_merge_decode_noalloc(const dbl_relay_merge_args *args, dbl_stream_t stream);

/* =============================================================================================
 * 5. Relay attention in the reference layout (training / prefill forward).
 *
 * Replaces RelayAttentionKernelOps::relay_attention_forward and run_relay_windowed_attention
 * (reuse/crates/dre-attention/src/relay_attention_kernel.rs:14-20, :311-340; kernel
 * relay_forward_kernel :38-130): query t of row b attends, in one softmax, to the keys of [t - 128,
 * t + 128] inside its inclusive document limits [doc_start, doc_end] and to the 16 relay slots of
 * its document doc_id; scores are q.k / 8.  q, k, v [B,H,T,64] and relay_k, relay_v
 * [documents,H,16,64] in dtype (f32 or bf16); doc_* [B,T] int32; o [B,H,T,64] in dtype;
 * normalization [B,H,T,2] f32 = (row maximum, sum of exp(score - maximum)).  A padding row
 * (doc_end < doc_start) writes o = 0 and (0, 1), as the reference.  head_dim must be 64 (the
 * reference asserts it).  All arrays contiguous and 16-byte aligned.  The forward's unused layout
 * tensors (doc_row, relay_start, relay_end) are not taken.  A live row whose doc_id is outside
 * [0, documents) gets no relay slots and records device error 101 (dbl_device_error).  documents
 * may be 0 (a batch of padding; relay_k and relay_v may then be NULL). */
typedef struct {
    int64_t batch, heads, time, head_dim, documents;
    int32_t dtype;
    const void *q, *k, *v;
    const void *relay_k, *relay_v;
    const int32_t *doc_id, *doc_start, *doc_end;
    void *o;
    float *normalization;
} dbl_relay_attention_args;

int dbl_relay_attention_forward(const dbl_relay_attention_args *args, dbl_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* DBL_GDN2_H */
