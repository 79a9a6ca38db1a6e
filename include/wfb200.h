/*
 * wfb200.h - C ABI of the B200-native WANferenz MoE decode path.
 *
 * Plain pointers, sizes and a cudaStream_t passed as void*; no torch types.
 * The workspace of wf_moe_forward must be zero-filled once when allocated;
 * the kernels leave their counters at zero after every call.
 * Every entry point returns an int status (WF_OK or a negative WF_E_* code);
 * wf_last_error() returns the message of the last failure on the calling
 * host thread.  No entry point allocates device memory (except the set-up
 * call wf_ep_alloc, which says so), synchronizes the
 * stream or reads device data back, except the load-time check
 * wf_fp4_scales_in_range() and the error-word reads wf_moe_read_error() and
 * wf_moe_read_error_noalloc(), which say so.
 *
 * Data formats (identical to the reference's tensors, so a reference
 * checkpoint's bytes are passed through unchanged):
 *   bf16        2-byte bfloat16, row-major
 *   e4m3        1-byte float8_e4m3fn
 *   e8m0        1-byte float8_e8m0fnu (power-of-two scale 2^(b-127))
 *   fp4 packed  float4_e2m1fn_x2: two E2M1 codes per byte, low nibble = even k
 *
 * Each declaration names the reference interface it replaces
 * (paths relative to the WANferenz project root).
 */
#ifndef WFB200_H
#define WFB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------- */
#define WF_OK 0
#define WF_E_SHAPE (-1)     /* unsupported or inconsistent dimensions          */
#define WF_E_DTYPE (-2)     /* unsupported scale kind / format flag            */
#define WF_E_EXPERT_ID (-3) /* an expert id or token id outside its range      */
#define WF_E_TIMEOUT (-4)   /* a device-side wait ran past its bound           */
#define WF_E_CUDA (-5)      /* a CUDA runtime call failed                      */
#define WF_E_RANGE (-6)     /* FP4 weight scales outside the exact range       */
#define WF_E_ARG (-7)       /* null pointer or workspace too small             */

/* scale kinds of activation / weight scale tensors */
#define WF_SCALE_F32 0  /* float32 scales                                   */
#define WF_SCALE_E8M0 1 /* e8m0 byte scales                                 */

/* router score functions: ModelArgs.score_func (architecture.py:59) */
#define WF_SCORE_SOFTMAX 0
#define WF_SCORE_SIGMOID 1
#define WF_SCORE_SQRTSOFTPLUS 2

/* One MoE layer's shapes and options: the ModelArgs fields read by Gate,
 * Expert and MoE (wanferenz/model/architecture.py:42-93, 674-794). */
typedef struct wf_moe_config {
    int32_t dim;             /* D: hidden size                         */
    int32_t inter_dim;       /* I: moe_inter_dim                       */
    int32_t n_experts;       /* E: n_routed_experts                    */
    int32_t n_local_experts; /* experts held by this rank (E / world)   */
    int32_t expert_offset;   /* first local expert id (rank * E_local)  */
    int32_t topk;            /* n_activated_experts                    */
    int32_t score_func;      /* WF_SCORE_*                             */
    int32_t hash_layer;      /* 1: indices = tid2eid[input_ids]        */
    int32_t ue8m0;           /* 1: power-of-two activation scales      */
    int32_t max_tokens;      /* capacity the workspace is sized for    */
    int64_t vocab;           /* rows of tid2eid (hash layers)          */
    float route_scale;       /* Gate.route_scale                       */
    float swiglu_limit;      /* Expert.swiglu_limit (0 = off)          */
} wf_moe_config;

/* Device pointers to one layer's weights, in the reference's bank layout
 * (wanferenz/kernels/fp4_grouped.py:136-201 for the routed bank,
 *  wanferenz/kernels/fp8_vector.py:316-351 for the shared w13 stack). */
typedef struct wf_moe_weights {
    const void *gate_w;       /* [E, D] bf16                               */
    const float *gate_bias;   /* [E] f32, or NULL on hash layers            */
    const int32_t *tid2eid;   /* [vocab, topk] int32 on hash layers, else NULL */
    const uint8_t *w13;       /* [E_local, 2I, D/2] fp4 packed (w1 rows, then w3 rows) */
    const uint8_t *w13_s;     /* [E_local, 2I, D/32] e8m0                   */
    const uint8_t *w2;        /* [E_local, D, I/2] fp4 packed               */
    const uint8_t *w2_s;      /* [E_local, D, I/32] e8m0                    */
    const uint8_t *shared_w13; /* [2I, D] e4m3 (w1 rows, then w3 rows)       */
    const void *shared_s13;   /* [2I/128, D/128] scale (shared_scale_kind)   */
    const uint8_t *shared_w2; /* [D, I] e4m3                               */
    const void *shared_s2;    /* [D/128, I/128] scale                       */
    int32_t shared_scale_kind; /* WF_SCALE_E8M0 or WF_SCALE_F32             */
} wf_moe_weights;

/* Last failure message of this host thread ("" when none). */
const char *wf_last_error(void);

/* Number of SMs of the current device (the persistent grid size). */
int wf_device_sm_count(void);

/* Bytes of device workspace wf_moe_forward needs for cfg->max_tokens tokens.
 * Allocate once (e.g. at layer load) and reuse; calls sharing one workspace
 * must be ordered on one stream. */
size_t wf_moe_workspace_bytes(const wf_moe_config *cfg);

/* Full MoE layer forward for T tokens: router, routed FP4 SwiGLU experts,
 * FP8 shared expert and the ascending-expert fp32 combine.
 * Replaces MoE.forward (wanferenz/model/architecture.py:777-794) and its GPU
 * patch grouped_forward (wanferenz/kernels/fp4_grouped.py:271-324).
 *   x          [T, D] bf16 (device)
 *   input_ids  [T] int64 (device; read on hash layers only, may be NULL otherwise)
 *   y          [T, D] bf16 output, or NULL when y_partial is given
 *   y_partial  [T, D] f32 output of the local experts' routed sum only
 *              (expert-parallel mode: the caller all-reduces it and calls
 *              wf_moe_finish), or NULL
 *   out_weights [T, topk] f32 and out_indices [T, topk] int64: the router's
 *              outputs (Gate.forward, architecture.py:696-718); may be NULL
 * Launches 3 kernels on `stream`; allocates nothing; no host sync. */
int wf_moe_forward(const wf_moe_config *cfg, const wf_moe_weights *w, const void *x,
                   const int64_t *input_ids, int32_t T, void *y, float *y_partial,
                   float *out_weights, int64_t *out_indices, void *workspace,
                   size_t workspace_bytes, void *stream);

/* wf_moe_forward with four caller-created cudaEvent_t recorded on `stream`
 * before the first and after each of the three kernels (measurement hook:
 * per-kernel durations without a profiler; the kernels then launch without
 * programmatic overlap, so each event pair brackets one kernel).  Not for use
 * inside stream capture.  No counterpart in the reference. */
int wf_moe_forward_timed(const wf_moe_config *cfg, const wf_moe_weights *w, const void *x,
                         const int64_t *input_ids, int32_t T, void *y, float *y_partial,
                         float *out_weights, int64_t *out_indices, void *workspace,
                         size_t workspace_bytes, void *stream, void *const *events);

/* Size of the module-scope device scratch wf_moe_forward_noalloc uses. */
#define WF_NOALLOC_SCRATCH_BYTES (4u << 20)

/* wf_moe_forward for callers that cannot allocate device memory: a caller
 * whose memory belongs to another allocator with nothing to hand out at call
 * time, or one that must not call into the CUDA allocator on its serving path
 * (cudaMalloc may synchronize the whole device).  The caller passes inputs and
 * outputs only; the scratch is a 4 MiB array in this library's device module
 * (WF_NOALLOC_SCRATCH_BYTES), which every device that loads the library keeps
 * until the process exits.  A T whose scratch would exceed it is rejected with
 * WF_E_SHAPE before anything runs: at the V4-Flash shapes (hidden 4096, inter
 * 2048, 256 experts, top-6) the limit is T = 48, at hidden 2048 / inter 1024 /
 * 64 experts it is T = 96.  The expert phases run on the mma.sync engine.
 * The first call in a device's context looks the array's device address up
 * (cudaGetSymbolAddress); make that first call before any stream capture.
 * Each call clears the array's completion counters (a cudaMemsetAsync on
 * `stream`) and calls no allocator.  The array's error word is not cleared:
 * it collects the flags of every call (an out-of-range token or expert id, a
 * timed-out device wait) until wf_moe_read_error_noalloc reads and clears it.
 * All calls on a device share the one array and it keeps the last call's
 * contents, so calls that overlap on the GPU (other streams, other threads)
 * race: order them on one stream.  No counterpart in the reference. */
int wf_moe_forward_noalloc(const wf_moe_config *cfg, const wf_moe_weights *w, const void *x,
                           const int64_t *input_ids, int32_t T, void *y, float *out_weights,
                           int64_t *out_indices, void *stream);

/* wf_moe_read_error for wf_moe_forward_noalloc: copies the static scratch's
 * error word to the host (synchronizes `stream`) and clears it; returns 0 or
 * the WF_E_* code of a flag set by any allocation-free call since the last
 * read (a timed-out device wait first).  Allocates nothing.  No counterpart in
 * the reference. */
int wf_moe_read_error_noalloc(void *stream);

/* Expert-parallel forward on a gathered batch with its routing given.  The
 * reference (MoE.forward, architecture.py:749-756, 785-794) has every rank
 * route the whole batch, run its local experts and the shared expert on all
 * of it, and all-reduce.  Here each rank routes only its own tokens
 * (wf_moe_route), the tokens and their routing are all-gathered, and this call
 * runs, on the gathered x [T, D] with in_weights / in_indices [T, topk]
 * (global expert ids):
 *   - the rank's local experts on every row (ascending expert id), and
 *   - the shared expert on rows [shared_row0, shared_row0 + shared_rows) only
 *     (the rank's own tokens; 0 rows for none), added to those rows,
 * into y_partial [T, D] f32.  Reduce-scattering y_partial over the ranks (each
 * rank's shared rows are its own) gives each rank routed + shared for its
 * rows, then wf_moe_to_bf16.  The result equals the whole-layer forward's up to
 * the fp32 order of the cross-rank sum.  Same workspace as wf_moe_forward. */
int wf_moe_forward_ep(const wf_moe_config *cfg, const wf_moe_weights *w, const void *x, int32_t T,
                      const float *in_weights, const int64_t *in_indices, int32_t shared_row0,
                      int32_t shared_rows, float *y_partial, void *workspace, size_t workspace_bytes,
                      void *stream);

/* ---- expert parallelism over peer memory ------------------------------
 * The reference's expert parallelism (MoE.forward under world_size > 1,
 * architecture.py:749-756, 785-794) routes the whole batch on every rank and
 * all-reduces the fp32 partial sums.  Here each rank routes only its own
 * tokens, and one fused launch moves the data over NVLink itself: the rank's
 * E4M3-quantized tokens and their routing go straight into every rank's
 * buffer, each rank runs its local experts on the gathered batch (and the
 * shared expert on its own rows), and writes each token's fp32 partial row
 * into the owner's buffer; a finish kernel sums the ranks' rows in rank
 * order and casts to bf16.  Ranks hand off through epoch flags in the
 * buffers (each rank's buffer counts its completed forwards, so captured CUDA
 * graphs replay correctly); every wait is bounded (WF_E_TIMEOUT).  Set-up: every rank
 * allocates one buffer (wf_ep_alloc, wf_ep_buffer_bytes), exports it
 * (wf_ipc_get_handle), and opens every other rank's (wf_ipc_open_handle). */
#define WF_IPC_HANDLE_BYTES 64
#define WF_EP_MAX_RANKS 8

/* Bytes of the per-rank buffer for `world` ranks; cfg->max_tokens is the
 * capacity of the gathered batch (world x tokens per rank). */
size_t wf_ep_buffer_bytes(const wf_moe_config *cfg, int32_t world);

/* Set-up only (the one entry point that allocates): cudaMalloc of an
 * expert-parallel buffer, zero-filled; wf_ep_free releases it. */
int wf_ep_alloc(size_t bytes, void **buf);
int wf_ep_free(void *buf);

/* CUDA IPC of a buffer between the ranks' processes: export (64 bytes),
 * map another process's buffer into this one, unmap. */
int wf_ipc_get_handle(const void *buf, void *handle);
int wf_ipc_open_handle(const void *handle, void **buf);
int wf_ipc_close_handle(void *buf);

/* One expert-parallel layer forward of this rank's T tokens x [T, D] (bf16),
 * on the fused engine: bufs[p] is rank p's buffer as mapped in this process
 * (bufs[rank] this rank's own); every rank of the group makes the same
 * sequence of calls, one stream each.  cfg: the rank's shard
 * (n_local_experts = E / world, expert_offset = rank * n_local_experts) and
 * max_tokens >= world * T.  Writes y [T, D] bf16 and, optionally, this rank's
 * routing (out_weights / out_indices [T, topk]).  Launches 2 kernels. */
int wf_moe_forward_ep_p2p(const wf_moe_config *cfg, const wf_moe_weights *w, const void *x,
                          const int64_t *input_ids, int32_t T, int32_t rank, int32_t world,
                          void *const *bufs, void *y, float *out_weights, int64_t *out_indices,
                          void *workspace, size_t workspace_bytes, void *stream);

/* dst[i] = bf16(src[i]) for i < n (round to nearest even): the last step of
 * MoE.forward's output (architecture.py:794) after the cross-rank sum. */
int wf_moe_to_bf16(const float *src, int64_t n, void *dst, void *stream);

/* y[i] = bf16(parts[0*n + i] + parts[1*n + i] + ... + parts[(P-1)*n + i]), summed
 * left to right in f32, for i < n (n a multiple of 4; parts 16-byte, y 8-byte
 * aligned): the combine after an all-to-all of the ranks' partial rows, the
 * reference's all_reduce + cast (architecture.py:791-794) in a fixed order that
 * does not depend on the collective's algorithm. */
int wf_moe_sum_ranks(const float *parts, int32_t P, int64_t n, void *y, void *stream);

/* Expert-parallel epilogue: y[t] = bf16(y_partial_reduced[t] + shared_out[row0 + t])
 * for t < T, where shared_out is the shared expert's output that the last
 * wf_moe_forward on this workspace left in it (architecture.py:791-794, after
 * dist.all_reduce; row0 selects this rank's rows of an all-gathered batch). */
int wf_moe_finish(const wf_moe_config *cfg, const float *y_partial_reduced, int32_t T,
                  int32_t row0, void *y, const void *workspace, size_t workspace_bytes,
                  void *stream);

/* Router only: Gate.forward (architecture.py:696-718).  Writes weights
 * [T, topk] f32 and indices [T, topk] int64 (descending biased score). */
int wf_moe_route(const wf_moe_config *cfg, const wf_moe_weights *w, const void *x,
                 const int64_t *input_ids, int32_t T, float *out_weights,
                 int64_t *out_indices, void *workspace, size_t workspace_bytes, void *stream);

/* Copies the workspace's device error word to the host (synchronizes the
 * stream) and clears it.  The word collects the flags of every call on this
 * workspace since it was last read; returns 0 or the negative WF_E_* code of
 * a flag that is set (a timed-out device wait first). */
int wf_moe_read_error(const void *workspace, size_t workspace_bytes, void *stream);

/* Bound, in SM clock cycles, of the layer kernels' waits on another role's
 * progress (a pipeline stage, an operand, an accumulator) for launches made
 * after this call, process-wide; cycles <= 0 restores the default (2e9 cycles,
 * about a second).  A wait that runs past it sets WF_E_TIMEOUT in the error
 * word and the kernel winds down: waits for the calling thread's own copies
 * and MMAs keep the default bound, so no CTA exits or frees tensor memory
 * with work in flight, and the context stays usable.  A failure-detection
 * hook (tests lower it so that a wait runs out); no counterpart in the
 * reference, whose waits are the host's (serving/chain.py:276-316). */
int wf_set_wait_limit(int64_t cycles);

/* Number of kernels this library has launched in this process, counting a
 * launch recorded into a stream capture once (measurement: the kernels a
 * timed region runs).  No counterpart in the reference. */
uint64_t wf_launch_count(void);

/* act_quant (wanferenz/kernels/torch_ops.py:33-49; TileLang reference.py:117-146):
 * x [M, K] bf16 -> q [M, K] e4m3 and s [M, K/block] scales of `scale_kind`.
 * ue8m0 != 0 rounds each scale up to a power of two (scale_fmt="ue8m0"). */
int wf_act_quant(const void *x, int64_t M, int64_t K, int32_t block, int32_t ue8m0, void *q,
                 void *s, int32_t scale_kind, void *stream);

/* fp4_act_quant (torch_ops.py:61-74; TileLang reference.py:212-232):
 * x [M, K] bf16 -> packed E2M1 [M, K/2] and e8m0 scales [M, K/32]. */
int wf_fp4_act_quant(const void *x, int64_t M, int64_t K, void *q, void *s, void *stream);

/* fp8_gemm (torch_ops.py:93-99; TileLang reference.py:292-311):
 * out[M, N] bf16 = (a * a_s) @ (b * b_s)^T with a [M, K] e4m3,
 * a_s [M, K/128], b [N, K] e4m3, b_s [ceil(N/128), K/128]. */
int wf_fp8_gemm(const void *a, const void *a_s, int32_t a_scale_kind, const void *b,
                const void *b_s, int32_t b_scale_kind, int64_t M, int64_t N, int64_t K,
                void *out, void *workspace, size_t workspace_bytes, void *stream);

/* fp4_gemm (torch_ops.py:102-108; TileLang reference.py:572-591):
 * out[M, N] bf16 = (a * a_s) @ (unpack(b) * b_s)^T with b [N, K/2] fp4
 * packed and b_s [N, K/32] e8m0. */
int wf_fp4_gemm(const void *a, const void *a_s, int32_t a_scale_kind, const void *b,
                const void *b_s, int64_t M, int64_t N, int64_t K, void *out, void *workspace,
                size_t workspace_bytes, void *stream);

/* grouped_fp4_gemm (wanferenz/kernels/fp4_grouped.py:96-128): slot g
 * multiplies a[g] [K] e4m3 by its own weights w[g] [N, K/2] fp4:
 * out[g, N] bf16 = (a[g] * a_s[g]) @ (unpack(w[g]) * w_s[g])^T. */
int wf_grouped_fp4_gemm(const void *a, const void *a_s, int32_t a_scale_kind, const void *w,
                        const void *w_s, int64_t G, int64_t N, int64_t K, void *out,
                        void *workspace, size_t workspace_bytes, void *stream);

/* Workspace bytes for the dense GEMM entry points above.  The workspace is
 * zero-filled once when allocated; its split-K counters return to zero at
 * the end of every call.  The library clears them again only when the shape
 * (or the engine) a workspace serves changes, so a workspace is used by one
 * stream at a time, and a call that failed (WF_E_TIMEOUT in the error word,
 * the first 4 bytes) leaves it to be re-zeroed by the caller. */
size_t wf_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K);

/* Load-time check that no FP4 weight scale byte is 0 or 255 (2^-127, the
 * subnormal the kernels do not decode, or NaN).  Synchronizes the stream.
 * Returns 1 (in range), 0 (not) or a negative WF_E_* code. */
int wf_fp4_scales_in_range(const uint8_t *scales, int64_t n, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* WFB200_H */
