/*
 * raon_cuda.h -- C ABI of the B200 (sm_100a) q4nx GEMV / MoE backend.
 *
 * This is the drop-in boundary for the GEMV and MoE entry points of the
 * reference's execution backend (raon-npu ``host/backend.py:65-204``, the
 * ``Backend`` ABC, implemented on the NPU by ``npu/backend.py``).  Every
 * function takes plain pointers and sizes, returns an ``int`` status
 * (RC_OK == 0) and leaves a thread-local message for ``rc_last_error``.
 *
 * Conventions (reference ``host/backend.py:9-14``): bf16 values travel as
 * uint16 bit patterns; an f32 activation gives an f32 result.  Device
 * pointers are CUDA device addresses on the context's device; ``stream``
 * arguments are ``cudaStream_t`` values (NULL = the context's own stream).
 */
#ifndef RAON_CUDA_H
#define RAON_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RC_OK 0
#define RC_ERR_INVALID 1   /* bad shape / dtype / id: the reference raises ValueError */
#define RC_ERR_NOT_FOUND 2 /* unknown weight handle: the reference raises KeyError   */
#define RC_ERR_CUDA 3      /* CUDA runtime failure: RuntimeError                      */
#define RC_ERR_TIMEOUT 4   /* a bounded device-side wait ran out: RuntimeError        */

#define RC_DTYPE_BF16 0
#define RC_DTYPE_F32 1

#define RC_ACT_SWIGLU 0 /* g*sigmoid(g)*u        (kernels/moe/reference.py:160-170) */
#define RC_ACT_SITU 1   /* SiTU-GLU with betas   (host/backend.py:47-62)            */

#define RC_ROUTER_SOFTMAX 0      /* softmax(x.Wr + b) -> top-k -> renormalise (b: router bias, 0 unless set) */
#define RC_ROUTER_SIGMOID_BIAS 1 /* sigmoid, top-k of score+bias (host/raon.py:1224-1247) */

/* Upload flags. */
#define RC_UPLOAD_SRC_DEVICE 1u /* ``packed`` is a device pointer, not host memory        */
#define RC_UPLOAD_GATE_UP 2u    /* rows are [gate; up] halves (kernels/moe/pack.py:136-172):
                                   store them interleaved so the GEMV epilogue can apply
                                   the GLU activation in registers                        */
#define RC_UPLOAD_DOWN_BFP16 4u /* rc_moe_set_expert: ``down`` is a bfp16ebs8 matrix in the
                                   reference's pack_bfp16_gemv bytes (its moe_b2 expert
                                   bundles, npu/backend.py:640-652), [hidden][inter_pad]
                                   at 9 bits a weight; every expert of a layer has the
                                   same down format.  Such a layer runs rc_moe_experts,
                                   rc_moe_experts_grouped and rc_moe_decode(_local)
                                   through the separate launches (T <= 16) and the
                                   prefill entry points on the register-fragment
                                   path; rc_moe_ep_decode refuses it.                     */

typedef struct rc_ctx rc_ctx;
typedef struct rc_weight rc_weight;

/* Thread-local text of the last failure on this thread (never NULL). */
const char *rc_last_error(void);

/* ABI version; bumps on any signature change. */
int rc_abi_version(void);

/* Create a context on ``device``: one CUDA stream, scratch memory, SM count.
 * Replaces the device/runner set-up of ``NpuBackend.__init__``
 * (npu/backend.py:2404-2485). */
int rc_init(int device, rc_ctx **out);
int rc_destroy(rc_ctx *ctx);

/* The context's stream as a ``cudaStream_t`` (for callers that order work on it). */
int rc_stream(rc_ctx *ctx, void **stream_out);

/* Block until all work on the context's device is done (its own stream and
 * any caller streams), then report any error word a kernel left
 * (RC_ERR_TIMEOUT for a bounded wait that gave up). */
int rc_sync(rc_ctx *ctx);

/* Number of SMs of the context's device (the persistent grids are sized by it). */
int rc_sm_count(rc_ctx *ctx, int *out);

/* Upload one q4nx matrix given as ``pack_gemv`` bytes (quant/q4nx.py:335-393,
 * rows=4: N % 128 == 0, K % 256 == 0, nbytes == N*K*5/8) and repack it once,
 * on the device, into the GEMV tile layout.  Replaces the bundle upload of
 * ``NpuBackend._get_weight_tensor`` (npu/backend.py:3127-3148), which hands the
 * same bytes to the NPU unchanged. */
int rc_upload_q4nx(rc_ctx *ctx, const uint8_t *packed, size_t nbytes, int n, int k,
                   unsigned flags, rc_weight **out);
/* Quantise an f32 [N, K] device matrix to q4nx and write its ``pack_gemv``
 * bytes (N*K*5/8, device memory), bit-identical to the reference's offline
 * converter ``quantize`` + ``pack_gemv`` (quant/q4nx.py:127-200,335-393).
 * Synchronous; RC_ERR_INVALID for non-finite input, as the reference. */
int rc_quantize_q4nx(rc_ctx *ctx, const float *w_dev, int n, int k, uint8_t *packed_dev, void *stream);

/* Upload a bfp16ebs8 matrix (9-bit block floating point: 8-column groups
 * sharing an exponent byte, int8 mantissas; the reference's second weight
 * format, quant/bfp16.py:1-60) from the reference's GEMV packing
 * ``pack_bfp16_gemv`` (quant/bfp16.py:190-292), N*K*9/8 bytes, kept unchanged
 * in HBM.  rc_gemv / rc_gemv_host then compute its GEMV as the reference's
 * kernels/gemv_bfp16 does (reference.py:118-182: exact products with bf16
 * activations, f32 accumulation, RTNE), bf16 activations only; the MoE, the
 * q4nx dequantiser and rc_gemv_noalloc take q4nx matrices only.  Flags:
 * RC_UPLOAD_SRC_DEVICE. */
int rc_upload_bfp16(rc_ctx *ctx, const uint8_t *packed, size_t nbytes, int n, int k, unsigned flags,
                    rc_weight **out);

int rc_weight_free(rc_weight *w);
int rc_weight_info(const rc_weight *w, int *n, int *k, size_t *device_bytes, unsigned *flags);

/* Attach an f32 bias [N] (host memory) to a matrix; ``rc_weight_bias`` returns
 * its device address for the ``bias_dev`` argument of rc_gemv.  The reference
 * adds ``<name>.bias`` in f32 before rounding (host/backend.py:410-413). */
int rc_weight_set_bias(rc_weight *w, const float *bias_host);
int rc_weight_bias(const rc_weight *w, const float **bias_dev);

/* Dequantise an uploaded matrix to f32 [N, K] (row-major, device memory):
 * ``f32(f64(min) + f64(scale) * code)``, bit-identical to the reference's
 * ``parse_gemv`` + ``dequantize_simple`` (quant/q4nx.py:203-223,396-438).
 * For an RC_UPLOAD_GATE_UP matrix the rows come back in the original
 * [gate; up] order. */
int rc_dequant_q4nx(rc_ctx *ctx, const rc_weight *w, float *out_dev, void *stream);

/* y[t, r] = x[t, :] . W[row0 + r, :] (+ bias[row0 + r]) for t < T, r < nrows.
 * Replaces ``Backend.linear`` / ``linear_batch`` (host/backend.py:71-83,
 * numpy oracle host/backend.py:402-417; NPU npu/backend.py:3569-3721).
 *   x_dtype RC_DTYPE_BF16, y_dtype RC_DTYPE_BF16: bf16 bits in, RTNE bf16 out
 *                                                 (the reference's contract);
 *   x_dtype RC_DTYPE_BF16, y_dtype RC_DTYPE_F32:  the same f32 sums, unrounded
 *                                                 (e.g. f32 logits);
 *   x_dtype RC_DTYPE_F32,  y_dtype RC_DTYPE_F32:  f32 in, f32 out.
 * row0 and nrows must be multiples of 16 (use a wider range and slice for
 * others).  ``bias`` is f32 [N] or NULL.  Any T >= 1; a row's result does
 * not depend on T or on the other rows (linear_batch == stacked linear). */
int rc_gemv(rc_ctx *ctx, const rc_weight *w, const void *x_dev, int x_dtype, int ldx, int T,
            void *y_dev, int y_dtype, int ldy, int row0, int nrows, const float *bias_dev,
            void *stream);

/* Same as rc_gemv on host buffers: copies x in, runs, copies y out, waits. */
int rc_gemv_host(rc_ctx *ctx, const rc_weight *w, const void *x_host, int x_dtype, int T,
                 void *y_host, const float *bias_dev);

/* ------------------------------------------------------------------ MoE ---
 * One MoE layer: n_experts routed experts (+ an optional shared expert, id
 * n_experts), each a q4nx [gate; up] matrix [2*inter, hidden] and a down
 * matrix [hidden, inter_pad] (inter zero-padded to a multiple of 256), both
 * as pack_gemv bytes -- the reference's expert packers
 * (kernels/moe/pack.py:136-224).  Expert parallelism: a rank loads the
 * experts it computes (rc_moe_decode_local). */
typedef struct rc_moe rc_moe;

int rc_moe_create(rc_ctx *ctx, int hidden, int inter, int n_experts, int has_shared, rc_moe **out);
int rc_moe_destroy(rc_moe *m);

/* Upload expert ``expert`` (0..n_experts-1, or n_experts for the shared one):
 * flags RC_UPLOAD_SRC_DEVICE and RC_UPLOAD_DOWN_BFP16. */
int rc_moe_set_expert(rc_moe *m, int expert, const uint8_t *gate_up, size_t gate_up_bytes,
                      const uint8_t *down, size_t down_bytes, unsigned flags);

/* Router weights bf16 [n_experts][hidden] (host) and, for the sigmoid+bias
 * router, the per-expert correction bias f32 [n_experts] (or NULL). */
int rc_moe_set_router(rc_moe *m, const uint16_t *router_w, const float *bias);

/* Decode path of rc_moe_decode / rc_moe_decode_local: enable != 0 (the
 * default) runs router, experts and combine as one persistent cooperative
 * kernel when the shape fits it; 0 always uses the separate launches.  Both
 * give the same bytes. */
int rc_moe_set_fused(rc_moe *m, int enable);

/* Phase stamps of the persistent decode kernel (rc_moe_decode, _local,
 * rc_moe_ep_decode), for measurement: while stamps_dev is set, every launch
 * writes, per CTA c, 16 global-timer readings in ns at stamps_dev[c*16 + i]
 * (0 where a phase does not apply): 0 start, 1 every rank's token rows
 * arrived (expert parallelism), 2 this CTA's router logits written, 3 the
 * grid passed the logits, 4 top-k and group table built, 5 token rows
 * staged, 6 this CTA's gate/up tiles done, 7 the activations its down tiles
 * read are complete, 8 its down tiles done, 9 every expert row of the
 * combined tokens written, 10 combine done, 11 the tokens' router keys in
 * shared memory, 12 the top-k ranks found, 13 the activation rows its down
 * tiles read staged, 14 its first down round's units computed, 15 that
 * round's tiles summed and written.  ``ctas`` >= the SM count;
 * NULL switches the stamps off.  No counterpart in the reference. */
int rc_moe_set_trace(rc_moe *m, unsigned long long *stamps_dev, int ctas);

/* Router for T <= 4096 tokens x [T][hidden] (device): top-k ids (best first,
 * lower index wins ties) and weights, optional f32 logits [T][n_experts].
 * Replaces the host router ``RaonModel._route_token`` (host/raon.py:1224-1247)
 * and the softmax top-k of the north-star configs. */
int rc_moe_route(rc_moe *m, const uint16_t *x_dev, int T, int k, int router, int renormalize,
                 float scaling, int32_t *ids_dev, float *w_dev, float *logits_dev, void *stream);

/* Routed experts of T <= 16 tokens for caller-supplied top-k ids / weights
 * [T][k] (device arrays, any order within a token, distinct ids):
 * ``Backend.moe_experts`` (host/backend.py:98-117, numpy
 * host/backend.py:466-510; NPU npu/backend.py:5029-5322) for T = 1.  Experts
 * are summed in ascending ID in f32, then RTNE.  with_shared != 0 also adds
 * the shared expert as ``_moe_token`` does (host/raon.py:1310-1327).
 * x [T][hidden] bf16, out [T][hidden] bf16. */
int rc_moe_experts(rc_moe *m, const uint16_t *x_dev, int T, const int32_t *ids_dev, const float *w_dev,
                   int k, int act, float gate_beta, float value_beta, int with_shared, uint16_t *out_dev,
                   void *stream);

/* rc_moe_experts on host buffers: copies in, runs, copies out, waits.
 * Validates the ids (range, loaded, distinct per token) as the reference's
 * ValueError checks do. */
int rc_moe_experts_host(rc_moe *m, const uint16_t *x_host, int T, const int32_t *ids_host,
                        const float *w_host, int k, int act, float gate_beta, float value_beta,
                        int with_shared, uint16_t *out_host);

/* ``moe_experts_grouped`` (npu/backend.py:4845-4979): routed sums
 * routed_out [T][hidden] and, when shared_gu [T][2*inter] (the shared
 * expert's gate | up rows, computed by the caller) is given, the shared
 * expert's down rows shared_out [T][hidden] = linear(shared_down,
 * RTNE(act(gate, up))).  T is 1..4096: above 16 tokens the routed experts run
 * on the prefill kernels (rc_moe_prefill_experts) and the shared rows in
 * 16-token chunks of the decode kernels; every token's bytes are those of a
 * call of at most 16 tokens. */
int rc_moe_experts_grouped(rc_moe *m, const uint16_t *x_dev, int T, const int32_t *ids_dev,
                           const float *w_dev, int k, const uint16_t *shared_gu_dev, int act,
                           float gate_beta, float value_beta, uint16_t *routed_out_dev,
                           uint16_t *shared_out_dev, void *stream);

/* The whole decode layer for T <= 16 tokens: router, routed + shared experts,
 * combine; optional copies of the selected ids / weights [T][k]. */
int rc_moe_decode(rc_moe *m, const uint16_t *x_dev, int T, int k, int router, int renormalize,
                  float scaling, int act, float gate_beta, float value_beta, uint16_t *out_dev,
                  int32_t *ids_dev, float *w_dev, void *stream);

/* rc_moe_decode, rc_moe_prefill and rc_moe_ep_decode on host buffers (the
 * entry a host runtime such as the reference's ``Backend`` binds): x_host
 * [T][hidden] (rc_moe_ep_decode_host: [tokens_per_rank][hidden]) is copied in
 * through pinned staging, the layer runs on ``stream`` (NULL: the context's),
 * out_host (and ids_host / w_host [T][k] when given) are copied back, and one
 * wait covers the results and the device error word.  Work the caller queued
 * on other streams is not waited for. */
int rc_moe_decode_host(rc_moe *m, const uint16_t *x_host, int T, int k, int router, int renormalize,
                       float scaling, int act, float gate_beta, float value_beta, uint16_t *out_host,
                       int32_t *ids_host, float *w_host, void *stream);
int rc_moe_prefill_host(rc_moe *m, const uint16_t *x_host, int T, int k, int router, int renormalize,
                        float scaling, int act, float gate_beta, float value_beta, uint16_t *out_host,
                        int32_t *ids_host, float *w_host, void *stream);
int rc_moe_ep_decode_host(rc_moe *m, const uint16_t *x_host, int k, int router, int renormalize,
                          float scaling, int act, float gate_beta, float value_beta, uint16_t *out_host,
                          void *stream);

/* Expert-parallel halves of rc_moe_decode.  decode_local routes all T tokens,
 * runs the routed experts [expert_lo, expert_hi) for every token and the
 * shared expert for tokens [shared_t0, shared_t0 + shared_tn), and writes the
 * slot rows slot_out [T][k+1][hidden] (slot r < k: the r-th selected expert in
 * ascending ID; slot k: the shared expert; zeros where another rank computes
 * the slot) and the slot weights slot_w [T][k].  Once the ranks' slot rows
 * are summed (each row is non-zero on at most one rank, so the sum is exact),
 * rc_moe_combine produces the same bytes as rc_moe_decode on one GPU. */
int rc_moe_decode_local(rc_moe *m, const uint16_t *x_dev, int T, int k, int router, int renormalize,
                        float scaling, int act, float gate_beta, float value_beta, int expert_lo,
                        int expert_hi, int shared_t0, int shared_tn, uint16_t *slot_out_dev,
                        float *slot_w_dev, void *stream);
int rc_moe_combine(rc_moe *m, const uint16_t *slot_out_dev, const float *slot_w_dev, int T, int k,
                   int with_shared, uint16_t *out_dev, void *stream);

/* Expert parallelism over peer memory (NVLink), the exchange inside the
 * decode kernel (replaces the reference's expert-parallel all-gather /
 * reduce-scatter around the local expert GEMVs, and the NCCL path through
 * rc_moe_decode_local).  ``world`` ranks, one process per GPU and every GPU
 * distinct (at most RC_EP_MAX_RANKS), each hold the routed experts
 * [rank*E/world, (rank+1)*E/world) plus the shared expert and decode
 * ``tokens_per_rank`` tokens per call (world * tokens_per_rank <= 16).
 *
 * rc_moe_ep_init allocates this rank's exchange buffer and writes an
 * RC_EP_HANDLE_BYTES blob to handle_out (its CUDA IPC handle, the GPU's UUID
 * and the geometry).  Once every rank has every blob, rc_moe_ep_open(peer)
 * maps each other rank's buffer; it checks that the blob is that rank's, of
 * the same geometry, and from a different GPU.  rc_moe_ep_decode is then one
 * persistent kernel per call: the rank's token rows are stored into every
 * peer's buffer, every rank routes all world*M tokens, computes its experts
 * for every token and the shared expert for its own, stores each expert row
 * straight into the buffer of the token's owner (exactly one rank writes each
 * row) and combines its own tokens into out_dev [M][hidden] -- the bytes of
 * rc_moe_decode on one GPU.  Every rank makes the same sequence of calls on
 * one stream.  Every wait for a peer is bounded (1 s): the call then fails
 * with RC_ERR_TIMEOUT at the next synchronising call, and the exchange state
 * is lost -- rc_moe_ep_decode refuses until rc_moe_ep_init and
 * rc_moe_ep_open are run again on every rank. */
#define RC_EP_MAX_RANKS 8
#define RC_EP_HANDLE_BYTES 128
int rc_moe_ep_init(rc_moe *m, int rank, int world, int tokens_per_rank, void *handle_out);
int rc_moe_ep_open(rc_moe *m, int peer, const void *handle);
int rc_moe_ep_decode(rc_moe *m, const uint16_t *x_dev, int k, int router, int renormalize, float scaling,
                     int act, float gate_beta, float value_beta, uint16_t *out_dev, void *stream);

/* Which kernel runs the prefill experts' GEMMs (same routing, plan and
 * combine; results within the oracle tolerance of each other):
 * RC_PREFILL_TCGEN05 (default) -- the tcgen05 grouped GEMM over 64-token
 * chunks (warp-specialised: TMA loads, bf16 expansion of the codes, MMAs
 * into one tensor-memory accumulator per 32-column group, promotion);
 * RC_PREFILL_GEMV -- a grouped GEMV over 8-token blocks with the decode
 * GEMV's register-fragment (mma.sync) unit arithmetic: a token's bytes equal
 * the decode path's, and it is the faster of the two below a few hundred
 * tokens.  rc_moe_experts_grouped always uses RC_PREFILL_GEMV for T > 16,
 * so its bytes do not depend on T.  Layers with bfp16ebs8 down matrices
 * always use RC_PREFILL_GEMV. */
#define RC_PREFILL_GEMV 0
#define RC_PREFILL_TCGEN05 1
int rc_moe_set_prefill_kernel(rc_moe *m, int kernel);

/* MoE prefill: the layer for T <= 4096 tokens over expert-sorted token rows
 * (the reference's grouped path, npu/backend.py:4845-4979 with
 * kernels/moe_grouped/planner.py:76-108,286-322; the experts' GEMMs as
 * rc_moe_set_prefill_kernel selects).  Same semantics as rc_moe_decode: router
 * (top-k ids / weights [T][k] copied out when given), routed experts summed
 * in ascending ID in f32 then RTNE, plus the shared expert.  x and out are
 * [T][hidden] bf16, 16-byte aligned.  Scratch grows on the first call for a
 * larger T (that call synchronises the device). */
int rc_moe_prefill(rc_moe *m, const uint16_t *x_dev, int T, int k, int router, int renormalize,
                   float scaling, int act, float gate_beta, float value_beta, uint16_t *out_dev,
                   int32_t *ids_dev, float *w_dev, void *stream);

/* rc_moe_prefill for caller-supplied routes ids / w [T][k] (distinct ids per
 * token; an id whose expert is not loaded sets the device error word).  On a
 * layer with a shared expert a route may also name it (id n_experts), like a
 * routed expert -- the expert-parallel prefill's jobs do so. */
int rc_moe_prefill_experts(rc_moe *m, const uint16_t *x_dev, int T, const int32_t *ids_dev,
                           const float *w_dev, int k, int act, float gate_beta, float value_beta,
                           int with_shared, uint16_t *out_dev, void *stream);

/* Expert-parallel halves of rc_moe_prefill, as rc_moe_decode_local /
 * rc_moe_combine: slot rows slot_out [T][k+1][hidden] of the routed experts
 * [expert_lo, expert_hi) and of the shared expert for tokens
 * [shared_t0, shared_t0 + shared_tn), zeros elsewhere, and the slot weights
 * [T][k]; after the ranks' slot rows are summed, rc_moe_prefill_combine gives
 * the bytes of rc_moe_prefill on one GPU. */
int rc_moe_prefill_local(rc_moe *m, const uint16_t *x_dev, int T, int k, int router, int renormalize,
                         float scaling, int act, float gate_beta, float value_beta, int expert_lo,
                         int expert_hi, int shared_t0, int shared_tn, uint16_t *slot_out_dev,
                         float *slot_w_dev, void *stream);
/* rc_moe_prefill_local for caller-supplied routes ids / w [T][k] (rank order,
 * as rc_moe_route returns them): the expert-parallel prefill routes each
 * rank's own tokens and exchanges the routes with the token rows, so no rank
 * routes another's tokens.  With the prefill router's routes (rc_moe_route,
 * T > 16) the slot rows and weights are those of rc_moe_prefill_local. */
int rc_moe_prefill_local_routes(rc_moe *m, const uint16_t *x_dev, int T, const int32_t *ids_dev,
                                const float *w_dev, int k, int act, float gate_beta, float value_beta,
                                int expert_lo, int expert_hi, int shared_t0, int shared_tn,
                                uint16_t *slot_out_dev, float *slot_w_dev, void *stream);
int rc_moe_prefill_combine(rc_moe *m, const uint16_t *slot_out_dev, const float *slot_w_dev, int T,
                           int k, int with_shared, uint16_t *out_dev, void *stream);

/* Token sampling on bf16 logits [T][ld] (device), the reference's
 * ``sample_token`` (serve/engine.py:84-140) in f64: presence penalty over each
 * token row's seen ids (concatenated in seen_dev, row t at
 * [seen_off[t], seen_off[t+1]); both NULL for none), then greedy argmax when
 * temperature <= 0, else top-k (1..1024, ties kept) -> top-p -> temperature ->
 * categorical draw with the caller's uniform u_dev[t] in [0, 1) (the value
 * numpy's Generator.random() would feed Generator.choice).  out_dev [T] int32.
 * A vocabulary-wide top-p without top-k is not supported (RC_ERR_INVALID). */
int rc_sample_tokens(rc_ctx *ctx, const uint16_t *logits_dev, int ld, int T, int V, int top_k,
                     double top_p, double temperature, double presence_penalty,
                     const int32_t *seen_dev, const int32_t *seen_off_dev, const double *u_dev,
                     int32_t *out_dev, void *stream);

/* out = RTNE(f32(a) + f32(b)) over n bf16 values (device, 16-byte aligned):
 * the residual add between the blocks of a decode step. */
int rc_add_bf16(rc_ctx *ctx, const uint16_t *a_dev, const uint16_t *b_dev, uint16_t *out_dev, long long n,
                void *stream);

/* Per row r of [rows][n]: s = f32(a) + f32(b); out = RTNE(s / sqrt(mean(s^2) + eps)) -- the
 * residual add followed by an RMS normalisation (no learned scale). */
int rc_add_rms_bf16(rc_ctx *ctx, const uint16_t *a_dev, const uint16_t *b_dev, uint16_t *out_dev, int rows,
                    int n, float eps, void *stream);

/* rc_gemv without any device allocation (this entry point has no counterpart
 * in the reference).  Arguments and results are those of rc_gemv, bit for
 * bit, for q4nx matrices only: a bfp16ebs8 matrix gets RC_ERR_INVALID.  The
 * context is the one the weight was uploaded with.
 *
 * Who needs it: callers that must not allocate device memory while they run
 * a GEMV -- a latency-critical serving thread that cannot afford the implicit
 * device-wide synchronisation cudaMalloc/cudaFree may perform, or a host that
 * reserves a fixed device-memory budget at start-up (weights, caches) and
 * forbids allocations afterwards.  rc_gemv may grow its scratch with
 * cudaMalloc on first use of a larger shape; this function never calls
 * cudaMalloc, cudaFree or anything that allocates.
 *
 * How: the split-K scratch (per-tile counters, per-warp partial sums) lives in
 * one static device array of 5,308,416 bytes that every GPU which loads this
 * library keeps until the process exits.  The first call on a device looks up
 * that array's device address (cudaGetSymbolAddress) with the device current;
 * make this first call before any stream capture.  Every call shares the
 * array, which keeps the last call's contents: each call clears the counters
 * it uses, and calls that overlap on the GPU (different streams or threads)
 * race -- keep them ordered on one stream.  The looked-up address is kept for
 * the life of the process: after a cudaDeviceReset (which also ends every
 * context and weight of this library on that device) the entry point must not
 * be called again in that process.
 *
 * Limits (RC_ERR_INVALID beyond them): nrows <= 262,144; the activations of
 * one launch must fit in shared memory -- K <= 5,120 for up to 16 bf16 rows
 * per call (8 f32 rows), K <= 10,240 for up to 8 bf16 rows per call. */
int rc_gemv_noalloc(const rc_weight *w, const void *x_dev, int x_dtype, int ldx, int T,
                    void *y_dev, int y_dtype, int ldy, int row0, int nrows,
                    const float *bias_dev, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* RAON_CUDA_H */
