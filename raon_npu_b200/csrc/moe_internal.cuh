// Definitions shared by the MoE translation units (decode: q4nx_moe.cu,
// prefill: q4nx_prefill.cu): limits, the per-layer device scratch and the
// layer object behind the C-ABI handle ``rc_moe``.
#pragma once

#include <stdint.h>

#include "rc_internal.cuh"

namespace rc {

constexpr int kMoeMaxK = 16;               // routed experts per token
constexpr int kMoeMaxTokens = 16;          // tokens per call: two 8-column mma blocks
constexpr int kPfMaxTokens = 4096;         // tokens per prefill call
constexpr int kMoeMaxExperts = 256;
constexpr int kMoeWarps = 16;
constexpr int kMoePartialBytes = 32 * 1024;   // per-CTA unit partials of one round
constexpr int kMoeMaxStages = 8;
constexpr int kMoeMaxGroupsPerCta = 4;     // down kernel: groups one CTA's tile range may touch

// Per-call device scratch of a layer.
struct MoeScratch {
  float *logits;           // [T][E]
  int *counter;            // [T + 1] arrival counters (per token, then "all tokens"), zero between calls
  int32_t *ids;            // [T][k] rank order (best first)
  float *weights;          // [T][k]
  int32_t *slot_expert;    // [T][k+1] ascending ID, then the shared expert (or -1)
  float *slot_w;           // [T][k]   weights in slot order
  int *n_groups;           // [1]
  int32_t *group_expert;   // [E+1]
  uint32_t *group_mask;    // [E+1] tokens of each group
  int32_t *group_dst;      // [E+1][16] slot row of (group, token)
  int *err;                // the context's device error word
};

// What one rank computes: routed experts [lo, hi) for every token, the shared
// expert (id E) for the tokens in shared_mask.
struct MoeOwned {
  int lo, hi;
  uint32_t shared_mask;
};

struct PfScratch;   // prefill scratch (q4nx_prefill.cu)

// Expert parallelism over peer memory: this rank's exchange buffer
//   [0, kEpFlagBytes)  u64 counters: [0] token-row arrivals (every rank adds
//                      1 per call), [2] calls done
//   tok                [world*M][hidden] bf16: every rank's token rows
//   red                [M][k+1][hidden/16][8] u64: the expert rows of this
//                      rank's tokens, each written by the rank that owns the
//                      expert (slot k: the shared expert, written here); word
//                      g of (token, slot, 16-column tile) holds rows g and
//                      g + 8 of the tile as bf16 (bits 0-31) and the number
//                      of the call that wrote it (bits 32-63)
constexpr int kEpMaxRanks = 8;
constexpr size_t kEpFlagBytes = 256;
struct MoeEp {
  int rank, world, M;
  uint8_t *base;                    // this rank's exchange buffer
  size_t bytes;
  uint8_t *peer[kEpMaxRanks];       // every rank's buffer, mapped here (own: base)
  bool mapped[kEpMaxRanks];
  uint8_t uuid[kEpMaxRanks][16];    // the GPU each buffer lives on
  uint8_t **peer_dev;               // device copy of peer[]
  unsigned epoch;                   // ctx->timeout_epoch at rc_moe_ep_init
};
// The blob rc_moe_ep_init hands out: IPC handle, GPU UUID, geometry.
struct MoeEpBlob {
  uint8_t ipc[64];
  uint8_t uuid[16];
  int32_t rank, world, M, hidden, n_experts, has_shared;
  uint64_t bytes;
};
static_assert(sizeof(MoeEpBlob) <= 128, "exchange blob exceeds RC_EP_HANDLE_BYTES");
inline size_t ep_tok_off() { return kEpFlagBytes; }
inline size_t ep_red_off(int world, int M, int hidden) { return kEpFlagBytes + (size_t)world * M * hidden * 2; }
inline size_t ep_bytes(int world, int M, int hidden) {
  return ep_red_off(world, M, hidden) + (size_t)M * (kMoeMaxK + 1) * hidden * 4;
}

// What the fused kernel needs of an expert-parallel call (null: one GPU).
struct MoeEpArgs {
  int rank, world, M;
  uint8_t *const *peer_dev;
  unsigned long long *flags;
  uint32_t tok_off, red_off;
  const uint16_t *x_own;
};

}  // namespace rc

// ------------------------------------------------------------- MoE object --
struct rc_moe {
  rc_ctx *ctx;
  int hidden, inter, inter_pad, n_experts, has_shared;
  rc_weight **gate_up;        // [E+1] host table of handles (null: not on this rank)
  rc_weight **down;
  const uint8_t **gu_tiles;   // [E+1] device pointer tables
  const uint8_t **dn_tiles;
  uint16_t *router_w;         // [E][hidden] bf16
  float *router_bias;         // [E]
  rc::MoeScratch s;
  uint16_t *act;              // [E+1][16][inter_pad]  (pad columns stay zero)
  uint16_t *down_out;         // [16][kMax+1][hidden]
  rc::PfScratch *pf;          // prefill scratch, grown on demand (null until the first prefill)
  int fused;                  // decode through the single persistent kernel when the shape fits
  unsigned long long *fz_bar; // grid-barrier arrival count of the persistent decode kernel (only grows)
  unsigned fz_epoch;          // ctx->timeout_epoch when fz_bar was last known consistent
  int *dc_cols;               // [hidden/16] down tiles written per output column tile (zero between calls)
  rc::MoeEp *ep;              // peer-memory expert parallelism (null until rc_moe_ep_init)
  int prefill_kernel;         // RC_PREFILL_GEMV (register fragments) or RC_PREFILL_TCGEN05
  int down_fmt;               // kFormatQ4nx or kFormatBfp16 (RC_UPLOAD_DOWN_BFP16), one for every expert
  unsigned long long *trace;  // phase stamps of the persistent decode kernel (rc_moe_set_trace; null: off)
  int trace_ctas;             // CTAs the trace buffer has room for
};

namespace rc {
// Phase stamps of the persistent decode kernel: per CTA, kTracePhases global
// timer readings (ns) at the phase boundaries below, written by thread 0.
enum TracePhase : int {
  kTrStart = 0,      // kernel entered (tables fetched, before any wait)
  kTrTokens,         // expert parallelism: every rank's token rows arrived
  kTrLogits,         // this CTA's router logits written
  kTrRouted,         // grid barrier after the logits passed
  kTrSelected,       // top-k, weights and group table built
  kTrStaged,         // token rows staged as mma fragments
  kTrGateUp,         // this CTA's gate/up tiles done
  kTrActReady,       // the activations this CTA's down tiles read are complete
  kTrDown,           // this CTA's down tiles done
  kTrRows,           // every expert row of the combined tokens is written (grid / peers)
  kTrEnd,            // combine done
  kTrKeys,           // selection: every router key of the tokens in shared memory
  kTrRanked,         // selection: the top-k ranks found
  kTrActStaged,      // down: the activation rows staged as mma fragments
  kTrDownUnits,      // down: this CTA's units computed (first round)
  kTrDownTiles,      // down: this CTA's tiles summed and written (first round)
  kTracePhases = 16
};
}  // namespace rc

namespace rc {
void pf_free(rc_moe *m);   // releases m->pf (q4nx_prefill.cu)
// Router for 16 < T <= 4096 tokens (q4nx_prefill.cu): ids / weights [T][k],
// logits [T][E] (each optional).
// Persistent decode kernel (q4nx_moe_decode.cu).
bool moe_fused_fits(const rc_moe *m, int T, int k, const MoeOwned &own);
bool moe_decode_shape_ok(const rc_moe *m, int T, int k, const MoeOwned &own);
int moe_decode_persistent(rc_moe *m, const uint16_t *x, int T, int k, int router, int renorm, float scaling,
                          int act, float gb, float vb, const MoeOwned &own, uint16_t *slot_rows, int zero_foreign,
                          uint16_t *out, int32_t *ids_out, float *w_out, float *slot_w_out, cudaStream_t s,
                          const MoeEpArgs *ep = nullptr);
int pf_route_tokens(rc_moe *m, const uint16_t *x_dev, int T, int k, int router, int renormalize, float scaling,
                    int32_t *ids_dev, float *w_dev, float *logits_dev, void *stream);
}  // namespace rc
