// MoE decode on the q4nx experts: router top-k, token grouping by expert,
// grouped expert GEMVs with the GLU activation fused into the gate/up
// epilogue, and the ascending-expert-ID combine.  Everything stays on the
// device, so a layer is a fixed chain of launches (graph-capturable) with no
// host round trip between router and experts.
//
// Reference semantics (raon-npu):
//   router      host/raon.py:1224-1247 (sigmoid + bias) and the softmax top-k
//               of the north-star configs; lower expert index wins ties.
//   experts     host/backend.py:466-510: per expert gate/up linear (bf16),
//               act -> RTNE, down linear (bf16); f32 weighted sum over the
//               experts in ascending ID, then RTNE.
//   shared      host/raon.py:1310-1327: out = RTNE(f32(routed) + f32(shared)).
//   grouped     npu/backend.py:4845-4979: T tokens, routed sums plus the shared
//               expert's down rows from caller-supplied shared gate/up rows.
//
// Work layout for T <= 16 tokens (one or two 8-column mma blocks):
//   groups      one per active expert, ascending ID, the shared expert last;
//               group g carries a token mask and, per token, the destination
//               slot row t*(k+1) + (position of the expert in the token's
//               ascending list; k for the shared expert).
//   gate/up     every warp takes whole row tiles of the group-major tile list
//               (tiles w, w+W, ...); all T tokens are staged once per CTA and
//               every tile computes all T columns, so an expert's weights are
//               read once however many tokens chose it; the epilogue keeps the
//               columns of the group's tokens:  act[g][t][col].
//   down        CTA c takes a contiguous range of the tile list, stages the
//               activation rows of the (at most 4) groups the range touches
//               and scatters row results to down_out[t*(k+1)+pos][row].
//   combine     per token, ascending ID, f32 multiply then add (no FMA), RTNE.
// No tile is split across warps and mma output columns do not interact, so an
// expert's output for a token is bit-identical whichever tokens, groups or
// ranks share the launch -- expert-parallel results equal single-GPU results
// byte for byte.
#include <string.h>

#include "moe_device.cuh"
#include "moe_internal.cuh"
#include "q4nx_core.cuh"
#include "rc_device.cuh"
#include "rc_internal.cuh"

namespace rc {

// ----------------------------------------------------------------- router --
struct RouteParams {
  const uint16_t *x;       // [T][ldx] bf16
  int ldx, tokens, hidden, n_experts, k, mode, renorm;
  float scaling;
  const uint16_t *wr;      // [E][hidden] bf16
  const float *bias;       // [E] (sigmoid mode)
  MoeScratch s;
  int shared_id;           // expert id of the shared expert, -1 if none
  MoeOwned own;
};

constexpr int kRouteThreads = 512;       // 16 warps: the slice order of the fused decode kernel
constexpr int kRouteSlice = 256;         // router columns per warp step: one 16-byte load per lane

// Phase 1 (CTA e = expert e, all T tokens): warp w takes the 256-column
// slices w, w+16, ...; a lane multiplies 8 columns, so every f64 chain is
// short; the warps' sums are added in warp order (the order of the fused
// decode kernel, so both round the same f64 sum).  The router row is fetched before waiting on the previous launch;
// the sums are exact f64 sums of exact bf16 x bf16 products, rounded once to
// f32.  Phase 2 (the last CTA to arrive, all threads): top-k by rank counting
// in the router order (larger first, NaN last, ties by lower index), the
// routing weights, the ascending-ID slot lists and the group table.
__global__ void __launch_bounds__(kRouteThreads) rc_moe_route_kernel(RouteParams p) {
  extern __shared__ __align__(16) uint8_t route_smem[];     // phase 2 arrays
  __shared__ double red[kRouteThreads / 32][kMoeMaxTokens];
  __shared__ uint32_t smask[kMoeMaxExperts + 1];
  __shared__ int sgidx[kMoeMaxExperts + 1];
  __shared__ int is_last;
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x, T = p.tokens;
  const int nslice = p.hidden / kRouteSlice;
  double acc[kMoeMaxTokens];
#pragma unroll
  for (int t = 0; t < kMoeMaxTokens; ++t) acc[t] = 0.0;
  bool waited = false;
  for (int sl = warp; sl < nslice; sl += kRouteThreads / 32) {
    const int col = sl * kRouteSlice + lane * 8;
    const uint4 wv = __ldg(reinterpret_cast<const uint4 *>(p.wr + (size_t)e * p.hidden + col));
    if (!waited) {
      pdl_wait_prior();                            // token rows come from the previous launch
      waited = true;
    }
    uint4 xv[kMoeMaxTokens];
#pragma unroll
    for (int t = 0; t < kMoeMaxTokens; ++t)
      if (t < T) xv[t] = *reinterpret_cast<const uint4 *>(p.x + (size_t)t * p.ldx + col);
    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
    double wd[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      wd[2 * j] = (double)bf16_to_f32(ww[j] & 0xFFFFu);
      wd[2 * j + 1] = (double)bf16_to_f32(ww[j] >> 16);
    }
#pragma unroll
    for (int t = 0; t < kMoeMaxTokens; ++t) {
      if (t < T) {
        const uint32_t xw[4] = {xv[t].x, xv[t].y, xv[t].z, xv[t].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[t] = fma((double)bf16_to_f32(xw[j] & 0xFFFFu), wd[2 * j], acc[t]);
          acc[t] = fma((double)bf16_to_f32(xw[j] >> 16), wd[2 * j + 1], acc[t]);
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kMoeMaxTokens; ++t) {
    if (t < T) {
      double a = acc[t];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
      if (lane == 0) red[warp][t] = a;
    }
  }
  __syncthreads();
  if (threadIdx.x < T) {
    double a = 0.0;
    for (int w = 0; w < kRouteThreads / 32; ++w) a += red[w][threadIdx.x];
    p.s.logits[(size_t)threadIdx.x * p.n_experts + e] = __double2float_rn(a);
  }
  // one release per CTA: the barrier orders the logit stores before thread
  // 0's (cumulative) fence and arrival
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int old = atomicAdd(p.s.counter, 1);
    is_last = old == (int)gridDim.x - 1;
    if (is_last) {
      atomicExch(p.s.counter, 0);
      __threadfence();
    }
  }
  __syncthreads();
  if (!is_last) return;

  // ---- phase 2 (last CTA)
  const int E = p.n_experts, k = p.k;
  float *val = reinterpret_cast<float *>(route_smem);      // [T][E]
  float *score = val + T * E;                               // [T][E]
  int *rank = reinterpret_cast<int *>(score + T * E);       // [T][E]
  int *sel = rank + T * E;                                  // [T][k] expert of each rank
  float *selw = reinterpret_cast<float *>(sel + T * k);     // [T][k] weight of each rank
  int32_t *slots = reinterpret_cast<int32_t *>(selw + T * k);   // [T][k+1] ascending slot lists
  for (int i = threadIdx.x; i < T * E; i += blockDim.x) {
    const float l = __ldcg(p.s.logits + i);
    float sc, v;
    if (p.mode == RC_ROUTER_SIGMOID_BIAS) {
      sc = __double2float_rn(1.0 / (1.0 + exp(-(double)l)));
      v = sc + p.bias[i % E];
    } else {
      sc = l + p.bias[i % E];          // softmax of the biased logits (bias zero unless set)
      v = sc;
    }
    score[i] = sc;
    val[i] = v;
  }
  __syncthreads();
  // rank of (t, e): experts ahead of it; P adjacent lanes split the count
  int P = 1;
  while (P < 32 && T * E * P * 2 <= kRouteThreads) P *= 2;
  const int items = T * E * P;
  for (int i0 = 0; i0 < items; i0 += blockDim.x) {
    const int i = i0 + threadIdx.x;
    int ahead = 0;
    int te = -1;
    if (i < items) {
      te = i / P;
      const int part = i - te * P;
      const int t = te / E, e0 = te - t * E;
      const float v = val[te];
      const float *row = val + t * E;
      const int per = (E + P - 1) / P;
      const int lo = part * per, hi = lo + per < E ? lo + per : E;
      for (int e2 = lo; e2 < hi; ++e2) ahead += route_before(row[e2], e2, v, e0) ? 1 : 0;
    }
    for (int o = 1; o < P; o <<= 1) ahead += __shfl_down_sync(0xffffffffu, ahead, o, P);
    if (i < items && (i % P) == 0) {
      rank[te] = ahead;
      const int t = te / E;
      if (ahead < k) sel[t * k + ahead] = te - t * E;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < T * k; i += blockDim.x) {
    const int t = i / k, r = i - t * k;
    const float *sc = score + t * E;
    const int *st = sel + t * k;
    float w;
    if (p.mode == RC_ROUTER_SIGMOID_BIAS) {
      float sum = 0.f;
      for (int r2 = 0; r2 < k; ++r2) sum += sc[st[r2]];
      w = sc[st[r]];
      if (p.renorm) w = w / (sum + 1e-20f);
      w = w * p.scaling;
    } else {
      // softmax over all experts then renormalised over the top-k equals the
      // softmax of the selected logits (the full denominator cancels)
      const float mx = sc[st[0]];
      float sum = 0.f;
      for (int r2 = 0; r2 < k; ++r2) sum += expf(sc[st[r2]] - mx);
      w = expf(sc[st[r]] - mx) / sum;
    }
    selw[i] = w;
    p.s.ids[i] = st[r];
    p.s.weights[i] = w;
  }
  __syncthreads();
  // ascending-ID slot lists: one warp per token, ballots over the experts
  for (int t = warp; t < T; t += kRouteThreads / 32) {
    int base = 0;
    for (int c = 0; c < E; c += 32) {
      const int e1 = c + lane;
      const int rk = e1 < E ? rank[t * E + e1] : k;
      const uint32_t b = __ballot_sync(0xffffffffu, rk < k);
      if (rk < k) {
        const int pos = base + __popc(b & ((1u << lane) - 1u));
        slots[t * (k + 1) + pos] = e1;
        p.s.slot_expert[t * (k + 1) + pos] = e1;
        p.s.slot_w[t * k + pos] = selw[t * k + rk];
      }
      base += __popc(b);
    }
    if (lane == 0) {
      slots[t * (k + 1) + k] = p.shared_id;
      p.s.slot_expert[t * (k + 1) + k] = p.shared_id;
    }
  }
  __syncthreads();
  if (warp == 0) build_groups(slots, T, k, E, p.own, p.s, smask, sgidx, lane);
}

// Slot lists from caller-supplied top ids / weights [T][k] (the
// Backend.moe_experts boundary): per token sort ascending by ID, append the
// shared expert; then the group table.  One warp.
__global__ void rc_moe_slots_kernel(const int32_t *ids, const float *w, int T, int k, int n_experts, int shared_id,
                                 MoeOwned own, MoeScratch s) {
  __shared__ uint32_t smask[kMoeMaxExperts + 1];
  __shared__ int sgidx[kMoeMaxExperts + 1];
  pdl_launch_dependents();
  pdl_wait_prior();
  const int lane = threadIdx.x & 31;
  if (threadIdx.x >= 32) return;
  for (int t = lane; t < T; t += 32) {
    const int32_t *id = ids + (size_t)t * k;
    const float *wt = w + (size_t)t * k;
    int order[kMoeMaxK];
    for (int r = 0; r < k; ++r) order[r] = r;
    for (int a = 1; a < k; ++a) {
      const int v = order[a];
      int b = a - 1;
      while (b >= 0 && id[order[b]] > id[v]) {
        order[b + 1] = order[b];
        --b;
      }
      order[b + 1] = v;
    }
    for (int r = 0; r < k; ++r) {
      s.slot_expert[(size_t)t * (k + 1) + r] = id[order[r]];
      s.slot_w[(size_t)t * k + r] = wt[order[r]];
    }
    s.slot_expert[(size_t)t * (k + 1) + k] = shared_id;
  }
  __threadfence_block();
  __syncwarp();
  build_groups(s.slot_expert, T, k, n_experts, own, s, smask, sgidx, lane);
}

// ------------------------------------------------------ grouped expert GEMV --
enum MoeEpi : int { kMoeEpiGlu = 0, kMoeEpiDown = 1 };

struct MoeGemvParams {
  const uint8_t *const *expert_tiles;  // [E+1]: t16 tiles of each expert matrix (null: not loaded)
  const int *n_groups;
  const int32_t *group_expert;
  const uint32_t *group_mask;
  const int32_t *group_dst;
  int skip_last_group;                 // gate/up: the shared group's activations come from elsewhere
  int group_tiles;                     // row tiles per expert matrix
  int kb;                              // K / 256
  int stages;
  int round_tiles;                     // tiles per reduction round of a CTA
  int T;                               // tokens of the call
  // activations (fields read by the shared staging code)
  const void *x;
  int x_dtype, ldx, tokens, slots, x_vec;
  // output
  uint16_t *y;
  int ldy;
  int act;
  float gate_beta, value_beta;
  int *err;
  // gate/up launch of an expert-parallel call: zero the slot rows another rank
  // computes (zero_rows [T*(k+1)][hidden], null otherwise)
  uint16_t *zero_rows;
  const int32_t *slot_expert;
  int k, hidden;
  MoeOwned own;
};

// EPI == kMoeEpiGlu: x = the T token rows; tile rows are interleaved
//   (gate g, up g) pairs; y = act rows, act[g][t][8*tile + g'] for the tokens of
//   group g (8*NTB rows per group).
// EPI == kMoeEpiDown: x = act; y = down_out rows, [t*(k+1)+pos][hidden].
//
// Partition: CTA c owns the contiguous tiles [c0, c1) of the group-major tile
// list; its units (tile, k-block) are dealt to the warps round-robin (unit u
// to warp u % 16) in rounds of p.round_tiles whole tiles.  Each unit's
// contribution goes to its own shared-memory partial; after a round's barrier
// one warp per tile sums the tile's partials in k-block order and runs the
// epilogue.  A tile's result therefore depends on the tile alone, never on
// the partition, the grid or the other groups of the launch.
template <int EPI, int NTB>
__global__ void __launch_bounds__(kMoeWarps * 32, 1) rc_moe_gemv_kernel(MoeGemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb = p.kb, k = kb * kUnitK, S = p.stages, R = p.round_tiles;
  uint8_t *ring = smem + warp * S * kUnitBytes;
  const uint32_t ring_s = smem_addr(ring);
  constexpr int kStageBlocks = EPI == kMoeEpiGlu ? NTB : NTB * kMoeMaxGroupsPerCta;
  uint8_t *sp = smem + kMoeWarps * S * kUnitBytes;
  uint32_t *xs = reinterpret_cast<uint32_t *>(sp);
  sp += xfrag_bytes(kStageBlocks, k);
  void *xa = sp;
  sp += xaux_bytes(kStageBlocks, k);
  float4 *part = reinterpret_cast<float4 *>(sp);           // [R*kb][NTB][32 lanes]
  sp += (size_t)R * kb * NTB * 32 * sizeof(float4);
  const uint32_t bar0 = smem_addr(sp) + warp * S * 8;

  pdl_launch_dependents();
  // The group table is written by the previous launch: wait before reading it.
  pdl_wait_prior();
  if (EPI == kMoeEpiGlu && p.zero_rows) {
    const int rows = p.T * (p.k + 1);
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {
      const int t = r / (p.k + 1), pos = r - t * (p.k + 1);
      const int e = p.slot_expert[r];
      const bool mine = pos < p.k ? (e >= p.own.lo && e < p.own.hi) : (e >= 0 && ((p.own.shared_mask >> t) & 1u));
      if (mine) continue;
      uint4 *dst = reinterpret_cast<uint4 *>(p.zero_rows + (size_t)r * p.hidden);
      for (int i = threadIdx.x; i < p.hidden / 8; i += blockDim.x) dst[i] = make_uint4(0, 0, 0, 0);
    }
  }
  const int ng = *p.n_groups - (p.skip_last_group ? 1 : 0);
  const int total = ng * p.group_tiles;
  const int per = (total + (int)gridDim.x - 1) / (int)gridDim.x;
  const int c0 = blockIdx.x * per;
  const int c1 = c0 + per < total ? c0 + per : total;
  const int n_tiles = c1 > c0 ? c1 - c0 : 0;
  int g_lo = 0;
  MoeGemvParams q = p;
  if (EPI == kMoeEpiDown) {
    // stage the activation rows of the groups the range touches (8*NTB rows each)
    g_lo = c0 / p.group_tiles;
    const int g_hi = n_tiles ? (c1 - 1) / p.group_tiles : g_lo - 1;
    q.x = static_cast<const uint16_t *>(p.x) + (size_t)g_lo * 8 * NTB * p.ldx;
    q.tokens = q.slots = (g_hi - g_lo + 1) * 8 * NTB;
  }
  // this warp's units: its chunk of every round (k-block-major order)
  RoundCursor cur;
  cur.init(n_tiles, R, kb, kMoeWarps, warp);
  RoundCursor iss = cur;                                   // the next unit to fetch (lane 0)
  auto unit_src = [&](const RoundCursor &c) -> const uint8_t * {
    const int tg = c0 + c.tile();
    const int grp = tg / p.group_tiles, tile = tg - grp * p.group_tiles;
    const uint8_t *b = p.expert_tiles[p.group_expert[grp]];
    return b ? b + ((size_t)tile * kb + c.kbi) * kUnitBytes : nullptr;
  };
  const uint64_t pol = policy_evict_first();
  int issued = 0;                                          // copies issued so far (lane 0)
  auto issue = [&](int sl) {
    const uint8_t *src = unit_src(iss);
    if (src) {
      mbar_arrive_expect_tx(bar0 + 8 * sl, kUnitBytes);
      bulk_copy_g2s(ring_s + sl * kUnitBytes, src, kUnitBytes, bar0 + 8 * sl, pol);
    } else {
      mbar_arrive_expect_tx(bar0 + 8 * sl, 0);   // nothing to fetch: complete the phase at once
    }
    iss.next();
    ++issued;
  };
  if (lane == 0 && cur.valid()) {
    for (int sl = 0; sl < S; ++sl) mbar_init(bar0 + 8 * sl, 1);
    mbar_fence_init();
    for (int sl = 0; sl < S && iss.valid(); ++sl) issue(sl);
  }
  build_activations<true>(q, kStageBlocks, xs, xa, threadIdx.x, blockDim.x);
  __syncthreads();

  const int n_rounds = round_count(n_tiles, R);
  int j = 0, slot_ring = 0;                                // units consumed, ring slot of the next
  uint32_t phase = 0;
  bool failed = false;
  int j_fail = 0;
  const int g = lane >> 2, qd = lane & 3;
  XFrag<NTB> xr;
  int xr_key = -1;                                         // (block, k-block) held in xr
  for (int r = 0; r < n_rounds; ++r) {
    for (; cur.valid() && cur.round == r; cur.next(), ++j) {
      const int kbi = cur.kbi;
      const int tg = c0 + cur.tile();
      const int grp = tg / p.group_tiles;
      if (!failed && !mbar_wait_bounded_warp(bar0 + 8 * slot_ring, phase)) {
        if (lane == 0) atomicCAS(p.err, 0, kErrWaitTimeout);
        failed = true;
        j_fail = j;
      }
      if (!failed && p.expert_tiles[p.group_expert[grp]] != nullptr) {
        const int blk = EPI == kMoeEpiGlu ? 0 : (grp - g_lo) * NTB;
        if (blk * kb + kbi != xr_key) {
          load_xfrag<NTB, true>(xr, xs, xa, kStageBlocks, blk, kb, kbi, lane);
          xr_key = blk * kb + kbi;
        }
        float4 Q[NTB];
        unit_result<NTB>(ring + slot_ring * kUnitBytes, xr, lane, Q);
        float4 *dst = part + (size_t)cur.slot() * NTB * 32 + lane;
#pragma unroll
        for (int tb = 0; tb < NTB; ++tb) dst[tb * 32] = Q[tb];
      }
      __syncwarp();
      if (!failed && lane == 0 && iss.valid()) issue(slot_ring);
      if (++slot_ring == S) slot_ring = 0, phase ^= 1u;
    }
    __syncthreads();
    // one warp per tile of this round: ordered sum of its units, epilogue
    const int t_lo = r * R, t_hi = t_lo + R < n_tiles ? t_lo + R : n_tiles;
    for (int ti = t_lo + warp; ti < t_hi; ti += kMoeWarps) {
      const int tg = c0 + ti;
      const int grp = tg / p.group_tiles, tile = tg - grp * p.group_tiles;
      const bool live = p.expert_tiles[p.group_expert[grp]] != nullptr;
      Acc<NTB> acc;
      acc_zero(acc);
      const float4 *src = part + (size_t)(ti - t_lo) * kb * NTB * 32 + lane;
      for (int kbi = 0; kbi < kb; ++kbi) {
        float4 v[NTB];
#pragma unroll
        for (int tb = 0; tb < NTB; ++tb) v[tb] = src[(kbi * NTB + tb) * 32];
        acc_add(acc, v);
      }
      const uint32_t mask = p.group_mask[grp];
#pragma unroll
      for (int tb = 0; tb < NTB; ++tb) {
#pragma unroll
        for (int e2 = 0; e2 < 2; ++e2) {
          const int t = tb * 8 + 2 * qd + e2;
          if (t >= p.T || !((mask >> t) & 1u)) continue;
          if (EPI == kMoeEpiGlu) {
            float v = 0.f;
            if (live) {
              const float gate = bf16_round(acc.v[tb][e2]);
              const float up = bf16_round(acc.v[tb][2 + e2]);
              v = p.act == RC_ACT_SITU ? act_situ(gate, up, p.gate_beta, p.value_beta) : act_swiglu(gate, up);
            }
            p.y[((size_t)grp * 8 * NTB + t) * p.ldy + tile * 8 + g] = f32_to_bf16_rne(v);
          } else {
            uint16_t *y = p.y + (size_t)p.group_dst[grp * kMoeMaxTokens + t] * p.ldy + tile * kUnitRows + g;
            y[0] = live ? f32_to_bf16_rne(acc.v[tb][e2]) : (uint16_t)0;
            y[8] = live ? f32_to_bf16_rne(acc.v[tb][2 + e2]) : (uint16_t)0;
          }
        }
      }
    }
    __syncthreads();
  }
  // after a timeout, wait (bounded) for the copies still in flight before the
  // CTA's shared memory is released
  if (failed && lane == 0) {
    for (int jj = j_fail; jj < issued; ++jj) mbar_wait_bounded(bar0 + 8 * (jj % S), (uint32_t)(jj / S) & 1u);
  }
}

// Shared-expert activations from caller-supplied gate|up rows [T][2*inter]
// (the grouped boundary): act[g_shared][t][c] = RTNE(act(gu[t][c], gu[t][inter + c]))
// for c < inter; the pad columns of act stay zero.
__global__ void rc_moe_shared_act_kernel(const uint16_t *gu, int T, int inter, int inter_pad, const int *n_groups,
                                      int rows_per_group, int act, float gb, float vb, uint16_t *act_out) {
  pdl_launch_dependents();
  pdl_wait_prior();
  const int t = blockIdx.y;
  uint16_t *dst = act_out + ((size_t)(*n_groups - 1) * rows_per_group + t) * inter_pad;
  const uint16_t *src = gu + (size_t)t * 2 * inter;
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < inter; c += gridDim.x * blockDim.x) {
    const float gate = bf16_to_f32(src[c]), up = bf16_to_f32(src[inter + c]);
    dst[c] = f32_to_bf16_rne(act == RC_ACT_SITU ? act_situ(gate, up, gb, vb) : act_swiglu(gate, up));
  }
}

// ---------------------------------------------------------------- combine --
// Per token t: routed = RTNE(sum_{slots in ascending ID} f32(down[t][s]) * w[t][s]);
// out = routed, or RTNE(f32(routed) + f32(down[t][k])) with the shared expert.
// routed_out / shared_out (optional) receive the routed sum and the shared
// expert's row (the grouped boundary returns them apart).  A thread owns 8
// columns and fetches all k+1 rows before summing (one memory round trip).
constexpr int kCombineThreads = 128;

__global__ void __launch_bounds__(kCombineThreads) rc_moe_combine_kernel(const uint16_t *down, const float *slot_w,
                                                                        int k, int with_shared, int hidden,
                                                                        uint16_t *out, uint16_t *routed_out,
                                                                        uint16_t *shared_out) {
  pdl_launch_dependents();
  pdl_wait_prior();
  const int t = blockIdx.y;
  const int v = blockIdx.x * blockDim.x + threadIdx.x;   // 8-column vector
  if (v * 8 >= hidden) return;
  const uint16_t *rows = down + (size_t)t * (k + 1) * hidden + (size_t)v * 8;
  const bool need_shared = with_shared || shared_out;
  uint4 r[kMoeMaxK];
  float w[kMoeMaxK];
#pragma unroll
  for (int s = 0; s < kMoeMaxK; ++s) {
    r[s] = make_uint4(0, 0, 0, 0);
    if (s < k) r[s] = __ldcg(reinterpret_cast<const uint4 *>(rows + (size_t)s * hidden));
  }
  // the shared row by its own load: selecting r[k] would index the array at
  // run time and move it to local memory
  const uint4 sh = need_shared ? __ldcg(reinterpret_cast<const uint4 *>(rows + (size_t)k * hidden))
                               : make_uint4(0, 0, 0, 0);
#pragma unroll
  for (int s = 0; s < kMoeMaxK; ++s) w[s] = s < k ? __ldcg(slot_w + (size_t)t * k + s) : 0.f;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  // product rounded, then sum rounded -- as the reference's f32 numpy update
  // (no fused multiply-add contraction)
#pragma unroll
  for (int s = 0; s < kMoeMaxK; ++s) {
    if (s < k) {
      const uint32_t q[4] = {r[s].x, r[s].y, r[s].z, r[s].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] = __fadd_rn(acc[2 * j], __fmul_rn(bf16_to_f32(q[j] & 0xFFFFu), w[s]));
        acc[2 * j + 1] = __fadd_rn(acc[2 * j + 1], __fmul_rn(bf16_to_f32(q[j] >> 16), w[s]));
      }
    }
  }
  const uint32_t shw[4] = {sh.x, sh.y, sh.z, sh.w};
  uint32_t ro[4], oo[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t lo = f32_to_bf16_rne(acc[2 * j]), hi = f32_to_bf16_rne(acc[2 * j + 1]);
    ro[j] = lo | (hi << 16);
    if (with_shared) {
      const uint32_t olo = f32_to_bf16_rne(bf16_to_f32(lo) + bf16_to_f32(shw[j] & 0xFFFFu));
      const uint32_t ohi = f32_to_bf16_rne(bf16_to_f32(hi) + bf16_to_f32(shw[j] >> 16));
      oo[j] = olo | (ohi << 16);
    } else {
      oo[j] = ro[j];
    }
  }
  const size_t o = (size_t)t * hidden + (size_t)v * 8;
  if (routed_out) *reinterpret_cast<uint4 *>(routed_out + o) = make_uint4(ro[0], ro[1], ro[2], ro[3]);
  if (shared_out) *reinterpret_cast<uint4 *>(shared_out + o) = sh;
  if (out) *reinterpret_cast<uint4 *>(out + o) = make_uint4(oo[0], oo[1], oo[2], oo[3]);
}

}  // namespace rc

using namespace rc;


namespace rc {

static size_t moe_smem_bytes(int stage_blocks, int k, int stages, int partial_bytes) {
  return (size_t)kMoeWarps * stages * (kUnitBytes + 8) + xfrag_bytes(stage_blocks, k) + xaux_bytes(stage_blocks, k) +
         partial_bytes;
}

template <int EPI, int NTB>
static cudaError_t launch_moe_gemv_t(const rc_ctx *ctx, MoeGemvParams p, int max_groups, cudaStream_t s) {
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(rc_moe_gemv_kernel<EPI, NTB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kGemvSmemLimit);
    if (e != cudaSuccess) return e;
    if (dev < 64) configured[dev] = true;
  }
  const int max_tiles = max_groups * p.group_tiles;
  int grid = ctx->sm_count;
  if (EPI == kMoeEpiDown) {
    // a CTA's contiguous range of `per` tiles touches at most
    // kMoeMaxGroupsPerCta groups when per - 1 <= (kMoeMaxGroupsPerCta - 1) * group_tiles
    while ((max_tiles + grid - 1) / grid - 1 > (kMoeMaxGroupsPerCta - 1) * p.group_tiles) grid *= 2;
  }
  const int per = (max_tiles + grid - 1) / grid;
  const int stage_blocks = EPI == kMoeEpiGlu ? NTB : NTB * kMoeMaxGroupsPerCta;
  const int k = p.kb * kUnitK;
  const int unit_partial = NTB * 32 * 16;                  // bytes per unit partial
  int R = kMoePartialBytes / (p.kb * unit_partial);
  if (R < 1) R = 1;
  if (R > per) R = per;
  const int units_per_warp = (per * p.kb + kMoeWarps - 1) / kMoeWarps;
  int S = units_per_warp < 2 ? 2 : (units_per_warp > kMoeMaxStages ? kMoeMaxStages : units_per_warp);
  while (S > 2 && moe_smem_bytes(stage_blocks, k, S, R * p.kb * unit_partial) > (size_t)kGemvSmemLimit) --S;
  while (R > 1 && moe_smem_bytes(stage_blocks, k, S, R * p.kb * unit_partial) > (size_t)kGemvSmemLimit) --R;
  const size_t smem = moe_smem_bytes(stage_blocks, k, S, R * p.kb * unit_partial);
  if (smem > (size_t)kGemvSmemLimit) return cudaErrorInvalidConfiguration;
  p.stages = S;
  p.round_tiles = R;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kMoeWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, rc_moe_gemv_kernel<EPI, NTB>, p);
}

template <int EPI>
static cudaError_t launch_moe_gemv(const rc_ctx *ctx, const MoeGemvParams &p, int max_groups, cudaStream_t s) {
  return p.T <= 8 ? launch_moe_gemv_t<EPI, 1>(ctx, p, max_groups, s)
                  : launch_moe_gemv_t<EPI, 2>(ctx, p, max_groups, s);
}

static cudaLaunchConfig_t small_cfg(dim3 grid, dim3 block, cudaStream_t s, cudaLaunchAttribute *attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// Upper bound of the group count, for launch sizing only (the kernels read the
// real count from the device).
static int max_groups(int T, int k, const MoeOwned &own) {
  const int owned = own.hi - own.lo;
  const int routed = T * k < owned ? T * k : owned;
  return routed + (own.shared_mask ? 1 : 0);
}

// gate/up with the GLU epilogue (the shared group's activations come from
// shared_gu instead when it is given), then the down GEMV into down_out
// [T][k+1][hidden].
static int moe_run_experts(rc_moe *m, const uint16_t *x, int T, int k, const MoeOwned &own, int act, float gb,
                           float vb, const uint16_t *shared_gu, uint16_t *down_out, bool zero_foreign,
                           cudaStream_t s) {
  const int ntb = T <= 8 ? 1 : 2;
  const int mg = max_groups(T, k, own);
  const bool glu_launch = mg - (shared_gu && own.shared_mask ? 1 : 0) > 0;
  if (zero_foreign && !glu_launch)
    RC_CUDA_TRY(cudaMemsetAsync(down_out, 0, (size_t)T * (k + 1) * m->hidden * 2, s));
  if (mg == 0) return RC_OK;
  MoeGemvParams g{};
  g.expert_tiles = m->gu_tiles;
  g.n_groups = m->s.n_groups;
  g.group_expert = m->s.group_expert;
  g.group_mask = m->s.group_mask;
  g.group_dst = m->s.group_dst;
  g.skip_last_group = shared_gu && own.shared_mask ? 1 : 0;
  g.group_tiles = m->inter / 8;              // interleaved gate/up: 8 intermediate columns per tile
  g.kb = m->hidden / kUnitK;
  g.T = T;
  g.x = x;
  g.x_dtype = RC_DTYPE_BF16;
  g.ldx = m->hidden;
  g.tokens = T;
  g.slots = T;
  g.x_vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (m->hidden * 2) % 16 == 0;
  g.y = m->act;
  g.ldy = m->inter_pad;
  g.act = act;
  g.gate_beta = gb;
  g.value_beta = vb;
  g.err = m->ctx->err;
  g.zero_rows = zero_foreign ? down_out : nullptr;
  g.slot_expert = m->s.slot_expert;
  g.k = k;
  g.hidden = m->hidden;
  g.own = own;
  cudaError_t e = cudaSuccess;
  if (mg - g.skip_last_group > 0) e = launch_moe_gemv<kMoeEpiGlu>(m->ctx, g, mg - g.skip_last_group, s);
  if (e != cudaSuccess) {
    set_error("moe gate/up launch: %s", cudaGetErrorString(e));
    return RC_ERR_CUDA;
  }
  if (g.skip_last_group) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = small_cfg(dim3((m->inter + 255) / 256, T), dim3(256), s, attr);
    e = cudaLaunchKernelEx(&cfg, rc_moe_shared_act_kernel, shared_gu, T, m->inter, m->inter_pad,
                           (const int *)m->s.n_groups, 8 * ntb, act, gb, vb, m->act);
    if (e != cudaSuccess) {
      set_error("moe shared activation launch: %s", cudaGetErrorString(e));
      return RC_ERR_CUDA;
    }
  }
  if (m->down_fmt == kFormatBfp16) {
    BfMoeDown b{};
    b.w = m->dn_tiles;
    b.n_groups = m->s.n_groups;
    b.group_expert = m->s.group_expert;
    b.group_mask = m->s.group_mask;
    b.group_dst = m->s.group_dst;
    b.dst_stride = kMoeMaxTokens;
    b.x = m->act;
    b.ldx = m->inter_pad;
    b.rows_per_group = 8 * ntb;
    b.T = T;
    b.hidden = m->hidden;
    b.inter_pad = m->inter_pad;
    b.y = down_out;
    b.ldy = m->hidden;
    b.max_groups = mg;
    b.err = m->ctx->err;
    return bfp16_moe_down(m->ctx, b, s);
  }
  MoeGemvParams d = g;
  d.expert_tiles = m->dn_tiles;
  d.skip_last_group = 0;
  d.zero_rows = nullptr;
  d.group_tiles = m->hidden / kUnitRows;
  d.kb = m->inter_pad / kUnitK;
  d.x = m->act;
  d.ldx = m->inter_pad;
  d.x_vec = 1;
  d.y = down_out;
  d.ldy = m->hidden;
  e = launch_moe_gemv<kMoeEpiDown>(m->ctx, d, mg, s);
  if (e != cudaSuccess) {
    set_error("moe down launch: %s", cudaGetErrorString(e));
    return RC_ERR_CUDA;
  }
  return RC_OK;
}

static int moe_combine(rc_moe *m, const uint16_t *down, const float *slot_w, int T, int k, int with_shared,
                       uint16_t *out, uint16_t *routed_out, uint16_t *shared_out, cudaStream_t s) {
  auto mis = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15) != 0; };
  RC_CHECK_ARG(!mis(down) && !mis(out) && !mis(routed_out) && !mis(shared_out),
               "MoE slot and output rows must be 16-byte aligned");
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = small_cfg(dim3((m->hidden / 8 + kCombineThreads - 1) / kCombineThreads, T),
                                     dim3(kCombineThreads), s, attr);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, rc_moe_combine_kernel, down, slot_w, k, with_shared, m->hidden, out,
                                           routed_out, shared_out);
  if (e != cudaSuccess) {
    set_error("moe combine launch: %s", cudaGetErrorString(e));
    return RC_ERR_CUDA;
  }
  return RC_OK;
}

static int moe_route(rc_moe *m, const uint16_t *x, int T, int k, int mode, int renorm, float scaling,
                     const MoeOwned &own, cudaStream_t s, const MoeScratch *scratch = nullptr) {
  RC_CHECK_ARG((reinterpret_cast<uintptr_t>(x) & 15) == 0, "token rows must be 16-byte aligned");
  RouteParams r{};
  r.x = x;
  r.ldx = m->hidden;
  r.tokens = T;
  r.hidden = m->hidden;
  r.n_experts = m->n_experts;
  r.k = k;
  r.mode = mode;
  r.renorm = renorm;
  r.scaling = scaling;
  r.wr = m->router_w;
  r.bias = m->router_bias;
  r.s = scratch ? *scratch : m->s;
  r.shared_id = m->has_shared ? m->n_experts : -1;
  r.own = own;
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess && (dev >= 64 || !configured[dev])) {
    constexpr int kPhase2Max = kMoeMaxTokens * kMoeMaxExperts * 12 + kMoeMaxTokens * kMoeMaxK * 8 +
                               kMoeMaxTokens * (kMoeMaxK + 1) * 4;
    e = cudaFuncSetAttribute(rc_moe_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPhase2Max);
    if (e == cudaSuccess && dev < 64) configured[dev] = true;
  }
  if (e != cudaSuccess) {
    set_error("moe router setup: %s", cudaGetErrorString(e));
    return RC_ERR_CUDA;
  }
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = small_cfg(dim3(m->n_experts), dim3(kRouteThreads), s, attr);
  const size_t need = (size_t)T * m->n_experts * 12 + (size_t)T * k * 8 + (size_t)T * (k + 1) * 4;
  cfg.dynamicSmemBytes = (need + 15) / 16 * 16;
  e = cudaLaunchKernelEx(&cfg, rc_moe_route_kernel, r);
  if (e != cudaSuccess) {
    set_error("moe router launch: %s", cudaGetErrorString(e));
    return RC_ERR_CUDA;
  }
  return RC_OK;
}

static int moe_slots(rc_moe *m, const int32_t *ids, const float *w, int T, int k, const MoeOwned &own,
                     cudaStream_t s) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = small_cfg(dim3(1), dim3(32), s, attr);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, rc_moe_slots_kernel, ids, w, T, k, m->n_experts,
                                           m->has_shared ? m->n_experts : -1, own, m->s);
  if (e != cudaSuccess) {
    set_error("moe slot list launch: %s", cudaGetErrorString(e));
    return RC_ERR_CUDA;
  }
  return RC_OK;
}

static uint32_t token_mask(int t0, int tn) {
  uint32_t m = 0;
  for (int t = t0; t < t0 + tn; ++t) m |= 1u << t;
  return m;
}

static int check_loaded(const rc_moe *m, const MoeOwned &own) {
  for (int e = own.lo; e < own.hi; ++e)
    RC_CHECK_ARG(m->gate_up[e] != nullptr, "expert %d is in the computed range but not loaded", e);
  RC_CHECK_ARG(!own.shared_mask || m->gate_up[m->n_experts] != nullptr, "the shared expert is not loaded");
  return RC_OK;
}

static MoeOwned all_owned(const rc_moe *m, int T, int with_shared) {
  MoeOwned o;
  o.lo = 0;
  o.hi = m->n_experts;
  o.shared_mask = with_shared ? token_mask(0, T) : 0u;
  return o;
}

}  // namespace rc

extern "C" {

int rc_moe_create(rc_ctx *ctx, int hidden, int inter, int n_experts, int has_shared, rc_moe **out) {
  RC_CHECK_ARG(ctx && out, "rc_moe_create: NULL argument");
  *out = nullptr;
  RC_CHECK_ARG(hidden > 0 && hidden % 256 == 0, "hidden (%d) must be a multiple of 256", hidden);
  RC_CHECK_ARG(inter > 0 && inter % 64 == 0, "intermediate size (%d) must be a multiple of 64", inter);
  RC_CHECK_ARG(n_experts > 0 && n_experts <= kMoeMaxExperts, "n_experts (%d) must be in 1..%d", n_experts,
               kMoeMaxExperts);
  RC_CUDA_TRY(cudaSetDevice(ctx->device));
  rc_moe *m = new rc_moe();
  m->ctx = ctx;
  m->hidden = hidden;
  m->inter = inter;
  m->inter_pad = (inter + 255) / 256 * 256;
  m->n_experts = n_experts;
  m->has_shared = has_shared ? 1 : 0;
  m->fused = 1;
  m->prefill_kernel = RC_PREFILL_TCGEN05;
  m->down_fmt = kFormatQ4nx;
  const int ne = n_experts + 1;
  m->gate_up = new rc_weight *[ne]();
  m->down = new rc_weight *[ne]();
  const int T = kMoeMaxTokens, K = kMoeMaxK;
  cudaError_t e = cudaMalloc(&m->gu_tiles, ne * sizeof(void *));
  if (e == cudaSuccess) e = cudaMalloc(&m->dn_tiles, ne * sizeof(void *));
  if (e == cudaSuccess) e = cudaMemset(m->gu_tiles, 0, ne * sizeof(void *));
  if (e == cudaSuccess) e = cudaMemset(m->dn_tiles, 0, ne * sizeof(void *));
  if (e == cudaSuccess) e = cudaMalloc(&m->router_w, (size_t)n_experts * hidden * 2);
  if (e == cudaSuccess) e = cudaMalloc(&m->router_bias, (size_t)n_experts * 4);
  if (e == cudaSuccess) e = cudaMemset(m->router_bias, 0, (size_t)n_experts * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->s.logits, (size_t)T * n_experts * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->s.counter, (T + 1) * 4);
  if (e == cudaSuccess) e = cudaMemset(m->s.counter, 0, (T + 1) * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->s.ids, T * K * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->s.weights, T * K * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->s.slot_expert, T * (K + 1) * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->s.slot_w, T * K * 4);
  m->s.err = ctx->err;
  if (e == cudaSuccess) e = cudaMalloc(&m->s.n_groups, 4);
  if (e == cudaSuccess) e = cudaMemset(m->s.n_groups, 0, 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->s.group_expert, ne * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->s.group_mask, ne * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->s.group_dst, (size_t)ne * kMoeMaxTokens * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->act, (size_t)ne * T * m->inter_pad * 2);
  if (e == cudaSuccess) e = cudaMemset(m->act, 0, (size_t)ne * T * m->inter_pad * 2);
  if (e == cudaSuccess) e = cudaMalloc(&m->down_out, (size_t)T * (K + 1) * hidden * 2);
  if (e != cudaSuccess) {
    set_error("rc_moe_create: %s", cudaGetErrorString(e));
    rc_moe_destroy(m);
    return RC_ERR_CUDA;
  }
  *out = m;
  return RC_OK;
}

// Unmaps the peers' exchange buffers and frees this rank's.
static void ep_release(rc_moe *m) {
  MoeEp *ep = m->ep;
  if (!ep) return;
  for (int r = 0; r < ep->world; ++r)
    if (r != ep->rank && ep->mapped[r]) cudaIpcCloseMemHandle(ep->peer[r]);
  cudaFree(ep->base);
  cudaFree(ep->peer_dev);
  delete ep;
  m->ep = nullptr;
}

int rc_moe_destroy(rc_moe *m) {
  if (!m) return RC_OK;
  cudaSetDevice(m->ctx->device);
  cudaDeviceSynchronize();
  pf_free(m);
  for (int e = 0; e <= m->n_experts; ++e) {
    if (m->gate_up && m->gate_up[e]) rc_weight_free(m->gate_up[e]);
    if (m->down && m->down[e]) rc_weight_free(m->down[e]);
  }
  delete[] m->gate_up;
  delete[] m->down;
  cudaFree(m->gu_tiles);
  cudaFree(m->dn_tiles);
  cudaFree(m->router_w);
  cudaFree(m->router_bias);
  cudaFree(m->s.logits);
  cudaFree(m->s.counter);
  cudaFree(m->s.ids);
  cudaFree(m->s.weights);
  cudaFree(m->s.slot_expert);
  cudaFree(m->s.slot_w);
  cudaFree(m->s.n_groups);
  cudaFree(m->s.group_expert);
  cudaFree(m->s.group_mask);
  cudaFree(m->s.group_dst);
  cudaFree(m->act);
  cudaFree(m->down_out);
  cudaFree(m->fz_bar);
  cudaFree(m->dc_cols);
  ep_release(m);
  delete m;
  return RC_OK;
}

int rc_moe_set_expert(rc_moe *m, int expert, const uint8_t *gate_up, size_t gate_up_bytes, const uint8_t *down,
                      size_t down_bytes, unsigned flags) {
  RC_CHECK_ARG(m && gate_up && down, "rc_moe_set_expert: NULL argument");
  RC_CHECK_ARG(expert >= 0 && expert <= m->n_experts, "expert id %d out of range 0..%d", expert, m->n_experts);
  RC_CHECK_ARG(expert < m->n_experts || m->has_shared, "this MoE layer has no shared expert");
  RC_CHECK_ARG((flags & ~(unsigned)(RC_UPLOAD_SRC_DEVICE | RC_UPLOAD_DOWN_BFP16)) == 0,
               "rc_moe_set_expert: unknown flags 0x%x", flags);
  const int fmt = (flags & RC_UPLOAD_DOWN_BFP16) ? kFormatBfp16 : kFormatQ4nx;
  for (int e = 0; e <= m->n_experts; ++e)
    RC_CHECK_ARG(e == expert || !m->down[e] || m->down[e]->format == fmt,
                 "rc_moe_set_expert: expert %d's down matrix is %s but expert %d's is %s (one format per layer)",
                 expert, fmt == kFormatBfp16 ? "bfp16ebs8" : "q4nx", e,
                 fmt == kFormatBfp16 ? "q4nx" : "bfp16ebs8");
  const unsigned src = flags & RC_UPLOAD_SRC_DEVICE;
  rc_weight *gu = nullptr, *dn = nullptr;
  int rc = rc_upload_q4nx(m->ctx, gate_up, gate_up_bytes, 2 * m->inter, m->hidden, src | RC_UPLOAD_GATE_UP, &gu);
  if (rc) return rc;
  rc = fmt == kFormatBfp16 ? rc_upload_bfp16(m->ctx, down, down_bytes, m->hidden, m->inter_pad, src, &dn)
                           : rc_upload_q4nx(m->ctx, down, down_bytes, m->hidden, m->inter_pad, src, &dn);
  if (rc) {
    rc_weight_free(gu);
    return rc;
  }
  if (m->gate_up[expert]) rc_weight_free(m->gate_up[expert]);
  if (m->down[expert]) rc_weight_free(m->down[expert]);
  m->gate_up[expert] = gu;
  m->down[expert] = dn;
  m->down_fmt = fmt;
  RC_CUDA_TRY(cudaMemcpy(m->gu_tiles + expert, &gu->tiles, sizeof(void *), cudaMemcpyHostToDevice));
  RC_CUDA_TRY(cudaMemcpy(m->dn_tiles + expert, &dn->tiles, sizeof(void *), cudaMemcpyHostToDevice));
  return RC_OK;
}

int rc_moe_set_fused(rc_moe *m, int enable) {
  RC_CHECK_ARG(m, "rc_moe_set_fused: NULL argument");
  m->fused = enable ? 1 : 0;
  return RC_OK;
}

int rc_moe_set_trace(rc_moe *m, unsigned long long *stamps_dev, int ctas) {
  RC_CHECK_ARG(m, "rc_moe_set_trace: NULL argument");
  RC_CHECK_ARG(!stamps_dev || ctas >= m->ctx->sm_count,
               "rc_moe_set_trace: the buffer must hold %d CTAs x %d stamps", m->ctx->sm_count, kTracePhases);
  m->trace = stamps_dev;
  m->trace_ctas = stamps_dev ? ctas : 0;
  return RC_OK;
}

int rc_moe_set_router(rc_moe *m, const uint16_t *router_w, const float *bias) {
  RC_CHECK_ARG(m && router_w, "rc_moe_set_router: NULL argument");
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  RC_CUDA_TRY(cudaMemcpy(m->router_w, router_w, (size_t)m->n_experts * m->hidden * 2, cudaMemcpyHostToDevice));
  if (bias) RC_CUDA_TRY(cudaMemcpy(m->router_bias, bias, (size_t)m->n_experts * 4, cudaMemcpyHostToDevice));
  return RC_OK;
}

#define RC_MOE_CHECK_TK(fn)                                                                              \
  RC_CHECK_ARG(T >= 1 && T <= kMoeMaxTokens, fn ": T must be 1..%d", kMoeMaxTokens);                    \
  RC_CHECK_ARG(k >= 1 && k <= kMoeMaxK && k <= m->n_experts, fn ": k must be 1..%d and <= n_experts", \
               kMoeMaxK)

int rc_moe_route(rc_moe *m, const uint16_t *x_dev, int T, int k, int router, int renormalize, float scaling,
                 int32_t *ids_dev, float *w_dev, float *logits_dev, void *stream) {
  RC_CHECK_ARG(m && x_dev, "rc_moe_route: NULL argument");
  RC_CHECK_ARG(router == RC_ROUTER_SOFTMAX || router == RC_ROUTER_SIGMOID_BIAS, "unknown router %d", router);
  if (T > kMoeMaxTokens)   // the prefill router (same arithmetic, one warp per token)
    return pf_route_tokens(m, x_dev, T, k, router, renormalize, scaling, ids_dev, w_dev, logits_dev, stream);
  RC_MOE_CHECK_TK("rc_moe_route");
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  const cudaStream_t s = pick_stream(m->ctx, stream);
  int rc = moe_route(m, x_dev, T, k, router, renormalize, scaling, all_owned(m, T, m->has_shared), s);
  if (rc) return rc;
  if (ids_dev) RC_CUDA_TRY(cudaMemcpyAsync(ids_dev, m->s.ids, (size_t)T * k * 4, cudaMemcpyDeviceToDevice, s));
  if (w_dev) RC_CUDA_TRY(cudaMemcpyAsync(w_dev, m->s.weights, (size_t)T * k * 4, cudaMemcpyDeviceToDevice, s));
  if (logits_dev)
    RC_CUDA_TRY(cudaMemcpyAsync(logits_dev, m->s.logits, (size_t)T * m->n_experts * 4, cudaMemcpyDeviceToDevice, s));
  return RC_OK;
}

int rc_moe_experts(rc_moe *m, const uint16_t *x_dev, int T, const int32_t *ids_dev, const float *w_dev, int k,
                   int act, float gate_beta, float value_beta, int with_shared, uint16_t *out_dev, void *stream) {
  RC_CHECK_ARG(m && x_dev && ids_dev && w_dev && out_dev, "rc_moe_experts: NULL argument");
  RC_MOE_CHECK_TK("rc_moe_experts");
  RC_CHECK_ARG(act == RC_ACT_SWIGLU || act == RC_ACT_SITU, "unknown activation %d", act);
  RC_CHECK_ARG(!with_shared || m->has_shared, "this MoE layer has no shared expert");
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  const cudaStream_t s = pick_stream(m->ctx, stream);
  const MoeOwned own = all_owned(m, T, with_shared);
  int rc = moe_slots(m, ids_dev, w_dev, T, k, own, s);
  if (rc) return rc;
  rc = moe_run_experts(m, x_dev, T, k, own, act, gate_beta, value_beta, nullptr, m->down_out, false, s);
  if (rc) return rc;
  return moe_combine(m, m->down_out, m->s.slot_w, T, k, with_shared, out_dev, nullptr, nullptr, s);
}

int rc_moe_experts_host(rc_moe *m, const uint16_t *x_host, int T, const int32_t *ids_host, const float *w_host,
                        int k, int act, float gate_beta, float value_beta, int with_shared, uint16_t *out_host) {
  RC_CHECK_ARG(m && x_host && ids_host && w_host && out_host, "rc_moe_experts_host: NULL argument");
  RC_MOE_CHECK_TK("rc_moe_experts_host");
  for (int t = 0; t < T; ++t) {
    for (int r = 0; r < k; ++r) {
      const int e = ids_host[t * k + r];
      RC_CHECK_ARG(e >= 0 && e < m->n_experts, "expert id %d out of range 0..%d", e, m->n_experts - 1);
      RC_CHECK_ARG(m->gate_up[e] != nullptr, "expert %d is not loaded", e);
      for (int r2 = 0; r2 < r; ++r2)
        RC_CHECK_ARG(ids_host[t * k + r2] != e, "token %d routes to expert %d twice", t, e);
    }
  }
  RC_CHECK_ARG(!with_shared || (m->has_shared && m->gate_up[m->n_experts]), "the shared expert is not loaded");
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  rc_ctx *ctx = m->ctx;
  const size_t x_bytes = (size_t)T * m->hidden * 2, id_bytes = (size_t)T * k * 4;
  const size_t off_ids = (x_bytes + 15) / 16 * 16, off_w = off_ids + (id_bytes + 15) / 16 * 16;
  const size_t xb = off_w + id_bytes, yb = (size_t)T * m->hidden * 2;
  int rc = ensure_host_staging(ctx, xb, yb);
  if (rc) return rc;
  uint8_t *px = static_cast<uint8_t *>(ctx->pin_x);
  memcpy(px, x_host, x_bytes);
  memcpy(px + off_ids, ids_host, id_bytes);
  memcpy(px + off_w, w_host, id_bytes);
  uint8_t *dx = static_cast<uint8_t *>(ctx->dev_x);
  if ((rc = host_copy_in(ctx, dx, px, xb, ctx->stream))) return rc;
  rc = rc_moe_experts(m, reinterpret_cast<const uint16_t *>(dx), T, reinterpret_cast<const int32_t *>(dx + off_ids),
                      reinterpret_cast<const float *>(dx + off_w), k, act, gate_beta, value_beta, with_shared,
                      static_cast<uint16_t *>(ctx->dev_y), nullptr);
  if (rc) return rc;
  if ((rc = host_copy_out_and_wait(ctx, ctx->pin_y, ctx->dev_y, yb, ctx->stream))) return rc;
  memcpy(out_host, ctx->pin_y, yb);
  return RC_OK;
}

int rc_moe_experts_grouped(rc_moe *m, const uint16_t *x_dev, int T, const int32_t *ids_dev, const float *w_dev,
                           int k, const uint16_t *shared_gu_dev, int act, float gate_beta, float value_beta,
                           uint16_t *routed_out_dev, uint16_t *shared_out_dev, void *stream) {
  RC_CHECK_ARG(m && x_dev && ids_dev && w_dev && routed_out_dev, "rc_moe_experts_grouped: NULL argument");
  RC_CHECK_ARG(act == RC_ACT_SWIGLU || act == RC_ACT_SITU, "unknown activation %d", act);
  RC_CHECK_ARG(!shared_gu_dev || (shared_out_dev && m->has_shared && m->down[m->n_experts]),
               "shared_gu needs shared_out and a loaded shared expert");
  if (T > kMoeMaxTokens) {
    // Prefill-sized call: the routed experts of all T tokens in one pass of
    // the register-fragment prefill kernels (a token's bytes equal the
    // decode path's, so the bytes do not depend on T), then the shared
    // expert's down rows in 16-token chunks of the decode kernels with no
    // routed expert in the computed range.
    const int kernel = m->prefill_kernel;
    m->prefill_kernel = RC_PREFILL_GEMV;
    int rc = rc_moe_prefill_experts(m, x_dev, T, ids_dev, w_dev, k, act, gate_beta, value_beta, 0, routed_out_dev,
                                    stream);
    m->prefill_kernel = kernel;
    if (rc || !shared_gu_dev) return rc;
    RC_CHECK_ARG((reinterpret_cast<uintptr_t>(shared_gu_dev) & 15) == 0 && (m->inter * 4) % 16 == 0,
                 "shared_gu rows must be 16-byte aligned");
    const cudaStream_t s = pick_stream(m->ctx, stream);
    for (int t0 = 0; t0 < T; t0 += kMoeMaxTokens) {
      const int tn = T - t0 < kMoeMaxTokens ? T - t0 : kMoeMaxTokens;
      MoeOwned own;
      own.lo = own.hi = 0;
      own.shared_mask = token_mask(0, tn);
      if ((rc = moe_slots(m, ids_dev + (size_t)t0 * k, w_dev + (size_t)t0 * k, tn, k, own, s))) return rc;
      if ((rc = moe_run_experts(m, x_dev + (size_t)t0 * m->hidden, tn, k, own, act, gate_beta, value_beta,
                                shared_gu_dev + (size_t)t0 * 2 * m->inter, m->down_out, false, s)))
        return rc;
      if ((rc = moe_combine(m, m->down_out, m->s.slot_w, tn, k, 0, nullptr, nullptr,
                            shared_out_dev + (size_t)t0 * m->hidden, s)))
        return rc;
    }
    return RC_OK;
  }
  RC_MOE_CHECK_TK("rc_moe_experts_grouped");
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  const cudaStream_t s = pick_stream(m->ctx, stream);
  const MoeOwned own = all_owned(m, T, shared_gu_dev != nullptr);
  int rc = moe_slots(m, ids_dev, w_dev, T, k, own, s);
  if (rc) return rc;
  rc = moe_run_experts(m, x_dev, T, k, own, act, gate_beta, value_beta, shared_gu_dev, m->down_out, false, s);
  if (rc) return rc;
  return moe_combine(m, m->down_out, m->s.slot_w, T, k, 0, nullptr, routed_out_dev,
                     shared_gu_dev ? shared_out_dev : nullptr, s);
}

int rc_moe_decode(rc_moe *m, const uint16_t *x_dev, int T, int k, int router, int renormalize, float scaling,
                  int act, float gate_beta, float value_beta, uint16_t *out_dev, int32_t *ids_dev, float *w_dev,
                  void *stream) {
  RC_CHECK_ARG(m && x_dev && out_dev, "rc_moe_decode: NULL argument");
  RC_MOE_CHECK_TK("rc_moe_decode");
  RC_CHECK_ARG(act == RC_ACT_SWIGLU || act == RC_ACT_SITU, "unknown activation %d", act);
  RC_CHECK_ARG(router == RC_ROUTER_SOFTMAX || router == RC_ROUTER_SIGMOID_BIAS, "unknown router %d", router);
  const MoeOwned own = all_owned(m, T, m->has_shared);
  int rc = check_loaded(m, own);
  if (rc) return rc;
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  const cudaStream_t s = pick_stream(m->ctx, stream);
  if ((reinterpret_cast<uintptr_t>(x_dev) & 15) == 0 && (reinterpret_cast<uintptr_t>(out_dev) & 15) == 0 &&
      moe_fused_fits(m, T, k, own))
    return moe_decode_persistent(m, x_dev, T, k, router, renormalize, scaling, act, gate_beta, value_beta, own,
                            m->down_out, 0, out_dev, ids_dev, w_dev, nullptr, s);
  rc = moe_route(m, x_dev, T, k, router, renormalize, scaling, own, s);
  if (rc) return rc;
  rc = moe_run_experts(m, x_dev, T, k, own, act, gate_beta, value_beta, nullptr, m->down_out, false, s);
  if (rc) return rc;
  rc = moe_combine(m, m->down_out, m->s.slot_w, T, k, m->has_shared, out_dev, nullptr, nullptr, s);
  if (rc) return rc;
  if (ids_dev) RC_CUDA_TRY(cudaMemcpyAsync(ids_dev, m->s.ids, (size_t)T * k * 4, cudaMemcpyDeviceToDevice, s));
  if (w_dev) RC_CUDA_TRY(cudaMemcpyAsync(w_dev, m->s.weights, (size_t)T * k * 4, cudaMemcpyDeviceToDevice, s));
  return RC_OK;
}

int rc_moe_decode_local(rc_moe *m, const uint16_t *x_dev, int T, int k, int router, int renormalize, float scaling,
                        int act, float gate_beta, float value_beta, int expert_lo, int expert_hi, int shared_t0,
                        int shared_tn, uint16_t *slot_out_dev, float *slot_w_dev, void *stream) {
  RC_CHECK_ARG(m && x_dev && slot_out_dev && slot_w_dev, "rc_moe_decode_local: NULL argument");
  RC_MOE_CHECK_TK("rc_moe_decode_local");
  RC_CHECK_ARG(act == RC_ACT_SWIGLU || act == RC_ACT_SITU, "unknown activation %d", act);
  RC_CHECK_ARG(router == RC_ROUTER_SOFTMAX || router == RC_ROUTER_SIGMOID_BIAS, "unknown router %d", router);
  RC_CHECK_ARG(0 <= expert_lo && expert_lo <= expert_hi && expert_hi <= m->n_experts,
               "expert range [%d, %d) outside 0..%d", expert_lo, expert_hi, m->n_experts);
  RC_CHECK_ARG(shared_tn == 0 || (m->has_shared && shared_t0 >= 0 && shared_tn > 0 && shared_t0 + shared_tn <= T),
               "shared token range [%d, +%d) invalid for T=%d", shared_t0, shared_tn, T);
  MoeOwned own;
  own.lo = expert_lo;
  own.hi = expert_hi;
  own.shared_mask = shared_tn ? token_mask(shared_t0, shared_tn) : 0u;
  int rc = check_loaded(m, own);
  if (rc) return rc;
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  const cudaStream_t s = pick_stream(m->ctx, stream);
  // The router writes the slot weights straight into slot_w_dev; slot rows of
  // experts computed elsewhere are zeroed by the gate/up launch, so the
  // ranks' slot rows can be summed in the exchange (x + 0 = x exactly).
  RC_CHECK_ARG((reinterpret_cast<uintptr_t>(slot_out_dev) & 15) == 0, "slot_out must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(x_dev) & 15) == 0 && moe_fused_fits(m, T, k, own))
    return moe_decode_persistent(m, x_dev, T, k, router, renormalize, scaling, act, gate_beta, value_beta, own,
                            slot_out_dev, 1, nullptr, nullptr, nullptr, slot_w_dev, s);
  MoeScratch sc = m->s;
  sc.slot_w = slot_w_dev;
  rc = moe_route(m, x_dev, T, k, router, renormalize, scaling, own, s, &sc);
  if (rc) return rc;
  return moe_run_experts(m, x_dev, T, k, own, act, gate_beta, value_beta, nullptr, slot_out_dev, true, s);
}

int rc_moe_combine(rc_moe *m, const uint16_t *slot_out_dev, const float *slot_w_dev, int T, int k, int with_shared,
                   uint16_t *out_dev, void *stream) {
  RC_CHECK_ARG(m && slot_out_dev && slot_w_dev && out_dev, "rc_moe_combine: NULL argument");
  RC_MOE_CHECK_TK("rc_moe_combine");
  RC_CHECK_ARG(!with_shared || m->has_shared, "this MoE layer has no shared expert");
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  return moe_combine(m, slot_out_dev, slot_w_dev, T, k, with_shared, out_dev, nullptr, nullptr,
                     pick_stream(m->ctx, stream));
}

int rc_moe_ep_init(rc_moe *m, int rank, int world, int tokens_per_rank, void *handle_out) {
  RC_CHECK_ARG(m && handle_out, "rc_moe_ep_init: NULL argument");
  RC_CHECK_ARG(world >= 2 && world <= kEpMaxRanks, "rc_moe_ep_init: world must be 2..%d", kEpMaxRanks);
  RC_CHECK_ARG(rank >= 0 && rank < world, "rc_moe_ep_init: rank %d outside 0..%d", rank, world - 1);
  RC_CHECK_ARG(tokens_per_rank >= 1 && world * tokens_per_rank <= kMoeMaxTokens,
               "rc_moe_ep_init: world * tokens_per_rank must be 1..%d", kMoeMaxTokens);
  RC_CHECK_ARG(m->n_experts >= world, "rc_moe_ep_init: %d experts cannot be split over %d ranks", m->n_experts,
               world);
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  RC_CUDA_TRY(cudaDeviceSynchronize());
  ep_release(m);
  MoeEp *ep = new MoeEp();
  ep->rank = rank;
  ep->world = world;
  ep->M = tokens_per_rank;
  ep->bytes = ep_bytes(world, tokens_per_rank, m->hidden);
  ep->epoch = m->ctx->timeout_epoch;
  m->ep = ep;
  cudaDeviceProp prop;
  MoeEpBlob blob{};
  cudaError_t e = cudaGetDeviceProperties(&prop, m->ctx->device);
  if (e == cudaSuccess) e = cudaMalloc(&ep->base, ep->bytes);
  if (e == cudaSuccess) e = cudaMemset(ep->base, 0, ep->bytes);
  if (e == cudaSuccess) e = cudaMalloc(&ep->peer_dev, kEpMaxRanks * sizeof(uint8_t *));
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, ep->base);
  if (e != cudaSuccess) {
    set_error("rc_moe_ep_init: %s", cudaGetErrorString(e));
    ep_release(m);
    return RC_ERR_CUDA;
  }
  ep->peer[rank] = ep->base;
  ep->mapped[rank] = true;
  memcpy(ep->uuid[rank], &prop.uuid, 16);
  memcpy(blob.ipc, &h, sizeof(h));
  memcpy(blob.uuid, &prop.uuid, 16);
  blob.rank = rank;
  blob.world = world;
  blob.M = tokens_per_rank;
  blob.hidden = m->hidden;
  blob.n_experts = m->n_experts;
  blob.has_shared = m->has_shared;
  blob.bytes = ep->bytes;
  memset(handle_out, 0, RC_EP_HANDLE_BYTES);
  memcpy(handle_out, &blob, sizeof(blob));
  return RC_OK;
}

int rc_moe_ep_open(rc_moe *m, int peer, const void *handle) {
  RC_CHECK_ARG(m && handle, "rc_moe_ep_open: NULL argument");
  MoeEp *ep = m->ep;
  RC_CHECK_ARG(ep, "rc_moe_ep_open: rc_moe_ep_init has not run");
  RC_CHECK_ARG(peer >= 0 && peer < ep->world, "rc_moe_ep_open: peer %d outside 0..%d", peer, ep->world - 1);
  MoeEpBlob blob;
  memcpy(&blob, handle, sizeof(blob));
  if (peer == ep->rank) {
    RC_CHECK_ARG(memcmp(blob.uuid, ep->uuid[peer], 16) == 0 && blob.rank == peer,
                 "rc_moe_ep_open: the blob given for this rank is not its own");
    return RC_OK;
  }
  RC_CHECK_ARG(!ep->mapped[peer], "rc_moe_ep_open: peer %d is already mapped", peer);
  RC_CHECK_ARG(blob.rank == peer && blob.world == ep->world && blob.M == ep->M && blob.hidden == m->hidden &&
                   blob.n_experts == m->n_experts && blob.has_shared == m->has_shared && blob.bytes == ep->bytes,
               "rc_moe_ep_open: the blob of peer %d describes another rank or layer geometry", peer);
  for (int r = 0; r < ep->world; ++r)
    RC_CHECK_ARG(!ep->mapped[r] || memcmp(blob.uuid, ep->uuid[r], 16) != 0,
                 "rc_moe_ep_open: peers %d and %d are on the same GPU (one rank per GPU)", peer, r);
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  cudaIpcMemHandle_t h;
  memcpy(&h, blob.ipc, sizeof(h));
  void *ptr = nullptr;
  RC_CUDA_TRY(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
  ep->peer[peer] = static_cast<uint8_t *>(ptr);
  ep->mapped[peer] = true;
  memcpy(ep->uuid[peer], blob.uuid, 16);
  RC_CUDA_TRY(cudaMemcpy(ep->peer_dev, ep->peer, kEpMaxRanks * sizeof(uint8_t *), cudaMemcpyHostToDevice));
  return RC_OK;
}

int rc_moe_ep_decode(rc_moe *m, const uint16_t *x_dev, int k, int router, int renormalize, float scaling, int act,
                     float gate_beta, float value_beta, uint16_t *out_dev, void *stream) {
  RC_CHECK_ARG(m && x_dev && out_dev, "rc_moe_ep_decode: NULL argument");
  MoeEp *ep = m->ep;
  RC_CHECK_ARG(ep, "rc_moe_ep_decode: rc_moe_ep_init has not run");
  for (int r = 0; r < ep->world; ++r)
    RC_CHECK_ARG(ep->mapped[r], "rc_moe_ep_decode: the buffer of rank %d is not mapped (rc_moe_ep_open)", r);
  if (ep->epoch != m->ctx->timeout_epoch) {
    set_error("rc_moe_ep_decode: a bounded wait gave up since rc_moe_ep_init; the exchange counters are lost, "
              "run rc_moe_ep_init and rc_moe_ep_open again on every rank");
    return RC_ERR_TIMEOUT;
  }
  const int T = ep->world * ep->M;
  RC_MOE_CHECK_TK("rc_moe_ep_decode");
  RC_CHECK_ARG(act == RC_ACT_SWIGLU || act == RC_ACT_SITU, "unknown activation %d", act);
  RC_CHECK_ARG(router == RC_ROUTER_SOFTMAX || router == RC_ROUTER_SIGMOID_BIAS, "unknown router %d", router);
  RC_CHECK_ARG((reinterpret_cast<uintptr_t>(x_dev) & 15) == 0 && (reinterpret_cast<uintptr_t>(out_dev) & 15) == 0,
               "rc_moe_ep_decode: x and out must be 16-byte aligned");
  MoeOwned own;
  own.lo = (int)((long long)ep->rank * m->n_experts / ep->world);
  own.hi = (int)((long long)(ep->rank + 1) * m->n_experts / ep->world);
  own.shared_mask = m->has_shared ? token_mask(ep->rank * ep->M, ep->M) : 0u;
  int rc = check_loaded(m, own);
  if (rc) return rc;
  RC_CHECK_ARG(m->down_fmt == kFormatQ4nx,
               "rc_moe_ep_decode: the persistent decode kernel takes q4nx down matrices, not bfp16ebs8");
  RC_CHECK_ARG(moe_decode_shape_ok(m, T, k, own),
               "rc_moe_ep_decode: T=%d k=%d does not fit the persistent decode kernel", T, k);
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  MoeEpArgs a;
  a.rank = ep->rank;
  a.world = ep->world;
  a.M = ep->M;
  a.peer_dev = ep->peer_dev;
  a.flags = reinterpret_cast<unsigned long long *>(ep->base);
  a.tok_off = (uint32_t)ep_tok_off();
  a.red_off = (uint32_t)ep_red_off(ep->world, ep->M, m->hidden);
  a.x_own = x_dev;
  return moe_decode_persistent(m, reinterpret_cast<const uint16_t *>(ep->base + ep_tok_off()), T, k, router,
                          renormalize, scaling, act, gate_beta, value_beta, own, m->down_out, 0, out_dev, nullptr,
                          nullptr, nullptr, pick_stream(m->ctx, stream), &a);
}


}  // extern "C"

// A layer call on host buffers: the token rows are copied in from pinned
// staging, ``run`` launches on the stream, the output rows (and the optional
// ids / weights [T_out][k]) are copied back with the error word, and one wait
// covers them (the copies are kernels: host_copy_in / host_copy_out_and_wait).
template <class Run>
static int moe_layer_host(rc_moe *m, const uint16_t *x_host, int T_in, int T_out, int k, uint16_t *out_host,
                          int32_t *ids_host, float *w_host, void *stream, Run run) {
  rc_ctx *ctx = m->ctx;
  RC_CUDA_TRY(cudaSetDevice(ctx->device));
  const cudaStream_t s = pick_stream(ctx, stream);
  const size_t xb = (size_t)T_in * m->hidden * 2, yb = (size_t)T_out * m->hidden * 2;
  const size_t rb = (size_t)T_out * k * 4;
  const size_t off_ids = (yb + 15) / 16 * 16, off_w = off_ids + (rb + 15) / 16 * 16;
  const size_t back = (ids_host || w_host) ? off_w + rb : yb;
  int rc = ensure_host_staging(ctx, xb, back);
  if (rc) return rc;
  memcpy(ctx->pin_x, x_host, xb);
  if ((rc = host_copy_in(ctx, ctx->dev_x, ctx->pin_x, xb, s))) return rc;
  uint8_t *dy = static_cast<uint8_t *>(ctx->dev_y);
  rc = run(static_cast<const uint16_t *>(ctx->dev_x), reinterpret_cast<uint16_t *>(dy),
           ids_host ? reinterpret_cast<int32_t *>(dy + off_ids) : nullptr,
           w_host ? reinterpret_cast<float *>(dy + off_w) : nullptr, static_cast<void *>(s));
  if (rc) return rc;
  if ((rc = host_copy_out_and_wait(ctx, ctx->pin_y, ctx->dev_y, back, s))) return rc;
  const uint8_t *py = static_cast<const uint8_t *>(ctx->pin_y);
  memcpy(out_host, py, yb);
  if (ids_host) memcpy(ids_host, py + off_ids, rb);
  if (w_host) memcpy(w_host, py + off_w, rb);
  return RC_OK;
}

extern "C" {

int rc_moe_decode_host(rc_moe *m, const uint16_t *x_host, int T, int k, int router, int renormalize, float scaling,
                       int act, float gate_beta, float value_beta, uint16_t *out_host, int32_t *ids_host,
                       float *w_host, void *stream) {
  RC_CHECK_ARG(m && x_host && out_host, "rc_moe_decode_host: NULL argument");
  RC_MOE_CHECK_TK("rc_moe_decode_host");
  return moe_layer_host(m, x_host, T, T, k, out_host, ids_host, w_host, stream,
                        [&](const uint16_t *x, uint16_t *y, int32_t *ids, float *w, void *st) {
                          return rc_moe_decode(m, x, T, k, router, renormalize, scaling, act, gate_beta, value_beta,
                                               y, ids, w, st);
                        });
}

int rc_moe_prefill_host(rc_moe *m, const uint16_t *x_host, int T, int k, int router, int renormalize, float scaling,
                        int act, float gate_beta, float value_beta, uint16_t *out_host, int32_t *ids_host,
                        float *w_host, void *stream) {
  RC_CHECK_ARG(m && x_host && out_host, "rc_moe_prefill_host: NULL argument");
  RC_CHECK_ARG(T >= 1 && T <= kPfMaxTokens, "rc_moe_prefill_host: T=%d outside 1..%d", T, kPfMaxTokens);
  RC_CHECK_ARG(k >= 1 && k <= kMoeMaxK, "rc_moe_prefill_host: k=%d outside 1..%d", k, kMoeMaxK);
  return moe_layer_host(m, x_host, T, T, k, out_host, ids_host, w_host, stream,
                        [&](const uint16_t *x, uint16_t *y, int32_t *ids, float *w, void *st) {
                          return rc_moe_prefill(m, x, T, k, router, renormalize, scaling, act, gate_beta, value_beta,
                                                y, ids, w, st);
                        });
}

int rc_moe_ep_decode_host(rc_moe *m, const uint16_t *x_host, int k, int router, int renormalize, float scaling,
                          int act, float gate_beta, float value_beta, uint16_t *out_host, void *stream) {
  RC_CHECK_ARG(m && x_host && out_host, "rc_moe_ep_decode_host: NULL argument");
  RC_CHECK_ARG(m->ep, "rc_moe_ep_decode_host: rc_moe_ep_init has not run");
  const int M = m->ep->M;
  return moe_layer_host(m, x_host, M, M, k, out_host, nullptr, nullptr, stream,
                        [&](const uint16_t *x, uint16_t *y, int32_t *, float *, void *st) {
                          return rc_moe_ep_decode(m, x, k, router, renormalize, scaling, act, gate_beta, value_beta,
                                                  y, st);
                        });
}

}  // extern "C"
