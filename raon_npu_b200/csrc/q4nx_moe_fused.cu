// The MoE decode layer for T <= 16 tokens as one persistent kernel: one CTA
// per SM (a cooperative launch, so every CTA is resident) runs the whole
// layer, phase after phase, with grid-wide barriers between the phases that
// exchange data through global memory:
//
//   1 logits     CTA c computes the logits of experts c, c + grid, ...
//                (f64 sums of exact bf16 products, rounded once to f32)
//   -- barrier --
//   2 selection  every CTA reads the T x E logits and repeats the selection
//                in its own shared memory: one warp per token takes the k
//                best experts in the router order (larger first, NaN last,
//                ties by lower index) by k warp-wide arg-max rounds, then the
//                weights, the ascending-ID slot lists and the group table --
//                identical inputs give identical tables, so no barrier is
//                needed after it
//   3 gate/up    the CTA's contiguous range of (group, row tile) tiles; units
//                dealt to 16 warps k-block-major (RoundCursor),
//                per-unit partials summed in k-block order (a tile's result
//                never depends on the partition); GLU epilogue -> act rows
//   -- barrier --
//   4 down       the same partition over the down tiles; the act rows of the
//                range's groups staged in shared memory; slot rows out
//   -- barrier --
//   5 combine    ascending-ID f32 sum (multiply then add, no FMA), RTNE, plus
//                the shared row
//
// Every warp streams its units through one ring of bulk copies that runs on
// from its gate/up units into its down units, so the down weights are in
// flight while gate/up is still computing.  The arithmetic of each tile, of
// the routing and of the combine is the one of the separate kernels in
// q4nx_moe.cu, so the bytes are the same.  Every wait is bounded.
#include "moe_internal.cuh"
#include "q4nx_core.cuh"
#include "rc_device.cuh"
#include "rc_internal.cuh"

namespace rc {

constexpr int kFzWarps = 16;
constexpr int kFzThreads = kFzWarps * 32;
constexpr int kFzMaxStages = 4;
constexpr int kFzChunks = kMoeMaxExperts / 32;        // router values a lane holds per token
// the "red" area: [16 warps][16 tokens] f64 partial logits, the barrier
// verdict word, then the peer buffer table (8 pointers) and the two phase
// ranges
constexpr int kFzRedBytes = kFzWarps * kMoeMaxTokens * 8 + 16;

struct MoeFusedParams {
  // tokens and router
  const uint16_t *x;                 // [T][hidden]
  int T, hidden, n_experts, k, mode, renorm;
  float scaling;
  const uint16_t *wr;                // [E][hidden]
  const float *bias;                 // [E]
  int shared_id;
  MoeOwned own;
  float *logits;                     // [T][E] scratch
  int32_t *ids_out;                  // [T][k] rank order (optional)
  float *w_out;                      // [T][k] (optional)
  float *slot_w_out;                 // [T][k] ascending-ID order (optional)
  // experts
  const uint8_t *const *gu_tiles;    // [E+1]
  const uint8_t *const *dn_tiles;    // [E+1]
  int inter, inter_pad;
  uint16_t *act;                     // [E+1][16][inter_pad]
  uint16_t *slot_rows;               // [T][k+1][hidden]
  int zero_foreign;                  // zero the slot rows of experts computed elsewhere
  uint16_t *out;                     // [T][hidden], null: no combine
  int act_kind;
  float gate_beta, value_beta;
  // launch geometry
  int stages, round_gu, round_dn;
  // shared-memory layout (byte offsets)
  int off_stage, off_part, off_tab, off_sel, off_red, off_bar;
  unsigned long long *bar;           // grid-barrier arrival count (only grows)
  int *err;
  // expert parallelism over peer memory (ep_world > 1): x is this rank's
  // exchange buffer's token rows, out its own tokens' rows
  int ep_world, ep_rank, ep_M;
  uint8_t *const *ep_peer;           // [world] every rank's exchange buffer
  unsigned long long *ep_flags;      // this rank's counters (token rows, expert rows, calls)
  uint32_t ep_tok_off, ep_red_off;   // byte offsets in an exchange buffer
  const uint16_t *ep_x_own;          // this rank's token rows [M][hidden]
  unsigned long long *trace;         // phase stamps [grid][kTracePhases] (null: off)
};

// Thread 0 records the global timer at a phase boundary (rc_moe_set_trace).
__device__ __forceinline__ void fz_stamp(const MoeFusedParams &p, int phase) {
  if (p.trace && threadIdx.x == 0) p.trace[(size_t)blockIdx.x * kTracePhases + phase] = global_timer_ns();
}

// what build_activations reads
struct FzStage {
  const void *x;
  int x_dtype, ldx, tokens, slots, x_vec, kb;
};

// Router order as an unsigned key: larger value -> larger key, -0 equal to
// +0, NaN (1) below every number, 0 = no candidate.  Equal keys are ordered
// by lower expert index, so (key, index) is the router order (route_before).
__device__ __forceinline__ uint32_t route_key(float v) {
  if (v != v) return 1u;
  uint32_t b = __float_as_uint(v);
  if (b == 0x80000000u) b = 0u;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// An expert's routing score and its router-order key: sigmoid(logit)
// (selected by score + bias), or the biased logit (softmax router; bias zero
// unless set).  Out of line: the unrolled selection calls it for each of a
// lane's experts, and one copy of the f64 exponential keeps the code small.
struct FzScore {
  uint32_t key;
  float score;
};
static __device__ __noinline__ FzScore fz_score(float l, float bias, int mode) {
  FzScore r;
  float v;
  if (mode == RC_ROUTER_SIGMOID_BIAS) {
    r.score = __double2float_rn(1.0 / (1.0 + exp(-(double)l)));
    v = r.score + bias;
  } else {
    r.score = l + bias;
    v = r.score;
  }
  r.key = route_key(v);
  return r;
}

// The group table of the ascending-ID slot lists, built by the whole CTA
// (the same table as build_groups): one group per expert of [own.lo, own.hi)
// that some token chose, ascending, then the shared expert for the tokens of
// own.shared_mask; per (group, token) the slot row t*(k+1) + position.
// Scratch: mask_s / gidx_s [E+1], cnt_s [(E+32)/32].
__device__ void fz_build_groups(const int32_t *slots, int T, int k, int E, MoeOwned own, int32_t *g_expert,
                                uint32_t *g_mask, int32_t *g_dst, int *n_groups, uint32_t *mask_s, int *gidx_s,
                                int *cnt_s, int *err) {
  const int tid = threadIdx.x, nth = blockDim.x, warp = tid >> 5, lane = tid & 31;
  for (int e = tid; e <= E; e += nth) mask_s[e] = e == E ? own.shared_mask : 0u;
  __syncthreads();
  for (int pr = tid; pr < T * k; pr += nth) {
    const int t = pr / k, r = pr - t * k;
    const int e = slots[t * (k + 1) + r];
    if (e >= own.lo && e < own.hi) atomicOr(mask_s + e, 1u << t);
    else if (e < 0 || e >= E) atomicCAS(err, 0, kErrBadExpert);
  }
  __syncthreads();
  const int nchunks = (E + 1 + 31) / 32;      // <= 9 <= warps
  uint32_t m = 0, b = 0;
  const int e = warp * 32 + lane;
  if (warp < nchunks) {
    m = e <= E ? mask_s[e] : 0u;
    b = __ballot_sync(0xffffffffu, m != 0u);
    if (lane == 0) cnt_s[warp] = __popc(b);
  }
  __syncthreads();
  if (warp < nchunks) {
    int base = 0;
    for (int c = 0; c < warp; ++c) base += cnt_s[c];
    if (m) {
      const int gi = base + __popc(b & ((1u << lane) - 1u));
      g_expert[gi] = e;
      g_mask[gi] = m;
      gidx_s[e] = gi;
    }
    if (warp == nchunks - 1 && lane == 0) *n_groups = base + __popc(b);
  }
  __syncthreads();
  for (int pr = tid; pr < T * (k + 1); pr += nth) {
    const int t = pr / (k + 1), r = pr - t * (k + 1);
    const int ex = slots[pr];
    const bool mine = r < k ? (ex >= own.lo && ex < own.hi) : (ex >= 0 && ((own.shared_mask >> t) & 1u));
    if (mine) g_dst[gidx_s[ex] * T + t] = pr;
  }
  __syncthreads();
}

// All CTAs meet.  Arrival n (counted over the layer's lifetime) belongs to
// barrier n / grid, which is complete when the count reaches the next
// multiple of the grid.  The arrival releases the CTA's writes (ordered
// before it by the CTA barrier), the acquiring load makes the other CTAs'
// writes visible.  Bounded: false after 1 s (error word set), CTA-uniform.
__device__ bool fz_grid_barrier(unsigned long long *bar, int *err, int *ok_s) {
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned long long old = atom_add_release_gpu(bar, 1ull);
    const unsigned long long target = (old / gridDim.x + 1) * gridDim.x;
    if (ld_acquire_gpu(bar) < target) {
      const uint64_t t0 = global_timer_ns();
      while (ld_acquire_gpu(bar) < target) {
        if (global_timer_ns() - t0 > 1000000000ull) {
          ok = 0;
          atomicCAS(err, 0, kErrWaitTimeout);
          break;
        }
      }
    }
    *ok_s = ok;
  }
  __syncthreads();
  return *ok_s != 0;
}

// Wait until a counter that peer GPUs add to reaches ``target``.  Bounded:
// false after 1 s (error word set), CTA-uniform.
__device__ bool fz_wait_sys(const unsigned long long *ctr, unsigned long long target, int *err, int *ok_s) {
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    if (ld_acquire_sys(ctr) < target) {
      const uint64_t t0 = global_timer_ns();
      while (ld_acquire_sys(ctr) < target) {
        if (global_timer_ns() - t0 > 1000000000ull) {
          ok = 0;
          atomicCAS(err, 0, kErrWaitTimeout);
          break;
        }
      }
    }
    *ok_s = ok;
  }
  __syncthreads();
  return *ok_s != 0;
}

// One phase's units: tiles [c0, c0 + n_tiles) of the group-major tile list,
// kb k-blocks each, rounds of R tiles (see RoundCursor).
struct FzRange {
  const uint8_t *const *g_ptr;       // [groups] tile base of each group (shared memory; null: not loaded)
  int c0, n_tiles, R, kb;
  FastDiv gt;                        // tiles per group

  __device__ __forceinline__ const uint8_t *src(const RoundCursor &c) const {
    const uint32_t tg = c0 + c.tile();
    const uint32_t grp = fdiv(tg, gt), tile = tg - grp * gt.d;
    const uint8_t *b = g_ptr[grp];
    return b ? b + ((size_t)tile * kb + c.kbi) * kUnitBytes : nullptr;
  }
};

// A warp's ring: the gate/up units of its chunks, then its down units.  The
// issue cursor runs up to S units ahead of consumption, across the phase
// boundary, so the first down weights are in flight during gate/up.
struct FzRing {
  RoundCursor iss;                   // next unit to fetch (lane 0)
  int iss_phase;                     // 0 gate/up, 1 down, 2 none left
  int slot, issued, consumed;
  uint32_t parity;
  bool failed;
};

__device__ __forceinline__ void fz_issue(FzRing &rg, const FzRange *ph, int warp, uint32_t ring_s, uint32_t bar0,
                                         uint64_t pol, int sl) {
  const uint8_t *src = ph[rg.iss_phase].src(rg.iss);
  if (src) {
    mbar_arrive_expect_tx(bar0 + 8 * sl, kUnitBytes);
    bulk_copy_g2s(ring_s + sl * kUnitBytes, src, kUnitBytes, bar0 + 8 * sl, pol);
  } else {
    mbar_arrive_expect_tx(bar0 + 8 * sl, 0);     // nothing to fetch: complete the phase at once
  }
  ++rg.issued;
  rg.iss.next();
  while (rg.iss_phase < 2 && !rg.iss.valid()) {
    if (++rg.iss_phase < 2) rg.iss.init(ph[1].n_tiles, ph[1].R, ph[1].kb, kFzWarps, warp);
  }
}

enum FzEpi : int { kFzGlu = 0, kFzDown = 1 };

// The GLU activation, out of line (one body for the epilogue's unrolled sites).
static __device__ __noinline__ float fz_glu(float gate, float up, int kind, float gb, float vb) {
  return kind == RC_ACT_SITU ? act_situ(gate, up, gb, vb) : act_swiglu(gate, up);
}

// One phase (gate/up or down) of this CTA over ph[EPI].  Each unit's result
// goes to its own shared-memory partial; after a round's barrier one warp per
// tile sums the tile's partials in k-block order and runs the epilogue, so a
// tile's result depends on the tile alone.
template <int EPI, int NTB>
__device__ void fz_phase(const MoeFusedParams &p, uint8_t *smem, const FzRange *ph, const uint32_t *g_mask,
                         const int *g_dst, int g_lo, FzRing &rg) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const FzRange &pr = ph[EPI];
  uint8_t *const *ep_peer_s = reinterpret_cast<uint8_t *const *>(smem + p.off_red + kFzRedBytes);
  const int S = p.stages;
  const int kb = pr.kb, k = kb * kUnitK, R = pr.R, n_tiles = pr.n_tiles;
  uint8_t *ring = smem + warp * S * kUnitBytes;
  const uint32_t ring_s = smem_addr(ring);
  const uint32_t bar0 = smem_addr(smem + p.off_bar) + warp * S * 8;
  const uint32_t *xs = reinterpret_cast<const uint32_t *>(smem + p.off_stage);
  constexpr int kBlocks = EPI == kFzGlu ? NTB : NTB * kMoeMaxGroupsPerCta;
  const void *xa = smem + p.off_stage + xfrag_bytes(kBlocks, k);
  XFrag<NTB> xr;
  int xr_key = -1;                              // (block, k-block) held in xr
  float4 *part = reinterpret_cast<float4 *>(smem + p.off_part);
  const uint64_t pol = policy_evict_first();
  const int n_rounds = round_count(n_tiles, R);
  RoundCursor cur;
  cur.init(n_tiles, R, kb, kFzWarps, warp);
  const int g = lane >> 2, qd = lane & 3;
  for (int r = 0; r < n_rounds; ++r) {
    for (; cur.valid() && cur.round == r; cur.next()) {
      const uint32_t grp = fdiv(pr.c0 + cur.tile(), pr.gt);
      if (!rg.failed) {
        if (mbar_wait_bounded_warp(bar0 + 8 * rg.slot, rg.parity)) {
          ++rg.consumed;
        } else {
          if (lane == 0) atomicCAS(p.err, 0, kErrWaitTimeout);
          rg.failed = true;
        }
      }
      if (!rg.failed && pr.g_ptr[grp] != nullptr) {
        const int blk = EPI == kFzGlu ? 0 : ((int)grp - g_lo) * NTB;
        if (blk * kb + cur.kbi != xr_key) {
          load_xfrag<NTB, true>(xr, xs, xa, kBlocks, blk, kb, cur.kbi, lane);
          xr_key = blk * kb + cur.kbi;
        }
        float4 Q[NTB];
        unit_result<NTB>(ring + rg.slot * kUnitBytes, xr, lane, Q);
        float4 *dst = part + (size_t)cur.slot() * NTB * 32 + lane;
#pragma unroll
        for (int tb = 0; tb < NTB; ++tb) dst[tb * 32] = Q[tb];
      }
      __syncwarp();
      if (!rg.failed && lane == 0 && rg.iss_phase < 2) fz_issue(rg, ph, warp, ring_s, bar0, pol, rg.slot);
      if (++rg.slot == S) rg.slot = 0, rg.parity ^= 1u;
    }
    __syncthreads();
    const int t_lo = r * R, t_hi = t_lo + R < n_tiles ? t_lo + R : n_tiles;
    for (int ti = t_lo + warp; ti < t_hi; ti += kFzWarps) {
      const uint32_t tg = pr.c0 + ti;
      const uint32_t grp = fdiv(tg, pr.gt), tile = tg - grp * pr.gt.d;
      const bool live = pr.g_ptr[grp] != nullptr;
      Acc<NTB> acc;
      acc_zero(acc);
      const float4 *src = part + (size_t)(ti - t_lo) * kb * NTB * 32 + lane;
      for (int kbi = 0; kbi < kb; ++kbi) {
        float4 v[NTB];
#pragma unroll
        for (int tb = 0; tb < NTB; ++tb) v[tb] = src[(kbi * NTB + tb) * 32];
        acc_add(acc, v);
      }
      const uint32_t mask = g_mask[grp];
#pragma unroll
      for (int tb = 0; tb < NTB; ++tb) {
#pragma unroll
        for (int e2 = 0; e2 < 2; ++e2) {
          const int t = tb * 8 + 2 * qd + e2;
          if (t >= p.T || !((mask >> t) & 1u)) continue;
          if (EPI == kFzGlu) {
            float v = 0.f;
            if (live) {
              const float gate = bf16_round(acc.v[tb][e2]);
              const float up = bf16_round(acc.v[tb][2 + e2]);
              v = fz_glu(gate, up, p.act_kind, p.gate_beta, p.value_beta);
            }
            p.act[((size_t)grp * 8 * NTB + t) * p.inter_pad + tile * 8 + g] = f32_to_bf16_rne(v);
          } else {
            const int srow = g_dst[grp * p.T + t];     // slot row t*(k+1) + position
            uint16_t *y;
            if (p.ep_world > 1) {
              // straight into the buffer of the token's owner
              const int tt = srow / (p.k + 1), pos = srow - tt * (p.k + 1);
              const int owner = tt / p.ep_M, tl = tt - owner * p.ep_M;
              y = reinterpret_cast<uint16_t *>(ep_peer_s[owner] + p.ep_red_off) +
                  ((size_t)tl * (p.k + 1) + pos) * p.hidden + tile * kUnitRows + g;
            } else {
              y = p.slot_rows + (size_t)srow * p.hidden + tile * kUnitRows + g;
            }
            y[0] = live ? f32_to_bf16_rne(acc.v[tb][e2]) : (uint16_t)0;
            y[8] = live ? f32_to_bf16_rne(acc.v[tb][2 + e2]) : (uint16_t)0;
          }
        }
      }
    }
    __syncthreads();
  }
}

template <int NTB>
__global__ void __launch_bounds__(kFzThreads, 1) rc_moe_fused_kernel(MoeFusedParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  int *ok_s = reinterpret_cast<int *>(smem + p.off_red + kFzWarps * kMoeMaxTokens * 8);
  uint8_t **ep_peer_s = reinterpret_cast<uint8_t **>(smem + p.off_red + kFzRedBytes);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = p.T, E = p.n_experts, k = p.k;
  const int gt_gu_i = p.inter / 8, kb_gu_i = p.hidden / kUnitK;
  const int gt_dn_i = p.hidden / kUnitRows, kb_dn_i = p.inter_pad / kUnitK;
  fz_stamp(p, kTrStart);
  if (p.trace && tid == 0 && p.ep_world <= 1) p.trace[(size_t)blockIdx.x * kTracePhases + kTrTokens] = 0;

  // ---- expert parallelism: every rank's token rows into every rank's buffer
  unsigned long long ep_calls = 0;
  if (p.ep_world > 1) {
    ep_calls = *reinterpret_cast<volatile unsigned long long *>(p.ep_flags + 2);
    if (tid < p.ep_world) ep_peer_s[tid] = p.ep_peer[tid];
    __syncthreads();
    if (blockIdx.x == 0) {
      const int n16 = p.ep_M * p.hidden / 8;
      const uint4 *src = reinterpret_cast<const uint4 *>(p.ep_x_own);
      for (int r = 0; r < p.ep_world; ++r) {
        uint4 *dst = reinterpret_cast<uint4 *>(ep_peer_s[r] + p.ep_tok_off) + (size_t)p.ep_rank * n16;
        for (int i = tid; i < n16; i += blockDim.x) dst[i] = src[i];
      }
      __syncthreads();
      if (tid == 0) {
        __threadfence_system();
        for (int r = 0; r < p.ep_world; ++r)
          red_add_release_sys(reinterpret_cast<unsigned long long *>(ep_peer_s[r]) + 0, 1ull);
      }
    }
  }

  // per-expert tables kept in shared memory for the whole kernel
  const uint8_t **all_gu = reinterpret_cast<const uint8_t **>(smem + p.off_tab);    // [E+1]
  const uint8_t **all_dn = all_gu + (E + 1);                                         // [E+1]
  const uint8_t **g_gu = all_dn + (E + 1);                                           // [E+1] per group
  const uint8_t **g_dn = g_gu + (E + 1);                                             // [E+1]
  float *bias_s = reinterpret_cast<float *>(g_dn + (E + 1));                        // [E+1]
  int32_t *g_expert = reinterpret_cast<int32_t *>(bias_s + (E + 1));                // [E+1]
  uint32_t *g_mask = reinterpret_cast<uint32_t *>(g_expert + (E + 1));              // [E+1]
  int32_t *g_dst = reinterpret_cast<int32_t *>(g_mask + (E + 1));                   // [E+1][16]
  int *n_groups_s = g_dst + (E + 1) * T;
  auto load_tables = [&](int first, int stride) {
    for (int i = first; i <= E; i += stride) {
      all_gu[i] = p.gu_tiles[i];
      all_dn[i] = p.dn_tiles[i];
      bias_s[i] = i < E ? p.bias[i] : 0.f;
    }
  };
  const int nslice = p.hidden / 256;
  const int busy = nslice < kFzWarps ? nslice : kFzWarps;   // warps with router columns
  // warps without router columns fetch the tables while the others compute
  if (busy < kFzWarps && warp >= busy) load_tables(tid - busy * 32, (kFzWarps - busy) * 32);

  if (p.ep_world > 1) {
    if (!fz_wait_sys(p.ep_flags + 0, (ep_calls + 1) * p.ep_world, p.err, ok_s)) return;
    fz_stamp(p, kTrTokens);
  }

  // ------------------------------------------------------------ 1 logits
  {
    double *red = reinterpret_cast<double *>(smem + p.off_red);     // [16 warps][16 tokens]
    for (int e = blockIdx.x; e < E; e += gridDim.x) {
      // tokens four at a time (a rolled loop: the kernel's code must stay
      // small); each token's sum runs in the same order as with all at once
      for (int t0 = 0; t0 < T; t0 += 4) {
        double acc[4] = {0.0, 0.0, 0.0, 0.0};
        for (int sl = warp; sl < nslice; sl += kFzWarps) {
          const int col = sl * 256 + lane * 8;
          const uint4 wv = __ldg(reinterpret_cast<const uint4 *>(p.wr + (size_t)e * p.hidden + col));
          uint4 xv[4];
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (t0 + q < T) xv[q] = __ldcg(reinterpret_cast<const uint4 *>(p.x + (size_t)(t0 + q) * p.hidden + col));
          const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
          double wd[8];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            wd[2 * j] = (double)bf16_to_f32(ww[j] & 0xFFFFu);
            wd[2 * j + 1] = (double)bf16_to_f32(ww[j] >> 16);
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if (t0 + q < T) {
              const uint32_t xw[4] = {xv[q].x, xv[q].y, xv[q].z, xv[q].w};
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                acc[q] = fma((double)bf16_to_f32(xw[j] & 0xFFFFu), wd[2 * j], acc[q]);
                acc[q] = fma((double)bf16_to_f32(xw[j] >> 16), wd[2 * j + 1], acc[q]);
              }
            }
          }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (t0 + q < T) {
            double a = acc[q];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
            if (lane == 0) red[warp * kMoeMaxTokens + t0 + q] = a;
          }
        }
      }
      __syncthreads();
      if (tid < T) {
        double a = 0.0;
        for (int w = 0; w < kFzWarps; ++w) a += red[w * kMoeMaxTokens + tid];
        p.logits[(size_t)tid * E + e] = __double2float_rn(a);
      }
      __syncthreads();
    }
  }
  if (busy == kFzWarps) load_tables(tid, blockDim.x);
  fz_stamp(p, kTrLogits);
  if (!fz_grid_barrier(p.bar, p.err, ok_s)) return;
  fz_stamp(p, kTrRouted);

  // --------------------------------------------------------- 2 selection
  int32_t *slots = reinterpret_cast<int32_t *>(smem + p.off_sel);                   // [T][k+1]
  float *slot_w = reinterpret_cast<float *>(slots + T * (k + 1));                   // [T][k]
  {
    // selection scratch in the staging area
    int32_t *sel_e = reinterpret_cast<int32_t *>(smem + p.off_stage);               // [T][k] rank order
    float *sel_sc = reinterpret_cast<float *>(sel_e + T * k);                       // [T][k] their scores
    uint32_t *mask_s = reinterpret_cast<uint32_t *>(sel_sc + T * k);                // [E+1]
    int *gidx_s = reinterpret_cast<int *>(mask_s + (E + 1));                        // [E+1]
    int *cnt_s = gidx_s + (E + 1);                                                  // [9]
    if (warp < T) {
      const int t = warp;
      uint32_t key[kFzChunks];
      float sc[kFzChunks];
#pragma unroll
      for (int c = 0; c < kFzChunks; ++c) {
        const int e = c * 32 + lane;
        key[c] = 0u;
        sc[c] = 0.f;
        if (e < E) {
          const FzScore r = fz_score(__ldcg(p.logits + (size_t)t * E + e), bias_s[e], p.mode);
          sc[c] = r.score;
          key[c] = r.key;
        }
      }
      // k rounds of arg-max over the experts not taken yet: the largest key,
      // the lowest index among equal keys (a lane's chunks ascend, so its
      // first best is its lowest)
      uint32_t taken = 0;
      for (int r = 0; r < k; ++r) {
        uint32_t bk = 0u;
        int be = 0x7FFFFFFF;
        float bs = 0.f;
#pragma unroll
        for (int c = 0; c < kFzChunks; ++c) {
          if (!((taken >> c) & 1u) && key[c] > bk) {
            bk = key[c];
            be = c * 32 + lane;
            bs = sc[c];
          }
        }
        const uint32_t kmax = __reduce_max_sync(0xffffffffu, bk);
        const int emin = (int)__reduce_min_sync(0xffffffffu, bk == kmax ? (unsigned)be : 0x7FFFFFFFu);
        const float ws = __shfl_sync(0xffffffffu, bs, emin & 31);
        if ((emin & 31) == lane) taken |= 1u << (emin >> 5);
        if (lane == 0) {
          sel_e[t * k + r] = emin;
          sel_sc[t * k + r] = ws;
        }
      }
      __syncwarp();
      if (lane < k) {
        const int r = lane;
        const float *ss = sel_sc + t * k;
        float w;
        if (p.mode == RC_ROUTER_SIGMOID_BIAS) {
          float sum = 0.f;
          for (int r2 = 0; r2 < k; ++r2) sum += ss[r2];
          w = ss[r];
          if (p.renorm) w = w / (sum + 1e-20f);
          w = w * p.scaling;
        } else {
          // softmax over all experts renormalised over the top-k equals the
          // softmax of the selected scores (the full denominator cancels)
          const float mx = ss[0];
          float sum = 0.f;
          for (int r2 = 0; r2 < k; ++r2) sum += expf(ss[r2] - mx);
          w = expf(ss[r] - mx) / sum;
        }
        const int e = sel_e[t * k + r];
        int pos = 0;
        for (int r2 = 0; r2 < k; ++r2) pos += sel_e[t * k + r2] < e ? 1 : 0;
        slots[t * (k + 1) + pos] = e;
        slot_w[t * k + pos] = w;
        if (blockIdx.x == 0) {
          if (p.ids_out) p.ids_out[t * k + r] = e;
          if (p.w_out) p.w_out[t * k + r] = w;
          if (p.slot_w_out) p.slot_w_out[t * k + pos] = w;
        }
      }
      if (lane == 0) slots[t * (k + 1) + k] = p.shared_id;
    }
    __syncthreads();
    fz_build_groups(slots, T, k, E, p.own, g_expert, g_mask, g_dst, n_groups_s, mask_s, gidx_s, cnt_s, p.err);
    for (int i = tid; i < *n_groups_s; i += blockDim.x) {
      g_gu[i] = all_gu[g_expert[i]];
      g_dn[i] = all_dn[g_expert[i]];
    }
    __syncthreads();
  }
  fz_stamp(p, kTrSelected);

  // ------------------------------------------------- partitions and ring
  const int ng = *n_groups_s;
  const int tot_gu = ng * gt_gu_i, tot_dn = ng * gt_dn_i;
  const int per_gu = (tot_gu + (int)gridDim.x - 1) / (int)gridDim.x;
  const int per_dn = (tot_dn + (int)gridDim.x - 1) / (int)gridDim.x;
  const int c0_gu = blockIdx.x * per_gu, c0_dn = blockIdx.x * per_dn;
  const int nt_gu = c0_gu < tot_gu ? (c0_gu + per_gu < tot_gu ? per_gu : tot_gu - c0_gu) : 0;
  const int nt_dn = c0_dn < tot_dn ? (c0_dn + per_dn < tot_dn ? per_dn : tot_dn - c0_dn) : 0;
  const int S = p.stages;
  const uint32_t bar0 = smem_addr(smem + p.off_bar) + warp * S * 8;
  // the two phases' ranges: per-CTA constants in shared memory (indexed by
  // the ring's current phase at run time)
  FzRange *ph = reinterpret_cast<FzRange *>(smem + p.off_red + kFzRedBytes + kEpMaxRanks * 8);
  if (tid == 0) {
    ph[0] = FzRange{g_gu, c0_gu, nt_gu, p.round_gu, kb_gu_i, make_fastdiv(gt_gu_i)};
    ph[1] = FzRange{g_dn, c0_dn, nt_dn, p.round_dn, kb_dn_i, make_fastdiv(gt_dn_i)};
  }
  __syncthreads();
  FzRing rg{};
  rg.iss.init(nt_gu, p.round_gu, kb_gu_i, kFzWarps, warp);
  rg.iss_phase = 0;
  while (rg.iss_phase < 2 && !rg.iss.valid()) {
    if (++rg.iss_phase < 2) rg.iss.init(nt_dn, p.round_dn, kb_dn_i, kFzWarps, warp);
  }
  if (lane == 0 && rg.iss_phase < 2) {
    const uint32_t ring_s = smem_addr(smem + warp * S * kUnitBytes);
    const uint64_t pol = policy_evict_first();
    for (int sl = 0; sl < S; ++sl) mbar_init(bar0 + 8 * sl, 1);
    mbar_fence_init();
    for (int sl = 0; sl < S && rg.iss_phase < 2; ++sl) fz_issue(rg, ph, warp, ring_s, bar0, pol, sl);
  }
  // expert parallelism: zero the slot rows other ranks compute
  if (p.zero_foreign) {
    const int rows = T * (k + 1);
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {
      const int t = r / (k + 1), pos = r - t * (k + 1);
      const int e = slots[r];
      const bool mine = pos < k ? (e >= p.own.lo && e < p.own.hi) : (e >= 0 && ((p.own.shared_mask >> t) & 1u));
      if (mine) continue;
      uint4 *dst = reinterpret_cast<uint4 *>(p.slot_rows + (size_t)r * p.hidden);
      for (int i = tid; i < p.hidden / 8; i += blockDim.x) dst[i] = make_uint4(0, 0, 0, 0);
    }
  }

  // ------------------------------------------------------------ 3 gate/up
  FzStage sx{p.x, RC_DTYPE_BF16, p.hidden, T, T, 1, kb_gu_i};
  build_activations<true, FzStage, kStageBf16Compact>(sx, NTB, reinterpret_cast<uint32_t *>(smem + p.off_stage),
                                                      smem + p.off_stage + xfrag_bytes(NTB, p.hidden), tid,
                                                      blockDim.x);
  __syncthreads();
  fz_stamp(p, kTrStaged);
  fz_phase<kFzGlu, NTB>(p, smem, ph, g_mask, g_dst, 0, rg);
  bool failed = __syncthreads_or(rg.failed) != 0;
  fz_stamp(p, kTrGateUp);
  if (!failed && !fz_grid_barrier(p.bar, p.err, ok_s)) failed = true;
  fz_stamp(p, kTrActReady);

  // --------------------------------------------------------------- 4 down
  if (!failed) {
    const int g_lo = c0_dn / gt_dn_i;
    const int g_hi = nt_dn ? (c0_dn + nt_dn - 1) / gt_dn_i : g_lo - 1;
    FzStage sa{p.act + (size_t)g_lo * 8 * NTB * p.inter_pad, RC_DTYPE_BF16, p.inter_pad,
               (g_hi - g_lo + 1) * 8 * NTB, (g_hi - g_lo + 1) * 8 * NTB, 1, kb_dn_i};
    build_activations<true, FzStage, kStageBf16Compact>(
        sa, NTB * kMoeMaxGroupsPerCta, reinterpret_cast<uint32_t *>(smem + p.off_stage),
        smem + p.off_stage + xfrag_bytes(NTB * kMoeMaxGroupsPerCta, p.inter_pad), tid, blockDim.x);
    __syncthreads();
    fz_phase<kFzDown, NTB>(p, smem, ph, g_mask, g_dst, g_lo, rg);
    failed = __syncthreads_or(rg.failed) != 0;
  }
  fz_stamp(p, kTrDown);
  if (p.ep_world > 1 && tid == 0) __threadfence_system();   // this CTA's rows to peers, before the barrier
  if (!failed && !fz_grid_barrier(p.bar, p.err, ok_s)) failed = true;
  if (p.ep_world > 1 && !failed) {
    // every rank's rows for this rank's tokens have been written once every
    // rank has passed its own barrier 3 and signalled
    if (blockIdx.x == 0 && tid == 0) {
      __threadfence_system();
      for (int r = 0; r < p.ep_world; ++r)
        red_add_release_sys(reinterpret_cast<unsigned long long *>(ep_peer_s[r]) + 1, 1ull);
    }
    if (!fz_wait_sys(p.ep_flags + 1, (ep_calls + 1) * p.ep_world, p.err, ok_s)) failed = true;
  }
  fz_stamp(p, kTrRows);

  // ------------------------------------------------------------ 5 combine
  if (!failed && p.out) {
    const int vecs = p.hidden / 8;
    const bool with_shared = p.shared_id >= 0 && p.own.shared_mask;
    const bool ep = p.ep_world > 1;
    const int n_out = ep ? p.ep_M : T;             // tokens combined here
    const uint16_t *ep_rows = ep ? reinterpret_cast<const uint16_t *>(ep_peer_s[p.ep_rank] + p.ep_red_off) : nullptr;
    for (int i = blockIdx.x * blockDim.x + tid; i < n_out * vecs; i += gridDim.x * blockDim.x) {
      const int to = i / vecs, v = i - to * vecs;      // output row
      const int t = ep ? p.ep_rank * p.ep_M + to : to;  // token of the call
      const uint16_t *rows = (ep ? ep_rows + (size_t)to * (k + 1) * p.hidden : p.slot_rows + (size_t)t * (k + 1) * p.hidden) +
                             (size_t)v * 8;
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
      for (int s = 0; s < k; ++s) {
        const uint4 r = __ldcg(reinterpret_cast<const uint4 *>(rows + (size_t)s * p.hidden));
        const float w = slot_w[t * k + s];
        const uint32_t q[4] = {r.x, r.y, r.z, r.w};
        // product rounded, then sum rounded (no fused multiply-add)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[2 * j] = __fadd_rn(acc[2 * j], __fmul_rn(bf16_to_f32(q[j] & 0xFFFFu), w));
          acc[2 * j + 1] = __fadd_rn(acc[2 * j + 1], __fmul_rn(bf16_to_f32(q[j] >> 16), w));
        }
      }
      const uint4 sh = with_shared ? __ldcg(reinterpret_cast<const uint4 *>(rows + (size_t)k * p.hidden))
                                   : make_uint4(0, 0, 0, 0);
      const uint32_t shw[4] = {sh.x, sh.y, sh.z, sh.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t lo = f32_to_bf16_rne(acc[2 * j]), hi = f32_to_bf16_rne(acc[2 * j + 1]);
        if (with_shared) {
          lo = f32_to_bf16_rne(bf16_to_f32(lo) + bf16_to_f32(shw[j] & 0xFFFFu));
          hi = f32_to_bf16_rne(bf16_to_f32(hi) + bf16_to_f32(shw[j] >> 16));
        }
        o[j] = lo | (hi << 16);
      }
      *reinterpret_cast<uint4 *>(p.out + (size_t)to * p.hidden + (size_t)v * 8) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  if (p.ep_world > 1 && !failed && blockIdx.x == 0 && tid == 0)
    *reinterpret_cast<volatile unsigned long long *>(p.ep_flags + 2) = ep_calls + 1;
  __syncthreads();
  fz_stamp(p, kTrEnd);
  // after a failure, the copies still in flight land before the CTA's shared
  // memory is released (ring indices consumed .. issued-1)
  if (failed && lane == 0) {
    for (int j = rg.consumed; j < rg.issued; ++j) mbar_wait_bounded(bar0 + 8 * (j % S), (uint32_t)(j / S) & 1u);
  }
}

// ------------------------------------------------------------------- host --
struct FzLayout {
  int stages, round_gu, round_dn, off_stage, off_part, off_tab, off_sel, off_red, off_bar, smem;
};

// The largest number of groups a call can have on this rank.
static int fz_max_groups(int T, int k, const MoeOwned &own) {
  const int owned = own.hi - own.lo;
  return (T * k < owned ? T * k : owned) + (own.shared_mask ? 1 : 0);
}

// Shared-memory layout of one call.  The deepest weight ring (up to 4 units
// per warp) comes first; the round partials hold at most the tiles a CTA can
// get in either phase, and shrink before the ring does.
static bool fz_layout(const rc_moe *m, int T, int k, const MoeOwned &own, FzLayout *L) {
  const int ntb = T <= 8 ? 1 : 2, E = m->n_experts, grid = m->ctx->sm_count;
  const int hidden = m->hidden, inter_pad = m->inter_pad;
  const int kb_gu = hidden / kUnitK, kb_dn = inter_pad / kUnitK;
  const int mg = fz_max_groups(T, k, own);
  const int per_gu = (mg * (m->inter / 8) + grid - 1) / grid;          // tiles per CTA, at most
  const int per_dn = (mg * (hidden / kUnitRows) + grid - 1) / grid;
  const size_t st_x = xfrag_bytes(ntb, hidden) + xaux_bytes(ntb, hidden);
  const size_t st_a = xfrag_bytes(ntb * kMoeMaxGroupsPerCta, inter_pad) + xaux_bytes(ntb * kMoeMaxGroupsPerCta,
                                                                                     inter_pad);
  const size_t st_sel = (size_t)T * k * 8 + (size_t)(E + 1) * 8 + 64;   // selection scratch
  size_t stage = st_x > st_a ? st_x : st_a;
  if (st_sel > stage) stage = st_sel;
  const size_t tab = (size_t)(E + 1) * (4 * 8 + 4 + 4 + 4 + 4 * T) + 16;   // expert and group tables
  const size_t sel = (size_t)T * (k + 1) * 4 + (size_t)T * k * 4;
  // + the barrier verdict word and the two phase ranges
  const size_t red = (size_t)kFzRedBytes + kEpMaxRanks * 8 + 2 * sizeof(FzRange);
  const int unit_part = ntb * 32 * 16;
  for (int S = kFzMaxStages; S >= 2; --S) {
    for (int cap = kMoePartialBytes; cap >= 4 * 1024; cap /= 2) {
      int R_gu = cap / (kb_gu * unit_part), R_dn = cap / (kb_dn * unit_part);
      if (R_gu < 1 || R_dn < 1) continue;
      if (R_gu > per_gu) R_gu = per_gu > 0 ? per_gu : 1;
      if (R_dn > per_dn) R_dn = per_dn > 0 ? per_dn : 1;
      const size_t part = (size_t)(R_gu * kb_gu > R_dn * kb_dn ? R_gu * kb_gu : R_dn * kb_dn) * unit_part;
      size_t off = (size_t)kFzWarps * S * kUnitBytes;
      const size_t o_stage = off;
      off += (stage + 15) / 16 * 16;
      const size_t o_part = off;
      off += part;
      const size_t o_tab = off;
      off += (tab + 15) / 16 * 16;
      const size_t o_sel = off;
      off += (sel + 15) / 16 * 16;
      const size_t o_red = off;
      off += red;
      const size_t o_bar = off;
      off += (size_t)kFzWarps * S * 8;
      if (off <= (size_t)kGemvSmemLimit) {
        *L = FzLayout{S, R_gu, R_dn, (int)o_stage, (int)o_part, (int)o_tab, (int)o_sel, (int)o_red, (int)o_bar,
                      (int)off};
        return true;
      }
    }
  }
  return false;
}

// Whether the fused kernel takes this call: it is switched on (rc_moe_set_fused)
// and the shape is one it can run.
bool moe_fused_fits(const rc_moe *m, int T, int k, const MoeOwned &own) {
  return m->fused && moe_persistent_shape_ok(m, T, k, own);
}

// Whether the fused kernel can run this shape: the shared-memory layout fits
// and a CTA's down range touches at most kMoeMaxGroupsPerCta groups.
bool moe_fused_shape_ok(const rc_moe *m, int T, int k, const MoeOwned &own) {
  if (m->down_fmt != kFormatQ4nx) return false;   // q4nx unit arithmetic only
  FzLayout L;
  if (!fz_layout(m, T, k, own, &L)) return false;
  const int max_groups = fz_max_groups(T, k, own);
  const int gt_dn = m->hidden / kUnitRows;
  const int per_dn = (max_groups * gt_dn + m->ctx->sm_count - 1) / m->ctx->sm_count;
  return per_dn - 1 <= (kMoeMaxGroupsPerCta - 1) * gt_dn;
}

// Runs the layer (out != null: combined rows into out) or its
// expert-parallel local half (out == null: slot rows, zeroed where another
// rank computes them, and the slot weights).  With ep, x is this rank's
// exchange buffer's token rows (every rank's tokens once the kernel has
// exchanged them), out this rank's own M rows.  The caller checked
// moe_fused_fits.
int moe_fused_decode(rc_moe *m, const uint16_t *x, int T, int k, int router, int renorm, float scaling, int act,
                     float gb, float vb, const MoeOwned &own, uint16_t *slot_rows, int zero_foreign, uint16_t *out,
                     int32_t *ids_out, float *w_out, float *slot_w_out, cudaStream_t s, const MoeEpArgs *ep) {
  const int ntb = T <= 8 ? 1 : 2;
  FzLayout L;
  if (!fz_layout(m, T, k, own, &L)) {
    set_error("fused MoE decode: no shared-memory layout for T=%d k=%d", T, k);
    return RC_ERR_INVALID;
  }
  rc_ctx *ctx = m->ctx;
  if (!m->fz_bar) {
    RC_CUDA_TRY(cudaMalloc(&m->fz_bar, sizeof(unsigned long long)));
    RC_CUDA_TRY(cudaMemset(m->fz_bar, 0, sizeof(unsigned long long)));
    m->fz_epoch = ctx->timeout_epoch;
  }
  if (m->fz_epoch != ctx->timeout_epoch) {
    // a bounded wait gave up since the last launch: the arrival count may be
    // left over from that launch
    RC_CUDA_TRY(cudaMemsetAsync(m->fz_bar, 0, sizeof(unsigned long long), s));
    m->fz_epoch = ctx->timeout_epoch;
  }
  MoeFusedParams p{};
  p.x = x;
  p.T = T;
  p.hidden = m->hidden;
  p.n_experts = m->n_experts;
  p.k = k;
  p.mode = router;
  p.renorm = renorm;
  p.scaling = scaling;
  p.wr = m->router_w;
  p.bias = m->router_bias;
  p.shared_id = m->has_shared ? m->n_experts : -1;
  p.own = own;
  p.logits = m->s.logits;
  p.ids_out = ids_out;
  p.w_out = w_out;
  p.slot_w_out = slot_w_out;
  p.gu_tiles = m->gu_tiles;
  p.dn_tiles = m->dn_tiles;
  p.inter = m->inter;
  p.inter_pad = m->inter_pad;
  p.act = m->act;
  p.slot_rows = slot_rows;
  p.zero_foreign = zero_foreign;
  p.out = out;
  p.act_kind = act;
  p.gate_beta = gb;
  p.value_beta = vb;
  p.stages = L.stages;
  p.round_gu = L.round_gu;
  p.round_dn = L.round_dn;
  p.off_stage = L.off_stage;
  p.off_part = L.off_part;
  p.off_tab = L.off_tab;
  p.off_sel = L.off_sel;
  p.off_red = L.off_red;
  p.off_bar = L.off_bar;
  p.bar = m->fz_bar;
  p.err = ctx->err;
  p.trace = m->trace;
  p.ep_world = 1;
  if (ep) {
    p.ep_world = ep->world;
    p.ep_rank = ep->rank;
    p.ep_M = ep->M;
    p.ep_peer = ep->peer_dev;
    p.ep_flags = ep->flags;
    p.ep_tok_off = ep->tok_off;
    p.ep_red_off = ep->red_off;
    p.ep_x_own = ep->x_own;
  }
  static bool configured[64][2] = {};
  int dev = 0;
  RC_CUDA_TRY(cudaGetDevice(&dev));
  if (dev >= 64 || !configured[dev][ntb - 1]) {
    if (ntb == 1)
      RC_CUDA_TRY(cudaFuncSetAttribute(rc_moe_fused_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kGemvSmemLimit));
    else
      RC_CUDA_TRY(cudaFuncSetAttribute(rc_moe_fused_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kGemvSmemLimit));
    if (dev < 64) configured[dev][ntb - 1] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctx->sm_count);
  cfg.blockDim = dim3(kFzThreads);
  cfg.dynamicSmemBytes = L.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;      // every CTA resident: the grid barriers are safe
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (ntb == 1)
    RC_CUDA_TRY(cudaLaunchKernelEx(&cfg, rc_moe_fused_kernel<1>, p));
  else
    RC_CUDA_TRY(cudaLaunchKernelEx(&cfg, rc_moe_fused_kernel<2>, p));
  return RC_OK;
}

}  // namespace rc
