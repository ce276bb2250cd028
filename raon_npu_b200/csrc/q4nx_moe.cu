// MoE decode on the q4nx experts: router top-k, grouped expert GEMVs with the
// GLU activation fused into the gate/up epilogue, and the ascending-expert-ID
// combine.  Everything stays on the device, so a layer is a fixed chain of
// launches (graph-capturable) with no host round trip between router and
// experts.
//
// Reference semantics (raon-npu):
//   router      host/raon.py:1224-1247 (sigmoid + bias) and the softmax top-k
//               of the north-star configs; lower expert index wins ties.
//   experts     host/backend.py:466-510: per expert gate/up linear (bf16),
//               act -> RTNE, down linear (bf16); f32 weighted sum over the
//               experts in ascending ID, then RTNE.
//   shared      host/raon.py:1310-1327: out = RTNE(f32(routed) + f32(shared)).
//
// Grouped GEMV partition: every warp owns whole row tiles (tiles w, w+W, ...
// of the slot-major tile list), so no tile is split and an expert's output is
// bit-identical whichever slots or ranks take part -- expert-parallel results
// equal single-GPU results byte for byte.
#include <string.h>

#include "q4nx_core.cuh"
#include "rc_device.cuh"
#include "rc_internal.cuh"

namespace rc {

constexpr int kMoeMaxK = 16;          // routed experts per token
constexpr int kMoeWarps = 8;
constexpr int kMoeMaxStages = 8;

struct rc_moe_impl;

// ----------------------------------------------------------------- router --
struct RouteParams {
  const uint16_t *x;       // [T][ldx] bf16
  int ldx, tokens, hidden, n_experts, k, mode, renorm;
  float scaling;
  const uint16_t *wr;      // [E][hidden] bf16
  const float *bias;       // [E] (sigmoid mode)
  float *logits;           // [T][E] f32 scratch (always written)
  int *counter;            // [T] arrival counters, zero between launches
  int32_t *ids;            // [T][k]   rank order (best first)
  float *weights;          // [T][k]
  int32_t *slot_expert;    // [T][k+1] ascending ID, then the shared expert (or -1)
  float *slot_w;           // [T][k]   weights in slot order
  int shared_id;           // expert id of the shared expert, -1 if none
};

constexpr int kRouteThreads = 256;
constexpr int kRouteExpertsPerCta = 8;   // one warp per expert

// Phase 1 (every CTA): logits of 8 experts for one token, f64 accumulation of
// exact bf16 x bf16 products, rounded once to f32.  Phase 2 (the last CTA of
// the token, by an arrival counter): top-k with "lower index wins" ties, the
// routing weights and the ascending-ID slot list.
__global__ void __launch_bounds__(kRouteThreads) moe_route_kernel(RouteParams p) {
  pdl_launch_dependents();
  pdl_wait_prior();
  const int t = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * kRouteExpertsPerCta + warp;
  const uint16_t *xr = p.x + (size_t)t * p.ldx;
  if (e < p.n_experts) {
    const uint16_t *wr = p.wr + (size_t)e * p.hidden;
    double acc = 0.0;
    for (int h = lane * 2; h < p.hidden; h += 64) {
      const uint32_t xv = *reinterpret_cast<const uint32_t *>(xr + h);
      const uint32_t wv = *reinterpret_cast<const uint32_t *>(wr + h);
      acc = fma((double)bf16_to_f32(xv & 0xFFFFu), (double)bf16_to_f32(wv & 0xFFFFu), acc);
      acc = fma((double)bf16_to_f32(xv >> 16), (double)bf16_to_f32(wv >> 16), acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) p.logits[(size_t)t * p.n_experts + e] = __double2float_rn(acc);
  }
  __threadfence();
  __syncthreads();
  __shared__ int is_last;
  if (threadIdx.x == 0) {
    const int old = atomicAdd(p.counter + t, 1);
    is_last = old == (int)gridDim.x - 1;
    if (is_last) atomicExch(p.counter + t, 0);
  }
  __syncthreads();
  if (!is_last || warp != 0) return;
  __threadfence();

  // ---- selection (one warp): value per expert, then k rounds of warp argmax
  const float *lg = p.logits + (size_t)t * p.n_experts;
  constexpr int kPer = 8;   // experts per lane (n_experts <= 256)
  float val[kPer], score[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int ei = lane + 32 * i;
    val[i] = -INFINITY;
    score[i] = 0.f;
    if (ei < p.n_experts) {
      const float l = __ldcg(lg + ei);
      if (p.mode == RC_ROUTER_SIGMOID_BIAS) {
        score[i] = __double2float_rn(1.0 / (1.0 + exp(-(double)l)));
        val[i] = score[i] + p.bias[ei];
      } else {
        score[i] = l;
        val[i] = l;
      }
    }
  }
  int sel[kMoeMaxK];
  float sel_score[kMoeMaxK];
  for (int r = 0; r < p.k; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int ei = lane + 32 * i;
      if (ei < p.n_experts && (val[i] > bv || (val[i] == bv && ei < bi))) bv = val[i], bi = ei;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) bv = ov, bi = oi;
    }
    sel[r] = bi;
    // the owner lane retires the winner and publishes its score
    float sc = 0.f;
#pragma unroll
    for (int i = 0; i < kPer; ++i)
      if (lane + 32 * i == bi) sc = score[i], val[i] = -INFINITY;
    sel_score[r] = __shfl_sync(0xffffffffu, sc, bi & 31);
  }
  if (lane != 0) return;
  // ---- routing weights
  float w[kMoeMaxK];
  if (p.mode == RC_ROUTER_SIGMOID_BIAS) {
    float sum = 0.f;
    for (int r = 0; r < p.k; ++r) sum += sel_score[r];
    for (int r = 0; r < p.k; ++r) {
      float c = sel_score[r];
      if (p.renorm) c = c / (sum + 1e-20f);
      w[r] = c * p.scaling;
    }
  } else {
    // softmax over all experts then renormalised over the top-k equals the
    // softmax of the selected logits (the full denominator cancels).
    const float mx = sel_score[0];
    float sum = 0.f;
    for (int r = 0; r < p.k; ++r) sum += expf(sel_score[r] - mx);
    for (int r = 0; r < p.k; ++r) w[r] = expf(sel_score[r] - mx) / sum;
  }
  for (int r = 0; r < p.k; ++r) {
    p.ids[(size_t)t * p.k + r] = sel[r];
    p.weights[(size_t)t * p.k + r] = w[r];
  }
  // ---- ascending-ID slot list (insertion sort of k <= 16 entries)
  int order[kMoeMaxK];
  for (int r = 0; r < p.k; ++r) order[r] = r;
  for (int a = 1; a < p.k; ++a) {
    const int v = order[a];
    int b = a - 1;
    while (b >= 0 && sel[order[b]] > sel[v]) {
      order[b + 1] = order[b];
      --b;
    }
    order[b + 1] = v;
  }
  int32_t *se = p.slot_expert + (size_t)t * (p.k + 1);
  float *sw = p.slot_w + (size_t)t * p.k;
  for (int r = 0; r < p.k; ++r) {
    se[r] = sel[order[r]];
    sw[r] = w[order[r]];
  }
  se[p.k] = p.shared_id;
}

// Slot list from caller-supplied top ids / weights (the Backend.moe_experts
// boundary): sort ascending by ID, append the shared expert.
__global__ void moe_slots_kernel(const int32_t *ids, const float *w, int k, int shared_id, int32_t *slot_expert,
                                 float *slot_w) {
  pdl_launch_dependents();
  pdl_wait_prior();
  if (threadIdx.x != 0) return;
  int order[kMoeMaxK];
  for (int r = 0; r < k; ++r) order[r] = r;
  for (int a = 1; a < k; ++a) {
    const int v = order[a];
    int b = a - 1;
    while (b >= 0 && ids[order[b]] > ids[v]) {
      order[b + 1] = order[b];
      --b;
    }
    order[b + 1] = v;
  }
  for (int r = 0; r < k; ++r) {
    slot_expert[r] = ids[order[r]];
    slot_w[r] = w[order[r]];
  }
  slot_expert[k] = shared_id;
}

// ------------------------------------------------------ grouped expert GEMV --
enum MoeEpi : int { kMoeEpiGlu = 0, kMoeEpiDown = 1 };

struct MoeGemvParams {
  const uint8_t *const *expert_tiles;  // per expert: t16 tiles, or null (not on this rank)
  const int32_t *slot_expert;          // [n_slots]: expert of each slot (-1: none)
  int n_slots;
  int slot_tiles;                      // row tiles per expert matrix
  int kb;                              // K / 256
  int stages;
  // activations (fields read by the shared staging code)
  const void *x;
  int x_dtype, ldx, tokens, slots, x_vec;
  // output
  uint16_t *y;
  long long y_slot_stride;             // elements between slots
  int ldy;                             // elements between token rows within a slot (glu)
  int act;
  float gate_beta, value_beta;
  int *err;
};

__device__ __forceinline__ const uint8_t *slot_base(const MoeGemvParams &p, int slot) {
  const int e = p.slot_expert[slot];
  return e < 0 ? nullptr : p.expert_tiles[e];
}

// EPI == kMoeEpiGlu: x = the token rows (shared by all slots); tile rows are
//   interleaved (gate g, up g) pairs; y[slot][t][8*tile + g] = bf16(act(gate, up)).
// EPI == kMoeEpiDown: x row s feeds slot s only (token block s/8, column s%8);
//   y[slot][row] = bf16(sum).
template <int EPI>
__global__ void __launch_bounds__(kMoeWarps * 32, 1) moe_gemv_kernel(MoeGemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb = p.kb, k = kb * kUnitK, S = p.stages;
  const int ntb = (p.slots + 7) >> 3;
  uint8_t *ring = smem + warp * S * kUnitBytes;
  const uint32_t ring_s = smem_addr(ring);
  uint8_t *cur = smem + kMoeWarps * S * kUnitBytes;
  uint32_t *xs = reinterpret_cast<uint32_t *>(cur);
  cur += xfrag_bytes(ntb, k);
  float *gs = reinterpret_cast<float *>(cur);
  cur += gsum_bytes(ntb, k);
  const uint32_t bar0 = smem_addr(cur) + warp * S * 8;

  const int W = gridDim.x * kMoeWarps;
  const int w = blockIdx.x * kMoeWarps + warp;
  const int total_tiles = p.n_slots * p.slot_tiles;
  const int my_tiles = w < total_tiles ? (total_tiles - 1 - w) / W + 1 : 0;
  const int n = my_tiles * kb;

  // unit j of this warp -> (slot, tile, kbi) and its source (null: skipped slot)
  auto unit_src = [&](int j) -> const uint8_t * {
    const int i = j / kb, kbi = j - i * kb;
    const int tg = w + i * W;
    const int slot = tg / p.slot_tiles, tile = tg - slot * p.slot_tiles;
    const uint8_t *b = slot_base(p, slot);
    return b ? b + ((size_t)tile * kb + kbi) * kUnitBytes : nullptr;
  };
  const uint64_t pol = policy_evict_first();
  auto issue = [&](int j, int sl) {
    const uint8_t *src = unit_src(j);
    if (src) {
      mbar_arrive_expect_tx(bar0 + 8 * sl, kUnitBytes);
      bulk_copy_g2s(ring_s + sl * kUnitBytes, src, kUnitBytes, bar0 + 8 * sl, pol);
    } else {
      mbar_arrive_expect_tx(bar0 + 8 * sl, 0);   // nothing to fetch: complete the phase at once
    }
  };
  pdl_launch_dependents();
  // The slot list is written by the previous launch (router / slot kernel):
  // wait before reading it.
  pdl_wait_prior();
  if (lane == 0 && n > 0) {
    for (int s = 0; s < S; ++s) mbar_init(bar0 + 8 * s, 1);
    mbar_fence_init();
    for (int j = 0; j < n && j < S; ++j) issue(j, j);
  }
  build_activations<true>(p, ntb, xs, gs, threadIdx.x, blockDim.x);
  __syncthreads();
  if (n == 0) return;

  Acc<1> acc;
  acc_zero(acc);
  int slot_ring = 0;
  uint32_t phase = 0;
  for (int j = 0; j < n; ++j) {
    const int i = j / kb, kbi = j - i * kb;
    const int tg = w + i * W;
    const int slot = tg / p.slot_tiles, tile = tg - slot * p.slot_tiles;
    const bool live = slot_base(p, slot) != nullptr;
    if (!mbar_wait_bounded(bar0 + 8 * slot_ring, phase)) {
      if (lane == 0) atomicCAS(p.err, 0, kErrWaitTimeout);
      int s2 = slot_ring;
      uint32_t ph2 = phase;
      for (int j2 = j + 1; j2 < n && j2 < j + S; ++j2) {
        if (++s2 == S) s2 = 0, ph2 ^= 1u;
        mbar_wait_bounded(bar0 + 8 * s2, ph2);
      }
      return;
    }
    if (live) {
      if (EPI == kMoeEpiGlu) {
        compute_unit<1, true>(ring + slot_ring * kUnitBytes, xs, gs, p, kbi, lane, acc);
      } else {
        const int tb = slot >> 3;   // token block holding this slot's activation row
        compute_unit<1, true>(ring + slot_ring * kUnitBytes, xs + (size_t)tb * (k / 64) * 256,
                              gs + (size_t)tb * kb * 64, p, kbi, lane, acc);
      }
    }
    __syncwarp();
    if (lane == 0 && j + S < n) issue(j + S, slot_ring);
    if (++slot_ring == S) slot_ring = 0, phase ^= 1u;
    if (kbi + 1 == kb) {
      // whole tile done: epilogue (skipped slots write zeros)
      const int g = lane >> 2, q = lane & 3;
      uint16_t *y = p.y + (size_t)slot * p.y_slot_stride;
      if (EPI == kMoeEpiGlu) {
        const int col = tile * 8 + g;
#pragma unroll
        for (int e2 = 0; e2 < 2; ++e2) {
          const int t = 2 * q + e2;
          if (t < p.tokens) {
            float v = 0.f;
            if (live) {
              const float gate = bf16_round(acc.v[0][e2]);
              const float up = bf16_round(acc.v[0][2 + e2]);
              v = p.act == RC_ACT_SITU ? act_situ(gate, up, p.gate_beta, p.value_beta) : act_swiglu(gate, up);
            }
            y[(size_t)t * p.ldy + col] = f32_to_bf16_rne(v);
          }
        }
      } else {
        const int c = slot & 7;
        if (q == (c >> 1)) {
          const int r0 = tile * kUnitRows + g;
          y[r0] = f32_to_bf16_rne(acc.v[0][c & 1]);
          y[r0 + 8] = f32_to_bf16_rne(acc.v[0][2 + (c & 1)]);
        }
      }
      acc_zero(acc);
    }
  }
}

// ---------------------------------------------------------------- combine --
// out = RTNE(sum_{slots in ascending ID} f32(down[s]) * w[s]); with a shared
// expert (slot k) out = RTNE(f32(out) + f32(down[k])).  routed_out (optional)
// receives the routed sum alone (the Backend.moe_experts contract).
__global__ void moe_combine_kernel(const uint16_t *down, long long slot_stride, const float *slot_w, int k,
                                   int with_shared, int hidden, uint16_t *out, uint16_t *routed_out) {
  pdl_launch_dependents();
  pdl_wait_prior();
  for (int h = blockIdx.x * blockDim.x + threadIdx.x; h < hidden; h += gridDim.x * blockDim.x) {
    float acc = 0.f;
    // product rounded, then sum rounded -- as the reference's f32 numpy update
    // (no fused multiply-add contraction)
    for (int s = 0; s < k; ++s)
      acc = __fadd_rn(acc, __fmul_rn(bf16_to_f32(down[(size_t)s * slot_stride + h]), slot_w[s]));
    const uint16_t routed = f32_to_bf16_rne(acc);
    if (routed_out) routed_out[h] = routed;
    if (out) {
      out[h] = with_shared ? f32_to_bf16_rne(bf16_to_f32(routed) + bf16_to_f32(down[(size_t)k * slot_stride + h]))
                           : routed;
    }
  }
}

}  // namespace rc

using namespace rc;

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
  // per-call scratch
  float *logits;              // [16][E]
  int *route_counter;         // [16]
  int32_t *ids, *slot_expert; // [16][kMax], [16][kMax+1]
  float *weights, *slot_w;
  uint16_t *act;              // [kMax+1][inter_pad]  (pad columns stay zero)
  uint16_t *down_out;         // [kMax+1][hidden]
};

namespace rc {

static int moe_stages(int ntb, int k, int units_per_warp) {
  int s = units_per_warp < 2 ? 2 : (units_per_warp > kMoeMaxStages ? kMoeMaxStages : units_per_warp);
  auto bytes = [&](int st) {
    return (size_t)kMoeWarps * st * (kUnitBytes + 8) + xfrag_bytes(ntb, k) + gsum_bytes(ntb, k);
  };
  while (s > 2 && bytes(s) > (size_t)kGemvSmemLimit) --s;
  return s;
}

template <int EPI>
static cudaError_t launch_moe_gemv(const rc_ctx *ctx, MoeGemvParams p, cudaStream_t s) {
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(moe_gemv_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvSmemLimit);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int total_tiles = p.n_slots * p.slot_tiles;
  int grid = (total_tiles + kMoeWarps - 1) / kMoeWarps;
  if (grid > ctx->sm_count) grid = ctx->sm_count;
  const int W = grid * kMoeWarps;
  const int tiles_per_warp = (total_tiles + W - 1) / W;
  const int ntb = (p.slots + 7) / 8;
  const int k = p.kb * kUnitK;
  p.stages = moe_stages(ntb, k, tiles_per_warp * p.kb);
  const size_t smem =
      (size_t)kMoeWarps * p.stages * (kUnitBytes + 8) + xfrag_bytes(ntb, k) + gsum_bytes(ntb, k);
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
  return cudaLaunchKernelEx(&cfg, moe_gemv_kernel<EPI>, p);
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

// Experts of one token for an already prepared slot list (slot_expert / slot_w
// on the device): gate/up GEMV with the GLU epilogue, then the down GEMV into
// down_out[slot].  n_slots = k (+1 with the shared expert).
static int moe_run_experts(rc_moe *m, const uint16_t *x, int n_slots, int act, float gb, float vb, cudaStream_t s) {
  MoeGemvParams g{};
  g.expert_tiles = m->gu_tiles;
  g.slot_expert = m->slot_expert;
  g.n_slots = n_slots;
  g.slot_tiles = m->inter / 8;              // interleaved gate/up: 8 intermediate columns per tile
  g.kb = m->hidden / kUnitK;
  g.x = x;
  g.x_dtype = RC_DTYPE_BF16;
  g.ldx = m->hidden;
  g.tokens = 1;
  g.slots = 1;
  g.x_vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (m->hidden * 2) % 16 == 0;
  g.y = m->act;
  g.y_slot_stride = m->inter_pad;
  g.ldy = m->inter_pad;
  g.act = act;
  g.gate_beta = gb;
  g.value_beta = vb;
  g.err = m->ctx->err;
  cudaError_t e = launch_moe_gemv<kMoeEpiGlu>(m->ctx, g, s);
  if (e != cudaSuccess) {
    set_error("moe gate/up launch: %s", cudaGetErrorString(e));
    return RC_ERR_CUDA;
  }
  MoeGemvParams d = g;
  d.expert_tiles = m->dn_tiles;
  d.slot_tiles = m->hidden / kUnitRows;
  d.kb = m->inter_pad / kUnitK;
  d.x = m->act;
  d.ldx = m->inter_pad;
  d.tokens = n_slots;
  d.slots = n_slots;
  d.x_vec = 1;
  d.y = m->down_out;
  d.y_slot_stride = m->hidden;
  d.ldy = m->hidden;
  e = launch_moe_gemv<kMoeEpiDown>(m->ctx, d, s);
  if (e != cudaSuccess) {
    set_error("moe down launch: %s", cudaGetErrorString(e));
    return RC_ERR_CUDA;
  }
  return RC_OK;
}

static int moe_combine(rc_moe *m, const uint16_t *down, const float *slot_w, int k, int with_shared, uint16_t *out,
                       uint16_t *routed_out, cudaStream_t s) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = small_cfg(dim3((m->hidden + 255) / 256), dim3(256), s, attr);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, moe_combine_kernel, down, (long long)m->hidden, slot_w, k,
                                           with_shared, m->hidden, out, routed_out);
  if (e != cudaSuccess) {
    set_error("moe combine launch: %s", cudaGetErrorString(e));
    return RC_ERR_CUDA;
  }
  return RC_OK;
}

static int moe_route(rc_moe *m, const uint16_t *x, int T, int k, int mode, int renorm, float scaling,
                     cudaStream_t s) {
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
  r.logits = m->logits;
  r.counter = m->route_counter;
  r.ids = m->ids;
  r.weights = m->weights;
  r.slot_expert = m->slot_expert;
  r.slot_w = m->slot_w;
  r.shared_id = m->has_shared ? m->n_experts : -1;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = small_cfg(
      dim3((m->n_experts + kRouteExpertsPerCta - 1) / kRouteExpertsPerCta, T), dim3(kRouteThreads), s, attr);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, moe_route_kernel, r);
  if (e != cudaSuccess) {
    set_error("moe router launch: %s", cudaGetErrorString(e));
    return RC_ERR_CUDA;
  }
  return RC_OK;
}

}  // namespace rc

extern "C" {

int rc_moe_create(rc_ctx *ctx, int hidden, int inter, int n_experts, int has_shared, rc_moe **out) {
  RC_CHECK_ARG(ctx && out, "rc_moe_create: NULL argument");
  *out = nullptr;
  RC_CHECK_ARG(hidden > 0 && hidden % 256 == 0, "hidden (%d) must be a multiple of 256", hidden);
  RC_CHECK_ARG(inter > 0 && inter % 64 == 0, "intermediate size (%d) must be a multiple of 64", inter);
  RC_CHECK_ARG(n_experts > 0 && n_experts <= 256, "n_experts (%d) must be in 1..256", n_experts);
  RC_CUDA_TRY(cudaSetDevice(ctx->device));
  rc_moe *m = new rc_moe();
  m->ctx = ctx;
  m->hidden = hidden;
  m->inter = inter;
  m->inter_pad = (inter + 255) / 256 * 256;
  m->n_experts = n_experts;
  m->has_shared = has_shared ? 1 : 0;
  const int ne = n_experts + 1;
  m->gate_up = new rc_weight *[ne]();
  m->down = new rc_weight *[ne]();
  cudaError_t e = cudaMalloc(&m->gu_tiles, ne * sizeof(void *));
  if (e == cudaSuccess) e = cudaMalloc(&m->dn_tiles, ne * sizeof(void *));
  if (e == cudaSuccess) e = cudaMemset(m->gu_tiles, 0, ne * sizeof(void *));
  if (e == cudaSuccess) e = cudaMemset(m->dn_tiles, 0, ne * sizeof(void *));
  if (e == cudaSuccess) e = cudaMalloc(&m->router_w, (size_t)n_experts * hidden * 2);
  if (e == cudaSuccess) e = cudaMalloc(&m->router_bias, (size_t)n_experts * 4);
  if (e == cudaSuccess) e = cudaMemset(m->router_bias, 0, (size_t)n_experts * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->logits, (size_t)kMoeMaxK * n_experts * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->route_counter, kMoeMaxK * 4);
  if (e == cudaSuccess) e = cudaMemset(m->route_counter, 0, kMoeMaxK * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->ids, kMoeMaxK * kMoeMaxK * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->weights, kMoeMaxK * kMoeMaxK * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->slot_expert, kMoeMaxK * (kMoeMaxK + 1) * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->slot_w, kMoeMaxK * kMoeMaxK * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->act, (size_t)(kMoeMaxK + 1) * m->inter_pad * 2);
  if (e == cudaSuccess) e = cudaMemset(m->act, 0, (size_t)(kMoeMaxK + 1) * m->inter_pad * 2);
  if (e == cudaSuccess) e = cudaMalloc(&m->down_out, (size_t)(kMoeMaxK + 1) * hidden * 2);
  if (e != cudaSuccess) {
    set_error("rc_moe_create: %s", cudaGetErrorString(e));
    rc_moe_destroy(m);
    return RC_ERR_CUDA;
  }
  *out = m;
  return RC_OK;
}

int rc_moe_destroy(rc_moe *m) {
  if (!m) return RC_OK;
  cudaSetDevice(m->ctx->device);
  cudaDeviceSynchronize();
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
  cudaFree(m->logits);
  cudaFree(m->route_counter);
  cudaFree(m->ids);
  cudaFree(m->weights);
  cudaFree(m->slot_expert);
  cudaFree(m->slot_w);
  cudaFree(m->act);
  cudaFree(m->down_out);
  delete m;
  return RC_OK;
}

int rc_moe_set_expert(rc_moe *m, int expert, const uint8_t *gate_up, size_t gate_up_bytes, const uint8_t *down,
                      size_t down_bytes, unsigned flags) {
  RC_CHECK_ARG(m && gate_up && down, "rc_moe_set_expert: NULL argument");
  RC_CHECK_ARG(expert >= 0 && expert <= m->n_experts, "expert id %d out of range 0..%d", expert, m->n_experts);
  RC_CHECK_ARG(expert < m->n_experts || m->has_shared, "this MoE layer has no shared expert");
  RC_CHECK_ARG((flags & ~(unsigned)RC_UPLOAD_SRC_DEVICE) == 0, "rc_moe_set_expert: unknown flags 0x%x", flags);
  rc_weight *gu = nullptr, *dn = nullptr;
  int rc = rc_upload_q4nx(m->ctx, gate_up, gate_up_bytes, 2 * m->inter, m->hidden, flags | RC_UPLOAD_GATE_UP, &gu);
  if (rc) return rc;
  rc = rc_upload_q4nx(m->ctx, down, down_bytes, m->hidden, m->inter_pad, flags, &dn);
  if (rc) {
    rc_weight_free(gu);
    return rc;
  }
  if (m->gate_up[expert]) rc_weight_free(m->gate_up[expert]);
  if (m->down[expert]) rc_weight_free(m->down[expert]);
  m->gate_up[expert] = gu;
  m->down[expert] = dn;
  RC_CUDA_TRY(cudaMemcpy(m->gu_tiles + expert, &gu->tiles, sizeof(void *), cudaMemcpyHostToDevice));
  RC_CUDA_TRY(cudaMemcpy(m->dn_tiles + expert, &dn->tiles, sizeof(void *), cudaMemcpyHostToDevice));
  return RC_OK;
}

int rc_moe_set_router(rc_moe *m, const uint16_t *router_w, const float *bias) {
  RC_CHECK_ARG(m && router_w, "rc_moe_set_router: NULL argument");
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  RC_CUDA_TRY(cudaMemcpy(m->router_w, router_w, (size_t)m->n_experts * m->hidden * 2, cudaMemcpyHostToDevice));
  if (bias) RC_CUDA_TRY(cudaMemcpy(m->router_bias, bias, (size_t)m->n_experts * 4, cudaMemcpyHostToDevice));
  return RC_OK;
}

int rc_moe_route(rc_moe *m, const uint16_t *x_dev, int T, int k, int router, int renormalize, float scaling,
                 int32_t *ids_dev, float *w_dev, float *logits_dev, void *stream) {
  RC_CHECK_ARG(m && x_dev, "rc_moe_route: NULL argument");
  RC_CHECK_ARG(T >= 1 && T <= kMoeMaxK, "rc_moe_route: T must be 1..%d", kMoeMaxK);
  RC_CHECK_ARG(k >= 1 && k <= kMoeMaxK && k <= m->n_experts, "rc_moe_route: k must be 1..%d", kMoeMaxK);
  RC_CHECK_ARG(router == RC_ROUTER_SOFTMAX || router == RC_ROUTER_SIGMOID_BIAS, "unknown router %d", router);
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  const cudaStream_t s = pick_stream(m->ctx, stream);
  int rc = moe_route(m, x_dev, T, k, router, renormalize, scaling, s);
  if (rc) return rc;
  if (ids_dev) RC_CUDA_TRY(cudaMemcpyAsync(ids_dev, m->ids, (size_t)T * k * 4, cudaMemcpyDeviceToDevice, s));
  if (w_dev) RC_CUDA_TRY(cudaMemcpyAsync(w_dev, m->weights, (size_t)T * k * 4, cudaMemcpyDeviceToDevice, s));
  if (logits_dev)
    RC_CUDA_TRY(cudaMemcpyAsync(logits_dev, m->logits, (size_t)T * m->n_experts * 4, cudaMemcpyDeviceToDevice, s));
  return RC_OK;
}

int rc_moe_experts(rc_moe *m, const uint16_t *x_dev, const int32_t *ids_dev, const float *w_dev, int k, int act,
                   float gate_beta, float value_beta, int with_shared, uint16_t *out_dev, void *stream) {
  RC_CHECK_ARG(m && x_dev && ids_dev && w_dev && out_dev, "rc_moe_experts: NULL argument");
  RC_CHECK_ARG(k >= 1 && k <= kMoeMaxK, "rc_moe_experts: k must be 1..%d", kMoeMaxK);
  RC_CHECK_ARG(act == RC_ACT_SWIGLU || act == RC_ACT_SITU, "unknown activation %d", act);
  RC_CHECK_ARG(!with_shared || m->has_shared, "this MoE layer has no shared expert");
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  const cudaStream_t s = pick_stream(m->ctx, stream);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = small_cfg(dim3(1), dim3(32), s, attr);
  RC_CUDA_TRY(cudaLaunchKernelEx(&cfg, moe_slots_kernel, ids_dev, w_dev, k, with_shared ? m->n_experts : -1,
                                 m->slot_expert, m->slot_w));
  int rc = moe_run_experts(m, x_dev, k + (with_shared ? 1 : 0), act, gate_beta, value_beta, s);
  if (rc) return rc;
  return moe_combine(m, m->down_out, m->slot_w, k, with_shared, out_dev, nullptr, s);
}

int rc_moe_experts_host(rc_moe *m, const uint16_t *x_host, const int32_t *ids_host, const float *w_host, int k,
                        int act, float gate_beta, float value_beta, int with_shared, uint16_t *out_host) {
  RC_CHECK_ARG(m && x_host && ids_host && w_host && out_host, "rc_moe_experts_host: NULL argument");
  RC_CHECK_ARG(k >= 1 && k <= kMoeMaxK, "rc_moe_experts_host: k must be 1..%d", kMoeMaxK);
  for (int r = 0; r < k; ++r) {
    RC_CHECK_ARG(ids_host[r] >= 0 && ids_host[r] < m->n_experts, "expert id %d out of range 0..%d", ids_host[r],
                 m->n_experts - 1);
    RC_CHECK_ARG(m->gate_up[ids_host[r]] != nullptr, "expert %d is not loaded", ids_host[r]);
  }
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  rc_ctx *ctx = m->ctx;
  const size_t xb = (size_t)m->hidden * 2 + kMoeMaxK * 8, yb = (size_t)m->hidden * 2;
  int rc = ensure_host_staging(ctx, xb, yb);
  if (rc) return rc;
  uint8_t *px = static_cast<uint8_t *>(ctx->pin_x);
  memcpy(px, x_host, (size_t)m->hidden * 2);
  memcpy(px + (size_t)m->hidden * 2, ids_host, (size_t)k * 4);
  memcpy(px + (size_t)m->hidden * 2 + kMoeMaxK * 4, w_host, (size_t)k * 4);
  uint8_t *dx = static_cast<uint8_t *>(ctx->dev_x);
  RC_CUDA_TRY(cudaMemcpyAsync(dx, px, xb, cudaMemcpyHostToDevice, ctx->stream));
  rc = rc_moe_experts(m, reinterpret_cast<const uint16_t *>(dx),
                      reinterpret_cast<const int32_t *>(dx + (size_t)m->hidden * 2),
                      reinterpret_cast<const float *>(dx + (size_t)m->hidden * 2 + kMoeMaxK * 4), k, act, gate_beta,
                      value_beta, with_shared, static_cast<uint16_t *>(ctx->dev_y), nullptr);
  if (rc) return rc;
  RC_CUDA_TRY(cudaMemcpyAsync(ctx->pin_y, ctx->dev_y, yb, cudaMemcpyDeviceToHost, ctx->stream));
  RC_CUDA_TRY(cudaStreamSynchronize(ctx->stream));
  rc = check_error_word(ctx);
  if (rc) return rc;
  memcpy(out_host, ctx->pin_y, yb);
  return RC_OK;
}

int rc_moe_decode(rc_moe *m, const uint16_t *x_dev, int k, int router, int renormalize, float scaling, int act,
                  float gate_beta, float value_beta, uint16_t *out_dev, int32_t *ids_dev, float *w_dev,
                  void *stream) {
  RC_CHECK_ARG(m && x_dev && out_dev, "rc_moe_decode: NULL argument");
  RC_CHECK_ARG(k >= 1 && k <= kMoeMaxK && k <= m->n_experts, "rc_moe_decode: k must be 1..%d", kMoeMaxK);
  RC_CHECK_ARG(act == RC_ACT_SWIGLU || act == RC_ACT_SITU, "unknown activation %d", act);
  RC_CHECK_ARG(router == RC_ROUTER_SOFTMAX || router == RC_ROUTER_SIGMOID_BIAS, "unknown router %d", router);
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  const cudaStream_t s = pick_stream(m->ctx, stream);
  int rc = moe_route(m, x_dev, 1, k, router, renormalize, scaling, s);
  if (rc) return rc;
  rc = moe_run_experts(m, x_dev, k + m->has_shared, act, gate_beta, value_beta, s);
  if (rc) return rc;
  rc = moe_combine(m, m->down_out, m->slot_w, k, m->has_shared, out_dev, nullptr, s);
  if (rc) return rc;
  if (ids_dev) RC_CUDA_TRY(cudaMemcpyAsync(ids_dev, m->ids, (size_t)k * 4, cudaMemcpyDeviceToDevice, s));
  if (w_dev) RC_CUDA_TRY(cudaMemcpyAsync(w_dev, m->weights, (size_t)k * 4, cudaMemcpyDeviceToDevice, s));
  return RC_OK;
}

int rc_moe_decode_local(rc_moe *m, const uint16_t *x_dev, int k, int router, int renormalize, float scaling, int act,
                        float gate_beta, float value_beta, uint16_t *slot_out_dev, float *slot_w_dev,
                        void *stream) {
  RC_CHECK_ARG(m && x_dev && slot_out_dev && slot_w_dev, "rc_moe_decode_local: NULL argument");
  RC_CHECK_ARG(k >= 1 && k <= kMoeMaxK && k <= m->n_experts, "rc_moe_decode_local: k must be 1..%d", kMoeMaxK);
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  const cudaStream_t s = pick_stream(m->ctx, stream);
  int rc = moe_route(m, x_dev, 1, k, router, renormalize, scaling, s);
  if (rc) return rc;
  rc = moe_run_experts(m, x_dev, k + m->has_shared, act, gate_beta, value_beta, s);
  if (rc) return rc;
  const int slots = k + m->has_shared;
  RC_CUDA_TRY(cudaMemcpyAsync(slot_out_dev, m->down_out, (size_t)slots * m->hidden * 2, cudaMemcpyDeviceToDevice, s));
  RC_CUDA_TRY(cudaMemcpyAsync(slot_w_dev, m->slot_w, (size_t)k * 4, cudaMemcpyDeviceToDevice, s));
  return RC_OK;
}

int rc_moe_combine(rc_moe *m, const uint16_t *slot_out_dev, const float *slot_w_dev, int k, int with_shared,
                   uint16_t *out_dev, void *stream) {
  RC_CHECK_ARG(m && slot_out_dev && slot_w_dev && out_dev, "rc_moe_combine: NULL argument");
  RC_CHECK_ARG(k >= 1 && k <= kMoeMaxK, "rc_moe_combine: k must be 1..%d", kMoeMaxK);
  RC_CHECK_ARG(!with_shared || m->has_shared, "this MoE layer has no shared expert");
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  return moe_combine(m, slot_out_dev, slot_w_dev, k, with_shared, out_dev, nullptr, pick_stream(m->ctx, stream));
}

}  // extern "C"
