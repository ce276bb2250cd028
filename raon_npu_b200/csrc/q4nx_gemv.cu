// q4nx weight-dequant-fused GEMV for T = 1..16 token rows (decode).
//
// Arithmetic.  For output row n and 32-column group g,
//     y[t,n] = sum_g scale[n,g] * D[t,n,g] + min[n,g] * S[t,g]
// with D = sum code*x over the group and S = sum x over the group -- the same
// factorisation the reference's NPU kernel uses (kernels/gemv/q4nx_gemv.cc:88-124),
// but with every product and partial sum kept in f32 (the reference's CPU
// oracle, host/backend.py:402-417, multiplies the f32-dequantised weights).
// Both terms run on the tensor cores (q4nx_core.cuh): codes as exact f16
// subnormals against block-scaled f16 activations, the min term as a K = 8
// contraction over the groups.
//
// Streaming.  A grid of at most one CTA per SM splits the matrix's units (16
// rows x 256 columns, 2560 B).  Two partitions, chosen from (N, K, SM count):
//   whole tiles: CTA c owns the row tiles [c*NT/G, (c+1)*NT/G).  Warp w takes
//     the tiles w, w+W, ... in chunks processed k-block by k-block (one
//     k-block's activation fragments in registers, one register accumulator
//     per tile) and finalises them itself; the last NT % W tiles run as
//     rounds whose units are spread over all warps, reduced in shared memory.
//   stream-K (a few tall tiles): all units split evenly over the grid in
//     contiguous ranges; split tiles reduced through global partials (the
//     last warp to arrive, by a per-tile counter, sums them and resets it).
// A tile's pieces are summed in a fixed order.  Each warp owns a ring of
// 2..12 units in shared memory fed by 1-D bulk copies (cp.async.bulk +
// mbarrier, L2 evict-first); for small matrices the ring holds the warp's
// whole range, so every byte is requested up front.  The partition and the
// order of every sum never depend on T, so a row's result is independent of
// the batch.
//
// Activations.  Each CTA stages the T x K activations once in shared memory,
// already permuted into mma B-fragment order, together with the group-sum
// fragments and block scales.  (For K too large to stage, a small prep kernel
// writes the same layout to global scratch and the unit loop reads it through
// the read-only path.)
//
// Launch chaining.  The kernel uses programmatic dependent launch: it issues
// its first weight copies while the previous kernel in the stream is still
// running and only waits (griddepcontrol.wait) before it reads activations or
// touches scratch, so back-to-back GEMVs overlap their HBM traffic.
#include <string.h>

#include <mutex>

#include "q4nx_core.cuh"
#include "rc_device.cuh"
#include "rc_internal.cuh"

namespace rc {

enum GemvEpilogue : int {
  kEpiBf16 = 0,   // y[t][n] = bf16_rne(acc + bias)
  kEpiF32 = 1,    // token slots (2t, 2t+1) carry the hi/lo bf16 split of an f32 row
  kEpiGlu = 2,    // unit rows (g, g+8) are (gate, up): y[t][8*tile+g] = bf16(act(bf16 g, bf16 u))
  kEpiF32Raw = 3, // bf16 activations, unrounded f32 output
};

struct GemvParams {
  const uint8_t *tiles;    // first unit of the row range, t16 layout
  int n_tiles;             // row tiles (16 rows) in the range
  int kb;                  // K / 256
  int active_warps;        // stream-K partition: warps that own units (<= units)
  int mode;                // GemvPartition
  int round_tiles;         // CTA-tile partition: tiles per reduction round
  int warps;               // warps per CTA (8 or 16)
  int stages;              // weight ring depth per warp
  int slots;               // token slots holding data (bf16: T, f32: 2T); others are never read back
  // activations: raw (staged path) ...
  const void *x;
  int x_dtype;
  int ldx;
  int tokens;              // real token rows (bf16/glu: <= 16, f32: <= 8)
  int x_vec;               // x rows 16-byte aligned: vector loads allowed
  // ... or pre-permuted in global scratch (large-K path)
  const uint32_t *xfrag;
  const void *aux;
  void *y;
  int ldy;
  const float *bias;       // f32 per row of the range, or null
  float *partials;
  int *counters;
  int *err;
  int act;
  float gate_beta, value_beta;
};

// Large-K path: the activations go to global scratch in the same layout.
__global__ void rc_gemv_prep_kernel(GemvParams p, int ntb, uint32_t *xfrag, void *aux) {
  pdl_launch_dependents();
  pdl_wait_prior();
  build_activations<false>(p, ntb, xfrag, aux, blockIdx.x * (long long)blockDim.x + threadIdx.x,
                           (long long)gridDim.x * blockDim.x);
}

// --------------------------------------------------------- main kernel --
// Balanced split of ``units`` over ``parts``: part i owns [i*U/P, (i+1)*U/P).
// 32-bit arithmetic; the host guarantees units * parts < 2^32.
__device__ __forceinline__ uint32_t split_start(uint32_t i, uint32_t units, uint32_t parts) {
  return i * units / parts;
}
// The part whose range contains unit u (all ranges non-empty: parts <= units).
__device__ __forceinline__ uint32_t split_owner(uint32_t u, uint32_t units, uint32_t parts) {
  return ((u + 1) * parts + units - 1) / units - 1;
}

template <int NTB, int EPI>
__device__ __forceinline__ void finalize_tile(const GemvParams &p, uint32_t tile, int lane, const Acc<NTB> &a) {
  const int g = lane >> 2, q = lane & 3;
  const int r0 = (int)tile * kUnitRows + g, r1 = r0 + 8;
#pragma unroll
  for (int tb = 0; tb < NTB; ++tb) {
    const int t0 = tb * 8 + 2 * q;
    // The bias is added only when present (no +0.0 that would turn -0.0 into +0.0).
    if (EPI == kEpiBf16 || EPI == kEpiF32Raw) {
      float v00 = a.v[tb][0], v01 = a.v[tb][1], v10 = a.v[tb][2], v11 = a.v[tb][3];
      if (p.bias) {
        const float b0 = p.bias[r0], b1 = p.bias[r1];
        v00 += b0;
        v01 += b0;
        v10 += b1;
        v11 += b1;
      }
      if (EPI == kEpiBf16) {
        uint16_t *y = static_cast<uint16_t *>(p.y);
        if (t0 < p.tokens) {
          y[(size_t)t0 * p.ldy + r0] = f32_to_bf16_rne(v00);
          y[(size_t)t0 * p.ldy + r1] = f32_to_bf16_rne(v10);
        }
        if (t0 + 1 < p.tokens) {
          y[(size_t)(t0 + 1) * p.ldy + r0] = f32_to_bf16_rne(v01);
          y[(size_t)(t0 + 1) * p.ldy + r1] = f32_to_bf16_rne(v11);
        }
      } else {
        float *y = static_cast<float *>(p.y);
        if (t0 < p.tokens) {
          y[(size_t)t0 * p.ldy + r0] = v00;
          y[(size_t)t0 * p.ldy + r1] = v10;
        }
        if (t0 + 1 < p.tokens) {
          y[(size_t)(t0 + 1) * p.ldy + r0] = v01;
          y[(size_t)(t0 + 1) * p.ldy + r1] = v11;
        }
      }
    } else if (EPI == kEpiF32) {
      float *y = static_cast<float *>(p.y);
      const int t = tb * 4 + q;
      if (t < p.tokens) {
        float v0 = a.v[tb][0] + a.v[tb][1], v1 = a.v[tb][2] + a.v[tb][3];
        if (p.bias) {
          v0 += p.bias[r0];
          v1 += p.bias[r1];
        }
        y[(size_t)t * p.ldy + r0] = v0;
        y[(size_t)t * p.ldy + r1] = v1;
      }
    } else {
      uint16_t *y = static_cast<uint16_t *>(p.y);
      const int col = (int)tile * 8 + g;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = t0 + e;
        if (t < p.tokens) {
          const float gate = bf16_round(a.v[tb][e]);
          const float up = bf16_round(a.v[tb][2 + e]);
          const float v = p.act == RC_ACT_SITU ? act_situ(gate, up, p.gate_beta, p.value_beta) : act_swiglu(gate, up);
          y[(size_t)t * p.ldy + col] = f32_to_bf16_rne(v);
        }
      }
    }
  }
}

// Global stream-K split tile: store this warp's partial; the last of the
// tile's warps to arrive (per-tile counter) sums all partials in warp order.
template <int NTB, int EPI>
__device__ void flush_split_global(const GemvParams &p, uint32_t tile, int slot, uint32_t gw, uint32_t units,
                                   int lane, const Acc<NTB> &acc) {
  const uint32_t W = (uint32_t)p.active_warps;
  float4 *part = reinterpret_cast<float4 *>(p.partials);
#pragma unroll
  for (int tb = 0; tb < NTB; ++tb)
    part[((gw * 2 + slot) * 2 + tb) * 32 + lane] = make_float4(acc.v[tb][0], acc.v[tb][1], acc.v[tb][2], acc.v[tb][3]);
  __threadfence();
  __syncwarp();
  const uint32_t first = tile * p.kb, last = first + p.kb - 1;
  const uint32_t w_first = split_owner(first, units, W), w_last = split_owner(last, units, W);
  int is_last = 0;
  if (lane == 0) {
    const int old = atomicAdd(p.counters + tile, 1);
    is_last = (old == (int)(w_last - w_first));
    if (is_last) atomicExch(p.counters + tile, 0);
  }
  is_last = __shfl_sync(0xffffffffu, is_last, 0);
  if (!is_last) return;
  __threadfence();
  Acc<NTB> sum;
  acc_zero(sum);
  // Up to 8/NTB pieces' loads in flight before they are added, in warp order.
  constexpr int kBatch = 8 / NTB;
  for (uint32_t w0 = w_first; w0 <= w_last; w0 += kBatch) {
    float4 v[kBatch][NTB];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const uint32_t w2 = w0 + i;
      if (w2 > w_last) break;
      const int s2 = (tile == split_start(w2, units, W) / p.kb) ? 0 : 1;
#pragma unroll
      for (int tb = 0; tb < NTB; ++tb)
        v[i][tb] = w2 == gw ? make_float4(acc.v[tb][0], acc.v[tb][1], acc.v[tb][2], acc.v[tb][3])
                            : __ldcg(part + ((w2 * 2 + s2) * 2 + tb) * 32 + lane);
    }
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      if (w0 + i > w_last) break;
      acc_add(sum, v[i]);
    }
  }
  finalize_tile<NTB, EPI>(p, tile, lane, sum);
}


// Partitions (chosen on the host from the shape and SM count only):
//   kPartTiles:   CTA c owns whole row tiles [c*NT/G, (c+1)*NT/G); its warps
//                 split that unit range evenly; a tile shared by several warps
//                 is reduced in shared memory after a CTA barrier.
//   kPartStreamK: warps split all units evenly across the grid; tiles shared
//                 by several warps are reduced through global partials.
enum GemvPartition : int { kPartTiles = 0, kPartStreamK = 1 };

// kPartTiles: CTA c owns the whole tiles [c*NT/G, (c+1)*NT/G), nt of them.
//   Main phase: warp w takes the whole tiles w, w+W, w+2W, ... (nt/W each, W
//   warps) in chunks of up to kChunk tiles; a chunk runs k-block by k-block,
//   so the warp loads a k-block's activation fragments once per chunk, adds
//   each unit's result into its tile's register accumulator and finalises its
//   own tiles -- no barrier, no shared partials.
//   Remainder: the last nt % W tiles in rounds (RoundCursor): unit results in
//   shared partials, summed per tile in k-block order after a barrier.
// Either way a tile's result is the sum of its units' results in k-block
// order, so it does not depend on the partition.
template <int NTB>
struct GemvChunk {
  static constexpr int kChunk = NTB == 1 ? 4 : 1;          // tiles per chunk (register accumulators)
};

// A warp's main-phase units in processing order: chunk, k-block, tile.
struct ChunkCursor {
  int per_warp, kb, W, w;
  int chunk, kbi, c, cn;
  __device__ __forceinline__ void init(int per_warp_, int kb_, int W_, int w_, int C) {
    per_warp = per_warp_, kb = kb_, W = W_, w = w_;
    chunk = 0, kbi = 0, c = 0;
    cn = per_warp < C ? per_warp : C;
  }
  __device__ __forceinline__ bool valid() const { return cn > 0; }
  __device__ __forceinline__ int tile(int C) const { return w + (chunk * C + c) * W; }
  __device__ __forceinline__ void next(int C) {
    if (++c < cn) return;
    c = 0;
    if (++kbi < kb) return;
    kbi = 0;
    ++chunk;
    const int left = per_warp - chunk * C;
    cn = left <= 0 ? 0 : (left < C ? left : C);
  }
};

template <int NTB, int EPI, bool STAGED>
__device__ __forceinline__ void gemv_rounds(const GemvParams &p, uint8_t *smem) {
  constexpr int C = GemvChunk<NTB>::kChunk;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  const int kb = p.kb, k = kb * kUnitK, S = p.stages, R = p.round_tiles;
  const int t0 = (int)((long long)blockIdx.x * p.n_tiles / gridDim.x);
  const int t1 = (int)((long long)(blockIdx.x + 1) * p.n_tiles / gridDim.x);
  const int nt = t1 - t0;
  const int per_warp = nt / nw, n_main = per_warp * nw, n_rem = nt - n_main;

  // shared memory: weight rings | activations | aux | round partials | barriers
  uint8_t *ring = smem + warp * S * kUnitBytes;
  const uint32_t ring_s = smem_addr(ring);
  uint8_t *sp = smem + nw * S * kUnitBytes;
  uint32_t *xs = reinterpret_cast<uint32_t *>(sp);
  if (STAGED) sp += xfrag_bytes(NTB, k);
  void *xa = sp;
  if (STAGED) sp += xaux_bytes(NTB, k);
  float4 *part = reinterpret_cast<float4 *>(sp);           // [R*kb][NTB][32 lanes]
  sp += (size_t)R * kb * NTB * 32 * sizeof(float4);
  const uint32_t bar0 = smem_addr(sp) + warp * S * 8;

  // the issue cursor: main-phase units, then the remainder's (lane 0)
  ChunkCursor im;
  im.init(per_warp, kb, nw, warp, C);
  RoundCursor ir;
  ir.init(n_rem, R, kb, nw, warp);
  const uint64_t pol = policy_evict_first();
  int issued = 0;
  auto issue = [&](int sl) {
    int tile, kbi;
    if (im.valid()) {
      tile = im.tile(C), kbi = im.kbi;
      im.next(C);
    } else {
      tile = n_main + ir.tile(), kbi = ir.kbi;
      ir.next();
    }
    mbar_arrive_expect_tx(bar0 + 8 * sl, kUnitBytes);
    bulk_copy_g2s(ring_s + sl * kUnitBytes, p.tiles + ((size_t)(t0 + tile) * kb + kbi) * kUnitBytes, kUnitBytes,
                  bar0 + 8 * sl, pol);
    ++issued;
  };
  const bool any = im.valid() || ir.valid();
  if (lane == 0 && any) {
    for (int sl = 0; sl < S; ++sl) mbar_init(bar0 + 8 * sl, 1);
    mbar_fence_init();
    for (int sl = 0; sl < S && (im.valid() || ir.valid()); ++sl) issue(sl);
  }
  pdl_launch_dependents();
  // Weights are in flight; now wait for the producer of x (and for any earlier
  // launch that shares the scratch) before touching anything it wrote.
  pdl_wait_prior();
  if (STAGED) {
    build_activations<true>(p, NTB, xs, xa, threadIdx.x, blockDim.x);
    __syncthreads();
  }
  const uint32_t *xf = STAGED ? xs : p.xfrag;
  const void *auxp = STAGED ? xa : p.aux;

  int j = 0, slot = 0, j_fail = 0;
  uint32_t phase = 0;
  bool failed = false;
  XFrag<NTB> xr;
  auto wait_unit = [&]() {
    if (!failed && !mbar_wait_bounded_warp(bar0 + 8 * slot, phase)) {
      if (lane == 0) atomicCAS(p.err, 0, kErrWaitTimeout);
      failed = true;
      j_fail = j;
    }
  };
  auto release_unit = [&]() {
    __syncwarp();
    if (!failed && lane == 0 && (im.valid() || ir.valid())) issue(slot);
    if (++slot == S) slot = 0, phase ^= 1u;
    ++j;
  };

  // ---- main phase
  for (int chunk = 0; chunk * C < per_warp; ++chunk) {
    const int cn = per_warp - chunk * C < C ? per_warp - chunk * C : C;
    Acc<NTB> acc[C];
#pragma unroll
    for (int c = 0; c < C; ++c) acc_zero(acc[c]);
    for (int kbi = 0; kbi < kb; ++kbi) {
      load_xfrag<NTB, STAGED>(xr, xf, auxp, NTB, 0, kb, kbi, lane);
#pragma unroll
      for (int c = 0; c < C; ++c) {
        if (c < cn) {
          wait_unit();
          if (!failed) unit_accumulate<NTB>(ring + slot * kUnitBytes, xr, lane, acc[c]);
          release_unit();
        }
      }
    }
    if (!failed) {
#pragma unroll
      for (int c = 0; c < C; ++c)
        if (c < cn) finalize_tile<NTB, EPI>(p, (uint32_t)(t0 + warp + (chunk * C + c) * nw), lane, acc[c]);
    }
  }

  // ---- remainder rounds
  RoundCursor cur;
  cur.init(n_rem, R, kb, nw, warp);
  const int n_rounds = round_count(n_rem, R);
  int xr_kbi = -1;
  for (int r = 0; r < n_rounds; ++r) {
    for (; cur.valid() && cur.round == r; cur.next()) {
      wait_unit();
      if (!failed) {
        if (cur.kbi != xr_kbi) {
          load_xfrag<NTB, STAGED>(xr, xf, auxp, NTB, 0, kb, cur.kbi, lane);
          xr_kbi = cur.kbi;
        }
        float4 Q[NTB];
        unit_result<NTB>(ring + slot * kUnitBytes, xr, lane, Q);
        float4 *dst = part + (size_t)cur.slot() * NTB * 32 + lane;
#pragma unroll
        for (int tb = 0; tb < NTB; ++tb) dst[tb * 32] = Q[tb];
      }
      release_unit();
    }
    __syncthreads();
    const int t_lo = r * R, t_hi = t_lo + R < n_rem ? t_lo + R : n_rem;
    for (int ti = t_lo + warp; ti < t_hi; ti += nw) {
      Acc<NTB> acc;
      acc_zero(acc);
      const float4 *src = part + (size_t)(ti - t_lo) * kb * NTB * 32 + lane;
      for (int kbi = 0; kbi < kb; ++kbi) {
        float4 v[NTB];
#pragma unroll
        for (int tb = 0; tb < NTB; ++tb) v[tb] = src[(kbi * NTB + tb) * 32];
        acc_add(acc, v);
      }
      finalize_tile<NTB, EPI>(p, (uint32_t)(t0 + n_main + ti), lane, acc);
    }
    __syncthreads();
  }
  // after a timeout, wait (bounded) for the copies still in flight before the
  // CTA's shared memory is released
  if (failed && lane == 0) {
    for (int jj = j_fail; jj < issued; ++jj) mbar_wait_bounded(bar0 + 8 * (jj % S), (uint32_t)(jj / S) & 1u);
  }
}

template <int NTB, int EPI, bool STAGED>
__global__ void __launch_bounds__(kGemvMaxWarps * 32, 1) rc_q4nx_gemv_kernel(GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  if (p.mode == kPartTiles) {
    gemv_rounds<NTB, EPI, STAGED>(p, smem);
    return;
  }
  // kPartStreamK: the warps of the grid split all units evenly (contiguous
  // ranges, k-block fastest); tiles shared by several warps are reduced
  // through global partials.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t kb = (uint32_t)p.kb;
  const int k = p.kb * kUnitK;
  uint32_t ub = 0, ue = 0;
  const uint32_t units = (uint32_t)p.n_tiles * kb;
  const int nw = blockDim.x >> 5;              // 8 or 16 warps
  const uint32_t gw = blockIdx.x * nw + warp;
  if (gw < (uint32_t)p.active_warps) {
    ub = split_start(gw, units, p.active_warps);
    ue = split_start(gw + 1, units, p.active_warps);
  }
  const int n = (int)(ue - ub);

  // ---- shared memory: weight rings | activations | aux | barriers
  const int S = p.stages;
  uint8_t *ring = smem + warp * S * kUnitBytes;
  const uint32_t ring_s = smem_addr(ring);
  uint8_t *cur_p = smem + nw * S * kUnitBytes;
  uint32_t *xs = reinterpret_cast<uint32_t *>(cur_p);
  if (STAGED) cur_p += xfrag_bytes(NTB, k);
  void *xa = cur_p;
  if (STAGED) cur_p += xaux_bytes(NTB, k);
  const uint32_t bar0 = smem_addr(cur_p) + warp * S * 8;

  const uint64_t pol = policy_evict_first();
  if (lane == 0 && n > 0) {
    for (int s = 0; s < S; ++s) mbar_init(bar0 + 8 * s, 1);
    mbar_fence_init();
    for (int j = 0; j < n && j < S; ++j) {
      mbar_arrive_expect_tx(bar0 + 8 * j, kUnitBytes);
      bulk_copy_g2s(ring_s + j * kUnitBytes, p.tiles + (size_t)(ub + j) * kUnitBytes, kUnitBytes, bar0 + 8 * j, pol);
    }
  }
  pdl_launch_dependents();
  // Weights are in flight; now wait for the producer of x (and for any earlier
  // launch that shares the scratch) before touching anything it wrote.
  pdl_wait_prior();
  if (STAGED) {
    build_activations<true>(p, NTB, xs, xa, threadIdx.x, blockDim.x);
    __syncthreads();
  }
  if (n == 0) return;
  const uint32_t *xf = STAGED ? xs : p.xfrag;
  const void *auxp = STAGED ? xa : p.aux;
  Acc<NTB> acc;
  acc_zero(acc);
  XFrag<NTB> xr;
  uint32_t tile = ub / kb, kbi = ub - tile * kb;
  uint32_t seg_k0 = kbi;     // first k-block of the current tile segment
  int seg = 0;               // 0 = the warp's first tile segment
  int slot = 0;
  uint32_t phase = 0;        // parity of the ring slot's current fill
  for (int j = 0; j < n; ++j) {
    if (!mbar_wait_bounded_warp(bar0 + 8 * slot, phase)) {
      if (lane == 0) atomicCAS(p.err, 0, kErrWaitTimeout);
      // Let the copies already issued (this unit's included) land before the
      // CTA's shared memory goes away.
      int s2 = slot;
      uint32_t ph2 = phase;
      for (int j2 = j; j2 < n && j2 < j + S; ++j2) {
        mbar_wait_bounded(bar0 + 8 * s2, ph2);
        if (++s2 == S) s2 = 0, ph2 ^= 1u;
      }
      return;
    }
    load_xfrag<NTB, STAGED>(xr, xf, auxp, NTB, 0, p.kb, (int)kbi, lane);
    unit_accumulate<NTB>(ring + slot * kUnitBytes, xr, lane, acc);
    __syncwarp();
    if (lane == 0 && j + S < n) {
      mbar_arrive_expect_tx(bar0 + 8 * slot, kUnitBytes);
      bulk_copy_g2s(ring_s + slot * kUnitBytes, p.tiles + (size_t)(ub + j + S) * kUnitBytes, kUnitBytes,
                    bar0 + 8 * slot, pol);
    }
    if (++slot == S) slot = 0, phase ^= 1u;
    const bool tile_end = kbi + 1 == kb;
    if (tile_end || j + 1 == n) {
      if (seg_k0 == 0 && tile_end)
        finalize_tile<NTB, EPI>(p, tile, lane, acc);
      else
        flush_split_global<NTB, EPI>(p, tile, seg ? 1 : 0, gw, units, lane, acc);
      acc_zero(acc);
      ++tile;
      kbi = 0;
      seg_k0 = 0;
      seg = 1;
    } else {
      ++kbi;
    }
  }
}

// ------------------------------------------------------------------ host --
constexpr int kGemvRoundBytes = 32 * 1024;   // round partials of the CTA-tile partition

// Tiles per round of the CTA-tile partition's remainder (the nt % W tiles
// left after the warps' whole tiles): no more than any CTA's remainder, and
// a round's unit partials fit kGemvRoundBytes (a function of the shape and
// T; results do not depend on it).
static int gemv_round_tiles(int ntb, int kb, int n_tiles, int grid, int warps) {
  const int lo = n_tiles / grid, hi = (n_tiles + grid - 1) / grid;   // CTA ranges hold lo or hi tiles
  int rem = hi % warps > lo % warps ? hi % warps : lo % warps;
  if (rem < 1) rem = 1;
  int r = kGemvRoundBytes / (kb * ntb * 32 * 16);
  if (r < 1) r = 1;
  return r < rem ? r : rem;
}

static size_t gemv_smem_bytes(int ntb, int k, bool staged, int stages, int nw, int round_tiles) {
  size_t b = (size_t)nw * stages * (kUnitBytes + 8);
  b += (size_t)round_tiles * (k / kUnitK) * ntb * 32 * 16;   // round partials (CTA-tile partition)
  if (staged) b += xfrag_bytes(ntb, k) + xaux_bytes(ntb, k);
  return b;
}

// Ring depth: deep enough to cover a warp's whole range for small matrices
// (everything requested at once), bounded by shared memory for large ones.
// Small rings keep the footprint low so consecutive launches can co-reside
// on an SM under programmatic dependent launch.
static int gemv_stages(int ntb, int k, bool staged, long long units_per_warp, int nw, int round_tiles) {
  int s = (int)(units_per_warp < 2 ? 2 : (units_per_warp > kGemvMaxStages ? kGemvMaxStages : units_per_warp));
  while (s > 2 && gemv_smem_bytes(ntb, k, staged, s, nw, round_tiles) > (size_t)kGemvSmemLimit) --s;
  return s;
}

static cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, size_t smem, cudaStream_t s, cudaLaunchAttribute *attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

template <int NTB, int EPI, bool STAGED>
static cudaError_t launch_main(const GemvParams &p, int grid, cudaStream_t s) {
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(rc_q4nx_gemv_kernel<NTB, EPI, STAGED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kGemvSmemLimit);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_config(dim3(grid), dim3(p.warps * 32),
                                      gemv_smem_bytes(NTB, p.kb * kUnitK, STAGED, p.stages, p.warps, p.round_tiles),
                                      s, attr);
  return cudaLaunchKernelEx(&cfg, rc_q4nx_gemv_kernel<NTB, EPI, STAGED>, p);
}

template <int NTB, bool STAGED>
static cudaError_t launch_epi(const GemvParams &p, int epi, int grid, cudaStream_t s) {
  switch (epi) {
    case kEpiBf16: return launch_main<NTB, kEpiBf16, STAGED>(p, grid, s);
    case kEpiF32: return launch_main<NTB, kEpiF32, STAGED>(p, grid, s);
    case kEpiF32Raw: return launch_main<NTB, kEpiF32Raw, STAGED>(p, grid, s);
    default: return launch_main<NTB, kEpiGlu, STAGED>(p, grid, s);
  }
}

// Grid of the persistent kernel for a given unit count: a function of the
// matrix shape and SM count only (never of T), so results are batch-invariant.
//
// Whole-tile CTA ranges are used when they balance the SMs within 25% (their
// split tiles reduce in shared memory); otherwise -- few tall tiles -- all
// units are split evenly over the grid's warps (global stream-K).
struct GemvGeometry {
  int mode, grid, warps, active_warps;
  long long units_per_warp;
  int tiles_per_cta;   // kPartTiles: the largest CTA range (0 for stream-K)
};

// Large matrices (>= 16 units per warp at 8 warps per SM) run one CTA of 16
// warps per SM, sharing one copy of the staged activations: latency hiding
// limits their stream.  Smaller ones run 8-warp CTAs, which leaves room for
// the next launch's CTA to co-reside under programmatic dependent launch.
GemvGeometry gemv_geometry(const rc_ctx *ctx, int n_tiles, int kb, int max_warps) {
  GemvGeometry g{};
  const long long units = (long long)n_tiles * kb;
  const long long sm = ctx->sm_count;
  const int nw = (units >= 16ll * kGemvWarps * sm && max_warps >= kGemvMaxWarps) ? kGemvMaxWarps : kGemvWarps;
  g.warps = nw;
  const long long gt = n_tiles < sm ? n_tiles : sm;
  const long long tiles_per_cta = (n_tiles + gt - 1) / gt;
  const bool balanced = tiles_per_cta * gt * 4 <= (long long)n_tiles * 5;
  const bool fits32 = units * (long long)(sm * nw) < (1ll << 32);
  if (balanced || !fits32) {
    g.mode = kPartTiles;
    g.grid = (int)gt;
    g.tiles_per_cta = (int)tiles_per_cta;
    g.active_warps = (int)(gt * nw);
    const long long cta_units = tiles_per_cta * kb;
    g.units_per_warp = (cta_units + nw - 1) / nw;
  } else {
    long long gr = (units + nw - 1) / nw;
    if (gr > sm) gr = sm;
    long long w = gr * nw;
    if (w > units) w = units;
    g.mode = kPartStreamK;
    g.grid = (int)gr;
    g.active_warps = (int)w;
    g.units_per_warp = (units + w - 1) / w;
  }
  return g;
}

// Whether ntb token blocks of K columns fit in shared memory next to the rings of nw warps.
static bool gemv_can_stage(int ntb, int k, int nw) {
  return gemv_smem_bytes(ntb, k, true, 2, nw, 1) <= (size_t)kGemvSmemLimit;
}

// One launch over <= 16 bf16 token rows (<= 8 f32 rows).
int gemv_launch(rc_ctx *ctx, const uint8_t *tiles, int n_tiles, int k, const void *x, int x_dtype, int ldx,
                int tokens, void *y, int ldy, const float *bias, int epi, int act, float gb, float vb,
                cudaStream_t s) {
  const int slots = x_dtype == RC_DTYPE_F32 ? 2 * tokens : tokens;
  const int ntb = slots > 8 ? 2 : 1;
  // The geometry must not depend on T (batch invariance): 16-warp CTAs only
  // where even two token blocks can be staged next to their rings.  Staging
  // itself may still fall back to global scratch; that changes no arithmetic.
  const GemvGeometry geo =
      gemv_geometry(ctx, n_tiles, k / kUnitK, gemv_can_stage(2, k, kGemvMaxWarps) ? kGemvMaxWarps : kGemvWarps);
  // Per-CTA staging repeats the whole of x in every CTA: worth it while that
  // work (items per thread) is at most twice a warp's units (measured on B200:
  // 2048x4096, 4096x2048 and 512x2048 at T = 1..16); otherwise one prep launch
  // spread over the grid stages x once (its launch overlaps the weight
  // prefetch under programmatic dependent launch).  Either way the fragments,
  // and so the results, are the same.
  const long long stage_items = (long long)slots * (k / 8) / (geo.warps * 32);
  const bool staged = gemv_can_stage(ntb, k, geo.warps) && stage_items <= 2 * geo.units_per_warp;
  int rc = ensure_gemv_scratch(ctx, staged ? 0 : k, n_tiles);
  if (rc) return rc;
  GemvParams p{};
  p.tiles = tiles;
  p.n_tiles = n_tiles;
  p.kb = k / kUnitK;
  p.x = x;
  p.x_dtype = x_dtype;
  p.ldx = ldx;
  p.tokens = tokens;
  p.slots = slots;
  const size_t esz = x_dtype == RC_DTYPE_F32 ? 4 : 2;
  p.x_vec = ((reinterpret_cast<uintptr_t>(x) & 15) == 0 && ((size_t)ldx * esz) % 16 == 0) ? 1 : 0;
  p.y = y;
  p.ldy = ldy;
  p.bias = bias;
  p.partials = ctx->partials;
  p.counters = ctx->counters;
  p.err = ctx->err;
  p.act = act;
  p.gate_beta = gb;
  p.value_beta = vb;
  cudaError_t e;
  if (!staged) {
    const unsigned xs = ctx->launch_seq++ % kXSlots;
    p.xfrag = ctx->xfrag + xs * xfrag_slot_words(ctx->xfrag_k);
    p.aux = ctx->gsum + xs * gsum_slot_floats(ctx->xfrag_k);
    const long long work = (long long)p.slots * (k / 8);
    long long pg = (work + 255) / 256;
    if (pg > ctx->sm_count) pg = ctx->sm_count;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pdl_config(dim3((unsigned)pg), dim3(256), 0, s, attr);
    e = cudaLaunchKernelEx(&cfg, rc_gemv_prep_kernel, p, ntb, const_cast<uint32_t *>(p.xfrag),
                           const_cast<void *>(p.aux));
    if (e != cudaSuccess) {
      set_error("gemv prep launch: %s", cudaGetErrorString(e));
      return RC_ERR_CUDA;
    }
  }
  const int grid = geo.grid;
  p.mode = geo.mode;
  p.warps = geo.warps;
  p.active_warps = geo.active_warps;
  p.round_tiles = geo.mode == kPartTiles ? gemv_round_tiles(ntb, k / kUnitK, n_tiles, geo.grid, geo.warps) : 0;
  p.stages = gemv_stages(ntb, k, staged, geo.units_per_warp, geo.warps, p.round_tiles);
  if (staged)
    e = ntb == 2 ? launch_epi<2, true>(p, epi, grid, s) : launch_epi<1, true>(p, epi, grid, s);
  else
    e = ntb == 2 ? launch_epi<2, false>(p, epi, grid, s) : launch_epi<1, false>(p, epi, grid, s);
  if (e != cudaSuccess) {
    set_error("gemv launch: %s", cudaGetErrorString(e));
    return RC_ERR_CUDA;
  }
  return RC_OK;
}

// ------------------------------------------------- allocation-free variant --
// Scratch of rc_gemv_noalloc: the per-tile arrival counters and the per-warp
// split-K partials of the stream-K partition, in one statically sized device
// array that every GPU loading this library holds until the process exits.
constexpr int kNoAllocMaxTiles = 16384;               // 262,144 output rows
constexpr int kNoAllocMaxWarps = 160 * kGemvMaxWarps; // 160 SMs x 16 warps
constexpr size_t kNoAllocCounterBytes = (size_t)kNoAllocMaxTiles * sizeof(int);
constexpr size_t kNoAllocPartialBytes = (size_t)kNoAllocMaxWarps * 2 * 2 * 32 * 4 * sizeof(float);
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocCounterBytes + kNoAllocPartialBytes];

// Device address of g_noalloc_scratch per device.  In host code the array's
// name is only a host-side stand-in, so the address comes from
// cudaGetSymbolAddress, looked up once per device with that device current.
static std::mutex g_noalloc_mu;
static void *g_noalloc_addr[64];

static int noalloc_scratch(int device, unsigned char **out) {
  RC_CHECK_ARG(device >= 0 && device < 64, "rc_gemv_noalloc: device %d out of range", device);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[device]) {
    void *ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || !ptr) {
      set_error("rc_gemv_noalloc: cudaGetSymbolAddress of the static scratch failed on device %d: %s", device,
                cudaGetErrorString(e));
      return RC_ERR_CUDA;
    }
    g_noalloc_addr[device] = ptr;
  }
  *out = static_cast<unsigned char *>(g_noalloc_addr[device]);
  return RC_OK;
}

// One launch of the GEMV kernel with its scratch in the static array: the same
// geometry and kernel as gemv_launch, restricted to shapes whose activations
// stage in shared memory (so no global activation scratch is needed).
static int gemv_launch_noalloc(rc_ctx *ctx, unsigned char *scratch, const uint8_t *tiles, int n_tiles, int k,
                               const void *x, int x_dtype, int ldx, int tokens, void *y, int ldy, const float *bias,
                               int epi, cudaStream_t s) {
  const int slots = x_dtype == RC_DTYPE_F32 ? 2 * tokens : tokens;
  const int ntb = slots > 8 ? 2 : 1;
  const GemvGeometry geo =
      gemv_geometry(ctx, n_tiles, k / kUnitK, gemv_can_stage(2, k, kGemvMaxWarps) ? kGemvMaxWarps : kGemvWarps);
  RC_CHECK_ARG(gemv_can_stage(ntb, k, geo.warps),
               "rc_gemv_noalloc: K=%d with %d token rows per launch does not fit in shared memory "
               "(use fewer rows per call, or rc_gemv)", k, tokens);
  RC_CHECK_ARG(geo.mode == kPartTiles || geo.active_warps <= kNoAllocMaxWarps,
               "rc_gemv_noalloc: %d warps exceed the static scratch (%d)", geo.active_warps, kNoAllocMaxWarps);
  int *counters = reinterpret_cast<int *>(scratch);
  // Every call shares the array and it keeps the last call's contents; the
  // counters must start at zero (a call that gave up a wait can leave them set).
  RC_CUDA_TRY(cudaMemsetAsync(counters, 0, (size_t)n_tiles * sizeof(int), s));
  GemvParams p{};
  p.tiles = tiles;
  p.n_tiles = n_tiles;
  p.kb = k / kUnitK;
  p.x = x;
  p.x_dtype = x_dtype;
  p.ldx = ldx;
  p.tokens = tokens;
  p.slots = slots;
  const size_t esz = x_dtype == RC_DTYPE_F32 ? 4 : 2;
  p.x_vec = ((reinterpret_cast<uintptr_t>(x) & 15) == 0 && ((size_t)ldx * esz) % 16 == 0) ? 1 : 0;
  p.y = y;
  p.ldy = ldy;
  p.bias = bias;
  p.partials = reinterpret_cast<float *>(scratch + kNoAllocCounterBytes);
  p.counters = counters;
  p.err = ctx->err;
  p.mode = geo.mode;
  p.warps = geo.warps;
  p.active_warps = geo.active_warps;
  p.round_tiles = geo.mode == kPartTiles ? gemv_round_tiles(ntb, k / kUnitK, n_tiles, geo.grid, geo.warps) : 0;
  p.stages = gemv_stages(ntb, k, true, geo.units_per_warp, geo.warps, p.round_tiles);
  const cudaError_t e =
      ntb == 2 ? launch_epi<2, true>(p, epi, geo.grid, s) : launch_epi<1, true>(p, epi, geo.grid, s);
  if (e != cudaSuccess) {
    set_error("rc_gemv_noalloc launch: %s", cudaGetErrorString(e));
    return RC_ERR_CUDA;
  }
  return RC_OK;
}

}  // namespace rc

using namespace rc;

extern "C" {

int rc_gemv(rc_ctx *ctx, const rc_weight *w, const void *x_dev, int x_dtype, int ldx, int T, void *y_dev,
            int y_dtype, int ldy, int row0, int nrows, const float *bias_dev, void *stream) {
  RC_CHECK_ARG(ctx && x_dev && y_dev, "rc_gemv: NULL argument");
  if (!w) {
    set_error("rc_gemv: unknown weight handle");
    return RC_ERR_NOT_FOUND;
  }
  RC_CHECK_ARG(!(w->flags & RC_UPLOAD_GATE_UP), "rc_gemv: a gate/up-interleaved matrix is only usable by the MoE path");
  RC_CHECK_ARG(x_dtype == RC_DTYPE_BF16 || x_dtype == RC_DTYPE_F32, "rc_gemv: x_dtype must be BF16 or F32");
  RC_CHECK_ARG(y_dtype == RC_DTYPE_F32 || (y_dtype == RC_DTYPE_BF16 && x_dtype == RC_DTYPE_BF16),
               "rc_gemv: y_dtype must be F32, or BF16 with BF16 activations");
  RC_CHECK_ARG(T >= 1, "rc_gemv: T must be >= 1 (got %d)", T);
  RC_CHECK_ARG(row0 >= 0 && nrows > 0 && row0 % kUnitRows == 0 && nrows % kUnitRows == 0 && row0 + nrows <= w->n,
               "rc_gemv: rows [%d, %d) must be 16-aligned inside [0, %d)", row0, row0 + nrows, w->n);
  RC_CHECK_ARG(ldx >= w->k, "rc_gemv: ldx (%d) < K (%d)", ldx, w->k);
  RC_CHECK_ARG(ldy >= nrows, "rc_gemv: ldy (%d) < nrows (%d)", ldy, nrows);
  RC_CUDA_TRY(cudaSetDevice(ctx->device));
  const cudaStream_t s = pick_stream(ctx, stream);
  if (w->format == kFormatBfp16) {
    RC_CHECK_ARG(x_dtype == RC_DTYPE_BF16, "rc_gemv: a bfp16ebs8 matrix takes bf16 activations");
    RC_CHECK_ARG((ldx % 8) == 0 && (reinterpret_cast<uintptr_t>(x_dev) & 15) == 0,
                 "rc_gemv: bfp16ebs8 activations must be 16-byte aligned rows (ldx a multiple of 8)");
    return bfp16_gemv(ctx, w, static_cast<const uint16_t *>(x_dev), ldx, T, y_dev, y_dtype, ldy, row0, nrows,
                      bias_dev ? bias_dev + row0 : nullptr, s);
  }
  const int per = x_dtype == RC_DTYPE_F32 ? kMaxTokensPerLaunch / 2 : kMaxTokensPerLaunch;
  const size_t xe = x_dtype == RC_DTYPE_F32 ? 4 : 2;
  const size_t ye = y_dtype == RC_DTYPE_F32 ? 4 : 2;
  const int epi = x_dtype == RC_DTYPE_F32 ? kEpiF32 : (y_dtype == RC_DTYPE_F32 ? kEpiF32Raw : kEpiBf16);
  const uint8_t *tiles = w->tiles + (size_t)(row0 / kUnitRows) * (w->k / kUnitK) * kUnitBytes;
  const float *bias = bias_dev ? bias_dev + row0 : nullptr;
  for (int t0 = 0; t0 < T; t0 += per) {
    const int tc = T - t0 < per ? T - t0 : per;
    const void *xc = static_cast<const uint8_t *>(x_dev) + (size_t)t0 * ldx * xe;
    void *yc = static_cast<uint8_t *>(y_dev) + (size_t)t0 * ldy * ye;
    int rc = gemv_launch(ctx, tiles, nrows / kUnitRows, w->k, xc, x_dtype, ldx, tc, yc, ldy, bias, epi, 0, 0.f,
                         0.f, s);
    if (rc) return rc;
  }
  return RC_OK;
}

int rc_gemv_host(rc_ctx *ctx, const rc_weight *w, const void *x_host, int x_dtype, int T, void *y_host,
                 const float *bias_dev) {
  RC_CHECK_ARG(ctx && x_host && y_host, "rc_gemv_host: NULL argument");
  if (!w) {
    set_error("rc_gemv_host: unknown weight handle");
    return RC_ERR_NOT_FOUND;
  }
  RC_CHECK_ARG(T >= 1, "rc_gemv_host: T must be >= 1 (got %d)", T);
  RC_CHECK_ARG(x_dtype == RC_DTYPE_BF16 || x_dtype == RC_DTYPE_F32, "rc_gemv_host: x_dtype must be BF16 or F32");
  RC_CUDA_TRY(cudaSetDevice(ctx->device));
  const size_t xe = x_dtype == RC_DTYPE_F32 ? 4 : 2;
  const size_t xb = (size_t)T * w->k * xe, yb = (size_t)T * w->n * xe;
  int rc = ensure_host_staging(ctx, xb, yb);
  if (rc) return rc;
  memcpy(ctx->pin_x, x_host, xb);
  if ((rc = host_copy_in(ctx, ctx->dev_x, ctx->pin_x, xb, ctx->stream))) return rc;
  rc = rc_gemv(ctx, w, ctx->dev_x, x_dtype, w->k, T, ctx->dev_y, x_dtype, w->n, 0, w->n, bias_dev, nullptr);
  if (rc) return rc;
  if ((rc = host_copy_out_and_wait(ctx, ctx->pin_y, ctx->dev_y, yb, ctx->stream))) return rc;
  memcpy(y_host, ctx->pin_y, yb);
  return RC_OK;
}

int rc_gemv_noalloc(const rc_weight *w, const void *x_dev, int x_dtype, int ldx, int T, void *y_dev, int y_dtype,
                    int ldy, int row0, int nrows, const float *bias_dev, void *stream) {
  RC_CHECK_ARG(x_dev && y_dev, "rc_gemv_noalloc: NULL argument");
  if (!w) {
    set_error("rc_gemv_noalloc: unknown weight handle");
    return RC_ERR_NOT_FOUND;
  }
  rc_ctx *ctx = w->ctx;
  RC_CHECK_ARG(w->format == kFormatQ4nx, "rc_gemv_noalloc: takes q4nx matrices only");
  RC_CHECK_ARG(!(w->flags & RC_UPLOAD_GATE_UP), "rc_gemv_noalloc: a gate/up-interleaved matrix is only usable by the MoE path");
  RC_CHECK_ARG(x_dtype == RC_DTYPE_BF16 || x_dtype == RC_DTYPE_F32, "rc_gemv_noalloc: x_dtype must be BF16 or F32");
  RC_CHECK_ARG(y_dtype == RC_DTYPE_F32 || (y_dtype == RC_DTYPE_BF16 && x_dtype == RC_DTYPE_BF16),
               "rc_gemv_noalloc: y_dtype must be F32, or BF16 with BF16 activations");
  RC_CHECK_ARG(T >= 1, "rc_gemv_noalloc: T must be >= 1 (got %d)", T);
  RC_CHECK_ARG(row0 >= 0 && nrows > 0 && row0 % kUnitRows == 0 && nrows % kUnitRows == 0 && row0 + nrows <= w->n,
               "rc_gemv_noalloc: rows [%d, %d) must be 16-aligned inside [0, %d)", row0, row0 + nrows, w->n);
  RC_CHECK_ARG(nrows / kUnitRows <= kNoAllocMaxTiles,
               "rc_gemv_noalloc: %d rows exceed the static scratch limit of %d rows", nrows,
               kNoAllocMaxTiles * kUnitRows);
  RC_CHECK_ARG(ldx >= w->k, "rc_gemv_noalloc: ldx (%d) < K (%d)", ldx, w->k);
  RC_CHECK_ARG(ldy >= nrows, "rc_gemv_noalloc: ldy (%d) < nrows (%d)", ldy, nrows);
  RC_CUDA_TRY(cudaSetDevice(ctx->device));
  unsigned char *scratch = nullptr;
  int rc = noalloc_scratch(ctx->device, &scratch);
  if (rc) return rc;
  const cudaStream_t s = pick_stream(ctx, stream);
  const int per = x_dtype == RC_DTYPE_F32 ? kMaxTokensPerLaunch / 2 : kMaxTokensPerLaunch;
  const size_t xe = x_dtype == RC_DTYPE_F32 ? 4 : 2;
  const size_t ye = y_dtype == RC_DTYPE_F32 ? 4 : 2;
  const int epi = x_dtype == RC_DTYPE_F32 ? kEpiF32 : (y_dtype == RC_DTYPE_F32 ? kEpiF32Raw : kEpiBf16);
  const uint8_t *tiles = w->tiles + (size_t)(row0 / kUnitRows) * (w->k / kUnitK) * kUnitBytes;
  const float *bias = bias_dev ? bias_dev + row0 : nullptr;
  for (int t0 = 0; t0 < T; t0 += per) {
    const int tc = T - t0 < per ? T - t0 : per;
    const void *xc = static_cast<const uint8_t *>(x_dev) + (size_t)t0 * ldx * xe;
    void *yc = static_cast<uint8_t *>(y_dev) + (size_t)t0 * ldy * ye;
    rc = gemv_launch_noalloc(ctx, scratch, tiles, nrows / kUnitRows, w->k, xc, x_dtype, ldx, tc, yc, ldy, bias, epi, s);
    if (rc) return rc;
  }
  return RC_OK;
}

}  // extern "C"
