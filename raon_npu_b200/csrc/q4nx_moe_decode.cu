// The MoE decode layer for T <= 16 tokens as one persistent kernel.
//
// One CTA per SM (cooperative launch: every CTA resident), 16 warps:
//
//   0 tokens     (expert parallelism) every rank's token rows arrive in this
//                rank's exchange buffer
//   1 stage      the CTA's router rows are requested; the token rows become
//                mma B fragments in shared memory, slot-compact (only the T
//                token columns are stored)
//   2 logits     CTA c computes the logits of experts c, c + grid, ...
//                (f64 sums of exact bf16 products, rounded once to f32)
//   -- grid barrier --
//   3 selection  every CTA takes each token's k best router keys (larger
//                first, NaN last, ties by lower index; one warp per token),
//                the weights, the ascending-ID slot lists and the group
//                table -- identical inputs, identical tables, no barrier
//   4 stream     the CTA's share of the layer -- a contiguous range of
//                (group, row tile) tiles of gate/up, then one of down -- is a
//                stream of 2560-byte units fetched in chunks of a few units
//                (one mbarrier, one to three bulk copies each) into a ring of
//                chunk slots; at T = 1 the whole share is requested at once
//   5 gate/up    rounds of whole tiles: unit i of a round goes to warp i % 16
//                (a warp keeps one k-block), each unit's result to its own
//                slot-compact partial; a tile is the sum of its units in
//                k-block order; GLU epilogue -> act rows
//   -- grid barrier --
//   6 down       act rows of the CTA's down groups staged slot-compact; the
//                same rounds; slot rows out (with expert parallelism, into
//                the buffer of the token's owner)
//   -- grid barrier (and, with expert parallelism, every rank's rows) --
//   7 combine    ascending-ID f32 sum (multiply then add, no FMA), RTNE, plus
//                the shared row
//
// The unit arithmetic, the partition of tiles over CTAs and the combine are
// those of the separate kernels in q4nx_moe.cu (a tile's result depends on
// the tile alone), so a token's bytes do not depend on which path ran.
// Every wait is bounded (1 s): it sets the error word and the kernel unwinds.
#include "moe_internal.cuh"
#include "q4nx_core.cuh"
#include "rc_device.cuh"
#include "rc_internal.cuh"

namespace rc {

constexpr int kDcWarps = 16;
constexpr int kDcThreads = kDcWarps * 32;
static_assert(kMoeMaxTokens <= kDcWarps, "the selection takes one warp per token");
constexpr int kDcChunk = 6;         // units per chunk
constexpr int kDcMaxChunks = 32;    // chunk slots at most (shared memory decides)
// dynamic shared memory of one CTA: the opt-in limit less the static copies
// of the parameters and the stream description
constexpr int kDcSmemLimit = kGemvSmemLimit - 1024;
// "red" area: [16 warps][16 tokens] f64 partial logits, the barrier verdict
// word, then the peer buffer table
constexpr int kDcRedBytes = kDcWarps * kMoeMaxTokens * 8 + 16;

struct DcParams {
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
  const uint8_t *const *gu_tiles;    // [E+1]
  const uint8_t *const *dn_tiles;    // [E+1]
  int inter, inter_pad;
  uint16_t *act;                     // [E+1][16][inter_pad]
  uint16_t *slot_rows;               // [T][k+1][hidden]
  int zero_foreign;                  // zero the slot rows of experts computed elsewhere
  uint16_t *out;                     // [T][hidden], null: no combine
  int act_kind;
  float gate_beta, value_beta;
  int chunk_slots;                   // B: chunk slots of the unit ring
  int round_units;                   // units a round may hold (partials)
  int stage_blk;                     // act blocks (groups) the staging area holds
  int col_down;                      // down tiles column-major, whole columns per CTA, combined in the CTA
  int off_buf, off_stage, off_part, off_tab, off_sel, off_red, off_bar;
  unsigned long long *bar;           // grid-barrier arrival count (only grows)
  int *cols;                         // [hidden/16] down tiles written per column tile (zero between calls)
  int *err;
  int ep_world, ep_rank, ep_M;
  uint8_t *const *ep_peer;
  unsigned long long *ep_flags;
  uint32_t ep_tok_off, ep_red_off;
  unsigned long long ep_call;        // this call's number (calls done before it), set in the kernel
  const uint16_t *ep_x_own;
  unsigned long long *trace;         // phase stamps [grid][kTracePhases] (null: off)
};

__device__ __forceinline__ void dc_stamp(const DcParams &p, int phase) {
  if (p.trace && threadIdx.x == 0) p.trace[(size_t)blockIdx.x * kTracePhases + phase] = global_timer_ns();
}

// Router order as an unsigned key: larger value -> larger key, -0 equal to
// +0, NaN (1) below every number.  Equal keys are ordered by lower expert
// index, so (key, index) is a strict total order.
__device__ __forceinline__ uint32_t dc_route_key(float v) {
  if (v != v) return 1u;
  uint32_t b = __float_as_uint(v);
  if (b == 0x80000000u) b = 0u;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// The sigmoid routing score, out of line (one copy of the f64 exponential).
static __device__ __noinline__ float dc_sigmoid(float l) { return __double2float_rn(1.0 / (1.0 + exp(-(double)l))); }

// --------------------------------------------------------- staging ------
// Slot-compact fragments of a staging area that holds nblk blocks (the token
// set, or one block per expert group) of Tsl token slots over kb k-blocks:
//   frag word ((((b*kb + kbi)*4 + s4)*Tsl + t)*4 + q)*8 + (s%4)*2 + j holds
//     the f16 pair {x'[t][16s+2q+8j], x'[t][16s+2q+8j+1]} of k16-step s of
//     k-block kbi (the mma B fragment of lane 4g+q for column g = t % 8);
//   bmin uint4 ((b*kb + kbi)*Tsl + t)*4 + q: bf16 {S'1, S'2, S'3, 0} pairs of
//     groups 2q, 2q+1 (the min-term fragment);
//   inv ((b*kb + kbi)*Tsl + t): the block's 2^-s.
// Values, scales and sums are those of stage_core (q4nx_core.cuh); only the
// storage is compact (no room for token columns that do not exist).
__host__ __device__ constexpr size_t dc_stage_bytes(int nblk, int tsl, int kb) {
  return (size_t)nblk * tsl * kb * (512 + 64 + 4);
}

// One warp per (block, slot, k-block) task; tasks w0, w0 + nw, ... of
// nblk * Tsl * kb.  Row of (b, t): src + (b * row_blk + t) * ld.  A warp
// requests the rows of up to kDcStageBatch tasks before it converts the
// first, so their L2 latencies overlap.
constexpr int kDcStageBatch = 3;

static __device__ __noinline__ void dc_stage(const uint16_t *src, int ld, int row_blk, int nblk, int tsl, int kb,
                                             uint8_t *area, int w0, int nw) {
  const int lane = threadIdx.x & 31;
  uint32_t *frag = reinterpret_cast<uint32_t *>(area);
  uint16_t *bmin16 = reinterpret_cast<uint16_t *>(area + (size_t)nblk * tsl * kb * 512);
  float *inv = reinterpret_cast<float *>(area + (size_t)nblk * tsl * kb * 576);
  const int ntask = nblk * tsl * kb;
#pragma unroll 1
  for (int i0 = w0; i0 < ntask; i0 += kDcStageBatch * nw) {
    uint4 raws[kDcStageBatch];
#pragma unroll
    for (int jb = 0; jb < kDcStageBatch; ++jb) {
      const int i = i0 + jb * nw;
      if (i < ntask) {
        const int b = i / (tsl * kb), r = i - b * tsl * kb, t = r / kb, kbi = r - t * kb;
        raws[jb] = __ldcg(reinterpret_cast<const uint4 *>(src + ((size_t)b * row_blk + t) * ld + kbi * kUnitK +
                                                          lane * 8));
      }
    }
#pragma unroll
    for (int jb = 0; jb < kDcStageBatch; ++jb) {
      const int i = i0 + jb * nw;
      if (i >= ntask) break;
      const int b = i / (tsl * kb), r = i - b * tsl * kb, t = r / kb, kbi = r - t * kb;
      const uint32_t w[4] = {raws[jb].x, raws[jb].y, raws[jb].z, raws[jb].w};
      float v[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[2 * j] = bf16_lo_f32(w[j]);
        v[2 * j + 1] = bf16_hi_f32(w[j]);
      }
      const int s = block_shift(warp_absmax(v));
      const float sc = pow2f(s);
      uint32_t hw[4];
      float part = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = v[2 * j] * sc, c = v[2 * j + 1] * sc;
        const __half2 h = __floats2half2_rn(a, c);
        hw[j] = *reinterpret_cast<const uint32_t *>(&h);
        part += a;   // a bf16 value times 2^s is exact in f16: sum the exact values
        part += c;
      }
      const size_t u = (size_t)b * kb + kbi;
      const int st = lane >> 1, jj = lane & 1;
      uint32_t *fw = frag + (((u * 4 + (st >> 2)) * tsl + t) * 4) * 8 + (st & 3) * 2 + jj;
#pragma unroll
      for (int q = 0; q < 4; ++q) fw[q * 8] = hw[q];
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      if ((lane & 3) == 0) {
        const int gi = lane >> 2;
        const float sp = part * 5.9604644775390625e-08f;   // S' 2^-24 (exact)
        const uint16_t s1 = f32_to_bf16_rne(sp);
        const float r1 = sp - bf16_to_f32(s1);
        const uint16_t s2 = f32_to_bf16_rne(r1);
        uint16_t *bw = bmin16 + ((u * tsl + t) * 4 + (gi >> 1)) * 8 + (gi & 1);
        bw[0] = s1;
        bw[2] = s2;
        bw[4] = f32_to_bf16_rne(r1 - bf16_to_f32(s2));
        bw[6] = 0;
      }
      if (lane == 0) inv[u * tsl + t] = pow2f(-s);
    }
  }
}

// The lane's fragments of k-block kbi of block blk.  Columns of token slots
// that do not exist read the last slot's data: mma columns do not interact,
// and those columns' results are never stored.
template <int NTB>
__device__ __forceinline__ void dc_load_frag(XFrag<NTB> &r, const uint8_t *area, int nblk, int tsl, int kb, int blk,
                                             int kbi, int lane) {
  const uint4 *frag = reinterpret_cast<const uint4 *>(area);
  const uint4 *bmin = reinterpret_cast<const uint4 *>(area + (size_t)nblk * tsl * kb * 512);
  const float *inv = reinterpret_cast<const float *>(area + (size_t)nblk * tsl * kb * 576);
  const int g = lane >> 2, q = lane & 3;
  const size_t u = (size_t)blk * kb + kbi;
  r.shared = true;
  r.step = 8 * tsl;
#pragma unroll
  for (int tb = 0; tb < NTB; ++tb) {
    const int t = min(tb * 8 + g, tsl - 1);
    const uint4 *xv = frag + ((u * 4 * tsl + t) * 4 + q) * 2;
    r.xv[tb] = xv;
    if (NTB == 1) {
#pragma unroll
      for (int s4 = 0; s4 < 4; ++s4) {
        r.xa[s4] = xv[s4 * r.step];
        r.xb[s4] = xv[s4 * r.step + 1];
      }
    }
    r.bm[tb] = bmin[(u * tsl + t) * 4 + q];
    const int t0 = min(tb * 8 + 2 * q, tsl - 1), t1 = min(tb * 8 + 2 * q + 1, tsl - 1);
    r.inv[tb] = make_float2(inv[u * tsl + t0], inv[u * tsl + t1]);
  }
}

// ------------------------------------------------------------ waits -----
// All CTAs meet (arrival n belongs to barrier n / grid).  Bounded: false after
// 1 s (error word set), CTA-uniform.
static __device__ __noinline__ bool dc_grid_barrier(unsigned long long *bar, int *err, int *ok_s) {
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

// Wait until a counter that peer GPUs add to reaches ``target``.  Bounded.
static __device__ __noinline__ bool dc_wait_sys(const unsigned long long *ctr, unsigned long long target, int *err,
                                                int *ok_s) {
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

// ------------------------------------------------------- unit stream ----
// The CTA's units: gate/up tiles [c0[0], c0[0] + nt[0]) of the group-major
// tile list (kb[0] k-blocks each), then down tiles [c0[1], c0[1] + nt[1]);
// unit s of the stream is (tile, k-block) in memory order, so each group's
// part of a phase is one contiguous byte range.
struct DcStream {
  const uint8_t *const *g_ptr[2];    // per phase: tile base of each group (shared memory)
  int c0[2], nt[2], kb[2], gt[2];
  int units0, units;                 // gate/up units; all units
  int nchunk;                        // chunks of kDcChunk units
  int col, ng;                       // down list column-major (tile = index / ng, group = index % ng)
};

// The global address and the contiguous extent (in units, <= n) of unit s.
__device__ __forceinline__ const uint8_t *dc_unit_src(const DcStream &st, int s, int n, int *run) {
  const int ph = s < st.units0 ? 0 : 1;
  const int u = ph ? s - st.units0 : s;
  const int kb = st.kb[ph];
  const int tg = st.c0[ph] + u / kb;                      // tile in the phase's list
  int grp, tile, left;
  if (ph == 1 && st.col) {
    // column-major: consecutive list entries are different experts
    tile = tg / st.ng, grp = tg - tile * st.ng;
    left = kb - (u % kb);
  } else {
    grp = tg / st.gt[ph], tile = tg - grp * st.gt[ph];
    // units left in this group of this phase
    const int grp_end_tile = (grp + 1) * st.gt[ph] < st.c0[ph] + st.nt[ph] ? (grp + 1) * st.gt[ph]
                                                                             : st.c0[ph] + st.nt[ph];
    left = (grp_end_tile - tg) * kb - (u % kb);
  }
  *run = left < n ? left : n;
  const uint8_t *b = st.g_ptr[ph][grp];
  return b ? b + ((size_t)tile * kb + u % kb) * kUnitBytes : nullptr;
}

// Request chunk j into its slot (one thread): one bulk copy per contiguous
// run (a chunk may cross a group or the phase boundary); units of experts
// that are not loaded here are not fetched.
static __device__ __noinline__ void dc_issue_chunk(const DcStream &st, int j, uint8_t *buf, uint32_t bar0,
                                                   int slots) {
  const int slot = j % slots;
  const uint32_t bar = bar0 + 8 * slot;
  const int s0 = j * kDcChunk, s1 = s0 + kDcChunk < st.units ? s0 + kDcChunk : st.units;
  const uint64_t pol = policy_evict_first();
  const uint32_t dst0 = smem_addr(buf) + slot * kDcChunk * kUnitBytes;
  // each contiguous run's bytes join the phase's transaction count before its
  // copy is issued; the single arrival comes last, so the phase cannot
  // complete before every run is accounted for
#pragma unroll 1
  for (int s = s0; s < s1;) {
    int run;
    const uint8_t *src = dc_unit_src(st, s, s1 - s, &run);
    if (src) {
      mbar_expect_tx(bar, run * kUnitBytes);
      bulk_copy_g2s(dst0 + (s - s0) * kUnitBytes, src, run * kUnitBytes, bar, pol);
    }
    s += run;
  }
  mbar_arrive(bar);
}

// Eight columns of one token: ascending-ID f32 sum (product rounded, then
// sum rounded) of the k slot rows at ``rows`` (stride ``hidden``) with the
// weights ``w``, RTNE, then RTNE(routed + shared row k) when with_shared.
template <bool SHARED_MEM = false>
__device__ __forceinline__ uint4 dc_combine8(const uint16_t *rows, int hidden, int k, const float *w,
                                             bool with_shared) {
  auto ld = [](const uint16_t *a) {
    return SHARED_MEM ? *reinterpret_cast<const uint4 *>(a) : __ldcg(reinterpret_cast<const uint4 *>(a));
  };
  const uint4 sh = with_shared ? ld(rows + (size_t)k * hidden) : make_uint4(0, 0, 0, 0);
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  // rows in batches of eight, all of a batch requested before any is summed
#pragma unroll 1
  for (int s0 = 0; s0 < k; s0 += 8) {
    uint4 r[8];
#pragma unroll
    for (int s = 0; s < 8; ++s)
      r[s] = s0 + s < k ? ld(rows + (size_t)(s0 + s) * hidden) : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      if (s0 + s < k) {
        const float ws = w[s0 + s];
        const uint32_t q[4] = {r[s].x, r[s].y, r[s].z, r[s].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[2 * j] = __fadd_rn(acc[2 * j], __fmul_rn(bf16_to_f32(q[j] & 0xFFFFu), ws));
          acc[2 * j + 1] = __fadd_rn(acc[2 * j + 1], __fmul_rn(bf16_to_f32(q[j] >> 16), ws));
        }
      }
    }
  }
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
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Request the chunks whose slots are free once the stream's first ``done``
// chunks are consumed (chunk j by lane 0 of warp j % 16).  Returns the new
// count of requested chunks (the same in every thread).
__device__ __forceinline__ int dc_refill(const DcStream &st, int issued, int done, uint8_t *buf, uint32_t bar0,
                                         int B) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hi = done + B < st.nchunk ? done + B : st.nchunk;
  if (lane == 0) {
#pragma unroll 1
    for (int j = issued + (warp - issued % kDcWarps + kDcWarps) % kDcWarps; j < hi; j += kDcWarps)
      dc_issue_chunk(st, j, buf, bar0, B);
  }
  return hi > issued ? hi : issued;
}

__device__ __forceinline__ float dc_glu(float gate, float up, int kind, float gb, float vb) {
  return kind == RC_ACT_SITU ? act_situ(gate, up, gb, vb) : act_swiglu(gate, up);
}

// Slot-compact partials: per unit of a round, the lanes whose result columns
// exist -- token block tb keeps lanes with quad index < qn(T, tb) -- as float4.
__host__ __device__ __forceinline__ int dc_qn(int T, int tb) {
  const int n = (T - 8 * tb + 1) / 2;
  return n < 0 ? 0 : (n > 4 ? 4 : n);
}

// One phase's rounds (ph 0: gate/up with the GLU epilogue, 1: down).
// ``issued``: chunks requested so far; returns (chunks requested << 1) | a
// wait ran out.  ``p`` and ``st`` live in shared memory.
// On one GPU the down phase also combines: the warp that writes the last
// down tile of an output column tile (column counter ``p.cols``, one
// arrival per group) sums that column tile of every token (``ng`` groups,
// slot weights ``slot_w``) and clears the counter for the next call.
template <int NTB>
__device__ __forceinline__ int dc_rounds(const DcParams &p, uint8_t *smem, const DcStream &st, int ph,
                                         const uint8_t *stage, int nblk, const uint32_t *g_mask,
                                         const int *g_dst, int g_lo, int issued, bool failed, int ng,
                                         const float *slot_w) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, T = p.T;
  uint8_t *const *ep_peer_s = reinterpret_cast<uint8_t *const *>(smem + p.off_red + kDcRedBytes);
  uint8_t *buf = smem + p.off_buf;
  const uint32_t bar0 = smem_addr(smem + p.off_bar);
  float4 *part = reinterpret_cast<float4 *>(smem + p.off_part);
  const int B = p.chunk_slots;
  const int kb = st.kb[ph], nt = st.nt[ph], gt = st.gt[ph], c0 = st.c0[ph];
  const int base = ph ? st.units0 : 0;
  const int qn0 = dc_qn(T, 0), qn1 = NTB == 2 ? dc_qn(T, 1) : 0, rec = 8 * (qn0 + qn1);
  const int g = lane >> 2, qd = lane & 3;
  const int tiles_per_round = p.round_units / kb;
  XFrag<NTB> xr;
  int xr_key = -1;
#pragma unroll 1
  for (int t0 = 0; t0 < nt; t0 += tiles_per_round) {
    const int t1 = t0 + tiles_per_round < nt ? t0 + tiles_per_round : nt;
    const int nu = (t1 - t0) * kb;
    bool wfail = false;                        // this warp gave up a wait
    if (!failed && warp < nu) {
      // unit i = warp + 16 n of the round: (tile, k-block) of the phase, its
      // group, its chunk and place in the chunk, advanced by 16 units a step
      // without divisions
      int u = t0 * kb + warp;
      int tile_r = u / kb, kbi = u - tile_r * kb;                // tile of the phase range
      // group and tile of the list entry; column-major lists step the group first
      const bool col = ph == 1 && st.col;
      const int inner_n = col ? ng : gt;
      int tg = c0 + tile_r, outer = tg / inner_n, inner = tg - outer * inner_n;
      int grp = col ? inner : outer;
      int sidx = base + u, j = sidx / kDcChunk, off = sidx - j * kDcChunk;
      int slot = j % B;
      uint32_t par = (uint32_t)(j / B) & 1u;
      const int dt = kDcWarps / kb, dk = kDcWarps - dt * kb;     // 16 units = dt tiles + dk k-blocks
      const int dj = kDcWarps / kDcChunk, doff = kDcWarps - dj * kDcChunk;
#pragma unroll 1
      for (int i = warp; i < nu; i += kDcWarps) {
        if (!mbar_wait_bounded_warp(bar0 + 8 * slot, par)) {
          if (lane == 0) atomicCAS(p.err, 0, kErrWaitTimeout);
          wfail = true;
          break;
        }
        if (st.g_ptr[ph][grp] != nullptr) {
          const int blk = ph ? grp - g_lo : 0;
          if (blk * kb + kbi != xr_key) {
            dc_load_frag<NTB>(xr, stage, nblk, T, kb, blk, kbi, lane);
            xr_key = blk * kb + kbi;
          }
          float4 Q[NTB];
          unit_result<NTB>(buf + ((size_t)slot * kDcChunk + off) * kUnitBytes, xr, lane, Q);
          float4 *dst = part + (size_t)i * rec;
          if (qd < qn0) dst[g * qn0 + qd] = Q[0];
          if (NTB == 2 && qd < qn1) dst[8 * qn0 + g * qn1 + qd] = Q[NTB - 1];
        }
        // next unit of this warp
        kbi += dk;
        int tstep = dt;
        if (kbi >= kb) kbi -= kb, ++tstep;
        inner += tstep;
        while (inner >= inner_n) inner -= inner_n, ++outer;
        grp = col ? inner : outer;
        off += doff;
        int cstep = dj;
        if (off >= kDcChunk) off -= kDcChunk, ++cstep;
        slot += cstep;
        while (slot >= B) slot -= B, par ^= 1u;
      }
    }
    // a wait that ran out in any warp stops the phase (CTA-uniform verdict)
    if (__syncthreads_or(wfail)) failed = true;
    if (ph == 1 && t0 == 0) dc_stamp(p, kTrDownUnits);
    if (!failed) {
      // a tile is the sum of its units' results in k-block order
#pragma unroll 1
      for (int ti = t0 + warp; ti < t1; ti += kDcWarps) {
        const int tg = c0 + ti;
        const bool col = ph == 1 && st.col;
        const int grp = col ? tg % ng : tg / gt, tile = col ? tg / ng : tg - (tg / gt) * gt;
        const bool live = st.g_ptr[ph][grp] != nullptr;
        Acc<NTB> acc;
        acc_zero(acc);
        const float4 *src = part + (size_t)(ti - t0) * kb * rec;
#pragma unroll 1
        for (int kbi = 0; kbi < kb; ++kbi) {
          float4 v[NTB];
          v[0] = qd < qn0 ? src[(size_t)kbi * rec + g * qn0 + qd] : make_float4(0.f, 0.f, 0.f, 0.f);
          if (NTB == 2)
            v[NTB - 1] = qd < qn1 ? src[(size_t)kbi * rec + 8 * qn0 + g * qn1 + qd] : make_float4(0.f, 0.f, 0.f, 0.f);
          acc_add(acc, v);
        }
        const uint32_t mask = g_mask[grp];
#pragma unroll
        for (int tb = 0; tb < NTB; ++tb) {
#pragma unroll
          for (int e2 = 0; e2 < 2; ++e2) {
            const int t = tb * 8 + 2 * qd + e2;
            if (t >= T || !((mask >> t) & 1u)) continue;
            if (ph == 0) {
              float v = 0.f;
              if (live) v = dc_glu(bf16_round(acc.v[tb][e2]), bf16_round(acc.v[tb][2 + e2]), p.act_kind,
                                   p.gate_beta, p.value_beta);
              p.act[((size_t)grp * 8 * NTB + t) * p.inter_pad + tile * 8 + g] = f32_to_bf16_rne(v);
            } else {
              const int srow = g_dst[grp * T + t];     // slot row t*(k+1) + position
              const uint32_t r0 = live ? f32_to_bf16_rne(acc.v[tb][e2]) : 0u;
              const uint32_t r1 = live ? f32_to_bf16_rne(acc.v[tb][2 + e2]) : 0u;
              if (!col && p.ep_world > 1) {
                // straight into the buffer of the token's owner: rows g and
                // g + 8 of the tile and this call's number in one 8-byte
                // store, so the owner needs no fence or flag to read them
                const int tt = srow / (p.k + 1), pos = srow - tt * (p.k + 1);
                const int owner = tt / p.ep_M, tl = tt - owner * p.ep_M;
                unsigned long long *wd = reinterpret_cast<unsigned long long *>(ep_peer_s[owner] + p.ep_red_off) +
                                         (((size_t)tl * (p.k + 1) + pos) * (p.hidden / kUnitRows) + tile) * 8 + g;
                st_relaxed_sys(wd, ((unsigned long long)(uint32_t)(p.ep_call + 1) << 32) | r0 | (r1 << 16));
              } else {
                // col: this CTA holds every expert row of the column tile --
                // rows [slot row][16 columns] in the (now free) staging area
                uint16_t *y = col ? reinterpret_cast<uint16_t *>(smem + p.off_stage) + (size_t)srow * kUnitRows + g
                                  : p.slot_rows + (size_t)srow * p.hidden + tile * kUnitRows + g;
                y[0] = (uint16_t)r0;
                y[8] = (uint16_t)r1;
              }
            }
          }
        }
        if (ph == 1 && !col && p.ep_world <= 1 && p.out) {
          // the last writer of column tile ``tile`` combines it (threadfence
          // reduction: stores, fence, count; the last counter sees them all)
          __syncwarp();
          int old = 0;
          if (lane == 0) {
            __threadfence();
            old = atomicAdd(p.cols + tile, 1);
          }
          old = __shfl_sync(0xffffffffu, old, 0);
          if (old == ng - 1) {
            __threadfence();
            const int t = lane >> 1, h = lane & 1;
            if (t < T) {
              const uint16_t *rows = p.slot_rows + (size_t)t * (p.k + 1) * p.hidden + tile * kUnitRows + h * 8;
              *reinterpret_cast<uint4 *>(p.out + (size_t)t * p.hidden + tile * kUnitRows + h * 8) =
                  dc_combine8(rows, p.hidden, p.k, slot_w + t * p.k, p.shared_id >= 0 && p.own.shared_mask);
            }
            if (lane == 0) p.cols[tile] = 0;
          }
        }
      }
    }
    __syncthreads();
    if (ph == 1 && t0 == 0) dc_stamp(p, kTrDownTiles);
    // chunks whose units all lie before this round's end are consumed: their
    // slots take the next chunks of the stream (chunk j by warp j % 16)
    if (!failed) issued = dc_refill(st, issued, (base + t1 * kb) / kDcChunk, buf, bar0, B);
  }
  return (issued << 1) | (failed ? 1 : 0);
}

// The combine of rows g and g + 8 of one column tile for one token from the
// expert-parallel exchange: word s*stride of ``w0`` (slot s) carries the two
// rows' bf16 values (bits 0-15, 16-31) and the number of the call that wrote
// them (bits 32-63).  Waits, until global time t0 + 1 s, for every slot's
// word of call ``want``, then sums exactly as dc_combine8 (ascending slots,
// f32 multiply then add, RTNE, plus the shared row); false on a timeout.
__device__ __forceinline__ bool dc_combine_tagged(const unsigned long long *w0, size_t stride, int k,
                                                  const float *w, bool with_shared, uint32_t want, uint64_t t0,
                                                  uint16_t *out) {
  const int ns = k + (with_shared ? 1 : 0);
  unsigned long long v[kMoeMaxK + 1];
  uint32_t pending = (ns >= 32 ? 0xFFFFFFFFu : (1u << ns) - 1u);
  while (true) {
#pragma unroll
    for (int s = 0; s < kMoeMaxK + 1; ++s) {
      if ((pending >> s) & 1u) {
        v[s] = ld_relaxed_sys(w0 + (size_t)s * stride);
        if ((uint32_t)(v[s] >> 32) == want) pending &= ~(1u << s);
      }
    }
    if (!pending) break;
    if (global_timer_ns() - t0 > 1000000000ull) return false;
  }
  float a0 = 0.f, a1 = 0.f;
#pragma unroll
  for (int s = 0; s < kMoeMaxK; ++s) {
    if (s < k) {
      const float ws = w[s];
      a0 = __fadd_rn(a0, __fmul_rn(bf16_to_f32((uint32_t)v[s] & 0xFFFFu), ws));
      a1 = __fadd_rn(a1, __fmul_rn(bf16_to_f32(((uint32_t)v[s] >> 16) & 0xFFFFu), ws));
    }
  }
  uint32_t r0 = f32_to_bf16_rne(a0), r1 = f32_to_bf16_rne(a1);
  if (with_shared) {
    uint32_t sh = 0;
#pragma unroll
    for (int s = 0; s < kMoeMaxK + 1; ++s)
      if (s == k) sh = (uint32_t)v[s];
    r0 = f32_to_bf16_rne(bf16_to_f32(r0) + bf16_to_f32(sh & 0xFFFFu));
    r1 = f32_to_bf16_rne(bf16_to_f32(r1) + bf16_to_f32(sh >> 16));
  }
  out[0] = (uint16_t)r0;
  out[8] = (uint16_t)r1;
  return true;
}

// ---------------------------------------------------------- routing -----
// The logits of experts blockIdx.x, + grid, ... for all T tokens, by warps
// 0 .. nlog-1 (nlog = the 256-column slices, at most 16): warp w sums the
// slices w, w + nlog, ... in f64 (exact bf16 products), the warps' sums are
// added in warp order and rounded once to f32.  ``wpre`` is the lane's router
// slice of this CTA's first expert, requested at kernel entry.  The logit
// warps meet on named barrier 1; the other warps stage meanwhile.
static __device__ __noinline__ void dc_logits(const DcParams &p, double *red, uint4 wpre, int nlog) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = p.T, E = p.n_experts, nslice = p.hidden / kUnitK;
  if (warp >= nlog) return;
  if (T <= 4) {
    // few tokens: one token at a time
#pragma unroll 1
    for (int e = blockIdx.x; e < E; e += gridDim.x) {
#pragma unroll 1
      for (int t = 0; t < T; ++t) {
        double acc = 0.0;
#pragma unroll 1
        for (int sl = warp; sl < nslice; sl += nlog) {
          const int col = sl * kUnitK + lane * 8;
          const uint4 wv = (e == (int)blockIdx.x && sl == warp)
                               ? wpre : __ldg(reinterpret_cast<const uint4 *>(p.wr + (size_t)e * p.hidden + col));
          const uint4 xv = __ldcg(reinterpret_cast<const uint4 *>(p.x + (size_t)t * p.hidden + col));
          const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w}, xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            acc = fma((double)bf16_to_f32(xw[j] & 0xFFFFu), (double)bf16_to_f32(ww[j] & 0xFFFFu), acc);
            acc = fma((double)bf16_to_f32(xw[j] >> 16), (double)bf16_to_f32(ww[j] >> 16), acc);
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) red[warp * kMoeMaxTokens + t] = acc;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(nlog * 32) : "memory");
      if (tid < T) {
        double a = 0.0;
#pragma unroll 1
        for (int w = 0; w < nlog; ++w) a += red[w * kMoeMaxTokens + tid];
        p.logits[(size_t)tid * E + e] = __double2float_rn(a);
      }
      asm volatile("bar.sync 1, %0;" ::"r"(nlog * 32) : "memory");
    }
    return;
  }
  // more tokens: every token's sum at once, the router slice read and widened once
#pragma unroll 1
  for (int e = blockIdx.x; e < E; e += gridDim.x) {
    double acc[kMoeMaxTokens];
#pragma unroll
    for (int t = 0; t < kMoeMaxTokens; ++t) acc[t] = 0.0;
#pragma unroll 1
    for (int sl = warp; sl < nslice; sl += nlog) {
      const int col = sl * kUnitK + lane * 8;
      const uint4 wv = (e == (int)blockIdx.x && sl == warp)
                           ? wpre : __ldg(reinterpret_cast<const uint4 *>(p.wr + (size_t)e * p.hidden + col));
      double wd[8];
      // eight tokens' slices are requested before the router slice is widened
#pragma unroll
      for (int t0 = 0; t0 < kMoeMaxTokens; t0 += 8) {
        if (t0 < T) {
          uint4 xv[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            if (t0 + i < T) xv[i] = __ldcg(reinterpret_cast<const uint4 *>(p.x + (size_t)(t0 + i) * p.hidden + col));
          if (t0 == 0) {
            const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              wd[2 * j] = (double)bf16_to_f32(ww[j] & 0xFFFFu);
              wd[2 * j + 1] = (double)bf16_to_f32(ww[j] >> 16);
            }
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            if (t0 + i < T) {
              const uint32_t xw[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                acc[t0 + i] = fma((double)bf16_to_f32(xw[j] & 0xFFFFu), wd[2 * j], acc[t0 + i]);
                acc[t0 + i] = fma((double)bf16_to_f32(xw[j] >> 16), wd[2 * j + 1], acc[t0 + i]);
              }
            }
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
        if (lane == 0) red[warp * kMoeMaxTokens + t] = a;
      }
    }
    asm volatile("bar.sync 1, %0;" ::"r"(nlog * 32) : "memory");
    if (tid < T) {
      double a = 0.0;
#pragma unroll 1
      for (int w = 0; w < nlog; ++w) a += red[w * kMoeMaxTokens + tid];
      p.logits[(size_t)tid * E + e] = __double2float_rn(a);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(nlog * 32) : "memory");
  }
}

// Selection by the whole CTA: the router keys of every (token, expert) pair,
// then per token (warp t) the k best in router order (a larger key, or an
// equal key and a lower index), best first; then per token (warp t, lane
// r < k) the weight, the ascending-ID slot position and the expert's token
// mask.  ``scratch`` holds T*E keys and scores.
static __device__ __noinline__ void dc_select(const DcParams &p, const float *bias_s, uint8_t *scratch,
                                              int32_t *slots, float *slot_w, int32_t *sel_e, float *sel_sc,
                                              uint32_t *mask_s) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int T = p.T, E = p.n_experts, k = p.k, n = T * E;
  // keys in rows of E4 (E rounded up to 4; the padding keys are 0, below
  // every router key, which are >= 1)
  const int E4 = (E + 3) & ~3;
  uint32_t *key_s = reinterpret_cast<uint32_t *>(scratch);
  float *sc_s = reinterpret_cast<float *>(key_s + T * E4);
#pragma unroll 1
  for (int i = tid; i < T * (E4 - E); i += kDcThreads) key_s[(i / (E4 - E)) * E4 + E + i % (E4 - E)] = 0u;
#pragma unroll 1
  for (int i = tid; i < n; i += kDcThreads) {
    const int t = i / E, e = i - t * E;
    const float l = __ldcg(p.logits + i);
    float sc, v;
    if (p.mode == RC_ROUTER_SIGMOID_BIAS) {
      sc = dc_sigmoid(l);
      v = sc + bias_s[e];
    } else {
      sc = l + bias_s[e];
      v = sc;
    }
    sc_s[i] = sc;
    key_s[t * E4 + e] = dc_route_key(v);
  }
  __syncthreads();
  dc_stamp(p, kTrKeys);
  // top-k: warp t takes token t's best key k times over -- the largest key,
  // the lowest expert index among equal ones (one warp max, one warp min),
  // then removes it (0 ranks below every router key) -- so the ranks follow
  // the strict order (key descending, index ascending)
#pragma unroll 1
  for (int t = warp; t < T; t += kDcWarps) {
    uint32_t kv[kMoeMaxExperts / 32];
#pragma unroll
    for (int j = 0; j < kMoeMaxExperts / 32; ++j) {
      const int e = lane + 32 * j;
      kv[j] = e < E ? key_s[t * E4 + e] : 0u;
    }
#pragma unroll 1
    for (int r = 0; r < k; ++r) {
      uint32_t bk = 0u;
      int bj = 0;
#pragma unroll
      for (int j = 0; j < kMoeMaxExperts / 32; ++j)
        if (kv[j] > bk) bk = kv[j], bj = j;
      const uint32_t mk = __reduce_max_sync(0xffffffffu, bk);
      const uint32_t mi = __reduce_min_sync(0xffffffffu, bk == mk ? (uint32_t)(lane + 32 * bj) : 0xFFFFFFFFu);
#pragma unroll
      for (int j = 0; j < kMoeMaxExperts / 32; ++j)
        if ((uint32_t)(lane + 32 * j) == mi) kv[j] = 0u;
      if (lane == 0) {
        sel_e[t * k + r] = (int32_t)mi;
        sel_sc[t * k + r] = sc_s[t * E + mi];
      }
    }
  }
  // warp t wrote token t's picks and reads them next (T <= 16 warps)
  __syncwarp();
  dc_stamp(p, kTrRanked);
  if (warp < T) {
    // lane r < k holds the token's r-th best expert; the weights' sums run
    // over the ranks in order (shuffles), as a single thread would add them
    const int t = warp, r = lane;
    const bool sel = r < k;
    const int e = sel ? sel_e[t * k + r] : 0x7FFFFFFF;
    const float sc = sel ? sel_sc[t * k + r] : 0.f;
    // (every rank's value is fetched first, then added in rank order)
    auto ranked_sum = [&](float v) {
      float vs[kMoeMaxK], acc = 0.f;
#pragma unroll
      for (int r2 = 0; r2 < kMoeMaxK; ++r2) vs[r2] = __shfl_sync(0xffffffffu, v, r2);
#pragma unroll
      for (int r2 = 0; r2 < kMoeMaxK; ++r2)
        if (r2 < k) acc += vs[r2];
      return acc;
    };
    float w;
    if (p.mode == RC_ROUTER_SIGMOID_BIAS) {
      const float sum = ranked_sum(sc);
      w = sc;
      if (p.renorm) w = w / (sum + 1e-20f);
      w = w * p.scaling;
    } else {
      // softmax over all experts renormalised over the top-k equals the
      // softmax of the selected scores (the full denominator cancels)
      const float ex = expf(sc - __shfl_sync(0xffffffffu, sc, 0));
      w = ex / ranked_sum(ex);
    }
    int pos = 0;
#pragma unroll
    for (int r2 = 0; r2 < kMoeMaxK; ++r2) {
      const int e2 = __shfl_sync(0xffffffffu, e, r2);
      pos += (r2 < k && e2 < e) ? 1 : 0;
    }
    if (sel) {
      slots[t * (k + 1) + pos] = e;
      slot_w[t * k + pos] = w;
      if (e >= p.own.lo && e < p.own.hi) atomicOr(mask_s + e, 1u << t);
      if (blockIdx.x == 0) {
        if (p.ids_out) p.ids_out[t * k + r] = e;
        if (p.w_out) p.w_out[t * k + r] = w;
        if (p.slot_w_out) p.slot_w_out[t * k + pos] = w;
      }
    }
    if (r == 0) slots[t * (k + 1) + k] = p.shared_id;
  }
  __syncthreads();
}

// The group table from the experts' token masks (warp 0, then the CTA): one
// group per expert of [own.lo, own.hi) that some token chose, ascending, then
// the shared expert for the tokens of own.shared_mask; per (group, token) the
// slot row t*(k+1) + position; the groups' tile tables.
static __device__ __noinline__ void dc_groups(const DcParams &p, const int32_t *slots, const uint32_t *mask_s,
                                              int *gidx_s, int32_t *g_expert, uint32_t *g_mask, int32_t *g_dst,
                                              int *n_groups, const uint8_t **all_gu, const uint8_t **all_dn,
                                              const uint8_t **g_gu, const uint8_t **g_dn) {
  const int tid = threadIdx.x, lane = tid & 31, T = p.T, k = p.k, E = p.n_experts;
  if (T == 1) {
    // one token: its ascending slot list (routed experts, then the shared
    // one) is the group list, the slot position the group's destination row
    if (tid < 32) {
      const int e = lane <= k ? slots[lane] : -1;
      const bool mine = lane < k ? (e >= p.own.lo && e < p.own.hi) : (lane == k && e >= 0 && (p.own.shared_mask & 1u));
      const uint32_t b = __ballot_sync(0xffffffffu, mine);
      if (mine) {
        const int gi = __popc(b & ((1u << lane) - 1u));
        g_expert[gi] = e;
        g_mask[gi] = 1u;
        gidx_s[e] = gi;
        g_dst[gi] = lane;
        g_gu[gi] = all_gu[e];
        g_dn[gi] = all_dn[e];
      }
      if (lane == 0) *n_groups = __popc(b);
    }
    __syncthreads();
    return;
  }
  if (tid < 32) {
    int base = 0;
#pragma unroll 1
    for (int c = 0; c <= E; c += 32) {
      const int e = c + lane;
      const uint32_t m = e <= E ? mask_s[e] : 0u;
      const uint32_t b = __ballot_sync(0xffffffffu, m != 0u);
      if (m) {
        const int gi = base + __popc(b & ((1u << lane) - 1u));
        g_expert[gi] = e;
        g_mask[gi] = m;
        gidx_s[e] = gi;
        g_gu[gi] = all_gu[e];
        g_dn[gi] = all_dn[e];
      }
      base += __popc(b);
    }
    if (lane == 0) *n_groups = base;
  }
  __syncthreads();
#pragma unroll 1
  for (int pr = tid; pr < T * (k + 1); pr += kDcThreads) {
    const int t = pr / (k + 1), r = pr - t * (k + 1);
    const int ex = slots[pr];
    const bool mine = r < k ? (ex >= p.own.lo && ex < p.own.hi) : (ex >= 0 && ((p.own.shared_mask >> t) & 1u));
    if (mine) g_dst[gidx_s[ex] * T + t] = pr;
  }
  __syncthreads();
}

// ------------------------------------------------------------- kernel ---
template <int NTB>
__global__ void __launch_bounds__(kDcThreads, 1) rc_moe_decode_kernel(DcParams p_arg) {
  extern __shared__ __align__(128) uint8_t smem[];
  // the parameters and the stream description are read by out-of-line
  // functions: shared-memory copies keep them off the thread stacks
  __shared__ DcParams p;
  __shared__ DcStream st;
  if (threadIdx.x == 0) p = p_arg;
  __syncthreads();
  int *ok_s = reinterpret_cast<int *>(smem + p.off_red + kDcWarps * kMoeMaxTokens * 8);
  uint8_t **ep_peer_s = reinterpret_cast<uint8_t **>(smem + p.off_red + kDcRedBytes);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int T = p.T, E = p.n_experts, k = p.k;
  const int gt_gu = p.inter / 8, kb_gu = p.hidden / kUnitK;
  const int gt_dn = p.hidden / kUnitRows, kb_dn = p.inter_pad / kUnitK;
  uint8_t *stage = smem + p.off_stage;
  dc_stamp(p, kTrStart);
  // Chaining: the next launch in the stream may start its CTAs as this
  // grid's CTAs leave their SMs (its prologue below reads only weights and
  // tables); it waits for this grid before it touches anything this grid
  // reads or writes.
  pdl_launch_dependents();

  // the lane's router slice of this CTA's first expert, in flight while the
  // tables load and the token rows are staged
  uint4 wpre = make_uint4(0, 0, 0, 0);
  if ((int)blockIdx.x < E && warp < p.hidden / kUnitK)
    wpre = __ldg(reinterpret_cast<const uint4 *>(p.wr + (size_t)blockIdx.x * p.hidden + warp * kUnitK + lane * 8));

  // The shared expert's weights do not depend on the routing: each CTA asks
  // L2 for its share of them now, so the stream finds them there.
  if (tid == 0 && p.shared_id >= 0 && p.own.shared_mask && p.gu_tiles[E] != nullptr) {
    const size_t gu_units = (size_t)gt_gu * kb_gu, dn_units = (size_t)gt_dn * kb_dn;
    const size_t a0 = gu_units * blockIdx.x / gridDim.x, a1 = gu_units * (blockIdx.x + 1) / gridDim.x;
    const size_t b0 = dn_units * blockIdx.x / gridDim.x, b1 = dn_units * (blockIdx.x + 1) / gridDim.x;
    if (a1 > a0) bulk_prefetch_l2(p.gu_tiles[E] + a0 * kUnitBytes, (uint32_t)((a1 - a0) * kUnitBytes));
    if (b1 > b0) bulk_prefetch_l2(p.dn_tiles[E] + b0 * kUnitBytes, (uint32_t)((b1 - b0) * kUnitBytes));
  }

  // the peer buffer table is fixed when the exchange is set up: read it now
  if (p.ep_world > 1 && tid < p.ep_world) ep_peer_s[tid] = p.ep_peer[tid];

  // the previous kernel in the stream (the producer of x, or the previous
  // call sharing this layer's counters and scratch) is complete from here on
  pdl_wait_prior();

  // ---- expert parallelism: every rank's token rows into every rank's buffer
  unsigned long long ep_calls = 0;
  if (p.ep_world > 1) {
    __syncthreads();
    // CTA r stores this rank's token rows into rank r's buffer and counts
    // them there: the ranks are served in parallel, one releasing add each
    // (the barrier orders the CTA's stores before thread 0's release)
    const int n16 = p.ep_M * p.hidden / 8;
    const uint4 *src = reinterpret_cast<const uint4 *>(p.ep_x_own);
#pragma unroll 1
    for (int r = blockIdx.x; r < p.ep_world; r += gridDim.x) {
      uint4 *dst = reinterpret_cast<uint4 *>(ep_peer_s[r] + p.ep_tok_off) + (size_t)p.ep_rank * n16;
      for (int i = tid; i < n16; i += blockDim.x) dst[i] = src[i];
      __syncthreads();
      if (tid == 0) red_add_release_sys(reinterpret_cast<unsigned long long *>(ep_peer_s[r]) + 0, 1ull);
    }
    // the calls made so far (the previous call of this layer wrote it)
    ep_calls = *reinterpret_cast<volatile unsigned long long *>(p.ep_flags + 2);
    if (tid == 0) p.ep_call = ep_calls;      // read by the down epilogue (after several barriers)
  }

  // per-expert tables kept in shared memory for the whole kernel
  const uint8_t **all_gu = reinterpret_cast<const uint8_t **>(smem + p.off_tab);    // [E+1]
  const uint8_t **all_dn = all_gu + (E + 1);
  const uint8_t **g_gu = all_dn + (E + 1);
  const uint8_t **g_dn = g_gu + (E + 1);
  float *bias_s = reinterpret_cast<float *>(g_dn + (E + 1));
  int32_t *g_expert = reinterpret_cast<int32_t *>(bias_s + (E + 1));
  uint32_t *g_mask = reinterpret_cast<uint32_t *>(g_expert + (E + 1));
  uint32_t *mask_s = g_mask + (E + 1);                                              // [E+1]
  int *gidx_s = reinterpret_cast<int *>(mask_s + (E + 1));                         // [E+1]
  int *n_groups_s = gidx_s + (E + 1);                                              // [4]
  int32_t *g_dst = n_groups_s + 4;                                                 // [E+1][T]
  // the tables are requested now and stored after the logits, so their
  // latency hides behind the router (E + 1 <= 512 entries, one per thread)
  const uint8_t *tab_gu = nullptr, *tab_dn = nullptr;
  float tab_bias = 0.f;
  if (tid <= E) {
    tab_gu = p.gu_tiles[tid];
    tab_dn = p.dn_tiles[tid];
    if (tid < E) tab_bias = p.bias[tid];
  }
  if (p.ep_world > 1) {
    if (!dc_wait_sys(p.ep_flags + 0, (ep_calls + 1) * p.ep_world, p.err, ok_s)) return;
    dc_stamp(p, kTrTokens);
  } else if (p.trace && tid == 0) {
    p.trace[(size_t)blockIdx.x * kTracePhases + kTrTokens] = 0;
  }

  // ------------------------------------------- 1 stage, 2 logits
  // warps 0 .. nlog-1 compute the logits while the others stage the tokens
  // (all warps stage after the logits when the slices take every warp)
  const int nlog = kb_gu < kDcWarps ? kb_gu : kDcWarps;
  if (nlog < kDcWarps) {
    if (warp >= nlog) dc_stage(p.x, p.hidden, 0, 1, T, kb_gu, stage, warp - nlog, kDcWarps - nlog);
    else dc_logits(p, reinterpret_cast<double *>(smem + p.off_red), wpre, nlog);
  } else {
    dc_logits(p, reinterpret_cast<double *>(smem + p.off_red), wpre, nlog);
    dc_stage(p.x, p.hidden, 0, 1, T, kb_gu, stage, warp, kDcWarps);
  }
  if (tid <= E) {
    all_gu[tid] = tab_gu;
    all_dn[tid] = tab_dn;
    bias_s[tid] = tab_bias;
    mask_s[tid] = tid == E ? p.own.shared_mask : 0u;
  }
  dc_stamp(p, kTrLogits);
  if (!dc_grid_barrier(p.bar, p.err, ok_s)) return;
  dc_stamp(p, kTrRouted);

  // -------------------------------------------------------- 3 selection
  int32_t *slots = reinterpret_cast<int32_t *>(smem + p.off_sel);                   // [T][k+1]
  float *slot_w = reinterpret_cast<float *>(slots + T * (k + 1));                   // [T][k]
  int32_t *sel_e = reinterpret_cast<int32_t *>(slot_w + T * k);                     // [T][k]
  float *sel_sc = reinterpret_cast<float *>(sel_e + T * k);                         // [T][k]
  // the unit buffer is free until the first chunk is requested: key scratch
  dc_select(p, bias_s, smem + p.off_buf, slots, slot_w, sel_e, sel_sc, mask_s);
  dc_groups(p, slots, mask_s, gidx_s, g_expert, g_mask, g_dst, n_groups_s, all_gu, all_dn, g_gu, g_dn);
  dc_stamp(p, kTrSelected);

  // ------------------------------------------- 4 partitions and stream
  const int ng = *n_groups_s;
  const int tot_gu = ng * gt_gu, tot_dn = ng * gt_dn;
  const int per_gu = (tot_gu + (int)gridDim.x - 1) / (int)gridDim.x;
  // column-major down: CTA c owns output column tile c of every group
  const int per_dn = p.col_down ? ng : (tot_dn + (int)gridDim.x - 1) / (int)gridDim.x;
  const int c0_gu = blockIdx.x * per_gu, c0_dn = blockIdx.x * per_dn;
  const int nt_gu = c0_gu < tot_gu ? (c0_gu + per_gu < tot_gu ? per_gu : tot_gu - c0_gu) : 0;
  const int nt_dn = c0_dn < tot_dn ? (c0_dn + per_dn < tot_dn ? per_dn : tot_dn - c0_dn) : 0;
  if (tid == 0) {
    st.g_ptr[0] = g_gu;
    st.g_ptr[1] = g_dn;
    st.c0[0] = c0_gu;
    st.c0[1] = c0_dn;
    st.nt[0] = nt_gu;
    st.nt[1] = nt_dn;
    st.kb[0] = kb_gu;
    st.kb[1] = kb_dn;
    st.gt[0] = gt_gu;
    st.gt[1] = gt_dn;
    st.units0 = nt_gu * kb_gu;
    st.units = st.units0 + nt_dn * kb_dn;
    st.nchunk = (st.units + kDcChunk - 1) / kDcChunk;
    st.col = p.col_down;
    st.ng = ng;
  }
  const int B = p.chunk_slots;
  const uint32_t bar0 = smem_addr(smem + p.off_bar);
  if (tid < B) mbar_init(bar0 + 8 * tid, 1);
  mbar_fence_init();
  __syncthreads();            // the barriers are initialised; the selection scratch in the ring is dead
  // chunks requested so far (the same count in every thread); chunk j by warp
  // j % 16.  Every chunk the ring holds is requested now, the gate/up ones
  // first in the stream; the rest follow as rounds free their slots.
  int issued = st.nchunk < B ? st.nchunk : B;
  if (lane == 0) {
#pragma unroll 1
    for (int j = warp; j < issued; j += kDcWarps) dc_issue_chunk(st, j, smem + p.off_buf, bar0, B);
  }
  // expert parallelism: zero the slot rows other ranks compute
  if (p.zero_foreign) {
    const int rows = T * (k + 1);
#pragma unroll 1
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {
      const int t = r / (k + 1), pos = r - t * (k + 1);
      const int e = slots[r];
      const bool mine = pos < k ? (e >= p.own.lo && e < p.own.hi) : (e >= 0 && ((p.own.shared_mask >> t) & 1u));
      if (mine) continue;
      uint4 *dst = reinterpret_cast<uint4 *>(p.slot_rows + (size_t)r * p.hidden);
#pragma unroll 1
      for (int i = tid; i < p.hidden / 8; i += blockDim.x) dst[i] = make_uint4(0, 0, 0, 0);
    }
  }
  dc_stamp(p, kTrStaged);

  // ------------------------------------------------------------ 5 gate/up
  bool failed = false;
  int rv = dc_rounds<NTB>(p, smem, st, 0, stage, 1, g_mask, g_dst, 0, issued, failed, ng, slot_w);
  issued = rv >> 1;
  failed = (rv & 1) != 0;
  // every gate/up unit is consumed (also in a CTA without gate/up tiles): the
  // down chunks take the free slots
  if (!failed) issued = dc_refill(st, issued, st.units0 / kDcChunk, smem + p.off_buf, bar0, B);
  dc_stamp(p, kTrGateUp);
  if (!failed && !dc_grid_barrier(p.bar, p.err, ok_s)) failed = true;
  dc_stamp(p, kTrActReady);

  // --------------------------------------------------------------- 6 down
  if (!failed) {
    const int g_lo = p.col_down ? 0 : c0_dn / gt_dn;
    const int g_hi = nt_dn ? (p.col_down ? ng - 1 : (c0_dn + nt_dn - 1) / gt_dn) : g_lo - 1;
    const int nblk = g_hi - g_lo + 1;
    if (nblk > 0)
      dc_stage(p.act + (size_t)g_lo * 8 * NTB * p.inter_pad, p.inter_pad, 8 * NTB, nblk, T, kb_dn, stage, warp,
               kDcWarps);
    __syncthreads();
    dc_stamp(p, kTrActStaged);
    rv = dc_rounds<NTB>(p, smem, st, 1, stage, nblk > 0 ? nblk : 1, g_mask, g_dst, g_lo, issued, failed, ng,
                        slot_w);
    issued = rv >> 1;
    failed = (rv & 1) != 0;
    if (!failed && p.col_down && nt_dn > 0) {
      // every expert row of column tile blockIdx.x is in this CTA: combine it
      // for every token straight from shared memory
      __syncthreads();
      const uint16_t *rows_s = reinterpret_cast<const uint16_t *>(stage);
      const bool with_shared = p.shared_id >= 0 && p.own.shared_mask;
      if (tid < 2 * T) {
        const int t = tid >> 1, h = tid & 1;
        *reinterpret_cast<uint4 *>(p.out + (size_t)t * p.hidden + blockIdx.x * kUnitRows + h * 8) =
            dc_combine8<true>(rows_s + (size_t)t * (k + 1) * kUnitRows + h * 8, kUnitRows, k, slot_w + t * k,
                              with_shared);
      }
    }
  }
  dc_stamp(p, kTrDown);
  if (p.ep_world > 1) {
    // expert parallelism: every expert row of this rank's tokens arrives
    // tagged with the call's number; thread (t, g) of a column tile waits for
    // rows g and g + 8 of every slot of token t, then combines them
    const bool with_shared = p.shared_id >= 0 && p.own.shared_mask;
    const unsigned long long *red =
        reinterpret_cast<const unsigned long long *>(ep_peer_s[p.ep_rank] + p.ep_red_off);
    if (tid == 0) *ok_s = 1;
    __syncthreads();
    const uint64_t tw = global_timer_ns();
#pragma unroll 1
    for (int c = blockIdx.x; c < gt_dn && !failed; c += gridDim.x) {
      if (p.out && tid < 8 * p.ep_M) {
        const int t = tid >> 3, g = tid & 7;
        if (!dc_combine_tagged(red + ((size_t)t * (k + 1) * gt_dn + c) * 8 + g, (size_t)gt_dn * 8, k,
                               slot_w + (p.ep_rank * p.ep_M + t) * k, with_shared, (uint32_t)(ep_calls + 1), tw,
                               p.out + (size_t)t * p.hidden + c * kUnitRows + g)) {
          atomicCAS(p.err, 0, kErrWaitTimeout);
          *ok_s = 0;
        }
      }
      __syncthreads();
      if (!*ok_s) failed = true;
    }
    dc_stamp(p, kTrRows);
  } else {
    // one GPU: the down phase combined each column tile as its last tile was written
    dc_stamp(p, kTrRows);
  }
  if (p.ep_world > 1 && !failed && blockIdx.x == 0 && tid == 0)
    *reinterpret_cast<volatile unsigned long long *>(p.ep_flags + 2) = ep_calls + 1;
  __syncthreads();
  dc_stamp(p, kTrEnd);
  // after a failure, the chunks still in flight land before the CTA's shared
  // memory is released: every slot's last requested chunk is waited for
  if (failed && tid == 0) {
#pragma unroll 1
    for (int j = issued - B > 0 ? issued - B : 0; j < issued; ++j)
      mbar_wait_bounded(bar0 + 8 * (j % B), (uint32_t)(j / B) & 1u);
  }
}

// ------------------------------------------------------------------- host --
struct DcLayout {
  int chunk_slots, round_units, stage_blk;
  int off_buf, off_stage, off_part, off_tab, off_sel, off_red, off_bar, smem;
};

static int dc_max_groups(int T, int k, const MoeOwned &own) {
  const int owned = own.hi - own.lo;
  return (T * k < owned ? T * k : owned) + (own.shared_mask ? 1 : 0);
}

// Shared-memory layout of one call.  Fixed parts: the staging area (token
// fragments, or the act fragments of the groups one CTA's down range can
// touch), the tables, the selection lists, the reduction area.  The rest is
// split between the unit ring (B chunk slots) and the round partials, a
// round holding at most B - 1 chunks of units and at least one tile of
// either phase.
// Column-major down (every group of one output column tile in one CTA,
// combined there): on one GPU with an output, when the output column tiles
// do not outnumber the CTAs and every group's activations of few tokens fit
// a small staging area.  The layout must also hold a CTA's units in one round.
static bool dc_col_down(const rc_moe *m, int T, int k, const MoeOwned &own) {
  const int gt_dn = m->hidden / kUnitRows, kb_dn = m->inter_pad / kUnitK;
  return gt_dn <= m->ctx->sm_count && dc_stage_bytes(dc_max_groups(T, k, own), T, kb_dn) <= 32 * 1024;
}

static bool dc_layout(const rc_moe *m, int T, int k, const MoeOwned &own, bool col, DcLayout *L) {
  const int ntb = T <= 8 ? 1 : 2, E = m->n_experts, grid = m->ctx->sm_count;
  const int hidden = m->hidden, inter_pad = m->inter_pad;
  const int kb_gu = hidden / kUnitK, kb_dn = inter_pad / kUnitK, gt_dn = hidden / kUnitRows;
  const int mg = dc_max_groups(T, k, own);
  const int per_dn = col ? mg : (mg * gt_dn + grid - 1) / grid;
  int blk = col ? mg : 1 + (per_dn + gt_dn - 2) / gt_dn;   // groups a CTA's down range can touch
  if (blk > mg) blk = mg > 0 ? mg : 1;
  size_t stage = dc_stage_bytes(1, T, kb_gu);
  const size_t st_a = dc_stage_bytes(blk, T, kb_dn);
  if (st_a > stage) stage = st_a;
  const size_t tab = (size_t)(E + 1) * (4 * 8 + 4 * 5 + 4 * T) + 16;
  const size_t sel = (size_t)T * (k + 1) * 4 + (size_t)T * k * 4 * 3;
  const size_t red = (size_t)kDcRedBytes + kEpMaxRanks * 8;
  const size_t pb = (size_t)128 * (dc_qn(T, 0) + (ntb == 2 ? dc_qn(T, 1) : 0));
  const int need = kb_gu > kb_dn ? kb_gu : kb_dn;           // units of the widest tile
  const size_t fixed = (stage + 15) / 16 * 16 + (tab + 15) / 16 * 16 + (sel + 15) / 16 * 16 +
                       (red + 15) / 16 * 16 + (size_t)kDcMaxChunks * 8;
  if (fixed >= (size_t)kDcSmemLimit) return false;
  const size_t rest = (size_t)kDcSmemLimit - fixed;
  if (col && (size_t)T * (k + 1) * kUnitRows * 2 > stage) return false;
  for (int B = kDcMaxChunks; B >= 2; --B) {
    const int ru = (B - 1) * kDcChunk;
    if (ru < need || (col && ru < per_dn * kb_dn)) break;
    const size_t bytes = (size_t)B * kDcChunk * kUnitBytes + ((size_t)ru * pb + 15) / 16 * 16;
    if (bytes > rest) continue;
    // the selection scratch (T*E keys and scores) lives in the unit ring
    if ((size_t)T * (E + 4) * 8 > (size_t)B * kDcChunk * kUnitBytes) continue;
    size_t off = 0;
    const size_t o_buf = off;
    off += (size_t)B * kDcChunk * kUnitBytes;
    const size_t o_stage = off;
    off += (stage + 15) / 16 * 16;
    const size_t o_part = off;
    off += ((size_t)ru * pb + 15) / 16 * 16;
    const size_t o_tab = off;
    off += (tab + 15) / 16 * 16;
    const size_t o_sel = off;
    off += (sel + 15) / 16 * 16;
    const size_t o_red = off;
    off += (red + 15) / 16 * 16;
    const size_t o_bar = off;
    off += (size_t)kDcMaxChunks * 8;
    *L = DcLayout{B, ru, blk, (int)o_buf, (int)o_stage, (int)o_part, (int)o_tab, (int)o_sel, (int)o_red,
                  (int)o_bar, (int)off};
    return true;
  }
  return false;
}

bool moe_decode_shape_ok(const rc_moe *m, int T, int k, const MoeOwned &own) {
  if (m->down_fmt != kFormatQ4nx) return false;   // q4nx unit arithmetic only
  DcLayout L;
  return dc_layout(m, T, k, own, false, &L);
}

int moe_decode_persistent(rc_moe *m, const uint16_t *x, int T, int k, int router, int renorm, float scaling,
                          int act, float gb, float vb, const MoeOwned &own, uint16_t *slot_rows, int zero_foreign,
                          uint16_t *out, int32_t *ids_out, float *w_out, float *slot_w_out, cudaStream_t s,
                          const MoeEpArgs *ep) {
  const int ntb = T <= 8 ? 1 : 2;
  DcLayout L;
  const bool col = ep == nullptr && out != nullptr && !zero_foreign && dc_col_down(m, T, k, own) &&
                   dc_layout(m, T, k, own, true, &L);
  if (!col && !dc_layout(m, T, k, own, false, &L)) {
    set_error("MoE decode: no shared-memory layout for T=%d k=%d", T, k);
    return RC_ERR_INVALID;
  }
  rc_ctx *ctx = m->ctx;
  const size_t cols_bytes = (size_t)(m->hidden / kUnitRows) * sizeof(int);
  if (!m->fz_bar) {
    RC_CUDA_TRY(cudaMalloc(&m->fz_bar, sizeof(unsigned long long)));
    RC_CUDA_TRY(cudaMemset(m->fz_bar, 0, sizeof(unsigned long long)));
    m->fz_epoch = ctx->timeout_epoch;
  }
  if (!m->dc_cols) {
    RC_CUDA_TRY(cudaMalloc(&m->dc_cols, cols_bytes));
    RC_CUDA_TRY(cudaMemset(m->dc_cols, 0, cols_bytes));
  }
  if (m->fz_epoch != ctx->timeout_epoch) {
    // a bounded wait gave up since the last launch: the arrival count and
    // the column counters may be left over from that launch
    RC_CUDA_TRY(cudaMemsetAsync(m->fz_bar, 0, sizeof(unsigned long long), s));
    RC_CUDA_TRY(cudaMemsetAsync(m->dc_cols, 0, cols_bytes, s));
    m->fz_epoch = ctx->timeout_epoch;
  }
  DcParams p{};
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
  p.chunk_slots = L.chunk_slots;
  p.round_units = L.round_units;
  p.stage_blk = L.stage_blk;
  p.col_down = col ? 1 : 0;
  p.off_buf = L.off_buf;
  p.off_stage = L.off_stage;
  p.off_part = L.off_part;
  p.off_tab = L.off_tab;
  p.off_sel = L.off_sel;
  p.off_red = L.off_red;
  p.off_bar = L.off_bar;
  p.bar = m->fz_bar;
  p.cols = m->dc_cols;
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
      RC_CUDA_TRY(cudaFuncSetAttribute(rc_moe_decode_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kDcSmemLimit));
    else
      RC_CUDA_TRY(cudaFuncSetAttribute(rc_moe_decode_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kDcSmemLimit));
    if (dev < 64) configured[dev][ntb - 1] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctx->sm_count);
  cfg.blockDim = dim3(kDcThreads);
  cfg.dynamicSmemBytes = L.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;      // every CTA resident: the grid barriers are safe
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (ntb == 1)
    RC_CUDA_TRY(cudaLaunchKernelEx(&cfg, rc_moe_decode_kernel<1>, p));
  else
    RC_CUDA_TRY(cudaLaunchKernelEx(&cfg, rc_moe_decode_kernel<2>, p));
  return RC_OK;
}

// Whether the persistent kernel takes this call: it is switched on
// (rc_moe_set_fused) and the shape is one it can run.
bool moe_fused_fits(const rc_moe *m, int T, int k, const MoeOwned &own) {
  return m->fused && moe_decode_shape_ok(m, T, k, own);
}

}  // namespace rc
