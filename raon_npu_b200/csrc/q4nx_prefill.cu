// MoE prefill on the q4nx experts: a grouped GEMM on the 5th-generation
// tensor cores (tcgen05, accumulators in tensor memory).
//
// Reference semantics are the decode path's (host/backend.py:466-510 per
// token; the grouped combine of kernels/moe_grouped/planner.py:286-322):
// gate/up linear (bf16), act -> RTNE, down linear (bf16), routed outputs
// summed in ascending expert ID in f32 then RTNE, plus the shared expert.
//
// Pipeline for T tokens (T <= 4096):
//   logits    f64 sums of exact bf16 products, rounded once to f32 (as decode)
//   select    one warp per token: top-k (lower index wins ties), weights,
//             ascending-ID slot list
//   plan      one CTA: per-expert token bitmaps -> expert-sorted row order
//             (tokens ascending within an expert), 64-row chunks
//   gate/up   tcgen05 grouped GEMM, epilogue GLU -> act rows (permuted order)
//   down      tcgen05 grouped GEMM -> down rows (permuted order)
//   combine   per token, its slot rows in ascending ID (f32 multiply, then
//             add, no FMA), RTNE, plus the shared row
//
// The grouped GEMM (one CTA per SM, persistent over work items (64-row chunk
// of one expert, 128-row weight tile), a k-block of 256 columns per step):
//   A  weight tile: the q4nx codes of 128 rows x 256 columns arrive by bulk
//      copy in the t16 upload layout and are written to shared memory as
//      bf16 (128 + code) -- exact -- in the 128-byte-swizzled K-major layout
//      the tensor core reads;
//   B  the chunk's 64 source rows x 256 columns: a gather pass first copies
//      the token rows into permuted order (the down GEMM's act rows already
//      are), so a chunk's rows are contiguous and arrive as four 64 x 64
//      TMA boxes in the same swizzle; the rows' per-32-column group sums S
//      (computed by that pass) arrive as a fifth box;
//   D  one tcgen05.mma chain of K = 32 per quantisation group into its own
//      tensor-memory accumulator (8 groups x 64 columns = 512 columns);
//   promotion: the thread of weight row r (TMEM lane r) reads the group
//      accumulators with tcgen05.ld and adds scale * D + (min - 128 scale) * S
//      in f32 registers -- the same arithmetic as the decode GEMV and as the
//      reference NPU kernel's per-group scaling (grouped_mmul.cc:196-254).
// Loads, expansion, MMAs and promotion run in different warps on mbarrier
// rings (see rc_pf_tc_kernel).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <string.h>

#include "moe_internal.cuh"
#include "q4nx_core.cuh"
#include "rc_device.cuh"
#include "rc_internal.cuh"

namespace rc {

constexpr int kPfRows = 128;         // weight rows per tile: MMA M, TMEM lanes
constexpr int kPfCols = 64;          // token columns per work item: max MMA N
constexpr int kPfBlk = 8;            // token rows per block of the register-fragment (mma.sync) path
constexpr int kPfTmemCols = 512;     // 8 group accumulators x 64 columns
constexpr int kPfGroups = 8;         // 32-column quantisation groups per 256-column block

// operand tiles of the tensor-core kernel
constexpr int kPfASub = kPfRows * 128;               // A: [128 rows x 128 B] per 64-column sub-tile
constexpr int kPfBSub = kPfCols * 128;               // B: [64 rows x 128 B] per 64-column sub-tile
constexpr int kPfBStage = 4 * kPfBSub;               // B of one 256-column k-block
constexpr int kPfUStage = 8 * kUnitBytes;            // the 8 units of a 128-row tile's k-block
constexpr int kPfPlanSmemMax = kGemvSmemLimit - 8 * 1024;   // dynamic part of the plan kernel (static: ~4.1 KB)

struct PfScratch {
  int T_cap, P_cap, chunk_cap, blk_cap, E1;
  float *logits;            // [T][E]
  int32_t *ids;             // [T][k] rank order
  float *weights;           // [T][k]
  int32_t *slot_expert;     // [T][k+1] ascending ID, then the shared expert (or -1)
  float *slot_w;            // [T][k]
  int32_t *slot_row;        // [T][k+1] permuted row of each slot, -1 if not computed here
  int32_t *row_token;       // [P] token of each permuted row
  int32_t *cnt, *off;       // [E+1]
  int32_t *n_chunks;        // [2]: 64-row chunks, 8-row blocks
  int32_t *chunk_expert, *chunk_row0, *chunk_n;
  uint16_t *act;            // [P][inter_pad]
  uint16_t *down;           // [P][hidden]
  int32_t *blk_expert, *blk_row0, *blk_n;   // 8-row token blocks of the permuted rows
  uint32_t *xf;             // the blocks' staged activations (f16 fragments), for K up to max(hidden, inter_pad)
  void *xaux;               // and their aux words
  uint16_t *x_perm;         // [P][hidden] token rows in permuted order (the gate/up GEMM's B rows)
  float *ssum_x, *ssum_act; // group sums of x_perm / act rows: [P][hidden / 32], [P][inter_pad / 32]
  CUtensorMap tm_x, tm_act, tm_sx, tm_sact;   // TMA maps of those four arrays (64-row boxes)
};

// ------------------------------------------------------------ small PTX --
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Descriptor of a K-major operand tile in the 128-byte swizzle layout: rows
// 128 B apart, 8-row groups 1024 B apart (version 1, SWIZZLE_128B).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor: f32 accumulator, bf16 A and B, both K-major, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// Byte offset of element (r, kk) (kk < 64) in a 128-byte-swizzled K-major tile.
__device__ __forceinline__ uint32_t sw128_off(int r, int kk) {
  return (r >> 3) * 1024 + (r & 7) * 128 + ((((kk >> 3) ^ r) & 7) << 4) + (kk & 7) * 2;
}
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(da), "l"(db), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t addr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(addr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- router --
// logits[t][e] = f32(sum_h f64(x[t][h]) * f64(wr[e][h])).  A CTA takes 8
// experts x 8*tpw tokens: the experts' router rows are staged in shared
// memory once and reused by all its tokens; each warp takes tpw tokens (4,
// or 2 when T is small, so the grid still fills the SMs), two at a time,
// each lane 8 columns per 256-column step, one f64 accumulator per (token,
// expert).  A token's sums do not depend on which warp takes it.
constexpr int kPfLogitExperts = 8, kPfLogitMaxTpw = 4;

__global__ void __launch_bounds__(256) rc_pf_logits_kernel(const uint16_t *x, int T, int hidden, const uint16_t *wr,
                                                        int E, float *logits, int tpw) {
  extern __shared__ __align__(16) uint8_t pf_logit_smem[];
  uint4 *w_s = reinterpret_cast<uint4 *>(pf_logit_smem);    // [8][hidden/8]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e0 = blockIdx.x * kPfLogitExperts, t0 = blockIdx.y * 8 * tpw;
  const int v8 = hidden / 8;
  for (int i = threadIdx.x; i < kPfLogitExperts * v8; i += blockDim.x) {
    const int ei = i / v8, c = i - ei * v8;
    w_s[i] = e0 + ei < E ? __ldg(reinterpret_cast<const uint4 *>(wr + (size_t)(e0 + ei) * hidden) + c)
                         : make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  // tokens in pairs: each router value is widened once for both tokens (the
  // widening runs on the f64 pipe like the sums); a token's sums are the same
  // chain of fused multiply-adds whether it is paired or not
  for (int tt = 0; tt < tpw; tt += 2) {
    const int ta = t0 + warp * tpw + tt;
    if (ta >= T) break;
    const bool two = tt + 1 < tpw && ta + 1 < T;
    const int tb = two ? ta + 1 : ta;
    double acc0[kPfLogitExperts], acc1[kPfLogitExperts];
#pragma unroll
    for (int ei = 0; ei < kPfLogitExperts; ++ei) acc0[ei] = acc1[ei] = 0.0;
    const uint4 *xra = reinterpret_cast<const uint4 *>(x + (size_t)ta * hidden);
    const uint4 *xrb = reinterpret_cast<const uint4 *>(x + (size_t)tb * hidden);
    // the next two slices of both rows are in flight while one is summed
    uint4 na = lane < v8 ? __ldg(xra + lane) : make_uint4(0, 0, 0, 0);
    uint4 nb = lane < v8 ? __ldg(xrb + lane) : make_uint4(0, 0, 0, 0);
    uint4 na2 = lane + 32 < v8 ? __ldg(xra + lane + 32) : make_uint4(0, 0, 0, 0);
    uint4 nb2 = lane + 32 < v8 ? __ldg(xrb + lane + 32) : make_uint4(0, 0, 0, 0);
    for (int c = lane; c < v8; c += 32) {
      const uint4 xa = na, xb = nb;
      na = na2;
      nb = nb2;
      if (c + 64 < v8) {
        na2 = __ldg(xra + c + 64);
        nb2 = __ldg(xrb + c + 64);
      }
      const uint32_t xsa[4] = {xa.x, xa.y, xa.z, xa.w}, xsb[4] = {xb.x, xb.y, xb.z, xb.w};
      double xda[8], xdb[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        xda[2 * j] = (double)bf16_to_f32(xsa[j] & 0xFFFFu);
        xda[2 * j + 1] = (double)bf16_to_f32(xsa[j] >> 16);
        xdb[2 * j] = (double)bf16_to_f32(xsb[j] & 0xFFFFu);
        xdb[2 * j + 1] = (double)bf16_to_f32(xsb[j] >> 16);
      }
#pragma unroll
      for (int ei = 0; ei < kPfLogitExperts; ++ei) {
        const uint4 wa = w_s[ei * v8 + c];
        const uint32_t ws[4] = {wa.x, wa.y, wa.z, wa.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const double wl = (double)bf16_to_f32(ws[j] & 0xFFFFu), wh = (double)bf16_to_f32(ws[j] >> 16);
          acc0[ei] = fma(xda[2 * j], wl, acc0[ei]);
          acc0[ei] = fma(xda[2 * j + 1], wh, acc0[ei]);
          acc1[ei] = fma(xdb[2 * j], wl, acc1[ei]);
          acc1[ei] = fma(xdb[2 * j + 1], wh, acc1[ei]);
        }
      }
    }
#pragma unroll
    for (int ei = 0; ei < kPfLogitExperts; ++ei) {
      double a0 = acc0[ei], a1 = acc1[ei];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        a0 += __shfl_xor_sync(0xffffffffu, a0, o);
        a1 += __shfl_xor_sync(0xffffffffu, a1, o);
      }
      if (lane == 0 && e0 + ei < E) {
        logits[(size_t)ta * E + e0 + ei] = __double2float_rn(a0);
        if (two) logits[(size_t)tb * E + e0 + ei] = __double2float_rn(a1);
      }
    }
  }
}

struct PfSelectParams {
  const float *logits;
  const float *bias;
  int T, E, k, mode, renorm, shared_id;
  float scaling;
  int32_t *ids;
  float *weights;
  int32_t *slot_expert;
  float *slot_w;
};

// One warp per token: k rounds of warp argmax (lower index wins ties), the
// routing weights, the ascending-ID slot list.
__global__ void __launch_bounds__(256) rc_pf_select_kernel(PfSelectParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= p.T) return;
  const float *lg = p.logits + (size_t)t * p.E;
  constexpr int kPer = kMoeMaxExperts / 32;
  float val[kPer], score[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int ei = lane + 32 * i;
    val[i] = -INFINITY;
    score[i] = 0.f;
    if (ei < p.E) {
      const float l = lg[ei];
      if (p.mode == RC_ROUTER_SIGMOID_BIAS) {
        score[i] = __double2float_rn(1.0 / (1.0 + exp(-(double)l)));
        val[i] = score[i] + p.bias[ei];
      } else {
        score[i] = l + p.bias[ei];
        val[i] = score[i];
      }
    }
  }
  int sel[kMoeMaxK];
  float sel_score[kMoeMaxK];
  uint32_t live = 0u;                 // bit i: expert lane + 32 i still selectable
#pragma unroll
  for (int i = 0; i < kPer; ++i)
    if (lane + 32 * i < p.E) live |= 1u << i;
#pragma unroll 1
  for (int r = 0; r < p.k; ++r) {
    float bv = 0.f;
    int bi = -1;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int ei = lane + 32 * i;
      if (((live >> i) & 1u) && (bi < 0 || route_before(val[i], ei, bv, bi))) bv = val[i], bi = ei;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi >= 0 && (bi < 0 || route_before(ov, oi, bv, bi))) bv = ov, bi = oi;
    }
    float sc = 0.f;
#pragma unroll
    for (int i = 0; i < kPer; ++i)
      if (lane + 32 * i == bi) sc = score[i], live &= ~(1u << i);
    sc = __shfl_sync(0xffffffffu, sc, bi & 31);
    if (lane == 0) {
      sel[r] = bi;
      sel_score[r] = sc;
    }
  }
  if (lane != 0) return;
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
    const float mx = sel_score[0];
    float sum = 0.f;
    for (int r = 0; r < p.k; ++r) sum += expf(sel_score[r] - mx);
    for (int r = 0; r < p.k; ++r) w[r] = expf(sel_score[r] - mx) / sum;
  }
  for (int r = 0; r < p.k; ++r) {
    p.ids[(size_t)t * p.k + r] = sel[r];
    p.weights[(size_t)t * p.k + r] = w[r];
  }
  int32_t *se = p.slot_expert + (size_t)t * (p.k + 1);
  float *sw = p.slot_w + (size_t)t * p.k;
  for (int r = 0; r < p.k; ++r) {   // ascending ID: position = number of smaller selected ids
    int pos = 0;
    for (int r2 = 0; r2 < p.k; ++r2) pos += sel[r2] < sel[r] ? 1 : 0;
    se[pos] = sel[r];
    sw[pos] = w[r];
  }
  se[p.k] = p.shared_id;
}

// Caller-supplied routes ids / w [T][k]: ascending-ID slot lists.
__global__ void rc_pf_slots_kernel(const int32_t *ids, const float *w, int T, int k, int shared_id, int32_t *slot_expert,
                                float *slot_w) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const int32_t *id = ids + (size_t)t * k;
  for (int r = 0; r < k; ++r) {
    int pos = 0;
    for (int r2 = 0; r2 < k; ++r2) pos += id[r2] < id[r] ? 1 : 0;
    slot_expert[(size_t)t * (k + 1) + pos] = id[r];
    slot_w[(size_t)t * k + pos] = w[(size_t)t * k + r];
  }
  slot_expert[(size_t)t * (k + 1) + k] = shared_id;
}

// ------------------------------------------------------------------ plan --
struct PfPlanParams {
  const int32_t *slot_expert;   // [T][k+1]
  int T, k, E1;                 // E1 = experts + 1 (index E = shared)
  int max_id;                   // caller routes name experts < max_id (E, or E + 1: the shared one too)
  int lo, hi;                   // routed experts computed here
  int st0, st1;                 // tokens whose shared expert is computed here
  int32_t *slot_row, *row_token, *cnt, *off, *n_chunks, *chunk_expert, *chunk_row0, *chunk_n;
  int chunk_cap;
  int32_t *blk_expert, *blk_row0, *blk_n;
  int blk_cap;
  int *err;
};

// One CTA.  Permuted rows are ordered by expert, then token: the row of
// (token t, expert e) is off[e] + #{t' < t choosing e}, counted with
// per-expert token bitmaps -- deterministic, independent of thread timing.
__global__ void __launch_bounds__(1024) rc_pf_plan_kernel(PfPlanParams p) {
  extern __shared__ uint32_t pf_plan_smem[];
  const int nw = (p.T + 31) / 32;
  uint32_t *mask = pf_plan_smem;                 // [E1][nw]
  uint32_t *pre = mask + (size_t)p.E1 * nw;      // [E1][nw] exclusive prefix popcounts
  __shared__ int s_cnt[kMoeMaxExperts + 1], s_off[kMoeMaxExperts + 1], s_cofs[kMoeMaxExperts + 1],
      s_bofs[kMoeMaxExperts + 1];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, nwarps = blockDim.x >> 5;
  const int k1 = p.k + 1;
  auto computed = [&](int t, int r, int e) {
    if (e < 0) return false;
    return r < p.k ? (e >= p.lo && e < p.hi) : (t >= p.st0 && t < p.st1);
  };
  for (int i = tid; i < p.E1 * nw; i += blockDim.x) mask[i] = 0u;
  __syncthreads();
  for (int i = tid; i < p.T * k1; i += blockDim.x) {
    const int t = i / k1, r = i - t * k1;
    const int e = p.slot_expert[i];
    if (r < p.k && (e < 0 || e >= p.max_id)) atomicCAS(p.err, 0, kErrBadExpert);   // caller id out of range
    else if (computed(t, r, e)) atomicOr(mask + (size_t)e * nw + (t >> 5), 1u << (t & 31));
  }
  __syncthreads();
  // per expert: exclusive prefix of popcounts over its words (one warp per expert)
  for (int e = warp; e < p.E1; e += nwarps) {
    int base = 0;
    for (int w0 = 0; w0 < nw; w0 += 32) {
      const int w = w0 + lane;
      const int c = w < nw ? __popc(mask[(size_t)e * nw + w]) : 0;
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (w < nw) pre[(size_t)e * nw + w] = base + incl - c;
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) s_cnt[e] = base;
  }
  __syncthreads();
  if (warp == 0) {
    // expert offsets and chunk offsets (ascending expert ID; the shared expert last)
    int base = 0, cbase = 0, bbase = 0;
    for (int e0 = 0; e0 < p.E1; e0 += 32) {
      const int e = e0 + lane;
      const int c = e < p.E1 ? s_cnt[e] : 0;
      const int nc = (c + kPfCols - 1) / kPfCols, nb = (c + kPfBlk - 1) / kPfBlk;
      int incl = c, cincl = nc, bincl = nb;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        const int cv = __shfl_up_sync(0xffffffffu, cincl, o);
        const int bv = __shfl_up_sync(0xffffffffu, bincl, o);
        if (lane >= o) incl += v, cincl += cv, bincl += bv;
      }
      if (e < p.E1) {
        s_off[e] = base + incl - c;
        s_cofs[e] = cbase + cincl - nc;
        s_bofs[e] = bbase + bincl - nb;
        p.cnt[e] = c;
        p.off[e] = base + incl - c;
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
      cbase += __shfl_sync(0xffffffffu, cincl, 31);
      bbase += __shfl_sync(0xffffffffu, bincl, 31);
    }
    if (lane == 0) {
      p.n_chunks[0] = cbase < p.chunk_cap ? cbase : p.chunk_cap;
      p.n_chunks[1] = bbase < p.blk_cap ? bbase : p.blk_cap;
      p.n_chunks[2] = base;                       // permuted rows in all
    }
  }
  __syncthreads();
  for (int i = tid; i < p.T * k1; i += blockDim.x) {
    const int t = i / k1, r = i - t * k1;
    const int e = p.slot_expert[i];
    int row = -1;
    if (!(r < p.k && (e < 0 || e >= p.max_id)) && computed(t, r, e)) {
      const uint32_t m = mask[(size_t)e * nw + (t >> 5)];
      row = s_off[e] + (int)pre[(size_t)e * nw + (t >> 5)] + __popc(m & ((1u << (t & 31)) - 1u));
      p.row_token[row] = t;
    }
    p.slot_row[i] = row;
  }
  for (int e = warp; e < p.E1; e += nwarps) {
    const int c = s_cnt[e], nc = (c + kPfCols - 1) / kPfCols, nb = (c + kPfBlk - 1) / kPfBlk;
    for (int j = lane; j < nc; j += 32) {
      const int ci = s_cofs[e] + j;
      if (ci < p.chunk_cap) {
        p.chunk_expert[ci] = e;
        p.chunk_row0[ci] = s_off[e] + j * kPfCols;
        p.chunk_n[ci] = c - j * kPfCols < kPfCols ? c - j * kPfCols : kPfCols;
      }
    }
    for (int j = lane; j < nb; j += 32) {
      const int bi = s_bofs[e] + j;
      if (bi < p.blk_cap) {
        p.blk_expert[bi] = e;
        p.blk_row0[bi] = s_off[e] + j * kPfBlk;
        p.blk_n[bi] = c - j * kPfBlk < kPfBlk ? c - j * kPfBlk : kPfBlk;
      }
    }
  }
}

// ---------------------------------------------------------- grouped GEMM --
// epilogues: the GLU of gate/up with either activation (one per kernel, so
// only one activation body is compiled into it), or the plain down rows
enum PfEpi : int { kPfEpiSwiglu = 0, kPfEpiSitu = 1, kPfEpiDown = 2 };

struct PfGemmParams {
  const uint8_t *const *expert_tiles;   // [E+1] t16 tiles (null: not loaded)
  int kb;                               // K / 256
  int m_tiles;                          // weight rows / 128
  const int32_t *n_chunks, *chunk_expert, *chunk_row0, *chunk_n;
  uint16_t *y;                          // gate/up: act [P][ld_y]; down: down [P][ld_y]
  int ld_y;
  float gate_beta, value_beta;
  int *err;
};

// ------------------------------------------- warp-specialised grouped GEMM --
// Warp roles, so that loads, code expansion, MMAs and promotion overlap:
//   warp 0        producer (one thread): unit bulk copies into a 3-stage
//                 ring; the chunk's rows and their group sums as TMA boxes
//                 into a 2-stage ring
//   warp 1        tensor memory owner; lane 0 issues the MMAs
//   warps 2..5    expand a stage's codes into bf16 A tiles, a part at a
//                 time
//   warps 6..13   promotion: TMEM lane quarter (warp & 3), token half
//                 ((warp - 6) >> 2); f32 accumulators in registers; the
//                 item's epilogue
// Tensor memory holds the 8 group accumulators of a k-block (8 x 64
// columns); a k-block runs in kTcParts parts, and each part's accumulators
// and A sub-tiles pass from expansion to MMAs to promotion on their own
// barriers, so the parts of one step overlap.
// Every wait is bounded and also watches a CTA-wide abort word, so a timeout
// in one role unwinds all of them.
constexpr int kTcWarps = 14;
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kTcConvThreads = 128;            // warps 2..5
constexpr int kTcPromoThreads = 256;           // warps 6..13
constexpr int kTcUStages = 3;
constexpr int kTcBStages = 2;
constexpr int kTcParts = 2;                    // a k-block's MMAs / promotion in 2 parts of 4 groups
constexpr int kTcGpp = kPfGroups / kTcParts;   // quantisation groups per part
constexpr int kTcSubs = 4 / kTcParts;          // 64-column A sub-tiles per part
constexpr int kTcTb = kTcGpp == 4 ? 8 : 16;    // token columns per TMEM read of a part's groups
constexpr int kTcA = 0;                        // the A parts
constexpr int kTcB = kTcA + 4 * kPfASub;       // kTcBStages x 4 sub-tiles x [64 rows x 128 B]
constexpr int kTcS = kTcB + kTcBStages * kPfBStage;                    // kTcBStages x [64 rows][8 groups] f32
constexpr int kTcU = kTcS + kTcBStages * kPfGroups * kPfCols * 4;      // kTcUStages x 8 units
constexpr int kTcBar = kTcU + kTcUStages * kPfUStage;
// barriers (8 bytes each): full_u[3] empty_u[3] full_b[2] empty_b[2] afull, amma, tfree [kTcParts] each
constexpr int kTcNumBars = 2 * kTcUStages + 2 * kTcBStages + 3 * kTcParts;
constexpr int kTcSmem = kTcBar + kTcNumBars * 8 + 16;
constexpr int kTcSmemAlloc = kTcSmem + 1024;
static_assert(kTcSmemAlloc <= kGemvSmemLimit, "warp-specialised GEMM shared memory");

struct TcBars {
  uint32_t full_u, empty_u, full_b, empty_b, afull, amma, tfree;
};

// Bounded wait that also gives up when another role has aborted.
__device__ __forceinline__ bool tc_wait(uint32_t bar, uint32_t parity, const volatile int *abort_word) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 16; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*abort_word) return false;
    if (global_timer_ns() - t0 > 1000000000ull) return false;
  }
}

// 2-D TMA tile load into this CTA's shared memory (no multicast), completing on ``bar``.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t addr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(addr));
}

template <int EPI>
__global__ void __launch_bounds__(kTcThreads, 1)
    rc_pf_tc_kernel(const __grid_constant__ PfGemmParams p, const __grid_constant__ CUtensorMap tm_b,
                    const __grid_constant__ CUtensorMap tm_s) {
  extern __shared__ uint8_t pf_raw_smem[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(pf_raw_smem) + 1023) & ~(uintptr_t)1023);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t bar0 = smem_addr(sm + kTcBar);
  const uint32_t bar_p = bar0 + 16 * kTcUStages + 16 * kTcBStages;   // the per-part barriers
  const TcBars bars{bar0, bar0 + 8 * kTcUStages, bar0 + 16 * kTcUStages, bar0 + 16 * kTcUStages + 8 * kTcBStages,
                    bar_p, bar_p + 8 * kTcParts, bar_p + 16 * kTcParts};
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + kTcBar + kTcNumBars * 8);
  volatile int *abort_word = reinterpret_cast<volatile int *>(sm + kTcBar + kTcNumBars * 8 + 4);

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(kPfTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    *abort_word = 0;
    for (int i = 0; i < kTcUStages; ++i) {
      mbar_init(bars.full_u + 8 * i, 1);
      mbar_init(bars.empty_u + 8 * i, kTcConvThreads + kTcPromoThreads);
    }
    for (int i = 0; i < kTcBStages; ++i) {
      mbar_init(bars.full_b + 8 * i, 1);
      mbar_init(bars.empty_b + 8 * i, 1 + kTcPromoThreads);
    }
    for (int q = 0; q < kTcParts; ++q) {
      mbar_init(bars.afull + 8 * q, kTcConvThreads);
      mbar_init(bars.amma + 8 * q, 1);
      mbar_init(bars.tfree + 8 * q, kTcPromoThreads);
    }
    mbar_fence_init();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const int n_chunks = *p.n_chunks;
  const int n_items = n_chunks * p.m_tiles;
  const int kb = p.kb;
  bool failed = false;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // One thread: per step the 8 weight units (bulk copies) and, as TMA tiles
    // of the permuted rows, the chunk's 64 source rows (four 64-column
    // swizzled boxes) and their group sums.
    int u_filled = 0, b_filled = 0;   // steps whose unit / row stage was issued
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      int step = 0;
      for (int item = blockIdx.x; item < n_items && !failed; item += gridDim.x) {
        const int chunk = item % n_chunks, m = item / n_chunks;
        const int e = p.chunk_expert[chunk], row0 = p.chunk_row0[chunk];
        const uint8_t *wt = p.expert_tiles[e];
        for (int kbi = 0; kbi < kb; ++kbi, ++step) {
          const int us = step % kTcUStages, bs = step % kTcBStages;
          if (step >= kTcUStages && !tc_wait(bars.empty_u + 8 * us, ((step / kTcUStages) - 1) & 1, abort_word)) {
            failed = true;
            break;
          }
          // an expert that is not loaded: the stage completes without data
          // (its outputs are garbage) and the call reports the error word
          mbar_arrive_expect_tx(bars.full_u + 8 * us, wt != nullptr ? kPfUStage : 0u);
          if (wt == nullptr) atomicCAS(p.err, 0, kErrWaitTimeout);
          if (wt != nullptr)
            for (int u = 0; u < 8; ++u)
              bulk_copy_g2s(smem_addr(sm + kTcU + us * kPfUStage + u * kUnitBytes),
                            wt + ((size_t)(8 * m + u) * kb + kbi) * kUnitBytes, kUnitBytes, bars.full_u + 8 * us,
                            pol);
          u_filled = step + 1;
          if (step >= kTcBStages && !tc_wait(bars.empty_b + 8 * bs, ((step / kTcBStages) - 1) & 1, abort_word)) {
            failed = true;
            break;
          }
          const uint32_t fb = bars.full_b + 8 * bs;
          mbar_arrive_expect_tx(fb, kPfBStage + kPfGroups * kPfCols * 4);
          const uint32_t sB = smem_addr(sm + kTcB + bs * kPfBStage);
#pragma unroll
          for (int j = 0; j < 4; ++j) tma_load_2d(sB + j * kPfBSub, &tm_b, kbi * kUnitK + 64 * j, row0, fb);
          tma_load_2d(smem_addr(sm + kTcS + bs * kPfGroups * kPfCols * 4), &tm_s, kbi * kPfGroups, row0, fb);
          b_filled = step + 1;
        }
      }
      if (failed) *abort_word = 1;
      // every copy issued lands before the shared memory goes away: wait for
      // the last fill of each stage (these complete whatever the other roles do)
      const int zero = 0;
      for (int us = 0; us < kTcUStages; ++us) {
        const int fills = (u_filled + kTcUStages - 1 - us) / kTcUStages;
        if (fills > 0) tc_wait(bars.full_u + 8 * us, (fills - 1) & 1, &zero);
      }
      for (int bs = 0; bs < kTcBStages; ++bs) {
        const int fills = (b_filled + kTcBStages - 1 - bs) / kTcBStages;
        if (fills > 0) tc_wait(bars.full_b + 8 * bs, (fills - 1) & 1, &zero);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    int step = 0;
    uint32_t commits[kTcParts] = {};   // completions issued on amma[q]
    for (int item = blockIdx.x; item < n_items && !failed; item += gridDim.x) {
      const int chunk = item % n_chunks;
      const int n16 = (p.chunk_n[chunk] + 15) & ~15;
      const uint32_t idesc = umma_idesc_bf16(kPfRows, n16);
      for (int kbi = 0; kbi < kb && !failed; ++kbi, ++step) {
        const int bs = step % kTcBStages;
        if (__any_sync(0xffffffffu, !tc_wait(bars.full_b + 8 * bs, (step / kTcBStages) & 1, abort_word))) {
          failed = true;
          break;
        }
        for (int q = 0; q < kTcParts; ++q) {
          if (__any_sync(0xffffffffu, !tc_wait(bars.afull + 8 * q, step & 1, abort_word) ||
                                          (step > 0 && !tc_wait(bars.tfree + 8 * q, (step - 1) & 1, abort_word)))) {
            failed = true;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            const uint64_t da = umma_desc_sw128(smem_addr(sm + kTcA + q * kTcSubs * kPfASub));
            const uint64_t db = umma_desc_sw128(smem_addr(sm + kTcB + bs * kPfBStage + q * kTcSubs * kPfBSub));
#pragma unroll
            for (int gg = 0; gg < kTcGpp; ++gg) {
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {
                const int kk = gg * 32 + hh * 16;      // column within the part: sub-tile kk / 64, column kk % 64
                umma_bf16(tbase + (kTcGpp * q + gg) * kPfCols,
                          da + (uint64_t)(((kk >> 6) * kPfASub + (kk & 63) * 2) >> 4),
                          db + (uint64_t)(((kk >> 6) * kPfBSub + (kk & 63) * 2) >> 4), idesc, (uint32_t)hh);
              }
            }
            umma_commit(bars.amma + 8 * q);
            if (q == kTcParts - 1) umma_commit(bars.empty_b + 8 * bs);
          }
          __syncwarp();
          ++commits[q];
        }
      }
    }
    if (failed) *abort_word = 1;
    // no MMA may still run when tensor memory is released (the abort word is
    // not consulted here: these commits always complete)
    const int zero = 0;
    for (int q = 0; q < kTcParts; ++q)
      if (commits[q] > 0) tc_wait(bars.amma + 8 * q, (commits[q] - 1) & 1, &zero);
  } else if (warp < 6) {
    // ----------------------------------------------------- code expansion
    const int ct = tid - 64;
    int step = 0;
    for (int item = blockIdx.x; item < n_items && !failed; item += gridDim.x) {
      for (int kbi = 0; kbi < kb && !failed; ++kbi, ++step) {
        const int us = step % kTcUStages;
        if (__any_sync(0xffffffffu, !tc_wait(bars.full_u + 8 * us, (step / kTcUStages) & 1, abort_word))) {
          failed = true;
          break;
        }
        const uint8_t *U = sm + kTcU + us * kPfUStage;
        for (int q = 0; q < kTcParts; ++q) {
          // the MMAs that read this A part in the previous step are done
          if (step > 0 && __any_sync(0xffffffffu, !tc_wait(bars.amma + 8 * q, (step - 1) & 1, abort_word))) {
            failed = true;
            break;
          }
          uint8_t *Ap = sm + kTcA + q * kTcSubs * kPfASub;
          constexpr int kPer = 128 / kTcParts;                // items of a unit in one part
#pragma unroll
          for (int j = 0; j < 8 / kTcParts; ++j) {
            const int gi = ct + kTcConvThreads * j;           // unit, k-step of the part, row group
            const int u = gi / kPer, rem = gi % kPer, s = 4 * kTcSubs * q + (rem >> 3), g = rem & 7;
            const uint8_t *base = U + u * kUnitBytes + ((s >> 2) * 32 + 4 * g) * 16 + (s & 3) * 4;
            // the four words sit 16 B apart: lanes start at word (g >> 1) so that
            // a warp's 32 loads fall in 32 different banks, then rotate back
            const int rot = (g >> 1) & 3;
            uint32_t v[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = *reinterpret_cast<const uint32_t *>(base + ((i + rot) & 3) * 16);
            const bool r1 = rot & 1, r2 = rot & 2;
            const uint32_t t0 = r1 ? v[3] : v[0], t1 = r1 ? v[0] : v[1], t2 = r1 ? v[1] : v[2], t3 = r1 ? v[2] : v[3];
            const uint32_t w[4] = {r2 ? t2 : t0, r2 ? t3 : t1, r2 ? t0 : t2, r2 ? t1 : t3};
            const int ra = 16 * u + g, rb = ra + 8;
            const int kk = 16 * (s & 3);
            uint8_t *As = Ap + ((s >> 2) - kTcSubs * q) * kPfASub;
            *reinterpret_cast<uint4 *>(As + sw128_off(ra, kk)) =
                make_uint4(codes_to_bf16x2<0>(w[0]), codes_to_bf16x2<0>(w[1]), codes_to_bf16x2<0>(w[2]),
                           codes_to_bf16x2<0>(w[3]));
            *reinterpret_cast<uint4 *>(As + sw128_off(ra, kk + 8)) =
                make_uint4(codes_to_bf16x2<2>(w[0]), codes_to_bf16x2<2>(w[1]), codes_to_bf16x2<2>(w[2]),
                           codes_to_bf16x2<2>(w[3]));
            *reinterpret_cast<uint4 *>(As + sw128_off(rb, kk)) =
                make_uint4(codes_to_bf16x2<1>(w[0]), codes_to_bf16x2<1>(w[1]), codes_to_bf16x2<1>(w[2]),
                           codes_to_bf16x2<1>(w[3]));
            *reinterpret_cast<uint4 *>(As + sw128_off(rb, kk + 8)) =
                make_uint4(codes_to_bf16x2<3>(w[0]), codes_to_bf16x2<3>(w[1]), codes_to_bf16x2<3>(w[2]),
                           codes_to_bf16x2<3>(w[3]));
          }
          fence_proxy_async();
          mbar_arrive(bars.afull + 8 * q);
        }
        if (!failed) mbar_arrive(bars.empty_u + 8 * us);
      }
    }
    if (failed) *abort_word = 1;
  } else {
    // ------------------------------------------------------------ promotion
    const int lq = warp & 3, ch = (warp - 6) >> 2;
    const int r_row = 32 * lq + lane;
    const int u_row = r_row >> 4, rr = r_row & 15;
    int step = 0;
    for (int item = blockIdx.x; item < n_items && !failed; item += gridDim.x) {
      const int chunk = item % n_chunks, m = item / n_chunks;
      const int row0 = p.chunk_row0[chunk], n = p.chunk_n[chunk];
      const int n16 = (n + 15) & ~15;
      const bool active = 32 * ch < n16;
      float2 acc[kPfCols / 4];
#pragma unroll
      for (int i = 0; i < kPfCols / 4; ++i) acc[i] = make_float2(0.f, 0.f);
      for (int kbi = 0; kbi < kb && !failed; ++kbi, ++step) {
        const int us = step % kTcUStages, bs = step % kTcBStages;
        if (__any_sync(0xffffffffu, !tc_wait(bars.full_u + 8 * us, (step / kTcUStages) & 1, abort_word))) {
          failed = true;
          break;
        }
        float sc[kPfGroups], mp[kPfGroups];
        {
          const uint8_t *P = sm + kTcU + us * kPfUStage + u_row * kUnitBytes + kUnitCodeBytes;
#pragma unroll
          for (int g = 0; g < kPfGroups; ++g) {
            const uint32_t pw = *reinterpret_cast<const uint32_t *>(P + ((rr & 7) * 8 + g) * 8 + (rr >> 3) * 4);
            sc[g] = bf16_lo_f32(pw);
            mp[g] = fmaf(-128.f, sc[g], bf16_hi_f32(pw));
          }
        }
        mbar_arrive(bars.empty_u + 8 * us);
        // the stage's group sums (TMA writes, acquired through the stage's barrier)
        if (__any_sync(0xffffffffu, !tc_wait(bars.full_b + 8 * bs, (step / kTcBStages) & 1, abort_word))) {
          failed = true;
          break;
        }
        const float *sS = reinterpret_cast<const float *>(sm + kTcS + bs * kPfGroups * kPfCols * 4);
#pragma unroll
        for (int q = 0; q < kTcParts; ++q) {
          if (failed || __any_sync(0xffffffffu, !tc_wait(bars.amma + 8 * q, step & 1, abort_word))) {
            failed = true;
            break;
          }
          tc_fence_after();
          if (active) {
            float2 a3[kTcGpp], sg[kTcGpp];
#pragma unroll
            for (int gg = 0; gg < kTcGpp; ++gg) {
              a3[gg] = make_float2(mp[kTcGpp * q + gg], mp[kTcGpp * q + gg]);
              sg[gg] = make_float2(sc[kTcGpp * q + gg], sc[kTcGpp * q + gg]);
            }
#pragma unroll
            for (int tb = 0; tb < 32 / kTcTb; ++tb) {
              // token columns past the chunk's MMA width hold nothing to promote
              if (kTcTb * tb >= n16 - 32 * ch) break;
              // kTcTb token columns of the part's group accumulators, one wait
              uint32_t v[kTcGpp][kTcTb];
#pragma unroll
              for (int gg = 0; gg < kTcGpp; ++gg) {
                const uint32_t ta = tbase + ((uint32_t)(32 * lq) << 16) + (kTcGpp * q + gg) * kPfCols + 32 * ch + kTcTb * tb;
                if constexpr (kTcTb == 8) tmem_ld8(ta, *reinterpret_cast<uint32_t(*)[8]>(&v[gg][0]));
                else tmem_ld16(ta, *reinterpret_cast<uint32_t(*)[16]>(&v[gg][0]));
              }
              tmem_wait_ld();
#pragma unroll
              for (int j = 0; j < kTcTb / 2; ++j) {
                const int t = 32 * ch + kTcTb * tb + 2 * j;
                float s0[kTcGpp], s1[kTcGpp];
                if constexpr (kTcGpp == 4) {
                  const float4 x0 = *reinterpret_cast<const float4 *>(sS + t * kPfGroups + kTcGpp * q);
                  const float4 x1 = *reinterpret_cast<const float4 *>(sS + (t + 1) * kPfGroups + kTcGpp * q);
                  s0[0] = x0.x, s0[1] = x0.y, s0[2] = x0.z, s0[3] = x0.w;
                  s1[0] = x1.x, s1[1] = x1.y, s1[2] = x1.z, s1[3] = x1.w;
                } else {
#pragma unroll
                  for (int gg = 0; gg < kTcGpp; ++gg) {
                    s0[gg] = sS[t * kPfGroups + kTcGpp * q + gg];
                    s1[gg] = sS[(t + 1) * kPfGroups + kTcGpp * q + gg];
                  }
                }
                float2 &ac = acc[(kTcTb / 2) * tb + j];
#pragma unroll
                for (int gg = 0; gg < kTcGpp; ++gg) {
                  ac = __ffma2_rn(a3[gg], make_float2(s0[gg], s1[gg]), ac);
                  ac = __ffma2_rn(sg[gg], make_float2(__uint_as_float(v[gg][2 * j]), __uint_as_float(v[gg][2 * j + 1])),
                                  ac);
                }
              }
            }
          }
          tc_fence_before();
          mbar_arrive(bars.tfree + 8 * q);
        }
        if (!failed) mbar_arrive(bars.empty_b + 8 * bs);
      }
      if (failed) break;
      // ---- epilogue: this warp's 32 token columns
      float a[kPfCols / 2];
#pragma unroll
      for (int i = 0; i < kPfCols / 4; ++i) a[2 * i] = acc[i].x, a[2 * i + 1] = acc[i].y;
      if (EPI != kPfEpiDown) {
        const int col = 8 * (8 * m + u_row) + rr;       // rows rr < 8: gate, rr >= 8: up of the same column
#pragma unroll
        for (int t = 0; t < kPfCols / 2; ++t) {
          const float up = __shfl_down_sync(0xffffffffu, a[t], 8);
          const int tok = 32 * ch + t;
          if (rr < 8 && tok < n) {
            const float gate = bf16_round(a[t]);
            const float u = bf16_round(up);
            const float v = EPI == kPfEpiSitu ? act_situ(gate, u, p.gate_beta, p.value_beta) : act_swiglu(gate, u);
            p.y[(size_t)(row0 + tok) * p.ld_y + col] = f32_to_bf16_rne(v);
          }
        }
      } else {
        const int col = kPfRows * m + r_row;
#pragma unroll
        for (int t = 0; t < kPfCols / 2; ++t) {
          const int tok = 32 * ch + t;
          if (tok < n) p.y[(size_t)(row0 + tok) * p.ld_y + col] = f32_to_bf16_rne(a[t]);
        }
      }
    }
    if (failed) *abort_word = 1;
  }
  if (failed && lane == 0) atomicCAS(p.err, 0, kErrWaitTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"(kPfTmemCols));
}

// Rows of the tensor-core GEMMs: for each of the *n_rows permuted rows r,
// source row row_token[r] (or r itself when row_token is null) copied to
// dst[r] (when dst is set), and its group sums s[r][g]: the group's four
// 8-column chunks in turn, each chunk's four bf16 pairs added pairwise first.
__global__ void rc_pf_rows_kernel(const uint16_t *src, int K, int ld, const int32_t *row_token, const int32_t *n_rows,
                                  uint16_t *dst, float *s) {
  const int groups = K / 32, total = *n_rows * groups;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int r = i / groups, g = i - r * groups;
    const int sr = row_token ? row_token[r] : r;
    const uint4 *p = reinterpret_cast<const uint4 *>(src + (size_t)sr * ld + 32 * g);
    uint4 v[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) v[c] = __ldg(p + c);
    if (dst) {
      uint4 *d = reinterpret_cast<uint4 *>(dst + (size_t)r * K + 32 * g);
#pragma unroll
      for (int c = 0; c < 4; ++c) d[c] = v[c];
    }
    float part = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint32_t w4[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) part += bf16_to_f32(w4[q] & 0xFFFFu) + bf16_to_f32(w4[q] >> 16);
    }
    s[i] = part;
  }
}

// ------------------------------------------------ register-fragment path --
// The experts' GEMMs as a grouped GEMV over 8-row token blocks, with the unit
// arithmetic of the decode GEMV (codes as exact f16 subnormals in mma.sync A
// fragments; activations as block-scaled f16 B fragments; min term on bf16
// mmas; per-unit partials summed per tile in k-block order).  tcgen05 needs
// a separate accumulator per 32-column quantisation group, so it pays 16 MMA
// instructions per (128-row tile, k-block) whatever the tile's token count;
// with the few tokens most experts get, these register fragments do the same
// work with far fewer instructions.

// Staged activations of the 8-row token blocks (slot 8 b + t = row t of block
// b; rows past the block's count zero), one warp per (slot, 256-column
// block).  Gate/up: row t of block b is x[row_token[row0 + t]]; down:
// act[row0 + t].
__global__ void __launch_bounds__(256) rc_pf_stage_blocks_kernel(const uint16_t *src, int K, const int32_t *row_token,
                                                              const int32_t *n_blocks, const int32_t *blk_row0,
                                                              const int32_t *blk_n, int blk_cap, uint32_t *xf,
                                                              void *aux) {
  const int nb = *n_blocks, KB = K / kUnitK, k64 = K / 64, lane = threadIdx.x & 31;
  const int total = nb * kPfBlk * KB;
  uint16_t *bmin16 = static_cast<uint16_t *>(aux);
  float *inv = reinterpret_cast<float *>(bmin16 + (size_t)blk_cap * KB * 256);
  const int nw = gridDim.x * (blockDim.x >> 5);
  for (int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < total; w += nw) {
    const int slot = w / KB, kbi = w - slot * KB;
    const int b = slot / kPfBlk, t = slot - b * kPfBlk;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
    if (t < blk_n[b]) {
      const int row = blk_row0[b] + t;
      const int srow = row_token ? row_token[row] : row;
      const uint4 raw = *reinterpret_cast<const uint4 *>(src + (size_t)srow * K + kbi * kUnitK + lane * 8);
      const uint32_t wd[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[2 * i] = bf16_lo_f32(wd[i]);
        v[2 * i + 1] = bf16_hi_f32(wd[i]);
      }
    }
    stage_core<true>(v, slot, kbi * 32 + lane, k64, KB, xf, bmin16, inv);
  }
}

struct PfGemvParams {
  const uint8_t *const *expert_tiles;   // [E+1] t16 tiles (null: not loaded)
  int kb, tiles;                        // k-blocks; 16-row tiles of an expert's matrix
  const int32_t *n_blocks, *blk_expert, *blk_row0, *blk_n;
  const uint32_t *xf;                   // staged blocks (rc_pf_stage_blocks_kernel)
  const void *xaux;
  int blk_cap;
  uint16_t *y;                          // gate/up: act [P][ld_y]; down: down [P][ld_y]
  int ld_y;
  float gate_beta, value_beta;
  int stages, round;                    // ring depth per warp; tiles per round
  int *err;
};
constexpr int kPgWarps = 16, kPgThreads = kPgWarps * 32;
constexpr int kPgPartBytes = 48 * 1024;

// One CTA per SM, persistent over a contiguous range of the block-major
// (block, 16-row tile) list; each warp streams its units (k-block-major
// within a round, RoundCursor) through a ring of bulk copies.
template <int EPI>
__global__ void __launch_bounds__(kPgThreads, 1) rc_pf_gemv_kernel(PfGemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, qd = lane & 3;
  const int S = p.stages, KB = p.kb, R = p.round;
  uint8_t *ring = smem + warp * S * kUnitBytes;
  const uint32_t ring_s = smem_addr(ring);
  float4 *part = reinterpret_cast<float4 *>(smem + kPgWarps * S * kUnitBytes);
  const uint32_t bar0 = smem_addr(smem + kPgWarps * S * kUnitBytes + kPgPartBytes) + warp * S * 8;
  const int nb = *p.n_blocks;
  const int total = nb * p.tiles;
  const int per = (total + (int)gridDim.x - 1) / (int)gridDim.x;
  const int c0 = blockIdx.x * per;
  const int nt = c0 < total ? (c0 + per < total ? per : total - c0) : 0;
  const FastDiv gt = make_fastdiv(p.tiles);
  RoundCursor iss, cur;
  iss.init(nt, R, KB, kPgWarps, warp);
  cur.init(nt, R, KB, kPgWarps, warp);
  int issued = 0, consumed = 0;
  auto issue = [&](int sl) {
    const uint32_t tg = c0 + iss.tile(), blk = fdiv(tg, gt), tile = tg - blk * gt.d;
    const uint8_t *wt = p.expert_tiles[p.blk_expert[blk]];
    if (wt) {
      mbar_arrive_expect_tx(bar0 + 8 * sl, kUnitBytes);
      bulk_copy_g2s_plain(ring_s + sl * kUnitBytes, wt + ((size_t)tile * KB + iss.kbi) * kUnitBytes, kUnitBytes,
                          bar0 + 8 * sl);
    } else {
      mbar_arrive_expect_tx(bar0 + 8 * sl, 0);     // nothing to fetch: complete the phase at once
    }
    ++issued;
    iss.next();
  };
  if (lane == 0) {
    for (int sl = 0; sl < S; ++sl) mbar_init(bar0 + 8 * sl, 1);
    mbar_fence_init();
    for (int sl = 0; sl < S && iss.valid(); ++sl) issue(sl);
  }
  __syncwarp();
  XFrag<1> xr;
  int xr_key = -1;
  int slot = 0;
  uint32_t parity = 0;
  bool failed = false;
  const int n_rounds = round_count(nt, R);
  for (int r = 0; r < n_rounds; ++r) {
    for (; cur.valid() && cur.round == r; cur.next()) {
      const uint32_t blk = fdiv(c0 + cur.tile(), gt);
      if (!failed) {
        if (mbar_wait_bounded_warp(bar0 + 8 * slot, parity)) {
          ++consumed;
        } else {
          if (lane == 0) atomicCAS(p.err, 0, kErrWaitTimeout);
          failed = true;
        }
      }
      if (!failed && p.expert_tiles[p.blk_expert[blk]] != nullptr) {
        if ((int)blk * KB + cur.kbi != xr_key) {
          load_xfrag<1, false>(xr, p.xf, p.xaux, p.blk_cap, blk, KB, cur.kbi, lane);
          xr_key = blk * KB + cur.kbi;
        }
        float4 Q[1];
        unit_result<1>(ring + slot * kUnitBytes, xr, lane, Q);
        part[(size_t)cur.slot() * 32 + lane] = Q[0];
      }
      __syncwarp();
      if (!failed && lane == 0 && iss.valid()) issue(slot);
      if (++slot == S) slot = 0, parity ^= 1u;
    }
    __syncthreads();
    const int t_lo = r * R, t_hi = t_lo + R < nt ? t_lo + R : nt;
    for (int ti = t_lo + warp; ti < t_hi; ti += kPgWarps) {
      const uint32_t tg = c0 + ti, blk = fdiv(tg, gt), tile = tg - blk * gt.d;
      const uint8_t *wt = p.expert_tiles[p.blk_expert[blk]];
      if (wt == nullptr) {
        if (lane == 0) atomicCAS(p.err, 0, kErrWaitTimeout);
        continue;
      }
      Acc<1> acc;
      acc_zero(acc);
      const float4 *src = part + (size_t)(ti - t_lo) * KB * 32 + lane;
      for (int kbi = 0; kbi < KB; ++kbi) {
        float4 v[1] = {src[kbi * 32]};
        acc_add(acc, v);
      }
      const int n = p.blk_n[blk], row0 = p.blk_row0[blk];
#pragma unroll
      for (int e2 = 0; e2 < 2; ++e2) {
        const int t = 2 * qd + e2;
        if (t >= n) continue;
        if (EPI != kPfEpiDown) {
          const float gate = bf16_round(acc.v[0][e2]);
          const float up = bf16_round(acc.v[0][2 + e2]);
          const float v = EPI == kPfEpiSitu ? act_situ(gate, up, p.gate_beta, p.value_beta) : act_swiglu(gate, up);
          p.y[(size_t)(row0 + t) * p.ld_y + tile * 8 + g] = f32_to_bf16_rne(v);
        } else {
          uint16_t *y = p.y + (size_t)(row0 + t) * p.ld_y + tile * kUnitRows + g;
          y[0] = f32_to_bf16_rne(acc.v[0][e2]);
          y[8] = f32_to_bf16_rne(acc.v[0][2 + e2]);
        }
      }
    }
    __syncthreads();
  }
  // after a failure, the copies still in flight land before the shared
  // memory is released
  if (failed && lane == 0) {
    for (int j = consumed; j < issued; ++j) mbar_wait_bounded(bar0 + 8 * (j % S), (uint32_t)(j / S) & 1u);
  }
}

// --------------------------------------------------------------- combine --
// Per token: routed = RTNE(sum over its slots in ascending ID of
// f32(down[row]) * w), then RTNE(f32(routed) + f32(shared row)).
constexpr int kPfCombineThreads = 128;

__global__ void __launch_bounds__(kPfCombineThreads) rc_pf_combine_kernel(const uint16_t *down, const int32_t *slot_row,
                                                                         const float *slot_w, int k, int with_shared,
                                                                         int hidden, uint16_t *out) {
  const int t = blockIdx.y;
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v * 8 >= hidden) return;
  const int32_t *sr = slot_row + (size_t)t * (k + 1);
  uint4 r[kMoeMaxK];
  float w[kMoeMaxK];
#pragma unroll
  for (int s = 0; s < kMoeMaxK; ++s) {
    r[s] = make_uint4(0, 0, 0, 0);
    w[s] = 0.f;
    if (s < k && sr[s] >= 0) {     // a slot without a row (bad caller id, flagged by the plan) adds nothing
      r[s] = __ldcg(reinterpret_cast<const uint4 *>(down + (size_t)sr[s] * hidden + (size_t)v * 8));
      w[s] = slot_w[(size_t)t * k + s];
    }
  }
  const uint4 sh = with_shared && sr[k] >= 0
                       ? __ldcg(reinterpret_cast<const uint4 *>(down + (size_t)sr[k] * hidden + (size_t)v * 8))
                       : make_uint4(0, 0, 0, 0);
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
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
  *reinterpret_cast<uint4 *>(out + (size_t)t * hidden + (size_t)v * 8) = make_uint4(o[0], o[1], o[2], o[3]);
}

// Expert-parallel slot rows: slot_out[t][r] = down[slot_row[t][r]], or zeros
// where the slot is computed on another rank.
__global__ void rc_pf_slot_rows_kernel(const uint16_t *down, const int32_t *slot_row, int hidden, uint16_t *slot_out) {
  const int i = blockIdx.x;                       // (token, slot)
  const int row = slot_row[i];
  for (int v = threadIdx.x; v * 8 < hidden; v += blockDim.x) {
    uint4 val = make_uint4(0, 0, 0, 0);
    if (row >= 0) val = __ldcg(reinterpret_cast<const uint4 *>(down + (size_t)row * hidden + (size_t)v * 8));
    *reinterpret_cast<uint4 *>(slot_out + (size_t)i * hidden + (size_t)v * 8) = val;
  }
}

__global__ void rc_pf_identity_rows_kernel(int32_t *rows, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) rows[i] = i;
}

// ------------------------------------------------------------------ host --
// A 2-D TMA map of a row-major [rows][cols] array with (box_cols x box_rows)
// boxes; rows past the end read as zeros.  The encoder is the driver's,
// reached through the runtime (no link against the driver library).
static bool tma_map_2d(CUtensorMap *map, void *base, CUtensorMapDataType type, int esize, int cols, size_t rows,
                       int box_cols, int box_rows, bool swizzle128, const char **why) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (encode == nullptr) {
    cudaDriverEntryPointQueryResult q{};
    void *fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || fn == nullptr) {
      *why = "cuTensorMapEncodeTiled is not available";
      return false;
    }
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  const cuuint64_t dim[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t stride[1] = {(cuuint64_t)cols * esize};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estride[2] = {1, 1};
  const CUresult r = encode(map, type, 2, base, dim, stride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    *why = "cuTensorMapEncodeTiled rejected a map";
    return false;
  }
  return true;
}

static void pf_release(PfScratch *s) {
  if (!s) return;
  cudaFree(s->logits);
  cudaFree(s->ids);
  cudaFree(s->weights);
  cudaFree(s->slot_expert);
  cudaFree(s->slot_w);
  cudaFree(s->slot_row);
  cudaFree(s->row_token);
  cudaFree(s->cnt);
  cudaFree(s->off);
  cudaFree(s->n_chunks);
  cudaFree(s->chunk_expert);
  cudaFree(s->chunk_row0);
  cudaFree(s->chunk_n);
  cudaFree(s->act);
  cudaFree(s->down);
  cudaFree(s->blk_expert);
  cudaFree(s->blk_row0);
  cudaFree(s->blk_n);
  cudaFree(s->xf);
  cudaFree(s->xaux);
  cudaFree(s->x_perm);
  cudaFree(s->ssum_x);
  cudaFree(s->ssum_act);
  delete s;
}

void pf_free(rc_moe *m) {
  pf_release(m->pf);
  m->pf = nullptr;
}

// Scratch for T tokens (grown, never shrunk).  Allocation synchronises the
// device, so size it before capturing a graph.
static int pf_scratch(rc_moe *m, int T) {
  if (m->pf && m->pf->T_cap >= T) return RC_OK;
  RC_CUDA_TRY(cudaDeviceSynchronize());
  pf_free(m);
  PfScratch *s = new PfScratch();
  const int E = m->n_experts, K = kMoeMaxK;
  s->T_cap = T;
  s->E1 = E + 1;
  s->P_cap = T * (K + 1);
  s->chunk_cap = s->P_cap / kPfCols + E + 1;
  s->blk_cap = s->P_cap / kPfBlk + E + 1;
  const int kmax = m->hidden > m->inter_pad ? m->hidden : m->inter_pad;
  const size_t P = (size_t)s->P_cap;
  cudaError_t e = cudaMalloc(&s->logits, (size_t)T * E * 4);
  if (e == cudaSuccess) e = cudaMalloc(&s->ids, (size_t)T * K * 4);
  if (e == cudaSuccess) e = cudaMalloc(&s->weights, (size_t)T * K * 4);
  if (e == cudaSuccess) e = cudaMalloc(&s->slot_expert, (size_t)T * (K + 1) * 4);
  if (e == cudaSuccess) e = cudaMalloc(&s->slot_w, (size_t)T * K * 4);
  if (e == cudaSuccess) e = cudaMalloc(&s->slot_row, (size_t)T * (K + 1) * 4);
  if (e == cudaSuccess) e = cudaMalloc(&s->row_token, P * 4);
  if (e == cudaSuccess) e = cudaMalloc(&s->cnt, (size_t)(E + 1) * 4);
  if (e == cudaSuccess) e = cudaMalloc(&s->off, (size_t)(E + 1) * 4);
  if (e == cudaSuccess) e = cudaMalloc(&s->n_chunks, 16);
  if (e == cudaSuccess) e = cudaMalloc(&s->blk_expert, (size_t)s->blk_cap * 4);
  if (e == cudaSuccess) e = cudaMalloc(&s->blk_row0, (size_t)s->blk_cap * 4);
  if (e == cudaSuccess) e = cudaMalloc(&s->blk_n, (size_t)s->blk_cap * 4);
  if (e == cudaSuccess) e = cudaMalloc(&s->xf, xfrag_bytes(s->blk_cap, kmax));
  if (e == cudaSuccess) e = cudaMalloc(&s->xaux, xaux_bytes(s->blk_cap, kmax));
  if (e == cudaSuccess) e = cudaMalloc(&s->x_perm, P * m->hidden * 2);
  if (e == cudaSuccess) e = cudaMalloc(&s->ssum_x, P * (m->hidden / 32) * 4);
  if (e == cudaSuccess) e = cudaMalloc(&s->ssum_act, P * (m->inter_pad / 32) * 4);
  if (e == cudaSuccess) e = cudaMalloc(&s->chunk_expert, (size_t)s->chunk_cap * 4);
  if (e == cudaSuccess) e = cudaMalloc(&s->chunk_row0, (size_t)s->chunk_cap * 4);
  if (e == cudaSuccess) e = cudaMalloc(&s->chunk_n, (size_t)s->chunk_cap * 4);
  if (e == cudaSuccess) e = cudaMalloc(&s->act, P * m->inter_pad * 2);
  if (e == cudaSuccess) e = cudaMemset(s->act, 0, P * m->inter_pad * 2);
  if (e == cudaSuccess) e = cudaMalloc(&s->down, P * m->hidden * 2);
  if (e != cudaSuccess) {
    pf_release(s);
    set_error("MoE prefill scratch for %d tokens: %s", T, cudaGetErrorString(e));
    return RC_ERR_CUDA;
  }
  const char *why = nullptr;
  if (!tma_map_2d(&s->tm_x, s->x_perm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, m->hidden, P, 64, 64, true, &why) ||
      !tma_map_2d(&s->tm_act, s->act, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, m->inter_pad, P, 64, 64, true, &why) ||
      !tma_map_2d(&s->tm_sx, s->ssum_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, m->hidden / 32, P, kPfGroups, 64, false,
                  &why) ||
      !tma_map_2d(&s->tm_sact, s->ssum_act, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, m->inter_pad / 32, P, kPfGroups, 64,
                  false, &why)) {
    pf_release(s);
    set_error("MoE prefill tensor maps: %s", why);
    return RC_ERR_CUDA;
  }
  m->pf = s;
  return RC_OK;
}

template <int EPI>
static cudaError_t pf_launch_tc(const rc_ctx *ctx, const PfGemmParams &p, const CUtensorMap &tm_b,
                                const CUtensorMap &tm_s, cudaStream_t s) {
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(rc_pf_tc_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmemAlloc);
    if (e != cudaSuccess) return e;
    if (dev < 64) configured[dev] = true;
  }
  // No programmatic overlap: a CTA of the next kernel must never sit on an SM
  // waiting for this grid while holding what this grid needs (tensor memory).
  rc_pf_tc_kernel<EPI><<<ctx->sm_count, kTcThreads, kTcSmemAlloc, s>>>(p, tm_b, tm_s);
  return cudaGetLastError();
}

// The permuted source rows of a tensor-core GEMM and their group sums.
static cudaError_t pf_rows(const rc_ctx *ctx, const uint16_t *src, int K, int ld, const int32_t *row_token,
                           const int32_t *n_rows, uint16_t *dst, float *ssum, cudaStream_t s) {
  rc_pf_rows_kernel<<<ctx->sm_count * 4, 256, 0, s>>>(src, K, ld, row_token, n_rows, dst, ssum);
  return cudaGetLastError();
}

template <int EPI>
static cudaError_t pf_launch_gemv(const rc_ctx *ctx, const PfGemvParams &p, size_t smem, cudaStream_t s) {
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(rc_pf_gemv_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvSmemLimit);
    if (e != cudaSuccess) return e;
    if (dev < 64) configured[dev] = true;
  }
  rc_pf_gemv_kernel<EPI><<<ctx->sm_count, kPgThreads, smem, s>>>(p);
  return cudaGetLastError();
}

struct PfRun {
  int T, k, act;
  float gb, vb;
  int lo, hi, st0, st1;        // computed experts / shared tokens
  int max_id;                  // routed ids below this (n_experts; + 1 when caller routes may name the shared expert)
};

// gate/up + down on the register-fragment path (after the plan): stage the
// blocks' rows, grouped GEMV, for each of the two matrices
static int pf_experts_gemv(rc_moe *m, const uint16_t *x, const PfRun &r, cudaStream_t s) {
  PfScratch *ps = m->pf;
  constexpr int kStages = 4;
  const size_t smem = (size_t)kPgWarps * kStages * kUnitBytes + kPgPartBytes + (size_t)kPgWarps * kStages * 8;
  PfGemvParams g{};
  g.expert_tiles = m->gu_tiles;
  g.kb = m->hidden / kUnitK;
  g.tiles = 2 * m->inter / kUnitRows;
  g.n_blocks = ps->n_chunks + 1;
  g.blk_expert = ps->blk_expert;
  g.blk_row0 = ps->blk_row0;
  g.blk_n = ps->blk_n;
  g.xf = ps->xf;
  g.xaux = ps->xaux;
  g.blk_cap = ps->blk_cap;
  g.y = ps->act;
  g.ld_y = m->inter_pad;
  g.gate_beta = r.gb;
  g.value_beta = r.vb;
  g.stages = kStages;
  g.round = kPgPartBytes / (g.kb * 32 * 16);
  g.err = m->ctx->err;
  rc_pf_stage_blocks_kernel<<<m->ctx->sm_count * 4, 256, 0, s>>>(x, m->hidden, ps->row_token, g.n_blocks, ps->blk_row0,
                                                               ps->blk_n, ps->blk_cap, ps->xf, ps->xaux);
  RC_CUDA_TRY(cudaGetLastError());
  if (r.act == RC_ACT_SITU)
    RC_CUDA_TRY(pf_launch_gemv<kPfEpiSitu>(m->ctx, g, smem, s));
  else
    RC_CUDA_TRY(pf_launch_gemv<kPfEpiSwiglu>(m->ctx, g, smem, s));
  if (m->down_fmt == kFormatBfp16) {
    BfMoeDown b{};
    b.w = m->dn_tiles;
    b.n_groups = g.n_blocks;
    b.group_expert = ps->blk_expert;
    b.blk_row0 = ps->blk_row0;
    b.blk_n = ps->blk_n;
    b.x = ps->act;
    b.ldx = m->inter_pad;
    b.T = 8;
    b.hidden = m->hidden;
    b.inter_pad = m->inter_pad;
    b.y = ps->down;
    b.ldy = m->hidden;
    b.max_groups = ps->blk_cap;
    b.err = m->ctx->err;
    return bfp16_moe_down(m->ctx, b, s);
  }
  PfGemvParams d = g;
  d.expert_tiles = m->dn_tiles;
  d.kb = m->inter_pad / kUnitK;
  d.tiles = m->hidden / kUnitRows;
  d.y = ps->down;
  d.ld_y = m->hidden;
  d.round = kPgPartBytes / (d.kb * 32 * 16);
  rc_pf_stage_blocks_kernel<<<m->ctx->sm_count * 4, 256, 0, s>>>(ps->act, m->inter_pad, nullptr, d.n_blocks,
                                                               ps->blk_row0, ps->blk_n, ps->blk_cap, ps->xf, ps->xaux);
  RC_CUDA_TRY(cudaGetLastError());
  RC_CUDA_TRY(pf_launch_gemv<kPfEpiDown>(m->ctx, d, smem, s));
  return RC_OK;
}

// plan + gate/up + down for slot lists already in m->pf (slot_expert, slot_w)
static int pf_experts(rc_moe *m, const uint16_t *x, const PfRun &r, cudaStream_t s) {
  PfScratch *ps = m->pf;
  PfPlanParams pp{};
  pp.slot_expert = ps->slot_expert;
  pp.T = r.T;
  pp.k = r.k;
  pp.E1 = m->n_experts + 1;
  pp.max_id = r.max_id;
  pp.lo = r.lo;
  pp.hi = r.hi;
  pp.st0 = r.st0;
  pp.st1 = r.st1;
  pp.slot_row = ps->slot_row;
  pp.row_token = ps->row_token;
  pp.cnt = ps->cnt;
  pp.off = ps->off;
  pp.n_chunks = ps->n_chunks;
  pp.chunk_expert = ps->chunk_expert;
  pp.chunk_row0 = ps->chunk_row0;
  pp.chunk_n = ps->chunk_n;
  pp.chunk_cap = ps->chunk_cap;
  pp.blk_expert = ps->blk_expert;
  pp.blk_row0 = ps->blk_row0;
  pp.blk_n = ps->blk_n;
  pp.blk_cap = ps->blk_cap;
  pp.err = m->ctx->err;
  const int nw = (r.T + 31) / 32;
  const size_t plan_smem = (size_t)2 * pp.E1 * nw * 4;
  RC_CHECK_ARG(plan_smem <= (size_t)kPfPlanSmemMax, "prefill plan of %d tokens x %d experts exceeds shared memory",
               r.T, pp.E1);
  static bool configured[64] = {};
  int dev = 0;
  RC_CUDA_TRY(cudaGetDevice(&dev));
  if (dev >= 64 || !configured[dev]) {
    RC_CUDA_TRY(cudaFuncSetAttribute(rc_pf_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfPlanSmemMax));
    if (dev < 64) configured[dev] = true;
  }
  rc_pf_plan_kernel<<<1, 1024, plan_smem, s>>>(pp);
  RC_CUDA_TRY(cudaGetLastError());

  // bfp16ebs8 down matrices: the register-fragment path's blocks feed the bfp16 grouped down kernel
  if (m->prefill_kernel == RC_PREFILL_GEMV || m->down_fmt == kFormatBfp16) return pf_experts_gemv(m, x, r, s);
  PfGemmParams g{};
  g.expert_tiles = m->gu_tiles;
  g.kb = m->hidden / kUnitK;
  g.m_tiles = 2 * m->inter / kPfRows;
  g.n_chunks = ps->n_chunks;
  g.chunk_expert = ps->chunk_expert;
  g.chunk_row0 = ps->chunk_row0;
  g.chunk_n = ps->chunk_n;
  g.y = ps->act;
  g.ld_y = m->inter_pad;
  g.gate_beta = r.gb;
  g.value_beta = r.vb;
  g.err = m->ctx->err;
  // the chunks' token rows in permuted order, with their group sums
  RC_CUDA_TRY(pf_rows(m->ctx, x, m->hidden, m->hidden, ps->row_token, ps->n_chunks + 2, ps->x_perm, ps->ssum_x, s));
  if (r.act == RC_ACT_SITU)
    RC_CUDA_TRY(pf_launch_tc<kPfEpiSitu>(m->ctx, g, ps->tm_x, ps->tm_sx, s));
  else
    RC_CUDA_TRY(pf_launch_tc<kPfEpiSwiglu>(m->ctx, g, ps->tm_x, ps->tm_sx, s));
  PfGemmParams d = g;
  d.expert_tiles = m->dn_tiles;
  d.kb = m->inter_pad / kUnitK;
  d.m_tiles = m->hidden / kPfRows;
  d.y = ps->down;
  d.ld_y = m->hidden;
  RC_CUDA_TRY(pf_rows(m->ctx, ps->act, m->inter_pad, m->inter_pad, nullptr, ps->n_chunks + 2, nullptr, ps->ssum_act,
                      s));
  RC_CUDA_TRY(pf_launch_tc<kPfEpiDown>(m->ctx, d, ps->tm_act, ps->tm_sact, s));
  return RC_OK;
}

static int pf_route(rc_moe *m, const uint16_t *x, int T, int k, int router, int renorm, float scaling,
                    cudaStream_t s) {
  PfScratch *ps = m->pf;
  const int E = m->n_experts;
  const size_t lsm = (size_t)kPfLogitExperts * m->hidden * 2;
  static bool configured[64] = {};
  int dev = 0;
  RC_CUDA_TRY(cudaGetDevice(&dev));
  if (dev >= 64 || !configured[dev]) {
    RC_CUDA_TRY(cudaFuncSetAttribute(rc_pf_logits_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvSmemLimit));
    if (dev < 64) configured[dev] = true;
  }
  RC_CHECK_ARG(lsm <= (size_t)kGemvSmemLimit, "hidden %d too large for the prefill router", m->hidden);
  // tokens per warp: 4 unless the grid would then have fewer CTAs than SMs,
  // and at least 2 (a warp's tokens go in pairs)
  const int gx = (E + kPfLogitExperts - 1) / kPfLogitExperts;
  int tpw = kPfLogitMaxTpw;
  while (tpw > 2 && (long long)gx * ((T + 8 * tpw - 1) / (8 * tpw)) < m->ctx->sm_count) tpw >>= 1;
  rc_pf_logits_kernel<<<dim3(gx, (T + 8 * tpw - 1) / (8 * tpw)), 256, lsm, s>>>(x, T, m->hidden, m->router_w, E,
                                                                           ps->logits, tpw);
  RC_CUDA_TRY(cudaGetLastError());
  PfSelectParams sp{};
  sp.logits = ps->logits;
  sp.bias = m->router_bias;
  sp.T = T;
  sp.E = E;
  sp.k = k;
  sp.mode = router;
  sp.renorm = renorm;
  sp.shared_id = m->has_shared ? E : -1;
  sp.scaling = scaling;
  sp.ids = ps->ids;
  sp.weights = ps->weights;
  sp.slot_expert = ps->slot_expert;
  sp.slot_w = ps->slot_w;
  rc_pf_select_kernel<<<(T + 7) / 8, 256, 0, s>>>(sp);
  RC_CUDA_TRY(cudaGetLastError());
  return RC_OK;
}

static int pf_check(rc_moe *m, const uint16_t *x, int T, int k, int act, int lo, int hi) {
  RC_CHECK_ARG(T >= 1 && T <= kPfMaxTokens, "prefill: T must be 1..%d", kPfMaxTokens);
  RC_CHECK_ARG(k >= 1 && k <= kMoeMaxK && k <= m->n_experts, "prefill: k must be 1..%d and <= n_experts", kMoeMaxK);
  RC_CHECK_ARG(act == RC_ACT_SWIGLU || act == RC_ACT_SITU, "unknown activation %d", act);
  RC_CHECK_ARG((reinterpret_cast<uintptr_t>(x) & 15) == 0, "token rows must be 16-byte aligned");
  RC_CHECK_ARG((2 * m->inter) % kPfRows == 0 && m->hidden % kPfRows == 0,
               "prefill needs 2*inter and hidden multiples of 128");
  for (int e = lo; e < hi; ++e) RC_CHECK_ARG(m->gate_up[e] != nullptr, "expert %d is not loaded", e);
  return RC_OK;
}

int pf_route_tokens(rc_moe *m, const uint16_t *x_dev, int T, int k, int router, int renormalize, float scaling,
                    int32_t *ids_dev, float *w_dev, float *logits_dev, void *stream) {
  RC_CHECK_ARG(T >= 1 && T <= kPfMaxTokens, "rc_moe_route: T must be 1..%d", kPfMaxTokens);
  RC_CHECK_ARG(k >= 1 && k <= kMoeMaxK && k <= m->n_experts, "rc_moe_route: k must be 1..%d and <= n_experts",
               kMoeMaxK);
  RC_CHECK_ARG((reinterpret_cast<uintptr_t>(x_dev) & 15) == 0, "token rows must be 16-byte aligned");
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  int rc = pf_scratch(m, T);
  if (rc) return rc;
  const cudaStream_t s = pick_stream(m->ctx, stream);
  if ((rc = pf_route(m, x_dev, T, k, router, renormalize, scaling, s))) return rc;
  if (ids_dev) RC_CUDA_TRY(cudaMemcpyAsync(ids_dev, m->pf->ids, (size_t)T * k * 4, cudaMemcpyDeviceToDevice, s));
  if (w_dev) RC_CUDA_TRY(cudaMemcpyAsync(w_dev, m->pf->weights, (size_t)T * k * 4, cudaMemcpyDeviceToDevice, s));
  if (logits_dev)
    RC_CUDA_TRY(
        cudaMemcpyAsync(logits_dev, m->pf->logits, (size_t)T * m->n_experts * 4, cudaMemcpyDeviceToDevice, s));
  return RC_OK;
}

}  // namespace rc

using namespace rc;

extern "C" {

int rc_moe_set_prefill_kernel(rc_moe *m, int kernel) {
  RC_CHECK_ARG(m, "rc_moe_set_prefill_kernel: NULL argument");
  RC_CHECK_ARG(kernel == RC_PREFILL_GEMV || kernel == RC_PREFILL_TCGEN05, "unknown prefill kernel %d", kernel);
  m->prefill_kernel = kernel;
  return RC_OK;
}

int rc_moe_prefill(rc_moe *m, const uint16_t *x_dev, int T, int k, int router, int renormalize, float scaling,
                   int act, float gate_beta, float value_beta, uint16_t *out_dev, int32_t *ids_dev, float *w_dev,
                   void *stream) {
  RC_CHECK_ARG(m && x_dev && out_dev, "rc_moe_prefill: NULL argument");
  RC_CHECK_ARG(router == RC_ROUTER_SOFTMAX || router == RC_ROUTER_SIGMOID_BIAS, "unknown router %d", router);
  RC_CHECK_ARG((reinterpret_cast<uintptr_t>(out_dev) & 15) == 0, "out must be 16-byte aligned");
  int rc = pf_check(m, x_dev, T, k, act, 0, m->n_experts);
  if (rc) return rc;
  RC_CHECK_ARG(!m->has_shared || m->gate_up[m->n_experts], "the shared expert is not loaded");
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  if ((rc = pf_scratch(m, T))) return rc;
  const cudaStream_t s = pick_stream(m->ctx, stream);
  if ((rc = pf_route(m, x_dev, T, k, router, renormalize, scaling, s))) return rc;
  PfRun r{T, k, act, gate_beta, value_beta, 0, m->n_experts, 0, m->has_shared ? T : 0, m->n_experts};
  if ((rc = pf_experts(m, x_dev, r, s))) return rc;
  rc_pf_combine_kernel<<<dim3((m->hidden / 8 + kPfCombineThreads - 1) / kPfCombineThreads, T), kPfCombineThreads, 0,
                      s>>>(m->pf->down, m->pf->slot_row, m->pf->slot_w, k, m->has_shared, m->hidden, out_dev);
  RC_CUDA_TRY(cudaGetLastError());
  if (ids_dev) RC_CUDA_TRY(cudaMemcpyAsync(ids_dev, m->pf->ids, (size_t)T * k * 4, cudaMemcpyDeviceToDevice, s));
  if (w_dev) RC_CUDA_TRY(cudaMemcpyAsync(w_dev, m->pf->weights, (size_t)T * k * 4, cudaMemcpyDeviceToDevice, s));
  return RC_OK;
}

int rc_moe_prefill_experts(rc_moe *m, const uint16_t *x_dev, int T, const int32_t *ids_dev, const float *w_dev,
                           int k, int act, float gate_beta, float value_beta, int with_shared, uint16_t *out_dev,
                           void *stream) {
  RC_CHECK_ARG(m && x_dev && ids_dev && w_dev && out_dev, "rc_moe_prefill_experts: NULL argument");
  RC_CHECK_ARG((reinterpret_cast<uintptr_t>(out_dev) & 15) == 0, "out must be 16-byte aligned");
  RC_CHECK_ARG(!with_shared || (m->has_shared && m->gate_up[m->n_experts]), "the shared expert is not loaded");
  int rc = pf_check(m, x_dev, T, k, act, 0, 0);
  if (rc) return rc;
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  if ((rc = pf_scratch(m, T))) return rc;
  const cudaStream_t s = pick_stream(m->ctx, stream);
  rc_pf_slots_kernel<<<(T + 127) / 128, 128, 0, s>>>(ids_dev, w_dev, T, k, with_shared ? m->n_experts : -1,
                                                 m->pf->slot_expert, m->pf->slot_w);
  RC_CUDA_TRY(cudaGetLastError());
  // every routed expert the caller names must be loaded: checked on the device
  // side by a null tile table entry (error word), so no host copy of the ids
  // a caller's route may name the shared expert (id n_experts) like a routed one
  const int max_id = m->n_experts + (m->has_shared ? 1 : 0);
  PfRun r{T, k, act, gate_beta, value_beta, 0, max_id, 0, with_shared ? T : 0, max_id};
  if ((rc = pf_experts(m, x_dev, r, s))) return rc;
  rc_pf_combine_kernel<<<dim3((m->hidden / 8 + kPfCombineThreads - 1) / kPfCombineThreads, T), kPfCombineThreads, 0,
                      s>>>(m->pf->down, m->pf->slot_row, m->pf->slot_w, k, with_shared, m->hidden, out_dev);
  RC_CUDA_TRY(cudaGetLastError());
  return RC_OK;
}

int rc_moe_prefill_local_routes(rc_moe *m, const uint16_t *x_dev, int T, const int32_t *ids_dev,
                                const float *w_dev, int k, int act, float gate_beta, float value_beta, int expert_lo,
                                int expert_hi, int shared_t0, int shared_tn, uint16_t *slot_out_dev, float *slot_w_dev,
                                void *stream) {
  RC_CHECK_ARG(m && x_dev && ids_dev && w_dev && slot_out_dev && slot_w_dev,
               "rc_moe_prefill_local_routes: NULL argument");
  RC_CHECK_ARG((reinterpret_cast<uintptr_t>(slot_out_dev) & 15) == 0, "slot_out must be 16-byte aligned");
  RC_CHECK_ARG(0 <= expert_lo && expert_lo <= expert_hi && expert_hi <= m->n_experts,
               "expert range [%d, %d) outside 0..%d", expert_lo, expert_hi, m->n_experts);
  RC_CHECK_ARG(shared_tn == 0 || (m->has_shared && shared_t0 >= 0 && shared_tn > 0 && shared_t0 + shared_tn <= T),
               "shared token range [%d, +%d) invalid for T=%d", shared_t0, shared_tn, T);
  int rc = pf_check(m, x_dev, T, k, act, expert_lo, expert_hi);
  if (rc) return rc;
  RC_CHECK_ARG(!shared_tn || m->gate_up[m->n_experts], "the shared expert is not loaded");
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  if ((rc = pf_scratch(m, T))) return rc;
  const cudaStream_t s = pick_stream(m->ctx, stream);
  // the caller's routes in ascending-ID slot order, as the router leaves them
  rc_pf_slots_kernel<<<(T + 127) / 128, 128, 0, s>>>(ids_dev, w_dev, T, k, m->has_shared ? m->n_experts : -1,
                                                 m->pf->slot_expert, m->pf->slot_w);
  RC_CUDA_TRY(cudaGetLastError());
  PfRun r{T, k, act, gate_beta, value_beta, expert_lo, expert_hi, shared_t0, shared_t0 + shared_tn, m->n_experts};
  if ((rc = pf_experts(m, x_dev, r, s))) return rc;
  rc_pf_slot_rows_kernel<<<T * (k + 1), 256, 0, s>>>(m->pf->down, m->pf->slot_row, m->hidden, slot_out_dev);
  RC_CUDA_TRY(cudaGetLastError());
  RC_CUDA_TRY(cudaMemcpyAsync(slot_w_dev, m->pf->slot_w, (size_t)T * k * 4, cudaMemcpyDeviceToDevice, s));
  return RC_OK;
}

int rc_moe_prefill_local(rc_moe *m, const uint16_t *x_dev, int T, int k, int router, int renormalize,
                         float scaling, int act, float gate_beta, float value_beta, int expert_lo, int expert_hi,
                         int shared_t0, int shared_tn, uint16_t *slot_out_dev, float *slot_w_dev, void *stream) {
  RC_CHECK_ARG(m && x_dev && slot_out_dev && slot_w_dev, "rc_moe_prefill_local: NULL argument");
  RC_CHECK_ARG(router == RC_ROUTER_SOFTMAX || router == RC_ROUTER_SIGMOID_BIAS, "unknown router %d", router);
  RC_CHECK_ARG((reinterpret_cast<uintptr_t>(slot_out_dev) & 15) == 0, "slot_out must be 16-byte aligned");
  RC_CHECK_ARG(0 <= expert_lo && expert_lo <= expert_hi && expert_hi <= m->n_experts,
               "expert range [%d, %d) outside 0..%d", expert_lo, expert_hi, m->n_experts);
  RC_CHECK_ARG(shared_tn == 0 || (m->has_shared && shared_t0 >= 0 && shared_tn > 0 && shared_t0 + shared_tn <= T),
               "shared token range [%d, +%d) invalid for T=%d", shared_t0, shared_tn, T);
  int rc = pf_check(m, x_dev, T, k, act, expert_lo, expert_hi);
  if (rc) return rc;
  RC_CHECK_ARG(!shared_tn || m->gate_up[m->n_experts], "the shared expert is not loaded");
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  if ((rc = pf_scratch(m, T))) return rc;
  const cudaStream_t s = pick_stream(m->ctx, stream);
  if ((rc = pf_route(m, x_dev, T, k, router, renormalize, scaling, s))) return rc;
  PfRun r{T, k, act, gate_beta, value_beta, expert_lo, expert_hi, shared_t0, shared_t0 + shared_tn, m->n_experts};
  if ((rc = pf_experts(m, x_dev, r, s))) return rc;
  rc_pf_slot_rows_kernel<<<T * (k + 1), 256, 0, s>>>(m->pf->down, m->pf->slot_row, m->hidden, slot_out_dev);
  RC_CUDA_TRY(cudaGetLastError());
  RC_CUDA_TRY(cudaMemcpyAsync(slot_w_dev, m->pf->slot_w, (size_t)T * k * 4, cudaMemcpyDeviceToDevice, s));
  return RC_OK;
}

int rc_moe_prefill_combine(rc_moe *m, const uint16_t *slot_out_dev, const float *slot_w_dev, int T, int k,
                           int with_shared, uint16_t *out_dev, void *stream) {
  RC_CHECK_ARG(m && slot_out_dev && slot_w_dev && out_dev, "rc_moe_prefill_combine: NULL argument");
  RC_CHECK_ARG(T >= 1 && T <= kPfMaxTokens && k >= 1 && k <= kMoeMaxK, "rc_moe_prefill_combine: bad T or k");
  RC_CHECK_ARG(!with_shared || m->has_shared, "this MoE layer has no shared expert");
  RC_CHECK_ARG(((reinterpret_cast<uintptr_t>(slot_out_dev) | reinterpret_cast<uintptr_t>(out_dev)) & 15) == 0,
               "slot rows and out must be 16-byte aligned");
  RC_CUDA_TRY(cudaSetDevice(m->ctx->device));
  const cudaStream_t s = pick_stream(m->ctx, stream);
  // slot rows laid out [T][k+1][hidden]: slot_row[t][r] = t*(k+1)+r
  int rc = pf_scratch(m, T);
  if (rc) return rc;
  // identity slot-row table, so that the combine kernel is shared with the
  // single-GPU path
  rc_pf_identity_rows_kernel<<<(T * (k + 1) + 255) / 256, 256, 0, s>>>(m->pf->slot_row, T * (k + 1));
  RC_CUDA_TRY(cudaGetLastError());
  rc_pf_combine_kernel<<<dim3((m->hidden / 8 + kPfCombineThreads - 1) / kPfCombineThreads, T), kPfCombineThreads, 0,
                      s>>>(slot_out_dev, m->pf->slot_row, slot_w_dev, k, with_shared, m->hidden, out_dev);
  RC_CUDA_TRY(cudaGetLastError());
  return RC_OK;
}

}  // extern "C"
