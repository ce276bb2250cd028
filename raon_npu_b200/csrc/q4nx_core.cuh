// Device code shared by the q4nx GEMV and the MoE expert GEMVs: activation
// staging in mma B-fragment order, the per-unit tensor-core inner product, and
// the f32 accumulator fragments.  Templates over a params type P that
// provides x, x_dtype, ldx, tokens, slots, x_vec and kb.
//
// Arithmetic of one unit (16 rows x 256 columns, 8 groups of 32 columns):
//     y[r] += sum_g scale[r,g] * sum_{k in g} code[r,k] x[k] + min[r,g] * S[g],
//     S[g] = sum_{k in g} x[k]
// (the factorisation of kernels/gemv/q4nx_gemv.cc:88-124, every product and
// partial sum in f32).
//
// Activations.  Each (token slot, 256-column block) is scaled by a power of
// two 2^s chosen from the block's largest magnitude (x' = x 2^s, |x'| < 2^15)
// and held as f16: exact for every bf16 value whose scaled magnitude is at
// least 2^-14 (all but values below 2^-29 of the block maximum, whose
// rounding moves a dot product by less than 2^-40 of its scale).
//
// Codes.  A nibble masked into the low bits of an f16 half-word IS an exact
// f16 value -- a subnormal: code * 2^-24 for bits 0-3 of each half-word and
// 16 code * 2^-24 for bits 4-7.  So one AND per two codes (and one shift per
// four) makes the mma's A operand, with no offset to cancel: rows g of a
// fragment take the bits 0-3 nibbles, rows g+8 the bits 4-7 nibbles, and
//     d[g] = 2^-24 sum code x',      d[g+8] = 2^-20 sum code x'
// (the tensor core multiplies f16 subnormals exactly).  The unit's result in
// the scaled domain, times 2^-24, is
//     P[r] = sum_g sc'[r,g] d[r,g] + min[r,g] S'[g] 2^-24
// with sc' = scale (rows g) or scale/16 (rows g+8).  The min term, a K = 8
// contraction over the groups, runs as three bf16 m16n8k8 mmas over S' 2^-24
// split into three bf16 parts (2^-25 relative).  The unit's result returns to
// x's scale exactly: Q = (2^24 P) 2^-s, two exact multiplies.  A tile's result
// is the sum of its units' Q in k-block order, whatever the partition.
#pragma once


#include "rc_device.cuh"
#include "rc_internal.cuh"

namespace rc {

// Staged activations (shared or global):
// xfrag (f16): for token block tb (8 slots) and k16-step s, lane l = 4g+q holds
//   word0 = {x'[slot g][16s+2q], x'[g][16s+2q+1]}, word1 = {x'[g][16s+2q+8], ..+9}
//   (the mma B fragment), stored so a lane reads 4 steps as two 16-byte loads:
//   word index ((tb*(K/64) + s/4)*32 + l)*8 + (s%4)*2 + {0,1}.
// aux, per (token block tb, k-block kb), u = tb*KB + kb:
//   bmin[u*32 + l]: a uint4 of bf16 pairs {S'1, S'2, S'3, -} (S' 2^-24 =
//     S'1 + S'2 + S'3) for token g, groups 2q and 2q+1 (the m16n8k8 B
//     fragments of the min term);
//   then inv[u*8 + slot]: the f32 2^-s of the slot's block.
// Token slots: bf16 input -> slot = token; f32 input -> slots 2t / 2t+1 hold
// the f16 hi part of token t and the f16 residual (each with its own scale;
// x = hi + lo to about 2^-22 relative).
__host__ __device__ constexpr size_t xfrag_bytes(int ntb, int k) { return (size_t)ntb * 16 * k; }
__host__ __device__ constexpr size_t xaux_bytes(int ntb, int k) { return (size_t)ntb * (k / 256) * (512 + 32); }

// Eight consecutive activations of a slot's token as f32 (0 past the tokens).
template <class P>
__device__ __forceinline__ void load8f(const P &p, int slot, int k, float (&v)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = 0.f;
  if (p.x_dtype == RC_DTYPE_BF16) {
    if (slot >= p.tokens) return;
    const uint16_t *row = static_cast<const uint16_t *>(p.x) + (size_t)slot * p.ldx + k;
    uint32_t w[4];
    if (p.x_vec) {
      const uint4 u = *reinterpret_cast<const uint4 *>(row);
      w[0] = u.x, w[1] = u.y, w[2] = u.z, w[3] = u.w;
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) w[i] = (uint32_t)row[2 * i] | ((uint32_t)row[2 * i + 1] << 16);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = bf16_lo_f32(w[i]);
      v[2 * i + 1] = bf16_hi_f32(w[i]);
    }
    return;
  }
  const int t = slot >> 1;
  if (t >= p.tokens) return;
  const float *row = static_cast<const float *>(p.x) + (size_t)t * p.ldx + k;
  if (p.x_vec) {
    const float4 a = *reinterpret_cast<const float4 *>(row), b = *reinterpret_cast<const float4 *>(row + 4);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = row[i];
  }
}

// Block exponent: 2^s brings the block maximum amax into [2^14, 2^15).  No
// scaling for a zero, subnormal, infinite or NaN maximum (NaN and inf stay
// what they are under any scale).
__device__ __forceinline__ int block_shift(float amax) {
  const int e = (int)(__float_as_uint(amax) >> 23);
  if (e == 0 || e >= 255) return 0;
  const int s = 141 - e;            // 14 - (e - 127)
  return s > 126 ? 126 : s;         // s >= 141 - 254 = -113
}

// Largest |v| over the warp (every lane of the warp calls it).
__device__ __forceinline__ float warp_absmax(const float (&v)[8]) {
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(v[i]));
  return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m)));
}

// One staged item: eight activations v of a slot (one warp = one 256-column
// block of that slot): block scale, f16 fragment words, group sums, aux words.
// Each group of 32 columns is summed as four sequential 8-element partials
// combined pairwise, a fixed order.  BF16: v came from bf16 input (slot =
// token); otherwise from f32 input, odd slots holding the residual of the
// even slot's f16 value.
template <bool BF16>
__device__ __forceinline__ void stage_core(float (&v)[8], int slot, int c8, int k64, int kb, uint32_t *xf,
                                           uint16_t *bmin16, float *inv) {
  int s = block_shift(warp_absmax(v));
  if (!BF16 && (slot & 1)) {
    // the residual of the hi slot's f16 value, with its own block scale
    const float sc = pow2f(s), isc = pow2f(-s);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] -= f16_to_f32(f32_to_f16_rn(v[i] * sc)) * isc;
    s = block_shift(warp_absmax(v));
  }
  const float sc = pow2f(s);
  uint32_t hw[4];
  float part = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a = v[2 * i] * sc, c = v[2 * i + 1] * sc;
    const __half2 h = __floats2half2_rn(a, c);
    hw[i] = *reinterpret_cast<const uint32_t *>(&h);
    if (BF16) {
      // a bf16 value times 2^s is exact in f16 (down to the f16 subnormal
      // range, 2^-29 of the block maximum): sum the exact values
      part += a;
      part += c;
    } else {
      const float2 f = __half22float2(h);
      part += f.x;
      part += f.y;
    }
  }
  const int kk = c8 * 8;
  const int st = kk >> 4, j = (kk >> 3) & 1, tb = slot >> 3, g = slot & 7;
  const size_t base = ((size_t)tb * k64 + (st >> 2)) * 32 * 8 + (st & 3) * 2 + j;
#pragma unroll
  for (int q = 0; q < 4; ++q) xf[base + (size_t)(g * 4 + q) * 8] = hw[q];
  part += __shfl_xor_sync(0xffffffffu, part, 1);
  part += __shfl_xor_sync(0xffffffffu, part, 2);
  if ((c8 & 3) == 0) {
    const int grp = c8 >> 2, kbi = grp >> 3, gi = grp & 7;
    const size_t u = (size_t)tb * kb + kbi;
    const float sp = part * 5.9604644775390625e-08f;   // S' 2^-24 (exact)
    const uint16_t s1 = f32_to_bf16_rne(sp);
    const float r1 = sp - bf16_to_f32(s1);
    const uint16_t s2 = f32_to_bf16_rne(r1);
    uint16_t *w = bmin16 + (u * 32 + g * 4 + (gi >> 1)) * 8 + (gi & 1);
    w[0] = s1;
    w[2] = s2;
    w[4] = f32_to_bf16_rne(r1 - bf16_to_f32(s2));
    w[6] = 0;
  }
  if ((c8 & 31) == 0) inv[((size_t)tb * kb + (c8 >> 5)) * 8 + g] = pow2f(-s);
}

// A staged bf16 item as an out-of-line call: the batched loop below calls it
// from several unrolled sites; one body keeps a kernel with many phases small
// enough for the instruction cache.
static __device__ __noinline__ void stage_item_bf16(uint4 raw, int slot, int c8, int k64, int kb, uint32_t *xf,
                                             uint16_t *bmin16, float *inv) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  float v[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = bf16_lo_f32(w[i]);
    v[2 * i + 1] = bf16_hi_f32(w[i]);
  }
  stage_core<true>(v, slot, c8, k64, kb, xf, bmin16, inv);
}

// How a build_activations instance is compiled: either input dtype (by
// p.x_dtype) with the item code inline (the GEMV kernels: fastest), or bf16
// input only with one out-of-line item body (the persistent decode kernel,
// whose many phases must share the instruction cache).
enum StageMode : int { kStageAny = 0, kStageBf16Compact = 1 };

// Build the fragment-ordered activations and their aux words for all token
// slots of ntb blocks.  Called by every thread of the CTA (or grid); ``stride``
// threads cooperate, ``first`` and ``stride`` multiples of 32 apart per warp,
// so a warp's 32 consecutive items are exactly one (slot, 256-column block):
// the block maximum is a warp reduction.  A thread issues the loads of a batch
// of items before processing any (one memory round trip per batch): 8 packed
// bf16 items, or 4 f32 items.
template <bool SHARED, class P, int DT = kStageAny>
__device__ __forceinline__ void build_activations(const P &p, int ntb, uint32_t *xf, void *aux, long long first,
                                                  long long stride) {
  const int k = p.kb * kUnitK, k64 = k / 64, c8n = k / 8;
  const size_t nu = (size_t)ntb * p.kb;
  uint16_t *bmin16 = static_cast<uint16_t *>(aux);
  float *inv = reinterpret_cast<float *>(bmin16 + nu * 256);
  // Only the slots that hold data are built: the B columns of empty slots feed
  // mma output columns that are never stored, so their contents do not matter.
  // 32-bit indices: slots <= 32 and K / 8 < 2^20, so total < 2^25
  const int total = p.slots * c8n;   // multiple of 32: whole warps iterate together
  const int first32 = (int)first, stride32 = (int)stride;
  if (DT == kStageBf16Compact || p.x_dtype == RC_DTYPE_BF16) {
    constexpr int kBatch = 8;
    for (int base0 = first32; base0 < total; base0 += stride32 * kBatch) {
      uint4 raw[kBatch];
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int idx = base0 + b * stride32;
        raw[b] = make_uint4(0, 0, 0, 0);
        if (idx < total) {
          const int slot = idx / c8n, c8 = idx - slot * c8n;
          if (slot < p.tokens) {
            const uint16_t *row = static_cast<const uint16_t *>(p.x) + (size_t)slot * p.ldx + c8 * 8;
            if (p.x_vec) {
              raw[b] = *reinterpret_cast<const uint4 *>(row);
            } else {
              uint32_t w[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) w[i] = (uint32_t)row[2 * i] | ((uint32_t)row[2 * i + 1] << 16);
              raw[b] = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
        }
      }
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        const int idx = base0 + b * stride32;
        if (idx >= total) break;
        const int slot = idx / c8n, c8 = idx - slot * c8n;
        if (DT == kStageBf16Compact) {
          stage_item_bf16(raw[b], slot, c8, k64, p.kb, xf, bmin16, inv);
        } else {
          const uint32_t w[4] = {raw[b].x, raw[b].y, raw[b].z, raw[b].w};
          float v[8];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            v[2 * i] = bf16_lo_f32(w[i]);
            v[2 * i + 1] = bf16_hi_f32(w[i]);
          }
          stage_core<true>(v, slot, c8, k64, p.kb, xf, bmin16, inv);
        }
      }
    }
    return;
  }
  if (DT == kStageBf16Compact) return;
  constexpr int kBatch = 4;
  for (int base0 = first32; base0 < total; base0 += stride32 * kBatch) {
    float v[kBatch][8];
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int idx = base0 + b * stride32;
      if (idx < total) {
        const int slot = idx / c8n, c8 = idx - slot * c8n;
        load8f(p, slot, c8 * 8, v[b]);
      }
    }
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const int idx = base0 + b * stride32;
      if (idx >= total) break;
      const int slot = idx / c8n, c8 = idx - slot * c8n;
      stage_core<false>(v[b], slot, c8, k64, p.kb, xf, bmin16, inv);
    }
  }
}

template <int NTB>
struct Acc {
  float v[NTB][4];
};

template <int NTB>
__device__ __forceinline__ void acc_zero(Acc<NTB> &a) {
#pragma unroll
  for (int tb = 0; tb < NTB; ++tb) a.v[tb][0] = a.v[tb][1] = a.v[tb][2] = a.v[tb][3] = 0.f;
}

template <int NTB>
__device__ __forceinline__ void acc_add(Acc<NTB> &s, const float4 (&v)[NTB]) {
#pragma unroll
  for (int tb = 0; tb < NTB; ++tb) {
    s.v[tb][0] += v[tb].x;
    s.v[tb][1] += v[tb].y;
    s.v[tb][2] += v[tb].z;
    s.v[tb][3] += v[tb].w;
  }
}

// One k-block of staged activations: the min-term fragment and the inverse
// scales of the lane's two columns in registers, per token block, and the B
// fragments of the block's 16 k16-steps -- in registers for one token block,
// read from the staging area per step for two (whose 64 registers would
// spill).
template <int NTB>
struct XFrag {
  uint4 xa[4], xb[4];                 // NTB == 1
  const uint4 *xv[NTB];               // NTB == 2: the lane's fragments of step 0
  int step;                           // NTB == 2: uint4 stride from one 4-step group to the next
  bool shared;
  uint4 bm[NTB];
  float2 inv[NTB];
};

template <int NTB>
__device__ __forceinline__ void xfrag_step(const XFrag<NTB> &r, int tb, int s4, uint4 &xa, uint4 &xb) {
  if (NTB == 1) {
    xa = r.xa[s4];
    xb = r.xb[s4];
  } else if (r.shared) {
    xa = r.xv[tb][s4 * r.step];
    xb = r.xv[tb][s4 * r.step + 1];
  } else {
    xa = __ldg(r.xv[tb] + s4 * r.step);
    xb = __ldg(r.xv[tb] + s4 * r.step + 1);
  }
}

// Load k-block kbi of token blocks tb0 .. tb0+NTB-1 of a staging area that
// holds nblocks token blocks of kb k-blocks.
template <int NTB, bool SHARED>
__device__ __forceinline__ void load_xfrag(XFrag<NTB> &r, const uint32_t *xf, const void *aux, int nblocks, int tb0,
                                           int kb, int kbi, int lane) {
  const int k64 = kb * 4, q = lane & 3;
  const size_t nu = (size_t)nblocks * kb;
  const uint4 *bm = static_cast<const uint4 *>(aux);
  const float *inv = reinterpret_cast<const float *>(bm + nu * 32);
  r.shared = SHARED;
  r.step = 64;
#pragma unroll
  for (int tb = 0; tb < NTB; ++tb) {
    const int blk = tb0 + tb;
    const size_t u = (size_t)blk * kb + kbi;
    const uint4 *xv = reinterpret_cast<const uint4 *>(xf + (((size_t)blk * k64 + kbi * 4) * 32 + lane) * 8);
    r.xv[tb] = xv;
    if (NTB == 1) {
#pragma unroll
      for (int s4 = 0; s4 < 4; ++s4) {
        r.xa[s4] = SHARED ? xv[s4 * 64] : __ldg(xv + s4 * 64);
        r.xb[s4] = SHARED ? xv[s4 * 64 + 1] : __ldg(xv + s4 * 64 + 1);
      }
    }
    const uint4 *bp = bm + u * 32 + lane;
    const float2 *ip = reinterpret_cast<const float2 *>(inv + u * 8 + 2 * q);
    r.bm[tb] = SHARED ? *bp : __ldg(bp);
    r.inv[tb] = SHARED ? *ip : __ldg(ip);
  }
}

// The eight codes of a word as f16 subnormal pairs in the mma A-fragment
// order: nibbles 0/4 -> a0 (code 2^-24), 1/5 -> a1 (16 code 2^-24), 2/6 -> a2,
// 3/7 -> a3.
__device__ __forceinline__ void codes_to_f16x4(uint32_t w, uint32_t &a0, uint32_t &a1, uint32_t &a2, uint32_t &a3) {
  const uint32_t w8 = w >> 8;
  a0 = w & 0x000F000Fu;
  a1 = w & 0x00F000F0u;
  a2 = w8 & 0x000F000Fu;
  a3 = w8 & 0x00F000F0u;
}

// The unit's result in the scaled domain times 2^-24, P (from zero).
template <int NTB>
__device__ __forceinline__ void unit_scaled(const uint8_t *unit, const XFrag<NTB> &r, int lane, Acc<NTB> &P) {
  const int g = lane >> 2, q = lane & 3;
  const uint4 *codes = reinterpret_cast<const uint4 *>(unit) + lane;
  const uint4 *params = reinterpret_cast<const uint4 *>(unit + kUnitCodeBytes + g * 64);
  {
    // min of groups 2q (x: row g, y: row g+8) and 2q+1 (z, w): the A fragment
    // of the K = 8 group contraction
    const uint4 pq = params[q];
    const uint32_t amn0 = __byte_perm(pq.x, pq.z, 0x7632), amn1 = __byte_perm(pq.y, pq.w, 0x7632);
#pragma unroll
    for (int tb = 0; tb < NTB; ++tb) {
      mma_bf16_1688<true>(P.v[tb], amn0, amn1, r.bm[tb].x);
      mma_bf16_1688<false>(P.v[tb], amn0, amn1, r.bm[tb].y);
      mma_bf16_1688<false>(P.v[tb], amn0, amn1, r.bm[tb].z);
    }
  }
#pragma unroll
  for (int s4 = 0; s4 < 4; ++s4) {
    const uint4 cw = codes[s4 * 32];
    const uint4 sm = params[s4];
    uint4 xa[NTB], xb[NTB];
#pragma unroll
    for (int tb = 0; tb < NTB; ++tb) xfrag_step(r, tb, s4, xa[tb], xb[tb]);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint32_t wa = half ? cw.z : cw.x;
      const uint32_t wb = half ? cw.w : cw.y;
      float d[NTB][4];
      {
        uint32_t a0, a1, a2, a3;
        codes_to_f16x4(wa, a0, a1, a2, a3);
#pragma unroll
        for (int tb = 0; tb < NTB; ++tb)
          mma_f16_16816_zero(d[tb], a0, a1, a2, a3, half ? xb[tb].x : xa[tb].x, half ? xb[tb].y : xa[tb].y);
      }
      {
        uint32_t a0, a1, a2, a3;
        codes_to_f16x4(wb, a0, a1, a2, a3);
#pragma unroll
        for (int tb = 0; tb < NTB; ++tb)
          mma_f16_16816(d[tb], a0, a1, a2, a3, half ? xb[tb].z : xa[tb].z, half ? xb[tb].w : xa[tb].w);
      }
      const uint32_t lo = half ? sm.z : sm.x;   // {scale[g], min[g]}
      const uint32_t hi = half ? sm.w : sm.y;   // {scale[g+8], min[g+8]}
      const float sc0 = bf16_lo_f32(lo), sc1 = bf16_lo_f32(hi) * 0.0625f;
#pragma unroll
      for (int tb = 0; tb < NTB; ++tb) {
        P.v[tb][0] = fmaf(sc0, d[tb][0], P.v[tb][0]);
        P.v[tb][1] = fmaf(sc0, d[tb][1], P.v[tb][1]);
        P.v[tb][2] = fmaf(sc1, d[tb][2], P.v[tb][2]);
        P.v[tb][3] = fmaf(sc1, d[tb][3], P.v[tb][3]);
      }
    }
  }
}

// acc += Q = (2^24 P) 2^-s (exact scalings, so the fused multiply-add rounds
// once, as the separate multiply and add would).
constexpr float kTwo24 = 16777216.f;

template <int NTB>
__device__ __forceinline__ void unit_accumulate(const uint8_t *unit, const XFrag<NTB> &r, int lane, Acc<NTB> &acc) {
  Acc<NTB> P;
  unit_scaled<NTB>(unit, r, lane, P);
#pragma unroll
  for (int tb = 0; tb < NTB; ++tb) {
    acc.v[tb][0] = fmaf(r.inv[tb].x, P.v[tb][0] * kTwo24, acc.v[tb][0]);
    acc.v[tb][1] = fmaf(r.inv[tb].y, P.v[tb][1] * kTwo24, acc.v[tb][1]);
    acc.v[tb][2] = fmaf(r.inv[tb].x, P.v[tb][2] * kTwo24, acc.v[tb][2]);
    acc.v[tb][3] = fmaf(r.inv[tb].y, P.v[tb][3] * kTwo24, acc.v[tb][3]);
  }
}

// The unit's result Q = (2^24 P) 2^-s as float4 per token block (for a
// partial slot).
template <int NTB>
__device__ __forceinline__ void unit_result(const uint8_t *unit, const XFrag<NTB> &r, int lane, float4 (&Q)[NTB]) {
  Acc<NTB> P;
  unit_scaled<NTB>(unit, r, lane, P);
#pragma unroll
  for (int tb = 0; tb < NTB; ++tb)
    Q[tb] = make_float4(r.inv[tb].x * (P.v[tb][0] * kTwo24), r.inv[tb].y * (P.v[tb][1] * kTwo24),
                        r.inv[tb].x * (P.v[tb][2] * kTwo24), r.inv[tb].y * (P.v[tb][3] * kTwo24));
}

// ------------------------------------------------------- round schedule --
// A CTA's tile range is processed in rounds of R tiles.  The units of a round
// (its tiles x kb k-blocks) are ordered k-block-major and cut into W equal
// contiguous chunks, one per warp: a warp meets one k-block in a round (two
// at a chunk boundary) and the same one round after round, so its activation
// fragments stay in registers.  Each unit's result goes to its own partial
// slot (ti*kb + kbi within the round); after the round's barrier the tile's
// partials are summed in k-block order, so a tile's result is the same
// whatever the partition.
struct RoundCursor {
  int n_tiles, R, kb, W, w;
  int round, Rr, u, u_end;   // round, its tile count, position in the round, end of the warp's chunk
  int kbi, ti;               // the unit: k-block and tile within the round

  __device__ __forceinline__ void start_round() {
    Rr = n_tiles - round * R < R ? n_tiles - round * R : R;
    const int U = Rr * kb;
    u = w * U / W;
    u_end = (w + 1) * U / W;
    kbi = u / Rr;
    ti = u - kbi * Rr;
  }
  __device__ __forceinline__ bool valid() const { return round * R < n_tiles; }
  __device__ __forceinline__ void skip_empty() {
    while (valid() && u >= u_end) {
      ++round;
      if (valid()) start_round();
    }
  }
  __device__ __forceinline__ void init(int n_tiles_, int R_, int kb_, int W_, int w_) {
    n_tiles = n_tiles_, R = R_, kb = kb_, W = W_, w = w_;
    round = 0;
    if (valid()) {
      start_round();
      skip_empty();
    }
  }
  __device__ __forceinline__ void next() {
    ++u;
    if (++ti == Rr) ti = 0, ++kbi;
    if (u >= u_end) {
      ++round;
      if (valid()) start_round();
      skip_empty();
    }
  }
  __device__ __forceinline__ int tile() const { return round * R + ti; }   // within the CTA's range
  __device__ __forceinline__ int slot() const { return ti * kb + kbi; }    // partial slot in the round
};

// Rounds of a CTA's range of n_tiles tiles.
__host__ __device__ __forceinline__ int round_count(int n_tiles, int R) { return (n_tiles + R - 1) / R; }

}  // namespace rc
