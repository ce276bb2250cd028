// Device code shared by the q4nx GEMV and the grouped MoE expert GEMV:
// activation staging in mma B-fragment order, the per-unit tensor-core inner
// product, and the f32 accumulator fragments.  Templates over a params type P
// that provides x, x_dtype, ldx, tokens, slots, x_vec and kb.
#pragma once

#include "rc_device.cuh"
#include "rc_internal.cuh"

namespace rc {

// Activation layout (shared or global):
// xfrag: for token block tb (8 token slots) and k16-step s, lane l = 4g+q holds
//   word0 = {x[slot g][16s+2q], x[g][16s+2q+1]}, word1 = {x[g][16s+2q+8], ..+9}
// (the mma B fragment); stored so a lane reads 4 steps as two 16-byte loads:
//   word index ((tb*(K/64) + s/4)*32 + l)*8 + (s%4)*2 + {0,1}.
// gsum: for tb, group grp = 8*kbi + gi and quad lane q, float2 {S[2q], S[2q+1]}
//   at float index ((((tb*KB + kbi)*4 + q)*8 + gi)*2.
// Token slots: bf16 input -> slot = token; f32 input -> slots 2t / 2t+1 hold
// the bf16 hi / lo parts of token t (x = hi + lo to 2^-17 relative).
__host__ __device__ constexpr size_t xfrag_bytes(int ntb, int k) { return (size_t)ntb * 16 * k; }
__host__ __device__ constexpr size_t gsum_bytes(int ntb, int k) { return (size_t)ntb * k; }

// Eight consecutive activations x[slot][k..k+8) as bf16 pairs.
template <class P>
__device__ __forceinline__ void load8(const P &p, int slot, int k, uint32_t (&w)[4]) {
  w[0] = w[1] = w[2] = w[3] = 0u;
  if (p.x_dtype == RC_DTYPE_BF16) {
    if (slot >= p.tokens) return;
    const uint16_t *row = static_cast<const uint16_t *>(p.x) + (size_t)slot * p.ldx + k;
    if (p.x_vec) {
      const uint4 v = *reinterpret_cast<const uint4 *>(row);
      w[0] = v.x, w[1] = v.y, w[2] = v.z, w[3] = v.w;
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) w[i] = (uint32_t)row[2 * i] | ((uint32_t)row[2 * i + 1] << 16);
    }
    return;
  }
  const int t = slot >> 1;
  if (t >= p.tokens) return;
  const float *row = static_cast<const float *>(p.x) + (size_t)t * p.ldx + k;
  float v[8];
  if (p.x_vec) {
    const float4 a = *reinterpret_cast<const float4 *>(row), b = *reinterpret_cast<const float4 *>(row + 4);
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = row[i];
  }
  uint32_t h[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint16_t hi = f32_to_bf16_rne(v[i]);
    h[i] = (slot & 1) ? f32_to_bf16_rne(v[i] - bf16_to_f32(hi)) : hi;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = h[2 * i] | (h[2 * i + 1] << 16);
}

// Build the fragment-ordered activations and group sums for all token slots
// of NTB blocks.  Called by every thread of the CTA (or grid); ``stride``
// threads cooperate.  Each group of 32 columns is summed as four sequential
// 8-element partials combined pairwise, a fixed order.
template <bool SHARED, class P>
__device__ __forceinline__ void build_activations(const P &p, int ntb, uint32_t *xf, float *gs,
                                                  long long first, long long stride) {
  const int k = p.kb * kUnitK, k64 = k / 64, c8n = k / 8;
  // Only the slots that hold data are built: the B columns of empty slots feed
  // mma output columns that are never stored, so their contents do not matter.
  const long long total = (long long)p.slots * c8n;   // multiple of 32: whole warps iterate together
  // Four chunks' loads are issued before any is used, so a thread pays one
  // memory round trip per four chunks instead of one per chunk.
  constexpr int kBatch = 4;
  for (long long base0 = first; base0 < total; base0 += stride * kBatch) {
    uint32_t w[kBatch][4];
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const long long idx = base0 + b * stride;
      if (idx < total) {
        const int slot = (int)(idx / c8n), c8 = (int)(idx - (long long)slot * c8n);
        load8(p, slot, c8 * 8, w[b]);
      }
    }
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const long long idx = base0 + b * stride;
      if (idx >= total) break;
      const int slot = (int)(idx / c8n), c8 = (int)(idx - (long long)slot * c8n);
      const int kk = c8 * 8;
      float part = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        part += bf16_to_f32(w[b][i] & 0xFFFFu);
        part += bf16_to_f32(w[b][i] >> 16);
      }
      const int s = kk >> 4, j = (kk >> 3) & 1, tb = slot >> 3, g = slot & 7;
      const size_t base = ((size_t)tb * k64 + (s >> 2)) * 32 * 8 + (s & 3) * 2 + j;
#pragma unroll
      for (int q = 0; q < 4; ++q) xf[base + (size_t)(g * 4 + q) * 8] = w[b][q];
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      if ((c8 & 3) == 0) {
        const int grp = c8 >> 2, kbi = grp >> 3, gi = grp & 7;
        gs[((((size_t)tb * p.kb + kbi) * 4 + (g >> 1)) * 8 + gi) * 2 + (g & 1)] = part;
      }
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

template <int NTB, bool STAGED, class P>
__device__ __forceinline__ void compute_unit(const uint8_t *unit, const uint32_t *xf, const float *gs,
                                             const P &p, int kbi, int lane, Acc<NTB> &acc) {
  const int g = lane >> 2, q = lane & 3;
  const uint4 *codes = reinterpret_cast<const uint4 *>(unit) + lane;
  const uint4 *params = reinterpret_cast<const uint4 *>(unit + kUnitCodeBytes + g * 64);
  const int k64 = p.kb * 4;
#pragma unroll
  for (int s4 = 0; s4 < 4; ++s4) {
    const uint4 cw = codes[s4 * 32];
    const uint4 sm = params[s4];
    uint4 xa[NTB], xb[NTB];
    float4 gsv[NTB];
#pragma unroll
    for (int tb = 0; tb < NTB; ++tb) {
      const uint4 *xv = reinterpret_cast<const uint4 *>(xf + ((tb * k64 + kbi * 4 + s4) * 32 + lane) * 8);
      const float4 *gp = reinterpret_cast<const float4 *>(gs + (((tb * p.kb + kbi) * 4 + q) * 8 + 2 * s4) * 2);
      if (STAGED) {
        xa[tb] = xv[0];
        xb[tb] = xv[1];
        gsv[tb] = gp[0];
      } else {
        xa[tb] = __ldg(xv);
        xb[tb] = __ldg(xv + 1);
        gsv[tb] = __ldg(gp);
      }
    }
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint32_t wa = half ? cw.z : cw.x;
      const uint32_t wb = half ? cw.w : cw.y;
      float d[NTB][4];
#pragma unroll
      for (int tb = 0; tb < NTB; ++tb) d[tb][0] = d[tb][1] = d[tb][2] = d[tb][3] = 0.f;
      {
        const uint32_t a0 = codes_to_bf16x2<0>(wa), a1 = codes_to_bf16x2<1>(wa);
        const uint32_t a2 = codes_to_bf16x2<2>(wa), a3 = codes_to_bf16x2<3>(wa);
#pragma unroll
        for (int tb = 0; tb < NTB; ++tb)
          mma_bf16_16816(d[tb], a0, a1, a2, a3, half ? xb[tb].x : xa[tb].x, half ? xb[tb].y : xa[tb].y);
      }
      {
        const uint32_t a0 = codes_to_bf16x2<0>(wb), a1 = codes_to_bf16x2<1>(wb);
        const uint32_t a2 = codes_to_bf16x2<2>(wb), a3 = codes_to_bf16x2<3>(wb);
#pragma unroll
        for (int tb = 0; tb < NTB; ++tb)
          mma_bf16_16816(d[tb], a0, a1, a2, a3, half ? xb[tb].z : xa[tb].z, half ? xb[tb].w : xa[tb].w);
      }
      const uint32_t lo = half ? sm.z : sm.x;   // {scale[g], min[g]}
      const uint32_t hi = half ? sm.w : sm.y;   // {scale[g+8], min[g+8]}
      const float sc0 = bf16_lo_f32(lo), mn0 = bf16_hi_f32(lo);
      const float sc1 = bf16_lo_f32(hi), mn1 = bf16_hi_f32(hi);
      const float mp0 = fmaf(-128.f, sc0, mn0), mp1 = fmaf(-128.f, sc1, mn1);
#pragma unroll
      for (int tb = 0; tb < NTB; ++tb) {
        const float S0 = half ? gsv[tb].z : gsv[tb].x;
        const float S1 = half ? gsv[tb].w : gsv[tb].y;
        acc.v[tb][0] = fmaf(sc0, d[tb][0], fmaf(mp0, S0, acc.v[tb][0]));
        acc.v[tb][1] = fmaf(sc0, d[tb][1], fmaf(mp0, S1, acc.v[tb][1]));
        acc.v[tb][2] = fmaf(sc1, d[tb][2], fmaf(mp1, S0, acc.v[tb][2]));
        acc.v[tb][3] = fmaf(sc1, d[tb][3], fmaf(mp1, S1, acc.v[tb][3]));
      }
    }
  }
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

}  // namespace rc
