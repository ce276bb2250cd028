// Device-side helpers: bf16 bit arithmetic, mbarrier / bulk-copy PTX wrappers,
// programmatic dependent launch controls, and the legacy-register bf16 mma.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rc {

// f32 -> bf16 bits, round to nearest even; every NaN becomes 0x7FC0 (the
// reference's converter, quant/q4nx.py:32-44, host/weights.py:104-115).
__device__ __forceinline__ uint16_t f32_to_bf16_rne(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FC0;
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

__device__ __forceinline__ float bf16_to_f32(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

__device__ __forceinline__ float bf16_round(float f) { return bf16_to_f32(f32_to_bf16_rne(f)); }

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier --
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Raise the transaction count a phase waits for, without arriving.
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Arrive (count 1) without a transaction count.
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase ``parity`` of a barrier, giving up after ``limit_ns`` of
// global time.  Returns false on timeout; callers record an error word and
// unwind instead of hanging the GPU.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  uint64_t limit_ns = 1000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > limit_ns) return false;
  }
}

// mbar_wait_bounded for a whole warp (every lane calls it): one verdict for
// all lanes, so a timeout never splits the warp before warp-wide instructions.
__device__ __forceinline__ bool mbar_wait_bounded_warp(uint32_t bar, uint32_t parity) {
  return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity));
}

// Router order: larger value first; NaN after every number; equal values (and
// NaNs among themselves) by lower index -- the order of numpy's stable argsort
// of the negated values, a strict total order even on NaN input.
__device__ __forceinline__ bool route_before(float a, int ia, float b, int ib) {
  const bool na = a != a, nb = b != b;
  if (na || nb) return nb ? (!na || ia < ib) : false;
  return a > b || (a == b && ia < ib);
}

// ---------------------------------------------------------- bulk copies --
// L2 policy for data that is streamed exactly once (weights).
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 1-D bulk copy global -> this CTA's shared memory, completing on ``bar``.
// Both addresses 16-byte aligned, ``bytes`` a multiple of 16.  The copy
// lands in the issuing CTA's own shared memory only.
__device__ __forceinline__ void bulk_copy_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

// The same without a cache hint (weights that several CTAs re-read soon).
// Prefetch ``bytes`` (a multiple of 16, 16-byte aligned) of global memory
// into L2 without a destination in shared memory.
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void bulk_copy_g2s_plain(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// ------------------------------------------------- grid-scope atomics --
__device__ __forceinline__ unsigned long long atom_add_release_gpu(unsigned long long *p, unsigned long long v) {
  unsigned long long old;
  asm volatile("atom.add.release.gpu.global.u64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
  return old;
}
__device__ __forceinline__ unsigned long long ld_acquire_gpu(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// System scope (peer GPUs over NVLink): a releasing add to a counter in
// another GPU's memory, and an acquiring load of a counter peers add to.
__device__ __forceinline__ void red_add_release_sys(unsigned long long *p, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys(unsigned long long *p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Division by a divisor fixed for a loop: q = umulhi(n, ceil(2^32 / d)),
// exact while n * d < 2^32 (the callers' tile and unit indices stay below
// 2^20 and their divisors below 2^12).
struct FastDiv {
  uint32_t d, m;
};
__host__ __device__ __forceinline__ FastDiv make_fastdiv(uint32_t d) {
  return FastDiv{d, d <= 1 ? 0u : 0xFFFFFFFFu / d + 1u};
}
__device__ __forceinline__ uint32_t fdiv(uint32_t n, FastDiv f) { return f.d <= 1 ? n : __umulhi(n, f.m); }

// ------------------------------------------- programmatic dependent launch --
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_prior() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// --------------------------------------------------------------------- mma --
// D(16x8 f32) += A(16x16 bf16, row) * B(16x8 bf16, col), register operands.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D(16x8 f32) = A(16x16 f16, row) * B(16x8 f16, col) (+ 0: the accumulator
// input is the zero register, so no accumulator needs clearing).
__device__ __forceinline__ void mma_f16_16816_zero(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                   uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}
// D(16x8 f32) += A(16x16 f16, row) * B(16x8 f16, col).
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// D(16x8 f32) (+)= A(16x8 bf16, row) * B(8x8 bf16, col); ZERO: accumulator input 0.
template <bool ZERO>
__device__ __forceinline__ void mma_bf16_1688(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  if (ZERO)
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(b0), "f"(0.f));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(b0));
}

// f32 -> f16 bits, round to nearest even.
__device__ __forceinline__ uint32_t f32_to_f16_rn(float f) { return __half_as_ushort(__float2half_rn(f)); }
__device__ __forceinline__ float f16_to_f32(uint32_t bits16) { return __half2float(__ushort_as_half((unsigned short)bits16)); }

// 2^s as f32 for |s| <= 126.
__device__ __forceinline__ float pow2f(int s) { return __uint_as_float((uint32_t)(s + 127) << 23); }

// Two 4-bit codes at bits [j*4, j*4+4) and [16+j*4, 16+j*4+4) -> bf16x2 {128+lo, 128+hi}.
template <int J>
__device__ __forceinline__ uint32_t codes_to_bf16x2(uint32_t w) {
  return ((w >> (4 * J)) & 0x000F000Fu) | 0x43004300u;
}

// {lo16, hi16} bf16 pair -> f32 values.
__device__ __forceinline__ float bf16_lo_f32(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi_f32(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// --------------------------------------------------------------- GLU acts --
// SiLU-GLU with the overflow-free sigmoid (kernels/moe/reference.py:160-170).
__device__ __forceinline__ float act_swiglu(float g, float u) {
  const float e = expf(-fabsf(g));
  const float sig = g >= 0.f ? 1.f / (1.f + e) : e / (1.f + e);
  return (g * sig) * u;
}

// SiTU-GLU: gb*tanh(g/gb)*sigmoid(g) * vb*tanh(v/vb) (host/backend.py:47-62).
__device__ __forceinline__ float act_situ(float g, float v, float gb, float vb) {
  const float sig = 1.f / (1.f + expf(-g));
  const float t1 = (gb * tanhf(g / gb)) * sig;
  const float t2 = vb * tanhf(v / vb);
  return t1 * t2;
}

}  // namespace rc
