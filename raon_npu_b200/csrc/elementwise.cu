// Elementwise glue of a decode step: the residual add of the hidden stream,
// plain or followed by an RMS normalisation; the staging copies of the
// host-buffer entry points.
#include "rc_device.cuh"
#include "rc_internal.cuh"

namespace rc {

// ------------------------------------------------------- host staging --
// The host-buffer entry points move their inputs and results between pinned
// host memory (mapped into the device's address space) and device memory with
// this kernel rather than with copy-engine transfers: chained to its
// neighbours by programmatic dependent launch it starts within about a
// microsecond of its predecessor, where a copy-engine transfer of a few KB
// costs several.  The copy out also carries the context's error word.
constexpr int kStageThreads = 256;

__global__ void __launch_bounds__(kStageThreads) rc_stage_copy_kernel(const uint8_t *src, uint8_t *dst, size_t bytes,
                                                                   const int *err_src, int *err_dst) {
  pdl_launch_dependents();
  pdl_wait_prior();
  const size_t n16 = bytes / 16, stride = (size_t)gridDim.x * blockDim.x;
  const size_t i0 = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (size_t i = i0; i < n16; i += stride)
    reinterpret_cast<uint4 *>(dst)[i] = reinterpret_cast<const uint4 *>(src)[i];
  for (size_t i = n16 * 16 + i0; i < bytes; i += stride) dst[i] = src[i];
  if (err_dst && i0 == 0) *err_dst = *reinterpret_cast<const volatile int *>(err_src);
}

static int stage_copy(rc_ctx *ctx, void *dst, const void *src, size_t bytes, bool with_err, cudaStream_t s) {
  if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) != 0) {
    set_error("host staging: buffers must be 16-byte aligned");
    return RC_ERR_INVALID;
  }
  long long blocks = (long long)((bytes / 16 + kStageThreads - 1) / kStageThreads);
  if (blocks < 1) blocks = 1;
  if (blocks > 4ll * ctx->sm_count) blocks = 4ll * ctx->sm_count;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(kStageThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  RC_CUDA_TRY(cudaLaunchKernelEx(&cfg, rc_stage_copy_kernel, static_cast<const uint8_t *>(src),
                                 static_cast<uint8_t *>(dst), bytes, with_err ? ctx->err : nullptr,
                                 with_err ? ctx->pin_err : nullptr));
  return RC_OK;
}

int host_copy_in(rc_ctx *ctx, void *dev, const void *pinned, size_t bytes, cudaStream_t s) {
  return stage_copy(ctx, dev, pinned, bytes, false, s);
}

int host_copy_out_and_wait(rc_ctx *ctx, void *pinned, const void *dev, size_t bytes, cudaStream_t s) {
  int rc = stage_copy(ctx, pinned, dev, bytes, true, s);
  if (rc) return rc;
  RC_CUDA_TRY(cudaStreamSynchronize(s));
  return report_error_word(ctx, *ctx->pin_err);
}

// out = RTNE(f32(a) + f32(b)), 8 bf16 per thread.
__global__ void rc_add_bf16_kernel(const uint16_t *a, const uint16_t *b, uint16_t *out, long long n) {
  pdl_launch_dependents();
  pdl_wait_prior();
  const long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (i + 8 <= n) {
    const uint4 va = *reinterpret_cast<const uint4 *>(a + i), vb = *reinterpret_cast<const uint4 *>(b + i);
    const uint32_t xa[4] = {va.x, va.y, va.z, va.w}, xb[4] = {vb.x, vb.y, vb.z, vb.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t lo = f32_to_bf16_rne(bf16_to_f32(xa[j] & 0xFFFFu) + bf16_to_f32(xb[j] & 0xFFFFu));
      const uint32_t hi = f32_to_bf16_rne(bf16_to_f32(xa[j] >> 16) + bf16_to_f32(xb[j] >> 16));
      o[j] = lo | (hi << 16);
    }
    *reinterpret_cast<uint4 *>(out + i) = make_uint4(o[0], o[1], o[2], o[3]);
  } else {
    for (long long j = i; j < n; ++j) out[j] = f32_to_bf16_rne(bf16_to_f32(a[j]) + bf16_to_f32(b[j]));
  }
}

// out[r] = RTNE(s / sqrt(mean(s^2) + eps)), s = f32(a[r]) + f32(b[r]): the
// residual add followed by an RMS normalisation without a learned scale, one
// CTA per row.
constexpr int kRmsThreads = 256;

__global__ void __launch_bounds__(kRmsThreads) rc_add_rms_bf16_kernel(const uint16_t *a, const uint16_t *b, uint16_t *out,
                                                                   int n, float eps) {
  pdl_launch_dependents();
  pdl_wait_prior();
  __shared__ float part[kRmsThreads / 32];
  const size_t base = (size_t)blockIdx.x * n;
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = bf16_to_f32(a[base + i]) + bf16_to_f32(b[base + i]);
    ss = fmaf(v, v, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kRmsThreads / 32; ++w) tot += part[w];
  const float scale = rsqrtf(tot / (float)n + eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = bf16_to_f32(a[base + i]) + bf16_to_f32(b[base + i]);
    out[base + i] = f32_to_bf16_rne(v * scale);
  }
}

}  // namespace rc

using namespace rc;

extern "C" int rc_add_rms_bf16(rc_ctx *ctx, const uint16_t *a_dev, const uint16_t *b_dev, uint16_t *out_dev, int rows,
                               int n, float eps, void *stream) {
  RC_CHECK_ARG(ctx && a_dev && b_dev && out_dev && rows >= 1 && n >= 1, "rc_add_rms_bf16: bad argument");
  RC_CUDA_TRY(cudaSetDevice(ctx->device));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows);
  cfg.blockDim = dim3(kRmsThreads);
  cfg.stream = pick_stream(ctx, stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  RC_CUDA_TRY(cudaLaunchKernelEx(&cfg, rc_add_rms_bf16_kernel, a_dev, b_dev, out_dev, n, eps));
  return RC_OK;
}

extern "C" int rc_add_bf16(rc_ctx *ctx, const uint16_t *a_dev, const uint16_t *b_dev, uint16_t *out_dev, long long n,
                           void *stream) {
  RC_CHECK_ARG(ctx && a_dev && b_dev && out_dev && n >= 0, "rc_add_bf16: bad argument");
  RC_CHECK_ARG(((reinterpret_cast<uintptr_t>(a_dev) | reinterpret_cast<uintptr_t>(b_dev) |
                 reinterpret_cast<uintptr_t>(out_dev)) & 15) == 0,
               "rc_add_bf16: buffers must be 16-byte aligned");
  if (n == 0) return RC_OK;
  RC_CUDA_TRY(cudaSetDevice(ctx->device));
  cudaLaunchConfig_t cfg = {};
  const long long threads = (n + 7) / 8;
  cfg.gridDim = dim3((unsigned)((threads + 255) / 256));
  cfg.blockDim = dim3(256);
  cfg.stream = pick_stream(ctx, stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  RC_CUDA_TRY(cudaLaunchKernelEx(&cfg, rc_add_bf16_kernel, a_dev, b_dev, out_dev, n));
  return RC_OK;
}
