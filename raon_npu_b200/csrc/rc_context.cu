// Context lifetime, error reporting and scratch management of the C ABI.
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>

#include "rc_internal.cuh"

namespace rc {

static thread_local char g_err[1024] = "no error";

void set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

cudaStream_t pick_stream(rc_ctx *ctx, void *stream) {
  return stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
}

// Scratch for one GEMV call over K columns and n_tiles row tiles.  Grows only;
// growth waits for the whole device (launches may sit on caller streams),
// allocates and zeroes counters, so it must not happen inside stream capture --
// warm a context up with its largest shapes first.  All launches that share a
// context's scratch must be ordered on one stream at a time.
int ensure_gemv_scratch(rc_ctx *ctx, int k, int n_tiles) {
  if ((size_t)k > ctx->xfrag_k) {
    size_t kk = (size_t)k;
    uint32_t *xf = nullptr;
    float *gs = nullptr;
    RC_CUDA_TRY(cudaDeviceSynchronize());
    RC_CUDA_TRY(cudaMalloc(&xf, kXSlots * xfrag_slot_words(kk) * sizeof(uint32_t)));
    RC_CUDA_TRY(cudaMalloc(&gs, kXSlots * gsum_slot_floats(kk) * sizeof(float)));
    if (ctx->xfrag) cudaFree(ctx->xfrag);
    if (ctx->gsum) cudaFree(ctx->gsum);
    ctx->xfrag = xf;
    ctx->gsum = gs;
    ctx->xfrag_k = kk;
  }
  if ((size_t)n_tiles > ctx->counters_cap) {
    size_t cap = (size_t)n_tiles;
    int *c = nullptr;
    RC_CUDA_TRY(cudaDeviceSynchronize());
    RC_CUDA_TRY(cudaMalloc(&c, cap * sizeof(int)));
    RC_CUDA_TRY(cudaMemset(c, 0, cap * sizeof(int)));
    if (ctx->counters) cudaFree(ctx->counters);
    ctx->counters = c;
    ctx->counters_cap = cap;
  }
  return RC_OK;
}

static int grow_pinned(void **p, size_t *cap, size_t need) {
  if (need <= *cap) return RC_OK;
  if (*p) cudaFreeHost(*p);
  *p = nullptr;
  *cap = 0;
  RC_CUDA_TRY(cudaMallocHost(p, need));
  *cap = need;
  return RC_OK;
}

static int grow_device(void **p, size_t *cap, size_t need) {
  if (need <= *cap) return RC_OK;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  RC_CUDA_TRY(cudaMalloc(p, need));
  *cap = need;
  return RC_OK;
}

// The status of an error word read back from the device (cleared when set).
int report_error_word(rc_ctx *ctx, int word) {
  if (word) {
    RC_CUDA_TRY(cudaMemset(ctx->err, 0, sizeof(int)));
    if (word == 2) {
      set_error("sampler: more than 2048 tokens tie at the top-k threshold (device error word 2)");
      return RC_ERR_INVALID;
    }
    if (word == 4) {
      set_error("MoE: an expert id outside 0..n_experts-1 reached the device (device error word 4)");
      return RC_ERR_INVALID;
    }
    if (word == 3) {
      set_error("sampler: the logits have no orderable value (NaN) (device error word 3)");
      return RC_ERR_INVALID;
    }
    ++ctx->timeout_epoch;
    set_error("a kernel gave up a bounded wait (device error word %d)", word);
    return RC_ERR_TIMEOUT;
  }
  return RC_OK;
}

// Report (and clear) the error word a kernel leaves when a bounded wait gives up.
int check_error_word(rc_ctx *ctx) {
  int word = 0;
  RC_CUDA_TRY(cudaMemcpy(&word, ctx->err, sizeof(int), cudaMemcpyDeviceToHost));
  return report_error_word(ctx, word);
}

int ensure_sample_scratch(rc_ctx *ctx, size_t bytes) {
  return grow_device(&ctx->sample_bits, &ctx->sample_bits_cap, bytes);
}

int ensure_host_staging(rc_ctx *ctx, size_t xb, size_t yb) {
  int rc;
  if ((rc = grow_pinned(&ctx->pin_x, &ctx->pin_x_cap, xb))) return rc;
  if ((rc = grow_pinned(&ctx->pin_y, &ctx->pin_y_cap, yb))) return rc;
  if (!ctx->pin_err) RC_CUDA_TRY(cudaMallocHost(reinterpret_cast<void **>(&ctx->pin_err), sizeof(int)));
  if ((rc = grow_device(&ctx->dev_x, &ctx->dev_x_cap, xb))) return rc;
  if ((rc = grow_device(&ctx->dev_y, &ctx->dev_y_cap, yb))) return rc;
  return RC_OK;
}

}  // namespace rc

using namespace rc;

extern "C" {

const char *rc_last_error(void) { return rc::g_err; }

int rc_abi_version(void) { return 1; }

int rc_init(int device, rc_ctx **out) {
  RC_CHECK_ARG(out != nullptr, "rc_init: out is NULL");
  *out = nullptr;
  int ndev = 0;
  RC_CUDA_TRY(cudaGetDeviceCount(&ndev));
  RC_CHECK_ARG(device >= 0 && device < ndev, "rc_init: device %d out of range (%d devices)", device, ndev);
  RC_CUDA_TRY(cudaSetDevice(device));
  int major = 0, minor = 0;
  RC_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
  RC_CUDA_TRY(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
  if (major != 10 || minor != 0) {
    set_error("rc_init: device %d is sm_%d%d; this library is built for sm_100a (B200) only", device,
              major, minor);
    return RC_ERR_CUDA;
  }
  rc_ctx *ctx = static_cast<rc_ctx *>(calloc(1, sizeof(rc_ctx)));
  if (!ctx) {
    set_error("rc_init: out of host memory");
    return RC_ERR_CUDA;
  }
  ctx->device = device;
  cudaError_t e = cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&ctx->err, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(ctx->err, 0, sizeof(int));
  if (e == cudaSuccess) e = cudaMalloc(&ctx->qflag, sizeof(int));
  if (e == cudaSuccess) {
    size_t warps = (size_t)ctx->sm_count * kGemvMaxWarps;   // stream-K partials: one slot pair per warp
    e = cudaMalloc(&ctx->partials, warps * 2 * 2 * 32 * 4 * sizeof(float));
  }
  if (e != cudaSuccess) {
    set_error("rc_init: %s", cudaGetErrorString(e));
    rc_destroy(ctx);
    return RC_ERR_CUDA;
  }
  *out = ctx;
  return RC_OK;
}

int rc_destroy(rc_ctx *ctx) {
  if (!ctx) return RC_OK;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  cudaFree(ctx->xfrag);
  cudaFree(ctx->gsum);
  cudaFree(ctx->partials);
  cudaFree(ctx->bf_partials);
  cudaFree(ctx->counters);
  cudaFree(ctx->err);
  cudaFree(ctx->qflag);
  cudaFree(ctx->dev_x);
  cudaFree(ctx->dev_y);
  cudaFree(ctx->sample_bits);
  if (ctx->pin_x) cudaFreeHost(ctx->pin_x);
  if (ctx->pin_y) cudaFreeHost(ctx->pin_y);
  if (ctx->pin_err) cudaFreeHost(ctx->pin_err);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  free(ctx);
  return RC_OK;
}

int rc_stream(rc_ctx *ctx, void **stream_out) {
  RC_CHECK_ARG(ctx && stream_out, "rc_stream: NULL argument");
  *stream_out = ctx->stream;
  return RC_OK;
}

int rc_sm_count(rc_ctx *ctx, int *out) {
  RC_CHECK_ARG(ctx && out, "rc_sm_count: NULL argument");
  *out = ctx->sm_count;
  return RC_OK;
}

int rc_sync(rc_ctx *ctx) {
  RC_CHECK_ARG(ctx, "rc_sync: NULL context");
  RC_CUDA_TRY(cudaSetDevice(ctx->device));
  // Device-wide: launches may have gone to caller streams as well as ctx->stream.
  RC_CUDA_TRY(cudaDeviceSynchronize());
  return check_error_word(ctx);
}

}  // extern "C"
