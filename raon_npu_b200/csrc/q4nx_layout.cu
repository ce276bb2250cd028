// Weight upload: the reference's pack_gemv bytes are repacked once, on the
// device, into the t16 tile layout the GEMV streams (layout described in
// rc_internal.cuh); plus the bit-exact dequantiser used to prove the repack.
#include "rc_device.cuh"
#include "rc_internal.cuh"

namespace rc {

struct RefLayout {
  const uint8_t *src;  // pack_gemv bytes (quant/q4nx.py:335-393, rows=4)
  int kb;              // K / 256
};

// Unit row r (0..15) of row tile ``tile`` -> logical matrix row.  For a
// [gate; up] matrix (``inter`` > 0) a tile holds gate rows 8*tile..+7 in unit
// rows 0..7 and the matching up rows in unit rows 8..15.
__device__ __forceinline__ int unit_row_to_matrix_row(int tile, int r, int inter) {
  if (inter == 0) return tile * kUnitRows + r;
  return r < 8 ? tile * 8 + r : inter + tile * 8 + (r - 8);
}

// Byte of the pack_gemv block holding (row n, k-block kbi) and the position of
// the 4-bit code of column kk (0..255) inside it (quant/q4nx.py:378-390).
__device__ __forceinline__ uint32_t ref_code(const RefLayout &L, int n, int kbi, int kk) {
  const int slice = n >> 7, rowblk = (n >> 5) & 3, r32 = n & 31;
  const size_t blk = ((size_t)slice * L.kb + kbi) * 4 + rowblk;
  const int h = r32 >> 4, rr = r32 & 15;
  const uint8_t b = L.src[blk * kRefBlockBytes + kRefParamBytes + (size_t)(h * kUnitK + kk) * 8 + (rr >> 1)];
  return (rr & 1) ? (b >> 4) : (b & 15u);
}

__device__ __forceinline__ uint32_t ref_scale_min(const RefLayout &L, int n, int kbi, int grp) {
  const int slice = n >> 7, rowblk = (n >> 5) & 3, r32 = n & 31;
  const size_t blk = ((size_t)slice * L.kb + kbi) * 4 + rowblk;
  const uint8_t *p = L.src + blk * kRefBlockBytes;
  const uint16_t s = *reinterpret_cast<const uint16_t *>(p + (grp * 32 + r32) * 2);
  const uint16_t m = *reinterpret_cast<const uint16_t *>(p + 512 + (grp * 32 + r32) * 2);
  return (uint32_t)s | ((uint32_t)m << 16);
}

// One thread per 32-bit word of the t16 layout (640 words per unit).
__global__ void rc_repack_kernel(RefLayout L, uint32_t *dst, long long units, int inter) {
  const long long words = units * (kUnitBytes / 4);
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < words;
       idx += (long long)gridDim.x * blockDim.x) {
    const long long unit = idx / (kUnitBytes / 4);
    const int wi = (int)(idx - unit * (kUnitBytes / 4));
    const int tile = (int)(unit / L.kb), kbi = (int)(unit - (long long)tile * L.kb);
    uint32_t word = 0;
    if (wi < kUnitCodeBytes / 4) {
      const int s4 = wi >> 7, lane = (wi >> 2) & 31, sub = wi & 3;
      const int s = s4 * 4 + sub, g = lane >> 2, q = lane & 3;
      const int n_lo = unit_row_to_matrix_row(tile, g, inter);
      const int n_hi = unit_row_to_matrix_row(tile, g + 8, inter);
      const int c0 = s * 16 + 2 * q;
      // nibble slot j (0..3) -> {row, column offset}: j0 (g, +0) j1 (g+8, +0) j2 (g, +8) j3 (g+8, +8);
      // the low half-word holds column c, the high half-word column c+1.
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = (j & 1) ? n_hi : n_lo;
        const int c = c0 + ((j & 2) ? 8 : 0);
        word |= ref_code(L, n, kbi, c) << (4 * j);
        word |= ref_code(L, n, kbi, c + 1) << (16 + 4 * j);
      }
    } else {
      const int j = wi - kUnitCodeBytes / 4;  // 0..127
      const int pair = j >> 1, upper = j & 1;
      const int g = pair >> 3, grp = pair & 7;
      const int n = unit_row_to_matrix_row(tile, g + (upper ? 8 : 0), inter);
      word = ref_scale_min(L, n, kbi, grp);
    }
    dst[idx] = word;
  }
}

// f32(f64(min) + f64(scale) * code), written in logical row order.
__global__ void rc_dequant_kernel(const uint32_t *tiles, float *out, int n_rows, int k, int inter) {
  const int kb = k / kUnitK;
  const long long total = (long long)n_rows * k;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(idx / k), col = (int)(idx - (long long)n * k);
    int tile, r;
    if (inter == 0) {
      tile = n / kUnitRows;
      r = n % kUnitRows;
    } else if (n < inter) {
      tile = n / 8;
      r = n % 8;
    } else {
      tile = (n - inter) / 8;
      r = 8 + (n - inter) % 8;
    }
    const int kbi = col / kUnitK, kk = col % kUnitK;
    const int s = kk / 16, c16 = kk % 16, grp = kk / 32;
    const int g = r & 7, rowhi = r >> 3;
    const int q = (c16 & 7) >> 1, odd = c16 & 1, upper8 = c16 >> 3;
    const int lane = g * 4 + q;
    const uint32_t *unit = tiles + ((size_t)tile * kb + kbi) * (kUnitBytes / 4);
    const uint32_t word = unit[((s >> 2) * 32 + lane) * 4 + (s & 3)];
    const int shift = upper8 * 8 + rowhi * 4 + odd * 16;
    const uint32_t code = (word >> shift) & 15u;
    const uint32_t sm = unit[kUnitCodeBytes / 4 + (g * 8 + grp) * 2 + rowhi];
    const double scale = (double)bf16_to_f32(sm & 0xFFFFu);
    const double mn = (double)bf16_to_f32(sm >> 16);
    out[idx] = __double2float_rn(__dadd_rn(mn, __dmul_rn(scale, (double)code)));
  }
}

// ------------------------------------------------------------- quantiser --
// bf16 directed rounding of an f32 value (quant/q4nx.py:57-106 on f32 input).
__device__ __forceinline__ float bf16_floor_f32(float f) {
  const uint32_t u = __float_as_uint(f);
  const uint32_t step = ((u >> 31) && (u & 0xFFFFu)) ? 1u : 0u;
  return __uint_as_float(((u >> 16) + step) << 16);
}
__device__ __forceinline__ float bf16_ceil_f32(float f) {
  const uint32_t u = __float_as_uint(f);
  const uint32_t step = (!(u >> 31) && (u & 0xFFFFu)) ? 1u : 0u;
  return __uint_as_float(((u >> 16) + step) << 16);
}
// f64 -> nearest f32 not below x, then bf16 ceiling (the f64 branch of bf16_ceil).
__device__ __forceinline__ float bf16_ceil_f64(double x) {
  float f = __double2float_rn(x);
  if ((double)f < x) f = nextafterf(f, INFINITY);
  return bf16_ceil_f32(f);
}
// Next bf16 toward +inf of an exact bf16 value, -0 treated as +0 (quant/q4nx.py:109-124).
__device__ __forceinline__ float bf16_next_up(float f) {
  uint32_t t = __float_as_uint(f) >> 16;
  if (t == 0x8000u) t = 0;
  uint32_t nxt;
  if (t == 0) nxt = 1;
  else if (t & 0x8000u) nxt = (t == 0x8001u) ? 0 : t - 1;
  else nxt = t + 1;
  return __uint_as_float(nxt << 16);
}

// One thread per (row pair, 32-column group): the two rows share the code
// bytes of pack_gemv (even row = low nibble).  Mirrors quant/q4nx.py:127-200
// with every f64 step an explicitly rounded IEEE operation, so codes, scales
// and mins are bit-identical to the reference's numpy quantiser.
__global__ void rc_quantize_pack_kernel(const float *w, int n, int k, uint8_t *out, int *flag) {
  const int groups = k / 32, kb = k / kUnitK;
  const long long work = (long long)(n / 2) * groups;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < work;
       idx += (long long)gridDim.x * blockDim.x) {
    const int pair = (int)(idx / groups), grp = (int)(idx - (long long)pair * groups);
    uint32_t codes[2][32];
    for (int h = 0; h < 2; ++h) {
      const int row = 2 * pair + h;
      const float *src = w + (size_t)row * k + grp * 32;
      float lo = src[0], hi = src[0];
      bool finite = true;
      for (int c = 0; c < 32; ++c) {
        const float v = src[c];
        finite = finite && isfinite(v);
        lo = fminf(lo, v);
        hi = fmaxf(hi, v);
      }
      if (!finite) {
        atomicOr(flag, 1);
        lo = hi = 0.f;
      }
      const float min_q = bf16_floor_f32(lo);
      const double base = (double)min_q, top = (double)hi;
      const double span = __dsub_rn(top, base);
      float scale = bf16_ceil_f64(__ddiv_rn(span, 15.0));
      for (int it = 0; it < 64 && isfinite(scale); ++it) {
        if (__dadd_rn(base, __dmul_rn(15.0, (double)scale)) >= top) break;
        scale = bf16_next_up(scale);
      }
      const bool flat = span == 0.0;
      if (flat) scale = 0.f;
      if (!isfinite(scale) || !isfinite(min_q)) atomicOr(flag, 2);
      const double div = flat ? 1.0 : (double)scale;
      for (int c = 0; c < 32; ++c) {
        double qv = rint(__ddiv_rn(__dsub_rn((double)src[c], base), div));
        qv = qv < 0.0 ? 0.0 : (qv > 15.0 ? 15.0 : qv);
        codes[h][c] = flat ? 0u : (uint32_t)qv;
      }
      // scale / min bf16 at [g][r] in the block header (quant/q4nx.py:372-382).
      const int slice = row >> 7, rowblk = (row >> 5) & 3, r32 = row & 31;
      const int kbi = grp >> 3, gi = grp & 7;
      uint8_t *blk = out + (((size_t)slice * kb + kbi) * 4 + rowblk) * kRefBlockBytes;
      reinterpret_cast<uint16_t *>(blk)[gi * 32 + r32] = (uint16_t)(__float_as_uint(scale) >> 16);
      reinterpret_cast<uint16_t *>(blk + 512)[gi * 32 + r32] = (uint16_t)(__float_as_uint(min_q) >> 16);
    }
    const int row = 2 * pair;
    const int slice = row >> 7, rowblk = (row >> 5) & 3, r32 = row & 31;
    const int h = r32 >> 4, rr = r32 & 15;
    const int kbi = grp >> 3, gi = grp & 7;
    uint8_t *blk = out + (((size_t)slice * kb + kbi) * 4 + rowblk) * kRefBlockBytes + kRefParamBytes;
    for (int c = 0; c < 32; ++c) {
      const int kk = gi * 32 + c;
      blk[(size_t)(h * kUnitK + kk) * 8 + (rr >> 1)] = (uint8_t)(codes[0][c] | (codes[1][c] << 4));
    }
  }
}

static int grid_for(long long work, int threads, int sm_count) {
  long long g = (work + threads - 1) / threads;
  long long cap = (long long)sm_count * 16;
  return (int)(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace rc

using namespace rc;

extern "C" {

int rc_upload_q4nx(rc_ctx *ctx, const uint8_t *packed, size_t nbytes, int n, int k, unsigned flags,
                   rc_weight **out) {
  RC_CHECK_ARG(ctx && packed && out, "rc_upload_q4nx: NULL argument");
  *out = nullptr;
  RC_CHECK_ARG(n > 0 && n % 128 == 0, "M (%d) must be a multiple of 128 (rows=4 * M_TILE=32)", n);
  RC_CHECK_ARG(k > 0 && k % 256 == 0, "K (%d) must be a multiple of K_TILE (256)", k);
  const size_t need = (size_t)n * k * 5 / 8;
  RC_CHECK_ARG(nbytes == need, "packed buffer is %zu bytes, expected %zu for %dx%d", nbytes, need, n, k);
  RC_CHECK_ARG((flags & ~(unsigned)(RC_UPLOAD_SRC_DEVICE | RC_UPLOAD_GATE_UP)) == 0, "unknown upload flags 0x%x",
               flags);
  RC_CUDA_TRY(cudaSetDevice(ctx->device));
  const int inter = (flags & RC_UPLOAD_GATE_UP) ? n / 2 : 0;

  rc_weight *w = new rc_weight();
  w->ctx = ctx;
  w->n = n;
  w->k = k;
  w->flags = flags;
  w->bytes = need;
  const uint8_t *src = packed;
  uint8_t *tmp = nullptr;
  cudaError_t e = cudaMalloc(&w->tiles, need);
  if (e == cudaSuccess && !(flags & RC_UPLOAD_SRC_DEVICE)) {
    e = cudaMalloc(&tmp, need);
    if (e == cudaSuccess) e = cudaMemcpyAsync(tmp, packed, need, cudaMemcpyHostToDevice, ctx->stream);
    src = tmp;
  }
  if (e == cudaSuccess) {
    RefLayout L{src, k / kUnitK};
    const long long units = (long long)(n / kUnitRows) * (k / kUnitK);
    const long long words = units * (kUnitBytes / 4);
    rc_repack_kernel<<<grid_for(words, 256, ctx->sm_count), 256, 0, ctx->stream>>>(
        L, reinterpret_cast<uint32_t *>(w->tiles), units, inter);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (tmp) cudaFree(tmp);
  if (e != cudaSuccess) {
    set_error("rc_upload_q4nx: %s", cudaGetErrorString(e));
    if (w->tiles) cudaFree(w->tiles);
    delete w;
    return RC_ERR_CUDA;
  }
  *out = w;
  return RC_OK;
}

int rc_quantize_q4nx(rc_ctx *ctx, const float *w_dev, int n, int k, uint8_t *packed_dev, void *stream) {
  RC_CHECK_ARG(ctx && w_dev && packed_dev, "rc_quantize_q4nx: NULL argument");
  RC_CHECK_ARG(n > 0 && n % 128 == 0, "M (%d) must be a multiple of 128 (rows=4 * M_TILE=32)", n);
  RC_CHECK_ARG(k > 0 && k % 256 == 0, "K (%d) must be a multiple of K_TILE (256)", k);
  RC_CUDA_TRY(cudaSetDevice(ctx->device));
  const cudaStream_t s = pick_stream(ctx, stream);
  RC_CUDA_TRY(cudaMemsetAsync(ctx->qflag, 0, sizeof(int), s));
  const long long work = (long long)(n / 2) * (k / 32);
  rc_quantize_pack_kernel<<<grid_for(work, 128, ctx->sm_count), 128, 0, s>>>(w_dev, n, k, packed_dev, ctx->qflag);
  RC_CUDA_TRY(cudaGetLastError());
  int flag = 0;
  RC_CUDA_TRY(cudaMemcpyAsync(&flag, ctx->qflag, sizeof(int), cudaMemcpyDeviceToHost, s));
  RC_CUDA_TRY(cudaStreamSynchronize(s));
  RC_CHECK_ARG(!(flag & 1), "Input weight matrix contains non-finite values (NaN or Inf)");
  RC_CHECK_ARG(!(flag & 2), "Quantization parameters (scale_q or min_q) overflowed to non-finite values");
  return RC_OK;
}

int rc_weight_free(rc_weight *w) {
  if (!w) return RC_OK;
  cudaSetDevice(w->ctx->device);
  cudaStreamSynchronize(w->ctx->stream);
  cudaFree(w->tiles);
  if (w->bias) cudaFree(w->bias);
  delete w;
  return RC_OK;
}

int rc_weight_set_bias(rc_weight *w, const float *bias_host) {
  if (!w) {
    set_error("rc_weight_set_bias: unknown weight handle");
    return RC_ERR_NOT_FOUND;
  }
  RC_CHECK_ARG(bias_host != nullptr, "rc_weight_set_bias: NULL bias");
  RC_CUDA_TRY(cudaSetDevice(w->ctx->device));
  if (!w->bias) RC_CUDA_TRY(cudaMalloc(&w->bias, (size_t)w->n * sizeof(float)));
  RC_CUDA_TRY(cudaMemcpyAsync(w->bias, bias_host, (size_t)w->n * sizeof(float), cudaMemcpyHostToDevice,
                              w->ctx->stream));
  RC_CUDA_TRY(cudaStreamSynchronize(w->ctx->stream));
  return RC_OK;
}

int rc_weight_bias(const rc_weight *w, const float **bias_dev) {
  if (!w) {
    set_error("rc_weight_bias: unknown weight handle");
    return RC_ERR_NOT_FOUND;
  }
  RC_CHECK_ARG(bias_dev != nullptr, "rc_weight_bias: NULL out");
  *bias_dev = w->bias;
  return RC_OK;
}

int rc_weight_info(const rc_weight *w, int *n, int *k, size_t *device_bytes, unsigned *flags) {
  if (!w) {
    set_error("rc_weight_info: unknown weight handle");
    return RC_ERR_NOT_FOUND;
  }
  if (n) *n = w->n;
  if (k) *k = w->k;
  if (device_bytes) *device_bytes = w->bytes;
  if (flags) *flags = w->flags;
  return RC_OK;
}

int rc_dequant_q4nx(rc_ctx *ctx, const rc_weight *w, float *out_dev, void *stream) {
  RC_CHECK_ARG(!w || w->format == kFormatQ4nx, "rc_dequant_q4nx: not a q4nx matrix");
  RC_CHECK_ARG(ctx && out_dev, "rc_dequant_q4nx: NULL argument");
  if (!w) {
    set_error("rc_dequant_q4nx: unknown weight handle");
    return RC_ERR_NOT_FOUND;
  }
  RC_CUDA_TRY(cudaSetDevice(ctx->device));
  const long long total = (long long)w->n * w->k;
  const int inter = (w->flags & RC_UPLOAD_GATE_UP) ? w->n / 2 : 0;
  rc_dequant_kernel<<<grid_for(total, 256, ctx->sm_count), 256, 0, pick_stream(ctx, stream)>>>(
      reinterpret_cast<const uint32_t *>(w->tiles), out_dev, w->n, w->k, inter);
  RC_CUDA_TRY(cudaGetLastError());
  return RC_OK;
}

}  // extern "C"
