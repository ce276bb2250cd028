// GEMV over 9-bit bfp16ebs8 weights (the reference's second weight format:
// quant/bfp16.py, kernels/gemv_bfp16/).  y[t][r] = bf16_rne(sum_k w[r][k] *
// x[t][k] (+ bias[r])), w[r][k] = m * 2**(max(e, 7) - 133) for the int8
// mantissa m and the exponent byte e its 8-column group shares
// (kernels/gemv_bfp16/reference.py:118-182).
//
// Layout: the reference's GEMV packing is kept byte for byte in HBM.  A
// 9216-byte block holds 32 rows x 256 columns as two halves of 16 rows; a half
// is 32 groups of [16 exponent bytes (one per row), 8 columns x 16 rows of
// mantissas, column-major]: 4608 contiguous bytes, the unit this kernel
// streams (one bulk copy each).  Blocks run ((slice * k_blocks + k) * 4 +
// block row) with 4 block rows (128 output rows) per slice.
//
// Work: (16-row tile, k-slice) items, dealt to the warps of a persistent grid
// (one CTA of 16 warps per SM), each warp streaming its items' units through a
// ring of bulk copies.  A lane takes 4 rows (row quad j) of 4 groups (group
// octet): per group it turns the 32 mantissas into f32 exactly (a byte
// permute onto 2**23, then one packed subtraction per two), sums each row's 8
// products with the token's activations in packed f32x2 lanes (columns 2c
// and 2c + 1; the products of an 8-bit mantissa and a bf16 value are exact),
// and adds the sum times the group's power-of-two scale (exact) into the
// row's accumulator.  The 8 lanes of a row quad are summed
// at the item's end.  With one k-slice the epilogue writes y; with several,
// f32 partials go to scratch and a finalize pass sums them in slice order, so
// the result does not depend on timing.
#include <string.h>

#include "rc_device.cuh"
#include "rc_internal.cuh"

namespace rc {

constexpr int kBfRows = 16;                         // rows of a unit (half block)
constexpr int kBfUnitBytes = 4608;                  // 32 groups x (16 + 128) bytes
constexpr int kBfGroupBytes = 144;
constexpr int kBfBlockBytes = 9216;
constexpr int kBfWarps = 16, kBfThreads = kBfWarps * 32, kBfStages = 3;
constexpr int kBfMaxTokens = 8;                     // tokens per launch
constexpr size_t kBfSmem = (size_t)kBfWarps * kBfStages * kBfUnitBytes + (size_t)kBfWarps * kBfStages * 8;

struct BfParams {
  const uint8_t *w;       // packed blocks of the whole matrix
  int tile0, n_tiles;     // first 16-row tile of the range, tiles in it
  int kb, slices, kps;    // k-blocks, k-slices per tile, k-blocks per slice
  const uint16_t *x;      // bf16 [T][ldx]
  int ldx, tokens;
  void *y;                // bf16 or f32 [T][ldy]
  int ldy;
  const float *bias;      // f32 per row of the range, or null
  float *partials;        // [slices][T][n_tiles * 16] when slices > 1
  int *err;
};

// Address of unit (16-row tile t, k-block kb) in the reference packing.
__device__ __forceinline__ const uint8_t *bf_unit(const uint8_t *w, int t, int kb, int KB) {
  const int br = t >> 1, half = t & 1, slice = br >> 2, r = br & 3;
  return w + ((size_t)((size_t)slice * KB + kb) * 4 + r) * kBfBlockBytes + half * kBfUnitBytes;
}

// Byte b of a word whose bytes were XOR'd with 0x80, as the f32 2**23 +
// (m + 128) (bits 0x4B0000bb); subtracting 2**23 + 128 leaves the int8
// mantissa m exactly.
__device__ __forceinline__ float bf_byte_bits(uint32_t biased, int b) {
  return __uint_as_float(__byte_perm(biased, 0x4B000000u, 0x7440u | (uint32_t)b));
}

// One unit (16 rows x 256 columns) into the accumulators of a lane: rows
// 4j..4j+3, groups go*4..go*4+3 of the unit, columns col0 + 8g.. of the
// activation rows tk with bit tk set in tmask (tk < TB).
template <int TB>
__device__ __forceinline__ void bf_unit_mac(const uint8_t *U, int j, int go, const uint16_t *x, int ldx, int col0,
                                            uint32_t tmask, float (&acc)[4][TB]) {
#pragma unroll 1
  for (int i = 0; i < 4; ++i) {
    const int g = go * 4 + i;                       // group of this unit (8 columns)
    const uint8_t *G = U + g * kBfGroupBytes;
    const uint32_t ew = *reinterpret_cast<const uint32_t *>(G + 4 * j);   // exponents of rows 4j..4j+3
    // mantissas of rows 4j..4j+3 as f32 pairs of adjacent columns (2cp, 2cp+1)
    float2 mf[4][4];
#pragma unroll
    for (int cp = 0; cp < 4; ++cp) {
      const uint32_t m0 = *reinterpret_cast<const uint32_t *>(G + 16 + 32 * cp + 4 * j) ^ 0x80808080u;
      const uint32_t m1 = *reinterpret_cast<const uint32_t *>(G + 32 + 32 * cp + 4 * j) ^ 0x80808080u;
#pragma unroll
      for (int r = 0; r < 4; ++r)
        mf[r][cp] = __fadd2_rn(make_float2(bf_byte_bits(m0, r), bf_byte_bits(m1, r)),
                               make_float2(-8388736.0f, -8388736.0f));   // 2**23 + 128
    }
    float sc[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      int e = (int)((ew >> (8 * r)) & 0xFFu);
      e = e < 7 ? 7 : e;                            // the reference kernel's clamp
      sc[r] = __uint_as_float((uint32_t)(e - 6) << 23);   // 2**(e - 133)
    }
    const int col = col0 + g * 8;
#pragma unroll
    for (int tk = 0; tk < TB; ++tk) {
      if ((tmask >> tk) & 1u) {
        const uint4 xv = __ldg(reinterpret_cast<const uint4 *>(x + (size_t)tk * ldx + col));
        const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
        float2 xf[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) xf[q] = make_float2(bf16_lo_f32(xw[q]), bf16_hi_f32(xw[q]));
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          float2 s2 = __fmul2_rn(mf[r][0], xf[0]);
#pragma unroll
          for (int cp = 1; cp < 4; ++cp) s2 = __ffma2_rn(mf[r][cp], xf[cp], s2);
          acc[r][tk] = fmaf(sc[r], s2.x + s2.y, acc[r][tk]);
        }
      }
    }
  }
}

template <int TB, bool F32OUT>
__global__ void __launch_bounds__(kBfThreads, 1) rc_bfp16_gemv_kernel(BfParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = lane & 3, go = lane >> 2;           // row quad, group octet
  uint8_t *ring = smem + warp * kBfStages * kBfUnitBytes;
  const uint32_t ring_s = smem_addr(ring);
  const uint32_t bar0 = smem_addr(smem + (size_t)kBfWarps * kBfStages * kBfUnitBytes) + warp * kBfStages * 8;
  const int W = gridDim.x * kBfWarps, w0 = blockIdx.x * kBfWarps + warp;
  const int items = p.n_tiles * p.slices;
  // the warp's unit sequence: items w0, w0 + W, ...; k-blocks of each item's slice
  auto item_kb = [&](int item, int &t, int &kb0, int &kb1) {
    t = item / p.slices;
    const int s = item - t * p.slices;
    kb0 = s * p.kps;
    kb1 = kb0 + p.kps < p.kb ? kb0 + p.kps : p.kb;
  };
  int iss_item = w0, iss_kb = 0, iss_t = 0, iss_kb1 = 0, issued = 0;
  if (iss_item < items) item_kb(iss_item, iss_t, iss_kb, iss_kb1);
  auto issue = [&](int sl) {
    mbar_arrive_expect_tx(bar0 + 8 * sl, kBfUnitBytes);
    bulk_copy_g2s_plain(ring_s + sl * kBfUnitBytes, bf_unit(p.w, p.tile0 + iss_t, iss_kb, p.kb), kBfUnitBytes,
                        bar0 + 8 * sl);
    ++issued;
    if (++iss_kb == iss_kb1) {
      iss_item += W;
      if (iss_item < items) item_kb(iss_item, iss_t, iss_kb, iss_kb1);
    }
  };
  if (lane == 0) {
    for (int sl = 0; sl < kBfStages; ++sl) mbar_init(bar0 + 8 * sl, 1);
    mbar_fence_init();
    for (int sl = 0; sl < kBfStages && iss_item < items; ++sl) issue(sl);
  }
  __syncwarp();
  int slot = 0, consumed = 0;
  uint32_t parity = 0;
  bool failed = false;
  for (int item = w0; item < items && !failed; item += W) {
    int t, kb0, kb1;
    item_kb(item, t, kb0, kb1);
    float acc[4][TB];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int tk = 0; tk < TB; ++tk) acc[r][tk] = 0.f;
    for (int kb = kb0; kb < kb1; ++kb) {
      if (!mbar_wait_bounded_warp(bar0 + 8 * slot, parity)) {
        if (lane == 0) atomicCAS(p.err, 0, kErrWaitTimeout);
        failed = true;
        break;
      }
      ++consumed;
      bf_unit_mac<TB>(ring + slot * kBfUnitBytes, j, go, p.x, p.ldx, kb * 256, (1u << p.tokens) - 1u, acc);
      __syncwarp();
      if (lane == 0 && iss_item < items) issue(slot);
      if (++slot == kBfStages) slot = 0, parity ^= 1u;
    }
    if (failed) break;
    // the 8 lanes of a row quad hold the sums of different groups
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int tk = 0; tk < TB; ++tk) {
        float v = acc[r][tk];
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        acc[r][tk] = v;
      }
    if (go == 0) {
      const int s = item - t * p.slices;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int row = t * kBfRows + 4 * j + r;    // within the range
#pragma unroll
        for (int tk = 0; tk < TB; ++tk) {
          if (tk >= p.tokens) continue;
          float v = acc[r][tk];
          if (p.slices > 1) {
            p.partials[((size_t)s * p.tokens + tk) * (p.n_tiles * kBfRows) + row] = v;
            continue;
          }
          if (p.bias) v += p.bias[row];
          if (F32OUT)
            static_cast<float *>(p.y)[(size_t)tk * p.ldy + row] = v;
          else
            static_cast<uint16_t *>(p.y)[(size_t)tk * p.ldy + row] = f32_to_bf16_rne(v);
        }
      }
    }
  }
  // after a failure, the copies still in flight land before the shared memory is released
  if (failed && lane == 0) {
    for (int q = consumed; q < issued; ++q)
      mbar_wait_bounded(bar0 + 8 * (q % kBfStages), (uint32_t)(q / kBfStages) & 1u);
  }
}

// Sum of the k-slices' partials in slice order, bias, output.
template <bool F32OUT>
__global__ void rc_bfp16_finalize_kernel(BfParams p) {
  const int rows = p.n_tiles * kBfRows;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * p.tokens) return;
  const int tk = i / rows, row = i - tk * rows;
  float v = 0.f;
  for (int s = 0; s < p.slices; ++s) v += p.partials[((size_t)s * p.tokens + tk) * rows + row];
  if (p.bias) v += p.bias[row];
  if (F32OUT)
    static_cast<float *>(p.y)[(size_t)tk * p.ldy + row] = v;
  else
    static_cast<uint16_t *>(p.y)[(size_t)tk * p.ldy + row] = f32_to_bf16_rne(v);
}

template <int TB, bool F32OUT>
static cudaError_t bf_launch(const rc_ctx *ctx, const BfParams &p, int grid, cudaStream_t s) {
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(rc_bfp16_gemv_kernel<TB, F32OUT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kBfSmem);
    if (e != cudaSuccess) return e;
    if (dev < 64) configured[dev] = true;
  }
  rc_bfp16_gemv_kernel<TB, F32OUT><<<grid, kBfThreads, kBfSmem, s>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess || p.slices == 1) return e;
  const int n = p.n_tiles * kBfRows * p.tokens;
  rc_bfp16_finalize_kernel<F32OUT><<<(n + 255) / 256, 256, 0, s>>>(p);
  return cudaGetLastError();
}

template <bool F32OUT>
static cudaError_t bf_dispatch(const rc_ctx *ctx, const BfParams &p, int grid, cudaStream_t s) {
  if (p.tokens <= 1) return bf_launch<1, F32OUT>(ctx, p, grid, s);
  if (p.tokens <= 2) return bf_launch<2, F32OUT>(ctx, p, grid, s);
  if (p.tokens <= 4) return bf_launch<4, F32OUT>(ctx, p, grid, s);
  return bf_launch<8, F32OUT>(ctx, p, grid, s);
}

// rows [row0, row0 + nrows) of a bfp16ebs8 matrix times T bf16 rows of x.
int bfp16_gemv(rc_ctx *ctx, const rc_weight *w, const uint16_t *x, int ldx, int T, void *y, int y_dtype, int ldy,
               int row0, int nrows, const float *bias, cudaStream_t s) {
  const int KB = w->k / 256, n_tiles = nrows / kBfRows;
  const int grid = ctx->sm_count;
  const long long warps = (long long)grid * kBfWarps;
  int slices = (int)((warps + n_tiles - 1) / n_tiles);
  if (slices > KB) slices = KB;
  if (slices < 1) slices = 1;
  const int kps = (KB + slices - 1) / slices;
  slices = (KB + kps - 1) / kps;                    // no empty slice
  for (int t0 = 0; t0 < T; t0 += kBfMaxTokens) {
    const int tc = T - t0 < kBfMaxTokens ? T - t0 : kBfMaxTokens;
    BfParams p{};
    p.w = w->tiles;
    p.tile0 = row0 / kBfRows;
    p.n_tiles = n_tiles;
    p.kb = KB;
    p.slices = slices;
    p.kps = kps;
    p.x = x + (size_t)t0 * ldx;
    p.ldx = ldx;
    p.tokens = tc;
    const size_t ye = y_dtype == RC_DTYPE_F32 ? 4 : 2;
    p.y = static_cast<uint8_t *>(y) + (size_t)t0 * ldy * ye;
    p.ldy = ldy;
    p.bias = bias;
    p.err = ctx->err;
    if (slices > 1) {
      const size_t need = (size_t)slices * tc * nrows * sizeof(float);
      if (need > ctx->bf_partials_cap) {
        RC_CUDA_TRY(cudaStreamSynchronize(s));
        cudaFree(ctx->bf_partials);
        ctx->bf_partials = nullptr;
        ctx->bf_partials_cap = 0;
        RC_CUDA_TRY(cudaMalloc(&ctx->bf_partials, need));
        ctx->bf_partials_cap = need;
      }
      p.partials = ctx->bf_partials;
    }
    const cudaError_t e = y_dtype == RC_DTYPE_F32 ? bf_dispatch<true>(ctx, p, grid, s)
                                                  : bf_dispatch<false>(ctx, p, grid, s);
    if (e != cudaSuccess) {
      set_error("bfp16 gemv launch: %s", cudaGetErrorString(e));
      return RC_ERR_CUDA;
    }
  }
  return RC_OK;
}

// Down projection of an MoE layer whose experts' down matrices are
// bfp16ebs8 (the reference's moe_b2 bundles, npu/backend.py:640-652): the
// groups of the slot table (expert, token mask, slot row per token) times
// their activation rows.  Items are (group, 16-row tile); a warp streams an
// item's k-blocks through its ring like the dense kernel and writes the
// group's tokens' rows of the tile as bf16 (zeros for an expert not loaded
// here, as the q4nx down kernel does).  Each output is one warp's f32 sum in
// k-block order, so a slot row does not depend on the grouping or the grid.
template <int TB, bool BLOCKS>
__global__ void __launch_bounds__(kBfThreads, 1) rc_bfp16_moe_down_kernel(BfMoeDown p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int j = lane & 3, go = lane >> 2;
  uint8_t *ring = smem + warp * kBfStages * kBfUnitBytes;
  const uint32_t ring_s = smem_addr(ring);
  const uint32_t bar0 = smem_addr(smem + (size_t)kBfWarps * kBfStages * kBfUnitBytes) + warp * kBfStages * 8;
  // Decode groups: items are dealt warp-major over the CTAs, so a grid larger
  // than items / 16 spreads a small item count over more SMs.  Prefill blocks:
  // CTA-major, so the tiles of one block (the same activation rows) share a
  // CTA's L1.
  const int W = gridDim.x * kBfWarps;
  const int w0 = BLOCKS ? blockIdx.x * kBfWarps + warp : warp * gridDim.x + blockIdx.x;
  const int tiles = p.hidden / kBfRows, KB = p.inter_pad / 256;
  const int items = *p.n_groups * tiles;
  auto weights = [&](int item) -> const uint8_t * {
    const int e = p.group_expert[item / tiles];
    return e >= 0 ? p.w[e] : nullptr;
  };
  int iss_item = w0, iss_kb = 0, issued = 0;
  auto issue = [&](int sl) {
    const uint8_t *w = weights(iss_item);
    if (w) {
      mbar_arrive_expect_tx(bar0 + 8 * sl, kBfUnitBytes);
      bulk_copy_g2s_plain(ring_s + sl * kBfUnitBytes, bf_unit(w, iss_item % tiles, iss_kb, KB), kBfUnitBytes,
                          bar0 + 8 * sl);
    } else {
      mbar_arrive_expect_tx(bar0 + 8 * sl, 0);      // nothing to fetch: the phase completes at once
    }
    ++issued;
    if (++iss_kb == KB) iss_kb = 0, iss_item += W;
  };
  if (lane == 0) {
    for (int sl = 0; sl < kBfStages; ++sl) mbar_init(bar0 + 8 * sl, 1);
    mbar_fence_init();
    for (int sl = 0; sl < kBfStages && iss_item < items; ++sl) issue(sl);
  }
  __syncwarp();
  int slot = 0, consumed = 0;
  uint32_t parity = 0;
  bool failed = false;
  for (int item = w0; item < items && !failed; item += W) {
    const int grp = item / tiles, t = item - grp * tiles;
    const bool live = weights(item) != nullptr;
    uint32_t mask;
    const uint16_t *xg;
    if (BLOCKS) {
      const int n = p.blk_n[grp];
      mask = n >= TB ? (TB >= 32 ? ~0u : (1u << TB) - 1u) : (1u << n) - 1u;
      xg = p.x + (size_t)p.blk_row0[grp] * p.ldx;
    } else {
      mask = p.group_mask[grp] & (p.T >= 32 ? ~0u : (1u << p.T) - 1u);
      xg = p.x + (size_t)grp * p.rows_per_group * p.ldx;
    }
    float acc[4][TB];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int tk = 0; tk < TB; ++tk) acc[r][tk] = 0.f;
    for (int kb = 0; kb < KB; ++kb) {
      if (!mbar_wait_bounded_warp(bar0 + 8 * slot, parity)) {
        if (lane == 0) atomicCAS(p.err, 0, kErrWaitTimeout);
        failed = true;
        break;
      }
      ++consumed;
      if (live) bf_unit_mac<TB>(ring + slot * kBfUnitBytes, j, go, xg, p.ldx, kb * 256, mask, acc);
      __syncwarp();
      if (lane == 0 && iss_item < items) issue(slot);
      if (++slot == kBfStages) slot = 0, parity ^= 1u;
    }
    if (failed) break;
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int tk = 0; tk < TB; ++tk) {
        float v = acc[r][tk];
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        acc[r][tk] = v;
      }
    if (go == 0) {
#pragma unroll
      for (int tk = 0; tk < TB; ++tk) {
        if (!((mask >> tk) & 1u)) continue;
        const size_t yrow = BLOCKS ? (size_t)p.blk_row0[grp] + tk : (size_t)p.group_dst[grp * p.dst_stride + tk];
        uint16_t *y = p.y + yrow * p.ldy + t * kBfRows + 4 * j;
#pragma unroll
        for (int r = 0; r < 4; ++r) y[r] = live ? f32_to_bf16_rne(acc[r][tk]) : (uint16_t)0;
      }
    }
  }
  if (failed && lane == 0) {
    for (int q = consumed; q < issued; ++q)
      mbar_wait_bounded(bar0 + 8 * (q % kBfStages), (uint32_t)(q / kBfStages) & 1u);
  }
}

template <int TB, bool BLOCKS = false>
static cudaError_t bf_moe_launch(const rc_ctx *ctx, const BfMoeDown &d, int grid, cudaStream_t s) {
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 64 || !configured[dev]) {
    e = cudaFuncSetAttribute(rc_bfp16_moe_down_kernel<TB, BLOCKS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kBfSmem);
    if (e != cudaSuccess) return e;
    if (dev < 64) configured[dev] = true;
  }
  rc_bfp16_moe_down_kernel<TB, BLOCKS><<<grid, kBfThreads, kBfSmem, s>>>(d);
  return cudaGetLastError();
}

int bfp16_moe_down(rc_ctx *ctx, const BfMoeDown &d, cudaStream_t s) {
  const bool blocks = d.blk_row0 != nullptr;
  RC_CHECK_ARG(blocks || (d.T >= 1 && d.T <= 16 && d.T <= d.rows_per_group && d.T <= d.dst_stride),
               "bfp16 MoE down: %d tokens outside 1..16", d.T);
  RC_CHECK_ARG(d.hidden % 128 == 0 && d.inter_pad % 256 == 0 && d.ldx % 8 == 0,
               "bfp16 MoE down: hidden %d / inter_pad %d not block-aligned", d.hidden, d.inter_pad);
  const long long items = (long long)d.max_groups * (d.hidden / kBfRows);
  if (items <= 0) return RC_OK;
  const long long want = (items + kBfWarps / 2 - 1) / (kBfWarps / 2);   // ~8 busy warps per SM for small counts
  const int grid = (int)(want < ctx->sm_count ? want : ctx->sm_count);
  cudaError_t e;
  if (blocks) e = bf_moe_launch<8, true>(ctx, d, grid, s);     // blocks of at most 8 rows
  else if (d.T <= 1) e = bf_moe_launch<1>(ctx, d, grid, s);
  else if (d.T <= 2) e = bf_moe_launch<2>(ctx, d, grid, s);
  else if (d.T <= 4) e = bf_moe_launch<4>(ctx, d, grid, s);
  else if (d.T <= 8) e = bf_moe_launch<8>(ctx, d, grid, s);
  else e = bf_moe_launch<16>(ctx, d, grid, s);
  if (e != cudaSuccess) {
    set_error("bfp16 MoE down launch: %s", cudaGetErrorString(e));
    return RC_ERR_CUDA;
  }
  return RC_OK;
}

}  // namespace rc

using namespace rc;

extern "C" {

int rc_upload_bfp16(rc_ctx *ctx, const uint8_t *packed, size_t nbytes, int n, int k, unsigned flags,
                    rc_weight **out) {
  RC_CHECK_ARG(ctx && packed && out, "rc_upload_bfp16: NULL argument");
  *out = nullptr;
  RC_CHECK_ARG(n > 0 && n % 128 == 0, "M (%d) must be a multiple of 128 (rows=4 * M_TILE=32)", n);
  RC_CHECK_ARG(k > 0 && k % 256 == 0, "K (%d) must be a multiple of K_TILE (256)", k);
  const size_t need = (size_t)n * k * 9 / 8;
  RC_CHECK_ARG(nbytes == need, "packed buffer is %zu bytes, expected %zu for %dx%d", nbytes, need, n, k);
  RC_CHECK_ARG((flags & ~(unsigned)RC_UPLOAD_SRC_DEVICE) == 0, "rc_upload_bfp16: unknown upload flags 0x%x", flags);
  RC_CUDA_TRY(cudaSetDevice(ctx->device));
  rc_weight *w = new rc_weight();
  w->ctx = ctx;
  w->n = n;
  w->k = k;
  w->flags = flags;
  w->format = kFormatBfp16;
  w->bytes = need;
  cudaError_t e = cudaMalloc(&w->tiles, need);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(w->tiles, packed, need,
                        (flags & RC_UPLOAD_SRC_DEVICE) ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                        ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) {
    set_error("rc_upload_bfp16: %s", cudaGetErrorString(e));
    if (w->tiles) cudaFree(w->tiles);
    delete w;
    return RC_ERR_CUDA;
  }
  *out = w;
  return RC_OK;
}

}  // extern "C"
