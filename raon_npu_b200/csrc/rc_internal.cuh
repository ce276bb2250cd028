// Internal definitions shared by the raon_cuda translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string>

#include "../../include/raon_cuda.h"

namespace rc {

// ----------------------------------------------------------- tile layout --
// GPU tile layout of a q4nx matrix ("t16"): the matrix is cut into units of
// 16 output rows x 256 input columns, stored unit after unit in
// (row-tile, k-block) order, 2560 bytes each (= 16*256*5/8, the same bits per
// weight as the reference's pack_gemv blocks):
//   bytes [0, 2048):   4-bit codes in mma.sync A-fragment order.  For k16-step
//                      s (0..15) and lane l (g = l/4, q = l%4) the 32-bit word at
//                      byte ((s/4)*32 + l)*16 + (s%4)*4 holds
//                        bits  0..3 / 16..19: code[g  ][16s+2q] / [16s+2q+1]
//                        bits  4..7 / 20..23: code[g+8][16s+2q] / [16s+2q+1]
//                        bits  8..11/ 24..27: code[g  ][16s+2q+8] / [16s+2q+9]
//                        bits 12..15/ 28..31: code[g+8][16s+2q+8] / [16s+2q+9]
//                      so ((w >> 4j) & 0x000F000F) | 0x43004300 is A register j
//                      as bf16x2 (128 + code), one 16-byte load per lane per
//                      4 k16-steps, 512 contiguous bytes per warp load.
//   bytes [2048,2560): per (g = 0..7, group 0..7) 8 bytes at 2048 + (g*8+group)*8:
//                      bf16 {scale[g], min[g], scale[g+8], min[g+8]}.
constexpr int kUnitRows = 16;
constexpr int kUnitK = 256;
constexpr int kUnitBytes = 2560;
constexpr int kUnitCodeBytes = 2048;
constexpr int kGroupsPerUnit = 8;

// Reference pack_gemv block (quant/q4nx.py:335-393).
constexpr int kRefBlockRows = 32;
constexpr int kRefBlockBytes = 5120;
constexpr int kRefParamBytes = 1024;

// GEMV persistent kernel geometry.
constexpr int kGemvWarps = 8;         // warps per CTA for small matrices (each with a private ring)
constexpr int kGemvMaxWarps = 16;     // warps per CTA for large matrices (one CTA per SM)
constexpr int kGemvMaxStages = 12;    // ring depth (units in flight) per warp; chosen per launch
constexpr int kGemvSmemLimit = 227 * 1024;   // opt-in dynamic shared memory per CTA on sm_100
constexpr int kMaxTokensPerLaunch = 16;   // two 8-token mma column blocks
// Activation scratch rotates over this many slots: consecutive launches chained
// by programmatic dependent launch may be resident together, and a launch must
// never read a slot that a still-running neighbour has cached.
constexpr int kXSlots = 4;

// Device error words (ctx->err): first failure wins.
constexpr int kErrWaitTimeout = 1;
constexpr int kErrBadExpert = 4;       // an expert id outside 0..E-1 reached the device

void set_error(const char *fmt, ...);

#define RC_CUDA_TRY(expr)                                                              \
  do {                                                                                 \
    cudaError_t _e = (expr);                                                           \
    if (_e != cudaSuccess) {                                                           \
      ::rc::set_error("%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), __FILE__, \
                      __LINE__);                                                       \
      return RC_ERR_CUDA;                                                              \
    }                                                                                  \
  } while (0)

#define RC_CHECK_ARG(cond, ...)        \
  do {                                 \
    if (!(cond)) {                     \
      ::rc::set_error(__VA_ARGS__);    \
      return RC_ERR_INVALID;           \
    }                                  \
  } while (0)

}  // namespace rc

// weight formats
constexpr int kFormatQ4nx = 0;    // 4-bit codes with per-32-column scale/min (t16 units)
constexpr int kFormatBfp16 = 1;   // 9-bit bfp16ebs8 in the reference's GEMV packing

struct rc_weight {
  rc_ctx *ctx;
  int n, k;            // logical rows (N) and columns (K)
  unsigned flags;      // RC_UPLOAD_* flags it was uploaded with
  int format;          // kFormatQ4nx or kFormatBfp16
  uint8_t *tiles;      // q4nx: t16 layout, n/16 * k/256 units; bfp16: the reference's packed bytes
  size_t bytes;
  float *bias;         // optional f32 [n] on the device
};

struct rc_ctx {
  int device;
  int sm_count;
  cudaStream_t stream;
  // GEMV scratch: fragment-ordered x, group sums, split-K partials, tile counters.
  uint32_t *xfrag;      // kXSlots x [2 token blocks][K/64][32 lanes][8 words]
  size_t xfrag_k;       // K capacity of one xfrag / gsum slot
  float *gsum;          // kXSlots x aux words of 2 token blocks (group-sum fragments, block scales)
  unsigned launch_seq;  // picks the activation slot of the next launch
  float *partials;      // [warps][2][2 token blocks][32 lanes][4]
  float *bf_partials;   // bfp16 GEMV k-slice partials [slices][T][rows]
  size_t bf_partials_cap;
  int *counters;        // [tiles], all zero between launches
  size_t counters_cap;
  int *err;             // device error word
  unsigned timeout_epoch;   // bumped whenever a bounded device wait is found to have given up
  int *qflag;           // quantiser status word (non-finite input / overflow)
  // Host staging of the host-buffer entry points (rc_*_host).
  void *pin_x, *pin_y;
  int *pin_err;         // pinned copy of the error word
  size_t pin_x_cap, pin_y_cap;
  void *dev_x, *dev_y;
  size_t dev_x_cap, dev_y_cap;
  // Sampler scratch: seen-token bitmaps.
  void *sample_bits;
  size_t sample_bits_cap;
};

namespace rc {
int ensure_gemv_scratch(rc_ctx *ctx, int k, int n_tiles);
int ensure_host_staging(rc_ctx *ctx, size_t xb, size_t yb);
int ensure_sample_scratch(rc_ctx *ctx, size_t bytes);
int check_error_word(rc_ctx *ctx);
int report_error_word(rc_ctx *ctx, int word);
// Host staging of the host-buffer entry points (elementwise.cu): pinned host
// memory <-> device memory by kernels on stream s; the copy out also brings
// the error word back, then waits for s and reports it.
int host_copy_in(rc_ctx *ctx, void *dev, const void *pinned, size_t bytes, cudaStream_t s);
int host_copy_out_and_wait(rc_ctx *ctx, void *pinned, const void *dev, size_t bytes, cudaStream_t s);
// Grouped down projection of an MoE layer with bfp16ebs8 down matrices
// (bfp16_gemv.cu).  Decode: the group tables of the q4nx MoE kernels.
// Prefill (blk_row0 != null): 8-row blocks of the permuted rows, block b =
// expert group_expert[b], rows blk_row0[b] .. + blk_n[b] of x and of y.
struct BfMoeDown {
  const uint8_t *const *w;      // [E+1] device table of expert down matrices [hidden][inter_pad] (null: not here)
  const int *n_groups;          // device: groups (decode) or blocks (prefill)
  const int32_t *group_expert;  // [group]
  const uint32_t *group_mask;   // [group] tokens of the group
  const int32_t *group_dst;     // [group][dst_stride] slot row of (group, token)
  int dst_stride;
  const int32_t *blk_row0, *blk_n;  // prefill blocks (null: decode groups)
  const uint16_t *x;            // activation of (group g, token t): row g * rows_per_group + t, stride ldx
  int ldx, rows_per_group, T;
  int hidden, inter_pad;
  uint16_t *y;                  // slot rows, stride ldy
  int ldy;
  int max_groups;               // upper bound of *n_groups (grid size only)
  int *err;
};
int bfp16_moe_down(rc_ctx *ctx, const BfMoeDown &d, cudaStream_t s);
int bfp16_gemv(rc_ctx *ctx, const rc_weight *w, const uint16_t *x, int ldx, int T, void *y, int y_dtype, int ldy,
               int row0, int nrows, const float *bias, cudaStream_t s);   // bfp16_gemv.cu
// Words of one xfrag slot / floats of one aux slot for K columns (2 token blocks).
inline size_t xfrag_slot_words(size_t k) { return 2 * k * 4; }
inline size_t gsum_slot_floats(size_t k) { return 17 * k / 16; }
cudaStream_t pick_stream(rc_ctx *ctx, void *stream);
}  // namespace rc
