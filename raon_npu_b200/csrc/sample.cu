// Token sampler on the bf16 lm-head logits: the reference's
// ``sample_token`` (serve/engine.py:84-140) in f64, one CTA per token row.
//
//   scores = f64(logit) - presence_penalty for the tokens already seen
//   temperature <= 0   -> argmax (first index of the maximum)
//   top-k (1..1024)    -> keep scores >= the k-th largest (ties kept)
//   top-p (< 1)        -> descending stable order, softmax, drop a token when
//                         the probability before it already reaches top_p
//                         (the top token always stays)
//   temperature        -> scores / T, softmax, categorical draw with the
//                         caller's uniform u: first index (ascending token id)
//                         whose normalised cumulative probability exceeds u
//                         (numpy Generator.choice)
//
// Top-k without a sort of the vocabulary: the scores of unseen tokens are
// bf16 values, so two 8-bit radix passes over their 16-bit keys give the k-th
// largest unseen score theta; every token of the top k (with ties) scores
// >= theta, so the candidates are the unseen tokens >= theta plus the seen
// tokens whose penalised score is >= theta.  Candidates are sorted in shared
// memory (bitonic, descending score, ascending index) and the rest runs on
// that short list.
#include "rc_device.cuh"
#include "rc_internal.cuh"

namespace rc {

constexpr int kSampleThreads = 1024;
constexpr int kSampleMaxCand = 2048;
constexpr int kSampleMaxVocab = 1 << 20;
constexpr int kSampleMaxTopK = 1024;
constexpr int kErrSampleCandidates = 2;    // device error word: too many tied candidates
constexpr int kErrSampleNoCandidates = 3;  // device error word: no orderable score (NaN logits)

struct SampleParams {
  const uint16_t *logits;    // [T][ld] bf16
  int ld, V, top_k;
  double top_p, temperature, penalty;
  const int32_t *seen;       // concatenated seen-token lists
  const int32_t *seen_off;   // [T+1] offsets into seen (null: none)
  const double *u;           // [T] uniform draws in [0, 1)
  int32_t *out;              // [T]
  uint32_t *seen_bits;       // [T][ceil(V/32)] scratch bitmap
  int *err;
};

// bf16 bits -> order-preserving 16-bit key (larger value -> larger key)
__device__ __forceinline__ uint32_t bf16_key(uint32_t b) { return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u); }

__global__ void __launch_bounds__(kSampleThreads) rc_sample_kernel(SampleParams p) {
  __shared__ double c_score[kSampleMaxCand];
  __shared__ int c_idx[kSampleMaxCand];
  __shared__ unsigned hist[256];
  __shared__ int s_count, s_digit, s_rank, s_done;
  __shared__ double s_red[kSampleThreads / 32];
  __shared__ int s_redi[kSampleThreads / 32];
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint16_t *row = p.logits + (size_t)t * p.ld;
  const int V = p.V, nwords = (V + 31) / 32;
  uint32_t *bits = p.seen_bits + (size_t)t * nwords;
  // seen tokens -> bitmap (duplicates collapse, as np.unique does)
  for (int i = tid; i < nwords; i += blockDim.x) bits[i] = 0u;
  __syncthreads();
  if (p.seen_off && p.penalty != 0.0) {
    for (int i = p.seen_off[t] + tid; i < p.seen_off[t + 1]; i += blockDim.x) {
      const int s = p.seen[i];
      if (s >= 0 && s < V) atomicOr(bits + (s >> 5), 1u << (s & 31));
    }
  }
  __syncthreads();
  auto seen_tok = [&](int i) -> bool { return p.seen_off && p.penalty != 0.0 && ((__ldcg(bits + (i >> 5)) >> (i & 31)) & 1u); };
  auto score = [&](int i) -> double {
    const double v = (double)bf16_to_f32(row[i]);
    return seen_tok(i) ? v - p.penalty : v;
  };

  if (p.temperature <= 0.0) {
    // greedy: first index of the maximum
    double best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < V; i += blockDim.x) {
      const double v = score(i);
      if (v > best || (v == best && i < bi)) best = v, bi = i;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const double ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) best = ov, bi = oi;
    }
    if (lane == 0) s_red[warp] = best, s_redi[warp] = bi;
    __syncthreads();
    if (tid == 0) {
      double b = s_red[0];
      int ix = s_redi[0];
      for (int w = 1; w < kSampleThreads / 32; ++w)
        if (s_red[w] > b || (s_red[w] == b && s_redi[w] < ix)) b = s_red[w], ix = s_redi[w];
      p.out[t] = ix;
    }
    return;
  }

  // ---- theta: the k-th largest score among unseen tokens (16-bit radix select)
  const int k = p.top_k;
  uint32_t prefix = 0;
  int rank = k;                 // rank still to find within the current prefix
  bool have_theta = true;
  for (int pass = 0; pass < 2; ++pass) {
    for (int i = tid; i < 256; i += blockDim.x) hist[i] = 0u;
    __syncthreads();
    const int shift = 8 - 8 * pass;
    for (int i = tid; i < V; i += blockDim.x) {
      if (seen_tok(i)) continue;
      const uint32_t key = bf16_key(row[i]);
      if (pass == 1 && (key >> 8) != prefix) continue;
      atomicAdd(hist + ((key >> shift) & 0xFFu), 1u);
    }
    __syncthreads();
    if (tid == 0) {
      int r = rank, d = 255;
      for (; d >= 0; --d) {
        if ((int)hist[d] >= r) break;
        r -= (int)hist[d];
      }
      s_digit = d;          // -1: fewer than `rank` unseen tokens in range
      s_rank = r;
    }
    __syncthreads();
    if (s_digit < 0) {
      have_theta = false;
      break;
    }
    prefix = pass == 0 ? (uint32_t)s_digit : ((prefix << 8) | (uint32_t)s_digit);
    rank = s_rank;
    __syncthreads();
  }
  double theta = -INFINITY;
  if (have_theta) {
    const uint32_t key = prefix;                  // 16-bit key of theta
    const uint32_t b = (key & 0x8000u) ? (key & 0x7FFFu) : (~key & 0xFFFFu);
    theta = (double)bf16_to_f32(b);
  }
  // ---- candidates: every token scoring >= theta
  if (tid == 0) s_count = 0, s_done = 0;
  __syncthreads();
  for (int i = tid; i < V; i += blockDim.x) {
    const double v = score(i);
    if (v >= theta) {
      const int slot = atomicAdd(&s_count, 1);
      if (slot < kSampleMaxCand) c_score[slot] = v, c_idx[slot] = i;
    }
  }
  __syncthreads();
  const int n = s_count;
  // n == 0 only when the scores are not ordered (NaN logits): report it
  // instead of drawing from an empty list
  if (n > kSampleMaxCand || n == 0) {
    if (tid == 0) {
      atomicCAS(p.err, 0, n == 0 ? kErrSampleNoCandidates : kErrSampleCandidates);
      p.out[t] = -1;
    }
    return;
  }
  // ---- bitonic sort of the candidates: descending score, ascending index
  int np2 = 1;
  while (np2 < n) np2 <<= 1;
  for (int i = n + tid; i < np2; i += blockDim.x) c_score[i] = -INFINITY, c_idx[i] = 0x7fffffff;
  __syncthreads();
  for (int size = 2; size <= np2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < np2; i += blockDim.x) {
        const int j = i ^ stride;
        if (j > i) {
          const bool up = (i & size) == 0;      // this half sorts "before" order
          const double a = c_score[i], b = c_score[j];
          const int ia = c_idx[i], ib = c_idx[j];
          const bool a_first = a > b || (a == b && ia < ib);
          if (a_first != up) {
            c_score[i] = b, c_score[j] = a;
            c_idx[i] = ib, c_idx[j] = ia;
          }
        }
      }
      __syncthreads();
    }
  }
  if (tid != 0) return;
  // ---- top-k, top-p, temperature, draw (short list, one thread)
  int keep = n;
  if (k > 0 && k < V && k <= n) {
    const double kth = c_score[k - 1];
    keep = k;
    while (keep < n && c_score[keep] >= kth) ++keep;
  }
  if (p.top_p >= 0.0 && p.top_p < 1.0) {
    const double m = c_score[0];
    double denom = 0.0;
    for (int i = 0; i < keep; ++i) denom += exp(c_score[i] - m);
    double cum = 0.0;
    int keep2 = keep;
    for (int i = 0; i < keep; ++i) {
      const double pr = exp(c_score[i] - m) / denom;
      cum += pr;
      if (i > 0 && cum - pr >= p.top_p) {
        keep2 = i;
        break;
      }
    }
    // tokens after the first removed one are removed as well (cum - pr only grows)
    keep = keep2;
  }
  // final softmax over the kept tokens, then the cumulative distribution in
  // ascending token id
  const double inv_t = p.temperature != 1.0 ? p.temperature : 1.0;
  double m = -INFINITY;
  for (int i = 0; i < keep; ++i) {
    const double s = p.temperature != 1.0 ? c_score[i] / inv_t : c_score[i];
    c_score[i] = s;
    m = s > m ? s : m;
  }
  double denom = 0.0;
  for (int i = 0; i < keep; ++i) denom += exp(c_score[i] - m);
  // insertion sort of the kept list by token id
  for (int a = 1; a < keep; ++a) {
    const double sv = c_score[a];
    const int iv = c_idx[a];
    int b = a - 1;
    while (b >= 0 && c_idx[b] > iv) {
      c_score[b + 1] = c_score[b];
      c_idx[b + 1] = c_idx[b];
      --b;
    }
    c_score[b + 1] = sv;
    c_idx[b + 1] = iv;
  }
  double total = 0.0;
  for (int i = 0; i < keep; ++i) {
    c_score[i] = exp(c_score[i] - m) / denom;   // probability
    total += c_score[i];
    c_score[i] = total;                          // cumulative
  }
  const double u = p.u[t];
  if (keep < 1) keep = 1;   // the top token always stays (n >= 1 here)
  int tok = c_idx[keep - 1];
  for (int i = 0; i < keep; ++i) {
    if (c_score[i] / total > u) {
      tok = c_idx[i];
      break;
    }
  }
  p.out[t] = tok;
}

}  // namespace rc

using namespace rc;

extern "C" {

int rc_sample_tokens(rc_ctx *ctx, const uint16_t *logits_dev, int ld, int T, int V, int top_k, double top_p,
                     double temperature, double presence_penalty, const int32_t *seen_dev,
                     const int32_t *seen_off_dev, const double *u_dev, int32_t *out_dev, void *stream) {
  RC_CHECK_ARG(ctx && logits_dev && u_dev && out_dev, "rc_sample_tokens: NULL argument");
  RC_CHECK_ARG(T >= 1 && V >= 1 && V <= kSampleMaxVocab && ld >= V, "rc_sample_tokens: bad T/V/ld");
  RC_CHECK_ARG(temperature <= 0.0 || (top_k >= 1 && top_k <= kSampleMaxTopK && top_k < V),
               "rc_sample_tokens: sampling needs top_k in 1..%d (and < V); a full-vocabulary top-p is not "
               "supported on the device", kSampleMaxTopK);
  RC_CHECK_ARG(!(presence_penalty != 0.0) || !seen_dev == !seen_off_dev, "seen and seen_off go together");
  RC_CUDA_TRY(cudaSetDevice(ctx->device));
  const size_t bytes = (size_t)T * ((V + 31) / 32) * 4;
  int rc = ensure_sample_scratch(ctx, bytes);
  if (rc) return rc;
  SampleParams p{};
  p.logits = logits_dev;
  p.ld = ld;
  p.V = V;
  p.top_k = top_k;
  p.top_p = top_p;
  p.temperature = temperature;
  p.penalty = presence_penalty;
  p.seen = seen_dev;
  p.seen_off = seen_dev ? seen_off_dev : nullptr;
  p.u = u_dev;
  p.out = out_dev;
  p.seen_bits = static_cast<uint32_t *>(ctx->sample_bits);
  p.err = ctx->err;
  rc_sample_kernel<<<T, kSampleThreads, 0, pick_stream(ctx, stream)>>>(p);
  RC_CUDA_TRY(cudaGetLastError());
  return RC_OK;
}

}  // extern "C"
