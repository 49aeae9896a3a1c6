// Kernel (d): fused greedy / temperature / top-p sampler, one CTA per row.
//
// Restates Decoder._sample (src/helios/runtime/qwen3/decode.py:457-473) and its
// batched use (src/helios/runtime/engine.py:470-492) without a sort:
//   * temperature 0: argmax, first index among equal maxima;
//   * otherwise p_i ~ exp(l_i / T - max / T). With top_p < 1, token i survives when
//     the mass of the tokens ranked before it (descending probability, ties by
//     ascending index) is <= top_p (the reference's shifted cumsum rule, :467-469).
//     Probability is monotone in the bf16 logit, so the cut is found by a two-level
//     radix select over the logit's 16-bit order key (256 + 256 bins of mass),
//     then by rank within the tied key;
//   * the draw: kept tokens in ascending index order, the first whose running
//     mass exceeds u * kept_mass for the caller's uniform u in [0, 1).
// Six passes over the row, all L2-resident after the first.
#pragma once

#include <climits>

#include "hb_common.cuh"

namespace hb {

constexpr int kSampleThreads = 1024;

struct SampleParams {
  const __nv_bfloat16* logits;  // [rows, row_stride]
  int64_t row_stride;
  int32_t rows, vocab;
  const float* temperature;  // [rows]
  const float* top_p;        // [rows]
  const float* uniforms;     // [rows]
  int64_t* out;              // [rows]
};

// Order-preserving 16-bit key of a bf16 value (larger value -> larger key).
__device__ __forceinline__ uint32_t bf16_key(__nv_bfloat16 v) {
  const uint16_t b = __bfloat16_as_ushort(v);
  return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
}

template <typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, Op op, T* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = red[lane];  // 32 warps exactly
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  return v;
}

// Exclusive block scan of one double per thread; returns this thread's prefix.
__device__ __forceinline__ double block_exclusive_scan(double v, double* red, double* total) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  double x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double n = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += n;
  }
  if (lane == 31) red[warp] = x;
  __syncthreads();
  if (warp == 0) {
    double w = red[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    red[lane] = w;
  }
  __syncthreads();
  const double before = (warp ? red[warp - 1] : 0.0) + x - v;
  *total = red[31];
  __syncthreads();
  return before;
}

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(SampleParams p) {
  __shared__ float fred[32];
  __shared__ int ired[32];
  __shared__ double dred[32];
  __shared__ float hist[256];
  __shared__ uint32_t cut_key;
  __shared__ float cut_mass_above;
  __shared__ int cut_found;
  __shared__ int chosen;

  const int row = blockIdx.x, tid = threadIdx.x;
  const __nv_bfloat16* lg = p.logits + static_cast<int64_t>(row) * p.row_stride;
  const int V = p.vocab;

  // Pass 1: max and its first index.
  float mx = -INFINITY;
  int arg = INT_MAX;
  for (int i = tid; i < V; i += kSampleThreads) {
    const float v = __bfloat162float(lg[i]);
    if (v > mx) { mx = v; arg = i; }  // strided order: first hit per thread is its smallest index
  }
  const float gmax = block_reduce(mx, [](float a, float b) { return fmaxf(a, b); }, fred);
  if (mx != gmax) arg = INT_MAX;
  const int garg = block_reduce(arg, [](int a, int b) { return min(a, b); }, ired);
  const float T = p.temperature[row];
  if (!(T > 0.f)) {
    if (tid == 0) p.out[row] = garg;
    return;
  }
  const float m = __fdiv_rn(gmax, T);
  const float top_p = p.top_p[row];

  // Pass 2: partition function Z.
  float z = 0.f;
  for (int i = tid; i < V; i += kSampleThreads) z += expf(__fdiv_rn(__bfloat162float(lg[i]), T) - m);
  const float Z = block_reduce(z, [](float a, float b) { return a + b; }, fred);

  uint32_t key_star = 0;        // tokens with key > key_star are kept
  int n_tie_keep = 0;           // how many tokens with key == key_star are kept (lowest indices)
  bool keep_all = !(top_p < 1.f);
  if (!keep_all) {
    const float target = top_p * Z;
    // Level 1: mass per high byte of the key.
    for (int b = tid; b < 256; b += kSampleThreads) hist[b] = 0.f;
    __syncthreads();
    for (int i = tid; i < V; i += kSampleThreads) {
      const __nv_bfloat16 v = lg[i];
      atomicAdd(&hist[bf16_key(v) >> 8], expf(__fdiv_rn(__bfloat162float(v), T) - m));
    }
    __syncthreads();
    if (tid == 0) {
      float cum = 0.f;
      cut_found = 0;
      for (int b = 255; b >= 0; --b) {
        if (cum <= target && target < cum + hist[b]) {
          cut_key = static_cast<uint32_t>(b);
          cut_mass_above = cum;
          cut_found = 1;
          break;
        }
        cum += hist[b];
      }
    }
    __syncthreads();
    if (!cut_found) {
      keep_all = true;
    } else {
      const uint32_t hi = cut_key;
      // Level 2: mass per low byte within the selected high byte.
      __syncthreads();
      for (int b = tid; b < 256; b += kSampleThreads) hist[b] = 0.f;
      __syncthreads();
      for (int i = tid; i < V; i += kSampleThreads) {
        const __nv_bfloat16 v = lg[i];
        const uint32_t k = bf16_key(v);
        if ((k >> 8) == hi) atomicAdd(&hist[k & 255u], expf(__fdiv_rn(__bfloat162float(v), T) - m));
      }
      __syncthreads();
      if (tid == 0) {
        float cum = cut_mass_above;
        int found = 0;
        for (int b = 255; b >= 0; --b) {
          if (hist[b] > 0.f && cum <= target && target < cum + hist[b]) {
            cut_key = (hi << 8) | static_cast<uint32_t>(b);
            cut_mass_above = cum;
            found = 1;
            break;
          }
          cum += hist[b];
        }
        cut_found = found;
      }
      __syncthreads();
      if (!cut_found) {
        keep_all = true;
      } else {
        key_star = cut_key;
        // All tokens sharing key_star share one probability e_star.
        const uint16_t bits = (key_star & 0x8000u) ? static_cast<uint16_t>(key_star & 0x7FFFu)
                                                   : static_cast<uint16_t>(~key_star & 0xFFFFu);
        const float e_star = expf(__fdiv_rn(__bfloat162float(__ushort_as_bfloat16(bits)), T) - m);
        const float room = target - cut_mass_above;
        n_tie_keep = static_cast<int>(floorf(room / e_star)) + 1;
      }
    }
  }

  // Passes 5 + 6: contiguous chunks in index order; kept mass per chunk, scan, locate u * M.
  const int chunk = (V + kSampleThreads - 1) / kSampleThreads;
  const int c0 = min(V, tid * chunk), c1 = min(V, c0 + chunk);
  // Rank of this chunk's first tie among all ties (index order).
  int ties = 0;
  if (!keep_all)
    for (int i = c0; i < c1; ++i) ties += bf16_key(lg[i]) == key_star;
  double unused;
  const int tie_before = static_cast<int>(block_exclusive_scan(static_cast<double>(ties), dred, &unused));
  double kept_sum = 0.0;
  int last_kept = -1;
  {
    int rank = tie_before;
    for (int i = c0; i < c1; ++i) {
      const __nv_bfloat16 v = lg[i];
      bool kept = keep_all;
      if (!kept) {
        const uint32_t k = bf16_key(v);
        kept = k > key_star || (k == key_star && rank++ < n_tie_keep);
      }
      if (kept) {
        kept_sum += expf(__fdiv_rn(__bfloat162float(v), T) - m);
        last_kept = i;
      }
    }
  }
  double total;
  const double before = block_exclusive_scan(kept_sum, dred, &total);
  const int glast = block_reduce(last_kept, [](int a, int b) { return max(a, b); }, ired);
  const double target = static_cast<double>(p.uniforms[row]) * total;
  if (tid == 0) chosen = glast;
  __syncthreads();
  if (kept_sum > 0.0 && before <= target && target < before + kept_sum) {
    double run = before;
    int rank = tie_before;
    for (int i = c0; i < c1; ++i) {
      const __nv_bfloat16 v = lg[i];
      bool kept = keep_all;
      if (!kept) {
        const uint32_t k = bf16_key(v);
        kept = k > key_star || (k == key_star && rank++ < n_tie_keep);
      }
      if (kept) {
        run += expf(__fdiv_rn(__bfloat162float(v), T) - m);
        if (run > target) {
          atomicMin(&chosen, i);
          break;
        }
      }
    }
  }
  __syncthreads();
  if (tid == 0) p.out[row] = chosen;
}

}  // namespace hb

namespace hb {

// Speculative verification of drafted rows (the acceptance loop of Engine._execute_batch,
// src/helios/runtime/engine.py:507-520). A row whose logit rows are its trailing lc
// tokens has prediction i (the greedy id after token count - lc + i) compared with the
// row's next token; the drafts accepted are the longest matching prefix, and the row
// emits predictions 0 .. accepted. A row with one logit row emits its prediction.
struct VerifyParams {
  const int64_t* tokens;         // [T] the tick's token ids, rows packed by cu_seq_q
  const int32_t* cu_seq_q;       // [B+1]
  const int32_t* logit_offsets;  // [B+1] first logit row of each row
  const int64_t* predictions;    // [logit rows] one id per logit row
  int32_t rows;
  int32_t* accepted;             // [B]
  int64_t* emitted;              // [logit rows]: row r writes logit_offsets[r] .. + accepted[r]
};

constexpr int kVerifyThreads = 128;

__global__ void __launch_bounds__(kVerifyThreads) verify_drafts_kernel(VerifyParams p) {
  const int r = blockIdx.x * kVerifyThreads + threadIdx.x;
  if (r >= p.rows) return;
  const int q0 = p.cu_seq_q[r], count = p.cu_seq_q[r + 1] - q0;
  const int l0 = p.logit_offsets[r], lc = p.logit_offsets[r + 1] - l0;
  if (lc < 1 || lc > count) {  // logit rows must be trailing tokens of the row
    raise_status(kStatusBadRow);
    p.accepted[r] = 0;
    return;
  }
  const int first = q0 + count - lc;  // token whose prediction is logit row l0
  int accepted = 0;
  while (accepted < lc - 1 && p.tokens[first + accepted + 1] == p.predictions[l0 + accepted]) ++accepted;
  for (int i = 0; i <= accepted; ++i) p.emitted[l0 + i] = p.predictions[l0 + i];
  p.accepted[r] = accepted;
}

}  // namespace hb
