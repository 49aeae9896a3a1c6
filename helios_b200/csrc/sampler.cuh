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
// Layout: each of the 32 warps owns one contiguous segment of the row and reads it in
// 256-element steps, lane l taking elements 8l .. 8l + 7 of a step as one 16-byte load,
// so every pass is coalesced and index order is (warp, step, lane, element). The mass
// histograms are per warp (no cross-warp atomics on the few bins a peaked distribution
// fills), index-ordered counts and sums are warp scans plus one block scan over the warps,
// and the last pass walks only the warp whose segment holds the draw.
//
// A top-p row first takes the short path: after the max pass (packed bf16 maxima), one pass
// collects the candidates (tokens whose weight can matter: logit >= x_floor), testing each
// 16-byte group by its maximum first since few groups hold one, each warp staging its own run
// of the list with its count in a register. The cut is then a single mass histogram over the
// candidates' keys (by distance below their top key, fixed-point masses, so the sums are exact
// and order-free), and only the kept tokens are sorted, by index, for the draw. Rows with more
// candidates than the list holds, or whose cut keeps every candidate, take the whole-row passes.
#pragma once

#include <climits>

#include "hb_common.cuh"

namespace hb {

constexpr int kSampleThreads = 1024;
constexpr int kSampleWarps = kSampleThreads / 32;
constexpr int kSampleUnroll = 4;  // groups a lane loads before using any (loads in flight)
// Weights below 2^-40 of the row's largest (which is exactly 1) are left out of the mass
// histograms that locate the top-p cut: even all 2^17+ of them together stay below
// 2^-23 of the partition function, the rounding of its own fp32 sum, so the cut is the
// one the full sums give; the kept mass and the draw still sum every kept token.
constexpr float kNegligibleWeight = 9.094947e-13f;  // 2^-40
// Top-p rows: tokens whose weight can matter (logit >= x_floor, a superset of the weights
// above kNegligibleWeight) are collected in one pass; when at most this many, the cut and the
// draw run on that list in shared memory instead of over the whole row again.
constexpr int kSampleCand = 4096;

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
__device__ __forceinline__ uint32_t bf16_key_bits(uint32_t b) { return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u); }
__device__ __forceinline__ uint32_t bf16_key(__nv_bfloat16 v) { return bf16_key_bits(__bfloat16_as_ushort(v)); }

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

// Exclusive scan of one value per warp (read from lane 0's argument) over the 32 warps in
// order; every thread gets its warp's prefix and the total.
template <typename T>
__device__ __forceinline__ T warps_exclusive_scan(T v, T* red, T* total) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    T w = red[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const T n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    red[lane] = w;  // inclusive
  }
  __syncthreads();
  const T before = warp ? red[warp - 1] : T(0);
  *total = red[31];
  __syncthreads();
  return before;
}

// Inclusive scan over the lanes of a warp.
template <typename T>
__device__ __forceinline__ T warp_inclusive_scan(T v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

// The 8 logits of group g (elements 8g .. 8g + 7, n of them inside the row) as bf16 bits.
__device__ __forceinline__ int load_group(const __nv_bfloat16* lg, int g, int V, bool vec_ok, uint32_t (&b)[8]) {
  const int i0 = 8 * g;
  const int n = min(8, V - i0);
  if (vec_ok && n == 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(lg + i0);
    b[0] = v.x & 0xFFFFu; b[1] = v.x >> 16; b[2] = v.y & 0xFFFFu; b[3] = v.y >> 16;
    b[4] = v.z & 0xFFFFu; b[5] = v.z >> 16; b[6] = v.w & 0xFFFFu; b[7] = v.w >> 16;
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) b[e] = e < n ? __bfloat16_as_ushort(lg[i0 + e]) : 0u;
  }
  return n;
}

__device__ __forceinline__ float bits_to_float(uint32_t b) { return __uint_as_float(b << 16); }

// Groups base + 32u + lane (u < kSampleUnroll) of a warp segment ending at g_end, all loads
// issued before any is used; n[u] = 0 past the segment.
__device__ __forceinline__ void load_groups(const __nv_bfloat16* lg, int base, int g_end, int V, bool vec_ok,
                                            uint32_t (&b)[kSampleUnroll][8], int (&n)[kSampleUnroll]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int u = 0; u < kSampleUnroll; ++u) {
    const int g = base + 32 * u + lane;
    n[u] = g < g_end ? load_group(lg, g, V, vec_ok, b[u]) : 0;
  }
}

constexpr int kSampleRawUnroll = 8;  // raw groups a lane loads before using any (max pass)

// The 8 logits of group g as four packed bf16 pairs (-inf past the row end); returns how many
// are in the row.
__device__ __forceinline__ int load_raw(const __nv_bfloat16* lg, int g, int V, bool vec_ok, uint4& r) {
  const int i0 = 8 * g;
  const int n = min(8, V - i0);
  if (vec_ok && n == 8) {
    r = *reinterpret_cast<const uint4*>(lg + i0);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t lo = 2 * k < n ? __bfloat16_as_ushort(lg[i0 + 2 * k]) : 0xFF80u;
      const uint32_t hi = 2 * k + 1 < n ? __bfloat16_as_ushort(lg[i0 + 2 * k + 1]) : 0xFF80u;
      w[k] = lo | (hi << 16);
    }
    r = make_uint4(w[0], w[1], w[2], w[3]);
  }
  return n;
}

// Largest of a group's 8 logits (packed bf16 maxima, NaN-ignoring as fmaxf), as a float.
__device__ __forceinline__ float group_max(const uint4& r) {
  auto h = [](uint32_t w) { return *reinterpret_cast<const __nv_bfloat162*>(&w); };
  const __nv_bfloat162 m = __hmax2(__hmax2(h(r.x), h(r.y)), __hmax2(h(r.z), h(r.w)));
  return fmaxf(__low2float(m), __high2float(m));
}

// Logit bits of element e (0..7, known when compiled) of a raw group.
__device__ __forceinline__ uint32_t raw_bits(const uint4& r, int e) {
  const uint32_t w = e < 2 ? r.x : e < 4 ? r.y : e < 6 ? r.z : r.w;
  return (e & 1) ? (w >> 16) : (w & 0xFFFFu);
}

// Appends the tokens of group g (its bits b, n of them in the row) whose logit reaches x_floor to
// list[0 .. cap) as (index << 16 | bits), reserving their slots with one shared-memory atomic
// per warp; every lane of the warp calls it. Slots past cap are counted but not written.
__device__ __forceinline__ void append_candidates(const uint32_t (&b)[8], int n, int g, float x_floor, int* count,
                                                  unsigned long long* list, int cap) {
  const int lane = threadIdx.x & 31;
  uint32_t mine = 0;
#pragma unroll
  for (int e = 0; e < 8; ++e) mine |= (e < n && bits_to_float(b[e]) >= x_floor) ? (1u << e) : 0u;
  const int cnt = __popc(mine);
  const int incl = warp_inclusive_scan(cnt);
  const int total = __shfl_sync(0xffffffffu, incl, 31);
  if (total == 0) return;  // warp-uniform
  int slot0 = 0;
  if (lane == 31) slot0 = atomicAdd(count, total);
  int slot = __shfl_sync(0xffffffffu, slot0, 31) + incl - cnt;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    if ((mine >> e) & 1u) {
      if (slot < cap) list[slot] = (static_cast<unsigned long long>(8 * g + e) << 16) | b[e];
      ++slot;
    }
  }
}

// The 256 bins of `hist` in descending key order (bin 255 first), by one warp: the first bin
// k with cum <= target < cum + hist[k] (and hist[k] > 0 when `nonempty`), where cum is `base`
// plus the mass of the bins above k. Returns the bin (or -1) and its cum; also the total mass.
__device__ __forceinline__ int warp_find_cut(const double* hist, double base, double target, bool nonempty,
                                             double* cum_out, double* total_out) {
  const int lane = threadIdx.x & 31;
  double h[8], sum = 0.0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    h[i] = hist[255 - (8 * lane + i)];
    sum += h[i];
  }
  const double incl = warp_inclusive_scan(sum);
  double c = base + incl - sum;
  int found = -1;
  double found_cum = 0.0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (found < 0 && (!nonempty || h[i] > 0.0) && c <= target && target < c + h[i]) {
      found = 255 - (8 * lane + i);
      found_cum = c;
    }
    c += h[i];
  }
  *total_out = __shfl_sync(0xffffffffu, incl, 31);
  const unsigned hit = __ballot_sync(0xffffffffu, found >= 0);
  if (hit == 0u) return -1;
  const int src = __ffs(hit) - 1;  // the lane with the highest bins
  *cum_out = __shfl_sync(0xffffffffu, found_cum, src);
  return __shfl_sync(0xffffffffu, found, src);
}

// Exclusive prefix of one value per thread over the block in thread order; also the total.
template <typename T>
__device__ __forceinline__ T block_exclusive_scan(T v, T* red, T* total) {
  const T incl = warp_inclusive_scan(v);
  const T warp_total = __shfl_sync(0xffffffffu, incl, 31);
  const T before = warps_exclusive_scan(warp_total, red, total);
  return before + incl - v;
}

// Ascending bitonic sort of n (<= kSampleCand) entries in shared memory, padded to a power of
// two with entries that sort last; called by every thread of the block.
__device__ void block_sort(unsigned long long* a, int n) {
  int n2 = 2;
  while (n2 < n) n2 <<= 1;
  for (int i = n + static_cast<int>(threadIdx.x); i < n2; i += kSampleThreads) a[i] = ~0ull;
  __syncthreads();
  for (int k = 2; k <= n2; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n2; i += kSampleThreads) {
        const int x = i ^ j;
        if (x > i) {
          const unsigned long long u = a[i], v = a[x];
          if ((u > v) == ((i & k) == 0)) {
            a[i] = v;
            a[x] = u;
          }
        }
      }
      __syncthreads();
    }
}

__device__ __forceinline__ uint32_t key_to_bits(uint32_t key) {
  return (key & 0x8000u) ? (key & 0x7FFFu) : (~key & 0xFFFFu);
}

// Masses of candidate tokens in fixed point: a weight in (kNegligibleWeight, 1] times 2^50,
// rounded to an integer (negligible weights count 0). Sums of at most kSampleCand of them stay
// below 2^62 and are exact, so every mass below is independent of the order it was summed in.
constexpr double kMassScale = 1125899906842624.0;  // 2^50
__device__ __forceinline__ unsigned long long mass_q(float w) {
  return w > kNegligibleWeight ? __double2ull_rn(static_cast<double>(w) * kMassScale) : 0ull;
}

// Shared memory the candidate path needs besides the candidate list (which, once read into
// registers, holds first the mass histogram and then the kept tokens).
struct CandidateScratch {
  unsigned long long ull_red[32];
  uint32_t u32_red[32];
  int n_kept, n_ties, cut_d, far;
  unsigned long long cut_cum;
};
constexpr int kCandBins = kSampleCand;  // key distances below the row's top key the histogram covers

// The cut and the draw of a top-p row from its candidate list (every token whose weight can
// matter; see kSampleCand), with the rules of the whole-row passes: only weights above
// kNegligibleWeight count toward the masses; in descending probability order (ties by
// ascending index) a token is kept when the mass before it is at most top_p * Z (the first
// always); the kept tokens are visited in index order and the first whose running mass exceeds
// u * kept mass is drawn (the last kept one when rounding leaves none). The cut comes from one
// mass histogram over the order key, binned by distance below the candidates' top key (tokens
// at one bf16 value share a bin, so few tokens meet in a bin's atomics) and scanned top down;
// tokens tied at the cut key are kept lowest index first. Only the kept tokens are sorted (by
// index) for the draw. Every thread of the block calls it. Returns false, with nothing written,
// when the cut keeps every candidate (tokens outside the list may then be kept too) or the
// candidates span more than kCandBins keys: the whole-row passes decide those rows.
// `cand` holds the list on entry and the kept tokens (index << 16 | bits) afterwards.
__device__ bool sample_candidates(const SampleParams& p, int row, int nc, unsigned long long* cand, float top_p,
                                  float T, float m, CandidateScratch& sc, int* chosen) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int R = kSampleCand / kSampleThreads;  // candidates (and histogram bins) per thread
  auto weight = [&](uint32_t bits) { return expf(__fdiv_rn(bits_to_float(bits), T) - m); };

  unsigned long long c[R], q[R];
  uint32_t key[R];
  uint32_t kmax = 0;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = tid + r * kSampleThreads;
    c[r] = i < nc ? cand[i] : 0ull;
    key[r] = i < nc ? bf16_key_bits(static_cast<uint32_t>(c[r] & 0xFFFFu)) : 0u;
    q[r] = i < nc ? mass_q(weight(static_cast<uint32_t>(c[r] & 0xFFFFu))) : 0ull;
    kmax = max(kmax, key[r]);
  }
  // The top key, and whether every candidate lies within kCandBins keys of it.
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
  if (lane == 0) sc.u32_red[warp] = kmax;
  if (tid == 0) sc.n_kept = sc.n_ties = sc.far = 0;
  __syncthreads();  // every candidate is in registers: `cand` is free for the histogram
  kmax = sc.u32_red[0];
#pragma unroll
  for (int w = 1; w < kSampleWarps; ++w) kmax = max(kmax, sc.u32_red[w]);
  bool far = false;
#pragma unroll
  for (int r = 0; r < R; ++r) far |= tid + r * kSampleThreads < nc && kmax - key[r] >= static_cast<uint32_t>(kCandBins);
  if (__any_sync(0xffffffffu, far) && lane == 0) sc.far = 1;
  unsigned long long* hist = cand;  // bin d: the mass of the tokens with key kmax - d
#pragma unroll
  for (int r = 0; r < R; ++r) hist[tid * R + r] = 0ull;
  __syncthreads();
  if (sc.far) return false;
#pragma unroll
  for (int r = 0; r < R; ++r)
    if (q[r]) atomicAdd(&hist[kmax - key[r]], q[r]);
  __syncthreads();
  // Scan top down (thread t owns bins R t .. R t + R - 1): Z, then the first bin with
  // cum <= top_p Z < cum + mass and mass > 0.
  unsigned long long h[R], local = 0;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    h[r] = hist[tid * R + r];
    local += h[r];
  }
  const unsigned long long incl = warp_inclusive_scan(local);
  if (lane == 31) sc.ull_red[warp] = incl;
  if (tid == 0) sc.cut_d = -1;
  __syncthreads();
  unsigned long long cum = incl - local, Z = 0;
  for (int w = 0; w < kSampleWarps; ++w) {
    if (w < warp) cum += sc.ull_red[w];
    Z += sc.ull_red[w];
  }
  const double target = static_cast<double>(top_p) * static_cast<double>(Z);
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (h[r] > 0 && static_cast<double>(cum) <= target && target < static_cast<double>(cum + h[r])) {
      sc.cut_d = tid * R + r;  // one bin at most meets this
      sc.cut_cum = cum;
    }
    cum += h[r];
  }
  __syncthreads();
  if (sc.cut_d < 0) return false;  // the cut keeps every candidate
  const uint32_t key_star = kmax - static_cast<uint32_t>(sc.cut_d);
  // Tokens tied at key_star share one weight: the first n_tie_keep of them (by index) are kept.
  const unsigned long long e_star = mass_q(weight(key_to_bits(key_star)));
  if (e_star == 0) return false;
  const int n_tie_keep =
      static_cast<int>(floor((target - static_cast<double>(sc.cut_cum)) / static_cast<double>(e_star))) + 1;
  unsigned long long* kept = cand;  // the histogram is read: the kept tokens go here
  // Kept tokens above the cut go to the front of `kept`, tokens at the cut to its back.
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = tid + r * kSampleThreads;
    const bool above = i < nc && key[r] > key_star, tie = i < nc && key[r] == key_star;
    const unsigned ma = __ballot_sync(0xffffffffu, above), mt = __ballot_sync(0xffffffffu, tie);
    int base_a = 0, base_t = 0;
    if (lane == 0) {
      if (ma) base_a = atomicAdd(&sc.n_kept, __popc(ma));
      if (mt) base_t = atomicAdd(&sc.n_ties, __popc(mt));
    }
    base_a = __shfl_sync(0xffffffffu, base_a, 0);
    base_t = __shfl_sync(0xffffffffu, base_t, 0);
    const unsigned below = (1u << lane) - 1u;
    if (above) kept[base_a + __popc(ma & below)] = c[r];
    if (tie) kept[kSampleCand - 1 - (base_t + __popc(mt & below))] = c[r];
  }
  __syncthreads();
  const int n_above = sc.n_kept, n_ties = sc.n_ties;
  const int t_keep = min(n_ties, n_tie_keep);
  if (n_above + t_keep >= nc) return false;
  // A tie is kept when fewer than n_tie_keep ties have a lower index (its rank, counted over
  // the tie list; the ties at one bf16 value are few). All ranks are taken before any write.
  bool keep_tie[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = tid + r * kSampleThreads;
    keep_tie[r] = false;
    if (i < nc && key[r] == key_star) {
      if (n_ties <= n_tie_keep) {
        keep_tie[r] = true;
      } else {
        const unsigned long long idx = c[r] >> 16;
        int rank = 0;
        for (int j = 0; j < n_ties; ++j) rank += (kept[kSampleCand - 1 - j] >> 16) < idx;
        keep_tie[r] = rank < n_tie_keep;
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const unsigned mk = __ballot_sync(0xffffffffu, keep_tie[r]);
    int base_k = 0;
    if (lane == 0 && mk) base_k = atomicAdd(&sc.n_kept, __popc(mk));
    base_k = __shfl_sync(0xffffffffu, base_k, 0);
    if (keep_tie[r]) kept[base_k + __popc(mk & ((1u << lane) - 1u))] = c[r];
  }
  __syncthreads();
  const int n_keep = sc.n_kept;  // n_above + t_keep
  block_sort(kept, n_keep);      // by index (the keys lead with it); pads within the list's 4096 entries

  // Kept mass in index order over a contiguous slice per thread, then the draw.
  const int per = (n_keep + kSampleThreads - 1) / kSampleThreads;
  const int lo = min(n_keep, tid * per), hi2 = min(n_keep, lo + per);
  unsigned long long kept_mass = 0;
  for (int i = lo; i < hi2; ++i) kept_mass += mass_q(weight(static_cast<uint32_t>(kept[i] & 0xFFFFu)));
  const unsigned long long kincl = warp_inclusive_scan(kept_mass);
  if (lane == 31) sc.ull_red[warp] = kincl;
  __syncthreads();
  unsigned long long before = kincl - kept_mass, kept_total = 0;
  for (int w = 0; w < kSampleWarps; ++w) {
    if (w < warp) before += sc.ull_red[w];
    kept_total += sc.ull_red[w];
  }
  const double draw = static_cast<double>(p.uniforms[row]) * static_cast<double>(kept_total);
  if (tid == 0) *chosen = static_cast<int>(kept[n_keep - 1] >> 16);  // the last kept (rounding)
  __syncthreads();
  if (kept_mass > 0 && static_cast<double>(before) <= draw && draw < static_cast<double>(before + kept_mass)) {
    unsigned long long run = before;
    for (int i = lo; i < hi2; ++i) {
      run += mass_q(weight(static_cast<uint32_t>(kept[i] & 0xFFFFu)));
      if (static_cast<double>(run) > draw) {
        atomicMin(chosen, static_cast<int>(kept[i] >> 16));
        break;
      }
    }
  }
  __syncthreads();
  if (tid == 0) p.out[row] = *chosen;
  return true;
}

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(SampleParams p) {
  __shared__ union {
    float whist[kSampleWarps][256];         // per-warp mass histograms (whole-row passes)
    unsigned long long cand[kSampleCand];   // candidates: token index << 16 | logit bits
  } sh;
  float (*whist)[256] = sh.whist;
  __shared__ double hist[256];                // their sum over the warps
  __shared__ float fred[32];
  __shared__ int ired[32];
  __shared__ double dred[32];
  __shared__ uint32_t cut_key;
  __shared__ double cut_mass_above, cut_target;
  __shared__ int cut_found;
  __shared__ int chosen;
  __shared__ int ncand;
  __shared__ CandidateScratch cscratch;

  const int row = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const __nv_bfloat16* lg = p.logits + static_cast<int64_t>(row) * p.row_stride;
  const int V = p.vocab;
  const bool vec_ok = (reinterpret_cast<uintptr_t>(lg) & 15) == 0;
  const int groups = (V + 7) / 8;
  const int gpw = (groups + kSampleWarps - 1) / kSampleWarps;  // groups per warp segment
  const int g_begin = min(groups, warp * gpw), g_end = min(groups, g_begin + gpw);

  const float T = p.temperature[row];
  const bool greedy = !(T > 0.f);
  // Pass 1: max (and, for a greedy row, its first index).
  float mx = -INFINITY;
  int arg = INT_MAX;
  for (int base = g_begin; greedy && base < g_end; base += 32 * kSampleUnroll) {
    uint32_t b[kSampleUnroll][8];
    int n[kSampleUnroll];
    load_groups(lg, base, g_end, V, vec_ok, b, n);
#pragma unroll
    for (int u = 0; u < kSampleUnroll; ++u)
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float v = bits_to_float(b[u][e]);
        if (e < n[u] && v > mx) { mx = v; arg = 8 * (base + 32 * u + lane) + e; }  // indices visited in order
      }
  }
  if (!greedy) {  // the maximum alone: packed maxima, twice the loads in flight
    for (int base = g_begin; base < g_end; base += 32 * kSampleRawUnroll) {
      uint4 r[kSampleRawUnroll];
      int n[kSampleRawUnroll];
#pragma unroll
      for (int u = 0; u < kSampleRawUnroll; ++u) {
        const int g = base + 32 * u + lane;
        n[u] = g < g_end ? load_raw(lg, g, V, vec_ok, r[u]) : 0;
      }
#pragma unroll
      for (int u = 0; u < kSampleRawUnroll; ++u)
        if (n[u] > 0) mx = fmaxf(mx, group_max(r[u]));
    }
  }
  const float gmax = block_reduce(mx, [](float a, float b) { return fmaxf(a, b); }, fred);
  if (mx != gmax) arg = INT_MAX;
  const int garg = block_reduce(arg, [](int a, int b) { return min(a, b); }, ired);
  if (greedy) {
    if (tid == 0) p.out[row] = garg;
    return;
  }
  const float m = __fdiv_rn(gmax, T);
  const float top_p = p.top_p[row];
  auto weight = [&](uint32_t bits) { return expf(__fdiv_rn(bits_to_float(bits), T) - m); };
  // Logits below x_floor have weight < e^-28 < kNegligibleWeight (x / T - m < -28 up to the
  // rounding of the division), so the histogram passes skip them without computing it.
  const float x_floor = T * (m - 28.f);

  if (top_p < 1.f) {
    // Candidate pass: every token with logit >= x_floor. Each warp stages the candidates of its
    // segment in its own kWarpCand entries of the list, counting in a register (no shared
    // counter for all warps to meet on), then the warps' runs are packed together in order.
    constexpr int kWarpCand = kSampleCand / kSampleWarps;
    int wcount = 0;  // the same in every lane
    unsigned long long* mine_list = sh.cand + warp * kWarpCand;
    for (int base = g_begin; base < g_end; base += 32 * kSampleUnroll) {
      uint4 r[kSampleUnroll];
      int n[kSampleUnroll];
#pragma unroll
      for (int u = 0; u < kSampleUnroll; ++u) {
        const int g = base + 32 * u + lane;
        n[u] = g < g_end ? load_raw(lg, g, V, vec_ok, r[u]) : 0;
      }
#pragma unroll
      for (int u = 0; u < kSampleUnroll; ++u) {
        // Most groups hold no candidate: their packed maximum is below the floor.
        uint32_t mine = 0;
        if (n[u] > 0 && group_max(r[u]) >= x_floor) {
#pragma unroll
          for (int e = 0; e < 8; ++e) mine |= (e < n[u] && bits_to_float(raw_bits(r[u], e)) >= x_floor) ? (1u << e) : 0u;
        }
        const int cnt = __popc(mine);
        const int incl = warp_inclusive_scan(cnt);
        const int total = __shfl_sync(0xffffffffu, incl, 31);
        if (total == 0) continue;  // warp-uniform
        int slot = wcount + incl - cnt;
        const int g = base + 32 * u + lane;
        while (mine) {
          const int e = __ffs(mine) - 1;
          mine &= mine - 1;
          const uint32_t w = e < 2 ? r[u].x : e < 4 ? r[u].y : e < 6 ? r[u].z : r[u].w;
          const uint32_t bits = (e & 1) ? (w >> 16) : (w & 0xFFFFu);
          if (slot < kWarpCand) mine_list[slot] = (static_cast<unsigned long long>(8 * g + e) << 16) | bits;
          ++slot;
        }
        wcount += total;
      }
    }
    int total_cand;
    const int woff = warps_exclusive_scan(wcount, ired, &total_cand);  // syncs the block
    const bool overflow = __syncthreads_or(wcount > kWarpCand);
    int nc = total_cand;
    if (!overflow) {
      // Pack the runs: every warp reads its entries before any is written over.
      unsigned long long v[kWarpCand / 32];
#pragma unroll
      for (int k = 0; k < kWarpCand / 32; ++k) v[k] = lane + 32 * k < wcount ? mine_list[lane + 32 * k] : 0ull;
      __syncthreads();
#pragma unroll
      for (int k = 0; k < kWarpCand / 32; ++k)
        if (lane + 32 * k < wcount) sh.cand[woff + lane + 32 * k] = v[k];
      __syncthreads();
    } else {
      // A segment held more candidates than its run: collect again through one shared counter.
      if (tid == 0) ncand = 0;
      __syncthreads();
      for (int base = g_begin; base < g_end; base += 32 * kSampleUnroll) {
        uint32_t b[kSampleUnroll][8];
        int n[kSampleUnroll];
        load_groups(lg, base, g_end, V, vec_ok, b, n);
#pragma unroll
        for (int u = 0; u < kSampleUnroll; ++u)
          append_candidates(b[u], n[u], base + 32 * u + lane, x_floor, &ncand, sh.cand, kSampleCand);
      }
      __syncthreads();
      nc = ncand;
    }
    if (nc <= kSampleCand && sample_candidates(p, row, nc, sh.cand, top_p, T, m, cscratch, &chosen)) return;
    __syncthreads();  // the candidate list's memory holds the histograms from here on
  }

  uint32_t key_star = 0;  // tokens with key > key_star are kept
  int n_tie_keep = 0;     // how many tokens with key == key_star are kept (lowest indices)
  bool keep_all = !(top_p < 1.f);
  if (!keep_all) {
    // Pass 2: mass per high byte of the key (its total is the partition function Z).
    for (int k = lane; k < 256; k += 32) whist[warp][k] = 0.f;
    __syncwarp();
    for (int base = g_begin; base < g_end; base += 32 * kSampleUnroll) {
      uint32_t b[kSampleUnroll][8];
      int n[kSampleUnroll];
      load_groups(lg, base, g_end, V, vec_ok, b, n);
#pragma unroll
      for (int u = 0; u < kSampleUnroll; ++u)
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (e >= n[u] || !(bits_to_float(b[u][e]) >= x_floor)) continue;
          const float w = weight(b[u][e]);
          if (w > kNegligibleWeight) atomicAdd(&whist[warp][bf16_key_bits(b[u][e]) >> 8], w);
        }
    }
    __syncthreads();
    if (tid < 256) {
      double t = 0.0;
      for (int w = 0; w < kSampleWarps; ++w) t += whist[w][tid];
      hist[tid] = t;
    }
    __syncthreads();
    if (warp == 0) {
      // Z first (the total of the bins), then the cut against top_p * Z.
      double cum = 0.0, Z = 0.0;
      warp_find_cut(hist, 0.0, -1.0, false, &cum, &Z);
      const double t = static_cast<double>(top_p) * Z;
      const int k = warp_find_cut(hist, 0.0, t, false, &cum, &Z);
      if (lane == 0) {
        cut_found = k >= 0;
        cut_key = static_cast<uint32_t>(k);
        cut_mass_above = cum;
        cut_target = t;
      }
    }
    __syncthreads();
    const double target = cut_target;
    if (!cut_found) {
      keep_all = true;
    } else {
      // Pass 3: mass per low byte within the selected high byte.
      const uint32_t hi = cut_key;
      __syncthreads();
      for (int k = lane; k < 256; k += 32) whist[warp][k] = 0.f;
      __syncwarp();
      for (int base = g_begin; base < g_end; base += 32 * kSampleUnroll) {
        uint32_t b[kSampleUnroll][8];
        int n[kSampleUnroll];
        load_groups(lg, base, g_end, V, vec_ok, b, n);
#pragma unroll
        for (int u = 0; u < kSampleUnroll; ++u)
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const uint32_t k = bf16_key_bits(b[u][e]);
            if (e < n[u] && (k >> 8) == hi && bits_to_float(b[u][e]) >= x_floor) {
              const float w = weight(b[u][e]);
              if (w > kNegligibleWeight) atomicAdd(&whist[warp][k & 255u], w);
            }
          }
      }
      __syncthreads();
      if (tid < 256) {
        double t = 0.0;
        for (int w = 0; w < kSampleWarps; ++w) t += whist[w][tid];
        hist[tid] = t;
      }
      __syncthreads();
      if (warp == 0) {
        double cum = 0.0, total = 0.0;
        const int k = warp_find_cut(hist, cut_mass_above, target, true, &cum, &total);
        if (lane == 0) {
          cut_found = k >= 0;
          cut_key = (hi << 8) | static_cast<uint32_t>(k);
          cut_mass_above = cum;
        }
      }
      __syncthreads();
      if (!cut_found) {
        keep_all = true;
      } else {
        key_star = cut_key;
        // All tokens sharing key_star share one probability e_star.
        const uint32_t bits = (key_star & 0x8000u) ? (key_star & 0x7FFFu) : (~key_star & 0xFFFFu);
        const double e_star = weight(bits);
        const double room = target - cut_mass_above;
        n_tie_keep = static_cast<int>(floor(room / e_star)) + 1;
      }
    }
  }

  // Pass 4: tokens tied at key_star before each warp's segment (index order).
  int tie_base = 0;
  if (!keep_all) {
    int ties = 0;
    for (int base = g_begin; base < g_end; base += 32 * kSampleUnroll) {
      uint32_t b[kSampleUnroll][8];
      int n[kSampleUnroll];
      load_groups(lg, base, g_end, V, vec_ok, b, n);
#pragma unroll
      for (int u = 0; u < kSampleUnroll; ++u)
#pragma unroll
        for (int e = 0; e < 8; ++e) ties += (e < n[u] && bf16_key_bits(b[u][e]) == key_star);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ties += __shfl_xor_sync(0xffffffffu, ties, o);
    int total_ties;
    tie_base = warps_exclusive_scan(ties, ired, &total_ties);
  }
  // Kept mass of this lane's group, in index order; `rank` is the lane's first tie rank.
  auto group_mass = [&](const uint32_t (&b)[8], int n, int g, int rank, double& mass, int& last) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if (e >= n) continue;
      bool kept = keep_all;
      if (!kept) {
        const uint32_t k = bf16_key_bits(b[e]);
        kept = k > key_star || (k == key_star && rank++ < n_tie_keep);
      }
      if (kept) {
        mass += static_cast<double>(weight(b[e]));
        last = 8 * g + e;
      }
    }
  };
  auto group_ties = [&](const uint32_t (&b)[8], int n) {
    int t = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) t += (!keep_all && e < n && bf16_key_bits(b[e]) == key_star);
    return t;
  };

  // Pass 5: kept mass per warp segment, then their scan.
  double seg_mass = 0.0;
  int last_kept = -1;
  {
    int rank_base = tie_base;
    for (int base = g_begin; base < g_end; base += 32 * kSampleUnroll) {
      uint32_t b[kSampleUnroll][8];
      int n[kSampleUnroll];
      load_groups(lg, base, g_end, V, vec_ok, b, n);
#pragma unroll
      for (int u = 0; u < kSampleUnroll; ++u) {
        const int g = base + 32 * u + lane;
        const int t = n[u] ? group_ties(b[u], n[u]) : 0;
        const int t_incl = warp_inclusive_scan(t);
        double mass = 0.0;
        if (n[u]) group_mass(b[u], n[u], g, rank_base + t_incl - t, mass, last_kept);
        seg_mass += mass;
        rank_base += __shfl_sync(0xffffffffu, t_incl, 31);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) seg_mass += __shfl_xor_sync(0xffffffffu, seg_mass, o);
  double total;
  const double before = warps_exclusive_scan(seg_mass, dred, &total);
  const int glast = block_reduce(last_kept, [](int a, int b) { return max(a, b); }, ired);
  const double target = static_cast<double>(p.uniforms[row]) * total;
  if (tid == 0) chosen = glast;
  __syncthreads();

  // Pass 6: the warp whose segment holds the target walks it in index order.
  if (seg_mass > 0.0 && before <= target && target < before + seg_mass) {
    double run = before;
    int rank_base = tie_base;
    for (int base = g_begin; base < g_end; base += 32) {
      const int g = base + lane;
      uint32_t b[8];
      const int n = g < g_end ? load_group(lg, g, V, vec_ok, b) : 0;
      const int t = n ? group_ties(b, n) : 0;
      const int t_incl = warp_inclusive_scan(t);
      double mass = 0.0;
      int unused = -1;
      if (n) group_mass(b, n, g, rank_base + t_incl - t, mass, unused);
      const double m_incl = warp_inclusive_scan(mass);
      const double step_total = __shfl_sync(0xffffffffu, m_incl, 31);
      if (run + step_total > target) {
        // The first lane whose running mass passes the target holds the draw (when rounding
        // leaves none, the last lane with kept mass in this step).
        const unsigned has = __ballot_sync(0xffffffffu, mass > 0.0);
        const unsigned passed = __ballot_sync(0xffffffffu, mass > 0.0 && run + m_incl > target);
        const int owner = passed ? __ffs(passed) - 1 : 31 - __clz(has);
        if (has != 0u && lane == owner) {
          double r = run + m_incl - mass;
          int rank = rank_base + t_incl - t;
          int pick = -1, lane_last = -1;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (e >= n) continue;
            bool kept = keep_all;
            if (!kept) {
              const uint32_t k = bf16_key_bits(b[e]);
              kept = k > key_star || (k == key_star && rank++ < n_tie_keep);
            }
            if (kept && pick < 0) {
              r += static_cast<double>(weight(b[e]));
              lane_last = 8 * g + e;
              if (r > target) pick = lane_last;
            }
          }
          atomicMin(&chosen, pick >= 0 ? pick : lane_last);
        }
        break;  // uniform: every lane saw the same step total
      }
      run += step_total;
      rank_base += __shfl_sync(0xffffffffu, t_incl, 31);
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
