// Row-wise kernels around the GEMMs of one decoder layer, plus the page copy.
//
//   rmsnorm           RMSNorm.forward over the hidden size (src/helios/runtime/qwen3/layers.py:36-40),
//                     optionally gathering rows first (the logit-row index_select of
//                     Qwen3Model._forward_packed, model.py:108-110).
//   add_rmsnorm       the residual add `x + sublayer(x)` (layers.py:220-232) rounded to bf16,
//                     fused with the RMSNorm that consumes it.
//   swiglu            down-projection input silu(gate) * up (layers.py:26-27) with the
//                     reference's rounding (silu rounded to bf16, then the product).
//   embed             token-embedding gather (model.py:97).
//   page_copy         copy whole KV pages of every layer (dense snapshot/restore copies,
//                     src/helios/runtime/qwen3/cache.py:109-147, for a paged pool).
// All of them are HBM-bound: 16-byte vector loads/stores, one CTA per row.
#pragma once

#include "hb_common.cuh"

namespace hb {

constexpr int kRowThreads = 256;
constexpr int kRowVecs = 8;  // up to 8 x 8 bf16 per thread: hidden <= 16384

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < static_cast<int>(blockDim.x >> 5) ? red[lane] : 0.f;
  t = warp_sum(t);
  __syncthreads();
  return t;
}

struct RowNormParams {
  const __nv_bfloat16* x;      // [rows_in, hidden]
  const __nv_bfloat16* y;      // [rows, hidden] or null (add_rmsnorm only)
  const int64_t* row_index;    // [rows] or null: gather x rows first
  const float* scale;          // [hidden]
  __nv_bfloat16* sum_out;      // [rows, hidden] or null: x + y
  __nv_bfloat16* norm_out;     // [rows, hidden]
  int32_t rows, hidden;
  int64_t rows_in;
  float eps;
};

__global__ void __launch_bounds__(kRowThreads) rmsnorm_kernel(RowNormParams p) {
  __shared__ float red[32];
  const int r = blockIdx.x;
  int64_t src_row = r;
  if (p.row_index != nullptr) {
    src_row = p.row_index[r];
    if (src_row < 0 || src_row >= p.rows_in) {
      if (threadIdx.x == 0) raise_status(kStatusBadRow);
      src_row = 0;
    }
  }
  const int nvec = p.hidden / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(p.x + src_row * p.hidden);
  const uint4* yr = p.y ? reinterpret_cast<const uint4*>(p.y + static_cast<int64_t>(r) * p.hidden) : nullptr;
  float v[kRowVecs][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kRowVecs; ++i) {
    const int vi = threadIdx.x + i * kRowThreads;
    if (vi < nvec) {
      unpack8(xr[vi], v[i]);
      if (yr) {
        float w[8];
        unpack8(yr[vi], w);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[i][e] = __bfloat162float(__float2bfloat16_rn(__fadd_rn(v[i][e], w[e])));
        reinterpret_cast<uint4*>(p.sum_out + static_cast<int64_t>(r) * p.hidden)[vi] = pack8(v[i]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = __fmaf_rn(v[i][e], v[i][e], ss);
    }
  }
  ss = block_sum(ss, red);
  const float inv = rsqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(p.hidden)), p.eps));
  const float4* sc = reinterpret_cast<const float4*>(p.scale);
  uint4* out = reinterpret_cast<uint4*>(p.norm_out + static_cast<int64_t>(r) * p.hidden);
#pragma unroll
  for (int i = 0; i < kRowVecs; ++i) {
    const int vi = threadIdx.x + i * kRowThreads;
    if (vi < nvec) {
      const float4 s0 = sc[2 * vi], s1 = sc[2 * vi + 1];
      const float s[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = __fmul_rn(__fmul_rn(v[i][e], inv), s[e]);
      out[vi] = pack8(o);
    }
  }
}

// Warp-per-row variant for hidden <= 32 * 8 * MAXV: every lane issues all of its
// 16-byte loads before reducing, and the reduction stays inside the warp.
constexpr int kNormWarps = 4;  // rows (warps) per CTA: small CTAs spread 2080 rows evenly over the SMs

template <int MAXV>
__global__ void __launch_bounds__(kNormWarps * 32) rmsnorm_warp_kernel(RowNormParams p) {
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * kNormWarps + (threadIdx.x >> 5);
  if (r >= p.rows) return;
  int64_t src_row = r;
  if (p.row_index != nullptr) {
    src_row = p.row_index[r];
    if (src_row < 0 || src_row >= p.rows_in) {
      if (lane == 0) raise_status(kStatusBadRow);
      src_row = 0;
    }
  }
  const int nvec = p.hidden / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(p.x + src_row * p.hidden);
  const uint4* yr = p.y ? reinterpret_cast<const uint4*>(p.y + static_cast<int64_t>(r) * p.hidden) : nullptr;
  uint4 raw[MAXV], raw_y[MAXV];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nvec) {
      raw[i] = xr[vi];
      if (yr) raw_y[i] = yr[vi];
    }
  }
  float v[MAXV][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nvec) {
      if (yr) {  // residual sum rounded to bf16 (one cvt per pair), stored, then reused as floats
        float a[8], w[8];
        unpack8(raw[i], a);
        unpack8(raw_y[i], w);
        const uint4 sum = make_uint4(pack_bf16(__fadd_rn(a[0], w[0]), __fadd_rn(a[1], w[1])),
                                     pack_bf16(__fadd_rn(a[2], w[2]), __fadd_rn(a[3], w[3])),
                                     pack_bf16(__fadd_rn(a[4], w[4]), __fadd_rn(a[5], w[5])),
                                     pack_bf16(__fadd_rn(a[6], w[6]), __fadd_rn(a[7], w[7])));
        reinterpret_cast<uint4*>(p.sum_out + static_cast<int64_t>(r) * p.hidden)[vi] = sum;
        unpack8(sum, v[i]);
      } else {
        unpack8(raw[i], v[i]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = __fmaf_rn(v[i][e], v[i][e], ss);
    }
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(p.hidden)), p.eps));
  const float4* sc = reinterpret_cast<const float4*>(p.scale);
  uint4* out = reinterpret_cast<uint4*>(p.norm_out + static_cast<int64_t>(r) * p.hidden);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nvec) {
      const float4 s0 = sc[2 * vi], s1 = sc[2 * vi + 1];
      const float s[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = __fmul_rn(__fmul_rn(v[i][e], inv), s[e]);
      out[vi] = pack8(o);
    }
  }
}

struct SwigluParams {
  const __nv_bfloat16* gate_up;  // [rows, 2 * inter]: gate then up
  __nv_bfloat16* out;            // [rows, inter]
  int64_t rows, inter;
};

// Grid: (column blocks, rows); each thread owns two 16-byte vectors of one row, so
// there is no per-element index division and four loads are in flight per thread.
constexpr int kSwigluThreads = 128;
constexpr int kSwigluVecs = 2;

__global__ void __launch_bounds__(kSwigluThreads) swiglu_kernel(SwigluParams p) {
  const int64_t nvec_row = p.inter / 8;
  for (int64_t r = blockIdx.y; r < p.rows; r += gridDim.y) {
    const uint4* row = reinterpret_cast<const uint4*>(p.gate_up + r * 2 * p.inter);
    uint4* out = reinterpret_cast<uint4*>(p.out + r * p.inter);
    const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kSwigluThreads * kSwigluVecs + threadIdx.x;
    uint4 g_raw[kSwigluVecs], u_raw[kSwigluVecs];
#pragma unroll
    for (int k = 0; k < kSwigluVecs; ++k) {
      const int64_t c = c0 + k * kSwigluThreads;
      if (c < nvec_row) {
        g_raw[k] = row[c];
        u_raw[k] = row[nvec_row + c];
      }
    }
#pragma unroll
    for (int k = 0; k < kSwigluVecs; ++k) {
      const int64_t c = c0 + k * kSwigluThreads;
      if (c < nvec_row) {
        float g[8], u[8], o[8];
        unpack8(g_raw[k], g);
        unpack8(u_raw[k], u);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          // silu(g) = g / (1 + e^-g) in fp32 with the fast exp and divide intrinsics
          // (fp32 error far below the bf16 rounding that follows; e^-g = inf gives -0,
          // as the exact quotient does), rounded to bf16, then times up, rounded.
          const float sl = __bfloat162float(__float2bfloat16_rn(__fdividef(g[e], 1.f + __expf(-g[e]))));
          o[e] = __fmul_rn(sl, u[e]);
        }
        out[c] = pack8(o);
      }
    }
  }
}

struct EmbedParams {
  const int64_t* ids;
  const __nv_bfloat16* table;  // [vocab, hidden]
  __nv_bfloat16* out;          // [tokens, hidden]
  int64_t tokens, vocab;
  int32_t hidden;
};

__global__ void __launch_bounds__(256) embed_kernel(EmbedParams p) {
  const int t = blockIdx.x;
  int64_t id = p.ids[t];
  if (id < 0 || id >= p.vocab) {
    if (threadIdx.x == 0) raise_status(kStatusBadToken);
    id = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(p.table + id * p.hidden);
  uint4* dst = reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(t) * p.hidden);
  for (int i = threadIdx.x; i < p.hidden / 8; i += blockDim.x) dst[i] = src[i];
}

struct PageCopyParams {
  uint8_t* base;              // first pool tensor
  int64_t tensor_stride;      // bytes between consecutive pool tensors (layers x {K, V})
  int32_t tensors;
  int64_t page_bytes;
  int64_t num_pages;
  const int32_t* src_pages;
  const int32_t* dst_pages;
  int32_t pairs;
};

__global__ void __launch_bounds__(256) page_copy_kernel(PageCopyParams p) {
  const int64_t vec_per_page = p.page_bytes / 16;
  const int64_t total = static_cast<int64_t>(p.pairs) * p.tensors * vec_per_page;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t v = i % vec_per_page;
    const int64_t rest = i / vec_per_page;
    const int tensor = static_cast<int>(rest % p.tensors);
    const int pair = static_cast<int>(rest / p.tensors);
    const int64_t s = p.src_pages[pair], d = p.dst_pages[pair];
    if (s < 0 || s >= p.num_pages || d < 0 || d >= p.num_pages) {
      if (v == 0 && tensor == 0) raise_status(kStatusBadPage);
      continue;
    }
    uint8_t* t = p.base + tensor * p.tensor_stride;
    reinterpret_cast<uint4*>(t + d * p.page_bytes)[v] = reinterpret_cast<const uint4*>(t + s * p.page_bytes)[v];
  }
}

}  // namespace hb
