// Kernel (b): fused per-head q/k RMSNorm + RoPE + paged KV append.
//
// Replaces, per decoder layer, the reference's chain
//   q_norm/k_norm  (RMSNorm.forward, src/helios/runtime/qwen3/layers.py:36-40),
//   apply_rope     (layers.py:54-72, with position_ids),
//   _write         (two index_copy_ into the pool, paged_cache.py:335-345)
// with one launch. One warp handles one (token, head) row of d elements; each
// lane holds d/32 contiguous elements, so the RoPE partner (i +- d/2) is lane ^ 16.
//
// Rounding points follow the reference exactly: the norm is fp32
// (x * rsqrt(mean(x^2) + eps)) * scale_fp32, rounded to bf16; RoPE then computes
// fl(fl(n * cos) + fl(rot(n) * sin)) in fp32 from that bf16 value and rounds to
// bf16 (no fused multiply-add, matching separate elementwise ops).
#pragma once

#include "hb_common.cuh"

namespace hb {

struct NormRopeParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t q_tok, q_head, k_tok, k_head, v_tok, v_head;  // element strides
  const float* q_scale;  // [d] or null: no norm
  const float* k_scale;  // [d] or null: no norm
  float eps;
  const float* cos;  // [rope_rows, d] or null: no rotation
  const float* sin;
  int64_t rope_rows;
  const int64_t* positions;    // [T]
  const int64_t* write_slots;  // [T]
  __nv_bfloat16* q_out;        // [T, H, d] or null
  __nv_bfloat16* key_pool;     // [pool_slots, Hkv, d]
  __nv_bfloat16* value_pool;   // [pool_slots, Hkv, d]
  int64_t pool_slots;
  int32_t tokens, heads, kv_heads;
};

template <int D>
__device__ __forceinline__ void load_row(const __nv_bfloat16* src, int lane, float (&x)[D / 32]) {
  constexpr int E = D / 32;
  if constexpr (E == 4) {
    const uint2 raw = *reinterpret_cast<const uint2*>(src + lane * E);
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
    x[0] = __low2float(a); x[1] = __high2float(a); x[2] = __low2float(b); x[3] = __high2float(b);
  } else {
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(src + lane * E);
    x[0] = __low2float(a); x[1] = __high2float(a);
  }
}

template <int D>
__device__ __forceinline__ void store_row(__nv_bfloat16* dst, int lane, const float (&x)[D / 32]) {
  constexpr int E = D / 32;
  if constexpr (E == 4) {
    uint2 raw;
    raw.x = pack_bf16(x[0], x[1]);
    raw.y = pack_bf16(x[2], x[3]);
    *reinterpret_cast<uint2*>(dst + lane * E) = raw;
  } else {
    *reinterpret_cast<uint32_t*>(dst + lane * E) = pack_bf16(x[0], x[1]);
  }
}

// Per-head RMSNorm then RoPE on one row held as d/32 values per lane. `scale`,
// `cs` and `sn` are this lane's slices (null scale: no norm; null cs: no rotation).
template <int D>
__device__ __forceinline__ void norm_rope_row(float (&x)[D / 32], int lane, const float* scale, float eps,
                                              const float* cs, const float* sn) {
  constexpr int E = D / 32;
  if (scale != nullptr) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) ss = __fmaf_rn(x[e], x[e], ss);
    ss = warp_sum(ss);
    const float inv = rsqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(D)), eps));
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(__fmul_rn(x[e], inv), scale[e])));
  }
  if (cs != nullptr) {
    float partner[E];
#pragma unroll
    for (int e = 0; e < E; ++e) partner[e] = __shfl_xor_sync(0xffffffffu, x[e], 16);
    const bool first_half = lane < 16;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float rot = first_half ? -partner[e] : partner[e];
      x[e] = __bfloat162float(__float2bfloat16_rn(__fadd_rn(__fmul_rn(x[e], cs[e]), __fmul_rn(rot, sn[e]))));
    }
  }
}

// One warp per (token, group of kRopeRowsPerWarp head rows): the warp issues its
// position, slot, row, scale and (after the position) cos/sin loads together, so a
// warp pays about two dependent memory latencies; thousands of warps run at once.
constexpr int kRopeWarps = 8;        // warps per CTA
constexpr int kRopeRowsPerWarp = 4;  // head rows per warp

template <int D>
__global__ void __launch_bounds__(kRopeWarps * 32) norm_rope_append_kernel(NormRopeParams p) {
  constexpr int E = D / 32;
  const int lane = threadIdx.x & 31;
  const int rows = p.heads + 2 * p.kv_heads;
  const int groups = (rows + kRopeRowsPerWarp - 1) / kRopeRowsPerWarp;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * kRopeWarps + (threadIdx.x >> 5);
  if (gw >= static_cast<int64_t>(p.tokens) * groups) return;
  const int t = static_cast<int>(gw / groups);
  const int row0 = static_cast<int>(gw % groups) * kRopeRowsPerWarp;
  const int64_t slot = p.write_slots[t];
  float x[kRopeRowsPerWarp][E];
#pragma unroll
  for (int i = 0; i < kRopeRowsPerWarp; ++i) {  // row loads first
    const int hr = row0 + i;
    if (hr >= rows) break;
    if (hr < p.heads) {
      if (p.q_out != nullptr) load_row<D>(p.q + t * p.q_tok + hr * p.q_head, lane, x[i]);
    } else if (hr < p.heads + p.kv_heads) {
      load_row<D>(p.k + t * p.k_tok + (hr - p.heads) * p.k_head, lane, x[i]);
    } else {
      load_row<D>(p.v + t * p.v_tok + (hr - p.heads - p.kv_heads) * p.v_head, lane, x[i]);
    }
  }
  float qsc[E], ksc[E], cs[E], sn[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    qsc[e] = p.q_scale != nullptr ? p.q_scale[lane * E + e] : 1.f;
    ksc[e] = p.k_scale != nullptr ? p.k_scale[lane * E + e] : 1.f;
  }
  bool rope_ok = p.cos == nullptr;
  if (p.cos != nullptr) {
    const int64_t pos = p.positions[t];
    if (pos >= 0 && pos < p.rope_rows) {
      rope_ok = true;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        cs[e] = p.cos[pos * D + lane * E + e];
        sn[e] = p.sin[pos * D + lane * E + e];
      }
    } else if (lane == 0) {
      raise_status(kStatusBadPosition);
    }
  }
  const bool slot_ok = slot >= 0 && slot < p.pool_slots;
  if (!slot_ok && lane == 0 && row0 + kRopeRowsPerWarp > p.heads) raise_status(kStatusBadSlot);
  const float* rope_c = p.cos != nullptr ? cs : nullptr;
  const float* rope_s = p.cos != nullptr ? sn : nullptr;
#pragma unroll
  for (int i = 0; i < kRopeRowsPerWarp; ++i) {
    const int hr = row0 + i;
    if (hr >= rows) break;
    if (hr < p.heads) {  // query head
      if (p.q_out == nullptr || !rope_ok) continue;
      norm_rope_row<D>(x[i], lane, p.q_scale != nullptr ? qsc : nullptr, p.eps, rope_c, rope_s);
      store_row<D>(p.q_out + (static_cast<int64_t>(t) * p.heads + hr) * D, lane, x[i]);
    } else if (hr < p.heads + p.kv_heads) {  // key head: norm + rope, then into the pool
      if (!slot_ok || !rope_ok) continue;
      norm_rope_row<D>(x[i], lane, p.k_scale != nullptr ? ksc : nullptr, p.eps, rope_c, rope_s);
      store_row<D>(p.key_pool + (slot * p.kv_heads + (hr - p.heads)) * D, lane, x[i]);
    } else {  // value head: copied as is
      if (!slot_ok) continue;
      store_row<D>(p.value_pool + (slot * p.kv_heads + (hr - p.heads - p.kv_heads)) * D, lane, x[i]);
    }
  }
}

}  // namespace hb
