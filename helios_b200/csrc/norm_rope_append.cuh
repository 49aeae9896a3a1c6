// Kernel (b): fused per-head q/k RMSNorm + RoPE + paged KV append.
//
// Replaces, per decoder layer, the reference's chain
//   q_norm/k_norm  (RMSNorm.forward, src/helios/runtime/qwen3/layers.py:36-40),
//   apply_rope     (layers.py:54-72, with position_ids),
//   _write         (two index_copy_ into the pool, paged_cache.py:335-345)
// with one launch (one CTA per token; layout below).
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

// One CTA per token. A head row of D bf16 values is spread over D/8 lanes, 16 B per
// lane (a 256 B row for D = 128 is one fully used 16-lane segment), so a warp moves
// 2 (D = 128) or 4 (D = 64) rows per instruction. Every thread first issues the loads
// of all its rows of the token (q, k and v rows are one contiguous span of the fused
// projection output), together with the token's position and write slot; the cos/sin
// slice of its lane and the norm scales follow. The RoPE partner of element i
// (i +- D/2) sits D/16 lanes away, and the row's sum of squares is a shuffle
// reduction within the row's lanes.
constexpr int kRopeThreads = 256;
constexpr int kRopeMaxRows = 3;  // rows one thread keeps in flight per pass (48 rows = one pass)

template <int D>
__global__ void __launch_bounds__(kRopeThreads, 4) norm_rope_append_kernel(NormRopeParams p) {
  constexpr int kLanes = D / 8;                    // lanes per head row
  constexpr int kSlots = kRopeThreads / kLanes;    // head rows handled side by side
  const int t = blockIdx.x;
  const int j = threadIdx.x % kLanes;              // this lane's 8 elements: 8j .. 8j+7
  const int slot0 = threadIdx.x / kLanes;
  // Rows of one warp may take different branches (q / k / v), so shuffles name only
  // the lanes of this thread's row; each row's lanes always take the same path.
  const unsigned row_mask = static_cast<unsigned>((1ull << kLanes) - 1) << ((threadIdx.x & 31) & ~(kLanes - 1));
  const int rows = p.heads + 2 * p.kv_heads;
  const int64_t slot = p.write_slots[t];
  const int64_t pos = p.cos != nullptr ? p.positions[t] : 0;
  const bool slot_ok = slot >= 0 && slot < p.pool_slots;
  const bool pos_ok = p.cos == nullptr || (pos >= 0 && pos < p.rope_rows);
  if (threadIdx.x == 0) {
    if (!slot_ok) raise_status(kStatusBadSlot);
    if (!pos_ok) raise_status(kStatusBadPosition);
  }
  for (int base = slot0; base < rows; base += kSlots * kRopeMaxRows) {
    uint4 raw[kRopeMaxRows];
#pragma unroll
    for (int i = 0; i < kRopeMaxRows; ++i) {  // all row loads first
      const int hr = base + i * kSlots;
      raw[i] = make_uint4(0, 0, 0, 0);
      if (hr >= rows) continue;
      const __nv_bfloat16* src;
      if (hr < p.heads) {
        if (p.q_out == nullptr) continue;
        src = p.q + t * p.q_tok + hr * p.q_head;
      } else if (hr < p.heads + p.kv_heads) {
        src = p.k + t * p.k_tok + (hr - p.heads) * p.k_head;
      } else {
        src = p.v + t * p.v_tok + (hr - p.heads - p.kv_heads) * p.v_head;
      }
      raw[i] = *reinterpret_cast<const uint4*>(src + 8 * j);
    }
    // cos and the signed sin of this lane's 8 elements: rot(x) = (-x2, x1), so the
    // first half multiplies its partner by -sin (negation is exact).
    float cs[8], sn[8];
    if (p.cos != nullptr && pos_ok) {
      const float4* c4 = reinterpret_cast<const float4*>(p.cos + pos * D + 8 * j);
      const float4* s4 = reinterpret_cast<const float4*>(p.sin + pos * D + 8 * j);
      const float4 c0 = c4[0], c1 = c4[1], s0 = s4[0], s1 = s4[1];
      const float sg = j < kLanes / 2 ? -1.f : 1.f;
      cs[0] = c0.x; cs[1] = c0.y; cs[2] = c0.z; cs[3] = c0.w; cs[4] = c1.x; cs[5] = c1.y; cs[6] = c1.z; cs[7] = c1.w;
      sn[0] = sg * s0.x; sn[1] = sg * s0.y; sn[2] = sg * s0.z; sn[3] = sg * s0.w;
      sn[4] = sg * s1.x; sn[5] = sg * s1.y; sn[6] = sg * s1.z; sn[7] = sg * s1.w;
    }
#pragma unroll
    for (int i = 0; i < kRopeMaxRows; ++i) {
      const int hr = base + i * kSlots;
      if (hr >= rows) break;  // uniform over the row's lanes
      if (hr >= p.heads + p.kv_heads) {  // value head: copied as is
        if (slot_ok) *reinterpret_cast<uint4*>(p.value_pool + (slot * p.kv_heads + (hr - p.heads - p.kv_heads)) * D + 8 * j) = raw[i];
        continue;
      }
      const bool is_q = hr < p.heads;
      if (is_q ? (p.q_out == nullptr || !pos_ok) : (!slot_ok || !pos_ok)) continue;
      // Every rounding point yields bf16 values, kept packed (one cvt.bf16x2 per pair) and
      // unpacked only where fp32 arithmetic follows.
      uint4 y = raw[i];
      const float* scale = is_q ? p.q_scale : p.k_scale;
      if (scale != nullptr) {  // RMSNorm over the row (fp32): bf16(fl(fl(x * inv) * scale))
        float x[8];
        unpack8(raw[i], x);
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) ss = __fmaf_rn(x[e], x[e], ss);
#pragma unroll
        for (int o = kLanes / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(row_mask, ss, o);
        // mean = ss / D: D is a power of two, so the product by 1 / D is the exact quotient.
        const float inv = rsqrtf(__fadd_rn(ss * (1.f / static_cast<float>(D)), p.eps));
        const float4 g0 = reinterpret_cast<const float4*>(scale + 8 * j)[0];
        const float4 g1 = reinterpret_cast<const float4*>(scale + 8 * j)[1];
        y.x = pack_bf16(__fmul_rn(__fmul_rn(x[0], inv), g0.x), __fmul_rn(__fmul_rn(x[1], inv), g0.y));
        y.y = pack_bf16(__fmul_rn(__fmul_rn(x[2], inv), g0.z), __fmul_rn(__fmul_rn(x[3], inv), g0.w));
        y.z = pack_bf16(__fmul_rn(__fmul_rn(x[4], inv), g1.x), __fmul_rn(__fmul_rn(x[5], inv), g1.y));
        y.w = pack_bf16(__fmul_rn(__fmul_rn(x[6], inv), g1.z), __fmul_rn(__fmul_rn(x[7], inv), g1.w));
      }
      if (p.cos != nullptr) {  // bf16(fl(fl(y cos) + fl(rot(y) sin))), rot(y) = (-y2, y1)
        uint4 other;  // the partner lane's 8 values, D/2 elements away
        other.x = __shfl_xor_sync(row_mask, y.x, kLanes / 2);
        other.y = __shfl_xor_sync(row_mask, y.y, kLanes / 2);
        other.z = __shfl_xor_sync(row_mask, y.z, kLanes / 2);
        other.w = __shfl_xor_sync(row_mask, y.w, kLanes / 2);
        float v[8], w[8];
        unpack8(y, v);
        unpack8(other, w);
        y.x = pack_bf16(__fadd_rn(__fmul_rn(v[0], cs[0]), __fmul_rn(w[0], sn[0])),
                        __fadd_rn(__fmul_rn(v[1], cs[1]), __fmul_rn(w[1], sn[1])));
        y.y = pack_bf16(__fadd_rn(__fmul_rn(v[2], cs[2]), __fmul_rn(w[2], sn[2])),
                        __fadd_rn(__fmul_rn(v[3], cs[3]), __fmul_rn(w[3], sn[3])));
        y.z = pack_bf16(__fadd_rn(__fmul_rn(v[4], cs[4]), __fmul_rn(w[4], sn[4])),
                        __fadd_rn(__fmul_rn(v[5], cs[5]), __fmul_rn(w[5], sn[5])));
        y.w = pack_bf16(__fadd_rn(__fmul_rn(v[6], cs[6]), __fmul_rn(w[6], sn[6])),
                        __fadd_rn(__fmul_rn(v[7], cs[7]), __fmul_rn(w[7], sn[7])));
      }
      __nv_bfloat16* dst = is_q ? p.q_out + (static_cast<int64_t>(t) * p.heads + hr) * D
                                : p.key_pool + (slot * p.kv_heads + (hr - p.heads)) * D;
      *reinterpret_cast<uint4*>(dst + 8 * j) = y;
    }
  }
}

}  // namespace hb
