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

// One CTA per token. A head row of D bf16 values is spread over D/8 lanes; lane j owns
// the 4 elements [4j, 4j+4) of the first half and their RoPE partners [D/2 + 4j, D/2 +
// 4j + 4) of the second half (two 8-byte loads per row; the 16 lanes of a D = 128 row
// read and write two full 128-byte halves), so the rotation needs no data from another
// lane. A warp moves two (D = 128) or four (D = 64) rows per instruction. Every thread
// first issues the loads of all its rows of the token (q, k and v rows are one
// contiguous span of the fused projection output), with the token's position and write
// slot; its cos/sin values and the norm scales follow. The row's sum of squares is a
// shuffle reduction within the row's lanes.
constexpr int kRopeThreads = 256;
constexpr int kRopeMaxRows = 3;  // rows one thread keeps in flight per pass (48 rows = one pass)

// Two fp32 products / sums / differences in one instruction (sm_100 f32x2), each rounded to
// nearest as its scalar form is.
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 d;
  asm("{.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rd;}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rd;}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
  float2 d;
  asm("{.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "sub.rn.f32x2 rd, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rd;}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 unpack2(uint32_t w) {
  const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&w);
  return make_float2(__low2float(h), __high2float(h));
}
__device__ __forceinline__ uint32_t pack2(float2 f) { return pack_bf16(f.x, f.y); }

__device__ __forceinline__ void unpack4(const uint2& v, float (&f)[4]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
  f[0] = __low2float(h[0]);
  f[1] = __high2float(h[0]);
  f[2] = __low2float(h[1]);
  f[3] = __high2float(h[1]);
}

// One lane's share of a head row's RMSNorm: the row's D values are spread over kLanes lanes
// (named by row_mask), this lane holding elements [4j, 4j+4) in ylo and [D/2 + 4j, D/2 + 4j
// + 4) in yhi as packed bf16, and ga / gb the norm scales at those elements. fp32 norm
// bf16(fl(fl(x * inv) * scale)) with inv = rsqrt(mean(x^2) + eps); the sum of squares is
// this lane's eight products in order, then a butterfly over the row's lanes.
template <int kLanes, int D>
__device__ __forceinline__ void norm_lane(uint2& ylo, uint2& yhi, const float4& ga, const float4& gb, float eps,
                                          unsigned row_mask) {
  float a[4], b[4];
  unpack4(ylo, a);
  unpack4(yhi, b);
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) ss = __fmaf_rn(a[e], a[e], ss);
#pragma unroll
  for (int e = 0; e < 4; ++e) ss = __fmaf_rn(b[e], b[e], ss);
#pragma unroll
  for (int o = kLanes / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(row_mask, ss, o);
  // mean = ss / D: D is a power of two, so the product by 1 / D is the exact quotient.
  const float inv = rsqrtf(__fadd_rn(ss * (1.f / static_cast<float>(D)), eps));
  const float2 inv2 = make_float2(inv, inv);
  ylo.x = pack2(mul2(mul2(make_float2(a[0], a[1]), inv2), make_float2(ga.x, ga.y)));
  ylo.y = pack2(mul2(mul2(make_float2(a[2], a[3]), inv2), make_float2(ga.z, ga.w)));
  yhi.x = pack2(mul2(mul2(make_float2(b[0], b[1]), inv2), make_float2(gb.x, gb.y)));
  yhi.y = pack2(mul2(mul2(make_float2(b[2], b[3]), inv2), make_float2(gb.z, gb.w)));
}

// One lane's share of RoPE, y * cos + rot(y) * sin with rot(y) = (-y_hi, y_lo):
// lo = fl(fl(y_lo c) - fl(y_hi s)), hi = fl(fl(y_hi c) + fl(y_lo s)), each rounded to bf16
// (negation is exact); c_lo/s_lo are the tables at this lane's first-half elements.
__device__ __forceinline__ void rope_lane(uint2& ylo, uint2& yhi, const float (&c_lo)[4], const float (&c_hi)[4],
                                          const float (&s_lo)[4], const float (&s_hi)[4]) {
  const float2 a01 = unpack2(ylo.x), a23 = unpack2(ylo.y), b01 = unpack2(yhi.x), b23 = unpack2(yhi.y);
  const float2 cl01 = make_float2(c_lo[0], c_lo[1]), cl23 = make_float2(c_lo[2], c_lo[3]);
  const float2 ch01 = make_float2(c_hi[0], c_hi[1]), ch23 = make_float2(c_hi[2], c_hi[3]);
  const float2 sl01 = make_float2(s_lo[0], s_lo[1]), sl23 = make_float2(s_lo[2], s_lo[3]);
  const float2 sh01 = make_float2(s_hi[0], s_hi[1]), sh23 = make_float2(s_hi[2], s_hi[3]);
  ylo = make_uint2(pack2(sub2(mul2(a01, cl01), mul2(b01, sl01))), pack2(sub2(mul2(a23, cl23), mul2(b23, sl23))));
  yhi = make_uint2(pack2(add2(mul2(b01, ch01), mul2(a01, sh01))), pack2(add2(mul2(b23, ch23), mul2(a23, sh23))));
}

// rope_lane with the table values as float4 (the same arithmetic).
__device__ __forceinline__ void rope_lane(uint2& ylo, uint2& yhi, const float4& cl, const float4& ch,
                                          const float4& sl, const float4& sh) {
  const float c_lo[4] = {cl.x, cl.y, cl.z, cl.w}, c_hi[4] = {ch.x, ch.y, ch.z, ch.w};
  const float s_lo[4] = {sl.x, sl.y, sl.z, sl.w}, s_hi[4] = {sh.x, sh.y, sh.z, sh.w};
  rope_lane(ylo, yhi, c_lo, c_hi, s_lo, s_hi);
}

template <int D>
__global__ void __launch_bounds__(kRopeThreads, 4) norm_rope_append_kernel(NormRopeParams p) {
  constexpr int kLanes = D / 8;                    // lanes per head row
  constexpr int kSlots = kRopeThreads / kLanes;    // head rows handled side by side
  constexpr int kHalf = D / 2;
  pdl_wait();     // the q|k|v projection ahead of this kernel has finished
  pdl_trigger();  // every CTA is resident once all have passed here: the attention may launch
  const int t = blockIdx.x;
  const int j = threadIdx.x % kLanes;              // elements 4j..4j+3 and D/2+4j..D/2+4j+3
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
  const __nv_bfloat16* q_tok = p.q + t * p.q_tok;
  const __nv_bfloat16* k_tok = p.k + t * p.k_tok;
  const __nv_bfloat16* v_tok = p.v + t * p.v_tok;
  for (int base = slot0; base < rows; base += kSlots * kRopeMaxRows) {
    uint2 lo[kRopeMaxRows], hi[kRopeMaxRows];
#pragma unroll
    for (int i = 0; i < kRopeMaxRows; ++i) {  // all row loads first
      const int hr = base + i * kSlots;
      lo[i] = hi[i] = make_uint2(0, 0);
      if (hr >= rows) continue;
      const __nv_bfloat16* src;
      if (hr < p.heads) {
        if (p.q_out == nullptr) continue;
        src = q_tok + hr * p.q_head;
      } else if (hr < p.heads + p.kv_heads) {
        src = k_tok + (hr - p.heads) * p.k_head;
      } else {
        src = v_tok + (hr - p.heads - p.kv_heads) * p.v_head;
      }
      lo[i] = *reinterpret_cast<const uint2*>(src + 4 * j);
      hi[i] = *reinterpret_cast<const uint2*>(src + kHalf + 4 * j);
    }
    // This lane's cos and sin at its two element groups.
    float c_lo[4], c_hi[4], s_lo[4], s_hi[4];
    if (p.cos != nullptr && pos_ok) {
      const float4 a = *reinterpret_cast<const float4*>(p.cos + pos * D + 4 * j);
      const float4 b = *reinterpret_cast<const float4*>(p.cos + pos * D + kHalf + 4 * j);
      const float4 c = *reinterpret_cast<const float4*>(p.sin + pos * D + 4 * j);
      const float4 d = *reinterpret_cast<const float4*>(p.sin + pos * D + kHalf + 4 * j);
      c_lo[0] = a.x; c_lo[1] = a.y; c_lo[2] = a.z; c_lo[3] = a.w;
      c_hi[0] = b.x; c_hi[1] = b.y; c_hi[2] = b.z; c_hi[3] = b.w;
      s_lo[0] = c.x; s_lo[1] = c.y; s_lo[2] = c.z; s_lo[3] = c.w;
      s_hi[0] = d.x; s_hi[1] = d.y; s_hi[2] = d.z; s_hi[3] = d.w;
    }
#pragma unroll
    for (int i = 0; i < kRopeMaxRows; ++i) {
      const int hr = base + i * kSlots;
      if (hr >= rows) break;  // uniform over the row's lanes
      if (hr >= p.heads + p.kv_heads) {  // value head: copied as is
        if (slot_ok) {
          __nv_bfloat16* dst = p.value_pool + (slot * p.kv_heads + (hr - p.heads - p.kv_heads)) * D;
          *reinterpret_cast<uint2*>(dst + 4 * j) = lo[i];
          *reinterpret_cast<uint2*>(dst + kHalf + 4 * j) = hi[i];
        }
        continue;
      }
      const bool is_q = hr < p.heads;
      if (is_q ? (p.q_out == nullptr || !pos_ok) : (!slot_ok || !pos_ok)) continue;
      // Every rounding point yields bf16 values, kept packed (one cvt.bf16x2 per pair) and
      // unpacked only where fp32 arithmetic follows.
      uint2 ylo = lo[i], yhi = hi[i];
      const float* scale = is_q ? p.q_scale : p.k_scale;
      if (scale != nullptr) {
        const float4 ga = *reinterpret_cast<const float4*>(scale + 4 * j);
        const float4 gb = *reinterpret_cast<const float4*>(scale + kHalf + 4 * j);
        norm_lane<kLanes, D>(ylo, yhi, ga, gb, p.eps, row_mask);
      }
      if (p.cos != nullptr) rope_lane(ylo, yhi, c_lo, c_hi, s_lo, s_hi);
      __nv_bfloat16* dst = is_q ? p.q_out + (static_cast<int64_t>(t) * p.heads + hr) * D
                                : p.key_pool + (slot * p.kv_heads + (hr - p.heads)) * D;
      *reinterpret_cast<uint2*>(dst + 4 * j) = ylo;
      *reinterpret_cast<uint2*>(dst + kHalf + 4 * j) = yhi;
    }
  }
}

}  // namespace hb
