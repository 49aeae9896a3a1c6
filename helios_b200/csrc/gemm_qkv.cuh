// q|k|v projection with the per-head q/k RMSNorm, RoPE and paged KV append in its epilogue,
// on tcgen05 tensor cores.
//
// Replaces, per decoder layer, the reference's chain
//   query(x), key(x), value(x)  (GroupedQueryAttention.forward,
//                                src/helios/runtime/qwen3/layers.py:132-146),
//   q_norm / k_norm             (RMSNorm.forward, layers.py:36-40),
//   apply_rope                  (layers.py:54-72, with position_ids),
//   _write                      (two index_copy_ into the pool, paged_cache.py:335-345)
// with one launch: the projection tile goes from TMEM through the epilogue to the rotated
// query rows and the pool pages; the [T, (H + 2 Hkv) d] projection output never reaches
// memory. The arithmetic is kernel (b)'s (norm_rope_append.cuh) with the same fp32 order:
// projection output rounded to bf16; norm bf16(fl(fl(x * inv) * scale)) with inv =
// rsqrt(mean(x^2) + eps), the sum of squares taken in kernel (b)'s order (sixteen partial
// sums of eight products, then its butterfly tree); RoPE fl(fl(n c) -/+ fl(rot(n) s)) rounded
// to bf16. Given the same projection values the rows are bit-identical to kernel (b)'s.
//
// A tile is 128 tokens x two heads (256 accumulator columns) of the fused main loop; the B
// boxes are weight rows 256 n .. 256 n + 255 of [Wq; Wk; Wv] (head_dim 128), so head row
// hr = 2 n + h sits at accumulator columns 128 h ..  Eight epilogue warps: warp (quad, h)
// takes head h for the 32 tokens of TMEM lane quadrant quad, thread = token, with the whole
// head row in registers (64 packed bf16 pairs): the norm needs no exchange and each RoPE
// partner (i, i + 64) is in the same thread. The tables come from hb_rope_gather as
// [w / 4][T][4] fp32 (token t's cos / sin row at its position, w = 64 when the tables'
// halves repeat, else 128), so the 32 threads of a warp read 512 contiguous bytes per load.
// Each thread writes its 256-byte row to q_out [T, H, 128] or to the pool slot
// write_slots[t] of key_pool / value_pool ([slots, Hkv, 128]). Bad slots or positions raise
// the device status and skip the row, as kernel (b) does.
#pragma once

#include "fused_gemm.cuh"
#include "norm_rope_append.cuh"

namespace hb {

constexpr int kQkvHeadDim = 128;

struct GemmQkvParams {
  int32_t m, k, tiles_m, tiles_n;
  int32_t heads, kv_heads;
  const float* q_scale;   // [128] or null: no norm
  const float* k_scale;   // [128] or null: no norm
  float eps;
  const float* rope_cos;  // [rope_width / 4][m][4] (hb_rope_gather) or null: no rotation
  const float* rope_sin;
  int32_t rope_width;     // 64: the tables' halves repeat; 128: full rows
  int64_t rope_rows;      // rows of the original tables (position check)
  const int64_t* positions;    // [m]
  const int64_t* write_slots;  // [m]
  __nv_bfloat16* q_out;        // [m, heads, 128]
  __nv_bfloat16* key_pool;     // [pool_slots, kv_heads, 128]
  __nv_bfloat16* value_pool;
  int64_t pool_slots;
};

struct QkvEpilogue {
  using Params = GemmQkvParams;
  static constexpr int D = kQkvHeadDim, kHalf = D / 2;
  static constexpr int kEpilogueWarps = 8;

  struct Prefetch {
    bool live, slot_ok, pos_ok;
    int64_t slot;
  };

  __device__ static int b_row(const Params&, int tile_n, int half) {
    return tile_n * (2 * kQkvHeadDim) + half * kQkvHeadDim;
  }

  // The token's write slot and position check, loaded while the tile's MMAs run.
  __device__ static void prefetch(const Params& p, int tile_m, int tile_n, const EpilogueWarp& ew, Prefetch& f) {
    const int row = tile_m * kGemmTileM + ew.quad * 32 + ew.lane;
    f.live = row < p.m;
    f.slot = -1;
    f.slot_ok = f.pos_ok = false;
    if (!f.live) return;
    f.slot = p.write_slots[row];
    f.slot_ok = f.slot >= 0 && f.slot < p.pool_slots;
    if (p.rope_cos != nullptr) {
      const int64_t pos = p.positions[row];
      f.pos_ok = pos >= 0 && pos < p.rope_rows;
    } else {
      f.pos_ok = true;
    }
    if (tile_n == 0 && ew.sub == 0) {  // report once per token
      if (!f.slot_ok) raise_status(kStatusBadSlot);
      if (!f.pos_ok) raise_status(kStatusBadPosition);
    }
  }

  __device__ static bool run(const Params& p, int tile_m, int tile_n, uint32_t acc, const EpilogueWarp& ew,
                             const Prefetch& f) {
    const int h = ew.sub;  // this warp's head of the tile
    const int hr = tile_n * 2 + h;
    const int row = tile_m * kGemmTileM + ew.quad * 32 + ew.lane;
    const uint32_t base = acc + h * D;
    const bool is_v = hr >= p.heads + p.kv_heads, is_q = hr < p.heads;
    // Columns in the order kernel (b)'s lanes hold them: chunk pairs (0..31, 64..95) then
    // (32..63, 96..127), so partial sums j = 0..7 then 8..15 complete one pair at a time.
    uint32_t w[D / 2];  // the head row as the projection returns it: bf16 pairs (2i, 2i + 1)
    float part[16];     // kernel (b)'s per-lane sums: elements 4j..4j+3 then 64+4j..64+4j+3
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float lo[32], hi[32];
      tmem_ld32(base + 32 * c, lo);
      tmem_ld32(base + kHalf + 32 * c, hi);
      tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        w[16 * c + e] = pack_bf16(lo[2 * e], lo[2 * e + 1]);
        w[kHalf / 2 + 16 * c + e] = pack_bf16(hi[2 * e], hi[2 * e + 1]);
      }
      if (!is_v) {
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          float a[4], b[4];
          unpack4(make_uint2(w[16 * c + 2 * jj], w[16 * c + 2 * jj + 1]), a);
          unpack4(make_uint2(w[kHalf / 2 + 16 * c + 2 * jj], w[kHalf / 2 + 16 * c + 2 * jj + 1]), b);
          float ss = 0.f;
#pragma unroll
          for (int e = 0; e < 4; ++e) ss = __fmaf_rn(a[e], a[e], ss);
#pragma unroll
          for (int e = 0; e < 4; ++e) ss = __fmaf_rn(b[e], b[e], ss);
          part[8 * c + jj] = ss;
        }
      }
    }
    if (!f.live) return true;
    __nv_bfloat16* dst;
    if (is_v) {  // value head: appended as is
      if (!f.slot_ok) return true;
      dst = p.value_pool + (f.slot * p.kv_heads + (hr - p.heads - p.kv_heads)) * D;
    } else {
      if (!f.pos_ok || (!is_q && !f.slot_ok)) return true;
      const float* scale = is_q ? p.q_scale : p.k_scale;
      if (scale != nullptr) {
        // Kernel (b)'s butterfly over its 16 lanes (xor 8, 4, 2, 1), as lane 0 adds.
        float t1[8], t2[4];
#pragma unroll
        for (int j = 0; j < 8; ++j) t1[j] = part[j] + part[j + 8];
#pragma unroll
        for (int j = 0; j < 4; ++j) t2[j] = t1[j] + t1[j + 4];
        const float ss = (t2[0] + t2[2]) + (t2[1] + t2[3]);
        const float inv = rsqrtf(__fadd_rn(ss * (1.f / static_cast<float>(D)), p.eps));
#pragma unroll
        for (int i = 0; i < D / 4; ++i) {
          const float4 g = *reinterpret_cast<const float4*>(scale + 4 * i);  // same for every thread
          float x[4];
          unpack4(make_uint2(w[2 * i], w[2 * i + 1]), x);
          w[2 * i] = pack_bf16(__fmul_rn(__fmul_rn(x[0], inv), g.x), __fmul_rn(__fmul_rn(x[1], inv), g.y));
          w[2 * i + 1] = pack_bf16(__fmul_rn(__fmul_rn(x[2], inv), g.z), __fmul_rn(__fmul_rn(x[3], inv), g.w));
        }
      }
      if (p.rope_cos != nullptr) {
        const int64_t tok_stride = static_cast<int64_t>(p.m) * 4;
        const float* cr = p.rope_cos + static_cast<int64_t>(row) * 4;
        const float* sr = p.rope_sin + static_cast<int64_t>(row) * 4;
        const int hi_group = p.rope_width == D ? kHalf / 4 : 0;  // where element 64 + i's value sits
#pragma unroll
        for (int g = 0; g < kHalf / 4; ++g) {  // elements 4g..4g+3 and their partners 64+4g..
          const float4 cl = *reinterpret_cast<const float4*>(cr + g * tok_stride);
          const float4 sl = *reinterpret_cast<const float4*>(sr + g * tok_stride);
          const float4 ch = *reinterpret_cast<const float4*>(cr + (g + hi_group) * tok_stride);
          const float4 sh = *reinterpret_cast<const float4*>(sr + (g + hi_group) * tok_stride);
          uint2 ylo = make_uint2(w[2 * g], w[2 * g + 1]);
          uint2 yhi = make_uint2(w[kHalf / 2 + 2 * g], w[kHalf / 2 + 2 * g + 1]);
          rope_lane(ylo, yhi, cl, ch, sl, sh);
          w[2 * g] = ylo.x;
          w[2 * g + 1] = ylo.y;
          w[kHalf / 2 + 2 * g] = yhi.x;
          w[kHalf / 2 + 2 * g + 1] = yhi.y;
        }
      }
      dst = is_q ? p.q_out + (static_cast<int64_t>(row) * p.heads + hr) * D
                 : p.key_pool + (f.slot * p.kv_heads + (hr - p.heads)) * D;
    }
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int q = 0; q < D / 8; ++q) d4[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    return true;
  }
};

// Per-token rope rows for the fused q|k|v epilogue: out[g][t][0..3] = table[positions[t]][4g ..
// 4g + 3] for g < width / 4, for cos and sin (zeros where the position is outside the
// tables). One thread per (g, t), t fastest, so the writes are contiguous.
struct RopeGatherParams {
  const float* cos;
  const float* sin;
  int64_t rope_rows;
  const int64_t* positions;
  int32_t tokens, width;
  float* out_cos;
  float* out_sin;
};

__global__ void __launch_bounds__(256) rope_gather_kernel(RopeGatherParams p) {
  pdl_wait();
  pdl_trigger();
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int groups = p.width / 4;
  if (idx >= static_cast<int64_t>(groups) * p.tokens) return;
  const int g = static_cast<int>(idx / p.tokens), t = static_cast<int>(idx % p.tokens);
  const int64_t pos = p.positions[t];
  float4 c = make_float4(0.f, 0.f, 0.f, 0.f), s = c;
  if (pos >= 0 && pos < p.rope_rows) {
    c = *reinterpret_cast<const float4*>(p.cos + pos * kQkvHeadDim + 4 * g);
    s = *reinterpret_cast<const float4*>(p.sin + pos * kQkvHeadDim + 4 * g);
  }
  reinterpret_cast<float4*>(p.out_cos)[idx] = c;
  reinterpret_cast<float4*>(p.out_sin)[idx] = s;
}

}  // namespace hb
