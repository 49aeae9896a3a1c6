// Gate|up projection with the SwiGLU product in its epilogue, on tcgen05 tensor cores.
//
// Replaces, in FeedForward.forward (src/helios/runtime/qwen3/layers.py:26-27), the two
// projections gate(x) and up(x) and silu(gate) * up: out = bf16(bf16(silu(bf16(x Wg^T)))
// * bf16(x Wu^T)), with every rounding point of the reference kept (each projection
// output rounded to bf16, silu computed in fp32 from it and rounded, then the product).
// The gate|up activations never reach memory: the GEMM output tile goes from TMEM
// through the epilogue straight to the [M, I] SwiGLU output.
//
// An output tile is 128 rows x 128 SwiGLU columns, one M128 x N256 accumulator of the
// fused main loop whose B operand stacks the 128 gate rows n0.. over the matching 128 up
// rows I + n0.. of the fused [gate; up] weight [2I, K]. The epilogue thread of a row loads
// 32 gate and 32 up columns at a time, applies the rounding chain above and stores 64-byte
// row chunks.
#pragma once

#include "fused_gemm.cuh"

namespace hb {

struct GemmSwigluParams {
  int32_t m, k, tiles_m, tiles_n;
  __nv_bfloat16* out;  // [m, inter]
  int32_t inter;
};

struct SwigluEpilogue {
  using Params = GemmSwigluParams;
  static constexpr int kEpilogueWarps = 4;  // one per TMEM lane quadrant (8 measured no faster)
  struct Prefetch {};

  __device__ static int b_row(const Params& p, int tile_n, int half) {
    return half == 0 ? tile_n * kGemmTileN : p.inter + tile_n * kGemmTileN;
  }

  __device__ static void prefetch(const Params&, int, int, const EpilogueWarp&, Prefetch&) {}

  __device__ static bool run(const Params& p, int tile_m, int tile_n, uint32_t acc, const EpilogueWarp& ew, const Prefetch&) {
    const int row = tile_m * kGemmTileM + ew.quad * 32 + ew.lane;  // thread = row (TMEM lane)
    __nv_bfloat16* dst = p.out + static_cast<int64_t>(row) * p.inter + tile_n * kGemmTileN;
#pragma unroll 1
    for (int c = 0; c < kGemmTileN / 32; ++c) {
      float g[32], u[32];
      tmem_ld32(acc + c * 32, g);
      tmem_ld32(acc + kGemmTileN + c * 32, u);
      tmem_wait_ld();
      if (row < p.m) {
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float o[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            // gate and up as the projections return them (bf16), silu(gate) in fp32
            // rounded to bf16 (fast exp/divide: error far below that rounding), product.
            const float gb = __bfloat162float(__float2bfloat16_rn(g[2 * e + h]));
            const float ub = __bfloat162float(__float2bfloat16_rn(u[2 * e + h]));
            const float sl = __bfloat162float(__float2bfloat16_rn(__fdividef(gb, 1.f + __expf(-gb))));
            o[h] = __fmul_rn(sl, ub);
          }
          w[e] = pack_bf16(o[0], o[1]);
        }
        uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q) d4[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
      }
    }
    return true;
  }
};

}  // namespace hb
