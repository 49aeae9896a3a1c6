// Greedy decoding head: the tied lm_head projection of the logit rows with the argmax in its
// epilogue, on tcgen05 tensor cores.
//
// Replaces, for rows sampled at temperature 0, the logits GEMM of Qwen3Model._forward_packed
// (src/helios/runtime/qwen3/model.py:108-110, output(norm(rows))) followed by the argmax of
// Decoder._sample (src/helios/runtime/qwen3/decode.py:458-460) and the batched sampling of
// Engine._execute_batch (src/helios/runtime/engine.py:472-473). The [rows, vocab] logits never
// reach memory.
//
// Each output tile of the fused main loop is 128 rows x 256 vocabulary columns (two 128-row
// boxes of the weight; rows past the vocabulary read as zeros and are skipped). The epilogue
// thread of a row rounds each logit to bf16 (the logits the reference takes the argmax of),
// keeps the first largest column of its 256, and folds it into the row's 64-bit key
// (ordered bf16 value << 32 | (2^32 - 1 - column)) with one atomicMax: the largest value wins
// and equal values go to the lowest column, as torch.argmax does. A NaN logit orders above
// every number (the reductions propagate NaN). argmax_finalize_kernel turns the keys into token
// ids and zeroes them for the next call.
#pragma once

#include "fused_gemm.cuh"

namespace hb {

struct GemmArgmaxParams {
  int32_t m, k, tiles_m, tiles_n;
  int32_t vocab;
  unsigned long long* best;  // [m] packed keys (above); zero before the call
};

// Unsigned order key of a float: larger float -> larger key; both zeros map to one key; NaN on top.
__device__ __forceinline__ uint32_t float_order_key(float v) {
  if (v != v) return 0xffffffffu;
  const uint32_t b = __float_as_uint(v == 0.f ? 0.f : v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

struct ArgmaxEpilogue {
  using Params = GemmArgmaxParams;
  static constexpr int kEpilogueWarps = 4;
  struct Prefetch {};

  __device__ static int b_row(const Params&, int tile_n, int half) { return (2 * tile_n + half) * kGemmTileN; }

  __device__ static void prefetch(const Params&, int, int, const EpilogueWarp&, Prefetch&) {}

  __device__ static bool run(const Params& p, int tile_m, int tile_n, uint32_t acc, const EpilogueWarp& ew, const Prefetch&) {
    const int row = tile_m * kGemmTileM + ew.quad * 32 + ew.lane;  // thread = row (TMEM lane)
    const int col0 = tile_n * 2 * kGemmTileN;
    const int ncols = min(2 * kGemmTileN, p.vocab - col0);
    uint32_t best_key = 0;
    int best_col = -1;
#pragma unroll 1
    for (int c = 0; c < 2 * kGemmTileN / 32; ++c) {
      float v[32];
      tmem_ld32(acc + c * 32, v);  // warp-collective: every lane loads, whatever its row
      tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int col = c * 32 + e;
        const uint32_t key = float_order_key(__bfloat162float(__float2bfloat16_rn(v[e])));
        if (col < ncols && (best_col < 0 || key > best_key)) {  // strict: the first of equals stays
          best_key = key;
          best_col = col;
        }
      }
    }
    if (row < p.m && best_col >= 0) {
      const unsigned long long packed = (static_cast<unsigned long long>(best_key) << 32) |
                                        static_cast<unsigned long long>(0xffffffffu - static_cast<uint32_t>(col0 + best_col));
      atomicMax(p.best + row, packed);
    }
    return true;
  }
};

// Token ids from the packed keys (-1 for a row the GEMM recorded nothing for, which only a
// kernel that gave up leaves); every key is left at zero for the next call.
__global__ void argmax_finalize_kernel(unsigned long long* best, int32_t m, int64_t* out_ids) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= m) return;
  const unsigned long long key = best[r];  // a recorded key is never zero (its value word is not)
  out_ids[r] = key == 0ull ? -1 : static_cast<int64_t>(0xffffffffu - static_cast<uint32_t>(key & 0xffffffffull));
  best[r] = 0ull;
}

}  // namespace hb
