// Gate|up projection with the SwiGLU product in its epilogue, on tcgen05 tensor cores.
//
// Replaces, in FeedForward.forward (src/helios/runtime/qwen3/layers.py:26-27), the two
// projections gate(x) and up(x) and silu(gate) * up: out = bf16(bf16(silu(bf16(x Wg^T)))
// * bf16(x Wu^T)), with every rounding point of the reference kept (each projection
// output rounded to bf16, silu computed in fp32 from it and rounded, then the product).
// The gate|up activations never reach memory: the GEMM output tile goes from TMEM
// through the epilogue straight to the [M, I] SwiGLU output.
//
// Persistent CTAs, one per SM (192 threads). An output tile is 128 rows x 128 SwiGLU
// columns, computed as one M128 x N256 accumulator whose B operand stacks the 128 gate
// rows over the matching 128 up rows of the fused [gate; up] weight [2I, K]:
//   warp 0     TMA producer: per 64-wide K step, the [128 x 64] A tile and the two
//              [128 x 64] B tiles (gate rows n0.., up rows I+n0..) into a 4-stage ring of
//              48 KB stages (128B swizzle; rows past M read as zeros);
//   warp 1     allocates 512 TMEM columns (two 256-column accumulators) and its lane 0
//              issues tcgen05.mma M128 N256 K16, four per K step, releasing each stage
//              with tcgen05.commit and handing each finished accumulator to the epilogue;
//   warps 2-5  epilogue, thread = output row (TMEM lane): loads 32 gate and 32 up columns
//              at a time, applies the rounding chain above and stores 64-byte row chunks;
//              the other accumulator is being filled by the next tile meanwhile.
// Tiles are walked M-fastest, so the CTAs running at once share few weight tiles and the
// activations (read by every column of tiles) stay in L2. Every spin-wait is bounded.
#pragma once

#include "hb_common.cuh"

namespace hb {

constexpr int kGemmTileM = 128;   // rows per tile (the MMA M)
constexpr int kGemmTileN = 128;   // SwiGLU columns per tile (the MMA N is 2x: gate | up)
constexpr int kGemmTileK = 64;    // K per stage: one 128-byte swizzled row
constexpr int kGemmStages = 4;
constexpr int kGemmThreads = 192;
constexpr uint32_t kGemmABytes = kGemmTileM * kGemmTileK * 2;      // 16 KB
constexpr uint32_t kGemmBHalf = kGemmTileN * kGemmTileK * 2;       // 16 KB (gate or up rows)
constexpr uint32_t kGemmStageBytes = kGemmABytes + 2 * kGemmBHalf;  // 48 KB
constexpr uint32_t kGemmSmemBytes = kGemmStages * kGemmStageBytes + 1024;
constexpr uint32_t kGemmAccCols = 2 * kGemmTileN;                  // 256 fp32 columns per accumulator

struct GemmSwigluParams {
  __nv_bfloat16* out;  // [m, inter]
  int32_t m, inter, k;
  int32_t tiles_m, tiles_n;
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__global__ void __launch_bounds__(kGemmThreads, 1) gemm_swiglu_kernel(GemmSwigluParams p,
                                                                     const __grid_constant__ CUtensorMap amap,
                                                                     const __grid_constant__ CUtensorMap bmap) {
  extern __shared__ __align__(1024) uint8_t dsm[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full[kGemmStages], empty[kGemmStages], acc_full[2], acc_empty[2], drain_bar;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_tiles = p.tiles_m * p.tiles_n;
  const int k_steps = p.k / kGemmTileK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemmStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_s, 2 * kGemmAccCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&amap);
      tma_prefetch_desc(&bmap);
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
        const int m0 = (t % p.tiles_m) * kGemmTileM, n0 = (t / p.tiles_m) * kGemmTileN;
        for (int ks = 0; ks < k_steps; ++ks, ++it) {
          const int s = it % kGemmStages;
          if (it >= kGemmStages && !mbar_wait(&empty[s], ((it / kGemmStages) - 1) & 1, &abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * kGemmStageBytes;
          mbar_expect_tx(&full[s], kGemmStageBytes);
          tma_load_2d(st, &amap, &full[s], ks * kGemmTileK, m0);
          tma_load_2d(st + kGemmABytes, &bmap, &full[s], ks * kGemmTileK, n0);
          tma_load_2d(st + kGemmABytes + kGemmBHalf, &bmap, &full[s], ks * kGemmTileK, p.inter + n0);
        }
      }
      // Never leave with copies in flight: the last stages issued complete (bounded).
      for (int j = max(0, it - kGemmStages); j < it; ++j) mbar_drain(&full[j % kGemmStages], (j / kGemmStages) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(kGemmTileM, kGemmAccCols, false, false);
      const uint64_t desc0 = smem_desc(smem_u32(smem), 16, 1024, kSwizzle128B);
      int it = 0, lt = 0;
      bool ok = true, issued = false;
      for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x, ++lt) {
        const int buf = lt & 1;
        if (lt >= 2 && !mbar_wait(&acc_empty[buf], ((lt >> 1) - 1) & 1, &abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * kGemmAccCols;
        for (int ks = 0; ks < k_steps; ++ks, ++it) {
          const int s = it % kGemmStages;
          if (!mbar_wait(&full[s], (it / kGemmStages) & 1, &abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t a = desc0 + static_cast<uint64_t>((s * kGemmStageBytes) >> 4);
          const uint64_t b = a + static_cast<uint64_t>(kGemmABytes >> 4);
#pragma unroll
          for (int kk = 0; kk < kGemmTileK / 16; ++kk)  // 32 bytes of K per MMA
            mma_ss(d, a + 2 * kk, b + 2 * kk, idesc, (ks > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&empty[s]);  // the stage is free once these MMAs have read it
          issued = true;
        }
        if (ok) mma_commit(&acc_full[buf]);
      }
      if (issued) {  // nothing may still write TMEM when it is freed
        mma_commit(&drain_bar);
        mbar_drain(&drain_bar, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2-5)
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // TMEM lane == tile row
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    int lt = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++lt) {
      const int buf = lt & 1;
      if (!mbar_wait(&acc_full[buf], (lt >> 1) & 1, &abort_flag)) break;
      tc_fence_after();
      const int row = (t % p.tiles_m) * kGemmTileM + r;
      const int n0 = (t / p.tiles_m) * kGemmTileN;
      const uint32_t acc = tmem + buf * kGemmAccCols + lane_base;
      __nv_bfloat16* dst = p.out + static_cast<int64_t>(row) * p.inter + n0;
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
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * kGemmAccCols);
  }
}

}  // namespace hb
