// Persistent tcgen05 GEMM main loop shared by the fused projections: out tile = epilogue(
// A[M, K] x B^T over a 128 x 256 accumulator in TMEM), with the epilogue a policy type.
//
// Persistent CTAs, one per SM (192 threads). A tile is 128 rows of A against 256 rows of the
// weight B [N_total, K], taken as two 128-row boxes whose first rows the epilogue names
// (b_row(tile_n, 0 / 1)): the gate|up GEMM stacks 128 gate rows over the matching 128 up
// rows, the greedy lm_head takes 256 consecutive vocabulary rows.
//   warp 0     TMA producer: per 64-wide K step, the [128 x 64] A tile and the two
//              [128 x 64] B boxes into a 4-stage ring of 48 KB stages (128B swizzle; rows
//              past M read as zeros);
//   warp 1     allocates 512 TMEM columns (two 256-column accumulators) and its lane 0
//              issues tcgen05.mma M128 N256 K16, four per K step, releasing each stage
//              with tcgen05.commit and handing each finished accumulator to the epilogue;
//   warps 2..  Epilogue::kEpilogueWarps epilogue warps (4, or 8 = two per TMEM lane
//              quadrant): Epilogue::run reads the accumulator rows of its quadrant while the
//              other accumulator is being filled by the next tile, then the accumulator is
//              handed back.
// Tiles are walked M-fastest, so the CTAs running at once share few weight tiles and the
// activations (read by every column of tiles) stay in L2. Every spin-wait is bounded.
//
// Epilogue policy interface:
//   using Params = ...;   // must hold int32_t m, k, tiles_m, tiles_n
//   static int b_row(const Params&, int tile_n, int half);        // first weight row of a box
//   static constexpr int kEpilogueWarps;      // 4 or 8
//   struct Prefetch;                          // what prefetch loads for run
//   static void prefetch(const Params&, int tile_m, int tile_n, const EpilogueWarp&, Prefetch&);
//                   // before the tile's accumulator is ready (overlaps its MMAs)
//   static bool run(const Params&, int tile_m, int tile_n, uint32_t acc, const EpilogueWarp& ew,
//                   const Prefetch&);
//                   // acc = TMEM address of column 0 of the quadrant's first row (lane
//                   // offset included); run by all 32 lanes together; false: give up
#pragma once

#include "hb_common.cuh"

namespace hb {

constexpr int kGemmTileM = 128;   // rows per tile (the MMA M)
constexpr int kGemmTileN = 128;   // rows of one B box (the MMA N is two boxes: 256)
constexpr int kGemmTileK = 64;    // K per stage: one 128-byte swizzled row
constexpr int kGemmStages = 4;
constexpr uint32_t kGemmABytes = kGemmTileM * kGemmTileK * 2;      // 16 KB
constexpr uint32_t kGemmBHalf = kGemmTileN * kGemmTileK * 2;       // 16 KB (one B box)
constexpr uint32_t kGemmStageBytes = kGemmABytes + 2 * kGemmBHalf;  // 48 KB
// Dynamic shared memory of one CTA: the stage ring plus 1 KB to align it to the 128-byte
// swizzle's 1024-byte period.
constexpr uint32_t kGemmSmemBytes = kGemmStages * kGemmStageBytes + 1024;
constexpr uint32_t kGemmAccCols = 2 * kGemmTileN;                  // 256 fp32 columns per accumulator

template <typename Epilogue>
constexpr int fused_gemm_threads() {
  return 64 + 32 * Epilogue::kEpilogueWarps;
}

// What one epilogue warp knows about itself. With 8 epilogue warps two warps share each TMEM
// lane quadrant (sub 0 and 1).
struct EpilogueWarp {
  int quad, sub, lane;  // TMEM lane quadrant (rows 32 quad ..), which of its warps, lane
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

template <typename Epilogue>
__global__ void __launch_bounds__(fused_gemm_threads<Epilogue>(), 1) fused_gemm_kernel(typename Epilogue::Params p,
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
      mbar_init(&acc_empty[b], 32 * Epilogue::kEpilogueWarps);
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
  pdl_wait();     // the setup above overlaps the kernel ahead; its outputs are read from here on
  pdl_trigger();  // every CTA is resident (grid <= SMs): the next kernel may launch and wait

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&amap);
      tma_prefetch_desc(&bmap);
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x) {
        const int m0 = (t % p.tiles_m) * kGemmTileM;
        const int b0 = Epilogue::b_row(p, t / p.tiles_m, 0), b1 = Epilogue::b_row(p, t / p.tiles_m, 1);
        for (int ks = 0; ks < k_steps; ++ks, ++it) {
          const int s = it % kGemmStages;
          if (it >= kGemmStages && !mbar_wait(&empty[s], ((it / kGemmStages) - 1) & 1, &abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * kGemmStageBytes;
          mbar_expect_tx(&full[s], kGemmStageBytes);
          tma_load_2d(st, &amap, &full[s], ks * kGemmTileK, m0);
          tma_load_2d(st + kGemmABytes, &bmap, &full[s], ks * kGemmTileK, b0);
          tma_load_2d(st + kGemmABytes + kGemmBHalf, &bmap, &full[s], ks * kGemmTileK, b1);
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
    // ------------------------------------------------------------ epilogue (warps 2..)
    const int quad = warp & 3;  // tcgen05.ld reaches TMEM lanes 32 (warp % 4) ..
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const EpilogueWarp ew{quad, (warp - 2) >> 2, lane};
    int lt = 0;
    typename Epilogue::Prefetch pre;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++lt) {
      const int buf = lt & 1;
      Epilogue::prefetch(p, t % p.tiles_m, t / p.tiles_m, ew, pre);  // overlaps the tile's MMAs
      if (!mbar_wait(&acc_full[buf], (lt >> 1) & 1, &abort_flag)) break;
      tc_fence_after();
      const bool ok = Epilogue::run(p, t % p.tiles_m, t / p.tiles_m, tmem + buf * kGemmAccCols + lane_base, ew, pre);
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
      if (!ok) break;
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
