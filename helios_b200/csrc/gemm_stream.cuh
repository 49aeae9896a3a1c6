// Weight-streaming GEMM for decode ticks: out[m][n] = sum_k x[m][k] * w[n][k] with few token
// rows (m <= 256) and a large weight, on tcgen05 tensor cores.
//
// Replaces, at decode-tick sizes, the projections of GroupedQueryAttention.forward
// (q|k|v and output, src/helios/runtime/qwen3/layers.py:131-146, :163-164) and of
// FeedForward.forward (gate|up and down, layers.py:26-27), which the reference runs as
// nn.Linear calls. With m <= 256 a GEMM is a stream over the weight (202 MB per Qwen3-4B layer,
// ~31 us at the copy peak): the work must spread over every SM and keep enough weight bytes in
// flight on each, whatever the weight's shape. A tiled GEMM with one CTA per 128-column output
// tile leaves most SMs idle on the 2560-column projections (20 tiles).
//
// So the weight is the MMA's A operand (128 weight rows = M) and the token rows its B operand
// (N = m rounded up to 32), and the work is split stream-K style: the (tile, 64-wide K step)
// sequence of the whole GEMM is cut into one equal contiguous range per CTA (persistent, one
// CTA per SM). A CTA accumulates each tile's part of its range in TMEM. A tile whose K range
// one CTA covers is written out directly; a tile split between CTAs has each part written as
// fp32 partials to the workspace, and the CTA that finishes the tile's last part (a per-tile
// arrival counter) adds the parts in part order, so the sum does not depend on which CTA
// finished first, writes the bf16 output and resets the counter to zero for the next call.
// Roles (192 threads):
//   warp 0     TMA producer: per K step the [128 x 64] weight box and the [n_pad x 64] token
//              box into a ring of stages (128B swizzle; token rows past m read as zeros);
//   warp 1     allocates 2 x n_pad TMEM columns (two accumulators) and its lane 0 issues
//              tcgen05.mma M128 N n_pad K16, four per K step;
//   warps 2-5  epilogue, thread = weight row (TMEM lane): the output or the partials of its
//              row, 32 token columns per tcgen05.ld.
// Every spin-wait is bounded.
#pragma once

#include "fused_gemm.cuh"  // tma_load_2d

namespace hb {

constexpr int kStreamTileRows = 128;  // weight rows per tile (the MMA M)
constexpr int kStreamTileK = 64;      // K per stage: one 128-byte swizzled row
constexpr int kStreamMaxTokens = 256;  // token rows (the MMA N: m rounded up to 32)
constexpr int kStreamThreads = 192;
constexpr uint32_t kStreamABytes = kStreamTileRows * kStreamTileK * 2;  // 16 KB
constexpr uint32_t kStreamSmemBudget = 200 * 1024;
constexpr int kStreamMaxStages = 8;
constexpr size_t kStreamCounterBytes = 4096;  // per-tile arrival counters ahead of the partials

struct StreamGemmParams {
  int32_t m, n_pad, n, k;         // token rows, MMA N (m rounded up to 32), weight rows, inner size
  int32_t tiles, ksteps, per_cta;  // n / 128, k / 64, (tile, K step) units per CTA
  int32_t stages;                  // ring stages
  int32_t max_parts;               // partial slots per tile in the workspace
  __nv_bfloat16* out;              // [m][n]
  int32_t* counters;               // [tiles], zero between calls
  float* partials;                 // [tiles][max_parts][128][n_pad]
};

__host__ __device__ inline uint32_t stream_stage_bytes(int n_pad) {
  return kStreamABytes + static_cast<uint32_t>(n_pad) * kStreamTileK * 2;
}

// First CTA whose range covers unit u.
__device__ __forceinline__ int stream_owner(const StreamGemmParams& p, int u) { return u / p.per_cta; }

__global__ void __launch_bounds__(kStreamThreads, 1) stream_gemm_kernel(StreamGemmParams p,
                                                                         const __grid_constant__ CUtensorMap wmap,
                                                                         const __grid_constant__ CUtensorMap xmap) {
  extern __shared__ __align__(1024) uint8_t dsm[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full[kStreamMaxStages], empty[kStreamMaxStages], acc_full[2], acc_empty[2], drain_bar;
  __shared__ uint64_t parts_written, decided;  // split tiles: all partials stored; last-arrival known
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_flag, last_arrival;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t stage_bytes = stream_stage_bytes(p.n_pad);
  const int total = p.tiles * p.ksteps;
  const int begin = blockIdx.x * p.per_cta;
  const int end = min(total, begin + p.per_cta);
  // Accumulator columns: n_pad rounded up to a power of two (TMEM allocations are).
  const uint32_t acc_cols = p.n_pad <= 32 ? 32u : p.n_pad <= 64 ? 64u : p.n_pad <= 128 ? 128u : 256u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(&drain_bar, 1);
    mbar_init(&parts_written, 128);
    mbar_init(&decided, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_s, 2 * acc_cols);
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
      tma_prefetch_desc(&wmap);
      tma_prefetch_desc(&xmap);
      int it = 0;
      for (int u = begin; u < end; ++u, ++it) {
        const int s = it % p.stages;
        if (it >= p.stages && !mbar_wait(&empty[s], ((it / p.stages) - 1) & 1, &abort_flag)) break;
        const int tile = u / p.ksteps, ks = u % p.ksteps;
        uint8_t* st = smem + s * stage_bytes;
        mbar_expect_tx(&full[s], stage_bytes);
        tma_load_2d(st, &wmap, &full[s], ks * kStreamTileK, tile * kStreamTileRows);
        tma_load_2d(st + kStreamABytes, &xmap, &full[s], ks * kStreamTileK, 0);
      }
      // Never leave with copies in flight: the last stages issued complete (bounded).
      for (int j = max(0, it - p.stages); j < it; ++j) mbar_drain(&full[j % p.stages], (j / p.stages) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(kStreamTileRows, p.n_pad, false, false);
      const uint64_t desc0 = smem_desc(smem_u32(smem), 16, 1024, kSwizzle128B);
      int it = 0, seg = 0;
      bool ok = true, issued = false;
      for (int u = begin; ok && u < end; ++seg) {
        const int tile = u / p.ksteps;
        const int seg_end = min(end, (tile + 1) * p.ksteps);
        const int buf = seg & 1;
        if (seg >= 2 && !mbar_wait(&acc_empty[buf], ((seg >> 1) - 1) & 1, &abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * acc_cols;
        for (int first = u; u < seg_end; ++u, ++it) {
          const int s = it % p.stages;
          if (!mbar_wait(&full[s], (it / p.stages) & 1, &abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t a = desc0 + static_cast<uint64_t>((s * stage_bytes) >> 4);
          const uint64_t b = a + static_cast<uint64_t>(kStreamABytes >> 4);
#pragma unroll
          for (int kk = 0; kk < kStreamTileK / 16; ++kk)  // 32 bytes of K per MMA
            mma_ss(d, a + 2 * kk, b + 2 * kk, idesc, (u > first || kk > 0) ? 1u : 0u);
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
    const int quad = warp & 3;  // tcgen05.ld reaches TMEM lanes 32 (warp % 4) ..
    const int r = quad * 32 + lane;  // weight row within the tile
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const int et = threadIdx.x - 64;  // 0..127
    int seg = 0, splits = 0;
    for (int u = begin; u < end; ++seg) {
      const int tile = u / p.ksteps;
      const int seg_end = min(end, (tile + 1) * p.ksteps);
      const int buf = seg & 1;
      // Parts of this tile: one per CTA whose range meets it, in CTA order.
      const int first_owner = stream_owner(p, tile * p.ksteps);
      const int last_owner = stream_owner(p, (tile + 1) * p.ksteps - 1);
      const int parts = last_owner - first_owner + 1;
      const int part = blockIdx.x - first_owner;
      if (!mbar_wait(&acc_full[buf], (seg >> 1) & 1, &abort_flag)) break;
      tc_fence_after();
      const uint32_t acc = tmem + buf * acc_cols + lane_base;
      const int col = tile * kStreamTileRows + r;  // output column
      if (parts == 1) {
#pragma unroll 1
        for (int c = 0; c < p.n_pad; c += 32) {
          float v[32];
          tmem_ld32(acc + c, v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (c + j < p.m) p.out[static_cast<int64_t>(c + j) * p.n + col] = __float2bfloat16_rn(v[j]);
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[buf]);
      } else {
        // Partials of this part, [128 rows][n_pad]: a thread writes and reads its row's values
        // as 16-byte vectors.
        const int64_t part_floats = static_cast<int64_t>(kStreamTileRows) * p.n_pad;
        float* mine = p.partials + (static_cast<int64_t>(tile) * p.max_parts + part) * part_floats + r * p.n_pad;
#pragma unroll 1
        for (int c = 0; c < p.n_pad; c += 32) {
          float v[32];
          tmem_ld32(acc + c, v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            __stcg(reinterpret_cast<float4*>(mine + c + j), make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[buf]);  // the accumulator is free: the parts are in memory
        // All 128 rows stored (bounded mbarrier waits, never an unbounded bar.sync), then one
        // thread counts this part in and tells the others whether it was the tile's last.
        __threadfence();
        mbar_arrive(&parts_written);
        if (et == 0) {
          const bool stored = mbar_wait(&parts_written, splits & 1, &abort_flag);
          last_arrival = stored && atomicAdd(p.counters + tile, 1) == parts - 1;
          mbar_arrive(&decided);
        }
        if (!mbar_wait(&decided, splits & 1, &abort_flag)) break;
        ++splits;
        if (last_arrival) {
          // The tile's last part: add every part in part order, write bf16, reset the counter.
          __threadfence();
          const float* row = p.partials + static_cast<int64_t>(tile) * p.max_parts * part_floats + r * p.n_pad;
#pragma unroll 1
          for (int j = 0; j < p.m; j += 4) {
            float4 sum = __ldcg(reinterpret_cast<const float4*>(row + j));
            for (int q = 1; q < parts; ++q) {
              const float4 v = __ldcg(reinterpret_cast<const float4*>(row + q * part_floats + j));
              sum.x += v.x;
              sum.y += v.y;
              sum.z += v.z;
              sum.w += v.w;
            }
            const float o[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
            for (int e = 0; e < 4; ++e)
              if (j + e < p.m) p.out[static_cast<int64_t>(j + e) * p.n + col] = __float2bfloat16_rn(o[e]);
          }
          if (et == 0) p.counters[tile] = 0;
        }
      }
      u = seg_end;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * acc_cols);
  }
}

}  // namespace hb
