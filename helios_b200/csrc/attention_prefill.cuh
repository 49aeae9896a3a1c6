// Kernel (c), prefill rows: causal paged GQA attention on tcgen05 tensor cores.
//
// Replaces the prefill-chunk part of the reference's paged varlen attention
// (PackedBatchCache.attend -> varlen_attn with block_table/seqused_k and
// window_size=(-1, 0), src/helios/runtime/qwen3/paged_cache.py:501-520).
//
// One CTA owns two query tiles of 128 rows each; a tile is (128 / GROUP)
// consecutive tokens of one sequence x the GROUP query heads that share KV head h.
// The two tiles are adjacent (2i and 2i+1 of a row), so they need the same key
// tiles (at most one more for the second), both stay busy for the CTA's whole
// life, and every K/V tile is read once for both. Keys go in steps of 128, so
// every tcgen05.mma is M128 x N128 x K16 (full rate) and each barrier handoff of
// the MMA thread is paid once per 128 keys. Roles (576 threads):
//   warp 0     TMA producer: both Q tiles once, then 128-key K and V tiles (four
//              128B-swizzled [64 keys][64 d] boxes each, each 64-key half from the
//              page the block table names) into 2-stage K and V rings;
//   warp 1     owns the TMEM allocation (512 columns: the S/P buffer of tile t at
//              128 t, its O accumulator at 256 + 128 t) and runs the issue loop as a
//              converged warp, one elected lane issuing S_t = Q_t K^T (both
//              operands in shared memory) and O_t += P_t V (P
//              read from TMEM, where the softmax wrote it over S_t), in a fixed
//              order with blocking waits: PV_0(j), S_0(j+1), PV_1(j), S_1(j+1). So
//              the tensor core computes one tile's P V and next S while the
//              softmax warps work on the other tile;
//   warps 2-9  softmax for tile 0, warps 10-17 for tile 1: the two warps of a
//              TMEM lane quadrant split the 128 key columns of each accumulator
//              row (thread = row, so no shuffles); they swap their half-row maxima
//              through shared memory (an mbarrier per row pair, so the wait is
//              bounded) and their row sums once at the end; each warp rescales and
//              writes its 64 of the 128 output columns. A quarter of the exponentials
//              run on the FMA pipe (exp2_fma2) beside the ex2 unit.
// O is rescaled (in TMEM) only when a row's running max grows by more than 2^8;
// exponents stay relative to the max in use, so P <= 2^8 and the final O / l is
// unchanged. Keys at or beyond seqused_k get their V rows zeroed so stale pool
// memory cannot reach the accumulator. The longest pairs (the last of a row) of
// every KV head are launched first.
#pragma once

#include "hb_common.cuh"
#include "attention_decode.cuh"

namespace hb {

constexpr int kPreRows = 128;     // rows per query tile
constexpr int kPreTiles = 2;      // query tiles per CTA
constexpr int kPreKeys = 128;     // keys per K/V tile (the N of S = Q K^T)
constexpr int kPreBoxKeys = 64;   // keys per TMA box (the box of the shared K/V tensor maps)
constexpr int kPreKStages = 2;
constexpr int kPreVStages = 2;
constexpr int kPreSoftmaxWarps = 8;  // per query tile: two warps per TMEM lane quadrant
constexpr int kPreSoftmaxThreads = kPreSoftmaxWarps * 32;
constexpr int kPreThreads = 64 + kPreTiles * kPreSoftmaxThreads;  // TMA warp, MMA warp, softmax
constexpr uint32_t kPreQBytes = kPreRows * 128 * 2;    // [128 rows][128 d] as two [128][64] d-halves
constexpr uint32_t kPreKVBytes = kPreKeys * 128 * 2;   // [128 keys][128 d] as two [128][64] d-halves
constexpr uint32_t kPreKVHalf = kPreKVBytes / 2;       // one d-half: [128 keys][64 d], 128 B rows
constexpr uint32_t kPreBoxBytes = kPreBoxKeys * 64 * 2;  // one TMA box: [64 keys][64 d]
constexpr uint32_t kPreSmemBytes = kPreTiles * kPreQBytes + (kPreKStages + kPreVStages) * kPreKVBytes + 1024;
// TMEM columns: S/P buffer of tile t at 128 t (S as fp32, then P as bf16 pairs over
// its first 64 columns once S has been read), O_t at 256 + 128 t.
constexpr uint32_t kPreTmemCols = 512;
constexpr uint32_t kPreTmemO = 256;
constexpr float kRescaleThreshold = 8.f;  // log2 units: rescale O when the max grows by more than 2^8

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Two fp32 fused multiply-adds in one instruction (sm_100 f32x2: two lanes of work per issue
// slot), d = a * b + c elementwise.
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                     float c1) {
  asm("{.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rd;}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

// 2^x for a pair of x <= 0 on the FMA pipe, beside the ex2 unit: x = n + f with n = round(x)
// (the 1.5 * 2^23 shifter) and f in [-0.5, 0.5]; 2^f from a cubic fitted here by weighted least
// squares (relative error 1.4e-4, far below P's bf16 rounding of 2^-9), then n added into the
// exponent field. x is clamped at -126 so the result stays a non-negative finite number: below it
// the result is ~2^-126 where ex2 gives 0, which P's bf16 rounding and the row sums ignore.
__device__ __forceinline__ void exp2_fma2(float& e0, float& e1, float x0, float x1) {
  constexpr float kShift = 12582912.f;
  constexpr float c0 = 0.99993980f, c1 = 0.69318938f, c2 = 0.24239314f, c3 = 0.05546971f;
  x0 = fmaxf(x0, -126.f);
  x1 = fmaxf(x1, -126.f);
  float t0, t1, n0, n1, f0, f1, p0, p1;
  fma2(t0, t1, x0, x1, 1.f, 1.f, kShift, kShift);     // t = x + shift: n in the low mantissa bits
  fma2(n0, n1, t0, t1, 1.f, 1.f, -kShift, -kShift);   // n = t - shift, exact
  fma2(f0, f1, n0, n1, -1.f, -1.f, x0, x1);           // f = x - n, exact
  fma2(p0, p1, f0, f1, c3, c3, c2, c2);
  fma2(p0, p1, p0, p1, f0, f1, c1, c1);
  fma2(p0, p1, p0, p1, f0, f1, c0, c0);
  e0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  e1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}

// Three-input maximum (sm_100): half the instructions of a two-input reduction.
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// PREFIX = false: prefill items, causal over each row's keys, bf16 output.
// PREFIX = true: prefix items (see AttentionParams::prefix_items): the query tiles hold the
// single tokens of consecutive rows that share their leading pages, every key of the item's
// split of those pages is visible to all of them (they sit past the shared keys), and each
// query row's (normalised output, log2-sum-exp) goes to its row's split record for the
// combine, beside the row's own decode splits.
template <int GROUP, bool PREFIX>
__global__ void __launch_bounds__(kPreThreads, 1) prefill_attention_kernel(AttentionParams p,
                                                                          const __grid_constant__ CUtensorMap qmap,
                                                                          const __grid_constant__ CUtensorMap kmap,
                                                                          const __grid_constant__ CUtensorMap vmap) {
  constexpr int D = 128;
  constexpr int kTileTokens = kPreRows / GROUP;
  extern __shared__ __align__(1024) uint8_t dsm[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = smem;                                   // tile t at t * kPreQBytes
  uint8_t* k_s = q_s + kPreTiles * kPreQBytes;           // stage s at s * kPreKVBytes
  uint8_t* v_s = k_s + kPreKStages * kPreKVBytes;

  __shared__ uint64_t q_full, k_full[kPreKStages], k_empty[kPreKStages], v_full[kPreVStages], v_empty[kPreVStages];
  __shared__ uint64_t s_full[kPreTiles], p_full[kPreTiles], o_done[kPreTiles], drain_bar;
  // Row max (per step parity) and final row sum exchanged by the two warps sharing a row.
  __shared__ float xmax[kPreTiles][2][2][kPreRows];
  __shared__ float xsum[kPreTiles][2][kPreRows];
  __shared__ uint64_t xbar[kPreTiles][4][2], lbar[kPreTiles][4];
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_flag;

  // Programmatic dependent launch. Right behind the decode (or prefix) grid, this grid starts
  // while that grid's CTAs still run: q, K and V are complete (that grid waited for them before
  // triggering) and this kernel does not read its output; one CTA (the last launched) waits for
  // it before it exits, so this grid completes after it. Behind the norm/RoPE/append kernel
  // instead, every CTA waits first.
  if (!p.prefill_after_decode) pdl_wait();
  pdl_trigger();
  const bool joins_decode = blockIdx.x == 0 && blockIdx.y == gridDim.y - 1;
  // KV head fastest; prefill items last to first: the longest query tiles of every head
  // launch first.
  const int n_items = PREFIX ? (p.counts != nullptr ? p.counts[3] : p.num_prefix)
                             : (p.counts != nullptr ? p.counts[1] : p.num_prefill);
  if (static_cast<int>(blockIdx.y) >= n_items) {  // past this tick's items (capacity grid)
    if (joins_decode) pdl_wait();
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x;
  // Keys [key_base, end) of the row's block table; query tiles at qs0 and qs1 (or none) of
  // the count queries from token q0.
  int row, q0, count, end, qs0, qs1, key_base = 0, split = 0;
  if constexpr (PREFIX) {
    const int32_t* item = p.prefix_items + kPrefixItemInts * static_cast<int>(blockIdx.y);
    row = item[0];
    count = item[1];
    key_base = item[2];
    end = item[3];
    split = item[4];
    const bool row_ok = row >= 0 && row < p.num_rows;
    q0 = row_ok ? p.cu_seq_q[row] : 0;
    // The members and their single tokens must exist, and the keys lie on the row's pages.
    const int limit = row_ok ? max(0, min(p.num_rows - row, p.tokens - q0)) : 0;
    if (count < 0 || count > limit || key_base < 0 || end < key_base || end > p.width * p.page_size) {
      if (threadIdx.x == 0) raise_status(kStatusBadRow);
      count = 0;
      end = key_base;
    }
    qs0 = 0;
    qs1 = count > kTileTokens ? kTileTokens : -1;
  } else {
    const int32_t* item = p.prefill_items + 3 * (n_items - 1 - static_cast<int>(blockIdx.y));
    row = item[0];
    q0 = p.cu_seq_q[row];
    count = p.cu_seq_q[row + 1] - q0;
    end = p.seqused_k[row];
    // Tile 0 starts at item[1]; tile 1 (if any) at item[2] > item[1], so nk0 <= nk1.
    qs0 = item[1];
    qs1 = item[2];
  }
  const int tc0 = max(0, min(kTileTokens, count - qs0));
  const int tc1 = qs1 >= 0 ? min(kTileTokens, count - qs1) : 0;
  int nk0, nk1;
  if constexpr (PREFIX) {
    const int n = (end - key_base + kPreKeys - 1) / kPreKeys;
    nk0 = tc0 > 0 ? n : 0;
    nk1 = tc1 > 0 ? n : 0;
  } else {
    nk0 = (min(end, end - count + qs0 + tc0) + kPreKeys - 1) / kPreKeys;
    nk1 = tc1 > 0 ? (min(end, end - count + qs1 + tc1) + kPreKeys - 1) / kPreKeys : 0;
  }
  const int n_all = max(nk0, nk1);

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < kPreKStages; ++s) { mbar_init(&k_full[s], 1); mbar_init(&k_empty[s], 1); }
    for (int s = 0; s < kPreVStages; ++s) { mbar_init(&v_full[s], 1); mbar_init(&v_empty[s], 1); }
    for (int t = 0; t < kPreTiles; ++t) {
      for (int qd = 0; qd < 4; ++qd) {
        mbar_init(&xbar[t][qd][0], 64);
        mbar_init(&xbar[t][qd][1], 64);
        mbar_init(&lbar[t][qd], 64);
      }
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], kPreSoftmaxThreads);
      mbar_init(&o_done[t], 1);
    }
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_base_s, kPreTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      const int q_tiles = tc1 > 0 ? 2 : 1;
      mbar_expect_tx(&q_full, q_tiles * kPreQBytes);
      for (int t = 0; t < q_tiles; ++t) {
        uint8_t* qt = q_s + t * kPreQBytes;
        const int tok = q0 + (t ? qs1 : qs0);
        tma_load_3d(qt, &qmap, &q_full, 0, h * GROUP, tok);
        tma_load_3d(qt + kPreQBytes / 2, &qmap, &q_full, 64, h * GROUP, tok);
      }
      int k_issued = 0, v_issued = 0, cached_pidx = -1, cached_page = -1;
      for (int j = 0; j < n_all; ++j) {
        // Pool rows of the two 64-key halves of key tile j. A half that starts at or past
        // the sequence end (its rows are masked and their V zeroed) re-reads the first
        // half's rows, so no page beyond the row's block-table entries is named.
        int tok[2];
        bool bad = false;
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
          const int key = key_base + j * kPreKeys + hb * kPreBoxKeys;
          if (hb == 1 && key >= end) { tok[1] = tok[0]; continue; }
          const int pidx = key / p.page_size;
          if (pidx != cached_pidx) {  // one block-table read per page
            cached_page = pidx < p.width ? p.block_table[static_cast<int64_t>(row) * p.width + pidx] : -1;
            cached_pidx = pidx;
          }
          if (cached_page < 0 || cached_page >= p.num_pages) bad = true;
          tok[hb] = cached_page * p.page_size + (key % p.page_size);
        }
        if (bad) {
          raise_status(kStatusBadPage);
          abort_flag = 1;
          break;
        }
        const int ks = j % kPreKStages, vs = j % kPreVStages;
        if (j >= kPreKStages && !mbar_wait(&k_empty[ks], ((j / kPreKStages) - 1) & 1, &abort_flag)) break;
        mbar_expect_tx(&k_full[ks], kPreKVBytes);
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
          uint8_t* dst = k_s + ks * kPreKVBytes + hb * kPreBoxBytes;
          tma_load_3d(dst, &kmap, &k_full[ks], 0, h, tok[hb]);
          tma_load_3d(dst + kPreKVHalf, &kmap, &k_full[ks], 64, h, tok[hb]);
        }
        ++k_issued;
        if (j >= kPreVStages && !mbar_wait(&v_empty[vs], ((j / kPreVStages) - 1) & 1, &abort_flag)) break;
        mbar_expect_tx(&v_full[vs], kPreKVBytes);
#pragma unroll
        for (int hb = 0; hb < 2; ++hb) {
          uint8_t* dst = v_s + vs * kPreKVBytes + hb * kPreBoxBytes;
          tma_load_3d(dst, &vmap, &v_full[vs], 0, h, tok[hb]);
          tma_load_3d(dst + kPreKVHalf, &vmap, &v_full[vs], 64, h, tok[hb]);
        }
        ++v_issued;
      }
      mbar_drain(&q_full, 0);
      if (abort_flag) {  // never leave with copies in flight
        for (int j = max(0, k_issued - kPreKStages); j < k_issued; ++j)
          mbar_drain(&k_full[j % kPreKStages], (j / kPreKStages) & 1);
        for (int j = max(0, v_issued - kPreVStages); j < v_issued; ++j)
          mbar_drain(&v_full[j % kPreVStages], (j / kPreVStages) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs the issue loop (waits by every lane, one elected lane issuing each
    // MMA and commit), so it stays converged and warp-uniform beside the 16 softmax warps.
    {
      constexpr uint32_t idesc_s = idesc_bf16(kPreRows, kPreKeys, false, false);
      constexpr uint32_t idesc_pv = idesc_bf16(kPreRows, D, false, true);
      bool ok = mbar_wait_warp(&q_full, 0, &abort_flag);
      // Operand descriptors are built once; per K step and stage only their start-address
      // field (low 14 bits, 16-byte units) moves, by offsets that never carry out of it
      // (shared memory is below 256 KB), so each MMA costs one add per operand.
      const uint64_t q_desc0 = smem_desc(smem_u32(q_s), 16, 1024, kSwizzle128B);
      const uint64_t k_desc0 = smem_desc(smem_u32(k_s), 16, 1024, kSwizzle128B);
      const uint64_t v_desc0 = smem_desc(smem_u32(v_s), kPreKVHalf, 1024, kSwizzle128B);
      auto issue_s = [&](int t, int j) {
        const uint64_t a = q_desc0 + static_cast<uint64_t>(t * (kPreQBytes >> 4));
        const uint64_t b = k_desc0 + static_cast<uint64_t>((j % kPreKStages) * (kPreKVBytes >> 4));
        const uint32_t d = tmem + kPreKeys * t;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {  // 16 of the 128 head dims per step
          const uint32_t qoff = ((kk >> 2) * (kPreQBytes / 2) + (kk & 3) * 32) >> 4;
          const uint32_t koff = ((kk >> 2) * kPreKVHalf + (kk & 3) * 32) >> 4;
          mma_ss_warp(d, a + qoff, b + koff, idesc_s, kk > 0);
        }
        mma_commit_warp(&s_full[t]);
      };
      auto issue_pv = [&](int t, int j) {
        const uint32_t p_tmem = tmem + kPreKeys * t;
        const uint64_t b = v_desc0 + static_cast<uint64_t>((j % kPreVStages) * (kPreKVBytes >> 4));
        const uint32_t d = tmem + kPreTmemO + t * 128;
#pragma unroll
        for (int kk = 0; kk < kPreKeys / 16; ++kk)  // 16 keys = 8 columns of P, 16 rows of V per step
          mma_ts_warp(d, p_tmem + kk * 8, b + ((kk * 2048) >> 4), idesc_pv, (j > 0 || kk > 0));
        mma_commit_warp(&o_done[t]);
      };
      // Fixed issue order with blocking waits (a poll of an mbarrier costs about as
      // much as an MMA, so the thread never polls): S of key tile 0 for both tiles,
      // then per key tile j: P V_0(j), S_0(j+1), P V_1(j), S_1(j+1). S_t(j+1)
      // overwrites the S/P buffer that P V_t(j) reads: tcgen05.mma of one thread run in
      // issue order, so it does so only after that P V has read it. Tile 0's P V of a
      // key tile goes first, so the V rows its softmax zeroes are zero for tile 1 too.
      const int nk[2] = {nk0, nk1};
      bool issued_any = false;
      int k_have = -1;  // highest key tile whose K stage is known to have landed
      auto need_k = [&](int x) -> bool {
        if (k_have >= x) return true;
        if (!mbar_wait_warp(&k_full[x % kPreKStages], (x / kPreKStages) & 1, &abort_flag)) return false;
        k_have = x;
        tc_fence_after();
        return true;
      };
      if (ok && n_all > 0) {
        ok = need_k(0);
        if (ok) {
#pragma unroll
          for (int t = 0; t < kPreTiles; ++t)
            if (nk[t] > 0) issue_s(t, 0);
          mma_commit_warp(&k_empty[0]);
          issued_any = true;
        }
      }
      for (int j = 0; ok && j < n_all; ++j) {
        if (!mbar_wait_warp(&v_full[j % kPreVStages], (j / kPreVStages) & 1, &abort_flag)) { ok = false; break; }
#pragma unroll
        for (int t = 0; t < kPreTiles; ++t) {
          if (j >= nk[t]) continue;
          if (!mbar_wait_warp(&p_full[t], j & 1, &abort_flag)) { ok = false; break; }
          tc_fence_after();
          issue_pv(t, j);
          if (j + 1 < nk[t]) {
            if (!need_k(j + 1)) { ok = false; break; }
            issue_s(t, j + 1);
          }
        }
        if (!ok) break;
        mma_commit_warp(&v_empty[j % kPreVStages]);  // V_j is free once these P V complete
        if (j + 1 < n_all) mma_commit_warp(&k_empty[(j + 1) % kPreKStages]);
      }
      if (issued_any) {  // nothing may still write TMEM when it is freed
        mma_commit_warp(&drain_bar);
        mbar_drain(&drain_bar, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warps
    const int sw = warp - 2;
    const int t = sw / kPreSoftmaxWarps;            // query tile of this warp
    const int half = (sw % kPreSoftmaxWarps) >> 2;  // key columns 64 half .. 64 half + 63 of S
    const int quad = warp & 3;                      // TMEM lane quadrant this warp may access
    const int r = quad * 32 + lane;                 // accumulator row == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tSP = tmem + kPreKeys * t + lane_base;
    const uint32_t tO = tmem + kPreTmemO + t * 128 + half * 64 + lane_base;  // this warp's 64 output columns
    const int tok = r / GROUP;
    const int qs = t ? qs1 : qs0;
    const bool row_valid = tok < (t ? tc1 : tc0);
    // Key position limit of this query row: bottom-right causal, or every key of a prefix item.
    const int qpos = !row_valid ? -1 : (PREFIX ? (1 << 30) : end - count + qs + tok);
    const int n = t ? nk1 : nk0;
    float m_used = -INFINITY, l = 0.f;  // running max (log2 units) the exponents are taken against
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (!mbar_wait(&s_full[t], j & 1, &abort_flag)) { ok = false; break; }
      tc_fence_after();
      float s[64];
      {
        float* s0 = s;
        float* s1 = s + 32;
        tmem_ld32(tSP + half * 64, *reinterpret_cast<float(*)[32]>(s0));
        tmem_ld32(tSP + half * 64 + 32, *reinterpret_cast<float(*)[32]>(s1));
        tmem_wait_ld();
      }
      const int key0 = key_base + j * kPreKeys + half * 64;
      if (!(key0 + 63 <= qpos && key0 + 64 <= end)) {  // edge of the causal or sequence range: mask
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const int key = key0 + c;
          s[c] = (key <= qpos && key < end) ? s[c] : -INFINITY;
        }
      }
      // Row max as 8 independent chains (fmaxf is exact in any order), then the
      // partner warp's half through shared memory.
      float m8[8];
#pragma unroll
      for (int c = 0; c < 8; ++c)
        m8[c] = max3(max3(s[c], s[c + 8], s[c + 16]), max3(s[c + 24], s[c + 32], s[c + 40]),
                     fmaxf(s[c + 48], s[c + 56]));
      const float mine = max3(max3(m8[0], m8[1], m8[2]), max3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
      xmax[t][j & 1][half][r] = mine;
      mbar_arrive(&xbar[t][quad][j & 1]);
      if (!mbar_wait(&xbar[t][quad][j & 1], (j >> 1) & 1, &abort_flag)) { ok = false; break; }
      const float mx = fmaxf(mine, xmax[t][j & 1][half ^ 1][r]) * p.scale_log2;
      // Lazy rescale: keep the max in use unless this tile's max exceeds it by 2^8.
      const bool grow = mx > m_used + kRescaleThreshold;
      const float m_new = grow ? mx : m_used;
      const float alpha = grow ? fast_exp2(m_used - m_new) : 1.f;  // m_used = -inf gives 0
      m_used = m_new;
      const float neg = m_new == -INFINITY ? 0.f : -m_new;
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
        // O must hold every P V so far before it is rescaled (tcgen05.ld/st are warp-collective).
        if (!mbar_wait(&o_done[t], (j - 1) & 1, &abort_flag)) { ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          float o[16];
          tmem_ld16(tO + cc * 16, o);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 16; ++c) o[c] *= alpha;
          tmem_st16(tO + cc * 16, o);
        }
        tmem_wait_st();
      }
      // P = exp2(S scale - max) as bf16 pairs over the first 64 columns of the S/P
      // buffer (this warp's 64 keys -> columns 32 half .. 32 half + 31). Both warps of
      // the row pair read their S before the max exchange above, so writing over it
      // is safe.
      float s8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int chunk = 0; chunk < 2; ++chunk) {
        uint32_t pw[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          float x0, x1;
          fma2(x0, x1, s[chunk * 32 + 2 * c], s[chunk * 32 + 2 * c + 1], p.scale_log2, p.scale_log2, neg, neg);
          float e0, e1;
          if ((c & 3) == 3) {  // a quarter of the pairs on the FMA pipe
            exp2_fma2(e0, e1, x0, x1);
          } else {
            e0 = fast_exp2(x0);
            e1 = fast_exp2(x1);
          }
          const int a = (2 * c) & 7;
          fma2(s8[a], s8[a + 1], e0, e1, 1.f, 1.f, s8[a], s8[a + 1]);
          pw[c] = pack_bf16(e0, e1);
        }
        tmem_st16u(tSP + half * 32 + chunk * 16, pw);
      }
      tmem_wait_st();
      l = l * alpha + (((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7])));
      // Stale pool rows past the sequence end are zeroed in this V stage by the first
      // query tile that uses key tile j (the MMA warp issues tile 1's P V of a key tile
      // after tile 0's), so both products read the zeros. Each warp of a row pair clears
      // its 64-column d-half of key row r.
      const int vkey0 = key_base + j * kPreKeys;
      const bool zeroer = t == 0 || j >= nk0;
      if (zeroer && vkey0 + kPreKeys > end && vkey0 + r >= end) {
        // V_j must have landed first, or its TMA write would land over the zeros.
        if (!mbar_wait(&v_full[j % kPreVStages], (j / kPreVStages) & 1, &abort_flag)) { ok = false; break; }
        uint8_t* vrow = v_s + (j % kPreVStages) * kPreKVBytes + half * kPreKVHalf;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) *reinterpret_cast<uint4*>(vrow + sw128(r, c8)) = make_uint4(0, 0, 0, 0);
        fence_proxy_async_smem();  // the zeros are read by the tensor core (async proxy)
      }
      tc_fence_before();
      mbar_arrive(&p_full[t]);
    }
    // P V completes in issue order: the last one done means all are.
    if (ok && n > 0 && mbar_wait(&o_done[t], (n - 1) & 1, &abort_flag)) {
      xsum[t][half][r] = l;
      mbar_arrive(&lbar[t][quad]);
      if (mbar_wait(&lbar[t][quad], 0, &abort_flag)) {
        const float total = l + xsum[t][half ^ 1][r];
        tc_fence_after();
        const float inv = total > 0.f ? 1.f / total : 0.f;
        __nv_bfloat16* o = nullptr;
        float* po = nullptr;  // prefix items: the member row's split record
        if constexpr (PREFIX) {
          if (row_valid) {
            const int member = row + qs + tok;
            const int rec_idx = p.row_records[member] + split;
            if (rec_idx < 0 || rec_idx >= p.record_capacity) {
              raise_status(kStatusBadRow);
            } else {
              const int64_t rec = static_cast<int64_t>(rec_idx) * p.heads + h * GROUP + r % GROUP;
              po = p.ws_out + rec * D + half * 64;
              if (half == 0) p.ws_lse[rec] = total > 0.f ? m_used + log2f(total) : -INFINITY;
            }
          }
        } else if (row_valid) {
          o = p.out + (static_cast<int64_t>(q0 + qs + tok) * p.heads + h * GROUP + r % GROUP) * D + half * 64;
        }
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          float v[16];
          tmem_ld16(tO + cc * 16, v);
          tmem_wait_ld();
          if (po != nullptr) {
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4)
              *reinterpret_cast<float4*>(po + cc * 16 + c4 * 4) =
                  make_float4(v[c4 * 4] * inv, v[c4 * 4 + 1] * inv, v[c4 * 4 + 2] * inv, v[c4 * 4 + 3] * inv);
          }
          if (o != nullptr) {
#pragma unroll
            for (int c8 = 0; c8 < 2; ++c8) {
              uint4 w;
              w.x = pack_bf16(v[c8 * 8 + 0] * inv, v[c8 * 8 + 1] * inv);
              w.y = pack_bf16(v[c8 * 8 + 2] * inv, v[c8 * 8 + 3] * inv);
              w.z = pack_bf16(v[c8 * 8 + 4] * inv, v[c8 * 8 + 5] * inv);
              w.w = pack_bf16(v[c8 * 8 + 6] * inv, v[c8 * 8 + 7] * inv);
              *reinterpret_cast<uint4*>(o + cc * 16 + c8 * 8) = w;
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kPreTmemCols);
  }
  if (joins_decode) pdl_wait();
}

}  // namespace hb
