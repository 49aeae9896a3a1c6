// Kernel (c), prefill rows: causal paged GQA attention on tcgen05 tensor cores.
//
// Replaces the prefill-chunk part of the reference's paged varlen attention
// (PackedBatchCache.attend -> varlen_attn with block_table/seqused_k and
// window_size=(-1, 0), src/helios/runtime/qwen3/paged_cache.py:501-520).
//
// One CTA owns two query tiles of 128 rows each; a tile is (128 / GROUP)
// consecutive tokens of one sequence x the GROUP query heads that share KV head h.
// The two tiles are adjacent (2i and 2i+1 of a row), so they need the same key
// tiles (up to two more for the second when a tile exceeds 32 tokens), both stay
// busy for the CTA's whole life, and every K/V tile is read once for both. Roles (320 threads):
//   warp 0     TMA producer: both Q tiles once, then 64-key K and V tiles (two
//              128B-swizzled [64][64] boxes each) from the pages the block table
//              names, into separate 3-stage K and V rings;
//   warp 1     owns the TMEM allocation (512 columns: S0, S1 at 0/64, O0, O1 at
//              128/256, P buffers at 384..511); lane 0 issues tcgen05.mma:
//              S_t = Q_t K^T (M=128, N=64, K=128, both operands in shared memory)
//              and O_t += P_t V (M=128, N=128, K=64, P read from TMEM),
//              committing to mbarriers;
//   warps 2-5  softmax for tile 0, warps 6-9 softmax for tile 1: thread i owns
//              accumulator row i (TMEM lane i), so row max and sum need no
//              shuffles; P is stored as bf16 pairs into one of the tile's two TMEM
//              P buffers (tcgen05.st), so the softmax of key tile j waits only for
//              the P V of key tile j-2 (or j-1 when O must be rescaled).
// The MMA thread polls both tiles' barriers and issues whichever S or P V is
// ready, so the tensor pipe works on one tile while the softmax warps work on
// the other. O is rescaled (in TMEM) only when a row's
// running max grows by more than 2^8; exponents stay relative to the max in use,
// so P <= 2^8 and the final O / l is unchanged. Keys at or beyond seqused_k get
// their V rows zeroed so stale pool memory cannot reach the accumulator. The
// longest pairs (the last of a row) of every KV head are launched first.
#pragma once

#include "hb_common.cuh"
#include "attention_decode.cuh"

namespace hb {

constexpr int kPreRows = 128;     // rows per query tile
constexpr int kPreTiles = 2;      // query tiles per CTA
constexpr int kPreKeys = 64;      // keys per K/V tile
constexpr int kPreKStages = 3;
constexpr int kPreVStages = 3;
constexpr int kPreThreads = 320;
constexpr uint32_t kPreQBytes = kPreRows * 128 * 2;   // [128][128] bf16 as two [128][64] boxes
constexpr uint32_t kPreKVBytes = kPreKeys * 128 * 2;  // [64][128] as two [64][64] boxes
constexpr uint32_t kPreSmemBytes = kPreTiles * kPreQBytes + (kPreKStages + kPreVStages) * kPreKVBytes + 1024;
// TMEM columns: S_t at 64 t, O_t at 128 + 128 t, P_{t,b} (bf16 pairs) at 384 + 32 (2 t + b).
constexpr uint32_t kPreTmemCols = 512;
constexpr uint32_t kPreTmemP = 384;
constexpr float kRescaleThreshold = 8.f;  // log2 units: rescale O when the max grows by more than 2^8

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int GROUP>
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
  __shared__ uint64_t s_full[kPreTiles], s_free[kPreTiles], p_full[kPreTiles][2], o_done[kPreTiles][2], drain_bar;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // KV head fastest, items last to first: the longest query tiles of every head launch first.
  const int h = blockIdx.x;
  const int32_t* item = p.prefill_items + 3 * (p.num_prefill - 1 - static_cast<int>(blockIdx.y));
  const int row = item[0];
  const int q0 = p.cu_seq_q[row];
  const int count = p.cu_seq_q[row + 1] - q0;
  const int end = p.seqused_k[row];
  // Tile 0 starts at item[1]; tile 1 (if any) at item[2] > item[1], so n_kv0 <= n_kv1.
  const int qs0 = item[1], qs1 = item[2];
  const int tc0 = min(kTileTokens, count - qs0);
  const int tc1 = qs1 >= 0 ? min(kTileTokens, count - qs1) : 0;
  const int nk0 = (min(end, end - count + qs0 + tc0) + kPreKeys - 1) / kPreKeys;
  const int nk1 = tc1 > 0 ? (min(end, end - count + qs1 + tc1) + kPreKeys - 1) / kPreKeys : 0;
  const int n_all = max(nk0, nk1);

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < kPreKStages; ++s) { mbar_init(&k_full[s], 1); mbar_init(&k_empty[s], 1); }
    for (int s = 0; s < kPreVStages; ++s) { mbar_init(&v_full[s], 1); mbar_init(&v_empty[s], 1); }
    for (int t = 0; t < kPreTiles; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&s_free[t], 128);
      for (int b = 0; b < 2; ++b) {
        mbar_init(&p_full[t][b], 128);
        mbar_init(&o_done[t][b], 1);
      }
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
      int k_issued = 0, v_issued = 0;
      for (int j = 0; j < n_all; ++j) {
        const int key = j * kPreKeys;
        const int pidx = key / p.page_size;
        const int page = pidx < p.width ? p.block_table[static_cast<int64_t>(row) * p.width + pidx] : -1;
        if (page < 0 || page >= p.num_pages) {
          raise_status(kStatusBadPage);
          abort_flag = 1;
          break;
        }
        const int tok = page * p.page_size + (key % p.page_size);
        const int ks = j % kPreKStages, vs = j % kPreVStages;
        if (j >= kPreKStages && !mbar_wait(&k_empty[ks], ((j / kPreKStages) - 1) & 1, &abort_flag)) break;
        mbar_expect_tx(&k_full[ks], kPreKVBytes);
        tma_load_3d(k_s + ks * kPreKVBytes, &kmap, &k_full[ks], 0, h, tok);
        tma_load_3d(k_s + ks * kPreKVBytes + kPreKVBytes / 2, &kmap, &k_full[ks], 64, h, tok);
        ++k_issued;
        if (j >= kPreVStages && !mbar_wait(&v_empty[vs], ((j / kPreVStages) - 1) & 1, &abort_flag)) break;
        mbar_expect_tx(&v_full[vs], kPreKVBytes);
        tma_load_3d(v_s + vs * kPreKVBytes, &vmap, &v_full[vs], 0, h, tok);
        tma_load_3d(v_s + vs * kPreKVBytes + kPreKVBytes / 2, &vmap, &v_full[vs], 64, h, tok);
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
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16(kPreRows, kPreKeys, false, false);
      constexpr uint32_t idesc_pv = idesc_bf16(kPreRows, D, false, true);
      bool ok = mbar_wait(&q_full, 0, &abort_flag);
      auto issue_s = [&](int t, int j) {
        const uint32_t q_addr = smem_u32(q_s + t * kPreQBytes);
        const uint32_t k_addr = smem_u32(k_s + (j % kPreKStages) * kPreKVBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t qoff = (kk >> 2) * (kPreQBytes / 2) + (kk & 3) * 32;
          const uint32_t koff = (kk >> 2) * (kPreKVBytes / 2) + (kk & 3) * 32;
          mma_ss(tmem + t * kPreKeys, smem_desc(q_addr + qoff, 16, 1024, kSwizzle128B),
                 smem_desc(k_addr + koff, 16, 1024, kSwizzle128B), idesc_s, kk > 0);
        }
        mma_commit(&s_full[t]);
      };
      auto issue_pv = [&](int t, int j) {
        const uint32_t p_tmem = tmem + kPreTmemP + (2 * t + (j & 1)) * (kPreKeys / 2);
        const uint32_t v_addr = smem_u32(v_s + (j % kPreVStages) * kPreKVBytes);
#pragma unroll
        for (int kk = 0; kk < kPreKeys / 16; ++kk)  // 16 keys = 8 columns of P per step
          mma_ts(tmem + 128 + t * 128, p_tmem + kk * 8,
                 smem_desc(v_addr + kk * 2048, kPreKVBytes / 2, 1024, kSwizzle128B), idesc_pv, (j > 0 || kk > 0));
        mma_commit(&o_done[t][j & 1]);
      };
      bool issued_any = false;
      // Non-blocking scheduler: issue whichever S or P V is ready for either query
      // tile, so one tile's softmax never holds up the other's tensor work. K (V) stage
      // j is released once every tile that needs key tile j has issued its S (P V).
      const int nk[2] = {nk0, nk1};
      int ns[2] = {0, 0}, npv[2] = {0, 0};
      int krel = 0, vrel = 0;
      uint64_t idle_since = globaltimer_ns();
      while (ok) {
        bool progress = false;
#pragma unroll
        for (int t = 0; t < kPreTiles; ++t) {
          const int j = ns[t];
          if (j < nk[t] && mbar_test(&k_full[j % kPreKStages], (j / kPreKStages) & 1) &&
              (j == 0 || mbar_test(&s_free[t], (j - 1) & 1))) {
            tc_fence_after();
            issue_s(t, j);
            ns[t] = j + 1;
            progress = issued_any = true;
          }
        }
        while (krel < n_all && (krel < ns[0] || krel >= nk[0]) && (krel < ns[1] || krel >= nk[1])) {
          mma_commit(&k_empty[krel % kPreKStages]);
          ++krel;
        }
#pragma unroll
        for (int t = 0; t < kPreTiles; ++t) {
          const int j = npv[t];
          if (j < nk[t] && mbar_test(&v_full[j % kPreVStages], (j / kPreVStages) & 1) &&
              mbar_test(&p_full[t][j & 1], (j >> 1) & 1)) {
            tc_fence_after();
            issue_pv(t, j);
            npv[t] = j + 1;
            progress = issued_any = true;
          }
        }
        while (vrel < n_all && (vrel < npv[0] || vrel >= nk[0]) && (vrel < npv[1] || vrel >= nk[1])) {
          mma_commit(&v_empty[vrel % kPreVStages]);
          ++vrel;
        }
        if (npv[0] == nk[0] && npv[1] == nk[1] && krel == n_all && vrel == n_all) break;
        if (progress) {
          idle_since = globaltimer_ns();
        } else if (*reinterpret_cast<volatile int*>(&abort_flag)) {
          ok = false;
        } else if (globaltimer_ns() - idle_since > kWaitLimitNs) {
          abort_flag = 1;
          raise_status(kStatusWaitTimeout);
          ok = false;
        }
      }
      if (issued_any) {  // nothing may still write TMEM when it is freed
        mma_commit(&drain_bar);
        mbar_drain(&drain_bar, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warpgroups
    const int t = (warp - 2) >> 2;   // query tile of this warpgroup
    const int quad = warp & 3;       // TMEM lane quadrant this warp may access
    const int r = quad * 32 + lane;  // accumulator row == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem + t * kPreKeys + lane_base, tO = tmem + 128 + t * 128 + lane_base;
    const int tok = r / GROUP;
    const int qs = t ? qs1 : qs0;
    const bool row_valid = tok < (t ? tc1 : tc0);
    const int qpos = row_valid ? end - count + qs + tok : -1;
    const int n = t ? nk1 : nk0;
    float m_used = -INFINITY, l = 0.f;  // running max (log2 units) the exponents are taken against
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      if (!mbar_wait(&s_full[t], j & 1, &abort_flag)) { ok = false; break; }
      tc_fence_after();
      float s[64];
      tmem_ld64(tS, s);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&s_free[t]);
      const int key0 = j * kPreKeys;
      if (!(key0 + kPreKeys - 1 <= qpos && key0 + kPreKeys <= end)) {  // edge tile: mask
#pragma unroll
        for (int c = 0; c < 64; ++c) {
          const int key = key0 + c;
          s[c] = (key <= qpos && key < end) ? s[c] : -INFINITY;
        }
      }
      // Max and sum as 8 independent chains (fmaxf is exact in any order; the sum
      // order only moves rounding of the normaliser).
      float m8[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) m8[c] = fmaxf(s[c], s[c + 8]);
#pragma unroll
      for (int c = 16; c < 64; c += 8) {
#pragma unroll
        for (int e = 0; e < 8; ++e) m8[e] = fmaxf(m8[e], s[c + e]);
      }
      float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])), fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
      mx *= p.scale_log2;
      // Lazy rescale: keep the max in use unless this tile's max exceeds it by 2^8.
      const bool grow = mx > m_used + kRescaleThreshold;
      const float m_new = grow ? mx : m_used;
      const float alpha = grow ? fast_exp2(m_used - m_new) : 1.f;  // m_used = -inf gives 0
      m_used = m_new;
      const float neg = m_new == -INFINITY ? 0.f : -m_new;
      float s8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        s[c] = fast_exp2(fmaf(s[c], p.scale_log2, neg));
        s8[c & 7] += s[c];
      }
      l = l * alpha + (((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7])));
      // P buffer j & 1 was last read by the P V of key tile j - 2.
      if (j >= 2 && !mbar_wait(&o_done[t][j & 1], ((j >> 1) - 1) & 1, &abort_flag)) { ok = false; break; }
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
        // O must hold every P V so far before it is rescaled (tcgen05.ld/st are warp-collective).
        if (!mbar_wait(&o_done[t][(j - 1) & 1], ((j - 1) >> 1) & 1, &abort_flag)) { ok = false; break; }
        tc_fence_after();
        {
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            float o[32];
            tmem_ld32(tO + cc * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] *= alpha;
            tmem_st32(tO + cc * 32, o);
          }
          tmem_wait_st();
        }
      }
      {  // P as bf16 pairs into this tile's TMEM P buffer j & 1 (row r = lane r)
        uint32_t pw[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) pw[c] = pack_bf16(s[2 * c], s[2 * c + 1]);
        tmem_st32u(tmem + kPreTmemP + (2 * t + (j & 1)) * (kPreKeys / 2) + lane_base, pw);
        tmem_wait_st();
      }
      // Stale pool rows past the sequence end are zeroed in this V stage by the first
      // query tile that uses key tile j: the MMA warp issues tile 0's P V before tile 1's,
      // so both products read the zeros.
      const bool zeroer = t == 0 || j >= nk0;
      if (zeroer && key0 + kPreKeys > end && r < kPreKeys && key0 + r >= end) {
        // V_j must have landed first, or its TMA write would land over the zeros.
        if (!mbar_wait(&v_full[j % kPreVStages], (j / kPreVStages) & 1, &abort_flag)) { ok = false; break; }
        uint8_t* vrow = v_s + (j % kPreVStages) * kPreKVBytes;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          *reinterpret_cast<uint4*>(vrow + sw128(r, c8)) = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(vrow + kPreKVBytes / 2 + sw128(r, c8)) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();  // the zeros are read by the tensor core (async proxy)
      }
      tc_fence_before();
      mbar_arrive(&p_full[t][j & 1]);
    }
    // P V completes in issue order: the last one done means all are.
    if (ok && n > 0 && mbar_wait(&o_done[t][(n - 1) & 1], ((n - 1) >> 1) & 1, &abort_flag)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* o = row_valid ? p.out + (static_cast<int64_t>(q0 + qs + tok) * p.heads + h * GROUP + r % GROUP) * D
                                   : nullptr;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        float v[32];
        tmem_ld32(tO + cc * 32, v);
        tmem_wait_ld();
        if (o != nullptr) {
#pragma unroll
          for (int c8 = 0; c8 < 4; ++c8) {
            uint4 w;
            w.x = pack_bf16(v[c8 * 8 + 0] * inv, v[c8 * 8 + 1] * inv);
            w.y = pack_bf16(v[c8 * 8 + 2] * inv, v[c8 * 8 + 3] * inv);
            w.z = pack_bf16(v[c8 * 8 + 4] * inv, v[c8 * 8 + 5] * inv);
            w.w = pack_bf16(v[c8 * 8 + 6] * inv, v[c8 * 8 + 7] * inv);
            *reinterpret_cast<uint4*>(o + cc * 32 + c8 * 8) = w;
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
}

}  // namespace hb
