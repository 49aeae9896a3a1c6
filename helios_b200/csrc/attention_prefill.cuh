// Kernel (c), prefill rows: causal paged GQA attention on tcgen05 tensor cores.
//
// Replaces the prefill-chunk part of the reference's paged varlen attention
// (PackedBatchCache.attend -> varlen_attn with block_table/seqused_k and
// window_size=(-1, 0), src/helios/runtime/qwen3/paged_cache.py:501-520).
//
// One CTA owns one query tile of 128 rows = (128 / GROUP) consecutive tokens of
// one sequence x the GROUP query heads that share KV head h, so every K/V tile is
// read once for the whole group. Roles (192 threads):
//   warp 0    TMA producer: the Q tile once, then 64-key K and V tiles (two
//             128B-swizzled [64][64] boxes each) from the pages the block table
//             names, into a 2-stage ring;
//   warp 1    owns the TMEM allocation (256 columns: S at 0..63, O at 128..255);
//             lane 0 issues tcgen05.mma: S = Q K^T (M=128, N=64, K=128) and
//             O += P V (M=128, N=128, K=64), committing to mbarriers;
//   warps 2-5 softmax: thread i owns accumulator row i (TMEM lane i), so the
//             row max and sum need no shuffles. P is written as bf16 into the
//             K slot of the same stage (K is dead once S is computed), in the
//             canonical 128B-swizzled K-major layout the next MMA reads.
// The online-softmax rescale of O is done in TMEM (tcgen05.ld/st) after the
// previous P V completes. Keys at or beyond seqused_k get their V rows zeroed
// so stale pool memory cannot reach the accumulator.
#pragma once

#include "hb_common.cuh"
#include "attention_decode.cuh"

namespace hb {

constexpr int kPreRows = 128;
constexpr int kPreKeys = 64;
constexpr int kPreThreads = 192;
constexpr uint32_t kPreQBytes = kPreRows * 128 * 2;   // [128][128] bf16 as two [128][64] boxes
constexpr uint32_t kPreKBytes = kPreKeys * 128 * 2;   // [64][128] as two [64][64] boxes (later P [128][64])
constexpr uint32_t kPreVBytes = kPreKeys * 128 * 2;
constexpr uint32_t kPreStageBytes = kPreKBytes + kPreVBytes;
constexpr uint32_t kPreSmemBytes = kPreQBytes + 2 * kPreStageBytes + 1024;
constexpr uint32_t kPreTmemCols = 256;

template <int GROUP>
__global__ void __launch_bounds__(kPreThreads, 1) prefill_attention_kernel(AttentionParams p,
                                                                          const __grid_constant__ CUtensorMap qmap,
                                                                          const __grid_constant__ CUtensorMap kmap,
                                                                          const __grid_constant__ CUtensorMap vmap) {
  constexpr int D = 128;
  constexpr int kTileTokens = kPreRows / GROUP;
  extern __shared__ __align__(1024) uint8_t dsm[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = smem;
  uint8_t* stage_s = smem + kPreQBytes;  // stage st: K/P at st*kPreStageBytes, V after it

  __shared__ uint64_t q_full, kv_full[2], kv_empty[2], s_full, s_free, p_full, o_done, drain_bar;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y;
  const int32_t* item = p.prefill_items + 2 * blockIdx.x;
  const int row = item[0], q_start = item[1];
  const int q0 = p.cu_seq_q[row];
  const int count = p.cu_seq_q[row + 1] - q0;
  const int end = p.seqused_k[row];
  const int tile_count = min(kTileTokens, count - q_start);         // valid tokens in this tile
  const int last_qpos = end - count + q_start + tile_count - 1;      // furthest query position
  const int n_kv = (min(end, last_qpos + 1) + kPreKeys - 1) / kPreKeys;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(&s_full, 1);
    mbar_init(&s_free, 128);
    mbar_init(&p_full, 128);
    mbar_init(&o_done, 1);
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
  const uint32_t tS = tmem, tO = tmem + 128;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      mbar_expect_tx(&q_full, kPreQBytes);
      tma_load_3d(q_s, &qmap, &q_full, 0, h * GROUP, q0 + q_start);
      tma_load_3d(q_s + kPreQBytes / 2, &qmap, &q_full, 64, h * GROUP, q0 + q_start);
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int st = j & 1;
        if (j >= 2 && !mbar_wait(&kv_empty[st], ((j >> 1) - 1) & 1, &abort_flag)) break;
        const int key = j * kPreKeys;
        const int pidx = key / p.page_size;
        const int page = pidx < p.width ? p.block_table[static_cast<int64_t>(row) * p.width + pidx] : -1;
        if (page < 0 || page >= p.num_pages) {
          raise_status(kStatusBadPage);
          abort_flag = 1;
          break;
        }
        const int tok = page * p.page_size + (key % p.page_size);
        uint8_t* ks = stage_s + st * kPreStageBytes;
        uint8_t* vs = ks + kPreKBytes;
        mbar_expect_tx(&kv_full[st], kPreStageBytes);
        tma_load_3d(ks, &kmap, &kv_full[st], 0, h, tok);
        tma_load_3d(ks + kPreKBytes / 2, &kmap, &kv_full[st], 64, h, tok);
        tma_load_3d(vs, &vmap, &kv_full[st], 0, h, tok);
        tma_load_3d(vs + kPreVBytes / 2, &vmap, &kv_full[st], 64, h, tok);
        ++issued;
      }
      mbar_drain(&q_full, 0);
      if (abort_flag)
        for (int j = max(0, issued - 2); j < issued; ++j) mbar_drain(&kv_full[j & 1], (j >> 1) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16(kPreRows, kPreKeys, false, false);
      constexpr uint32_t idesc_pv = idesc_bf16(kPreRows, D, false, true);
      const uint32_t q_addr = smem_u32(q_s);
      bool ok = mbar_wait(&q_full, 0, &abort_flag);
      bool issued_any = false;
      for (int j = 0; ok && j < n_kv; ++j) {
        const int st = j & 1;
        const uint32_t k_addr = smem_u32(stage_s + st * kPreStageBytes);
        if (!mbar_wait(&kv_full[st], (j >> 1) & 1, &abort_flag)) { ok = false; break; }
        if (j > 0 && !mbar_wait(&s_free, (j - 1) & 1, &abort_flag)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (kPreQBytes / 2) + (kk & 3) * 32;
          const uint32_t koff = (kk >> 2) * (kPreKBytes / 2) + (kk & 3) * 32;
          mma_ss(tS, smem_desc(q_addr + off, 16, 1024, kSwizzle128B), smem_desc(k_addr + koff, 16, 1024, kSwizzle128B),
                 idesc_s, kk > 0);
        }
        mma_commit(&s_full);
        issued_any = true;
        if (j > 0) {
          const int pj = j - 1, pst = pj & 1;
          if (!mbar_wait(&p_full, pj & 1, &abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t p_addr = smem_u32(stage_s + pst * kPreStageBytes);
          const uint32_t v_addr = p_addr + kPreKBytes;
#pragma unroll
          for (int kk = 0; kk < kPreKeys / 16; ++kk)
            mma_ss(tO, smem_desc(p_addr + kk * 32, 16, 1024, kSwizzle128B),
                   smem_desc(v_addr + kk * 2048, kPreVBytes / 2, 1024, kSwizzle128B), idesc_pv, (pj > 0 || kk > 0));
          mma_commit(&o_done);
          mma_commit(&kv_empty[pst]);
        }
      }
      if (ok && n_kv > 0) {
        const int pj = n_kv - 1, pst = pj & 1;
        if (mbar_wait(&p_full, pj & 1, &abort_flag)) {
          tc_fence_after();
          const uint32_t p_addr = smem_u32(stage_s + pst * kPreStageBytes);
          const uint32_t v_addr = p_addr + kPreKBytes;
#pragma unroll
          for (int kk = 0; kk < kPreKeys / 16; ++kk)
            mma_ss(tO, smem_desc(p_addr + kk * 32, 16, 1024, kSwizzle128B),
                   smem_desc(v_addr + kk * 2048, kPreVBytes / 2, 1024, kSwizzle128B), idesc_pv, (pj > 0 || kk > 0));
          mma_commit(&o_done);
          mma_commit(&kv_empty[pst]);
        }
      }
      if (issued_any) {  // nothing may still write TMEM when it is freed
        mma_commit(&drain_bar);
        mbar_drain(&drain_bar, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warpgroup
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // accumulator row == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(quad * 32) << 16;
    const int tok = r / GROUP;
    const bool row_valid = tok < tile_count;
    const int qpos = row_valid ? end - count + q_start + tok : -1;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int st = j & 1;
      if (!mbar_wait(&s_full, j & 1, &abort_flag)) { ok = false; break; }
      tc_fence_after();
      float s[64];
      tmem_ld32(tS + lane_base + 0, *reinterpret_cast<float(*)[32]>(&s[0]));
      tmem_ld32(tS + lane_base + 32, *reinterpret_cast<float(*)[32]>(&s[32]));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&s_free);
      const int key0 = j * kPreKeys;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const int key = key0 + c;
        s[c] = (key <= qpos && key < end) ? s[c] * p.scale_log2 : -INFINITY;
        mx = fmaxf(mx, s[c]);
      }
      const float mn = fmaxf(m, mx);
      const float base = mn == -INFINITY ? 0.f : mn;
      const float alpha = exp2f(m - base);
      m = mn;
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        s[c] = exp2f(s[c] - base);
        sum += s[c];
      }
      l = l * alpha + sum;
      if (j > 0) {
        if (!mbar_wait(&o_done, (j - 1) & 1, &abort_flag)) { ok = false; break; }
        tc_fence_after();
        // tcgen05.ld/st are warp-collective: rescale when any row of the warp moved its max.
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            float o[32];
            tmem_ld32(tO + lane_base + cc * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] *= alpha;
            tmem_st32(tO + lane_base + cc * 32, o);
          }
          tmem_wait_st();
        }
      }
      // P (bf16) into this stage's K slot, canonical 128B-swizzled K-major rows.
      uint8_t* ps = stage_s + st * kPreStageBytes;
#pragma unroll
      for (int c8 = 0; c8 < 8; ++c8) {
        uint4 v;
        v.x = pack_bf16(s[c8 * 8 + 0], s[c8 * 8 + 1]);
        v.y = pack_bf16(s[c8 * 8 + 2], s[c8 * 8 + 3]);
        v.z = pack_bf16(s[c8 * 8 + 4], s[c8 * 8 + 5]);
        v.w = pack_bf16(s[c8 * 8 + 6], s[c8 * 8 + 7]);
        *reinterpret_cast<uint4*>(ps + sw128(r, c8)) = v;
      }
      if (key0 + kPreKeys > end && r < kPreKeys && key0 + r >= end) {
        uint8_t* vs = ps + kPreKBytes;
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          *reinterpret_cast<uint4*>(vs + sw128(r, c8)) = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(vs + kPreVBytes / 2 + sw128(r, c8)) = make_uint4(0, 0, 0, 0);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full);
    }
    if (ok && n_kv > 0 && mbar_wait(&o_done, (n_kv - 1) & 1, &abort_flag)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* o = row_valid ? p.out + (static_cast<int64_t>(q0 + q_start + tok) * p.heads + h * GROUP + r % GROUP) * D
                                   : nullptr;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        float v[32];
        tmem_ld32(tO + lane_base + cc * 32, v);
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
