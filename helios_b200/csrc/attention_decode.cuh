// Kernel (c), decode rows: split-K paged GQA attention (flash-decoding).
//
// Replaces the decode part of the reference's paged varlen attention call
// (PackedBatchCache.attend -> varlen_attn(..., block_table, seqused_k,
// window_size=(-1, 0), num_splits=1), src/helios/runtime/qwen3/paged_cache.py:501-520;
// PagedBatchCache.attend, :301-333). The reference runs with num_splits=1, which
// leaves most SMs idle when a tick holds few long decode rows; here each
// (row, split of split_keys keys, KV head) is one CTA.
//
// Semantics (bottom-right causal, as the reference's window_size=(-1, 0)): query
// i of a row with `count` queries and `end = seqused_k` keys sits at key position
// end - count + i and sees keys 0..that position. Scale is applied to q.k in fp32.
//
// Structure per CTA (160 threads): warp 4 is the TMA producer, streaming 64-key
// K and V tiles of one KV head ([64 keys][128 d] bf16, two 128B-swizzled boxes
// each) from the page the block table names into a 3-stage ring; warps 0-3
// consume them with m16n8k16 warp MMAs. All query rows of the GQA group
// (count * group <= 64) share every K/V tile, so K/V bytes cross HBM once per
// (row, KV head). With 16 query rows, the 4 warps split the 64 keys of a tile
// and merge their (max, sum, acc) at the end; with 64 rows each warp owns 16
// rows. Results of a multi-split row go to a float workspace as (normalised
// output, log2-sum-exp) and are merged by decode_combine_kernel.
#pragma once

#include "hb_common.cuh"

namespace hb {

struct AttentionParams {
  const __nv_bfloat16* q;   // [T, H, D]
  __nv_bfloat16* out;       // [T, H, D]
  const int32_t* block_table;  // [B, W]
  const int32_t* cu_seq_q;     // [B+1]
  const int32_t* seqused_k;    // [B]
  const int32_t* decode_items;   // [n][4] row, split, partial_base, n_splits
  const int32_t* prefill_items;  // [n][3] row, query start of tile 2i, of tile 2i+1 or -1
  // Optional device counts {decode items, prefill pairs, partial records} written by the
  // tick-pack kernel: when set, grids are sized to capacities and CTAs past a count exit
  // (a launch that stays valid, e.g. in a CUDA graph, while the work list changes).
  const int32_t* counts;
  // Set when the prefill kernel is launched right behind the decode kernel (programmatic
  // dependent launch): it then reads q, K and V without waiting (the decode kernel waited
  // for them before triggering), and one of its CTAs waits for the decode grid before
  // exiting, so the prefill grid completes after the decode grid.
  int32_t prefill_after_decode;
  float* ws_out;   // [records, H, D]
  float* ws_lse;   // [records, H]
  int32_t width, num_pages, page_size, heads, kv_heads, split_keys, tokens;
  int32_t num_prefill;  // prefill items (the kernel walks them from the last, heaviest, first)
  float scale_log2;  // softmax scale * log2(e)
};

constexpr int kDecTileKeys = 64;
constexpr int kDecStages = 3;
constexpr int kDecConsumerWarps = 4;
constexpr int kDecThreads = (kDecConsumerWarps + 1) * 32;
constexpr uint32_t kDecHalfBytes = kDecTileKeys * 128;                 // one [64][64] bf16 box
constexpr uint32_t kDecTileBytes = 2 * kDecHalfBytes;                  // K or V tile, D = 128
constexpr uint32_t kDecStageBytes = 2 * kDecTileBytes;                 // K + V
constexpr uint32_t kDecSmemBytes = kDecStages * kDecStageBytes + 1024;  // + alignment slack
constexpr int kMergeStride = 132;  // floats per row of the split merge scratch (padded: no bank conflicts)
static_assert(kDecConsumerWarps * 16 * kMergeStride * 4 <= kDecStages * kDecStageBytes, "merge scratch fits the ring");

template <int GROUP>
__global__ void __launch_bounds__(kDecThreads, 2) decode_attention_kernel(AttentionParams p,
                                                                      const __grid_constant__ CUtensorMap kmap,
                                                                      const __grid_constant__ CUtensorMap vmap) {
  constexpr int D = 128;
  extern __shared__ __align__(1024) uint8_t dsm[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full_bar[kDecStages], empty_bar[kDecStages];
  __shared__ int abort_flag;
  __shared__ float merge_ml[kDecConsumerWarps][16][2];

  pdl_wait();     // q, K and V from the norm/RoPE/append kernel ahead of this one
  pdl_trigger();  // the prefill kernel (or the split combine) may launch behind this grid
  if (p.counts != nullptr && static_cast<int>(blockIdx.x) >= p.counts[0]) return;  // past this tick's items
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y;
  const int32_t* item = p.decode_items + 4 * blockIdx.x;
  const int row = item[0], split = item[1], pbase = item[2], nsplit = item[3];
  const int q0 = p.cu_seq_q[row];
  const int count = p.cu_seq_q[row + 1] - q0;
  const int end = p.seqused_k[row];
  const int kb = split * p.split_keys;
  const int ke = min(end, kb + p.split_keys);
  const int n_tiles = (ke - kb + kDecTileKeys - 1) / kDecTileKeys;
  const int qrows = count * GROUP;
  const int m_tiles = qrows <= 16 ? 1 : (qrows <= 32 ? 2 : 4);
  const int key_split = kDecConsumerWarps / m_tiles;  // warps sharing one m-tile
  const int kpw = kDecTileKeys / key_split;           // keys per warp per tile

  if (threadIdx.x == 0) {
    for (int s = 0; s < kDecStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kDecConsumerWarps);
    }
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kDecConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      int issued = 0, cached_pidx = -1, cached_page = -1;
      for (int t = 0; t < n_tiles; ++t) {
        const int stage = t % kDecStages;
        if (t >= kDecStages && !mbar_wait(&empty_bar[stage], ((t / kDecStages) - 1) & 1, &abort_flag)) break;
        const int key = kb + t * kDecTileKeys;
        const int pidx = key / p.page_size;
        if (pidx != cached_pidx) {  // one block-table read per page, not per key tile
          cached_page = pidx < p.width ? p.block_table[static_cast<int64_t>(row) * p.width + pidx] : -1;
          cached_pidx = pidx;
        }
        const int page = cached_page;
        if (page < 0 || page >= p.num_pages) {
          raise_status(kStatusBadPage);
          abort_flag = 1;
          break;
        }
        const int tok = page * p.page_size + (key % p.page_size);
        uint8_t* ks = smem + stage * kDecStageBytes;
        uint8_t* vs = ks + kDecTileBytes;
        mbar_expect_tx(&full_bar[stage], kDecStageBytes);
        tma_load_3d(ks, &kmap, &full_bar[stage], 0, h, tok);
        tma_load_3d(ks + kDecHalfBytes, &kmap, &full_bar[stage], 64, h, tok);
        tma_load_3d(vs, &vmap, &full_bar[stage], 0, h, tok);
        tma_load_3d(vs + kDecHalfBytes, &vmap, &full_bar[stage], 64, h, tok);
        ++issued;
      }
      // Never leave with copies in flight: wait (bounded) for every issued tile.
      if (abort_flag) {
        for (int t = max(0, issued - kDecStages); t < issued; ++t) mbar_drain(&full_bar[t % kDecStages], (t / kDecStages) & 1);
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int mt = warp / key_split, kpart = warp % key_split;
  const int g4 = lane >> 2, c4 = lane & 3;
  // Query A-fragments for rows mt*16 + g4 and +8: 8 k-steps of 16 dims.
  uint32_t qa[8][4];
  {
    const int ja = mt * 16 + g4, jb = ja + 8;
    const __nv_bfloat16* pa = ja < qrows ? p.q + (static_cast<int64_t>(q0 + ja / GROUP) * p.heads + h * GROUP + ja % GROUP) * D : nullptr;
    const __nv_bfloat16* pb = jb < qrows ? p.q + (static_cast<int64_t>(q0 + jb / GROUP) * p.heads + h * GROUP + jb % GROUP) * D : nullptr;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int d0 = kk * 16 + 2 * c4;
      qa[kk][0] = pa ? *reinterpret_cast<const uint32_t*>(pa + d0) : 0u;
      qa[kk][1] = pb ? *reinterpret_cast<const uint32_t*>(pb + d0) : 0u;
      qa[kk][2] = pa ? *reinterpret_cast<const uint32_t*>(pa + d0 + 8) : 0u;
      qa[kk][3] = pb ? *reinterpret_cast<const uint32_t*>(pb + d0 + 8) : 0u;
    }
  }
  // Key position limit per query row (bottom-right causal) for rows g4, g4+8.
  const int ja = mt * 16 + g4, jb = ja + 8;
  const int qpos_a = ja < qrows ? end - count + ja / GROUP : -1;
  const int qpos_b = jb < qrows ? end - count + jb / GROUP : -1;

  float acc[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;

  for (int t = 0; t < n_tiles; ++t) {
    const int stage = t % kDecStages;
    if (!mbar_wait(&full_bar[stage], (t / kDecStages) & 1, &abort_flag)) break;
    const uint32_t ks = smem_u32(smem + stage * kDecStageBytes);
    const uint32_t vs = ks + kDecTileBytes;
    const int key0 = kb + t * kDecTileKeys;
    const int mykey0 = kpart * kpw;  // within the tile
    // Keys at or past the split end may be stale or uninitialised pool memory:
    // zero their V rows (this warp only reads its own key range) so 0 * NaN cannot occur.
    if (key0 + kDecTileKeys > ke) {
      uint8_t* vgen = smem + stage * kDecStageBytes + kDecTileBytes;
      for (int kr = mykey0 + (lane >> 3); kr < mykey0 + kpw; kr += 4) {
        if (key0 + kr >= ke) {
          const int chunk = lane & 7;
          *reinterpret_cast<uint4*>(vgen + sw128(kr, chunk)) = make_uint4(0, 0, 0, 0);
          *reinterpret_cast<uint4*>(vgen + kDecHalfBytes + sw128(kr, chunk)) = make_uint4(0, 0, 0, 0);
        }
      }
      fence_proxy_async_smem();  // these generic writes precede the stage's next TMA fill
      __syncwarp();
    }
    // ---- S = Q K^T over this warp's keys: kpw/8 n-tiles.
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int np = 0; np < 4; ++np) {  // pairs of 8-key n-tiles
      if (np * 16 >= kpw) break;
      const int kr = mykey0 + np * 16 + (lane & 7) + ((lane >> 4) << 3);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int chunk = kk * 2 + ((lane >> 3) & 1);
        const uint32_t addr = ks + (chunk >> 3) * kDecHalfBytes + sw128(kr, chunk & 7);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(addr, b0, b1, b2, b3);
        mma_16816(s[2 * np], qa[kk], b0, b1);
        mma_16816(s[2 * np + 1], qa[kk], b2, b3);
      }
    }
    // ---- mask, online softmax (log2 domain)
    const int nt_count = kpw / 8;
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      if (n >= nt_count) break;
      const int key = key0 + mykey0 + n * 8 + 2 * c4;
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const bool ok = key + e < ke;
        s[n][e] = (ok && key + e <= qpos_a) ? s[n][e] * p.scale_log2 : -INFINITY;
        s[n][2 + e] = (ok && key + e <= qpos_b) ? s[n][2 + e] * p.scale_log2 : -INFINITY;
        mx_a = fmaxf(mx_a, s[n][e]);
        mx_b = fmaxf(mx_b, s[n][2 + e]);
      }
    }
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
    const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
    const float base_a = mn_a == -INFINITY ? 0.f : mn_a, base_b = mn_b == -INFINITY ? 0.f : mn_b;
    const float alpha_a = exp2f(m_a - base_a), alpha_b = exp2f(m_b - base_b);
    m_a = mn_a;
    m_b = mn_b;
    l_a *= alpha_a;
    l_b *= alpha_b;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      acc[n][0] *= alpha_a; acc[n][1] *= alpha_a;
      acc[n][2] *= alpha_b; acc[n][3] *= alpha_b;
    }
    uint32_t pa[8][2];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      if (n >= nt_count) break;
      const float p0 = exp2f(s[n][0] - base_a), p1 = exp2f(s[n][1] - base_a);
      const float p2 = exp2f(s[n][2] - base_b), p3 = exp2f(s[n][3] - base_b);
      l_a += p0 + p1;
      l_b += p2 + p3;
      pa[n][0] = pack_bf16(p0, p1);
      pa[n][1] = pack_bf16(p2, p3);
    }
    // ---- O += P V: one k-step per 16 keys, 16 dim n-tiles.
#pragma unroll
    for (int np = 0; np < 4; ++np) {
      if (np * 16 >= kpw) break;
      const uint32_t a[4] = {pa[2 * np][0], pa[2 * np][1], pa[2 * np + 1][0], pa[2 * np + 1][1]};
      const int kr = mykey0 + np * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {  // pairs of 8-dim n-tiles
        const int chunk = dp * 2 + (lane >> 4);
        const uint32_t addr = vs + (chunk >> 3) * kDecHalfBytes + sw128(kr, chunk & 7);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(addr, b0, b1, b2, b3);
        mma_16816(acc[2 * dp], a, b0, b1);
        mma_16816(acc[2 * dp + 1], a, b2, b3);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[stage]);
  }

  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);

  // Merge the warps that split the keys of one m-tile (through the idle stage ring).
  asm volatile("bar.sync 1, %0;" ::"n"(kDecConsumerWarps * 32) : "memory");
  if (abort_flag) return;
  if (key_split > 1) {
    float* scratch = reinterpret_cast<float*>(smem) + warp * (16 * kMergeStride);
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      const int col = n * 8 + 2 * c4;
      *reinterpret_cast<float2*>(scratch + g4 * kMergeStride + col) = make_float2(acc[n][0], acc[n][1]);
      *reinterpret_cast<float2*>(scratch + (g4 + 8) * kMergeStride + col) = make_float2(acc[n][2], acc[n][3]);
    }
    if (c4 == 0) {
      merge_ml[warp][g4][0] = m_a; merge_ml[warp][g4][1] = l_a;
      merge_ml[warp][g4 + 8][0] = m_b; merge_ml[warp][g4 + 8][1] = l_b;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kDecConsumerWarps * 32) : "memory");
    if (kpart != 0) return;
    float mt_a = -INFINITY, mt_b = -INFINITY;
    for (int w = warp; w < warp + key_split; ++w) {
      mt_a = fmaxf(mt_a, merge_ml[w][g4][0]);
      mt_b = fmaxf(mt_b, merge_ml[w][g4 + 8][0]);
    }
    const float ba = mt_a == -INFINITY ? 0.f : mt_a, bb = mt_b == -INFINITY ? 0.f : mt_b;
    float la = 0.f, lb = 0.f;
#pragma unroll
    for (int n = 0; n < 16; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
    for (int w = warp; w < warp + key_split; ++w) {
      const float wa = exp2f(merge_ml[w][g4][0] - ba), wb = exp2f(merge_ml[w][g4 + 8][0] - bb);
      la += wa * merge_ml[w][g4][1];
      lb += wb * merge_ml[w][g4 + 8][1];
      const float* sc = reinterpret_cast<const float*>(smem) + w * (16 * kMergeStride);
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        const int col = n * 8 + 2 * c4;
        const float2 xa = *reinterpret_cast<const float2*>(sc + g4 * kMergeStride + col);
        const float2 xb = *reinterpret_cast<const float2*>(sc + (g4 + 8) * kMergeStride + col);
        acc[n][0] += wa * xa.x; acc[n][1] += wa * xa.y;
        acc[n][2] += wb * xb.x; acc[n][3] += wb * xb.y;
      }
    }
    m_a = mt_a; m_b = mt_b; l_a = la; l_b = lb;
  }

  // ---- write rows ja (g4) and jb (g4 + 8)
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int j = half ? jb : ja;
    if (j >= qrows) continue;
    const float m = half ? m_b : m_a, l = half ? l_b : l_a;
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const int tq = j / GROUP, head = h * GROUP + j % GROUP;
    if (nsplit == 1) {
      __nv_bfloat16* o = p.out + (static_cast<int64_t>(q0 + tq) * p.heads + head) * D;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        const int col = n * 8 + 2 * c4;
        *reinterpret_cast<uint32_t*>(o + col) = pack_bf16(acc[n][2 * half] * inv, acc[n][2 * half + 1] * inv);
      }
    } else {
      const int64_t rec = static_cast<int64_t>(pbase + tq) * p.heads + head;
      float* o = p.ws_out + rec * D;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        const int col = n * 8 + 2 * c4;
        *reinterpret_cast<float2*>(o + col) = make_float2(acc[n][2 * half] * inv, acc[n][2 * half + 1] * inv);
      }
      if (c4 == 0) p.ws_lse[rec] = l > 0.f ? m + log2f(l) : -INFINITY;
    }
  }
}

// Merge the splits of every multi-split decode row: out = sum_s w_s o_s / sum_s w_s
// with w_s = 2^(lse_s - max lse). One CTA per (split-0 item, KV head); each warp merges
// one query row, lane l owning dims 4l..4l+3, so every split's loads are in flight at once.
constexpr int kCombineMaxSplits = 8;

template <int GROUP>
__global__ void __launch_bounds__(128) decode_combine_kernel(AttentionParams p) {
  constexpr int D = 128;
  pdl_wait();  // the kernel ahead (decode, or prefill, which completes after decode) has finished
  if (p.counts != nullptr && static_cast<int>(blockIdx.x) >= p.counts[0]) return;
  const int32_t* item = p.decode_items + 4 * blockIdx.x;
  if (item[1] != 0 || item[3] <= 1) return;
  const int row = item[0], pbase = item[2], nsplit = item[3];
  const int h = blockIdx.y;
  const int q0 = p.cu_seq_q[row];
  const int count = p.cu_seq_q[row + 1] - q0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int j = warp; j < count * GROUP; j += 4) {
    const int tq = j / GROUP, head = h * GROUP + j % GROUP;
    float mx = -INFINITY;
    for (int s0 = 0; s0 < nsplit; s0 += 32) {
      const int s = s0 + lane;
      const float v = s < nsplit ? p.ws_lse[static_cast<int64_t>(pbase + s * count + tq) * p.heads + head] : -INFINITY;
      mx = fmaxf(mx, warp_max(v));
    }
    const float base = mx == -INFINITY ? 0.f : mx;
    float4 num = make_float4(0.f, 0.f, 0.f, 0.f);
    float den = 0.f;
    for (int s0 = 0; s0 < nsplit; s0 += kCombineMaxSplits) {
      const int n = min(kCombineMaxSplits, nsplit - s0);
      float4 part[kCombineMaxSplits];
      float w[kCombineMaxSplits];
#pragma unroll
      for (int i = 0; i < kCombineMaxSplits; ++i) {
        if (i < n) {
          const int64_t rec = static_cast<int64_t>(pbase + (s0 + i) * count + tq) * p.heads + head;
          w[i] = p.ws_lse[rec];
          part[i] = reinterpret_cast<const float4*>(p.ws_out + rec * D)[lane];
        }
      }
#pragma unroll
      for (int i = 0; i < kCombineMaxSplits; ++i) {
        if (i < n) {
          const float wi = exp2f(w[i] - base);
          den += wi;
          num.x += wi * part[i].x; num.y += wi * part[i].y; num.z += wi * part[i].z; num.w += wi * part[i].w;
        }
      }
    }
    const float inv = den > 0.f ? 1.f / den : 0.f;
    uint2 packed;
    packed.x = pack_bf16(num.x * inv, num.y * inv);
    packed.y = pack_bf16(num.z * inv, num.w * inv);
    reinterpret_cast<uint2*>(p.out + (static_cast<int64_t>(q0 + tq) * p.heads + head) * D)[lane] = packed;
  }
}

}  // namespace hb
