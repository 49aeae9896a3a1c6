// Kernel (c), decode rows: split-K paged GQA attention (flash-decoding).
//
// Replaces the decode part of the reference's paged varlen attention call
// (PackedBatchCache.attend -> varlen_attn(..., block_table, seqused_k,
// window_size=(-1, 0), num_splits=1), src/helios/runtime/qwen3/paged_cache.py:501-520;
// PagedBatchCache.attend, :301-333). The reference runs with num_splits=1, which
// leaves most SMs idle when a tick holds few long decode rows; here the work unit is
// (row, split of split_keys keys, KV head): see the decode item layout in tick_pack.cuh. Keys
// that rows share through restored pages run as prefix items on the tensor cores instead
// (attention_prefill.cuh); their records join the rows' own splits in the combine.
//
// Semantics (bottom-right causal, as the reference's window_size=(-1, 0)): query
// i of a row with `count` queries and `end = seqused_k` keys sits at key position
// end - count + i and sees keys 0..that position. Scale is applied to q.k in fp32.
//
// A unit is worked by a producer warp and 4 consumer warps over a 3-stage ring of 32 KB
// stages: the producer streams the 64-key K and V tiles of one KV head ([64 keys][128 d]
// bf16, two 128B-swizzled boxes each) from the page the block table names; the consumers
// run m16n8k16 warp MMAs (decode_tile). All query rows of the GQA group (count * group <=
// 64) share every K/V tile, so K/V bytes cross HBM once per (row, KV head). With 16 query
// rows, the 4 warps split the 64 keys of a tile and merge their (max, sum, acc) at the
// unit's end through shared memory (decode_merge); with 64 rows each warp owns 16 rows.
// Results of a multi-split row go to a float workspace as (normalised output,
// log2-sum-exp) and are merged by decode_combine_kernel. Two grids:
//   decode_attention_kernel   one CTA (160 threads) per unit, two CTAs per SM: while one
//                             CTA starts or merges, the other streams. Used alone.
//   decode_persistent_kernel  at most one CTA per SM, each two independent halves of the
//                             above walking units claimed from a global ticket; the
//                             producer tags the ring stage of each unit's first tile with
//                             the unit's metadata and streams across unit boundaries, and a
//                             unit's last stage serves as its merge scratch. Used when prefill
//                             work is launched behind it: its CTAs past decode_ctas exit at
//                             once and leave their SMs to the prefill grid, which then runs
//                             beside the decode CTAs (decode is HBM-bound, prefill
//                             tensor-bound).
#pragma once

#include "hb_common.cuh"

namespace hb {

struct AttentionParams {
  const __nv_bfloat16* q;   // [T, H, D]
  __nv_bfloat16* out;       // [T, H, D]
  const int32_t* block_table;  // [B, W]
  const int32_t* cu_seq_q;     // [B+1]
  const int32_t* seqused_k;    // [B]
  const int32_t* decode_items;   // [n][6] row, first key, end key, record base, splits of the row, 0
  const int32_t* row_records;    // [rows+1] first partial record of each row
  int32_t num_rows;
  int32_t record_capacity;       // partial records the workspace holds
  const int32_t* prefill_items;  // [n][3] row, query start of tile 2i, of tile 2i+1 or -1
  // [n][5] first row, rows, first key, end key, prefix split index: query tiles of the single
  // tokens of consecutive rows sharing a prefix, against one split of the shared keys
  const int32_t* prefix_items;
  // Optional device counts {decode items, prefill pairs, partial records, prefix items}
  // written by the tick-pack kernel: when set, grids are sized to capacities and CTAs past a
  // count exit (a launch that stays valid, e.g. in a CUDA graph, while the work list changes).
  const int32_t* counts;
  // Set when the prefill kernel is launched right behind the decode kernel (programmatic
  // dependent launch): it then reads q, K and V without waiting (the decode kernel waited
  // for them before triggering), and one of its CTAs waits for the decode grid before
  // exiting, so the prefill grid completes after the decode grid.
  int32_t prefill_after_decode;
  // Set when the (per-unit) decode grid is launched right behind the prefix grid: it reads q,
  // K and V without waiting (the prefix grid waited for them before triggering), and its last
  // CTA waits for the prefix grid, so the decode grid completes after it.
  int32_t decode_after_prefix;
  int32_t num_decode;   // decode items (without counts)
  int32_t decode_ctas;  // decode CTAs that stay when prefill work runs beside the decode grid
  // The next unclaimed decode unit: zero before the decode grid, reset to zero by the
  // combine grid behind it (so a workspace that starts zeroed stays ready for the next call).
  int32_t* work_counter;
  float* ws_out;   // [records, H, D]
  float* ws_lse;   // [records, H]
  int32_t width, num_pages, page_size, heads, kv_heads, split_keys, tokens;
  int32_t num_prefill;  // prefill items (the kernel walks them from the last, heaviest, first)
  int32_t num_prefix;   // prefix items (without counts)
  float scale_log2;  // softmax scale * log2(e)
};

constexpr int kDecTileKeys = 64;
constexpr int kDecStages = 3;
constexpr int kDecConsumerWarps = 4;
constexpr int kDecSubThreads = (kDecConsumerWarps + 1) * 32;          // one unit's warps
constexpr int kDecSubs = 2;                                            // halves of a persistent CTA
constexpr int kDecPersistentThreads = kDecSubs * kDecSubThreads;
constexpr uint32_t kDecHalfBytes = kDecTileKeys * 128;                 // one [64][64] bf16 box
constexpr uint32_t kDecTileBytes = 2 * kDecHalfBytes;                  // K or V tile, D = 128
constexpr uint32_t kDecStageBytes = 2 * kDecTileBytes;                 // K + V
constexpr uint32_t kDecRingBytes = kDecStages * kDecStageBytes;
constexpr uint32_t kDecSmemBytes = kDecRingBytes + 1024;               // + alignment slack
constexpr uint32_t kDecPersistentSmemBytes = kDecSubs * kDecRingBytes + 1024;
constexpr int kMergeStride = 132;  // floats per row of the split merge scratch (padded: no bank conflicts)
// The key-split merge writes the accumulators of at most 3 warps into one stage.
static_assert((kDecConsumerWarps - 1) * 16 * kMergeStride * 4 <= kDecStageBytes, "merge scratch fits a stage");

// What a consumer warp needs to know about its unit.
struct DecodeUnit {
  int h, row, q0, count, end, kb, ke, n_tiles, rec, nsplit;
  int qrows, key_split, kpw, mt, kpart;
};

constexpr int kDecodeItemInts = 6;
constexpr int kPrefixItemInts = 5;

// From decode item `it` (the tick-pack layout), q0 / count / end of its row.
template <int GROUP>
__device__ __forceinline__ DecodeUnit decode_unit(const AttentionParams& p, int h, const int4& ia, const int2& ib,
                                                  int q0, int count, int end, int consumer_warp) {
  DecodeUnit u;
  u.h = h;
  u.row = ia.x;
  u.kb = ia.y;
  u.ke = ia.z;
  u.rec = ia.w;
  u.nsplit = ib.x;
  u.q0 = q0;
  u.count = count;
  u.end = end;
  u.n_tiles = (u.ke - u.kb + kDecTileKeys - 1) / kDecTileKeys;
  u.qrows = count * GROUP;
  const int m_tiles = u.qrows <= 16 ? 1 : (u.qrows <= 32 ? 2 : 4);
  u.key_split = kDecConsumerWarps / m_tiles;  // warps sharing one m-tile
  u.kpw = kDecTileKeys / u.key_split;         // keys per warp per tile
  u.mt = consumer_warp / u.key_split;
  u.kpart = consumer_warp % u.key_split;
  return u;
}

// The decode item as two vectors plus its row's query range and key end.
__device__ __forceinline__ void decode_item(const AttentionParams& p, int index, int4& ia, int2& ib, int& q0,
                                            int& count, int& end) {
  const int32_t* it = p.decode_items + kDecodeItemInts * index;
  ia = make_int4(it[0], it[1], it[2], it[3]);
  ib = make_int2(it[4], it[5]);
  q0 = p.cu_seq_q[ia.x];
  count = p.cu_seq_q[ia.x + 1] - q0;
  end = p.seqused_k[ia.x];
}

// Key position limit of query row j (bottom-right causal).
template <int GROUP>
__device__ __forceinline__ int decode_qpos(const DecodeUnit& u, int j) {
  if (j >= u.qrows) return -1;
  return u.end - u.count + j / GROUP;
}

// Query A-fragments for rows mt*16 + g4 and +8 of the unit: 8 k-steps of 16 dims.
template <int GROUP>
__device__ __forceinline__ void decode_load_q(const AttentionParams& p, const DecodeUnit& u, int lane,
                                              uint32_t (&qa)[8][4]) {
  constexpr int D = 128;
  const int g4 = lane >> 2, c4 = lane & 3;
  const int ja = u.mt * 16 + g4, jb = ja + 8;
  const __nv_bfloat16* pa =
      ja < u.qrows ? p.q + (static_cast<int64_t>(u.q0 + ja / GROUP) * p.heads + u.h * GROUP + ja % GROUP) * D : nullptr;
  const __nv_bfloat16* pb =
      jb < u.qrows ? p.q + (static_cast<int64_t>(u.q0 + jb / GROUP) * p.heads + u.h * GROUP + jb % GROUP) * D : nullptr;
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    const int d0 = kk * 16 + 2 * c4;
    qa[kk][0] = pa ? *reinterpret_cast<const uint32_t*>(pa + d0) : 0u;
    qa[kk][1] = pb ? *reinterpret_cast<const uint32_t*>(pb + d0) : 0u;
    qa[kk][2] = pa ? *reinterpret_cast<const uint32_t*>(pa + d0 + 8) : 0u;
    qa[kk][3] = pb ? *reinterpret_cast<const uint32_t*>(pb + d0 + 8) : 0u;
  }
}

// One 64-key K/V tile (stage at `stage`, first key key0) into the warp's online softmax
// state: S = Q K^T over the warp's keys, mask, rescale, O += P V.
template <int GROUP>
__device__ __forceinline__ void decode_tile(const AttentionParams& p, const DecodeUnit& u, uint8_t* stage, int key0,
                                            int lane, int qpos_a, int qpos_b, const uint32_t (&qa)[8][4],
                                            float (&acc)[16][4], float& m_a, float& m_b, float& l_a, float& l_b) {
  const int c4 = lane & 3;
  const uint32_t ks = smem_u32(stage);
  const uint32_t vs = ks + kDecTileBytes;
  const int kpw = u.kpw;
  const int mykey0 = u.kpart * kpw;  // within the tile
  // Keys at or past the split end may be stale or uninitialised pool memory:
  // zero their V rows (this warp only reads its own key range) so 0 * NaN cannot occur.
  if (key0 + kDecTileKeys > u.ke) {
    uint8_t* vgen = stage + kDecTileBytes;
    for (int kr = mykey0 + (lane >> 3); kr < mykey0 + kpw; kr += 4) {
      if (key0 + kr >= u.ke) {
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
      const bool ok = key + e < u.ke;
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
}

// The key-split merge of the unit's warps (called by all 4 consumer warps of the unit after
// a barrier; `scratch` holds (kDecConsumerWarps - 1) x 16 x kMergeStride floats, `ml` the
// warps' (max, sum) rows). Warps with kpart > 0 publish their state; the kpart 0 warp of each
// m-tile folds the others into its own. `sync` is the unit's consumer barrier.
template <typename Sync>
__device__ __forceinline__ void decode_merge(const DecodeUnit& u, int cw, int lane, float* scratch,
                                             float (*ml)[16][2], float (&acc)[16][4], float& m_a, float& m_b,
                                             float& l_a, float& l_b, Sync sync) {
  const int g4 = lane >> 2, c4 = lane & 3;
  const int key_split = u.key_split, mt = u.mt, kpart = u.kpart;
  if (kpart != 0) {
    float* mine = scratch + (mt * (key_split - 1) + kpart - 1) * (16 * kMergeStride);
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      const int col = n * 8 + 2 * c4;
      *reinterpret_cast<float2*>(mine + g4 * kMergeStride + col) = make_float2(acc[n][0], acc[n][1]);
      *reinterpret_cast<float2*>(mine + (g4 + 8) * kMergeStride + col) = make_float2(acc[n][2], acc[n][3]);
    }
  }
  if (c4 == 0) {
    ml[cw][g4][0] = m_a; ml[cw][g4][1] = l_a;
    ml[cw][g4 + 8][0] = m_b; ml[cw][g4 + 8][1] = l_b;
  }
  sync();
  if (kpart != 0) return;
  float mt_a = -INFINITY, mt_b = -INFINITY;
  for (int w = cw; w < cw + key_split; ++w) {
    mt_a = fmaxf(mt_a, ml[w][g4][0]);
    mt_b = fmaxf(mt_b, ml[w][g4 + 8][0]);
  }
  const float ba = mt_a == -INFINITY ? 0.f : mt_a, bb = mt_b == -INFINITY ? 0.f : mt_b;
  const float wa0 = exp2f(m_a - ba), wb0 = exp2f(m_b - bb);
  float la = wa0 * l_a, lb = wb0 * l_b;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    acc[n][0] *= wa0; acc[n][1] *= wa0;
    acc[n][2] *= wb0; acc[n][3] *= wb0;
  }
  for (int k = 1; k < key_split; ++k) {
    const int w = cw + k;
    const float wa = exp2f(ml[w][g4][0] - ba), wb = exp2f(ml[w][g4 + 8][0] - bb);
    la += wa * ml[w][g4][1];
    lb += wb * ml[w][g4 + 8][1];
    const float* sc = scratch + (mt * (key_split - 1) + k - 1) * (16 * kMergeStride);
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

// Rows mt*16 + g4 and +8 of the unit: bf16 output (one split) or a split record.
template <int GROUP>
__device__ __forceinline__ void decode_store(const AttentionParams& p, const DecodeUnit& u, int lane,
                                             const float (&acc)[16][4], float m_a, float m_b, float l_a, float l_b) {
  constexpr int D = 128;
  const int g4 = lane >> 2, c4 = lane & 3;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int j = u.mt * 16 + g4 + 8 * half;
    if (j >= u.qrows) continue;
    const float m = half ? m_b : m_a, l = half ? l_b : l_a;
    const float inv = l > 0.f ? 1.f / l : 0.f;
    const int tq = j / GROUP, head = u.h * GROUP + j % GROUP;
    if (u.nsplit == 1) {
      __nv_bfloat16* o = p.out + (static_cast<int64_t>(u.q0 + tq) * p.heads + head) * D;
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        const int col = n * 8 + 2 * c4;
        *reinterpret_cast<uint32_t*>(o + col) = pack_bf16(acc[n][2 * half] * inv, acc[n][2 * half + 1] * inv);
      }
    } else {
      if (u.rec + tq < 0 || u.rec + tq >= p.record_capacity) {
        raise_status(kStatusBadRow);
        continue;
      }
      const int64_t rec = static_cast<int64_t>(u.rec + tq) * p.heads + head;
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

// Issue one K/V tile (key `key` of `row`, KV head h) into `stage`; false on a bad page.
__device__ __forceinline__ bool decode_issue_tile(const AttentionParams& p, const CUtensorMap* kmap,
                                                  const CUtensorMap* vmap, uint8_t* stage, uint64_t* full, int row,
                                                  int h, int key, int& cached_pidx, int& cached_page) {
  const int pidx = key / p.page_size;
  if (pidx != cached_pidx) {  // one block-table read per page, not per key tile
    cached_page = pidx < p.width ? p.block_table[static_cast<int64_t>(row) * p.width + pidx] : -1;
    cached_pidx = pidx;
  }
  const int page = cached_page;
  if (page < 0 || page >= p.num_pages) {
    raise_status(kStatusBadPage);
    return false;
  }
  const int tok = page * p.page_size + (key % p.page_size);
  mbar_expect_tx(full, kDecStageBytes);
  tma_load_3d(stage, kmap, full, 0, h, tok);
  tma_load_3d(stage + kDecHalfBytes, kmap, full, 64, h, tok);
  tma_load_3d(stage + kDecTileBytes, vmap, full, 0, h, tok);
  tma_load_3d(stage + kDecTileBytes + kDecHalfBytes, vmap, full, 64, h, tok);
  return true;
}

template <int GROUP>
__global__ void __launch_bounds__(kDecSubThreads, 2) decode_attention_kernel(AttentionParams p,
                                                                         const __grid_constant__ CUtensorMap kmap,
                                                                         const __grid_constant__ CUtensorMap vmap) {
  extern __shared__ __align__(1024) uint8_t dsm[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full_bar[kDecStages], empty_bar[kDecStages];
  __shared__ int abort_flag;
  __shared__ float merge_ml[kDecConsumerWarps][16][2];

  // q, K and V from the norm/RoPE/append kernel ahead of this one (or, behind the prefix grid,
  // already complete: see decode_after_prefix).
  if (!p.decode_after_prefix || blockIdx.x == gridDim.x - 1) pdl_wait();
  pdl_trigger();  // the prefill kernel (or the split combine) may launch behind this grid
  // KV heads fastest: the CTAs of one item's heads run together and read the same pool rows
  // (each its own 256 bytes of every 2 KB token row).
  const int item = static_cast<int>(blockIdx.x) / p.kv_heads, head = static_cast<int>(blockIdx.x) % p.kv_heads;
  if (p.counts != nullptr && item >= p.counts[0]) return;  // past this tick's items
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int4 ia;
  int2 ib;
  int q0, count, end;
  decode_item(p, item, ia, ib, q0, count, end);
  const int row = ia.x;
  const DecodeUnit u = decode_unit<GROUP>(p, head, ia, ib, q0, count, end, warp);

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
      for (int t = 0; t < u.n_tiles; ++t) {
        const int stage = t % kDecStages;
        if (t >= kDecStages && !mbar_wait(&empty_bar[stage], ((t / kDecStages) - 1) & 1, &abort_flag)) break;
        if (!decode_issue_tile(p, &kmap, &vmap, smem + stage * kDecStageBytes, &full_bar[stage], row, u.h,
                               u.kb + t * kDecTileKeys, cached_pidx, cached_page)) {
          abort_flag = 1;
          break;
        }
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
  const int g4 = lane >> 2;
  uint32_t qa[8][4];
  decode_load_q<GROUP>(p, u, lane, qa);
  // Key position limit per query row (bottom-right causal) for rows g4, g4+8.
  const int ja = u.mt * 16 + g4, jb = ja + 8;
  const int qpos_a = decode_qpos<GROUP>(u, ja), qpos_b = decode_qpos<GROUP>(u, jb);
  float acc[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  for (int t = 0; t < u.n_tiles; ++t) {
    const int stage = t % kDecStages;
    if (!mbar_wait(&full_bar[stage], (t / kDecStages) & 1, &abort_flag)) break;
    decode_tile<GROUP>(p, u, smem + stage * kDecStageBytes, u.kb + t * kDecTileKeys, lane, qpos_a, qpos_b, qa, acc,
                       m_a, m_b, l_a, l_b);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[stage]);
  }
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);

  // Merge the warps that split the keys of one m-tile (through the idle stage ring).
  named_barrier_sync(1, kDecConsumerWarps * 32);
  if (abort_flag) return;
  if (u.key_split > 1) {
    decode_merge(u, warp, lane, reinterpret_cast<float*>(smem), merge_ml, acc, m_a, m_b, l_a, l_b,
                 [] { named_barrier_sync(1, kDecConsumerWarps * 32); });
    if (u.kpart != 0) return;
  }
  decode_store<GROUP>(p, u, lane, acc, m_a, m_b, l_a, l_b);
}

template <int GROUP>
__global__ void __launch_bounds__(kDecPersistentThreads, 1) decode_persistent_kernel(
    AttentionParams p, const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap) {
  extern __shared__ __align__(1024) uint8_t dsm[];
  uint8_t* smem_base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full_bars[kDecSubs][kDecStages], empty_bars[kDecSubs][kDecStages];
  __shared__ int abort_flag;
  __shared__ float merge_ml[kDecSubs][kDecConsumerWarps][16][2];
  // The unit whose first tile a stage holds, with its metadata: {unit, row, first key, end
  // key}, {record, splits, unused, first query}, {queries, keys}; unit -1: no more units.
  __shared__ int4 unit_meta[kDecSubs][kDecStages][3];

  pdl_wait();     // q, K and V from the norm/RoPE/append kernel ahead of this one
  pdl_trigger();  // the prefill kernel (or the split combine) may launch behind this grid
  const int n_items = p.counts != nullptr ? p.counts[0] : p.num_decode;
  const bool beside_prefill =
      (p.counts != nullptr ? p.counts[1] + p.counts[3] : p.num_prefill + p.num_prefix) > 0;
  const int active = beside_prefill ? min(static_cast<int>(gridDim.x), p.decode_ctas) : static_cast<int>(gridDim.x);
  if (static_cast<int>(blockIdx.x) >= active) return;  // the SM is left to the prefill grid
  const int units = n_items * p.kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = warp / (kDecConsumerWarps + 1), cw = warp % (kDecConsumerWarps + 1);
  uint8_t* smem = smem_base + sub * kDecRingBytes;
  uint64_t* full_bar = full_bars[sub];
  uint64_t* empty_bar = empty_bars[sub];
  int4* metas = &unit_meta[sub][0][0];  // ordered by the barrier operations around each access

  if (threadIdx.x == 0) {
    for (int h = 0; h < kDecSubs; ++h)
      for (int s = 0; s < kDecStages; ++s) {
        mbar_init(&full_bars[h][s], 1);
        mbar_init(&empty_bars[h][s], kDecConsumerWarps);
      }
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (cw == kDecConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      int it = 0;  // tiles issued by this half, across units
      bool ok = true;
      // Units are claimed two ahead and the next unit's metadata is loaded while this one's
      // tiles stream, so the ring keeps filling across unit boundaries.
      auto load_meta = [&](int unit, int4& a, int4& b, int4& c) {
        int4 ia;
        int2 ib;
        int q0, count, end;
        decode_item(p, unit / p.kv_heads, ia, ib, q0, count, end);
        a = make_int4(unit, ia.x, ia.y, ia.z);
        b = make_int4(ia.w, ib.x, ib.y, q0);
        c = make_int4(count, end, 0, 0);
      };
      int u = atomicAdd(p.work_counter, 1);
      int u_next = atomicAdd(p.work_counter, 1);
      int4 a = make_int4(0, 0, 0, 0), b = a, c = a;
      if (u < units) load_meta(u, a, b, c);
      while (ok && u < units) {
        int4 na = make_int4(0, 0, 0, 0), nb = na, nc = na;
        int u_after = units;
        if (u_next < units) {  // issued now, used after this unit's tiles
          load_meta(u_next, na, nb, nc);
          u_after = atomicAdd(p.work_counter, 1);
        }
        const int h = u % p.kv_heads, row = a.y;
        const int kb = a.z, ke = a.w;
        const int n_tiles = (ke - kb + kDecTileKeys - 1) / kDecTileKeys;
        int cached_pidx = -1, cached_page = -1;
        for (int t = 0; t < n_tiles; ++t) {
          const int stage = it % kDecStages;
          if (it >= kDecStages && !mbar_wait(&empty_bar[stage], ((it / kDecStages) - 1) & 1, &abort_flag)) {
            ok = false;
            break;
          }
          if (t == 0) {  // published by the expect_tx arrive of the tile's issue
            metas[3 * stage] = a;
            metas[3 * stage + 1] = b;
            metas[3 * stage + 2] = c;
          }
          if (!decode_issue_tile(p, &kmap, &vmap, smem + stage * kDecStageBytes, &full_bar[stage], row, h,
                                 kb + t * kDecTileKeys, cached_pidx, cached_page)) {
            abort_flag = 1;
            ok = false;
            break;
          }
          ++it;
        }
        u = u_next;
        u_next = u_after;
        a = na;
        b = nb;
        c = nc;
      }
      // End of work: a stage tagged -1, completed by a plain arrive (no bytes).
      if (ok) {
        const int stage = it % kDecStages;
        if (it < kDecStages || mbar_wait(&empty_bar[stage], ((it / kDecStages) - 1) & 1, &abort_flag)) {
          metas[3 * stage] = make_int4(-1, 0, 0, 0);
          mbar_arrive(&full_bar[stage]);
        } else {
          ok = false;
        }
      }
      // Never leave with copies in flight: wait (bounded) for every issued tile.
      if (!ok || abort_flag) {
        for (int j = max(0, it - kDecStages); j < it; ++j) mbar_drain(&full_bar[j % kDecStages], (j / kDecStages) & 1);
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int g4 = lane >> 2;
  const auto sync = [sub] { named_barrier_sync(1 + sub, kDecConsumerWarps * 32); };
  int it = 0;  // tiles consumed by this half, across units
  while (true) {
    // The stage of the next unit's first tile (or the end tag). Every consumer warp of the
    // half meets here, so an abort is seen by all of them at once.
    const bool got = mbar_wait(&full_bar[it % kDecStages], (it / kDecStages) & 1, &abort_flag);
    sync();
    if (!got || abort_flag) break;
    const int4 ma = metas[3 * (it % kDecStages)];
    if (ma.x < 0) break;
    const int4 mb = metas[3 * (it % kDecStages) + 1];
    const int4 mc = metas[3 * (it % kDecStages) + 2];
    const DecodeUnit u = decode_unit<GROUP>(p, ma.x % p.kv_heads, make_int4(ma.y, ma.z, ma.w, mb.x),
                                            make_int2(mb.y, mb.z), mb.w, mc.x, mc.y, cw);
    uint32_t qa[8][4];
    decode_load_q<GROUP>(p, u, lane, qa);
    const int ja = u.mt * 16 + g4, jb = ja + 8;
    const int qpos_a = decode_qpos<GROUP>(u, ja), qpos_b = decode_qpos<GROUP>(u, jb);
    float acc[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
    for (int t = 0; t < u.n_tiles; ++t) {
      const int stage = (it + t) % kDecStages;
      if (t > 0 && !mbar_wait(&full_bar[stage], ((it + t) / kDecStages) & 1, &abort_flag)) break;
      decode_tile<GROUP>(p, u, smem + stage * kDecStageBytes, u.kb + t * kDecTileKeys, lane, qpos_a, qpos_b, qa, acc,
                         m_a, m_b, l_a, l_b);
      __syncwarp();
      // The unit's last stage stays with the consumers when it becomes the merge scratch.
      if (lane == 0 && !(t == u.n_tiles - 1 && u.key_split > 1)) mbar_arrive(&empty_bar[stage]);
    }
    const int last_stage = (it + u.n_tiles - 1) % kDecStages;
    it += u.n_tiles;
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
    // Every consumer warp of the half gets here (waits are bounded); the abort flag is read
    // after the barrier, so all of them leave together.
    sync();
    if (abort_flag) break;
    if (u.key_split > 1) {
      decode_merge(u, cw, lane, reinterpret_cast<float*>(smem + last_stage * kDecStageBytes), merge_ml[sub], acc, m_a,
                   m_b, l_a, l_b, sync);
      // The scratch is read; hand the stage back to the producer (after ordering these
      // generic accesses before its next TMA fill).
      fence_proxy_async_smem();
      sync();
      if (lane == 0) mbar_arrive(&empty_bar[last_stage]);
      if (u.kpart != 0) continue;
    }
    decode_store<GROUP>(p, u, lane, acc, m_a, m_b, l_a, l_b);
  }
}

// Merge the splits of every multi-split decode row: out = sum_s w_s o_s / sum_s w_s
// with w_s = 2^(lse_s - max lse). One CTA per (row, KV head): the row's records are
// row_records[r] .. row_records[r + 1], split s of query token tq at + s * count + tq (rows
// with one split wrote their output directly; prefill rows have none). Each warp merges one
// query row, lane l owning dims 4l..4l+3, so every split's loads are in flight at once.
constexpr int kCombineMaxSplits = 8;

template <int GROUP>
__global__ void __launch_bounds__(128) decode_combine_kernel(AttentionParams p) {
  constexpr int D = 128;
  pdl_wait();  // the kernel ahead (decode, or prefill, which completes after decode) has finished
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) *p.work_counter = 0;  // for the next call
  const int row = blockIdx.x, h = blockIdx.y;
  const int q0 = p.cu_seq_q[row];
  const int count = p.cu_seq_q[row + 1] - q0;
  const int pbase = p.row_records[row];
  const int records = p.row_records[row + 1] - pbase;
  if (count <= 0 || records <= count) return;  // one split (written directly) or a prefill row
  if (pbase < 0 || pbase + records > p.record_capacity) {
    if (threadIdx.x == 0) raise_status(kStatusBadRow);
    return;
  }
  const int nsplit = records / count;
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
