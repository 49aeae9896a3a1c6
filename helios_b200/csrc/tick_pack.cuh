// Kernel (a): GPU-side tick packing.
//
// One scheduler tick selects rows (requests) and a token count per row. The
// reference builds the attention metadata for that selection in Python lists
// (PackedBatchCache.prepare_packed, src/helios/runtime/qwen3/paged_cache.py:418-494;
// PagedBatchCache.prepare, :221-270) and copies each list to the device. Here the
// host uploads only O(rows + new pages) integers and one CTA expands them:
//
//   * page updates are applied to a device-resident page arena
//     ([slots, arena_width] int32, one slot per live request cache);
//   * block-scans over rows give cu_seq_q, cu_seq_k, seqused_k, logit offsets and
//     the attention work-list offsets;
//   * block_table[r, j] = arena[slot_r, j] for j < n_pages_r, else 0;
//   * per token: position = length_r + i, write slot = page(pos / P) * P + pos % P,
//     and the owning row;
//   * logit_indices: the trailing logit_count_r tokens of each row;
//   * the attention work lists: split-K items for decode-class rows
//     (count <= decode_max_tokens) and, for prefill-class rows, pairs of adjacent
//     query tiles (2i, 2i+1) of a row with m tiles. Tiles of at most 32 tokens
//     (GROUP >= 4) read the same 64-key tiles, so the two stay busy together; larger
//     tiles differ by at most two key tiles;
//   * shared-prefix groups: consecutive single-token decode rows whose block tables
//     start with the same shared_len keys (pages restored by aliasing) form a group. The
//     group's first row carries group_rows = n. Its keys [0, shared_len) are split every
//     prefix_split_keys keys once for all n rows: prefix items, each up to two query tiles
//     (2 x prefill_tile_tokens consecutive rows of the group, one token each) against one
//     split of the shared pages, run on the tensor cores by the prefill kernel; each row's
//     own decode items cover only [shared_len, end). The row's partial records are the
//     prefix splits, then its tail splits, merged by the split combine.
//
// Decode item (6 int32): row, first key, end key, record base of the item (row record base
// + split * count), splits of the row, 0.
// Prefix item (5 int32): first row, rows (<= 2 x prefill_tile_tokens), first key, end key,
// prefix split index s (member i's record: row_records[first row + i] + s).
// Every output write is bounded by the capacity the host sized it for; an entry
// that would fall outside is skipped and reported in the status word.
#pragma once

#include "attention_decode.cuh"  // kDecodeItemInts: the decode item layout
#include "hb_common.cuh"

namespace hb {

constexpr int kTickRowFields = 7;  // slot, length, count, logit_count, n_pages, shared_len, group_rows

struct TickPackParams {
  const int32_t* rows;     // [B][kTickRowFields]
  const int32_t* updates;  // [U][3] slot, page position, page index
  int32_t* arena;          // [slots][arena_width]
  int32_t num_rows, num_updates, arena_width, arena_slots, page_size, width, num_pages;
  int32_t decode_max_tokens, split_keys, prefill_tile_tokens, prefix_split_keys;
  int32_t* block_table;    // [B][width]
  int32_t* cu_seq_q;       // [B+1]
  int32_t* cu_seq_k;       // [B+1]
  int32_t* seqused_k;      // [B]
  int64_t* positions;      // [T]
  int64_t* write_slots;    // [T]
  int32_t* token_row;      // [T]
  int64_t* logit_indices;  // [logit_capacity]
  int32_t* decode_items;   // [decode_capacity][kDecodeItemInts] (above)
  int32_t* prefill_items;  // [prefill_capacity][3] row, first tile start, second tile start or -1
  int32_t total_tokens, logit_capacity, decode_capacity, prefill_capacity;
  int32_t* counts;         // optional [4]: decode items, prefill pairs, partial records, prefix items (capped)
  int32_t* row_records;    // [B+1] first partial record of each row (exclusive prefix)
  int32_t* prefix_items;   // [prefix_capacity][kPrefixItemInts] (above)
  int32_t prefix_capacity;
};

constexpr int kTickThreads = 1024;

__device__ __forceinline__ int row_splits(int end, int split_keys) { return (end + split_keys - 1) / split_keys; }

// A decode row's own keys: the nearest whole number of split_keys (at least one), cut into
// near-equal parts on 64-key boundaries, so no row ends in a sliver of a split (a unit of a
// few keys costs a whole CTA's start and merge). split_keys >= 256, so every part holds at
// least 170 keys.
__device__ __forceinline__ int tail_split_count(int keys, int split_keys) {
  return max(1, (keys + split_keys / 2) / split_keys);
}
__device__ __forceinline__ int tail_split_start(int keys, int n, int k) {
  return k >= n ? keys : static_cast<int>((static_cast<int64_t>(keys) * k / n) & ~int64_t(63));
}

// Decode items, prefix items and partial records of row r (see the header).
struct RowWork {
  int items, records, prefix_splits, tail_splits, prefix_items;
};
__device__ __forceinline__ RowWork row_work(const TickPackParams& p, int r) {
  const int32_t* row = p.rows + kTickRowFields * r;
  const int32_t end = row[1] + row[2], cnt = row[2], shared = row[5], group = row[6];
  RowWork w{0, 0, 0, 0, 0};
  if (cnt > p.decode_max_tokens) return w;
  if (shared > 0) {
    const int pair_rows = 2 * p.prefill_tile_tokens;
    w.prefix_splits = row_splits(shared, p.prefix_split_keys);
    w.tail_splits = tail_split_count(end - shared, p.split_keys);
    w.items = w.tail_splits;
    w.records = (w.prefix_splits + w.tail_splits) * cnt;
    w.prefix_items = group > 0 ? ((group + pair_rows - 1) / pair_rows) * w.prefix_splits : 0;
  } else {
    w.tail_splits = tail_split_count(end, p.split_keys);
    w.items = w.tail_splits;
    w.records = w.tail_splits * cnt;
  }
  return w;
}
__device__ __forceinline__ int row_prefill_items(int count, int tile_tokens) {
  return ((count + tile_tokens - 1) / tile_tokens + 1) / 2;  // tiles, paired
}

__global__ void __launch_bounds__(kTickThreads) tick_pack_kernel(TickPackParams p) {
  extern __shared__ int32_t sm[];
  const int B = p.num_rows;
  // Exclusive offsets per row, B+1 entries each.
  int32_t* q_off = sm;
  int32_t* k_off = q_off + (B + 1);
  int32_t* l_off = k_off + (B + 1);
  int32_t* d_off = l_off + (B + 1);
  int32_t* r_off = d_off + (B + 1);
  int32_t* f_off = r_off + (B + 1);
  int32_t* x_off = f_off + (B + 1);  // prefix items
  __shared__ int32_t warp_tot[32][7];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // 1. Page-arena updates (pages acquired or restored since the last tick).
  for (int u = tid; u < p.num_updates; u += kTickThreads) {
    const int32_t slot = p.updates[3 * u], pos = p.updates[3 * u + 1], page = p.updates[3 * u + 2];
    if (slot < 0 || slot >= p.arena_slots || pos < 0 || pos >= p.arena_width || page < 0 || page >= p.num_pages) {
      raise_status(kStatusBadPage);
      continue;
    }
    p.arena[static_cast<int64_t>(slot) * p.arena_width + pos] = page;
  }

  // 2. Block scan over rows. Each thread owns a contiguous chunk of rows.
  const int per = (B + kTickThreads - 1) / kTickThreads;
  const int r0 = min(B, tid * per), r1 = min(B, r0 + per);
  int32_t s[7] = {0, 0, 0, 0, 0, 0, 0};
  for (int r = r0; r < r1; ++r) {
    const int32_t len = p.rows[kTickRowFields * r + 1], cnt = p.rows[kTickRowFields * r + 2];
    const int32_t lc = p.rows[kTickRowFields * r + 3];
    const int32_t end = len + cnt;
    s[0] += cnt;
    s[1] += end;
    s[2] += lc;
    if (cnt <= p.decode_max_tokens) {
      const RowWork w = row_work(p, r);
      s[3] += w.items;
      s[4] += w.records;
      s[6] += w.prefix_items;
    } else {
      s[5] += row_prefill_items(cnt, p.prefill_tile_tokens);
    }
  }
  int32_t incl[7];
#pragma unroll
  for (int f = 0; f < 7; ++f) {
    int32_t v = s[f];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t n = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += n;
    }
    incl[f] = v;
    if (lane == 31) warp_tot[warp][f] = v;
  }
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int f = 0; f < 7; ++f) {
      int32_t v = warp_tot[lane][f];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int32_t n = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += n;
      }
      warp_tot[lane][f] = v;  // inclusive over warps
    }
  }
  __syncthreads();
  int32_t base[7];
#pragma unroll
  for (int f = 0; f < 7; ++f) base[f] = (warp ? warp_tot[warp - 1][f] : 0) + incl[f] - s[f];
  for (int r = r0; r < r1; ++r) {
    const int32_t len = p.rows[kTickRowFields * r + 1], cnt = p.rows[kTickRowFields * r + 2];
    const int32_t lc = p.rows[kTickRowFields * r + 3];
    const int32_t end = len + cnt;
    q_off[r] = base[0];
    k_off[r] = base[1];
    l_off[r] = base[2];
    d_off[r] = base[3];
    r_off[r] = base[4];
    f_off[r] = base[5];
    x_off[r] = base[6];
    base[0] += cnt;
    base[1] += end;
    base[2] += lc;
    if (cnt <= p.decode_max_tokens) {
      const RowWork w = row_work(p, r);
      base[3] += w.items;
      base[4] += w.records;
      base[6] += w.prefix_items;
    } else {
      base[5] += row_prefill_items(cnt, p.prefill_tile_tokens);
    }
  }
  if (tid == kTickThreads - 1) {
    q_off[B] = base[0];
    k_off[B] = base[1];
    l_off[B] = base[2];
    d_off[B] = base[3];
    r_off[B] = base[4];
    f_off[B] = base[5];
    x_off[B] = base[6];
    if (p.counts != nullptr) {  // work-list sizes for launches sized to capacities
      p.counts[0] = min(base[3], p.decode_capacity);
      p.counts[1] = min(base[5], p.prefill_capacity);
      p.counts[2] = base[4];
      p.counts[3] = min(base[6], p.prefix_capacity);
    }
  }
  __syncthreads();

  // 3. Row-level outputs, logit rows and attention work items.
  for (int r = tid; r <= B; r += kTickThreads) {
    p.cu_seq_q[r] = q_off[r];
    p.cu_seq_k[r] = k_off[r];
    if (p.row_records != nullptr) p.row_records[r] = r_off[r];
  }
  for (int r = tid; r < B; r += kTickThreads) {
    const int32_t len = p.rows[kTickRowFields * r + 1], cnt = p.rows[kTickRowFields * r + 2];
    const int32_t lc = p.rows[kTickRowFields * r + 3];
    const int32_t end = len + cnt;
    p.seqused_k[r] = end;
    for (int i = 0; i < lc; ++i) {
      if (l_off[r] + i >= p.logit_capacity) { raise_status(kStatusBadRow); break; }
      p.logit_indices[l_off[r] + i] = static_cast<int64_t>(q_off[r + 1] - lc + i);
    }
    if (cnt <= p.decode_max_tokens) {
      const RowWork w = row_work(p, r);
      const int32_t shared = p.rows[kTickRowFields * r + 5], group = p.rows[kTickRowFields * r + 6];
      const int nsplit = w.prefix_splits + w.tail_splits;
      int at = d_off[r];
      for (int k = 0; k < w.tail_splits; ++k, ++at) {  // this row's own keys [shared, end)
        if (at >= p.decode_capacity) { raise_status(kStatusBadRow); break; }
        int32_t* it = p.decode_items + kDecodeItemInts * at;
        const int own = end - shared;
        it[0] = r;
        it[1] = shared + tail_split_start(own, w.tail_splits, k);
        it[2] = shared + tail_split_start(own, w.tail_splits, k + 1);
        it[3] = r_off[r] + (w.prefix_splits + k) * cnt;
        it[4] = nsplit;
        it[5] = 0;
      }
      if (group > 0) {  // the group's shared keys [0, shared), once for its `group` rows
        const int pair_rows = 2 * p.prefill_tile_tokens;
        int px = x_off[r];
        for (int k = 0; k < w.prefix_splits; ++k) {
          for (int i = 0; i < group; i += pair_rows, ++px) {
            if (px >= p.prefix_capacity) { raise_status(kStatusBadRow); break; }
            int32_t* it = p.prefix_items + kPrefixItemInts * px;
            it[0] = r + i;
            it[1] = min(pair_rows, group - i);
            it[2] = k * p.prefix_split_keys;
            it[3] = min(shared, (k + 1) * p.prefix_split_keys);
            it[4] = k;
          }
        }
      }
    } else {
      const int tiles = (cnt + p.prefill_tile_tokens - 1) / p.prefill_tile_tokens;
      for (int i = 0; i < (tiles + 1) / 2; ++i) {
        if (f_off[r] + i >= p.prefill_capacity) { raise_status(kStatusBadRow); break; }
        int32_t* it = p.prefill_items + 3 * (f_off[r] + i);
        it[0] = r;
        it[1] = 2 * i * p.prefill_tile_tokens;
        it[2] = 2 * i + 1 < tiles ? (2 * i + 1) * p.prefill_tile_tokens : -1;
      }
    }
  }

  // 4. Block table rows from the arena, zero-padded to `width`.
  const int64_t cells = static_cast<int64_t>(B) * p.width;
  for (int64_t c = tid; c < cells; c += kTickThreads) {
    const int r = static_cast<int>(c / p.width), j = static_cast<int>(c % p.width);
    const int32_t slot = p.rows[kTickRowFields * r], npages = p.rows[kTickRowFields * r + 4];
    int32_t v = 0;
    if (j < npages) {
      v = (j < p.arena_width && slot >= 0 && slot < p.arena_slots)
              ? p.arena[static_cast<int64_t>(slot) * p.arena_width + j]
              : -1;
      if (v < 0 || v >= p.num_pages) {
        raise_status(kStatusBadPage);
        v = 0;
      }
    }
    p.block_table[c] = v;
  }

  // 5. Per-token positions, KV write slots and owning rows.
  for (int t = tid; t < p.total_tokens && t < q_off[B]; t += kTickThreads) {
    int lo = 0, hi = B;  // largest r with q_off[r] <= t
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (q_off[mid] <= t) lo = mid; else hi = mid;
    }
    const int r = lo;
    const int32_t slot = p.rows[kTickRowFields * r], len = p.rows[kTickRowFields * r + 1];
    const int32_t npages = p.rows[kTickRowFields * r + 4];
    const int32_t pos = len + (t - q_off[r]);
    const int32_t pidx = pos / p.page_size;
    int32_t page = 0;
    if (pidx < npages && pidx < p.arena_width && slot >= 0 && slot < p.arena_slots) {
      page = p.arena[static_cast<int64_t>(slot) * p.arena_width + pidx];
    } else {
      raise_status(kStatusBadPage);
    }
    p.positions[t] = pos;
    p.write_slots[t] = static_cast<int64_t>(page) * p.page_size + (pos % p.page_size);
    p.token_row[t] = r;
  }
}

}  // namespace hb
