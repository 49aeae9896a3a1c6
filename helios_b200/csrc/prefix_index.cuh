// Device-resident prefix-cache index: chained block hashes and a digest hash table.
//
// Replaces the host side of the reference's prefix lookup on the admission path
// (src/helios/runtime/prefix_cache.py:86-110 hash_token_blocks / build_token_blocks, and the
// probe loop of PrefixCache.longest_prefix, :208-222). A prompt is cut into blocks of
// block_size tokens (the last one may be partial); block i's key is
//     SHA-256(digest of block i-1 || "[t0,t1,...]")
// with the token ids written in decimal ASCII, comma-separated, no spaces (the JSON the
// reference hashes), and no parent bytes for block 0. SHA-256 itself follows FIPS 180-4.
//
// hash_blocks_kernel: one warp per prompt walks its blocks in order (each digest feeds the
// next block's message); its lanes format 32 tokens at a time into a shared-memory ring and
// compress each full 64-byte chunk together; digests land at digests[(block_offsets[p] + i) * 32].
//
// The index is an open-addressing table of slots {state, value, digest[8 words]} (48 bytes):
// state 0 empty, 1 live, 3 removed. Keys are SHA-256 digests, so their first word is already
// uniform and picks the home slot; probing is linear. Insertions claim the first empty or
// removed slot with atomicCAS (the host inserts only keys that are absent, each once per
// batch); removals mark the live slot of a key removed; a lookup stops at an empty slot.
// prefix_lookup_kernel: one thread per prompt probes its full blocks in order and stops at the
// first miss, so matched[p] blocks match, as longest_prefix's loop does.
#pragma once

#include "hb_common.cuh"

namespace hb {

constexpr int kIndexSlotWords = 12;  // state, value, 8 digest words, 2 spare (48-byte slots)
constexpr uint32_t kSlotEmpty = 0, kSlotLive = 1, kSlotRemoved = 3;

// First 32 bits of the fractional parts of the cube roots of the first 64 primes (FIPS 180-4).
__constant__ uint32_t kSha256K[64] = {
    0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
    0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
    0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
    0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
    0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
    0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
    0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
    0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};

__device__ __forceinline__ uint32_t rotr32(uint32_t x, int n) { return __funnelshift_r(x, x, n); }

// One SHA-256 compression of the 16 big-endian message words w into h.
__device__ __forceinline__ void sha256_compress(uint32_t (&h)[8], uint32_t (&w)[16]) {
  uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
#pragma unroll
  for (int i = 0; i < 64; ++i) {
    if (i >= 16) {
      const uint32_t w15 = w[(i - 15) & 15], w2 = w[(i - 2) & 15];
      const uint32_t s0 = rotr32(w15, 7) ^ rotr32(w15, 18) ^ (w15 >> 3);
      const uint32_t s1 = rotr32(w2, 17) ^ rotr32(w2, 19) ^ (w2 >> 10);
      w[i & 15] += s0 + w[(i - 7) & 15] + s1;
    }
    const uint32_t S1 = rotr32(e, 6) ^ rotr32(e, 11) ^ rotr32(e, 25);
    const uint32_t ch = (e & f) ^ (~e & g);
    const uint32_t t1 = hh + S1 + ch + kSha256K[i] + w[i & 15];
    const uint32_t S0 = rotr32(a, 2) ^ rotr32(a, 13) ^ rotr32(a, 22);
    const uint32_t maj = (a & b) ^ (a & c) ^ (b & c);
    hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + S0 + maj;
  }
  h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
}

__device__ __forceinline__ int decimal_digits(uint32_t v) {
  int n = 1;
  for (uint32_t p = 10u; n < 10 && v >= p; p *= 10u) ++n;
  return n;
}

constexpr int kHashWarps = 4;     // prompts per CTA (one warp each)
constexpr int kHashRing = 512;    // message bytes staged per warp (a 64-byte chunk is consumed at a time)

// Compress every full 64-byte chunk staged in the ring (all lanes, identical data).
__device__ __forceinline__ void drain_ring(uint32_t (&h)[8], const uint8_t* ring, int64_t head, int64_t& tail) {
  __syncwarp();
  while (head - tail >= 64) {
    const uint32_t* c = reinterpret_cast<const uint32_t*>(ring + (tail & (kHashRing - 1)));
    uint32_t w[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) w[j] = __byte_perm(c[j], 0, 0x0123);  // big-endian words
    sha256_compress(h, w);
    tail += 64;
  }
  __syncwarp();
}

// One warp per prompt. Per block the warp's lanes format 32 tokens at a time (decimal digits,
// a comma before every token but the block's first) into a shared-memory ring at offsets from
// a warp scan of their lengths; every full 64-byte chunk is then compressed by all lanes at
// once on identical data, so the state stays warp-uniform. The parent digest leads each
// block's message after the first; padding is the FIPS 180-4 0x80, zeros, 64-bit bit length.
__global__ void __launch_bounds__(kHashWarps * 32) hash_blocks_kernel(const int32_t* tokens, const int64_t* offsets,
                                                                     int32_t prompts, int32_t block_size,
                                                                     const int64_t* block_offsets, uint8_t* digests) {
  __shared__ __align__(16) uint8_t ring_all[kHashWarps][kHashRing];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pr = blockIdx.x * kHashWarps + warp;
  if (pr >= prompts) return;
  uint8_t* ring = ring_all[warp];
  const int64_t t0 = offsets[pr], t1 = offsets[pr + 1];
  const int64_t nblocks = (t1 - t0 + block_size - 1) / block_size;
  uint32_t h[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int64_t head = 0, tail = 0;  // ring positions (bytes written, bytes compressed)
  for (int64_t b = 0; b < nblocks; ++b) {
    uint32_t parent[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) parent[j] = h[j];
    h[0] = 0x6a09e667u; h[1] = 0xbb67ae85u; h[2] = 0x3c6ef372u; h[3] = 0xa54ff53au;
    h[4] = 0x510e527fu; h[5] = 0x9b05688cu; h[6] = 0x1f83d9abu; h[7] = 0x5be0cd19u;
    head = tail = 0;
    if (b > 0) {  // the parent digest, big-endian
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (lane == j) *reinterpret_cast<uint32_t*>(ring + 4 * j) = __byte_perm(parent[j], 0, 0x0123);
    }
    if (lane == 0) ring[b > 0 ? 32 : 0] = '[';
    head = b > 0 ? 33 : 1;
    const int64_t lo = t0 + b * block_size, hi = min(t1, lo + block_size);
    for (int64_t base = lo; base < hi; base += 32) {
      const int64_t t = base + lane;
      uint32_t v = 0;
      int len = 0, nd = 0;
      if (t < hi) {
        const int32_t tok = tokens[t];
        if (tok < 0) raise_status(kStatusBadToken);  // the host rejects these before the launch
        v = static_cast<uint32_t>(max(tok, 0));
        nd = decimal_digits(v);
        len = nd + (t > lo ? 1 : 0);
      }
      int incl = len;  // warp inclusive scan of the byte lengths
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      if (len > 0) {
        int64_t at = head + incl - len;
        if (t > lo) ring[(at++) & (kHashRing - 1)] = ',';
        for (int k = nd - 1; k >= 0; --k) {
          ring[(at + k) & (kHashRing - 1)] = static_cast<uint8_t>('0' + v % 10u);
          v /= 10u;
        }
      }
      head += __shfl_sync(0xffffffffu, incl, 31);
      drain_ring(h, ring, head, tail);
    }
    if (lane == 0) ring[head & (kHashRing - 1)] = ']';
    ++head;
    // Padding: 0x80, zeros up to 56 mod 64, then the message length in bits (big-endian).
    const uint64_t bits = static_cast<uint64_t>(head) * 8;
    const int zeros = static_cast<int>((119 - (head % 64)) % 64);  // head + 1 + zeros == 56 (mod 64)
    const int pad = 1 + zeros + 8;
    for (int k = lane; k < pad; k += 32) {
      uint8_t byte = 0;
      if (k == 0) byte = 0x80;
      else if (k > zeros) byte = static_cast<uint8_t>(bits >> (8 * (pad - 1 - k)));
      ring[(head + k) & (kHashRing - 1)] = byte;
    }
    head += pad;
    drain_ring(h, ring, head, tail);
    uint8_t* out = digests + (block_offsets[pr] + b) * 32;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (lane == j) *reinterpret_cast<uint32_t*>(out + 4 * j) = __byte_perm(h[j], 0, 0x0123);
  }
}

__device__ __forceinline__ void load_digest(const uint8_t* d, uint32_t (&k)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
    k[j] = (static_cast<uint32_t>(d[4 * j]) << 24) | (static_cast<uint32_t>(d[4 * j + 1]) << 16) |
           (static_cast<uint32_t>(d[4 * j + 2]) << 8) | static_cast<uint32_t>(d[4 * j + 3]);
}

__device__ __forceinline__ bool slot_holds(const uint32_t* slot, const uint32_t (&k)[8]) {
  bool eq = true;
#pragma unroll
  for (int j = 0; j < 8; ++j) eq &= slot[2 + j] == k[j];
  return eq;
}

// Slot of a live key, or -1. Every probe loop is bounded by the table size.
__device__ __forceinline__ int index_find(const uint32_t* table, int32_t slots, const uint32_t (&k)[8]) {
  const uint32_t mask = static_cast<uint32_t>(slots) - 1u;
  for (int i = 0; i < slots; ++i) {
    const int s = static_cast<int>((k[0] + static_cast<uint32_t>(i)) & mask);
    const uint32_t* slot = table + static_cast<int64_t>(s) * kIndexSlotWords;
    const uint32_t st = slot[0];
    if (st == kSlotEmpty) return -1;
    if (st == kSlotLive && slot_holds(slot, k)) return s;
  }
  return -1;
}

__global__ void prefix_index_insert_kernel(uint32_t* table, int32_t slots, const uint8_t* digests,
                                           const int32_t* values, int32_t n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  uint32_t k[8];
  load_digest(digests + static_cast<int64_t>(i) * 32, k);
  const uint32_t mask = static_cast<uint32_t>(slots) - 1u;
  for (int probe = 0; probe < slots; ++probe) {
    const int s = static_cast<int>((k[0] + static_cast<uint32_t>(probe)) & mask);
    uint32_t* slot = table + static_cast<int64_t>(s) * kIndexSlotWords;
    const uint32_t st = slot[0];
    if (st != kSlotEmpty && st != kSlotRemoved) continue;  // live, or taken by this batch
    // Claim an empty or removed slot (2: being written) so no other insert of this batch takes it.
    if (atomicCAS(slot, st, 2u) != st) continue;
    slot[1] = static_cast<uint32_t>(values[i]);
#pragma unroll
    for (int j = 0; j < 8; ++j) slot[2 + j] = k[j];
    __threadfence();
    atomicExch(slot, kSlotLive);
    return;
  }
  raise_status(kStatusIndexFull);  // no free slot: the host keeps the load factor at most 1/2
}

__global__ void prefix_index_remove_kernel(uint32_t* table, int32_t slots, const uint8_t* digests, int32_t n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  uint32_t k[8];
  load_digest(digests + static_cast<int64_t>(i) * 32, k);
  const int s = index_find(table, slots, k);
  if (s >= 0) table[static_cast<int64_t>(s) * kIndexSlotWords] = kSlotRemoved;
}

// One thread per prompt: values of its leading full blocks that are in the index, up to the
// first block that is not.
__global__ void __launch_bounds__(128) prefix_lookup_kernel(const uint32_t* table, int32_t slots,
                                                            const uint8_t* digests, const int64_t* block_offsets,
                                                            const int32_t* full_blocks, int32_t prompts,
                                                            int32_t* matched, int32_t* values) {
  const int pr = blockIdx.x * blockDim.x + threadIdx.x;
  if (pr >= prompts) return;
  const int64_t base = block_offsets[pr];
  int count = 0;
  for (int b = 0; b < full_blocks[pr]; ++b) {
    uint32_t k[8];
    load_digest(digests + (base + b) * 32, k);
    const int s = index_find(table, slots, k);
    if (s < 0) break;
    values[base + b] = static_cast<int32_t>(table[static_cast<int64_t>(s) * kIndexSlotWords + 1]);
    ++count;
  }
  matched[pr] = count;
}

}  // namespace hb
