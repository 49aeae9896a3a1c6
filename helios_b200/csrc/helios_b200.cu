// C-ABI of libhelios_b200.so: the packed-tick hot path for sm_100a.
//
// Every entry point takes raw device pointers, sizes and a cudaStream_t, borrows
// the memory for the duration of the launch and allocates nothing. Each returns
// 0 on success or a negative code (HB_ERR_*) with a message in hb_last_error().
// Declarations and the reference interface each one replaces: include/helios_b200.h.
#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <utility>

#include "../../include/helios_b200.h"
#include "attention_decode.cuh"
#include "attention_prefill.cuh"
#include "gemm_swiglu.cuh"
#include "hb_common.cuh"
#include "lm_head_argmax.cuh"
#include "model_ops.cuh"
#include "norm_rope_append.cuh"
#include "prefix_index.cuh"
#include "sampler.cuh"
#include "tick_pack.cuh"

namespace {

thread_local char g_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(HB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return HB_OK;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// ---- cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 3-D bf16 tensor map: dims (inner, mid, outer) with byte strides for mid and outer,
// 128-byte swizzle, box (box0, box1, box2). Out-of-range boxes are zero-filled.
int encode_3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1, uint64_t s2,
              uint32_t b0, uint32_t b1, uint32_t b2) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(HB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {s1, s2};
  const cuuint32_t box[3] = {b0, b1, b2};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(HB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return HB_OK;
}

// 2-D bf16 tensor map over a row-major [rows][cols] matrix (cols contiguous, row stride
// in bytes), 128-byte swizzle, box (box0 columns, box1 rows); rows past the end read as zeros.
int encode_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t row_bytes, uint32_t b0,
              uint32_t b1) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(HB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {b0, b1};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(HB_ERR_CUDA, "cuTensorMapEncodeTiled (2-D) failed (%d)", static_cast<int>(r));
  return HB_OK;
}

int sm_count() {
  static int count[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (count[dev] == 0) cudaDeviceGetAttribute(&count[dev], cudaDevAttrMultiProcessorCount, dev);
  return count[dev];
}

// Per-device one-time opt-in to large dynamic shared memory.
template <typename K>
int ensure_smem(K kernel, int bytes, bool (&done)[64]) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fail(HB_ERR_CUDA, "cudaGetDevice failed");
  if (!done[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return fail(HB_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    // Take the whole unified L1/shared array as shared memory, so two ~100 KB CTAs fit per SM.
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return fail(HB_ERR_CUDA, "cudaFuncSetAttribute(carveout): %s", cudaGetErrorString(e));
    done[dev] = true;
  }
  return HB_OK;
}

bool g_dec_smem[4][64], g_decp_smem[4][64], g_pre_smem[4][64], g_prx_smem[4][64], g_tick_smem[64], g_gemm_smem[64], g_argmax_smem[64];

constexpr int kDefaultOverlapDecodeSms = 100;

// SMs the decode grid keeps when a call also has prefill work (its other CTAs exit at once and
// leave their SMs to the prefill grid, which runs beside it); 0: the decode grid keeps all.
std::atomic<int> g_overlap_decode_sms{kDefaultOverlapDecodeSms};



// Split-K workspace of hb_paged_attention_static_workspace: one fixed array per GPU,
// for callers that cannot allocate device memory. In host code the name stands for a
// host-side shadow, so its device address is looked up once per device.
constexpr size_t kStaticWorkspaceFloats = HB_STATIC_WORKSPACE_BYTES / sizeof(float);
static __device__ __align__(256) float g_static_workspace[kStaticWorkspaceFloats];
std::mutex g_static_ws_mutex;
void* g_static_ws_ptr[64];

int group_slot(int group) { return group == 1 ? 0 : group == 2 ? 1 : group == 4 ? 2 : 3; }

// Launch with programmatic stream serialization: the kernel may start before the kernel
// ahead of it in the stream has finished, once that one's CTAs have all triggered (the
// kernels of this library wait with griddepcontrol.wait before reading what the kernel
// ahead of them wrote).
template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Persistent fused GEMM launch: one CTA per SM at most, programmatic serialization.
template <typename Epi>
int launch_fused_gemm(const typename Epi::Params& p, const CUtensorMap& amap, const CUtensorMap& bmap,
                      bool (&smem_done)[64], cudaStream_t stream, const char* what) {
  const int tiles = p.tiles_m * p.tiles_n;
  const int sms = sm_count();
  if (sms <= 0) return fail(HB_ERR_CUDA, "cannot read the SM count");
  constexpr uint32_t smem = hb::kGemmSmemBytes;
  if (int rc = ensure_smem(hb::fused_gemm_kernel<Epi>, smem, smem_done)) return rc;
  const cudaError_t e = launch_pdl(hb::fused_gemm_kernel<Epi>, dim3(static_cast<unsigned>(std::min(tiles, sms))),
                                   dim3(hb::fused_gemm_threads<Epi>()), smem, stream, p, amap, bmap);
  if (e != cudaSuccess) return fail(HB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return check_launch(what);
}

// RMSNorm launch: a CTA per row for few rows or hidden beyond 4096, else a warp per row.
int launch_rmsnorm(const hb::RowNormParams& p, cudaStream_t stream, const char* what) {
  const int nvec = p.hidden / 8;
  // Few rows (a decode tick's): a CTA per row, so each row's loads, sum and stores are spread
  // over 256 threads instead of one warp's long dependent chain (the launch is latency-bound).
  const int sms = sm_count();
  if (sms > 0 && p.rows <= 2 * sms) {
    hb::rmsnorm_kernel<<<p.rows, hb::kRowThreads, 0, stream>>>(p);
    return check_launch(what);
  }
  const unsigned warp_blocks = static_cast<unsigned>((p.rows + hb::kNormWarps - 1) / hb::kNormWarps);
  if (nvec <= 32 * 4)
    hb::rmsnorm_warp_kernel<4><<<warp_blocks, hb::kNormWarps * 32, 0, stream>>>(p);
  else if (nvec <= 32 * 8)
    hb::rmsnorm_warp_kernel<8><<<warp_blocks, hb::kNormWarps * 32, 0, stream>>>(p);
  else if (nvec <= 32 * 10)  // hidden 2560 (Qwen3-4B)
    hb::rmsnorm_warp_kernel<10><<<warp_blocks, hb::kNormWarps * 32, 0, stream>>>(p);
  else if (nvec <= 32 * 16)
    hb::rmsnorm_warp_kernel<16><<<warp_blocks, hb::kNormWarps * 32, 0, stream>>>(p);
  else
    hb::rmsnorm_kernel<<<p.rows, hb::kRowThreads, 0, stream>>>(p);
  return check_launch(what);
}

// One thread waits for phase 0 of a fresh mbarrier that no thread arrives at: the bounded
// wait must run out after limit_cycles, raise the wait-timeout status bit and return.
__global__ void wait_timeout_selftest_kernel(long long limit_cycles, int32_t* result) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    hb::mbar_init(&bar, 1);
    abort_flag = 0;
    hb::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool ok = hb::mbar_wait(&bar, 0, &abort_flag, limit_cycles);
    result[0] = ok ? 1 : 0;
    result[1] = abort_flag;
  }
}

}  // namespace

extern "C" {

int hb_version(void) { return HB_VERSION; }

const char* hb_last_error(void) { return g_error; }

int hb_device_status(uint32_t* status, int clear) {
  if (status == nullptr) return fail(HB_ERR_INVALID, "status is null");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail(HB_ERR_CUDA, "synchronize: %s", cudaGetErrorString(e));
  e = cudaMemcpyFromSymbol(status, hb::g_status, sizeof(uint32_t));
  if (e != cudaSuccess) return fail(HB_ERR_CUDA, "read status: %s", cudaGetErrorString(e));
  if (clear) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(hb::g_status, &zero, sizeof(uint32_t));
    if (e != cudaSuccess) return fail(HB_ERR_CUDA, "clear status: %s", cudaGetErrorString(e));
  }
  return HB_OK;
}

int hb_selftest_wait_timeout(int64_t limit_cycles, int32_t* result, cudaStream_t stream) {
  if (limit_cycles < 1 || limit_cycles > (int64_t(1) << 31))
    return fail(HB_ERR_INVALID, "limit_cycles %lld outside [1, 2^31]", static_cast<long long>(limit_cycles));
  if (result == nullptr || !aligned(result, 4)) return fail(HB_ERR_INVALID, "result must be a device int32[2]");
  wait_timeout_selftest_kernel<<<1, 32, 0, stream>>>(limit_cycles, result);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(HB_ERR_CUDA, "wait_timeout_selftest_kernel: %s", cudaGetErrorString(e));
  return HB_OK;
}

int hb_tick_pack(const int32_t* rows, int32_t num_rows, const int32_t* updates, int32_t num_updates, int32_t* arena,
                 int32_t arena_slots, int32_t arena_width, int32_t page_size, int32_t width, int32_t num_pages,
                 int32_t decode_max_tokens, int32_t split_keys, int32_t prefill_tile_tokens,
                 int32_t prefix_split_keys, int32_t total_tokens, int32_t* block_table, int32_t* cu_seq_q,
                 int32_t* cu_seq_k, int32_t* seqused_k, int64_t* positions, int64_t* write_slots, int32_t* token_row,
                 int64_t* logit_indices, int32_t logit_capacity, int32_t* decode_items, int32_t decode_capacity,
                 int32_t* prefill_items, int32_t prefill_capacity, int32_t* prefix_items, int32_t prefix_capacity,
                 int32_t* counts, int32_t* row_records, cudaStream_t stream) {
  if (num_rows < 1 || num_rows > HB_MAX_TICK_ROWS)
    return fail(HB_ERR_INVALID, "num_rows %d outside [1, %d]", num_rows, HB_MAX_TICK_ROWS);
  if (rows == nullptr || arena == nullptr || block_table == nullptr || cu_seq_q == nullptr || cu_seq_k == nullptr ||
      seqused_k == nullptr)
    return fail(HB_ERR_INVALID, "null metadata pointer");
  if (num_updates < 0 || (num_updates > 0 && updates == nullptr)) return fail(HB_ERR_INVALID, "bad page updates");
  if (page_size < 1 || width < 1 || arena_width < 1 || arena_slots < 1 || num_pages < 1 || split_keys < page_size ||
      split_keys % page_size != 0 || prefill_tile_tokens < 1 || total_tokens < 0 || prefix_split_keys < page_size ||
      prefix_split_keys % page_size != 0)
    return fail(HB_ERR_INVALID, "bad tick sizes");
  if (total_tokens > 0 && (positions == nullptr || write_slots == nullptr || token_row == nullptr))
    return fail(HB_ERR_INVALID, "null per-token output");
  if ((logit_capacity > 0 && logit_indices == nullptr) || (decode_capacity > 0 && decode_items == nullptr) ||
      (prefill_capacity > 0 && prefill_items == nullptr) || (prefix_capacity > 0 && prefix_items == nullptr) ||
      logit_capacity < 0 || decode_capacity < 0 || prefill_capacity < 0 || prefix_capacity < 0)
    return fail(HB_ERR_INVALID, "bad output capacities");
  hb::TickPackParams p{rows, updates, arena, num_rows, num_updates, arena_width, arena_slots, page_size, width,
                       num_pages, decode_max_tokens, split_keys, prefill_tile_tokens, prefix_split_keys, block_table,
                       cu_seq_q, cu_seq_k, seqused_k, positions, write_slots, token_row, logit_indices, decode_items,
                       prefill_items, total_tokens, logit_capacity, decode_capacity, prefill_capacity, counts,
                       row_records, prefix_items, prefix_capacity};
  const int smem = 7 * (num_rows + 1) * static_cast<int>(sizeof(int32_t));
  if (int rc = ensure_smem(hb::tick_pack_kernel, 7 * (HB_MAX_TICK_ROWS + 1) * 4, g_tick_smem)) return rc;
  hb::tick_pack_kernel<<<1, hb::kTickThreads, smem, stream>>>(p);
  return check_launch("tick_pack_kernel");
}

int hb_qk_norm_rope_append(const void* q, int64_t q_token_stride, int64_t q_head_stride, const void* k,
                           int64_t k_token_stride, int64_t k_head_stride, const void* v, int64_t v_token_stride,
                           int64_t v_head_stride, const float* q_scale, const float* k_scale, float eps,
                           const float* cos, const float* sin, int64_t rope_rows, const int64_t* positions,
                           const int64_t* write_slots, void* q_out, void* key_pool, void* value_pool,
                           int64_t pool_slots, int32_t tokens, int32_t heads, int32_t kv_heads, int32_t head_dim,
                           cudaStream_t stream) {
  if (tokens < 0 || heads < 1 || kv_heads < 1 || heads % kv_heads) return fail(HB_ERR_INVALID, "bad head counts");
  if (head_dim != 64 && head_dim != 128) return fail(HB_ERR_UNSUPPORTED, "head_dim %d (supported: 64, 128)", head_dim);
  if (tokens == 0) return HB_OK;
  if (k == nullptr || v == nullptr || key_pool == nullptr || value_pool == nullptr || write_slots == nullptr)
    return fail(HB_ERR_INVALID, "null key/value pointer");
  if (q_out != nullptr && q == nullptr) return fail(HB_ERR_INVALID, "q_out without q");
  if ((cos == nullptr) != (sin == nullptr) || (cos != nullptr && positions == nullptr))
    return fail(HB_ERR_INVALID, "rope tables need cos, sin and positions");
  // Every row is moved as 16-byte vectors: bases 16-byte aligned, strides multiples of 8 elements.
  const bool strides_ok = k_token_stride % 8 == 0 && k_head_stride % 8 == 0 && v_token_stride % 8 == 0 &&
                          v_head_stride % 8 == 0 && (q == nullptr || (q_token_stride % 8 == 0 && q_head_stride % 8 == 0));
  if (!strides_ok || !aligned(k, 16) || !aligned(v, 16) || (q && !aligned(q, 16)) || (q_out && !aligned(q_out, 16)) ||
      !aligned(key_pool, 16) || !aligned(value_pool, 16))
    return fail(HB_ERR_INVALID, "q/k/v rows and pools must be 16-byte aligned (strides multiples of 8 elements)");
  if ((q_scale && !aligned(q_scale, 16)) || (k_scale && !aligned(k_scale, 16)) || (cos && !aligned(cos, 16)) ||
      (sin && !aligned(sin, 16)))
    return fail(HB_ERR_INVALID, "norm scales and rope tables must be 16-byte aligned");
  hb::NormRopeParams p{static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
                       static_cast<const __nv_bfloat16*>(v), q_token_stride, q_head_stride, k_token_stride,
                       k_head_stride, v_token_stride, v_head_stride, q_scale, k_scale, eps, cos, sin, rope_rows,
                       positions, write_slots, static_cast<__nv_bfloat16*>(q_out),
                       static_cast<__nv_bfloat16*>(key_pool), static_cast<__nv_bfloat16*>(value_pool), pool_slots,
                       tokens, heads, kv_heads};
  const dim3 blocks(static_cast<unsigned>(tokens));  // one CTA per token
  const cudaError_t e = head_dim == 128
                            ? launch_pdl(hb::norm_rope_append_kernel<128>, blocks, dim3(hb::kRopeThreads), 0, stream, p)
                            : launch_pdl(hb::norm_rope_append_kernel<64>, blocks, dim3(hb::kRopeThreads), 0, stream, p);
  if (e != cudaSuccess) return fail(HB_ERR_CUDA, "norm_rope_append_kernel: %s", cudaGetErrorString(e));
  return check_launch("norm_rope_append_kernel");
}

// Workspace: kWorkspaceHeader bytes of decode work counters, then the split-K partials
// ([records][heads][head_dim] outputs, then [records][heads] log2-sum-exps).
constexpr size_t kWorkspaceHeader = 256;

size_t hb_attention_workspace_bytes(int32_t partial_records, int32_t heads, int32_t head_dim) {
  if (heads <= 0 || head_dim <= 0) return 0;
  const size_t records = partial_records > 0 ? static_cast<size_t>(partial_records) : 0;
  return kWorkspaceHeader + records * heads * (head_dim + 1) * sizeof(float);
}

int hb_paged_attention(const void* q, const void* key_pool, const void* value_pool, int64_t num_pages,
                       int32_t page_size, const int32_t* block_table, int32_t width, const int32_t* cu_seq_q,
                       const int32_t* seqused_k, int32_t num_rows, const int32_t* row_records,
                       const int32_t* decode_items, int32_t num_decode_items,
                       const int32_t* prefill_items, int32_t num_prefill_items, const int32_t* prefix_items,
                       int32_t num_prefix_items, const int32_t* counts, int32_t partial_records,
                       int32_t split_keys, int32_t total_tokens, int32_t heads, int32_t kv_heads, int32_t head_dim,
                       float scale, void* workspace, size_t workspace_bytes, void* out, cudaStream_t stream) {
  if (head_dim != 128) return fail(HB_ERR_UNSUPPORTED, "paged attention supports head_dim 128, got %d", head_dim);
  if (heads < 1 || kv_heads < 1 || heads % kv_heads) return fail(HB_ERR_INVALID, "bad head counts");
  const int group = heads / kv_heads;
  if (group != 1 && group != 2 && group != 4 && group != 8)
    return fail(HB_ERR_UNSUPPORTED, "query heads per KV head must be 1, 2, 4 or 8 (got %d)", group);
  if (page_size % hb::kDecTileKeys != 0 || split_keys % page_size != 0 || split_keys < page_size)
    return fail(HB_ERR_INVALID, "page_size must be a multiple of 64 and split_keys of page_size");
  if (num_decode_items < 0 || num_prefill_items < 0 || num_prefix_items < 0 || total_tokens < 0 || num_pages < 1 ||
      width < 1 || partial_records < 0 || num_rows < 1 || num_rows > HB_MAX_TICK_ROWS)
    return fail(HB_ERR_INVALID, "bad work sizes");
  if ((num_decode_items > 0 || num_prefix_items > 0) && row_records == nullptr)
    return fail(HB_ERR_INVALID, "null row records");
  // Prefix items add their splits to rows that also have decode items: the combine behind the
  // decode grid merges them.
  if (num_prefix_items > 0 && num_decode_items == 0)
    return fail(HB_ERR_INVALID, "prefix items without decode items");
  if (num_pages * page_size > (int64_t(1) << 31)) return fail(HB_ERR_UNSUPPORTED, "pool exceeds 2^31 tokens");
  if (q == nullptr || key_pool == nullptr || value_pool == nullptr || out == nullptr || block_table == nullptr ||
      cu_seq_q == nullptr || seqused_k == nullptr)
    return fail(HB_ERR_INVALID, "null attention pointer");
  if (!aligned(key_pool, 16) || !aligned(value_pool, 16) || !aligned(q, 16) || !aligned(out, 16))
    return fail(HB_ERR_INVALID, "q, out and pools must be 16-byte aligned");
  const size_t need = hb_attention_workspace_bytes(partial_records, heads, head_dim);
  if (workspace_bytes < need || workspace == nullptr || !aligned(workspace, 16))
    return fail(HB_ERR_INVALID, "workspace holds %zu bytes, needs %zu (16-byte aligned)", workspace_bytes, need);
  if (total_tokens == 0) return HB_OK;

  hb::AttentionParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.block_table = block_table;
  p.cu_seq_q = cu_seq_q;
  p.seqused_k = seqused_k;
  p.decode_items = decode_items;
  p.row_records = row_records;
  p.num_rows = num_rows;
  p.record_capacity = partial_records;
  p.prefill_items = prefill_items;
  p.prefix_items = prefix_items;
  p.work_counter = static_cast<int32_t*>(workspace);
  p.ws_out = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kWorkspaceHeader);
  p.ws_lse = p.ws_out + static_cast<size_t>(partial_records > 0 ? partial_records : 0) * heads * head_dim;
  p.width = width;
  p.num_pages = static_cast<int32_t>(num_pages);
  p.page_size = page_size;
  p.heads = heads;
  p.kv_heads = kv_heads;
  p.split_keys = split_keys;
  p.tokens = total_tokens;
  p.num_prefill = num_prefill_items;
  p.num_prefix = num_prefix_items;
  p.counts = counts;
  p.scale_log2 = scale * 1.4426950408889634f;

  const uint64_t pool_tokens = static_cast<uint64_t>(num_pages) * page_size;
  const uint64_t row_bytes = static_cast<uint64_t>(kv_heads) * head_dim * 2;
  CUtensorMap kmap, vmap;
  if (int rc = encode_3d(&kmap, key_pool, head_dim, kv_heads, pool_tokens, head_dim * 2, row_bytes, 64, 1,
                         hb::kDecTileKeys))
    return rc;
  if (int rc = encode_3d(&vmap, value_pool, head_dim, kv_heads, pool_tokens, head_dim * 2, row_bytes, 64, 1,
                         hb::kDecTileKeys))
    return rc;
  const int gs = group_slot(group);
  if (num_decode_items > 0 && decode_items == nullptr) return fail(HB_ERR_INVALID, "null decode items");
  if (static_cast<int64_t>(num_decode_items) * kv_heads > INT32_MAX)
    return fail(HB_ERR_UNSUPPORTED, "decode items x KV heads exceed 2^31");
  if (num_prefill_items > 0 && prefill_items == nullptr) return fail(HB_ERR_INVALID, "null prefill items");
  if (num_prefix_items > 0 && prefix_items == nullptr) return fail(HB_ERR_INVALID, "null prefix items");

  // Launch order on the caller's stream, each grid behind the previous one with programmatic
  // dependent launch; completions are ordered through grid-dependency waits (each grid that
  // skips its initial wait has one CTA wait for the grid ahead before it exits, see
  // prefill_after_decode / decode_after_prefix, and the combine waits last).
  //   Without prefill items: prefix -> decode -> combine. The decode grid runs one CTA per
  //   unit, two per SM; its CTAs fill the SMs the prefix tiles leave and take the rest as
  //   they finish.
  //   With prefill items: decode -> prefix -> prefill -> combine, the decode grid persistent:
  //   its CTAs past decode_ctas exit at once so that the tensor-core tiles start on those SMs
  //   while the decode CTAs stream K/V (decode is HBM-bound, the tiles tensor-bound).
  if (num_prefill_items > 65535 || num_prefix_items > 65535)
    return fail(HB_ERR_UNSUPPORTED, "more than 65535 prefill tile pairs or prefix items in one call");
  const int overlap_sms = g_overlap_decode_sms.load();
  const bool beside = num_decode_items > 0 && num_prefill_items > 0 && overlap_sms > 0;
  const bool prefix_first = num_prefix_items > 0 && !beside;
  int decode_grid = 0;
  if (beside) {
    const int sms = sm_count();
    if (sms <= 0) return fail(HB_ERR_CUDA, "cannot read the SM count");
    decode_grid = std::min(sms, (num_decode_items * kv_heads + hb::kDecSubs - 1) / hb::kDecSubs);
  }
  p.num_decode = num_decode_items;
  p.decode_ctas = std::max(1, std::min(overlap_sms, decode_grid));
  p.prefill_after_decode = num_decode_items > 0 ? 1 : 0;

  // Everything that can fail before a launch (the prefill tensor map, the shared-memory
  // opt-ins) is done first, so an early return never leaves the decode grid queued without
  // the combine that resets its work ticket.
  CUtensorMap qmap;
  if (num_prefill_items > 0 || num_prefix_items > 0) {
#define HB_PREFILL_PREP(G)                                                                                      \
  do {                                                                                                          \
    if (int rc = encode_3d(&qmap, q, head_dim, heads, total_tokens, head_dim * 2,                               \
                           static_cast<uint64_t>(heads) * head_dim * 2, 64, G, hb::kPreRows / G))               \
      return rc;                                                                                                \
    if (num_prefill_items > 0)                                                                                  \
      if (int rc = ensure_smem(hb::prefill_attention_kernel<G, false>, hb::kPreSmemBytes, g_pre_smem[gs]))      \
        return rc;                                                                                              \
    if (num_prefix_items > 0)                                                                                   \
      if (int rc = ensure_smem(hb::prefill_attention_kernel<G, true>, hb::kPreSmemBytes, g_prx_smem[gs]))       \
        return rc;                                                                                              \
  } while (0)
    switch (group) {
      case 1: HB_PREFILL_PREP(1); break;
      case 2: HB_PREFILL_PREP(2); break;
      case 4: HB_PREFILL_PREP(4); break;
      default: HB_PREFILL_PREP(8); break;
    }
#undef HB_PREFILL_PREP
  }
  if (num_decode_items > 0) {
#define HB_DECODE_PREP(G)                                                                                       \
  do {                                                                                                          \
    if (beside) {                                                                                               \
      if (int rc = ensure_smem(hb::decode_persistent_kernel<G>, hb::kDecPersistentSmemBytes, g_decp_smem[gs]))  \
        return rc;                                                                                              \
    } else if (int rc = ensure_smem(hb::decode_attention_kernel<G>, hb::kDecSmemBytes, g_dec_smem[gs])) {       \
      return rc;                                                                                                \
    }                                                                                                           \
  } while (0)
    switch (group) {
      case 1: HB_DECODE_PREP(1); break;
      case 2: HB_DECODE_PREP(2); break;
      case 4: HB_DECODE_PREP(4); break;
      default: HB_DECODE_PREP(8); break;
    }
#undef HB_DECODE_PREP
  }

  // Once the persistent decode grid is queued, its work ticket is nonzero until the combine
  // grid resets it. If a later launch fails, a 4-byte memset queued behind the decode grid
  // resets it instead (it allocates nothing), so the next call on this workspace starts at 0.
  bool ticket_queued = false;
  auto fail_after_decode = [&](int rc) {
    if (ticket_queued) cudaMemsetAsync(workspace, 0, sizeof(int32_t), stream);
    return rc;
  };
  auto launch_prefix = [&]() -> int {
#define HB_PREFIX(G)                                                                                            \
  do {                                                                                                          \
    const cudaError_t e = launch_pdl(hb::prefill_attention_kernel<G, true>, dim3(kv_heads, num_prefix_items),   \
                                     dim3(hb::kPreThreads), hb::kPreSmemBytes, stream, p, qmap, kmap, vmap);     \
    if (e != cudaSuccess)                                                                                       \
      return fail_after_decode(fail(HB_ERR_CUDA, "prefill_attention_kernel<prefix>: %s", cudaGetErrorString(e))); \
  } while (0)
    switch (group) {
      case 1: HB_PREFIX(1); break;
      case 2: HB_PREFIX(2); break;
      case 4: HB_PREFIX(4); break;
      default: HB_PREFIX(8); break;
    }
#undef HB_PREFIX
    return HB_OK;
  };
  if (prefix_first) {  // first behind the norm/RoPE/append kernel: every prefix CTA waits for it
    p.prefill_after_decode = 0;
    if (int rc = launch_prefix()) return rc;
    p.decode_after_prefix = 1;
  }
  p.prefill_after_decode = num_decode_items > 0 ? 1 : 0;
  if (num_decode_items > 0) {
#define HB_DECODE(G)                                                                                            \
  do {                                                                                                          \
    cudaError_t e;                                                                                              \
    if (beside) {                                                                                               \
      e = launch_pdl(hb::decode_persistent_kernel<G>, dim3(decode_grid), dim3(hb::kDecPersistentThreads),       \
                     hb::kDecPersistentSmemBytes, stream, p, kmap, vmap);                                       \
    } else {                                                                                                    \
      e = launch_pdl(hb::decode_attention_kernel<G>, dim3(num_decode_items * kv_heads), dim3(hb::kDecSubThreads), \
                     hb::kDecSmemBytes, stream, p, kmap, vmap);                                                 \
    }                                                                                                           \
    if (e != cudaSuccess) return fail(HB_ERR_CUDA, "decode attention: %s", cudaGetErrorString(e));              \
  } while (0)
    switch (group) {
      case 1: HB_DECODE(1); break;
      case 2: HB_DECODE(2); break;
      case 4: HB_DECODE(4); break;
      default: HB_DECODE(8); break;
    }
#undef HB_DECODE
    ticket_queued = beside;
  }
  if (num_prefix_items > 0 && !prefix_first) {
    if (int rc = launch_prefix()) return rc;
  }
  if (num_prefill_items > 0) {
    const dim3 grid(kv_heads, num_prefill_items);
#define HB_PREFILL(G)                                                                                           \
  do {                                                                                                          \
    const cudaError_t e = launch_pdl(hb::prefill_attention_kernel<G, false>, grid, dim3(hb::kPreThreads),       \
                                     hb::kPreSmemBytes, stream, p, qmap, kmap, vmap);                           \
    if (e != cudaSuccess)                                                                                       \
      return fail_after_decode(fail(HB_ERR_CUDA, "prefill_attention_kernel: %s", cudaGetErrorString(e)));      \
  } while (0)
    switch (group) {
      case 1: HB_PREFILL(1); break;
      case 2: HB_PREFILL(2); break;
      case 4: HB_PREFILL(4); break;
      default: HB_PREFILL(8); break;
    }
#undef HB_PREFILL
  }
  if (num_decode_items > 0 && (partial_records > 0 || beside)) {  // also resets the decode work ticket
    const dim3 grid(num_rows, kv_heads);
#define HB_COMBINE(G)                                                                                          \
  do {                                                                                                         \
    const cudaError_t e = launch_pdl(hb::decode_combine_kernel<G>, grid, dim3(128), 0, stream, p);             \
    if (e != cudaSuccess)                                                                                      \
      return fail_after_decode(fail(HB_ERR_CUDA, "decode_combine_kernel: %s", cudaGetErrorString(e)));       \
  } while (0)
    switch (group) {
      case 1: HB_COMBINE(1); break;
      case 2: HB_COMBINE(2); break;
      case 4: HB_COMBINE(4); break;
      default: HB_COMBINE(8); break;
    }
#undef HB_COMBINE
  }
  return HB_OK;
}

int hb_attention_set_overlap(int32_t decode_sms) {
  if (decode_sms < 0) return fail(HB_ERR_INVALID, "decode_sms must be >= 0");
  g_overlap_decode_sms.store(decode_sms);
  return HB_OK;
}

int hb_paged_attention_static_workspace(const void* q, const void* key_pool, const void* value_pool,
                                       int64_t num_pages, int32_t page_size, const int32_t* block_table,
                                       int32_t width, const int32_t* cu_seq_q, const int32_t* seqused_k,
                                       int32_t num_rows, const int32_t* row_records,
                                       const int32_t* decode_items, int32_t num_decode_items,
                                       const int32_t* prefill_items, int32_t num_prefill_items,
                                       const int32_t* prefix_items, int32_t num_prefix_items,
                                       const int32_t* counts, int32_t partial_records, int32_t split_keys,
                                       int32_t total_tokens, int32_t heads, int32_t kv_heads, int32_t head_dim,
                                       float scale, void* out, cudaStream_t stream) {
  const size_t need = hb_attention_workspace_bytes(partial_records, heads, head_dim);
  if (need > HB_STATIC_WORKSPACE_BYTES)
    return fail(HB_ERR_INVALID,
                "split-K partials need %zu bytes, more than the built-in %u-byte workspace; "
                "use hb_paged_attention with a caller workspace or larger split_keys",
                need, HB_STATIC_WORKSPACE_BYTES);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fail(HB_ERR_CUDA, "cudaGetDevice failed");
  void* ws = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_static_ws_mutex);
    if (g_static_ws_ptr[dev] == nullptr) {
      // Once per device, with that device current: the array's device address.
      const cudaError_t e = cudaGetSymbolAddress(&g_static_ws_ptr[dev], g_static_workspace);
      if (e != cudaSuccess) {
        g_static_ws_ptr[dev] = nullptr;
        return fail(HB_ERR_CUDA, "cudaGetSymbolAddress(static workspace): %s", cudaGetErrorString(e));
      }
    }
    ws = g_static_ws_ptr[dev];
  }
  return hb_paged_attention(q, key_pool, value_pool, num_pages, page_size, block_table, width, cu_seq_q, seqused_k,
                            num_rows, row_records, decode_items, num_decode_items, prefill_items, num_prefill_items,
                            prefix_items, num_prefix_items, counts, partial_records,
                            split_keys, total_tokens, heads, kv_heads, head_dim, scale, ws, HB_STATIC_WORKSPACE_BYTES,
                            out, stream);
}

int hb_rmsnorm(const void* x, int64_t rows_in, const int64_t* row_index, const float* scale, float eps, void* out,
               int32_t rows, int32_t hidden, cudaStream_t stream) {
  if (rows < 0 || hidden < 8 || hidden % 8 || hidden > 8 * hb::kRowVecs * hb::kRowThreads)
    return fail(HB_ERR_UNSUPPORTED, "hidden %d must be a multiple of 8 up to %d", hidden,
                8 * hb::kRowVecs * hb::kRowThreads);
  if (rows == 0) return HB_OK;
  if (x == nullptr || scale == nullptr || out == nullptr) return fail(HB_ERR_INVALID, "null rmsnorm pointer");
  if (!aligned(x, 16) || !aligned(out, 16) || !aligned(scale, 16))
    return fail(HB_ERR_INVALID, "rmsnorm pointers must be 16-byte aligned");
  hb::RowNormParams p{static_cast<const __nv_bfloat16*>(x), nullptr, row_index, scale, nullptr,
                      static_cast<__nv_bfloat16*>(out), rows, hidden, row_index ? rows_in : rows, eps};
  return launch_rmsnorm(p, stream, "rmsnorm_kernel");
}

int hb_add_rmsnorm(const void* x, const void* y, const float* scale, float eps, void* sum_out, void* norm_out,
                   int32_t rows, int32_t hidden, cudaStream_t stream) {
  if (rows < 0 || hidden < 8 || hidden % 8 || hidden > 8 * hb::kRowVecs * hb::kRowThreads)
    return fail(HB_ERR_UNSUPPORTED, "hidden %d must be a multiple of 8 up to %d", hidden,
                8 * hb::kRowVecs * hb::kRowThreads);
  if (rows == 0) return HB_OK;
  if (x == nullptr || y == nullptr || scale == nullptr || sum_out == nullptr || norm_out == nullptr)
    return fail(HB_ERR_INVALID, "null add_rmsnorm pointer");
  if (!aligned(x, 16) || !aligned(y, 16) || !aligned(sum_out, 16) || !aligned(norm_out, 16) || !aligned(scale, 16))
    return fail(HB_ERR_INVALID, "add_rmsnorm pointers must be 16-byte aligned");
  hb::RowNormParams p{static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(y), nullptr, scale,
                      static_cast<__nv_bfloat16*>(sum_out), static_cast<__nv_bfloat16*>(norm_out), rows, hidden,
                      rows, eps};
  return launch_rmsnorm(p, stream, "add_rmsnorm_kernel");
}

int hb_swiglu(const void* gate_up, void* out, int64_t rows, int64_t inter, cudaStream_t stream) {
  if (rows < 0 || inter < 8 || inter % 8)
    return fail(HB_ERR_UNSUPPORTED, "inter %lld must be a multiple of 8", static_cast<long long>(inter));
  if (rows == 0) return HB_OK;
  if (gate_up == nullptr || out == nullptr || !aligned(gate_up, 16) || !aligned(out, 16))
    return fail(HB_ERR_INVALID, "swiglu pointers must be non-null and 16-byte aligned");
  hb::SwigluParams p{static_cast<const __nv_bfloat16*>(gate_up), static_cast<__nv_bfloat16*>(out), rows, inter};
  const int64_t per_block = hb::kSwigluThreads * hb::kSwigluVecs;
  const dim3 grid(static_cast<unsigned>((inter / 8 + per_block - 1) / per_block),
                  static_cast<unsigned>(std::min<int64_t>(rows, 65535)));
  hb::swiglu_kernel<<<grid, hb::kSwigluThreads, 0, stream>>>(p);
  return check_launch("swiglu_kernel");
}

int hb_embedding(const int64_t* ids, const void* table, int64_t vocab, void* out, int64_t tokens, int32_t hidden,
                 cudaStream_t stream) {
  if (tokens < 0 || hidden < 8 || hidden % 8)
    return fail(HB_ERR_UNSUPPORTED, "hidden %d must be a multiple of 8", hidden);
  if (tokens == 0) return HB_OK;
  if (ids == nullptr || table == nullptr || out == nullptr || !aligned(table, 16) || !aligned(out, 16))
    return fail(HB_ERR_INVALID, "embedding pointers must be non-null and 16-byte aligned");
  hb::EmbedParams p{ids, static_cast<const __nv_bfloat16*>(table), static_cast<__nv_bfloat16*>(out), tokens, vocab,
                    hidden};
  hb::embed_kernel<<<static_cast<unsigned>(tokens), 256, 0, stream>>>(p);
  return check_launch("embed_kernel");
}

int hb_page_copy(void* pool_base, int64_t tensor_stride_bytes, int32_t tensors, int64_t page_bytes, int64_t num_pages,
                 const int32_t* src_pages, const int32_t* dst_pages, int32_t pairs, cudaStream_t stream) {
  if (pairs < 0 || tensors < 1 || page_bytes < 16 || page_bytes % 16 || num_pages < 1)
    return fail(HB_ERR_INVALID, "bad page copy sizes");
  if (pairs == 0) return HB_OK;
  if (pool_base == nullptr || src_pages == nullptr || dst_pages == nullptr || !aligned(pool_base, 16) ||
      tensor_stride_bytes % 16)
    return fail(HB_ERR_INVALID, "page copy pointers must be non-null and 16-byte aligned");
  hb::PageCopyParams p{static_cast<uint8_t*>(pool_base), tensor_stride_bytes, tensors, page_bytes, num_pages,
                       src_pages, dst_pages, pairs};
  const int64_t vecs = static_cast<int64_t>(pairs) * tensors * (page_bytes / 16);
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((vecs + 255) / 256, 148 * 8));
  hb::page_copy_kernel<<<blocks, 256, 0, stream>>>(p);
  return check_launch("page_copy_kernel");
}

int hb_sample(const void* logits, int64_t row_stride, int32_t rows, int32_t vocab, const float* temperature,
              const float* top_p, const float* uniforms, int64_t* out_ids, cudaStream_t stream) {
  if (rows < 0 || vocab < 1 || row_stride < vocab) return fail(HB_ERR_INVALID, "bad sampler sizes");
  if (rows == 0) return HB_OK;
  if (logits == nullptr || temperature == nullptr || top_p == nullptr || uniforms == nullptr || out_ids == nullptr)
    return fail(HB_ERR_INVALID, "null sampler pointer");
  hb::SampleParams p{static_cast<const __nv_bfloat16*>(logits), row_stride, rows, vocab, temperature, top_p, uniforms,
                     out_ids};
  hb::sample_kernel<<<rows, hb::kSampleThreads, 0, stream>>>(p);
  return check_launch("sample_kernel");
}

int hb_gemm_swiglu(const void* x, int32_t m, int32_t k, const void* w_gate_up, int32_t inter, void* out,
                   cudaStream_t stream) {
  if (m < 0 || k < 1 || inter < 1) return fail(HB_ERR_INVALID, "bad GEMM sizes");
  if (k % hb::kGemmTileK != 0 || inter % hb::kGemmTileN != 0)
    return fail(HB_ERR_UNSUPPORTED, "gate|up GEMM needs K %% %d == 0 and intermediate %% %d == 0 (got %d, %d)",
                hb::kGemmTileK, hb::kGemmTileN, k, inter);
  if (m == 0) return HB_OK;
  if (x == nullptr || w_gate_up == nullptr || out == nullptr || !aligned(x, 16) || !aligned(w_gate_up, 16) ||
      !aligned(out, 16))
    return fail(HB_ERR_INVALID, "gate|up GEMM pointers must be non-null and 16-byte aligned");
  CUtensorMap amap, bmap;
  const uint64_t row_bytes = static_cast<uint64_t>(k) * 2;
  if (int rc = encode_2d(&amap, x, k, m, row_bytes, hb::kGemmTileK, hb::kGemmTileM)) return rc;
  if (int rc = encode_2d(&bmap, w_gate_up, k, 2 * static_cast<uint64_t>(inter), row_bytes, hb::kGemmTileK,
                         hb::kGemmTileN))
    return rc;
  hb::GemmSwigluParams p{m, k, (m + hb::kGemmTileM - 1) / hb::kGemmTileM, inter / hb::kGemmTileN,
                         static_cast<__nv_bfloat16*>(out), inter};
  return launch_fused_gemm<hb::SwigluEpilogue>(p, amap, bmap, g_gemm_smem, stream, "fused_gemm_kernel<swiglu>");
}

int hb_lm_head_argmax(const void* x, int32_t m, int32_t k, const void* weight, int32_t vocab,
                      unsigned long long* best, int64_t* out_ids, cudaStream_t stream) {
  if (m < 0 || k < 1 || vocab < 1) return fail(HB_ERR_INVALID, "bad lm_head sizes");
  if (k % hb::kGemmTileK != 0)
    return fail(HB_ERR_UNSUPPORTED, "lm_head argmax needs K %% %d == 0 (got %d)", hb::kGemmTileK, k);
  if (m == 0) return HB_OK;
  if (x == nullptr || weight == nullptr || best == nullptr || out_ids == nullptr || !aligned(x, 16) ||
      !aligned(weight, 16) || !aligned(best, 8) || !aligned(out_ids, 8))
    return fail(HB_ERR_INVALID, "lm_head argmax pointers must be non-null, x and weight 16-byte aligned");
  CUtensorMap amap, bmap;
  const uint64_t row_bytes = static_cast<uint64_t>(k) * 2;
  if (int rc = encode_2d(&amap, x, k, m, row_bytes, hb::kGemmTileK, hb::kGemmTileM)) return rc;
  if (int rc = encode_2d(&bmap, weight, k, vocab, row_bytes, hb::kGemmTileK, hb::kGemmTileN)) return rc;
  hb::GemmArgmaxParams p{m, k, (m + hb::kGemmTileM - 1) / hb::kGemmTileM,
                         (vocab + 2 * hb::kGemmTileN - 1) / (2 * hb::kGemmTileN), vocab, best};
  if (int rc = launch_fused_gemm<hb::ArgmaxEpilogue>(p, amap, bmap, g_argmax_smem, stream, "fused_gemm_kernel<argmax>"))
    return rc;
  hb::argmax_finalize_kernel<<<(m + 127) / 128, 128, 0, stream>>>(best, m, out_ids);
  return check_launch("argmax_finalize_kernel");
}

int hb_hash_token_blocks(const int32_t* tokens, const int64_t* offsets, int32_t prompts, int32_t block_size,
                         const int64_t* block_offsets, uint8_t* digests, cudaStream_t stream) {
  if (prompts < 0 || block_size < 1) return fail(HB_ERR_INVALID, "bad prompt count or block size");
  if (prompts == 0) return HB_OK;
  if (tokens == nullptr || offsets == nullptr || block_offsets == nullptr || digests == nullptr)
    return fail(HB_ERR_INVALID, "null block-hash pointer");
  hb::hash_blocks_kernel<<<(prompts + hb::kHashWarps - 1) / hb::kHashWarps, hb::kHashWarps * 32, 0, stream>>>(
      tokens, offsets, prompts, block_size, block_offsets, digests);
  return check_launch("hash_blocks_kernel");
}

static bool index_slots_ok(int32_t slots) { return slots >= 1 && (slots & (slots - 1)) == 0; }

int hb_prefix_index_insert(uint32_t* table, int32_t slots, const uint8_t* digests, const int32_t* values, int32_t n,
                           cudaStream_t stream) {
  if (!index_slots_ok(slots) || n < 0) return fail(HB_ERR_INVALID, "index slots must be a power of two, n >= 0");
  if (n == 0) return HB_OK;
  if (table == nullptr || digests == nullptr || values == nullptr) return fail(HB_ERR_INVALID, "null index pointer");
  hb::prefix_index_insert_kernel<<<(n + 127) / 128, 128, 0, stream>>>(table, slots, digests, values, n);
  return check_launch("prefix_index_insert_kernel");
}

int hb_prefix_index_remove(uint32_t* table, int32_t slots, const uint8_t* digests, int32_t n, cudaStream_t stream) {
  if (!index_slots_ok(slots) || n < 0) return fail(HB_ERR_INVALID, "index slots must be a power of two, n >= 0");
  if (n == 0) return HB_OK;
  if (table == nullptr || digests == nullptr) return fail(HB_ERR_INVALID, "null index pointer");
  hb::prefix_index_remove_kernel<<<(n + 127) / 128, 128, 0, stream>>>(table, slots, digests, n);
  return check_launch("prefix_index_remove_kernel");
}

int hb_prefix_index_lookup(const uint32_t* table, int32_t slots, const uint8_t* digests, const int64_t* block_offsets,
                           const int32_t* full_blocks, int32_t prompts, int32_t* matched, int32_t* values,
                           cudaStream_t stream) {
  if (!index_slots_ok(slots) || prompts < 0)
    return fail(HB_ERR_INVALID, "index slots must be a power of two, prompts >= 0");
  if (prompts == 0) return HB_OK;
  if (table == nullptr || digests == nullptr || block_offsets == nullptr || full_blocks == nullptr ||
      matched == nullptr || values == nullptr)
    return fail(HB_ERR_INVALID, "null index pointer");
  hb::prefix_lookup_kernel<<<(prompts + 127) / 128, 128, 0, stream>>>(table, slots, digests, block_offsets,
                                                                       full_blocks, prompts, matched, values);
  return check_launch("prefix_lookup_kernel");
}


int hb_verify_drafts(const int64_t* tokens, const int32_t* cu_seq_q, const int32_t* logit_offsets,
                     const int64_t* predictions, int32_t rows, int32_t* accepted, int64_t* emitted,
                     cudaStream_t stream) {
  if (rows < 0 || rows > HB_MAX_TICK_ROWS) return fail(HB_ERR_INVALID, "rows %d outside [0, %d]", rows, HB_MAX_TICK_ROWS);
  if (rows == 0) return HB_OK;
  if (tokens == nullptr || cu_seq_q == nullptr || logit_offsets == nullptr || predictions == nullptr ||
      accepted == nullptr || emitted == nullptr)
    return fail(HB_ERR_INVALID, "null verification pointer");
  hb::VerifyParams p{tokens, cu_seq_q, logit_offsets, predictions, rows, accepted, emitted};
  const unsigned blocks = static_cast<unsigned>((rows + hb::kVerifyThreads - 1) / hb::kVerifyThreads);
  hb::verify_drafts_kernel<<<blocks, hb::kVerifyThreads, 0, stream>>>(p);
  return check_launch("verify_drafts_kernel");
}

}  // extern "C"
