// KV append: scatter this step's K/V rows into the paged pool by slot.
//
// Replaces PagedKVCache.write (src/nanovllm_ascend/npu/paged_kv_cache.py:44-69),
// i.e. pool_flat.index_copy_(0, slot_mapping, rows) for K and for V.
//
// HBM-bound byte movement: algorithmic traffic per token is
// 2 (K,V) * row_bytes read + 2 * row_bytes written + 8 B of slot.
// Each thread moves 16-byte words (LDG.128 / STG.128); one warp covers 512
// contiguous bytes of a row, so both the gather side (token-major inputs) and
// the scatter side (one whole pool row per slot) are fully coalesced. K and V
// go in the same launch; several independent words per thread are in flight
// before the first store so small (decode-sized) appends are latency-, not
// issue-bound.
#include "host_common.h"
#include "nvk_common.cuh"

namespace nvk {
namespace {

constexpr int kAppendThreads = 256;
constexpr int64_t kBulkMinTokens = 1024;  // below this the register path's one round trip is shorter
constexpr int kAppendUnroll = 4;

__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// One work item = one 16-byte word of one token's K row and the matching word
// of its V row. words_per_row = num_kv_heads * head_dim * 2 / 16.
__global__ void __launch_bounds__(kAppendThreads) kv_append_kernel(
    const uint4* __restrict__ key, const uint4* __restrict__ value, int64_t key_stride_w, int64_t value_stride_w,
    uint4* __restrict__ key_cache, uint4* __restrict__ value_cache, const int64_t* __restrict__ slots,
    int64_t num_tokens, int64_t num_slots, int words_per_row, int* __restrict__ error_word) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t total = num_tokens * words_per_row;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; base < total;
       base += stride * kAppendUnroll) {
    uint4 kv[kAppendUnroll], vv[kAppendUnroll];
    int64_t dst[kAppendUnroll];
#pragma unroll
    for (int u = 0; u < kAppendUnroll; ++u) {
      const int64_t i = base + u * stride;
      dst[u] = -1;
      if (i < total) {
        const int64_t t = i / words_per_row;
        const int w = static_cast<int>(i - t * words_per_row);
        const int64_t s = __ldg(slots + t);
        if (s >= 0 && s < num_slots) {
          dst[u] = s * words_per_row + w;
          kv[u] = ldg_stream(key + t * key_stride_w + w);
          vv[u] = ldg_stream(value + t * value_stride_w + w);
        } else if (error_word != nullptr && w == 0) {
          atomicOr(error_word, kErrBadSlot);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kAppendUnroll; ++u) {
      if (dst[u] >= 0) {
        key_cache[dst[u]] = kv[u];
        value_cache[dst[u]] = vv[u];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Large appends (prefill-sized): whole rows move by TMA bulk copies, global ->
// shared -> global, so reads and writes stream concurrently without a
// register round trip. Each of kBulkWarps warps per CTA owns an interleaved
// set of rows and a ring of kBulkStages (K row, V row) stages; its lane 0
// keeps up to kBulkStages - kBulkLag rows loading while the stores of the
// last kBulkLag rows drain, reusing a stage once its store has read it
// (cp.async.bulk.wait_group.read). Slots come 32 at a time, one per lane.
constexpr int kBulkWarps = 4;
constexpr int kBulkStages = 12;
constexpr int kBulkLag = 4;  // stores in flight per warp before a stage is reused
constexpr int kBulkMaxRowBytes = 2048;

struct BulkSmem {
  alignas(128) uint8_t k[kBulkWarps][kBulkStages][kBulkMaxRowBytes];
  alignas(128) uint8_t v[kBulkWarps][kBulkStages][kBulkMaxRowBytes];
  uint64_t full[kBulkWarps][kBulkStages];
};

__global__ void __launch_bounds__(kBulkWarps * 32, 1) kv_append_bulk_kernel(
    const uint8_t* __restrict__ key, const uint8_t* __restrict__ value, int64_t key_stride_b, int64_t value_stride_b,
    uint8_t* __restrict__ key_cache, uint8_t* __restrict__ value_cache, const int64_t* __restrict__ slots,
    int64_t num_tokens, int64_t num_slots, int row_bytes, int* __restrict__ error_word) {
  extern __shared__ uint8_t smem_raw[];
  BulkSmem& sm = *reinterpret_cast<BulkSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    for (int s = 0; s < kBulkStages; ++s) mbar_init(&sm.full[warp][s], 1);
    fence_mbar_init();
  }
  __syncwarp();
  pdl_launch_dependents();
  pdl_wait();
  const int64_t nw = static_cast<int64_t>(gridDim.x) * kBulkWarps;
  const int64_t w0 = static_cast<int64_t>(blockIdx.x) * kBulkWarps + warp;
  const int64_t n = w0 < num_tokens ? (num_tokens - w0 + nw - 1) / nw : 0;  // rows of this warp: w0 + i * nw
  const uint32_t rb = static_cast<uint32_t>(row_bytes);
  int64_t loaded = 0;  // rows whose load lane 0 has issued (in order)
  auto issue_load = [&](int64_t i) {
    ++loaded;
    const int s = static_cast<int>(i % kBulkStages);
    const int64_t t = w0 + i * nw;
    mbar_arrive_expect_tx(&sm.full[warp][s], 2 * rb);
    bulk_load(sm.k[warp][s], key + t * key_stride_b, rb, &sm.full[warp][s]);
    bulk_load(sm.v[warp][s], value + t * value_stride_b, rb, &sm.full[warp][s]);
  };
  bool ok = true;
  int64_t slot_chunk = 0;
  if (lane == 0)
    for (int64_t i = 0; i < n && i < kBulkStages; ++i) issue_load(i);
  for (int64_t i = 0; i < n; ++i) {
    if ((i & 31) == 0) {  // this lane's slot of the next 32 rows
      const int64_t ii = i + lane;
      slot_chunk = ii < n ? slots[w0 + ii * nw] : -1;
    }
    const int64_t slot = __shfl_sync(0xffffffffu, slot_chunk, static_cast<int>(i & 31));
    if (lane == 0) {
      const int s = static_cast<int>(i % kBulkStages);
      if (ok && !mbar_wait(&sm.full[warp][s], static_cast<uint32_t>((i / kBulkStages) & 1))) ok = false;
      if (ok && slot >= 0 && slot < num_slots) {
        bulk_store(key_cache + slot * rb, sm.k[warp][s], rb);
        bulk_store(value_cache + slot * rb, sm.v[warp][s], rb);
      } else if (ok && error_word != nullptr) {
        atomicOr(error_word, kErrBadSlot);
      }
      bulk_commit();  // one group per row, empty for a skipped row
      // The stage of row i - kBulkLag + 1 is free once at most kBulkLag - 1
      // newer store groups still read shared memory; refill it.
      const int64_t nxt = i - kBulkLag + 1 + kBulkStages;
      if (ok && i >= kBulkLag - 1 && nxt < n) {
        bulk_wait_read<kBulkLag - 1>();
        issue_load(nxt);
      }
    }
  }
  if (lane == 0) {
    if (!ok && error_word != nullptr) atomicOr(error_word, kErrWaitTimeout);
    // Drain: every load issued lands and every store completes before exit.
    for (int64_t i = loaded > kBulkStages ? loaded - kBulkStages : 0; i < loaded; ++i)
      (void)mbar_wait(&sm.full[warp][i % kBulkStages], static_cast<uint32_t>((i / kBulkStages) & 1));
    bulk_wait_all();
  }
}

}  // namespace
}  // namespace nvk

extern "C" int nvk_kv_append(const void* key, const void* value, int64_t key_token_stride,
                             int64_t value_token_stride, void* key_cache, void* value_cache,
                             const int64_t* slot_mapping, int64_t num_tokens, int64_t num_slots, int num_kv_heads,
                             int head_dim, int* error_word, nvk_stream_t stream) {
  using namespace nvk;
  if (num_tokens < 0 || num_slots < 0 || num_kv_heads <= 0 || head_dim <= 0)
    return fail(NVK_ERR_INVALID_ARGUMENT, "kv_append: negative or zero size (tokens=%lld slots=%lld kvh=%d d=%d)",
                (long long)num_tokens, (long long)num_slots, num_kv_heads, head_dim);
  if (num_tokens == 0) return NVK_OK;
  const int64_t row_bytes = static_cast<int64_t>(num_kv_heads) * head_dim * 2;
  if (row_bytes % 16 != 0)
    return fail(NVK_ERR_UNSUPPORTED, "kv_append: row of %lld bytes is not a multiple of 16", (long long)row_bytes);
  if (!key || !value || !key_cache || !value_cache || !slot_mapping)
    return fail(NVK_ERR_INVALID_ARGUMENT, "kv_append: null pointer");
  if (!aligned16(key) || !aligned16(value) || !aligned16(key_cache) || !aligned16(value_cache))
    return fail(NVK_ERR_INVALID_ARGUMENT, "kv_append: buffers must be 16-byte aligned");
  if ((key_token_stride * 2) % 16 != 0 || (value_token_stride * 2) % 16 != 0 ||
      key_token_stride < num_kv_heads * head_dim || value_token_stride < num_kv_heads * head_dim)
    return fail(NVK_ERR_INVALID_ARGUMENT, "kv_append: token strides (%lld, %lld) must cover a row and be 16-byte multiples",
                (long long)key_token_stride, (long long)value_token_stride);
  const int words_per_row = static_cast<int>(row_bytes / 16);
  const int64_t total = num_tokens * words_per_row;
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (num_tokens >= kBulkMinTokens && row_bytes <= kBulkMaxRowBytes) {
    const size_t smem = sizeof(BulkSmem) + 128;
    int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(&kv_append_bulk_kernel), smem);
    if (rc != NVK_OK) return rc;
    const int64_t warps_needed = (num_tokens + 7) / 8;  // at least ~8 rows per warp
    const int64_t want = (warps_needed + kBulkWarps - 1) / kBulkWarps;
    const int grid = static_cast<int>(want < sms ? want : sms);
    const cudaError_t e = launch_pdl(kv_append_bulk_kernel, dim3(grid), dim3(kBulkWarps * 32), smem,
                                     reinterpret_cast<cudaStream_t>(stream), static_cast<const uint8_t*>(key),
                                     static_cast<const uint8_t*>(value), key_token_stride * 2, value_token_stride * 2,
                                     static_cast<uint8_t*>(key_cache), static_cast<uint8_t*>(value_cache),
                                     slot_mapping, num_tokens, num_slots, static_cast<int>(row_bytes), error_word);
    return check_cuda(e, "kv_append (bulk) launch");
  }
  const int64_t want = (total + int64_t(kAppendThreads) * kAppendUnroll - 1) / (int64_t(kAppendThreads) * kAppendUnroll);
  const int blocks = static_cast<int>(want < int64_t(sms) * 8 ? (want > 0 ? want : 1) : int64_t(sms) * 8);
  const cudaError_t e = launch_pdl(kv_append_kernel, dim3(blocks), dim3(kAppendThreads), 0,
                                   reinterpret_cast<cudaStream_t>(stream), static_cast<const uint4*>(key),
                                   static_cast<const uint4*>(value), key_token_stride * 2 / 16,
                                   value_token_stride * 2 / 16, static_cast<uint4*>(key_cache),
                                   static_cast<uint4*>(value_cache), slot_mapping, num_tokens, num_slots,
                                   words_per_row, error_word);
  return check_cuda(e, "kv_append launch");
}
