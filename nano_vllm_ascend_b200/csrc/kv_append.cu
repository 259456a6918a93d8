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
