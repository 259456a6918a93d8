// Fused per-head RMSNorm of q and k, rotary embedding ("half" mode) and the
// KV append -- the prologue of Qwen3Attention.forward
// (src/nanovllm_ascend/models/qwen3.py:83-96): q_norm / k_norm
// (layers/layernorm.py:12-17, npu_rms_norm over head_dim), then
// apply_rotary_pos_emb_tnd (layers/rotary_embedding.py:58-99, npu_rotary_mul
// rotary_mode="half" with cos/sin rows of the fp32 tables cast to bf16),
// then PagedKVCache.write of the rotated k and of v. One read of q, k, v;
// the rotated q goes to q_out, k and v go to the pool rows of their slots.
//
// One warp per 8 head rows of a token, four rows at a time (cos/sin loaded
// once per warp).
// Lane l holds dims {2l, 2l+1} and {64+2l, 64+2l+1} of a row, so each
// rotation pair (i, i+64) is in one lane: a warp reduction for the mean
// square, then
//   y  = bf16(x * rsqrt(mean(x^2) + eps) * w)                (fp32 arithmetic)
//   out = bf16(y * cos + rotate_half(y) * sin),  rotate_half(y) = (-y[64:], y[:64])
// HBM-bound elementwise work: per token (H + KVH) * 256 B read and written for
// q and k, KVH * 256 B copied for v.
#include "host_common.h"
#include "nvk_common.cuh"

namespace nvk {
namespace {

constexpr int kD = 128;
constexpr int kWarps = 8;

__device__ __forceinline__ float2 bf16x2_to_f32(uint32_t w) { return make_float2(bf16lo_to_f32(w), bf16hi_to_f32(w)); }
__device__ __forceinline__ float round_bf16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

struct NormRopeArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t q_stride, k_stride, v_stride;  // elements between tokens
  const __nv_bfloat16* q_weight;
  const __nv_bfloat16* k_weight;
  const float* cos_table;  // [max_pos, 128] fp32
  const float* sin_table;
  int max_pos;
  const int64_t* positions;
  const int64_t* slots;
  __nv_bfloat16* q_out;  // [T, H, 128] contiguous
  __nv_bfloat16* key_cache;
  __nv_bfloat16* value_cache;
  int64_t num_tokens, num_slots;
  int num_heads, num_kv_heads;
  int group_rows;  // head rows per warp, a multiple of 4
  float eps;
  int* err;
};

// Normalises and rotates one 128-dim head row held as lane dims {2l, 2l+1}
// (w_lo) and {64+2l, 65+2l} (w_hi); the cos/sin pairs are this lane's.
__device__ __forceinline__ void norm_rope_row(uint32_t w_lo, uint32_t w_hi, float2 g0, float2 g1, float2 c0,
                                              float2 c1, float2 s0, float2 s1, float eps, uint32_t& o_lo,
                                              uint32_t& o_hi) {
  const float2 x0 = bf16x2_to_f32(w_lo), x1 = bf16x2_to_f32(w_hi);
  float ss = x0.x * x0.x + x0.y * x0.y + x1.x * x1.x + x1.y * x1.y;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float rinv = rsqrtf(ss * (1.f / kD) + eps);
  // normalised row, rounded to bf16 as the norm's output is
  const float y0 = round_bf16(x0.x * rinv * g0.x), y1 = round_bf16(x0.y * rinv * g0.y);
  const float y2 = round_bf16(x1.x * rinv * g1.x), y3 = round_bf16(x1.y * rinv * g1.y);
  // out[i] = y[i] cos[i] - y[i+64] sin[i];  out[i+64] = y[i+64] cos[i+64] + y[i] sin[i+64]
  o_lo = pack_bf16x2(y0 * c0.x - y2 * s0.x, y1 * c0.y - y3 * s0.y);
  o_hi = pack_bf16x2(y2 * c1.x + y0 * s1.x, y3 * c1.y + y1 * s1.y);
}

// One warp per group of group_rows head rows of one token (rows: the q heads,
// then the k heads, then the v heads): the token's position, slot and
// cos/sin pairs are loaded once per group, and the group's rows go kBatch at
// a time (loads of kBatch rows in flight before their reductions).
constexpr int kBatch = 8;

__global__ void __launch_bounds__(kWarps * 32) qk_norm_rope_append_kernel(const NormRopeArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const float2 gq0 = bf16x2_to_f32(*reinterpret_cast<const uint32_t*>(a.q_weight + 2 * lane));
  const float2 gq1 = bf16x2_to_f32(*reinterpret_cast<const uint32_t*>(a.q_weight + 64 + 2 * lane));
  const float2 gk0 = bf16x2_to_f32(*reinterpret_cast<const uint32_t*>(a.k_weight + 2 * lane));
  const float2 gk1 = bf16x2_to_f32(*reinterpret_cast<const uint32_t*>(a.k_weight + 64 + 2 * lane));
  const int nrows = a.num_heads + 2 * a.num_kv_heads;
  const int nqk = a.num_heads + a.num_kv_heads;
  const int groups = (nrows + a.group_rows - 1) / a.group_rows;
  const int64_t items = a.num_tokens * groups;
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5); w < items;
       w += static_cast<int64_t>(gridDim.x) * kWarps) {
    const int64_t t = w / groups;
    const int r_lo = static_cast<int>(w - t * groups) * a.group_rows;
    const int r_hi = min(r_lo + a.group_rows, nrows);
    const int64_t slot = a.slots[t];
    const bool slot_ok = slot >= 0 && slot < a.num_slots;
    if (!slot_ok && lane == 0 && r_lo == 0 && a.err) atomicOr(a.err, kErrBadSlot);
    float2 c0 = make_float2(0.f, 0.f), c1 = c0, s0 = c0, s1 = c0;
    if (r_lo < nqk) {
      int64_t p = a.positions[t];
      if (p < 0 || p >= a.max_pos) {
        if (lane == 0 && r_lo == 0 && a.err) atomicOr(a.err, kErrContextTooLong);
        p = p < 0 ? 0 : a.max_pos - 1;
      }
      const float* cr = a.cos_table + p * kD;
      const float* sr = a.sin_table + p * kD;
      // cos/sin rows cast to bf16 (apply_rotary_pos_emb_tnd casts them to q's dtype)
      c0 = make_float2(round_bf16(cr[2 * lane]), round_bf16(cr[2 * lane + 1]));
      c1 = make_float2(round_bf16(cr[64 + 2 * lane]), round_bf16(cr[65 + 2 * lane]));
      s0 = make_float2(round_bf16(sr[2 * lane]), round_bf16(sr[2 * lane + 1]));
      s1 = make_float2(round_bf16(sr[64 + 2 * lane]), round_bf16(sr[65 + 2 * lane]));
    }
    for (int r0 = r_lo; r0 < r_hi; r0 += kBatch) {
      uint32_t lo[kBatch], hi[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int r = r0 + u;
        const __nv_bfloat16* src = r < a.num_heads ? a.q + t * a.q_stride + r * kD
                                 : r < nqk       ? a.k + t * a.k_stride + (r - a.num_heads) * kD
                                                 : a.v + t * a.v_stride + (r - nqk) * kD;
        lo[u] = r < r_hi ? *reinterpret_cast<const uint32_t*>(src + 2 * lane) : 0u;
        hi[u] = r < r_hi ? *reinterpret_cast<const uint32_t*>(src + 64 + 2 * lane) : 0u;
      }
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int r = r0 + u;
        if (r >= r_hi) break;
        __nv_bfloat16* dst;
        uint32_t o_lo = lo[u], o_hi = hi[u];
        if (r < nqk) {
          const bool is_q = r < a.num_heads;
          norm_rope_row(lo[u], hi[u], is_q ? gq0 : gk0, is_q ? gq1 : gk1, c0, c1, s0, s1, a.eps, o_lo, o_hi);
          if (!is_q && !slot_ok) continue;
          dst = is_q ? a.q_out + (t * a.num_heads + r) * kD : a.key_cache + (slot * a.num_kv_heads + r - a.num_heads) * kD;
        } else {  // v: a raw copy
          if (!slot_ok) continue;
          dst = a.value_cache + (slot * a.num_kv_heads + r - nqk) * kD;
        }
        *reinterpret_cast<uint32_t*>(dst + 2 * lane) = o_lo;
        *reinterpret_cast<uint32_t*>(dst + 64 + 2 * lane) = o_hi;
      }
    }
  }
}

}  // namespace
}  // namespace nvk

extern "C" int nvk_qk_norm_rope_append(const void* query, const void* key, const void* value, int64_t query_stride,
                                       int64_t key_stride, int64_t value_stride, const void* q_weight,
                                       const void* k_weight, float eps, const float* cos_table,
                                       const float* sin_table, int max_position, const int64_t* positions,
                                       void* query_out, void* key_cache, void* value_cache,
                                       const int64_t* slot_mapping, int64_t num_tokens, int64_t num_slots,
                                       int num_heads, int num_kv_heads, int head_dim, int* error_word,
                                       nvk_stream_t stream) {
  using namespace nvk;
  if (num_tokens < 0 || num_heads <= 0 || num_kv_heads <= 0 || num_slots < 0 || max_position <= 0)
    return fail(NVK_ERR_INVALID_ARGUMENT, "qk_norm_rope_append: bad sizes (tokens=%lld heads=%d kv_heads=%d)",
                (long long)num_tokens, num_heads, num_kv_heads);
  if (head_dim != kD) return fail(NVK_ERR_UNSUPPORTED, "qk_norm_rope_append: head_dim %d unsupported (128 only)",
                                  head_dim);
  if (num_tokens == 0) return NVK_OK;
  if (!query || !key || !value || !q_weight || !k_weight || !cos_table || !sin_table || !positions || !query_out ||
      !key_cache || !value_cache || !slot_mapping)
    return fail(NVK_ERR_INVALID_ARGUMENT, "qk_norm_rope_append: null pointer");
  auto al4 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; };
  if (!al4(query) || !al4(key) || !al4(value) || !al4(q_weight) || !al4(k_weight) || !al4(query_out) ||
      query_stride % 2 || key_stride % 2 || value_stride % 2 || query_stride < int64_t(num_heads) * kD ||
      key_stride < int64_t(num_kv_heads) * kD || value_stride < int64_t(num_kv_heads) * kD)
    return fail(NVK_ERR_INVALID_ARGUMENT, "qk_norm_rope_append: rows must be 4-byte aligned and strides cover a row");
  NormRopeArgs a;
  a.q = static_cast<const __nv_bfloat16*>(query);
  a.k = static_cast<const __nv_bfloat16*>(key);
  a.v = static_cast<const __nv_bfloat16*>(value);
  a.q_stride = query_stride;
  a.k_stride = key_stride;
  a.v_stride = value_stride;
  a.q_weight = static_cast<const __nv_bfloat16*>(q_weight);
  a.k_weight = static_cast<const __nv_bfloat16*>(k_weight);
  a.cos_table = cos_table;
  a.sin_table = sin_table;
  a.max_pos = max_position;
  a.positions = positions;
  a.slots = slot_mapping;
  a.q_out = static_cast<__nv_bfloat16*>(query_out);
  a.key_cache = static_cast<__nv_bfloat16*>(key_cache);
  a.value_cache = static_cast<__nv_bfloat16*>(value_cache);
  a.num_tokens = num_tokens;
  a.num_slots = num_slots;
  a.num_heads = num_heads;
  a.num_kv_heads = num_kv_heads;
  a.eps = eps;
  a.err = error_word;
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // A whole token per warp (cos/sin loaded once per token) when the tokens
  // alone give every SM 16 warps; else four rows per warp, for parallelism.
  const int nrows = num_heads + 2 * num_kv_heads;
  const int group_rows = num_tokens >= int64_t(sms) * 16 ? (nrows + 3) / 4 * 4 : 4;
  a.group_rows = group_rows;
  const int64_t groups = (nrows + group_rows - 1) / group_rows;
  const int64_t want = (num_tokens * groups + kWarps - 1) / kWarps;
  const int grid = static_cast<int>(want < int64_t(sms) * 16 ? want : int64_t(sms) * 16);
  return check_cuda(launch_pdl(qk_norm_rope_append_kernel, dim3(grid), dim3(kWarps * 32), 0,
                               reinterpret_cast<cudaStream_t>(stream), a),
                    "qk_norm_rope_append launch");
}
