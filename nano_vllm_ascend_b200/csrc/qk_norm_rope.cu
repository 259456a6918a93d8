// Fused per-head RMSNorm of q and k, rotary embedding ("half" mode) and the
// KV append -- the prologue of Qwen3Attention.forward
// (src/nanovllm_ascend/models/qwen3.py:83-96): q_norm / k_norm
// (layers/layernorm.py:12-17, npu_rms_norm over head_dim), then
// apply_rotary_pos_emb_tnd (layers/rotary_embedding.py:58-99, npu_rotary_mul
// rotary_mode="half" with cos/sin rows of the fp32 tables cast to bf16),
// then PagedKVCache.write of the rotated k and of v. One read of q, k, v;
// the rotated q goes to q_out, k and v go to the pool rows of their slots.
//
// Half a warp per head row: lane l of a half holds dims {4l .. 4l+3} and
// {64+4l .. 64+4l+3} (two 8-byte words), so each rotation pair (i, i+64) is
// in one lane and a row is two coalesced 128-byte loads. A warp works on a
// group of rows of one token (its position, slot and cos/sin loaded once)
// and keeps kPairs row pairs (2 * kPairs rows) of loads in flight before
// their reductions: a 16-lane reduction for the mean square, then
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
constexpr int kPairs = 8;  // row pairs in flight per warp

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
  int group_rows;  // head rows per warp, even
  float eps;
  int* err;
};

__device__ __forceinline__ void unpack4(uint2 w, float (&x)[4]) {
  x[0] = bf16lo_to_f32(w.x);
  x[1] = bf16hi_to_f32(w.x);
  x[2] = bf16lo_to_f32(w.y);
  x[3] = bf16hi_to_f32(w.y);
}

__device__ __forceinline__ uint2 load8(const __nv_bfloat16* p) { return *reinterpret_cast<const uint2*>(p); }

// Normalises and rotates one 128-dim head row held by a half warp as this
// lane's dims {4l .. 4l+3} (w_lo) and {64+4l .. 64+4l+3} (w_hi); g_*, c_*, s_*
// are this lane's weights and bf16-rounded cos/sin values as bf16 pairs.
// Every lane of the warp must call it (the reduction shuffles stay inside
// each half).
__device__ __forceinline__ void norm_rope_row(uint2 w_lo, uint2 w_hi, uint2 g_lo, uint2 g_hi, uint2 c_lo, uint2 c_hi,
                                              uint2 s_lo, uint2 s_hi, float eps, uint2& o_lo, uint2& o_hi) {
  float x0[4], x1[4];
  unpack4(w_lo, x0);
  unpack4(w_hi, x1);
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) ss += x0[k] * x0[k] + x1[k] * x1[k];
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float rinv = rsqrtf(ss * (1.f / kD) + eps);
  float g0[4], g1[4], y0[4], y1[4], r0[4], r1[4];
  unpack4(g_lo, g0);
  unpack4(g_hi, g1);
#pragma unroll
  for (int k = 0; k < 4; ++k) {  // normalised row, rounded to bf16 as the norm's output is
    y0[k] = round_bf16(x0[k] * rinv * g0[k]);
    y1[k] = round_bf16(x1[k] * rinv * g1[k]);
  }
  float c0[4], c1[4], s0[4], s1[4];
  unpack4(c_lo, c0);
  unpack4(c_hi, c1);
  unpack4(s_lo, s0);
  unpack4(s_hi, s1);
  // out[i] = y[i] cos[i] - y[i+64] sin[i];  out[i+64] = y[i+64] cos[i+64] + y[i] sin[i+64]
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    r0[k] = y0[k] * c0[k] - y1[k] * s0[k];
    r1[k] = y1[k] * c1[k] + y0[k] * s1[k];
  }
  o_lo = make_uint2(pack_bf16x2(r0[0], r0[1]), pack_bf16x2(r0[2], r0[3]));
  o_hi = make_uint2(pack_bf16x2(r1[0], r1[1]), pack_bf16x2(r1[2], r1[3]));
}

// bf16 rounding of four fp32 table values, packed as two bf16 pairs.
__device__ __forceinline__ uint2 table4(const float* p) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  return make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
}

__global__ void __launch_bounds__(kWarps * 32, 2) qk_norm_rope_append_kernel(const NormRopeArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int half = lane >> 4, hl = lane & 15;
  const int d_lo = 4 * hl, d_hi = 64 + 4 * hl;
  const uint2 gq_lo = load8(a.q_weight + d_lo), gq_hi = load8(a.q_weight + d_hi);
  const uint2 gk_lo = load8(a.k_weight + d_lo), gk_hi = load8(a.k_weight + d_hi);
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
    uint2 c_lo = make_uint2(0u, 0u), c_hi = c_lo, s_lo = c_lo, s_hi = c_lo;
    if (r_lo < nqk) {
      int64_t p = a.positions[t];
      if (p < 0 || p >= a.max_pos) {
        if (lane == 0 && r_lo == 0 && a.err) atomicOr(a.err, kErrContextTooLong);
        p = p < 0 ? 0 : a.max_pos - 1;
      }
      // cos/sin rows cast to bf16 (apply_rotary_pos_emb_tnd casts them to q's dtype)
      c_lo = table4(a.cos_table + p * kD + d_lo);
      c_hi = table4(a.cos_table + p * kD + d_hi);
      s_lo = table4(a.sin_table + p * kD + d_lo);
      s_hi = table4(a.sin_table + p * kD + d_hi);
    }
    for (int r0 = r_lo; r0 < r_hi; r0 += 2 * kPairs) {
      uint2 lo[kPairs], hi[kPairs];
#pragma unroll
      for (int u = 0; u < kPairs; ++u) {
        const int r = r0 + 2 * u + half;
        const __nv_bfloat16* src = r < a.num_heads ? a.q + t * a.q_stride + r * kD
                                 : r < nqk       ? a.k + t * a.k_stride + (r - a.num_heads) * kD
                                                 : a.v + t * a.v_stride + (r - nqk) * kD;
        const bool in = r < r_hi;
        lo[u] = in ? load8(src + d_lo) : make_uint2(0u, 0u);
        hi[u] = in ? load8(src + d_hi) : make_uint2(0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < kPairs; ++u) {
        if (r0 + 2 * u >= r_hi) break;  // warp-uniform: both halves are past the group's end
        const int r = r0 + 2 * u + half;
        const bool is_q = r < a.num_heads;
        uint2 o_lo = lo[u], o_hi = hi[u];
        if (r0 + 2 * u < nqk) {  // at least one half holds a q or k row: the whole warp reduces
          uint2 n_lo, n_hi;
          norm_rope_row(lo[u], hi[u], is_q ? gq_lo : gk_lo, is_q ? gq_hi : gk_hi, c_lo, c_hi, s_lo, s_hi, a.eps,
                        n_lo, n_hi);
          if (r < nqk) {
            o_lo = n_lo;
            o_hi = n_hi;
          }
        }
        if (r >= r_hi) continue;
        __nv_bfloat16* dst;
        if (is_q) {
          dst = a.q_out + (t * a.num_heads + r) * kD;
        } else {
          if (!slot_ok) continue;
          dst = r < nqk ? a.key_cache + (slot * a.num_kv_heads + r - a.num_heads) * kD
                        : a.value_cache + (slot * a.num_kv_heads + r - nqk) * kD;
        }
        *reinterpret_cast<uint2*>(dst + d_lo) = o_lo;
        *reinterpret_cast<uint2*>(dst + d_hi) = o_hi;
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
  auto al8 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; };
  if (!al8(query) || !al8(key) || !al8(value) || !al8(q_weight) || !al8(k_weight) || !al8(query_out) ||
      query_stride % 4 || key_stride % 4 || value_stride % 4 || query_stride < int64_t(num_heads) * kD ||
      key_stride < int64_t(num_kv_heads) * kD || value_stride < int64_t(num_kv_heads) * kD)
    return fail(NVK_ERR_INVALID_ARGUMENT,
                "qk_norm_rope_append: rows must be 8-byte aligned (strides multiples of 4) and strides cover a row");
  if (!aligned16(cos_table) || !aligned16(sin_table))
    return fail(NVK_ERR_INVALID_ARGUMENT, "qk_norm_rope_append: cos/sin tables must be 16-byte aligned");
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
  const int group_rows = num_tokens >= int64_t(sms) * 16 ? (nrows + 1) / 2 * 2 : 4;  // even: rows go in pairs
  a.group_rows = group_rows;
  const int64_t groups = (nrows + group_rows - 1) / group_rows;
  const int64_t want = (num_tokens * groups + kWarps - 1) / kWarps;
  const int grid = static_cast<int>(want < int64_t(sms) * 16 ? want : int64_t(sms) * 16);
  return check_cuda(launch_pdl(qk_norm_rope_append_kernel, dim3(grid), dim3(kWarps * 32), 0,
                               reinterpret_cast<cudaStream_t>(stream), a),
                    "qk_norm_rope_append launch");
}
