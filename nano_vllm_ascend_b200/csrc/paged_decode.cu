// Paged GQA decode attention (one query token per sequence).
//
// Replaces torch_npu._npu_paged_attention as called from
// src/nanovllm_ascend/layers/npu_paged_attention.py:58,89 (and the graph
// task update at src/nanovllm_ascend/npu/acl_graph.py:232):
//   out[b,h] = softmax(scale * q[b,h] . K[b,:,g(h)]^T) . V[b,:,g(h)]
// over the first context_lens[b] tokens reached through block_tables[b].
//
// B200 design (HBM-bound: every KV byte is read exactly once):
//  * grid = (split, kv_head, seq). A CTA owns one KV head of one sequence over
//    `blocks_per_split` pool blocks and serves ALL query heads of that GQA
//    group from the same KV read.
//  * warp 4 = producer: stages the split's block ids in shared memory, then
//    one lane streams 64-token stages of K and V (two 64-dim halves each) with
//    3-D TMA tile loads (box {64 dims, 1 head, <=32 tokens}, 128-byte swizzle)
//    into a STAGES-deep ring guarded by full/empty mbarriers.
//  * warps 0-3 = consumers: each owns 16 tokens of a stage. LPT = 2*QPK lanes
//    share a token, each holding 64/QPK dims of every query head of the group
//    in registers (q pre-scaled by scale*log2 e), so q and the f32
//    accumulators take 64 registers each whatever the GQA ratio. The lane ->
//    (token, 16-byte chunk) map is chosen against the 128-byte swizzle so that
//    every quarter-warp of a 128-bit shared load hits 8 distinct bank groups.
//  * online softmax in base 2 with lazy rescaling (the running max only moves
//    when a tile max exceeds it by more than 2^8), per warp; warps merge once
//    at the end through shared memory.
//  * split-K without a second launch: every split writes (m, l, o) partials;
//    the last CTA of a (seq, kv_head) to arrive (atomic ticket) merges them and
//    resets the ticket, so the workspace is reusable and graph-capturable.
#include <cfloat>
#include <mutex>

#include "host_common.h"
#include "nvk_common.cuh"

namespace nvk {
namespace {

constexpr int kD = 128;
constexpr int kTile = 64;  // tokens per pipeline stage
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kHalfBytes = kTile * 128;        // 64 tokens x 64 dims x bf16
constexpr int kStageBytes = 4 * kHalfBytes;    // K lo, K hi, V lo, V hi
constexpr int kTokPerWarp = kTile / kConsumerWarps;
constexpr int kMaxSplitBlocks = 256;
constexpr int kStages = 3;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct DecodeArgs {
  __nv_bfloat16* out;
  const __nv_bfloat16* q;
  const int32_t* block_tables;
  const int32_t* context_lens;
  float* ws_o;
  float2* ws_ml;
  int* ws_cnt;
  int* err;
  int bt_stride;
  int max_blocks;
  int num_blocks;
  int block_size;
  int log2_bs;
  int sub_rows;
  int num_heads;
  int num_kv_heads;
  int blocks_per_split;
  int max_splits;
  float scale_log2;
};

template <int QPK>
struct Layout {
  static constexpr int kLPT = 2 * QPK;         // lanes per token
  static constexpr int kDPL = kD / kLPT;       // dims per lane
  static constexpr int kNCH = kDPL / 8;        // 16-byte chunks per lane
  static constexpr int kTPP = 32 / kLPT;       // tokens per warp pass
  static constexpr int kNP = kTokPerWarp / kTPP;  // passes per stage
  static_assert(kNCH >= 1 && kNP >= 1, "bad GQA ratio");
};

template <int QPK>
struct Smem {
  alignas(1024) uint8_t stage[kStages][kStageBytes];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  int blocks[kMaxSplitBlocks];
  float red_m[kConsumerWarps][QPK];
  float red_l[kConsumerWarps][QPK];
  float red_o[kConsumerWarps][QPK][kD];
  int last;
};

// Two CTAs per SM while q + accumulators fit (QPK <= 2); one above that.
template <int QPK>
__global__ void __launch_bounds__(kThreads, (QPK <= 2) ? 2 : 1) paged_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                   const __grid_constant__ CUtensorMap vmap,
                                                                   const DecodeArgs a) {
  using Lay = Layout<QPK>;
  constexpr int LPT = Lay::kLPT, DPL = Lay::kDPL, NCH = Lay::kNCH, TPP = Lay::kTPP, NP = Lay::kNP;

  const int split = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  int L = a.context_lens[b];
  if (L < 0) L = 0;
  if (L > a.max_blocks * a.block_size) {
    if (threadIdx.x == 0 && split == 0) atomicOr(a.err, kErrContextTooLong);
    L = a.max_blocks * a.block_size;
  }
  const int nblk = (L + a.block_size - 1) >> a.log2_bs;
  int nsplit = (nblk + a.blocks_per_split - 1) / a.blocks_per_split;
  if (nsplit < 1) nsplit = 1;
  if (split >= nsplit) return;  // uniform over the CTA

  extern __shared__ uint8_t smem_raw[];
  Smem<QPK>& sm = *reinterpret_cast<Smem<QPK>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int split_blk0 = split * a.blocks_per_split;
  const int split_nblk = min(a.blocks_per_split, nblk - split_blk0);
  const int tok_begin = split_blk0 * a.block_size;
  const int tok_end = min(L, tok_begin + a.blocks_per_split * a.block_size);
  const int ntiles = tok_end > tok_begin ? (tok_end - tok_begin + kTile - 1) / kTile : 0;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer --
    const int32_t* bt = a.block_tables + static_cast<int64_t>(b) * a.bt_stride + split_blk0;
    for (int i = lane; i < split_nblk; i += 32) {
      int blk = bt[i];
      if (blk < 0 || blk >= a.num_blocks) {
        atomicOr(a.err, kErrBadBlockId);
        blk = a.num_blocks;  // fully out of the tensor map: TMA fills zeros
      }
      sm.blocks[i] = blk;
    }
    __syncwarp();
    if (lane == 0) {
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      int issued = 0;
      bool ok = true;
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % kStages;
        if (t >= kStages && !mbar_wait(&sm.empty[s], ((t / kStages) - 1) & 1)) {
          atomicOr(a.err, kErrWaitTimeout);
          ok = false;
          break;
        }
        const int tile_tok = tok_begin + t * kTile;
        const int nsub = min(kTile / a.sub_rows, (tok_end - tile_tok + a.sub_rows - 1) / a.sub_rows);
        mbar_arrive_expect_tx(&sm.full[s], static_cast<uint32_t>(nsub * 4 * a.sub_rows * 128));
        uint8_t* st = sm.stage[s];
        for (int u = 0; u < nsub; ++u) {
          const int tok = tile_tok + u * a.sub_rows;
          const int blk = sm.blocks[(tok >> a.log2_bs) - split_blk0];
          const int row = blk * a.block_size + (tok & (a.block_size - 1));
          const int off = u * a.sub_rows * 128;
          tma_load_3d(st + 0 * kHalfBytes + off, &kmap, &sm.full[s], 0, g, row);
          tma_load_3d(st + 1 * kHalfBytes + off, &kmap, &sm.full[s], 64, g, row);
          tma_load_3d(st + 2 * kHalfBytes + off, &vmap, &sm.full[s], 0, g, row);
          tma_load_3d(st + 3 * kHalfBytes + off, &vmap, &sm.full[s], 64, g, row);
        }
        ++issued;
      }
      if (!ok) {
        // Drain: wait (bounded) for the copies this CTA still has in flight.
        for (int t = max(0, issued - kStages); t < issued; ++t)
          (void)mbar_wait(&sm.full[t % kStages], (t / kStages) & 1);
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers --
  int tok_in_pass, j;
  if constexpr (LPT == 16) {
    tok_in_pass = lane >> 4;
    j = lane & 15;
  } else {
    const int qtr = lane >> 3, r = lane & 7;
    j = r % LPT;
    tok_in_pass = (qtr / LPT) * 8 + (qtr % LPT) + LPT * (r / LPT);
  }

  const int h0 = g * QPK;
  float qr[QPK][DPL];
#pragma unroll
  for (int h = 0; h < QPK; ++h) {
    const __nv_bfloat16* qh = a.q + (static_cast<int64_t>(b) * a.num_heads + h0 + h) * kD;
#pragma unroll
    for (int i = 0; i < NCH; ++i) {
      const int gc = j + LPT * i;
      const uint4 w = *reinterpret_cast<const uint4*>(qh + gc * 8);
      const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        qr[h][i * 8 + 2 * e] = bf16lo_to_f32(ww[e]) * a.scale_log2;
        qr[h][i * 8 + 2 * e + 1] = bf16hi_to_f32(ww[e]) * a.scale_log2;
      }
    }
  }

  float m_run[QPK], l_run[QPK], acc[QPK][DPL];
#pragma unroll
  for (int h = 0; h < QPK; ++h) {
    m_run[h] = -INFINITY;
    l_run[h] = 0.f;
#pragma unroll
    for (int k = 0; k < DPL; ++k) acc[h][k] = 0.f;
  }

  for (int t = 0; t < ntiles; ++t) {
    const int s = t % kStages;
    if (!mbar_wait(&sm.full[s], (t / kStages) & 1)) {
      if (lane == 0) atomicOr(a.err, kErrWaitTimeout);
      break;
    }
    const uint32_t base = smem_u32(sm.stage[s]);
    const int tile_tok = tok_begin + t * kTile;

    float sc[NP][QPK];
#pragma unroll
    for (int p = 0; p < NP; ++p) {
      const int tl = warp * kTokPerWarp + p * TPP + tok_in_pass;
      const uint32_t row = base + tl * 128;
      const int sw = tl & 7;
      float dot[QPK];
#pragma unroll
      for (int h = 0; h < QPK; ++h) dot[h] = 0.f;
#pragma unroll
      for (int i = 0; i < NCH; ++i) {
        const int gc = j + LPT * i;
        const uint4 kw = ld_shared_v4(row + (gc >> 3) * kHalfBytes + (((gc & 7) ^ sw) << 4));
        const uint32_t ww[4] = {kw.x, kw.y, kw.z, kw.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float lo = bf16lo_to_f32(ww[e]), hi = bf16hi_to_f32(ww[e]);
#pragma unroll
          for (int h = 0; h < QPK; ++h) {
            dot[h] = fmaf(lo, qr[h][i * 8 + 2 * e], dot[h]);
            dot[h] = fmaf(hi, qr[h][i * 8 + 2 * e + 1], dot[h]);
          }
        }
      }
#pragma unroll
      for (int h = 0; h < QPK; ++h) {
#pragma unroll
        for (int off = 1; off < LPT; off <<= 1) dot[h] += __shfl_xor_sync(0xffffffffu, dot[h], off);
      }
      const bool valid = tile_tok + tl < tok_end;
#pragma unroll
      for (int h = 0; h < QPK; ++h) sc[p][h] = valid ? dot[h] : -INFINITY;
    }

    // Warp-wide tile max per head; lazy rescale of the running state.
#pragma unroll
    for (int h = 0; h < QPK; ++h) {
      float mx = sc[0][h];
#pragma unroll
      for (int p = 1; p < NP; ++p) mx = fmaxf(mx, sc[p][h]);
#pragma unroll
      for (int off = LPT; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      if (mx > m_run[h] + kRescaleThreshold) {
        const float alpha = fast_exp2(m_run[h] - mx);  // 0 when m_run = -inf
        m_run[h] = mx;
        l_run[h] *= alpha;
#pragma unroll
        for (int k = 0; k < DPL; ++k) acc[h][k] *= alpha;
      }
    }

#pragma unroll
    for (int p = 0; p < NP; ++p) {
      const int tl = warp * kTokPerWarp + p * TPP + tok_in_pass;
      if (tile_tok + tl < tok_end) {  // rows past the context may hold any bits
        float pr[QPK];
#pragma unroll
        for (int h = 0; h < QPK; ++h) {
          pr[h] = fast_exp2(sc[p][h] - m_run[h]);
          l_run[h] += pr[h];
        }
        const uint32_t row = base + 2 * kHalfBytes + tl * 128;
        const int sw = tl & 7;
#pragma unroll
        for (int i = 0; i < NCH; ++i) {
          const int gc = j + LPT * i;
          const uint4 vw = ld_shared_v4(row + (gc >> 3) * kHalfBytes + (((gc & 7) ^ sw) << 4));
          const uint32_t ww[4] = {vw.x, vw.y, vw.z, vw.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float lo = bf16lo_to_f32(ww[e]), hi = bf16hi_to_f32(ww[e]);
#pragma unroll
            for (int h = 0; h < QPK; ++h) {
              acc[h][i * 8 + 2 * e] = fmaf(pr[h], lo, acc[h][i * 8 + 2 * e]);
              acc[h][i * 8 + 2 * e + 1] = fmaf(pr[h], hi, acc[h][i * 8 + 2 * e + 1]);
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[s]);
  }

  // Reduce the token lanes of the warp (all lanes of one token hold the same l).
#pragma unroll
  for (int h = 0; h < QPK; ++h) {
#pragma unroll
    for (int off = LPT; off < 32; off <<= 1) {
      l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], off);
#pragma unroll
      for (int k = 0; k < DPL; ++k) acc[h][k] += __shfl_xor_sync(0xffffffffu, acc[h][k], off);
    }
  }
  if (tok_in_pass == 0) {
#pragma unroll
    for (int h = 0; h < QPK; ++h) {
#pragma unroll
      for (int i = 0; i < NCH; ++i) {
        const int gc = j + LPT * i;
#pragma unroll
        for (int e = 0; e < 8; ++e) sm.red_o[warp][h][gc * 8 + e] = acc[h][i * 8 + e];
      }
    }
  }
  if (lane == 0) {
#pragma unroll
    for (int h = 0; h < QPK; ++h) {
      sm.red_m[warp][h] = m_run[h];
      sm.red_l[warp][h] = l_run[h];
    }
  }
  named_barrier_sync(1, kConsumerWarps * 32);

  // Merge the 4 warps: thread d owns output dim d of every head in the group.
  const int d = threadIdx.x;
  float o_cta[QPK], m_cta[QPK], l_cta[QPK];
#pragma unroll
  for (int h = 0; h < QPK; ++h) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, sm.red_m[w][h]);
    float o = 0.f, l = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float mw = sm.red_m[w][h];
        const float sc_w = (mw == -INFINITY) ? 0.f : fast_exp2(mw - M);
        o = fmaf(sc_w, sm.red_o[w][h][d], o);
        l = fmaf(sc_w, sm.red_l[w][h], l);
      }
    }
    o_cta[h] = o;
    m_cta[h] = M;
    l_cta[h] = l;
  }

  __nv_bfloat16* out = a.out + (static_cast<int64_t>(b) * a.num_heads + h0) * kD;
  if (nsplit == 1) {
#pragma unroll
    for (int h = 0; h < QPK; ++h) out[h * kD + d] = __float2bfloat16_rn(l_cta[h] > 0.f ? o_cta[h] / l_cta[h] : 0.f);
    return;
  }

  const int64_t pair = static_cast<int64_t>(b) * a.num_kv_heads + g;
  const int64_t part0 = pair * a.max_splits * QPK;
#pragma unroll
  for (int h = 0; h < QPK; ++h) {
    const int64_t idx = part0 + static_cast<int64_t>(split) * QPK + h;
    a.ws_o[idx * kD + d] = o_cta[h];
    if (d == 0) a.ws_ml[idx] = make_float2(m_cta[h], l_cta[h]);
  }
  __threadfence();
  named_barrier_sync(1, kConsumerWarps * 32);
  if (d == 0) sm.last = (atomicAdd(a.ws_cnt + pair, 1) == nsplit - 1);
  named_barrier_sync(1, kConsumerWarps * 32);
  if (!sm.last) return;
  __threadfence();

#pragma unroll
  for (int h = 0; h < QPK; ++h) {
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, __ldcg(&a.ws_ml[part0 + sp * QPK + h]).x);
    float o = 0.f, l = 0.f;
    if (M != -INFINITY) {
      for (int sp = 0; sp < nsplit; ++sp) {
        const float2 ml = __ldcg(&a.ws_ml[part0 + sp * QPK + h]);
        const float w = (ml.x == -INFINITY) ? 0.f : fast_exp2(ml.x - M);
        o = fmaf(w, __ldcg(&a.ws_o[(part0 + sp * QPK + h) * kD + d]), o);
        l = fmaf(w, ml.y, l);
      }
    }
    out[h * kD + d] = __float2bfloat16_rn(l > 0.f ? o / l : 0.f);
  }
  if (d == 0) a.ws_cnt[pair] = 0;
}

struct WsLayout {
  size_t cnt_off, ml_off, o_off, total;
};

WsLayout ws_layout(int batch, int num_heads, int num_kv_heads, int max_splits) {
  auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
  const int qpk = num_heads / num_kv_heads;
  const size_t pairs = static_cast<size_t>(batch) * num_kv_heads;
  const size_t parts = pairs * static_cast<size_t>(max_splits) * qpk;
  WsLayout w;
  w.cnt_off = 256;  // [0, 256): device error word
  w.ml_off = w.cnt_off + up(pairs * sizeof(int));
  w.o_off = w.ml_off + up(parts * sizeof(float2));
  w.total = w.o_off + up(parts * kD * sizeof(float));
  return w;
}

template <int QPK>
int launch(const CUtensorMap& km, const CUtensorMap& vm, const DecodeArgs& a, int batch, cudaStream_t stream) {
  const size_t smem = sizeof(Smem<QPK>) + 1024;
  int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(&paged_decode_kernel<QPK>), smem);
  if (rc != NVK_OK) return rc;
  const dim3 grid(a.max_splits, a.num_kv_heads, batch);
  paged_decode_kernel<QPK><<<grid, kThreads, smem, stream>>>(km, vm, a);
  return check_cuda(cudaGetLastError(), "paged_decode launch");
}

}  // namespace
}  // namespace nvk

extern "C" int nvk_paged_decode_workspace_size(int batch, int num_heads, int num_kv_heads, int head_dim,
                                               int max_splits, size_t* bytes) {
  using namespace nvk;
  if (!bytes) return fail(NVK_ERR_INVALID_ARGUMENT, "workspace_size: null output pointer");
  if (batch < 0 || num_heads <= 0 || num_kv_heads <= 0 || max_splits <= 0 || num_heads % num_kv_heads != 0)
    return fail(NVK_ERR_INVALID_ARGUMENT, "workspace_size: bad sizes (batch=%d heads=%d kv_heads=%d splits=%d)",
                batch, num_heads, num_kv_heads, max_splits);
  if (head_dim != kD) return fail(NVK_ERR_UNSUPPORTED, "workspace_size: head_dim %d unsupported (128 only)", head_dim);
  *bytes = ws_layout(batch, num_heads, num_kv_heads, max_splits).total;
  return NVK_OK;
}

extern "C" int nvk_paged_decode(void* out, const void* query, const void* key_cache, const void* value_cache,
                                int num_blocks, int block_size, const int32_t* block_tables, int block_table_stride,
                                int max_blocks_per_seq, const int32_t* context_lens, int batch, int num_heads,
                                int num_kv_heads, int head_dim, float scale, int blocks_per_split, int max_splits,
                                void* workspace, size_t workspace_bytes, nvk_stream_t stream) {
  using namespace nvk;
  if (batch < 0 || num_blocks <= 0 || num_heads <= 0 || num_kv_heads <= 0)
    return fail(NVK_ERR_INVALID_ARGUMENT, "paged_decode: bad sizes (batch=%d blocks=%d heads=%d kv_heads=%d)", batch,
                num_blocks, num_heads, num_kv_heads);
  if (batch == 0) return NVK_OK;
  if (head_dim != kD) return fail(NVK_ERR_UNSUPPORTED, "paged_decode: head_dim %d unsupported (128 only)", head_dim);
  if (num_heads % num_kv_heads != 0)
    return fail(NVK_ERR_INVALID_ARGUMENT, "paged_decode: num_heads %d not a multiple of num_kv_heads %d", num_heads,
                num_kv_heads);
  const int qpk = num_heads / num_kv_heads;
  if (qpk != 1 && qpk != 2 && qpk != 4 && qpk != 8)
    return fail(NVK_ERR_UNSUPPORTED, "paged_decode: GQA ratio %d unsupported (1, 2, 4, 8)", qpk);
  if (block_size < 16 || block_size > 256 || (block_size & (block_size - 1)) != 0)
    return fail(NVK_ERR_UNSUPPORTED, "paged_decode: block_size %d unsupported (power of two in [16, 256])",
                block_size);
  if (blocks_per_split <= 0 || blocks_per_split > kMaxSplitBlocks)
    return fail(NVK_ERR_INVALID_ARGUMENT, "paged_decode: blocks_per_split %d outside [1, %d]", blocks_per_split,
                kMaxSplitBlocks);
  if (max_blocks_per_seq <= 0 || block_table_stride < max_blocks_per_seq)
    return fail(NVK_ERR_INVALID_ARGUMENT, "paged_decode: block table width %d / stride %d invalid",
                max_blocks_per_seq, block_table_stride);
  if (max_splits < (max_blocks_per_seq + blocks_per_split - 1) / blocks_per_split || max_splits > 65535)
    return fail(NVK_ERR_INVALID_ARGUMENT, "paged_decode: max_splits %d < ceil(%d / %d)", max_splits,
                max_blocks_per_seq, blocks_per_split);
  if (batch > 65535 || num_kv_heads > 65535)
    return fail(NVK_ERR_UNSUPPORTED, "paged_decode: batch %d or kv heads %d above grid limit", batch, num_kv_heads);
  if (!out || !query || !key_cache || !value_cache || !block_tables || !context_lens)
    return fail(NVK_ERR_INVALID_ARGUMENT, "paged_decode: null pointer");
  if (!aligned16(out) || !aligned16(query))
    return fail(NVK_ERR_INVALID_ARGUMENT, "paged_decode: q/out must be 16-byte aligned");
  const WsLayout wl = ws_layout(batch, num_heads, num_kv_heads, max_splits);
  if (!workspace || workspace_bytes < wl.total || !aligned16(workspace))
    return fail(NVK_ERR_WORKSPACE, "paged_decode: workspace %zu bytes < %zu needed (or misaligned)", workspace_bytes,
                wl.total);

  const int64_t rows = static_cast<int64_t>(num_blocks) * block_size;
  const int sub_rows = block_size < 32 ? block_size : 32;
  CUtensorMap km, vm;
  int rc = kv_tensor_map(&km, key_cache, rows, num_kv_heads, sub_rows);
  if (rc != NVK_OK) return rc;
  rc = kv_tensor_map(&vm, value_cache, rows, num_kv_heads, sub_rows);
  if (rc != NVK_OK) return rc;

  uint8_t* ws = static_cast<uint8_t*>(workspace);
  DecodeArgs a;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.q = static_cast<const __nv_bfloat16*>(query);
  a.block_tables = block_tables;
  a.context_lens = context_lens;
  a.err = reinterpret_cast<int*>(ws);
  a.ws_cnt = reinterpret_cast<int*>(ws + wl.cnt_off);
  a.ws_ml = reinterpret_cast<float2*>(ws + wl.ml_off);
  a.ws_o = reinterpret_cast<float*>(ws + wl.o_off);
  a.bt_stride = block_table_stride;
  a.max_blocks = max_blocks_per_seq;
  a.num_blocks = num_blocks;
  a.block_size = block_size;
  a.log2_bs = __builtin_ctz(static_cast<unsigned>(block_size));
  a.sub_rows = sub_rows;
  a.num_heads = num_heads;
  a.num_kv_heads = num_kv_heads;
  a.blocks_per_split = blocks_per_split;
  a.max_splits = max_splits;
  a.scale_log2 = scale * 1.4426950408889634f;

  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (qpk) {
    case 1: return launch<1>(km, vm, a, batch, st);
    case 2: return launch<2>(km, vm, a, batch, st);
    case 4: return launch<4>(km, vm, a, batch, st);
    default: return launch<8>(km, vm, a, batch, st);
  }
}

// ---------------------------------------------------------------------------
// Allocation-free decode entry point.
//
// Some callers cannot allocate device memory where they run attention: a
// plugin's enqueue callback inside a host framework that owns every device
// buffer and forbids allocating there, a binding from a language with no
// device allocator of its own (cgo, JNI, N-API), or a latency-critical serving
// thread that must not take cudaMalloc's implicit device synchronisation. For
// them the split-K scratch lives in a fixed array in this library's device
// memory instead of a caller-provided workspace. The array costs
// kNoAllocScratchBytes on every GPU that loads the library, until the process
// exits.
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // 16 MiB per device
constexpr int kNoAllocMaxDevices = 64;

}  // namespace

static __device__ __align__(256) uint8_t g_noalloc_decode_scratch[kNoAllocScratchBytes];

namespace {

// Device address of the scratch array on the current device. The symbol's
// host-side name is only a handle: the address is fetched with
// cudaGetSymbolAddress once per device (with that device current) and cached.
int noalloc_scratch(void** out) {
  static std::mutex mu;
  static void* addr[kNoAllocMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return nvk::check_cuda(e, "paged_decode_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return nvk::fail(NVK_ERR_UNSUPPORTED, "paged_decode_noalloc: device %d above %d", dev, kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_decode_scratch);
    if (e != cudaSuccess) return nvk::check_cuda(e, "paged_decode_noalloc: cudaGetSymbolAddress");
    addr[dev] = p;
  }
  *out = addr[dev];
  return NVK_OK;
}

}  // namespace

extern "C" int nvk_paged_decode_noalloc(void* out, const void* query, const void* key_cache,
                                        const void* value_cache, int num_blocks, int block_size,
                                        const int32_t* block_tables, int block_table_stride, int max_blocks_per_seq,
                                        const int32_t* context_lens, int batch, int num_heads, int num_kv_heads,
                                        int head_dim, float scale, int blocks_per_split, int max_splits,
                                        nvk_stream_t stream) {
  using namespace nvk;
  size_t need = 0;
  size_t header = 0;
  const bool sane = batch > 0 && num_heads > 0 && num_kv_heads > 0 && num_heads % num_kv_heads == 0 &&
                    max_splits > 0 && head_dim == kD;
  if (sane) {
    const WsLayout wl = ws_layout(batch, num_heads, num_kv_heads, max_splits);
    need = wl.total;
    header = wl.ml_off;  // error word + arrival counters
    if (need > kNoAllocScratchBytes)
      return fail(NVK_ERR_UNSUPPORTED,
                  "paged_decode_noalloc: %zu bytes of split-K scratch needed, the static scratch holds %zu "
                  "(fewer splits, a smaller batch, or nvk_paged_decode with a caller workspace)",
                  need, kNoAllocScratchBytes);
  }
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc != NVK_OK) return rc;
  if (sane) {
    // The array keeps the previous call's contents: clear the error word and
    // the arrival counters, which must start at zero.
    rc = check_cuda(cudaMemsetAsync(scratch, 0, header, reinterpret_cast<cudaStream_t>(stream)),
                    "paged_decode_noalloc: clear scratch header");
    if (rc != NVK_OK) return rc;
  }
  return nvk_paged_decode(out, query, key_cache, value_cache, num_blocks, block_size, block_tables,
                          block_table_stride, max_blocks_per_seq, context_lens, batch, num_heads, num_kv_heads,
                          head_dim, scale, blocks_per_split, max_splits, scratch, kNoAllocScratchBytes, stream);
}
