// LM head + greedy argmax on the device, one launch for the whole batch.
//
// Replaces, for greedy sampling, Qwen3ForCausalLM's lm_head
// (src/nanovllm_ascend/models/qwen3.py:196,221: bf16 logits = hidden . W^T)
// followed by Sampler.sample's torch.argmax (layers/sampler.py:13-14) and the
// per-sequence .item() of ModelRunner.decode (model_runner.py:284-286): the
// kernel writes the next token id of every row into device memory, which the
// host reads with one copy.
//
// A skinny GEMM, HBM-bound on the weight (vocab x hidden bf16, read once):
//  * persistent grid, CTA c takes a contiguous range of 128-row vocab tiles;
//  * warp 4 (producer): per tile and 64-wide hidden chunk, TMA loads of the
//    weight chunk [128 x 64] and the hidden chunk [N x 64] (rows >= batch are
//    zero-filled) into a kStages ring, 128-byte swizzle;
//  * warp 5 (MMA): logits^T[128 vocab x N batch] += W_chunk . H_chunk^T, four
//    M=128 K=16 UMMAs per chunk, f32 accumulators in TMEM (two tile buffers);
//  * warps 0-3 (epilogue): thread r owns vocab row r of the tile; each logit
//    is rounded to bf16 (the reference's logits dtype), then per batch row a
//    warp/CTA (max, first index) reduction; the CTA's best of every batch
//    row goes to a packed 64-bit atomicMax (ordered value, complemented
//    index: ties pick the smallest index, as torch.argmax does); the CTA that
//    finishes last turns the packed words into int64 token ids and resets
//    them. Every mbarrier wait is bounded.
#include "host_common.h"
#include "nvk_common.cuh"
#include "tcgen05.cuh"

namespace nvk {
namespace {

constexpr int kTileRows = 128;  // vocab rows per tile (UMMA M)
constexpr int kChunk = 64;      // hidden elements per chunk (one 128-byte swizzle atom)
constexpr int kStages = 6;
constexpr int kMaxN = 128;      // padded batch (UMMA N)
constexpr int kWChunkBytes = kTileRows * kChunk * 2;  // 16 KB
constexpr int kHChunkBytes = kMaxN * kChunk * 2;      // 16 KB at the largest batch
constexpr int kThreads = 6 * 32;
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr uint32_t kTmemCols = 2 * kMaxN;

struct HeadArgs {
  unsigned long long* best;  // [batch] packed (ordered logit, ~index)
  int* done;                 // CTAs finished this call
  int64_t* token_ids;        // [batch]
  int* err;
  int vocab, hidden, batch, n_pad, tiles;
};

struct HeadSmem {
  alignas(1024) uint8_t w[kStages][kWChunkBytes];
  alignas(1024) uint8_t h[kStages][kHChunkBytes];
  uint64_t full[kStages], empty[kStages];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t fin;
  float red_v[4][kMaxN];
  int red_i[4][kMaxN];
  uint32_t tmem_base;
};

static_assert(sizeof(HeadSmem) + 1024 <= 232448, "lm_head_argmax shared memory exceeds the 227 KB per-CTA limit");

__device__ __forceinline__ uint32_t ordered_bits(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(kThreads, 1) lm_head_argmax_kernel(const __grid_constant__ CUtensorMap wmap,
                                                                     const __grid_constant__ CUtensorMap hmap,
                                                                     const HeadArgs a) {
  extern __shared__ uint8_t smem_raw[];
  HeadSmem& sm = *reinterpret_cast<HeadSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, ctas = gridDim.x;
  const int t_lo = static_cast<int>(static_cast<int64_t>(a.tiles) * c / ctas);
  const int t_hi = static_cast<int>(static_cast<int64_t>(a.tiles) * (c + 1) / ctas);
  const int nchunks = a.hidden / kChunk;
  const int64_t total = static_cast<int64_t>(t_hi - t_lo) * nchunks;
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.acc_full[i], 1);
      mbar_init(&sm.acc_empty[i], 128);
    }
    mbar_init(&sm.fin, 1);
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();
  const uint32_t tmem = sm.tmem_base;

  if (warp == kProducerWarp) {
    if (lane == 0) {
      tma_prefetch_desc(&wmap);
      tma_prefetch_desc(&hmap);
      const uint32_t hbytes = static_cast<uint32_t>(a.n_pad) * kChunk * 2;
      int64_t q = 0;
      bool ok = true;
      for (; ok && q < total; ++q) {
        const int st = static_cast<int>(q % kStages);
        if (q >= kStages && !mbar_wait(&sm.empty[st], static_cast<uint32_t>((q / kStages) - 1) & 1)) {
          ok = false;
          break;
        }
        const int tile = t_lo + static_cast<int>(q / nchunks);
        const int k = static_cast<int>(q % nchunks);
        mbar_arrive_expect_tx(&sm.full[st], kWChunkBytes + hbytes);
        // W viewed as [vocab, hidden/128, 128]: chunk k is half (k & 1) of column block k / 2
        tma_load_3d(sm.w[st], &wmap, &sm.full[st], (k & 1) * 64, k >> 1, tile * kTileRows);
        tma_load_3d(sm.h[st], &hmap, &sm.full[st], (k & 1) * 64, k >> 1, 0);
      }
      if (!ok) atomicOr(a.err, kErrWaitTimeout);
      for (int64_t j = q > kStages ? q - kStages : 0; j < q; ++j)
        (void)mbar_wait(&sm.full[j % kStages], static_cast<uint32_t>(j / kStages) & 1);
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(kTileRows, a.n_pad, false);
      bool ok = true;
      int64_t q = 0;
      for (int t = 0; ok && t < t_hi - t_lo; ++t) {
        const int ab = t & 1;
        if (t >= 2 && !mbar_wait(&sm.acc_empty[ab], ((t >> 1) - 1) & 1)) {
          ok = false;
          break;
        }
        for (int k = 0; k < nchunks; ++k, ++q) {
          const int st = static_cast<int>(q % kStages);
          if (!mbar_wait(&sm.full[st], static_cast<uint32_t>(q / kStages) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t wa = smem_u32(sm.w[st]), ha = smem_u32(sm.h[st]);
#pragma unroll
          for (int kk = 0; kk < kChunk / 16; ++kk)
            umma_f16_ss(tmem + ab * kMaxN, smem_desc_sw128(wa + kk * 32, 16, 1024), smem_desc_sw128(ha + kk * 32, 16, 1024),
                        idesc, (k > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&sm.empty[st]);
        }
        if (ok) umma_commit(&sm.acc_full[ab]);
      }
      if (!ok) atomicOr(a.err, kErrWaitTimeout);
      umma_commit(&sm.fin);
      (void)mbar_wait(&sm.fin, 0);
    }
  } else {
    // ----------------------------------------------------------- epilogue ----
    const int r = tid;  // vocab row within the tile = TMEM lane
    const uint32_t t_lane = static_cast<uint32_t>(warp * 32) << 16;
    float best_v = -INFINITY;  // thread b < batch keeps batch row b's best so far
    int best_i = 0x7fffffff;
    bool ok = true;
    for (int t = 0; t < t_hi - t_lo; ++t) {
      const int ab = t & 1;
      if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&sm.acc_full[ab], (t >> 1) & 1));
      const int row = (t_lo + t) * kTileRows + r;
      for (int n0 = 0; n0 < a.n_pad; n0 += 32) {
        uint32_t v[32];
        if (ok) {
          tc_fence_after();
          tmem_ld32(tmem + ab * kMaxN + n0 + t_lane, v);
          tmem_ld_wait();
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          // the reference's logits are bf16: round first, then compare
          float x = (ok && row < a.vocab) ? __bfloat162float(__float2bfloat16_rn(__uint_as_float(v[e]))) : -INFINITY;
          int xi = row;
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) {
            const float y = __shfl_xor_sync(0xffffffffu, x, off);
            const int yi = __shfl_xor_sync(0xffffffffu, xi, off);
            if (y > x || (y == x && yi < xi)) {
              x = y;
              xi = yi;
            }
          }
          if (lane == 0) {
            sm.red_v[warp][n0 + e] = x;
            sm.red_i[warp][n0 + e] = xi;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&sm.acc_empty[ab]);  // the accumulator buffer may take tile t + 2
      named_barrier_sync(1, 128);
      if (r < a.batch) {
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const float y = sm.red_v[w][r];
          const int yi = sm.red_i[w][r];
          if (y > best_v || (y == best_v && yi < best_i)) {
            best_v = y;
            best_i = yi;
          }
        }
      }
      named_barrier_sync(1, 128);  // red[] is rewritten by the next tile
    }
    if (!ok && r == 0) atomicOr(a.err, kErrWaitTimeout);
    if (r < a.batch && best_i != 0x7fffffff) {
      const unsigned long long key = (static_cast<unsigned long long>(ordered_bits(best_v)) << 32) |
                                     (0xffffffffull - static_cast<unsigned long long>(best_i));
      atomicMax(a.best + r, key);
    }
    // The last CTA to finish decodes the winners and resets the words.
    named_barrier_sync(1, 128);
    if (r == 0) {
      __threadfence();
      const int old = atomicAdd(a.done, 1);
      sm.red_i[0][0] = (old == ctas - 1);
    }
    named_barrier_sync(1, 128);
    if (sm.red_i[0][0]) {
      __threadfence();
      for (int b = r; b < a.batch; b += 128) {
        const unsigned long long key = atomicExch(a.best + b, 0ull);
        a.token_ids[b] = static_cast<int64_t>(0xffffffffull - (key & 0xffffffffull));
      }
      if (r == 0) *a.done = 0;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) {
    __syncwarp();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace
}  // namespace nvk

extern "C" int nvk_lm_head_argmax_workspace_size(int batch, size_t* bytes) {
  if (!bytes || batch < 0) return nvk::fail(NVK_ERR_INVALID_ARGUMENT, "lm_head_argmax_workspace_size: bad arguments");
  *bytes = 256 + static_cast<size_t>(batch) * 8;
  return NVK_OK;
}

extern "C" int nvk_lm_head_argmax(const void* hidden, int64_t hidden_stride, const void* weight, int vocab_size,
                                  int hidden_size, int batch, int64_t* token_ids, void* workspace,
                                  size_t workspace_bytes, int num_ctas, int* error_word, nvk_stream_t stream) {
  using namespace nvk;
  if (batch < 0 || vocab_size <= 0 || hidden_size <= 0 || num_ctas < 0)
    return fail(NVK_ERR_INVALID_ARGUMENT, "lm_head_argmax: bad sizes (batch=%d vocab=%d hidden=%d)", batch, vocab_size,
                hidden_size);
  if (batch == 0) return NVK_OK;
  if (batch > kMaxN) return fail(NVK_ERR_UNSUPPORTED, "lm_head_argmax: batch %d above %d", batch, kMaxN);
  if (hidden_size % 128 != 0)
    return fail(NVK_ERR_UNSUPPORTED, "lm_head_argmax: hidden size %d not a multiple of 128", hidden_size);
  if (!hidden || !weight || !token_ids || !workspace || !error_word)
    return fail(NVK_ERR_INVALID_ARGUMENT, "lm_head_argmax: null pointer");
  if (workspace_bytes < 256 + static_cast<size_t>(batch) * 8 || !aligned16(workspace) || !aligned16(hidden) ||
      !aligned16(weight) || (hidden_stride * 2) % 16 != 0 || hidden_stride < hidden_size)
    return fail(NVK_ERR_INVALID_ARGUMENT, "lm_head_argmax: workspace too small or misaligned rows");
  int ctas = num_ctas;
  if (ctas == 0) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&ctas, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return check_cuda(e, "lm_head_argmax: SM count");
  }
  const int tiles = (vocab_size + kTileRows - 1) / kTileRows;
  if (ctas > tiles) ctas = tiles;
  const int n_pad = batch <= 16 ? 16 : (batch <= 32 ? 32 : (batch <= 64 ? 64 : 128));
  CUtensorMap wm, hm;
  int rc;
  // W as [vocab, hidden/128, 128] (box 64 x 1 x 128 rows); H as [batch, hidden/128, 128] (box 64 x 1 x n_pad rows)
  if ((rc = kv_tensor_map(&wm, weight, vocab_size, hidden_size / 128, kTileRows)) != NVK_OK) return rc;
  if ((rc = kv_tensor_map(&hm, hidden, batch, hidden_size / 128, n_pad, hidden_stride)) != NVK_OK) return rc;
  const size_t smem = sizeof(HeadSmem) + 1024;
  rc = ensure_dynamic_smem(reinterpret_cast<const void*>(&lm_head_argmax_kernel), smem);
  if (rc != NVK_OK) return rc;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  HeadArgs a;
  a.done = reinterpret_cast<int*>(ws);
  a.best = reinterpret_cast<unsigned long long*>(ws + 256);
  a.token_ids = token_ids;
  a.err = error_word;
  a.vocab = vocab_size;
  a.hidden = hidden_size;
  a.batch = batch;
  a.n_pad = n_pad;
  a.tiles = tiles;
  return check_cuda(launch_pdl(lm_head_argmax_kernel, dim3(ctas), dim3(kThreads), smem,
                               reinterpret_cast<cudaStream_t>(stream), wm, hm, a),
                    "lm_head_argmax launch");
}
