// Causal prefill attention on the sm_100a tensor cores (tcgen05 + TMEM).
//
// Replaces torch_npu.npu_fused_infer_attention_score as called from
// src/nanovllm_ascend/layers/npu_prefill_attention.py:82-112 (TND layout,
// sparse_mode=3): paged mode reads the whole KV of a sequence (cached prefix
// + rows appended this step) through its block table with absolute kv
// lengths; dense mode reads contiguous K/V rows delimited by cumulative
// lengths. Masking is bottom-right aligned: query i of a sequence with Lq
// queries and Lk keys sees key j iff j <= Lk - Lq + i.
//
// One CTA = 128 query rows of one sequence x one query head; two CTAs share
// an SM (96 KB of shared memory and 256 TMEM columns each), so that one
// CTA's softmax runs while the other's MMAs do.
//   warp 4 (producer): TMA loads of the Q tile once, then 64-key K and V
//     tiles (half a pool block each, 128-byte swizzle = the canonical UMMA
//     operand layout): K into a 2-stage ring freed as soon as S has read it,
//     V into a 2-stage ring freed by PV; K runs two tiles ahead of V, and
//     the block ids come 32 at a time (one parallel load per warp).
//   warp 5 (MMA): allocates 256 TMEM columns (S/P double buffered: 0-63,
//     64-127; O: 128-255) and one lane issues S = Q K^T (8 x M128 N64 K16,
//     both K-major) one key tile ahead of O += P V (4 x M128 N128 K16, P read
//     from TMEM where the softmax wrote it over S(j), V MN-major from smem),
//     so the tensor core computes S(j+1) while the softmax warps work on
//     tile j; S(j+2) reuses the columns of P(j) and so waits for P V(j);
//     tcgen05.commit signals the mbarriers.
//   warps 0-3 (softmax): thread r owns query row r = TMEM lane r: loads its
//     S row in two halves (tcgen05.ld), masks, base-2 online softmax with
//     lazy rescaling of O in TMEM (only when the running max grows by more
//     than 2^8), packed f32x2 exponent arguments and row sums, writes P as
//     bf16 pairs into the first 32 columns of its S buffer (tcgen05.st),
//     and at the end normalises its O row and stores it.
// Every mbarrier wait is bounded; on a timeout the CTA records the error,
// drains its in-flight copies and MMAs, frees TMEM and exits.
#include "host_common.h"
#include "nvk_common.cuh"
#include "tcgen05.cuh"

namespace nvk {
namespace {

constexpr int kD = 128;
constexpr int kRows = 128;                   // query rows per CTA
constexpr int kKeys = 64;                    // keys per K/V tile (half a 128-token pool block)
constexpr int kQHalfBytes = kRows * 128;     // one 64-dim half of the Q tile
constexpr int kQTileBytes = 2 * kQHalfBytes;
constexpr int kKVHalfBytes = kKeys * 128;    // one 64-dim half of a K or V tile
constexpr int kKVTileBytes = 2 * kKVHalfBytes;
constexpr int kKStages = 2;
constexpr int kVStages = 2;
constexpr int kSoftmaxThreads = 128;
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr int kThreads = 6 * 32;
constexpr int kSBufs = 2;            // S/P buffers in TMEM
constexpr uint32_t kTmemCols = 256;  // S0, S1 (64 columns each), O (128): two CTAs share an SM's 512
constexpr int kCtasPerSm = 2;        // two softmax warpgroups per SM hide each other's latency
constexpr float kRescaleThreshold = 8.0f;

struct PrefillArgs {
  __nv_bfloat16* out;
  const int32_t* block_tables;
  const int32_t* cu_q;
  const int32_t* kv_lens;  // paged: absolute kv length per sequence
  const int32_t* cu_kv;    // dense: cumulative kv rows
  int* err;
  int bt_stride;
  int num_blocks;
  int num_heads;
  int qpk;
  int paged;
  float scale_log2;
};

struct PrefillSmem {
  alignas(1024) uint8_t q[kQTileBytes];
  alignas(1024) uint8_t k[kKStages][kKVTileBytes];
  alignas(1024) uint8_t v[kVStages][kKVTileBytes];
  uint64_t bar_q;
  uint64_t full_k[kKStages], k_empty[kKStages];
  uint64_t full_v[kVStages], v_empty[kVStages];
  uint64_t s_full[kSBufs];
  uint64_t p_full[kSBufs];   // P(j) written into S buffer j % 2
  uint64_t pv_done[kSBufs];  // PV(j) complete (S buffer j % 2 free again)
  uint64_t fin;
  uint32_t tmem_base;
  volatile int abort;
};

static_assert(kCtasPerSm * (sizeof(PrefillSmem) + 1024 + 1024) <= 233472,
              "prefill shared memory does not let two CTAs share an SM");

__device__ __forceinline__ void flag_error(const PrefillArgs& a, PrefillSmem& sm, int code) {
  if (a.err) atomicOr(a.err, code);
  sm.abort = 1;
}

__global__ void __launch_bounds__(kThreads, kCtasPerSm) prefill_kernel(const __grid_constant__ CUtensorMap qmap,
                                                              const __grid_constant__ CUtensorMap kmap,
                                                              const __grid_constant__ CUtensorMap vmap,
                                                              const PrefillArgs a) {
  const int qt = gridDim.x - 1 - blockIdx.x;  // heaviest (last) query tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  pdl_launch_dependents();
  pdl_wait();
  const int q0 = a.cu_q[b];
  const int lq = a.cu_q[b + 1] - q0;
  if (qt * kRows >= lq) return;
  const int lk = a.paged ? a.kv_lens[b] : (a.cu_kv[b + 1] - a.cu_kv[b]);
  const int kv_row0 = a.paged ? 0 : a.cu_kv[b];
  const int g = h / a.qpk;
  const int i_last = min(qt * kRows + kRows - 1, lq - 1);
  const int lim_last = min(lk - lq + i_last, lk - 1);
  const int n_kv = lim_last < 0 ? 0 : lim_last / kKeys + 1;  // 64-key tiles

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  __nv_bfloat16* out_row = nullptr;
  const int i = qt * kRows + tid;  // query row within the sequence (softmax threads)
  if (tid < kSoftmaxThreads && i < lq) out_row = a.out + (static_cast<int64_t>(q0 + i) * a.num_heads + h) * kD;

  if (n_kv == 0) {  // no visible key for any row of this tile: zeros
    if (out_row) {
      for (int c = 0; c < kD; c += 8) *reinterpret_cast<uint4*>(out_row + c) = make_uint4(0, 0, 0, 0);
    }
    return;
  }

  extern __shared__ uint8_t smem_raw[];
  PrefillSmem& sm =
      *reinterpret_cast<PrefillSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  if (tid == 0) {
    mbar_init(&sm.bar_q, 1);
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&sm.full_k[s], 1);
      mbar_init(&sm.k_empty[s], 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&sm.full_v[s], 1);
      mbar_init(&sm.v_empty[s], 1);
    }
    for (int i = 0; i < kSBufs; ++i) {
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.p_full[i], kSoftmaxThreads);
      mbar_init(&sm.pv_done[i], 1);
    }
    mbar_init(&sm.fin, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t tmem_s = tmem;            // S(j), then P(j), in columns (j % 2) * 64
  const uint32_t tmem_o = tmem + kSBufs * kKeys;

  if (warp == kProducerWarp) {
    // -------------------------------------------------------- producer ----
    // The whole warp walks the tiles (block ids come 32 at a time, one per
    // lane); lane 0 waits for ring slots and issues the copies.
    if (lane == 0) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      mbar_arrive_expect_tx(&sm.bar_q, kQTileBytes);
      tma_load_3d(sm.q, &qmap, &sm.bar_q, 0, h, q0 + qt * kRows);
      tma_load_3d(sm.q + kQHalfBytes, &qmap, &sm.bar_q, 64, h, q0 + qt * kRows);
    }
    const int32_t* bt = a.block_tables + static_cast<int64_t>(b) * a.bt_stride;
    // First pool row of 64-key tile j (tile j is half j & 1 of block j / 2);
    // `chunk` holds this lane's block id for tile j & ~31 + lane and is
    // refreshed when j crosses a multiple of 32 (each caller passes its own
    // register and consecutive j).
    auto row_of = [&](int j, int& chunk) -> int {
      if ((j & 31) == 0) {
        const int jj = j + lane;
        int blk = 0;
        if (a.paged && jj < n_kv) {
          blk = bt[jj >> 1];
          if (blk < 0 || blk >= a.num_blocks) {
            if (a.err) atomicOr(a.err, kErrBadBlockId);
            blk = a.num_blocks;  // fully outside the tensor map: zero fill
          }
        }
        chunk = blk;
      }
      const int blk = __shfl_sync(0xffffffffu, chunk, j & 31);
      return a.paged ? blk * kRows + (j & 1) * kKeys : kv_row0 + j * kKeys;
    };
    int k_chunk = 0, v_chunk = 0, k_issued = 0, v_issued = 0;
    bool ok = true;
    auto load_k = [&](int j) {
      const int row = row_of(j, k_chunk);
      const int st = j % kKStages;
      if (lane == 0) {
        if (j >= kKStages && !mbar_wait(&sm.k_empty[st], ((j / kKStages) - 1) & 1)) {
          ok = false;
        } else {
          mbar_arrive_expect_tx(&sm.full_k[st], kKVTileBytes);
          tma_load_3d(sm.k[st], &kmap, &sm.full_k[st], 0, g, row);
          tma_load_3d(sm.k[st] + kKVHalfBytes, &kmap, &sm.full_k[st], 64, g, row);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      k_issued += ok ? 1 : 0;
    };
    auto load_v = [&](int j) {
      const int row = row_of(j, v_chunk);
      const int st = j % kVStages;
      if (lane == 0) {
        if (j >= kVStages && !mbar_wait(&sm.v_empty[st], ((j / kVStages) - 1) & 1)) {
          ok = false;
        } else {
          mbar_arrive_expect_tx(&sm.full_v[st], kKVTileBytes);
          tma_load_3d(sm.v[st], &vmap, &sm.full_v[st], 0, g, row);
          tma_load_3d(sm.v[st] + kKVHalfBytes, &vmap, &sm.full_v[st], 64, g, row);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      v_issued += ok ? 1 : 0;
    };
    for (int j = 0; ok && j < 2 && j < n_kv; ++j) load_k(j);
    for (int t = 0; ok && t < n_kv && !sm.abort; ++t) {
      if (t + 2 < n_kv) load_k(t + 2);
      if (ok) load_v(t);
    }
    if (lane == 0) {
      if (!ok) flag_error(a, sm, kErrWaitTimeout);
      // Drain every copy this CTA issued before it may exit.
      (void)mbar_wait(&sm.bar_q, 0);
      for (int j = max(0, k_issued - kKStages); j < k_issued; ++j)
        (void)mbar_wait(&sm.full_k[j % kKStages], (j / kKStages) & 1);
      for (int j = max(0, v_issued - kVStages); j < v_issued; ++j)
        (void)mbar_wait(&sm.full_v[j % kVStages], (j / kVStages) & 1);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------- MMA ----
    if (lane == 0) {
      constexpr uint32_t idesc_qk = umma_idesc_bf16(kRows, kKeys, false);
      constexpr uint32_t idesc_pv = umma_idesc_bf16(kRows, kD, true);
      const uint32_t q_addr = smem_u32(sm.q);
      bool ok = mbar_wait(&sm.bar_q, 0);
      if (!ok) flag_error(a, sm, kErrWaitTimeout);
      // S(j) = Q K(j)^T into S buffer j % 2, once K(j) has landed and PV(j-2)
      // has read P(j-2) out of that buffer.
      auto issue_s = [&](int j) -> bool {
        const int s = j % kSBufs, ks = j % kKStages;
        if (!mbar_wait(&sm.full_k[ks], (j / kKStages) & 1)) return false;
        if (j >= kSBufs && !mbar_wait(&sm.pv_done[s], ((j / kSBufs) - 1) & 1)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sm.k[ks]);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t qoff = (kk >> 2) * kQHalfBytes + (kk & 3) * 32;
          const uint32_t koff = (kk >> 2) * kKVHalfBytes + (kk & 3) * 32;
          umma_f16_ss(tmem_s + s * kKeys, smem_desc_sw128(q_addr + qoff, 16, 1024),
                      smem_desc_sw128(k_addr + koff, 16, 1024), idesc_qk, kk > 0);
        }
        umma_commit(&sm.s_full[s]);
        umma_commit(&sm.k_empty[ks]);  // K(j) slot free once S(j) has read it
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < n_kv; ++j) {
        const int s = j % kSBufs;
        if (j + 1 < n_kv && !issue_s(j + 1)) { ok = false; break; }
        if (!mbar_wait(&sm.p_full[s], (j / kSBufs) & 1)) { ok = false; break; }
        const int vs = j % kVStages;
        if (!mbar_wait(&sm.full_v[vs], (j / kVStages) & 1)) { ok = false; break; }
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sm.v[vs]);
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk) {
          const uint64_t vb = smem_desc_sw128(v_addr + kk * 16 * 128, kKVHalfBytes, 1024);
          umma_f16_ts(tmem_o, tmem_s + s * kKeys + kk * 8, vb, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&sm.v_empty[vs]);
        umma_commit(&sm.pv_done[s]);
      }
      if (!ok) flag_error(a, sm, kErrWaitTimeout);
      // All MMAs of this CTA complete before TMEM is released.
      umma_commit(&sm.fin);
      (void)mbar_wait(&sm.fin, 0);
    }
  } else {
    // --------------------------------------------------------- softmax ----
    const int lim = (i < lq) ? (lk - lq + i) : (lk - 1);
    const uint32_t t_lane = static_cast<uint32_t>(warp * 32) << 16;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      // warp-uniform outcome: the tcgen05.ld/st below need a converged warp
      const int sb = j % kSBufs;
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.s_full[sb], (j / kSBufs) & 1))) { ok = false; break; }
      tc_fence_after();
      // S row in two 32-column halves: the second half loads while the
      // first half's maximum is taken.
      uint32_t sr[2][32];
      tmem_ld32(tmem_s + sb * kKeys + t_lane, sr[0]);
      tmem_ld_wait();
      tmem_ld32(tmem_s + sb * kKeys + t_lane + 32, sr[1]);
      const int kbase = j * kKeys;
      const bool need_mask = kbase + kKeys - 1 > lim;
      // The max is taken over raw scores (scale > 0), the scale folded into
      // the exponent's FMA below; max is exact, so its order is free.
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        if (c == 1) tmem_ld_wait();
        if (need_mask) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (kbase + c * 32 + e > lim) sr[c][e] = __float_as_uint(-INFINITY);
        }
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          mx0 = fmax3(mx0, __uint_as_float(sr[c][e]), __uint_as_float(sr[c][e + 1]));
          mx1 = fmax3(mx1, __uint_as_float(sr[c][e + 2]), __uint_as_float(sr[c][e + 3]));
        }
      }
      const float mraw = fmaxf(mx0, mx1);
      const float mt = mraw * a.scale_log2;
      const float m_new = fmaxf(m, mt);
      const bool resc = m_new > m + kRescaleThreshold;
      const float alpha = resc ? fast_exp2(m - m_new) : 1.f;
      // O rows change only when one of this warp's rows rescales; then
      // PV(j-1) must be complete first.
      if (j > 0 && __any_sync(0xffffffffu, resc)) {
        if (!__all_sync(0xffffffffu, mbar_wait(&sm.pv_done[(j - 1) % kSBufs], ((j - 1) / kSBufs) & 1))) { ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld32(tmem_o + t_lane + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st32(tmem_o + t_lane + c * 32, o);
        }
        tmem_st_wait();
      }
      if (resc) {
        l *= alpha;
        m = m_new;
      }
      const float neg_mu = (m == -INFINITY) ? 0.f : -m;
      const uint64_t sc2 = f32x2_pack(a.scale_log2, a.scale_log2);
      const uint64_t nm2 = f32x2_pack(neg_mu, neg_mu);
      uint64_t sum2[2] = {f32x2_pack(0.f, 0.f), f32x2_pack(0.f, 0.f)};  // two add chains
      // P over the first 32 columns of the S buffer (S is in registers now):
      // column k holds keys 2k and 2k+1 of this row as a bf16 pair.
#pragma unroll
      for (int c = 0; c < 2; ++c) {  // 32 keys -> 16 columns at a time
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const uint64_t x2 = f32x2_fma(
              f32x2_pack(__uint_as_float(sr[c][2 * e]), __uint_as_float(sr[c][2 * e + 1])), sc2, nm2);
          float x0, x1;
          f32x2_unpack(x2, x0, x1);
          const float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
          sum2[e & 1] = f32x2_add(sum2[e & 1], f32x2_pack(p0, p1));
          w[e] = pack_bf16x2(p0, p1);
        }
        tmem_st16(tmem_s + sb * kKeys + c * 16 + t_lane, w);
      }
      float s_lo, s_hi;
      f32x2_unpack(f32x2_add(sum2[0], sum2[1]), s_lo, s_hi);
      l += s_lo + s_hi;
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&sm.p_full[sb]);
    }
    if (ok && !__all_sync(0xffffffffu, mbar_wait(&sm.pv_done[(n_kv - 1) % kSBufs], ((n_kv - 1) / kSBufs) & 1))) ok = false;
    if (!ok) {
      flag_error(a, sm, kErrWaitTimeout);
    } else {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(tmem_o + t_lane + c * 32, o);
        tmem_ld_wait();
        if (out_row) {
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint4 wv;
            wv.x = pack_bf16x2(__uint_as_float(o[q4 * 8 + 0]) * inv, __uint_as_float(o[q4 * 8 + 1]) * inv);
            wv.y = pack_bf16x2(__uint_as_float(o[q4 * 8 + 2]) * inv, __uint_as_float(o[q4 * 8 + 3]) * inv);
            wv.z = pack_bf16x2(__uint_as_float(o[q4 * 8 + 4]) * inv, __uint_as_float(o[q4 * 8 + 5]) * inv);
            wv.w = pack_bf16x2(__uint_as_float(o[q4 * 8 + 6]) * inv, __uint_as_float(o[q4 * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(out_row + c * 32 + q4 * 8) = wv;
          }
        }
      }
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

int launch_prefill(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm, const PrefillArgs& a,
                   int batch, int max_q_len, cudaStream_t stream) {
  const size_t smem = sizeof(PrefillSmem) + 1024;
  int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(&prefill_kernel), smem);
  if (rc != NVK_OK) return rc;
  const dim3 grid((max_q_len + kRows - 1) / kRows, a.num_heads, batch);
  return check_cuda(launch_pdl(prefill_kernel, grid, dim3(kThreads), smem, stream, qm, km, vm, a), "prefill launch");
}

int check_common(const void* out, const void* query, int batch, int total_q, int max_q_len, int num_heads,
                 int num_kv_heads, int head_dim, const char* who) {
  if (batch < 0 || total_q < 0 || max_q_len < 0 || num_heads <= 0 || num_kv_heads <= 0)
    return fail(NVK_ERR_INVALID_ARGUMENT, "%s: bad sizes (batch=%d total_q=%d max_q_len=%d heads=%d kv_heads=%d)",
                who, batch, total_q, max_q_len, num_heads, num_kv_heads);
  if (head_dim != kD) return fail(NVK_ERR_UNSUPPORTED, "%s: head_dim %d unsupported (128 only)", who, head_dim);
  if (num_heads % num_kv_heads != 0)
    return fail(NVK_ERR_INVALID_ARGUMENT, "%s: num_heads %d not a multiple of num_kv_heads %d", who, num_heads,
                num_kv_heads);
  if (batch > 65535 || num_heads > 65535)
    return fail(NVK_ERR_UNSUPPORTED, "%s: batch %d or heads %d above grid limit", who, batch, num_heads);
  if (!out || !query) return fail(NVK_ERR_INVALID_ARGUMENT, "%s: null pointer", who);
  if (!aligned16(out) || !aligned16(query))
    return fail(NVK_ERR_INVALID_ARGUMENT, "%s: q/out must be 16-byte aligned", who);
  return NVK_OK;
}

}  // namespace
}  // namespace nvk

extern "C" int nvk_paged_prefill(void* out, const void* query, const void* key_cache, const void* value_cache,
                                 int num_blocks, int block_size, const int32_t* block_tables, int block_table_stride,
                                 const int32_t* cu_seqlens_q, const int32_t* kv_lens, int batch, int total_q,
                                 int max_q_len, int num_heads, int num_kv_heads, int head_dim, float scale,
                                 int* error_word, nvk_stream_t stream) {
  using namespace nvk;
  int rc = check_common(out, query, batch, total_q, max_q_len, num_heads, num_kv_heads, head_dim, "paged_prefill");
  if (rc != NVK_OK) return rc;
  if (batch == 0 || total_q == 0 || max_q_len == 0) return NVK_OK;
  if (block_size != kRows)
    return fail(NVK_ERR_UNSUPPORTED, "paged_prefill: block_size %d unsupported (128 only)", block_size);
  if (num_blocks <= 0 || !key_cache || !value_cache || !block_tables || !cu_seqlens_q || !kv_lens)
    return fail(NVK_ERR_INVALID_ARGUMENT, "paged_prefill: null pointer or empty pool");
  if (block_table_stride <= 0) return fail(NVK_ERR_INVALID_ARGUMENT, "paged_prefill: bad block table stride");
  CUtensorMap qm, km, vm;
  if ((rc = kv_tensor_map(&qm, query, total_q, num_heads, kRows)) != NVK_OK) return rc;
  const int64_t rows = static_cast<int64_t>(num_blocks) * block_size;
  if ((rc = kv_tensor_map(&km, key_cache, rows, num_kv_heads, kKeys)) != NVK_OK) return rc;
  if ((rc = kv_tensor_map(&vm, value_cache, rows, num_kv_heads, kKeys)) != NVK_OK) return rc;
  PrefillArgs a{};
  a.out = static_cast<__nv_bfloat16*>(out);
  a.block_tables = block_tables;
  a.cu_q = cu_seqlens_q;
  a.kv_lens = kv_lens;
  a.cu_kv = nullptr;
  a.err = error_word;
  a.bt_stride = block_table_stride;
  a.num_blocks = num_blocks;
  a.num_heads = num_heads;
  a.qpk = num_heads / num_kv_heads;
  a.paged = 1;
  a.scale_log2 = scale * 1.4426950408889634f;
  return launch_prefill(qm, km, vm, a, batch, max_q_len, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int nvk_dense_prefill(void* out, const void* query, const void* key, const void* value,
                                 const int32_t* cu_seqlens_q, const int32_t* cu_seqlens_kv, int batch, int total_q,
                                 int total_kv, int max_q_len, int num_heads, int num_kv_heads, int head_dim,
                                 float scale, int* error_word, nvk_stream_t stream) {
  using namespace nvk;
  int rc = check_common(out, query, batch, total_q, max_q_len, num_heads, num_kv_heads, head_dim, "dense_prefill");
  if (rc != NVK_OK) return rc;
  if (batch == 0 || total_q == 0 || max_q_len == 0) return NVK_OK;
  if (total_kv <= 0 || !key || !value || !cu_seqlens_q || !cu_seqlens_kv)
    return fail(NVK_ERR_INVALID_ARGUMENT, "dense_prefill: null pointer or no keys");
  CUtensorMap qm, km, vm;
  if ((rc = kv_tensor_map(&qm, query, total_q, num_heads, kRows)) != NVK_OK) return rc;
  if ((rc = kv_tensor_map(&km, key, total_kv, num_kv_heads, kKeys)) != NVK_OK) return rc;
  if ((rc = kv_tensor_map(&vm, value, total_kv, num_kv_heads, kKeys)) != NVK_OK) return rc;
  PrefillArgs a{};
  a.out = static_cast<__nv_bfloat16*>(out);
  a.block_tables = nullptr;
  a.cu_q = cu_seqlens_q;
  a.kv_lens = nullptr;
  a.cu_kv = cu_seqlens_kv;
  a.err = error_word;
  a.bt_stride = 0;
  a.num_blocks = 0;
  a.num_heads = num_heads;
  a.qpk = num_heads / num_kv_heads;
  a.paged = 0;
  a.scale_log2 = scale * 1.4426950408889634f;
  return launch_prefill(qm, km, vm, a, batch, max_q_len, reinterpret_cast<cudaStream_t>(stream));
}
