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
// One CTA = 128 query rows of one sequence x TWO query heads of one GQA
// group ("streams" 0 and 1; one stream when the group size is odd), one CTA
// per SM. Both streams read the same 128-key K and V tiles (one pool block
// each), so every K/V byte staged in shared memory feeds two heads.
// Tensor memory (all 512 columns): S/P of stream s at columns s*128, its O
// accumulator at 256 + s*128.
//   warp 8 (producer): TMA loads of the two Q tiles once, then per key tile
//     the K and the V tile (two 64-dim halves each, 128-byte swizzle = the
//     canonical UMMA operand layout) into 2-stage rings; block ids 32 at a
//     time (one parallel load per warp).
//   warp 9 (MMA, one elected lane): S_s(0) = Q_s K(0)^T for both streams,
//     then per tile j and stream s: wait for P_s(j), issue O_s += P_s(j) V(j)
//     (P read from TMEM where the softmax wrote it over S_s, V MN-major from
//     smem) and right behind it S_s(j+1) = Q_s K(j+1)^T into the same
//     columns. tcgen05.mma executes in issue order, so S_s(j+1) overwrites
//     P_s(j) only after the P V has read it, and the tensor pipe always has
//     the other stream's work queued while one stream's softmax runs.
//   warps 0-3 / 4-7 (softmax of stream 0 / 1): thread r owns query row r =
//     TMEM lane r: loads its 128-key S row (one round of tcgen05.ld), masks,
//     base-2 online softmax, P written as bf16 pairs into the first 64
//     columns of its S (tcgen05.st), lazy rescaling of O (only when the
//     running max grew by more than 2^8; S_s(j) having landed means P V(j-1)
//     is done, so O may be rescaled before P_s(j) is signalled), and at the
//     end normalises its O row and stores it.
// Ten warps put three on one SM sub-partition, whose register file holds
// 3 x 32 x 168 registers: the kernel is held to 168 registers a thread.
// Every mbarrier wait is bounded; on a timeout the CTA records the error,
// drains its in-flight copies and MMAs, frees TMEM and exits.
#include "host_common.h"
#include "nvk_common.cuh"
#include "tcgen05.cuh"

namespace nvk {
namespace {

constexpr int kD = 128;
constexpr int kRows = 128;                // query rows per CTA (UMMA M)
constexpr int kKeys = 128;                // keys per K/V tile: one 128-token pool block
constexpr int kHalfBytes = 128 * 128;     // one 64-dim half of a 128-row tile
constexpr int kTileBytes = 2 * kHalfBytes;
constexpr int kStages = 2;                // K and V ring depth
constexpr int kStreams = 2;               // query heads per CTA
constexpr int kStreamThreads = 128;       // softmax threads per stream
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 10 * 32;
constexpr uint32_t kTmemCols = 512;       // S0 | S1 | O0 | O1, 128 columns each
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
  int paired;  // two heads per CTA (qpk even)
  int paged;
  float scale_log2;
};

struct PrefillSmem {
  alignas(1024) uint8_t q[kStreams][kTileBytes];
  alignas(1024) uint8_t k[kStages][kTileBytes];
  alignas(1024) uint8_t v[kStages][kTileBytes];
  uint64_t bar_q;
  uint64_t full_k[kStages], k_empty[kStages];
  uint64_t full_v[kStages], v_empty[kStages];
  uint64_t s_full[kStreams];  // S_s(j) in TMEM (and, in issue order, P V_s(j-1) done)
  uint64_t p_full[kStreams];  // P_s(j) written by the stream's 128 softmax threads
  uint64_t o_done[kStreams];  // O_s += P_s(j) V(j) complete
  uint64_t fin;
  uint32_t tmem_base;
  volatile int abort;
};

static_assert(sizeof(PrefillSmem) + 1024 <= 232448, "prefill shared memory exceeds one SM's 227 KB");

// The first 16 of 32 registers into 16 consecutive 32-bit TMEM columns of
// this thread's lane (warp-collective).
__device__ __forceinline__ void tmem_st16_first(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// O row of this thread (four 32-column chunks) times alpha, in TMEM.
__device__ __forceinline__ void rescale_o(uint32_t tmem_o, float alpha) {
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t o[32];
    tmem_ld32(tmem_o + c * 32, o);
    tmem_ld_wait();
#pragma unroll
    for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
    tmem_st32(tmem_o + c * 32, o);
  }
}

__device__ __forceinline__ void flag_error(const PrefillArgs& a, PrefillSmem& sm, int code) {
  if (a.err) atomicOr(a.err, code);
  sm.abort = 1;
}

__global__ void __maxnreg__(168) prefill_kernel(const __grid_constant__ CUtensorMap qmap,
                                                const __grid_constant__ CUtensorMap kmap,
                                                const __grid_constant__ CUtensorMap vmap, const PrefillArgs a) {
  const int qt = gridDim.x - 1 - blockIdx.x;  // heaviest (last) query tiles first
  const int b = blockIdx.z;
  const int nstreams = a.paired ? 2 : 1;
  const int h0 = blockIdx.y * nstreams;  // query heads h0 .. h0 + nstreams - 1, one KV group
  pdl_launch_dependents();
  pdl_wait();
  const int q0 = a.cu_q[b];
  const int lq = a.cu_q[b + 1] - q0;
  if (qt * kRows >= lq) return;
  const int lk = a.paged ? a.kv_lens[b] : (a.cu_kv[b + 1] - a.cu_kv[b]);
  const int kv_row0 = a.paged ? 0 : a.cu_kv[b];
  const int g = h0 / a.qpk;
  const int i_last = min(qt * kRows + kRows - 1, lq - 1);
  const int lim_last = min(lk - lq + i_last, lk - 1);
  const int n_kv = lim_last < 0 ? 0 : lim_last / kKeys + 1;  // 128-key tiles

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int stream = warp >> 2;                  // softmax warps 0-3 / 4-7
  const int r = tid & (kStreamThreads - 1);      // query row within the tile = TMEM lane
  const int i = qt * kRows + r;                  // query row within the sequence
  __nv_bfloat16* out_row = nullptr;
  if (warp < 8 && stream < nstreams && i < lq)
    out_row = a.out + (static_cast<int64_t>(q0 + i) * a.num_heads + h0 + stream) * kD;

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
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full_k[s], 1);
      mbar_init(&sm.k_empty[s], 1);
      mbar_init(&sm.full_v[s], 1);
      mbar_init(&sm.v_empty[s], 1);
    }
    for (int s = 0; s < kStreams; ++s) {
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.p_full[s], kStreamThreads);
      mbar_init(&sm.o_done[s], 1);
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

  if (warp == kProducerWarp) {
    // -------------------------------------------------------- producer ----
    if (lane == 0) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      mbar_arrive_expect_tx(&sm.bar_q, nstreams * kTileBytes);
      for (int s = 0; s < nstreams; ++s) {
        tma_load_3d(sm.q[s], &qmap, &sm.bar_q, 0, h0 + s, q0 + qt * kRows);
        tma_load_3d(sm.q[s] + kHalfBytes, &qmap, &sm.bar_q, 64, h0 + s, q0 + qt * kRows);
      }
    }
    const int32_t* bt = a.block_tables + static_cast<int64_t>(b) * a.bt_stride;
    int ids = 0, k_issued = 0, v_issued = 0;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      // warp-uniform stop decision (lane 0's view of the abort flag)
      if (__shfl_sync(0xffffffffu, (ok ? 0 : 1) | sm.abort, 0)) break;
      if ((j & 31) == 0 && a.paged) {  // block ids of tiles j .. j+31, one per lane
        const int jj = j + lane;
        int blk = 0;
        if (jj < n_kv) {
          blk = bt[jj];
          if (blk < 0 || blk >= a.num_blocks) {
            if (a.err) atomicOr(a.err, kErrBadBlockId);
            blk = a.num_blocks;  // fully outside the tensor map: zero fill
          }
        }
        ids = blk;
      }
      const int blk = __shfl_sync(0xffffffffu, ids, j & 31);
      const int row = a.paged ? blk * kKeys : kv_row0 + j * kKeys;
      const int st = j % kStages;
      if (lane == 0) {
        if (j >= kStages && !mbar_wait(&sm.k_empty[st], ((j / kStages) - 1) & 1)) {
          ok = false;
        } else {
          mbar_arrive_expect_tx(&sm.full_k[st], kTileBytes);
          tma_load_3d(sm.k[st], &kmap, &sm.full_k[st], 0, g, row);
          tma_load_3d(sm.k[st] + kHalfBytes, &kmap, &sm.full_k[st], 64, g, row);
          ++k_issued;
          if (j >= kStages && !mbar_wait(&sm.v_empty[st], ((j / kStages) - 1) & 1)) {
            ok = false;
          } else {
            mbar_arrive_expect_tx(&sm.full_v[st], kTileBytes);
            tma_load_3d(sm.v[st], &vmap, &sm.full_v[st], 0, g, row);
            tma_load_3d(sm.v[st] + kHalfBytes, &vmap, &sm.full_v[st], 64, g, row);
            ++v_issued;
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (lane == 0) {
      if (!ok) flag_error(a, sm, kErrWaitTimeout);
      // Drain every copy this CTA issued before it may exit.
      (void)mbar_wait(&sm.bar_q, 0);
      for (int j = max(0, k_issued - kStages); j < k_issued; ++j)
        (void)mbar_wait(&sm.full_k[j % kStages], (j / kStages) & 1);
      for (int j = max(0, v_issued - kStages); j < v_issued; ++j)
        (void)mbar_wait(&sm.full_v[j % kStages], (j / kStages) & 1);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------- MMA ----
    if (lane == 0) {
      constexpr uint32_t idesc_qk = umma_idesc_bf16(kRows, kKeys, false);
      constexpr uint32_t idesc_pv = umma_idesc_bf16(kRows, kD, true);
      auto issue_s = [&](int s, int j) {  // S_s(j) = Q_s K(j)^T
        const uint32_t q_addr = smem_u32(sm.q[s]);
        const uint32_t k_addr = smem_u32(sm.k[j % kStages]);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
          umma_f16_ss(tmem + s * kKeys, smem_desc_sw128(q_addr + off, 16, 1024),
                      smem_desc_sw128(k_addr + off, 16, 1024), idesc_qk, kk > 0);
        }
        umma_commit(&sm.s_full[s]);
      };
      auto issue_pv = [&](int s, int j) {  // O_s += P_s(j) V(j)
        const uint32_t v_addr = smem_u32(sm.v[j % kStages]);
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk) {
          const uint64_t vb = smem_desc_sw128(v_addr + kk * 16 * 128, kHalfBytes, 1024);
          umma_f16_ts(tmem + 256 + s * kD, tmem + s * kKeys + kk * 8, vb, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&sm.o_done[s]);
      };
      bool ok = mbar_wait(&sm.bar_q, 0) && mbar_wait(&sm.full_k[0], 0);
      if (ok) {
        tc_fence_after();
        for (int s = 0; s < nstreams; ++s) issue_s(s, 0);
        umma_commit(&sm.k_empty[0]);
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        const int st = j % kStages;
        if (!mbar_wait(&sm.full_v[st], (j / kStages) & 1)) { ok = false; break; }
        const bool more = j + 1 < n_kv;
        for (int s = 0; ok && s < nstreams; ++s) {
          if (!mbar_wait(&sm.p_full[s], j & 1)) { ok = false; break; }
          if (s == 0 && more && !mbar_wait(&sm.full_k[(j + 1) % kStages], ((j + 1) / kStages) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(s, j);
          if (s == nstreams - 1) umma_commit(&sm.v_empty[st]);
          if (more) {
            issue_s(s, j + 1);
            if (s == nstreams - 1) umma_commit(&sm.k_empty[(j + 1) % kStages]);
          }
        }
      }
      if (!ok) flag_error(a, sm, kErrWaitTimeout);
      // All MMAs of this CTA complete before TMEM is released.
      umma_commit(&sm.fin);
      (void)mbar_wait(&sm.fin, 0);
    }
  } else if (stream < nstreams) {
    // --------------------------------------------------------- softmax ----
    const int lim = (i < lq) ? (lk - lq + i) : (lk - 1);
    const uint32_t t_lane = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tmem_s = tmem + stream * kKeys + t_lane;
    const uint32_t tmem_o = tmem + 256 + stream * kD + t_lane;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      // warp-uniform outcome: the tcgen05.ld/st below need a converged warp
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.s_full[stream], j & 1))) { ok = false; break; }
      tc_fence_after();
      const int kbase = j * kKeys;
      // The whole 128-key S row in one round of TMEM loads.
      uint32_t sr[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tmem_s + c * 32, sr[c]);
      tmem_ld_wait();
      if (kbase + kKeys - 1 > lim) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (kbase + c * 32 + e > lim) sr[c][e] = __float_as_uint(-INFINITY);
      }
      // The max is taken over raw scores (scale > 0), the scale folded into
      // the exponent's FMA below; max is exact, so its order is free.
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          mx0 = fmax3(mx0, __uint_as_float(sr[c][e]), __uint_as_float(sr[c][e + 1]));
          mx1 = fmax3(mx1, __uint_as_float(sr[c][e + 2]), __uint_as_float(sr[c][e + 3]));
        }
      const float mt = fmaxf(mx0, mx1) * a.scale_log2;
      const float m_new = fmaxf(m, mt);
      const bool resc = m_new > m + kRescaleThreshold;
      const float alpha = resc ? fast_exp2(m - m_new) : 1.f;
      if (resc) {
        l *= alpha;
        m = m_new;
      }
      const float neg_mu = (m == -INFINITY) ? 0.f : -m;
      const float sc = a.scale_log2;
      float sum[4] = {0.f, 0.f, 0.f, 0.f};  // independent add chains
      // P over the first 64 columns of the S buffer (S is in registers now):
      // column k holds keys 2k and 2k+1 of this row as a bf16 pair.
#pragma unroll
      for (int c = 0; c < 4; ++c) {  // 32 keys -> 16 columns at a time
        // word e of P overwrites score e, already read at pair e / 2 <= e
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float p0 = fast_exp2(fmaf(__uint_as_float(sr[c][2 * e]), sc, neg_mu));
          const float p1 = fast_exp2(fmaf(__uint_as_float(sr[c][2 * e + 1]), sc, neg_mu));
          sum[(2 * e) & 3] += p0;
          sum[(2 * e + 1) & 3] += p1;
          sr[c][e] = pack_bf16x2(p0, p1);
        }
        tmem_st16_first(tmem_s + c * 16, sr[c]);
      }
      l += (sum[0] + sum[1]) + (sum[2] + sum[3]);
      // S_s(j) has landed, so P V(j-1) -- issued before it -- is complete: O
      // may be rescaled now (rows of this warp, when one of them needs it),
      // before this tile's P is signalled and P V(j) issued.
      if (j > 0 && __any_sync(0xffffffffu, resc)) rescale_o(tmem_o, alpha);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&sm.p_full[stream]);
    }
    if (ok && !__all_sync(0xffffffffu, mbar_wait(&sm.o_done[stream], (n_kv - 1) & 1))) ok = false;
    if (!ok) {
      flag_error(a, sm, kErrWaitTimeout);
    } else {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld32(tmem_o + c * 32, o);
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
  const int groups = a.paired ? a.num_heads / 2 : a.num_heads;
  const dim3 grid((max_q_len + kRows - 1) / kRows, groups, batch);
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
  a.paired = a.qpk % 2 == 0;
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
  a.paired = a.qpk % 2 == 0;
  a.paged = 0;
  a.scale_log2 = scale * 1.4426950408889634f;
  return launch_prefill(qm, km, vm, a, batch, max_q_len, reinterpret_cast<cudaStream_t>(stream));
}
