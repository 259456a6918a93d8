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
// Work item = 128 query rows of one sequence x one query head. The grid is
// persistent (one CTA per SM); CTA c takes items c, c + C, c + 2C, ... in an
// order that puts the heaviest query tiles first. Per item the 128-key K and
// V tiles (one pool block each) stream through shared memory.
// Tensor memory (512 columns): S/P double buffered at 0 and 128, O at 256,
// the item's Q as the A operand of S = Q K^T at 384 / 448 (double buffered
// across items), so an S UMMA reads only K from shared memory.
//   warp 8 (producer): per item a TMA load of the Q tile into one of two
//     staging buffers, then per key tile the K and V tiles (two 64-dim halves
//     each, 128-byte swizzle = the canonical UMMA operand layout) into
//     2-stage rings; block ids 32 at a time (one parallel load per warp).
//   warp 9 (MMA, one elected lane): S(j) = Q K(j)^T (A from TMEM) into S
//     buffer j % 2, two tiles ahead of O += P(j) V(j) (P from TMEM where the
//     softmax wrote it over S(j), V MN-major from smem); S(j+2) is issued
//     right behind P V(j) (tcgen05.mma executes in issue order, so it
//     overwrites P(j) only after the P V has read it). An item's first two S
//     tiles are issued behind the previous item's last P V, while the
//     softmax warps still write that item's output.
//   warps 0-7 (softmax, two warpgroups): query row r = TMEM lane r belongs
//     to thread r of both warpgroups; warpgroup wg handles keys wg*64 ..
//     wg*64+63 of every tile and dims wg*64 .. wg*64+63 of Q and O, so that
//     each sub-partition's exponentials spread over two warps. Per item the
//     copy of the Q row halves from the staging buffer into TMEM; per tile 64
//     scores in one round of tcgen05.ld, mask, the row max exchanged through
//     shared memory, base-2 online softmax, P written as bf16 pairs into the
//     warpgroup's 32 columns of its S buffer (tcgen05.st), lazy rescaling of
//     its half of O (only when the running max grew by more than 2^8, after
//     P V(j-1) completed); per item the next item's Q copy, the row sums
//     exchanged, the normalised O rows staged in the item's own Q staging
//     buffer (O released) and stored two whole rows per warp instruction.
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
constexpr int kRows = 128;                // query rows per item (UMMA M)
constexpr int kKeys = 128;                // keys per K/V tile: one 128-token pool block
constexpr int kHalfBytes = 128 * 128;     // one 64-dim half of a 128-row tile
constexpr int kTileBytes = 2 * kHalfBytes;
constexpr int kStages = 2;                // K, V and Q ring depth
constexpr int kSoftmaxThreads = 128;      // per warpgroup; two warpgroups share every row
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 10 * 32;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256;           // O accumulator
constexpr uint32_t kColQ = 384;           // Q(item) at kColQ + (item % 2) * 64
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
  int batch;
  int qtiles;  // query tiles of the longest sequence
  float scale_log2;
};

struct PrefillSmem {
  alignas(1024) uint8_t q[kStages][kTileBytes];
  alignas(1024) uint8_t k[kStages][kTileBytes];
  alignas(1024) uint8_t v[kStages][kTileBytes];
  uint64_t q_full[kStages], q_empty[kStages], q_tmem[kStages];
  uint64_t full_k[kStages], k_empty[kStages];
  uint64_t full_v[kStages], v_empty[kStages];
  uint64_t s_full[2];   // S(j) in buffer j % 2
  uint64_t p_full[2];   // P(j) written over it by the 256 softmax threads
  uint64_t pv_done[2];  // O += P V(j) complete, barrier j % 2 (one phase per two tiles, so a
                        // wait is never two phases behind its barrier)
  uint64_t o_free;      // one phase per item: its O has been read out
  uint64_t fin;
  uint64_t max_ready[2];    // both halves' row maxima of tile j written (barrier j % 2)
  uint64_t sum_ready;       // both halves' row sums of an item written
  uint64_t staged;          // an item's normalised rows are in the staging buffer
  float rowmax[2][2][kRows];  // [tile parity][warpgroup][row]: per-half row maxima
  float rowsum[2][kRows];     // [warpgroup][row]: per-half row sums of an item
  uint32_t tmem_base;
  volatile int abort;
};

static_assert(sizeof(PrefillSmem) + 1024 <= 232448, "prefill shared memory exceeds one SM's 227 KB");

// One work item: query tile qt of head h of sequence b. Every role walks the
// same list; `next` skips items without rows and reports their key tiles.
struct Item {
  int w, qt, h, b, q0, lq, lk, kv_row0, n_kv;
};

__device__ __forceinline__ bool load_item(const PrefillArgs& a, int w, Item& it) {
  const int per_tile = a.num_heads * a.batch;
  it.w = w;
  it.qt = a.qtiles - 1 - w / per_tile;  // heaviest (last) query tiles first
  const int rem = w - (a.qtiles - 1 - it.qt) * per_tile;
  it.h = rem % a.num_heads;
  it.b = rem / a.num_heads;
  it.q0 = a.cu_q[it.b];
  it.lq = a.cu_q[it.b + 1] - it.q0;
  if (it.qt * kRows >= it.lq) return false;
  it.lk = a.paged ? a.kv_lens[it.b] : (a.cu_kv[it.b + 1] - a.cu_kv[it.b]);
  it.kv_row0 = a.paged ? 0 : a.cu_kv[it.b];
  const int i_last = min(it.qt * kRows + kRows - 1, it.lq - 1);
  const int lim_last = min(it.lk - it.lq + i_last, it.lk - 1);
  it.n_kv = lim_last < 0 ? 0 : lim_last / kKeys + 1;
  return true;
}

// Next item of this CTA at or after list position w that has key tiles
// (items with rows but no visible key are handed to `zero_rows`).
template <typename ZeroRows>
__device__ __forceinline__ bool next_item(const PrefillArgs& a, int& w, int total, Item& it, ZeroRows&& zero_rows) {
  for (; w < total; w += gridDim.x) {
    if (!load_item(a, w, it)) continue;
    if (it.n_kv == 0) {
      zero_rows(it);
      continue;
    }
    return true;
  }
  return false;
}

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

// Half (64 columns) of this thread's O row times alpha, in TMEM.
__device__ __forceinline__ void rescale_o_half(uint32_t tmem_o, float alpha) {
#pragma unroll 1
  for (int c = 0; c < 2; ++c) {
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
                                                              const __grid_constant__ CUtensorMap vmap,
                                                              const PrefillArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int total = a.qtiles * a.num_heads * a.batch;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  extern __shared__ uint8_t smem_raw[];
  PrefillSmem& sm =
      *reinterpret_cast<PrefillSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.q_full[s], 1);
      mbar_init(&sm.q_empty[s], 2 * kSoftmaxThreads);
      mbar_init(&sm.q_tmem[s], 2 * kSoftmaxThreads);
      mbar_init(&sm.full_k[s], 1);
      mbar_init(&sm.k_empty[s], 1);
      mbar_init(&sm.full_v[s], 1);
      mbar_init(&sm.v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.p_full[s], 2 * kSoftmaxThreads);
    }
    mbar_init(&sm.pv_done[0], 1);
    mbar_init(&sm.pv_done[1], 1);
    mbar_init(&sm.o_free, 2 * kSoftmaxThreads);
    mbar_init(&sm.max_ready[0], 2 * kSoftmaxThreads);
    mbar_init(&sm.max_ready[1], 2 * kSoftmaxThreads);
    mbar_init(&sm.sum_ready, 2 * kSoftmaxThreads);
    mbar_init(&sm.staged, 2 * kSoftmaxThreads);
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
  auto no_zero = [](const Item&) {};

  if (warp == kProducerWarp) {
    // -------------------------------------------------------- producer ----
    if (lane == 0) {
      tma_prefetch_desc(&qmap);
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
    }
    int w = blockIdx.x, qi = 0, g = 0, q_issued = 0, k_issued = 0, v_issued = 0;
    bool ok = true;
    Item it;
    while (ok && next_item(a, w, total, it, no_zero)) {
      const int qs = qi % kStages;
      if (lane == 0) {
        if (qi >= kStages && !mbar_wait(&sm.q_empty[qs], ((qi / kStages) - 1) & 1)) {
          ok = false;
        } else {
          mbar_arrive_expect_tx(&sm.q_full[qs], kTileBytes);
          tma_load_3d(sm.q[qs], &qmap, &sm.q_full[qs], 0, it.h, it.q0 + it.qt * kRows);
          tma_load_3d(sm.q[qs] + kHalfBytes, &qmap, &sm.q_full[qs], 64, it.h, it.q0 + it.qt * kRows);
          ++q_issued;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      const int kvh = it.h / a.qpk;
      const int32_t* bt = a.block_tables + static_cast<int64_t>(it.b) * a.bt_stride;
      int ids = 0;
      for (int j = 0; ok && j < it.n_kv; ++j, ++g) {
        if (__shfl_sync(0xffffffffu, sm.abort, 0)) { ok = false; break; }
        if ((j & 31) == 0 && a.paged) {  // block ids of tiles j .. j+31, one per lane
          const int jj = j + lane;
          int blk = 0;
          if (jj < it.n_kv) {
            blk = bt[jj];
            if (blk < 0 || blk >= a.num_blocks) {
              if (a.err) atomicOr(a.err, kErrBadBlockId);
              blk = a.num_blocks;  // fully outside the tensor map: zero fill
            }
          }
          ids = blk;
        }
        const int blk = __shfl_sync(0xffffffffu, ids, j & 31);
        const int row = a.paged ? blk * kKeys : it.kv_row0 + j * kKeys;
        const int st = g % kStages;
        if (lane == 0) {
          if (g >= kStages && !mbar_wait(&sm.k_empty[st], ((g / kStages) - 1) & 1)) {
            ok = false;
          } else {
            mbar_arrive_expect_tx(&sm.full_k[st], kTileBytes);
            tma_load_3d(sm.k[st], &kmap, &sm.full_k[st], 0, kvh, row);
            tma_load_3d(sm.k[st] + kHalfBytes, &kmap, &sm.full_k[st], 64, kvh, row);
            ++k_issued;
            if (g >= kStages && !mbar_wait(&sm.v_empty[st], ((g / kStages) - 1) & 1)) {
              ok = false;
            } else {
              mbar_arrive_expect_tx(&sm.full_v[st], kTileBytes);
              tma_load_3d(sm.v[st], &vmap, &sm.full_v[st], 0, kvh, row);
              tma_load_3d(sm.v[st] + kHalfBytes, &vmap, &sm.full_v[st], 64, kvh, row);
              ++v_issued;
            }
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
      }
      ++qi;
      w += gridDim.x;
    }
    if (lane == 0) {
      if (!ok) flag_error(a, sm, kErrWaitTimeout);
      // Drain every copy this CTA issued before it may exit.
      for (int j = max(0, q_issued - kStages); j < q_issued; ++j)
        (void)mbar_wait(&sm.q_full[j % kStages], (j / kStages) & 1);
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
      bool ok = true;
      // S(g) = Q(item qi) K(g)^T into S buffer g % 2 (A from TMEM, B from smem)
      auto issue_s = [&](int g, int qi) -> bool {
        const int st = g % kStages;
        if (!mbar_wait(&sm.full_k[st], (g / kStages) & 1)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sm.k[st]);
        const uint32_t q_col = tmem + kColQ + (qi % 2) * 64;
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
          umma_f16_ts(tmem + (g % 2) * kKeys, q_col + kk * 8, smem_desc_sw128(k_addr + off, 16, 1024), idesc_qk,
                      kk > 0);
        }
        umma_commit(&sm.s_full[g % 2]);
        umma_commit(&sm.k_empty[st]);
        return true;
      };
      // S of an item's first two tiles, once its Q is in TMEM
      auto start_item = [&](const Item& it, int g0, int qi) -> bool {
        if (!mbar_wait(&sm.q_tmem[qi % 2], (qi / 2) & 1)) return false;
        tc_fence_after();
        for (int j = 0; j < 2 && j < it.n_kv; ++j)
          if (!issue_s(g0 + j, qi)) return false;
        return true;
      };
      int w = blockIdx.x, qi = 0, g = 0;
      Item it;
      bool have = next_item(a, w, total, it, no_zero);
      if (have) ok = start_item(it, 0, 0);
      while (ok && have) {
        for (int j = 0; j < it.n_kv; ++j, ++g) {
          const int b2 = g % 2, st = g % kStages;
          if (!mbar_wait(&sm.p_full[b2], (g / 2) & 1) || !mbar_wait(&sm.full_v[st], (g / kStages) & 1) ||
              (j == 0 && qi > 0 && !mbar_wait(&sm.o_free, (qi - 1) & 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t v_addr = smem_u32(sm.v[st]);
#pragma unroll
          for (int kk = 0; kk < kKeys / 16; ++kk) {
            const uint64_t vb = smem_desc_sw128(v_addr + kk * 16 * 128, kHalfBytes, 1024);
            umma_f16_ts(tmem + kColO, tmem + b2 * kKeys + kk * 8, vb, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&sm.v_empty[st]);
          umma_commit(&sm.pv_done[b2]);
          if (j + 2 < it.n_kv && !issue_s(g + 2, qi)) {
            ok = false;
            break;
          }
        }
        if (!ok) break;
        ++qi;
        w += gridDim.x;
        have = next_item(a, w, total, it, no_zero);
        if (have) ok = start_item(it, g, qi);
      }
      if (!ok) flag_error(a, sm, kErrWaitTimeout);
      // All MMAs of this CTA complete before TMEM is released.
      umma_commit(&sm.fin);
      (void)mbar_wait(&sm.fin, 0);
    }
  } else {
    // --------------------------------------------------------- softmax ----
    // Two warpgroups share every row: warpgroup wg takes keys wg*64 .. wg*64+63
    // of each tile (and dims wg*64 .. of Q and O); both track the same running
    // max, exchanged once per tile, and their own row sums.
    const int wg = warp >> 2;               // 0 or 1
    const int r = tid & (kRows - 1);        // query row within the tile = TMEM lane
    const uint32_t t_lane = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tmem_o = tmem + kColO + wg * 64 + t_lane;
    // Rows of an item that sees no key: zeros (each warpgroup its half of the dims).
    auto zero_rows = [&](const Item& z) {
      const int i = z.qt * kRows + r;
      if (i < z.lq) {
        __nv_bfloat16* row = a.out + (static_cast<int64_t>(z.q0 + i) * a.num_heads + z.h) * kD + wg * 64;
        for (int c = 0; c < 64; c += 8) *reinterpret_cast<uint4*>(row + c) = make_uint4(0, 0, 0, 0);
      }
    };
    // This warpgroup's half (64 dims) of Q row r of item qi from the staging
    // buffer into TMEM (the A operand of S).
    auto copy_q = [&](int qi) -> bool {
      const int qs = qi % kStages;
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.q_full[qs], (qi / kStages) & 1))) return false;
      uint32_t words[32];
      const uint8_t* base = sm.q[qs] + wg * kHalfBytes + r * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {  // 16-byte chunk c of the row sits at chunk c ^ (r % 8) (128-byte swizzle)
        const uint4 v4 = *reinterpret_cast<const uint4*>(base + ((c ^ (r & 7)) << 4));
        words[4 * c + 0] = v4.x;
        words[4 * c + 1] = v4.y;
        words[4 * c + 2] = v4.z;
        words[4 * c + 3] = v4.w;
      }
      // (the stage is released after this item's epilogue, which uses it as scratch)
      tmem_st32(tmem + kColQ + (qi % 2) * 64 + wg * 32 + t_lane, words);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&sm.q_tmem[qi % 2]);
      return true;
    };
    int w = blockIdx.x, qi = 0, g = 0;
    bool ok = true;
    Item it;
    bool have = next_item(a, w, total, it, zero_rows);
    if (have) ok = copy_q(0);
    while (ok && have) {
      const int i = it.qt * kRows + r;
      const int lim = (i < it.lq) ? (it.lk - it.lq + i) : (it.lk - 1);
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < it.n_kv; ++j, ++g) {
        const int b2 = g % 2;
        const uint32_t tmem_s = tmem + b2 * kKeys + t_lane;
        // warp-uniform outcome: the tcgen05.ld/st below need a converged warp
        if (!__all_sync(0xffffffffu, mbar_wait(&sm.s_full[b2], (g / 2) & 1))) { ok = false; break; }
        tc_fence_after();
        const int kbase = j * kKeys + wg * 64;
        uint32_t sr[2][32];
        tmem_ld32(tmem_s + wg * 64, sr[0]);
        tmem_ld32(tmem_s + wg * 64 + 32, sr[1]);
        tmem_ld_wait();
        if (kbase + 63 > lim) {
#pragma unroll
          for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (kbase + c * 32 + e > lim) sr[c][e] = __float_as_uint(-INFINITY);
        }
        // The max is taken over raw scores (scale > 0), the scale folded into
        // the exponent's FMA below; max is exact, so its order is free.
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            mx0 = fmax3(mx0, __uint_as_float(sr[c][e]), __uint_as_float(sr[c][e + 1]));
            mx1 = fmax3(mx1, __uint_as_float(sr[c][e + 2]), __uint_as_float(sr[c][e + 3]));
          }
        // Row max over both halves: exchanged through shared memory (one slot
        // per tile parity, so the next tile's writes cannot race these reads).
        // (it also orders both warpgroups' score reads before the P writes below)
        sm.rowmax[b2][wg][r] = fmaxf(mx0, mx1);
        tc_fence_before();
        mbar_arrive(&sm.max_ready[b2]);
        if (!__all_sync(0xffffffffu, mbar_wait(&sm.max_ready[b2], (g / 2) & 1))) { ok = false; break; }
        tc_fence_after();
        const float mt = fmaxf(sm.rowmax[b2][0][r], sm.rowmax[b2][1][r]) * a.scale_log2;
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
        // P of keys wg*64 .. wg*64+63 into columns wg*32 .. wg*32+31 of the S
        // buffer (column k holds keys 2k and 2k+1 as a bf16 pair): columns
        // whose scores both warpgroups read before the exchange above.
#pragma unroll
        for (int c = 0; c < 2; ++c) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {  // word e of P overwrites score e, already read
            const float p0 = fast_exp2(fmaf(__uint_as_float(sr[c][2 * e]), sc, neg_mu));
            const float p1 = fast_exp2(fmaf(__uint_as_float(sr[c][2 * e + 1]), sc, neg_mu));
            sum[(2 * e) & 3] += p0;
            sum[(2 * e + 1) & 3] += p1;
            sr[c][e] = pack_bf16x2(p0, p1);
          }
          tmem_st16_first(tmem_s + wg * 32 + c * 16, sr[c]);
        }
        l += (sum[0] + sum[1]) + (sum[2] + sum[3]);
        // This warpgroup's half of the O rows rescales (rarely) once P V(j-1)
        // is complete, before this tile's P is signalled and P V(j) issued.
        if (j > 0 && __any_sync(0xffffffffu, resc)) {
          if (!__all_sync(0xffffffffu, mbar_wait(&sm.pv_done[(g - 1) % 2], ((g - 1) / 2) & 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
          rescale_o_half(tmem_o, alpha);
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&sm.p_full[b2]);
      }
      if (!ok) break;
      // The next item's Q goes into TMEM now, so that its first S tiles are
      // computed while this item's output is written.
      const int g_last = g - 1;
      int w_next = w + gridDim.x;
      Item nx;
      const bool have_next = next_item(a, w_next, total, nx, zero_rows);
      if (have_next && !copy_q(qi + 1)) { ok = false; break; }
      sm.rowsum[wg][r] = l;
      mbar_arrive(&sm.sum_ready);
      // P V completes in issue order: the last tile's implies the item's.
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.pv_done[g_last % 2], (g_last / 2) & 1))) {
        ok = false;
        break;
      }
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.sum_ready, qi & 1))) {  // both row sums written
        ok = false;
        break;
      }
      tc_fence_after();
      // Output through the item's Q staging buffer (free since its copy into
      // TMEM): thread r writes its half of the normalised row there (16-byte
      // chunk c of row r at chunk c ^ (r % 16): conflict-free), then every
      // warp stores two whole rows per instruction, so the global writes are
      // coalesced.
      const float lt = sm.rowsum[0][r] + sm.rowsum[1][r];
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      uint8_t* scratch = sm.q[qi % kStages];
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t o[32];
        tmem_ld32(tmem_o + c * 32, o);
        tmem_ld_wait();
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          uint4 wv;
          wv.x = pack_bf16x2(__uint_as_float(o[q4 * 8 + 0]) * inv, __uint_as_float(o[q4 * 8 + 1]) * inv);
          wv.y = pack_bf16x2(__uint_as_float(o[q4 * 8 + 2]) * inv, __uint_as_float(o[q4 * 8 + 3]) * inv);
          wv.z = pack_bf16x2(__uint_as_float(o[q4 * 8 + 4]) * inv, __uint_as_float(o[q4 * 8 + 5]) * inv);
          wv.w = pack_bf16x2(__uint_as_float(o[q4 * 8 + 6]) * inv, __uint_as_float(o[q4 * 8 + 7]) * inv);
          const int chunk = wg * 8 + c * 4 + q4;
          *reinterpret_cast<uint4*>(scratch + r * 256 + ((chunk ^ (r & 15)) << 4)) = wv;
        }
      }
      // O is read out: the next item's first P V may overwrite it.
      tc_fence_before();
      mbar_arrive(&sm.o_free);
      mbar_arrive(&sm.staged);
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.staged, qi & 1))) {  // the staged rows are complete
        ok = false;
        break;
      }
      {
        const int c = lane & 15;
        const int lq_rows = it.lq - it.qt * kRows;  // valid rows of this tile
#pragma unroll 4
        for (int k = 0; k < 8; ++k) {
          const int row = warp * 16 + k * 2 + (lane >> 4);
          if (row < lq_rows) {
            const uint4 v4 = *reinterpret_cast<const uint4*>(scratch + row * 256 + ((c ^ (row & 15)) << 4));
            __nv_bfloat16* dst =
                a.out + (static_cast<int64_t>(it.q0 + it.qt * kRows + row) * a.num_heads + it.h) * kD + c * 8;
            *reinterpret_cast<uint4*>(dst) = v4;
          }
        }
      }
      // The scratch reads are done: the stage may take the Q tile of the
      // item after next (an async-proxy write).
      fence_proxy_async_smem();
      mbar_arrive(&sm.q_empty[qi % kStages]);
      ++qi;
      w = w_next;
      it = nx;
      have = have_next;
    }
    if (!ok) flag_error(a, sm, kErrWaitTimeout);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) {
    __syncwarp();
    tmem_dealloc(tmem, kTmemCols);
  }
}

int launch_prefill(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm, PrefillArgs a,
                   int max_q_len, cudaStream_t stream) {
  const size_t smem = sizeof(PrefillSmem) + 1024;
  int rc = ensure_dynamic_smem(reinterpret_cast<const void*>(&prefill_kernel), smem);
  if (rc != NVK_OK) return rc;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  a.qtiles = (max_q_len + kRows - 1) / kRows;
  const int64_t items = static_cast<int64_t>(a.qtiles) * a.num_heads * a.batch;
  if (items > (int64_t(1) << 30))
    return fail(NVK_ERR_UNSUPPORTED, "prefill: %lld work items above the kernel's range", (long long)items);
  const int grid = static_cast<int>(items < sms ? items : sms);
  return check_cuda(launch_pdl(prefill_kernel, dim3(grid), dim3(kThreads), smem, stream, qm, km, vm, a),
                    "prefill launch");
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
  a.batch = batch;
  a.scale_log2 = scale * 1.4426950408889634f;
  return launch_prefill(qm, km, vm, a, max_q_len, reinterpret_cast<cudaStream_t>(stream));
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
  a.batch = batch;
  a.scale_log2 = scale * 1.4426950408889634f;
  return launch_prefill(qm, km, vm, a, max_q_len, reinterpret_cast<cudaStream_t>(stream));
}
