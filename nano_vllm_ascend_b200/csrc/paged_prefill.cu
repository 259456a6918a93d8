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
// Work item = 128 query rows of one sequence x two query heads of one GQA
// group ("streams" 0 and 1; one stream when the group size is odd). Both
// streams read the same 128-key K and V tiles (one pool block each), so each
// K/V byte staged in shared memory feeds two heads. The grid is persistent
// (one CTA per SM); CTA c takes items c, c + C, c + 2C, ... in an order that
// puts the heaviest query tiles first.
// Tensor memory (512 columns): S/P of stream s at s * 128, its O accumulator
// at 256 + s * 128.
//   warp 8 (producer): walks the item list and publishes each item's
//     descriptor through a 4-slot shared-memory ring (the other roles never
//     read the item metadata from global memory); per item the TMA loads of
//     the streams' Q tiles (once the previous item's last S has read their
//     buffers), then per key tile the K and V tiles (two 64-dim halves each,
//     128-byte swizzle = the canonical UMMA operand layout) into 2-stage
//     rings; block ids 32 at a time (one parallel load per warp).
//   warp 9 (MMA; the whole warp runs the loop, an elected lane issues):
//     per tile j and stream s, once the first 64 keys of P_s(j) are written,
//     O_s += P V over them, then over the other 64 (P read from TMEM where
//     the softmax wrote it over S_s, V MN-major from smem), and right behind
//     it S_s(j+1) = Q_s K(j+1)^T into the same columns. tcgen05.mma executes
//     in issue order, so S_s(j+1) overwrites P_s(j) only after the P V has
//     read it, and the tensor pipe has the other stream's work queued while
//     one stream's softmax runs. An item's first S tiles are issued behind
//     the previous item's last P V.
//   warps 0-3 / 4-7 (softmax of stream 0 / 1): thread r owns query row r =
//     TMEM lane r. Per tile the 128 scores of its row in one round of
//     tcgen05.ld, the mask, base-2 online softmax, P written as bf16 pairs
//     over the first 64 columns of S_s (tcgen05.st) in two halves, each
//     signalled once stored; lazy rescaling of O_s (only when the running
//     max grew by more than 2^8; S_s(j) having landed means P V_s(j-1),
//     issued before it, is complete). Per item, once its last P V_s has
//     completed, the normalised O_s rows go out through a staging buffer:
//     each warp stores the 32 rows its own lanes staged as whole 128-byte
//     row halves (coalesced), and O_s is released to the next item.
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
constexpr int kStages = 2;                // K and V ring depth
constexpr int kStreams = 2;               // query heads per item
constexpr int kStreamThreads = 128;       // softmax threads per stream
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 10 * 32;
constexpr uint32_t kTmemCols = 512;       // S_0 | S_1 | O_0 | O_1, 128 columns each
constexpr uint32_t kColO = 256;
constexpr float kRescaleThreshold = 8.0f;
constexpr int kItemRing = 4;              // item descriptors published ahead by the producer

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
  int paired;  // two heads per item (GQA group size even)
  int paged;
  int batch;
  int qtiles;  // query tiles of the longest sequence
  float scale_log2;
};

// One work item: query tile qt of heads h0 .. h0 + streams - 1 of sequence b
// (n_kv < 0: no further item).
struct Item {
  int qt, h0, kvh, b, q0, lq, lk, kv_row0, n_kv;
};

struct PrefillSmem {
  alignas(1024) uint8_t q[kStreams][kTileBytes];
  alignas(1024) uint8_t k[kStages][kTileBytes];
  alignas(1024) uint8_t v[kStages][kTileBytes];
  alignas(1024) uint8_t stage[kStreams][kHalfBytes];  // epilogue: 64 dims of 128 output rows per stream
  Item items[kItemRing];
  uint64_t item_full[kItemRing];                 // items[i % ring] written (one phase per use)
  uint64_t q_full[kStreams], q_empty[kStreams];  // one phase per item
  uint64_t full_k[kStages], k_empty[kStages];
  uint64_t full_v[kStages], v_empty[kStages];
  uint64_t s_full[kStreams];   // S_s(j) in TMEM (and, in issue order, P V_s(j-1) done)
  uint64_t p_lo[kStreams];     // P_s(j) of keys 0-63 written by the stream's 128 softmax threads
  uint64_t p_hi[kStreams];     // P_s(j) of keys 64-127 written
  uint64_t o_ready[kStreams];  // an item's last P V_s complete (one phase per item)
  uint64_t o_free[kStreams];   // an item's O_s read out (one phase per item)
  uint64_t fin;
  uint32_t tmem_base;
  volatile int abort;
};

static_assert(sizeof(PrefillSmem) + 1024 <= 232448, "prefill shared memory exceeds one SM's 227 KB");

// The producer walks the item list; `next_item` skips items without rows and
// hands the ones whose rows see no key to `zero_rows`.
__device__ __forceinline__ int item_streams(const PrefillArgs& a) { return a.paired ? kStreams : 1; }

__device__ __forceinline__ bool load_item(const PrefillArgs& a, int w, Item& it) {
  const int ns = item_streams(a);
  const int groups = a.num_heads / ns;  // head groups per sequence
  const int per_tile = groups * a.batch;
  const int t = w / per_tile;
  it.qt = a.qtiles - 1 - t;  // heaviest (last) query tiles first
  const int rem = w - t * per_tile;
  it.h0 = (rem % groups) * ns;
  it.kvh = it.h0 / a.qpk;  // both heads of a pair share it: h0 even, group size even
  it.b = rem / groups;
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

__device__ __forceinline__ void flag_error(const PrefillArgs& a, PrefillSmem& sm, int code) {
  if (a.err) atomicOr(a.err, code);
  sm.abort = 1;
}

__global__ void __maxnreg__(168) prefill_kernel(const __grid_constant__ CUtensorMap qmap,
                                                const __grid_constant__ CUtensorMap kmap,
                                                const __grid_constant__ CUtensorMap vmap, const PrefillArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int ns = item_streams(a);
  const int total = a.qtiles * (a.num_heads / ns) * a.batch;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  extern __shared__ uint8_t smem_raw[];
  PrefillSmem& sm =
      *reinterpret_cast<PrefillSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full_k[s], 1);
      mbar_init(&sm.k_empty[s], 1);
      mbar_init(&sm.full_v[s], 1);
      mbar_init(&sm.v_empty[s], 1);
    }
    for (int s = 0; s < kStreams; ++s) {
      mbar_init(&sm.q_full[s], 1);
      mbar_init(&sm.q_empty[s], 1);
      mbar_init(&sm.s_full[s], 1);
      mbar_init(&sm.p_lo[s], kStreamThreads);
      mbar_init(&sm.p_hi[s], kStreamThreads);
      mbar_init(&sm.o_ready[s], 1);
      mbar_init(&sm.o_free[s], kStreamThreads);
    }
    for (int i = 0; i < kItemRing; ++i) mbar_init(&sm.item_full[i], 1);
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
    }
    // Rows of an item that sees no key: zeros (two rows per warp instruction).
    auto zero_rows = [&](const Item& z) {
      const int rows = min(kRows, z.lq - z.qt * kRows);
      for (int s = 0; s < ns; ++s)
        for (int rr = lane >> 4; rr < rows; rr += 2) {
          __nv_bfloat16* row = a.out + (static_cast<int64_t>(z.q0 + z.qt * kRows + rr) * a.num_heads + z.h0 + s) * kD;
          *reinterpret_cast<uint4*>(row + (lane & 15) * 8) = make_uint4(0, 0, 0, 0);
        }
    };
    int w = blockIdx.x, qi = 0, g = 0, k_issued = 0, v_issued = 0;
    bool ok = true;
    while (true) {
      Item it;
      const bool have = next_item(a, w, total, it, zero_rows);
      if (lane == 0) {
        // The Q buffers, and with them the ring slot (read by every role
        // before the previous item's last S), are free once the previous
        // item's last S of each stream has completed.
        for (int s = 0; s < ns && ok && qi > 0; ++s)
          if (!mbar_wait(&sm.q_empty[s], (qi - 1) & 1)) ok = false;
        Item& slot = sm.items[qi % kItemRing];
        slot = it;
        if (!have || !ok) slot.n_kv = -1;
        mbar_arrive(&sm.item_full[qi % kItemRing]);
        if (have && ok) {
          for (int s = 0; s < ns; ++s) {
            mbar_arrive_expect_tx(&sm.q_full[s], kTileBytes);
            tma_load_3d(sm.q[s], &qmap, &sm.q_full[s], 0, it.h0 + s, it.q0 + it.qt * kRows);
            tma_load_3d(sm.q[s] + kHalfBytes, &qmap, &sm.q_full[s], 64, it.h0 + s, it.q0 + it.qt * kRows);
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!have || !ok) break;
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
            tma_load_3d(sm.k[st], &kmap, &sm.full_k[st], 0, it.kvh, row);
            tma_load_3d(sm.k[st] + kHalfBytes, &kmap, &sm.full_k[st], 64, it.kvh, row);
            ++k_issued;
            if (g >= kStages && !mbar_wait(&sm.v_empty[st], ((g / kStages) - 1) & 1)) {
              ok = false;
            } else {
              mbar_arrive_expect_tx(&sm.full_v[st], kTileBytes);
              tma_load_3d(sm.v[st], &vmap, &sm.full_v[st], 0, it.kvh, row);
              tma_load_3d(sm.v[st] + kHalfBytes, &vmap, &sm.full_v[st], 64, it.kvh, row);
              ++v_issued;
            }
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
      }
      ++qi;
      w += gridDim.x;
      if (!ok) break;
    }
    if (lane == 0) {
      if (!ok) flag_error(a, sm, kErrWaitTimeout);
      // Drain every copy this CTA issued before it may exit (a Q buffer is
      // reloaded only after its previous load was consumed, so only the last
      // load of each stream can be in flight).
      for (int s = 0; s < ns; ++s)
        if (qi > 0) (void)mbar_wait(&sm.q_full[s], (qi - 1) & 1);
      for (int j = max(0, k_issued - kStages); j < k_issued; ++j)
        (void)mbar_wait(&sm.full_k[j % kStages], (j / kStages) & 1);
      for (int j = max(0, v_issued - kStages); j < v_issued; ++j)
        (void)mbar_wait(&sm.full_v[j % kStages], (j / kStages) & 1);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------- MMA ----
    constexpr uint32_t idesc_qk = umma_idesc_bf16(kRows, kKeys, false);
    constexpr uint32_t idesc_pv = umma_idesc_bf16(kRows, kD, true);
    bool ok = true;
    auto wait_all = [](uint64_t* bar, uint32_t parity) { return __all_sync(0xffffffffu, mbar_wait(bar, parity)); };
    auto commit = [](uint64_t* bar) {
      if (elect_one_sync()) umma_commit(bar);
      __syncwarp();
    };
    auto issue_s = [&](int s, int st) {  // S_s = Q_s K(stage st)^T
      const uint32_t q_addr = smem_u32(sm.q[s]);
      const uint32_t k_addr = smem_u32(sm.k[st]);
#pragma unroll
      for (int kk = 0; kk < kD / 16; ++kk) {
        const uint32_t off = (kk >> 2) * kHalfBytes + (kk & 3) * 32;
        const uint64_t qa = smem_desc_sw128(q_addr + off, 16, 1024);
        const uint64_t kb = smem_desc_sw128(k_addr + off, 16, 1024);
        if (elect_one_sync()) umma_f16_ss(tmem + s * kKeys, qa, kb, idesc_qk, kk > 0);
        __syncwarp();
      }
      commit(&sm.s_full[s]);
    };
    // O_s (+)= P_s V(stage st) over the keys of 16-key steps kk0 .. kk0 + 3
    auto issue_pv = [&](int s, int st, int kk0, bool first) {
      const uint32_t v_addr = smem_u32(sm.v[st]);
#pragma unroll
      for (int kk = kk0; kk < kk0 + 4; ++kk) {
        const uint64_t vb = smem_desc_sw128(v_addr + kk * 16 * 128, kHalfBytes, 1024);
        if (elect_one_sync())
          umma_f16_ts(tmem + kColO + s * kD, tmem + s * kKeys + kk * 8, vb, idesc_pv, (!first || kk > 0) ? 1u : 0u);
        __syncwarp();
      }
    };
    int qi = 0, g = 0;
    while (ok) {
      if (!wait_all(&sm.item_full[qi % kItemRing], (qi / kItemRing) & 1)) { ok = false; break; }
      const Item it = sm.items[qi % kItemRing];
      if (it.n_kv < 0) break;
      // First S tiles of the item: behind the previous item's last P V in
      // issue order, so they overwrite its P only after it was read.
      {
        const int st = g % kStages;
        if (!wait_all(&sm.full_k[st], (g / kStages) & 1)) { ok = false; break; }
        for (int s = 0; s < ns && ok; ++s) {
          if (!wait_all(&sm.q_full[s], qi & 1)) { ok = false; break; }
          tc_fence_after();
          issue_s(s, st);
          if (it.n_kv == 1) commit(&sm.q_empty[s]);
        }
        if (!ok) break;
        commit(&sm.k_empty[st]);
      }
      for (int j = 0; j < it.n_kv && ok; ++j, ++g) {
        const int st = g % kStages, st1 = (g + 1) % kStages;
        const bool more = j + 1 < it.n_kv;
        if (!wait_all(&sm.full_v[st], (g / kStages) & 1) ||
            (more && !wait_all(&sm.full_k[st1], ((g + 1) / kStages) & 1))) {
          ok = false;
          break;
        }
        for (int s = 0; s < ns; ++s) {
          // the P V of the first 64 keys goes out while the softmax still
          // computes the exponentials of the other 64
          if (!wait_all(&sm.p_lo[s], g & 1) || (j == 0 && qi > 0 && !wait_all(&sm.o_free[s], (qi - 1) & 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(s, st, 0, j == 0);
          if (!wait_all(&sm.p_hi[s], g & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(s, st, 4, false);
          if (more) {
            issue_s(s, st1);
            if (j + 2 == it.n_kv) commit(&sm.q_empty[s]);  // the item's last S_s
          } else {
            commit(&sm.o_ready[s]);
          }
        }
        if (!ok) break;
        commit(&sm.v_empty[st]);
        if (more) commit(&sm.k_empty[st1]);
      }
      ++qi;
    }
    if (!ok && lane == 0) flag_error(a, sm, kErrWaitTimeout);
    // All MMAs of this CTA complete before TMEM is released.
    commit(&sm.fin);
    (void)mbar_wait(&sm.fin, 0);
  } else if ((warp >> 2) < ns) {
    // --------------------------------------------------------- softmax ----
    const int s = warp >> 2;
    const int r = tid & (kStreamThreads - 1);  // query row within the tile = TMEM lane
    const uint32_t t_lane = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tmem_s = tmem + s * kKeys + t_lane;
    const uint32_t tmem_o = tmem + kColO + s * kD + t_lane;
    const float sc = a.scale_log2;
    uint8_t* stage = sm.stage[s];
    int qi = 0, g = 0;
    bool ok = true;
    while (ok) {
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.item_full[qi % kItemRing], (qi / kItemRing) & 1))) {
        ok = false;
        break;
      }
      const Item it = sm.items[qi % kItemRing];
      if (it.n_kv < 0) break;
      const int i = it.qt * kRows + r;
      const int lim = (i < it.lq) ? (it.lk - it.lq + i) : (it.lk - 1);
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < it.n_kv; ++j, ++g) {
        // warp-uniform outcome: the tcgen05.ld/st below need a converged warp
        if (!__all_sync(0xffffffffu, mbar_wait(&sm.s_full[s], g & 1))) { ok = false; break; }
        tc_fence_after();
        const int kbase = j * kKeys;
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
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; e += 2) mx[c] = fmax3(mx[c], __uint_as_float(sr[c][e]), __uint_as_float(sr[c][e + 1]));
        const float mt = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * sc;
        const float m_new = fmaxf(m, mt);
        const bool resc = m_new > m + kRescaleThreshold;
        const float alpha = resc ? fast_exp2(m - m_new) : 1.f;
        if (resc) {
          l *= alpha;
          m = m_new;
        }
        const float neg_mu = (m == -INFINITY) ? 0.f : -m;
        float sum[4] = {0.f, 0.f, 0.f, 0.f};  // independent add chains
        // P over the first 64 columns of S_s (column k holds keys 2k and 2k+1
        // as a bf16 pair): word e of chunk c overwrites score e, already read.
        // Keys 0-63 are signalled first, so that their P V starts while the
        // exponentials of keys 64-127 are computed.
        auto exps = [&](int c) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float p0 = fast_exp2(fmaf(__uint_as_float(sr[c][2 * e]), sc, neg_mu));
            const float p1 = fast_exp2(fmaf(__uint_as_float(sr[c][2 * e + 1]), sc, neg_mu));
            sum[(2 * e) & 3] += p0;
            sum[(2 * e + 1) & 3] += p1;
            sr[c][e] = pack_bf16x2(p0, p1);
          }
          tmem_st16_first(tmem_s + c * 16, sr[c]);
        };
        exps(0);
        exps(1);
        // O_s rescales (rarely) before any P V of this tile: S_s(j) landed,
        // so P V_s(j-1) is complete.
        if (j > 0 && __any_sync(0xffffffffu, resc)) {
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
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&sm.p_lo[s]);
        exps(2);
        exps(3);
        l += (sum[0] + sum[1]) + (sum[2] + sum[3]);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&sm.p_hi[s]);
      }
      if (!ok) break;
      // The item's last P V_s complete: normalise the O_s rows and store them
      // through stage[s], one 64-dim half at a time: thread r writes its row
      // half there (16-byte chunk c of row r at chunk c ^ (r % 8): conflict
      // free), then its warp stores the 32 row halves its lanes wrote, four
      // whole 128-byte row halves per instruction, so the global writes are
      // coalesced and no warp waits for another.
      if (!__all_sync(0xffffffffu, mbar_wait(&sm.o_ready[s], qi & 1))) { ok = false; break; }
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int rows = min(kRows, it.lq - it.qt * kRows);
      const int row0 = (warp & 3) * 32;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t o[32];
          tmem_ld32(tmem_o + h * 64 + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const uint32_t x = pack_bf16x2(__uint_as_float(o[q4 * 8 + 0]) * inv, __uint_as_float(o[q4 * 8 + 1]) * inv);
            const uint32_t y = pack_bf16x2(__uint_as_float(o[q4 * 8 + 2]) * inv, __uint_as_float(o[q4 * 8 + 3]) * inv);
            const uint32_t z = pack_bf16x2(__uint_as_float(o[q4 * 8 + 4]) * inv, __uint_as_float(o[q4 * 8 + 5]) * inv);
            const uint32_t u = pack_bf16x2(__uint_as_float(o[q4 * 8 + 6]) * inv, __uint_as_float(o[q4 * 8 + 7]) * inv);
            const int chunk = c * 4 + q4;
            st_shared_v4(smem_u32(stage + r * 128 + ((chunk ^ (r & 7)) << 4)), x, y, z, u);
          }
        }
        if (h == 1) {  // O_s is read out: the next item's first P V_s may overwrite it
          tc_fence_before();
          mbar_arrive(&sm.o_free[s]);
        }
        __syncwarp();  // this warp's 32 row halves are in stage[s]
#pragma unroll 4
        for (int k = 0; k < 8; ++k) {
          const int row = row0 + k * 4 + (lane >> 3), c16 = lane & 7;
          if (row < rows) {
            const uint4 v4 = ld_shared_v4(smem_u32(stage + row * 128 + ((c16 ^ (row & 7)) << 4)));
            __nv_bfloat16* dst = a.out +
                                 (static_cast<int64_t>(it.q0 + it.qt * kRows + row) * a.num_heads + it.h0 + s) * kD +
                                 h * 64 + c16 * 8;
            *reinterpret_cast<uint4*>(dst) = v4;
          }
        }
        __syncwarp();  // read out before the next half overwrites the rows
      }
      if (!ok) break;
      ++qi;
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
  a.paired = (a.qpk % 2 == 0) ? 1 : 0;
  const int64_t items = static_cast<int64_t>(a.qtiles) * (a.num_heads / (a.paired ? kStreams : 1)) * a.batch;
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
