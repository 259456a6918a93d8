// Paged GQA decode attention (one query token per sequence) on the sm_100a
// tensor cores, as a persistent, continuously streaming kernel.
//
// Replaces torch_npu._npu_paged_attention as called from
// src/nanovllm_ascend/layers/npu_paged_attention.py:58,89 (and the graph
// task update at src/nanovllm_ascend/npu/acl_graph.py:232):
//   out[b,h] = softmax(scale * q[b,h] . K[b,:,g(h)]^T) . V[b,:,g(h)]
// over the first context_lens[b] tokens reached through block_tables[b].
//
// HBM-bound: every KV byte is read once. Design:
//  * work = 128-token tiles of every (sequence, KV head) pair, linearised
//    sequence-major. The grid is persistent (one CTA per SM); CTA c takes the
//    contiguous range [c*T/C, (c+1)*T/C) of the T tiles, so loads stream
//    without per-CTA fill/drain and the load balance is within one tile.
//    A range holds whole pairs ("segments") plus at most a partial pair at
//    each end; a pair split across CTAs is merged by the CTA that completes
//    it: a CTA that finds every other piece already published (acquire load
//    of the pair's ticket) fetches them while its own piece is computed and
//    merges in registers; otherwise it publishes its piece (two partial
//    slots per CTA, acq_rel ticket) and the last publisher merges.
//  * warp 11 (scheduler): scans the context lengths into the schedule and
//    walks the CTA's segments ahead of the producer: per segment a TMA load
//    of the group's QPK query rows into a zero-padded 16-row operand, per
//    chunk of tiles one parallel round of block-id loads into a ring, and
//    (fused append) the step's new K/V row before any copy of its tile. The
//    scan and the first chunk's ids come from step metadata and are done
//    before griddepcontrol.wait.
//  * warp 4 (producer): per tile, TMA loads of the K and V tile (box {64
//    dims, 1 head, <=32 tokens}, 128-byte swizzle, only the sub-boxes that
//    hold context tokens, L2 evict_first) into a 3-stage ring.
//  * warps 5 and 10 (MMA issuers, one elected thread each): warp 5 issues
//    S^T[128 tok x 16] = K[128 x 128] . Qpad^T (A and B K-major), warp 10
//    O^T[128 dims x 16] += V^T . P^T (A = the V tile read MN-major, B = P^T
//    K-major): M=128 N=16 K=16 UMMAs with f32 accumulators in TMEM (S double
//    buffered, O and the query operand four deep, so short segments do not
//    wait on each other), completion via tcgen05.commit. Two issuers keep the
//    S of later tiles flowing while PV waits for the softmax; the producer
//    publishes each tile's segment facts beside its K/V stage, so neither
//    issuer walks the schedule.
//  * warps 0-3 (softmax): thread t owns token t of S^T (and dim t of O^T).
//    Base-2 online softmax per query head with lazy rescaling (the reference
//    max moves only when a tile max exceeds it by more than 2^8); the tile
//    max is exchanged across the 4 warps once per tile; P^T goes to shared
//    memory as bf16; l is summed once per segment.
//  * warps 6-9 (epilogue): thread e owns dim e of O^T: per segment the
//    normalised output row (to every rank's output over NVLink in gather
//    mode), or the partial (numerator, max, denominator) of a split pair,
//    published for the merge.
// Every mbarrier wait is bounded (%globaltimer); a timeout sets the error
// word, the CTA drains its copies and MMAs, frees TMEM and exits.
#include <cfloat>
#include <mutex>

#include "host_common.h"
#include "nvk_common.cuh"
#include "tcgen05.cuh"

namespace nvk {
namespace {

constexpr int kD = 128;
constexpr int kTile = 128;          // tokens per tile
constexpr int kHalf = kTile * 128;  // one 64-dim half of a K or V tile
constexpr int kKV = 2 * kHalf;      // one K (or V) tile
constexpr int kStages = 3;
constexpr int kN = 16;              // UMMA N: the GQA group, zero padded
constexpr int kQHalf = kN * 128;    // 16 rows x 64 dims
constexpr int kQBytes = 2 * kQHalf;
constexpr int kMaxSeqs = 1024;      // sequences per launch (tile prefix in smem)
constexpr int kSoftmaxThreads = 128;
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;                 // issues S = K Q^T
constexpr int kEpilogueWarp0 = 6;           // warps 6-9: one per TMEM lane quarter
constexpr int kEpilogueThreads = 128;
constexpr int kPvWarp = 10;                 // issues O += V^T P^T
constexpr int kSchedWarp = 11;              // walks the schedule, stages block ids, loads queries
constexpr int kThreads = 12 * 32;
constexpr int kQBufs = 4;           // query operands in flight (one per segment)
constexpr int kOBufs = 4;           // O accumulators in flight (one per segment)
constexpr uint32_t kTmemCols = 128; // S: 0-31 (2 x 16), O: 32-95 (4 x 16)
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr int kChunkTiles = 32;            // most tiles per staged chunk of block ids
constexpr int kRingSlots = 4;              // staged chunks in flight between scheduler and producer
constexpr int kSlotIds = 64;               // block ids per chunk
constexpr int kMaxMergePieces = 32;        // pieces staged per merge pass
constexpr int kTicketStride = 32;          // ints: one 128-byte line per ticket (no shared lines)

struct DecodeArgs {
  __nv_bfloat16* out;
  const void* query;  // only warmed in L2 here; read through the tensor map
  const int32_t* block_tables;
  const int32_t* context_lens;
  float* ws_o;    // [C][2][QPK][kD] partial numerators
  float2* ws_ml;  // [C][2][QPK] partial (reference max, denominator)
  int* ws_cnt;    // [batch * KVH] arrival tickets, back at zero after every call
  int* err;
  int batch;
  int bt_stride;
  int max_blocks;
  int num_blocks;
  int block_size;
  int log2_bs;
  int sub_rows;
  int chunk_tiles;  // tiles per chunk: every chunk's block ids fit in kSlotIds
  // Output rows: (b, local query head h) goes to head head_offset + h of a
  // [batch, out_heads, 128] array -- `out`, or with world > 0 every rank's
  // gathered output peer_out[r] (see gather_signal).
  int out_heads, head_offset;
  int world, rank;
  __nv_bfloat16* peer_out[NVK_MAX_PEERS];
  uint32_t* peer_sig[NVK_MAX_PEERS];
  uint32_t* my_sig;
  int* done;  // CTAs finished this call (gather mode), back at zero after it
  // Gather mode timing, accumulated over calls in the workspace header:
  // [0] ns from CTA 0's release (griddepcontrol.wait) to the last CTA's
  // arrival, [1] ns the last CTA then waited for every rank's epoch,
  // [2] calls, [3] this call's release time (written by CTA 0).
  unsigned long long* timing;
  // Fused append (new_slots != nullptr): this step's token of sequence b,
  // rows k_new/v_new + b * stride (16-byte words, heads and dims packed), is
  // written to pool slot new_slots[b] before any of its tiles is read.
  const uint4* k_new;
  const uint4* v_new;
  int64_t k_new_stride_w, v_new_stride_w;
  const int64_t* new_slots;
  uint4* kc_words;
  uint4* vc_words;
  int64_t num_slots;
  int num_heads;
  int num_kv_heads;
  int qpk;
  float scale_log2;
};

// What the producer knows about the tile in a K/V stage, published with the
// stage's TMA transaction (written before the arrive that sets its byte count,
// read after a wait on that barrier) so that no other role walks segments.
enum TileFlags : int { kFirstTile = 1, kLastTile = 2 };
struct TileInfo {
  int seg;     // segment ordinal within this CTA
  int flags;   // kFirstTile / kLastTile of the segment
  int nvalid;  // context tokens in the tile (1..128)
  int b, g, n, ntiles, pair_t0, slot;
};

// One chunk of a segment (at most chunk_tiles tiles), staged by the scheduler
// warp for the producer: where it lies and its block ids. nt == 0 ends the walk.
struct Chunk {
  int seg, b, g, len, i, nt, seg_i0, seg_ntiles, n, pair_t0, slot, blk0;
  int ids[kSlotIds];
};

struct Smem {
  alignas(1024) uint8_t k[kStages][kKV];
  alignas(1024) uint8_t v[kStages][kKV];
  alignas(1024) uint8_t q[kQBufs][kQBytes];
  alignas(1024) uint8_t p[2][kQBytes];
  int tiles_before[kMaxSeqs + 1];
  uint8_t last_rows[kMaxSeqs];           // context tokens in each sequence's last tile (1..128)
  Chunk ring[kRingSlots];
  uint64_t ring_full[kRingSlots], ring_empty[kRingSlots];
  float red[2][4][8];
  int warp_ok[2][4];
  int resc_ok[4];  // rescale-path exchange (its own slot: warp_ok[] belongs to the tile)
  TileInfo info[kStages];
  uint64_t full_k[kStages], full_v[kStages], kv_empty[kStages];
  uint64_t q_full[kQBufs], q_empty[kQBufs];
  uint64_t s_full[2], s_free[2], p_full[2], pv_done[2];
  uint64_t o_full[kOBufs], o_empty[kOBufs];
  uint64_t fin;
  uint32_t tmem_base;
  int total_tiles;
  int b_lo, b_hi;  // sequences holding this CTA's first and last tile
  // softmax -> epilogue hand-off, one per O buffer
  struct SegInfo {
    int b, g, n, ntiles, pair_t0, slot;
    float m[8];
    float l_part[4][8];
  } seg_info[kOBufs];
  uint64_t seg_ready[kOBufs];
  int pre_last[2];  // per partial segment: every other piece of its pair was already published
  int last[2];      // per partial segment: this CTA's publish was the pair's last
  float2 mml[kMaxMergePieces * 8];          // (m, l) of the pieces being merged
  int epi_ok[4];
  volatile int abort;
};

__device__ __forceinline__ int seq_tiles(int len) { return (len + kTile - 1) / kTile; }

// The T tiles of a launch split into C contiguous ranges: CTA c gets
// q = T / C tiles, plus one more if c < r = T % C. Range starts and owners are
// then multiplications and one 32-bit divide by a per-launch constant (no
// 64-bit divisions on the critical path), and empty ranges (T < C) all sit at
// the end, so the CTAs holding pieces of one pair are contiguous.
struct Sched {
  int total, ctas, q, r, big;  // big = r * (q + 1): tiles held by the longer ranges
};

__device__ __forceinline__ Sched make_sched(int total, int ctas) {
  Sched sc;
  sc.total = total;
  sc.ctas = ctas;
  sc.q = total / ctas;
  sc.r = total - sc.q * ctas;
  sc.big = sc.r * (sc.q + 1);
  return sc;
}

__device__ __forceinline__ int range_lo(int c, const Sched& sc) { return c * sc.q + min(c, sc.r); }

// CTA whose range holds linear tile t.
__device__ __forceinline__ int cta_of(int t, const Sched& sc) {
  return t < sc.big ? t / (sc.q + 1) : sc.r + (t - sc.big) / max(sc.q, 1);  // q >= 1 whenever t >= big
}

// Partial slot of CTA cc for a pair starting at pair_t0: 0 when the pair is
// the first segment of cc's range (the range starts inside the pair), else 1.
__device__ __forceinline__ int64_t part_index(int cc, int pair_t0, const Sched& sc, int qpk) {
  const int slot = (range_lo(cc, sc) >= pair_t0) ? 0 : 1;
  return (static_cast<int64_t>(cc) * 2 + slot) * qpk;
}

// One contiguous run of tiles of one (sequence, KV head) pair inside this CTA.
struct Segment {
  int b, g, len, i0, n, ntiles, pair_t0, start;
};

// The segment of sequence b (which must hold tile t) that starts at tile t
// and ends at its pair's end or at hi.
__device__ __forceinline__ Segment make_segment(const Smem& sm, const DecodeArgs& a, int b, int t, int hi) {
  Segment s;
  s.b = b;
  s.n = sm.tiles_before[b + 1] - sm.tiles_before[b];
  const int off = t - a.num_kv_heads * sm.tiles_before[b];
  s.g = off / s.n;
  s.i0 = off - s.g * s.n;
  s.ntiles = min(hi - t, s.n - s.i0);
  s.pair_t0 = t - s.i0;
  s.start = t;
  s.len = (s.n - 1) * kTile + sm.last_rows[b];  // a segment exists only when s.n >= 1
  return s;
}

// Order in which a CTA walks its range [lo, hi): first the (at most two)
// partial segments -- pieces of pairs shared with the neighbouring CTAs --
// then the whole pairs. Both pieces of every split pair are thus finished
// early in every CTA, and their merge overlaps the streaming of whole pairs
// instead of trailing the kernel. Every role follows the same order.
// The sequences holding tiles lo and hi-1 come from the schedule scan, and
// whole pairs follow one another, so no step searches.
struct SegIter {
  int lo, hi;
  int f_b, l_b, s1;  // sequences holding tiles lo and hi-1; start of the last segment
  int cb, cg, ct;    // whole-pair cursor: pair (cb, cg) starts at tile ct ...
  int m1;            // ... and whole pairs end at tile m1
  int phase, npartial;
  bool f_emit, l_emit;

  __device__ __forceinline__ void init(const Smem& sm, const DecodeArgs& a, int lo_, int hi_) {
    lo = lo_;
    hi = hi_;
    phase = 0;
    npartial = 0;
    f_emit = l_emit = false;
    ct = m1 = hi;
    f_b = l_b = s1 = cb = cg = 0;
    if (lo >= hi) return;
    f_b = sm.b_lo;
    const Segment f = make_segment(sm, a, f_b, lo, hi);
    const int e0 = lo + f.ntiles;
    if (e0 >= hi) {  // a single segment
      f_emit = true;
      npartial = (f.ntiles != f.n) ? 1 : 0;
      return;
    }
    l_b = sm.b_hi;
    const Segment l = make_segment(sm, a, l_b, hi - 1, hi);
    s1 = max(e0, l.pair_t0);  // start of the last segment
    f_emit = f.ntiles != f.n;
    l_emit = (hi - s1) != l.n;
    npartial = int(f_emit) + int(l_emit);
    ct = f_emit ? e0 : lo;
    m1 = l_emit ? s1 : hi;
    cb = f_b;
    cg = f.g;
    if (f_emit && ct < m1) advance(sm, a.num_kv_heads);
  }

  // Next pair in linear order (one exists: the cursor is below m1).
  __device__ __forceinline__ void advance(const Smem& sm, int kvh) {
    if (++cg == kvh) {
      cg = 0;
      do {
        ++cb;
      } while (sm.tiles_before[cb + 1] == sm.tiles_before[cb]);  // sequences without tiles own no pair
    }
  }

  __device__ __forceinline__ bool next(const Smem& sm, const DecodeArgs& a, Segment& s) {
    if (phase == 0) {
      phase = 1;
      if (f_emit) {
        s = make_segment(sm, a, f_b, lo, hi);
        return true;
      }
    }
    if (phase == 1) {
      phase = 2;
      if (l_emit) {
        s = make_segment(sm, a, l_b, s1, hi);
        return true;
      }
    }
    if (ct >= m1) return false;
    s.b = cb;
    s.g = cg;
    s.n = sm.tiles_before[cb + 1] - sm.tiles_before[cb];
    s.len = (s.n - 1) * kTile + sm.last_rows[cb];
    s.i0 = 0;
    s.ntiles = s.n;
    s.pair_t0 = ct;
    s.start = ct;
    ct += s.n;
    if (ct < m1) advance(sm, a.num_kv_heads);
    return true;
  }
};

// Stores output element d of (sequence b, local query head qh). In gather
// mode into this rank's own gathered output; push_rows then copies whole
// rows to the other ranks.
__device__ __forceinline__ void store_out(const DecodeArgs& a, int b, int qh, int d, float v) {
  const int64_t off = (static_cast<int64_t>(b) * a.out_heads + a.head_offset + qh) * kD + d;
  const __nv_bfloat16 x = __float2bfloat16_rn(v);
  if (a.world == 0) {
    a.out[off] = x;
    return;
  }
  a.peer_out[a.rank][off] = x;
}

// Gather mode: the rows (sequence b, local query heads h0 .. h0 + nh - 1),
// which the 128 epilogue threads have just stored into this rank's output
// (ordered by the named barrier the caller took), copied to every other
// rank's output over NVLink, 16 bytes a store (the rows are contiguous).
__device__ __forceinline__ void push_rows(const DecodeArgs& a, int b, int h0, int nh, int e) {
  const int64_t off = (static_cast<int64_t>(b) * a.out_heads + a.head_offset + h0) * kD;
  const int chunks = nh * (kD * 2 / 16);
  const uint4* src = reinterpret_cast<const uint4*>(a.peer_out[a.rank] + off);
  for (int i = e; i < (a.world - 1) * chunks; i += kEpilogueThreads) {
    const int p = i / chunks, k = i - p * chunks;
    const int r = p < a.rank ? p : p + 1;  // every rank but this one
    reinterpret_cast<uint4*>(a.peer_out[r] + off)[k] = src[k];
  }
}

constexpr int kEpochSlot = NVK_MAX_PEERS;  // signal word holding this rank's call count

// Completion of the in-kernel gather (thread 0 of every CTA, after the CTA's
// last output store): each CTA fences its stores at system scope and takes a
// ticket; the last CTA posts this call's epoch to every rank's signal area and
// waits until every rank has posted the same epoch to ours. Then every rank's
// rows of this call are in our buffer when the kernel completes. The wait is
// bounded (kWaitLimitNs -> kErrPeerTimeout).
__device__ __forceinline__ void gather_signal(const DecodeArgs& a, int ctas) {
  __threadfence_system();
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(a.done) : "memory");
  if (old != ctas - 1) return;
  __threadfence_system();
  *a.done = 0;  // for the next call, which the kernel boundary orders after this one
  const uint32_t epoch = a.my_sig[kEpochSlot] + 1;
  a.my_sig[kEpochSlot] = epoch;
  // The fence above already publishes every CTA's rows at system scope, so
  // the flags go out as relaxed stores: a release store per rank would carry
  // a system-scope fence of its own each (at 8 ranks ~12 us per launch).
#pragma unroll
  for (int r = 0; r < NVK_MAX_PEERS; ++r)
    if (r < a.world) st_relaxed_sys(a.peer_sig[r] + a.rank, epoch);
  const uint64_t t0 = globaltimer_ns();
  for (int r = 0; r < a.world; ++r) {
    while (static_cast<int>(ld_acquire_sys(a.my_sig + r) - epoch) < 0) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        atomicOr(a.err, kErrPeerTimeout);
        return;
      }
    }
  }
  // (CTA 0's release time is ordered before this by the acq_rel ticket)
  a.timing[0] += t0 - a.timing[3];
  a.timing[1] += globaltimer_ns() - t0;
  a.timing[2] += 1;
}

__device__ __forceinline__ void flag_error(const DecodeArgs& a, Smem& sm, int code) {
  atomicOr(a.err, code);
  sm.abort = 1;
}

// QPK consecutive 32-bit TMEM columns of this thread's lane (warp-collective).
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, int qpk, float (&v)[8]) {
  uint32_t r[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (qpk == 1) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r[0]) : "r"(taddr));
  } else if (qpk == 2) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(taddr));
  } else if (qpk == 4) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
  } else {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                   "=r"(r[7])
                 : "r"(taddr));
  }
  tmem_ld_wait();
#pragma unroll
  for (int h = 0; h < 8; ++h) v[h] = __uint_as_float(r[h]);
}

__device__ __forceinline__ void tmem_st_cols(uint32_t taddr, int qpk, const float (&v)[8]) {
  uint32_t r[8];
#pragma unroll
  for (int h = 0; h < 8; ++h) r[h] = __float_as_uint(v[h]);
  if (qpk == 1) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(r[0]) : "memory");
  } else if (qpk == 2) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x2.b32 [%0], {%1, %2};" ::"r"(taddr), "r"(r[0]), "r"(r[1])
                 : "memory");
  } else if (qpk == 4) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3])
                 : "memory");
  } else {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
  }
  tmem_st_wait();
}

constexpr int kFastPieces = 4;  // other pieces of a pair fetched in one round of loads

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Merges pair (b, g), split over the CTAs c_first .. c_first + pieces - 1,
// from the published partials of every piece (this CTA's included) and
// resets its ticket. Called by the 128 epilogue threads of the CTA whose
// publish was the pair's last (thread e owns dim d).
template <int QPK>
__device__ __forceinline__ void merge_published(Smem& sm, const DecodeArgs& a, const Sched& sc, int e, int d, int b,
                                                int g, int pair_t0, int c_first, int pieces, int* ticket) {
  if (pieces <= kFastPieces) {
    float2 ml[kFastPieces][QPK];
    float ov[kFastPieces][QPK];
#pragma unroll
    for (int u = 0; u < kFastPieces; ++u) {
#pragma unroll
      for (int h = 0; h < QPK; ++h) {
        const bool use = u < pieces;
        const int64_t pp = use ? part_index(c_first + u, pair_t0, sc, QPK) + h : 0;
        ml[u][h] = use ? __ldcg(&a.ws_ml[pp]) : make_float2(-INFINITY, 0.f);
        ov[u][h] = use ? __ldcg(&a.ws_o[pp * kD + d]) : 0.f;
      }
    }
#pragma unroll
    for (int h = 0; h < QPK; ++h) {
      float M = -INFINITY;
#pragma unroll
      for (int u = 0; u < kFastPieces; ++u) M = fmaxf(M, ml[u][h].x);
      float num = 0.f, den = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int u = 0; u < kFastPieces; ++u) {
          if (ml[u][h].x == -INFINITY) continue;
          const float w = fast_exp2(ml[u][h].x - M);
          num = fmaf(w, ov[u][h], num);
          den = fmaf(w, ml[u][h].y, den);
        }
      }
      store_out(a, b, g * QPK + h, d, den > 0.f ? num / den : 0.f);
    }
  } else {
    // Many pieces (a long pair over many CTAs): staged passes through smem.
    float num[QPK], den[QPK], M[QPK];
#pragma unroll
    for (int h = 0; h < QPK; ++h) {
      num[h] = 0.f;
      den[h] = 0.f;
      M[h] = -INFINITY;
    }
    for (int c0 = c_first; c0 < c_first + pieces; c0 += kMaxMergePieces) {
      const int n = min(kMaxMergePieces, c_first + pieces - c0);
      for (int r = e; r < n * QPK; r += kEpilogueThreads)
        sm.mml[r] = __ldcg(&a.ws_ml[part_index(c0 + r / QPK, pair_t0, sc, QPK) + (r % QPK)]);
      named_barrier_sync(2, kEpilogueThreads);
#pragma unroll
      for (int h = 0; h < QPK; ++h) {
        float mg = M[h];
        for (int p = 0; p < n; ++p) mg = fmaxf(mg, sm.mml[p * QPK + h].x);
        const float s_old = (M[h] == -INFINITY) ? 0.f : fast_exp2(M[h] - mg);
        num[h] *= s_old;
        den[h] *= s_old;
        M[h] = mg;
        for (int p = 0; p < n; ++p) {
          const float2 ml = sm.mml[p * QPK + h];
          if (ml.x == -INFINITY) continue;
          const float w = fast_exp2(ml.x - mg);
          num[h] = fmaf(w, __ldcg(&a.ws_o[(part_index(c0 + p, pair_t0, sc, QPK) + h) * kD + d]), num[h]);
          den[h] = fmaf(w, ml.y, den[h]);
        }
      }
      named_barrier_sync(2, kEpilogueThreads);  // staging is rewritten by the next group
    }
#pragma unroll
    for (int h = 0; h < QPK; ++h) store_out(a, b, g * QPK + h, d, den[h] > 0.f ? num[h] / den[h] : 0.f);
  }
  if (e == 0) *ticket = 0;  // every piece has arrived: ready for the next call
}

template <int QPK>
__global__ void __launch_bounds__(kThreads, 1) paged_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                                                                   const __grid_constant__ CUtensorMap vmap,
                                                                   const __grid_constant__ CUtensorMap qmap,
                                                                   const DecodeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, ctas = gridDim.x;
  const int kvh = a.num_kv_heads;

  if (tid == 32) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full_k[s], 1);
      mbar_init(&sm.full_v[s], 1);
      mbar_init(&sm.kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.s_free[i], kSoftmaxThreads);
      mbar_init(&sm.p_full[i], kSoftmaxThreads);
      mbar_init(&sm.pv_done[i], 1);
    }
    for (int i = 0; i < kQBufs; ++i) {
      mbar_init(&sm.q_full[i], 1);
      mbar_init(&sm.q_empty[i], 1);
    }
    for (int i = 0; i < kOBufs; ++i) {
      mbar_init(&sm.o_full[i], 1);
      mbar_init(&sm.o_empty[i], kEpilogueThreads);
      mbar_init(&sm.seg_ready[i], kSoftmaxThreads);
    }
    for (int i = 0; i < kRingSlots; ++i) {
      mbar_init(&sm.ring_full[i], 32);  // every scheduler lane, after its own id stores
      mbar_init(&sm.ring_empty[i], 1);
    }
    mbar_init(&sm.fin, 2);  // one commit from each MMA-issuing thread
    sm.abort = 0;
    fence_mbar_init();
  }
  // Zero the padded Q and P operands once (rows >= QPK are never written).
  for (int i = tid; i < kQBufs * kQBytes / 16; i += kThreads) reinterpret_cast<uint4*>(sm.q[0])[i] = make_uint4(0, 0, 0, 0);
  for (int i = tid; i < 2 * kQBytes / 16; i += kThreads) reinterpret_cast<uint4*>(sm.p[0])[i] = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();
  if (warp == kMmaWarp) {
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  pdl_launch_dependents();
  // Programmatic dependent launch: context_lens and block_tables are step
  // metadata written before the step's first kernel (host copies, or a
  // metadata kernel that does not trigger its dependents early), so the
  // schedule and the first chunk's block ids are computed before
  // griddepcontrol.wait, while the predecessor drains. Everything the predecessor may write (queries, new K/V rows, the
  // pool, outputs, workspace) is touched only after each warp's own wait.
  {
    const int64_t bt_bytes = (int64_t(a.batch - 1) * a.bt_stride + a.max_blocks) * 4;
    prefetch_l2_range(a.block_tables, bt_bytes, c, ctas, tid, kThreads);
    prefetch_l2_range(a.query, int64_t(a.batch) * a.num_heads * kD * 2, c, ctas, tid, kThreads);
  }
  // ---- per-sequence tile prefix: every CTA derives the same schedule ----
  // All lengths are loaded at once (one round trip), then warp 0 scans them
  // in place.
  for (int b = tid; b < a.batch; b += kThreads) sm.tiles_before[b] = a.context_lens[b];
  __syncthreads();
  if (warp == 0) {
    int carry = 0;
    for (int base = 0; base < a.batch; base += 32) {
      const int b = base + lane;
      int n = 0;
      if (b < a.batch) {
        int len = sm.tiles_before[b];
        if (len > a.max_blocks * a.block_size) {
          if (c == 0) atomicOr(a.err, kErrContextTooLong);
          len = a.max_blocks * a.block_size;
        }
        len = max(len, 0);
        n = seq_tiles(len);
        sm.last_rows[b] = static_cast<uint8_t>(len - (n - 1) * kTile);  // unused when n == 0
      }
      int incl = n;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += y;
      }
      if (b < a.batch) sm.tiles_before[b] = carry + incl - n;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      sm.tiles_before[a.batch] = carry;
      sm.total_tiles = carry * kvh;
    }
    // Sequences holding this CTA's first and last tile: the largest b with
    // kvh * tiles_before[b] <= t is the count of such b, less one.
    __syncwarp();
    const int total = carry * kvh;
    if (total > 0) {
      const Sched sc0 = make_sched(total, ctas);
      const int t_lo = range_lo(c, sc0), t_hi = range_lo(c + 1, sc0) - 1;
      int n_lo = 0, n_hi = 0;
      for (int b = lane; b < a.batch; b += 32) {
        const int v = kvh * sm.tiles_before[b];
        n_lo += (v <= t_lo) ? 1 : 0;
        n_hi += (v <= t_hi) ? 1 : 0;
      }
      n_lo = __reduce_add_sync(0xffffffffu, n_lo);
      n_hi = __reduce_add_sync(0xffffffffu, n_hi);
      if (lane == 0) {
        sm.b_lo = max(n_lo - 1, 0);
        sm.b_hi = max(n_hi - 1, 0);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp != kSchedWarp) pdl_wait();  // the scheduler waits after staging its first chunk
  if (a.world > 0 && c == 0 && tid == 0) a.timing[3] = globaltimer_ns();

  const int total = sm.total_tiles;
  const Sched sc = make_sched(total, ctas);
  const int lo = total > 0 ? range_lo(c, sc) : 0;
  const int hi = total > 0 ? range_lo(c + 1, sc) : 0;
  const uint32_t tmem = sm.tmem_base;

  if (warp == kSchedWarp) {
    // ------------------------------------------------------- scheduler ----
    // Walks this CTA's segments ahead of the producer: per segment the TMA
    // load of the group's query rows; per chunk of tiles, one parallel round
    // of block-id loads into a ring slot. The producer then only issues K/V
    // copies, so no segment start waits on a global round trip.
    if (lane == 0) tma_prefetch_desc(&qmap);
    int chunk = 0, seg = 0;
    bool ok = true, waited = false;
    SegIter it;
    it.init(sm, a, lo, hi);
    Segment s;
    auto load_q = [&](int sg, const Segment& sq) {  // lane 0
      const int qb = sg % kQBufs;
      if (sg >= kQBufs && !mbar_wait(&sm.q_empty[qb], ((sg / kQBufs) - 1) & 1)) ok = false;
      if (ok) {
        mbar_arrive_expect_tx(&sm.q_full[qb], static_cast<uint32_t>(2 * QPK * 128));
        tma_load_3d(sm.q[qb], &qmap, &sm.q_full[qb], 0, sq.g * QPK, sq.b);
        tma_load_3d(sm.q[qb] + kQHalf, &qmap, &sm.q_full[qb], 64, sq.g * QPK, sq.b);
      }
    };
    auto claim = [&](int ch) -> bool {  // ring slot of chunk ch is free
      if (ch < kRingSlots) return true;
      return __all_sync(0xffffffffu, mbar_wait(&sm.ring_empty[ch % kRingSlots], ((ch / kRingSlots) - 1) & 1));
    };
    for (; ok && it.next(sm, a, s); ++seg) {
      if (waited && lane == 0) load_q(seg, s);  // the first segment's query: after the wait below
      ok = __shfl_sync(0xffffffffu, ok, 0);
      const int32_t* bt = a.block_tables + static_cast<int64_t>(s.b) * a.bt_stride;
      for (int i = s.i0; ok && i < s.i0 + s.ntiles; i += a.chunk_tiles, ++chunk) {
        if (!claim(chunk)) {
          ok = false;
          break;
        }
        Chunk& ck = sm.ring[chunk % kRingSlots];
        const int nt = min(a.chunk_tiles, s.i0 + s.ntiles - i);
        const int blk0 = (i * kTile) >> a.log2_bs;
        const int blk1 = (min((i + nt) * kTile, s.len) - 1) >> a.log2_bs;  // inclusive, blk1 - blk0 < kSlotIds
        for (int k = lane; k <= blk1 - blk0; k += 32) {
          int blk = bt[blk0 + k];
          if (blk < 0 || blk >= a.num_blocks) {
            atomicOr(a.err, kErrBadBlockId);
            blk = a.num_blocks;  // fully outside the tensor map: zero fill
          }
          ck.ids[k] = blk;
        }
        if (!waited) {
          // First chunk: its ids are staged from step metadata; now wait for
          // the predecessor before the query copy and the fused append.
          __syncwarp();
          pdl_wait();
          waited = true;
          if (lane == 0) load_q(seg, s);
          ok = __shfl_sync(0xffffffffu, ok, 0);
        }
        if (lane == 0) {
          ck.seg = seg;
          ck.b = s.b;
          ck.g = s.g;
          ck.len = s.len;
          ck.i = i;
          ck.nt = nt;
          ck.seg_i0 = s.i0;
          ck.seg_ntiles = s.ntiles;
          ck.n = s.n;
          ck.pair_t0 = s.pair_t0;
          ck.slot = (s.start == lo) ? 0 : 1;
          ck.blk0 = blk0;
        }
        if (a.new_slots != nullptr && i + nt == s.n) {
          // Fused append: this chunk holds the pair's last tile, which only
          // this CTA reads, so it writes the new token's row of head s.g
          // first (K by lanes 0-15, V by lanes 16-31, 16 bytes each). The
          // slot must be the sequence's last context position.
          __syncwarp();  // ck.ids written by every lane
          const int last = s.len - 1;
          const int blk = ck.ids[(last >> a.log2_bs) - blk0];
          const int64_t want = static_cast<int64_t>(blk) * a.block_size + (last & (a.block_size - 1));
          const int64_t slot = a.new_slots[s.b];
          if (slot == want && blk < a.num_blocks) {
            const int w = s.g * (kD * 2 / 16) + (lane & 15);
            const int64_t row = slot * kvh * (kD * 2 / 16) + w;
            if (lane < 16) a.kc_words[row] = a.k_new[s.b * a.k_new_stride_w + w];
            else a.vc_words[row] = a.v_new[s.b * a.v_new_stride_w + w];
          } else if (lane == 0) {
            atomicOr(a.err, kErrBadSlot);
          }
          fence_proxy_async_global();  // the producer's TMA copies of this tile come after the ring arrive
        }
        mbar_arrive(&sm.ring_full[chunk % kRingSlots]);
      }
    }
    // End marker (skipped when a wait failed: the producer's own wait then
    // runs out and it stops too).
    if (ok && claim(chunk)) {
      if (lane == 0) sm.ring[chunk % kRingSlots].nt = 0;
      mbar_arrive(&sm.ring_full[chunk % kRingSlots]);
    }
    if (lane == 0) {
      if (!ok) flag_error(a, sm, kErrWaitTimeout);
      // Drain: every query copy lands before the CTA may exit.
      for (int sg = max(0, seg - kQBufs); sg < seg; ++sg) (void)mbar_wait(&sm.q_full[sg % kQBufs], (sg / kQBufs) & 1);
    }
  } else if (warp == kProducerWarp) {
    // -------------------------------------------------------- producer ----
    // Lane 0 turns each staged chunk into K and V tile copies (one per
    // sub-box holding context tokens) and publishes each tile's segment
    // facts with its stage.
    if (lane == 0) {
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
      // K/V are read exactly once per launch: keep them from evicting the
      // workspace partials, block tables and queries other CTAs still need.
      const uint64_t stream_policy = l2_policy_evict_first();
      int j = 0;
      bool ok = true;
      for (int chunk = 0; ok; ++chunk) {
        const int rs = chunk % kRingSlots;
        if (!mbar_wait(&sm.ring_full[rs], (chunk / kRingSlots) & 1)) {
          ok = false;
          break;
        }
        const Chunk& ck = sm.ring[rs];
        const int nt = ck.nt;
        if (nt == 0) break;
        const int seg = ck.seg, b = ck.b, g = ck.g, len = ck.len, seg_i0 = ck.seg_i0, seg_last = ck.seg_i0 + ck.seg_ntiles - 1;
        const int blk0 = ck.blk0;
        for (int ii = ck.i; ii < ck.i + nt; ++ii, ++j) {
          const int st = j % kStages;
          if (j >= kStages && !mbar_wait(&sm.kv_empty[st], ((j / kStages) - 1) & 1)) {
            ok = false;
            break;
          }
          const int tok0 = ii * kTile;
          const int nvalid = min(kTile, len - tok0);
          const int nsub = (nvalid + a.sub_rows - 1) / a.sub_rows;
          const uint32_t bytes = static_cast<uint32_t>(nsub * a.sub_rows * 128 * 2);
          TileInfo& ti = sm.info[st];
          ti.seg = seg;
          ti.flags = (ii == seg_i0 ? kFirstTile : 0) | (ii == seg_last ? kLastTile : 0);
          ti.nvalid = nvalid;
          ti.b = b;
          ti.g = g;
          ti.n = ck.n;
          ti.ntiles = ck.seg_ntiles;
          ti.pair_t0 = ck.pair_t0;
          ti.slot = ck.slot;
          mbar_arrive_expect_tx(&sm.full_k[st], bytes);
          mbar_arrive_expect_tx(&sm.full_v[st], bytes);
          for (int u = 0; u < nsub; ++u) {
            const int tok = tok0 + u * a.sub_rows;
            const int blk = ck.ids[(tok >> a.log2_bs) - blk0];
            const int row = blk * a.block_size + (tok & (a.block_size - 1));
            const int off = u * a.sub_rows * 128;
            tma_load_3d_hint(sm.k[st] + off, &kmap, &sm.full_k[st], 0, g, row, stream_policy);
            tma_load_3d_hint(sm.k[st] + kHalf + off, &kmap, &sm.full_k[st], 64, g, row, stream_policy);
            tma_load_3d_hint(sm.v[st] + off, &vmap, &sm.full_v[st], 0, g, row, stream_policy);
            tma_load_3d_hint(sm.v[st] + kHalf + off, &vmap, &sm.full_v[st], 64, g, row, stream_policy);
          }
        }
        mbar_arrive(&sm.ring_empty[rs]);  // the chunk's ids are no longer read
      }
      if (!ok) flag_error(a, sm, kErrWaitTimeout);
      // Drain: every copy this CTA issued lands before the CTA may exit.
      for (int jj = max(0, j - kStages); jj < j; ++jj) {
        (void)mbar_wait(&sm.full_k[jj % kStages], (jj / kStages) & 1);
        (void)mbar_wait(&sm.full_v[jj % kStages], (jj / kStages) & 1);
      }
    }
  } else if (warp == kMmaWarp) {
    // -------------------------------------------------------- MMA: S ----
    // S^T(j) = K(j) Qpad^T into S buffer j % 2, as soon as K(j) has landed and
    // the softmax has read S(j-2). Runs ahead of the PV issuer.
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_bf16(kTile, kN, false);  // A = K, B = Qpad
      bool ok = true;
      for (int j = 0; j < hi - lo; ++j) {
        const int st = j % kStages, sb = j & 1;
        if (!mbar_wait(&sm.full_k[st], (j / kStages) & 1)) {
          ok = false;
          break;
        }
        const int seg = sm.info[st].seg, flags = sm.info[st].flags;
        const int qb = seg % kQBufs;
        if (((flags & kFirstTile) && !mbar_wait(&sm.q_full[qb], (seg / kQBufs) & 1)) ||
            (j >= 2 && !mbar_wait(&sm.s_free[sb], ((j >> 1) - 1) & 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sm.k[st]);
        const uint32_t q_addr = smem_u32(sm.q[qb]);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t koff = (kk >> 2) * kHalf + (kk & 3) * 32;
          const uint32_t qoff = (kk >> 2) * kQHalf + (kk & 3) * 32;
          umma_f16_ss(tmem + sb * kN, smem_desc_sw128(k_addr + koff, 16, 1024),
                      smem_desc_sw128(q_addr + qoff, 16, 1024), idesc_s, kk > 0);
        }
        umma_commit(&sm.s_full[sb]);
        if (flags & kLastTile) umma_commit(&sm.q_empty[qb]);  // the segment's query is no longer read
      }
      if (!ok) flag_error(a, sm, kErrWaitTimeout);
      umma_commit(&sm.fin);
      (void)mbar_wait(&sm.fin, 0);  // every MMA of both issuers completes before TMEM is freed
    }
  } else if (warp == kPvWarp) {
    // ------------------------------------------------------- MMA: PV ----
    // O^T(seg) += V(j)^T P^T(j) once the softmax has written P(j). Its commit
    // frees the K/V stage: P(j) exists only after S(j), hence K(j), is done.
    if (lane == 0) {
      constexpr uint32_t idesc_o = umma_idesc_bf16(kD, kN, false) | (1u << 15);  // A = V^T (MN-major), B = P^T
      bool ok = true;
      for (int j = 0; j < hi - lo; ++j) {
        const int st = j % kStages, sb = j & 1;
        if (!mbar_wait(&sm.p_full[sb], (j >> 1) & 1) || !mbar_wait(&sm.full_v[st], (j / kStages) & 1)) {
          ok = false;
          break;
        }
        const int seg = sm.info[st].seg, flags = sm.info[st].flags;
        const int ob = seg % kOBufs;
        if ((flags & kFirstTile) && seg >= kOBufs && !mbar_wait(&sm.o_empty[ob], ((seg / kOBufs) - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sm.v[st]);
        const uint32_t p_addr = smem_u32(sm.p[sb]);
        const uint32_t o_tmem = tmem + 32 + ob * kN;
        const uint32_t acc0 = (flags & kFirstTile) ? 0u : 1u;
#pragma unroll
        for (int kk = 0; kk < kTile / 16; ++kk) {
          const uint64_t va = smem_desc_sw128(v_addr + kk * 16 * 128, kHalf, 1024);
          const uint64_t pb = smem_desc_sw128(p_addr + (kk >> 2) * kQHalf + (kk & 3) * 32, 16, 1024);
          umma_f16_ss(o_tmem, va, pb, idesc_o, kk > 0 ? 1u : acc0);
        }
        umma_commit(&sm.kv_empty[st]);
        umma_commit(&sm.pv_done[sb]);
        if (flags & kLastTile) umma_commit(&sm.o_full[ob]);
      }
      if (!ok) flag_error(a, sm, kErrWaitTimeout);
      umma_commit(&sm.fin);
    }
  } else if (warp < 4) {
    // --------------------------------------------------------- softmax ----
    const uint32_t t_lane = static_cast<uint32_t>(warp * 32) << 16;
    bool all_ok = true;
    float m_ref[QPK], l_t[QPK];
#pragma unroll
    for (int h = 0; h < QPK; ++h) {
      m_ref[h] = -INFINITY;
      l_t[h] = 0.f;
    }
    for (int j = 0; j < hi - lo; ++j) {
      const int st = j % kStages, sb = j & 1, rb = j & 1;
      // K(j) landed (and with it the tile info); S(j) ready; P buffer sb free
      // (PV(j-2) done); V(j) landed when rows past the context must be zeroed.
      bool ok = mbar_wait(&sm.full_k[st], (j / kStages) & 1) && mbar_wait(&sm.s_full[sb], (j >> 1) & 1);
      if (j >= 2) ok = ok && mbar_wait(&sm.pv_done[sb], ((j - 2) >> 1) & 1);
      TileInfo ti{};
      if (ok) ti = sm.info[st];  // read before p_full(j): the stage is refilled only after PV(j)
      if (ok && ti.nvalid < kTile) ok = mbar_wait(&sm.full_v[st], (j / kStages) & 1);
      ok = __all_sync(0xffffffffu, ok);  // tcgen05.ld below needs a converged warp
      const bool first = (ti.flags & kFirstTile) != 0;
      const int ob = ti.seg % kOBufs;
      const uint32_t o_tmem = tmem + 32 + ob * kN + t_lane;
      const bool valid = tid < ti.nvalid;
      if (first) {
#pragma unroll
        for (int h = 0; h < QPK; ++h) {
          m_ref[h] = -INFINITY;
          l_t[h] = 0.f;
        }
      }
      float sv8[8];
      float sv[QPK];
      if (ok) {
        tc_fence_after();
        tmem_ld_cols(tmem + sb * kN + t_lane, QPK, sv8);
        tc_fence_before();
        mbar_arrive(&sm.s_free[sb]);
      }
#pragma unroll
      for (int h = 0; h < QPK; ++h) {
        sv[h] = (ok && valid) ? sv8[h] * a.scale_log2 : -INFINITY;
        float x = sv[h];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, off));
        if (lane == 0) sm.red[rb][warp][h] = x;
      }
      if (lane == 0) sm.warp_ok[rb][warp] = ok;
      named_barrier_sync(1, kSoftmaxThreads);
      all_ok = sm.warp_ok[rb][0] && sm.warp_ok[rb][1] && sm.warp_ok[rb][2] && sm.warp_ok[rb][3];
      if (!all_ok) break;
      bool any_resc = false;
      float alpha[QPK];
#pragma unroll
      for (int h = 0; h < QPK; ++h) {
        const float mt = fmaxf(fmaxf(sm.red[rb][0][h], sm.red[rb][1][h]), fmaxf(sm.red[rb][2][h], sm.red[rb][3][h]));
        alpha[h] = 1.f;
        if (mt > m_ref[h] + kRescaleThreshold) {
          alpha[h] = fast_exp2(m_ref[h] - mt);  // 0 when m_ref = -inf
          m_ref[h] = mt;
          l_t[h] *= alpha[h];
          any_resc = true;
        }
      }
      if (any_resc && !first) {
        // O^T lane t is dim t; PV(j-1) must be complete before O changes.
        bool okr = __all_sync(0xffffffffu, mbar_wait(&sm.pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1));
        if (lane == 0) sm.resc_ok[warp] = okr;
        named_barrier_sync(1, kSoftmaxThreads);
        all_ok = sm.resc_ok[0] && sm.resc_ok[1] && sm.resc_ok[2] && sm.resc_ok[3];
        if (!all_ok) break;
        float o[8];
        tc_fence_after();
        tmem_ld_cols(o_tmem, QPK, o);
#pragma unroll
        for (int h = 0; h < QPK; ++h) o[h] *= alpha[h];
        tmem_st_cols(o_tmem, QPK, o);
      }
      if (!valid) {
        // Rows past the context hold arbitrary bits; P is 0 there, but the
        // tensor core still multiplies them, so they become zeros.
        const uint32_t vrow = smem_u32(sm.v[st]) + tid * 128;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          st_shared_v4(vrow + cc * 16, 0, 0, 0, 0);
          st_shared_v4(vrow + kHalf + cc * 16, 0, 0, 0, 0);
        }
      }
      // P^T[h][token], K-major SW128: tokens 0-63 in the first 2 KiB half.
      const uint32_t p_base = smem_u32(sm.p[sb]) + (tid >> 6) * kQHalf + (tid & 7) * 2;
      const int chunk = (tid & 63) >> 3;
#pragma unroll
      for (int h = 0; h < QPK; ++h) {
        const float mu = (m_ref[h] == -INFINITY) ? 0.f : m_ref[h];
        const float p = valid ? fast_exp2(sv[h] - mu) : 0.f;
        l_t[h] += p;
        const __nv_bfloat16 pb = __float2bfloat16_rn(p);
        const uint32_t addr = p_base + h * 128 + ((chunk ^ (h & 7)) << 4);
        asm volatile("st.shared.b16 [%0], %1;" ::"r"(addr), "h"(*reinterpret_cast<const uint16_t*>(&pb))
                     : "memory");
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&sm.p_full[sb]);
      if (!(ti.flags & kLastTile)) continue;
      // Hand the segment's (m, l) to the epilogue warps and go on streaming;
      // the info slot is free once the epilogue released segment seg-kOBufs.
      const int seg = ti.seg;
      if (seg >= kOBufs && !__all_sync(0xffffffffu, mbar_wait(&sm.o_empty[ob], ((seg / kOBufs) - 1) & 1))) {
        all_ok = false;
        break;
      }
      typename Smem::SegInfo& info = sm.seg_info[ob];
#pragma unroll
      for (int h = 0; h < QPK; ++h) {
        float x = l_t[h];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
        if (lane == 0) info.l_part[warp][h] = x;
        if (tid == 0) info.m[h] = m_ref[h];
      }
      if (tid == 0) {
        info.b = ti.b;
        info.g = ti.g;
        info.n = ti.n;
        info.ntiles = ti.ntiles;
        info.pair_t0 = ti.pair_t0;
        info.slot = ti.slot;
      }
      mbar_arrive(&sm.seg_ready[ob]);
    }
    if (!all_ok) flag_error(a, sm, kErrWaitTimeout);
  } else {
    // ------------------------------------------------------- epilogue ----
    // Warps 6-9: thread e owns dim d of O^T (TMEM lane d). Per segment:
    // normalise and store, or keep a partial piece; then publish the pieces
    // once and merge the pairs this CTA completes last.
    const int ew = warp - kEpilogueWarp0;
    const int e = ew * 32 + lane;
    const int d = (warp & 3) * 32 + lane;
    const uint32_t t_lane = static_cast<uint32_t>((warp & 3) * 32) << 16;
    bool ok = true;
    int seg = 0;
    SegIter it;
    it.init(sm, a, lo, hi);
    Segment s;
    // Never leaves the walk early and takes every named barrier of a partial
    // segment, even after a failed wait: the epilogue warps stay in step.
    int npart = 0;
    for (; it.next(sm, a, s); ++seg) {
      const int ob = seg % kOBufs;
      const bool part = s.ntiles != s.n;
      const int pi = npart & 1;
      // A piece of a pair shared with other CTAs. If every other piece is
      // already published, this CTA merges the pair: the others' partials are
      // fetched now, while its own piece is still being computed, and it
      // publishes nothing. Otherwise it publishes its piece after computing it.
      int c_first = 0, pieces = 1;
      int* ticket = nullptr;
      bool pre_last = false;
      float2 pml[kFastPieces][QPK];
      float po[kFastPieces][QPK];
      if (part) {
        c_first = cta_of(s.pair_t0, sc);
        pieces = cta_of(s.pair_t0 + s.n - 1, sc) - c_first + 1;  // CTAs holding tiles are contiguous
        ticket = a.ws_cnt + static_cast<int64_t>(s.b * kvh + s.g) * kTicketStride;
        if (e == 0) sm.pre_last[pi] = (pieces - 1 <= kFastPieces) && ld_acquire_gpu(ticket) == pieces - 1;
        named_barrier_sync(2, kEpilogueThreads);  // one decision for all epilogue threads
        pre_last = sm.pre_last[pi] != 0;
        if (pre_last) {
#pragma unroll
          for (int u = 0; u < kFastPieces; ++u) {
            const int cc = c_first + (u < c - c_first ? u : u + 1);  // every piece but this CTA's
#pragma unroll
            for (int h = 0; h < QPK; ++h) {
              const bool use = u < pieces - 1;
              const int64_t pp = use ? part_index(cc, s.pair_t0, sc, QPK) + h : 0;
              pml[u][h] = use ? __ldcg(&a.ws_ml[pp]) : make_float2(-INFINITY, 0.f);
              po[u][h] = use ? __ldcg(&a.ws_o[pp * kD + d]) : 0.f;
            }
          }
        }
      }
      if (ok) ok = mbar_wait(&sm.seg_ready[ob], (seg / kOBufs) & 1) && mbar_wait(&sm.o_full[ob], (seg / kOBufs) & 1);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        float o[8];
        tc_fence_after();
        tmem_ld_cols(tmem + 32 + ob * kN + t_lane, QPK, o);
        const typename Smem::SegInfo& info = sm.seg_info[ob];
        float l_sum[QPK], m_seg[QPK];
#pragma unroll
        for (int h = 0; h < QPK; ++h) {
          l_sum[h] = info.l_part[0][h] + info.l_part[1][h] + info.l_part[2][h] + info.l_part[3][h];
          m_seg[h] = info.m[h];
        }
        tc_fence_before();
        mbar_arrive(&sm.o_empty[ob]);
        if (!part) {  // the whole pair lies in this CTA
#pragma unroll
          for (int h = 0; h < QPK; ++h) store_out(a, s.b, s.g * QPK + h, d, l_sum[h] > 0.f ? o[h] / l_sum[h] : 0.f);
        } else if (pre_last) {  // merge this piece (registers) with the fetched ones
#pragma unroll
          for (int h = 0; h < QPK; ++h) {
            float M = m_seg[h];
#pragma unroll
            for (int u = 0; u < kFastPieces; ++u) M = fmaxf(M, pml[u][h].x);
            float num = 0.f, den = 0.f;
            if (M != -INFINITY) {
              if (m_seg[h] != -INFINITY) {
                const float w = fast_exp2(m_seg[h] - M);
                num = w * o[h];
                den = w * l_sum[h];
              }
#pragma unroll
              for (int u = 0; u < kFastPieces; ++u) {
                if (pml[u][h].x == -INFINITY) continue;
                const float w = fast_exp2(pml[u][h].x - M);
                num = fmaf(w, po[u][h], num);
                den = fmaf(w, pml[u][h].y, den);
              }
            }
            store_out(a, s.b, s.g * QPK + h, d, den > 0.f ? num / den : 0.f);
          }
          if (e == 0) *ticket = 0;  // every other piece arrived and none will touch it again this call
        } else {  // this CTA's piece, for whichever CTA merges the pair
          const int64_t slot_part = part_index(c, s.pair_t0, sc, QPK);
#pragma unroll
          for (int h = 0; h < QPK; ++h) {
            a.ws_o[(slot_part + h) * kD + d] = o[h];
            if (e == 0) a.ws_ml[slot_part + h] = make_float2(m_seg[h], l_sum[h]);
          }
        }
      }
      if (a.world > 1 && (!part || pre_last)) {  // this CTA completed the pair: its rows go to the peers
        named_barrier_sync(2, kEpilogueThreads);
        push_rows(a, s.b, s.g * QPK, QPK, e);
      }
      if (part && !pre_last) {
        // Publish: one acq_rel ticket releases the piece (every epilogue
        // thread's stores, ordered by the barrier) and acquires the others'.
        if (lane == 0) sm.epi_ok[ew] = ok;
        named_barrier_sync(2, kEpilogueThreads);
        if (e == 0) {
          const bool all_ok = sm.epi_ok[0] && sm.epi_ok[1] && sm.epi_ok[2] && sm.epi_ok[3];
          int last = 0;
          if (all_ok) {
            int old;
            asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(ticket) : "memory");
            last = (old == pieces - 1);
          } else {
            flag_error(a, sm, kErrWaitTimeout);
          }
          sm.last[pi] = last;
        }
        named_barrier_sync(2, kEpilogueThreads);
        if (sm.last[pi]) {
          merge_published<QPK>(sm, a, sc, e, d, s.b, s.g, s.pair_t0, c_first, pieces, ticket);
          if (a.world > 1) {
            named_barrier_sync(2, kEpilogueThreads);
            push_rows(a, s.b, s.g * QPK, QPK, e);
          }
        }
      }
      if (part) ++npart;
    }
    if (!ok) flag_error(a, sm, kErrWaitTimeout);

    // Sequences without context own no tile: their outputs are zeros (and
    // a fused append still writes their row, as the reference's write would).
    for (int b = c; b < a.batch; b += ctas) {
      if (sm.tiles_before[b + 1] == sm.tiles_before[b]) {
        for (int h = 0; h < a.num_heads; ++h) store_out(a, b, h, e, 0.f);
        if (a.world > 1) {
          named_barrier_sync(2, kEpilogueThreads);
          push_rows(a, b, 0, a.num_heads, e);
        }
        if (a.new_slots != nullptr) {
          const int64_t slot = a.new_slots[b];
          const int words = kvh * (kD * 2 / 16);
          if (slot >= 0 && slot < a.num_slots) {
            for (int w = e; w < words; w += kEpilogueThreads) {
              a.kc_words[slot * words + w] = a.k_new[b * a.k_new_stride_w + w];
              a.vc_words[slot * words + w] = a.v_new[b * a.v_new_stride_w + w];
            }
          } else if (e == 0) {
            atomicOr(a.err, kErrBadSlot);
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
  if (a.world > 0 && tid == 0) gather_signal(a, ctas);
}

static_assert(sizeof(Smem) + 1024 <= 232448, "decode shared memory exceeds the 227 KB per-CTA limit");

struct WsLayout {
  size_t cnt_off, ml_off, o_off, total;
};

// [0, 256): error word (byte 0), gather-mode CTA counter (64) and timing sums (128..159) |
// tickets [batch * KVH], one per 128-byte line | (m, l) [C][2][QPK] | o [C][2][QPK][128]
WsLayout ws_layout(int batch, int num_heads, int num_kv_heads, int ctas) {
  auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
  const int qpk = num_heads / num_kv_heads;
  const size_t parts = static_cast<size_t>(ctas) * 2 * qpk;
  WsLayout w;
  w.cnt_off = 256;
  w.ml_off = w.cnt_off + up(static_cast<size_t>(batch) * num_kv_heads * kTicketStride * sizeof(int));
  w.o_off = w.ml_off + up(parts * sizeof(float2));
  w.total = w.o_off + up(parts * kD * sizeof(float));
  return w;
}

int resolve_ctas(int num_ctas, int* out) {
  if (num_ctas > 0) {
    *out = num_ctas;
    return NVK_OK;
  }
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return check_cuda(e, "paged_decode: SM count");
  *out = sms;
  return NVK_OK;
}

}  // namespace
}  // namespace nvk

extern "C" int nvk_paged_decode_workspace_size(int batch, int num_heads, int num_kv_heads, int head_dim,
                                               int num_ctas, size_t* bytes) {
  using namespace nvk;
  if (!bytes) return fail(NVK_ERR_INVALID_ARGUMENT, "workspace_size: null output pointer");
  if (batch < 0 || num_heads <= 0 || num_kv_heads <= 0 || num_ctas < 0 || num_heads % num_kv_heads != 0)
    return fail(NVK_ERR_INVALID_ARGUMENT, "workspace_size: bad sizes (batch=%d heads=%d kv_heads=%d ctas=%d)",
                batch, num_heads, num_kv_heads, num_ctas);
  if (head_dim != kD) return fail(NVK_ERR_UNSUPPORTED, "workspace_size: head_dim %d unsupported (128 only)", head_dim);
  int ctas = 0;
  const int rc = resolve_ctas(num_ctas, &ctas);
  if (rc != NVK_OK) return rc;
  *bytes = ws_layout(batch, num_heads, num_kv_heads, ctas).total;
  return NVK_OK;
}

namespace nvk {
namespace {

// This step's token rows for a fused append (see nvk_paged_decode_append).
struct AppendRows {
  const void* key;
  const void* value;
  int64_t key_stride, value_stride;  // elements between consecutive tokens
  const int64_t* slots;
};

// Where a gathering decode call stores its rows (see nvk_paged_decode_gather).
struct GatherTargets {
  void* const* out_peers;
  void* const* signal_peers;
  int world, rank, out_heads, head_offset;
};

// Every host-side argument check of a decode call except the workspace's.
int decode_check_args(const void* out, const void* query, const void* key_cache, const void* value_cache,
                      int num_blocks, int block_size, const int32_t* block_tables, int block_table_stride,
                      int max_blocks_per_seq, const int32_t* context_lens, int batch, int num_heads,
                      int num_kv_heads, int head_dim, int num_ctas, const GatherTargets* gt, const AppendRows* ap) {
  if (batch < 0 || num_blocks <= 0 || num_heads <= 0 || num_kv_heads <= 0 || num_ctas < 0)
    return fail(NVK_ERR_INVALID_ARGUMENT, "paged_decode: bad sizes (batch=%d blocks=%d heads=%d kv_heads=%d ctas=%d)",
                batch, num_blocks, num_heads, num_kv_heads, num_ctas);
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
  if (max_blocks_per_seq <= 0 || block_table_stride < max_blocks_per_seq)
    return fail(NVK_ERR_INVALID_ARGUMENT, "paged_decode: block table width %d / stride %d invalid",
                max_blocks_per_seq, block_table_stride);
  if ((!gt && !out) || !query || !key_cache || !value_cache || !block_tables || !context_lens)
    return fail(NVK_ERR_INVALID_ARGUMENT, "paged_decode: null pointer");
  if ((!gt && !aligned16(out)) || !aligned16(query))
    return fail(NVK_ERR_INVALID_ARGUMENT, "paged_decode: q/out must be 16-byte aligned");
  if (ap) {
    const int64_t row = static_cast<int64_t>(num_kv_heads) * kD;
    if (!ap->key || !ap->value || !ap->slots || !aligned16(ap->key) || !aligned16(ap->value) ||
        ap->key_stride < row || ap->value_stride < row || ap->key_stride % 8 != 0 || ap->value_stride % 8 != 0)
      return fail(NVK_ERR_INVALID_ARGUMENT,
                  "paged_decode_append: new rows null, misaligned or strides (%lld, %lld) below a row / not 16-byte",
                  (long long)ap->key_stride, (long long)ap->value_stride);
  }
  return NVK_OK;
}

int decode_impl(void* out, const void* query, const void* key_cache, const void* value_cache, int num_blocks,
                int block_size, const int32_t* block_tables, int block_table_stride, int max_blocks_per_seq,
                const int32_t* context_lens, int batch, int num_heads, int num_kv_heads, int head_dim, float scale,
                int num_ctas, void* workspace, size_t workspace_bytes, const GatherTargets* gt, const AppendRows* ap,
                nvk_stream_t stream) {
  int rc = decode_check_args(out, query, key_cache, value_cache, num_blocks, block_size, block_tables,
                             block_table_stride, max_blocks_per_seq, context_lens, batch, num_heads, num_kv_heads,
                             head_dim, num_ctas, gt, ap);
  if (rc != NVK_OK || batch == 0) return rc;
  const int qpk = num_heads / num_kv_heads;
  int ctas = 0;
  rc = resolve_ctas(num_ctas, &ctas);
  if (rc != NVK_OK) return rc;
  const WsLayout wl = ws_layout(batch, num_heads, num_kv_heads, ctas);
  if (!workspace || workspace_bytes < wl.total || !aligned16(workspace))
    return fail(NVK_ERR_WORKSPACE, "paged_decode: workspace %zu bytes < %zu needed (or misaligned)", workspace_bytes,
                wl.total);

  const int64_t rows = static_cast<int64_t>(num_blocks) * block_size;
  const int sub_rows = block_size < 32 ? block_size : 32;
  CUtensorMap km, vm, qm;
  if ((rc = kv_tensor_map(&km, key_cache, rows, num_kv_heads, sub_rows)) != NVK_OK) return rc;
  if ((rc = kv_tensor_map(&vm, value_cache, rows, num_kv_heads, sub_rows)) != NVK_OK) return rc;
  const size_t smem = sizeof(Smem) + 1024;
  const void* kernel = qpk == 1   ? reinterpret_cast<const void*>(&paged_decode_kernel<1>)
                       : qpk == 2 ? reinterpret_cast<const void*>(&paged_decode_kernel<2>)
                       : qpk == 4 ? reinterpret_cast<const void*>(&paged_decode_kernel<4>)
                                  : reinterpret_cast<const void*>(&paged_decode_kernel<8>);
  rc = ensure_dynamic_smem(kernel, smem);
  if (rc != NVK_OK) return rc;

  uint8_t* ws = static_cast<uint8_t*>(workspace);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // Sequences go in chunks of kMaxSeqs launches (the schedule lives in smem).
  for (int b0 = 0; b0 < batch; b0 += kMaxSeqs) {
    const int nb = batch - b0 < kMaxSeqs ? batch - b0 : kMaxSeqs;
    const void* qb = static_cast<const uint8_t*>(query) + static_cast<size_t>(b0) * num_heads * kD * 2;
    // q as [nb, heads, 128]: box {64 dims, QPK heads, 1 sequence}
    if ((rc = kv_tensor_map(&qm, qb, nb, num_heads, 1, 0, qpk)) != NVK_OK) return rc;
    DecodeArgs a;
    const int out_heads = gt ? gt->out_heads : num_heads;
    const size_t out_skip = static_cast<size_t>(b0) * out_heads * kD;
    a.out = gt ? nullptr : static_cast<__nv_bfloat16*>(out) + out_skip;
    a.out_heads = out_heads;
    a.head_offset = gt ? gt->head_offset : 0;
    a.world = gt ? gt->world : 0;
    a.rank = gt ? gt->rank : 0;
    for (int r = 0; r < NVK_MAX_PEERS; ++r) {
      const bool on = gt && r < gt->world;
      a.peer_out[r] = on ? static_cast<__nv_bfloat16*>(gt->out_peers[r]) + out_skip : nullptr;
      a.peer_sig[r] = on ? static_cast<uint32_t*>(gt->signal_peers[r]) : nullptr;
    }
    a.my_sig = gt ? static_cast<uint32_t*>(gt->signal_peers[gt->rank]) : nullptr;
    a.done = reinterpret_cast<int*>(ws + 64);
    a.timing = reinterpret_cast<unsigned long long*>(ws + 128);
    a.new_slots = ap ? ap->slots + b0 : nullptr;
    a.k_new = ap ? static_cast<const uint4*>(ap->key) + b0 * (ap->key_stride / 8) : nullptr;
    a.v_new = ap ? static_cast<const uint4*>(ap->value) + b0 * (ap->value_stride / 8) : nullptr;
    a.k_new_stride_w = ap ? ap->key_stride / 8 : 0;
    a.v_new_stride_w = ap ? ap->value_stride / 8 : 0;
    a.kc_words = static_cast<uint4*>(const_cast<void*>(key_cache));
    a.vc_words = static_cast<uint4*>(const_cast<void*>(value_cache));
    a.num_slots = rows;
    a.query = qb;
    a.block_tables = block_tables + static_cast<int64_t>(b0) * block_table_stride;
    a.context_lens = context_lens + b0;
    a.err = reinterpret_cast<int*>(ws);
    a.ws_cnt = reinterpret_cast<int*>(ws + wl.cnt_off) + static_cast<size_t>(b0) * num_kv_heads * kTicketStride;
    a.ws_ml = reinterpret_cast<float2*>(ws + wl.ml_off);
    a.ws_o = reinterpret_cast<float*>(ws + wl.o_off);
    a.batch = nb;
    a.bt_stride = block_table_stride;
    a.max_blocks = max_blocks_per_seq;
    a.num_blocks = num_blocks;
    a.block_size = block_size;
    a.log2_bs = __builtin_ctz(static_cast<unsigned>(block_size));
    a.sub_rows = sub_rows;
    a.chunk_tiles = block_size >= 64 ? kChunkTiles : kSlotIds * block_size / kTile;
    a.num_heads = num_heads;
    a.num_kv_heads = num_kv_heads;
    a.qpk = qpk;
    a.scale_log2 = scale * 1.4426950408889634f;
    cudaError_t e;
    switch (qpk) {
      case 1: e = launch_pdl(paged_decode_kernel<1>, dim3(ctas), dim3(kThreads), smem, st, km, vm, qm, a); break;
      case 2: e = launch_pdl(paged_decode_kernel<2>, dim3(ctas), dim3(kThreads), smem, st, km, vm, qm, a); break;
      case 4: e = launch_pdl(paged_decode_kernel<4>, dim3(ctas), dim3(kThreads), smem, st, km, vm, qm, a); break;
      default: e = launch_pdl(paged_decode_kernel<8>, dim3(ctas), dim3(kThreads), smem, st, km, vm, qm, a); break;
    }
    rc = check_cuda(e, "paged_decode launch");
    if (rc != NVK_OK) return rc;
  }
  return NVK_OK;
}

}  // namespace
}  // namespace nvk

extern "C" int nvk_paged_decode(void* out, const void* query, const void* key_cache, const void* value_cache,
                                int num_blocks, int block_size, const int32_t* block_tables, int block_table_stride,
                                int max_blocks_per_seq, const int32_t* context_lens, int batch, int num_heads,
                                int num_kv_heads, int head_dim, float scale, int num_ctas, void* workspace,
                                size_t workspace_bytes, nvk_stream_t stream) {
  return nvk::decode_impl(out, query, key_cache, value_cache, num_blocks, block_size, block_tables,
                          block_table_stride, max_blocks_per_seq, context_lens, batch, num_heads, num_kv_heads,
                          head_dim, scale, num_ctas, workspace, workspace_bytes, nullptr, nullptr, stream);
}

extern "C" int nvk_paged_decode_append(void* out, const void* query, void* key_cache, void* value_cache,
                                       int num_blocks, int block_size, const int32_t* block_tables,
                                       int block_table_stride, int max_blocks_per_seq, const int32_t* context_lens,
                                       int batch, int num_heads, int num_kv_heads, int head_dim, float scale,
                                       int num_ctas, void* workspace, size_t workspace_bytes, const void* key,
                                       const void* value, int64_t key_token_stride, int64_t value_token_stride,
                                       const int64_t* slot_mapping, nvk_stream_t stream) {
  const nvk::AppendRows ap{key, value, key_token_stride, value_token_stride, slot_mapping};
  return nvk::decode_impl(out, query, key_cache, value_cache, num_blocks, block_size, block_tables,
                          block_table_stride, max_blocks_per_seq, context_lens, batch, num_heads, num_kv_heads,
                          head_dim, scale, num_ctas, workspace, workspace_bytes, nullptr, &ap, stream);
}

extern "C" int nvk_paged_decode_gather(const void* query, void* key_cache, void* value_cache,
                                       int num_blocks, int block_size, const int32_t* block_tables,
                                       int block_table_stride, int max_blocks_per_seq, const int32_t* context_lens,
                                       int batch, int num_heads, int num_kv_heads, int head_dim, float scale,
                                       int num_ctas, void* workspace, size_t workspace_bytes,
                                       void* const* out_peers, void* const* signal_peers, int world, int rank,
                                       int out_heads, int head_offset, const void* key, const void* value,
                                       int64_t key_token_stride, int64_t value_token_stride,
                                       const int64_t* slot_mapping, nvk_stream_t stream) {
  using namespace nvk;
  if (world < 1 || world > NVK_MAX_PEERS || rank < 0 || rank >= world)
    return fail(NVK_ERR_INVALID_ARGUMENT, "paged_decode_gather: rank %d / world %d invalid (world 1..%d)", rank,
                world, NVK_MAX_PEERS);
  if (head_offset < 0 || num_heads <= 0 || out_heads < head_offset + num_heads)
    return fail(NVK_ERR_INVALID_ARGUMENT, "paged_decode_gather: heads [%d, %d) outside the %d output heads",
                head_offset, head_offset + num_heads, out_heads);
  if (!out_peers || !signal_peers) return fail(NVK_ERR_INVALID_ARGUMENT, "paged_decode_gather: null peer arrays");
  for (int r = 0; r < world; ++r) {
    if (!out_peers[r] || !aligned16(out_peers[r]) || !signal_peers[r] ||
        (reinterpret_cast<uintptr_t>(signal_peers[r]) & 3u) != 0)
      return fail(NVK_ERR_INVALID_ARGUMENT, "paged_decode_gather: rank %d buffers null or misaligned", r);
  }
  const GatherTargets gt{out_peers, signal_peers, world, rank, out_heads, head_offset};
  const AppendRows ap{key, value, key_token_stride, value_token_stride, slot_mapping};
  return decode_impl(nullptr, query, key_cache, value_cache, num_blocks, block_size, block_tables,
                     block_table_stride, max_blocks_per_seq, context_lens, batch, num_heads, num_kv_heads, head_dim,
                     scale, num_ctas, workspace, workspace_bytes, &gt, slot_mapping ? &ap : nullptr, stream);
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

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

// Unique id of the CUDA context current on this thread (0 if none). Ids are
// never reused within a process, so a context created after a device reset,
// or a second context a plugin host made current on the same device, gets a
// fresh one. The driver functions are resolved through the runtime, like
// cuTensorMapEncodeTiled, so the library does not link libcuda.
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of the scratch array in the current context. The symbol's
// host-side name is only a handle: the address is fetched with
// cudaGetSymbolAddress once per CUDA context (the first call on a device does
// it, with that device current) and cached under the context's id.
int noalloc_scratch(void** out) {
  struct Entry {
    unsigned long long ctx_id;
    void* addr;
  };
  static std::mutex mu;
  static Entry cache[kNoAllocMaxDevices] = {};
  static int next = 0;
  std::lock_guard<std::mutex> lock(mu);
  unsigned long long id = current_context_id();
  if (id != 0) {
    for (const Entry& e : cache)
      if (e.ctx_id == id) {
        *out = e.addr;
        return NVK_OK;
      }
  }
  void* p = nullptr;
  // With no context current yet this call also initialises the device's primary context.
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_decode_scratch);
  if (e != cudaSuccess) return nvk::check_cuda(e, "paged_decode_noalloc: cudaGetSymbolAddress");
  if (id == 0) id = current_context_id();
  if (id != 0) {
    cache[next] = Entry{id, p};
    next = (next + 1) % kNoAllocMaxDevices;
  }
  *out = p;
  return NVK_OK;
}

}  // namespace

extern "C" int nvk_paged_decode_noalloc(void* out, const void* query, const void* key_cache,
                                        const void* value_cache, int num_blocks, int block_size,
                                        const int32_t* block_tables, int block_table_stride, int max_blocks_per_seq,
                                        const int32_t* context_lens, int batch, int num_heads, int num_kv_heads,
                                        int head_dim, float scale, int num_ctas, nvk_stream_t stream) {
  using namespace nvk;
  // Arguments first, so that a call refused for them queues nothing on the stream.
  int rc = decode_check_args(out, query, key_cache, value_cache, num_blocks, block_size, block_tables,
                             block_table_stride, max_blocks_per_seq, context_lens, batch, num_heads, num_kv_heads,
                             head_dim, num_ctas, nullptr, nullptr);
  if (rc != NVK_OK || batch == 0) return rc;
  int ctas = 0;
  rc = resolve_ctas(num_ctas, &ctas);
  if (rc != NVK_OK) return rc;
  const WsLayout wl = ws_layout(batch, num_heads, num_kv_heads, ctas);
  if (wl.total > kNoAllocScratchBytes)
    return fail(NVK_ERR_UNSUPPORTED,
                "paged_decode_noalloc: %zu bytes of split-K scratch needed, the static scratch holds %zu "
                "(a smaller batch, or nvk_paged_decode with a caller workspace)",
                wl.total, kNoAllocScratchBytes);
  void* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc != NVK_OK) return rc;
  // The array keeps the previous call's contents: clear the error word and
  // the arrival tickets, which must start at zero.
  rc = check_cuda(cudaMemsetAsync(scratch, 0, wl.ml_off, reinterpret_cast<cudaStream_t>(stream)),
                  "paged_decode_noalloc: clear scratch header");
  if (rc != NVK_OK) return rc;
  return nvk_paged_decode(out, query, key_cache, value_cache, num_blocks, block_size, block_tables,
                          block_table_stride, max_blocks_per_seq, context_lens, batch, num_heads, num_kv_heads,
                          head_dim, scale, num_ctas, scratch, kNoAllocScratchBytes, stream);
}

extern "C" int nvk_paged_decode_noalloc_error(int* error_word, nvk_stream_t stream) {
  using namespace nvk;
  if (!error_word) return fail(NVK_ERR_INVALID_ARGUMENT, "paged_decode_noalloc_error: null output pointer");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  int rc = check_cuda(cudaStreamIsCapturing(st, &cap), "paged_decode_noalloc_error: capture status");
  if (rc != NVK_OK) return rc;
  if (cap != cudaStreamCaptureStatusNone)
    return fail(NVK_ERR_INVALID_ARGUMENT, "paged_decode_noalloc_error: the stream is capturing (this call waits)");
  void* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc != NVK_OK) return rc;
  int word = 0;
  rc = check_cuda(cudaMemcpyAsync(&word, scratch, sizeof(int), cudaMemcpyDeviceToHost, st),
                  "paged_decode_noalloc_error: copy");
  if (rc != NVK_OK) return rc;
  rc = check_cuda(cudaStreamSynchronize(st), "paged_decode_noalloc_error: synchronize");
  if (rc != NVK_OK) return rc;
  *error_word = word;
  return NVK_OK;
}
