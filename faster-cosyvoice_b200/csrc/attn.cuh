// attn.cuh -- ragged multi-head attention over packed documents.
//
// Semantics (modules.py:349-407 with the masks of mask.py:127-158, 223-229;
// FlashInfer ragged prefill in flashinfer_attention.py:36-142): for document
// d with rows [cu[d], cu[d+1]), head h, query q:
//     o = softmax(q K^T / 8 + mask) V
// with keys k < L_d and, when chunk > 0, only k // chunk <= q // chunk.
// The mask is evaluated arithmetically (nothing is materialised) and key
// tiles past the last visible key of a query tile are never loaded.  A
// document's result depends only on its own rows (no split-KV), so outputs
// are invariant to batch composition.
//
// Work list: (128-row query tile, head) items; tiles come from the host as
// (doc, q0) pairs ordered by cost, most expensive first.
#pragma once

#include "fcv_common.cuh"

namespace fcv {

constexpr int kQkvStride = 3072;
constexpr int kAttnQTile = 128;

// Last visible key (exclusive) for the query rows [q0, q0+rows) of a document of length L.
__device__ __forceinline__ int kv_limit(int q0, int rows, int L, int chunk) {
  const int q_last = min(q0 + rows - 1, L - 1);
  if (chunk <= 0) return L;
  return min(L, (q_last / chunk + 1) * chunk);
}

// Where a document's queries and keys live.  Queries (and outputs) are rows
// [cu[d], cu[d+1]) of the packed Q buffer.  A document may continue a cached
// prefix (streaming prefix reuse): its first query row then sits at absolute
// position pos0[d], and its keys are rows kv_base[d] .. kv_base[d] + pos0[d] + L
// of a separate K/V buffer (the cache, prefix keys first).  Without pos0 /
// kv_base the keys are the document's own rows of the QKV buffer.
struct AttnSrc {
  const int32_t* cu;
  const int32_t* pos0;     // null: 0
  const int32_t* kv_base;  // null: cu[d]
};

// ------------------------------------------------------------------ bf16 (tcgen05)
// Persistent: each CTA walks work items (128-row query tile, head) c, c+grid, ...
// (tiles arrive most expensive first).  6 warps per CTA, 2 CTAs per SM:
//   warp 0   TMA: Q of each item into one of two buffers, K/V tiles of 64 keys
//            into a 4-stage ring
//   warp 1   owns TMEM (S at columns 0..63, P at 64..95, two O buffers of 80
//            columns at 96 and 176) and issues tcgen05.mma: S_g = Q K_g^T, then
//            O += P_g [V_g | 1] with P_g read from TMEM
//   warps 2-5 softmax: TMEM lane quarter = warp % 4, one query row per lane and
//            all 64 keys of a tile per thread, so row maxima stay in registers.
//            A 32-key half that no row of the warp can see (past the document
//            or the chunk limit) is neither loaded nor exponentiated: its P is 0.
// The softmax row sum comes from the tensor core: V is extended by a constant
// shared block whose first column is 1 (reached through the descriptor's
// leading byte offset), so O column 64 holds sum_k P[q,k] in the same bf16 P
// that multiplies V.  Exponentials use a per-row reference max that moves only
// when a tile max exceeds it by more than 8 (log2 units); O (with its sum
// column) in TMEM is rescaled only then.  S_{g+1} -- possibly the next item's
// first tile -- is issued as soon as S_g has been read, and the next item's Q is
// loaded while the current item finishes, so items overlap.
// Barrier invariant: every mbarrier is waited on with a parity that its
// producer cannot have advanced past by two phases (per-buffer barriers for Q
// and O; P is written only after the previous P.V is done), so parity waits
// never alias.  P lives in TMEM, so no shared-memory round trip per tile.
constexpr int kTcKv = 64;
constexpr int kTcSmemQ = 128 * 128;      // 16 KB per Q buffer
constexpr int kTcSmemKV = kTcKv * 128;   // 8 KB per K or V tile
constexpr int kTcKvStages = 4;
constexpr int kTcOffK = 2 * kTcSmemQ;
constexpr int kTcOffV = kTcOffK + kTcKvStages * kTcSmemKV;
constexpr int kTcOffOnes = kTcOffV + kTcKvStages * kTcSmemKV;  // 64 x 64 bf16, column 0 = 1
// TMEM columns: S [0, 64), P [64, 96) (bf16 pairs), O buffers [96, 176) and [176, 256)
constexpr int kTcColP = 64;
constexpr int kTcColO = 96;
constexpr int kTcOffBar = kTcOffOnes + kTcSmemKV;
// mbarrier slots (8 bytes each), derived from the stage count
constexpr int kBarQFull = 0;
constexpr int kBarQEmpty = kBarQFull + 2;
constexpr int kBarKvFull = kBarQEmpty + 2;
constexpr int kBarKvEmpty = kBarKvFull + kTcKvStages;
constexpr int kBarSFull = kBarKvEmpty + kTcKvStages;
constexpr int kBarSEmpty = kBarSFull + 1;
constexpr int kBarPFull = kBarSEmpty + 1;
constexpr int kBarODone = kBarPFull + 1;
constexpr int kBarOEmpty = kBarODone + 1;
constexpr int kBarOFinal = kBarOEmpty + 2;  // [2] last P.V of an item done, per O buffer
constexpr int kBarDrain = kBarOFinal + 2;
constexpr int kBarCount = kBarDrain + 1;
constexpr int kTcBarBytes = 256;
static_assert(kBarCount * 8 + 8 <= kTcBarBytes, "attention barrier area too small");
constexpr int kTcSmemBytes = 1024 + kTcOffBar + kTcBarBytes;
constexpr int kTcOCols = 80;  // 64 output columns + the row sum + 15 zero columns
constexpr float kRescaleThreshold = 8.0f;

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 32 TMEM lanes x 32 consecutive columns <- 32 registers per thread.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// One work item: query rows [q0, q0 + 128) of a document (local indices), one
// head.  base / L: the document's query rows; pos0: absolute position of local
// row 0; kvb / Lkv: its first key row and key count (pos0 + L).
struct AttnItem {
  int base, L, q0, head, n_kv, pos0, kvb, Lkv;
};

// Item `it` from its work-list entry tl (already loaded).
__device__ __forceinline__ AttnItem attn_item_at(const AttnSrc& src, int2 tl, int chunk, int it) {
  AttnItem a;
  a.head = it & 15;
  a.q0 = tl.y;
  a.base = src.cu[tl.x];
  a.L = src.cu[tl.x + 1] - a.base;
  a.pos0 = src.pos0 ? __ldg(src.pos0 + tl.x) : 0;
  a.kvb = src.kv_base ? __ldg(src.kv_base + tl.x) : a.base;
  a.Lkv = a.pos0 + a.L;
  // the tile's last query row in absolute positions bounds its visible keys
  const int q_last = a.pos0 + min(a.q0 + kAttnQTile - 1, a.L - 1);
  const int lim = chunk > 0 ? min(a.Lkv, (q_last / chunk + 1) * chunk) : a.Lkv;
  a.n_kv = (lim + kTcKv - 1) / kTcKv;
  return a;
}

__device__ __forceinline__ AttnItem attn_item(const AttnSrc& src, const int2* tiles, int chunk, int it) {
  return attn_item_at(src, tiles[it >> 4], chunk, it);
}

// A CTA's items with the descriptor lookups run ahead: while item `it` is
// processed, the item after it is already resolved (its cu loads in flight)
// and the work-list entry of the one after that is loading, so no role waits
// on a dependent global load at an item boundary.  Items come either round
// robin (positions first, first + stride, ... of the work list) or from a
// host-built schedule: positions [beg, end) of a per-CTA item list.
struct ItemFeed {
  AttnSrc cu;
  const int2* tiles;
  const int32_t* list;  // schedule items, or null for round robin
  int chunk, end, stride, pos, it, it1, it2;
  AttnItem cur, nxt;
  int2 tl2;
  __device__ __forceinline__ int item_at(int p) const { return list ? __ldg(list + p) : p; }
  // Round robin when sched is null; else sched = [offsets (gridDim + 1) | items].
  __device__ __forceinline__ bool init(const AttnSrc& cu_, const int2* tiles_, int chunk_, int n_items,
                                       const int32_t* sched) {
    cu = cu_;
    tiles = tiles_;
    chunk = chunk_;
    if (sched) {
      list = sched + gridDim.x + 1;
      pos = __ldg(sched + blockIdx.x);
      end = __ldg(sched + blockIdx.x + 1);
      stride = 1;
    } else {
      list = nullptr;
      pos = blockIdx.x;
      end = n_items;
      stride = gridDim.x;
    }
    if (pos >= end) return false;
    it = item_at(pos);
    cur = attn_item(cu, tiles, chunk, it);
    if (pos + stride < end) {
      it1 = item_at(pos + stride);
      nxt = attn_item(cu, tiles, chunk, it1);
    }
    if (pos + 2 * stride < end) {
      it2 = item_at(pos + 2 * stride);
      tl2 = tiles[it2 >> 4];
    }
    return true;
  }
  __device__ __forceinline__ bool advance() {
    pos += stride;
    if (pos >= end) return false;
    it = it1;
    cur = nxt;
    if (pos + stride < end) {
      it1 = it2;
      nxt = attn_item_at(cu, tl2, chunk, it1);
    }
    if (pos + 2 * stride < end) {
      it2 = item_at(pos + 2 * stride);
      tl2 = tiles[it2 >> 4];
    }
    return true;
  }
};

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

constexpr int kTcThreads = 192;  // warp 0 TMA, warp 1 MMA, warps 2-5 softmax (one per TMEM lane quarter)
constexpr int kTcSoftmaxWarps = 4;

__global__ void __launch_bounds__(kTcThreads, 2)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                   const AttnSrc src, const int2* __restrict__ tiles, int n_tiles,
                   const int32_t* __restrict__ n_tiles_dev, const int32_t* __restrict__ sched, int chunk,
                   int k_col, int v_col, bf16* __restrict__ out) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t s0 = smem_u32(smem);
  const uint32_t sQ = s0, sK = s0 + kTcOffK, sV = s0 + kTcOffV, sOnes = s0 + kTcOffOnes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kTcOffBar);
  uint64_t* q_full = bars + kBarQFull;     // [2]
  uint64_t* q_empty = bars + kBarQEmpty;   // [2]
  uint64_t* kv_full = bars + kBarKvFull;   // [kTcKvStages]
  uint64_t* kv_empty = bars + kBarKvEmpty; // [kTcKvStages]
  uint64_t* s_full = bars + kBarSFull;
  uint64_t* s_empty = bars + kBarSEmpty;
  uint64_t* p_full = bars + kBarPFull;     // P_g written
  uint64_t* o_done = bars + kBarODone;     // P_g [V_g|1] complete (P free, O updated)
  uint64_t* o_empty = bars + kBarOEmpty;   // [2] final O of an item read, per O buffer
  uint64_t* o_final = bars + kBarOFinal;   // [2] final O of an item complete, per O buffer
  uint64_t* drain = bars + kBarDrain;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kBarCount);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&q_full[i]), 1);
      mbar_init(smem_u32(&q_empty[i]), 1);
      mbar_init(smem_u32(&o_empty[i]), kTcSoftmaxWarps);
      mbar_init(smem_u32(&o_final[i]), 1);
    }
    for (int i = 0; i < kTcKvStages; ++i) {
      mbar_init(smem_u32(&kv_full[i]), 1);
      mbar_init(smem_u32(&kv_empty[i]), 1);
    }
    mbar_init(smem_u32(p_full), kTcSoftmaxWarps);
    mbar_init(smem_u32(o_done), 1);
    mbar_init(smem_u32(s_full), 1);
    mbar_init(smem_u32(s_empty), kTcSoftmaxWarps);
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmKV);
  }
  if (warp >= 2 && threadIdx.x - 64 < 64) {
    // constant [1 0 ... 0] rows extending V (128-byte swizzle: chunk c of row r at c ^ (r % 8))
    const int r = threadIdx.x - 64;
    uint8_t* row = smem + kTcOffOnes + r * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(row + c * 16) = make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(row + ((0 ^ (r & 7)) << 4)) = make_uint4(0x3F80u, 0, 0, 0);  // bf16 1.0 in column 0
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  griddep_wait();
  griddep_launch();
  // work-list length: a launch parameter, or (CUDA-graph buckets) read from the
  // device and clamped to the capacity the launch was sized for
  const int n_items = (n_tiles_dev ? min(max(__ldg(n_tiles_dev), 0), n_tiles) : n_tiles) * 16;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      int g = 0, i = 0;
      bool ok = true;
      ItemFeed feed;
      for (bool have = feed.init(src, tiles, chunk, n_items, sched); have && ok;
           have = feed.advance(), ++i) {
        const AttnItem a = feed.cur;
        const int qb = i & 1;
        if (!mbar_wait(smem_u32(&q_empty[qb]), ((i >> 1) & 1) ^ 1, 221, abort_flag)) { ok = false; break; }
        mbar_arrive_expect_tx(smem_u32(&q_full[qb]), kTcSmemQ);
        tma_load_2d(sQ + qb * kTcSmemQ, &tmQ, smem_u32(&q_full[qb]), a.head * 64, a.base + a.q0);
        for (int j = 0; j < a.n_kv; ++j, ++g) {
          const int st = g % kTcKvStages;
          if (!mbar_wait(smem_u32(&kv_empty[st]), ((g / kTcKvStages) & 1) ^ 1, 222, abort_flag)) { ok = false; break; }
          const uint32_t fb = smem_u32(&kv_full[st]);
          mbar_arrive_expect_tx(fb, 2 * kTcSmemKV);
          tma_load_2d(sK + st * kTcSmemKV, &tmKV, fb, k_col + a.head * 64, a.kvb + j * kTcKv);
          tma_load_2d(sV + st * kTcSmemKV, &tmKV, fb, v_col + a.head * 64, a.kvb + j * kTcKv);
        }
      }
      // wait for our own copies before the CTA may exit (all phases already issued)
      for (int k = (g > kTcKvStages ? g - kTcKvStages : 0); k < g; ++k)
        mbar_wait(smem_u32(&kv_full[k % kTcKvStages]), (k / kTcKvStages) & 1, 223, nullptr);
      for (int k = (i > 2 ? i - 2 : 0); k < i; ++k) mbar_wait(smem_u32(&q_full[k & 1]), (k >> 1) & 1, 224, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer: S of the next tile, then P.V of the current one
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, kTcKv, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, kTcOCols, false, true);  // [V|1] is MN-major
      struct Cur {
        int it, i, j, n_kv;
      };
      // the S cursor runs at most one tile ahead of the P.V cursor, and the feed
      // follows the S cursor's item
      ItemFeed feed;
      auto first = [&](Cur& c) -> bool {
        c.i = 0;
        c.j = 0;
        if (!feed.init(src, tiles, chunk, n_items, sched)) return false;
        c.it = feed.it;
        c.n_kv = feed.cur.n_kv;
        return true;
      };
      auto next = [&](Cur& c) -> bool {
        if (++c.j < c.n_kv) return true;
        if (!feed.advance()) return false;
        c.it = feed.it;
        c.i += 1;
        c.j = 0;
        c.n_kv = feed.cur.n_kv;
        return true;
      };
      auto issue_s = [&](const Cur& c, int g) -> bool {
        const int qb = c.i & 1;
        if (c.j == 0 && !mbar_wait(smem_u32(&q_full[qb]), (c.i >> 1) & 1, 225, abort_flag)) return false;
        if (!mbar_wait(smem_u32(&kv_full[g % kTcKvStages]), (g / kTcKvStages) & 1, 226, abort_flag)) return false;
        if (g > 0 && !mbar_wait(smem_u32(s_empty), (g - 1) & 1, 227, abort_flag)) return false;
        tc_fence_after();
        const uint64_t dq = sdesc_sw128(sQ + qb * kTcSmemQ);
        const uint64_t dk = sdesc_sw128(sK + (g % kTcKvStages) * kTcSmemKV);
#pragma unroll
        for (int k = 0; k < 4; ++k) umma_bf16(tmem, dq + 2 * k, dk + 2 * k, idesc_s, k != 0);
        umma_commit(smem_u32(s_full));
        if (c.j == c.n_kv - 1) umma_commit(smem_u32(&q_empty[qb]));  // Q free once this S is done
        return true;
      };
      auto issue_pv = [&](const Cur& c, int g) -> bool {
        const int ob = c.i & 1;
        if (!mbar_wait(smem_u32(p_full), g & 1, 228, abort_flag)) return false;
        if (c.j == 0 && !mbar_wait(smem_u32(&o_empty[ob]), ((c.i >> 1) & 1) ^ 1, 229, abort_flag)) return false;
        tc_fence_after();
        const uint32_t va = sV + (g % kTcKvStages) * kTcSmemKV;
        const uint64_t dv = sdesc_sw128_lbo(va, sOnes - va);
#pragma unroll
        for (int k = 0; k < 4; ++k)  // 16 keys per step: P +8 TMEM columns, V +2048 B (16 rows of 128 B)
          umma_bf16_ts(tmem + kTcColO + ob * kTcOCols, tmem + kTcColP + 8 * k, dv + 128 * k, idesc_o,
                       (c.j | k) != 0);
        umma_commit(smem_u32(o_done));
        umma_commit(smem_u32(&kv_empty[g % kTcKvStages]));
        if (c.j == c.n_kv - 1) umma_commit(smem_u32(&o_final[ob]));  // the item's O is complete
        return true;
      };
      Cur pc, sc;
      bool have = first(pc);
      sc = pc;
      bool ok = !have || issue_s(sc, 0);
      int g = 0;
      while (have && ok) {
        sc = pc;
        const bool more = next(sc);
        if (more && !issue_s(sc, g + 1)) break;
        if (!issue_pv(pc, g)) break;
        pc = sc;
        have = more;
        ++g;
      }
      umma_commit(smem_u32(drain));
      mbar_wait(smem_u32(drain), 0, 230, nullptr);
    }
  } else {
    // ---------------- softmax warps 2..5: TMEM lane quarter qd = warp % 4, one query row per lane
    const int qd = warp & 3;
    const int r = qd * 32 + lane;  // row within the tile = TMEM lane
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(qd * 32) << 16);
    const float sl2 = 0.125f * kLog2e;  // softmax scale in log2 units
    int g = 0, i = 0;
    bool ok = true;
    // An item's output is read from TMEM after the next item's first tile: by
    // then its last P.V has long finished (o_final), so that wait is off the
    // critical path.  The pending item's O buffer is not written again before
    // that read (its next user is two items later and waits for o_empty).
    bool pend = false;
    int p_i = 0, p_row = 0;
    long p_out = 0;
    auto epilogue = [&]() -> bool {
      if (!mbar_wait(smem_u32(&o_final[p_i & 1]), (p_i >> 1) & 1, 234, abort_flag)) return false;
      tc_fence_after();
      const uint32_t po = lane_base + kTcColO + (p_i & 1) * kTcOCols;
      // two 32-column halves, then the row sum (column 64); O is released after the last read
      uint32_t oa[32];
      const uint32_t lsum = tmem_ld1(po + 64);
      tmem_ld32(po, oa);
      tmem_wait_ld();
      const float l = __uint_as_float(lsum);
      const float inv = l > 0.f ? 1.f / l : 0.f;
      bf16* orow = out + p_out;
      if (p_row) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint4 u;
          u.x = pack_bf16x2(__uint_as_float(oa[8 * c]) * inv, __uint_as_float(oa[8 * c + 1]) * inv);
          u.y = pack_bf16x2(__uint_as_float(oa[8 * c + 2]) * inv, __uint_as_float(oa[8 * c + 3]) * inv);
          u.z = pack_bf16x2(__uint_as_float(oa[8 * c + 4]) * inv, __uint_as_float(oa[8 * c + 5]) * inv);
          u.w = pack_bf16x2(__uint_as_float(oa[8 * c + 6]) * inv, __uint_as_float(oa[8 * c + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + 8 * c) = u;
        }
      }
      tmem_ld32(po + 32, oa);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&o_empty[p_i & 1]));
      if (p_row) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint4 u;
          u.x = pack_bf16x2(__uint_as_float(oa[8 * c]) * inv, __uint_as_float(oa[8 * c + 1]) * inv);
          u.y = pack_bf16x2(__uint_as_float(oa[8 * c + 2]) * inv, __uint_as_float(oa[8 * c + 3]) * inv);
          u.z = pack_bf16x2(__uint_as_float(oa[8 * c + 4]) * inv, __uint_as_float(oa[8 * c + 5]) * inv);
          u.w = pack_bf16x2(__uint_as_float(oa[8 * c + 6]) * inv, __uint_as_float(oa[8 * c + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + 32 + 8 * c) = u;
        }
      }
      pend = false;
      return true;
    };
    ItemFeed feed;
    for (bool have = feed.init(src, tiles, chunk, n_items, sched); have && ok;
         have = feed.advance(), ++i) {
      const AttnItem a = feed.cur;
      const int qa = a.q0 + r;                                   // local query row
      const int qabs = a.pos0 + qa;                              // its absolute position
      const int lim = chunk > 0 ? min(a.Lkv, (qabs / chunk + 1) * chunk) : a.Lkv;  // visible keys [0, lim)
      const int wlim = __reduce_max_sync(0xffffffffu, lim);                    // any row of this warp
      const uint32_t o_addr = lane_base + kTcColO + (i & 1) * kTcOCols;
      float m_ref = -INFINITY;
      for (int j = 0; j < a.n_kv; ++j, ++g) {
        if (!mbar_wait(smem_u32(s_full), g & 1, 231, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const int k0 = j * kTcKv;
        const bool hi = wlim > k0 + 32;  // warp-uniform: keys k0+32.. visible to some row
        uint32_t s0[32], s1[32];
        tmem_ld32(lane_base, s0);
        if (hi) tmem_ld32(lane_base + 32, s1);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(s_empty));
        const int nvis = lim - k0;
        if (nvis < 64) {
#pragma unroll
          for (int c = 0; c < 32; ++c)
            if (c >= nvis) s0[c] = __float_as_uint(-INFINITY);
          if (hi) {
#pragma unroll
            for (int c = 0; c < 32; ++c)
              if (c + 32 >= nvis) s1[c] = __float_as_uint(-INFINITY);
          }
        }
        float m4[4];
#pragma unroll
        for (int t = 0; t < 4; ++t)
          m4[t] = fmax3(fmax3(__uint_as_float(s0[8 * t]), __uint_as_float(s0[8 * t + 1]), __uint_as_float(s0[8 * t + 2])),
                        fmax3(__uint_as_float(s0[8 * t + 3]), __uint_as_float(s0[8 * t + 4]), __uint_as_float(s0[8 * t + 5])),
                        fmaxf(__uint_as_float(s0[8 * t + 6]), __uint_as_float(s0[8 * t + 7])));
        if (hi) {
#pragma unroll
          for (int t = 0; t < 4; ++t)
            m4[t] = fmax3(m4[t],
                          fmax3(__uint_as_float(s1[8 * t]), __uint_as_float(s1[8 * t + 1]), __uint_as_float(s1[8 * t + 2])),
                          fmax3(fmax3(__uint_as_float(s1[8 * t + 3]), __uint_as_float(s1[8 * t + 4]),
                                      __uint_as_float(s1[8 * t + 5])),
                                __uint_as_float(s1[8 * t + 6]), __uint_as_float(s1[8 * t + 7])));
        }
        const float m_tile = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * sl2;
        const bool need = m_tile > m_ref + kRescaleThreshold;
        const float m_new = need ? m_tile : m_ref;
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          // rescale this row of O and its sum column: wait for P_{g-1} [V|1], then scale
          if (!mbar_wait(smem_u32(o_done), (g - 1) & 1, 232, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const float alpha = need ? ex2_approx(m_ref - m_new) : 1.0f;
          // O columns 0..63 in two pieces, then the sum column (rare path: one buffer)
#pragma unroll 1
          for (int piece = 0; piece < 2; ++piece) {
            uint32_t oa[32];
            tmem_ld32(o_addr + 32 * piece, oa);
            tmem_wait_ld();
#pragma unroll
            for (int d = 0; d < 32; ++d) oa[d] = __float_as_uint(__uint_as_float(oa[d]) * alpha);
            tmem_st32(o_addr + 32 * piece, oa);
          }
          const uint32_t lsum = tmem_ld1(o_addr + 64);
          tmem_wait_ld();
          tmem_st1(o_addr + 64, __float_as_uint(__uint_as_float(lsum) * alpha));
          tmem_wait_st();
        }
        m_ref = m_new;
        const float mo = m_ref == -INFINITY ? 0.f : m_ref;
        uint32_t pw[32];  // P_g of this row: 64 keys as bf16 pairs
#pragma unroll
        for (int c = 0; c < 16; ++c)
          pw[c] = pack_bf16x2(ex2_approx(fmaf(__uint_as_float(s0[2 * c]), sl2, -mo)),
                              ex2_approx(fmaf(__uint_as_float(s0[2 * c + 1]), sl2, -mo)));
        if (hi) {
#pragma unroll
          for (int c = 0; c < 16; ++c)
            pw[16 + c] = pack_bf16x2(ex2_approx(fmaf(__uint_as_float(s1[2 * c]), sl2, -mo)),
                                     ex2_approx(fmaf(__uint_as_float(s1[2 * c + 1]), sl2, -mo)));
        } else {
#pragma unroll
          for (int c = 16; c < 32; ++c) pw[c] = 0u;
        }
        // P_g -> TMEM; its columns were last read by P.V of tile g-1
        if (g >= 1 && !mbar_wait(smem_u32(o_done), (g - 1) & 1, 233, abort_flag)) { ok = false; break; }
        tc_fence_after();
        tmem_st32(lane_base + kTcColP, pw);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(p_full));
        if (pend && !epilogue()) { ok = false; break; }
      }
      if (!ok) break;
      pend = true;
      p_i = i;
      p_row = qa < a.L;
      p_out = (long)(a.base + qa) * 1024 + a.head * 64;
    }
    if (ok && pend) epilogue();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ------------------------------------------------------------------ fp32 (CUDA cores)
// One thread per query row (128 per CTA), 32-key tiles in shared memory.
__global__ void __launch_bounds__(128) attn_f32_kernel(const float* __restrict__ qkv, const AttnSrc src,
                                                       const float* __restrict__ kv, long kv_rows, long kv_stride,
                                                       int k_col, int v_col, const int2* __restrict__ tiles,
                                                       const int32_t* __restrict__ n_tiles_dev, int chunk,
                                                       float* __restrict__ out) {
  griddep_wait();
  griddep_launch();
  if (n_tiles_dev && (int)blockIdx.x >= __ldg(n_tiles_dev)) return;  // grid sized for the capacity
  __shared__ float sK[32][64];
  __shared__ float sV[32][64];
  const AttnItem a = attn_item_at(src, tiles[blockIdx.x], chunk, (int)blockIdx.y);
  const int head = blockIdx.y;
  const int q = a.q0 + threadIdx.x;  // local query row
  const bool valid = q < a.L;
  float qv[64], o[64];
  const float* qrow = qkv + (long)(a.base + (valid ? q : 0)) * kQkvStride + head * 64;
#pragma unroll
  for (int d = 0; d < 64; ++d) {
    qv[d] = qrow[d] * 0.125f;
    o[d] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const int kv_end = a.n_kv * kTcKv < a.Lkv ? a.n_kv * kTcKv : a.Lkv;
  const int qabs = a.pos0 + q;
  const int my_end = valid ? (chunk > 0 ? min(a.Lkv, (qabs / chunk + 1) * chunk) : a.Lkv) : 0;
  for (int k0 = 0; k0 < kv_end; k0 += 32) {
    __syncthreads();
    for (int i = threadIdx.x; i < 32 * 64; i += 128) {
      const int r = i >> 6, c = i & 63;
      const int k = k0 + r;
      const long row = (long)a.kvb + k;
      const bool in = k < a.Lkv && row >= 0 && row < kv_rows;  // rows outside the buffer read as 0
      const long off = (in ? row : 0) * kv_stride + head * 64 + c;
      sK[r][c] = in ? kv[off + k_col] : 0.f;
      sV[r][c] = in ? kv[off + v_col] : 0.f;
    }
    __syncthreads();
    const int kmax = min(32, my_end - k0);
    for (int kk = 0; kk < kmax; ++kk) {
      float sdot = 0.f;
#pragma unroll
      for (int d = 0; d < 64; ++d) sdot = fmaf(qv[d], sK[kk][d], sdot);
      const float m_new = fmaxf(m, sdot);
      const float corr = expf(m - m_new);
      const float pexp = expf(sdot - m_new);
      l = l * corr + pexp;
#pragma unroll
      for (int d = 0; d < 64; ++d) o[d] = fmaf(pexp, sV[kk][d], o[d] * corr);
      m = m_new;
    }
  }
  if (valid) {
    const float inv = 1.f / l;
    float* orow = out + (long)(a.base + q) * 1024 + head * 64;
#pragma unroll
    for (int d = 0; d < 64; ++d) orow[d] = o[d] * inv;
  }
}

}  // namespace fcv
