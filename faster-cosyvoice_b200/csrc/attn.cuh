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
// Work list: (384-row query block, head) items; blocks come from the host as
// (doc, q0) pairs ordered by cost, most expensive first.
#pragma once

#include "fcv_common.cuh"

namespace fcv {

constexpr int kQkvStride = 3072;
constexpr int kAttnQTile = 384;  // query rows of one work-list entry

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
// Work list: (doc, q0) entries of up to kAttnQTile = 384 query rows, most
// expensive first; an item is an entry and one head.  Its rows form three
// 128-row query tiles (TMEM lanes) that share every K/V tile.
constexpr int kFaTiles = 3;    // query tiles per item
constexpr int kFaRows = 128;   // rows of one query tile
constexpr int kFaKv = 64;      // keys of one K/V tile (S tiles are 128 x 64)
constexpr int kFaStages = 6;   // K/V ring depth (4 to 8 measured within 1 %; 6 best on short chunked documents)
constexpr int kFaSmemQ = kFaTiles * kFaRows * 128;  // the query tiles of an item, 48 KB
constexpr int kFaSmemKV = kFaKv * 128;               // one K or V tile, 8 KB
constexpr int kFaOffK = 2 * kFaSmemQ;                // Q of two items in flight
constexpr int kFaOffV = kFaOffK + kFaStages * kFaSmemKV;
constexpr int kFaOffBar = kFaOffV + kFaStages * kFaSmemKV;
static_assert(kAttnQTile == kFaTiles * kFaRows, "work-list entries are whole items");
// mbarriers, per query tile t where indexed [kFaTiles]
constexpr int kFbQFull = 0, kFbQEmpty = 2, kFbKvFull = 4, kFbKvEmpty = kFbKvFull + kFaStages;
constexpr int kFbSFull = kFbKvEmpty + kFaStages, kFbSEmpty = kFbSFull + kFaTiles, kFbPFull = kFbSEmpty + kFaTiles;
constexpr int kFbODone = kFbPFull + kFaTiles, kFbOFinal = kFbODone + kFaTiles, kFbOEmpty = kFbOFinal + kFaTiles;
constexpr int kFaRing = 4;  // slots of the work-item ring
constexpr int kFbInfoFull = kFbOEmpty + kFaTiles, kFbInfoEmpty = kFbInfoFull + kFaRing;
constexpr int kFbDrain = kFbInfoEmpty + kFaRing, kFbCount = kFbDrain + kFaTiles;
// barrier area: the mbarriers, the TMEM slot and abort flag, then the item ring
constexpr int kFaRingOff = (kFbCount * 8 + 8 + 15) / 16 * 16;
// TMEM (one CTA per SM): S_t (fp32, 64 columns) at 64 t, P_t (bf16 pairs, 32
// columns) at 192 + 32 t, O_t (fp32, 64 columns) at 288 + 64 t; 480 of 512.
constexpr int kFaColS = 0, kFaColP = kFaTiles * kFaKv, kFaColO = kFaColP + kFaTiles * kFaKv / 2;
static_assert(kFaColO + 64 * kFaTiles <= 512, "TMEM columns");
constexpr int kFaSoftmaxWarps = 4;  // per query tile: one per TMEM lane quarter
// warps 0..11 softmax (query tile = warp / 4); warpgroup 12-15: warp 12 TMA, warp 13 + t
// issues the MMAs of query tile t
constexpr int kFaThreads = 32 * (kFaSoftmaxWarps * kFaTiles + 4);
// Register budgets (setmaxnreg, per warpgroup): launched at 128 per thread
// (512 x 128 = 65,536), the producer warpgroup gives back down to 96 and the
// three softmax warpgroups grow to 136: 4 x 32 x 96 + 12 x 32 x 136 = 64,512.
constexpr int kFaRegsLaunch = 128, kFaRegsProducer = 96, kFaRegsSoftmax = 136;
static_assert(4 * 32 * kFaRegsProducer + kFaTiles * 4 * 32 * kFaRegsSoftmax <= kFaThreads * kFaRegsLaunch,
              "register split exceeds the launch allocation");
constexpr float kRescaleThreshold = 8.0f;  // log2 units
// Exponentials of pairs p with p % 8 < kFaPolyPairs run as a polynomial on the FMA
// pipe, the rest on the special-function unit (16 results per clock per SM, the
// bound of this kernel at head dim 64).  Measured on a B200 for 32 documents of
// 3000 rows: 0 of 8 pairs 682 TFLOP/s, 1 727, 2 741, 3 699, 4 671.
constexpr int kFaPolyPairs = 2;

struct FaItem {
  int base, L, q0, head, pos0, kvb, Lkv;
  int n[kFaTiles];  // key tiles of each query tile (0: the tile lies past the document)
  int nkv;          // key tiles of the item
};
// What the MMA and softmax roles need of an item, published by the TMA thread
// through a ring in shared memory (n[0] == 0 marks the end of the CTA's items).
struct FaSlot {
  int base, L, q0, head, pos0, Lkv;
  int n[kFaTiles];
};
constexpr int kFaBarBytes = (kFaRingOff + kFaRing * static_cast<int>(sizeof(FaSlot)) + 127) / 128 * 128;
constexpr int kFaSmemBytes = 1024 + kFaOffBar + kFaBarBytes;
static_assert(kFaSmemBytes <= 227 * 1024, "attention shared memory");

// Key tiles visible to query rows ending at absolute position q_last.
__device__ __forceinline__ int fa_key_tiles(int q_last, int Lkv, int chunk) {
  const int lim = chunk > 0 ? min(Lkv, (q_last / chunk + 1) * chunk) : Lkv;
  return (lim + kFaKv - 1) / kFaKv;
}

__device__ __forceinline__ FaItem fa_item_at(const AttnSrc& src, int2 tl, int chunk, int it) {
  FaItem a;
  a.head = it & 15;
  a.q0 = tl.y;
  a.base = src.cu[tl.x];
  a.L = src.cu[tl.x + 1] - a.base;
  a.pos0 = src.pos0 ? __ldg(src.pos0 + tl.x) : 0;
  a.kvb = src.kv_base ? __ldg(src.kv_base + tl.x) : a.base;
  a.Lkv = a.pos0 + a.L;
  a.nkv = 0;
#pragma unroll
  for (int t = 0; t < kFaTiles; ++t) {
    const int r0 = a.q0 + kFaRows * t;
    a.n[t] = r0 < a.L ? fa_key_tiles(a.pos0 + min(r0 + kFaRows - 1, a.L - 1), a.Lkv, chunk) : 0;
    a.nkv = max(a.nkv, a.n[t]);
  }
  return a;
}

// A CTA's items with the descriptor lookups run ahead (used by the TMA thread,
// which publishes each item to the others): while item `it` is processed, the
// item after it is already resolved and the work-list entry of the one after
// that is loading.  Items come round robin (first, first + stride, ... of the
// work list) or from a host-built schedule: positions [beg, end) of a per-CTA
// item list.
struct FaFeed {
  AttnSrc src;
  const int2* tiles;
  const int32_t* list;  // schedule items, or null for round robin
  int chunk, end, stride, pos, it, it1, it2;
  FaItem cur, nxt;
  int2 tl2;
  __device__ __forceinline__ int item_at(int p) const { return list ? __ldg(list + p) : p; }
  // Round robin when sched is null; else sched = [offsets (gridDim + 1) | items].
  __device__ __forceinline__ bool init(const AttnSrc& src_, const int2* tiles_, int chunk_, int n_items,
                                       const int32_t* sched) {
    src = src_;
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
    cur = fa_item_at(src, tiles[it >> 4], chunk, it);
    if (pos + stride < end) {
      it1 = item_at(pos + stride);
      nxt = fa_item_at(src, tiles[it1 >> 4], chunk, it1);
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
      nxt = fa_item_at(src, tl2, chunk, it1);
    }
    if (pos + 2 * stride < end) {
      it2 = item_at(pos + 2 * stride);
      tl2 = tiles[it2 >> 4];
    }
    return true;
  }
};

// ---- packed float32 pairs (sm_100 f32x2 instructions: one issue slot per pair)
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                     float c1) {
  asm("{\n\t.reg .b64 a, b, c, d;\n\t"
      "mov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\tmov.b64 c, {%6, %7};\n\t"
      "fma.rn.f32x2 d, a, b, c;\n\tmov.b64 {%0, %1}, d;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
__device__ __forceinline__ void add2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 a, b, d;\n\t"
      "mov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
      "add.rn.f32x2 d, a, b;\n\tmov.b64 {%0, %1}, d;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 2^x for a pair on the FMA pipe.  Range reduction x = n + f with n = rint(x)
// (adding 1.5 * 2^23 leaves rint(x) in the low mantissa bits), f in [-1/2, 1/2];
// 2^f from a cubic with p(0) = 1 whose other coefficients minimise the maximum
// relative error on [-1/2, 1/2] (a linear program; max 1.0e-4, far below the
// bf16 rounding of P); 2^n by adding n to the exponent field.  x is clamped at
// -127: there f = 0 and p = 1 exactly, so the sum of the fields is +0.0 -- the
// -inf of a masked key gives exactly 0, like ex2 -- and every x >= -127 keeps a
// non-negative exponent field.
__device__ __forceinline__ void exp2_poly2(float x0, float x1, float& y0, float& y1) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  constexpr float c1 = 0.6932829022407532f, c2 = 0.2422109693288803f, c3 = 0.055009059607982635f;
  x0 = fmaxf(x0, -127.0f);
  x1 = fmaxf(x1, -127.0f);
  float t0, t1, n0, n1, f0, f1, p0, p1;
  add2(t0, t1, x0, x1, kRound, kRound);
  add2(n0, n1, t0, t1, -kRound, -kRound);
  fma2(f0, f1, n0, n1, -1.0f, -1.0f, x0, x1);
  fma2(p0, p1, c3, c3, f0, f1, c2, c2);
  fma2(p0, p1, p0, p1, f0, f1, c1, c1);
  fma2(p0, p1, p0, p1, f0, f1, 1.0f, 1.0f);
  y0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  y1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}

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

// Persistent, one CTA per SM.  Per item (three 128-row query tiles of one head):
//   warp 12  TMA: the item's query tiles into one of two buffers, K/V tiles of 64
//            keys into a 6-stage ring shared by the query tiles; it also resolves
//            each item once and publishes it to the other roles (item ring)
//   warp 13+t  issues slot t's tcgen05.mma: S_t = Q K_j^T, then O_t += P_t V_j
//            with P_t read from TMEM; S of key tile j+1 is issued before P.V of
//            tile j, so the tensor core works while softmax runs.  One issuer per
//            slot keeps the slots independent (a slot's slow softmax never holds
//            back another slot's MMAs); they share only the K/V ring, whose
//            stages return when every slot is done with them.  Warp 13 also owns
//            TMEM.
//   warps 4t..4t+3  softmax of slot t, one row per thread (TMEM lane quarter =
//            warp % 4).  Three warps per SM sub-partition keep the exponential
//            units busy while the others load S, take row maxima or wait.
// Slot t takes query tile (t + i) mod 3 of the CTA's i-th item: under a causal
// chunk mask the last tile of an item sees the most keys, and a short item has
// tiles past its document, so a fixed assignment would give one slot most of the
// work; rotating spreads it, and slots whose tile ends early run ahead into the
// next item as far as the Q buffers and the K/V ring allow.
// Row maxima move only when a tile exceeds the reference max by more than
// kRescaleThreshold (log2 units); O in TMEM and the row sum are then rescaled
// (rare).  An item's O is read after the next item's first P is written (its
// last P.V has finished by then), and that item's first P.V waits for the read.
// Barrier invariant: every wait uses a parity its producer cannot have advanced
// past by two phases.
__global__ void __launch_bounds__(kFaThreads, 1)
    attn_fa_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                   const AttnSrc src, const int2* __restrict__ tiles, int n_tiles,
                   const int32_t* __restrict__ n_tiles_dev, const int32_t* __restrict__ sched, int chunk,
                   int k_col, int v_col, bf16* __restrict__ out) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t s0 = smem_u32(smem);
  const uint32_t sQ = s0, sK = s0 + kFaOffK, sV = s0 + kFaOffV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kFaOffBar);
  auto bar = [&](int i) { return smem_u32(bars + i); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kFbCount);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  FaSlot* ring = reinterpret_cast<FaSlot*>(smem + kFaOffBar + kFaRingOff);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kProducerWarp = kFaSoftmaxWarps * kFaTiles;  // first warp of the producer warpgroup

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(kFbQFull + i), 1);
      mbar_init(bar(kFbQEmpty + i), kFaTiles);  // one arrival per MMA issuer
    }
    for (int t = 0; t < kFaTiles; ++t) {
      mbar_init(bar(kFbSFull + t), 1);
      mbar_init(bar(kFbSEmpty + t), kFaSoftmaxWarps);
      mbar_init(bar(kFbPFull + t), kFaSoftmaxWarps);
      mbar_init(bar(kFbODone + t), 1);
      mbar_init(bar(kFbOFinal + t), 1);
      mbar_init(bar(kFbOEmpty + t), kFaSoftmaxWarps);
    }
    for (int i = 0; i < kFaStages; ++i) {
      mbar_init(bar(kFbKvFull + i), 1);
      mbar_init(bar(kFbKvEmpty + i), kFaTiles);  // one arrival per MMA issuer
    }
    for (int i = 0; i < kFaRing; ++i) {
      mbar_init(bar(kFbInfoFull + i), 1);
      mbar_init(bar(kFbInfoEmpty + i), kFaTiles + kFaSoftmaxWarps * kFaTiles);  // the MMA issuers, every softmax warp
    }
    for (int t = 0; t < kFaTiles; ++t) mbar_init(bar(kFbDrain + t), 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmKV);
  }
  if (warp == kProducerWarp + 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
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

  if (warp >= kProducerWarp) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kFaRegsProducer));
    if (warp == kProducerWarp && lane == 0) {
      // ---------------- TMA producer
      int g = 0, i = 0;
      bool ok = true;
      FaFeed feed;
      auto publish = [&](const FaItem& a, bool last) -> bool {
        const int sl = i % kFaRing;
        if (!mbar_wait(bar(kFbInfoEmpty + sl), ((i / kFaRing) & 1) ^ 1, 240, abort_flag)) return false;
        FaSlot& o = ring[sl];
        o.base = a.base, o.L = a.L, o.q0 = a.q0, o.head = a.head, o.pos0 = a.pos0, o.Lkv = a.Lkv;
#pragma unroll
        for (int t = 0; t < kFaTiles; ++t) o.n[t] = a.n[t];
        if (last) o.n[0] = 0;
        mbar_arrive(bar(kFbInfoFull + sl));
        return true;
      };
      bool have = feed.init(src, tiles, chunk, n_items, sched);
      for (; have && ok; have = feed.advance(), ++i) {
        const FaItem a = feed.cur;
        const int qb = i & 1;
        if (!publish(a, false)) { ok = false; break; }
        if (!mbar_wait(bar(kFbQEmpty + qb), ((i >> 1) & 1) ^ 1, 241, abort_flag)) { ok = false; break; }
        mbar_arrive_expect_tx(bar(kFbQFull + qb), kFaSmemQ);
#pragma unroll
        for (int t = 0; t < kFaTiles; ++t)  // tiles past the document load rows of the next one (or zeros): unused
          tma_load_2d(sQ + qb * kFaSmemQ + t * kFaRows * 128, &tmQ, bar(kFbQFull + qb), a.head * 64,
                      a.base + a.q0 + kFaRows * t);
        for (int j = 0; j < a.nkv; ++j, ++g) {
          const int st = g % kFaStages;
          if (!mbar_wait(bar(kFbKvEmpty + st), ((g / kFaStages) & 1) ^ 1, 242, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(bar(kFbKvFull + st), 2 * kFaSmemKV);
          tma_load_2d(sK + st * kFaSmemKV, &tmKV, bar(kFbKvFull + st), k_col + a.head * 64, a.kvb + j * kFaKv);
          tma_load_2d(sV + st * kFaSmemKV, &tmKV, bar(kFbKvFull + st), v_col + a.head * 64, a.kvb + j * kFaKv);
        }
      }
      if (ok) publish(FaItem{}, true);  // end of the CTA's items
      // wait for our own copies before the CTA may exit (all phases already issued)
      for (int k = (g > kFaStages ? g - kFaStages : 0); k < g; ++k)
        mbar_wait(bar(kFbKvFull + k % kFaStages), (k / kFaStages) & 1, 243, nullptr);
      for (int k = (i > 2 ? i - 2 : 0); k < i; ++k) mbar_wait(bar(kFbQFull + (k & 1)), (k >> 1) & 1, 244, nullptr);
    } else if (warp > kProducerWarp && warp <= kProducerWarp + kFaTiles && lane == 0) {
      // ---------------- MMA issuer of query tile t
      const int t = warp - kProducerWarp - 1;
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, kFaKv, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, 64, false, true);  // V is MN-major
      int sc = 0, pvc = 0, items_t = 0;  // S / P.V tiles issued, items having this tile
      // pending P.V (issued after S of the next key tile) of key tile pv_g
      int pv_g = 0, pv_item = 0;
      bool pv_on = false, pv_first = false, pv_last = false, ok = true, pend = false;
      // P.V of the pending key tile (if this tile has one), then its K/V stage returned
      auto issue_pv = [&]() -> bool {
        if (pv_on) {
          if (!mbar_wait(bar(kFbPFull + t), pvc & 1, 245, abort_flag)) return false;
          if (pv_first && !mbar_wait(bar(kFbOEmpty + t), (pv_item & 1) ^ 1, 246, abort_flag)) return false;
          tc_fence_after();
          const uint64_t dv = sdesc_sw128(sV + (pv_g % kFaStages) * kFaSmemKV);
#pragma unroll
          for (int k = 0; k < kFaKv / 16; ++k)  // 16 keys per step: P +8 TMEM columns, V +2048 B (16 rows of 128 B)
            umma_bf16_ts(tmem + kFaColO + 64 * t, tmem + kFaColP + (kFaKv / 2) * t + 8 * k, dv + 128 * k, idesc_o,
                         (!pv_first || k != 0) ? 1u : 0u);
          umma_commit(bar(kFbODone + t));
          if (pv_last) umma_commit(bar(kFbOFinal + t));
          ++pvc;
          umma_commit(bar(kFbKvEmpty + pv_g % kFaStages));  // after this tile's MMAs that read the stage
        } else {
          mbar_arrive(bar(kFbKvEmpty + pv_g % kFaStages));  // this tile never read the stage
        }
        return true;
      };
      int g = 0;
      for (int i = 0; ok; ++i) {
        const int sl = i % kFaRing;
        if (!mbar_wait(bar(kFbInfoFull + sl), (i / kFaRing) & 1, 239, abort_flag)) { ok = false; break; }
        const FaSlot a = ring[sl];
        mbar_arrive(bar(kFbInfoEmpty + sl));
        if (a.n[0] == 0) break;  // no more items
        const int rt = (t + i) % kFaTiles;  // the item's query tile this issuer takes (rotates per item)
        int nkv = 0, nt = 0;
#pragma unroll
        for (int u = 0; u < kFaTiles; ++u) {
          nkv = max(nkv, a.n[u]);
          if (u == rt) nt = a.n[u];
        }
        const int qb = i & 1;
        // Arrivals that release a Q buffer or a K/V stage without an MMA behind them
        // come only after that buffer's load completed: the load cannot complete
        // before the buffer's previous phase did, so no issuer can arrive twice in
        // one phase however far ahead of the others it runs.
        if (!mbar_wait(bar(kFbQFull + qb), (i >> 1) & 1, 247, abort_flag)) { ok = false; break; }
        if (nt == 0) mbar_arrive(bar(kFbQEmpty + qb));  // this tile reads no Q of the item
        for (int j = 0; j < nkv && ok; ++j, ++g) {
          const int st = g % kFaStages;
          if (!mbar_wait(bar(kFbKvFull + st), (g / kFaStages) & 1, 248, abort_flag)) { ok = false; break; }
          if (j < nt) {
            if (sc > 0 && !mbar_wait(bar(kFbSEmpty + t), (sc - 1) & 1, 249, abort_flag)) { ok = false; break; }
            tc_fence_after();
            const uint64_t dq = sdesc_sw128(sQ + qb * kFaSmemQ + rt * kFaRows * 128);
            const uint64_t dk = sdesc_sw128(sK + st * kFaSmemKV);
#pragma unroll
            for (int k = 0; k < 4; ++k) umma_bf16(tmem + kFaColS + kFaKv * t, dq + 2 * k, dk + 2 * k, idesc_s, k != 0);
            umma_commit(bar(kFbSFull + t));
            ++sc;
            if (j == nt - 1) umma_commit(bar(kFbQEmpty + qb));  // Q_t free once this S is done
          }
          if (pend && !issue_pv()) { ok = false; break; }
          pv_g = g;
          pv_on = j < nt;
          pv_first = j == 0;
          pv_last = j == nt - 1;
          pv_item = items_t;
          pend = true;
        }
        items_t += nt > 0 ? 1 : 0;
      }
      if (ok && pend) issue_pv();
      umma_commit(bar(kFbDrain + t));
      mbar_wait(bar(kFbDrain + t), 0, 250, nullptr);
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kFaRegsSoftmax));
    // ---------------- softmax of query tile t: one row per thread
    const int t = warp >> 2;
    const int qd = warp & 3;
    const int r = qd * 32 + lane;  // row within the tile = TMEM lane
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(qd * 32) << 16);
    const uint32_t colS = lane_base + kFaColS + kFaKv * t, colP = lane_base + kFaColP + (kFaKv / 2) * t,
                   colO = lane_base + kFaColO + 64 * t;
    const float sl2 = 0.125f * kLog2e;  // softmax scale in log2 units
    int cnt = 0, it_t = 0;
    bool ok = true;
    // deferred epilogue of the previous item of this tile
    bool pend = false, p_row = false;
    int p_idx = 0;
    long p_out = 0;
    float p_l = 1.f;
    auto epilogue = [&]() -> bool {
      if (!mbar_wait(bar(kFbOFinal + t), p_idx & 1, 251, abort_flag)) return false;
      tc_fence_after();
      const float inv = p_l > 0.f ? 1.f / p_l : 0.f;
      bf16* orow = out + p_out;
      // four 16-column pieces, each stored as it arrives; O is released after the last read
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t o[16];
        tmem_ld16(colO + 16 * c, o);
        tmem_wait_ld();
        if (c == 3) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(kFbOEmpty + t));
        }
        if (p_row) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            uint4 u;
            u.x = pack_bf16x2(__uint_as_float(o[8 * h + 0]) * inv, __uint_as_float(o[8 * h + 1]) * inv);
            u.y = pack_bf16x2(__uint_as_float(o[8 * h + 2]) * inv, __uint_as_float(o[8 * h + 3]) * inv);
            u.z = pack_bf16x2(__uint_as_float(o[8 * h + 4]) * inv, __uint_as_float(o[8 * h + 5]) * inv);
            u.w = pack_bf16x2(__uint_as_float(o[8 * h + 6]) * inv, __uint_as_float(o[8 * h + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + 16 * c + 8 * h) = u;
          }
        }
      }
      pend = false;
      return true;
    };
    for (int i = 0; ok; ++i) {
      const int sl = i % kFaRing;
      if (!mbar_wait(bar(kFbInfoFull + sl), (i / kFaRing) & 1, 238, abort_flag)) { ok = false; break; }
      const FaSlot a = ring[sl];
      __syncwarp();
      if (lane == 0) mbar_arrive(bar(kFbInfoEmpty + sl));
      if (a.n[0] == 0) break;  // no more items
      const int rt = (t + i) % kFaTiles;  // the item's query tile this slot takes (rotates per item)
      int ntile = 0;
#pragma unroll
      for (int u = 0; u < kFaTiles; ++u)
        if (u == rt) ntile = a.n[u];
      if (ntile == 0) continue;  // this query tile lies past the document
      const int qa = a.q0 + kFaRows * rt + r;  // local query row
      const int qabs = a.pos0 + qa;           // its absolute position
      const int lim = chunk > 0 ? min(a.Lkv, (qabs / chunk + 1) * chunk) : a.Lkv;  // visible keys [0, lim)
      const bool row_ok = qa < a.L;
      const bool warp_rows = __any_sync(0xffffffffu, row_ok);  // the warp has a row of the document
      const int wmax = __reduce_max_sync(0xffffffffu, lim), wmin = __reduce_min_sync(0xffffffffu, lim);
      float m_ref = -INFINITY;
      float lsum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // four independent pair accumulators of the row sum
      for (int j = 0; j < ntile; ++j, ++cnt) {
        if (!mbar_wait(bar(kFbSFull + t), cnt & 1, 252, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const int k0 = j * kFaKv;
        // 32-key halves that some row of the warp sees (warp-uniform)
        const int nch = warp_rows ? min(2, max(0, (wmax - k0 + 31) / 32)) : 0;
        uint32_t s[64];
        tmem_ld32(colS, *reinterpret_cast<uint32_t(*)[32]>(s));
        if (nch > 1) tmem_ld32(colS + 32, *reinterpret_cast<uint32_t(*)[32]>(s + 32));
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kFbSEmpty + t));
        if (wmin < k0 + kFaKv) {  // a row of the warp stops inside this tile: mask its invisible keys
          const int nvis = lim - k0;
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c >= nvis) s[c] = __float_as_uint(-INFINITY);
        }
        float mt = -INFINITY;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          if (c < nch) {
            float m8[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const uint32_t* v = s + 32 * c + 8 * u;
              m8[u] = fmax3(fmax3(__uint_as_float(v[0]), __uint_as_float(v[1]), __uint_as_float(v[2])),
                            fmax3(__uint_as_float(v[3]), __uint_as_float(v[4]), __uint_as_float(v[5])),
                            fmaxf(__uint_as_float(v[6]), __uint_as_float(v[7])));
            }
            mt = fmax3(mt, fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3]));
          }
        }
        const float m_tile = mt * sl2;
        const bool need = m_tile > m_ref + kRescaleThreshold;
        const float m_new = need ? m_tile : m_ref;
        // O_t must hold P.V of every earlier key tile before it is rescaled, and P_t is
        // free once P.V of this tile's previous key tile is done: the exponentials
        // below run first, overlapping that P.V, unless a rescale needs O now (rare)
        bool o_ready = cnt == 0;
        if (j > 0 && __any_sync(0xffffffffu, need)) {
          if (!mbar_wait(bar(kFbODone + t), (cnt - 1) & 1, 253, abort_flag)) { ok = false; break; }
          tc_fence_after();
          o_ready = true;
          // rescale this row of O and its sum (the max grew by more than the threshold)
          const float alpha = need ? ex2_approx(m_ref - m_new) : 1.0f;
#pragma unroll 1
          for (int piece = 0; piece < 4; ++piece) {
            uint32_t o[16];
            tmem_ld16(colO + 16 * piece, o);
            tmem_wait_ld();
#pragma unroll
            for (int d = 0; d < 16; ++d) o[d] = __float_as_uint(__uint_as_float(o[d]) * alpha);
            tmem_st16(colO + 16 * piece, o);
          }
          tmem_wait_st();
#pragma unroll
          for (int u = 0; u < 8; ++u) lsum[u] *= alpha;
        }
        m_ref = m_new;
        const float mo = m_ref == -INFINITY ? 0.f : m_ref;
        uint32_t pw[32];  // P of this row: 64 keys as bf16 pairs
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          if (c < nch) {
#pragma unroll
            for (int p = 0; p < 16; ++p) {
              float x0, x1, e0, e1;
              fma2(x0, x1, __uint_as_float(s[32 * c + 2 * p]), __uint_as_float(s[32 * c + 2 * p + 1]), sl2, sl2, -mo,
                   -mo);
              if (p % 8 < kFaPolyPairs) {
                exp2_poly2(x0, x1, e0, e1);
              } else {
                e0 = ex2_approx(x0);
                e1 = ex2_approx(x1);
              }
              add2(lsum[2 * (p & 3)], lsum[2 * (p & 3) + 1], lsum[2 * (p & 3)], lsum[2 * (p & 3) + 1], e0, e1);
              pw[16 * c + p] = pack_bf16x2(e0, e1);
            }
          } else {
#pragma unroll
            for (int p = 0; p < 16; ++p) pw[16 * c + p] = 0u;
          }
        }
        if (!o_ready) {
          if (!mbar_wait(bar(kFbODone + t), (cnt - 1) & 1, 254, abort_flag)) { ok = false; break; }
          tc_fence_after();
        }
        tmem_st32(colP, pw);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(kFbPFull + t));
        if (pend && !epilogue()) { ok = false; break; }
      }
      if (!ok) break;
      pend = true;
      p_idx = it_t++;
      p_row = row_ok;
      p_out = (long)(a.base + qa) * 1024 + a.head * 64;
      p_l = ((lsum[0] + lsum[1]) + (lsum[2] + lsum[3])) + ((lsum[4] + lsum[5]) + (lsum[6] + lsum[7]));
    }
    if (ok && pend) epilogue();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kProducerWarp + 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ fp32 (CUDA cores)
// One thread per query row (384 per CTA: one work-list entry), 32-key tiles in
// shared memory.
__global__ void __launch_bounds__(kAttnQTile) attn_f32_kernel(const float* __restrict__ qkv, const AttnSrc src,
                                                              const float* __restrict__ kv, long kv_rows,
                                                              long kv_stride, int k_col, int v_col,
                                                              const int2* __restrict__ tiles,
                                                              const int32_t* __restrict__ n_tiles_dev, int chunk,
                                                              float* __restrict__ out) {
  griddep_wait();
  griddep_launch();
  if (n_tiles_dev && (int)blockIdx.x >= __ldg(n_tiles_dev)) return;  // grid sized for the capacity
  __shared__ float sK[32][64];
  __shared__ float sV[32][64];
  const FaItem a = fa_item_at(src, tiles[blockIdx.x], chunk, (int)blockIdx.y);
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
  const int kv_end = a.nkv * kFaKv < a.Lkv ? a.nkv * kFaKv : a.Lkv;
  const int qabs = a.pos0 + q;
  const int my_end = valid ? (chunk > 0 ? min(a.Lkv, (qabs / chunk + 1) * chunk) : a.Lkv) : 0;
  for (int k0 = 0; k0 < kv_end; k0 += 32) {
    __syncthreads();
    for (int i = threadIdx.x; i < 32 * 64; i += blockDim.x) {
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
