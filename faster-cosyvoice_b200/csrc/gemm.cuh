// gemm.cuh -- GEMMs of the DiT estimator with fused epilogues.
//
//   bf16: persistent tcgen05 kernel.  One CTA per SM, 6 warps:
//         warp 0 issues TMA loads of A/B k-blocks into a multi-stage ring,
//         warp 1 owns TMEM and issues tcgen05.mma (128 x BN x 16) into one of
//         two TMEM accumulators, warps 2-5 drain the other accumulator with
//         tcgen05.ld and run the epilogue (bias, GELU, partial RoPE, gated
//         residual, Mish, unpack) straight to global memory.
//   f32:  CUDA-core FFMA tiles with the same epilogues (the exact-fp32 mode;
//         tcgen05 has no fp32-input kind).
//
// "Conv" mode turns the kernel into the implicit GEMM of the causal grouped
// position convolution (modules.py:115-144): A is a *gapped* activation
// buffer in which each document is preceded by 30 zero rows, output tile
// column block g (64 wide) is convolution group g, and k-block t (64 wide) is
// tap t, whose A tile is the same 64 columns shifted by t - 30 rows.
#pragma once

#include "fcv_common.cuh"

namespace fcv {

enum Epi : int {
  EPI_BIAS = 0,       // C(act) = acc + b
  EPI_GELU = 1,       // C(act) = gelu_tanh(acc + b)
  EPI_ROPE = 2,       // C(act) = acc + b with partial RoPE on columns [0,64) and [1024,1088)
  EPI_GATE_RES = 3,   // h(f32)[row] += gate[doc] * (acc + b)
  EPI_F32 = 4,        // C(f32) = acc + b
  EPI_EMBED_GAP = 5,  // C(act)[row + 30*(doc+1)] = acc + b   (embed -> gapped buffer)
  EPI_MISH_GAP = 6,   // gapped row g: C(act)[g] = mish(acc + b) unless gap_rows[g] < 0
  EPI_MISH_RES = 7,   // gapped row g, packed p = gap_rows[g] >= 0: h(f32)[p] = mish(acc+b) + res[g]
  EPI_UNPACK = 8,     // out(act)[doc, col, pos] = acc + b   (proj_out -> (B, 80, T))
  EPI_SILU = 9,       // C(act) = silu(acc + b)
  EPI_LRELU = 10,     // C(act) = leaky_relu(acc + b, 0.01)   (pre-lookahead conv1)
};

constexpr int kConvPad = 30;  // kernel_size - 1 zero rows before every document

struct EpiParams {
  int epi;
  int M, N;            // rows of A / columns of C
  void* C;
  long ldc;            // elements
  const float* bias;   // may be null
  const int32_t* aux;  // positions (ROPE), doc_ids (GATE_RES, EMBED_GAP, UNPACK), gap_rows (MISH_*)
  const int32_t* aux2; // positions (UNPACK)
  const void* res;     // gapped residual rows (MISH_RES), act dtype, row stride 1024
  const float* gate;
  long gate_stride;
  const float* rope_cos;
  const float* rope_sin;
  int T;               // padded length (UNPACK)
  void* C2;            // EPI_F32: when set, also C2(act)[row*1024 + col] = silu(acc + b)
  int out_f32;         // EPI_UNPACK: float32 output instead of act
};

// Apply the epilogue to W consecutive columns [col0, col0+W) of one row.
// W is even and col0 is a multiple of W, so RoPE pairs (2j, 2j+1) never split.
template <typename Tact, int W>
__device__ __forceinline__ void epilogue_apply(const EpiParams& p, int row, int col0, float* v) {
  if (row >= p.M) return;
  const bool full = (col0 + W) <= p.N;
  if (p.bias != nullptr) {
#pragma unroll
    for (int j = 0; j < W; ++j)
      if (full || col0 + j < p.N) v[j] += __ldg(p.bias + col0 + j);
  }
  int out_row = row;
  switch (p.epi) {
    case EPI_GELU:
#pragma unroll
      for (int j = 0; j < W; ++j) v[j] = gelu_tanh(v[j]);
      break;
    case EPI_ROPE: {
      const int c = col0 & 1023;
      if (col0 < 2048 && c < 64) {
        const int pos = __ldg(p.aux + row);
#pragma unroll
        for (int j = 0; j < W; j += 2) {
          const int i = (c + j) >> 1;
          if (c + j < 64) {
            const float cs = __ldg(p.rope_cos + (long)pos * 32 + i);
            const float sn = __ldg(p.rope_sin + (long)pos * 32 + i);
            const float a = v[j], b = v[j + 1];
            v[j] = a * cs - b * sn;
            v[j + 1] = b * cs + a * sn;
          }
        }
      }
      break;
    }
    case EPI_GATE_RES: {
      const int doc = __ldg(p.aux + row);
      const float* g = p.gate + (long)doc * p.gate_stride + col0;
      float* h = reinterpret_cast<float*>(p.C) + (long)row * p.ldc + col0;
      if (full && W % 4 == 0) {
#pragma unroll
        for (int j = 0; j < W; j += 4) {
          const float4 gv = __ldg(reinterpret_cast<const float4*>(g + j));
          float4 hv = *reinterpret_cast<float4*>(h + j);
          hv.x += gv.x * v[j];
          hv.y += gv.y * v[j + 1];
          hv.z += gv.z * v[j + 2];
          hv.w += gv.w * v[j + 3];
          *reinterpret_cast<float4*>(h + j) = hv;
        }
      } else {
        for (int j = 0; j < W; ++j)
          if (col0 + j < p.N) h[j] += g[j] * v[j];
      }
      return;
    }
    case EPI_SILU:
#pragma unroll
      for (int j = 0; j < W; ++j) v[j] = silu(v[j]);
      break;
    case EPI_LRELU:
#pragma unroll
      for (int j = 0; j < W; ++j) v[j] = leaky_relu(v[j]);
      break;
    case EPI_F32: {
      if (p.C2 != nullptr) {
        Tact* c2 = reinterpret_cast<Tact*>(p.C2) + (long)row * 1024 + col0;
        for (int j = 0; j < W; ++j)
          if (col0 + j < p.N) c2[j] = from_f<Tact>(silu(v[j]));
      }
      float* c = reinterpret_cast<float*>(p.C) + (long)row * p.ldc + col0;
      if (full && W % 4 == 0) {
#pragma unroll
        for (int j = 0; j < W; j += 4)
          *reinterpret_cast<float4*>(c + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      } else {
        for (int j = 0; j < W; ++j)
          if (col0 + j < p.N) c[j] = v[j];
      }
      return;
    }
    case EPI_EMBED_GAP:
      out_row = row + kConvPad * (__ldg(p.aux + row) + 1);
      break;
    case EPI_MISH_GAP:
      if (__ldg(p.aux + row) < 0) return;
#pragma unroll
      for (int j = 0; j < W; ++j) v[j] = mish(v[j]);
      break;
    case EPI_MISH_RES: {
      const int pr = __ldg(p.aux + row);
      if (pr < 0) return;
      const Tact* r = reinterpret_cast<const Tact*>(p.res) + (long)row * 1024 + col0;
      float* h = reinterpret_cast<float*>(p.C) + (long)pr * p.ldc + col0;
      if constexpr (sizeof(Tact) == 2 && W % 8 == 0) {
        // 16-byte residual loads and stores (rows of 1024, col0 a multiple of W)
#pragma unroll
        for (int j = 0; j < W; j += 8) {
          const uint4 u = *reinterpret_cast<const uint4*>(r + j);
          const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
          float rr[8];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w4[k]));
            rr[2 * k] = f.x;
            rr[2 * k + 1] = f.y;
          }
          *reinterpret_cast<float4*>(h + j) = make_float4(mish(v[j]) + rr[0], mish(v[j + 1]) + rr[1],
                                                          mish(v[j + 2]) + rr[2], mish(v[j + 3]) + rr[3]);
          *reinterpret_cast<float4*>(h + j + 4) = make_float4(mish(v[j + 4]) + rr[4], mish(v[j + 5]) + rr[5],
                                                              mish(v[j + 6]) + rr[6], mish(v[j + 7]) + rr[7]);
        }
      } else {
#pragma unroll
        for (int j = 0; j < W; ++j) h[j] = mish(v[j]) + to_f<Tact>(r[j]);
      }
      return;
    }
    case EPI_UNPACK: {
      const int doc = __ldg(p.aux + row);
      const int pos = __ldg(p.aux2 + row);
      const long off = (long)doc * p.N * p.T + pos;
      if (p.out_f32) {
        float* o = reinterpret_cast<float*>(p.C) + off;
#pragma unroll
        for (int j = 0; j < W; ++j)
          if (col0 + j < p.N) o[(long)(col0 + j) * p.T] = v[j];
      } else {
        Tact* o = reinterpret_cast<Tact*>(p.C) + off;
#pragma unroll
        for (int j = 0; j < W; ++j)
          if (col0 + j < p.N) o[(long)(col0 + j) * p.T] = from_f<Tact>(v[j]);
      }
      return;
    }
    default:
      break;
  }
  // plain activation store at out_row
  Tact* c = reinterpret_cast<Tact*>(p.C) + (long)out_row * p.ldc + col0;
  if constexpr (sizeof(Tact) == 2) {
    if (full && W % 8 == 0) {
#pragma unroll
      for (int j = 0; j < W; j += 8) {
        uint4 u;
        u.x = pack_bf16x2(v[j], v[j + 1]);
        u.y = pack_bf16x2(v[j + 2], v[j + 3]);
        u.z = pack_bf16x2(v[j + 4], v[j + 5]);
        u.w = pack_bf16x2(v[j + 6], v[j + 7]);
        *reinterpret_cast<uint4*>(c + j) = u;
      }
      return;
    }
  } else {
    if (full && W % 4 == 0) {
#pragma unroll
      for (int j = 0; j < W; j += 4)
        *reinterpret_cast<float4*>(c + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      return;
    }
  }
  for (int j = 0; j < W; ++j)
    if (col0 + j < p.N) c[j] = from_f<Tact>(v[j]);
}

// ============================================================== tcgen05 GEMM

struct TcGemmArgs {
  int num_kb;      // k-blocks of 64
  int m_blocks;
  int n_blocks;
  // pair kernel: tiles [0, full_tiles) are 256 x 256; the remaining m_blocks*n_blocks
  // - full_tiles tiles (the last, partial wave) are each split into `split` (1 or 2)
  // pieces of 256 x (256/split), spread over more CTA pairs; num_tiles counts pieces
  int full_tiles;
  int split;
  int num_tiles;
  int conv;        // tc_conv_kernel: set for the causal grouped convolution
  int tma_out;     // 0: direct stores; 1: TMA store of act/f32 tiles; 2: TMA reduce-add into f32 h
  EpiParams epi;
};

template <int BN>
struct TcGemmCfg {
  static constexpr int BM = 128;
  static constexpr int BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI_WARPS = 8;
  // two 32-row x 128-byte staging tiles per epilogue warp (TMA output paths only; BN < 128 stores directly)
  static constexpr int STAGING_BYTES = BN >= 128 ? EPI_WARPS * 8192 : 0;
  static constexpr int BIAS_BYTES = 0;
  static constexpr int BAR_BYTES = 256;
  static constexpr int BUDGET = 227 * 1024 - 1024 - STAGING_BYTES - BIAS_BYTES - BAR_BYTES;
  static constexpr int STAGES = BUDGET / STAGE_BYTES > 8 ? 8 : BUDGET / STAGE_BYTES;
  static constexpr int TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64 ? 64 : (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512)));
  static constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGES * STAGE_BYTES + STAGING_BYTES + BIAS_BYTES + BAR_BYTES;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
};

// Write one thread's 128-byte row piece (8 x 16 B) into a 32-row staging tile in
// the 128-byte-swizzled layout TMA expects (16-byte chunk c of row r at c ^ (r % 8)).
__device__ __forceinline__ void stage_row128(uint8_t* stage, int r, const uint32_t (&w)[32]) {
  uint8_t* row = stage + r * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint4 u = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
    *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) << 4)) = u;
  }
}

// Bias of output columns col0..col0+31 added to v (warp-uniform loads, served by
// L1).  Only the TMA output paths use it; they require N % 32 == 0, so a piece
// with col0 < N lies entirely inside the bias vector.
__device__ __forceinline__ void add_bias32(const EpiParams& P, int col0, float (&v)[32]) {
  if (P.bias == nullptr || col0 >= P.N) return;
  const float4* b4 = reinterpret_cast<const float4*>(P.bias + col0);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 b = __ldg(b4 + j);
    v[4 * j] += b.x;
    v[4 * j + 1] += b.y;
    v[4 * j + 2] += b.z;
    v[4 * j + 3] += b.w;
  }
}

// bf16 epilogue on 32 accumulator columns held as raw bits in r[]: adds the bias,
// applies GELU / SiLU / partial RoPE and packs bf16 pairs into r[0..15].
__device__ __forceinline__ void epi_bf16_half(const EpiParams& P, uint32_t (&r)[32], int col0, int pos) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  add_bias32(P, col0, v);
  if (P.epi == EPI_GELU) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(v[j]);
  } else if (P.epi == EPI_SILU) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = silu(v[j]);
  } else if (P.epi == EPI_LRELU) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = leaky_relu(v[j]);
  } else if (P.epi == EPI_ROPE && col0 < 2048 && (col0 & 1023) < 64) {
    const int i0 = (col0 & 1023) >> 1;  // first rotary pair of this 32-column piece (0 or 16)
    // 16 consecutive table entries per row, 64-byte aligned: four 16-byte loads each
    const float4* cs = reinterpret_cast<const float4*>(P.rope_cos + (long)pos * 32 + i0);
    const float4* sn = reinterpret_cast<const float4*>(P.rope_sin + (long)pos * 32 + i0);
    float cv[16], sv[16];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4 c4 = __ldg(cs + k), s4 = __ldg(sn + k);
      cv[4 * k] = c4.x; cv[4 * k + 1] = c4.y; cv[4 * k + 2] = c4.z; cv[4 * k + 3] = c4.w;
      sv[4 * k] = s4.x; sv[4 * k + 1] = s4.y; sv[4 * k + 2] = s4.z; sv[4 * k + 3] = s4.w;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float a = v[2 * i], b = v[2 * i + 1];
      v[2 * i] = a * cv[i] - b * sv[i];
      v[2 * i + 1] = b * cv[i] + a * sv[i];
    }
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) r[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
}

// Drain one accumulator slab through the epilogue: TMEM lanes q*32..q*32+31
// (output rows row_base + q*32 + lane) and HALF columns starting at TMEM
// address taddr (output columns n0..).  Direct stores, TMA stores of 32-row x
// 128-byte tiles, or TMA reduce-add, as args.tma_out says.
template <int HALF, typename Tact>
__device__ __forceinline__ void epilogue_slab(const TcGemmArgs& args, const CUtensorMap* tmC, uint32_t taddr,
                                              int row_base, int q, int lane, int n0, uint8_t* stage_buf,
                                              int& sbuf) {
  const EpiParams& P = args.epi;
  const int row = row_base + q * 32 + lane;
  if (args.tma_out == 0) {
#pragma unroll 1
    for (int c = 0; c < HALF / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      tmem_wait_ld();
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
      const int col0 = n0 + c * 32;
      if (col0 < P.N) epilogue_apply<Tact, 32>(P, row, col0, v);
    }
  } else if (args.tma_out == 1 && sizeof(Tact) == 2 && P.epi != EPI_F32) {
    // bf16 tiles: 64 columns (128 B per row) per TMA store
    const int pos = (P.epi == EPI_ROPE && row < P.M) ? __ldg(P.aux + row) : 0;
#pragma unroll 1
    for (int c = 0; c < HALF / 64; ++c) {
      uint32_t r0[32], r1[32];
      tmem_ld32(taddr + c * 64, r0);
      tmem_ld32(taddr + c * 64 + 32, r1);
      tmem_wait_ld();
      const int col0 = n0 + c * 64;
      // in place: bits -> float (+ bias, activation) -> packed bf16 pairs in r0[0..15], r1[0..15]
      epi_bf16_half(P, r0, col0, pos);
      epi_bf16_half(P, r1, col0 + 32, pos);
      uint32_t w[32];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        w[j] = r0[j];
        w[16 + j] = r1[j];
      }
      if (col0 < P.N && row_base + q * 32 < P.M) {  // warp-uniform
        // staging tiles alternate per issued store: the group before the most
        // recent one read this tile, and wait_group.read 1 covers it
        uint8_t* sb = stage_buf + (sbuf & 1) * 4096;
        ++sbuf;
        if (lane == 0) bulk_wait_read1();
        __syncwarp();
        stage_row128(sb, lane, w);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(tmC, smem_u32(sb), col0, row_base + q * 32);
          bulk_commit();
        }
      }
    }
  } else {
    // f32 tiles: 32 columns (128 B per row) per TMA store (EPI_F32) or reduce-add (EPI_GATE_RES)
    const float* grow = nullptr;
    if (P.epi == EPI_GATE_RES) {
      const int doc = row < P.M ? __ldg(P.aux + row) : 0;
      grow = P.gate + (long)doc * P.gate_stride;
    }
#pragma unroll 1
    for (int c = 0; c < HALF / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      const int col0 = n0 + c * 32;
      float g[32];
      if (grow != nullptr) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 gv = __ldg(reinterpret_cast<const float4*>(grow + col0 + j));
          g[j] = gv.x; g[j + 1] = gv.y; g[j + 2] = gv.z; g[j + 3] = gv.w;
        }
      }
      tmem_wait_ld();
      float x[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) x[j] = __uint_as_float(r[j]);
      add_bias32(P, col0, x);
      uint32_t w[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) w[j] = __float_as_uint(grow != nullptr ? x[j] * g[j] : x[j]);
      if (col0 < P.N && row_base + q * 32 < P.M) {  // warp-uniform
        uint8_t* sb = stage_buf + (sbuf & 1) * 4096;
        ++sbuf;
        if (lane == 0) bulk_wait_read1();
        __syncwarp();
        stage_row128(sb, lane, w);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (args.tma_out == 2) tma_reduce_add_2d(tmC, smem_u32(sb), col0, row_base + q * 32);
          else tma_store_2d(tmC, smem_u32(sb), col0, row_base + q * 32);
          bulk_commit();
        }
      }
    }
  }
}

template <int BN, typename Tact>
__global__ void __launch_bounds__(TcGemmCfg<BN>::THREADS, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, const TcGemmArgs args) {
  using Cfg = TcGemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int HALF = BN / 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = smem + STAGES * Cfg::STAGE_BYTES;
  uint8_t* bar_area = staging + Cfg::STAGING_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(bar_area);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      mbar_init(smem_u32(&tempty[a]), Cfg::EPI_WARPS);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (args.tma_out) tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x != 0) {  // thread 0 (the producer) waits after its weight prefetch
    griddep_wait();
    griddep_launch();
  }

  const int num_tiles = args.m_blocks * args.n_blocks;
  const uint32_t smem_base = smem_u32(smem);

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      int stage = 0;
      uint32_t phase = 0;
      long issued = 0;
      bool ok = true;
      // The weights are not written by earlier kernels: load the first tile's B
      // stages before waiting for the previous kernel (overlaps its tail).
      int pre = 0;
      if (static_cast<int>(blockIdx.x) < num_tiles) {
        const int n_blk0 = blockIdx.x % args.n_blocks;
        pre = min(STAGES, args.num_kb);
        for (int kb = 0; kb < pre; ++kb) {
          const uint32_t fb = smem_u32(&full[kb]);
          mbar_arrive_expect_tx(fb, Cfg::STAGE_BYTES);
          tma_load_2d(smem_base + kb * Cfg::STAGE_BYTES + Cfg::A_BYTES, &tmB, fb, kb * 64, n_blk0 * BN);
        }
      }
      griddep_wait();
      griddep_launch();
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m_blk = tile / args.n_blocks;
        const int n_blk = tile - m_blk * args.n_blocks;
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1, 101, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t sa = smem_base + stage * Cfg::STAGE_BYTES;
          const uint32_t sb = sa + Cfg::A_BYTES;
          const uint32_t fb = smem_u32(&full[stage]);
          if (issued >= pre) mbar_arrive_expect_tx(fb, Cfg::STAGE_BYTES);
          tma_load_2d(sa, &tmA, fb, kb * 64, m_blk * 128);
          if (issued >= pre) tma_load_2d(sb, &tmB, fb, kb * 64, n_blk * BN);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Drain the loads that may still be in flight before the CTA exits.
        long n = issued < STAGES ? issued : STAGES;
        int s = stage;
        uint32_t ph = phase;
        for (long i = 0; i < n; ++i) {
          if (--s < 0) {
            s = STAGES - 1;
            ph ^= 1;
          }
          mbar_wait(smem_u32(&full[s]), ph, 102, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc = idesc_bf16_f32(128, BN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1, 103, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait(smem_u32(&full[stage]), phase, 104, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_base + stage * Cfg::STAGE_BYTES;
          const uint32_t sb = sa + Cfg::A_BYTES;
          const uint64_t da = sdesc_sw128(sa);
          const uint64_t db = sdesc_sw128(sb);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            // +32 bytes per 16-element K step inside the 128-byte swizzle atom
            umma_bf16(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0);
          }
          umma_commit(smem_u32(&empty[stage]));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(smem_u32(&tfull[acc]));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      // Make sure no MMA is still writing TMEM when the CTA tears down.
      umma_commit(smem_u32(drain));
      mbar_wait(smem_u32(drain), 0, 105, nullptr);
    }
  } else {
    // ---------------- epilogue warps 2..9: TMEM lane quarter = warp % 4, column half = (warp-2)/4
    const int ew = warp - 2;
    const int q = warp & 3;
    const int col_begin = (ew >> 2) * HALF;
    uint8_t* stage_buf = staging + ew * 8192;
    int sbuf = 0;
    const EpiParams& P = args.epi;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int m_blk = tile / args.n_blocks;
      const int n_blk = tile - m_blk * args.n_blocks;
      const int n0 = n_blk * BN + col_begin;  // first output column of this warp
      if (!mbar_wait(smem_u32(&tfull[acc]), acc_phase, 106, abort_flag)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN + col_begin;
      epilogue_slab<HALF, Tact>(args, &tmC, taddr, m_blk * 128, q, lane, n0, stage_buf, sbuf);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&tempty[acc]));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (lane == 0) bulk_wait0();
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ============================================================== tcgen05 GEMM, CTA pairs
// Same roles and epilogue as tc_gemm_kernel, but a cluster of two CTAs on an SM
// pair computes 256 x 256 tiles with cta_group::2 MMAs: each CTA TMA-loads its
// own 128 rows of A and its own 128 rows of B (no multicast), the completion
// bytes of both land on the leader's (even CTA's) full barrier, the leader
// issues M=256 x N=256 MMAs and multicasts its commits to both CTAs' barriers,
// and each CTA drains its 128-row half of the accumulator from its own TMEM.
// Per SM this halves the operand bytes per MMA compared with 128 x 256 tiles.
struct TcPairCfg {
  static constexpr int BK = 64;
  static constexpr int A_BYTES = 128 * BK * 2;
  static constexpr int B_BYTES = 128 * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI_WARPS = 8;
  static constexpr int HALF = 128;  // columns per epilogue warp
  static constexpr int STAGING_BYTES = EPI_WARPS * 8192;  // two 32-row x 128-byte tiles per epilogue warp
  static constexpr int BIAS_BYTES = 0;
  static constexpr int BAR_BYTES = 256;
  static constexpr int BUDGET = 227 * 1024 - 1024 - STAGING_BYTES - BIAS_BYTES - BAR_BYTES;
  static constexpr int STAGES = BUDGET / STAGE_BYTES > 8 ? 8 : BUDGET / STAGE_BYTES;
  static constexpr int TMEM_COLS = 512;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + STAGING_BYTES + BIAS_BYTES + BAR_BYTES;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
};

// Tile `v` of the pair kernel: output rows m_blk*256.., columns n0..n0+nt-1.
struct PairTile {
  int m_blk, n0, nt;
};
template <bool SPLIT>
__device__ __forceinline__ PairTile pair_tile(const TcGemmArgs& a, int v) {
  PairTile t;
  int f = v, part = 0;
  t.nt = 256;
  if (SPLIT && v >= a.full_tiles) {
    const int u = v - a.full_tiles;
    f = a.full_tiles + u / a.split;
    part = u - (u / a.split) * a.split;
    t.nt = 256 / a.split;
  }
  t.m_blk = f / a.n_blocks;
  t.n0 = (f - t.m_blk * a.n_blocks) * 256 + part * t.nt;
  return t;
}

// SPLIT: the launch splits its last wave's tiles (pieces of 256 x 128 or 256 x 64).
template <typename Tact, bool SPLIT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(TcPairCfg::THREADS, 1)
    tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmB64, const __grid_constant__ CUtensorMap tmC,
                        const TcGemmArgs args) {
  using Cfg = TcPairCfg;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = smem + STAGES * Cfg::STAGE_BYTES;
  uint8_t* bar_area = staging + Cfg::STAGING_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(bar_area);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      mbar_init(smem_u32(&tempty[a]), 2 * Cfg::EPI_WARPS);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (SPLIT) tma_prefetch_desc(&tmB64);
    if (args.tma_out) tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x != 0) {  // thread 0 (the producer) waits after its weight prefetch
    griddep_wait();
    griddep_launch();
  }

  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int num_tiles = args.num_tiles;  // 256 x 256 tiles, then the split pieces of the last wave
  const uint32_t smem_base = smem_u32(smem);
  // B rows per CTA (nt / 2) for a piece of width nt, through the map whose box has that height
  auto b_map = [&](int nt) -> const CUtensorMap* { return (!SPLIT || nt == 256) ? &tmB : &tmB64; };
  auto stage_bytes = [&](int nt) -> uint32_t { return SPLIT ? Cfg::A_BYTES + (nt / 2) * Cfg::BK * 2 : Cfg::STAGE_BYTES; };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs)
      int stage = 0;
      uint32_t phase = 0;
      long issued = 0;
      bool ok = true;
      // weight (B) stages of the first tile before waiting for the previous kernel
      int pre = 0;
      if (pair < num_tiles) {
        const PairTile t0 = pair_tile<SPLIT>(args, pair);
        pre = min(STAGES, args.num_kb);
        for (int kb = 0; kb < pre; ++kb) {
          const uint32_t fb = smem_u32(&full[kb]);
          if (leader) mbar_arrive_expect_tx(fb, 2 * stage_bytes(t0.nt));
          tma_load_2d_pair(smem_base + kb * Cfg::STAGE_BYTES + Cfg::A_BYTES, b_map(t0.nt), to_leader(fb), kb * 64,
                           t0.n0 + rank * (t0.nt / 2));
        }
      }
      griddep_wait();
      griddep_launch();
      for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
        const PairTile pt = pair_tile<SPLIT>(args, tile);
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1, 121, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t sa = smem_base + stage * Cfg::STAGE_BYTES;
          const uint32_t sb = sa + Cfg::A_BYTES;
          const uint32_t fb = smem_u32(&full[stage]);
          if (leader && issued >= pre) mbar_arrive_expect_tx(fb, 2 * stage_bytes(pt.nt));
          tma_load_2d_pair(sa, &tmA, to_leader(fb), kb * 64, pt.m_blk * 256 + rank * 128);
          if (issued >= pre) tma_load_2d_pair(sb, b_map(pt.nt), to_leader(fb), kb * 64, pt.n0 + rank * (pt.nt / 2));
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok && leader) {
        // the leader's full barriers count both CTAs' bytes: drain what may be in flight
        long n = issued < STAGES ? issued : STAGES;
        int s = stage;
        uint32_t ph = phase;
        for (long i = 0; i < n; ++i) {
          if (--s < 0) {
            s = STAGES - 1;
            ph ^= 1;
          }
          mbar_wait(smem_u32(&full[s]), ph, 122, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (leader only)
      constexpr uint32_t idesc256 = idesc_bf16_f32(256, 256, false, false);
      constexpr uint32_t idesc128 = idesc_bf16_f32(256, 128, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
        const int nt = pair_tile<SPLIT>(args, tile).nt;
        const uint32_t idesc = (!SPLIT || nt == 256) ? idesc256 : idesc128;
        if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1, 123, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * 256;
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait(smem_u32(&full[stage]), phase, 124, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_base + stage * Cfg::STAGE_BYTES;
          const uint32_t sb = sa + Cfg::A_BYTES;
          const uint64_t da = sdesc_sw128(sa);
          const uint64_t db = sdesc_sw128(sb);
#pragma unroll
          for (int k = 0; k < 4; ++k) umma_bf16_pair(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb | k) != 0);
          umma_commit_pair_mc(smem_u32(&empty[stage]), 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair_mc(smem_u32(&tfull[acc]), 0x3);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      umma_commit_pair(smem_u32(drain));
      mbar_wait(smem_u32(drain), 0, 125, nullptr);
    }
  } else {
    // ---------------- epilogue warps 2..9 (both CTAs): this CTA's 128 rows of each tile
    const int ew = warp - 2;
    const int q = warp & 3;
    uint8_t* stage_buf = staging + ew * 8192;
    int sbuf = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = pair; tile < num_tiles; tile += npairs) {
      const PairTile pt = pair_tile<SPLIT>(args, tile);
      // the two warps of a TMEM lane quarter split the tile's columns
      const int width = pt.nt / 2;
      const int col_begin = (ew >> 2) * width;
      if (!mbar_wait(smem_u32(&tfull[acc]), acc_phase, 126, abort_flag)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * 256 + col_begin;
      if (!SPLIT || width == 128)
        epilogue_slab<128, Tact>(args, &tmC, taddr, pt.m_blk * 256 + rank * 128, q, lane, pt.n0 + col_begin,
                                 stage_buf, sbuf);
      else
        epilogue_slab<64, Tact>(args, &tmC, taddr, pt.m_blk * 256 + rank * 128, q, lane, pt.n0 + col_begin,
                                stage_buf, sbuf);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(to_leader(smem_u32(&tempty[acc])));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (lane == 0) bulk_wait0();
    __syncwarp();
  }
  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its peer may still signal it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

// ============================================================== tcgen05 causal grouped convolution
// Implicit GEMM of the grouped causal convolutions of the input embedding
// (CausalConvPositionEmbedding, kernel 31, 16 groups of 64 channels;
// flashinfer_dit.py:615-654) on the gapped buffer: for group n,
//   out[g, n*64 + c] = bias + sum_t sum_i A[g + t - 30, n*64 + i] * W[n*64 + c, t*64 + i].
// The 128 output rows of a tile need input rows g0-30 .. g0+127; they are loaded
// ONCE (160 rows, TMA zero-fills rows before the buffer) and tap t is the MMA on
// rows t .. t+127 of that tile (descriptor moved by t rows).  The group's
// weights stream through a ring of stages of 4 taps (4 x 64 x 64), so the MMA
// thread waits and commits once per 16 MMAs.
// Persistent, one CTA per SM: warp 0 TMA, warp 1 MMA, warps 2-9 epilogue, two
// per TMEM lane quarter with 32 columns each (direct stores through
// epilogue_apply: Mish into the gapped buffer, or Mish plus residual into the
// packed fp32 stream).
struct ConvCfg {
  static constexpr int A_ROWS = 160;
  static constexpr int A_BYTES = A_ROWS * 128;  // 20 KB, a multiple of 1024
  static constexpr int B_BYTES = 64 * 128;      // one tap of one group
  static constexpr int UNIT_TAPS = 4;           // taps per ring stage
  static constexpr int UNIT_BYTES = UNIT_TAPS * B_BYTES;
  static constexpr int B_STAGES = 4;
  static constexpr int TAPS = 31;
  static constexpr int UNITS = (TAPS + UNIT_TAPS - 1) / UNIT_TAPS;  // 8 per tile, the last with 3 taps
  static constexpr int THREADS = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
  static constexpr int OFF_B = 2 * A_BYTES;
  static constexpr int OFF_BAR = OFF_B + B_STAGES * UNIT_BYTES;
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM_BYTES = 1024 + OFF_BAR + BAR_BYTES;
  static constexpr int TMEM_COLS = 128;  // two 64-column accumulators
  static constexpr int EPI_WARPS = 8;
};
static_assert((2 + 2 + 2 * ConvCfg::B_STAGES + 2 + 2 + 1) * 8 + 8 <= ConvCfg::BAR_BYTES, "conv barrier area");

template <typename Tact>
__global__ void __launch_bounds__(ConvCfg::THREADS, 1)
    tc_conv_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const TcGemmArgs args) {
  using Cfg = ConvCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t s0 = smem_u32(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::OFF_BAR);
  uint64_t* a_full = bars;                      // [2]
  uint64_t* a_empty = bars + 2;                 // [2]
  uint64_t* b_full = bars + 4;                  // [B_STAGES]
  uint64_t* b_empty = b_full + Cfg::B_STAGES;   // [B_STAGES]
  uint64_t* tfull = b_empty + Cfg::B_STAGES;    // [2]
  uint64_t* tempty = tfull + 2;                 // [2]
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&a_full[i]), 1);
      mbar_init(smem_u32(&a_empty[i]), 1);
      mbar_init(smem_u32(&tfull[i]), 1);
      mbar_init(smem_u32(&tempty[i]), Cfg::EPI_WARPS);
    }
    for (int i = 0; i < Cfg::B_STAGES; ++i) {
      mbar_init(smem_u32(&b_full[i]), 1);
      mbar_init(smem_u32(&b_empty[i]), 1);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x != 0) {  // thread 0 (the producer) waits after its weight prefetch
    griddep_wait();
    griddep_launch();
  }
  const int n_groups = args.n_blocks;
  const int num_tiles = args.m_blocks * n_groups;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      long bi = 0;  // weight stages in ring order
      long b_issued = 0;
      int ti = 0, a_issued = 0;
      bool ok = true;
      auto load_unit = [&](int st, int u, int grp) {
        const int taps = min(Cfg::UNIT_TAPS, Cfg::TAPS - u * Cfg::UNIT_TAPS);
        const uint32_t fb = smem_u32(&b_full[st]);
        mbar_arrive_expect_tx(fb, taps * Cfg::B_BYTES);
        for (int j = 0; j < taps; ++j)
          tma_load_2d(s0 + Cfg::OFF_B + st * Cfg::UNIT_BYTES + j * Cfg::B_BYTES, &tmB, fb,
                      (u * Cfg::UNIT_TAPS + j) * 64, grp * 64);
      };
      int pre = 0;
      if (static_cast<int>(blockIdx.x) < num_tiles) {
        pre = Cfg::B_STAGES < Cfg::UNITS ? Cfg::B_STAGES : Cfg::UNITS;
        for (int u = 0; u < pre; ++u) load_unit(u, u, blockIdx.x % n_groups);
        b_issued = pre;
      }
      griddep_wait();
      griddep_launch();
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++ti) {
        const int m_blk = tile / n_groups;
        const int grp = tile - m_blk * n_groups;
        const int ab = ti & 1;
        if (!mbar_wait(smem_u32(&a_empty[ab]), ((ti >> 1) & 1) ^ 1, 141, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(smem_u32(&a_full[ab]), Cfg::A_BYTES);
        tma_load_2d(s0 + ab * Cfg::A_BYTES, &tmA, smem_u32(&a_full[ab]), grp * 64, m_blk * 128 - kConvPad);
        ++a_issued;
        for (int u = 0; u < Cfg::UNITS; ++u, ++bi) {
          if (bi < pre) continue;  // loaded before the wait on the previous kernel
          const int st = static_cast<int>(bi % Cfg::B_STAGES);
          if (!mbar_wait(smem_u32(&b_empty[st]), ((bi / Cfg::B_STAGES) & 1) ^ 1, 142, abort_flag)) {
            ok = false;
            break;
          }
          load_unit(st, u, grp);
          ++b_issued;
        }
      }
      if (!ok) {
        // let the copies that may still be in flight land before the CTA exits
        for (long k = (b_issued > Cfg::B_STAGES ? b_issued - Cfg::B_STAGES : 0); k < b_issued; ++k)
          mbar_wait(smem_u32(&b_full[k % Cfg::B_STAGES]), (k / Cfg::B_STAGES) & 1, 147, nullptr);
        for (int k = (a_issued > 2 ? a_issued - 2 : 0); k < a_issued; ++k)
          mbar_wait(smem_u32(&a_full[k & 1]), (k >> 1) & 1, 148, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer: 31 taps of 4 K-steps per tile
      constexpr uint32_t idesc = idesc_bf16_f32(128, 64, false, false);
      long bi = 0;
      int ti = 0, acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++ti) {
        const int ab = ti & 1;
        if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1, 143, abort_flag)) break;
        if (!mbar_wait(smem_u32(&a_full[ab]), (ti >> 1) & 1, 144, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * 64;
        const uint32_t sa = s0 + ab * Cfg::A_BYTES;
        for (int u = 0; u < Cfg::UNITS; ++u, ++bi) {
          const int st = static_cast<int>(bi % Cfg::B_STAGES);
          if (!mbar_wait(smem_u32(&b_full[st]), (bi / Cfg::B_STAGES) & 1, 145, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int taps = min(Cfg::UNIT_TAPS, Cfg::TAPS - u * Cfg::UNIT_TAPS);
          for (int j = 0; j < taps; ++j) {
            const int tap = u * Cfg::UNIT_TAPS + j;
            const uint64_t da = sdesc_sw128_row(sa, tap);
            const uint64_t db = sdesc_sw128(s0 + Cfg::OFF_B + st * Cfg::UNIT_BYTES + j * Cfg::B_BYTES);
#pragma unroll
            for (int k = 0; k < 4; ++k) umma_bf16(d_tmem, da + 2 * k, db + 2 * k, idesc, (tap | k) != 0);
          }
          umma_commit(smem_u32(&b_empty[st]));
        }
        if (!ok) break;
        umma_commit(smem_u32(&tfull[acc]));
        umma_commit(smem_u32(&a_empty[ab]));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      umma_commit(smem_u32(drain));
      mbar_wait(smem_u32(drain), 0, 146, nullptr);
    }
  } else {
    // ---------------- epilogue warps 2..9: lane quarter q, 32 columns (half ch) of the tile
    const int q = warp & 3;
    const int ch = (warp - 2) >> 2;
    const EpiParams& P = args.epi;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int m_blk = tile / n_groups;
      const int grp = tile - m_blk * n_groups;
      if (!mbar_wait(smem_u32(&tfull[acc]), acc_phase, 149, abort_flag)) break;
      tc_fence_after();
      const int row = m_blk * 128 + q * 32 + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * 64 + ch * 32;
      {
        uint32_t r[32];
        tmem_ld32(taddr, r);
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        epilogue_apply<Tact, 32>(P, row, grp * 64 + ch * 32, v);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&tempty[acc]));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ============================================================== fp32 SIMT GEMM

struct SimtGemmArgs {
  const float* A;
  long lda;
  const float* W;  // (N, K) row-major
  int M, N, K;
  int conv;        // implicit-conv A addressing (K = 31*64, N tile = one group)
  EpiParams epi;
};

// 64x64 tile, 256 threads, 4x4 outputs per thread (4 consecutive columns).
__global__ void __launch_bounds__(256) simt_gemm_f32_kernel(const SimtGemmArgs a) {
  griddep_wait();
  griddep_launch();
  __shared__ float As[16][64 + 4];
  __shared__ float Bs[16][64 + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  const int lr = threadIdx.x >> 2;        // 0..63 (row of the tile being loaded)
  const int lk = (threadIdx.x & 3) * 4;   // 0,4,8,12
  for (int k0 = 0; k0 < a.K; k0 += 16) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int k = k0 + lk + j;
      // A element
      float av = 0.f;
      const int m = m0 + lr;
      if (m < a.M && k < a.K) {
        if (a.conv) {
          const int tap = k >> 6, ci = k & 63;
          const int r = m + tap - kConvPad;
          if (r >= 0) av = a.A[(long)r * a.lda + blockIdx.x * 64 + ci];
        } else {
          av = a.A[(long)m * a.lda + k];
        }
      }
      As[lk + j][lr] = av;
      float bv = 0.f;
      const int n = n0 + lr;
      if (n < a.N && k < a.K) bv = a.W[(long)n * a.K + k];
      Bs[lk + j][lr] = bv;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      float ar[4], br[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) ar[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) br[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
    }
    __syncthreads();
  }
  const int col0 = n0 + tx * 4;
  if (col0 >= a.N) return;
#pragma unroll
  for (int i = 0; i < 4; ++i) epilogue_apply<float, 4>(a.epi, m0 + ty * 4 + i, col0, acc[i]);
}

}  // namespace fcv
