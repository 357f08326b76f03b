// HiFT vocoder decode on packed rows (CausalHiFTGenerator.inference,
// cosyvoice/hifigan/generator.py:728-740, structure of builders.py:38-50).
//
// Every signal of the vocoder is stored time-major over the packed documents of
// one batch: a level with C channels is (rows, C) with each request's rows
// contiguous, its start in a cu array of the layout block.  All convolutions
// are causal within a document (zero outside it), so one launch serves every
// request; the reference runs the vocoder once per request (token2wav.py:130-131).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "fcv_common.cuh"

namespace hift {

using fcv::griddep_launch;
using fcv::griddep_wait;

enum Pre { PRE_NONE = 0, PRE_LEAKY = 1, PRE_SNAKE = 2 };
enum Epi { EPI_STORE = 0, EPI_ELU = 1, EPI_SNAKE = 2, EPI_RES = 3, EPI_RES_ACC = 4, EPI_RES_ACC_AVG = 5 };

constexpr int kUpTotal = 480;   // samples per mel frame: 8 * 5 * 3 upsampling * hop 4
constexpr int kHarm = 9;        // fundamental + 8 harmonics (nb_harmonics=8)
constexpr int kNfft = 16;
constexpr int kHop = 4;
constexpr int kBins = 9;        // n_fft / 2 + 1

// One convolution over packed rows.
//   out[r, co] = epi(b[co] + sum_{j < k} sum_ci w[j][ci][co] * pre(x[src(r, j), ci]))
// Output row r of document d (local t) reads, at tap j, position
// idx = c * stride + j * dil - pad_left of the document's input, where c = t (or
// the ReflectionPad1d((1, 0)) remap t == 0 -> 1, t -> t - 1 with reflect_first);
// with up > 1 the input is first repeated up times (nearest upsampling), so idx
// addresses the repeated sequence and reads input row idx / up.  Positions
// outside [0, up * lim) are zero padding; lim = in_lim[d + 1] - in_lim[d].
// Besides out, the epilogue can store up to 3 Snake activations of the final
// value (act_out[q] = snake(out; act_alpha[q])): the next convolutions' inputs,
// computed once per element instead of once per tap and channel tile.
template <typename T>
struct ConvArgs {
  const void* x;
  int x_pitch;
  const int* in_off;   // (n_docs + 1) input row offsets
  const int* in_lim;   // (n_docs + 1) cu array whose differences bound the readable input
  const int* out_cu;   // (n_docs + 1) output row offsets
  int n_docs, rows_out;
  const T* w;          // [k][cin_pad][cout_pad]
  const T* b;          // [cout_pad]
  int cin, cin_pad, cout, cout_pad, k, dil, stride, up, pad_left, reflect_first;
  int vec;             // rows load as float4: float input, cin % 16 == 0, x_pitch % 4 == 0, 16-byte base
  int pre;
  float slope;
  const float* pre_alpha;
  const float* pre_inv;
  int epi;
  const float* post_alpha;
  const float* post_inv;
  const T* res;
  const T* acc;
  T* out;
  int out_pitch;
  int n_act;
  T* act_out[3];
  const float* act_alpha[3];
  const float* act_inv[3];
  const float* tw_hi;  // tensor-core path: weights [k][cout][cin] split into a tf32 head ...
  const float* tw_lo;  // ... and the float32 remainder (null: SIMT path)
};

__device__ __forceinline__ int find_doc(const int* __restrict__ cu, int n_docs, int r) {
  int lo = 0, hi = n_docs;  // largest d with cu[d] <= r
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(cu + mid) <= r) lo = mid; else hi = mid;
  }
  return lo;
}

// Snake (activation.py:73-84): x + inv * sin(x * alpha)^2, inv = 1 / (alpha + 1e-9)
// precomputed in float32 on the host; each product and sum rounded separately
// like the reference's tensor ops.
__device__ __forceinline__ float snake(float x, float a, float inv) {
  const float s = sinf(__fmul_rn(x, a));
  return __fadd_rn(x, __fmul_rn(inv, __fmul_rn(s, s)));
}

template <typename T>
__device__ __forceinline__ T pre_act(T v, int pre, float slope, const float* alpha, const float* inv, int ci) {
  if (pre == PRE_LEAKY) return v < T(0) ? v * T(slope) : v;
  if (pre == PRE_SNAKE) return T(snake(float(v), __ldg(alpha + ci), __ldg(inv + ci)));
  return v;
}

template <typename T>
__device__ __forceinline__ T add_rn(T a, T b) { return a + b; }
template <>
__device__ __forceinline__ float add_rn<float>(float a, float b) { return __fadd_rn(a, b); }

// Four consecutive shared-memory elements (16-byte aligned for float: one 128-bit load).
__device__ __forceinline__ void load4(float* d, const float* s) {
  const float4 v = *reinterpret_cast<const float4*>(s);
  d[0] = v.x;
  d[1] = v.y;
  d[2] = v.z;
  d[3] = v.w;
}
__device__ __forceinline__ void load4(double* d, const double* s) {
  const double2 v0 = *reinterpret_cast<const double2*>(s), v1 = *reinterpret_cast<const double2*>(s + 2);
  d[0] = v0.x;
  d[1] = v0.y;
  d[2] = v1.x;
  d[3] = v1.y;
}

// SIMT implicit-GEMM tile: 128 output rows x 64 output channels, 128 threads,
// each 8 rows x 8 channels; K = taps x input channels in steps of BK (one row of
// BK channels loaded per thread), operands double-buffered in shared memory
// through registers.  The accumulation order over (tap, channel) is the same
// for every output element whatever its tile, so packed documents give the
// same bits as single ones.
template <typename Tin, typename T>
__global__ void __launch_bounds__(128, sizeof(T) == 8 ? 2 : 4) conv_kernel(ConvArgs<T> p) {
  griddep_wait();
  griddep_launch();
  constexpr int BM = 128, BN = 64, NT = 128;
  constexpr int BK = sizeof(T) == 8 ? 8 : 16;
  constexpr int NB = BK * BN / NT;     // weights one thread loads per step
  __shared__ __align__(16) T As[2][BK][BM + 4];
  __shared__ __align__(16) T Bs[2][BK][BN];
  const int tid = threadIdx.x;
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  const Tin* __restrict__ x = static_cast<const Tin*>(p.x);

  // the A row this thread loads, and its document geometry
  const int r_ld = m0 + tid;
  int base = 0, pos0 = 0, lim_up = 0;
  const bool row_ok = r_ld < p.rows_out;
  if (row_ok) {
    const int d = find_doc(p.out_cu, p.n_docs, r_ld);
    const int t = r_ld - __ldg(p.out_cu + d);
    const int c = p.reflect_first ? (t == 0 ? 1 : t - 1) : t;
    base = __ldg(p.in_off + d);
    lim_up = (__ldg(p.in_lim + d + 1) - __ldg(p.in_lim + d)) * p.up;
    pos0 = c * p.stride - p.pad_left;
  }
  const int n_ci = p.cin_pad / BK;
  const int n_iter = p.k * n_ci;

  T a_reg[BK];
  T b_reg[NB];
  int ld_j = 0, ld_c = 0;   // tap and channel chunk of the next load
  auto load = [&]() {
    const int idx = pos0 + ld_j * p.dil;
    const bool ok = row_ok && idx >= 0 && idx < lim_up;
    const int ci0 = ld_c * BK;
    if (ok) {
      const Tin* src = x + (size_t)(base + (p.up == 1 ? idx : idx / p.up)) * p.x_pitch + ci0;
      if (sizeof(Tin) == 4 && p.vec) {
#pragma unroll
        for (int q = 0; q < BK; q += 4) {
          const float4 v4 = __ldg(reinterpret_cast<const float4*>(src) + q / 4);
          a_reg[q] = T(v4.x);
          a_reg[q + 1] = T(v4.y);
          a_reg[q + 2] = T(v4.z);
          a_reg[q + 3] = T(v4.w);
        }
      } else {
#pragma unroll
        for (int q = 0; q < BK; ++q) a_reg[q] = ci0 + q < p.cin ? T(src[q]) : T(0);
      }
      if (p.pre != PRE_NONE) {
#pragma unroll
        for (int q = 0; q < BK; ++q)
          if (ci0 + q < p.cin) a_reg[q] = pre_act<T>(a_reg[q], p.pre, p.slope, p.pre_alpha, p.pre_inv, ci0 + q);
      }
    } else {
#pragma unroll
      for (int q = 0; q < BK; ++q) a_reg[q] = T(0);
    }
    const T* wsrc = p.w + ((size_t)ld_j * p.cin_pad + ci0) * p.cout_pad + n0;
#pragma unroll
    for (int q = 0; q < NB; ++q) {
      const int e = tid + q * NT;
      b_reg[q] = __ldg(wsrc + (size_t)(e / BN) * p.cout_pad + (e % BN));
    }
    if (++ld_c == n_ci) {
      ld_c = 0;
      ++ld_j;
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int q = 0; q < BK; ++q) As[buf][q][tid] = a_reg[q];
#pragma unroll
    for (int q = 0; q < NB; ++q) {
      const int e = tid + q * NT;
      Bs[buf][e / BN][e % BN] = b_reg[q];
    }
  };

  const int tx = tid & 15, ty = tid >> 4;   // rows tx*4 (+64), channels ty*4 (+32)
  T accum[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) accum[i][jj] = T(0);

  load();
  store(0);
  __syncthreads();
  for (int it = 0; it < n_iter; ++it) {
    const int buf = it & 1;
    if (it + 1 < n_iter) load();
    // partial unroll: the fully unrolled step (~1100 instructions) stalled on instruction fetch
#pragma unroll 4
    for (int kk = 0; kk < BK; ++kk) {
      T a[8], bv[8];
      load4(a, &As[buf][kk][tx * 4]);
      load4(a + 4, &As[buf][kk][64 + tx * 4]);
      load4(bv, &Bs[buf][kk][ty * 4]);
      load4(bv + 4, &Bs[buf][kk][32 + ty * 4]);
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) accum[i][jj] = fma(a[i], bv[jj], accum[i][jj]);
    }
    if (it + 1 < n_iter) store(buf ^ 1);
    __syncthreads();
  }

  // epilogue
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = m0 + (i < 4 ? tx * 4 + i : 64 + tx * 4 + (i - 4));
    if (r >= p.rows_out) continue;
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      const int co = n0 + (jj < 4 ? ty * 4 + jj : 32 + ty * 4 + (jj - 4));
      if (co >= p.cout) continue;
      T v = add_rn<T>(accum[i][jj], p.b[co]);
      const size_t o = (size_t)r * p.out_pitch + co;
      switch (p.epi) {
        case EPI_ELU: v = v > T(0) ? v : T(exp(double(v)) - 1.0); break;
        case EPI_SNAKE: v = T(snake(float(v), __ldg(p.post_alpha + co), __ldg(p.post_inv + co))); break;
        case EPI_RES: v = add_rn<T>(v, p.res[o]); break;
        case EPI_RES_ACC: v = add_rn<T>(p.acc[o], add_rn<T>(v, p.res[o])); break;
        case EPI_RES_ACC_AVG: v = T(__fdiv_rn(float(add_rn<T>(p.acc[o], add_rn<T>(v, p.res[o]))), 3.0f)); break;
        default: break;
      }
      p.out[o] = v;
      for (int q = 0; q < p.n_act; ++q)
        p.act_out[q][o] = T(snake(float(v), __ldg(p.act_alpha[q] + co), __ldg(p.act_inv[q] + co)));
    }
  }
}


// ---------------------------------------------------------------- tensor-core residual convolutions
// Stride-1 convolutions (the 72 residual-block convolutions, 88 % of the vocoder's
// FLOPs) on tcgen05 kind::tf32
// with float32 accuracy: each operand is split into a tf32 head h (x rounded to
// the nearest tf32, low 13 mantissa bits zero) and the remainder l = x - h (exact,
// |l| <= 2^-11 |x|), and D += Ah*Bh + Ah*Bl + Al*Bh (the Al*Bl term is below
// float32 rounding).
//
// The kernel also handles nearest upsampling, the first-row reflection and a
// leaky-ReLU input (applied while splitting), but the three upsampling convolutions
// (K up to 8192) run on the SIMT kernel: on the tensor cores they took the speech
// output to 1.007e-4 rel-L2 of the reference's, past the 1e-4 test bound, for a gain
// of about 8 % of the vocoder time.
//
// One CTA computes 128 output rows x N (= C_out) channels, accumulating in N TMEM
// columns.  Warps 0-3 produce: each thread gathers its output row's input row for
// the current tap with cp.async (zero-filled outside the document), 32 channels
// (128 bytes) per stage, splits it into head and remainder in shared memory and
// loads 128-byte rows of the pre-split weights; warp 4 issues the MMAs; warps 0-3
// then read the accumulator rows back and run the same epilogue as the SIMT kernel.
// Shared-memory tiles use the 128-byte swizzle (16-byte chunk c of row r stored at
// chunk c ^ (r & 7)), the layout the MMA descriptors describe.
template <int N>
struct ResConvCfg {
  static constexpr int S = N == 128 ? 3 : 2;                       // pipeline stages (N = 64: two CTAs per SM)
  static constexpr int A_BYTES = 128 * 128;                        // 128 rows x 32 floats
  static constexpr int B_BYTES = N * 128;
  static constexpr int STAGE = 2 * A_BYTES + 2 * B_BYTES;          // head and remainder of A and B
  static constexpr int SMEM_BYTES = 1024 + S * STAGE + 256;
  static constexpr int THREADS = 160;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int PENDING>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(PENDING) : "memory"); }

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor: kind::tf32, A = B = tf32 (format 2), D = f32, both K-major.
__host__ __device__ constexpr uint32_t idesc_tf32_f32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

template <int N>
__global__ void __launch_bounds__(160, N == 64 ? 2 : 1) res_conv_tc_kernel(ConvArgs<float> p) {
  using Cfg = ResConvCfg<N>;
  constexpr int S = Cfg::S;
  griddep_wait();
  griddep_launch();
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = (fcv::smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* base = smem_raw + (base_u32 - fcv::smem_u32(smem_raw));
  const uint32_t bar0 = base_u32 + S * Cfg::STAGE;   // full[S], empty[S], done
  int* abort_flag = reinterpret_cast<int*>(base + S * Cfg::STAGE + 8 * (2 * S + 1));
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(base + S * Cfg::STAGE + 8 * (2 * S + 1) + 4);
  auto full = [&](int st) { return bar0 + 8u * st; };
  auto empty = [&](int st) { return bar0 + 8u * (S + st); };
  const uint32_t done = bar0 + 8u * (2 * S);
  auto a_hi = [&](int st) { return base_u32 + st * Cfg::STAGE; };
  auto a_lo = [&](int st) { return a_hi(st) + Cfg::A_BYTES; };
  auto b_hi = [&](int st) { return a_hi(st) + 2 * Cfg::A_BYTES; };
  auto b_lo = [&](int st) { return b_hi(st) + Cfg::B_BYTES; };

  const int tid = threadIdx.x, warp = tid >> 5;
  const int m0 = blockIdx.x * 128;
  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      fcv::mbar_init(full(i), 128);
      fcv::mbar_init(empty(i), 1);
    }
    fcv::mbar_init(done, 1);
    *abort_flag = 0;
    fcv::fence_mbar_init();
  }
  if (warp == 4) {
    fcv::tmem_alloc(fcv::smem_u32(tmem_slot), N);
    fcv::tmem_relinquish();
  }
  fcv::tc_fence_before();
  __syncthreads();
  fcv::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_ci = p.cin / 32;
  const int n_iter = p.k * n_ci;
  volatile int* abrt = abort_flag;

  if (warp < 4) {
    // ---- producer: row tid of the tile
    const int r = m0 + tid;
    const bool row_ok = r < p.rows_out;
    int rbase = 0, pos0 = 0, lim = 0;
    if (row_ok) {
      const int d = find_doc(p.out_cu, p.n_docs, r);
      const int t = r - __ldg(p.out_cu + d);
      rbase = __ldg(p.in_off + d);
      lim = (__ldg(p.in_lim + d + 1) - __ldg(p.in_lim + d)) * p.up;   // positions of the upsampled input
      pos0 = (p.reflect_first ? (t == 0 ? 1 : t - 1) : t) - p.pad_left;
    }
    const float* xin = static_cast<const float*>(p.x);
    auto issue = [&](int it) {
      const int st = it % S, j = it / n_ci, ci0 = (it - j * n_ci) * 32;
      const int idx = pos0 + j * p.dil;
      const bool ok = row_ok && idx >= 0 && idx < lim;
      const float* src = ok ? xin + (size_t)(rbase + (p.up == 1 ? idx : idx / p.up)) * p.x_pitch + ci0 : xin;
      const uint32_t arow = a_hi(st) + tid * 128;
#pragma unroll
      for (int q = 0; q < 8; ++q) cp_async16(arow + ((q ^ (tid & 7)) << 4), src + 4 * q, ok ? 16u : 0u);
#pragma unroll
      for (int m = 0; m < N / 16; ++m) {
        const int e = tid + 128 * m, co = e >> 3, q = e & 7;
        const size_t off = ((size_t)j * p.cout + co) * p.cin + ci0 + 4 * q;
        const uint32_t dst = co * 128 + ((q ^ (co & 7)) << 4);
        cp_async16(b_hi(st) + dst, p.tw_hi + off, 16u);
        cp_async16(b_lo(st) + dst, p.tw_lo + off, 16u);
      }
    };
    bool ok_run = true;
    for (int it = 0; it < S - 1; ++it) {
      if (it < n_iter) issue(it);
      cp_async_commit();
    }
    for (int it = 0; it < n_iter && ok_run; ++it) {
      // stage it has landed once at most S - 2 newer groups are pending
      cp_async_wait<S - 2>();
      // split this thread's row of stage it into head and remainder, hand it to the MMA
      const int st = it % S;
      float4* hrow = reinterpret_cast<float4*>(base + (a_hi(st) - base_u32) + tid * 128);
      float4* lrow = reinterpret_cast<float4*>(base + (a_lo(st) - base_u32) + tid * 128);
#pragma unroll
      for (int qq = 0; qq < 8; ++qq) {
        const int q = qq ^ (tid & 7);   // swizzled order: the 8 threads of a phase hit distinct banks
        float4 v = hrow[q];
        if (p.pre == PRE_LEAKY) {   // leaky ReLU of the input, as the SIMT kernel applies on load
          v.x = v.x < 0.f ? v.x * p.slope : v.x;
          v.y = v.y < 0.f ? v.y * p.slope : v.y;
          v.z = v.z < 0.f ? v.z * p.slope : v.z;
          v.w = v.w < 0.f ? v.w * p.slope : v.w;
        }
        float4 h, l;
        h.x = __uint_as_float((__float_as_uint(v.x) + 0x1000u) & 0xFFFFE000u);
        h.y = __uint_as_float((__float_as_uint(v.y) + 0x1000u) & 0xFFFFE000u);
        h.z = __uint_as_float((__float_as_uint(v.z) + 0x1000u) & 0xFFFFE000u);
        h.w = __uint_as_float((__float_as_uint(v.w) + 0x1000u) & 0xFFFFE000u);
        l.x = v.x - h.x;
        l.y = v.y - h.y;
        l.z = v.z - h.z;
        l.w = v.w - h.w;
        hrow[q] = h;
        lrow[q] = l;
      }
      fcv::fence_proxy_async_smem();
      fcv::mbar_arrive(full(st));
      // then refill the slot the previous step's MMAs read (stage it + S - 1)
      const int nxt = it + S - 1;
      if (nxt < n_iter) {
        if (nxt >= S && !fcv::mbar_wait(empty(nxt % S), ((nxt - S) / S) & 1, 260, abrt)) { ok_run = false; break; }
        issue(nxt);
      }
      cp_async_commit();
    }
    cp_async_wait<0>();
    // ---- epilogue: accumulator row tid (TMEM lane 32 * warp + lane)
    // tcgen05.ld is warp-collective: the whole warp reads the accumulator or none of it
    const bool ready = __all_sync(0xffffffffu, ok_run && fcv::mbar_wait(done, 0, 261, abrt));
    fcv::tc_fence_after();
    if (ready) {
      for (int c0 = 0; c0 < N; c0 += 32) {
        uint32_t acc_r[32];
        fcv::tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + c0, acc_r);
        fcv::tmem_wait_ld();
        if (!row_ok) continue;
        // this thread's 32 consecutive outputs of row r: every operand is loaded before
        // anything is stored (res / acc may alias out), 16 bytes at a time
        const size_t o0 = (size_t)r * p.out_pitch + c0;
        float v[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) v[c] = __fadd_rn(__uint_as_float(acc_r[c]), __ldg(p.b + c0 + c));
        if (p.epi == EPI_SNAKE) {
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] = snake(v[c], __ldg(p.post_alpha + c0 + c), __ldg(p.post_inv + c0 + c));
        } else if (p.epi >= EPI_RES) {
          float rv[32], av[32];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 t = reinterpret_cast<const float4*>(p.res + o0)[q];
            rv[4 * q] = t.x;
            rv[4 * q + 1] = t.y;
            rv[4 * q + 2] = t.z;
            rv[4 * q + 3] = t.w;
          }
          if (p.epi != EPI_RES) {
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 t = reinterpret_cast<const float4*>(p.acc + o0)[q];
              av[4 * q] = t.x;
              av[4 * q + 1] = t.y;
              av[4 * q + 2] = t.z;
              av[4 * q + 3] = t.w;
            }
          }
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            float u = __fadd_rn(v[c], rv[c]);
            if (p.epi == EPI_RES_ACC) u = __fadd_rn(av[c], u);
            if (p.epi == EPI_RES_ACC_AVG) u = __fdiv_rn(__fadd_rn(av[c], u), 3.0f);
            v[c] = u;
          }
        }
        float4* outv = reinterpret_cast<float4*>(p.out + o0);
#pragma unroll
        for (int q = 0; q < 8; ++q) outv[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        for (int a = 0; a < p.n_act; ++a) {
          float4* actv = reinterpret_cast<float4*>(p.act_out[a] + o0);
          const float* al = p.act_alpha[a] + c0;
          const float* ai = p.act_inv[a] + c0;
#pragma unroll
          for (int q = 0; q < 8; ++q)
            actv[q] = make_float4(snake(v[4 * q], __ldg(al + 4 * q), __ldg(ai + 4 * q)),
                                  snake(v[4 * q + 1], __ldg(al + 4 * q + 1), __ldg(ai + 4 * q + 1)),
                                  snake(v[4 * q + 2], __ldg(al + 4 * q + 2), __ldg(ai + 4 * q + 2)),
                                  snake(v[4 * q + 3], __ldg(al + 4 * q + 3), __ldg(ai + 4 * q + 3)));
        }
      }
    }
  } else if (tid == 128) {
    // ---- MMA issuer
    constexpr uint32_t idesc = idesc_tf32_f32(128, N);
    bool ok_run = true;
    for (int it = 0; it < n_iter; ++it) {
      const int st = it % S;
      if (!fcv::mbar_wait(full(st), (it / S) & 1, 262, abrt)) { ok_run = false; break; }
      fcv::tc_fence_after();
      const uint64_t dah = fcv::sdesc_sw128(a_hi(st)), dal = fcv::sdesc_sw128(a_lo(st));
      const uint64_t dbh = fcv::sdesc_sw128(b_hi(st)), dbl = fcv::sdesc_sw128(b_lo(st));
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        umma_tf32(tmem, dah + 2 * kk, dbh + 2 * kk, idesc, (it | kk) != 0);
        umma_tf32(tmem, dah + 2 * kk, dbl + 2 * kk, idesc, 1);
        umma_tf32(tmem, dal + 2 * kk, dbh + 2 * kk, idesc, 1);
      }
      fcv::umma_commit(empty(st));
    }
    if (ok_run) fcv::umma_commit(done);
  }
  fcv::tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    fcv::tc_fence_after();
    fcv::tmem_dealloc(tmem, N);
  }
}

// f0 = |classifier(h)| (f0_predictor.py:101-103) in float64, rounded to float32
// (generator.py:732).  One warp per frame.
__global__ void f0_head_kernel(const double* __restrict__ h, int rows, int C, const double* __restrict__ w,
                               double b, float* __restrict__ f0) {
  griddep_wait();
  griddep_launch();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  double s = 0.0;
  for (int c = lane; c < C; c += 32) s = fma(h[(size_t)warp * C + c], w[c], s);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) f0[warp] = float(fabs(s + b));
}

// Per-frame source sines (SineGen2._f02sine, generator.py:214-233 in causal
// inference mode): radian step rad = (f0 * h / 24000) mod 1 per frame and
// harmonic, phase = float32(float64 prefix sum of rad) * 2 * pi * 480, held for
// the frame's 480 samples; writes 0.1 * sin(phase) as (frames, 9).  One block per
// document; the prefix sum runs in document order in float64, one thread per
// harmonic, like torch.cumsum's double accumulator on the CPU.
__global__ void __launch_bounds__(256) source_phase_kernel(const float* __restrict__ f0, const int* __restrict__ f0_cu,
                                                           float* __restrict__ sines) {
  griddep_wait();
  griddep_launch();
  constexpr int CH = 256;
  __shared__ float rad[CH][kHarm];
  __shared__ double carry[kHarm];
  const int d = blockIdx.x;
  const int off = f0_cu[d], n = f0_cu[d + 1] - off;
  if (threadIdx.x < kHarm) carry[threadIdx.x] = 0.0;
  for (int f0c = 0; f0c < n; f0c += CH) {
    const int cnt = min(CH, n - f0c);
    __syncthreads();
    for (int e = threadIdx.x; e < cnt * kHarm; e += blockDim.x) {
      const int f = e / kHarm, h = e - f * kHarm;
      const float fn = __fmul_rn(f0[off + f0c + f], float(h + 1));
      rad[f][h] = fmodf(__fdiv_rn(fn, 24000.0f), 1.0f);
    }
    __syncthreads();
    if (threadIdx.x < kHarm) {
      const int h = threadIdx.x;
      double c = carry[h];
      for (int f = 0; f < cnt; ++f) {
        c += double(rad[f][h]);
        rad[f][h] = float(c);
      }
      carry[h] = c;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < cnt * kHarm; e += blockDim.x) {
      const int f = e / kHarm, h = e - f * kHarm;
      float ph = __fmul_rn(__fmul_rn(rad[f][h], 2.0f), 3.14159265358979323846f);
      ph = __fmul_rn(ph, float(kUpTotal));
      sines[(size_t)(off + f0c + f) * kHarm + h] = __fmul_rn(sinf(ph), 0.1f);
    }
  }
}

// Excitation s (SineGen2.forward + SourceModuleHnNSF, generator.py:241-262, 321-336):
// per sample, with frame f = t / 480 and uv = f0 > 10:
//   e_h = sine[f, h] * uv + amp * noise[t, h],  amp = uv ? 0.003 : 0.1 / 3
//   s = tanh(sum_h lw[h] e_h + lb)
// noise is the module's fixed uniform table, read from sample 0 in every document.
__global__ void source_kernel(const float* __restrict__ f0, const float* __restrict__ sines,
                              const int* __restrict__ f0_cu, const int* __restrict__ src_cu, int n_docs, int n_src,
                              const float* __restrict__ noise, const float* __restrict__ lw, float lb,
                              float* __restrict__ s) {
  griddep_wait();
  griddep_launch();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_src) return;
  const int d = find_doc(src_cu, n_docs, i);
  const int t = i - src_cu[d];
  const int fr = f0_cu[d] + t / kUpTotal;
  const float fv = f0[fr];
  const bool voiced = fv > 10.0f;
  const float amp = voiced ? 0.003f : __fdiv_rn(0.1f, 3.0f);
  const float* nz = noise + (size_t)t * kHarm;
  const float* sn = sines + (size_t)fr * kHarm;
  float y = 0.0f;
#pragma unroll
  for (int h = 0; h < kHarm; ++h) {
    const float e = __fadd_rn(voiced ? sn[h] : 0.0f, __fmul_rn(amp, nz[h]));
    y = fmaf(__ldg(lw + h), e, y);
  }
  s[i] = tanhf(__fadd_rn(y, lb));
}

// STFT of the excitation (torch.stft(s, 16, 4, 16, periodic hann, center=True,
// reflect), generator.py:413-419) as (frames, 18) rows: 9 real parts, 9
// imaginary parts.  One thread per frame; float64 DFT of the 16 windowed samples.
__global__ void stft_kernel(const float* __restrict__ s, const int* __restrict__ src_cu,
                            const int* __restrict__ stft_cu, int n_docs, int n_rows, float* __restrict__ spec) {
  griddep_wait();
  griddep_launch();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n_rows) return;
  const int d = find_doc(stft_cu, n_docs, r);
  const int m = r - stft_cu[d];
  const int off = src_cu[d], T = src_cu[d + 1] - off;
  double xw[kNfft];
#pragma unroll
  for (int n = 0; n < kNfft; ++n) {
    int q = m * kHop - kNfft / 2 + n;
    q = q < 0 ? -q : (q >= T ? 2 * (T - 1) - q : q);
    double sw, cw;
    sincospi(double(n) / 8.0, &sw, &cw);
    xw[n] = double(s[off + q]) * (0.5 - 0.5 * cw);
  }
#pragma unroll
  for (int k = 0; k < kBins; ++k) {
    double re = 0.0, im = 0.0;
#pragma unroll
    for (int n = 0; n < kNfft; ++n) {
      double sv, cv;
      sincospi(double((k * n) & 15) / 8.0, &sv, &cv);
      re = fma(xw[n], cv, re);
      im = fma(-xw[n], sv, im);
    }
    spec[(size_t)r * 18 + k] = float(re);
    spec[(size_t)r * 18 + kBins + k] = float(im);
  }
}

// Magnitude/phase head (generator.py:713-714, 421-424): per frame and bin,
// mag = min(exp(x[k]), 100), ph = sin(x[9 + k]); spectrum (mag cos ph, mag sin ph).
__global__ void spectrum_kernel(const float* __restrict__ post, int n_rows, float2* __restrict__ spec) {
  griddep_wait();
  griddep_launch();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_rows * kBins) return;
  const int r = i / kBins, k = i - r * kBins;
  const float mag = fminf(expf(post[(size_t)r * 18 + k]), 100.0f);
  const float ph = sinf(post[(size_t)r * 18 + kBins + k]);
  spec[i] = make_float2(__fmul_rn(mag, cosf(ph)), __fmul_rn(mag, sinf(ph)));
}

// Centred inverse STFT (torch.istft, generator.py:425-426) with the window-square
// envelope, then the +-0.99 clamp (:719).  One thread per output sample: sample n
// of a document sits at n + 8 of the overlap-add buffer and sums the one-sided
// inverse DFT of every frame covering it.  Documents with fewer samples than
// 4 * (frames - 1) (non-final chunks drop their last 480) just stop early.
__global__ void istft_kernel(const float2* __restrict__ spec, const int* __restrict__ frame_cu,
                             const int* __restrict__ audio_cu, int n_docs, int n_audio, float* __restrict__ audio) {
  griddep_wait();
  griddep_launch();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_audio) return;
  const int d = find_doc(audio_cu, n_docs, i);
  const int n = i - audio_cu[d];
  const int f_off = frame_cu[d], F = frame_cu[d + 1] - f_off;
  const int pos = n + kNfft / 2;
  const int m_lo = max(0, (pos - kNfft + kHop) / kHop), m_hi = min(F - 1, pos / kHop);
  double y = 0.0, env = 0.0;
  for (int m = m_lo; m <= m_hi; ++m) {
    const int q = pos - m * kHop;   // 0..15
    const float2* sp = spec + (size_t)(f_off + m) * kBins;
    double v = double(sp[0].x) + ((q & 1) ? -double(sp[8].x) : double(sp[8].x));
#pragma unroll
    for (int k = 1; k < 8; ++k) {
      double sv, cv;
      sincospi(double((k * q) & 15) / 8.0, &sv, &cv);
      v += 2.0 * (double(sp[k].x) * cv - double(sp[k].y) * sv);
    }
    v *= 1.0 / kNfft;
    double sw, cw;
    sincospi(double(q) / 8.0, &sw, &cw);
    const double w = 0.5 - 0.5 * cw;
    y = fma(w, v, y);
    env = fma(w, w, env);
  }
  const float o = float(y / env);
  audio[i] = fminf(fmaxf(o, -0.99f), 0.99f);
}

}  // namespace hift
