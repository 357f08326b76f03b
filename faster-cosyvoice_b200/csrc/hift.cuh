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
