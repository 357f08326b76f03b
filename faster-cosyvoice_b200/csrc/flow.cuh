// flow.cuh -- packed flow front end (flashinfer_flow.py:118-281): the windows of the
// pre-lookahead convolutions over packed token rows, mu rows at the mel rate,
// the speaker projection, prompt condition rows, channel-major -> row packing
// (noise), and the packed-row input gather of the estimator.
//
// Token rows are packed per document: document b owns input token rows
// [icu[b], icu[b+1]) (context tokens of a non-final stream included) and output
// token rows [ocu[b], ocu[b+1]); mel rows are [ratio*ocu[b], ratio*ocu[b+1]).
// None of these kernels is on the per-NFE critical path except
// embed_rows_kernel; they run once per flow call.
#pragma once

#include "fcv_common.cuh"

namespace fcv {

constexpr int kFlowIn = 80;     // token feature width (input_size, builders.py:40)
constexpr int kFlowHid = 1024;  // PreLookaheadLayer channels (builders.py:42-43)
constexpr int kLookK = 4;       // conv1 kernel = pre_lookahead_len + 1 (upsample_encoder.py:61-65)
constexpr int kCausalK = 3;     // conv2 kernel (upsample_encoder.py:66-69)

__device__ __forceinline__ int clamp_token(int tk, int vocab) {
  // clamp(min=0) as the reference (flashinfer_flow.py:148); ids >= vocab are
  // rejected on the host, the upper clamp only keeps the read in bounds
  return tk < 0 ? 0 : (tk >= vocab ? vocab - 1 : tk);
}

// conv1 window of output token row p of document b (upsample_encoder.py:77-84):
// a1[ocu[b]+p, k*80 + c] = table[tok[icu[b]+p+k], c] for p+k < L_in, else 0.
// Grid (ceil(max_out/8), B), 256 threads: one warp per row.
template <typename T>
__global__ void __launch_bounds__(256) token_window_kernel(const int32_t* __restrict__ tokens,
                                                           const int32_t* __restrict__ icu,
                                                           const int32_t* __restrict__ ocu,
                                                           const T* __restrict__ table, int vocab,
                                                           T* __restrict__ a1) {
  griddep_wait();
  griddep_launch();
  const int b = blockIdx.y;
  const int i0 = icu[b], L = icu[b + 1] - i0;
  const int o0 = ocu[b], n = ocu[b + 1] - o0;
  const int lane = threadIdx.x & 31;
  for (int p = blockIdx.x * 8 + (threadIdx.x >> 5); p < n; p += gridDim.x * 8) {
    T* dst = a1 + (long)(o0 + p) * (kLookK * kFlowIn);
#pragma unroll
    for (int k = 0; k < kLookK; ++k) {
      const int q = p + k;
      const T* src = q < L ? table + (long)clamp_token(tokens[i0 + q], vocab) * kFlowIn : nullptr;
      for (int c = lane; c < kFlowIn; c += 32) dst[k * kFlowIn + c] = src ? src[c] : from_f<T>(0.f);
    }
  }
}

// conv2 window (causal, two zero rows on the left: upsample_encoder.py:86-87):
// a2[o0+p, k*1024 + c] = h1[o0+p-2+k, c] for p-2+k >= 0, else 0.  16-byte copies;
// h1 and a2 rows are 16-byte aligned.  Grid (ceil(max_out/8), B), one warp per row.
template <typename T>
__global__ void __launch_bounds__(256) causal_window_kernel(const int32_t* __restrict__ ocu,
                                                            const T* __restrict__ h1, T* __restrict__ a2) {
  griddep_wait();
  griddep_launch();
  constexpr int V = kFlowHid * (int)sizeof(T) / 16;  // 16-byte vectors per tap
  const int b = blockIdx.y;
  const int o0 = ocu[b], n = ocu[b + 1] - o0;
  const int lane = threadIdx.x & 31;
  for (int p = blockIdx.x * 8 + (threadIdx.x >> 5); p < n; p += gridDim.x * 8) {
    uint4* dst = reinterpret_cast<uint4*>(a2 + (long)(o0 + p) * (kCausalK * kFlowHid));
#pragma unroll
    for (int k = 0; k < kCausalK; ++k) {
      const int q = p - (kCausalK - 1) + k;
      const uint4* src = q >= 0 ? reinterpret_cast<const uint4*>(h1 + (long)(o0 + q) * kFlowHid) : nullptr;
      for (int v = lane; v < V; v += 32) dst[k * V + v] = src ? __ldg(src + v) : make_uint4(0, 0, 0, 0);
    }
  }
}

// mu rows at the mel rate (upsample_encoder.py:91 residual, flashinfer_flow.py:153
// repeat_interleave): mu[ratio*o0 + m, c] = c2[o0 + m/ratio, c] + table[tok[i0 + m/ratio], c].
// Grid (ceil(ratio*max_out/8), B), one warp per mel row.
template <typename T>
__global__ void __launch_bounds__(256) mu_rows_kernel(const int32_t* __restrict__ tokens,
                                                      const int32_t* __restrict__ icu,
                                                      const int32_t* __restrict__ ocu,
                                                      const T* __restrict__ table, int vocab,
                                                      const float* __restrict__ c2, int ratio,
                                                      T* __restrict__ mu) {
  griddep_wait();
  griddep_launch();
  const int b = blockIdx.y;
  const int i0 = icu[b];
  const int o0 = ocu[b], n = (ocu[b + 1] - o0) * ratio;
  const int lane = threadIdx.x & 31;
  for (int m = blockIdx.x * 8 + (threadIdx.x >> 5); m < n; m += gridDim.x * 8) {
    const int p = m / ratio;
    const T* e = table + (long)clamp_token(tokens[i0 + p], vocab) * kFlowIn;
    const float* h = c2 + (long)(o0 + p) * kFlowIn;
    T* dst = mu + ((long)o0 * ratio + m) * kFlowIn;
    for (int c = lane; c < kFlowIn; c += 32) dst[c] = from_f<T>(h[c] + to_f<T>(e[c]));
  }
}

// Speaker projection (flashinfer_flow.py:145-146, 219-220): x = spk / max(|spk|, 1e-12)
// rounded to the weight type, out = W x + b.  One block of 128 threads per row.
template <typename Tin, typename T>
__global__ void __launch_bounds__(128) speaker_projection_kernel(const Tin* __restrict__ spk, int dim,
                                                                 const T* __restrict__ w,
                                                                 const float* __restrict__ bias, int n_out,
                                                                 T* __restrict__ out) {
  griddep_wait();
  griddep_launch();
  extern __shared__ float xs[];  // dim
  __shared__ float part[4];
  const int b = blockIdx.x;
  float ss = 0.f;
  for (int c = threadIdx.x; c < dim; c += blockDim.x) {
    const float v = to_f<Tin>(spk[(long)b * dim + c]);
    xs[c] = v;
    ss += v * v;
  }
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  const float nrm = sqrtf(part[0] + part[1] + part[2] + part[3]);
  const float inv = 1.0f / fmaxf(nrm, 1e-12f);
  for (int c = threadIdx.x; c < dim; c += blockDim.x) xs[c] = to_f<T>(from_f<T>(xs[c] * inv));
  __syncthreads();
  for (int o = threadIdx.x; o < n_out; o += blockDim.x) {
    const T* wr = w + (long)o * dim;
    float acc = bias ? bias[o] : 0.f;
    for (int c = 0; c < dim; ++c) acc += to_f<T>(wr[c]) * xs[c];
    out[(long)b * n_out + o] = from_f<T>(acc);
  }
}

// Prompt condition rows (flashinfer_flow.py:95-115): cond[mcu[b] + m, c] =
// prompt[pcu[b] + m, c] for m < Lp_b, else 0.  Grid (ceil(max_mel/8), B).
template <typename T>
__global__ void __launch_bounds__(256) prompt_rows_kernel(const T* __restrict__ prompt,
                                                          const int32_t* __restrict__ pcu,
                                                          const int32_t* __restrict__ mcu, T* __restrict__ cond) {
  griddep_wait();
  griddep_launch();
  const int b = blockIdx.y;
  const int p0 = pcu[b], lp = pcu[b + 1] - p0;
  const int m0 = mcu[b], n = mcu[b + 1] - m0;
  const int lane = threadIdx.x & 31;
  for (int m = blockIdx.x * 8 + (threadIdx.x >> 5); m < n; m += gridDim.x * 8) {
    T* dst = cond + (long)(m0 + m) * kFlowIn;
    const T* src = m < lp ? prompt + (long)(p0 + m) * kFlowIn : nullptr;
    for (int c = lane; c < kFlowIn; c += 32) dst[c] = src ? src[c] : from_f<T>(0.f);
  }
}

// Channel-major padded -> packed rows: dst[cu[b] + p, c] = src[b*bstride + c*T + p]
// for p < L_b (80 channels).  Grid (ceil(max_len/32), B), 256 threads, a 32-position
// tile transposed through shared memory (both sides coalesced).
template <typename Ts, typename Td>
__global__ void __launch_bounds__(256) pack_rows_kernel(const Ts* __restrict__ src, long bstride, int T_,
                                                        const int32_t* __restrict__ cu, Td* __restrict__ dst) {
  griddep_wait();
  griddep_launch();
  __shared__ float tile[kFlowIn][33];
  const int b = blockIdx.y;
  const int p0 = blockIdx.x * 32;
  const int L = cu[b + 1] - cu[b];
  if (p0 >= L) return;
  const int w = threadIdx.x >> 5, pp = threadIdx.x & 31;
  for (int c = w; c < kFlowIn; c += 8)
    tile[c][pp] = p0 + pp < L ? to_f<Ts>(src[(long)b * bstride + (long)c * T_ + p0 + pp]) : 0.f;
  __syncthreads();
  const long row0 = cu[b] + p0;
  for (int i = threadIdx.x; i < 32 * kFlowIn; i += blockDim.x) {
    const int r = i / kFlowIn, c = i - r * kFlowIn;
    if (p0 + r < L) dst[(row0 + r) * kFlowIn + c] = from_f<Td>(tile[c][r]);
  }
}

// Estimator input over packed rows (dit.py:91-96 order):
// a_in[n, :] = [x[n, :], cond[n, :], mu[n, :], spks[doc[n], :]], every operand (rows, 80).
// 16-byte copies (an 80-element row is 160 or 320 bytes).  One warp per row.
template <typename T>
__global__ void __launch_bounds__(256) embed_rows_kernel(const T* __restrict__ x, const T* __restrict__ cond,
                                                         const T* __restrict__ mu, const T* __restrict__ spks,
                                                         const int32_t* __restrict__ doc, long N,
                                                         T* __restrict__ a_in) {
  griddep_wait();
  griddep_launch();
  constexpr int V = kFlowIn * (int)sizeof(T) / 16;  // vectors per 80-element row
  const int lane = threadIdx.x & 31;
  for (long n = blockIdx.x * 8L + (threadIdx.x >> 5); n < N; n += gridDim.x * 8L) {
    uint4* dst = reinterpret_cast<uint4*>(a_in + n * (4 * kFlowIn));
    const long srow = (long)__ldg(doc + n) * kFlowIn;
    for (int v = lane; v < 4 * V; v += 32) {
      const int s = v / V;
      const T* base = s == 0 ? x + n * kFlowIn : (s == 1 ? cond + n * kFlowIn : (s == 2 ? mu + n * kFlowIn : spks + srow));
      dst[v] = __ldg(reinterpret_cast<const uint4*>(base) + (v - s * V));
    }
  }
}

// ------------------------------------------------------------------ streaming prefix reuse
// A document continuing a cached prefix runs only its rows from absolute
// position pos0[d] on.  The kernels below give it the cached state of the
// earlier rows: RoPE positions, the convolutions' left context and the keys.

// positions[n] += pos0[doc[n]] (absolute RoPE positions of the new rows).
__global__ void offset_positions_kernel(const int32_t* __restrict__ doc, const int32_t* __restrict__ pos0, long N,
                                        int32_t* __restrict__ positions) {
  griddep_wait();
  griddep_launch();
  for (long n = blockIdx.x * (long)blockDim.x + threadIdx.x; n < N; n += (long)gridDim.x * blockDim.x)
    positions[n] += __ldg(pos0 + __ldg(doc + n));
}

// The 30 gap rows in front of document d (rows cu[d] + 30 d + r of both gapped
// buffers) take the cached left context ctx[d][buffer][r] ((B, 2, 30, 1024));
// the group after the last document stays zero.  Grid (30, B + 1).
template <typename T>
__global__ void gap_context_kernel(const int32_t* __restrict__ cu, int B, const T* __restrict__ ctx,
                                   T* __restrict__ buf0, T* __restrict__ buf1) {
  griddep_wait();
  griddep_launch();
  const int d = blockIdx.y, r = blockIdx.x;
  const long g = (long)cu[d] + 30L * d + r;
  constexpr int kVec = 16 / sizeof(T);
  const uint4 z = make_uint4(0, 0, 0, 0);
  const T* c0 = d < B ? ctx + ((long)d * 2 * 30 + r) * kFlowHid : nullptr;
  const T* c1 = d < B ? ctx + ((long)d * 2 * 30 + 30 + r) * kFlowHid : nullptr;
  for (int c = threadIdx.x * kVec; c < kFlowHid; c += blockDim.x * kVec) {
    *reinterpret_cast<uint4*>(buf0 + g * kFlowHid + c) = c0 ? *reinterpret_cast<const uint4*>(c0 + c) : z;
    *reinterpret_cast<uint4*>(buf1 + g * kFlowHid + c) = c1 ? *reinterpret_cast<const uint4*>(c1 + c) : z;
  }
}

// The next call's left context of document d: the 30 rows ending before its
// local row row0[d] (row0[d] < 0: keep nothing, the caller keeps the old one).
// Rows before local row 0 come from this call's context ctx_in.  Writes
// ctx_out[d][buffer][r] from the gapped buffers (document d's local row p is
// gapped row cu[d] + 30 (d + 1) + p).  Grid (30, B).
template <typename T>
__global__ void context_save_kernel(const int32_t* __restrict__ cu, const int32_t* __restrict__ row0,
                                    const T* __restrict__ ctx_in, const T* __restrict__ buf0,
                                    const T* __restrict__ buf1, T* __restrict__ ctx_out) {
  griddep_wait();
  griddep_launch();
  const int d = blockIdx.y, r = blockIdx.x;
  const int start = __ldg(row0 + d);
  if (start < 0) return;
  const int p = start - 30 + r;  // local row feeding context row r
  constexpr int kVec = 16 / sizeof(T);
  const T* s0;
  const T* s1;
  if (p >= 0) {
    const long g = (long)cu[d] + 30L * (d + 1) + p;
    s0 = buf0 + g * kFlowHid;
    s1 = buf1 + g * kFlowHid;
  } else {
    s0 = ctx_in + ((long)d * 2 * 30 + 30 + p) * kFlowHid;
    s1 = ctx_in + ((long)d * 2 * 30 + 60 + p) * kFlowHid;
  }
  T* o0 = ctx_out + ((long)d * 2 * 30 + r) * kFlowHid;
  T* o1 = ctx_out + ((long)d * 2 * 30 + 30 + r) * kFlowHid;
  for (int c = threadIdx.x * kVec; c < kFlowHid; c += blockDim.x * kVec) {
    *reinterpret_cast<uint4*>(o0 + c) = *reinterpret_cast<const uint4*>(s0 + c);
    *reinterpret_cast<uint4*>(o1 + c) = *reinterpret_cast<const uint4*>(s1 + c);
  }
}

// Append the new rows' keys and values to the cache: cache[kv_base[d] + pos][0:2048]
// = qkv[n][1024:3072] with pos the row's absolute position.  One warp per row.
// A destination outside the cache's `rows` is skipped and reported (code 251).
template <typename T>
__global__ void __launch_bounds__(256) kv_append_kernel(const T* __restrict__ qkv, const int32_t* __restrict__ doc,
                                                        const int32_t* __restrict__ positions,
                                                        const int32_t* __restrict__ kv_base, long N, long rows,
                                                        T* __restrict__ cache) {
  griddep_wait();
  griddep_launch();
  constexpr int V = 2048 * (int)sizeof(T) / 16;
  const int lane = threadIdx.x & 31;
  for (long n = blockIdx.x * 8L + (threadIdx.x >> 5); n < N; n += gridDim.x * 8L) {
    const long dst = (long)__ldg(kv_base + __ldg(doc + n)) + __ldg(positions + n);
    if (dst < 0 || dst >= rows) {
      if (lane == 0) record_error(251);
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(qkv + n * 3072 + 1024);
    uint4* out = reinterpret_cast<uint4*>(cache + dst * 2048);
    for (int v = lane; v < V; v += 32) out[v] = __ldg(src + v);
  }
}

}  // namespace fcv
