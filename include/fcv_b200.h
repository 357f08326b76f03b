/*
 * fcv_b200.h -- C ABI of the B200-native packed DiT estimator.
 *
 * The library replaces the GPU work of the reference estimator
 * (faster_cosyvoice/token2wav/flashinfer_dit.py, FlashInferDiT) for one
 * hot path: the 22-block flow-matching DiT evaluated over cross-request
 * packed (ragged) batches.  Every entry point is stateless, takes raw device
 * pointers, sizes and a cudaStream_t (passed as void*), enqueues work on that
 * stream and returns an int status:
 *
 *    0  FCV_OK
 *   -1  FCV_EINVAL     invalid argument (message in fcv_last_error())
 *   -2  FCV_EUNSUPPORTED  shape / dtype outside what the kernels implement
 *   -3  FCV_ECUDA      a CUDA runtime/driver call failed
 *   -4  FCV_EDEVICE    a kernel reported a device-side error (bounded wait
 *                      expired); read it with fcv_device_error()
 *
 * The library never allocates device memory on the compute path: callers pass
 * a workspace sized by fcv_dit_workspace_bytes().  Nothing is synchronised
 * inside the compute entry points (no host<->device traffic), so every
 * compute entry point can be captured into a CUDA graph.
 *
 * Layout conventions (all row-major, C order):
 *   padded inputs x, mu, cond : (B, 80, T)  element type = dtype
 *   spks                      : (B, 80)     dtype
 *   t                         : (B,)        dtype
 *   packed activations        : (N, 1024)   N = sum of document lengths
 *   qkv                       : (N, 3072)   [Q | K | V], head h of Q at
 *                                           columns h*64 .. h*64+63 (NHD)
 *   cu_seqlens                : (B+1,) int32, cu[0] = 0, cu[B] = N
 */
#ifndef FCV_B200_H
#define FCV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FCV_OK 0
#define FCV_EINVAL (-1)
#define FCV_EUNSUPPORTED (-2)
#define FCV_ECUDA (-3)
#define FCV_EDEVICE (-4)

/* element types */
#define FCV_DTYPE_F32 0
#define FCV_DTYPE_BF16 1

/* fixed model geometry (builders.py:17-21) */
#define FCV_DIM 1024
#define FCV_HEADS 16
#define FCV_DIM_HEAD 64
#define FCV_FF_INNER 2048
#define FCV_MEL 80
#define FCV_IN_FEAT 320
#define FCV_CONV_K 31
#define FCV_CONV_GROUPS 16
#define FCV_ROPE_DIM 64

/* GEMM epilogues for fcv_gemm() */
#define FCV_EPI_BIAS 0          /* C = A W^T + b                           */
#define FCV_EPI_BIAS_GELU 1     /* C = gelu_tanh(A W^T + b)                */
#define FCV_EPI_BIAS_ROPE_QKV 2 /* C = A W^T + b, partial RoPE on Q/K head 0 */
#define FCV_EPI_BIAS_GATE_RES 3 /* h(f32) += gate[doc] * (A W^T + b)       */
#define FCV_EPI_BIAS_F32 4      /* C(f32) = A W^T + b                      */

/* Version / diagnostics ------------------------------------------------- */
int fcv_version(void);
/* Thread-local description of the last failure of this thread. */
const char* fcv_last_error(void);
/* Reads and clears the device error word of the current device (synchronises
 * the given stream).  *code = 0 when no kernel has reported an error. */
int fcv_device_error(int* code, void* stream);
/* Self-test of the bounded waits (no counterpart in the reference, whose
 * kernels come from FlashInfer, Triton and cuBLAS): one CTA in which one
 * thread waits on an mbarrier that nothing completes.  After limit_ns
 * (0 < limit_ns <= 4 s) the wait gives up, records device error 901 and
 * raises the CTA's abort flag, on which a second waiter (4 x limit_ns)
 * returns at once; observed (a device int32[2]) gets 0 for each wait that
 * returned false.  Lets a caller check that a stalled pipeline ends with an
 * error code the host can read (fcv_device_error) and leaves the context
 * usable, without faulting the GPU. */
int fcv_selftest_wait_expiry(unsigned long long limit_ns, int32_t* observed, void* stream);

/* Weights ---------------------------------------------------------------- */
/* Derived inference weights (FlashInferDiT.finalize_weights,
 * flashinfer_dit.py:228-313).  Matrices have element type `dtype`; biases and
 * tables are float32.  All pointers are device pointers. */
typedef struct fcv_dit_weights {
  int depth;          /* number of DiT blocks (22)                            */
  int dtype;          /* FCV_DTYPE_BF16 or FCV_DTYPE_F32                      */
  const void* time_w1;   /* (1024, 256)  time_embed.time_mlp.0.weight         */
  const float* time_b1;  /* (1024)                                            */
  const void* time_w2;   /* (1024, 1024) time_embed.time_mlp.2.weight         */
  const float* time_b2;  /* (1024)                                            */
  const void* ada_w;     /* (depth*6144 + 2048, 1024) all AdaLN projections   */
  const float* ada_b;    /* (depth*6144 + 2048), +1 folded into the scales    */
  const void* in_w;      /* (1024, 320)  input_embed.proj.weight              */
  const float* in_b;     /* (1024)                                            */
  const void* conv1_w;   /* (1024, 31*64) row g*64+co, column tap*64+ci        */
  const float* conv1_b;  /* (1024)                                            */
  const void* conv2_w;   /* (1024, 31*64)                                     */
  const float* conv2_b;  /* (1024)                                            */
  const void* qkv_w;     /* (depth, 3072, 1024) cat(to_q, to_k, to_v)          */
  const float* qkv_b;    /* (depth, 3072)                                     */
  const void* o_w;       /* (depth, 1024, 1024) attn.to_out.0                 */
  const float* o_b;      /* (depth, 1024)                                     */
  const void* ff1_w;     /* (depth, 2048, 1024) ff.ff.0.0                     */
  const float* ff1_b;    /* (depth, 2048)                                     */
  const void* ff2_w;     /* (depth, 1024, 2048) ff.ff.2                       */
  const float* ff2_b;    /* (depth, 1024)                                     */
  const void* out_w;     /* (80, 1024)   proj_out.weight                      */
  const float* out_b;    /* (80)                                              */
  const float* rope_cos; /* (rope_max_len, 32) cos(p * 10000^(-2j/64))        */
  const float* rope_sin; /* (rope_max_len, 32)                                */
  int rope_max_len;
} fcv_dit_weights;

/* One packed batch -------------------------------------------------------- */
typedef struct fcv_dit_batch {
  int B;             /* sequences (CFG rows included)                          */
  int T;             /* padded length of x / mu / cond / out                   */
  int N;             /* packed rows, sum of lengths                            */
  int max_len;       /* longest document                                      */
  int chunk;         /* 0: full attention inside a document; >0: chunk-causal */
  const void* x;     /* (B, 80, T) */
  const void* mu;    /* (B, 80, T) */
  const void* cond;  /* (B, 80, T) */
  const void* spks;  /* (B, 80)    */
  const void* t;     /* (B,)       */
  const int32_t* cu_seqlens;  /* (B+1)  device                                */
  const int32_t* doc_ids;     /* (N)    device                                */
  const int32_t* positions;   /* (N)    device                                */
  const int32_t* gap_rows;    /* (N + 30*(B+1)) device, see fcv_pack_layout   */
  const int32_t* attn_tiles;  /* (n_attn_tiles, 2) device: (doc, q0), 128 rows */
  int n_attn_tiles;
  void* out;         /* (B, 80, T); padding frames zeroed                      */
  int out_f32;       /* 0: out has element type dtype; 1: out is float32       */
  int packed;        /* 1: x, mu, cond and out are packed rows (N, 80) in
                      * document order (cu_seqlens), T is unused and nothing
                      * is padded; rows and spks 16-byte aligned.  0: the
                      * padded (B, 80, T) layout above.  The packed form
                      * serves the device-packed flow (flashinfer_flow.py
                      * 118-281 without its padded intermediate tensors).   */
  const int32_t* n_attn_tiles_dev; /* optional (device int): the work list's
                      * length, read on the device at run time; n_attn_tiles
                      * is then only its capacity.  Lets one captured CUDA
                      * graph serve every batch composition of a bucket
                      * (the packed counterpart of the reference's graph
                      * buckets, flashinfer_dit.py:742-826).               */
  const int32_t* attn_sched;  /* optional (device): per-CTA attention items from
                      * fcv_attn_schedule, for attn_sched_ctas CTAs; null:
                      * items dealt round robin.  Results do not depend on it. */
  int attn_sched_ctas;
  /* Streaming prefix reuse (optional; all null = off).  Document d continues
   * a prefix of doc_pos0[d] frames computed by earlier calls, whose state is
   * cached: it runs only its new rows, positions must be absolute (see
   * fcv_offset_positions), and packed must be 1.  Frames of chunks that were
   * complete in the previous call keep bit-identical trajectories, so the
   * result equals recomputing the whole prefix (flashinfer_flow.py:215-221). */
  const int32_t* doc_pos0;    /* (B) device: absolute position of d's first row   */
  const int32_t* doc_kv_base; /* (B) device: d's first row in a block's K/V cache */
  void* kv_cache;             /* device: depth consecutive blocks of kv_layer_rows
                               * x 2048 ([K | V], element type dtype); the new
                               * rows' K/V are appended at doc_kv_base[d] + their
                               * absolute positions, attention reads all keys
                               * [0, doc_pos0[d] + L_d) from it                  */
  long kv_layer_rows;
  const void* conv_ctx;       /* (B, 2, 30, 1024) device, dtype: left context of
                               * the two position convolutions (zeros for a
                               * fresh document)                                 */
  void* conv_ctx_out;         /* optional (B, 2, 30, 1024), not conv_ctx: the
                               * next call's context, the 30 rows before local
                               * row ctx_row0[d] (< 0: not written)             */
  const int32_t* ctx_row0;
  const float* shared_mods;   /* optional (device): one modulation row (depth*6144
                               * + 2048 floats, fcv_dit_modulations) that every
                               * document uses -- the ODE solver's documents
                               * share t (flashinfer_flow.py:55-58), and the
                               * schedule's ten t values repeat on every call --
                               * so the time embedding and the AdaLN GEMM are
                               * skipped; t is then unused                       */
} fcv_dit_batch;

/* Layout ------------------------------------------------------------------ */
/* Document lengths from a right-padded 0/1 mask (B, 1, T) of element type
 * dtype: lengths[b] = number of entries > 0.5.
 * Replaces flashinfer_dit.py:460 (mask[:, 0].sum(-1)); counts exactly. */
int fcv_mask_lengths(const void* mask, int dtype, int B, int T, int32_t* lengths,
                     void* stream);

/* Packed layout from device lengths (B,).  Replaces
 * FlashInferDiT._get_packed_layout (flashinfer_dit.py:364-405) and
 * RaggedAttentionRunner._make_indptr (flashinfer_attention.py:82-86):
 *   gather[n]    = b*T + p          (int64, for row n = cu[b] + p)
 *   doc_ids[n]   = b                (int32)
 *   positions[n] = p                (int32)
 *   cu_seqlens   = [0, cumsum(lengths)] (int32)
 * plus gap_rows (length max_rows + 30*(B+1), int32): the embedding's causal
 * convolution stores each document behind 30 zero rows; gap_rows[g] is the
 * packed row held by row g of that gapped layout, or -1 for a zero row.
 * max_rows bounds N (B*T is always safe); entries past N are not written. */
int fcv_pack_layout(const int32_t* lengths, int B, int T, int max_rows, int64_t* gather,
                    int32_t* doc_ids, int32_t* positions, int32_t* cu_seqlens,
                    int32_t* gap_rows, void* stream);

/* Scatter packed rows (N, 80) back to a zeroed padded (B, 80, T) tensor
 * (flashinfer_dit.py:535-543). */
int fcv_unpack_output(const void* packed, int dtype, const int32_t* cu_seqlens, int B, int T,
                      int N, void* out, void* stream);

/* Row kernels (flashinfer_kernels.py) ------------------------------------- */
/* out[n] = LN(h[n]) * scale[doc[n]] + shift[doc[n]]; LN affine-free, eps 1e-6,
 * float32 statistics.  h: (N,1024) of h_dtype; out: (N,1024) of out_dtype;
 * shift/scale rows are float32 at stride mod_stride (elements).
 * Replaces layer_norm_modulate_packed (flashinfer_kernels.py:83-108, 327-348). */
int fcv_ln_modulate(const void* h, int h_dtype, const float* shift, const float* scale,
                    const int32_t* doc_ids, long mod_stride, int N, void* out, int out_dtype,
                    void* stream);

/* h_out = h + gate[doc]*r ; norm = LN(h_out)*scale[doc] + shift[doc].
 * Replaces gate_residual_layer_norm_modulate_packed
 * (flashinfer_kernels.py:110-145, 351-378). h/h_out/r/norm share `dtype`. */
int fcv_gate_res_ln_modulate(const void* h, const float* gate, const void* r,
                             const float* shift, const float* scale,
                             const int32_t* doc_ids, long mod_stride, int N, void* h_out,
                             void* norm, int dtype, void* stream);

/* GEMM -------------------------------------------------------------------- */
/* C[M, Nout] = A[M, K] * W[Nout, K]^T + bias, epilogue `epi`, element type
 * dtype for A/W (bf16 -> tcgen05 tensor cores, f32 -> CUDA cores).
 * Replaces F.linear (flashinfer_dit.py:490, 500, 512, 535).
 * For FCV_EPI_BIAS_ROPE_QKV: aux_i32 = positions (M), rope tables required.
 * For FCV_EPI_BIAS_GATE_RES: C is the float32 residual h, aux_i32 = doc_ids,
 * gate rows at `gate` with stride gate_stride. */
int fcv_gemm(const void* A, const void* W, const float* bias, int M, int Nout, int K,
             int dtype, int epi, void* C, const int32_t* aux_i32, const float* gate,
             long gate_stride, const float* rope_cos, const float* rope_sin, void* stream);

/* Attention --------------------------------------------------------------- */
/* Ragged multi-head attention over packed documents: for every document d,
 * head h and query row q: softmax(Q K^T / 8 + mask) V, where the mask keeps
 * keys k < L_d, and, when chunk > 0, only k // chunk <= q // chunk.
 * qkv: (N, 3072) [Q|K|V] element type dtype; out: (N, 1024); N = cu_seqlens[B].
 * tiles: (n_tiles, 2) int32 (doc, q0) list of work-list entries of up to 384
 * query rows (three 128-row query tiles sharing their K/V tiles), built by
 * fcv_attn_tiles().  sched (device, optional): the balanced per-CTA item
 * list of fcv_attn_schedule for sched_ctas CTAs; null deals items round
 * robin (the result is the same either way).  Replaces the FlashInfer ragged
 * prefill of flashinfer_attention.py:36-142 + flashinfer_dit.py:501. */
int fcv_attention(const void* qkv, int dtype, const int32_t* cu_seqlens, int B, int N,
                  int max_len, int chunk, const int32_t* tiles, int n_tiles,
                  const int32_t* sched, int sched_ctas, void* out, void* stream);

/* Host helper: fill `tiles` (capacity `cap` pairs, host memory) with the
 * 384-row work-list entries of the documents, most expensive first.  Returns the
 * number of tiles or a negative status. */
int fcv_attn_tiles(const int32_t* lengths_host, int B, int chunk, int32_t* tiles, int cap);

/* Host helpers for a balanced attention launch (the FlashInfer plan's load
 * balancing, flashinfer_attention.py:110-120, done once per batch
 * composition).  fcv_attn_ctas: the CTA count of the persistent attention
 * launch for n_tiles work-list entries on the current device.
 * fcv_attn_schedule: assign the 16 * n_tiles items (tile t, head h) = t*16+h
 * to n_ctas CTAs, longest first to the least loaded (cost = the 128 x 64
 * key tiles of its one to three query tiles + 1; one CTA per SM);
 * writes offsets (n_ctas + 1) then the items grouped by CTA into `sched`
 * (capacity cap ints).  Returns the ints written or a negative status. */
int fcv_attn_ctas(int n_tiles);
int fcv_attn_schedule(const int32_t* lengths_host, int B, int chunk, const int32_t* tiles, int n_tiles,
                      int n_ctas, int32_t* sched, int cap);

/* Time embedding + AdaLN ---------------------------------------------------- */
/* temb (B,1024) f32 = TimestepEmbedding(t) (modules.py:606-616); silu_act
 * (B,1024, element type dtype) = SiLU(temb) for the modulation GEMM.  The
 * silu_act buffer must hold B*2304 elements: rows B*1024.. are scratch for the
 * sinusoid and the hidden layer.  In bf16 mode the sinusoid argument is
 * bf16(1000*t) and the sinusoid is rounded to bf16, as the reference computes
 * them in the input dtype. */
int fcv_time_embed(const fcv_dit_weights* w, const void* t, int B, float* temb,
                   void* silu_act, void* stream);

/* Allocation-free time embedding (no counterpart in the reference; the
 * reference only ever runs inside PyTorch, whose caching allocator hands out
 * its scratch).  Same result as fcv_time_embed, but silu_act only has to hold
 * the (B, 1024) outputs: the sinusoid and hidden-layer scratch rows live in a
 * file-scope device array of this library.  For callers that cannot allocate
 * device memory themselves: a host that binds only this C ABI and has no
 * device allocator of its own, code that runs while a stream is being
 * captured into a CUDA graph (cudaMalloc is not allowed then), or a real-time
 * audio thread that must not enter the allocator (it may synchronise the
 * device).  Limits and sharing:
 *   - B <= FCV_NOALLOC_MAX_B (512); larger B returns FCV_EINVAL.
 *   - The array holds FCV_NOALLOC_MAX_B * 1280 float32 (2.5 MiB); every GPU on
 *     which the library is loaded keeps it until the process exits.
 *   - The first call on a device looks up the array's device address with
 *     that device current; make that first call before any stream capture.
 *   - All calls on one device share the array, which keeps the last call's
 *     contents (nothing in it needs to start at zero): calls that overlap on
 *     the GPU (e.g. on two streams at once) race and must be serialised. */
#define FCV_NOALLOC_MAX_B 512
int fcv_time_embed_noalloc(const fcv_dit_weights* w, const void* t, int B, float* temb,
                           void* silu_act, void* stream);

/* ODE --------------------------------------------------------------------- */
/* Fused CFG combine + Euler step on (R, 80, T) float32 samples
 * (flashinfer_flow.py:55-70): x += dt * ((1+r) d[:R] - r d[R:]), d (2R, 80, T)
 * of element type d_dtype.  When x_next is not NULL it receives the next
 * estimator input, the CFG-repeated sample (2R, 80, T) in x_next_dtype. */
int fcv_cfg_euler(float* x, const void* d, int d_dtype, int R, int T, float dt, float cfg_rate,
                  void* x_next, int x_next_dtype, void* stream);

/* Tracing ----------------------------------------------------------------- */
/* Kernel classes timed by the executor when profiling is on. */
#define FCV_CAT_GEMM_QKV 0
#define FCV_CAT_GEMM_OUT 1
#define FCV_CAT_GEMM_FF1 2
#define FCV_CAT_GEMM_FF2 3
#define FCV_CAT_ATTENTION 4
#define FCV_CAT_LN 5
#define FCV_CAT_EMBED 6
#define FCV_CAT_ADALN 7
#define FCV_CAT_OUTPUT 8
#define FCV_CAT_COUNT 9
/* When on, fcv_dit_forward brackets every launch with CUDA events on its
 * stream (the reference has no equivalent; it has only host wall clocks). */
int fcv_profile_enable(int on);
/* Synchronises the recorded events and writes, per class, the summed device
 * milliseconds and the number of launches since the last collect. */
int fcv_profile_collect(float* ms, int* launches, int n_categories);
/* Number of kernels this library has launched in this process. */
long fcv_launch_count(void);

/* Whole estimator call ---------------------------------------------------- */
/* Bytes of workspace fcv_dit_forward needs for N packed rows, B sequences. */
size_t fcv_dit_workspace_bytes(int N, int B, int depth, int dtype);

/* One estimator evaluation (FlashInferDiT.forward -> _forward_packed,
 * flashinfer_dit.py:315-362, 447-543): embed, 22 DiT blocks, final norm,
 * proj_out, unpack into batch->out.  `workspace` must be 256-byte aligned. */
int fcv_dit_forward(const fcv_dit_weights* w, const fcv_dit_batch* batch, void* workspace,
                    size_t workspace_bytes, void* stream);

/* The AdaLN modulation row of one timestep (TimestepEmbedding + every block's
 * AdaLayerNormZero and the final norm, flashinfer_dit.py:430-445) for
 * fcv_dit_batch.shared_mods: t is one value of the weights' dtype on the
 * device, mods receives depth*6144 + 2048 floats; workspace as
 * fcv_dit_workspace_bytes(0, 1, depth, dtype). */
int fcv_dit_modulations(const fcv_dit_weights* w, const void* t, float* mods, void* workspace,
                        size_t workspace_bytes, void* stream);

/* positions[n] += doc_pos0[doc_ids[n]]: absolute positions for documents that
 * continue a cached prefix (see fcv_dit_batch).  Apply once per layout. */
int fcv_offset_positions(int32_t* positions, const int32_t* doc_ids, const int32_t* doc_pos0, int N,
                         void* stream);

/* Packed flow front end ----------------------------------------------------
 * Device-packed replacement of the per-request Python front end of
 * flow_inference_batched / flow_inference_batched_streaming
 * (flashinfer_flow.py:118-281; CausalMaskedDiffWithDiT.inference, flow.py:365-409).
 * Token rows are packed per request: request b owns input tokens
 * [token_cu[b], token_cu[b+1]) -- for a non-final stream the last 3 of them
 * are lookahead context -- and output token rows [out_cu[b], out_cu[b+1]),
 * out_len = in_len (final / offline) or in_len - 3 (non-final).  Its mel rows
 * are [ratio*out_cu[b], ratio*out_cu[b+1]). */
typedef struct fcv_flow_weights {
  int dtype;             /* FCV_DTYPE_*: element type of the tables and rows    */
  int vocab;             /* rows of the token table (6561)                      */
  const void* embed;     /* (vocab, 80) input_embedding.weight                  */
  const void* conv1_w;   /* (1024, 4*80): conv1.weight[o, c, k] at [o, k*80+c]  */
  const float* conv1_b;  /* (1024)                                              */
  const void* conv2_w;   /* (80, 3*1024): conv2.weight[o, c, k] at [o, k*1024+c] */
  const float* conv2_b;  /* (80)                                                */
} fcv_flow_weights;

/* Workspace bytes of fcv_flow_frontend for n_out_tokens output token rows. */
size_t fcv_flow_workspace_bytes(int n_out_tokens, int dtype);

/* mu_rows (ratio*n_out_tokens, 80), element type w->dtype, = the
 * PreLookaheadLayer (upsample_encoder.py:55-92) over every request's embedded
 * tokens (flashinfer_flow.py:148-149, 171-182), repeat-interleaved to the mel
 * rate (:150, 183).  Token ids are clamped at 0 (:148); ids >= vocab must be
 * rejected by the caller.  max_out_len = longest out_len. */
int fcv_flow_frontend(const fcv_flow_weights* w, const int32_t* tokens, const int32_t* token_cu,
                      const int32_t* out_cu, int B, int n_out_tokens, int max_out_len, int ratio,
                      void* workspace, size_t workspace_bytes, void* mu_rows, void* stream);

/* out (B, n_out) = W normalize(spk) + b: F.normalize then spk_embed_affine_layer
 * (flashinfer_flow.py:145-146, 219-220).  spk (B, dim) of spk_dtype; W (n_out,
 * dim) and out of dtype; the normalised vector is rounded to dtype as the
 * reference's module computes in its own dtype. */
int fcv_speaker_projection(const void* spk, int spk_dtype, int B, int dim, const void* w, const float* b,
                           int n_out, void* out, int dtype, void* stream);

/* cond rows (mel_cu[B], 80) of dtype: the prompt Mel of request b in its first
 * prompt_cu[b+1]-prompt_cu[b] rows, zeros after (_copy_prompt_features,
 * flashinfer_flow.py:95-115).  prompt (prompt_cu[B], 80) of dtype; every prompt
 * must fit its request (checked on the host by the caller). */
int fcv_prompt_rows(const void* prompt, const int32_t* prompt_cu, const int32_t* mel_cu, int B,
                    int max_mel_len, void* cond, int dtype, void* stream);

/* Channel-major padded (B, 80, T) -> packed rows: dst[cu[b]+p, c] =
 * src[b*batch_stride + c*T + p] for p < cu[b+1]-cu[b].  batch_stride 0
 * broadcasts one sequence (the fixed noise prefix, flashinfer_flow.py:266). */
int fcv_pack_rows(const void* src, int src_dtype, long batch_stride, int T, const int32_t* cu, int B,
                  int max_len, void* dst, int dst_dtype, void* stream);

/* ------------------------------------------------------------------ HiFT vocoder
 * CausalHiFTGenerator (cosyvoice/hifigan/generator.py:578-740) as built by
 * builders.py:38-50, over packed requests.  Replaces the per-request
 * hift.inference(speech_feat=mel, finalize=...) calls of token2wav.py:130-131
 * and :194-195 with one call for a whole batch.
 *
 * Convolutions are indexed 0..79 in this order:
 *   0            conv_pre                       80 -> 512, k 5, right look-ahead 4
 *   1..3         ups.{0,1,2}                    nearest x8/x5/x3 then k 16/11/7 causal
 *   4..6         source_downs.{0,1,2}           18 -> 256/128/64, k 30/6/1, stride 15/3/1
 *   7 + 6i + 2s  source_resblocks.{i}.convs1.{s} (+1: convs2.{s}), i, s in 0..2
 *   25 + 6n + 2s resblocks.{n}.convs1.{s}       (+1: convs2.{s}), n = 3 level + kernel, 0..8
 *   79           conv_post                      64 -> 18, k 7 causal
 * Weights (weight norm folded) are float32 [k][roundup(C_in, 16)][roundup(C_out, 64)],
 * zero in the padding; biases float32 [roundup(C_out, 64)].  Snake parameters
 * are given at the index of the convs1 they surround: snake_alpha / snake_inv
 * (activations1, applied to convs1's input) and snake2_alpha / snake2_inv
 * (activations2, applied to convs1's output); inv = 1 / (alpha + 1e-9) in float32.
 * The f0 predictor (f0_predictor.py:60-103) is float64: condnet convs 0..4 as
 * [k][C_in][512] (k 4 then 3), classifier (512) + bias. */
#define FCV_HIFT_CONVS 80
#define FCV_HIFT_SAMPLES_PER_FRAME 480

typedef struct fcv_hift_weights {
  const float* conv_w[FCV_HIFT_CONVS];
  const float* conv_b[FCV_HIFT_CONVS];
  const float* snake_alpha[FCV_HIFT_CONVS];
  const float* snake_inv[FCV_HIFT_CONVS];
  const float* snake2_alpha[FCV_HIFT_CONVS];
  const float* snake2_inv[FCV_HIFT_CONVS];
  /* Residual-block convolutions (7..78) on the tensor cores: weights as
   * [k][C_out][C_in] float32 split into a tf32 head (w rounded to the nearest tf32,
   * low 13 mantissa bits zero) and the float32 remainder w - head; null runs the
   * convolution on the SIMT path. */
  const float* tc_w_hi[FCV_HIFT_CONVS];
  const float* tc_w_lo[FCV_HIFT_CONVS];
  const double* f0_w[5];
  const double* f0_b[5];
  const double* f0_cls_w;
  double f0_cls_b;
  const float* source_w;     /* m_source.l_linear.weight (9) */
  float source_b;            /* m_source.l_linear.bias */
  const float* noise;        /* (noise_rows, 9) l_sin_gen.sine_waves (generator.py:187) */
  long long noise_rows;
} fcv_hift_weights;

/* Per-document row layout, 9 int32 cu arrays of n_docs + 1 entries each, in
 * this order (L = given mel frames, F0 = L offline or L - 3 non-final, X = F0 or
 * F0 - 4 non-final):
 *   mel (L), f0 (F0), x (X), source (480 F0), stft (120 F0 + 1),
 *   level0 (8 X), level1 (40 X), level2 (120 X + 1), audio (480 X, non-final 480 X - 480). */
#define FCV_HIFT_LAYOUT_ARRAYS 9

typedef struct fcv_hift_batch {
  int n_docs;
  const float* mel;          /* packed mel rows (rows of the mel array, 80) */
  const int32_t* layout;     /* device, FCV_HIFT_LAYOUT_ARRAYS * (n_docs + 1) int32 */
  int rows[FCV_HIFT_LAYOUT_ARRAYS]; /* host copy of each array's last entry (totals) */
  int max_src;               /* longest document's source samples (480 F0): noise rows needed */
  float* audio;              /* (rows[8]) packed speech samples */
  float* source;             /* optional (rows[3]) excitation s (generator.py:737) */
  float* f0;                 /* optional (rows[1]) f0 */
} fcv_hift_batch;

/* Workspace bytes of fcv_hift_forward for these totals (rows as in fcv_hift_batch). */
size_t fcv_hift_workspace_bytes(const int* rows);

/* speech = CausalHiFTGenerator.inference(mel, finalize) (generator.py:728-740)
 * of every document: f0 predictor, source excitation, STFT, decode network,
 * inverse STFT and clamp, documents independent (causal per document).  The
 * noise table must hold max_src rows.  float32 like the reference's module
 * (float64 f0 predictor). */
int fcv_hift_forward(const fcv_hift_weights* w, const fcv_hift_batch* batch, void* workspace,
                     size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FCV_B200_H */
