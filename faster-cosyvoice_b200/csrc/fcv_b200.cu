// fcv_b200.cu -- C ABI of the B200 DiT estimator (include/fcv_b200.h).
//
// One translation unit: the kernels live in the .cuh files included below and
// share the device error word.  Host code here validates arguments, encodes
// TMA tensor maps, picks tile shapes and launches; fcv_dit_forward is the
// native executor of one estimator call (embed, 22 DiT blocks, output).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "fcv_b200.h"
#include "fcv_common.cuh"
#include "gemm.cuh"
#include "attn.cuh"
#include "rows.cuh"
#include "flow.cuh"
#include "hift.cuh"

using namespace fcv;

namespace {

thread_local std::string t_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

#define FCV_CUDA(expr)                                                                 \
  do {                                                                                 \
    cudaError_t e_ = (expr);                                                           \
    if (e_ != cudaSuccess)                                                             \
      return fail(FCV_ECUDA, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, \
                  __LINE__);                                                           \
  } while (0)

#define FCV_LAUNCH_CHECK(name)                                                          \
  do {                                                                                 \
    count_launch();                                                                    \
    cudaError_t e_ = cudaGetLastError();                                               \
    if (e_ != cudaSuccess) return fail(FCV_ECUDA, "launch of %s failed: %s", name, cudaGetErrorString(e_)); \
  } while (0)

#define FCV_TRY(expr)      \
  do {                     \
    int s_ = (expr);       \
    if (s_ != FCV_OK) return s_; \
  } while (0)



inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// ------------------------------------------------------------------ tracing
// Launch counter and optional CUDA-event timing of the executor's launches.
std::atomic<long> g_launches{0};
struct ProfState {
  bool on = false;
  std::vector<cudaEvent_t> pool;
  size_t next = 0;
  std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> marks;
  int open_cat = -1;
  cudaEvent_t open_ev = nullptr;
};
ProfState g_prof;
std::mutex g_prof_mu;

inline void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

// Programmatic dependent launch: kernels on one stream may start their
// prologue while the previous kernel finishes (every kernel opens with
// griddepcontrol.wait before touching memory).  FCV_PDL=0 in the environment
// launches them with plain stream serialisation instead.
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("FCV_PDL");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
int launch_k_opt(bool pdl, const char* name, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                 cudaStream_t s, Args... args) {
  count_launch();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (pdl && pdl_enabled()) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
  if (e != cudaSuccess) return fail(FCV_ECUDA, "launch of %s failed: %s", name, cudaGetErrorString(e));
  return FCV_OK;
}
template <typename... KArgs, typename... Args>
int launch_k(const char* name, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
             Args... args) {
  return launch_k_opt(true, name, kernel, grid, block, smem, s, args...);
}
#define FCV_LAUNCH(...)                        \
  do {                                         \
    const int rc_ = launch_k(__VA_ARGS__);     \
    if (rc_ != FCV_OK) return rc_;             \
  } while (0)

cudaEvent_t prof_event() {
  if (g_prof.next >= g_prof.pool.size()) return nullptr;
  return g_prof.pool[g_prof.next++];
}
// Record an event; inside a stream capture it becomes an external event node, so
// every replay of the graph records it where host code can read it.
void prof_record(cudaEvent_t e, cudaStream_t s) {
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &st) == cudaSuccess && st == cudaStreamCaptureStatusActive)
    cudaEventRecordWithFlags(e, s, cudaEventRecordExternal);
  else
    cudaEventRecord(e, s);
}
void prof_begin(int cat, cudaStream_t s) {
  if (!g_prof.on) return;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  cudaEvent_t e = prof_event();
  if (!e) return;
  prof_record(e, s);
  g_prof.open_cat = cat;
  g_prof.open_ev = e;
}
void prof_end(cudaStream_t s) {
  if (!g_prof.on) return;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  if (g_prof.open_ev == nullptr) return;
  cudaEvent_t e = prof_event();
  if (!e) {
    g_prof.open_ev = nullptr;
    return;
  }
  prof_record(e, s);
  g_prof.marks.push_back({g_prof.open_cat, {g_prof.open_ev, e}});
  g_prof.open_ev = nullptr;
}
struct ProfScope {
  cudaStream_t s;
  ProfScope(int cat, cudaStream_t st) : s(st) { prof_begin(cat, st); }
  ~ProfScope() { prof_end(s); }
};

// ------------------------------------------------------------------ tensor maps
typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                      const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                      const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                      CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PFN_encodeTiled_t encode_fn() {
  static PFN_encodeTiled_t fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled_t>(p);
  });
  return fn;
}

// 2-D tensor of `rows` x `cols` (row stride `ld` elements) with a box of
// box_cols x box_rows, 128-byte swizzle, zero fill out of bounds.
int make_tmap(CUtensorMap* m, const void* ptr, bool f32, long rows, long cols, long ld, int box_cols, int box_rows) {
  PFN_encodeTiled_t enc = encode_fn();
  if (!enc) return fail(FCV_ECUDA, "cuTensorMapEncodeTiled unavailable");
  const int es = f32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || ((ld * es) & 15))
    return fail(FCV_EINVAL, "TMA operand must be 16-byte aligned with a 16-byte multiple row stride");
  cuuint64_t gdim[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t gstride[1] = {static_cast<cuuint64_t>(ld * es)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                   const_cast<void*>(ptr), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FCV_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return FCV_OK;
}

int make_tmap_bf16(CUtensorMap* m, const void* ptr, long rows, long cols, long ld, int box_rows) {
  return make_tmap(m, ptr, false, rows, cols, ld, 64, box_rows);
}

// ------------------------------------------------------------------ GEMM launch
struct GemmCall {
  const void* A;
  long lda;        // elements
  long a_rows;     // rows of A (M, or gapped rows in conv mode)
  const void* W;   // (N, K)
  const float* bias;
  int M, N, K;
  int conv;
  EpiParams epi;
};

int choose_tma_out(const GemmCall& g, int bn);
int make_out_map(CUtensorMap* tc, const GemmCall& g, int tma_out, const CUtensorMap& fallback);

template <int BN, typename Tact>
int launch_tc(const GemmCall& g, cudaStream_t s) {
  using Cfg = TcGemmCfg<BN>;
  CUtensorMap ta, tb, tc;
  FCV_TRY(make_tmap_bf16(&ta, g.A, g.a_rows, g.K, g.lda, 128));
  FCV_TRY(make_tmap_bf16(&tb, g.W, g.N, g.K, g.K, BN));
  TcGemmArgs args{};
  args.num_kb = (g.K + 63) / 64;
  args.m_blocks = (g.M + 127) / 128;
  args.n_blocks = (g.N + BN - 1) / BN;
  args.epi = g.epi;
  args.tma_out = choose_tma_out(g, BN);
  FCV_TRY(make_out_map(&tc, g, args.tma_out, ta));
  const int tiles = args.m_blocks * args.n_blocks;
  const int grid = std::min(tiles, num_sms());
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    FCV_CUDA(cudaFuncSetAttribute(tc_gemm_kernel<BN, Tact>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  Cfg::SMEM_BYTES));
    attr_set[dev & 63] = true;
  }
  FCV_LAUNCH("tc_gemm_kernel", tc_gemm_kernel<BN, Tact>, dim3(grid), dim3(Cfg::THREADS), Cfg::SMEM_BYTES, s, ta, tb, tc, args);
  return FCV_OK;
}

// Output path of a GEMM: TMA store/reduce of 32-row x 128-byte tiles where the
// epilogue writes a plain row-major tile; direct per-thread stores otherwise.
int choose_tma_out(const GemmCall& g, int bn) {
  const int e = g.epi.epi;
  if (bn < 128) return 0;
  if ((e == EPI_BIAS || e == EPI_GELU || e == EPI_ROPE || e == EPI_SILU || e == EPI_LRELU) && g.N % 64 == 0) return 1;
  if (e == EPI_F32 && g.epi.C2 == nullptr && g.N % 32 == 0) return 1;
  if (e == EPI_GATE_RES && g.N % 32 == 0) return 2;
  return 0;
}

int make_out_map(CUtensorMap* tc, const GemmCall& g, int tma_out, const CUtensorMap& fallback) {
  if (tma_out == 1 && g.epi.epi != EPI_F32) return make_tmap(tc, g.epi.C, false, g.M, g.N, g.epi.ldc, 64, 32);
  if (tma_out != 0) return make_tmap(tc, g.epi.C, true, g.M, g.N, g.epi.ldc, 32, 32);
  *tc = fallback;  // unused by the kernel
  return FCV_OK;
}

// Clusters of two CTAs that can be resident at once (persistent grid size).
int max_pairs() {
  static int cached[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  int& c = cached[dev & 63];
  if (c == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * num_sms(), 1, 1);
    cfg.blockDim = dim3(TcPairCfg::THREADS, 1, 1);
    cfg.dynamicSmemBytes = TcPairCfg::SMEM_BYTES;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, tc_gemm_pair_kernel<bf16, false>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = num_sms() / 2;
    }
    c = std::min(n, num_sms() / 2);
  }
  return c;
}

template <typename Tact>
int launch_tc_pair(const GemmCall& g, cudaStream_t s) {
  using Cfg = TcPairCfg;
  CUtensorMap ta, tb, tb64, tc;
  FCV_TRY(make_tmap_bf16(&ta, g.A, g.a_rows, g.K, g.lda, 128));
  FCV_TRY(make_tmap_bf16(&tb, g.W, g.N, g.K, g.K, 128));
  TcGemmArgs args{};
  args.num_kb = (g.K + 63) / 64;
  args.m_blocks = (g.M + 255) / 256;
  args.n_blocks = (g.N + 255) / 256;
  // Persistent grid of CTA pairs.  For N <= 1024 the tiles of a last, partial
  // wave are split into two 256 x 128 pieces when the pieces still fit in one
  // wave.  A piece loads the whole A tile, so it is load-bound at ~3/4 of a tile
  // time; measured on B200 this shortens the 1-2 wave GEMMs (out, FF2) by ~5 %
  // and lengthens the many-wave QKV GEMM, so wider outputs are not split.
  const int tiles = args.m_blocks * args.n_blocks;
  const int grid_pairs = max_pairs();
  const int rem = tiles % grid_pairs;
  int split = 1;
  if (rem != 0 && args.n_blocks <= 4 && rem * 2 <= grid_pairs) split = 2;
  args.split = split;
  args.full_tiles = split > 1 ? tiles - rem : tiles;
  args.num_tiles = args.full_tiles + (tiles - args.full_tiles) * split;
  if (split > 1) FCV_TRY(make_tmap_bf16(&tb64, g.W, g.N, g.K, g.K, 64));
  else tb64 = tb;
  args.conv = 0;
  args.epi = g.epi;
  args.tma_out = choose_tma_out(g, 256);
  FCV_TRY(make_out_map(&tc, g, args.tma_out, ta));
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    FCV_CUDA(cudaFuncSetAttribute(tc_gemm_pair_kernel<Tact, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  Cfg::SMEM_BYTES));
    FCV_CUDA(cudaFuncSetAttribute(tc_gemm_pair_kernel<Tact, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  Cfg::SMEM_BYTES));
    attr_set[dev & 63] = true;
  }
  const int launch_pairs = std::max(1, std::min(args.num_tiles, grid_pairs));
  if (split > 1)
    FCV_LAUNCH("tc_gemm_pair_kernel", tc_gemm_pair_kernel<Tact, true>, dim3(2 * launch_pairs), dim3(Cfg::THREADS),
               Cfg::SMEM_BYTES, s, ta, tb, tb64, tc, args);
  else
    FCV_LAUNCH("tc_gemm_pair_kernel", tc_gemm_pair_kernel<Tact, false>, dim3(2 * launch_pairs), dim3(Cfg::THREADS),
               Cfg::SMEM_BYTES, s, ta, tb, tb64, tc, args);
  return FCV_OK;
}

// Causal grouped convolution (bf16): A = gapped buffer (a_rows x 1024, 160-row
// windows), B = (1024, 31*64) weights, one 64-channel group per tile column.
template <typename Tact>
int launch_conv(const GemmCall& g, cudaStream_t s) {
  using Cfg = ConvCfg;
  CUtensorMap ta, tb;
  FCV_TRY(make_tmap_bf16(&ta, g.A, g.a_rows, 1024, g.lda, Cfg::A_ROWS));
  FCV_TRY(make_tmap_bf16(&tb, g.W, g.N, g.K, g.K, 64));
  TcGemmArgs args{};
  args.num_kb = Cfg::TAPS;
  args.m_blocks = (g.M + 127) / 128;
  args.n_blocks = g.N / 64;
  args.conv = 1;
  args.epi = g.epi;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    FCV_CUDA(cudaFuncSetAttribute(tc_conv_kernel<Tact>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES));
    attr_set[dev & 63] = true;
  }
  const int tiles = args.m_blocks * args.n_blocks;
  FCV_LAUNCH("tc_conv_kernel", tc_conv_kernel<Tact>, dim3(std::min(tiles, num_sms())), dim3(Cfg::THREADS),
             Cfg::SMEM_BYTES, s, ta, tb, args);
  return FCV_OK;
}

int run_gemm(const GemmCall& g, int dtype, cudaStream_t s) {
  if (g.M <= 0 || g.N <= 0) return FCV_OK;
  if (dtype == FCV_DTYPE_BF16) {
    if (g.conv) return launch_conv<bf16>(g, s);
    if (g.K % 64 != 0) return fail(FCV_EUNSUPPORTED, "bf16 GEMM needs K %% 64 == 0 (K=%d)", g.K);
    // CTA pairs (256-row tiles) once there are rows to fill them.  Up to 1536 rows the
    // single-SM kernel is faster (a chain of the 88 block GEMMs of one estimator call,
    // measured on B200: 400 rows 959 vs 1162 us, 800 rows 1071 vs 1186 us, 1400 rows
    // 1219 vs 1255 us; 1600 rows 1319 vs 1307 us), and a GEMM of at most 128 rows (time
    // MLP, AdaLN modulation) is bound by streaming its weights either way
    if (g.N >= 256 && g.M > 1536) return launch_tc_pair<bf16>(g, s);
    const long mb = (g.M + 127) / 128;
    const long t256 = mb * ((g.N + 255) / 256);
    // 128-wide tiles only when 256-wide ones leave SMs idle: the AdaLN weight
    // stream (M = 16, N = 137216) runs at 4.2 TB/s on 256-wide tiles, 3.8 TB/s on 128
    if (g.N <= 128 || t256 < 2L * num_sms()) return launch_tc<128, bf16>(g, s);
    return launch_tc<256, bf16>(g, s);
  }
  SimtGemmArgs a;
  a.A = static_cast<const float*>(g.A);
  a.lda = g.lda;
  a.W = static_cast<const float*>(g.W);
  a.M = g.M;
  a.N = g.N;
  a.K = g.K;
  a.conv = g.conv;
  a.epi = g.epi;
  dim3 grid((g.N + 63) / 64, (g.M + 63) / 64);
  FCV_LAUNCH("simt_gemm_f32_kernel", simt_gemm_f32_kernel, dim3(grid), dim3(256), 0, s, a);
  return FCV_OK;
}

EpiParams make_epi(int epi, int M, int N, void* C, long ldc, const float* bias) {
  EpiParams e;
  memset(&e, 0, sizeof(e));
  e.epi = epi;
  e.M = M;
  e.N = N;
  e.C = C;
  e.ldc = ldc;
  e.bias = bias;
  return e;
}

// ------------------------------------------------------------------ attention launch
// Keys of a launch: by default the documents' own rows of the QKV buffer; for
// documents continuing a cached prefix, a K/V cache of `rows` x 2048 ([K | V])
// with per-document first key rows and absolute query offsets.
struct KvSrc {
  const void* kv = nullptr;  // null: the QKV buffer itself
  long rows = 0;
  const int32_t* pos0 = nullptr;
  const int32_t* kv_base = nullptr;
};

int run_attention(const void* qkv, int dtype, const int32_t* cu, int chunk, const int32_t* tiles,
                  int n_tiles, void* out, long n_rows, cudaStream_t s, const int32_t* n_tiles_dev = nullptr,
                  const int32_t* sched = nullptr, int sched_ctas = 0, const KvSrc& kvs = KvSrc()) {
  if (n_tiles <= 0) return FCV_OK;
  dim3 grid(n_tiles, FCV_HEADS);
  const int2* t2 = reinterpret_cast<const int2*>(tiles);
  const bool cached = kvs.kv != nullptr;
  AttnSrc src;
  src.cu = cu;
  src.pos0 = cached ? kvs.pos0 : nullptr;
  src.kv_base = cached ? kvs.kv_base : nullptr;
  const int k_col = cached ? 0 : 1024, v_col = cached ? 1024 : 2048;
  if (dtype == FCV_DTYPE_BF16) {
    // Q tiles of 128 rows from the (N, 3072) [Q|K|V] buffer; K/V tiles of kFaKv rows from it or the cache
    CUtensorMap tq, tkv;
    FCV_TRY(make_tmap(&tq, qkv, false, n_rows, 3072, 3072, 64, kFaRows));
    if (cached)
      FCV_TRY(make_tmap(&tkv, kvs.kv, false, kvs.rows, 2048, 2048, 64, kFaKv));
    else
      FCV_TRY(make_tmap(&tkv, qkv, false, n_rows, 3072, 3072, 64, kFaKv));
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev & 63]) {
      FCV_CUDA(cudaFuncSetAttribute(attn_fa_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kFaSmemBytes));
      attr[dev & 63] = true;
    }
    const int items = n_tiles * FCV_HEADS;
    // persistent, one CTA per SM (all 512 TMEM columns); a host schedule fixes the CTA count it was built for
    const int ctas = sched ? sched_ctas : std::min(items, num_sms());
    if (sched && (sched_ctas < 1 || sched_ctas > num_sms()))
      return fail(FCV_EINVAL, "attention schedule built for %d CTAs", sched_ctas);
    // Plain stream order: the work items are dealt to CTAs by index, and CTAs that
    // start early on the SMs freed first by the previous kernel would unbalance it.
    const int rc = launch_k_opt(false, "attn_fa_kernel", attn_fa_kernel, dim3(ctas), dim3(kFaThreads), kFaSmemBytes,
                                s, tq, tkv, src, t2, n_tiles, n_tiles_dev, sched, chunk, k_col, v_col,
                                static_cast<bf16*>(out));
    if (rc != FCV_OK) return rc;
  } else {
    const float* kv = cached ? static_cast<const float*>(kvs.kv) : static_cast<const float*>(qkv);
    const long kv_stride = cached ? 2048 : 3072;
    const long kv_rows = cached ? kvs.rows : n_rows;
    FCV_LAUNCH("attn_f32_kernel", attn_f32_kernel, dim3(grid), dim3(kAttnQTile), 0, s, static_cast<const float*>(qkv), src,
               kv, kv_rows, kv_stride, k_col, v_col, t2, n_tiles_dev, chunk, static_cast<float*>(out));
  }
  return FCV_OK;
}

template <typename Th, typename To>
int launch_ln(const void* h, const float* shift, const float* scale, const int32_t* doc_ids, long stride,
              int N, void* out, cudaStream_t s) {
  if (N <= 0) return FCV_OK;
  if (reinterpret_cast<uintptr_t>(h) & 15) return fail(FCV_EINVAL, "layer norm: h must be 16-byte aligned");
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    FCV_CUDA(cudaFuncSetAttribute(ln_modulate_kernel<Th, To>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  ln_smem_bytes<Th>()));
    attr[dev & 63] = true;
  }
  const int grid = std::min(num_sms(), (N + kLnWarps - 1) / kLnWarps);
  FCV_LAUNCH("ln_modulate_kernel", ln_modulate_kernel<Th, To>, dim3(grid), dim3(kLnWarps * 32), ln_smem_bytes<Th>(), s, 
      static_cast<const Th*>(h), shift, scale, doc_ids, stride, N, static_cast<To*>(out));
  return FCV_OK;
}

int run_ln(const void* h, int h_dtype, const float* shift, const float* scale, const int32_t* doc_ids,
           long stride, int N, void* out, int out_dtype, cudaStream_t s) {
  if (h_dtype == FCV_DTYPE_F32 && out_dtype == FCV_DTYPE_BF16)
    return launch_ln<float, bf16>(h, shift, scale, doc_ids, stride, N, out, s);
  if (h_dtype == FCV_DTYPE_F32 && out_dtype == FCV_DTYPE_F32)
    return launch_ln<float, float>(h, shift, scale, doc_ids, stride, N, out, s);
  if (h_dtype == FCV_DTYPE_BF16 && out_dtype == FCV_DTYPE_BF16)
    return launch_ln<bf16, bf16>(h, shift, scale, doc_ids, stride, N, out, s);
  if (h_dtype == FCV_DTYPE_BF16 && out_dtype == FCV_DTYPE_F32)
    return launch_ln<bf16, float>(h, shift, scale, doc_ids, stride, N, out, s);
  return fail(FCV_EINVAL, "unknown dtype");
}

bool valid_dtype(int d) { return d == FCV_DTYPE_F32 || d == FCV_DTYPE_BF16; }
size_t dsize(int d) { return d == FCV_DTYPE_BF16 ? 2 : 4; }
size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Workspace carve-up for fcv_dit_forward.
struct Workspace {
  float* temb;
  void* tsin;
  void* th1;
  void* silu;
  float* mods;
  float* h;
  void* a_in;
  void* gap0;
  void* gap1;
  void* norm;
  void* qkv;
  void* attn;
  void* mid;
  size_t total;
};

Workspace carve(uint8_t* base, int N, int B, int depth, int dtype) {
  const size_t es = dsize(dtype);
  const long G = (long)N + 30L * (B + 1);
  const long MS = (long)depth * 6144 + 2048;
  Workspace w;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    void* p = base ? base + off : nullptr;
    off += align256(bytes);
    return p;
  };
  w.temb = static_cast<float*>(take((size_t)B * 1024 * 4));
  w.tsin = take((size_t)std::max(B, 1) * 256 * es);
  w.th1 = take((size_t)std::max(B, 1) * 1024 * es);
  w.silu = take((size_t)std::max(B, 1) * 1024 * es);
  w.mods = static_cast<float*>(take((size_t)B * MS * 4));
  w.h = static_cast<float*>(take((size_t)N * 1024 * 4));
  w.a_in = take((size_t)N * 320 * es);
  w.gap0 = take((size_t)G * 1024 * es);
  w.gap1 = take((size_t)G * 1024 * es);
  w.norm = take((size_t)N * 1024 * es);
  w.qkv = take((size_t)N * 3072 * es);
  w.attn = take((size_t)N * 1024 * es);
  w.mid = take((size_t)N * 2048 * es);
  w.total = off;
  return w;
}

// temb = W2 silu(W1 sinus(t) + b1) + b2 ; silu_act = silu(temb)  (modules.py:606-616)
template <typename T>
int run_time_embed(const fcv_dit_weights* w, const void* t, int B, void* tsin, void* th1, float* temb,
                   void* silu_act, cudaStream_t s) {
  const int dtype = w->dtype;
  FCV_LAUNCH("time_sinusoid_kernel", time_sinusoid_kernel<T>, dim3(B), dim3(128), 0, s, static_cast<const T*>(t), dtype == FCV_DTYPE_BF16 ? 1 : 0,
                                            static_cast<T*>(tsin));
  GemmCall g1{};
  g1.A = tsin; g1.lda = 256; g1.a_rows = B; g1.W = w->time_w1; g1.M = B; g1.N = 1024; g1.K = 256;
  g1.epi = make_epi(EPI_SILU, B, 1024, th1, 1024, w->time_b1);
  FCV_TRY(run_gemm(g1, dtype, s));
  GemmCall g2{};
  g2.A = th1; g2.lda = 1024; g2.a_rows = B; g2.W = w->time_w2; g2.M = B; g2.N = 1024; g2.K = 1024;
  g2.epi = make_epi(EPI_F32, B, 1024, temb, 1024, w->time_b2);
  g2.epi.C2 = silu_act;
  return run_gemm(g2, dtype, s);
}

template <typename T>
int forward_impl(const fcv_dit_weights* w, const fcv_dit_batch* bt, const Workspace& ws, cudaStream_t s) {
  const int dtype = w->dtype;
  const int N = bt->N, B = bt->B, depth = w->depth;
  const long MS = (long)depth * 6144 + 2048;
  const long G = (long)N + 30L * (B + 1);
  const int G_rows = N + 30 * B;  // gapped rows that can hold data

  // 1. time embedding + all AdaLN projections (one GEMM, flashinfer_dit.py:430-445), or one
  // precomputed row shared by every document (the ODE solver's documents share t): stride 0
  const float* mods = bt->shared_mods ? bt->shared_mods : ws.mods;
  const long mstride = bt->shared_mods ? 0 : MS;
  if (!bt->shared_mods) {
    ProfScope ps(FCV_CAT_ADALN, s);
    FCV_TRY(run_time_embed<T>(w, bt->t, B, ws.tsin, ws.th1, ws.temb, ws.silu, s));
    GemmCall g{};
    g.A = ws.silu; g.lda = 1024; g.a_rows = B; g.W = w->ada_w; g.M = B; g.N = (int)MS; g.K = 1024;
    g.epi = make_epi(EPI_F32, B, (int)MS, ws.mods, MS, w->ada_b);
    FCV_TRY(run_gemm(g, dtype, s));
  }
  // frames p >= L_b of a padded (B, 80, T) output are zero (all of them when N = 0)
  auto zero_pad = [&]() -> int {
    const dim3 zgrid(80, B);
    if (bt->out_f32)
      FCV_LAUNCH("zero_padding_kernel", zero_padding_kernel<float>, zgrid, dim3(128), 0, s, bt->cu_seqlens, B, bt->T,
                 static_cast<float*>(bt->out));
    else
      FCV_LAUNCH("zero_padding_kernel", zero_padding_kernel<T>, zgrid, dim3(128), 0, s, bt->cu_seqlens, B, bt->T,
                 static_cast<T*>(bt->out));
    return FCV_OK;
  };
  if (N == 0) return (bt->packed || B == 0 || bt->T == 0) ? FCV_OK : zero_pad();

  // 2. input embedding: gather, proj (K=320), causal grouped conv x2 + Mish + residual
  {
    ProfScope ps(FCV_CAT_EMBED, s);
    if (bt->packed) {
      const int grid = (int)std::min<long>((N + 7) / 8, 16L * num_sms());
      FCV_LAUNCH("embed_rows_kernel", embed_rows_kernel<T>, dim3(grid), dim3(256), 0, s, static_cast<const T*>(bt->x),
                 static_cast<const T*>(bt->cond), static_cast<const T*>(bt->mu), static_cast<const T*>(bt->spks),
                 bt->doc_ids, (long)N, static_cast<T*>(ws.a_in));
    } else {
      dim3 grid((bt->T + 31) / 32, B);
      FCV_LAUNCH("embed_gather_kernel", embed_gather_kernel<T>, dim3(grid), dim3(256), 0, s, static_cast<const T*>(bt->x), static_cast<const T*>(bt->cond),
                                                  static_cast<const T*>(bt->mu), static_cast<const T*>(bt->spks),
                                                  bt->cu_seqlens, bt->T, static_cast<T*>(ws.a_in));
    }
    if (bt->conv_ctx)  // continuing documents: the cached rows are the convolutions' left context
      FCV_LAUNCH("gap_context_kernel", gap_context_kernel<T>, dim3(30, B + 1), dim3(128), 0, s, bt->cu_seqlens, B,
                 static_cast<const T*>(bt->conv_ctx), static_cast<T*>(ws.gap0), static_cast<T*>(ws.gap1));
    else
      FCV_LAUNCH("zero_gap_rows_kernel", zero_gap_rows_kernel<T>, dim3(30, B + 1), dim3(128), 0, s, bt->cu_seqlens,
                 static_cast<T*>(ws.gap0), static_cast<T*>(ws.gap1));
    GemmCall g{};
    g.A = ws.a_in; g.lda = 320; g.a_rows = N; g.W = w->in_w; g.M = N; g.N = 1024; g.K = 320;
    g.epi = make_epi(EPI_EMBED_GAP, N, 1024, ws.gap0, 1024, w->in_b);
    g.epi.aux = bt->doc_ids;
    FCV_TRY(run_gemm(g, dtype, s));
    GemmCall c1{};
    c1.A = ws.gap0; c1.lda = 1024; c1.a_rows = G; c1.W = w->conv1_w; c1.M = G_rows; c1.N = 1024;
    c1.K = 31 * 64; c1.conv = 1;
    c1.epi = make_epi(EPI_MISH_GAP, G_rows, 1024, ws.gap1, 1024, w->conv1_b);
    c1.epi.aux = bt->gap_rows;
    FCV_TRY(run_gemm(c1, dtype, s));
    if (bt->conv_ctx_out)  // both convolution inputs are in place: keep the next call's context
      FCV_LAUNCH("context_save_kernel", context_save_kernel<T>, dim3(30, B), dim3(128), 0, s, bt->cu_seqlens,
                 bt->ctx_row0, static_cast<const T*>(bt->conv_ctx), static_cast<const T*>(ws.gap0),
                 static_cast<const T*>(ws.gap1), static_cast<T*>(bt->conv_ctx_out));
    GemmCall c2 = c1;
    c2.A = ws.gap1; c2.W = w->conv2_w;
    c2.epi = make_epi(EPI_MISH_RES, G_rows, 1024, ws.h, 1024, w->conv2_b);
    c2.epi.aux = bt->gap_rows;
    c2.epi.res = ws.gap0;
    FCV_TRY(run_gemm(c2, dtype, s));
  }

  // 3. DiT blocks (flashinfer_dit.py:485-533; DiTBlock.forward modules.py:516-530)
  const size_t es = dsize(dtype);
  for (int i = 0; i < depth; ++i) {
    const float* mi = mods + (long)i * 6144;
    {
      ProfScope ps(FCV_CAT_LN, s);
      FCV_TRY(run_ln(ws.h, FCV_DTYPE_F32, mi + 0, mi + 1024, bt->doc_ids, mstride, N, ws.norm, dtype, s));
    }
    GemmCall q{};
    q.A = ws.norm; q.lda = 1024; q.a_rows = N; q.M = N; q.N = 3072; q.K = 1024;
    q.W = static_cast<const uint8_t*>(w->qkv_w) + (size_t)i * 3072 * 1024 * es;
    q.epi = make_epi(EPI_ROPE, N, 3072, ws.qkv, 3072, w->qkv_b + (long)i * 3072);
    q.epi.aux = bt->positions;
    q.epi.rope_cos = w->rope_cos;
    q.epi.rope_sin = w->rope_sin;
    {
      ProfScope ps(FCV_CAT_GEMM_QKV, s);
      FCV_TRY(run_gemm(q, dtype, s));
    }
    KvSrc kvs;
    if (bt->kv_cache) {
      // this block's cache: the prefix keys of earlier calls, then the new rows' keys appended
      kvs.kv = static_cast<const uint8_t*>(bt->kv_cache) + (size_t)i * bt->kv_layer_rows * 2048 * es;
      kvs.rows = bt->kv_layer_rows;
      kvs.pos0 = bt->doc_pos0;
      kvs.kv_base = bt->doc_kv_base;
      const int grid = (int)std::min<long>((N + 7) / 8, 16L * num_sms());
      FCV_LAUNCH("kv_append_kernel", kv_append_kernel<T>, dim3(grid), dim3(256), 0, s, static_cast<const T*>(ws.qkv),
                 bt->doc_ids, bt->positions, bt->doc_kv_base, (long)N, bt->kv_layer_rows,
                 static_cast<T*>(const_cast<void*>(kvs.kv)));
    }
    {
      ProfScope ps(FCV_CAT_ATTENTION, s);
      FCV_TRY(run_attention(ws.qkv, dtype, bt->cu_seqlens, bt->chunk, bt->attn_tiles, bt->n_attn_tiles,
                            ws.attn, N, s, bt->n_attn_tiles_dev, bt->attn_sched, bt->attn_sched_ctas, kvs));
    }
    GemmCall o{};
    o.A = ws.attn; o.lda = 1024; o.a_rows = N; o.M = N; o.N = 1024; o.K = 1024;
    o.W = static_cast<const uint8_t*>(w->o_w) + (size_t)i * 1024 * 1024 * es;
    o.epi = make_epi(EPI_GATE_RES, N, 1024, ws.h, 1024, w->o_b + (long)i * 1024);
    o.epi.aux = bt->doc_ids;
    o.epi.gate = mi + 2048;
    o.epi.gate_stride = mstride;
    {
      ProfScope ps(FCV_CAT_GEMM_OUT, s);
      FCV_TRY(run_gemm(o, dtype, s));
    }
    {
      ProfScope ps(FCV_CAT_LN, s);
      FCV_TRY(run_ln(ws.h, FCV_DTYPE_F32, mi + 3072, mi + 4096, bt->doc_ids, mstride, N, ws.norm, dtype, s));
    }
    GemmCall f1{};
    f1.A = ws.norm; f1.lda = 1024; f1.a_rows = N; f1.M = N; f1.N = 2048; f1.K = 1024;
    f1.W = static_cast<const uint8_t*>(w->ff1_w) + (size_t)i * 2048 * 1024 * es;
    f1.epi = make_epi(EPI_GELU, N, 2048, ws.mid, 2048, w->ff1_b + (long)i * 2048);
    {
      ProfScope ps(FCV_CAT_GEMM_FF1, s);
      FCV_TRY(run_gemm(f1, dtype, s));
    }
    GemmCall f2{};
    f2.A = ws.mid; f2.lda = 2048; f2.a_rows = N; f2.M = N; f2.N = 1024; f2.K = 2048;
    f2.W = static_cast<const uint8_t*>(w->ff2_w) + (size_t)i * 1024 * 2048 * es;
    f2.epi = make_epi(EPI_GATE_RES, N, 1024, ws.h, 1024, w->ff2_b + (long)i * 1024);
    f2.epi.aux = bt->doc_ids;
    f2.epi.gate = mi + 5120;
    f2.epi.gate_stride = mstride;
    {
      ProfScope ps(FCV_CAT_GEMM_FF2, s);
      FCV_TRY(run_gemm(f2, dtype, s));
    }
  }

  // 4. final AdaLN (chunk order scale, shift: modules.py:260-265), proj_out, unpack
  const float* mf = mods + (long)depth * 6144;
  ProfScope ps_out(FCV_CAT_OUTPUT, s);
  FCV_TRY(run_ln(ws.h, FCV_DTYPE_F32, mf + 1024, mf + 0, bt->doc_ids, mstride, N, ws.norm, dtype, s));
  if (bt->packed) {
    // packed output rows (N, 80): a plain row-major store, nothing to unpack or zero
    GemmCall po{};
    po.A = ws.norm; po.lda = 1024; po.a_rows = N; po.M = N; po.N = 80; po.K = 1024; po.W = w->out_w;
    po.epi = make_epi(bt->out_f32 ? EPI_F32 : EPI_BIAS, N, 80, bt->out, 80, w->out_b);
    FCV_TRY(run_gemm(po, dtype, s));
    return FCV_OK;
  }
  FCV_TRY(zero_pad());
  GemmCall po{};
  po.A = ws.norm; po.lda = 1024; po.a_rows = N; po.M = N; po.N = 80; po.K = 1024; po.W = w->out_w;
  po.epi = make_epi(EPI_UNPACK, N, 80, bt->out, 0, w->out_b);
  po.epi.aux = bt->doc_ids;
  po.epi.aux2 = bt->positions;
  po.epi.T = bt->T;
  po.epi.out_f32 = bt->out_f32 ? 1 : 0;
  FCV_TRY(run_gemm(po, dtype, s));
  return FCV_OK;
}

}  // namespace

// ====================================================================== allocation-free entry point
// Scratch of fcv_time_embed_noalloc: FCV_NOALLOC_MAX_B rows of the sinusoid
// (256) plus the hidden layer (1024), sized for float32.  Host code must not
// use this name as a device address; it looks the address up per device.
static __device__ __align__(256) float g_noalloc_time_scratch[FCV_NOALLOC_MAX_B * 1280];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {nullptr};

// Device address of g_noalloc_time_scratch on the current device (looked up
// once per device, with that device current).
int noalloc_scratch(void** out) {
  int dev = -1;
  FCV_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(FCV_EUNSUPPORTED, "fcv_time_embed_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_time_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(FCV_ECUDA, "fcv_time_embed_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return FCV_OK;
}
}  // namespace

// ====================================================================== C ABI

extern "C" {

int fcv_version(void) { return 1; }

const char* fcv_last_error(void) { return t_last_error.c_str(); }

int fcv_device_error(int* code, void* stream) {
  if (!code) return fail(FCV_EINVAL, "code is null");
  FCV_CUDA(cudaStreamSynchronize(as_stream(stream)));
  int v = 0;
  FCV_CUDA(cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)));
  const int zero = 0;
  FCV_CUDA(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)));
  *code = v;
  return FCV_OK;
}

// Self-test of the bounded waits every pipelined kernel uses: thread 0 waits on an
// mbarrier that nothing completes and gives up after limit_ns, recording code 901
// and raising the CTA's abort flag; thread 32 waits on the same barrier with four
// times the limit and leaves when it sees the flag.  observed[i] = 1 if waiter i's
// wait succeeded (never expected), 0 if it returned false.
__global__ void __launch_bounds__(64) wait_expiry_kernel(unsigned long long limit_ns, int* observed) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0)
    observed[0] = mbar_wait(smem_u32(&bar), 0, 901, &abort_flag, limit_ns) ? 1 : 0;
  else if (threadIdx.x == 32)
    observed[1] = mbar_wait(smem_u32(&bar), 0, 902, &abort_flag, 4 * limit_ns) ? 1 : 0;
}

int fcv_selftest_wait_expiry(unsigned long long limit_ns, int32_t* observed, void* stream) {
  if (!observed || limit_ns == 0 || limit_ns > kWaitLimitNs)
    return fail(FCV_EINVAL, "fcv_selftest_wait_expiry: observed must be a device int[2], 0 < limit_ns <= %llu",
                kWaitLimitNs);
  FCV_LAUNCH("wait_expiry_kernel", wait_expiry_kernel, dim3(1), dim3(64), 0, as_stream(stream), limit_ns, observed);
  return FCV_OK;
}

int fcv_mask_lengths(const void* mask, int dtype, int B, int T, int32_t* lengths, void* stream) {
  if (!mask || !lengths || B < 0 || T < 0) return fail(FCV_EINVAL, "fcv_mask_lengths: bad arguments");
  if (!valid_dtype(dtype)) return fail(FCV_EINVAL, "fcv_mask_lengths: bad dtype");
  if (B == 0) return FCV_OK;
  if (dtype == FCV_DTYPE_BF16)
    FCV_LAUNCH("mask_lengths_kernel", mask_lengths_kernel<bf16>, dim3(B), dim3(256), 0, as_stream(stream), static_cast<const bf16*>(mask), T, lengths);
  else
    FCV_LAUNCH("mask_lengths_kernel", mask_lengths_kernel<float>, dim3(B), dim3(256), 0, as_stream(stream), static_cast<const float*>(mask), T, lengths);
  return FCV_OK;
}

int fcv_pack_layout(const int32_t* lengths, int B, int T, int max_rows, int64_t* gather, int32_t* doc_ids,
                    int32_t* positions, int32_t* cu_seqlens, int32_t* gap_rows, void* stream) {
  if (!lengths || !doc_ids || !positions || !cu_seqlens || B < 1 || T < 0 || max_rows < 0)
    return fail(FCV_EINVAL, "fcv_pack_layout: bad arguments");
  cudaStream_t s = as_stream(stream);
  FCV_LAUNCH("lengths_scan_kernel", lengths_scan_kernel, dim3(1), dim3(1024), 0, s, lengths, B, cu_seqlens);
  const long work = std::max<long>((long)max_rows + 30L * (B + 1), 1);
  const int grid = (int)std::min<long>((work + 255) / 256, 8L * num_sms());
  FCV_LAUNCH("layout_fill_kernel", layout_fill_kernel, dim3(grid), dim3(256), 0, s, cu_seqlens, B, T, max_rows, gather, doc_ids, positions, gap_rows);
  return FCV_OK;
}

int fcv_unpack_output(const void* packed, int dtype, const int32_t* cu_seqlens, int B, int T, int N, void* out,
                      void* stream) {
  (void)N;
  if (!packed || !cu_seqlens || !out || B < 0 || T < 0) return fail(FCV_EINVAL, "fcv_unpack_output: bad arguments");
  if (!valid_dtype(dtype)) return fail(FCV_EINVAL, "fcv_unpack_output: bad dtype");
  const long total = (long)B * 80 * T;
  if (total == 0) return FCV_OK;
  const int grid = (int)std::min<long>((total + 255) / 256, 4096);
  if (dtype == FCV_DTYPE_BF16)
    FCV_LAUNCH("unpack_kernel", unpack_kernel<bf16>, dim3(grid), dim3(256), 0, as_stream(stream), static_cast<const bf16*>(packed), cu_seqlens, B, T,
                                                            static_cast<bf16*>(out));
  else
    FCV_LAUNCH("unpack_kernel", unpack_kernel<float>, dim3(grid), dim3(256), 0, as_stream(stream), static_cast<const float*>(packed), cu_seqlens, B, T,
                                                             static_cast<float*>(out));
  return FCV_OK;
}

int fcv_ln_modulate(const void* h, int h_dtype, const float* shift, const float* scale, const int32_t* doc_ids,
                    long mod_stride, int N, void* out, int out_dtype, void* stream) {
  if (!h || !shift || !scale || !doc_ids || !out || N < 0) return fail(FCV_EINVAL, "fcv_ln_modulate: bad arguments");
  if (!valid_dtype(h_dtype) || !valid_dtype(out_dtype)) return fail(FCV_EINVAL, "fcv_ln_modulate: bad dtype");
  if ((mod_stride & 3) || (reinterpret_cast<uintptr_t>(shift) & 15) || (reinterpret_cast<uintptr_t>(scale) & 15))
    return fail(FCV_EINVAL, "fcv_ln_modulate: modulation rows must be 16-byte aligned");
  return run_ln(h, h_dtype, shift, scale, doc_ids, mod_stride, N, out, out_dtype, as_stream(stream));
}

int fcv_gate_res_ln_modulate(const void* h, const float* gate, const void* r, const float* shift, const float* scale,
                             const int32_t* doc_ids, long mod_stride, int N, void* h_out, void* norm, int dtype,
                             void* stream) {
  if (!h || !gate || !r || !shift || !scale || !doc_ids || !h_out || !norm || N < 0)
    return fail(FCV_EINVAL, "fcv_gate_res_ln_modulate: bad arguments");
  if (!valid_dtype(dtype)) return fail(FCV_EINVAL, "fcv_gate_res_ln_modulate: bad dtype");
  if ((mod_stride & 3) || (reinterpret_cast<uintptr_t>(shift) & 15) || (reinterpret_cast<uintptr_t>(scale) & 15))
    return fail(FCV_EINVAL, "fcv_gate_res_ln_modulate: modulation rows must be 16-byte aligned");
  if (N == 0) return FCV_OK;
  cudaStream_t s = as_stream(stream);
  if (dtype == FCV_DTYPE_BF16)
    FCV_LAUNCH("gate_res_ln_modulate_kernel", gate_res_ln_modulate_kernel<bf16>, dim3((N + 7) / 8), dim3(256), 0, s, 
        static_cast<const bf16*>(h), gate, static_cast<const bf16*>(r), shift, scale, doc_ids, mod_stride, N,
        static_cast<bf16*>(h_out), static_cast<bf16*>(norm));
  else
    FCV_LAUNCH("gate_res_ln_modulate_kernel", gate_res_ln_modulate_kernel<float>, dim3((N + 7) / 8), dim3(256), 0, s, 
        static_cast<const float*>(h), gate, static_cast<const float*>(r), shift, scale, doc_ids, mod_stride, N,
        static_cast<float*>(h_out), static_cast<float*>(norm));
  return FCV_OK;
}

int fcv_gemm(const void* A, const void* W, const float* bias, int M, int Nout, int K, int dtype, int epi, void* C,
             const int32_t* aux_i32, const float* gate, long gate_stride, const float* rope_cos,
             const float* rope_sin, void* stream) {
  if (!A || !W || !C || M < 0 || Nout <= 0 || K <= 0) return fail(FCV_EINVAL, "fcv_gemm: bad arguments");
  if (!valid_dtype(dtype)) return fail(FCV_EINVAL, "fcv_gemm: bad dtype");
  int internal;
  switch (epi) {
    case FCV_EPI_BIAS: internal = EPI_BIAS; break;
    case FCV_EPI_BIAS_GELU: internal = EPI_GELU; break;
    case FCV_EPI_BIAS_ROPE_QKV:
      if (!aux_i32 || !rope_cos || !rope_sin) return fail(FCV_EINVAL, "fcv_gemm: RoPE needs positions and tables");
      if (Nout != 3072) return fail(FCV_EINVAL, "fcv_gemm: RoPE epilogue expects Nout = 3072");
      if ((reinterpret_cast<uintptr_t>(rope_cos) & 15) || (reinterpret_cast<uintptr_t>(rope_sin) & 15))
        return fail(FCV_EINVAL, "fcv_gemm: RoPE tables must be 16-byte aligned");
      internal = EPI_ROPE;
      break;
    case FCV_EPI_BIAS_GATE_RES:
      if (!aux_i32 || !gate) return fail(FCV_EINVAL, "fcv_gemm: gated residual needs doc_ids and gate");
      if ((gate_stride & 3) || (reinterpret_cast<uintptr_t>(gate) & 15) || (Nout & 3))
        return fail(FCV_EINVAL, "fcv_gemm: gate rows must be 16-byte aligned");
      internal = EPI_GATE_RES;
      break;
    case FCV_EPI_BIAS_F32: internal = EPI_F32; break;
    default: return fail(FCV_EINVAL, "fcv_gemm: unknown epilogue %d", epi);
  }
  const bool f32_out = internal == EPI_GATE_RES || internal == EPI_F32;
  const size_t out_es = f32_out ? 4 : dsize(dtype);
  if (((size_t)Nout * out_es) % 16 != 0 || (reinterpret_cast<uintptr_t>(C) & 15))
    return fail(FCV_EINVAL, "fcv_gemm: output rows must be 16-byte aligned");
  GemmCall g{};
  g.A = A; g.lda = K; g.a_rows = M; g.W = W; g.M = M; g.N = Nout; g.K = K;
  g.epi = make_epi(internal, M, Nout, C, Nout, bias);
  g.epi.aux = aux_i32;
  g.epi.gate = gate;
  g.epi.gate_stride = gate_stride;
  g.epi.rope_cos = rope_cos;
  g.epi.rope_sin = rope_sin;
  return run_gemm(g, dtype, as_stream(stream));
}

int fcv_attention(const void* qkv, int dtype, const int32_t* cu_seqlens, int B, int N, int max_len, int chunk,
                  const int32_t* tiles, int n_tiles, const int32_t* sched, int sched_ctas, void* out, void* stream) {
  (void)B;
  (void)max_len;
  if (!qkv || !cu_seqlens || !out || (n_tiles > 0 && !tiles) || chunk < 0 || N < 0)
    return fail(FCV_EINVAL, "fcv_attention: bad arguments");
  if (!valid_dtype(dtype)) return fail(FCV_EINVAL, "fcv_attention: bad dtype");
  if (N == 0) return FCV_OK;
  return run_attention(qkv, dtype, cu_seqlens, chunk, tiles, n_tiles, out, N, as_stream(stream), nullptr, sched,
                       sched_ctas);
}

int fcv_attn_tiles(const int32_t* lengths_host, int B, int chunk, int32_t* tiles, int cap) {
  if (!lengths_host || !tiles || B < 0 || cap < 0 || chunk < 0) return fail(FCV_EINVAL, "fcv_attn_tiles: bad arguments");
  struct Item {
    long cost;
    int doc, q0;
  };
  std::vector<Item> items;
  for (int d = 0; d < B; ++d) {
    const int L = lengths_host[d];
    if (L < 0) return fail(FCV_EINVAL, "fcv_attn_tiles: negative length");
    for (int q0 = 0; q0 < L; q0 += kAttnQTile) {
      const int rows = std::min(kAttnQTile, L - q0);
      const int q_last = q0 + rows - 1;
      const int kv = chunk > 0 ? std::min(L, (q_last / chunk + 1) * chunk) : L;
      items.push_back({(long)rows * kv, d, q0});
    }
  }
  if ((int)items.size() > cap) return fail(FCV_EINVAL, "fcv_attn_tiles: capacity %d < %zu tiles", cap, items.size());
  std::stable_sort(items.begin(), items.end(), [](const Item& a, const Item& b) { return a.cost > b.cost; });
  for (size_t i = 0; i < items.size(); ++i) {
    tiles[2 * i] = items[i].doc;
    tiles[2 * i + 1] = items[i].q0;
  }
  return (int)items.size();
}

int fcv_attn_ctas(int n_tiles) {
  if (n_tiles < 0) return fail(FCV_EINVAL, "fcv_attn_ctas: negative tile count");
  return std::max(1, std::min(n_tiles * FCV_HEADS, num_sms()));
}

int fcv_attn_schedule(const int32_t* lengths_host, int B, int chunk, const int32_t* tiles, int n_tiles, int n_ctas,
                      int32_t* sched, int cap) {
  if (!lengths_host || (n_tiles > 0 && !tiles) || !sched || B < 0 || chunk < 0 || n_tiles < 0 || n_ctas < 1)
    return fail(FCV_EINVAL, "fcv_attn_schedule: bad arguments");
  const long items = (long)n_tiles * FCV_HEADS;
  const long need = n_ctas + 1 + items;
  if (need > cap) return fail(FCV_EINVAL, "fcv_attn_schedule: capacity %d < %ld", cap, need);
  // item cost: the S and P.V tiles (128 rows x kFaKv keys) of its query tiles plus
  // one for the per-item work (Q load, output)
  std::vector<std::pair<long, int>> order;  // (cost, item), most expensive first
  order.reserve(items);
  auto key_tiles = [&](int L, int q_last) {
    const int kv = chunk > 0 ? std::min(L, (q_last / chunk + 1) * chunk) : L;
    return (long)((kv + kFaKv - 1) / kFaKv);
  };
  for (int t = 0; t < n_tiles; ++t) {
    const int d = tiles[2 * t], q0 = tiles[2 * t + 1];
    if (d < 0 || d >= B) return fail(FCV_EINVAL, "fcv_attn_schedule: tile %d names document %d", t, d);
    const int L = lengths_host[d];
    long cost = 1;
    for (int u = 0; u < kFaTiles && q0 + kFaRows * u < L; ++u)
      cost += key_tiles(L, std::min(q0 + kFaRows * (u + 1), L) - 1);
    for (int h = 0; h < FCV_HEADS; ++h) order.push_back({cost, t * FCV_HEADS + h});
  }
  std::stable_sort(order.begin(), order.end(), [](const auto& a, const auto& b) { return a.first > b.first; });
  // longest processing time first: each item to the least loaded CTA
  std::vector<std::vector<int>> per(n_ctas);
  std::vector<std::pair<long, int>> heap;  // (load, cta), min-heap
  heap.reserve(n_ctas);
  for (int c = 0; c < n_ctas; ++c) heap.push_back({0, c});
  auto cmp = [](const auto& a, const auto& b) { return a.first != b.first ? a.first > b.first : a.second > b.second; };
  std::make_heap(heap.begin(), heap.end(), cmp);
  for (const auto& it : order) {
    std::pop_heap(heap.begin(), heap.end(), cmp);
    auto& slot = heap.back();
    per[slot.second].push_back(it.second);
    slot.first += it.first;
    std::push_heap(heap.begin(), heap.end(), cmp);
  }
  int32_t* off = sched;
  int32_t* list = sched + n_ctas + 1;
  long k = 0;
  for (int c = 0; c < n_ctas; ++c) {
    off[c] = (int32_t)k;
    for (int v : per[c]) list[k++] = v;
  }
  off[n_ctas] = (int32_t)k;
  return (int)need;
}

int fcv_time_embed(const fcv_dit_weights* w, const void* t, int B, float* temb, void* silu_act, void* stream) {
  if (!w || !t || !temb || !silu_act || B < 0) return fail(FCV_EINVAL, "fcv_time_embed: bad arguments");
  if (!valid_dtype(w->dtype)) return fail(FCV_EINVAL, "fcv_time_embed: bad dtype");
  if (B == 0) return FCV_OK;
  cudaStream_t s = as_stream(stream);
  // silu_act holds (B, 1024) outputs followed by (B, 256) + (B, 1024) scratch rows
  uint8_t* base = static_cast<uint8_t*>(silu_act);
  const size_t es = dsize(w->dtype);
  void* tsin = base + (size_t)B * 1024 * es;
  void* th1 = base + (size_t)B * 1280 * es;
  if (w->dtype == FCV_DTYPE_BF16) return run_time_embed<bf16>(w, t, B, tsin, th1, temb, silu_act, s);
  return run_time_embed<float>(w, t, B, tsin, th1, temb, silu_act, s);
}

int fcv_time_embed_noalloc(const fcv_dit_weights* w, const void* t, int B, float* temb, void* silu_act,
                           void* stream) {
  if (!w || !t || !temb || !silu_act || B < 0) return fail(FCV_EINVAL, "fcv_time_embed_noalloc: bad arguments");
  if (!valid_dtype(w->dtype)) return fail(FCV_EINVAL, "fcv_time_embed_noalloc: bad dtype");
  if (B > FCV_NOALLOC_MAX_B)
    return fail(FCV_EINVAL, "fcv_time_embed_noalloc: B=%d exceeds the static scratch limit of %d sequences", B,
                FCV_NOALLOC_MAX_B);
  if (B == 0) return FCV_OK;
  void* scratch = nullptr;
  FCV_TRY(noalloc_scratch(&scratch));
  cudaStream_t s = as_stream(stream);
  uint8_t* base = static_cast<uint8_t*>(scratch);
  void* tsin = base;                                            // (B, 256) sinusoid
  void* th1 = base + (size_t)B * 256 * dsize(w->dtype);         // (B, 1024) hidden layer
  if (w->dtype == FCV_DTYPE_BF16) return run_time_embed<bf16>(w, t, B, tsin, th1, temb, silu_act, s);
  return run_time_embed<float>(w, t, B, tsin, th1, temb, silu_act, s);
}

int fcv_cfg_euler(float* x, const void* d, int d_dtype, int R, int T, float dt, float cfg_rate, void* x_next,
                  int x_next_dtype, void* stream) {
  if (!x || !d || R < 0 || T < 0) return fail(FCV_EINVAL, "fcv_cfg_euler: bad arguments");
  if (!valid_dtype(d_dtype) || !valid_dtype(x_next_dtype)) return fail(FCV_EINVAL, "fcv_cfg_euler: bad dtype");
  const long per = 80L * T;
  const long total = (long)R * per;
  if (total == 0) return FCV_OK;
  const int grid = (int)std::min<long>((total + 255) / 256, 8L * num_sms());
  cudaStream_t s = as_stream(stream);
  const bool db = d_dtype == FCV_DTYPE_BF16, nb = x_next_dtype == FCV_DTYPE_BF16;
  if (db && nb)
    FCV_LAUNCH("cfg_euler_kernel", cfg_euler_kernel<bf16, bf16>, dim3(grid), dim3(256), 0, s, x, static_cast<const bf16*>(d), R, per, dt, cfg_rate,
                                                      static_cast<bf16*>(x_next));
  else if (db)
    FCV_LAUNCH("cfg_euler_kernel", cfg_euler_kernel<bf16, float>, dim3(grid), dim3(256), 0, s, x, static_cast<const bf16*>(d), R, per, dt, cfg_rate,
                                                       static_cast<float*>(x_next));
  else if (nb)
    FCV_LAUNCH("cfg_euler_kernel", cfg_euler_kernel<float, bf16>, dim3(grid), dim3(256), 0, s, x, static_cast<const float*>(d), R, per, dt, cfg_rate,
                                                       static_cast<bf16*>(x_next));
  else
    FCV_LAUNCH("cfg_euler_kernel", cfg_euler_kernel<float, float>, dim3(grid), dim3(256), 0, s, x, static_cast<const float*>(d), R, per, dt, cfg_rate,
                                                        static_cast<float*>(x_next));
  return FCV_OK;
}

int fcv_profile_enable(int on) {
  std::lock_guard<std::mutex> lk(g_prof_mu);
  if (on && g_prof.pool.empty()) {
    g_prof.pool.resize(16384);
    for (auto& e : g_prof.pool) FCV_CUDA(cudaEventCreate(&e));
  }
  g_prof.on = on != 0;
  return FCV_OK;
}

int fcv_profile_collect(float* ms, int* launches, int n_categories) {
  if (!ms || !launches || n_categories < 0) return fail(FCV_EINVAL, "fcv_profile_collect: bad arguments");
  std::lock_guard<std::mutex> lk(g_prof_mu);
  for (int c = 0; c < n_categories; ++c) {
    ms[c] = 0.f;
    launches[c] = 0;
  }
  for (auto& m : g_prof.marks) {
    FCV_CUDA(cudaEventSynchronize(m.second.second));
    float t = 0.f;
    FCV_CUDA(cudaEventElapsedTime(&t, m.second.first, m.second.second));
    if (m.first >= 0 && m.first < n_categories) {
      ms[m.first] += t;
      launches[m.first] += 1;
    }
  }
  g_prof.marks.clear();
  g_prof.next = 0;
  g_prof.open_ev = nullptr;
  return FCV_OK;
}

long fcv_launch_count(void) { return g_launches.load(); }

size_t fcv_dit_workspace_bytes(int N, int B, int depth, int dtype) {
  if (N < 0 || B < 0 || depth < 0 || !valid_dtype(dtype)) return 0;
  return carve(nullptr, N, B, depth, dtype).total;
}

int fcv_dit_forward(const fcv_dit_weights* w, const fcv_dit_batch* bt, void* workspace, size_t workspace_bytes,
                    void* stream) {
  if (!w || !bt || !workspace) return fail(FCV_EINVAL, "fcv_dit_forward: null argument");
  if (!valid_dtype(w->dtype)) return fail(FCV_EINVAL, "fcv_dit_forward: bad dtype");
  if (w->depth < 1) return fail(FCV_EINVAL, "fcv_dit_forward: depth must be >= 1");
  if (bt->B < 1 || bt->N < 0 || bt->chunk < 0 || (!bt->packed && (bt->T < 1 || bt->N > (long)bt->B * bt->T)))
    return fail(FCV_EINVAL, "fcv_dit_forward: bad batch geometry B=%d T=%d N=%d", bt->B, bt->T, bt->N);
  if (bt->kv_cache || bt->doc_pos0 || bt->conv_ctx) {
    // streaming prefix reuse: every piece of the cached state is needed, on packed rows
    if (!bt->kv_cache || !bt->doc_pos0 || !bt->doc_kv_base || !bt->conv_ctx || !bt->packed || bt->kv_layer_rows < 1)
      return fail(FCV_EINVAL, "fcv_dit_forward: a cached prefix needs packed rows, kv_cache, kv_layer_rows, "
                              "doc_pos0, doc_kv_base and conv_ctx");
    if (bt->conv_ctx_out && (!bt->ctx_row0 || bt->conv_ctx_out == bt->conv_ctx))
      return fail(FCV_EINVAL, "fcv_dit_forward: conv_ctx_out needs ctx_row0 and a buffer other than conv_ctx");
    if (reinterpret_cast<uintptr_t>(bt->kv_cache) & 15)
      return fail(FCV_EINVAL, "fcv_dit_forward: kv_cache must be 16-byte aligned");
  }
  if (bt->packed) {
    const void* rows[5] = {bt->x, bt->mu, bt->cond, bt->spks, bt->out};
    for (const void* r : rows)
      if (reinterpret_cast<uintptr_t>(r) & 15)
        return fail(FCV_EINVAL, "fcv_dit_forward: packed rows and spks must be 16-byte aligned");
  }
  if ((reinterpret_cast<uintptr_t>(w->rope_cos) & 15) || (reinterpret_cast<uintptr_t>(w->rope_sin) & 15))
    return fail(FCV_EINVAL, "fcv_dit_forward: RoPE tables must be 16-byte aligned");
  if (bt->max_len > w->rope_max_len)
    return fail(FCV_EUNSUPPORTED, "fcv_dit_forward: document of %d frames exceeds the RoPE table (%d)", bt->max_len,
                w->rope_max_len);
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return fail(FCV_EINVAL, "fcv_dit_forward: workspace must be 256-byte aligned");
  Workspace ws = carve(static_cast<uint8_t*>(workspace), bt->N, bt->B, w->depth, w->dtype);
  if (ws.total > workspace_bytes)
    return fail(FCV_EINVAL, "fcv_dit_forward: workspace of %zu bytes < %zu needed", workspace_bytes, ws.total);
  cudaStream_t s = as_stream(stream);
  if (w->dtype == FCV_DTYPE_BF16) return forward_impl<bf16>(w, bt, ws, s);
  return forward_impl<float>(w, bt, ws, s);
}


int fcv_dit_modulations(const fcv_dit_weights* w, const void* t, float* mods, void* workspace, size_t workspace_bytes,
                        void* stream) {
  if (!w || !t || !mods || !workspace) return fail(FCV_EINVAL, "fcv_dit_modulations: null argument");
  if (!valid_dtype(w->dtype) || w->depth < 1) return fail(FCV_EINVAL, "fcv_dit_modulations: bad weights");
  if (reinterpret_cast<uintptr_t>(workspace) & 255)
    return fail(FCV_EINVAL, "fcv_dit_modulations: workspace must be 256-byte aligned");
  Workspace ws = carve(static_cast<uint8_t*>(workspace), 0, 1, w->depth, w->dtype);
  if (ws.total > workspace_bytes)
    return fail(FCV_EINVAL, "fcv_dit_modulations: workspace of %zu bytes < %zu needed", workspace_bytes, ws.total);
  cudaStream_t s = as_stream(stream);
  const long MS = (long)w->depth * 6144 + 2048;
  if (w->dtype == FCV_DTYPE_BF16)
    FCV_TRY(run_time_embed<bf16>(w, t, 1, ws.tsin, ws.th1, ws.temb, ws.silu, s));
  else
    FCV_TRY(run_time_embed<float>(w, t, 1, ws.tsin, ws.th1, ws.temb, ws.silu, s));
  GemmCall g{};
  g.A = ws.silu; g.lda = 1024; g.a_rows = 1; g.W = w->ada_w; g.M = 1; g.N = (int)MS; g.K = 1024;
  g.epi = make_epi(EPI_F32, 1, (int)MS, mods, MS, w->ada_b);
  return run_gemm(g, w->dtype, s);
}

int fcv_offset_positions(int32_t* positions, const int32_t* doc_ids, const int32_t* doc_pos0, int N, void* stream) {
  if (!positions || !doc_ids || !doc_pos0 || N < 0) return fail(FCV_EINVAL, "fcv_offset_positions: bad arguments");
  if (N == 0) return FCV_OK;
  const int grid = (int)std::min<long>((N + 255) / 256, 8L * num_sms());
  FCV_LAUNCH("offset_positions_kernel", offset_positions_kernel, dim3(grid), dim3(256), 0, as_stream(stream), doc_ids,
             doc_pos0, (long)N, positions);
  return FCV_OK;
}

// ====================================================================== packed flow front end
size_t fcv_flow_workspace_bytes(int n_out_tokens, int dtype) {
  if (n_out_tokens < 0 || !valid_dtype(dtype)) return 0;
  const size_t es = dtype == FCV_DTYPE_BF16 ? 2 : 4;
  auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
  const size_t n = (size_t)n_out_tokens;
  return up(n * kLookK * kFlowIn * es) + up(n * kFlowHid * es) + up(n * kCausalK * kFlowHid * es) +
         up(n * kFlowIn * 4);
}

int fcv_flow_frontend(const fcv_flow_weights* w, const int32_t* tokens, const int32_t* token_cu, const int32_t* out_cu,
                      int B, int n_out_tokens, int max_out_len, int ratio, void* workspace, size_t workspace_bytes,
                      void* mu_rows, void* stream) {
  if (!w || !tokens || !token_cu || !out_cu || !mu_rows || B < 0 || n_out_tokens < 0 || max_out_len < 0 || ratio < 1)
    return fail(FCV_EINVAL, "fcv_flow_frontend: bad arguments");
  if (!valid_dtype(w->dtype) || w->vocab < 1 || !w->embed || !w->conv1_w || !w->conv2_w)
    return fail(FCV_EINVAL, "fcv_flow_frontend: bad weights");
  if (B == 0 || n_out_tokens == 0) return FCV_OK;
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(FCV_EINVAL, "fcv_flow_frontend: workspace must be 256-byte aligned");
  const size_t need = fcv_flow_workspace_bytes(n_out_tokens, w->dtype);
  if (workspace_bytes < need)
    return fail(FCV_EINVAL, "fcv_flow_frontend: workspace of %zu bytes < %zu needed", workspace_bytes, need);
  const int dtype = w->dtype;
  const size_t es = dtype == FCV_DTYPE_BF16 ? 2 : 4;
  auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
  const size_t n = (size_t)n_out_tokens;
  uint8_t* base = static_cast<uint8_t*>(workspace);
  void* a1 = base;
  void* h1 = base + up(n * kLookK * kFlowIn * es);
  void* a2 = static_cast<uint8_t*>(h1) + up(n * kFlowHid * es);
  float* c2 = reinterpret_cast<float*>(static_cast<uint8_t*>(a2) + up(n * kCausalK * kFlowHid * es));
  cudaStream_t s = as_stream(stream);
  const dim3 tgrid((max_out_len + 7) / 8, B);
  const dim3 mgrid(((long)max_out_len * ratio + 7) / 8, B);
  // conv1 (kernel 4, right lookahead) + LeakyReLU, conv2 (kernel 3, causal) as GEMMs on windows
  GemmCall g1{};
  g1.A = a1; g1.lda = kLookK * kFlowIn; g1.a_rows = n_out_tokens; g1.W = w->conv1_w;
  g1.M = n_out_tokens; g1.N = kFlowHid; g1.K = kLookK * kFlowIn;
  g1.epi = make_epi(EPI_LRELU, n_out_tokens, kFlowHid, h1, kFlowHid, w->conv1_b);
  GemmCall g2{};
  g2.A = a2; g2.lda = kCausalK * kFlowHid; g2.a_rows = n_out_tokens; g2.W = w->conv2_w;
  g2.M = n_out_tokens; g2.N = kFlowIn; g2.K = kCausalK * kFlowHid;
  g2.epi = make_epi(EPI_F32, n_out_tokens, kFlowIn, c2, kFlowIn, w->conv2_b);
  if (dtype == FCV_DTYPE_BF16) {
    FCV_LAUNCH("token_window_kernel", token_window_kernel<bf16>, tgrid, dim3(256), 0, s, tokens, token_cu, out_cu,
               static_cast<const bf16*>(w->embed), w->vocab, static_cast<bf16*>(a1));
    FCV_TRY(run_gemm(g1, dtype, s));
    FCV_LAUNCH("causal_window_kernel", causal_window_kernel<bf16>, tgrid, dim3(256), 0, s, out_cu,
               static_cast<const bf16*>(h1), static_cast<bf16*>(a2));
    FCV_TRY(run_gemm(g2, dtype, s));
    FCV_LAUNCH("mu_rows_kernel", mu_rows_kernel<bf16>, mgrid, dim3(256), 0, s, tokens, token_cu, out_cu,
               static_cast<const bf16*>(w->embed), w->vocab, c2, ratio, static_cast<bf16*>(mu_rows));
  } else {
    FCV_LAUNCH("token_window_kernel", token_window_kernel<float>, tgrid, dim3(256), 0, s, tokens, token_cu, out_cu,
               static_cast<const float*>(w->embed), w->vocab, static_cast<float*>(a1));
    FCV_TRY(run_gemm(g1, dtype, s));
    FCV_LAUNCH("causal_window_kernel", causal_window_kernel<float>, tgrid, dim3(256), 0, s, out_cu,
               static_cast<const float*>(h1), static_cast<float*>(a2));
    FCV_TRY(run_gemm(g2, dtype, s));
    FCV_LAUNCH("mu_rows_kernel", mu_rows_kernel<float>, mgrid, dim3(256), 0, s, tokens, token_cu, out_cu,
               static_cast<const float*>(w->embed), w->vocab, c2, ratio, static_cast<float*>(mu_rows));
  }
  return FCV_OK;
}

int fcv_speaker_projection(const void* spk, int spk_dtype, int B, int dim, const void* w, const float* b, int n_out,
                           void* out, int dtype, void* stream) {
  if (!spk || !w || !out || B < 0 || dim < 1 || dim > 4096 || n_out < 1)
    return fail(FCV_EINVAL, "fcv_speaker_projection: bad arguments");
  if (!valid_dtype(spk_dtype) || !valid_dtype(dtype)) return fail(FCV_EINVAL, "fcv_speaker_projection: bad dtype");
  if (B == 0) return FCV_OK;
  cudaStream_t s = as_stream(stream);
  const size_t smem = (size_t)dim * sizeof(float);
  const bool sb = spk_dtype == FCV_DTYPE_BF16, ob = dtype == FCV_DTYPE_BF16;
  if (sb && ob)
    FCV_LAUNCH("speaker_projection_kernel", speaker_projection_kernel<bf16, bf16>, dim3(B), dim3(128), smem, s,
               static_cast<const bf16*>(spk), dim, static_cast<const bf16*>(w), b, n_out, static_cast<bf16*>(out));
  else if (ob)
    FCV_LAUNCH("speaker_projection_kernel", speaker_projection_kernel<float, bf16>, dim3(B), dim3(128), smem, s,
               static_cast<const float*>(spk), dim, static_cast<const bf16*>(w), b, n_out, static_cast<bf16*>(out));
  else if (sb)
    FCV_LAUNCH("speaker_projection_kernel", speaker_projection_kernel<bf16, float>, dim3(B), dim3(128), smem, s,
               static_cast<const bf16*>(spk), dim, static_cast<const float*>(w), b, n_out, static_cast<float*>(out));
  else
    FCV_LAUNCH("speaker_projection_kernel", speaker_projection_kernel<float, float>, dim3(B), dim3(128), smem, s,
               static_cast<const float*>(spk), dim, static_cast<const float*>(w), b, n_out, static_cast<float*>(out));
  return FCV_OK;
}

int fcv_prompt_rows(const void* prompt, const int32_t* prompt_cu, const int32_t* mel_cu, int B, int max_mel_len,
                    void* cond, int dtype, void* stream) {
  if (!prompt_cu || !mel_cu || !cond || B < 0 || max_mel_len < 0) return fail(FCV_EINVAL, "fcv_prompt_rows: bad arguments");
  if (!valid_dtype(dtype)) return fail(FCV_EINVAL, "fcv_prompt_rows: bad dtype");
  if (B == 0 || max_mel_len == 0) return FCV_OK;
  const dim3 grid((max_mel_len + 7) / 8, B);
  cudaStream_t s = as_stream(stream);
  if (dtype == FCV_DTYPE_BF16)
    FCV_LAUNCH("prompt_rows_kernel", prompt_rows_kernel<bf16>, grid, dim3(256), 0, s, static_cast<const bf16*>(prompt),
               prompt_cu, mel_cu, static_cast<bf16*>(cond));
  else
    FCV_LAUNCH("prompt_rows_kernel", prompt_rows_kernel<float>, grid, dim3(256), 0, s, static_cast<const float*>(prompt),
               prompt_cu, mel_cu, static_cast<float*>(cond));
  return FCV_OK;
}

int fcv_pack_rows(const void* src, int src_dtype, long batch_stride, int T, const int32_t* cu, int B, int max_len,
                  void* dst, int dst_dtype, void* stream) {
  if (!src || !cu || !dst || B < 0 || max_len < 0 || T < max_len || batch_stride < 0)
    return fail(FCV_EINVAL, "fcv_pack_rows: bad arguments");
  if (!valid_dtype(src_dtype) || !valid_dtype(dst_dtype)) return fail(FCV_EINVAL, "fcv_pack_rows: bad dtype");
  if (B == 0 || max_len == 0) return FCV_OK;
  const dim3 grid((max_len + 31) / 32, B);
  cudaStream_t s = as_stream(stream);
  const bool sb = src_dtype == FCV_DTYPE_BF16, db = dst_dtype == FCV_DTYPE_BF16;
  if (sb && db)
    FCV_LAUNCH("pack_rows_kernel", pack_rows_kernel<bf16, bf16>, grid, dim3(256), 0, s, static_cast<const bf16*>(src),
               batch_stride, T, cu, static_cast<bf16*>(dst));
  else if (sb)
    FCV_LAUNCH("pack_rows_kernel", pack_rows_kernel<bf16, float>, grid, dim3(256), 0, s, static_cast<const bf16*>(src),
               batch_stride, T, cu, static_cast<float*>(dst));
  else if (db)
    FCV_LAUNCH("pack_rows_kernel", pack_rows_kernel<float, bf16>, grid, dim3(256), 0, s, static_cast<const float*>(src),
               batch_stride, T, cu, static_cast<bf16*>(dst));
  else
    FCV_LAUNCH("pack_rows_kernel", pack_rows_kernel<float, float>, grid, dim3(256), 0, s, static_cast<const float*>(src),
               batch_stride, T, cu, static_cast<float*>(dst));
  return FCV_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- HiFT vocoder
namespace {

struct HiftGeom {
  int cin, cout, k, dil, stride, up, pad;
};

// Geometry of convolution idx (the index order of fcv_hift_weights), from the
// module structure of generator.py:616-676 with builders.py:38-50's sizes.
HiftGeom hift_geom(int idx) {
  static const int ch[3] = {256, 128, 64}, upr[3] = {8, 5, 3}, upk[3] = {16, 11, 7};
  static const int sdk[3] = {30, 6, 1}, sds[3] = {15, 3, 1};
  static const int srk[3] = {7, 7, 11}, rbk[3] = {3, 7, 11}, dil[3] = {1, 3, 5};
  if (idx == 0) return {80, 512, 5, 1, 1, 1, 0};  // look-ahead 4: reads t .. t + 4
  if (idx <= 3) {
    const int i = idx - 1;
    return {i == 0 ? 512 : ch[i - 1], ch[i], upk[i], 1, 1, upr[i], upk[i] - 1};
  }
  if (idx <= 6) {
    const int i = idx - 4;
    return {18, ch[i], sdk[i], 1, sds[i], 1, sds[i] - 1};
  }
  if (idx <= 78) {
    const bool src = idx <= 24;
    const int q = src ? idx - 7 : idx - 25, n = q / 6, s = (q % 6) / 2, second = q % 2;
    const int level = src ? n : n / 3, k = src ? srk[n] : rbk[n % 3];
    const int d = second ? 1 : dil[s];
    return {ch[level], ch[level], k, d, 1, 1, (k - 1) * d};
  }
  return {64, 18, 7, 1, 1, 1, 6};
}

inline int round_up(int v, int m) { return (v + m - 1) / m * m; }

size_t hift_level_floats(const int* rows) {
  return std::max({(size_t)rows[5] * 256, (size_t)rows[6] * 128, (size_t)rows[7] * 64, (size_t)1});
}

template <int N>
int hift_res_conv_tc(const hift::ConvArgs<float>& a, cudaStream_t s) {
  using Cfg = hift::ResConvCfg<N>;
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    FCV_CUDA(cudaFuncSetAttribute(hift::res_conv_tc_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  Cfg::SMEM_BYTES));
    attr_set[dev & 63] = true;
  }
  FCV_LAUNCH("hift_res_conv_tc_kernel", hift::res_conv_tc_kernel<N>, dim3((a.rows_out + 127) / 128),
             dim3(Cfg::THREADS), Cfg::SMEM_BYTES, s, a);
  return FCV_OK;
}

template <typename Tin, typename T>
int hift_conv(const hift::ConvArgs<T>& a, cudaStream_t s) {
  if (a.rows_out == 0) return FCV_OK;
  if constexpr (sizeof(T) == 4 && sizeof(Tin) == 4) {
    if (a.tw_hi && a.tw_lo) {
      // tensor-core path: stride 1, no pre-activation but leaky ReLU, 32-channel K
      // chunks, 16-byte aligned rows
      if (a.stride != 1 || (a.pre != hift::PRE_NONE && a.pre != hift::PRE_LEAKY) || a.cin % 32 ||
          a.cout != a.out_pitch || (a.x_pitch % 4) || (reinterpret_cast<uintptr_t>(a.x) & 15))
        return fail(FCV_EUNSUPPORTED, "fcv_hift_forward: convolution not eligible for the tensor-core path");
      if (a.cout == 64) return hift_res_conv_tc<64>(a, s);
      if (a.cout == 128) return hift_res_conv_tc<128>(a, s);
      if (a.cout == 256) return hift_res_conv_tc<256>(a, s);
      return fail(FCV_EUNSUPPORTED, "fcv_hift_forward: tensor-core convolution needs 64, 128 or 256 channels");
    }
  }
  const dim3 grid((a.rows_out + 127) / 128, a.cout_pad / 64);
  FCV_LAUNCH("hift_conv_kernel", hift::conv_kernel<Tin, T>, grid, dim3(128), 0, s, a);
  return FCV_OK;
}

// Float32 convolution idx from x (rows on in_off / in_lim) to out (rows on out_cu).
hift::ConvArgs<float> hift_args(const fcv_hift_weights* w, int idx, const void* x, const int* in_off, const int* in_lim,
                                const int* out_cu, int n_docs, int rows_out, float* out) {
  const HiftGeom g = hift_geom(idx);
  hift::ConvArgs<float> a{};
  a.x = x;
  a.x_pitch = g.cin;
  a.in_off = in_off;
  a.in_lim = in_lim;
  a.out_cu = out_cu;
  a.n_docs = n_docs;
  a.rows_out = rows_out;
  a.w = w->conv_w[idx];
  a.b = w->conv_b[idx];
  if (idx >= 7 && idx <= 78) {   // residual blocks (the upsampling convolutions stay on SIMT: see hift.cuh)
    a.tw_hi = w->tc_w_hi[idx];
    a.tw_lo = w->tc_w_lo[idx];
  }
  a.cin = g.cin;
  a.cin_pad = round_up(g.cin, 16);
  a.cout = g.cout;
  a.cout_pad = round_up(g.cout, 64);
  a.k = g.k;
  a.dil = g.dil;
  a.stride = g.stride;
  a.up = g.up;
  a.pad_left = g.pad;
  a.vec = g.cin % 16 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  a.out = out;
  a.out_pitch = g.cout;
  return a;
}

}  // namespace

extern "C" {

size_t fcv_hift_workspace_bytes(const int* rows) {
  if (!rows) return 0;
  for (int i = 0; i < FCV_HIFT_LAYOUT_ARRAYS; ++i)
    if (rows[i] < 0) return 0;
  auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
  const size_t lvl = up(hift_level_floats(rows) * 4);
  return 2 * up((size_t)rows[1] * 512 * 8) + up((size_t)rows[1] * 4) + up((size_t)rows[1] * 9 * 4) +
         up((size_t)rows[3] * 4) + up((size_t)rows[4] * 18 * 4) + up((size_t)rows[2] * 512 * 4) + 10 * lvl +
         up((size_t)rows[7] * 18 * 4) + up((size_t)rows[7] * 9 * 8);
}

int fcv_hift_forward(const fcv_hift_weights* w, const fcv_hift_batch* b, void* workspace, size_t workspace_bytes,
                     void* stream) {
  using namespace hift;
  if (!w || !b || b->n_docs < 0) return fail(FCV_EINVAL, "fcv_hift_forward: bad arguments");
  // A batch of non-final chunks that each hold only their look-ahead frames has no
  // audio (rows[8] == 0) but still a source excitation and f0 (rows[3], rows[1]):
  // the f0/source stage runs whenever any of them is non-empty.
  if (b->n_docs == 0 || (b->rows[1] == 0 && b->rows[3] == 0 && b->rows[8] == 0)) return FCV_OK;
  if (!b->mel || !b->layout || (!b->audio && b->rows[8] > 0))
    return fail(FCV_EINVAL, "fcv_hift_forward: null mel, layout or audio");
  for (int i = 0; i < FCV_HIFT_CONVS; ++i)
    if (!w->conv_w[i] || !w->conv_b[i]) return fail(FCV_EINVAL, "fcv_hift_forward: convolution %d has no weights", i);
  for (int i = 0; i < 5; ++i)
    if (!w->f0_w[i] || !w->f0_b[i]) return fail(FCV_EINVAL, "fcv_hift_forward: f0 convolution %d has no weights", i);
  if (!w->f0_cls_w || !w->source_w || !w->noise) return fail(FCV_EINVAL, "fcv_hift_forward: missing weights");
  if (b->max_src < 0 || (long long)b->max_src > w->noise_rows)
    return fail(FCV_EINVAL, "fcv_hift_forward: a document needs %d noise rows, the table holds %lld", b->max_src,
                w->noise_rows);
  const int* rows = b->rows;
  for (int i = 0; i < FCV_HIFT_LAYOUT_ARRAYS; ++i)
    if (rows[i] < 0) return fail(FCV_EINVAL, "fcv_hift_forward: negative row total");
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255))
    return fail(FCV_EINVAL, "fcv_hift_forward: workspace must be 256-byte aligned");
  const size_t need = fcv_hift_workspace_bytes(rows);
  if (workspace_bytes < need)
    return fail(FCV_EINVAL, "fcv_hift_forward: workspace of %zu bytes < %zu needed", workspace_bytes, need);
  const int D = b->n_docs;
  const int* L = b->layout;
  const int *mel_cu = L, *f0_cu = L + (D + 1), *x_cu = L + 2 * (D + 1), *src_cu = L + 3 * (D + 1),
            *stft_cu = L + 4 * (D + 1), *audio_cu = L + 8 * (D + 1);
  const int* lvl_cu[3] = {L + 5 * (D + 1), L + 6 * (D + 1), L + 7 * (D + 1)};
  const int lvl_rows[3] = {rows[5], rows[6], rows[7]};

  auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
  uint8_t* p = static_cast<uint8_t*>(workspace);
  auto take = [&](size_t bytes) {
    void* r = p;
    p += up(bytes);
    return r;
  };
  double* f0a = static_cast<double*>(take((size_t)rows[1] * 512 * 8));
  double* f0b = static_cast<double*>(take((size_t)rows[1] * 512 * 8));
  float* f0 = static_cast<float*>(take((size_t)rows[1] * 4));
  float* sines = static_cast<float*>(take((size_t)rows[1] * 9 * 4));
  float* s_src = static_cast<float*>(take((size_t)rows[3] * 4));
  float* spec_in = static_cast<float*>(take((size_t)rows[4] * 18 * 4));
  float* x0 = static_cast<float*>(take((size_t)rows[2] * 512 * 4));
  const size_t lvl = hift_level_floats(rows) * 4;
  float* xb[2] = {static_cast<float*>(take(lvl)), static_cast<float*>(take(lvl))};
  float* tmp = static_cast<float*>(take(lvl));
  float* y = static_cast<float*>(take(lvl));
  float* xs = static_cast<float*>(take(lvl));
  float* si = static_cast<float*>(take(lvl));
  float* act = static_cast<float*>(take(lvl));   // Snake input of the next convs1 inside a residual block
  float* actx[3] = {static_cast<float*>(take(lvl)), static_cast<float*>(take(lvl)), static_cast<float*>(take(lvl))};
  float* post = static_cast<float*>(take((size_t)rows[7] * 18 * 4));
  float2* spec_out = static_cast<float2*>(take((size_t)rows[7] * 9 * 8));
  cudaStream_t s = as_stream(stream);

  // ---- f0 predictor (float64): condnet 0 (k 4, look-ahead 3) + 4 x (k 3, causal), ELU after each
  for (int i = 0; i < 5; ++i) {
    ConvArgs<double> a{};
    a.x = i == 0 ? static_cast<const void*>(b->mel) : static_cast<const void*>(i % 2 ? f0a : f0b);
    a.x_pitch = i == 0 ? 80 : 512;
    a.in_off = i == 0 ? mel_cu : f0_cu;
    a.in_lim = a.in_off;
    a.out_cu = f0_cu;
    a.n_docs = D;
    a.rows_out = rows[1];
    a.w = w->f0_w[i];
    a.b = w->f0_b[i];
    a.cin = i == 0 ? 80 : 512;
    a.cin_pad = a.cin;
    a.cout = a.cout_pad = 512;
    a.k = i == 0 ? 4 : 3;
    a.dil = a.stride = a.up = 1;
    a.pad_left = i == 0 ? 0 : 2;
    a.epi = EPI_ELU;
    a.out = i % 2 ? f0b : f0a;
    a.out_pitch = 512;
    if (i == 0) FCV_TRY((hift_conv<float, double>(a, s)));
    else FCV_TRY((hift_conv<double, double>(a, s)));
  }
  if (rows[1] > 0) {
    FCV_LAUNCH("hift_f0_head_kernel", f0_head_kernel, dim3((rows[1] + 7) / 8), dim3(256), 0, s, f0a, rows[1], 512,
               w->f0_cls_w, w->f0_cls_b, f0);
    // ---- source excitation and its STFT
    FCV_LAUNCH("hift_source_phase_kernel", source_phase_kernel, dim3(D), dim3(256), 0, s, f0, f0_cu, sines);
  }
  if (rows[3] > 0)
    FCV_LAUNCH("hift_source_kernel", source_kernel, dim3((rows[3] + 255) / 256), dim3(256), 0, s, f0, sines, f0_cu,
               src_cu, D, rows[3], w->noise, w->source_w, w->source_b, s_src);
  if (rows[4] > 0)
    FCV_LAUNCH("hift_stft_kernel", stft_kernel, dim3((rows[4] + 127) / 128), dim3(128), 0, s, s_src, src_cu, stft_cu,
               D, rows[4], spec_in);

  auto copy_source_f0 = [&]() -> int {
    if (b->source && rows[3] > 0)
      FCV_CUDA(cudaMemcpyAsync(b->source, s_src, (size_t)rows[3] * 4, cudaMemcpyDeviceToDevice, s));
    if (b->f0 && rows[1] > 0) FCV_CUDA(cudaMemcpyAsync(b->f0, f0, (size_t)rows[1] * 4, cudaMemcpyDeviceToDevice, s));
    return FCV_OK;
  };
  if (rows[8] == 0) return copy_source_f0();  // no audio frame to decode

  // ---- decode: conv_pre reads the first F0 mel frames of each request (look-ahead 4 of them)
  FCV_TRY((hift_conv<float, float>(hift_args(w, 0, b->mel, mel_cu, f0_cu, x_cu, D, rows[2], x0), s)));
  const float* x_prev = x0;
  const int* prev_cu = x_cu;
  for (int i = 0; i < 3; ++i) {
    float* x = xb[i & 1];
    const int* cu = lvl_cu[i];
    const int n = lvl_rows[i];
    auto ca = [&](int idx, const void* in, const int* in_cu, float* out) {
      return hift_args(w, idx, in, in_cu, in_cu, cu, D, n, out);
    };
    ConvArgs<float> a = hift_args(w, 1 + i, x_prev, prev_cu, prev_cu, cu, D, n, x);
    a.pre = PRE_LEAKY;
    a.slope = 0.1f;
    a.reflect_first = i == 2;
    FCV_TRY((hift_conv<float, float>(a, s)));
    // Every convs1 reads its Snake input (activations1) ready-made: the convolution
    // producing that input stores it from its epilogue (act_out).
    auto add_act = [&](ConvArgs<float>& c, float* dst, int c1) {
      c.act_out[c.n_act] = dst;
      c.act_alpha[c.n_act] = w->snake_alpha[c1];
      c.act_inv[c.n_act] = w->snake_inv[c1];
      ++c.n_act;
    };
    const int src_first = 7 + 6 * i, rb0 = 25 + 6 * (3 * i);
    ConvArgs<float> sd = ca(4 + i, spec_in, stft_cu, si);
    add_act(sd, act, src_first);
    FCV_TRY((hift_conv<float, float>(sd, s)));
    // one residual block: per dilation, conv1 with activations2 in its epilogue, then
    // conv2 + residual storing the next stage's activations1; the last conv2 may fold
    // in the sum that follows (last_epi) and store other blocks' first inputs (acts)
    auto resblock = [&](int first, const float* in, const float* in_act, float* work, int last_epi, float* last_out,
                        const float* acc, bool acts) {
      const float* cur = in;
      for (int st = 0; st < 3; ++st) {
        const int c1 = first + 2 * st;
        ConvArgs<float> a1 = ca(c1, st == 0 ? in_act : act, cu, tmp);
        a1.epi = EPI_SNAKE;
        a1.post_alpha = w->snake2_alpha[c1];
        a1.post_inv = w->snake2_inv[c1];
        FCV_TRY((hift_conv<float, float>(a1, s)));
        ConvArgs<float> a2 = ca(c1 + 1, tmp, cu, work);
        a2.epi = EPI_RES;
        a2.res = cur;
        if (st < 2) add_act(a2, act, c1 + 2);
        if (st == 2 && last_epi != EPI_RES) {
          a2.epi = last_epi;
          a2.acc = acc;
          a2.out = last_out;
        }
        if (st == 2 && acts)
          for (int j = 0; j < 3; ++j) add_act(a2, actx[j], rb0 + 6 * j);
        FCV_TRY((hift_conv<float, float>(a2, s)));
        cur = work;
      }
      return FCV_OK;
    };
    // source branch: si = resblock(si); x = x + si folded into its last conv2, which
    // also stores the three blocks' first Snake inputs
    FCV_TRY(resblock(src_first, si, act, si, EPI_RES_ACC, x, x, true));
    // xs = rb0(x); xs += rb1(x); x = (xs + rb2(x)) / 3
    FCV_TRY(resblock(rb0, x, actx[0], xs, EPI_RES, xs, nullptr, false));
    FCV_TRY(resblock(rb0 + 6, x, actx[1], y, EPI_RES_ACC, xs, xs, false));
    FCV_TRY(resblock(rb0 + 12, x, actx[2], y, EPI_RES_ACC_AVG, x, xs, false));
    x_prev = x;
    prev_cu = cu;
  }
  // ---- conv_post (leaky 0.01 on load), magnitude/phase head, inverse STFT
  ConvArgs<float> ap = hift_args(w, 79, x_prev, prev_cu, prev_cu, prev_cu, D, rows[7], post);
  ap.pre = PRE_LEAKY;
  ap.slope = 0.01f;
  FCV_TRY((hift_conv<float, float>(ap, s)));
  FCV_LAUNCH("hift_spectrum_kernel", spectrum_kernel, dim3((rows[7] * 9 + 255) / 256), dim3(256), 0, s, post, rows[7],
             spec_out);
  FCV_LAUNCH("hift_istft_kernel", istft_kernel, dim3((rows[8] + 255) / 256), dim3(256), 0, s, spec_out, lvl_cu[2],
             audio_cu, D, rows[8], b->audio);
  return copy_source_f0();
}

}  // extern "C"
