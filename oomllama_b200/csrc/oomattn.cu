// Host side of the oomattn C ABI (include/oomattn.h): context lifetime, host
// validation, the paged-cache bookkeeping that mirrors LayerKVCache /
// ModelKVCache (src/oomllama_turbo.rs:26-104), tensor maps, split planning and
// kernel launches.  Everything here is plain host C++ over the CUDA runtime;
// every kernel it launches is this library's own (no cuBLAS or other compute
// library).
#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#include "../../include/oomattn.h"
#include "common.cuh"
#include "decode.cuh"
#include "gemm.cuh"
#include "params.cuh"
#include "prefill.cuh"
#include "q8_linear.cuh"
#include "q8_tc.cuh"
#include "rope_append.cuh"

using namespace oomattn;

namespace {

int split_cap(int kv_dtype) { return kv_dtype == OOMATTN_DTYPE_BF16 ? kMaxSplitsBf16 : kMaxSplits; }
static_assert(kMaxGroup * kMaxSplits <= kDecWarps * kMaxGroup * kMergeStride,
              "the f32 decode merge stages [group][splits] lse values over the per-warp O area");
constexpr unsigned long long kDefaultTimeoutNs = 2000000000ull;  // bounded device waits: 2 s
constexpr int kPfMinKeyChunk = 4;  // key tiles per unit of a key-split prefill, at least

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

}  // namespace

struct oomattn_ctx {
  oomattn_config cfg;
  int device = 0;
  cudaStream_t stream = nullptr;
  std::string err;
  int num_sms = 148;
  int group = 1;
  int max_pages_per_seq = 0;
  int n_pool_pages = 0;  // cfg.n_pages + null page
  size_t esize = 4;
  float scale = 0.f;
  unsigned long long timeout_ns = kDefaultTimeoutNs;
  int test_flags = 0;  // OOMATTN_TEST_* launch flags (tests only)
  // device state
  void* kpool = nullptr;
  void* vpool = nullptr;
  int* d_block_table = nullptr;
  float* d_cos = nullptr;
  float* d_sin = nullptr;
  float* d_part_o = nullptr;
  float* d_part_lse = nullptr;
  unsigned* d_counters = nullptr;
  int* d_status = nullptr;
  CUtensorMap kmap{}, vmap{};
  bool have_maps = false;
  int prefill_regs = 0;  // compiled register count of the prefill kernel
  int kf_q8_regs = 0;    // and of the Q8 tensor-core linear (its register split needs kKfLaunchRegs)
  // host mirrors (authoritative for lengths; updated at enqueue time)
  std::vector<int> h_block_table;  // [max_seqs][max_pages_per_seq]
  std::vector<int> h_len;          // [n_layers][max_seqs]
  std::vector<int> h_pos_off;      // [max_seqs]
  std::vector<float> h_cos, h_sin; // [max_seq_len][64]
  // lazily grown scratch for the layer step
  float* d_scratch = nullptr;
  size_t scratch_bytes = 0;
  // K-F (tensor-core linear): the split / converted operand planes
  uint8_t* d_kf = nullptr;
  size_t kf_bytes = 0;
  // key-split prefill: the chunks' partial O and lse
  uint8_t* d_pf_part = nullptr;
  size_t pf_part_bytes = 0;
  // Q8 linear: activation splits and split-K partials, and per-row-tile
  // arrival counters (zero between launches)
  uint8_t* d_q8_scratch = nullptr;
  size_t q8_scratch_bytes = 0;
  unsigned* d_q8_counters = nullptr;
  int q8_counters_n = 0;
  // decoder-layer step: normalised activations, projections, MLP intermediates
  float* d_layer_scratch = nullptr;
  size_t layer_scratch_bytes = 0;
  // model step: the residual stream between layers and the logits
  float* d_model_scratch = nullptr;
  size_t model_scratch_bytes = 0;
  // argmax: per-(row, chunk) (value, index) partials
  void* d_argmax_part = nullptr;
  size_t argmax_part_bytes = 0;
  // the last decode schedule and the page counts it was planned for (every
  // layer of a step, and every step until a row crosses a page, reuses it)
  std::vector<int> sched_key;
  DecodeSched sched;
  int sched_items = 0;
};

namespace {

int fail(oomattn_ctx* ctx, int code, const char* fmt, ...) {
  if (ctx) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    ctx->err = buf;
  }
  return code;
}

#define CK(call)                                                                                     \
  do {                                                                                               \
    cudaError_t e_ = (call);                                                                         \
    if (e_ != cudaSuccess) return fail(ctx, OOMATTN_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

#define CKLAUNCH()                                                                                          \
  do {                                                                                                      \
    cudaError_t e_ = cudaGetLastError();                                                                    \
    if (e_ != cudaSuccess) return fail(ctx, OOMATTN_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e_)); \
  } while (0)

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// f32 RoPE table exactly as the reference builds it on the host
// (src/oomllama_turbo.rs:753-761): inv_freq = 1 / theta^(2i/d) with f32 powf,
// angle = (f32)pos * inv_freq, cos/sin in f32.
void build_rope_table(float theta, int n_pos, std::vector<float>& c, std::vector<float>& s) {
  const int half = kHeadDim / 2;
  std::vector<float> inv(half);
  for (int i = 0; i < half; ++i) {
    volatile float e = (2.0f * (float)i) / (float)kHeadDim;
    inv[i] = 1.0f / powf(theta, e);
  }
  c.resize((size_t)n_pos * half);
  s.resize((size_t)n_pos * half);
  for (int p = 0; p < n_pos; ++p) {
    const float pos = (float)p;
    for (int i = 0; i < half; ++i) {
      volatile float a = pos * inv[i];
      c[(size_t)p * half + i] = cosf(a);
      s[(size_t)p * half + i] = sinf(a);
    }
  }
}

int encode_pool_map(oomattn_ctx* ctx, void* base, CUtensorMap* map) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(ctx, OOMATTN_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const uint64_t rows = (uint64_t)ctx->cfg.n_layers * ctx->n_pool_pages * ctx->cfg.n_kv_heads * kPageSize;
  cuuint64_t dims[2] = {(cuuint64_t)kHeadDim, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)kHeadDim * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)kPageSize};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ctx, OOMATTN_ERR_CUDA, "cuTensorMapEncodeTiled(pool) failed: %d", (int)r);
  return OOMATTN_OK;
}

int encode_q_map(oomattn_ctx* ctx, const void* q, int n_new, CUtensorMap* map) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(ctx, OOMATTN_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[3] = {(cuuint64_t)kHeadDim, (cuuint64_t)ctx->cfg.n_heads, (cuuint64_t)n_new};
  cuuint64_t strides[2] = {(cuuint64_t)kHeadDim * 2, (cuuint64_t)ctx->cfg.n_heads * kHeadDim * 2};
  cuuint32_t box[3] = {64, 1, 128};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ctx, OOMATTN_ERR_CUDA, "cuTensorMapEncodeTiled(q) failed: %d", (int)r);
  return OOMATTN_OK;
}

// The prefill output [n_new][n_heads][128] (f32 or bf16) as the target of
// the epilogue's TMA stores: boxes of 128 rows x 128 bytes (32 f32 or 64 bf16
// columns) of one head, 128-byte swizzled; rows past n_new are clipped.
int encode_out_map(oomattn_ctx* ctx, void* out, int n_new, bool bf16, CUtensorMap* map) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(ctx, OOMATTN_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const uint64_t es = bf16 ? 2 : 4;
  cuuint64_t dims[3] = {(cuuint64_t)kHeadDim, (cuuint64_t)ctx->cfg.n_heads, (cuuint64_t)n_new};
  cuuint64_t strides[2] = {(cuuint64_t)kHeadDim * es, (cuuint64_t)ctx->cfg.n_heads * kHeadDim * es};
  cuuint32_t box[3] = {(cuuint32_t)(128 / es), 1, 128};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, out, dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ctx, OOMATTN_ERR_CUDA, "cuTensorMapEncodeTiled(out) failed: %d", (int)r);
  return OOMATTN_OK;
}

KVPool make_pool(const oomattn_ctx* ctx) {
  KVPool p;
  p.k = ctx->kpool;
  p.v = ctx->vpool;
  p.block_table = ctx->d_block_table;
  p.max_pages_per_seq = ctx->max_pages_per_seq;
  p.n_pool_pages = ctx->n_pool_pages;
  p.n_kv = ctx->cfg.n_kv_heads;
  p.kv_bf16 = ctx->cfg.kv_dtype == OOMATTN_DTYPE_BF16;
  return p;
}

int check_layer(oomattn_ctx* ctx, int layer) {
  if (layer < 0 || layer >= ctx->cfg.n_layers)
    return fail(ctx, OOMATTN_ERR_OUT_OF_RANGE, "layer %d outside [0, %d)", layer, ctx->cfg.n_layers);
  return OOMATTN_OK;
}

int check_seq(oomattn_ctx* ctx, int seq) {
  if (seq < 0 || seq >= ctx->cfg.max_seqs)
    return fail(ctx, OOMATTN_ERR_OUT_OF_RANGE, "sequence %d outside [0, %d)", seq, ctx->cfg.max_seqs);
  return OOMATTN_OK;
}

// Slots [from, to) of `seq` must sit in assigned pages.
int check_slots(oomattn_ctx* ctx, int seq, int from, int to) {
  if (to > ctx->max_pages_per_seq * kPageSize)
    return fail(ctx, OOMATTN_ERR_OUT_OF_RANGE, "sequence %d: %d slots exceed max_seq_len capacity %d", seq, to,
                ctx->max_pages_per_seq * kPageSize);
  const int null_page = ctx->n_pool_pages - 1;
  for (int lp = from / kPageSize; lp * kPageSize < to; ++lp)
    if (ctx->h_block_table[(size_t)seq * ctx->max_pages_per_seq + lp] == null_page)
      return fail(ctx, OOMATTN_ERR_OUT_OF_RANGE, "sequence %d: logical page %d (slot %d) has no pool page", seq, lp,
                  std::max(from, lp * kPageSize));
  return OOMATTN_OK;
}

int validate_dtype(oomattn_ctx* ctx, int dt, const char* what) {
  if (dt != OOMATTN_DTYPE_F32 && dt != OOMATTN_DTYPE_BF16)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "%s: unknown dtype %d", what, dt);
  return OOMATTN_OK;
}

int ensure_scratch(oomattn_ctx* ctx, size_t bytes) {
  if (bytes <= ctx->scratch_bytes) return OOMATTN_OK;
  if (ctx->d_scratch) {
    cudaStreamSynchronize(ctx->stream);
    cudaFree(ctx->d_scratch);
    ctx->d_scratch = nullptr;
    ctx->scratch_bytes = 0;
  }
  if (cudaMalloc(&ctx->d_scratch, bytes) != cudaSuccess)
    return fail(ctx, OOMATTN_ERR_NO_MEMORY, "scratch allocation of %zu bytes failed", bytes);
  ctx->scratch_bytes = bytes;
  return OOMATTN_OK;
}

// ------------------------------------------------------------------ K-F host side
// A 2D row-major tensor [outer][inner] of 16-bit or f32 elements as a TMA map
// with 128-byte-swizzled boxes [box_outer][box_inner]; reads past the edges
// fill zeros and stores past them are dropped.
int encode_2d(oomattn_ctx* ctx, const void* base, CUtensorMapDataType dt, int es, uint64_t inner, uint64_t outer,
              uint32_t box_inner, uint32_t box_outer, CUtensorMap* map) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(ctx, OOMATTN_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)inner * es};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ctx, OOMATTN_ERR_CUDA, "cuTensorMapEncodeTiled(linear operand) failed: %d", (int)r);
  return OOMATTN_OK;
}

uint8_t* kf_scratch(oomattn_ctx* ctx, size_t bytes, int* rc) {
  *rc = OOMATTN_OK;
  if (bytes > ctx->kf_bytes) {
    if (ctx->d_kf) {
      cudaStreamSynchronize(ctx->stream);
      cudaFree(ctx->d_kf);
      ctx->d_kf = nullptr;
      ctx->kf_bytes = 0;
    }
    if (cudaMalloc(&ctx->d_kf, bytes) != cudaSuccess) {
      *rc = fail(ctx, OOMATTN_ERR_NO_MEMORY, "linear operand scratch of %zu bytes failed", bytes);
      return nullptr;
    }
    ctx->kf_bytes = bytes;
  }
  return ctx->d_kf;
}

size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

// One tensor-core linear launch: out [M][N] = A [M][K] . B [N][K]^T over the
// given 16-bit planes (bf16, or fp16 for Q8 with the promotion operands).
template <bool Q8, int BPLANES>
int kf_launch(oomattn_ctx* ctx, int M, int N, int K, const void* a_hi, const void* a_lo, const void* b_hi,
              const void* b_lo, const float* bias, const float* residual, float* out, const float* scale_t = nullptr,
              const float* min_t = nullptr, const float* xsum = nullptr) {
  const CUtensorMapDataType dt16 = Q8 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap am_hi, am_lo, bm_hi, bm_lo, om, rm;
  int rc = encode_2d(ctx, a_hi, dt16, 2, K, M, kKfBK, kKfBM, &am_hi);
  if (!rc) rc = encode_2d(ctx, a_lo, dt16, 2, K, M, kKfBK, kKfBM, &am_lo);
  if (!rc) rc = encode_2d(ctx, b_hi, dt16, 2, K, N, kKfBK, kKfBN, &bm_hi);
  if (!rc) rc = encode_2d(ctx, BPLANES == 2 ? b_lo : b_hi, dt16, 2, K, N, kKfBK, kKfBN, &bm_lo);
  if (!rc) rc = encode_2d(ctx, out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, M, 32, kKfBM, &om);
  if (!rc) rc = encode_2d(ctx, residual ? residual : out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, M, 32, kKfBM, &rm);
  if (rc) return rc;
  KfArgs a;
  a.M = M;
  a.N = N;
  a.K = K;
  a.m_tiles = (M + kKfBM - 1) / kKfBM;
  a.n_tiles = (N + kKfBN - 1) / kKfBN;
  a.bias = bias;
  a.scale_t = scale_t;
  a.min_t = min_t;
  a.xsum = xsum;
  a.has_residual = residual != nullptr;
  a.status = ctx->d_status;
  a.timeout_ns = ctx->timeout_ns;
  const long long grid = (long long)a.m_tiles * a.n_tiles;
  if (grid >= (1ll << 31)) return fail(ctx, OOMATTN_ERR_OUT_OF_RANGE, "linear of %d x %d too large", M, N);
  kf_gemm_kernel<Q8, BPLANES><<<(unsigned)grid, kKfThreads, kKfSmemBytes, ctx->stream>>>(am_hi, am_lo, bm_hi, bm_lo,
                                                                                         om, rm, a);
  CKLAUNCH();
  return OOMATTN_OK;
}

// One output of an f32 (or bf16-weight) linear: out = x W^T (+ bias) (+ residual).
struct KfJob {
  const void* w;  // [n][k], f32 or bf16
  int w_bf16;
  int n;
  const float* bias;
  const float* residual;  // [m][n] or null (may alias out)
  float* out;             // [m][n]
};

// x [m][k] f32 times several weight matrices of the same width on the tensor
// cores: x is split into bf16 hi/lo planes once, each f32 W into its planes.
int kf_linear_f32(oomattn_ctx* ctx, const float* x, int m, int k, const KfJob* jobs, int n_jobs) {
  if (m <= 0) return OOMATTN_OK;
  if (k % 8 || (reinterpret_cast<uintptr_t>(x) & 15))
    return fail(ctx, OOMATTN_ERR_UNSUPPORTED, "the tensor-core linear needs k %% 8 == 0 and 16-byte aligned x");
  size_t wmax = 0;
  for (int j = 0; j < n_jobs; ++j) {
    const KfJob& jb = jobs[j];
    if (jb.n % 4 || !jb.w || !jb.out || (reinterpret_cast<uintptr_t>(jb.w) & 15) ||
        (reinterpret_cast<uintptr_t>(jb.out) & 15) || (jb.bias && (reinterpret_cast<uintptr_t>(jb.bias) & 15)) ||
        (jb.residual && (reinterpret_cast<uintptr_t>(jb.residual) & 15)))
      return fail(ctx, OOMATTN_ERR_UNSUPPORTED,
                  "the tensor-core linear needs rows %% 4 == 0 and 16-byte aligned weights, bias and outputs");
    if (!jb.w_bf16) wmax = std::max(wmax, (size_t)jb.n * k);
  }
  const size_t xb = align256((size_t)m * k * 2), wb = align256(wmax * 2);
  int rc;
  uint8_t* sc = kf_scratch(ctx, 2 * xb + 2 * wb, &rc);
  if (rc) return rc;
  uint16_t* xh = reinterpret_cast<uint16_t*>(sc);
  uint16_t* xl = reinterpret_cast<uint16_t*>(sc + xb);
  uint16_t* wh = reinterpret_cast<uint16_t*>(sc + 2 * xb);
  uint16_t* wl = reinterpret_cast<uint16_t*>(sc + 2 * xb + wb);
  const size_t xn4 = (size_t)m * k / 4;
  kf_split_bf16_kernel<<<(unsigned)std::min<size_t>((xn4 + 255) / 256, (size_t)ctx->num_sms * 8), 256, 0,
                         ctx->stream>>>(x, xh, xl, xn4);
  CKLAUNCH();
  for (int j = 0; j < n_jobs; ++j) {
    const KfJob& jb = jobs[j];
    if (jb.w_bf16) {
      rc = kf_launch<false, 1>(ctx, m, jb.n, k, xh, xl, jb.w, nullptr, jb.bias, jb.residual, jb.out);
    } else {
      const size_t wn4 = (size_t)jb.n * k / 4;
      kf_split_bf16_kernel<<<(unsigned)std::min<size_t>((wn4 + 255) / 256, (size_t)ctx->num_sms * 8), 256, 0,
                             ctx->stream>>>(static_cast<const float*>(jb.w), wh, wl, wn4);
      CKLAUNCH();
      rc = kf_launch<false, 2>(ctx, m, jb.n, k, xh, xl, wh, wl, jb.bias, jb.residual, jb.out);
    }
    if (rc) return rc;
  }
  return OOMATTN_OK;
}

// f32 GEMV for T <= 16 tokens (f32 weights): y = x W^T (+ bias) (+ residual).
int f32_gemv(oomattn_ctx* ctx, const float* x, const float* w, int T, int n, int k, const float* bias,
             const float* residual, float* y) {
  if (k % 4 || ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) & 15))
    return fail(ctx, OOMATTN_ERR_UNSUPPORTED, "the f32 GEMV needs k %% 4 == 0 and 16-byte aligned x and W");
  const int grid = (int)(((long long)(n + 1) / 2 * 32 + 255) / 256);
#define OOMATTN_GEMV_T(TT) \
  case TT: f32_gemv_kernel<TT><<<grid, 256, 0, ctx->stream>>>(x, w, bias, residual, y, n, k); break;
  switch (T) {
    OOMATTN_GEMV_T(1) OOMATTN_GEMV_T(2) OOMATTN_GEMV_T(3) OOMATTN_GEMV_T(4) OOMATTN_GEMV_T(5) OOMATTN_GEMV_T(6)
    OOMATTN_GEMV_T(7) OOMATTN_GEMV_T(8) OOMATTN_GEMV_T(9) OOMATTN_GEMV_T(10) OOMATTN_GEMV_T(11)
    OOMATTN_GEMV_T(12) OOMATTN_GEMV_T(13) OOMATTN_GEMV_T(14) OOMATTN_GEMV_T(15) OOMATTN_GEMV_T(16)
    default: return fail(ctx, OOMATTN_ERR_INVALID_ARG, "f32 GEMV of %d tokens", T);
  }
#undef OOMATTN_GEMV_T
  CKLAUNCH();
  return OOMATTN_OK;
}

// Fills the SeqBatch of an append over rows [r0, r0+n) and advances the host lengths.
int plan_append(oomattn_ctx* ctx, int layer, int n, const int32_t* seq_ids, int n_new, SeqBatch& sb) {
  sb.n = n;
  for (int z = 0; z < n; ++z) {
    const int seq = seq_ids[z];
    int rc = check_seq(ctx, seq);
    if (rc) return rc;
    for (int w = 0; w < z; ++w)
      if (sb.seq[w] == seq) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "sequence %d appears twice in one append", seq);
    const int len = ctx->h_len[(size_t)layer * ctx->cfg.max_seqs + seq];
    const int pos = ctx->h_pos_off[seq] + len;
    if (pos + n_new > ctx->cfg.max_seq_len)
      return fail(ctx, OOMATTN_ERR_OUT_OF_RANGE, "sequence %d: positions up to %d exceed max_seq_len %d", seq,
                  pos + n_new - 1, ctx->cfg.max_seq_len);
    rc = check_slots(ctx, seq, len, len + n_new);
    if (rc) return rc;
    sb.seq[z] = seq;
    sb.len[z] = len;
    sb.pos[z] = pos;
  }
  return OOMATTN_OK;
}

void commit_append(oomattn_ctx* ctx, int layer, const SeqBatch& sb, int n_new) {
  for (int z = 0; z < sb.n; ++z) ctx->h_len[(size_t)layer * ctx->cfg.max_seqs + sb.seq[z]] += n_new;
}

AppendArgs base_append_args(oomattn_ctx* ctx, int layer, int n_new) {
  AppendArgs ap;
  memset(&ap, 0, sizeof(ap));
  ap.cos_t = ctx->d_cos;
  ap.sin_t = ctx->d_sin;
  ap.max_pos = ctx->cfg.max_seq_len;
  ap.n_heads = ctx->cfg.n_heads;
  ap.n_new = n_new;
  ap.layer = layer;
  ap.variant = ctx->cfg.rope_variant;
  ap.rope_k = 1;
  ap.status = ctx->d_status;
  return ap;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// A launch as a programmatic dependent of the kernel before it on the stream:
// it may start while that kernel runs; the kernel waits (griddepcontrol.wait)
// before it touches anything the earlier kernel reads or writes.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Vectorised K-A epilogue over T tokens (one template instance per input /
// q-output / cache dtype combination).
int launch_rope_append(oomattn_ctx* ctx, const AppendArgs& ap, const SeqBatch& sb, int T) {
  const void* ptrs[] = {ap.q, ap.k, ap.v, ap.q_out, ap.bq, ap.bk, ap.bv};
  for (const void* p : ptrs)
    if (p && !aligned16(p)) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "tensors and biases must be 16-byte aligned");
  const int hq = ctx->cfg.n_heads, hkv = ctx->cfg.n_kv_heads;
  const long long units = (long long)T * ((ap.k ? (hq + 2 * hkv) * 8 : hq * 8) - (ap.q ? 0 : hq * 8));
  if (units >= (1ll << 31)) return fail(ctx, OOMATTN_ERR_OUT_OF_RANGE, "%d tokens in one append call", T);
  // four CTAs per SM, each thread looping over several 16-element units (measured: 16.1 us for a
  // 4096-token bf16 prefill against 18.1 us with one unit per thread)
  const int grid = (int)std::max<long long>(1, std::min<long long>((units + 255) / 256, (long long)ctx->num_sms * 4));
  const KVPool pool = make_pool(ctx);
  const int combo = (ap.in_bf16 ? 4 : 0) | (ap.q_out_bf16 ? 2 : 0) | (pool.kv_bf16 ? 1 : 0);
  cudaError_t le = cudaSuccess;
#define OOMATTN_RA(I, Q, K) le = launch_pdl(rope_append_kernel<I, Q, K>, dim3(grid), dim3(256), 0, ctx->stream, ap, pool, sb, T)
  switch (combo) {
    case 0: OOMATTN_RA(false, false, false); break;
    case 1: OOMATTN_RA(false, false, true); break;
    case 2: OOMATTN_RA(false, true, false); break;
    case 3: OOMATTN_RA(false, true, true); break;
    case 4: OOMATTN_RA(true, false, false); break;
    case 5: OOMATTN_RA(true, false, true); break;
    case 6: OOMATTN_RA(true, true, false); break;
    default: OOMATTN_RA(true, true, true); break;
  }
#undef OOMATTN_RA
  if (le != cudaSuccess) return fail(ctx, OOMATTN_ERR_CUDA, "append launch: %s", cudaGetErrorString(le));
  return OOMATTN_OK;
}

// Split-KV decode schedule.  Row z's pages are split into ns_z = ceil(pages_z
// / t) near-equal ranges (at most max_splits) for each kv head, and the rows
// are ordered by range size, longest first, so that the block scheduler's
// in-order hand-out of CTAs to free slots is a longest-processing-time list
// schedule.  t is the best of three candidates -- the smallest t that gives at
// most 1, 2 or 3 waves of CTAs on the resident slots -- scored by simulating
// that list schedule with kDecodeFillPages pages of fixed cost per CTA
// (pipeline fill and merge).  Returns the number of items (the grid size).
constexpr int kDecodeFillPages = 12;     // bf16 cache
constexpr int kDecodeFillPagesF32 = 12;  // f32 cache (measured insensitive: 4 to 200 chose the same plans on C1)
constexpr int kDecodeMaxSimSlots = 2048;

long long lpt_makespan(const int* size, const int* count, int groups, int slots, int fill, long long* heap) {
  // min-heap of slot finish times, in pages
  for (int i = 0; i < slots; ++i) heap[i] = 0;
  for (int gi = 0; gi < groups; ++gi) {
    for (int k = 0; k < count[gi]; ++k) {
      heap[0] += size[gi] + fill;  // the earliest free slot takes the item; sift it down
      int i = 0;
      for (;;) {
        const int l = 2 * i + 1, r = l + 1;
        int m = i;
        if (l < slots && heap[l] < heap[m]) m = l;
        if (r < slots && heap[r] < heap[m]) m = r;
        if (m == i) break;
        std::swap(heap[i], heap[m]);
        i = m;
      }
    }
  }
  long long mx = 0;
  for (int i = 0; i < slots; ++i) mx = std::max(mx, heap[i]);
  return mx;
}

int plan_decode(const SeqBatch& sb, int n_kv, int slots, int max_splits, int fill, DecodeSched& sched) {
  slots = std::max(1, std::min(slots, kDecodeMaxSimSlots));
  int pages[kMaxBatch];
  int mp = 0;
  for (int z = 0; z < sb.n; ++z) {
    pages[z] = sb.len[z] > 0 ? (sb.len[z] + kPageSize - 1) / kPageSize : 0;
    mp = std::max(mp, pages[z]);
  }
  const int t_lo = std::max(1, (mp + max_splits - 1) / max_splits);
  const int t_hi = std::max(t_lo, mp);
  auto ns_of = [&](int p, int t) { return p > 0 ? (p + t - 1) / t : 1; };
  auto ctas_of = [&](int t) {
    long long c = 0;
    for (int z = 0; z < sb.n; ++z) c += (long long)ns_of(pages[z], t) * n_kv;
    return c;
  };
  // candidates: the smallest t giving at most 1, 2 or 3 waves (ctas falls as
  // t grows), and for batches too small to fill one wave, whole rows cut in
  // 1, 2, 4 or 8 ranges
  int cand[7];
  int n_cand = 0;
  for (int w = 1; w <= 3; ++w) {
    int lo = t_lo, hi = t_hi;
    while (lo < hi) {
      const int mid = lo + (hi - lo) / 2;
      if (ctas_of(mid) <= (long long)w * slots) hi = mid; else lo = mid + 1;
    }
    cand[n_cand++] = lo;
  }
  for (int k = 1; k <= 8; k *= 2) {
    const int t = std::max(t_lo, (mp + k - 1) / k);
    if (t > cand[0]) cand[n_cand++] = t;
  }
  long long heap[kDecodeMaxSimSlots];
  int order[kMaxBatch], size[kMaxBatch], count[kMaxBatch];
  int best_t = cand[0];
  long long best_cost = -1;
  for (int ci = 0; ci < n_cand; ++ci) {
    const int t = cand[ci];
    if (std::find(cand, cand + ci, t) != cand + ci) continue;
    for (int z = 0; z < sb.n; ++z) order[z] = z;
    auto range = [&](int z) { const int p = pages[z]; return p > 0 ? (p + ns_of(p, t) - 1) / ns_of(p, t) : 0; };
    std::sort(order, order + sb.n, [&](int x, int y) { return range(x) > range(y); });
    for (int r = 0; r < sb.n; ++r) {
      size[r] = range(order[r]);
      count[r] = ns_of(pages[order[r]], t) * n_kv;
    }
    const long long cost = lpt_makespan(size, count, sb.n, slots, fill, heap);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best_t = t;
    }
  }
  // the chosen schedule
  sched.n = sb.n;
  for (int z = 0; z < sb.n; ++z) order[z] = z;
  auto range_best = [&](int z) {
    const int p = pages[z];
    return p > 0 ? (p + ns_of(p, best_t) - 1) / ns_of(p, best_t) : 0;
  };
  std::sort(order, order + sb.n, [&](int x, int y) { return range_best(x) > range_best(y); });
  int items = 0;
  for (int r = 0; r < sb.n; ++r) {
    sched.order[r] = order[r];
    sched.nsplit[r] = ns_of(pages[order[r]], best_t);
    sched.item0[r] = items;
    items += sched.nsplit[r] * n_kv;
  }
  sched.item0[sb.n] = items;
  return items;
}

int launch_decode_rows(oomattn_ctx* ctx, int layer, const SeqBatch& sb, const float* q, float* out, float* lse,
                       int o_stride, int lse_stride) {
  const int n_kv = ctx->cfg.n_kv_heads;
  const int slots = ctx->num_sms * (ctx->cfg.kv_dtype == OOMATTN_DTYPE_BF16 ? kDecCtasPerSm : 3);
  int key[kMaxBatch + 1];
  key[0] = sb.n;
  for (int z = 0; z < sb.n; ++z) key[z + 1] = sb.len[z] > 0 ? (sb.len[z] + kPageSize - 1) / kPageSize : 0;
  if (ctx->sched_key.size() != (size_t)sb.n + 1 || !std::equal(key, key + sb.n + 1, ctx->sched_key.begin())) {
    ctx->sched_items = plan_decode(sb, n_kv, slots, split_cap(ctx->cfg.kv_dtype),
                                   ctx->cfg.kv_dtype == OOMATTN_DTYPE_BF16 ? kDecodeFillPages : kDecodeFillPagesF32,
                                   ctx->sched);
    ctx->sched_key.assign(key, key + sb.n + 1);
  }
  const DecodeSched& sched = ctx->sched;
  const int n_items = ctx->sched_items;
  if (n_items == 0) return OOMATTN_OK;
  DecodeArgs a;
  a.q = q;
  a.out = out;
  a.lse = lse;
  a.o_stride = o_stride;
  a.lse_stride = lse_stride;
  a.test_flags = ctx->test_flags;
  a.layer = layer;
  a.n_heads = ctx->cfg.n_heads;
  a.group = ctx->group;
  a.max_splits = split_cap(ctx->cfg.kv_dtype);
  a.qscale = ctx->scale * 1.4426950408889634f;
  a.part_o = ctx->d_part_o;
  a.part_lse = ctx->d_part_lse;
  a.counters = ctx->d_counters;
  a.status = ctx->d_status;
  a.timeout_ns = ctx->timeout_ns;
  KVPool pool = make_pool(ctx);
  // a programmatic dependent of the append before it (see prefetch_then_wait)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_items);
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t le;
  if (ctx->cfg.kv_dtype == OOMATTN_DTYPE_BF16) {
    cfg.blockDim = dim3((kDecWarps + 1) * 32);
    cfg.dynamicSmemBytes = kDecSmemBytes;
    le = cudaLaunchKernelEx(&cfg, decode_bf16_kernel, ctx->kmap, ctx->vmap, pool, a, sb, sched);
  } else {
    cfg.blockDim = dim3(kDecWarps * 32);
    le = cudaLaunchKernelEx(&cfg, decode_f32_kernel, pool, a, sb, sched);
  }
  if (le != cudaSuccess) return fail(ctx, OOMATTN_ERR_CUDA, "decode launch: %s", cudaGetErrorString(le));
  CKLAUNCH();
  return OOMATTN_OK;
}

}  // namespace

namespace {
// Decode rows in launches of at most kMaxBatch rows; (row, head) outputs at
// out + (row * n_heads + head) * o_stride and lse + (row * n_heads + head) * lse_stride.
int decode_rows_impl(oomattn_ctx* ctx, int layer, int n_rows, const int32_t* seq_ids, const int32_t* lens,
                     const float* q, float* out, float* lse, int o_stride, int lse_stride) {
  int rc = check_layer(ctx, layer);
  if (rc) return rc;
  DeviceGuard dg(ctx->device);
  const int hq = ctx->cfg.n_heads;
  for (int r0 = 0; r0 < n_rows; r0 += kMaxBatch) {
    const int n = std::min(kMaxBatch, n_rows - r0);
    SeqBatch sb;
    sb.n = n;
    for (int z = 0; z < n; ++z) {
      const int seq = seq_ids[r0 + z];
      rc = check_seq(ctx, seq);
      if (rc) return rc;
      const int cur = ctx->h_len[(size_t)layer * ctx->cfg.max_seqs + seq];
      const int len = lens ? lens[r0 + z] : cur;
      if (len < 0 || len > cur)
        return fail(ctx, OOMATTN_ERR_OUT_OF_RANGE, "row %d: length %d outside [0, %d]", r0 + z, len, cur);
      sb.seq[z] = seq;
      sb.len[z] = len;
      sb.pos[z] = 0;
    }
    rc = launch_decode_rows(ctx, layer, sb, q + (size_t)r0 * hq * kHeadDim, out + (size_t)r0 * hq * o_stride,
                            lse ? lse + (size_t)r0 * hq * lse_stride : nullptr, o_stride, lse_stride);
    if (rc) return rc;
  }
  return OOMATTN_OK;
}

// The GEMV is a programmatic dependent of the kernel before it: it launches
// during that kernel's tail and waits (griddepcontrol.wait) before reading x.
template <int T, bool WBF16>
cudaError_t launch_gemv(const GemvArgs& ga, const KVPool& pool, const SeqBatch& sb, int grid, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, qkv_gemv_rope_append_kernel<T, WBF16>, ga, pool, sb);
}
}  // namespace

extern "C" {

const char* oomattn_version(void) { return "oomattn 0.1 (sm_100a)"; }

const char* oomattn_last_error(const oomattn_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

int oomattn_create(const oomattn_config* cfg, int device, void* stream, oomattn_ctx** out) {
  if (!cfg || !out) return OOMATTN_ERR_INVALID_ARG;
  *out = nullptr;
  const oomattn_config& c = *cfg;
  if (c.head_dim != kHeadDim || c.page_size != kPageSize || c.n_heads <= 0 || c.n_kv_heads <= 0 ||
      c.n_heads % c.n_kv_heads != 0 || c.n_heads / c.n_kv_heads > kMaxGroup || c.n_layers <= 0 ||
      c.max_seq_len <= 0 || c.max_seqs <= 0 || c.n_pages <= 0 || c.hidden_size < 0 || !(c.rope_theta > 0.f) ||
      (c.kv_dtype != OOMATTN_DTYPE_F32 && c.kv_dtype != OOMATTN_DTYPE_BF16) ||
      (c.rope_variant != OOMATTN_ROPE_SPLIT_HALF && c.rope_variant != OOMATTN_ROPE_INTERLEAVED))
    return OOMATTN_ERR_BAD_CONFIG;
  const long long rows = (long long)c.n_layers * (c.n_pages + 1) * c.n_kv_heads * kPageSize;
  if (rows >= (1ll << 31)) return OOMATTN_ERR_BAD_CONFIG;

  oomattn_ctx* ctx = new oomattn_ctx();
  ctx->cfg = c;
  ctx->device = device;
  ctx->stream = reinterpret_cast<cudaStream_t>(stream);
  ctx->group = c.n_heads / c.n_kv_heads;
  ctx->max_pages_per_seq = (c.max_seq_len + kPageSize - 1) / kPageSize;
  ctx->n_pool_pages = c.n_pages + 1;
  ctx->esize = c.kv_dtype == OOMATTN_DTYPE_BF16 ? 2 : 4;
  ctx->scale = c.softmax_scale > 0.f ? c.softmax_scale : 1.0f / sqrtf((float)kHeadDim);
  DeviceGuard dg(device);
  auto bail = [&](int code) {
    oomattn_destroy(ctx);
    return code;
  };
  if (cudaSetDevice(device) != cudaSuccess) return bail(OOMATTN_ERR_CUDA);
  cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device);
  const size_t pool_bytes = (size_t)rows * kHeadDim * ctx->esize;
  if (cudaMalloc(&ctx->kpool, pool_bytes) != cudaSuccess || cudaMalloc(&ctx->vpool, pool_bytes) != cudaSuccess)
    return bail(OOMATTN_ERR_NO_MEMORY);
  if (cudaMemset(ctx->kpool, 0, pool_bytes) != cudaSuccess || cudaMemset(ctx->vpool, 0, pool_bytes) != cudaSuccess)
    return bail(OOMATTN_ERR_CUDA);
  const size_t bt_n = (size_t)c.max_seqs * ctx->max_pages_per_seq;
  ctx->h_block_table.assign(bt_n, ctx->n_pool_pages - 1);
  ctx->h_len.assign((size_t)c.n_layers * c.max_seqs, 0);
  ctx->h_pos_off.assign(c.max_seqs, 0);
  if (cudaMalloc(&ctx->d_block_table, bt_n * sizeof(int)) != cudaSuccess) return bail(OOMATTN_ERR_NO_MEMORY);
  if (cudaMemcpy(ctx->d_block_table, ctx->h_block_table.data(), bt_n * sizeof(int), cudaMemcpyHostToDevice) !=
      cudaSuccess)
    return bail(OOMATTN_ERR_CUDA);
  build_rope_table(c.rope_theta, c.max_seq_len, ctx->h_cos, ctx->h_sin);
  const size_t tab = ctx->h_cos.size() * sizeof(float);
  if (cudaMalloc(&ctx->d_cos, tab) != cudaSuccess || cudaMalloc(&ctx->d_sin, tab) != cudaSuccess)
    return bail(OOMATTN_ERR_NO_MEMORY);
  if (cudaMemcpy(ctx->d_cos, ctx->h_cos.data(), tab, cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(ctx->d_sin, ctx->h_sin.data(), tab, cudaMemcpyHostToDevice) != cudaSuccess)
    return bail(OOMATTN_ERR_CUDA);
  const size_t parts = (size_t)kMaxBatch * c.n_heads * split_cap(c.kv_dtype);
  if (cudaMalloc(&ctx->d_part_o, parts * kHeadDim * sizeof(float)) != cudaSuccess ||
      cudaMalloc(&ctx->d_part_lse, parts * sizeof(float)) != cudaSuccess ||
      cudaMalloc(&ctx->d_counters, (size_t)kMaxBatch * c.n_kv_heads * sizeof(unsigned)) != cudaSuccess ||
      cudaMalloc(&ctx->d_status, sizeof(int)) != cudaSuccess)
    return bail(OOMATTN_ERR_NO_MEMORY);
  if (cudaMemset(ctx->d_counters, 0, (size_t)kMaxBatch * c.n_kv_heads * sizeof(unsigned)) != cudaSuccess ||
      cudaMemset(ctx->d_status, 0, sizeof(int)) != cudaSuccess)
    return bail(OOMATTN_ERR_CUDA);
  if (c.kv_dtype == OOMATTN_DTYPE_BF16) {
    if (encode_pool_map(ctx, ctx->kpool, &ctx->kmap) || encode_pool_map(ctx, ctx->vpool, &ctx->vmap))
      return bail(OOMATTN_ERR_CUDA);
    ctx->have_maps = true;
  }
  if (cudaFuncSetAttribute(decode_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDecSmemBytes) !=
          cudaSuccess ||
      cudaFuncSetAttribute(prefill_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmemBytes) !=
          cudaSuccess ||
      cudaFuncSetAttribute(q8_linear_xs_kernel<2, 2, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)q8_xs_smem_bytes(2, q8_xs_max_chunks(2))) != cudaSuccess ||
      cudaFuncSetAttribute(q8_linear_xs_kernel<2, 1, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)q8_xs_smem_bytes(2, q8_xs_max_chunks(2))) != cudaSuccess ||
      cudaFuncSetAttribute(q8_linear_xs_kernel<1, 2, kQ8Xs1S2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)q8_xs_smem_bytes(1, q8_xs_max_chunks(1))) != cudaSuccess ||
      cudaFuncSetAttribute(q8_linear_xs_kernel<1, 1, kQ8Xs1S1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)q8_xs_smem_bytes(1, q8_xs_max_chunks(1))) != cudaSuccess ||
      cudaFuncSetAttribute(kf_gemm_kernel<false, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kKfSmemBytes) !=
          cudaSuccess ||
      cudaFuncSetAttribute(kf_gemm_kernel<false, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kKfSmemBytes) !=
          cudaSuccess ||
      cudaFuncSetAttribute(kf_gemm_kernel<true, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kKfSmemBytes) !=
          cudaSuccess ||
      cudaFuncSetAttribute(q8_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmemBytes) != cudaSuccess)
    return bail(OOMATTN_ERR_CUDA);
  cudaFuncAttributes fa;
  if (cudaFuncGetAttributes(&fa, prefill_bf16_kernel) != cudaSuccess) return bail(OOMATTN_ERR_CUDA);
  ctx->prefill_regs = fa.numRegs;
  if (cudaFuncGetAttributes(&fa, kf_gemm_kernel<true, 1>) != cudaSuccess) return bail(OOMATTN_ERR_CUDA);
  ctx->kf_q8_regs = fa.numRegs;
  if (cudaDeviceSynchronize() != cudaSuccess) return bail(OOMATTN_ERR_CUDA);
  *out = ctx;
  return OOMATTN_OK;
}

int oomattn_destroy(oomattn_ctx* ctx) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  DeviceGuard dg(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  void* ptrs[] = {ctx->kpool,     ctx->vpool,      ctx->d_block_table, ctx->d_cos,    ctx->d_sin,
                  ctx->d_part_o,  ctx->d_part_lse, ctx->d_counters,    ctx->d_status, ctx->d_scratch,
                  ctx->d_q8_scratch, ctx->d_q8_counters, ctx->d_layer_scratch, ctx->d_model_scratch,
                  ctx->d_argmax_part, ctx->d_kf, ctx->d_pf_part};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  delete ctx;
  return OOMATTN_OK;
}

int oomattn_set_stream(oomattn_ctx* ctx, void* stream) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  ctx->stream = reinterpret_cast<cudaStream_t>(stream);
  return OOMATTN_OK;
}

int oomattn_sync(oomattn_ctx* ctx) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  DeviceGuard dg(ctx->device);
  CK(cudaStreamSynchronize(ctx->stream));
  int st = 0;
  CK(cudaMemcpy(&st, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost));
  if (st) {
    CK(cudaMemset(ctx->d_status, 0, sizeof(int)));
    // a linear that gave up on a wait may have left cut-tile arrivals behind
    if (ctx->d_q8_counters) CK(cudaMemset(ctx->d_q8_counters, 0, sizeof(unsigned) * ctx->q8_counters_n));
    if (st & kDevErrTimeout) return fail(ctx, OOMATTN_ERR_TIMEOUT, "a device-side wait timed out (status %d)", st);
    if (st & kDevErrRange)
      return fail(ctx, OOMATTN_ERR_DEVICE_CHECK,
                  "prefill met a cached V value of magnitude >= 65536, outside the fp16 P.V product (status %d)", st);
    if (st & kDevErrFormat)
      return fail(ctx, OOMATTN_ERR_DEVICE_CHECK,
                  "q8_repack met a block whose length field disagrees with its position (status %d)", st);
    if (st & kDevErrX16)
      return fail(ctx, OOMATTN_ERR_DEVICE_CHECK,
                  "q8_linear met an activation of magnitude >= 65504, outside its fp16 hi/lo split (status %d)", st);
    return fail(ctx, OOMATTN_ERR_DEVICE_CHECK, "a device-side index check failed (status %d)", st);
  }
  return OOMATTN_OK;
}

int oomattn_reset(oomattn_ctx* ctx) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  std::fill(ctx->h_len.begin(), ctx->h_len.end(), 0);
  return OOMATTN_OK;
}

int oomattn_seq_len(const oomattn_ctx* ctx, int32_t layer, int32_t seq, int32_t* out_len) {
  if (!ctx || !out_len) return OOMATTN_ERR_INVALID_ARG;
  if (layer < 0 || layer >= ctx->cfg.n_layers || seq < 0 || seq >= ctx->cfg.max_seqs) return OOMATTN_ERR_OUT_OF_RANGE;
  *out_len = ctx->h_len[(size_t)layer * ctx->cfg.max_seqs + seq];
  return OOMATTN_OK;
}

int oomattn_set_block_table(oomattn_ctx* ctx, int32_t seq, const int32_t* pages, int32_t n) {
  if (!ctx || (n > 0 && !pages) || n < 0) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad block-table arguments");
  int rc = check_seq(ctx, seq);
  if (rc) return rc;
  if (n > ctx->max_pages_per_seq)
    return fail(ctx, OOMATTN_ERR_OUT_OF_RANGE, "%d pages exceed max_seq_len / 16 = %d", n, ctx->max_pages_per_seq);
  for (int i = 0; i < n; ++i)
    if (pages[i] < 0 || pages[i] >= ctx->cfg.n_pages)
      return fail(ctx, OOMATTN_ERR_OUT_OF_RANGE, "page id %d outside [0, %d)", pages[i], ctx->cfg.n_pages);
  int* row = ctx->h_block_table.data() + (size_t)seq * ctx->max_pages_per_seq;
  for (int i = 0; i < ctx->max_pages_per_seq; ++i) row[i] = i < n ? pages[i] : ctx->n_pool_pages - 1;
  DeviceGuard dg(ctx->device);
  CK(cudaMemcpyAsync(ctx->d_block_table + (size_t)seq * ctx->max_pages_per_seq, row,
                     ctx->max_pages_per_seq * sizeof(int), cudaMemcpyHostToDevice, ctx->stream));
  CK(cudaStreamSynchronize(ctx->stream));  // the host row may change again before the copy would run
  return OOMATTN_OK;
}

int oomattn_set_position_offset(oomattn_ctx* ctx, int32_t seq, int32_t offset) {
  if (!ctx || offset < 0) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad position offset");
  int rc = check_seq(ctx, seq);
  if (rc) return rc;
  ctx->h_pos_off[seq] = offset;
  return OOMATTN_OK;
}

int oomattn_set_seq_len(oomattn_ctx* ctx, int32_t layer, int32_t seq, int32_t len) {
  if (!ctx || len < 0) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad length");
  int rc = check_layer(ctx, layer);
  if (!rc) rc = check_seq(ctx, seq);
  if (!rc) rc = check_slots(ctx, seq, 0, len);
  if (rc) return rc;
  ctx->h_len[(size_t)layer * ctx->cfg.max_seqs + seq] = len;
  return OOMATTN_OK;
}

int oomattn_kv_pool(const oomattn_ctx* ctx, void** k_pool, void** v_pool) {
  if (!ctx || !k_pool || !v_pool) return OOMATTN_ERR_INVALID_ARG;
  *k_pool = ctx->kpool;
  *v_pool = ctx->vpool;
  return OOMATTN_OK;
}

int oomattn_kv_write(oomattn_ctx* ctx, int32_t layer, int32_t seq, const void* k, const void* v, int32_t n,
                     int32_t src_dtype) {
  if (!ctx || !k || !v || n < 0) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad kv_write arguments");
  int rc = check_layer(ctx, layer);
  if (!rc) rc = validate_dtype(ctx, src_dtype, "kv_write");
  if (rc) return rc;
  if (n == 0) return OOMATTN_OK;
  SeqBatch sb;
  int32_t sid = seq;
  rc = plan_append(ctx, layer, 1, &sid, n, sb);
  if (rc) return rc;
  AppendArgs ap = base_append_args(ctx, layer, n);
  ap.q = nullptr;
  ap.k = k;
  ap.v = v;
  ap.in_bf16 = src_dtype == OOMATTN_DTYPE_BF16;
  ap.rope_k = 0;  // K is stored as given: no rotation
  DeviceGuard dg(ctx->device);
  rc = launch_rope_append(ctx, ap, sb, n);
  if (rc) return rc;
  CKLAUNCH();
  commit_append(ctx, layer, sb, n);
  return OOMATTN_OK;
}

int oomattn_kv_read(oomattn_ctx* ctx, int32_t layer, int32_t seq, void* k_out, void* v_out) {
  if (!ctx || !k_out || !v_out) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad kv_read arguments");
  int rc = check_layer(ctx, layer);
  if (!rc) rc = check_seq(ctx, seq);
  if (rc) return rc;
  DeviceGuard dg(ctx->device);
  CK(cudaStreamSynchronize(ctx->stream));
  const int L = ctx->h_len[(size_t)layer * ctx->cfg.max_seqs + seq];
  const int n_kv = ctx->cfg.n_kv_heads;
  const size_t es = ctx->esize;
  std::vector<uint8_t> page(kPageSize * kHeadDim * es);
  for (int lp = 0; lp * kPageSize < L; ++lp) {
    const int pg = ctx->h_block_table[(size_t)seq * ctx->max_pages_per_seq + lp];
    const int nt = std::min(kPageSize, L - lp * kPageSize);
    for (int g = 0; g < n_kv; ++g) {
      const size_t off = (((size_t)layer * ctx->n_pool_pages + pg) * n_kv + g) * kPageSize * kHeadDim * es;
      for (int which = 0; which < 2; ++which) {
        const uint8_t* src = (const uint8_t*)(which ? ctx->vpool : ctx->kpool) + off;
        CK(cudaMemcpy(page.data(), src, page.size(), cudaMemcpyDeviceToHost));
        uint8_t* dst = (uint8_t*)(which ? v_out : k_out) + ((size_t)g * L + (size_t)lp * kPageSize) * kHeadDim * es;
        memcpy(dst, page.data(), (size_t)nt * kHeadDim * es);
      }
    }
  }
  return OOMATTN_OK;
}

int oomattn_rope_table(const oomattn_ctx* ctx, int32_t pos0, int32_t n, float* cos_out, float* sin_out) {
  if (!ctx || !cos_out || !sin_out || n < 0 || pos0 < 0) return OOMATTN_ERR_INVALID_ARG;
  if (pos0 + n > ctx->cfg.max_seq_len) return OOMATTN_ERR_OUT_OF_RANGE;
  memcpy(cos_out, ctx->h_cos.data() + (size_t)pos0 * 64, (size_t)n * 64 * sizeof(float));
  memcpy(sin_out, ctx->h_sin.data() + (size_t)pos0 * 64, (size_t)n * 64 * sizeof(float));
  return OOMATTN_OK;
}

int oomattn_compute_rope_table(float theta, int32_t head_dim, int32_t pos0, int32_t n, float* cos_out,
                               float* sin_out) {
  if (!cos_out || !sin_out || n < 0 || pos0 < 0 || !(theta > 0.f)) return OOMATTN_ERR_INVALID_ARG;
  if (head_dim != kHeadDim) return OOMATTN_ERR_BAD_CONFIG;
  std::vector<float> c, s;
  build_rope_table(theta, pos0 + n, c, s);
  memcpy(cos_out, c.data() + (size_t)pos0 * 64, (size_t)n * 64 * sizeof(float));
  memcpy(sin_out, s.data() + (size_t)pos0 * 64, (size_t)n * 64 * sizeof(float));
  return OOMATTN_OK;
}

int oomattn_rope_append(oomattn_ctx* ctx, int32_t layer, int32_t n_seqs, const int32_t* seq_ids, int32_t n_new,
                        const void* q, const void* k, const void* v, int32_t in_dtype, const float* bq,
                        const float* bk, const float* bv, void* q_out, int32_t q_out_dtype) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  if (!seq_ids || !q || !k || !v || !q_out || n_seqs <= 0 || n_new <= 0)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad rope_append arguments");
  int rc = check_layer(ctx, layer);
  if (!rc) rc = validate_dtype(ctx, in_dtype, "rope_append input");
  if (!rc) rc = validate_dtype(ctx, q_out_dtype, "rope_append q_out");
  if (rc) return rc;
  DeviceGuard dg(ctx->device);
  const int in_es = in_dtype == OOMATTN_DTYPE_BF16 ? 2 : 4, out_es = q_out_dtype == OOMATTN_DTYPE_BF16 ? 2 : 4;
  for (int r0 = 0; r0 < n_seqs; r0 += kMaxBatch) {
    const int n = std::min(kMaxBatch, n_seqs - r0);
    SeqBatch sb;
    rc = plan_append(ctx, layer, n, seq_ids + r0, n_new, sb);
    if (rc) return rc;
    const size_t t0 = (size_t)r0 * n_new;
    AppendArgs ap = base_append_args(ctx, layer, n_new);
    ap.q = (const uint8_t*)q + t0 * ctx->cfg.n_heads * kHeadDim * in_es;
    ap.k = (const uint8_t*)k + t0 * ctx->cfg.n_kv_heads * kHeadDim * in_es;
    ap.v = (const uint8_t*)v + t0 * ctx->cfg.n_kv_heads * kHeadDim * in_es;
    ap.in_bf16 = in_dtype == OOMATTN_DTYPE_BF16;
    ap.q_out = (uint8_t*)q_out + t0 * ctx->cfg.n_heads * kHeadDim * out_es;
    ap.q_out_bf16 = q_out_dtype == OOMATTN_DTYPE_BF16;
    ap.bq = bq;
    ap.bk = bk;
    ap.bv = bv;
    rc = launch_rope_append(ctx, ap, sb, n * n_new);
    if (rc) return rc;
    CKLAUNCH();
    commit_append(ctx, layer, sb, n_new);
  }
  return OOMATTN_OK;
}

int oomattn_rope_q(oomattn_ctx* ctx, int32_t n_rows, const int32_t* positions, const void* q, int32_t in_dtype,
                   const float* bq, void* q_out, int32_t q_out_dtype) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  if (!positions || !q || !q_out || n_rows <= 0) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad rope_q arguments");
  int rc = validate_dtype(ctx, in_dtype, "rope_q input");
  if (!rc) rc = validate_dtype(ctx, q_out_dtype, "rope_q q_out");
  if (rc) return rc;
  DeviceGuard dg(ctx->device);
  const int in_es = in_dtype == OOMATTN_DTYPE_BF16 ? 2 : 4, out_es = q_out_dtype == OOMATTN_DTYPE_BF16 ? 2 : 4;
  for (int r0 = 0; r0 < n_rows; r0 += kMaxBatch) {
    const int n = std::min(kMaxBatch, n_rows - r0);
    SeqBatch sb;
    sb.n = n;
    for (int z = 0; z < n; ++z) {
      const int pos = positions[r0 + z];
      if (pos < 0 || pos >= ctx->cfg.max_seq_len)
        return fail(ctx, OOMATTN_ERR_OUT_OF_RANGE, "row %d: position %d outside [0, %d)", r0 + z, pos,
                    ctx->cfg.max_seq_len);
      sb.seq[z] = 0;
      sb.len[z] = 0;
      sb.pos[z] = pos;
    }
    AppendArgs ap = base_append_args(ctx, 0, 1);
    ap.q = (const uint8_t*)q + (size_t)r0 * ctx->cfg.n_heads * kHeadDim * in_es;
    ap.k = nullptr;  // q rows only: nothing is appended
    ap.v = nullptr;
    ap.in_bf16 = in_dtype == OOMATTN_DTYPE_BF16;
    ap.q_out = (uint8_t*)q_out + (size_t)r0 * ctx->cfg.n_heads * kHeadDim * out_es;
    ap.q_out_bf16 = q_out_dtype == OOMATTN_DTYPE_BF16;
    ap.bq = bq;
    rc = launch_rope_append(ctx, ap, sb, n);
    if (rc) return rc;
  }
  return OOMATTN_OK;
}

int oomattn_qkv_rope_append(oomattn_ctx* ctx, int32_t layer, int32_t n_seqs, const int32_t* seq_ids, int32_t n_new,
                            const float* x, const void* wq, const void* wk, const void* wv, int32_t w_dtype,
                            const float* bq, const float* bk, const float* bv, void* q_out, int32_t q_out_dtype) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  if (!seq_ids || !x || !wq || !wk || !wv || !q_out || n_seqs <= 0 || n_new <= 0)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad qkv_rope_append arguments");
  int rc = check_layer(ctx, layer);
  if (!rc) rc = validate_dtype(ctx, w_dtype, "weights");
  if (!rc) rc = validate_dtype(ctx, q_out_dtype, "q_out");
  if (rc) return rc;
  const int H = ctx->cfg.hidden_size;
  if (H <= 0 || H % 8 != 0) return fail(ctx, OOMATTN_ERR_BAD_CONFIG, "hidden_size %d must be a positive multiple of 8", H);
  DeviceGuard dg(ctx->device);
  const long long T = (long long)n_seqs * n_new;
  const int nq = ctx->cfg.n_heads * kHeadDim, nk = ctx->cfg.n_kv_heads * kHeadDim;
  if (T <= kGemvMaxT) {
    SeqBatch sb;
    rc = plan_append(ctx, layer, n_seqs, seq_ids, n_new, sb);
    if (rc) return rc;
    GemvArgs ga;
    ga.x = x;
    ga.wq = wq;
    ga.wk = wk;
    ga.wv = wv;
    ga.w_bf16 = w_dtype == OOMATTN_DTYPE_BF16;
    ga.hidden = H;
    ga.T = (int)T;
    ga.ap = base_append_args(ctx, layer, n_new);
    ga.ap.q_out = q_out;
    ga.ap.q_out_bf16 = q_out_dtype == OOMATTN_DTYPE_BF16;
    ga.ap.bq = bq;
    ga.ap.bk = bk;
    ga.ap.bv = bv;
    const int grid = (ctx->cfg.n_heads + 2 * ctx->cfg.n_kv_heads) * 8;
    KVPool pool = make_pool(ctx);
#define OOMATTN_GEMV_CASE(TT)                                                                          \
  case TT:                                                                                             \
    le = ga.w_bf16 ? launch_gemv<TT, true>(ga, pool, sb, grid, ctx->stream)                            \
                   : launch_gemv<TT, false>(ga, pool, sb, grid, ctx->stream);                          \
    break;
    cudaError_t le = cudaSuccess;
    switch ((int)T) {
      OOMATTN_GEMV_CASE(1)
      OOMATTN_GEMV_CASE(2)
      OOMATTN_GEMV_CASE(3)
      OOMATTN_GEMV_CASE(4)
      OOMATTN_GEMV_CASE(5)
      OOMATTN_GEMV_CASE(6)
      OOMATTN_GEMV_CASE(7)
      OOMATTN_GEMV_CASE(8)
      OOMATTN_GEMV_CASE(9)
      OOMATTN_GEMV_CASE(10)
      OOMATTN_GEMV_CASE(11)
      OOMATTN_GEMV_CASE(12)
      OOMATTN_GEMV_CASE(13)
      OOMATTN_GEMV_CASE(14)
      OOMATTN_GEMV_CASE(15)
      OOMATTN_GEMV_CASE(16)
    }
#undef OOMATTN_GEMV_CASE
    if (le != cudaSuccess) return fail(ctx, OOMATTN_ERR_CUDA, "qkv gemv launch: %s", cudaGetErrorString(le));
    commit_append(ctx, layer, sb, n_new);
    return OOMATTN_OK;
  }
  // Larger T: tensor-core projections (K-F) into scratch, then the K-A epilogue kernel.
  const int wb = w_dtype == OOMATTN_DTYPE_BF16;
  const size_t proj_bytes = (size_t)T * (nq + 2 * nk) * sizeof(float);
  rc = ensure_scratch(ctx, proj_bytes);
  if (rc) return rc;
  float* sq = ctx->d_scratch;
  float* sk = sq + (size_t)T * nq;
  float* sv = sk + (size_t)T * nk;
  const KfJob jobs[3] = {{wq, wb, nq, nullptr, nullptr, sq}, {wk, wb, nk, nullptr, nullptr, sk},
                         {wv, wb, nk, nullptr, nullptr, sv}};
  rc = kf_linear_f32(ctx, x, (int)T, H, jobs, 3);
  if (rc) return rc;
  return oomattn_rope_append(ctx, layer, n_seqs, seq_ids, n_new, sq, sk, sv, OOMATTN_DTYPE_F32, bq, bk, bv, q_out,
                             q_out_dtype);
}

int oomattn_linear(oomattn_ctx* ctx, const float* x, const void* w, int32_t w_dtype, int32_t n_tokens, int32_t rows,
                   int32_t cols, const float* bias, float* y) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  if (!x || !w || !y || n_tokens < 0 || rows <= 0 || cols <= 0)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad linear arguments");
  int rc = validate_dtype(ctx, w_dtype, "linear weights");
  if (rc) return rc;
  if (n_tokens == 0) return OOMATTN_OK;
  DeviceGuard dg(ctx->device);
  if (n_tokens <= kGemvMaxT && w_dtype == OOMATTN_DTYPE_F32)
    return f32_gemv(ctx, x, static_cast<const float*>(w), n_tokens, rows, cols, bias, nullptr, y);
  const KfJob job{w, w_dtype == OOMATTN_DTYPE_BF16, rows, bias, nullptr, y};
  return kf_linear_f32(ctx, x, n_tokens, cols, &job, 1);
}

int oomattn_decode(oomattn_ctx* ctx, int32_t layer, int32_t n_rows, const int32_t* seq_ids, const int32_t* lens,
                   const float* q, float* out, float* lse) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  if (!seq_ids || !q || !out || n_rows <= 0) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad decode arguments");
  return decode_rows_impl(ctx, layer, n_rows, seq_ids, lens, q, out, lse, kHeadDim, 1);
}

int oomattn_decode_packed(oomattn_ctx* ctx, int32_t layer, int32_t n_rows, const int32_t* seq_ids,
                          const int32_t* lens, const float* q, float* packed) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  if (!seq_ids || !q || !packed || n_rows <= 0)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad decode_packed arguments");
  if (reinterpret_cast<uintptr_t>(packed) % 16 != 0)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "packed must be 16-byte aligned");
  return decode_rows_impl(ctx, layer, n_rows, seq_ids, lens, q, packed, packed + kHeadDim, OOMATTN_PACKED_STRIDE,
                          OOMATTN_PACKED_STRIDE);
}

int oomattn_merge_partials(oomattn_ctx* ctx, int32_t n_parts, int32_t n_rows, const float* parts, const float* lses,
                           float* out, float* lse_out) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  if (!parts || !lses || !out || n_parts <= 0 || n_rows < 0)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad merge arguments");
  if (n_rows == 0) return OOMATTN_OK;
  DeviceGuard dg(ctx->device);
  merge_partials_kernel<<<n_rows, kHeadDim, 0, ctx->stream>>>(parts, lses, kHeadDim, 1, n_parts, n_rows, out,
                                                               lse_out);
  CKLAUNCH();
  return OOMATTN_OK;
}

int oomattn_merge_packed(oomattn_ctx* ctx, int32_t n_parts, int32_t n_rows, const float* packed, float* out,
                         float* lse_out) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  if (!packed || !out || n_parts <= 0 || n_rows < 0)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad merge_packed arguments");
  if (n_rows == 0) return OOMATTN_OK;
  DeviceGuard dg(ctx->device);
  merge_partials_kernel<<<n_rows, kHeadDim, 0, ctx->stream>>>(packed, packed + kHeadDim, OOMATTN_PACKED_STRIDE,
                                                               OOMATTN_PACKED_STRIDE, n_parts, n_rows, out, lse_out);
  CKLAUNCH();
  return OOMATTN_OK;
}

int oomattn_set_wait_limit(oomattn_ctx* ctx, uint64_t timeout_ns) {
  if (!ctx || timeout_ns == 0) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "the wait limit must be positive");
  ctx->timeout_ns = timeout_ns;
  return OOMATTN_OK;
}

int oomattn_set_test_flags(oomattn_ctx* ctx, int32_t flags) {
  if (!ctx || (flags & ~(OOMATTN_TEST_DROP_DECODE_COPIES | OOMATTN_TEST_DROP_LINEAR_COPIES)))
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "unknown test flags %d", flags);
  ctx->test_flags = flags;
  return OOMATTN_OK;
}

int oomattn_prefill(oomattn_ctx* ctx, int32_t layer, int32_t seq, int32_t n_new, const void* q, void* out,
                    int32_t out_dtype, float* lse) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  if (n_new <= 0) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad prefill arguments");
  const int32_t all[2] = {0, (n_new + 255) / 256};
  return oomattn_prefill_blocks(ctx, layer, seq, n_new, q, out, out_dtype, lse, 1, all);
}

int oomattn_prefill_blocks(oomattn_ctx* ctx, int32_t layer, int32_t seq, int32_t n_new, const void* q, void* out,
                           int32_t out_dtype, float* lse, int32_t n_ranges, const int32_t* ranges) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  if (!q || !out || n_new <= 0 || !ranges || n_ranges <= 0)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad prefill arguments");
  int rc = check_layer(ctx, layer);
  if (!rc) rc = check_seq(ctx, seq);
  if (!rc) rc = validate_dtype(ctx, out_dtype, "prefill out");
  if (rc) return rc;
  if (ctx->cfg.kv_dtype != OOMATTN_DTYPE_BF16)
    return fail(ctx, OOMATTN_ERR_UNSUPPORTED, "the tensor-core prefill needs a bf16 cache");
  // The kernel's register split (setmaxnreg) balances only at this launch count.
  if (ctx->prefill_regs != kPfLaunchRegs)
    return fail(ctx, OOMATTN_ERR_UNSUPPORTED, "prefill kernel compiled with %d registers per thread, expected %d",
                ctx->prefill_regs, kPfLaunchRegs);
  if (reinterpret_cast<uintptr_t>(q) % 16 != 0 || reinterpret_cast<uintptr_t>(out) % 16 != 0)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "q and out must be 16-byte aligned");
  const int L = ctx->h_len[(size_t)layer * ctx->cfg.max_seqs + seq];
  if (n_new > L) return fail(ctx, OOMATTN_ERR_OUT_OF_RANGE, "n_new %d exceeds the cached length %d", n_new, L);
  const int n_pairs = (n_new + 255) / 256;
  if (n_ranges > kPfMaxRanges)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "%d block ranges (at most %d)", n_ranges, kPfMaxRanges);
  PrefillArgs a;
  memset(&a, 0, sizeof(a));
  // ranges sorted by descending start; they must lie in [0, n_pairs) and not overlap
  int order[kPfMaxRanges];
  for (int r = 0; r < n_ranges; ++r) order[r] = r;
  std::sort(order, order + n_ranges, [&](int x, int y) { return ranges[2 * x] > ranges[2 * y]; });
  long long blocks = 0;
  for (int i = 0; i < n_ranges; ++i) {
    const int lo = ranges[2 * order[i]], hi = ranges[2 * order[i] + 1];
    if (lo < 0 || hi > n_pairs || lo >= hi)
      return fail(ctx, OOMATTN_ERR_OUT_OF_RANGE, "block range [%d, %d) outside [0, %d) or empty", lo, hi, n_pairs);
    if (i > 0 && hi > a.range_lo[i - 1])
      return fail(ctx, OOMATTN_ERR_INVALID_ARG, "block ranges overlap");
    a.range_lo[i] = lo;
    a.range_hi[i] = hi;
    blocks += hi - lo;
  }
  a.n_ranges = n_ranges;
  DeviceGuard dg(ctx->device);
  // Key split: when one work unit (the pair with the most key tiles) would run
  // much longer than the launch's work per SM -- a sharded rank's few heads --
  // the units are cut into chunks of about that per-SM share of key tiles, so
  // the heaviest block no longer sets the launch time; their partials are
  // merged by one more kernel.  A whole 28-head 4096-token launch is not split.
  const int prefix = L - n_new;
  auto pair_tiles = [&](int p) { return (prefix + std::min(n_new, 256 * p + 256) + 127) / 128; };
  long long work = 0;
  int max_tiles = 1;
  for (int i = 0; i < n_ranges; ++i)
    for (int p = a.range_lo[i]; p < a.range_hi[i]; ++p) {
      work += (long long)pair_tiles(p) * ctx->cfg.n_heads;
      max_tiles = std::max(max_tiles, pair_tiles(p));
    }
  const int per_sm = (int)((work + ctx->num_sms - 1) / ctx->num_sms);
  int key_chunk = max_tiles;
  if (2 * max_tiles > 3 * per_sm) key_chunk = std::max(kPfMinKeyChunk, per_sm);
  const int n_chunks = (max_tiles + key_chunk - 1) / key_chunk;
  a.key_chunk = key_chunk;
  a.n_pad = (n_new + 127) / 128 * 128;
  a.part_lse = nullptr;
  float* part_o = nullptr;
  CUtensorMap qmap, omap, pmap;
  rc = encode_q_map(ctx, q, n_new, &qmap);
  if (!rc) rc = encode_out_map(ctx, out, n_new, out_dtype == OOMATTN_DTYPE_BF16, &omap);
  if (rc) return rc;
  pmap = omap;
  if (n_chunks > 1) {
    const size_t rows_all = (size_t)n_chunks * a.n_pad;
    const size_t ob = rows_all * ctx->cfg.n_heads * kHeadDim * 4, lb = rows_all * ctx->cfg.n_heads * 4;
    if (ob + lb > ctx->pf_part_bytes) {
      if (ctx->d_pf_part) {
        cudaStreamSynchronize(ctx->stream);
        cudaFree(ctx->d_pf_part);
        ctx->d_pf_part = nullptr;
        ctx->pf_part_bytes = 0;
      }
      if (cudaMalloc(&ctx->d_pf_part, ob + lb) != cudaSuccess)
        return fail(ctx, OOMATTN_ERR_NO_MEMORY, "prefill partial scratch of %zu bytes failed", ob + lb);
      ctx->pf_part_bytes = ob + lb;
    }
    part_o = reinterpret_cast<float*>(ctx->d_pf_part);
    a.part_lse = reinterpret_cast<float*>(ctx->d_pf_part + ob);
    rc = encode_out_map(ctx, part_o, (int)rows_all, false, &pmap);
    if (rc) return rc;
  }
  a.out = out;
  a.out_bf16 = out_dtype == OOMATTN_DTYPE_BF16;
  a.lse = lse;
  a.n_new = n_new;
  a.prefix = L - n_new;
  a.seq = seq;
  a.layer = layer;
  a.n_heads = ctx->cfg.n_heads;
  a.group = ctx->group;
  a.n_pairs = n_pairs;
  a.qscale = ctx->scale * 1.4426950408889634f;
  a.status = ctx->d_status;
  a.timeout_ns = ctx->timeout_ns;
  prefill_bf16_kernel<<<dim3((unsigned)(blocks * a.n_heads), n_chunks), kPfThreads, kPfSmemBytes, ctx->stream>>>(
      qmap, ctx->kmap, ctx->vmap, omap, pmap, make_pool(ctx), a);
  CKLAUNCH();
  if (n_chunks > 1) {
    const long long warps = (long long)n_new * a.n_heads;
    prefill_chunk_merge_kernel<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, ctx->stream>>>(part_o, a);
    CKLAUNCH();
  }
  return OOMATTN_OK;
}

int oomattn_attention_forward_with_bias(oomattn_ctx* ctx, int32_t layer, int32_t batch, int32_t seq_len,
                                        const float* x, const float* wq, const float* wk, const float* wv,
                                        const float* wo, int32_t o_out, const float* bq, const float* bk,
                                        const float* bv, float* out) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  if (!x || !wq || !wk || !wv || !wo || !out || batch <= 0 || seq_len <= 0 || o_out <= 0)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad attention_forward_with_bias arguments");
  if (batch > ctx->cfg.max_seqs)
    return fail(ctx, OOMATTN_ERR_OUT_OF_RANGE, "batch %d exceeds max_seqs %d", batch, ctx->cfg.max_seqs);
  int rc = check_layer(ctx, layer);
  if (rc) return rc;
  DeviceGuard dg(ctx->device);
  const long long T = (long long)batch * seq_len;
  const int hq = ctx->cfg.n_heads, qo = hq * kHeadDim;
  const bool use_prefill = ctx->cfg.kv_dtype == OOMATTN_DTYPE_BF16 && seq_len > 16;
  // scratch: q (f32) | attention out (f32) | q bf16 for the prefill path
  const size_t q_bytes = (size_t)T * qo * sizeof(float);
  const size_t need = 2 * q_bytes + (use_prefill ? (size_t)T * qo * 2 : 0);
  // projection scratch is separate from the q/attention buffers; allocate both in one block
  const size_t proj = T > kGemvMaxT ? (size_t)T * (qo + 2 * ctx->cfg.n_kv_heads * kHeadDim) * sizeof(float) : 0;
  rc = ensure_scratch(ctx, need + proj + 256);
  if (rc) return rc;
  float* qbuf = (float*)((uint8_t*)ctx->d_scratch + proj);
  float* abuf = (float*)((uint8_t*)qbuf + q_bytes);
  void* qb16 = (uint8_t*)abuf + q_bytes;
  std::vector<int32_t> seqs(batch);
  for (int b = 0; b < batch; ++b) seqs[b] = b;
  std::vector<int> plen(batch);
  for (int b = 0; b < batch; ++b) plen[b] = ctx->h_len[(size_t)layer * ctx->cfg.max_seqs + b];
  // K-A (the cuBLAS branch writes its projections at the start of the scratch block)
  if (T <= kGemvMaxT) {
    rc = oomattn_qkv_rope_append(ctx, layer, batch, seqs.data(), seq_len, x, wq, wk, wv, OOMATTN_DTYPE_F32, bq, bk,
                                 bv, use_prefill ? qb16 : (void*)qbuf,
                                 use_prefill ? OOMATTN_DTYPE_BF16 : OOMATTN_DTYPE_F32);
  } else {
    float* sq = ctx->d_scratch;
    float* sk = sq + (size_t)T * qo;
    float* sv = sk + (size_t)T * ctx->cfg.n_kv_heads * kHeadDim;
    const int nk = ctx->cfg.n_kv_heads * kHeadDim;
    const int H = ctx->cfg.hidden_size;
    const KfJob jobs[3] = {{wq, 0, qo, nullptr, nullptr, sq}, {wk, 0, nk, nullptr, nullptr, sk},
                           {wv, 0, nk, nullptr, nullptr, sv}};
    rc = kf_linear_f32(ctx, x, (int)T, H, jobs, 3);
    if (rc) return rc;
    rc = oomattn_rope_append(ctx, layer, batch, seqs.data(), seq_len, sq, sk, sv, OOMATTN_DTYPE_F32, bq, bk, bv,
                             use_prefill ? qb16 : (void*)qbuf, use_prefill ? OOMATTN_DTYPE_BF16 : OOMATTN_DTYPE_F32);
  }
  if (rc) return rc;
  // attention
  if (use_prefill) {
    for (int b = 0; b < batch; ++b) {
      rc = oomattn_prefill(ctx, layer, b, seq_len, (uint8_t*)qb16 + (size_t)b * seq_len * qo * 2,
                           abuf + (size_t)b * seq_len * qo, OOMATTN_DTYPE_F32, nullptr);
      if (rc) return rc;
    }
  } else {
    // one decode row per new token: token s of sequence b sees slots 0..P_b+s
    std::vector<int32_t> rs(T), rl(T);
    for (int b = 0; b < batch; ++b)
      for (int s = 0; s < seq_len; ++s) {
        rs[(size_t)b * seq_len + s] = b;
        rl[(size_t)b * seq_len + s] = plen[b] + s + 1;
      }
    rc = oomattn_decode(ctx, layer, (int)T, rs.data(), rl.data(), qbuf, abuf, nullptr);
    if (rc) return rc;
  }
  // o_proj: out = attn . Wo^T   (src/oomllama_turbo.rs:715-720): a GEMV for decode-sized
  // token counts, the tensor-core linear above that
  if (T <= kGemvMaxT) return f32_gemv(ctx, abuf, wo, (int)T, o_out, qo, nullptr, nullptr, out);
  const KfJob oj{wo, 0, o_out, nullptr, nullptr, out};
  return kf_linear_f32(ctx, abuf, (int)T, qo, &oj, 1);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Decode with no device allocation.
//
// Some callers cannot call cudaMalloc on the decode path: a host whose device
// memory is owned by another allocator (an inference server's pooled arena, a
// framework plugin that is handed only tensors), or a latency-critical loop in
// which an allocation could synchronise the device or fail under memory
// pressure.  oomattn_decode_static_scratch serves them: it runs the same
// split-KV decode kernels over KV memory the caller owns, and keeps the
// split-KV partials in a fixed array that is part of this library's device
// image instead of in allocated scratch.  It creates no context and calls no
// allocating routine (no cudaMalloc, cudaFree, cuBLAS or torch).
// ---------------------------------------------------------------------------
#include <mutex>

namespace {

constexpr int kStaticPartSlots = 16384;  // (row, q head, split) partials held at once
constexpr int kStaticMaxKv = 64;         // kv heads per launch covered by the counters
constexpr size_t kStaticPartOBytes = (size_t)kStaticPartSlots * kHeadDim * sizeof(float);  // 8 MiB
constexpr size_t kStaticPartLseBytes = (size_t)kStaticPartSlots * sizeof(float);          // 64 KiB
constexpr size_t kStaticCounterBytes = (size_t)kMaxBatch * kStaticMaxKv * sizeof(unsigned);  // 32 KiB
constexpr size_t kStaticStatusBytes = 256;  // one int: the kernels' error bits, kept until read
constexpr size_t kStaticScratchBytes = kStaticPartOBytes + kStaticPartLseBytes + kStaticCounterBytes +
                                       kStaticStatusBytes;
constexpr int kStaticMaxDevices = 64;

// The scratch: every GPU that loads this library holds one copy until the
// process exits.  All calls on a device share it.  Its last 256 bytes hold
// the status word the kernels OR their error bits into; it starts at zero
// (static device memory is zero-initialised) and is cleared only when
// oomattn_decode_static_scratch_status reads it.
static __device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];

std::mutex g_static_mu;
void* g_static_scratch[kStaticMaxDevices] = {};

int static_fail(char* buf, int32_t len, int code, const char* fmt, ...) {
  if (buf && len > 0) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, (size_t)len, fmt, ap);
    va_end(ap);
  }
  return code;
}

}  // namespace

extern "C" int oomattn_decode_static_scratch(int device, void* stream, int32_t kv_dtype, const void* k_pool,
                                             const void* v_pool, int32_t n_pool_pages, const int32_t* block_table,
                                             int32_t max_pages_per_seq, int32_t n_heads, int32_t n_kv_heads,
                                             float softmax_scale, int32_t n_rows, const int32_t* seq_ids,
                                             const int32_t* lens, const float* q, float* out, float* lse,
                                             char* errbuf, int32_t errbuf_len) {
  if (errbuf && errbuf_len > 0) errbuf[0] = '\0';
  if (!k_pool || !v_pool || !block_table || !seq_ids || !lens || !q || !out)
    return static_fail(errbuf, errbuf_len, OOMATTN_ERR_INVALID_ARG, "null pointer argument");
  if (kv_dtype != OOMATTN_DTYPE_F32 && kv_dtype != OOMATTN_DTYPE_BF16)
    return static_fail(errbuf, errbuf_len, OOMATTN_ERR_INVALID_ARG, "unknown kv dtype %d", kv_dtype);
  if (device < 0 || device >= kStaticMaxDevices)
    return static_fail(errbuf, errbuf_len, OOMATTN_ERR_OUT_OF_RANGE, "device %d outside [0, %d)", device,
                       kStaticMaxDevices);
  if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || n_heads / n_kv_heads > kMaxGroup)
    return static_fail(errbuf, errbuf_len, OOMATTN_ERR_BAD_CONFIG, "n_heads %d / n_kv_heads %d unsupported",
                       n_heads, n_kv_heads);
  if (n_rows <= 0 || n_rows > kMaxBatch)
    return static_fail(errbuf, errbuf_len, OOMATTN_ERR_OUT_OF_RANGE,
                       "n_rows %d outside [1, %d]: the static scratch serves at most %d rows per call", n_rows,
                       kMaxBatch, kMaxBatch);
  if (n_kv_heads > kStaticMaxKv)
    return static_fail(errbuf, errbuf_len, OOMATTN_ERR_OUT_OF_RANGE,
                       "n_kv_heads %d exceeds the static scratch's %d", n_kv_heads, kStaticMaxKv);
  if (n_pool_pages <= 0 || max_pages_per_seq <= 0 ||
      (long long)n_pool_pages * n_kv_heads * kPageSize >= (1ll << 31))
    return static_fail(errbuf, errbuf_len, OOMATTN_ERR_OUT_OF_RANGE, "pool of %d pages unsupported", n_pool_pages);
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15u)
    return static_fail(errbuf, errbuf_len, OOMATTN_ERR_INVALID_ARG, "q and out must be 16-byte aligned");
  SeqBatch sb;
  sb.n = n_rows;
  for (int z = 0; z < n_rows; ++z) {
    if (lens[z] < 0 || lens[z] > max_pages_per_seq * kPageSize)
      return static_fail(errbuf, errbuf_len, OOMATTN_ERR_OUT_OF_RANGE, "row %d: length %d outside [0, %d]", z,
                         lens[z], max_pages_per_seq * kPageSize);
    if (seq_ids[z] < 0)
      return static_fail(errbuf, errbuf_len, OOMATTN_ERR_OUT_OF_RANGE, "row %d: negative sequence id", z);
    sb.seq[z] = seq_ids[z];
    sb.len[z] = lens[z];
    sb.pos[z] = 0;
  }

  DeviceGuard dg(device);
  int num_sms = 148;
  cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, device);
  void* scratch = nullptr;
  {
    // Set-up, once per device with that device current: the array's device
    // address (its name in host code is only a host-side stand-in) and the
    // decode kernel's shared-memory limit.
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (!g_static_scratch[device]) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_decode_scratch);
      if (e != cudaSuccess || !p)
        return static_fail(errbuf, errbuf_len, OOMATTN_ERR_CUDA, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      e = cudaFuncSetAttribute(decode_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDecSmemBytes);
      if (e != cudaSuccess)
        return static_fail(errbuf, errbuf_len, OOMATTN_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      g_static_scratch[device] = p;
    }
    scratch = g_static_scratch[device];
  }
  float* part_o = reinterpret_cast<float*>(scratch);
  float* part_lse = reinterpret_cast<float*>(static_cast<unsigned char*>(scratch) + kStaticPartOBytes);
  unsigned* counters =
      reinterpret_cast<unsigned*>(static_cast<unsigned char*>(scratch) + kStaticPartOBytes + kStaticPartLseBytes);
  int* status = reinterpret_cast<int*>(static_cast<unsigned char*>(scratch) + kStaticPartOBytes +
                                       kStaticPartLseBytes + kStaticCounterBytes);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

  // Split plan as in oomattn_decode, capped so that every (row, q head, split)
  // partial fits the static array: nsplit <= slots / (rows * heads).
  const int cap_splits = std::max(1, std::min(split_cap(kv_dtype), kStaticPartSlots / (n_rows * n_heads)));
  DecodeSched sched;
  const int n_items = plan_decode(sb, n_kv_heads, num_sms * (kv_dtype == OOMATTN_DTYPE_BF16 ? kDecCtasPerSm : 3), cap_splits,
                                  kv_dtype == OOMATTN_DTYPE_BF16 ? kDecodeFillPages : kDecodeFillPagesF32, sched);
  if (n_items == 0) return OOMATTN_OK;

  // The counters must start at zero; a previous call that ended early could
  // have left some set, so they are cleared on every call.
  cudaError_t e = cudaMemsetAsync(counters, 0, (size_t)n_rows * n_kv_heads * sizeof(unsigned), st);
  if (e != cudaSuccess)
    return static_fail(errbuf, errbuf_len, OOMATTN_ERR_CUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));

  KVPool pool;
  pool.k = const_cast<void*>(k_pool);
  pool.v = const_cast<void*>(v_pool);
  pool.block_table = block_table;
  pool.max_pages_per_seq = max_pages_per_seq;
  pool.n_pool_pages = n_pool_pages;
  pool.n_kv = n_kv_heads;
  pool.kv_bf16 = kv_dtype == OOMATTN_DTYPE_BF16;
  DecodeArgs a;
  a.q = q;
  a.out = out;
  a.lse = lse;
  a.o_stride = kHeadDim;
  a.lse_stride = 1;
  a.test_flags = 0;
  a.layer = 0;
  a.n_heads = n_heads;
  a.group = n_heads / n_kv_heads;
  a.max_splits = cap_splits;
  a.qscale = (softmax_scale > 0.f ? softmax_scale : 1.0f / sqrtf((float)kHeadDim)) * 1.4426950408889634f;
  a.part_o = part_o;
  a.part_lse = part_lse;
  a.counters = counters;
  a.status = status;  // read and cleared by oomattn_decode_static_scratch_status
  a.timeout_ns = kDefaultTimeoutNs;
  if (pool.kv_bf16) {
    // Tensor maps are encoded on the host into kernel parameters: no allocation.
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return static_fail(errbuf, errbuf_len, OOMATTN_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    CUtensorMap maps[2];
    const void* bases[2] = {k_pool, v_pool};
    for (int m = 0; m < 2; ++m) {
      cuuint64_t dims[2] = {(cuuint64_t)kHeadDim, (cuuint64_t)n_pool_pages * n_kv_heads * kPageSize};
      cuuint64_t strides[1] = {(cuuint64_t)kHeadDim * 2};
      cuuint32_t box[2] = {64, (cuuint32_t)kPageSize};
      cuuint32_t estr[2] = {1, 1};
      CUresult r = enc(&maps[m], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(bases[m]), dims, strides,
                       box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS)
        return static_fail(errbuf, errbuf_len, OOMATTN_ERR_INVALID_ARG,
                           "pool pointer rejected by cuTensorMapEncodeTiled (%d): it must be 16-byte aligned", (int)r);
    }
    decode_bf16_kernel<<<n_items, (kDecWarps + 1) * 32, kDecSmemBytes, st>>>(maps[0], maps[1], pool, a, sb, sched);
  } else {
    decode_f32_kernel<<<n_items, kDecWarps * 32, 0, st>>>(pool, a, sb, sched);
  }
  e = cudaGetLastError();
  if (e != cudaSuccess)
    return static_fail(errbuf, errbuf_len, OOMATTN_ERR_CUDA, "kernel launch: %s", cudaGetErrorString(e));
  return OOMATTN_OK;
}

extern "C" int oomattn_decode_static_scratch_status(int device, void* stream, int32_t* flags_out, char* errbuf,
                                                    int32_t errbuf_len) {
  if (errbuf && errbuf_len > 0) errbuf[0] = '\0';
  if (flags_out) *flags_out = 0;
  if (device < 0 || device >= kStaticMaxDevices)
    return static_fail(errbuf, errbuf_len, OOMATTN_ERR_OUT_OF_RANGE, "device %d outside [0, %d)", device,
                       kStaticMaxDevices);
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_static_mu);
    scratch = g_static_scratch[device];
  }
  if (!scratch) return OOMATTN_OK;  // no call has run on this device
  DeviceGuard dg(device);
  int* status = reinterpret_cast<int*>(static_cast<unsigned char*>(scratch) + kStaticPartOBytes +
                                       kStaticPartLseBytes + kStaticCounterBytes);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int h = 0;
  cudaError_t e = cudaMemcpyAsync(&h, status, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && h) {
    e = cudaMemsetAsync(status, 0, sizeof(int), st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  }
  if (e != cudaSuccess)
    return static_fail(errbuf, errbuf_len, OOMATTN_ERR_CUDA, "reading the status word: %s", cudaGetErrorString(e));
  if (flags_out) *flags_out = h;
  if (h & kDevErrTimeout)
    return static_fail(errbuf, errbuf_len, OOMATTN_ERR_TIMEOUT, "a decode wait gave up (status %d)", h);
  if (h & kDevErrBounds)
    return static_fail(errbuf, errbuf_len, OOMATTN_ERR_DEVICE_CHECK,
                       "a block-table page id was outside [0, n_pool_pages) and read as the last pool page (status %d)",
                       h);
  if (h) return static_fail(errbuf, errbuf_len, OOMATTN_ERR_DEVICE_CHECK, "device check failed (status %d)", h);
  return OOMATTN_OK;
}

// ------------------------------------------------------------------ K-E: Q8 weights

extern "C" int oomattn_q8_unpack(const uint8_t* stream, uint64_t stream_bytes, int64_t n_values, uint8_t* q_out,
                                 float* scale_out, float* min_out, char* errbuf, int32_t errbuf_len) {
  auto err = [&](const char* what, long long block, long long val) {
    if (errbuf && errbuf_len > 0) snprintf(errbuf, (size_t)errbuf_len, "block %lld: %s (%lld)", block, what, val);
    return OOMATTN_ERR_INVALID_ARG;
  };
  if (!stream || !q_out || !scale_out || !min_out || n_values < 0) return err("null pointer or negative size", -1, n_values);
  // OomLoader::dequantize_tensor_into (src/quant.rs:431-463): per block
  // [f32 scale][f32 min][u32 len][len bytes], min(256, values left) values each
  uint64_t off = 0;
  int64_t pos = 0;
  for (int64_t b = 0; pos < n_values; ++b) {
    if (off > stream_bytes || stream_bytes - off < 12) return err("header past the end of the stream, offset", b, (long long)off);
    float sc, mn;
    uint32_t len;
    memcpy(&sc, stream + off, 4);
    memcpy(&mn, stream + off + 4, 4);
    memcpy(&len, stream + off + 8, 4);
    off += 12;
    const int64_t want = std::min<int64_t>(256, n_values - pos);
    if ((int64_t)len != want) return err("length is not min(256, values left), length", b, (long long)len);
    if (stream_bytes - off < len) return err("data past the end of the stream, offset", b, (long long)off);
    memcpy(q_out + pos, stream + off, len);
    scale_out[b] = sc;
    min_out[b] = mn;
    off += len;
    pos += len;
  }
  return OOMATTN_OK;
}

namespace {

int ensure_q8_scratch(oomattn_ctx* ctx, size_t bytes, int row_tiles) {
  if (bytes > ctx->q8_scratch_bytes) {
    if (ctx->d_q8_scratch) {
      cudaStreamSynchronize(ctx->stream);
      cudaFree(ctx->d_q8_scratch);
      ctx->d_q8_scratch = nullptr;
      ctx->q8_scratch_bytes = 0;
    }
    if (cudaMalloc(&ctx->d_q8_scratch, bytes) != cudaSuccess)
      return fail(ctx, OOMATTN_ERR_NO_MEMORY, "q8 scratch allocation of %zu bytes failed", bytes);
    ctx->q8_scratch_bytes = bytes;
  }
  if (row_tiles > ctx->q8_counters_n) {
    if (ctx->d_q8_counters) {
      cudaStreamSynchronize(ctx->stream);
      cudaFree(ctx->d_q8_counters);
      ctx->d_q8_counters = nullptr;
      ctx->q8_counters_n = 0;
    }
    if (cudaMalloc(&ctx->d_q8_counters, sizeof(unsigned) * row_tiles) != cudaSuccess)
      return fail(ctx, OOMATTN_ERR_NO_MEMORY, "q8 counter allocation failed");
    CK(cudaMemsetAsync(ctx->d_q8_counters, 0, sizeof(unsigned) * row_tiles, ctx->stream));
    ctx->q8_counters_n = row_tiles;
  }
  return OOMATTN_OK;
}

// The linear kernel is a programmatic dependent of the x-split kernel before
// it: it launches while that kernel runs, issues its first weight loads, and
// waits for the split only before it reads x.
template <int NT, int MT, int S, bool XA>
cudaError_t launch_q8_linear(const Q8Args& a, int row_blocks, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.splits, row_blocks);
  cfg.blockDim = dim3(kQ8Warps * 32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, q8_linear_kernel<NT, MT, S, XA>, a);
}

}  // namespace

namespace {

// One output of a Q8 pass: y = x W^T (+ bias) (+ residual).
struct Q8Job {
  const oomattn_q8_matrix* w;
  const float* bias;
  const float* residual;
  float* y;
};

int check_q8_matrix(oomattn_ctx* ctx, const oomattn_q8_matrix* w, int cols) {
  if (!w || !w->q || !w->scale || !w->min) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "null Q8 matrix pointer");
  if (w->rows <= 0 || w->cols <= 0) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad Q8 matrix shape");
  if (w->rows % 16 || w->cols % kQ8Chunk)
    return fail(ctx, OOMATTN_ERR_UNSUPPORTED, "Q8 linear needs rows %% 16 == 0 and cols %% 64 == 0 (got %d x %d)",
                w->rows, w->cols);
  if (cols >= 0 && w->cols != cols)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "Q8 matrix has %d columns, the input %d", w->cols, cols);
  if (reinterpret_cast<uintptr_t>(w->q) % 16) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "q must be 16-byte aligned");
  return OOMATTN_OK;
}

struct Q8Plan {
  int mt, row_blocks, splits, cps;
};

// Tall or large matrices use row blocks of 32 rows (two row tiles per warp
// share each x fragment), others 16 rows for more CTAs.  Split-K only when the row blocks
// alone leave SMs idle, keeping at least one chunk per warp of a CTA (more,
// shorter CTAs only add pipeline fill and merge).
Q8Plan plan_q8(const oomattn_ctx* ctx, int rows, int cols, int nt) {
  Q8Plan p;
  const int nchunks = cols / kQ8Chunk;
  // two row tiles per warp for tall matrices (gate+up at 16 tokens: 57.6
  // against 66.6 us for two 8-token CTAs per weight tile) and, at one token
  // tile, for large short ones (the down projection: 25.1 against 26.9 us at
  // one token; at 16 tokens it halves the CTAs for no gain)
  p.mt = (rows >= 64 * ctx->num_sms || (nt == 1 && (long long)rows * cols >= (32ll << 20))) ? 2 : 1;
  p.row_blocks = (rows + 16 * p.mt - 1) / (16 * p.mt);
  const int want = std::max(1, (ctx->num_sms + p.row_blocks - 1) / p.row_blocks);
  p.splits = std::max(1, std::min(want, nchunks / kQ8Warps));
  p.cps = (nchunks + p.splits - 1) / p.splits;
  p.splits = (nchunks + p.cps - 1) / p.cps;
  return p;
}

// The form with x staged in shared memory (q8_linear_xs_kernel), for passes
// the tensor-core form below does not take (with cols % 256 and rows % 128 it
// takes 9-16 tokens, and any count on a wave of row tiles): for matrices
// of at least 32 M weights, one CTA per SM over a row group of 256 * MT rows
// and a column range of 8 to 96 / NT chunks.  MT and the ranges minimise
// waves x (MT x chunks per range + kQ8XsFixed), a fixed cost for staging x,
// filling the ring and the merge in units of 256 rows x one chunk; ties go to
// fewer ranges, then to MT = 1.
//  - Two token tiles (9..16 tokens): always.  Measured at 16 tokens
//    (Qwen2.5-7B shapes, us, against the register-x form): gate+up MT 2: 51.2
//    (57.7), gate MT 1: 29.2 (30.6), down MT 1: 35.6 (41.9), LM head MT 2: 206
//    (226); MT 2 with 3- or 4-deep rings spills and loses.
//  - One token tile: only when the plan fits in one wave and gives each warp
//    at least 30 chunks, where staging x and filling the 8-deep ring are
//    amortised: gate+up 30.8 (35.7) at 1 token, 32.0 (37.4) at 8; down 20.7
//    (25.0) at 1 token.  Shorter runs lose: gate (two 28-chunk ranges) 19.3
//    against 19.4 at 1 token and 22.0 against 20.7 at 8; the LM head (4.01
//    waves) 137 against 132.
constexpr int kQ8XsFixed = 8;
struct Q8XsPlan {
  int mt, groups, splits, cps;
};
bool q8_xs_size_ok(int total_rows, int cols) {
  return (long long)total_rows * cols >= (32ll << 20) && cols / kQ8Chunk >= 8;
}
Q8XsPlan plan_q8_xs(const oomattn_ctx* ctx, const Q8Job* jobs, int n_jobs, int nchunks, int nt) {
  Q8XsPlan best{1, 0, 1, nchunks};
  long long best_cost = -1;
  for (int mt = 2; mt >= 1; --mt) {
    int groups = 0;
    for (int j = 0; j < n_jobs; ++j) groups += (jobs[j].w->rows + 256 * mt - 1) / (256 * mt);
    const int mx = q8_xs_max_chunks(nt);
    for (int s = (nchunks + mx - 1) / mx; s <= std::max(1, nchunks / 8); ++s) {
      const int cps = (nchunks + s - 1) / s;
      const int splits = (nchunks + cps - 1) / cps;
      const long long waves = ((long long)groups * splits + ctx->num_sms - 1) / ctx->num_sms;
      const long long cost = waves * (mt * cps + kQ8XsFixed);
      if (best_cost < 0 || cost < best_cost || (cost == best_cost && mt < best.mt)) {
        best_cost = cost;
        best = {mt, groups, splits, cps};
      }
    }
  }
  return best;
}

template <int NT, int MT, int S>
cudaError_t launch_q8_linear_xs(const Q8Args& a, int groups, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.splits, groups);
  cfg.blockDim = dim3(kQ8XsWarps * 32);
  cfg.dynamicSmemBytes = q8_xs_smem_bytes(NT, a.chunks_per_split);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, q8_linear_xs_kernel<NT, MT, S>, a);
}

// Runs every job (up to kQ8MaxMats, all of the same width) on the same input:
// x, or silu(x) * up when `up` is given.  Tokens run in passes of up to 16
// (two MMA token tiles; each weight byte is read once per pass): one x split
// per pass, then one linear launch over all jobs' row blocks, a programmatic
// dependent of the split.
// The tensor-core form of a decode-sized pass (q8_tc_kernel) for large
// matrices: rows in tiles of 128, all of a launch's matrices' tiles in one
// persistent grid of at most one CTA per SM, each CTA an equal range of the
// (row tile, 256-column block) units.  It takes passes of 9 or more tokens,
// and passes of any size over matrices of at least a wave of row tiles (the
// gate/up pair, the LM head); a smaller matrix with few tokens leaves each
// CTA too little to stream and stays on the CUDA-core form.
#ifndef OOMATTN_Q8_TC_MIN_TOKENS
#define OOMATTN_Q8_TC_MIN_TOKENS 9
#endif
constexpr int kQ8TcMinTokens = OOMATTN_Q8_TC_MIN_TOKENS;
struct Q8TcPlan {
  int row_tiles, units, grid;
};
bool q8_tc_fits(const Q8Job* jobs, int n_jobs, int total_rows, int cols) {
  if (!q8_xs_size_ok(total_rows, cols) || cols % 256 || cols > 256 * kTcMaxBlocks) return false;
  for (int j = 0; j < n_jobs; ++j)
    if (jobs[j].w->rows % kTcRows) return false;
  return true;
}
Q8TcPlan plan_q8_tc(const oomattn_ctx* ctx, int total_rows, int cols) {
  Q8TcPlan p;
  p.row_tiles = total_rows / kTcRows;
  p.units = p.row_tiles * (cols / 256);
  p.grid = std::max(1, std::min(ctx->num_sms, p.units));
  return p;
}

int launch_q8_tc(oomattn_ctx* ctx, const Q8Job* jobs, int n_jobs, int cols, int t0, int nt, const uint8_t* digits,
                 const float* xsum, const float* sx, float* part, int total_rows) {
  const Q8TcPlan p = plan_q8_tc(ctx, total_rows, cols);
  CUtensorMap wm[kTcMaxMats], dm;
  int rc = encode_2d(ctx, digits, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, cols, kTcDigitRows, kTcCols, kTcDigitRows, &dm);
  if (rc) return rc;
  Q8TcArgs a;
  memset(&a, 0, sizeof(a));
  a.n_mats = n_jobs;
  a.cols = cols;
  a.xsum = xsum;
  a.sx = sx;
  a.n_tokens = nt;
  a.units = p.units;
  a.part = part;
  a.counters = ctx->d_q8_counters;
  a.status = ctx->d_status;
  a.timeout_ns = ctx->timeout_ns;
  a.test_flags = ctx->test_flags;
  int tiles = 0;
  for (int j = 0; j < n_jobs; ++j) {
    const oomattn_q8_matrix* w = jobs[j].w;
    rc = encode_2d(ctx, w->q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, cols, w->rows, kTcCols, kTcRows, &wm[j]);
    if (rc) return rc;
    Q8TcMat& m = a.m[j];
    m.scale = w->scale;
    m.min = w->min;
    m.rows = w->rows;
    m.rb_begin = tiles;
    m.bias = jobs[j].bias;
    m.residual = jobs[j].residual ? jobs[j].residual + (size_t)t0 * w->rows : nullptr;
    m.y = jobs[j].y + (size_t)t0 * w->rows;
    tiles += w->rows / kTcRows;
  }
  for (int j = n_jobs; j < kTcMaxMats; ++j) wm[j] = wm[0];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = kTcSmemBytes;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t le = cudaLaunchKernelEx(&cfg, q8_tc_kernel, wm[0], wm[1], wm[2], dm, a);
  if (le != cudaSuccess) return fail(ctx, OOMATTN_ERR_CUDA, "q8 tensor-core pass launch: %s", cudaGetErrorString(le));
  return OOMATTN_OK;
}

// Prefill-sized Q8 linears on the tensor cores (K-F): the input is normalised
// (rmsnorm_kernel) when norm_w is given and split into fp16 hi/lo planes with
// its block sums once; each matrix is converted to fp16 with its scales and
// minima transposed, then multiplied with the block promotion.  Above this
// many tokens the weight conversion costs less than re-reading the weights
// once per 16-token pass of K-E.
constexpr int kKfQ8MinTokens = 64;

bool kf_q8_fits(const Q8Job* jobs, int n_jobs) {
  for (int j = 0; j < n_jobs; ++j) {
    const Q8Job& jb = jobs[j];
    if (jb.w->cols % kKfQ8Block || jb.w->rows % 4) return false;
    const uintptr_t al = reinterpret_cast<uintptr_t>(jb.y) | reinterpret_cast<uintptr_t>(jb.bias) |
                         reinterpret_cast<uintptr_t>(jb.residual);
    if (al & 15) return false;
  }
  return true;
}

int kf_linear_q8(oomattn_ctx* ctx, const Q8Job* jobs, int n_jobs, const float* x, const float* up, int m,
                 const float* norm_w, float eps) {
  const int k = jobs[0].w->cols;
  size_t wmax = 0;
  for (int j = 0; j < n_jobs; ++j) wmax = std::max(wmax, (size_t)jobs[j].w->rows * k);
  const size_t xnb = norm_w ? align256((size_t)m * k * 4) : 0, xb = align256((size_t)m * k * 2);
  const size_t sb = align256((size_t)m * (k / kKfQ8Block) * 4), wb = align256(wmax * 2);
  const size_t tb = align256(wmax / kKfQ8Block * 4);
  int rc;
  uint8_t* sc = kf_scratch(ctx, xnb + 2 * xb + sb + wb + 2 * tb, &rc);
  if (rc) return rc;
  float* xn = reinterpret_cast<float*>(sc);
  uint16_t* xh = reinterpret_cast<uint16_t*>(sc + xnb);
  uint16_t* xl = reinterpret_cast<uint16_t*>(sc + xnb + xb);
  float* xsum = reinterpret_cast<float*>(sc + xnb + 2 * xb);
  uint16_t* w16 = reinterpret_cast<uint16_t*>(sc + xnb + 2 * xb + sb);
  float* st = reinterpret_cast<float*>(sc + xnb + 2 * xb + sb + wb);
  float* mt = reinterpret_cast<float*>(sc + xnb + 2 * xb + sb + wb + tb);
  if (norm_w) {
    rmsnorm_kernel<<<m, kNormThreads, 0, ctx->stream>>>(x, norm_w, eps, k, xn);
    CKLAUNCH();
    x = xn;
  }
  const long long warps = (long long)m * (k / kKfQ8Block);
  kf_prep_x16_kernel<<<(unsigned)std::min<long long>((warps + 7) / 8, (long long)ctx->num_sms * 16), 256, 0,
                       ctx->stream>>>(x, up, xh, xl, xsum, m, k, ctx->d_status);
  CKLAUNCH();
  for (int j = 0; j < n_jobs; ++j) {
    const oomattn_q8_matrix* w = jobs[j].w;
    kf_prep_w8_kernel<<<ctx->num_sms * 8, 256, 0, ctx->stream>>>(w->q, w->scale, w->min, w16, st, mt, w->rows, k);
    CKLAUNCH();
    rc = kf_launch<true, 1>(ctx, m, w->rows, k, xh, xl, w16, nullptr, jobs[j].bias, jobs[j].residual, jobs[j].y, st,
                            mt, xsum);
    if (rc) return rc;
  }
  return OOMATTN_OK;
}

int q8_run(oomattn_ctx* ctx, const Q8Job* jobs, int n_jobs, const float* x, const float* up, int n_tokens,
           const float* norm_w = nullptr, float eps = 0.f) {
  if (!x || n_tokens < 0) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad Q8 input");
  if (reinterpret_cast<uintptr_t>(x) % 16 || (up && reinterpret_cast<uintptr_t>(up) % 16) ||
      (norm_w && reinterpret_cast<uintptr_t>(norm_w) % 16))
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "x must be 16-byte aligned");
  if (n_jobs < 1 || n_jobs > kQ8MaxMats) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad Q8 job count");
  const int cols = jobs[0].w ? jobs[0].w->cols : 0;
  int total_rows = 0;
  for (int j = 0; j < n_jobs; ++j) {
    int rc = check_q8_matrix(ctx, jobs[j].w, cols);
    if (rc) return rc;
    if (!jobs[j].y) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "null Q8 output");
    total_rows += jobs[j].w->rows;
  }
  // all jobs run in one launch per pass, planned on their rows together
  size_t part_floats = 0;
  int max_blocks = 1;
  for (int nt = 1; nt <= 2; ++nt) {
    const Q8Plan p = plan_q8(ctx, total_rows, cols, nt);
    int blocks = 0;
    for (int j = 0; j < n_jobs; ++j) blocks += (jobs[j].w->rows + 16 * p.mt - 1) / (16 * p.mt);
    part_floats = std::max(part_floats, (size_t)p.splits * 8 * nt * total_rows);
    max_blocks = std::max(max_blocks, blocks);
    if (q8_xs_size_ok(total_rows, cols)) {
      const Q8XsPlan xp = plan_q8_xs(ctx, jobs, n_jobs, cols / kQ8Chunk, nt);
      part_floats = std::max(part_floats, (size_t)xp.splits * 8 * nt * total_rows);
      max_blocks = std::max(max_blocks, xp.groups);
    }
  }
  const bool tc_fits = q8_tc_fits(jobs, n_jobs, total_rows, cols);
  bool tc_wide = false;  // a wave of row tiles or more
  if (tc_fits) {
    const Q8TcPlan tp = plan_q8_tc(ctx, total_rows, cols);
    tc_wide = tp.row_tiles >= ctx->num_sms;
    part_floats = std::max(part_floats, (size_t)tp.grid * 2 * 16 * kTcRows);
    max_blocks = std::max(max_blocks, tp.row_tiles);
  }
  if (n_tokens == 0) return OOMATTN_OK;
  if (n_tokens > kKfQ8MinTokens && ctx->kf_q8_regs == kKfLaunchRegs && kf_q8_fits(jobs, n_jobs))
    return kf_linear_q8(ctx, jobs, n_jobs, x, up, n_tokens, norm_w, eps);
  const int group = 16;
  const int nchunks = cols / kQ8Chunk;
  const size_t xw = (size_t)group * (cols / 2);
  const size_t bytes = 2 * xw * 4 + (size_t)group * nchunks * 4 + (size_t)group * (cols / 256) * 4 +
                       part_floats * 4 + 256;
  int rc = ensure_q8_scratch(ctx, bytes, max_blocks);
  if (rc) return rc;
  uint32_t* xh = reinterpret_cast<uint32_t*>(ctx->d_q8_scratch);
  uint32_t* xl = xh + xw;
  float* xsum = reinterpret_cast<float*>(xl + xw);
  float* sx = xsum + (size_t)group * nchunks;  // [16][cols / 256], the integer form's digit scales
  float* part = sx + (size_t)group * (cols / 256);
  for (int t0 = 0; t0 < n_tokens; t0 += group) {
    const int nt = std::min(group, n_tokens - t0);
    if (tc_fits && (nt >= kQ8TcMinTokens || tc_wide)) {
      // the integer tensor-core pass: x as digits (the 64 x cols bytes over the xh/xl area)
      uint8_t* digits = reinterpret_cast<uint8_t*>(xh);
      const dim3 dgrid(16, (cols / 256 + kDigitBlocksPerCta - 1) / kDigitBlocksPerCta);
      const cudaError_t de =
          launch_pdl(q8_digits_kernel, dgrid, dim3(256), 0, ctx->stream, x + (size_t)t0 * cols,
                     up ? up + (size_t)t0 * cols : nullptr, norm_w, eps, nt, cols, digits, xsum, sx, ctx->d_status);
      if (de != cudaSuccess) return fail(ctx, OOMATTN_ERR_CUDA, "digit split launch: %s", cudaGetErrorString(de));
      rc = launch_q8_tc(ctx, jobs, n_jobs, cols, t0, nt, digits, xsum, sx, part, total_rows);
      if (rc) return rc;
      continue;
    }
    if (norm_w) {
      const dim3 ngrid(nt, (nchunks + kNormThreads / 32 - 1) / (kNormThreads / 32));
      rmsnorm_prep_x_kernel<<<ngrid, kNormThreads, 0, ctx->stream>>>(x + (size_t)t0 * cols, norm_w, eps, cols, xh,
                                                                     xl, xsum, ctx->d_status);
    } else {
      const long long prep_warps = (long long)nt * nchunks;
      q8_prep_x_kernel<<<(unsigned)((prep_warps + 7) / 8), 256, 0, ctx->stream>>>(
          x + (size_t)t0 * cols, up ? up + (size_t)t0 * cols : nullptr, nt, cols, xh, xl, xsum, ctx->d_status);
    }
    CKLAUNCH();
    const int ntiles = nt > 8 ? 2 : 1;
    const Q8Plan p = plan_q8(ctx, total_rows, cols, ntiles);
    Q8XsPlan xp{p.mt, 0, p.splits, p.cps};
    bool xs = false;
    if (q8_xs_size_ok(total_rows, cols)) {
      const Q8XsPlan t = plan_q8_xs(ctx, jobs, n_jobs, nchunks, ntiles);
      xs = ntiles == 2 || ((long long)t.groups * t.splits <= ctx->num_sms && t.cps >= 30);
      if (xs) xp = t;
    }
    const int rows_per_block = xs ? 256 * xp.mt : 16 * p.mt;
    Q8Args a;
    memset(&a, 0, sizeof(a));
    a.n_mats = n_jobs;
    a.cols = cols;
    a.xh = xh;
    a.xl = xl;
    a.xsum = xsum;
    a.n_tokens = nt;
    a.counters = ctx->d_q8_counters;
    a.splits = xp.splits;
    a.chunks_per_split = xp.cps;
    a.status = ctx->d_status;
    int blocks = 0;
    size_t row_prefix = 0;
    for (int j = 0; j < n_jobs; ++j) {
      const oomattn_q8_matrix* w = jobs[j].w;
      Q8Mat& m = a.m[j];
      m.q = w->q;
      m.scale = w->scale;
      m.min = w->min;
      m.rows = w->rows;
      m.rb_begin = blocks;
      m.bias = jobs[j].bias;
      m.residual = jobs[j].residual ? jobs[j].residual + (size_t)t0 * w->rows : nullptr;
      m.y = jobs[j].y + (size_t)t0 * w->rows;
      m.part = part + (size_t)xp.splits * 8 * ntiles * row_prefix;  // [splits][8 NT][rows]
      blocks += (w->rows + rows_per_block - 1) / rows_per_block;
      row_prefix += w->rows;
    }
    // one token tile: x read a chunk ahead; two: x read at use, with a 3-deep
    // weight ring for one row tile and a 2-deep one for two
    const cudaError_t le =
        xs ? (ntiles == 2 ? (xp.mt == 2 ? launch_q8_linear_xs<2, 2, 2>(a, blocks, ctx->stream)
                                        : launch_q8_linear_xs<2, 1, 4>(a, blocks, ctx->stream))
                          : (xp.mt == 2 ? launch_q8_linear_xs<1, 2, kQ8Xs1S2>(a, blocks, ctx->stream)
                                        : launch_q8_linear_xs<1, 1, kQ8Xs1S1>(a, blocks, ctx->stream)))
                           : ntiles == 2 ? (p.mt == 2 ? launch_q8_linear<2, 2, 2, false>(a, blocks, ctx->stream)
                                                    : launch_q8_linear<2, 1, 3, false>(a, blocks, ctx->stream))
                           : p.mt == 2 ? launch_q8_linear<1, 2, 2, true>(a, blocks, ctx->stream)
                                       : launch_q8_linear<1, 1, 2, true>(a, blocks, ctx->stream);
    if (le != cudaSuccess) return fail(ctx, OOMATTN_ERR_CUDA, "q8_linear launch: %s", cudaGetErrorString(le));
  }
  return OOMATTN_OK;
}

// Per-context buffers of the layer step (grown on demand).
float* layer_scratch(oomattn_ctx* ctx, size_t floats, int* rc) {
  if (floats * 4 > ctx->layer_scratch_bytes) {
    if (ctx->d_layer_scratch) {
      cudaStreamSynchronize(ctx->stream);
      cudaFree(ctx->d_layer_scratch);
      ctx->d_layer_scratch = nullptr;
      ctx->layer_scratch_bytes = 0;
    }
    if (cudaMalloc(&ctx->d_layer_scratch, floats * 4) != cudaSuccess) {
      *rc = fail(ctx, OOMATTN_ERR_NO_MEMORY, "layer scratch allocation of %zu bytes failed", floats * 4);
      return nullptr;
    }
    ctx->layer_scratch_bytes = floats * 4;
  }
  *rc = OOMATTN_OK;
  return ctx->d_layer_scratch;
}

int run_rmsnorm(oomattn_ctx* ctx, const float* x, const float* w, float eps, int n_tokens, int hidden, float* out) {
  if (!x || !w || !out || n_tokens < 0 || hidden <= 0) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad rmsnorm arguments");
  if (hidden % 4 || !aligned16(x) || !aligned16(w) || !aligned16(out))
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "rmsnorm needs hidden %% 4 == 0 and 16-byte aligned rows");
  if (n_tokens == 0) return OOMATTN_OK;
  rmsnorm_kernel<<<n_tokens, kNormThreads, 0, ctx->stream>>>(x, w, eps, hidden, out);
  CKLAUNCH();
  return OOMATTN_OK;
}

}  // namespace

extern "C" int oomattn_q8_linear(oomattn_ctx* ctx, const oomattn_q8_matrix* w, const float* x, int32_t n_tokens,
                                 const float* bias, float* y) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  if (!y) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "null pointer");
  DeviceGuard dg(ctx->device);
  const Q8Job job{w, bias, nullptr, y};
  return q8_run(ctx, &job, 1, x, nullptr, n_tokens);
}

extern "C" int oomattn_rmsnorm(oomattn_ctx* ctx, const float* x, const float* weight, float eps, int32_t n_tokens,
                               int32_t hidden, float* out) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  DeviceGuard dg(ctx->device);
  return run_rmsnorm(ctx, x, weight, eps, n_tokens, hidden, out);
}

extern "C" int oomattn_q8_mlp(oomattn_ctx* ctx, const oomattn_q8_matrix* gate, const oomattn_q8_matrix* up,
                              const oomattn_q8_matrix* down, const float* x, int32_t n_tokens, const float* residual,
                              float* y) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  if (!gate || !up || !down || !y) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "null pointer");
  if (gate->rows != up->rows || gate->cols != up->cols || down->cols != gate->rows || down->rows != gate->cols)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "MLP shapes disagree: gate %dx%d, up %dx%d, down %dx%d", gate->rows,
                gate->cols, up->rows, up->cols, down->rows, down->cols);
  if (n_tokens <= 0) return n_tokens == 0 ? OOMATTN_OK : fail(ctx, OOMATTN_ERR_INVALID_ARG, "negative n_tokens");
  DeviceGuard dg(ctx->device);
  int rc;
  const size_t inter = (size_t)gate->rows;
  float* g = layer_scratch(ctx, 2 * inter * n_tokens + 64, &rc);
  if (rc) return rc;
  float* u = g + inter * n_tokens + 32;  // 128-byte offset keeps both 16-byte aligned
  const Q8Job gu[2] = {{gate, nullptr, nullptr, g}, {up, nullptr, nullptr, u}};
  rc = q8_run(ctx, gu, 2, x, nullptr, n_tokens);
  if (rc) return rc;
  const Q8Job dn{down, nullptr, residual, y};
  return q8_run(ctx, &dn, 1, g, u, n_tokens);
}

extern "C" int oomattn_decoder_layer_q8(oomattn_ctx* ctx, int32_t layer, int32_t n_seqs, const int32_t* seq_ids,
                                        const float* x, const oomattn_q8_layer* w, float* out) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  if (!seq_ids || !x || !w || !out || n_seqs <= 0)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad decoder_layer_q8 arguments");
  const int H = ctx->cfg.hidden_size, hq = ctx->cfg.n_heads, hkv = ctx->cfg.n_kv_heads;
  const int nq = hq * kHeadDim, nkv = hkv * kHeadDim;
  if (w->q.rows != nq || w->k.rows != nkv || w->v.rows != nkv || w->q.cols != H || w->k.cols != H ||
      w->v.cols != H || w->o.rows != H || w->o.cols != nq || w->gate.cols != H || w->up.cols != H ||
      w->up.rows != w->gate.rows || w->down.rows != H || w->down.cols != w->gate.rows)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "decoder_layer_q8 weight shapes do not match the configuration");
  if (!w->input_norm || !w->post_norm) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "null norm weights");
  int rc = check_layer(ctx, layer);
  if (rc) return rc;
  DeviceGuard dg(ctx->device);
  const size_t B = (size_t)n_seqs, inter = (size_t)w->gate.rows;
  // scratch: q, k, v, rotated q, attention output, residual stream h
  const size_t need = B * (H + 3 * nq + 2 * nkv) + 8 * 32;
  float* sb = layer_scratch(ctx, need + 2 * inter * B + 64, &rc);
  if (rc) return rc;
  auto carve = [&](size_t n) {
    float* p = sb;
    sb += (n + 31) / 32 * 32;  // 128-byte aligned pieces
    return p;
  };
  float* q = carve(B * nq);
  float* k = carve(B * nkv);
  float* v = carve(B * nkv);
  float* qr = carve(B * nq);
  float* att = carve(B * nq);
  float* h = carve(B * H);
  float* g = carve(B * inter);
  float* u = carve(B * inter);
  // GhostDecoderLayer::forward_turbo (src/oomllama.rs:387-402): h = x + attn(norm(x)); out = h + mlp(norm(h))
  // (the RMSNorms run inside the x splits of the linears that read them)
  const Q8Job qkv[3] = {{&w->q, w->bq, nullptr, q}, {&w->k, w->bk, nullptr, k}, {&w->v, w->bv, nullptr, v}};
  rc = q8_run(ctx, qkv, 3, x, nullptr, n_seqs, w->input_norm, w->eps);
  if (rc) return rc;
  rc = oomattn_rope_append(ctx, layer, n_seqs, seq_ids, 1, q, k, v, OOMATTN_DTYPE_F32, nullptr, nullptr, nullptr, qr,
                           OOMATTN_DTYPE_F32);
  if (rc) return rc;
  rc = oomattn_decode(ctx, layer, n_seqs, seq_ids, nullptr, qr, att, nullptr);
  if (rc) return rc;
  const Q8Job o{&w->o, nullptr, x, h};
  rc = q8_run(ctx, &o, 1, att, nullptr, n_seqs);
  if (rc) return rc;
  const Q8Job gu[2] = {{&w->gate, nullptr, nullptr, g}, {&w->up, nullptr, nullptr, u}};
  rc = q8_run(ctx, gu, 2, h, nullptr, n_seqs, w->post_norm, w->eps);
  if (rc) return rc;
  const Q8Job dn{&w->down, nullptr, h, out};
  return q8_run(ctx, &dn, 1, g, u, n_seqs);
}

extern "C" int oomattn_embed_q8(oomattn_ctx* ctx, const oomattn_q8_matrix* emb, const int32_t* token_ids,
                                int32_t n_tokens, float* out) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  if (!emb || !emb->q || !emb->scale || !emb->min || !token_ids || !out || n_tokens < 0 || emb->rows <= 0 ||
      emb->cols <= 0)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad embed_q8 arguments");
  if (n_tokens == 0) return OOMATTN_OK;
  DeviceGuard dg(ctx->device);
  embed_q8_kernel<<<n_tokens, 256, 0, ctx->stream>>>(emb->q, emb->scale, emb->min, emb->rows, emb->cols, token_ids,
                                                     out, ctx->d_status);
  CKLAUNCH();
  return OOMATTN_OK;
}

extern "C" int oomattn_argmax(oomattn_ctx* ctx, const float* logits, int32_t n_rows, int32_t n, int32_t* ids) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  if (!logits || !ids || n_rows < 0 || n <= 0) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad argmax arguments");
  if (n_rows == 0) return OOMATTN_OK;
  DeviceGuard dg(ctx->device);
  // about 4 CTAs per SM over all rows, at least 2048 logits per CTA
  const int want = std::max(1, (4 * ctx->num_sms + n_rows - 1) / n_rows);
  const int chunks = std::max(1, std::min({want, (n + 2047) / 2048, 1024}));
  const int chunk = (n + chunks - 1) / chunks;
  const int n_chunks = (n + chunk - 1) / chunk;
  const size_t need = (size_t)n_rows * n_chunks * 8;
  if (need > ctx->argmax_part_bytes) {
    if (ctx->d_argmax_part) {
      cudaStreamSynchronize(ctx->stream);
      cudaFree(ctx->d_argmax_part);
      ctx->d_argmax_part = nullptr;
      ctx->argmax_part_bytes = 0;
    }
    if (cudaMalloc(&ctx->d_argmax_part, need) != cudaSuccess)
      return fail(ctx, OOMATTN_ERR_NO_MEMORY, "argmax scratch allocation of %zu bytes failed", need);
    ctx->argmax_part_bytes = need;
  }
  float* pv = static_cast<float*>(ctx->d_argmax_part);
  int* pi = reinterpret_cast<int*>(pv + (size_t)n_rows * n_chunks);
  argmax_partial_kernel<<<dim3(n_chunks, n_rows), kArgmaxThreads, 0, ctx->stream>>>(logits, n, chunk, pv, pi);
  CKLAUNCH();
  argmax_final_kernel<<<n_rows, kArgmaxThreads, 0, ctx->stream>>>(logits, n, n_chunks, pv, pi, ids);
  CKLAUNCH();
  return OOMATTN_OK;
}

extern "C" int oomattn_decode_step_q8(oomattn_ctx* ctx, const oomattn_q8_model* m, int32_t n_seqs,
                                      const int32_t* seq_ids, const int32_t* tokens, int32_t* next, float* logits) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  if (!m || !m->layers || !seq_ids || !tokens || !next || n_seqs <= 0)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad decode_step_q8 arguments");
  if (m->n_layers <= 0 || m->n_layers > ctx->cfg.n_layers)
    return fail(ctx, OOMATTN_ERR_OUT_OF_RANGE, "model has %d layers, the context %d", m->n_layers, ctx->cfg.n_layers);
  const int H = ctx->cfg.hidden_size;
  if (m->embed.cols != H || m->lm_head.cols != H || !m->final_norm)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "embedding / LM head width or final norm does not match hidden %d", H);
  DeviceGuard dg(ctx->device);
  const size_t B = (size_t)n_seqs, vocab = (size_t)m->lm_head.rows;
  const size_t xf = (B * H + 31) / 32 * 32;
  const size_t need = (2 * xf + (logits ? 0 : B * vocab) + 64) * 4;
  if (need > ctx->model_scratch_bytes) {
    if (ctx->d_model_scratch) {
      cudaStreamSynchronize(ctx->stream);
      cudaFree(ctx->d_model_scratch);
      ctx->d_model_scratch = nullptr;
      ctx->model_scratch_bytes = 0;
    }
    if (cudaMalloc(&ctx->d_model_scratch, need) != cudaSuccess)
      return fail(ctx, OOMATTN_ERR_NO_MEMORY, "model scratch allocation of %zu bytes failed", need);
    ctx->model_scratch_bytes = need;
  }
  float* xa = ctx->d_model_scratch;
  float* xb = xa + xf;
  float* lg = logits ? logits : xb + xf;
  // OomLlamaModel::forward_turbo (src/oomllama.rs:504-553) for one new token per sequence, then the greedy
  // pick of the generation loop (:973-976, :1000-1003)
  int rc = oomattn_embed_q8(ctx, &m->embed, tokens, n_seqs, xa);
  if (rc) return rc;
  for (int l = 0; l < m->n_layers; ++l) {
    rc = oomattn_decoder_layer_q8(ctx, l, n_seqs, seq_ids, xa, &m->layers[l], xb);
    if (rc) return rc;
    std::swap(xa, xb);
  }
  const Q8Job head{&m->lm_head, nullptr, nullptr, lg};
  rc = q8_run(ctx, &head, 1, xa, nullptr, n_seqs, m->final_norm, m->eps);
  if (rc) return rc;
  return oomattn_argmax(ctx, lg, n_seqs, (int)vocab, next);
}

extern "C" int oomattn_prefill_step_q8(oomattn_ctx* ctx, const oomattn_q8_model* m, int32_t n_seqs,
                                       const int32_t* seq_ids, int32_t n_new, const int32_t* tokens, int32_t* next,
                                       float* logits) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  if (!m || !m->layers || !seq_ids || !tokens || !next || n_seqs <= 0 || n_new <= 0)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad prefill_step_q8 arguments");
  if (m->n_layers <= 0 || m->n_layers > ctx->cfg.n_layers)
    return fail(ctx, OOMATTN_ERR_OUT_OF_RANGE, "model has %d layers, the context %d", m->n_layers, ctx->cfg.n_layers);
  if (ctx->cfg.kv_dtype != OOMATTN_DTYPE_BF16)
    return fail(ctx, OOMATTN_ERR_UNSUPPORTED, "the model prefill runs the tensor-core attention: bf16 cache needed");
  const int H = ctx->cfg.hidden_size, hq = ctx->cfg.n_heads, hkv = ctx->cfg.n_kv_heads;
  const int nq = hq * kHeadDim, nkv = hkv * kHeadDim;
  if (m->embed.cols != H || m->lm_head.cols != H || !m->final_norm)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "embedding / LM head width or final norm does not match hidden %d", H);
  for (int l = 0; l < m->n_layers; ++l) {
    const oomattn_q8_layer* w = &m->layers[l];
    if (w->q.rows != nq || w->k.rows != nkv || w->v.rows != nkv || w->q.cols != H || w->k.cols != H ||
        w->v.cols != H || w->o.rows != H || w->o.cols != nq || w->gate.cols != H || w->up.cols != H ||
        w->up.rows != w->gate.rows || w->down.rows != H || w->down.cols != w->gate.rows || !w->input_norm ||
        !w->post_norm)
      return fail(ctx, OOMATTN_ERR_INVALID_ARG, "layer %d: weight shapes do not match the configuration", l);
  }
  DeviceGuard dg(ctx->device);
  const size_t T = (size_t)n_seqs * n_new, B = (size_t)n_seqs, vocab = (size_t)m->lm_head.rows;
  const size_t inter = (size_t)m->layers[0].gate.rows;
  auto up32 = [](size_t n) { return (n + 31) / 32 * 32; };  // 128-byte aligned pieces
  // model scratch: the residual stream (two buffers), the last token of each sequence, the logits
  const size_t need_m = (2 * up32(T * H) + up32(B * H) + (logits ? 0 : up32(B * vocab)) + 64) * 4;
  if (need_m > ctx->model_scratch_bytes) {
    if (ctx->d_model_scratch) {
      cudaStreamSynchronize(ctx->stream);
      cudaFree(ctx->d_model_scratch);
      ctx->d_model_scratch = nullptr;
      ctx->model_scratch_bytes = 0;
    }
    if (cudaMalloc(&ctx->d_model_scratch, need_m) != cudaSuccess)
      return fail(ctx, OOMATTN_ERR_NO_MEMORY, "model scratch allocation of %zu bytes failed", need_m);
    ctx->model_scratch_bytes = need_m;
  }
  float* xa = ctx->d_model_scratch;
  float* xb = xa + up32(T * H);
  float* xlast = xb + up32(T * H);
  float* lg = logits ? logits : xlast + up32(B * H);
  // layer scratch: q, k, v, rotated q (bf16), attention output, h, gate, up
  int rc;
  float* sb = layer_scratch(ctx, up32(T * nq) * 3 + up32(T * nkv) * 2 + up32(T * nq / 2) + up32(T * H) +
                                     2 * up32(T * inter) + 64, &rc);
  if (rc) return rc;
  auto carve = [&](size_t n) {
    float* p = sb;
    sb += up32(n);
    return p;
  };
  float* q = carve(T * nq);
  float* k = carve(T * nkv);
  float* v = carve(T * nkv);
  uint16_t* qr = reinterpret_cast<uint16_t*>(carve(T * nq / 2 + 1));
  float* att = carve(T * nq);
  float* h = carve(T * H);
  float* g = carve(T * inter);
  float* u = carve(T * inter);
  // OomLlamaModel::forward_turbo (src/oomllama.rs:504-553) over a prompt of n_new tokens per sequence:
  // every token's K/V enters each layer's cache, attention is causal over the sequence (K-C), and the
  // last token's logits give the first greedy pick (src/oomllama.rs:969-976)
  rc = oomattn_embed_q8(ctx, &m->embed, tokens, (int32_t)T, xa);
  if (rc) return rc;
  for (int l = 0; l < m->n_layers; ++l) {
    const oomattn_q8_layer* w = &m->layers[l];
    const Q8Job qkv[3] = {{&w->q, w->bq, nullptr, q}, {&w->k, w->bk, nullptr, k}, {&w->v, w->bv, nullptr, v}};
    rc = q8_run(ctx, qkv, 3, xa, nullptr, (int)T, w->input_norm, w->eps);
    if (rc) return rc;
    rc = oomattn_rope_append(ctx, l, n_seqs, seq_ids, n_new, q, k, v, OOMATTN_DTYPE_F32, nullptr, nullptr, nullptr,
                             qr, OOMATTN_DTYPE_BF16);
    if (rc) return rc;
    for (int b = 0; b < n_seqs; ++b) {
      rc = oomattn_prefill(ctx, l, seq_ids[b], n_new, qr + (size_t)b * n_new * nq, att + (size_t)b * n_new * nq,
                           OOMATTN_DTYPE_F32, nullptr);
      if (rc) return rc;
    }
    const Q8Job o{&w->o, nullptr, xa, h};
    rc = q8_run(ctx, &o, 1, att, nullptr, (int)T);
    if (rc) return rc;
    const Q8Job gu[2] = {{&w->gate, nullptr, nullptr, g}, {&w->up, nullptr, nullptr, u}};
    rc = q8_run(ctx, gu, 2, h, nullptr, (int)T, w->post_norm, w->eps);
    if (rc) return rc;
    const Q8Job dn{&w->down, nullptr, h, xb};
    rc = q8_run(ctx, &dn, 1, g, u, (int)T);
    if (rc) return rc;
    std::swap(xa, xb);
  }
  // the last prompt token of each sequence
  CK(cudaMemcpy2DAsync(xlast, (size_t)H * 4, xa + (size_t)(n_new - 1) * H, (size_t)n_new * H * 4, (size_t)H * 4, B,
                       cudaMemcpyDeviceToDevice, ctx->stream));
  const Q8Job head{&m->lm_head, nullptr, nullptr, lg};
  rc = q8_run(ctx, &head, 1, xlast, nullptr, n_seqs, m->final_norm, m->eps);
  if (rc) return rc;
  return oomattn_argmax(ctx, lg, n_seqs, (int)vocab, next);
}

// ------------------------------------------------------------------ .oom files
namespace {
bool rd_u32(const uint8_t* f, uint64_t bytes, uint64_t off, uint32_t* v) {
  if (off + 4 > bytes) return false;
  memcpy(v, f + off, 4);  // little endian, as the writer stores it
  return true;
}
}  // namespace

// OomLoader::load's metadata scan (src/quant.rs:320-367) over a file image,
// with every field and block bounds-checked (the reference stops silently at
// a truncated tensor; here that is an error).
extern "C" int oomattn_oom_scan(const uint8_t* file, uint64_t bytes, oomattn_oom_tensor* out, int32_t max_tensors,
                                int32_t* n_tensors, char* errbuf, int32_t errbuf_len) {
  auto bad = [&](const char* fmt, long long a, long long b) {
    if (errbuf && errbuf_len > 0) snprintf(errbuf, (size_t)errbuf_len, fmt, a, b);
    return OOMATTN_ERR_INVALID_ARG;
  };
  if (!file || !n_tensors || (max_tensors > 0 && !out)) return bad("null argument (%lld %lld)", 0, 0);
  if (bytes < 12 || memcmp(file, "OOML", 4) != 0) return bad("not an .oom file (%lld bytes, magic %lld)", (long long)bytes, 0);
  uint32_t version = 0, count = 0;
  rd_u32(file, bytes, 4, &version);
  rd_u32(file, bytes, 8, &count);
  *n_tensors = (int32_t)count;
  uint64_t off = 12;
  for (uint32_t t = 0; t < count; ++t) {
    uint32_t name_len = 0, num_blocks = 0, total = 0;
    if (!rd_u32(file, bytes, off, &name_len) || off + 4 + name_len + 9 > bytes)
      return bad("tensor %lld: header past the end of the file (offset %lld)", t, (long long)off);
    const uint64_t name_off = off + 4;
    off = name_off + name_len;
    const uint8_t qt = file[off];
    off += 1;
    rd_u32(file, bytes, off, &num_blocks);
    rd_u32(file, bytes, off + 4, &total);
    off += 8;
    const uint64_t data_off = off;
    for (uint32_t b = 0; b < num_blocks; ++b) {
      uint32_t len = 0;
      if (!rd_u32(file, bytes, off + 8, &len) || off + 12 + (uint64_t)len > bytes)
        return bad("tensor %lld: block %lld past the end of the file", t, b);
      off += 12 + (uint64_t)len;
    }
    if ((int32_t)t < max_tensors) {
      oomattn_oom_tensor& m = out[t];
      m.name_offset = name_off;
      m.name_len = name_len;
      m.quant_type = qt;
      m.num_blocks = num_blocks;
      m.total_values = total;
      m.data_offset = data_off;
      m.data_bytes = off - data_off;
    }
  }
  (void)version;
  return OOMATTN_OK;
}

extern "C" int oomattn_q8_repack(oomattn_ctx* ctx, const uint8_t* blocks, uint64_t bytes, int64_t n_values,
                                 uint8_t* q, float* scale, float* min) {
  if (!ctx) return OOMATTN_ERR_INVALID_ARG;
  if (!blocks || !q || !scale || !min || n_values <= 0) return fail(ctx, OOMATTN_ERR_INVALID_ARG, "bad q8_repack arguments");
  const long long nb = (n_values + 255) / 256;
  const uint64_t expect = (uint64_t)nb * 12 + (uint64_t)n_values;
  if (bytes != expect)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "a Q8 stream of %lld values has %llu bytes, not %llu", (long long)n_values,
                (unsigned long long)bytes, (unsigned long long)expect);
  if (reinterpret_cast<uintptr_t>(q) % 8 || reinterpret_cast<uintptr_t>(scale) % 4 ||
      reinterpret_cast<uintptr_t>(min) % 4)
    return fail(ctx, OOMATTN_ERR_INVALID_ARG, "q must be 8-byte and scale/min 4-byte aligned");
  DeviceGuard dg(ctx->device);
  const uintptr_t p = reinterpret_cast<uintptr_t>(blocks);
  const uint32_t* base_w = reinterpret_cast<const uint32_t*>(p & ~uintptr_t(3));
  const int warps = 8;
  q8_repack_kernel<<<(unsigned)((nb + warps - 1) / warps), warps * 32, 0, ctx->stream>>>(
      base_w, (uint32_t)(p & 3), n_values, nb, q, scale, min, ctx->d_status);
  CKLAUNCH();
  return OOMATTN_OK;
}
