/*
 * oomattn -- B200 (sm_100a) grouped-query attention step for OomLlama, behind
 * a plain C ABI.
 *
 * What it replaces (paths relative to the jaspertvdm/oomllama project root):
 *   TurboEngine::new / reset / seq_len            src/oomllama_turbo.rs:528-538, 726-733
 *   TurboEngine::attention_forward_with_bias       src/oomllama_turbo.rs:618-723
 *   LayerKVCache / ModelKVCache (append, get, ...) src/oomllama_turbo.rs:26-104
 *   TurboEngine::apply_rope, apply_rope,
 *   apply_rope_llama, compute_rope_freqs           src/oomllama_turbo.rs:376-467, 737-786
 *   flash_attention_forward                        src/oomllama_turbo.rs:304-369
 *   attention_head / softmax (CPU scalar path)     src/oom_inference.rs:152-164, 240-272
 *
 * Conventions
 *  - Every function returns an oomattn_status (0 = OK).  Nothing aborts or
 *    throws across the ABI; oomattn_last_error() holds the message of the last
 *    failure on a context.  Invalid shapes, indices and positions are rejected
 *    on the host before any GPU work is queued.
 *  - Device pointers are raw CUDA device addresses owned by the caller;
 *    host pointers are marked "host".  All GPU work is queued on the context's
 *    stream (oomattn_set_stream); nothing synchronises the host except
 *    oomattn_sync and oomattn_kv_read.
 *  - A context owns the paged K/V pools of all layers, the block tables, the
 *    RoPE table and the split-KV scratch.  One context per device per host
 *    thread; calls on one context are not thread-safe (the reference engine
 *    sits behind a Mutex / RwLock, src/python.rs:38, src/main.rs:617).
 *  - head_dim is 128 and a page holds 16 tokens.  Tensor layouts are
 *    row-major: tokens [T][heads][128]; weights [out][in] (HF/GGUF layout,
 *    src/oomllama_turbo.rs:637).
 */
#ifndef OOMATTN_H
#define OOMATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OOMATTN_ABI_VERSION 1

typedef enum oomattn_status {
  OOMATTN_OK = 0,
  OOMATTN_ERR_INVALID_ARG = 1,  /* null pointer, negative size, unknown enum value */
  OOMATTN_ERR_BAD_CONFIG = 2,   /* unsupported head_dim / page size, heads not divisible */
  OOMATTN_ERR_OUT_OF_RANGE = 3, /* layer, sequence, page or position outside its range */
  OOMATTN_ERR_CUDA = 4,         /* a CUDA runtime / driver call failed */
  OOMATTN_ERR_NCCL = 5,         /* reserved for communicator failures */
  OOMATTN_ERR_TIMEOUT = 6,      /* a bounded device-side wait gave up */
  OOMATTN_ERR_NO_MEMORY = 7,    /* device allocation failed */
  OOMATTN_ERR_UNSUPPORTED = 8,  /* valid request this build does not implement */
  OOMATTN_ERR_DEVICE_CHECK = 9  /* a kernel's own index check failed */
} oomattn_status;

enum { OOMATTN_DTYPE_F32 = 0, OOMATTN_DTYPE_BF16 = 1 };
/* Floats per (row, q head) in the packed decode output: O in [0, 128), the
 * natural-log LSE at 128, 3 floats of padding (16-byte aligned rows). */
#define OOMATTN_PACKED_STRIDE 132
/* Test-only flags (oomattn_set_test_flags). */
enum { OOMATTN_TEST_DROP_DECODE_COPIES = 1, OOMATTN_TEST_DROP_LINEAR_COPIES = 2 };
/* RoPE pairing: split-half pairs (x[i], x[i+64]) -- apply_rope_llama,
 * src/oomllama_turbo.rs:443-467, and TurboEngine::apply_rope :737-786;
 * interleaved pairs (x[2i], x[2i+1]) -- apply_rope, :402-438. */
enum { OOMATTN_ROPE_SPLIT_HALF = 0, OOMATTN_ROPE_INTERLEAVED = 1 };

/* TurboConfig (src/oomllama_turbo.rs:474-497) plus the fields the reference
 * hard-codes (theta, :746) or leaves implicit (paging, cache dtype). */
typedef struct oomattn_config {
  int32_t n_layers;     /* TurboConfig::n_layers */
  int32_t hidden_size;  /* TurboConfig::hidden_size (projection input width) */
  int32_t n_heads;      /* TurboConfig::n_heads (q heads held by this context) */
  int32_t n_kv_heads;   /* TurboConfig::n_kv_heads; n_heads / n_kv_heads <= 8 */
  int32_t head_dim;     /* must be 128 */
  int32_t max_seq_len;  /* TurboConfig::max_seq_len: RoPE positions are < this */
  int32_t max_seqs;     /* sequence slots (batch rows) */
  int32_t page_size;    /* must be 16 */
  int32_t n_pages;      /* pages per layer pool shared by all sequences */
  int32_t kv_dtype;     /* OOMATTN_DTYPE_F32 or OOMATTN_DTYPE_BF16 */
  int32_t rope_variant; /* OOMATTN_ROPE_* */
  float rope_theta;     /* 1e6 for Qwen2.5, 5e5 for Llama-3 */
  float softmax_scale;  /* <= 0 selects 1/sqrt(head_dim) (src/oomllama_turbo.rs:688) */
} oomattn_config;

typedef struct oomattn_ctx oomattn_ctx;

/* ---------------------------------------------------------------- lifecycle */

/* Version string of the library build. */
const char* oomattn_version(void);

/* TurboEngine::new (src/oomllama_turbo.rs:528-538).  Allocates the pools
 * (zeroed), the RoPE table (host-computed in f32 as :753-761) and scratch on
 * `device`; `stream` is a cudaStream_t (NULL = legacy default stream). */
int oomattn_create(const oomattn_config* cfg, int device, void* stream, oomattn_ctx** out);
int oomattn_destroy(oomattn_ctx* ctx);
const char* oomattn_last_error(const oomattn_ctx* ctx);
int oomattn_set_stream(oomattn_ctx* ctx, void* stream);
/* Waits for the context's stream and reports device-side check failures
 * (OOMATTN_ERR_TIMEOUT / OOMATTN_ERR_DEVICE_CHECK), clearing them. */
int oomattn_sync(oomattn_ctx* ctx);

/* Limit of every bounded device-side wait of this context's kernels (default
 * 2 s).  A wait that runs out records OOMATTN_ERR_TIMEOUT for oomattn_sync and
 * ends its kernel.  No counterpart in the reference (it has no device waits). */
int oomattn_set_wait_limit(oomattn_ctx* ctx, uint64_t timeout_ns);

/* Test-only launch flags, 0 in normal use.  OOMATTN_TEST_DROP_DECODE_COPIES
 * makes the bf16 decode's copy producer issue nothing, so that its consumers'
 * bounded waits run out: a test of the timeout path that faults nothing.
 * OOMATTN_TEST_DROP_LINEAR_COPIES does the same for the Q8 tensor-core pass
 * (its MMA issuer's and promoters' waits run out).  No counterpart in the
 * reference. */
int oomattn_set_test_flags(oomattn_ctx* ctx, int32_t flags);

/* TurboEngine::reset / ModelKVCache::clear (src/oomllama_turbo.rs:95-99,
 * 726-728): every layer's length of every sequence becomes 0.  Page
 * assignments are kept. */
int oomattn_reset(oomattn_ctx* ctx);

/* TurboEngine::seq_len / LayerKVCache::seq_len (src/oomllama_turbo.rs:32,
 * 731-733), per layer and sequence (the reference reads layer 0 only). */
int oomattn_seq_len(const oomattn_ctx* ctx, int32_t layer, int32_t seq, int32_t* out_len /* host */);

/* ------------------------------------------------------------ cache layout */

/* Assigns pool pages to a sequence: logical page i of `seq` (tokens
 * 16i..16i+15) lives in pool page pages[i] in every layer.  Unassigned logical
 * pages point at a zero null page.  pages: host array of n ids in
 * [0, n_pages). */
int oomattn_set_block_table(oomattn_ctx* ctx, int32_t seq, const int32_t* pages /* host */, int32_t n);

/* Absolute RoPE position of the sequence's cache slot 0 (default 0).  A
 * context that holds a later slice of a split context sets it to the slice
 * start, so appended tokens rotate at their global position. */
int oomattn_set_position_offset(oomattn_ctx* ctx, int32_t seq, int32_t offset);

/* Sets a sequence's cached length in one layer without writing data (the
 * pool contents written by other means, e.g. oomattn_kv_pool, are taken as
 * already rotated). */
int oomattn_set_seq_len(oomattn_ctx* ctx, int32_t layer, int32_t seq, int32_t len);

/* Device addresses of the K and V pools: element (layer, page, kv, slot, d)
 * at (((layer*(n_pages+1) + page)*n_kv + kv)*16 + slot)*128 + d, in kv_dtype.
 * Page n_pages is the null page. */
int oomattn_kv_pool(const oomattn_ctx* ctx, void** k_pool, void** v_pool);

/* LayerKVCache::append (src/oomllama_turbo.rs:41-55) of already-rotated rows:
 * k, v: device [n][n_kv][128] in src_dtype appended after the current length. */
int oomattn_kv_write(oomattn_ctx* ctx, int32_t layer, int32_t seq, const void* k, const void* v, int32_t n,
                     int32_t src_dtype);

/* LayerKVCache::get (src/oomllama_turbo.rs:57-63): copies the layer's cache of
 * `seq` to host k_out, v_out [n_kv][len][128] in kv_dtype (synchronises). */
int oomattn_kv_read(oomattn_ctx* ctx, int32_t layer, int32_t seq, void* k_out /* host */, void* v_out /* host */);

/* Host copy of the f32 RoPE table rows [pos0, pos0+n) as cos, sin
 * [n][64] (compute_rope_freqs, src/oomllama_turbo.rs:376-396). */
int oomattn_rope_table(const oomattn_ctx* ctx, int32_t pos0, int32_t n, float* cos_out /* host */,
                       float* sin_out /* host */);

/* compute_rope_freqs (src/oomllama_turbo.rs:376-396) without a context: the
 * same host f32 table, rows [pos0, pos0+n), head_dim 128. */
int oomattn_compute_rope_table(float theta, int32_t head_dim, int32_t pos0, int32_t n, float* cos_out /* host */,
                               float* sin_out /* host */);

/* ---------------------------------------------------------------- K-A */

/* Bias + RoPE + paged append for already-projected rows (epilogue of
 * src/oomllama_turbo.rs:647-681).  Rows are n_seqs x n_new tokens, token t of
 * sequence seq_ids[t / n_new] at position offset + len + t % n_new.
 *   q: [T][n_heads][128]  k, v: [T][n_kv][128]  in in_dtype (device)
 *   bq, bk, bv: f32 biases or NULL   q_out: [T][n_heads][128] in q_out_dtype
 * Every sequence's length grows by n_new in `layer`. */
int oomattn_rope_append(oomattn_ctx* ctx, int32_t layer, int32_t n_seqs, const int32_t* seq_ids /* host */,
                        int32_t n_new, const void* q, const void* k, const void* v, int32_t in_dtype,
                        const float* bq, const float* bk, const float* bv, void* q_out, int32_t q_out_dtype);

/* The q half of the RoPE step (TurboEngine::apply_rope, src/oomllama_turbo.rs:
 * 737-786, and apply_rope :402-438, by the context's variant) at explicit
 * positions, with nothing appended: q rows [n_rows][n_heads][128] in in_dtype
 * (+ bq f32 or NULL) -> q_out in q_out_dtype; positions (host) < max_seq_len.
 * Used by the ranks of a split context that do not hold the new token's slot:
 * they attend with the same rotated query as the rank that appends it. */
int oomattn_rope_q(oomattn_ctx* ctx, int32_t n_rows, const int32_t* positions /* host */, const void* q,
                   int32_t in_dtype, const float* bq, void* q_out, int32_t q_out_dtype);

/* Fused QKV projection + bias + RoPE + append (src/oomllama_turbo.rs:638-681).
 *   x: f32 [T][hidden]; wq [n_heads*128][hidden], wk/wv [n_kv*128][hidden] in
 *   w_dtype; bq/bk/bv f32 or NULL; q_out as in oomattn_rope_append.
 * T <= 16 runs one fused GEMV kernel (weights read once); larger T runs the
 * tensor-core linear (as oomattn_linear) followed by the K-A epilogue kernel. */
int oomattn_qkv_rope_append(oomattn_ctx* ctx, int32_t layer, int32_t n_seqs, const int32_t* seq_ids /* host */,
                            int32_t n_new, const float* x, const void* wq, const void* wk, const void* wv,
                            int32_t w_dtype, const float* bq, const float* bk, const float* bv, void* q_out,
                            int32_t q_out_dtype);

/* ---------------------------------------------------------------- K-B */

/* One-query-per-row GQA attention over the paged cache (split-KV flash
 * decode with an in-kernel LSE merge).  Row z attends to the first lens[z]
 * slots of sequence seq_ids[z] (lens NULL: the whole current length).
 *   q: f32 [n_rows][n_heads][128] rotated; out: f32 [n_rows][n_heads][128];
 *   lse: f32 [n_rows][n_heads] natural-log LSE of the scaled scores, or NULL. */
int oomattn_decode(oomattn_ctx* ctx, int32_t layer, int32_t n_rows, const int32_t* seq_ids /* host */,
                   const int32_t* lens /* host, may be NULL */, const float* q, float* out, float* lse);

/* oomattn_decode with the outputs packed for the split-context exchange
 * (flash_attention_forward's decode rows, src/oomllama_turbo.rs:304-369):
 * packed [n_rows][n_heads][OOMATTN_PACKED_STRIDE] f32 (16-byte aligned), O
 * at [0, 128) and the natural-log LSE at 128, so one collective moves both. */
int oomattn_decode_packed(oomattn_ctx* ctx, int32_t layer, int32_t n_rows, const int32_t* seq_ids /* host */,
                          const int32_t* lens /* host, may be NULL */, const float* q, float* packed);

/* K-B2 / K-D merge: combine n_parts split-context results of n_rows rows:
 * parts [n_parts][n_rows][128] (each normalised), lses [n_parts][n_rows]
 * (natural log); out [n_rows][128], lse_out [n_rows] or NULL. */
int oomattn_merge_partials(oomattn_ctx* ctx, int32_t n_parts, int32_t n_rows, const float* parts, const float* lses,
                           float* out, float* lse_out);

/* The same merge over packed partials [n_parts][n_rows][OOMATTN_PACKED_STRIDE]
 * (the all-gathered outputs of oomattn_decode_packed, n_rows = rows x heads). */
int oomattn_merge_packed(oomattn_ctx* ctx, int32_t n_parts, int32_t n_rows, const float* packed, float* out,
                         float* lse_out);

/* Decode for callers that cannot allocate device memory.  No counterpart in
 * the reference.  Some hosts cannot call cudaMalloc while decoding: their
 * device memory belongs to another allocator (a serving arena, a framework
 * that hands a plugin only tensors), or an allocation in their token loop
 * could synchronise the GPU or fail under memory pressure.  This entry point
 * needs no context and allocates nothing: it runs the split-KV decode kernels
 * over the caller's own paged K/V memory and keeps the split partials in a
 * fixed 8.1 MiB array inside the library's device image (every GPU that loads
 * the library holds one copy until the process exits).
 *   device, stream: the GPU and cudaStream_t to run on
 *   kv_dtype: OOMATTN_DTYPE_BF16 or OOMATTN_DTYPE_F32
 *   k_pool, v_pool: [n_pool_pages][n_kv_heads][16][128] in kv_dtype, 16-byte aligned
 *   block_table: device int32 [n_block_rows][max_pages_per_seq]
 *   q, out: f32 [n_rows][n_heads][128]; lse: f32 [n_rows][n_heads] or NULL
 *   seq_ids, lens (host): row z attends to the first lens[z] slots of block-table row seq_ids[z]
 *   errbuf (host, optional): receives a message when the call fails
 * The caller keeps these rules, which only the device can check:
 *   - every seq_ids[z] is below the block table's row count n_block_rows (the
 *     kernels read row seq_ids[z] without knowing how many rows there are);
 *   - every page id a row reaches is below n_pool_pages.  A larger id is read as
 *     the pool's last page and reported by oomattn_decode_static_scratch_status,
 *     so the pool should end with a zeroed page that no sequence uses;
 *   - slots past lens[z] in a row's last page hold finite values (they are
 *     weighted by zero, and 0 x inf or 0 x NaN would reach the output).
 * Limits: n_rows <= 128, n_kv_heads <= 64, n_heads / n_kv_heads <= 8; larger
 * requests return OOMATTN_ERR_OUT_OF_RANGE.  The split count is capped so
 * that n_rows * n_heads * splits <= 16384.  The first call on a device looks
 * up the array's address and must come before any stream capture on that
 * device.  All calls on a device share the array: calls whose GPU work
 * overlaps (different streams, other host threads) race and must be ordered
 * by the caller.  Device-side errors (an out-of-range page id, a wait that
 * gave up) accumulate in a status word inside the same array until
 * oomattn_decode_static_scratch_status reads them. */
int oomattn_decode_static_scratch(int device, void* stream, int32_t kv_dtype, const void* k_pool, const void* v_pool,
                                  int32_t n_pool_pages, const int32_t* block_table, int32_t max_pages_per_seq,
                                  int32_t n_heads, int32_t n_kv_heads, float softmax_scale, int32_t n_rows,
                                  const int32_t* seq_ids /* host */, const int32_t* lens /* host */, const float* q,
                                  float* out, float* lse, char* errbuf /* host, may be NULL */, int32_t errbuf_len);

/* The device-side error bits that oomattn_decode_static_scratch calls on
 * `device` have recorded since the last read, and clears them: waits for
 * `stream`, writes the bits to *flags_out (host) and returns OOMATTN_OK (none),
 * OOMATTN_ERR_TIMEOUT or OOMATTN_ERR_DEVICE_CHECK.  Allocates nothing.  No
 * counterpart in the reference. */
int oomattn_decode_static_scratch_status(int device, void* stream, int32_t* flags_out /* host */,
                                         char* errbuf /* host, may be NULL */, int32_t errbuf_len);

/* ---------------------------------------------------------------- K-C */

/* Causal prefill of the n_new newest tokens of `seq` (bf16 cache only):
 * query i (absolute slot len-n_new+i) attends to slots 0..len-n_new+i.
 *   q: bf16 [n_new][n_heads][128] rotated; out: [n_new][n_heads][128] in
 *   out_dtype; lse: f32 [n_new][n_heads] or NULL. */
int oomattn_prefill(oomattn_ctx* ctx, int32_t layer, int32_t seq, int32_t n_new, const void* q, void* out,
                    int32_t out_dtype, float* lse);

/* oomattn_prefill for some of the 256-row query blocks only: block b is query
 * rows [256 b, 256 b + 256) of the n_new; the launch computes the blocks of the
 * n_ranges ranges [ranges[2i], ranges[2i+1]) (host, at most 4, disjoint, inside
 * [0, ceil(n_new / 256))) and writes only their rows of out and lse.  A rank of
 * a prefill sharded beyond the kv-head count takes a zig-zag share of the
 * blocks (flash_attention_forward's causal path, src/oomllama_turbo.rs:344-368,
 * split over GPUs; the reference has no multi-GPU attention). */
int oomattn_prefill_blocks(oomattn_ctx* ctx, int32_t layer, int32_t seq, int32_t n_new, const void* q, void* out,
                           int32_t out_dtype, float* lse, int32_t n_ranges, const int32_t* ranges /* host */);

/* ------------------------------------------------------- linear projections */

/* y[t][r] = sum_c x[t][c] * w[r][c] (+ bias[r]): candle's x @ W^T of the
 * projections (src/oomllama_turbo.rs:643-645) and of o_proj (:715-720).
 *   x f32 [n_tokens][cols], w [rows][cols] in w_dtype, bias f32 [rows] or
 *   NULL, y f32 [n_tokens][rows]; device pointers, 16-byte aligned.
 * Up to 16 tokens with f32 weights: a GEMV that streams W once.  Otherwise
 * the tcgen05 tensor-core linear: x (and f32 W) split into bf16 hi + lo
 * planes, three products per tile (two for bf16 W), f32 accumulation --
 * within 1e-4 of the f32 product at unit-scale activations.  Needs
 * cols % 8 == 0 and rows % 4 == 0. */
int oomattn_linear(oomattn_ctx* ctx, const float* x, const void* w, int32_t w_dtype, int32_t n_tokens, int32_t rows,
                   int32_t cols, const float* bias, float* y);

/* ------------------------------------------------------- the layer step */

/* TurboEngine::attention_forward_with_bias (src/oomllama_turbo.rs:618-723) for
 * batch rows 0..batch-1 (sequence slot b = batch row b), seq_len new tokens
 * each: QKV + bias -> RoPE at each sequence's own length -> append ->
 * causal GQA attention -> o_proj.  f32 activations and weights:
 *   x [batch][seq_len][hidden]; wq [n_heads*128][hidden]; wk, wv
 *   [n_kv*128][hidden]; wo [o_out][n_heads*128]; bq/bk/bv or NULL;
 *   out [batch][seq_len][o_out]. */
int oomattn_attention_forward_with_bias(oomattn_ctx* ctx, int32_t layer, int32_t batch, int32_t seq_len,
                                        const float* x, const float* wq, const float* wk, const float* wv,
                                        const float* wo, int32_t o_out, const float* bq, const float* bk,
                                        const float* bv, float* out);

/* ------------------------------------------- K-E: GPU-resident Q8 weights */

/* A Q8 matrix W [rows][cols] resident on the device, row-major ([out][in], the
 * HF layout of the projections and MLP weights).  Values are quantised in
 * blocks of 256 consecutive values of the row-major flattening, as the .oom
 * writer cuts them (src/gguf2oom.rs:719-770); block b covers values
 * [256 b, 256 b + 256):
 *   W[r][c] = min[b] + (float)q[r * cols + c] * scale[b],  b = (r * cols + c) / 256
 * (BlockQ8View::dequantize_fast, src/quant.rs:201-224).
 *   q: uint8 [rows * cols] (16-byte aligned); scale, min: f32 [ceil(rows*cols/256)].
 * It replaces the reference's per-call path, OomLoader::dequantize_tensor
 * (src/quant.rs:413-468) into an f32 host buffer and its upload in
 * GhostLayer::materialize (src/oomllama.rs:425-439). */
typedef struct oomattn_q8_matrix {
  const uint8_t* q;
  const float* scale;
  const float* min;
  int32_t rows;
  int32_t cols;
} oomattn_q8_matrix;

/* Unpack the block stream of one .oom Q8 tensor -- the bytes that follow its
 * header, n_blocks = ceil(n_values / 256) blocks of [f32 scale][f32 min]
 * [u32 len][len bytes q], little endian (src/gguf2oom.rs:823-826) -- into host
 * arrays q_out[n_values], scale_out[n_blocks] and min_out[n_blocks].  The walk
 * is OomLoader::dequantize_tensor_into's (src/quant.rs:431-463); every block
 * must hold min(256, values left) bytes and lie inside the stream, otherwise
 * OOMATTN_ERR_INVALID_ARG.  Host only: needs no context or GPU. */
int oomattn_q8_unpack(const uint8_t* stream /* host */, uint64_t stream_bytes, int64_t n_values,
                      uint8_t* q_out /* host */, float* scale_out /* host */, float* min_out /* host */,
                      char* errbuf /* host, may be NULL */, int32_t errbuf_len);

/* y[t][r] = sum_c x[t][c] * W[r][c]  (+ bias[r] when bias is not NULL), for
 * t < n_tokens: the reference's matvec (src/oom_inference.rs:168-180) and
 * candle's x @ W^T (src/oomllama_turbo.rs:643-645) on dequantised weights,
 * without materialising them.  f32 activations: x [n_tokens][cols],
 * y [n_tokens][rows], bias [rows] -- all device pointers.  rows must be a
 * multiple of 16 and cols of 64; |x| < 65504 (x enters the tensor cores as an
 * fp16 hi/lo pair; larger values are reported by oomattn_sync as
 * OOMATTN_ERR_DEVICE_CHECK).  Up to 64 tokens the weights stream through
 * 16-token passes; more tokens (a prefill chunk), with cols % 256 == 0, run
 * the tcgen05 tensor-core linear: W converted to fp16 q values once per call,
 * each 256-value block's dot products promoted with its scale and min. */
int oomattn_q8_linear(oomattn_ctx* ctx, const oomattn_q8_matrix* w /* host struct */, const float* x,
                      int32_t n_tokens, const float* bias, float* y);

/* ------------------------------------------- the layer steps around attention */

/* GhostRMSNorm::forward (src/oomllama.rs:200-211): out[t] = x[t] /
 * sqrt(mean(x[t]^2) + eps) * weight, f32, x and out [n_tokens][hidden],
 * weight [hidden]; hidden % 4 == 0, 16-byte aligned rows (device). */
int oomattn_rmsnorm(oomattn_ctx* ctx, const float* x, const float* weight, float eps, int32_t n_tokens,
                    int32_t hidden, float* out);

/* GhostMlp::forward (src/oomllama.rs:230-242) on resident Q8 weights, plus
 * the decoder layer's residual add (src/oomllama.rs:401):
 *   y = down(silu(gate(x)) * up(x)) (+ residual)
 * gate, up [inter][hidden]; down [hidden][inter]; x, y, residual
 * [n_tokens][hidden] f32 (residual may alias y, or be NULL).  The gated
 * activation is formed while down's input is split, without a buffer of its
 * own. */
int oomattn_q8_mlp(oomattn_ctx* ctx, const oomattn_q8_matrix* gate, const oomattn_q8_matrix* up,
                   const oomattn_q8_matrix* down, const float* x, int32_t n_tokens, const float* residual, float* y);

/* The Q8 weights of one decoder layer (GhostDecoderLayer, src/oomllama.rs:366-402). */
typedef struct oomattn_q8_layer {
  oomattn_q8_matrix q, k, v, o;      /* [n_heads*128][hidden], [n_kv*128][hidden] x2, [hidden][n_heads*128] */
  oomattn_q8_matrix gate, up, down;  /* [inter][hidden] x2, [hidden][inter] */
  const float* bq;                   /* attention biases (Qwen), f32 or NULL */
  const float* bk;
  const float* bv;
  const float* input_norm;           /* RMSNorm weights [hidden] */
  const float* post_norm;
  float eps;                         /* rms_norm_eps */
} oomattn_q8_layer;

/* GhostDecoderLayer::forward_turbo (src/oomllama.rs:387-402) for one new token
 * of each of n_seqs sequences (decode), Q8 weights resident on the device:
 *   h = x + o_proj(attention(rope(qkv(rmsnorm(x)))))      (the token is appended)
 *   out = h + mlp(rmsnorm(h))
 * x, out [n_seqs][hidden] f32 (device); sequence seq_ids[b] is batch row b. */
int oomattn_decoder_layer_q8(oomattn_ctx* ctx, int32_t layer, int32_t n_seqs, const int32_t* seq_ids /* host */,
                             const float* x, const oomattn_q8_layer* w /* host struct */, float* out);

/* ------------------------------------------------------------------ .oom files */

/* One tensor of an .oom file: OomTensorMeta (src/quant.rs:307-312) plus where
 * its name and blocks lie in the file image.  quant_type: 0 f32 (one block of
 * raw values), 8 Q8, 4 Q4, 2 Q2. */
typedef struct oomattn_oom_tensor {
  uint64_t name_offset;  /* the name's bytes (not terminated) */
  uint32_t name_len;
  uint32_t quant_type;
  uint32_t num_blocks;
  uint32_t total_values;
  uint64_t data_offset;  /* first block header: OomTensorMeta::offset */
  uint64_t data_bytes;   /* all its blocks: headers and data */
} oomattn_oom_tensor;

/* OomLoader::load's scan (src/quant.rs:320-367) of a file image in host
 * memory: "OOML", u32 version, u32 tensor count, then per tensor u32 name
 * length, name, u8 quant type, u32 blocks, u32 values and its blocks
 * (src/gguf2oom.rs:708-716, :782-829).  Fills out[0..min(count, max_tensors))
 * and *n_tensors = count.  A field or block past the end of the image is
 * OOMATTN_ERR_INVALID_ARG (the reference stops silently).  Host only. */
int oomattn_oom_scan(const uint8_t* file /* host */, uint64_t bytes, oomattn_oom_tensor* out /* host */,
                     int32_t max_tensors, int32_t* n_tensors /* host */, char* errbuf /* host, may be NULL */,
                     int32_t errbuf_len);

/* The device-side repack of one Q8 tensor: its block stream (the bytes at
 * data_offset, data_bytes long, already in device memory, at any byte
 * alignment and readable to the next 4-byte boundary past its end) into the
 * resident layout q [n_values], scale and min [ceil(n_values / 256)] that
 * oomattn_q8_unpack produces on the host.  A block whose length field is not
 * min(256, values left) is reported by oomattn_sync as OOMATTN_ERR_DEVICE_CHECK. */
int oomattn_q8_repack(oomattn_ctx* ctx, const uint8_t* blocks, uint64_t bytes, int64_t n_values, uint8_t* q,
                      float* scale, float* min);

/* ------------------------------------------------ embedding, LM head, greedy pick */

/* out[t] = row token_ids[t] of the embedding table emb [vocab][hidden],
 * dequantised (min + (f32)q * scale): embed_w.embedding(tokens) of
 * OomLlamaModel::forward_turbo (src/oomllama.rs:508-515).  token_ids
 * [n_tokens] int32 and out [n_tokens][hidden] f32 are device pointers; an id
 * outside [0, vocab) gives a zero row and OOMATTN_ERR_DEVICE_CHECK at
 * oomattn_sync. */
int oomattn_embed_q8(oomattn_ctx* ctx, const oomattn_q8_matrix* emb /* host struct */, const int32_t* token_ids,
                     int32_t n_tokens, float* out);

/* ids[r] = argmax of logits[r][0..n): the generation loop's greedy pick
 * (src/oomllama.rs:973-976, :1000-1003; candle's argmax scans from element 0
 * and moves only to a strictly larger value: lowest index among equal values,
 * NaN skipped unless in element 0, which then gives 0).  Device pointers. */
int oomattn_argmax(oomattn_ctx* ctx, const float* logits, int32_t n_rows, int32_t n, int32_t* ids);

/* A whole Q8 model (OomLlamaModel, src/oomllama.rs:462-500). */
typedef struct oomattn_q8_model {
  int32_t n_layers;                /* <= the context's n_layers; layer l uses KV layer l */
  const oomattn_q8_layer* layers;  /* host array [n_layers] */
  oomattn_q8_matrix embed;         /* [vocab][hidden] */
  oomattn_q8_matrix lm_head;       /* [vocab][hidden] */
  const float* final_norm;         /* [hidden] (device) */
  float eps;
} oomattn_q8_model;

/* One decode step of the whole model for n_seqs sequences, one new token each
 * (OomLlamaModel::forward_turbo, src/oomllama.rs:504-553, then the greedy pick
 * of the generation loop, :1000-1003): embedding of tokens[b], every decoder
 * layer (each appends the token to its KV cache), the final RMSNorm, the LM
 * head and argmax into next[b].  tokens, next [n_seqs] int32 (device; next may
 * alias tokens, so steps chain on the device); logits [n_seqs][vocab] f32
 * (device) or NULL to keep them in library scratch.  seq_ids [n_seqs] is host
 * memory, sequence seq_ids[b] is batch row b.  The sequences' lengths grow by
 * one. */
int oomattn_decode_step_q8(oomattn_ctx* ctx, const oomattn_q8_model* m /* host struct */, int32_t n_seqs,
                           const int32_t* seq_ids /* host */, const int32_t* tokens, int32_t* next, float* logits);

/* The prompt of n_seqs sequences through the whole model
 * (OomLlamaModel::forward_turbo over all prompt tokens, src/oomllama.rs:504-553,
 * as GhostLlamaModel's generate calls it, :969-970), then the first greedy pick:
 * tokens [n_seqs][n_new] int32 (device) are embedded, every decoder layer
 * appends their K/V to its cache (K-A), attends causally over each sequence
 * (K-C) and runs its projections and MLP on the tensor cores (Q8 weights); the
 * final RMSNorm, LM head and argmax of each sequence's last prompt token give
 * next[b] (device; logits [n_seqs][vocab] or NULL).  Needs a bf16 cache; the
 * sequences' lengths grow by n_new in every layer. */
int oomattn_prefill_step_q8(oomattn_ctx* ctx, const oomattn_q8_model* m /* host struct */, int32_t n_seqs,
                            const int32_t* seq_ids /* host */, int32_t n_new, const int32_t* tokens, int32_t* next,
                            float* logits);


#ifdef __cplusplus
}
#endif

#endif /* OOMATTN_H */
