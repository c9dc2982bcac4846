// K-E: x @ W^T for GPU-resident Q8 weights, without materialising W.
//
// Semantics: y[t][r] = sum_c x[t][c] * W[r][c] (+ bias[r]) with
// W[r][c] = min_b + q[r][c] * scale_b, b the 256-value block of the row-major
// flattening (BlockQ8View::dequantize_fast, src/quant.rs:201-224; the matvec
// src/oom_inference.rs:168-180).  The block's affine map is applied after the
// dot product, per 64-column chunk (a chunk never straddles a block because
// cols is a multiple of 64):
//   sum_k x_k (min + q_k s) = s * sum_k q_k x_k + min * sum_k x_k.
//
// Tensor-core form (mma.sync m16n8k16, fp16 in, f32 accumulate):
//  - A = 1024 + q as fp16: the bit pattern 0x6400 | q, built from the weight
//    bytes with one byte permute per two values; exact for q <= 255.
//  - B = x split into fp16 hi + lo (about 22 significant bits), two MMAs per
//    k-step; products are exact in the f32 accumulator.
//  - D = sum (1024 + q) x, so the chunk's contribution is
//      s * D + (min - 1024 s) * X,   X = sum_k x_k over the chunk.
//  - The k order inside a chunk is permuted so that each thread's A values
//    are 16 consecutive weight bytes of a row and its B values 16 consecutive
//    x values of a token (the dot product does not depend on the order).
// A warp covers 16 * MT rows x 64 columns per chunk and all tokens in tiles of
// 8, reading the next chunk's operands while it computes the current one; a
// CTA's 8 warps split its column range and reduce in shared memory, and
// split-K CTAs of the same rows merge through a partial buffer: the last CTA
// to arrive (a per-row-block counter) sums the splits in order, so results do
// not depend on CTA timing.
//
// Roofline: HBM-bound for decode-sized token counts; algorithmic bytes per
// launch = rows * cols (q) + 8 * ceil(rows * cols / 256) (scale, min)
// + 4 * (n_tokens * cols + n_tokens * rows) (x, y).
#pragma once
#include <cuda_fp16.h>

#include "common.cuh"

namespace oomattn {

constexpr int kQ8Warps = 8;            // warps per CTA
constexpr int kQ8Chunk = 64;           // columns per chunk

// One matrix of a launch: its weights, epilogue operands and output.  A
// launch runs up to kQ8MaxMats matrices of the same width on the same x (the
// q, k and v projections; gate and up); matrix i owns the grid's row blocks
// from rb_begin.
constexpr int kQ8MaxMats = 3;
struct Q8Mat {
  const uint8_t* q;
  const float* scale;
  const float* min;
  int rows;
  int rb_begin;
  const float* bias;      // [rows] or null
  const float* residual;  // [n_tokens][rows] added to y, or null (may alias y)
  float* y;               // [n_tokens][rows]
  float* part;            // [splits][8 * token tiles][rows]: split-K partial sums
};

struct Q8Args {
  Q8Mat m[kQ8MaxMats];
  int n_mats;
  int cols;
  const uint32_t* xh;   // [n_tokens][cols / 2] fp16 pairs: x rounded to fp16
  const uint32_t* xl;   // [n_tokens][cols / 2] fp16 pairs: x - hi rounded to fp16
  const float* xsum;    // [n_tokens][cols / 64]
  int n_tokens;
  unsigned* counters;   // [row blocks]: arrivals, zero between launches
  int splits;
  int chunks_per_split;
  int* status;
};

// What one CTA uses: its matrix's fields and the launch's shared ones.
struct Q8View {
  const uint8_t* q;
  const float* scale;
  const float* min;
  int rows;
  int rb;  // row block within the matrix
  const float* bias;
  const float* residual;
  float* y;
  float* part;
  int cols;
  int n_tokens;
  int splits;
};

// Field-wise selects keep the parameter array in constant space (a dynamic
// index would copy it to local memory).
__device__ __forceinline__ Q8View q8_view(const Q8Args& A, int rbg) {
  const int j = (A.n_mats > 1 && rbg >= A.m[1].rb_begin) + (A.n_mats > 2 && rbg >= A.m[2].rb_begin);
#define Q8_SEL(f) (j == 0 ? A.m[0].f : (j == 1 ? A.m[1].f : A.m[2].f))
  Q8View v;
  v.q = Q8_SEL(q);
  v.scale = Q8_SEL(scale);
  v.min = Q8_SEL(min);
  v.rows = Q8_SEL(rows);
  v.rb = rbg - Q8_SEL(rb_begin);
  v.bias = Q8_SEL(bias);
  v.residual = Q8_SEL(residual);
  v.y = Q8_SEL(y);
  v.part = Q8_SEL(part);
#undef Q8_SEL
  v.cols = A.cols;
  v.n_tokens = A.n_tokens;
  v.splits = A.splits;
  return v;
}

// y = x W^T + bias + residual for one output element (the residual add of a
// decoder layer, src/oomllama.rs:391, :401).
__device__ __forceinline__ float q8_epilogue(const Q8View& a, int tok, int row, float v) {
  if (a.bias) v += a.bias[row];
  if (a.residual) v += a.residual[(size_t)tok * a.rows + row];
  return v;
}

// x -> (hi, lo) fp16 pairs and per-chunk sums.  One warp per (token, 64-column
// chunk): lane l owns columns 2l, 2l+1.  The chunk sum is a fixed shuffle
// tree, so it does not depend on timing.  |x| >= 65504 has no fp16 image: it
// is reported through the status word.
// With `up` given, the split input is the MLP's gated activation
// silu(x) * up = x * sigmoid(x) * up (GhostMlp::forward, src/oomllama.rs:230-242),
// so the down projection reads it without a separate kernel or buffer.
__global__ void q8_prep_x_kernel(const float* __restrict__ x, const float* __restrict__ up, int n_tokens, int cols,
                                 uint32_t* xh, uint32_t* xl, float* xsum, int* status) {
  // the linear kernel may launch now: it waits for this grid before it reads
  // the split.  (This kernel launches after the one before it; launched as its
  // programmatic dependent, resident beside a tensor-core pass, it slowed a
  // Qwen2.5-7B layer's four linears at 1 token from 68 to 101 us.)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int lane = threadIdx.x & 31;
  const int nchunks = cols / kQ8Chunk;
  const long long w = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (w >= (long long)n_tokens * nchunks) return;
  const int t = (int)(w / nchunks), ch = (int)(w % nchunks);
  float2 v = *reinterpret_cast<const float2*>(x + (size_t)t * cols + ch * kQ8Chunk + 2 * lane);
  if (up) {
    const float2 u = *reinterpret_cast<const float2*>(up + (size_t)t * cols + ch * kQ8Chunk + 2 * lane);
    v.x = v.x * (1.f / (1.f + expf(-v.x))) * u.x;
    v.y = v.y * (1.f / (1.f + expf(-v.y))) * u.y;
  }
  const __half2 hi = __floats2half2_rn(v.x, v.y);
  const float2 hf = __half22float2(hi);
  const __half2 lo = __floats2half2_rn(v.x - hf.x, v.y - hf.y);
  if (!(fabsf(v.x) < 65504.f) || !(fabsf(v.y) < 65504.f)) report_error(status, kDevErrX16);
  const size_t o = (size_t)t * (cols / 2) + ch * (kQ8Chunk / 2) + lane;
  xh[o] = *reinterpret_cast<const uint32_t*>(&hi);
  xl[o] = *reinterpret_cast<const uint32_t*>(&lo);
  float s = v.x + v.y;
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) s += __shfl_xor_sync(0xffffffffu, s, d);
  if (lane == 0) xsum[(size_t)t * nchunks + ch] = s;
}

// 16 weight bytes of a row, streamed past L1 (each byte is read once).
__device__ __forceinline__ uint4 ldg_stream16(const uint8_t* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// D(16x8, f32) += A(16x16, f16, row) * B(16x8, f16, col)
__device__ __forceinline__ void mma_f16_16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// fp16 pair (1024 + byte 2i, 1024 + byte 2i + 1) of a word of four weight bytes.
__device__ __forceinline__ uint32_t q8_pair(uint32_t w, uint32_t sel) { return __byte_perm(w, 0x64646464u, sel); }

// The weight bytes of one 64-column chunk for a warp's MT row tiles (rows g
// and g + 8 of each: 16 bytes each), and their blocks' scale and min.
template <int MT>
struct Q8W {
  uint4 qa[MT], qb[MT];
  float sa[MT], ma[MT], sb[MT], mb[MT];
};

// The x fragments of one chunk for NT token tiles: hi / lo pairs of token
// 8n + g (the thread's 16 columns) and the chunk sums of tokens 8n + 2c and
// 8n + 2c + 1.
template <int NT>
struct Q8X {
  uint32_t bh[NT][8], bl[NT][8];
  float x0[NT], x1[NT];
};

// Per-thread addresses that do not change along the column range.
template <int NT, int MT>
struct Q8Base {
  long long fa[MT];        // flattened index of row g of each row tile (row g + 8 is 8 rows on)
  bool live[MT];           // row tile inside the matrix
  const uint32_t* xh[NT];  // token 8n + g, this thread's 8 words of a chunk (null past n_tokens)
  const float* xs0[NT];    // chunk sums of token 8n + 2c (8n + 2c + 1 follows a row later)
  bool has0[NT], has1[NT];
  long long xlo;           // xl - xh in words
  long long row8;          // 8 * cols
  int nchunks;
};

// The weight bytes and their blocks' scale and min (independent of x).
template <int NT, int MT>
__device__ __forceinline__ void q8_load_w(const Q8View& a, const Q8Base<NT, MT>& b, int ch, Q8W<MT>& d) {
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    if (!b.live[m]) {  // a row block's last tile may lie past the matrix
      d.qa[m] = d.qb[m] = make_uint4(0, 0, 0, 0);
      d.sa[m] = d.ma[m] = d.sb[m] = d.mb[m] = 0.f;
      continue;
    }
    const long long f = b.fa[m] + ch * kQ8Chunk;
    d.qa[m] = ldg_stream16(a.q + f);
    d.qb[m] = ldg_stream16(a.q + f + b.row8);
    const long long ba = f >> 8, bb = (f + b.row8) >> 8;
    d.sa[m] = __ldg(a.scale + ba);
    d.ma[m] = __ldg(a.min + ba);
    d.sb[m] = __ldg(a.scale + bb);
    d.mb[m] = __ldg(a.min + bb);
  }
}

// The x fragments and chunk sums (written by the split kernel; cache hits).
template <int NT, int MT>
__device__ __forceinline__ void q8_load_x(const Q8Base<NT, MT>& b, int ch, Q8X<NT>& d) {
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    if (b.xh[n]) {  // tokens past n_tokens contribute zero and are not read
      const uint32_t* ph = b.xh[n] + ch * (kQ8Chunk / 2);
      const uint4 h0 = __ldg(reinterpret_cast<const uint4*>(ph));
      const uint4 h1 = __ldg(reinterpret_cast<const uint4*>(ph + 4));
      const uint4 l0 = __ldg(reinterpret_cast<const uint4*>(ph + b.xlo));
      const uint4 l1 = __ldg(reinterpret_cast<const uint4*>(ph + b.xlo + 4));
      d.bh[n][0] = h0.x; d.bh[n][1] = h0.y; d.bh[n][2] = h0.z; d.bh[n][3] = h0.w;
      d.bh[n][4] = h1.x; d.bh[n][5] = h1.y; d.bh[n][6] = h1.z; d.bh[n][7] = h1.w;
      d.bl[n][0] = l0.x; d.bl[n][1] = l0.y; d.bl[n][2] = l0.z; d.bl[n][3] = l0.w;
      d.bl[n][4] = l1.x; d.bl[n][5] = l1.y; d.bl[n][6] = l1.z; d.bl[n][7] = l1.w;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) d.bh[n][e] = d.bl[n][e] = 0u;
    }
    d.x0[n] = b.has0[n] ? __ldg(b.xs0[n] + ch) : 0.f;
    d.x1[n] = b.has1[n] ? __ldg(b.xs0[n] + b.nchunks + ch) : 0.f;
  }
}

template <int NT, int MT>
__device__ __forceinline__ void q8_compute_chunk(const Q8W<MT>& w, const Q8X<NT>& d, float (&acc)[MT][NT][4]) {
  constexpr bool kOneChain = NT * MT >= 4;
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    // A fragments of the 4 k-steps: step s takes bytes 4s..4s+3 of the thread's 16
    const uint32_t wa[4] = {w.qa[m].x, w.qa[m].y, w.qa[m].z, w.qa[m].w};
    const uint32_t wb[4] = {w.qb[m].x, w.qb[m].y, w.qb[m].z, w.qb[m].w};
    uint32_t af[4][4];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      af[s][0] = q8_pair(wa[s], 0x4140u);
      af[s][1] = q8_pair(wb[s], 0x4140u);
      af[s][2] = q8_pair(wa[s], 0x4342u);
      af[s][3] = q8_pair(wb[s], 0x4342u);
    }
    const float ka = w.ma[m] - 1024.f * w.sa[m], kb = w.mb[m] - 1024.f * w.sb[m];
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      // hi and lo products accumulate in two independent chains, or, with four
      // or more (row tile, token tile) pairs, in one: the pairs already give
      // independent MMAs, and the registers go to the weight ring
      float dh[4] = {0.f, 0.f, 0.f, 0.f}, dl[4] = {0.f, 0.f, 0.f, 0.f};
      float(&dlo)[4] = kOneChain ? dh : dl;
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        mma_f16_16816(dh, af[s][0], af[s][1], af[s][2], af[s][3], d.bh[n][2 * s], d.bh[n][2 * s + 1]);
        mma_f16_16816(dlo, af[s][0], af[s][1], af[s][2], af[s][3], d.bl[n][2 * s], d.bl[n][2 * s + 1]);
      }
      // rows g, g + 8 x tokens 8n + 2c, 8n + 2c + 1
      acc[m][n][0] = fmaf(w.sa[m], dh[0] + dl[0], fmaf(ka, d.x0[n], acc[m][n][0]));
      acc[m][n][1] = fmaf(w.sa[m], dh[1] + dl[1], fmaf(ka, d.x1[n], acc[m][n][1]));
      acc[m][n][2] = fmaf(w.sb[m], dh[2] + dl[2], fmaf(kb, d.x0[n], acc[m][n][2]));
      acc[m][n][3] = fmaf(w.sb[m], dh[3] + dl[3], fmaf(kb, d.x1[n], acc[m][n][3]));
    }
  }
}

// A CTA owns 16 * MT rows and a column range; its 8 warps take the range's
// chunks round-robin, each chunk for all MT row tiles and NT token tiles.
// Each warp keeps the weights of its next S - 1 chunks in flight in a
// register ring (the loop is unrolled by S so ring slots are static).  The x
// fragments are cache hits: with XA they are read one chunk ahead into a
// second buffer (S even, so buffer indices stay static), otherwise just
// before use, which leaves the registers to the weight ring.
template <int NT, int MT, int S, bool XA>
__global__ void __launch_bounds__(kQ8Warps * 32, 2) q8_linear_kernel(const Q8Args args) {
  static_assert(S >= 2 && (!XA || S % 2 == 0), "ring depth");
  __shared__ float red[kQ8Warps][MT][NT][4][32];
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const Q8View a = q8_view(args, blockIdx.y);
  const int sp = blockIdx.x;
  const int rb = a.rb;
  const int row0 = rb * 16 * MT;
  const int nchunks = a.cols / kQ8Chunk;
  const int c0 = sp * args.chunks_per_split, c1 = min(nchunks, c0 + args.chunks_per_split);

  Q8Base<NT, MT> b;
  b.row8 = 8LL * a.cols;
  b.xlo = args.xl - args.xh;
  b.nchunks = nchunks;
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    b.live[m] = row0 + 16 * m < a.rows;
    b.fa[m] = (long long)(row0 + 16 * m + g) * a.cols + 16 * c;  // block lookups ignore the low 8 bits
  }
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    const int tok = 8 * n + g, t0 = 8 * n + 2 * c;
    b.xh[n] = tok < a.n_tokens ? args.xh + (size_t)tok * (a.cols / 2) + 8 * c : nullptr;
    b.xs0[n] = args.xsum + (size_t)t0 * nchunks;
    b.has0[n] = t0 < a.n_tokens;
    b.has1[n] = t0 + 1 < a.n_tokens;
  }

  float acc[MT][NT][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[m][n][e] = 0.f;

  Q8W<MT> w[S];
  Q8X<NT> xf[XA ? 2 : 1];
  int ch = c0 + warp;
  // the first S - 1 chunks' weights do not depend on the x split: load them,
  // then wait for the split kernel (launched before this one) to complete
#pragma unroll
  for (int s = 0; s < S - 1; ++s)
    if (ch + s * kQ8Warps < c1) q8_load_w<NT, MT>(a, b, ch + s * kQ8Warps, w[s]);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (XA && ch < c1) q8_load_x<NT, MT>(b, ch, xf[0]);
  while (ch < c1) {
#pragma unroll
    for (int s = 0; s < S; ++s) {
      if (ch >= c1) break;
      const int nx = ch + (S - 1) * kQ8Warps;
      if (nx < c1) q8_load_w<NT, MT>(a, b, nx, w[(s + S - 1) % S]);
      if (XA) {
        if (ch + kQ8Warps < c1) q8_load_x<NT, MT>(b, ch + kQ8Warps, xf[(s + 1) & 1]);
        q8_compute_chunk<NT, MT>(w[s], xf[s & 1], acc);
      } else {
        q8_load_x<NT, MT>(b, ch, xf[0]);
        q8_compute_chunk<NT, MT>(w[s], xf[0], acc);
      }
      ch += kQ8Warps;
    }
  }

  // the CTA's warps cover disjoint chunks of the same rows: sum them in warp order
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) red[warp][m][n][e][lane] = acc[m][n][e];
  __syncthreads();
  const int tp = 8 * NT;
  const int rows_cta = 16 * MT;
  float* part = a.part + (size_t)sp * tp * a.rows;
  for (int i = threadIdx.x; i < MT * NT * 128; i += blockDim.x) {
    const int m = i / (NT * 128), n = (i / 128) % NT, e = (i / 32) & 3, l = i & 31;
    float v = 0.f;
#pragma unroll
    for (int w8 = 0; w8 < kQ8Warps; ++w8) v += red[w8][m][n][e][l];
    const int row = row0 + 16 * m + (l >> 2) + ((e & 2) ? 8 : 0);
    const int tok = 8 * n + 2 * (l & 3) + (e & 1);
    if (row >= a.rows || tok >= a.n_tokens) continue;
    if (a.splits == 1)
      a.y[(size_t)tok * a.rows + row] = q8_epilogue(a, tok, row, v);
    else
      part[(size_t)tok * a.rows + row] = v;
  }
  if (a.splits == 1) return;
  // split-K merge: the last CTA of this row block sums the splits in order
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atom_add_acq_rel_gpu(&args.counters[blockIdx.y], 1u);
    s_last = (prev == (unsigned)a.splits - 1);
  }
  __syncthreads();
  if (!s_last) return;
  for (int i = threadIdx.x; i < rows_cta * a.n_tokens; i += blockDim.x) {
    const int tok = i / rows_cta, row = row0 + i % rows_cta;
    if (row >= a.rows) continue;
    float v = 0.f;
    for (int s = 0; s < a.splits; ++s)
      v += __ldcg(a.part + ((size_t)s * tp + tok) * a.rows + row);
    a.y[(size_t)tok * a.rows + row] = q8_epilogue(a, tok, row, v);
  }
  if (threadIdx.x == 0) args.counters[blockIdx.y] = 0;
}

// ------------------------------------------------- 16 tokens, x in shared memory
// Form for 9..16 tokens on large matrices.  At 16 tokens the x fragments of a
// chunk (16 tokens x 64 columns as fp16 hi + lo: 4 KB) outweigh the chunk's
// weight bytes per warp (1-2 KB), and in the form above every CTA re-reads its
// whole column range of x from L2.  Here a CTA of 16 warps (one per SM, all
// 64K registers) owns 16 * 16 * MT rows and one column range: it stages the
// range's x hi / lo words and chunk sums in shared memory once, then each warp
// streams its own 16 * MT rows across the range with an S-deep weight ring,
// reading x fragments from shared memory.  Token rows are padded to 4 words
// past a multiple of 32 so that the 16-byte fragment loads of a warp's 8
// tokens fall in distinct banks.  Each warp owns its rows, so there is no
// reduction across warps; CTAs of other column ranges merge through the
// split-K partial buffer in split order, as above.
constexpr int kQ8XsWarps = 16;
// chunks per range: 96 / NT (x staging: 96 x 64 columns x 8 tokens x 4 B = 192 KB)
__host__ __device__ constexpr int q8_xs_max_chunks(int nt) { return 96 / nt; }
constexpr int kQ8Xs1S2 = 3, kQ8Xs1S1 = 8;  // one token tile: ring depth for MT = 2 and MT = 1

__host__ __device__ constexpr int q8_xs_stride(int cps) { return cps * 32 + 4; }  // words per token row
__host__ __device__ constexpr size_t q8_xs_smem_bytes(int nt, int cps) {
  return ((size_t)16 * nt * q8_xs_stride(cps) + (size_t)8 * nt * (cps + 1)) * 4;
}

template <int NT, int MT, int S>
__global__ void __launch_bounds__(kQ8XsWarps * 32, 1) q8_linear_xs_kernel(const Q8Args args) {
  constexpr int TR = 8 * NT;  // staged token rows
  extern __shared__ __align__(16) uint32_t xs[];
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const Q8View a = q8_view(args, blockIdx.y);
  const int nchunks = a.cols / kQ8Chunk;
  const int cps = args.chunks_per_split;
  const int sp = blockIdx.x;
  const int c0 = sp * cps, c1 = min(nchunks, c0 + cps);
  const int stride = q8_xs_stride(cps);
  uint32_t* xs_h = xs;
  uint32_t* xs_l = xs + TR * stride;
  float* xs_s = reinterpret_cast<float*>(xs + 2 * TR * stride);  // [TR][cps + 1]
  const int rows_cta = kQ8XsWarps * 16 * MT;
  const int row0 = a.rb * rows_cta + warp * 16 * MT;

  Q8Base<NT, MT> b;
  b.row8 = 8LL * a.cols;
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    b.live[m] = row0 + 16 * m < a.rows;
    b.fa[m] = (long long)(row0 + 16 * m + g) * a.cols + 16 * c;
  }
  Q8W<MT> w[S];
  int ch = c0;
  // the first S - 1 chunks' weights do not depend on the x split
#pragma unroll
  for (int s = 0; s < S - 1; ++s)
    if (ch + s < c1) q8_load_w<NT, MT>(a, b, ch + s, w[s]);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // stage the range's x: TR token rows of hi and lo words (zero past n_tokens)
  // and their chunk sums
  {
    const int q4 = (c1 - c0) * 8;  // 16-byte words per token row
    const size_t xrow = (size_t)a.cols / 2;
    for (int i = threadIdx.x; i < TR * q4; i += blockDim.x) {
      const int t = i / q4, k = (i - t * q4) * 4;
      uint4 h = make_uint4(0, 0, 0, 0), l = make_uint4(0, 0, 0, 0);
      if (t < a.n_tokens) {
        h = __ldg(reinterpret_cast<const uint4*>(args.xh + t * xrow + (size_t)c0 * 32 + k));
        l = __ldg(reinterpret_cast<const uint4*>(args.xl + t * xrow + (size_t)c0 * 32 + k));
      }
      *reinterpret_cast<uint4*>(xs_h + t * stride + k) = h;
      *reinterpret_cast<uint4*>(xs_l + t * stride + k) = l;
    }
    for (int i = threadIdx.x; i < TR * (c1 - c0); i += blockDim.x) {
      const int t = i / (c1 - c0), k = i - t * (c1 - c0);
      xs_s[t * (cps + 1) + k] = t < a.n_tokens ? __ldg(args.xsum + (size_t)t * nchunks + c0 + k) : 0.f;
    }
  }
  __syncthreads();

  float acc[MT][NT][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[m][n][e] = 0.f;
  while (ch < c1) {
#pragma unroll
    for (int s = 0; s < S; ++s) {
      if (ch >= c1) break;
      const int nx = ch + S - 1;
      if (nx < c1) q8_load_w<NT, MT>(a, b, nx, w[(s + S - 1) % S]);
      const int cl = ch - c0;
      Q8X<NT> xf;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const uint32_t* ph = xs_h + (8 * n + g) * stride + cl * 32 + 8 * c;
        const uint32_t* pl = xs_l + (8 * n + g) * stride + cl * 32 + 8 * c;
        const uint4 h0 = *reinterpret_cast<const uint4*>(ph), h1 = *reinterpret_cast<const uint4*>(ph + 4);
        const uint4 l0 = *reinterpret_cast<const uint4*>(pl), l1 = *reinterpret_cast<const uint4*>(pl + 4);
        xf.bh[n][0] = h0.x; xf.bh[n][1] = h0.y; xf.bh[n][2] = h0.z; xf.bh[n][3] = h0.w;
        xf.bh[n][4] = h1.x; xf.bh[n][5] = h1.y; xf.bh[n][6] = h1.z; xf.bh[n][7] = h1.w;
        xf.bl[n][0] = l0.x; xf.bl[n][1] = l0.y; xf.bl[n][2] = l0.z; xf.bl[n][3] = l0.w;
        xf.bl[n][4] = l1.x; xf.bl[n][5] = l1.y; xf.bl[n][6] = l1.z; xf.bl[n][7] = l1.w;
        xf.x0[n] = xs_s[(8 * n + 2 * c) * (cps + 1) + cl];
        xf.x1[n] = xs_s[(8 * n + 2 * c + 1) * (cps + 1) + cl];
      }
      q8_compute_chunk<NT, MT>(w[s], xf, acc);
      ++ch;
    }
  }

  // each warp owns its rows: write y, or this range's partial sums
  const int tp = 8 * NT;
  float* part = a.part + (size_t)sp * tp * a.rows;
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = row0 + 16 * m + g + ((e & 2) ? 8 : 0);
        const int tok = 8 * n + 2 * c + (e & 1);
        if (row >= a.rows || tok >= a.n_tokens) continue;
        if (a.splits == 1)
          a.y[(size_t)tok * a.rows + row] = q8_epilogue(a, tok, row, acc[m][n][e]);
        else
          part[(size_t)tok * a.rows + row] = acc[m][n][e];
      }
  if (a.splits == 1) return;
  // the last CTA of this row group sums the ranges in order
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atom_add_acq_rel_gpu(&args.counters[blockIdx.y], 1u);
    s_last = (prev == (unsigned)a.splits - 1);
  }
  __syncthreads();
  if (!s_last) return;
  const int rg0 = a.rb * rows_cta;
  for (int i = threadIdx.x; i < rows_cta * a.n_tokens; i += blockDim.x) {
    const int tok = i / rows_cta, row = rg0 + i % rows_cta;
    if (row >= a.rows) continue;
    float v = 0.f;
    for (int s = 0; s < a.splits; ++s) v += __ldcg(a.part + ((size_t)s * tp + tok) * a.rows + row);
    a.y[(size_t)tok * a.rows + row] = q8_epilogue(a, tok, row, v);
  }
  if (threadIdx.x == 0) args.counters[blockIdx.y] = 0;
}

// ------------------------------------------------------------------ RMSNorm
// out[t] = x[t] / sqrt(mean(x[t]^2) + eps) * w  (GhostRMSNorm::forward,
// src/oomllama.rs:200-211), f32.  One CTA per token: the sum of squares is a
// fixed-order block reduction; the division and square root are IEEE.
constexpr int kNormThreads = 256;
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(const float* __restrict__ x,
                                                               const float* __restrict__ w, float eps, int hidden,
                                                               float* __restrict__ out) {
  __shared__ float part[kNormThreads / 32];
  const int t = blockIdx.x;
  const float* xr = x + (size_t)t * hidden;
  float s = 0.f;
#pragma unroll 4  // the loads go out together; the sum keeps its order
  for (int i = threadIdx.x * 4; i < hidden; i += kNormThreads * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) s += __shfl_xor_sync(0xffffffffu, s, d);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < kNormThreads / 32; ++k) tot += part[k];
  const float denom = sqrtf(tot / (float)hidden + eps);
  float* orow = out + (size_t)t * hidden;
  for (int i = threadIdx.x * 4; i < hidden; i += kNormThreads * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    const float4 g = *reinterpret_cast<const float4*>(w + i);
    *reinterpret_cast<float4*>(orow + i) =
        make_float4(v.x / denom * g.x, v.y / denom * g.y, v.z / denom * g.z, v.w / denom * g.w);
  }
}

// RMSNorm fused into the x split of the linear that reads it: CTAs (token,
// group of 8 chunks) each form the row's sum of squares exactly as
// rmsnorm_kernel does, then their warps split the normalised row
// x / sqrt(mean(x^2) + eps) * w chunk by chunk exactly as q8_prep_x_kernel does.  The normalised row itself is not
// stored: only the linears read it (src/oomllama.rs:389, :395, :549).
__global__ void __launch_bounds__(kNormThreads) rmsnorm_prep_x_kernel(const float* __restrict__ x,
                                                                      const float* __restrict__ w, float eps,
                                                                      int cols, uint32_t* xh, uint32_t* xl,
                                                                      float* xsum, int* status) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // as in q8_prep_x_kernel
  __shared__ float part[kNormThreads / 32];
  const int t = blockIdx.x;
  const float* xr = x + (size_t)t * cols;
  float s = 0.f;
#pragma unroll 4  // the loads go out together; the sum keeps its order
  for (int i = threadIdx.x * 4; i < cols; i += kNormThreads * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) s += __shfl_xor_sync(0xffffffffu, s, d);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < kNormThreads / 32; ++k) tot += part[k];
  const float denom = sqrtf(tot / (float)cols + eps);
  const int lane = threadIdx.x & 31;
  const int nchunks = cols / kQ8Chunk;
  // blockIdx.y picks this CTA's 8 chunks: every CTA of a token forms the same
  // sum of squares (read from L2), so a token's split is spread over several SMs
  for (int ch = blockIdx.y * (kNormThreads / 32) + (threadIdx.x >> 5); ch < nchunks;
       ch += gridDim.y * (kNormThreads / 32)) {
    const int c = ch * kQ8Chunk + 2 * lane;
    const float2 xv = *reinterpret_cast<const float2*>(xr + c);
    const float2 g = *reinterpret_cast<const float2*>(w + c);
    const float2 v = make_float2(xv.x / denom * g.x, xv.y / denom * g.y);
    const __half2 hi = __floats2half2_rn(v.x, v.y);
    const float2 hf = __half22float2(hi);
    const __half2 lo = __floats2half2_rn(v.x - hf.x, v.y - hf.y);
    if (!(fabsf(v.x) < 65504.f) || !(fabsf(v.y) < 65504.f)) report_error(status, kDevErrX16);
    const size_t o = (size_t)t * (cols / 2) + ch * (kQ8Chunk / 2) + lane;
    xh[o] = *reinterpret_cast<const uint32_t*>(&hi);
    xl[o] = *reinterpret_cast<const uint32_t*>(&lo);
    float cs = v.x + v.y;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) cs += __shfl_xor_sync(0xffffffffu, cs, d);
    if (lane == 0) xsum[(size_t)t * nchunks + ch] = cs;
  }
}

// ---------------------------------------------------------- .oom block repack
// A Q8 tensor's block stream as the .oom writer lays it down
// (src/gguf2oom.rs:782-829): block b = [f32 scale][f32 min][u32 len][len bytes]
// with len = min(256, n - 256 b), so block b starts at byte 268 b.  One warp
// per block: lane l moves bytes 8l..8l+7 of the block's data into q and lane 0
// the scale and min.  The stream may start at any byte (a tensor inside a
// whole uploaded file): words are read 4-byte aligned and funnel-shifted.  A
// length field that disagrees with the block's position is reported.
constexpr int kQ8BlockBytes = 12 + 256;

__device__ __forceinline__ uint32_t oom_word(const uint32_t* base_w, uint32_t shift, long long byte_off) {
  // 4 bytes starting at byte_off of a stream whose first byte lies `shift` bytes into base_w[0]
  const long long b = byte_off + shift;
  const uint32_t lo = base_w[b >> 2];
  if ((b & 3) == 0) return lo;  // the next word is read only when the 4 bytes reach into it
  return __funnelshift_r(lo, base_w[(b >> 2) + 1], (uint32_t)(b & 3) * 8);
}

__global__ void q8_repack_kernel(const uint32_t* __restrict__ base_w, uint32_t shift, long long n_values,
                                 long long n_blocks, uint8_t* __restrict__ q, float* __restrict__ scale,
                                 float* __restrict__ mn, int* status) {
  const long long blk = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (blk >= n_blocks) return;
  const int lane = threadIdx.x & 31;
  const long long off = blk * kQ8BlockBytes;
  const int len = (int)min(256LL, n_values - blk * 256);
  if (lane == 0) {
    scale[blk] = __uint_as_float(oom_word(base_w, shift, off));
    mn[blk] = __uint_as_float(oom_word(base_w, shift, off + 4));
    if ((int)oom_word(base_w, shift, off + 8) != len) report_error(status, kDevErrFormat);
  }
  const int b0 = lane * 8;
  if (b0 >= len) return;
  uint8_t* dst = q + blk * 256 + b0;
  if (b0 + 8 <= len) {
    const uint32_t w0 = oom_word(base_w, shift, off + 12 + b0), w1 = oom_word(base_w, shift, off + 16 + b0);
    *reinterpret_cast<uint2*>(dst) = make_uint2(w0, w1);  // q is 8-byte aligned per lane (blocks of 256)
  } else {
    for (int i = b0; i < len; ++i) {
      const long long b = off + 12 + i + shift;
      dst[i - b0] = (uint8_t)(base_w[b >> 2] >> ((b & 3) * 8));
    }
  }
}

// ------------------------------------------------------------------ embedding, argmax
// out[t] = row ids[t] of a Q8 matrix [vocab][hidden], dequantised exactly as
// the reference reads a Q8 tensor (min + (f32)q * scale, src/quant.rs:201-224),
// the embedding gather of src/oomllama.rs:508-515.  One CTA per token.  A
// token id outside [0, vocab) is reported and gives a zero row.
__global__ void embed_q8_kernel(const uint8_t* __restrict__ q, const float* __restrict__ scale,
                                const float* __restrict__ mn, int vocab, int hidden, const int* __restrict__ ids,
                                float* __restrict__ out, int* status) {
  const int t = blockIdx.x;
  const int id = ids[t];
  float* orow = out + (size_t)t * hidden;
  if ((unsigned)id >= (unsigned)vocab) {
    if (threadIdx.x == 0) report_error(status, kDevErrBounds);
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) orow[i] = 0.f;
    return;
  }
  const long long base = (long long)id * hidden;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    const long long f = base + i;
    orow[i] = __fadd_rn(mn[f >> 8], __fmul_rn((float)q[f], scale[f >> 8]));
  }
}

// ids[r] = argmax over logits[r][0..n) (the greedy pick, src/oomllama.rs:973-976,
// :1000-1003, i.e. candle-core 0.9.1's argmax: a scan from element 0 that moves
// only to a strictly larger value).  So: the largest value, the lowest index
// among equal ones, NaN skipped -- except that a NaN in element 0 is never left
// and gives 0.  Two stages: CTAs (chunk, row) reduce ranges of a row to
// (value, index) pairs, then one CTA per row reduces those.  "Larger value,
// then lower index" is associative and commutative, so the result does not
// depend on how the row is cut.
constexpr int kArgmaxThreads = 256;

__device__ __forceinline__ void argmax_take(float& bv, int& bi, float v, int i, int none) {
  if (i != none && (bi == none || v > bv || (v == bv && i < bi))) {
    bv = v;
    bi = i;
  }
}

// (value, index) of the whole block; valid in thread 0.  `none` marks "no candidate".
__device__ __forceinline__ void argmax_block(float& bv, int& bi, int none) {
  __shared__ float sv[kArgmaxThreads / 32];
  __shared__ int si[kArgmaxThreads / 32];
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, d);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, d);
    argmax_take(bv, bi, ov, oi, none);
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = bv;
    si[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0)
    for (int k = 1; k < (int)(blockDim.x >> 5); ++k) argmax_take(bv, bi, sv[k], si[k], none);
}

__global__ void __launch_bounds__(kArgmaxThreads) argmax_partial_kernel(const float* __restrict__ logits, int n,
                                                                        int chunk, float* part_v, int* part_i) {
  const int r = blockIdx.y, c = blockIdx.x;
  const float* row = logits + (size_t)r * n;
  const int b = c * chunk, e = min(n, b + chunk);
  float bv = -INFINITY;
  int bi = n;  // none yet
  for (int i = b + threadIdx.x; i < e; i += blockDim.x) {
    const float v = row[i];
    if (v == v) argmax_take(bv, bi, v, i, n);  // NaN is never larger
  }
  argmax_block(bv, bi, n);
  if (threadIdx.x == 0) {
    part_v[(size_t)r * gridDim.x + c] = bv;
    part_i[(size_t)r * gridDim.x + c] = bi;
  }
}

__global__ void __launch_bounds__(kArgmaxThreads) argmax_final_kernel(const float* __restrict__ logits, int n,
                                                                      int chunks, const float* part_v,
                                                                      const int* part_i, int* __restrict__ ids) {
  const int r = blockIdx.x;
  float bv = -INFINITY;
  int bi = n;
  for (int c = threadIdx.x; c < chunks; c += blockDim.x)
    argmax_take(bv, bi, part_v[(size_t)r * chunks + c], part_i[(size_t)r * chunks + c], n);
  argmax_block(bv, bi, n);
  if (threadIdx.x == 0) {
    const float first = logits[(size_t)r * n];
    ids[r] = (bi == n || first != first) ? 0 : bi;
  }
}

}  // namespace oomattn
