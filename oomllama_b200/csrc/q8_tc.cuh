// K-E, tensor-core form for decode-sized token counts on large matrices:
// y[t][r] = sum_c x[t][c] W[r][c] (+ bias) (+ residual) for up to 16 tokens,
// W resident as Q8 (BlockQ8View::dequantize_fast, src/quant.rs:201-224), on the
// integer tensor cores (tcgen05.mma kind::i8, u8 x u8 -> s32, exact).
//
// The weight bytes enter the MMA as they are stored: A = q (u8), straight from
// the TMA-loaded shared-memory tile, with no conversion.  x is written by
// q8_digits_kernel as three base-128 digits per value relative to the largest
// magnitude sx of its 256-column block (per token):
//   x = sx / 127 * (e0 + e1 / 128 + e2 / 16384),  e0 in [-127, 127], e1, e2 in [-64, 64]
// (about 21 significant bits of sx), each digit stored as e + 128 (u8).  B
// has 64 rows: digit d of token t in row 16 d + t, and row 48 all ones, so the
// MMA also forms S = sum q, and every 256-column block's contribution is
//   sum_k q_k x_k = sx / 127 * ((D0 - 128 S) + (D1 - 128 S) / 128 + (D2 - 128 S) / 16384)
//   block: scale * that + min * X_t,   X_t = sum of x over the block,
// the block's affine map applied after its dot product (src/quant.rs:201-224).
// Every D stays below 2^24 (255 * 255 * 256), so the integer sums are exact
// and convert to f32 exactly.
//
//   warp 4       TMA producer (one lane): per stage a [128 rows][128 columns]
//                weight box (16 KB) and the stage's [64 rows][128 columns]
//                digit box (8 KB), 128-byte swizzled, into an 8-stage ring
//                (192 KB in flight per SM)
//   warp 5       MMA issuer (one lane): M = 128 weight rows, N = 64, K = 32:
//                4 MMAs per stage; the D of a 256-column block in one of four
//                TMEM buffers
//   warps 0-3    promoters: thread r holds row r's 16 accumulators; the
//                blocks' token sums and scales sit in shared memory, and each
//                row's block scale and min arrive by cp.async into an 8-deep
//                shared-memory ring ahead of the block's D
// The kernel is persistent: the work is the launch's (row tile, 256-column
// block) units in row-tile order (the matrices of a launch -- q/k/v,
// gate/up -- one after another), and CTA c takes the contiguous range
// [c U / G, (c + 1) U / G) of the U units, so every SM streams the same
// number of weight bytes and its ring runs on from one row tile into the
// next.  A row tile that a range covers whole is written directly; one cut
// between CTAs leaves each CTA's partial sums in its first or last slot, and
// the last CTA to finish the tile adds them in column order, so results do
// not depend on CTA timing.
#pragma once
#include "common.cuh"
#include "prefill.cuh"
#include "q8_linear.cuh"

namespace oomattn {

constexpr int kTcRows = 128;                       // weight rows per row tile (TMEM lanes)
constexpr int kTcCols = 128;                       // columns per stage
constexpr int kTcStages = 8;
constexpr int kTcWBytes = kTcRows * kTcCols;       // 16 KB of Q8 weights per stage
constexpr int kTcXBytes = 64 * kTcCols;            // 8 KB: 64 digit rows x 128 columns
constexpr int kTcStageBytes = kTcWBytes + kTcXBytes;
constexpr int kTcDBufs = 4;                        // D buffers of 64 TMEM columns
constexpr int kTcMaxBlocks = 128;                  // cols <= 32768: the blocks' token operands in shared memory
constexpr int kTcOpBytes = kTcMaxBlocks * 16 * 8;
constexpr int kTcSmAhead = 8;                      // blocks of row scales and minima in flight
constexpr int kTcSmBytes = kTcSmAhead * kTcRows * 8;
constexpr int kTcSmemBytes = kTcStages * kTcStageBytes + kTcOpBytes + kTcSmBytes + 1024 + 256;
constexpr int kTcThreads = 192;
constexpr int kTcMaxMats = 3;
constexpr int kTcDigitRows = 64;                   // B rows: 3 digits x 16 tokens, the ones row, zeros

struct Q8TcMat {
  const float* scale;
  const float* min;
  int rows;               // a multiple of 128
  int rb_begin;           // first row tile of this matrix in the launch's tile order
  const float* bias;      // [rows] or null
  const float* residual;  // [n_tokens][rows] or null (may alias y)
  float* y;               // [n_tokens][rows]
};

struct Q8TcArgs {
  Q8TcMat m[kTcMaxMats];
  int n_mats;
  int cols;
  const float* xsum;      // [16][cols / 64] sums of x per 64-column chunk
  const float* sx;        // [16][cols / 256] each token's largest |x| per 256-column block
  int n_tokens;           // <= 16
  int units;              // row tiles x 256-column blocks
  float* part;            // [gridDim.x][2][16][128]: a CTA's partial first and last row tiles
  unsigned* counters;     // [row tiles]: arrivals at a cut tile, zero between launches
  int* status;
  unsigned long long timeout_ns;
  int test_flags;         // 0 outside tests
};

// CTA c's units start at c U / G; the CTA holding unit u is the last c whose
// start is <= u.
__device__ __forceinline__ int tc_unit_begin(int c, int units, int g) {
  return (int)((long long)c * units / g);
}
__device__ __forceinline__ int tc_cta_of(int u, int units, int g) {
  return (int)(((long long)(u + 1) * g - 1) / units);
}
__device__ __forceinline__ int tc_mat_of(const Q8TcArgs& a, int tile) {
  int mi = 0;
#pragma unroll
  for (int j = 1; j < kTcMaxMats; ++j)
    if (j < a.n_mats && tile >= a.m[j].rb_begin) mi = j;
  return mi;
}
#define OOMATTN_TC_FIELD(a, mi, f) ((mi) == 0 ? (a).m[0].f : ((mi) == 1 ? (a).m[1].f : (a).m[2].f))


// kind::i8 instruction descriptor: s32 accumulate, A and B unsigned 8-bit,
// both K-major, M = 128, N = 64.
__host__ __device__ constexpr uint32_t tc_i8_idesc() {
  return (2u << 4) | ((64u >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi, uint32_t b_lo,
                                          uint32_t b_hi, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "mov.b64 da, {%1, %2};\n\t"
      "mov.b64 db, {%3, %4};\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], da, db, %5, p;\n\t}" ::"r"(d_tmem),
      "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
      : "memory");
}

__global__ void __launch_bounds__(kTcThreads, 1)
    q8_tc_kernel(const __grid_constant__ CUtensorMap wmap0, const __grid_constant__ CUtensorMap wmap1,
                 const __grid_constant__ CUtensorMap wmap2, const __grid_constant__ CUtensorMap dmap,
                 const Q8TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float2* s_op = reinterpret_cast<float2*>(smem + kTcStages * kTcStageBytes);  // [kb][16]: (block sum, sx / 127)
  float2* s_sm = reinterpret_cast<float2*>(smem + kTcStages * kTcStageBytes + kTcOpBytes);  // [kTcSmAhead][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kTcStages * kTcStageBytes + kTcOpBytes + kTcSmBytes);
  uint64_t* full = bars;                   // [kTcStages]: weights + digits of a stage landed
  uint64_t* empty = full + kTcStages;      // [kTcStages]: the stage's MMAs completed
  uint64_t* d_full = empty + kTcStages;    // [kTcDBufs]: a block's D complete
  uint64_t* d_empty = d_full + kTcDBufs;   // [kTcDBufs]: the promoters have read D
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(d_empty + kTcDBufs);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kbt = a.cols / 256;  // 256-column blocks per row tile
  const int u_begin = tc_unit_begin(blockIdx.x, a.units, gridDim.x);
  const int n_blocks = tc_unit_begin(blockIdx.x + 1, a.units, gridDim.x) - u_begin;
  const int n_st = 2 * n_blocks;
  const int tile0 = u_begin / kbt, kb0 = u_begin - tile0 * kbt;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < kTcDBufs; ++b) {
      mbar_init(&d_full[b], 1);
      mbar_init(&d_empty[b], 4);
    }
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, 64 * kTcDBufs);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // D buffer j at column 64 j

  if (warp == 4) {
    // ------------------------------------------------ TMA producer
    // (kTestDropLinearCopies: a test makes the MMA issuer's and promoters'
    // bounded waits run out by issuing nothing; they record kDevErrTimeout.)
    if (lane == 0 && !(a.test_flags & kTestDropLinearCopies)) {
      prefetch_tensormap(&wmap0);
      if (a.n_mats > 1) prefetch_tensormap(&wmap1);
      if (a.n_mats > 2) prefetch_tensormap(&wmap2);
      prefetch_tensormap(&dmap);
      // stage i: block i / 2 of the range, its (i % 2)-th 128 columns
      int tile = tile0, kb = kb0, half = 0;
      auto issue_w = [&](int s) {
        const int mi = tc_mat_of(a, tile);
        const CUtensorMap* wm = mi == 0 ? &wmap0 : (mi == 1 ? &wmap1 : &wmap2);
        const int r0 = (tile - OOMATTN_TC_FIELD(a, mi, rb_begin)) * kTcRows;
        tma_load_2d(smem + s * kTcStageBytes, wm, &full[s], kb * 256 + half * kTcCols, r0);
      };
      auto advance = [&]() {
        half ^= 1;
        if (!half && ++kb == kbt) {
          kb = 0;
          ++tile;
        }
      };
      // the first stages' weights go out before the digit split this kernel
      // depends on has finished (programmatic dependent launch)
      const int pre = min(n_st, kTcStages);
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], kTcStageBytes);
        issue_w(i);
        advance();
      }
      asm volatile("griddepcontrol.wait;" ::: "memory");
      for (int i = 0; i < pre; ++i) {
        const int u = u_begin + (i >> 1), kbi = u % kbt;
        tma_load_2d(smem + i * kTcStageBytes + kTcWBytes, &dmap, &full[i], kbi * 256 + (i & 1) * kTcCols, 0);
      }
      int issued = pre;
      for (int i = pre; i < n_st; ++i) {
        const int s = i % kTcStages;
        if (!mbar_wait(&empty[s], ((i / kTcStages) - 1) & 1, a.status, a.timeout_ns)) break;
        mbar_arrive_expect_tx(&full[s], kTcStageBytes);
        issue_w(s);
        tma_load_2d(smem + s * kTcStageBytes + kTcWBytes, &dmap, &full[s], kb * 256 + half * kTcCols, 0);
        advance();
        issued = i + 1;
      }
      // drain: the last copies this lane issued land before the CTA can exit
      for (int i = max(0, issued - kTcStages); i < issued; ++i)
        mbar_wait(&full[i % kTcStages], (i / kTcStages) & 1, a.status, a.timeout_ns);
    }
  } else if (warp == 5) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = tc_i8_idesc();
      const uint64_t d0 = make_sdesc(smem_u32(smem), 16, 1024);
      const uint32_t dlo = (uint32_t)d0, dhi = (uint32_t)(d0 >> 32);
      bool ok = true;
      for (int i = 0; i < n_st && ok; ++i) {
        const int s = i % kTcStages, b = i >> 1, first = (i & 1) == 0;
        const int db = b % kTcDBufs;
        ok = mbar_wait(&full[s], (i / kTcStages) & 1, a.status, a.timeout_ns);
        if (ok && first && b >= kTcDBufs)
          ok = mbar_wait(&d_empty[db], ((b / kTcDBufs) - 1) & 1, a.status, a.timeout_ns);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + 64 * db;
        const uint32_t wa = dlo + (uint32_t)((s * kTcStageBytes) >> 4);
        const uint32_t xb = wa + (uint32_t)(kTcWBytes >> 4);
#pragma unroll
        for (int kk = 0; kk < kTcCols / 32; ++kk)  // 32 columns (bytes) per k-step of the 128-byte row
          mma_i8_ss(d, wa + kk * 2, dhi, xb + kk * 2, dhi, idesc, (first && kk == 0) ? 0u : 1u);
        tc_commit(&empty[s]);
        if (!first) tc_commit(&d_full[db]);
      }
    }
  } else {
    // ------------------------------------------------ promoters (warps 0-3)
    const int r = warp * 32 + lane;  // weight row within the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    asm volatile("griddepcontrol.wait;" ::: "memory");  // sx and xsum come from the digit split
    // the next kernel may launch now; it waits for this grid before it
    // touches anything this one reads or writes
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    // only the blocks of this CTA's range: kb0, kb0 + 1, ... (mod kbt)
    const int n_kb = min(n_blocks, kbt);
#pragma unroll 4
    for (int i = threadIdx.x; i < n_kb * 16; i += 128) {
      int kb = kb0 + (i >> 4);
      if (kb >= kbt) kb -= kbt;
      const int t = i & 15;
      float2 v = make_float2(0.f, 0.f);
      if (t < a.n_tokens) {
        const float4 x4 = __ldg(reinterpret_cast<const float4*>(a.xsum + (size_t)t * (a.cols / 64) + 4 * kb));
        v = make_float2((x4.x + x4.y) + (x4.z + x4.w), __ldg(a.sx + (size_t)t * kbt + kb) * (1.f / 127.f));
      }
      s_op[kb * 16 + t] = v;
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    // this row's scale and min of block b go to ring slot b % kTcSmAhead, one
    // cp.async group per block (empty past the range), kTcSmAhead - 1 blocks
    // ahead of the block being promoted; each thread reads only what it copied
    int p_tile = tile0, p_kb = kb0;
    auto fetch = [&](int b) {
      if (b < n_blocks) {
        const int mi = tc_mat_of(a, p_tile);
        const size_t blk = (size_t)((p_tile - OOMATTN_TC_FIELD(a, mi, rb_begin)) * kTcRows + r) * kbt + p_kb;
        float2* dst = s_sm + (b % kTcSmAhead) * kTcRows + r;
        cp_async4(&dst->x, OOMATTN_TC_FIELD(a, mi, scale) + blk);
        cp_async4(&dst->y, OOMATTN_TC_FIELD(a, mi, min) + blk);
        if (++p_kb == kbt) {
          p_kb = 0;
          ++p_tile;
        }
      }
      cp_async_commit();
    };
#pragma unroll 1
    for (int b = 0; b < kTcSmAhead - 1; ++b) fetch(b);
    float acc[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) acc[t] = 0.f;
    __shared__ int s_last;
    int tile = tile0, kb = kb0;
    bool ok = true;
    for (int b = 0; b < n_blocks; ++b) {
      fetch(b + kTcSmAhead - 1);
      cp_async_wait<kTcSmAhead - 1>();  // block b's group has landed
      const float2 scmn = s_sm[(b % kTcSmAhead) * kTcRows + r];
      const float sc = scmn.x, mn = scmn.y;
      const int db = b % kTcDBufs;
      ok = mbar_wait(&d_full[db], (b / kTcDBufs) & 1, a.status, a.timeout_ns);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t dr[64];
      OOMATTN_TMEM_LD32(tmem + lane_off + 64 * db, dr);
      OOMATTN_TMEM_LD32(tmem + lane_off + 64 * db + 32, (dr + 32));
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&d_empty[db]);
      const float4* op = reinterpret_cast<const float4*>(s_op + kb * 16);
      const int s128 = 128 * (int)dr[48];  // 128 x the sum of the block's q of this row
#pragma unroll
      for (int t2 = 0; t2 < 8; ++t2) {
        const float4 xu = op[t2];  // (X, unit) of tokens 2 t2 and 2 t2 + 1
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int t = 2 * t2 + h;
          const float X = h ? xu.z : xu.x, unit = h ? xu.w : xu.y;
          const float e0 = (float)((int)dr[t] - s128), e1 = (float)((int)dr[16 + t] - s128);
          const float e2 = (float)((int)dr[32 + t] - s128);
          const float dot = unit * (e0 + (e1 * (1.f / 128.f) + e2 * (1.f / 16384.f)));
          acc[t] = fmaf(sc, dot, fmaf(mn, X, acc[t]));
        }
      }
      if (kb == kbt - 1 || b == n_blocks - 1) {
        // ---------------------------------------------- the end of a row tile's segment
        const int mi = tc_mat_of(a, tile);
        const int rows = OOMATTN_TC_FIELD(a, mi, rows);
        const int R = (tile - OOMATTN_TC_FIELD(a, mi, rb_begin)) * kTcRows + r;
        const float* bias = OOMATTN_TC_FIELD(a, mi, bias);
        const float* residual = OOMATTN_TC_FIELD(a, mi, residual);
        float* y = OOMATTN_TC_FIELD(a, mi, y);
        const int seg_kb0 = tile == tile0 ? kb0 : 0;
        if (seg_kb0 == 0 && kb == kbt - 1) {
#pragma unroll
          for (int t = 0; t < 16; ++t) {
            if (t < a.n_tokens) {
              float v = acc[t];
              if (bias) v += bias[R];
              if (residual) v += residual[(size_t)t * rows + R];
              y[(size_t)t * rows + R] = v;
            }
          }
        } else {
          float* pp = a.part + ((size_t)blockIdx.x * 2 + (tile == tile0 ? 0 : 1)) * 16 * kTcRows;
#pragma unroll
          for (int t = 0; t < 16; ++t)
            if (t < a.n_tokens) pp[t * kTcRows + r] = acc[t];
          const int c_lo = tc_cta_of(tile * kbt, a.units, gridDim.x);
          const int c_hi = tc_cta_of(tile * kbt + kbt - 1, a.units, gridDim.x);
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (r == 0) s_last = atom_add_acq_rel_gpu(&a.counters[tile], 1u) == (unsigned)(c_hi - c_lo);
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (s_last) {
            // the last CTA of the tile adds its segments in column order;
            // two segments' 16 token sums are loaded together, this CTA's
            // own taken from its registers
            auto seg = [&](int c, float* p) {
              if (c > c_hi) {
#pragma unroll
                for (int t = 0; t < 16; ++t) p[t] = 0.f;
              } else if (c == (int)blockIdx.x) {
#pragma unroll
                for (int t = 0; t < 16; ++t) p[t] = acc[t];
              } else {
                const int slot = tc_unit_begin(c, a.units, gridDim.x) >= tile * kbt ? 0 : 1;
                const float* pc = a.part + ((size_t)c * 2 + slot) * 16 * kTcRows + r;
#pragma unroll
                for (int t = 0; t < 16; ++t) p[t] = t < a.n_tokens ? __ldcg(pc + t * kTcRows) : 0.f;
              }
            };
            float v[16];
#pragma unroll
            for (int t = 0; t < 16; ++t) v[t] = 0.f;
            for (int c = c_lo; c <= c_hi; c += 2) {
              float p0[16], p1[16];
              seg(c, p0);
              seg(c + 1, p1);
#pragma unroll
              for (int t = 0; t < 16; ++t) v[t] = (v[t] + p0[t]) + p1[t];
            }
#pragma unroll
            for (int t = 0; t < 16; ++t) {
              if (t < a.n_tokens) {
                float o = v[t];
                if (bias) o += bias[R];
                if (residual) o += residual[(size_t)t * rows + R];
                y[(size_t)t * rows + R] = o;
              }
            }
            if (r == 0) a.counters[tile] = 0u;
          }
        }
#pragma unroll
        for (int t = 0; t < 16; ++t) acc[t] = 0.f;
      }
      if (++kb == kbt) {
        kb = 0;
        ++tile;
      }
    }
    cp_async_wait<0>();  // no copy into this CTA's shared memory outlives it
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 64 * kTcDBufs);
  }
}

// The x split of the integer form, for up to 16 tokens: CTAs (token slot,
// group of 8 256-column blocks), one warp per block.  The row the linear reads
// -- x, x RMS-normalised with weight w (the row's sum of squares formed by
// every CTA exactly as rmsnorm_kernel forms it), or the gated activation
// silu(x) * up (as q8_prep_x_kernel forms it) -- gives per block its largest
// magnitude sx, three base-128 digits per value (+128, u8) into rows t, 16 + t
// and 32 + t of digits [64][cols], and its sums over each 64-column chunk (a
// fixed shuffle tree).  A slot past n_tokens writes zero digits (128).  The
// CTAs of slot 0 also write the ones row (48) and the zero rows (49-63) of
// their columns.  A non-finite value is reported through the status word.
constexpr int kDigitBlocksPerCta = 8;
__global__ void __launch_bounds__(256) q8_digits_kernel(const float* __restrict__ x, const float* __restrict__ up,
                                                        const float* __restrict__ norm_w, float eps, int n_tokens,
                                                        int cols, uint8_t* __restrict__ digits,
                                                        float* __restrict__ xsum, float* __restrict__ sx,
                                                        int* status) {
  // launched as a programmatic dependent of the kernel before it: x, and the
  // digit buffers the previous pass may still read, are touched only after it
  // ends; then the tensor-core pass may launch (one kernel of lookahead)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ float red[8];
  const int t = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, wp = tid >> 5;
  const int kb_total = cols / 256;
  const int kb = blockIdx.y * kDigitBlocksPerCta + wp;  // this warp's 256-column block
  const bool has_block = kb < kb_total;
  const int c0 = kb * 256 + lane * 8;  // this lane's 8 columns
  if (t == 0 && has_block) {
#pragma unroll
    for (int rr = 48; rr < 64; ++rr)
      *reinterpret_cast<uint2*>(digits + (size_t)rr * cols + c0) =
          rr == 48 ? make_uint2(0x01010101u, 0x01010101u) : make_uint2(0u, 0u);
  }
  if (t >= n_tokens) {
    if (has_block)
#pragma unroll
      for (int d = 0; d < 3; ++d)
        *reinterpret_cast<uint2*>(digits + (size_t)(16 * d + t) * cols + c0) = make_uint2(0x80808080u, 0x80808080u);
    return;
  }
  const float* xr = x + (size_t)t * cols;
  float denom = 1.f;
  if (norm_w) {
    // the sum of squares exactly as rmsnorm_kernel forms it (every CTA of the token forms it)
    float s = 0.f;
#pragma unroll 4  // the loads go out together; the sum keeps its order
    for (int i = tid * 4; i < cols; i += 256 * 4) {
      const float4 v = *reinterpret_cast<const float4*>(xr + i);
      s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) s += __shfl_xor_sync(0xffffffffu, s, d);
    if (lane == 0) red[wp] = s;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) tot += red[k];
    denom = sqrtf(tot / (float)cols + eps);
  }
  if (!has_block) return;
  float v[8];
  {
    const float4 p = *reinterpret_cast<const float4*>(xr + c0), q = *reinterpret_cast<const float4*>(xr + c0 + 4);
    v[0] = p.x; v[1] = p.y; v[2] = p.z; v[3] = p.w; v[4] = q.x; v[5] = q.y; v[6] = q.z; v[7] = q.w;
  }
  if (norm_w) {
    const float4 p = *reinterpret_cast<const float4*>(norm_w + c0), q = *reinterpret_cast<const float4*>(norm_w + c0 + 4);
    const float w8[8] = {p.x, p.y, p.z, p.w, q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = v[i] / denom * w8[i];
  }
  if (up) {
    const float* ur = up + (size_t)t * cols + c0;
    const float4 p = *reinterpret_cast<const float4*>(ur), q = *reinterpret_cast<const float4*>(ur + 4);
    const float u8[8] = {p.x, p.y, p.z, p.w, q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = v[i] * (1.f / (1.f + expf(-v[i]))) * u8[i];
  }
  float mx = 0.f;
  bool bad = false;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    bad |= !(fabsf(v[i]) <= 3.0e38f);
    mx = fmaxf(mx, fabsf(v[i]));
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, d));
  if (bad) report_error(status, kDevErrX16);
  if (lane == 0) sx[(size_t)t * kb_total + kb] = mx;
  const float k127 = mx > 0.f ? 127.f / mx : 0.f;
  uint32_t e[3][2] = {{0u, 0u}, {0u, 0u}, {0u, 0u}};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float z = v[i] * k127;
    const float d0 = fminf(127.f, fmaxf(-127.f, rintf(z)));
    const float r1 = (z - d0) * 128.f;
    const float d1 = fminf(64.f, fmaxf(-64.f, rintf(r1)));
    const float r2 = (r1 - d1) * 128.f;
    const float d2 = fminf(64.f, fmaxf(-64.f, rintf(r2)));
    e[0][i >> 2] |= (uint32_t)((int)d0 + 128) << (8 * (i & 3));
    e[1][i >> 2] |= (uint32_t)((int)d1 + 128) << (8 * (i & 3));
    e[2][i >> 2] |= (uint32_t)((int)d2 + 128) << (8 * (i & 3));
  }
#pragma unroll
  for (int d = 0; d < 3; ++d)
    *reinterpret_cast<uint2*>(digits + (size_t)(16 * d + t) * cols + c0) = make_uint2(e[d][0], e[d][1]);
  // the 64-column chunk sums: lanes 8j..8j+7 hold chunk j of the block
  float s = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
#pragma unroll
  for (int d = 4; d > 0; d >>= 1) s += __shfl_xor_sync(0xffffffffu, s, d);
  if ((lane & 7) == 0) xsum[(size_t)t * (cols / 64) + kb * 4 + (lane >> 3)] = s;
}

}  // namespace oomattn
