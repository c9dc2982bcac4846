// K-E, tensor-core form for decode-sized token counts on large matrices:
// y[t][r] = sum_c x[t][c] W[r][c] (+ bias) (+ residual) for up to 16 tokens,
// W resident as Q8 (BlockQ8View::dequantize_fast, src/quant.rs:201-224), with
// the arithmetic of q8_linear_kernel: A = 1024 + q as fp16 (exact), x split
// into fp16 hi + lo, and per 256-value block of a row
//   sum_k x_k (min + q_k s) = s * D + (min - 1024 s) * X,   D = sum_k (1024 + q_k) x_k.
//
// The pass is HBM-bound: every weight byte is read once, so what matters is
// how many bytes are in flight and how little each byte costs on the SM.
//   warp 12      TMA producer (one lane): per stage a [128 rows][128 columns]
//                Q8 weight box (16 KB, 128-byte swizzled) and the stage's x
//                hi/lo boxes ([16 tokens][64 columns] fp16, 4 x 2 KB), into an
//                8-stage ring (192 KB in flight per SM).  A token past n_tokens
//                reads as zero (the x maps end there).
//   warps 0-7    converters in two groups of four (one warp per TMEM lane
//                quarter each) taking alternate stages: thread r reads weight
//                row r's 128 bytes of the stage from shared memory
//                (conflict-free under the swizzle), forms 1024 + q as fp16
//                pairs with one byte permute per pair, and writes them straight
//                into TMEM as the MMA's A operand (tcgen05.st; four 64-column
//                slots), so the fp16 weights never touch shared memory.
//   warps 8-11   promoters: thread r holds row r's accumulators and adds each
//                finished 256-column block, acc[t] += s (D_hi[t] + D_lo[t]) +
//                c X[t], with the block's scale, min and x sums loaded before
//                it waits for the block (their L2 latency kept off the
//                converters' path), then writes the result.
//   warp 13      MMA issuer (one lane): tcgen05.mma kind::f16, M = 128 weight
//                rows, N = 32 (16 tokens x {hi, lo}), K = 16, A from TMEM, B (x)
//                from shared memory; D of a block in one of two TMEM buffers.
// Matrices of a launch (q/k/v, gate/up) split the grid's row tiles; a matrix
// with few row tiles is also split along its columns (grid.y), and the last
// CTA of a row tile to finish adds the splits' partial sums in split order,
// so results do not depend on CTA timing.
#pragma once
#include <cuda_fp16.h>

#include "common.cuh"
#include "prefill.cuh"
#include "q8_linear.cuh"

namespace oomattn {

constexpr int kTcRows = 128;                       // weight rows per CTA (TMEM lanes)
constexpr int kTcCols = 128;                       // columns per stage
constexpr int kTcStages = 8;
constexpr int kTcWBytes = kTcRows * kTcCols;       // 16 KB of Q8 weights per stage
constexpr int kTcXBytes = 32 * kTcCols * 2;        // 8 KB: 16 tokens x {hi, lo} x 128 columns fp16
constexpr int kTcStageBytes = kTcWBytes + kTcXBytes;
constexpr int kTcSmemBytes = kTcStages * kTcStageBytes + 1024 + 256;
constexpr int kTcThreads = 448;
constexpr int kTcSlots = 4;                        // TMEM A slots of 64 columns
constexpr int kTcMaxMats = 3;

struct Q8TcMat {
  const float* scale;
  const float* min;
  int rows;
  int rb_begin;           // first row tile of this matrix in the grid
  const float* bias;      // [rows] or null
  const float* residual;  // [n_tokens][rows] or null (may alias y)
  float* y;               // [n_tokens][rows]
  float* part;            // [splits][16][rows]: split partial sums
};

struct Q8TcArgs {
  Q8TcMat m[kTcMaxMats];
  int n_mats;
  int cols;
  const float* xsum;      // [16][cols / 64] sums of x per 64-column chunk
  int n_tokens;           // <= 16
  int splits;             // column ranges per row tile
  int stages_per_split;   // even: a range holds whole 256-column blocks
  unsigned* counters;     // [row tiles]: arrivals, zero between launches
  int* status;
  unsigned long long timeout_ns;
};

// M = 128, N = 32, fp16 x fp16 -> f32, A from TMEM (K-major), B K-major.
__host__ __device__ constexpr uint32_t tc_idesc() {
  return (1u << 4) | ((32u >> 3) << 17) | ((128u >> 4) << 24);
}

#define OOMATTN_TMEM_LD16(taddr, r)                                                                              \
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, " \
               "[%16];"                                                                                          \
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),  \
                 "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),         \
                 "=r"(r[15])                                                                                     \
               : "r"(taddr))

__global__ void __launch_bounds__(kTcThreads, 1)
    q8_tc_kernel(const __grid_constant__ CUtensorMap wmap0, const __grid_constant__ CUtensorMap wmap1,
                 const __grid_constant__ CUtensorMap wmap2, const __grid_constant__ CUtensorMap xhmap,
                 const __grid_constant__ CUtensorMap xlmap, const Q8TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kTcStages * kTcStageBytes);
  uint64_t* full = bars;                   // [kTcStages]: weights + x of a stage landed
  uint64_t* empty = full + kTcStages;      // [kTcStages]: 4 converter warps + the MMA commit
  uint64_t* a_full = empty + kTcStages;    // [kTcSlots]: a TMEM A slot written (4 converter warps)
  uint64_t* a_empty = a_full + kTcSlots;   // [kTcSlots]: the MMAs reading the slot completed
  uint64_t* d_full = a_empty + kTcSlots;   // [2]: a block's D complete
  uint64_t* d_empty = d_full + 2;          // [2]: the converters have read D
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(d_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // this CTA's matrix and row tile
  const int rb = blockIdx.x;
  int mi = 0;
#pragma unroll
  for (int j = 1; j < kTcMaxMats; ++j)
    if (j < a.n_mats && rb >= a.m[j].rb_begin) mi = j;
  const CUtensorMap* wmap = mi == 0 ? &wmap0 : (mi == 1 ? &wmap1 : &wmap2);
  const Q8TcMat& M = a.m[mi];
  const int r0 = (rb - M.rb_begin) * kTcRows;
  const int split = blockIdx.y;
  const int n_stages_all = a.cols / kTcCols;
  const int s_begin = split * a.stages_per_split;
  const int n_st = max(0, min(n_stages_all - s_begin, a.stages_per_split));
  const int n_blocks = n_st / 2;
  const int kb_total = a.cols / 256;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 5);
    }
    for (int b = 0; b < kTcSlots; ++b) {
      mbar_init(&a_full[b], 4);
      mbar_init(&a_empty[b], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&d_full[b], 1);
      mbar_init(&d_empty[b], 4);
    }
    fence_mbar_init();
  }
  if (warp == 13) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // A slots at columns 0, 64, 128, 192; D buffers at 256 and 288
  constexpr uint32_t kDCol = 64 * kTcSlots;

  if (warp == 12) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tensormap(wmap);
      prefetch_tensormap(&xhmap);
      prefetch_tensormap(&xlmap);
      auto load_x = [&](int i) {
        uint8_t* xs = smem + (i % kTcStages) * kTcStageBytes + kTcWBytes;
        const int c = (s_begin + i) * kTcCols;
        tma_load_2d(xs, &xhmap, &full[i % kTcStages], c, 0);
        tma_load_2d(xs + 2048, &xlmap, &full[i % kTcStages], c, 0);
        tma_load_2d(xs + 4096, &xhmap, &full[i % kTcStages], c + 64, 0);
        tma_load_2d(xs + 6144, &xlmap, &full[i % kTcStages], c + 64, 0);
      };
      // the first stages' weights go out before the x split this kernel
      // depends on has finished (programmatic dependent launch)
      const int pre = min(n_st, kTcStages);
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], kTcStageBytes);
        tma_load_2d(smem + i * kTcStageBytes, wmap, &full[i], (s_begin + i) * kTcCols, r0);
      }
      asm volatile("griddepcontrol.wait;" ::: "memory");
      for (int i = 0; i < pre; ++i) load_x(i);
      int issued = pre;
      for (int i = pre; i < n_st; ++i) {
        const int s = i % kTcStages;
        if (!mbar_wait(&empty[s], ((i / kTcStages) - 1) & 1, a.status, a.timeout_ns)) break;
        mbar_arrive_expect_tx(&full[s], kTcStageBytes);
        tma_load_2d(smem + s * kTcStageBytes, wmap, &full[s], (s_begin + i) * kTcCols, r0);
        load_x(i);
        issued = i + 1;
      }
      for (int i = max(0, issued - kTcStages); i < issued; ++i)
        mbar_wait(&full[i % kTcStages], (i / kTcStages) & 1, a.status, a.timeout_ns);
    }
  } else if (warp == 13) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = tc_idesc();
      const uint64_t d0 = make_sdesc(smem_u32(smem), 16, 1024);
      const uint32_t dlo = (uint32_t)d0, dhi = (uint32_t)(d0 >> 32);
      bool ok = true;
      for (int i = 0; i < n_st && ok; ++i) {
        const int s = i % kTcStages, slot = i % kTcSlots, b = i >> 1, first = (i & 1) == 0;
        ok = mbar_wait(&full[s], (i / kTcStages) & 1, a.status, a.timeout_ns) &&
             mbar_wait(&a_full[slot], (i / kTcSlots) & 1, a.status, a.timeout_ns);
        if (ok && first && b >= 2) ok = mbar_wait(&d_empty[b & 1], ((b >> 1) - 1) & 1, a.status, a.timeout_ns);
        if (!ok) break;
        tc_fence_after();
        const uint32_t d = tmem + kDCol + 32 * (b & 1);
        const uint32_t xs = dlo + (uint32_t)((s * kTcStageBytes + kTcWBytes) >> 4);
#pragma unroll
        for (int kk = 0; kk < kTcCols / 16; ++kk) {
          // B: k-step kk of the [32 rows][64 columns] half (kk / 4), 32 bytes per step
          const uint32_t bd = xs + (uint32_t)((kk >> 2) * (4096 >> 4) + (kk & 3) * 2);
          mma_ts_lh(d, tmem + slot * 64 + kk * 8, bd, dhi, idesc, (first && kk == 0) ? 0u : 1u);
        }
        tc_commit(&a_empty[slot]);
        tc_commit(&empty[s]);
        if (!first) tc_commit(&d_full[b & 1]);
      }
    }
  } else if (warp < 8) {
    // ------------------------------------------------ converters (warps 0-7)
    const int grp = warp >> 2;             // converts the stages i with i % 2 == grp
    const int r = (warp & 3) * 32 + lane;  // weight row within the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t rsw = (uint32_t)(r & 7);
    bool ok = true;
    for (int i = grp; i < n_st && ok; i += 2) {
      const int s = i % kTcStages, slot = i % kTcSlots;
      ok = mbar_wait(&full[s], (i / kTcStages) & 1, a.status, a.timeout_ns);
      if (ok && i >= kTcSlots) ok = mbar_wait(&a_empty[slot], ((i / kTcSlots) - 1) & 1, a.status, a.timeout_ns);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      // row r's 128 weight bytes: 8 chunks of 16, chunk j at position j ^ (r % 8);
      // each half (64 columns) converted and stored to TMEM in turn
      const uint32_t row = smem_u32(smem + s * kTcStageBytes) + (uint32_t)r * 128u;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t w[32];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int j = hf * 4 + jj;
          uint32_t q0, q1, q2, q3;
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(q0), "=r"(q1), "=r"(q2), "=r"(q3)
                       : "r"(row + ((((uint32_t)j) ^ rsw) << 4)));
          const uint32_t qs[4] = {q0, q1, q2, q3};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            w[8 * jj + 2 * u] = __byte_perm(qs[u], 0x64646464u, 0x4140);      // bytes 0, 1 -> 1024 + q
            w[8 * jj + 2 * u + 1] = __byte_perm(qs[u], 0x64646464u, 0x4342);  // bytes 2, 3
          }
        }
        OOMATTN_TMEM_ST32(tmem + lane_off + slot * 64 + hf * 32, w);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&a_full[slot]);
        mbar_arrive(&empty[s]);  // the weights of the stage are read
      }
    }
  } else if (warp < 12) {
    // ------------------------------------------------ promoters (warps 8-11)
    const int r = (warp & 3) * 32 + lane;
    const int R = r0 + r;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    float acc[16];
#pragma unroll
    for (int t = 0; t < 16; ++t) acc[t] = 0.f;
    asm volatile("griddepcontrol.wait;" ::: "memory");  // xsum comes from the x split
    bool ok = true;
    for (int b = 0; b < n_blocks && ok; ++b) {
      // this block's operands first: their latency overlaps the wait for D
      const int kb = s_begin / 2 + b;  // 256-column block within the row
      float sc = 0.f, c = 0.f;
      if (R < M.rows) {
        const size_t blk = (size_t)R * kb_total + kb;
        sc = __ldg(M.scale + blk);
        c = __ldg(M.min + blk) - 1024.f * sc;
      }
      float X[16];
      const float* xs = a.xsum + 4 * kb;
#pragma unroll
      for (int t = 0; t < 16; ++t) {
        if (t < a.n_tokens) {
          const float4 x4 = __ldg(reinterpret_cast<const float4*>(xs + (size_t)t * (a.cols / 64)));
          X[t] = (x4.x + x4.y) + (x4.z + x4.w);
        } else {
          X[t] = 0.f;
        }
      }
      ok = mbar_wait(&d_full[b & 1], (b >> 1) & 1, a.status, a.timeout_ns);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      uint32_t dr[32];
      OOMATTN_TMEM_LD16(tmem + lane_off + kDCol + 32 * (b & 1), dr);
      OOMATTN_TMEM_LD16(tmem + lane_off + kDCol + 32 * (b & 1) + 16, (dr + 16));
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&d_empty[b & 1]);
#pragma unroll
      for (int t = 0; t < 16; ++t)
        acc[t] = fmaf(sc, __uint_as_float(dr[t]) + __uint_as_float(dr[16 + t]), fmaf(c, X[t], acc[t]));
    }
    ok = __all_sync(0xffffffffu, ok);
    // ------------------------------------------------ epilogue
    if (ok && R < M.rows) {
      if (a.splits == 1) {
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          if (t < a.n_tokens) {
            float v = acc[t];
            if (M.bias) v += M.bias[R];
            if (M.residual) v += M.residual[(size_t)t * M.rows + R];
            M.y[(size_t)t * M.rows + R] = v;
          }
        }
      } else {
#pragma unroll
        for (int t = 0; t < 16; ++t)
          if (t < a.n_tokens) M.part[((size_t)split * 16 + t) * M.rows + R] = acc[t];
      }
    }
    if (a.splits > 1) {
      // the last CTA of this row tile adds the splits in order
      __shared__ int s_last;
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (r == 0) s_last = atomicAdd(&a.counters[rb], 1u) == (unsigned)(a.splits - 1);
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (s_last) {
        __threadfence();
        if (R < M.rows) {
          for (int t = 0; t < a.n_tokens; ++t) {
            float v = 0.f;
            for (int sp = 0; sp < a.splits; ++sp) v += __ldcg(M.part + ((size_t)sp * 16 + t) * M.rows + R);
            if (M.bias) v += M.bias[R];
            if (M.residual) v += M.residual[(size_t)t * M.rows + R];
            M.y[(size_t)t * M.rows + R] = v;
          }
        }
        if (r == 0) a.counters[rb] = 0u;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 13) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace oomattn
