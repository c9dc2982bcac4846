// K-F: x @ W^T on the 5th-generation tensor cores, for token counts where the
// projection is a real contraction (prefill chunks): TMA-fed, tcgen05.mma
// with the accumulator in TMEM, epilogue through TMA stores.
//
// Semantics: out[t][n] = sum_k x[t][k] * W[n][k] (+ bias[n]) (+ residual[t][n])
// -- candle's x @ W^T (src/oomllama_turbo.rs:643-645, :715-720) and the
// matvec of src/oom_inference.rs:168-180 -- for f32 activations, with W in
// one of three forms:
//   * f32 (split): x and W are split on the device into bf16 hi + lo planes
//     (x = xh + xl, W = Wh + Wl, each part rounded to nearest) and the tile
//     accumulates xh.Wh + xh.Wl + xl.Wh in f32: about 16 significant bits per
//     product; the dropped xl.Wl term is below 2^-16 of |x w|;
//   * bf16: xh.W + xl.W;
//   * Q8 (BlockQ8View::dequantize_fast, src/quant.rs:201-224): W = min_b +
//     q * scale_b per 256-value block of the row-major flattening.  x is split
//     into fp16 hi + lo (about 22 significant bits) and q enters as fp16 (exact
//     for 0..255).  Every 256-column block's partial product D_b = sum q x is
//     promoted by the epilogue warps into a register accumulator:
//       acc += scale_b * D_b + min_b * X_b,    X_b = sum of x over the block,
//     the affine map of the block applied after its dot product, as K-E does.
//
// Tile: 128 tokens (TMEM lanes) x 256 weight rows (TMEM columns) per CTA; K
// in stages of 64 (one 128-byte swizzle row of 16-bit values).  Warps:
//   warp 0       TMA producer (one lane): A planes [128][64], B planes [256][64]
//   warp 1       MMA issuer (one lane): M = 128, N = 256, K = 16 per MMA
//   warps 2-3    idle
//   warps 4-11   epilogue: warp w reads TMEM lanes 32 (w % 4).., columns
//                128 ((w - 4) / 4).. -- one token row and 128 columns per thread
// The Q8 form keeps 128 accumulators per epilogue thread in registers: its
// warpgroup 0 gives registers back (setmaxnreg) to the two epilogue
// warpgroups, as the prefill kernel does (launch at 168 per thread, 88 / 208).
// Q8 tiles double-buffer D_b in TMEM (2 x 256 columns), so the tensor core
// fills block b + 1 while the epilogue promotes block b.  The result is staged
// in shared memory over the (then idle) operand ring, 128-byte swizzled, and
// leaves through TMA stores that clip rows past M and columns past N; the
// residual arrives the same way, by TMA loads into the staging area.
//
// Tiles are visited in groups of kKfGroupM token tiles, so the weight tiles a
// wave streams are reused by several token tiles while they are in L2.
#pragma once
#include <cuda_fp16.h>

#include "common.cuh"
#include "prefill.cuh"

namespace oomattn {

constexpr int kKfBM = 128;
constexpr int kKfBN = 256;
constexpr int kKfBK = 64;
constexpr int kKfWarps = 12;
constexpr int kKfThreads = kKfWarps * 32;
constexpr int kKfEpiThreads = 256;
constexpr int kKfATile = kKfBM * kKfBK * 2;  // 16 KB per A plane per stage
constexpr int kKfBTile = kKfBN * kKfBK * 2;  // 32 KB per B plane per stage
constexpr int kKfRingBytes = 192 * 1024;
constexpr int kKfSmemBytes = kKfRingBytes + 1024 + 256;
constexpr int kKfGroupM = 8;
constexpr int kKfQ8Block = 256;  // K per Q8 block: 4 stages
constexpr int kKfLaunchRegs = 168;  // the Q8 form's register split holds only at this compiled count
static_assert(128 * 88 + 256 * 208 <= kKfThreads * kKfLaunchRegs, "register split exceeds the launch allocation");

template <bool Q8, int BPLANES>
struct KfShape {
  static constexpr int kStageBytes = 2 * kKfATile + BPLANES * kKfBTile;
  static constexpr int kStages = kKfRingBytes / kStageBytes;  // 2 (f32 split), 3 (bf16, Q8)
  static_assert(kStages >= 2, "ring too small");
};

struct KfArgs {
  int M, N, K;
  int m_tiles, n_tiles;
  const float* bias;      // [N] or null
  const float* scale_t;   // Q8: [K / 256][N] block scales, transposed
  const float* min_t;     // Q8: [K / 256][N] block minima, transposed
  const float* xsum;      // Q8: [M][K / 256] sums of x over each block
  int has_residual;
  int* status;
  unsigned long long timeout_ns;
};

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
__device__ __forceinline__ bool epi_bar_and(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, 256, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}

// Instruction descriptor, kind::f16: f32 accumulate, A and B both bf16 (or
// both fp16), both K-major, M = 128, N = 256.
__host__ __device__ constexpr uint32_t kf_idesc(bool bf16) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((uint32_t)(kKfBN >> 3) << 17) |
         ((uint32_t)(kKfBM >> 4) << 24);
}

template <bool Q8, int BPLANES>
__global__ void __launch_bounds__(kKfThreads, 1)
    kf_gemm_kernel(const __grid_constant__ CUtensorMap amap_hi, const __grid_constant__ CUtensorMap amap_lo,
                   const __grid_constant__ CUtensorMap bmap_hi, const __grid_constant__ CUtensorMap bmap_lo,
                   const __grid_constant__ CUtensorMap omap, const __grid_constant__ CUtensorMap rmap,
                   const KfArgs a) {
  using S = KfShape<Q8, BPLANES>;
  constexpr int kStages = S::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kKfRingBytes);
  uint64_t* full = bars;                  // [kStages]
  uint64_t* empty = full + kStages;       // [kStages]
  uint64_t* d_full = empty + kStages;     // [2]: accumulator buffer ready (Q8: block b in buffer b % 2)
  uint64_t* d_empty = d_full + 2;         // [2]: Q8: the epilogue has read the buffer
  uint64_t* res_full = d_empty + 2;       // the residual tile has landed in the staging area
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(res_full + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grouped raster: kKfGroupM token tiles share a run of weight tiles
  int m_tile, n_tile;
  {
    const int per_group = kKfGroupM * a.n_tiles;
    const int grp = (int)blockIdx.x / per_group;
    const int first = grp * kKfGroupM;
    const int gm = min(a.m_tiles - first, kKfGroupM);
    const int w = (int)blockIdx.x - grp * per_group;
    m_tile = first + w % gm;
    n_tile = w / gm;
  }
  const int m0 = m_tile * kKfBM, n0 = n_tile * kKfBN;
  const int n_k = (a.K + kKfBK - 1) / kKfBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&d_full[b], 1);
      mbar_init(&d_empty[b], kKfEpiThreads / 32);
    }
    mbar_init(res_full, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

#define OOMATTN_KF_DEC() \
  if constexpr (Q8) asm volatile("setmaxnreg.dec.sync.aligned.u32 88;")
#define OOMATTN_KF_INC() \
  if constexpr (Q8) asm volatile("setmaxnreg.inc.sync.aligned.u32 208;")
  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    OOMATTN_KF_DEC();
    if (lane == 0) {
      prefetch_tensormap(&amap_hi);
      prefetch_tensormap(&amap_lo);
      prefetch_tensormap(&bmap_hi);
      if (BPLANES == 2) prefetch_tensormap(&bmap_lo);
      int issued = 0;
      for (int kt = 0; kt < n_k; ++kt) {
        const int s = kt % kStages;
        if (kt >= kStages && !mbar_wait(&empty[s], ((kt / kStages) - 1) & 1, a.status, a.timeout_ns)) break;
        uint8_t* st = smem + s * S::kStageBytes;
        mbar_arrive_expect_tx(&full[s], S::kStageBytes);
        tma_load_2d(st, &amap_hi, &full[s], kt * kKfBK, m0);
        tma_load_2d(st + kKfATile, &amap_lo, &full[s], kt * kKfBK, m0);
        tma_load_2d(st + 2 * kKfATile, &bmap_hi, &full[s], kt * kKfBK, n0);
        if (BPLANES == 2) tma_load_2d(st + 2 * kKfATile + kKfBTile, &bmap_lo, &full[s], kt * kKfBK, n0);
        issued = kt + 1;
      }
      // drain: the last copies this lane issued land before the CTA can exit,
      // also when a wait above gave up
      for (int kt = max(0, issued - kStages); kt < issued; ++kt)
        mbar_wait(&full[kt % kStages], (kt / kStages) & 1, a.status, a.timeout_ns);
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    OOMATTN_KF_DEC();
    if (lane == 0) {
      constexpr uint32_t idesc = kf_idesc(!Q8);
      const uint64_t d0 = make_sdesc(smem_u32(smem), 16, 1024);
      const uint32_t dlo = (uint32_t)d0, dhi = (uint32_t)(d0 >> 32);
      bool ok = true;
      for (int kt = 0; kt < n_k && ok; ++kt) {
        const int s = kt % kStages;
        ok = mbar_wait(&full[s], (kt / kStages) & 1, a.status, a.timeout_ns);
        if (!ok) break;
        tc_fence_after();
        int buf = 0;
        bool first_of_acc = kt == 0;
        if (Q8) {
          const int b = kt / (kKfQ8Block / kKfBK);
          buf = b & 1;
          first_of_acc = kt % (kKfQ8Block / kKfBK) == 0;
          if (first_of_acc && b >= 2) {
            ok = mbar_wait(&d_empty[buf], ((b >> 1) - 1) & 1, a.status, a.timeout_ns);
            if (!ok) break;
            tc_fence_after();
          }
        }
        const uint32_t d = tmem + buf * kKfBN;
        const uint32_t st = dlo + (uint32_t)(s * S::kStageBytes >> 4);
        const uint32_t ah = st, al = st + (kKfATile >> 4);
        const uint32_t bh = st + (2 * kKfATile >> 4), bl = bh + (kKfBTile >> 4);
#pragma unroll
        for (int k16 = 0; k16 < kKfBK / 16; ++k16) {
          const uint32_t o = (uint32_t)k16 * 2;  // 32 bytes per k-step inside the 128-byte row
          const uint32_t acc0 = (first_of_acc && k16 == 0) ? 0u : 1u;
          mma_ss_lh(d, ah + o, dhi, bh + o, dhi, idesc, acc0);
          if (BPLANES == 2) mma_ss_lh(d, ah + o, dhi, bl + o, dhi, idesc, 1u);
          mma_ss_lh(d, al + o, dhi, bh + o, dhi, idesc, 1u);
        }
        tc_commit(&empty[s]);
        if (Q8 && (kt % (kKfQ8Block / kKfBK) == (kKfQ8Block / kKfBK) - 1 || kt == n_k - 1)) tc_commit(&d_full[buf]);
      }
      if (!Q8 && ok) tc_commit(&d_full[0]);
    }
  } else if (warp < 4) {
    OOMATTN_KF_DEC();  // idle warps
  } else {
    // ------------------------------------------------ epilogue (warps 4-11)
    OOMATTN_KF_INC();
    const int quarter = warp & 3;
    const int half = (warp - 4) >> 2;
    const int r = quarter * 32 + lane;  // token row within the tile
    const int t = m0 + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int c0 = half * 128;  // first column (within the tile) of this thread
    bool ok = true;
    float acc[Q8 ? 128 : 1];
    if (Q8) {
#pragma unroll
      for (int j = 0; j < 128; ++j) acc[j] = 0.f;
      const int kb_total = a.K / kKfQ8Block;
      for (int b = 0; b < kb_total; ++b) {
        const int buf = b & 1;
        ok = mbar_wait(&d_full[buf], (b >> 1) & 1, a.status, a.timeout_ns);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        const float xs = t < a.M ? __ldg(a.xsum + (size_t)t * kb_total + b) : 0.f;
        const float* sc = a.scale_t + (size_t)b * a.N + n0 + c0;
        const float* mn = a.min_t + (size_t)b * a.N + n0 + c0;
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t dr[32];
          OOMATTN_TMEM_LD32(tmem + lane_off + buf * kKfBN + c0 + ch * 32, dr);
          tmem_wait_ld();
#pragma unroll
          for (int v = 0; v < 8; ++v) {
            const int j = ch * 32 + 4 * v;
            float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f), m4 = s4;
            if (n0 + c0 + j < a.N) {  // N % 4 == 0: a group of 4 is wholly inside or outside
              s4 = __ldg(reinterpret_cast<const float4*>(sc + j));
              m4 = __ldg(reinterpret_cast<const float4*>(mn + j));
            }
            acc[j + 0] = fmaf(s4.x, __uint_as_float(dr[4 * v + 0]), fmaf(m4.x, xs, acc[j + 0]));
            acc[j + 1] = fmaf(s4.y, __uint_as_float(dr[4 * v + 1]), fmaf(m4.y, xs, acc[j + 1]));
            acc[j + 2] = fmaf(s4.z, __uint_as_float(dr[4 * v + 2]), fmaf(m4.z, xs, acc[j + 2]));
            acc[j + 3] = fmaf(s4.w, __uint_as_float(dr[4 * v + 3]), fmaf(m4.w, xs, acc[j + 3]));
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&d_empty[buf]);
      }
    } else {
      ok = mbar_wait(&d_full[0], 0, a.status, a.timeout_ns);
      tc_fence_after();
    }
    // all 256 epilogue threads agree before the staging area (the operand
    // ring, idle once the last MMA has completed) is written
    ok = epi_bar_and(ok);
    if (ok) {
      uint8_t* stage = smem;  // 8 boxes of [128 rows][32 f32], 16 KB each
      const bool leader = warp == 4 && lane == 0;
      if (a.has_residual) {
        if (leader) {
          prefetch_tensormap(&rmap);
          mbar_arrive_expect_tx(res_full, 8 * 16384);
          for (int bx = 0; bx < 8; ++bx) tma_load_2d(stage + bx * 16384, &rmap, res_full, n0 + 32 * bx, m0);
        }
        ok = mbar_wait(res_full, 0, a.status, a.timeout_ns);
        ok = epi_bar_and(ok);
      }
      if (ok) {
        const uint32_t row_base = smem_u32(stage) + (uint32_t)r * 128u;
        const uint32_t rsw = (uint32_t)(r & 7);
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          const int box = half * 4 + ch;
          const int nb = n0 + c0 + ch * 32;  // first column of the box
          float v[32];
          if (Q8) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = acc[ch * 32 + j];
          } else {
            uint32_t dr[32];
            OOMATTN_TMEM_LD32(tmem + lane_off + c0 + ch * 32, dr);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(dr[j]);
          }
          if (a.bias) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              if (nb + j < a.N) {
                const float4 b4 = __ldg(reinterpret_cast<const float4*>(a.bias + nb + j));
                v[j] += b4.x;
                v[j + 1] += b4.y;
                v[j + 2] += b4.z;
                v[j + 3] += b4.w;
              }
            }
          }
          const uint32_t bx_addr = row_base + (uint32_t)box * 16384u;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint32_t addr = bx_addr + (((uint32_t)c ^ rsw) << 4);
            float x0 = v[4 * c], x1 = v[4 * c + 1], x2 = v[4 * c + 2], x3 = v[4 * c + 3];
            if (a.has_residual) {
              float4 rv;
              asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                           : "=f"(rv.x), "=f"(rv.y), "=f"(rv.z), "=f"(rv.w)
                           : "r"(addr));
              x0 += rv.x;
              x1 += rv.y;
              x2 += rv.z;
              x3 += rv.w;
            }
            st_shared_v4(addr, __float_as_uint(x0), __float_as_uint(x1), __float_as_uint(x2), __float_as_uint(x3));
          }
        }
        fence_proxy_async_smem();
        epi_bar();
        if (leader) {
          prefetch_tensormap(&omap);
          for (int bx = 0; bx < 8; ++bx) tma_store_2d(&omap, stage + bx * 16384, n0 + 32 * bx, m0);
          bulk_commit_group();
          bulk_wait_group_read0();
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
#undef OOMATTN_KF_DEC
#undef OOMATTN_KF_INC
}

// ------------------------------------------------------------ operand preparation
// x (f32, 4 n4 values) -> bf16 hi = rn(x) and lo = rn(x - hi).
__global__ void kf_split_bf16_kernel(const float* __restrict__ x, uint16_t* __restrict__ hi,
                                     uint16_t* __restrict__ lo, size_t n4) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    const float4 v = __ldg(reinterpret_cast<const float4*>(x) + i);
    uint32_t h0, l0, h1, l1;
    split_bf16x2(v.x, v.y, h0, l0);
    split_bf16x2(v.z, v.w, h1, l1);
    reinterpret_cast<uint2*>(hi)[i] = make_uint2(h0, h1);
    reinterpret_cast<uint2*>(lo)[i] = make_uint2(l0, l1);
  }
}

// Q8 activations: x [M][K] f32 -> fp16 hi = rn(x), lo = rn(x - hi), and the
// sum of x over every 256-column block (one warp per (token, block), a fixed
// reduction order).  |x| >= 65504 has no fp16 image: it is reported.
// With `up` given, the split input is the MLP's gated activation silu(x) * up
// (GhostMlp::forward, src/oomllama.rs:230-242), formed as q8_prep_x_kernel
// forms it.
__global__ void kf_prep_x16_kernel(const float* __restrict__ x, const float* __restrict__ up,
                                   uint16_t* __restrict__ hi, uint16_t* __restrict__ lo, float* __restrict__ xsum,
                                   int M, int K, int* status) {
  const int kb = K / kKfQ8Block;
  const long long units = (long long)M * kb;
  const int lane = threadIdx.x & 31;
  for (long long u = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; u < units;
       u += ((long long)gridDim.x * blockDim.x) >> 5) {
    const int t = (int)(u / kb), b = (int)(u - (long long)t * kb);
    const size_t base = (size_t)t * K + (size_t)b * kKfQ8Block + lane * 8;
    const float4 p = __ldg(reinterpret_cast<const float4*>(x + base));
    const float4 q = __ldg(reinterpret_cast<const float4*>(x + base + 4));
    float v[8] = {p.x, p.y, p.z, p.w, q.x, q.y, q.z, q.w};
    if (up) {
      const float4 pu = __ldg(reinterpret_cast<const float4*>(up + base));
      const float4 qu = __ldg(reinterpret_cast<const float4*>(up + base + 4));
      const float u[8] = {pu.x, pu.y, pu.z, pu.w, qu.x, qu.y, qu.z, qu.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = v[i] * (1.f / (1.f + expf(-v[i]))) * u[i];
    }
    uint32_t h[4], l[4];
    bool big = false;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      big |= !(fabsf(v[2 * i]) < 65504.f) || !(fabsf(v[2 * i + 1]) < 65504.f);
      h[i] = pack_f16(v[2 * i], v[2 * i + 1]);
      const __half2 hh = *reinterpret_cast<const __half2*>(&h[i]);
      const float2 hf = __half22float2(hh);
      l[i] = pack_f16(v[2 * i] - hf.x, v[2 * i + 1] - hf.y);
      s += v[2 * i] + v[2 * i + 1];
    }
    if (big) report_error(status, kDevErrX16);
    *reinterpret_cast<uint4*>(hi + base) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo + base) = make_uint4(l[0], l[1], l[2], l[3]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) xsum[(size_t)t * kb + b] = s;
  }
}

// Q8 weights: q [N][K] uint8 -> fp16 (exact), and the block scales and minima
// of the row-major flattening transposed to [K / 256][N], so that a tile's
// values for one block are contiguous.
__global__ void kf_prep_w8_kernel(const uint8_t* __restrict__ q, const float* __restrict__ scale,
                                  const float* __restrict__ mn, uint16_t* __restrict__ w16, float* __restrict__ scale_t,
                                  float* __restrict__ min_t, int N, int K) {
  const size_t n16 = (size_t)N * K / 16;
  const size_t tid = blockIdx.x * (size_t)blockDim.x + threadIdx.x, stride = (size_t)gridDim.x * blockDim.x;
  for (size_t i = tid; i < n16; i += stride) {
    const uint4 w = __ldg(reinterpret_cast<const uint4*>(q) + i);
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
    uint32_t o[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      o[2 * k] = pack_f16((float)(u[k] & 0xffu), (float)((u[k] >> 8) & 0xffu));
      o[2 * k + 1] = pack_f16((float)((u[k] >> 16) & 0xffu), (float)(u[k] >> 24));
    }
    reinterpret_cast<uint4*>(w16)[2 * i] = make_uint4(o[0], o[1], o[2], o[3]);
    reinterpret_cast<uint4*>(w16)[2 * i + 1] = make_uint4(o[4], o[5], o[6], o[7]);
  }
  const int kb = K / kKfQ8Block;
  const size_t nb = (size_t)N * kb;
  for (size_t i = tid; i < nb; i += stride) {
    const int n = (int)(i / kb), b = (int)(i - (size_t)n * kb);
    scale_t[(size_t)b * N + n] = __ldg(scale + i);
    min_t[(size_t)b * N + n] = __ldg(mn + i);
  }
}

// f32 GEMV for a few tokens: y[t][n] = sum_k x[t][k] W[n][k] (+ bias[n]) (+
// residual[t][n]), W f32 [N][K] streamed once with 128-bit loads; one warp per
// two rows, x read through L1/L2 (T <= 16, K % 4 == 0).  HBM-bound: the decode
// form of the f32 layer's o_proj.
template <int T>
__global__ void __launch_bounds__(256) f32_gemv_kernel(const float* __restrict__ x, const float* __restrict__ W,
                                                       const float* __restrict__ bias,
                                                       const float* __restrict__ residual, float* __restrict__ y,
                                                       int N, int K) {
  const int warp = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  const int n = 2 * warp;
  if (n >= N) return;
  const bool two = n + 1 < N;
  const float* w0 = W + (size_t)n * K;
  const float* w1 = W + (size_t)(two ? n + 1 : n) * K;
  float acc0[T], acc1[T];
#pragma unroll
  for (int t = 0; t < T; ++t) acc0[t] = acc1[t] = 0.f;
  for (int k = lane * 4; k < K; k += 128) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(w0 + k));
    const float4 b = __ldg(reinterpret_cast<const float4*>(w1 + k));
#pragma unroll
    for (int t = 0; t < T; ++t) {
      const float4 xv = __ldg(reinterpret_cast<const float4*>(x + (size_t)t * K + k));
      acc0[t] = fmaf(a.x, xv.x, fmaf(a.y, xv.y, fmaf(a.z, xv.z, fmaf(a.w, xv.w, acc0[t]))));
      acc1[t] = fmaf(b.x, xv.x, fmaf(b.y, xv.y, fmaf(b.z, xv.z, fmaf(b.w, xv.w, acc1[t]))));
    }
  }
#pragma unroll
  for (int t = 0; t < T; ++t) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      acc0[t] += __shfl_xor_sync(0xffffffffu, acc0[t], off);
      acc1[t] += __shfl_xor_sync(0xffffffffu, acc1[t], off);
    }
  }
  // lane t writes token t (each unrolled step indexes its registers statically)
#pragma unroll
  for (int t = 0; t < T; ++t) {
    if (lane == t) {
      float v0 = acc0[t] + (bias ? bias[n] : 0.f);
      if (residual) v0 += residual[(size_t)t * N + n];
      y[(size_t)t * N + n] = v0;
      if (two) {
        float v1 = acc1[t] + (bias ? bias[n + 1] : 0.f);
        if (residual) v1 += residual[(size_t)t * N + n + 1];
        y[(size_t)t * N + n + 1] = v1;
      }
    }
  }
}

}  // namespace oomattn
