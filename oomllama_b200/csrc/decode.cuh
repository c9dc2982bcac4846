// K-B / K-B2: split-KV GQA flash-decode over the paged cache, with the
// log-sum-exp merge of the splits done by the last CTA of each (row, kv head).
//
// Work unit: one CTA per item (row z, kv head g, split) of a DecodeSched.  The
// CTA streams pages [split*pps, (split+1)*pps) of row z's block table, pps =
// ceil(pages / nsplit), and serves all `group` q heads that read kv head g
// (q head h -> kv head h / group, the repeat_interleave grouping of
// oomllama_turbo.rs:313-316), so each KV byte is read from HBM once per step
// instead of `group` times.  Items come longest first, so the block scheduler,
// which hands CTAs out in grid order to whichever slot frees first, runs a
// longest-processing-time list schedule over rows of different lengths.
//
// bf16 cache (decode_bf16_kernel): a producer warp moves each (page, kv head)
// chunk -- 16 tokens x 128 dims, two 2 KB TMA boxes with the 128-byte swizzle --
// into a 2-stage shared-memory ring (mbarrier complete_tx), three CTAs per SM;
// four consumer warps each take one page per stage.  Per page a warp computes
//   S^T[16 tok x 8 heads] = K[16 x 128] . Q^T        (m16n8k16, Q split hi+lo)
// then an online softmax per head column (exp2 of log2e-prescaled scores), and
//   O^T[128 x 8] += V^T[128 x 16] . P^T[16 x 8]       (P split hi+lo)
// with P^T moved into the B-operand layout by movmatrix.  The hi/lo splits
// make the bf16 tensor-core products carry ~16 significant bits of the f32
// query and probabilities; the cached K/V are bf16 by contract.
//
// f32 cache (decode_f32_kernel): plain 128-bit loads and f32 FMAs (the f32
// path's 1e-4 tolerance rules out bf16/tf32 products); same split/merge.
#pragma once
#include "common.cuh"
#include "params.cuh"

namespace oomattn {

constexpr int kDecWarps = 4;                       // consumer warps per CTA
// 2 stages x 3 CTAs per SM: 192 KB in flight per SM, as with 3 stages x 2
// CTAs, but with half again as many CTAs to overlap one another's fill and
// merge (C4 0.966 -> 0.992 of HBM, C3 0.923 -> 0.934; a 16-row, 67 MB decode
// 18.0 -> 18.3 us).  The registers drop from 155 to 128 without spills.
constexpr int kDecStages = 2;
constexpr int kDecCtasPerSm = 3;
constexpr int kChunkBytes = kPageSize * kHeadDim * 2;           // one (page, kv head) bf16 chunk: 4 KB
constexpr int kDecStageBytes = 2 * kDecWarps * kChunkBytes;     // K and V of 4 pages: 32 KB
constexpr int kDecSmemBytes = kDecStages * kDecStageBytes + 1024 + 2 * kDecStages * 8 + 64 + kMaxGroup * 32 * 4;

constexpr int kF32Tok = 4;                 // f32 path: tokens loaded and scored together
constexpr int kMergeStride = kHeadDim + 4;  // padded row of the per-warp O staging area
struct MergeSmem {
  float m[kDecWarps][kMaxGroup];
  float l[kDecWarps][kMaxGroup];
  float o[kDecWarps][kMaxGroup][kMergeStride];
};

__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// The last CTA's merge when it has a shared-memory area to stage into (the
// bf16 kernel's page ring, free by then): every (q head, split) partial O row
// of the (row, kv head) is copied in by cp.async (one warp per row, one lane
// per 16 bytes, no index division; chunks of cs splits when they do not all
// fit).  While the copies fly, the 16 threads of each q head load its split
// lse values (two each), reduce the maximum by shuffles and write each
// split's weight 2^(lse - M) once to shared memory; the unrolled sums then
// read only shared memory.  A thread's dims are 4t..4t+3 and 64+4t..64+4t+3,
// so a quarter-warp's 16-byte reads are consecutive.  Against loading the
// partials eight splits ahead into registers with every thread computing
// every weight, the last CTA's merge (globaltimer stamps) takes 1.8-2.4 us
// instead of 2.2-4 us at 6-32 splits; the decode of a 16-row, 67 MB layer
// 18.3 -> 16.6 us.  The sums still run in split order, so the result is the
// same to the bit.
__device__ __forceinline__ void merge_splits_staged(const DecodeArgs& a, int z, int g, int nsplit, int tid,
                                                    float* stage, int stage_floats, float* s_w) {
  const int j = tid >> 4, da = (tid & 15) * 4, db = da + kHeadDim / 2;
  const int warp = tid >> 5, lane = tid & 31;
  const bool active = j < a.group;
  const size_t head0 = (size_t)z * a.n_heads + (size_t)g * a.group;
  const int cs = max(1, min(nsplit, stage_floats / (a.group * kHeadDim)));
  // the 16 threads of a q head (a half-warp) hold its split lse values, two
  // each (splits t and t + 16)
  static_assert(kMaxSplitsBf16 <= 32, "two split weights per thread of a half-warp");
  const int t = tid & 15;
  float w0 = -INFINITY, w1 = -INFINITY;
  if (active) {
    const float* lrow = a.part_lse + (head0 + j) * a.max_splits;
    if (t < nsplit) w0 = __ldcg(lrow + t);
    if (t + 16 < nsplit) w1 = __ldcg(lrow + t + 16);
  }
  auto issue = [&](int s0) {
    const int n = min(cs, nsplit - s0);
    for (int jj = 0; jj < a.group; ++jj) {
      const float* src = a.part_o + ((head0 + jj) * a.max_splits + s0) * kHeadDim + lane * 4;
      float* dst = stage + (size_t)jj * cs * kHeadDim + lane * 4;
      for (int s = warp; s < n; s += kDecWarps) cp_async16_cg(dst + s * kHeadDim, src + (size_t)s * kHeadDim);
    }
    cp_async_commit();
  };
  issue(0);
  float M = fmaxf(w0, w1);
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  // the weights go to shared memory once, for the half-warp's unrolled sums
  float* w_j = s_w + (active ? j : 0) * 32;
  if (active) {
    w_j[t] = (w0 == -INFINITY) ? 0.f : exp2f(w0 - M);
    w_j[t + 16] = (w1 == -INFINITY) ? 0.f : exp2f(w1 - M);
  }
  __syncwarp();
  float wsum = 0.f, acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int s0 = 0; s0 < nsplit; s0 += cs) {
    if (s0 > 0) {
      consumer_bar();  // every thread is done with the previous chunk
      issue(s0);
    }
    cp_async_wait<0>();
    consumer_bar();
    if (active) {
      const int n = min(cs, nsplit - s0);
      const float* st = stage + (size_t)j * cs * kHeadDim;
#pragma unroll 8
      for (int s = 0; s < n; ++s) {
        const float wt = w_j[s0 + s];
        wsum += wt;
        const float4 u = *reinterpret_cast<const float4*>(st + s * kHeadDim + da);
        const float4 v = *reinterpret_cast<const float4*>(st + s * kHeadDim + db);
        acc[0] += wt * u.x; acc[1] += wt * u.y; acc[2] += wt * u.z; acc[3] += wt * u.w;
        acc[4] += wt * v.x; acc[5] += wt * v.y; acc[6] += wt * v.z; acc[7] += wt * v.w;
      }
    }
  }
  if (active) {
    const int h = g * a.group + j;
    const float inv = 1.f / wsum;
    float* orow = a.out + ((size_t)z * a.n_heads + h) * a.o_stride;
    *reinterpret_cast<float4*>(orow + da) = make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv);
    *reinterpret_cast<float4*>(orow + db) = make_float4(acc[4] * inv, acc[5] * inv, acc[6] * inv, acc[7] * inv);
    if (a.lse && (tid & 15) == 0)
      a.lse[((size_t)z * a.n_heads + h) * a.lse_stride] = (M + log2f(wsum)) * 0.69314718055994531f;
  }
}

// Combine the four warps' (m, l, O) of this CTA, then either write the final
// row (single split) or this split's normalised partial; the last CTA of the
// (row, kv head) to finish merges all partials:
//   M = max lse_s ; O = sum 2^(lse_s - M) O_s / sum 2^(lse_s - M) ;
//   lse = M + log2(sum 2^(lse_s - M))   (base 2; stored as natural log).
// Runs on the 128 consumer threads (tid 0..127).  With a staging area
// (`stage`, and `s_w` for the weights) the merge is merge_splits_staged;
// without one (the f32 kernel, which holds no shared ring) the partials are
// loaded into registers.
__device__ __forceinline__ void combine_and_store(const MergeSmem& ms, const DecodeArgs& a, int z, int g, int split,
                                                  int nsplit, int n_kv, int tid, int* s_last, float* stage,
                                                  int stage_floats, float* s_w) {
  const int j = tid >> 4;                       // q head within the group
  const int da = (tid & 15) * 4, db = da + 64;  // the thread's output dims: da..da+3, db..db+3
  const bool active = j < a.group;
  const int h = g * a.group + j;
  float acc[8];
  float lse2 = -INFINITY;
  if (active) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, ms.m[w][j]);
    float lsum = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) {
      const float mw = ms.m[w][j];
      const float wt = (mw == -INFINITY) ? 0.f : exp2f(mw - M);
      lsum += wt * ms.l[w][j];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[i] += wt * ms.o[w][j][da + i];
        acc[4 + i] += wt * ms.o[w][j][db + i];
      }
    }
    const float inv = 1.f / lsum;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] *= inv;
    lse2 = M + log2f(lsum);
    if (nsplit == 1) {
      float* orow = a.out + ((size_t)z * a.n_heads + h) * a.o_stride;
      *reinterpret_cast<float4*>(orow + da) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      *reinterpret_cast<float4*>(orow + db) = make_float4(acc[4], acc[5], acc[6], acc[7]);
      if (a.lse && (tid & 15) == 0)
        a.lse[((size_t)z * a.n_heads + h) * a.lse_stride] = lse2 * 0.69314718055994531f;
    } else {
      const size_t prow = ((size_t)z * a.n_heads + h) * a.max_splits + split;
      float* prow_o = a.part_o + prow * kHeadDim;
      *reinterpret_cast<float4*>(prow_o + da) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      *reinterpret_cast<float4*>(prow_o + db) = make_float4(acc[4], acc[5], acc[6], acc[7]);
      if ((tid & 15) == 0) a.part_lse[prow] = lse2;
    }
  }
  if (nsplit == 1) return;
  consumer_bar();
  if (tid == 0) {
    const unsigned prev = atom_add_acq_rel_gpu(&a.counters[(size_t)z * n_kv + g], 1u);
    *s_last = (prev == (unsigned)(nsplit - 1));
  }
  consumer_bar();
  if (!*s_last) return;
  if (stage != nullptr) {
    merge_splits_staged(a, z, g, nsplit, tid, stage, stage_floats, s_w);
    if (tid == 0) a.counters[(size_t)z * n_kv + g] = 0u;
    return;
  }
  // every (q head, split) lse in one round of loads, staged over the per-warp
  // O area (its last reader passed the barriers above); then each thread's
  // partial O loads run eight splits ahead
  float* lse_s = const_cast<float*>(&ms.o[0][0][0]);  // [kMaxGroup][nsplit]
  for (int i = tid; i < a.group * nsplit; i += kDecWarps * 32) {
    const int jj = i / nsplit, s = i - jj * nsplit;
    lse_s[i] = __ldcg(a.part_lse + ((size_t)z * a.n_heads + g * a.group + jj) * a.max_splits + s);
  }
  consumer_bar();
  if (active) {
    const size_t prow0 = ((size_t)z * a.n_heads + h) * a.max_splits;
    const float* ls_j = lse_s + j * nsplit;
    float M = -INFINITY;
    for (int s = 0; s < nsplit; ++s) M = fmaxf(M, ls_j[s]);
    float wsum = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll 8
    for (int s = 0; s < nsplit; ++s) {
      const float ls = ls_j[s];
      const float wt = (ls == -INFINITY) ? 0.f : exp2f(ls - M);
      wsum += wt;
      const float* pp = a.part_o + (prow0 + s) * kHeadDim;
      const float4 u = __ldcg(reinterpret_cast<const float4*>(pp + da));
      const float4 v = __ldcg(reinterpret_cast<const float4*>(pp + db));
      acc[0] += wt * u.x; acc[1] += wt * u.y; acc[2] += wt * u.z; acc[3] += wt * u.w;
      acc[4] += wt * v.x; acc[5] += wt * v.y; acc[6] += wt * v.z; acc[7] += wt * v.w;
    }
    const float inv = 1.f / wsum;
    float* orow = a.out + ((size_t)z * a.n_heads + h) * a.o_stride;
    *reinterpret_cast<float4*>(orow + da) = make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv);
    *reinterpret_cast<float4*>(orow + db) = make_float4(acc[4] * inv, acc[5] * inv, acc[6] * inv, acc[7] * inv);
    if (a.lse && (tid & 15) == 0)
      a.lse[((size_t)z * a.n_heads + h) * a.lse_stride] = (M + log2f(wsum)) * 0.69314718055994531f;
  }
  if (tid == 0) a.counters[(size_t)z * n_kv + g] = 0u;
}

// A row with no visible keys gets O = 0 and lse = -inf (written by split 0).
// Item i of the schedule: the last row slot whose items start at or before i.
struct DecodeItem {
  int z, g, split, nsplit, pb, pe;
};
__device__ __forceinline__ DecodeItem decode_item(const DecodeSched& s, const SeqBatch& sb, int i) {
  int lo = 0, hi = s.n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s.item0[mid] <= i) lo = mid; else hi = mid - 1;
  }
  DecodeItem it;
  it.z = s.order[lo];
  const int ns = s.nsplit[lo];
  const int j = i - s.item0[lo];
  it.g = j / ns;
  it.split = j - it.g * ns;
  const int n_pages = (sb.len[it.z] + kPageSize - 1) / kPageSize;
  const int pps = n_pages > 0 ? (n_pages + ns - 1) / ns : 0;
  it.pb = it.split * pps;
  it.pe = min(it.pb + pps, n_pages);
  it.nsplit = pps > 0 ? (n_pages + pps - 1) / pps : 1;
  return it;
}

// The kernel is launched as a programmatic dependent of the one before it
// (the RoPE + append): while that one finishes, pull the first pages of this
// item's K/V into L2, then wait for it before reading q or the cache.
constexpr int kDecPrefetchPages = 8;
__device__ __forceinline__ void prefetch_then_wait(const KVPool& pool, const DecodeArgs& a, int seq, int g, int pb,
                                                   int pe, int elem_bytes) {
  const int np = min(pe - pb, kDecPrefetchPages);
  if (np > 0) {
    const int lines = kPageSize * kHeadDim * elem_bytes / 128;  // 128-byte lines per (page, kv head) chunk
    const int* bt = pool.block_table + (size_t)seq * pool.max_pages_per_seq;
    for (int i = threadIdx.x; i < np * 2 * lines; i += blockDim.x) {
      const int pi = pb + i / (2 * lines), r = i % (2 * lines);
      const int page = __ldg(bt + pi);
      if ((unsigned)page >= (unsigned)pool.n_pool_pages) continue;  // reported by the main loop
      const size_t chunk = ((size_t)(a.layer * pool.n_pool_pages + page) * pool.n_kv + g) * kPageSize * kHeadDim;
      const char* base = static_cast<const char*>(r < lines ? pool.k : pool.v) + chunk * elem_bytes;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(base + (size_t)(r % lines) * 128));
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void write_empty_row(const DecodeArgs& a, int z, int g) {
  for (int i = threadIdx.x; i < a.group * kHeadDim; i += blockDim.x) {
    const int h = g * a.group + i / kHeadDim;
    a.out[((size_t)z * a.n_heads + h) * a.o_stride + (i % kHeadDim)] = 0.f;
    if (a.lse && (i % kHeadDim) == 0) a.lse[((size_t)z * a.n_heads + h) * a.lse_stride] = -INFINITY;
  }
}

__global__ void __launch_bounds__((kDecWarps + 1) * 32, kDecCtasPerSm)
    decode_bf16_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                       const KVPool pool, const DecodeArgs a, const __grid_constant__ SeqBatch sb,
                       const __grid_constant__ DecodeSched sched) {
  // a programmatic dependent (the next layer's QKV GEMV) may launch now; it
  // waits for this grid before it reads or writes anything
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kDecStages * kDecStageBytes);
  uint64_t* empty = full + kDecStages;
  int* s_last = reinterpret_cast<int*>(empty + kDecStages);
  float* s_w = reinterpret_cast<float*>(s_last + 16);  // [kMaxGroup][32] merge weights

  const DecodeItem item = decode_item(sched, sb, blockIdx.x);
  const int split = item.split, g = item.g, z = item.z;
  const int seq = sb.seq[z];
  const int L = sb.len[z];
  const int pb = item.pb, pe = item.pe;
  prefetch_then_wait(pool, a, seq, g, pb, pe, 2);
  if (pb >= pe) {
    if (L <= 0 && split == 0) write_empty_row(a, z, g);
    return;
  }
  const int nsplit = item.nsplit;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_iter = (pe - pb + kDecWarps - 1) / kDecWarps;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kDecStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDecWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kDecWarps) {
    // ---------------- producer: one elected lane issues the TMA loads
    // (kTestDropDecodeCopies: a test makes the consumers' bounded waits run
    // out by issuing nothing; they record kDevErrTimeout and the CTA ends.)
    if (lane == 0 && !(a.test_flags & kTestDropDecodeCopies)) {
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      const int* bt = pool.block_table + (size_t)seq * pool.max_pages_per_seq;
      for (int it = 0; it < n_iter; ++it) {
        const int s = it % kDecStages;
        if (it >= kDecStages) {
          if (!mbar_wait(&empty[s], ((it / kDecStages) - 1) & 1, a.status, a.timeout_ns)) break;
        }
        const int p0 = pb + it * kDecWarps;
        const int np = min(kDecWarps, pe - p0);
        mbar_arrive_expect_tx(&full[s], (uint32_t)(np * 2 * kChunkBytes));
        uint8_t* kst = smem + s * kDecStageBytes;
        uint8_t* vst = kst + kDecWarps * kChunkBytes;
        for (int j = 0; j < np; ++j) {
          int page = __ldg(bt + p0 + j);
          if ((unsigned)page >= (unsigned)pool.n_pool_pages) {
            report_error(a.status, kDevErrBounds);
            page = pool.n_pool_pages - 1;
          }
          const int row = ((a.layer * pool.n_pool_pages + page) * pool.n_kv + g) * kPageSize;
          tma_load_2d(kst + j * kChunkBytes, &kmap, &full[s], 0, row);
          tma_load_2d(kst + j * kChunkBytes + kChunkBytes / 2, &kmap, &full[s], 64, row);
          tma_load_2d(vst + j * kChunkBytes, &vmap, &full[s], 0, row);
          tma_load_2d(vst + j * kChunkBytes + kChunkBytes / 2, &vmap, &full[s], 64, row);
        }
      }
    }
    return;
  }

  // ---------------- consumers
  // Q^T as the B operand of S^T = K Q^T: lane holds head lane/4, dims
  // kk*16 + 2*(lane%4) + {0,1} and +8, prescaled by scale*log2(e), split hi/lo.
  uint32_t qh[8][2], ql[8][2];
  {
    const int hq = lane >> 2;
    const bool valid = hq < a.group;
    const float* qp = a.q + ((size_t)z * a.n_heads + g * a.group + (valid ? hq : 0)) * kHeadDim;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int d0 = kk * 16 + 2 * (lane & 3);
      const float2 x01 = valid ? *reinterpret_cast<const float2*>(qp + d0) : make_float2(0.f, 0.f);
      const float2 x89 = valid ? *reinterpret_cast<const float2*>(qp + d0 + 8) : make_float2(0.f, 0.f);
      split_bf16x2(x01.x * a.qscale, x01.y * a.qscale, qh[kk][0], ql[kk][0]);
      split_bf16x2(x89.x * a.qscale, x89.y * a.qscale, qh[kk][1], ql[kk][1]);
    }
  }
  float o[8][4];
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int lrow = lane & 7, lmat = lane >> 3;

  for (int it = 0; it < n_iter; ++it) {
    const int s = it % kDecStages;
    if (!mbar_wait(&full[s], (it / kDecStages) & 1, a.status, a.timeout_ns)) break;
    const int pi = pb + it * kDecWarps + warp;
    if (pi < pe) {
      const uint32_t kbase = smem_u32(smem + s * kDecStageBytes + warp * kChunkBytes);
      const uint32_t vbase = kbase + kDecWarps * kChunkBytes;
      float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(kbase + sw128_off(lrow + (lmat & 1) * 8, kk * 16 + (lmat >> 1) * 8), a0, a1, a2, a3);
        mma_bf16_16816(sc, a0, a1, a2, a3, qh[kk][0], qh[kk][1]);
        mma_bf16_16816(sc, a0, a1, a2, a3, ql[kk][0], ql[kk][1]);
      }
      const int t0 = pi * kPageSize + (lane >> 2);
      if (t0 >= L) sc[0] = sc[1] = -INFINITY;
      if (t0 + 8 >= L) sc[2] = sc[3] = -INFINITY;
      float mt0 = fmaxf(sc[0], sc[2]), mt1 = fmaxf(sc[1], sc[3]);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mt0 = fmaxf(mt0, __shfl_xor_sync(0xffffffffu, mt0, off));
        mt1 = fmaxf(mt1, __shfl_xor_sync(0xffffffffu, mt1, off));
      }
      const float mn0 = fmaxf(m0, mt0), mn1 = fmaxf(m1, mt1);
      const float al0 = exp2f(m0 - mn0), al1 = exp2f(m1 - mn1);
      m0 = mn0;
      m1 = mn1;
      const float p0 = exp2f(sc[0] - mn0), p1 = exp2f(sc[1] - mn1);
      const float p2 = exp2f(sc[2] - mn0), p3 = exp2f(sc[3] - mn1);
      l0 = l0 * al0 + (p0 + p2);
      l1 = l1 * al1 + (p1 + p3);
      uint32_t xh, xl, yh, yl;
      split_bf16x2(p0, p1, xh, xl);
      split_bf16x2(p2, p3, yh, yl);
      const uint32_t bxh = movmatrix_trans(xh), bxl = movmatrix_trans(xl);
      const uint32_t byh = movmatrix_trans(yh), byl = movmatrix_trans(yl);
#pragma unroll
      for (int mt = 0; mt < 8; ++mt) {
        o[mt][0] *= al0;
        o[mt][1] *= al1;
        o[mt][2] *= al0;
        o[mt][3] *= al1;
        uint32_t a0, a1, a2, a3;
        ldsm_x4_trans(vbase + sw128_off(lrow + (lmat >> 1) * 8, mt * 16 + (lmat & 1) * 8), a0, a1, a2, a3);
        mma_bf16_16816(o[mt], a0, a1, a2, a3, bxh, byh);
        mma_bf16_16816(o[mt], a0, a1, a2, a3, bxl, byl);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // per-warp l: sum the partial sums of the 8 lanes sharing a head column
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  consumer_bar();  // every consumer is done with the stage buffers
  MergeSmem& ms = *reinterpret_cast<MergeSmem*>(smem);
  const int h0 = 2 * (lane & 3);
  if (lane < 4) {
    ms.m[warp][h0] = m0;
    ms.m[warp][h0 + 1] = m1;
    ms.l[warp][h0] = l0;
    ms.l[warp][h0 + 1] = l1;
  }
#pragma unroll
  for (int mt = 0; mt < 8; ++mt) {
    const int d = mt * 16 + (lane >> 2);
    ms.o[warp][h0][d] = o[mt][0];
    ms.o[warp][h0 + 1][d] = o[mt][1];
    ms.o[warp][h0][d + 8] = o[mt][2];
    ms.o[warp][h0 + 1][d + 8] = o[mt][3];
  }
  consumer_bar();
  // the merge stages partials over the page ring (MergeSmem's last reader is
  // past the barriers before the merge)
  combine_and_store(ms, a, z, g, split, nsplit, pool.n_kv, threadIdx.x, s_last, reinterpret_cast<float*>(smem),
                    kDecStages * kDecStageBytes / 4, s_w);
}

__global__ void __launch_bounds__(kDecWarps * 32)
    decode_f32_kernel(const KVPool pool, const DecodeArgs a, const __grid_constant__ SeqBatch sb,
                      const __grid_constant__ DecodeSched sched) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // as in decode_bf16_kernel
  __shared__ MergeSmem ms;
  __shared__ int s_last;
  const DecodeItem item = decode_item(sched, sb, blockIdx.x);
  const int split = item.split, g = item.g, z = item.z;
  const int seq = sb.seq[z];
  const int L = sb.len[z];
  const int pb = item.pb, pe = item.pe;
  prefetch_then_wait(pool, a, seq, g, pb, pe, 4);
  if (pb >= pe) {
    if (L <= 0 && split == 0) write_empty_row(a, z, g);
    return;
  }
  const int nsplit = item.nsplit;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* kp = reinterpret_cast<const float*>(pool.k);
  const float* vp = reinterpret_cast<const float*>(pool.v);
  const int* bt = pool.block_table + (size_t)seq * pool.max_pages_per_seq;

  float4 q[kMaxGroup], o[kMaxGroup];
  float m[kMaxGroup], l[kMaxGroup];
#pragma unroll
  for (int j = 0; j < kMaxGroup; ++j) {
    if (j < a.group) {
      const float4 t = *reinterpret_cast<const float4*>(
          a.q + ((size_t)z * a.n_heads + g * a.group + j) * kHeadDim + lane * 4);
      q[j] = make_float4(t.x * a.qscale, t.y * a.qscale, t.z * a.qscale, t.w * a.qscale);
    } else {
      q[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    o[j] = make_float4(0.f, 0.f, 0.f, 0.f);
    m[j] = -INFINITY;
    l[j] = 0.f;
  }
  // the CTA's tokens in groups of kF32Tok (a group never crosses a page),
  // dealt to the warps in turn; a group's loads issue together and its scores
  // reduce as independent shuffle chains; the running max and sums are
  // updated once per group
  const int tok_end = min(pe * kPageSize, L);
  for (int g0 = pb * kPageSize + warp * kF32Tok; g0 < tok_end; g0 += kDecWarps * kF32Tok) {
    const int pi = g0 / kPageSize;
    int page = __ldg(bt + pi);
    if ((unsigned)page >= (unsigned)pool.n_pool_pages) {
      if (lane == 0) report_error(a.status, kDevErrBounds);
      page = pool.n_pool_pages - 1;
    }
    const size_t base = ((size_t)(a.layer * pool.n_pool_pages + page) * pool.n_kv + g) * kPageSize * kHeadDim;
    const int t0 = g0 - pi * kPageSize;             // first slot of the group in its page
    const int nt = min(kPageSize, tok_end - pi * kPageSize);  // valid slots of the page
    {
      float4 kv[kF32Tok], vv[kF32Tok];
#pragma unroll
      for (int u = 0; u < kF32Tok; ++u) {
        const int t = min(t0 + u, nt - 1);  // past the last token: reloaded, then masked
        kv[u] = __ldg(reinterpret_cast<const float4*>(kp + base + t * kHeadDim) + lane);
        vv[u] = __ldg(reinterpret_cast<const float4*>(vp + base + t * kHeadDim) + lane);
      }
#pragma unroll
      for (int j = 0; j < kMaxGroup; ++j) {
        if (j < a.group) {
          float sc[kF32Tok];
#pragma unroll
          for (int u = 0; u < kF32Tok; ++u)
            sc[u] = q[j].x * kv[u].x + q[j].y * kv[u].y + q[j].z * kv[u].z + q[j].w * kv[u].w;
#pragma unroll
          for (int off = 16; off > 0; off >>= 1)
#pragma unroll
            for (int u = 0; u < kF32Tok; ++u) sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], off);
          float mn = m[j];
#pragma unroll
          for (int u = 0; u < kF32Tok; ++u)
            if (t0 + u < nt) mn = fmaxf(mn, sc[u]);
          const float al = exp2f(m[j] - mn);
          m[j] = mn;
          l[j] *= al;
          o[j].x *= al;
          o[j].y *= al;
          o[j].z *= al;
          o[j].w *= al;
#pragma unroll
          for (int u = 0; u < kF32Tok; ++u) {
            if (t0 + u < nt) {
              const float p = exp2f(sc[u] - mn);
              l[j] += p;
              o[j].x += p * vv[u].x;
              o[j].y += p * vv[u].y;
              o[j].z += p * vv[u].z;
              o[j].w += p * vv[u].w;
            }
          }
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kMaxGroup; ++j) {
    if (lane == 0) {
      ms.m[warp][j] = m[j];
      ms.l[warp][j] = l[j];
    }
    *reinterpret_cast<float4*>(&ms.o[warp][j][lane * 4]) = o[j];
  }
  __syncthreads();
  combine_and_store(ms, a, z, g, split, nsplit, pool.n_kv, threadIdx.x, &s_last, nullptr, 0, nullptr);
}

// K-B2 standalone: merge P split-context partials (from P GPUs or P launches)
// given as normalised O_p and natural-log lse_p; partial (p, r) has its O at
// parts + (p * n_rows + r) * part_stride and its lse at lses[(p * n_rows + r) *
// lse_stride] (128 / 1 for separate [P][rows][128] and [P][rows] arrays, 132 /
// 132 for the packed (O, lse) rows that one collective moves).
__global__ void merge_partials_kernel(const float* __restrict__ parts, const float* __restrict__ lses,
                                      int part_stride, int lse_stride, int n_parts, int n_rows,
                                      float* __restrict__ out, float* __restrict__ lse_out) {
  const int r = blockIdx.x;
  const int d = threadIdx.x;  // 128 threads
  if (r >= n_rows) return;
  float M = -INFINITY;
  for (int p = 0; p < n_parts; ++p) M = fmaxf(M, lses[((size_t)p * n_rows + r) * lse_stride]);
  if (M == -INFINITY) {
    out[(size_t)r * kHeadDim + d] = 0.f;
    if (lse_out && d == 0) lse_out[r] = -INFINITY;
    return;
  }
  float acc = 0.f, wsum = 0.f;
  for (int p = 0; p < n_parts; ++p) {
    const float lp = lses[((size_t)p * n_rows + r) * lse_stride];
    const float wt = (lp == -INFINITY) ? 0.f : expf(lp - M);
    wsum += wt;
    acc += wt * parts[((size_t)p * n_rows + r) * part_stride + d];
  }
  out[(size_t)r * kHeadDim + d] = acc / wsum;
  if (lse_out && d == 0) lse_out[r] = M + logf(wsum);
}

}  // namespace oomattn
