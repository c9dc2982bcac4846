// K-A: bias + RoPE + paged KV append, standalone (epilogue-only, for
// projections computed elsewhere) and fused behind a QKV GEMV for decode-sized
// token counts.
//
// Reference semantics (oomllama_turbo.rs:638-681): q = x Wq^T + bq, k = x Wk^T
// + bk, v = x Wv^T + bv (bias added after the product, :648-656), then RoPE on
// q and k at position pos(token) and LayerKVCache::append of k, v (:41-55).
// RoPE pairs (x0, x1) are (x[i], x[i+64]) for the split-half variant
// (apply_rope_llama :443-467 and TurboEngine::apply_rope :773-783) or
// (x[2i], x[2i+1]) for the interleaved one (apply_rope :402-438):
//   x0' = x0*cos - x1*sin ; x1' = x0*sin + x1*cos
// with every product and sum separately rounded (__fmul_rn/__fadd_rn keep
// nvcc from contracting them into FMAs), using the host-built f32 cos/sin
// table, so rotated values are bit-identical to the f32 reference arithmetic.
// K/V stored in a bf16 cache and q written as bf16 are rounded to nearest even.
#pragma once
#include "common.cuh"
#include "params.cuh"

namespace oomattn {

__device__ __forceinline__ void rope_pair(float x0, float x1, float c, float s, float& y0, float& y1) {
  const float a = __fmul_rn(x0, c), b = __fmul_rn(x1, s);
  const float e = __fmul_rn(x0, s), f = __fmul_rn(x1, c);
  y0 = __fsub_rn(a, b);
  y1 = __fadd_rn(e, f);
}

__device__ __forceinline__ float load_elem(const void* p, size_t i, int bf16) {
  return bf16 ? bf16_bits_to_f32(reinterpret_cast<const uint16_t*>(p)[i]) : reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_elem(void* p, size_t i, float x, int bf16) {
  if (bf16)
    reinterpret_cast<uint16_t*>(p)[i] = f32_to_bf16_bits(x);
  else
    reinterpret_cast<float*>(p)[i] = x;
}

// Element offset of (layer, slot, kv head g, dim 0) in the pool, resolving the
// slot through the block table.  Returns false when the page is out of range.
__device__ __forceinline__ bool cache_offset(const KVPool& pool, int layer, int seq, int slot, int g, size_t& off) {
  const int lp = slot / kPageSize;
  if ((unsigned)lp >= (unsigned)pool.max_pages_per_seq) return false;
  const int page = pool.block_table[(size_t)seq * pool.max_pages_per_seq + lp];
  if ((unsigned)page >= (unsigned)(pool.n_pool_pages - 1)) return false;  // the null page is never written
  off = (((size_t)(layer * pool.n_pool_pages + page) * pool.n_kv + g) * kPageSize + (slot % kPageSize)) * kHeadDim;
  return true;
}

// Rotate / store one (q or k) pair or copy one v pair of token t.
// item < n_heads*64: q pairs; < (n_heads+n_kv)*64: k pairs; else v pairs.
// vals: the un-rotated (biased) pair values.
__device__ __forceinline__ void emit_pair(const AppendArgs& ap, const KVPool& pool, const SeqBatch& sb, int t,
                                          int item, float x0, float x1) {
  const int nq = ap.n_heads * 64, nk = pool.n_kv * 64;
  const int row = t / ap.n_new, s = t % ap.n_new;
  const int pos = sb.pos[row] + s;
  const int sec = item < nq ? 0 : (item < nq + nk ? 1 : 2);
  const int local = sec == 0 ? item : (sec == 1 ? item - nq : item - nq - nk);
  const int head = local / 64, i = local % 64;
  const int i0 = (ap.variant == 1 || sec == 2) ? 2 * i : i;
  const int i1 = (ap.variant == 1 || sec == 2) ? 2 * i + 1 : i + 64;
  float y0 = x0, y1 = x1;
  if (sec == 0 || (sec == 1 && ap.rope_k)) {
    if ((unsigned)pos >= (unsigned)ap.max_pos) {
      report_error(ap.status, kDevErrBounds);
      return;
    }
    rope_pair(x0, x1, ap.cos_t[(size_t)pos * 64 + i], ap.sin_t[(size_t)pos * 64 + i], y0, y1);
  }
  if (sec == 0) {
    const size_t o = ((size_t)t * ap.n_heads + head) * kHeadDim;
    store_elem(ap.q_out, o + i0, y0, ap.q_out_bf16);
    store_elem(ap.q_out, o + i1, y1, ap.q_out_bf16);
  } else {
    size_t off;
    if (!cache_offset(pool, ap.layer, sb.seq[row], sb.len[row] + s, head, off)) {
      report_error(ap.status, kDevErrBounds);
      return;
    }
    void* dst = sec == 1 ? pool.k : pool.v;
    store_elem(dst, off + i0, y0, pool.kv_bf16);
    store_elem(dst, off + i1, y1, pool.kv_bf16);
  }
}

// 8 consecutive elements of a bf16 or f32 row as f32 (one or two 128-bit loads).
template <bool BF16>
__device__ __forceinline__ void load8(const void* p, size_t i, float* x) {
  if (BF16) {
    const uint4 w = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p) + i);
    const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      x[2 * k] = bf16_lo_f32(u[k]);
      x[2 * k + 1] = bf16_hi_f32(u[k]);
    }
  } else {
    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i);
    const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i + 4);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
  }
}

template <bool BF16>
__device__ __forceinline__ void store8(void* p, size_t i, const float* x) {
  if (BF16) {
    uint4 w;
    w.x = pack_bf16(x[0], x[1]);
    w.y = pack_bf16(x[2], x[3]);
    w.z = pack_bf16(x[4], x[5]);
    w.w = pack_bf16(x[6], x[7]);
    *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p) + i) = w;
  } else {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(p) + i) = make_float4(x[0], x[1], x[2], x[3]);
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(p) + i + 4) = make_float4(x[4], x[5], x[6], x[7]);
  }
}

__device__ __forceinline__ void add_bias8(float* x, const float* b) {
  const float4 u = *reinterpret_cast<const float4*>(b), v = *reinterpret_cast<const float4*>(b + 4);
  x[0] = __fadd_rn(x[0], u.x); x[1] = __fadd_rn(x[1], u.y); x[2] = __fadd_rn(x[2], u.z); x[3] = __fadd_rn(x[3], u.w);
  x[4] = __fadd_rn(x[4], v.x); x[5] = __fadd_rn(x[5], v.y); x[6] = __fadd_rn(x[6], v.z); x[7] = __fadd_rn(x[7], v.w);
}

// Epilogue-only K-A, vectorised.  A unit is 16 elements of one head that close
// under the RoPE pairing -- 8 pairs i = 8c..8c+7:
//   interleaved: elements [16c, 16c+16) (pair i = (2i, 2i+1))
//   split-half:  elements [8c, 8c+8) and [64+8c, 64+8c+8) (pair i = (i, i+64))
//   V:           elements [16c, 16c+16), copied
// so every thread moves 128-bit vectors and reads its 8 cos/sin values as two
// float4s.  The rotation arithmetic is rope_pair's, bit for bit.
// grid-stride over T tokens x (n_heads + 2 n_kv) heads x 8 units.
template <bool IN_BF16, bool Q_BF16, bool KV_BF16>
__global__ void __launch_bounds__(256)
    rope_append_kernel(const AppendArgs ap, const KVPool pool, const __grid_constant__ SeqBatch sb, int T) {
  // launched as a programmatic dependent of the kernel before it (the QKV
  // projection): q/k/v and the cache are touched only after that kernel ends;
  // then the decode that follows may launch (it waits for this grid before reading)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int hq = ap.n_heads, hkv = pool.n_kv;
  const int units_tok = (hq + 2 * hkv) * 8;
  const int first = ap.q ? 0 : hq * 8;         // no q: K/V rows only
  const int last = ap.k ? units_tok : hq * 8;  // no k/v: q rows only (nothing is appended)
  const int per_tok = last - first;
  const int total = T * per_tok;  // < 2^31 (checked on the host): 32-bit index arithmetic
  for (int w = blockIdx.x * blockDim.x + threadIdx.x; w < total; w += gridDim.x * blockDim.x) {
    const int t = w / per_tok;
    const int u = first + (w - t * per_tok);
    const int sec = u < hq * 8 ? 0 : (u < (hq + hkv) * 8 ? 1 : 2);
    const int lu = sec == 0 ? u : (sec == 1 ? u - hq * 8 : u - (hq + hkv) * 8);
    const int head = lu >> 3, c = lu & 7;
    const bool split = ap.variant == 0 && sec < 2;
    const int e0 = split ? 8 * c : 16 * c;         // first element of the first 8
    const int e1 = split ? 64 + 8 * c : 16 * c + 8;  // first element of the second 8
    const void* src = sec == 0 ? ap.q : (sec == 1 ? ap.k : ap.v);
    const size_t base = ((size_t)t * (sec == 0 ? hq : hkv) + head) * kHeadDim;
    float a[8], b[8];
    load8<IN_BF16>(src, base + e0, a);
    load8<IN_BF16>(src, base + e1, b);
    const float* bias = sec == 0 ? ap.bq : (sec == 1 ? ap.bk : ap.bv);
    if (bias) {
      add_bias8(a, bias + head * kHeadDim + e0);
      add_bias8(b, bias + head * kHeadDim + e1);
    }
    const int row = t / ap.n_new, s = t % ap.n_new;
    if (sec == 0 || (sec == 1 && ap.rope_k)) {
      const int pos = sb.pos[row] + s;
      if ((unsigned)pos >= (unsigned)ap.max_pos) {
        report_error(ap.status, kDevErrBounds);
        continue;
      }
      const float4* cp = reinterpret_cast<const float4*>(ap.cos_t + (size_t)pos * 64 + 8 * c);
      const float4* sp = reinterpret_cast<const float4*>(ap.sin_t + (size_t)pos * 64 + 8 * c);
      const float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
      const float cs[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
      const float sn[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
      if (split) {
        // pair k: (a[k], b[k])
#pragma unroll
        for (int k = 0; k < 8; ++k) rope_pair(a[k], b[k], cs[k], sn[k], a[k], b[k]);
      } else {
        // pairs 0..3 in a (a[2k], a[2k+1]), pairs 4..7 in b
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          rope_pair(a[2 * k], a[2 * k + 1], cs[k], sn[k], a[2 * k], a[2 * k + 1]);
          rope_pair(b[2 * k], b[2 * k + 1], cs[k + 4], sn[k + 4], b[2 * k], b[2 * k + 1]);
        }
      }
    }
    if (sec == 0) {
      const size_t o = ((size_t)t * hq + head) * kHeadDim;
      store8<Q_BF16>(ap.q_out, o + e0, a);
      store8<Q_BF16>(ap.q_out, o + e1, b);
    } else {
      size_t off;
      if (!cache_offset(pool, ap.layer, sb.seq[row], sb.len[row] + s, head, off)) {
        report_error(ap.status, kDevErrBounds);
        continue;
      }
      void* dst = sec == 1 ? pool.k : pool.v;
      store8<KV_BF16>(dst, off + e0, a);
      store8<KV_BF16>(dst, off + e1, b);
    }
  }
}

// Fused QKV GEMV + bias + RoPE + append for T <= kGemvMaxT tokens.
// One CTA owns 16 output rows that are closed under the RoPE pairing (for the
// split-half variant rows c*8..c*8+7 and 64+c*8.. of one head; otherwise 16
// adjacent rows), so the rotation completes inside the CTA.  8 warps x 2 rows;
// each warp streams its weight rows with 128-bit loads (HBM-bound on W).
constexpr int kGemvMaxT = 16;

// x (f32) -> bf16 (RNE) for the cuBLAS projection of bf16 weights, whose
// GEMM takes both operands in one type.
__global__ void f32_to_bf16_kernel(const float* __restrict__ x, uint16_t* __restrict__ y, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    y[i] = f32_to_bf16_bits(x[i]);
}

#ifndef OOMATTN_GEMV_PRE
#define OOMATTN_GEMV_PRE 12
#endif
// f32 weight chunks (of 128 columns per warp) each lane loads before the wait:
// C1 step 26.7 us with none, 22.7 with 8, 20.9 with 10, 20.1 with 12, 27.2 with
// 14 and 25.8 with 16 (the registers then cut the resident CTAs)
constexpr int kGemvPre = OOMATTN_GEMV_PRE;

template <int T, bool WBF16>
__global__ void __launch_bounds__(256)
    qkv_gemv_rope_append_kernel(const GemvArgs ga, const KVPool pool, const __grid_constant__ SeqBatch sb) {
  // the decode that follows may launch now: it waits for this grid before reading
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  __shared__ float y[16][T];
  const AppendArgs& ap = ga.ap;
  const int grp = blockIdx.x;
  const int nq_grp = ap.n_heads * 8, nk_grp = pool.n_kv * 8;
  const int sec = grp < nq_grp ? 0 : (grp < nq_grp + nk_grp ? 1 : 2);
  const int lg = sec == 0 ? grp : (sec == 1 ? grp - nq_grp : grp - nq_grp - nk_grp);
  const int head = lg / 8, c = lg % 8;
  const bool split_half = (ap.variant == 0) && sec < 2;
  const void* W = sec == 0 ? ga.wq : (sec == 1 ? ga.wk : ga.wv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int H = ga.hidden;

  // the warp's two rows stream together: twice the loads in flight, and each
  // x vector is read once for both
  size_t wrow[2];
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int r = warp * 2 + rr;  // 0..15
    const int drow = split_half ? (r < 8 ? c * 8 + r : 64 + c * 8 + (r - 8)) : c * 16 + r;
    wrow[rr] = (size_t)(head * kHeadDim + drow) * H;
  }
  // Launched as a programmatic dependent of the kernel before it (in a token
  // loop, the previous layer's decode), so its launch overlaps that kernel's
  // tail; it waits for it before it reads x or writes q and the cache.  The
  // weights do not depend on that kernel: with f32 weights each lane's first
  // kGemvPre chunks of both rows are loaded into registers before the wait
  // (C1 step 20.1 against 26.7 us).  Pulling the rows into L2 instead was
  // slower (29.9 us for all rows, 26.8 for the first 4 KB of each row).
  float4 pa[WBF16 ? 1 : kGemvPre], pb[WBF16 ? 1 : kGemvPre];
  if (!WBF16) {
    const float* wp0 = reinterpret_cast<const float*>(W) + wrow[0];
    const float* wp1 = reinterpret_cast<const float*>(W) + wrow[1];
#pragma unroll
    for (int u = 0; u < kGemvPre; ++u) {
      const int j = lane * 4 + u * 128;
      if (j < H) {
        pa[u] = __ldcs(reinterpret_cast<const float4*>(wp0 + j));
        pb[u] = __ldcs(reinterpret_cast<const float4*>(wp1 + j));
      }
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  float acc[2][T];
#pragma unroll
  for (int rr = 0; rr < 2; ++rr)
#pragma unroll
    for (int t = 0; t < T; ++t) acc[rr][t] = 0.f;
  if (WBF16) {
    const uint16_t* wp0 = reinterpret_cast<const uint16_t*>(W) + wrow[0];
    const uint16_t* wp1 = reinterpret_cast<const uint16_t*>(W) + wrow[1];
#pragma unroll 2
    for (int j = lane * 8; j < H; j += 256) {
      const uint4 wa = __ldcs(reinterpret_cast<const uint4*>(wp0 + j));
      const uint4 wb = __ldcs(reinterpret_cast<const uint4*>(wp1 + j));
      const float w0[8] = {bf16_lo_f32(wa.x), bf16_hi_f32(wa.x), bf16_lo_f32(wa.y), bf16_hi_f32(wa.y),
                           bf16_lo_f32(wa.z), bf16_hi_f32(wa.z), bf16_lo_f32(wa.w), bf16_hi_f32(wa.w)};
      const float w1[8] = {bf16_lo_f32(wb.x), bf16_hi_f32(wb.x), bf16_lo_f32(wb.y), bf16_hi_f32(wb.y),
                           bf16_lo_f32(wb.z), bf16_hi_f32(wb.z), bf16_lo_f32(wb.w), bf16_hi_f32(wb.w)};
#pragma unroll
      for (int t = 0; t < T; ++t) {
        const float4 x0 = __ldg(reinterpret_cast<const float4*>(ga.x + (size_t)t * H + j));
        const float4 x1 = __ldg(reinterpret_cast<const float4*>(ga.x + (size_t)t * H + j + 4));
        acc[0][t] += x0.x * w0[0] + x0.y * w0[1] + x0.z * w0[2] + x0.w * w0[3] + x1.x * w0[4] + x1.y * w0[5] +
                     x1.z * w0[6] + x1.w * w0[7];
        acc[1][t] += x0.x * w1[0] + x0.y * w1[1] + x0.z * w1[2] + x0.w * w1[3] + x1.x * w1[4] + x1.y * w1[5] +
                     x1.z * w1[6] + x1.w * w1[7];
      }
    }
  } else {
    const float* wp0 = reinterpret_cast<const float*>(W) + wrow[0];
    const float* wp1 = reinterpret_cast<const float*>(W) + wrow[1];
    // the preloaded chunks first, then the rest in the same column order
#pragma unroll
    for (int u = 0; u < kGemvPre; ++u) {
      const int j = lane * 4 + u * 128;
      if (j < H) {
#pragma unroll
        for (int t = 0; t < T; ++t) {
          const float4 x = __ldg(reinterpret_cast<const float4*>(ga.x + (size_t)t * H + j));
          acc[0][t] += x.x * pa[u].x + x.y * pa[u].y + x.z * pa[u].z + x.w * pa[u].w;
          acc[1][t] += x.x * pb[u].x + x.y * pb[u].y + x.z * pb[u].z + x.w * pb[u].w;
        }
      }
    }
#pragma unroll 8
    for (int j = lane * 4 + kGemvPre * 128; j < H; j += 128) {  // 16 loads of 16 bytes in flight per lane
      const float4 wa = __ldcs(reinterpret_cast<const float4*>(wp0 + j));
      const float4 wb = __ldcs(reinterpret_cast<const float4*>(wp1 + j));
#pragma unroll
      for (int t = 0; t < T; ++t) {
        const float4 x = __ldg(reinterpret_cast<const float4*>(ga.x + (size_t)t * H + j));
        acc[0][t] += x.x * wa.x + x.y * wa.y + x.z * wa.z + x.w * wa.w;
        acc[1][t] += x.x * wb.x + x.y * wb.y + x.z * wb.z + x.w * wb.w;
      }
    }
  }
#pragma unroll
  for (int rr = 0; rr < 2; ++rr)
#pragma unroll
    for (int t = 0; t < T; ++t) {
      float v = acc[rr][t];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0) y[warp * 2 + rr][t] = v;
    }
  __syncthreads();
  // epilogue: 8 pairs x T tokens
  for (int idx = threadIdx.x; idx < 8 * ga.T; idx += blockDim.x) {
    const int pr = idx % 8, t = idx / 8;
    // pair pr = rows (pr, pr+8) for split-half; (2pr, 2pr+1) otherwise
    const int r0 = split_half ? pr : 2 * pr, r1 = split_half ? pr + 8 : 2 * pr + 1;
    const int d0 = split_half ? c * 8 + pr : c * 16 + 2 * pr;
    const int d1 = split_half ? 64 + c * 8 + pr : d0 + 1;
    float x0 = y[r0][t], x1 = y[r1][t];
    const float* b = sec == 0 ? ap.bq : (sec == 1 ? ap.bk : ap.bv);
    if (b) {
      x0 = __fadd_rn(x0, b[head * kHeadDim + d0]);
      x1 = __fadd_rn(x1, b[head * kHeadDim + d1]);
    }
    // pair index in emit_pair's numbering: split-half pair i = d0; interleaved i = d0 / 2
    const int i = split_half ? d0 : d0 / 2;
    const int item = (sec == 0 ? 0 : (sec == 1 ? ap.n_heads * 64 : (ap.n_heads + pool.n_kv) * 64)) + head * 64 + i;
    emit_pair(ap, pool, sb, t, item, x0, x1);
  }
}

}  // namespace oomattn
