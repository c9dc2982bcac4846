// K-C: causal GQA prefill on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Semantics: flash_attention_forward with causal=true (oomllama_turbo.rs:304-369)
// for the n_new newest tokens of one sequence: query i (cache slot
// P + i, P = cache length before the chunk) sees key slots 0..P+i, scale
// 1/sqrt(128), GQA grouping h -> h / group.  Scores and softmax statistics are
// f32.  S = Q K^T runs as bf16 x bf16 (the cache and q are bf16 by contract);
// O += P V runs as fp16 x fp16 with V converted exactly from bf16 and P
// rounded to fp16 (11 significant bits), f32 accumulate throughout.
//
// CTA work unit: one q head and 256 query rows held as two 128-row tiles
// (Q0, Q1).  Warp roles (384 threads):
//   warp 0      TMA producer: Q0/Q1 once, then K_j and V_j (128 keys each,
//               gathered page by page from the paged pool) into a 3-stage K
//               ring and a 2-stage V ring
//   warp 1      MMA issuer (one lane): S_i = Q_i K_j^T and O_i += P_i V_j
//   warps 2-3   rewrite each landed V tile in place from bf16 to fp16
//   warps 4-7   softmax of tile Q0, warps 8-11 softmax of tile Q1: one query
//               row per thread, read from TMEM, online softmax with a lazily
//               rescaled O (only when the running max grows by > 2^8), P
//               written back into TMEM over the S columns as fp16, then the
//               final O / l epilogue, staged in shared memory (over the
//               tile's Q buffer) and written by TMA stores
// The two softmax groups ping-pong: while one computes exponentials the tensor
// core runs the other tile's MMAs.
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512);
// P of tile i aliases columns [0,64) of S_i (two fp16 per column).
// Shared memory: Q0, Q1 (2 x 32 KB) + 3 K stages + 2 V stages of 32 KB, all
// 128-byte swizzled; each operand is two 64-column halves of [128 rows][128 B].
#pragma once
#include "common.cuh"
#include "params.cuh"

namespace oomattn {

constexpr int kPfThreads = 384;
constexpr int kPfConvThreads = 64;                // warps 2-3 convert V tiles bf16 -> fp16
constexpr int kPfKStages = 3;                     // K ring: a stage frees once both S MMAs of its tile finish
constexpr int kPfVStages = 2;                     // V ring: a stage frees once both P.V MMAs finish
constexpr int kTileBytes = 128 * kHeadDim * 2;    // 32 KB: one 128 x 128 bf16 operand tile
constexpr int kHalfTileBytes = kTileBytes / 2;    // one 64-column half
constexpr int kPfSmemBytes = (2 + kPfKStages + kPfVStages) * kTileBytes + 1024 + 256;
constexpr float kRescaleThreshold = 8.0f;         // log2 units: rescale O only when the max grows by > 256x
constexpr int kPfLaunchRegs = 168;                // 65536 / 384, rounded down to a multiple of 8
constexpr int kPfProducerRegs = 88;
constexpr int kPfSoftmaxRegs = 208;
static_assert(128 * kPfProducerRegs + 256 * kPfSoftmaxRegs <= kPfThreads * kPfLaunchRegs,
              "register split exceeds the launch allocation");

constexpr int kPfMaxRanges = 4;

struct PrefillArgs {
  void* out;           // [n_new][n_heads][128]
  int out_bf16;
  float* lse;          // [n_new][n_heads] natural log, or null
  int n_new;
  int prefix;          // P: cache slots before the chunk
  int seq;
  int layer;
  int n_heads;
  int group;
  int n_pairs;         // ceil(n_new / 256)
  // The 256-row query blocks ("pairs") this launch computes: ranges [lo, hi)
  // ordered by descending lo, so that taking each range from its top gives
  // the whole grid in descending causal work (one range [0, n_pairs) by
  // default; a rank of a sharded prefill takes its zig-zag share).
  int n_ranges;
  int range_lo[kPfMaxRanges];
  int range_hi[kPfMaxRanges];
  // Key split: grid.y indexes chunks of key_chunk 128-key tiles; a unit
  // (pair, head, chunk) covers key tiles [chunk * key_chunk, + key_chunk).
  // A pair whose last tile needs more than key_chunk key tiles writes each
  // chunk's normalised O and lse as partials (rows padded to n_pad per chunk)
  // for prefill_chunk_merge_kernel; other pairs write out directly.
  int key_chunk;
  int n_pad;           // n_new rounded up to 128
  float* part_lse;     // [chunks][n_pad][n_heads] natural log
  float qscale;        // softmax scale * log2(e)
  int* status;
  unsigned long long timeout_ns;
};

// ------------------------------------------------------------ tcgen05 PTX
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Same two MMAs with each descriptor given as 32-bit halves (lo carries the
// start address), so callers advance only a 32-bit register per k-step.
__device__ __forceinline__ void mma_ss_lh(uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi, uint32_t b_lo, uint32_t b_hi,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "mov.b64 da, {%1, %2};\n\t"
      "mov.b64 db, {%3, %4};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %5, p;\n\t}" ::"r"(d_tmem),
      "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_ts_lh(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t b_hi,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 db;\n\t"
      "setp.ne.b32 p, %5, 0;\n\t"
      "mov.b64 db, {%2, %3};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %4, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

#define OOMATTN_TMEM_LD32(taddr, r)                                                                               \
  asm volatile(                                                                                                   \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18," \
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                                              \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),            \
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),      \
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),    \
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])     \
      : "r"(taddr))

#define OOMATTN_TMEM_ST32(taddr, r)                                                                                \
  asm volatile(                                                                                                    \
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17," \
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),                                \
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),           \
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),   \
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),  \
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])                                                   \
      : "memory")

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------ epilogue helpers
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}
// Named barrier over the 128 threads (4 warps) of one softmax tile.
__device__ __forceinline__ void tile_bar(int id) { asm volatile("bar.sync %0, 128;" ::"r"(id) : "memory"); }
// The same barrier, returning whether `pred` holds in all 128 threads.
__device__ __forceinline__ bool tile_bar_and(int id, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %2, 0;\n\t"
      "bar.red.and.pred q, %1, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(id), "r"((uint32_t)pred)
      : "memory");
  return r != 0;
}
// 3D tiled bulk-tensor store from this CTA's shared memory (innermost x a multiple of 16 bytes).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until every committed bulk store has finished reading its shared memory.
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor (sm_100 format): start address, leading /
// stride byte offsets (16-byte units), version 1, layout type 2 = 128B swizzle.
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;   // descriptor version for sm_100
  d |= (uint64_t)2 << 61;   // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: f32 accumulate, A and B both bf16 (or
// both fp16), M = 128, N = 128; b_mn_major selects an N-contiguous B operand
// (V in P.V).
__host__ __device__ constexpr uint32_t make_idesc_f16kind(bool bf16, bool b_mn_major) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         ((128u >> 3) << 17) | ((128u >> 4) << 24);
}
__host__ __device__ constexpr uint32_t make_idesc_bf16(bool b_mn_major) { return make_idesc_f16kind(true, b_mn_major); }

// ------------------------------------------------------------ the kernel
__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_bf16_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap omap,
                        const __grid_constant__ CUtensorMap pmap, const KVPool pool, const PrefillArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                // [2 tiles][2 halves][128][128 B]
  uint8_t* sK = smem + 2 * kTileBytes;               // [K stage][2 halves][128][128 B]
  uint8_t* sV = sK + kPfKStages * kTileBytes;        // [V stage][2 halves][128][128 B]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kPfVStages * kTileBytes);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;                       // [kPfKStages]
  uint64_t* k_empty = k_full + kPfKStages;           // [kPfKStages]
  uint64_t* v_full = k_empty + kPfKStages;           // [kPfVStages]
  uint64_t* v_empty = v_full + kPfVStages;           // [kPfVStages]
  uint64_t* v_conv = v_empty + kPfVStages;           // [kPfVStages]: V stage converted to fp16
  uint64_t* s_full = v_conv + kPfVStages;            // [2]
  uint64_t* p_full = s_full + 2;                     // [2 tiles][2 halves of P]
  uint64_t* o_full = p_full + 4;                     // [2]
  uint64_t* mma_done = o_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // heaviest work first: block b -> the (b / n_heads)-th pair of the ranges
  // taken top down, head b % n_heads
  const int h = blockIdx.x % a.n_heads;
  int pair = 0;
  {
    // unrolled with constant indices, so the ranges are read from the
    // parameter space rather than copied to a local array
    int k = (int)(blockIdx.x / a.n_heads);
    bool found = false;
#pragma unroll
    for (int r = 0; r < kPfMaxRanges; ++r) {
      const int n = a.range_hi[r] - a.range_lo[r];
      if (!found && r < a.n_ranges) {
        if (k < n) {
          pair = a.range_hi[r] - 1 - k;
          found = true;
        } else {
          k -= n;
        }
      }
    }
  }
  const int g = h / a.group;
  const int q0 = pair * 256;
  int rows_valid[2], ntile[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    rows_valid[i] = max(0, min(128, a.n_new - (q0 + 128 * i)));
    // KV tiles needed by the last valid row (slot P + q0 + 128 i + rows - 1)
    ntile[i] = rows_valid[i] > 0 ? (a.prefix + q0 + 128 * i + rows_valid[i] + 127) / 128 : 0;
  }
  // this unit's chunk of key tiles: absolute tiles jb + j for local j < ntl[i]
  const int jb = (int)blockIdx.y * a.key_chunk;
  int ntl[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) ntl[i] = max(0, min(ntile[i], jb + a.key_chunk) - jb);
  const int n_kv_tiles = max(ntl[0], ntl[1]);
  if (n_kv_tiles == 0) return;  // a chunk past this pair's keys: the whole CTA leaves
  const bool split_pair = max(ntile[0], ntile[1]) > a.key_chunk;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kPfKStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < kPfVStages; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&v_conv[s], kPfConvThreads);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[2 * i], 4);      // one elected lane per softmax warp
      mbar_init(&p_full[2 * i + 1], 4);
      mbar_init(&o_full[i], 1);
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Register split: the kernel launches with kPfLaunchRegs per thread (the host
  // checks the compiled count before launching); warpgroup 0 (TMA, MMA and two
  // idle warps) gives (168-88)*128 registers back at the top of its branches and
  // the two softmax warpgroups take (208-168)*256 -- the same number, so the
  // increase never waits.
#define OOMATTN_REGS_DEC() asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kPfProducerRegs))
#define OOMATTN_REGS_INC() asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kPfSoftmaxRegs))

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    OOMATTN_REGS_DEC();
    if (lane == 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      prefetch_tensormap(&omap);
      prefetch_tensormap(&pmap);
      mbar_arrive_expect_tx(q_full, 2 * kTileBytes);
      for (int i = 0; i < 2; ++i)
        for (int c = 0; c < 2; ++c)
          tma_load_3d(sQ + i * kTileBytes + c * kHalfTileBytes, &qmap, q_full, c * 64, h, q0 + 128 * i);
      const int* bt = pool.block_table + (size_t)a.seq * pool.max_pages_per_seq;
      const int null_page = pool.n_pool_pages - 1;
      // The pool rows of a 128-key tile: its 8 pages' block-table entries, read
      // together (one latency per tile, shared by K and V; the next tile's are
      // fetched while this tile's copies are issued).
      auto tile_rows = [&](int j, int* rows) {
        int pages[8];
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const int lp = j * 8 + p;
          pages[p] = lp < pool.max_pages_per_seq ? __ldg(bt + lp) : null_page;
        }
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          int page = pages[p];
          if ((unsigned)page >= (unsigned)pool.n_pool_pages) {
            report_error(a.status, kDevErrBounds);
            page = null_page;
          }
          rows[p] = ((a.layer * pool.n_pool_pages + page) * pool.n_kv + g) * kPageSize;
        }
      };
      // one 128-key tile = 8 pages x two 64-column boxes of 16 rows, stacked at 2 KB steps
      auto load_tile = [&](uint8_t* dst, const CUtensorMap* map, uint64_t* bar, const int* rows) {
        mbar_arrive_expect_tx(bar, kTileBytes);
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          tma_load_2d(dst + p * 2048, map, bar, 0, rows[p]);
          tma_load_2d(dst + p * 2048 + kHalfTileBytes, map, bar, 64, rows[p]);
        }
      };
      bool ok = true;
      int rows[8], next_rows[8];
      if (n_kv_tiles > 0) tile_rows(jb, rows);
      for (int j = 0; j < n_kv_tiles && ok; ++j) {
        const int sk = j % kPfKStages, sv = j % kPfVStages;
        if (j >= kPfKStages) ok = mbar_wait(&k_empty[sk], ((j / kPfKStages) - 1) & 1, a.status, a.timeout_ns);
        if (!ok) break;
        load_tile(sK + sk * kTileBytes, &kmap, &k_full[sk], rows);
        if (j + 1 < n_kv_tiles) tile_rows(jb + j + 1, next_rows);
        if (j >= kPfVStages) ok = mbar_wait(&v_empty[sv], ((j / kPfVStages) - 1) & 1, a.status, a.timeout_ns);
        if (!ok) break;
        load_tile(sV + sv * kTileBytes, &vmap, &v_full[sv], rows);
#pragma unroll
        for (int p = 0; p < 8; ++p) rows[p] = next_rows[p];
      }
      // drain: the last loads this lane issued land before the CTA can exit
      for (int j = max(0, n_kv_tiles - kPfKStages); j < n_kv_tiles; ++j)
        mbar_wait(&k_full[j % kPfKStages], (j / kPfKStages) & 1, a.status, a.timeout_ns);
      for (int j = max(0, n_kv_tiles - kPfVStages); j < n_kv_tiles; ++j)
        mbar_wait(&v_full[j % kPfVStages], (j / kPfVStages) & 1, a.status, a.timeout_ns);
      mbar_wait(q_full, 0, a.status, a.timeout_ns);
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    OOMATTN_REGS_DEC();
    if (lane == 0) {
      constexpr uint32_t idesc_qk = make_idesc_bf16(false);
      constexpr uint32_t idesc_pv = make_idesc_f16kind(false, true);  // P fp16 x V fp16
      bool ok = mbar_wait(q_full, 0, a.status, a.timeout_ns);
      tc_fence_after();
      // Descriptor bases are built once; each MMA only adds a compile-time
      // offset (in 16-byte units) to the start-address field, which cannot
      // carry out of its 14 bits because shared memory ends below 256 KB.  This
      // keeps the single issuing thread at a few instructions per MMA, ahead of
      // the 64-cycle MMA rate even while it shares its scheduler with softmax warps.
      const uint64_t dq = make_sdesc(smem_u32(sQ), 16, 1024);
      const uint64_t dk = make_sdesc(smem_u32(sK), 16, 1024);
      const uint64_t dv = make_sdesc(smem_u32(sV), kHalfTileBytes, 1024);
      const uint32_t dq_hi = (uint32_t)(dq >> 32), dk_hi = (uint32_t)(dk >> 32), dv_hi = (uint32_t)(dv >> 32);
      // S_i(j) = Q_i K_j^T : 8 k-steps of 16 dims; halves at +16 KB, steps +32 B inside a half
      auto issue_s = [&](int i, int j) {
        const uint32_t a0 = (uint32_t)dq + i * (kTileBytes >> 4);
        const uint32_t b0 = (uint32_t)dk + (j % kPfKStages) * (kTileBytes >> 4);
        const uint32_t d = tmem + i * 128;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * (kHalfTileBytes >> 4) + (kk & 3) * 2;
          mma_ss_lh(d, a0 + off, dq_hi, b0 + off, dk_hi, idesc_qk, kk > 0 ? 1u : 0u);
        }
      };
      // O_i (+)= P_i V_j in fp16 x fp16 : 8 k-steps of 16 keys; P from TMEM
      // (8 columns per step); V (converted to fp16 in place) N-major: LBO =
      // 16 KB between 64-dim halves, SBO = 1 KB between 8-key groups
      // one half = keys [64*half, 64*half+64): k-steps 4*half .. 4*half+3
      auto issue_pv_half = [&](int i, int j, int half) {
        const uint32_t b0 = (uint32_t)dv + (j % kPfVStages) * (kTileBytes >> 4);
        const uint32_t d = tmem + 256 + i * 128, p = tmem + i * 128;
        const uint32_t first = (j > 0 || half > 0) ? 1u : 0u;
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const int kk = half * 4 + k4;
          mma_ts_lh(d, p + kk * 8, b0 + kk * (2048 >> 4), dv_hi, idesc_pv, k4 > 0 ? 1u : first);
        }
      };
      int k_waited = -1, v_waited = -1;
      auto wait_k = [&](int j) {
        if (ok && j > k_waited) {
          ok = mbar_wait(&k_full[j % kPfKStages], (j / kPfKStages) & 1, a.status, a.timeout_ns);
          tc_fence_after();
          k_waited = j;
        }
      };
      auto wait_v = [&](int j) {
        if (ok && j > v_waited) {
          ok = mbar_wait(&v_conv[j % kPfVStages], (j / kPfVStages) & 1, a.status, a.timeout_ns);
          tc_fence_after();
          v_waited = j;
        }
      };
      // tile i uses K/V tile j when j < ntile[i]; ntile[1] >= ntile[0] unless Q1 is empty,
      // so the last user of a tile in issue order is Q1 when Q1 uses it, else Q0
      auto last_user = [&](int j) { return j < ntl[1] ? 1 : 0; };
      // Each commit tracks every MMA issued before it, so committing a ring's
      // "empty" barrier right after the last MMA that reads the stage frees it
      // as soon as those MMAs finish.
      if (ok && n_kv_tiles > 0) {
        wait_k(0);
        for (int i = 0; i < 2 && ok; ++i)
          if ((i ? ntl[1] : ntl[0]) > 0) {
            issue_s(i, 0);
            tc_commit(&s_full[i]);
          }
        tc_commit(&k_empty[0]);
      }
      for (int j = 0; j < n_kv_tiles && ok; ++j) {
        for (int i = 0; i < 2 && ok; ++i) {
          if (j >= (i ? ntl[1] : ntl[0])) continue;
          wait_v(j);
          if (!ok) break;
          ok = mbar_wait(&p_full[2 * i], j & 1, a.status, a.timeout_ns);
          if (!ok) break;
          tc_fence_after();
          issue_pv_half(i, j, 0);
          ok = mbar_wait(&p_full[2 * i + 1], j & 1, a.status, a.timeout_ns);
          if (!ok) break;
          tc_fence_after();
          issue_pv_half(i, j, 1);
          if (i == last_user(j)) tc_commit(&v_empty[j % kPfVStages]);
          if (j + 1 < (i ? ntl[1] : ntl[0])) {
            wait_k(j + 1);
            if (!ok) break;
            issue_s(i, j + 1);
            tc_commit(&s_full[i]);
            if (i == last_user(j + 1)) tc_commit(&k_empty[(j + 1) % kPfKStages]);
          } else {
            tc_commit(&o_full[i]);
          }
        }
      }
      // every MMA this lane issued has completed before TMEM can be released
      tc_commit(mma_done);
      mbar_wait(mma_done, 0, a.status, a.timeout_ns);
    }
  } else if (warp < 4) {
    // ------------------------------------------------ V converters (warps 2-3)
    // Each V tile lands as bf16; these 64 threads rewrite it in place as fp16
    // (exact for |v| < 65536) so that P.V runs as an fp16 x fp16 MMA with P
    // carrying 11 significant bits.  A bf16 value of magnitude >= 65536 has no
    // fp16 image: it is reported through the status word.
    OOMATTN_REGS_DEC();
    const int ct = threadIdx.x - 64;  // 0..63
    bool ok = true;
    uint32_t big = 0;
    for (int j = 0; j < n_kv_tiles && ok; ++j) {
      const int s = j % kPfVStages;
      ok = mbar_wait(&v_full[s], (j / kPfVStages) & 1, a.status, a.timeout_ns);
      if (!ok) break;
      uint4* tile = reinterpret_cast<uint4*>(sV + s * kTileBytes);
#pragma unroll 4
      for (int c = ct; c < kTileBytes / 16; c += kPfConvThreads) {
        uint4 w = tile[c];
        big = max(big, max_exp_bf16x8(w.x, w.y, w.z, w.w));
        w.x = bf16x2_to_f16x2(w.x);
        w.y = bf16x2_to_f16x2(w.y);
        w.z = bf16x2_to_f16x2(w.z);
        w.w = bf16x2_to_f16x2(w.w);
        tile[c] = w;
      }
      fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
      mbar_arrive(&v_conv[s]);
    }
    if (big >= 0x4780u) report_error(a.status, kDevErrRange);
  } else {
    // ------------------------------------------------ softmax / epilogue
    OOMATTN_REGS_INC();
    const int i = (warp - 4) >> 2;           // q tile
    const int quarter = warp & 3;            // TMEM lane quarter of this warp
    const int r = quarter * 32 + lane;       // row within the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int row_in_chunk = q0 + 128 * i + r;
    const int qslot = a.prefix + row_in_chunk;  // absolute cache slot of this query
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    const float cl = a.qscale;
    for (int j = 0; j < (i ? ntl[1] : ntl[0]) && ok; ++j) {
      ok = mbar_wait(&s_full[i], j & 1, a.status, a.timeout_ns);
      if (!ok) break;
      tc_fence_after();
      uint32_t sr[128];
      OOMATTN_TMEM_LD32((tmem + i * 128) + lane_off + 0, (sr + 0));
      OOMATTN_TMEM_LD32((tmem + i * 128) + lane_off + 32, (sr + 32));
      OOMATTN_TMEM_LD32((tmem + i * 128) + lane_off + 64, (sr + 64));
      OOMATTN_TMEM_LD32((tmem + i * 128) + lane_off + 96, (sr + 96));
      tmem_wait_ld();
      const int lim = qslot - (jb + j) * 128;  // columns c <= lim are visible
      if (__any_sync(0xffffffffu, lim < 127)) {
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (c > lim) sr[c] = __float_as_uint(-INFINITY);
      }
      // row max: 8 independent 3-input max chains, then a short tree
      float mv[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mv[k] = fmaxf(__uint_as_float(sr[2 * k]), __uint_as_float(sr[2 * k + 1]));
#pragma unroll
      for (int c = 16; c < 128; c += 16)
#pragma unroll
        for (int k = 0; k < 8; ++k)
          mv[k] = max3f(mv[k], __uint_as_float(sr[c + 2 * k]), __uint_as_float(sr[c + 2 * k + 1]));
      const float mx = max3f(max3f(mv[0], mv[1], mv[2]), max3f(mv[3], mv[4], mv[5]), fmaxf(mv[6], mv[7]));
      const float mxs = mx * cl;
      bool need = false;
      float alpha = 1.f;
      if (j == 0) {
        m_used = mxs;
      } else if (mxs > m_used + kRescaleThreshold) {
        need = true;
        alpha = exp2f(m_used - mxs);
        m_used = mxs;
        l *= alpha;
      }
      // O must be rescaled before the first P.V of this tile: that MMA is
      // released with P's first half below.  (Rare: lazy rescale.)
      if (__any_sync(0xffffffffu, need)) {
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t orr[32];
          OOMATTN_TMEM_LD32((tmem + 256 + i * 128) + lane_off + ch * 32, orr);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 32; ++c) orr[c] = __float_as_uint(__uint_as_float(orr[c]) * alpha);
          OOMATTN_TMEM_ST32((tmem + 256 + i * 128) + lane_off + ch * 32, orr);
        }
      }
      // P in fp16 (11 significant bits, 8x finer than bf16; p <= 2^8 after the
      // lazy rescale, far inside fp16 range) packed in place over the scores
      // (step c reads sr[2c], sr[2c+1] and writes sr[c], c <= 2c) and stored
      // into S columns [0,64) in two halves of 64 keys.  Each half is released
      // to the MMA thread on its own barrier, so the P.V of keys 0..63 runs
      // while keys 64..127 are still being exponentiated.  One elected lane per
      // warp arrives (barrier count 4).  The scale-and-shift and the row sum
      // run as packed f32x2 FMA-pipe instructions, the exponential on MUFU.
      const uint64_t cl2 = f2_pack(cl, cl);
      // a row with no visible key yet (possible only in a key-split chunk past
      // its own slot) keeps m = -inf: shift by 0 so its masked scores give p = 0
      const float m_eff = m_used == -INFINITY ? 0.f : m_used;
      const uint64_t nm2 = f2_pack(-m_eff, -m_eff);
      uint64_t acc[4] = {0, 0, 0, 0};
#pragma unroll
      for (int half = 0; half < 2; ++half) {
#pragma unroll
        for (int cc = 0; cc < 32; ++cc) {
          const int c = half * 32 + cc;
          const uint64_t t = f2_fma(f2_pack(__uint_as_float(sr[2 * c]), __uint_as_float(sr[2 * c + 1])), cl2, nm2);
          const float p0 = ex2_ftz(f2_lo(t)), p1 = ex2_ftz(f2_hi(t));
          acc[c & 3] = f2_add(acc[c & 3], f2_pack(p0, p1));
          sr[c] = pack_f16(p0, p1);
        }
        OOMATTN_TMEM_ST32((tmem + i * 128) + lane_off + half * 32, (sr + half * 32));
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[2 * i + half]);
      }
      const uint64_t acc2 = f2_add(f2_add(acc[0], acc[1]), f2_add(acc[2], acc[3]));
      l += f2_lo(acc2) + f2_hi(acc2);
    }
    // Epilogue: O / l staged in shared memory and written by TMA stores.
    // The staging area is this tile's Q buffer (every MMA that read it has
    // completed once o_full fires), 32 KB: f32 output goes out in two rounds
    // of 64 columns, bf16 in one.  Each round is two boxes of [128 rows][128 B]
    // in the 128-byte-swizzled layout, so a warp's 16-byte shared stores hit
    // distinct banks; one thread of the tile issues the stores, which clip the
    // rows past n_new.  The tile's 128 threads agree on the outcome of the
    // bounded o_full wait before any of them enters a named barrier.
    if ((i ? ntl[1] : ntl[0]) > 0) {
      bool okw = ok && mbar_wait(&o_full[i], 0, a.status, a.timeout_ns);
      tc_fence_after();
      okw = tile_bar_and(1 + i, okw);
      if (okw) {
        const float inv = l > 0.f ? 1.f / l : 0.f;  // l = 0: no visible key in this chunk
        uint8_t* stage = sQ + i * kTileBytes;
        const uint32_t st0 = smem_u32(stage) + (uint32_t)r * 128u;
        const uint32_t rsw = (uint32_t)(r & 7);
        const bool issuer = quarter == 0 && lane == 0;
        // a split pair's chunk goes to its partial rows: chunk y at rows [y * n_pad, ...)
        const CUtensorMap* tmap = split_pair ? &pmap : &omap;
        const int qrow0 = (split_pair ? (int)blockIdx.y * a.n_pad : 0) + q0 + 128 * i;
        if (a.out_bf16 && !split_pair) {  // partials stay f32
#pragma unroll
          for (int b = 0; b < 2; ++b) {  // box b: columns [64 b, 64 b + 64)
            uint32_t orr[64];
            OOMATTN_TMEM_LD32((tmem + 256 + i * 128) + lane_off + b * 64, orr);
            OOMATTN_TMEM_LD32((tmem + 256 + i * 128) + lane_off + b * 64 + 32, (orr + 32));
            tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 8; ++c)
              st_shared_v4(st0 + b * kHalfTileBytes + (((uint32_t)c ^ rsw) << 4),
                           pack_bf16(__uint_as_float(orr[8 * c + 0]) * inv, __uint_as_float(orr[8 * c + 1]) * inv),
                           pack_bf16(__uint_as_float(orr[8 * c + 2]) * inv, __uint_as_float(orr[8 * c + 3]) * inv),
                           pack_bf16(__uint_as_float(orr[8 * c + 4]) * inv, __uint_as_float(orr[8 * c + 5]) * inv),
                           pack_bf16(__uint_as_float(orr[8 * c + 6]) * inv, __uint_as_float(orr[8 * c + 7]) * inv));
          }
          fence_proxy_async_smem();
          tile_bar(1 + i);
          if (issuer) {
            tma_store_3d(tmap, stage, 0, h, qrow0);
            tma_store_3d(tmap, stage + kHalfTileBytes, 64, h, qrow0);
            bulk_commit_group();
            bulk_wait_group_read0();
          }
        } else {
#pragma unroll
          for (int c2 = 0; c2 < 2; ++c2) {  // round c2: columns [64 c2, 64 c2 + 64)
            if (c2 == 1) tile_bar(1 + i);  // the issuer has seen round 0's reads of the staging area end
#pragma unroll
            for (int b = 0; b < 2; ++b) {  // box b: 32 columns
              uint32_t orr[32];
              OOMATTN_TMEM_LD32((tmem + 256 + i * 128) + lane_off + (2 * c2 + b) * 32, orr);
              tmem_wait_ld();
#pragma unroll
              for (int c = 0; c < 8; ++c)
                st_shared_v4(st0 + b * kHalfTileBytes + (((uint32_t)c ^ rsw) << 4),
                             __float_as_uint(__uint_as_float(orr[4 * c + 0]) * inv),
                             __float_as_uint(__uint_as_float(orr[4 * c + 1]) * inv),
                             __float_as_uint(__uint_as_float(orr[4 * c + 2]) * inv),
                             __float_as_uint(__uint_as_float(orr[4 * c + 3]) * inv));
            }
            fence_proxy_async_smem();
            tile_bar(1 + i);
            if (issuer) {
              tma_store_3d(tmap, stage, 64 * c2, h, qrow0);
              tma_store_3d(tmap, stage + kHalfTileBytes, 64 * c2 + 32, h, qrow0);
              bulk_commit_group();
              bulk_wait_group_read0();
            }
          }
        }
        const bool valid = r < (i ? rows_valid[1] : rows_valid[0]);
        if (valid && split_pair)
          a.part_lse[((size_t)blockIdx.y * a.n_pad + row_in_chunk) * a.n_heads + h] =
              (l > 0.f ? (m_used + log2f(l)) * 0.69314718055994531f : -INFINITY);
        else if (valid && a.lse)
          a.lse[(size_t)row_in_chunk * a.n_heads + h] = (l > 0.f ? (m_used + log2f(l)) * 0.69314718055994531f : -INFINITY);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// The rows of key-split pairs: out[row][h] = sum_c w_c O_c / sum_c w_c with
// w_c = e^(lse_c - max lse) over the chunks that hold work for the row's tile
// (chunk c does when c * key_chunk < the tile's key-tile count; a row that
// sees no key of such a chunk has its lse at -inf there, and chunk 0, which
// holds key 0, is never empty).  One warp per (row,
// head), 4 dimensions per lane; rows of unsplit pairs, or outside the
// launch's block ranges, were written by the prefill kernel itself.
__global__ void prefill_chunk_merge_kernel(const float* __restrict__ part_o, const PrefillArgs a) {
  const long long item = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (item >= (long long)a.n_new * a.n_heads) return;
  const int row = (int)(item / a.n_heads), h = (int)(item - (long long)row * a.n_heads);
  const int pair = row >> 8;
  bool mine = false;
#pragma unroll
  for (int r = 0; r < kPfMaxRanges; ++r)
    if (r < a.n_ranges && pair >= a.range_lo[r] && pair < a.range_hi[r]) mine = true;
  const int pair_end = min(a.n_new, 256 * pair + 256);
  if (!mine || (a.prefix + pair_end + 127) / 128 <= a.key_chunk) return;
  const int tile_end = min(a.n_new, (row / 128) * 128 + 128);
  const int nt = (a.prefix + tile_end + 127) / 128;
  const int nc = (nt + a.key_chunk - 1) / a.key_chunk;
  float M = -INFINITY;
  for (int c = 0; c < nc; ++c) M = fmaxf(M, a.part_lse[((size_t)c * a.n_pad + row) * a.n_heads + h]);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float wsum = 0.f;
  for (int c = 0; c < nc; ++c) {
    const float w = expf(a.part_lse[((size_t)c * a.n_pad + row) * a.n_heads + h] - M);
    const float4 o = __ldg(reinterpret_cast<const float4*>(part_o + (((size_t)c * a.n_pad + row) * a.n_heads + h) *
                                                           kHeadDim) + lane);
    wsum += w;
    acc.x += w * o.x;
    acc.y += w * o.y;
    acc.z += w * o.z;
    acc.w += w * o.w;
  }
  const float inv = 1.f / wsum;
  const size_t o_off = ((size_t)row * a.n_heads + h) * kHeadDim + lane * 4;
  if (a.out_bf16) {
    uint2 v;
    v.x = pack_bf16(acc.x * inv, acc.y * inv);
    v.y = pack_bf16(acc.z * inv, acc.w * inv);
    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(a.out) + o_off) = v;
  } else {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(a.out) + o_off) =
        make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
  }
  if (a.lse && lane == 0) a.lse[(size_t)row * a.n_heads + h] = M + logf(wsum);
}

}  // namespace oomattn
