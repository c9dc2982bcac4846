// Shared device helpers for the sm_100a attention kernels: mbarriers with
// bounded waits, TMA tile loads into the issuing CTA only, legacy-MMA fragments for the
// decode path, bf16 packing, and the error-status word every kernel reports to.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace oomattn {

// Status bits a kernel ORs into the context's device status word.
enum : int {
  kDevErrTimeout = 1,      // a bounded wait on an mbarrier gave up
  kDevErrBounds = 2,       // a page / position index failed its device check
  kDevErrTmem = 4,         // tensor-memory allocation returned an unusable address
  kDevErrRange = 8,        // a cached V value of magnitude >= 65536 met the fp16 P.V product
  kDevErrX16 = 16,         // a Q8-linear activation of magnitude >= 65504 met its fp16 hi/lo split
  kDevErrFormat = 32,      // a .oom Q8 block's length field disagrees with its position in the tensor
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void report_error(int* status, int bit) {
  if (status) atomicOr(status, bit);
}

// ---------------------------------------------------------------- mbarriers
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Asynchronous global -> shared copies (per thread, no registers held while
// in flight): 4 bytes through L1, 16 bytes through L2 only (data that other
// CTAs wrote during this launch, which this SM's L1 may hold stale).
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16_cg(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait until the barrier's phase with the given parity has completed.  Gives
// up after `timeout_ns` of wall time, records kDevErrTimeout and returns false,
// so a lost arrival ends the kernel with an error instead of hanging the GPU.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, uint64_t timeout_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 255u) == 0) {
      if (global_timer_ns() - t0 > timeout_ns) {
        report_error(status, kDevErrTimeout);
        return false;
      }
    }
  }
}

// An arrival at a counter shared by CTAs that merge partial results: one
// thread's acquire-release add after a barrier of the threads that wrote their
// partials releases those writes (the barrier orders them before it) and
// acquires the partials the earlier arrivals released, so neither side needs
// a fence in every thread.
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// ---------------------------------------------------------------- TMA loads
// 2D tiled bulk-tensor load into this CTA's shared memory, completing on `bar`.
// x is the innermost coordinate; callers keep x * element size a multiple of
// 16 bytes.  Every TMA load in this library lands in the issuing CTA's own
// shared memory and reads this GPU's own memory.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- legacy MMA
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                              uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D(16x8,f32) += A(16x16,bf16,row) * B(16x8,bf16,col)
__device__ __forceinline__ void mma_bf16_16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// ---------------------------------------------------------------- bf16 bits
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);  // .x = lo (low 16 bits), .y = hi
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float bf16_lo_f32(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi_f32(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// Split (a, b) into hi = bf16(x) and lo = bf16(x - hi) pairs so that two
// bf16 MMAs reproduce the f32 operand to ~16 significant bits.
__device__ __forceinline__ void split_bf16x2(float a, float b, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16(a, b);
  lo = pack_bf16(a - bf16_lo_f32(hi), b - bf16_hi_f32(hi));
}

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float x) {
  __nv_bfloat16 h = __float2bfloat16_rn(x);
  return *reinterpret_cast<uint16_t*>(&h);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }

// ---------------------------------------------------------------- Blackwell scalar helpers
// Hardware base-2 exponential (MUFU), flushing results below 2^-126 to 0.
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float m;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(a), "f"(b), "f"(c));
  return m;
}
// Two f32 lanes in one 64-bit register for the packed FMA-pipe instructions.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  return ((uint64_t)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// fp16 pair (round to nearest even): a in the low half, b in the high half.
__device__ __forceinline__ uint32_t pack_f16(float a, float b) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(b), "f"(a));
  return d;
}
// bf16 pair -> fp16 pair (exact for |x| < 65536; larger magnitudes become inf).
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t x) {
  return pack_f16(__uint_as_float(x << 16), __uint_as_float(x & 0xffff0000u));
}
// Largest bf16 exponent field (bits 14..7 of a half, as 0x0000..0x7f80) among
// the eight bf16 values of four packed pairs.
__device__ __forceinline__ uint32_t max_exp_bf16x8(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  const uint32_t m = __vmaxu2(__vmaxu2(a & 0x7f807f80u, b & 0x7f807f80u), __vmaxu2(c & 0x7f807f80u, d & 0x7f807f80u));
  return max(m & 0xffffu, m >> 16);
}
// bf16 pair holding the upper 16 bits (truncation) of a (low half) and b (high half).
__device__ __forceinline__ uint32_t trunc_bf16x2(float a, float b) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, 0x7632;" : "=r"(d) : "r"(__float_as_uint(a)), "r"(__float_as_uint(b)));
  return d;
}

// Byte offset of element column e (0..127) of row r inside one 16-row x
// 128-column bf16 block stored as two 64-column halves of 16 x 128 B with the
// TMA 128-byte swizzle (16-byte chunk index XOR row % 8).
__device__ __forceinline__ uint32_t sw128_off(int r, int e) {
  return (uint32_t)((e >> 6) * 2048 + r * 128 + ((((e & 63) >> 3) ^ (r & 7)) << 4) + ((e & 7) << 1));
}

}  // namespace oomattn
