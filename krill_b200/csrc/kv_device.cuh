// kv_device.cuh — device helpers shared by the attention kernels: bounded
// mbarrier waits, bulk async copies, the m16n8k16 tensor-core MMA, the
// reference-exact u8 -> f16 dequantization and the sub-block geometry.
#pragma once
#include "internal.h"

namespace krill {
namespace {

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ uint32_t mbar_try_wait(uint32_t bar, uint32_t phase) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(phase)
      : "memory");
  return done;
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
// Every kernel with bounded waits keeps two shared-memory words: cta_abort[0]
// (set once a wait of the CTA ran out) and cta_abort[1], the pool's wait
// limit in microseconds (a launch parameter), set when the CTA starts.
__device__ __forceinline__ void init_wait_state(volatile int* cta_abort, int wait_us) {
  cta_abort[0] = 0;
  cta_abort[1] = wait_us > 0 ? wait_us : kDefaultWaitUs;
}
// Bound of a device-side wait in units of 1,024 ns (elapsed globaltimer ns
// >> 10): the pool's limit, or about 20 us once the CTA has already seen a
// timeout.
__device__ __forceinline__ uint32_t wait_limit_units(volatile int* cta_abort) {
  return cta_abort[0] ? 20u : (uint32_t)cta_abort[1];
}
// Bounded wait: gives up after the pool's limit (100 ms by default), records
// the error and returns false. The bound is far above any legitimate wait (a
// 17 KB copy) yet short enough that a fault ends the launch instead of
// hanging the GPU.
__device__ bool mbar_wait(uint32_t bar, uint32_t phase, volatile int* cta_abort, int* err) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint32_t limit = wait_limit_units(cta_abort);
  const uint64_t t0 = globaltimer();
  for (;;) {
    // the clock is read once per 16 polls: it is off the wake-up path
    for (int k = 0; k < 16; ++k)
      if (mbar_try_wait(bar, phase)) return true;
    if (((globaltimer() - t0) >> 10) > limit) {
      *cta_abort = 1;
      atomicOr(err, kErrTimeout);
      return false;
    }
  }
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma16816_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Two u8 codes (bytes selected by `sel` from w) -> f16x2 dequantized with the
// reference's rounding: f16_rn(f16_rn(c * s) + z). PRMT builds 1024 + c
// exactly (exponent byte 0x64), the subtraction of 1024 is exact.
__device__ __forceinline__ uint32_t deq2(uint32_t w, uint32_t sel, uint32_t s2, uint32_t z2) {
  __half2 c = u2h(__byte_perm(w, 0x64646464u, sel));
  c = __hsub2_rn(c, u2h(0x64006400u));
  c = __hmul2_rn(c, u2h(s2));
  c = __hadd2_rn(c, u2h(z2));
  return h2u(c);
}

// Same result with one operation less, exact whenever |s| < 64:
// fma(1024 + c, s, -1024*s) rounds the exact product c*s once (-1024*s is
// exact in f16, subnormal s included), then + z rounds again.
__device__ __forceinline__ uint32_t deq2_fast(uint32_t w, uint32_t sel, uint32_t s2, uint32_t ns2,
                                              uint32_t z2) {
  __half2 c = u2h(__byte_perm(w, 0x64646464u, sel));
  c = __hfma2(c, u2h(s2), u2h(ns2));
  c = __hadd2_rn(c, u2h(z2));
  return h2u(c);
}
__device__ __forceinline__ uint32_t neg1024(uint32_t s2) {
  return h2u(__hmul2_rn(u2h(s2), u2h(0xE400E400u)));  // -1024 in f16
}

template <int D, int NG, int FMT = kFmtInt8>
struct SubGeom {
  static constexpr int G = D / NG;
  static constexpr int T = FMT == kFmtBf16 ? sub_tokens_raw(D) : sub_tokens(D);
  static constexpr int SPB = kBlockTokens / T;
  static constexpr int NU = T / 16;          // 16-token m-tiles per sub-block
  static constexpr int TPT = T / 4;          // tokens per lane chunk (V rows)
  static constexpr int SB = FMT == kFmtBf16 ? T * 4 * D : T * (2 * D + 8 * NG);
  static constexpr int VOFF = FMT == kFmtBf16 ? T * D * 2 : T * D;
  static constexpr int META = 2 * T * D;     // int8 only
  // meta array a, group gi, token t -> byte offset (int8 only)
  static __device__ __forceinline__ int meta(int a, int gi, int t) {
    return META + ((a * NG + gi) * T + t) * 2;
  }
};

__device__ __forceinline__ uint32_t f2h2(float lo, float hi) {
  return h2u(__floats2half2_rn(lo, hi));
}
// bf16 pair -> f16 pair; exact for magnitudes in the f16 normal range
__device__ __forceinline__ uint32_t bf2h2(uint32_t w) {
  return f2h2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

__device__ __forceinline__ void store_out(void* out, int dtype, int64_t i, float v) {
  if (dtype == 0)
    reinterpret_cast<__half*>(out)[i] = __float2half_rn(v);
  else if (dtype == 1)
    reinterpret_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<float*>(out)[i] = v;
}

}  // namespace
}  // namespace krill
