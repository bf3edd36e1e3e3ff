// kv_quant.cuh — the per-token quantizer core of the warp-per-token append
// kernels (kv_ops.cu): a warp quantizes one token's K and V rows, lanes
// [k*LPG, (k+1)*LPG) holding one group of EPL elements each. Reference: QuantizedKVCache.quantizePerHead
// (Sources/KrillCache/QuantizedKVCache.swift:181-197), applied per
// `group_size` slice of head_dim, every rounding step the reference's.
#pragma once
#include "internal.h"

namespace krill {
namespace {

template <int EPL>
struct VecIn;  // EPL 16-bit inputs per lane
template <> struct VecIn<2> { using T = uint32_t; };
template <> struct VecIn<4> { using T = uint2; };
template <> struct VecIn<8> { using T = uint4; };

__device__ inline float bits_to_float(uint16_t b, int dtype) {
  return dtype == 0 ? __half2float(__ushort_as_half(b)) : __bfloat162float(__ushort_as_bfloat16(b));
}

// Quantize EPL elements held by this lane; lanes [k*LPG, (k+1)*LPG) form one
// group. Returns codes packed little-endian in `codes`, plus the group's f16
// scale / zero bits.
// code = trunc(clip(RN(a / s), 0, 255)) for a = rn_in(x - mn) >= 0, bit for bit
// as with the IEEE divide the reference performs, without a divide per
// element.
//   qa = RN(a * rinv), rinv = RN(1 / s), is within 2^-23 (relative: two
//   roundings of 2^-24) of the exact quotient q, i.e. within 3.1e-5 for
//   q <= 256. trunc(RN(q)) only changes where q crosses m_k = k - h_k, the
//   midpoint below an integer k (h_k = half the spacing of the floats just
//   below k, 2^(E-24) with 2^E the binade of k - 0.5; h_k <= 2^-17 for
//   k <= 256). So when qa lies at least 1e-4 from the nearest integer k,
//   trunc(qa) = trunc(RN(q)).
//   Otherwise RN(q) >= k exactly when q >= m_k (a tie rounds to k, whose
//   significand is even), i.e. when a - k s + h_k s >= 0. r = fma(-k, s, a)
//   is exact there (|a - k s| < 1.4e-4 s, a multiple of the smaller of the
//   two operands' spacings, needs fewer than 24 bits), h_k s is exact (a
//   power-of-two scaling), and the sign of RN(r + h_k s) is the sign of the
//   exact sum (no underflow: both are multiples of 2^-75 at these
//   magnitudes). About 0.2 % (f16) to 2 % (bf16) of N(0,1) elements take
//   that branch; the group minimum (a = 0) gives 0. Non-finite or
//   out-of-range quotients fall back to the divide.
// s24 = s * 2^-24.
__device__ __forceinline__ uint8_t code_of(float a, float s, float rinv, float s24) {
  if (a == 0.0f) return 0;
  const float qa = a * rinv;
  const float k = rintf(qa);
  if (!(qa < 512.0f)) {  // NaN / inf / out of range: the divide decides
    const float n = fminf(fmaxf(__fdiv_rn(a, s), 0.0f), 255.0f);
    return (uint8_t)__float2int_rz(n);
  }
  if (fabsf(qa - k) >= 1e-4f) return (uint8_t)__float2int_rz(fminf(qa, 255.0f));
  if (k >= 256.0f) return 255;
  if (k <= 0.0f) return 0;
  const float r = fmaf(-k, s, a);
  const float p2 = __uint_as_float(__float_as_uint(k - 0.5f) & 0x7f800000u);
  const float up = r + s24 * p2;
  return (uint8_t)(__float2int_rz(k) - (up >= 0.0f ? 0 : 1));
}

template <int EPL, int LPG>
__device__ inline void quantize_lane(const float (&x)[EPL], int dtype, int variant,
                                     uint8_t (&codes)[EPL], uint16_t& s16, uint16_t& z16) {
  float mn = x[0], mx = x[0];
#pragma unroll
  for (int e = 1; e < EPL; ++e) { mn = fminf(mn, x[e]); mx = fmaxf(mx, x[e]); }
#pragma unroll
  for (int off = 1; off < LPG; off <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  }
  float d = round_in(mx - mn, dtype);
  float scale;
  if (variant == 0) {
    scale = fmaxf(__fdiv_rn(d, 255.0f), 1e-8f);
  } else {
    scale = fmaxf(round_in(__fdiv_rn(d, 255.0f), dtype), round_in(1e-8f, dtype));
  }
  if (variant == 0) {
    const float rinv = __frcp_rn(scale);
    const float s24 = scale * 5.9604644775390625e-08f;  // 2^-24
#pragma unroll
    for (int e = 0; e < EPL; ++e) codes[e] = code_of(round_in(x[e] - mn, dtype), scale, rinv, s24);
  } else {
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      float n = round_in(__fdiv_rn(round_in(x[e] - mn, dtype), scale), dtype);
      n = fminf(fmaxf(n, 0.0f), 255.0f);
      codes[e] = (uint8_t)__float2int_rz(n);
    }
  }
  s16 = __half_as_ushort(__float2half_rn(scale));
  z16 = __half_as_ushort(__float2half_rn(mn));
}

template <int EPL>
__device__ inline void load_row(const void* src, int64_t elem_off, int lane, int dtype,
                                float (&x)[EPL]) {
  using T = typename VecIn<EPL>::T;
  const T* p = reinterpret_cast<const T*>(reinterpret_cast<const uint16_t*>(src) + elem_off) + lane;
  T v = *p;
  const uint16_t* h = reinterpret_cast<const uint16_t*>(&v);
#pragma unroll
  for (int e = 0; e < EPL; ++e) x[e] = bits_to_float(h[e], dtype);
}

template <int EPL>
__device__ inline void store_kcodes(uint8_t* sb, int D, int t, int lane, const uint8_t (&c)[EPL]) {
  int64_t off = sb_kcode(D, t, lane * EPL);
  if constexpr (EPL == 2) {
    *reinterpret_cast<uint16_t*>(sb + off) = (uint16_t)(c[0] | (c[1] << 8));
  } else if constexpr (EPL == 4) {
    *reinterpret_cast<uint32_t*>(sb + off) =
        (uint32_t)c[0] | ((uint32_t)c[1] << 8) | ((uint32_t)c[2] << 16) | ((uint32_t)c[3] << 24);
  } else {
    uint2 w;
    w.x = (uint32_t)c[0] | ((uint32_t)c[1] << 8) | ((uint32_t)c[2] << 16) | ((uint32_t)c[3] << 24);
    w.y = (uint32_t)c[4] | ((uint32_t)c[5] << 8) | ((uint32_t)c[6] << 16) | ((uint32_t)c[7] << 24);
    *reinterpret_cast<uint2*>(sb + off) = w;
  }
}

// One token's K and V rows (input row elem_off / D), K rotated at `pos` when a
// rotary table is given, quantized per group: the per-token core shared by
// both append kernels, so both produce the same bits.
template <int EPL>
__device__ __forceinline__ typename VecIn<EPL>::T load_raw(const void* src, int64_t elem_off,
                                                            int lane) {
  using T = typename VecIn<EPL>::T;
  return *(reinterpret_cast<const T*>(reinterpret_cast<const uint16_t*>(src) + elem_off) + lane);
}
template <int EPL>
__device__ __forceinline__ void raw_to_float(const typename VecIn<EPL>::T& r, int dtype,
                                             float (&x)[EPL]) {
  const uint16_t* h = reinterpret_cast<const uint16_t*>(&r);
#pragma unroll
  for (int e = 0; e < EPL; ++e) x[e] = bits_to_float(h[e], dtype);
}

template <int EPL, int LPG>
__device__ __forceinline__ void quant_values(float (&xk)[EPL], float (&xv)[EPL], int64_t pos, int D,
                                             int lane, int dtype, int variant,
                                             const RopeTable& rope, uint8_t (&ck)[EPL],
                                             uint8_t (&cv)[EPL], uint16_t& sk, uint16_t& zk,
                                             uint16_t& sv, uint16_t& zv);

template <int EPL, int LPG>
__device__ __forceinline__ void quant_token(const void* __restrict__ k, const void* __restrict__ v,
                                            int64_t elem_off, int64_t pos, int D, int lane,
                                            int dtype, int variant, const RopeTable& rope,
                                            uint8_t (&ck)[EPL], uint8_t (&cv)[EPL], uint16_t& sk,
                                            uint16_t& zk, uint16_t& sv, uint16_t& zv) {
  float xk[EPL], xv[EPL];
  load_row<EPL>(k, elem_off, lane, dtype, xk);
  load_row<EPL>(v, elem_off, lane, dtype, xv);
  quant_values<EPL, LPG>(xk, xv, pos, D, lane, dtype, variant, rope, ck, cv, sk, zk, sv, zv);
}

template <int EPL, int LPG>
__device__ __forceinline__ void quant_values(float (&xk)[EPL], float (&xv)[EPL], int64_t pos, int D,
                                             int lane, int dtype, int variant,
                                             const RopeTable& rope, uint8_t (&ck)[EPL],
                                             uint8_t (&cv)[EPL], uint16_t& sk, uint16_t& zk,
                                             uint16_t& sv, uint16_t& zv) {
  if (rope.cos) {
    // Rotate-half RoPE at the token's absolute position (MLXFast.RoPE with
    // traditional: false): element d < D/2 pairs with d + D/2, which lives 16
    // lanes away. Unfused f32 products and sum, then the input-dtype rounding
    // the reference's rotated K carries before it is quantized.
    const int half = D / 2;
    const float* cr = rope.cos + pos * half;
    const float* sr = rope.sin + pos * half;
    float other[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) other[e] = __shfl_xor_sync(0xffffffffu, xk[e], 16);
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const int i = (lane * EPL + e) % half;
      const float c = __ldg(cr + i), sn = __ldg(sr + i);
      const float y = lane < 16 ? __fsub_rn(__fmul_rn(xk[e], c), __fmul_rn(other[e], sn))
                                : __fadd_rn(__fmul_rn(other[e], sn), __fmul_rn(xk[e], c));
      xk[e] = round_in(y, dtype);
    }
  }
  quantize_lane<EPL, LPG>(xk, dtype, variant, ck, sk, zk);
  quantize_lane<EPL, LPG>(xv, dtype, variant, cv, sv, zv);
}

}  // namespace
}  // namespace krill
