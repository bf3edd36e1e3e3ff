// kv_ops.cu — fused quantize+append, and the gather/scatter kernels behind
// snapshots, restores and the continuous-batch stack/scatter glue.
//
// Quantizer: reference QuantizedKVCache.quantizePerHead
// (Sources/KrillCache/QuantizedKVCache.swift:181-197), applied per
// `group_size` slice of head_dim. Every rounding step is the reference's
// (MLX CPU-device semantics), so codes, scales and zeros are bit-exact:
//   mn/mx exact; d = rn_in(mx - mn); scale = max(d / 255f, 1e-8f) in f32
//   (IEEE divide, __fdiv_rn); code = trunc(clip(rn_in(x - mn) / scale, 0, 255));
//   stored scale f16_rn(scale), zero f16_rn(mn).
// Dequantize (:200-204): f16_rn(f16_rn(f16(code) * scale) + zero).
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

// One warp per (layer, seq, kv-head, new token): quantize its K row and V row
// and write codes + meta straight into the destination sub-block (appends of
// a few tokens, i.e. decode steps).
template <int EPL, int LPG>
__global__ void __launch_bounds__(256) append_quantize_kernel(uint8_t* __restrict__ pool, Geom geom,
                                                              const AppendDst* __restrict__ dst,
                                                              int layer_begin, int layer_count,
                                                              int n_seqs, int n_new,
                                                              const void* __restrict__ k,
                                                              const void* __restrict__ v, int dtype,
                                                              int* __restrict__ large_scale,
                                                              RopeTable rope) {
  // A decode step's attention kernel may be launched as this kernel's
  // programmatic dependent: let it be scheduled now (it waits for this grid's
  // completion before it reads the pool).
  asm volatile("griddepcontrol.launch_dependents;");
  const int lane = threadIdx.x & 31;
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t total = (int64_t)layer_count * n_seqs * geom.Hkv * n_new;
  if (w >= total) return;
  const int D = geom.D;
  const int tok = (int)(w % n_new);
  const int64_t rest = w / n_new;
  const int h = (int)(rest % geom.Hkv);
  const int64_t ls = rest / geom.Hkv;  // li * n_seqs + si
  const int li = (int)(ls / n_seqs);
  const AppendDst d = dst[ls * n_new + tok];
  const int slot = d.pos & (kBlockTokens - 1);
  const int t = slot % geom.subt;
  uint8_t* sb = pool + (((int64_t)d.block * geom.L + (layer_begin + li)) * geom.Hkv + h) * geom.page_bytes +
                (int64_t)(slot / geom.subt) * geom.sb_bytes;

  uint8_t ck[EPL], cv[EPL];
  uint16_t sk, zk, sv, zv;
  quant_token<EPL, LPG>(k, v, w * D, d.pos, D, lane, dtype, geom.quant_variant, rope, ck, cv, sk, zk,
                        sv, zv);

  store_kcodes<EPL>(sb, D, t, lane, ck);
#pragma unroll
  for (int e = 0; e < EPL; ++e) sb[sb_vcode(D, t, lane * EPL + e)] = cv[e];
  if ((lane % LPG) == 0) {
    const int gi = lane / LPG;
    const int NG = geom.NG;
    *reinterpret_cast<uint16_t*>(sb + sb_meta(D, NG, 0, gi, t)) = sk;
    *reinterpret_cast<uint16_t*>(sb + sb_meta(D, NG, 1, gi, t)) = zk;
    *reinterpret_cast<uint16_t*>(sb + sb_meta(D, NG, 2, gi, t)) = sv;
    *reinterpret_cast<uint16_t*>(sb + sb_meta(D, NG, 3, gi, t)) = zv;
    if ((sk & 0x7fffu) >= 0x5400u || (sv & 0x7fffu) >= 0x5400u) atomicOr(large_scale, 1);
  }
}

// Appends of many tokens (prefill chunks): one CTA of 8 warps per (layer, seq,
// kv head, destination sub-block). Each warp quantizes tokens with the same
// per-token core and writes its K row directly (one coalesced row), but the
// transposed V codes and the scales / zeros, which the one-warp-per-token
// kernel scatters as single bytes and halves, are staged in shared memory and
// written row by row: 16-byte stores when the call covers the whole sub-block,
// else only the covered slots (other tokens of the sub-block stay untouched).
template <int EPL, int LPG>
__global__ void __launch_bounds__(256) append_tile_kernel(uint8_t* __restrict__ pool, Geom geom,
                                                          const AppendDst* __restrict__ dst,
                                                          int layer_begin, int n_seqs, int n_new,
                                                          int n_chunks, const void* __restrict__ k,
                                                          const void* __restrict__ v, int dtype,
                                                          int* __restrict__ large_scale,
                                                          RopeTable rope) {
  asm volatile("griddepcontrol.launch_dependents;");  // as in append_quantize_kernel
  extern __shared__ __align__(16) uint8_t app_smem[];
  const int D = geom.D, T = geom.subt, NG = geom.NG;
  int64_t b = blockIdx.x;
  const int c = (int)(b % n_chunks);
  b /= n_chunks;
  const int h = (int)(b % geom.Hkv);
  const int64_t ls = b / geom.Hkv;  // li * n_seqs + si
  // positions of the call's tokens for this (layer, seq): [p0, p0 + n_new);
  // chunk c is the c-th sub-block they touch
  const int64_t p0 = dst[ls * n_chunks].pos;
  const int64_t cs = p0 - p0 % T + (int64_t)c * T;  // first position of the sub-block
  const int64_t s0 = max(p0, cs), e0 = min(p0 + n_new, cs + T);
  if (s0 >= e0) return;
  const int t_lo = (int)(s0 - cs), t_hi = (int)(e0 - cs);
  const AppendDst d0 = dst[ls * n_chunks + c];
  const int slot0 = d0.pos & (kBlockTokens - 1);
  uint8_t* sb = pool + (((int64_t)d0.block * geom.L + (layer_begin + (ls / n_seqs))) * geom.Hkv + h) *
                           geom.page_bytes +
                (int64_t)(slot0 / T) * geom.sb_bytes;
  // V codes token-major, rows of D + 4 bytes: a lane stores its EPL codes of a
  // token as one packed word (consecutive lanes, consecutive words), and the
  // odd word count per row spreads the column reads of the write-out over
  // the banks
  const int S = D + 4;
  uint8_t* vtile = app_smem;                                                   // [T][S]
  uint16_t* mtile = reinterpret_cast<uint16_t*>(app_smem + (size_t)T * S);  // [4][NG][T]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  bool large = false;
  for (int t = t_lo + warp; t < t_hi; t += 8) {
    uint8_t ck[EPL], cv[EPL];
    uint16_t sk, zk, sv, zv;
    quant_token<EPL, LPG>(k, v, ((ls * geom.Hkv + h) * n_new + (cs + t - p0)) * D, cs + t, D, lane,
                          dtype, geom.quant_variant, rope, ck, cv, sk, zk, sv, zv);
    store_kcodes<EPL>(sb, D, t, lane, ck);
    {
      uint8_t* vp = vtile + t * S + lane * EPL;
      if constexpr (EPL == 2) {
        *reinterpret_cast<uint16_t*>(vp) = (uint16_t)(cv[0] | (cv[1] << 8));
      } else {
#pragma unroll
        for (int w4 = 0; w4 < EPL / 4; ++w4)
          reinterpret_cast<uint32_t*>(vp)[w4] =
              (uint32_t)cv[4 * w4] | ((uint32_t)cv[4 * w4 + 1] << 8) |
              ((uint32_t)cv[4 * w4 + 2] << 16) | ((uint32_t)cv[4 * w4 + 3] << 24);
      }
    }
    if ((lane % LPG) == 0) {
      const int gi = lane / LPG;
      mtile[(0 * NG + gi) * T + t] = sk;
      mtile[(1 * NG + gi) * T + t] = zk;
      mtile[(2 * NG + gi) * T + t] = sv;
      mtile[(3 * NG + gi) * T + t] = zv;
      large |= (sk & 0x7fffu) >= 0x5400u || (sv & 0x7fffu) >= 0x5400u;
    }
  }
  if (large) atomicOr(large_scale, 1);
  __syncthreads();
  uint8_t* vdst = sb + sb_voff(D);
  uint16_t* mdst = reinterpret_cast<uint16_t*>(sb + sb_meta_off(D));
  if (t_lo == 0 && t_hi == T) {
    // 16 tokens of one V row per 16-byte store, gathered from the token-major tile
    const int cpr = T / 16, nv = D * cpr, nm = 4 * NG * T * 2 / 16;
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
      const int r = i / cpr, t0 = (i % cpr) * 16;
      uint32_t w[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint8_t* c = vtile + (t0 + 4 * q) * S + r;
        w[q] = (uint32_t)c[0] | ((uint32_t)c[S] << 8) | ((uint32_t)c[2 * S] << 16) |
               ((uint32_t)c[3 * S] << 24);
      }
      reinterpret_cast<uint4*>(vdst)[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
    for (int i = threadIdx.x; i < nm; i += blockDim.x)
      reinterpret_cast<uint4*>(mdst)[i] = reinterpret_cast<const uint4*>(mtile)[i];
  } else {
    const int wdt = t_hi - t_lo;
    for (int i = threadIdx.x; i < D * wdt; i += blockDim.x) {
      const int r = i / wdt, t = t_lo + i % wdt;
      vdst[r * T + t] = vtile[t * S + r];
    }
    for (int i = threadIdx.x; i < 4 * NG * wdt; i += blockDim.x) {
      const int r = i / wdt, t = t_lo + i % wdt;
      mdst[r * T + t] = mtile[r * T + t];
    }
  }
}

// Raw bf16 pools (the unquantized comparison format): copy one token's K row
// and V column; one warp per (layer, seq, head, token), bf16 inputs.
__global__ void append_raw_kernel(uint8_t* __restrict__ pool, Geom geom,
                                  const AppendDst* __restrict__ dst, int layer_begin,
                                  int layer_count, int n_seqs, int n_new,
                                  const uint16_t* __restrict__ k, const uint16_t* __restrict__ v) {
  asm volatile("griddepcontrol.launch_dependents;");  // as in append_quantize_kernel
  const int lane = threadIdx.x & 31;
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t total = (int64_t)layer_count * n_seqs * geom.Hkv * n_new;
  if (w >= total) return;
  const int D = geom.D;
  const int tok = (int)(w % n_new);
  const int64_t rest = w / n_new;
  const int h = (int)(rest % geom.Hkv);
  const int64_t ls = rest / geom.Hkv;  // li * n_seqs + si
  const int li = (int)(ls / n_seqs);
  const AppendDst d = dst[ls * n_new + tok];
  const int slot = d.pos & (kBlockTokens - 1);
  const int t = slot % geom.subt;
  uint8_t* sb = pool + (((int64_t)d.block * geom.L + (layer_begin + li)) * geom.Hkv + h) * geom.page_bytes +
                (int64_t)(slot / geom.subt) * geom.sb_bytes;
  const int64_t elem_off = w * D;
  for (int c = lane; c < D / 8; c += 32)
    *reinterpret_cast<uint4*>(sb + raw_koff(D, t, 8 * c)) =
        *reinterpret_cast<const uint4*>(k + elem_off + 8 * c);
  for (int e = lane; e < D; e += 32)
    *reinterpret_cast<uint16_t*>(sb + raw_voff(D, geom.subt, t, e)) = v[elem_off + e];
}

// Gather rows [p0, p0+S) of one (seq, layer) into the reference snapshot
// layout; one thread per (head, row, element-of-8). mode 0: raw codes + meta;
// mode 1: dequantized f16 (keys/values are f16 outputs).
__global__ void gather_kernel(const uint8_t* __restrict__ pool, Geom geom, int layer,
                              const int32_t* __restrict__ bt, int64_t p0, int64_t S,
                              GatherOut out) {
  const int D = geom.D, NG = geom.NG, G = geom.G;
  const int per_row = D / 8;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)geom.Hkv * S * per_row;
  if (idx >= total) return;
  const int e8 = (int)(idx % per_row);
  const int64_t hr = idx / per_row;
  const int64_t i = hr % S;
  const int h = (int)(hr / S);
  const int64_t pos = p0 + i;
  int64_t bidx = pos >> 8;
  if (geom.ring > 0) bidx %= geom.ring;
  const int blk = bt[bidx];
  const int slot = (int)(pos & 255);
  const int t = slot % geom.subt;
  const uint8_t* sb = pool + (((int64_t)blk * geom.L + layer) * geom.Hkv + h) * geom.page_bytes +
                      (int64_t)(slot / geom.subt) * geom.sb_bytes;
  const int64_t orow = (int64_t)h * out.rows_total + out.row_off + i;
  const int d0 = e8 * 8;
  uint8_t kc[8], vc[8];
  // 8 consecutive K codes sit inside one 16-byte chunk.
  const uint2 kw = *reinterpret_cast<const uint2*>(sb + sb_kcode(D, t, d0));
  const uint8_t* kb = reinterpret_cast<const uint8_t*>(&kw);
#pragma unroll
  for (int e = 0; e < 8; ++e) { kc[e] = kb[e]; vc[e] = sb[sb_vcode(D, t, d0 + e)]; }
  const int gi = d0 / G;
  const uint16_t ks = *reinterpret_cast<const uint16_t*>(sb + sb_meta(D, NG, 0, gi, t));
  const uint16_t kz = *reinterpret_cast<const uint16_t*>(sb + sb_meta(D, NG, 1, gi, t));
  const uint16_t vs = *reinterpret_cast<const uint16_t*>(sb + sb_meta(D, NG, 2, gi, t));
  const uint16_t vz = *reinterpret_cast<const uint16_t*>(sb + sb_meta(D, NG, 3, gi, t));
  if (out.mode == 0) {
    if (out.keys) *reinterpret_cast<uint2*>(out.keys + orow * D + d0) = kw;
    if (out.values) {
      uint2 vw;
      vw.x = vc[0] | (vc[1] << 8) | (vc[2] << 16) | ((uint32_t)vc[3] << 24);
      vw.y = vc[4] | (vc[5] << 8) | (vc[6] << 16) | ((uint32_t)vc[7] << 24);
      *reinterpret_cast<uint2*>(out.values + orow * D + d0) = vw;
    }
    if ((d0 % G) == 0) {
      const int64_t m = orow * NG + gi;
      if (out.key_scales) out.key_scales[m] = ks;
      if (out.key_zeros) out.key_zeros[m] = kz;
      if (out.value_scales) out.value_scales[m] = vs;
      if (out.value_zeros) out.value_zeros[m] = vz;
    }
  } else {
    const __half hks = __ushort_as_half(ks), hkz = __ushort_as_half(kz);
    const __half hvs = __ushort_as_half(vs), hvz = __ushort_as_half(vz);
    __half* ok = reinterpret_cast<__half*>(out.keys);
    __half* ov = reinterpret_cast<__half*>(out.values);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if (ok) ok[orow * D + d0 + e] = __hadd_rn(__hmul_rn(__ushort2half_rn(kc[e]), hks), hkz);
      if (ov) ov[orow * D + d0 + e] = __hadd_rn(__hmul_rn(__ushort2half_rn(vc[e]), hvs), hvz);
    }
  }
}

// Scatter rows from the snapshot layout into a sequence's pages (restore,
// scatter-back). Row i of the input (at in.row_off + i) lands at position p0+i.
__global__ void scatter_kernel(uint8_t* __restrict__ pool, Geom geom, int layer,
                               const int32_t* __restrict__ bt, int64_t p0, int64_t S, ScatterIn in,
                               int* __restrict__ large_scale) {
  const int D = geom.D, NG = geom.NG, G = geom.G;
  const int per_row = D / 8;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t total = (int64_t)geom.Hkv * S * per_row;
  if (idx >= total) return;
  const int e8 = (int)(idx % per_row);
  const int64_t hr = idx / per_row;
  const int64_t i = hr % S;
  const int h = (int)(hr / S);
  const int64_t pos = p0 + i;
  int64_t bidx = pos >> 8;
  if (geom.ring > 0) bidx %= geom.ring;
  const int blk = bt[bidx];
  const int slot = (int)(pos & 255);
  const int t = slot % geom.subt;
  uint8_t* sb = pool + (((int64_t)blk * geom.L + layer) * geom.Hkv + h) * geom.page_bytes +
                (int64_t)(slot / geom.subt) * geom.sb_bytes;
  const int64_t irow = (int64_t)h * in.rows_total + in.row_off + i;
  const int d0 = e8 * 8;
  const uint2 kw = *reinterpret_cast<const uint2*>(in.keys + irow * D + d0);
  const uint2 vw = *reinterpret_cast<const uint2*>(in.values + irow * D + d0);
  *reinterpret_cast<uint2*>(sb + sb_kcode(D, t, d0)) = kw;
  const uint8_t* vb = reinterpret_cast<const uint8_t*>(&vw);
#pragma unroll
  for (int e = 0; e < 8; ++e) sb[sb_vcode(D, t, d0 + e)] = vb[e];
  if ((d0 % G) == 0) {
    const int gi = d0 / G;
    const int64_t m = irow * NG + gi;
    *reinterpret_cast<uint16_t*>(sb + sb_meta(D, NG, 0, gi, t)) = in.key_scales[m];
    *reinterpret_cast<uint16_t*>(sb + sb_meta(D, NG, 1, gi, t)) = in.key_zeros[m];
    *reinterpret_cast<uint16_t*>(sb + sb_meta(D, NG, 2, gi, t)) = in.value_scales[m];
    *reinterpret_cast<uint16_t*>(sb + sb_meta(D, NG, 3, gi, t)) = in.value_zeros[m];
    if ((in.key_scales[m] & 0x7fffu) >= 0x5400u || (in.value_scales[m] & 0x7fffu) >= 0x5400u)
      atomicOr(large_scale, 1);
  }
}

}  // namespace

cudaError_t launch_append(const Geom& g, uint8_t* pool, const AppendDst* d_dst, int layer_begin,
                          int layer_count, int n_seqs, int n_new, const void* k, const void* v,
                          int dtype, int* large_scale, RopeTable rope, cudaStream_t stream) {
  const int64_t warps = (int64_t)layer_count * n_seqs * g.Hkv * n_new;
  if (warps == 0) return cudaSuccess;
  const int threads = 256;
  const int64_t blocks = (warps * 32 + threads - 1) / threads;
  if (g.fmt == kFmtBf16) {
    if (dtype != 1 || rope.cos) return cudaErrorInvalidValue;
    append_raw_kernel<<<(unsigned)blocks, threads, 0, stream>>>(
        pool, g, d_dst, layer_begin, layer_count, n_seqs, n_new,
        static_cast<const uint16_t*>(k), static_cast<const uint16_t*>(v));
    return cudaGetLastError();
  }
  const int epl = g.D / 32;
  const int lpg = g.G / epl;
  // Multi-token appends take the tiled kernel (whole sub-blocks per CTA);
  // decode-sized ones keep one warp per token.
  const bool tiled = append_uses_tiles(n_new);
  const int n_chunks = append_tile_chunks(n_new, g.subt);
  const int64_t tiles = (int64_t)layer_count * n_seqs * g.Hkv * n_chunks;
  const size_t tile_smem = (size_t)g.subt * (g.D + 4) + (size_t)4 * g.NG * g.subt * 2;
#define KRILL_APPEND(E, P)                                                                    \
  if (epl == E && lpg == P) {                                                                  \
    if (tiled) {                                                                               \
      append_tile_kernel<E, P><<<(unsigned)tiles, threads, tile_smem, stream>>>(               \
          pool, g, d_dst, layer_begin, n_seqs, n_new, n_chunks, k, v, dtype, large_scale,      \
          rope);                                                                               \
    } else {                                                                                   \
      append_quantize_kernel<E, P><<<(unsigned)blocks, threads, 0, stream>>>(                  \
          pool, g, d_dst, layer_begin, layer_count, n_seqs, n_new, k, v, dtype, large_scale,   \
          rope);                                                                               \
    }                                                                                          \
    return cudaGetLastError();                                                                 \
  }
  KRILL_APPEND(2, 32)   // D=64,  G=64
  KRILL_APPEND(4, 16)   // D=128, G=64
  KRILL_APPEND(4, 32)   // D=128, G=128
  KRILL_APPEND(8, 8)    // D=256, G=64
  KRILL_APPEND(8, 16)   // D=256, G=128
  KRILL_APPEND(8, 32)   // D=256, G=256
#undef KRILL_APPEND
  return cudaErrorInvalidValue;
}

cudaError_t launch_gather(const Geom& g, const uint8_t* pool, int layer, const int32_t* d_bt,
                          int64_t p0, int64_t S, const GatherOut& out, cudaStream_t stream) {
  const int64_t total = (int64_t)g.Hkv * S * (g.D / 8);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  gather_kernel<<<(unsigned)((total + threads - 1) / threads), threads, 0, stream>>>(pool, g, layer,
                                                                                     d_bt, p0, S, out);
  return cudaGetLastError();
}

cudaError_t launch_scatter(const Geom& g, uint8_t* pool, int layer, const int32_t* d_bt, int64_t p0,
                           int64_t S, const ScatterIn& in, int* large_scale, cudaStream_t stream) {
  const int64_t total = (int64_t)g.Hkv * S * (g.D / 8);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  scatter_kernel<<<(unsigned)((total + threads - 1) / threads), threads, 0, stream>>>(
      pool, g, layer, d_bt, p0, S, in, large_scale);
  return cudaGetLastError();
}

}  // namespace krill
