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
#include "kv_quant.cuh"

namespace krill {
namespace {


// One warp per (layer, seq, kv-head, new token): quantize its K row and V row
// and write codes + meta straight into the destination sub-block (appends of
// a few tokens, i.e. decode steps).
// DT: input dtype (0 f16, 1 bf16), compile-time so the roundings fold.
template <int EPL, int LPG, int DT>
__global__ void __launch_bounds__(256) append_quantize_kernel(uint8_t* __restrict__ pool, Geom geom,
                                                              const AppendDst* __restrict__ dst,
                                                              int layer_begin, int layer_count,
                                                              int n_seqs, int n_new,
                                                              const void* __restrict__ k,
                                                              const void* __restrict__ v,
                                                              int* __restrict__ large_scale,
                                                              RopeTable rope) {
  constexpr int dtype = DT;
  // A decode step's attention kernel may be launched as this kernel's
  // programmatic dependent: let it be scheduled now (it waits for this grid's
  // completion before it reads the pool).
  asm volatile("griddepcontrol.launch_dependents;");
  const int lane = threadIdx.x & 31;
  const int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t total = (int64_t)layer_count * n_seqs * geom.Hkv * n_new;
  if (w >= total) return;
  constexpr int D = 32 * EPL, T = sub_tokens(D), NG = 32 / LPG;
  const int tok = (int)(w % n_new);
  const int64_t rest = w / n_new;
  const int h = (int)(rest % geom.Hkv);
  const int64_t ls = rest / geom.Hkv;  // li * n_seqs + si
  const int li = (int)(ls / n_seqs);
  const AppendDst d = dst[ls * n_new + tok];
  const int slot = d.pos & (kBlockTokens - 1);
  const int t = slot % T;
  uint8_t* sb = pool + (((int64_t)d.block * geom.L + (layer_begin + li)) * geom.Hkv + h) * geom.page_bytes +
                (int64_t)(slot / T) * geom.sb_bytes;

  uint8_t ck[EPL], cv[EPL];
  uint16_t sk, zk, sv, zv;
  quant_token<EPL, LPG>(k, v, w * D, d.pos, D, lane, dtype, geom.quant_variant, rope, ck, cv, sk, zk,
                        sv, zv);

  store_kcodes<EPL>(sb, D, t, lane, ck);
#pragma unroll
  for (int e = 0; e < EPL; ++e) sb[sb_vcode(D, t, lane * EPL + e)] = cv[e];
  if ((lane % LPG) == 0) {
    const int gi = lane / LPG;
    *reinterpret_cast<uint16_t*>(sb + sb_meta(D, NG, 0, gi, t)) = sk;
    *reinterpret_cast<uint16_t*>(sb + sb_meta(D, NG, 1, gi, t)) = zk;
    *reinterpret_cast<uint16_t*>(sb + sb_meta(D, NG, 2, gi, t)) = sv;
    *reinterpret_cast<uint16_t*>(sb + sb_meta(D, NG, 3, gi, t)) = zv;
    if ((sk & 0x7fffu) >= 0x5400u || (sv & 0x7fffu) >= 0x5400u) atomicOr(large_scale, 1);
  }
}

// Appends of many tokens (prefill chunks): one CTA of T/4 warps per (layer,
// sequence, kv head, destination sub-block of T tokens). Warp w owns the
// sub-block's tokens [4w, 4w + 4): it issues the loads of all its rows
// first, quantizes them token by token (the same per-token core as
// append_quantize_kernel, so both produce the same bits), writes each K row
// as it goes, and keeps its lane's V codes and the group scales/zeros in
// registers. The V rows ([D][T], tokens contiguous) and the meta arrays
// ([4][NG][T]) then leave with one store per lane per row segment (4 bytes of
// V, 8 bytes of meta), with no shared-memory transpose. Tokens
// of the sub-block outside the call's range [t_lo, t_hi) are left untouched
// (byte stores on a partly covered segment).
template <int EPL, int LPG, int DT>
__global__ void __launch_bounds__(8 * sub_tokens(32 * EPL), 128 / sub_tokens(32 * EPL)) append_tile_kernel(uint8_t* __restrict__ pool, Geom geom,
                                                          const AppendDst* __restrict__ dst,
                                                          int layer_begin, int n_seqs, int n_new,
                                                          int n_chunks, const void* __restrict__ k,
                                                          const void* __restrict__ v,
                                                          int* __restrict__ large_scale,
                                                          RopeTable rope) {
  asm volatile("griddepcontrol.launch_dependents;");  // as in append_quantize_kernel
  constexpr int dtype = DT;
  constexpr int D = 32 * EPL, T = sub_tokens(D), NG = 32 / LPG, TPW = 4;
  constexpr int VW = 1;  // 32-bit words of one V row segment
  using In = typename VecIn<EPL>::T;
  uint32_t b = blockIdx.x;
  const int c = (int)(b % (uint32_t)n_chunks);
  b /= (uint32_t)n_chunks;
  const int h = (int)(b % (uint32_t)geom.Hkv);
  const int64_t ls = b / (uint32_t)geom.Hkv;  // li * n_seqs + si
  // positions of the call's tokens for this (layer, seq): [p0, p0 + n_new);
  // chunk c is the c-th sub-block they touch
  const int64_t p0 = dst[ls * n_chunks].pos;
  const int64_t cs = p0 - p0 % T + (int64_t)c * T;  // first position of the sub-block
  const int64_t s0 = max(p0, cs), e0 = min(p0 + n_new, cs + T);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int w0 = warp * TPW;
  const int t_lo = max((int)(s0 - cs), w0), t_hi = min((int)(e0 - cs), w0 + TPW);
  if (t_lo >= t_hi) return;
  const AppendDst d0 = dst[ls * n_chunks + c];
  const int slot0 = d0.pos & (kBlockTokens - 1);
  uint8_t* sb = pool +
                (((int64_t)d0.block * geom.L + (layer_begin + (int)((uint32_t)ls / (uint32_t)n_seqs))) *
                     geom.Hkv + h) * geom.page_bytes +
                (int64_t)(slot0 / T) * geom.sb_bytes;
  const int64_t row0 = (ls * geom.Hkv + h) * n_new + (cs - p0);  // input row of token t: row0 + t
  In rk[TPW], rv[TPW];
#pragma unroll
  for (int i = 0; i < TPW; ++i) {
    const int t = w0 + i;
    if (t >= t_lo && t < t_hi) {
      rk[i] = load_raw<EPL>(k, (row0 + t) * D, lane);
      rv[i] = load_raw<EPL>(v, (row0 + t) * D, lane);
    }
  }
  uint32_t vw[EPL][VW];  // this lane's V codes: element e, tokens w0.. packed by byte
  uint32_t mw[4][TPW / 2];  // this group's K/V scale and zero per token, two f16 per word
#pragma unroll
  for (int e = 0; e < EPL; ++e)
#pragma unroll
    for (int q = 0; q < VW; ++q) vw[e][q] = 0u;
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int q = 0; q < TPW / 2; ++q) mw[a][q] = 0u;
  bool large = false;
#pragma unroll
  for (int i = 0; i < TPW; ++i) {
    const int t = w0 + i;
    if (t < t_lo || t >= t_hi) continue;
    float xk[EPL], xv[EPL];
    raw_to_float<EPL>(rk[i], dtype, xk);
    raw_to_float<EPL>(rv[i], dtype, xv);
    uint8_t ck[EPL], cv[EPL];
    uint16_t sk, zk, sv, zv;
    quant_values<EPL, LPG>(xk, xv, cs + t, D, lane, dtype, geom.quant_variant, rope, ck, cv, sk, zk,
                           sv, zv);
    store_kcodes<EPL>(sb, D, t, lane, ck);
#pragma unroll
    for (int e = 0; e < EPL; ++e) vw[e][i / 4] |= (uint32_t)cv[e] << (8 * (i % 4));
    const int sh = 16 * (i % 2);
    mw[0][i / 2] |= (uint32_t)sk << sh;
    mw[1][i / 2] |= (uint32_t)zk << sh;
    mw[2][i / 2] |= (uint32_t)sv << sh;
    mw[3][i / 2] |= (uint32_t)zv << sh;
    large |= (sk & 0x7fffu) >= 0x5400u || (sv & 0x7fffu) >= 0x5400u;
  }
  const bool full = t_lo == w0 && t_hi == w0 + TPW;
  uint8_t* vdst = sb + sb_voff(D);
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    uint8_t* row = vdst + (lane * EPL + e) * T + w0;
    if (full) {
      *reinterpret_cast<uint32_t*>(row) = vw[e][0];
    } else {
#pragma unroll
      for (int i = 0; i < TPW; ++i)
        if (w0 + i >= t_lo && w0 + i < t_hi) row[i] = (uint8_t)(vw[e][i / 4] >> (8 * (i % 4)));
    }
  }
  if ((lane % LPG) == 0) {
    const int gi = lane / LPG;
    uint16_t* mdst = reinterpret_cast<uint16_t*>(sb + sb_meta_off(D));
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      uint16_t* m = mdst + (a * NG + gi) * T + w0;
      if (full) {
        *reinterpret_cast<uint2*>(m) = make_uint2(mw[a][0], mw[a][1]);
      } else {
#pragma unroll
        for (int i = 0; i < TPW; ++i)
          if (w0 + i >= t_lo && w0 + i < t_hi) m[i] = (uint16_t)(mw[a][i / 2] >> (16 * (i % 2)));
      }
    }
    if (large) atomicOr(large_scale, 1);
  }
}

// ---------------------------------------------------------------------------
// Row-per-lane append for multi-token calls (prefill chunks), quantization
// variant KRILL_QUANT_F32. Each lane owns one token of a sub-block (a warp =
// 32 consecutive tokens) and quantizes whole groups of its own K and V rows,
// so the group min/max needs no shuffles, and the V codes ([D][T], tokens
// contiguous) and the scales/zeros ([4][NG][T]) leave as 32 consecutive
// tokens per store instruction. Same arithmetic as quantize_lane, so the
// codes are the same bits:
//  - min/max over the group's input values (exact in any order);
//  - d = rn_in(mx - mn) in f32, scale = max(RN(d / 255), 1e-8);
//  - a = rn_in(x - mn): taken as the input dtype's own RN subtraction
//    (HSUB2). That equals rounding the f32 difference: the f32 difference of
//    two 16-bit floats is exact unless their exponents are far apart, and then
//    the f32 rounding moves it by less than 2^-24 relative while the input
//    dtype's rounding midpoints lie at least 2^-12 away, so both round alike;
//  - code_of(a, ...) as above.
// code_of without branches, for groups whose range d is finite (then every
// quotient is at most 256, so qa < 2^22 and the magic-number rounding
// below is exact). qa + 1.5 * 2^23 rounds qa to the nearest integer k in
// the low mantissa bits (ki, kf); trunc(qa) = k - (qa < k). The near-integer
// test is the exact one of code_of; both results are computed and selected.
// For k = 0 (a = 0 included) it yields 0.
__device__ __forceinline__ uint32_t code_nb(float a, float s, float rinv, float s24) {
  const float qa = a * rinv;
  const float m = qa + 12582912.0f;
  const int ki = __float_as_int(m) - 0x4B400000;
  const float kf = m - 12582912.0f;
  const float diff = qa - kf;
  const float r = fmaf(-kf, s, a);
  const float p2 = __uint_as_float(__float_as_uint(kf - 0.5f) & 0x7f800000u);
  const float up = fmaf(s24, p2, r);
  const bool down = fabsf(diff) >= 1e-4f ? diff < 0.0f : up < 0.0f;
  return (uint32_t)min(ki - (down ? 1 : 0), 255);
}

__device__ __forceinline__ uint32_t code_exact(float a, float s) {
  return (uint32_t)__float2int_rz(fminf(fmaxf(__fdiv_rn(a, s), 0.0f), 255.0f));
}

// The codes of one group by the IEEE divide, element by element (groups with
// a non-finite value; kept out of line).
__device__ __noinline__ void codes_by_divide(const uint32_t* w, int n, float mn, float s, int dt,
                                             uint32_t* codes) {
  for (int e = 0; e < n; ++e) {
    const uint32_t bits = (w[e / 2] >> (16 * (e % 2))) & 0xffffu;
    const float x = dt == 0 ? __half2float(__ushort_as_half((uint16_t)bits)) : __uint_as_float(bits << 16);
    const uint32_t c = code_exact(round_in(x - mn, dt), s);
    if (e % 4 == 0) codes[e / 4] = c;
    else codes[e / 4] |= c << (8 * (e % 4));
  }
}

template <int DT>
struct Pair;  // two packed 16-bit values of the input dtype
template <> struct Pair<0> {
  using T = __half2;
  static __device__ __forceinline__ T from(uint32_t w) { return *reinterpret_cast<T*>(&w); }
  static __device__ __forceinline__ uint32_t bits(T v) { return *reinterpret_cast<uint32_t*>(&v); }
  static __device__ __forceinline__ float lo(T v) { return __low2float(v); }
  static __device__ __forceinline__ float hi(T v) { return __high2float(v); }
};
template <> struct Pair<1> {
  using T = __nv_bfloat162;
  static __device__ __forceinline__ T from(uint32_t w) { return *reinterpret_cast<T*>(&w); }
  static __device__ __forceinline__ uint32_t bits(T v) { return *reinterpret_cast<uint32_t*>(&v); }
  static __device__ __forceinline__ float lo(T v) { return __uint_as_float(bits(v) << 16); }
  static __device__ __forceinline__ float hi(T v) { return __uint_as_float(bits(v) & 0xffff0000u); }
};

// Quantize one group of G values held as G/2 packed pairs; codes packed four
// per word, little-endian.
template <int G, int DT>
__device__ __forceinline__ void quantize_group_row(const uint32_t (&w)[G / 2], uint32_t (&codes)[G / 4],
                                                   uint16_t& s16, uint16_t& z16) {
  using P = Pair<DT>;
  typename P::T mn2 = P::from(w[0]), mx2 = mn2;
#pragma unroll
  for (int j = 1; j < G / 2; ++j) {
    mn2 = __hmin2(mn2, P::from(w[j]));
    mx2 = __hmax2(mx2, P::from(w[j]));
  }
  const float mn = fminf(P::lo(mn2), P::hi(mn2));
  const float mx = fmaxf(P::lo(mx2), P::hi(mx2));
  const float d = round_in(mx - mn, DT);
  const float scale = fmaxf(__fdiv_rn(d, 255.0f), 1e-8f);
  const float rinv = __frcp_rn(scale);
  const float s24 = scale * 5.9604644775390625e-08f;  // 2^-24
  typename P::T mnv;
  if constexpr (DT == 0) mnv = __float2half2_rn(mn);  // exact: mn is an input value
  else mnv = __float2bfloat162_rn(mn);
  if (isfinite(d)) {
#pragma unroll
    for (int j = 0; j < G / 2; ++j) {
      const typename P::T a2 = __hsub2_rn(P::from(w[j]), mnv);
      const uint32_t pr = code_nb(P::lo(a2), scale, rinv, s24) | (code_nb(P::hi(a2), scale, rinv, s24) << 8);
      if (j % 2 == 0) codes[j / 2] = pr;
      else codes[j / 2] |= pr << 16;
    }
  } else {  // a non-finite input in the group: the divide decides every code
    // (through copies, so that only this rare path hands arrays to the
    // out-of-line function and w / codes can stay in registers)
    uint32_t wt[G / 2], ct[G / 4];
#pragma unroll
    for (int j = 0; j < G / 2; ++j) wt[j] = w[j];
    codes_by_divide(wt, G, mn, scale, DT, ct);
#pragma unroll
    for (int j = 0; j < G / 4; ++j) codes[j] = ct[j];
  }
  s16 = __half_as_ushort(__float2half_rn(scale));
  z16 = __half_as_ushort(__float2half_rn(mn));
}

// Warp-cooperative staging of 32 rows of B bytes each (row r at src + r *
// stride bytes, only rows with valid[r]) into shared memory, 16-byte chunks
// XOR-swizzled by (row & 7) so that each lane can then read its own row with
// conflict-free 16-byte loads. Coalesced: one instruction covers 512
// consecutive bytes of the rows.
template <int B>
__device__ __forceinline__ void stage_rows(uint8_t* __restrict__ buf, const uint8_t* __restrict__ src,
                                           int64_t stride, uint32_t valid, int lane) {
  constexpr int CPR = B / 16;  // chunks per row
#pragma unroll 4
  for (int q = lane; q < 32 * CPR; q += 32) {
    const int r = q / CPR, c = q % CPR;
    if ((valid >> r) & 1u) {
      const uint4 x = __ldg(reinterpret_cast<const uint4*>(src + r * stride) + c);
      *reinterpret_cast<uint4*>(buf + r * B + 16 * (c ^ (r & 7))) = x;
    }
  }
}
// This lane's row (row = lane) from a staged buffer: N 32-bit words starting
// at byte offset off (a multiple of 16).
template <int B, int N>
__device__ __forceinline__ void row_words(const uint8_t* __restrict__ buf, int lane, int off,
                                          uint32_t (&w)[N]) {
#pragma unroll
  for (int i = 0; i < N / 4; ++i) {
    const int c = off / 16 + i;
    const uint4 x = *reinterpret_cast<const uint4*>(buf + lane * B + 16 * (c ^ (lane & 7)));
    w[4 * i] = x.x;
    w[4 * i + 1] = x.y;
    w[4 * i + 2] = x.z;
    w[4 * i + 3] = x.w;
  }
}

// Rotate-half RoPE of one pair of half-rows: lo holds elements [e0, e0 + n),
// hi the elements h = D/2 further; same arithmetic as quant_values (unfused
// f32 products and sum, rounded to the input dtype).
template <int N, int DT>
__device__ __forceinline__ void rope_pairs(uint32_t (&lo)[N / 2], uint32_t (&hi)[N / 2],
                                           const uint32_t (&cw)[N], const uint32_t (&sw)[N]) {
  using P = Pair<DT>;
#pragma unroll
  for (int j = 0; j < N / 2; ++j) {
    const float cx = __uint_as_float(cw[2 * j]), cy = __uint_as_float(cw[2 * j + 1]);
    const float sx = __uint_as_float(sw[2 * j]), sy = __uint_as_float(sw[2 * j + 1]);
    const typename P::T x1 = P::from(lo[j]), x2 = P::from(hi[j]);
    const float a0 = P::lo(x1), a1 = P::hi(x1), b0 = P::lo(x2), b1 = P::hi(x2);
    const float y0 = __fsub_rn(__fmul_rn(a0, cx), __fmul_rn(b0, sx));
    const float y1 = __fsub_rn(__fmul_rn(a1, cy), __fmul_rn(b1, sy));
    const float z0 = __fadd_rn(__fmul_rn(a0, sx), __fmul_rn(b0, cx));
    const float z1 = __fadd_rn(__fmul_rn(a1, sy), __fmul_rn(b1, cy));
    if constexpr (DT == 0) {
      lo[j] = P::bits(__floats2half2_rn(y0, y1));
      hi[j] = P::bits(__floats2half2_rn(z0, z1));
    } else {
      lo[j] = P::bits(__floats2bfloat162_rn(y0, y1));
      hi[j] = P::bits(__floats2bfloat162_rn(z0, z1));
    }
  }
}

// Stores one group's results for token t: K codes into the token-major row
// (16-byte chunks, odd rows swizzled for D >= 128) or V codes into column t
// of the transposed rows; scale and zero into meta arrays (a, a + 1).
template <int D, int G, bool IS_K>
__device__ __forceinline__ void store_group_row(bool mine, uint8_t* __restrict__ sb, int g, int t,
                                                const uint32_t (&codes)[G / 4], uint16_t s16,
                                                uint16_t z16) {
  constexpr int T = sub_tokens(D), NG = D / G;
  if (!mine) return;
  if constexpr (IS_K) {
#pragma unroll
    for (int ch = 0; ch < G / 16; ++ch) {
      const int d = g * G + 16 * ch;
      *reinterpret_cast<uint4*>(sb + sb_kcode(D, t, d)) =
          make_uint4(codes[4 * ch], codes[4 * ch + 1], codes[4 * ch + 2], codes[4 * ch + 3]);
    }
  } else {
    uint8_t* col = sb + sb_voff(D) + (int64_t)(g * G) * T + t;
#pragma unroll
    for (int e = 0; e < G; ++e) col[e * T] = (uint8_t)(codes[e / 4] >> (8 * (e % 4)));
  }
  uint16_t* meta = reinterpret_cast<uint16_t*>(sb + sb_meta_off(D));
  const int a = IS_K ? 0 : 2;
  meta[(a * NG + g) * T + t] = s16;
  meta[((a + 1) * NG + g) * T + t] = z16;
}

// Writes N 32-bit words back into this lane's row of a staged buffer.
template <int B, int N>
__device__ __forceinline__ void row_words_put(uint8_t* __restrict__ buf, int lane, int off,
                                              const uint32_t (&w)[N]) {
#pragma unroll
  for (int i = 0; i < N / 4; ++i) {
    const int c = off / 16 + i;
    *reinterpret_cast<uint4*>(buf + lane * B + 16 * (c ^ (lane & 7))) =
        make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
  }
}

// Rotates this lane's staged K row in place (rotate-half: element d < D/2
// with d + D/2) with the caller's cos/sin rows at the warp's 32 positions (f32
// rows of D/2 values, row of lane r at table + r * D/2), 16 elements at a
// time. Each lane reads its own position's cos/sin straight from the table
// (every head and layer of a call reads the same rows, so they are cache
// hits); lanes of tokens outside the call read nothing and rotate zeros.
template <int D, int DT>
__device__ __forceinline__ void rope_row_in_place(uint8_t* kbuf, const float* cos_rows,
                                                  const float* sin_rows, uint32_t valid, int lane) {
  constexpr int H = D / 2, B = 2 * D;
  const bool own = (valid >> lane) & 1u;
  const uint4* cr = reinterpret_cast<const uint4*>(cos_rows + (int64_t)lane * H);
  const uint4* sr = reinterpret_cast<const uint4*>(sin_rows + (int64_t)lane * H);
#pragma unroll 1
  for (int jc = 0; jc < H / 16; ++jc) {
    uint32_t cw[16], sw[16];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 z = make_uint4(0u, 0u, 0u, 0u);
      const uint4 x = own ? __ldg(cr + 4 * jc + c) : z;
      const uint4 y = own ? __ldg(sr + 4 * jc + c) : z;
      cw[4 * c] = x.x; cw[4 * c + 1] = x.y; cw[4 * c + 2] = x.z; cw[4 * c + 3] = x.w;
      sw[4 * c] = y.x; sw[4 * c + 1] = y.y; sw[4 * c + 2] = y.z; sw[4 * c + 3] = y.w;
    }
    uint32_t l8[8], h8[8];
    row_words<B, 8>(kbuf, lane, 2 * 16 * jc, l8);
    row_words<B, 8>(kbuf, lane, 2 * (H + 16 * jc), h8);
    rope_pairs<16, DT>(l8, h8, cw, sw);
    row_words_put<B, 8>(kbuf, lane, 2 * 16 * jc, l8);
    row_words_put<B, 8>(kbuf, lane, 2 * (H + 16 * jc), h8);
  }
}

// One warp per 32 consecutive tokens of a destination sub-block (T/32 warps
// per sub-block, two warps per CTA). The warp stages its K rows (and, with
// RoPE, its cos/sin rows) in shared memory with coalesced loads, then each
// lane quantizes its own token's groups; then the same for V.
template <int D, int G, int DT, bool ROPE>
__global__ void __launch_bounds__(64) append_rows_kernel(uint8_t* __restrict__ pool, Geom geom,
                                                         const AppendDst* __restrict__ dst,
                                                         int layer_begin, int n_seqs, int n_new,
                                                         int n_chunks, int64_t n_tiles,
                                                         const void* __restrict__ k,
                                                         const void* __restrict__ v,
                                                         int* __restrict__ large_scale,
                                                         RopeTable rope) {
  asm volatile("griddepcontrol.launch_dependents;");  // as in append_quantize_kernel
  constexpr int T = sub_tokens(D), NG = D / G, WPT = T / 32, H = D / 2, B = 2 * D;
  extern __shared__ __align__(16) uint8_t rows_smem[];
  const int lane = threadIdx.x & 31, wl = threadIdx.x >> 5;
  constexpr int WSMEM = 32 * B;  // shared memory per warp: its 32 staged rows
  uint8_t* kbuf = rows_smem + (size_t)wl * WSMEM;
  const int64_t wg = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t tile = wg / WPT;
  if (tile >= n_tiles) return;
  const int c = (int)(tile % n_chunks);
  const int64_t b = tile / n_chunks;
  const int h = (int)(b % geom.Hkv);
  const int64_t ls = b / geom.Hkv;  // li * n_seqs + si
  const int64_t p0 = dst[ls * n_chunks].pos;
  const int64_t cs = p0 - p0 % T + (int64_t)c * T;  // first position of the sub-block
  const int tw0 = (int)(wg % WPT) * 32;               // the warp's first token in the sub-block
  const int t = tw0 + lane;
  const int64_t pos = cs + t;
  const bool mine = pos >= p0 && pos < p0 + n_new;  // one of the call's tokens
  const uint32_t valid = __ballot_sync(0xffffffffu, mine);
  if (valid == 0u) return;
  const AppendDst d0 = dst[ls * n_chunks + c];
  const int slot0 = d0.pos & (kBlockTokens - 1);
  uint8_t* sb = pool + (((int64_t)d0.block * geom.L + (layer_begin + (int)(ls / n_seqs))) * geom.Hkv + h) *
                           geom.page_bytes +
                (int64_t)(slot0 / T) * geom.sb_bytes;
  // input rows of the warp's tokens: row of token tw0 + r at first + r * D
  const int64_t first = ((ls * geom.Hkv + h) * n_new + (cs + tw0 - p0)) * D;
  bool large = false;
  uint16_t s16, z16;
  stage_rows<B>(kbuf, reinterpret_cast<const uint8_t*>(static_cast<const uint16_t*>(k) + first), B, valid,
                lane);
  const int64_t prow = (cs + tw0) * H;  // cos/sin row of token tw0
  __syncwarp();
  // every lane runs the arithmetic (the RoPE staging inside is warp-wide);
  // only the call's tokens store
  if constexpr (ROPE)
    rope_row_in_place<D, DT>(kbuf, rope.cos + prow, rope.sin + prow, valid, lane);
#pragma unroll 1
  for (int g = 0; g < NG; ++g) {
    uint32_t w[G / 2], codes[G / 4];
    row_words<B, G / 2>(kbuf, lane, 2 * g * G, w);
    quantize_group_row<G, DT>(w, codes, s16, z16);
    store_group_row<D, G, true>(mine, sb, g, t, codes, s16, z16);
    large |= (s16 & 0x7fffu) >= 0x5400u;
  }
  __syncwarp();
  stage_rows<B>(kbuf, reinterpret_cast<const uint8_t*>(static_cast<const uint16_t*>(v) + first), B, valid,
                lane);
  __syncwarp();
  {
#pragma unroll 1
    for (int g = 0; g < NG; ++g) {
      uint32_t w[G / 2], codes[G / 4];
      row_words<B, G / 2>(kbuf, lane, 2 * g * G, w);
      quantize_group_row<G, DT>(w, codes, s16, z16);
      store_group_row<D, G, false>(mine, sb, g, t, codes, s16, z16);
      large |= (s16 & 0x7fffu) >= 0x5400u;
    }
  }
  if (mine && large) atomicOr(large_scale, 1);
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
  const int tile_threads = 32 * g.subt / 4;  // one warp per 4 tokens of a sub-block
  // Multi-token appends with the f32 quantizer: one lane per token.
  if (tiled && g.quant_variant == KRILL_QUANT_F32 && g.G <= 128) {
    const int64_t n_tiles = tiles;
    const int64_t warps_rows = n_tiles * (g.subt / 32);
    const unsigned rows_blocks = (unsigned)((warps_rows + 1) / 2);  // two warps per CTA
    const size_t rows_smem = (size_t)2 * 32 * 2 * g.D;  // two warps' staged rows
    // above 48 KB of dynamic shared memory a kernel needs the opt-in (D = 256
    // with RoPE: 96 KB); the attribute is per device, set on every such call
#define KRILL_ROWS_SMEM(DD, GG, DTT)                                                             \
    if (rows_smem > 48 * 1024) {                                                               \
      cudaError_t e = cudaFuncSetAttribute(append_rows_kernel<DD, GG, DTT, true>,              \
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,         \
                                           (int)rows_smem);                                     \
      if (e != cudaSuccess) return e;                                                          \
    }
#define KRILL_ROWS(DD, GG)                                                                     \
    if (g.D == DD && g.G == GG) {                                                              \
      if (rope.cos) {                                                                          \
        if (dtype == 0) { KRILL_ROWS_SMEM(DD, GG, 0) }                                         \
        else { KRILL_ROWS_SMEM(DD, GG, 1) }                                                    \
      }                                                                                        \
      if (dtype == 0 && rope.cos)                                                              \
        append_rows_kernel<DD, GG, 0, true><<<rows_blocks, 64, rows_smem, stream>>>(                  \
            pool, g, d_dst, layer_begin, n_seqs, n_new, n_chunks, n_tiles, k, v, large_scale, rope); \
      else if (dtype == 0)                                                                     \
        append_rows_kernel<DD, GG, 0, false><<<rows_blocks, 64, rows_smem, stream>>>(                 \
            pool, g, d_dst, layer_begin, n_seqs, n_new, n_chunks, n_tiles, k, v, large_scale, rope); \
      else if (rope.cos)                                                                       \
        append_rows_kernel<DD, GG, 1, true><<<rows_blocks, 64, rows_smem, stream>>>(                  \
            pool, g, d_dst, layer_begin, n_seqs, n_new, n_chunks, n_tiles, k, v, large_scale, rope); \
      else                                                                                     \
        append_rows_kernel<DD, GG, 1, false><<<rows_blocks, 64, rows_smem, stream>>>(                 \
            pool, g, d_dst, layer_begin, n_seqs, n_new, n_chunks, n_tiles, k, v, large_scale, rope); \
      return cudaGetLastError();                                                               \
    }
    KRILL_ROWS(64, 64)
    KRILL_ROWS(128, 64)
    KRILL_ROWS(128, 128)
    KRILL_ROWS(256, 64)
    KRILL_ROWS(256, 128)
#undef KRILL_ROWS
#undef KRILL_ROWS_SMEM
  }
#define KRILL_APPEND(E, P)                                                                    \
  if (epl == E && lpg == P) {                                                                  \
    if (tiled) {                                                                               \
      if (dtype == 0)                                                                          \
        append_tile_kernel<E, P, 0><<<(unsigned)tiles, tile_threads, 0, stream>>>(             \
            pool, g, d_dst, layer_begin, n_seqs, n_new, n_chunks, k, v, large_scale, rope);    \
      else                                                                                     \
        append_tile_kernel<E, P, 1><<<(unsigned)tiles, tile_threads, 0, stream>>>(             \
            pool, g, d_dst, layer_begin, n_seqs, n_new, n_chunks, k, v, large_scale, rope);    \
    } else if (dtype == 0) {                                                                   \
      append_quantize_kernel<E, P, 0><<<(unsigned)blocks, threads, 0, stream>>>(               \
          pool, g, d_dst, layer_begin, layer_count, n_seqs, n_new, k, v, large_scale, rope);   \
    } else {                                                                                   \
      append_quantize_kernel<E, P, 1><<<(unsigned)blocks, threads, 0, stream>>>(               \
          pool, g, d_dst, layer_begin, layer_count, n_seqs, n_new, k, v, large_scale, rope);   \
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
