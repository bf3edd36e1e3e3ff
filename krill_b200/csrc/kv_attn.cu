// kv_attn.cu — int8 decode attention, dequantize fused into q·Kᵀ and ·V.
//
// Replaces, for one query token per (layer, sequence): the full-cache
// dequantize of QuantizedKVCache.update (Sources/KrillCache/QuantizedKVCache.swift:71-74,
// dequantize :200-204) and MLXFast.scaledDotProductAttention with GQA
// (Sources/KrillCore/Gemma4Model.swift:516, Attention.swift:95). K/V are
// dequantized tile by tile with the reference's two fp16 roundings, so the
// only differences from the reference math are fp32 accumulation order and
// the fp16 rounding of the softmax weights fed to the ·V product.
//
// Structure (persistent, one CTA per SM):
//   - the host plans work items = (layer, seq, kv-head, range of 64-token
//     sub-blocks) and assigns them to CTAs by longest-processing-time;
//   - a producer warp streams each item's sub-blocks HBM -> shared memory with
//     plain bulk async copies (cp.async.bulk, one CTA each) into an NSTAGE ring
//     guarded by mbarriers;
//   - NCW consumer warps take the item's sub-blocks round-robin. Tensor-core
//     path (mma.sync m16n8k16, f16 in / f32 accumulate):
//        Sᵀ[16 tok × 8 heads] = Kdeq[16 tok × D] · Qᵀ[D × 8]   (GQA group <= 8)
//        Oᵀ[D × 8]           += Vdeqᵀ[D × 16 tok] · Pᵀ[16 tok × 8]
//     with Pᵀ obtained from the Sᵀ accumulators by movmatrix.trans, online
//     softmax in the exp2 domain;
//   - warps of one head combine in shared memory; a unit split over several
//     items writes fp32 partial records, merged by attn_combine_kernel in
//     bandwidth-bound plans and, in latency-bound plans, by the item that
//     arrives last (an epoch-tagged counter per unit and head).
//   - in a decode step the kernel may be launched as the append kernel's
//     programmatic dependent; every thread waits for that grid
//     (griddepcontrol.wait) before reading the pool.
// Every mbarrier wait is bounded; on timeout the kernel raises an error flag
// and runs to completion instead of hanging.
#include <algorithm>
#include <atomic>
#include <cstdio>

#include "kv_device.cuh"

namespace krill {
namespace {

// A consumer may reach a stage several uses ahead of the producer (its
// stages are HPR*R apart and it may skip items), and a parity wait cannot
// tell phase u+1 from phase u-1. The producer therefore tags each stage with
// the sequence number it is filling before arming the barrier; a consumer
// first waits (bounded) for its own tag, after which the parity wait is exact.
__device__ bool wait_tag(volatile uint32_t* tag, uint32_t want, volatile int* cta_abort, int* err) {
  if (*tag == want) return true;
  const uint32_t limit = wait_limit_units(cta_abort);
  const uint64_t t0 = globaltimer();
  while (*tag != want) {
    if (((globaltimer() - t0) >> 10) > limit) {
      *cta_abort = 1;
      atomicOr(err, kErrTimeout);
      return false;
    }
  }
  return true;
}

// Bounded wait for a shared-memory word to reach `want`; on timeout raises the
// error flag and returns.
__device__ __forceinline__ void wait_count(volatile uint32_t* cnt, uint32_t want, volatile int* cta_abort,
                                           int* err) {
  const uint32_t limit = wait_limit_units(cta_abort);
  const uint64_t t0 = globaltimer();
  while (*cnt < want) {
    if (((globaltimer() - t0) >> 10) > limit) {
      *cta_abort = 1;
      atomicOr(err, kErrTimeout);
      return;
    }
  }
}

__device__ __forceinline__ uint32_t movm_trans(uint32_t x) {
  uint32_t y;
  asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// True when every K and V scale of the sub-block has |s| < 64 (and is finite),
// i.e. the fast dequant is exact for the whole sub-block. Warp-uniform.
template <int D, int NG>
__device__ __forceinline__ bool scales_small(const uint8_t* __restrict__ sb, int lane) {
  using SG = SubGeom<D, NG>;
  constexpr int BYTES = NG * SG::T * 2;  // one [NG][T] f16 array
  bool big = false;
  for (int off = lane * 16; off < 2 * BYTES; off += 512) {
    const int a = off / BYTES;  // 0: K scales, 1: V scales (meta array 2)
    const uint4 w = *reinterpret_cast<const uint4*>(sb + SG::META + a * 2 * BYTES + (off - a * BYTES));
    big |= (__vcmpgeu2(w.x & 0x7fff7fffu, 0x54005400u) | __vcmpgeu2(w.y & 0x7fff7fffu, 0x54005400u) |
            __vcmpgeu2(w.z & 0x7fff7fffu, 0x54005400u) | __vcmpgeu2(w.w & 0x7fff7fffu, 0x54005400u)) != 0;
  }
  return !__any_sync(0xffffffffu, big);
}

template <int D>
struct TCState {
  float o[D / 16][4];
  float m[2], l[2];
  uint32_t qf[D / 64][8];
};


// This lane's Qᵀ fragments for one (unit, head): q[head = r][16*(tig+4hh) +
// 0..15], fetched as raw words ahead of use (fetch_q) so that the next item's
// query arrives while the current one computes, then converted (set_q).
template <int D>
struct QRaw {
  uint4 w[D / 64][2];
};

// Column r = lane / 4 of the tile (see AttnUnit::nq): query r / g, head r % g.
template <int D>
__device__ __forceinline__ void fetch_q(QRaw<D>& qr, const void* q, int64_t row_elem, int g, int cols,
                                        int64_t row_elems, int lane) {
  const int r = lane >> 2, tig = lane & 3;
  const int64_t cbase = row_elem + col_off(r, g, row_elems, D);
#pragma unroll
  for (int hh = 0; hh < D / 64; ++hh) {
    if (r < cols) {
      const int64_t e = cbase + 16 * (tig + 4 * hh);
      const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(q) + e);
      qr.w[hh][0] = __ldg(p);
      qr.w[hh][1] = __ldg(p + 1);
    } else {
      qr.w[hh][0] = make_uint4(0u, 0u, 0u, 0u);
      qr.w[hh][1] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

// st.qf from fetched words (bf16 queries become f16 for the int8 path).
template <int D, int FMT = kFmtInt8>
__device__ __forceinline__ void set_q(TCState<D>& st, const QRaw<D>& qr, int q_dtype) {
#pragma unroll
  for (int hh = 0; hh < D / 64; ++hh) {
    const uint4 a = qr.w[hh][0], b = qr.w[hh][1];
    uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (FMT == kFmtInt8 && q_dtype == 1) {  // bf16 -> f16 (exact in the f16 normal range)
        __nv_bfloat162 bv = *reinterpret_cast<__nv_bfloat162*>(&w[i]);
        float2 f = __bfloat1622float2(bv);
        w[i] = f2h2(f.x, f.y);
      }
      st.qf[hh][i] = w[i];
    }
  }
}

template <int D>
__device__ __forceinline__ void reset_state(TCState<D>& st) {
#pragma unroll
  for (int mt = 0; mt < D / 16; ++mt)
#pragma unroll
    for (int c = 0; c < 4; ++c) st.o[mt][c] = 0.f;
  st.m[0] = st.m[1] = -INFINITY;
  st.l[0] = st.l[1] = 0.f;
}

// Process one 64-token sub-block resident in shared memory at `sb` for QT
// query tiles of 8 columns (st[q]; QT = 2 for multi-query units of more than
// 8 columns): each K and V fragment is dequantized once and feeds the MMAs of
// every tile. pos0 = absolute position of its token 0; tokens outside
// [t_lo, t_hi) are masked (only checked when `boundary`), and for this lane's
// two columns 2*tig and 2*tig + 1 of tile q also those at or past th[q][0] /
// th[q][1] (<= t_hi).
template <int D, int NG, bool FAST, int QT>
__device__ __forceinline__ void tc_subblock(const uint8_t* __restrict__ sb, TCState<D> (&st)[QT],
                                            int lane, float scale_log2, bool boundary, int pos0,
                                            int t_lo, int t_hi, const int (&th)[QT][2]) {
  using SG = SubGeom<D, NG>;
  constexpr bool SWZ = D >= 128;
  const int r = lane >> 2, tig = lane & 3;
  const uint32_t selh = (r & 1) ? 0x3232u : 0x1010u;

  // ---- K phase: Sᵀ = Kdeq · Qᵀ for NU m-tiles of 16 tokens ----
  // Rows r and r + 8 of m-tile u hold tokens TPT*(r>>1) + 4u + (r&1) and that
  // plus 2: after movmatrix.trans this is exactly the token order of the V
  // fragments, where lane tig holds tokens TPT*tig + 4u + 0..3.
  constexpr int NU = SG::NU, TPT = SG::TPT;
  float s[QT][NU][4];
#pragma unroll
  for (int u = 0; u < NU; ++u) {
    const int tbase = TPT * (r >> 1) + 4 * u;
    const int ta = tbase + (r & 1);
    const int tb = ta + 2;
    float acc[QT][4];
#pragma unroll
    for (int q = 0; q < QT; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
#pragma unroll
    for (int hh = 0; hh < D / 64; ++hh) {
      const int grp = (64 * hh) / SG::G;
      const int chunk = tig + 4 * hh;
      const int phys = SWZ ? (chunk ^ ((r & 1) << 2)) : chunk;
      const uint4 wa = *reinterpret_cast<const uint4*>(sb + ta * D + phys * 16);
      const uint4 wb = *reinterpret_cast<const uint4*>(sb + tb * D + phys * 16);
      const uint2 ks4 = *reinterpret_cast<const uint2*>(sb + SG::meta(0, grp, tbase));
      const uint2 kz4 = *reinterpret_cast<const uint2*>(sb + SG::meta(1, grp, tbase));
      const uint32_t sA = __byte_perm(ks4.x, 0, selh), sB = __byte_perm(ks4.y, 0, selh);
      const uint32_t zA = __byte_perm(kz4.x, 0, selh), zB = __byte_perm(kz4.y, 0, selh);
      const uint32_t wav[4] = {wa.x, wa.y, wa.z, wa.w};
      const uint32_t wbv[4] = {wb.x, wb.y, wb.z, wb.w};
      const uint32_t nsA = neg1024(sA), nsB = neg1024(sB);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        uint32_t a0, a1, a2, a3;
        if constexpr (FAST) {
          a0 = deq2_fast(wav[k], 0x4140u, sA, nsA, zA);
          a1 = deq2_fast(wbv[k], 0x4140u, sB, nsB, zB);
          a2 = deq2_fast(wav[k], 0x4342u, sA, nsA, zA);
          a3 = deq2_fast(wbv[k], 0x4342u, sB, nsB, zB);
        } else {
          a0 = deq2(wav[k], 0x4140u, sA, zA);
          a1 = deq2(wbv[k], 0x4140u, sB, zB);
          a2 = deq2(wav[k], 0x4342u, sA, zA);
          a3 = deq2(wbv[k], 0x4342u, sB, zB);
        }
#pragma unroll
        for (int q = 0; q < QT; ++q)
          mma16816(acc[q], a0, a1, a2, a3, st[q].qf[hh][2 * k], st[q].qf[hh][2 * k + 1]);
      }
    }
#pragma unroll
    for (int q = 0; q < QT; ++q) {
#pragma unroll
      for (int c = 0; c < 4; ++c) s[q][u][c] = acc[q][c] * scale_log2;
      if (boundary) {  // fragment: [0] (ta, col 2tig), [1] (ta, 2tig+1), [2] (tb, 2tig), [3] (tb, 2tig+1)
        const int pa = pos0 + ta, pb = pos0 + tb;
        if (pa < t_lo || pa >= th[q][0]) s[q][u][0] = -INFINITY;
        if (pa < t_lo || pa >= th[q][1]) s[q][u][1] = -INFINITY;
        if (pb < t_lo || pb >= th[q][0]) s[q][u][2] = -INFINITY;
        if (pb < t_lo || pb >= th[q][1]) s[q][u][3] = -INFINITY;
      }
    }
  }

  // ---- online softmax per tile (heads 2*tig, 2*tig+1 live in this lane) ----
  uint32_t pb[QT][NU][2];
#pragma unroll
  for (int q = 0; q < QT; ++q) {
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int u = 0; u < NU; ++u) {
      mx0 = fmaxf(mx0, fmaxf(s[q][u][0], s[q][u][2]));
      mx1 = fmaxf(mx1, fmaxf(s[q][u][1], s[q][u][3]));
    }
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const float mn0 = fmaxf(st[q].m[0], mx0), mn1 = fmaxf(st[q].m[1], mx1);
    const float b0 = (mn0 == -INFINITY) ? 0.f : mn0;
    const float b1 = (mn1 == -INFINITY) ? 0.f : mn1;
    const float al0 = exp2f(st[q].m[0] - b0), al1 = exp2f(st[q].m[1] - b1);
    st[q].m[0] = mn0;
    st[q].m[1] = mn1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int u = 0; u < NU; ++u) {
      const float p0 = exp2f(s[q][u][0] - b0), p1 = exp2f(s[q][u][1] - b1);
      const float p2 = exp2f(s[q][u][2] - b0), p3 = exp2f(s[q][u][3] - b1);
      ps0 += p0 + p2;
      ps1 += p1 + p3;
      pb[q][u][0] = movm_trans(f2h2(p0, p1));
      pb[q][u][1] = movm_trans(f2h2(p2, p3));
    }
    st[q].l[0] = st[q].l[0] * al0 + ps0;
    st[q].l[1] = st[q].l[1] * al1 + ps1;
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt) {
      st[q].o[mt][0] *= al0;
      st[q].o[mt][1] *= al1;
      st[q].o[mt][2] *= al0;
      st[q].o[mt][3] *= al1;
    }
  }

  // ---- V phase: Oᵀ += Vdeqᵀ · Pᵀ ----
  const uint8_t* vt = sb + SG::VOFF;
#pragma unroll
  for (int grp = 0; grp < NG; ++grp) {
    // this lane's TPT tokens: TPT*tig .. TPT*tig + TPT - 1 (TPT/2 words of two)
    constexpr int NW = TPT / 2;
    uint32_t vs[NW], vz[NW];
#pragma unroll
    for (int c = 0; c < NW / 4; ++c) {
      const uint4 sw = *reinterpret_cast<const uint4*>(sb + SG::meta(2, grp, TPT * tig + 8 * c));
      const uint4 zw = *reinterpret_cast<const uint4*>(sb + SG::meta(3, grp, TPT * tig + 8 * c));
      vs[4 * c] = sw.x; vs[4 * c + 1] = sw.y; vs[4 * c + 2] = sw.z; vs[4 * c + 3] = sw.w;
      vz[4 * c] = zw.x; vz[4 * c + 1] = zw.y; vz[4 * c + 2] = zw.z; vz[4 * c + 3] = zw.w;
    }
    if (boundary) {
      // Invalid tokens get scale = zero = 0 so their (possibly stale) codes
      // dequantize to exactly 0 and cannot inject non-finite values.
#pragma unroll
      for (int i = 0; i < NW; ++i) {
        const int p = pos0 + TPT * tig + 2 * i;
        const uint32_t m = ((p >= t_lo && p < t_hi) ? 0x0000ffffu : 0u) |
                           ((p + 1 >= t_lo && p + 1 < t_hi) ? 0xffff0000u : 0u);
        vs[i] &= m;
        vz[i] &= m;
      }
    }
    uint32_t nvs[NW];
#pragma unroll
    for (int i = 0; i < NW; ++i) nvs[i] = FAST ? neg1024(vs[i]) : 0u;
#pragma unroll
    for (int mi = 0; mi < SG::G / 16; ++mi) {
      const int mt = grp * (SG::G / 16) + mi;
      const int d = 16 * mt + r;
      uint32_t xv[NU], yv[NU];
      if constexpr (NU == 4) {
        const uint4 x = *reinterpret_cast<const uint4*>(vt + d * SG::T + TPT * tig);
        const uint4 y = *reinterpret_cast<const uint4*>(vt + (d + 8) * SG::T + TPT * tig);
        xv[0] = x.x; xv[1] = x.y; xv[2] = x.z; xv[3] = x.w;
        yv[0] = y.x; yv[1] = y.y; yv[2] = y.z; yv[3] = y.w;
      } else {
        const uint2 x = *reinterpret_cast<const uint2*>(vt + d * SG::T + TPT * tig);
        const uint2 y = *reinterpret_cast<const uint2*>(vt + (d + 8) * SG::T + TPT * tig);
        xv[0] = x.x; xv[1] = x.y;
        yv[0] = y.x; yv[1] = y.y;
      }
#pragma unroll
      for (int u = 0; u < NU; ++u) {
        uint32_t a0, a1, a2, a3;
        if constexpr (FAST) {
          a0 = deq2_fast(xv[u], 0x4140u, vs[2 * u], nvs[2 * u], vz[2 * u]);
          a1 = deq2_fast(yv[u], 0x4140u, vs[2 * u], nvs[2 * u], vz[2 * u]);
          a2 = deq2_fast(xv[u], 0x4342u, vs[2 * u + 1], nvs[2 * u + 1], vz[2 * u + 1]);
          a3 = deq2_fast(yv[u], 0x4342u, vs[2 * u + 1], nvs[2 * u + 1], vz[2 * u + 1]);
        } else {
          a0 = deq2(xv[u], 0x4140u, vs[2 * u], vz[2 * u]);
          a1 = deq2(yv[u], 0x4140u, vs[2 * u], vz[2 * u]);
          a2 = deq2(xv[u], 0x4342u, vs[2 * u + 1], vz[2 * u + 1]);
          a3 = deq2(yv[u], 0x4342u, vs[2 * u + 1], vz[2 * u + 1]);
        }
#pragma unroll
        for (int q = 0; q < QT; ++q) mma16816(st[q].o[mt], a0, a1, a2, a3, pb[q][u][0], pb[q][u][1]);
      }
    }
  }
}


// Process one raw bf16 sub-block (the unquantized comparison format):
// Sᵀ = K·Qᵀ on bf16 tensor cores (K and q are bf16, exact products), then the
// same online softmax and Oᵀ += Vᵀ·Pᵀ in f16 with V converted exactly (V
// magnitudes beyond the f16 range are not supported). Same fragment
// permutation as tc_subblock, so q fragments and the state are shared.
template <int D>
__device__ __forceinline__ void tc_subblock_raw(const uint8_t* __restrict__ sb, TCState<D>& st,
                                                int lane, float scale_log2, bool boundary, int pos0,
                                                int t_lo, int t_hi) {
  using SG = SubGeom<D, 1, kFmtBf16>;
  constexpr int NU = SG::NU, TPT = SG::TPT;
  const int r = lane >> 2, tig = lane & 3;
  float s[NU][4];
#pragma unroll
  for (int u = 0; u < NU; ++u) {
    const int ta = TPT * (r >> 1) + 4 * u + (r & 1);
    const int tb = ta + 2;  // same parity as ta
    const int sw = ta & 1;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int hh = 0; hh < D / 64; ++hh) {
      // logical 16-byte chunks c, c+1 (d = 16 (tig + 4 hh) .. + 15) sit at
      // physical chunks c ^ sw, (c + 1) ^ sw of their row
      const int c = 2 * (tig + 4 * hh);
      const uint8_t* ra = sb + (size_t)ta * D * 2;
      const uint8_t* rb = sb + (size_t)tb * D * 2;
      const uint4 a0 = *reinterpret_cast<const uint4*>(ra + ((c ^ sw) << 4));
      const uint4 a1 = *reinterpret_cast<const uint4*>(ra + (((c + 1) ^ sw) << 4));
      const uint4 b0 = *reinterpret_cast<const uint4*>(rb + ((c ^ sw) << 4));
      const uint4 b1 = *reinterpret_cast<const uint4*>(rb + (((c + 1) ^ sw) << 4));
      const uint32_t wa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const uint32_t wb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int k = 0; k < 4; ++k)
        mma16816_bf16(acc, wa[2 * k], wb[2 * k], wa[2 * k + 1], wb[2 * k + 1], st.qf[hh][2 * k],
                      st.qf[hh][2 * k + 1]);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) s[u][c] = acc[c] * scale_log2;
    if (boundary) {
      const int pa = pos0 + ta, pb = pos0 + tb;
      if (pa < t_lo || pa >= t_hi) s[u][0] = s[u][1] = -INFINITY;
      if (pb < t_lo || pb >= t_hi) s[u][2] = s[u][3] = -INFINITY;
    }
  }
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int u = 0; u < NU; ++u) {
    mx0 = fmaxf(mx0, fmaxf(s[u][0], s[u][2]));
    mx1 = fmaxf(mx1, fmaxf(s[u][1], s[u][3]));
  }
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
  }
  const float mn0 = fmaxf(st.m[0], mx0), mn1 = fmaxf(st.m[1], mx1);
  const float b0 = (mn0 == -INFINITY) ? 0.f : mn0;
  const float b1 = (mn1 == -INFINITY) ? 0.f : mn1;
  const float al0 = exp2f(st.m[0] - b0), al1 = exp2f(st.m[1] - b1);
  st.m[0] = mn0;
  st.m[1] = mn1;
  float ps0 = 0.f, ps1 = 0.f;
  uint32_t pb[NU][2];
#pragma unroll
  for (int u = 0; u < NU; ++u) {
    const float p0 = exp2f(s[u][0] - b0), p1 = exp2f(s[u][1] - b1);
    const float p2 = exp2f(s[u][2] - b0), p3 = exp2f(s[u][3] - b1);
    ps0 += p0 + p2;
    ps1 += p1 + p3;
    pb[u][0] = movm_trans(f2h2(p0, p1));
    pb[u][1] = movm_trans(f2h2(p2, p3));
  }
  st.l[0] = st.l[0] * al0 + ps0;
  st.l[1] = st.l[1] * al1 + ps1;
#pragma unroll
  for (int mt = 0; mt < D / 16; ++mt) {
    st.o[mt][0] *= al0;
    st.o[mt][1] *= al1;
    st.o[mt][2] *= al0;
    st.o[mt][3] *= al1;
  }
  // ---- V: rows d and d + 8, this lane's tokens TPT*tig .. +TPT-1 ----
  const uint8_t* vt = sb + SG::VOFF;
  constexpr int NW = TPT / 2;  // bf16 pairs per row
  uint32_t vmask[NW];
#pragma unroll
  for (int i = 0; i < NW; ++i) {
    // invalid tokens read as zero so stale contents cannot inject non-finite values
    const int pp = pos0 + TPT * tig + 2 * i;
    vmask[i] = !boundary ? 0xffffffffu
                         : (((pp >= t_lo && pp < t_hi) ? 0x0000ffffu : 0u) |
                            ((pp + 1 >= t_lo && pp + 1 < t_hi) ? 0xffff0000u : 0u));
  }
#pragma unroll
  for (int mt = 0; mt < D / 16; ++mt) {
    const int d = 16 * mt + r;
    uint32_t xv[NW], yv[NW];
#pragma unroll
    for (int q4 = 0; q4 < NW / 4; ++q4) {
      const uint4 x = *reinterpret_cast<const uint4*>(vt + ((size_t)d * SG::T + TPT * tig) * 2 + 16 * q4);
      const uint4 y = *reinterpret_cast<const uint4*>(vt + ((size_t)(d + 8) * SG::T + TPT * tig) * 2 + 16 * q4);
      xv[4 * q4] = x.x; xv[4 * q4 + 1] = x.y; xv[4 * q4 + 2] = x.z; xv[4 * q4 + 3] = x.w;
      yv[4 * q4] = y.x; yv[4 * q4 + 1] = y.y; yv[4 * q4 + 2] = y.z; yv[4 * q4 + 3] = y.w;
    }
#pragma unroll
    for (int u = 0; u < NU; ++u) {
      const uint32_t a0 = bf2h2(xv[2 * u] & vmask[2 * u]);
      const uint32_t a1 = bf2h2(yv[2 * u] & vmask[2 * u]);
      const uint32_t a2 = bf2h2(xv[2 * u + 1] & vmask[2 * u + 1]);
      const uint32_t a3 = bf2h2(yv[2 * u + 1] & vmask[2 * u + 1]);
      mma16816(st.o[mt], a0, a1, a2, a3, pb[u][0], pb[u][1]);
    }
  }
}

template <int D, int NG, int NCW, int R, int NSTAGE, int FMT = kFmtInt8>
struct AttnSmem {
  static constexpr int SB = SubGeom<D, NG, FMT>::SB;
  static constexpr int STAGE_BYTES = NSTAGE * SB;
  static constexpr int BAR_OFF = STAGE_BYTES;                 // 2*NSTAGE u64
  static constexpr int NV = D / 16 * 4 + 4;                   // per-lane state floats
  static constexpr int CB_OFF = BAR_OFF + 2 * NSTAGE * 8;     // [NCW - NCW/R][NV][32] f32
  static constexpr int CB_BYTES = R > 1 ? (NCW - NCW / R) * NV * 32 * 4 : 0;
  static constexpr int TAG_OFF = CB_OFF + CB_BYTES;           // [NSTAGE] u32 stage tags
  static constexpr int MISC_OFF = TAG_OFF + ((NSTAGE * 4 + 15) / 16) * 16;  // abort flag
  static constexpr int TOTAL = MISC_OFF + 16;
};

// Number of 64-token stages that fit next to the rest of the shared memory.
template <int D, int NG, int NCW, int R, int FMT = kFmtInt8>
constexpr int stages_for() {
  constexpr int fixed = AttnSmem<D, NG, NCW, R, 0, FMT>::TOTAL;
  constexpr int n = (232448 - fixed - 2 * 16 * 8) / SubGeom<D, NG, FMT>::SB;
  return n > 16 ? 16 : n;
}

// Merge a split unit's n_split partial records for kv head h into the output,
// in one warp: the piece that finished last does this in place of a combine
// kernel. The arithmetic and its order are those of attn_combine_kernel
// (max, then the weighted sums in record order), so both give the same bits.
// Records written by other CTAs are read through L2 (ld.global.cg).
template <int D>
__device__ __forceinline__ void merge_split(const AttnParams& p, const AttnUnit& un, int h, int lane) {
  const int g = p.g, n = un.n_split, cols = unit_cols(un, g);
  const int64_t row_elems = (int64_t)p.Hq * D;
  const int64_t stride = (int64_t)p.Hkv * partial_floats(D);
  const float* base = p.partials + ((int64_t)un.first_split * p.Hkv + h) * partial_floats(D);
  // lane j < g: max and normalizer of query head j
  float M = -INFINITY, Ls = 0.f;
  if (lane < cols) {
#pragma unroll 8
    for (int i = 0; i < n; ++i) M = fmaxf(M, __ldcg(base + i * stride + lane));
#pragma unroll 8
    for (int i = 0; i < n; ++i) {
      const float mi = __ldcg(base + i * stride + lane);
      Ls += (mi == -INFINITY) ? 0.f : __ldcg(base + i * stride + 8 + lane) * exp2f(mi - M);
    }
  }
  const float inv = 1.f / Ls;
  constexpr int NC = D / 32;  // output dims per lane and query head
  float acc[8][NC];
#pragma unroll
  for (int hq = 0; hq < 8; ++hq)
#pragma unroll
    for (int c = 0; c < NC; ++c) acc[hq][c] = 0.f;
#pragma unroll 2
  for (int i = 0; i < n; ++i) {
    const float* ri = base + i * stride;
    const float mj = lane < cols ? __ldcg(ri + lane) : -INFINITY;
    const float wj = (mj == -INFINITY) ? 0.f : exp2f(mj - M);
#pragma unroll
    for (int hq = 0; hq < 8; ++hq) {
      if (hq < cols) {
        const float mh = __shfl_sync(0xffffffffu, mj, hq);
        const float wh = __shfl_sync(0xffffffffu, wj, hq);
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          const float o = __ldcg(ri + 16 + hq * D + lane + 32 * c);
          acc[hq][c] = (mh == -INFINITY) ? acc[hq][c] : acc[hq][c] + o * wh;
        }
      }
    }
  }
  const int64_t orow = ((int64_t)un.qo_row * p.Hq + (int64_t)h * g) * D;
#pragma unroll
  for (int hq = 0; hq < 8; ++hq) {
    if (hq < cols) {
      const float ih = __shfl_sync(0xffffffffu, inv, hq);
#pragma unroll
      for (int c = 0; c < NC; ++c)
        store_out(p.out, p.out_dtype, orow + col_off(hq, g, row_elems, D) + lane + 32 * c, acc[hq][c] * ih);
    }
  }
}

// Count this piece's arrival at (unit, head h); true for the piece that
// completes the unit (n_split - n_pre decode pieces; the n_pre prefix records
// were finished by an earlier kernel). Called by the whole warp after its
// partial record is stored.
__device__ __forceinline__ bool arrive_split(const AttnParams& p, const AttnUnit& un, int h, int lane) {
  __threadfence();  // this lane's record stores, device-wide, before the count
  __syncwarp();
  int last = 0;
  if (lane == 0) {
    unsigned long long* c = p.split_ctr + (int64_t)un.first_split * p.Hkv + h;
    const unsigned long long need = (unsigned long long)(un.n_split - un.n_pre);
    unsigned long long old = *reinterpret_cast<volatile unsigned long long*>(c);
    int tries = 0;
    for (; tries < (1 << 16); ++tries) {
      const unsigned long long cnt = (old >> 32) == p.epoch ? (old & 0xffffffffull) : 0ull;
      const unsigned long long got = atomicCAS(c, old, ((unsigned long long)p.epoch << 32) | (cnt + 1));
      if (got == old) {
        last = cnt + 1 == need;
        break;
      }
      old = got;
    }
    if (tries == (1 << 16)) atomicOr(p.err, kErrTimeout);
    if (last) __threadfence();  // the other pieces' records, before reading them
  }
  return __shfl_sync(0xffffffffu, last, 0) != 0;
}

// Finish one (item, head) in the warp that holds the merged state: write the
// normalized output, or a partial record plus, for the piece that arrives
// last, the merge of the unit's records.
template <int D>
__device__ __forceinline__ void finish_head(const AttnParams& p, TCState<D>& st, float l0,
                                            float l1, const AttnUnit& un, const AttnItem& item,
                                            int h, int lane) {
  const int r = lane >> 2, tig = lane & 3;
  const int g = p.g;
  const int Hkv = p.Hkv;
  const int64_t orow = ((int64_t)un.qo_row * p.Hq + (int64_t)h * g) * D;
  const int h0 = 2 * tig, h1 = 2 * tig + 1;
  const int cols = unit_cols(un, g);
  if (un.n_split == 1) {
    if (un.n_pre > 0) {
      // merge the shared-prefix records the cascade kernel completed earlier
      // in the stream (heads beyond the GQA group hold no data and are unused)
      // (loops unrolled and the O loads unconditional, so that the loads of
      // a record, and of two records, are in flight together)
      const float* rec = p.partials + ((int64_t)un.first_split * Hkv + h) * partial_floats(D);
      const int64_t stride = (int64_t)Hkv * partial_floats(D);
      const int n_pre = un.n_pre;
      float M0 = st.m[0], M1 = st.m[1];
#pragma unroll 4
      for (int i = 0; i < n_pre; ++i) {
        M0 = fmaxf(M0, rec[i * stride + (h0 & 7)]);
        M1 = fmaxf(M1, rec[i * stride + (h1 & 7)]);
      }
      const float a0 = st.m[0] == -INFINITY ? 0.f : exp2f(st.m[0] - M0);
      const float a1 = st.m[1] == -INFINITY ? 0.f : exp2f(st.m[1] - M1);
      l0 *= a0;
      l1 *= a1;
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt) {
        st.o[mt][0] *= a0;
        st.o[mt][1] *= a1;
        st.o[mt][2] *= a0;
        st.o[mt][3] *= a1;
      }
      // Records of heads h0, h1 >= g are never written: their words are read
      // (the buffer spans all 8 head slots) but always discarded by the
      // selects, as are the words of empty records (b == 0).
#pragma unroll 2
      for (int i = 0; i < n_pre; ++i) {
        const float* ri = rec + i * stride;
        const float m0 = ri[h0 & 7], m1 = ri[h1 & 7];
        const float lv0 = ri[8 + (h0 & 7)], lv1 = ri[8 + (h1 & 7)];
        float ov[D / 16][4];
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt) {
          ov[mt][0] = ri[16 + (h0 & 7) * D + 16 * mt + r];
          ov[mt][2] = ri[16 + (h0 & 7) * D + 16 * mt + r + 8];
          ov[mt][1] = ri[16 + (h1 & 7) * D + 16 * mt + r];
          ov[mt][3] = ri[16 + (h1 & 7) * D + 16 * mt + r + 8];
        }
        const float b0 = m0 == -INFINITY ? 0.f : exp2f(m0 - M0);
        const float b1 = m1 == -INFINITY ? 0.f : exp2f(m1 - M1);
        const bool t0 = b0 != 0.f && h0 < cols, t1 = b1 != 0.f && h1 < cols;
        l0 = t0 ? l0 + lv0 * b0 : l0;
        l1 = t1 ? l1 + lv1 * b1 : l1;
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt) {
          st.o[mt][0] = t0 ? st.o[mt][0] + ov[mt][0] * b0 : st.o[mt][0];
          st.o[mt][2] = t0 ? st.o[mt][2] + ov[mt][2] * b0 : st.o[mt][2];
          st.o[mt][1] = t1 ? st.o[mt][1] + ov[mt][1] * b1 : st.o[mt][1];
          st.o[mt][3] = t1 ? st.o[mt][3] + ov[mt][3] * b1 : st.o[mt][3];
        }
      }
    }
    const float i0 = 1.f / l0, i1 = 1.f / l1;
    const int64_t row_elems = (int64_t)p.Hq * D;
    const int64_t o0 = orow + col_off(h0, g, row_elems, D), o1 = orow + col_off(h1, g, row_elems, D);
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt) {
      const int d = 16 * mt + r;
      if (h0 < cols) {
        store_out(p.out, p.out_dtype, o0 + d, st.o[mt][0] * i0);
        store_out(p.out, p.out_dtype, o0 + d + 8, st.o[mt][2] * i0);
      }
      if (h1 < cols) {
        store_out(p.out, p.out_dtype, o1 + d, st.o[mt][1] * i1);
        store_out(p.out, p.out_dtype, o1 + d + 8, st.o[mt][3] * i1);
      }
    }
    return;
  }
  const int64_t rec = ((int64_t)un.first_split + item.idx) * Hkv + h;
  float* part = p.partials + rec * partial_floats(D);
#pragma unroll
  for (int mt = 0; mt < D / 16; ++mt) {
    const int d = 16 * mt + r;
    part[16 + h0 * D + d] = st.o[mt][0];
    part[16 + h0 * D + d + 8] = st.o[mt][2];
    part[16 + h1 * D + d] = st.o[mt][1];
    part[16 + h1 * D + d + 8] = st.o[mt][3];
  }
  if (r == 0) {
    part[h0] = st.m[0];
    part[h1] = st.m[1];
    part[8 + h0] = l0;
    part[8 + h1] = l1;
  }
  if (p.split_ctr != nullptr && arrive_split(p, un, h, lane)) merge_split<D>(p, un, h, lane);
}

// Merge the partial records of split units: one CTA per (split unit, kv head).
template <int D>
__global__ void __launch_bounds__(128) attn_combine_kernel(AttnParams p) {
  const int Hkv = p.Hkv, g = p.g;
  const int u = p.split_units[blockIdx.x / Hkv];
  const int h = blockIdx.x % Hkv;
  const AttnUnit un = p.units[u];
  const float* base = p.partials + ((int64_t)un.first_split * Hkv + h) * partial_floats(D);
  const int64_t stride = (int64_t)Hkv * partial_floats(D);
  // (loops unrolled so that several records' loads are in flight; the sums
  // keep record order)
  const int cols = unit_cols(un, g);
  const int64_t row_elems = (int64_t)p.Hq * D;
  __shared__ float sm[8], sinv[8];
  if (threadIdx.x < cols) {
    const int hq = threadIdx.x;
    float M = -INFINITY;
#pragma unroll 8
    for (int i = 0; i < un.n_split; ++i) M = fmaxf(M, base[i * stride + hq]);
    float Ls = 0.f;
#pragma unroll 8
    for (int i = 0; i < un.n_split; ++i) {
      const float mi = base[i * stride + hq];
      const float li = base[i * stride + 8 + hq];
      Ls += (mi == -INFINITY) ? 0.f : li * exp2f(mi - M);
    }
    sm[hq] = M;
    sinv[hq] = 1.f / Ls;
  }
  __syncthreads();
  const int64_t orow = ((int64_t)un.qo_row * p.Hq + (int64_t)h * g) * D;
  for (int idx = threadIdx.x; idx < cols * D; idx += blockDim.x) {
    const int hq = idx / D, d = idx - hq * D;
    const float M = sm[hq];
    float Os = 0.f;
#pragma unroll 4
    for (int i = 0; i < un.n_split; ++i) {
      const float mi = base[i * stride + hq];
      const float oi = base[i * stride + 16 + hq * D + d];
      Os = (mi != -INFINITY) ? Os + oi * exp2f(mi - M) : Os;
    }
    store_out(p.out, p.out_dtype, orow + col_off(hq, g, row_elems, D) + d, Os * sinv[hq]);
  }
}

// Work split inside a CTA: an item covers hg kv heads; HPR = NCW / R of them
// are processed at once, each by R warps (R = 1 when hg >= NCW), in hg / HPR
// rounds. For an item of n_sb sub-blocks the
// producer issues, per round, sub-block k of head hr as stage J0 + k*HPR + hr;
// warp (hr, r) takes the sub-blocks k = r, r + R, ...
// Threads: NCW consumer warps (two warpgroups) + one producer warpgroup, of
// which one warp issues the copies. At start the producer warpgroup gives its
// registers back (setmaxnreg.dec to 56) and the consumers take them
// (setmaxnreg.inc to 224): 128*56 + 256*224 = 384*168, the launch budget.
// (With 40 the producer's metadata prefetch spilled; 224 still holds every
// consumer without spills.)
constexpr int kProducerRegs = 56;
constexpr int kConsumerRegs = 224;

// Consumer warps of attn_tc_kernel. FAST selects the one-fma dequantization,
// exact only while every scale in the pool is below 64 in magnitude; the
// kernel picks one specialization per launch from the pool's large-scale flag
// (set by the kernels that store scales), so the hot loop carries one path.
// QT = 2: every unit of the launch is the first 8 columns of a multi-query
// unit whose other columns are the next unit (AttnUnit::nq; its shadow, with
// the same sequence, layer and pieces, but its own queries, bounds and
// records); both tiles are computed from each staged sub-block.
template <int D, int NG, int NCW, int R, int NSTAGE, int FMT, bool FAST, int QT>
__device__ __forceinline__ void attn_consume(const AttnParams& p, uint8_t* smem, uint8_t* stages,
                                             uint32_t bar_base, volatile int* cta_abort,
                                             volatile uint32_t* tags, int warp, int lane, int it0,
                                             int it1, int rounds) {
  using SM = AttnSmem<D, NG, NCW, R, NSTAGE, FMT>;
  constexpr int SB = SM::SB;
  constexpr int HPR = NCW / R;
  static_assert(QT == 1 || (R == 1 && FMT == kFmtInt8), "two query tiles: one warp per head, int8");
  const int hr = warp / R, rr = warp % R;
  TCState<D> sts[QT];
  TCState<D>& st = sts[0];
  uint32_t J = 0;
  AttnItem item_next{};
  AttnUnit un_next{};
  // The query of the next (item, round) is fetched while this one computes:
  // the next item's unit after this warp's first sub-block (the item record
  // has arrived by then), its q words after the second, so neither load
  // stalls the warp. qr always holds the q of the (item, round) about to run.
  QRaw<D> qr;
  auto q_row = [&](const AttnUnit& u, int hh) {
    return ((int64_t)u.qo_row * p.Hq + (int64_t)hh * p.g) * D;
  };
  const int64_t q_row_elems = (int64_t)p.Hq * D;
  // query index (within a multi-query unit) of this lane's two columns
  const int col_q0 = D <= 128 ? (2 * (lane & 3)) / p.g : 0;
  const int col_q1 = D <= 128 ? (2 * (lane & 3) + 1) / p.g : 0;
  if (it0 < it1) {
    item_next = p.items[it0];
    un_next = p.units[item_next.unit];
    if constexpr (QT == 1)
      fetch_q<D>(qr, p.q, q_row(un_next, item_next.h0 + hr), p.g, unit_cols(un_next, p.g),
                 q_row_elems, lane);
  }
  for (int it = it0; it < it1; ++it) {
    const AttnItem item = item_next;
    const AttnUnit un = un_next;
    if (it + 1 < it1) item_next = p.items[it + 1];
    const int n_sb = item.sb_end - item.sb_begin;
    for (int rd = 0; rd < rounds; ++rd) {
      const int h = item.h0 + rd * HPR + hr;
      // with two tiles both queries are fetched here (no prefetch across the
      // item, whose registers the second tile needs); items are long
      if constexpr (QT == 2)
        fetch_q<D>(qr, p.q, q_row(un, h), p.g, unit_cols(un, p.g), q_row_elems, lane);
      reset_state(st);
      set_q<D, FMT>(st, qr, p.q_dtype);
      // the shadow unit's queries (second tile), fetched here: items are long
      // (the shadow record is read again at the finish, not kept in registers)
      AttnUnit un2 = un;
      if constexpr (QT == 2) {
        un2 = p.units[item.unit + 1];
        QRaw<D> qr2;
        fetch_q<D>(qr2, p.q, q_row(un2, h), p.g, unit_cols(un2, p.g), q_row_elems, lane);
        reset_state(sts[1]);
        set_q<D, FMT>(sts[1], qr2, p.q_dtype);
      }
      // prefetch state: 0 nothing yet, 1 next unit requested, 2 next q fetched
      int pf = 0;
      auto prefetch_step = [&]() {
        if (rd + 1 < rounds) {  // next round: same unit, the next head group
          if constexpr (QT == 1)
            fetch_q<D>(qr, p.q, q_row(un, h + HPR), p.g, unit_cols(un, p.g), q_row_elems, lane);
          pf = 2;
        } else if (it + 1 >= it1) {
          pf = 2;
        } else if (pf == 0) {
          un_next = p.units[item_next.unit];
          pf = 1;
        } else {
          if constexpr (QT == 1)
            fetch_q<D>(qr, p.q, q_row(un_next, item_next.h0 + hr), p.g, unit_cols(un_next, p.g),
                       q_row_elems, lane);
          pf = 2;
        }
      };
      // per-column bounds of a multi-query unit (AttnUnit::nq); the tiles'
      // union of positions is [t_lo, t_hi), the first column's bound b_min
      int th[QT][2];
      int b_min = INT32_MAX, t_hi = 0;
#pragma unroll
      for (int q = 0; q < QT; ++q) {
        const AttnUnit& uq = q == 0 ? un : un2;
        const int nq1 = uq.nq > 1 ? uq.nq - 1 : 0;  // column c: t_hi - (nq - 1 - c / g)
        if constexpr (D <= 128) {  // per-lane quotients computed once per launch
          th[q][0] = uq.t_hi - (nq1 - min(col_q0, nq1));
          th[q][1] = uq.t_hi - (nq1 - min(col_q1, nq1));
        } else {  // (at head_dim 256 two more live registers cost spills)
          th[q][0] = uq.t_hi - (nq1 - (2 * (lane & 3)) / p.g);
          th[q][1] = uq.t_hi - (nq1 - (2 * (lane & 3) + 1) / p.g);
        }
        b_min = min(b_min, uq.t_hi - nq1);
        t_hi = max(t_hi, uq.t_hi);
      }
      for (int k = rr; k < n_sb; k += R) {
        const uint32_t jj = J + (uint32_t)k * HPR + hr;
        const uint32_t stage = jj % NSTAGE;
        wait_tag(tags + stage, jj, cta_abort, p.err);
        mbar_wait(bar_base + 8 * stage, (jj / NSTAGE) & 1, cta_abort, p.err);
        const int j = item.sb_begin + k;
        constexpr int T = SubGeom<D, NG, FMT>::T;
        const int pos0 = j * T;
        const bool boundary = pos0 < un.t_lo || pos0 + T > b_min;
        const uint8_t* sbp = stages + (size_t)stage * SB;
        if constexpr (FMT == kFmtBf16)
          tc_subblock_raw<D>(sbp, st, lane, p.scale_log2, boundary, pos0, un.t_lo, un.t_hi);
        else
          tc_subblock<D, NG, FAST, QT>(sbp, sts, lane, p.scale_log2, boundary, pos0, un.t_lo, t_hi, th);
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_base + 8 * (NSTAGE + stage));
        if (pf < 2) prefetch_step();
      }
      while (pf < 2) prefetch_step();
      J += (uint32_t)n_sb * HPR;

      float l0 = st.l[0], l1 = st.l[1];
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, off);
        l1 += __shfl_xor_sync(0xffffffffu, l1, off);
      }
      if constexpr (R > 1) {
        // merge the R warps of this head through a lane-major buffer
        float* cb = reinterpret_cast<float*>(smem + SM::CB_OFF);
        const int nbar = 1 + hr;
        asm volatile("bar.sync %0, %1;" ::"r"(nbar), "r"(R * 32) : "memory");  // buffer free
        if (rr != 0) {
          float* mine = cb + (size_t)(hr * (R - 1) + rr - 1) * SM::NV * 32;
#pragma unroll
          for (int mt = 0; mt < D / 16; ++mt)
#pragma unroll
            for (int c = 0; c < 4; ++c) mine[(mt * 4 + c) * 32 + lane] = st.o[mt][c];
          mine[(D / 4 + 0) * 32 + lane] = st.m[0];
          mine[(D / 4 + 1) * 32 + lane] = st.m[1];
          mine[(D / 4 + 2) * 32 + lane] = l0;
          mine[(D / 4 + 3) * 32 + lane] = l1;
        }
        asm volatile("bar.sync %0, %1;" ::"r"(nbar), "r"(R * 32) : "memory");
        if (rr == 0) {
#pragma unroll
          for (int w = 1; w < R; ++w) {
            const float* o = cb + (size_t)(hr * (R - 1) + w - 1) * SM::NV * 32;
            const float m0 = o[(D / 4 + 0) * 32 + lane], m1 = o[(D / 4 + 1) * 32 + lane];
            const float M0 = fmaxf(st.m[0], m0), M1 = fmaxf(st.m[1], m1);
            const float a0 = (st.m[0] == -INFINITY) ? 0.f : exp2f(st.m[0] - M0);
            const float a1 = (st.m[1] == -INFINITY) ? 0.f : exp2f(st.m[1] - M1);
            const float b0 = (m0 == -INFINITY) ? 0.f : exp2f(m0 - M0);
            const float b1 = (m1 == -INFINITY) ? 0.f : exp2f(m1 - M1);
            l0 = l0 * a0 + o[(D / 4 + 2) * 32 + lane] * b0;
            l1 = l1 * a1 + o[(D / 4 + 3) * 32 + lane] * b1;
#pragma unroll
            for (int mt = 0; mt < D / 16; ++mt) {
              st.o[mt][0] = st.o[mt][0] * a0 + o[(mt * 4 + 0) * 32 + lane] * b0;
              st.o[mt][1] = st.o[mt][1] * a1 + o[(mt * 4 + 1) * 32 + lane] * b1;
              st.o[mt][2] = st.o[mt][2] * a0 + o[(mt * 4 + 2) * 32 + lane] * b0;
              st.o[mt][3] = st.o[mt][3] * a1 + o[(mt * 4 + 3) * 32 + lane] * b1;
            }
            st.m[0] = M0;
            st.m[1] = M1;
          }
        }
      }
      if (rr == 0) finish_head<D>(p, st, l0, l1, un, item, h, lane);
      if constexpr (QT == 2) {
        float m0 = sts[1].l[0], m1 = sts[1].l[1];
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          m0 += __shfl_xor_sync(0xffffffffu, m0, off);
          m1 += __shfl_xor_sync(0xffffffffu, m1, off);
        }
        finish_head<D>(p, sts[1], m0, m1, p.units[item.unit + 1], item, h, lane);
      }
    }
  }
}

template <int D, int NG, int NCW, int R, int NSTAGE, int FMT, int QT = 1>
__global__ void __launch_bounds__((NCW + 4) * 32, 1) attn_tc_kernel(AttnParams p) {
  static_assert(NCW == 8, "two consumer warpgroups");
  using SM = AttnSmem<D, NG, NCW, R, NSTAGE, FMT>;
  constexpr int SB = SM::SB;
  constexpr int HPR = NCW / R;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* stages = smem;
  const uint32_t bar_base = smem_u32(smem + SM::BAR_OFF);
  volatile int* cta_abort = reinterpret_cast<volatile int*>(smem + SM::MISC_OFF);
  volatile uint32_t* tags = reinterpret_cast<volatile uint32_t*>(smem + SM::TAG_OFF);
  volatile uint32_t* stall_word = reinterpret_cast<volatile uint32_t*>(smem + SM::MISC_OFF + 8);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(bar_base + 8 * s, 1);             // full: producer arrive + tx
      mbar_init(bar_base + 8 * (NSTAGE + s), 1);  // empty: the consuming warp
    }
    for (int s = 0; s < NSTAGE; ++s) tags[s] = 0xffffffffu;
    init_wait_state(cta_abort, p.wait_us);
    *stall_word = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // Launched as the programmatic dependent of a decode step's append (see
  // launch_tc), this grid may start while the append runs: wait for it to
  // complete before reading the pool or the large-scale flag it writes.
  // Without that launch attribute this returns at once.
  asm volatile("griddepcontrol.wait;" ::: "memory");

  const int it0 = p.cta_off[blockIdx.x], it1 = p.cta_off[blockIdx.x + 1];
  const int Hkv = p.Hkv;
  const int rounds = p.hg / HPR;

  if (warp >= NCW) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProducerRegs));
    // Testing only (the pool's kDevTestStall word): an otherwise idle warp of
    // CTA 0 waits for a word that nothing raises, so that its bounded wait
    // runs out (error flag set; the launch still ends, its outputs not valid).
    if (warp == NCW + 1 && blockIdx.x == 0 && lane == 0 &&
        reinterpret_cast<volatile const int*>(p.err)[kDevTestStall] != 0)
      wait_count(stall_word, 1u, cta_abort, p.err);
    if (warp != NCW) return;
    // ---------------- producer ----------------
    // The lanes fetch an item's block ids together (one coalesced load per 32
    // blocks); lane 0 issues the bulk copies with no dependent global load in
    // the issue loop.
    // The next item's record, unit and first 32 block ids are fetched while
    // this item's copies are issued (one step per issued sub-block), so that
    // the chain item -> unit -> block table never idles the copy engine
    // between items.
    const int64_t blk_stride = (int64_t)p.L * Hkv * p.page_bytes;
    constexpr int SPB = SubGeom<D, NG, FMT>::SPB;
    auto first_blocks = [&](const AttnItem& itm, const AttnUnit& u) {
      const int b0 = itm.sb_begin / SPB;
      const int nblk = (itm.sb_end - 1) / SPB - b0 + 1;
      int bi = b0 + lane;
      if (p.ring > 0) bi %= p.ring;
      return lane < nblk ? p.bt[(int64_t)u.si * p.bt_stride + bi] : 0;
    };
    AttnItem item_n{};
    AttnUnit un_n{};
    int blk_n = 0;
    if (it0 < it1) {
      item_n = p.items[it0];
      un_n = p.units[item_n.unit];
      blk_n = first_blocks(item_n, un_n);
    }
    uint32_t J = 0;
    for (int it = it0; it < it1; ++it) {
      const AttnItem item = item_n;
      const AttnUnit un = un_n;
      const int blk_first = blk_n;
      const bool more = it + 1 < it1;
      if (more) item_n = p.items[it + 1];
      int pf = more ? 0 : 2;  // 0: next record requested, 1: its unit, 2: its block ids
      auto prefetch_step = [&]() {
        if (pf == 0) {
          un_n = p.units[item_n.unit];
          pf = 1;
        } else if (pf == 1) {
          blk_n = first_blocks(item_n, un_n);
          pf = 2;
        }
      };
      const int32_t* bt = p.bt + (int64_t)un.si * p.bt_stride;
      const int n_sb = item.sb_end - item.sb_begin;
      const int b0 = item.sb_begin / SPB;
      const int nblk = (item.sb_end - 1) / SPB - b0 + 1;
      for (int rd = 0; rd < rounds; ++rd) {
        const uint8_t* layer_base =
            p.pool + ((int64_t)un.layer * Hkv + item.h0 + rd * HPR) * p.page_bytes;
        for (int c0 = 0; c0 < nblk; c0 += 32) {
          int bi = b0 + c0 + lane;
          if (p.ring > 0) bi %= p.ring;
          const int blk = c0 == 0 ? blk_first : (c0 + lane < nblk) ? bt[bi] : 0;
          const int jlo = max(item.sb_begin, (b0 + c0) * SPB);
          const int jhi = min(item.sb_end, (b0 + c0 + 32) * SPB);
          for (int j = jlo; j < jhi; ++j) {
            const int b = __shfl_sync(0xffffffffu, blk, j / SPB - b0 - c0);
            if (lane == 0) {
              const uint8_t* sb_src = layer_base + (int64_t)b * blk_stride + (int64_t)(j % SPB) * SB;
              for (int hr = 0; hr < HPR; ++hr) {
                const uint32_t Jh = J + (uint32_t)(j - item.sb_begin) * HPR + hr;
                const uint32_t stage = Jh % NSTAGE;
                if (Jh >= (uint32_t)NSTAGE)
                  mbar_wait(bar_base + 8 * (NSTAGE + stage), ((Jh / NSTAGE) - 1) & 1, cta_abort,
                            p.err);
                const uint32_t full = bar_base + 8 * stage;
                tags[stage] = Jh;  // released by the arrive below
                mbar_expect_tx(full, SB);
                bulk_g2s(smem_u32(stages + (size_t)stage * SB), sb_src + (int64_t)hr * p.page_bytes,
                         SB, full);
              }
            }
            if (pf < 2) prefetch_step();
          }
        }
        J += (uint32_t)n_sb * HPR;
      }
      while (pf < 2) prefetch_step();
    }
    return;
  }

  // ---------------- consumers ----------------
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kConsumerRegs));
  if (FMT == kFmtInt8 && *reinterpret_cast<volatile const int*>(p.large_scale) != 0)
    attn_consume<D, NG, NCW, R, NSTAGE, FMT, false, QT>(p, smem, stages, bar_base, cta_abort, tags, warp,
                                                    lane, it0, it1, rounds);
  else
    attn_consume<D, NG, NCW, R, NSTAGE, FMT, true, QT>(p, smem, stages, bar_base, cta_abort, tags, warp,
                                                   lane, it0, it1, rounds);
}

template <int D, int NG, int NCW, int R, int FMT, int QT = 1>
cudaError_t launch_tc(const AttnParams& p, int grid, cudaStream_t stream) {
  constexpr int NSTAGE = stages_for<D, NG, NCW, R, FMT>();
  using SM = AttnSmem<D, NG, NCW, R, NSTAGE, FMT>;
  static_assert(NSTAGE >= 4, "too few stages");
  static_assert(SM::TOTAL <= 232448, "shared memory budget");
  // the shared-memory opt-in is a per-device attribute: set it once per device
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    // setmaxnreg.inc waits until the producer's released registers cover it:
    // refuse to launch a build whose register count would not balance
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, attn_tc_kernel<D, NG, NCW, R, NSTAGE, FMT, QT>);
    if (e != cudaSuccess) return e;
    if (fa.numRegs * (NCW + 4) * 32 < 128 * kProducerRegs + NCW * 32 * kConsumerRegs)
      return cudaErrorInvalidConfiguration;
    e = cudaFuncSetAttribute(attn_tc_kernel<D, NG, NCW, R, NSTAGE, FMT, QT>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, SM::TOTAL);
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit);
  }
  if (p.pdl) {
    // programmatic dependent of the append launched just before it
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3((NCW + 4) * 32);
    cfg.dynamicSmemBytes = SM::TOTAL;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, attn_tc_kernel<D, NG, NCW, R, NSTAGE, FMT, QT>, p);
  }
  attn_tc_kernel<D, NG, NCW, R, NSTAGE, FMT, QT><<<grid, (NCW + 4) * 32, SM::TOTAL, stream>>>(p);
  return cudaGetLastError();
}

template <int D, int NG, int NCW, int FMT = kFmtInt8>
cudaError_t launch_tc_r(const AttnParams& p, int grid, cudaStream_t stream) {
  const int hpr = p.hg < NCW ? p.hg : NCW;
  if (NCW % hpr != 0 || p.hg % hpr != 0) return cudaErrorInvalidValue;
  cudaError_t e = cudaErrorInvalidValue;
  if (p.qt == 2) {  // two query tiles per unit: one warp per head only
    if constexpr (FMT == kFmtInt8 && D <= 128)
      if (hpr == NCW) e = launch_tc<D, NG, NCW, 1, FMT, 2>(p, grid, stream);
  } else switch (NCW / hpr) {
    case 1: e = launch_tc<D, NG, NCW, 1, FMT>(p, grid, stream); break;
    case 2: e = launch_tc<D, NG, NCW, 2, FMT>(p, grid, stream); break;
    case 4: e = launch_tc<D, NG, NCW, 4, FMT>(p, grid, stream); break;
    case 8:
      if constexpr (NCW == 8) e = launch_tc<D, NG, NCW, 8, FMT>(p, grid, stream);
      break;
    default: break;
  }
  if (e != cudaSuccess || p.n_split_units == 0 || p.split_ctr != nullptr) return e;
  attn_combine_kernel<D><<<p.n_split_units * p.Hkv, 128, 0, stream>>>(p);
  return cudaGetLastError();
}


// ---------------------------------------------------------------------------
// CUDA-core variant (attn_impl = KRILL_ATTN_CUDA_CORE), kept as the
// measured alternative to the tensor-core path. Same planner, partial records
// and combine kernel; reads the pages straight from global memory (no staging).
// One warp per kv head of an item; lane l owns head-dim slice
// [l*EPD, (l+1)*EPD). Tokens go in batches of TB = 32/GQ: each lane forms
// partial q.k dot products for TB tokens x GQ query heads over its slice, a
// 31-shuffle reduce-scatter leaves lane L with the full score of
// (token L / GQ, head L % GQ), the scores are broadcast back, and every lane
// accumulates p.v for its slice with FMAs. Dequantization is the reference's
// (two fp16 roundings), as on the tensor-core path.
template <int D, int NG, int GQ>
__global__ void __launch_bounds__(256) attn_cc_kernel(AttnParams p) {
  using SG = SubGeom<D, NG>;
  constexpr int T = SG::T, SPB = SG::SPB, EPD = D / 32, G = D / NG;
  constexpr int TB = 32 / GQ;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int it0 = p.cta_off[blockIdx.x], it1 = p.cta_off[blockIdx.x + 1];
  const int Hkv = p.Hkv;
  const int64_t blk_stride = (int64_t)p.L * Hkv * p.page_bytes;
  const int d0 = lane * EPD;
  const int grp = d0 / G;
  for (int it = it0; it < it1; ++it) {
    const AttnItem item = p.items[it];
    const AttnUnit un = p.units[item.unit];
    const int32_t* bt = p.bt + (int64_t)un.si * p.bt_stride;
    for (int h = item.h0 + warp; h < item.h0 + p.hg; h += 8) {
      const int64_t qrow = ((int64_t)un.qo_row * p.Hq + (int64_t)h * GQ) * D;
      float qv[GQ][EPD];
#pragma unroll
      for (int hq = 0; hq < GQ; ++hq)
#pragma unroll
        for (int e = 0; e < EPD; ++e) qv[hq][e] = load_in(p.q, qrow + hq * D + d0 + e, p.q_dtype);
      float o[GQ][EPD], m[GQ], l[GQ];
#pragma unroll
      for (int hq = 0; hq < GQ; ++hq) {
        m[hq] = -INFINITY;
        l[hq] = 0.f;
#pragma unroll
        for (int e = 0; e < EPD; ++e) o[hq][e] = 0.f;
      }
      const uint8_t* head_base = p.pool + ((int64_t)un.layer * Hkv + h) * p.page_bytes;
      for (int j = item.sb_begin; j < item.sb_end; ++j) {
        int bi = j / SPB;
        if (p.ring > 0) bi %= p.ring;
        const uint8_t* sb = head_base + (int64_t)__ldg(bt + bi) * blk_stride + (int64_t)(j % SPB) * SG::SB;
        const int pos0 = j * T;
        for (int t0 = 0; t0 < T; t0 += TB) {
          // ---- partial q.k over this lane's slice ----
          float part[32];
#pragma unroll
          for (int tt = 0; tt < TB; ++tt) {
            const int t = t0 + tt;
            const __half s = __ushort_as_half(*reinterpret_cast<const uint16_t*>(sb + SG::meta(0, grp, t)));
            const __half z = __ushort_as_half(*reinterpret_cast<const uint16_t*>(sb + SG::meta(1, grp, t)));
            const uint8_t* kr = sb + sb_kcode(D, t, d0);
            float kf[EPD];
#pragma unroll
            for (int e = 0; e < EPD; ++e)
              kf[e] = __half2float(__hadd_rn(__hmul_rn(__ushort2half_rn(kr[e]), s), z));
#pragma unroll
            for (int hq = 0; hq < GQ; ++hq) {
              float a = 0.f;
#pragma unroll
              for (int e = 0; e < EPD; ++e) a = fmaf(qv[hq][e], kf[e], a);
              part[tt * GQ + hq] = a;
            }
          }
          // ---- reduce-scatter: lane L ends with the sum of part[L] ----
#pragma unroll
          for (int off = 16, n = 32; off >= 1; off >>= 1, n >>= 1) {
            const bool up = lane & off;
#pragma unroll
            for (int i = 0; i < n / 2; ++i) {
              const float send = up ? part[i] : part[i + n / 2];
              const float keep = up ? part[i + n / 2] : part[i];
              part[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
            }
          }
          const int my_t = pos0 + t0 + lane / GQ;
          float sc = part[0] * p.scale_log2;
          if (my_t < un.t_lo || my_t >= un.t_hi) sc = -INFINITY;
          // ---- online softmax per head (lanes with the same lane % GQ) ----
          float mx = sc;
#pragma unroll
          for (int off = GQ; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
          float pv[32];
          float alpha[GQ];
#pragma unroll
          for (int hq = 0; hq < GQ; ++hq) {
            const float mb = __shfl_sync(0xffffffffu, mx, hq);
            const float mn = fmaxf(m[hq], mb);
            const float base = (mn == -INFINITY) ? 0.f : mn;
            alpha[hq] = exp2f(m[hq] - base);
            m[hq] = mn;
          }
          const float my_base = (m[lane % GQ] == -INFINITY) ? 0.f : m[lane % GQ];
          const float my_p = exp2f(sc - my_base);
#pragma unroll
          for (int i = 0; i < 32; ++i) pv[i] = __shfl_sync(0xffffffffu, my_p, i);
#pragma unroll
          for (int hq = 0; hq < GQ; ++hq) {
            float ls = 0.f;
#pragma unroll
            for (int tt = 0; tt < TB; ++tt) ls += pv[tt * GQ + hq];
            l[hq] = l[hq] * alpha[hq] + ls;
#pragma unroll
            for (int e = 0; e < EPD; ++e) o[hq][e] *= alpha[hq];
          }
          // ---- p.v over this lane's slice ----
#pragma unroll
          for (int tt = 0; tt < TB; ++tt) {
            const int t = t0 + tt;
            const int pt = pos0 + t;
            const bool valid = pt >= un.t_lo && pt < un.t_hi;
            const __half s = __ushort_as_half(*reinterpret_cast<const uint16_t*>(sb + SG::meta(2, grp, t)));
            const __half z = __ushort_as_half(*reinterpret_cast<const uint16_t*>(sb + SG::meta(3, grp, t)));
#pragma unroll
            for (int e = 0; e < EPD; ++e) {
              const uint8_t c = sb[sb_vcode(D, t, d0 + e)];
              const float vf = valid ? __half2float(__hadd_rn(__hmul_rn(__ushort2half_rn(c), s), z)) : 0.f;
#pragma unroll
              for (int hq = 0; hq < GQ; ++hq) o[hq][e] = fmaf(pv[tt * GQ + hq], vf, o[hq][e]);
            }
          }
        }
      }
      // ---- finish: output, or a partial record of a split unit ----
      if (un.n_split == 1) {
#pragma unroll
        for (int hq = 0; hq < GQ; ++hq) {
          const float inv = 1.f / l[hq];
#pragma unroll
          for (int e = 0; e < EPD; ++e) store_out(p.out, p.out_dtype, qrow + hq * D + d0 + e, o[hq][e] * inv);
        }
      } else {
        const int64_t rec = ((int64_t)un.first_split + item.idx) * Hkv + h;
        float* part = p.partials + rec * partial_floats(D);
#pragma unroll
        for (int hq = 0; hq < GQ; ++hq) {
#pragma unroll
          for (int e = 0; e < EPD; ++e) part[16 + hq * D + d0 + e] = o[hq][e];
          if (lane == 0) {
            part[hq] = m[hq];
            part[8 + hq] = l[hq];
          }
        }
      }
    }
  }
}

template <int D, int NG>
cudaError_t launch_cc(const AttnParams& p, int grid, cudaStream_t stream) {
  cudaError_t e = cudaErrorInvalidValue;
  switch (p.g) {
    case 1: attn_cc_kernel<D, NG, 1><<<grid, 256, 0, stream>>>(p); e = cudaGetLastError(); break;
    case 2: attn_cc_kernel<D, NG, 2><<<grid, 256, 0, stream>>>(p); e = cudaGetLastError(); break;
    case 4: attn_cc_kernel<D, NG, 4><<<grid, 256, 0, stream>>>(p); e = cudaGetLastError(); break;
    case 8: attn_cc_kernel<D, NG, 8><<<grid, 256, 0, stream>>>(p); e = cudaGetLastError(); break;
    default: break;
  }
  if (e != cudaSuccess || p.n_split_units == 0) return e;
  attn_combine_kernel<D><<<p.n_split_units * p.Hkv, 128, 0, stream>>>(p);
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_combine(const Geom& g, const AttnParams& p, cudaStream_t stream) {
  if (p.n_split_units == 0) return cudaSuccess;
  const unsigned blocks = (unsigned)p.n_split_units * p.Hkv;
  if (g.D == 64) attn_combine_kernel<64><<<blocks, 128, 0, stream>>>(p);
  else if (g.D == 128) attn_combine_kernel<128><<<blocks, 128, 0, stream>>>(p);
  else if (g.D == 256) attn_combine_kernel<256><<<blocks, 128, 0, stream>>>(p);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

namespace {
template <int D, int NG, int NCW, int R, int FMT>
int tc_desc(char* buf, size_t cap) {
  return snprintf(buf, cap, "attn_tc_kernel<%d,%d,%d,%d,%d,%d>", D, NG, NCW, R,
                  stages_for<D, NG, NCW, R, FMT>(), FMT);
}
template <int D, int NG, int FMT = kFmtInt8>
int tc_desc_r(const AttnParams& p, char* buf, size_t cap) {
  const int hpr = p.hg < 8 ? p.hg : 8;
  if (p.qt == 2)
    return snprintf(buf, cap, "attn_tc_kernel<%d,%d,8,1,%d,%d,2>", D, NG, stages_for<D, NG, 8, 1, FMT>(), FMT);
  if (hpr <= 0 || 8 % hpr != 0) return snprintf(buf, cap, "none");
  switch (8 / hpr) {
    case 1: return tc_desc<D, NG, 8, 1, FMT>(buf, cap);
    case 2: return tc_desc<D, NG, 8, 2, FMT>(buf, cap);
    case 4: return tc_desc<D, NG, 8, 4, FMT>(buf, cap);
    default: return tc_desc<D, NG, 8, 8, FMT>(buf, cap);
  }
}
}  // namespace

// Names the kernel instances launch_attention(g, p, grid, impl) runs, in
// launch order, joined by '+'. For introspection (krill_pool_last_kernels).
void describe_attention(const Geom& g, const AttnParams& p, int grid, int impl, char* buf,
                        size_t cap) {
  size_t n = 0;
  auto put = [&](int w) { n = std::min(cap - 1, n + (size_t)(w > 0 ? w : 0)); };
  if (cap == 0) return;
  buf[0] = 0;
  if (p.sh_grid > 0)
    put(snprintf(buf + n, cap - n, "%s<%d,%d>+",
                 !shared_uses_umma(g, impl) ? "attn_shared_kernel"
                 : p.sh_pair                ? "attn_shared_pair_kernel"
                                            : "attn_shared_umma_kernel",
                 g.D, g.NG));
  if (grid > 0) {
    if (impl == 1) put(snprintf(buf + n, cap - n, "attn_cc_kernel<%d,%d,%d>", g.D, g.NG, p.g));
    else if (g.fmt == kFmtBf16 && g.D == 64) put(tc_desc_r<64, 1, kFmtBf16>(p, buf + n, cap - n));
    else if (g.fmt == kFmtBf16) put(tc_desc_r<128, 1, kFmtBf16>(p, buf + n, cap - n));
    else if (g.D == 64) put(tc_desc_r<64, 1>(p, buf + n, cap - n));
    else if (g.D == 128 && g.NG == 2) put(tc_desc_r<128, 2>(p, buf + n, cap - n));
    else if (g.D == 128) put(tc_desc_r<128, 1>(p, buf + n, cap - n));
    else if (g.NG == 4) put(tc_desc_r<256, 4>(p, buf + n, cap - n));
    else put(tc_desc_r<256, 1>(p, buf + n, cap - n));
    if (p.split_ctr != nullptr && p.n_split_units > 0 && impl != 1)
      put(snprintf(buf + n, cap - n, "[merge in kernel]"));
  }
  if (attn_needs_combine(p, grid, impl))
    put(snprintf(buf + n, cap - n, "%sattn_combine_kernel<%d>", n > 0 && buf[n - 1] != '+' ? "+" : "", g.D));
  if (n > 0 && buf[n - 1] == '+') buf[--n] = 0;
}

cudaError_t launch_attention(const Geom& g, const AttnParams& p, int grid, int impl,
                             cudaStream_t stream) {
  if (p.sh_grid > 0) {  // shared-prefix fragments first: they fill partial records
    const cudaError_t e = shared_uses_umma(g, impl) ? launch_shared_umma(g, p, stream)
                                                    : launch_shared(g, p, stream);
    if (e != cudaSuccess) return e;
  }
  if (grid <= 0) return launch_combine(g, p, stream);  // everything was in cascade items
  if (impl == 1) {  // KRILL_ATTN_CUDA_CORE
    if (g.D == 64 && g.NG == 1) return launch_cc<64, 1>(p, grid, stream);
    if (g.D == 128 && g.NG == 2) return launch_cc<128, 2>(p, grid, stream);
    if (g.D == 128 && g.NG == 1) return launch_cc<128, 1>(p, grid, stream);
    if (g.D == 256 && g.NG == 4) return launch_cc<256, 4>(p, grid, stream);
    if (g.D == 256 && g.NG == 1) return launch_cc<256, 1>(p, grid, stream);
    return cudaErrorInvalidValue;
  }
  if (g.fmt == kFmtBf16) {  // raw bf16 pools: G = D
    if (g.D == 64) return launch_tc_r<64, 1, 8, kFmtBf16>(p, grid, stream);
    if (g.D == 128) return launch_tc_r<128, 1, 8, kFmtBf16>(p, grid, stream);
    return cudaErrorInvalidValue;
  }
  if (g.D == 64 && g.NG == 1) return launch_tc_r<64, 1, 8>(p, grid, stream);
  if (g.D == 128 && g.NG == 2) return launch_tc_r<128, 2, 8>(p, grid, stream);
  if (g.D == 128 && g.NG == 1) return launch_tc_r<128, 1, 8>(p, grid, stream);
  if (g.D == 256 && g.NG == 4) return launch_tc_r<256, 4, 8>(p, grid, stream);
  if (g.D == 256 && g.NG == 1) return launch_tc_r<256, 1, 8>(p, grid, stream);
  return cudaErrorInvalidValue;
}

}  // namespace krill
