// kv_shared.cu — cascade attention over a prefix shared by several sequences.
//
// In the reference every request that restored the same prefix-cache entry
// (PrefixCache.lookupQuantized + restore, Sources/KrillEngine/InferenceEngine.swift:1305-1320)
// owns a private copy of the prefix and attends it on its own
// (MLXFast.scaledDotProductAttention, Sources/KrillCore/Gemma4Model.swift:516).
// Here the forked sequences share the prefix's blocks, and this kernel reads
// and dequantizes them once per (layer, kv head) for all member queries: the
// shared part of decode attention becomes a small GEMM-shaped problem
// (rows = member sequences x GQA group, columns = prefix tokens) instead of a
// per-request stream over the same bytes.
//
// Structure (persistent, one CTA per SM, 12 warps):
//   - warp 8 streams the prefix's raw sub-blocks HBM -> shared memory with
//     bulk async copies (cp.async.bulk) into a kShNR-stage mbarrier ring;
//   - warps 9-11 dequantize each raw sub-block once, with the reference's two
//     fp16 roundings, into f16 tiles (K [T][D], V [D][T], 16-byte chunks XOR
//     swizzled so every ldmatrix is bank-conflict free), kShNF stages;
//   - warps 0-7 own 32 query rows each (16 at D = 256) and run a flash-
//     attention style update per 32-token chunk with mma.sync m16n8k16
//     (f16 in, f32 accumulate): S = Q·Kᵀ with Q and K fragments from ldmatrix,
//     online softmax in the exp2 domain, O += P·V with P taken straight from
//     the S accumulators. The running max is only raised when a row's max
//     grows by more than 8 (log2 units), so the O rescale is rare; P then
//     stays below 256 and the final O / l is unchanged.
// Each item's result is one fp32 partial record per member (record `slot` of
// the member's unit); attn_combine_kernel merges it with the suffix pieces.
// Every wait is bounded (the pool's wait_timeout_us, then 20 us after the
// first timeout) and sets the pool's error flag instead of hanging.
#include <atomic>

#include "kv_device.cuh"

namespace krill {
namespace {

constexpr int kShNF = 2;           // f16 tile stages
constexpr int kShNR = 4;           // raw sub-block stages
constexpr int kShDeqWarps = 3;     // warps 9-11
constexpr int kShProducerRegs = 56;
constexpr int kShConsumerRegs = 224;  // 128*56 + 256*224 = 384*168, the launch budget

__device__ __forceinline__ void ldm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                       uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Physical 16-byte chunk of logical chunk c in row r of a tile whose rows hold
// CPR chunks. The 8 rows of an ldmatrix 8x8 matrix (same logical chunk) land
// in 8 distinct 16-byte bank groups.
template <int CPR>
__device__ __forceinline__ int swz(int r, int c) {
  static_assert(CPR == 4 || CPR % 8 == 0, "tile row length");
  if constexpr (CPR == 4)
    return c ^ ((r >> 1) & 3);
  else
    return c ^ (r & 7);
}

template <int D, int NG>
struct ShSmem {
  using SG = SubGeom<D, NG>;
  static constexpr int T = SG::T;
  static constexpr int ROWS = sh_rows(D);
  static constexpr int RPW = ROWS / 8;   // query rows per consumer warp
  static constexpr int MT = RPW / 16;    // 16-row m-tiles per warp
  static constexpr int QROW = D * 2;     // bytes of one f16 query row
  static constexpr int KT = T * D * 2;   // f16 K tile [T][D]
  static constexpr int VT = D * T * 2;   // f16 V tile [D][T]
  static constexpr int Q_OFF = 0;
  static constexpr int F_OFF = ROWS * QROW;
  static constexpr int R_OFF = F_OFF + kShNF * (KT + VT);
  static constexpr int BAR_OFF = R_OFF + kShNR * SG::SB;
  // raw full [NR] | raw empty [NR] | f16 full [NF] | f16 empty [NF]
  static constexpr int MISC_OFF = BAR_OFF + (2 * kShNR + 2 * kShNF) * 8;
  static constexpr int TOTAL = MISC_OFF + 16;
  static_assert(SG::SB % 16 == 0, "bulk copies move 16-byte multiples");
};

// One raw sub-block -> f16 K tile [T][D] and V tile [D][T], by the 96
// dequantizer threads (thread index t0). Values are the reference's
// f16_rn(f16_rn(code * scale) + zero) (QuantizedKVCache.swift:200-204).
template <int D, int NG>
__device__ __forceinline__ void sh_dequant(const uint8_t* __restrict__ raw, uint8_t* __restrict__ kt,
                                           uint8_t* __restrict__ vt, int t0) {
  using SG = SubGeom<D, NG>;
  constexpr int T = SG::T, G = SG::G;
  constexpr int NDT = kShDeqWarps * 32;
  // K codes: token-major rows (odd rows' 16-byte chunks swizzled by 4 when
  // D >= 128); one scale / zero per (token, group)
  for (int i = t0; i < T * (D / 16); i += NDT) {
    const int t = i / (D / 16), c = i % (D / 16);
    const int pc = D >= 128 ? (c ^ ((t & 1) << 2)) : c;
    const uint4 w = *reinterpret_cast<const uint4*>(raw + t * D + pc * 16);
    const int gi = (16 * c) / G;
    const uint32_t s = *reinterpret_cast<const uint16_t*>(raw + SG::meta(0, gi, t));
    const uint32_t z = *reinterpret_cast<const uint16_t*>(raw + SG::meta(1, gi, t));
    const uint32_t s2 = s | (s << 16), z2 = z | (z << 16);
    uint4 lo, hi;
    lo.x = deq2(w.x, 0x4140u, s2, z2);
    lo.y = deq2(w.x, 0x4342u, s2, z2);
    lo.z = deq2(w.y, 0x4140u, s2, z2);
    lo.w = deq2(w.y, 0x4342u, s2, z2);
    hi.x = deq2(w.z, 0x4140u, s2, z2);
    hi.y = deq2(w.z, 0x4342u, s2, z2);
    hi.z = deq2(w.w, 0x4140u, s2, z2);
    hi.w = deq2(w.w, 0x4342u, s2, z2);
    uint8_t* row = kt + t * (D * 2);
    *reinterpret_cast<uint4*>(row + swz<D / 8>(t, 2 * c) * 16) = lo;
    *reinterpret_cast<uint4*>(row + swz<D / 8>(t, 2 * c + 1) * 16) = hi;
  }
  // V codes: transposed [D][T]; scale / zero per (token, group), so each
  // pair of tokens takes its own pair of scales
  for (int i = t0; i < D * (T / 16); i += NDT) {
    const int d = i / (T / 16), c = i % (T / 16);
    const uint4 w = *reinterpret_cast<const uint4*>(raw + SG::VOFF + d * T + c * 16);
    const int gi = d / G;
    const uint4 sa = *reinterpret_cast<const uint4*>(raw + SG::meta(2, gi, 16 * c));
    const uint4 sb = *reinterpret_cast<const uint4*>(raw + SG::meta(2, gi, 16 * c + 8));
    const uint4 za = *reinterpret_cast<const uint4*>(raw + SG::meta(3, gi, 16 * c));
    const uint4 zb = *reinterpret_cast<const uint4*>(raw + SG::meta(3, gi, 16 * c + 8));
    uint4 lo, hi;
    lo.x = deq2(w.x, 0x4140u, sa.x, za.x);
    lo.y = deq2(w.x, 0x4342u, sa.y, za.y);
    lo.z = deq2(w.y, 0x4140u, sa.z, za.z);
    lo.w = deq2(w.y, 0x4342u, sa.w, za.w);
    hi.x = deq2(w.z, 0x4140u, sb.x, zb.x);
    hi.y = deq2(w.z, 0x4342u, sb.y, zb.y);
    hi.z = deq2(w.w, 0x4140u, sb.z, zb.z);
    hi.w = deq2(w.w, 0x4342u, sb.w, zb.w);
    uint8_t* row = vt + d * (T * 2);
    *reinterpret_cast<uint4*>(row + swz<T / 8>(d, 2 * c) * 16) = lo;
    *reinterpret_cast<uint4*>(row + swz<T / 8>(d, 2 * c + 1) * 16) = hi;
  }
}

// This warp's RPW query rows of an item -> f16 rows in shared memory (rows
// past the item's n_rows are zero).
template <int D, int RPW>
__device__ __forceinline__ void sh_load_q(const AttnParams& p, const ShItem& item, int row0,
                                          uint8_t* qs, int lane) {
  constexpr int CPR = D / 8;
  const int gq = p.g;
  for (int i = lane; i < RPW * CPR; i += 32) {
    const int rr = i / CPR, c = i % CPR;
    const int R = row0 + rr;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (R < item.n_rows) {
      const int mem = R / gq, jq = R - mem * gq;
      const int64_t qrow = p.units[p.sh_members[item.mem_off + mem]].qo_row;
      const uint4* src = reinterpret_cast<const uint4*>(
                             static_cast<const uint16_t*>(p.q) +
                             ((qrow * p.Hq + (int64_t)item.h * gq + jq) * D)) + c;
      v = __ldg(src);
      if (p.q_dtype == 1) {  // bf16 -> f16 (exact in the f16 normal range)
        uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&wv[k]));
          wv[k] = f2h2(f.x, f.y);
        }
        v = make_uint4(wv[0], wv[1], wv[2], wv[3]);
      }
    }
    *reinterpret_cast<uint4*>(qs + rr * (D * 2) + swz<CPR>(rr, c) * 16) = v;
  }
}

// One f16 K/V tile (T tokens) against this warp's query rows.
template <int D, int NG>
__device__ __forceinline__ void sh_tile(uint32_t qw, uint32_t kt, uint32_t vt,
                                        float (&o)[ShSmem<D, NG>::MT][D / 8][4],
                                        float (&m)[ShSmem<D, NG>::MT][2],
                                        float (&l)[ShSmem<D, NG>::MT][2], int lane,
                                        float scale_log2) {
  using SM = ShSmem<D, NG>;
  constexpr int T = SM::T, MT = SM::MT;
  constexpr int KROW = D * 2, VROW = T * 2;
  const int l7 = lane & 7, hi8 = (lane >> 3) & 1, hi16 = lane >> 4;
#pragma unroll
  for (int c0 = 0; c0 < T; c0 += 32) {
    // ---- S = Q · Kᵀ for 32 tokens (4 n-tiles of 8) ----
    float s[MT][4][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) s[mt][nt][c] = 0.f;
#pragma unroll
    for (int kc = 0; kc < D / 16; ++kc) {
      uint32_t a[MT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int row = 16 * mt + l7 + 8 * hi8;
        ldm_x4(qw + row * (D * 2) + (((2 * kc + hi16) ^ l7) << 4), a[mt][0], a[mt][1], a[mt][2],
               a[mt][3]);
      }
      uint32_t b[4][2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int tok = c0 + 16 * hh + l7 + 8 * hi16;
        ldm_x4(kt + tok * KROW + (((2 * kc + hi8) ^ l7) << 4), b[2 * hh][0], b[2 * hh][1],
               b[2 * hh + 1][0], b[2 * hh + 1][1]);
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
          mma16816(s[mt][nt], a[mt][0], a[mt][1], a[mt][2], a[mt][3], b[nt][0], b[nt][1]);
    }
    // ---- online softmax: rows r (hf = 0) and r + 8 (hf = 1) of each m-tile ----
    float mx[MT][2];
    bool grow = false;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        float v = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          s[mt][nt][2 * hf] *= scale_log2;
          s[mt][nt][2 * hf + 1] *= scale_log2;
          v = fmaxf(v, fmaxf(s[mt][nt][2 * hf], s[mt][nt][2 * hf + 1]));
        }
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
        mx[mt][hf] = v;
        grow |= v > m[mt][hf] + 8.f;
      }
    if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const float mn = fmaxf(m[mt][hf], mx[mt][hf]);
          const float al = exp2f(m[mt][hf] - mn);
          m[mt][hf] = mn;
          l[mt][hf] *= al;
#pragma unroll
          for (int dt = 0; dt < D / 8; ++dt) {
            o[mt][dt][2 * hf] *= al;
            o[mt][dt][2 * hf + 1] *= al;
          }
        }
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        float ps = 0.f;
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
          const float p0 = exp2f(s[mt][nt][2 * hf] - m[mt][hf]);
          const float p1 = exp2f(s[mt][nt][2 * hf + 1] - m[mt][hf]);
          s[mt][nt][2 * hf] = p0;
          s[mt][nt][2 * hf + 1] = p1;
          ps += p0 + p1;
        }
        l[mt][hf] += ps;
      }
    // ---- O += P · V: P's A fragments are the S accumulators packed to f16 ----
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      uint32_t pa[MT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        pa[mt][0] = f2h2(s[mt][2 * kk][0], s[mt][2 * kk][1]);
        pa[mt][1] = f2h2(s[mt][2 * kk][2], s[mt][2 * kk][3]);
        pa[mt][2] = f2h2(s[mt][2 * kk + 1][0], s[mt][2 * kk + 1][1]);
        pa[mt][3] = f2h2(s[mt][2 * kk + 1][2], s[mt][2 * kk + 1][3]);
      }
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        const int drow = 16 * dp + l7 + 8 * hi16;
        const int chunk = c0 / 8 + 2 * kk + hi8;
        uint32_t b0, b1, b2, b3;
        ldm_x4(vt + drow * VROW + (swz<T / 8>(drow, chunk) << 4), b0, b1, b2, b3);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          mma16816(o[mt][2 * dp], pa[mt][0], pa[mt][1], pa[mt][2], pa[mt][3], b0, b1);
          mma16816(o[mt][2 * dp + 1], pa[mt][0], pa[mt][1], pa[mt][2], pa[mt][3], b2, b3);
        }
      }
    }
  }
}

template <int D, int NG>
__global__ void __launch_bounds__(384, 1) attn_shared_kernel(AttnParams p) {
  using SM = ShSmem<D, NG>;
  using SG = SubGeom<D, NG>;
  constexpr int SB = SG::SB, RPW = SM::RPW, MT = SM::MT;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_rf = sbase + SM::BAR_OFF, bar_re = bar_rf + 8 * kShNR;
  const uint32_t bar_ff = bar_re + 8 * kShNR, bar_fe = bar_ff + 8 * kShNF;
  volatile int* cta_abort = reinterpret_cast<volatile int*>(smem + SM::MISC_OFF);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < kShNR; ++s) {
      mbar_init(bar_rf + 8 * s, 1);            // copy issuer arrive + tx bytes
      mbar_init(bar_re + 8 * s, kShDeqWarps);  // each dequantizer warp
    }
    for (int s = 0; s < kShNF; ++s) {
      mbar_init(bar_ff + 8 * s, kShDeqWarps);
      mbar_init(bar_fe + 8 * s, 8);            // each consumer warp
    }
    init_wait_state(cta_abort, p.wait_us);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const int it0 = p.sh_cta_off[blockIdx.x], it1 = p.sh_cta_off[blockIdx.x + 1];
  const int Hkv = p.Hkv;

  if (warp >= 8) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kShProducerRegs));
    if (warp == 8) {
      if (lane != 0) return;
      // ---------------- copy issuer ----------------
      const int64_t blk_stride = (int64_t)p.L * Hkv * p.page_bytes;
      uint32_t J = 0;
      for (int it = it0; it < it1; ++it) {
        const ShItem item = p.sh_items[it];
        const int32_t* bt = p.bt + (int64_t)item.leader * p.bt_stride;
        const uint8_t* page = p.pool + ((int64_t)item.layer * Hkv + item.h) * p.page_bytes;
        for (int j = item.sb_begin; j < item.sb_end; ++j, ++J) {
          const int b = __ldg(bt + j / SG::SPB);
          const uint32_t s = J % kShNR;
          if (J >= (uint32_t)kShNR)
            mbar_wait(bar_re + 8 * s, ((J / kShNR) - 1) & 1, cta_abort, p.err);
          mbar_expect_tx(bar_rf + 8 * s, SB);
          bulk_g2s(sbase + SM::R_OFF + s * SB,
                   page + (int64_t)b * blk_stride + (int64_t)(j % SG::SPB) * SB, SB, bar_rf + 8 * s);
        }
      }
      // every issued copy has landed before this CTA may exit
      for (uint32_t k = J > (uint32_t)kShNR ? J - kShNR : 0; k < J; ++k)
        mbar_wait(bar_rf + 8 * (k % kShNR), (k / kShNR) & 1, cta_abort, p.err);
      return;
    }
    // ---------------- dequantizers ----------------
    const int t0 = tid - 9 * 32;
    uint32_t J = 0;
    for (int it = it0; it < it1; ++it) {
      const ShItem item = p.sh_items[it];
      for (int j = item.sb_begin; j < item.sb_end; ++j, ++J) {
        const uint32_t rs = J % kShNR, fs = J % kShNF;
        mbar_wait(bar_rf + 8 * rs, (J / kShNR) & 1, cta_abort, p.err);
        if (J >= (uint32_t)kShNF)
          mbar_wait(bar_fe + 8 * fs, ((J / kShNF) - 1) & 1, cta_abort, p.err);
        uint8_t* kt = smem + SM::F_OFF + fs * (SM::KT + SM::VT);
        sh_dequant<D, NG>(smem + SM::R_OFF + rs * SB, kt, kt + SM::KT, t0);
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(bar_re + 8 * rs);
          mbar_arrive(bar_ff + 8 * fs);
        }
      }
    }
    return;
  }

  // ---------------- consumers: warp w owns query rows [w*RPW, (w+1)*RPW) ----------------
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kShConsumerRegs));
  const int r = lane >> 2, tq = lane & 3;
  const int row0 = warp * RPW;
  uint8_t* qs = smem + SM::Q_OFF + row0 * SM::QROW;
  const uint32_t qw = sbase + SM::Q_OFF + row0 * SM::QROW;
  const int gq = p.g;
  float o[MT][D / 8][4];
  float m[MT][2], l[MT][2];
  uint32_t J = 0;
  for (int it = it0; it < it1; ++it) {
    const ShItem item = p.sh_items[it];
    const bool active = row0 < item.n_rows;  // warp-uniform
    if (active) {
      sh_load_q<D, RPW>(p, item, row0, qs, lane);
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
        for (int dt = 0; dt < D / 8; ++dt)
#pragma unroll
          for (int c = 0; c < 4; ++c) o[mt][dt][c] = 0.f;
        m[mt][0] = m[mt][1] = -INFINITY;
        l[mt][0] = l[mt][1] = 0.f;
      }
    }
    __syncwarp();
    for (int j = item.sb_begin; j < item.sb_end; ++j, ++J) {
      const uint32_t fs = J % kShNF;
      mbar_wait(bar_ff + 8 * fs, (J / kShNF) & 1, cta_abort, p.err);
      if (active) {
        const uint32_t kt = sbase + SM::F_OFF + fs * (SM::KT + SM::VT);
        sh_tile<D, NG>(qw, kt, kt + SM::KT, o, m, l, lane, p.scale_log2);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_fe + 8 * fs);
    }
    if (!active) continue;
    // ---- partial records: one per (member, kv head) row group ----
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        float lv = l[mt][hf];
        lv += __shfl_xor_sync(0xffffffffu, lv, 1);
        lv += __shfl_xor_sync(0xffffffffu, lv, 2);
        const int R = row0 + 16 * mt + 8 * hf + r;
        if (R >= item.n_rows) continue;
        const int mem = R / gq, jq = R - mem * gq;
        const AttnUnit un = p.units[p.sh_members[item.mem_off + mem]];
        float* part = p.partials +
                      ((int64_t)(un.first_split + item.slot) * Hkv + item.h) * partial_floats(D);
#pragma unroll
        for (int dt = 0; dt < D / 8; ++dt)
          *reinterpret_cast<float2*>(part + 16 + jq * D + 8 * dt + 2 * tq) =
              make_float2(o[mt][dt][2 * hf], o[mt][dt][2 * hf + 1]);
        if (tq == 0) {
          part[jq] = m[mt][hf];
          part[8 + jq] = lv;
          // the first fragment also marks this pair's unused slots empty
          if (item.slot == 0)
            for (int sl = item.n_frag; sl < p.n_pslots; ++sl) {
              float* e = p.partials +
                         ((int64_t)(un.first_split + sl) * Hkv + item.h) * partial_floats(D);
              e[jq] = -INFINITY;
              e[8 + jq] = 0.f;
            }
        }
      }
  }
}

template <int D, int NG>
cudaError_t launch_sh(const AttnParams& p, cudaStream_t stream) {
  using SM = ShSmem<D, NG>;
  static_assert(SM::TOTAL <= 232448, "shared memory budget");
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    // setmaxnreg.inc waits until released registers cover it: refuse a build
    // whose launch register count would not balance the split
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, attn_shared_kernel<D, NG>);
    if (e != cudaSuccess) return e;
    if (fa.numRegs * 384 < 128 * kShProducerRegs + 256 * kShConsumerRegs)
      return cudaErrorInvalidConfiguration;
    e = cudaFuncSetAttribute(attn_shared_kernel<D, NG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SM::TOTAL);
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit);
  }
  attn_shared_kernel<D, NG><<<p.sh_grid, 384, SM::TOTAL, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_shared(const Geom& g, const AttnParams& p, cudaStream_t stream) {
  if (p.sh_grid <= 0) return cudaSuccess;
  if (g.D == 64 && g.NG == 1) return launch_sh<64, 1>(p, stream);
  if (g.D == 128 && g.NG == 2) return launch_sh<128, 2>(p, stream);
  if (g.D == 128 && g.NG == 1) return launch_sh<128, 1>(p, stream);
  if (g.D == 256 && g.NG == 4) return launch_sh<256, 4>(p, stream);
  if (g.D == 256 && g.NG == 1) return launch_sh<256, 1>(p, stream);
  return cudaErrorInvalidValue;
}

}  // namespace krill
