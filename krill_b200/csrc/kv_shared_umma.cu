// kv_shared_umma.cu — cascade attention over a shared prefix on the
// 5th-generation tensor cores (tcgen05.mma, accumulators in tensor memory).
//
// Same work items and results as kv_shared.cu (forks of one prefix-cache
// entry attend the common blocks once per (layer, kv head); see there for the
// reference mapping), for head_dim 64 and 128. An item covers up to 256 query
// rows as two 128-row halves that share every K/V tile. One CTA per SM, 20
// warps:
//   - warp 9 streams raw sub-blocks HBM -> shared memory (cp.async.bulk);
//   - warps 10-19 dequantize each raw sub-block once (the reference's two
//     fp16 roundings) into f16 K [64 tok][D] and V [D][64 tok] tiles laid out
//     as the tensor core's canonical K-major 128-byte-swizzled operands;
//   - warp 8 owns the tensor memory (512 columns) and one of its lanes issues
//     the MMAs, per half h:
//       S_h  = Q_h · K_jᵀ     (M = 128 query rows, N = 64 tokens, K = D)
//       O_h += P_h · V_j      (M = 128, N = D, K = 64 tokens)
//     with S double-buffered in tensor memory so the softmax of tile j
//     overlaps S of tile j+1; each group of MMAs is committed to an mbarrier;
//   - warps 4h .. 4h+3 (thread t = query row t of half h = tensor-memory
//     lane t) read S with tcgen05.ld, run the online softmax in the exp2
//     domain (one ex2.approx.ftz and one fma per score) and write P_h as f16
//     into a swizzled shared tile. The running max
//     is only raised when a row's max grows by more than 8 (log2 units); the
//     rare O rescale is a tcgen05.ld / st round trip after the previous P·V
//     has completed. At the end of an item they read O and write the fp32
//     partial records.
// Every wait is bounded (the pool's wait_timeout_us, then 20 us after the
// first timeout) and sets the pool's error flag; the tensor memory is released on every path.
#include <atomic>

#include "kv_device.cuh"

namespace krill {
namespace {

constexpr int kUmNF = 3;         // f16 K/V tile stages
constexpr int kUmNR = 2;         // raw sub-block stages
constexpr int kUmDeqWarps = 10;  // warps 10-19
constexpr int kUmThreads = 640;  // 20 warps
// Register split (setmaxnreg): the two softmax warpgroups hold a 64-column S
// row per thread and take 120; the MMA, copy and dequantizer warpgroups give
// theirs back to 80. 256*120 + 384*80 = 61,440 = 640*96, the launch budget.
// (Of the splits that fit, this one spills least.)
constexpr int kUmSoftmaxRegs = 120;
constexpr int kUmOtherRegs = 80;
// tensor memory: half h owns columns [256h, 256h + 256): O_h at +0 (D columns),
// S_h double buffer at +128 and +192
constexpr uint32_t kUmCols = 512;
constexpr uint32_t kUmS0 = 128;

// ---- tensor-core primitives (PTX ISA 8.6+, sm_100a) ----
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// generic-proxy shared-memory writes -> visible to the tensor core (async proxy)
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrives on the mbarrier once every MMA this thread issued so far completed
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// 32 consecutive fp32 columns of this thread's tensor-memory lane; the wait
// sits in the same statement so no use of the registers can precede it.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

// Shared-memory matrix descriptor of a K-major operand in the canonical
// 128-byte-swizzle layout: rows of 64 f16 (128 B), 8-row groups of 1024 B
// stacked contiguously, 16-byte chunk c of row r stored at chunk c ^ (r & 7).
// Advancing along K by 16 elements inside a swizzle atom adds 32 B to the
// start address; the next 64-element atom starts rows * 128 B further.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);  // start address
  d |= (uint64_t)1 << 16;                            // leading byte offset (unused when swizzled)
  d |= (uint64_t)(1024 >> 4) << 32;                  // stride byte offset: next 8-row group
  d |= (uint64_t)1 << 46;                            // descriptor version for sm_100
  d |= (uint64_t)2 << 61;                            // 128-byte swizzle
  return d;
}
// Instruction descriptor: f16 A and B, f32 accumulator, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// Byte offset of 16-byte chunk c (along K) of row r in a K-major SW128 tile of
// `rows` rows.
__device__ __forceinline__ uint32_t sw128_off(int rows, int r, int c) {
  return (uint32_t)((c >> 3) * rows * 128 + (r >> 3) * 1024 + (r & 7) * 128 + (((c & 7) ^ (r & 7)) << 4));
}


template <int D, int NG>
struct UmSmem {
  using SG = SubGeom<D, NG>;
  static_assert(SG::T == 64, "one 64-token sub-block per tile");
  static constexpr int QH_BYTES = 128 * D * 2;  // one 128-row half of the Q tile
  static constexpr int P_BYTES = 128 * 64 * 2;  // one half's P tile
  static constexpr int K_BYTES = 64 * D * 2;
  static constexpr int V_BYTES = D * 64 * 2;
  static constexpr int Q_OFF = 0;                     // 2 halves
  static constexpr int P_OFF = Q_OFF + 2 * QH_BYTES;  // 2 halves
  static constexpr int KV_OFF = P_OFF + 2 * P_BYTES;
  static constexpr int KV_STAGE = K_BYTES + V_BYTES;
  static constexpr int RAW_OFF = KV_OFF + kUmNF * KV_STAGE;
  static constexpr int BAR_OFF = RAW_OFF + kUmNR * SG::SB;
  // raw full/empty [NR], kv full/empty [NF]; per half: s full [2], p full,
  // pv done, q full; fin
  static constexpr int B_RF = 0, B_RE = kUmNR, B_KF = 2 * kUmNR, B_KE = 2 * kUmNR + kUmNF,
                       B_SF = 2 * kUmNR + 2 * kUmNF,  // [half][2]
                       B_PF = B_SF + 4, B_PD = B_PF + 2, B_QF = B_PD + 2, B_FIN = B_QF + 2,
                       NBAR = B_FIN + 1;
  static constexpr int MISC_OFF = BAR_OFF + NBAR * 8;  // tmem address, abort flag
  static constexpr int TOTAL = MISC_OFF + 16;
  static_assert(SG::SB % 16 == 0 && KV_STAGE % 1024 == 0 && QH_BYTES % 1024 == 0, "alignment");
};

// One raw sub-block -> f16 K tile [64 tok][D] and V tile [D][64 tok] in the
// SW128 K-major layout; values f16_rn(f16_rn(code * scale) + zero)
// (QuantizedKVCache.swift:200-204). t0 = dequantizer thread index. Each
// thread first loads all of its items (codes and their scales / zeros), then
// converts and stores them, so the shared-memory latencies overlap. When every
// scale of an item is below 64 in magnitude the product is formed by one fma
// (exact then, see deq2_fast).
__device__ __forceinline__ uint32_t small2(uint32_t s2) {  // both halves |s| < 64
  return __vcmpgeu2(s2 & 0x7fff7fffu, 0x54005400u);
}
__device__ __forceinline__ uint4 deq16(uint4 w, const uint32_t (&s)[8], const uint32_t (&z)[8],
                                       bool fast, bool hi) {
  const int o = hi ? 4 : 0;
  const uint32_t a = hi ? w.z : w.x, b = hi ? w.w : w.y;
  uint4 r;
  if (fast) {
    r.x = deq2_fast(a, 0x4140u, s[o], neg1024(s[o]), z[o]);
    r.y = deq2_fast(a, 0x4342u, s[o + 1], neg1024(s[o + 1]), z[o + 1]);
    r.z = deq2_fast(b, 0x4140u, s[o + 2], neg1024(s[o + 2]), z[o + 2]);
    r.w = deq2_fast(b, 0x4342u, s[o + 3], neg1024(s[o + 3]), z[o + 3]);
  } else {
    r.x = deq2(a, 0x4140u, s[o], z[o]);
    r.y = deq2(a, 0x4342u, s[o + 1], z[o + 1]);
    r.z = deq2(b, 0x4140u, s[o + 2], z[o + 2]);
    r.w = deq2(b, 0x4342u, s[o + 3], z[o + 3]);
  }
  return r;
}
template <int D, int NG>
__device__ __forceinline__ void um_dequant(const uint8_t* __restrict__ raw, uint8_t* __restrict__ kt,
                                           uint8_t* __restrict__ vt, int t0) {
  using SG = SubGeom<D, NG>;
  constexpr int G = SG::G;
  constexpr int NDT = kUmDeqWarps * 32;
  constexpr int NK = 64 * (D / 16), NV = D * 4;  // 16-element items
  constexpr int KI = (NK + NDT - 1) / NDT, VI = (NV + NDT - 1) / NDT;
  // ---- K: token-major codes (odd rows' chunks swizzled by 4 when D >= 128),
  // one scale / zero per (token, group) ----
  uint4 kw[KI];
  uint32_t ks[KI], kz[KI];
#pragma unroll
  for (int k = 0; k < KI; ++k) {
    const int i = t0 + k * NDT;
    if (i < NK) {
      const int t = i / (D / 16), c = i % (D / 16);
      const int pc = D >= 128 ? (c ^ ((t & 1) << 2)) : c;
      kw[k] = *reinterpret_cast<const uint4*>(raw + t * D + pc * 16);
      ks[k] = *reinterpret_cast<const uint16_t*>(raw + SG::meta(0, (16 * c) / G, t));
      kz[k] = *reinterpret_cast<const uint16_t*>(raw + SG::meta(1, (16 * c) / G, t));
    }
  }
  // ---- V: transposed codes [D][64]; scale / zero per (token, group) ----
  uint4 vw[VI], vs[VI][2], vz[VI][2];
#pragma unroll
  for (int k = 0; k < VI; ++k) {
    const int i = t0 + k * NDT;
    if (i < NV) {
      const int d = i >> 2, c = i & 3, gi = d / G;
      vw[k] = *reinterpret_cast<const uint4*>(raw + SG::VOFF + d * 64 + c * 16);
      vs[k][0] = *reinterpret_cast<const uint4*>(raw + SG::meta(2, gi, 16 * c));
      vs[k][1] = *reinterpret_cast<const uint4*>(raw + SG::meta(2, gi, 16 * c + 8));
      vz[k][0] = *reinterpret_cast<const uint4*>(raw + SG::meta(3, gi, 16 * c));
      vz[k][1] = *reinterpret_cast<const uint4*>(raw + SG::meta(3, gi, 16 * c + 8));
    }
  }
#pragma unroll
  for (int k = 0; k < KI; ++k) {
    const int i = t0 + k * NDT;
    if (i < NK) {
      const int t = i / (D / 16), c = i % (D / 16);
      const uint32_t s2 = ks[k] | (ks[k] << 16), z2 = kz[k] | (kz[k] << 16);
      const uint32_t s8[8] = {s2, s2, s2, s2, s2, s2, s2, s2};
      const uint32_t z8[8] = {z2, z2, z2, z2, z2, z2, z2, z2};
      const bool fast = small2(s2) == 0;
      *reinterpret_cast<uint4*>(kt + sw128_off(64, t, 2 * c)) = deq16(kw[k], s8, z8, fast, false);
      *reinterpret_cast<uint4*>(kt + sw128_off(64, t, 2 * c + 1)) = deq16(kw[k], s8, z8, fast, true);
    }
  }
#pragma unroll
  for (int k = 0; k < VI; ++k) {
    const int i = t0 + k * NDT;
    if (i < NV) {
      const int d = i >> 2, c = i & 3;
      const uint32_t s8[8] = {vs[k][0].x, vs[k][0].y, vs[k][0].z, vs[k][0].w,
                              vs[k][1].x, vs[k][1].y, vs[k][1].z, vs[k][1].w};
      const uint32_t z8[8] = {vz[k][0].x, vz[k][0].y, vz[k][0].z, vz[k][0].w,
                              vz[k][1].x, vz[k][1].y, vz[k][1].z, vz[k][1].w};
      const bool fast = (small2(s8[0]) | small2(s8[1]) | small2(s8[2]) | small2(s8[3]) |
                         small2(s8[4]) | small2(s8[5]) | small2(s8[6]) | small2(s8[7])) == 0;
      // the codes of tokens 8-15 take the scales of words 4-7
      *reinterpret_cast<uint4*>(vt + sw128_off(D, d, 2 * c)) = deq16(vw[k], s8, z8, fast, false);
      *reinterpret_cast<uint4*>(vt + sw128_off(D, d, 2 * c + 1)) = deq16(vw[k], s8, z8, fast, true);
    }
  }
}

// 2^x by the special-function unit (ex2.approx.ftz.f32: one instruction;
// results below 2^-126 flush to zero, immaterial next to a row sum >= 1).
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float max64(const float (&a)[32], const float (&b)[32]) {
  float m[8];
#pragma unroll
  for (int k = 0; k < 8; ++k)
    m[k] = fmaxf(fmaxf(fmaxf(a[4 * k], a[4 * k + 1]), fmaxf(a[4 * k + 2], a[4 * k + 3])),
                 fmaxf(fmaxf(b[4 * k], b[4 * k + 1]), fmaxf(b[4 * k + 2], b[4 * k + 3])));
#pragma unroll
  for (int k = 0; k < 4; ++k) m[k] = fmaxf(m[k], m[k + 4]);
  return fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
}

template <int D, int NG>
__global__ void __launch_bounds__(kUmThreads, 1) attn_shared_umma_kernel(AttnParams p) {
  using SM = UmSmem<D, NG>;
  using SG = SubGeom<D, NG>;
  constexpr int SB = SG::SB;
  extern __shared__ __align__(1024) uint8_t smem[];
  // The swizzled operand tiles need 1024-byte alignment. The dynamic shared
  // memory of a kernel without static shared memory starts 1024-aligned on
  // sm_100; should that not hold, the launch reports an error instead of
  // computing with misplaced tiles.
  const uint32_t sbase = smem_u32(smem);
  if (sbase & 1023u) {
    if (threadIdx.x == 0) atomicOr(p.err, kErrBadArg);
    return;
  }
  auto bar = [&](int i) { return sbase + SM::BAR_OFF + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + SM::MISC_OFF);
  volatile int* cta_abort = reinterpret_cast<volatile int*>(smem + SM::MISC_OFF + 4);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < kUmNR; ++s) {
      mbar_init(bar(SM::B_RF + s), 1);            // copy issuer arrive + tx bytes
      mbar_init(bar(SM::B_RE + s), kUmDeqWarps);  // dequantizer warps
    }
    for (int s = 0; s < kUmNF; ++s) {
      mbar_init(bar(SM::B_KF + s), kUmDeqWarps);
      mbar_init(bar(SM::B_KE + s), 1);            // MMA commit
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(bar(SM::B_SF + 2 * h), 1);        // MMA commit
      mbar_init(bar(SM::B_SF + 2 * h + 1), 1);
      mbar_init(bar(SM::B_PF + h), 4);            // the half's softmax warps
      mbar_init(bar(SM::B_PD + h), 1);            // MMA commit
      mbar_init(bar(SM::B_QF + h), 4);
    }
    mbar_init(bar(SM::B_FIN), 1);
    init_wait_state(cta_abort, p.wait_us);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 8) {
    tmem_alloc(smem_u32(tmem_slot), kUmCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int it0 = p.sh_cta_off[blockIdx.x], it1 = p.sh_cta_off[blockIdx.x + 1];
  const int Hkv = p.Hkv;

  // Each warpgroup adjusts its registers at one point of its own branch
  // (setmaxnreg is .sync.aligned over the warpgroup): warpgroups 2-4 (MMA,
  // copies, dequantizers) give registers back, 0-1 (softmax) take them.
  if (warp >= 8) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kUmOtherRegs));
  if (warp == 9) {
    // ---------------- copy issuer ----------------
    if (lane == 0) {
      const int64_t blk_stride = (int64_t)p.L * Hkv * p.page_bytes;
      uint32_t J = 0;
      for (int it = it0; it < it1; ++it) {
        const ShItem item = p.sh_items[it];
        const int32_t* bt = p.bt + (int64_t)item.leader * p.bt_stride;
        const uint8_t* page = p.pool + ((int64_t)item.layer * Hkv + item.h) * p.page_bytes;
        for (int j = item.sb_begin; j < item.sb_end; ++j, ++J) {
          const int b = __ldg(bt + j / SG::SPB);
          const uint32_t s = J % kUmNR;
          if (J >= (uint32_t)kUmNR)
            mbar_wait(bar(SM::B_RE + s), ((J / kUmNR) - 1) & 1, cta_abort, p.err);
          mbar_expect_tx(bar(SM::B_RF + s), SB);
          bulk_g2s(sbase + SM::RAW_OFF + s * SB,
                   page + (int64_t)b * blk_stride + (int64_t)(j % SG::SPB) * SB, SB,
                   bar(SM::B_RF + s));
        }
      }
      // every issued copy has landed before the CTA may exit
      for (uint32_t k = J > (uint32_t)kUmNR ? J - kUmNR : 0; k < J; ++k)
        mbar_wait(bar(SM::B_RF + k % kUmNR), (k / kUmNR) & 1, cta_abort, p.err);
    }
  } else if (warp >= 10) {
    // ---------------- dequantizers ----------------
    const int t0 = tid - 10 * 32;
    uint32_t J = 0;
    for (int it = it0; it < it1; ++it) {
      const ShItem item = p.sh_items[it];
      for (int j = item.sb_begin; j < item.sb_end; ++j, ++J) {
        const uint32_t rs = J % kUmNR, fs = J % kUmNF;
        mbar_wait(bar(SM::B_RF + rs), (J / kUmNR) & 1, cta_abort, p.err);
        if (J >= (uint32_t)kUmNF)
          mbar_wait(bar(SM::B_KE + fs), ((J / kUmNF) - 1) & 1, cta_abort, p.err);
        uint8_t* kt = smem + SM::KV_OFF + fs * SM::KV_STAGE;
        um_dequant<D, NG>(smem + SM::RAW_OFF + rs * SB, kt, kt + SM::K_BYTES, t0);
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(bar(SM::B_RE + rs));
          mbar_arrive(bar(SM::B_KF + fs));
        }
      }
    }
  } else {
    // ---------------- MMA issuer (warp 8) ----------------
    if (lane == 0) {
      constexpr uint32_t idS = umma_idesc(128, 64), idO = umma_idesc(128, D);
      uint32_t cnt0 = 0, cnt1 = 0;  // tiles processed by each half
      uint32_t qn0 = 0, qn1 = 0;    // items processed by each half
      uint32_t J = 0;
      // Shared-memory descriptors built once: per K/V stage and per half. An
      // operand at a fixed byte offset o from a tile's start is its tile
      // descriptor plus o / 16 (the start-address field; every address here
      // is below 256 KB, so the addition never carries out of the field).
      const uint64_t dK0 = sw128_desc(sbase + SM::KV_OFF);
      const uint64_t dV0 = sw128_desc(sbase + SM::KV_OFF + SM::K_BYTES);
      const uint64_t dQ0 = sw128_desc(sbase + SM::Q_OFF);
      const uint64_t dP0 = sw128_desc(sbase + SM::P_OFF);
      // O_h += P_h · V of K/V stage st (P_h ready: PF observed by the caller)
      auto issue_pv = [&](int h, uint32_t st, bool first) {
        const uint64_t pd = dP0 + (uint64_t)(h * (SM::P_BYTES >> 4));
        const uint64_t vd = dV0 + (uint64_t)(st * (SM::KV_STAGE >> 4));
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma_f16(tmem + 256u * h, pd + (uint64_t)(2 * ks), vd + (uint64_t)(2 * ks), idO,
                   (!first || ks > 0) ? 1u : 0u);
        umma_commit(bar(SM::B_PD + h));  // O_h updated, P_h free
      };
      for (int it = it0; it < it1; ++it) {
        const ShItem item = p.sh_items[it];
        const int n = item.sb_end - item.sb_begin;
        const int nh = (item.n_rows + 127) >> 7;
        mbar_wait(bar(SM::B_QF), qn0 & 1, cta_abort, p.err);
        ++qn0;
        if (nh > 1) {
          mbar_wait(bar(SM::B_QF + 1), qn1 & 1, cta_abort, p.err);
          ++qn1;
        }
        tc_fence_after();
        // S of tile js goes out once its K/V tiles are ready and its S buffer
        // has been read (the softmax of tile js-2 is done, i.e. P·V of js-2 was
        // issued); P·V of tile jp once both halves' P are ready. Whichever is
        // ready first is issued, so neither chain waits on the other.
        int js = 0, jp = 0;
        uint32_t spins = 0;
        uint64_t idle_since = 0;
        while (jp < n) {
          bool progressed = false;
          if (js < n && js <= jp + 1) {
            const uint32_t Jc = J + js, st = Jc % kUmNF;
            if (mbar_try_wait(bar(SM::B_KF + st), (Jc / kUmNF) & 1)) {
              tc_fence_after();
              const uint64_t kd = dK0 + (uint64_t)(st * (SM::KV_STAGE >> 4));
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                if (h >= nh) break;
                const uint32_t c = (h == 0 ? cnt0 : cnt1) + js;
                const uint64_t qd = dQ0 + (uint64_t)(h * (SM::QH_BYTES >> 4));
                const uint32_t sc = tmem + 256u * h + kUmS0 + 64u * (c & 1);
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks)
                  umma_f16(sc, qd + (uint64_t)(((ks >> 2) * (128 * 128) + 32 * (ks & 3)) >> 4),
                           kd + (uint64_t)(((ks >> 2) * (64 * 128) + 32 * (ks & 3)) >> 4), idS,
                           ks > 0 ? 1u : 0u);
                umma_commit(bar(SM::B_SF + 2 * h + (c & 1)));
              }
              ++js;
              progressed = true;
            }
          }
          if (jp < js && mbar_try_wait(bar(SM::B_PF), (cnt0 + jp) & 1) &&
              (nh < 2 || mbar_try_wait(bar(SM::B_PF + 1), (cnt1 + jp) & 1))) {
            tc_fence_after();
            const uint32_t st = (J + jp) % kUmNF;
            issue_pv(0, st, jp == 0);
            if (nh > 1) issue_pv(1, st, jp == 0);
            umma_commit(bar(SM::B_KE + st));  // K/V stage free
            ++jp;
            progressed = true;
          }
          if (progressed) {
            spins = 0;
            idle_since = 0;
          } else if ((++spins & 63u) == 0) {  // bounded: no progress within the pool's wait limit
            const uint64_t now = globaltimer();
            if (idle_since == 0) idle_since = now;
            if (((now - idle_since) >> 10) > wait_limit_units(cta_abort)) {
              *cta_abort = 1;
              atomicOr(p.err, kErrTimeout);
              break;
            }
          }
        }
        cnt0 += (uint32_t)n;
        if (nh > 1) cnt1 += (uint32_t)n;
        J += (uint32_t)n;
      }
      // every MMA has completed before the tensor memory is released
      umma_commit(bar(SM::B_FIN));
      mbar_wait(bar(SM::B_FIN), 0, cta_abort, p.err);
    }
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kUmSoftmaxRegs));
    // ---------------- softmax / epilogue: half h, thread t = its query row t ----------------
    const int h = warp >> 2;
    const int t = tid & 127;
    const int row = 128 * h + t;
    const uint32_t lane_addr = tmem + 256u * h + ((uint32_t)((warp & 3) * 32) << 16);
    const int gq = p.g;
    uint32_t cnt = 0;
    for (int it = it0; it < it1; ++it) {
      const ShItem item = p.sh_items[it];
      const int n = item.sb_end - item.sb_begin;
      if (128 * h >= item.n_rows) continue;  // this half has no rows in the item
      // ---- this row's query -> the half's Q tile (K-major SW128, 128 rows) ----
      {
        uint8_t* qs = smem + SM::Q_OFF + h * SM::QH_BYTES;
        int64_t qoff = -1;
        if (row < item.n_rows) {
          const int mem = row / gq, jq = row - mem * gq;
          const int64_t qrow = p.units[p.sh_members[item.mem_off + mem]].qo_row;
          qoff = (qrow * p.Hq + (int64_t)item.h * gq + jq) * D;
        }
#pragma unroll 4
        for (int c = 0; c < D / 8; ++c) {
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (qoff >= 0) {
            v = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.q) + qoff) + c);
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
          *reinterpret_cast<uint4*>(qs + sw128_off(128, t, c)) = v;
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(SM::B_QF + h));
      }
      float m = -INFINITY, l = 0.f;
      uint8_t* pb = smem + SM::P_OFF + h * SM::P_BYTES;
      for (int j = 0; j < n; ++j) {
        const uint32_t c = cnt + j;
        mbar_wait(bar(SM::B_SF + 2 * h + (c & 1)), (c >> 1) & 1, cta_abort, p.err);
        tc_fence_after();
        float s0[32], s1[32];
        tmem_ld32(lane_addr + kUmS0 + 64u * (c & 1), s0);
        tmem_ld32(lane_addr + kUmS0 + 64u * (c & 1) + 32u, s1);
        // The scale enters the exponent through one fma per score; the max
        // is taken unscaled (scaling by sc > 0 keeps the order and rounds
        // monotonically, so max(s) * sc == max(s * sc)). A non-positive
        // scale is applied up front instead.
        float sc = p.scale_log2;
        if (!(sc > 0.f)) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            s0[i] *= sc;
            s1[i] *= sc;
          }
          sc = 1.f;
        }
        if (item.causal >= 0) {  // tokens after this row's own position
          const int pos0 = (item.sb_begin + j) * 64;
          const int lim = item.causal + row / gq - pos0;  // last visible token in this tile
          if (lim < 63) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              if (i > lim) s0[i] = -INFINITY;
              if (32 + i > lim) s1[i] = -INFINITY;
            }
          }
        }
        const float mx = max64(s0, s1) * sc;
        // O_h and P_h were last used by the P·V of tile c-1: wait for it only
        // where they are touched (rare O rescale, then the P write)
        bool pv_done = j == 0;
        if (j == 0) {
          m = mx;  // O is overwritten by this item's first P·V
        } else {
          const bool grow = mx > m + 8.f || (m == -INFINITY && mx > -INFINITY);
          if (__any_sync(0xffffffffu, grow)) {
            mbar_wait(bar(SM::B_PD + h), (c - 1) & 1, cta_abort, p.err);
            tc_fence_after();
            pv_done = true;
            const float mn = grow ? mx : m;
            const float al = m == -INFINITY ? 0.f : exp2f(m - mn);
            m = mn;
            l *= al;
#pragma unroll 1
            for (int cc = 0; cc < D / 32; ++cc) {
              float o[32];
              tmem_ld32(lane_addr + 32u * cc, o);
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] *= al;
              tmem_st32(lane_addr + 32u * cc, o);
            }
          }
        }
        float ps[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) ps[k] = 0.f;
        // a row that has seen no visible token yet (causal) keeps m = -inf
        const float nb = m == -INFINITY ? 0.f : -m;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          s0[i] = ex2_ftz(fmaf(s0[i], sc, nb));
          s1[i] = ex2_ftz(fmaf(s1[i], sc, nb));
          ps[i & 7] += s0[i] + s1[i];
        }
        l += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
        if (!pv_done) mbar_wait(bar(SM::B_PD + h), (c - 1) & 1, cta_abort, p.err);
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          const float* src = cc < 4 ? s0 + 8 * cc : s1 + 8 * (cc - 4);
          uint4 w;
          w.x = f2h2(src[0], src[1]);
          w.y = f2h2(src[2], src[3]);
          w.z = f2h2(src[4], src[5]);
          w.w = f2h2(src[6], src[7]);
          *reinterpret_cast<uint4*>(pb + sw128_off(128, t, cc)) = w;
        }
        fence_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar(SM::B_PF + h));
      }
      if (n > 0) {
        // ---- epilogue: O row -> partial record `slot` of the member's unit ----
        mbar_wait(bar(SM::B_PD + h), (cnt + n - 1) & 1, cta_abort, p.err);
        tc_fence_after();
        float* part = nullptr;
        int jq = 0;
        const AttnUnit* un = nullptr;
        if (row < item.n_rows) {
          const int mem = row / gq;
          jq = row - mem * gq;
          un = p.units + p.sh_members[item.mem_off + mem];
          part = p.partials +
                 ((int64_t)(un->first_split + item.slot) * Hkv + item.h) * partial_floats(D);
        }
#pragma unroll 1
        for (int cc = 0; cc < D / 32; ++cc) {
          float o[32];
          tmem_ld32(lane_addr + 32u * cc, o);
          if (part) {
            float4* dst = reinterpret_cast<float4*>(part + 16 + jq * D + 32 * cc);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
          }
        }
        if (part) {
          part[jq] = m;
          part[8 + jq] = l;
          if (item.slot == 0)
            for (int sl = item.n_frag; sl < p.n_pslots; ++sl) {
              float* e =
                  p.partials + ((int64_t)(un->first_split + sl) * Hkv + item.h) * partial_floats(D);
              e[jq] = -INFINITY;
              e[8 + jq] = 0.f;
            }
        }
        tc_fence_before();
      }
      cnt += (uint32_t)n;
    }
  }
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, kUmCols);
  }
}

template <int D, int NG>
cudaError_t launch_um(const AttnParams& p, cudaStream_t stream) {
  using SM = UmSmem<D, NG>;
  static_assert(SM::TOTAL <= 232448, "shared memory budget");
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    // setmaxnreg.inc waits until the released registers cover it: refuse to
    // launch a build whose register count would not balance
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, attn_shared_umma_kernel<D, NG>);
    if (e != cudaSuccess) return e;
    if (fa.numRegs * kUmThreads < 256 * kUmSoftmaxRegs + (kUmThreads - 256) * kUmOtherRegs)
      return cudaErrorInvalidConfiguration;
    e = cudaFuncSetAttribute(attn_shared_umma_kernel<D, NG>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, SM::TOTAL);
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit);
  }
  attn_shared_umma_kernel<D, NG><<<p.sh_grid, kUmThreads, SM::TOTAL, stream>>>(p);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// CTA-pair variant (tcgen05 cta_group::2). The same items, with each item's
// two 128-row halves on the two CTAs of a cluster (rank r owns rows
// [128r, 128r + 128)). One M = 256 instruction then computes both halves:
//   S = Q · K_jᵀ   (M = 256, N = 64 tokens, K = D): D/16 instructions per tile
//   O += P · V_j   (M = 256, N = D, K = 64 tokens): 4 instructions per tile
// instead of 2 × (D/16 + 4) per tile and SM, and the tensor core splits the
// B operand along N between the pair: rank r holds tokens [32r, 32r + 32) of
// the K tile and head-dim rows [rD/2, (r+1)D/2) of the V tile, so each CTA
// copies and dequantizes half of every sub-block. The MMAs are issued by one
// thread of rank 0 and read both CTAs' shared memory; each CTA's tensor
// memory receives its own rows.
//
// Per CTA, 20 warps:
//   - warps 0-7: softmax, thread = (row t = 32 (w % 4) + lane, column half
//     w / 4): 32 scores per tile, the row max exchanged with the partner
//     thread through shared memory (named barrier of the two warps);
//   - warp 8: tensor memory (both CTAs, cta_group::2); rank 0 lane 0 issues;
//   - warp 9: bulk copies of this CTA's half of each raw sub-block;
//   - warps 10-19: dequantize that half into the K / V half tiles.
// Cross-CTA signals: the dequantizers and the softmax warps of both CTAs
// arrive on rank 0's K/V-full, P-full and Q-full barriers (remote arrive,
// release at cluster scope); rank 0's commits arrive on both CTAs' S-full,
// P·V-done, K/V-free and final barriers (tcgen05.commit to the CTA mask
// 0b11); every wait on a barrier that the other CTA arrives on acquires at
// cluster scope. The kernel has no early exit after its first cluster
// barrier: every thread reaches the closing one, after which the tensor
// memory is released. Waits are bounded as in the one-CTA kernel.
constexpr int kPrNF = 5;           // K/V half-tile stages
constexpr int kPrNR = 4;           // raw half-sub-block stages
constexpr uint32_t kPrCols = 256;  // O at [0, D); S double buffer at D and D + 64

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// arrive on the mbarrier at the same offset in CTA `rank` of the cluster
__device__ __forceinline__ void mbar_arrive_at(uint32_t bar, uint32_t rank) {
  asm volatile(
      "{\n\t.reg .b32 ra;\n\t"
      "mapa.shared::cluster.u32 ra, %0, %1;\n\t"
      "mbarrier.arrive.release.cluster.shared::cluster.b64 _, [ra];\n\t}" ::"r"(bar),
      "r"(rank)
      : "memory");
}
__device__ __forceinline__ uint32_t mbar_try_wait_cl(uint32_t bar, uint32_t phase) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(phase)
      : "memory");
  return done;
}
// bounded wait on a barrier that the other CTA of the pair arrives on
__device__ bool mbar_wait_cl(uint32_t bar, uint32_t phase, volatile int* cta_abort, int* err) {
  if (mbar_try_wait_cl(bar, phase)) return true;
  const uint32_t limit = wait_limit_units(cta_abort);
  const uint64_t t0 = globaltimer();
  for (;;) {
    for (int k = 0; k < 16; ++k)
      if (mbar_try_wait_cl(bar, phase)) return true;
    if (((globaltimer() - t0) >> 10) > limit) {
      *cta_abort = 1;
      atomicOr(err, kErrTimeout);
      return false;
    }
  }
}
__device__ __forceinline__ void tmem_alloc2(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void umma2_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrives on the mbarrier at this offset in both CTAs of the pair once every
// MMA this thread issued so far completed
__device__ __forceinline__ void umma2_commit_both(uint32_t bar) {
  const uint16_t both = 3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
      "[%0], %1;" ::"r"(bar),
      "h"(both)
      : "memory");
}
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

template <int D, int NG>
struct PrSmem {
  using SG = SubGeom<D, NG>;
  static_assert(SG::T == 64, "one 64-token sub-block per tile");
  static constexpr int Q_BYTES = 128 * D * 2;         // this CTA's 128 rows
  static constexpr int P_BYTES = 128 * 64 * 2;
  static constexpr int KH_BYTES = 32 * D * 2;         // K half tile: 32 tokens x D
  static constexpr int VH_BYTES = (D / 2) * 64 * 2;   // V half tile: D/2 rows x 64 tokens
  static constexpr int KV_STAGE = KH_BYTES + VH_BYTES;
  static constexpr int RK_BYTES = 32 * D;             // raw K codes of the 32 tokens
  static constexpr int RV_BYTES = (D / 2) * 64;       // raw V codes of the D/2 rows
  static constexpr int RM_BYTES = 8 * NG * 64;        // all scales / zeros [4][NG][64] f16
  static constexpr int RAW_STAGE = RK_BYTES + RV_BYTES + RM_BYTES;
  static constexpr int Q_OFF = 0;
  static constexpr int P_OFF = Q_OFF + Q_BYTES;
  static constexpr int KV_OFF = P_OFF + P_BYTES;
  static constexpr int RAW_OFF = KV_OFF + kPrNF * KV_STAGE;
  static constexpr int XM_OFF = RAW_OFF + kPrNR * RAW_STAGE;  // row max exchange [2][2][128] f32
  static constexpr int XL_OFF = XM_OFF + 2 * 2 * 128 * 4;      // row sum exchange [2][128] f32
  static constexpr int BAR_OFF = XL_OFF + 2 * 128 * 4;
  // raw full / empty [NR], K/V full / free [NF], S full [2], P full, P·V
  // done, Q full, final. K/V full, P full and Q full are used in rank 0 only.
  static constexpr int B_RF = 0, B_RE = kPrNR, B_KF = 2 * kPrNR, B_KE = 2 * kPrNR + kPrNF,
                       B_SF = 2 * kPrNR + 2 * kPrNF, B_PF = B_SF + 2, B_PD = B_PF + 1,
                       B_QF = B_PD + 1, B_FIN = B_QF + 1, NBAR = B_FIN + 1;
  static constexpr int MISC_OFF = BAR_OFF + NBAR * 8;  // tmem address, abort flag, wait limit
  static constexpr int TOTAL = MISC_OFF + 16;
  static_assert(Q_BYTES % 1024 == 0 && P_BYTES % 1024 == 0 && KH_BYTES % 1024 == 0 &&
                    KV_STAGE % 1024 == 0 && RAW_STAGE % 16 == 0 && RK_BYTES % 16 == 0,
                "alignment");
};

// This CTA's half of one raw sub-block -> f16 K half tile [32 tok][D] and V
// half tile [D/2][64 tok], SW128 K-major; values f16_rn(f16_rn(code * scale)
// + zero) (QuantizedKVCache.swift:200-204), as um_dequant.
template <int D, int NG>
__device__ __forceinline__ void pr_dequant(const uint8_t* __restrict__ raw, uint8_t* __restrict__ kt,
                                           uint8_t* __restrict__ vt, int rank, int t0) {
  using SM = PrSmem<D, NG>;
  constexpr int G = D / NG;
  constexpr int NDT = kUmDeqWarps * 32;
  constexpr int NK = 32 * (D / 16), NV = (D / 2) * 4;  // 16-element items
  constexpr int KI = (NK + NDT - 1) / NDT, VI = (NV + NDT - 1) / NDT;
  constexpr int MB = SM::RK_BYTES + SM::RV_BYTES;
  auto meta = [](int a, int gi, int t) { return MB + ((a * NG + gi) * 64 + t) * 2; };
  uint4 kw[KI];
  uint32_t ks[KI], kz[KI];
#pragma unroll
  for (int k = 0; k < KI; ++k) {
    const int i = t0 + k * NDT;
    if (i < NK) {
      const int t = i / (D / 16), c = i % (D / 16);
      const int pc = D >= 128 ? (c ^ ((t & 1) << 2)) : c;  // row parity = token parity
      kw[k] = *reinterpret_cast<const uint4*>(raw + t * D + pc * 16);
      ks[k] = *reinterpret_cast<const uint16_t*>(raw + meta(0, (16 * c) / G, 32 * rank + t));
      kz[k] = *reinterpret_cast<const uint16_t*>(raw + meta(1, (16 * c) / G, 32 * rank + t));
    }
  }
  uint4 vw[VI], vs[VI][2], vz[VI][2];
#pragma unroll
  for (int k = 0; k < VI; ++k) {
    const int i = t0 + k * NDT;
    if (i < NV) {
      const int d = i >> 2, c = i & 3, gi = ((D / 2) * rank + d) / G;
      vw[k] = *reinterpret_cast<const uint4*>(raw + SM::RK_BYTES + d * 64 + c * 16);
      vs[k][0] = *reinterpret_cast<const uint4*>(raw + meta(2, gi, 16 * c));
      vs[k][1] = *reinterpret_cast<const uint4*>(raw + meta(2, gi, 16 * c + 8));
      vz[k][0] = *reinterpret_cast<const uint4*>(raw + meta(3, gi, 16 * c));
      vz[k][1] = *reinterpret_cast<const uint4*>(raw + meta(3, gi, 16 * c + 8));
    }
  }
#pragma unroll
  for (int k = 0; k < KI; ++k) {
    const int i = t0 + k * NDT;
    if (i < NK) {
      const int t = i / (D / 16), c = i % (D / 16);
      const uint32_t s2 = ks[k] | (ks[k] << 16), z2 = kz[k] | (kz[k] << 16);
      const uint32_t s8[8] = {s2, s2, s2, s2, s2, s2, s2, s2};
      const uint32_t z8[8] = {z2, z2, z2, z2, z2, z2, z2, z2};
      const bool fast = small2(s2) == 0;
      *reinterpret_cast<uint4*>(kt + sw128_off(32, t, 2 * c)) = deq16(kw[k], s8, z8, fast, false);
      *reinterpret_cast<uint4*>(kt + sw128_off(32, t, 2 * c + 1)) = deq16(kw[k], s8, z8, fast, true);
    }
  }
#pragma unroll
  for (int k = 0; k < VI; ++k) {
    const int i = t0 + k * NDT;
    if (i < NV) {
      const int d = i >> 2, c = i & 3;
      const uint32_t s8[8] = {vs[k][0].x, vs[k][0].y, vs[k][0].z, vs[k][0].w,
                              vs[k][1].x, vs[k][1].y, vs[k][1].z, vs[k][1].w};
      const uint32_t z8[8] = {vz[k][0].x, vz[k][0].y, vz[k][0].z, vz[k][0].w,
                              vz[k][1].x, vz[k][1].y, vz[k][1].z, vz[k][1].w};
      const bool fast = (small2(s8[0]) | small2(s8[1]) | small2(s8[2]) | small2(s8[3]) |
                         small2(s8[4]) | small2(s8[5]) | small2(s8[6]) | small2(s8[7])) == 0;
      *reinterpret_cast<uint4*>(vt + sw128_off(D / 2, d, 2 * c)) = deq16(vw[k], s8, z8, fast, false);
      *reinterpret_cast<uint4*>(vt + sw128_off(D / 2, d, 2 * c + 1)) = deq16(vw[k], s8, z8, fast, true);
    }
  }
}

__device__ __forceinline__ float max32(const float (&a)[32]) {
  float m[8];
#pragma unroll
  for (int k = 0; k < 8; ++k)
    m[k] = fmaxf(fmaxf(a[4 * k], a[4 * k + 1]), fmaxf(a[4 * k + 2], a[4 * k + 3]));
#pragma unroll
  for (int k = 0; k < 4; ++k) m[k] = fmaxf(m[k], m[k + 4]);
  return fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
}

template <int D, int NG>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kUmThreads, 1)
    attn_shared_pair_kernel(AttnParams p) {
  using SM = PrSmem<D, NG>;
  using SG = SubGeom<D, NG>;
  constexpr int SB = SG::SB;
  extern __shared__ __align__(1024) uint8_t smem[];
  // Both CTAs run the same launch configuration, so both see the same base
  // and take this exit together (before any cluster barrier).
  const uint32_t sbase = smem_u32(smem);
  if (sbase & 1023u) {
    if (threadIdx.x == 0) atomicOr(p.err, kErrBadArg);
    return;
  }
  auto bar = [&](int i) { return sbase + SM::BAR_OFF + 8u * (uint32_t)i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + SM::MISC_OFF);
  volatile int* cta_abort = reinterpret_cast<volatile int*>(smem + SM::MISC_OFF + 4);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  if (tid == 0) {
    for (int s = 0; s < kPrNR; ++s) {
      mbar_init(bar(SM::B_RF + s), 1);            // copy issuer arrive + tx bytes
      mbar_init(bar(SM::B_RE + s), kUmDeqWarps);  // this CTA's dequantizer warps
    }
    for (int s = 0; s < kPrNF; ++s) {
      mbar_init(bar(SM::B_KF + s), 2 * kUmDeqWarps);  // both CTAs' dequantizers (rank 0)
      mbar_init(bar(SM::B_KE + s), 1);                // MMA commit
    }
    mbar_init(bar(SM::B_SF), 1);
    mbar_init(bar(SM::B_SF + 1), 1);
    mbar_init(bar(SM::B_PF), 16);  // both CTAs' 8 softmax warps (rank 0)
    mbar_init(bar(SM::B_PD), 1);
    mbar_init(bar(SM::B_QF), 16);
    mbar_init(bar(SM::B_FIN), 1);
    init_wait_state(cta_abort, p.wait_us);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 8) {
    tmem_alloc2(smem_u32(tmem_slot), kPrCols);
    tmem_relinquish2();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the pair's barriers and tensor memory exist before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int pair = blockIdx.x >> 1;
  const int it0 = p.sh_cta_off[pair], it1 = p.sh_cta_off[pair + 1];
  const int Hkv = p.Hkv;

  if (warp >= 8) {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kUmOtherRegs));
  if (warp == 9) {
    // ---------------- copy issuer: this CTA's half of each sub-block ----------------
    if (lane == 0) {
      const int64_t blk_stride = (int64_t)p.L * Hkv * p.page_bytes;
      const int64_t k_off = (int64_t)32 * rank * D;
      const int64_t v_off = SG::VOFF + (int64_t)(D / 2) * rank * 64;
      uint32_t J = 0;
      for (int it = it0; it < it1; ++it) {
        const ShItem item = p.sh_items[it];
        const int32_t* bt = p.bt + (int64_t)item.leader * p.bt_stride;
        const uint8_t* page = p.pool + ((int64_t)item.layer * Hkv + item.h) * p.page_bytes;
        for (int j = item.sb_begin; j < item.sb_end; ++j, ++J) {
          const int b = __ldg(bt + j / SG::SPB);
          const uint32_t s = J % kPrNR;
          if (J >= (uint32_t)kPrNR)
            mbar_wait(bar(SM::B_RE + s), ((J / kPrNR) - 1) & 1, cta_abort, p.err);
          const uint8_t* src = page + (int64_t)b * blk_stride + (int64_t)(j % SG::SPB) * SB;
          const uint32_t dst = sbase + SM::RAW_OFF + s * SM::RAW_STAGE;
          mbar_expect_tx(bar(SM::B_RF + s), SM::RAW_STAGE);
          bulk_g2s(dst, src + k_off, SM::RK_BYTES, bar(SM::B_RF + s));
          bulk_g2s(dst + SM::RK_BYTES, src + v_off, SM::RV_BYTES, bar(SM::B_RF + s));
          bulk_g2s(dst + SM::RK_BYTES + SM::RV_BYTES, src + SG::META, SM::RM_BYTES,
                   bar(SM::B_RF + s));
        }
      }
      for (uint32_t k = J > (uint32_t)kPrNR ? J - kPrNR : 0; k < J; ++k)
        mbar_wait(bar(SM::B_RF + k % kPrNR), (k / kPrNR) & 1, cta_abort, p.err);
    }
  } else if (warp >= 10) {
    // ---------------- dequantizers ----------------
    const int t0 = tid - 10 * 32;
    uint32_t J = 0;
    for (int it = it0; it < it1; ++it) {
      const ShItem item = p.sh_items[it];
      for (int j = item.sb_begin; j < item.sb_end; ++j, ++J) {
        const uint32_t rs = J % kPrNR, fs = J % kPrNF;
        mbar_wait(bar(SM::B_RF + rs), (J / kPrNR) & 1, cta_abort, p.err);
        if (J >= (uint32_t)kPrNF)
          mbar_wait_cl(bar(SM::B_KE + fs), ((J / kPrNF) - 1) & 1, cta_abort, p.err);
        uint8_t* kt = smem + SM::KV_OFF + fs * SM::KV_STAGE;
        pr_dequant<D, NG>(smem + SM::RAW_OFF + rs * SM::RAW_STAGE, kt, kt + SM::KH_BYTES, (int)rank,
                          t0);
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(bar(SM::B_RE + rs));
          mbar_arrive_at(bar(SM::B_KF + fs), 0);
        }
      }
    }
  } else if (rank == 0) {
    // ---------------- MMA issuer (rank 0, warp 8) ----------------
    if (lane == 0) {
      constexpr uint32_t idS = umma_idesc(256, 64), idO = umma_idesc(256, D);
      uint32_t cnt = 0, qn = 0, J = 0;
      const uint64_t dK0 = sw128_desc(sbase + SM::KV_OFF);
      const uint64_t dV0 = sw128_desc(sbase + SM::KV_OFF + SM::KH_BYTES);
      const uint64_t dQ0 = sw128_desc(sbase + SM::Q_OFF);
      const uint64_t dP0 = sw128_desc(sbase + SM::P_OFF);
      for (int it = it0; it < it1; ++it) {
        const ShItem item = p.sh_items[it];
        const int n = item.sb_end - item.sb_begin;
        mbar_wait_cl(bar(SM::B_QF), qn & 1, cta_abort, p.err);
        ++qn;
        tc_fence_after();
        int js = 0, jp = 0;
        uint32_t spins = 0;
        uint64_t idle_since = 0;
        while (jp < n) {
          bool progressed = false;
          if (js < n && js <= jp + 1) {
            const uint32_t Jc = J + js, st = Jc % kPrNF;
            if (mbar_try_wait_cl(bar(SM::B_KF + st), (Jc / kPrNF) & 1)) {
              tc_fence_after();
              const uint32_t c = cnt + js;
              const uint64_t kd = dK0 + (uint64_t)(st * (SM::KV_STAGE >> 4));
              const uint32_t sc = tmem + (uint32_t)D + 64u * (c & 1);
#pragma unroll
              for (int ks = 0; ks < D / 16; ++ks)
                umma2_f16(sc, dQ0 + (uint64_t)(((ks >> 2) * (128 * 128) + 32 * (ks & 3)) >> 4),
                          kd + (uint64_t)(((ks >> 2) * (32 * 128) + 32 * (ks & 3)) >> 4), idS,
                          ks > 0 ? 1u : 0u);
              umma2_commit_both(bar(SM::B_SF + (c & 1)));
              ++js;
              progressed = true;
            }
          }
          if (jp < js && mbar_try_wait_cl(bar(SM::B_PF), (cnt + jp) & 1)) {
            tc_fence_after();
            const uint32_t st = (J + jp) % kPrNF;
            const uint64_t vd = dV0 + (uint64_t)(st * (SM::KV_STAGE >> 4));
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              umma2_f16(tmem, dP0 + (uint64_t)(2 * ks), vd + (uint64_t)(2 * ks), idO,
                        (jp > 0 || ks > 0) ? 1u : 0u);
            umma2_commit_both(bar(SM::B_PD));       // O updated, P free
            umma2_commit_both(bar(SM::B_KE + st));  // K/V stage free in both CTAs
            ++jp;
            progressed = true;
          }
          if (progressed) {
            spins = 0;
            idle_since = 0;
          } else if ((++spins & 63u) == 0) {  // bounded: no progress within the pool's wait limit
            const uint64_t now = globaltimer();
            if (idle_since == 0) idle_since = now;
            if (((now - idle_since) >> 10) > wait_limit_units(cta_abort)) {
              *cta_abort = 1;
              atomicOr(p.err, kErrTimeout);
              break;
            }
          }
        }
        cnt += (uint32_t)n;
        J += (uint32_t)n;
      }
      // every MMA has completed (in both CTAs) before the tensor memory is released
      umma2_commit_both(bar(SM::B_FIN));
      mbar_wait_cl(bar(SM::B_FIN), 0, cta_abort, p.err);
    }
  } else {
    // rank 1, warp 8: the MMAs that write this CTA's tensor memory have
    // completed before it is released
    if (lane == 0) mbar_wait_cl(bar(SM::B_FIN), 0, cta_abort, p.err);
  }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kUmSoftmaxRegs));
    // ---------------- softmax / epilogue: row t, column half ch ----------------
    const int ch = warp >> 2;
    const int t = ((warp & 3) << 5) | lane;
    const int row = 128 * (int)rank + t;  // row of the item
    const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t nbar = 1 + (uint32_t)(warp & 3);  // named barrier of warps w and w ^ 4
    float* xm = reinterpret_cast<float*>(smem + SM::XM_OFF);
    float* xl = reinterpret_cast<float*>(smem + SM::XL_OFF);
    const int gq = p.g;
    uint8_t* pb = smem + SM::P_OFF;
    uint32_t cnt = 0;
    for (int it = it0; it < it1; ++it) {
      const ShItem item = p.sh_items[it];
      const int n = item.sb_end - item.sb_begin;
      // ---- this row's query, column half ch -> the Q tile (K-major SW128) ----
      {
        uint8_t* qs = smem + SM::Q_OFF;
        int64_t qoff = -1;
        if (row < item.n_rows) {
          const int mem = row / gq, jq = row - mem * gq;
          const int64_t qrow = p.units[p.sh_members[item.mem_off + mem]].qo_row;
          qoff = (qrow * p.Hq + (int64_t)item.h * gq + jq) * D;
        }
#pragma unroll 4
        for (int c = ch * (D / 16); c < (ch + 1) * (D / 16); ++c) {
          uint4 v = make_uint4(0u, 0u, 0u, 0u);
          if (qoff >= 0) {
            v = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.q) + qoff) + c);
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
          *reinterpret_cast<uint4*>(qs + sw128_off(128, t, c)) = v;
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive_at(bar(SM::B_QF), 0);
      }
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < n; ++j) {
        const uint32_t c = cnt + j;
        mbar_wait_cl(bar(SM::B_SF + (c & 1)), (c >> 1) & 1, cta_abort, p.err);
        tc_fence_after();
        float s[32];
        tmem_ld32(lane_addr + (uint32_t)D + 64u * (c & 1) + 32u * (uint32_t)ch, s);
        float sc = p.scale_log2;
        if (!(sc > 0.f)) {
#pragma unroll
          for (int i = 0; i < 32; ++i) s[i] *= sc;
          sc = 1.f;
        }
        if (item.causal >= 0) {  // tokens after this row's own position
          const int pos0 = (item.sb_begin + j) * 64 + 32 * ch;
          const int lim = item.causal + row / gq - pos0;  // last visible column of this half
          if (lim < 31) {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (i > lim) s[i] = -INFINITY;
          }
        }
        // the row max over both column halves: each thread posts its half's
        // max, the two warps of the row meet at their named barrier
        float mx = max32(s) * sc;
        float* xp = xm + (c & 1) * 256;
        xp[ch * 128 + t] = mx;
        named_sync(nbar, 64);
        mx = fmaxf(mx, xp[(ch ^ 1) * 128 + t]);
        // both threads of a row hold the same m and mx, so they take the
        // same branch (and __any_sync agrees between the row's two warps)
        bool pv_done = j == 0;
        if (j == 0) {
          m = mx;
        } else {
          const bool grow = mx > m + 8.f || (m == -INFINITY && mx > -INFINITY);
          if (__any_sync(0xffffffffu, grow)) {
            mbar_wait_cl(bar(SM::B_PD), (c - 1) & 1, cta_abort, p.err);
            tc_fence_after();
            pv_done = true;
            const float mn = grow ? mx : m;
            const float al = m == -INFINITY ? 0.f : exp2f(m - mn);
            m = mn;
            l *= al;
#pragma unroll 1
            for (int cc = 0; cc < D / 64; ++cc) {
              const uint32_t oa = lane_addr + (uint32_t)(ch * (D / 2) + 32 * cc);
              float o[32];
              tmem_ld32(oa, o);
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] *= al;
              tmem_st32(oa, o);
            }
          }
        }
        float ps[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) ps[k] = 0.f;
        const float nb = m == -INFINITY ? 0.f : -m;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          s[i] = ex2_ftz(fmaf(s[i], sc, nb));
          ps[i & 7] += s[i];
        }
        l += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
        if (!pv_done) mbar_wait_cl(bar(SM::B_PD), (c - 1) & 1, cta_abort, p.err);
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          uint4 w;
          w.x = f2h2(s[8 * cc + 0], s[8 * cc + 1]);
          w.y = f2h2(s[8 * cc + 2], s[8 * cc + 3]);
          w.z = f2h2(s[8 * cc + 4], s[8 * cc + 5]);
          w.w = f2h2(s[8 * cc + 6], s[8 * cc + 7]);
          *reinterpret_cast<uint4*>(pb + sw128_off(128, t, 4 * ch + cc)) = w;
        }
        fence_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_at(bar(SM::B_PF), 0);
      }
      if (n > 0) {
        // ---- epilogue: O row (this thread's D/2 columns) -> partial record ----
        mbar_wait_cl(bar(SM::B_PD), (cnt + n - 1) & 1, cta_abort, p.err);
        tc_fence_after();
        xl[ch * 128 + t] = l;
        named_sync(nbar, 64);
        const float lt = l + xl[(ch ^ 1) * 128 + t];
        named_sync(nbar, 64);  // the buffer is free for the next item
        float* part = nullptr;
        int jq = 0;
        const AttnUnit* un = nullptr;
        if (row < item.n_rows) {
          const int mem = row / gq;
          jq = row - mem * gq;
          un = p.units + p.sh_members[item.mem_off + mem];
          part = p.partials +
                 ((int64_t)(un->first_split + item.slot) * Hkv + item.h) * partial_floats(D);
        }
#pragma unroll 1
        for (int cc = 0; cc < D / 64; ++cc) {
          const int col = ch * (D / 2) + 32 * cc;
          float o[32];
          tmem_ld32(lane_addr + (uint32_t)col, o);
          if (part) {
            float4* dst = reinterpret_cast<float4*>(part + 16 + jq * D + col);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
          }
        }
        if (part && ch == 0) {
          part[jq] = m;
          part[8 + jq] = lt;
          if (item.slot == 0)
            for (int sl = item.n_frag; sl < p.n_pslots; ++sl) {
              float* e =
                  p.partials + ((int64_t)(un->first_split + sl) * Hkv + item.h) * partial_floats(D);
              e[jq] = -INFINITY;
              e[8 + jq] = 0.f;
            }
        }
        tc_fence_before();
      }
      cnt += (uint32_t)n;
    }
  }
  __syncthreads();
  cluster_sync_all();  // no cross-CTA access remains once both CTAs pass this
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc2(tmem, kPrCols);
  }
}

template <int D, int NG>
cudaError_t configure_pair() {
  using SM = PrSmem<D, NG>;
  static_assert(SM::TOTAL <= 232448, "shared memory budget");
  static std::atomic<uint64_t> configured{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (!(configured.load() & bit)) {
    cudaFuncAttributes fa;
    e = cudaFuncGetAttributes(&fa, attn_shared_pair_kernel<D, NG>);
    if (e != cudaSuccess) return e;
    if (fa.numRegs * kUmThreads < 256 * kUmSoftmaxRegs + (kUmThreads - 256) * kUmOtherRegs)
      return cudaErrorInvalidConfiguration;
    e = cudaFuncSetAttribute(attn_shared_pair_kernel<D, NG>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, SM::TOTAL);
    if (e != cudaSuccess) return e;
    configured.fetch_or(bit);
  }
  return cudaSuccess;
}

template <int D, int NG>
cudaError_t launch_pair(const AttnParams& p, cudaStream_t stream) {
  using SM = PrSmem<D, NG>;
  cudaError_t e = configure_pair<D, NG>();
  if (e != cudaSuccess) return e;
  attn_shared_pair_kernel<D, NG><<<2 * p.sh_grid, kUmThreads, SM::TOTAL, stream>>>(p);
  return cudaGetLastError();
}

// Clusters of two CTAs of the pair kernel resident at once on the current device.
template <int D, int NG>
int pair_capacity() {
  using SM = PrSmem<D, NG>;
  if (configure_pair<D, NG>() != cudaSuccess) return 0;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * (sms / 2)));
  cfg.blockDim = dim3(kUmThreads);
  cfg.dynamicSmemBytes = SM::TOTAL;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, attn_shared_pair_kernel<D, NG>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return clusters;
}

}  // namespace

bool shared_uses_umma(const Geom& g, int impl) {
  return (impl == KRILL_ATTN_TENSOR_CORE || impl == KRILL_ATTN_TENSOR_CORE_PAIR) && g.D <= 128;
}

int shared_pair_capacity(const Geom& g) {
  if (g.fmt != kFmtInt8) return 0;
  if (g.D == 64 && g.NG == 1) return pair_capacity<64, 1>();
  if (g.D == 128 && g.NG == 2) return pair_capacity<128, 2>();
  if (g.D == 128 && g.NG == 1) return pair_capacity<128, 1>();
  return 0;
}

cudaError_t launch_shared_umma(const Geom& g, const AttnParams& p, cudaStream_t stream) {
  if (p.sh_grid <= 0) return cudaSuccess;
  if (p.sh_pair) {
    if (g.D == 64 && g.NG == 1) return launch_pair<64, 1>(p, stream);
    if (g.D == 128 && g.NG == 2) return launch_pair<128, 2>(p, stream);
    if (g.D == 128 && g.NG == 1) return launch_pair<128, 1>(p, stream);
    return cudaErrorInvalidValue;
  }
  if (g.D == 64 && g.NG == 1) return launch_um<64, 1>(p, stream);
  if (g.D == 128 && g.NG == 2) return launch_um<128, 2>(p, stream);
  if (g.D == 128 && g.NG == 1) return launch_um<128, 1>(p, stream);
  return cudaErrorInvalidValue;
}

}  // namespace krill
