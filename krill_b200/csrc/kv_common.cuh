// kv_common.cuh — page geometry and device helpers shared by the kernels.
//
// HBM layout of one pool (one layer group on one GPU):
//   pool = blocks[num_blocks]; block = pages[num_layers][num_kv_heads];
//   page = 256 tokens = sub-blocks of T tokens (T = 64, or 32 for D = 256 so
//   that every sub-block is about 17 KB); each sub-block is one contiguous run
//   of SB = T * (2*D + 8*NG) bytes:
//     [0, T*D)             K codes, token-major rows of D bytes; for D >= 128
//                          the 16-byte chunks of odd rows are XOR-swizzled by 4
//                          so the decode kernel's shared-memory reads are
//                          bank-conflict free
//     [T*D, 2*T*D)         V codes transposed: D rows of T token bytes, so the
//                          tensor-core fragments along the token axis are
//                          contiguous bytes
//     [2*T*D, ...)         K scales, K zeros, V scales, V zeros: [NG][T] f16 each
// A sub-block is the unit one bulk (TMA) copy moves into shared memory.
//
// Raw bf16 pools (the unquantized comparison format) use the same blocks and
// pages with sub-blocks of T = 32 tokens (64 at D = 64) of T * 4 * D bytes:
//     [0, 2*T*D)           K rows, token-major bf16; the 16-byte chunks of odd
//                          rows swapped pairwise (chunk ^ 1) so the decode
//                          kernel's shared-memory reads are conflict free
//     [2*T*D, 4*T*D)       V transposed: D rows of T bf16
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace krill {

constexpr int kBlockTokens = 256;
// Tokens per sub-block for head dim D.
__host__ __device__ constexpr int sub_tokens(int D) { return D >= 256 ? 32 : 64; }
// Tokens per sub-block of a raw bf16 pool.
__host__ __device__ constexpr int sub_tokens_raw(int D) { return D >= 128 ? 32 : 64; }
// Pool formats.
constexpr int kFmtInt8 = 0;
constexpr int kFmtBf16 = 1;

struct Geom {
  int L;        // layers in the pool
  int Hkv;      // kv heads
  int Hq;       // query heads
  int g;        // Hq / Hkv
  int D;        // head dim
  int G;        // group size
  int NG;       // D / G
  int ring;     // blocks in a windowed sequence's ring; 0 = full history
  int window;   // sliding window (tokens); 0 = full history
  int quant_variant;
  int fmt;      // kFmtInt8 or kFmtBf16
  int subt;     // tokens per sub-block
  int spb;      // sub-blocks per 256-token block
  int64_t sb_bytes;
  int64_t page_bytes;
  int64_t block_bytes;
};

inline Geom make_geom(int L, int Hkv, int Hq, int D, int G, int ring, int window, int qv,
                      int fmt = kFmtInt8) {
  Geom g;
  g.L = L; g.Hkv = Hkv; g.Hq = Hq; g.g = Hq / Hkv; g.D = D; g.G = G; g.NG = D / G;
  g.ring = ring; g.window = window; g.quant_variant = qv; g.fmt = fmt;
  g.subt = fmt == kFmtBf16 ? sub_tokens_raw(D) : sub_tokens(D);
  g.spb = kBlockTokens / g.subt;
  g.sb_bytes = fmt == kFmtBf16 ? (int64_t)g.subt * 4 * D : (int64_t)g.subt * (2 * D + 8 * g.NG);
  g.page_bytes = g.sb_bytes * g.spb;
  g.block_bytes = g.page_bytes * L * Hkv;
  return g;
}

// Byte offsets inside a sub-block.
__host__ __device__ inline int64_t sb_voff(int D) { return (int64_t)sub_tokens(D) * D; }
__host__ __device__ inline int64_t sb_meta_off(int D) { return (int64_t)2 * sub_tokens(D) * D; }
// meta array a (0 = K scale, 1 = K zero, 2 = V scale, 3 = V zero), group gi, token t
__host__ __device__ inline int64_t sb_meta(int D, int NG, int a, int gi, int t) {
  return sb_meta_off(D) + ((int64_t)(a * NG + gi) * sub_tokens(D) + t) * 2;
}
// Physical byte offset of K code (token t in sub-block, element d).
__host__ __device__ inline int64_t sb_kcode(int D, int t, int d) {
  int chunk = d >> 4;
  if (D >= 128) chunk ^= (t & 1) << 2;
  return (int64_t)t * D + chunk * 16 + (d & 15);
}
__host__ __device__ inline int64_t sb_vcode(int D, int t, int d) {
  return sb_voff(D) + (int64_t)d * sub_tokens(D) + t;
}

// Raw bf16 sub-block of T tokens: byte offsets of K (token t, element d) and
// V (element d, token t).
__host__ __device__ inline int64_t raw_koff(int D, int t, int d) {
  return ((int64_t)t * D + (((d >> 3) ^ (t & 1)) << 3) + (d & 7)) * 2;
}
__host__ __device__ inline int64_t raw_voff(int D, int T, int t, int d) {
  return ((int64_t)T * D + (int64_t)d * T + t) * 2;
}

// Error flag bits written by kernels (pool-owned int, read + cleared by host).
constexpr int kErrTimeout = 1;
constexpr int kErrBadArg = 2;
// The pool's device words (int32): [0] error flag bits, [1] large-scale flag,
// [2] scratch of the peer fetch, [5] testing only: non-zero makes a wait of
// CTA 0 in the next decode launches run out.
constexpr int kDevWords = 8;
constexpr int kDevTestStall = 5;
constexpr int kDefaultWaitUs = 100000;  // 100 ms

#ifdef __CUDACC__
__device__ inline float load_in(const void* p, int64_t i, int dtype) {
  return dtype == 0 ? __half2float(reinterpret_cast<const __half*>(p)[i])
                    : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}
// Round a float to the input dtype (f16 or bf16), RN-even, back to float.
__device__ inline float round_in(float v, int dtype) {
  return dtype == 0 ? __half2float(__float2half_rn(v)) : __bfloat162float(__float2bfloat16_rn(v));
}
__device__ inline uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
#endif

}  // namespace krill
