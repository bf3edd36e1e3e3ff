// krill_oracle.cpp — CPU restatement of Krill's int8 KV-cache path.
//
// TEST INFRASTRUCTURE ONLY. This library is the parity checker for the
// CUDA product in krill_b200/; it is loaded only by tests/, by
// __graft_entry__.smoke() and by bench.py's CPU-baseline arm. The product
// never links or calls it.
//
// Parity status: PARTIALLY PINNED. The reference (Swift + mlx-swift 0.31.4,
// macOS arm64 only) cannot be built or run on Linux, and mlx is not vendored,
// so no reference output exists to pin against. What pins this restatement:
//   * the reference's own known-answer and tolerance tests, restated in
//     tests/test_oracle.py (Weyl round-trip bound of
//     Tests/KrillEngineTests/QuantizedKVCacheUnitTests.swift:17-84, LCP=5 of
//     Tests/KrillCoreTests/QuantizedPrefixCacheTests.swift:92-121, the
//     append/truncate orderings of Tests/KrillCoreTests/KVCacheTests.swift);
//   * the published FNV-1a 64 test vectors for the prefix-cache key;
//   * an independent numpy restatement of the quantizer (tests/golden/gen_golden.py).
// The SDPA values themselves are unpinned (the reference delegates to
// MLXFast.scaledDotProductAttention, whose source is not available here), so
// the oracle uses the mathematical definition in float64.
//
// Numeric recipe (reference: Sources/KrillCache/QuantizedKVCache.swift:181-204,
// MLX CPU-device semantics):
//   mn = min_d x, mx = max_d x                      (exact, input dtype)
//   d  = rn_in(mx - mn)                             (input-dtype subtract)
//   scale32 = max(f32(d) / 255.0f, 1e-8f)           (f16 / f32 array -> f32)
//   n  = f32(rn_in(x - mn)) / scale32               (f32 RN divide)
//   code = (uint8) trunc(clip(n, 0, 255))           (asType(.uint8) truncates)
//   stored scale = f16_rn(scale32), zero = f16_rn(mn)
//   dequant = f16_rn(f16_rn(f16(code) * scale) + zero)
// The reference applies this over the whole head_dim; group_size G < D applies
// the identical recipe independently to each G-wide slice (G == D is the
// reference scheme exactly).
// Variant KRILL_QUANT_F16 keeps scale and quotient in the input dtype, for the
// case where mlx-swift's MLXArray(Float) scalars were weakly typed (unverified).

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

namespace {

// ---------------------------------------------------------------- f16 / bf16
inline uint32_t f2u(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
inline float u2f(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000) << 16;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t man = h & 0x3ff;
  if (exp == 0) {
    if (man == 0) return u2f(sign);
    // subnormal: man * 2^-24
    float v = (float)man * 5.9604644775390625e-08f;
    return sign ? -v : v;
  }
  if (exp == 31) return u2f(sign | 0x7f800000u | (man << 13));
  return u2f(sign | ((exp + 112) << 23) | (man << 13));
}

// IEEE round-to-nearest-even float32 -> binary16.
uint16_t f32_to_f16(float f) {
  uint32_t x = f2u(f);
  uint16_t sign = (uint16_t)((x >> 16) & 0x8000);
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) {  // inf / nan
    return (uint16_t)(sign | 0x7c00 | (ax > 0x7f800000u ? 0x200 : 0));
  }
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00);  // rounds to inf
  if (ax < 0x38800000u) {
    // result is subnormal or zero: value = ax_float; quantum 2^-24
    float a = u2f(ax);
    // a * 2^24 rounded to nearest even integer
    float scaled = a * 16777216.0f;  // exact (power of two)
    float r = std::nearbyint(scaled);  // default rounding mode: nearest-even
    return (uint16_t)(sign | (uint16_t)r);
  }
  uint32_t exp = (ax >> 23) - 112;   // rebias 127 -> 15
  uint32_t man = ax & 0x7fffff;
  uint32_t h = (exp << 10) | (man >> 13);
  uint32_t rem = man & 0x1fff;
  if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h += 1;
  return (uint16_t)(sign | h);
}

float bf16_to_f32(uint16_t b) { return u2f((uint32_t)b << 16); }

uint16_t f32_to_bf16(float f) {
  uint32_t x = f2u(f);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40);
  uint32_t lsb = (x >> 16) & 1;
  x += 0x7fffu + lsb;
  return (uint16_t)(x >> 16);
}

inline float load_in(uint16_t v, int dtype) { return dtype == 0 ? f16_to_f32(v) : bf16_to_f32(v); }
inline float round_in(float v, int dtype) {
  return dtype == 0 ? f16_to_f32(f32_to_f16(v)) : bf16_to_f32(f32_to_bf16(v));
}
inline float round_f16(float v) { return f16_to_f32(f32_to_f16(v)); }

// One G-wide group: the reference quantizer restated step by step.
void quantize_group(const uint16_t* x, int dtype, int G, int variant, uint8_t* codes,
                    uint16_t* scale_out, uint16_t* zero_out) {
  float mn = load_in(x[0], dtype), mx = mn;
  for (int i = 1; i < G; ++i) {
    float v = load_in(x[i], dtype);
    mn = std::min(mn, v);
    mx = std::max(mx, v);
  }
  float d = round_in(mx - mn, dtype);       // QuantizedKVCache.swift:185 (maxVal - minVal)
  float scale;
  if (variant == 0) {
    scale = d / 255.0f;                     // :185  f16/bf16 array / f32 scalar -> f32
    scale = std::max(scale, 1e-8f);         // :187  maximum(scale, 1e-8)
  } else {
    scale = round_in(d / 255.0f, dtype);
    scale = std::max(scale, round_in(1e-8f, dtype));
  }
  for (int i = 0; i < G; ++i) {
    float diff = round_in(load_in(x[i], dtype) - mn, dtype);  // :192 (x - minVal)
    float n = diff / scale;                                   // :192 / safeScale
    if (variant != 0) n = round_in(n, dtype);
    n = std::min(std::max(n, 0.0f), 255.0f);                  // :193 clip(0, 255)
    codes[i] = (uint8_t)(int)n;                               // :194 asType(.uint8) truncates
  }
  *scale_out = f32_to_f16(scale);                             // :196 safeScale.asType(.float16)
  *zero_out = f32_to_f16(mn);                                 // :196 minVal.asType(.float16)
}

}  // namespace

extern "C" {

// f16/bf16 helpers exported for the tests.
uint16_t oracle_f32_to_f16(float f) { return f32_to_f16(f); }
float oracle_f16_to_f32(uint16_t h) { return f16_to_f32(h); }
uint16_t oracle_f32_to_bf16(float f) { return f32_to_bf16(f); }
float oracle_bf16_to_f32(uint16_t b) { return bf16_to_f32(b); }

// Quantize `rows` rows of D elements (dtype 0 = f16, 1 = bf16, given as bits).
// Outputs: codes [rows][D], scales/zeros [rows][D/G] as f16 bits.
// Reference: QuantizedKVCache.quantizePerHead (QuantizedKVCache.swift:181-197).
void oracle_quantize(const uint16_t* x, int dtype, int64_t rows, int D, int G, int variant,
                     uint8_t* codes, uint16_t* scales, uint16_t* zeros) {
  int ng = D / G;
  for (int64_t r = 0; r < rows; ++r)
    for (int g = 0; g < ng; ++g)
      quantize_group(x + r * D + g * G, dtype, G, variant, codes + r * D + g * G,
                     scales + r * ng + g, zeros + r * ng + g);
}

// Dequantize to f16 bits exactly as QuantizedKVCache.dequantize
// (QuantizedKVCache.swift:200-204): f16(code) * scale, then + zero, each
// rounded to f16.
void oracle_dequantize(const uint8_t* codes, const uint16_t* scales, const uint16_t* zeros,
                       int64_t rows, int D, int G, uint16_t* out) {
  int ng = D / G;
  for (int64_t r = 0; r < rows; ++r)
    for (int i = 0; i < D; ++i) {
      float s = f16_to_f32(scales[r * ng + i / G]);
      float z = f16_to_f32(zeros[r * ng + i / G]);
      float prod = round_f16((float)codes[r * D + i] * s);
      out[r * D + i] = f32_to_f16(prod + z);
    }
}

// Float64 scaled-dot-product attention for one query token with GQA:
// q [Hq][D], k/v [Hkv][L][D] (the reference's [B,H,S,D] layout, B = 1),
// out [Hq][D]. Query head h reads kv head h / (Hq / Hkv), matching MLX's GQA
// broadcast used by MLXFast.scaledDotProductAttention
// (Gemma4Model.swift:516, Attention.swift:95).
void oracle_sdpa_f64(const double* q, const double* k, const double* v, int Hq, int Hkv,
                     int64_t L, int D, double scale, double* out) {
  int grp = Hq / Hkv;
  std::vector<double> s((size_t)std::max<int64_t>(L, 1));
  for (int h = 0; h < Hq; ++h) {
    int kh = h / grp;
    const double* qh = q + (size_t)h * D;
    double m = -INFINITY;
    for (int64_t t = 0; t < L; ++t) {
      const double* kt = k + ((size_t)kh * L + t) * D;
      double acc = 0.0;
      for (int d = 0; d < D; ++d) acc += qh[d] * kt[d];
      s[t] = acc * scale;
      m = std::max(m, s[t]);
    }
    double l = 0.0;
    for (int64_t t = 0; t < L; ++t) { s[t] = std::exp(s[t] - m); l += s[t]; }
    for (int d = 0; d < D; ++d) {
      double acc = 0.0;
      for (int64_t t = 0; t < L; ++t) acc += s[t] * v[((size_t)kh * L + t) * D + d];
      out[(size_t)h * D + d] = L > 0 ? acc / l : 0.0;
    }
  }
}

// FNV-1a 64 over `n` bytes (reference: PrefixCache.cacheKey, PrefixCache.swift:526-530).
uint64_t oracle_fnv1a64(const uint8_t* data, int64_t n) {
  uint64_t h = 14695981039346656037ull;
  for (int64_t i = 0; i < n; ++i) { h ^= data[i]; h *= 1099511628211ull; }
  return h;
}

// Prefix-cache key (PrefixCache.swift:513-532): schema 3 || dtype tag ||
// modelId utf8 || 0xFF || mediaHash utf8 (if non-empty) || 0xFF || tokens as
// little-endian Int64 bytes.
uint64_t oracle_prefix_key(const int64_t* tokens, int64_t n, const char* model_id,
                           const char* media_hash, int dtype_tag) {
  std::string data;
  data.push_back((char)3);
  data.push_back((char)dtype_tag);
  data.append(model_id ? model_id : "");
  data.push_back((char)0xFF);
  if (media_hash && media_hash[0]) data.append(media_hash);
  data.push_back((char)0xFF);
  data.append(reinterpret_cast<const char*>(tokens), (size_t)n * 8);
  return oracle_fnv1a64(reinterpret_cast<const uint8_t*>(data.data()), (int64_t)data.size());
}

// ---------------------------------------------------------------------------
// CPU baseline: the reference's per-step dataflow (QuantizedKVCache.update,
// QuantizedKVCache.swift:49-75, then SDPA) for a batch of sequences:
//   1. quantize the new token's K and V per head;
//   2. concatenate onto the stored u8 codes and f16 scales/zeros (a full copy
//      of all six tensors, as `concatenated` does);
//   3. dequantize the whole cache to f16;
//   4. SDPA with GQA in float32, f16 output.
// State lives in caller-owned host buffers per (seq, layer) in the reference
// [Hkv][S][D] layout with capacity `cap` rows; the concat is restated as a
// copy into a second buffer (ping-pong) to keep the O(L) copy the reference
// pays. Work is split over (seq, layer) across `threads` std::threads.
struct BaselineCache {
  int Hkv, D, G, ng;
  int64_t len, cap;
  std::vector<uint8_t> kc, vc, kc2, vc2;
  std::vector<uint16_t> ks, kz, vs, vz, ks2, kz2, vs2, vz2;
};

void* oracle_baseline_create(int Hkv, int D, int G, int64_t len, int64_t cap, uint64_t seed) {
  auto* c = new BaselineCache();
  c->Hkv = Hkv; c->D = D; c->G = G; c->ng = D / G; c->len = len; c->cap = cap;
  size_t codes = (size_t)Hkv * cap * D, meta = (size_t)Hkv * cap * c->ng;
  c->kc.resize(codes); c->vc.resize(codes); c->kc2.resize(codes); c->vc2.resize(codes);
  for (auto* m : {&c->ks, &c->kz, &c->vs, &c->vz, &c->ks2, &c->kz2, &c->vs2, &c->vz2}) m->resize(meta);
  uint64_t st = seed * 0x9E3779B97F4A7C15ull + 1;
  auto rnd = [&]() { st ^= st << 13; st ^= st >> 7; st ^= st << 17; return st; };
  for (int h = 0; h < Hkv; ++h)
    for (int64_t t = 0; t < len; ++t) {
      size_t row = (size_t)h * cap + t;
      for (int d = 0; d < D; ++d) {
        c->kc[row * D + d] = (uint8_t)rnd();
        c->vc[row * D + d] = (uint8_t)rnd();
      }
      for (int g = 0; g < c->ng; ++g) {
        c->ks[row * c->ng + g] = f32_to_f16(0.02f);
        c->vs[row * c->ng + g] = f32_to_f16(0.02f);
        c->kz[row * c->ng + g] = f32_to_f16(-2.5f);
        c->vz[row * c->ng + g] = f32_to_f16(-2.5f);
      }
    }
  return c;
}

void oracle_baseline_destroy(void* p) { delete static_cast<BaselineCache*>(p); }

static void baseline_step_one(BaselineCache* c, const uint16_t* knew, const uint16_t* vnew,
                              const uint16_t* q, int Hq, int dtype, float scale, uint16_t* out) {
  int Hkv = c->Hkv, D = c->D, G = c->G, ng = c->ng;
  int64_t L = c->len, L1 = L + 1;
  if (L1 > c->cap) return;
  // 1. quantize the new rows
  std::vector<uint8_t> qk((size_t)Hkv * D), qv((size_t)Hkv * D);
  std::vector<uint16_t> sk((size_t)Hkv * ng), zk((size_t)Hkv * ng), sv((size_t)Hkv * ng), zv((size_t)Hkv * ng);
  oracle_quantize(knew, dtype, Hkv, D, G, 0, qk.data(), sk.data(), zk.data());
  oracle_quantize(vnew, dtype, Hkv, D, G, 0, qv.data(), sv.data(), zv.data());
  // 2. concatenate: copy old rows + new row into the other buffer, then swap
  for (int h = 0; h < Hkv; ++h) {
    size_t base = (size_t)h * c->cap;
    std::memcpy(&c->kc2[base * D], &c->kc[base * D], (size_t)L * D);
    std::memcpy(&c->vc2[base * D], &c->vc[base * D], (size_t)L * D);
    std::memcpy(&c->kc2[(base + L) * D], &qk[(size_t)h * D], D);
    std::memcpy(&c->vc2[(base + L) * D], &qv[(size_t)h * D], D);
    for (auto pr : {std::make_pair(&c->ks, &c->ks2), std::make_pair(&c->kz, &c->kz2),
                    std::make_pair(&c->vs, &c->vs2), std::make_pair(&c->vz, &c->vz2)})
      std::memcpy(&(*pr.second)[base * ng], &(*pr.first)[base * ng], (size_t)L * ng * 2);
    std::memcpy(&c->ks2[(base + L) * ng], &sk[(size_t)h * ng], ng * 2);
    std::memcpy(&c->kz2[(base + L) * ng], &zk[(size_t)h * ng], ng * 2);
    std::memcpy(&c->vs2[(base + L) * ng], &sv[(size_t)h * ng], ng * 2);
    std::memcpy(&c->vz2[(base + L) * ng], &zv[(size_t)h * ng], ng * 2);
  }
  std::swap(c->kc, c->kc2); std::swap(c->vc, c->vc2);
  std::swap(c->ks, c->ks2); std::swap(c->kz, c->kz2);
  std::swap(c->vs, c->vs2); std::swap(c->vz, c->vz2);
  c->len = L1;
  // 3. dequantize the full cache to f16 (a transient, as the reference does)
  std::vector<uint16_t> kd((size_t)Hkv * L1 * D), vd((size_t)Hkv * L1 * D);
  for (int h = 0; h < Hkv; ++h) {
    size_t base = (size_t)h * c->cap;
    oracle_dequantize(&c->kc[base * D], &c->ks[base * ng], &c->kz[base * ng], L1, D, G,
                      &kd[(size_t)h * L1 * D]);
    oracle_dequantize(&c->vc[base * D], &c->vs[base * ng], &c->vz[base * ng], L1, D, G,
                      &vd[(size_t)h * L1 * D]);
  }
  // 4. SDPA in float32 with GQA, f16 output
  int grp = Hq / Hkv;
  std::vector<float> s((size_t)L1), acc((size_t)D);
  for (int h = 0; h < Hq; ++h) {
    int kh = h / grp;
    float m = -INFINITY;
    for (int64_t t = 0; t < L1; ++t) {
      const uint16_t* kt = &kd[((size_t)kh * L1 + t) * D];
      float a = 0.f;
      for (int d = 0; d < D; ++d) a += load_in(q[(size_t)h * D + d], dtype) * f16_to_f32(kt[d]);
      s[t] = a * scale;
      m = std::max(m, s[t]);
    }
    float l = 0.f;
    for (int64_t t = 0; t < L1; ++t) { s[t] = std::exp(s[t] - m); l += s[t]; }
    std::fill(acc.begin(), acc.end(), 0.f);
    for (int64_t t = 0; t < L1; ++t) {
      const uint16_t* vt = &vd[((size_t)kh * L1 + t) * D];
      for (int d = 0; d < D; ++d) acc[d] += s[t] * f16_to_f32(vt[d]);
    }
    for (int d = 0; d < D; ++d) out[(size_t)h * D + d] = f32_to_f16(acc[d] / l);
  }
}

// Run one decode step over `n` caches (e.g. n = seqs × layers) on `threads`
// threads. knew/vnew: [n][Hkv][D]; q/out: [n][Hq][D] (16-bit bits).
void oracle_baseline_step(void** caches, int64_t n, const uint16_t* knew, const uint16_t* vnew,
                          const uint16_t* q, int Hq, int dtype, float scale, uint16_t* out,
                          int threads) {
  if (n <= 0) return;
  std::atomic<int64_t> next{0};
  auto worker = [&]() {
    for (;;) {
      int64_t i = next.fetch_add(1);
      if (i >= n) break;
      auto* c = static_cast<BaselineCache*>(caches[i]);
      size_t kvo = (size_t)i * c->Hkv * c->D, qo = (size_t)i * Hq * c->D;
      baseline_step_one(c, knew + kvo, vnew + kvo, q + qo, Hq, dtype, scale, out + qo);
    }
  };
  threads = std::max(1, threads);
  std::vector<std::thread> pool;
  for (int t = 1; t < threads; ++t) pool.emplace_back(worker);
  worker();
  for (auto& th : pool) th.join();
}

int oracle_hardware_concurrency() { return (int)std::thread::hardware_concurrency(); }

}  // extern "C"
