// host.cpp — host side of the B200 KV-cache library: block pool accounting,
// sequences (per-layer lengths over one shared block table), copy-on-write,
// the decode-attention planner, the prefix cache, and every C-ABI entry
// point declared in include/krill_kv.h.
//
// The reference keeps one MLXArray set per layer per request and lets Swift
// ARC reference-count them (Sources/KrillCache/QuantizedKVCache.swift,
// PrefixCache.swift). Here the same state is a table of 256-token blocks per
// sequence; blocks carry explicit reference counts so that prefix entries and
// forked sequences share them without copies.
#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <deque>
#include <filesystem>
#include <list>
#include <map>
#include <mutex>
#include <queue>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "../../include/krill_kv.h"
#include "internal.h"

using namespace krill;

namespace {

thread_local std::string g_err;

krill_status_t fail(krill_status_t code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

#define CUDA_TRY(expr)                                                                       \
  do {                                                                                       \
    cudaError_t _e = (expr);                                                                 \
    if (_e != cudaSuccess) return fail(KRILL_ERR_CUDA, "%s: %s", #expr, cudaGetErrorString(_e)); \
  } while (0)

#define TRY(expr)                        \
  do {                                   \
    krill_status_t _s = (expr);          \
    if (_s != KRILL_OK) return _s;       \
  } while (0)

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (dev < 0) return;
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != dev) {
      cudaSetDevice(dev);
      prev = cur;
    }
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

struct Seq {
  uint32_t gen = 0;
  bool alive = false;
  std::vector<int32_t> blocks;  // full history: block i holds positions [256i, 256i+256);
                                // windowed: ring slot i, -1 until first written
  std::vector<int64_t> len;     // per layer: tokens seen (sequenceLength)
  std::vector<int64_t> ret;     // per layer: rows retained (== len on full history)
};

// Pinned host + device staging buffer for one launch's metadata packet; the
// event guards reuse until every kernel reading it has finished.
struct StageSlot {
  uint8_t* h = nullptr;
  uint8_t* d = nullptr;
  size_t cap = 0;
  cudaEvent_t ev = nullptr;
  bool pending = false;
  bool owned = false;  // h/d allocated for this slot (else a slice of the pool's arena)
};
constexpr int kStageSlots = 16;
// Every slot starts as a slice of one pinned + one device arena made with the
// pool, so no call allocates staging until a packet outgrows its slice.
constexpr size_t kStageSliceBytes = 1 << 20;

// An append whose destinations were planned but whose upload and launch are
// left to the caller (see do_append).
struct DeferredAppend {
  std::vector<AppendDst> dst;
  int32_t lb = 0, lc = 0, n_seqs = 0, n_new = 0, dtype = 0;
  const void* k = nullptr;
  const void* v = nullptr;
  bool pending = false;  // planned, not launched yet
};

// Decode-attention planner buffers, reused across calls.
__global__ void or_flag_kernel(int* dst, const int* src) { *dst |= *src; }

struct Plan {
  std::vector<Seq*> sv;
  std::vector<AttnUnit> units;
  std::vector<AttnItem> items, items_tmp;
  std::vector<size_t> run_start, run_cur;
  std::vector<int64_t> bucket;
  std::vector<int32_t> order, owner, count, fill;
  std::vector<uint64_t> heap;
  std::vector<uint8_t> dry;
  std::vector<int64_t> nsb;
  std::vector<int32_t> split_units;
  // cascade (shared-prefix / causal) planning
  struct Pair {
    int32_t layer, leader;
    int64_t n_sb;
    int32_t mem_off, n_rows, h, causal;
  };
  std::vector<Pair> pairs;
  std::vector<int32_t> gorder, gstart, gmembers, seq_sh;
  std::vector<int64_t> gshared;
  std::vector<ShItem> sh_items;
  std::vector<int32_t> sh_members, sh_cta;
  int last_C = 0, last_HG = 0, last_grid = 0;
  int64_t last_items = 0;
  int last_groups = 0, last_pslots = 0, last_sh_grid = 0;
  int64_t last_sh_items = 0;
  char last_kernels[192] = {0};  // kernel instances of the last launch
};

}  // namespace

struct krill_pool_s {
  krill_pool_cfg cfg{};
  Geom geom{};
  int device = -1;
  bool host_only = true;
  uint8_t* d_pool = nullptr;
  std::vector<int32_t> refcnt;
  std::vector<int32_t> free_blocks;
  std::vector<Seq> seqs;
  std::vector<uint32_t> free_slots;
  int num_sms = 148;
  int pair_slots = 74;  // CTA pairs of the cascade kernel resident at once (0: none)
  float* d_partials = nullptr;
  int64_t partials_cap = 0;
  unsigned long long* d_split_ctr = nullptr;  // arrival counters, one per partial record
  uint32_t attn_epoch = 0;                    // launches of the decode kernel (never 0 in use)
  int64_t kernels = 0;  // device kernels launched since the last krill_pool_kernel_count
  std::map<std::string, uint8_t*> ipc_maps;  // other processes' pools opened here (handle bytes)
  int* d_err = nullptr;
  StageSlot stage[kStageSlots];
  int stage_next = 0;
  uint8_t* stage_arena_h = nullptr;  // kStageSlots slices of kStageSliceBytes
  uint8_t* stage_arena_d = nullptr;
  std::recursive_mutex mu;
  // kernel timing (measurement hook): event pairs around each launch
  bool profiling = false;
  struct Timed {
    cudaEvent_t a, b;
    int kind;  // 0 = attention, 1 = append
  };
  std::vector<Timed> timed;
  std::vector<cudaEvent_t> spare_events;
  Plan plan;
  DeferredAppend deferred;  // krill_decode_step's append, folded into the attention packet
  // krill_decode_step_host: device staging for the step's inputs and output,
  // the two copy streams and the per-chunk events that order them.
  struct HostIo {
    uint8_t* d = nullptr;
    int64_t cap = 0;
    cudaStream_t h2d = nullptr, d2h = nullptr;
    std::vector<cudaEvent_t> ev;
  } io;

  int64_t ring_tokens() const { return (int64_t)geom.ring * kBlockTokens; }
  bool windowed() const { return cfg.window > 0; }
  uint8_t* block_ptr(int32_t b) const { return d_pool + (int64_t)b * geom.block_bytes; }
};

namespace {

// ---------------------------------------------------------------- blocks
krill_status_t block_alloc(krill_pool_t p, int32_t* out) {
  if (p->free_blocks.empty())
    return fail(KRILL_ERR_OOM, "block pool exhausted (%lld blocks)", (long long)p->cfg.num_blocks);
  int32_t b = p->free_blocks.back();
  p->free_blocks.pop_back();
  p->refcnt[b] = 1;
  *out = b;
  return KRILL_OK;
}
void block_ref(krill_pool_t p, int32_t b) { p->refcnt[b] += 1; }
void block_unref(krill_pool_t p, int32_t b) {
  if (b < 0) return;
  if (--p->refcnt[b] == 0) p->free_blocks.push_back(b);
}

// ---------------------------------------------------------------- sequences
krill_status_t seq_get(krill_pool_t p, krill_seq_t h, Seq** out) {
  uint32_t slot = (uint32_t)(h & 0xffffffffu), gen = (uint32_t)(h >> 32);
  if (slot >= p->seqs.size() || !p->seqs[slot].alive || p->seqs[slot].gen != gen)
    return fail(KRILL_ERR_INVALID, "stale or unknown sequence handle 0x%llx", (unsigned long long)h);
  *out = &p->seqs[slot];
  return KRILL_OK;
}

krill_status_t seq_new(krill_pool_t p, krill_seq_t* out, Seq** sp) {
  uint32_t slot;
  if (!p->free_slots.empty()) {
    slot = p->free_slots.back();
    p->free_slots.pop_back();
  } else {
    slot = (uint32_t)p->seqs.size();
    p->seqs.emplace_back();
  }
  Seq& s = p->seqs[slot];
  s.gen += 1;
  s.alive = true;
  s.blocks.clear();
  if (p->windowed()) s.blocks.assign(p->geom.ring, -1);
  s.len.assign(p->geom.L, 0);
  s.ret.assign(p->geom.L, 0);
  *out = ((uint64_t)s.gen << 32) | slot;
  if (sp) *sp = &s;
  return KRILL_OK;
}

void seq_drop_blocks(krill_pool_t p, Seq& s) {
  for (int32_t b : s.blocks) block_unref(p, b);
  s.blocks.clear();
  if (p->windowed()) s.blocks.assign(p->geom.ring, -1);
}

// Full-history pools: release blocks past the longest layer.
void seq_trim_blocks(krill_pool_t p, Seq& s) {
  if (p->windowed()) return;
  int64_t mx = 0;
  for (int64_t l : s.len) mx = std::max(mx, l);
  size_t need = (size_t)((mx + kBlockTokens - 1) / kBlockTokens);
  while (s.blocks.size() > need) {
    block_unref(p, s.blocks.back());
    s.blocks.pop_back();
  }
}

// Make block-table index `idx` writable: allocate it, or copy it if shared.
krill_status_t seq_writable_block(krill_pool_t p, Seq& s, int64_t idx, cudaStream_t stream) {
  if (!p->windowed()) {
    while ((int64_t)s.blocks.size() <= idx) {
      int32_t b = -1;
      TRY(block_alloc(p, &b));
      s.blocks.push_back(b);
    }
  } else if (s.blocks[idx] < 0) {
    int32_t b = -1;
    TRY(block_alloc(p, &b));
    s.blocks[idx] = b;
    return KRILL_OK;
  }
  int32_t b = s.blocks[idx];
  if (p->refcnt[b] > 1) {
    int32_t nb = -1;
    TRY(block_alloc(p, &nb));
    if (!p->host_only)
      CUDA_TRY(cudaMemcpyAsync(p->block_ptr(nb), p->block_ptr(b), (size_t)p->geom.block_bytes,
                               cudaMemcpyDeviceToDevice, stream));
    block_unref(p, b);
    s.blocks[idx] = nb;
  }
  return KRILL_OK;
}

int64_t block_index(krill_pool_t p, int64_t pos) {
  int64_t bi = pos / kBlockTokens;
  return p->windowed() ? bi % p->geom.ring : bi;
}

// ---------------------------------------------------------------- staging
krill_status_t stage_acquire(krill_pool_t p, size_t bytes, StageSlot** out) {
  StageSlot& s = p->stage[p->stage_next];
  p->stage_next = (p->stage_next + 1) % kStageSlots;
  if (s.pending) {
    CUDA_TRY(cudaEventSynchronize(s.ev));
    s.pending = false;
  }
  if (!s.ev) CUDA_TRY(cudaEventCreateWithFlags(&s.ev, cudaEventDisableTiming));
  if (s.cap < bytes) {
    if (s.owned) {
      if (s.h) cudaFreeHost(s.h);
      if (s.d) cudaFree(s.d);
    }
    s.h = nullptr;
    s.d = nullptr;
    s.cap = 0;
    s.owned = true;
    size_t cap = kStageSliceBytes;
    while (cap < bytes) cap *= 2;
    CUDA_TRY(cudaMallocHost(&s.h, cap));
    CUDA_TRY(cudaMalloc(&s.d, cap));
    s.cap = cap;
  }
  *out = &s;
  return KRILL_OK;
}

krill_status_t stage_upload(StageSlot* s, size_t bytes, cudaStream_t stream) {
  CUDA_TRY(cudaMemcpyAsync(s->d, s->h, bytes, cudaMemcpyHostToDevice, stream));
  return KRILL_OK;
}

krill_status_t stage_release(StageSlot* s, cudaStream_t stream) {
  CUDA_TRY(cudaEventRecord(s->ev, stream));
  s->pending = true;
  return KRILL_OK;
}

size_t align16(size_t x) { return (x + 15) & ~(size_t)15; }

cudaEvent_t take_event(krill_pool_t p) {
  if (!p->spare_events.empty()) {
    cudaEvent_t e = p->spare_events.back();
    p->spare_events.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

// Record an event pair around `launch` when profiling is on.
template <typename F>
cudaError_t timed_launch(krill_pool_t p, int kind, cudaStream_t stream, F&& launch) {
  if (!p->profiling) return launch();
  cudaEvent_t a = take_event(p), b = take_event(p);
  cudaEventRecord(a, stream);
  cudaError_t e = launch();
  cudaEventRecord(b, stream);
  p->timed.push_back({a, b, kind});
  return e;
}

krill_status_t require_device(krill_pool_t p) {
  if (p->host_only) return fail(KRILL_ERR_NO_DEVICE, "compute call on a host-only pool");
  return KRILL_OK;
}

krill_status_t check_dtype16(int32_t dt, const char* what) {
  if (dt != KRILL_DTYPE_F16 && dt != KRILL_DTYPE_BF16)
    return fail(KRILL_ERR_INVALID, "%s dtype must be F16 or BF16 (got %d)", what, dt);
  return KRILL_OK;
}

krill_status_t check_aligned(const void* ptr, const char* what) {
  if (((uintptr_t)ptr & 15) != 0) return fail(KRILL_ERR_INVALID, "%s must be 16-byte aligned", what);
  return KRILL_OK;
}

krill_status_t check_layers(krill_pool_t p, int32_t lb, int32_t lc) {
  if (lb < 0 || lc < 0 || lb + lc > p->geom.L)
    return fail(KRILL_ERR_INVALID, "layer range [%d, %d) outside [0, %d)", lb, lb + lc, p->geom.L);
  return KRILL_OK;
}

// ---------------------------------------------------------------- append
// On a host-only (dry-run) pool the block accounting, copy-on-write decisions
// and length updates run, and the device work is skipped.
// With `deferred` the destinations go to deferred->dst (host) and the upload
// and launch are left to the caller (krill_decode_step folds them into the
// attention's metadata packet); the bookkeeping is the same.
krill_status_t launch_deferred_append(krill_pool_t p, DeferredAppend& da, const AppendDst* d_dst,
                                      cudaStream_t stream);

krill_status_t do_append(krill_pool_t p, int32_t n_seqs, const krill_seq_t* seqs, int32_t lb,
                         int32_t lc, int32_t n_new, const void* k, const void* v, int32_t dtype,
                         cudaStream_t stream, RopeTable rope = RopeTable{nullptr, nullptr, 0},
                         DeferredAppend* deferred = nullptr) {
  TRY(check_layers(p, lb, lc));
  TRY(check_dtype16(dtype, "k/v"));
  if (rope.cos) {
    if (p->geom.fmt != kFmtInt8) return fail(KRILL_ERR_INVALID, "the RoPE append needs an int8 pool");
    if (!rope.sin) return fail(KRILL_ERR_INVALID, "null rope_sin");
    if ((reinterpret_cast<uintptr_t>(rope.cos) | reinterpret_cast<uintptr_t>(rope.sin)) & 3)
      return fail(KRILL_ERR_INVALID, "rope tables must be 4-byte aligned");
  }
  if (p->geom.fmt == kFmtBf16 && dtype != KRILL_DTYPE_BF16)
    return fail(KRILL_ERR_INVALID, "a bf16 pool stores bf16 K/V: k/v dtype must be BF16");
  if (n_seqs < 0 || n_new < 0) return fail(KRILL_ERR_INVALID, "negative count");
  if (n_seqs == 0 || lc == 0 || n_new == 0) return KRILL_OK;
  if (!seqs || (!p->host_only && (!k || !v))) return fail(KRILL_ERR_INVALID, "null k/v/seqs");
  if (p->windowed() && n_new > p->cfg.max_append)
    return fail(KRILL_ERR_INVALID, "n_new %d exceeds the windowed pool's max_append %d", n_new,
                p->cfg.max_append);
  std::vector<Seq*> sv(n_seqs);
  for (int i = 0; i < n_seqs; ++i) TRY(seq_get(p, seqs[i], &sv[i]));
  for (int i = 0; i < n_seqs; ++i)
    for (int j = 0; j < i; ++j)
      if (sv[i] == sv[j]) return fail(KRILL_ERR_INVALID, "sequence listed twice in one call");
  if (rope.cos)
    for (int i = 0; i < n_seqs; ++i)
      for (int li = 0; li < lc; ++li)
        if (sv[i]->len[lb + li] + n_new > rope.rows)
          return fail(KRILL_ERR_INVALID, "position %lld beyond the %lld-row rope table",
                      (long long)(sv[i]->len[lb + li] + n_new - 1), (long long)rope.rows);
  // tiled appends (int8 pools) take one entry per touched sub-block
  const bool tiled = append_uses_tiles(n_new) && p->geom.fmt == kFmtInt8;
  const int n_chunks = append_tile_chunks(n_new, p->geom.subt);
  const size_t n_dst = (size_t)lc * n_seqs * (tiled ? n_chunks : n_new);
  StageSlot* slot = nullptr;
  std::vector<AppendDst> dry;
  AppendDst* dst;
  if (deferred && !p->host_only) {
    deferred->dst.resize(n_dst);
    dst = deferred->dst.data();
  } else if (p->host_only) {
    dry.resize(n_dst);
    dst = dry.data();
  } else {
    TRY(stage_acquire(p, n_dst * sizeof(AppendDst), &slot));
    dst = reinterpret_cast<AppendDst*>(slot->h);
  }
  for (int si = 0; si < n_seqs; ++si) {
    Seq& s = *sv[si];
    // make every touched block writable first (allocation / copy-on-write)
    for (int li = 0; li < lc; ++li) {
      int64_t p0 = s.len[lb + li];
      if (p0 + n_new > INT32_MAX) return fail(KRILL_ERR_INVALID, "sequence too long");
      int64_t b0 = p0 / kBlockTokens, b1 = (p0 + n_new - 1) / kBlockTokens;
      for (int64_t bi = b0; bi <= b1; ++bi)
        TRY(seq_writable_block(p, s, p->windowed() ? bi % p->geom.ring : bi, stream));
    }
    for (int li = 0; li < lc; ++li) {
      int64_t p0 = s.len[lb + li];
      if (tiled) {
        const int64_t T = p->geom.subt, base = p0 - p0 % T;
        for (int c = 0; c < n_chunks; ++c) {
          const int64_t pos = std::max<int64_t>(p0, base + c * T);
          AppendDst& d = dst[((size_t)li * n_seqs + si) * n_chunks + c];
          d.block = pos < p0 + n_new ? s.blocks[block_index(p, pos)] : -1;
          d.pos = (int32_t)std::min<int64_t>(pos, INT32_MAX);
        }
        continue;
      }
      for (int t = 0; t < n_new; ++t) {
        int64_t pos = p0 + t;
        AppendDst& d = dst[((size_t)li * n_seqs + si) * n_new + t];
        d.block = s.blocks[block_index(p, pos)];
        d.pos = (int32_t)pos;
      }
    }
  }
  if (deferred && !p->host_only) {
    deferred->lb = lb;
    deferred->lc = lc;
    deferred->n_seqs = n_seqs;
    deferred->n_new = n_new;
    deferred->dtype = dtype;
    deferred->k = k;
    deferred->v = v;
    deferred->pending = true;
  } else if (!p->host_only) {
    TRY(stage_upload(slot, n_dst * sizeof(AppendDst), stream));
    CUDA_TRY(timed_launch(p, 1, stream, [&] {
      return launch_append(p->geom, p->d_pool, reinterpret_cast<const AppendDst*>(slot->d), lb, lc,
                           n_seqs, n_new, k, v, dtype, p->d_err + 1, rope, stream);
    }));
    p->kernels += 1;
    TRY(stage_release(slot, stream));
  }
  for (int si = 0; si < n_seqs; ++si) {
    Seq& s = *sv[si];
    for (int li = 0; li < lc; ++li) {
      const int L = lb + li;
      s.len[L] += n_new;
      if (p->windowed())
        s.ret[L] = std::min<int64_t>(s.ret[L], p->cfg.window - 1) + n_new;
      else
        s.ret[L] = s.len[L];
    }
  }
  return KRILL_OK;
}

// The append kernel of a deferred append, its destinations at d_dst (device).
krill_status_t launch_deferred_append(krill_pool_t p, DeferredAppend& da, const AppendDst* d_dst,
                                      cudaStream_t stream) {
  da.pending = false;
  CUDA_TRY(timed_launch(p, 1, stream, [&] {
    return launch_append(p->geom, p->d_pool, d_dst, da.lb, da.lc, da.n_seqs, da.n_new, da.k, da.v,
                         da.dtype, p->d_err + 1, RopeTable{nullptr, nullptr, 0}, stream);
  }));
  p->kernels += 1;
  return KRILL_OK;
}

// A deferred append that its attention call did not launch (it failed before
// its launches): uploaded and launched on its own, so that the advanced
// lengths always have their K/V.
krill_status_t flush_deferred_append(krill_pool_t p, DeferredAppend& da, cudaStream_t stream) {
  if (!da.pending) return KRILL_OK;
  StageSlot* slot = nullptr;
  const size_t bytes = da.dst.size() * sizeof(AppendDst);
  TRY(stage_acquire(p, bytes, &slot));
  std::memcpy(slot->h, da.dst.data(), bytes);
  TRY(stage_upload(slot, bytes, stream));
  TRY(launch_deferred_append(p, da, reinterpret_cast<const AppendDst*>(slot->d), stream));
  return stage_release(slot, stream);
}

// ---------------------------------------------------------------- attention
krill_status_t ensure_scratch(krill_pool_t p, int64_t records, int64_t /*unused*/) {
  const int64_t pf = partial_floats(p->geom.D);
  if (records * pf > p->partials_cap) {
    // grows rarely (first launches); the free must not race kernels in flight
    CUDA_TRY(cudaDeviceSynchronize());
    if (p->d_partials) cudaFree(p->d_partials);
    if (p->d_split_ctr) cudaFree(p->d_split_ctr);
    p->d_partials = nullptr;
    p->d_split_ctr = nullptr;
    p->partials_cap = 0;
    int64_t cap = std::max<int64_t>(records * pf * 3 / 2, 1 << 20);
    CUDA_TRY(cudaMalloc(&p->d_partials, (size_t)cap * sizeof(float)));
    const int64_t n_ctr = cap / pf + 1;
    CUDA_TRY(cudaMalloc(&p->d_split_ctr, (size_t)n_ctr * sizeof(unsigned long long)));
    CUDA_TRY(cudaMemset(p->d_split_ctr, 0, (size_t)n_ctr * sizeof(unsigned long long)));
    p->partials_cap = cap;
  }
  return KRILL_OK;
}

krill_status_t do_attention(krill_pool_t p, int32_t n_seqs, const krill_seq_t* seqs, int32_t lb,
                            int32_t lc, const void* q, int32_t q_dtype, void* out,
                            int32_t out_dtype, float scale, cudaStream_t stream,
                            int32_t n_query = 1, DeferredAppend* pre = nullptr) {
  TRY(check_layers(p, lb, lc));
  if (n_query < 1) return fail(KRILL_ERR_INVALID, "n_query must be positive");
  if (n_query > 1 && p->windowed())
    return fail(KRILL_ERR_INVALID, "multi-query verify attention needs a full-history pool");
  // Many queries per sequence (chunked prefill, long verify) run as causal
  // tcgen05 cascade items: the sequence's K/V is read once per query block.
  const bool causal_path = n_query > 1 && p->geom.fmt == kFmtInt8 &&
                           shared_uses_umma(p->geom, p->cfg.attn_impl) &&
                           (int64_t)n_query * p->geom.g >= 64;
  TRY(check_dtype16(q_dtype, "q"));
  if (p->geom.fmt == kFmtBf16 && q_dtype != KRILL_DTYPE_BF16)
    return fail(KRILL_ERR_INVALID, "attention over a bf16 pool takes a BF16 q");
  if (out_dtype != KRILL_DTYPE_F16 && out_dtype != KRILL_DTYPE_BF16 && out_dtype != KRILL_DTYPE_F32)
    return fail(KRILL_ERR_INVALID, "out dtype must be F16, BF16 or F32");
  if (n_seqs < 0) return fail(KRILL_ERR_INVALID, "negative n_seqs");
  if (n_seqs == 0 || lc == 0) return KRILL_OK;
  if (!seqs || (!p->host_only && (!q || !out))) return fail(KRILL_ERR_INVALID, "null q/out/seqs");
  TRY(check_aligned(q, "q"));
  TRY(check_aligned(out, "out"));
  const Geom& g = p->geom;
  Plan& pl = p->plan;
  pl.sv.resize(n_seqs);
  int64_t bt_stride = 1;
  for (int i = 0; i < n_seqs; ++i) {
    TRY(seq_get(p, seqs[i], &pl.sv[i]));
    bt_stride = std::max<int64_t>(bt_stride, (int64_t)pl.sv[i]->blocks.size());
  }
  // ---- shared-prefix groups (cascade) ----
  // Sequences whose block tables begin with the same physical blocks (forks of
  // one prefix-cache entry) attend that common prefix through cascade items
  // that read and dequantize it once for all of them; each member's decode
  // items then start where the shared part ends. Only on full-history pools
  // with a tensor-core implementation and adaptive splitting: a fixed
  // split_tokens promises results that do not depend on the rest of the batch.
  pl.gstart.clear();
  pl.gmembers.clear();
  pl.gshared.clear();
  pl.seq_sh.assign((size_t)n_seqs, 0);
  const int64_t min_tok = p->cfg.cascade_min_tokens == 0 ? 256 : p->cfg.cascade_min_tokens;
  if (!p->windowed() && g.fmt == kFmtInt8 && p->cfg.attn_impl != KRILL_ATTN_CUDA_CORE &&
      p->cfg.split_tokens == 0 && n_query == 1 &&
      p->cfg.cascade_min_tokens >= 0 && n_seqs >= 2) {
    const size_t min_blocks = (size_t)std::max<int64_t>(1, (min_tok + kBlockTokens - 1) / kBlockTokens);
    pl.gorder.clear();
    for (int si = 0; si < n_seqs; ++si)
      if (pl.sv[si]->blocks.size() >= min_blocks) pl.gorder.push_back(si);
    std::sort(pl.gorder.begin(), pl.gorder.end(), [&](int32_t a, int32_t b) {
      const auto& x = pl.sv[a]->blocks;
      const auto& y = pl.sv[b]->blocks;
      return std::lexicographical_compare(x.begin(), x.end(), y.begin(), y.end()) ||
             (x == y && a < b);
    });
    auto lcp = [&](int32_t a, int32_t b) {
      const auto& x = pl.sv[a]->blocks;
      const auto& y = pl.sv[b]->blocks;
      const size_t n = std::min(x.size(), y.size());
      size_t i = 0;
      while (i < n && x[i] == y[i]) ++i;
      return i;
    };
    for (size_t i = 0; i < pl.gorder.size();) {
      size_t j = i + 1, common = SIZE_MAX;
      while (j < pl.gorder.size()) {
        const size_t c = lcp(pl.gorder[j - 1], pl.gorder[j]);
        if (c < min_blocks) break;
        common = std::min(common, c);
        ++j;
      }
      if (j - i >= 2) {
        // whole common blocks, strictly below every member's length at every
        // layer of the call (each member keeps at least one own token)
        int64_t S = (int64_t)common * kBlockTokens;
        for (size_t k = i; k < j; ++k)
          for (int li = 0; li < lc; ++li) S = std::min<int64_t>(S, pl.sv[pl.gorder[k]]->len[lb + li] - 1);
        S -= S % g.subt;
        if (S >= min_tok) {
          pl.gstart.push_back((int32_t)pl.gmembers.size());
          pl.gshared.push_back(S);
          for (size_t k = i; k < j; ++k) {
            pl.gmembers.push_back(pl.gorder[k]);
            pl.seq_sh[pl.gorder[k]] = (int32_t)(S / g.subt);
          }
        }
      }
      i = j;
    }
  }
  const int n_groups = (int)pl.gshared.size();
  pl.gstart.push_back((int32_t)pl.gmembers.size());
  // ---- units (layer, seq[, query]) ----
  // With n_query > 1 (speculative verify) the last n_query tokens of each
  // sequence are the queries: query j sees the cache up to and including its
  // own token and none of the later drafts (buildBatchedVerifyMask,
  // BatchedDecode.swift:299-312). On the int8 tensor-core decode kernel up to
  // 8 / g consecutive queries share one unit as further columns of its query
  // tile, each column masked at its own query's bound (AttnUnit::nq), so the
  // cache is read once per unit instead of once per query; otherwise (and on
  // the causal cascade path) one unit per query.
  const int fold = (n_query > 1 && !causal_path && g.fmt == kFmtInt8 &&
                    p->cfg.attn_impl != KRILL_ATTN_CUDA_CORE)
                       ? std::max(1, std::min(n_query, 8 / g.g))
                       : 1;
  const int q_units = (n_query + fold - 1) / fold;  // units per (layer, sequence)
  // Two units per sequence on a decode kernel with one warp per kv head:
  // the second unit (the shadow) becomes the second 8-column query tile of
  // the first one's items, so each sub-block is staged once for both; the
  // shadow keeps its own queries, bounds and partial records, and has no
  // items of its own.
  const bool qt2 = q_units == 2 && !causal_path && g.fmt == kFmtInt8 && g.D <= 128 &&
                   g.Hkv >= 8 && p->cfg.attn_impl != KRILL_ATTN_CUDA_CORE;
  const int64_t n_units = (int64_t)lc * n_seqs * q_units;
  pl.units.resize((size_t)n_units);
  pl.nsb.resize((size_t)n_units);
  int64_t total_sb = 0;
  for (int li = 0; li < lc; ++li) {
    const int L = lb + li;
    for (int si = 0; si < n_seqs; ++si) {
      const Seq& s = *pl.sv[si];
      const int64_t len = s.len[L];
      if (len <= 0) return fail(KRILL_ERR_INVALID, "attention over an empty cache (layer %d)", L);
      if (len < n_query)
        return fail(KRILL_ERR_INVALID, "%d queries need their tokens in the cache (layer %d holds %lld)",
                    n_query, L, (long long)len);
      for (int k = 0; k < q_units; ++k) {
        const int j0 = k * fold, nq = std::min(fold, n_query - j0);  // queries j0 .. j0 + nq - 1
        const int64_t t_hi = len - n_query + j0 + nq;                // the last one's bound
        const int64_t t_lo = p->windowed() ? len - std::min<int64_t>(s.ret[L], p->cfg.window) : 0;
        const int64_t ui = ((int64_t)li * n_seqs + si) * q_units + k;
        AttnUnit& u = pl.units[ui];
        u.qo_row = (int32_t)(((int64_t)li * n_seqs + si) * n_query + j0);
        u.si = si;
        u.layer = L;
        u.t_lo = (int32_t)t_lo;
        u.t_hi = (int32_t)t_hi;
        u.n_pre = 0;
        u.nq = nq;
        pl.nsb[ui] = causal_path ? 0
                                 : (t_hi + g.subt - 1) / g.subt -
                                       std::max<int64_t>(t_lo / g.subt, pl.seq_sh[si]);
        total_sb += pl.nsb[ui];
        if (qt2 && k == 1) {  // the shadow's range is the pair's: its items cover both
          total_sb -= pl.nsb[ui - 1];
          pl.nsb[ui - 1] = pl.nsb[ui];
        }
      }
    }
  }
  // ---- decomposition: sequence piece length C (sub-blocks) and kv heads per
  // item HG. A fixed split_tokens keeps C fixed and HG = Hkv, so a sequence's
  // result does not depend on the batch; otherwise both follow the batch
  // shape: the largest pieces such that one item is at most a quarter of a
  // CTA's share, halving the head group when even 8-sub-block pieces are too
  // coarse (small batches). Results depend only on shapes, never on contents.
  int C, HG = g.Hkv;
  bool latency_bound = false;
  if (p->cfg.split_tokens > 0) {
    C = std::max(1, p->cfg.split_tokens / g.subt);
  } else if ((latency_bound = !qt2 && (int64_t)8 * g.Hkv >
                                          std::max<int64_t>(1, total_sb * g.Hkv / p->num_sms / 4))) {
    // Small batch (8-sub-block items of all kv heads would exceed a quarter of
    // a CTA's share): the step is latency-bound, and its time is about the
    // largest item plus, where a sequence is split over CTAs, the merge of
    // the pieces through global memory. Splitting heads costs less: the R =
    // 8 / HG warps of one head share its sub-blocks and merge in shared
    // memory. So for each head group HG, take the shortest pieces (at least
    // R sub-blocks, one per warp) that give at most one item per CTA, and
    // keep the (HG, C) with the least estimated time in sub-blocks per warp:
    // the item's share, plus for a split plan about 3 for the fence, count
    // and merge latency and 1/8 per piece the merge reads.
    const int W = attn_warps(g.D);
    int64_t max_nsb = 1;
    for (int64_t ui = 0; ui < n_units; ++ui) max_nsb = std::max<int64_t>(max_nsb, pl.nsb[ui]);
    auto n_items_for = [&](int hg, int64_t c) {
      int64_t n = 0;
      for (int64_t ui = 0; ui < n_units; ++ui) n += (pl.nsb[ui] + c - 1) / c;
      return n * (g.Hkv / hg);
    };
    double best = 1e300;
    C = 1;
    for (int hg = g.Hkv; hg >= 1; hg /= 2) {
      if (g.Hkv % hg != 0 || !(hg % W == 0 || W % hg == 0)) break;
      const int64_t cmin = std::max(1, W / hg);
      int64_t lo = cmin, hi = std::max<int64_t>(cmin, max_nsb);  // items fall as C grows
      while (lo < hi) {
        const int64_t mid = (lo + hi) / 2;
        if (n_items_for(hg, mid) > p->num_sms) lo = mid + 1;
        else hi = mid;
      }
      const int64_t items = n_items_for(hg, lo);
      const int64_t waves = (items + p->num_sms - 1) / p->num_sms;
      const bool split = lo < max_nsb;
      const double cost = (double)(waves * lo * hg) / W + (split ? 3.0 + (double)((max_nsb + lo - 1) / lo) / 8.0 : 0.0);
      if (cost < best) {
        best = cost;
        HG = hg;
        C = (int)std::min<int64_t>(lo, INT32_MAX);
      }
      if (hg % 2 != 0) break;
    }
  } else {
    const int64_t quarter = std::max<int64_t>(1, total_sb * g.Hkv / p->num_sms / 4);
    C = 8;
    while (C < 128 && (int64_t)(2 * C) * HG <= quarter) C *= 2;
  }
  // ---- cascade items: (layer, row block, kv head) pairs cut into fragments.
  // A pair is either a shared-prefix group (rows = member sequences x GQA
  // group, tokens = the common blocks) or, on the causal path, a block of one
  // sequence's queries (rows = queries x GQA group, tokens = everything up to
  // the block's last query, masked per row). The pairs' sub-blocks are laid
  // end to end and split into equal contiguous ranges, one per CTA; the
  // fragment index within a pair is its partial-record slot. Pairs that read
  // the same blocks are adjacent, so the CTAs working on them share L2.
  pl.sh_items.clear();
  pl.sh_members.clear();
  pl.sh_cta.clear();
  pl.pairs.clear();
  int n_pslots = 0, sh_grid = 0;
  {
    const int mem_cap = std::max(1, shared_rows(g, p->cfg.attn_impl) / g.g);
    for (int gi = 0; gi < n_groups; ++gi) {
      const int32_t* mem = pl.gmembers.data() + pl.gstart[gi];
      const int n_mem = pl.gstart[gi + 1] - pl.gstart[gi];
      for (int li = 0; li < lc; ++li)
        for (int mb = 0; mb < n_mem; mb += mem_cap) {
          const int nm = std::min(mem_cap, n_mem - mb);
          const int32_t mem_off = (int32_t)pl.sh_members.size();
          for (int k = 0; k < nm; ++k) pl.sh_members.push_back((int32_t)((int64_t)li * n_seqs + mem[mb + k]));
          for (int h = 0; h < g.Hkv; ++h)
            pl.pairs.push_back(Plan::Pair{lb + li, mem[0], pl.gshared[gi] / g.subt, mem_off, nm * g.g, h, -1});
        }
    }
    if (causal_path)
      for (int li = 0; li < lc; ++li)
        for (int si = 0; si < n_seqs; ++si) {
          const int64_t len = pl.sv[si]->len[lb + li];
          for (int q0 = 0; q0 < n_query; q0 += mem_cap) {
            const int nq = std::min(mem_cap, n_query - q0);
            const int32_t mem_off = (int32_t)pl.sh_members.size();
            for (int k = 0; k < nq; ++k)
              pl.sh_members.push_back((int32_t)(((int64_t)li * n_seqs + si) * n_query + q0 + k));
            const int64_t first_pos = len - n_query + q0;  // position of the block's first query
            const int64_t n_sb = (first_pos + nq + g.subt - 1) / g.subt;
            for (int h = 0; h < g.Hkv; ++h)
              pl.pairs.push_back(Plan::Pair{lb + li, si, n_sb, mem_off, nq * g.g, h, (int32_t)first_pos});
          }
        }
  }
  // Under KRILL_ATTN_TENSOR_CORE_PAIR, items of more than 128 rows run on CTA
  // pairs (one M = 256 instruction for both halves, each CTA dequantizing
  // half of every sub-block); a pair then takes the place of one CTA in the
  // split below.
  bool sh_pair = false;
  if (!pl.pairs.empty() && p->cfg.attn_impl == KRILL_ATTN_TENSOR_CORE_PAIR && p->pair_slots > 0 &&
      shared_uses_umma(g, p->cfg.attn_impl))
    for (const Plan::Pair& pr : pl.pairs) sh_pair = sh_pair || pr.n_rows > 128;
  if (!pl.pairs.empty()) {
    int64_t W = 0;
    for (const Plan::Pair& pr : pl.pairs) W += pr.n_sb;
    constexpr int64_t kMinFragment = 8;  // sub-blocks
    const int64_t workers = sh_pair ? p->pair_slots : p->num_sms;
    const int64_t grid_sh =
        std::max<int64_t>(1, std::min<int64_t>(workers, (W + kMinFragment - 1) / kMinFragment));
    const int64_t per = (W + grid_sh - 1) / grid_sh;
    sh_grid = (int)((W + per - 1) / per);
    pl.sh_cta.assign((size_t)sh_grid + 1, 0);
    int64_t pos = 0;
    for (const Plan::Pair& pr : pl.pairs) {
      const int64_t a = pos, b = pos + pr.n_sb;
      const int64_t first = a / per, last = (b - 1) / per;
      for (int64_t c = first; c <= last; ++c) {
        ShItem it{};
        it.layer = pr.layer;
        it.leader = pr.leader;
        it.sb_begin = (int32_t)(std::max(a, c * per) - a);
        it.sb_end = (int32_t)(std::min(b, (c + 1) * per) - a);
        it.mem_off = pr.mem_off;
        it.n_rows = (int16_t)pr.n_rows;
        it.h = (int16_t)pr.h;
        it.slot = (int16_t)(c - first);
        it.n_frag = (int16_t)(last - first + 1);
        it.causal = pr.causal;
        pl.sh_items.push_back(it);
        pl.sh_cta[(size_t)c + 1] += 1;
      }
      n_pslots = std::max<int>(n_pslots, (int)(last - first + 1));
      pos = b;
    }
    for (int c = 0; c < sh_grid; ++c) pl.sh_cta[(size_t)c + 1] += pl.sh_cta[(size_t)c];
  }
  // ---- items ----
  pl.items.clear();
  int64_t split_count = 0;
  pl.split_units.clear();
  // In a latency-bound plan the decode piece that arrives last merges its
  // split unit, which saves the combine kernel's launch and its serial
  // latency. A bandwidth-bound plan keeps the combine kernel: there the
  // fence and count that every split piece would pay cost more than the
  // combine's ~1 % of the step. Units without decode pieces always need it.
  bool merge_in_kernel = latency_bound && !causal_path;
  for (int64_t ui = 0; ui < n_units; ++ui) {
    AttnUnit& u = pl.units[ui];
    if (causal_path) {  // every record comes from the causal cascade items
      u.first_split = (int32_t)split_count;
      u.n_pre = 0;
      u.n_split = (int32_t)n_pslots;
      split_count += n_pslots;
      pl.split_units.push_back((int32_t)ui);
      continue;
    }
    const int64_t n_sb = pl.nsb[ui];
    const int64_t n_it = (n_sb + C - 1) / C;
    const int64_t base = n_sb / n_it, extra = n_sb % n_it;
    const int sh_sb = pl.seq_sh[u.si];
    // cascaded units: records [0, n_pslots) come from the cascade items. A
    // single suffix piece merges them itself when it finishes; several go
    // through the combine kernel with the prefix records as pieces 0..
    const int64_t off = sh_sb > 0 ? n_pslots : 0;
    u.first_split = (int32_t)split_count;
    u.n_pre = 0;
    if (sh_sb > 0 && n_it == 1) {
      u.n_split = 1;
      u.n_pre = n_pslots;
      split_count += n_pslots;
    } else {
      u.n_split = (int32_t)(off + n_it);
      u.n_pre = (int32_t)off;
      if (u.n_split > 1 && n_it < 1) merge_in_kernel = false;
      if (u.n_split > 1) {
        split_count += u.n_split;
        pl.split_units.push_back((int32_t)ui);
      }
    }
    if (qt2 && (ui % 2) == 1) continue;  // a shadow: tile 2 of the previous unit's items
    int64_t b = std::max<int64_t>(u.t_lo / g.subt, sh_sb);
    for (int64_t i = 0; i < n_it; ++i) {
      const int64_t sz = base + (i < extra ? 1 : 0);
      for (int h0 = 0; h0 < g.Hkv; h0 += HG)
        pl.items.push_back(AttnItem{(int32_t)ui, (int32_t)b, (int32_t)(b + sz),
                                    (int16_t)(u.n_split == 1 ? 0 : off + i), (int16_t)h0});
      b += sz;
    }
  }
  if (q_units > 1 && !causal_path) {
    // The units of one (layer, sequence) in a multi-query call read the same
    // blocks: interleave their items (piece by piece) so that the assignment
    // below, stable for equal sizes, hands matching pieces to CTAs side by
    // side, and the second read of each sub-block is served from L2.
    pl.items_tmp.clear();
    pl.items_tmp.reserve(pl.items.size());
    size_t a = 0;
    while (a < pl.items.size()) {
      const int32_t grp = pl.items[a].unit / q_units;
      size_t b = a;
      while (b < pl.items.size() && pl.items[b].unit / q_units == grp) ++b;
      // [a, b) holds the group's units, each a contiguous run, in unit order
      pl.run_start.clear();
      for (size_t i = a; i < b; ++i)
        if (i == a || pl.items[i].unit != pl.items[i - 1].unit) pl.run_start.push_back(i);
      const size_t nr = pl.run_start.size();
      pl.run_start.push_back(b);
      pl.run_cur.assign(pl.run_start.begin(), pl.run_start.end() - 1);
      for (size_t left = b - a; left > 0;)
        for (size_t r = 0; r < nr; ++r)
          if (pl.run_cur[r] < pl.run_start[r + 1]) {
            pl.items_tmp.push_back(pl.items[pl.run_cur[r]++]);
            --left;
          }
      a = b;
    }
    pl.items.swap(pl.items_tmp);
  }
  if (!p->host_only) TRY(ensure_scratch(p, split_count * g.Hkv, 0));
  // ---- longest-processing-time assignment of items to persistent CTAs ----
  // Items are at most C sub-blocks, so a counting sort orders them by size.
  const int64_t n_items = (int64_t)pl.items.size();
  const int grid =
      (int)std::min<int64_t>((int64_t)p->num_sms * attn_ctas_per_sm(p->cfg.attn_impl), n_items);
  pl.bucket.assign((size_t)C + 2, 0);
  for (const AttnItem& it : pl.items) pl.bucket[C - (it.sb_end - it.sb_begin)] += 1;
  for (int i = 1; i <= C + 1; ++i) pl.bucket[i] += pl.bucket[i - 1];
  pl.order.resize((size_t)n_items);
  for (int64_t i = n_items - 1; i >= 0; --i) {
    const AttnItem& it = pl.items[i];
    pl.order[--pl.bucket[C - (it.sb_end - it.sb_begin)]] = (int32_t)i;
  }
  pl.owner.resize((size_t)n_items);
  pl.count.assign((size_t)grid, 0);
  // min-heap of (load << 20 | cta): one integer compare orders by load, then
  // by CTA index
  pl.heap.resize((size_t)grid);
  for (int c = 0; c < grid; ++c) pl.heap[c] = (uint64_t)c;  // already a min-heap
  auto sift_down = [&](size_t i) {
    const size_t n = pl.heap.size();
    uint64_t* h = pl.heap.data();
    const uint64_t v = h[i];
    for (;;) {
      size_t l = 2 * i + 1;
      if (l >= n) break;
      if (l + 1 < n && h[l + 1] < h[l]) ++l;
      if (h[l] >= v) break;
      h[i] = h[l];
      i = l;
    }
    h[i] = v;
  };
  if (n_items <= grid) {  // one item per CTA (latency-bound plans): no heap
    for (int64_t r = 0; r < n_items; ++r) {
      pl.owner[pl.order[r]] = (int32_t)r;
      pl.count[r] = 1;
    }
  } else {
    for (int32_t i : pl.order) {
      uint64_t& top = pl.heap[0];
      const int32_t c = (int32_t)(top & 0xfffffu);
      pl.owner[i] = c;
      pl.count[c] += 1;
      top += (uint64_t)(pl.items[i].sb_end - pl.items[i].sb_begin) << 20;
      sift_down(0);
    }
  }
  // ---- metadata packet: units | items (grouped by CTA) | cta offsets | block tables ----
  const size_t units_bytes = align16((size_t)n_units * sizeof(AttnUnit));
  const size_t items_bytes = align16((size_t)n_items * sizeof(AttnItem));
  const size_t off_bytes = align16((size_t)(grid + 1) * sizeof(int32_t));
  const size_t bt_bytes = align16((size_t)n_seqs * bt_stride * sizeof(int32_t));
  const size_t su_bytes = align16((pl.split_units.size() + 1) * sizeof(int32_t));
  const size_t shi_bytes = align16(pl.sh_items.size() * sizeof(ShItem));
  const size_t shc_bytes = align16(pl.sh_cta.size() * sizeof(int32_t));
  const size_t shm_bytes = align16(pl.sh_members.size() * sizeof(int32_t));
  const size_t sh_off = units_bytes + items_bytes + off_bytes + bt_bytes + su_bytes;
  // a deferred append's destinations ride in the same packet (one upload)
  const size_t pre_off = sh_off + shi_bytes + shc_bytes + shm_bytes;
  const size_t pre_bytes = pre && pre->pending ? align16(pre->dst.size() * sizeof(AppendDst)) : 0;
  const size_t total = pre_off + pre_bytes;
  StageSlot* slot = nullptr;
  uint8_t* h;
  if (p->host_only) {
    pl.dry.resize(total);
    h = pl.dry.data();
  } else {
    TRY(stage_acquire(p, total, &slot));
    h = slot->h;
  }
  std::memcpy(h, pl.units.data(), (size_t)n_units * sizeof(AttnUnit));
  AttnItem* hi = reinterpret_cast<AttnItem*>(h + units_bytes);
  int32_t* off = reinterpret_cast<int32_t*>(h + units_bytes + items_bytes);
  off[0] = 0;
  for (int c = 0; c < grid; ++c) off[c + 1] = off[c] + pl.count[c];
  pl.fill.assign(off, off + grid);
  for (int32_t i : pl.order) hi[pl.fill[pl.owner[i]]++] = pl.items[i];
  int32_t* bt = reinterpret_cast<int32_t*>(h + units_bytes + items_bytes + off_bytes);
  for (int si = 0; si < n_seqs; ++si) {
    const Seq& s = *pl.sv[si];
    const size_t nb = s.blocks.size();
    if (nb) std::memcpy(bt + si * bt_stride, s.blocks.data(), nb * sizeof(int32_t));
    for (int64_t j = (int64_t)nb; j < bt_stride; ++j) bt[si * bt_stride + j] = -1;
  }
  int32_t* su = reinterpret_cast<int32_t*>(h + units_bytes + items_bytes + off_bytes + bt_bytes);
  if (!pl.split_units.empty())
    std::memcpy(su, pl.split_units.data(), pl.split_units.size() * sizeof(int32_t));
  if (sh_grid > 0) {
    std::memcpy(h + sh_off, pl.sh_items.data(), pl.sh_items.size() * sizeof(ShItem));
    std::memcpy(h + sh_off + shi_bytes, pl.sh_cta.data(), pl.sh_cta.size() * sizeof(int32_t));
    std::memcpy(h + sh_off + shi_bytes + shc_bytes, pl.sh_members.data(),
                pl.sh_members.size() * sizeof(int32_t));
  }
  if (pre_bytes) std::memcpy(h + pre_off, pre->dst.data(), pre->dst.size() * sizeof(AppendDst));
  pl.last_groups = n_groups;
  pl.last_pslots = n_pslots;
  pl.last_sh_grid = sh_pair ? 2 * sh_grid : sh_grid;
  pl.last_sh_items = (int64_t)pl.sh_items.size();
  pl.last_C = C;
  pl.last_HG = HG;
  pl.last_items = n_items;
  pl.last_grid = grid;
  {
    // the kernel instances this plan launches (dry runs included); only the
    // fields the description reads are set
    static unsigned long long ctr_tag;
    AttnParams dp{};
    dp.hg = HG;
    dp.qt = qt2 ? 2 : 1;
    dp.g = g.g;
    dp.n_split_units = (int)pl.split_units.size();
    dp.split_ctr = merge_in_kernel ? &ctr_tag : nullptr;
    dp.sh_grid = sh_grid;
    dp.sh_pair = sh_pair ? 1 : 0;
    describe_attention(g, dp, grid, p->cfg.attn_impl, pl.last_kernels, sizeof(pl.last_kernels));
  }
  if (p->host_only) return KRILL_OK;  // dry run: planned, nothing launched
  TRY(stage_upload(slot, total, stream));
  AttnParams ap{};
  ap.pool = p->d_pool;
  ap.page_bytes = g.page_bytes;
  ap.sb_bytes = g.sb_bytes;
  ap.L = g.L;
  ap.Hkv = g.Hkv;
  ap.Hq = g.Hq;
  ap.g = g.g;
  ap.ring = g.ring;
  ap.units = reinterpret_cast<const AttnUnit*>(slot->d);
  ap.items = reinterpret_cast<const AttnItem*>(slot->d + units_bytes);
  ap.cta_off = reinterpret_cast<const int32_t*>(slot->d + units_bytes + items_bytes);
  ap.bt = reinterpret_cast<const int32_t*>(slot->d + units_bytes + items_bytes + off_bytes);
  ap.bt_stride = (int)bt_stride;
  ap.hg = HG;
  ap.qt = qt2 ? 2 : 1;
  ap.split_units = reinterpret_cast<const int32_t*>(slot->d + units_bytes + items_bytes + off_bytes + bt_bytes);
  ap.n_split_units = (int)pl.split_units.size();
  ap.q = q;
  ap.q_dtype = q_dtype;
  ap.out = out;
  ap.out_dtype = out_dtype;
  ap.scale_log2 = scale * 1.4426950408889634f;
  ap.partials = p->d_partials;
  ap.split_ctr = merge_in_kernel ? p->d_split_ctr : nullptr;
  if (++p->attn_epoch == 0) p->attn_epoch = 1;
  ap.epoch = p->attn_epoch;
  ap.err = p->d_err;
  ap.wait_us = p->cfg.wait_timeout_us;
  ap.large_scale = p->d_err + 1;
  if (sh_grid > 0) {
    ap.sh_items = reinterpret_cast<const ShItem*>(slot->d + sh_off);
    ap.sh_cta_off = reinterpret_cast<const int32_t*>(slot->d + sh_off + shi_bytes);
    ap.sh_members = reinterpret_cast<const int32_t*>(slot->d + sh_off + shi_bytes + shc_bytes);
    ap.sh_grid = sh_grid;
    ap.sh_pair = sh_pair ? 1 : 0;
    ap.n_pslots = n_pslots;
  }
  if (pre_bytes) {
    const krill_status_t st =
        launch_deferred_append(p, *pre, reinterpret_cast<const AppendDst*>(slot->d + pre_off), stream);
    if (st != KRILL_OK) {
      stage_release(slot, stream);
      return st;
    }
    // the decode kernel follows the append directly (no cascade kernel
    // between them): let it start while the append runs
    ap.pdl = (sh_grid == 0 && grid > 0 && p->cfg.attn_impl != KRILL_ATTN_CUDA_CORE) ? 1 : 0;
  }
  CUDA_TRY(timed_launch(p, 0, stream, [&] { return launch_attention(g, ap, grid, p->cfg.attn_impl, stream); }));
  p->kernels += (grid > 0 ? 1 : 0) + (attn_needs_combine(ap, grid, p->cfg.attn_impl) ? 1 : 0) +
                (sh_grid > 0 ? 1 : 0);
  TRY(stage_release(slot, stream));
  return KRILL_OK;
}

// ---------------------------------------------------------------- gather helpers
// Rows physically available for a layer: positions [p0, p0 + S).
void layer_span(krill_pool_t p, const Seq& s, int L, int64_t* p0, int64_t* S) {
  if (p->windowed()) {
    *S = std::min<int64_t>(s.ret[L], p->ring_tokens());
    *p0 = s.len[L] - *S;
  } else {
    *S = s.len[L];
    *p0 = 0;
  }
}

krill_status_t upload_bt(krill_pool_t p, const Seq& s, cudaStream_t stream, StageSlot** out) {
  size_t n = std::max<size_t>(1, s.blocks.size());
  StageSlot* slot;
  TRY(stage_acquire(p, n * sizeof(int32_t), &slot));
  int32_t* bt = reinterpret_cast<int32_t*>(slot->h);
  for (size_t i = 0; i < n; ++i) bt[i] = i < s.blocks.size() ? s.blocks[i] : -1;
  TRY(stage_upload(slot, n * sizeof(int32_t), stream));
  *out = slot;
  return KRILL_OK;
}

krill_status_t do_restore(krill_pool_t p, Seq& s, int32_t layer, int64_t rows, int64_t total_seen,
                          const ScatterIn& in, cudaStream_t stream) {
  if (rows < 0 || total_seen < rows) return fail(KRILL_ERR_INVALID, "bad restore span");
  if (!p->windowed() && rows != total_seen)
    return fail(KRILL_ERR_INVALID, "full-history restore needs rows == total_seen");
  if (p->windowed() && rows > p->ring_tokens())
    return fail(KRILL_ERR_INVALID, "restore of %lld rows exceeds the ring (%lld)", (long long)rows,
                (long long)p->ring_tokens());
  if (!p->host_only && rows > 0 &&
      (!in.keys || !in.values || !in.key_scales || !in.key_zeros || !in.value_scales ||
       !in.value_zeros))
    return fail(KRILL_ERR_INVALID, "restore needs all six tensors");
  const int64_t p0 = total_seen - rows;
  if (rows > 0) {
    int64_t b0 = p0 / kBlockTokens, b1 = (total_seen - 1) / kBlockTokens;
    for (int64_t bi = b0; bi <= b1; ++bi)
      TRY(seq_writable_block(p, s, p->windowed() ? bi % p->geom.ring : bi, stream));
    if (!p->host_only) {
      StageSlot* slot;
      TRY(upload_bt(p, s, stream, &slot));
      CUDA_TRY(launch_scatter(p->geom, p->d_pool, layer, reinterpret_cast<const int32_t*>(slot->d),
                              p0, rows, in, p->d_err + 1, stream));
      p->kernels += 1;
      TRY(stage_release(slot, stream));
    }
  }
  s.len[layer] = total_seen;
  s.ret[layer] = rows;
  seq_trim_blocks(p, s);
  return KRILL_OK;
}

}  // namespace

// =====================================================================
// C ABI
// =====================================================================
extern "C" {

const char* krill_last_error_string(void) { return g_err.c_str(); }
const char* krill_version(void) { return "krill-kv-b200 0.1.0 (sm_100a)"; }

krill_status_t krill_pool_create(const krill_pool_cfg* cfg_in, int32_t device, krill_pool_t* out) {
  if (!cfg_in || !out) return fail(KRILL_ERR_INVALID, "null argument");
  krill_pool_cfg cfg = *cfg_in;
  if (cfg.num_layers <= 0 || cfg.num_kv_heads <= 0 || cfg.num_q_heads <= 0)
    return fail(KRILL_ERR_INVALID, "layers and heads must be positive");
  if (cfg.num_q_heads % cfg.num_kv_heads != 0 || cfg.num_q_heads / cfg.num_kv_heads > 8)
    return fail(KRILL_ERR_INVALID, "num_q_heads must be a multiple of num_kv_heads, ratio <= 8");
  if (cfg.head_dim != 64 && cfg.head_dim != 128 && cfg.head_dim != 256)
    return fail(KRILL_ERR_INVALID, "head_dim must be 64, 128 or 256");
  if (cfg.group_size == 0) cfg.group_size = 64;
  if (cfg.group_size != 64 && cfg.group_size != cfg.head_dim)
    return fail(KRILL_ERR_INVALID, "group_size must be 64 or head_dim");
  {
    // decode attention processes min(Hkv, W) kv heads at a time, W = 8 warps:
    // Hkv must divide W or be a multiple of it
    const int W = 8;
    const int hpr = std::min(cfg.num_kv_heads, W);
    if (W % hpr != 0 || cfg.num_kv_heads % hpr != 0)
      return fail(KRILL_ERR_INVALID, "num_kv_heads must divide %d or be a multiple of it", W);
  }
  if (cfg.window == 1 || cfg.window < 0) return fail(KRILL_ERR_INVALID, "window must be 0 or > 1");
  if (cfg.max_append <= 0) cfg.max_append = 256;
  if (cfg.quant_variant != KRILL_QUANT_F32 && cfg.quant_variant != KRILL_QUANT_INPUT_DTYPE)
    return fail(KRILL_ERR_INVALID, "bad quant_variant");
  if (cfg.attn_impl != KRILL_ATTN_TENSOR_CORE && cfg.attn_impl != KRILL_ATTN_CUDA_CORE &&
      cfg.attn_impl != KRILL_ATTN_TENSOR_CORE_SYNC && cfg.attn_impl != KRILL_ATTN_TENSOR_CORE_PAIR)
    return fail(KRILL_ERR_INVALID, "bad attn_impl");
  if (cfg.split_tokens < 0 || cfg.split_tokens % 64 != 0)
    return fail(KRILL_ERR_INVALID, "split_tokens must be 0 (adaptive) or a multiple of 64");
  if (cfg.num_blocks <= 0 || cfg.num_blocks > INT32_MAX)
    return fail(KRILL_ERR_INVALID, "num_blocks out of range");
  if (cfg.wait_timeout_us < 0) return fail(KRILL_ERR_INVALID, "wait_timeout_us must be >= 0");
  if (cfg.kv_format != KRILL_KV_INT8 && cfg.kv_format != KRILL_KV_BF16)
    return fail(KRILL_ERR_INVALID, "kv_format must be KRILL_KV_INT8 or KRILL_KV_BF16");
  if (cfg.kv_format == KRILL_KV_BF16) {
    if (cfg.head_dim > 128) return fail(KRILL_ERR_INVALID, "bf16 pools support head_dim 64 and 128");
    if (cfg.attn_impl == KRILL_ATTN_CUDA_CORE)
      return fail(KRILL_ERR_INVALID, "bf16 pools use the tensor-core attention");
    cfg.group_size = cfg.head_dim;  // no quantization groups
  }
  int ring = 0;
  if (cfg.window > 0) {
    int64_t need = (int64_t)cfg.window - 1 + cfg.max_append;
    ring = (int)((need + kBlockTokens - 1) / kBlockTokens);
  }
  auto* p = new krill_pool_s();
  p->cfg = cfg;
  p->geom = make_geom(cfg.num_layers, cfg.num_kv_heads, cfg.num_q_heads, cfg.head_dim,
                      cfg.group_size, ring, cfg.window, cfg.quant_variant,
                      cfg.kv_format == KRILL_KV_BF16 ? kFmtBf16 : kFmtInt8);
  p->device = device;
  p->host_only = device < 0;
  p->refcnt.assign((size_t)cfg.num_blocks, 0);
  p->free_blocks.reserve((size_t)cfg.num_blocks);
  for (int64_t b = cfg.num_blocks - 1; b >= 0; --b) p->free_blocks.push_back((int32_t)b);
  if (!p->host_only) {
    DeviceGuard dg(device);
    cudaError_t e = cudaSetDevice(device);
    size_t bytes = (size_t)cfg.num_blocks * (size_t)p->geom.block_bytes;
    if (e == cudaSuccess) e = cudaMalloc(&p->d_pool, bytes);
    if (e == cudaSuccess) e = cudaMemset(p->d_pool, 0, bytes);
    // [0] error flag, [1] large-scale flag (a stored scale with |s| >= 64)
    if (e == cudaSuccess) e = cudaMalloc(&p->d_err, kDevWords * sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(p->d_err, 0, kDevWords * sizeof(int));
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&p->num_sms, cudaDevAttrMultiProcessorCount, device);
    if (e == cudaSuccess) e = cudaMallocHost(&p->stage_arena_h, kStageSlots * kStageSliceBytes);
    if (e == cudaSuccess) e = cudaMalloc(&p->stage_arena_d, kStageSlots * kStageSliceBytes);
    if (e == cudaSuccess)
      for (int i = 0; i < kStageSlots; ++i) {
        p->stage[i].h = p->stage_arena_h + (size_t)i * kStageSliceBytes;
        p->stage[i].d = p->stage_arena_d + (size_t)i * kStageSliceBytes;
        p->stage[i].cap = kStageSliceBytes;
      }
    // The allocation-free entry point's scratch is resolved here, with the
    // pool's device current, so that the driver reserves it (a module load
    // under lazy loading) at pool creation rather than inside a decode call.
    if (e == cudaSuccess) e = krill::noalloc_prepare(device);
    // CTA pairs of the cascade kernel that fit at once (0: single-CTA cascade)
    if (e == cudaSuccess && cfg.attn_impl == KRILL_ATTN_TENSOR_CORE_PAIR &&
        shared_uses_umma(p->geom, cfg.attn_impl))
      p->pair_slots = std::min(krill::shared_pair_capacity(p->geom), p->num_sms / 2);
    if (e != cudaSuccess) {
      krill_status_t code = (e == cudaErrorMemoryAllocation) ? KRILL_ERR_OOM : KRILL_ERR_CUDA;
      if (p->d_pool) cudaFree(p->d_pool);
      if (p->d_err) cudaFree(p->d_err);
      if (p->stage_arena_h) cudaFreeHost(p->stage_arena_h);
      if (p->stage_arena_d) cudaFree(p->stage_arena_d);
      delete p;
      cudaGetLastError();
      return fail(code, "pool allocation on device %d failed: %s", device, cudaGetErrorString(e));
    }
  }
  *out = p;
  return KRILL_OK;
}

krill_status_t krill_pool_destroy(krill_pool_t p) {
  if (!p) return KRILL_OK;
  if (!p->host_only) {
    DeviceGuard dg(p->device);
    cudaDeviceSynchronize();
    for (auto& s : p->stage) {
      if (s.owned && s.h) cudaFreeHost(s.h);
      if (s.owned && s.d) cudaFree(s.d);
      if (s.ev) cudaEventDestroy(s.ev);
    }
    if (p->stage_arena_h) cudaFreeHost(p->stage_arena_h);
    if (p->stage_arena_d) cudaFree(p->stage_arena_d);
    for (auto& e : p->timed) {
      cudaEventDestroy(e.a);
      cudaEventDestroy(e.b);
    }
    for (auto e : p->spare_events) cudaEventDestroy(e);
    for (auto e : p->io.ev) cudaEventDestroy(e);
    if (p->io.h2d) cudaStreamDestroy(p->io.h2d);
    if (p->io.d2h) cudaStreamDestroy(p->io.d2h);
    if (p->io.d) cudaFree(p->io.d);
    for (auto& m : p->ipc_maps) cudaIpcCloseMemHandle(m.second);
    if (p->d_pool) cudaFree(p->d_pool);
    if (p->d_partials) cudaFree(p->d_partials);
    if (p->d_split_ctr) cudaFree(p->d_split_ctr);
    if (p->d_err) cudaFree(p->d_err);
  }
  delete p;
  return KRILL_OK;
}

krill_status_t krill_pool_block_bytes(krill_pool_t p, int64_t* bytes) {
  if (!p || !bytes) return fail(KRILL_ERR_INVALID, "null argument");
  *bytes = p->geom.block_bytes;
  return KRILL_OK;
}

krill_status_t krill_pool_free_blocks(krill_pool_t p, int64_t* n) {
  if (!p || !n) return fail(KRILL_ERR_INVALID, "null argument");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  *n = (int64_t)p->free_blocks.size();
  return KRILL_OK;
}

krill_status_t krill_pool_block_refcount(krill_pool_t p, int32_t block, int32_t* rc) {
  if (!p || !rc) return fail(KRILL_ERR_INVALID, "null argument");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  if (block < 0 || block >= (int64_t)p->refcnt.size()) return fail(KRILL_ERR_INVALID, "bad block id");
  *rc = p->refcnt[block];
  return KRILL_OK;
}

krill_status_t krill_pool_device_error(krill_pool_t p, int32_t* flag) {
  if (!p || !flag) return fail(KRILL_ERR_INVALID, "null argument");
  *flag = 0;
  if (p->host_only) return KRILL_OK;
  DeviceGuard dg(p->device);
  int v = 0;
  CUDA_TRY(cudaMemcpy(&v, p->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (v) CUDA_TRY(cudaMemset(p->d_err, 0, sizeof(int)));
  *flag = v;
  return KRILL_OK;
}

krill_status_t krill_pool_test_stall(krill_pool_t p, int32_t enable) {
  if (!p) return fail(KRILL_ERR_INVALID, "null pool");
  if (p->host_only) return fail(KRILL_ERR_NO_DEVICE, "test stall on a host-only pool");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  DeviceGuard dg(p->device);
  const int v = enable ? 1 : 0;
  CUDA_TRY(cudaDeviceSynchronize());
  CUDA_TRY(cudaMemcpy(p->d_err + kDevTestStall, &v, sizeof(int), cudaMemcpyHostToDevice));
  return KRILL_OK;
}

krill_status_t krill_pool_set_profiling(krill_pool_t p, int32_t enable) {
  if (!p) return fail(KRILL_ERR_INVALID, "null pool");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  p->profiling = enable != 0 && !p->host_only;
  return KRILL_OK;
}

krill_status_t krill_pool_kernel_count(krill_pool_t p, int64_t* kernels) {
  if (!p || !kernels) return fail(KRILL_ERR_INVALID, "null argument");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  *kernels = p->kernels;
  p->kernels = 0;
  return KRILL_OK;
}

krill_status_t krill_pool_kernel_times(krill_pool_t p, double* attn_ms, int32_t* attn_launches,
                                       double* append_ms, int32_t* append_launches) {
  if (!p) return fail(KRILL_ERR_INVALID, "null pool");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  DeviceGuard dg(p->device);
  double t[2] = {0.0, 0.0};
  int32_t n[2] = {0, 0};
  for (auto& e : p->timed) {
    CUDA_TRY(cudaEventSynchronize(e.b));
    float ms = 0.f;
    CUDA_TRY(cudaEventElapsedTime(&ms, e.a, e.b));
    t[e.kind] += ms;
    n[e.kind] += 1;
    p->spare_events.push_back(e.a);
    p->spare_events.push_back(e.b);
  }
  p->timed.clear();
  if (attn_ms) *attn_ms = t[0];
  if (attn_launches) *attn_launches = n[0];
  if (append_ms) *append_ms = t[1];
  if (append_launches) *append_launches = n[1];
  return KRILL_OK;
}

krill_status_t krill_pool_last_plan(krill_pool_t p, int32_t* piece_subblocks, int32_t* heads_per_item,
                                    int64_t* items, int32_t* ctas) {
  if (!p) return fail(KRILL_ERR_INVALID, "null pool");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  if (piece_subblocks) *piece_subblocks = p->plan.last_C;
  if (heads_per_item) *heads_per_item = p->plan.last_HG;
  if (items) *items = p->plan.last_items;
  if (ctas) *ctas = p->plan.last_grid;
  return KRILL_OK;
}

krill_status_t krill_pool_last_kernels(krill_pool_t p, char* buf, int32_t cap) {
  if (!p || !buf || cap <= 0) return fail(KRILL_ERR_INVALID, "null pool or buffer");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  snprintf(buf, (size_t)cap, "%s", p->plan.last_kernels);
  return KRILL_OK;
}

krill_status_t krill_pool_last_cascade(krill_pool_t p, int32_t* groups, int64_t* shared_items,
                                       int32_t* prefix_slots, int32_t* ctas) {
  if (!p) return fail(KRILL_ERR_INVALID, "null pool");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  if (groups) *groups = p->plan.last_groups;
  if (shared_items) *shared_items = p->plan.last_sh_items;
  if (prefix_slots) *prefix_slots = p->plan.last_pslots;
  if (ctas) *ctas = p->plan.last_sh_grid;
  return KRILL_OK;
}

krill_status_t krill_seq_create(krill_pool_t p, krill_seq_t* out) {
  if (!p || !out) return fail(KRILL_ERR_INVALID, "null argument");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  return seq_new(p, out, nullptr);
}

krill_status_t krill_seq_release(krill_pool_t p, krill_seq_t h) {
  if (!p) return fail(KRILL_ERR_INVALID, "null pool");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  Seq* s = nullptr;
  TRY(seq_get(p, h, &s));
  seq_drop_blocks(p, *s);
  s->alive = false;
  s->len.clear();
  s->ret.clear();
  p->free_slots.push_back((uint32_t)(h & 0xffffffffu));
  return KRILL_OK;
}

krill_status_t krill_seq_reset(krill_pool_t p, krill_seq_t h) {
  if (!p) return fail(KRILL_ERR_INVALID, "null pool");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  Seq* s = nullptr;
  TRY(seq_get(p, h, &s));
  seq_drop_blocks(p, *s);
  std::fill(s->len.begin(), s->len.end(), 0);
  std::fill(s->ret.begin(), s->ret.end(), 0);
  return KRILL_OK;
}

krill_status_t krill_seq_length(krill_pool_t p, krill_seq_t h, int32_t layer, int64_t* len) {
  if (!p || !len) return fail(KRILL_ERR_INVALID, "null argument");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  Seq* s = nullptr;
  TRY(seq_get(p, h, &s));
  if (layer < 0 || layer >= p->geom.L) return fail(KRILL_ERR_INVALID, "bad layer");
  *len = s->len[layer];
  return KRILL_OK;
}

krill_status_t krill_seq_retained(krill_pool_t p, krill_seq_t h, int32_t layer, int64_t* n) {
  if (!p || !n) return fail(KRILL_ERR_INVALID, "null argument");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  Seq* s = nullptr;
  TRY(seq_get(p, h, &s));
  if (layer < 0 || layer >= p->geom.L) return fail(KRILL_ERR_INVALID, "bad layer");
  *n = s->ret[layer];
  return KRILL_OK;
}

krill_status_t krill_seq_memory_bytes(krill_pool_t p, krill_seq_t h, int32_t layer, int64_t* bytes) {
  if (!p || !bytes) return fail(KRILL_ERR_INVALID, "null argument");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  Seq* s = nullptr;
  TRY(seq_get(p, h, &s));
  if (layer < 0 || layer >= p->geom.L) return fail(KRILL_ERR_INVALID, "bad layer");
  int64_t p0, S;
  layer_span(p, *s, layer, &p0, &S);
  const Geom& g = p->geom;
  // QuantizedKVCache.memorySizeBytes: u8 K+V plus 4 f16 arrays per row (per group)
  *bytes = 2 * S * g.Hkv * g.D + 4 * S * g.Hkv * g.NG * 2;
  return KRILL_OK;
}

krill_status_t krill_seq_can_truncate(krill_pool_t p, krill_seq_t h, int64_t n, int32_t* ok) {
  if (!p || !ok) return fail(KRILL_ERR_INVALID, "null argument");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  Seq* s = nullptr;
  TRY(seq_get(p, h, &s));
  bool good = n >= 0;
  if (p->windowed())
    for (int L = 0; L < p->geom.L && good; ++L)
      good = n >= s->len[L] - s->ret[L] && n <= s->len[L];
  *ok = good ? 1 : 0;
  return KRILL_OK;
}

krill_status_t krill_seq_truncate(krill_pool_t p, krill_seq_t h, int64_t n) {
  if (!p) return fail(KRILL_ERR_INVALID, "null pool");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  Seq* s = nullptr;
  TRY(seq_get(p, h, &s));
  if (n < 0) return KRILL_OK;  // QuantizedKVCache.truncate ignores negative lengths (:138)
  if (p->windowed()) {
    for (int L = 0; L < p->geom.L; ++L)
      if (n < s->len[L] && n < s->len[L] - s->ret[L])
        return fail(KRILL_ERR_INVALID, "truncate(to: %lld) below the retained range of layer %d",
                    (long long)n, L);
    for (int L = 0; L < p->geom.L; ++L)
      if (n < s->len[L]) {
        s->ret[L] -= s->len[L] - n;
        s->len[L] = n;
      }
  } else {
    for (int L = 0; L < p->geom.L; ++L)
      if (n < s->len[L]) s->len[L] = s->ret[L] = n;
    seq_trim_blocks(p, *s);
  }
  return KRILL_OK;
}

krill_status_t krill_seq_blocks(krill_pool_t p, krill_seq_t h, int32_t* ids, int32_t cap, int32_t* n) {
  if (!p || !n) return fail(KRILL_ERR_INVALID, "null argument");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  Seq* s = nullptr;
  TRY(seq_get(p, h, &s));
  *n = (int32_t)s->blocks.size();
  for (int32_t i = 0; i < *n && i < cap && ids; ++i) ids[i] = s->blocks[i];
  return KRILL_OK;
}

krill_status_t krill_append_quantize(krill_pool_t p, int32_t n_seqs, const krill_seq_t* seqs,
                                     int32_t layer_begin, int32_t layer_count, int32_t n_new,
                                     const void* k_new, const void* v_new, int32_t dtype,
                                     void* stream) {
  if (!p) return fail(KRILL_ERR_INVALID, "null pool");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  DeviceGuard dg(p->device);
  return do_append(p, n_seqs, seqs, layer_begin, layer_count, n_new, k_new, v_new, dtype,
                   (cudaStream_t)stream);
}

krill_status_t krill_append_quantize_rope(krill_pool_t p, int32_t n_seqs, const krill_seq_t* seqs,
                                          int32_t layer_begin, int32_t layer_count, int32_t n_new,
                                          const void* k_new, const void* v_new, int32_t dtype,
                                          const float* rope_cos, const float* rope_sin,
                                          int64_t rope_rows, void* stream) {
  if (!p) return fail(KRILL_ERR_INVALID, "null pool");
  if (!rope_cos || !rope_sin || rope_rows <= 0) return fail(KRILL_ERR_INVALID, "null rope table");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  DeviceGuard dg(p->device);
  return do_append(p, n_seqs, seqs, layer_begin, layer_count, n_new, k_new, v_new, dtype,
                   (cudaStream_t)stream, RopeTable{rope_cos, rope_sin, rope_rows});
}

krill_status_t krill_decode_attention(krill_pool_t p, int32_t n_seqs, const krill_seq_t* seqs,
                                      int32_t layer_begin, int32_t layer_count, const void* q,
                                      int32_t q_dtype, void* out, int32_t out_dtype, float scale,
                                      void* stream) {
  if (!p) return fail(KRILL_ERR_INVALID, "null pool");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  DeviceGuard dg(p->device);
  return do_attention(p, n_seqs, seqs, layer_begin, layer_count, q, q_dtype, out, out_dtype, scale,
                      (cudaStream_t)stream);
}

krill_status_t krill_verify_attention(krill_pool_t p, int32_t n_seqs, const krill_seq_t* seqs,
                                      int32_t layer_begin, int32_t layer_count, int32_t n_query,
                                      const void* q, int32_t q_dtype, void* out, int32_t out_dtype,
                                      float scale, void* stream) {
  if (!p) return fail(KRILL_ERR_INVALID, "null pool");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  DeviceGuard dg(p->device);
  return do_attention(p, n_seqs, seqs, layer_begin, layer_count, q, q_dtype, out, out_dtype, scale,
                      (cudaStream_t)stream, n_query);
}

krill_status_t krill_prefill_attention(krill_pool_t p, int32_t n_seqs, const krill_seq_t* seqs,
                                       int32_t layer_begin, int32_t layer_count, int32_t n_query,
                                       const void* q, int32_t q_dtype, void* out, int32_t out_dtype,
                                       float scale, void* stream) {
  return krill_verify_attention(p, n_seqs, seqs, layer_begin, layer_count, n_query, q, q_dtype, out,
                                out_dtype, scale, stream);
}

krill_status_t krill_decode_step(krill_pool_t p, int32_t n_seqs, const krill_seq_t* seqs,
                                 int32_t layer_begin, int32_t layer_count, const void* k_new,
                                 const void* v_new, int32_t kv_dtype, const void* q,
                                 int32_t q_dtype, void* out, int32_t out_dtype, float scale,
                                 void* stream) {
  if (!p) return fail(KRILL_ERR_INVALID, "null pool");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  DeviceGuard dg(p->device);
  // The append's destinations travel in the attention's metadata packet: one
  // upload per step, then the append and attention launches.
  DeferredAppend& da = p->deferred;
  da.pending = false;
  TRY(do_append(p, n_seqs, seqs, layer_begin, layer_count, 1, k_new, v_new, kv_dtype,
                (cudaStream_t)stream, RopeTable{nullptr, nullptr, 0}, &da));
  const krill_status_t st = do_attention(p, n_seqs, seqs, layer_begin, layer_count, q, q_dtype, out,
                                         out_dtype, scale, (cudaStream_t)stream, 1, &da);
  if (da.pending) {
    // keep the error of the attention call, whatever the fallback returns
    const std::string msg = krill_last_error_string();
    flush_deferred_append(p, da, (cudaStream_t)stream);
    if (st != KRILL_OK) set_error(st, msg.c_str());
  }
  return st;
}

krill_status_t krill_decode_step_host(krill_pool_t p, int32_t n_seqs, const krill_seq_t* seqs,
                                      int32_t layer_begin, int32_t layer_count, const void* k_new,
                                      const void* v_new, int32_t kv_dtype, const void* q,
                                      int32_t q_dtype, void* out, int32_t out_dtype, float scale,
                                      int32_t layer_chunk, void* stream) {
  if (!p) return fail(KRILL_ERR_INVALID, "null pool");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  TRY(require_device(p));
  TRY(check_layers(p, layer_begin, layer_count));
  TRY(check_dtype16(kv_dtype, "k/v"));
  TRY(check_dtype16(q_dtype, "q"));
  if (out_dtype != KRILL_DTYPE_F16 && out_dtype != KRILL_DTYPE_BF16 && out_dtype != KRILL_DTYPE_F32)
    return fail(KRILL_ERR_INVALID, "out dtype must be F16, BF16 or F32");
  if (n_seqs < 1 || !seqs) return fail(KRILL_ERR_INVALID, "need at least one sequence");
  if (!k_new || !v_new || !q || !out) return fail(KRILL_ERR_INVALID, "null host buffer");
  if (layer_chunk < 0) return fail(KRILL_ERR_INVALID, "layer_chunk must be >= 0");
  DeviceGuard dg(p->device);
  const Geom& g = p->geom;
  // Bytes per layer of each buffer; the buffers are layer-major, so a chunk of
  // layers is one contiguous range of each.
  const int64_t kv_l = (int64_t)n_seqs * g.Hkv * g.D * 2;
  const int64_t q_l = (int64_t)n_seqs * g.Hq * g.D * 2;
  const int64_t o_l = (int64_t)n_seqs * g.Hq * g.D * (out_dtype == KRILL_DTYPE_F32 ? 4 : 2);
  const int64_t k_off = 0, v_off = align16(kv_l * layer_count), q_off = 2 * v_off;
  const int64_t o_off = q_off + (int64_t)align16(q_l * layer_count);
  const int64_t need = o_off + (int64_t)align16(o_l * layer_count);
  if (need > p->io.cap) {
    CUDA_TRY(cudaDeviceSynchronize());  // earlier steps may still read the old staging
    if (p->io.d) cudaFree(p->io.d);
    p->io.d = nullptr;
    p->io.cap = 0;
    CUDA_TRY(cudaMalloc(&p->io.d, need));
    p->io.cap = need;
  }
  if (!p->io.h2d) CUDA_TRY(cudaStreamCreateWithFlags(&p->io.h2d, cudaStreamNonBlocking));
  if (!p->io.d2h) CUDA_TRY(cudaStreamCreateWithFlags(&p->io.d2h, cudaStreamNonBlocking));
  // Chunking (layer_chunk = 0: one chunk). Measured at the Llama-3.1-8B
  // batch of 32 (12.6 MB in, 8.4 MB out per step): 4 chunks overlap the
  // copies but their launches lose more to ramp-up and tail (1.96 ms of
  // kernels against 1.60 ms in one launch) than the 0.33 ms of copies they
  // hide, so the default keeps the step in one launch.
  int chunk = layer_chunk == 0 ? (int)layer_count : std::min(layer_chunk, (int)layer_count);
  const int n_ch = (layer_count + chunk - 1) / chunk;
  while ((int)p->io.ev.size() < 2 + 2 * n_ch) {
    cudaEvent_t e = nullptr;
    CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    p->io.ev.push_back(e);
  }
  cudaStream_t s = (cudaStream_t)stream;
  cudaEvent_t ev_start = p->io.ev[0], ev_end = p->io.ev[1];
  uint8_t* d = p->io.d;
  // A query in page-locked host memory is read in place by the attention
  // kernels through its device mapping: its transfer then overlaps the cache
  // reads instead of preceding them. Other host memory is copied first.
  const uint8_t* q_mapped = nullptr;
  {
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, q) == cudaSuccess && attr.type == cudaMemoryTypeHost &&
        attr.devicePointer != nullptr && ((uintptr_t)attr.devicePointer & 15) == 0)
      q_mapped = static_cast<const uint8_t*>(attr.devicePointer);
    cudaGetLastError();  // an unregistered pointer leaves an error to clear
  }
  // Everything earlier on `stream` (the previous step's reads of the staging
  // and its output copies, which it joined) precedes this step's uploads.
  CUDA_TRY(cudaEventRecord(ev_start, s));
  CUDA_TRY(cudaStreamWaitEvent(p->io.h2d, ev_start, 0));
  auto copy_in = [&](int c) -> krill_status_t {
    const int64_t c0 = (int64_t)c * chunk, lc = std::min<int64_t>(chunk, layer_count - c0);
    CUDA_TRY(cudaMemcpyAsync(d + k_off + c0 * kv_l, (const uint8_t*)k_new + c0 * kv_l, lc * kv_l,
                             cudaMemcpyHostToDevice, p->io.h2d));
    CUDA_TRY(cudaMemcpyAsync(d + v_off + c0 * kv_l, (const uint8_t*)v_new + c0 * kv_l, lc * kv_l,
                             cudaMemcpyHostToDevice, p->io.h2d));
    if (!q_mapped)
      CUDA_TRY(cudaMemcpyAsync(d + q_off + c0 * q_l, (const uint8_t*)q + c0 * q_l, lc * q_l,
                               cudaMemcpyHostToDevice, p->io.h2d));
    CUDA_TRY(cudaEventRecord(p->io.ev[2 + c], p->io.h2d));
    return KRILL_OK;
  };
  // Chunk c+1's inputs are queued after chunk c's metadata uploads, so that
  // those small copies never wait behind the next chunk's inputs.
  krill_status_t rc = copy_in(0);
  int issued = rc == KRILL_OK ? 1 : 0;
  for (int c = 0; c < n_ch && rc == KRILL_OK; ++c) {
    const int64_t c0 = (int64_t)c * chunk;
    const int32_t lc = (int32_t)std::min<int64_t>(chunk, layer_count - c0);
    CUDA_TRY(cudaStreamWaitEvent(s, p->io.ev[2 + c], 0));
    // as krill_decode_step: the append rides in the attention's packet
    DeferredAppend& da = p->deferred;
    da.pending = false;
    rc = do_append(p, n_seqs, seqs, layer_begin + (int32_t)c0, lc, 1, d + k_off + c0 * kv_l,
                   d + v_off + c0 * kv_l, kv_dtype, s, RopeTable{nullptr, nullptr, 0}, &da);
    if (rc == KRILL_OK)
      rc = do_attention(p, n_seqs, seqs, layer_begin + (int32_t)c0, lc,
                        (q_mapped ? q_mapped : d + q_off) + c0 * q_l, q_dtype, d + o_off + c0 * o_l,
                        out_dtype, scale, s, 1, &da);
    if (da.pending) {
      const std::string msg = krill_last_error_string();
      flush_deferred_append(p, da, s);
      if (rc != KRILL_OK) set_error(rc, msg.c_str());
    }
    if (rc != KRILL_OK) break;
    if (c + 1 < n_ch) {
      rc = copy_in(c + 1);
      if (rc != KRILL_OK) break;
      ++issued;
    }
    CUDA_TRY(cudaEventRecord(p->io.ev[2 + n_ch + c], s));
    CUDA_TRY(cudaStreamWaitEvent(p->io.d2h, p->io.ev[2 + n_ch + c], 0));
    CUDA_TRY(cudaMemcpyAsync((uint8_t*)out + c0 * o_l, d + o_off + c0 * o_l, (int64_t)lc * o_l,
                             cudaMemcpyDeviceToHost, p->io.d2h));
  }
  // Join the copy streams back into `stream` even after an error, so that
  // nothing of this call is left running unordered.
  if (issued > 0) CUDA_TRY(cudaStreamWaitEvent(s, p->io.ev[2 + issued - 1], 0));
  CUDA_TRY(cudaEventRecord(ev_end, p->io.d2h));
  CUDA_TRY(cudaStreamWaitEvent(s, ev_end, 0));
  return rc;
}

krill_status_t krill_seq_snapshot_quantized(krill_pool_t p, krill_seq_t h, int32_t layer,
                                            void* keys, void* values, void* key_scales,
                                            void* key_zeros, void* value_scales,
                                            void* value_zeros, void* stream) {
  if (!p) return fail(KRILL_ERR_INVALID, "null pool");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  if (p->geom.fmt != kFmtInt8) return fail(KRILL_ERR_INVALID, "quantized snapshots need an int8 pool");
  TRY(require_device(p));
  DeviceGuard dg(p->device);
  Seq* s = nullptr;
  TRY(seq_get(p, h, &s));
  if (layer < 0 || layer >= p->geom.L) return fail(KRILL_ERR_INVALID, "bad layer");
  int64_t p0, S;
  layer_span(p, *s, layer, &p0, &S);
  if (S == 0) return KRILL_OK;
  StageSlot* slot;
  TRY(upload_bt(p, *s, (cudaStream_t)stream, &slot));
  GatherOut o{};
  o.keys = (uint8_t*)keys;
  o.values = (uint8_t*)values;
  o.key_scales = (uint16_t*)key_scales;
  o.key_zeros = (uint16_t*)key_zeros;
  o.value_scales = (uint16_t*)value_scales;
  o.value_zeros = (uint16_t*)value_zeros;
  o.row_off = 0;
  o.rows_total = S;
  o.mode = 0;
  CUDA_TRY(launch_gather(p->geom, p->d_pool, layer, reinterpret_cast<const int32_t*>(slot->d), p0, S,
                         o, (cudaStream_t)stream));
  p->kernels += 1;
  return stage_release(slot, (cudaStream_t)stream);
}

krill_status_t krill_seq_snapshot_dequantized(krill_pool_t p, krill_seq_t h, int32_t layer,
                                              void* keys, void* values, void* stream) {
  if (!p) return fail(KRILL_ERR_INVALID, "null pool");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  if (p->geom.fmt != kFmtInt8) return fail(KRILL_ERR_INVALID, "quantized snapshots need an int8 pool");
  TRY(require_device(p));
  DeviceGuard dg(p->device);
  Seq* s = nullptr;
  TRY(seq_get(p, h, &s));
  if (layer < 0 || layer >= p->geom.L) return fail(KRILL_ERR_INVALID, "bad layer");
  int64_t p0, S;
  layer_span(p, *s, layer, &p0, &S);
  if (S == 0) return KRILL_OK;
  StageSlot* slot;
  TRY(upload_bt(p, *s, (cudaStream_t)stream, &slot));
  GatherOut o{};
  o.keys = (uint8_t*)keys;
  o.values = (uint8_t*)values;
  o.rows_total = S;
  o.mode = 1;
  CUDA_TRY(launch_gather(p->geom, p->d_pool, layer, reinterpret_cast<const int32_t*>(slot->d), p0, S,
                         o, (cudaStream_t)stream));
  p->kernels += 1;
  return stage_release(slot, (cudaStream_t)stream);
}

krill_status_t krill_seq_restore_quantized(krill_pool_t p, krill_seq_t h, int32_t layer,
                                           int64_t rows, int64_t total_seen, const void* keys,
                                           const void* values, const void* key_scales,
                                           const void* key_zeros, const void* value_scales,
                                           const void* value_zeros, void* stream) {
  if (!p) return fail(KRILL_ERR_INVALID, "null pool");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  if (p->geom.fmt != kFmtInt8) return fail(KRILL_ERR_INVALID, "quantized snapshots need an int8 pool");
  DeviceGuard dg(p->device);
  Seq* s = nullptr;
  TRY(seq_get(p, h, &s));
  if (layer < 0 || layer >= p->geom.L) return fail(KRILL_ERR_INVALID, "bad layer");
  ScatterIn in{};
  in.keys = (const uint8_t*)keys;
  in.values = (const uint8_t*)values;
  in.key_scales = (const uint16_t*)key_scales;
  in.key_zeros = (const uint16_t*)key_zeros;
  in.value_scales = (const uint16_t*)value_scales;
  in.value_zeros = (const uint16_t*)value_zeros;
  in.row_off = 0;
  in.rows_total = rows;
  return do_restore(p, *s, layer, rows, total_seen, in, (cudaStream_t)stream);
}

krill_status_t krill_stack_left_padded(krill_pool_t p, int32_t n_seqs, const krill_seq_t* seqs,
                                       int32_t layer, int64_t s_max, void* keys, void* values,
                                       void* key_scales, void* key_zeros, void* value_scales,
                                       void* value_zeros, void* stream) {
  if (!p) return fail(KRILL_ERR_INVALID, "null pool");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  if (p->geom.fmt != kFmtInt8) return fail(KRILL_ERR_INVALID, "quantized snapshots need an int8 pool");
  TRY(require_device(p));
  DeviceGuard dg(p->device);
  if (layer < 0 || layer >= p->geom.L) return fail(KRILL_ERR_INVALID, "bad layer");
  if (n_seqs <= 0) return KRILL_OK;
  const Geom& g = p->geom;
  cudaStream_t st = (cudaStream_t)stream;
  std::vector<Seq*> sv(n_seqs);
  for (int i = 0; i < n_seqs; ++i) {
    TRY(seq_get(p, seqs[i], &sv[i]));
    int64_t p0, S;
    layer_span(p, *sv[i], layer, &p0, &S);
    if (S > s_max) return fail(KRILL_ERR_INVALID, "row %d longer than s_max", i);
  }
  const size_t codes = (size_t)n_seqs * g.Hkv * s_max * g.D;
  const size_t meta = (size_t)n_seqs * g.Hkv * s_max * g.NG * 2;
  if (keys) CUDA_TRY(cudaMemsetAsync(keys, 0, codes, st));
  if (values) CUDA_TRY(cudaMemsetAsync(values, 0, codes, st));
  for (void* m : {key_scales, key_zeros, value_scales, value_zeros})
    if (m) CUDA_TRY(cudaMemsetAsync(m, 0, meta, st));
  for (int i = 0; i < n_seqs; ++i) {
    int64_t p0, S;
    layer_span(p, *sv[i], layer, &p0, &S);
    if (S == 0) continue;
    StageSlot* slot;
    TRY(upload_bt(p, *sv[i], st, &slot));
    const size_t co = (size_t)i * g.Hkv * s_max * g.D, mo = (size_t)i * g.Hkv * s_max * g.NG;
    GatherOut o{};
    o.keys = keys ? (uint8_t*)keys + co : nullptr;
    o.values = values ? (uint8_t*)values + co : nullptr;
    o.key_scales = key_scales ? (uint16_t*)key_scales + mo : nullptr;
    o.key_zeros = key_zeros ? (uint16_t*)key_zeros + mo : nullptr;
    o.value_scales = value_scales ? (uint16_t*)value_scales + mo : nullptr;
    o.value_zeros = value_zeros ? (uint16_t*)value_zeros + mo : nullptr;
    o.row_off = s_max - S;
    o.rows_total = s_max;
    o.mode = 0;
    CUDA_TRY(launch_gather(g, p->d_pool, layer, reinterpret_cast<const int32_t*>(slot->d), p0, S, o, st));
    p->kernels += 1;
    TRY(stage_release(slot, st));
  }
  return KRILL_OK;
}

krill_status_t krill_scatter_back(krill_pool_t p, int32_t n_seqs, const krill_seq_t* seqs,
                                  int32_t layer, const int64_t* base_lens, int64_t s_max,
                                  int64_t steps, const void* keys, const void* values,
                                  const void* key_scales, const void* key_zeros,
                                  const void* value_scales, const void* value_zeros,
                                  void* stream) {
  if (!p) return fail(KRILL_ERR_INVALID, "null pool");
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  if (p->geom.fmt != kFmtInt8) return fail(KRILL_ERR_INVALID, "quantized snapshots need an int8 pool");
  TRY(require_device(p));
  DeviceGuard dg(p->device);
  if (layer < 0 || layer >= p->geom.L) return fail(KRILL_ERR_INVALID, "bad layer");
  if (n_seqs <= 0) return KRILL_OK;
  if (!base_lens || steps < 0) return fail(KRILL_ERR_INVALID, "bad base_lens/steps");
  const Geom& g = p->geom;
  const int64_t width = s_max + steps;
  for (int i = 0; i < n_seqs; ++i) {
    Seq* s = nullptr;
    TRY(seq_get(p, seqs[i], &s));
    if (base_lens[i] < 0 || base_lens[i] > s_max) return fail(KRILL_ERR_INVALID, "bad base_len");
    const int64_t rows = base_lens[i] + steps;
    const size_t co = (size_t)i * g.Hkv * width * g.D, mo = (size_t)i * g.Hkv * width * g.NG;
    ScatterIn in{};
    in.keys = (const uint8_t*)keys + co;
    in.values = (const uint8_t*)values + co;
    in.key_scales = (const uint16_t*)key_scales + mo;
    in.key_zeros = (const uint16_t*)key_zeros + mo;
    in.value_scales = (const uint16_t*)value_scales + mo;
    in.value_zeros = (const uint16_t*)value_zeros + mo;
    in.row_off = s_max - base_lens[i];
    in.rows_total = width;
    int64_t total_seen = rows;
    if (p->windowed()) total_seen = std::max<int64_t>(s->len[layer], rows);
    TRY(do_restore(p, *s, layer, std::min<int64_t>(rows, p->windowed() ? p->ring_tokens() : rows),
                   total_seen, in, (cudaStream_t)stream));
  }
  return KRILL_OK;
}

krill_status_t krill_build_decode_mask(const int64_t* lengths, int32_t n, int64_t s_max,
                                       int64_t total_len, float* out) {
  if (n < 0 || (n > 0 && (!lengths || !out)) || total_len < s_max)
    return fail(KRILL_ERR_INVALID, "bad mask arguments");
  for (int r = 0; r < n; ++r) {
    const int64_t pad = s_max - lengths[r];
    for (int64_t j = 0; j < total_len; ++j) out[(int64_t)r * total_len + j] = (j < pad) ? -10000.0f : 0.0f;
  }
  return KRILL_OK;
}

}  // extern "C"

// =====================================================================
// Prefix cache
// =====================================================================
struct krill_prefix_entry_s {
  std::atomic<int> refs{1};  // one for the cache map + one per outstanding hit
  uint64_t key = 0;
  std::vector<int64_t> tokens;
  std::string model, media;
  std::vector<int32_t> blocks;
  std::vector<int64_t> len, ret;
  int64_t n_tokens = 0;
};

struct DiskTier;

struct krill_prefix_s {
  krill_pool_t pool = nullptr;
  int max_entries = 8;
  int min_len = 8;
  std::unordered_map<uint64_t, krill_prefix_entry_t> map;
  std::list<uint64_t> lru;  // front = least recently used
  std::mutex mu;
  DiskTier* disk = nullptr;  // persistent tier, null when disabled
};

namespace {

constexpr uint8_t kKeySchema = 3;
constexpr uint8_t kDtypeInt8 = 2;

// FNV-1a 64 state after the key header (schema, dtype, model, 0xFF, media, 0xFF).
uint64_t key_header(const char* model, const char* media, int dtype_tag) {
  uint64_t h = 14695981039346656037ull;
  auto mix = [&](uint8_t b) {
    h ^= b;
    h *= 1099511628211ull;
  };
  mix(kKeySchema);
  mix((uint8_t)dtype_tag);
  for (const char* c = model ? model : ""; *c; ++c) mix((uint8_t)*c);
  mix(0xFF);
  if (media)
    for (const char* c = media; *c; ++c) mix((uint8_t)*c);
  mix(0xFF);
  return h;
}
uint64_t key_extend(uint64_t h, int64_t token) {
  uint64_t t = (uint64_t)token;
  for (int i = 0; i < 8; ++i) {
    h ^= (uint8_t)(t >> (8 * i));
    h *= 1099511628211ull;
  }
  return h;
}

void entry_unref(krill_prefix_t pc, krill_prefix_entry_t e) {
  if (e->refs.fetch_sub(1) == 1) {
    std::lock_guard<std::recursive_mutex> lk(pc->pool->mu);
    for (int32_t b : e->blocks) block_unref(pc->pool, b);
    delete e;
  }
}

void lru_touch(krill_prefix_t pc, uint64_t key) {
  pc->lru.remove(key);
  pc->lru.push_back(key);
}

void evict_locked(krill_prefix_t pc, uint64_t key) {
  auto it = pc->map.find(key);
  if (it == pc->map.end()) return;
  krill_prefix_entry_t e = it->second;
  pc->map.erase(it);
  pc->lru.remove(key);
  entry_unref(pc, e);
}

// ---------------------------------------------------------------------
// Disk tier (PrefixCache.swift:496-501 file naming, :553-581 load, :583-648
// write + byte budget, :650-695 LRU eviction to a 90 % low-water mark). An
// int8 entry is one safetensors file `<key %016llx>.q8.safetensors` holding,
// per layer i, `layer_{i}_qk` / `_qv` (U8 [1, Hkv, S, D]) and `_ks` / `_kz` /
// `_vs` / `_vz` (F16 [1, Hkv, S, D/G]): the reference's names, dtypes and
// shapes (G = D is the reference's one-scale-per-head layout). Writes run on a
// per-cache worker thread (the reference's serial disk queue); a disk hit is
// read back into pool blocks through the restore kernel. Disk-loaded entries
// carry no tokens, so longest-prefix matching skips them, as in the reference.
struct StTensor {
  std::string dtype;
  std::vector<int64_t> shape;
  int64_t begin = 0, end = 0;
};

// Minimal JSON reader for a safetensors header: an object of tensor records
// ({"dtype", "shape", "data_offsets"}) plus an optional "__metadata__".
struct JsonCursor {
  const std::string& s;
  size_t i = 0;
  void ws() {
    while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
  }
  bool eat(char c) {
    ws();
    if (i < s.size() && s[i] == c) {
      ++i;
      return true;
    }
    return false;
  }
  bool str(std::string& out) {
    ws();
    if (i >= s.size() || s[i] != '"') return false;
    ++i;
    out.clear();
    while (i < s.size() && s[i] != '"') {
      if (s[i] == '\\') {
        if (i + 1 >= s.size()) return false;
        const char c = s[i + 1];
        if (c == 'u') {  // tensor names are ASCII; keep a placeholder
          if (i + 5 >= s.size()) return false;
          out += '?';
          i += 6;
          continue;
        }
        out += c == 'n' ? '\n' : c == 't' ? '\t' : c;
        i += 2;
        continue;
      }
      out += s[i++];
    }
    if (i >= s.size()) return false;
    ++i;
    return true;
  }
  bool num(int64_t& v) {
    ws();
    size_t j = i;
    if (j < s.size() && s[j] == '-') ++j;
    if (j >= s.size() || s[j] < '0' || s[j] > '9') return false;
    while (j < s.size() && s[j] >= '0' && s[j] <= '9') ++j;
    v = std::strtoll(s.c_str() + i, nullptr, 10);
    i = j;
    return true;
  }
  bool skip() {
    ws();
    if (i >= s.size()) return false;
    const char c = s[i];
    if (c == '"') {
      std::string t;
      return str(t);
    }
    if (c == '{') {
      ++i;
      if (eat('}')) return true;
      do {
        std::string k;
        if (!str(k) || !eat(':') || !skip()) return false;
      } while (eat(','));
      return eat('}');
    }
    if (c == '[') {
      ++i;
      if (eat(']')) return true;
      do {
        if (!skip()) return false;
      } while (eat(','));
      return eat(']');
    }
    const size_t j = i;
    while (i < s.size() && (isalnum((unsigned char)s[i]) || s[i] == '-' || s[i] == '+' || s[i] == '.')) ++i;
    return i > j;
  }
};

bool parse_st_header(const std::string& js, std::map<std::string, StTensor>* out) {
  JsonCursor p{js};
  if (!p.eat('{')) return false;
  if (p.eat('}')) return true;
  do {
    std::string name;
    if (!p.str(name) || !p.eat(':')) return false;
    if (name == "__metadata__") {
      if (!p.skip()) return false;
      continue;
    }
    StTensor t;
    if (!p.eat('{')) return false;
    if (!p.eat('}')) {
      do {
        std::string f;
        if (!p.str(f) || !p.eat(':')) return false;
        if (f == "dtype") {
          if (!p.str(t.dtype)) return false;
        } else if (f == "shape") {
          if (!p.eat('[')) return false;
          if (!p.eat(']')) {
            do {
              int64_t v;
              if (!p.num(v)) return false;
              t.shape.push_back(v);
            } while (p.eat(','));
            if (!p.eat(']')) return false;
          }
        } else if (f == "data_offsets") {
          int64_t a, b;
          if (!p.eat('[') || !p.num(a) || !p.eat(',') || !p.num(b) || !p.eat(']')) return false;
          t.begin = a;
          t.end = b;
        } else if (!p.skip()) {
          return false;
        }
      } while (p.eat(','));
      if (!p.eat('}')) return false;
    }
    (*out)[name] = t;
  } while (p.eat(','));
  return p.eat('}');
}

}  // namespace

struct DiskTier {
  krill_prefix_t pc = nullptr;
  std::string dir;
  int64_t budget = 0;  // bytes; < 0 unbounded
  std::thread worker;
  std::mutex mu;  // queue, counters
  std::condition_variable cv, idle;
  std::deque<krill_prefix_entry_t> queue;
  int busy = 0;
  bool stop = false;
  int64_t counter = 0;
  bool seeded = false;
  cudaStream_t wstream = nullptr, lstream = nullptr;
  uint8_t* d_w = nullptr;  // writer device scratch: block table + one layer
  size_t d_w_cap = 0;
  uint8_t* h_w = nullptr;  // writer pinned host buffer: one layer
  size_t h_w_cap = 0;
  std::mutex lmu;  // loader scratch
  uint8_t* d_l = nullptr;
  size_t d_l_cap = 0;
};

namespace {

namespace fs = std::filesystem;

std::string disk_path(const DiskTier* dt, uint64_t key) {
  char name[40];
  std::snprintf(name, sizeof(name), "%016llx.q8.safetensors", (unsigned long long)key);
  return dt->dir + "/" + name;
}

// Bytes of one layer of an S-token entry: codes K, V, then K/V scale and zero.
int64_t disk_layer_bytes(const Geom& g, int64_t S) {
  return 2 * (int64_t)g.Hkv * S * g.D + 8 * (int64_t)g.Hkv * S * g.NG;
}

std::string st_header(const Geom& g, int64_t S) {
  std::string h = "{";
  int64_t off = 0;
  const int64_t codes = (int64_t)g.Hkv * S * g.D, meta = (int64_t)g.Hkv * S * g.NG * 2;
  const char* names[6] = {"qk", "qv", "ks", "kz", "vs", "vz"};
  char buf[256];
  for (int L = 0; L < g.L; ++L)
    for (int a = 0; a < 6; ++a) {
      const bool c = a < 2;
      const int64_t n = c ? codes : meta;
      std::snprintf(buf, sizeof(buf),
                    "%s\"layer_%d_%s\":{\"dtype\":\"%s\",\"shape\":[1,%d,%lld,%d],\"data_offsets\":[%lld,%lld]}",
                    h.size() > 1 ? "," : "", L, names[a], c ? "U8" : "F16", g.Hkv, (long long)S,
                    c ? g.D : g.NG, (long long)off, (long long)(off + n));
      h += buf;
      off += n;
    }
  h += "}";
  while (h.size() % 8) h += ' ';
  return h;
}

void disk_evict_to_low_water(DiskTier* dt) {
  if (dt->budget <= 0) return;
  const int64_t low = dt->budget - dt->budget / 10;
  std::vector<std::pair<fs::file_time_type, std::pair<fs::path, int64_t>>> files;
  int64_t total = 0;
  std::error_code ec;
  for (const auto& de : fs::directory_iterator(dt->dir, ec)) {
    if (de.path().extension() != ".safetensors") continue;
    const int64_t sz = (int64_t)de.file_size(ec);
    files.push_back({de.last_write_time(ec), {de.path(), sz}});
    total += sz;
  }
  if (total > dt->budget) {
    std::sort(files.begin(), files.end(),
              [](const auto& a, const auto& b) { return a.first < b.first; });
    for (const auto& f : files) {
      if (total <= low) break;
      if (fs::remove(f.second.first, ec)) total -= f.second.second;
    }
  }
  dt->counter = total;
  dt->seeded = true;
}

int64_t disk_scan_bytes(const DiskTier* dt) {
  int64_t total = 0;
  std::error_code ec;
  for (const auto& de : fs::directory_iterator(dt->dir, ec))
    if (de.path().extension() == ".safetensors") total += (int64_t)de.file_size(ec);
  return total;
}

// Worker: gather every layer of the entry (gather kernel, mode 0) and write
// the file under a temporary name, then rename it into place.
bool disk_write_entry(DiskTier* dt, krill_prefix_entry_t e) {
  krill_pool_t p = dt->pc->pool;
  const Geom& g = p->geom;
  const int64_t S = e->n_tokens;
  if (S <= 0) return false;
  const int64_t lb = disk_layer_bytes(g, S);
  const size_t nb = e->blocks.size();
  const size_t bt_bytes = (nb * sizeof(int32_t) + 255) & ~size_t(255);
  if (cudaSetDevice(p->device) != cudaSuccess) return false;
  if (dt->d_w_cap < bt_bytes + (size_t)lb) {
    if (dt->d_w) cudaFree(dt->d_w);
    dt->d_w = nullptr;
    dt->d_w_cap = 0;
    if (cudaMalloc(&dt->d_w, bt_bytes + (size_t)lb) != cudaSuccess) return false;
    dt->d_w_cap = bt_bytes + (size_t)lb;
  }
  if (dt->h_w_cap < (size_t)lb) {
    if (dt->h_w) cudaFreeHost(dt->h_w);
    dt->h_w = nullptr;
    dt->h_w_cap = 0;
    if (cudaMallocHost(&dt->h_w, (size_t)lb) != cudaSuccess) return false;
    dt->h_w_cap = (size_t)lb;
  }
  const std::string path = disk_path(dt, e->key), tmp = path + ".tmp";
  FILE* f = std::fopen(tmp.c_str(), "wb");
  if (!f) return false;
  const std::string hdr = st_header(g, S);
  const uint64_t hl = hdr.size();
  bool ok = std::fwrite(&hl, 8, 1, f) == 1 && std::fwrite(hdr.data(), 1, hdr.size(), f) == hdr.size();
  ok = ok && cudaMemcpyAsync(dt->d_w, e->blocks.data(), nb * sizeof(int32_t), cudaMemcpyHostToDevice,
                             dt->wstream) == cudaSuccess;
  const int64_t codes = (int64_t)g.Hkv * S * g.D, meta = (int64_t)g.Hkv * S * g.NG * 2;
  uint8_t* d = dt->d_w + bt_bytes;
  for (int L = 0; ok && L < g.L; ++L) {
    GatherOut o{};
    o.keys = d;
    o.values = d + codes;
    o.key_scales = reinterpret_cast<uint16_t*>(d + 2 * codes);
    o.key_zeros = reinterpret_cast<uint16_t*>(d + 2 * codes + meta);
    o.value_scales = reinterpret_cast<uint16_t*>(d + 2 * codes + 2 * meta);
    o.value_zeros = reinterpret_cast<uint16_t*>(d + 2 * codes + 3 * meta);
    o.row_off = 0;
    o.rows_total = S;
    o.mode = 0;
    ok = launch_gather(g, p->d_pool, L, reinterpret_cast<const int32_t*>(dt->d_w), 0, S, o,
                       dt->wstream) == cudaSuccess &&
         cudaMemcpyAsync(dt->h_w, d, (size_t)lb, cudaMemcpyDeviceToHost, dt->wstream) == cudaSuccess &&
         cudaStreamSynchronize(dt->wstream) == cudaSuccess &&
         std::fwrite(dt->h_w, 1, (size_t)lb, f) == (size_t)lb;
  }
  ok = (std::fclose(f) == 0) && ok;
  std::error_code ec;
  if (!ok) {
    fs::remove(tmp, ec);
    return false;
  }
  const int64_t prior = fs::exists(path, ec) ? (int64_t)fs::file_size(path, ec) : 0;
  fs::rename(tmp, path, ec);
  if (ec) {
    fs::remove(tmp, ec);
    return false;
  }
  const int64_t now = (int64_t)fs::file_size(path, ec);
  bool over;
  {
    std::lock_guard<std::mutex> lk(dt->mu);
    if (!dt->seeded) {
      dt->counter = disk_scan_bytes(dt);
      dt->seeded = true;
    } else {
      dt->counter += now - prior;
    }
    over = dt->budget > 0 && dt->counter > dt->budget;
    if (over) disk_evict_to_low_water(dt);
  }
  return true;
}

void disk_worker(DiskTier* dt) {
  for (;;) {
    krill_prefix_entry_t e;
    {
      std::unique_lock<std::mutex> lk(dt->mu);
      dt->cv.wait(lk, [&] { return dt->stop || !dt->queue.empty(); });
      if (dt->queue.empty()) return;  // stop requested and drained
      e = dt->queue.front();
      dt->queue.pop_front();
      dt->busy += 1;
    }
    disk_write_entry(dt, e);
    entry_unref(dt->pc, e);
    {
      std::lock_guard<std::mutex> lk(dt->mu);
      dt->busy -= 1;
      if (dt->queue.empty() && dt->busy == 0) dt->idle.notify_all();
    }
  }
}

void disk_wait(DiskTier* dt) {
  std::unique_lock<std::mutex> lk(dt->mu);
  dt->idle.wait(lk, [&] { return dt->queue.empty() && dt->busy == 0; });
}

void disk_shutdown(DiskTier* dt) {
  {
    std::lock_guard<std::mutex> lk(dt->mu);
    dt->stop = true;
  }
  dt->cv.notify_all();
  if (dt->worker.joinable()) dt->worker.join();
  cudaSetDevice(dt->pc->pool->device);
  if (dt->wstream) cudaStreamDestroy(dt->wstream);
  if (dt->lstream) cudaStreamDestroy(dt->lstream);
  if (dt->d_w) cudaFree(dt->d_w);
  if (dt->h_w) cudaFreeHost(dt->h_w);
  if (dt->d_l) cudaFree(dt->d_l);
  delete dt;
}

// Disk probe of one key: a missing or unreadable file, or one whose shapes do
// not fit this pool, is a miss (KRILL_ERR_NOT_FOUND); a hit is read into new
// pool blocks (restore kernel) and returned as an entry holding one map
// reference. The file's modification time is refreshed (the LRU recency).
krill_status_t disk_load(DiskTier* dt, uint64_t key, int64_t S, const char* model, const char* media,
                         krill_prefix_entry_t* out) {
  krill_pool_t p = dt->pc->pool;
  const Geom& g = p->geom;
  const std::string path = disk_path(dt, key);
  std::error_code ec;
  if (!fs::exists(path, ec)) return KRILL_ERR_NOT_FOUND;
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f) return KRILL_ERR_NOT_FOUND;
  uint64_t hl = 0;
  std::string hdr;
  std::vector<uint8_t> data;
  bool ok = std::fread(&hl, 8, 1, f) == 1 && hl < (uint64_t)1 << 28;
  if (ok) {
    hdr.resize(hl);
    ok = std::fread(&hdr[0], 1, hl, f) == hl;
  }
  std::map<std::string, StTensor> ts;
  ok = ok && parse_st_header(hdr, &ts);
  const int64_t lb = disk_layer_bytes(g, S);
  const int64_t codes = (int64_t)g.Hkv * S * g.D, meta = (int64_t)g.Hkv * S * g.NG * 2;
  // every layer present with this pool's shapes
  const char* names[6] = {"qk", "qv", "ks", "kz", "vs", "vz"};
  int64_t max_end = 0;
  for (int L = 0; ok && L < g.L; ++L)
    for (int a = 0; ok && a < 6; ++a) {
      auto it = ts.find("layer_" + std::to_string(L) + "_" + names[a]);
      if (it == ts.end()) {
        ok = false;
        break;
      }
      const StTensor& t = it->second;
      const bool c = a < 2;
      ok = t.dtype == (c ? "U8" : "F16") && t.shape.size() == 4 && t.shape[0] == 1 &&
           t.shape[1] == g.Hkv && t.shape[2] == S && t.shape[3] == (c ? g.D : g.NG) &&
           t.end - t.begin == (c ? codes : meta) && t.begin >= 0;
      max_end = std::max(max_end, t.end);
    }
  ok = ok && ts.count("layer_" + std::to_string(g.L) + "_qk") == 0;  // no extra layers
  if (ok) {
    data.resize((size_t)max_end);
    ok = std::fread(data.data(), 1, data.size(), f) == data.size();
  }
  std::fclose(f);
  if (!ok) return KRILL_ERR_NOT_FOUND;

  std::lock_guard<std::mutex> llk(dt->lmu);
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  DeviceGuard dg(p->device);
  if (dt->d_l_cap < (size_t)lb) {
    if (dt->d_l) cudaFree(dt->d_l);
    dt->d_l = nullptr;
    dt->d_l_cap = 0;
    CUDA_TRY(cudaMalloc(&dt->d_l, (size_t)lb));
    dt->d_l_cap = (size_t)lb;
  }
  krill_seq_t h;
  Seq* s = nullptr;
  TRY(seq_new(p, &h, &s));
  krill_status_t st = KRILL_OK;
  for (int L = 0; st == KRILL_OK && L < g.L; ++L) {
    uint8_t* d = dt->d_l;
    const std::string pre = "layer_" + std::to_string(L) + "_";
    const int64_t offs[6] = {0, codes, 2 * codes, 2 * codes + meta, 2 * codes + 2 * meta,
                             2 * codes + 3 * meta};
    for (int a = 0; a < 6 && st == KRILL_OK; ++a) {
      const StTensor& t = ts[pre + names[a]];
      if (cudaMemcpyAsync(d + offs[a], data.data() + t.begin, (size_t)(t.end - t.begin),
                          cudaMemcpyHostToDevice, dt->lstream) != cudaSuccess)
        st = fail(KRILL_ERR_CUDA, "disk tier upload failed");
    }
    if (st != KRILL_OK) break;
    ScatterIn in{};
    in.keys = d;
    in.values = d + codes;
    in.key_scales = reinterpret_cast<const uint16_t*>(d + offs[2]);
    in.key_zeros = reinterpret_cast<const uint16_t*>(d + offs[3]);
    in.value_scales = reinterpret_cast<const uint16_t*>(d + offs[4]);
    in.value_zeros = reinterpret_cast<const uint16_t*>(d + offs[5]);
    in.row_off = 0;
    in.rows_total = S;
    st = do_restore(p, *s, L, S, S, in, dt->lstream);
    // the layer scratch is reused by the next layer
    if (st == KRILL_OK && cudaStreamSynchronize(dt->lstream) != cudaSuccess)
      st = fail(KRILL_ERR_CUDA, "disk tier restore failed");
  }
  if (st == KRILL_OK) {
    auto* e = new krill_prefix_entry_s();
    const size_t nb = (size_t)((S + kBlockTokens - 1) / kBlockTokens);
    e->blocks.assign(s->blocks.begin(), s->blocks.begin() + nb);
    for (int32_t b : e->blocks) block_ref(p, b);
    e->len.assign(g.L, S);
    e->ret.assign(g.L, S);
    e->n_tokens = S;
    e->key = key;
    e->model = model ? model : "";
    e->media = media ? media : "";
    *out = e;
    fs::last_write_time(path, fs::file_time_type::clock::now(), ec);
  }
  seq_drop_blocks(p, *s);
  s->alive = false;
  s->len.clear();
  s->ret.clear();
  p->free_slots.push_back((uint32_t)(h & 0xffffffffu));
  return st;
}

}  // namespace

extern "C" {

uint64_t krill_prefix_key(const int64_t* tokens, int64_t n, const char* model_id,
                          const char* media_hash, int32_t dtype_tag) {
  uint64_t h = key_header(model_id, media_hash, dtype_tag);
  for (int64_t i = 0; i < n; ++i) h = key_extend(h, tokens[i]);
  return h;
}

krill_status_t krill_prefix_create(krill_pool_t pool, int32_t max_entries, int32_t min_len,
                                   krill_prefix_t* out) {
  if (!pool || !out) return fail(KRILL_ERR_INVALID, "null argument");
  if (max_entries <= 0) return fail(KRILL_ERR_INVALID, "max_memory_entries must be positive");
  auto* pc = new krill_prefix_s();
  pc->pool = pool;
  pc->max_entries = max_entries;
  pc->min_len = std::max(1, min_len);
  *out = pc;
  return KRILL_OK;
}

krill_status_t krill_prefix_clear(krill_prefix_t pc) {
  if (!pc) return fail(KRILL_ERR_INVALID, "null prefix cache");
  {
    std::lock_guard<std::mutex> lk(pc->mu);
    std::vector<uint64_t> keys;
    for (auto& kv : pc->map) keys.push_back(kv.first);
    for (uint64_t k : keys) evict_locked(pc, k);
  }
  if (pc->disk) {  // and the disk tier's files (PrefixCache.swift:403-415)
    DiskTier* dt = pc->disk;
    disk_wait(dt);
    std::error_code ec;
    for (const auto& de : std::filesystem::directory_iterator(dt->dir, ec)) {
      const std::string name = de.path().filename().string();
      if (name.size() > 12 && (name.compare(name.size() - 12, 12, ".safetensors") == 0 ||
                               name.compare(name.size() - 4, 4, ".tmp") == 0))
        std::filesystem::remove(de.path(), ec);
    }
    std::lock_guard<std::mutex> lk(dt->mu);
    dt->counter = 0;
    dt->seeded = true;
  }
  return KRILL_OK;
}

krill_status_t krill_prefix_set_disk(krill_prefix_t pc, const char* cache_dir, int64_t budget_bytes) {
  if (!pc) return fail(KRILL_ERR_INVALID, "null prefix cache");
  if (pc->disk) {
    disk_shutdown(pc->disk);
    pc->disk = nullptr;
  }
  if (budget_bytes == 0) return KRILL_OK;  // disabled (PrefixCache.swift:585)
  if (!cache_dir || !*cache_dir) return fail(KRILL_ERR_INVALID, "empty cache_dir");
  krill_pool_t p = pc->pool;
  if (p->host_only) return fail(KRILL_ERR_NO_DEVICE, "the disk tier needs a device pool");
  if (p->geom.fmt != kFmtInt8) return fail(KRILL_ERR_INVALID, "the disk tier stores int8 pools");
  std::error_code ec;
  std::filesystem::create_directories(cache_dir, ec);
  if (ec) return fail(KRILL_ERR_INVALID, "cannot create %s: %s", cache_dir, ec.message().c_str());
  auto* dt = new DiskTier();
  dt->pc = pc;
  dt->dir = cache_dir;
  dt->budget = budget_bytes;
  DeviceGuard dg(p->device);
  if (cudaStreamCreateWithFlags(&dt->wstream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&dt->lstream, cudaStreamNonBlocking) != cudaSuccess) {
    if (dt->wstream) cudaStreamDestroy(dt->wstream);
    delete dt;
    return fail(KRILL_ERR_CUDA, "cannot create disk-tier streams");
  }
  dt->worker = std::thread(disk_worker, dt);
  pc->disk = dt;
  return KRILL_OK;
}

krill_status_t krill_prefix_wait_disk(krill_prefix_t pc) {
  if (!pc) return fail(KRILL_ERR_INVALID, "null prefix cache");
  if (pc->disk) disk_wait(pc->disk);
  return KRILL_OK;
}

krill_status_t krill_prefix_disk_count(krill_prefix_t pc, int32_t* count) {
  if (!pc || !count) return fail(KRILL_ERR_INVALID, "null argument");
  *count = 0;
  if (!pc->disk) return KRILL_OK;
  std::error_code ec;
  for (const auto& de : std::filesystem::directory_iterator(pc->disk->dir, ec))
    if (de.path().extension() == ".safetensors") *count += 1;
  return KRILL_OK;
}

krill_status_t krill_prefix_destroy(krill_prefix_t pc) {
  if (!pc) return KRILL_OK;
  if (pc->disk) {  // finish pending writes, keep the files
    disk_shutdown(pc->disk);
    pc->disk = nullptr;
  }
  {
    std::lock_guard<std::mutex> lk(pc->mu);
    std::vector<uint64_t> keys;
    for (auto& kv : pc->map) keys.push_back(kv.first);
    for (uint64_t k : keys) evict_locked(pc, k);
  }
  delete pc;
  return KRILL_OK;
}

krill_status_t krill_prefix_memory_count(krill_prefix_t pc, int32_t* count) {
  if (!pc || !count) return fail(KRILL_ERR_INVALID, "null argument");
  std::lock_guard<std::mutex> lk(pc->mu);
  *count = (int32_t)pc->map.size();
  return KRILL_OK;
}

static void insert_locked(krill_prefix_t pc, krill_prefix_entry_t e) {
  auto it = pc->map.find(e->key);
  if (it != pc->map.end()) evict_locked(pc, e->key);  // same key: replace
  while ((int)pc->map.size() >= pc->max_entries && !pc->lru.empty())
    evict_locked(pc, pc->lru.front());
  pc->map[e->key] = e;
  pc->lru.push_back(e->key);
}

krill_status_t krill_prefix_store(krill_prefix_t pc, krill_seq_t seq, const int64_t* tokens,
                                  int64_t n, const char* model_id, const char* media_hash) {
  if (!pc) return fail(KRILL_ERR_INVALID, "null prefix cache");
  if (n < pc->min_len) return KRILL_OK;  // PrefixCache.storeQuantized guard (:375)
  if (!tokens) return fail(KRILL_ERR_INVALID, "null tokens");
  krill_pool_t p = pc->pool;
  auto* e = new krill_prefix_entry_s();
  {
    std::lock_guard<std::recursive_mutex> lk(p->mu);
    Seq* s = nullptr;
    krill_status_t st = seq_get(p, seq, &s);
    if (st != KRILL_OK) {
      delete e;
      return st;
    }
    for (int L = 0; L < p->geom.L; ++L) {
      const bool ok = p->windowed() ? s->len[L] == n : s->len[L] >= n;
      if (!ok) {
        delete e;
        return fail(KRILL_ERR_INVALID, "layer %d holds %lld tokens, cannot store a %lld-token prefix",
                    L, (long long)s->len[L], (long long)n);
      }
    }
    if (p->windowed()) {
      e->blocks = s->blocks;
      e->len = s->len;
      e->ret = s->ret;
    } else {
      const size_t nb = (size_t)((n + kBlockTokens - 1) / kBlockTokens);
      e->blocks.assign(s->blocks.begin(), s->blocks.begin() + nb);
      e->len.assign(p->geom.L, n);
      e->ret.assign(p->geom.L, n);
    }
    for (int32_t b : e->blocks)
      if (b >= 0) block_ref(p, b);
  }
  e->tokens.assign(tokens, tokens + n);
  e->model = model_id ? model_id : "";
  e->media = media_hash ? media_hash : "";
  e->n_tokens = n;
  e->key = krill_prefix_key(tokens, n, model_id, media_hash, kDtypeInt8);
  {
    std::lock_guard<std::mutex> lk(pc->mu);
    insert_locked(pc, e);
    if (pc->disk && !p->windowed()) e->refs.fetch_add(1);  // held by the disk writer
  }
  if (pc->disk && !p->windowed()) {  // write-behind (PrefixCache.swift:396-399)
    {
      std::lock_guard<std::mutex> lk(pc->disk->mu);
      pc->disk->queue.push_back(e);
    }
    pc->disk->cv.notify_one();
  }
  return KRILL_OK;
}

krill_status_t krill_prefix_lookup(krill_prefix_t pc, const int64_t* tokens, int64_t n,
                                   const char* model_id, const char* media_hash,
                                   krill_prefix_entry_t* entry, int64_t* prefix_length) {
  if (!pc || !entry || !prefix_length) return fail(KRILL_ERR_INVALID, "null argument");
  *entry = nullptr;
  *prefix_length = 0;
  if (n < pc->min_len || !tokens) return KRILL_ERR_NOT_FOUND;
  // Running FNV-1a over the tokens gives the key of every prefix length in one
  // pass; probe in the reference's scan order (PrefixCache.swift:283-305).
  std::vector<uint64_t> keys((size_t)n + 1);
  keys[0] = key_header(model_id, media_hash, kDtypeInt8);
  for (int64_t i = 0; i < n; ++i) keys[i + 1] = key_extend(keys[i], tokens[i]);
  const int64_t step = std::max(1, pc->min_len / 2);
  for (int64_t check = n; check >= pc->min_len; check -= step) {
    {
      std::lock_guard<std::mutex> lk(pc->mu);
      auto it = pc->map.find(keys[check]);
      if (it != pc->map.end()) {
        lru_touch(pc, it->first);
        it->second->refs.fetch_add(1);
        *entry = it->second;
        *prefix_length = check;
        return KRILL_OK;
      }
    }
    // then the disk tier, with the map unlocked (PrefixCache.swift:296-301)
    if (pc->disk && !pc->pool->windowed()) {
      krill_prefix_entry_t e = nullptr;
      const krill_status_t st = disk_load(pc->disk, keys[check], check, model_id, media_hash, &e);
      if (st == KRILL_OK) {
        std::lock_guard<std::mutex> lk(pc->mu);
        insert_locked(pc, e);
        e->refs.fetch_add(1);
        *entry = e;
        *prefix_length = check;
        return KRILL_OK;
      }
      if (st != KRILL_ERR_NOT_FOUND) return st;
    }
  }
  return KRILL_ERR_NOT_FOUND;
}

krill_status_t krill_prefix_lookup_longest(krill_prefix_t pc, const int64_t* tokens, int64_t n,
                                           const char* model_id, const char* media_hash,
                                           krill_prefix_entry_t* entry, int64_t* prefix_length) {
  if (!pc || !entry || !prefix_length) return fail(KRILL_ERR_INVALID, "null argument");
  *entry = nullptr;
  *prefix_length = 0;
  if (n < pc->min_len || !tokens) return KRILL_ERR_NOT_FOUND;
  const std::string model = model_id ? model_id : "", media = media_hash ? media_hash : "";
  std::lock_guard<std::mutex> lk(pc->mu);
  krill_prefix_entry_t best = nullptr;
  int64_t best_len = 0;
  for (auto& kv : pc->map) {
    krill_prefix_entry_t e = kv.second;
    if (e->model != model || e->media != media || e->tokens.empty()) continue;
    const int64_t m = std::min<int64_t>(n, (int64_t)e->tokens.size());
    int64_t i = 0;
    while (i < m && tokens[i] == e->tokens[i]) ++i;
    if (i >= pc->min_len && i > best_len) {
      best_len = i;
      best = e;
    }
  }
  if (!best) return KRILL_ERR_NOT_FOUND;
  lru_touch(pc, best->key);
  best->refs.fetch_add(1);
  *entry = best;
  *prefix_length = best_len;
  return KRILL_OK;
}

krill_status_t krill_prefix_entry_length(krill_prefix_entry_t e, int64_t* stored_length) {
  if (!e || !stored_length) return fail(KRILL_ERR_INVALID, "null argument");
  *stored_length = e->n_tokens;
  return KRILL_OK;
}

krill_status_t krill_prefix_entry_release(krill_prefix_t pc, krill_prefix_entry_t e) {
  if (!pc || !e) return fail(KRILL_ERR_INVALID, "null argument");
  entry_unref(pc, e);
  return KRILL_OK;
}

krill_status_t krill_seq_fork_prefix(krill_prefix_t pc, krill_prefix_entry_t e, int64_t keep,
                                     krill_seq_t* out) {
  if (!pc || !e || !out) return fail(KRILL_ERR_INVALID, "null argument");
  krill_pool_t p = pc->pool;
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  if (keep < 0 || keep > e->n_tokens)
    return fail(KRILL_ERR_INVALID, "keep %lld outside [0, %lld]", (long long)keep, (long long)e->n_tokens);
  if (p->windowed())
    for (int L = 0; L < p->geom.L; ++L)
      if (keep < e->len[L] - e->ret[L])
        return fail(KRILL_ERR_INVALID, "keep %lld below the retained window of layer %d",
                    (long long)keep, L);
  Seq* s = nullptr;
  TRY(seq_new(p, out, &s));
  if (p->windowed()) {
    s->blocks = e->blocks;
    for (int L = 0; L < p->geom.L; ++L) {
      s->len[L] = keep;
      s->ret[L] = e->ret[L] - (e->len[L] - keep);
    }
  } else {
    const size_t nb = (size_t)((keep + kBlockTokens - 1) / kBlockTokens);
    s->blocks.assign(e->blocks.begin(), e->blocks.begin() + nb);
    std::fill(s->len.begin(), s->len.end(), keep);
    std::fill(s->ret.begin(), s->ret.end(), keep);
  }
  for (int32_t b : s->blocks)
    if (b >= 0) block_ref(p, b);
  return KRILL_OK;
}

krill_status_t krill_prefix_peer_fetch(krill_prefix_t dst, krill_prefix_t src,
                                       krill_prefix_entry_t se, void* stream,
                                       krill_prefix_entry_t* out) {
  if (!dst || !src || !se || !out) return fail(KRILL_ERR_INVALID, "null argument");
  krill_pool_t dp = dst->pool, sp = src->pool;
  if (dp->host_only || sp->host_only) return fail(KRILL_ERR_NO_DEVICE, "peer fetch needs device pools");
  const Geom &a = dp->geom, &b = sp->geom;
  if (a.L != b.L || a.Hkv != b.Hkv || a.D != b.D || a.G != b.G || a.ring != b.ring ||
      dp->cfg.window != sp->cfg.window)
    return fail(KRILL_ERR_INVALID, "peer fetch between pools of different geometry");
  auto* e = new krill_prefix_entry_s();
  {
    std::lock_guard<std::recursive_mutex> lk(dp->mu);
    DeviceGuard dg(dp->device);
    if (dp->device != sp->device) {
      int can = 0;
      cudaDeviceCanAccessPeer(&can, dp->device, sp->device);
      if (can) {
        cudaError_t pe = cudaDeviceEnablePeerAccess(sp->device, 0);
        if (pe != cudaSuccess && pe != cudaErrorPeerAccessAlreadyEnabled) {
          delete e;
          return fail(KRILL_ERR_PEER, "cudaDeviceEnablePeerAccess: %s", cudaGetErrorString(pe));
        }
        cudaGetLastError();
      }
    }
    e->blocks.assign(se->blocks.size(), -1);
    for (size_t i = 0; i < se->blocks.size(); ++i) {
      if (se->blocks[i] < 0) continue;
      krill_status_t st = block_alloc(dp, &e->blocks[i]);
      if (st != KRILL_OK) {
        for (int32_t bb : e->blocks) block_unref(dp, bb);
        delete e;
        return st;
      }
      cudaError_t ce = cudaMemcpyPeerAsync(dp->block_ptr(e->blocks[i]), dp->device,
                                           sp->block_ptr(se->blocks[i]), sp->device,
                                           (size_t)a.block_bytes, (cudaStream_t)stream);
      if (ce != cudaSuccess) {
        for (int32_t bb : e->blocks) block_unref(dp, bb);
        delete e;
        return fail(KRILL_ERR_PEER, "cudaMemcpyPeerAsync: %s", cudaGetErrorString(ce));
      }
    }
    // the copied blocks may hold large scales: fold the source pool's flag
    // into this pool's, in stream order (peer copy into a scratch word, then OR)
    cudaError_t ce = cudaMemcpyPeerAsync(dp->d_err + 2, dp->device, sp->d_err + 1, sp->device,
                                         sizeof(int), (cudaStream_t)stream);
    if (ce == cudaSuccess) {
      or_flag_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(dp->d_err + 1, dp->d_err + 2);
      ce = cudaGetLastError();
    }
    if (ce != cudaSuccess) {
      for (int32_t bb : e->blocks) block_unref(dp, bb);
      delete e;
      return fail(KRILL_ERR_PEER, "flag copy: %s", cudaGetErrorString(ce));
    }
    dp->kernels += 1;
  }
  e->key = se->key;
  e->tokens = se->tokens;
  e->model = se->model;
  e->media = se->media;
  e->len = se->len;
  e->ret = se->ret;
  e->n_tokens = se->n_tokens;
  std::lock_guard<std::mutex> lk(dst->mu);
  insert_locked(dst, e);
  e->refs.fetch_add(1);
  *out = e;
  return KRILL_OK;
}

// ---- cross-process fetch (one process per GPU) ----
// Entry descriptor, little-endian: "KKV1", geometry (L, Hkv, D, G, format,
// window, ring, block bytes), key, length, large-scale flag, block ids,
// per-layer length / retained, model id, media hash, tokens.
}  // extern "C"
namespace {
struct DescWriter {
  std::vector<uint8_t> b;
  template <class T>
  void put(T v) {
    const uint8_t* p = reinterpret_cast<const uint8_t*>(&v);
    b.insert(b.end(), p, p + sizeof(T));
  }
  void bytes(const void* p, size_t n) {
    b.insert(b.end(), (const uint8_t*)p, (const uint8_t*)p + n);
  }
};
struct DescReader {
  const uint8_t* p;
  size_t n, i = 0;
  bool ok = true;
  template <class T>
  T get() {
    T v{};
    if (i + sizeof(T) > n) {
      ok = false;
      return v;
    }
    std::memcpy(&v, p + i, sizeof(T));
    i += sizeof(T);
    return v;
  }
  bool bytes(void* out, size_t m) {
    if (i + m > n) return ok = false;
    std::memcpy(out, p + i, m);
    i += m;
    return true;
  }
};
}  // namespace
extern "C" {

krill_status_t krill_pool_ipc_handle(krill_pool_t p, void* handle) {
  if (!p || !handle) return fail(KRILL_ERR_INVALID, "null argument");
  if (p->host_only) return fail(KRILL_ERR_NO_DEVICE, "a host-only pool has no device memory");
  DeviceGuard dg(p->device);
  cudaIpcMemHandle_t h;
  CUDA_TRY(cudaIpcGetMemHandle(&h, p->d_pool));
  std::memcpy(handle, &h, sizeof(h));
  return KRILL_OK;
}

krill_status_t krill_prefix_entry_describe(krill_prefix_t pc, krill_prefix_entry_t e, void* buf,
                                           int64_t cap, int64_t* size) {
  if (!pc || !e || !size) return fail(KRILL_ERR_INVALID, "null argument");
  krill_pool_t p = pc->pool;
  const Geom& g = p->geom;
  int32_t large = 0;
  if (!p->host_only) {
    DeviceGuard dg(p->device);
    CUDA_TRY(cudaDeviceSynchronize());  // appends in flight may still raise the flag
    CUDA_TRY(cudaMemcpy(&large, p->d_err + 1, sizeof(int32_t), cudaMemcpyDeviceToHost));
  }
  DescWriter w;
  w.bytes("KKV1", 4);
  for (int32_t v : {g.L, g.Hkv, g.D, g.G, g.fmt, g.window, g.ring}) w.put<int32_t>(v);
  w.put<int64_t>(g.block_bytes);
  w.put<uint64_t>(e->key);
  w.put<int64_t>(e->n_tokens);
  w.put<int32_t>(large != 0);
  w.put<int32_t>((int32_t)e->blocks.size());
  for (int32_t b : e->blocks) w.put<int32_t>(b);
  for (int L = 0; L < g.L; ++L) w.put<int64_t>(e->len[L]);
  for (int L = 0; L < g.L; ++L) w.put<int64_t>(e->ret[L]);
  w.put<int32_t>((int32_t)e->model.size());
  w.bytes(e->model.data(), e->model.size());
  w.put<int32_t>((int32_t)e->media.size());
  w.bytes(e->media.data(), e->media.size());
  w.put<int64_t>((int64_t)e->tokens.size());
  if (!e->tokens.empty()) w.bytes(e->tokens.data(), e->tokens.size() * sizeof(int64_t));
  *size = (int64_t)w.b.size();
  if (!buf) return KRILL_OK;  // size query
  if (cap < *size) return fail(KRILL_ERR_INVALID, "descriptor needs %lld bytes", (long long)*size);
  std::memcpy(buf, w.b.data(), w.b.size());
  return KRILL_OK;
}

krill_status_t krill_prefix_import(krill_prefix_t dst, const void* pool_handle, const void* desc,
                                   int64_t desc_size, void* stream, krill_prefix_entry_t* out) {
  if (!dst || !pool_handle || !desc || !out) return fail(KRILL_ERR_INVALID, "null argument");
  krill_pool_t dp = dst->pool;
  if (dp->host_only) return fail(KRILL_ERR_NO_DEVICE, "import needs a device pool");
  const Geom& g = dp->geom;
  DescReader r{static_cast<const uint8_t*>(desc), (size_t)std::max<int64_t>(0, desc_size)};
  char magic[4];
  if (!r.bytes(magic, 4) || std::memcmp(magic, "KKV1", 4) != 0)
    return fail(KRILL_ERR_INVALID, "not an entry descriptor");
  int32_t geo[7];
  for (auto& v : geo) v = r.get<int32_t>();
  const int64_t block_bytes = r.get<int64_t>();
  if (!r.ok || geo[0] != g.L || geo[1] != g.Hkv || geo[2] != g.D || geo[3] != g.G || geo[4] != g.fmt ||
      geo[5] != g.window || geo[6] != g.ring || block_bytes != g.block_bytes)
    return fail(KRILL_ERR_INVALID, "import between pools of different geometry");
  auto* e = new krill_prefix_entry_s();
  e->key = r.get<uint64_t>();
  e->n_tokens = r.get<int64_t>();
  const int32_t large = r.get<int32_t>();
  const int32_t nb = r.get<int32_t>();
  std::vector<int32_t> src_blocks(nb > 0 && nb < (1 << 24) ? nb : 0);
  for (auto& b : src_blocks) b = r.get<int32_t>();
  e->len.resize(g.L);
  e->ret.resize(g.L);
  for (auto& v : e->len) v = r.get<int64_t>();
  for (auto& v : e->ret) v = r.get<int64_t>();
  int32_t ml = r.get<int32_t>();
  if (ml >= 0 && ml < (1 << 20)) {
    e->model.resize(ml);
    r.bytes(&e->model[0], ml);
  } else {
    r.ok = false;
  }
  int32_t dl = r.get<int32_t>();
  if (dl >= 0 && dl < (1 << 20)) {
    e->media.resize(dl);
    r.bytes(&e->media[0], dl);
  } else {
    r.ok = false;
  }
  const int64_t nt = r.get<int64_t>();
  if (nt >= 0 && nt < ((int64_t)1 << 30)) {
    e->tokens.resize((size_t)nt);
    if (nt) r.bytes(e->tokens.data(), (size_t)nt * sizeof(int64_t));
  } else {
    r.ok = false;
  }
  if (!r.ok || (int32_t)src_blocks.size() != nb) {
    delete e;
    return fail(KRILL_ERR_INVALID, "truncated entry descriptor");
  }
  {
    std::lock_guard<std::recursive_mutex> lk(dp->mu);
    DeviceGuard dg(dp->device);
    // map the owner's pool once per (handle) in this process
    const std::string hk(static_cast<const char*>(pool_handle), sizeof(cudaIpcMemHandle_t));
    uint8_t* src = nullptr;
    auto it = dp->ipc_maps.find(hk);
    if (it != dp->ipc_maps.end()) {
      src = it->second;
    } else {
      cudaIpcMemHandle_t h;
      std::memcpy(&h, pool_handle, sizeof(h));
      void* ptr = nullptr;
      const cudaError_t ce = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
      if (ce != cudaSuccess) {
        delete e;
        return fail(KRILL_ERR_PEER, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(ce));
      }
      src = static_cast<uint8_t*>(ptr);
      dp->ipc_maps[hk] = src;
    }
    e->blocks.assign(src_blocks.size(), -1);
    for (size_t i = 0; i < src_blocks.size(); ++i) {
      if (src_blocks[i] < 0) continue;
      krill_status_t st = block_alloc(dp, &e->blocks[i]);
      cudaError_t ce = cudaSuccess;
      if (st == KRILL_OK)
        ce = cudaMemcpyAsync(dp->block_ptr(e->blocks[i]), src + (int64_t)src_blocks[i] * g.block_bytes,
                             (size_t)g.block_bytes, cudaMemcpyDeviceToDevice, (cudaStream_t)stream);
      if (st != KRILL_OK || ce != cudaSuccess) {
        for (int32_t bb : e->blocks) block_unref(dp, bb);
        delete e;
        return st != KRILL_OK ? st : fail(KRILL_ERR_PEER, "peer copy: %s", cudaGetErrorString(ce));
      }
    }
    if (large) CUDA_TRY(cudaMemsetAsync(dp->d_err + 1, 1, 1, (cudaStream_t)stream));
  }
  std::lock_guard<std::mutex> lk(dst->mu);
  insert_locked(dst, e);
  e->refs.fetch_add(1);
  *out = e;
  return KRILL_OK;
}

}  // extern "C"

// =====================================================================
// Metadata for the allocation-free decode attention (kv_noalloc.cu)
// =====================================================================
namespace krill {

krill_status_t set_error(krill_status_t code, const char* msg) { return fail(code, "%s", msg); }

// Plans a decode-attention launch for krill_decode_attention_noalloc without
// touching the pool's staging buffers or scratch, and without any heap
// allocation on the success path: the metadata packet is written straight
// into `buf` (host memory owned by the caller) using only fixed-size stack
// state. Decomposition: every item covers all kv heads of a (layer,
// sequence) and at most 64 sub-blocks (4096 tokens); items are dealt to CTAs
// in serpentine order of decreasing size. On return `np->ap` holds every
// launch parameter except the device pointers into the scratch, whose byte
// offsets are in `np`.
krill_status_t noalloc_plan(krill_pool_t p, int32_t n_seqs, const krill_seq_t* seqs, int32_t lb,
                            int32_t lc, const void* q, int32_t q_dtype, void* out, int32_t out_dtype,
                            float scale, uint8_t* buf, size_t buf_cap, NoAllocPlan* np) {
  constexpr int C = 64;
  constexpr int kMaxCtas = 1024;
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  if (p->host_only) return fail(KRILL_ERR_NO_DEVICE, "compute call on a host-only pool");
  TRY(check_layers(p, lb, lc));
  TRY(check_dtype16(q_dtype, "q"));
  if (p->geom.fmt == kFmtBf16 && q_dtype != KRILL_DTYPE_BF16)
    return fail(KRILL_ERR_INVALID, "attention over a bf16 pool takes a BF16 q");
  if (out_dtype != KRILL_DTYPE_F16 && out_dtype != KRILL_DTYPE_BF16 && out_dtype != KRILL_DTYPE_F32)
    return fail(KRILL_ERR_INVALID, "out dtype must be F16, BF16 or F32");
  if (n_seqs <= 0 || lc <= 0) return fail(KRILL_ERR_INVALID, "nothing to attend");
  if (!seqs || !q || !out) return fail(KRILL_ERR_INVALID, "null q/out/seqs");
  TRY(check_aligned(q, "q"));
  TRY(check_aligned(out, "out"));
  const Geom& g = p->geom;
  // pass 1: sizes
  int64_t bt_stride = 1, n_items = 0, splits = 0, n_split_units = 0;
  for (int i = 0; i < n_seqs; ++i) {
    Seq* s = nullptr;
    TRY(seq_get(p, seqs[i], &s));
    bt_stride = std::max<int64_t>(bt_stride, (int64_t)s->blocks.size());
  }
  auto span = [&](const Seq& s, int L, int64_t* t_lo, int64_t* sb0, int64_t* n_sb) {
    const int64_t len = s.len[L];
    *t_lo = p->windowed() ? len - std::min<int64_t>(s.ret[L], p->cfg.window) : 0;
    *sb0 = *t_lo / g.subt;
    *n_sb = (len + g.subt - 1) / g.subt - *sb0;
  };
  for (int li = 0; li < lc; ++li)
    for (int si = 0; si < n_seqs; ++si) {
      Seq* s = nullptr;
      TRY(seq_get(p, seqs[si], &s));
      if (s->len[lb + li] <= 0)
        return fail(KRILL_ERR_INVALID, "attention over an empty cache (layer %d)", lb + li);
      int64_t t_lo, sb0, n_sb;
      span(*s, lb + li, &t_lo, &sb0, &n_sb);
      const int64_t n_it = (n_sb + C - 1) / C;
      n_items += n_it;
      if (n_it > 1) {
        splits += n_it;
        n_split_units += 1;
      }
    }
  const int64_t n_units = (int64_t)lc * n_seqs;
  const int grid = (int)std::min<int64_t>(std::min(p->num_sms, kMaxCtas), n_items);
  NoAllocPlan& o = *np;
  o.units_off = 0;
  o.items_off = align16((size_t)n_units * sizeof(AttnUnit));
  o.cta_off_off = o.items_off + align16((size_t)n_items * sizeof(AttnItem));
  o.bt_off = o.cta_off_off + align16((size_t)(grid + 1) * sizeof(int32_t));
  o.su_off = o.bt_off + align16((size_t)n_seqs * bt_stride * sizeof(int32_t));
  o.packet_bytes = o.su_off + align16((size_t)(n_split_units + 1) * sizeof(int32_t));
  o.partials_off = (o.packet_bytes + 255) & ~(size_t)255;
  o.records = (int64_t)splits * g.Hkv;
  o.total_bytes = o.partials_off + (size_t)splits * g.Hkv * partial_floats(g.D) * sizeof(float);
  if (o.total_bytes > buf_cap)
    return fail(KRILL_ERR_INVALID,
                "decode attention needs %zu bytes of scratch, above the %zu-byte limit of the "
                "allocation-free entry point (use krill_decode_attention, or fewer/shorter "
                "sequences per call)",
                o.total_bytes, buf_cap);
  // pass 2: units, split list, block tables
  AttnUnit* units = reinterpret_cast<AttnUnit*>(buf + o.units_off);
  int32_t* su = reinterpret_cast<int32_t*>(buf + o.su_off);
  int64_t split_base = 0, n_su = 0;
  for (int li = 0; li < lc; ++li)
    for (int si = 0; si < n_seqs; ++si) {
      Seq* s = nullptr;
      TRY(seq_get(p, seqs[si], &s));
      int64_t t_lo, sb0, n_sb;
      span(*s, lb + li, &t_lo, &sb0, &n_sb);
      const int64_t n_it = (n_sb + C - 1) / C;
      const int64_t ui = (int64_t)li * n_seqs + si;
      units[ui] = AttnUnit{(int32_t)ui, si, lb + li, (int32_t)t_lo, (int32_t)s->len[lb + li],
                           (int32_t)split_base, (int32_t)n_it, 0};
      if (n_it > 1) {
        split_base += n_it;
        su[n_su++] = (int32_t)ui;
      }
    }
  int32_t* bt = reinterpret_cast<int32_t*>(buf + o.bt_off);
  for (int si = 0; si < n_seqs; ++si) {
    Seq* s = nullptr;
    TRY(seq_get(p, seqs[si], &s));
    for (int64_t j = 0; j < bt_stride; ++j)
      bt[si * bt_stride + j] = j < (int64_t)s->blocks.size() ? s->blocks[j] : -1;
  }
  // pass 3: items in decreasing size, dealt serpentine to CTAs. CTA c gets
  // items i with serp(i) = c; count them first to lay the CTA ranges out.
  int32_t* off = reinterpret_cast<int32_t*>(buf + o.cta_off_off);
  int32_t fill[kMaxCtas];
  auto serp = [&](int64_t i) {
    const int64_t round = i / grid, pos = i % grid;
    return (int)((round & 1) ? grid - 1 - pos : pos);
  };
  for (int c = 0; c < grid; ++c) fill[c] = 0;
  for (int64_t i = 0; i < n_items; ++i) fill[serp(i)] += 1;
  off[0] = 0;
  for (int c = 0; c < grid; ++c) {
    off[c + 1] = off[c] + fill[c];
    fill[c] = off[c];
  }
  AttnItem* hi = reinterpret_cast<AttnItem*>(buf + o.items_off);
  int64_t rank = 0;
  for (int sz = C; sz >= 1; --sz)
    for (int64_t ui = 0; ui < n_units; ++ui) {
      const AttnUnit& u = units[ui];
      const int64_t sb0 = u.t_lo / g.subt;
      const int64_t n_sb = (u.t_hi + g.subt - 1) / g.subt - sb0;
      const int64_t n_it = u.n_split, base = n_sb / n_it, extra = n_sb % n_it;
      int64_t b = sb0;
      for (int64_t i = 0; i < n_it; ++i) {
        const int64_t piece = base + (i < extra ? 1 : 0);
        if (piece == sz)
          hi[fill[serp(rank++)]++] = AttnItem{(int32_t)ui, (int32_t)b, (int32_t)(b + piece), (int16_t)i, 0};
        b += piece;
      }
    }
  AttnParams& ap = o.ap;
  ap = AttnParams{};
  ap.pool = p->d_pool;
  ap.page_bytes = g.page_bytes;
  ap.sb_bytes = g.sb_bytes;
  ap.L = g.L;
  ap.Hkv = g.Hkv;
  ap.Hq = g.Hq;
  ap.g = g.g;
  ap.ring = g.ring;
  ap.hg = g.Hkv;
  ap.bt_stride = (int)bt_stride;
  ap.n_split_units = (int)n_su;
  ap.q = q;
  ap.q_dtype = q_dtype;
  ap.out = out;
  ap.out_dtype = out_dtype;
  ap.scale_log2 = scale * 1.4426950408889634f;
  ap.err = p->d_err;
  ap.wait_us = p->cfg.wait_timeout_us;
  ap.large_scale = p->d_err + 1;
  o.geom = g;
  o.grid = grid;
  o.impl = p->cfg.attn_impl;
  o.device = p->device;
  return KRILL_OK;
}

void count_kernels(krill_pool_t p, int n) {
  std::lock_guard<std::recursive_mutex> lk(p->mu);
  p->kernels += n;
}

std::recursive_mutex& pool_mutex(krill_pool_t p) { return p->mu; }

}  // namespace krill
