// internal.h — declarations shared between the host library (host.cpp) and
// the CUDA kernels. Not part of the public ABI (that is include/krill_kv.h).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "../../include/krill_kv.h"
#include "kv_common.cuh"

namespace krill {

// Destination of one appended token for one (layer, seq): the physical block
// and the absolute position (slot = pos % 256).
struct AppendDst {
  int32_t block;
  int32_t pos;
};

struct GatherOut {
  uint8_t* keys;          // mode 0: u8 codes; mode 1: f16
  uint8_t* values;
  uint16_t* key_scales;   // f16 bits (mode 0 only)
  uint16_t* key_zeros;
  uint16_t* value_scales;
  uint16_t* value_zeros;
  int64_t row_off;        // first output row (stacking)
  int64_t rows_total;     // output rows per head
  int mode;               // 0 = raw codes + meta, 1 = dequantized f16
};

struct ScatterIn {
  const uint8_t* keys;
  const uint8_t* values;
  const uint16_t* key_scales;
  const uint16_t* key_zeros;
  const uint16_t* value_scales;
  const uint16_t* value_zeros;
  int64_t row_off;
  int64_t rows_total;
};

// One decode-attention unit: (layer, sequence) over all of its kv heads, with
// the attended positions [t_lo, t_hi). Its sub-block range is split into
// n_split sequence pieces; an item is one piece for one group of kv heads.
struct AttnUnit {
  int32_t qo_row;       // li * n_seqs + si : row of q/out
  int32_t si;           // sequence index in the call (block-table row)
  int32_t layer;        // absolute layer in the pool
  int32_t t_lo, t_hi;   // attended positions
  int32_t first_split;  // partial record of (piece i, head h): (first_split + i) * Hkv + h
  int32_t n_split;
  int32_t n_pre;        // prefix records [first_split, + n_pre) written by the cascade
                        // kernel: with n_split == 1 merged by the decode item that
                        // finishes; with n_split > 1 the first n_pre of the n_split
                        // records (the decode pieces arrive as the other n_split - n_pre)
  int32_t nq;           // consecutive queries of one sequence held as columns of the
                        // query tile (multi-query verify; 0 or 1: one query). Column
                        // c is query c / g (row qo_row + c / g), kv-group head c % g,
                        // and sees positions below t_hi - (nq - 1 - c / g)
};

// Columns of a unit's query tile (at most 8) and the element offset of column
// c in q / out relative to the unit's first row and head group.
__host__ __device__ inline int unit_cols(const AttnUnit& u, int g) { return g * (u.nq > 1 ? u.nq : 1); }
__host__ __device__ inline int64_t col_off(int c, int g, int64_t row_elems, int D) {
  return (int64_t)(c / g) * row_elems + (int64_t)(c % g) * D;
}

struct AttnItem {
  int32_t unit;
  int32_t sb_begin;  // logical sub-block range (positions 64*sb ...)
  int32_t sb_end;
  int16_t idx;       // sequence piece within its unit
  int16_t h0;        // first kv head of the item's head group
};

// Cascade (shared-prefix) attention. Sequences of one call whose block tables
// begin with the same physical blocks attend that common prefix together: a
// work item is a fragment [sb_begin, sb_end) of the prefix's sub-blocks for
// one (layer, kv head) and up to sh_rows(D) query rows (member sequences x
// GQA group), read and dequantized once for all of them. Its result is the
// partial record `slot` of every member unit; the members' own suffixes go
// through the decode kernel as later pieces and the combine kernel merges.
struct ShItem {
  int32_t layer;     // absolute layer in the pool
  int32_t leader;    // block-table row holding the shared blocks
  int32_t sb_begin;  // sub-block range of the shared prefix
  int32_t sb_end;
  int32_t mem_off;   // first member unit id in the members array
  int16_t n_rows;    // members * g, at most sh_rows(D)
  int16_t h;         // kv head
  int16_t slot;      // partial-record slot of this fragment
  int16_t n_frag;    // fragments of this (members, layer, head)
  int32_t causal;    // -1: every row sees every token. Else the rows are the
                     // queries (row / g) of one sequence at positions causal +
                     // row / g, each seeing tokens up to its own (multi-query
                     // verify / chunked prefill)
};

// Query rows of one cascade item: 8 consumer warps x 32 rows (16 at D = 256,
// whose fp32 output rows need twice the registers).
__host__ __device__ constexpr int sh_rows(int D) { return D >= 256 ? 128 : 256; }

struct AttnParams {
  const uint8_t* pool;
  int64_t page_bytes, sb_bytes;
  int L, Hkv, Hq, g, ring;
  int hg;                  // kv heads per item (divides Hkv)
  int qt;                  // query tiles per unit: 1, or 2 (each unit followed by its
                           // shadow unit, AttnUnit::nq; int8, head_dim <= 128, hg = 8)
  const AttnUnit* units;
  const AttnItem* items;
  const int32_t* cta_off;  // [grid + 1] item ranges per CTA
  const int32_t* bt;       // [n_seqs][bt_stride]
  int bt_stride;
  const int32_t* split_units;  // units with n_split > 1
  int n_split_units;
  // Arrival counters of split units, one per partial record ((first_split +
  // i) * Hkv + h, only i = 0 used): the decode piece that arrives last merges
  // the unit's records. Each word is (epoch << 32 | arrivals); a word from
  // another epoch counts as zero, so the counters never need clearing.
  // nullptr: the combine kernel merges instead.
  unsigned long long* split_ctr;
  uint32_t epoch;
  const void* q;
  int q_dtype;
  void* out;
  int out_dtype;
  float scale_log2;  // softmax scale * log2(e)
  float* partials;   // [splits * Hkv][16 + 8*D]
  int* err;
  int wait_us;       // bound of every device-side wait, microseconds (0: default)
  const int* large_scale;  // non-zero once the pool holds a scale with |s| >= 64
  // cascade items (sh_grid = 0: none)
  const ShItem* sh_items;
  const int32_t* sh_cta_off;  // [sh_grid + 1]
  const int32_t* sh_members;  // unit ids
  int sh_grid;                // CTAs, or CTA pairs when sh_pair (sh_cta_off per pair)
  int sh_pair;                // 1: the tcgen05 cascade runs as CTA pairs (cta_group::2)
  int n_pslots;               // prefix record slots per cascaded unit
  // host side only: launch the decode kernel as the programmatic dependent of
  // the append kernel launched just before it on the stream
  int pdl;
};

// Rotary table for the fused RoPE append: cos / sin [rows][D/2] f32 (device),
// indexed by absolute position; cos == nullptr means no rotation.
struct RopeTable {
  const float* cos;
  const float* sin;
  int64_t rows;
};

// Appends of at least this many tokens per (layer, sequence) into an int8
// pool run the tiled append kernel (one CTA per destination sub-block). Their
// destination list is compact: per (layer, sequence), append_tile_chunks
// entries, entry c giving the block and position of the first new token in
// the c-th sub-block the call touches (unused entries past the last one).
inline bool append_uses_tiles(int n_new) { return n_new >= 16; }
inline int append_tile_chunks(int n_new, int subt) { return (n_new + subt - 1) / subt + 1; }

// Kernels that store scales raise *large_scale when one has |s| >= 64 (the
// one-fma dequantization is exact only below that).
cudaError_t launch_append(const Geom& g, uint8_t* pool, const AppendDst* d_dst, int layer_begin,
                          int layer_count, int n_seqs, int n_new, const void* k, const void* v,
                          int dtype, int* large_scale, RopeTable rope, cudaStream_t stream);
cudaError_t launch_gather(const Geom& g, const uint8_t* pool, int layer, const int32_t* d_bt,
                          int64_t p0, int64_t S, const GatherOut& out, cudaStream_t stream);
cudaError_t launch_scatter(const Geom& g, uint8_t* pool, int layer, const int32_t* d_bt, int64_t p0,
                           int64_t S, const ScatterIn& in, int* large_scale, cudaStream_t stream);
// grid = number of persistent CTAs (cta_off has grid + 1 entries). Launches
// the cascade kernel when p.sh_grid > 0, then the decode kernel and, when
// some unit is split, the combine kernel.
cudaError_t launch_attention(const Geom& g, const AttnParams& p, int grid, int impl,
                             cudaStream_t stream);
// Names the kernel instances launch_attention would run for these arguments.
void describe_attention(const Geom& g, const AttnParams& p, int grid, int impl, char* buf,
                        size_t cap);
cudaError_t launch_shared(const Geom& g, const AttnParams& p, cudaStream_t stream);
// Merge the partial records of p.split_units (attn_combine_kernel) on its own.
cudaError_t launch_combine(const Geom& g, const AttnParams& p, cudaStream_t stream);
// True when launch_attention runs the combine kernel: split units whose records
// are not merged by the last-arriving decode piece (no counters, no decode
// kernel, or the CUDA-core variant).
inline bool attn_needs_combine(const AttnParams& p, int grid, int impl) {
  return p.n_split_units > 0 && (grid <= 0 || impl == 1 || p.split_ctr == nullptr);
}
// The cascade runs on tcgen05 (accumulators in tensor memory, 256 query rows
// per item as two 128-row halves) for head_dim <= 128 under
// KRILL_ATTN_TENSOR_CORE; otherwise on mma.sync (sh_rows(D) rows per item).
bool shared_uses_umma(const Geom& g, int impl);
// Clusters of two CTAs of the pair cascade kernel that fit on the current
// device at once (0: no pair kernel for this geometry, or no device).
int shared_pair_capacity(const Geom& g);
cudaError_t launch_shared_umma(const Geom& g, const AttnParams& p, cudaStream_t stream);
inline int shared_rows(const Geom& g, int impl) { return shared_uses_umma(g, impl) ? 256 : sh_rows(g.D); }
// Launch description produced for the allocation-free decode attention:
// byte offsets of the metadata and partial records inside the caller's
// scratch, plus the launch parameters (pointers into the scratch unset).
struct NoAllocPlan {
  size_t units_off, items_off, cta_off_off, bt_off, su_off;
  size_t packet_bytes, partials_off, total_bytes;
  int64_t records;  // partial records (split pieces x kv heads)
  AttnParams ap;
  Geom geom;
  int grid, impl, device;
};

// Plans a launch of the allocation-free decode attention into `buf` (host).
krill_status_t noalloc_plan(krill_pool_t p, int32_t n_seqs, const krill_seq_t* seqs, int32_t lb,
                            int32_t lc, const void* q, int32_t q_dtype, void* out, int32_t out_dtype,
                            float scale, uint8_t* buf, size_t buf_cap, NoAllocPlan* np);
// Adds n to the pool's launched-kernel count (krill_pool_kernel_count).
void count_kernels(krill_pool_t p, int n);
// The pool's call mutex (recursive): held across planning and launch so that
// no other thread frees or appends to a planned sequence in between.
std::recursive_mutex& pool_mutex(krill_pool_t p);
// Resolves the allocation-free entry point's device scratch on `device`
// (which must be current). Under lazy module loading this is the moment the
// driver loads the module and reserves the scratch, so pool creation calls it
// instead of the first decode call. Idempotent; thread-safe.
cudaError_t noalloc_prepare(int device);
// Sets the thread-local message returned by krill_last_error_string().
krill_status_t set_error(krill_status_t code, const char* msg);

// Consumer warps per attention CTA for head_dim D.
inline int attn_warps(int /*D*/) { return 8; }
// Resident CTAs per SM the planner targets: one persistent tensor-core CTA
// (it fills the shared memory), four of the lighter CUDA-core variant.
inline int attn_ctas_per_sm(int impl) { return impl == 1 ? 4 : 1; }
// Floats per partial record for head_dim D.
__host__ __device__ inline int64_t partial_floats(int D) { return 16 + 8 * (int64_t)D; }

}  // namespace krill
