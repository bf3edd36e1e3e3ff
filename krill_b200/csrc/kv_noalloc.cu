// kv_noalloc.cu — decode attention that allocates no memory.
//
// krill_decode_attention grows two kinds of memory on demand: pinned host +
// device staging for each launch's metadata (work items, block tables) and a
// device buffer for the per-piece partial results of long sequences. Some
// callers cannot let the library allocate at decode time: an engine that
// reserves all device memory up front for its own allocator (so a cudaMalloc
// from the library would fail or fragment its arena), a serving loop that
// must not take the driver's allocation locks in the middle of a step, or a
// host that accounts for every device byte itself. This entry point serves
// them: it does the same decode attention with its scratch in a fixed array
// compiled into the library (KRILL_NOALLOC_SCRATCH_BYTES, present on every
// GPU that loads the library until the process exits) and a fixed host
// buffer for the metadata, and it calls no cudaMalloc, cudaFree,
// cudaMallocHost or other allocating routine.
//
// The array's name in host code is only a stand-in for the device symbol, not
// a device address, so the address kernels receive comes from
// cudaGetSymbolAddress, looked up once per device with that device current.
// krill_pool_create does that lookup for its device (noalloc_prepare): under
// lazy module loading (the CUDA default since 12.2) the lookup is what makes
// the driver load this module and reserve the scratch, so that reservation
// happens when a pool is created, not in the middle of decoding.
#include <mutex>

#include "internal.h"

namespace {

// The scratch every call shares: metadata packet, then partial records.
static __device__ __align__(256) uint8_t g_noalloc_scratch[KRILL_NOALLOC_SCRATCH_BYTES];
// Arrival counters of split units (one per partial record; zero at load,
// epoch-tagged after that). The scratch holds at most 16 MiB / (4 * (16 + 8 *
// 64)) = 7,943 records, so 8,192 counters cover every head_dim.
constexpr int kNoallocCounters = 8192;
static __device__ unsigned long long g_noalloc_ctr[kNoallocCounters];

constexpr int kMaxDevices = 64;
std::mutex g_mu;                        // one call at a time through the shared buffers
void* g_scratch_addr[kMaxDevices];      // device address of g_noalloc_scratch per device
void* g_ctr_addr[kMaxDevices];          // device address of g_noalloc_ctr per device
uint32_t g_epoch[kMaxDevices];          // decode launches per device
alignas(64) uint8_t g_host_packet[KRILL_NOALLOC_SCRATCH_BYTES];  // host side of the metadata

}  // namespace

// Looks up both symbols' device addresses for `device` (current), once.
// Caller holds g_mu.
static cudaError_t resolve_locked(int device) {
  if (g_scratch_addr[device] && g_ctr_addr[device]) return cudaSuccess;
  void* a = nullptr;
  void* c = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&a, g_noalloc_scratch);
  if (e == cudaSuccess) e = cudaGetSymbolAddress(&c, g_noalloc_ctr);
  if (e != cudaSuccess) return e;
  if (!a || !c) return cudaErrorInvalidSymbol;
  g_scratch_addr[device] = a;
  g_ctr_addr[device] = c;
  return cudaSuccess;
}

cudaError_t krill::noalloc_prepare(int device) {
  if (device < 0 || device >= kMaxDevices) return cudaSuccess;  // no-alloc calls reject it
  std::lock_guard<std::mutex> lk(g_mu);
  return resolve_locked(device);
}

extern "C" krill_status_t krill_decode_attention_noalloc(krill_pool_t pool, int32_t n_seqs,
                                                         const krill_seq_t* seqs,
                                                         int32_t layer_begin, int32_t layer_count,
                                                         const void* q, int32_t q_dtype, void* out,
                                                         int32_t out_dtype, float scale,
                                                         void* stream) {
  using namespace krill;
  if (!pool) return set_error(KRILL_ERR_INVALID, "null pool");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Lock order: g_mu, then the pool's mutex, held across planning and launch
  // so that no other thread changes a planned sequence before its launch.
  std::lock_guard<std::mutex> lk(g_mu);
  std::lock_guard<std::recursive_mutex> plk(pool_mutex(pool));
  NoAllocPlan np;
  krill_status_t st = noalloc_plan(pool, n_seqs, seqs, layer_begin, layer_count, q, q_dtype, out,
                                   out_dtype, scale, g_host_packet, sizeof(g_host_packet), &np);
  if (st != KRILL_OK) return st;
  if (np.device < 0 || np.device >= kMaxDevices)
    return set_error(KRILL_ERR_INVALID, "device index out of range for the no-alloc scratch");
  // The metadata is copied from g_host_packet, which the next call rewrites.
  // A copy recorded into a graph would read it at replay time, so a call on a
  // stream under capture is refused.
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cap) != cudaSuccess) {
    cudaError_t e = cudaGetLastError();
    return set_error(KRILL_ERR_CUDA, cudaGetErrorString(e));
  }
  if (cap != cudaStreamCaptureStatusNone)
    return set_error(KRILL_ERR_INVALID,
                     "krill_decode_attention_noalloc cannot be called on a stream under capture "
                     "(its metadata comes from a host buffer that later calls overwrite)");
  int prev = -1;
  cudaGetDevice(&prev);
  if (prev != np.device) cudaSetDevice(np.device);
  krill_status_t rc = KRILL_OK;
  do {
    // normally done by krill_pool_create already
    cudaError_t e = resolve_locked(np.device);
    if (e != cudaSuccess) {
      rc = set_error(KRILL_ERR_CUDA, cudaGetErrorString(e));
      break;
    }
    uint8_t* base = static_cast<uint8_t*>(g_scratch_addr[np.device]);
    // Pageable source: for a host-to-device cudaMemcpyAsync from pageable
    // memory the runtime stages the bytes before the call returns, so the
    // next call may overwrite g_host_packet.
    e = cudaMemcpyAsync(base, g_host_packet, np.packet_bytes, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) {
      rc = set_error(KRILL_ERR_CUDA, cudaGetErrorString(e));
      break;
    }
    AttnParams ap = np.ap;
    ap.units = reinterpret_cast<const AttnUnit*>(base + np.units_off);
    ap.items = reinterpret_cast<const AttnItem*>(base + np.items_off);
    ap.cta_off = reinterpret_cast<const int32_t*>(base + np.cta_off_off);
    ap.bt = reinterpret_cast<const int32_t*>(base + np.bt_off);
    ap.split_units = reinterpret_cast<const int32_t*>(base + np.su_off);
    ap.partials = reinterpret_cast<float*>(base + np.partials_off);
    if (np.records <= kNoallocCounters) {
      ap.split_ctr = static_cast<unsigned long long*>(g_ctr_addr[np.device]);
      if (++g_epoch[np.device] == 0) g_epoch[np.device] = 1;
      ap.epoch = g_epoch[np.device];
    }
    e = launch_attention(np.geom, ap, np.grid, np.impl, s);
    if (e == cudaSuccess) count_kernels(pool, 1 + (attn_needs_combine(ap, np.grid, np.impl) ? 1 : 0));
    if (e != cudaSuccess) rc = set_error(KRILL_ERR_CUDA, cudaGetErrorString(e));
  } while (false);
  if (prev >= 0 && prev != np.device) cudaSetDevice(prev);
  return rc;
}
