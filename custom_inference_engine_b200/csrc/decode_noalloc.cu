// cie_decode_attention_noalloc: split-KV decode attention whose scratch lives
// in a fixed device array owned by this library, for callers that cannot hand
// the library any device memory of their own.
//
// Some callers cannot allocate: a host that only received device pointers
// through an FFI and has no device allocator of its own, or a serving
// process that reserved all of HBM up front for weights and the KV pool, where
// another cudaMalloc would fail or, since cudaMalloc / cudaFree synchronise
// the device, stall the decode loop. This entry point takes inputs and
// outputs only and calls no allocator.
//
// The scratch is the file-scope array below (CIE_DECODE_NOALLOC_SCRATCH_BYTES).
// Every GPU that loads the library holds one copy until the process exits.
// Host code cannot use the array's name as a device address, so each call made
// outside a stream capture looks the address up with cudaGetSymbolAddress
// (with the call's device current) and caches it per device; a call made while
// its stream is capturing uses that cache, so make the first call on a device
// before any stream capture. Looking the address up again on every uncaptured
// call keeps it right after a device reset, which reloads the module at a
// possibly different address. All calls on a device share the array and it
// keeps the last call's contents; nothing in it has to start at zero (every split writes its whole
// partial before the merge reads it). Two calls that overlap on the GPU (two
// streams, or two graphs replayed concurrently) race on the array.
#include <mutex>

#include "cie_common.cuh"
#include "cie_host.h"

namespace cie {
namespace noalloc {

constexpr size_t kScratchBytes = CIE_DECODE_NOALLOC_SCRATCH_BYTES;
static_assert(kScratchBytes % 256 == 0, "scratch size must keep 256-byte alignment");

static __device__ __align__(256) float g_decode_scratch[kScratchBytes / sizeof(float)];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {};
std::mutex g_mu;

// Device address of g_decode_scratch on the current device: looked up again on
// every call whose stream is not capturing, taken from the per-device cache
// while it is (no runtime lookup is recorded into a graph).
int scratch_address(cudaStream_t stream, void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(CIE_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(CIE_ERR_UNSUPPORTED, "device ordinal %d", dev);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(stream, &cap);
  if (e != cudaSuccess)
    return fail(CIE_ERR_CUDA, "cudaStreamIsCapturing: %s", cudaGetErrorString(e));
  std::lock_guard<std::mutex> lk(g_mu);
  if (cap == cudaStreamCaptureStatusNone) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(CIE_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    g_scratch_addr[dev] = p;
  } else if (g_scratch_addr[dev] == nullptr) {
    return fail(CIE_ERR_INVALID_ARGUMENT,
                "first cie_decode_attention_noalloc call on device %d is inside a stream "
                "capture; make one call on this device before capturing",
                dev);
  }
  *out = g_scratch_addr[dev];
  return CIE_OK;
}

}  // namespace noalloc
}  // namespace cie

extern "C" int cie_decode_attention_noalloc(
    const void* q, const void* k, const void* v, const int64_t* lens, const int64_t* slot_ids,
    const int64_t* block_table, void* o, int batch, int num_q_heads, int num_kv_heads,
    int head_dim, int page_size, int64_t n_pages, int64_t n_slots, int64_t bt_stride,
    int64_t kv_page_stride, int64_t kv_head_stride, int num_splits, cie_stream_t stream) {
  using namespace cie;
  // the same argument checks (and status codes) as cie_decode_attention first,
  // so that only a request that is valid but too large reports CIE_ERR_WORKSPACE
  int S = 0;
  const int st = decode::check_args(q, k, v, lens, slot_ids, block_table, o, batch, num_q_heads,
                                    num_kv_heads, head_dim, page_size, n_pages, n_slots,
                                    bt_stride, kv_page_stride, kv_head_stride, num_splits,
                                    nullptr, &S);
  if (st != CIE_OK || S == 0) return st;
  const size_t need = cie_decode_workspace_bytes(batch, num_q_heads, head_dim, S);
  if (need > noalloc::kScratchBytes)
    return fail(CIE_ERR_WORKSPACE,
                "batch %d x %d splits needs %zu scratch bytes; the built-in scratch holds %zu "
                "(use fewer splits, a smaller batch, or cie_decode_attention with a workspace)",
                batch, S, need, noalloc::kScratchBytes);
  void* scratch = nullptr;
  if (need > 0) {
    const int sa = noalloc::scratch_address(reinterpret_cast<cudaStream_t>(stream), &scratch);
    if (sa != CIE_OK) return sa;
  }
  return cie_decode_attention(q, k, v, lens, slot_ids, block_table, o, scratch,
                              need > 0 ? noalloc::kScratchBytes : 0, batch, num_q_heads,
                              num_kv_heads, head_dim, page_size, n_pages, n_slots, bt_stride,
                              kv_page_stride, kv_head_stride, S, stream);
}
