// Split-KV decode for callers that cannot allocate device memory.
//
// Some callers cannot call cudaMalloc or any allocating library routine around the
// attention call: code running where allocation is forbidden or would break determinism
// of the memory footprint (a serving loop with a fixed, pre-planned memory budget, a
// host runtime without a CUDA allocator of its own, a foreign-language binding that only
// passes plain pointers).  am_q4_decode needs a caller-provided workspace for its per-split
// partial results; this entry point instead takes that scratch from one fixed array
// compiled into the library, so the caller passes only the cache, the queries and the
// output.
//
// The scratch is a file-scope device array of AM_STATIC_DECODE_SCRATCH_BYTES (16 MiB).
// Every GPU that loads this library holds it until the process exits.  Requests needing
// more scratch are rejected with AM_ERR_WORKSPACE.  All calls share the one array and it
// keeps the previous call's contents; the decode kernels write every partial they later
// read within the same call, so nothing in it has to start at zero.  Calls that overlap on
// the GPU (different streams, or different host threads, on the same device) race on the
// array and must be serialized by the caller.
//
// The device address of the array is looked up once per device with cudaGetSymbolAddress
// (the array's host-side name is only a stand-in, not a device address) on the first call
// made with that device current; make that first call before any stream capture begins.
// The cached address belongs to the device's current context: after cudaDeviceReset (or
// any teardown of the primary context) it is stale.  A call that ends in a CUDA error
// drops the cached address so the next call looks it up again; callers that reset a
// device should expect the first call afterwards to repeat the lookup.
#include <mutex>

#include "am_common.cuh"
#include "am_internal.h"

namespace am {

constexpr size_t kStaticDecodeScratchBytes = size_t(16) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_decode_scratch[kStaticDecodeScratchBytes];

static std::mutex g_scratch_mu;
static void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_decode_scratch on the current device (looked up once per device).
static int static_scratch(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_error("am_q4_decode_noalloc: no usable current CUDA device (%s)", cudaGetErrorString(e));
    (void)cudaGetLastError();
    return AM_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("am_q4_decode_noalloc: cudaGetSymbolAddress failed on device %d (%s)", dev,
                cudaGetErrorString(e));
      (void)cudaGetLastError();
      return AM_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return AM_OK;
}

// Drop the current device's cached address (after a CUDA error it may belong to a context
// that no longer exists); the next call repeats the lookup.
static void forget_static_scratch() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    (void)cudaGetLastError();
    return;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  g_scratch_ptr[dev] = nullptr;
}

}  // namespace am

extern "C" int am_q4_decode_noalloc(const am_q4_cache* cache, const am_attn_args* args,
                                    void* stream) {
  using namespace am;
  clear_error();
  if (cache == nullptr || args == nullptr) {
    set_error("am_q4_decode_noalloc: cache and args are required");
    return AM_ERR_INVALID;
  }
  // Sizes that cannot describe a call are reported by am_q4_decode's own argument checks
  // (AM_ERR_INVALID) before the scratch size is computed from them; nothing is launched.
  if (args->batch < 0 || args->q_len < 0 || args->max_kv_len < 0 || args->n_q_heads <= 0 ||
      cache->n_kv_heads <= 0 || args->n_q_heads % cache->n_kv_heads != 0) {
    return am_q4_decode(cache, args, nullptr, 0, stream);
  }
  const size_t need = am_q4_decode_workspace_bytes(cache, args);
  if (need > kStaticDecodeScratchBytes) {
    set_error("am_q4_decode_noalloc: this call needs %zu bytes of scratch but the static scratch "
              "holds %zu bytes; use am_q4_decode with a caller-provided workspace",
              need, kStaticDecodeScratchBytes);
    return AM_ERR_WORKSPACE;
  }
  void* scratch = nullptr;
  int rc = static_scratch(&scratch);
  if (rc != AM_OK) return rc;
  rc = am_q4_decode(cache, args, scratch, kStaticDecodeScratchBytes, stream);
  if (rc == AM_ERR_CUDA) forget_static_scratch();
  return rc;
}
