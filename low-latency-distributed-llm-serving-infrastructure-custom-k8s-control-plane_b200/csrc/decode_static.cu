// Allocation-free entry point for the split-K paged decode.
//
// Some callers of this library cannot allocate device memory when they decode: a serving process
// that sized its KV block pool to nearly all free HBM at start-up (a later cudaMalloc would fail
// or fragment what is left), a caller bound through a plain C foreign-function layer that has no
// device allocator of its own, or a latency-critical loop that must not pay for cudaMalloc /
// cudaFree and the device-wide synchronisation they bring.  b200_paged_decode needs a scratch
// workspace (split plan, work list, merge counters, split partials) that such callers would have
// to allocate; b200_paged_decode_static takes it from a fixed array in device memory instead.
//
// The array is a file-scope static __device__ buffer of B200_DECODE_STATIC_SCRATCH_BYTES (64 MiB):
// every GPU that loads this library holds it until the process exits.  Its device address is
// looked up with cudaGetSymbolAddress the first time the entry point runs on a device (with that
// device current); make that first call before any stream capture begins.  All calls on a device
// share the one array and it keeps whatever the previous call left in it: the split-plan kernel
// that runs first in every call resets the header and the merge counters, which are the only
// parts that must start at zero.  Calls whose work overlaps on the GPU (different streams, or
// different host threads without ordering) race on the array; serialise them.
#include <mutex>
#include <string>

#include "attention.cuh"

namespace {

constexpr size_t kStaticScratchBytes = B200_DECODE_STATIC_SCRATCH_BYTES;
constexpr int kMaxDevices = 128;

std::mutex g_setup_mutex;
void* g_scratch_address[kMaxDevices] = {};

}  // namespace

static __device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];

namespace {

// Device address of g_decode_scratch for the current device (set-up on first use per device).
int scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    b200::set_last_error((std::string("b200_paged_decode_static: cudaGetDevice: ") +
                          cudaGetErrorString(e)).c_str());
    return B200_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    b200::set_last_error("b200_paged_decode_static: device ordinal out of range");
    return B200_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_address[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || p == nullptr) {
      b200::set_last_error((std::string("b200_paged_decode_static: cudaGetSymbolAddress: ") +
                            cudaGetErrorString(e)).c_str());
      return B200_ERR_CUDA;
    }
    g_scratch_address[dev] = p;
  }
  *out = g_scratch_address[dev];
  return B200_OK;
}

}  // namespace

extern "C" int b200_paged_decode_static(const B200DecodeParams* p, void* stream) {
  if (p == nullptr) {
    b200::set_last_error("b200_paged_decode_static: null params");
    return B200_ERR_INVALID_ARGUMENT;
  }
  const size_t need = b200_paged_decode_workspace_bytes(p);
  if (need > kStaticScratchBytes) {
    b200::set_last_error(("b200_paged_decode_static: this batch needs " + std::to_string(need) +
                          " bytes of decode scratch, more than the " +
                          std::to_string(kStaticScratchBytes) +
                          " bytes the allocation-free decode holds; use b200_paged_decode with "
                          "a caller-provided workspace or a smaller batch")
                             .c_str());
    return B200_ERR_INVALID_ARGUMENT;
  }
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != B200_OK) return rc;
  return b200_paged_decode(p, scratch, kStaticScratchBytes, stream);
}
