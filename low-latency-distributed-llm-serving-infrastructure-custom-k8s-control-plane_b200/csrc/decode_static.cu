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
// looked up with cudaGetSymbolAddress the first time the entry point runs in a CUDA context of a
// device (with that device current); make that first call before any stream capture begins.  The
// address is cached together with the context it belongs to, so after a cudaDeviceReset (which
// destroys the context and reloads the module in a new one) the next call looks it up again
// instead of reusing a stale address.  All calls on a device share the one array and it keeps
// whatever the previous call left in it: the split-plan kernel that runs first in every call
// resets the header and the merge counters, which are the only parts that must start at zero.
// Calls whose work overlaps on the GPU (different streams, or different host threads without
// ordering) race on the array; serialise them.
#include <cuda.h>

#include <mutex>
#include <string>

#include "attention.cuh"

namespace {

constexpr size_t kStaticScratchBytes = B200_DECODE_STATIC_SCRATCH_BYTES;
constexpr int kMaxDevices = 128;

struct ScratchEntry {
  CUcontext ctx;  // the context the cached address belongs to
  void* address;
};

std::mutex g_setup_mutex;
ScratchEntry g_scratch[kMaxDevices] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// cuCtxGetCurrent through the runtime's driver entry point (no link-time libcuda dependency).
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

}  // namespace

static __device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];

namespace {

int setup_fail(const char* what, cudaError_t e) {
  b200::set_last_error((std::string("b200_paged_decode_static: ") + what + ": " +
                        cudaGetErrorString(e)).c_str());
  return B200_ERR_CUDA;
}

// Device address of g_decode_scratch in the current context (looked up once per context).
int scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return setup_fail("cudaGetDevice", e);
  if (dev < 0 || dev >= kMaxDevices) {
    b200::set_last_error("b200_paged_decode_static: device ordinal out of range");
    return B200_ERR_UNSUPPORTED;
  }
  CtxGetCurrentFn get_ctx = ctx_get_current();
  if (get_ctx == nullptr) {
    b200::set_last_error("b200_paged_decode_static: cuCtxGetCurrent is unavailable");
    return B200_ERR_CUDA;
  }
  CUcontext ctx = nullptr;  // null until the runtime has set up this thread's context
  if (get_ctx(&ctx) != CUDA_SUCCESS) {
    b200::set_last_error("b200_paged_decode_static: cannot read the current CUDA context");
    return B200_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  ScratchEntry& entry = g_scratch[dev];
  if (ctx == nullptr || entry.address == nullptr || entry.ctx != ctx) {
    void* p = nullptr;
    // Also makes the device's primary context current when none was.
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || p == nullptr) return setup_fail("cudaGetSymbolAddress", e);
    if (get_ctx(&ctx) != CUDA_SUCCESS || ctx == nullptr) {
      b200::set_last_error("b200_paged_decode_static: cannot read the current CUDA context");
      return B200_ERR_CUDA;
    }
    entry.ctx = ctx;
    entry.address = p;
  }
  *out = entry.address;
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
