// m5b_linear_noalloc: the online projection of m5b_linear for callers that
// cannot allocate device memory.
//
// Some hosts cannot hand this library a workspace: a serving process whose
// device memory is already committed to its own pool and budgeted to the
// byte, a plugin whose host framework forbids extension code from allocating,
// or a hot path where cudaMalloc's implicit device synchronisation is not
// acceptable.  This entry point needs nothing from them but inputs and
// outputs: the per-token codes and scales live in one file-scope device array
// of fixed size that is part of the library's device image.  Every GPU that
// loads the library reserves it (64 MiB + 64 KiB) for as long as the library
// stays loaded.
//
// Rules for callers:
//   * Limits: m * k <= 67,108,864 codes and m <= 16,384 rows; larger calls
//     are rejected with M5B_EINVAL and a message, nothing is launched.
//   * The array is shared by every call on a device and keeps the previous
//     call's contents.  Nothing in it has to start at zero: each call writes
//     every code and scale it later reads.  Two calls whose kernels overlap
//     on the GPU (different streams, no ordering between them) race on the
//     array and may corrupt each other's results; order them on one stream
//     or with events.
//   * The device address of the array is looked up once per device, with
//     that device current, on the first call made on that device (a
//     cudaGetSymbolAddress host call).  Make that first call before any
//     stream capture.  The address is cached together with the identity of
//     the device's CUDA context; a call that finds a different context
//     current (after cudaDeviceReset the library's device image is loaded
//     again and the array may sit elsewhere) looks the address up again, so
//     the first call after a reset must also come before any stream capture.
//   * It allocates nothing: no cudaMalloc, no cudaFree, no allocating
//     library routine.
#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "m5b200.h"
#include "m5b_internal.h"

namespace {

constexpr int64_t kCodeBytes = int64_t(64) << 20;   // codes: m * k bytes
constexpr int64_t kMaxRows = 16384;                   // scales: m * 4 bytes
constexpr int64_t kScratchBytes = kCodeBytes + kMaxRows * int64_t(sizeof(float));

// The scratch array.  In host code this name is only a stand-in for the
// symbol; its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_linear_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
struct ScratchSlot {
  unsigned long long ctx_id;  // identity of the context the address belongs to
  void* addr;
};
ScratchSlot g_scratch[kMaxDevices] = {};

// Driver entry points for the current context's unique id (cuCtxGetId gives
// every context a distinct id for the life of the process, unlike the
// CUcontext handle, which a new context may reuse).
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);
CtxGetCurrentFn g_ctx_current = nullptr;
CtxGetIdFn g_ctx_id = nullptr;
std::once_flag g_ctx_once;

// Id of the context current on this thread, or 0 when none is (or the
// driver lacks the query).
unsigned long long current_context_id() {
  std::call_once(g_ctx_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_current = reinterpret_cast<CtxGetCurrentFn>(fn);
    fn = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_ctx_id = reinterpret_cast<CtxGetIdFn>(fn);
  });
  if (!g_ctx_current || !g_ctx_id) return 0;
  CUcontext ctx = nullptr;
  if (g_ctx_current(&ctx) != CUDA_SUCCESS || !ctx) return 0;
  unsigned long long id = 0;
  if (g_ctx_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of g_linear_scratch on the current device: looked up with
// cudaGetSymbolAddress on the first call on the device, with that device
// current, and again whenever the current context is not the one the cached
// address was taken in.
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  ScratchSlot& slot = g_scratch[dev];
  const unsigned long long id = current_context_id();
  if (!slot.addr || id == 0 || id != slot.ctx_id) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_linear_scratch);  // also makes the context current
    if (e != cudaSuccess) return e;
    slot.addr = p;
    slot.ctx_id = current_context_id();
  }
  *out = slot.addr;
  return cudaSuccess;
}

}  // namespace

extern "C" int m5b_linear_noalloc(const void* x, int x_dtype, int64_t m, int64_t k,
                                  int block_size, const int8_t* signs, const void* wq,
                                  const float* w_scales, int64_t n, int mode, void* out,
                                  int out_dtype, void* stream) {
  if (m <= 0 || k <= 0) return m5b::set_last_error(M5B_EINVAL, "A and B must be nonempty matrices");
  // Rows first, then k against the code bytes left per row: m * k itself
  // could overflow int64 for absurd k.
  if (m > kMaxRows || k > kCodeBytes / m)
    return m5b::set_last_error(
        M5B_EINVAL,
        "m5b_linear_noalloc holds at most 67108864 codes (m*k) and 16384 rows in its fixed "
        "device scratch; use m5b_linear with a workspace for larger inputs");
  void* scratch = nullptr;
  const cudaError_t e = scratch_address(&scratch);
  if (e != cudaSuccess)
    return m5b::set_last_error(M5B_ECUDA, "cudaGetSymbolAddress of the scratch array failed");
  return m5b_linear(x, x_dtype, m, k, block_size, signs, wq, w_scales, n, mode, out, out_dtype,
                    scratch, kScratchBytes, stream);
}
