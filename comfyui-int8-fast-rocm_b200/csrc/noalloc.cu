// A W8A8 GEMM entry point that allocates no memory: the split-K scratch
// lives in a fixed array in this library's device image.
//
// Who needs it: callers that cannot allocate device memory at the moment
// they run the GEMM -- an engine that reserves all of its GPU memory up
// front and forbids allocations afterwards, a caller inside a
// memory-pressure callback, a plugin host that owns the allocator and hands
// out only input and output buffers, or code replayed where an allocation
// would fail.  qlin_gemm_w8a8_splitk asks the caller for scratch; this entry
// uses the array below instead, so the caller only passes inputs and
// outputs.
//
// The array costs every GPU that loads the library kNoAllocScratchBytes of
// device memory until the process exits, whether or not this entry is
// called.  Its address is looked up once per device (cudaGetSymbolAddress,
// which is not an allocation) on that device's first call.  Every call
// shares the array: calls that overlap on the GPU (different streams, or
// several host threads) race on it, and the caller must serialise them.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/qlinear_b200.h"
#include "internal.h"

namespace qlin {
namespace {

// Largest split-K scratch a plan needs on a 148-SM B200: a 64 KB header
// plus at most 48 partial slots of 256 KB (one wave of split units), 12.1
// MiB; 16 MiB leaves room.  A plan that needs more is refused.
constexpr size_t kNoAllocScratchBytes = 16u << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
void* g_scratch_ptr[kMaxDevices] = {};  // device address of the array, per device

// The array's device address on the current device (looked up on the
// device's first call).  A host-side `g_noalloc_scratch` is only a stand-in
// symbol, never a device address, so the kernel is always given this one.
int scratch_address(void** ptr) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(QLIN_ERR_UNSUPPORTED, "device index above 63");
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(split-K scratch array)");
    g_scratch_ptr[dev] = p;
  }
  *ptr = g_scratch_ptr[dev];
  return QLIN_OK;
}

}  // namespace

int launch_gemm_splitk_noalloc(int kind, const int8_t* a, const int8_t* b, const float* a_scale,
                               const float* w_scale, const void* bias, void* out, int out_dt, int64_t M, int64_t N,
                               int64_t K, cudaStream_t stream) {
  const size_t need = splitk_scratch_bytes(M, N, K);
  if (need > kNoAllocScratchBytes)
    return fail(QLIN_ERR_UNSUPPORTED, "split-K scratch of " + std::to_string(need) +
                                          " bytes exceeds the library's fixed array of " +
                                          std::to_string(kNoAllocScratchBytes) + " bytes");
  void* scratch = nullptr;
  if (need > 0) {
    int rc = scratch_address(&scratch);
    if (rc) return rc;
    // the counters and flags must start at zero; an earlier call that ended
    // early (a timed-out wait) may have left them set
    cudaError_t e = cudaMemsetAsync(scratch, 0, splitk_header_bytes(), stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(split-K scratch header)");
  }
  return launch_gemm_splitk(kind, a, b, a_scale, w_scale, bias, out, out_dt, M, N, K, scratch, need, stream);
}

}  // namespace qlin
