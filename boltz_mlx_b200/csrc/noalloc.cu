// triattn_forward_noalloc: one triangle-attention layer that needs no workspace from its caller.
//
// Some callers cannot allocate device memory when they run a layer: a plugin whose host hands it
// device pointers for inputs and outputs but forbids cudaMalloc after start-up, a serving process
// whose memory is carved up once by an allocator it does not own, or code that must keep a fixed
// device footprint known at load time.  For them the layer's scratch (the tri-bias table, the
// q/k/v/g operand images, the attention output before projection and the mask bias) lives in the
// fixed array below.  A GPU holds the array from the moment this file's module is loaded on it until
// process exit: under CUDA's default lazy module loading (CUDA_MODULE_LOADING=LAZY) that is the first
// triattn_forward_noalloc call on the device, whose symbol lookup loads the module and reserves the
// 48 MiB; with CUDA_MODULE_LOADING=EAGER it is library load.  A caller that hands the rest of its
// device memory to another allocator should make one small call (e.g. N = 1) on each device first.
//
// Limits and rules:
//   * The array holds kScratchBytes = 48 MiB.  A call is accepted when its workspace,
//     triattn_workspace_bytes(B, N, N, dtype), fits: roughly N <= 128 for B = 1 in every dtype
//     (e.g. N = 128 needs 20.3 MB in fp16/bf16 and 42.3 MB in fp32).  Larger calls return
//     TRIATTN_ENOSPACE with the sizes in triattn_last_error_string() and launch nothing.
//   * Nothing here allocates or frees: no cudaMalloc, no cudaFree, no allocating library routine.
//   * The first call on a device (with that device current) looks up the array's device address
//     with cudaGetSymbolAddress and caches it; make that first call before any stream capture.
//   * All calls share the one array and it keeps the previous call's contents.  No region has to
//     start at zero: within a call every byte the kernels read is written earlier in the same call.
//     Two calls that overlap on the GPU (different streams, or different host threads on one
//     device) race on the array; serialise them.
#include <cstdio>
#include <mutex>

#include "triattn.h"
#include "triattn_internal.cuh"

namespace {

constexpr size_t kScratchBytes = 48ull << 20;

// In host code `g_noalloc_scratch` names a host-side stand-in, not device memory: only the address
// returned by cudaGetSymbolAddress may be handed to a kernel.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

// Device address of the scratch array for the current device, looked up once per device.
int scratch_for_current_device(void** out) {
  static void* cache[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return triattn::record_error(TRIATTN_ECUDA, "cudaGetDevice", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return triattn::record_error(TRIATTN_EUNSUPPORTED, "device index above 63", "");
  std::lock_guard<std::mutex> lk(mu);
  if (!cache[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e == cudaErrorMemoryAllocation)
      return triattn::record_error(TRIATTN_ECUDA, "cudaGetSymbolAddress(scratch)",
                                   "no device memory left for the 48 MiB scratch array (reserved when the "
                                   "module loads, on the first call under lazy loading)");
    if (e != cudaSuccess || p == nullptr)
      return triattn::record_error(TRIATTN_ECUDA, "cudaGetSymbolAddress(scratch)", cudaGetErrorString(e));
    cache[dev] = p;
  }
  *out = cache[dev];
  return TRIATTN_OK;
}

}  // namespace

extern "C" int triattn_forward_noalloc(const float* z, const float* mask, const void* packed, int B, int N,
                                       int starting, float inf, int dtype, int add_residual, float* out,
                                       void* stream) {
  const size_t need = triattn_workspace_bytes(B, N, N, dtype);
  if (need == 0 || (dtype != TRIATTN_F32 && dtype != TRIATTN_F16 && dtype != TRIATTN_BF16))
    // invalid sizes or dtype: let the regular entry point report them (it checks before any CUDA call)
    return triattn_forward(z, mask, packed, B, N, starting, inf, dtype, add_residual, out, nullptr, 0, stream);
  if (need > kScratchBytes) {
    char msg[160];
    snprintf(msg, sizeof(msg), "B=%d N=%d needs %zu bytes of scratch; the static array holds %zu", B, N, need,
             kScratchBytes);
    return triattn::record_error(TRIATTN_ENOSPACE, "triattn_forward_noalloc", msg);
  }
  void* ws = nullptr;
  if (int r = scratch_for_current_device(&ws)) return r;
  return triattn_forward(z, mask, packed, B, N, starting, inf, dtype, add_residual, out, ws, kScratchBytes, stream);
}
