// Cross-GPU barrier of the peer-store exchange (one process per GPU, memory shared through CUDA IPC).
//
// Each rank owns a flag block of `world` 32-bit slots in IPC-shared device memory.  A barrier with
// epoch e: lane t (< world) publishes e into slot [rank] of rank t's block (a system-scope release
// store over NVLink), then waits until slot [t] of its own block holds e or later (system-scope
// acquire loads).  Epochs only grow, so a late signal from the previous barrier cannot satisfy this
// one.  The wait is bounded: after TRIATTN_WAIT_NS (or as soon as a kernel records an error while
// this barrier waits) the lane records DEV_PEER_TIMEOUT and returns, so a rank that never arrives
// cannot hang this GPU.  An error already in the status word when the barrier starts (a stale one,
// from an earlier launch) does not end the wait: skipping a barrier would let the exchange's remote
// stores race, so every barrier waits for every peer unless a NEW error appears meanwhile.
#include <algorithm>
#include <cstdint>

#include "sm100.cuh"
#include "triattn_internal.cuh"

namespace triattn {

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(32) peer_barrier_kernel(const unsigned long long* __restrict__ flag_ptrs, int rank,
                                                          int world, unsigned epoch, int* status) {
  const int t = threadIdx.x;
  if (t >= world) return;
  const int status_at_entry = *reinterpret_cast<volatile int*>(status);
  __threadfence_system();  // this GPU's earlier writes (previous kernels included) before the signal
  st_release_sys(reinterpret_cast<unsigned*>(flag_ptrs[t]) + rank, epoch);
  const unsigned* mine = reinterpret_cast<const unsigned*>(flag_ptrs[rank]) + t;
  uint64_t t0 = 0;
  for (uint32_t spin = 0;; ++spin) {
    if (static_cast<int>(ld_acquire_sys(mine) - epoch) >= 0) break;
    if ((spin & 63u) == 0u) {
      if (*reinterpret_cast<volatile int*>(status) != status_at_entry) return;  // a new error meanwhile
      const uint64_t now = global_timer_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > TRIATTN_WAIT_NS) {
        atomicCAS(status, 0, DEV_PEER_TIMEOUT);
        return;
      }
    }
    __nanosleep(200);
  }
  __threadfence_system();
}

cudaError_t launch_peer_barrier(const unsigned long long* flag_ptrs, int rank, int world, unsigned epoch,
                                int* status, cudaStream_t st) {
  peer_barrier_kernel<<<1, 32, 0, st>>>(flag_ptrs, rank, world, epoch, status);
  return cudaGetLastError();
}

}  // namespace triattn

namespace triattn {

// Copy `bytes` (a multiple of 16) at byte `offset` of this rank's buffer to the same offset of every
// other rank's buffer (dst_ptrs[t] = rank t's buffer as mapped here): 16-byte loads from local HBM,
// stores over NVLink, all peers interleaved so every link carries traffic at once.  The stores are
// made visible system-wide before the kernel ends (a triattn_peer_barrier publishes them).
__global__ void __launch_bounds__(256) peer_broadcast_kernel(const unsigned long long* __restrict__ dst_ptrs,
                                                             int rank, int world, size_t offset, size_t n16) {
  const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(dst_ptrs[rank]) + offset);
  const int lane = threadIdx.x & 31;
  const size_t peers = (size_t)(world - 1);
  // work unit = 32 consecutive 16-byte chunks (512 B) for one peer; units cycle over the peers
  const size_t units = (n16 + 31) / 32 * peers;
  const size_t nwarps = (size_t)gridDim.x * (blockDim.x >> 5);
  for (size_t u = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; u < units; u += nwarps) {
    const size_t g = u / peers;
    int t = (int)(u - g * peers);
    t += (t >= rank);
    const size_t k = g * 32 + lane;
    if (k < n16) reinterpret_cast<uint4*>(reinterpret_cast<char*>(dst_ptrs[t]) + offset)[k] = __ldg(src + k);
  }
  __threadfence_system();
}

cudaError_t launch_peer_broadcast(const unsigned long long* dst_ptrs, int rank, int world, size_t offset, size_t bytes,
                                  int num_sms, cudaStream_t st) {
  if (world < 2 || bytes == 0) return cudaSuccess;
  const size_t n16 = bytes / 16, units = (n16 + 31) / 32 * (size_t)(world - 1);
  const int grid = (int)std::max<size_t>(1, std::min<size_t>((size_t)num_sms * 4, (units + 7) / 8));
  peer_broadcast_kernel<<<grid, 256, 0, st>>>(dst_ptrs, rank, world, offset, n16);
  return cudaGetLastError();
}

}  // namespace triattn
