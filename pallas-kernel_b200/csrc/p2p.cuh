// Peer-memory regions of the sequence-parallel state exchange (one process per GPU, every
// rank's region mapped into every process).  A region: a 4 KB control block -- flags[2][64]
// (the epoch whose slot rank j has written, per slot parity), the epoch of this rank's last
// exchange, a block counter -- then slots[2][world][per] of fp32 packed (state | decay),
// per = ns + nd.  Exchange e uses slot parity e & 1.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace tops {
namespace p2p {

constexpr size_t CTRL = 4096;
constexpr int MAX_WORLD = 64;

// A kernel that produces a rank's packed (state | decay) and stores it straight into every
// rank's region: the device table of regions, this rank's own, and, when the decay is not
// the kernel's own result, the decay to pack beside the state.
struct PeerPush {
  void* const* regions;
  void* own;
  int rank, world;
  const float* decay_in;
};

__device__ __forceinline__ uint32_t* flags(void* region) { return reinterpret_cast<uint32_t*>(region); }
__device__ __forceinline__ uint32_t* epoch_word(void* region) {
  return reinterpret_cast<uint32_t*>(static_cast<char*>(region) + 1024);
}
__device__ __forceinline__ uint32_t* done_word(void* region) {
  return reinterpret_cast<uint32_t*>(static_cast<char*>(region) + 1028);
}
__device__ __forceinline__ float* slots(void* region) { return reinterpret_cast<float*>(static_cast<char*>(region) + CTRL); }
__device__ __forceinline__ uint32_t ld_volatile(const uint32_t* p) { return *reinterpret_cast<const volatile uint32_t*>(p); }
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// The epoch of the exchange a push kernel is making (read by every block at its start; the
// previous push on this stream advanced it).
__device__ __forceinline__ uint32_t next_epoch(void* own) { return ld_volatile(epoch_word(own)) + 1u; }

// Float offset of rank `rank`'s slot of parity `epoch & 1` inside a region's slots.
__device__ __forceinline__ size_t slot_offset(uint32_t epoch, int world, int rank, size_t per) {
  return ((size_t)(epoch & 1u) * world + rank) * per;
}

// End of a push kernel, called by every thread of every block after its stores: each block
// fences its stores system-wide and counts itself; the last block then writes the epoch into
// every region's flag for `rank` (release stores) and advances this rank's epoch.
__device__ __forceinline__ void signal(void* const* regions, void* own, int world, int rank, uint32_t epoch) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned nblocks = gridDim.x * gridDim.y * gridDim.z;
    if (atomicAdd(done_word(own), 1u) == nblocks - 1) {
      __threadfence_system();
      for (int p = 0; p < world; ++p) st_release_sys(flags(regions[p]) + (epoch & 1u) * MAX_WORLD + rank, epoch);
      *done_word(own) = 0u;
      *epoch_word(own) = epoch;
    }
  }
}

}  // namespace p2p
}  // namespace tops
