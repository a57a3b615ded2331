// peer_barrier.cuh — stream-ordered barrier between the GPUs of a fused all-gather.
//
// After a GEMM has stored its output tiles into every rank's buffer over peer memory
// (gemm_a8w4_decode.cuh with peers > 0), each rank must know that all the others have
// finished writing into its buffer before anything reads it. Each rank owns `world`+1
// uint32 words: flags[rank][j] is the last epoch rank j announced, flags[rank][world] the
// number of barriers this rank has passed (only this rank touches it). One warp takes the
// next epoch from that counter, announces it in every rank's array (a system-scope release
// store into peer memory) and waits until its own array holds epochs >= this one from every
// rank (acquire loads). The epoch lives in device memory, not in the launch arguments, so
// a CUDA graph that captured the launch replays correctly. Epochs only grow, so the flags
// never need resetting. The wait is bounded (2 s unless the caller gives another limit):
// when it runs out the kernel sets a status bit (arc_device_status) and returns, so a
// missing peer cannot hang the GPU.
#pragma once

#include "sm100.cuh"

namespace arcb {
namespace peer {

constexpr uint32_t kMaxPeers = 8;

struct BarrierParams {
  uint32_t* flags[kMaxPeers];  // rank i's flag array (world + 1 words), mapped into this process
  uint32_t world, rank;
  uint64_t timeout_ns;         // bound of the wait for the peers' announcements
};

__global__ void __launch_bounds__(32, 1) peer_barrier_kernel(const __grid_constant__ BarrierParams b) {
  const uint32_t i = threadIdx.x;
  // Launched with programmatic dependent launch: the next kernel in the stream (the next
  // GEMM) may start its prologue and weight prefetch now; it reads and writes outputs only
  // after this kernel has completed.
  pdl_launch_dependents();
  // The GEMM before this kernel in the stream must have completed (its peer stores
  // performed) before anything is announced.
  pdl_wait();
  uint32_t* counter = b.flags[b.rank] + b.world;
  const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(counter) + 1u;
  // Make the GEMM's peer stores visible system-wide before announcing them.
  __threadfence_system();
  if (i < b.world) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(b.flags[i] + b.rank), "r"(epoch) : "memory");
    const uint32_t* f = b.flags[b.rank] + i;
    const uint64_t start = globaltimer_ns();
#pragma unroll 1
    for (uint32_t it = 0;; ++it) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
      if (static_cast<int32_t>(v - epoch) >= 0) break;
      if ((it & 63u) == 63u && globaltimer_ns() - start > b.timeout_ns) {
        atomicOr(&g_arc_status, kStatusTimeoutPeer);
        break;
      }
      __nanosleep(128);
    }
  }
  __syncwarp();  // every lane has read the counter
  if (i == 0) *counter = epoch;
}

}  // namespace peer
}  // namespace arcb
