// Symmetric heap over NVLink / NVSwitch and device-side signalling.
//
// Each rank cudaMallocs one heap of the same size; its CUDA-IPC handle is exchanged over the process group and
// every peer's heap is mapped (cudaIpcOpenMemHandle), so buffer `off` of rank r is at peer_base[r] + off on every
// GPU. This one mechanism replaces the reference's three (DeepGEMM SymBuffer, torch symmetric memory, legacy IPC
// shard maps: cuda_moe_prefill.py:4025, rehome_transport.py:60-65, cuda_peer_read.py:196-217).
//
// Signals: 32-bit epoch words. `signal_peers` writes (release, system scope) epoch e into slot [my_rank] of a flag
// array on every peer; `wait_flags` spins (acquire, system scope) until every slot of the local array reaches e,
// bounded by %globaltimer — on timeout it records an error code in a status word and returns.
#include <stdio.h>
#include "common.cuh"
#include "ptx.cuh"

namespace cb {

CB_DEVICE void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
CB_DEVICE uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
CB_DEVICE void red_release_sys_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// One thread per peer: flag[peer][slot] = epoch, after all prior writes of this stream are visible system-wide.
__global__ void signal_peers_kernel(const uint64_t* __restrict__ peer_flag_ptrs, int world, int slot, uint32_t epoch) {
  cb::pdl_entry();
  __threadfence_system();
  const int r = threadIdx.x;
  if (r < world) st_release_sys(reinterpret_cast<uint32_t*>(peer_flag_ptrs[r]) + slot, epoch);
}

// Wait until flags[0..world) >= epoch (wrap-safe comparison), bounded.
__global__ void wait_flags_kernel(const uint32_t* __restrict__ flags, int world, uint32_t epoch, int* status,
                                  unsigned long long limit_ns) {
  cb::pdl_entry();
  const int r = threadIdx.x;
  if (r >= world) return;
  const uint64_t t0 = globaltimer();
  uint32_t n = 0;
  while (int32_t(ld_acquire_sys(flags + r) - epoch) < 0) {
    if ((++n & 63u) == 0 && globaltimer() - t0 > limit_ns) {
      if (status) atomicCAS(status, 0, kErrTimeoutPeer);
      return;
    }
  }
}

// Barrier across ranks, safe to capture in a CUDA graph: the epoch is a device counter advanced by the kernel.
// All prior writes of this stream (including P2P stores into peers' heaps) are made visible system-wide, the new
// epoch is published into slot [my_rank] of every peer's flag array, then the kernel waits (bounded) until every
// rank has published an epoch >= its own.
__global__ void p2p_barrier_kernel(const uint64_t* __restrict__ peer_flag_ptrs, int world, int my_rank,
                                   uint32_t* __restrict__ epoch_ctr, const uint32_t* __restrict__ my_flags,
                                   int* __restrict__ status, unsigned long long limit_ns) {
  cb::pdl_entry();
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0) {
    s_epoch = *epoch_ctr + 1u;
    *epoch_ctr = s_epoch;
    __threadfence_system();
  }
  __syncthreads();
  const uint32_t e = s_epoch;
  const int r = threadIdx.x;
  if (r < world) st_release_sys(reinterpret_cast<uint32_t*>(peer_flag_ptrs[r]) + my_rank, e);
  // once an error is recorded the ranks are out of step: signal (so healthy peers are not held up) but do not
  // wait, so that the failure surfaces at the next host check instead of every barrier waiting its full limit
  const bool failed = status != nullptr && *reinterpret_cast<volatile int*>(status) != 0;
  if (r < world && !failed) {
    const uint64_t t0 = globaltimer();
    uint32_t n = 0;
    while (int32_t(ld_acquire_sys(my_flags + r) - e) < 0) {
      if ((++n & 63u) == 0 && globaltimer() - t0 > limit_ns) {
        if (status) atomicCAS(status, 0, kErrTimeoutPeer);
        break;
      }
    }
  }
  __syncthreads();
}

cudaError_t p2p_barrier(const uint64_t* peer_flag_ptrs, int world, int my_rank, uint32_t* epoch_ctr,
                        const uint32_t* my_flags, int* status, uint64_t limit_ns, cudaStream_t s) {
  if (world > 32) return cudaErrorInvalidValue;
  cb::launch_k(p2p_barrier_kernel, 1, 32, 0, s, peer_flag_ptrs, world, my_rank, epoch_ctr, my_flags, status, limit_ns);
  return cudaGetLastError();
}

cudaError_t signal_peers(const uint64_t* peer_flag_ptrs, int world, int slot, uint32_t epoch, cudaStream_t s) {
  cb::launch_k(signal_peers_kernel, 1, 32, 0, s, peer_flag_ptrs, world, slot, epoch);
  return cudaGetLastError();
}

cudaError_t wait_flags(const uint32_t* flags, int world, uint32_t epoch, int* status, uint64_t limit_ns,
                       cudaStream_t s) {
  cb::launch_k(wait_flags_kernel, 1, 32, 0, s, flags, world, epoch, status, limit_ns);
  return cudaGetLastError();
}

}  // namespace cb
