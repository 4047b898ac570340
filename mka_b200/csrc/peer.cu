// Cross-GPU flag barrier for the head-sharded layer.
//
// The ranks of one sequence group (one process per GPU of a box) exchange the
// attention output and the o_proj output by storing straight into each other's
// buffers through peer mappings (CUDA IPC of plain cudaMalloc allocations; no
// NVLink multicast object is involved). This barrier orders those stores: each
// rank owns a flag array with one 32-bit slot per rank of the group, mapped
// into every other rank. Arriving at barrier number `epoch`, rank r stores
// `epoch` into slot r of every rank's array (release, system scope) and then
// waits until every slot of its own array has reached `epoch` (acquire). It
// runs in stream order, so everything the rank launched before it - including
// stores into peer memory - is visible to the others once they pass it.
//
// Epochs grow by one per barrier, so a peer that has already moved on to the
// next barrier also counts as arrived, and no reset is ever needed. Every wait
// is bounded (2 s of %globaltimer): when it runs out the kernel sets
// kStatusPeerTimeout in the device status word and returns, so a rank that
// never arrives ends the barrier with an error the host can read instead of a
// hung GPU.
//
// The reference has no distributed code in the layer (its DDP / tensor
// parallel use lives in scripts/train_hf_patch.py:97-129); this replaces the
// NCCL all-gather of the attention output in front of o_proj.
#include "fmka_internal.h"
#include "ptx.cuh"

namespace fmka {

namespace {

struct PeerFlags {
  uint32_t* f[kMaxPeers];
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ bool reached(uint32_t v, uint32_t epoch) { return (int32_t)(v - epoch) >= 0; }

// One thread per rank j of the group: announce this rank to j, then wait for
// j's announcement in this rank's own array.
__global__ void peer_barrier_kernel(PeerFlags fl, int rank, int n, uint32_t epoch, uint32_t* status) {
  const int j = threadIdx.x;
  if (j >= n) return;
  __threadfence_system();
  st_release_sys(fl.f[j] + rank, epoch);
  const uint32_t* mine = fl.f[rank] + j;
  if (reached(ld_acquire_sys(mine), epoch)) return;
  const uint64_t t0 = globaltimer_ns();
  while (!reached(ld_acquire_sys(mine), epoch)) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      if (status) atomicOr(status, kStatusPeerTimeout);
      return;
    }
    __nanosleep(128);
  }
}

}  // namespace

int launch_peer_barrier(uint32_t* const* flags, int rank, int n, uint32_t epoch, cudaStream_t stream) {
  if (n < 1 || n > kMaxPeers || rank < 0 || rank >= n)
    return set_error(kErrInvalidArgument, "peer_barrier: rank / group size out of range");
  PeerFlags fl;
  for (int j = 0; j < kMaxPeers; ++j) {
    fl.f[j] = j < n ? flags[j] : nullptr;
    if (j < n && (fl.f[j] == nullptr || (reinterpret_cast<uintptr_t>(fl.f[j]) & 3u)))
      return set_error(kErrInvalidArgument, "peer_barrier: flag arrays must be non-null and 4-byte aligned");
  }
  peer_barrier_kernel<<<1, 32, 0, stream>>>(fl, rank, n, epoch, device_status_word());
  return check_cuda(cudaGetLastError(), "peer_barrier launch");
}

}  // namespace fmka
