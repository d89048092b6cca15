// Peer-memory exchange primitives shared by the head-sharding kernels (heads.cu) and the generic exchange entry points
// (exchange.cu): the identity phase's two all_to_all_single calls (reference train/speedrun/run.py:3888, 3906) done
// as stores into the destination ranks' buffers over NVLink (CUDA IPC mappings, plain loads and stores, no
// multicast), with a per-(slot, source) epoch flag instead of a collective's completion.
//
// Every rank's exchange buffer starts with NOISE_EXCHANGE_HEAD_BYTES of control words:
//   flags[slot][src]   uint32, offset (slot * 64 + src) * 4: the last epoch rank src published into this buffer
//   counter[slot]      uint32, offset 512 + slot * 4: blocks of this rank's current send that have finished (local)
// A send kernel's blocks store their share, fence at system scope and count themselves; the last block resets the
// counter and publishes the epoch to every destination's flag with a system-scope release store. The receiver's
// wait kernel spins (bounded) on its own flags with system-scope acquire loads.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "noise_b200.h"

namespace noise {
namespace xch {

constexpr int FLAG_WORDS = 64;
constexpr int COUNTER_OFFSET = 512;

struct Peers {
  char* base[NOISE_MAX_PEERS];
  int rank, world;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Called once by every thread of every block after the block's last store of the send: the grid's last block
// publishes `epoch` to flags[slot][rank] of every destination.
__device__ __forceinline__ void send_done(const Peers& P, int slot, uint32_t epoch) {
  __shared__ int last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* counter = reinterpret_cast<uint32_t*>(P.base[P.rank] + COUNTER_OFFSET) + slot;
    const uint32_t blocks = gridDim.x * gridDim.y * gridDim.z;
    last = atomicAdd(counter, 1u) == blocks - 1;
    if (last) {
      atomicExch(counter, 0u);
      __threadfence_system();
      for (int p = 0; p < P.world; ++p)
        st_release_sys(reinterpret_cast<uint32_t*>(P.base[p]) + slot * FLAG_WORDS + P.rank, epoch);
    }
  }
}

// A peers description the send kernels accept: 1 <= world <= 8 ranks, rank < world, every base mapped, 16-byte
// aligned.
inline int peers_check(const noise_peers_t* peers, xch::Peers* out) {
  if (!peers) return NOISE_ERR_ARGUMENT;
  if (peers->world < 1 || peers->world > NOISE_MAX_PEERS || peers->rank < 0 || peers->rank >= peers->world)
    return NOISE_ERR_SHAPE;
  for (int p = 0; p < NOISE_MAX_PEERS; ++p) {
    out->base[p] = p < peers->world ? static_cast<char*>(peers->base[p]) : nullptr;
    if (p < peers->world && !peers->base[p]) return NOISE_ERR_ARGUMENT;
    if (p < peers->world && (reinterpret_cast<uintptr_t>(peers->base[p]) & 15)) return NOISE_ERR_ALIGN;
  }
  out->rank = peers->rank;
  out->world = peers->world;
  return NOISE_OK;
}

}  // namespace xch
}  // namespace noise
