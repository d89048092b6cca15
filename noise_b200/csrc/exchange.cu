// The identity phase's exchanges over peer memory (reference train/speedrun/run.py:3887-3912: the heads-in and
// heads-out all_to_all_single and their waits): buffer allocation and IPC mapping, the generic all-to-all send and the
// receiver's bounded wait. The protocol (epoch flags, block counter) is described in exchange.cuh; the fused pack +
// send of the heads-in exchange is in heads.cu.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>

#include "exchange.cuh"
#include "noise_b200.h"
#include "ptx.cuh"

namespace noise {
namespace xch {

// Chunk p (n16 16-byte words) of send into rank p's buffer at dst_offset + rank * chunk, then the flag. The grid walks
// 4 KB tiles (one block's stores) with the destination varying fastest and staggered by this rank, so the blocks,
// and the ranks at any moment, write to different destinations instead of every sender to one at a time.
__global__ void __launch_bounds__(256) alltoall_peer_kernel(const uint4* __restrict__ send, int64_t n16,
                                                            const __grid_constant__ Peers peers, int64_t dst_offset,
                                                            int slot, uint32_t epoch) {
  const int W = peers.world;
  const int64_t tiles = (n16 + blockDim.x - 1) / blockDim.x * W;
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int p = static_cast<int>((t % W + peers.rank) % W);
    const int64_t j = (t / W) * blockDim.x + threadIdx.x;
    if (j < n16) {
      uint4* dst = reinterpret_cast<uint4*>(peers.base[p] + dst_offset) + peers.rank * n16 + j;
      *dst = send[p * n16 + j];
    }
  }
  send_done(peers, slot, epoch);
}

// One thread per source rank: spin on this rank's flag (slot, w) until it reaches epoch (wrap-safe compare), at most
// limit_ns of global time; on a timeout the status word records NOISE_DEVICE_TIMEOUT.
__global__ void exchange_wait_kernel(const uint32_t* __restrict__ flags, int world, uint32_t epoch, int64_t limit_ns,
                                     int* status) {
  const int w = threadIdx.x;
  if (w < world) {
    const uint32_t* f = flags + w;
    if (static_cast<int32_t>(ld_acquire_sys(f) - epoch) < 0) {
      const uint64_t start = global_ns();
      for (uint32_t spin = 1;; ++spin) {
        if (static_cast<int32_t>(ld_acquire_sys(f) - epoch) >= 0) break;
        if ((spin & 63u) == 0) {
          if (*(volatile int*)status != 0) break;
          if (global_ns() - start > static_cast<uint64_t>(limit_ns)) {
            record_error(status, NOISE_DEV_TIMEOUT);
            break;
          }
          __nanosleep(200);
        }
      }
    }
  }
  __syncthreads();
}

}  // namespace xch
}  // namespace noise

using namespace noise::xch;

extern "C" {

int noise_exchange_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  if (!ptr || !ipc_handle) return NOISE_ERR_ARGUMENT;
  if (bytes < NOISE_EXCHANGE_HEAD_BYTES) return NOISE_ERR_SHAPE;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return NOISE_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return NOISE_ERR_CUDA;
  }
  static_assert(sizeof(h) == NOISE_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return NOISE_OK;
}

int noise_exchange_open(const void* ipc_handle, void** ptr) {
  if (!ipc_handle || !ptr) return NOISE_ERR_ARGUMENT;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_exchange_close(void* ptr) {
  if (!ptr) return NOISE_ERR_ARGUMENT;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_exchange_free(void* ptr) {
  if (!ptr) return NOISE_ERR_ARGUMENT;
  return cudaFree(ptr) == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_exchange_wait(const noise_peers_t* peers, int slot, uint32_t epoch, int64_t limit_ns, void* workspace,
                        void* stream) {
  Peers P;
  int rc = peers_check(peers, &P);
  if (rc) return rc;
  if (!workspace) return NOISE_ERR_WORKSPACE;
  if (slot < 0 || slot > 1 || limit_ns <= 0) return NOISE_ERR_SHAPE;
  const uint32_t* flags = reinterpret_cast<const uint32_t*>(P.base[P.rank]) + slot * FLAG_WORDS;
  exchange_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flags, P.world, epoch, limit_ns,
                                                                        static_cast<int*>(workspace));
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_alltoall_peer(const void* send, size_t chunk_bytes, const noise_peers_t* peers, size_t dst_offset, int slot,
                        uint32_t epoch, void* stream) {
  if (!send) return NOISE_ERR_ARGUMENT;
  Peers P;
  int rc = peers_check(peers, &P);
  if (rc) return rc;
  if (slot < 0 || slot > 1 || chunk_bytes == 0) return NOISE_ERR_SHAPE;
  if (chunk_bytes % 16 || dst_offset % 16 || dst_offset < NOISE_EXCHANGE_HEAD_BYTES ||
      (reinterpret_cast<uintptr_t>(send) & 15))
    return NOISE_ERR_ALIGN;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev))
    return NOISE_ERR_CUDA;
  const int64_t n16 = static_cast<int64_t>(chunk_bytes / 16);
  const int blocks = static_cast<int>(std::min<int64_t>((n16 * P.world + 255) / 256, static_cast<int64_t>(sms) * 8));
  alltoall_peer_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(send), n16, P, static_cast<int64_t>(dst_offset), slot, epoch);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

}  // extern "C"
