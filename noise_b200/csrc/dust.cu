// Dust's LM-head slab jitter (reference train/val/dust.py:265-303, DUST.head_error) on sm_100a.
//
// The clean softcapped logits' exponentials are summed once per row in 16 slabs of 256 columns (head_prep_kernel).
// Each chunk of n draws jitters one slab of the cached raw logits (raw + sigma a, a ~ N(0, 1) bf16 from the caller's
// generator) and recomputes each draw's cross-entropy from the other slabs' cached sums (head_error_chunk_kernel):
//   loss = log(total - slab_sum + sum_j e^(softcap(raw_j + sigma a_j))) - target logit (the jittered one if the target
//   falls in the slab), reward = clean_loss - loss (0 where the target is -1), centred across the batch rows at each
//   position, and error[b, t, slab] -= bf16(sum_n bf16(reward / sigma) a) (the reference's bf16 einsum).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "noise_b200.h"

namespace noise {
namespace dust {

constexpr int SLAB = 256;
constexpr int SLABS = NOISE_VOCAB / SLAB;  // 16
constexpr float CAP = 15.f;

__device__ __forceinline__ float softcap(float x) { return CAP * tanhf(x / CAP); }

template <typename T>
__device__ __forceinline__ float ld(const T* p, int64_t i) {
  return static_cast<float>(p[i]);
}
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  return __bfloat162float(p[i]);
}

// One block (256 threads) per row: slab_sums[row, s] = sum of e^(softcap(raw)) over slab s, total = their sum,
// clean_target = softcap(raw[target]) with target = max(y, 0).
template <typename T>
__global__ void __launch_bounds__(256) head_prep_kernel(const T* __restrict__ raw, int64_t ld_raw,
                                                        const int64_t* __restrict__ y, float* __restrict__ slab_sums,
                                                        float* __restrict__ total, float* __restrict__ clean_target) {
  __shared__ float part[SLABS][8];
  const int64_t row = blockIdx.x;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  // warp w covers slabs 2 w, 2 w + 1
  for (int k = 0; k < 2; ++k) {
    const int s = 2 * w + k;
    float acc = 0.f;
    for (int j = lane; j < SLAB; j += 32) acc += expf(softcap(ld(raw, row * ld_raw + s * SLAB + j)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) part[s][0] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int s = 0; s < SLABS; ++s) {
      slab_sums[row * SLABS + s] = part[s][0];
      tot += part[s][0];
    }
    total[row] = tot;
    const int64_t tg = y[row] < 0 ? 0 : y[row];
    clean_target[row] = softcap(ld(raw, row * ld_raw + tg));
  }
}

// One block (256 threads) per position t: all B batch rows and n draws of one slab.
template <typename T>
__global__ void __launch_bounds__(256) head_error_chunk_kernel(
    const T* __restrict__ raw, int64_t ld_raw, const __nv_bfloat16* __restrict__ a, const int64_t* __restrict__ y,
    const float* __restrict__ clean_loss, const float* __restrict__ slab_sums, const float* __restrict__ total,
    const float* __restrict__ clean_target, int B, int Tn, int n, int slab, float sigma, float* __restrict__ error) {
  extern __shared__ float rew[];  // [n][B]
  const int t = blockIdx.x;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int lo = slab * SLAB;
  // rewards: warp per (draw, batch row)
  for (int pair = w; pair < n * B; pair += 8) {
    const int d = pair / B, b = pair % B;
    const int64_t row = static_cast<int64_t>(b) * Tn + t;
    const int64_t arow = (static_cast<int64_t>(d) * B + b) * Tn + t;  // a [n * B, T, 256]
    const int64_t tg = y[row] < 0 ? 0 : y[row];
    const bool in_slab = tg >= lo && tg < lo + SLAB;
    float acc = 0.f, tl = 0.f;
    for (int j = lane; j < SLAB; j += 32) {
      const float c = softcap(ld(raw, row * ld_raw + lo + j) + sigma * __bfloat162float(a[arow * SLAB + j]));
      acc += expf(c);
      if (in_slab && lo + j == tg) tl = c;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      acc += __shfl_xor_sync(0xffffffffu, acc, o);
      tl += __shfl_xor_sync(0xffffffffu, tl, o);
    }
    if (lane == 0) {
      const float partition = total[row] - slab_sums[row * SLABS + slab] + acc;
      const float loss = logf(partition) - (in_slab ? tl : clean_target[row]);
      rew[d * B + b] = y[row] != -1 ? clean_loss[row] - loss : 0.f;
    }
  }
  __syncthreads();
  if (B > 1 && threadIdx.x < n) {  // centre across the batch rows at this position
    float m = 0.f;
    for (int b = 0; b < B; ++b) m += rew[threadIdx.x * B + b];
    m /= B;
    for (int b = 0; b < B; ++b) rew[threadIdx.x * B + b] -= m;
  }
  __syncthreads();
  // error[b, t, lo + j] -= bf16(sum_n bf16(reward / sigma) a[n, b, t, j]); thread j = column
  const int j = threadIdx.x;
  for (int b = 0; b < B; ++b) {
    float acc = 0.f;
    for (int d = 0; d < n; ++d) {
      const float r = __bfloat162float(__float2bfloat16_rn(rew[d * B + b] / sigma));
      acc = fmaf(r, __bfloat162float(a[((static_cast<int64_t>(d) * B + b) * Tn + t) * SLAB + j]), acc);
    }
    error[(static_cast<int64_t>(b) * Tn + t) * ld_raw + lo + j] -= __bfloat162float(__float2bfloat16_rn(acc));
  }
}

}  // namespace dust
}  // namespace noise

using namespace noise::dust;

extern "C" {

int noise_head_error_prep(const void* raw, int raw_dtype, int64_t raw_stride, const int64_t* targets, int rows,
                          float* slab_sums, float* total, float* clean_target, void* stream) {
  if (!raw || !targets || !slab_sums || !total || !clean_target) return NOISE_ERR_ARGUMENT;
  if (raw_dtype != NOISE_DTYPE_F32 && raw_dtype != NOISE_DTYPE_BF16) return NOISE_ERR_ARGUMENT;
  if (rows < 0 || raw_stride < NOISE_VOCAB) return NOISE_ERR_SHAPE;
  if (rows == 0) return NOISE_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (raw_dtype == NOISE_DTYPE_BF16)
    head_prep_kernel<__nv_bfloat16><<<rows, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(raw), raw_stride, targets,
                                                         slab_sums, total, clean_target);
  else
    head_prep_kernel<float><<<rows, 256, 0, s>>>(static_cast<const float*>(raw), raw_stride, targets, slab_sums,
                                                 total, clean_target);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_head_error_chunk(const void* raw, int raw_dtype, int64_t raw_stride, const void* noise,
                           const int64_t* targets, const float* clean_loss, const float* slab_sums,
                           const float* total, const float* clean_target, int batch, int tokens, int draws, int slab,
                           float sigma, float* error, void* stream) {
  if (!raw || !noise || !targets || !clean_loss || !slab_sums || !total || !clean_target || !error)
    return NOISE_ERR_ARGUMENT;
  if (raw_dtype != NOISE_DTYPE_F32 && raw_dtype != NOISE_DTYPE_BF16) return NOISE_ERR_ARGUMENT;
  if (batch < 1 || tokens < 1 || draws < 1 || slab < 0 || slab >= SLABS || raw_stride < NOISE_VOCAB ||
      draws * batch > 8192)
    return NOISE_ERR_SHAPE;
  const size_t smem = static_cast<size_t>(draws) * batch * sizeof(float);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const __nv_bfloat16* a = static_cast<const __nv_bfloat16*>(noise);
  if (raw_dtype == NOISE_DTYPE_BF16)
    head_error_chunk_kernel<__nv_bfloat16><<<tokens, 256, smem, s>>>(
        static_cast<const __nv_bfloat16*>(raw), raw_stride, a, targets, clean_loss, slab_sums, total, clean_target,
        batch, tokens, draws, slab, sigma, error);
  else
    head_error_chunk_kernel<float><<<tokens, 256, smem, s>>>(static_cast<const float*>(raw), raw_stride, a, targets,
                                                             clean_loss, slab_sums, total, clean_target, batch,
                                                             tokens, draws, slab, sigma, error);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

}  // extern "C"
