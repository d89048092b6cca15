// The seed-rebuilt ES update of EGGROLL (reference archive/10M/train/val/eggroll.py:151-167) on sm_100a.
//
// G_P = -(1 / count) sum_j w_j a_j b_j^T for every parameter P, where (a_j, b_j) is pair j's slice of the fixed noise
// buffer at offsets[P, j] (a = first `out` values, b = next `in`), then AdamW. For matrices the sum over pairs is a GEMM
// with K = pairs: rank1_operands_kernel builds A' [out, Kp] = -w_j a_j[o] / count and B' [in, Kp] = b_j[i] in fp32
// (or bf16; transposed through shared memory; columns j >= pairs are zero so Kp may be padded), and the tcgen05 GEMM
// computes G = A' B'^T at tf32 (noise_gemm_tf32_tn: the reference's fp32 matmul at 'high' precision, eggroll.py:184)
// or bf16 (noise_gemm_bf16_tn). Parameters too small for GEMM tiles (the value-embedding gates
// [8, 32], the mixing scalars [8]) use rank1_small_kernel directly. adam_kernel is torch.optim.AdamW's update
// (weight_decay = 0) for one flat fp32 tensor.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "noise_b200.h"

namespace noise {
namespace update {

constexpr int TJ = 64;  // pairs per tile
constexpr int TE = 64;  // vector elements per tile

__device__ __forceinline__ void store_operand(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
__device__ __forceinline__ void store_operand(float* p, float v) { *p = v; }

// One block: pairs j0 .. j0 + 63, elements e0 .. e0 + 63 of the a (or b) vectors.
// dst[e][j] = scale_j * buffer[off_j + shift + e] (bf16, or fp32 for the tf32 GEMM), zero for j >= pairs.
template <class Out>
__global__ void __launch_bounds__(256) rank1_operands_kernel(const float* __restrict__ buffer,
                                                             const int64_t* __restrict__ off,
                                                             const float* __restrict__ weight, float wscale,
                                                             int64_t shift, int n_elem, int pairs, int kp,
                                                             Out* __restrict__ dst) {
  __shared__ float tile[TJ][TE + 1];
  const int j0 = blockIdx.x * TJ, e0 = blockIdx.y * TE;
  const int tx = threadIdx.x & 63, ty = threadIdx.x >> 6;  // 64 x 4
  for (int jj = ty; jj < TJ; jj += 4) {
    const int j = j0 + jj, e = e0 + tx;
    float v = 0.f;
    if (j < pairs && e < n_elem) {
      v = buffer[off[j] + shift + e];
      if (weight) v *= weight[j] * wscale;
    }
    tile[jj][tx] = v;
  }
  __syncthreads();
  for (int ee = ty; ee < TE; ee += 4) {
    const int e = e0 + ee, j = j0 + tx;
    if (e < n_elem && j < kp) store_operand(dst + static_cast<int64_t>(e) * kp + j, tile[tx][ee]);
  }
}

// out[o, i] (+)= scale * sum_j w_j a_j[o] b_j[i] in fp32, a_j = buffer + off_j, b_j = a_j + n_out (or b_j = a_j with
// n_out = 1, a = 1: the 1-D case eps_j[i]). One thread per output element.
__global__ void __launch_bounds__(256) rank1_small_kernel(const float* __restrict__ buffer,
                                                          const int64_t* __restrict__ off,
                                                          const float* __restrict__ weight, float scale, int n_out,
                                                          int n_in, int one_d, int pairs, float* __restrict__ out) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= n_out * n_in) return;
  const int o = idx / n_in, i = idx - o * n_in;
  float acc = 0.f;
  for (int j = 0; j < pairs; ++j) {
    const float* base = buffer + off[j];
    const float av = one_d ? 1.f : base[o];
    const float bv = one_d ? base[i] : base[n_out + i];
    acc = fmaf(weight[j] * av, bv, acc);
  }
  out[idx] = acc * scale;
}

// torch.optim.AdamW (weight_decay = 0): m = b1 m + (1 - b1) g; v = b2 v + (1 - b2) g^2;
// p -= (lr / (1 - b1^t)) m / (sqrt(v) / sqrt(1 - b2^t) + eps).
__global__ void __launch_bounds__(256) adam_kernel(float* __restrict__ p, float* __restrict__ m,
                                                   float* __restrict__ v, const float* __restrict__ g, int64_t n,
                                                   float lr, float b1, float b2, float eps, float bc1, float bc2_sqrt) {
  const float step_size = lr / bc1;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float gi = g[i];
    const float mi = b1 * m[i] + (1.f - b1) * gi;
    const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    m[i] = mi;
    v[i] = vi;
    const float denom = sqrtf(vi) / bc2_sqrt + eps;
    p[i] -= step_size * mi / denom;
  }
}

}  // namespace update
}  // namespace noise

using namespace noise::update;

extern "C" {

int noise_rank1_operands(const float* buffer, const int64_t* offsets, const float* weight, float weight_scale,
                         int64_t shift, int n_elem, int pairs, int k_padded, void* dst, void* stream) {
  if (!buffer || !offsets || !dst) return NOISE_ERR_ARGUMENT;
  if (n_elem < 1 || pairs < 1 || k_padded < pairs || shift < 0) return NOISE_ERR_SHAPE;
  dim3 grid((k_padded + TJ - 1) / TJ, (n_elem + TE - 1) / TE);
  rank1_operands_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      buffer, offsets, weight, weight_scale, shift, n_elem, pairs, k_padded, static_cast<__nv_bfloat16*>(dst));
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_rank1_operands_f32(const float* buffer, const int64_t* offsets, const float* weight, float weight_scale,
                             int64_t shift, int n_elem, int pairs, int k_padded, float* dst, void* stream) {
  if (!buffer || !offsets || !dst) return NOISE_ERR_ARGUMENT;
  if (n_elem < 1 || pairs < 1 || k_padded < pairs || shift < 0) return NOISE_ERR_SHAPE;
  dim3 grid((k_padded + TJ - 1) / TJ, (n_elem + TE - 1) / TE);
  rank1_operands_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      buffer, offsets, weight, weight_scale, shift, n_elem, pairs, k_padded, dst);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_rank1_small(const float* buffer, const int64_t* offsets, const float* weight, float scale, int n_out,
                      int n_in, int one_d, int pairs, float* out, void* stream) {
  if (!buffer || !offsets || !weight || !out) return NOISE_ERR_ARGUMENT;
  if (n_out < 1 || n_in < 1 || pairs < 0) return NOISE_ERR_SHAPE;
  const int n = n_out * n_in;
  rank1_small_kernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      buffer, offsets, weight, scale, n_out, n_in, one_d, pairs, out);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_adam_step(float* param, float* exp_avg, float* exp_avg_sq, const float* grad, int64_t n, float lr,
                    float beta1, float beta2, float eps, int step, void* stream) {
  if (!param || !exp_avg || !exp_avg_sq || !grad) return NOISE_ERR_ARGUMENT;
  if (n < 0 || step < 1) return NOISE_ERR_SHAPE;
  if (n == 0) return NOISE_OK;
  const float bc1 = 1.f - powf(beta1, static_cast<float>(step));
  const float bc2 = 1.f - powf(beta2, static_cast<float>(step));
  int blocks = static_cast<int>((n + 255) / 256);
  if (blocks > 148 * 8) blocks = 148 * 8;
  adam_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(param, exp_avg, exp_avg_sq, grad, n, lr, beta1,
                                                                     beta2, eps, bc1, sqrtf(bc2));
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

}  // extern "C"
