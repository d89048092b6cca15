// The identity phase's readout cycle (reference train/speedrun/run.py:3569-3686) on sm_100a: the per-logit part of
// the cycle weights, the cycle's finish, and coordinate_change (the LM head's finite coordinate change).
//
// top_credit(model, x, y) moves each token's final stream x along the 512 directions of a signed Hadamard basis h by a
// step sigma rms(x) and reads the change of the softcapped cross-entropy through the LM head without recomputing the
// logits: with base = x W (logits), c = h W, z = base inv0, the moved partition sum_v e^(softcap(z + step c_v inv /
// inv0 ...)) is expanded to third order in the step, so it needs per token f = e^(15 tanh(z / 15)) times its softcap
// derivatives g1, g2, g3 (this file's cycle_weights_kernel) contracted with c, c^2, c^3 (GEMMs), then combined per
// (token, direction) in cycle_finish_kernel.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "noise_b200.h"

namespace noise {
namespace cycle {

constexpr int D = NOISE_N_EMBD;   // 512
constexpr int V = NOISE_VOCAB;    // 4096
constexpr float CAP = 15.f;       // SOFTCAP
constexpr float EPS = 1.1920928955078125e-07f;

template <int N>
__device__ __forceinline__ void block_sums(float (&v)[N], float* red) {  // 256 threads; every thread gets the sums
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < N; ++i)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v[i] += __shfl_xor_sync(0xffffffffu, v[i], o);
  __syncthreads();
  if (lane == 0)
#pragma unroll
    for (int i = 0; i < N; ++i) red[i * 8 + w] = v[i];
  __syncthreads();
#pragma unroll
  for (int i = 0; i < N; ++i) {
    float s = 0.f;
    for (int k = 0; k < 8; ++k) s += red[i * 8 + k];
    v[i] = s;
  }
}

__device__ __forceinline__ float softcap(float x) { return CAP * tanhf(x / CAP); }

// One block per token: sq = |x|^2, inv0 = rsqrt(sq / 512 + eps); over the 4096 logits z = base inv0,
// t = tanh(z / 15), f = e^(15 t), g1 = 1 - t^2, d1 = -2 t g1 / 15, d2 = -2 g1 (1 - 3 t^2) / 15^2, g2 = g1^2 + d1,
// g3 = g1^3 + 3 g1 d1 + d2: fg1 = f g1 (fp32), fast = bf16(f z g2, f z^2 g3, f g2, f z g3, f g3), total = sum f,
// rows = (sum f z g1, sum f z^2 g2, sum f z^3 g3), base_y = base[y].
__global__ void __launch_bounds__(256) cycle_weights_kernel(const float* __restrict__ x, const float* __restrict__ base,
                                                            const int64_t* __restrict__ y, int n,
                                                            float* __restrict__ fg1, __nv_bfloat16* __restrict__ fast,
                                                            float* __restrict__ rows, float* __restrict__ total,
                                                            float* __restrict__ sq_out, float* __restrict__ base_y) {
  __shared__ float red[4 * 8];
  const int64_t tok = blockIdx.x;
  float sq[1] = {0.f};
  for (int i = threadIdx.x; i < D; i += 256) {
    const float v = x[tok * D + i];
    sq[0] += v * v;
  }
  block_sums(sq, red);
  const float inv0 = rsqrtf(sq[0] / D + EPS);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const int64_t nv = static_cast<int64_t>(n) * V;
  for (int v = threadIdx.x; v < V; v += 256) {
    const int64_t o = tok * V + v;
    const float b = base[o];
    const float z = b * inv0;
    const float t = tanhf(z / CAP);
    const float f = expf(CAP * t);
    const float g1 = 1.f - t * t;
    const float d1 = -2.f * t * g1 / CAP;
    const float d2 = -2.f * g1 * (1.f - 3.f * t * t) / (CAP * CAP);
    const float g2 = g1 * g1 + d1, g3 = g1 * g1 * g1 + 3.f * g1 * d1 + d2;
    const float fz = f * z, fzz = f * z * z;
    acc[0] += f;
    acc[1] += fz * g1;
    acc[2] += fzz * g2;
    acc[3] += fzz * z * g3;
    fg1[o] = f * g1;
    fast[o] = __float2bfloat16_rn(fz * g2);
    fast[nv + o] = __float2bfloat16_rn(fzz * g3);
    fast[2 * nv + o] = __float2bfloat16_rn(f * g2);
    fast[3 * nv + o] = __float2bfloat16_rn(fz * g3);
    fast[4 * nv + o] = __float2bfloat16_rn(f * g3);
    if (v == y[tok]) base_y[tok] = b;
  }
  block_sums(acc, red);
  if (threadIdx.x == 0) {
    total[tok] = acc[0];
    rows[tok * 3] = acc[1];
    rows[tok * 3 + 1] = acc[2];
    rows[tok * 3 + 2] = acc[3];
    sq_out[tok] = sq[0];
  }
}

// Per (token i, direction r): steps = sigma max(sqrt(sq / 512), 1e-6); inv = rsqrt((sq + 2 steps dots + steps^2 512)
// / 512 + eps); inv0 = rsqrt(sq / 512 + eps); delta = inv / inv0 - 1; s = steps inv; the moved partition ratio from
// the contractions (exact = fg1 c^T; prods = bf16 of fast_k c^(1, 1, 2, 2, 3)^T) and the rows; out = (moved - clean) /
// steps with clean = log(total) - softcap(base_y inv0), moved = log(total) + log1p(ratio / total) -
// softcap((base_y + steps c[r, y]) inv).
__global__ void __launch_bounds__(256) cycle_finish_kernel(const float* __restrict__ dots, const float* __restrict__ sq,
                                                           const float* __restrict__ exact,
                                                           const float* __restrict__ prods,
                                                           const float* __restrict__ rows,
                                                           const float* __restrict__ total,
                                                           const float* __restrict__ base_y,
                                                           const float* __restrict__ c, const int64_t* __restrict__ y,
                                                           int n, int R, float sigma, float* __restrict__ out) {
  const int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (idx >= static_cast<int64_t>(n) * R) return;
  const int64_t i = idx / R;
  const int r = static_cast<int>(idx - i * R);
  const int64_t nr = static_cast<int64_t>(n) * R;
  const float sqi = sq[i];
  const float steps = sigma * fmaxf(sqrtf(sqi / D), 1e-6f);
  const float inv = rsqrtf((sqi + 2.f * steps * dots[idx] + steps * steps * D) / D + EPS);
  const float inv0 = rsqrtf(sqi / D + EPS);
  const float delta = inv / inv0 - 1.f, s = steps * inv;
  auto bf = [](float v) { return __bfloat162float(__float2bfloat16_rn(v)); };  // the bf16 GEMM outputs
  const float f0 = bf(prods[idx]), f1 = bf(prods[nr + idx]), f2 = bf(prods[2 * nr + idx]);
  const float f3 = bf(prods[3 * nr + idx]), f4 = bf(prods[4 * nr + idx]);
  const float* rw = rows + i * 3;
  const float ratio = s * exact[idx] + delta * s * f0 + 0.5f * delta * delta * s * f1 + 0.5f * s * s * f2 +
                      0.5f * delta * s * s * f3 + s * s * s / 6.f * f4 + delta * rw[0] +
                      0.5f * delta * delta * rw[1] + delta * delta * delta / 6.f * rw[2];
  const float tot = total[i], part = logf(tot), by = base_y[i];
  const float clean = part - softcap(by * inv0);
  const float moved = part + log1pf(ratio / tot) - softcap((by + steps * c[static_cast<int64_t>(r) * V + y[i]]) * inv);
  out[idx] = (moved - clean) / steps;
}

// coordinate_change (run.py:3569-3577), one block per row: z = softcap(raw), up / down = softcap(raw +- hs),
// w = softmax(z); (log1p(w expm1(up - z)) - log1p(w expm1(down - z)) - [v = y] (up - down)) / (2 hs).
template <typename T>
__global__ void __launch_bounds__(256) coordinate_change_kernel(const T* __restrict__ raw,
                                                                const int64_t* __restrict__ targets, float hs,
                                                                float* __restrict__ out) {
  __shared__ float red[2 * 8];
  const int64_t row = blockIdx.x;
  const T* rr = raw + row * V;
  float zmax[1] = {-3.402823466e38f};
  for (int v = threadIdx.x; v < V; v += 256) zmax[0] = fmaxf(zmax[0], softcap(static_cast<float>(rr[v])));
  {  // block max
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) zmax[0] = fmaxf(zmax[0], __shfl_xor_sync(0xffffffffu, zmax[0], o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = zmax[0];
    __syncthreads();
    float m = red[0];
    for (int k = 1; k < 8; ++k) m = fmaxf(m, red[k]);
    zmax[0] = m;
  }
  float se[1] = {0.f};
  for (int v = threadIdx.x; v < V; v += 256) se[0] += expf(softcap(static_cast<float>(rr[v])) - zmax[0]);
  block_sums(se, red);
  const int64_t y = targets[row];
  for (int v = threadIdx.x; v < V; v += 256) {
    const float a = static_cast<float>(rr[v]);
    const float z = softcap(a), up = softcap(a + hs), down = softcap(a - hs);
    const float w = expf(z - zmax[0]) / se[0];
    float ch = log1pf(w * expm1f(up - z)) - log1pf(w * expm1f(down - z));
    if (v == y) ch -= up - down;
    out[row * V + v] = ch / (2.f * hs);
  }
}

}  // namespace cycle
}  // namespace noise

using namespace noise::cycle;

extern "C" {

int noise_cycle_weights(const float* x, const float* base, const int64_t* targets, int tokens, float* fg1, void* fast,
                        float* rows, float* total, float* sq, float* base_y, void* stream) {
  if (!x || !base || !targets || !fg1 || !fast || !rows || !total || !sq || !base_y) return NOISE_ERR_ARGUMENT;
  if (tokens < 0) return NOISE_ERR_SHAPE;
  if (tokens == 0) return NOISE_OK;
  cycle_weights_kernel<<<tokens, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, base, targets, tokens, fg1, static_cast<__nv_bfloat16*>(fast), rows, total, sq, base_y);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_cycle_finish(const float* dots, const float* sq, const float* exact, const float* prods, const float* rows,
                       const float* total, const float* base_y, const float* c, const int64_t* targets, int tokens,
                       int directions, float sigma, float* out, void* stream) {
  if (!dots || !sq || !exact || !prods || !rows || !total || !base_y || !c || !targets || !out)
    return NOISE_ERR_ARGUMENT;
  if (tokens < 0 || directions < 1) return NOISE_ERR_SHAPE;
  if (tokens == 0) return NOISE_OK;
  const int64_t total_n = static_cast<int64_t>(tokens) * directions;
  cycle_finish_kernel<<<static_cast<unsigned>((total_n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      dots, sq, exact, prods, rows, total, base_y, c, targets, tokens, directions, sigma, out);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_coordinate_change(const void* raw, int raw_dtype, const int64_t* targets, int rows, float head_sigma,
                            float* out, void* stream) {
  if (!raw || !targets || !out) return NOISE_ERR_ARGUMENT;
  if (raw_dtype != NOISE_DTYPE_F32 && raw_dtype != NOISE_DTYPE_BF16) return NOISE_ERR_ARGUMENT;
  if (rows < 0 || !(head_sigma > 0.f)) return NOISE_ERR_SHAPE;
  if (rows == 0) return NOISE_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (raw_dtype == NOISE_DTYPE_BF16)
    coordinate_change_kernel<__nv_bfloat16><<<rows, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(raw), targets,
                                                                  head_sigma, out);
  else
    coordinate_change_kernel<float><<<rows, 256, 0, s>>>(static_cast<const float*>(raw), targets, head_sigma, out);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

}  // extern "C"
