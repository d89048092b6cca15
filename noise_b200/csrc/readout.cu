// The track-1 readout scorers' custom ops (reference train/val/run.py, `recipe` section: noise_record::future_scores
// :1633-1750, noise_record::key_response and noise_record::routed_response :541-637, noise_record::
// future_query_response :1780-1835) on sm_100a.
//
// All four are attention-like reductions of a finite change of one side of a softmax over head_dim 64. Each has a
// tcgen05 form (the *_ws entry points: query_tc.cuh, column_tc.cuh for future_scores / key_response, routed_tc.cuh;
// the reference's tf32x3 dots as kind::tf32 MMAs, routed_response's bf16 dots as kind::f16 with bf16-rounded
// outputs) and the fp32 CUDA-core form in this file (the entry points without a workspace):
//   future_scores  out[h, p, m] = sum over receivers s with 0 < s - (start + m) <= window of
//                  (a (e^x - 1) c + (a + a (e^x - 1)) g . dv) / (1 + a (e^x - 1)),  x = q_s . dk_pm / 8,
//                  a = A[h, s, m], c = C[h, s, m], g = target_s;
//   key_response   out[h, p, m] = sum over queries s of change / (1 + change) c, change = a (e^(q_s . dk_pm / 8) - 1)
//                  (A is zero outside the source's window, as the attention probabilities it is);
//   query_response out[m, p, h] = (sum_k change v_k - sum_k change base) / (1 + sum_k change),
//                  change = P[h, m, k] (e^(dq_mph . k_k / 8) - 1);
//   routed_response out[m, p, h] = bf16(w V) + (e^-dlse - 1) rest, w = bf16(p (e^(ds - dlse) - 1)),
//                  ds = bf16(dq . k) / 8, dlse = log1p(sum_k p (e^ds - 1)) over the routed keys.
// The CUDA-core kernels keep their per-column (or per-probe) state in registers, stage the other side's tiles in
// shared memory, and never materialise a [receiver x column] tensor.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "noise_b200.h"

namespace noise {
namespace readout {

constexpr int D = 64;
constexpr float SCALE = 0.125f;  // 64 ** -0.5

struct View3 {
  const float* p;
  int64_t s0, s1, s2;
  __device__ __forceinline__ float at(int64_t i, int64_t j, int64_t k) const { return p[i * s0 + j * s1 + k * s2]; }
};

static View3 view(const noise_view3_t& v) { return View3{v.data, v.stride0, v.stride1, v.stride2}; }

// ---------------------------------------------------------------------------------------------------------------
// future_scores / key_response: one block = 64 columns (col = p * M + m) of one head; thread t owns column t % 64
// (its dk, dv in registers) and receivers s = 4 i + t / 64 of each 32-receiver tile; q (and target) tiles are
// staged in shared memory and read as broadcasts.
// ---------------------------------------------------------------------------------------------------------------
constexpr int FC = 64;  // columns per block
constexpr int FQ = 32;  // receivers per tile

template <bool VALUES>
__global__ void __launch_bounds__(256) column_scores_kernel(View3 q, View3 g, const float* __restrict__ dk,
                                                            const float* __restrict__ dv, View3 a, View3 c, int T,
                                                            int M, int P, int source_start, int query_start,
                                                            int window, float* __restrict__ out) {
  __shared__ __align__(16) float sq[FQ][D];
  __shared__ __align__(16) float sg[VALUES ? FQ : 1][D];
  __shared__ float red[4][FC];
  const int h = blockIdx.y, tid = threadIdx.x;
  const int lc = tid % FC, grp = tid / FC;
  const int col = blockIdx.x * FC + lc;
  const bool live = col < P * M;
  const int m = live ? col % M : 0;
  float k[D], v[VALUES ? D : 1];
  {
    const float* kp = dk + (static_cast<int64_t>(h) * P * M + (live ? col : 0)) * D;
#pragma unroll
    for (int d = 0; d < D; d += 4) {
      const float4 t4 = *reinterpret_cast<const float4*>(kp + d);
      k[d] = t4.x, k[d + 1] = t4.y, k[d + 2] = t4.z, k[d + 3] = t4.w;
    }
    if constexpr (VALUES) {
      const float* vp = dv + (static_cast<int64_t>(h) * P * M + (live ? col : 0)) * D;
#pragma unroll
      for (int d = 0; d < D; d += 4) {
        const float4 t4 = *reinterpret_cast<const float4*>(vp + d);
        v[d] = t4.x, v[d + 1] = t4.y, v[d + 2] = t4.z, v[d + 3] = t4.w;
      }
    }
  }
  // receivers this block can need: the union of its columns' windows (block columns are consecutive)
  const int c_lo = blockIdx.x * FC, c_hi = min(c_lo + FC, P * M) - 1;
  const int m_lo = (c_hi / M > c_lo / M) ? 0 : c_lo % M;
  const int m_hi = (c_hi / M > c_lo / M) ? M - 1 : c_hi % M;
  // future_scores: s in (start + m, start + m + window]; key_response: query index s with absolute position
  // query_start + s in [source_start + m, source_start + m + window]
  const int off = VALUES ? 1 : 0;
  const int base = VALUES ? source_start : source_start - query_start;
  const int s_first = max(0, base + m_lo + off), s_last = min(T - 1, base + m_hi + window);
  const int my_first = base + m + off, my_last = base + m + window;
  float acc = 0.f;
  for (int s0 = s_first - s_first % FQ; s0 <= s_last; s0 += FQ) {
    __syncthreads();
    for (int i = tid; i < FQ * D; i += 256) {
      const int r = i / D, d = i % D, s = s0 + r;
      sq[r][d] = s < T ? q.at(h, s, d) : 0.f;
      if constexpr (VALUES) sg[r][d] = s < T ? g.at(h, s, d) : 0.f;
    }
    __syncthreads();
#pragma unroll 1
    for (int r = grp; r < FQ; r += 4) {
      const int s = s0 + r;
      if (!live || s < my_first || s > my_last || s >= T) continue;
      float x0 = 0.f, x1 = 0.f, y0 = 0.f, y1 = 0.f;
#pragma unroll
      for (int d = 0; d < D; d += 4) {
        const float4 qq = *reinterpret_cast<const float4*>(&sq[r][d]);
        x0 = fmaf(qq.x, k[d], x0);
        x1 = fmaf(qq.y, k[d + 1], x1);
        x0 = fmaf(qq.z, k[d + 2], x0);
        x1 = fmaf(qq.w, k[d + 3], x1);
        if constexpr (VALUES) {
          const float4 gg = *reinterpret_cast<const float4*>(&sg[r][d]);
          y0 = fmaf(gg.x, v[d], y0);
          y1 = fmaf(gg.y, v[d + 1], y1);
          y0 = fmaf(gg.z, v[d + 2], y0);
          y1 = fmaf(gg.w, v[d + 3], y1);
        }
      }
      const float x = (x0 + x1) * SCALE;
      const float av = a.at(h, s, m), cv = c.at(h, s, m);
      const float changed = av * expm1f(x);
      if constexpr (VALUES)
        acc += (changed * cv + (av + changed) * (y0 + y1)) / (1.f + changed);
      else
        acc += changed / (1.f + changed) * cv;
    }
  }
  red[grp][lc] = acc;
  __syncthreads();
  if (grp == 0 && live)
    out[static_cast<int64_t>(h) * P * M + col] = (red[0][lc] + red[1][lc]) + (red[2][lc] + red[3][lc]);
}

// ---------------------------------------------------------------------------------------------------------------
// query_response: one block = 32 probes of one (token m, head h); key tiles of 64 (skipped when every probability
// in the tile is zero); phase 1 change[p][k] into shared memory, phase 2 numerator[p][d] += change V.
// ---------------------------------------------------------------------------------------------------------------
constexpr int QP = 32, QK = 64;
constexpr int QUERY_SMEM = ((QP + QK) * (D + 4) + QK * D + QP * (QK + 1) + QK) * 4;

__global__ void __launch_bounds__(256) query_response_kernel(const float* __restrict__ dq, View3 keys, View3 values,
                                                             View3 prob, View3 base, int Mt, int P, int H, int T,
                                                             float* __restrict__ out) {
  extern __shared__ __align__(16) float qsm[];
  float(*sdq)[D + 4] = reinterpret_cast<float(*)[D + 4]>(qsm);              // [QP][D + 4]
  float(*sk)[D + 4] = reinterpret_cast<float(*)[D + 4]>(qsm + QP * (D + 4));  // [QK][D + 4]
  float(*sv)[D] = reinterpret_cast<float(*)[D]>(qsm + (QP + QK) * (D + 4));   // [QK][D]
  float(*sch)[QK + 1] = reinterpret_cast<float(*)[QK + 1]>(qsm + (QP + QK) * (D + 4) + QK * D);  // [QP][QK + 1]
  float* sa = qsm + (QP + QK) * (D + 4) + QK * D + QP * (QK + 1);           // [QK]
  __shared__ int any;
  const int tm = blockIdx.y / H, h = blockIdx.y % H, tid = threadIdx.x;
  const int p0 = blockIdx.x * QP;
  for (int i = tid; i < QP * D; i += 256) {
    const int r = i / D, d = i % D, p = p0 + r;
    sdq[r][d] = p < P ? dq[((static_cast<int64_t>(tm) * P + p) * H + h) * D + d] : 0.f;
  }
  const int pr = tid / 8, part = tid % 8;  // phase 1: probe pr, keys part + 8 e; phase 2: dims 8 part .. 8 part + 7
  float num[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  float partition = 0.f;
  for (int k0 = 0; k0 < T; k0 += QK) {
    __syncthreads();
    if (tid == 0) any = 0;
    __syncthreads();
    if (tid < QK) {
      const int kk = k0 + tid;
      const float av = kk < T ? prob.at(h, tm, kk) : 0.f;
      sa[tid] = av;
      if (av != 0.f) any = 1;
    }
    __syncthreads();
    if (!any) continue;  // a causal / window-masked tile contributes exactly nothing
    for (int i = tid; i < QK * D; i += 256) {
      const int r = i / D, d = i % D, kk = k0 + r;
      sk[r][d] = kk < T ? keys.at(h, kk, d) : 0.f;
      sv[r][d] = kk < T ? values.at(h, kk, d) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int kr = part + 8 * e;  // rows 68 floats apart: the 8 parts hit distinct banks
      float x0 = 0.f, x1 = 0.f;
#pragma unroll
      for (int d = 0; d < D; d += 4) {
        const float4 qq = *reinterpret_cast<const float4*>(&sdq[pr][d]);
        const float4 kk4 = *reinterpret_cast<const float4*>(&sk[kr][d]);
        x0 = fmaf(qq.x, kk4.x, x0);
        x1 = fmaf(qq.y, kk4.y, x1);
        x0 = fmaf(qq.z, kk4.z, x0);
        x1 = fmaf(qq.w, kk4.w, x1);
      }
      sch[pr][kr] = sa[kr] * expm1f((x0 + x1) * SCALE);
    }
    __syncthreads();
#pragma unroll 4
    for (int kr = 0; kr < QK; ++kr) {
      const float ch = sch[pr][kr];
      partition += ch;
      const float4 v0 = *reinterpret_cast<const float4*>(&sv[kr][part * 8]);
      const float4 v1 = *reinterpret_cast<const float4*>(&sv[kr][part * 8 + 4]);
      num[0] = fmaf(ch, v0.x, num[0]);
      num[1] = fmaf(ch, v0.y, num[1]);
      num[2] = fmaf(ch, v0.z, num[2]);
      num[3] = fmaf(ch, v0.w, num[3]);
      num[4] = fmaf(ch, v1.x, num[4]);
      num[5] = fmaf(ch, v1.y, num[5]);
      num[6] = fmaf(ch, v1.z, num[6]);
      num[7] = fmaf(ch, v1.w, num[7]);
    }
  }
  const int p = p0 + pr;
  if (p < P) {
    float* o = out + ((static_cast<int64_t>(tm) * P + p) * H + h) * D + part * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = (num[e] - partition * base.at(h, tm, part * 8 + e)) / (1.f + partition);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// routed_response: one block = 32 probes of one (token, head) against its K <= 256 routed keys (bf16 operands).
// ---------------------------------------------------------------------------------------------------------------
constexpr int RP = 32, RK = 256;

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__global__ void __launch_bounds__(256) routed_response_kernel(const __nv_bfloat16* __restrict__ dq,
                                                              const __nv_bfloat16* __restrict__ keys,
                                                              const __nv_bfloat16* __restrict__ values,
                                                              const float* __restrict__ prob,
                                                              const float* __restrict__ rest, int P, int H, int K,
                                                              float* __restrict__ out) {
  extern __shared__ __align__(16) float rsm[];
  // shared memory sized by the routed keys K (K <= 256)
  constexpr int KP = D + 4;         // key row pitch: the 8 key-parts of a quarter warp hit distinct banks
  const int KS = K + 1;             // row pitch of the ds / weight rows
  float* sk = rsm;                  // [K][D + 4] keys (fp32 copies of bf16)
  float* sv = sk + K * KP;          // [K][D] values
  float* sds = sv + K * D;          // [RP][K + 1] ds, then the bf16 weights
  float* sq = sds + RP * KS;        // [RP][D] probes
  float* sp = sq + RP * D;          // [K] probabilities
  float* sdl = sp + K;              // [RP] dlse
  const int tm = blockIdx.y / H, h = blockIdx.y % H, tid = threadIdx.x;
  const int p0 = blockIdx.x * RP;
  const int64_t kvb = (static_cast<int64_t>(tm) * H + h) * K;
  for (int i = tid; i < K * D; i += 256) {
    const int r = i / D, d = i % D;
    sk[r * KP + d] = __bfloat162float(keys[(kvb + r) * D + d]);
    sv[r * D + d] = __bfloat162float(values[(kvb + r) * D + d]);
  }
  for (int i = tid; i < K; i += 256) sp[i] = prob[kvb + i];
  for (int i = tid; i < RP * D; i += 256) {
    const int r = i / D, d = i % D, p = p0 + r;
    sq[i] = p < P ? __bfloat162float(dq[((static_cast<int64_t>(tm) * P + p) * H + h) * D + d]) : 0.f;
  }
  __syncthreads();
  // ds[p][k] = bf16(q . k) / 8 (the dot's bf16 output, as the reference's); 8 threads per probe (one warp holds 4
  // probes), the probe row in registers, key rows read as float4
  const int pr = tid / 8, part = tid % 8;
  float qv[D];
#pragma unroll
  for (int d = 0; d < D; d += 4) {
    const float4 t4 = *reinterpret_cast<const float4*>(sq + pr * D + d);
    qv[d] = t4.x, qv[d + 1] = t4.y, qv[d + 2] = t4.z, qv[d + 3] = t4.w;
  }
  float lsum = 0.f;
  for (int kr = part; kr < K; kr += 8) {
    float x0 = 0.f, x1 = 0.f;
#pragma unroll
    for (int d = 0; d < D; d += 4) {
      const float4 k4 = *reinterpret_cast<const float4*>(sk + kr * KP + d);
      x0 = fmaf(qv[d], k4.x, x0);
      x1 = fmaf(qv[d + 1], k4.y, x1);
      x0 = fmaf(qv[d + 2], k4.z, x0);
      x1 = fmaf(qv[d + 3], k4.w, x1);
    }
    const float ds = bf16r(x0 + x1) * SCALE;
    sds[pr * KS + kr] = ds;
    lsum += sp[kr] * expm1f(ds);
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
  const float dlse = log1pf(lsum);
  for (int kr = part; kr < K; kr += 8) sds[pr * KS + kr] = bf16r(sp[kr] * expm1f(sds[pr * KS + kr] - dlse));
  if (part == 0) sdl[pr] = dlse;
  __syncwarp();  // a probe's weights come from its own 8 threads, all in this warp
  // moved[p][d] = bf16(sum_k w[p][k] v[k][d]) + (e^-dlse - 1) rest[d]; thread: probe pr, dims 8 part .. + 7
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
  for (int kr = 0; kr < K; ++kr) {
    const float w = sds[pr * KS + kr];
    const float4 v0 = *reinterpret_cast<const float4*>(sv + kr * D + part * 8);
    const float4 v1 = *reinterpret_cast<const float4*>(sv + kr * D + part * 8 + 4);
    acc[0] = fmaf(w, v0.x, acc[0]);
    acc[1] = fmaf(w, v0.y, acc[1]);
    acc[2] = fmaf(w, v0.z, acc[2]);
    acc[3] = fmaf(w, v0.w, acc[3]);
    acc[4] = fmaf(w, v1.x, acc[4]);
    acc[5] = fmaf(w, v1.y, acc[5]);
    acc[6] = fmaf(w, v1.z, acc[6]);
    acc[7] = fmaf(w, v1.w, acc[7]);
  }
  const int p = p0 + pr;
  if (p < P) {
    const float em = expm1f(-sdl[pr]);
    const float* rs = rest + (static_cast<int64_t>(tm) * H + h) * D + part * 8;
    float* o = out + ((static_cast<int64_t>(tm) * P + p) * H + h) * D + part * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = bf16r(acc[e]) + em * rs[e];
  }
}

constexpr int routed_smem(int K) { return (K * (D + 4) + K * D + RP * (K + 1) + RP * D + K + RP) * 4; }

static bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace readout
}  // namespace noise

#include "query_tc.cuh"
#include "routed_tc.cuh"
#include "column_tc.cuh"

namespace {

PFN_cuTensorMapEncodeTiled_v12000 qt_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// fp32 [outer, inner] rows, box_rows x 32-column boxes (128 bytes), 128-byte swizzle
int qt_map(CUtensorMap* map, const float* base, uint64_t inner, uint64_t outer, uint32_t box_rows = 64) {
  auto fn = qt_encode();
  if (!fn) return NOISE_ERR_CUDA;
  if (reinterpret_cast<uintptr_t>(base) & 15) return NOISE_ERR_ALIGN;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * 4};
  cuuint32_t box[2] = {32, box_rows};
  cuuint32_t el[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, el,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NOISE_OK : NOISE_ERR_CUDA;
}

// bf16 rows of 64 (128 bytes): a 2-D [outer, 64] map with 64 x box_rows boxes, or (heads > 0) the 3-D (64, heads,
// outer) view of a [outer, heads, 64] buffer with 64 x 1 x box_rows boxes; 128-byte swizzle
int rt_map(CUtensorMap* map, const void* base, uint64_t outer, int heads, uint32_t box_rows) {
  auto fn = qt_encode();
  if (!fn) return NOISE_ERR_CUDA;
  if (reinterpret_cast<uintptr_t>(base) & 15) return NOISE_ERR_ALIGN;
  const uint32_t rank = heads > 0 ? 3 : 2;
  cuuint64_t dims[3] = {64, heads > 0 ? static_cast<cuuint64_t>(heads) : outer, outer};
  cuuint64_t strides[2] = {128, heads > 0 ? static_cast<cuuint64_t>(heads) * 128 : 0};
  cuuint32_t box[3] = {64, heads > 0 ? 1u : box_rows, box_rows};
  cuuint32_t el[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims, strides, box, el,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NOISE_OK : NOISE_ERR_CUDA;
}

// e^x - 1 of the library's own (expm1_f2) over n values, two per thread: the numerics check of the scorers' exponential
__global__ void __launch_bounds__(256) expm1_check_kernel(const float* __restrict__ x, float* __restrict__ out,
                                                          int64_t n) {
  for (int64_t i = 2 * (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x); i < n;
       i += 2 * static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float2 e = noise::expm1_f2(make_float2(x[i], i + 1 < n ? x[i + 1] : 0.f));
    out[i] = e.x;
    if (i + 1 < n) out[i + 1] = e.y;
  }
}

// future_scores / key_response on tcgen05: 256-byte status block, then q (and target) as tf32 hi / lo planes
size_t ct_plane_bytes(int heads, int tokens) {
  return static_cast<size_t>(heads) * ((tokens + 63) / 64 * 64) * noise::readout::D * 4;
}

template <bool VALUES>
int column_ws(const noise_view3_t* q, const noise_view3_t* target, const float* dk, const float* dv,
              const noise_view3_t* a, const noise_view3_t* c, int heads, int tokens, int probes, int sources,
              int first_off, int span, float* out, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace noise::readout;
  using L = CtLayout<VALUES>;
  const size_t plane = ct_plane_bytes(heads, tokens);
  if (!workspace || workspace_bytes < 256 + (VALUES ? 4 : 2) * plane) return NOISE_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) || !a16(dk) || (VALUES && !a16(dv))) return NOISE_ERR_ALIGN;
  const int64_t cols = static_cast<int64_t>(probes) * sources;
  if (cols > 0x7FFFFFFF) return NOISE_ERR_SHAPE;
  // the kernel's TMA row coordinates (head h's rows at h Tp) are int32
  if (static_cast<int64_t>(heads) * ((tokens + 63) / 64 * 64) > 0x7FFFFFFF) return NOISE_ERR_SHAPE;
  const int tp = (tokens + 63) / 64 * 64;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* status = static_cast<int*>(workspace);
  float* qhi = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + 256);
  float* qlo = qhi + plane / 4;
  float* ghi = qlo + plane / 4;
  float* glo = ghi + plane / 4;
  CtMaps maps;
  int rc;
  const uint64_t rows = static_cast<uint64_t>(heads) * tp;
  if ((rc = qt_map(&maps.qhi, qhi, D, rows, CT_RECV)) || (rc = qt_map(&maps.qlo, qlo, D, rows, CT_RECV))) return rc;
  if (VALUES) {
    if ((rc = qt_map(&maps.ghi, ghi, D, rows, CT_RECV)) || (rc = qt_map(&maps.glo, glo, D, rows, CT_RECV))) return rc;
  } else {
    maps.ghi = maps.qhi;
    maps.glo = maps.qlo;
  }
  if (cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess) return NOISE_ERR_CUDA;
  col_split_kernel<<<dim3(tp / 64, heads), 256, 0, s>>>(view(*q), tokens, tp, qhi, qlo);
  if (VALUES) col_split_kernel<<<dim3(tp / 64, heads), 256, 0, s>>>(view(*target), tokens, tp, ghi, glo);
  if (cudaFuncSetAttribute(column_tc_kernel<VALUES>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM))
    return NOISE_ERR_CUDA;
  CtArgs args{dk, dv, view(*a), view(*c), out, tokens, sources, probes, heads, tp, first_off, span, status};
  column_tc_kernel<VALUES><<<dim3(static_cast<unsigned>((cols + CT_COLS - 1) / CT_COLS), heads), CT_THREADS, L::SMEM,
                             s>>>(maps, args);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

// workspace: 256-byte status block, keys hi / lo and values^T hi / lo (fp32, H * Tp * 64 each), live flags
struct QtWorkspace {
  int64_t nt, tp, plane, live_bytes;
  QtWorkspace(int tokens, int heads, int keys_len)
      : nt((keys_len + noise::readout::QT_KEYS - 1) / noise::readout::QT_KEYS), tp(nt * noise::readout::QT_KEYS),
        plane(static_cast<int64_t>(heads) * tp * noise::readout::D * 4),
        live_bytes((static_cast<int64_t>(heads) * tokens * nt + 255) / 256 * 256) {}
  size_t bytes() const { return static_cast<size_t>(256 + 4 * plane + live_bytes); }
};

}  // namespace

using namespace noise::readout;

extern "C" {

int noise_future_scores(const noise_view3_t* q, const noise_view3_t* target, const float* dk, const float* dv,
                        const noise_view3_t* a, const noise_view3_t* contrast, int heads, int tokens, int probes,
                        int sources, int source_start, int window, float* out, void* stream) {
  if (!q || !target || !dk || !dv || !a || !contrast || !out || !q->data || !target->data || !a->data ||
      !contrast->data)
    return NOISE_ERR_ARGUMENT;
  if (heads < 1 || tokens < 1 || probes < 1 || sources < 1 || window < 0) return NOISE_ERR_SHAPE;
  if (!a16(dk) || !a16(dv)) return NOISE_ERR_ALIGN;
  dim3 grid((probes * sources + FC - 1) / FC, heads);
  column_scores_kernel<true><<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      view(*q), view(*target), dk, dv, view(*a), view(*contrast), tokens, sources, probes, source_start, 0, window,
      out);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_key_response(const noise_view3_t* q, const float* dk, const noise_view3_t* a, const noise_view3_t* c,
                       int heads, int tokens, int probes, int sources, int source_start, int query_start, int window,
                       float* out, void* stream) {
  if (!q || !dk || !a || !c || !out || !q->data || !a->data || !c->data) return NOISE_ERR_ARGUMENT;
  if (heads < 1 || tokens < 1 || probes < 1 || sources < 1 || window < 0) return NOISE_ERR_SHAPE;
  if (!a16(dk)) return NOISE_ERR_ALIGN;
  dim3 grid((probes * sources + FC - 1) / FC, heads);
  column_scores_kernel<false><<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      view(*q), view(*q), dk, dk, view(*a), view(*c), tokens, sources, probes, source_start, query_start, window,
      out);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_query_response(const float* dq, const noise_view3_t* keys, const noise_view3_t* values,
                         const noise_view3_t* probabilities, const noise_view3_t* base, int tokens, int probes,
                         int heads, int keys_len, float* out, void* stream) {
  if (!dq || !keys || !values || !probabilities || !base || !out || !keys->data || !values->data ||
      !probabilities->data || !base->data)
    return NOISE_ERR_ARGUMENT;
  if (tokens < 1 || probes < 1 || heads < 1 || keys_len < 1) return NOISE_ERR_SHAPE;
  if (cudaFuncSetAttribute(query_response_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, QUERY_SMEM))
    return NOISE_ERR_CUDA;
  dim3 grid((probes + QP - 1) / QP, tokens * heads);
  query_response_kernel<<<grid, 256, QUERY_SMEM, static_cast<cudaStream_t>(stream)>>>(
      dq, view(*keys), view(*values), view(*probabilities), view(*base), tokens, probes, heads, keys_len, out);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_expm1_f32(const float* x, float* out, int64_t n, void* stream) {
  if (!x || !out) return NOISE_ERR_ARGUMENT;
  if (n < 0) return NOISE_ERR_SHAPE;
  if (n == 0) return NOISE_OK;
  const int64_t blocks = std::min<int64_t>((n + 511) / 512, 4096);
  expm1_check_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, out, n);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_routed_response_ws(const void* dq, const void* keys, const void* values, const float* probabilities,
                             const float* rest, int tokens, int probes, int heads, int keys_len, float* out,
                             void* workspace, size_t workspace_bytes, void* stream) {
  if (!dq || !keys || !values || !probabilities || !rest || !out) return NOISE_ERR_ARGUMENT;
  if (tokens < 1 || probes < 1 || heads < 1 || keys_len < 1 || keys_len > RK) return NOISE_ERR_SHAPE;
  if (!workspace || workspace_bytes < NOISE_STATUS_BYTES) return NOISE_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) || !a16(out)) return NOISE_ERR_ALIGN;
  RtArgs a{};
  a.prob = probabilities;
  a.rest = rest;
  a.out = out;
  a.M = tokens;
  a.P = probes;
  a.H = heads;
  a.K = keys_len;
  a.Kp = (keys_len + 31) / 32 * 32;
  a.G = 2 * a.Kp <= 256 ? 2 : 1;
  a.PB = (probes + 63) / 64;
  const int64_t items = static_cast<int64_t>(tokens) * heads * a.PB;
  if (items > 0x7FFFFFFF - 1) return NOISE_ERR_SHAPE;
  // the kernel's TMA row coordinates are int32: a probe block's first row tok P + 64 pb, an item's first key mh K
  if (static_cast<int64_t>(tokens) * probes + 64 > 0x7FFFFFFF ||
      static_cast<int64_t>(tokens) * heads * keys_len + a.Kp > 0x7FFFFFFF)
    return NOISE_ERR_SHAPE;
  a.items = static_cast<int>(items);
  a.tiles = (a.items + a.G - 1) / a.G;
  a.status = static_cast<int*>(workspace);
  RtMaps maps;
  int rc;
  const uint64_t kv_rows = static_cast<uint64_t>(tokens) * heads * keys_len;
  if ((rc = rt_map(&maps.q, dq, static_cast<uint64_t>(tokens) * probes, heads, 64)) ||
      (rc = rt_map(&maps.kv, keys, kv_rows, 0, static_cast<uint32_t>(a.Kp))) ||
      (rc = rt_map(&maps.v, values, kv_rows, 0, static_cast<uint32_t>(a.Kp))))
    return rc;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
    return NOISE_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(a.status, 0, sizeof(int), s) != cudaSuccess) return NOISE_ERR_CUDA;
  const auto kernel = a.Kp <= 128 ? routed_tc_kernel<1> : routed_tc_kernel<2>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, RT_SMEM)) return NOISE_ERR_CUDA;
  kernel<<<std::min(a.tiles, sms), RT_THREADS, RT_SMEM, s>>>(maps, a);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

size_t noise_future_scores_workspace_bytes(int heads, int tokens) {
  return heads < 1 || tokens < 1 ? 0 : 256 + 4 * ct_plane_bytes(heads, tokens);
}

size_t noise_key_response_workspace_bytes(int heads, int tokens) {
  return heads < 1 || tokens < 1 ? 0 : 256 + 2 * ct_plane_bytes(heads, tokens);
}

int noise_future_scores_ws(const noise_view3_t* q, const noise_view3_t* target, const float* dk, const float* dv,
                           const noise_view3_t* a, const noise_view3_t* contrast, int heads, int tokens, int probes,
                           int sources, int source_start, int window, float* out, void* workspace,
                           size_t workspace_bytes, void* stream) {
  if (!q || !target || !dk || !dv || !a || !contrast || !out || !q->data || !target->data || !a->data ||
      !contrast->data)
    return NOISE_ERR_ARGUMENT;
  if (heads < 1 || tokens < 1 || probes < 1 || sources < 1 || window < 0) return NOISE_ERR_SHAPE;
  // receivers 0 < s - (start + m) <= window: s in [start + m + 1, start + m + window]
  return column_ws<true>(q, target, dk, dv, a, contrast, heads, tokens, probes, sources, source_start + 1, window - 1,
                         out, workspace, workspace_bytes, stream);
}

int noise_key_response_ws(const noise_view3_t* q, const float* dk, const noise_view3_t* a, const noise_view3_t* c,
                          int heads, int tokens, int probes, int sources, int source_start, int query_start,
                          int window, float* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!q || !dk || !a || !c || !out || !q->data || !a->data || !c->data) return NOISE_ERR_ARGUMENT;
  if (heads < 1 || tokens < 1 || probes < 1 || sources < 1 || window < 0) return NOISE_ERR_SHAPE;
  // query index s with query_start + s in [source_start + m, source_start + m + window]
  return column_ws<false>(q, q, dk, dk, a, c, heads, tokens, probes, sources, source_start - query_start, window, out,
                          workspace, workspace_bytes, stream);
}

size_t noise_query_response_workspace_bytes(int tokens, int probes, int heads, int keys_len) {
  if (tokens < 1 || probes < 1 || heads < 1 || keys_len < 1) return 0;
  if (keys_len > QT_MAX_TILES * QT_KEYS) return 256;  // the CUDA-core kernel: the status word only
  return QtWorkspace(tokens, heads, keys_len).bytes();
}

int noise_query_response_ws(const float* dq, const noise_view3_t* keys, const noise_view3_t* values,
                            const noise_view3_t* probabilities, const noise_view3_t* base, int tokens, int probes,
                            int heads, int keys_len, float* out, void* workspace, size_t workspace_bytes,
                            void* stream) {
  if (!dq || !keys || !values || !probabilities || !base || !out || !keys->data || !values->data ||
      !probabilities->data || !base->data)
    return NOISE_ERR_ARGUMENT;
  if (tokens < 1 || probes < 1 || heads < 1 || keys_len < 1) return NOISE_ERR_SHAPE;
  const QtWorkspace w(tokens, heads, keys_len);
  if (!workspace || workspace_bytes < noise_query_response_workspace_bytes(tokens, probes, heads, keys_len))
    return NOISE_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) || !a16(dq) || !a16(out)) return NOISE_ERR_ALIGN;
  if (keys_len > QT_MAX_TILES * QT_KEYS) {  // longer than the live-tile list holds: the CUDA-core kernel
    if (cudaMemsetAsync(workspace, 0, sizeof(int), static_cast<cudaStream_t>(stream)) != cudaSuccess)
      return NOISE_ERR_CUDA;  // its status word reads 0: that kernel has no waits to give up
    return noise_query_response(dq, keys, values, probabilities, base, tokens, probes, heads, keys_len, out, stream);
  }
  const int64_t rows = static_cast<int64_t>(tokens) * probes;
  const int64_t items = (rows + QT_ROWS - 1) / QT_ROWS * heads;
  if (items > 0x7FFFFFFF || heads * w.tp > 0x7FFFFFFF) return NOISE_ERR_SHAPE;  // int32 TMA rows h Tp + k
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* status = static_cast<int*>(workspace);
  float* khi = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + 256);
  float* klo = khi + w.plane / 4;
  float* vhi = klo + w.plane / 4;
  float* vlo = vhi + w.plane / 4;
  uint8_t* live = reinterpret_cast<uint8_t*>(vlo + w.plane / 4);
  QtMaps maps;
  int rc;
  const uint64_t krows = static_cast<uint64_t>(heads) * w.tp, vrows = static_cast<uint64_t>(heads) * D;
  if ((rc = qt_map(&maps.khi, khi, D, krows)) || (rc = qt_map(&maps.klo, klo, D, krows)) ||
      (rc = qt_map(&maps.vhi, vhi, w.tp, vrows)) || (rc = qt_map(&maps.vlo, vlo, w.tp, vrows)))
    return rc;
  if (cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess) return NOISE_ERR_CUDA;
  qr_split_kernel<<<dim3(static_cast<unsigned>(w.nt), heads), 256, 0, s>>>(view(*keys), view(*values), keys_len,
                                                                           static_cast<int>(w.tp), khi, klo, vhi, vlo);
  const int64_t warps = static_cast<int64_t>(heads) * tokens * w.nt;
  qr_live_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, s>>>(
      view(*probabilities), heads, tokens, keys_len, static_cast<int>(w.nt), live);
  if (cudaFuncSetAttribute(query_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, QT_SMEM))
    return NOISE_ERR_CUDA;
  const noise_view3_t& pv = *probabilities;
  const int vec = pv.stride2 == 1 && pv.stride1 % 4 == 0 && pv.stride0 % 4 == 0 && a16(pv.data);
  QtArgs a{dq, view(pv), view(*base), live, out, tokens, probes, heads, keys_len, static_cast<int>(w.nt),
           static_cast<int>(w.tp), vec, status};
  query_tc_kernel<<<static_cast<unsigned>(items), QT_THREADS, QT_SMEM, s>>>(maps, a);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_routed_response(const void* dq, const void* keys, const void* values, const float* probabilities,
                          const float* rest, int tokens, int probes, int heads, int keys_len, float* out,
                          void* stream) {
  if (!dq || !keys || !values || !probabilities || !rest || !out) return NOISE_ERR_ARGUMENT;
  if (tokens < 1 || probes < 1 || heads < 1 || keys_len < 1 || keys_len > RK) return NOISE_ERR_SHAPE;
  if (cudaFuncSetAttribute(routed_response_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, routed_smem(RK)))
    return NOISE_ERR_CUDA;
  dim3 grid((probes + RP - 1) / RP, tokens * heads);
  routed_response_kernel<<<grid, 256, routed_smem(keys_len), static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(dq), static_cast<const __nv_bfloat16*>(keys),
      static_cast<const __nv_bfloat16*>(values), probabilities, rest, probes, heads, keys_len, out);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

}  // extern "C"
