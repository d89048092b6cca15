// The true-path readout's scorer (reference train/val/run.py, `readout` section :5900-6040) on sm_100a: the per-row
// statistics pass (stats_kernel), and the score of every moved row of a token against block j's future moment tables
// (staged_kernel, from the bf16 projection of the raw moves; readout_kernel, from the projected change itself).
//
// For each row (a move of token t) and head h: the change of the token's rotated, RMS-normed key dk and value dv,
//   dk = dr m - r0 (g (i m)^2 / (i + m)),  i = rsqrt(|r0|^2 / 64 + eps), m = rsqrt(|r0|^2 / 64 + g + eps),
//   g = (2 r0 . dr + |dr|^2) / 64,
// is scored against the tables of (t, h): dk . U / 8 + dv . W + bf16(dk) M1 dk / 64 + bf16(dk) M2 dv / 8, plus (DIAG)
// the exact receiver s = t, and (SELF) the token's own output change written as bf16.
// Layout: one warp per row; lane l owns the features l and l + 32 (a rotary pair: each is the other's RoPE partner).
// A block is 64 rows of one token; per head the token's M1, M2 (bf16 64 x 64) are staged in shared memory once for
// all of them. The *_ws entry points run the M1 / M2 terms on tcgen05 instead (staged_tc.cuh).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <mutex>

#include "noise_b200.h"
#include "ptx.cuh"

namespace noise {
namespace scorer {

constexpr int H = NOISE_N_HEAD, D = NOISE_HEAD_DIM, W = NOISE_N_EMBD;
constexpr float NEPS = 1.1920928955078125e-07f;  // the kernels' RMS eps (finfo(float32).eps)
constexpr int ROWS = 64;                         // rows per block (8 warps x 8 rows)

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float bf(const __nv_bfloat16* p, int64_t i) { return __bfloat162float(p[i]); }
__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// stats: per row p < n of token t (delta rows d_rows apart): DB = bf16(d), ST = (inv', inv' / inv0 - 1) of the input
// RMSNorm at x + d, x = X[start + t], sqx = |x|^2.
__global__ void __launch_bounds__(256) stats_kernel(const float* __restrict__ delta, const float* __restrict__ X,
                                                    const float* __restrict__ sqx, __nv_bfloat16* __restrict__ db,
                                                    float* __restrict__ st, int start, int n, int d_rows, float eps) {
  const int lane = threadIdx.x & 31;
  const int p = blockIdx.x * 8 + (threadIdx.x >> 5), t = blockIdx.y;
  if (p >= n) return;
  const int tok = start + t;
  const float* d = delta + (static_cast<int64_t>(t) * d_rows + p) * W;
  const float* x = X + static_cast<int64_t>(tok) * W;
  __nv_bfloat16* o = db + (static_cast<int64_t>(t) * n + p) * W;
  float dotx = 0.f, sqd = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = 4 * lane + 128 * i;
    const float4 dv = *reinterpret_cast<const float4*>(d + c);
    const float4 xv = *reinterpret_cast<const float4*>(x + c);
    dotx += dv.x * xv.x + dv.y * xv.y + dv.z * xv.z + dv.w * xv.w;
    sqd += dv.x * dv.x + dv.y * dv.y + dv.z * dv.z + dv.w * dv.w;
    __nv_bfloat162 lo = __floats2bfloat162_rn(dv.x, dv.y), hi = __floats2bfloat162_rn(dv.z, dv.w);
    *reinterpret_cast<uint2*>(o + c) = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
  }
  dotx = warp_sum(dotx);
  sqd = warp_sum(sqd);
  if (lane == 0) {
    const float sq = sqx[tok];
    const float inv0 = rsqrtf(sq / W + eps), inv = rsqrtf((sq + 2.f * dotx + sqd) / W + eps);
    float* s = st + (static_cast<int64_t>(t) * n + p) * 2;
    s[0] = inv;
    s[1] = (inv - inv0) / inv0;
  }
}

struct Tables {
  const float *U, *WV;                   // [T, H, 64]
  const __nv_bfloat16 *M1, *M2;          // [T, H, 64, 64]
  const float *QD, *GD, *AD, *CD, *VT, *OT;  // [T, H, 64], [T, H, 64], [T, H], [T, H], [T, H, 64], [T, H, 64]
};

struct StagedArgs {
  const __nv_bfloat16* up;  // [m * n, NC]: d W_k^T | d W_v^T | d[:32] W_g^T (padded to 16)
  const float* st;          // [m * n, 2]
  const float *r0, *vc;     // [T, H, 64] rotated clean raw key, [T, 512] raw value (global token rows)
  const float *gz, *ve;     // [T, H] gate logits, [T, H, 64] value embedding (GATED)
  const float *cs, *sn;     // [T, 32]
  Tables tab;
  float* out;               // [m, n]
  __nv_bfloat16* se;        // [m, se_rows, 512] (SELF)
  int start, n, se_rows, nc, diag;
};

struct DirectArgs {
  const float* pj;          // [m, P, 2, H, 64] projected key / value change
  const float* r0;          // [m, H, 64] (chunk rows)
  const float *cs, *sn;     // cos / sin rows of the chunk's tokens, strided
  int64_t csm, csf, snm, snf;
  const float *gc, *ve;     // [m, P, H] gate change, [m, H, 64] value embedding (chunk rows; GATED)
  Tables tab;
  float* out;               // [m, P]
  __nv_bfloat16* se;        // [m, P, 512] (SELF)
  int start, P, diag;
};

// A lane's values of the per-(token, head) tables that every row of the token reads: its two features of QD, GD, U,
// W (and, SELF, VT - OT) and the scalars AD, CD.
struct HeadVals {
  float qd0, qd1, gd0, gd1, u0, u1, w0, w1, vo0, vo1, ad, cd;
};

template <bool SELF>
__device__ __forceinline__ HeadVals head_vals(const Tables& tb, int64_t row, int lane) {
  const int64_t v = row * D;
  HeadVals hv;
  hv.qd0 = tb.QD[v + lane], hv.qd1 = tb.QD[v + lane + 32];
  hv.gd0 = tb.GD[v + lane], hv.gd1 = tb.GD[v + lane + 32];
  hv.u0 = tb.U[v + lane], hv.u1 = tb.U[v + lane + 32];
  hv.w0 = tb.WV[v + lane], hv.w1 = tb.WV[v + lane + 32];
  hv.vo0 = SELF ? tb.VT[v + lane] - tb.OT[v + lane] : 0.f;
  hv.vo1 = SELF ? tb.VT[v + lane + 32] - tb.OT[v + lane + 32] : 0.f;
  hv.ad = tb.AD[row], hv.cd = tb.CD[row];
  return hv;
}

// Three (or two) independent butterfly sums at once: the same sums as warp_sum, their shuffle chains interleaved.
__device__ __forceinline__ void warp_sum3(float& a, float& b, float& c) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
    c += __shfl_xor_sync(0xffffffffu, c, o);
  }
}
__device__ __forceinline__ void warp_sum2(float& a, float& b) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
}

// One head of one row: dr, dv (the lane's two features), the clean rotated key r0 (and its square sum over the head,
// the same for every row of the head) -> the change dk of the rotated, RMS-normed key (the lane's features in dk0,
// dk1) and the row's score part without the moment tables: the exact receiver s = t (DIAG), the self-edge (SELF,
// written) and dk . U / 8 + dv . W (every lane holds the sum). Two rounds of reductions: the growth and both dv dots
// together, then both dk dots.
template <bool SELF>
__device__ __forceinline__ float head_change_v(float dr0, float dr1, float dv0, float dv1, float r00, float r01,
                                               float square, const HeadVals& hv, int lane, int diag,
                                               __nv_bfloat16* se_row, float& dk0, float& dk1) {
  float grow = 2.f * (r00 * dr0 + r01 * dr1) + dr0 * dr0 + dr1 * dr1;
  float gdot = dv0 * hv.gd0 + dv1 * hv.gd1, wdot = dv0 * hv.w0 + dv1 * hv.w1;
  warp_sum3(grow, gdot, wdot);
  grow /= D;
  const float inverse = rsqrtf(square / D + NEPS), moved = rsqrtf(square / D + grow + NEPS);
  const float shrink = grow * (inverse * moved) * (inverse * moved) / (inverse + moved);
  dk0 = dr0 * moved - r00 * shrink;
  dk1 = dr1 * moved - r01 * shrink;
  float xq = dk0 * hv.qd0 + dk1 * hv.qd1, udot = dk0 * hv.u0 + dk1 * hv.u1;
  warp_sum2(xq, udot);
  float total = 0.f;
  if (diag || SELF) {  // the receiver s = t, exactly
    const float x = xq * 0.125f;
    const float a = hv.ad, e = expm1f(x);
    const float gain = a * e / (1.f + a * e), vgain = (a + a * e) / (1.f + a * e);
    if (diag) total += gain * hv.cd + vgain * gdot;
    if (SELF) {
      se_row[lane] = __float2bfloat16_rn(gain * hv.vo0 + vgain * dv0);
      se_row[lane + 32] = __float2bfloat16_rn(gain * hv.vo1 + vgain * dv1);
    }
  }
  total += udot * 0.125f + wdot;
  return total;
}

template <bool SELF>
__device__ __forceinline__ float head_change(float dr0, float dr1, float dv0, float dv1, float r00, float r01,
                                             const Tables& tb, int64_t row, int lane, int diag,
                                             __nv_bfloat16* se_row, float& dk0, float& dk1) {
  return head_change_v<SELF>(dr0, dr1, dv0, dv1, r00, r01, warp_sum(r00 * r00 + r01 * r01),
                             head_vals<SELF>(tb, row, lane), lane, diag, se_row, dk0, dk1);
}

// head_change plus the moment tables on the CUDA cores: bf16(dk) M1 dk / 64 + bf16(dk) M2 dv / 8, the lane forming
// columns lane, lane + 32 of bf16(dk) M from the tables staged in shared memory
template <bool SELF>
__device__ __forceinline__ float score_head(float dr0, float dr1, float dv0, float dv1, float r00, float r01,
                                            const Tables& tb, int64_t row, int lane, const __nv_bfloat16* sm1,
                                            const __nv_bfloat16* sm2, float* sdk, int diag, __nv_bfloat16* se_row) {
  float dk0, dk1;
  float total = head_change<SELF>(dr0, dr1, dv0, dv1, r00, r01, tb, row, lane, diag, se_row, dk0, dk1);
  sdk[lane] = bf16r(dk0);
  sdk[lane + 32] = bf16r(dk1);
  __syncwarp();
  float c10 = 0.f, c11 = 0.f, c20 = 0.f, c21 = 0.f;
#pragma unroll 8
  for (int i = 0; i < D; ++i) {
    const float k = sdk[i];
    c10 = fmaf(k, __bfloat162float(sm1[i * D + lane]), c10);
    c11 = fmaf(k, __bfloat162float(sm1[i * D + lane + 32]), c11);
    c20 = fmaf(k, __bfloat162float(sm2[i * D + lane]), c20);
    c21 = fmaf(k, __bfloat162float(sm2[i * D + lane + 32]), c21);
  }
  __syncwarp();
  total += warp_sum((c10 * dk0 + c11 * dk1) * (1.f / D) + (c20 * dv0 + c21 * dv1) * 0.125f);
  return total;
}

__device__ __forceinline__ void stage_tables(const Tables& tb, int64_t row, __nv_bfloat16* sm1, __nv_bfloat16* sm2) {
  const uint4* g1 = reinterpret_cast<const uint4*>(tb.M1 + row * D * D);
  const uint4* g2 = reinterpret_cast<const uint4*>(tb.M2 + row * D * D);
  for (int i = threadIdx.x; i < D * D / 8; i += 256) {
    reinterpret_cast<uint4*>(sm1)[i] = g1[i];
    reinterpret_cast<uint4*>(sm2)[i] = g2[i];
  }
}

template <bool GATED, bool SELF>
__global__ void __launch_bounds__(256) staged_kernel(const __grid_constant__ StagedArgs a) {
  __shared__ __align__(16) __nv_bfloat16 sm1[D * D], sm2[D * D];
  __shared__ float sdk[8][D];
  __shared__ float sgc[ROWS][H];
  __shared__ float sinv[ROWS], scoef[ROWS], stot[ROWS];  // per row (a warp touches only its own rows)
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int t = blockIdx.y, p0 = blockIdx.x * ROWS;
  const int tok = a.start + t;
  for (int k = 0; k < 8; ++k) {
    const int rl = wib + 8 * k, p = p0 + rl;
    const bool live = p < a.n;
    const float iv = live ? a.st[(static_cast<int64_t>(t) * a.n + p) * 2] : 1.f;
    const float cf = live ? a.st[(static_cast<int64_t>(t) * a.n + p) * 2 + 1] : 0.f;
    if (lane == 0) {
      sinv[rl] = iv;
      scoef[rl] = cf;
      stot[rl] = 0.f;
    }
    if constexpr (GATED) {  // gate change per head: 2 (sigmoid(gz + inv ug + coef gz) - sigmoid(gz))
      if (lane < H) {
        const float gz = a.gz[static_cast<int64_t>(tok) * H + lane];
        const float ug = live ? bf(a.up, (static_cast<int64_t>(t) * a.n + p) * a.nc + 2 * W + lane) : 0.f;
        const float z = gz + iv * ug + cf * gz;
        sgc[rl][lane] = 2.f * (1.f / (1.f + __expf(-z)) - 1.f / (1.f + __expf(-gz)));
      }
    }
  }
  const float c = a.cs[static_cast<int64_t>(tok) * (D / 2) + lane], s = a.sn[static_cast<int64_t>(tok) * (D / 2) + lane];
  for (int h = 0; h < H; ++h) {
    const int64_t row = static_cast<int64_t>(tok) * H + h;
    __syncthreads();
    stage_tables(a.tab, row, sm1, sm2);
    __syncthreads();
    const float r00 = a.r0[row * D + lane], r01 = a.r0[row * D + lane + 32];
    const float vc0 = a.vc[static_cast<int64_t>(tok) * W + h * D + lane];
    const float vc1 = a.vc[static_cast<int64_t>(tok) * W + h * D + lane + 32];
    float ve0 = 0.f, ve1 = 0.f;
    if constexpr (GATED) {
      ve0 = a.ve[row * D + lane];
      ve1 = a.ve[row * D + lane + 32];
    }
#pragma unroll 1
    for (int k = 0; k < 8; ++k) {
      const int rl = wib + 8 * k, p = p0 + rl;
      if (p >= a.n) break;
      const float iv = sinv[rl], cf = scoef[rl];
      const int64_t ur = (static_cast<int64_t>(t) * a.n + p) * a.nc;
      const float uk0 = bf(a.up, ur + h * D + lane), uk1 = bf(a.up, ur + h * D + lane + 32);
      const float uv0 = bf(a.up, ur + W + h * D + lane), uv1 = bf(a.up, ur + W + h * D + lane + 32);
      const float dr0 = iv * (uk0 * c + uk1 * s) + cf * r00;
      const float dr1 = iv * (uk1 * c - uk0 * s) + cf * r01;
      float dv0 = iv * uv0 + cf * vc0, dv1 = iv * uv1 + cf * vc1;
      if constexpr (GATED) {
        const float gc = sgc[rl][h];
        dv0 += gc * ve0;
        dv1 += gc * ve1;
      }
      __nv_bfloat16* se_row =
          SELF ? a.se + (static_cast<int64_t>(t) * a.se_rows + p) * W + h * D : nullptr;
      const float part = score_head<SELF>(dr0, dr1, dv0, dv1, r00, r01, a.tab, row, lane, sm1, sm2, sdk[wib], a.diag,
                                          se_row);
      if (lane == 0) stot[rl] += part;
    }
  }
  for (int k = 0; k < 8; ++k) {
    const int rl = wib + 8 * k, p = p0 + rl;
    if (p < a.n && lane == 0) a.out[static_cast<int64_t>(t) * a.n + p] = stot[rl];
  }
}

template <bool GATED, bool SELF>
__global__ void __launch_bounds__(256) direct_kernel(const __grid_constant__ DirectArgs a) {
  __shared__ __align__(16) __nv_bfloat16 sm1[D * D], sm2[D * D];
  __shared__ float sdk[8][D];
  __shared__ float stot[ROWS];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int t = blockIdx.y, p0 = blockIdx.x * ROWS;
  const int tok = a.start + t;
  if (lane == 0)
    for (int k = 0; k < 8; ++k) stot[wib + 8 * k] = 0.f;
  const float c = a.cs[t * a.csm + lane * a.csf], s = a.sn[t * a.snm + lane * a.snf];
  for (int h = 0; h < H; ++h) {
    const int64_t row = static_cast<int64_t>(tok) * H + h;
    __syncthreads();
    stage_tables(a.tab, row, sm1, sm2);
    __syncthreads();
    const int64_t lr = (static_cast<int64_t>(t) * H + h) * D;  // chunk rows of r0 / ve
    const float r00 = a.r0[lr + lane], r01 = a.r0[lr + lane + 32];
#pragma unroll 1
    for (int k = 0; k < 8; ++k) {
      const int p = p0 + wib + 8 * k;
      if (p >= a.P) break;
      const int64_t base = ((static_cast<int64_t>(t) * a.P + p) * 2 * H + h) * D;
      const float pk0 = a.pj[base + lane], pk1 = a.pj[base + lane + 32];
      const float dr0 = pk0 * c + pk1 * s, dr1 = -pk0 * s + pk1 * c;
      float dv0 = a.pj[base + H * D + lane], dv1 = a.pj[base + H * D + lane + 32];
      if constexpr (GATED) {
        const float gc = a.gc[(static_cast<int64_t>(t) * a.P + p) * H + h];
        dv0 += gc * a.ve[lr + lane];
        dv1 += gc * a.ve[lr + lane + 32];
      }
      __nv_bfloat16* se_row = SELF ? a.se + (static_cast<int64_t>(t) * a.P + p) * W + h * D : nullptr;
      const float part = score_head<SELF>(dr0, dr1, dv0, dv1, r00, r01, a.tab, row, lane, sm1, sm2, sdk[wib], a.diag,
                                          se_row);
      if (lane == 0) stot[wib + 8 * k] += part;
    }
  }
  for (int k = 0; k < 8; ++k) {
    const int p = p0 + wib + 8 * k;
    if (p < a.P && lane == 0) a.out[static_cast<int64_t>(t) * a.P + p] = stot[wib + 8 * k];
  }
}

static Tables tables(const noise_scorer_tables_t& t) {
  return Tables{t.U, t.W, static_cast<const __nv_bfloat16*>(t.M1), static_cast<const __nv_bfloat16*>(t.M2), t.QD,
                t.GD, t.AD, t.CD, t.VT, t.OT};
}

static bool tables_ok(const noise_scorer_tables_t& t, bool self) {
  if (!t.U || !t.W || !t.M1 || !t.M2 || !t.QD || !t.GD || !t.AD || !t.CD) return false;
  if (self && (!t.VT || !t.OT)) return false;
  return (reinterpret_cast<uintptr_t>(t.M1) & 15) == 0 && (reinterpret_cast<uintptr_t>(t.M2) & 15) == 0;
}

}  // namespace scorer
}  // namespace noise

#include "staged_tc.cuh"

using namespace noise::scorer;

namespace {

PFN_cuTensorMapEncodeTiled_v12000 stc_encode() {
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

// bf16 moment tables [rows, 64] (rows = tokens x 8 heads x 64), 64 x 64 boxes, 128-byte swizzle
int stc_map(CUtensorMap* map, const void* base, uint64_t rows) {
  auto fn = stc_encode();
  if (!fn) return NOISE_ERR_CUDA;
  if (reinterpret_cast<uintptr_t>(base) & 15) return NOISE_ERR_ALIGN;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(D), rows};
  cuuint64_t strides[1] = {D * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(D), static_cast<cuuint32_t>(D)};
  cuuint32_t el[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, el,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NOISE_OK : NOISE_ERR_CUDA;
}

}  // namespace

extern "C" {

int noise_readout_stats(const float* delta, const float* x, const float* sqx, void* db, float* st, int start, int n,
                        int d_rows, int tokens, float eps, void* stream) {
  if (!delta || !x || !sqx || !db || !st) return NOISE_ERR_ARGUMENT;
  if (n < 0 || tokens < 0 || d_rows < n || start < 0) return NOISE_ERR_SHAPE;
  if (n == 0 || tokens == 0) return NOISE_OK;
  if ((reinterpret_cast<uintptr_t>(delta) | reinterpret_cast<uintptr_t>(x)) & 15 ||
      reinterpret_cast<uintptr_t>(db) & 7)
    return NOISE_ERR_ALIGN;
  stats_kernel<<<dim3((n + 7) / 8, tokens), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      delta, x, sqx, static_cast<__nv_bfloat16*>(db), st, start, n, d_rows, eps);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_readout_staged(const void* up, const float* st, const float* r0, const float* vc, const float* gz,
                         const float* ve, const float* cs, const float* sn, const noise_scorer_tables_t* tab,
                         float* out, void* se, int start, int n, int se_rows, int tokens, int nc, int diag,
                         void* stream) {
  if (!up || !st || !r0 || !vc || !cs || !sn || !tab || !out) return NOISE_ERR_ARGUMENT;
  const bool gated = gz != nullptr, self = se != nullptr;
  if ((gated && !ve) || !tables_ok(*tab, self)) return NOISE_ERR_ARGUMENT;
  if (n < 0 || tokens < 0 || start < 0 || nc < 2 * W + (gated ? 16 : 0) || (self && se_rows < n))
    return NOISE_ERR_SHAPE;
  if (n == 0 || tokens == 0) return NOISE_OK;
  StagedArgs a{static_cast<const __nv_bfloat16*>(up), st, r0, vc, gz, ve, cs, sn, tables(*tab), out,
               static_cast<__nv_bfloat16*>(se), start, n, se_rows, nc, diag};
  dim3 grid((n + ROWS - 1) / ROWS, tokens);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (gated && self) staged_kernel<true, true><<<grid, 256, 0, s>>>(a);
  else if (gated) staged_kernel<true, false><<<grid, 256, 0, s>>>(a);
  else if (self) staged_kernel<false, true><<<grid, 256, 0, s>>>(a);
  else staged_kernel<false, false><<<grid, 256, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_readout_staged_ws(const void* up, const float* st, const float* r0, const float* vc, const float* gz,
                            const float* ve, const float* cs, const float* sn, const noise_scorer_tables_t* tab,
                            float* out, void* se, int start, int n, int se_rows, int tokens, int nc, int diag,
                            void* workspace, size_t workspace_bytes, void* stream) {
  if (!up || !st || !r0 || !vc || !cs || !sn || !tab || !out) return NOISE_ERR_ARGUMENT;
  const bool gated = gz != nullptr, self = se != nullptr;
  if ((gated && !ve) || !tables_ok(*tab, self)) return NOISE_ERR_ARGUMENT;
  if (n < 0 || tokens < 0 || start < 0 || nc < 2 * W + (gated ? 16 : 0) || (self && se_rows < n))
    return NOISE_ERR_SHAPE;
  if (!workspace || workspace_bytes < NOISE_STATUS_BYTES) return NOISE_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return NOISE_ERR_ALIGN;
  if (n == 0 || tokens == 0) return NOISE_OK;
  StagedArgs a{static_cast<const __nv_bfloat16*>(up), st, r0, vc, gz, ve, cs, sn, tables(*tab), out,
               static_cast<__nv_bfloat16*>(se), start, n, se_rows, nc, diag};
  // the kernel's TMA row coordinate tok H D is int32
  if ((static_cast<int64_t>(start) + tokens) * H * D > 0x7FFFFFFF) return NOISE_ERR_SHAPE;
  StcMaps maps;
  const uint64_t rows = (static_cast<uint64_t>(start) + tokens) * H * D;
  int rc;
  if ((rc = stc_map(&maps.m1, tab->M1, rows)) || (rc = stc_map(&maps.m2, tab->M2, rows))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* status = static_cast<int*>(workspace);
  if (cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess) return NOISE_ERR_CUDA;
  auto kernel = gated ? (self ? staged_tc_kernel<true, true, StagedArgs> : staged_tc_kernel<true, false, StagedArgs>)
                      : (self ? staged_tc_kernel<false, true, StagedArgs> : staged_tc_kernel<false, false, StagedArgs>);
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, STC_SMEM)) return NOISE_ERR_CUDA;
  kernel<<<dim3((n + STC_ROWS - 1) / STC_ROWS, tokens), STC_THREADS, STC_SMEM, s>>>(maps, a, status);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_readout_direct_ws(const float* pj, const float* r0, const float* cs, int64_t cs_token_stride,
                            int64_t cs_pair_stride, const float* sn, int64_t sn_token_stride, int64_t sn_pair_stride,
                            const float* gc, const float* ve, const noise_scorer_tables_t* tab, float* out, void* se,
                            int start, int probes, int tokens, int diag, void* workspace, size_t workspace_bytes,
                            void* stream) {
  if (!pj || !r0 || !cs || !sn || !tab || !out) return NOISE_ERR_ARGUMENT;
  const bool gated = gc != nullptr, self = se != nullptr;
  if ((gated && !ve) || !tables_ok(*tab, self)) return NOISE_ERR_ARGUMENT;
  if (probes < 0 || tokens < 0 || start < 0) return NOISE_ERR_SHAPE;
  if (!workspace || workspace_bytes < NOISE_STATUS_BYTES) return NOISE_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return NOISE_ERR_ALIGN;
  if (probes == 0 || tokens == 0) return NOISE_OK;
  DirectArgs a{pj, r0, cs, sn, cs_token_stride, cs_pair_stride, sn_token_stride, sn_pair_stride, gc, ve, tables(*tab),
               out, static_cast<__nv_bfloat16*>(se), start, probes, diag};
  // the kernel's TMA row coordinate tok H D is int32
  if ((static_cast<int64_t>(start) + tokens) * H * D > 0x7FFFFFFF) return NOISE_ERR_SHAPE;
  StcMaps maps;
  const uint64_t rows = (static_cast<uint64_t>(start) + tokens) * H * D;
  int rc;
  if ((rc = stc_map(&maps.m1, tab->M1, rows)) || (rc = stc_map(&maps.m2, tab->M2, rows))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* status = static_cast<int*>(workspace);
  if (cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess) return NOISE_ERR_CUDA;
  auto kernel = gated ? (self ? staged_tc_kernel<true, true, DirectArgs> : staged_tc_kernel<true, false, DirectArgs>)
                      : (self ? staged_tc_kernel<false, true, DirectArgs> : staged_tc_kernel<false, false, DirectArgs>);
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, STC_SMEM)) return NOISE_ERR_CUDA;
  kernel<<<dim3((probes + STC_ROWS - 1) / STC_ROWS, tokens), STC_THREADS, STC_SMEM, s>>>(maps, a, status);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_readout_direct(const float* pj, const float* r0, const float* cs, int64_t cs_token_stride,
                         int64_t cs_pair_stride, const float* sn, int64_t sn_token_stride, int64_t sn_pair_stride,
                         const float* gc, const float* ve, const noise_scorer_tables_t* tab, float* out, void* se,
                         int start, int probes, int tokens, int diag, void* stream) {
  if (!pj || !r0 || !cs || !sn || !tab || !out) return NOISE_ERR_ARGUMENT;
  const bool gated = gc != nullptr, self = se != nullptr;
  if ((gated && !ve) || !tables_ok(*tab, self)) return NOISE_ERR_ARGUMENT;
  if (probes < 0 || tokens < 0 || start < 0) return NOISE_ERR_SHAPE;
  if (probes == 0 || tokens == 0) return NOISE_OK;
  DirectArgs a{pj, r0, cs, sn, cs_token_stride, cs_pair_stride, sn_token_stride, sn_pair_stride, gc, ve, tables(*tab),
               out, static_cast<__nv_bfloat16*>(se), start, probes, diag};
  dim3 grid((probes + ROWS - 1) / ROWS, tokens);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (gated && self) direct_kernel<true, true><<<grid, 256, 0, s>>>(a);
  else if (gated) direct_kernel<true, false><<<grid, 256, 0, s>>>(a);
  else if (self) direct_kernel<false, true><<<grid, 256, 0, s>>>(a);
  else direct_kernel<false, false><<<grid, 256, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

}  // extern "C"
