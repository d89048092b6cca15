// Credit-readout kernels of Noise's speedrun (reference train/speedrun/moment_kernels.py) on sm_100a.
//
// Rows are (layer, head, sequence) slices of one attention map: [rows, T, 64]. Receiver/query s and key t interact
// iff 0 <= s - t <= window. Five kernels:
//   implicit_ctx    per query: lse = logsumexp_t q.k / 8 and center = sum_t p (hub . v)       (moment_kernels.py:80-194)
//   value_pass      per key: sum_s exp(q_s.k_t / 8 - lse_s) src_s, src split into bf16 hi + lo (:612-717)
//   key_moments     per key and raw direction: degree-2 moment response of the receivers' softmax (key scan, :467-607,
//                   with tf32 logits on fp32 operands; and the identity phase's key moments, :370-462, bf16 operands,
//                   full causal, value sums)
//   query_moments   per query and raw direction: numerator / denominator moments of its own softmax (:197-365)
// All run on warp-level tensor cores (mma.sync bf16 m16n8k16, tf32 m16n8k8), 4 warps x 16 rows per CTA, with
// cp.async-staged shared-memory tiles. The moment dots take bf16 operands exactly where the reference rounds to bf16.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <mutex>
#include <type_traits>

#include "noise_b200.h"
#include "ptx.cuh"
#include "warp_mma.cuh"

namespace noise {
namespace credit {

constexpr float LOG2E = 1.4426950408889634f;
constexpr int D = 64;
constexpr int PITCH_F32 = 68;  // padded fp32 row (floats): conflict-free tf32 fragment loads

struct Rows {
  void* data;
  int64_t layer_stride, token_stride;
  int heads;
  const int32_t* map;
  int block_rows;  // > 0: the blocked layout (row blocks of block_rows rows, tokens split over source GPUs)
  int64_t per_gpu, gpu_stride;
  __device__ __forceinline__ int64_t base(int row) const {
    int l = row / heads;
    if (map) l = map[l];
    return static_cast<int64_t>(l) * layer_stride + static_cast<int64_t>(row % heads) * D;
  }
  // element offset of (row, t, 0); T = tokens per row
  __device__ __forceinline__ int64_t at(int row, int t, int T) const {
    if (block_rows > 0) {  // moment_kernels._query_coefficients / _query_store addressing (:200-220)
      const int blk = row / block_rows;
      const int64_t n = static_cast<int64_t>(row - blk * block_rows) * T + t;
      return blk * layer_stride + (n / per_gpu) * gpu_stride + (n % per_gpu) * token_stride;
    }
    return base(row) + static_cast<int64_t>(t) * token_stride;
  }
};

__host__ Rows to_rows(const noise_rows_t& r) {
  return Rows{r.data, r.layer_stride, r.token_stride, r.heads, r.layer_map, r.block_rows, r.per_gpu, r.gpu_stride};
}

// A contiguous [rows, T, 64] tensor as a view.
__host__ Rows stacked_rows(const void* data, int T) {
  return Rows{const_cast<void*>(data), static_cast<int64_t>(T) * D, D, 1, nullptr, 0, 0, 0};
}

// One element of a raw-coordinate view (fp32 or bf16) as fp32.
__device__ __forceinline__ float raw_at(const Rows& r, bool bf16, int64_t i) {
  return bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(r.data)[i]) : static_cast<const float*>(r.data)[i];
}

// ---------------------------------------------------------------------------------------------------------------
// tile staging
// ---------------------------------------------------------------------------------------------------------------
// bf16 [R][64] tile, rows `stride` elements apart, into the swizzled layout swz(row, chunk).
template <int R>
__device__ __forceinline__ void stage_bf16(uint32_t sbase, const __nv_bfloat16* g, int64_t stride, int tid) {
#pragma unroll
  for (int i = tid; i < R * 8; i += 128) {
    const int row = i >> 3, ch = i & 7;
    cp_async16(sbase + swz(row, ch), g + row * stride + ch * 8);
  }
}

// fp32 [R][64] tile, rows `stride` floats apart, into a [R][PITCH_F32] padded tile.
template <int R>
__device__ __forceinline__ void stage_f32(uint32_t sbase, const float* g, int64_t stride, int tid) {
#pragma unroll
  for (int i = tid; i < R * 16; i += 128) {
    const int row = i >> 4, ch = i & 15;
    cp_async16(sbase + static_cast<uint32_t>((row * PITCH_F32 + ch * 4) * 4), g + row * stride + ch * 4);
  }
}

__device__ __forceinline__ void st_bf16(uint8_t* base, uint32_t byte, float v) {
  *reinterpret_cast<__nv_bfloat16*>(base + byte) = __float2bfloat16_rn(v);
}

// A fragment (16 rows from r0, k-step kk of 16) from a swizzled bf16 [*][64] tile.
__device__ __forceinline__ void frag_a(uint32_t s, int r0, int kk, int lane, uint32_t (&a)[4]) {
  ldsm_x4(s + swz(r0 + (lane & 15), 2 * kk + (lane >> 4)), a[0], a[1], a[2], a[3]);
}
// B fragments of two 8-wide n-tiles (n rows np*16 ..) for k-step kk, from a swizzled [n][64 k] tile.
__device__ __forceinline__ void frag_b(uint32_t s, int np, int kk, int lane, uint32_t (&b)[4]) {
  ldsm_x4(s + swz(np * 16 + (lane & 7) + ((lane >> 4) << 3), 2 * kk + ((lane >> 3) & 1)), b[0], b[1], b[2], b[3]);
}
// B fragments (transposed source): k rows kk*16 .., n columns np*16 .. of a swizzled [k][64 n] tile.
__device__ __forceinline__ void frag_bt(uint32_t s, int kk, int np, int lane, uint32_t (&b)[4]) {
  ldsm_x4_t(s + swz(kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), 2 * np + (lane >> 4)), b[0], b[1], b[2], b[3]);
}
// Same for a padded bf16 [k][cols] tile with a row pitch of `pitch` bytes.
__device__ __forceinline__ void frag_bt_pitch(uint32_t s, int pitch, int kk, int np, int lane, uint32_t (&b)[4]) {
  const int row = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
  const int col = np * 16 + (lane >> 4) * 8;
  ldsm_x4_t(s + static_cast<uint32_t>(row * pitch + col * 2), b[0], b[1], b[2], b[3]);
}
// tf32 A fragment (rows r0 + g, r0 + g + 8; k columns 8 kk + q, + 4) from a padded fp32 tile.
__device__ __forceinline__ void frag_a_tf32(const float* t, int r0, int kk, int lane, uint32_t (&a)[4]) {
  const int g = lane >> 2, q = lane & 3;
  const float* p = t + (r0 + g) * PITCH_F32 + 8 * kk + q;
  a[0] = to_tf32(p[0]);
  a[1] = to_tf32(p[8 * PITCH_F32]);
  a[2] = to_tf32(p[4]);
  a[3] = to_tf32(p[8 * PITCH_F32 + 4]);
}
// tf32 B fragment of n-tile nt (n rows 8 nt + g), k-step kk, from a padded fp32 [n][64 k] tile.
__device__ __forceinline__ void frag_b_tf32(const float* t, int nt, int kk, int lane, uint32_t (&b)[2]) {
  const int g = lane >> 2, q = lane & 3;
  const float* p = t + (8 * nt + g) * PITCH_F32 + 8 * kk + q;
  b[0] = to_tf32(p[0]);
  b[1] = to_tf32(p[4]);
}

// 16 x (8 NT) block of q.k-like dot products: rows = this warp's rows of tile A, columns = rows of tile B.
template <bool BF16, int NT>
__device__ __forceinline__ void dot_block(uint32_t sa, uint32_t sb, int r0, int lane, float (&acc)[NT][4]) {
#pragma unroll
  for (int n = 0; n < NT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  if constexpr (BF16) {
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      frag_a(sa, r0, kk, lane, a);
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        uint32_t b[4];
        frag_b(sb, np, kk, lane, b);
        mma_bf16(acc[2 * np], a[0], a[1], a[2], a[3], b[0], b[1]);
        mma_bf16(acc[2 * np + 1], a[0], a[1], a[2], a[3], b[2], b[3]);
      }
    }
  } else {
    const float* ta = reinterpret_cast<const float*>(__cvta_shared_to_generic(sa));
    const float* tb = reinterpret_cast<const float*>(__cvta_shared_to_generic(sb));
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t a[4];
      frag_a_tf32(ta, r0, kk, lane, a);
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        uint32_t b[2];
        frag_b_tf32(tb, n, kk, lane, b);
        mma_tf32(acc[n], a[0], a[1], a[2], a[3], b[0], b[1]);
      }
    }
  }
}

// Pack a 16 x 16 slice (n-tiles 2 j, 2 j + 1) of a C-fragment block into an A fragment (bf16).
template <int NT>
__device__ __forceinline__ void pack_a(const float (&x)[NT][4], int j, uint32_t (&a)[4]) {
  a[0] = pack_bf16x2(x[2 * j][0], x[2 * j][1]);
  a[1] = pack_bf16x2(x[2 * j][2], x[2 * j][3]);
  a[2] = pack_bf16x2(x[2 * j + 1][0], x[2 * j + 1][1]);
  a[3] = pack_bf16x2(x[2 * j + 1][2], x[2 * j + 1][3]);
}

template <bool BF16>
__host__ __device__ constexpr int tile_bytes(int rows) {
  return BF16 ? rows * 128 : rows * PITCH_F32 * 4;
}

template <bool BF16, int R>
__device__ __forceinline__ void stage_tile(uint32_t s, const void* g, int64_t stride, int tid) {
  if constexpr (BF16)
    stage_bf16<R>(s, static_cast<const __nv_bfloat16*>(g), stride, tid);
  else
    stage_f32<R>(s, static_cast<const float*>(g), stride, tid);
}

// ---------------------------------------------------------------------------------------------------------------
// implicit_ctx: lse and center per query (online softmax over the window)
// ---------------------------------------------------------------------------------------------------------------
struct CtxArgs {
  const void *q, *k, *v, *hub;  // [rows, T, 64] contiguous, bf16 or fp32
  float *lse, *center;          // [rows, T]
  int T, window;
};

template <bool BF16>
__global__ void __launch_bounds__(128) implicit_ctx_kernel(CtxArgs p) {
  constexpr int TB = tile_bytes<BF16>(64);
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nq = p.T / 64;
  const int qt = nq - 1 - blockIdx.x, row = blockIdx.y;
  const int q0 = qt * 64;
  const size_t es = BF16 ? 2 : 4;
  const int64_t base = static_cast<int64_t>(row) * p.T * D;
  auto at = [&](const void* t, int64_t off) { return static_cast<const uint8_t*>(t) + (base + off) * es; };
  const uint32_t sQ = smem_u32(smem), sH = sQ + TB;
  const uint32_t sK0 = sQ + 2 * TB;  // stage i: K at sK0 + 2 i TB, V at + TB
  const int lo = q0 - p.window >= 0 ? (q0 - p.window) / 64 : 0;
  const int hi = qt;
  stage_tile<BF16, 64>(sQ, at(p.q, int64_t(q0) * D), D, tid);
  stage_tile<BF16, 64>(sH, at(p.hub, int64_t(q0) * D), D, tid);
  stage_tile<BF16, 64>(sK0, at(p.k, int64_t(lo) * 64 * D), D, tid);
  stage_tile<BF16, 64>(sK0 + TB, at(p.v, int64_t(lo) * 64 * D), D, tid);
  cp_async_commit();
  const int r0 = warp * 16;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f}, ssum[2] = {0.f, 0.f};
  for (int kt = lo; kt <= hi; ++kt) {
    const int buf = (kt - lo) & 1;
    const uint32_t sK = sK0 + buf * 2 * TB, sV = sK + TB;
    if (kt < hi) {
      const uint32_t nK = sK0 + (buf ^ 1) * 2 * TB;
      stage_tile<BF16, 64>(nK, at(p.k, int64_t(kt + 1) * 64 * D), D, tid);
      stage_tile<BF16, 64>(nK + TB, at(p.v, int64_t(kt + 1) * 64 * D), D, tid);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    float s[8][4], sc[8][4];
    dot_block<BF16, 8>(sQ, sK, r0, lane, s);
    dot_block<BF16, 8>(sH, sV, r0, lane, sc);
    const bool mask = kt == hi || (q0 - p.window >= 0 && kt == lo);
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int tq = q0 + r0 + (lane >> 2) + 8 * hr;
      float mx = -INFINITY;
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float x = s[n][2 * hr + e] * 0.125f;
          if (mask) {
            const int sk = kt * 64 + n * 8 + 2 * (lane & 3) + e;
            if (sk > tq || tq - sk > p.window) x = -INFINITY;
          }
          s[n][2 * hr + e] = x;
          mx = fmaxf(mx, x);
        }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(m[hr], mx);
      const float ms = mn == -INFINITY ? 0.f : mn;
      const float scale = ex2_approx((m[hr] - ms) * LOG2E);
      float rs = 0.f, rw = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float pr = ex2_approx((s[n][2 * hr + e] - ms) * LOG2E);
          rs += pr;
          rw += pr * sc[n][2 * hr + e];
        }
      m[hr] = mn;
      l[hr] = l[hr] * scale + rs;
      ssum[hr] = ssum[hr] * scale + rw;
    }
    __syncthreads();
  }
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    float lt = l[hr], st = ssum[hr];
    lt += __shfl_xor_sync(0xffffffffu, lt, 1);
    lt += __shfl_xor_sync(0xffffffffu, lt, 2);
    st += __shfl_xor_sync(0xffffffffu, st, 1);
    st += __shfl_xor_sync(0xffffffffu, st, 2);
    if ((lane & 3) == 0) {
      const int tq = q0 + r0 + (lane >> 2) + 8 * hr;
      p.lse[static_cast<int64_t>(row) * p.T + tq] = m[hr] + logf(lt);
      p.center[static_cast<int64_t>(row) * p.T + tq] = st / lt;
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// value_pass: out_t = sum_{s: 0 <= s - t <= W} exp(q_s.k_t / 8 - lse_s) src_s   (src as bf16 hi + lo)
// ---------------------------------------------------------------------------------------------------------------
struct ValueArgs {
  const void *q, *k;  // [rows, T, 64] contiguous, bf16 or fp32
  const float* lse;   // [rows, T]
  Rows src, out;      // fp32 views
  int T, window;
};

template <bool BF16>
__global__ void __launch_bounds__(128) value_pass_kernel(ValueArgs p) {
  constexpr int TB = tile_bytes<BF16>(64);
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row = blockIdx.y, t0 = blockIdx.x * 64;
  const size_t es = BF16 ? 2 : 4;
  const int64_t base = static_cast<int64_t>(row) * p.T * D;
  auto at = [&](const void* t, int64_t off) { return static_cast<const uint8_t*>(t) + (base + off) * es; };
  const uint32_t sK = smem_u32(smem), sQ0 = sK + TB;  // Q stage i at sQ0 + i TB
  uint8_t* hl = smem + 3 * TB;                           // bf16 hi tile, lo tile
  float* lse_s = reinterpret_cast<float*>(hl + 2 * 64 * 128);
  const uint32_t sHi = smem_u32(hl), sLo = sHi + 64 * 128;
  const float* src_row = static_cast<const float*>(p.src.data) + p.src.base(row);
  const int first = t0 / 64;
  const int last = min((t0 + 63 + p.window) / 64, p.T / 64 - 1);
  stage_tile<BF16, 64>(sK, at(p.k, int64_t(t0) * D), D, tid);
  stage_tile<BF16, 64>(sQ0, at(p.q, int64_t(first) * 64 * D), D, tid);
  cp_async_commit();
  const int r0 = warp * 16;
  float acc[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
  for (int it = first; it <= last; ++it) {
    const int buf = (it - first) & 1;
    const uint32_t sQ = sQ0 + buf * TB;
    // src tile -> bf16 hi / lo (registers -> shared; the previous iteration's readers are past the barrier)
    const int s0 = it * 64;
#pragma unroll
    for (int i = tid; i < 64 * 16; i += 128) {
      const int r = i >> 4, c4 = (i & 15) * 4;
      const float4 v = *reinterpret_cast<const float4*>(src_row + static_cast<int64_t>(s0 + r) * p.src.token_stride + c4);
      const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float h = bf16_round(vv[e]);
        const uint32_t off = swz(r, (c4 + e) >> 3) + ((c4 + e) & 7) * 2;
        st_bf16(hl, off, h);
        st_bf16(hl + 64 * 128, off, vv[e] - h);
      }
    }
    if (tid < 64) lse_s[tid] = p.lse[static_cast<int64_t>(row) * p.T + s0 + tid];
    if (it < last) {
      stage_tile<BF16, 64>(sQ0 + (buf ^ 1) * TB, at(p.q, int64_t(it + 1) * 64 * D), D, tid);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    float s[8][4];
    dot_block<BF16, 8>(sK, sQ, r0, lane, s);  // [key t][receiver s]
    const bool mask = it == first || s0 + 63 - t0 > p.window;
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int tk = t0 + r0 + (lane >> 2) + 8 * (e >> 1);
        const int sr = s0 + n * 8 + 2 * (lane & 3) + (e & 1);
        float pr = ex2_approx((s[n][e] * 0.125f - lse_s[sr - s0]) * LOG2E);
        if (mask && (sr < tk || sr - tk > p.window)) pr = 0.f;
        s[n][e] = pr;
      }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      pack_a(s, kk, a);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b[4];
        frag_bt(sHi, kk, np, lane, b);
        mma_bf16(acc[2 * np], a[0], a[1], a[2], a[3], b[0], b[1]);
        mma_bf16(acc[2 * np + 1], a[0], a[1], a[2], a[3], b[2], b[3]);
        frag_bt(sLo, kk, np, lane, b);
        mma_bf16(acc[2 * np], a[0], a[1], a[2], a[3], b[0], b[1]);
        mma_bf16(acc[2 * np + 1], a[0], a[1], a[2], a[3], b[2], b[3]);
      }
    }
    __syncthreads();
  }
  float* out = static_cast<float*>(p.out.data) + p.out.base(row);
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int tk = t0 + r0 + (lane >> 2) + 8 * hr;
#pragma unroll
    for (int n = 0; n < 8; ++n)
      *reinterpret_cast<float2*>(out + static_cast<int64_t>(tk) * p.out.token_stride + n * 8 + 2 * (lane & 3)) =
          make_float2(acc[n][2 * hr], acc[n][2 * hr + 1]);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// key_moments: key scan (SCAN) and the identity phase's key moments (IDENT)
// ---------------------------------------------------------------------------------------------------------------
// Feature layout of the receivers' pair features (x_i = side[s][i] / 8, y_i = side[s][i + 32] / 8):
//   f2[s][2 i + u] = (x_i, y_i)[u], g2[s][2 i + u] = (x_i^2, y_i^2)[u]  (swizzled [32][64] bf16)
//   xy[s][c] = x_P y_P with P = pxy(c) = 8 (c / 8) + 4 (c % 2) + (c % 8) / 2  (padded [32][40] bf16)
// so that a thread's C-fragment columns of p2 / q2 / r2 (features 2P, 2P + 1 for P = 4 n + q) and of qxy (column
// permuted) refer to the same rotary pairs P = 4 n' + q, n' = 0..7.
__device__ __forceinline__ int pxy(int c) { return 8 * (c >> 3) + 4 * (c & 1) + ((c & 7) >> 1); }

struct KeyArgs {
  const void *qp, *kp, *values, *hub;  // [rows, T, 64]: fp32 (SCAN) or bf16 (IDENT)
  const float* side;                   // IDENT: receivers' fp32 pair-feature source [rows, T, 64]; SCAN uses qp
  Rows raw;                            // raw key coordinates (rows, T, 64) view
  int raw_bf16;                        // raw holds bf16 (else fp32)
  int out_bf16;                        // out / vout hold bf16 (else fp32)
  const float* sq;                     // IDENT: [rows, T]
  const float* steps;                  // IDENT: [rows, T]
  const float *lse, *center;           // [rows, T] (center = hub_out for IDENT)
  const float *cosb, *sinb;            // [T, 32] fp32
  Rows out, vout;                      // output views; vout.data NULL = no value credit
  int T, window;
  float sigma;
};

constexpr int KB = 32;  // receivers per iteration

template <bool IDENT>
struct KeyLayout {
  static constexpr bool BF16 = IDENT;
  static constexpr int TK = tile_bytes<BF16>(64);        // key-side tile (K or V)
  static constexpr int TR = tile_bytes<BF16>(KB);        // receiver-side tile (Q or Hub)
  static constexpr int TS = IDENT ? KB * PITCH_F32 * 4 : 0;  // side tile (IDENT)
  static constexpr int STAGE = 2 * TR + TS + 2 * KB * 4;  // Q, Hub, side, lse, center
  static constexpr int FEAT = 2 * KB * 128 + KB * 80 + (IDENT ? 0 : 2 * KB * 128);  // f2, g2, xy, hub hi/lo
  static constexpr int SMEM = 2 * TK + 2 * STAGE + FEAT;
};

template <bool IDENT>
__global__ void __launch_bounds__(128) key_moments_kernel(KeyArgs p) {
  using L = KeyLayout<IDENT>;
  constexpr bool BF16 = L::BF16;
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q = lane & 3;
  const int row = blockIdx.y, t0 = blockIdx.x * 64;
  const size_t es = BF16 ? 2 : 4;
  const int64_t base = static_cast<int64_t>(row) * p.T * D;
  auto at = [&](const void* t, int64_t off) { return static_cast<const uint8_t*>(t) + (base + off) * es; };
  const uint32_t s0a = smem_u32(smem);
  const uint32_t sK = s0a, sV = s0a + L::TK, sStage = s0a + 2 * L::TK;
  uint8_t* feat = smem + 2 * L::TK + 2 * L::STAGE;
  const uint32_t sF2 = smem_u32(feat), sG2 = sF2 + KB * 128, sXY = sG2 + KB * 128, sHi = sXY + KB * 80,
                 sLo = sHi + KB * 128;
  const bool values = p.vout.data != nullptr;
  const int window = IDENT ? p.T : p.window;
  const int first = t0 / KB;
  const int last = min((t0 + 63 + window) / KB, p.T / KB - 1);

  auto stage = [&](int it, int buf) {
    const uint32_t s = sStage + buf * L::STAGE;
    stage_tile<BF16, KB>(s, at(p.qp, int64_t(it) * KB * D), D, tid);
    stage_tile<BF16, KB>(s + L::TR, at(p.hub, int64_t(it) * KB * D), D, tid);
    if constexpr (IDENT) stage_f32<KB>(s + 2 * L::TR, p.side + base + int64_t(it) * KB * D, D, tid);
  };
  stage_tile<BF16, 64>(sK, at(p.kp, int64_t(t0) * D), D, tid);
  stage_tile<BF16, 64>(sV, at(p.values, int64_t(t0) * D), D, tid);
  stage(first, 0);
  cp_async_commit();

  const int r0 = warp * 16;
  float p2[8][4], q2[8][4], r2[8][4], qxy[4][4], va[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) p2[n][e] = q2[n][e] = r2[n][e] = va[n][e] = 0.f;
#pragma unroll
  for (int n = 0; n < 4; ++n) qxy[n][0] = qxy[n][1] = qxy[n][2] = qxy[n][3] = 0.f;
  float s1[2] = {0.f, 0.f}, s2[2] = {0.f, 0.f};

  for (int it = first; it <= last; ++it) {
    const int buf = (it - first) & 1;
    const uint32_t sQ = sStage + buf * L::STAGE, sH = sQ + L::TR;
    uint8_t* stg = smem + 2 * L::TK + buf * L::STAGE;
    float* lse_s = reinterpret_cast<float*>(stg + 2 * L::TR + L::TS);
    float* ctr_s = lse_s + KB;
    const int s0 = it * KB;
    if (tid < KB) {
      lse_s[tid] = p.lse[static_cast<int64_t>(row) * p.T + s0 + tid];
    } else if (tid < 2 * KB) {
      ctr_s[tid - KB] = p.center[static_cast<int64_t>(row) * p.T + s0 + tid - KB];
    }
    if (it < last) {
      stage(it + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    // receivers' pair features (and hub hi / lo for the scan's value credit)
    {
      const float* side = IDENT ? reinterpret_cast<const float*>(stg + 2 * L::TR)
                                : reinterpret_cast<const float*>(stg);  // SCAN: the fp32 qp tile
      for (int i = tid; i < KB * 32; i += 128) {
        const int r = i >> 5, pr = i & 31;
        const float x = side[r * PITCH_F32 + pr] * 0.125f, y = side[r * PITCH_F32 + pr + 32] * 0.125f;
        const int f = 2 * pr;
        st_bf16(feat, swz(r, f >> 3) + (f & 7) * 2, x);
        st_bf16(feat, swz(r, (f + 1) >> 3) + ((f + 1) & 7) * 2, y);
        st_bf16(feat + KB * 128, swz(r, f >> 3) + (f & 7) * 2, x * x);
        st_bf16(feat + KB * 128, swz(r, (f + 1) >> 3) + ((f + 1) & 7) * 2, y * y);
        const int P = pxy(pr);
        const float xp = side[r * PITCH_F32 + P] * 0.125f, yp = side[r * PITCH_F32 + P + 32] * 0.125f;
        st_bf16(feat + 2 * KB * 128, r * 80 + pr * 2, xp * yp);
      }
      if constexpr (!IDENT) {
        if (values) {
          const float* hub = reinterpret_cast<const float*>(stg + L::TR);
          for (int i = tid; i < KB * 64; i += 128) {
            const int r = i >> 6, c = i & 63;
            const float v = hub[r * PITCH_F32 + c], h = bf16_round(v);
            const uint32_t off = swz(r, c >> 3) + (c & 7) * 2;
            st_bf16(feat + 2 * KB * 128 + KB * 80, off, h);
            st_bf16(feat + 3 * KB * 128 + KB * 80, off, v - h);
          }
        }
      }
    }
    __syncthreads();
    float lg[4][4], sc[4][4];
    dot_block<BF16, 4>(sK, sQ, r0, lane, lg);  // k_t . q_s
    dot_block<BF16, 4>(sV, sH, r0, lane, sc);  // v_t . hub_s
    float w1[4][4], w2[4][4], w2l[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int hr = e >> 1;
        const int tk = t0 + r0 + g + 8 * hr;
        const int cs = n * 8 + 2 * q + (e & 1);
        const int sr = s0 + cs;
        const bool valid = sr >= tk && sr - tk <= window;
        const float logit = lg[n][e] * 0.125f;
        const float a = valid ? ex2_approx((logit - lse_s[cs]) * LOG2E) : 0.f;
        const float c = IDENT ? sc[n][e] - ctr_s[cs] : (valid ? sc[n][e] - ctr_s[cs] : 0.f);
        const float x1 = a * c, x2 = (0.5f * a - a * a) * c;
        w1[n][e] = x1;
        w2[n][e] = x2;
        w2l[n][e] = x2 * logit;
        s1[hr] += x1 * logit;
        s2[hr] += x2 * logit * logit;
        lg[n][e] = a;  // reused: probabilities for the value credit
      }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint32_t a1[4], a2[4], a3[4], ap[4];
      pack_a(w1, j, a1);
      pack_a(w2, j, a2);
      pack_a(w2l, j, a3);
      pack_a(lg, j, ap);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b[4];
        frag_bt(sF2, j, np, lane, b);
        mma_bf16(p2[2 * np], a1[0], a1[1], a1[2], a1[3], b[0], b[1]);
        mma_bf16(p2[2 * np + 1], a1[0], a1[1], a1[2], a1[3], b[2], b[3]);
        mma_bf16(r2[2 * np], a3[0], a3[1], a3[2], a3[3], b[0], b[1]);
        mma_bf16(r2[2 * np + 1], a3[0], a3[1], a3[2], a3[3], b[2], b[3]);
        frag_bt(sG2, j, np, lane, b);
        mma_bf16(q2[2 * np], a2[0], a2[1], a2[2], a2[3], b[0], b[1]);
        mma_bf16(q2[2 * np + 1], a2[0], a2[1], a2[2], a2[3], b[2], b[3]);
        if (values) {
          if constexpr (IDENT) {
            frag_bt(sH, j, np, lane, b);
            mma_bf16(va[2 * np], ap[0], ap[1], ap[2], ap[3], b[0], b[1]);
            mma_bf16(va[2 * np + 1], ap[0], ap[1], ap[2], ap[3], b[2], b[3]);
          } else {
            frag_bt(sHi, j, np, lane, b);
            mma_bf16(va[2 * np], ap[0], ap[1], ap[2], ap[3], b[0], b[1]);
            mma_bf16(va[2 * np + 1], ap[0], ap[1], ap[2], ap[3], b[2], b[3]);
            frag_bt(sLo, j, np, lane, b);
            mma_bf16(va[2 * np], ap[0], ap[1], ap[2], ap[3], b[0], b[1]);
            mma_bf16(va[2 * np + 1], ap[0], ap[1], ap[2], ap[3], b[2], b[3]);
          }
        }
      }
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        uint32_t b[4];
        frag_bt_pitch(sXY, 80, j, np, lane, b);
        mma_bf16(qxy[2 * np], a2[0], a2[1], a2[2], a2[3], b[0], b[1]);
        mma_bf16(qxy[2 * np + 1], a2[0], a2[1], a2[2], a2[3], b[2], b[3]);
      }
    }
    __syncthreads();
  }

  // epilogue: per key row and raw direction d = P, P + 32 (P = 4 n' + q)
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    float a1 = s1[hr], a2 = s2[hr];
    a1 += __shfl_xor_sync(0xffffffffu, a1, 1);
    a1 += __shfl_xor_sync(0xffffffffu, a1, 2);
    a2 += __shfl_xor_sync(0xffffffffu, a2, 1);
    a2 += __shfl_xor_sync(0xffffffffu, a2, 2);
    const int tk = t0 + r0 + g + 8 * hr;
    const int64_t ro = p.raw.at(row, tk, p.T);
    const bool rb = p.raw_bf16;
    float sqv, stepv, den;
    if constexpr (IDENT) {
      sqv = p.sq[static_cast<int64_t>(row) * p.T + tk];
      stepv = p.steps[static_cast<int64_t>(row) * p.T + tk];
      den = sqv / D + 1e-6f;
    } else {
      float part = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const int P = 4 * n + q;
        const float r0 = raw_at(p.raw, rb, ro + P), r1 = raw_at(p.raw, rb, ro + P + 32);
        part += r0 * r0 + r1 * r1;
      }
      part += __shfl_xor_sync(0xffffffffu, part, 1);
      part += __shfl_xor_sync(0xffffffffu, part, 2);
      sqv = part / D;
      stepv = p.sigma * fmaxf(sqrtf(sqv), 1e-6f);
      den = sqv + 1.1920928955078125e-07f;
    }
    const float rs = rsqrtf(den);
    const int64_t oo = p.out.at(row, tk, p.T);
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int P = 4 * n + q;
      const float px = p2[n][2 * hr], py = p2[n][2 * hr + 1];
      const float qx = q2[n][2 * hr], qy = q2[n][2 * hr + 1];
      const float rx = r2[n][2 * hr], ry = r2[n][2 * hr + 1];
      const float cxy = qxy[n >> 1][(n & 1) + 2 * hr];
      const float cs = p.cosb[static_cast<int64_t>(tk) * 32 + P], sn = p.sinb[static_cast<int64_t>(tk) * 32 + P];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int d = P + 32 * half;
        const float ratio = (2.f * stepv * raw_at(p.raw, rb, ro + d) + stepv * stepv) / D / den;
        const float ca = expm1f(-0.5f * log1pf(ratio));
        const float cb = stepv * rs * (1.f + ca);
        const float bu = cb * (half ? sn : cs), bw = cb * (half ? cs : -sn);
        const float resp = px * bu + py * bw + qx * bu * bu + qy * bw * bw + 2.f * cxy * bu * bw +
                           2.f * ca * (rx * bu + ry * bw) + a1 * ca + a2 * ca * ca;
        if (p.out_bf16)
          static_cast<__nv_bfloat16*>(p.out.data)[oo + d] = __float2bfloat16_rn(resp / stepv);
        else
          static_cast<float*>(p.out.data)[oo + d] = resp / stepv;
      }
    }
    if (values) {
      const int64_t vo = p.vout.at(row, tk, p.T);
      if (p.out_bf16) {
        __nv_bfloat16* vb = static_cast<__nv_bfloat16*>(p.vout.data) + vo;
#pragma unroll
        for (int n = 0; n < 8; ++n)
          *reinterpret_cast<__nv_bfloat162*>(vb + n * 8 + 2 * q) = __floats2bfloat162_rn(va[n][2 * hr], va[n][2 * hr + 1]);
      } else {
        float* vf = static_cast<float*>(p.vout.data) + vo;
#pragma unroll
        for (int n = 0; n < 8; ++n)
          *reinterpret_cast<float2*>(vf + n * 8 + 2 * q) = make_float2(va[n][2 * hr], va[n][2 * hr + 1]);
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// query_moments: per query s and raw query coordinate, zn / (1 + zd) / step
// ---------------------------------------------------------------------------------------------------------------
// Each CTA handles 64 queries and one half ("part") of the 32 rotary pairs. Feature blocks over the part's 16 pairs,
// [32 keys][16] bf16 (pitch 48 B), columns permuted: column c holds pair pq(c) = 8 (c / 8) + 4 (c % 2) + (c % 8) / 2,
// so a thread's C-fragment columns (n, e) all refer to pair 8 n + 4 e + q of the part.
__device__ __forceinline__ int pq16(int c) { return 8 * (c >> 3) + 4 * (c & 1) + ((c & 7) >> 1); }

struct QueryArgs {
  const __nv_bfloat16 *q, *k, *v, *hub;  // [rows, T, 64]
  Rows raw;                              // raw query coordinates (rows, T, 64) view
  int raw_bf16;
  const float *sq, *steps, *lse, *hub_out;  // [rows, T]
  const float* side;                     // keys' pair-feature source [rows, T, 64] fp32
  const float *cosb, *sinb;              // [T, 32]
  Rows out;
  int out_bf16;
  int T, window;
};

constexpr int QB = 32;                  // keys per iteration
constexpr int QF = QB * 48;             // one feature block
constexpr int Q_STAGE = 2 * QB * 128 + QB * 36 * 4 + 2 * QB * 0;  // K, V, side (part's 32 columns, pitch 36)
constexpr int Q_SMEM = 2 * 64 * 128 + 2 * Q_STAGE + 5 * QF;

__global__ void __launch_bounds__(128) query_moments_kernel(QueryArgs p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q = lane & 3;
  const int nq = p.T / 64;
  const int qt = nq - 1 - blockIdx.x;
  const int row = blockIdx.y >> 1, part = blockIdx.y & 1;
  const int q0 = qt * 64;
  const int64_t base = static_cast<int64_t>(row) * p.T * D;
  const uint32_t sQ = smem_u32(smem), sH = sQ + 64 * 128, sSt = sH + 64 * 128;
  uint8_t* feat = smem + 2 * 64 * 128 + 2 * Q_STAGE;
  const uint32_t sF = smem_u32(feat);  // blocks: x, y, xx, yy, xy
  const int first = q0 - p.window >= 0 ? (q0 - p.window) / QB : 0;
  const int last = (q0 + 63) / QB;

  auto stage = [&](int it, int buf) {
    const uint32_t s = sSt + buf * Q_STAGE;
    stage_bf16<QB>(s, p.k + base + int64_t(it) * QB * D, D, tid);
    stage_bf16<QB>(s + QB * 128, p.v + base + int64_t(it) * QB * D, D, tid);
    // the part's 16 x columns and 16 y columns of side: 4 + 4 chunks of 16 bytes per key
    for (int i = tid; i < QB * 8; i += 128) {
      const int r = i >> 3, ch = i & 7;
      const int col = (ch < 4 ? part * 16 : 32 + part * 16) + (ch & 3) * 4;
      cp_async16(s + 2 * QB * 128 + static_cast<uint32_t>((r * 36 + ch * 4) * 4),
                 p.side + base + static_cast<int64_t>(it * QB + r) * D + col);
    }
  };
  stage_bf16<64>(sQ, p.q + base + int64_t(q0) * D, D, tid);
  stage_bf16<64>(sH, p.hub + base + int64_t(q0) * D, D, tid);
  stage(first, 0);
  cp_async_commit();

  const int r0 = warp * 16;
  float nm[5][2][4], dm[5][2][4], lm[2][2][4], mm[2][2][4];
#pragma unroll
  for (int b = 0; b < 5; ++b)
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) nm[b][n][e] = dm[b][n][e] = 0.f;
#pragma unroll
  for (int b = 0; b < 2; ++b)
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) lm[b][n][e] = mm[b][n][e] = 0.f;
  float s1n[2] = {0.f, 0.f}, s2n[2] = {0.f, 0.f}, s1d[2] = {0.f, 0.f}, s2d[2] = {0.f, 0.f};
  float lse_r[2], hout_r[2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int64_t i = static_cast<int64_t>(row) * p.T + q0 + r0 + g + 8 * hr;
    lse_r[hr] = p.lse[i];
    hout_r[hr] = p.hub_out[i];
  }

  for (int it = first; it <= last; ++it) {
    const int buf = (it - first) & 1;
    const uint32_t sK = sSt + buf * Q_STAGE, sV = sK + QB * 128;
    const float* side = reinterpret_cast<const float*>(smem + 2 * 64 * 128 + buf * Q_STAGE + 2 * QB * 128);
    if (it < last) {
      stage(it + 1, buf ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    for (int i = tid; i < QB * 16; i += 128) {
      const int r = i >> 4, c = i & 15;
      const int P = pq16(c);  // pair within the part
      const float x = side[r * 36 + P] * 0.125f, y = side[r * 36 + 16 + P] * 0.125f;
      const uint32_t off = static_cast<uint32_t>(r * 48 + c * 2);
      st_bf16(feat, off, x);
      st_bf16(feat + QF, off, y);
      st_bf16(feat + 2 * QF, off, x * x);
      st_bf16(feat + 3 * QF, off, y * y);
      st_bf16(feat + 4 * QF, off, x * y);
    }
    __syncthreads();
    float lg[4][4], cc[4][4];
    dot_block<true, 4>(sQ, sK, r0, lane, lg);  // q_s . k_t
    dot_block<true, 4>(sH, sV, r0, lane, cc);  // hub_s . v_t
    float wn[4][4], wnl[4][4], al[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int hr = e >> 1;
        const int sq_ = q0 + r0 + g + 8 * hr;
        const int tk = it * QB + n * 8 + 2 * q + (e & 1);
        const float logit = lg[n][e] * 0.125f;
        float a = ex2_approx((logit - lse_r[hr]) * LOG2E);
        if (tk > sq_ || sq_ - tk > p.window) a = 0.f;
        const float c = cc[n][e] - hout_r[hr];
        const float w = a * c;
        wn[n][e] = w;
        wnl[n][e] = w * logit;
        al[n][e] = a * logit;
        lg[n][e] = a;
        s1n[hr] += w * logit;
        s2n[hr] += w * logit * logit;
        s1d[hr] += a * logit;
        s2d[hr] += a * logit * logit;
      }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint32_t aw[4], aa[4], awl[4], aal[4];
      pack_a(wn, j, aw);
      pack_a(lg, j, aa);
      pack_a(wnl, j, awl);
      pack_a(al, j, aal);
#pragma unroll
      for (int b = 0; b < 5; ++b) {
        uint32_t f[4];
        const int row_ = j * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        ldsm_x4_t(sF + b * QF + static_cast<uint32_t>(row_ * 48 + (lane >> 4) * 16), f[0], f[1], f[2], f[3]);
        mma_bf16(nm[b][0], aw[0], aw[1], aw[2], aw[3], f[0], f[1]);
        mma_bf16(nm[b][1], aw[0], aw[1], aw[2], aw[3], f[2], f[3]);
        mma_bf16(dm[b][0], aa[0], aa[1], aa[2], aa[3], f[0], f[1]);
        mma_bf16(dm[b][1], aa[0], aa[1], aa[2], aa[3], f[2], f[3]);
        if (b < 2) {
          mma_bf16(lm[b][0], awl[0], awl[1], awl[2], awl[3], f[0], f[1]);
          mma_bf16(lm[b][1], awl[0], awl[1], awl[2], awl[3], f[2], f[3]);
          mma_bf16(mm[b][0], aal[0], aal[1], aal[2], aal[3], f[0], f[1]);
          mma_bf16(mm[b][1], aal[0], aal[1], aal[2], aal[3], f[2], f[3]);
        }
      }
    }
    __syncthreads();
  }

#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    float v1n = s1n[hr], v2n = s2n[hr], v1d = s1d[hr], v2d = s2d[hr];
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      v1n += __shfl_xor_sync(0xffffffffu, v1n, o);
      v2n += __shfl_xor_sync(0xffffffffu, v2n, o);
      v1d += __shfl_xor_sync(0xffffffffu, v1d, o);
      v2d += __shfl_xor_sync(0xffffffffu, v2d, o);
    }
    const int sq_ = q0 + r0 + g + 8 * hr;
    const int64_t ti = static_cast<int64_t>(row) * p.T + sq_;
    const float sqv = p.sq[ti], stepv = p.steps[ti];
    const float den = sqv / D + 1e-6f, rs = rsqrtf(den);
    const int64_t ro = p.raw.at(row, sq_, p.T);
    const int64_t ob = p.out.at(row, sq_, p.T);
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int P = part * 16 + 8 * n + 4 * e + q;
        const int k = e + 2 * hr;
        const float cs = p.cosb[static_cast<int64_t>(sq_) * 32 + P], sn = p.sinb[static_cast<int64_t>(sq_) * 32 + P];
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int d = P + 32 * half;
          const float change = (2.f * stepv * raw_at(p.raw, p.raw_bf16, ro + d) + stepv * stepv) / D / den;
          const float ca = expm1f(-0.5f * log1pf(change));
          const float b = stepv * rs * (1.f + ca);
          const float bu = b * (half ? sn : cs), bw = b * (half ? cs : -sn);
          const float zn = nm[0][n][k] * bu + nm[1][n][k] * bw + 0.5f * (nm[2][n][k] * bu * bu + nm[3][n][k] * bw * bw) +
                           nm[4][n][k] * bu * bw + ca * (lm[0][n][k] * bu + lm[1][n][k] * bw) + v1n * ca +
                           v2n * (0.5f * ca * ca);
          const float zd = dm[0][n][k] * bu + dm[1][n][k] * bw + 0.5f * (dm[2][n][k] * bu * bu + dm[3][n][k] * bw * bw) +
                           dm[4][n][k] * bu * bw + ca * (mm[0][n][k] * bu + mm[1][n][k] * bw) + v1d * ca +
                           v2d * (0.5f * ca * ca);
          const float z = bf16_round(zn / (1.f + zd) / stepv);
          if (p.out_bf16)
            static_cast<__nv_bfloat16*>(p.out.data)[ob + d] = __float2bfloat16_rn(z);
          else
            static_cast<float*>(p.out.data)[ob + d] = z;
        }
      }
  }
}

static bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// A (by-layer / by-token) view the vectorised kernels accept: 16-byte aligned rows, no blocked layout.
static bool rows_ok(const noise_rows_t& r, bool f32) {
  return r.data && r.heads >= 1 && r.block_rows == 0 && a16(r.data) && (r.token_stride * (f32 ? 4 : 2)) % 16 == 0 &&
         (r.layer_stride * (f32 ? 4 : 2)) % 16 == 0;
}

// A view the moment-score epilogues accept (blocked allowed): element-aligned scalar accesses, and with `pairs` the
// value sums' two-element stores (even strides).
static bool view_ok(const noise_rows_t& r, bool bf16, bool pairs) {
  const int64_t esz = bf16 ? 2 : 4, align = pairs ? 2 * esz : esz;
  if (!r.data || r.heads < 1 || (reinterpret_cast<uintptr_t>(r.data) % align)) return false;
  if (r.block_rows < 0 || (r.block_rows > 0 && (r.per_gpu < 1 || r.heads != 1 || r.layer_map))) return false;
  if (pairs && ((r.token_stride | r.layer_stride | r.gpu_stride) & 1)) return false;
  return true;
}

}  // namespace credit
}  // namespace noise

#include "context_tc.cuh"
#include "keymom_tc.cuh"
#include "querymom_tc.cuh"
#include "value_tc.cuh"

using namespace noise::credit;

namespace {

// A _ws entry point that falls through to a kernel without bounded waits still leaves the caller's status word
// reading 0, as its contract says.
int fall_through_status(void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace || workspace_bytes < sizeof(int) || (reinterpret_cast<uintptr_t>(workspace) & 3)) return NOISE_OK;
  return cudaMemsetAsync(workspace, 0, sizeof(int), static_cast<cudaStream_t>(stream)) == cudaSuccess ? NOISE_OK
                                                                                                   : NOISE_ERR_CUDA;
}

PFN_cuTensorMapEncodeTiled_v12000 tv_encode() {
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

// [n, 64] bf16 rows, box 128 rows x 64 with 128-byte swizzle; or (lse) fp32 [rows, T], box 1 x 128, no swizzle
int tv_map(CUtensorMap* map, const void* base, bool bf16, uint64_t inner, uint64_t outer) {
  auto fn = tv_encode();
  if (!fn) return NOISE_ERR_CUDA;
  if (reinterpret_cast<uintptr_t>(base) & 15) return NOISE_ERR_ALIGN;
  const uint64_t es = bf16 ? 2 : 4;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * es};
  cuuint32_t box[2] = {bf16 ? 64u : static_cast<cuuint32_t>(TV_B), bf16 ? static_cast<cuuint32_t>(TV_B) : 1u};
  cuuint32_t el[2] = {1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                  const_cast<void*>(base), dims, strides, box, el, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  bf16 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NOISE_OK : NOISE_ERR_CUDA;
}

// bf16 [n, 64] rows with KM_R-row boxes (the key moments' receiver-side tiles), 128-byte swizzle
int km_map(CUtensorMap* map, const void* base, uint64_t n) {
  auto fn = tv_encode();
  if (!fn) return NOISE_ERR_CUDA;
  if (reinterpret_cast<uintptr_t>(base) & 15) return NOISE_ERR_ALIGN;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(D), n};
  cuuint64_t strides[1] = {D * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(KM_R)};
  cuuint32_t el[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, el,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NOISE_OK : NOISE_ERR_CUDA;
}

// [n, 64] rows of bf16 or fp32 with box_rows x box_cols boxes, 128-byte swizzle (box_cols x element = 128 bytes)
int km_map_rows(CUtensorMap* map, const void* base, bool bf16, uint64_t n, uint32_t box_cols, uint32_t box_rows) {
  auto fn = tv_encode();
  if (!fn) return NOISE_ERR_CUDA;
  if (reinterpret_cast<uintptr_t>(base) & 15) return NOISE_ERR_ALIGN;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(D), n};
  cuuint64_t strides[1] = {D * (bf16 ? 2u : 4u)};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t el[2] = {1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                  const_cast<void*>(base), dims, strides, box, el, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NOISE_OK : NOISE_ERR_CUDA;
}

// fp32 [rows, T] with KM_R x 1 boxes (per-receiver lse / center of one receiver tile)
int km_map_f32(CUtensorMap* map, const float* base, uint64_t t, uint64_t rows) {
  auto fn = tv_encode();
  if (!fn) return NOISE_ERR_CUDA;
  if (reinterpret_cast<uintptr_t>(base) & 15) return NOISE_ERR_ALIGN;
  cuuint64_t dims[2] = {t, rows};
  cuuint64_t strides[1] = {t * 4};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(KM_R), 1};
  cuuint32_t el[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, el,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NOISE_OK : NOISE_ERR_CUDA;
}

int tv_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return n;
}

}  // namespace

extern "C" {

int noise_implicit_key_context(const void* q, const void* k, const void* values, const void* hub, int dtype, int rows,
                               int tokens, int window, float* lse, float* center, void* stream) {
  if (!q || !k || !values || !hub || !lse || !center) return NOISE_ERR_ARGUMENT;
  if (dtype != NOISE_DTYPE_F32 && dtype != NOISE_DTYPE_BF16) return NOISE_ERR_ARGUMENT;
  if (rows < 1 || tokens < 64 || tokens % 64 || window < 0 || window % 64) return NOISE_ERR_SHAPE;
  if (!a16(q) || !a16(k) || !a16(values) || !a16(hub)) return NOISE_ERR_ALIGN;
  CtxArgs a{q, k, values, hub, lse, center, tokens, window};
  const bool bf = dtype == NOISE_DTYPE_BF16;
  const int smem = (bf ? 64 * 128 : 64 * PITCH_F32 * 4) * 6;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  dim3 grid(tokens / 64, rows);
  if (bf) {
    if (cudaFuncSetAttribute(implicit_ctx_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) return NOISE_ERR_CUDA;
    implicit_ctx_kernel<true><<<grid, 128, smem, s>>>(a);
  } else {
    if (cudaFuncSetAttribute(implicit_ctx_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) return NOISE_ERR_CUDA;
    implicit_ctx_kernel<false><<<grid, 128, smem, s>>>(a);
  }
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_implicit_key_context_ws(const void* q, const void* k, const void* values, const void* hub, int dtype,
                                  int rows, int tokens, int window, float* lse, float* center, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  if (!q || !k || !values || !hub || !lse || !center) return NOISE_ERR_ARGUMENT;
  if (dtype != NOISE_DTYPE_F32 && dtype != NOISE_DTYPE_BF16) return NOISE_ERR_ARGUMENT;
  if (dtype != NOISE_DTYPE_BF16 || tokens % TC_B) {  // fp32 operands (tf32 dots) or T % 128 != 0: the warp-MMA kernel
    if (const int rc = fall_through_status(workspace, workspace_bytes, stream)) return rc;
    return noise_implicit_key_context(q, k, values, hub, dtype, rows, tokens, window, lse, center, stream);
  }
  if (rows < 1 || window < 0 || window % 64) return NOISE_ERR_SHAPE;
  if (!a16(q) || !a16(k) || !a16(values) || !a16(hub)) return NOISE_ERR_ALIGN;
  if (!workspace || workspace_bytes < NOISE_STATUS_BYTES) return NOISE_ERR_WORKSPACE;
  const int sms = tv_sms();
  if (sms < 1) return NOISE_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint64_t n = static_cast<uint64_t>(rows) * tokens;
  CUtensorMap mq, mk, mh, mv;
  int rc;
  if ((rc = tv_map(&mq, q, true, D, n)) || (rc = tv_map(&mk, k, true, D, n)) || (rc = tv_map(&mh, hub, true, D, n)) ||
      (rc = tv_map(&mv, values, true, D, n)))
    return rc;
  int* status = static_cast<int*>(workspace);
  if (cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess) return NOISE_ERR_CUDA;
  if (cudaFuncSetAttribute(context_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM))
    return NOISE_ERR_CUDA;
  const TContextArgs a{tokens, std::min(window, tokens), rows, lse, center, status};
  const int items = (tokens / TC_B + 1) / 2 * rows;
  context_tc_kernel<<<std::min(items, sms), TC_THREADS, TC_SMEM, s>>>(mq, mk, mh, mv, a);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_value_pass(const void* q, const void* k, int dtype, const float* lse, const noise_rows_t* source,
                     const noise_rows_t* out, int rows, int tokens, int window, void* stream) {
  if (!q || !k || !lse || !source || !out) return NOISE_ERR_ARGUMENT;
  if (dtype != NOISE_DTYPE_F32 && dtype != NOISE_DTYPE_BF16) return NOISE_ERR_ARGUMENT;
  if (rows < 1 || tokens < 64 || tokens % 64 || window < 0) return NOISE_ERR_SHAPE;
  if (!a16(q) || !a16(k) || !rows_ok(*source, true) || !rows_ok(*out, true)) return NOISE_ERR_ALIGN;
  ValueArgs a{q, k, lse, to_rows(*source), to_rows(*out), tokens, window};
  const bool bf = dtype == NOISE_DTYPE_BF16;
  const int tb = bf ? 64 * 128 : 64 * PITCH_F32 * 4;
  const int smem = 3 * tb + 2 * 64 * 128 + 64 * 4;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  dim3 grid(tokens / 64, rows);
  if (bf) {
    if (cudaFuncSetAttribute(value_pass_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) return NOISE_ERR_CUDA;
    value_pass_kernel<true><<<grid, 128, smem, s>>>(a);
  } else {
    if (cudaFuncSetAttribute(value_pass_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) return NOISE_ERR_CUDA;
    value_pass_kernel<false><<<grid, 128, smem, s>>>(a);
  }
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

size_t noise_value_pass_workspace_bytes(int rows, int tokens) {
  if (rows < 1 || tokens < 1) return 0;
  return 256 + 2 * static_cast<size_t>(rows) * tokens * D * sizeof(__nv_bfloat16);
}

int noise_value_pass_ws(const void* q, const void* k, int dtype, const float* lse, const noise_rows_t* source,
                        const noise_rows_t* out, int rows, int tokens, int window, void* workspace,
                        size_t workspace_bytes, void* stream) {
  if (!q || !k || !lse || !source || !out) return NOISE_ERR_ARGUMENT;
  if (dtype != NOISE_DTYPE_F32 && dtype != NOISE_DTYPE_BF16) return NOISE_ERR_ARGUMENT;
  if (dtype != NOISE_DTYPE_BF16 || tokens % TV_B) {  // fp32 operands or T % 128 != 0: the warp-MMA kernel
    if (const int rc = fall_through_status(workspace, workspace_bytes, stream)) return rc;
    return noise_value_pass(q, k, dtype, lse, source, out, rows, tokens, window, stream);
  }
  if (rows < 1 || window < 0) return NOISE_ERR_SHAPE;
  if (!a16(q) || !a16(k) || !a16(lse) || !rows_ok(*source, true) || !rows_ok(*out, true)) return NOISE_ERR_ALIGN;
  if (!workspace || workspace_bytes < noise_value_pass_workspace_bytes(rows, tokens)) return NOISE_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return NOISE_ERR_ALIGN;
  const int sms = tv_sms();
  if (sms < 1) return NOISE_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* status = static_cast<int*>(workspace);
  __nv_bfloat16* hi = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(workspace) + 256);
  __nv_bfloat16* lo = hi + static_cast<int64_t>(rows) * tokens * D;
  const uint64_t n = static_cast<uint64_t>(rows) * tokens;
  CUtensorMap mk, mq, mhi, mlo, mlse;
  int rc;
  if ((rc = tv_map(&mk, k, true, D, n)) || (rc = tv_map(&mq, q, true, D, n)) || (rc = tv_map(&mhi, hi, true, D, n)) ||
      (rc = tv_map(&mlo, lo, true, D, n)) || (rc = tv_map(&mlse, lse, false, tokens, rows)))
    return rc;
  if (cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess) return NOISE_ERR_CUDA;
  const int64_t n4 = static_cast<int64_t>(n) * (D / 4);
  const int split_blocks = static_cast<int>(std::min<int64_t>((n4 + 255) / 256, static_cast<int64_t>(sms) * 8));
  split_source_kernel<<<split_blocks, 256, 0, s>>>(to_rows(*source), tokens, n4, hi, lo);
  if (cudaFuncSetAttribute(value_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TV_SMEM)) return NOISE_ERR_CUDA;
  const TValueArgs a{tokens, std::min(window, tokens), rows, to_rows(*out), status};
  const int items = (tokens / TV_B + 1) / 2 * rows;
  value_tc_kernel<<<std::min(items, sms), TV_THREADS, TV_SMEM, s>>>(mk, mq, mhi, mlo, mlse, a);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_key_scan(const float* qp, const float* kp, const float* k_raw, const float* lse, const float* values,
                   const float* hub, const float* center, const float* cos, const float* sin, int rows, int tokens,
                   int window, float sigma, const noise_rows_t* key_out, const noise_rows_t* value_out, void* stream) {
  if (!qp || !kp || !k_raw || !lse || !values || !hub || !center || !cos || !sin || !key_out) return NOISE_ERR_ARGUMENT;
  if (rows < 1 || tokens < 64 || tokens % 64 || window < 0) return NOISE_ERR_SHAPE;
  if (!a16(qp) || !a16(kp) || !a16(values) || !a16(hub) || !rows_ok(*key_out, true)) return NOISE_ERR_ALIGN;
  if (value_out && value_out->data && !rows_ok(*value_out, true)) return NOISE_ERR_ALIGN;
  KeyArgs a{};
  a.qp = qp;
  a.kp = kp;
  a.values = values;
  a.hub = hub;
  a.raw = stacked_rows(k_raw, tokens);
  a.lse = lse;
  a.center = center;
  a.cosb = cos;
  a.sinb = sin;
  a.out = to_rows(*key_out);
  a.vout = value_out ? to_rows(*value_out) : Rows{};
  a.T = tokens;
  a.window = window;
  a.sigma = sigma;
  const int smem = KeyLayout<false>::SMEM;
  if (cudaFuncSetAttribute(key_moments_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) return NOISE_ERR_CUDA;
  key_moments_kernel<false><<<dim3(tokens / 64, rows), 128, smem, static_cast<cudaStream_t>(stream)>>>(a);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

size_t noise_key_scan_workspace_bytes(int rows, int tokens) {
  if (rows < 1 || tokens < 1) return 0;
  return 256 + 5 * static_cast<size_t>(rows) * tokens * D * sizeof(__nv_bfloat16);
}

int noise_key_scan_ws(const float* qp, const float* kp, const float* k_raw, const float* lse, const float* values,
                      const float* hub, const float* center, const float* cos, const float* sin, int rows, int tokens,
                      int window, float sigma, const noise_rows_t* key_out, const noise_rows_t* value_out,
                      void* workspace, size_t workspace_bytes, void* stream) {
  if (!qp || !kp || !k_raw || !lse || !values || !hub || !center || !cos || !sin || !key_out) return NOISE_ERR_ARGUMENT;
  const bool with_values = value_out && value_out->data;
  auto vec_ok = [&](const noise_rows_t& r) {  // fp32 views with 16-byte strides (the kernel's vector stores)
    return r.data && rows_ok(r, true) && r.block_rows == 0;
  };
  if (tokens % KM_B || !vec_ok(*key_out) || (with_values && !vec_ok(*value_out)) || !a16(cos) || !a16(sin) ||
      !a16(lse) || !a16(center)) {
    if (const int rc = fall_through_status(workspace, workspace_bytes, stream)) return rc;
    return noise_key_scan(qp, kp, k_raw, lse, values, hub, center, cos, sin, rows, tokens, window, sigma, key_out,
                          value_out, stream);
  }
  if (rows < 1 || window < 0) return NOISE_ERR_SHAPE;
  if (!a16(qp) || !a16(kp) || !a16(values) || !a16(hub)) return NOISE_ERR_ALIGN;
  if (!workspace || workspace_bytes < noise_key_scan_workspace_bytes(rows, tokens)) return NOISE_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return NOISE_ERR_ALIGN;
  const int sms = tv_sms();
  if (sms < 1) return NOISE_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* status = static_cast<int*>(workspace);
  const int64_t n = static_cast<int64_t>(rows) * tokens;
  __nv_bfloat16* f2 = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(workspace) + 256);
  __nv_bfloat16* g2 = f2 + n * D;
  __nv_bfloat16* xy = g2 + n * D;
  __nv_bfloat16* hi = xy + n * D;
  __nv_bfloat16* lo = hi + n * D;
  KeyMomMaps m;
  int rc;
  // the logits' and scores' operands go to the kind::tf32 MMAs as they are: the tensor core reads the tf32 part of
  // each fp32 value, as the reference's Triton kernel's tf32 dots do on this GPU (no rounding pass)
  if ((rc = km_map_rows(&m.k, kp, false, n, 32, KM_B)) || (rc = km_map_rows(&m.v, values, false, n, 32, KM_B)) ||
      (rc = km_map_rows(&m.q, qp, false, n, 32, KM_R)) || (rc = km_map_rows(&m.h, hub, false, n, 32, KM_R)) ||
      (rc = km_map(&m.f2, f2, n)) || (rc = km_map(&m.g2, g2, n)) || (rc = km_map(&m.xy, xy, n)) ||
      (rc = km_map(&m.hi, hi, n)) || (rc = km_map(&m.lo, lo, n)) || (rc = km_map_f32(&m.lse, lse, tokens, rows)) ||
      (rc = km_map_f32(&m.ctr, center, tokens, rows)))
    return rc;
  if (cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess) return NOISE_ERR_CUDA;
  const int64_t n_pairs = n * 32;
  keymom_features_kernel<<<static_cast<int>(std::min<int64_t>((n_pairs + 255) / 256, static_cast<int64_t>(sms) * 8)),
                           256, 0, s>>>(qp, n_pairs, f2, g2, xy);
  if (with_values) {
    const Rows hub_rows = stacked_rows(hub, tokens);
    const int64_t n4 = n * (D / 4);
    split_source_kernel<<<static_cast<int>(std::min<int64_t>((n4 + 255) / 256, static_cast<int64_t>(sms) * 8)), 256,
                          0, s>>>(hub_rows, tokens, n4, hi, lo);
  }
  KeyMomTcArgs a{};
  a.T = tokens;
  a.window = std::min(window, tokens);
  a.rows = rows;
  a.raw = stacked_rows(k_raw, tokens);
  a.raw_bf16 = 0;
  a.out_bf16 = 0;
  a.sigma = sigma;
  a.cosb = cos;
  a.sinb = sin;
  a.out = to_rows(*key_out);
  a.vout = with_values ? to_rows(*value_out) : Rows{};
  a.status = status;
  const int items = tokens / KM_B * rows;
  // without value credits the stages drop the hub's hi / lo tiles, leaving room for a third stage
  auto launch = [&](auto vals_tag) {
    constexpr bool VALS = decltype(vals_tag)::value;
    if (cudaFuncSetAttribute(keymom_tc_kernel<true, VALS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             KmLayout<true, VALS>::SMEM))
      return NOISE_ERR_CUDA;
    keymom_tc_kernel<true, VALS><<<std::min(items, sms), KM_THREADS, KmLayout<true, VALS>::SMEM, s>>>(m, a);
    return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
  };
  return with_values ? launch(std::true_type{}) : launch(std::false_type{});
}

int noise_moment_key_scores_v(const void* q, const void* k, const void* v, const void* hub, const noise_rows_t* raw,
                              int raw_dtype, const float* sq, const float* side, const float* cos, const float* sin,
                              const float* lse, const float* hub_out, const float* steps, int rows, int tokens,
                              const noise_rows_t* out, const noise_rows_t* values_out, int out_dtype, void* stream) {
  if (!q || !k || !v || !hub || !raw || !sq || !side || !cos || !sin || !lse || !hub_out || !steps || !out || !values_out)
    return NOISE_ERR_ARGUMENT;
  if ((raw_dtype != NOISE_DTYPE_F32 && raw_dtype != NOISE_DTYPE_BF16) ||
      (out_dtype != NOISE_DTYPE_F32 && out_dtype != NOISE_DTYPE_BF16))
    return NOISE_ERR_ARGUMENT;
  if (rows < 1 || tokens < 64 || tokens % 64) return NOISE_ERR_SHAPE;
  const bool ob = out_dtype == NOISE_DTYPE_BF16;
  if (!a16(q) || !a16(k) || !a16(v) || !a16(hub) || !a16(side) || !view_ok(*raw, raw_dtype == NOISE_DTYPE_BF16, false) ||
      !view_ok(*out, ob, false) || !view_ok(*values_out, ob, true))
    return NOISE_ERR_ALIGN;
  KeyArgs a{};
  a.qp = q;
  a.kp = k;
  a.values = v;
  a.hub = hub;
  a.side = side;
  a.raw = to_rows(*raw);
  a.raw_bf16 = raw_dtype == NOISE_DTYPE_BF16;
  a.out_bf16 = ob;
  a.sq = sq;
  a.steps = steps;
  a.lse = lse;
  a.center = hub_out;
  a.cosb = cos;
  a.sinb = sin;
  a.out = to_rows(*out);
  a.vout = to_rows(*values_out);
  a.T = tokens;
  a.window = tokens;
  const int smem = KeyLayout<true>::SMEM;
  if (cudaFuncSetAttribute(key_moments_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) return NOISE_ERR_CUDA;
  key_moments_kernel<true><<<dim3(tokens / 64, rows), 128, smem, static_cast<cudaStream_t>(stream)>>>(a);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

size_t noise_moment_key_scores_workspace_bytes(int rows, int tokens) {
  if (rows < 1 || tokens < 1) return 0;
  return 256 + 3 * static_cast<size_t>(rows) * tokens * D * sizeof(__nv_bfloat16);
}

int noise_moment_key_scores_ws(const void* q, const void* k, const void* v, const void* hub, const noise_rows_t* raw,
                               int raw_dtype, const float* sq, const float* side, const float* cos, const float* sin,
                               const float* lse, const float* hub_out, const float* steps, int rows, int tokens,
                               const noise_rows_t* out, const noise_rows_t* values_out, int out_dtype, void* workspace,
                               size_t workspace_bytes, void* stream) {
  if (!q || !k || !v || !hub || !raw || !sq || !side || !cos || !sin || !lse || !hub_out || !steps || !out || !values_out)
    return NOISE_ERR_ARGUMENT;
  if ((raw_dtype != NOISE_DTYPE_F32 && raw_dtype != NOISE_DTYPE_BF16) ||
      (out_dtype != NOISE_DTYPE_F32 && out_dtype != NOISE_DTYPE_BF16))
    return NOISE_ERR_ARGUMENT;
  const bool ob = out_dtype == NOISE_DTYPE_BF16;
  // the tcgen05 kernel stores 16 consecutive outputs per vector: every view stride a 16-byte multiple
  auto vec_ok = [&](const noise_rows_t& r) {
    const int64_t es = ob ? 2 : 4;
    return r.data && a16(r.data) && (r.layer_stride * es) % 16 == 0 && (r.token_stride * es) % 16 == 0 &&
           (r.block_rows == 0 || (r.gpu_stride * es) % 16 == 0);
  };
  if (tokens % KM_B || !vec_ok(*out) || !vec_ok(*values_out) || !a16(cos) || !a16(sin)) {
    if (const int rc = fall_through_status(workspace, workspace_bytes, stream)) return rc;
    return noise_moment_key_scores_v(q, k, v, hub, raw, raw_dtype, sq, side, cos, sin, lse, hub_out, steps, rows,
                                     tokens, out, values_out, out_dtype, stream);
  }
  if (rows < 1) return NOISE_ERR_SHAPE;
  if (!a16(q) || !a16(k) || !a16(v) || !a16(hub) || !a16(side) || !a16(lse) || !a16(hub_out) ||
      !view_ok(*raw, raw_dtype == NOISE_DTYPE_BF16, false) || !view_ok(*out, ob, false) ||
      !view_ok(*values_out, ob, true))
    return NOISE_ERR_ALIGN;
  if (!workspace || workspace_bytes < noise_moment_key_scores_workspace_bytes(rows, tokens)) return NOISE_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return NOISE_ERR_ALIGN;
  const int sms = tv_sms();
  if (sms < 1) return NOISE_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* status = static_cast<int*>(workspace);
  const int64_t n = static_cast<int64_t>(rows) * tokens;
  __nv_bfloat16* f2 = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(workspace) + 256);
  __nv_bfloat16* g2 = f2 + n * D;
  __nv_bfloat16* xy = g2 + n * D;
  KeyMomMaps m;
  int rc;
  if ((rc = tv_map(&m.k, k, true, D, n)) || (rc = tv_map(&m.v, v, true, D, n)) ||
      (rc = km_map(&m.q, q, n)) || (rc = km_map(&m.h, hub, n)) || (rc = km_map(&m.f2, f2, n)) ||
      (rc = km_map(&m.g2, g2, n)) || (rc = km_map(&m.xy, xy, n)) || (rc = km_map_f32(&m.lse, lse, tokens, rows)) ||
      (rc = km_map_f32(&m.ctr, hub_out, tokens, rows)))
    return rc;
  m.hi = m.lo = m.xy;  // unused by the identity-phase variant
  if (cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess) return NOISE_ERR_CUDA;
  const int64_t n_pairs = n * 32;
  keymom_features_kernel<<<static_cast<int>(std::min<int64_t>((n_pairs + 255) / 256, static_cast<int64_t>(sms) * 8)),
                           256, 0, s>>>(side, n_pairs, f2, g2, xy);
  if (cudaFuncSetAttribute(keymom_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           KmLayout<false>::SMEM))
    return NOISE_ERR_CUDA;
  KeyMomTcArgs a{};
  a.T = tokens;
  a.window = tokens;
  a.rows = rows;
  a.raw = to_rows(*raw);
  a.raw_bf16 = raw_dtype == NOISE_DTYPE_BF16;
  a.out_bf16 = ob;
  a.sq = sq;
  a.steps = steps;
  a.cosb = cos;
  a.sinb = sin;
  a.out = to_rows(*out);
  a.vout = to_rows(*values_out);
  a.status = status;
  const int items = tokens / KM_B * rows;
  keymom_tc_kernel<false><<<std::min(items, sms), KM_THREADS, KmLayout<false>::SMEM, s>>>(m, a);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_moment_key_scores(const void* q, const void* k, const void* v, const void* hub, const float* raw,
                            const float* sq, const float* side, const float* cos, const float* sin, const float* lse,
                            const float* hub_out, const float* steps, int rows, int tokens, const noise_rows_t* out,
                            const noise_rows_t* values_out, void* stream) {
  if (!raw || !out || !values_out) return NOISE_ERR_ARGUMENT;
  if (!rows_ok(*out, true) || !rows_ok(*values_out, true)) return NOISE_ERR_ALIGN;
  const noise_rows_t rv{const_cast<float*>(raw), static_cast<int64_t>(tokens) * D, D, 1, nullptr, 0, 0, 0};
  return noise_moment_key_scores_v(q, k, v, hub, &rv, NOISE_DTYPE_F32, sq, side, cos, sin, lse, hub_out, steps, rows,
                                   tokens, out, values_out, NOISE_DTYPE_F32, stream);
}

int noise_moment_query_scores_v(const void* q, const void* k, const void* v, const void* hub, const noise_rows_t* raw,
                                int raw_dtype, const float* sq, const float* side, const float* cos, const float* sin,
                                const float* lse, const float* hub_out, const float* steps, int rows, int tokens,
                                int window, const noise_rows_t* out, int out_dtype, void* stream) {
  if (!q || !k || !v || !hub || !raw || !sq || !side || !cos || !sin || !lse || !hub_out || !steps || !out)
    return NOISE_ERR_ARGUMENT;
  if ((raw_dtype != NOISE_DTYPE_F32 && raw_dtype != NOISE_DTYPE_BF16) ||
      (out_dtype != NOISE_DTYPE_F32 && out_dtype != NOISE_DTYPE_BF16))
    return NOISE_ERR_ARGUMENT;
  if (rows < 1 || tokens < 64 || tokens % 64 || window < 0) return NOISE_ERR_SHAPE;
  if (!a16(q) || !a16(k) || !a16(v) || !a16(hub) || !a16(side) || !view_ok(*raw, raw_dtype == NOISE_DTYPE_BF16, false) ||
      !view_ok(*out, out_dtype == NOISE_DTYPE_BF16, false))
    return NOISE_ERR_ALIGN;
  QueryArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.hub = static_cast<const __nv_bfloat16*>(hub);
  a.raw = to_rows(*raw);
  a.raw_bf16 = raw_dtype == NOISE_DTYPE_BF16;
  a.sq = sq;
  a.steps = steps;
  a.lse = lse;
  a.hub_out = hub_out;
  a.side = side;
  a.cosb = cos;
  a.sinb = sin;
  a.out = to_rows(*out);
  a.out_bf16 = out_dtype == NOISE_DTYPE_BF16;
  a.T = tokens;
  a.window = window < tokens ? window : tokens;
  if (cudaFuncSetAttribute(query_moments_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Q_SMEM)) return NOISE_ERR_CUDA;
  query_moments_kernel<<<dim3(tokens / 64, 2 * rows), 128, Q_SMEM, static_cast<cudaStream_t>(stream)>>>(a);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

size_t noise_moment_query_scores_workspace_bytes(int rows, int tokens) {
  if (rows < 1 || tokens < 1) return 0;
  return 256 + 3 * static_cast<size_t>(rows) * tokens * D * sizeof(__nv_bfloat16);
}

int noise_moment_query_scores_ws(const void* q, const void* k, const void* v, const void* hub, const noise_rows_t* raw,
                                 int raw_dtype, const float* sq, const float* side, const float* cos, const float* sin,
                                 const float* lse, const float* hub_out, const float* steps, int rows, int tokens,
                                 int window, const noise_rows_t* out, int out_dtype, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  if (!q || !k || !v || !hub || !raw || !sq || !side || !cos || !sin || !lse || !hub_out || !steps || !out)
    return NOISE_ERR_ARGUMENT;
  if ((raw_dtype != NOISE_DTYPE_F32 && raw_dtype != NOISE_DTYPE_BF16) ||
      (out_dtype != NOISE_DTYPE_F32 && out_dtype != NOISE_DTYPE_BF16))
    return NOISE_ERR_ARGUMENT;
  const bool ob = out_dtype == NOISE_DTYPE_BF16;
  // the tcgen05 kernel stores 8 consecutive outputs per vector: every view stride a 16-byte multiple
  auto vec_ok = [&](const noise_rows_t& r) {
    const int64_t es = ob ? 2 : 4;
    return r.data && a16(r.data) && (r.layer_stride * es) % 16 == 0 && (r.token_stride * es) % 16 == 0 &&
           (r.block_rows == 0 || (r.gpu_stride * es) % 16 == 0);
  };
  if (tokens % QM_B || !vec_ok(*out) || !a16(cos) || !a16(sin)) {
    if (const int rc = fall_through_status(workspace, workspace_bytes, stream)) return rc;
    return noise_moment_query_scores_v(q, k, v, hub, raw, raw_dtype, sq, side, cos, sin, lse, hub_out, steps, rows,
                                       tokens, window, out, out_dtype, stream);
  }
  if (rows < 1 || window < 0) return NOISE_ERR_SHAPE;
  if (!a16(q) || !a16(k) || !a16(v) || !a16(hub) || !a16(side) ||
      !view_ok(*raw, raw_dtype == NOISE_DTYPE_BF16, false) || !view_ok(*out, ob, false))
    return NOISE_ERR_ALIGN;
  if (!workspace || workspace_bytes < noise_moment_query_scores_workspace_bytes(rows, tokens))
    return NOISE_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return NOISE_ERR_ALIGN;
  const int sms = tv_sms();
  if (sms < 1) return NOISE_ERR_CUDA;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* status = static_cast<int*>(workspace);
  const int64_t n = static_cast<int64_t>(rows) * tokens;
  __nv_bfloat16* fa = reinterpret_cast<__nv_bfloat16*>(static_cast<uint8_t*>(workspace) + 256);
  __nv_bfloat16* fb = fa + n * D;
  __nv_bfloat16* fc = fb + n * D;
  QueryMomMaps m;
  int rc;
  if ((rc = tv_map(&m.q, q, true, D, n)) || (rc = tv_map(&m.h, hub, true, D, n)) || (rc = km_map(&m.k, k, n)) ||
      (rc = km_map(&m.v, v, n)) || (rc = km_map(&m.fa, fa, n)) || (rc = km_map(&m.fb, fb, n)) ||
      (rc = km_map(&m.fc, fc, n)))
    return rc;
  if (cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess) return NOISE_ERR_CUDA;
  const int64_t n_pairs = n * 32;
  querymom_features_kernel<<<static_cast<int>(
                                 std::min<int64_t>((n_pairs + 255) / 256, static_cast<int64_t>(sms) * 8)),
                             256, 0, s>>>(side, n_pairs, fa, fb, fc);
  if (cudaFuncSetAttribute(querymom_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, QM_SMEM))
    return NOISE_ERR_CUDA;
  QueryMomTcArgs a{};
  a.T = tokens;
  a.window = std::min(window, tokens);
  a.rows = rows;
  a.raw = to_rows(*raw);
  a.raw_bf16 = raw_dtype == NOISE_DTYPE_BF16;
  a.out_bf16 = ob;
  a.sq = sq;
  a.steps = steps;
  a.lse = lse;
  a.hub_out = hub_out;
  a.cosb = cos;
  a.sinb = sin;
  a.out = to_rows(*out);
  a.status = status;
  const int items = tokens / QM_B * rows;
  querymom_tc_kernel<<<std::min(items, sms), QM_THREADS, QM_SMEM, s>>>(m, a);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_moment_query_scores(const void* q, const void* k, const void* v, const void* hub, const float* raw,
                              const float* sq, const float* side, const float* cos, const float* sin, const float* lse,
                              const float* hub_out, const float* steps, int rows, int tokens, int window,
                              const noise_rows_t* out, int out_dtype, void* stream) {
  if (!raw) return NOISE_ERR_ARGUMENT;
  const noise_rows_t rv{const_cast<float*>(raw), static_cast<int64_t>(tokens) * D, D, 1, nullptr, 0, 0, 0};
  return noise_moment_query_scores_v(q, k, v, hub, &rv, NOISE_DTYPE_F32, sq, side, cos, sin, lse, hub_out, steps, rows,
                                     tokens, window, out, out_dtype, stream);
}

}  // extern "C"
