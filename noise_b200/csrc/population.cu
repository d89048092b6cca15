// Population-perturbed forward of Noise's fixed GPT on sm_100a.
//
// Replaces eggroll.population_loss (reference archive/10M/train/val/eggroll.py:66-103): m members, each the GPT
// of utils/model.py with every matrix and embedding perturbed by sign_j a_j b_j^T and every mixing scalar by
// sign_j eps_j, all evaluated on one shared token row. Rows of every activation are (member, token) pairs,
// row r = j * T + t, so a 128-row GEMM tile belongs to one member (T % 128 == 0).
//
// Per block (8 blocks), 6 kernels:
//   norm_kernel<BLOCK>   mixing resid x + x0l x0 (x0 recomputed from wte + rank-1 term), RMS norm -> bf16 h,
//                        rank-1 dot products h.b for q, k, v, the value-embedding gate
//   GEMM + EpiQKV        h [M,512] x Wqkv^T [512,1536]; epilogue adds sign (h.b) a, RoPE + RMS norm of q and k,
//                        gated value embedding of v; writes q, k, v bf16 [m, H, T, 64]
//   attention_kernel     windowed causal softmax(q k^T / 8) v (mma.sync), writes y bf16 [M,512] and the per-head
//                        partial dots y.b of the c_proj perturbation
//   GEMM + EpiResid      x += y Wproj^T + sign (y.b) a
//   norm_kernel<MID>     RMS norm -> bf16 h, h.b of c_fc
//   GEMM + EpiFC         relu(h Wfc^T + sign (h.b) a)^2 -> bf16 hidden [M,2048], partial dots hidden.b of mlp.c_proj
//   GEMM + EpiResid      x += hidden Wmproj^T + sign (hidden.b) a
// then norm_kernel<FINAL> and GEMM + EpiHeadCE (LM head, softcap 15 tanh(z/15), cross-entropy against the target,
// logits never leave the SM) and member_reduce_kernel (per-member mean or sum).
//
// Rounding follows the reference under torch.autocast('cuda', bfloat16): every matmul takes bf16 operands and
// returns bf16; the rank-1 correction sign bf16(x.b) a and the residual stream stay fp32.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "gemm.cuh"
#include "noise_b200.h"
#include "ptx.cuh"
#include "warp_mma.cuh"

namespace noise {

constexpr int D = NOISE_N_EMBD;  // 512
constexpr int H = NOISE_N_HEAD;  // 8
constexpr int HD = NOISE_HEAD_DIM;  // 64
constexpr int F = 4 * NOISE_N_EMBD;  // 2048
constexpr int V = NOISE_VOCAB;  // 4096
constexpr float RMS_EPS = 1.1920928955078125e-07f;  // torch.finfo(float32).eps: F.rms_norm(eps=None) on fp32
constexpr float LOG2E = 1.4426950408889634f;
constexpr int GEMM_BN = 256;
constexpr int GEMM_STAGES = 3;

struct Slice {
  const float* a;
  const float* b;
  const int64_t* off;
  int64_t as, bs;
  __device__ __forceinline__ const float* A(int j) const { return a + (off ? off[j] : j * as); }
  __device__ __forceinline__ const float* B(int j) const { return b + (off ? off[j] : j * bs); }
};

static Slice to_slice(const noise_slice_t& s) { return Slice{s.a, s.b, s.off, s.a_stride, s.b_stride}; }

// ---------------------------------------------------------------------------------------------------------------
// Norm / mixing kernel: one warp per row, lane l holds columns 4 l + 128 i + {0..3}, i = 0..3.
// ---------------------------------------------------------------------------------------------------------------
enum NormMode { NORM_BLOCK = 0, NORM_MID = 1, NORM_FINAL = 2 };

struct NormArgs {
  int layer, T, M;
  const int64_t* idx;  // token ids: member j, position t reads idx[j * row_stride + t]
  int64_t row_stride;  // 0: every member reads the same row
  const float* sign;
  float* x;            // residual stream [M, 512] fp32
  __nv_bfloat16* h;    // out [M, 512] bf16
  float* svec;         // out [M, 4]: BLOCK (s_q, s_k, s_v, s_gate); MID s_fc; FINAL s_head (slot 0)
  float* gate;         // out [M, 8] (BLOCK, value-embedding layers)
  const float* wte;
  Slice n_wte, n_resid, n_x0;
  const float* resid_l;
  const float* x0_l;
  Slice nb0, nb1, nb2;  // b sources of the dot products (BLOCK: c_q, c_k, c_v; MID: c_fc; FINAL: lm_head)
  const float* wgate;  // [8, 32] fp32 or NULL
  Slice n_gate;
  int no_mix;          // BLOCK: x is the block's input as is (no x0 mixing; Dust's block_forward)
};

constexpr int NORM_ROWS = 64;  // rows per block: T % 128 == 0, so a block's rows are one member's

// dot of the row's bf16-rounded h (lane's 16 columns) with a bf16-rounded b staged in shared memory, rounded to bf16
// as autocast returns it
__device__ __forceinline__ float dot_staged(const float (&hb)[16], const float* sb, int lane) {
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 bv = *reinterpret_cast<const float4*>(sb + 4 * lane + 128 * i);
    acc[i] = fmaf(hb[4 * i + 0], bv.x, fmaf(hb[4 * i + 1], bv.y, fmaf(hb[4 * i + 2], bv.z, hb[4 * i + 3] * bv.w)));
  }
  return bf16_round(warp_sum((acc[0] + acc[1]) + (acc[2] + acc[3])));
}

// One block = NORM_ROWS consecutive rows of one member; each warp takes every eighth row. The member's noise vectors
// (read in place from the noise buffer at arbitrary 4-byte offsets) are staged once per block in shared memory,
// already rounded to bf16 where autocast rounds them: the b of every rank-1 dot this kernel forms (BLOCK: c_q, c_k,
// c_v and the ve_gate; MID: c_fc; FINAL: lm_head), the embedding's b (fp32), and bf16(ve_gate) itself.
template <int MODE>
__global__ void __launch_bounds__(256) norm_kernel(NormArgs p) {
  __shared__ __align__(16) float sb[3][D];
  __shared__ __align__(16) float swb[MODE == NORM_BLOCK ? D : 4];
  __shared__ __align__(16) float sgw[MODE == NORM_BLOCK ? (H + 1) * 32 : 4];  // bf16(W_gate) [8][32], bf16(b_gate)
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int row0 = blockIdx.x * NORM_ROWS;
  const int j = row0 / p.T;
  {
    const float* b0 = p.nb0.B(j);
    for (int i = threadIdx.x; i < D; i += 256) {
      sb[0][i] = bf16_round(b0[i]);
      if (MODE == NORM_BLOCK) {
        sb[1][i] = bf16_round(p.nb1.B(j)[i]);
        sb[2][i] = bf16_round(p.nb2.B(j)[i]);
        swb[i] = p.n_wte.B(j)[i];
      }
    }
    if (MODE == NORM_BLOCK && p.wgate)
      for (int i = threadIdx.x; i < (H + 1) * 32; i += 256)
        sgw[i] = bf16_round(i < H * 32 ? p.wgate[i] : p.n_gate.B(j)[i - H * 32]);
  }
  __syncthreads();
  const float sg = p.sign[j];

  for (int rr = wib; rr < NORM_ROWS; rr += 8) {
    const int r = row0 + rr;
    if (r >= p.M) break;
    const int t = r - j * p.T;
    float x[16];
    float* xrow = p.x + static_cast<int64_t>(r) * D;

    if (MODE == NORM_BLOCK && !p.no_mix) {
      // x0 = norm(wte[idx] + sign a[idx] b), eggroll.py:61-63, 74
      const int64_t tok = p.idx[j * p.row_stride + t];
      const float* w = p.wte + tok * D;
      const float sa = sg * p.n_wte.A(j)[tok];
      float x0[16], ss0[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 wv = *reinterpret_cast<const float4*>(w + 4 * lane + 128 * i);
        const float4 bv = *reinterpret_cast<const float4*>(swb + 4 * lane + 128 * i);
        x0[4 * i + 0] = wv.x + sa * bv.x;
        x0[4 * i + 1] = wv.y + sa * bv.y;
        x0[4 * i + 2] = wv.z + sa * bv.z;
        x0[4 * i + 3] = wv.w + sa * bv.w;
        ss0[i] = x0[4 * i] * x0[4 * i] + x0[4 * i + 1] * x0[4 * i + 1] + x0[4 * i + 2] * x0[4 * i + 2] +
                 x0[4 * i + 3] * x0[4 * i + 3];
      }
      const float inv0 = rsqrtf(warp_sum((ss0[0] + ss0[1]) + (ss0[2] + ss0[3])) / D + RMS_EPS);
#pragma unroll
      for (int i = 0; i < 16; ++i) x0[i] *= inv0;
      // mixing, eggroll.py:77-79
      const float resid = p.resid_l[p.layer] + sg * p.n_resid.A(j)[p.layer];
      const float mix = p.x0_l[p.layer] + sg * p.n_x0.A(j)[p.layer];
      if (p.layer == 0) {
#pragma unroll
        for (int i = 0; i < 16; ++i) x[i] = resid * x0[i] + mix * x0[i];
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 xv = *reinterpret_cast<const float4*>(xrow + 4 * lane + 128 * i);
          x[4 * i + 0] = resid * xv.x + mix * x0[4 * i + 0];
          x[4 * i + 1] = resid * xv.y + mix * x0[4 * i + 1];
          x[4 * i + 2] = resid * xv.z + mix * x0[4 * i + 2];
          x[4 * i + 3] = resid * xv.w + mix * x0[4 * i + 3];
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
        *reinterpret_cast<float4*>(xrow + 4 * lane + 128 * i) =
            make_float4(x[4 * i + 0], x[4 * i + 1], x[4 * i + 2], x[4 * i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 xv = *reinterpret_cast<const float4*>(xrow + 4 * lane + 128 * i);
        x[4 * i + 0] = xv.x;
        x[4 * i + 1] = xv.y;
        x[4 * i + 2] = xv.z;
        x[4 * i + 3] = xv.w;
      }
    }

    // h = norm(x) in fp32, rounded to bf16 as autocast feeds it to the matmuls
    float ss4[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      ss4[i] = x[4 * i] * x[4 * i] + x[4 * i + 1] * x[4 * i + 1] + x[4 * i + 2] * x[4 * i + 2] +
               x[4 * i + 3] * x[4 * i + 3];
    const float inv = rsqrtf(warp_sum((ss4[0] + ss4[1]) + (ss4[2] + ss4[3])) / D + RMS_EPS);
    float hb[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) hb[i] = bf16_round(x[i] * inv);
    __nv_bfloat16* hrow = p.h + static_cast<int64_t>(r) * D;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint2 pk;
      pk.x = pack_bf16x2(hb[4 * i + 0], hb[4 * i + 1]);
      pk.y = pack_bf16x2(hb[4 * i + 2], hb[4 * i + 3]);
      *reinterpret_cast<uint2*>(hrow + 4 * lane + 128 * i) = pk;
    }

    float* sv = p.svec + static_cast<int64_t>(r) * 4;
    if (MODE == NORM_BLOCK) {
      const float sq = dot_staged(hb, sb[0], lane);
      const float sk = dot_staged(hb, sb[1], lane);
      const float svv = dot_staged(hb, sb[2], lane);
      float sgate = 0.f;
      if (p.wgate) {
        // value-embedding gate 2 sigmoid(lowrank(h[:32], W_g, a, b)), eggroll.py:88; h[:32] lives in lanes 0..7
        // (i = 0): lane l < 8 holds h[4 l .. 4 l + 3]
        const float* ag = p.n_gate.A(j);
        float part[H + 1];
#pragma unroll
        for (int hh = 0; hh <= H; ++hh) {
          part[hh] = 0.f;
          if (lane < 8) {
            const float4 wv = *reinterpret_cast<const float4*>(sgw + hh * 32 + 4 * lane);
            part[hh] = hb[0] * wv.x + hb[1] * wv.y + hb[2] * wv.z + hb[3] * wv.w;
          }
        }
        // nine 8-lane sums at once
#pragma unroll
        for (int o = 4; o > 0; o >>= 1)
#pragma unroll
          for (int hh = 0; hh <= H; ++hh) part[hh] += __shfl_xor_sync(0xffffffffu, part[hh], o);
        sgate = bf16_round(__shfl_sync(0xffffffffu, part[H], 0));
        float gsel = 0.f;
#pragma unroll
        for (int hh = 0; hh < H; ++hh) {
          const float z = bf16_round(__shfl_sync(0xffffffffu, part[hh], 0)) + sg * sgate * ag[hh];
          if (lane == hh) gsel = 2.f / (1.f + __expf(-z));
        }
        if (lane < H) p.gate[static_cast<int64_t>(r) * H + lane] = gsel;
      }
      if (lane == 0) *reinterpret_cast<float4*>(sv) = make_float4(sq, sk, svv, sgate);
    } else {
      const float s0 = dot_staged(hb, sb[0], lane);
      if (lane == 0) sv[0] = s0;
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// GEMM epilogues
// ---------------------------------------------------------------------------------------------------------------
// Warp staging tile: 32 rows x 128 bytes, 16-byte chunk c of row r stored at chunk c ^ (r % 8) (conflict-free both
// when a thread writes its own row and when 8 lanes read one row). Rows of a warp's chunk are consecutive rows of the
// GEMM output, so after staging, lane L handles chunk L % 8 of rows L / 8 + 4 i: every global access of the warp
// covers 4 whole rows of 128 bytes (4 cache lines) instead of 32 lines.
__device__ __forceinline__ uint32_t stg_addr(uint32_t stg, int r, int c) {
  return stg + static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}
__device__ __forceinline__ void sts128(uint32_t a, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a) : "memory");
  return v;
}

// q, k: + sign (h.b) a, RoPE (utils/model.py:55-58), RMS norm over the head; v: + sign (h.b) a + gate ve
// (eggroll.py:82-90). Writes bf16 [m, H, T, 64].
struct EpiQKV {
  static constexpr int CH = 64;
  static constexpr bool PIPELINED = false;
  int T;
  const float* sign;
  const float* svec;
  const float* gate;  // NULL on blocks without value embeddings
  const int64_t* idx;
  int64_t row_stride;
  const __nv_bfloat16* cosb;
  const __nv_bfloat16* sinb;
  const float* vew;  // value-embedding table [4096, 512] fp32, or (ve_rows) one row per output row, or NULL
  int ve_rows;       // vew holds the value embedding of each row (Dust's captured rows): no token gather, no noise
  Slice nq, nk, nv, nve;
  __nv_bfloat16* q;
  __nv_bfloat16* k;
  __nv_bfloat16* v;
  int j, t, col0;
  float sg;
  float* scratch;
  uint32_t stg;

  __device__ __forceinline__ void row_begin(int row, int) {
    j = row / T;
    t = row - j * T;
    sg = sign[j];
  }
  // the tile's slice of a (q, k or v section) into shared memory
  __device__ __forceinline__ void stage(int row0, int c0, float* s, int tid) {
    col0 = c0;
    const int jj = row0 / T, sec = c0 / D;
    const float* a = (sec == 0 ? nq.A(jj) : sec == 1 ? nk.A(jj) : nv.A(jj)) + (c0 % D);
    s[tid] = a[tid];
  }
  __device__ __forceinline__ void tile_end(int, int, int) {}
  __device__ __forceinline__ void row_end(int, int) {}
  __device__ __forceinline__ void chunk(int row, int col, float* val) {
    const int sec = col / D, hh = (col % D) / HD;
    const float coef = sg * svec[static_cast<int64_t>(row) * 4 + sec];
    const float2 coef2 = make_float2(coef, coef);
    const float4* a4 = reinterpret_cast<const float4*>(scratch + (col - col0));
    // columns in pairs: one packed bf16 conversion per rounding (its fp32 values are the halves shifted back) and
    // fp32x2 FMAs, with the rounding of scalar ones
#pragma unroll
    for (int d = 0; d < HD; d += 4) {
      const float4 av = a4[d / 4];
      const float2 u0 = __ffma2_rn(coef2, make_float2(av.x, av.y), unpack_bf16x2(pack_bf16x2(val[d], val[d + 1])));
      const float2 u1 =
          __ffma2_rn(coef2, make_float2(av.z, av.w), unpack_bf16x2(pack_bf16x2(val[d + 2], val[d + 3])));
      val[d + 0] = u0.x;
      val[d + 1] = u0.y;
      val[d + 2] = u1.x;
      val[d + 3] = u1.y;
    }
    __nv_bfloat16* dst;
    if (sec < 2) {
      const uint4* cr = reinterpret_cast<const uint4*>(cosb + static_cast<int64_t>(t) * (HD / 2));
      const uint4* sr = reinterpret_cast<const uint4*>(sinb + static_cast<int64_t>(t) * (HD / 2));
      float ss4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int g = 0; g < 4; ++g) {  // 8 rotary pairs per 16-byte load of the bf16 tables
        const uint4 cv = cr[g], sv = sr[g];
        const __nv_bfloat162* c2 = reinterpret_cast<const __nv_bfloat162*>(&cv);
        const __nv_bfloat162* s2 = reinterpret_cast<const __nv_bfloat162*>(&sv);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int d = 8 * g + e;
          const float c = e & 1 ? __high2float(c2[e >> 1]) : __low2float(c2[e >> 1]);
          const float s = e & 1 ? __high2float(s2[e >> 1]) : __low2float(s2[e >> 1]);
          const float x1 = val[d], x2 = val[d + HD / 2];
          const float o1 = x1 * c + x2 * s;
          const float o2 = x1 * -s + x2 * c;
          val[d] = o1;
          val[d + HD / 2] = o2;
          ss4[e & 3] += o1 * o1 + o2 * o2;
        }
      }
      const float inv = rsqrtf(((ss4[0] + ss4[1]) + (ss4[2] + ss4[3])) / HD + RMS_EPS);
      const float2 inv2 = make_float2(inv, inv);
#pragma unroll
      for (int d = 0; d < HD; d += 2) {
        const float2 w = __fmul2_rn(make_float2(val[d], val[d + 1]), inv2);
        val[d] = w.x;
        val[d + 1] = w.y;
      }
      dst = sec == 0 ? q : k;
    } else {
      if (gate) {
        const float g = gate[static_cast<int64_t>(row) * H + hh];
        if (ve_rows) {
          const float4* vr = reinterpret_cast<const float4*>(vew + static_cast<int64_t>(row) * D + hh * HD);
#pragma unroll
          for (int d4 = 0; d4 < HD / 4; ++d4) {
            const float4 w4 = vr[d4];
            val[4 * d4 + 0] += g * w4.x;
            val[4 * d4 + 1] += g * w4.y;
            val[4 * d4 + 2] += g * w4.z;
            val[4 * d4 + 3] += g * w4.w;
          }
          dst = v;
          goto staged;
        }
        const int64_t tok = idx[j * row_stride + t];
        const float4* ver = reinterpret_cast<const float4*>(vew + tok * D + hh * HD);
        const float sa = sg * nve.A(j)[tok];
        const float* __restrict__ bve = nve.B(j) + hh * HD;
#pragma unroll
        for (int d4 = 0; d4 < HD / 4; ++d4) {
          const float4 w4 = ver[d4];
          val[4 * d4 + 0] += g * (w4.x + sa * bve[4 * d4 + 0]);
          val[4 * d4 + 1] += g * (w4.y + sa * bve[4 * d4 + 1]);
          val[4 * d4 + 2] += g * (w4.z + sa * bve[4 * d4 + 2]);
          val[4 * d4 + 3] += g * (w4.w + sa * bve[4 * d4 + 3]);
        }
      }
      dst = v;
    }
  staged:
    // this thread's head row (128 bytes) -> staging; then rows t0 .. t0 + 31 of the head, 4 per instruction
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int d = 0; d < HD; d += 8)
      sts128(stg_addr(stg, lane, d / 8), make_uint4(pack_bf16x2(val[d], val[d + 1]), pack_bf16x2(val[d + 2], val[d + 3]),
                                                   pack_bf16x2(val[d + 4], val[d + 5]), pack_bf16x2(val[d + 6], val[d + 7])));
    __syncwarp();
    uint4* out = reinterpret_cast<uint4*>(dst + ((static_cast<int64_t>(j) * H + hh) * T + (t - lane)) * HD);
    const int c = lane & 7;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = (lane >> 3) + 4 * i;
      out[r * 8 + c] = lds128(stg_addr(stg, r, c));
    }
    __syncwarp();
  }
};

// x += bf16(acc) + sign bf16(sum of the row's partial dots) a  (c_proj and mlp.c_proj, eggroll.py:92-93).
struct EpiResid {
  static constexpr int CH = 64;
  static constexpr bool PIPELINED = false;
  int T, nparts;
  const float* sign;
  const float* parts;  // [M, nparts] partial dots of the input row with this linear's b
  const float* jit;    // [M, 512] fp32 added to the linear's output, or NULL (Dust's attn / mlp jitter sites)
  Slice n;
  float* x;
  float coef;
  int col0;
  float* scratch;
  uint32_t stg;

  __device__ __forceinline__ void row_begin(int row, int) {
    const int j = row / T;
    const float* pr = parts + static_cast<int64_t>(row) * nparts;
    float s = 0.f;
    for (int i = 0; i < nparts; ++i) s += pr[i];
    coef = sign[j] * bf16_round(s);
  }
  __device__ __forceinline__ void stage(int row0, int c0, float* s, int tid) {
    col0 = c0;
    s[tid] = n.A(row0 / T)[c0 + tid];
  }
  __device__ __forceinline__ void tile_end(int, int, int) {}
  __device__ __forceinline__ void row_end(int, int) {}
  __device__ __forceinline__ void chunk(int row, int col, float* acc) {
    const int lane = threadIdx.x & 31, c = lane & 7;
    // x of rows row - lane .. + 31, columns col .. col + 63 (two 32-column halves, 4 whole 128-byte row segments per
    // instruction): every load is issued first, so the warp has 8 KB of the residual stream in flight while it
    // forms y (the epilogue is bound by the latency of these loads)
    float4* xr = reinterpret_cast<float4*>(x + static_cast<int64_t>(row - lane) * D + col) + c;
    float4 xv[16];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int i = 0; i < 8; ++i) xv[8 * h + i] = xr[((lane >> 3) + 4 * i) * (D / 4) + 8 * h];
    const float4* a4 = reinterpret_cast<const float4*>(scratch + (col - col0));
    const float2 coef2 = make_float2(coef, coef);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      // the linear's output for this thread's row (32 columns, 128 bytes) -> staging; columns in pairs: one packed
      // bf16 conversion per rounding and fp32x2 FMAs, with the rounding of scalar ones
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 av = a4[8 * h + i];
        const float* ac = acc + 32 * h + 4 * i;
        float2 y0 = __ffma2_rn(coef2, make_float2(av.x, av.y), unpack_bf16x2(pack_bf16x2(ac[0], ac[1])));
        float2 y1 = __ffma2_rn(coef2, make_float2(av.z, av.w), unpack_bf16x2(pack_bf16x2(ac[2], ac[3])));
        if (jit) {
          const float4 jv =
              *reinterpret_cast<const float4*>(jit + static_cast<int64_t>(row) * D + col + 32 * h + 4 * i);
          y0 = __fadd2_rn(y0, make_float2(jv.x, jv.y));
          y1 = __fadd2_rn(y1, make_float2(jv.z, jv.w));
        }
        sts128(stg_addr(stg, lane, i), make_uint4(__float_as_uint(y0.x), __float_as_uint(y0.y),
                                                  __float_as_uint(y1.x), __float_as_uint(y1.y)));
      }
      __syncwarp();
      // x += y for rows row - lane .. + 31
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = (lane >> 3) + 4 * i;
        const uint4 yv = lds128(stg_addr(stg, r, c));
        const float4 xo = xv[8 * h + i];
        const float2 s0 =
            __fadd2_rn(make_float2(xo.x, xo.y), make_float2(__uint_as_float(yv.x), __uint_as_float(yv.y)));
        const float2 s1 =
            __fadd2_rn(make_float2(xo.z, xo.w), make_float2(__uint_as_float(yv.z), __uint_as_float(yv.w)));
        xr[r * (D / 4) + 8 * h] = make_float4(s0.x, s0.y, s1.x, s1.y);
      }
      __syncwarp();
    }
  }
};

// hidden = bf16(relu(bf16(acc) + sign bf16(h.b_fc) a_fc)^2), and per N tile the partial dot hidden.b_mproj
// (the next linear's rank-1 input dot), eggroll.py:93.
template <bool JIT>
struct EpiFCImpl {
  static constexpr int CH = 64;
  static constexpr bool PIPELINED = true;
  static constexpr int NPARTS = 2 * (F / GEMM_BN);  // per row: one partial dot per (N tile, column half)
  int T;
  const float* sign;
  const float* svec;
  Slice nfc, nmp;
  __nv_bfloat16* hidden;
  const float* jit;  // JIT: [M, 2048] fp32 added to the pre-activation (Dust's fc jitter site)
  float* pdot;  // [M, NPARTS]
  float coef;
  float2 pd[4];  // eight partial sums (independent FMA chains), updated two at a time by packed fp32x2 FMAs
  int col0;
  float* scratch;
  uint32_t stg;

  __device__ __forceinline__ void row_begin(int row, int) {
    const int j = row / T;
    coef = sign[j] * svec[static_cast<int64_t>(row) * 4];
#pragma unroll
    for (int i = 0; i < 4; ++i) pd[i] = make_float2(0.f, 0.f);
  }
  // the tile's slices of a_fc and of the bf16-rounded b of mlp.c_proj into shared memory
  __device__ __forceinline__ void stage(int row0, int c0, float* s, int tid) {
    col0 = c0;
    const int j = row0 / T;
    s[tid] = nfc.A(j)[c0 + tid];
    s[GEMM_BN + tid] = bf16_round(nmp.B(j)[c0 + tid]);
  }
  __device__ __forceinline__ void tile_end(int row, int nb, int part) {
    pdot[static_cast<int64_t>(row) * NPARTS + 2 * nb + part] =
        ((pd[0].x + pd[0].y) + (pd[1].x + pd[1].y)) + ((pd[2].x + pd[2].y) + (pd[3].x + pd[3].y));
#pragma unroll
    for (int i = 0; i < 4; ++i) pd[i] = make_float2(0.f, 0.f);
  }
  __device__ __forceinline__ void row_end(int, int) {}
  // Columns in pairs: each bf16 rounding is one packed conversion (its fp32 values are the halves shifted back), and
  // the rank-1 term, the square and the partial dots are packed fp32x2 operations with the rounding of scalar ones.
  __device__ __forceinline__ void chunk(int row, int col, float* acc) {
    const int lane = threadIdx.x & 31;
    const float* ap = scratch + (col - col0);
    const float* bp = ap + GEMM_BN;
    const float2 coef2 = make_float2(coef, coef);
#pragma unroll
    for (int i = 0; i < CH; i += 8) {
      uint32_t pk[4];
      const float4 a0 = *reinterpret_cast<const float4*>(ap + i), a1 = *reinterpret_cast<const float4*>(ap + i + 4);
      const float4 b0 = *reinterpret_cast<const float4*>(bp + i), b1 = *reinterpret_cast<const float4*>(bp + i + 4);
      const float2 av[4] = {make_float2(a0.x, a0.y), make_float2(a0.z, a0.w), make_float2(a1.x, a1.y),
                            make_float2(a1.z, a1.w)};
      const float2 bv[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w), make_float2(b1.x, b1.y),
                            make_float2(b1.z, b1.w)};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float2 u = __ffma2_rn(coef2, av[e], unpack_bf16x2(pack_bf16x2(acc[i + 2 * e], acc[i + 2 * e + 1])));
        if constexpr (JIT) {
          const float* jp = jit + static_cast<int64_t>(row) * F + col + i + 2 * e;
          u = __fadd2_rn(u, make_float2(jp[0], jp[1]));
        }
        const float2 rl = make_float2(fmaxf(u.x, 0.f), fmaxf(u.y, 0.f));
        pk[e] = pack_bf16x2_f2(__fmul2_rn(rl, rl));
        pd[e] = __ffma2_rn(unpack_bf16x2(pk[e]), bv[e], pd[e]);
      }
      sts128(stg_addr(stg, lane, i / 8), make_uint4(pk[0], pk[1], pk[2], pk[3]));
    }
    __syncwarp();
    // rows row - lane .. + 31 of hidden, columns col .. col + CH - 1: whole CH * 2-byte row segments, NC 16-byte
    // pieces per row, 32 / NC rows per instruction
    constexpr int NC = CH / 8;
    uint4* out = reinterpret_cast<uint4*>(hidden + static_cast<int64_t>(row - lane) * F + col);
    const int c = lane % NC;
#pragma unroll
    for (int k = 0; k < NC; ++k) {
      const int rr = lane / NC + (32 / NC) * k;
      out[rr * (F / 8) + c] = lds128(stg_addr(stg, rr, c));
    }
    __syncwarp();
  }
};
using EpiFC = EpiFCImpl<false>;     // the population forward
using EpiFCJit = EpiFCImpl<true>;   // Dust's block rerun with an fc jitter site

// LM head: z = bf16(acc) + sign bf16(h.b) a; c = 15 tanh(z / 15); per row the cross-entropy
// log sum_v exp(c_v) - c_target (eggroll.py:96-102). Since c <= 15, exp(c - 15) never overflows, so the
// log-sum-exp needs no running maximum.
struct EpiHeadCE {
  static constexpr int CH = 32;
  static constexpr bool PIPELINED = false;
  int T;
  const float* sign;
  const float* svec;
  const int64_t* targets;  // member j, position t: targets[j * row_stride + t]
  int64_t row_stride;
  Slice n;
  float2* ce2;  // [M, 2]: per column half, (sum exp(c - 15), c_target or 0)
  int64_t tgt;
  float coef, sum, zt;
  int col0;
  float* scratch;
  uint32_t stg;

  __device__ __forceinline__ void row_begin(int row, int) {
    const int j = row / T;
    tgt = targets[j * row_stride + (row - j * T)];
    coef = sign[j] * svec[static_cast<int64_t>(row) * 4];
    sum = 0.f;
    zt = 0.f;
  }
  __device__ __forceinline__ void stage(int row0, int c0, float* s, int tid) {
    col0 = c0;
    s[tid] = n.A(row0 / T)[c0 + tid];
  }
  __device__ __forceinline__ void tile_end(int, int, int) {}
  __device__ __forceinline__ void row_end(int row, int part) { ce2[static_cast<int64_t>(row) * 2 + part] = make_float2(sum, zt); }
  // With u = e^(2 z / 15): 15 tanh(z / 15) - 15 = -30 / (u + 1), so exp(c - 15) = 2^(-30 log2(e) / (u + 1)): one
  // ex2 and one reciprocal, then the outer 2^x: three MUFU operations (an FMA-polynomial 2^x measured slower).
  // c itself is only needed at the target column: c = 15 - 30 / (u + 1).
  __device__ __forceinline__ void chunk(int, int col, float* acc) {
    const float4* a4 = reinterpret_cast<const float4*>(scratch + (col - col0));
#pragma unroll
    for (int i = 0; i < CH; i += 4) {
      const float4 av = a4[i / 4];
      const float aa[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float z = bf16_round_alu(acc[i + e]) + coef * aa[e];
        const float inv = rcp_approx(ex2_approx(z * (2.f / 15.f * LOG2E)) + 1.f);  // 1 / (u + 1)
        sum += ex2_approx(inv * (-30.f * LOG2E));
        if (col + i + e == tgt) zt = 15.f - 30.f * inv;
      }
    }
  }
};

// Plain fp32 store of the accumulator: D[row, col] = acc (the tcgen05 core without any fused arithmetic).
// Plain store of D (fp32, row-major, leading dimension ldd) for rows < m and columns < n: the M and N tails of a
// GEMM whose last tiles reach past the operands (TMA fills those operand rows with zeros).
struct EpiStore {
  static constexpr int CH = 32;
  static constexpr bool PIPELINED = false;
  float* d;
  int ldd, m, n;
  float* scratch;
  uint32_t stg;
  __device__ __forceinline__ void stage(int, int, float*, int) {}
  __device__ __forceinline__ void row_begin(int, int) {}
  __device__ __forceinline__ void tile_end(int, int, int) {}
  __device__ __forceinline__ void row_end(int, int) {}
  __device__ __forceinline__ void chunk(int row, int col, float* acc) {
    if (row >= m || col >= n) return;  // n % CH == 0: a chunk is wholly inside or outside
    float4* out = reinterpret_cast<float4*>(d + static_cast<int64_t>(row) * ldd + col);
#pragma unroll
    for (int i = 0; i < CH / 4; ++i) out[i] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
  }
};

// ---------------------------------------------------------------------------------------------------------------
// Windowed causal attention (mma.sync m16n8k16 bf16, FA2-style online softmax).
// q, k, v: bf16 [m*H, T, 64]; key s visible to query t iff 0 <= t - s <= window (utils/model.py:17-21).
// Writes y bf16 [M, 512] (row j*T + t, columns h*64 + d) and ydot[row, h] = sum_d bf16(y) bf16(b_cproj).
// ---------------------------------------------------------------------------------------------------------------
constexpr int ATT_BQ = 64, ATT_BK = 64;

struct AttnArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  __nv_bfloat16* y;
  float* ydot;
  int T, window;
  Slice nproj;  // c_proj noise (b used)
};

__device__ __forceinline__ void load_tile_async(uint32_t sbase, const __nv_bfloat16* g, int tid) {
  // 64 rows x 128 B = 512 16-byte chunks, 128 threads x 4
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = tid + 128 * i;
    const int row = c >> 3, ch = c & 7;
    cp_async16(sbase + swz(row, ch), g + row * 64 + ch * 8);
  }
}

__global__ void __launch_bounds__(128) attention_kernel(AttnArgs p) {
  __shared__ __align__(128) uint8_t smem[ATT_BQ * 128 + 4 * ATT_BK * 128];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_qt = p.T / ATT_BQ;
  const int qt = n_qt - 1 - blockIdx.x;  // heaviest tiles first
  const int bh = blockIdx.y;             // member * H + head
  const int j = bh / H, hh = bh - j * H;
  const int q0 = qt * ATT_BQ;
  const int64_t base = static_cast<int64_t>(bh) * p.T * HD;
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK[2] = {sQ + ATT_BQ * 128, sQ + ATT_BQ * 128 + ATT_BK * 128};
  const uint32_t sV[2] = {sQ + ATT_BQ * 128 + 2 * ATT_BK * 128, sQ + ATT_BQ * 128 + 3 * ATT_BK * 128};

  const int lo = q0 - p.window >= 0 ? (q0 - p.window) / ATT_BK : 0;  // window % 64 == 0
  const int hi = q0 / ATT_BK;

  load_tile_async(sQ, p.q + base + static_cast<int64_t>(q0) * HD, tid);
  load_tile_async(sK[0], p.k + base + static_cast<int64_t>(lo) * ATT_BK * HD, tid);
  load_tile_async(sV[0], p.v + base + static_cast<int64_t>(lo) * ATT_BK * HD, tid);
  cp_async_commit();

  float o[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  uint32_t qf[4][4];
  const float sl2 = 0.125f * LOG2E;
  const int r_lo = warp * 16 + (lane >> 2);  // this thread's rows within the q tile: r_lo, r_lo + 8

  for (int kt = lo; kt <= hi; ++kt) {
    const int buf = (kt - lo) & 1;
    if (kt < hi) {
      load_tile_async(sK[buf ^ 1], p.k + base + static_cast<int64_t>(kt + 1) * ATT_BK * HD, tid);
      load_tile_async(sV[buf ^ 1], p.v + base + static_cast<int64_t>(kt + 1) * ATT_BK * HD, tid);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (kt == lo) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int row = warp * 16 + (lane & 15), ch = kk * 2 + (lane >> 4);
        ldsm_x4(sQ + swz(row, ch), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    // S = Q K^T: 16 rows x 64 keys per warp
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // pairs of 8-key tiles
        const int key = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int ch = kk * 2 + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(sK[buf] + swz(key, ch), b0, b1, b2, b3);
        mma_bf16(s[2 * np], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
        mma_bf16(s[2 * np + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b2, b3);
      }
    }
    // masks: diagonal tile (key <= query) and the window's first tile (query - key <= window)
    const bool diag = kt == hi, edge = (q0 - p.window >= 0) && kt == lo;
    if (diag || edge) {
#pragma unroll
      for (int n = 0; n < 8; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int rq = r_lo + ((e >> 1) << 3);
          const int key = n * 8 + ((lane & 3) << 1) + (e & 1);
          const int tq = q0 + rq, sk = kt * ATT_BK + key;
          if (sk > tq || tq - sk > p.window) s[n][e] = -INFINITY;
        }
    }
    // online softmax (base 2)
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float mx = -INFINITY;
#pragma unroll
      for (int n = 0; n < 8; ++n) mx = fmaxf(mx, fmaxf(s[n][2 * hr], s[n][2 * hr + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mnew = fmaxf(mrow[hr], mx);
      const float msafe = mnew == -INFINITY ? 0.f : mnew;
      const float scale = ex2_approx((mrow[hr] - msafe) * sl2);
      mrow[hr] = mnew;
      float rs = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        s[n][2 * hr] = ex2_approx((s[n][2 * hr] - msafe) * sl2);
        s[n][2 * hr + 1] = ex2_approx((s[n][2 * hr + 1] - msafe) * sl2);
        rs += s[n][2 * hr] + s[n][2 * hr + 1];
        o[n][2 * hr] *= scale;
        o[n][2 * hr + 1] *= scale;
      }
      lrow[hr] = lrow[hr] * scale + rs;
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {  // 16 keys per step
      const uint32_t a0 = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      const uint32_t a1 = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      const uint32_t a2 = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      const uint32_t a3 = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // pairs of 8-dim tiles
        const int key = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int ch = np * 2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(sV[buf] + swz(key, ch), b0, b1, b2, b3);
        mma_bf16(o[2 * np], a0, a1, a2, a3, b0, b1);
        mma_bf16(o[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();
  }

  // epilogue: normalise, bf16, y and the c_proj rank-1 partial dot
  float lsum[2];
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    float l = lrow[hr];
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    lsum[hr] = 1.f / l;
  }
  const float* bproj = p.nproj.B(j) + hh * HD;
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int tq = q0 + r_lo + hr * 8;
    const int64_t row = static_cast<int64_t>(j) * p.T + tq;
    __nv_bfloat16* yr = p.y + row * D + hh * HD;
    float dp = 0.f;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int d = n * 8 + ((lane & 3) << 1);
      const float y0 = bf16_round(o[n][2 * hr] * lsum[hr]);
      const float y1 = bf16_round(o[n][2 * hr + 1] * lsum[hr]);
      *reinterpret_cast<uint32_t*>(yr + d) = pack_bf16x2(y0, y1);
      dp += y0 * bf16_round(bproj[d]) + y1 * bf16_round(bproj[d + 1]);
    }
    dp += __shfl_xor_sync(0xffffffffu, dp, 1);
    dp += __shfl_xor_sync(0xffffffffu, dp, 2);
    if ((lane & 3) == 0) p.ydot[row * H + hh] = dp;
  }
}

}  // namespace noise
#include "attention_tc.cuh"
namespace noise {

// ---------------------------------------------------------------------------------------------------------------
// Reductions of the per-row cross-entropy. Row r's loss is 15 + log(sum) - c_target from its two column halves'
// (sum exp(c - 15), c_target); a negative target (F.cross_entropy's ignore_index, -1 in GPT.forward) adds nothing.
// All sums run in a fixed order: the results are deterministic.
// ---------------------------------------------------------------------------------------------------------------
__device__ __forceinline__ float row_ce(float4 c) { return 15.f + logf(c.x + c.z) - (c.y + c.w); }

// out[j] = scale * sum of member j's token losses; cnt[j] (if given) = its number of counted tokens.
__global__ void __launch_bounds__(256) member_reduce_kernel(const float4* ce2, const int64_t* targets, int T,
                                                            int64_t row_stride, float scale, float* out, float* cnt) {
  __shared__ float part[8], npart[8];
  const int j = blockIdx.x;
  float s = 0.f, n = 0.f;
  for (int t = threadIdx.x; t < T; t += 256) {
    if (targets[j * row_stride + t] < 0) continue;
    s += row_ce(ce2[static_cast<int64_t>(j) * T + t]);
    n += 1.f;
  }
  s = warp_sum(s);
  n = warp_sum(n);
  if ((threadIdx.x & 31) == 0) {
    part[threadIdx.x >> 5] = s;
    npart[threadIdx.x >> 5] = n;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f, ntot = 0.f;
    for (int w = 0; w < 8; ++w) {
      tot += part[w];
      ntot += npart[w];
    }
    out[j] = tot * scale;
    if (cnt) cnt[j] = ntot;
  }
}

// reduction 'none': out[r] = loss of row r (0 for an ignored target).
__global__ void __launch_bounds__(256) token_loss_kernel(const float4* ce2, const int64_t* targets, int T,
                                                         int64_t row_stride, int64_t M, float* out) {
  for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; r < M;
       r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t j = r / T, t = r - j * T;
    out[r] = targets[j * row_stride + t] < 0 ? 0.f : row_ce(ce2[r]);
  }
}

// One scalar over all members (one block, fp64 accumulation): sum, or sum / counted tokens for the mean.
__global__ void __launch_bounds__(256) total_kernel(const float* sums, const float* cnt, int n, int mean, float* out) {
  __shared__ double part[8], npart[8];
  double s = 0.0, c = 0.0;
  for (int j = threadIdx.x; j < n; j += 256) {
    s += sums[j];
    c += cnt[j];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    c += __shfl_xor_sync(0xffffffffu, c, o);
  }
  if ((threadIdx.x & 31) == 0) {
    part[threadIdx.x >> 5] = s;
    npart[threadIdx.x >> 5] = c;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double tot = 0.0, ntot = 0.0;
    for (int w = 0; w < 8; ++w) {
      tot += part[w];
      ntot += npart[w];
    }
    out[0] = static_cast<float>(mean ? tot / ntot : tot);  // mean of no counted token: nan, as torch gives
  }
}

__global__ void pack_bf16_kernel(const float4* __restrict__ src, uint2* __restrict__ dst, int64_t n4) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float4 v = src[i];
    dst[i] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  }
}

__global__ void clear_status_kernel(int* status) { *status = 0; }

// ---------------------------------------------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// 2-D row-major [outer, inner] tensor of bf16 (or, f32, fp32) values, box [box_outer, 128 bytes] with 128-byte
// swizzle; reads past the tensor's edge fill with zeros.
static int make_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint32_t box_outer,
                    bool f32 = false) {
  auto fn = encode_fn();
  if (!fn) return NOISE_ERR_CUDA;
  const uint64_t es_bytes = f32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (inner * es_bytes) % 16) return NOISE_ERR_ALIGN;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {inner * es_bytes};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / es_bytes), box_outer};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NOISE_OK : NOISE_ERR_CUDA;
}

static int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return n;
}

static thread_local int g_launches = 0;
// Optional per-launch timing (noise_profile_start/stop): an event pair around every launch, labelled by kind.
enum LaunchKind {
  K_NORM_BLOCK, K_GEMM_QKV, K_ATTENTION, K_GEMM_PROJ, K_NORM_MID, K_GEMM_FC, K_GEMM_MPROJ, K_NORM_FINAL,
  K_GEMM_HEAD, K_REDUCE, K_GEMM_PLAIN, K_KINDS
};
struct Profiler {
  bool on = false;
  int capacity = 0, used = 0;
  cudaEvent_t* ev = nullptr;
  int* kind = nullptr;
};
static thread_local Profiler g_prof;
static thread_local int g_kind = 0;

static inline void launch_begin(cudaStream_t s, int kind) {
  g_kind = kind;
  if (g_prof.on && g_prof.used < g_prof.capacity) cudaEventRecord(g_prof.ev[2 * g_prof.used], s);
}
static inline void launch_end(cudaStream_t s) {
  if (g_prof.on && g_prof.used < g_prof.capacity) {
    cudaEventRecord(g_prof.ev[2 * g_prof.used + 1], s);
    g_prof.kind[g_prof.used++] = g_kind;
  }
  ++g_launches;
}

template <class Epi>
static int run_gemm(const void* A, int M, int K, const void* B, int N, const Epi& epi, int* status, cudaStream_t s,
                    int kind) {
  using L = GemmLayout<GEMM_BN, GEMM_STAGES>;
  if (M % GEMM_BM || N % GEMM_BN || K % GEMM_BK) return NOISE_ERR_SHAPE;
  CUtensorMap ma, mb;
  int rc = make_map(&ma, A, K, M, GEMM_BM);
  if (rc) return rc;
  rc = make_map(&mb, B, K, N, GEMM_BN);
  if (rc) return rc;
  auto kern = gemm_bf16_tn_kernel<GEMM_BN, GEMM_STAGES, Epi>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM_BYTES) != cudaSuccess)
    return NOISE_ERR_CUDA;
  const int m_tiles = M / GEMM_BM;
  int sms = sm_count();
  if (sms <= 0) return NOISE_ERR_CUDA;
  const int grid = m_tiles < sms ? m_tiles : sms;
  launch_begin(s, kind);
  kern<<<grid, GEMM_THREADS, L::SMEM_BYTES, s>>>(ma, mb, m_tiles, N / GEMM_BN, K / GEMM_BK, epi, status);
  launch_end(s);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

// D[m, n] = A[m, k] B[n, k]^T with a plain fp32 store, any m >= 1, n % 32 == 0 and k a whole number of 16 bytes:
// the last M / N / K tiles read zeros past the operands' edges and store only rows < m, columns < n.
template <bool TF32>
static int run_gemm_plain(const void* A, int M, int K, const void* B, int N, float* D, int* status, cudaStream_t s) {
  using L = GemmLayout<GEMM_BN, GEMM_STAGES>;
  constexpr int KE = TF32 ? GEMM_BK / 2 : GEMM_BK;
  if (M < 1 || N < 32 || N % 32 || K < 1) return NOISE_ERR_SHAPE;
  CUtensorMap ma, mb;
  int rc = make_map(&ma, A, K, M, GEMM_BM, TF32);
  if (rc) return rc;
  if ((rc = make_map(&mb, B, K, N, GEMM_BN, TF32))) return rc;
  EpiStore e{D, N, M, N};
  auto kern = gemm_bf16_tn_kernel<GEMM_BN, GEMM_STAGES, EpiStore, TF32>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM_BYTES) != cudaSuccess)
    return NOISE_ERR_CUDA;
  const int m_tiles = (M + GEMM_BM - 1) / GEMM_BM;
  int sms = sm_count();
  if (sms <= 0) return NOISE_ERR_CUDA;
  const int grid = m_tiles < sms ? m_tiles : sms;
  launch_begin(s, K_GEMM_PLAIN);
  kern<<<grid, GEMM_THREADS, L::SMEM_BYTES, s>>>(ma, mb, m_tiles, (N + GEMM_BN - 1) / GEMM_BN, (K + KE - 1) / KE, e,
                                                 status);
  launch_end(s);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

// attention_item's order for every attention launch: NOISE_B200_ATTN_ORDER "1" (head rows in per-CTA blocks) or "2"
// (head-major, items claimed from a launch-wide counter), else 0 (the launch-wide heaviest-first order)
static int attention_order() {
  static const int order = [] {
    const char* e = getenv("NOISE_B200_ATTN_ORDER");
    return e && (e[0] == '1' || e[0] == '2') && e[1] == '\0' ? e[0] - '0' : 0;
  }();
  return order;
}

static int run_attention(const void* q, const void* k, const void* v, int M, int T, int members,
                         const TAttnArgs& args, cudaStream_t s) {
  CUtensorMap mq, mk, mv;
  int rc;
  const uint64_t rows = static_cast<uint64_t>(M) * H;  // q, k, v are head-major [members * H * T, 64]
  if ((rc = make_map(&mq, q, HD, rows, TA_BQ)) || (rc = make_map(&mk, k, HD, rows, TA_BK)) ||
      (rc = make_map(&mv, v, HD, rows, TA_BK)))
    return rc;
  TAttnArgs a = args;
  a.bh = members * H;
  a.order = attention_order();
  const bool dyn = a.order == 2;
  auto kern = args.jit ? (dyn ? attention_tc_kernel<true, true> : attention_tc_kernel<true, false>)
                       : (dyn ? attention_tc_kernel<false, true> : attention_tc_kernel<false, false>);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, TA_SMEM) != cudaSuccess)
    return NOISE_ERR_CUDA;
  const int sms = sm_count();
  if (sms <= 0) return NOISE_ERR_CUDA;
  if (dyn) {  // the work counter: word 32 of the workspace's 256-byte status block (word 0 is the status)
    a.next_item = a.status + 32;
    if (cudaMemsetAsync(a.next_item, 0, sizeof(int), s) != cudaSuccess) return NOISE_ERR_CUDA;
  }
  launch_begin(s, K_ATTENTION);
  const int items = (T / TA_BQ + 1) / 2 * a.bh;
  kern<<<items < sms ? items : sms, TA_THREADS, TA_SMEM, s>>>(mq, mk, mv, a);
  launch_end(s);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

struct Workspace {
  int* status;
  float* x;
  __nv_bfloat16 *h, *q, *k, *v, *y, *hidden;
  float *svec, *gate, *ydot, *pdot;
  float2* ce2;
  float* zeros;   // V zero floats: the noise of the un-perturbed forward
  float* zsign;   // [members] zero signs
  float* msum;    // [members] per-member loss sums
  float* mcnt;    // [members] per-member counted tokens
  size_t bytes;
};

static size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

static Workspace carve(void* ws, int64_t M) {
  Workspace w{};
  size_t off = NOISE_STATUS_BYTES;
  auto take = [&](size_t n) {
    void* p = ws ? static_cast<uint8_t*>(ws) + off : nullptr;
    off += align256(n);
    return p;
  };
  w.status = static_cast<int*>(ws);
  w.x = static_cast<float*>(take(M * D * 4));
  w.h = static_cast<__nv_bfloat16*>(take(M * D * 2));
  w.q = static_cast<__nv_bfloat16*>(take(M * D * 2));
  w.k = static_cast<__nv_bfloat16*>(take(M * D * 2));
  w.v = static_cast<__nv_bfloat16*>(take(M * D * 2));
  w.y = static_cast<__nv_bfloat16*>(take(M * D * 2));
  w.hidden = static_cast<__nv_bfloat16*>(take(M * F * 2));
  w.svec = static_cast<float*>(take(M * 4 * 4));
  w.gate = static_cast<float*>(take(M * H * 4));
  w.ydot = static_cast<float*>(take(M * H * 4));
  w.pdot = static_cast<float*>(take(M * EpiFC::NPARTS * 4));
  w.ce2 = static_cast<float2*>(take(M * 2 * 8));
  const int64_t mmax = M / GEMM_BM + 1;  // rows per member >= 128
  w.zeros = static_cast<float*>(take(V * 4));
  w.zsign = static_cast<float*>(take(mmax * 4));
  w.msum = static_cast<float*>(take(mmax * 4));
  w.mcnt = static_cast<float*>(take(mmax * 4));
  w.bytes = off;
  return w;
}

// Scratch of noise_head_loss: the status word, h, the head dots, the cross-entropy halves and the zero noise.
static Workspace carve_head(void* ws, int64_t rows) {
  Workspace w{};
  size_t off = NOISE_STATUS_BYTES;
  auto take = [&](size_t n) {
    void* p = ws ? static_cast<uint8_t*>(ws) + off : nullptr;
    off += align256(n);
    return p;
  };
  w.status = static_cast<int*>(ws);
  w.h = static_cast<__nv_bfloat16*>(take(rows * D * 2));
  w.svec = static_cast<float*>(take(rows * 4 * 4));
  w.ce2 = static_cast<float2*>(take(rows * 2 * 8));
  w.zeros = static_cast<float*>(take(V * 4));
  w.zsign = static_cast<float*>(take(4));
  w.bytes = off;
  return w;
}

}  // namespace noise


using namespace noise;

extern "C" {

int noise_attention_item(int order, int item, int head_rows, int pairs, int grid, int* pair, int* head_row) {
  if (!pair || !head_row || order < 0 || order > 2) return NOISE_ERR_ARGUMENT;
  const int64_t items = static_cast<int64_t>(head_rows) * pairs;
  if (head_rows < 1 || pairs < 1 || items > 0x7FFFFFFF || grid < 1 || grid > items || item < 0 || item >= items)
    return NOISE_ERR_SHAPE;
  attention_item(order, item, head_rows, pairs, grid, *pair, *head_row);
  return NOISE_OK;
}

int noise_param_index(int block, int which) {
  if (block < 0 || block >= NOISE_N_LAYER) return -1;
  if (which == NOISE_P_VE) return (block & 1) ? 56 + block / 2 : -1;
  if (which == NOISE_P_VEGATE && !(block & 1)) return -1;
  int idx = 3;  // first block tensor
  for (int b = 0; b < block; ++b) idx += (b & 1) ? 7 : 6;
  static const int even[7] = {0, 1, 2, 3, -1, 4, 5};
  static const int odd[7] = {0, 1, 2, 3, 4, 5, 6};
  const int k = (block & 1) ? odd[which] : even[which];
  return k < 0 ? -1 : idx + k;
}

size_t noise_population_workspace_bytes(int members, int tokens) {
  if (members < 1 || tokens < 1) return 0;
  return carve(nullptr, static_cast<int64_t>(members) * tokens).bytes;
}

}  // extern "C"

namespace noise {

static int check_model(const noise_gpt_t* model) {
  for (int l = 0; l < NOISE_N_LAYER; ++l) {
    if (!model->wqkv[l] || !model->wproj[l] || !model->wfc[l] || !model->wmproj[l]) return NOISE_ERR_ARGUMENT;
    if ((l & 1) && (!model->wgate[l] || !model->ve[l])) return NOISE_ERR_ARGUMENT;
  }
  if (!model->whead || !model->wte || !model->resid_lambdas || !model->x0_lambdas || !model->cos || !model->sin)
    return NOISE_ERR_ARGUMENT;
  return NOISE_OK;
}

static int check_device() {
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NOISE_ERR_CUDA;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  return major == 10 ? NOISE_OK : NOISE_ERR_DEVICE;
}

// Checks shared by the whole-model entries: members x tokens rows, T a multiple of 128 up to the rotary tables' 2048.
static int check_forward(const noise_gpt_t* model, int members, int tokens, void* workspace, size_t workspace_bytes,
                         Workspace* w) {
  if (members < 1 || tokens < GEMM_BM || tokens > 2048 || tokens % GEMM_BM) return NOISE_ERR_SHAPE;
  const int64_t M = static_cast<int64_t>(members) * tokens;
  if (M > (int64_t(1) << 31) / F) return NOISE_ERR_SHAPE;
  *w = carve(workspace, M);
  if (!workspace || workspace_bytes < w->bytes) return NOISE_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return NOISE_ERR_ALIGN;
  const int rc = check_model(model);
  return rc ? rc : check_device();
}

// The perturbed forward up to the per-row cross-entropy halves in w.ce2: member j reads token row
// idx + j * row_stride (row_stride 0: one shared row, as eggroll.py:143), its noise from nz and its sign from sign.
static int run_forward(const noise_gpt_t* model, const noise_slice_t* nz, const float* sign, const int64_t* idx,
                       const int64_t* targets, int64_t row_stride, int members, int T, const Workspace& w,
                       cudaStream_t s) {
  const int64_t M = static_cast<int64_t>(members) * T;
  const int Mi = static_cast<int>(M);
  int rc;
  if (cudaMemsetAsync(w.status, 0, sizeof(int), s) != cudaSuccess) return NOISE_ERR_CUDA;
  const int norm_blocks = static_cast<int>((M + NORM_ROWS - 1) / NORM_ROWS);

  for (int l = 0; l < NOISE_N_LAYER; ++l) {
    const bool ve = l & 1;
    NormArgs na{};
    na.layer = l;
    na.T = T;
    na.M = Mi;
    na.idx = idx;
    na.row_stride = row_stride;
    na.sign = sign;
    na.x = w.x;
    na.h = w.h;
    na.svec = w.svec;
    na.gate = w.gate;
    na.wte = model->wte;
    na.n_wte = to_slice(nz[NOISE_PARAM_WTE]);
    na.n_resid = to_slice(nz[NOISE_PARAM_RESID]);
    na.n_x0 = to_slice(nz[NOISE_PARAM_X0]);
    na.resid_l = model->resid_lambdas;
    na.x0_l = model->x0_lambdas;
    na.nb0 = to_slice(nz[noise_param_index(l, NOISE_P_CQ)]);
    na.nb1 = to_slice(nz[noise_param_index(l, NOISE_P_CK)]);
    na.nb2 = to_slice(nz[noise_param_index(l, NOISE_P_CV)]);
    na.wgate = ve ? model->wgate[l] : nullptr;
    if (ve) na.n_gate = to_slice(nz[noise_param_index(l, NOISE_P_VEGATE)]);
    launch_begin(s, K_NORM_BLOCK);
    norm_kernel<NORM_BLOCK><<<norm_blocks, 256, 0, s>>>(na);
    launch_end(s);

    EpiQKV eq{};
    eq.T = T;
    eq.sign = sign;
    eq.svec = w.svec;
    eq.gate = ve ? w.gate : nullptr;
    eq.idx = idx;
    eq.row_stride = row_stride;
    eq.cosb = static_cast<const __nv_bfloat16*>(model->cos);
    eq.sinb = static_cast<const __nv_bfloat16*>(model->sin);
    eq.vew = ve ? model->ve[l] : nullptr;
    eq.nq = na.nb0;
    eq.nk = na.nb1;
    eq.nv = na.nb2;
    if (ve) eq.nve = to_slice(nz[noise_param_index(l, NOISE_P_VE)]);
    eq.q = w.q;
    eq.k = w.k;
    eq.v = w.v;
    if ((rc = run_gemm(w.h, Mi, D, model->wqkv[l], 3 * D, eq, w.status, s, K_GEMM_QKV))) return rc;

    TAttnArgs aa{};
    aa.T = T;
    aa.window = (l % 4 == 3 || l == NOISE_N_LAYER - 1) ? 2048 : 1024;  // SSSL, last block L
    aa.y = w.y;
    aa.ydot = w.ydot;
    aa.nproj = to_slice(nz[noise_param_index(l, NOISE_P_CPROJ)]);
    aa.status = w.status;
    if ((rc = run_attention(w.q, w.k, w.v, Mi, T, members, aa, s))) return rc;

    EpiResid er{};
    er.T = T;
    er.nparts = H;
    er.sign = sign;
    er.parts = w.ydot;
    er.n = aa.nproj;
    er.x = w.x;
    if ((rc = run_gemm(w.y, Mi, D, model->wproj[l], D, er, w.status, s, K_GEMM_PROJ))) return rc;

    NormArgs nm = na;
    nm.nb0 = to_slice(nz[noise_param_index(l, NOISE_P_CFC)]);
    launch_begin(s, K_NORM_MID);
    norm_kernel<NORM_MID><<<norm_blocks, 256, 0, s>>>(nm);
    launch_end(s);

    EpiFC ef{};
    ef.T = T;
    ef.sign = sign;
    ef.svec = w.svec;
    ef.nfc = nm.nb0;
    ef.nmp = to_slice(nz[noise_param_index(l, NOISE_P_MPROJ)]);
    ef.hidden = w.hidden;
    ef.pdot = w.pdot;
    if ((rc = run_gemm(w.h, Mi, D, model->wfc[l], F, ef, w.status, s, K_GEMM_FC))) return rc;

    EpiResid em{};
    em.T = T;
    em.nparts = EpiFC::NPARTS;
    em.sign = sign;
    em.parts = w.pdot;
    em.n = ef.nmp;
    em.x = w.x;
    if ((rc = run_gemm(w.hidden, Mi, F, model->wmproj[l], D, em, w.status, s, K_GEMM_MPROJ))) return rc;
  }

  NormArgs nf{};
  nf.T = T;
  nf.M = Mi;
  nf.idx = idx;
  nf.row_stride = row_stride;
  nf.sign = sign;
  nf.x = w.x;
  nf.h = w.h;
  nf.svec = w.svec;
  nf.nb0 = to_slice(nz[NOISE_PARAM_HEAD]);
  launch_begin(s, K_NORM_FINAL);
  norm_kernel<NORM_FINAL><<<norm_blocks, 256, 0, s>>>(nf);
  launch_end(s);

  EpiHeadCE eh{};
  eh.T = T;
  eh.sign = sign;
  eh.svec = w.svec;
  eh.targets = targets;
  eh.row_stride = row_stride;
  eh.n = nf.nb0;
  eh.ce2 = w.ce2;
  if ((rc = run_gemm(w.h, Mi, D, model->whead, V, eh, w.status, s, K_GEMM_HEAD))) return rc;

  return NOISE_OK;
}

// nz[i] = the zero noise (a = b = w.zeros for every member) and w.zsign = 0 for `members` members.
static int zero_noise(const Workspace& w, int members, noise_slice_t* nz, cudaStream_t s) {
  if (cudaMemsetAsync(w.zeros, 0, V * sizeof(float), s) != cudaSuccess) return NOISE_ERR_CUDA;
  if (cudaMemsetAsync(w.zsign, 0, members * sizeof(float), s) != cudaSuccess) return NOISE_ERR_CUDA;
  for (int i = 0; i < NOISE_N_PARAMS; ++i) nz[i] = noise_slice_t{w.zeros, w.zeros, nullptr, 0, 0};
  return NOISE_OK;
}

// reduction 'none': one loss per row into out[M]
static int token_losses(const Workspace& w, const int64_t* targets, int T, int64_t row_stride, int64_t M, float* out,
                        cudaStream_t s) {
  launch_begin(s, K_REDUCE);
  token_loss_kernel<<<static_cast<int>(std::min<int64_t>((M + 255) / 256, 148 * 16)), 256, 0, s>>>(
      reinterpret_cast<const float4*>(w.ce2), targets, T, row_stride, M, out);
  launch_end(s);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

}  // namespace noise

extern "C" {

int noise_population_loss(const noise_gpt_t* model, const noise_slice_t* nz, const float* sign, const int64_t* idx,
                          const int64_t* targets, int members, int tokens, int reduction, float* losses,
                          void* workspace, size_t workspace_bytes, void* stream) {
  if (!model || !nz || !sign || !idx || !targets || !losses) return NOISE_ERR_ARGUMENT;
  if (reduction != NOISE_REDUCTION_MEAN && reduction != NOISE_REDUCTION_SUM && reduction != NOISE_REDUCTION_NONE)
    return NOISE_ERR_ARGUMENT;
  Workspace w;
  int rc = check_forward(model, members, tokens, workspace, workspace_bytes, &w);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  g_launches = 0;
  if ((rc = run_forward(model, nz, sign, idx, targets, 0, members, tokens, w, s))) return rc;
  if (reduction == NOISE_REDUCTION_NONE)
    return token_losses(w, targets, tokens, 0, static_cast<int64_t>(members) * tokens, losses, s);
  launch_begin(s, K_REDUCE);
  member_reduce_kernel<<<members, 256, 0, s>>>(reinterpret_cast<const float4*>(w.ce2), targets, tokens, 0,
                                               reduction == NOISE_REDUCTION_MEAN ? 1.f / tokens : 1.f, losses,
                                               nullptr);
  launch_end(s);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

size_t noise_gpt_workspace_bytes(int rows, int tokens) { return noise_population_workspace_bytes(rows, tokens); }

int noise_gpt_loss(const noise_gpt_t* model, const int64_t* idx, const int64_t* targets, int rows, int tokens,
                   int reduction, float* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!model || !idx || !targets || !out) return NOISE_ERR_ARGUMENT;
  if (reduction != NOISE_REDUCTION_MEAN && reduction != NOISE_REDUCTION_SUM && reduction != NOISE_REDUCTION_NONE)
    return NOISE_ERR_ARGUMENT;
  Workspace w;
  int rc = check_forward(model, rows, tokens, workspace, workspace_bytes, &w);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  g_launches = 0;
  noise_slice_t nz[NOISE_N_PARAMS];
  if ((rc = zero_noise(w, rows, nz, s))) return rc;
  if ((rc = run_forward(model, nz, w.zsign, idx, targets, tokens, rows, tokens, w, s))) return rc;
  if (reduction == NOISE_REDUCTION_NONE)
    return token_losses(w, targets, tokens, tokens, static_cast<int64_t>(rows) * tokens, out, s);
  launch_begin(s, K_REDUCE);
  member_reduce_kernel<<<rows, 256, 0, s>>>(reinterpret_cast<const float4*>(w.ce2), targets, tokens, tokens, 1.f,
                                            w.msum, w.mcnt);
  total_kernel<<<1, 256, 0, s>>>(w.msum, w.mcnt, rows, reduction == NOISE_REDUCTION_MEAN, out);
  launch_end(s);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

size_t noise_head_loss_workspace_bytes(int rows) {
  if (rows < 1) return 0;
  return carve_head(nullptr, rows).bytes;
}

int noise_head_loss(const float* x, const void* weight, const int64_t* targets, int rows, float* out, void* workspace,
                    size_t workspace_bytes, void* stream) {
  if (!x || !weight || !targets || !out) return NOISE_ERR_ARGUMENT;
  if (rows < GEMM_BM || rows % GEMM_BM || rows > (1 << 22)) return NOISE_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(weight) & 15)) return NOISE_ERR_ALIGN;
  const Workspace w = carve_head(workspace, rows);
  if (!workspace || workspace_bytes < w.bytes) return NOISE_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return NOISE_ERR_ALIGN;
  int rc = check_device();
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  g_launches = 0;
  if (cudaMemsetAsync(w.status, 0, sizeof(int), s) != cudaSuccess) return NOISE_ERR_CUDA;
  noise_slice_t nz[NOISE_N_PARAMS];
  if ((rc = zero_noise(w, 1, nz, s))) return rc;
  // one "member" of `rows` rows; the final norm reads x in place (NORM_FINAL never writes it)
  NormArgs nf{};
  nf.T = rows;
  nf.M = rows;
  nf.sign = w.zsign;
  nf.x = const_cast<float*>(x);
  nf.h = w.h;
  nf.svec = w.svec;
  nf.nb0 = to_slice(nz[NOISE_PARAM_HEAD]);
  launch_begin(s, K_NORM_FINAL);
  norm_kernel<NORM_FINAL><<<(rows + NORM_ROWS - 1) / NORM_ROWS, 256, 0, s>>>(nf);
  launch_end(s);
  EpiHeadCE eh{};
  eh.T = rows;
  eh.sign = w.zsign;
  eh.svec = w.svec;
  eh.targets = targets;
  eh.row_stride = 0;
  eh.n = nf.nb0;
  eh.ce2 = w.ce2;
  if ((rc = run_gemm(w.h, rows, D, weight, V, eh, w.status, s, K_GEMM_HEAD))) return rc;
  return token_losses(w, targets, rows, 0, rows, out, s);
}

size_t noise_block_workspace_bytes(int seqs, int tokens) { return noise_population_workspace_bytes(seqs, tokens); }

int noise_block_forward(const noise_gpt_t* model, int layer, float* x, const float* ve, const noise_jitter_t* jit,
                        int seqs, int tokens, int window, void* workspace, size_t workspace_bytes, void* stream) {
  if (!model || !x || layer < 0 || layer >= NOISE_N_LAYER) return NOISE_ERR_ARGUMENT;
  if (!model->wqkv[layer] || !model->wproj[layer] || !model->wfc[layer] || !model->wmproj[layer] || !model->cos ||
      !model->sin)
    return NOISE_ERR_ARGUMENT;
  const bool gated = model->wgate[layer] != nullptr;
  if (gated != (ve != nullptr)) return NOISE_ERR_ARGUMENT;  // a value-embedding block takes its ve rows, others none
  if (seqs < 1 || tokens < GEMM_BM || tokens > 2048 || tokens % GEMM_BM || window < 0) return NOISE_ERR_SHAPE;
  const int64_t M = static_cast<int64_t>(seqs) * tokens;
  if (M > (int64_t(1) << 31) / F) return NOISE_ERR_SHAPE;
  const Workspace w = carve(workspace, M);
  if (!workspace || workspace_bytes < w.bytes) return NOISE_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (ve && (reinterpret_cast<uintptr_t>(ve) & 15)))
    return NOISE_ERR_ALIGN;
  int rc = check_device();
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int T = tokens, Mi = static_cast<int>(M);
  g_launches = 0;
  if (cudaMemsetAsync(w.status, 0, sizeof(int), s) != cudaSuccess) return NOISE_ERR_CUDA;
  noise_slice_t nz[NOISE_N_PARAMS];
  if ((rc = zero_noise(w, seqs, nz, s))) return rc;
  const Slice zs = to_slice(nz[0]);
  const int norm_blocks = static_cast<int>((M + NORM_ROWS - 1) / NORM_ROWS);
  const noise_jitter_t none{};
  const noise_jitter_t& j = jit ? *jit : none;

  NormArgs na{};
  na.layer = layer;
  na.T = T;
  na.M = Mi;
  na.sign = w.zsign;
  na.x = x;
  na.h = w.h;
  na.svec = w.svec;
  na.gate = w.gate;
  na.n_wte = na.n_resid = na.n_x0 = na.nb0 = na.nb1 = na.nb2 = na.n_gate = zs;
  na.wgate = gated ? model->wgate[layer] : nullptr;
  na.no_mix = 1;
  launch_begin(s, K_NORM_BLOCK);
  norm_kernel<NORM_BLOCK><<<norm_blocks, 256, 0, s>>>(na);
  launch_end(s);

  EpiQKV eq{};
  eq.T = T;
  eq.sign = w.zsign;
  eq.svec = w.svec;
  eq.gate = gated ? w.gate : nullptr;
  eq.cosb = static_cast<const __nv_bfloat16*>(model->cos);
  eq.sinb = static_cast<const __nv_bfloat16*>(model->sin);
  eq.vew = ve;
  eq.ve_rows = 1;
  eq.nq = eq.nk = eq.nv = eq.nve = zs;
  eq.q = w.q;
  eq.k = w.k;
  eq.v = w.v;
  if ((rc = run_gemm(w.h, Mi, D, model->wqkv[layer], 3 * D, eq, w.status, s, K_GEMM_QKV))) return rc;

  TAttnArgs aa{};
  aa.T = T;
  aa.window = window;
  aa.y = w.y;
  aa.ydot = w.ydot;
  aa.nproj = zs;
  aa.status = w.status;
  aa.jit = j.o;
  if ((rc = run_attention(w.q, w.k, w.v, Mi, T, seqs, aa, s))) return rc;

  EpiResid er{};
  er.T = T;
  er.nparts = H;
  er.sign = w.zsign;
  er.parts = w.ydot;
  er.n = zs;
  er.x = x;
  er.jit = j.attn;
  if ((rc = run_gemm(w.y, Mi, D, model->wproj[layer], D, er, w.status, s, K_GEMM_PROJ))) return rc;

  NormArgs nm = na;
  nm.wgate = nullptr;
  launch_begin(s, K_NORM_MID);
  norm_kernel<NORM_MID><<<norm_blocks, 256, 0, s>>>(nm);
  launch_end(s);

  auto fc_epi = [&](auto& ef) {
    ef.T = T;
    ef.sign = w.zsign;
    ef.svec = w.svec;
    ef.nfc = ef.nmp = zs;
    ef.hidden = w.hidden;
    ef.pdot = w.pdot;
    ef.jit = j.fc;
    return run_gemm(w.h, Mi, D, model->wfc[layer], F, ef, w.status, s, K_GEMM_FC);
  };
  if (j.fc) {
    EpiFCJit ef{};
    rc = fc_epi(ef);
  } else {
    EpiFC ef{};
    rc = fc_epi(ef);
  }
  if (rc) return rc;

  EpiResid em{};
  em.T = T;
  em.nparts = EpiFC::NPARTS;
  em.sign = w.zsign;
  em.parts = w.pdot;
  em.n = zs;
  em.x = x;
  em.jit = j.mlp;
  if ((rc = run_gemm(w.hidden, Mi, F, model->wmproj[layer], D, em, w.status, s, K_GEMM_MPROJ))) return rc;
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

// ---------------------------------------------------------------------------------------------------------------
// No-allocation variant of noise_population_loss. Its scratch is this file-scope device array, which every GPU that
// loads the library holds until the process exits. In host code `g_static_scratch` is only a host-side stand-in
// for the symbol, never a device address: its device address is looked up once per device with
// cudaGetSymbolAddress (with that device current) and only that address reaches the kernels.
// ---------------------------------------------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_static_scratch[NOISE_STATIC_SCRATCH_BYTES];
static void* g_static_scratch_addr[NOISE_STATIC_MAX_DEVICES];
static std::mutex g_static_scratch_mutex;

namespace noise {

// Device address of the current device's copy of g_static_scratch, after checking that `stream` belongs to that
// device (a stream of another device would run the kernels against the wrong GPU's array).
static int static_scratch(cudaStream_t stream, void** out) {
  int dev = 0, sdev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NOISE_ERR_CUDA;
  if (dev < 0 || dev >= NOISE_STATIC_MAX_DEVICES) return NOISE_ERR_ARGUMENT;
  if (cudaStreamGetDevice(stream, &sdev) != cudaSuccess) return NOISE_ERR_CUDA;
  if (sdev != dev) return NOISE_ERR_ARGUMENT;
  std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
  if (!g_static_scratch_addr[dev]) {  // first call on this device: resolve the array's device address
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_static_scratch) != cudaSuccess || !addr) return NOISE_ERR_CUDA;
    g_static_scratch_addr[dev] = addr;
  }
  *out = g_static_scratch_addr[dev];
  return NOISE_OK;
}

}  // namespace noise

int noise_population_loss_noalloc(const noise_gpt_t* model, const noise_slice_t* noise, const float* sign,
                                  const int64_t* idx, const int64_t* targets, int members, int tokens, int reduction,
                                  float* losses, void* stream) {
  const size_t need = noise_population_workspace_bytes(members, tokens);
  if (need == 0) return NOISE_ERR_SHAPE;
  if (need > NOISE_STATIC_SCRATCH_BYTES) return NOISE_ERR_TOO_LARGE;
  void* scratch = nullptr;
  const int rc = static_scratch(static_cast<cudaStream_t>(stream), &scratch);
  if (rc) return rc;
  // The status word at the head of the scratch is cleared by noise_population_loss itself; every other buffer is
  // fully written before it is read, so stale contents of an earlier call never leak into this one.
  return noise_population_loss(model, noise, sign, idx, targets, members, tokens, reduction, losses, scratch,
                               NOISE_STATIC_SCRATCH_BYTES, stream);
}

int noise_read_static_status(int* status, void* stream) {
  if (!status) return NOISE_ERR_ARGUMENT;
  void* scratch = nullptr;
  const int rc = static_scratch(static_cast<cudaStream_t>(stream), &scratch);
  if (rc) return rc;
  return noise_read_status(scratch, status, stream);
}

int noise_gemm_bf16_tn(const void* a, const void* b, float* d, int m, int n, int k, void* workspace,
                       void* stream) {
  if (!a || !b || !d || !workspace) return NOISE_ERR_ARGUMENT;
  if (m < 1 || n < 32 || n % 32 || k < 8 || k % 8) return NOISE_ERR_SHAPE;
  if (reinterpret_cast<uintptr_t>(d) & 15) return NOISE_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(workspace, 0, sizeof(int), s) != cudaSuccess) return NOISE_ERR_CUDA;
  g_launches = 0;
  return run_gemm_plain<false>(a, m, k, b, n, d, static_cast<int*>(workspace), s);
}

int noise_gemm_tf32_tn(const float* a, const float* b, float* d, int m, int n, int k, void* workspace,
                       void* stream) {
  if (!a || !b || !d || !workspace) return NOISE_ERR_ARGUMENT;
  if (m < 1 || n < 32 || n % 32 || k < 4 || k % 4) return NOISE_ERR_SHAPE;
  if (reinterpret_cast<uintptr_t>(d) & 15) return NOISE_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(workspace, 0, sizeof(int), s) != cudaSuccess) return NOISE_ERR_CUDA;
  g_launches = 0;
  return run_gemm_plain<true>(a, m, k, b, n, d, static_cast<int*>(workspace), s);
}

int noise_pack_bf16(const float* src, void* dst, int64_t n, void* stream) {
  if (!src || !dst || n < 0) return NOISE_ERR_ARGUMENT;
  if (n % 8 || (reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(dst) & 15))
    return NOISE_ERR_ALIGN;
  if (n == 0) return NOISE_OK;
  const int64_t n4 = n / 4;
  int blocks = static_cast<int>((n4 + 255) / 256);
  if (blocks > 148 * 16) blocks = 148 * 16;
  pack_bf16_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(reinterpret_cast<const float4*>(src),
                                                                           static_cast<uint2*>(dst), n4);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_read_status(const void* workspace, int* status, void* stream) {
  if (!workspace || !status) return NOISE_ERR_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(status, workspace, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess) return NOISE_ERR_CUDA;
  return cudaStreamSynchronize(s) == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_clear_status(void* workspace, void* stream) {
  if (!workspace) return NOISE_ERR_ARGUMENT;
  clear_status_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<int*>(workspace));
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

const char* noise_status_string(int status) {
  switch (status) {
    case NOISE_OK: return "ok";
    case NOISE_ERR_SHAPE: return "unsupported shape";
    case NOISE_ERR_ALIGN: return "misaligned pointer or stride";
    case NOISE_ERR_WORKSPACE: return "workspace missing or too small";
    case NOISE_ERR_ARGUMENT: return "invalid argument (NULL pointer, bad enum value, or a stream or device index the entry point does not take)";
    case NOISE_ERR_CUDA: return "CUDA call failed";
    case NOISE_ERR_DEVICE: return "not an sm_100 device";
    case NOISE_ERR_TOO_LARGE: return "members x tokens exceed the static scratch of the no-allocation entry point";
    default: return "unknown status";
  }
}

int noise_last_launch_count(void) { return g_launches; }

int noise_profile_start(int capacity) {
  if (capacity < 1) return NOISE_ERR_ARGUMENT;
  noise_profile_stop(nullptr, nullptr, 0);
  g_prof.ev = new cudaEvent_t[2 * capacity];
  g_prof.kind = new int[capacity];
  for (int i = 0; i < 2 * capacity; ++i) {
    if (cudaEventCreate(&g_prof.ev[i]) != cudaSuccess) {
      g_prof.capacity = i / 2;
      noise_profile_stop(nullptr, nullptr, 0);
      return NOISE_ERR_CUDA;
    }
  }
  g_prof.capacity = capacity;
  g_prof.used = 0;
  g_prof.on = true;
  return NOISE_OK;
}

int noise_profile_stop(float* kind_ms, int* kind_count, int nkinds) {
  int rc = NOISE_OK;
  if (kind_ms && kind_count) {
    for (int k = 0; k < nkinds; ++k) kind_ms[k] = 0.f, kind_count[k] = 0;
    for (int i = 0; i < g_prof.used; ++i) {
      float ms = 0.f;
      if (cudaEventSynchronize(g_prof.ev[2 * i + 1]) != cudaSuccess ||
          cudaEventElapsedTime(&ms, g_prof.ev[2 * i], g_prof.ev[2 * i + 1]) != cudaSuccess) {
        rc = NOISE_ERR_CUDA;
        break;
      }
      const int k = g_prof.kind[i];
      if (k < nkinds) kind_ms[k] += ms, kind_count[k] += 1;
    }
  }
  if (g_prof.ev) {
    for (int i = 0; i < 2 * g_prof.capacity; ++i) cudaEventDestroy(g_prof.ev[i]);
    delete[] g_prof.ev;
    delete[] g_prof.kind;
  }
  g_prof = Profiler{};
  return rc;
}

}  // extern "C"
