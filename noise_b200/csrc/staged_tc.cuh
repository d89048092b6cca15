// The true-path readout scorer's staged_kernel (reference train/val/run.py :5985-6040) and readout_kernel
// (:5906-5965) with their moment-table terms on tcgen05: per head, bf16(dk) M1 and bf16(dk) M2 for a block's 128 rows are kind::f16 MMAs (M = 128 rows, N = 64,
// K = 64; the reference's tl.dot of the same bf16 operands, fp32 accumulation), and each row's dot of those rows with
// its fp32 dk / dv is one thread's sum over a TMEM row. Everything else (dk, dv from the bf16 projection, the RMS norm
// and RoPE, the exact receiver, the self-edge, dk . U / 8 + dv . W) stays head_change's warp-per-row arithmetic.
//
// A block is 128 rows (moves or probes) of one token (two blocks per SM), 8 warps. Per head h:
//   warp phase   warp w takes rows w, w + 8, ..: head_change, then bf16(dk) into the 128-byte-swizzled K-major A tile
//                and fp32 dk, dv into padded rows of shared memory (zero for rows past the token's count);
//   MMAs         thread 0: D1 = A M1, D2 = A M2 into TMEM (tables M1, M2 of (t, h) by TMA as the MN-major B
//                operands), committed to an mbarrier; then the next head's tables;
//   TMEM phase   warp w: TMEM lane quarter w % 4; warps 0..3 sum D1 . dk, warps 4..7 D2 . dv over their rows.
#pragma once
#include <type_traits>

namespace noise {
namespace scorer {

constexpr int STC_ROWS = 128, STC_THREADS = 256, STC_PAD = D + 1;
constexpr int STC_A = 0;                              // bf16 [128][64], 128-byte swizzle: 16 KB
constexpr int STC_TB = STC_A + STC_ROWS * 128;        // M1, M2 bf16 [64][64] each: 16 KB
constexpr int STC_DK = STC_TB + 2 * D * D * 2;        // fp32 [128][65]
constexpr int STC_DV = STC_DK + STC_ROWS * STC_PAD * 4;
constexpr int STC_ROW = STC_DV + STC_ROWS * STC_PAD * 4;  // inv, coef, tot, q1, q2 [128] fp32; gate change [128][H]
constexpr int STC_BAR = STC_ROW + 5 * STC_ROWS * 4 + STC_ROWS * H * 4;
constexpr int STC_SMEM = STC_BAR + 64 + 1024;
static_assert(2 * STC_SMEM <= 228 * 1024, "two blocks per SM");

struct StcMaps {
  CUtensorMap m1, m2;  // bf16 [T * H * 64, 64], 64 x 64 boxes, 128-byte swizzle
};

// Args = StagedArgs (staged_kernel: the change from the bf16 projection of the raw move and the stats pass) or
// DirectArgs (readout_kernel, run.py:5906-5965: from the projected change itself, per-chunk r0 / ve / cos / sin rows)
template <bool GATED, bool SELF, class Args>
__global__ void __launch_bounds__(STC_THREADS, 2)
    staged_tc_kernel(const __grid_constant__ StcMaps maps, const __grid_constant__ Args a, int* status) {
  constexpr bool DIRECT = std::is_same<Args, DirectArgs>::value;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* sdk = reinterpret_cast<float*>(smem + STC_DK);
  float* sdv = reinterpret_cast<float*>(smem + STC_DV);
  float* sinv = reinterpret_cast<float*>(smem + STC_ROW);
  float* scoef = sinv + STC_ROWS;
  float* stot = scoef + STC_ROWS;
  float* sq1 = stot + STC_ROWS;
  float* sq2 = sq1 + STC_ROWS;
  float* sgc = sq2 + STC_ROWS;  // [128][H]
  uint64_t* tb_full = reinterpret_cast<uint64_t*>(smem + STC_BAR);
  uint64_t* mma_done = tb_full + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(mma_done + 1);
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int t = blockIdx.y, p0 = blockIdx.x * STC_ROWS;
  const int tok = a.start + t;
  const uint32_t sbase = smem_u32(smem);
  int nrows;
  if constexpr (DIRECT) nrows = a.P;
  else nrows = a.n;

  if (threadIdx.x == 0) {
    mbar_init(tb_full, 1);
    mbar_init(mma_done, 1);
    fence_barrier_init();
  }
  if (wib == 0) {
    tmem_alloc(tmem_holder, 128);
    tmem_relinquish();
  }
  // per row (staged): the stats pass's inverse RMS and coefficient, the gate change per head (GATED)
  for (int k = 0; k < STC_ROWS / 8; ++k) {
    const int rl = wib + 8 * k, p = p0 + rl;
    if (lane == 0) stot[rl] = 0.f;
    if constexpr (!DIRECT) {
      const bool live = p < a.n;
      const float iv = live ? a.st[(static_cast<int64_t>(t) * a.n + p) * 2] : 1.f;
      const float cf = live ? a.st[(static_cast<int64_t>(t) * a.n + p) * 2 + 1] : 0.f;
      if (lane == 0) {
        sinv[rl] = iv;
        scoef[rl] = cf;
      }
      if constexpr (GATED) {  // gate change per head: 2 (sigmoid(gz + inv ug + coef gz) - sigmoid(gz))
        if (lane < H) {
          const float gz = a.gz[static_cast<int64_t>(tok) * H + lane];
          const float ug = live ? bf(a.up, (static_cast<int64_t>(t) * a.n + p) * a.nc + 2 * W + lane) : 0.f;
          const float z = gz + iv * ug + cf * gz;
          sgc[rl * H + lane] = 2.f * (1.f / (1.f + __expf(-z)) - 1.f / (1.f + __expf(-gz)));
        }
      }
    }
  }
  sq1[threadIdx.x & (STC_ROWS - 1)] = 0.f;
  sq2[threadIdx.x & (STC_ROWS - 1)] = 0.f;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&maps.m1);
    tma_prefetch_desc(&maps.m2);
    mbar_arrive_expect_tx(tb_full, 2 * D * D * 2);
    tma_load_2d(smem + STC_TB, &maps.m1, tb_full, 0, tok * H * D);
    tma_load_2d(smem + STC_TB + D * D * 2, &maps.m2, tb_full, 0, tok * H * D);
  }
  float c, s;
  if constexpr (DIRECT) {
    c = a.cs[t * a.csm + lane * a.csf];
    s = a.sn[t * a.snm + lane * a.snf];
  } else {
    c = a.cs[static_cast<int64_t>(tok) * (D / 2) + lane];
    s = a.sn[static_cast<int64_t>(tok) * (D / 2) + lane];
  }
  bool ok = true;
  for (int h = 0; h < H; ++h) {
    const int64_t row = static_cast<int64_t>(tok) * H + h;
    // the clean rotated key (and, gated, the value embedding): global token rows (staged) or chunk rows (direct)
    const int64_t kr = DIRECT ? (static_cast<int64_t>(t) * H + h) * D : row * D;
    const float r00 = a.r0[kr + lane], r01 = a.r0[kr + lane + 32];
    float vc0 = 0.f, vc1 = 0.f;
    if constexpr (!DIRECT) {
      vc0 = a.vc[static_cast<int64_t>(tok) * W + h * D + lane];
      vc1 = a.vc[static_cast<int64_t>(tok) * W + h * D + lane + 32];
    }
    float ve0 = 0.f, ve1 = 0.f;
    if constexpr (GATED) {
      ve0 = a.ve[kr + lane];
      ve1 = a.ve[kr + lane + 32];
    }
    const HeadVals hv = head_vals<SELF>(a.tab, row, lane);  // the head's table values, once for all its rows
    const float square = warp_sum(r00 * r00 + r01 * r01);   // |r0|^2 of the head, the same for all its rows
    // warp phase: head_change per row, bf16(dk) into A (element (r, f) at r * 128 + ((f / 8) ^ (r % 8)) * 16 + (f % 8) * 2)
    // a row's four raw inputs (the lane's key and value features), loaded one row ahead of their use
    float in0 = 0.f, in1 = 0.f, in2 = 0.f, in3 = 0.f;
    auto load_in = [&](int k) {
      const int p = p0 + wib + 8 * k;
      if (p >= nrows) return;
      if constexpr (DIRECT) {
        const int64_t base = ((static_cast<int64_t>(t) * a.P + p) * 2 * H + h) * D;
        in0 = a.pj[base + lane], in1 = a.pj[base + lane + 32];
        in2 = a.pj[base + H * D + lane], in3 = a.pj[base + H * D + lane + 32];
      } else {
        const int64_t ur = (static_cast<int64_t>(t) * a.n + p) * a.nc;
        in0 = bf(a.up, ur + h * D + lane), in1 = bf(a.up, ur + h * D + lane + 32);
        in2 = bf(a.up, ur + W + h * D + lane), in3 = bf(a.up, ur + W + h * D + lane + 32);
      }
    };
    load_in(0);
#pragma unroll 1
    for (int k = 0; k < STC_ROWS / 8; ++k) {
      const int rl = wib + 8 * k, p = p0 + rl;
      const float x0 = in0, x1 = in1, x2 = in2, x3 = in3;
      if (k + 1 < STC_ROWS / 8) load_in(k + 1);
      float dk0 = 0.f, dk1 = 0.f, dv0 = 0.f, dv1 = 0.f;
      if (p < nrows) {
        float dr0, dr1, gc = 0.f;
        __nv_bfloat16* se_row = nullptr;
        if constexpr (DIRECT) {
          dr0 = x0 * c + x1 * s;
          dr1 = -x0 * s + x1 * c;
          dv0 = x2;
          dv1 = x3;
          if constexpr (GATED) gc = a.gc[(static_cast<int64_t>(t) * a.P + p) * H + h];
          if constexpr (SELF) se_row = a.se + (static_cast<int64_t>(t) * a.P + p) * W + h * D;
        } else {
          const float iv = sinv[rl], cf = scoef[rl];
          dr0 = iv * (x0 * c + x1 * s) + cf * r00;
          dr1 = iv * (x1 * c - x0 * s) + cf * r01;
          dv0 = iv * x2 + cf * vc0;
          dv1 = iv * x3 + cf * vc1;
          if constexpr (GATED) gc = sgc[rl * H + h];
          if constexpr (SELF) se_row = a.se + (static_cast<int64_t>(t) * a.se_rows + p) * W + h * D;
        }
        if constexpr (GATED) {
          dv0 += gc * ve0;
          dv1 += gc * ve1;
        }
        const float part =
            head_change_v<SELF>(dr0, dr1, dv0, dv1, r00, r01, square, hv, lane, a.diag, se_row, dk0, dk1);
        if (lane == 0) stot[rl] += part;
      }
      const uint32_t arow = sbase + STC_A + rl * 128 + (lane & 7) * 2;
      const uint16_t b0 = __bfloat16_as_ushort(__float2bfloat16_rn(dk0));
      const uint16_t b1 = __bfloat16_as_ushort(__float2bfloat16_rn(dk1));
      asm volatile("st.shared.u16 [%0], %1;" ::"r"(arow + ((((lane >> 3)) ^ (rl & 7)) << 4)), "h"(b0) : "memory");
      asm volatile("st.shared.u16 [%0], %1;" ::"r"(arow + ((((lane >> 3) + 4) ^ (rl & 7)) << 4)), "h"(b1) : "memory");
      sdk[rl * STC_PAD + lane] = dk0;
      sdk[rl * STC_PAD + lane + 32] = dk1;
      sdv[rl * STC_PAD + lane] = dv0;
      sdv[rl * STC_PAD + lane + 32] = dv1;
    }
    fence_proxy_async_smem();  // A goes to the tensor core through the async proxy
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // MMAs: D1 = A M1 (TMEM columns 0..63), D2 = A M2 (64..127); M as MN-major B (N = f' contiguous, K = f rows)
    if (wib == 0) {
      constexpr uint32_t id = idesc_bf16(STC_ROWS, D, false, true);
      const bool have = ok && mbar_wait_warp(tb_full, static_cast<uint32_t>(h) & 1u, status);
      if (have) {
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint64_t ad = sdesc_kmajor_sw128(sbase + STC_A) + 2u * k;
          if (elect_one()) tc_mma(tmem, ad, sdesc_mnmajor_sw128(sbase + STC_TB + k * 2048, 16), id, k > 0);
          if (elect_one())
            tc_mma(tmem + 64, ad, sdesc_mnmajor_sw128(sbase + STC_TB + D * D * 2 + k * 2048, 16), id, k > 0);
        }
      }
      if (elect_one()) tc_commit(mma_done);  // arrives also when nothing was issued, so every thread's wait ends
    }
    const bool done = mbar_wait_warp(mma_done, static_cast<uint32_t>(h) & 1u, status);
    ok = ok && done;
    tc_fence_after();
    // the tables' buffer is free once the MMAs have completed: the next head's
    if (threadIdx.x == 0 && ok && h + 1 < H) {
      mbar_arrive_expect_tx(tb_full, 2 * D * D * 2);
      tma_load_2d(smem + STC_TB, &maps.m1, tb_full, 0, (tok * H + h + 1) * D);
      tma_load_2d(smem + STC_TB + D * D * 2, &maps.m2, tb_full, 0, (tok * H + h + 1) * D);
    }
    // TMEM phase: row r's D1 . dk (warps 0..3) or D2 . dv (warps 4..7)
    if (ok) {
      const int quarter = wib & 3, part = wib >> 2;
      const int r = quarter * 32 + lane;
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + part * 64;
      const float* x = (part ? sdv : sdk) + r * STC_PAD;
      float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float dv[32];
        tmem_ld32(taddr + half * 32, dv);
        tc_wait_ld();
        reg_fence<32>(dv);
#pragma unroll
        for (int f = 0; f < 32; f += 2) {
          acc0 = fmaf(dv[f], x[half * 32 + f], acc0);
          acc1 = fmaf(dv[f + 1], x[half * 32 + f + 1], acc1);
        }
      }
      (part ? sq2 : sq1)[r] += acc0 + acc1;
    }
    tc_fence_before();
    __syncthreads();  // A, dk / dv and TMEM are free for the next head
    tc_fence_after();
  }
  if (threadIdx.x < STC_ROWS && ok) {
    const int p = p0 + threadIdx.x;
    if (p < nrows)
      a.out[static_cast<int64_t>(t) * nrows + p] =
          stot[threadIdx.x] + sq1[threadIdx.x] * (1.f / D) + sq2[threadIdx.x] * 0.125f;
  }
  __syncthreads();
  if (wib == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

}  // namespace scorer
}  // namespace noise
