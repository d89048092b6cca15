// noise_record::future_scores and noise_record::key_response on tcgen05 (sm_100a): reference train/val/run.py
// :1696-1725 (score_kernel) and :571-593 (finite_attention_kernels' key_response), whose dots run
// tl.dot(..., input_precision="tf32x3"). Per head h and column col = (probe p, source m):
//   S[s, col] = q_s . dk_col / 8,  VS[s, col] = target_s . dv_col           (tf32x3, fp32 accumulate)
//   future_scores  out[h, p, m] = sum over receivers 0 < s - (start + m) <= window of
//                  (ch c + (a + ch) VS) / (1 + ch),  ch = a (e^S - 1),  a = A[h, s, m], c = C[h, s, m]
//   key_response   out[h, p, m] = sum over queries query_start + s in [source_start + m, .. + window] of
//                  ch / (1 + ch) c
// The columns are the MMA rows (M = 128): S^T = dk q^T, so each epilogue thread owns a column and its sum over
// receivers stays in a register, as the reference's per-column result does.
//
// Before the kernel, col_split_kernel writes q (and target) as tf32 hi / lo planes [H, Tp, 64] (Tp = T rounded up to
// 64, zero rows past T), K-major and TMA-loadable. One CTA per 128 consecutive columns of a head; its receivers are
// the union of its columns' windows, in 32-receiver tiles. 320 threads:
//   warp 0      TMA: per receiver tile q hi / lo (and target hi / lo) into a ring of 2 stages (4 for key_response);
//   warp 1      TMEM (256 columns: S and VS, 32 each, 4 buffers) and the MMAs: S^T (and VS^T) of a tile, 24
//               kind::tf32 MMAs 128 x 32 x 8 each (hi.hi + hi.lo + lo.hi per K-step), A = dk (dv) from shared
//               memory;
//   warps 2..9  warp w: columns of TMEM lane quarter w % 4, receivers 16 ((w - 2) / 4) .. + 15 of each tile; a and
//               c loaded a tile ahead; at the end the two halves' sums meet in shared memory.
// All threads first stage the block's dk (and dv) rows as tf32 hi / lo into 128-byte-swizzled K-major tiles.
#pragma once
#include "ptx.cuh"

namespace noise {
namespace readout {

constexpr int CT_COLS = 128, CT_RECV = 32, CT_THREADS = 320, CT_EPI = 8;
constexpr int CT_SB = 4;  // S (and VS) buffers in TMEM: the MMAs run up to CT_SB - 1 tiles ahead of the epilogue
constexpr int CT_HALF = CT_COLS * 128;    // 128 rows x 32 fp32 (one K-major half of 64 dims): 16 KB
constexpr int CT_OP = CT_RECV * 128;      // 32 receivers x 32 fp32: 4 KB
constexpr int CT_B = 4 * CT_OP;           // hi half 0, hi half 1, lo half 0, lo half 1 of q (or target): 16 KB

template <bool VALUES>
struct CtLayout {
  static constexpr int A = VALUES ? 2 : 1;       // dk (and dv)
  static constexpr int DKH = 0, DKL = 2 * CT_HALF, DVH = 4 * CT_HALF, DVL = 6 * CT_HALF;
  static constexpr int RING = A * 4 * CT_HALF;   // after dk hi / lo (and dv hi / lo)
  static constexpr int STAGE = A * CT_B;         // q (and target)
  static constexpr int STAGES = VALUES ? 2 : 4;
  static constexpr int SUMS = RING + STAGES * STAGE;  // [2][128] fp32
  static constexpr int BAR = SUMS + 2 * CT_COLS * 4;
  static constexpr int SMEM = BAR + 256 + 1024;
  static_assert(SMEM <= 227 * 1024, "shared memory per CTA");
};

struct CtArgs {
  const float *dk, *dv;  // contiguous [H, P, M, 64]
  View3 a, c;            // (H, T, M)
  float* out;            // [H, P, M]
  int T, M, P, H, Tp;
  int first_off;         // a column of source m sees receivers s with first_off + m <= s <= first_off + m + span
  int span;
  int* status;
};

struct CtMaps {
  CUtensorMap qhi, qlo, ghi, glo;  // fp32 [H * Tp, 64], 32-row x 32 boxes, 128-byte swizzle
};

// q (or target) -> tf32 hi / lo [H, Tp, 64], rows >= T zero; grid (Tp / 64, H)
__global__ void __launch_bounds__(256) col_split_kernel(View3 x, int T, int Tp, float* __restrict__ hi,
                                                        float* __restrict__ lo) {
  const int h = blockIdx.y, s0 = blockIdx.x * 64;
  for (int i = threadIdx.x; i < 64 * D; i += 256) {
    const int s = s0 + i / D, d = i % D;
    const float v = s < T ? x.at(h, s, d) : 0.f;
    const float vh = tf32_hi(v);
    const int64_t o = (static_cast<int64_t>(h) * Tp + s) * D + d;
    hi[o] = vh;
    lo[o] = v - vh;
  }
}

template <bool VALUES>
__global__ void __launch_bounds__(CT_THREADS, 1)
    column_tc_kernel(const __grid_constant__ CtMaps m, const __grid_constant__ CtArgs p) {
  using L = CtLayout<VALUES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint64_t* full = bar;                  // STAGES
  uint64_t* empty = full + L::STAGES;    // STAGES
  uint64_t* s_full = empty + L::STAGES;  // CT_SB
  uint64_t* s_empty = s_full + CT_SB;    // CT_SB
  uint64_t* drain = s_empty + CT_SB;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, ncols = p.P * p.M;
  const int c_lo = blockIdx.x * CT_COLS, c_hi = min(c_lo + CT_COLS, ncols) - 1;
  // the block's receivers: the union of its columns' windows (its columns are consecutive)
  const bool wraps = c_hi / p.M > c_lo / p.M;
  const int m_lo = wraps ? 0 : c_lo % p.M, m_hi = wraps ? p.M - 1 : c_hi % p.M;
  const int s_first = max(0, p.first_off + m_lo), s_last = min(p.T - 1, p.first_off + m_hi + p.span);
  const int t_first = s_first / CT_RECV;
  const int n = s_first <= s_last ? s_last / CT_RECV - t_first + 1 : 0;

  if (threadIdx.x == 0) {
    for (int b = 0; b < L::STAGES; ++b) {
      mbar_init(&full[b], 1);
      mbar_init(&empty[b], 1);
    }
    for (int b = 0; b < CT_SB; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], CT_EPI);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&m.qhi);
    tma_prefetch_desc(&m.qlo);
    if (VALUES) {
      tma_prefetch_desc(&m.ghi);
      tma_prefetch_desc(&m.glo);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 64 * CT_SB);
    tmem_relinquish();
  }
  // dk (dv) rows of the block as tf32 hi / lo: float4 q of a row = 16-byte chunk q % 8 of half q / 8, swizzled
  const uint32_t sbase = smem_u32(smem);
  for (int f = threadIdx.x; f < CT_COLS * 16; f += CT_THREADS) {
    const int r = f >> 4, q = f & 15, col = c_lo + r;
    const uint32_t off = static_cast<uint32_t>((q >> 3) * CT_HALF + r * 128 + (((q & 7) ^ (r & 7)) << 4));
#pragma unroll
    for (int o = 0; o < L::A; ++o) {
      const float* src = o == 0 ? p.dk : p.dv;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (col < ncols) x = *reinterpret_cast<const float4*>(src + (static_cast<int64_t>(h) * ncols + col) * D + q * 4);
      const float4 xh = make_float4(tf32_hi(x.x), tf32_hi(x.y), tf32_hi(x.z), tf32_hi(x.w));
      const float4 xl = make_float4(x.x - xh.x, x.y - xh.y, x.z - xh.z, x.w - xh.w);
      asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(sbase + (o ? L::DVH : L::DKH) + off), "f"(xh.x),
                   "f"(xh.y), "f"(xh.z), "f"(xh.w)
                   : "memory");
      asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(sbase + (o ? L::DVL : L::DKL) + off), "f"(xl.x),
                   "f"(xl.y), "f"(xl.z), "f"(xl.w)
                   : "memory");
    }
  }
  fence_proxy_async_smem();  // the tensor core reads these through the async proxy
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int j = 0; j < n; ++j) {
        const int b = j % L::STAGES;
        if (!mbar_wait(&empty[b], (static_cast<uint32_t>(j / L::STAGES) & 1u) ^ 1u, p.status)) break;
        uint8_t* st = smem + L::RING + b * L::STAGE;
        const int y = h * p.Tp + (t_first + j) * CT_RECV;
        mbar_arrive_expect_tx(&full[b], L::STAGE);
        tma_load_2d(st, &m.qhi, &full[b], 0, y);
        tma_load_2d(st + CT_OP, &m.qhi, &full[b], 32, y);
        tma_load_2d(st + 2 * CT_OP, &m.qlo, &full[b], 0, y);
        tma_load_2d(st + 3 * CT_OP, &m.qlo, &full[b], 32, y);
        if (VALUES) {
          tma_load_2d(st + CT_B, &m.ghi, &full[b], 0, y);
          tma_load_2d(st + CT_B + CT_OP, &m.ghi, &full[b], 32, y);
          tma_load_2d(st + CT_B + 2 * CT_OP, &m.glo, &full[b], 0, y);
          tma_load_2d(st + CT_B + 3 * CT_OP, &m.glo, &full[b], 32, y);
        }
        ++issued;
      }
      // no TMA write may still be in flight when the CTA exits
      for (int j = max(issued - L::STAGES, 0); j < issued; ++j)
        mbar_wait(&full[j % L::STAGES], static_cast<uint32_t>(j / L::STAGES) & 1u, p.status);
    }
  } else if (warp == 1) {
    constexpr uint32_t id = idesc_tf32(CT_COLS, CT_RECV);
    // A (dk or dv) x B (q or target tile) into accumulator d: per K-step of 8 dims lo.hi, hi.lo, then hi.hi
    auto product = [&](uint32_t d, uint32_t ahi, uint32_t alo, uint32_t b) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t ho = k >> 2, kk = 2u * (k & 3);
        const uint64_t ah = sdesc_kmajor_sw128(ahi + ho * CT_HALF) + kk;
        const uint64_t al = sdesc_kmajor_sw128(alo + ho * CT_HALF) + kk;
        const uint64_t bh = sdesc_kmajor_sw128(b + ho * CT_OP) + kk;
        const uint64_t bl = sdesc_kmajor_sw128(b + 2 * CT_OP + ho * CT_OP) + kk;
        if (elect_one()) tc_mma_tf32(d, al, bh, id, k > 0);
        if (elect_one()) tc_mma_tf32(d, ah, bl, id, 1u);
        if (elect_one()) tc_mma_tf32(d, ah, bh, id, 1u);
      }
    };
    for (int j = 0; j < n; ++j) {
      const int b = j % L::STAGES, sb = j % CT_SB;
      if (!mbar_wait_warp(&full[b], static_cast<uint32_t>(j / L::STAGES) & 1u, p.status) ||
          !mbar_wait_warp(&s_empty[sb], (static_cast<uint32_t>(j / CT_SB) & 1u) ^ 1u, p.status))
        break;
      tc_fence_after();
      const uint32_t st = sbase + L::RING + b * L::STAGE;
      product(tmem + sb * 64, sbase + L::DKH, sbase + L::DKL, st);
      if (VALUES) product(tmem + sb * 64 + 32, sbase + L::DVH, sbase + L::DVL, st + CT_B);
      if (elect_one()) tc_commit(&s_full[sb]);
      if (elect_one()) tc_commit(&empty[b]);
    }
    if (elect_one()) tc_commit(drain);
    mbar_wait_warp(drain, 0, p.status);
  } else {
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane, col = c_lo + r;
    const bool valid = col < ncols;
    const int mc = valid ? col % p.M : 0;
    const int lo_s = p.first_off + mc, hi_s = lo_s + p.span;  // this column's receivers
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    // a and c of this column for receivers s0 + 16 half .. + 15 of tile jj, a tile ahead of their use
    float an[16], cn[16];
    // this column's a and c rows (receiver stride s1): one base pointer each, stepped per receiver
    const float* acol = p.a.p + h * p.a.s0 + mc * p.a.s2;
    const float* ccol = p.c.p + h * p.c.s0 + mc * p.c.s2;
    auto fetch = [&](int jj) {
      const int s0 = (t_first + jj) * CT_RECV + half * 16;
      const float* ap = acol + s0 * p.a.s1;
      const float* cp = ccol + s0 * p.c.s1;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const bool in = valid && s0 + i < p.T;
        an[i] = in ? *ap : 0.f;
        cn[i] = in ? *cp : 0.f;
        ap += p.a.s1;
        cp += p.c.s1;
      }
    };
    float acc = 0.f;
    bool ok = true;
    if (n > 0) fetch(0);
    for (int j = 0; j < n; ++j) {
      const int sb = j % CT_SB;
      float av[16], cv[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) av[i] = an[i], cv[i] = cn[i];
      if (j + 1 < n) fetch(j + 1);
      if (!mbar_wait_warp(&s_full[sb], static_cast<uint32_t>(j / CT_SB) & 1u, p.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[16], vv[16];
      tmem_ld16(trow + sb * 64 + half * 16, sv);
      if (VALUES) tmem_ld16(trow + sb * 64 + 32 + half * 16, vv);
      tc_wait_ld();
      reg_fence<16>(sv);
      if (VALUES) reg_fence<16>(vv);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[sb]);
      const int s0 = (t_first + j) * CT_RECV + half * 16;
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        const float2 e = expm1_f2(__fmul2_rn(make_float2(sv[i], sv[i + 1]), make_float2(SCALE, SCALE)));
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int s = s0 + i + u;
          const float ev = u ? e.y : e.x;
          const float ch = av[i + u] * ev;
          float term;
          // fast division (2 ulp for a denominator in the normal range, as Triton's default fp32 division)
          if constexpr (VALUES)
            term = __fdividef(ch * cv[i + u] + (av[i + u] + ch) * vv[i + u], 1.f + ch);
          else
            term = __fdividef(ch, 1.f + ch) * cv[i + u];
          if (valid && s >= lo_s && s <= hi_s && s < p.T) acc += term;
        }
      }
    }
    float* sums = reinterpret_cast<float*>(smem + L::SUMS);
    sums[half * CT_COLS + r] = acc;
    const bool all = bar_and<CT_THREADS - 64>(ok);
    if (half == 0 && valid && all)
      p.out[static_cast<int64_t>(h) * ncols + col] = sums[r] + sums[CT_COLS + r];
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 64 * CT_SB);
  }
}

}  // namespace readout
}  // namespace noise
