// The identity phase's query moments on tcgen05 (sm_100a): per query s and raw query coordinate d the change of the
// query's own softmax readout under a finite step of q_raw[s, d] (reference train/speedrun/moment_kernels.py:197-365,
// moment_query_scores; bf16 q / k / v / hub, keys 0 <= s - t <= window).
//
// Per query s and key t (logit x = q_s . k_t / 8, a = e^(x - lse_s), c = hub_s . v_t - hub_out_s, w = a c):
//   numerator moments   NX0, NY0, NX1, NY1, NXY = sum bf16(w) (x_t, y_t, x_t^2, y_t^2, x_t y_t)
//   denominator moments DX0, DY0, DX1, DY1, DXY = sum bf16(a) (same features)
//   LX0, LY0 = sum bf16(w x) (x_t, y_t), MX0, MY0 = sum bf16(a x) (x_t, y_t)
//   s1n = sum w x, s2n = sum w x^2, s1d = sum a x, s2d = sum a x^2 (fp32)
// with the keys' pair features x_i, y_i of side / 8 (bf16, from querymom_features_kernel), then per query the
// response zn / (1 + zd) / step of every raw coordinate through RoPE and the RMS norm, rounded to bf16.
//
// One work item = one 128-query tile of one row; keys stream in 32-wide tiles. 320 threads, one CTA per SM:
//   warp 0      TMA: Q, H once per item; per key tile k, v and the features fa = (x | y), fb = (x^2 | y^2),
//               fc = (x y | 0) (32 rows each, adjacent: fa | fb | fc is one 160-wide MN-major operand) into a
//               5-stage ring;
//   warp 1      TMEM (512 columns): S = Q K^T, C = H V^T (32 columns each), the accumulators N = W (fa | fb | fc)
//               (160), D = A (fa | fb | fc) (160), L = WL fa (64), M = AL fa (64); the whole warp runs the issue
//               loop and an elect.sync lane issues S / C of tile j + 1 (once the weight warps have read tile j's)
//               ahead of the moment MMAs of tile j;
//   warps 2..9  warp w: query rows of TMEM lane quarter w % 4, keys half (w - 2) / 4 of each tile: the four weights
//               as bf16 into one of two 64-byte-swizzled buffers; at the item's end the response epilogue for its 16
//               rotary pairs.
#pragma once
#include "ptx.cuh"

namespace noise {
namespace credit {

constexpr int QM_B = 128, QM_R = 32, QM_STAGES = 5, QM_THREADS = 320;
constexpr int QM_QT = QM_B * 128;       // [128][64] bf16 query-side tile: 16 KB
constexpr int QM_RT = QM_R * 128;       // [32][64] bf16 key-side tile: 4 KB
constexpr int QM_WT = QM_B * QM_R * 2;  // [128][32] bf16 weight matrix (64-byte rows): 8 KB
constexpr int QM_Q = 0, QM_H = QM_QT, QM_W = 2 * QM_QT;  // W: 2 buffers x (W, A, WL, AL)
constexpr int QM_RING = QM_W + 8 * QM_WT;
constexpr int QM_SK = 0, QM_SV = QM_RT, QM_SFA = 2 * QM_RT, QM_SFB = 3 * QM_RT, QM_SFC = 4 * QM_RT;
constexpr int QM_STAGE = 5 * QM_RT;
constexpr int QM_SUMS = QM_RING + QM_STAGES * QM_STAGE;  // s1n, s2n, s1d, s2d per (half, query row)
constexpr int QM_BAR = QM_SUMS + 4 * 2 * 128 * 4;
constexpr int QM_SMEM = QM_BAR + 256 + 1024;
// TMEM columns
constexpr uint32_t QM_TS = 0, QM_TC = 32, QM_TN = 64, QM_TD = 224, QM_TL = 384, QM_TM = 448;

struct QueryMomTcArgs {
  int T, window, rows;
  Rows raw;
  int raw_bf16, out_bf16;
  const float *sq, *steps, *lse, *hub_out;  // [rows, T]
  const float *cosb, *sinb;                 // [T, 32]
  Rows out;
  int* status;
};

struct QueryMomMaps {
  CUtensorMap q, h;          // bf16 [rows * T, 64], 128-row boxes
  CUtensorMap k, v;          // bf16 [rows * T, 64], 32-row boxes
  CUtensorMap fa, fb, fc;    // bf16 [rows * T, 64], 32-row boxes
};

// The keys' pair features of side / 8 (fp32 [rows * T, 64]): fa = (x_0..x_31, y_0..y_31), fb = (x_i^2 .., y_i^2 ..),
// fc = (x_i y_i .., 32 zeros), bf16 [rows * T, 64] each; one thread per (token, pair).
__global__ void __launch_bounds__(256) querymom_features_kernel(const float* __restrict__ side, int64_t n_pairs,
                                                               __nv_bfloat16* __restrict__ fa,
                                                               __nv_bfloat16* __restrict__ fb,
                                                               __nv_bfloat16* __restrict__ fc) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n_pairs;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t tok = i >> 5;
    const int pr = static_cast<int>(i & 31);
    const float x = side[tok * 64 + pr] * 0.125f, y = side[tok * 64 + pr + 32] * 0.125f;
    fa[tok * 64 + pr] = __float2bfloat16_rn(x);
    fa[tok * 64 + 32 + pr] = __float2bfloat16_rn(y);
    fb[tok * 64 + pr] = __float2bfloat16_rn(x * x);
    fb[tok * 64 + 32 + pr] = __float2bfloat16_rn(y * y);
    fc[tok * 64 + pr] = __float2bfloat16_rn(x * y);
    fc[tok * 64 + 32 + pr] = __float2bfloat16_rn(0.f);
  }
}

// 32 lanes x 8 consecutive 32-bit columns (issued only: the caller waits with tc_wait_ld).
__device__ __forceinline__ void qm_tmem_ld8(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

__global__ void __launch_bounds__(QM_THREADS, 1)
    querymom_tc_kernel(const __grid_constant__ QueryMomMaps m, const __grid_constant__ QueryMomTcArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + QM_BAR);
  uint64_t* q_full = bar;
  uint64_t* q_empty = bar + 1;
  uint64_t* st_full = bar + 2;              // STAGES
  uint64_t* st_empty = st_full + QM_STAGES;  // STAGES
  uint64_t* s_full = st_empty + QM_STAGES;
  uint64_t* s_empty = s_full + 1;
  uint64_t* w_full = s_empty + 1;  // 2 (weight buffers)
  uint64_t* w_empty = w_full + 2;  // 2
  uint64_t* acc_full = w_empty + 2;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* drain = acc_empty + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqt = p.T / QM_B;
  const int items = nqt * p.rows;
  // item w: query tile nqt - 1 - w / rows (the last tiles see the most keys: heaviest first) of row w % rows; its
  // key tiles run from the window's start to the tile's last query
  auto tiles_of = [&](int qt, int& lo, int& hi) {
    const int first = qt * QM_B - p.window;
    lo = first > 0 ? first / QM_R : 0;
    hi = (qt * QM_B + QM_B - 1) / QM_R;
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < QM_STAGES; ++s) {
      mbar_init(&st_full[s], 1);
      mbar_init(&st_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, 8);  // one arrival per weight warp (its lanes joined by __syncwarp first)
    for (int b = 0; b < 2; ++b) {
      mbar_init(&w_full[b], 8);
      mbar_init(&w_empty[b], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 8);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    const CUtensorMap* maps[7] = {&m.q, &m.h, &m.k, &m.v, &m.fa, &m.fb, &m.fc};
    for (int i = 0; i < 7; ++i) tma_prefetch_desc(maps[i]);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const uint32_t sbase = smem_u32(smem);

  if (warp == 0) {
    if (lane == 0) {
      int sv = 0, nitem = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++nitem) {
        const int qt = nqt - 1 - w / p.rows, row = w % p.rows;
        const int row0 = row * p.T;
        int lo, hi;
        tiles_of(qt, lo, hi);
        if (!mbar_wait(q_empty, (static_cast<uint32_t>(nitem) & 1u) ^ 1u, p.status)) break;
        mbar_arrive_expect_tx(q_full, 2 * QM_QT);
        tma_load_2d(smem + QM_Q, &m.q, q_full, 0, row0 + qt * QM_B);
        tma_load_2d(smem + QM_H, &m.h, q_full, 0, row0 + qt * QM_B);
        for (int j = lo; j <= hi; ++j, ++sv) {
          const int sl = sv % QM_STAGES;
          if (!mbar_wait(&st_empty[sl], (static_cast<uint32_t>(sv / QM_STAGES) & 1u) ^ 1u, p.status)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + QM_RING + sl * QM_STAGE;
          uint64_t* b = &st_full[sl];
          const int r = row0 + j * QM_R;
          mbar_arrive_expect_tx(b, QM_STAGE);
          tma_load_2d(st + QM_SK, &m.k, b, 0, r);
          tma_load_2d(st + QM_SV, &m.v, b, 0, r);
          tma_load_2d(st + QM_SFA, &m.fa, b, 0, r);
          tma_load_2d(st + QM_SFB, &m.fb, b, 0, r);
          tma_load_2d(st + QM_SFC, &m.fc, b, 0, r);
        }
      }
      if (nitem > 0) mbar_wait(q_full, static_cast<uint32_t>(nitem - 1) & 1u, p.status);
      for (int j = sv - 1; j >= 0 && j >= sv - QM_STAGES; --j)
        mbar_wait(&st_full[j % QM_STAGES], static_cast<uint32_t>(j / QM_STAGES) & 1u, p.status);
    }
  } else if (warp == 1) {
    {  // the whole warp runs the issuer; one elected lane issues the MMAs and commits
      constexpr uint32_t id_s = idesc_bf16(QM_B, QM_R);               // S, C: B = k / v rows (K-major)
      constexpr uint32_t id_n = idesc_bf16(QM_B, 160, false, true);   // N, D: B = fa | fb | fc (MN-major)
      constexpr uint32_t id_l = idesc_bf16(QM_B, 64, false, true);    // L, M: B = fa
      int sv = 0, nitem = 0;
      bool ok = true;
      auto moments = [&](int svj, bool first) {
        const int wb = svj & 1;
        if (!mbar_wait_warp(&w_full[wb], static_cast<uint32_t>(svj >> 1) & 1u, p.status)) return false;
        tc_fence_after();
        const uint32_t st = sbase + QM_RING + (svj % QM_STAGES) * QM_STAGE;
        const uint32_t w = sbase + QM_W + wb * 4 * QM_WT;  // W, A, WL, AL
#pragma unroll
        for (int ks = 0; ks < QM_R / 16; ++ks) {
          const uint32_t acc = (first && ks == 0) ? 0u : 1u;
          const uint64_t fd = sdesc_mnmajor_sw128(st + QM_SFA + ks * 2048, QM_RT);
          if (elect_one()) tc_mma(tmem + QM_TN, km_sdesc_kmajor_sw64(w) + 2u * ks, fd, id_n, acc);
          if (elect_one()) tc_mma(tmem + QM_TD, km_sdesc_kmajor_sw64(w + QM_WT) + 2u * ks, fd, id_n, acc);
          if (elect_one()) tc_mma(tmem + QM_TL, km_sdesc_kmajor_sw64(w + 2 * QM_WT) + 2u * ks, fd, id_l, acc);
          if (elect_one()) tc_mma(tmem + QM_TM, km_sdesc_kmajor_sw64(w + 3 * QM_WT) + 2u * ks, fd, id_l, acc);
        }
        if (elect_one()) tc_commit(&w_empty[wb]);
        if (elect_one()) tc_commit(&st_empty[svj % QM_STAGES]);
        return true;
      };
      // S / C of the tile with global index svj (the single S / C buffer is free once the weight warps read the
      // previous tile's)
      auto scores = [&](int svj) {
        const int sl = svj % QM_STAGES;
        if (!mbar_wait_warp(&st_full[sl], static_cast<uint32_t>(svj / QM_STAGES) & 1u, p.status) ||
            !mbar_wait_warp(s_empty, (static_cast<uint32_t>(svj) & 1u) ^ 1u, p.status))
          return false;
        tc_fence_after();
        const uint32_t st = sbase + QM_RING + sl * QM_STAGE;
        const uint64_t qd = sdesc_kmajor_sw128(sbase + QM_Q), hd = sdesc_kmajor_sw128(sbase + QM_H);
        const uint64_t kd = sdesc_kmajor_sw128(st + QM_SK), vd = sdesc_kmajor_sw128(st + QM_SV);
#pragma unroll
        for (int k = 0; k < 4; ++k)
              if (elect_one()) tc_mma(tmem + QM_TS, qd + 2u * k, kd + 2u * k, id_s, k > 0);
#pragma unroll
        for (int k = 0; k < 4; ++k)
              if (elect_one()) tc_mma(tmem + QM_TC, hd + 2u * k, vd + 2u * k, id_s, k > 0);
        if (elect_one()) tc_commit(&s_full[0]);
        return true;
      };
      for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++nitem) {
        const int qt = nqt - 1 - w / p.rows;
        int lo, hi;
        tiles_of(qt, lo, hi);
        if (!mbar_wait_warp(q_full, static_cast<uint32_t>(nitem) & 1u, p.status)) {
          ok = false;
          break;
        }
        ok = scores(sv);
        for (int j = lo; j <= hi && ok; ++j, ++sv) {
          if (j + 1 <= hi) ok = scores(sv + 1);
          if (ok && j == lo) ok = mbar_wait_warp(acc_empty, (static_cast<uint32_t>(nitem) & 1u) ^ 1u, p.status);
          if (ok) ok = moments(sv, j == lo);
        }
        if (ok) {
          if (elect_one()) tc_commit(q_empty);
          if (elect_one()) tc_commit(acc_full);
        }
      }
      if (elect_one()) tc_commit(drain);
      mbar_wait_warp(drain, 0, p.status);
    }
  } else {
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;  // query row of the tile
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t trow = tmem + lane_base;
    float* sums = reinterpret_cast<float*>(smem + QM_SUMS);  // [half][4][128]: s1n, s2n, s1d, s2d
    constexpr float SL2 = 0.125f * 1.4426950408889634f;
    constexpr float L2E = 1.4426950408889634f;
    int sv = 0, nitem = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++nitem) {
      const int qt = nqt - 1 - w / p.rows, row = w % p.rows;
      const int sq = qt * QM_B + r;
      const int64_t ti = static_cast<int64_t>(row) * p.T + sq;
      const float lse_r = p.lse[ti], hout_r = p.hub_out[ti];
      int lo, hi;
      tiles_of(qt, lo, hi);
      // even / odd keys' partial sums
      float2 s1n = make_float2(0.f, 0.f), s2n = s1n, s1d = s1n, s2d = s1n;
      for (int j = lo; j <= hi && ok; ++j, ++sv) {
        if (!mbar_wait(s_full, static_cast<uint32_t>(sv) & 1u, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float s[16], c[16];
        tmem_ld16(trow + QM_TS + half * 16, s);
        tmem_ld16(trow + QM_TC + half * 16, c);
        tc_wait_ld();
        reg_fence<16>(s);
        reg_fence<16>(c);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_empty);
        const int t0 = j * QM_R + half * 16;
        const bool full = t0 + 15 <= qt * QM_B && qt * QM_B + QM_B - 1 - t0 <= p.window;
        uint32_t pw[8], pa[8], pwl[8], pal[8];
        // keys in pairs: packed fp32x2 arithmetic, two exponentials on the MUFU pipe
        const float2 nl = make_float2(-lse_r * L2E, -lse_r * L2E), nh = make_float2(-hout_r, -hout_r);
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          const float2 sc = make_float2(s[e], s[e + 1]);
          const float2 logit = __fmul2_rn(sc, make_float2(0.125f, 0.125f));
          const float2 arg = __ffma2_rn(sc, make_float2(SL2, SL2), nl);
          float2 a = make_float2(ex2_approx(arg.x), ex2_approx(arg.y));
          if (!full) {
            if (t0 + e > sq || sq - (t0 + e) > p.window) a.x = 0.f;
            if (t0 + e + 1 > sq || sq - (t0 + e + 1) > p.window) a.y = 0.f;
          }
          const float2 wn = __fmul2_rn(a, __fadd2_rn(make_float2(c[e], c[e + 1]), nh));
          const float2 wl = __fmul2_rn(wn, logit), al = __fmul2_rn(a, logit);
          s1n = __fadd2_rn(s1n, wl);
          s2n = __ffma2_rn(wl, logit, s2n);
          s1d = __fadd2_rn(s1d, al);
          s2d = __ffma2_rn(al, logit, s2d);
          pw[e / 2] = pack_bf16x2(wn.x, wn.y);
          pa[e / 2] = pack_bf16x2(a.x, a.y);
          pwl[e / 2] = pack_bf16x2(wl.x, wl.y);
          pal[e / 2] = pack_bf16x2(al.x, al.y);
        }
        const int b = sv & 1;
        if (!mbar_wait(&w_empty[b], (static_cast<uint32_t>(sv >> 1) & 1u) ^ 1u, p.status)) {
          ok = false;
          break;
        }
        // row r, keys half * 16 .. + 15: 16-byte chunks half * 2 + i of the 64-byte row, 64-byte swizzle
        const uint32_t wrow = sbase + QM_W + b * 4 * QM_WT + r * 64;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const uint32_t off = static_cast<uint32_t>(((half * 2 + i) ^ ((r >> 1) & 3)) << 4);
          km_st_v4(wrow + off, pw[4 * i], pw[4 * i + 1], pw[4 * i + 2], pw[4 * i + 3]);
          km_st_v4(wrow + QM_WT + off, pa[4 * i], pa[4 * i + 1], pa[4 * i + 2], pa[4 * i + 3]);
          km_st_v4(wrow + 2 * QM_WT + off, pwl[4 * i], pwl[4 * i + 1], pwl[4 * i + 2], pwl[4 * i + 3]);
          km_st_v4(wrow + 3 * QM_WT + off, pal[4 * i], pal[4 * i + 1], pal[4 * i + 2], pal[4 * i + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&w_full[b]);
      }
      ok = __all_sync(0xffffffffu, ok);
      sums[(half * 4) * 128 + r] = s1n.x + s1n.y;
      sums[(half * 4 + 1) * 128 + r] = s2n.x + s2n.y;
      sums[(half * 4 + 2) * 128 + r] = s1d.x + s1d.y;
      sums[(half * 4 + 3) * 128 + r] = s2d.x + s2d.y;
      if (!bar_and<QM_THREADS - 64>(ok)) {
        ok = false;
        break;
      }
      const float v1n = sums[r] + sums[4 * 128 + r], v2n = sums[128 + r] + sums[5 * 128 + r];
      const float v1d = sums[2 * 128 + r] + sums[6 * 128 + r], v2d = sums[3 * 128 + r] + sums[7 * 128 + r];
      // per query: ratio = (2 step raw + step^2) / 64 / den = ka raw + kb, z = bf16(zn / (1 + zd) / step)
      const float stepv = p.steps[ti];
      const float den = p.sq[ti] / D + 1e-6f;
      const float inv = 1.f / (D * den);
      const float ka = 2.f * stepv * inv, kb = stepv * stepv * inv, cbk = stepv * rsqrtf(den), rstep = 1.f / stepv;
      const int64_t ro = p.raw.at(row, sq, p.T);
      const int64_t oo = p.out.at(row, sq, p.T);
      // a thread whose wait gives up skips the epilogue but still reaches the item's closing barrier
      const bool got = __all_sync(0xffffffffu, mbar_wait(acc_full, static_cast<uint32_t>(nitem) & 1u, p.status));
      tc_fence_after();
#pragma unroll 1
      for (int g8 = 0; g8 < (got ? 2 : 0); ++g8) {
        const int P0 = half * 16 + g8 * 8;  // this chunk's 8 rotary pairs
        float nx[8], ny[8], nxx[8], nyy[8], nxy[8], dx[8], dy[8], dxx[8], dyy[8], dxy[8], lx[8], ly[8], mx[8], my[8];
        qm_tmem_ld8(trow + QM_TN + P0, nx);
        qm_tmem_ld8(trow + QM_TN + 32 + P0, ny);
        qm_tmem_ld8(trow + QM_TN + 64 + P0, nxx);
        qm_tmem_ld8(trow + QM_TN + 96 + P0, nyy);
        qm_tmem_ld8(trow + QM_TN + 128 + P0, nxy);
        qm_tmem_ld8(trow + QM_TD + P0, dx);
        qm_tmem_ld8(trow + QM_TD + 32 + P0, dy);
        qm_tmem_ld8(trow + QM_TD + 64 + P0, dxx);
        qm_tmem_ld8(trow + QM_TD + 96 + P0, dyy);
        qm_tmem_ld8(trow + QM_TD + 128 + P0, dxy);
        qm_tmem_ld8(trow + QM_TL + P0, lx);
        qm_tmem_ld8(trow + QM_TL + 32 + P0, ly);
        qm_tmem_ld8(trow + QM_TM + P0, mx);
        qm_tmem_ld8(trow + QM_TM + 32 + P0, my);
        tc_wait_ld();
        reg_fence<8>(nx);
        reg_fence<8>(ny);
        reg_fence<8>(nxx);
        reg_fence<8>(nyy);
        reg_fence<8>(nxy);
        reg_fence<8>(dx);
        reg_fence<8>(dy);
        reg_fence<8>(dxx);
        reg_fence<8>(dyy);
        reg_fence<8>(dxy);
        reg_fence<8>(lx);
        reg_fence<8>(ly);
        reg_fence<8>(mx);
        reg_fence<8>(my);
        if (g8 == 1) {  // every accumulator column of this item has been read
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(acc_empty);
        }
        const float4 c0 = *reinterpret_cast<const float4*>(p.cosb + static_cast<int64_t>(sq) * 32 + P0);
        const float4 c1 = *reinterpret_cast<const float4*>(p.cosb + static_cast<int64_t>(sq) * 32 + P0 + 4);
        const float4 n0 = *reinterpret_cast<const float4*>(p.sinb + static_cast<int64_t>(sq) * 32 + P0);
        const float4 n1 = *reinterpret_cast<const float4*>(p.sinb + static_cast<int64_t>(sq) * 32 + P0 + 4);
        const float csv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
        const float snv[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
#pragma unroll 1
        for (int hf = 0; hf < 2; ++hf) {  // coordinates d = P + 32 hf
          float res[8], rv[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) rv[i] = raw_at(p.raw, p.raw_bf16, ro + P0 + i + 32 * hf);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            // ca = (1 + ratio)^(-1/2) - 1 = -ratio s^2 / (1 + s), s = (1 + ratio)^(-1/2) (the reference's
            // expm1(-log1p(ratio) / 2), without the cancellation of s - 1)
            const float ratio = fmaf(ka, rv[i], kb);
            const float srt = rsqrtf(1.f + ratio);
            const float ca = __fdividef(-ratio * srt * srt, 1.f + srt);
            const float bb = cbk * (1.f + ca);
            const float bu = bb * (hf ? snv[i] : csv[i]), bw = bb * (hf ? csv[i] : -snv[i]);
            const float zn = nx[i] * bu + ny[i] * bw + 0.5f * (nxx[i] * bu * bu + nyy[i] * bw * bw) +
                             nxy[i] * bu * bw + ca * (lx[i] * bu + ly[i] * bw) + v1n * ca + v2n * (0.5f * ca * ca);
            const float zd = dx[i] * bu + dy[i] * bw + 0.5f * (dxx[i] * bu * bu + dyy[i] * bw * bw) +
                             dxy[i] * bu * bw + ca * (mx[i] * bu + my[i] * bw) + v1d * ca + v2d * (0.5f * ca * ca);
            res[i] = bf16_round(zn / (1.f + zd) * rstep);
          }
          const int64_t o = oo + P0 + 32 * hf;  // 8 consecutive coordinates (host: 16-byte strides)
          if (p.out_bf16) {
            *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out.data) + o) =
                make_uint4(pack_bf16x2(res[0], res[1]), pack_bf16x2(res[2], res[3]), pack_bf16x2(res[4], res[5]),
                           pack_bf16x2(res[6], res[7]));
          } else {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out.data) + o);
            dst[0] = make_float4(res[0], res[1], res[2], res[3]);
            dst[1] = make_float4(res[4], res[5], res[6], res[7]);
          }
        }
      }
      // both halves have read sums before the next item overwrites them
      if (!bar_and<QM_THREADS - 64>(got)) {
        ok = false;
        break;
      }
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace credit
}  // namespace noise
