// Key moments on tcgen05 (sm_100a): per key t and raw key coordinate d the degree-2 moment response of the receivers'
// softmax to a finite step of k_raw[t, d], and the value sums sum_s p hub_s. Two variants of one kernel:
//   IDENT  the identity phase's key moments (reference train/speedrun/moment_kernels.py:368-462,
//          moment_key_scores): bf16 q / k / v / hub, full causal window, the key's sq and step given;
//   SCAN   the key scan (moment_kernels.py:467-607, key_credits / key_and_raw_value_credits): fp32 q / k / v / hub
//          with tf32 logits and scores (kind::tf32 MMAs), receivers 0 <= s - t <= window, the key's step from its
//          own raw coordinates, and the optional value credits with hub split into bf16 hi + lo.
//
// Per key t and receiver s (logit x = q_s . k_t / 8, p = e^(x - lse_s), c = hub_s . v_t - center_s):
//   w1 = p c, w2 = (p / 2 - p^2) c, w2l = w2 x;  s1 = sum w1 x, s2 = sum w2 x^2 (fp32)
//   P2 = sum bf16(w1) f2_s, R2 = sum bf16(w2l) f2_s, Q2 = sum bf16(w2) g2_s, QXY = sum bf16(w2) xy_s,
//   VA = sum bf16(p) hub_s (IDENT) or sum bf16(p) (hi_s + lo_s) (SCAN)
// with the receivers' pair features f2 = (x_i, y_i), g2 = (x_i^2, y_i^2), xy = x_i y_i of side / 8 (bf16, from
// keymom_features_kernel), then per key the response of every raw coordinate through RoPE and the RMS norm.
//
// One work item = one 128-key tile of one row; receivers stream in 32-wide tiles. 320 threads, one CTA per SM:
//   warp 0      TMA: K, V once per item; per receiver tile q, hub, f2, g2, xy (and hi, lo) and lse / center into
//               a ring (5 stages IDENT, 2 SCAN);
//   warp 1      TMEM (512 columns): S = K Q^T and C = V H^T (32 columns each, double-buffered), the accumulators
//               P2 (64), R2 (64), Q2 | QXY (96: g2 and xy as one 96-wide B operand) and VA (64); the whole warp
//               runs the issue loop and an elect.sync lane issues S / C of tile j + AHEAD ahead of the moment MMAs of
//               tile j (M = 128 keys, K = 32 receivers);
//   warps 2..9  warp w: key rows of TMEM lane quarter w % 4, receivers half (w - 2) / 4 of each tile: the weights
//               as bf16 into one of two 64-byte-swizzled shared buffers (the moment MMAs' A operands), so a tile's
//               weights are written while the previous tile's moment MMAs run; at the item's end the response
//               epilogue for its 16 rotary pairs and 32 value columns.
#pragma once
#include "ptx.cuh"

namespace noise {
namespace credit {

constexpr int KM_B = 128, KM_R = 32, KM_THREADS = 320;
constexpr int KM_KT = KM_B * 128;       // [128][64] bf16 (or [128][32] fp32) key-side tile: 16 KB
constexpr int KM_RT = KM_R * 128;       // [32][64] bf16 (or [32][32] fp32) receiver-side tile: 4 KB
constexpr int KM_WT = KM_B * KM_R * 2;  // [128][32] bf16 weight matrix (64-byte rows): 8 KB
// TMEM columns: S / C buffer b at 64 b (S) and 64 b + 32 (C)
constexpr uint32_t KM_TSC = 0, KM_TP2 = 128, KM_TR2 = 192, KM_TQ2 = 256, KM_TXY = 320, KM_TVA = 384;

// VALS: the value sums are computed (always for IDENT; for SCAN when value credits are requested, which adds the hub's
// hi / lo tiles to every stage and leaves room for 2 stages instead of 3)
template <bool SCAN, bool VALS = true>
struct KmLayout {
  static constexpr int KV = SCAN ? 2 * KM_KT : KM_KT;  // K or V: fp32 as two 32-wide halves (128-byte rows)
  static constexpr int RQ = SCAN ? 2 * KM_RT : KM_RT;  // q or hub of a receiver tile
  static constexpr int K = 0, V = KV, W = 2 * KV;       // W: 2 buffers x (W1, W2, W2L, P)
  static constexpr int RING = W + 8 * KM_WT;
  // stage: q, hub, f2, g2, xy (g2 and xy adjacent: one 96-wide MN-major operand), [hi, lo], lse, center
  static constexpr int SQ = 0, SH = RQ, SF2 = 2 * RQ, SG2 = SF2 + KM_RT, SXY = SG2 + KM_RT, SHI = SXY + KM_RT,
                       SLO = SHI + KM_RT;
  static constexpr int SLSE = SCAN && VALS ? SLO + KM_RT : SHI, SCTR = SLSE + 128;
  static constexpr int STAGE = (SCTR + 128 + 1023) / 1024 * 1024;
  static constexpr int STAGES = SCAN ? (VALS ? 2 : 3) : 5;
  static constexpr int AHEAD = STAGES >= 3 ? 2 : 1;  // S / C run this many receiver tiles ahead of the moment MMAs
  static constexpr int SUMS = RING + STAGES * STAGE;  // s1, s2 and (SCAN) |raw|^2 per (half, key row)
  static constexpr int BAR = SUMS + 3 * 2 * 128 * 4;
  static constexpr int SMEM = BAR + 256 + 1024;
  static_assert(SMEM <= 227 * 1024, "shared memory per CTA");
};

// K-major operand in 64-byte swizzled rows (32 bf16 of K per row): 8-row groups 512 bytes apart, layout type 4
// (SWIZZLE_64B); the K step inside a row advances the start address by 32 bytes per 16 bf16 values.
__device__ __forceinline__ uint64_t km_sdesc_kmajor_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(512u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(4u) << 61;
  return d;
}

struct KeyMomTcArgs {
  int T, window, rows;
  Rows raw;
  int raw_bf16, out_bf16;
  const float *sq, *steps;     // IDENT: [rows, T]
  float sigma;                 // SCAN: step = sigma max(rms(k_raw[t]), 1e-6)
  const float *cosb, *sinb;    // [T, 32]
  Rows out, vout;              // vout.data NULL (SCAN): no value credits
  int* status;
};

// The receivers' pair features of side / 8 (fp32 [rows * T, 64]): f2 = (x_i, y_i) interleaved, g2 = (x_i^2,
// y_i^2) interleaved, xy = (x_i y_i, then 32 zeros), bf16 [rows * T, 64] each; one thread per (token, pair).
__global__ void __launch_bounds__(256) keymom_features_kernel(const float* __restrict__ side, int64_t n_pairs,
                                                             __nv_bfloat16* __restrict__ f2,
                                                             __nv_bfloat16* __restrict__ g2,
                                                             __nv_bfloat16* __restrict__ xy) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n_pairs;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t tok = i >> 5;
    const int pr = static_cast<int>(i & 31);
    const float x = side[tok * 64 + pr] * 0.125f, y = side[tok * 64 + pr + 32] * 0.125f;
    reinterpret_cast<uint32_t*>(f2 + tok * 64)[pr] = pack_bf16x2(x, y);
    reinterpret_cast<uint32_t*>(g2 + tok * 64)[pr] = pack_bf16x2(x * x, y * y);
    xy[tok * 64 + pr] = __float2bfloat16_rn(x * y);
    xy[tok * 64 + 32 + pr] = __float2bfloat16_rn(0.f);
  }
}

__device__ __forceinline__ void km_st_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
struct KeyMomMaps {
  CUtensorMap k, v;                // [rows * T, 64]: bf16 128 x 64 boxes (IDENT) or fp32 128 x 32 boxes (SCAN)
  CUtensorMap q, h;                // [rows * T, 64]: bf16 32 x 64 boxes or fp32 32 x 32 boxes
  CUtensorMap f2, g2, xy, hi, lo;  // bf16 [rows * T, 64], 32 x 64 boxes
  CUtensorMap lse, ctr;            // fp32 [rows, T], 32 x 1 boxes
};

template <bool SCAN, bool VALS = true>
__global__ void __launch_bounds__(KM_THREADS, 1)
    keymom_tc_kernel(const __grid_constant__ KeyMomMaps m, const __grid_constant__ KeyMomTcArgs p) {
  using L = KmLayout<SCAN, VALS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L::BAR);
  uint64_t* kv_full = bar;
  uint64_t* kv_empty = bar + 1;
  uint64_t* st_full = bar + 2;               // STAGES
  uint64_t* st_empty = st_full + L::STAGES;  // STAGES
  uint64_t* s_full = st_empty + L::STAGES;   // 2 (S / C buffers)
  uint64_t* s_empty = s_full + 2;            // 2
  uint64_t* w_full = s_empty + 2;            // 2 (weight buffers)
  uint64_t* w_empty = w_full + 2;            // 2
  uint64_t* acc_full = w_empty + 2;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* drain = acc_empty + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkt = p.T / KM_B, nrt = p.T / KM_R;
  const int items = nkt * p.rows;
  constexpr bool values = !SCAN || VALS;
  // item w: key tile w / rows (the first tiles have the most receivers: heaviest first) of row w % rows; its
  // receiver tiles run from the key tile's first receivers to the window's end
  auto tiles_of = [&](int kt, int& lo, int& hi) {
    lo = kt * KM_B / KM_R;
    hi = min((kt * KM_B + KM_B - 1 + p.window) / KM_R, nrt - 1);
  };

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_empty, 1);
    for (int s = 0; s < L::STAGES; ++s) {
      mbar_init(&st_full[s], 1);
      mbar_init(&st_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 8);  // one arrival per weight warp (its lanes joined by __syncwarp first)
      mbar_init(&w_full[b], 8);
      mbar_init(&w_empty[b], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 8);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    const CUtensorMap* maps[11] = {&m.k, &m.v, &m.q, &m.h, &m.f2, &m.g2, &m.xy, &m.lse, &m.ctr, &m.hi, &m.lo};
    for (int i = 0; i < (SCAN && values ? 11 : 9); ++i) tma_prefetch_desc(maps[i]);
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
      const uint32_t stage_tx = 2 * L::RQ + 3 * KM_RT + (SCAN && values ? 2 * KM_RT : 0) + 2 * KM_R * 4;
      for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++nitem) {
        const int kt = w / p.rows, row = w % p.rows;
        const int row0 = row * p.T;
        int lo, hi;
        tiles_of(kt, lo, hi);
        if (!mbar_wait(kv_empty, (static_cast<uint32_t>(nitem) & 1u) ^ 1u, p.status)) break;
        mbar_arrive_expect_tx(kv_full, 2 * L::KV);
        tma_load_2d(smem + L::K, &m.k, kv_full, 0, row0 + kt * KM_B);
        tma_load_2d(smem + L::V, &m.v, kv_full, 0, row0 + kt * KM_B);
        if constexpr (SCAN) {  // the fp32 rows' second 32-wide half
          tma_load_2d(smem + L::K + KM_KT, &m.k, kv_full, 32, row0 + kt * KM_B);
          tma_load_2d(smem + L::V + KM_KT, &m.v, kv_full, 32, row0 + kt * KM_B);
        }
        for (int j = lo; j <= hi; ++j, ++sv) {
          const int sl = sv % L::STAGES;
          if (!mbar_wait(&st_empty[sl], (static_cast<uint32_t>(sv / L::STAGES) & 1u) ^ 1u, p.status)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + L::RING + sl * L::STAGE;
          uint64_t* b = &st_full[sl];
          const int r = row0 + j * KM_R;
          mbar_arrive_expect_tx(b, stage_tx);
          tma_load_2d(st + L::SQ, &m.q, b, 0, r);
          tma_load_2d(st + L::SH, &m.h, b, 0, r);
          if constexpr (SCAN) {
            tma_load_2d(st + L::SQ + KM_RT, &m.q, b, 32, r);
            tma_load_2d(st + L::SH + KM_RT, &m.h, b, 32, r);
            if (values) {
              tma_load_2d(st + L::SHI, &m.hi, b, 0, r);
              tma_load_2d(st + L::SLO, &m.lo, b, 0, r);
            }
          }
          tma_load_2d(st + L::SF2, &m.f2, b, 0, r);
          tma_load_2d(st + L::SG2, &m.g2, b, 0, r);
          tma_load_2d(st + L::SXY, &m.xy, b, 0, r);
          tma_load_2d(st + L::SLSE, &m.lse, b, j * KM_R, row);
          tma_load_2d(st + L::SCTR, &m.ctr, b, j * KM_R, row);
        }
      }
      if (nitem > 0) mbar_wait(kv_full, static_cast<uint32_t>(nitem - 1) & 1u, p.status);
      for (int j = sv - 1; j >= 0 && j >= sv - L::STAGES; --j)
        mbar_wait(&st_full[j % L::STAGES], static_cast<uint32_t>(j / L::STAGES) & 1u, p.status);
    }
  } else if (warp == 1) {
    {  // the whole warp runs the issuer; one elected lane issues the MMAs and commits
      constexpr uint32_t id_s = SCAN ? idesc_tf32(KM_B, KM_R) : idesc_bf16(KM_B, KM_R);  // S, C (K-major B)
      constexpr uint32_t id_f = idesc_bf16(KM_B, 64, false, true);   // P2, R2, VA: B MN-major
      constexpr uint32_t id_q = idesc_bf16(KM_B, 96, false, true);   // Q2 | QXY
      int sv = 0, nitem = 0;
      bool ok = true;
      // the moment MMAs of the receiver tile with global index svj (the item's first when first)
      auto moments = [&](int svj, bool first) {
        const int wb = svj & 1;
        if (!mbar_wait_warp(&w_full[wb], static_cast<uint32_t>(svj >> 1) & 1u, p.status)) return false;
        tc_fence_after();
        const uint32_t st = sbase + L::RING + (svj % L::STAGES) * L::STAGE;
        const uint32_t w = sbase + L::W + wb * 4 * KM_WT;  // W1, W2, W2L, P
#pragma unroll
        for (int ks = 0; ks < KM_R / 16; ++ks) {
          const uint32_t acc = (first && ks == 0) ? 0u : 1u;
          const uint64_t f2d = sdesc_mnmajor_sw128(st + L::SF2 + ks * 2048, 16);
          if (elect_one()) tc_mma(tmem + KM_TP2, km_sdesc_kmajor_sw64(w) + 2u * ks, f2d, id_f, acc);
          if (elect_one()) tc_mma(tmem + KM_TR2, km_sdesc_kmajor_sw64(w + 2 * KM_WT) + 2u * ks, f2d, id_f, acc);
          if (elect_one()) tc_mma(tmem + KM_TQ2, km_sdesc_kmajor_sw64(w + KM_WT) + 2u * ks,
                 sdesc_mnmajor_sw128(st + L::SG2 + ks * 2048, KM_RT), id_q, acc);
          if constexpr (SCAN) {
            if (values) {
              const uint64_t pd = km_sdesc_kmajor_sw64(w + 3 * KM_WT) + 2u * ks;
              if (elect_one()) tc_mma(tmem + KM_TVA, pd, sdesc_mnmajor_sw128(st + L::SHI + ks * 2048, 16), id_f, acc);
              if (elect_one()) tc_mma(tmem + KM_TVA, pd, sdesc_mnmajor_sw128(st + L::SLO + ks * 2048, 16), id_f, 1u);
            }
          } else {
            if (elect_one()) tc_mma(tmem + KM_TVA, km_sdesc_kmajor_sw64(w + 3 * KM_WT) + 2u * ks,
                   sdesc_mnmajor_sw128(st + L::SH + ks * 2048, 16), id_f, acc);
          }
        }
        if (elect_one()) tc_commit(&w_empty[wb]);
        if (elect_one()) tc_commit(&st_empty[svj % L::STAGES]);
        return true;
      };
      for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++nitem) {
        const int kt = w / p.rows;
        int lo, hi;
        tiles_of(kt, lo, hi);
        if (!mbar_wait_warp(kv_full, static_cast<uint32_t>(nitem) & 1u, p.status)) {
          ok = false;
          break;
        }
        // the accumulators are free once the previous item's epilogue has read them (S / C may start before)
        auto acc_free = [&]() { return mbar_wait_warp(acc_empty, (static_cast<uint32_t>(nitem) & 1u) ^ 1u, p.status); };
        // S / C of the tile with global index svj into buffer svj & 1 (free once the tile two back was read)
        auto scores = [&](int svj) {
          const int sl = svj % L::STAGES, b = svj & 1;
          if (!mbar_wait_warp(&st_full[sl], static_cast<uint32_t>(svj / L::STAGES) & 1u, p.status) ||
              !mbar_wait_warp(&s_empty[b], (static_cast<uint32_t>(svj >> 1) & 1u) ^ 1u, p.status))
            return false;
          tc_fence_after();
          const uint32_t st = sbase + L::RING + sl * L::STAGE;
          const uint32_t ts = tmem + KM_TSC + b * 64;
          if constexpr (SCAN) {  // tf32: 8 K-steps of 8, 4 per 32-wide half
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const uint32_t ho = (k >> 2);
              if (elect_one()) tc_mma_tf32(ts, sdesc_kmajor_sw128(sbase + L::K + ho * KM_KT) + 2u * (k & 3),
                          sdesc_kmajor_sw128(st + L::SQ + ho * KM_RT) + 2u * (k & 3), id_s, k > 0);
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const uint32_t ho = (k >> 2);
              if (elect_one()) tc_mma_tf32(ts + 32, sdesc_kmajor_sw128(sbase + L::V + ho * KM_KT) + 2u * (k & 3),
                          sdesc_kmajor_sw128(st + L::SH + ho * KM_RT) + 2u * (k & 3), id_s, k > 0);
            }
          } else {
            const uint64_t kd = sdesc_kmajor_sw128(sbase + L::K), vd = sdesc_kmajor_sw128(sbase + L::V);
            const uint64_t qd = sdesc_kmajor_sw128(st + L::SQ), hd = sdesc_kmajor_sw128(st + L::SH);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              if (elect_one()) tc_mma(ts, kd + 2u * k, qd + 2u * k, id_s, k > 0);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              if (elect_one()) tc_mma(ts + 32, vd + 2u * k, hd + 2u * k, id_s, k > 0);
          }
          if (elect_one()) tc_commit(&s_full[b]);
          return true;
        };
        // S / C run AHEAD tiles ahead of the moment MMAs, so a tile's moments issue as soon as its weights are
        // written (not behind the next tile's loads)
        const int sv0 = sv;
        for (int a = 0; a < L::AHEAD && ok && lo + a <= hi; ++a) ok = scores(sv0 + a);
        for (int j = lo; j <= hi && ok; ++j, ++sv) {
          if (j == lo) ok = acc_free();
          if (ok) ok = moments(sv, j == lo);
          if (ok && j + L::AHEAD <= hi) ok = scores(sv + L::AHEAD);
        }
        if (ok) {
          if (elect_one()) tc_commit(kv_empty);
          if (elect_one()) tc_commit(acc_full);
        }
      }
      if (elect_one()) tc_commit(drain);
      mbar_wait_warp(drain, 0, p.status);
    }
  } else {
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;  // key row of the tile
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t trow = tmem + lane_base;
    float* sums = reinterpret_cast<float*>(smem + L::SUMS);  // [half][3][128]: s1, s2, |raw|^2
    constexpr float SL2 = 0.125f * 1.4426950408889634f;
    constexpr float L2E = 1.4426950408889634f;
    int sv = 0, nitem = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++nitem) {
      const int kt = w / p.rows, row = w % p.rows;
      const int tk = kt * KM_B + r;
      int lo, hi;
      tiles_of(kt, lo, hi);
      float2 s1p = make_float2(0.f, 0.f), s2p = make_float2(0.f, 0.f);  // even / odd receivers' partial sums
      for (int j = lo; j <= hi && ok; ++j, ++sv) {
        const int b = sv & 1;
        if (!mbar_wait(&s_full[b], static_cast<uint32_t>(sv >> 1) & 1u, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float s[16], c[16];
        tmem_ld16(trow + KM_TSC + b * 64 + half * 16, s);
        tmem_ld16(trow + KM_TSC + b * 64 + 32 + half * 16, c);
        tc_wait_ld();
        reg_fence<16>(s);
        reg_fence<16>(c);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[b]);
        const uint8_t* st = smem + L::RING + (sv % L::STAGES) * L::STAGE;
        const float* lse = reinterpret_cast<const float*>(st + L::SLSE) + half * 16;
        const float* ctr = reinterpret_cast<const float*>(st + L::SCTR) + half * 16;
        const int s0 = j * KM_R + half * 16;
        const bool full = s0 >= kt * KM_B + KM_B - 1 && s0 + 15 - kt * KM_B <= p.window;
        uint32_t pw1[8], pw2[8], pw2l[8], pp[8];
        // receivers in pairs: packed fp32x2 arithmetic, two exponentials on the MUFU pipe
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          const float2 sc = make_float2(s[e], s[e + 1]);
          const float2 logit = __fmul2_rn(sc, make_float2(0.125f, 0.125f));
          const float2 arg = __ffma2_rn(sc, make_float2(SL2, SL2), __fmul2_rn(make_float2(-lse[e], -lse[e + 1]),
                                                                               make_float2(L2E, L2E)));
          float2 a = make_float2(ex2_approx(arg.x), ex2_approx(arg.y));
          if (!full) {
            if (s0 + e < tk || s0 + e - tk > p.window) a.x = 0.f;
            if (s0 + e + 1 < tk || s0 + e + 1 - tk > p.window) a.y = 0.f;
          }
          const float2 cc = __fadd2_rn(make_float2(c[e], c[e + 1]), make_float2(-ctr[e], -ctr[e + 1]));
          const float2 x1 = __fmul2_rn(a, cc);
          const float2 half_a = __fmul2_rn(make_float2(0.5f, 0.5f), a);
          const float2 x2 = __fmul2_rn(__ffma2_rn(make_float2(-a.x, -a.y), a, half_a), cc);  // (a / 2 - a^2) c
          const float2 x2l = __fmul2_rn(x2, logit);
          s1p = __ffma2_rn(x1, logit, s1p);
          s2p = __ffma2_rn(x2l, logit, s2p);
          pw1[e / 2] = pack_bf16x2(x1.x, x1.y);
          pw2[e / 2] = pack_bf16x2(x2.x, x2.y);
          pw2l[e / 2] = pack_bf16x2(x2l.x, x2l.y);
          pp[e / 2] = pack_bf16x2(a.x, a.y);
        }
        if (!mbar_wait(&w_empty[b], (static_cast<uint32_t>(sv >> 1) & 1u) ^ 1u, p.status)) {
          ok = false;
          break;
        }
        // row r, receivers half * 16 .. + 15: 16-byte chunks half * 2 + i of the 64-byte row, 64-byte swizzle
        const uint32_t wrow = sbase + L::W + b * 4 * KM_WT + r * 64;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const uint32_t off = static_cast<uint32_t>(((half * 2 + i) ^ ((r >> 1) & 3)) << 4);
          km_st_v4(wrow + off, pw1[4 * i], pw1[4 * i + 1], pw1[4 * i + 2], pw1[4 * i + 3]);
          km_st_v4(wrow + KM_WT + off, pw2[4 * i], pw2[4 * i + 1], pw2[4 * i + 2], pw2[4 * i + 3]);
          km_st_v4(wrow + 2 * KM_WT + off, pw2l[4 * i], pw2l[4 * i + 1], pw2l[4 * i + 2], pw2l[4 * i + 3]);
          km_st_v4(wrow + 3 * KM_WT + off, pp[4 * i], pp[4 * i + 1], pp[4 * i + 2], pp[4 * i + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&w_full[b]);
      }
      ok = __all_sync(0xffffffffu, ok);
      // the two halves' s1 / s2 of each key row
      // this thread's 32 raw coordinates d = half * 16 + i and 32 + half * 16 + i (and SCAN: their square sum)
      const int64_t ro = p.raw.at(row, tk, p.T);
      float rv[32];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        rv[i] = raw_at(p.raw, p.raw_bf16, ro + half * 16 + i);
        rv[16 + i] = raw_at(p.raw, p.raw_bf16, ro + 32 + half * 16 + i);
      }
      float rsq = 0.f;
      if constexpr (SCAN) {
#pragma unroll
        for (int i = 0; i < 32; ++i) rsq = fmaf(rv[i], rv[i], rsq);
      }
      sums[(half * 3) * 128 + r] = s1p.x + s1p.y;
      sums[(half * 3 + 1) * 128 + r] = s2p.x + s2p.y;
      sums[(half * 3 + 2) * 128 + r] = rsq;
      if (!bar_and<KM_THREADS - 64>(ok)) {
        ok = false;
        break;
      }
      const float a1 = sums[r] + sums[3 * 128 + r], a2 = sums[128 + r] + sums[4 * 128 + r];
      const float rsq_all = sums[2 * 128 + r] + sums[5 * 128 + r];
      // a thread whose wait gives up skips the epilogue but still reaches the item's closing barrier
      const bool got = __all_sync(0xffffffffu, mbar_wait(acc_full, static_cast<uint32_t>(nitem) & 1u, p.status));
      tc_fence_after();
      // response per raw coordinate d = P and P + 32 of this half's pairs P = half * 16 + g * 8 + i, 8 pairs at a time
      float stepv, den;
      if constexpr (SCAN) {  // the key's own step: sigma max(rms(k_raw[t]), 1e-6), RMS eps = finfo(fp32).eps
        const float sqv = rsq_all / D;
        stepv = p.sigma * fmaxf(sqrtf(sqv), 1e-6f);
        den = sqv + 1.1920928955078125e-07f;
      } else {
        stepv = p.steps[static_cast<int64_t>(row) * p.T + tk];
        den = p.sq[static_cast<int64_t>(row) * p.T + tk] / D + 1e-6f;
      }
      // per key: ratio = (2 step raw + step^2) / 64 / den = ka raw + kb, response / step = response * rstep
      const float inv = 1.f / (D * den);
      const float ka = 2.f * stepv * inv, kb = stepv * stepv * inv, cbk = stepv * rsqrtf(den), rstep = 1.f / stepv;
      const int64_t oo = p.out.at(row, tk, p.T);
#pragma unroll 1
      for (int g8 = 0; g8 < (got ? 2 : 0); ++g8) {
        float p2[16], r2[16], q2[16], xy[16];
        tmem_ld16(trow + KM_TP2 + half * 32 + g8 * 16, p2);
        tmem_ld16(trow + KM_TR2 + half * 32 + g8 * 16, r2);
        tmem_ld16(trow + KM_TQ2 + half * 32 + g8 * 16, q2);
        tmem_ld16(trow + KM_TXY + half * 16, xy);
        tc_wait_ld();
        reg_fence<16>(p2);
        reg_fence<16>(r2);
        reg_fence<16>(q2);
        reg_fence<16>(xy);
        const int P0 = half * 16 + g8 * 8;  // this chunk's 8 rotary pairs: cos / sin as two float4 each
        const float4 c0 = *reinterpret_cast<const float4*>(p.cosb + static_cast<int64_t>(tk) * 32 + P0);
        const float4 c1 = *reinterpret_cast<const float4*>(p.cosb + static_cast<int64_t>(tk) * 32 + P0 + 4);
        const float4 n0 = *reinterpret_cast<const float4*>(p.sinb + static_cast<int64_t>(tk) * 32 + P0);
        const float4 n1 = *reinterpret_cast<const float4*>(p.sinb + static_cast<int64_t>(tk) * 32 + P0 + 4);
        const float csv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
        const float snv[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
#pragma unroll 1
        for (int hf = 0; hf < 2; ++hf) {  // coordinates d = P + 32 hf
          float res[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            // ca = (1 + ratio)^(-1/2) - 1 = -ratio s^2 / (1 + s), s = (1 + ratio)^(-1/2): no cancellation for small
            // ratios (the reference's expm1(-log1p(ratio) / 2))
            const float ratio = fmaf(ka, (g8 ? (hf ? rv[24 + i] : rv[8 + i]) : (hf ? rv[16 + i] : rv[i])), kb);
            const float sr = rsqrtf(1.f + ratio);
            const float ca = __fdividef(-ratio * sr * sr, 1.f + sr);
            const float cb = cbk * (1.f + ca);
            const float bu = cb * (hf ? snv[i] : csv[i]), bw = cb * (hf ? csv[i] : -snv[i]);
            const float cxy = g8 ? xy[8 + i] : xy[i];
            const float resp = p2[2 * i] * bu + p2[2 * i + 1] * bw + q2[2 * i] * bu * bu + q2[2 * i + 1] * bw * bw +
                               2.f * cxy * bu * bw + 2.f * ca * (r2[2 * i] * bu + r2[2 * i + 1] * bw) + a1 * ca +
                               a2 * ca * ca;
            res[i] = resp * rstep;
          }
          const int64_t o = oo + hf * 32 + half * 16 + g8 * 8;  // 8 consecutive coordinates (host: 16-byte strides)
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
      // value sums: 32 columns of VA
      float va[32];
      if (values && got) {
        tmem_ld32(trow + KM_TVA + half * 32, va);
        tc_wait_ld();
        reg_fence<32>(va);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
      if (!values || !got) {
        if (!bar_and<KM_THREADS - 64>(got)) {  // both halves have read sums before the next item overwrites them
          ok = false;
          break;
        }
        continue;
      }
      const int64_t vo = p.vout.at(row, tk, p.T) + half * 32;
      if (p.out_bf16) {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.vout.data) + vo);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          dst[q] = make_uint4(pack_bf16x2(va[8 * q], va[8 * q + 1]), pack_bf16x2(va[8 * q + 2], va[8 * q + 3]),
                              pack_bf16x2(va[8 * q + 4], va[8 * q + 5]), pack_bf16x2(va[8 * q + 6], va[8 * q + 7]));
      } else {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.vout.data) + vo);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          dst[q] = make_float4(va[4 * q], va[4 * q + 1], va[4 * q + 2], va[4 * q + 3]);
      }
      if (!bar_and<KM_THREADS - 64>(true)) {  // both halves have read sums before the next item overwrites them
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
