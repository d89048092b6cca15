// The identity phase's key moments on tcgen05 (sm_100a): per key t and raw key coordinate d the degree-2 moment
// response of the receivers' softmax to a finite step of k_raw[t, d], and the value sums sum_s p hub_s (reference
// train/speedrun/moment_kernels.py:368-462, moment_key_scores; bf16 operands, full causal window).
//
// Per key t and receiver s >= t (logit x = q_s . k_t / 8, p = e^(x - lse_s), c = hub_s . v_t - center_s):
//   w1 = p c, w2 = (p / 2 - p^2) c, w2l = w2 x;  s1 = sum w1 x, s2 = sum w2 x^2 (fp32)
//   P2 = sum bf16(w1) f2_s, R2 = sum bf16(w2l) f2_s, Q2 = sum bf16(w2) g2_s, QXY = sum bf16(w2) xy_s,
//   VA = sum bf16(p) hub_s
// with the receivers' pair features f2 = (x_i, y_i), g2 = (x_i^2, y_i^2), xy = x_i y_i of side / 8 (bf16, from
// keymom_features_kernel), then per key the response of every raw coordinate through RoPE and the RMS norm.
//
// One work item = one 128-key tile of one row; receivers stream in 64-wide tiles. 320 threads, one CTA per SM:
//   warp 0      TMA: K, V once per item; per receiver tile q, hub, f2, g2, xy (64 rows each) and lse / center
//               into a 2-stage ring;
//   warp 1      TMEM (512 columns): S (64) = K Q^T, C (64) = V H^T, then the accumulators P2 (64), R2 (64),
//               Q2 | QXY (128: g2 and the zero-padded xy as one 128-wide B operand) and VA (64); one lane issues
//               S / C of tile j, then the moment MMAs of tile j - 1 (M = 128 keys, K = 64 receivers);
//   warps 2..9  warp w: key rows of TMEM lane quarter w % 4, receiver half (w - 2) / 4 of each tile: the weights
//               as bf16 into swizzled shared memory (the moment MMAs' A operands); at the item's end the response
//               epilogue for its 16 rotary pairs and 32 value columns.
#pragma once
#include "ptx.cuh"

namespace noise {
namespace credit {

constexpr int KM_B = 128, KM_R = 64, KM_STAGES = 2, KM_THREADS = 320;
constexpr int KM_KT = KM_B * 128;            // [128][64] bf16 key-side tile: 16 KB
constexpr int KM_RT = KM_R * 128;            // [64][64] bf16 receiver-side tile: 8 KB
constexpr int KM_K = 0, KM_V = KM_KT;
constexpr int KM_W = 2 * KM_KT;              // W1, W2, W2L, P: [128][64] bf16 each
constexpr int KM_RING = KM_W + 4 * KM_KT;
// stage: q, hub, f2, g2, xy (g2 and xy adjacent: one 128-wide MN-major operand), then lse, center (64 floats each)
constexpr int KM_SQ = 0, KM_SH = KM_RT, KM_SF2 = 2 * KM_RT, KM_SG2 = 3 * KM_RT, KM_SXY = 4 * KM_RT,
              KM_SLSE = 5 * KM_RT, KM_SCTR = KM_SLSE + 256;
constexpr int KM_STAGE = 5 * KM_RT + 1024;
constexpr int KM_SUMS = KM_RING + KM_STAGES * KM_STAGE;  // s1 / s2 per (half, key row): 2 x 2 x 128 floats
constexpr int KM_BAR = KM_SUMS + 2048;
constexpr int KM_SMEM = KM_BAR + 256 + 1024;
// TMEM columns
constexpr uint32_t KM_TS = 0, KM_TC = 64, KM_TP2 = 128, KM_TR2 = 192, KM_TQ2 = 256, KM_TXY = 320, KM_TVA = 384;

struct KeyMomTcArgs {
  int T, window, rows;
  Rows raw;
  int raw_bf16, out_bf16;
  const float *sq, *steps;     // [rows, T]
  const float *cosb, *sinb;    // [T, 32]
  Rows out, vout;
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
__device__ __forceinline__ void km_bar_sync() {  // named barrier 1 over the 256 weight / epilogue threads
  asm volatile("bar.sync 1, 256;" ::: "memory");
}

struct KeyMomMaps {
  CUtensorMap k, v;           // bf16 [rows * T, 64], 128-row boxes
  CUtensorMap q, h, f2, g2, xy;  // bf16 [rows * T, 64], 64-row boxes
  CUtensorMap lse, ctr;       // fp32 [rows, T], 64 x 1 boxes
};

__global__ void __launch_bounds__(KM_THREADS, 1)
    keymom_tc_kernel(const __grid_constant__ KeyMomMaps m, const __grid_constant__ KeyMomTcArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + KM_BAR);
  uint64_t* kv_full = bar;
  uint64_t* kv_empty = bar + 1;
  uint64_t* st_full = bar + 2;              // STAGES
  uint64_t* st_empty = st_full + KM_STAGES;  // STAGES
  uint64_t* s_full = st_empty + KM_STAGES;
  uint64_t* s_empty = s_full + 1;
  uint64_t* w_full = s_empty + 1;
  uint64_t* w_empty = w_full + 1;
  uint64_t* acc_full = w_empty + 1;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* drain = acc_empty + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkt = p.T / KM_B, nrt = p.T / KM_R;
  const int items = nkt * p.rows;
  // item w: key tile w / rows (the first tiles have the most receivers: heaviest first) of row w % rows; its
  // receiver tiles run from the key tile's first 64 receivers to the window's end
  auto tiles_of = [&](int kt, int& lo, int& hi) {
    lo = kt * KM_B / KM_R;
    hi = min((kt * KM_B + KM_B - 1 + p.window) / KM_R, nrt - 1);
  };

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_empty, 1);
    for (int s = 0; s < KM_STAGES; ++s) {
      mbar_init(&st_full[s], 1);
      mbar_init(&st_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, 256);
    mbar_init(w_full, 256);
    mbar_init(w_empty, 1);
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 256);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    const CUtensorMap* maps[9] = {&m.k, &m.v, &m.q, &m.h, &m.f2, &m.g2, &m.xy, &m.lse, &m.ctr};
    for (int i = 0; i < 9; ++i) tma_prefetch_desc(maps[i]);
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
        const int kt = w / p.rows, row = w % p.rows;
        const int row0 = row * p.T;
        int lo, hi;
        tiles_of(kt, lo, hi);
        if (!mbar_wait(kv_empty, (static_cast<uint32_t>(nitem) & 1u) ^ 1u, p.status)) break;
        mbar_arrive_expect_tx(kv_full, 2 * KM_KT);
        tma_load_2d(smem + KM_K, &m.k, kv_full, 0, row0 + kt * KM_B);
        tma_load_2d(smem + KM_V, &m.v, kv_full, 0, row0 + kt * KM_B);
        for (int j = lo; j <= hi; ++j, ++sv) {
          const int sl = sv % KM_STAGES;
          if (!mbar_wait(&st_empty[sl], (static_cast<uint32_t>(sv / KM_STAGES) & 1u) ^ 1u, p.status)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + KM_RING + sl * KM_STAGE;
          uint64_t* b = &st_full[sl];
          const int r = row0 + j * KM_R;
          mbar_arrive_expect_tx(b, 5 * KM_RT + 2 * KM_R * 4);
          tma_load_2d(st + KM_SQ, &m.q, b, 0, r);
          tma_load_2d(st + KM_SH, &m.h, b, 0, r);
          tma_load_2d(st + KM_SF2, &m.f2, b, 0, r);
          tma_load_2d(st + KM_SG2, &m.g2, b, 0, r);
          tma_load_2d(st + KM_SXY, &m.xy, b, 0, r);
          tma_load_2d(st + KM_SLSE, &m.lse, b, j * KM_R, row);
          tma_load_2d(st + KM_SCTR, &m.ctr, b, j * KM_R, row);
        }
      }
      if (nitem > 0) mbar_wait(kv_full, static_cast<uint32_t>(nitem - 1) & 1u, p.status);
      for (int j = sv - 1; j >= 0 && j >= sv - KM_STAGES; --j)
        mbar_wait(&st_full[j % KM_STAGES], static_cast<uint32_t>(j / KM_STAGES) & 1u, p.status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_bf16(KM_B, KM_R);             // S, C: B = q / hub rows (K-major)
      constexpr uint32_t id_f = idesc_bf16(KM_B, 64, false, true);  // P2, R2, VA: B MN-major
      constexpr uint32_t id_q = idesc_bf16(KM_B, 128, false, true);  // Q2 | QXY
      int sv = 0, nitem = 0;
      bool ok = true;
      // the moment MMAs of the receiver tile in ring slot svj (the item's first when first)
      auto moments = [&](int svj, bool first) {
        if (!mbar_wait(w_full, static_cast<uint32_t>(svj) & 1u, p.status)) return false;
        tc_fence_after();
        const uint32_t st = sbase + KM_RING + (svj % KM_STAGES) * KM_STAGE;
        const uint32_t w = sbase + KM_W;
#pragma unroll
        for (int ks = 0; ks < KM_R / 16; ++ks) {
          const uint32_t acc = (first && ks == 0) ? 0u : 1u;
          const uint64_t f2d = sdesc_mnmajor_sw128(st + KM_SF2 + ks * 2048, 16);
          tc_mma(tmem + KM_TP2, sdesc_kmajor_sw128(w) + 2u * ks, f2d, id_f, acc);
          tc_mma(tmem + KM_TR2, sdesc_kmajor_sw128(w + 2 * KM_KT) + 2u * ks, f2d, id_f, acc);
          tc_mma(tmem + KM_TQ2, sdesc_kmajor_sw128(w + KM_KT) + 2u * ks,
                 sdesc_mnmajor_sw128(st + KM_SG2 + ks * 2048, KM_RT), id_q, acc);
          tc_mma(tmem + KM_TVA, sdesc_kmajor_sw128(w + 3 * KM_KT) + 2u * ks,
                 sdesc_mnmajor_sw128(st + KM_SH + ks * 2048, 16), id_f, acc);
        }
        tc_commit(w_empty);
        tc_commit(&st_empty[svj % KM_STAGES]);
        return true;
      };
      for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++nitem) {
        const int kt = w / p.rows;
        int lo, hi;
        tiles_of(kt, lo, hi);
        if (!mbar_wait(kv_full, static_cast<uint32_t>(nitem) & 1u, p.status) ||
            !mbar_wait(acc_empty, (static_cast<uint32_t>(nitem) & 1u) ^ 1u, p.status)) {
          ok = false;
          break;
        }
        const int sv0 = sv;
        for (int j = lo; j <= hi && ok; ++j, ++sv) {
          const int sl = sv % KM_STAGES;
          if (!mbar_wait(&st_full[sl], static_cast<uint32_t>(sv / KM_STAGES) & 1u, p.status) ||
              !mbar_wait(s_empty, (static_cast<uint32_t>(sv) & 1u) ^ 1u, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = sbase + KM_RING + sl * KM_STAGE;
          const uint64_t kd = sdesc_kmajor_sw128(sbase + KM_K), vd = sdesc_kmajor_sw128(sbase + KM_V);
          const uint64_t qd = sdesc_kmajor_sw128(st + KM_SQ), hd = sdesc_kmajor_sw128(st + KM_SH);
#pragma unroll
          for (int k = 0; k < 4; ++k) tc_mma(tmem + KM_TS, kd + 2u * k, qd + 2u * k, id_s, k > 0);
#pragma unroll
          for (int k = 0; k < 4; ++k) tc_mma(tmem + KM_TC, vd + 2u * k, hd + 2u * k, id_s, k > 0);
          tc_commit(s_full);
          if (j > lo) ok = moments(sv - 1, j - 1 == lo);
        }
        if (ok) ok = moments(sv - 1, hi == lo);
        if (ok) {
          tc_commit(kv_empty);
          tc_commit(acc_full);
        }
        (void)sv0;
      }
      tc_commit(drain);
      mbar_wait(drain, 0, p.status);
    }
  } else {
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;  // key row of the tile
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t trow = tmem + lane_base;
    float* sums = reinterpret_cast<float*>(smem + KM_SUMS);  // [half][2][128]
    constexpr float SL2 = 0.125f * 1.4426950408889634f;
    constexpr float L2E = 1.4426950408889634f;
    int sv = 0, nitem = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++nitem) {
      const int kt = w / p.rows, row = w % p.rows;
      const int tk = kt * KM_B + r;
      int lo, hi;
      tiles_of(kt, lo, hi);
      float s1 = 0.f, s2 = 0.f;
      for (int j = lo; j <= hi && ok; ++j, ++sv) {
        if (!mbar_wait(s_full, static_cast<uint32_t>(sv) & 1u, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float s[32], c[32];
        tmem_ld32(trow + KM_TS + half * 32, s);
        tmem_ld32(trow + KM_TC + half * 32, c);
        tc_wait_ld();
        reg_fence<32>(s);
        reg_fence<32>(c);
        tc_fence_before();
        mbar_arrive(s_empty);
        const uint8_t* st = smem + KM_RING + (sv % KM_STAGES) * KM_STAGE;
        const float* lse = reinterpret_cast<const float*>(st + KM_SLSE) + half * 32;
        const float* ctr = reinterpret_cast<const float*>(st + KM_SCTR) + half * 32;
        const int s0 = j * KM_R + half * 32;
        const bool full = s0 >= tk - r + KM_B - 1 && s0 + 31 - (tk - r) <= p.window;
        uint32_t pw1[16], pw2[16], pw2l[16], pp[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float x1v[2], x2v[2], x2lv[2], av[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const float logit = s[e + u] * 0.125f;
            float a = ex2_approx(fmaf(s[e + u], SL2, -lse[e + u] * L2E));
            if (!full) {
              const int sr = s0 + e + u;
              if (sr < tk || sr - tk > p.window) a = 0.f;
            }
            const float cc = c[e + u] - ctr[e + u];
            const float x1 = a * cc, x2 = (0.5f * a - a * a) * cc;
            s1 += x1 * logit;
            s2 += x2 * logit * logit;
            x1v[u] = x1;
            x2v[u] = x2;
            x2lv[u] = x2 * logit;
            av[u] = a;
          }
          pw1[e / 2] = pack_bf16x2(x1v[0], x1v[1]);
          pw2[e / 2] = pack_bf16x2(x2v[0], x2v[1]);
          pw2l[e / 2] = pack_bf16x2(x2lv[0], x2lv[1]);
          pp[e / 2] = pack_bf16x2(av[0], av[1]);
        }
        if (!mbar_wait(w_empty, (static_cast<uint32_t>(sv) & 1u) ^ 1u, p.status)) {
          ok = false;
          break;
        }
        // row r, receivers half * 32 .. + 31: 16-byte chunks half * 4 + i of the 128-byte row, 128-byte swizzle
        const uint32_t wrow = sbase + KM_W + r * 128;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t off = static_cast<uint32_t>(((half * 4 + i) ^ (r & 7)) << 4);
          km_st_v4(wrow + off, pw1[4 * i], pw1[4 * i + 1], pw1[4 * i + 2], pw1[4 * i + 3]);
          km_st_v4(wrow + KM_KT + off, pw2[4 * i], pw2[4 * i + 1], pw2[4 * i + 2], pw2[4 * i + 3]);
          km_st_v4(wrow + 2 * KM_KT + off, pw2l[4 * i], pw2l[4 * i + 1], pw2l[4 * i + 2], pw2l[4 * i + 3]);
          km_st_v4(wrow + 3 * KM_KT + off, pp[4 * i], pp[4 * i + 1], pp[4 * i + 2], pp[4 * i + 3]);
        }
        fence_proxy_async_smem();
        mbar_arrive(w_full);
      }
      if (!ok) break;
      // the two halves' s1 / s2 of each key row
      sums[(half * 2) * 128 + r] = s1;
      sums[(half * 2 + 1) * 128 + r] = s2;
      km_bar_sync();
      const float a1 = sums[r] + sums[2 * 128 + r], a2 = sums[128 + r] + sums[3 * 128 + r];
      if (!mbar_wait(acc_full, static_cast<uint32_t>(nitem) & 1u, p.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float p2[32], r2[32], q2[32], xy[16];
      tmem_ld32(trow + KM_TP2 + half * 32, p2);
      tmem_ld32(trow + KM_TR2 + half * 32, r2);
      tmem_ld32(trow + KM_TQ2 + half * 32, q2);
      tmem_ld16(trow + KM_TXY + half * 16, xy);
      tc_wait_ld();
      reg_fence<32>(p2);
      reg_fence<32>(r2);
      reg_fence<32>(q2);
      reg_fence<16>(xy);
      // response per raw coordinate d = P and P + 32 of this half's pairs P = half * 16 + i
      const int64_t ro = p.raw.at(row, tk, p.T);
      const float sqv = p.sq[static_cast<int64_t>(row) * p.T + tk];
      const float stepv = p.steps[static_cast<int64_t>(row) * p.T + tk];
      const float den = sqv / D + 1e-6f;
      const float rs = rsqrtf(den);
      float res[32];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int P = half * 16 + i;
        const float px = p2[2 * i], py = p2[2 * i + 1], qx = q2[2 * i], qy = q2[2 * i + 1];
        const float rx = r2[2 * i], ry = r2[2 * i + 1], cxy = xy[i];
        const float cs = p.cosb[static_cast<int64_t>(tk) * 32 + P], sn = p.sinb[static_cast<int64_t>(tk) * 32 + P];
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int d = P + 32 * hf;
          const float ratio = (2.f * stepv * raw_at(p.raw, p.raw_bf16, ro + d) + stepv * stepv) / D / den;
          const float ca = expm1f(-0.5f * log1pf(ratio));
          const float cb = stepv * rs * (1.f + ca);
          const float bu = cb * (hf ? sn : cs), bw = cb * (hf ? cs : -sn);
          const float resp = px * bu + py * bw + qx * bu * bu + qy * bw * bw + 2.f * cxy * bu * bw +
                             2.f * ca * (rx * bu + ry * bw) + a1 * ca + a2 * ca * ca;
          res[hf * 16 + i] = resp / stepv;
        }
      }
      const int64_t oo = p.out.at(row, tk, p.T);
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int64_t o = oo + hf * 32 + half * 16;  // 16 consecutive coordinates, 16-byte aligned (host check)
        if (p.out_bf16) {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out.data) + o);
#pragma unroll
          for (int q = 0; q < 2; ++q)
            dst[q] = make_uint4(pack_bf16x2(res[hf * 16 + 8 * q], res[hf * 16 + 8 * q + 1]),
                                pack_bf16x2(res[hf * 16 + 8 * q + 2], res[hf * 16 + 8 * q + 3]),
                                pack_bf16x2(res[hf * 16 + 8 * q + 4], res[hf * 16 + 8 * q + 5]),
                                pack_bf16x2(res[hf * 16 + 8 * q + 6], res[hf * 16 + 8 * q + 7]));
        } else {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out.data) + o);
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[q] = make_float4(res[hf * 16 + 4 * q], res[hf * 16 + 4 * q + 1], res[hf * 16 + 4 * q + 2],
                                 res[hf * 16 + 4 * q + 3]);
        }
      }
      // value sums: 32 columns of VA
      float va[32];
      tmem_ld32(trow + KM_TVA + half * 32, va);
      tc_wait_ld();
      reg_fence<32>(va);
      tc_fence_before();
      mbar_arrive(acc_empty);
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
      km_bar_sync();  // both halves have read sums before the next item overwrites them
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
