// noise_record::future_query_response on tcgen05 (sm_100a): reference train/val/run.py :1780-1815 (query_kernel),
// whose two dots run tl.dot(..., input_precision="tf32x3"). Per head h and (token m, probe p) row:
//   S[row, k] = dq[m, p, h] . keys[h, k]                     (tf32x3: hi.hi + hi.lo + lo.hi, fp32 accumulate)
//   change[row, k] = probabilities[h, m, k] (e^(S / 8) - 1)   (fp32, in the epilogue warps)
//   numerator[row] = sum_k change v_k (tf32x3), partition[row] = sum_k change (fp32)
//   out[m, p, h] = (numerator - partition base[h, m]) / (1 + partition)
// A 64-key tile of a token whose probabilities sum to <= 0 contributes nothing, as the reference skips it.
//
// Before the kernel, qr_split_kernel writes keys as tf32 hi / lo [H, Tp, 64] and values transposed as tf32 hi / lo
// [H, 64, Tp] (Tp = T rounded up to 64, zero keys beyond T), so every operand is K-major and TMA-loadable, and
// qr_live_kernel marks each (head, token, 64-key tile) whose probabilities sum above zero.
//
// One CTA per item = 128 (token, probe) rows of one head (the MMA's M; with 64 probes, two tokens), the latest
// tokens (the most live keys) launched first; its live key tiles are the union of its tokens'. 576 threads:
//   warp 0      the item's live-tile list (ballot over the live flags), then TMA: per tile the keys' hi / lo
//               (K ring, 3 stages of 32 KB) and the values' hi / lo (V ring, 2 stages of 32 KB);
//   warp 1      TMEM (512 columns): S (64 columns, 3 buffers), change hi / lo (64 + 64, double-buffered) and the
//               numerator O (64). The whole warp runs the issue loop, an elect.sync lane issues: S of tile j + 2
//               (24 MMAs 128 x 64 x 8, A = dq from shared memory) before O += change_j V_j (24 MMAs, A = change
//               from tensor memory), so S is ready when the epilogue reaches a tile and the tensor pipe always
//               holds queued work (with S one tile ahead it idled between the phases);
//   warps 2..17 warp w: rows of TMEM lane quarter w % 4, key columns 16 ((w - 2) / 4) .. + 15 of each tile: change
//               (e^x - 1 by expm1_f2, packed fp32x2 arithmetic) and its tf32 hi / lo into TMEM; at the end the same
//               16 dims of O, the partition, and the output.
// All threads first stage the item's dq rows as tf32 hi / lo into 128-byte-swizzled K-major tiles (32 KB each).
#pragma once
#include "ptx.cuh"

namespace noise {
namespace readout {

constexpr int QT_ROWS = 128, QT_KEYS = 64;
constexpr int QT_EPI = 16, QT_COLS = QT_KEYS / (QT_EPI / 4);  // epilogue warps; key columns (and O dims) per warp
constexpr int QT_THREADS = 64 + 32 * QT_EPI;
constexpr int QT_MAX_TILES = 512;  // keys_len <= 32,768 (the live-tile list is uint16 in shared memory)
// S runs QT_AHEAD tiles ahead of the O MMAs: QT_AHEAD + 1 S buffers in TMEM and K stages in shared memory
constexpr int QT_AHEAD = 2, QT_NS = QT_AHEAD + 1;
// shared memory (1024-byte aligned): dq hi / lo as two 16 KB halves (32 fp32 dims per 128-byte row) each; a K ring of
// QT_NS stages and a V ring of 2, a stage = hi half 0, hi half 1, lo half 0, lo half 1 of 8 KB (64 rows x 128 bytes)
constexpr int QT_HALF = QT_ROWS * 128;
constexpr int QT_OP = QT_KEYS * 128;
constexpr int QT_STAGE = 4 * QT_OP;
constexpr int QT_DQH = 0, QT_DQL = 2 * QT_HALF;
constexpr int QT_KR = 4 * QT_HALF, QT_VR = QT_KR + QT_NS * QT_STAGE;
constexpr int QT_SUMS = QT_KR;  // [QT_EPI / 4][128] fp32 partitions: the K ring, free once every MMA has completed
constexpr int QT_LIST = QT_VR + 2 * QT_STAGE;  // uint16 [QT_MAX_TILES], then the count
constexpr int QT_BAR = QT_LIST + QT_MAX_TILES * 2 + 16;
constexpr int QT_SMEM = QT_BAR + 256 + 1024;
static_assert(QT_BAR % 8 == 0, "mbarrier alignment");
static_assert(QT_SMEM <= 227 * 1024, "shared memory per CTA");
static_assert(QT_EPI / 4 * QT_ROWS * 4 <= QT_NS * QT_STAGE, "partitions fit the K ring");
// TMEM columns: S buffer b at 64 b; change buffer c: hi at QT_TCH + 128 c, lo 64 further; O at QT_TO (512 in all)
constexpr uint32_t QT_TS = 0, QT_TCH = 64 * QT_NS, QT_TO = QT_TCH + 256;
static_assert(QT_TO + 64 <= 512, "tensor memory columns");

struct QtArgs {
  const float* dq;      // contiguous [M, P, H, 64]
  View3 prob, base;     // (H, M, T), (H, M, 64)
  const uint8_t* live;  // [H, M, NT]
  float* out;           // contiguous [M, P, H, 64]
  int M, P, H, T, NT, Tp;
  int vec;              // probability rows contiguous and 16-byte aligned: float4 loads
  int* status;
};

struct QtMaps {
  CUtensorMap khi, klo;  // fp32 [H * Tp, 64], 64-row x 32 boxes, 128-byte swizzle
  CUtensorMap vhi, vlo;  // fp32 [H * 64, Tp], 64-row x 32 boxes, 128-byte swizzle
};

// keys -> tf32 hi / lo [H, Tp, 64]; values -> transposed tf32 hi / lo [H, 64, Tp]; keys >= T are zero. One block per
// (64-key tile, head).
__global__ void __launch_bounds__(256) qr_split_kernel(View3 keys, View3 values, int T, int Tp,
                                                       float* __restrict__ khi, float* __restrict__ klo,
                                                       float* __restrict__ vhi, float* __restrict__ vlo) {
  __shared__ float tile[QT_KEYS][D + 1];
  const int h = blockIdx.y, k0 = blockIdx.x * QT_KEYS;
  for (int i = threadIdx.x; i < QT_KEYS * D; i += 256) {
    const int kr = i / D, d = i % D, k = k0 + kr;
    const float x = k < T ? keys.at(h, k, d) : 0.f;
    const float xh = tf32_hi(x);
    const int64_t o = (static_cast<int64_t>(h) * Tp + k) * D + d;
    khi[o] = xh;
    klo[o] = x - xh;
    tile[kr][d] = k < T ? values.at(h, k, d) : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < QT_KEYS * D; i += 256) {
    const int d = i / QT_KEYS, kr = i % QT_KEYS;
    const float x = tile[kr][d];
    const float xh = tf32_hi(x);
    const int64_t o = (static_cast<int64_t>(h) * D + d) * Tp + k0 + kr;
    vhi[o] = xh;
    vlo[o] = x - xh;
  }
}

// live[h, m, t] = 1 when token m's probabilities over key tile t sum above zero (the reference's tile test,
// `tl.sum(a, 0) > 0`); one warp per (head, token, tile).
__global__ void __launch_bounds__(256) qr_live_kernel(View3 prob, int H, int M, int T, int NT,
                                                      uint8_t* __restrict__ live) {
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= static_cast<int64_t>(H) * M * NT) return;  // whole warps
  const int t = static_cast<int>(w % NT);
  const int64_t hm = w / NT;
  const int m = static_cast<int>(hm % M), h = static_cast<int>(hm / M);
  const int k = t * QT_KEYS + lane;
  float s = (k < T ? prob.at(h, m, k) : 0.f) + (k + 32 < T ? prob.at(h, m, k + 32) : 0.f);
  s = warp_sum(s);
  if (lane == 0) live[w] = s > 0.f ? 1 : 0;
}

__device__ __forceinline__ void qt_st_v4(uint32_t addr, float4 v) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

__global__ void __launch_bounds__(QT_THREADS, 1)
    query_tc_kernel(const __grid_constant__ QtMaps m, const __grid_constant__ QtArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + QT_BAR);
  uint64_t* k_full = bar;              // QT_NS
  uint64_t* k_empty = k_full + QT_NS;  // QT_NS
  uint64_t* s_full = k_empty + QT_NS;  // QT_NS
  uint64_t* s_empty = s_full + QT_NS;  // QT_NS
  uint64_t* v_full = s_empty + QT_NS;  // 2
  uint64_t* v_empty = v_full + 2;      // 2
  uint64_t* c_full = v_empty + 2;      // 2
  uint64_t* c_empty = c_full + 2;      // 2
  uint64_t* o_full = c_empty + 2;
  uint64_t* drain = o_full + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  uint16_t* list = reinterpret_cast<uint16_t*>(smem + QT_LIST);
  int* count = reinterpret_cast<int*>(smem + QT_LIST + QT_MAX_TILES * 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t R = static_cast<int64_t>(p.M) * p.P;
  const int RB = static_cast<int>((R + QT_ROWS - 1) / QT_ROWS);
  const int h = blockIdx.x % p.H;
  const int64_t r0 = static_cast<int64_t>(RB - 1 - blockIdx.x / p.H) * QT_ROWS;  // the latest tokens first

  if (threadIdx.x == 0) {
    for (int b = 0; b < QT_NS; ++b) {
      mbar_init(&k_full[b], 1);
      mbar_init(&k_empty[b], 1);
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], QT_EPI);  // one arrival per epilogue warp (its lanes joined by __syncwarp first)
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&v_full[b], 1);
      mbar_init(&v_empty[b], 1);
      mbar_init(&c_full[b], QT_EPI);
      mbar_init(&c_empty[b], 1);
    }
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&m.khi);
      tma_prefetch_desc(&m.klo);
      tma_prefetch_desc(&m.vhi);
      tma_prefetch_desc(&m.vlo);
    }
    // the item's live key tiles: live for any of its tokens
    const int tm0 = static_cast<int>(r0 / p.P);
    const int tm1 = static_cast<int>((min(r0 + QT_ROWS, R) - 1) / p.P);
    int n = 0;
    for (int t0 = 0; t0 < p.NT; t0 += 32) {
      const int t = t0 + lane;
      bool any = false;
      if (t < p.NT)
        for (int tm = tm0; tm <= tm1 && !any; ++tm) any = p.live[(static_cast<int64_t>(h) * p.M + tm) * p.NT + t] != 0;
      const uint32_t bal = __ballot_sync(0xffffffffu, any);
      if (any) list[n + __popc(bal & ((1u << lane) - 1u))] = static_cast<uint16_t>(t);
      n += __popc(bal);
    }
    if (lane == 0) *count = n;
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  // dq rows r0 .. r0 + 127 as tf32 hi / lo: float4 q of a row = 16-byte chunk q % 8 of half q / 8, swizzled by row % 8
  const uint32_t sbase = smem_u32(smem);
  for (int f = threadIdx.x; f < QT_ROWS * 16; f += QT_THREADS) {
    const int r = f >> 4, q = f & 15;
    const int64_t rr = r0 + r;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (rr < R) x = *reinterpret_cast<const float4*>(p.dq + (rr * p.H + h) * D + q * 4);
    const float4 hi = make_float4(tf32_hi(x.x), tf32_hi(x.y), tf32_hi(x.z), tf32_hi(x.w));
    const float4 lo = make_float4(x.x - hi.x, x.y - hi.y, x.z - hi.z, x.w - hi.w);
    const uint32_t off = static_cast<uint32_t>((q >> 3) * QT_HALF + r * 128 + (((q & 7) ^ (r & 7)) << 4));
    qt_st_v4(sbase + QT_DQH + off, hi);
    qt_st_v4(sbase + QT_DQL + off, lo);
  }
  fence_proxy_async_smem();  // the tensor core reads these through the async proxy
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int n = *count;

  if (warp == 0) {
    if (lane == 0) {
      // K tiles run QT_AHEAD ahead of V tiles, in the order the MMAs consume them: K(0) .. K(AHEAD - 1), then V(j),
      // K(j + AHEAD) for each j
      int nk = 0, nv = 0;
      auto load_k = [&](int j) {
        const int b = j % QT_NS;
        if (!mbar_wait(&k_empty[b], (static_cast<uint32_t>(j / QT_NS) & 1u) ^ 1u, p.status)) return false;
        uint8_t* ks = smem + QT_KR + b * QT_STAGE;
        const int y = h * p.Tp + list[j] * QT_KEYS;
        mbar_arrive_expect_tx(&k_full[b], QT_STAGE);
        tma_load_2d(ks, &m.khi, &k_full[b], 0, y);
        tma_load_2d(ks + QT_OP, &m.khi, &k_full[b], 32, y);
        tma_load_2d(ks + 2 * QT_OP, &m.klo, &k_full[b], 0, y);
        tma_load_2d(ks + 3 * QT_OP, &m.klo, &k_full[b], 32, y);
        ++nk;
        return true;
      };
      auto load_v = [&](int j) {
        const int b = j & 1;
        if (!mbar_wait(&v_empty[b], (static_cast<uint32_t>(j >> 1) & 1u) ^ 1u, p.status)) return false;
        uint8_t* vs = smem + QT_VR + b * QT_STAGE;
        const int k0 = list[j] * QT_KEYS;
        mbar_arrive_expect_tx(&v_full[b], QT_STAGE);
        tma_load_2d(vs, &m.vhi, &v_full[b], k0, h * D);
        tma_load_2d(vs + QT_OP, &m.vhi, &v_full[b], k0 + 32, h * D);
        tma_load_2d(vs + 2 * QT_OP, &m.vlo, &v_full[b], k0, h * D);
        tma_load_2d(vs + 3 * QT_OP, &m.vlo, &v_full[b], k0 + 32, h * D);
        ++nv;
        return true;
      };
      bool ok = true;
      for (int j = 0; j < QT_AHEAD && j < n && ok; ++j) ok = load_k(j);
      for (int j = 0; j < n && ok; ++j) {
        ok = load_v(j);
        if (ok && j + QT_AHEAD < n) ok = load_k(j + QT_AHEAD);
      }
      // no TMA write may still be in flight when the CTA exits (a pipeline that gave up included)
      for (int j = max(nk - QT_NS, 0); j < nk; ++j)
        mbar_wait(&k_full[j % QT_NS], static_cast<uint32_t>(j / QT_NS) & 1u, p.status);
      for (int j = max(nv - 2, 0); j < nv; ++j) mbar_wait(&v_full[j & 1], static_cast<uint32_t>(j >> 1) & 1u, p.status);
    }
  } else if (warp == 1) {
    constexpr uint32_t id = idesc_tf32(QT_ROWS, 64);
    // S_j = dq K_j^T into S buffer j % QT_NS: per K-step of 8 dims the small terms first (lo.hi, hi.lo, then hi.hi)
    auto scores = [&](int j) {
      const int b = j % QT_NS;
      const uint32_t par = static_cast<uint32_t>(j / QT_NS) & 1u;
      if (!mbar_wait_warp(&k_full[b], par, p.status) || !mbar_wait_warp(&s_empty[b], par ^ 1u, p.status))
        return false;
      tc_fence_after();
      const uint32_t ks = sbase + QT_KR + b * QT_STAGE, ts = tmem + QT_TS + b * 64;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t ho = k >> 2, kk = 2u * (k & 3);
        const uint64_t ah = sdesc_kmajor_sw128(sbase + QT_DQH + ho * QT_HALF) + kk;
        const uint64_t al = sdesc_kmajor_sw128(sbase + QT_DQL + ho * QT_HALF) + kk;
        const uint64_t bh = sdesc_kmajor_sw128(ks + ho * QT_OP) + kk;
        const uint64_t bl = sdesc_kmajor_sw128(ks + 2 * QT_OP + ho * QT_OP) + kk;
        if (elect_one()) tc_mma_tf32(ts, al, bh, id, k > 0);
        if (elect_one()) tc_mma_tf32(ts, ah, bl, id, 1u);
        if (elect_one()) tc_mma_tf32(ts, ah, bh, id, 1u);
      }
      if (elect_one()) tc_commit(&s_full[b]);
      if (elect_one()) tc_commit(&k_empty[b]);
      return true;
    };
    // O += change_j V_j: A = change hi / lo from TMEM (8 columns per K-step of 8 keys), B = V^T (keys as K)
    auto numerator = [&](int j) {
      const int b = j & 1;
      const uint32_t par = static_cast<uint32_t>(j >> 1) & 1u;
      if (!mbar_wait_warp(&v_full[b], par, p.status) || !mbar_wait_warp(&c_full[b], par, p.status)) return false;
      tc_fence_after();
      const uint32_t vs = sbase + QT_VR + b * QT_STAGE, ch = tmem + QT_TCH + b * 128;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t ho = k >> 2, kk = 2u * (k & 3);
        const uint64_t bh = sdesc_kmajor_sw128(vs + ho * QT_OP) + kk;
        const uint64_t bl = sdesc_kmajor_sw128(vs + 2 * QT_OP + ho * QT_OP) + kk;
        if (elect_one()) tc_mma_ts_tf32(tmem + QT_TO, ch + 64 + k * 8, bh, id, (j > 0 || k > 0) ? 1u : 0u);
        if (elect_one()) tc_mma_ts_tf32(tmem + QT_TO, ch + k * 8, bl, id, 1u);
        if (elect_one()) tc_mma_ts_tf32(tmem + QT_TO, ch + k * 8, bh, id, 1u);
      }
      if (elect_one()) tc_commit(&v_empty[b]);
      if (elect_one()) tc_commit(&c_empty[b]);
      return true;
    };
    // S of tiles 0 .. AHEAD - 1, then per tile j: S(j + AHEAD), O += change_j V_j
    bool ok = true;
    for (int j = 0; j < QT_AHEAD && j < n && ok; ++j) ok = scores(j);
    for (int j = 0; j < n && ok; ++j) {
      if (j + QT_AHEAD < n) ok = scores(j + QT_AHEAD);
      if (ok) ok = numerator(j);
    }
    if (elect_one()) tc_commit(o_full);
    if (elect_one()) tc_commit(drain);
    mbar_wait_warp(drain, 0, p.status);
  } else {
    const int quarter = warp & 3, cg = (warp - 2) >> 2;  // TMEM lane quarter; column group of QT_COLS
    const int r = quarter * 32 + lane;
    const int64_t rr = r0 + r;
    const bool valid = rr < R;
    const int tm = valid ? static_cast<int>(rr / p.P) : 0;
    const uint8_t* lv = p.live + (static_cast<int64_t>(h) * p.M + tm) * p.NT;
    const float* prow = p.prob.p + h * p.prob.s0 + tm * p.prob.s1;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    float2 part = make_float2(0.f, 0.f);
    bool ok = true;
    // a row's probabilities and its token's live flag for tile index jj, loaded one tile ahead of their use; every
    // valid row loads, the flag masks later, so no load waits on another
    float an[QT_COLS];
    uint8_t mine_n = 0;
    auto fetch = [&](int jj) {
      const int kb = list[jj] * QT_KEYS + cg * QT_COLS;
      mine_n = valid ? lv[list[jj]] : 0;
      if (valid && p.vec && kb + QT_COLS <= p.T) {
#pragma unroll
        for (int c = 0; c < QT_COLS; c += 4) {
          const float4 v = *reinterpret_cast<const float4*>(prow + kb + c);
          an[c] = v.x, an[c + 1] = v.y, an[c + 2] = v.z, an[c + 3] = v.w;
        }
      } else {
#pragma unroll
        for (int c = 0; c < QT_COLS; ++c) an[c] = (valid && kb + c < p.T) ? prow[(kb + c) * p.prob.s2] : 0.f;
      }
    };
    if (n > 0) fetch(0);
    for (int j = 0; j < n && ok; ++j) {
      const int b = j & 1, sb = j % QT_NS;
      const uint32_t par = static_cast<uint32_t>(j >> 1) & 1u, spar = static_cast<uint32_t>(j / QT_NS) & 1u;
      // a row whose own token's tile is not live takes nothing from it (the reference skips the tile there), even
      // where e^x would overflow
      const bool mine = mine_n != 0;
      float a[QT_COLS];
#pragma unroll
      for (int c = 0; c < QT_COLS; ++c) a[c] = an[c];
      if (j + 1 < n) fetch(j + 1);
      if (!mbar_wait_warp(&s_full[sb], spar, p.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[QT_COLS];
      tmem_ld16(trow + QT_TS + sb * 64 + cg * QT_COLS, s);
      tc_wait_ld();
      reg_fence<QT_COLS>(s);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[sb]);
      uint32_t hi[QT_COLS], lo[QT_COLS];
      if (mine) {
#pragma unroll
        for (int c = 0; c < QT_COLS; c += 2) {
          const float2 e = expm1_f2(__fmul2_rn(make_float2(s[c], s[c + 1]), make_float2(SCALE, SCALE)));
          const float2 ch = __fmul2_rn(make_float2(a[c], a[c + 1]), e);
          part = __fadd2_rn(part, ch);
          const float2 chh = make_float2(tf32_hi(ch.x), tf32_hi(ch.y));
          const float2 chl = __fadd2_rn(ch, make_float2(-chh.x, -chh.y));
          hi[c] = __float_as_uint(chh.x), hi[c + 1] = __float_as_uint(chh.y);
          lo[c] = __float_as_uint(chl.x), lo[c + 1] = __float_as_uint(chl.y);
        }
      } else {
#pragma unroll
        for (int c = 0; c < QT_COLS; ++c) hi[c] = lo[c] = 0u;
      }
      if (!mbar_wait_warp(&c_empty[b], par ^ 1u, p.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      tmem_st16(trow + QT_TCH + b * 128 + cg * QT_COLS, hi);
      tmem_st16(trow + QT_TCH + b * 128 + 64 + cg * QT_COLS, lo);
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&c_full[b]);
    }
    // after o_full every MMA has completed and every K tile was consumed: the K ring holds the partitions
    const bool got = mbar_wait_warp(o_full, 0, p.status);
    float* sums = reinterpret_cast<float*>(smem + QT_SUMS);
    sums[cg * QT_ROWS + r] = part.x + part.y;
    const bool all = bar_and<QT_THREADS - 64>(ok && got);  // every column group's partition is in shared memory
    float total = 0.f;
#pragma unroll
    for (int g = 0; g < QT_EPI / 4; ++g) total += sums[g * QT_ROWS + r];
    float o[QT_COLS];
    if (all && n > 0) {
      tc_fence_after();
      tmem_ld16(trow + QT_TO + cg * QT_COLS, o);
      tc_wait_ld();
      reg_fence<QT_COLS>(o);
    } else {
#pragma unroll
      for (int c = 0; c < QT_COLS; ++c) o[c] = 0.f;
    }
    if (valid && all) {
      const float den = 1.f + total;
      float4* dst = reinterpret_cast<float4*>(p.out + (rr * p.H + h) * D + cg * QT_COLS);
#pragma unroll
      for (int c = 0; c < QT_COLS; c += 4) {
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = (o[c + e] - total * p.base.at(h, tm, cg * QT_COLS + c + e)) / den;
        dst[c / 4] = make_float4(v[0], v[1], v[2], v[3]);
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

}  // namespace readout
}  // namespace noise
