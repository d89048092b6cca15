// noise_record::routed_response on tcgen05 (sm_100a): reference train/val/run.py :548-569 (finite_attention_kernels'
// `routed`), :604-619. Per (token m, head h) item, its K routed keys / values (bf16) and probabilities p_k, and each
// probe row dq[m, p, h] (bf16):
//   ds_k = bf16(dq . k_k) / 8                             (the bf16 output of the first dot)
//   dlse = log1p(sum_k p_k (e^ds_k - 1))
//   w_k = bf16(p_k (e^(ds_k - dlse) - 1)),  out = bf16(sum_k w_k v_k) + (e^-dlse - 1) rest[m, h]
// Both dots are kind::f16 MMAs with fp32 accumulation, rounded to bf16 as the reference's tl.dot outputs are.
//
// A tile is G items: G = 2 when the keys padded to 32 (Kp) fit twice in one MMA's N (Kp <= 128), else 1. Its 128
// MMA rows are item g's 64 probes at rows 64 g .. 64 g + 63 (one 64-probe block; more probes make more items):
//   S [128 x G Kp] = Q [128 x 64] [K_0; K_1]^T    (each row uses only its own item's Kp columns)
//   O [128 x 64]   = W [128 x G Kp] [V_0; V_1]    (W in TMEM, block-diagonal: zero outside a row's own keys)
// Keys past K inside a Kp box are the next item's (or TMA's zero fill): their p is masked to 0, so they add nothing.
// Persistent CTAs (one per SM), 576 threads:
//   warp 0      TMA: per tile the G items' probe rows (a 3-D map over dq's (row, head, dim)), keys and values into
//               one of 2 stages (80 KB each);
//   warp 1      TMEM (512 columns: S 256, W 128, O 64) and the MMAs: S of tile t + 1 (4) as soon as the epilogue
//               has read S(t), then O(t) (G Kp / 16) once it has written W(t);
//   warps 2..17 warp w: rows of TMEM lane quarter w % 4, 32-key pieces (w - 2) / 4 and + 4 of its item. First pass:
//               e = e^ds - 1 (kept in registers) and its p-weighted sum; the 4 warps of a row exchange partial sums
//               in shared memory for sigma; second pass: W = bf16(p (e - sigma) / (1 + sigma)) into TMEM; then
//               dims 16 ((w - 2) / 4) .. + 15 of O and the output. The first pass of tile t + 1 runs before O(t) is
//               read, so the O MMAs overlap it. The probabilities are staged in shared memory two tiles ahead.
#pragma once
#include "ptx.cuh"

namespace noise {
namespace readout {

constexpr int RT_THREADS = 576, RT_EPI = 16;
constexpr int RT_Q = 64 * 128;             // one item's 64 probe rows, 128 bytes each
constexpr int RT_KV = 256 * 128;           // keys (or values) of a tile: G Kp <= 256 rows
constexpr int RT_STAGE = 2 * RT_Q + 2 * RT_KV;  // Q0, Q1, K, V
constexpr int RT_SUMS = 2 * RT_STAGE;      // [2 tiles][4 pieces][128 rows] fp32
constexpr int RT_PROB = RT_SUMS + 2 * 4 * 128 * 4;  // [3 tiles][256] fp32: a tile's probabilities, slot-major
constexpr int RT_BAR = RT_PROB + 3 * 256 * 4;
constexpr int RT_SMEM = RT_BAR + 256 + 1024;
static_assert(RT_SMEM <= 227 * 1024, "shared memory per CTA");
constexpr uint32_t RT_TS = 0, RT_TW = 256, RT_TO = 384;

struct RtArgs {
  const float* prob;  // [M, H, K]
  const float* rest;  // [M, H, 64]
  float* out;         // [M, P, H, 64]
  int M, P, H, K, Kp, G, PB, items, tiles;
  int* status;
};

struct RtMaps {
  CUtensorMap q;   // bf16 dq as (dim 64, head H, row M * P), 64 x 1 x 64 boxes, 128-byte swizzle
  CUtensorMap kv;  // bf16 keys as [M * H * K, 64], 64 x Kp boxes
  CUtensorMap v;   // bf16 values, same
};

// NP: 32-key pieces per epilogue warp and row, ceil(Kp / 128) (1 up to 128 keys, 2 up to 256)
template <int NP>
__global__ void __launch_bounds__(RT_THREADS, 1)
    routed_tc_kernel(const __grid_constant__ RtMaps m, const __grid_constant__ RtArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + RT_BAR);
  uint64_t* st_full = bar;        // 2
  uint64_t* st_empty = bar + 2;   // 2
  uint64_t* s_full = bar + 4;
  uint64_t* w_full = bar + 5;
  uint64_t* o_full = bar + 6;
  uint64_t* acc_free = bar + 7;
  uint64_t* drain = bar + 8;
  uint64_t* s_free = bar + 9;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bar + 10);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NS = p.G * p.Kp;  // S columns = O's K extent

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&st_full[s], 1);
      mbar_init(&st_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(w_full, RT_EPI);
    mbar_init(o_full, 1);
    mbar_init(acc_free, RT_EPI);
    mbar_init(drain, 1);
    mbar_init(s_free, RT_EPI);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&m.q);
    tma_prefetch_desc(&m.kv);
    tma_prefetch_desc(&m.v);
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
  // the item of tile slot g (the tile's last slot repeats a valid item when items is odd, so its shared memory holds
  // finite keys and values: they meet zero weights)
  auto item_of = [&](int t, int g) { return min(t * p.G + g, p.items - 1); };

  if (warp == 0) {
    if (lane == 0) {
      int lt = 0;
      const uint32_t bytes = static_cast<uint32_t>(p.G * (RT_Q + 2 * p.Kp * 128));
      for (int t = blockIdx.x; t < p.tiles; t += gridDim.x, ++lt) {
        const int s = lt & 1;
        if (!mbar_wait(&st_empty[s], (static_cast<uint32_t>(lt >> 1) & 1u) ^ 1u, p.status)) break;
        uint8_t* st = smem + s * RT_STAGE;
        mbar_arrive_expect_tx(&st_full[s], bytes);
        for (int g = 0; g < p.G; ++g) {
          const int it = item_of(t, g);
          const int pb = it % p.PB, mh = it / p.PB, tok = mh / p.H, hd = mh % p.H;
          tma_load_3d(st + g * RT_Q, &m.q, &st_full[s], 0, hd, tok * p.P + pb * 64);
          tma_load_2d(st + 2 * RT_Q + g * p.Kp * 128, &m.kv, &st_full[s], 0, mh * p.K);
          tma_load_2d(st + 2 * RT_Q + RT_KV + g * p.Kp * 128, &m.v, &st_full[s], 0, mh * p.K);
        }
      }
      // no TMA write may still be in flight when the CTA exits
      for (int j = max(lt - 2, 0); j < lt; ++j)
        mbar_wait(&st_full[j & 1], static_cast<uint32_t>(j >> 1) & 1u, p.status);
    }
  } else if (warp == 1) {
    const uint32_t id_s = idesc_bf16(128, NS);
    constexpr uint32_t id_o = idesc_bf16(128, 64, false, true);  // V as the MN-major B operand
    // S(lt): the stage's operands have landed and the epilogue's first pass has read S(lt - 1)
    auto scores = [&](int lt) {
      const int s = lt & 1;
      if (!mbar_wait_warp(&st_full[s], static_cast<uint32_t>(lt >> 1) & 1u, p.status) ||
          (lt > 0 && !mbar_wait_warp(s_free, static_cast<uint32_t>(lt - 1) & 1u, p.status)))
        return false;
      tc_fence_after();
      const uint32_t st = sbase + s * RT_STAGE;
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (elect_one())
          tc_mma(tmem + RT_TS, sdesc_kmajor_sw128(st) + 2u * k, sdesc_kmajor_sw128(st + 2 * RT_Q) + 2u * k, id_s, k > 0);
      if (elect_one()) tc_commit(s_full);
      return true;
    };
    // O(lt) = W V: the epilogue has written W(lt) and read O(lt - 1)
    auto values = [&](int lt) {
      const uint32_t par = static_cast<uint32_t>(lt) & 1u;
      if (!mbar_wait_warp(w_full, par, p.status) || !mbar_wait_warp(acc_free, par ^ 1u, p.status)) return false;
      tc_fence_after();
      const uint32_t st = sbase + (lt & 1) * RT_STAGE;
      for (int ks = 0; ks < NS / 16; ++ks)
        if (elect_one())
          tc_mma_ts(tmem + RT_TO, tmem + RT_TW + ks * 8, sdesc_mnmajor_sw128(st + 2 * RT_Q + RT_KV + ks * 2048, 16),
                    id_o, ks > 0);
      if (elect_one()) tc_commit(o_full);
      if (elect_one()) tc_commit(&st_empty[lt & 1]);
      return true;
    };
    // S of the next tile goes in as soon as the epilogue has read this tile's S, ahead of this tile's O
    const int nt = (p.tiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) / gridDim.x;
    bool ok = nt > 0 && scores(0);
    for (int lt = 0; lt < nt && ok; ++lt) {
      if (lt + 1 < nt) ok = scores(lt + 1);
      if (ok) ok = values(lt);
    }
    if (elect_one()) tc_commit(drain);
    mbar_wait_warp(drain, 0, p.status);
  } else {
    const int quarter = warp & 3, cg = (warp - 2) >> 2;
    const int r = quarter * 32 + lane, g = r >> 6;  // MMA row; its tile slot (warp-uniform)
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    float* sums = reinterpret_cast<float*>(smem + RT_SUMS);
    float* probs = reinterpret_cast<float*>(smem + RT_PROB);
    const int pieces = p.Kp / 32;
    const int et = threadIdx.x - 64;  // 0 .. 511
    const int nt = (p.tiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) / gridDim.x;
    auto tile_of = [&](int lt) { return static_cast<int>(blockIdx.x) + lt * static_cast<int>(gridDim.x); };
    // local tile lt's probabilities into buffer lt % 3: slot g's keys at g Kp .. g Kp + Kp - 1, zero past K. A buffer
    // is written two barriers before its first read and after the last read of its previous tile
    auto stage_probs = [&](int lt) {
      if (lt < nt && et < p.G * p.Kp) {
        const int sg = et / p.Kp, k = et % p.Kp;
        const int mh = item_of(tile_of(lt), sg) / p.PB;
        probs[(lt % 3) * 256 + et] = k < p.K ? p.prob[static_cast<int64_t>(mh) * p.K + k] : 0.f;
      }
    };
    stage_probs(0);
    stage_probs(1);
    // W starts zero: a row's weights are only ever written in its own item's columns (block-diagonal)
    {
      uint32_t z[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) z[c] = 0u;
      for (int c = cg * 16; c < 128; c += 64) tmem_st16(trow + RT_TW + c, z);
      tc_wait_st();
    }
    tc_fence_before();
    // every epilogue warp reaches the named barrier the same number of times, whatever happened: a warp whose bounded
    // wait gave up arrives with false, all of them see the AND, and from then on they only keep the count
    bool ok = bar_and<RT_THREADS - 64>(true);
    tc_fence_after();
    float e[NP][32];  // e^ds - 1 of this warp's pieces of the row's own keys, from the first pass to the second
    // first pass of local tile lt: e and its p-weighted partial sum into sums[lt & 1]; then S may be overwritten
    auto pass1 = [&](int lt) {
      const bool got = ok && mbar_wait_warp(s_full, static_cast<uint32_t>(lt) & 1u, p.status);
      const float* pk = probs + (lt % 3) * 256 + g * p.Kp;
      float2 acc = make_float2(0.f, 0.f);
      if (got) {
        tc_fence_after();
        if (g < p.G) {
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            const int pc = cg + 4 * i;
            if (pc < pieces) {
              float sv[32];
              tmem_ld32(trow + RT_TS + g * p.Kp + pc * 32, sv);
              tc_wait_ld();
              reg_fence<32>(sv);
#pragma unroll
              for (int c = 0; c < 32; c += 2) {
                const int k = pc * 32 + c;
                // the dot's bf16 output: one packed conversion (round to nearest even) and its exact widening
                const float2 ev = expm1_f2(__fmul2_rn(unpack_bf16x2(pack_bf16x2(sv[c], sv[c + 1])),
                                                      make_float2(SCALE, SCALE)));
                e[i][c] = ev.x, e[i][c + 1] = ev.y;
                if (k < p.K) acc.x = fmaf(pk[k], ev.x, acc.x);
                if (k + 1 < p.K) acc.y = fmaf(pk[k + 1], ev.y, acc.y);
              }
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_free);
      }
      sums[(lt & 1) * 512 + cg * 128 + r] = acc.x + acc.y;
      return got;
    };
    // second pass (after the barrier): e^(ds - dlse) - 1 = (e - sigma) / (1 + sigma), as 1 + sigma = e^dlse, so
    // w_k = bf16(p_k (e_k - sigma) / (1 + sigma)) into W (bf16 pairs, the TS operand's K-major packing); returns
    // dlse. 1 + sigma <= 0 makes dlse, and the reference's weights with it, NaN: so here too
    auto pass2 = [&](int lt) {
      const float* sb = sums + (lt & 1) * 512;
      const float sigma = (sb[r] + sb[128 + r]) + (sb[256 + r] + sb[384 + r]);
      const float inv = 1.f + sigma > 0.f ? 1.f / (1.f + sigma) : __int_as_float(0x7FC00000);
      const float* pk = probs + (lt % 3) * 256 + g * p.Kp;
      if (g < p.G) {
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          const int pc = cg + 4 * i;
          if (pc < pieces) {
            uint32_t wv[16];
#pragma unroll
            for (int c = 0; c < 32; c += 2) {
              const int k = pc * 32 + c;
              const float2 d = __fmul2_rn(__fadd2_rn(make_float2(e[i][c], e[i][c + 1]), make_float2(-sigma, -sigma)),
                                          make_float2(inv, inv));
              const float w0 = k < p.K ? pk[k] * d.x : 0.f, w1 = k + 1 < p.K ? pk[k + 1] * d.y : 0.f;
              wv[c / 2] = pack_bf16x2(w0, w1);
            }
            tmem_st16(trow + RT_TW + (g * p.Kp + pc * 32) / 2, wv);
          }
        }
        tc_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(w_full);
      return log1pf(sigma);
    };
    // software pipeline over the CTA's tiles: pass 1 of tile lt + 1 runs while O(lt) is on the tensor pipe
    float dlse = 0.f;
    if (nt > 0) {
      const bool got = pass1(0);
      ok = bar_and<RT_THREADS - 64>(got);
      stage_probs(2);
      if (ok) dlse = pass2(0);
    }
    for (int lt = 0; lt < nt; ++lt) {
      const bool got1 = lt + 1 < nt ? pass1(lt + 1) : true;
      // O(lt): read, release, finish and store
      const bool have = ok && mbar_wait_warp(o_full, static_cast<uint32_t>(lt) & 1u, p.status);
      if (have) {
        tc_fence_after();
        float o[16];
        tmem_ld16(trow + RT_TO + cg * 16, o);
        tc_wait_ld();
        reg_fence<16>(o);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_free);
        const int t = tile_of(lt);
        const int it = item_of(t, g);
        const int pb = it % p.PB, mh = it / p.PB, tok = mh / p.H, hd = mh % p.H;
        const int probe = pb * 64 + (r & 63);
        if (g < p.G && t * p.G + g < p.items && probe < p.P) {
          const float em = expm1f(-dlse);
          const float* rs = p.rest + static_cast<int64_t>(mh) * 64 + cg * 16;
          float4* dst = reinterpret_cast<float4*>(
              p.out + ((static_cast<int64_t>(tok) * p.P + probe) * p.H + hd) * 64 + cg * 16);
#pragma unroll
          for (int c = 0; c < 16; c += 4) {
            const float2 o01 = unpack_bf16x2(pack_bf16x2(o[c], o[c + 1]));
            const float2 o23 = unpack_bf16x2(pack_bf16x2(o[c + 2], o[c + 3]));
            dst[c / 4] = make_float4(o01.x + em * rs[c], o01.y + em * rs[c + 1], o23.x + em * rs[c + 2],
                                     o23.y + em * rs[c + 3]);
          }
        }
      }
      ok = ok && have;
      if (lt + 1 < nt) {
        ok = bar_and<RT_THREADS - 64>(ok && got1);
        stage_probs(lt + 3);
        if (ok) dlse = pass2(lt + 1);
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
