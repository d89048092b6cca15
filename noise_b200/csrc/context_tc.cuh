// The credit path's per-query context on tcgen05 (sm_100a), bf16 inputs: lse_t = logsumexp_{s: 0 <= t - s <= window}
// q_t . k_s / 8 and center_t = sum_s p(t, s) (hub_t . v_s) (reference train/speedrun/moment_kernels.py:137-194,
// implicit_key_context_edges; the reference's dots are tf32 on bf16 operands, i.e. exact products with fp32 sums,
// which the bf16 tensor-core MMA also computes).
//
// One work item = two adjacent 128-query tiles A, B of one row sharing every 128-key tile; 320 threads, one CTA per
// SM, persistent, heaviest items first:
//   warp 0      TMA: Q_A, Q_B, H_A, H_B once per item, then the item's key tiles (k and v rows) into a 3-stage ring
//               (128-byte swizzle);
//   warp 1      TMEM: per group g the logits S_g = Q_g K^T and the scores C_g = H_g V^T (128 columns each, 512 in
//               all); one lane issues the 8 MMAs per (group, key tile) (M = 128 queries, N = 128 keys, K = 64);
//   warps 2..9  two groups of 4 warps (tiles A, B), one query row per thread: 32-column chunks of S and C from TMEM,
//               masked only on the diagonal and window-edge tiles, an online maximum (rescaling l and the weighted
//               sum when it grows), p = 2^(s log2(e) / 8 - m log2(e)) on the MUFU pipe, l += p, sum += p c; at the end
//               lse = m + log(l), center = sum / l, one coalesced store each.
#pragma once
#include <type_traits>

#include "ptx.cuh"

namespace noise {
namespace credit {

constexpr int TC_B = 128, TC_STAGES = 3, TC_THREADS = 320;
constexpr int TC_TILE = 128 * 128;                      // bytes of one [128][64] bf16 tile
constexpr int TC_Q = 0;                                 // Q_A, Q_B, H_A, H_B
constexpr int TC_RING = TC_Q + 4 * TC_TILE;             // stage: K, V
constexpr int TC_BAR = TC_RING + TC_STAGES * 2 * TC_TILE;
constexpr int TC_SMEM = TC_BAR + 256 + 1024;

struct TContextArgs {
  int T, window, rows;
  float *lse, *center;  // [rows, T]
  int* status;
};

struct TCRange {
  int lo, hi;  // key tiles [lo, hi] of query tile qt
};
__device__ __forceinline__ TCRange tc_range(int qt, int window) {
  const int first = qt * TC_B - window;
  return TCRange{first > 0 ? first / TC_B : 0, qt};
}
// every key of tile kt is visible to every query of tile qt: no mask
__device__ __forceinline__ bool tc_full(int qt, int kt, int window) {
  const int q0 = qt * TC_B, k0 = kt * TC_B;
  return k0 + TC_B - 1 <= q0 && q0 + TC_B - 1 - k0 <= window;
}

__global__ void __launch_bounds__(TC_THREADS, 1)
    context_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tmh, const __grid_constant__ CUtensorMap tmv,
                      TContextArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + TC_BAR);
  uint64_t* q_full = bar;                  // the item's Q / H tiles landed
  uint64_t* q_empty = bar + 1;             // every MMA of the item done
  uint64_t* kv_full = bar + 2;             // STAGES
  uint64_t* kv_empty = kv_full + TC_STAGES;
  uint64_t* s_full = kv_empty + TC_STAGES;  // per group
  uint64_t* s_empty = s_full + 2;
  uint64_t* drain = s_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = p.T / TC_B;
  const int npairs = (nt + 1) / 2;
  const int items = npairs * p.rows;

  // work item w: query-tile pair (npairs - 1 - w / rows: the last pairs see the most keys) of row w % rows
  struct Item {
    int row, qa, qb, lo, hi;
    bool has_b;
    TCRange ra, rb;
  };
  auto item = [&](int w) {
    Item it;
    const int pi = npairs - 1 - w / p.rows;
    it.row = w % p.rows;
    it.qa = 2 * pi;
    it.qb = 2 * pi + 1;
    it.has_b = it.qb < nt;
    it.ra = tc_range(it.qa, p.window);
    it.rb = it.has_b ? tc_range(it.qb, p.window) : TCRange{1, 0};
    it.lo = it.ra.lo;
    it.hi = it.has_b ? it.rb.hi : it.ra.hi;
    return it;
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < TC_STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&s_full[g], 1);
      mbar_init(&s_empty[g], 4);  // one arrival per warp of the group (after its __syncwarp)
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmq);
    tma_prefetch_desc(&tmk);
    tma_prefetch_desc(&tmh);
    tma_prefetch_desc(&tmv);
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
      int kv = 0, nitem = 0;  // key tiles issued, items started
      bool ok = true;
      for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++nitem) {
        const Item it = item(w);
        const int row0 = it.row * p.T;
        if (!mbar_wait(q_empty, (static_cast<uint32_t>(nitem) & 1u) ^ 1u, p.status)) break;
        mbar_arrive_expect_tx(q_full, (it.has_b ? 4 : 2) * TC_TILE);
        tma_load_2d(smem + TC_Q, &tmq, q_full, 0, row0 + it.qa * TC_B);
        tma_load_2d(smem + TC_Q + 2 * TC_TILE, &tmh, q_full, 0, row0 + it.qa * TC_B);
        if (it.has_b) {
          tma_load_2d(smem + TC_Q + TC_TILE, &tmq, q_full, 0, row0 + it.qb * TC_B);
          tma_load_2d(smem + TC_Q + 3 * TC_TILE, &tmh, q_full, 0, row0 + it.qb * TC_B);
        }
        for (int kt = it.lo; kt <= it.hi; ++kt, ++kv) {
          const int sl = kv % TC_STAGES;
          if (!mbar_wait(&kv_empty[sl], (static_cast<uint32_t>(kv / TC_STAGES) & 1u) ^ 1u, p.status)) {
            ok = false;
            break;
          }
          uint8_t* stage = smem + TC_RING + sl * 2 * TC_TILE;
          mbar_arrive_expect_tx(&kv_full[sl], 2 * TC_TILE);
          tma_load_2d(stage, &tmk, &kv_full[sl], 0, row0 + kt * TC_B);
          tma_load_2d(stage + TC_TILE, &tmv, &kv_full[sl], 0, row0 + kt * TC_B);
        }
      }
      // drain: the last Q load and the last STAGES ring loads land before the CTA exits
      if (nitem > 0) mbar_wait(q_full, static_cast<uint32_t>(nitem - 1) & 1u, p.status);
      for (int j = kv - 1; j >= 0 && j >= kv - TC_STAGES; --j)
        mbar_wait(&kv_full[j % TC_STAGES], static_cast<uint32_t>(j / TC_STAGES) & 1u, p.status);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(TC_B, TC_B);
      int kv = 0, nitem = 0;
      int s_count[2] = {0, 0};
      bool ok = true;
      for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++nitem) {
        const Item it = item(w);
        const TCRange rg[2] = {it.ra, it.rb};
        if (!mbar_wait(q_full, static_cast<uint32_t>(nitem) & 1u, p.status)) break;
        for (int kt = it.lo; kt <= it.hi && ok; ++kt, ++kv) {
          const int sl = kv % TC_STAGES;
          if (!mbar_wait(&kv_full[sl], static_cast<uint32_t>(kv / TC_STAGES) & 1u, p.status)) {
            ok = false;
            break;
          }
          const uint32_t kd0 = sbase + TC_RING + sl * 2 * TC_TILE;
          for (int g = 0; g < 2 && ok; ++g) {
            if (kt < rg[g].lo || kt > rg[g].hi) continue;
            if (!mbar_wait(&s_empty[g], (static_cast<uint32_t>(s_count[g]) & 1u) ^ 1u, p.status)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t qd = sdesc_kmajor_sw128(sbase + TC_Q + g * TC_TILE);
            const uint64_t hd = sdesc_kmajor_sw128(sbase + TC_Q + (2 + g) * TC_TILE);
            const uint64_t kd = sdesc_kmajor_sw128(kd0), vd = sdesc_kmajor_sw128(kd0 + TC_TILE);
#pragma unroll
            for (int k = 0; k < 4; ++k) tc_mma(tmem + g * 256, qd + 2u * k, kd + 2u * k, idesc, k > 0);
#pragma unroll
            for (int k = 0; k < 4; ++k) tc_mma(tmem + g * 256 + TC_B, hd + 2u * k, vd + 2u * k, idesc, k > 0);
            tc_commit(&s_full[g]);
            ++s_count[g];
          }
          tc_commit(&kv_empty[sl]);
        }
        if (ok) tc_commit(q_empty);
      }
      tc_commit(drain);  // every MMA of this CTA done before TMEM is freed
      mbar_wait(drain, 0, p.status);
    }
  } else {
    // groups: warps 2..5 -> query tile A, 6..9 -> B; thread = query row of the group's tile
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + g * 256, c_addr = s_addr + TC_B;
    constexpr float SL2 = 0.125f * 1.4426950408889634f;
    constexpr float L2E = 1.4426950408889634f;
    int cnt = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < items && ok; w += gridDim.x) {
      const Item it = item(w);
      if (g == 1 && !it.has_b) continue;
      const TCRange rg = g == 0 ? it.ra : it.rb;
      const int tq = (g == 0 ? it.qa : it.qb) * TC_B + r;
      const int qt = g == 0 ? it.qa : it.qb;
      float m = -INFINITY, l = 0.f, sum = 0.f;
      auto tile = [&](auto masked_tag, int kt) {
        constexpr bool MASKED = decltype(masked_tag)::value;
#pragma unroll 1
        for (int c = 0; c < TC_B; c += 32) {
          float s[32], cc[32];
          tmem_ld32(s_addr + c, s);
          tmem_ld32(c_addr + c, cc);
          tc_wait_ld();
          reg_fence<32>(s);
          reg_fence<32>(cc);
          if (c + 32 == TC_B) {  // the tile's last chunk is in registers: TMEM may take the next tile
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s_empty[g]);
          }
          if constexpr (MASKED) {
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const int sk = kt * TC_B + c + e;
              if (sk > tq || tq - sk > p.window) s[e] = -INFINITY;
            }
          }
          float mx = s[0];
#pragma unroll
          for (int e = 1; e < 32; ++e) mx = fmaxf(mx, s[e]);
          const float mn = fmaxf(m, mx * 0.125f);
          if (mn > m) {  // a new maximum: rescale what has been summed (m = -inf the first time: both are 0)
            const float scale = ex2_approx((m - mn) * L2E);
            l *= scale;
            sum *= scale;
            m = mn;
          }
          if (m == -INFINITY) continue;  // every logit so far masked
          const float off = -m * L2E;
          // pairs: packed fp32x2 arithmetic into even / odd partial sums
          float2 l2 = make_float2(0.f, 0.f), sum2 = make_float2(0.f, 0.f);
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float2 arg = __ffma2_rn(make_float2(s[e], s[e + 1]), make_float2(SL2, SL2), make_float2(off, off));
            const float2 pe = make_float2(ex2_approx(arg.x), ex2_approx(arg.y));  // masked: 2^-inf = 0
            l2 = __fadd2_rn(l2, pe);
            sum2 = __ffma2_rn(pe, make_float2(cc[e], cc[e + 1]), sum2);
          }
          l += l2.x + l2.y;
          sum += sum2.x + sum2.y;
        }
      };
      for (int kt = rg.lo; kt <= rg.hi && ok; ++kt, ++cnt) {
        if (!mbar_wait(&s_full[g], static_cast<uint32_t>(cnt) & 1u, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (tc_full(qt, kt, p.window))
          tile(std::false_type{}, kt);
        else
          tile(std::true_type{}, kt);
      }
      if (!ok) break;
      const int64_t o = static_cast<int64_t>(it.row) * p.T + tq;
      p.lse[o] = m + logf(l);
      p.center[o] = sum / l;
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
