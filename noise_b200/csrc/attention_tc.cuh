// Windowed causal attention on tcgen05 (sm_100a) for the population forward: softmax(q k^T / 8) v with key s
// visible to query t iff 0 <= t - s <= window (reference utils/model.py:17-31, flex attention).
//
// q and k reach this kernel RMS-normalised per head (utils/model.py:94; EpiQKV), so |q|, |k| <= 8 (8.03 after bf16
// rounding) and every logit q.k / 8 <= 8.03. Softmax is shift invariant, so the kernel uses the fixed offset 8 in place
// of a running row maximum: p = exp(q.k / 8 - 8) <= 1.03 never overflows, there is no max pass and no rescaling of the
// accumulator, and O = sum_j P_j V_j accumulates straight in tensor memory across key tiles.
//
// One CTA per (member x head, pair of 128-query tiles A = 2i, B = 2i + 1), 320 threads:
//   warp 0      TMA: Q_A, Q_B once, then 128-key K / V tiles (the union of both tiles' key ranges) into a 3-stage
//               ring (128-byte swizzle); both query tiles share every K / V load;
//   warp 1      TMEM (512 columns: S_A, S_B 128 each, O_A, O_B 64 each, P_A, P_B 64 each); the whole warp runs
//               the issue loop and an elect.sync lane issues, per key tile, S_w = Q_w K^T (M=128, N=128, K=64) for
//               each tile w that sees it, then O_w += P_w V of
//               the previous key tile (M=128, N=64, K=128; P the A operand read from tensor memory, V an MN-major
//               shared-memory operand);
//   warps 2..5  softmax group A, warps 6..9 group B: one query row per thread; S_w is read with one batched
//               tcgen05.ld and released at once, P = exp2(s log2(e) / 8 - 8 log2(e)) goes as packed bf16 pairs into
//               the group's P columns of tensor memory (tcgen05.st; the A operand of the next O MMA, so the MMAs read
//               only V from shared memory), every exponential on the MUFU pipe (moving a share to an FMA
//               polynomial measured slower); at the end y = O / l (bf16) and the per-head partial dot y . b of the
//               c_proj rank-1 term.
// Only the diagonal key tile and the window's first tile take the masked path.
#pragma once
#include <type_traits>

#include "ptx.cuh"

namespace noise {

constexpr int TA_BQ = 128, TA_BK = 128, TA_STAGES = 3, TA_THREADS = 320;
constexpr int TA_TILE = 128 * 128;  // bytes of one [128][64] bf16 tile
constexpr int TA_Q = 0;             // Q_A, Q_B
constexpr int TA_K = TA_Q + 2 * TA_TILE;
constexpr int TA_V = TA_K + TA_STAGES * TA_TILE;
constexpr int TA_P = TA_V + TA_STAGES * TA_TILE;  // epilogue staging per group: y rows, the head's b
constexpr int TA_BAR = TA_P + 4 * TA_TILE;
constexpr int TA_SMEM = TA_BAR + 256 + 1024;
constexpr uint32_t TA_TS = 0, TA_TO = 256, TA_TP = 384;  // TMEM columns: S_A | S_B, O_A | O_B, P_A | P_B

struct TAttnArgs {
  int T, window;
  int bh;            // member x head rows of q / k / v (each T tokens)
  __nv_bfloat16* y;  // [M, 512]
  float* ydot;       // [M, 8]
  Slice nproj;       // c_proj noise: b used
  int* status;
  const float* jit;  // [M, 512] fp32 added to the attention output before c_proj, or NULL (Dust's o jitter site)
  int order;         // attention_item's order
  int* next_item;    // order 2: the launch's next unclaimed work item (zeroed before the launch)
};

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void st_shared_f32(uint32_t addr, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// Work item w of a launch over bh head rows (member x head), npairs pairs of 128-query tiles each, dealt round-robin
// to `grid` persistent CTAs (CTA c takes w = c, c + grid, ...): its pair index pi and head row.
//   order 0: heaviest pair first over the whole launch, head rows inner, so each round of the grid takes one pair
//            level (equal cost); a head row's pairs are 1 / npairs of the launch apart, so its keys and values come
//            from HBM once per pair.
//   order 1: blocks of `grid` head rows, each block heaviest pair first: CTA c takes every pair of head row
//            blk grid + c in turn, so the row's keys and values come from HBM once and then from L2, while each round
//            still takes one pair level. The rows past the last whole block are dealt heaviest first over all CTAs.
//   order 2: head-major, a row's pairs heaviest first; the CTAs claim items in this order from a launch-wide counter
//            as they finish their previous one, so the CTAs working on a head row at once share its keys and values
//            through L2 within a few items, and the unequal costs of the pair levels balance dynamically.
// All are bijections of [0, npairs bh) onto (pair, row).
__host__ __device__ inline void attention_item(int order, int w, int bh, int npairs, int grid, int& pi, int& row) {
  if (order == 2) {  // head-major, heaviest pair first within a row; the items are claimed dynamically
    pi = npairs - 1 - w % npairs;
    row = w / npairs;
    return;
  }
  const int per = grid * npairs, full = order == 1 ? bh / grid : 0;
  if (w < full * per) {
    const int r = w % per;
    pi = npairs - 1 - r / grid;
    row = w / per * grid + r % grid;
  } else {
    const int rest = bh - full * grid, r = w - full * per;
    pi = npairs - 1 - r / rest;
    row = full * grid + r % rest;
  }
}

// Key-tile range [lo, hi] of query tile qt and whether its first tile is cut by the window.
struct TileRange {
  int lo, hi;
  bool edge;
};
__device__ __forceinline__ TileRange tile_range(int qt, int window) {
  const int q0 = qt * TA_BQ;
  const bool edge = q0 - window >= 0;
  return TileRange{edge ? (q0 - window) / TA_BK : 0, q0 / TA_BK, edge};
}

// JIT: add TAttnArgs::jit to the attention output (Dust's o jitter site). DYN: take work items in order 2 from the
// launch-wide counter p.next_item (the producer lane claims one, then hands its index to the MMA and softmax warps
// through a 2-slot ring in shared memory); otherwise CTA c takes items c, c + grid, ...
template <bool JIT, bool DYN>
__global__ void __launch_bounds__(TA_THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                        const __grid_constant__ CUtensorMap tmv, TAttnArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + TA_BAR);
  uint64_t* q_full = bar;                    // Q_A / Q_B of the current item landed
  uint64_t* q_empty = bar + 1;               // every S MMA of the current item done
  uint64_t* kv_full = bar + 2;               // STAGES
  uint64_t* kv_empty = kv_full + TA_STAGES;  // STAGES
  uint64_t* s_full = kv_empty + TA_STAGES;   // per group
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_empty + 2;
  uint64_t* p_empty = p_full + 2;
  uint64_t* o_full = p_empty + 2;            // [0]: all MMAs of the item done ([1] unused)
  uint64_t* o_empty = o_full + 2;            // per group: the group's warps read its O
  uint64_t* drain = o_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  uint64_t* item_full = bar + 22;                           // DYN: slot's item index written (2)
  uint64_t* item_empty = bar + 24;                          // DYN: slot read by the MMA warp and 8 softmax warps (2)
  volatile int* item_slot = reinterpret_cast<int*>(bar + 26);  // DYN: 2 item indices (-1: no more work)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = p.T / TA_BQ;
  const int npairs = (nq + 1) / 2;
  const int items = npairs * p.bh;

  // work item w: pair pi of head-row bh (attention_item: every round of CTAs takes equal-cost items)
  struct Item {
    int bh, qa, qb, lo, hi;
    bool has_b;
    TileRange ra, rb;
  };
  auto item = [&](int w) {
    Item it;
    int pi;
    attention_item(p.order, w, p.bh, npairs, static_cast<int>(gridDim.x), pi, it.bh);
    it.qa = 2 * pi;
    it.qb = 2 * pi + 1;
    it.has_b = it.qb < nq;
    it.ra = tile_range(it.qa, p.window);
    it.rb = it.has_b ? tile_range(it.qb, p.window) : TileRange{it.ra.lo, it.ra.lo - 1, false};
    it.lo = it.ra.lo;
    it.hi = it.has_b ? it.rb.hi : it.ra.hi;
    return it;
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < TA_STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 4);  // one arrival per softmax warp of the group (after its __syncwarp)
      mbar_init(&p_full[b], 4);
      mbar_init(&p_empty[b], 1);
      mbar_init(&o_full[b], 1);
      mbar_init(&o_empty[b], 4);
    }
    mbar_init(drain, 1);
    if constexpr (DYN) {
      for (int b = 0; b < 2; ++b) {
        mbar_init(&item_full[b], 1);
        mbar_init(&item_empty[b], 9);
      }
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmq);
    tma_prefetch_desc(&tmk);
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
  // the CTA's n-th work item without DYN: c + n grid (-1 past the launch's items)
  auto static_item = [&](int n) {
    const int w = static_cast<int>(blockIdx.x) + n * static_cast<int>(gridDim.x);
    return w < items ? w : -1;
  };
  // DYN, the producer lane: claim the launch's next item for the CTA's n-th and hand its index over in slot n % 2
  // (-1 once the launch's items are gone; -2 if the slot's wait gave up)
  auto claim_item = [&](int n) {
    const int slot = n & 1;
    if (!mbar_wait(&item_empty[slot], (static_cast<uint32_t>(n >> 1) & 1u) ^ 1u, p.status)) return -2;
    int w = atomicAdd(p.next_item, 1);
    if (w >= items) w = -1;
    item_slot[slot] = w;
    mbar_arrive(&item_full[slot]);
    return w;
  };
  // DYN, the MMA and softmax warps: the CTA's n-th item index from slot n % 2, then the slot is released (one arrival
  // per warp); the wait is warp-wide, so every lane of a warp gets the same index
  auto take_item = [&](int n) {
    const int slot = n & 1;
    if (!mbar_wait_warp(&item_full[slot], static_cast<uint32_t>(n >> 1) & 1u, p.status)) return -2;
    const int w = item_slot[slot];
    __syncwarp();
    if (lane == 0) mbar_arrive(&item_empty[slot]);
    return w;
  };

  if (warp == 0) {
    if (lane == 0) {
      int kv = 0, nitem = 0;  // K / V tiles issued, items started
      bool ok = true;
      auto next = [&](int n) {
        if constexpr (DYN) return claim_item(n);
        else return static_item(n);
      };
      for (int w = next(0); w >= 0 && ok; ++nitem, w = ok ? next(nitem) : -1) {
        const Item it = item(w);
        const int row0 = it.bh * p.T;
        if (!mbar_wait(q_empty, (static_cast<uint32_t>(nitem) & 1u) ^ 1u, p.status)) break;
        mbar_arrive_expect_tx(q_full, (it.has_b ? 2 : 1) * TA_TILE);
        tma_load_2d(smem + TA_Q, &tmq, q_full, 0, row0 + it.qa * TA_BQ);
        if (it.has_b) tma_load_2d(smem + TA_Q + TA_TILE, &tmq, q_full, 0, row0 + it.qb * TA_BQ);
        for (int kt = it.lo; kt <= it.hi; ++kt, ++kv) {
          const int st = kv % TA_STAGES;
          if (!mbar_wait(&kv_empty[st], (static_cast<uint32_t>(kv / TA_STAGES) & 1u) ^ 1u, p.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[st], 2 * TA_TILE);
          tma_load_2d(smem + TA_K + st * TA_TILE, &tmk, &kv_full[st], 0, row0 + kt * TA_BK);
          tma_load_2d(smem + TA_V + st * TA_TILE, &tmv, &kv_full[st], 0, row0 + kt * TA_BK);
        }
      }
      // drain: the last Q load and the last STAGES K / V loads must land before the CTA exits
      if (nitem > 0) mbar_wait(q_full, static_cast<uint32_t>(nitem - 1) & 1u, p.status);
      for (int j = kv - 1; j >= 0 && j >= kv - TA_STAGES; --j)
        mbar_wait(&kv_full[j % TA_STAGES], static_cast<uint32_t>(j / TA_STAGES) & 1u, p.status);
    }
  } else if (warp == 1) {
    {  // the whole warp runs the issuer; one elected lane issues the MMAs and commits
      constexpr uint32_t idesc_s = idesc_bf16(TA_BQ, TA_BK);
      constexpr uint32_t idesc_pv = idesc_bf16(TA_BQ, 64, false, true);
      int kv = 0, nitem = 0;
      int s_count[2] = {0, 0}, pv_count[2] = {0, 0};
      bool ok = true;
      auto next = [&](int n) {
        if constexpr (DYN) return take_item(n);
        else return static_item(n);
      };
      for (int w = next(0); w >= 0 && ok; ++nitem, w = ok ? next(nitem) : -1) {
        const Item it = item(w);
        const TileRange rg[2] = {it.ra, it.rb};
        auto sees = [&](int g, int kt) { return kt >= rg[g].lo && kt <= rg[g].hi; };
        int first_pv[2] = {1, 1};  // the item's first O MMA overwrites the accumulator
        bool o_free = false;       // both groups have read O of the previous item
        auto issue_pv = [&](int g, int kt, int kvi) {  // O_g += P_g V of key tile kt (ring slot of tile kvi)
          const int st = kvi % TA_STAGES;
          // the item's first O MMA overwrites O: both groups must have read theirs (item nitem - 1). Waiting for both
          // keeps o_full at most one phase ahead of every group's wait on it, inactive group B included.
          if (!o_free) {
            const uint32_t par = (static_cast<uint32_t>(nitem) & 1u) ^ 1u;
            if (!mbar_wait_warp(&o_empty[0], par, p.status) || !mbar_wait_warp(&o_empty[1], par, p.status))
              return false;
            o_free = true;
          }
          if (!mbar_wait_warp(&p_full[g], static_cast<uint32_t>(pv_count[g]) & 1u, p.status)) return false;
          tc_fence_after();
          const uint32_t vbase = sbase + TA_V + st * TA_TILE;
#pragma unroll
          for (int ks = 0; ks < TA_BK / 16; ++ks) {  // P columns ks * 8 .. + 7: keys 16 ks .. 16 ks + 15
            const uint64_t bd = sdesc_mnmajor_sw128(vbase + ks * 2048, 16);
            if (elect_one())
              tc_mma_ts(tmem + TA_TO + g * 64, tmem + TA_TP + g * 64 + ks * 8, bd, idesc_pv, !(first_pv[g] && ks == 0));
          }
          first_pv[g] = 0;
          if (elect_one()) tc_commit(&p_empty[g]);
          ++pv_count[g];
          return true;
        };
        if (!mbar_wait_warp(q_full, static_cast<uint32_t>(nitem) & 1u, p.status)) {
          ok = false;
          break;
        }
        const int kv0 = kv;
        for (int kt = it.lo; kt <= it.hi && ok; ++kt, ++kv) {
          const int st = kv % TA_STAGES;
          if (!mbar_wait_warp(&kv_full[st], static_cast<uint32_t>(kv / TA_STAGES) & 1u, p.status)) {
            ok = false;
            break;
          }
          const uint64_t kd = sdesc_kmajor_sw128(sbase + TA_K + st * TA_TILE);
          for (int g = 0; g < 2 && ok; ++g) {
            if (!sees(g, kt)) continue;
            if (!mbar_wait_warp(&s_empty[g], (static_cast<uint32_t>(s_count[g]) & 1u) ^ 1u, p.status)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t qd = sdesc_kmajor_sw128(sbase + TA_Q + g * TA_TILE);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              if (elect_one()) tc_mma(tmem + g * TA_BK, qd + 2u * k, kd + 2u * k, idesc_s, k > 0);
            if (elect_one()) tc_commit(&s_full[g]);
            ++s_count[g];
          }
          if (kt == it.hi && ok && elect_one()) tc_commit(q_empty);  // the item's last S MMAs read Q
          if (kt > it.lo && ok) {  // O MMAs of the previous key tile, then release its ring slot
            for (int g = 0; g < 2 && ok; ++g)
              if (sees(g, kt - 1)) ok = issue_pv(g, kt - 1, kv - 1);
            if (elect_one()) tc_commit(&kv_empty[(kv - 1) % TA_STAGES]);
          }
        }
        if (ok) {
          for (int g = 0; g < 2 && ok; ++g)
            if (sees(g, it.hi)) ok = issue_pv(g, it.hi, kv0 + (it.hi - it.lo));
          if (elect_one()) {
            tc_commit(&kv_empty[(kv - 1) % TA_STAGES]);
            tc_commit(&o_full[0]);
          }
        }
      }
      if (elect_one()) tc_commit(drain);  // every MMA of this CTA done before TMEM is freed
      mbar_wait_warp(drain, 0, p.status);
    }
  } else {
    // softmax groups: warps 2..5 -> group A, 6..9 -> group B; thread = query row of the group's tile
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + g * TA_BK;
    const uint32_t p_addr = tmem + lane_base + TA_TP + g * 64;  // this row's 64 P columns
    constexpr float SL2 = 0.125f * 1.4426950408889634f;  // 1/8 in base 2
    constexpr float OFF = 8.f * 1.4426950408889634f;     // the fixed offset 8 in base 2
    int cnt = 0, nitem = 0;
    bool ok = true;
    auto next = [&](int n) {
      if constexpr (DYN) return take_item(n);
      else return static_item(n);
    };
    for (int w = next(0); w >= 0 && ok; ++nitem, w = ok ? next(nitem) : -1) {
      const Item it = item(w);
      const TileRange rg = g == 0 ? it.ra : it.rb;
      const int tq = (g == 0 ? it.qa : it.qb) * TA_BQ + r;
      const bool active = g == 0 || it.has_b;
      float l = 0.f;
      auto tile = [&](auto masked_tag, int kt) {
        constexpr bool MASKED = decltype(masked_tag)::value;
        float v[TA_BK];
#pragma unroll
        for (int c = 0; c < TA_BK; c += 32) tmem_ld32(s_addr + c, v + c);
        tc_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[g]);  // S is in registers: the next S MMA may overwrite it
        uint32_t pk[TA_BK / 2];
        // packed fp32x2 FMA / add (one instruction for two keys; the same rounding as two scalar ones)
        float2 rs2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < TA_BK; c += 8) {
          float pe[8];
#pragma unroll
          for (int e = 0; e < 8; e += 2) {
            const float2 x = __ffma2_rn(make_float2(v[c + e], v[c + e + 1]), make_float2(SL2, SL2),
                                        make_float2(-OFF, -OFF));
            pe[e] = ex2_approx(x.x);
            pe[e + 1] = ex2_approx(x.y);
            if constexpr (MASKED) {
#pragma unroll
              for (int i = 0; i < 2; ++i) {
                const int key = kt * TA_BK + c + e + i;
                if (key > tq || tq - key > p.window) pe[e + i] = 0.f;
              }
            }
            rs2 = __fadd2_rn(rs2, make_float2(pe[e], pe[e + 1]));
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) pk[c / 2 + e] = pack_bf16x2(pe[2 * e], pe[2 * e + 1]);
        }
        const float rs = rs2.x + rs2.y;
        // the P buffer is free once the previous O MMA of this group completed
        if (!mbar_wait(&p_empty[g], (static_cast<uint32_t>(cnt) & 1u) ^ 1u, p.status)) return false;
        __syncwarp();  // tcgen05.st is warp-aligned
        tc_fence_after();
        // column i of the row holds keys 2 i (low half) and 2 i + 1 (high half)
#pragma unroll
        for (int c = 0; c < TA_BK / 2; c += 16) tmem_st16(p_addr + c, pk + c);
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[g]);
        l += rs;
        return true;
      };
      if (active) {
        for (int kt = rg.lo; kt <= rg.hi && ok; ++kt, ++cnt) {
          if (!mbar_wait(&s_full[g], static_cast<uint32_t>(cnt) & 1u, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const bool masked = kt == rg.hi || (rg.edge && kt == rg.lo);
          ok = masked ? tile(std::true_type{}, kt) : tile(std::false_type{}, kt);
        }
      }
      // this head's 64 values of the c_proj noise b, two per lane: loaded before the wait for O, so their latency
      // overlaps it
      float bq0 = 0.f, bq1 = 0.f;
      if (ok && active) {
        const float* bproj = p.nproj.B(it.bh / NOISE_N_HEAD) + (it.bh % NOISE_N_HEAD) * 64;
        bq0 = bproj[lane];
        bq1 = bproj[lane + 32];
      }
      if (!ok || !mbar_wait(&o_full[0], static_cast<uint32_t>(nitem) & 1u, p.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float o[64];
      const uint32_t o_addr = tmem + lane_base + TA_TO + g * 64;
      tmem_ld32(o_addr, o);
      tmem_ld32(o_addr + 32, o + 32);
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[g]);
      if (active) {
        const int j = it.bh / NOISE_N_HEAD, hh = it.bh % NOISE_N_HEAD;
        const int64_t row = static_cast<int64_t>(j) * p.T + tq;
        const float inv = 1.f / l;
        // The warp's own 32 rows of this group's staging area (only this warp uses them): sub-tile 1 holds the
        // head's b, sub-tile 0 stages the y rows (16-byte chunk c of row rl at c ^ (rl % 8)) so the global stores
        // cover whole 128-byte row segments.
        const uint32_t wst = sbase + TA_P + g * 2 * TA_TILE + quarter * 32 * 128;
        const uint32_t wb = wst + TA_TILE;
        st_shared_f32(wb + lane * 4, bf16_round(bq0));
        st_shared_f32(wb + (lane + 32) * 4, bf16_round(bq1));
        __syncwarp();
        float dp[2] = {0.f, 0.f};
#pragma unroll
        for (int d = 0; d < 64; d += 8) {
          const uint4 b0 = ld_shared_v4(wb + d * 4), b1 = ld_shared_v4(wb + d * 4 + 16);
          const float bv[8] = {__uint_as_float(b0.x), __uint_as_float(b0.y), __uint_as_float(b0.z),
                               __uint_as_float(b0.w), __uint_as_float(b1.x), __uint_as_float(b1.y),
                               __uint_as_float(b1.z), __uint_as_float(b1.w)};
          float yv[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            yv[e] = bf16_round(o[d + e] * inv);
            if constexpr (JIT) yv[e] = bf16_round(yv[e] + p.jit[row * NOISE_N_EMBD + hh * 64 + d + e]);
            dp[e & 1] = fmaf(yv[e], bv[e], dp[e & 1]);
          }
          st_shared_v4(wst + lane * 128 + (((d >> 3) ^ (lane & 7)) << 4), pack_bf16x2(yv[0], yv[1]),
                       pack_bf16x2(yv[2], yv[3]), pack_bf16x2(yv[4], yv[5]), pack_bf16x2(yv[6], yv[7]));
        }
        p.ydot[row * NOISE_N_HEAD + hh] = dp[0] + dp[1];
        __syncwarp();
        const int64_t row_w0 = row - lane;  // the warp's 32 rows are consecutive
        const int c = lane & 7;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int rl = (lane >> 3) + 4 * i;
          *reinterpret_cast<uint4*>(p.y + (row_w0 + rl) * NOISE_N_EMBD + hh * 64 + c * 8) =
              ld_shared_v4(wst + rl * 128 + ((c ^ (rl & 7)) << 4));
        }
        __syncwarp();
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

}  // namespace noise
