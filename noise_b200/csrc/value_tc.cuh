// The credit value pass on tcgen05 (sm_100a), bf16 inputs: out_t = sum_{s: 0 <= s - t <= window}
// exp(q_s . k_t / 8 - lse_s) source_s (reference train/speedrun/moment_kernels.py:612-661, _value_pass), P rounded
// to bf16 and the fp32 source split into bf16 hi + lo (both products accumulate in fp32), as the reference's.
//
// It is the population attention with the roles of queries and keys swapped: one work item = two adjacent 128-key
// tiles A, B of one row sharing every 128-receiver tile; 320 threads, one CTA per SM, persistent:
//   warp 0      TMA: K_A, K_B once, then per receiver tile its q rows, source hi / lo rows and lse values into a
//               2-stage ring (128-byte swizzle for the bf16 tiles);
//   warp 1      TMEM (S_A, S_B 128 columns each, O double-buffered 2 x (64 + 64)); the whole warp runs the issue
//               loop and an elect.sync lane issues S_g = K_g Q^T (M=128 keys, N=128 receivers, K=64) and
//               O_g += P_g hi + P_g lo (M=128, N=64, K=128; hi / lo MN-major operands);
//   warps 2..9  two groups of 4 warps (tile A, tile B), one key row per thread: P = exp2(s log2(e) / 8 - lse_s
//               log2(e)) (<= 1), masked to 0 <= s - t <= window, as bf16 into swizzled shared memory; at the end O
//               (fp32) to the output view.
// The source hi / lo tensors come from split_source_kernel (this file), one pass over the source.
#pragma once
#include <type_traits>

#include "ptx.cuh"

namespace noise {
namespace credit {

__device__ __forceinline__ void tv_st_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

constexpr int TV_B = 128, TV_STAGES = 2, TV_THREADS = 320;
constexpr int TV_TILE = 128 * 128;  // bytes of one [128][64] bf16 tile
constexpr int TV_K = 0;                                   // K_A, K_B
constexpr int TV_RING = TV_K + 2 * TV_TILE;               // stage: Q, hi, lo tiles, then 128 lse floats
constexpr int TV_STAGE = 3 * TV_TILE + 1024;              // (lse padded to keep the tiles 1024-byte aligned)
constexpr int TV_P = TV_RING + TV_STAGES * TV_STAGE;      // P_A, P_B: 2 sub-tiles each (receivers 0..63, 64..127)
constexpr int TV_BAR = TV_P + 4 * TV_TILE;
constexpr int TV_SMEM = TV_BAR + 256 + 1024;

struct TValueArgs {
  int T, window, rows;
  Rows out;      // fp32 [rows, T, 64] view
  int* status;
};

struct TVRange {
  int lo, hi;  // receiver tiles [lo, hi] of key tile kt
};
__device__ __forceinline__ TVRange tv_range(int kt, int window, int nt) {
  return TVRange{kt, min((kt * TV_B + TV_B - 1 + window) / TV_B, nt - 1)};
}
// every receiver of tile st sees every key of tile kt: no mask
__device__ __forceinline__ bool tv_full(int kt, int st, int window) {
  const int t0 = kt * TV_B, s0 = st * TV_B;
  return s0 >= t0 + TV_B - 1 && s0 + TV_B - 1 - t0 <= window;
}

// hi = bf16(source), lo = bf16(source - hi) as contiguous [rows, T, 64] bf16; one thread per 4 channels
__global__ void __launch_bounds__(256) split_source_kernel(Rows src, int T, int64_t n4, __nv_bfloat16* __restrict__ hi,
                                                           __nv_bfloat16* __restrict__ lo) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t tok = i / 16;
    const int c4 = static_cast<int>(i % 16) * 4;
    const int row = static_cast<int>(tok / T), t = static_cast<int>(tok % T);
    const float4 v = *reinterpret_cast<const float4*>(static_cast<const float*>(src.data) + src.base(row) +
                                                      static_cast<int64_t>(t) * src.token_stride + c4);
    const float h0 = bf16_round(v.x), h1 = bf16_round(v.y), h2 = bf16_round(v.z), h3 = bf16_round(v.w);
    *reinterpret_cast<uint2*>(hi + tok * 64 + c4) = make_uint2(pack_bf16x2(h0, h1), pack_bf16x2(h2, h3));
    *reinterpret_cast<uint2*>(lo + tok * 64 + c4) =
        make_uint2(pack_bf16x2(v.x - h0, v.y - h1), pack_bf16x2(v.z - h2, v.w - h3));
  }
}

__global__ void __launch_bounds__(TV_THREADS, 1)
    value_tc_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmq,
                    const __grid_constant__ CUtensorMap tmhi, const __grid_constant__ CUtensorMap tmlo,
                    const __grid_constant__ CUtensorMap tmlse, TValueArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + TV_BAR);
  uint64_t* k_full = bar;                     // K_A / K_B of the current item landed
  uint64_t* k_empty = bar + 1;                // every S MMA of the current item done
  uint64_t* st_full = bar + 2;                // STAGES
  uint64_t* st_empty = st_full + TV_STAGES;   // STAGES
  uint64_t* s_full = st_empty + TV_STAGES;    // per group
  uint64_t* s_empty = s_full + 2;
  uint64_t* p_full = s_empty + 2;
  uint64_t* p_empty = p_full + 2;
  uint64_t* o_full = p_empty + 2;             // per O buffer (items alternate)
  uint64_t* o_empty = o_full + 2;
  uint64_t* drain = o_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = p.T / TV_B;
  const int npairs = (nt + 1) / 2;
  const int items = npairs * p.rows;

  // work item w: key-tile pair pi (the first pairs see the most receivers: heaviest first) of row
  struct Item {
    int row, ka, kb, lo, hi;
    bool has_b;
    TVRange ra, rb;
  };
  auto item = [&](int w) {
    Item it;
    const int pi = w / p.rows;
    it.row = w % p.rows;
    it.ka = 2 * pi;
    it.kb = 2 * pi + 1;
    it.has_b = it.kb < nt;
    it.ra = tv_range(it.ka, p.window, nt);
    it.rb = it.has_b ? tv_range(it.kb, p.window, nt) : TVRange{1, 0};
    it.lo = it.ra.lo;
    it.hi = it.has_b ? max(it.ra.hi, it.rb.hi) : it.ra.hi;
    return it;
  };

  if (threadIdx.x == 0) {
    mbar_init(k_full, 1);
    mbar_init(k_empty, 1);
    for (int s = 0; s < TV_STAGES; ++s) {
      mbar_init(&st_full[s], 1);
      mbar_init(&st_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 4);  // one arrival per warp (after its __syncwarp)
      mbar_init(&p_full[b], 4);
      mbar_init(&p_empty[b], 1);
      mbar_init(&o_full[b], 1);
      mbar_init(&o_empty[b], 8);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmk);
    tma_prefetch_desc(&tmq);
    tma_prefetch_desc(&tmhi);
    tma_prefetch_desc(&tmlo);
    tma_prefetch_desc(&tmlse);
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
      int sv = 0, nitem = 0;  // receiver tiles issued, items started
      bool ok = true;
      for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++nitem) {
        const Item it = item(w);
        const int row0 = it.row * p.T;
        if (!mbar_wait(k_empty, (static_cast<uint32_t>(nitem) & 1u) ^ 1u, p.status)) break;
        mbar_arrive_expect_tx(k_full, (it.has_b ? 2 : 1) * TV_TILE);
        tma_load_2d(smem + TV_K, &tmk, k_full, 0, row0 + it.ka * TV_B);
        if (it.has_b) tma_load_2d(smem + TV_K + TV_TILE, &tmk, k_full, 0, row0 + it.kb * TV_B);
        for (int st = it.lo; st <= it.hi; ++st, ++sv) {
          const int sl = sv % TV_STAGES;
          if (!mbar_wait(&st_empty[sl], (static_cast<uint32_t>(sv / TV_STAGES) & 1u) ^ 1u, p.status)) {
            ok = false;
            break;
          }
          uint8_t* stage = smem + TV_RING + sl * TV_STAGE;
          mbar_arrive_expect_tx(&st_full[sl], 3 * TV_TILE + TV_B * 4);
          tma_load_2d(stage, &tmq, &st_full[sl], 0, row0 + st * TV_B);
          tma_load_2d(stage + TV_TILE, &tmhi, &st_full[sl], 0, row0 + st * TV_B);
          tma_load_2d(stage + 2 * TV_TILE, &tmlo, &st_full[sl], 0, row0 + st * TV_B);
          tma_load_2d(stage + 3 * TV_TILE, &tmlse, &st_full[sl], st * TV_B, it.row);
        }
      }
      // drain: the last K load and the last STAGES ring loads must land before the CTA exits
      if (nitem > 0) mbar_wait(k_full, static_cast<uint32_t>(nitem - 1) & 1u, p.status);
      for (int j = sv - 1; j >= 0 && j >= sv - TV_STAGES; --j)
        mbar_wait(&st_full[j % TV_STAGES], static_cast<uint32_t>(j / TV_STAGES) & 1u, p.status);
    }
  } else if (warp == 1) {
    {  // the whole warp runs the issuer; one elected lane issues the MMAs and commits
      constexpr uint32_t idesc_s = idesc_bf16(TV_B, TV_B);
      constexpr uint32_t idesc_pv = idesc_bf16(TV_B, 64, false, true);
      int sv = 0, nitem = 0;
      int s_count[2] = {0, 0}, pv_count[2] = {0, 0};
      bool ok = true;
      for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++nitem) {
        const Item it = item(w);
        const int ob = nitem & 1;
        const TVRange rg[2] = {it.ra, it.rb};
        auto sees = [&](int g, int st) { return st >= rg[g].lo && st <= rg[g].hi; };
        int first_pv[2] = {1, 1};
        auto issue_pv = [&](int g, int svi) {  // O_g += P_g hi + P_g lo of the receiver tile in ring slot svi
          const int sl = svi % TV_STAGES;
          if (!mbar_wait_warp(&p_full[g], static_cast<uint32_t>(pv_count[g]) & 1u, p.status)) return false;
          tc_fence_after();
          const uint32_t pbase = sbase + TV_P + g * 2 * TV_TILE;
          const uint32_t stage = sbase + TV_RING + sl * TV_STAGE;
#pragma unroll
          for (int part = 0; part < 2; ++part) {  // hi, lo
            const uint32_t bbase = stage + (1 + part) * TV_TILE;
#pragma unroll
            for (int ks = 0; ks < TV_B / 16; ++ks) {
              const uint64_t ad = sdesc_kmajor_sw128(pbase + (ks >> 2) * TV_TILE) + 2u * (ks & 3);
              const uint64_t bd = sdesc_mnmajor_sw128(bbase + ks * 2048, 16);
              if (elect_one())
                tc_mma(tmem + 256 + ob * 128 + g * 64, ad, bd, idesc_pv, !(first_pv[g] && part == 0 && ks == 0));
            }
          }
          first_pv[g] = 0;
          if (elect_one()) tc_commit(&p_empty[g]);
          ++pv_count[g];
          return true;
        };
        if (!mbar_wait_warp(&o_empty[ob], (static_cast<uint32_t>(nitem >> 1) & 1u) ^ 1u, p.status) ||
            !mbar_wait_warp(k_full, static_cast<uint32_t>(nitem) & 1u, p.status)) {
          ok = false;
          break;
        }
        const int sv0 = sv;
        for (int st = it.lo; st <= it.hi && ok; ++st, ++sv) {
          const int sl = sv % TV_STAGES;
          if (!mbar_wait_warp(&st_full[sl], static_cast<uint32_t>(sv / TV_STAGES) & 1u, p.status)) {
            ok = false;
            break;
          }
          const uint64_t qd = sdesc_kmajor_sw128(sbase + TV_RING + sl * TV_STAGE);
          for (int g = 0; g < 2 && ok; ++g) {
            if (!sees(g, st)) continue;
            if (!mbar_wait_warp(&s_empty[g], (static_cast<uint32_t>(s_count[g]) & 1u) ^ 1u, p.status)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t kd = sdesc_kmajor_sw128(sbase + TV_K + g * TV_TILE);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              if (elect_one()) tc_mma(tmem + g * TV_B, kd + 2u * k, qd + 2u * k, idesc_s, k > 0);
            if (elect_one()) tc_commit(&s_full[g]);
            ++s_count[g];
          }
          if (st == it.hi && ok && elect_one()) tc_commit(k_empty);  // the item's last S MMAs read K
          if (st > it.lo && ok) {  // O MMAs of the previous receiver tile, then release its ring slot
            for (int g = 0; g < 2 && ok; ++g)
              if (sees(g, st - 1)) ok = issue_pv(g, sv - 1);
            if (elect_one()) tc_commit(&st_empty[(sv - 1) % TV_STAGES]);
          }
        }
        if (ok) {
          for (int g = 0; g < 2 && ok; ++g)
            if (sees(g, it.hi)) ok = issue_pv(g, sv0 + (it.hi - it.lo));
          if (elect_one()) tc_commit(&st_empty[(sv - 1) % TV_STAGES]);
          if (elect_one()) tc_commit(&o_full[ob]);
        }
      }
      if (elect_one()) tc_commit(drain);  // every MMA of this CTA done before TMEM is freed
      mbar_wait_warp(drain, 0, p.status);
    }
  } else {
    // groups: warps 2..5 -> key tile A, 6..9 -> B; thread = key row of the group's tile
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + g * TV_B;
    const uint32_t prow = sbase + TV_P + g * 2 * TV_TILE + r * 128;
    constexpr float SL2 = 0.125f * 1.4426950408889634f;
    constexpr float L2E = 1.4426950408889634f;
    int cnt = 0, nitem = 0, sv = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++nitem) {
      const Item it = item(w);
      const int ob = nitem & 1;
      const TVRange rg = g == 0 ? it.ra : it.rb;
      const int tk = (g == 0 ? it.ka : it.kb) * TV_B + r;
      const bool active = g == 0 || it.has_b;
      const int kt = g == 0 ? it.ka : it.kb;
      auto tile = [&](auto masked_tag, int st, int svi) {
        constexpr bool MASKED = decltype(masked_tag)::value;
        float v[TV_B];
#pragma unroll
        for (int c = 0; c < TV_B; c += 32) tmem_ld32(s_addr + c, v + c);
        tc_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_empty[g]);
        const float* lse = reinterpret_cast<const float*>(smem + TV_RING + (svi % TV_STAGES) * TV_STAGE + 3 * TV_TILE);
#pragma unroll
        for (int c = 0; c < TV_B; c += 8) {
          const float4 l0 = *reinterpret_cast<const float4*>(lse + c), l1 = *reinterpret_cast<const float4*>(lse + c + 4);
          const float lv[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
          float pe[8];
#pragma unroll
          for (int e = 0; e < 8; e += 2) {  // pairs: packed fp32x2 FMAs, the rounding of scalar ones
            const float2 nl = __fmul2_rn(make_float2(-lv[e], -lv[e + 1]), make_float2(L2E, L2E));
            const float2 arg = __ffma2_rn(make_float2(v[c + e], v[c + e + 1]), make_float2(SL2, SL2), nl);
            pe[e] = ex2_approx(arg.x);
            pe[e + 1] = ex2_approx(arg.y);
          }
          if constexpr (MASKED) {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int s = st * TV_B + c + e;
              if (s < tk || s - tk > p.window) pe[e] = 0.f;
            }
          }
          if (c == 0 && !mbar_wait(&p_empty[g], (static_cast<uint32_t>(cnt) & 1u) ^ 1u, p.status)) return false;
          const int chunk = (c & 63) >> 3;  // receivers c .. c + 7: sub-tile c / 64, chunk (c % 64) / 8, 128-B swizzle
          tv_st_v4(prow + (c >> 6) * TV_TILE + ((chunk ^ (r & 7)) << 4), pack_bf16x2(pe[0], pe[1]),
                       pack_bf16x2(pe[2], pe[3]), pack_bf16x2(pe[4], pe[5]), pack_bf16x2(pe[6], pe[7]));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[g]);
        return true;
      };
      // the item's receiver tiles run through ring slots sv .. sv + (hi - lo); this group's start at lo_g
      if (active) {
        for (int st = rg.lo; st <= rg.hi && ok; ++st, ++cnt) {
          if (!mbar_wait(&s_full[g], static_cast<uint32_t>(cnt) & 1u, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int svi = sv + (st - it.lo);
          ok = tv_full(kt, st, p.window) ? tile(std::false_type{}, st, svi) : tile(std::true_type{}, st, svi);
        }
      }
      sv += it.hi - it.lo + 1;
      if (!ok || !mbar_wait(&o_full[ob], static_cast<uint32_t>(nitem >> 1) & 1u, p.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float o[64];
      const uint32_t o_addr = tmem + lane_base + 256 + ob * 128 + g * 64;
      tmem_ld32(o_addr, o);
      tmem_ld32(o_addr + 32, o + 32);
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[ob]);
      if (active) {
        float* out = static_cast<float*>(p.out.data) + p.out.base(it.row) + static_cast<int64_t>(tk) * p.out.token_stride;
#pragma unroll
        for (int d = 0; d < 64; d += 4)
          *reinterpret_cast<float4*>(out + d) = make_float4(o[d], o[d + 1], o[d + 2], o[d + 3]);
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
