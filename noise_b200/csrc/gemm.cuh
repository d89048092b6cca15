// Persistent, warp-specialised "TN" GEMM for sm_100a: D[M, N] = A[M, K] . B[N, K]^T with both operands K-major in
// HBM (activations row-major, nn.Linear weights [out, in]), fp32 accumulation in tensor memory, and a fused per-row
// epilogue supplied as a functor. Operands are bf16 (kind::f16) or, with TF32, fp32 read as tf32 (kind::tf32: what
// torch.set_float32_matmul_precision('high') gives an fp32 matmul). A shared-memory tile row is 128 bytes either way:
// 64 bf16 or 32 fp32 values of K.
//
// Roles (320 threads, one CTA per SM):
//   warp 0      one lane issues TMA tile loads (128-byte swizzle) into a STAGES-deep shared-memory ring;
//   warp 1      allocates 2 x BN TMEM columns (double-buffered accumulator); one lane issues tcgen05.mma
//               (M = 128, N = BN, K = 16 per instruction) and tcgen05.commit to release ring slots / publish tiles;
//   warps 2..9  epilogue: warp w reads TMEM lane quarter (w % 4), i.e. one output row per thread; the two warps of a
//               quarter split the tile's columns into halves (part 0 / 1). Column chunks come from tcgen05.ld 32x32b
//               and go to the functor; then the accumulator buffer is released.
// Schedule: CTA c owns row blocks c, c + grid, ...; for each it walks all N tiles in order, so an epilogue can carry
// per-row state (a running log-sum-exp, a partial dot product) across the N tiles of its row.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "ptx.cuh"

namespace noise {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_EPI_WARPS = 8;
constexpr int GEMM_THREADS = 64 + 32 * GEMM_EPI_WARPS;

// Named barrier 1 over the epilogue warps, returning the AND of every thread's predicate.
__device__ __forceinline__ bool epi_barrier_and(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\t"
      "bar.red.and.pred p, 1, %2, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred)), "n"(32 * GEMM_EPI_WARPS)
      : "memory");
  return r != 0;
}

// CH accumulator columns of this thread's row from TMEM (issued only: the caller waits with tc_wait_ld).
template <int CH>
__device__ __forceinline__ void load_chunk(uint32_t taddr, float* v) {
  if constexpr (CH == 64) {
    tmem_ld32(taddr, v);
    tmem_ld32(taddr + 32, v + 32);
  } else if constexpr (CH == 32) {
    tmem_ld32(taddr, v);
  } else {
    tmem_ld16(taddr, v);
  }
}

template <int BN, int STAGES>
struct GemmLayout {
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;
  static constexpr int B_BYTES = BN * GEMM_BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int SCRATCH_BYTES = 4 * 2 * BN;  // per accumulator buffer: two fp32 vectors of the tile's width
  static constexpr int SCRATCH_OFFSET = STAGES * STAGE_BYTES;
  static constexpr int STAGING_BYTES = 4096;         // per epilogue warp: one 32-row x 128-byte chunk
  static constexpr int STAGING_OFFSET = SCRATCH_OFFSET + 2 * SCRATCH_BYTES;
  static constexpr int BAR_OFFSET = STAGING_OFFSET + GEMM_EPI_WARPS * STAGING_BYTES;
  static constexpr int SMEM_BYTES = BAR_OFFSET + 8 * (2 * STAGES + 5) + 16 + 1024;  // + 1024 alignment slack
  static constexpr int TMEM_COLS = 2 * BN;
  static_assert(BN % 16 == 0 && BN >= 32 && BN <= 256, "tcgen05 M=128 needs N in [16, 256], N % 16 == 0");
  static_assert((TMEM_COLS & (TMEM_COLS - 1)) == 0, "TMEM allocation must be a power of two");
};

// Epilogue functor contract (all methods run on a thread that owns `row` and column half `part` of every tile):
//   static constexpr int CH;                          columns per TMEM load (16, 32 or 64)
//   static constexpr bool PIPELINED;                  load chunk i + 1 from TMEM while chunk i is processed (two
//                                                     register buffers: for epilogues with registers to spare)
//   void row_begin(int row, int part);                before the first N tile of the row block
//   void stage(int row0, int col0, float* s, int tid); before every tile, all 256 epilogue threads (tid 0..255):
//                                                     may fill s[0 .. 2 BN) (16-byte aligned shared memory) with
//                                                     per-tile vectors; the tile's chunks run after a barrier
//   float* scratch; uint32_t stg;                     set by the kernel: the staged vectors of the current tile, and
//                                                     the shared address of the warp's 4 KB staging tile
//   void chunk(int row, int col, float* v);           v[0..CH) = D[row, col .. col + CH) (may be modified in place)
//   void tile_end(int row, int n_tile, int part);     after the last chunk of the thread's half of a tile
//   void row_end(int row, int part);                  after the last N tile
template <int BN, int STAGES, class Epi, bool TF32 = false>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_bf16_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        int m_tiles, int n_tiles, int k_blocks, Epi epi, int* status) {
  using L = GemmLayout<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFFSET);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;
  uint64_t* acce = accf + 2;
  uint64_t* drain = acce + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], GEMM_EPI_WARPS);  // one arrival per epilogue warp (after its __syncwarp)
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, L::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int mb = blockIdx.x; mb < m_tiles && ok; mb += gridDim.x)
        for (int nb = 0; nb < n_tiles && ok; ++nb)
          for (int kb = 0; kb < k_blocks; ++kb) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, status)) {
              ok = false;
              break;
            }
            uint8_t* a = smem + stage * L::STAGE_BYTES;
            mbar_arrive_expect_tx(&full[stage], L::STAGE_BYTES);
            constexpr int KE = TF32 ? GEMM_BK / 2 : GEMM_BK;  // K elements of a 128-byte tile row
            tma_load_2d(a, &tmA, &full[stage], kb * KE, mb * GEMM_BM);
            tma_load_2d(a + L::A_BYTES, &tmB, &full[stage], kb * KE, nb * BN);
            ++issued;
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
      // Drain: the last min(issued, STAGES) loads must have landed before the CTA may exit.
      for (int i = 0; i < STAGES && i < issued; ++i) {
        if (--stage < 0) {
          stage = STAGES - 1;
          phase ^= 1u;
        }
        mbar_wait(&full[stage], phase, status);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = TF32 ? idesc_tf32(GEMM_BM, BN) : idesc_bf16(GEMM_BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int t = 0;
      bool ok = true;
      for (int mb = blockIdx.x; mb < m_tiles && ok; mb += gridDim.x)
        for (int nb = 0; nb < n_tiles && ok; ++nb, ++t) {
          const int buf = t & 1;
          const uint32_t use = static_cast<uint32_t>(t >> 1);
          if (!mbar_wait(&acce[buf], (use & 1u) ^ 1u, status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + static_cast<uint32_t>(buf * BN);
          for (int kb = 0; kb < k_blocks; ++kb) {
            if (!mbar_wait(&full[stage], phase, status)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a = smem_u32(smem + stage * L::STAGE_BYTES);
            const uint64_t ad = sdesc_kmajor_sw128(a), bd = sdesc_kmajor_sw128(a + L::A_BYTES);
#pragma unroll
            for (int k = 0; k < GEMM_BK / 16; ++k) {  // +32 bytes along K = +2 in the 16-byte address field
              if constexpr (TF32)
                tc_mma_tf32(d, ad + 2u * k, bd + 2u * k, idesc, (kb | k) != 0);
              else
                tc_mma(d, ad + 2u * k, bd + 2u * k, idesc, (kb | k) != 0);
            }
            tc_commit(&empty[stage]);
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (ok) tc_commit(&accf[buf]);
        }
      // Drain every MMA this thread issued before TMEM is freed.
      tc_commit(drain);
      mbar_wait(drain, 0, status);
    }
  } else {
    Epi e = epi;  // per-thread copy: the functor may carry per-row state
    // this warp's 32 x 128-byte staging tile (rows swizzled in 16-byte chunks: chunk c of row r at c ^ (r % 8)), for
    // epilogues that turn a thread-per-row chunk into row-contiguous global accesses
    e.stg = smem_u32(smem + L::STAGING_OFFSET + (warp - 2) * L::STAGING_BYTES);
    const int quarter = warp & 3;
    const int part = (warp - 2) >> 2;  // column half of every tile this warp handles
    const int r_in = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    constexpr int HALF = BN / 2;
    static_assert(HALF % Epi::CH == 0, "epilogue chunk must divide half a tile");
    int t = 0;
    bool ok = true;
    for (int mb = blockIdx.x; mb < m_tiles && ok; mb += gridDim.x) {
      const int row = mb * GEMM_BM + r_in;
      e.row_begin(row, part);
      for (int nb = 0; nb < n_tiles; ++nb, ++t) {
        const int buf = t & 1;
        const uint32_t use = static_cast<uint32_t>(t >> 1);
        const bool waited = mbar_wait(&accf[buf], use & 1u, status);
        tc_fence_after();
        // per-tile shared vectors (double-buffered by accumulator buffer: the barrier of tile t + 1 orders every
        // reader of tile t before the writers of tile t + 2). The barrier also ANDs every epilogue thread's wait
        // result, so all of them leave the loop together when a bounded wait gives up.
        float* scratch = reinterpret_cast<float*>(smem + L::SCRATCH_OFFSET + buf * L::SCRATCH_BYTES);
        e.stage(mb * GEMM_BM, nb * BN, scratch, threadIdx.x - 64);
        ok = epi_barrier_and(waited);
        e.scratch = scratch;
        if (ok && !Epi::PIPELINED) {
          const uint32_t base = tmem + lane_base + static_cast<uint32_t>(buf * BN + part * HALF);
#pragma unroll 1
          for (int c = 0; c < HALF; c += Epi::CH) {
            float v[Epi::CH];
            load_chunk<Epi::CH>(base + c, v);
            tc_wait_ld();
            reg_fence<Epi::CH>(v);
            e.chunk(row, nb * BN + part * HALF + c, v);
          }
          e.tile_end(row, nb, part);
        } else if (ok) {
          const uint32_t base = tmem + lane_base + static_cast<uint32_t>(buf * BN + part * HALF);
          // two register buffers: chunk i + 1 is loaded from TMEM while chunk i is processed (a rolled loop over
          // chunk pairs, so only two copies of the chunk code exist)
          constexpr int NCH = HALF / Epi::CH;
          static_assert(NCH % 2 == 0, "pipelined epilogues need an even number of chunks per half tile");
          const int col = nb * BN + part * HALF;
          float va[Epi::CH], vb[Epi::CH];
          load_chunk<Epi::CH>(base, va);
          tc_wait_ld();
          reg_fence<Epi::CH>(va);
#pragma unroll 1
          for (int i = 0; i < NCH; i += 2) {
            load_chunk<Epi::CH>(base + (i + 1) * Epi::CH, vb);
            e.chunk(row, col + i * Epi::CH, va);
            tc_wait_ld();
            reg_fence<Epi::CH>(vb);
            if (i + 2 < NCH) load_chunk<Epi::CH>(base + (i + 2) * Epi::CH, va);
            e.chunk(row, col + (i + 1) * Epi::CH, vb);
            if (i + 2 < NCH) {
              tc_wait_ld();
              reg_fence<Epi::CH>(va);
            }
          }
          e.tile_end(row, nb, part);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acce[buf]);
        if (!ok) break;
      }
      if (ok) e.row_end(row, part);
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

}  // namespace noise
