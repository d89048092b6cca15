// The identity phase's batched GEMMs (reference train/speedrun/id_kernels.py, called from speedrun/run.py:3818-3913
// identity_grad) on sm_100a tensor cores:
//   hidden_credits_fused  out[l] = bf16(slope(U_l, step_l) * float(bf16(credb[l] @ w_out_t[l])))   (:19-84)
//   square_credit_grads   out[j L + l] = bf16(n1s[l]^T @ B_jl), B_jl[tok, w 64 + d] = got2[w, l, j, tok, d] (:87-133)
//   at_b_layers           out[l] = bf16(A_l^T @ B_l)                                                 (:136-170)
// with slope(u, s) = (max(u + s, 0)^2 - max(u - s, 0)^2) / (2 s), the central difference of relu^2.
//
// One persistent, warp-specialised kernel for all three (320 threads, one CTA per SM):
//   warp 0      one lane: TMA loads into a 4-deep ring of (A, B) k-blocks of 64. An operand stored K-contiguous (the
//               hidden credits' A) is one 128 x 64 box with 128-byte swizzle; an operand stored MN-contiguous (every
//               A^T and every B here) is loaded as 64 x 64 boxes, one per 64-wide MN chunk, so a chunk may come from a
//               different tensor (square_credit_grads' B: one got2 plane per world rank w);
//   warp 1      one lane: tcgen05.mma M = 128, N = BN, K = 16 into a double-buffered TMEM accumulator (2 x BN columns);
//   warps 2..9  epilogue: warp w reads TMEM lane quarter w % 4 (one output row per thread) and column half
//               (w - 2) / 4 of the tile, applies the op's rounding (and the slope), stores bf16.
// Work items are (batch, row tile, column tile), column tiles fastest, so concurrently running CTAs share the A tile
// and the batch's B in L2. Every wait is bounded (ptx.cuh): on a timeout the status word is set and the kernel
// unwinds.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "noise_b200.h"
#include "ptx.cuh"

namespace noise {
namespace idk {

constexpr int BM = 128, BK = 64, STAGES = 4, EPI_WARPS = 8, THREADS = 64 + 32 * EPI_WARPS;
constexpr int SUB = 64 * 128;         // one 64 x 64 bf16 sub-tile (128-byte rows)
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int MAX_MAPS = 8;

enum Op { HIDDEN = 0, AT_B = 1, SQUARE = 2 };

template <int BN>
struct Layout {
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int BAR_OFFSET = STAGES * STAGE_BYTES;
  static constexpr int SMEM = BAR_OFFSET + 256 + 1024;  // barriers + TMEM holder, 1024 alignment slack
  static constexpr int TMEM_COLS = 2 * BN;
};

struct Maps {
  CUtensorMap a[MAX_MAPS];  // per A matrix (layer)
  CUtensorMap b[MAX_MAPS];  // per B matrix (layer); SQUARE: b[0] spans got2 as [W L 3 M, 64]
};

struct Args {
  int batches, m_tiles, n_tiles, k_blocks;
  int layers;                 // SQUARE: batch = j layers + l
  int planes_rows;            // SQUARE: tokens per got2 plane (M)
  __nv_bfloat16* out;         // [batches, m_tiles BM, ldo]
  int64_t out_batch;          // elements between batches
  int ldo;
  const __nv_bfloat16* u[MAX_MAPS];  // HIDDEN: U_l [M, N] row-major
  const float* step;                 // HIDDEN: [L, M]
  int* status;
};

// fp32, no contraction: the reference's (up * up - down * down) / (2 * step), the divide as a multiply by the row's
// correctly rounded 1 / (2 step) (within an fp32 ulp of the quotient; the result is then rounded to bf16)
__device__ __forceinline__ float slope_of(float u, float s, float inv2s) {
  const float up = fmaxf(__fadd_rn(u, s), 0.f), down = fmaxf(__fsub_rn(u, s), 0.f);
  return __fmul_rn(__fsub_rn(__fmul_rn(up, up), __fmul_rn(down, down)), inv2s);
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&p);
}

template <int OP, int BN>
__global__ void __launch_bounds__(THREADS, 1) idgemm_kernel(const __grid_constant__ Maps maps, const __grid_constant__ Args p) {
  using L = Layout<BN>;
  constexpr bool A_MN = OP != HIDDEN;  // A stored MN-contiguous (A^T given)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFFSET);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;
  uint64_t* acce = accf + 2;
  uint64_t* drain = acce + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_batch = p.m_tiles * p.n_tiles;
  const int items = p.batches * per_batch;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], EPI_WARPS);  // one arrival per epilogue warp (after its __syncwarp)
    }
    mbar_init(drain, 1);
    fence_barrier_init();
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
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < items && ok; w += gridDim.x) {
        const int batch = w / per_batch, rem = w - batch * per_batch;
        const int mb = rem / p.n_tiles, nb = rem - mb * p.n_tiles;
        const int la = OP == SQUARE ? batch % p.layers : batch;  // A matrix
        const CUtensorMap* ma = &maps.a[la];
        const CUtensorMap* mbm = &maps.b[OP == SQUARE ? 0 : batch];
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, p.status)) {
            ok = false;
            break;
          }
          uint8_t* a = smem + stage * L::STAGE_BYTES;
          uint8_t* b = a + A_BYTES;
          mbar_arrive_expect_tx(&full[stage], L::STAGE_BYTES);
          if constexpr (A_MN) {
            tma_load_2d(a, ma, &full[stage], mb * BM, kb * BK);
            tma_load_2d(a + SUB, ma, &full[stage], mb * BM + 64, kb * BK);
          } else {
            tma_load_2d(a, ma, &full[stage], kb * BK, mb * BM);
          }
#pragma unroll
          for (int c = 0; c < BN / 64; ++c) {
            if constexpr (OP == SQUARE) {  // chunk c of columns nb BN + 64 c is got2[w, l, j] with w its head
              const int wr = (nb * BN) / 64 + c, l = batch % p.layers, j = batch / p.layers;
              const int plane = (wr * p.layers + l) * 3 + j;
              tma_load_2d(b + c * SUB, mbm, &full[stage], 0, plane * p.planes_rows + kb * BK);
            } else {
              tma_load_2d(b + c * SUB, mbm, &full[stage], nb * BN + 64 * c, kb * BK);
            }
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      for (int i = 0; i < STAGES && i < issued; ++i) {  // drain: every issued load lands before the CTA exits
        if (--stage < 0) {
          stage = STAGES - 1;
          phase ^= 1u;
        }
        mbar_wait(&full[stage], phase, p.status);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(BM, BN, A_MN, true);
      int stage = 0, t = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int w = blockIdx.x; w < items && ok; w += gridDim.x, ++t) {
        const int buf = t & 1;
        if (!mbar_wait(&acce[buf], (static_cast<uint32_t>(t >> 1) & 1u) ^ 1u, p.status)) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(buf * BN);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + stage * L::STAGE_BYTES), b = a + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // MN-major: 16 K rows = 2048 bytes further, 64-wide MN chunks SUB apart (LBO); K-major: +32 bytes
            const uint64_t ad = A_MN ? sdesc_mnmajor_sw128(a + k * 2048, SUB) : sdesc_kmajor_sw128(a) + 2u * k;
            const uint64_t bd = sdesc_mnmajor_sw128(b + k * 2048, SUB);
            tc_mma(d, ad, bd, idesc, (kb | k) != 0);
          }
          tc_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (ok) tc_commit(&accf[buf]);
      }
      tc_commit(drain);
      mbar_wait(drain, 0, p.status);
    }
  } else {
    const int quarter = warp & 3, part = (warp - 2) >> 2;
    const int r_in = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    constexpr int HALF = BN / 2;
    int t = 0;
    for (int w = blockIdx.x; w < items; w += gridDim.x, ++t) {
      const int batch = w / per_batch, rem = w - batch * per_batch;
      const int mb = rem / p.n_tiles, nb = rem - mb * p.n_tiles;
      const int buf = t & 1;
      if (!mbar_wait(&accf[buf], static_cast<uint32_t>(t >> 1) & 1u, p.status)) break;
      tc_fence_after();
      const int row = mb * BM + r_in;
      const int col0 = nb * BN + part * HALF;
      __nv_bfloat16* orow = p.out + batch * p.out_batch + static_cast<int64_t>(row) * p.ldo + col0;
      float s = 0.f, inv2s = 0.f;
      const __nv_bfloat16* urow = nullptr;
      if constexpr (OP == HIDDEN) {
        s = p.step[static_cast<int64_t>(batch) * p.m_tiles * BM + row];
        inv2s = 1.f / __fmul_rn(2.f, s);  // once per row: the per-element divide becomes a multiply
        urow = p.u[batch] + static_cast<int64_t>(row) * p.ldo + col0;
      }
      const uint32_t base = tmem + lane_base + static_cast<uint32_t>(buf * BN + part * HALF);
      uint32_t uw[16];
      auto load_u = [&](int c) {  // the chunk's 32 pre-activations, issued ahead of their use
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 q = *reinterpret_cast<const uint4*>(urow + c + 8 * i);
          uw[4 * i] = q.x, uw[4 * i + 1] = q.y, uw[4 * i + 2] = q.z, uw[4 * i + 3] = q.w;
        }
      };
      if constexpr (OP == HIDDEN) load_u(0);
#pragma unroll 1
      for (int c = 0; c < HALF; c += 32) {
        float v[32];
        tmem_ld32(base + c, v);
        tc_wait_ld();
        reg_fence<32>(v);
        if constexpr (OP == HIDDEN) {
          float u[32];
#pragma unroll
          for (int i = 0; i < 32; ++i)  // bf16 -> fp32 is the 16 bits shifted up
            u[i] = __uint_as_float((i & 1) ? (uw[i >> 1] & 0xffff0000u) : (uw[i >> 1] << 16));
          if (c + 32 < HALF) load_u(c + 32);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float read = __bfloat162float(__float2bfloat16_rn(v[i]));
            v[i] = __fmul_rn(slope_of(u[i], s, inv2s), read);
          }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
          *reinterpret_cast<uint4*>(orow + c + 8 * i) =
              make_uint4(pack2(v[8 * i], v[8 * i + 1]), pack2(v[8 * i + 2], v[8 * i + 3]),
                         pack2(v[8 * i + 4], v[8 * i + 5]), pack2(v[8 * i + 6], v[8 * i + 7]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[buf]);
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

}  // namespace idk
}  // namespace noise

using namespace noise::idk;

namespace {

PFN_cuTensorMapEncodeTiled_v12000 idk_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// bf16 row-major [rows, cols] with a 128-byte swizzled box of box_rows x 64 columns
int idk_map(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows) {
  auto fn = idk_encode();
  if (!fn) return NOISE_ERR_CUDA;
  if (!base) return NOISE_ERR_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (cols * 2) % 16) return NOISE_ERR_ALIGN;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t el[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, el,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NOISE_OK : NOISE_ERR_CUDA;
}

int idk_sms() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return n;
}

template <int OP, int BN>
int idk_launch(const Maps& maps, Args a, cudaStream_t s) {
  using L = Layout<BN>;
  const int sms = idk_sms();
  if (sms < 1) return NOISE_ERR_CUDA;
  if (cudaMemsetAsync(a.status, 0, sizeof(int), s) != cudaSuccess) return NOISE_ERR_CUDA;
  if (cudaFuncSetAttribute(idgemm_kernel<OP, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM))
    return NOISE_ERR_CUDA;
  const int items = a.batches * a.m_tiles * a.n_tiles;
  idgemm_kernel<OP, BN><<<std::min(items, sms), THREADS, L::SMEM, s>>>(maps, a);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

// BN = 256 where the output width allows it (fewer B re-reads per A tile) and the grid still fills the SMs, else 128
template <int OP>
int idk_run(const Maps& maps, Args a, int n, cudaStream_t s) {
  if (n % 256 == 0 && a.batches * a.m_tiles * (n / 256) >= idk_sms()) {
    a.n_tiles = n / 256;
    return idk_launch<OP, 256>(maps, a, s);
  }
  a.n_tiles = n / 128;
  return idk_launch<OP, 128>(maps, a, s);
}

bool a16p(const void* p) { return p && (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

extern "C" {

int noise_hidden_credits(const void* const* us, const float* steps, const void* credb, const void* w_out_t,
                         int layers, int m, int n, int k, void* out, void* workspace, size_t workspace_bytes,
                         void* stream) {
  if (!us || !steps || !credb || !w_out_t || !out) return NOISE_ERR_ARGUMENT;
  if (!workspace || workspace_bytes < NOISE_STATUS_BYTES) return NOISE_ERR_WORKSPACE;
  if (layers < 1 || layers > MAX_MAPS || m < 1 || n < 1 || k < 1 || m % BM || n % 128 || k % BK)
    return NOISE_ERR_SHAPE;
  if (!a16p(out) || !a16p(credb) || !a16p(w_out_t)) return NOISE_ERR_ALIGN;
  Maps maps;
  Args a{};
  for (int l = 0; l < layers; ++l) {
    if (!a16p(us[l])) return us[l] ? NOISE_ERR_ALIGN : NOISE_ERR_ARGUMENT;
    const auto* A = static_cast<const __nv_bfloat16*>(credb) + static_cast<int64_t>(l) * m * k;
    const auto* B = static_cast<const __nv_bfloat16*>(w_out_t) + static_cast<int64_t>(l) * k * n;
    int rc;
    if ((rc = idk_map(&maps.a[l], A, k, m, BM)) || (rc = idk_map(&maps.b[l], B, n, k, 64))) return rc;
    a.u[l] = static_cast<const __nv_bfloat16*>(us[l]);
  }
  a.batches = layers;
  a.m_tiles = m / BM;
  a.k_blocks = k / BK;
  a.layers = layers;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.out_batch = static_cast<int64_t>(m) * n;
  a.ldo = n;
  a.step = steps;
  a.status = static_cast<int*>(workspace);
  return idk_run<HIDDEN>(maps, a, n, static_cast<cudaStream_t>(stream));
}

int noise_at_b_layers(const void* const* as, const void* const* bs, int layers, int k, int p, int q, void* out,
                      void* workspace, size_t workspace_bytes, void* stream) {
  if (!as || !bs || !out) return NOISE_ERR_ARGUMENT;
  if (!workspace || workspace_bytes < NOISE_STATUS_BYTES) return NOISE_ERR_WORKSPACE;
  if (layers < 1 || layers > MAX_MAPS || k < 1 || p < 1 || q < 1 || k % BK || p % BM || q % 128)
    return NOISE_ERR_SHAPE;
  if (!a16p(out)) return NOISE_ERR_ALIGN;
  Maps maps;
  Args a{};
  for (int l = 0; l < layers; ++l) {
    int rc;
    if ((rc = idk_map(&maps.a[l], as[l], p, k, 64)) || (rc = idk_map(&maps.b[l], bs[l], q, k, 64))) return rc;
  }
  a.batches = layers;
  a.m_tiles = p / BM;
  a.k_blocks = k / BK;
  a.layers = layers;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.out_batch = static_cast<int64_t>(p) * q;
  a.ldo = q;
  a.status = static_cast<int*>(workspace);
  return idk_run<AT_B>(maps, a, q, static_cast<cudaStream_t>(stream));
}

int noise_square_credit_grads(const void* const* n1s, const void* got2, int world, int layers, int m, int d,
                              void* out, void* workspace, size_t workspace_bytes, void* stream) {
  if (!n1s || !got2 || !out) return NOISE_ERR_ARGUMENT;
  if (!workspace || workspace_bytes < NOISE_STATUS_BYTES) return NOISE_ERR_WORKSPACE;
  if (layers < 1 || layers > MAX_MAPS || world < 1 || m < 1 || m % BK || d % BM || world * 64 != d)
    return NOISE_ERR_SHAPE;
  if (!a16p(out)) return NOISE_ERR_ALIGN;
  Maps maps;
  Args a{};
  int rc;
  for (int l = 0; l < layers; ++l)
    if ((rc = idk_map(&maps.a[l], n1s[l], d, m, 64))) return rc;
  if ((rc = idk_map(&maps.b[0], got2, 64, static_cast<uint64_t>(world) * layers * 3 * m, 64))) return rc;
  a.batches = 3 * layers;
  a.m_tiles = d / BM;
  a.k_blocks = m / BK;
  a.layers = layers;
  a.planes_rows = m;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.out_batch = static_cast<int64_t>(d) * d;
  a.ldo = d;
  a.status = static_cast<int*>(workspace);
  return idk_run<SQUARE>(maps, a, d, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
