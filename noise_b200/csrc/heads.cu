// The identity phase's head-sharding kernels (reference train/speedrun/run.py:3694-3804) on sm_100a.
//
// The identity phase moves every layer's attention pieces from token-sharded to head-sharded over an all_to_all:
//   pack_heads   (run.py:3698-3731)  per head h, layer l, token: q, k, v, attention output o and target pieces (64
//                each, bf16) and the lse's fp32 bits, one 322-element bf16 row of the (H, L, n, 322) send buffer;
//   head_prep    (run.py:3734-3796)  from the received (W, L, N, 322) buffer: RoPE + RMS-normed queries and keys
//                (bf16 and fp32), their raw square norms and finite-difference steps, the keys' pair features,
//                values and hubs, lse and hub . o, reordered to (layer, source rank, token) rows;
//   id_head_scores (run.py:3799-3803) head_prep, then the query- and key-moment credits (credit.cu) reading the raw
//                coordinates in place from the received buffer and writing the bf16 (W, L, 3, N, 64) return buffer.
// All of it is memory-bound byte movement plus a few flops per element: one warp per 322-element row, every global
// access a 128-byte warp-contiguous segment.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "exchange.cuh"
#include "noise_b200.h"

namespace noise {
namespace heads {

constexpr int H = NOISE_N_HEAD;     // 8
constexpr int HD = NOISE_HEAD_DIM;  // 64
constexpr int PACK = NOISE_PACK;    // 5 * 64 + 2
constexpr int WARPS = 8;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

struct PackArgs {
  noise_head_pieces_t layer[NOISE_MAX_PACK_LAYERS];
  int L, n, T;
  uint32_t* out;  // (H, L, n, PACK) bf16 as 32-bit words (a row is PACK / 2 words)
};

// grid (ceil(n / 8), H, L): warp w of block x copies token x * 8 + w of head blockIdx.y, layer blockIdx.z.
// Row (h, l, tok) of the pack: 161 32-bit words (5 pieces x 32 words, then the lse's fp32 bits), one warp.
__device__ __forceinline__ void pack_row(const PackArgs& a, int h, int l, int tok, uint32_t* dst, int lane) {
  const noise_head_pieces_t& P = a.layer[l];
  const void* src[5] = {P.q, P.k, P.v, P.o, P.target};
  const int64_t stride[5] = {P.q_stride, P.k_stride, P.v_stride, P.o_stride, P.target_stride};
#pragma unroll
  for (int piece = 0; piece < 5; ++piece) {
    const uint32_t* s = reinterpret_cast<const uint32_t*>(static_cast<const __nv_bfloat16*>(src[piece]) +
                                                          tok * stride[piece] + h * HD);
    dst[piece * 32 + lane] = s[lane];
  }
  if (lane == 0) {
    const int64_t li = (static_cast<int64_t>(tok / a.T) * H + h) * a.T + tok % a.T;  // lse (rows, H, T)
    dst[5 * 32] = __float_as_uint(P.lse[li]);
  }
}

__global__ void __launch_bounds__(256) pack_heads_kernel(const __grid_constant__ PackArgs a) {
  const int lane = threadIdx.x & 31;
  const int tok = blockIdx.x * WARPS + (threadIdx.x >> 5);
  if (tok >= a.n) return;
  const int h = blockIdx.y, l = blockIdx.z;
  pack_row(a, h, l, tok, a.out + (static_cast<int64_t>(h * a.L + l) * a.n + tok) * (PACK / 2), lane);
}

// The pack written straight into the destination ranks' exchange buffers, then the send's epoch flag
// (exchange.cuh). A warp packs 4 consecutive tokens of one (head, layer) into shared memory (2,576 bytes: 161
// 16-byte words, since 4 rows of 644 bytes start 16-byte aligned) and stores them with 16-byte stores, so every
// NVLink write is a 512-byte warp-contiguous segment. Grid-stride over the (h, l, 4-token) groups.
constexpr int GROUP = 4;
constexpr int GROUP_WORDS = GROUP * PACK / 2;  // 644 32-bit words = 161 x 16 bytes

__global__ void __launch_bounds__(256) pack_heads_peer_kernel(const __grid_constant__ PackArgs a,
                                                              const __grid_constant__ xch::Peers peers,
                                                              int64_t dst_offset, int slot, uint32_t epoch) {
  __shared__ __align__(16) uint32_t stage[WARPS][GROUP_WORDS];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int hp = H / peers.world;  // heads per destination rank
  const int groups_per_hl = a.n / GROUP;
  const int64_t groups = static_cast<int64_t>(H) * a.L * groups_per_hl;
  uint32_t* st = stage[warp];
  for (int64_t gi = static_cast<int64_t>(blockIdx.x) * WARPS + warp; gi < groups;
       gi += static_cast<int64_t>(gridDim.x) * WARPS) {
    // the head varies fastest and starts at this rank's own heads: the warps of a block, and the ranks at any moment,
    // write to different destinations, so no destination's NVLink ingress is shared by every sender at once
    const int h = static_cast<int>((gi % H + static_cast<int64_t>(peers.rank) * hp) % H);
    const int64_t rest = gi / H;
    const int l = static_cast<int>(rest % a.L);
    const int tok0 = static_cast<int>(rest / a.L) * GROUP;
#pragma unroll
    for (int r = 0; r < GROUP; ++r) pack_row(a, h, l, tok0 + r, st + r * (PACK / 2), lane);
    __syncwarp();
    const int p = h / hp;
    const int64_t drow = (static_cast<int64_t>(peers.rank * hp + h % hp) * a.L + l) * a.n + tok0;
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint32_t*>(peers.base[p] + dst_offset) + drow * (PACK / 2));
    const uint4* src = reinterpret_cast<const uint4*>(st);
    for (int i = lane; i < GROUP_WORDS / 4; i += 32) dst[i] = src[i];
    __syncwarp();
  }
  xch::send_done(peers, slot, epoch);
}

struct PrepArgs {
  const __nv_bfloat16* got;  // (W, L, N, PACK)
  const float *cosb, *sinb;  // [T, 32] fp32
  int W, L, N, T;
  float sigma, eps;
  noise_head_prep_t o;
};

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&p);
}

// One warp per received row, in the buffer's order (source rank, layer, token): lane j owns rotary pair j.
__global__ void __launch_bounds__(256) head_prep_kernel(const __grid_constant__ PrepArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t src = static_cast<int64_t>(blockIdx.x) * WARPS + (threadIdx.x >> 5);
  if (src >= static_cast<int64_t>(a.W) * a.L * a.N) return;
  const int i = static_cast<int>(src % a.N);
  const int wl = static_cast<int>(src / a.N);
  const int layer = wl % a.L, w = wl / a.L;
  const int64_t dst = (static_cast<int64_t>(layer) * a.W + w) * a.N + i;
  const int pos = i % a.T;
  const __nv_bfloat16* row = a.got + src * PACK;
  const float c = a.cosb[pos * 32 + lane], s = a.sinb[pos * 32 + lane];

#pragma unroll
  for (int j = 0; j < 2; ++j) {  // j = 0: queries, 1: keys
    const float x1 = __bfloat162float(row[j * HD + lane]), x2 = __bfloat162float(row[j * HD + 32 + lane]);
    float r1 = x1 * c + x2 * s;
    float r2 = x1 * -s + x2 * c;
    const float inv = rsqrtf(warp_sum(r1 * r1 + r2 * r2) / HD + a.eps);
    const float sq = warp_sum(x1 * x1 + x2 * x2);
    r1 *= inv;
    r2 *= inv;
    __nv_bfloat16* o16 = static_cast<__nv_bfloat16*>(j ? a.o.k16 : a.o.q16) + dst * HD;
    o16[lane] = __float2bfloat16_rn(r1);
    o16[lane + 32] = __float2bfloat16_rn(r2);
    float* o32 = j ? a.o.k32 : a.o.q32;
    if (o32) {
      o32[dst * HD + lane] = r1;
      o32[dst * HD + 32 + lane] = r2;
    }
    if (j == 1 && a.o.f2) {  // the keys' pair features (moment_kernels._pair_features), x = r1 / 8, y = r2 / 8
      const float x = r1 * 0.125f, y = r2 * 0.125f;
      reinterpret_cast<uint32_t*>(static_cast<__nv_bfloat16*>(a.o.f2) + dst * HD)[lane] = pack2(x, y);
      static_cast<__nv_bfloat16*>(a.o.xy)[dst * (HD / 2) + lane] = __float2bfloat16_rn(x * y);
      reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(a.o.f4) + dst * 2 * HD)[lane] =
          make_uint2(pack2(x, x * x), pack2(y, y * y));
    }
    if (lane == 0) {
      (j ? a.o.sq_k : a.o.sq_q)[dst] = sq;
      (j ? a.o.steps_k : a.o.steps_q)[dst] = a.sigma * fmaxf(sqrtf(sq / HD), 1e-6f);
    }
  }
  // values and hubs copied; hub_out = hub . o in fp32; lse from its fp32 bits
  const uint32_t* w32 = reinterpret_cast<const uint32_t*>(row);
  const uint32_t vw = w32[64 + lane], ow = w32[96 + lane], hw = w32[128 + lane];
  reinterpret_cast<uint32_t*>(static_cast<__nv_bfloat16*>(a.o.v16) + dst * HD)[lane] = vw;
  reinterpret_cast<uint32_t*>(static_cast<__nv_bfloat16*>(a.o.hub16) + dst * HD)[lane] = hw;
  const float2 of = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ow));
  const float2 hf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&hw));
  const float ho = warp_sum(hf.x * of.x + hf.y * of.y);
  if (lane == 0) {
    a.o.hub_out[dst] = ho;
    a.o.lse[dst] = __uint_as_float(w32[PACK / 2 - 1]);
  }
}

static bool a4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3) == 0; }
static bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
static size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

static int prep_checks(const void* got, int world, int layers, int n, const float* cos, const float* sin, int tokens) {
  if (!got || !cos || !sin) return NOISE_ERR_ARGUMENT;
  if (world < 1 || layers < 1 || n < 32 || n % 32 || tokens < 1 || (static_cast<int64_t>(world) * n) % tokens)
    return NOISE_ERR_SHAPE;
  if (!a4(got)) return NOISE_ERR_ALIGN;
  return NOISE_OK;
}

static int launch_prep(const void* got, int world, int layers, int n, const float* cos, const float* sin, int tokens,
                       float sigma, float eps, const noise_head_prep_t& o, cudaStream_t s) {
  PrepArgs a{};
  a.got = static_cast<const __nv_bfloat16*>(got);
  a.cosb = cos;
  a.sinb = sin;
  a.W = world;
  a.L = layers;
  a.N = n;
  a.T = tokens;
  a.sigma = sigma;
  a.eps = eps;
  a.o = o;
  const int64_t total = static_cast<int64_t>(world) * layers * n;
  head_prep_kernel<<<static_cast<unsigned>((total + WARPS - 1) / WARPS), 256, 0, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

// Scratch of noise_id_head_scores: head_prep's outputs for `total` received rows (no pair features: the moment
// kernels derive them from the fp32 keys).
struct IdScratch {
  noise_head_prep_t o;
  size_t bytes;
};

static IdScratch carve(void* ws, int64_t total) {
  IdScratch w{};
  size_t off = 0;
  auto take = [&](size_t nb) {
    void* p = ws ? static_cast<uint8_t*>(ws) + off : nullptr;
    off += align256(nb);
    return p;
  };
  w.o.q16 = take(total * HD * 2);
  w.o.k16 = take(total * HD * 2);
  w.o.v16 = take(total * HD * 2);
  w.o.hub16 = take(total * HD * 2);
  w.o.q32 = static_cast<float*>(take(total * HD * 4));
  w.o.k32 = static_cast<float*>(take(total * HD * 4));
  float** scal[6] = {&w.o.lse, &w.o.hub_out, &w.o.sq_q, &w.o.sq_k, &w.o.steps_q, &w.o.steps_k};
  for (float** p : scal) *p = static_cast<float*>(take(total * 4));
  w.bytes = off;
  return w;
}

}  // namespace heads
}  // namespace noise

using namespace noise::heads;

static int pack_args(const noise_head_pieces_t* layers, int n_layers, int tokens, int seq_len, PackArgs* a) {
  if (!layers) return NOISE_ERR_ARGUMENT;
  if (n_layers < 1 || n_layers > NOISE_MAX_PACK_LAYERS || tokens < 16 || tokens % 16 || seq_len < 1 ||
      tokens % seq_len)
    return NOISE_ERR_SHAPE;
  for (int l = 0; l < n_layers; ++l) {
    const noise_head_pieces_t& P = layers[l];
    if (!P.q || !P.k || !P.v || !P.o || !P.target || !P.lse) return NOISE_ERR_ARGUMENT;
    const void* ptr[5] = {P.q, P.k, P.v, P.o, P.target};
    const int64_t st[5] = {P.q_stride, P.k_stride, P.v_stride, P.o_stride, P.target_stride};
    for (int k = 0; k < 5; ++k) {
      if (st[k] < H * HD) return NOISE_ERR_SHAPE;
      if (!a4(ptr[k]) || (st[k] & 1)) return NOISE_ERR_ALIGN;
    }
    a->layer[l] = P;
  }
  a->L = n_layers;
  a->n = tokens;
  a->T = seq_len;
  return NOISE_OK;
}

extern "C" {

int noise_pack_heads(const noise_head_pieces_t* layers, int n_layers, int tokens, int seq_len, void* out, void* stream) {
  if (!layers || !out) return NOISE_ERR_ARGUMENT;
  PackArgs a{};
  int rc = pack_args(layers, n_layers, tokens, seq_len, &a);
  if (rc) return rc;
  if (!a4(out)) return NOISE_ERR_ALIGN;
  a.out = static_cast<uint32_t*>(out);
  dim3 grid((tokens + WARPS - 1) / WARPS, H, n_layers);
  pack_heads_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_pack_heads_peer(const noise_head_pieces_t* layers, int n_layers, int tokens, int seq_len,
                          const noise_peers_t* peers, size_t dst_offset, int slot, uint32_t epoch, void* stream) {
  PackArgs a{};
  int rc = pack_args(layers, n_layers, tokens, seq_len, &a);
  if (rc) return rc;
  noise::xch::Peers P;
  if ((rc = noise::xch::peers_check(peers, &P))) return rc;
  if (H % P.world || slot < 0 || slot > 1) return NOISE_ERR_SHAPE;
  if (dst_offset < NOISE_EXCHANGE_HEAD_BYTES || dst_offset % 16) return NOISE_ERR_ALIGN;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev))
    return NOISE_ERR_CUDA;
  const int64_t groups = static_cast<int64_t>(H) * n_layers * (tokens / GROUP);
  const int blocks = static_cast<int>(std::min<int64_t>((groups + WARPS - 1) / WARPS, static_cast<int64_t>(sms) * 8));
  pack_heads_peer_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      a, P, static_cast<int64_t>(dst_offset), slot, epoch);
  return cudaGetLastError() == cudaSuccess ? NOISE_OK : NOISE_ERR_CUDA;
}

int noise_head_prep(const void* got, int world, int layers, int n, const float* cos, const float* sin, int tokens,
                    float sigma, float eps, const noise_head_prep_t* out, void* stream) {
  int rc = prep_checks(got, world, layers, n, cos, sin, tokens);
  if (rc) return rc;
  if (!out || !out->q16 || !out->k16 || !out->v16 || !out->hub16 || !out->q32 || !out->lse || !out->hub_out ||
      !out->sq_q || !out->sq_k || !out->steps_q || !out->steps_k)
    return NOISE_ERR_ARGUMENT;
  if ((out->f2 || out->f4 || out->xy) && !(out->f2 && out->f4 && out->xy)) return NOISE_ERR_ARGUMENT;
  const void* vec[7] = {out->q16, out->k16, out->v16, out->hub16, out->f2, out->f4, out->xy};
  for (const void* p : vec)
    if (p && !a16(p)) return NOISE_ERR_ALIGN;
  if (!a16(out->q32) || (out->k32 && !a16(out->k32))) return NOISE_ERR_ALIGN;
  return launch_prep(got, world, layers, n, cos, sin, tokens, sigma, eps, *out, static_cast<cudaStream_t>(stream));
}

// The moment kernels' own workspace (a status word and the pair features; the query and key passes run one after the
// other and share it) sits at the head of id_head_scores' workspace, head_prep's outputs after it.
static size_t moment_ws_bytes(int64_t total) { return 256 + 3 * static_cast<size_t>(total) * HD * 2; }

size_t noise_id_head_scores_workspace_bytes(int world, int layers, int n) {
  if (world < 1 || layers < 1 || n < 1) return 0;
  const int64_t total = static_cast<int64_t>(world) * layers * n;
  return moment_ws_bytes(total) + carve(nullptr, total).bytes;
}

int noise_id_head_scores(const void* got, int world, int layers, int n, const float* cos, const float* sin, int tokens,
                         float sigma, float eps, void* back, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = prep_checks(got, world, layers, n, cos, sin, tokens);
  if (rc) return rc;
  if (!back) return NOISE_ERR_ARGUMENT;
  if (tokens < 64 || tokens % 64) return NOISE_ERR_SHAPE;
  const int64_t total = static_cast<int64_t>(world) * layers * n;
  const size_t mws = moment_ws_bytes(total);
  const IdScratch w = carve(workspace ? static_cast<uint8_t*>(workspace) + mws : nullptr, total);
  if (!workspace || workspace_bytes < mws + w.bytes) return NOISE_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return NOISE_ERR_ALIGN;
  if (!a4(back)) return NOISE_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((rc = launch_prep(got, world, layers, n, cos, sin, tokens, sigma, eps, w.o, s))) return rc;

  const int b = static_cast<int>(static_cast<int64_t>(world) * n / tokens);  // rows per layer
  const int rows = layers * b;
  // got (W, L, N, PACK): the raw queries at element 0 of a row, the raw keys at element 64
  noise_rows_t raw{};
  raw.data = const_cast<void*>(got);
  raw.heads = 1;
  raw.block_rows = b;
  raw.layer_stride = static_cast<int64_t>(n) * PACK;
  raw.gpu_stride = static_cast<int64_t>(layers) * n * PACK;
  raw.token_stride = PACK;
  raw.per_gpu = n;
  // back (W, L, 3, N, 64): slot 0 query credits, 1 key credits, 2 value sums
  noise_rows_t out{};
  out.data = back;
  out.heads = 1;
  out.block_rows = b;
  out.layer_stride = 3 * static_cast<int64_t>(n) * HD;
  out.gpu_stride = static_cast<int64_t>(layers) * 3 * n * HD;
  out.token_stride = HD;
  out.per_gpu = n;
  const noise_head_prep_t& o = w.o;
  // T % 128 == 0: the tcgen05 moment kernels (their status word at the workspace's head); else the warp-MMA ones
  rc = noise_moment_query_scores_ws(o.q16, o.k16, o.v16, o.hub16, &raw, NOISE_DTYPE_BF16, o.sq_q, o.k32, cos, sin,
                                    o.lse, o.hub_out, o.steps_q, rows, tokens, tokens, &out, NOISE_DTYPE_BF16,
                                    workspace, mws, stream);
  if (rc) return rc;
  noise_rows_t rawk = raw, keys = out, vals = out;
  rawk.data = const_cast<__nv_bfloat16*>(static_cast<const __nv_bfloat16*>(got) + HD);
  keys.data = static_cast<__nv_bfloat16*>(back) + static_cast<int64_t>(n) * HD;
  vals.data = static_cast<__nv_bfloat16*>(back) + 2 * static_cast<int64_t>(n) * HD;
  return noise_moment_key_scores_ws(o.q16, o.k16, o.v16, o.hub16, &rawk, NOISE_DTYPE_BF16, o.sq_k, o.q32, cos, sin,
                                    o.lse, o.hub_out, o.steps_k, rows, tokens, &keys, &vals, NOISE_DTYPE_BF16, workspace,
                                    mws, stream);
}

}  // extern "C"
