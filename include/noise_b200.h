/* noise_b200 — C ABI of the B200 (sm_100a) hot path of Noise's forward-only training.
 *
 * Every pointer is a device pointer unless stated; every entry point enqueues work on `stream` (a cudaStream_t,
 * NULL = legacy default stream), performs no allocation, no host synchronisation and no host read of device data,
 * and returns NOISE_OK or a NOISE_ERR_* status for arguments it rejects before launching anything. Scratch memory
 * is caller-owned (`workspace`); its first NOISE_STATUS_BYTES hold a device status word that kernels set when a
 * bounded wait gives up (read it with noise_read_status after synchronising).
 *
 * The reference is pure Python (PyTorch + Triton/Gluon JIT kernels), so these functions replace Python entry points;
 * each declaration names the reference function it stands in for (path:line inside the reference project).
 */
#ifndef NOISE_B200_H
#define NOISE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NOISE_OK 0
#define NOISE_ERR_SHAPE 1       /* unsupported size (e.g. T not a multiple of 128, members < 1) */
#define NOISE_ERR_ALIGN 2       /* a pointer or stride violates the 16-byte TMA / vector alignment rule */
#define NOISE_ERR_WORKSPACE 3   /* workspace NULL or smaller than the *_workspace_bytes query */
#define NOISE_ERR_ARGUMENT 4    /* NULL required pointer, bad enum value, or a stream of another device */
#define NOISE_ERR_CUDA 5        /* a CUDA runtime/driver call failed (launch, tensor-map encode, attributes) */
#define NOISE_ERR_DEVICE 6      /* not an sm_100 device */
#define NOISE_ERR_TOO_LARGE 7   /* size beyond the static scratch of noise_population_loss_noalloc */

#define NOISE_STATUS_BYTES 256

/* Device status word values (noise_read_status). */
#define NOISE_DEVICE_OK 0
#define NOISE_DEVICE_TIMEOUT 1     /* a bounded mbarrier/flag wait gave up; outputs are invalid */

/* Model dimensions of the fixed GPT (reference utils/model.py:34-43). */
#define NOISE_N_LAYER 8
#define NOISE_N_HEAD 8
#define NOISE_HEAD_DIM 64
#define NOISE_N_EMBD 512
#define NOISE_VOCAB 4096
#define NOISE_N_PARAMS 60

/* Index of each parameter in the reference's GPT.named_parameters() order (60 tensors):
 * 0 resid_lambdas, 1 x0_lambdas, 2 transformer.wte.weight, then per block i the attn.c_q, attn.c_k, attn.c_v,
 * attn.c_proj, [attn.ve_gate on odd blocks], mlp.c_fc, mlp.c_proj weights, then 55 lm_head.weight and
 * 56..59 value_embeds.{1,3,5,7}.weight. noise_param_index() returns the index of block i's tensor `which`. */
enum noise_block_param {
  NOISE_P_CQ = 0, NOISE_P_CK = 1, NOISE_P_CV = 2, NOISE_P_CPROJ = 3, NOISE_P_VEGATE = 4, NOISE_P_CFC = 5,
  NOISE_P_MPROJ = 6, NOISE_P_VE = 7
};
int noise_param_index(int block, int which);
#define NOISE_PARAM_RESID 0
#define NOISE_PARAM_X0 1
#define NOISE_PARAM_WTE 2
#define NOISE_PARAM_HEAD 55

/* Rank-1 perturbation slices of one parameter for m members (reference eggroll.py:122-128). Member j's out-side
 * vector a_j starts at a + off[j] and its in-side vector b_j at b + off[j] (fp32). For the EGGROLL buffer,
 * a = buffer, b = buffer + out and off[j] = offsets[param][direction_j]; for materialised per-member tensors
 * a [m, out] / b [m, in], pass off = NULL and the strides instead: a_j = a + j * a_stride, b_j = b + j * b_stride.
 * 1-D parameters (the mixing scalars) use a only: eps_j = a + off[j] (or a + j * a_stride). */
typedef struct {
  const float* a;
  const float* b;
  const int64_t* off;
  int64_t a_stride;
  int64_t b_stride;
} noise_slice_t;

/* The model's weights as the CUDA path consumes them: matrices packed to bf16 once per update (noise_pack_bf16),
 * embeddings and mixing scalars fp32 (EGGROLL keeps them fp32, eggroll.py:50-52), RoPE tables bf16
 * [>= T, 32] (utils/model.py:177-183). */
typedef struct {
  const void* wqkv[NOISE_N_LAYER];   /* bf16 [1536, 512]: rows 0..511 c_q, 512..1023 c_k, 1024..1535 c_v */
  const void* wproj[NOISE_N_LAYER];  /* bf16 [512, 512] attn.c_proj */
  const void* wfc[NOISE_N_LAYER];    /* bf16 [2048, 512] mlp.c_fc */
  const void* wmproj[NOISE_N_LAYER]; /* bf16 [512, 2048] mlp.c_proj */
  const float* wgate[NOISE_N_LAYER]; /* fp32 [8, 32] attn.ve_gate on odd blocks, NULL on even blocks */
  const void* whead;                 /* bf16 [4096, 512] lm_head */
  const float* wte;                  /* fp32 [4096, 512] */
  const float* ve[NOISE_N_LAYER];    /* fp32 [4096, 512] value_embeds on odd blocks, NULL on even blocks */
  const float* resid_lambdas;        /* fp32 [8] */
  const float* x0_lambdas;           /* fp32 [8] */
  const void* cos;                   /* bf16 [>= T, 32] */
  const void* sin;                   /* bf16 [>= T, 32] */
} noise_gpt_t;

/* Loss reductions: MEAN / SUM over a member's (or, for noise_gpt_loss, all rows') tokens; NONE one loss per token.
 * A negative target (F.cross_entropy's ignore_index, -1 in GPT.forward) contributes 0 and is not counted. */
#define NOISE_REDUCTION_MEAN 0
#define NOISE_REDUCTION_SUM 1
#define NOISE_REDUCTION_NONE 2

/* ---------------------------------------------------------------------------------------------------------------
 * Credit-readout kernels (reference train/speedrun/moment_kernels.py). Rows are (layer, head, sequence) slices of
 * one attention map, [rows, T, 64]; receiver/query s and key t interact iff 0 <= s - t <= window. T % 64 == 0.
 * ------------------------------------------------------------------------------------------------------------- */
#define NOISE_DTYPE_F32 0
#define NOISE_DTYPE_BF16 1

/* A [rows, T, 64] view: element (row, t, c) at data + L * layer_stride + (row % heads) * 64 + t * token_stride + c,
 * L = row / heads, or layer_map[row / heads] when layer_map (int32, device) is set. The reference's stacked layout is
 * heads = 1, layer_stride = T * 64, token_stride = 64; its "by token" (layers, T, heads * 64) views
 * (moment_kernels.py:66-74) are heads = H, layer_stride = stride(0), token_stride = stride(1). 16-byte aligned.
 * With block_rows > 0 (heads = 1, no layer_map; moment-score raw inputs and outputs only) the blocked layout of the
 * identity phase's all_to_all buffers (moment_kernels.py:200-220, run.py:3799-3803): element (row, t, c) at
 * data + (row / block_rows) * layer_stride + (n / per_gpu) * gpu_stride + (n % per_gpu) * token_stride + c,
 * n = (row % block_rows) * T + t; e.g. a (W, L, N, C) buffer is block_rows = rows / L, layer_stride = stride(1),
 * gpu_stride = stride(0), token_stride = stride(2), per_gpu = N. Zero-initialised trailing fields mean "not blocked". */
typedef struct {
  void* data;
  int64_t layer_stride;
  int64_t token_stride;
  int heads;
  const int32_t* layer_map;
  int block_rows;
  int64_t per_gpu;
  int64_t gpu_stride;
} noise_rows_t;

/* lse[row, s] = logsumexp_t q_s.k_t / 8 and center[row, s] = sum_t p(s, t) (hub_s . v_t) over the window; q, k,
 * values, hub contiguous [rows, T, 64] of `dtype` (fp32 operands use tf32 dots, as the reference's PREC = 'tf32').
 * Replaces moment_kernels.implicit_key_context_edges (moment_kernels.py:137-194); window % 64 == 0. */
int noise_implicit_key_context(const void* q, const void* k, const void* values, const void* hub, int dtype, int rows,
                               int tokens, int window, float* lse, float* center, void* stream);

/* noise_implicit_key_context with a workspace of at least NOISE_STATUS_BYTES (the device status word): bf16 operands
 * with T % 128 == 0 run on tcgen05 (S = Q K^T and the scores H V^T into TMEM per pair of 128-query tiles, an online
 * softmax on 32-column chunks); anything else falls through to noise_implicit_key_context. Same results
 * (moment_kernels.py:137-194); window % 64 == 0. */
int noise_implicit_key_context_ws(const void* q, const void* k, const void* values, const void* hub, int dtype,
                                  int rows, int tokens, int window, float* lse, float* center, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* out[row, t] = sum_{s: 0 <= s - t <= window} exp(q_s.k_t / 8 - lse_s) source[row, s] (64 channels), the
 * probabilities rounded to bf16 and the fp32 source split into bf16 hi + lo, fp32 accumulation. Replaces
 * moment_kernels._value_pass / _value_credit_kernel (moment_kernels.py:612-717) and value_gluon.value_pass_gluon:
 * raw_value_credits(_by_token), terminal_value_credits(_into). q, k contiguous [rows, T, 64] of `dtype`. */
int noise_value_pass(const void* q, const void* k, int dtype, const float* lse, const noise_rows_t* source,
                     const noise_rows_t* out, int rows, int tokens, int window, void* stream);

/* Bytes of the caller's workspace for noise_value_pass_ws: a 256-byte status block, then the source's bf16 hi and lo
 * halves ([rows, T, 64] each). 0 for rows < 1 or tokens < 1. */
size_t noise_value_pass_workspace_bytes(int rows, int tokens);

/* noise_value_pass with a caller workspace (256-byte aligned, noise_value_pass_workspace_bytes large): bf16 q / k with
 * T % 128 == 0 run on tcgen05 (one pass splitting the source into bf16 hi / lo, then a persistent kernel computing
 * S = K Q^T into TMEM and O += P hi + P lo per pair of 128-key tiles); anything else falls through to
 * noise_value_pass. Same result definition as noise_value_pass (moment_kernels.py:612-717). The workspace's first
 * int32 is the device status after the call completes: 0, or 1 if a pipeline wait gave up (the output is then
 * incomplete). */
int noise_value_pass_ws(const void* q, const void* k, int dtype, const float* lse, const noise_rows_t* source,
                        const noise_rows_t* out, int rows, int tokens, int window, void* workspace,
                        size_t workspace_bytes, void* stream);

/* Key credits: per key t and raw key coordinate d, the degree-2 moment response of the receivers' softmax to a finite
 * step sigma * rms(k_raw[t]) of k_raw[t, d] through RoPE and the RMS norm (moment_kernels.py:467-607; key_gluon.py);
 * with value_out (data != NULL) also the raw value credit sum_s p hub_s. All inputs fp32 contiguous; cos / sin
 * [T, 32]; key_out / value_out fp32 views. */
int noise_key_scan(const float* qp, const float* kp, const float* k_raw, const float* lse, const float* values,
                   const float* hub, const float* center, const float* cos, const float* sin, int rows, int tokens,
                   int window, float sigma, const noise_rows_t* key_out, const noise_rows_t* value_out, void* stream);

/* Bytes of the caller's workspace for noise_key_scan_ws: a 256-byte status block, the receivers' pair features and
 * the hub's bf16 hi / lo halves (bf16 [rows, T, 64] x 5). 0 for rows < 1 or tokens < 1. */
size_t noise_key_scan_workspace_bytes(int rows, int tokens);

/* noise_key_scan with a caller workspace (256-byte aligned): T % 128 == 0 with 16-byte-aligned, non-blocked key_out /
 * value_out views runs on tcgen05 (the logits and scores as kind::tf32 MMAs reading the fp32 operands as they are,
 * which is how the reference's Triton tf32 dots run on this GPU; the moment sums as bf16 MMAs; the same kernel as
 * noise_moment_key_scores_ws); anything else falls through to noise_key_scan (tf32 operands rounded to nearest).
 * Same results (moment_kernels.py:467-607). */
int noise_key_scan_ws(const float* qp, const float* kp, const float* k_raw, const float* lse, const float* values,
                      const float* hub, const float* center, const float* cos, const float* sin, int rows, int tokens,
                      int window, float sigma, const noise_rows_t* key_out, const noise_rows_t* value_out,
                      void* workspace, size_t workspace_bytes, void* stream);

/* The identity phase's key credits and value sums (moment_kernels._moment_keys_kernel, :370-462): receivers s >= t
 * (full causal), q, k, v, hub bf16 [rows, T, 64]; raw (the keys' raw coordinates), side (the queries' fp32 pair
 * feature source) fp32 [rows, T, 64]; sq, steps (keys'), lse, hub_out (receivers') [rows, T]; out, values_out fp32
 * views. */
int noise_moment_key_scores(const void* q, const void* k, const void* v, const void* hub, const float* raw,
                            const float* sq, const float* side, const float* cos, const float* sin, const float* lse,
                            const float* hub_out, const float* steps, int rows, int tokens, const noise_rows_t* out,
                            const noise_rows_t* values_out, void* stream);

/* noise_moment_key_scores with raw as a view of `raw_dtype` (fp32 or bf16, blocked allowed) and out / values_out
 * views of `out_dtype`: the reference kernel's strided raw (RAW_BLK, RAW_GPU, RAW_STRIDE) and out arguments, as the
 * identity phase passes them (raw = the received heads' key pieces, out / values = its bf16 return buffer). */
int noise_moment_key_scores_v(const void* q, const void* k, const void* v, const void* hub, const noise_rows_t* raw,
                              int raw_dtype, const float* sq, const float* side, const float* cos, const float* sin,
                              const float* lse, const float* hub_out, const float* steps, int rows, int tokens,
                              const noise_rows_t* out, const noise_rows_t* values_out, int out_dtype, void* stream);

/* Bytes of the caller's workspace for noise_moment_key_scores_ws: a 256-byte status block, then the receivers' pair
 * features (bf16 [rows, T, 64] x 3). 0 for rows < 1 or tokens < 1. */
size_t noise_moment_key_scores_workspace_bytes(int rows, int tokens);

/* noise_moment_key_scores_v with a caller workspace (256-byte aligned): T % 128 == 0 with out / values_out views whose
 * strides are 16-byte multiples run on tcgen05 (a pass writing the receivers' pair features as bf16, then one
 * persistent kernel per 128-key tile: S = K Q^T and the scores V H^T into TMEM, the moment weights as bf16 A operands,
 * the five moment sums as tcgen05 MMAs, the response epilogue from TMEM); anything else falls through to
 * noise_moment_key_scores_v. Same results (moment_kernels.py:368-462). */
int noise_moment_key_scores_ws(const void* q, const void* k, const void* v, const void* hub, const noise_rows_t* raw,
                               int raw_dtype, const float* sq, const float* side, const float* cos, const float* sin,
                               const float* lse, const float* hub_out, const float* steps, int rows, int tokens,
                               const noise_rows_t* out, const noise_rows_t* values_out, int out_dtype, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Query credits: per query s and raw query coordinate d, zn / (1 + zd) / steps_s from the numerator / denominator
 * moments of its own softmax (moment_kernels._moment_queries_kernel, :197-365), rounded to bf16 (stored as bf16 or
 * as fp32 per out_dtype). q, k, v, hub bf16 [rows, T, 64]; raw (queries' raw coordinates), side (the keys' fp32 pair
 * feature source, kp at the reference's call site) fp32 [rows, T, 64]; sq, steps, lse, hub_out [rows, T]. */
int noise_moment_query_scores(const void* q, const void* k, const void* v, const void* hub, const float* raw,
                              const float* sq, const float* side, const float* cos, const float* sin, const float* lse,
                              const float* hub_out, const float* steps, int rows, int tokens, int window,
                              const noise_rows_t* out, int out_dtype, void* stream);

/* noise_moment_query_scores with raw as a view of `raw_dtype` (fp32 or bf16, blocked allowed) and out any view of
 * `out_dtype` (blocked allowed): the reference's strided raw / out arguments (moment_kernels.py:319-336). */
int noise_moment_query_scores_v(const void* q, const void* k, const void* v, const void* hub, const noise_rows_t* raw,
                                int raw_dtype, const float* sq, const float* side, const float* cos, const float* sin,
                                const float* lse, const float* hub_out, const float* steps, int rows, int tokens,
                                int window, const noise_rows_t* out, int out_dtype, void* stream);

/* Bytes of the caller's workspace for noise_moment_query_scores_ws: a 256-byte status block, then the keys' pair
 * features (bf16 [rows, T, 64] x 3). 0 for rows < 1 or tokens < 1. */
size_t noise_moment_query_scores_workspace_bytes(int rows, int tokens);

/* noise_moment_query_scores_v with a caller workspace (256-byte aligned): T % 128 == 0 with an out view whose strides
 * are 16-byte multiples runs on tcgen05 (a pass writing the keys' pair features as bf16, then one persistent kernel per
 * 128-query tile: S = Q K^T and the scores H V^T into TMEM, the four moment weights as bf16 A operands, the numerator,
 * denominator and logit-weighted moments as 160- and 64-wide tcgen05 MMAs, the response epilogue from TMEM); anything
 * else falls through to noise_moment_query_scores_v. Same results (moment_kernels.py:197-365). */
int noise_moment_query_scores_ws(const void* q, const void* k, const void* v, const void* hub, const noise_rows_t* raw,
                                 int raw_dtype, const float* sq, const float* side, const float* cos, const float* sin,
                                 const float* lse, const float* hub_out, const float* steps, int rows, int tokens,
                                 int window, const noise_rows_t* out, int out_dtype, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * The seed-rebuilt ES update (reference archive/10M/train/val/eggroll.py:151-167).
 * ------------------------------------------------------------------------------------------------------------- */

/* GEMM operands of the rebuild G = -(1 / count) sum_j w_j a_j b_j^T of one matrix parameter, straight from the noise
 * buffer: dst[e, j] = weight_scale * weight[j] * buffer[offsets[j] + shift + e] as bf16 (weight NULL: no scaling),
 * e < n_elem, j < pairs, and 0 for pairs <= j < k_padded. dst is [n_elem, k_padded] row-major. With shift = 0 and
 * the fitness weights this is A' (the out-side vectors); with shift = out and weight NULL it is B' (in-side); then
 * noise_gemm_bf16_tn(A', B', G, out, in, k_padded) gives G. Replaces the loop of eggroll.py:156-163. */
int noise_rank1_operands(const float* buffer, const int64_t* offsets, const float* weight, float weight_scale,
                         int64_t shift, int n_elem, int pairs, int k_padded, void* dst, void* stream);

/* noise_rank1_operands with fp32 output (dst float [n_elem, k_padded]): the operands of the tf32 update GEMM
 * (noise_gemm_tf32_tn), for the reference's fp32 rebuild at 'high' precision (eggroll.py:159-160, :184). */
int noise_rank1_operands_f32(const float* buffer, const int64_t* offsets, const float* weight, float weight_scale,
                             int64_t shift, int n_elem, int pairs, int k_padded, float* dst, void* stream);

/* out[o, i] = scale * sum_j weight[j] a_j[o] b_j[i] (fp32) for parameters too small for GEMM tiles: a_j =
 * buffer + offsets[j], b_j = a_j + n_out; with one_d != 0 the 1-D case out[i] = scale * sum_j weight[j] eps_j[i],
 * eps_j = buffer + offsets[j] (eggroll.py:162-163). */
int noise_rank1_small(const float* buffer, const int64_t* offsets, const float* weight, float scale, int n_out,
                      int n_in, int one_d, int pairs, float* out, void* stream);

/* torch.optim.AdamW with weight_decay = 0 (the reference's optimizer, eggroll.py:164-167, 205) on one flat fp32
 * tensor: exp_avg, exp_avg_sq updated in place, param -= (lr / (1 - beta1^step)) exp_avg /
 * (sqrt(exp_avg_sq) / sqrt(1 - beta2^step) + eps). */
int noise_adam_step(float* param, float* exp_avg, float* exp_avg_sq, const float* grad, int64_t n, float lr,
                    float beta1, float beta2, float eps, int step, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * Identity-phase head sharding (reference train/speedrun/run.py:3694-3804): the all_to_all send buffer, the
 * received heads' preparation and their moment credits.
 * ------------------------------------------------------------------------------------------------------------- */
#define NOISE_PACK (5 * NOISE_HEAD_DIM + 2) /* bf16 elements per packed row: q, k, v, o, target pieces + lse bits */
#define NOISE_MAX_PACK_LAYERS 16

/* One layer's pieces for noise_pack_heads: q, k, v, o (attention output) and target bf16 [tokens, >= 512] with row
 * strides in elements (even, 4-byte aligned rows; head h at columns 64 h .. 64 h + 63); lse fp32 [tokens / T, 8, T]. */
typedef struct {
  const void* q;
  const void* k;
  const void* v;
  const void* o;
  const void* target;
  int64_t q_stride, k_stride, v_stride, o_stride, target_stride;
  const float* lse;
} noise_head_pieces_t;

/* out (8, n_layers, tokens, NOISE_PACK) bf16: row (h, l, t) = head h's 64 columns of q, k, v, o, target of layer l at
 * token t, then the fp32 bits of lse[t / T, h, t % T] in its last two elements. Replaces run.py's pack_heads_kernel
 * / _pack_heads_kernel (:3698-3731); tokens % 16 == 0, tokens % seq_len == 0, n_layers <= 16. */
int noise_pack_heads(const noise_head_pieces_t* layers, int n_layers, int tokens, int seq_len, void* out, void* stream);

/* Outputs of noise_head_prep, rows = layers * world * n / T of T tokens each: q16, k16, v16, hub16 bf16 [rows, T, 64];
 * q32 fp32 [rows, T, 64]; k32 fp32 [rows, T, 64] or NULL (the reference does not keep it); the keys' pair features
 * f2 bf16 [rows, T, 64] (x_i, y_i interleaved), f4 [rows, T, 128] (x_i, x_i^2, y_i, y_i^2), xy [rows, T, 32], all three
 * or none; lse, hub_out (= hub . o), sq_q, sq_k (raw square norms), steps_q, steps_k fp32 [rows, T]. */
typedef struct {
  void* q16;
  void* k16;
  void* v16;
  void* hub16;
  float* q32;
  float* k32;
  void* f2;
  void* f4;
  void* xy;
  float* lse;
  float* hub_out;
  float* sq_q;
  float* sq_k;
  float* steps_q;
  float* steps_k;
} noise_head_prep_t;

/* The received heads from got (world, layers, n, NOISE_PACK) bf16: received row (w, l, i) becomes output token
 * (l * world + w) * n + i at position i % T; queries and keys RoPE'd (cos / sin fp32 [T, 32]) and RMS-normed with
 * eps, steps = sigma * max(sqrt(sq / 64), 1e-6). Replaces run.py's head_prep_fused / _head_prep_kernel (:3734-3796;
 * the reference calls it with sigma = KEY_SIGMA 0.003, eps = NORM_EPS 1e-6). n % 32 == 0, world * n % T == 0. */
int noise_head_prep(const void* got, int world, int layers, int n, const float* cos, const float* sin, int tokens,
                    float sigma, float eps, const noise_head_prep_t* out, void* stream);

/* Bytes of scratch noise_id_head_scores needs (its first int is the device status word of the tcgen05 moment
 * kernels). */
size_t noise_id_head_scores_workspace_bytes(int world, int layers, int n);

/* run.py's id_head_scores (:3799-3803): noise_head_prep, then the query-moment credits (full causal window) into
 * back[:, :, 0] and the key-moment credits and value sums into back[:, :, 1] and back[:, :, 2], the raw coordinates
 * read in place from got's q and k pieces. back: bf16 (world, layers, 3, n, 64). T % 64 == 0. */
int noise_id_head_scores(const void* got, int world, int layers, int n, const float* cos, const float* sin, int tokens,
                         float sigma, float eps, void* back, void* workspace, size_t workspace_bytes, void* stream);

/* The identity phase's two all_to_all_single exchanges (run.py:3887-3888 heads in, :3905-3906 heads out, completed by
 * heads_in.wait() :3902 / heads_out.wait() :3912) over peer memory: every rank owns one exchange buffer (device memory
 * from noise_exchange_alloc, mapped into the other ranks with CUDA IPC: plain NVLink loads and stores, no multicast).
 * Its first NOISE_EXCHANGE_HEAD_BYTES are control words (epoch flags per (slot, source rank), a local block counter
 * per slot); the rest holds the received data at offsets the caller chooses. A send writes chunk p of its data into
 * rank p's buffer at dst_offset + rank * chunk (all_to_all_single's layout) and then publishes `epoch` in rank p's
 * flag (slot, rank); noise_exchange_wait on rank p returns (on the stream) once every source's flag of the slot has
 * reached `epoch`. Epochs grow by one per exchange and slot; one exchange per slot is in flight at a time, and a rank
 * may send epoch e + 1 into a buffer only after its owner has finished reading epoch e (the identity phase's order:
 * heads out of step e is received before heads in of step e + 1 is sent). */
#define NOISE_MAX_PEERS 8
#define NOISE_EXCHANGE_HEAD_BYTES 1024
#define NOISE_IPC_HANDLE_BYTES 64
typedef struct {
  void* base[NOISE_MAX_PEERS]; /* every rank's exchange buffer as mapped in this process (own one included) */
  int rank;
  int world;
} noise_peers_t;

/* A zeroed exchange buffer of `bytes` (cudaMalloc, so it can be shared) and its IPC handle (NOISE_IPC_HANDLE_BYTES). */
int noise_exchange_alloc(size_t bytes, void** ptr, void* ipc_handle);
/* Map another rank's exchange buffer from its IPC handle (peer access enabled). */
int noise_exchange_open(const void* ipc_handle, void** ptr);
/* Unmap a buffer from noise_exchange_open. */
int noise_exchange_close(void* ptr);
/* Free a buffer from noise_exchange_alloc (after every other rank has closed its mapping). */
int noise_exchange_free(void* ptr);

/* Stream-ordered wait until flags (slot, w) of this rank's buffer reach epoch for every w < world; a wait longer than
 * limit_ns sets the workspace's status word to NOISE_DEVICE_TIMEOUT (NOISE_STATUS_BYTES workspace). */
int noise_exchange_wait(const noise_peers_t* peers, int slot, uint32_t epoch, int64_t limit_ns, void* workspace,
                        void* stream);

/* all_to_all_single over peer memory: chunk p of send (chunk_bytes, 16-byte multiple) to rank p's buffer at
 * dst_offset + rank * chunk_bytes, then epoch to flag (slot, rank) of every rank. Replaces the heads-out
 * dist.all_to_all_single(got2, back) (run.py:3905-3906). */
int noise_alltoall_peer(const void* send, size_t chunk_bytes, const noise_peers_t* peers, size_t dst_offset, int slot,
                        uint32_t epoch, void* stream);

/* noise_pack_heads fused with the heads-in exchange (run.py:3885-3888): row (h, l, t) of the pack goes straight to
 * rank p = h / (8 / world) at dst_offset + ((rank * (8 / world) + h % (8 / world)) * n_layers + l) * tokens + t rows
 * of NOISE_PACK bf16 (the all_to_all_single output layout), then epoch to flag (slot, rank) of every rank. world
 * divides 8. */
int noise_pack_heads_peer(const noise_head_pieces_t* layers, int n_layers, int tokens, int seq_len,
                          const noise_peers_t* peers, size_t dst_offset, int slot, uint32_t epoch, void* stream);

/* The identity phase's batched GEMMs (tcgen05, fp32 accumulation, bf16 out); each takes a workspace of at least
 * NOISE_STATUS_BYTES (the device status word) and at most 8 layers.
 *
 * out[l] = bf16(slope(us[l], steps[l]) * float(bf16(credb[l] @ w_out_t[l]))) with slope(u, s) = (max(u + s, 0)^2 -
 * max(u - s, 0)^2) / (2 s) in fp32: credb bf16 (layers, m, k), w_out_t bf16 (layers, k, n), us[l] bf16 (m, n), steps
 * fp32 (layers, m), out bf16 (layers, m, n); all contiguous; m % 128, n % 128, k % 64 == 0. Replaces
 * id_kernels.hidden_credits_fused / _hidden_credit_kernel (id_kernels.py:19-84; run.py:3818-3820). */
int noise_hidden_credits(const void* const* us, const float* steps, const void* credb, const void* w_out_t,
                         int layers, int m, int n, int k, void* out, void* workspace, size_t workspace_bytes,
                         void* stream);

/* out[l] = bf16(as[l]^T @ bs[l]) for as[l] bf16 (k, p), bs[l] bf16 (k, q) row-major, out bf16 (layers, p, q)
 * contiguous; k % 64, p % 128, q % 128 == 0. Replaces id_kernels.at_b_layers / _at_b_kernel (id_kernels.py:136-170;
 * run.py:3895-3896, 3911). */
int noise_at_b_layers(const void* const* as, const void* const* bs, int layers, int k, int p, int q, void* out,
                      void* workspace, size_t workspace_bytes, void* stream);

/* out[j * layers + l] = bf16(n1s[l]^T @ B_jl), B_jl[tok, w * 64 + c] = got2[w, l, j, tok, c]: n1s[l] bf16 (m, d)
 * row-major, got2 bf16 (world, layers, 3, m, 64) contiguous (the received heads_out), out bf16 (3 layers, d, d);
 * world * 64 == d, d % 128 == 0, m % 64 == 0. Replaces id_kernels.square_credit_grads / _square_credit_kernel
 * (id_kernels.py:87-133; run.py:3913). */
int noise_square_credit_grads(const void* const* n1s, const void* got2, int world, int layers, int m, int d,
                              void* out, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * Track-1 readout scorers (reference train/val/run.py, `recipe` section): the noise_record custom ops, head_dim 64,
 * fp32 arithmetic (the reference's tf32x3 dots are fp32-accurate).
 * ------------------------------------------------------------------------------------------------------------- */
/* A strided fp32 3-D view: element (i, j, k) at data[i * stride0 + j * stride1 + k * stride2] (torch strides). */
typedef struct {
  const float* data;
  int64_t stride0, stride1, stride2;
} noise_view3_t;

/* noise_record::future_scores (run.py:1729-1745; dense form joint_scores :1671-1681): out[h, p, m] (fp32 [H, P, M])
 * = sum over receivers s in (source_start + m, source_start + m + window] of (a (e^x - 1) c + (a + a (e^x - 1))
 * target_s . dv) / (1 + a (e^x - 1)), x = q_s . dk / 8, a = a[h, s, m], c = contrast[h, s, m]. q, target (H, T, 64)
 * views; dk, dv contiguous fp32 [H, P, M, 64] (16-byte aligned). */
int noise_future_scores(const noise_view3_t* q, const noise_view3_t* target, const float* dk, const float* dv,
                        const noise_view3_t* a, const noise_view3_t* contrast, int heads, int tokens, int probes,
                        int sources, int source_start, int window, float* out, void* stream);

/* noise_record::key_response (run.py:622-632, kernel :571-602): out[h, p, m] = sum over queries s (absolute position
 * query_start + s in [source_start + m, source_start + m + window]) of change / (1 + change) c[h, s, m],
 * change = a[h, s, m] (e^(q_s . dk / 8) - 1). q (H, T, 64) view; dk contiguous fp32 [H, P, M, 64]. */
int noise_key_response(const noise_view3_t* q, const float* dk, const noise_view3_t* a, const noise_view3_t* c,
                       int heads, int tokens, int probes, int sources, int source_start, int query_start, int window,
                       float* out, void* stream);

/* Bytes of the caller's workspace for noise_future_scores_ws / noise_key_response_ws: a 256-byte status block, then q
 * (and, for future_scores, target) as tf32 hi / lo planes, fp32 [heads, Tp, 64] each (Tp = tokens rounded up to 64).
 * 0 for an argument < 1. */
size_t noise_future_scores_workspace_bytes(int heads, int tokens);
size_t noise_key_response_workspace_bytes(int heads, int tokens);

/* noise_future_scores / noise_key_response on tcgen05 with a caller workspace (256-byte aligned, the *_workspace_bytes
 * query large; dk, dv 16-byte aligned): both dots at the reference kernels' tf32x3 precision (run.py:1714-1715, :585)
 * as kind::tf32 MMAs with the (probe, source) columns as the 128 MMA rows, so each column's sum over its receivers
 * stays in one thread; receivers stream in 32-row tiles over the union of a block's windows, each column masked to its
 * own. Same result definitions. The workspace's first int32 is the device status after the call completes: 0, or 1 if
 * a pipeline wait gave up (the output is then incomplete). heads x tokens (rounded up to 64) below 2^31 (int32 TMA row
 * coordinates; NOISE_ERR_SHAPE otherwise). */
int noise_future_scores_ws(const noise_view3_t* q, const noise_view3_t* target, const float* dk, const float* dv,
                           const noise_view3_t* a, const noise_view3_t* contrast, int heads, int tokens, int probes,
                           int sources, int source_start, int window, float* out, void* workspace,
                           size_t workspace_bytes, void* stream);
int noise_key_response_ws(const noise_view3_t* q, const float* dk, const noise_view3_t* a, const noise_view3_t* c,
                          int heads, int tokens, int probes, int sources, int source_start, int query_start,
                          int window, float* out, void* workspace, size_t workspace_bytes, void* stream);

/* noise_record::future_query_response (run.py:1818-1834, kernel :1780-1815): out[m, p, h] (fp32 [M, P, H, 64]) =
 * (sum_k change v_k - (sum_k change) base[h, m]) / (1 + sum_k change), change = probabilities[h, m, k]
 * (e^(dq[m, p, h] . k_k / 8) - 1). dq contiguous fp32 [M, P, H, 64]; keys, values (H, T, 64), probabilities (H, M, T),
 * base (H, M, 64) views. */
int noise_query_response(const float* dq, const noise_view3_t* keys, const noise_view3_t* values,
                         const noise_view3_t* probabilities, const noise_view3_t* base, int tokens, int probes,
                         int heads, int keys_len, float* out, void* stream);

/* The library's own fp32 e^x - 1 (the one the tcgen05 query_response evaluates: Cody-Waite reduction by ln2, degree-8
 * Taylor polynomial, no MUFU) over n device values; a numerics check against CUDA's expm1f. */
int noise_expm1_f32(const float* x, float* out, int64_t n, void* stream);

/* Bytes of the caller's workspace for noise_query_response_ws: a 256-byte status block, the keys and the transposed
 * values as tf32 hi / lo planes (fp32 [heads, Tp, 64] each, Tp = keys_len rounded up to 64) and one live flag per
 * (head, token, 64-key tile); 256 (the status block) when keys_len > 32,768. 0 for any argument < 1. */
size_t noise_query_response_workspace_bytes(int tokens, int probes, int heads, int keys_len);

/* noise_query_response on tcgen05 with a caller workspace (256-byte aligned, noise_query_response_workspace_bytes
 * large; dq and out 16-byte aligned): both dots at the reference kernel's tf32x3 precision (run.py:1808,1813), one
 * CTA per 128 (token, probe) rows of a head, S and change V as kind::tf32 MMAs with the change in tensor memory.
 * keys_len > 32,768 falls through to noise_query_response. Same result definition. The workspace's first int32 is
 * the device status after the call completes: 0, or 1 if a pipeline wait gave up (the output is then incomplete).
 * heads x Tp below 2^31 (int32 TMA row coordinates; NOISE_ERR_SHAPE otherwise). */
int noise_query_response_ws(const float* dq, const noise_view3_t* keys, const noise_view3_t* values,
                            const noise_view3_t* probabilities, const noise_view3_t* base, int tokens, int probes,
                            int heads, int keys_len, float* out, void* workspace, size_t workspace_bytes,
                            void* stream);

/* noise_record::routed_response (run.py:604-619, kernel :548-569): out[m, p, h] = bf16(w V) + (e^-dlse - 1) rest,
 * w = bf16(p_k (e^(ds - dlse) - 1)), ds = bf16(dq . k) / 8, dlse = log1p(sum_k p_k (e^ds - 1)). dq bf16
 * [M, P, H, 64], keys, values bf16 [M, H, K, 64], probabilities fp32 [M, H, K], rest fp32 [M, H, 64], all
 * contiguous; K <= 256. */
int noise_routed_response(const void* dq, const void* keys, const void* values, const float* probabilities,
                          const float* rest, int tokens, int probes, int heads, int keys_len, float* out,
                          void* stream);

/* noise_routed_response on tcgen05 with a workspace of at least NOISE_STATUS_BYTES (256-byte aligned; its first int32
 * is the device status after the call: 0, or 1 if a pipeline wait gave up and the output is incomplete); out 16-byte
 * aligned; keys_len <= 256; tokens x probes and tokens x heads x keys_len below 2^31 (the kernel's TMA row
 * coordinates are int32; NOISE_ERR_SHAPE otherwise). Both dots are kind::f16 MMAs (fp32 accumulation, outputs rounded
 * to bf16 as the reference kernel's tl.dot outputs are, run.py:561,565): two (token, head) items share the 128 MMA
 * rows when keys_len padded to 32 is at most 128, their weights block-diagonal in tensor memory. Same result
 * definition. */
int noise_routed_response_ws(const void* dq, const void* keys, const void* values, const float* probabilities,
                             const float* rest, int tokens, int probes, int heads, int keys_len, float* out,
                             void* workspace, size_t workspace_bytes, void* stream);

/* The true-path readout's scorer (reference train/val/run.py, `readout` section :5900-6040): width 512, 8 heads of
 * 64. Moment tables of one block, per (global token, head): U, W fp32 [T, 8, 64]; M1, M2 bf16 [T, 8, 64, 64] (16-byte
 * aligned); QD, GD fp32 [T, 8, 64]; AD, CD fp32 [T, 8]; VT, OT fp32 [T, 8, 64] (the self-edge only). */
typedef struct {
  const float* U;
  const float* W;
  const void* M1;
  const void* M2;
  const float* QD;
  const float* GD;
  const float* AD;
  const float* CD;
  const float* VT;
  const float* OT;
} noise_scorer_tables_t;

/* stats_kernel (:5968-5988): for the first n rows of each of `tokens` tokens of delta [tokens, d_rows, 512] fp32:
 * db bf16 [tokens, n, 512] = bf16(d), st fp32 [tokens, n, 2] = (inv', inv' / inv0 - 1) of the RMSNorm at x + d,
 * x = x[start + t] fp32 [T, 512], sqx[start + t] = |x|^2, eps as given. */
int noise_readout_stats(const float* delta, const float* x, const float* sqx, void* db, float* st, int start, int n,
                        int d_rows, int tokens, float eps, void* stream);

/* staged_kernel (:5991-6040): the rows' score against the tables from up bf16 [tokens * n, nc] (the projection
 * d W_k^T | d W_v^T | d[:32] W_g^T padded to 16), st (noise_readout_stats), r0 fp32 [T, 8, 64] (rotated clean raw
 * key), vc fp32 [T, 512] (raw value), gz fp32 [T, 8] and ve fp32 [T, 8, 64] (both NULL: no value-embedding gate),
 * cs / sn fp32 [T, 32]: out fp32 [tokens, n]; with se (bf16 [tokens, se_rows, 512]) also the self-edge; diag: add the
 * exact receiver s = t. */
int noise_readout_staged(const void* up, const float* st, const float* r0, const float* vc, const float* gz,
                         const float* ve, const float* cs, const float* sn, const noise_scorer_tables_t* tab,
                         float* out, void* se, int start, int n, int se_rows, int tokens, int nc, int diag,
                         void* stream);

/* noise_readout_staged with the moment-table terms on tcgen05 and a workspace of at least NOISE_STATUS_BYTES
 * (256-byte aligned; its first int32 is the device status after the call: 0, or 1 if a bounded wait gave up and out is
 * incomplete): per head bf16(dk) M1 and bf16(dk) M2 for 128 rows of a token as kind::f16 MMAs (the reference's
 * tl.dot of the same bf16 operands, run.py:6032-6033), each row's dot with its fp32 dk / dv one thread's sum over a
 * TMEM row; the rest as noise_readout_staged. Same arguments and results. (start + tokens) x 512 moment-table rows
 * below 2^31 (int32 TMA row coordinates; NOISE_ERR_SHAPE otherwise; noise_readout_direct_ws likewise). */
int noise_readout_staged_ws(const void* up, const float* st, const float* r0, const float* vc, const float* gz,
                            const float* ve, const float* cs, const float* sn, const noise_scorer_tables_t* tab,
                            float* out, void* se, int start, int n, int se_rows, int tokens, int nc, int diag,
                            void* workspace, size_t workspace_bytes, void* stream);

/* readout_kernel (:5906-5965): the same score from the projected change pj fp32 [tokens, probes, 2, 8, 64] (key and
 * value parts), r0 fp32 [tokens, 8, 64], cos / sin rows of the chunk's tokens (strided: token, pair), gc fp32
 * [tokens, probes, 8] and ve fp32 [tokens, 8, 64] (both NULL: ungated): out fp32 [tokens, probes]; se bf16
 * [tokens, probes, 512] or NULL. Tables at global token start + t. */
int noise_readout_direct(const float* pj, const float* r0, const float* cs, int64_t cs_token_stride,
                         int64_t cs_pair_stride, const float* sn, int64_t sn_token_stride, int64_t sn_pair_stride,
                         const float* gc, const float* ve, const noise_scorer_tables_t* tab, float* out, void* se,
                         int start, int probes, int tokens, int diag, void* stream);

/* noise_readout_direct with the moment-table terms on tcgen05 (as noise_readout_staged_ws: bf16(dk) M1 / M2 as
 * kind::f16 MMAs over 128 probes of a token, run.py:5952-5953) and a workspace of at least NOISE_STATUS_BYTES
 * (256-byte aligned; first int32 the device status). Same arguments and results. */
int noise_readout_direct_ws(const float* pj, const float* r0, const float* cs, int64_t cs_token_stride,
                            int64_t cs_pair_stride, const float* sn, int64_t sn_token_stride, int64_t sn_pair_stride,
                            const float* gc, const float* ve, const noise_scorer_tables_t* tab, float* out, void* se,
                            int start, int probes, int tokens, int diag, void* workspace, size_t workspace_bytes,
                            void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * The identity phase's readout cycle (reference train/speedrun/run.py:3569-3686), width 512, vocabulary 4096,
 * softcap 15. The GEMMs between these kernels (x W, h W, x h^T, fg1 c^T in fp32; fast_k c^p^T in bf16; the final
 * (moved - clean) / steps h) are the caller's.
 * ------------------------------------------------------------------------------------------------------------- */
/* _cycle_weights_kernel with cycle_scales' |x|^2 (run.py:3596-3647): per token of x fp32 [tokens, 512] and its
 * logits base fp32 [tokens, 4096]: fg1 fp32 [tokens, 4096] = f g1; fast bf16 [5, tokens, 4096] = (f z g2, f z^2 g3,
 * f g2, f z g3, f g3); rows fp32 [tokens, 3] = (sum f z g1, sum f z^2 g2, sum f z^3 g3); total, sq (|x|^2), base_y
 * (= base[targets]) fp32 [tokens]. */
int noise_cycle_weights(const float* x, const float* base, const int64_t* targets, int tokens, float* fg1, void* fast,
                        float* rows, float* total, float* sq, float* base_y, void* stream);

/* cycle_scales + cycle_finish up to its last GEMM (run.py:3588-3597, 3650-3662): out fp32 [tokens, directions] =
 * (moved - clean) / steps per (token, direction) from dots = x h^T, sq, exact = fg1 c^T and prods fp32
 * [5, tokens, directions] (the bf16 GEMMs' fp32 accumulators, rounded to bf16 here as the reference's bf16 outputs),
 * rows, total, base_y, c fp32 [directions, 4096], targets int64 [tokens], sigma (SIGMA 0.005). */
int noise_cycle_finish(const float* dots, const float* sq, const float* exact, const float* prods, const float* rows,
                       const float* total, const float* base_y, const float* c, const int64_t* targets, int tokens,
                       int directions, float sigma, float* out, void* stream);

/* coordinate_change (run.py:3569-3577): out fp32 [rows, 4096] = (log1p(w expm1(up - z)) - log1p(w expm1(down - z))
 * - onehot(targets) (up - down)) / (2 head_sigma), z = softcap(raw), up / down = softcap(raw +- head_sigma),
 * w = softmax(z); raw fp32 or bf16 [rows, 4096] contiguous. */
int noise_coordinate_change(const void* raw, int raw_dtype, const int64_t* targets, int rows, float head_sigma,
                            float* out, void* stream);

/* Bytes of scratch noise_population_loss needs for `members` members of `tokens` tokens each. */
size_t noise_population_workspace_bytes(int members, int tokens);

/* Per-member cross-entropy of m rank-1-perturbed copies of the GPT on one shared token row.
 * Replaces eggroll.population_loss (archive/10M/train/val/eggroll.py:66-103) and the lowrank/lowrank_embed
 * helpers it calls (:56-63); the perturbed weights are never materialised: every linear layer is a tcgen05 GEMM
 * whose epilogue adds sign_j (x . b_j) a_j.
 *   noise[NOISE_N_PARAMS]: host array of slices in named_parameters order; sign[m] fp32 (+-sigma);
 *   idx[T], targets[T] int64 token ids; losses[m] fp32 out (mean or sum over T per `reduction`), or with
 *   NOISE_REDUCTION_NONE losses[m * T], member-major (the reference's `ce` before its .mean(-1), eggroll.py:101-102).
 * Requirements: T % 128 == 0, 128 <= T <= 2048, members >= 1. */
int noise_population_loss(const noise_gpt_t* model, const noise_slice_t* noise, const float* sign,
                          const int64_t* idx, const int64_t* targets, int members, int tokens, int reduction,
                          float* losses, void* workspace, size_t workspace_bytes, void* stream);

/* The attention kernel's work schedule (host function, no device work; the forward's flex attention,
 * utils/model.py:24-31, has no counterpart): work item `item` of a launch over head_rows (member x head) rows of
 * `pairs` pairs of 128-query tiles, dealt round-robin to `grid` persistent CTAs, is pair *pair of head row *head_row.
 * order 0: heaviest pair first over the launch (the forward's default); order 1: blocks of `grid` head rows, each CTA
 * taking every pair of one row in turn so the row's keys and values are re-read from L2; order 2: head-major, a row's
 * pairs heaviest first, which the kernel's CTAs claim from a launch-wide counter as they finish (grid unused). The
 * forward uses order 1 or 2 when the environment variable NOISE_B200_ATTN_ORDER is "1" or "2"; order 2 keeps its
 * counter in word 32 of the workspace's status block. */
int noise_attention_item(int order, int item, int head_rows, int pairs, int grid, int* pair, int* head_row);

/* Bytes of scratch noise_gpt_loss needs for `rows` rows of `tokens` tokens. */
size_t noise_gpt_workspace_bytes(int rows, int tokens);

/* The un-perturbed forward and loss on `rows` distinct token rows: GPT.forward(idx, targets, loss_reduction)
 * (utils/model.py:193-209) with softcap 15 and ignore_index -1, computed as the population forward does (bf16
 * tensor-core linears with fp32 accumulation and an fp32 residual stream, fp32 embeddings: the autocast numerics of
 * EGGROLL's make_model weights, eggroll.py:38-53). idx, targets int64 [rows, T] row-major. out: one float (MEAN:
 * sum / counted tokens; SUM) or [rows * T] (NONE). Requirements as noise_population_loss. */
int noise_gpt_loss(const noise_gpt_t* model, const int64_t* idx, const int64_t* targets, int rows, int tokens,
                   int reduction, float* out, void* workspace, size_t workspace_bytes, void* stream);

/* Dust's additive jitter sites of one block (train/val/dust.py:102-125), each fp32 row-major or NULL: o [rows, 512]
 * on the attention output before c_proj, attn [rows, 512] on c_proj's output, fc [rows, 2048] on c_fc's
 * pre-activation, mlp [rows, 512] on mlp.c_proj's output. */
typedef struct {
  const float* o;
  const float* attn;
  const float* fc;
  const float* mlp;
} noise_jitter_t;

/* Bytes of scratch noise_block_forward needs for `seqs` sequences of `tokens` tokens. */
size_t noise_block_workspace_bytes(int seqs, int tokens);

/* Dust's block_forward (train/val/dust.py:102-125): one block `layer` of the un-perturbed model on x fp32
 * [seqs * tokens, 512] (the block's input, already mixed; updated in place to its output) with the jitter sites
 * added; ve fp32 [seqs * tokens, 512] (the captured value-embedding rows) on value-embedding blocks, NULL on the
 * others; window as the reference passes it. Numerics as the population forward's (bf16 linears, fp32 stream).
 * Requirements as noise_population_loss (tokens % 128 == 0, <= 2048); the model needs the layer's weights and the
 * RoPE tables only. */
int noise_block_forward(const noise_gpt_t* model, int layer, float* x, const float* ve, const noise_jitter_t* jit,
                        int seqs, int tokens, int window, void* workspace, size_t workspace_bytes, void* stream);

/* DUST.head_error's cached clean sums (train/val/dust.py:272-278): per row of raw [rows, >= 4096] (fp32 or bf16,
 * row stride raw_stride elements): slab_sums fp32 [rows, 16] = sum over each 256-column slab of e^(softcap(raw)),
 * total fp32 [rows], clean_target fp32 [rows] = softcap(raw[max(target, 0)]). */
int noise_head_error_prep(const void* raw, int raw_dtype, int64_t raw_stride, const int64_t* targets, int rows,
                          float* slab_sums, float* total, float* clean_target, void* stream);

/* One chunk of DUST.head_error (dust.py:281-301): `draws` jitters noise bf16 [draws * batch, tokens, 256] of slab
 * `slab` of raw (rows b * tokens + t); each draw's loss from the cached sums, its reward clean_loss - loss (0 where the
 * target is -1) centred across the batch rows, and error fp32 [rows, raw_stride] columns of the slab -=
 * bf16(sum over draws of bf16(reward / sigma) noise). draws * batch <= 8192. */
int noise_head_error_chunk(const void* raw, int raw_dtype, int64_t raw_stride, const void* noise,
                           const int64_t* targets, const float* clean_loss, const float* slab_sums,
                           const float* total, const float* clean_target, int batch, int tokens, int draws, int slab,
                           float sigma, float* error, void* stream);

/* Bytes of scratch noise_head_loss needs for `rows` rows. */
size_t noise_head_loss_workspace_bytes(int rows);

/* Per-token loss of the final norm, LM head, softcap 15 and cross-entropy (reduction 'none', ignore_index -1):
 * replaces dust.head_loss (train/val/dust.py:94-99) and the tail of GPT.forward (utils/model.py:202-208).
 *   x fp32 [rows, 512] (the residual stream); weight bf16 [>= 4096, 512] row-major (rows past the vocabulary are
 *   ignored, as the reference's [..., :vocab]); targets int64 [rows]; out fp32 [rows].
 * Requirements: rows % 128 == 0, 128 <= rows <= 2^22; x and weight 16-byte aligned. */
int noise_head_loss(const float* x, const void* weight, const int64_t* targets, int rows, float* out, void* workspace,
                    size_t workspace_bytes, void* stream);

/* No counterpart in the reference: noise_population_loss for callers that cannot allocate device memory — a host
 * that embeds this library without a CUDA allocator of its own (a C/FFI caller that must not call cudaMalloc, which
 * synchronises the device, on its hot path), or one whose memory pool is fully reserved by the time it evaluates.
 * Same arguments and results as noise_population_loss minus the workspace: the scratch is a file-scope
 * __device__ array of NOISE_STATIC_SCRATCH_BYTES that every GPU which loads the library holds until exit, so
 * members * tokens is limited to what fits in it (noise_population_workspace_bytes(members, tokens) <=
 * NOISE_STATIC_SCRATCH_BYTES, about 4,400 rows, e.g. 2 members x 2048 tokens); larger sizes return
 * NOISE_ERR_TOO_LARGE before anything is launched. Nothing is allocated: no cudaMalloc/cudaFree, no allocating
 * library routine. The first call on a device looks up the array's device address (cudaGetSymbolAddress, with
 * that device current); make that first call before any stream capture. All calls share the one array and it
 * keeps the last call's contents (the status word is cleared at the start of each call): calls that overlap on the
 * GPU (concurrent streams, or threads sharing a device) race on it, so serialise them. `stream` must belong to the
 * current device (the array used is the current device's): a stream of another device, or a current device index
 * at or above NOISE_STATIC_MAX_DEVICES, returns NOISE_ERR_ARGUMENT. The device status word is the array's first int;
 * read it with noise_read_static_status. */
#define NOISE_STATIC_SCRATCH_BYTES (48u << 20)
#define NOISE_STATIC_MAX_DEVICES 64
int noise_population_loss_noalloc(const noise_gpt_t* model, const noise_slice_t* noise, const float* sign,
                                  const int64_t* idx, const int64_t* targets, int members, int tokens, int reduction,
                                  float* losses, void* stream);

/* No counterpart in the reference: the device status word of noise_population_loss_noalloc's static scratch on the
 * current device, copied to *status after `stream` (which must belong to the current device) is synchronised.
 * NOISE_DEVICE_TIMEOUT there means a bounded wait of the last call gave up and its losses are not valid. */
int noise_read_static_status(int* status, void* stream);

/* D[m, n] (fp32, row-major) = A[m, k] . B[n, k]^T for bf16 row-major A and B, on the persistent tcgen05/TMA GEMM
 * that every linear layer of noise_population_loss runs on, with a plain store epilogue. Stands in for the cuBLAS
 * GEMM autocast issues for `x @ weight.t()` (eggroll.py:58; utils/model.py:83-85) and for the bf16 moment products
 * of the readout cycle (train/speedrun/run.py:3681-3685). m >= 1, n % 32 == 0, k % 8 == 0 (partial tiles read zeros
 * past the edges and store only inside D); A, B, D 16-byte aligned; `workspace` holds at least NOISE_STATUS_BYTES
 * (the device status word). */
int noise_gemm_bf16_tn(const void* a, const void* b, float* d, int m, int n, int k, void* workspace, void* stream);

/* The same GEMM on fp32 A and B read as tf32 (tcgen05 kind::tf32, fp32 accumulation): an fp32 matmul at
 * torch.set_float32_matmul_precision('high'), which the reference sets for its fp32 contractions — the seed-rebuilt
 * update (archive/10M/train/val/eggroll.py:159-160, precision set at :184) and the readout cycle's x W, h W, x h^T,
 * fg1 c^T and out h (train/speedrun/run.py:3673-3686, precision set at :4447). m >= 1, n % 32 == 0, k % 4 == 0. */
int noise_gemm_tf32_tn(const float* a, const float* b, float* d, int m, int n, int k, void* workspace, void* stream);

/* fp32 -> bf16 (round to nearest even) of n values; both pointers 16-byte aligned, n % 8 == 0.
 * Replaces autocast's per-call weight casts inside the reference's linears (eggroll.py:58 under
 * torch.autocast, eggroll.py:144). */
int noise_pack_bf16(const float* src, void* dst, int64_t n, void* stream);

/* Copy the device status word at the head of `workspace` to *status (synchronises `stream`). */
int noise_read_status(const void* workspace, int* status, void* stream);

/* Clear the device status word (enqueued on `stream`). */
int noise_clear_status(void* workspace, void* stream);

/* Human-readable name of a NOISE_ERR_* status. */
const char* noise_status_string(int status);

/* Number of kernels the most recent successful noise_population_loss call on this thread enqueued. */
int noise_last_launch_count(void);

/* Per-launch timing with CUDA events (no counterpart in the reference, which times whole updates with CUDA events,
 * train/speedrun/run.py:4262-4263). After noise_profile_start(capacity), every launch of noise_population_loss /
 * noise_gemm_bf16_tn on this thread records an event pair around itself on its stream (up to `capacity` launches).
 * noise_profile_stop synchronises on the recorded events, adds the elapsed milliseconds per kernel kind into
 * kind_ms[k] / kind_count[k] (k < nkinds; kinds: 0 norm+mix, 1 QKV GEMM, 2 attention, 3 c_proj GEMM, 4 mid norm,
 * 5 c_fc GEMM, 6 mlp.c_proj GEMM, 7 final norm, 8 LM-head+CE GEMM, 9 member reduce, 10 plain GEMM), frees the
 * events and turns timing off (kind_ms / kind_count may be NULL to discard). */
int noise_profile_start(int capacity);
int noise_profile_stop(float* kind_ms, int* kind_count, int nkinds);

#ifdef __cplusplus
}
#endif

#endif /* NOISE_B200_H */
