/*
 * so101_b200.h — C ABI of the B200 SmolVLA chunk kernels (libso101_b200.so).
 *
 * Every entry point takes device pointers, element strides, sizes and a cudaStream_t, launches
 * asynchronously on that stream, allocates nothing, and returns an int status (0 = ok, see
 * SO101_ERR_*). Nothing here takes or returns a framework type; the Python engine binds these
 * with ctypes, and any other host language can bind them the same way.
 *
 * Each entry point names the reference (so101-smolvla-edge, paths relative to its
 * src/so101_smolvla_edge/) function or kernel it replaces.
 */
#ifndef SO101_B200_H
#define SO101_B200_H

#include <stdint.h>
#include <cuda_runtime.h>

#if defined(__GNUC__)
#define SO101_API __attribute__((visibility("default")))
#else
#define SO101_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------------------- */
#define SO101_OK 0
#define SO101_ERR_ARG 1         /* a size, stride, pointer alignment or dtype is unsupported */
#define SO101_ERR_LAUNCH 2      /* the CUDA launch failed (cudaGetLastError after the launch) */
#define SO101_ERR_WORKSPACE 3   /* split-K workspace or ticket array too small */
#define SO101_ERR_TIMEOUT 4     /* a device wait hit its bound (read with so101_device_status) */
#define SO101_ERR_DRIVER 5      /* a driver entry point (TMA descriptors, current context) is unavailable */

/* ---- element types --------------------------------------------------------------------- */
#define SO101_BF16 0
#define SO101_F32 1
#define SO101_I8 2

/* ---- GEMM epilogues -------------------------------------------------------------------- */
#define SO101_EPI_NONE 0      /* y = acc (+ bias)                                           */
#define SO101_EPI_GELU 1      /* y = gelu_tanh(acc + bias)                                   */
#define SO101_EPI_SILU_GATE 2 /* w = [gate; up] (2N x K): y = silu(x@gate^T) * (x@up^T)     */

/* Epilogue operands of so101_gemm, applied in this order to the fp32 (or dequantized int32)
 * accumulator of output element (m, n):
 *   v  = acc * x_scale * w_scale[n]            (int8 operands only)
 *   v += bias[n]                               (bias != NULL)
 *   v  = gelu(v) | silu(v) * v_up              (epilogue)
 *   v *= out_scale
 *   v += residual[(m % r_period) * ldr + n]    (residual != NULL; r_period 0 = no period)
 *   y[row(m) * ldy + n] = cast(v)              (I8: clamp(rint(v / y_qscale), -128, 127))
 * row(m) = (m / row_group) * row_stride + m % row_group when row_group > 0, else m.
 * y may alias residual (each element is read before it is written, by the same thread).
 *
 * RMSNorm split between two GEMMs (the reference launches rms_norm before these GEMMs,
 * pkg/model/smolvla_triton.py:87,101,114,126): rmsnorm(x) W^T = rstd[m] (x * w) W^T, so with the
 * operand bf16(x * w) written by the producer of the residual stream x (y16, y16_scale = w),
 *   rms_ss != NULL: first v *= rsqrt(sum_{s < rms_slots} rms_ss[m * rms_ld + s] / rms_n + rms_eps)
 * (rms_slots <= 64, rms_ld a multiple of 4, rms_ss 16-byte aligned) where rms_ss holds sums of
 * squares of the residual rows written by its producer:
 *   stat_ss != NULL: stat_ss[m * stat_ld + slot] = sum of the final v^2 over one of the disjoint
 *   feature ranges of row m, slots [0, so101_gemm_stat_slots(...)), summed in slot order
 *   y16 != NULL: y16[row(m) * ld16 + n] = bf16(final v * y16_scale[n]), the next GEMM's operand
 *   (y16_scale: the next norm's weight, fp32, 16-byte aligned; NULL: 1)
 * stat_ss / y16 need the vectorised bf16 epilogues (so101_gemm_stat_slots says whether the plan
 * has one), no GELU, an fp32 residual if any and N a multiple of 16. Zero fields mean "off".
 * The weights stay as they are: scaling the activations rather than the weights by w rounds once
 * per element, as the reference's rms_norm does. */
typedef struct so101_epilogue {
  int epilogue;
  const float* bias;
  const void* residual;
  int64_t ldr;
  int r_type;
  int64_t r_period;
  float out_scale;
  const float* w_scale;
  float x_scale;
  float y_qscale;
  int64_t row_group;
  int64_t row_stride;
  const float* rms_ss;
  int rms_slots;
  int64_t rms_ld;
  float rms_n;
  float rms_eps;
  float* stat_ss;
  int64_t stat_ld;
  void* y16;
  int64_t ld16;
  const float* y16_scale;
} so101_epilogue;

/* Tile configuration; zero-initialised fields mean "pick" (the heuristic of so101_gemm_pick). */
typedef struct so101_gemm_config {
  int swap;    /* 1: weights on the MMA M side (few token rows), 0: tokens on the M side */
  int bn;      /* MMA N: 16, 32, 48, 64 (swap) or 64, 128, 256, 192 (tokens on M; 192:   */
               /* persistent kernel or CTA pair only, no SiLU gate)                      */
  int splits;  /* K splits, reduced in split order (deterministic)                        */
  int stages;  /* shared-memory pipeline depth (0: chosen from the problem)               */
  int flags;   /* SO101_GEMM_* bits                                                       */
} so101_gemm_config;

/* so101_gemm_config.flags. By default split-K partials are reduced on chip across a thread-block
 * cluster (splits <= 8) and large problems with tokens on the MMA M side run the persistent
 * kernel (one CTA per SM, double-buffered TMEM accumulators). */
#define SO101_GEMM_GLOBAL_SPLITK 1     /* reduce split-K partials through the workspace       */
#define SO101_GEMM_PERSISTENT 2        /* tokens on M, no split: always the persistent kernel */
#define SO101_GEMM_ONE_TILE_PER_CTA 4  /* tokens on M: never the persistent kernel            */
#define SO101_GEMM_PAIR 8              /* tokens on M, no split, bn 128/192/256 (192 without  */
                                       /* the SiLU gate): CTA-pair tiles                      */
                                       /* (256 x bn per two SMs, cta_group::2 MMAs)           */

/* y (M x N) = epilogue(x (M x K) @ w (N x K)^T) on tcgen05 tensor cores, TMA-fed.
 * Replaces kernels/gemm.py:48-96 (so101_gemm) and :350-398 (linear), the cuBLAS F.linear calls of
 * model/smolvla.py:152-156 and the TensorRT vision GEMMs (model/trt_vision.py:102-163, int8).
 * a_type SO101_BF16 (kind::f16, fp32 accumulate) or SO101_I8 (kind::i8, int32 accumulate).
 * Requires: 16-byte aligned x, w; K * elem_size and ldx, ldw a multiple of 16 bytes.
 * workspace: fp32 split-K partials; tickets: int32 counters, zero before the first call and left
 * zero by every call; both are used only by SO101_GEMM_GLOBAL_SPLITK plans (and splits > 8).
 * Bytes needed: so101_gemm_workspace. cfg may be NULL. */
SO101_API int so101_gemm(int a_type, const void* x, int64_t ldx, const void* w, int64_t ldw, void* y,
               int64_t ldy, int y_type, int64_t M, int64_t N, int64_t K,
               const so101_epilogue* epi, const so101_gemm_config* cfg, void* workspace,
               int64_t workspace_bytes, int* tickets, int64_t n_tickets, cudaStream_t stream);

/* How many statistics slots (stat_ss) the plan of this problem writes; SO101_ERR_ARG when its
 * epilogue cannot produce them. No counterpart in the reference, whose RMSNorm is a GEMM prologue. */
SO101_API int so101_gemm_stat_slots(int a_type, int64_t M, int64_t N, int64_t K, int epilogue,
                                    const so101_gemm_config* cfg, int* slots);

/* The configuration so101_gemm would pick for this problem on this device (cfg out). */
SO101_API int so101_gemm_pick(int a_type, int64_t M, int64_t N, int64_t K, int epilogue,
                    so101_gemm_config* cfg);

/* Split-K workspace bytes and ticket count a configuration needs. */
SO101_API int so101_gemm_workspace(int a_type, int64_t M, int64_t N, int64_t K, int epilogue,
                         const so101_gemm_config* cfg, int64_t* workspace_bytes,
                         int64_t* n_tickets);

/* Grouped-query flash attention, bf16 in, fp32 online softmax (exp2), P rounded to bf16 for PV.
 * Replaces kernels/attention.py:27-120 (so101_attention) and the SDPA calls of
 * model/smolvla.py:182, 298, 303, 312-325.
 * q: (Lq, >= nq*hd) rows of stride ldq, head h at columns [h*hd, (h+1)*hd); k, v: (Lk, nkv*hd).
 * Query head h reads kv head h / (nq / nkv). Key j is visible to query i iff
 * j < causal_from || j <= i + q_offset. cos/sin (Lq x hd/2) rotate q on load (NULL: none).
 * batch: independent problems at element strides bq, bk, bv, bo. o: (Lq, nq*hd) in o_type
 * (SO101_BF16, or SO101_I8 quantized by o_qscale). hd: 32, 64 or 128. */
SO101_API int so101_attention(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                    int64_t ldv, void* o, int64_t ldo, int o_type, float o_qscale, int64_t Lq,
                    int64_t Lk, int nq, int nkv, int hd, int64_t causal_from, int64_t q_offset,
                    const float* cos, const float* sin, int batch, int64_t bq, int64_t bk,
                    int64_t bv, int64_t bo, cudaStream_t stream);

/* so101_attention where keys j >= own_from (and their values) are the current step's own rows,
 * read from row j - own_from of k_own / v_own (row stride ld_own, batch stride b_own: the fused
 * q|k|v output) instead of k / v, and rotated on chip by k_cos / k_sin (row j - own_from, hd/2
 * columns) exactly as so101_rope_kv rotates cache rows. Replaces the rope_kv launch that writes the
 * expert's own rows into the K/V cache before each self-attention (kernels/rope.py:17-66 followed
 * by kernels/attention.py:27-120). hd 64; k_own, v_own 16-byte aligned. */
SO101_API int so101_attention_rows(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                                   int64_t ldv, void* o, int64_t ldo, int o_type, float o_qscale, int64_t Lq,
                                   int64_t Lk, int nq, int nkv, int hd, int64_t causal_from, int64_t q_offset,
                                   const float* cos, const float* sin, int batch, int64_t bq, int64_t bk,
                                   int64_t bv, int64_t bo, const void* k_own, const void* v_own, int64_t ld_own,
                                   int64_t b_own, int64_t own_from, const float* k_cos, const float* k_sin,
                                   cudaStream_t stream);

/* Attention fused with its output projection and residual (the few query rows of one
 * observation): y = residual + attention(q, k, v) @ w_o^T, attention arguments and mask as
 * so101_attention_rows (k_own NULL: every key from k / v), bf16 attention output rows, hd 64,
 * nq <= 16 query heads (one cluster of nq CTAs per 128-feature output tile). y and residual fp32
 * (rows b * Lq + i; residual may be y), w_o (n_out x nq * 64) bf16 with row stride ldw. Optional
 * y16 = bf16(y * y16_scale[col]) and stat_ss[row * stat_ld + tile] = the row's sum of squares over
 * output tile `tile` (ceil(n_out / 128) statistics slots, the rms_ss/rms_slots of the next GEMM's
 * so101_epilogue). The projection sums heads in head order: deterministic; not bit-identical to
 * so101_attention followed by so101_gemm (which sums K in another order). Replaces the expert's
 * attention launch and o-projection launch, model/smolvla_triton.py:118-125 (attention, then
 * lin(a, exp.{i}.o, residual=e); the torch path's model/smolvla.py:298-304).
 * SO101_ERR_ARG when the GPU cannot hold a cluster of nq CTAs. */
SO101_API int so101_attention_o(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v,
                                int64_t ldv, int64_t Lq, int64_t Lk, int nq, int nkv, int hd,
                                int64_t causal_from, int64_t q_offset, const float* cos, const float* sin,
                                int batch, int64_t bq, int64_t bk, int64_t bv, const void* k_own,
                                const void* v_own, int64_t ld_own, int64_t b_own, int64_t own_from,
                                const float* k_cos, const float* k_sin, const void* w_o, int64_t ldw,
                                int64_t n_out, float* y, int64_t ldy, const float* residual, int64_t ldr,
                                void* y16, int64_t ld16, const float* y16_scale, float* stat_ss,
                                int64_t stat_ld, cudaStream_t stream);

/* The SwiGLU MLP block of the few token rows of one observation in one launch:
 * y = residual + (silu(rs * x @ w_gate^T) * (rs * x @ w_up^T)) @ w_down^T, x (batch * rows x k)
 * bf16 with rows <= 64 per observation, rs = rsqrt(sum of the row's rms_slots statistics / k +
 * rms_eps) (rms_ss NULL: rs = 1), w_gate_up (2 * mlp x k: gate rows, then up rows) and w_down
 * (n_out x mlp) bf16, mlp a multiple of 128 and at most 2048 (one cluster of mlp / 128 CTAs per
 * 128-feature output tile, each owning 128 hidden features; hidden activations rounded to bf16
 * as the unfused chain stores them). y, residual, y16, y16_scale and stat_ss as
 * so101_attention_o. Replaces model/smolvla_triton.py:126-128 (rms_norm ln_post, lin gate_up with
 * the SiLU gate, lin down with the residual; the torch path's model/smolvla.py:305-307).
 * SO101_ERR_ARG when the GPU cannot hold a cluster of mlp / 128 CTAs. */
SO101_API int so101_mlp(const void* x, int64_t ldx, int64_t rows, int batch, int64_t k, const float* rms_ss,
                        int rms_slots, int64_t rms_ld, float rms_eps, const void* w_gate_up, int64_t ldw1,
                        int64_t mlp, const void* w_down, int64_t ldw2, int64_t n_out, float* y, int64_t ldy,
                        const float* residual, int64_t ldr, void* y16, int64_t ld16, const float* y16_scale,
                        float* stat_ss, int64_t stat_ld, cudaStream_t stream);

/* y (rows x n) = x * rsqrt(mean(x^2) + eps) * w, statistics in fp32, one rounding to y_type.
 * x_type SO101_F32 or SO101_BF16. Replaces kernels/norm.py:14-42 and model/smolvla.py:72-74. */
SO101_API int so101_rms_norm(const void* x, int64_t ldx, int x_type, const float* w, void* y,
                   int64_t ldy, int y_type, int64_t rows, int64_t n, float eps,
                   cudaStream_t stream);

/* Statistics of an fp32 residual stream for an RMSNorm finished in the consuming GEMM
 * (so101_epilogue.rms_ss): per row the sum of squares of its n values into stat_ss[row * stat_ld]
 * (one slot) and bf16(row * w) into y16 (ld16; w: the norm weight, 16-byte aligned, NULL: 1).
 * Replaces the reference's rms_norm launch (pkg/kernels/norm.py:14-42) where no GEMM epilogue
 * produced the statistics (the first norm of a pass). */
SO101_API int so101_rms_stats(const float* x, int64_t ldx, int64_t rows, int64_t n, const float* w, void* y16,
                              int64_t ld16, float* stat_ss, int64_t stat_ld, cudaStream_t stream);

/* LayerNorm (fp32 statistics, fp32 affine) of x (rows x n) fp32 into y_type (SO101_BF16 or
 * SO101_I8 with y_qscale). shuffle > 1 writes the SmolVLM pixel shuffle of each image's
 * tokens_per_image rows (model/smolvla.py:105-114) instead of row order. Replaces the
 * F.layer_norm + pixel_shuffle of model/smolvla.py:174-175, 189. */
SO101_API int so101_layer_norm(const float* x, int64_t ldx, const float* w, const float* b, void* y,
                     int64_t ldy, int y_type, float y_qscale, int64_t rows, int64_t n, float eps,
                     int shuffle, int64_t tokens_per_image, cudaStream_t stream);

/* Rotate the key columns of fused qkv rows into k_out and copy the value columns into v_out
 * (v_out may be NULL), fp32 rotation, bf16 store. Replaces kernels/rope.py:17-66.
 * qkv: (rows, (nq + 2 nkv) hd) stride ldqkv; cos/sin: (rows, hd/2); batch strides in elements. */
SO101_API int so101_rope_kv(const void* qkv, int64_t ldqkv, int nq, int nkv, int hd, const float* cos,
                  const float* sin, void* k_out, int64_t ldk, void* v_out, int64_t ldv,
                  int64_t rows, int batch, int64_t b_qkv, int64_t b_k, int64_t b_v,
                  cudaStream_t stream);

/* Camera frames to SigLIP patch rows: uint8 (n_img, h, w, 3) -> /255 -> bilinear resize
 * (align_corners=False) to (rh, rw) -> zero pad on the left and top to S x S -> *2-1 -> patches
 * (n_img * (S/P)^2, 3*P*P) in bf16 (or int8 with y_qscale). Replaces model/engine.py:236-245 and
 * the patch unfold of model/smolvla.py:166-168. */
SO101_API int so101_preprocess(const uint8_t* img, int n_img, int h, int w, int rh, int rw, int S, int P,
                     void* patches, int y_type, float y_qscale, cudaStream_t stream);

/* Preprocessed frames to SigLIP patch rows: px (n_img, 3, S, S) float32 in [-1, 1] -> patches
 * (n_img * (S/P)^2, 3*P*P) in bf16, int8 (with y_qscale) or fp32. The patch unfold of
 * model/smolvla.py:166-168 for callers that hand over px, as the reference's TrtVision input
 * (model/trt_vision.py:212-252) is. */
SO101_API int so101_patchify(const float* px, int n_img, int S, int P, void* patches, int y_type, float y_qscale,
                             cudaStream_t stream);

/* SigLIP patch embedding straight from camera frames at the model's size (no resize): uint8
 * (n_img, S, S, 3) -> per 16 x 16 patch, (v / 255) * 2 - 1 in bf16, unfolded as channel, row,
 * column -> y (n_img * (S/16)^2, N) fp32 = patches @ w^T + bias + pos[row % period]. The
 * preprocessing of model/engine.py:236-245 and the unfold of model/smolvla.py:166-168 run inside
 * the patch GEMM's operand producer (the patch rows never reach global memory); the result equals
 * so101_preprocess followed by so101_gemm bit for bit. w: (N, 768) bf16, N a multiple of 256;
 * S a multiple of 16 with G = S / 16 dividing 128 and G^2 a multiple of 128 (every 128
 * consecutive patches are whole patch rows of one frame: S = 256, 512); every pointer 16-byte
 * aligned. */
SO101_API int so101_patch_embed(const uint8_t* img, int n_img, int S, const void* w, int64_t ldw, int64_t N,
                                const float* bias, const float* pos, int64_t period, float* y, int64_t ldy,
                                cudaStream_t stream);

/* Dense fp32 linear on CUDA cores (the reference keeps these small MLPs fp32):
 * y[m, n] = act(x[m, :] @ w[n, :] + bias[n] (+ bias2[n])), act 0 none, 2 SiLU (act 1 is
 * accepted and means none: SiLU belongs on the producer's output). K, ldx, ldw multiples of 4,
 * x and w 16-byte aligned.
 * Replaces the fp32 F.linear calls of model/smolvla.py:282-285, 309 and engine.py:251. */
SO101_API int so101_linear_f32(const float* x, int64_t ldx, const float* w, int64_t ldw, const float* bias,
                     const float* bias2, float* y, int64_t ldy, int64_t M, int64_t N, int64_t K,
                     int act, cudaStream_t stream);

/* x (M x K fp32, row stride ldx) -> y (M x 3K bf16, row stride ldy) = [bf16(x) | bf16(x) |
 * bf16(x - bf16(x))]: with w3 = [W_hi | W_lo | W_hi] (W_hi = bf16(W), W_lo = bf16(W - W_hi)),
 * so101_gemm(y, w3) is the fp32 linear x W^T to about 2^-16 relative on the tensor cores (the
 * split's lo x lo term dropped). K a multiple of 4, x 16-byte and y 8-byte aligned. No reference
 * counterpart: the engine's batched form of the fp32 linear of model/smolvla.py:285. */
SO101_API int so101_split_bf16x3(const float* x, int64_t ldx, int64_t M, int64_t K, void* y, int64_t ldy,
                                 cudaStream_t stream);

/* The expert's output head and Euler step, per row m of e (M x K): x_t[m, :] += dt *
 * (rms_norm(e[m], norm_w) @ w_out^T + b_out). Replaces model/smolvla.py:308-309 and
 * engine.py:263-271 (x_t + dt * v_t). */
SO101_API int so101_expert_out(const float* e, int64_t lde, const float* norm_w, float eps,
                     const float* w_out, const float* b_out, float* x_t, int64_t ldx,
                     int64_t M, int64_t N, int64_t K, float dt, cudaStream_t stream);

/* Prefix tail rows per observation: lang rows copied from lang (lang_len x d) and the state row
 * state_w @ pad((state - mean) / (std + 1e-8)) + state_b written at rows [tail_row, tail_row +
 * lang_len] of each observation's prefix (stride prefix_rows rows of ldp). Replaces
 * model/engine.py:247-252. */
SO101_API int so101_prefix_tail(const float* state, int state_dim, const float* s_mean,
                      const float* s_std, const float* state_w, int max_state,
                      const float* state_b, const float* lang, int lang_len, int d,
                      float* prefix, int64_t ldp, int64_t prefix_rows, int64_t tail_row,
                      int batch, cudaStream_t stream);

/* Undo the action representation and normalisation: x_t (batch, H, max_action) fp32 ->
 * out (batch, H, action_dim). repr 0 absolute, 1 delta, 2 velocity (cumulative over H).
 * Replaces model/engine.py:281-291. */
SO101_API int so101_finish(const float* x_t, int max_action, const float* state, int state_dim,
                 const float* s_mean, const float* s_std, const float* r_mean,
                 const float* r_std, const float* a_mean, const float* a_std, float* out,
                 int action_dim, int H, int repr, int batch, cudaStream_t stream);

/* Per-tensor max |x| of a (rows x n) matrix (x_type SO101_F32 or SO101_BF16) folded into
 * *amax with atomicMax (int8 calibration; tests/test_ov_engine.py:222-225 semantics). */
SO101_API int so101_absmax(const void* x, int64_t ldx, int x_type, int64_t rows, int64_t n, float* amax,
                 cudaStream_t stream);

/* Per-output-channel symmetric int8 weights: w_q[n, k] = clamp(rint(w[n, k] / s[n]), -127, 127),
 * s[n] = max(max_k |w[n, k]| / 127, 1e-8), from bf16 or fp32 w (model/trt_vision.py:131-133). */
SO101_API int so101_quantize_weight(const void* w, int w_type, int64_t N, int64_t K, int8_t* w_q,
                          float* scale, cudaStream_t stream);

/* Device status word: 0, or the SO101_ERR_* a kernel recorded (bounded waits). Synchronous:
 * reads a device variable. so101_clear_device_status resets it. */
SO101_API int so101_device_status(void);
SO101_API int so101_clear_device_status(void);

/* so101_gemm for callers that cannot allocate device memory. No counterpart in the reference.
 * Some hosts cannot call cudaMalloc when they need a GEMM: code running inside CUDA-graph capture,
 * a real-time control loop that forbids allocation after start-up, a foreign-language runtime
 * that reaches the GPU only through this library. This entry point takes no workspace: its split-K
 * scratch (at most 8 MiB of partials and 4096 tile tickets) is a file-scope device array that
 * every GPU loading the library holds until the process exits. Problems whose split-K plan needs
 * more return SO101_ERR_WORKSPACE. It allocates nothing and frees nothing; the tickets are
 * cleared on the stream before each launch. The first call on a device looks the array's device
 * address up (cudaGetSymbolAddress, with that device current): make that first call before any
 * stream capture. The address is kept beside the device's current context and looked up again
 * when that context changes (after cudaDeviceReset), so make the first call after a reset outside
 * capture too. All calls share the one array, so calls that overlap on the GPU (other streams,
 * other host threads) race; keep them ordered on one stream. */
SO101_API int so101_gemm_static(int a_type, const void* x, int64_t ldx, const void* w, int64_t ldw,
                                void* y, int64_t ldy, int y_type, int64_t M, int64_t N, int64_t K,
                                const so101_epilogue* epi, const so101_gemm_config* cfg,
                                cudaStream_t stream);

/* Programmatic dependent launch for the GEMM kernels (0 off, default; 1 on): each GEMM may start
 * streaming its weights while the previous kernel on the stream drains. */
SO101_API int so101_set_pdl(int enable);

/* ----------------------------------------------------------------- persistent expert step
 * The action expert's layers for one denoising step of ONE observation (rows <= 64 action rows)
 * as a single cooperative kernel: per layer RMSNorm -> q|k|v (RoPE on k, k/v written into the
 * cache rows [prefix_len, prefix_len + rows)) -> attention -> o + residual -> RMSNorm -> SwiGLU
 * gate/up -> down + residual, with grid barriers between the phases. It replaces the chain of
 * per-op launches the reference's TritonPath.velocity makes for the 16 expert layers
 * (pkg/model/smolvla_triton.py:106-130, the loop over layers); the reference has no fused
 * counterpart. Requirements: head_dim 64, n_layers <= 16, exp_dim and mlp_dim multiples of 8,
 * every pointer 16-byte aligned, bf16 weights, fp32 norm weights, fp32 e. */
typedef struct so101_expert_layer {
  const void* w_attn;     /* self: [q; k; v] rows (q_dim + 2 kv_dim) x exp_dim; cross: q rows q_dim x exp_dim */
  const void* w_o;        /* exp_dim x q_dim */
  const void* w_gate_up;  /* 2 mlp_dim x exp_dim: gate rows, then up rows */
  const void* w_down;     /* exp_dim x mlp_dim */
  const float* ln_in;     /* exp_dim */
  const float* ln_post;   /* exp_dim */
  void* k;                /* self: key cache, (prefix_len + rows) x kv_dim bf16; cross: prefix_len x kv_dim */
  void* v;
  int self_attn;
} so101_expert_layer;

typedef struct so101_expert_step {
  int n_layers, rows, prefix_len, exp_dim, q_dim, kv_dim, n_heads, n_kv, head_dim, mlp_dim;
  float eps;
  so101_expert_layer layer[16];
  float* e;                /* rows x exp_dim fp32 residual stream, updated in place */
  void* q;                 /* rows x q_dim bf16 scratch */
  void* attn;              /* rows x q_dim bf16 scratch */
  void* act;               /* rows x mlp_dim bf16 scratch */
  const float* cos_self;   /* rows x head_dim / 2: RoPE of the step's own positions */
  const float* sin_self;
  const float* cos_cross;  /* rows x head_dim / 2: RoPE of the cross-attention queries */
  const float* sin_cross;
  void* workspace;         /* so101_expert_step_workspace bytes; 16-byte aligned */
  int64_t workspace_bytes;
} so101_expert_step;

SO101_API int so101_expert_step_workspace(const so101_expert_step* s, int64_t* bytes);
SO101_API int so101_expert_step_run(const so101_expert_step* s, cudaStream_t stream);

/* Test hook for the bounded waits of so101_expert_step_run (no counterpart in the reference, whose
 * kernels never wait on one another). wait_limit_ns bounds each grid-barrier and split-count wait
 * (0: the default 2 s; at most 2 s); withhold_cta >= 0 makes that CTA leave at its first grid
 * barrier without arriving, so every other CTA gives up after the bound, records
 * SO101_ERR_TIMEOUT in the device status word and returns (its weight copies landed, its TMEM
 * freed); -1 turns it off. Read at each launch: eager launches only, a captured graph keeps the
 * values of its capture. */
SO101_API int so101_expert_step_test_hooks(int64_t wait_limit_ns, int withhold_cta);

/* The CUDA error string behind this thread's most recent SO101_ERR_LAUNCH ("" if none). No
 * counterpart in the reference, whose TensorRT enqueue reports a bare failure. */
SO101_API const char* so101_last_error(void);

/* Library version string and the compute capability it was built for ("sm_100a"). */
SO101_API const char* so101_version(void);

#ifdef __cplusplus
}
#endif
#endif /* SO101_B200_H */
