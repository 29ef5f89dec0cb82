/*
 * joyomni_b200.h -- C ABI of the B200-native (sm_100a) joyomni_ops hot path.
 *
 * Every entry point takes plain device pointers, element counts, element
 * strides (in elements, not bytes), a dtype code and a cudaStream_t passed as
 * `void*`, and returns an int status (JO_OK == 0, negative on error).  Nothing
 * here allocates device memory but jo_ipc_alloc (the IPC-shareable buffers of
 * the copy-engine K/V gather); outputs are caller-owned.  No C++ exception
 * crosses this boundary; jo_last_error() returns the message of the last
 * failing call made on the calling host thread.
 *
 * Kernels are compiled for sm_100a only.  A call on any other device fails
 * with JO_ERR_UNSUPPORTED.
 *
 * Each declaration names the reference interface it replaces
 * (jammm/JoyAI-Video-Edit, paths relative to the reference project root).
 */
#ifndef JOYOMNI_B200_H_
#define JOYOMNI_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define JO_API __attribute__((visibility("default")))
#else
#define JO_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------- */
#define JO_OK 0
#define JO_ERR_INVALID (-1)     /* null pointer, bad option value          */
#define JO_ERR_SHAPE (-2)       /* sizes inconsistent or out of range      */
#define JO_ERR_ALIGN (-3)       /* pointer / stride alignment violated     */
#define JO_ERR_DTYPE (-4)       /* unsupported dtype code                   */
#define JO_ERR_CUDA (-5)        /* CUDA runtime / launch error              */
#define JO_ERR_UNSUPPORTED (-6) /* current device is not sm_100             */

/* ---- dtype codes ----------------------------------------------------- */
#define JO_F32 0
#define JO_F16 1
#define JO_BF16 2
#define JO_E4M3 3 /* float8_e4m3fn */

/* ---- norm codes (fused_norm_scale_shift.cu:153) ---------------------- */
#define JO_NORM_LAYER 0
#define JO_NORM_RMS 1

JO_API int jo_abi_version(void);
JO_API const char* jo_status_name(int status);
JO_API const char* jo_last_error(void);
/* Number of kernel launches issued by this library since load (all threads). */
JO_API uint64_t jo_launch_count(void);
/* Device-side faults recorded on the current device since the last call (then
 * cleared): a kernel whose bounded wait on an mbarrier expired counts one,
 * stops issuing work, frees its tensor memory and returns instead of hanging.
 * Synchronises the current device. */
JO_API int jo_device_fault_count(uint32_t* count);

/* ====================================================================== *
 *  Drop-in replacements of torch.ops.joyomni_ops.* (csrc/pybind.cpp:52-75)
 * ====================================================================== */

/* rmsnorm: out = x * rsqrt(mean(x^2) + eps) * weight, fp32 math, one rounding.
 * Replaces joyomni_ops::rmsnorm (joyomni_ops/csrc/rmsnorm.cu:107-126).
 * x/out: [rows, cols] with row strides; weight: [cols].  dtype: F32/F16/BF16. */
JO_API int jo_rmsnorm(void* out, int64_t out_row_stride, const void* x, int64_t x_row_stride,
               const void* weight, int64_t rows, int64_t cols, int dtype, float eps,
               void* stream);

/* fused_norm_scale_shift: out = Norm(x; gamma, beta) * (1 + scale) + shift.
 * Replaces joyomni_ops::fused_norm_scale_shift
 * (joyomni_ops/csrc/fused_norm_scale_shift.cu:364-403).
 * norm: JO_NORM_LAYER or JO_NORM_RMS.  gamma/beta: [cols] or NULL (beta is
 * LayerNorm-only).  scale/shift: [mod_rows, cols] with mod_rows == 1
 * (broadcast over all rows) or mod_rows == rows, row stride mod_row_stride. */
JO_API int jo_norm_scale_shift(void* out, int64_t out_row_stride, const void* x, int64_t x_row_stride,
                        const void* gamma, const void* beta, const void* scale,
                        const void* shift, int64_t mod_rows, int64_t mod_row_stride,
                        int64_t rows, int64_t cols, int norm, int dtype, float eps,
                        void* stream);

/* fused_qk_norm_rope_3d_paired (in place): per head RMSNorm(eps)*weight, then
 * interleaved-pair RoPE with bf16 cos/sin [seq_len, head_dim/2].  q, k:
 * contiguous bf16 [batch, seq_len*num_heads, head_dim]; k_pre_rope (optional)
 * receives the normalised k before rotation.  head_dim in {64, 128, 256}.
 * Replaces joyomni_ops::fused_qk_norm_rope_3d_paired
 * (joyomni_ops/csrc/fused_qknorm_rope_3d_kernel.cu:280-319). */
JO_API int jo_qk_norm_rope_3d_paired(void* q, void* k, int64_t batch, int64_t seq_len,
                              int64_t num_heads, int64_t head_dim, float eps,
                              const void* q_weight, const void* k_weight, const void* cos,
                              const void* sin, void* k_pre_rope, void* stream);

/* A [B=1, L, H, D=128] bf16 view: element (l, h, d) at ptr[l*sl + h*sh + d]. */
typedef struct jo_view4 {
  const void* ptr;
  int64_t len;      /* L */
  int64_t stride_l; /* elements */
  int64_t stride_h; /* elements */
} jo_view4;

/* fused_joint_qkv_pack: out_q = [img_q | RMSNorm(txt_q)], out_k = [cache_k |
 * img_k | RMSNorm(txt_k)], out_v = [cache_v | img_v | txt_v], all bf16
 * contiguous [1, *, heads, 128].  The text RMSNorm rounds the normalised value
 * to bf16 before the weight multiply (double rounding, as the model's RMSNorm).
 * cache_k.ptr == NULL means no cache.
 * Replaces joyomni_ops::fused_joint_qkv_pack
 * (joyomni_ops/csrc/fused_joint_qkv_pack.cu:237-342). */
JO_API int jo_joint_qkv_pack(void* out_q, void* out_k, void* out_v, jo_view4 img_q, jo_view4 img_k,
                      jo_view4 img_v, jo_view4 txt_q, jo_view4 txt_k, jo_view4 txt_v,
                      jo_view4 cache_k, jo_view4 cache_v, const void* txt_q_weight,
                      const void* txt_k_weight, int64_t heads, float eps, void* stream);

/* fused_cached_kv_pack: concatenates one or two pre-RoPE K/V segments into
 * contiguous bf16 [1, len0+len1, heads, 128] and applies interleaved RoPE to K
 * with fp32 full-width cos/sin [len0+len1, 128].  key1.ptr == NULL: one segment.
 * value0.ptr == NULL (with out_value and value1.ptr NULL): keys only, no values
 * copied (the rotation of a cache whose values stay where they are).
 * Replaces joyomni_ops::fused_cached_kv_pack
 * (joyomni_ops/csrc/fused_joint_qkv_pack.cu:344-415). */
JO_API int jo_cached_kv_pack(void* out_key, void* out_value, jo_view4 key0, jo_view4 value0,
                      jo_view4 key1, jo_view4 value1, const float* cos, const float* sin,
                      int64_t heads, void* stream);

/* sgl_per_token_quant_fp8: per row s = max(amax|x|, 1e-8) / 448 (IEEE fp32),
 * q = e4m3(clamp(x / s, -448, 448)) (IEEE division, round-to-nearest-even).
 * These are the semantics of the reference's PyTorch path
 * (deploy/xvideo/models/dit/fp8_linear.py:38-43); all-zero rows get
 * s = 1e-8/448 and q = 0.  x: F16/BF16 [rows, cols]; out_q: e4m3 [rows, cols];
 * out_s: fp32 [rows].
 * Replaces joyomni_ops::sgl_per_token_quant_fp8
 * (joyomni_ops/csrc/per_token_quant_fp8.cu:148-176). */
JO_API int jo_per_token_quant_fp8(void* out_q, int64_t q_row_stride, float* out_s, const void* x,
                           int64_t x_row_stride, int64_t rows, int64_t cols, int dtype,
                           void* stream);

/* fp8_scaled_mm: D[m,n] = out_dtype( scale_a[m] * (sum_k A[m,k]*B[k,n]) *
 * scale_b[n] (+ bias[n]) ), fp32 accumulation in tensor memory (tcgen05).
 * A: e4m3 row-major [M,K] (row stride lda); B: e4m3 column-major [K,N]
 * (element (k,n) at b[n*ldb + k]); D row-major [M,N] (row stride ldd).
 * out_dtype: JO_BF16 or JO_F16; bias (optional) has out_dtype.
 * K, lda, ldb must be multiples of 16; ldd*esize a multiple of 16 bytes.
 * Replaces joyomni_ops::fp8_scaled_mm (joyomni_ops/csrc/fp8_gemm.cu:1450-1546,
 * sm100 path :797-1170). */
JO_API int jo_fp8_scaled_mm(void* d, int64_t ldd, const void* a, int64_t lda, const void* b,
                     int64_t ldb, const float* scale_a, const float* scale_b,
                     const void* bias, int64_t m, int64_t n, int64_t k, int out_dtype,
                     void* stream);

/* FP8 GEMM with the gated residual in the epilogue:
 *   D = residual + gate[n] * ((A.B) * sB[n] * sA[m] (+ bias[n]))
 * the down-projection + gated residual of each MLP (dit.py:536-538:
 * Fp8Linear, then sgl_fused_ops.fused_add_gate = torch.addcmul(res, x, gate)) in
 * one pass: the product is not rounded to D's dtype before the residual.
 * residual [M, N] (row stride ldr), gate [N], both of D's dtype; D may alias
 * residual (same rows, same stride).  Other arguments as jo_fp8_scaled_mm. */
JO_API int jo_fp8_scaled_mm_gated_residual(void* d, int64_t ldd, const void* a, int64_t lda, const void* b,
                                           int64_t ldb, const float* scale_a, const float* scale_b, const void* bias,
                                           const void* residual, int64_t ldr, const void* gate, int64_t m, int64_t n,
                                           int64_t k, int out_dtype, void* stream);

/* The MLP's fc1 -> GELU -> per-token FP8 (dit.py:508-513: Fp8Linear, F.gelu
 * tanh, then the next Fp8Linear's per-token quantisation, fp8_linear.py:38-43):
 *   y = y_dtype(GELU_tanh(y_dtype((A.B) * sB[n] * sA[m] (+ bias[n]))))
 *   out_s[m] = max(max_n |y[m,n]|, 1e-8) / 448; out_q = e4m3(y / out_s[m])
 * GELU and the per-row amax run in the GEMM epilogue; a second kernel quantises
 * y.  q and out_s equal jo_per_token_quant_fp8 applied to
 * jo_gelu_tanh(jo_fp8_scaled_mm(...)) bit for bit.
 * y: caller workspace [M, N] of y_dtype (row stride ldy), left holding the GELU
 * output; amax: caller workspace of M uint32 (zeroed here on the stream);
 * out_q: e4m3 [M, N] (row stride ldq, a multiple of 8 bytes, >= N); out_s:
 * fp32 [M].  Other arguments as jo_fp8_scaled_mm; N > 0.  Three stream
 * operations: a memset of amax, the GEMM, the quantisation. */
JO_API int jo_fp8_scaled_mm_gelu_quant(void* out_q, int64_t ldq, float* out_s, void* y, int64_t ldy,
                                       uint32_t* amax, const void* a, int64_t lda, const void* b,
                                       int64_t ldb, const float* scale_a, const float* scale_b,
                                       const void* bias, int64_t m, int64_t n, int64_t k, int y_dtype,
                                       void* stream);

/* ====================================================================== *
 *  New fused ops on the same path (no single reference kernel)
 * ====================================================================== */

/* qkv_norm_rope_pack: one pass from the QKV projection output to packed
 * q/k/v.  qkv: bf16 [tokens, 3*heads*head_dim] (row stride qkv_row_stride),
 * laid out (K H D) as in dit.py:409-411.  q and k get per-head
 * RMSNorm(eps)*weight and interleaved RoPE with bf16 cos/sin
 * [tokens, head_dim/2] (single rounding, as
 * joyomni_ops/csrc/fused_qknorm_rope_3d_kernel.cu:200-231); v is copied.
 * Output element (h, t, d) of q/k/v is written at out[h*out_stride_h +
 * t*out_stride_t + d]: head-major [heads, tokens, D] is (tokens*D, D),
 * token-major [tokens, heads, D] is (D, heads*D).  k_pre_rope (optional,
 * same layout) receives normalised k before rotation.  head_dim in {64,128,256}.
 * Text mode (cos == sin == NULL): no rotation, and the q/k RMSNorm rounds twice
 * as the model's RMSNorm does (bf16(x*rsqrt(mean+eps)), then bf16(. * w);
 * dit.py:289-296, the text rows of fused_joint_qkv_pack.cu:59-79).
 * Replaces the chain deploy/xvideo/models/dit/dit.py:408-429 ->
 * sgl_fused_ops.py:137-168 (two .contiguous() copies + the paired kernel) and
 * the q/k/v part of fused_joint_qkv_pack. */
JO_API int jo_qkv_norm_rope_pack(void* out_q, void* out_k, void* out_v, void* k_pre_rope,
                          int64_t out_stride_h, int64_t out_stride_t, const void* qkv,
                          int64_t qkv_row_stride, int64_t tokens, int64_t heads,
                          int64_t head_dim, const void* q_weight, const void* k_weight,
                          const void* cos, const void* sin, float eps, void* stream);

/* jo_qkv_norm_rope_pack from and to host memory, pipelined: the qkv rows are
 * uploaded chunk_tokens tokens at a time on h2d_stream, each chunk is packed on
 * `stream` once its upload has landed, and its q/k/v rows are downloaded on
 * d2h_stream once packed, so both directions of the host link and the kernel
 * overlap (one cudaMemcpyAsync per chunk for the input, one per output tensor
 * per chunk; a 2-D copy for head-major outputs).  host_qkv: bf16 [tokens,
 * 3*heads*head_dim] contiguous; host_q/k/v and dev_q/k/v share one layout,
 * head-major [heads, tokens, D] (out_stride_h = tokens*D, out_stride_t = D) or
 * token-major [tokens, heads, D] (D, heads*D).  dev_qkv/dev_q/k/v: caller-owned
 * device staging of the same sizes.  Host buffers should be pinned (pageable
 * memory works but serialises the copies).  The copy streams wait for the work
 * already queued on `stream`, and `stream` waits for the last download before
 * anything queued after the call: synchronising `stream` covers the whole call.
 * h2d_stream and d2h_stream must be non-null (not the legacy default stream).
 * Replaces, for a host-resident chunk, the upload + jo_qkv_norm_rope_pack +
 * download that a caller would otherwise issue back to back on one stream. */
JO_API int jo_qkv_norm_rope_pack_host(void* host_q, void* host_k, void* host_v, int64_t out_stride_h,
                                      int64_t out_stride_t, const void* host_qkv, void* dev_q, void* dev_k,
                                      void* dev_v, void* dev_qkv, int64_t tokens, int64_t heads, int64_t head_dim,
                                      const void* q_weight, const void* k_weight, const void* cos, const void* sin,
                                      float eps, int64_t chunk_tokens, void* stream, void* h2d_stream,
                                      void* d2h_stream);

/* Merge of two partial attention outputs over disjoint key sets A and B by
 * their log-sum-exps: per (row s, head h), m = max(lA, lB),
 * out = (e^(lA-m) oA + e^(lB-m) oB) / (e^(lA-m) + e^(lB-m)), fp32 math, one
 * rounding.  oA/oB/out: bf16 or fp16 [rows, heads, head_dim] views, element
 * (s, h, d) at p[s*stride_s + h*stride_h + d]; lse_a/lse_b: fp32 natural-log
 * log-sum-exps of the scaled scores, element (h, s) at p[h*stride_h + s*stride_s].
 * Attention over [cache | chunk | text] keys (deploy/xvideo/models/dit/dit.py:
 * 154-189, 498) is the merge of the attention over the cache rows and over the
 * rest, so the cache part can run while the chunk's K/V are still being
 * gathered from the other ranks.  No single reference kernel. */
JO_API int jo_attn_merge(void* out, int64_t out_stride_s, int64_t out_stride_h, const void* o_a, int64_t a_stride_s,
                         int64_t a_stride_h, const float* lse_a, int64_t lse_a_stride_h, int64_t lse_a_stride_s,
                         const void* o_b, int64_t b_stride_s, int64_t b_stride_h, const float* lse_b,
                         int64_t lse_b_stride_h, int64_t lse_b_stride_s, int64_t rows, int64_t heads,
                         int64_t head_dim, int dtype, void* stream);

/* gated residual: out = residual + x * gate (fp32 math, one rounding); gate is
 * [gate_rows, cols] with gate_rows in {1, rows}.
 * Replaces fused_add_gate = torch.addcmul
 * (deploy/xvideo/models/dit/sgl_fused_ops.py:302-305). */
JO_API int jo_gated_residual(void* out, int64_t out_row_stride, const void* residual,
                      int64_t res_row_stride, const void* x, int64_t x_row_stride,
                      const void* gate, int64_t gate_rows, int64_t gate_row_stride,
                      int64_t rows, int64_t cols, int dtype, void* stream);

/* gated residual + Norm + modulate, one pass:
 *   h   = dtype(residual + x * gate)           (written to out_h)
 *   out = Norm(h; gamma, beta) * (1 + scale) + shift
 * Replaces dit.py:525-534 (fused_add_gate followed by fused_layernorm_modulate). */
JO_API int jo_gated_residual_norm_scale_shift(
    void* out_h, int64_t h_row_stride, void* out, int64_t out_row_stride,
    const void* residual, int64_t res_row_stride, const void* x, int64_t x_row_stride,
    const void* gate, int64_t gate_rows, int64_t gate_row_stride, const void* gamma,
    const void* beta, const void* scale, const void* shift, int64_t mod_rows,
    int64_t mod_row_stride, int64_t rows, int64_t cols, int norm, int dtype, float eps,
    void* stream);

/* GELU, tanh approximation: out = 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))).
 * Replaces F.gelu(x, approximate="tanh") (deploy/xvideo/models/dit/dit.py:87-89). */
JO_API int jo_gelu_tanh(void* out, const void* x, int64_t n, int dtype, void* stream);

/* SiLU-gated multiply: out[r, c] = silu(a[r, c]) * b[r, c] (fp32 math). */
JO_API int jo_silu_mul(void* out, int64_t out_row_stride, const void* a, int64_t a_row_stride,
                const void* b, int64_t b_row_stride, int64_t rows, int64_t cols, int dtype,
                void* stream);

/* Sinusoidal timestep embedding (the diffusers Timesteps projection used at
 * deploy/xvideo/models/dit/dit.py:574-575,614): out fp32 [batch, dim],
 * freq_i = exp(-ln(max_period) * i / (dim/2 - downscale_freq_shift)),
 * e = [sin(scale*t*f), cos(scale*t*f)], halves swapped when flip_sin_to_cos. */
JO_API int jo_timestep_embedding(float* out, const float* t, int64_t batch, int64_t dim,
                          int flip_sin_to_cos, float downscale_freq_shift, float scale,
                          float max_period, void* stream);

/* Timestep conditioning MLP, the WanTimeTextImageEmbedding timestep branch
 * (deploy/xvideo/models/dit/dit.py:574-579, 605-620; replaces Timesteps +
 * TimestepEmbedding + act_fn + time_proj, four modules and seven kernels):
 *   e = bf16(sinusoid(t)) [B, freq_dim] (flip_sin_to_cos, shift 0, max_period),
 *   s1 = bf16(silu(bf16(e @ w1^T + b1))), s2 = bf16(silu(bf16(s1 @ w2^T + b2))),
 *   vec = bf16(s2 @ w3^T + b3) [B, proj_dim].
 * w1 bf16 [dim, freq_dim], w2 [dim, dim], w3 [proj_dim, dim] row-major; biases
 * bf16 or NULL; t fp32 [B].  freq_dim, dim <= 4096, multiples of 8.
 * scratch: caller-owned device memory of >= 4 * B * dim bytes (16-byte aligned)
 * that receives s1 then s2 (bf16 [B, dim] each). */
JO_API int jo_timestep_mlp(void* vec, const float* t, int64_t batch, const void* w1, const void* b1,
                           int64_t freq_dim, int64_t dim, const void* w2, const void* b2, const void* w3,
                           const void* b3, int64_t proj_dim, void* scratch, int64_t scratch_bytes,
                           float max_period, void* stream);

/* jo_timestep_mlp with the ModulateWan table add folded into time_proj's
 * epilogue: besides vec, writes mods[t, b, :] = bf16(tables[t, :] + vec[b, :])
 * for every t < n_tables (vec rounded to bf16 first, as the module adds the bf16
 * time_proj output).  One launch serves every block and stream of a forward:
 * tables bf16 [n_tables, proj_dim] (each block's img_mod / txt_mod
 * modulate_table, [6, D] flattened), mods bf16 [n_tables, batch, proj_dim].
 * Replaces ModulateWan.forward (deploy/xvideo/models/dit/dit.py:103-116), one
 * torch add per block and stream, after the timestep branch (dit.py:574-579,
 * 605-620).  Other arguments as jo_timestep_mlp. */
JO_API int jo_timestep_mlp_modulate(void* vec, void* mods, const void* tables, int64_t n_tables, const float* t,
                                    int64_t batch, const void* w1, const void* b1, int64_t freq_dim, int64_t dim,
                                    const void* w2, const void* b2, const void* w3, const void* b3, int64_t proj_dim,
                                    void* scratch, int64_t scratch_bytes, float max_period, void* stream);

/* jo_timestep_mlp without the scratch argument, for callers that cannot
 * allocate device memory.  No counterpart in the reference.  The two bf16
 * intermediates go to a file-scope device array of 256 KB, so
 * batch * dim <= 65536 (larger sizes return JO_ERR_SHAPE); nothing in it has to
 * start at zero (every call writes s1 and s2 before reading them).  The array is
 * shared by every call on a device: calls whose kernels overlap on the GPU (other
 * streams, other threads) race on it.  The array's address is looked up with
 * cudaGetSymbolAddress on the first call on each device (with that device
 * current), and again on the first call after the device's context was
 * re-created (cudaDeviceReset); make that first call before any stream capture:
 * a lookup requested while `stream` is capturing returns JO_ERR_INVALID with a
 * message saying so.  Allocates nothing. */
JO_API int jo_timestep_mlp_noalloc(void* vec, const float* t, int64_t batch, const void* w1, const void* b1,
                                   int64_t freq_dim, int64_t dim, const void* w2, const void* b2, const void* w3,
                                   const void* b3, int64_t proj_dim, float max_period, void* stream);

/* RMSNorm -> per-token FP8 quant, one pass: y = dtype(rmsnorm(x)*w) is rounded
 * to dtype in registers, then quantised with the jo_per_token_quant_fp8
 * semantics.  Oracle: quant(_torch_rmsnorm(x, w, eps)). */
JO_API int jo_rmsnorm_quant_fp8(void* out_q, int64_t q_row_stride, float* out_s, const void* x,
                         int64_t x_row_stride, const void* weight, int64_t rows, int64_t cols,
                         int dtype, float eps, void* stream);

/* Norm + modulate -> per-token FP8 quant, one pass (the input of every
 * Fp8Linear QKV / MLP-up projection, dit.py:402-408 and :529-535 ->
 * fp8_linear.py:133-140): y = dtype(Norm(x)*(1+scale)+shift), then quantised. */
JO_API int jo_norm_scale_shift_quant_fp8(void* out_q, int64_t q_row_stride, float* out_s,
                                  const void* x, int64_t x_row_stride, const void* gamma,
                                  const void* beta, const void* scale, const void* shift,
                                  int64_t mod_rows, int64_t mod_row_stride, int64_t rows,
                                  int64_t cols, int norm, int dtype, float eps, void* stream);

/* GELU-tanh -> per-token FP8 quant, one pass: y = dtype(gelu_tanh(x)) is rounded
 * to dtype in registers, then quantised with the jo_per_token_quant_fp8
 * semantics.  Replaces the MLP's activation + the down-projection's quant
 * (deploy/xvideo/models/dit/dit.py:508-513 -> fp8_linear.py:133-140). */
JO_API int jo_gelu_quant_fp8(void* out_q, int64_t q_row_stride, float* out_s, const void* x,
                             int64_t x_row_stride, int64_t rows, int64_t cols, int dtype, void* stream);

/* gated residual + Norm + modulate -> per-token FP8 quant, one pass:
 *   h = dtype(residual + x * gate) (written to out_h),
 *   (out_q, out_s) = quant(dtype(Norm(h) * (1 + scale) + shift)).
 * Replaces dit.py:525-535 (fused_add_gate, fused_layernorm_modulate and the
 * MLP-up projection's quant). */
JO_API int jo_gated_residual_norm_scale_shift_quant_fp8(
    void* out_h, int64_t h_row_stride, void* out_q, int64_t q_row_stride, float* out_s,
    const void* residual, int64_t res_row_stride, const void* x, int64_t x_row_stride,
    const void* gate, int64_t gate_rows, int64_t gate_row_stride, const void* gamma,
    const void* beta, const void* scale, const void* shift, int64_t mod_rows,
    int64_t mod_row_stride, int64_t rows, int64_t cols, int norm, int dtype, float eps,
    void* stream);

/* ---- copy-engine K/V all-gather between the ranks of one node --------- *
 * Replaces the NCCL all_gather_into_tensor of the chunk's K/V at the attention
 * boundary of the sequence-parallel block (deploy/xvideo/models/dit/dit.py:
 * 154-189, 498; one process per GPU): every rank maps the other ranks' K/V
 * buffers over CUDA IPC and pulls their blocks with the copy engines over
 * NVLink, so no SM is taken from the attention that the gather overlaps.  The
 * host side (joyomni_ops.chain) orders the steps with two flag words per peer. */
#define JO_IPC_HANDLE_BYTES 64

/* cudaMalloc of `bytes` (a whole allocation, as IPC export requires), zeroed
 * (synchronously); jo_ipc_free releases it. */
JO_API int jo_ipc_alloc(int64_t bytes, void** ptr);
JO_API int jo_ipc_free(void* ptr);
/* The IPC handle (JO_IPC_HANDLE_BYTES bytes) of an allocation made by
 * jo_ipc_alloc, for another process on the node to open. */
JO_API int jo_ipc_handle(const void* ptr, void* handle);
/* Maps another process's allocation into the current device's context with
 * peer access (cudaIpcMemLazyEnablePeerAccess); jo_ipc_close unmaps it. */
JO_API int jo_ipc_open(const void* handle, void** ptr);
JO_API int jo_ipc_close(void* ptr);
/* One kernel on `stream`: after a system-wide fence, stores `value` with
 * release semantics into each non-null 8-byte word peer_flags[q], q < world
 * (<= 16): this rank's flag word in each peer's (mapped) flag array. */
JO_API int jo_peer_signal(void* const* peer_flags, int world, uint64_t value, void* stream);
/* One kernel on `stream`: waits until flags[q] >= value (acquire loads) for
 * every q < world other than `skip`.  Bounded: after 2 s without progress the
 * device fault counter (jo_device_fault_count) is raised and the kernel
 * returns, so a rank that never signals ends in a recorded fault. */
JO_API int jo_peer_wait(const uint64_t* flags, int world, int skip, uint64_t value, void* stream);
/* cudaMemcpyAsync of `bytes` device bytes on `stream` (a peer's mapped memory
 * as the source: a copy-engine transfer over NVLink). */
JO_API int jo_peer_copy(void* dst, const void* src, int64_t bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* JOYOMNI_B200_H_ */
