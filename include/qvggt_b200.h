/*
 * qvggt_b200 -- C ABI of the B200 (sm_100a) kernels for QVGGT's quantised
 * transformer hot path.
 *
 * Every entry point takes raw device pointers, sizes and a CUDA stream
 * (cudaStream_t passed as void*; NULL = legacy default stream) and returns
 * QVGGT_OK or an error code; qvggt_last_error() gives the message of the last
 * failure on the calling thread.  Kernels are launched asynchronously on the
 * stream; nothing here synchronises.  Tensors are dense row-major unless a
 * stride argument says otherwise.  fp16 means IEEE binary16.
 *
 * Reference citations are paths inside the QVGGT repository
 * (E/ = qvggt/runtime/awq_inference_engine/csrc/).
 */
#ifndef QVGGT_B200_H
#define QVGGT_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QVGGT_OK 0
#define QVGGT_ERR_INVALID 1      /* bad shape or argument */
#define QVGGT_ERR_UNSUPPORTED 2  /* configuration the kernels do not implement */
#define QVGGT_ERR_CUDA 3         /* CUDA runtime / launch error */
#define QVGGT_ERR_TIMEOUT 4      /* a bounded device-side wait gave up */
#define QVGGT_ERR_ALIGN 5        /* pointer or stride not 16-byte aligned */

#define QVGGT_DTYPE_F16 0

/* Library version (major*10000 + minor*100 + patch). */
int qvggt_version(void);

/* Message of the last error returned on this thread ("" if none). */
const char* qvggt_last_error(void);

/* Device status word of the current device: 0, or the code of the first
 * bounded device-side wait that gave up since the last clear.  Synchronises
 * the current device.  clear != 0 resets the word to 0 afterwards. */
int qvggt_device_status(uint32_t* status_out, int clear);

/* Budget of every bounded device-side wait (default 2 s). */
int qvggt_set_wait_timeout_ns(uint64_t ns);

/* Number of kernels this library launched on this process (all devices). */
uint64_t qvggt_launch_count(void);

/* ---------------------------------------------------------------- W4A16 */

/* out[M, N] = in_feats[M, K] . deq(qweight)^T (+ bias), fp16 in / fp16 out,
 * fp32 accumulation (tcgen05, TMEM).  qweight int16 [N/4, K] in the AWQ
 * interleaved layout of pack_intweight(interleave=4, kstride=64);
 * scales / scaled_zeros fp16 [gpad, N], gpad >= K / group_size.
 * Requirements: N % 128 == 0, K % group_size == 0, group_size % 64 == 0.
 * bias may be NULL; with a bias the result is half(half(acc) + bias), the same
 * two roundings as the reference's GEMM followed by `out + self.bias`.
 * Replaces gemm_forward_cuda_new (E/quantization_new/gemm/gemm_cuda.cu:1125-1235,
 * bound at E/pybind.cpp:21) and the bias add of WQLinear.forward
 * (qvggt/runtime/awq/qmodule.py:361-367). */
int qvggt_w4a16_gemm(const void* in_feats, const void* qweight, const void* scales, const void* scaled_zeros,
                     const void* bias, void* out, int64_t M, int64_t N, int64_t K, int64_t gpad,
                     int32_t group_size, void* stream);

/* qvggt_w4a16_gemm with bf16 in_feats, scales, scaled_zeros, bias and out
 * (same qweight).  Dequantisation w = q * s + sz in one bf16x2 fma, bf16
 * operands on the tensor cores, fp32 accumulation, out = bf16(acc) (with a
 * bias: bf16(bf16(acc) + bias)).  Replaces the bf16 instantiation of
 * gemm_forward_cuda_new (E/quantization_new/gemm/gemm_cuda.cu:1146 dispatches
 * nv_bfloat16 through the same kernels; dequantize.cuh:53-90). */
int qvggt_w4a16_gemm_bf16(const void* in_feats, const void* qweight, const void* scales, const void* scaled_zeros,
                          const void* bias, void* out, int64_t M, int64_t N, int64_t K, int64_t gpad,
                          int32_t group_size, void* stream);

/* Same GEMM with a fused epilogue for the VGGT block:
 *   act == 1: out = gelu_erf(half(half(acc) + bias))          (fc1 -> GELU)
 *   resid != NULL: resid[M, ldr] += half(half(half(acc)+bias) * gamma)
 *                  (out must equal resid; LayerScale residual of proj / fc2)
 * New entry point (the reference runs these as separate PyTorch ops after
 * WQLinear.forward, qmodule.py:333-369). */
int qvggt_w4a16_linear_ex(const void* in_feats, int64_t lda, const void* qweight, const void* scales,
                          const void* scaled_zeros, const void* bias, void* out, int64_t ldo, int64_t M, int64_t N,
                          int64_t K, int64_t gpad, int32_t group_size, int32_t act, const void* resid,
                          int64_t ldr, const void* gamma, void* stream);

/* The qkv projection of a VGGT block with the q/k/v split, the optional per-head
 * LayerNorm (qk_norm != 0; qn_w/qn_b/kn_w/kn_b fp16 [64]) and the 2-D RoPE
 * fused into the W4A16 GEMM epilogue: y = half(half(in . deq(W)^T) + bias)
 * over N = 3*dim columns [q | k | v]; q -> q_out [M, dim] and [k | v] ->
 * kv_out [M, 2*dim], with q and k rotated exactly as qvggt_qkv_rope2d does
 * (same position rule and fp16 rounding points).  weight_kind 0 = W4A16
 * (qweight/scales/scaled_zeros/gpad/group_size), 1 = dense fp16 [N, K] in
 * `qweight` (scales ignored).  New entry point (the reference model runs the
 * split and RoPE in PyTorch after WQLinear.forward). */
int qvggt_qkv_rope_linear(const void* in_feats, int32_t weight_kind, const void* qweight, const void* scales,
                          const void* scaled_zeros, int64_t gpad, int32_t group_size, const void* bias, void* q_out,
                          void* kv_out, int64_t M, int64_t K, int32_t dim, int64_t token_offset,
                          int32_t tokens_per_frame, int32_t patch_start, int32_t grid_w, const void* cos_tab,
                          const void* sin_tab, int32_t max_pos, int32_t qk_norm, const void* qn_w, const void* qn_b,
                          const void* kn_w, const void* kn_b, float eps, void* stream);

/* Dense fp16 linear with the same fused epilogues (weight fp16 [N, K]); used
 * for the unquantised DINOv2 patch-embed blocks.  No reference counterpart
 * (the reference runs these layers in PyTorch). */
int qvggt_f16_linear_ex(const void* in_feats, int64_t lda, const void* weight, const void* bias, void* out,
                        int64_t ldo, int64_t M, int64_t N, int64_t K, int32_t act, const void* resid, int64_t ldr,
                        const void* gamma, void* stream);

/* Small-M linear (1 <= M <= 256 rows; N % 128 == 0, K % 64 == 0): the same
 * result and epilogues as qvggt_w4a16_linear_ex (weight_kind 0: AWQ int4
 * qweight/scales/scaled_zeros/gpad/group_size) or qvggt_f16_linear_ex
 * (weight_kind 1: fp16 weight [N, K] in `weight`, scales ignored), or
 * qvggt_w4a16_gemm_bf16 (weight_kind 2: AWQ int4 with bf16 activations,
 * scales, bias and output; act = 0 and resid = NULL only), computed
 * with the rows as the tensor-core N dimension and K split across the CTAs
 * of a thread-block cluster (partials summed on chip in a fixed order; no
 * workspace).  Replaces the small-M path of gemm_forward_cuda_new,
 * gemm_w4a16_T1 with its split-K semaphore
 * (E/quantization_new/gemm/gemm_cuda.cu:312-751, 1154-1205). */
int qvggt_small_linear(int32_t weight_kind, const void* in_feats, int64_t lda, const void* weight, const void* scales,
                       const void* scaled_zeros, int64_t gpad, int32_t group_size, const void* bias, void* out,
                       int64_t ldo, int64_t M, int64_t N, int64_t K, int32_t act, const void* resid, int64_t ldr,
                       const void* gamma, void* stream);

/* Launch plan qvggt_small_linear uses for (M, N, K) on the current device:
 * info[0] padded rows (MMA N), info[1] CTAs per cluster (K splits),
 * info[2] 64-wide k-blocks per CTA, info[3] CTAs, info[4] clusters of that
 * size the device holds at once.  Part of the same small-M replacement
 * (E/quantization_new/gemm/gemm_cuda.cu:1154-1205 picks its tiles by M). */
int qvggt_small_linear_plan(int32_t weight_kind, int64_t M, int64_t N, int64_t K, int32_t* info);

/* out[m, N] = in_feats[m, K] . deq(qweight)^T (+ bias) for 1 <= m <= 16.
 * Any group_size that is a multiple of 32 and divides K.
 * Replaces gemv_forward_cuda_new (E/quantization_new/gemv/gemv_cuda.cu:197-281,
 * bound at E/pybind.cpp:22; reference: m <= 7, group_size 128 only). */
int qvggt_w4a16_gemv(const void* in_feats, const void* qweight, const void* scales, const void* scaled_zeros,
                     const void* bias, void* out, int64_t m, int64_t N, int64_t K, int64_t gpad,
                     int32_t group_size, void* stream);

/* qvggt_w4a16_gemv with bf16 in_feats, scales, scaled_zeros, bias and out:
 * bf16 dequantisation as qvggt_w4a16_gemm_bf16, products summed in fp32,
 * out = bf16(sum) (+ bias).  Replaces the bf16 instantiation of
 * gemv_forward_cuda_new (E/quantization_new/gemv/gemv_cuda.cu:210-217, 59,
 * 130-133: the reference sums in bf16). */
int qvggt_w4a16_gemv_bf16(const void* in_feats, const void* qweight, const void* scales, const void* scaled_zeros,
                          const void* bias, void* out, int64_t m, int64_t N, int64_t K, int64_t gpad,
                          int32_t group_size, void* stream);

/* ----------------------------------------------------------------- W8A8 */

/* out[M, N] fp16 = half(float(acc) * (wscales[n] * ascales[m]))                (bias == NULL)
 *              or half(fma(float(acc) * wscales[n], ascales[m], bias[n]))      (bias != NULL)
 * acc = sum_k in[m, k] * w[n, k] in int32 (tcgen05 kind::i8, TMEM).
 * in int8 [M, K], w int8 [N, K], wscales fp16 [N], ascales fp16 [M].
 * Requirements: N % 128 == 0, K % 128 == 0.
 * Replaces w8a8_gemm_forward_cuda and w8a8_gemm_fuse_bias_forward_cuda
 * (E/w8a8/w8a8_gemm_cuda.cu:881-922 and :564-607, E/pybind.cpp:27-28). */
int qvggt_w8a8_gemm(const int8_t* in, const int8_t* w, const void* wscales, const void* ascales, const void* bias,
                    void* out, int64_t M, int64_t N, int64_t K, void* stream);

/* The W8A8 GEMM of a VGGT block with the LayerScale residual fused:
 * resid[M, N] += half(half(y) * gamma), y as in qvggt_w8a8_gemm (bias may be
 * NULL).  New entry point (the reference has no caller of its W8A8 GEMM). */
int qvggt_w8a8_gemm_residual(const int8_t* in, const int8_t* w, const void* wscales, const void* ascales,
                             const void* bias, const void* gamma, void* resid, int64_t M, int64_t N, int64_t K,
                             void* stream);

/* Raw int32 accumulators acc[M, N] of the same GEMM (for bit-exact checks).
 * No reference counterpart (the reference never exposes its accumulators). */
int qvggt_i8_gemm_i32(const int8_t* in, const int8_t* w, int32_t* acc, int64_t M, int64_t N, int64_t K,
                      void* stream);

/* Per-token dynamic int8 quantisation: scale[t] = half(amax_t / 127),
 * out = rni_sat(x * (127 / amax_t)).  in fp16 [tokens, hidden].
 * Replaces invoke_quant (E/w8a8/quantization.cu:81-96, E/pybind.cpp:29). */
int qvggt_invoke_quant(int8_t* out, const void* in, void* scale, int64_t tokens, int64_t hidden, void* stream);

/* LayerNorm (var = E[x^2] - E[x]^2) + int8 quantisation.
 * per_token != 0: out = rni_sat(ln * 127 / amax), scale_io[t] = half(amax/127)
 *   (amax over fp16-rounded ln, floor half(1e-6)); beta used.
 * per_token == 0: out = rni_sat(half(ln) * scale_io[0]) with scale_io a
 *   per-tensor fp16 input; beta ignored (the reference passes none).
 * Replaces rms_norm_general (E/w8a8/layernorm.cu:155-191, E/pybind.cpp:30-32). */
int qvggt_layernorm_quant(int8_t* out, const void* in, const void* gamma, const void* beta, void* scale_io,
                          int64_t tokens, int64_t hidden, float eps, int32_t per_token, void* stream);

/* tmp = gelu_tanh(in) in fp16 arithmetic; scale[t] = half(amax_t / 127) with
 * the reference's |t| rule (t > 1e-4 ? t : -t); out = rni_sat(half(127/amax) * tmp).
 * Replaces gelu_and_quant (E/w8a8/act.cu:77-90, E/pybind.cpp:36). */
int qvggt_gelu_quant(int8_t* out, const void* in, void* scale, void* tmp, int64_t tokens, int64_t d, void* stream);

/* ---------------------------------------------------------------- norms */

/* out = LayerNorm(in) * gamma + beta, fp16 in/out, fp32 statistics
 * (two-pass mean / variance).  rows of `hidden` (multiple of 256, <= 8192).
 * New entry point: the VGGT pre-norm (nn.LayerNorm, run by PyTorch in the
 * reference model). */
int qvggt_layernorm(const void* in, const void* gamma, const void* beta, void* out, int64_t tokens, int64_t hidden,
                    float eps, void* stream);

/* ----------------------------------------------------------------- RoPE */

/* Reference rotate-half RoPE with explicit per-(b, s) angles:
 * in [s, b, h, d] with element strides in_strides[4], freqs fp32 [b, s, d2],
 * out [s, b, h, d] with element strides out_strides[4]; dims >= d2 copied.
 * Replaces fused_rope_with_pos_forward_func (E/rope_new/fused_rope_with_pos.cu:122-164,
 * E/pybind.cpp:26); the caller allocates `out` with the strides it wants. */
int qvggt_rope_with_pos(const void* in, const float* freqs, void* out, int64_t s, int64_t b, int64_t h, int64_t d,
                        int64_t d2, const int64_t* in_strides, const int64_t* out_strides, void* stream);

/* VGGT 2-D RoPE fused with the q/k/v split of the qkv projection output.
 * qkv fp16 [T, 3*H*64] (token-major, [q | k | v], head-major inside each);
 * q_out [T, H*64] (roped), kv_out [T, 2*H*64] ([k roped | v]).
 * Token t's position: p = (t + token_offset) % tokens_per_frame; p < patch_start
 * -> (0, 0) else ((p-patch_start)/grid_w + 1, (p-patch_start)%grid_w + 1).
 * cos_tab / sin_tab fp16 [max_pos, 32] (the per-half tables of the model).
 * qk_norm != 0 applies LayerNorm over each head's 64 dims to q and k first
 * (weights qn_w/qn_b/kn_w/kn_b fp16 [64]).  New entry point. */
int qvggt_qkv_rope2d(const void* qkv, void* q_out, void* kv_out, int64_t T, int32_t heads, int64_t token_offset,
                     int32_t tokens_per_frame, int32_t patch_start, int32_t grid_w, const void* cos_tab,
                     const void* sin_tab, int32_t max_pos, int32_t qk_norm, const void* qn_w, const void* qn_b,
                     const void* kn_w, const void* kn_b, float eps, void* stream);

/* ------------------------------------------------------------ attention */

/* Flash attention, head_dim 64, non-causal, softmax(q k^T / 8) v, tcgen05.
 * Token-major layouts: q [batches*Lq rows, q_stride] with head h at column
 * h*64; k / v rows of kv_stride elements, head h at k_col0 + h*64 and
 * v_col0 + h*64; out [batches*Lq, o_stride], head h at column h*64.
 * Batch b covers q rows [b*Lq, (b+1)*Lq) and kv rows [b*Lkv, (b+1)*Lkv).
 * Strides are in elements and must be multiples of 8.
 * New entry point (the reference model runs PyTorch SDPA). */
int qvggt_attention(const void* q, int64_t q_stride, const void* kv, int64_t kv_stride, int64_t k_col0,
                    int64_t v_col0, void* out, int64_t o_stride, int64_t batches, int64_t Lq, int64_t Lkv,
                    int32_t heads, void* stream);

/* qvggt_attention over a chosen subset of each batch's keys, in pieces that
 * merge exactly (the frame-sharded global block of the aggregator: a rank
 * attends to its own K/V rows while the all-gather of the other ranks' rows is
 * in flight, then to those rows, and the two results are merged).
 *
 * Keys: rows [seg0_start, seg0_start + seg0_len) and
 * [seg1_start, seg1_start + seg1_len) of each batch's Lkv rows (seg1_len may
 * be 0; seg0_len > 0).
 * splits: 1..4 CTAs share each (batch, head, 256-query block), each over a
 * consecutive part of the keys; their results are merged on the device by the
 * last of them to finish (no CTA waits for another).  splits > 1 needs
 * `scratch` of qvggt_attention_scratch_bytes() bytes (16-byte aligned); its
 * first bytes are cleared on `stream` before the launch, so calls on one
 * stream may share it, calls that may overlap on the GPU may not.
 * lse (fp32 [batches][heads][Lq]) holds ln(sum_k exp(q.k / 8)) of each row:
 *   lse_mode 0: not used;  1: written;  2: `out` and `lse` hold the result of
 *   an earlier call over other keys of the same rows, which is merged with
 *   this call's; both are overwritten with the merged result.
 * qvggt_attention_plan() gives the split count the library would choose for a
 * shape on the current device (fewest waves of CTAs over its SMs) and the
 * scratch it needs.
 * New entry points (the reference model runs PyTorch SDPA). */
int qvggt_attention_ex(const void* q, int64_t q_stride, const void* kv, int64_t kv_stride, int64_t k_col0,
                       int64_t v_col0, void* out, int64_t o_stride, int64_t batches, int64_t Lq, int64_t Lkv,
                       int64_t seg0_start, int64_t seg0_len, int64_t seg1_start, int64_t seg1_len, int32_t heads,
                       int32_t splits, int32_t lse_mode, float* lse, void* scratch, int64_t scratch_bytes,
                       void* stream);
int qvggt_attention_plan(int64_t batches, int64_t Lq, int64_t keys, int32_t heads, int32_t* splits,
                         int64_t* scratch_bytes);
int qvggt_attention_scratch_bytes(int64_t batches, int64_t Lq, int32_t heads, int32_t splits,
                                  int64_t* scratch_bytes);

/* qvggt_attention_ex over all keys (lse_mode 0) with `splits` (1..4) split-KV
 * CTAs, for callers that cannot allocate device memory: it allocates nothing.
 * Its scratch is a fixed 64 MiB array in the library's device memory, present
 * on every GPU that loads the library until the process exits; a shape whose
 * scratch (qvggt_attention_scratch_bytes) exceeds 64 MiB is rejected with
 * QVGGT_ERR_UNSUPPORTED.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress, with that device current); make that
 * first call before any stream capture.  All calls on a device share the array
 * and leave their data in it; each call clears the counters it needs on
 * `stream` before its kernel, so calls in order on one stream are safe, and
 * calls whose kernels may run at the same time on the GPU (other streams,
 * other host threads) race.  Same arguments and results as qvggt_attention_ex.
 * No counterpart in the reference. */
int qvggt_attention_split_static(const void* q, int64_t q_stride, const void* kv, int64_t kv_stride,
                                 int64_t k_col0, int64_t v_col0, void* out, int64_t o_stride, int64_t batches,
                                 int64_t Lq, int64_t Lkv, int32_t heads, int32_t splits, void* stream);

/* Attention over short sequences with head_dim 128 (the camera-head trunk:
 * 16 heads x 128 over the S <= 256 camera tokens of each batch),
 * softmax(q k^T / sqrt(128)) v on CUDA cores in fp32.  Same token-major
 * layout as qvggt_attention with heads at column h*128 and Lq = Lkv = L.
 * New entry point (the reference model runs PyTorch SDPA in its camera head,
 * loader.py:338-344 quantises the trunk's linears around it). */
int qvggt_attention_small(const void* q, int64_t q_stride, const void* kv, int64_t kv_stride, int64_t k_col0,
                          int64_t v_col0, void* out, int64_t o_stride, int64_t batches, int64_t L, int32_t heads,
                          void* stream);

/* ---------------------------------------------------------- patch embed */

/* images fp16 [S, 3, H, W] (pixels in [0, 1]) -> patches fp16
 * [S*(H/patch)*(W/patch), k_pad]: column c*patch^2 + ky*patch + kx holds
 * half(half(x - mean[c]) / std[c]), columns >= 3*patch^2 are zero.  Turns the
 * patch-embed convolution of the DINOv2 front into a GEMM.  No reference
 * counterpart (the model runs the convolution in PyTorch). */
int qvggt_patchify(const void* images, void* out, int64_t S, int32_t H, int32_t W, int32_t patch, int32_t k_pad,
                   const float* mean3, const float* std3, void* stream);

/* out [S, P, C]: rows p < n_special of frame f copy specials[set][p] (set = 1
 * for every frame whose global index f + frame_offset > 0 when two_sets != 0,
 * else 0); rows p >= n_special copy src row
 * f*src_rows_per_frame + src_row_offset + (p - n_special).  If pos != NULL,
 * pos[p] (fp16 [P, C]) is added (one fp16 rounding).  Builds the DINOv2 token
 * sequence (cls / registers / patches + position embedding) and the aggregator
 * sequence (camera / registers / patch tokens).  No reference counterpart. */
int qvggt_assemble_tokens(const void* src, int64_t src_rows_per_frame, int64_t src_row_offset, const void* specials,
                          int32_t n_special, int32_t two_sets, const void* pos, void* out, int64_t S, int32_t P,
                          int32_t C, int64_t frame_offset, void* stream);

/* Kernel configuration of every large-M GEMM entry point (W4A16, dense fp16,
 * int8): 0 = chosen per shape (default: the configuration with the fewest
 * estimated cycles, waves of tiles over the SMs x time per tile), 1 = CTA
 * pairs with 256 x 256 tiles, 2 = one SM per 128 x 256 tile, 3 = one SM per
 * 128 x 128 tile.  A forced configuration a shape cannot use falls back to
 * the automatic choice.  Process-wide; for tuning and tests.  The
 * QVGGT_GEMM_CONFIG environment variable sets the initial value.  No
 * reference counterpart (the reference picks its GEMM by M alone,
 * gemm_cuda.cu:1154-1232). */
int qvggt_set_gemm_config(int32_t cfg);

/* ------------------------------------------------------- post-processing */

/* Camera matrices from VGGT's pose encoding "absT_quaR_FoV": pose_enc fp32
 * [n, 9] = (t, quaternion x y z w, fov_h, fov_w) -> extrinsics fp32 [n, 3, 4] =
 * [R | t] and, when `intrinsics` is not NULL, intrinsics fp32 [n, 3, 3]
 * (fx = (w/2) / tan(fov_w/2), fy = (h/2) / tan(fov_h/2), fields of view
 * clamped to [1e-6, pi - 1e-6], focal lengths to [1, 1e6], principal point
 * (w/2, h/2)).  Replaces qvggt/common/pose_enc.py:7-65
 * (pose_encoding_to_extri_intri) and rotation.py:4-25 (quat_to_mat). */
int qvggt_pose_encoding_to_extri_intri(const float* pose_enc, int64_t n, int32_t image_h, int32_t image_w,
                                        float* extrinsics, float* intrinsics, void* stream);

/* World points from depth maps: depth fp32 [S, H, W] (16-byte aligned),
 * extrinsics fp32 [S, 3, 4], intrinsics fp32 [S, 3, 3] -> world_points fp32
 * [S, H, W, 3] (16-byte aligned) = R^T (cam - t) with cam = ((u - cu) d / fu,
 * (v - cv) d / fv, d), fu and fv floored at 1e-6; every pixel is converted
 * (no mask), as in the reference.  Replaces qvggt/common/geometry.py:43-96
 * (unproject_depth_map_to_point_map, computed there in numpy on the host). */
int qvggt_unproject_depth(const float* depth, int64_t S, int32_t H, int32_t W, const float* extrinsics,
                          const float* intrinsics, float* world_points, void* stream);

/* ------------------------------------------------------------- self-test */

/* Runs one kernel whose bounded wait waits on an mbarrier nothing arrives on;
 * it must give up after the wait budget and report QVGGT_ERR_TIMEOUT through
 * the status word (which this call clears).  Synchronises.  For tests of the
 * failure path; faults nothing. */
int qvggt_selftest_wait_timeout(uint64_t timeout_ns, uint32_t* status_out);

#ifdef __cplusplus
}
#endif

#endif /* QVGGT_B200_H */
