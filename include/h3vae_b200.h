/*
 * h3vae_b200.h -- C ABI of the B200-native H3 video-VAE INT8 encode/decode path.
 *
 * Every entry point takes raw device pointers, int64 sizes, an explicit CUDA
 * stream, and returns 0 on success or a negative H3B_E* status (the message is
 * available from h3b_last_error()).  No entry point allocates device memory:
 * producers that need scratch take a caller-provided workspace whose size is
 * reported by the matching *_workspace_size query.  No C++ exception crosses
 * this boundary.  Tensors are dense unless a stride argument says otherwise;
 * "NDHWC" means PyTorch's channels_last_3d layout of a logical [B,C,D,H,W].
 *
 * Citations "ref: file:line" point into fishelegs/ComfyUI-H3VAE-PyOpt 0.2.0,
 * the interface each function replaces.
 */
#ifndef H3VAE_B200_H_
#define H3VAE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* h3b_stream_t; /* == cudaStream_t */

enum {
  H3B_OK = 0,
  H3B_EINVAL = -1,      /* bad pointer / shape / stride / dtype contract  */
  H3B_EUNSUPPORTED = -2, /* geometry outside the implemented contract     */
  H3B_ECUDA = -3,       /* CUDA runtime or driver error                    */
  H3B_EDEVICE = -4      /* device-side error word set (bounded wait expired) */
};

/* ---- library / error plumbing ------------------------------------------ */

/* Message for the last failing call on this host thread ("" if none). */
const char* h3b_last_error(void);

/* ABI version (major*100 + minor). */
int h3b_abi_version(void);

/* Reads (and with clear!=0 resets) the device error word of the current
 * device.  Synchronizes the device.  *bits==0 means no kernel reported a
 * timeout or invariant failure. */
int h3b_device_error(unsigned int* bits, int clear);

/* Failure-detection probe (diagnostic; no counterpart in the reference).
 * Launches one warp that waits on an mbarrier nothing arrives at, through the
 * same bounded wait every kernel of this library uses, with the given poll
 * limit (1 .. 2^20) instead of the library-wide one.  The wait runs out, ORs
 * the barrier-timeout bit (1) into the device error word and the kernel
 * returns; the call synchronizes `stream` and returns H3B_EDEVICE when the bit
 * is set.  Nothing traps and nothing waits without a bound; the context stays
 * usable.  The bit stays set until h3b_device_error(&bits, 1) clears it. */
int h3b_probe_wait_timeout(uint32_t poll_limit, h3b_stream_t stream);

/* ---- (a4) INT8 implicit-GEMM 3-D convolution ---------------------------- */

/* Valid (unpadded) 3-D convolution of an already padded, already quantized
 * NDHWC int8 activation with packed int8 weights, int32 accumulation on the
 * tcgen05 tensor cores (TMEM accumulators), and the dequantizing epilogue
 *   out = fp16( fma(acc * x_scale, w_scale[n], bias[n]) )   (bias optional)
 * written to an NDHWC fp16 tensor with caller strides (channel stride 1).
 *   qx        int8  [B, D, H, W, C] contiguous (x_dims = {B, D, H, W, C})
 *   qw        int8  [O, kd*kh*kw*C], tap-major / channel-minor packing
 *   x_scale   fp32 scalar (per-tensor activation scale, device pointer)
 *   w_scale   fp32 [O];  bias fp16 [O] or NULL
 *   out       fp16, element strides out_strides = {sB, sD, sH, sW}
 *   residual  optional fp16 tensor with the strides of out: out = fp16(fp16(conv) + residual),
 *             the residual block's `x + h` (ref: opt/encoder_fused_norm_bias.py:140) fused in
 *   acc_out   optional int32 [B, Do, Ho, Wo, O] contiguous raw accumulators
 *   causal_zero_frames: 2 when the producer guarantees that input frames 0
 *     and 1 are exact zeros (the causal pad); the kernel then skips the
 *     temporal taps that only read them.  0 = full reduction.
 * ref: opt/encoder_int8.py:509-588 (_conv3d_from_quantized),
 *      opt/encoder_int8_pipeline.py:16-121 (SKIP_CAUSAL_ZEROS kernel) */
int h3b_conv3d_i8(const int8_t* qx, const int64_t* x_dims, const int8_t* qw, int64_t out_channels,
                  int kd, int kh, int kw, int sd, int sh, int sw, const float* x_scale,
                  const float* w_scale, const void* bias, void* out, const int64_t* out_strides,
                  const void* residual, int32_t* acc_out, int causal_zero_frames, h3b_stream_t stream);

/* fp16 valid conv3d on the tensor cores (tcgen05 kind::f16, fp32 accumulate):
 * the encoder/decoder convolutions outside the INT8 scope -- stride-2
 * downsample convs, 1x1x1 shortcuts, conv_out, the decoder's upsampling convs.
 *   x         fp16 NDHWC contiguous [B, D, H, W, C] (already padded), C % 64 == 0
 *   x_dims    {B, D, H, W, C}
 *   w         fp16 [O, kd*kh*kw*C] tap-major, channel-minor
 *   strides   1 or 2 per axis (a stride-2 conv reads every other pixel through
 *             TMA element strides)
 *   bias      fp16 [O] or NULL: out = fp16(acc + bias) with an fp32 accumulator
 *   out       fp16 [B, Do, Ho, Wo, O] at out_strides {sB, sD, sH, sW} (elements)
 *   residual  optional fp16 tensor with out's strides: out = fp16(fp16(conv) + residual)
 *   causal_zero_frames: 2 when input frames 0 and 1 are the causal zero pad;
 *             taps that only read them are skipped
 * Replaces the cuDNN F.conv3d calls of the fp16 encoder/decoder path,
 * ref: opt/encoder_fused_residual_pack.py:85 (stride-2 downsample after the
 *      residual pack), opt/encoder_fused_batched_norm.py:83,94,96 (suffix
 *      convs), opt/encoder_internal_padding.py:34 (padded causal conv) */
int h3b_conv3d_f16(const void* x, const int64_t* x_dims, const void* w, int64_t out_channels,
                   int kd, int kh, int kw, int sd, int sh, int sw, const void* bias, void* out,
                   const int64_t* out_strides, const void* residual, int causal_zero_frames,
                   h3b_stream_t stream);

/* Encoder input conv with the pixel normalization and the causal/reflect pad
 * fused in: x fp16 logical [B, Cin, T, H, W] (element strides5, Cin <= 4) ->
 *   n = fp16(((x + 1) * 0.5 - mean[c]) / std[c])   (fp32; skipped when both
 *       normalization pointers are NULL)
 *   padded: reflect 1 in H/W (zero when H or W is 1), 2 zero frames in front
 *   out = fp16(conv3x3x3(padded, w) + bias), fp32 accumulate, NDHWC [B,T,H,W,O]
 * w: fp16 [O, 27*Cin] tap-major, channel-minor; O = 128.
 * workspace >= h3b_conv_in_workspace_size(B, T, H, W) bytes (8-byte aligned;
 * it holds the padded normalized pixels).
 * ref: h3vae_runtime.py:566-570 (_normalize_pixels) and the encoder's first
 *      causal conv, opt/encoder_staged_batch.py:16-17 (EncoderPrefix.conv_in),
 *      opt/encoder_internal_padding.py:27-36 (causal padding of the conv) */
size_t h3b_conv_in_workspace_size(int64_t B, int64_t T, int64_t H, int64_t W);
int h3b_conv_in_f16(const void* x, const int64_t* dims5, const int64_t* strides5, const float* norm_mean,
                    const float* norm_std, const void* w, int64_t out_channels, const void* bias,
                    void* out, void* workspace, size_t workspace_bytes, h3b_stream_t stream);

/* Decoder latent conv-in operand: the causal 3x3x3 conv's input unrolled into
 * GEMM rows.  x fp16 logical [B, C, T, H, W] (element strides5, C % 8 == 0) ->
 * out fp16 [B*T*H*W, 27*C] (16-byte aligned), row (b, t, y, x), column
 * (kd*9 + kh*3 + kw)*C + c = x[b, c, t+kd-2, y+kh-1, x+kw-1] with the two
 * causal zero frames in front and reflect padding 1 in H/W (zero padding when
 * H or W is 1).  out times a [N, 27*C] weight (h3b_gemm_f16) is the conv.
 * ref: the decoder's first causal conv on the latent (klvae module, built by
 *      h3vae_runtime.py:218-247; not in the checkout) with the causal padding
 *      of opt/encoder_internal_padding.py:27-36 */
int h3b_im2col_causal_f16(const void* x, const int64_t* dims5, const int64_t* strides5, void* out,
                          h3b_stream_t stream);

/* Decoder output conv to RGB: 3x3x3 valid conv from C channels (C % 64 == 0,
 * C <= 256) to 3, fp32 accumulate, + bias.  The 27 taps are packed into the
 * MMA's N dimension (see conv_rgb.cu) so each input row is read once per
 * temporal tap.
 *   x         fp16 NDHWC contiguous padded [B, T+2, H+2, W+2, C]; x_dims {B, T+2, H+2, W+2, C}
 *   w_packed  fp16 [3 * 32, C]: row kd*32 + kh*9 + kw*3 + o holds W[o, :, kd, kh, kw]
 *             (rows kd*32 + 27..31 are zero)
 *   bias      fp16 [3] or NULL
 *   out       fp16 planar [B, 3, T, H, W]
 * Replaces the cuDNN F.conv3d of the decoder's last conv (the reference runs
 * the model's conv_out through cuDNN, h3vae_runtime.py:524-564 decode path) */
int h3b_conv3d_rgb_f16(const void* x, const int64_t* x_dims, const void* w_packed, const void* bias, void* out,
                       h3b_stream_t stream);

/* Per-token activation scales (one fp32 scale per spatio-temporal position;
 * BASELINE config 1 / the north_star's per-token quantisation): INT8 conv whose
 * input carries scales x_scales[B, D, H, W] for the padded positions.  Every
 * 128-channel k-block's integer partial is dequantized with the scale of the
 * input position it read: out = fp16(fma(sum_kb float(P_kb) * s_x, w_scale[o],
 * bias[o])) (+ residual as in h3b_conv3d_i8).  C % 128 == 0.  The reference's
 * encoder path is per-tensor (h3b_conv3d_i8); this is the per-token variant of
 * ref: opt/encoder_int8.py:509-588 with the per-row scales of
 * opt/int8_swiglu_fused.py:28-38 moved to the conv's input positions. */
int h3b_conv3d_i8_token(const int8_t* qx, const int64_t* x_dims, const int8_t* qw, int64_t out_channels,
                        int kd, int kh, int kw, int sd, int sh, int sw, const float* x_scales,
                        const float* w_scale, const void* bias, void* out, const int64_t* out_strides,
                        const void* residual, int causal_zero_frames, h3b_stream_t stream);

/* Per-token INT8 producer: the GroupNorm/SiLU/pad of h3b_norm_pad_quant, then
 * per padded position scale = absmax over its C channels * fp32(1/127) (0 -> 1)
 * and q = clamp(half_away(z / scale), +-127).  C in {128, 256, 512}.
 *   q       int8 NDHWC [B, D+2, H+2, W+2, C];  scales fp32 [B, D+2, H+2, W+2]
 *   workspace >= h3b_norm_workspace_size(B, C, D, H, W)
 * ref: opt/encoder_int8_norm.py:77-110 with per-position instead of per-tensor scales */
int h3b_norm_pad_quant_token(const void* x, int64_t B, int64_t C, int64_t D, int64_t H, int64_t W,
                             const void* pre_bias, const void* gamma, const void* beta, float eps, int8_t* q,
                             float* scales, void* workspace, size_t workspace_bytes, h3b_stream_t stream);

/* ---- (a2) per-tensor activation quantization ---------------------------- */

/* scale = max|x| * fp32(1/127) (0 -> 1);  q = clamp(half_away(x / scale), +-127)
 * x: fp16 logical [B,C,D,H,W] with element strides; q: int8 NDHWC contiguous.
 * workspace >= h3b_quantize_tensor_workspace_size() bytes.
 * ref: opt/encoder_int8.py:384-426 (quantize_activation_tensor) */
size_t h3b_quantize_tensor_workspace_size(void);
int h3b_quantize_tensor_i8(const void* x, const int64_t* dims5, const int64_t* strides5, int8_t* q,
                           float* scale, void* workspace, size_t workspace_bytes, h3b_stream_t stream);

/* ---- (a3) GroupNorm(32) + SiLU + reflect/causal pad producers ----------- */

/* Workspace for the per-frame GroupNorm statistics of x [B,C,D,H,W]. */
size_t h3b_norm_workspace_size(int64_t B, int64_t C, int64_t D, int64_t H, int64_t W);

/* INT8 producer.  x: fp16 NDHWC [B,D,H,W,C].  Optional pre_bias (fp16 [C])
 * is added and rounded to fp16 first.  Per (b, frame, group) statistics;
 * z = fp16(((v-mean)*rstd)*gamma+beta); s = fp16(silu(z)); reflect pad 1 in
 * H and W, two zero frames in front; per-tensor scale = max|s| * fp32(1/127);
 * q = half_away(s/scale).  Output q: int8 NDHWC [B, D+2, H+2, W+2, C].
 * ref: opt/encoder_int8_norm.py:77-110 (quantized_temporal_norm_pad),
 *      opt/encoder_int8_norm_recompute.py:11-49, opt/encoder_fused_temporal_norm.py:13-51 */
int h3b_norm_pad_quant(const void* x, int64_t B, int64_t C, int64_t D, int64_t H, int64_t W,
                       const void* pre_bias, const void* gamma, const void* beta, float eps, int8_t* q,
                       float* scale, void* workspace, size_t workspace_bytes, h3b_stream_t stream);

/* Allocation-free INT8 producer: the same computation and output as
 * h3b_norm_pad_quant, for callers that cannot allocate device memory at the
 * call site -- e.g. a host that hands the library only the input and output
 * buffers carved from its own pre-sized pool and has no allocator (and no
 * spare workspace) to offer.  The scratch is a 4 MiB static device array that
 * every GPU loading the library holds until exit; shapes whose
 * h3b_norm_workspace_size() exceeds 4 MiB are rejected with H3B_EUNSUPPORTED
 * (e.g. B=4, C=128, D=17, 256x256 needs about 1.2 MiB and fits).
 * Every call resolves the array's address on the current device
 * (cudaGetSymbolAddress; nothing is cached, so a device reset does not leave
 * a stale address); the first call on a device also loads the module there,
 * so make that first call before any stream capture.  All calls share the one
 * array, which keeps the last call's contents: calls that overlap on
 * the GPU (other streams, other host threads) race on it, so serialize them.
 * No cudaMalloc / cudaFree or allocating library routine is called.
 * No counterpart in the reference: its producer always allocates its scratch
 * through PyTorch (opt/encoder_int8_norm.py:77-110 is the computation). */
int h3b_norm_pad_quant_noalloc(const void* x, int64_t B, int64_t C, int64_t D, int64_t H, int64_t W,
                               const void* pre_bias, const void* gamma, const void* beta, float eps, int8_t* q,
                               float* scale, h3b_stream_t stream);

/* FP16 producer with the same arithmetic, writing y: fp16 NDHWC
 * [B, D+2, H+2, W+2, C] (padded) for the fp16 convolutions.
 * ref: opt/encoder_fused_temporal_norm.py:54-80 (temporal_norm_pack),
 *      opt/encoder_fused_norm_bias.py:43-99 (bias_temporal_norm_pack),
 *      opt/encoder_fused_batched_norm.py:16-73 (batched_temporal_norm_pack) */
int h3b_norm_pad_f16(const void* x, int64_t B, int64_t C, int64_t D, int64_t H, int64_t W,
                     const void* pre_bias, const void* gamma, const void* beta, float eps, void* y,
                     void* workspace, size_t workspace_bytes, h3b_stream_t stream);

/* Nearest upsampling folded into the fp16 producer: x [B,C,D,H,W] (NDHWC) is
 * read as up(x) -- spatial factor up_spatial (1 or 2), causal temporal
 * doubling when up_temporal = 1 (frame 0 once, later frames twice: D -> 2D-1)
 * -- and y = pad(silu(GN(up(x) [+ pre_bias]))) is written as fp16 NDHWC
 * [B, D'+2, H'+2, W'+2, C] without materializing up(x).  Replication leaves
 * each frame's statistics unchanged, so they come from the source frame.
 * Workspace: h3b_norm_workspace_size(B, C, D, H, W).
 * ref: the causal conv3d upsampling stages of the klvae decoder
 * (h3vae_runtime.py:542, external) fed through
 *      opt/encoder_fused_temporal_norm.py:54-80 (norm/pack arithmetic) */
int h3b_upsample_norm_pad_f16(const void* x, int64_t B, int64_t C, int64_t D, int64_t H, int64_t W, int up_spatial,
                              int up_temporal, const void* pre_bias, const void* gamma, const void* beta, float eps,
                              void* y, void* workspace, size_t workspace_bytes, h3b_stream_t stream);

/* ---- (a6) residual + bias + downsample pad pack ------------------------- */

/* y = fp16(r + (x + bias)) computed in fp32; right/bottom reflect pad +1,
 * two zero frames in front.  x, r: fp16 NDHWC [B,D,H,W,C]; y: fp16 NDHWC
 * [B, D+2, H+1, W+1, C].
 * ref: opt/encoder_fused_residual_pack.py:13-50 (residual_downsample_pack) */
int h3b_residual_pack(const void* x, const void* r, const void* bias, int64_t B, int64_t C, int64_t D,
                      int64_t H, int64_t W, void* y, h3b_stream_t stream);

/* ---- (a9) INT8 GEMM family (decoder linears) ----------------------------- */

/* out[m, n] = fp16( fma(acc[m,n] * a_scale[m], w_scale[n], bias[n]) )
 * qa int8 [M,K] (row stride K), qw int8 [N,K], a_scale fp32 [M], w_scale fp32
 * [N], bias fp16 [N] or NULL, out fp16 with row stride ldo.  K % 16 == 0.
 * acc_out: optional int32 [M,N] raw accumulators.
 * ref: opt/int8_swiglu_fused.py:78-107 (prequantized_linear, the CK
 *      cutlass_int8_dequant contract restated at opt/int8_ffn_up_fused.py:78-84) */
int h3b_gemm_i8(const int8_t* qa, const float* a_scale, const int8_t* qw, const float* w_scale,
                const void* bias, int64_t M, int64_t N, int64_t K, void* out, int64_t ldo,
                int32_t* acc_out, h3b_stream_t stream);

/* Attention-out GEMM with the residual and the RMS statistics of the next
 * norm fused into its epilogue.  Per element of row m, column n:
 *   a   = fp16( fma(acc * a_scale[m], w_scale[n], bias[n]) )   (the linear)
 *   raw = fma(a, gate[n], x[m, n]);   h[m, n] = fp16(raw)
 * h is written instead of a (row stride ldh; h may alias x: every element is
 * read before it is written, by the same thread), and the sum of raw^2 (h^2
 * with round_stats) over each half of each 128-column tile goes to
 * row_sumsq[m, 0 .. h3b_gemm_i8_residual_parts(N)) (fp32, caller-provided).
 * h3b_rms_quant_parts then finishes the norm and the row quantization without
 * reading a.  ref: opt/int8_attention_out.py (out_linear: prequantized_linear,
 * opt/int8_swiglu_fused.py:78-107) followed by opt/int8_norm_quant.py:23-70
 * (residual_quant, the residual + RMSNorm + row quantization of norm2) */
int64_t h3b_gemm_i8_residual_parts(int64_t N);
int h3b_gemm_i8_residual(const int8_t* qa, const float* a_scale, const int8_t* qw, const float* w_scale,
                         const void* bias, int64_t M, int64_t N, int64_t K, const void* x, const void* gate,
                         int round_stats, void* h, int64_t ldh, float* row_sumsq, h3b_stream_t stream);

/* The rest of residual_quant for an h and its partial sums from
 * h3b_gemm_i8_residual: inv = rsqrt(sum of the row's `parts` partials / K +
 * eps) (summed in index order), act = fp16(h * inv * w), CK row quantization
 * -> q int8 [M,K], s fp32 [M]; norm_out (fp16 act) optional.
 * ref: opt/int8_norm_quant.py:23-44 (from the inv step on) */
int h3b_rms_quant_parts(const void* h, const float* row_sumsq, int64_t parts, const void* w, int64_t M, int64_t K,
                        float eps, int8_t* q, float* s, void* norm_out, h3b_stream_t stream);

/* FFN-up GEMM with the SwiGLU epilogue.  qw is the unmodified [2F, K] weight
 * (rows 0..F-1 gate, F..2F-1 up); per column j:
 *   g = fp16(fma(acc_g*s, ws[j], b[j])), u = fp16(fma(acc_u*s, ws[F+j], b[F+j]))
 *   act[m, j] = fp16( g / (1 + exp(-g)) * u )
 * ref: opt/int8_ffn_up_fused.py:51-90 (up_swiglu) */
int h3b_gemm_i8_swiglu(const int8_t* qa, const float* a_scale, const int8_t* qw, const float* w_scale,
                       const void* bias, int64_t M, int64_t F, int64_t K, void* act, h3b_stream_t stream);

/* fp16 decoder profile (decode_fusions without int8_decode): the same tcgen05
 * GEMM with fp16 operands (kind::f16, fp32 accumulate).
 *   h3b_gemm_f16:        out[m, n] = fp16(acc[m,n] + bias[n])
 *   h3b_gemm_f16_swiglu: g = fp16(acc_g + b[j]), u = fp16(acc_u + b[F+j]),
 *                        act[m, j] = fp16( g / (1 + exp(-g)) * u ) in fp32
 * a fp16 [M,K] (row stride K), w fp16 [N,K] (SwiGLU: [2F,K], rows 0..F-1 gate,
 * F..2F-1 up), bias fp16 or NULL, out fp16 with row stride ldo (SwiGLU: F).
 * K % 8 == 0, a and w 16-byte aligned.
 * ref: opt/fp16_swiglu_gemm.py:20-47 (w1_swiglu kernel: fp32 accumulate, bias,
 *      fp16 rounding of gate/up, fp32 SwiGLU); the plain fp16 linears of the
 *      same profile are the model's nn.Linear layers. */
int h3b_gemm_f16(const void* a, const void* w, const void* bias, int64_t M, int64_t N, int64_t K, void* out,
                 int64_t ldo, h3b_stream_t stream);
int h3b_gemm_f16_swiglu(const void* a, const void* w, const void* bias, int64_t M, int64_t F, int64_t K, void* act,
                        h3b_stream_t stream);

/* QKV GEMM with the fused per-head QK RMSNorm + rotary epilogue.  qw rows are
 * laid out per head as [q(64) | k(64) | v(64)] (N = heads*192).  For each
 * token m = b*tokens + t and head h:
 *   qkv = fp16(fma(acc*s, ws, bias));  q' = fp16(q * rsqrt(mean(q^2) + eps))
 *   q_out[d] = fp16(q'[d]*cos[d]) + fp16(rot(q')[d]*sin[d]) for d < R, q'[d] after
 * (same for k), v passes through.  cos/sin: fp16 [M, R], R in {0,16,32,48,64}.  q/k/v outputs are
 * fp16 [batch, heads, tokens, 64].
 * ref: opt/decoder_fused_qk_rope.py:13-54 (_qk_rope / qk_rope) fused behind
 *      opt/int8_qkv.py:33-41 (INT8 to_qkv) */
int h3b_gemm_i8_qkv_rope(const int8_t* qa, const float* a_scale, const int8_t* qw, const float* w_scale,
                         const void* bias, int64_t batch, int64_t tokens, int64_t heads, int64_t K,
                         const void* cos_t, const void* sin_t, int64_t rot_dims, float eps, void* q_out,
                         void* k_out, void* v_out, h3b_stream_t stream);

/* ---- (a12/a13) decoder row producers ------------------------------------ */

/* Row quantization (CK contract): s = max(amax*fp32(1/127), 1e-30),
 * q = clamp(rint(fp16(x / fp16(s))), -128, 127), NaN -> -128.
 * x fp16 [M,K] row stride ldx.  ref: opt/int8_ffn_up_fused.py:92-105 */
int h3b_row_quant(const void* x, int64_t M, int64_t K, int64_t ldx, int8_t* q, float* s, h3b_stream_t stream);

/* SwiGLU of [gate | up] rows then row quantization.
 * ref: opt/int8_swiglu_fused.py:22-66 (quantize_swiglu) */
int h3b_swiglu_quant(const void* x, int64_t M, int64_t K, int8_t* q, float* s, h3b_stream_t stream);

/* raw = fma(a, g, x); h = fp16(raw); inv = rsqrt(mean(stat^2) + eps) with
 * stat = round_stats ? h : raw; act = fp16(h*inv*w); row quantization of act.
 * h may alias x (in-place residual).  norm_out (fp16 act) is optional.
 * ref: opt/int8_norm_quant.py:23-70 (residual_quant),
 *      opt/int8_norm1_producer.py:29-61 (residual_norm_quant) */
int h3b_residual_rms_quant(const void* x, const void* a, const void* g, const void* w, int64_t M, int64_t K,
                           float eps, int round_stats, void* h, int8_t* q, float* s, void* norm_out,
                           h3b_stream_t stream);

/* y = fp16(x * rsqrt(mean(x^2) + eps) * gamma).  ref: opt/decoder_block0_norm.py:39-59 */
int h3b_rms_norm_f16(const void* x, const void* gamma, int64_t M, int64_t K, float eps, void* y,
                     h3b_stream_t stream);

/* RMSNorm followed by row quantization (block-0 norm1 feeding the INT8 QKV).
 * ref: opt/decoder_block0_norm.py:39-59 then opt/kitchen_int8.py:20-37 */
int h3b_rms_quant(const void* x, const void* gamma, int64_t M, int64_t K, float eps, int8_t* q, float* s,
                  h3b_stream_t stream);

/* raw = fma(o, gate, h); LayerNorm(raw) over K; y = fp16(fma(n, gamma, beta)).
 * ref: opt/decoder_final_norm.py:35-72 (final_residual_ln_w8) */
int h3b_final_residual_layernorm(const void* h, const void* o, const void* gate, const void* gamma,
                                 const void* beta, int64_t M, int64_t K, float eps, void* y,
                                 h3b_stream_t stream);

/* Standalone QK RMSNorm + rotary on a [b, n, 3*H*D] qkv tensor (D = 64),
 * writing q, k as fp16 [b, n, H, D].  ref: opt/decoder_fused_qk_rope.py:13-54 */
int h3b_qk_rope(const void* qkv, const void* cos_t, const void* sin_t, int64_t batch, int64_t tokens,
                int64_t heads, int64_t rot_dims, float eps, void* q_out, void* k_out, h3b_stream_t stream);

/* ---- (a11) attention ----------------------------------------------------- */

/* Non-causal softmax(q k^T * scale) v, fp16 in/out, fp32 softmax, head dim 64.
 * q/k/v: fp16 with element strides {batch, head, token} (dim stride 1);
 * out: fp16 with element strides {batch, head, token}.
 * ref: opt/decoder_fused_qk_rope.py:73 (perform_attention -> PyTorch SDPA) */
int h3b_attention_f16(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
                      const void* v, const int64_t* v_strides, void* out, const int64_t* out_strides,
                      int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len, float scale,
                      h3b_stream_t stream);

/* ---- (a15) pixel finalization ------------------------------------------- */

/* out = clamp(x*std[c] + mean[c], 0, 1) in fp32 without FMA, NaN preserved.
 * x: fp16 (x_is_fp16=1) or fp32 logical [B,3,T,H,W] with element strides;
 * out: fp32 contiguous.  ref: opt/fp16_finalize.py:24-54 (finalize_pixels) */
int h3b_finalize_pixels(const void* x, int x_is_fp16, const int64_t* dims5, const int64_t* strides5,
                        const float* std3, const float* mean3, float* out, h3b_stream_t stream);

/* ---- (a8, a15) overlap blend ------------------------------------------- */

/* canvas[c,t,y,x] += fp32(tile[c,t,y,x]) * weight[y,x], product and sum each
 * rounded once in fp32 (no FMA).  tile: fp16 (tile_is_fp16=1) or fp32 of
 * logical shape dims4 = {C,T,H,W} with element strides; weight: fp32 [H,W]
 * contiguous; canvas: fp32 window of the same logical shape with element
 * strides (a view into the blend canvas).  Each tile's weight map makes the
 * sum over tiles equal the reference's sequential ramp-blend and trim.
 * ref: h3vae_runtime.py:623-639 (_encode_spatial_tiled blend / trim),
 *      h3vae_runtime.py:457-477 (decoder tile tasks). */
int h3b_blend_accumulate(const void* tile, int tile_is_fp16, const int64_t* dims4, const int64_t* tile_strides4,
                         const float* weight, float* canvas, const int64_t* canvas_strides4, h3b_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* H3VAE_B200_H_ */
