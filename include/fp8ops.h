/*
 * fp8ops.h — C ABI of the B200 (sm_100a) FP8 hot path.
 *
 * Every entry point takes raw device pointers, sizes and a CUDA stream, enqueues
 * its kernels on that stream and returns a status code.  None of them allocates
 * device memory or synchronises: buffers (outputs and workspaces) are owned by
 * the caller, so the calls can be captured in CUDA graphs.  Scales are fp32
 * scalars in device memory (the reference keeps them as 0-d CUDA tensors and
 * never reads them on the host).
 *
 * FP8 tensors are float8_e4m3fn bytes.  "scale" is the dequantisation scale
 * s = amax / 448 of the reference (x ~= q * s).
 *
 * Reference interfaces (fattorib/diffusion-profiled, diffusion/fp8_kernels.py)
 * that each entry point replaces are cited per function.  The reference is
 * Python + Triton; its "FFI" is the Python call into the Triton launcher, so the
 * binding a maintainer adds is a ctypes layer (diffusion-profiled_b200/fp8_b200/
 * _lib.py is that layer: one restype / argtypes entry per function below).
 *
 * Delayed-scaling casts fold their scale in the last CTA of the launch: each such
 * launch takes the next of 8192 ticket counters (per device) in rotation and
 * leaves it at zero.  Launches that can run at the same time (on different
 * streams) must be fewer than 8192 folding launches apart in issue order.
 */
#ifndef FP8OPS_H_
#define FP8OPS_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ABI-compatible with cudaStream_t / CUstream. NULL = legacy default stream. */
typedef struct CUstream_st* fp8_stream_t;

/* Status codes. */
#define FP8_OK 0
#define FP8_ERR_INVALID_ARGUMENT 1 /* bad pointer, size, alignment or shape      */
#define FP8_ERR_UNSUPPORTED 2      /* shape outside what the kernels implement    */
#define FP8_ERR_CUDA 3             /* a CUDA runtime / driver call failed          */
#define FP8_ERR_WORKSPACE 4        /* workspace too small                          */

/* Epilogues of the forward GEMM / conv. */
#define FP8_EPILOGUE_NONE 0      /* y = acc * sa * sb                              */
#define FP8_EPILOGUE_BIAS 1      /* y = acc * sa * sb + bias[n]                    */
#define FP8_EPILOGUE_BIAS_SILU 2 /* y = silu(acc * sa * sb + bias[n])              */

/* Version of this ABI (incremented on any signature change). */
int fp8_abi_version(void);

/* Copies the calling thread's last error message (NUL-terminated, truncated to
 * len) into buf and returns the status code of that error (FP8_OK if none). */
int fp8_last_error(char* buf, size_t len);

/* Reads and clears the device-side error word of the current device (kernels
 * record a code there when a bounded wait inside them times out).  Synchronises
 * `stream`.  *code_out = 0 means no device error was recorded. */
int fp8_device_error(int* code_out, fp8_stream_t stream);

/* Failure-path self test (no counterpart in the reference, which has no
 * bounded waits).  Launches one CTA that waits, through the same bounded
 * mbarrier wait every kernel of this library uses, on a barrier that nothing
 * arrives on, with a limit of limit_ns (0 < limit_ns <= 1e9) instead of the
 * kernels' 2 s.  The wait gives up, records error code 199 in the device error
 * word and the kernel returns; *returned (device int) becomes 1.  The context
 * stays usable.  Read the code with fp8_device_error. */
int fp8_selftest_wait_timeout(uint64_t limit_ns, int* returned, fp8_stream_t stream);

/* Number of streaming multiprocessors of the current device (launch sizing). */
int fp8_sm_count(int* out);

/* Number of kernels this library has launched in this process (host-side
 * launches; replays of a captured CUDA graph are not counted). */
int fp8_kernel_launch_count(unsigned long long* out);

/* ------------------------------------------------------------------ quantize */

/* Bytes of fp32 workspace the quantize calls need for n elements. */
size_t fp8_quantize_workspace_bytes(int64_t n);

/* Current (just-in-time) per-tensor scaling of n bf16 values:
 *   *scale_out = amax>0 ? amax/448 : 1;  q = e4m3(clamp(x / *scale_out, +-448)).
 * Replaces quantize_fp8 (fp8_kernels.py:559-601) and its kernels
 * partial_amax_kernel (:54-64), finalize_amax_kernel (:90-102) and
 * quantize_fp8_kernel (:105-120).  The element order of x is irrelevant (the
 * reference also treats the tensor as flat memory); q has the same order. */
int fp8_quantize_current(const void* x_bf16, void* q_e4m3, float* scale_out, void* workspace,
                         size_t workspace_bytes, int64_t n, fp8_stream_t stream);

/* Allocation-free variant of fp8_quantize_current (same results, bit for bit).
 * No counterpart in the reference: it exists for callers that cannot allocate
 * device memory, e.g. a runtime whose device memory is entirely owned by
 * another allocator (a host framework that reserves the whole device at start),
 * or a foreign-language host reached over FFI that has no device allocator of
 * its own.  It takes no workspace: its scratch (the per-CTA amax partials) is a
 * static 8 KB array inside this library, one per device, held until the process
 * exits.  Limit: that array has 2048 slots; a call whose amax pass would need
 * more (a device with more than 256 SMs) is rejected with FP8_ERR_UNSUPPORTED.
 * The first call on a device looks up the array's device address; make that
 * first call before any stream capture.  All calls share the one array: calls
 * that overlap on the GPU (different streams, no ordering between them) race
 * and may produce wrong scales; serialise them. */
int fp8_quantize_current_noalloc(const void* x_bf16, void* q_e4m3, float* scale_out, int64_t n,
                                 fp8_stream_t stream);

/* Workspace bytes of fp8_quantize_current_multi for `count` tensors. */
size_t fp8_quantize_multi_workspace_bytes(int count);

/* fp8_quantize_current on `count` (1..4) tensors at once: one amax launch and one
 * cast launch stream all of them, each tensor keeps its own amax and scale and
 * gets exactly the bytes fp8_quantize_current would write.  The reference
 * quantizes a conv's input and weight back to back (fp8_kernels.py:642-650 ->
 * quantize_fp8 :559-601, twice); this is that pair in two launches instead of
 * four, or in one where the shared-memory-resident form applies
 * (fp8_set_quantize_resident).  x[i], q[i], scale_out[i], n[i] as for
 * fp8_quantize_current. */
int fp8_quantize_current_multi(int count, const void* const* x_bf16, void* const* q_e4m3, float* const* scale_out,
                               const int64_t* n, void* workspace, size_t workspace_bytes, fp8_stream_t stream);

/* Delayed scaling: q = e4m3(clamp(x / *prev_scale, +-448)) and
 * *scale_curr_out = scale of x's own amax.
 * Replaces quantize_fp8_delayed (fp8_kernels.py:518-556) and
 * partial_amax_kernel_delayed (:69-87) + finalize_amax_kernel (:90-102). */
int fp8_quantize_delayed(const void* x_bf16, void* q_e4m3, const float* prev_scale, float* scale_curr_out,
                         void* workspace, size_t workspace_bytes, int64_t n, fp8_stream_t stream);

/* --------------------------------------------------------------- transposes */

/* dst[c][r] = src[r][c] for a rows x cols byte matrix.
 * Replaces transpose_fp8_2d_kernel (fp8_kernels.py:321-337). */
int fp8_transpose_2d(const void* src, void* dst, int64_t rows, int64_t cols, fp8_stream_t stream);

/* Conv weight re-layout for the data-grad: wq [Cout][3][3][Cin] (channels_last
 * [Cout,Cin,3,3]) -> wq_t [Cin][3][3][Cout], so that fp8_conv3x3_dgrad reads a
 * K-major B operand.  No reference counterpart: the reference's dX kernel
 * gathers W with strided loads (fp8_kernels.py:306-309). */
int fp8_conv_weight_transpose(const void* wq, void* wq_t, int cout, int cin, fp8_stream_t stream);

/* fp8_conv_weight_transpose of `count` (1..64) weights in one launch (Cout and
 * Cin multiples of 64, 16-byte aligned): the re-laid-out weights of every
 * data-grad of a training step, made once per step next to the batched weight
 * quantize instead of inside each fp8_conv3x3_dgrad_w call. */
int fp8_conv_weight_transpose_batch(int count, const void* const* wq, void* const* wq_t, const int* cout,
                                    const int* cin, fp8_stream_t stream);

/* ------------------------------------------------------------ 3x3 conv (pad 1) */

/* y[n,h,w,co] = epi( sum_{kh,kw,ci} xq[n,h+kh-1,w+kw-1,ci] * wq[co,kh,kw,ci] * sx * sw )
 * xq: NHWC e4m3 [B][H][W][Cin]; wq: [Cout][3][3][Cin]; y: NHWC bf16 [B][H][W][Cout];
 * bias: bf16 [Cout] (only read by the bias epilogues, else may be NULL).
 * Replaces conv2d_fwd_fp8_prequantized + conv2d_fwd_fp8_kernel
 * (fp8_kernels.py:604-639, :168-247).  Cin, Cout: multiples of 128; the width
 * must divide 128 and a 128-pixel tile must cover whole rows of one image or
 * whole images (true for every shape in SUPPORTED_UNET_SHAPES). */
int fp8_conv3x3_fwd(const void* xq, const void* wq, void* y, const float* sx, const float* sw, const void* bias,
                    int epilogue, int batch, int height, int width, int cin, int cout, fp8_stream_t stream);

/* Workspace bytes of fp8_conv3x3_dgrad_w (0 when it reads wq in place). */
size_t fp8_conv3x3_dgrad_w_workspace_bytes(int batch, int height, int width, int cin, int cout);

/* fp8_conv3x3_dgrad on the forward's weights wq [Cout][3][3][Cin]: where the
 * transposed halo kernel applies (Cout = 128 at 32x32 and 16x16) it reads wq in
 * place as an MN-major operand; otherwise it writes the [Cin][3][3][Cout]
 * re-layout into the workspace first.  Same result as fp8_conv_weight_transpose
 * followed by fp8_conv3x3_dgrad (reference fp8_kernels.py:671-709). */
int fp8_conv3x3_dgrad_w(const void* dyq, const void* wq, void* dx, const float* sdy, const float* sw, int batch,
                        int height, int width, int cin, int cout, void* workspace, size_t workspace_bytes,
                        fp8_stream_t stream);

/* dx[n,h,w,ci] = sum_{kh,kw,co} dyq[n,h+1-kh,w+1-kw,co] * wq[co,kh,kw,ci] * sdy * sw
 * dyq: NHWC e4m3 [B][H][W][Cout]; wq_t: [Cin][3][3][Cout] (fp8_conv_weight_transpose
 * of the forward's wq); dx: NHWC bf16 [B][H][W][Cin].
 * Replaces conv2d_bwd_input_fp8_prequantized + conv2d_dx_fp8_kernel
 * (fp8_kernels.py:671-709, :250-318). */
int fp8_conv3x3_dgrad(const void* dyq, const void* wq_t, void* dx, const float* sdy, const float* sw, int batch,
                      int height, int width, int cin, int cout, fp8_stream_t stream);

/* Workspace bytes of fp8_conv3x3_wgrad: one fp32 accumulator of Cout*9*Cin
 * elements (split_k does not change it; 0 for unsupported geometry). */
size_t fp8_conv3x3_wgrad_workspace_bytes(int batch, int height, int width, int cin, int cout, int split_k);

/* dw[co,kh,kw,ci] = sum_{n,h,w} dyq[n,h,w,co] * xq[n,h+kh-1,w+kw-1,ci] * sx * sdy
 * xq: NHWC e4m3 [B][H][W][Cin]; dyq: NHWC e4m3 [B][H][W][Cout]; dw: bf16
 * [Cout][3][3][Cin] (channels_last [Cout,Cin,3,3]).  Split-K over pixels
 * (split_k <= 0: the library's choice); the splits' fp32 sums are added in L2
 * into the workspace accumulator (zeroed by this call), so their order of
 * addition is not fixed.
 * Replaces conv2d_bwd_weight_fp8_prequantized (fp8_kernels.py:723-808) with
 * its transpose_fp8_2d_kernel, conv2d_dw_fp8_kernel and
 * conv2d_dw_reduce_fp8_kernel (:321-337, :385-468). */
int fp8_conv3x3_wgrad(const void* xq, const void* dyq, void* dw, const float* sx, const float* sdy, int batch,
                      int height, int width, int cin, int cout, int split_k, void* workspace,
                      size_t workspace_bytes, fp8_stream_t stream);

/* fp8_conv3x3_wgrad with dw fp32 [Cout][3][3][Cin] (16-byte aligned): the same
 * bf16 values, widened.  That is the gradient the reference's fp32 conv weight
 * receives: Conv2dFP8Specialized.backward returns the bf16 dW
 * (fp8_kernels.py:875-913) and autograd casts it to the parameter's dtype; here
 * the reduce pass writes it directly, with no separate cast launch. */
int fp8_conv3x3_wgrad_f32(const void* xq, const void* dyq, float* dw, const float* sx, const float* sdy, int batch,
                          int height, int width, int cin, int cout, int split_k, void* workspace,
                          size_t workspace_bytes, fp8_stream_t stream);

/* --------------------------------------------------------------- FP8 linear */

/* out[m,n] = epi( sum_k a[m,k] * b[n,k] * sa * sb ), a: [M][K] e4m3, b: [N][K]
 * e4m3 (the nn.Linear weight layout), out: [M][N] bf16, bias: bf16 [N].
 * No reference kernel: the reference runs these linears (unet.py:101, 171-172,
 * 331-336) in bf16; this is the new scaled FP8 GEMM.  K % 16 == 0, N % 32 == 0. */
int fp8_gemm(const void* a, const void* b, void* out, const float* sa, const float* sb, const void* bias,
             int epilogue, int64_t m, int64_t n, int64_t k, fp8_stream_t stream);

/* Workspace bytes of fp8_gemm_wgrad: one fp32 accumulator of N*K elements. */
size_t fp8_gemm_wgrad_workspace_bytes(int64_t m, int64_t n, int64_t k, int split_k);

/* dw[n,k] = sum_m dy[m,n] * x[m,k] * sdy * sx; dy: [M][N] e4m3, x: [M][K] e4m3,
 * dw: [N][K] bf16.  N, K multiples of 128.  No reference counterpart. */
int fp8_gemm_wgrad(const void* dy, const void* x, void* dw, const float* sdy, const float* sx, int64_t m,
                   int64_t n, int64_t k, int split_k, void* workspace, size_t workspace_bytes,
                   fp8_stream_t stream);

/* Tuning override for the K-major GEMM tile (bm_sub in {1,2}, bn in {64,128,256})
 * and the weight-gradient column group (g in {1,2,3}); 0 restores the built-in
 * choice.  Process-wide; meant for benchmarks and tests. */
int fp8_set_tile_override(int bm_sub, int bn, int wgrad_group);

/* Algorithm of fp8_conv3x3_fwd / fp8_conv3x3_dgrad: 0 = the library's choice
 * (for 32x32 and 16x16 images the transposed halo kernel when the reduced
 * dimension is 128 channels, else the single-CTA halo kernel; the tap-by-tap
 * GEMM for other sizes), 1 = always tap-by-tap, 2 = single-CTA halo wherever
 * it applies, 3 = CTA-pair halo where the reduced dimension is 128 channels
 * (else as 2), 4 = transposed halo where it applies (else as 2).
 * Process-wide; meant for benchmarks and tests. */
int fp8_set_conv_algo(int algo);

/* Programmatic dependent launch.  Every kernel of the library waits for the
 * previous kernel on its stream (griddepcontrol.wait) before its first global
 * memory access; a kernel launched with programmatic stream serialization can
 * therefore start, and set up shared memory, barriers and tensor memory, while
 * the previous kernel drains.  mode 0 = plain stream order (the default), 1 = the
 * attribute on the tensor-core kernels, 2 = on every kernel.  Process-wide;
 * meant for benchmarks and tests. */
int fp8_set_pdl(int mode);

/* What the delayed-scaling histories record for a tensor whose amax is 0 (an
 * all-zero weight, or the all-zero output gradient of a layer whose only path
 * back runs through FP8 convs on their first, uncalibrated call).
 * mode 0 (default): the reference's entry, the tensor's scale 1.0
 * (finalize_amax_kernel, fp8_kernels.py:90-102, stored by unet.py:84-89 and
 * fp8_kernels.py:887-889); the history max then stays >= 1.0 for the next
 * window-length calls and e4m3 flushes values below ~1e-3 of that tensor to 0.
 * mode 1: 0.0, so the tensor adds nothing to the history max (the next cast
 * uses the largest scale of the tensors that had values).  Applies to the
 * entry points that update histories on the device (the *_window calls and
 * fp8_quantize_weights_delayed); the scale outputs keep the reference value.
 * Process-wide, read when a call launches its kernels (a captured CUDA graph
 * keeps the mode it was captured with).  No counterpart in the reference. */
int fp8_set_empty_tensor_history(int mode);

/* Current-scaling quantize (fp8_quantize_current, _multi, _noalloc) of aligned
 * tensors with sizes that are multiples of 8: enable = 1 (default) runs it as one
 * cooperative launch that keeps each SM's share of the tensors in shared memory
 * between the amax and the cast (x read from memory once), where the shares fit
 * and the tensors hold at least 6 MB of bf16 (below that the two passes are
 * about as fast); enable = 0 always uses the two passes.
 * Same bytes and scales either way.  Process-wide; for benchmarks and tests. */
int fp8_set_quantize_resident(int enable);

/* Weight gradients (fp8_conv3x3_wgrad, _f32, fp8_gemm_wgrad): enable = 1 folds
 * the conversion of the fp32 split-K accumulator into the weight-gradient launch
 * (a cooperative launch whose CTAs meet at a grid barrier) when its grid fits one
 * CTA per SM; enable = 0 (default: the barrier costs more than the launch it
 * saves) converts in a second launch.  Same results either way.  Process-wide;
 * for benchmarks and tests. */
int fp8_set_wgrad_fused(int enable);

/* Tuning override for the quantize grids: CTAs per SM of the amax pass and of
 * the cast pass (1..8; 0 restores the built-in choice).  Process-wide. */
int fp8_set_quantize_override(int amax_blocks_per_sm, int cast_blocks_per_sm);

/* ---- GroupNorm + FiLM + SiLU + dropout (the activations that feed the FP8 convs).
 * No reference kernel: these replace the torch ops of the reference ResBlock,
 * norm1 -> silu (unet.py:151) and norm2 -> (scale + 1) * h + shift -> silu ->
 * dropout (unet.py:157-159), with one statistics pass and one apply pass.
 * x, dx: NHWC [n][hw][c] (channels_last), bf16 (x_fp32 = 0) or fp32 (x_fp32 = 1);
 * out, dy: NHWC bf16; all 16-byte aligned; c a multiple of 8, c <= 512,
 * c % groups == 0.  gamma, beta: fp32 [c].
 * film: nullable bf16 [n][film_ld], FiLM scale at film[i*film_ld + ch] and shift
 * at film[i*film_ld + c + ch] (the chunk of the time-embedding projection).
 * seed: nullable device int64 (dropout off when null or p == 0); element e is
 * kept when a 16-bit slice of splitmix64 of (seed, e / 4) is >= p * 65536.
 * stats: fp32 [n][2][groups] (mean, rstd), written by the forward and read by
 * the backward.  totals (backward): fp32 [n][3][c] = per sample and channel the
 * sums over pixels of df, df * z and df * xhat, where f = (scale + 1) * z + shift
 * and z = gamma * xhat + beta; the caller forms d gamma = sum_n (scale+1) * totals[2],
 * d beta = sum_n (scale+1) * totals[0], d scale = totals[1], d shift = totals[0]. */
size_t fp8_gn_workspace_bytes(int n, int hw, int c);

int fp8_gn_act_fwd(const void* x, int x_fp32, const float* gamma, const float* beta, const void* film,
                   int film_ld, const int64_t* seed, float p, float eps, float* stats, void* out, int n, int hw,
                   int c, int groups, void* workspace, size_t workspace_bytes, fp8_stream_t stream);

int fp8_gn_act_bwd(const void* x, int x_fp32, const void* dy, const float* gamma, const float* beta,
                   const void* film, int film_ld, const int64_t* seed, float p, float eps, const float* stats,
                   float* totals, void* dx, int n, int hw, int c, int groups, void* workspace,
                   size_t workspace_bytes, fp8_stream_t stream);

/* fp8_gn_act_bwd with a second gradient of x added: dx = RN(RN(dx_norm) +
 * dx_add) in x's dtype, dx_add laid out like x (16-byte aligned).  That is the
 * sum autograd forms for the input of a residual block with an identity skip,
 * read by norm1 and by the join (unet.py:151, 161), without the separate add. */
int fp8_gn_act_bwd_accumulate(const void* x, int x_fp32, const void* dy, const float* gamma, const float* beta,
                              const void* film, int film_ld, const int64_t* seed, float p, float eps,
                              const float* stats, float* totals, const void* dx_add, void* dx, int n, int hw, int c,
                              int groups, void* workspace, size_t workspace_bytes, fp8_stream_t stream);

/* fp8_gn_act_bwd for a bf16 x that is the output of a delayed-scaling FP8 conv
 * (the residual block's conv_1 before norm2, unet.py:151-159): dx (bf16) is
 * also written as e4m3 to dxq, cast with max(window[0 .. window_len)) -- which
 * goes to *scale_used_out -- and dx's own scale is stored at
 * window[*window_pos] (position kept): bit for bit what that conv's backward
 * gets from fp8_quantize_delayed_window(dx, window, window_pos, advance = 0)
 * (reference fp8_kernels.py:875-889), without reading dx again.  Workspace:
 * fp8_gn_act_bwd_quant_workspace_bytes. */
size_t fp8_gn_act_bwd_quant_workspace_bytes(int n, int hw, int c);
int fp8_gn_act_bwd_quant(const void* x, const void* dy, const float* gamma, const float* beta, const void* film,
                         int film_ld, const int64_t* seed, float p, float eps, const float* stats, float* totals,
                         void* dx, void* dxq, float* window, int window_len, int64_t* window_pos,
                         float* scale_used_out, int n, int hw, int c, int groups, void* workspace,
                         size_t workspace_bytes, fp8_stream_t stream);

/* LayerNorm over the last dimension of `tokens` rows of c channels (the
 * attention-block norm of reference unet.py:174, :187, nn.LayerNorm(C) with
 * elementwise affine): y = bf16((x - mean) * rstd * gamma + beta), rstd =
 * 1 / sqrt(biased var + eps).  The reference computes it in fp32 under autocast
 * and the qkv projection casts it to bf16; this writes the bf16 directly.
 * x is bf16 (x_fp32 = 0) or fp32; mean_rstd: fp32 [tokens][2] for the backward.
 * c % 8 == 0, c <= 1024; x, y 16-byte aligned. */
int fp8_layer_norm_fwd(const void* x, int x_fp32, const float* gamma, const float* beta, float eps, void* y_bf16,
                       float* mean_rstd, int64_t tokens, int c, fp8_stream_t stream);

/* Workspace bytes of fp8_layer_norm_bwd. */
size_t fp8_layer_norm_workspace_bytes(int64_t tokens, int c);

/* Backward of fp8_layer_norm_fwd: dx (x's dtype) from the bf16 dy, and the
 * parameter gradients dgamma = sum_t dy * xhat, dbeta = sum_t dy (fp32 [c],
 * overwritten; summed per CTA and then over CTAs in a fixed order). */
int fp8_layer_norm_bwd(const void* x, int x_fp32, const void* dy_bf16, const float* gamma, const float* mean_rstd,
                       void* dx, float* dgamma, float* dbeta, int64_t tokens, int c, void* workspace,
                       size_t workspace_bytes, fp8_stream_t stream);

/* Parameter gradients of the group-norm chain from fp8_gn_act_bwd's totals
 * [n][3c] (sums of df, df*z, df*xhat per sample and channel):
 *   dgamma[c] = sum_n (s + 1) * T[n][2c..], dbeta[c] = sum_n (s + 1) * T[n][0..]
 * with s the FiLM scale (0 without FiLM), and with FiLM the bf16 gradient of
 * its (scale, shift) rows, dfilm[n] = (T[n][c..2c), T[n][0..c)).  One launch;
 * fixed summation order (deterministic).  film / dfilm may be NULL together. */
int fp8_gn_param_grads(const float* totals, const void* film, int film_ld, int n, int c, float* dgamma,
                       float* dbeta, void* dfilm, int dfilm_ld, fp8_stream_t stream);

/* Nearest-neighbour resampling of the UNet (reference unet.py:368-383,
 * F.interpolate(..., mode="nearest"), which bf16 autocast runs in fp32) on NHWC
 * tensors; dtype codes: 0 = bf16, 1 = fp32.  c, c1, c2 multiples of 8; all
 * tensors 16-byte aligned.
 * fp8_resample_down2     : y (fp32) [n][h/2][w/2][c] = x[n][2i][2j][c] (scale 0.5)
 * fp8_resample_down2_bwd : dx [n][h][w][c] = dy at even (i, j), else 0 (dx dtype given)
 * fp8_up_cat     : y [n][h][w][c1 + c2] = (a[n][i/f][j/f][:], s[n][i][j][:]) with f = 2
 *                  (upsample, scale 2) or 1, in y's dtype: the upsample and the
 *                  skip concatenation (torch.cat, which promotes to the wider dtype)
 *                  as one pass
 * fp8_up_cat_bwd : da = fp32 sum of dy over each f x f block (channels 0..c1),
 *                  ds = dy channels c1..c1+c2, each in its own dtype */
int fp8_resample_down2(const void* x, int x_dtype, float* y, int n, int h, int w, int c, fp8_stream_t stream);
int fp8_resample_down2_bwd(const float* dy, void* dx, int dx_dtype, int n, int h, int w, int c,
                           fp8_stream_t stream);
int fp8_up_cat(const void* a, int a_dtype, const void* s, int s_dtype, void* y, int y_dtype, int n, int h, int w,
               int c1, int c2, int factor, fp8_stream_t stream);
int fp8_up_cat_bwd(const void* dy, int y_dtype, void* da, int a_dtype, void* ds, int s_dtype, int n, int h, int w,
                   int c1, int c2, int factor, fp8_stream_t stream);

/* fp8_up_cat with an fp32 y and a second output y_bf16 = bf16(y) (round to
 * nearest even): the concatenation the next residual block normalises and the
 * copy bf16 autocast makes of it for that block's 1x1 skip conv (reference
 * unet.py:139, 161, an nn.Conv2d reading the fp32 tensor), in one pass.
 * fp8_up_cat_pair_bwd: the gradient of y is dy + dy_bf16 (fp32 sum, the one
 * autograd forms for the two readers), then as fp8_up_cat_bwd. */
int fp8_up_cat_pair(const void* a, int a_dtype, const void* s, int s_dtype, float* y, void* y_bf16, int n, int h,
                    int w, int c1, int c2, int factor, fp8_stream_t stream);
int fp8_up_cat_pair_bwd(const float* dy, const void* dy_bf16, void* da, int a_dtype, void* ds, int s_dtype, int n,
                        int h, int w, int c1, int c2, int factor, fp8_stream_t stream);

/* Delayed scaling with the scale history kept on the device (reference
 * Conv2dFP8 bookkeeping, unet.py:69-91, fp8_kernels.py:841-853, 883-889):
 * the cast divides by max(window[0 .. window_len)) -- the module's
 * torch.max(amax_window) -- and writes that value to *scale_used_out (the
 * dequantisation scale of q, for the contraction); afterwards this tensor's
 * own scale (amax/448, 1.0 for amax 0) is stored at window[*window_pos] and,
 * when `advance`, *window_pos = (*window_pos + 1) % window_len.  One cast pass
 * whose last CTA folds the scale; no torch.max / scatter / position launches. */
int fp8_quantize_delayed_window(const void* x_bf16, void* q_e4m3, float* window, int window_len,
                                int64_t* window_pos, int advance, float* scale_used_out, void* workspace,
                                size_t workspace_bytes, int64_t n, fp8_stream_t stream);

/* The delayed quantize of up to 64 fp32 weight tensors in three launches (all FP8
 * conv weights of a model, once per step): tensor t is rounded to bf16 (the
 * reference's weight.to(bfloat16), fp8_kernels.py:836), cast with
 * max(windows[t][0 .. window_len)) -- written to *scale_used[t] -- and its own
 * scale stored at windows[t][*pos[t]]; the positions are not advanced (the
 * module's activation quantize, fp8_quantize_delayed_window with advance = 1,
 * writes at the same position and steps it).  Same bytes and histories as one
 * fp8_quantize_delayed_window per weight.  Pointer arrays are host memory. */
size_t fp8_quantize_weights_delayed_workspace_bytes(int count, const int64_t* n);
int fp8_quantize_weights_delayed(int count, const float* const* w, void* const* q, const int64_t* n,
                                 float* const* windows, int window_len, const int64_t* const* pos,
                                 float* const* scale_used, void* workspace, size_t workspace_bytes,
                                 fp8_stream_t stream);

/* The training step's tail in one pass over the parameters: gradient clipping
 * to max_grad_norm (torch.nn.utils.clip_grad_norm_; none when <= 0), AdamW
 * (decoupled weight decay, bias corrections from the device step count, which
 * this call increments) and, when ema != NULL, the EMA of the weights after the
 * update, ema = RN(ema * ema_beta) + RN((1 - ema_beta) * p) (reference
 * ddpm.py:20-25).  fp32 tensors; pointer arrays are host memory. */
size_t fp8_adamw_ema_workspace_bytes(int count, const int64_t* n);
int fp8_adamw_ema_step(int count, float* const* params, const float* const* grads, float* const* exp_avg,
                       float* const* exp_avg_sq, float* const* ema, const int64_t* n, float* step, float lr,
                       float beta1, float beta2, float eps, float weight_decay, float ema_beta, float max_grad_norm,
                       void* workspace, size_t workspace_bytes, fp8_stream_t stream);

/* fp8_gn_act_quant_fwd with the scale history of fp8_quantize_delayed_window. */
int fp8_gn_act_quant_fwd_window(const void* x, int x_fp32, const float* gamma, const float* beta, const void* film,
                                int film_ld, const int64_t* seed, float p, float eps, float* window, int window_len,
                                int64_t* window_pos, int advance, float* scale_used_out, float* stats, void* q_e4m3,
                                int n, int hw, int c, int groups, void* workspace, size_t workspace_bytes,
                                fp8_stream_t stream);

/* The UNet's residual join y = (a + b) / d (reference unet.py:161, :203 with
 * d = sqrt 2) as its bf16-autocast ops compute it: the sum rounded to y's dtype,
 * then times inv_divisor = RN32(1 / d), rounded again (torch divides by a host
 * scalar as a multiplication by its fp32 reciprocal).  The backward writes
 * g = RN_y(dy * inv_divisor) to da and db in their own dtypes.  n elements of
 * one dense layout, n % 8 == 0; dtype codes as fp8_up_cat. */
int fp8_add_scale(const void* a, int a_dtype, const void* b, int b_dtype, void* y, int y_dtype, int64_t n,
                  float inv_divisor, fp8_stream_t stream);
int fp8_add_scale_bwd(const void* dy, int y_dtype, void* da, int a_dtype, void* db, int b_dtype, int64_t n,
                      float inv_divisor, fp8_stream_t stream);

/* fp8_add_scale_bwd where b is the bf16 output of a delayed-scaling FP8 conv:
 * db (bf16) is also written as e4m3 to dbq, cast with max(window[0 ..
 * window_len)) -- which goes to *scale_used_out -- and db's own scale (amax /
 * 448) is stored at window[*window_pos] with the position kept: bit for bit
 * what the conv's backward gets from fp8_quantize_delayed_window(db, window,
 * window_pos, advance = 0) (reference Conv2dFP8Specialized.backward,
 * fp8_kernels.py:875-889), without reading db again.  Workspace:
 * fp8_add_scale_bwd_quant_workspace_bytes(n). */
size_t fp8_add_scale_bwd_quant_workspace_bytes(int64_t n);
int fp8_add_scale_bwd_quant(const void* dy, int y_dtype, void* da, int a_dtype, void* db_bf16, void* dbq_e4m3,
                            float* window, int window_len, int64_t* window_pos, float* scale_used_out, int64_t n,
                            float inv_divisor, void* workspace, size_t workspace_bytes, fp8_stream_t stream);

/* Workspace bytes of fp8_gn_act_quant_fwd. */
size_t fp8_gn_act_quant_workspace_bytes(int n, int hw, int c);

/* fp8_gn_act_fwd fused with the delayed-scaling quantize of its output, for the
 * FP8 conv that consumes it (the conv input x of reference
 * Conv2dFP8Specialized.forward, fp8_kernels.py:835-845, is
 * silu(norm1(x)) / dropout(silu((scale+1)*norm2(h)+shift)), unet.py:151, 157-159):
 *   q_e4m3[i]       = e4m3(clamp(bf16(a[i]) / *prev_scale, -448, 448))
 *   *scale_curr_out = amax|bf16(a)| / 448 (1.0 when the amax is 0)
 * bit for bit what fp8_gn_act_fwd followed by fp8_quantize_delayed gives, in one
 * statistics pass and one apply pass that writes only the e4m3 bytes and whose
 * last CTA folds the scale.  stats as in fp8_gn_act_fwd (for the backward). */
int fp8_gn_act_quant_fwd(const void* x, int x_fp32, const float* gamma, const float* beta, const void* film,
                         int film_ld, const int64_t* seed, float p, float eps, const float* prev_scale,
                         float* stats, void* q_e4m3, float* scale_curr_out, int n, int hw, int c, int groups,
                         void* workspace, size_t workspace_bytes, fp8_stream_t stream);

/* ------------------------------------------------------------ batched casts */

/* dst[t][i] = src[t][i] for count (1..64) dense tensors of n[t] elements, one
 * launch: to_bf16 != 0 casts fp32 -> bf16 (round to nearest even), else bf16
 * -> fp32 (exact).  Replaces the per-weight casts bf16 autocast makes for the
 * reference's bf16 layers (attention projections unet.py:171-172, 1x1 skip
 * convs :139, time-embedding linears :101, :331-336) and the casts of their
 * bf16 weight gradients back to the fp32 parameters' dtype. */
int fp8_cast_batch(int count, const void* const* src, void* const* dst, const int64_t* n, int to_bf16,
                   fp8_stream_t stream);

/* ------------------------------------------------------------ FP8 attention */

/* FP8 self-attention of the attention blocks, forward.  Replaces
 * F.scaled_dot_product_attention(q, k, v) with q, k, v = chunk(qkv, 3) split
 * into `heads` heads of head_dim channels (diffusion/unet.py:189-199), which the
 * reference runs in bf16; the reference has no FP8 attention kernel.
 *   qkv:  bf16 [batch][seq][ld_qkv], q of head h at columns h*64, k at C + h*64,
 *         v at 2C + h*64 (C = heads * 64) -- the qkv projection's output rows.
 *   o:    bf16 [batch][seq][ld_o], head h at columns h*64 (the layout the
 *         output projection reads).
 *   lse:  fp32 [batch][heads][seq], log-sum-exp of each query's logits.
 *   scales: fp32 [batch][heads][4], the e4m3 scales of q, k, v (amax/448 of each
 *         head's slice) and 0.
 * q, k and v are quantized per (image, head) with the reference's per-tensor
 * scale s = amax/448 (fp8_kernels.py:90-102) as e4m3(x * (1/s)) (one multiply by
 * the fp32 reciprocal), S = q k^T / sqrt(64) and O = P v run on the FP8
 * tensor cores with P quantized as e4m3(p * 448); softmax in fp32.
 * head_dim must be 64; seq a multiple of 16 in [16, 256]; qkv, o 16-byte
 * aligned, ld_qkv and ld_o multiples of 8. */
int fp8_attention_fwd(const void* qkv, void* o, float* lse, float* scales, int batch, int seq, int heads,
                      int head_dim, int ld_qkv, int ld_o, fp8_stream_t stream);

/* Backward of fp8_attention_fwd: dqkv (bf16, qkv's layout) from qkv, the
 * forward's o, lse and scales and the output gradient dout (o's layout).  The
 * gradient of the forward with straight-through quantizers, computed on the
 * bf16 tensor cores from the e4m3 values of q, k and v. */
int fp8_attention_bwd(const void* qkv, const void* o, const void* dout, const float* lse, const float* scales,
                      void* dqkv, int batch, int seq, int heads, int head_dim, int ld_qkv, int ld_o,
                      fp8_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FP8OPS_H_ */
