/* C ABI of the B200 (sm_100a) kernels for the trellis-coded W2A8 Linear.
 *
 * Drop-in boundary for the reference's kernel wrappers (ForeverBlue816/yanlongvla, deploy/tcq_kernels/kernels.py):
 * each entry point below replaces one Python wrapper of that file (cited per function), keeps its argument meaning,
 * and adds the shapes and the stream the wrapper used to read from tensors / torch.cuda.current_stream().
 *
 * Conventions (all entry points):
 *   - every buffer is a device pointer allocated and owned by the caller; the library allocates nothing and keeps no
 *     per-call state, so calls can be captured in a CUDA graph. The one exception is tcq_gemm_tcq_noalloc: it keeps
 *     its scratch in one fixed array inside the library that every call on a device shares (calls that overlap on
 *     the GPU race on it), and its first call on a device, which looks up that array's address, must come before
 *     any stream capture;
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream);
 *   - kernels are launched with programmatic dependent launch and read a layer's constants (the packed trellis
 *     stream `bits`, its table `t8`, row scales, sign vectors, norm weights) before waiting for the work queued
 *     before them on the stream; everything else (activations, accumulators, token scales, outputs) only after. A
 *     kernel launched the ordinary way completes before the next launch starts, so it may write those constants;
 *     a writer that itself releases its dependents early (griddepcontrol.launch_dependents) needs an event wait or
 *     a stream synchronization before the call;
 *   - optional outputs / inputs may be NULL where stated (the reference passes None for them, cuda_rt.py:90-91);
 *   - BF16 values are passed as uint16_t bit patterns; dtype codes are TCQ_DT_*;
 *   - the return value is a tcq_status: 0 on success; shapes and alignment are validated on the host before any
 *     launch, so a non-zero status means nothing was launched (TCQ_ERR_LAUNCH: the launch itself failed; for
 *     tcq_gemm_tcq_noalloc a clear of its own scratch array may already be queued on the stream then).
 */
#ifndef TCQ_B200_H
#define TCQ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TCQ_ABI_VERSION 1

enum tcq_status {
    TCQ_OK = 0,
    TCQ_ERR_SHAPE = 1,     /* a size is not supported (e.g. width not a multiple of 16, or above the limit)   */
    TCQ_ERR_ALIGN = 2,     /* a pointer or leading dimension breaks the 16-byte alignment the kernel needs     */
    TCQ_ERR_DTYPE = 3,     /* unknown dtype code                                                              */
    TCQ_ERR_ARG = 4,       /* a required pointer is NULL, or an argument is out of range                        */
    TCQ_ERR_LAUNCH = 5,    /* the CUDA launch failed (cudaGetLastError after the launch)                        */
    TCQ_ERR_DEVICE = 6,    /* no usable device, or not an sm_100 device                                         */
    TCQ_ERR_WORKSPACE = 7  /* the workspace is missing or smaller than the *_workspace() query returned           */
};

enum tcq_dtype { TCQ_DT_BF16 = 0, TCQ_DT_F32 = 1, TCQ_DT_F16 = 2, TCQ_DT_I32 = 3 };

/* Library version and status text. */
int tcq_abi_version(void);
const char* tcq_status_string(int status);

/* ------------------------------------------------------------------------------------------------ rotation + quantizer
 * Row widths K / N are multiples of 16 and at most 16384; rows are rotated by the block Walsh over the binary
 * decomposition of the width (tcq_format.py:26-55). */

/* Replaces kernels.pre (kernels.py:602-606; kernel k_pre_*, kernels.py:208-219): x (M, K) BF16/F16/F32 -> sign flip
 * by su (K,), block Walsh, per-token absmax INT8. Outputs q (M, K) int8 and/or q4 (K/4, ldq) int32 words (4
 * consecutive inputs per word, token = column; NULL = not written), scale (M,) float32. */
int tcq_pre(const void* x, int x_dtype, const int8_t* su, int8_t* q, int32_t* q4, float* scale,
            int M, int K, int ldq, void* stream);

/* The per-token INT8 quantizer alone, without rotation (tcq_format.quantize_tokens, tcq_format.py:119-122), for
 * W8A8 layers that are not rotated (benchmark config 3, the vision tower): x (M, K) BF16/F16/F32 -> q (M, K) int8,
 * scale (M,) float32 = absmax / 127 (1 for an all-zero row). */
int tcq_quantize(const void* x, int x_dtype, int8_t* q, float* scale, int M, int K, void* stream);

/* Replaces kernels.pre2 (kernels.py:631-633; k_pre2, kernels.py:295-307): x = BF16(g * u) of two BF16 (M, K) inputs,
 * then as tcq_pre. */
int tcq_pre2(const uint16_t* g, const uint16_t* u, const int8_t* su, int8_t* q, int32_t* q4, float* scale,
             int M, int K, int ldq, void* stream);

/* Replaces kernels.pre_h (kernels.py:677-680; k_preh_*, kernels.py:309-317): rotated activations as BF16, h (M, K)
 * row-major and/or hT (K, ldh) with token = column. */
int tcq_pre_h(const void* x, int x_dtype, const int8_t* su, uint16_t* h, uint16_t* hT, int M, int K, int ldh,
              void* stream);

/* Replaces kernels.post (kernels.py:612-615; k_post_*, kernels.py:221-230): for token t, columns col0 .. col0+N of
 * the accumulator row acc (M, lda): z = ((float)a * s[t]) * rs[i] (acc_dtype I32), a (F32, already scaled) or
 * bf2f(a) * rs[i] (BF16); then block Walsh, * sv[i], + bias[i] (bias may be NULL), BF16 y (M, N).
 * s and rs may be NULL when acc_dtype does not use them. */
int tcq_post(const void* acc, int acc_dtype, const float* s, const float* rs, const int8_t* sv, const float* bias,
             uint16_t* y, int M, int N, int lda, int col0, void* stream);

/* Replaces kernels.post3 (kernels.py:618-621; k_post3_*, kernels.py:232-247): three layers (q / k / v) sharing the
 * accumulator row, columns [0,n0), [n0,n0+n1), [n0+n1, n0+n1+n2); rs / sv / bias concatenated. */
int tcq_post3(const void* acc, int acc_dtype, const float* s, const float* rs, const int8_t* sv, const float* bias,
              uint16_t* y0, uint16_t* y1, uint16_t* y2, int M, int n0, int n1, int n2, int lda, void* stream);

/* Replaces kernels.postg (kernels.py:624-628; k_postg_*, kernels.py:249-261): up to three layers sharing the row, one
 * thread block per (token, layer); act0 != 0 applies the activation table lut (65536 BF16 entries indexed by the BF16
 * bit pattern) to the first layer's output. Unused layers: n = 0 and y = NULL. */
int tcq_postg(const void* acc, int acc_dtype, const float* s, const float* rs, const int8_t* sv, const float* bias,
              const uint16_t* lut, uint16_t* y0, uint16_t* y1, uint16_t* y2, int M, int n0, int n1, int n2, int lda,
              int act0, void* stream);

/* Replaces kernels.mid2 (kernels.py:641-644; k_mid2_*, kernels.py:263-278): gated-MLP middle. acc (M, lda) holds
 * gate | up (columns [0,N) and [N,2N)); rs, sv concatenated (2N); g = lut(BF16(post(gate))), u = BF16(post(up)),
 * x = BF16(g * u), then sign su (N,), block Walsh and INT8 quantizer as tcq_pre. lut = GELU-tanh (Gemma) or SiLU
 * (SwiGLU) table. */
int tcq_mid2(const void* acc, int acc_dtype, const float* s, const float* rs, const int8_t* sv, const uint16_t* lut,
             const int8_t* su, int8_t* q, int32_t* q4, float* scale, int M, int N, int lda, int ldq, void* stream);

/* Replaces kernels.mid1 (kernels.py:647-650; k_mid1_*, kernels.py:280-292): plain-MLP middle,
 * x = lut(BF16(post(acc) + bias)) -> sign su, block Walsh, INT8. */
int tcq_mid1(const void* acc, int acc_dtype, const float* s, const float* rs, const int8_t* sv, const float* bias,
             const uint16_t* lut, const int8_t* su, int8_t* q, int32_t* q4, float* scale, int M, int N, int lda,
             int ldq, void* stream);

/* Standalone randomized Walsh rotation (the rotation op; tcq_format.py:44-55 with the signs of :130 / :145):
 * forward y = fwht(x * signs), inverse y = fwht(x) * signs; x (M, D) BF16/F16/F32, y (M, D) BF16 or F32. */
int tcq_rotate(const void* x, int x_dtype, const int8_t* signs, void* y, int y_dtype, int M, int D, int inverse,
               void* stream);

/* ------------------------------------------------------------------------------------------------ trellis weights
 * bits: (m/16 * n/16, 32) uint16 words, 512 bits per 16 x 16 tile, tiles row-major (tcq_format.py:3-12, 58-63);
 * t8: (512, 2) int8 table (tcq_format.py:74-77); m, n multiples of 16. */

/* Replaces kernels.decode (kernels.py:653-656; k_decode, kernels.py:339-349): dense INT8 W (m, n) row-major. */
int tcq_decode(const uint16_t* bits, const int8_t* t8, int8_t* out, int m, int n, void* stream);

/* Replaces kernels.decode_bf16 (kernels.py:683-686; k_decode_bf16, kernels.py:320-337): tb (512, 2) BF16 bit
 * patterns of the INT8 table values; out (m, n) BF16. */
int tcq_decode_bf16(const uint16_t* bits, const uint16_t* tb, uint16_t* out, int m, int n, void* stream);

/* Replaces kernels.gemm_w8 (kernels.py:662-668; k_gemm_w8, kernels.py:365-399): INT8-resident small-M product.
 * W (N, K) int8, q4 (K/4, M) int32 words, s (M,), rs (N,) -> z (M, N) float32 = ((float)acc * s[t]) * rs[n].
 * 1 <= M <= 16. */
int tcq_gemm_w8(const int8_t* W, const int32_t* q4, const float* s, const float* rs, float* z, int M, int N, int K,
                void* stream);

/* Workspace of tcq_gemm_tcq in bytes for (M, N). The workspace must be zero-filled before its first use; every
 * successful call leaves it zero-filled again. */
size_t tcq_gemm_tcq_workspace(int M, int N);

/* Replaces kernels.gemm_tcq (kernels.py:671-673; k_gemm_tcq, kernels.py:403-427): trellis decode fused into the
 * small-M product; the decoded weights never leave the SM. Up to three layers concatenated along the output rows
 * (q / k / v, gate / up): tile rows < nb0 use table 0 of t8 (3 x 1024 bytes), < nb1 table 1, else table 2
 * (nb = 1 << 30: unused). z (M, N) float32 = ((float)acc * s[t]) * rs[n], bit-exact. 1 <= M <= 16.
 * workspace: tcq_gemm_tcq_workspace(M, N) bytes, see above. */
int tcq_gemm_tcq(const uint16_t* bits, const int8_t* t8, const int32_t* q4, const float* s, const float* rs, float* z,
                 int M, int N, int K, int nb0, int nb1, void* workspace, size_t workspace_bytes, void* stream);

/* No counterpart in the reference. The fused decode-GEMV of tcq_gemm_tcq for callers that cannot allocate device
 * memory (e.g. a real-time control loop that must not call cudaMalloc, or a plugin host that owns every device
 * buffer): same arguments and bit-identical results, no workspace argument. Its scratch is a fixed ~2 MiB array inside
 * this library (held on every GPU that loads it until exit); the first call on a device looks up its address (make
 * that first call before any stream capture). Limits: 1 <= M <= 16, N <= 32768, M * N <= 524288, else TCQ_ERR_SHAPE.
 * Calls share the array: calls that overlap on the GPU (different streams or threads) race. Allocates nothing. */
int tcq_gemm_tcq_noalloc(const uint16_t* bits, const int8_t* t8, const int32_t* q4, const float* s, const float* rs,
                         float* z, int M, int N, int K, int nb0, int nb1, void* stream);

/* Largest M * N tcq_gemm_tcq_noalloc accepts. */
size_t tcq_gemm_tcq_noalloc_max_elements(void);

/* ------------------------------------------------------------------------------------------------ W8A8 INT8 GEMM
 * q (M, K) int8 row-major (tokens), W (N, K) int8 row-major (output channels); K a multiple of 16; q, W 16-byte
 * aligned. tcgen05 tensor cores (kind::i8), exact INT32 accumulation. */

/* Replaces torch._int_mm(q, W.t()) as the reference calls it (modules.py:86; tcq_format.py:110-116):
 * acc (M, N) int32 = q W^T, exact. */
int tcq_int_mm(const int8_t* q, const int8_t* W, int32_t* acc, int M, int N, int K, void* stream);

/* The reference's product + scale epilogue in one launch (tcq_format.py:135; benchmark config 3):
 * out (M, N) = ((float)acc * s_tok[t]) * s_ch[n] as BF16 (out_dtype TCQ_DT_BF16) or FP32 (TCQ_DT_F32). */
int tcq_int8_gemm(const int8_t* q, const int8_t* W, const float* s_tok, const float* s_ch, void* out, int out_dtype,
                  int M, int N, int K, void* stream);

/* tcq_int8_gemm with BF16 output and the layer's bias (and activation) in the epilogue (no counterpart in the
 * reference, whose vision tower is not W8A8: this is the W8A8 Linear of the policy's vision tower, followed there by a
 * BF16 tensor add of its bias and, for the MLP's first layer, the tanh GELU): out = act(BF16(BF16(z) + bias)),
 * z = ((float)acc * s_tok[t]) * s_ch[n], i.e. the result of int8_gemm, then `+ bias`, then the activation, in PyTorch
 * BF16 arithmetic bit for bit. bias (N,) BF16 or NULL; act_lut the 65536-entry BF16 table of the activation
 * (kernels.act_table) or NULL. */
int tcq_int8_gemm_bias(const int8_t* q, const int8_t* W, const float* s_tok, const float* s_ch, const uint16_t* bias,
                       const uint16_t* act_lut, uint16_t* out, int M, int N, int K, void* stream);

/* Workspace of tcq_gemm_tcq_tc in bytes for (M, N); same zero-filled contract as tcq_gemm_tcq_workspace. */
size_t tcq_gemm_tcq_tc_workspace(int M, int N);

/* kernels.pre + kernels.gemm_tcq in one launch for 1 <= M <= 4 tokens and K <= 8192 (no single counterpart in the
 * reference, which launches kernels.pre then kernels.gemm_tcq, kernels.py:602-606, 671-673): every CTA rotates and
 * quantizes x (M, K) BF16 / F16 / F32 with the input signs su itself, as tcq_pre would (same bits), and runs the fused
 * decode-GEMV on the result; z as tcq_gemm_tcq. Workspace: tcq_gemm_tcq_workspace(M, N) bytes, same contract. */
int tcq_gemm_tcq_x(const uint16_t* bits, const int8_t* t8, const void* x, int x_dtype, const int8_t* su, const float* rs,
                   float* z, int M, int N, int K, int nb0, int nb1, void* workspace, size_t workspace_bytes, void* stream);

/* Tensor-core form of kernels.gemm_tcq (kernels.py:671-673) for 1 <= M <= 256 tokens, and the on-the-fly prefill
 * product of the reference (k_decode + torch._int_mm, modules.py:81-86) without the dense INT8 weights: the trellis
 * stream is decoded straight into shared memory and consumed by tcgen05.mma.kind::i8. q (M, K) int8 row-major
 * (tcq_pre's q output), z (M, N) float32 = ((float)acc * s[t]) * rs[n], bit-exact. Layer bounds nb0 / nb1 (tile rows)
 * must be multiples of 8 (128 output rows) or >= N/16. workspace: tcq_gemm_tcq_tc_workspace(M, N) bytes. */
int tcq_gemm_tcq_tc(const uint16_t* bits, const int8_t* t8, const int8_t* q, const float* s, const float* rs, float* z,
                    int M, int N, int K, int nb0, int nb1, void* workspace, size_t workspace_bytes, void* stream);

/* W2 float-activation products (kernels.gemmf_tcq / gemmf_w8, kernels.py:677-696; kernels k_gemmf_*, kernels.py:
 * 430-489): hT (K, ldh) BF16 rotated activations from tcq_pre_h (token = column), INT8-table weights (the trellis
 * stream decoded in the kernel with the per-layer tables of t8 and layer bounds nb0 / nb1 in tile rows, or INT8
 * resident W (N, K)), FP32 accumulation; z (M, N) = (sum_k w h) * rs. Any M (launched in chunks of 16 tokens). The sum
 * order is fixed (reproducible) but differs from a float64 sum: this path is checked to a tolerance. */
int tcq_gemmf_tcq(const uint16_t* bits, const int8_t* t8, const uint16_t* hT, const float* rs, float* z, int M, int N, int K,
                  int ldh, int nb0, int nb1, void* stream);
int tcq_gemmf_w8(const int8_t* W, const uint16_t* hT, const float* rs, float* z, int M, int N, int K, int ldh, void* stream);

/* Policy glue around the quantized layers (no counterpart in the reference's kernels: its model code runs these as
 * PyTorch ops, e.g. RMSNorm as float/pow/mean/rsqrt/mul/mul/cast). One launch per call, one block per token row.
 *
 * tcq_add_norm: h = x + y (BF16 add; written to h when h != NULL, y may be NULL for a plain norm), then
 * kind 0 RMSNorm n = (h * rsqrt(sum(h^2) / D + eps)) * w, kind 1 LayerNorm n = ((h - mean) * rsqrt(var + eps)) * w + b
 * (w, b (D,) of dtype wb_dtype, TCQ_DT_F32 or TCQ_DT_BF16; NULL = 1 / 0); with mod_scale / mod_shift (BF16 vectors, row stride ld_mod, one per group of
 * mod_rows rows) n = n * (1 + mod_scale) + mod_shift (the DiT's AdaLN). out = BF16(n). x, y, h, out (M, D) BF16,
 * D a multiple of 16, at most 32768. Row sums run in a fixed order: results are reproducible run to run. */
int tcq_add_norm(const uint16_t* x, const uint16_t* y, uint16_t* h, uint16_t* out, const void* w, const void* b, int wb_dtype,
                 const uint16_t* mod_scale, const uint16_t* mod_shift, int mod_rows, int ld_mod, float eps, int kind, int M,
                 int D, void* stream);

/* Fused chain across a residual block boundary: one layer's post-rotation fused with the next layer's pre-rotation
 * through the residual add and norm between them (no single counterpart in the reference, which runs kernels.post,
 * the model's PyTorch add + norm and kernels.pre, kernels.py:602-628): per token row
 *   y = tcq_post(acc, ...) (acc != NULL; acc_dtype I32 with s / rs, or F32 z already scaled) or y = the BF16 tensor y,
 *   h = BF16(x + y) -> h (h = x without y), n = the norm of tcq_add_norm (same arguments, same arithmetic and order)
 *   -> n when n != NULL, and with su != NULL q / q4 / scale = tcq_pre(BF16(n), su) of the next layer; with su == NULL
 *   and q or q4 given, q / q4 / scale = the plain per-token INT8 quantization of BF16(n) (tcq_quantize's arithmetic,
 *   for a W8A8 next layer).
 * Each stage is bit-identical to the separate entry point. x, y, h, n (M, N) BF16; acc (M, lda) from column col0. */
int tcq_chain(const void* acc, int acc_dtype, const float* s, const float* rs, const int8_t* sv, const float* bias, int lda,
              int col0, const uint16_t* y, const uint16_t* x, uint16_t* h, uint16_t* n, const void* w, const void* b,
              int wb_dtype, const uint16_t* mod_scale, const uint16_t* mod_shift, int mod_rows, int ld_mod, float eps,
              int kind, const int8_t* su, int8_t* q, int32_t* q4, float* scale, int ldq, int M, int N, void* stream);

/* Rotary position embedding, half-split form: for each of `heads` heads of width D in row r (position r % T) and
 * j < D/2, (a, b) = (x[j], x[j + D/2]) -> (BF16(a cos - b sin), BF16(a sin + b cos)) in FP32 with one rounding per
 * operation. x (rows, ldx) and out (rows, ldo) BF16 (out may equal x), cos / sin (T, D/2) FP32. */
int tcq_rope(const uint16_t* x, uint16_t* out, const float* cos_t, const float* sin_t, int rows, int T, int heads, int D,
             int ldx, int ldo, void* stream);

/* Self-test of the failure path (no counterpart in the reference): one thread waits, through the same bounded wait the
 * tcgen05 kernels use, on a barrier that nothing arrives at; after limit_us (1 .. 1e6) microseconds the wait gives up,
 * raises device error flag 1 and the kernel returns. Nothing faults and the context stays usable. */
int tcq_selftest_wait_expiry(unsigned limit_us, void* stream);

/* Device error flags raised by bounded waits inside the kernels (1 = a pipeline wait expired and the kernel stopped
 * early). Synchronizes the current device. reset != 0 clears the flags. Returns -1 if the flags cannot be read. */
int tcq_device_error(int reset);

#ifdef __cplusplus
}
#endif
#endif /* TCQ_B200_H */
