/*
 * xgb.h — C ABI of the xgen_b200 library (libxgb.so): the B200 (sm_100a)
 * kernels behind xGen's sequence-parallel MiniMax-H3 attention hot path.
 *
 * Conventions shared by every entry point:
 *   - Plain pointers to device memory, sizes and strides in ELEMENTS, and a
 *     cudaStream_t passed as `void* stream` (NULL = legacy default stream).
 *   - Return XGB_OK (0) or a negative status; never throw, never exit.
 *   - No entry point allocates device memory. Kernels that need scratch
 *     take a caller-provided workspace and export a *_workspace() sizing
 *     function.
 *   - Work is enqueued on `stream` only; calls are thread-compatible.
 *   - dtype codes: XGB_BF16 or XGB_F16 for 16-bit floating inputs.
 *
 * Each declaration cites the reference (lightnateriver/xGen) function whose
 * behaviour it reproduces, as path:line within that project.
 */
#ifndef XGB_H_
#define XGB_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define XGB_OK 0
#define XGB_ERR_ARG (-1)       /* null pointer or out-of-range parameter */
#define XGB_ERR_SHAPE (-2)     /* sizes the kernel does not support */
#define XGB_ERR_STRIDE (-3)    /* strides the kernel does not support */
#define XGB_ERR_ALIGN (-4)     /* pointer/stride alignment requirement not met */
#define XGB_ERR_LAUNCH (-5)    /* CUDA reported an error for the launch */
#define XGB_ERR_DEVICE (-6)    /* current device is not an sm_100 part */
#define XGB_ERR_WORKSPACE (-7) /* workspace missing or smaller than required */

#define XGB_BF16 0
#define XGB_F16 1

/* Library ABI version (major*100 + minor). */
int xgb_version(void);

/* Human-readable name of a status code (static string). */
const char* xgb_status_string(int status);

/* ---- Elementwise operators, bit-exact with the reference Triton kernels ---- */

/* Rotate-half RoPE over the first `rotary` channels of contiguous bf16
 * Q and K [batch, seq, heads, width]; cos/sin fp32 [seq, rotary], rounded to
 * bf16 before use; every product rounded to bf16 as eager PyTorch does.
 * Replaces _partial_rope / try_h3_partial_rope,
 * x_base/x_base/operator/h3_partial_rope.py:9-47. */
int xgb_partial_rope(const void* q, const void* k, const float* cos, const float* sin,
                     void* q_out, void* k_out, int64_t batch, int64_t seq, int64_t heads,
                     int64_t width, int64_t rotary, void* stream);

/* Per-head RMSNorm of strided bf16 Q/K views [batch, seq, heads, width]
 * (q_strides/k_strides = element strides of batch, seq, head; channel
 * stride must be 1) times the bf16 weight, then optional rotate-half RoPE
 * over `rotary` channels (rotary = 0 disables; cos/sin may then be NULL).
 * Outputs are contiguous. Replaces _qk_rms / try_h3_qk_rms,
 * x_base/x_base/operator/h3_qk_rms.py:9-84. */
int xgb_qk_rms(const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
               const void* q_weight, const void* k_weight, float q_eps, float k_eps,
               const float* cos, const float* sin, int64_t rotary, void* q_out, void* k_out,
               int64_t batch, int64_t seq, int64_t heads, int64_t width, void* stream);

/* AdaLN indexed modulation (modulation = 1):
 *     out = bf16(bf16(x * bf16(1 + table[idx])) + addend[idx])
 * or gated residual (modulation = 0):
 *     out = bf16(bf16(x * table[idx]) + addend)
 * x/out contiguous bf16 [batch, seq, width]; table/addend rows strided by
 * table_stride/addend_stride elements (addend contiguous like x when
 * modulation = 0); indices int64 [seq].
 * Replaces _indexed_affine / _apply,
 * x_base/x_base/operator/h3_indexed_affine.py:9-49. */
int xgb_indexed_affine(const void* x, const void* table, int64_t table_stride,
                       const void* addend, int64_t addend_stride, const int64_t* indices,
                       void* out, int64_t batch, int64_t seq, int64_t width, int modulation,
                       void* stream);

/* Gate-first packed SwiGLU: out[r, c] = bf16(bf16(g / (1 + exp(-g))) * v)
 * with g = x[r, c], v = x[r, width + c]; x bf16 [rows, 2*width] contiguous.
 * When amax_out is non-NULL it receives max |out| (NaN-propagating) — the
 * caller zeroes it first (it is combined with atomic max).
 * Replaces _swiglu / gate_first_swiglu,
 * x_base/x_base/operator/h3_swiglu.py:15-41. */
int xgb_swiglu(const void* x, void* out, int64_t rows, int64_t width, float* amax_out,
               void* stream);

/* ---- PHAA FP8 wire format (per-row e4m3 + fp32 scale) ---- */

/* Encode `streams` (1 or 3) tensors into the PHAA byte wire. Each source is
 * a 4-D view [peers, seq, batch, heads] of rows of `width` channels with
 * element strides strides[4*s + 0..3] for source s (channel stride 1).
 * Wire row = width e4m3 bytes + one fp32 scale, scale = max(amax/448,
 * 1e-12); per peer the packet holds stream 0 rows, stream 1 rows, stream 2
 * rows, then `peer_padding` zero bytes.
 * When rotary > 0, streams 0 and 1 (Q, K) first get the rotate-half RoPE of
 * xgb_partial_rope using cos/sin rows indexed by the `seq` coordinate —
 * the two reference kernels fused, bit-exact with running them in turn.
 * Replaces _encode, x_base/x_base/phaa/fp8_transport.py:26-63 (and the
 * send side of fp8_all_to_all_many, :85-140). */
int xgb_fp8_wire_encode(const void* const* sources, const int64_t* strides, int streams,
                        int64_t peers, int64_t seq, int64_t batch, int64_t heads, int64_t width,
                        int dtype, const float* cos, const float* sin, int64_t rotary,
                        int64_t peer_padding, uint8_t* payload, void* stream);

/* Decode the wire into `streams` contiguous outputs of rows*width elements
 * (dest = e4m3 * scale, rounded to dtype). rows = total rows per stream.
 * Replaces _decode, x_base/x_base/phaa/fp8_transport.py:66-78. */
int xgb_fp8_wire_decode(const uint8_t* payload, void* const* dests, int streams, int64_t rows,
                        int64_t peers, int64_t width, int64_t peer_padding, int dtype,
                        void* stream);

/* xgb_fp8_wire_encode with a sequence mask: rows whose global sequence
 * index peer*seq + s is >= valid_seq are not read and encode as zeros with
 * scale 1e-12 (0 < valid_seq <= peers*seq; peers*seq means all rows). The
 * async exchange's fused return pack encodes the attention output
 * [batch, head, valid_seq, D] through the view [peers, seq, batch, head]
 * with strides (seq*sS, sS, sB, sH).
 * Replaces _encode with RETURN_SEQ / STRIDED,
 * x_base/x_base/phaa/fp8_async_transport.py:14-50, and _pack_exchange,
 * :129-181. */
int xgb_fp8_wire_encode_view(const void* const* sources, const int64_t* strides, int streams,
                             int64_t peers, int64_t seq, int64_t batch, int64_t heads,
                             int64_t width, int dtype, const float* cos, const float* sin,
                             int64_t rotary, int64_t valid_seq, int64_t peer_padding,
                             uint8_t* payload, void* stream);

/* Decode the wire into `streams` destinations addressed, like the encode's
 * sources, as [peers, seq, batch, heads] views with element strides
 * strides[4*s + 0..3] (channel stride 1); rows with peer*seq + s >=
 * valid_seq are skipped. Wire rows are in [peer, seq, batch, head] order.
 * Covers the direct gather (destination = attention input [batch, head,
 * valid_seq, D]) and the direct return (destination = [batch, seq, heads*D]
 * at the chunk's head offset) of the async exchange.
 * Replaces _decode / _unpack_exchange,
 * x_base/x_base/phaa/fp8_async_transport.py:53-81, :184-193. */
int xgb_fp8_wire_decode_view(const uint8_t* payload, void* const* dests, const int64_t* strides,
                             int streams, int64_t peers, int64_t seq, int64_t batch,
                             int64_t heads, int64_t width, int64_t valid_seq,
                             int64_t peer_padding, int dtype, void* stream);

/* An SP exchange's encode and all-to-all in one kernel: encodes `streams`
 * (1, or 3 for Q/K/V) bf16 [peers, seq, batch, heads] views of 128 channels
 * (strides as xgb_fp8_wire_encode_view, multiples of 8; sources 16-byte
 * aligned), with the fused rotate-half RoPE of streams 0 and 1 when streams
 * is 3 (rotary a multiple of 32, 0 for none), and stores each peer's
 * section, byte for byte as xgb_fp8_wire_encode_view with peer_padding 0
 * writes it, at peer_dst[p] (16-byte aligned; normally peer p's receive
 * buffer at this rank's section, a peer pointer reached over NVLink).
 * peers <= 8, heads <= 12, seq*batch a multiple of 4.
 * Replaces the encode + dist.all_to_all_single pair of fp8_all_to_all_many /
 * fp8_all_to_all, x_base/x_base/phaa/fp8_transport.py:85-144. */
int xgb_fp8_wire_encode_peers(const void* const* sources, const int64_t* strides, int streams,
                              int64_t peers, int64_t seq, int64_t batch, int64_t heads,
                              const float* cos, const float* sin, int64_t rotary, int64_t valid_seq,
                              uint8_t* const* peer_dst, void* stream);

/* Store `value` into each of n (<= 64) flag words (normally in peer GPUs'
 * buffers), after a system-scope fence and with release semantics, on
 * `stream`. */
int xgb_peer_signal(int* const* flags, int n, int value, void* stream);

/* Wait on `stream` until each of n (<= 64) flag words holds at least
 * `value` (acquire, system scope). After limit_ns it records a timeout in
 * *error_flag (device int, may be NULL) and lets the stream continue. */
int xgb_peer_wait(int* const* flags, int n, int value, int64_t limit_ns, int* error_flag,
                  void* stream);

/* ---- FP8 Linear activation quantisation ---- */

/* Bytes of workspace xgb_fp8_quantize_per_tensor needs for n elements. */
int64_t xgb_fp8_quantize_per_tensor_workspace(int64_t n);

/* Per-tensor dynamic e4m3: scale = max(amax(|x|)/448, FLT_MIN),
 * out = e4m3(clamp(x/scale, +-448)); scale_out = one fp32 on the device.
 * Replaces quantize_per_tensor (x_base/x_base/operator/h3_fp8.py:9-12) and
 * quantize_activation + activation_abs_peak
 * (h3_fp8_quant.py:18-25, h3_abs_peak.py:14-25). */
int xgb_fp8_quantize_per_tensor(const void* x, int dtype, int64_t n, uint8_t* out,
                                float* scale_out, void* workspace, int64_t workspace_bytes,
                                void* stream);

/* xgb_fp8_quantize_per_tensor for callers that cannot allocate device
 * memory at call time (a plugin whose host runtime owns every allocation, a
 * server that plans all of HBM up front, a latency-critical path that cannot
 * take cudaMalloc's implicit device synchronisation). Same inputs, outputs
 * and results as xgb_fp8_quantize_per_tensor, but the per-block peak scratch
 * is a fixed 256 KiB array inside the library, so no workspace is passed and
 * nothing is allocated. Limit: n <= 536,870,912 elements (65,536 peak
 * blocks of 8,192); larger n returns XGB_ERR_SHAPE. The first call on each
 * device resolves the array's device address (make it before any stream
 * capture); every GPU that loads the library keeps the array until exit; all
 * calls share it, so calls whose kernels overlap on one device race.
 * No counterpart in the reference: it is an addition of this library. */
int xgb_fp8_quantize_per_tensor_noalloc(const void* x, int dtype, int64_t n, uint8_t* out,
                                        float* scale_out, void* stream);

/* The two halves of xgb_fp8_quantize_per_tensor, for a scale shared by a
 * process group: xgb_fp8_abs_peak_scale writes scale_out = max(amax/448,
 * FLT_MIN) (workspace as for xgb_fp8_quantize_per_tensor); the caller may
 * then all-reduce it with MAX; xgb_fp8_quantize_with_scale writes
 * out = e4m3(clamp(x/scale, +-448)) with the device scalar *scale.
 * Replace quantize_activation(x, group=...),
 * x_base/x_base/operator/h3_fp8_quant.py:18-25 (used by H3FP8TPLinear,
 * h3_fp8.py:58-68). */
int xgb_fp8_abs_peak_scale(const void* x, int dtype, int64_t n, float* scale_out, void* workspace,
                           int64_t workspace_bytes, void* stream);
int xgb_fp8_quantize_with_scale(const void* x, int dtype, int64_t n, const float* scale,
                                uint8_t* out, void* stream);

/* Per-token dynamic e4m3 (the per-token scaling of the B200 FP8 Linear):
 * scales[r] = max(amax(|x[r,:]|)/448, FLT_MIN), out[r,c] = e4m3(x/scale).
 * x rows strided by row_stride elements; out contiguous [rows, cols].
 * Per-token counterpart of quantize_activation,
 * x_base/x_base/operator/h3_fp8_quant.py:18-25. */
int xgb_fp8_quantize_per_token(const void* x, int dtype, int64_t rows, int64_t cols,
                               int64_t row_stride, uint8_t* out, float* scales, void* stream);

/* ---- FP8 GEMM (tcgen05 kind::f8f6f4) ---- */

/* out[m, n] = bf16(acc[m, n] * (scale_a[m*sa_stride] * scale_w[n*sw_stride])
 *                  + bias[n])
 * with acc = sum_k a[m, k] * w[n, k] in fp32; a [M, K] and w [N, K] e4m3
 * row-major (16-byte aligned, K and N multiples of 16); scale strides 0
 * (per-tensor scalar) or 1 (per row / per output channel); bias bf16 [N]
 * or NULL; out bf16 rows ldo elements apart. activation: 0 none, 1 GELU
 * (erf), 2 GELU (tanh approximation), applied after the bias (FFN up),
 * 3 gate-first SwiGLU: w rows (and scale_w, bias) interleaved in groups of
 * 128 as [gate j..j+127 | value j..j+127] (N % 256 == 0), and
 *     out[m, j] = bf16(bf16(silu(yg)) * yv), yg/yv the bf16 plain results
 * of the gate/value rows, N/2 output columns (replaces the separate
 * gate_first_swiglu pass, x_base/x_base/operator/h3_swiglu.py:15-41).
 * When gate != NULL the AdaLN gated residual is fused in, with the
 * reference's rounding after each op:
 *     out[m, n] = bf16(bf16(y * gate[gate_index[m]*ldg + n]) + residual[m*ldr + n])
 * error_flag as for the attention kernels.
 * Replaces torch._scaled_mm in H3FP8Linear._local_forward
 * (x_base/x_base/operator/h3_fp8.py:48-68) and the gated `_apply` after the
 * output projections (x_base/x_base/operator/h3_indexed_affine.py:52-61). */
int xgb_fp8_gemm(const uint8_t* a, const uint8_t* w, int64_t M, int64_t N, int64_t K,
                 const float* scale_a, int64_t scale_a_stride, const float* scale_w,
                 int64_t scale_w_stride, const void* bias, int activation, void* out, int64_t ldo,
                 const void* gate, int64_t ldg, const int64_t* gate_index, const void* residual,
                 int64_t ldr, int* error_flag, void* stream);

/* AdaLN prologue of an FP8 Linear, one HBM pass per row of x [rows, width]
 * (rows = batch * seq, row stride ldx):
 *   n = norm(x) rounded to bf16, norm_kind 0 = LayerNorm without affine,
 *       1 = RMSNorm times the bf16 weight (weight may be NULL), eps
 *   h = bf16(bf16(n * bf16(1 + scale[t])) + shift[t]),  t = indices[row % seq]
 *   out = e4m3(h / s), out_scale[row] = s = max(amax|h| / 448, FLT_MIN)
 * scale/shift are bf16 table rows (strides lds/ldsh); out_bf16 (optional)
 * receives h. width <= 6144. With out = out_scale = NULL (out_bf16 set) it
 * is the final layer's output AdaLN, norm_out + modulation
 * (x_diffusers/x_diffusers/framework/transformer/minimax_h3.py:672-696).
 * Replaces norm1/norm2 + `_apply(..., modulation=True)` of the H3 block
 * (x_base/x_base/operator/h3_indexed_affine.py:52-61,
 * x_diffusers/x_diffusers/framework/transformer/h3_npu_fusion.py:339-356)
 * plus the next FP8 Linear's activation quantisation. */
int xgb_norm_modulate_quant(const void* x, int64_t ldx, int64_t rows, int64_t width, int64_t seq,
                            int norm_kind, const void* weight, float eps, const void* scale,
                            int64_t lds, const void* shift, int64_t ldsh, const int64_t* indices,
                            uint8_t* out, float* out_scale, void* out_bf16, void* stream);

/* ---- Attention (tcgen05 / TMEM / TMA kernels) ---- */

/* Bytes of workspace xgb_sage_prepare needs (16-byte aligned; its contents
 * need no initialisation). */
int64_t xgb_sage_prepare_workspace(int64_t batch, int64_t heads, int64_t seq);

/* Sage quantisation of post-A2A Q/K/V views [batch, heads, seq, head_dim]
 * (element strides b, h, s, d with d = 1; bf16 or fp16), head_dim = 128:
 *   K <- K - mean over the seq real tokens (per head, per channel)
 *   Q <- Q * sm_scale * log2(e); Q, K int8 per 64-token block (amax/127)
 *   V e4m3 per channel: v_scale = max(amax/448, FLT_MIN)
 * Outputs (16-byte aligned): q8/k8/v8 [batch*heads][S_pad][128] with
 * S_pad = roundup(seq, 128) (rows >= seq zero), q_scale/k_scale
 * [batch*heads][S_pad/64], v_scale [batch*heads][128].
 * One cooperative kernel launch (one or two CTAs per SM) reads Q, K and V
 * once, quantises Q and gathers the K/V statistics, then quantises K and V;
 * its grid barriers give up after 2 s and record a timeout in *error_flag
 * (device int, may be NULL), as the attention kernels do.
 * Replaces the quantisation inside `sageattn` as called at
 * x_base/x_base/operator/attention.py:363-375 (SageAttention 2.2.0, not in
 * the reference tree; algorithm per the SageAttention2 paper). */
int xgb_sage_prepare(const void* q, const int64_t* q_strides, const void* k,
                     const int64_t* k_strides, const void* v, const int64_t* v_strides, int dtype,
                     int64_t batch, int64_t heads, int64_t seq, int64_t head_dim, float sm_scale,
                     int8_t* q8, float* q_scale, int8_t* k8, float* k_scale, uint8_t* v8,
                     float* v_scale, void* workspace, int64_t workspace_bytes, int* error_flag,
                     void* stream);

/* xgb_sage_prepare of bf16 Q/K/V with the rotate-half RoPE of the first
 * `rotary` channels of Q and K applied as they are read (rotary a multiple
 * of 16, <= 128): cos/sin fp32 [seq, rotary] (16-byte aligned rows of the
 * attention's sequence positions); each rotated value is
 * bf16(bf16(x*bf16(cos)) + bf16(+-partner*bf16(sin))), the reference's
 * rounding. Replaces `try_h3_partial_rope` (x_base/x_base/operator/
 * h3_partial_rope.py:9-47) followed by the quantisation inside `sageattn`
 * (x_base/x_base/operator/attention.py:363-375); the outputs equal
 * xgb_partial_rope + xgb_sage_prepare. Same workspace as xgb_sage_prepare. */
int xgb_sage_prepare_rope(const void* q, const int64_t* q_strides, const void* k,
                          const int64_t* k_strides, const void* v, const int64_t* v_strides,
                          int64_t batch, int64_t heads, int64_t seq, int64_t head_dim, float sm_scale,
                          const float* cos, const float* sin, int64_t rotary, int8_t* q8,
                          float* q_scale, int8_t* k8, float* k_scale, uint8_t* v8, float* v_scale,
                          void* workspace, int64_t workspace_bytes, int* error_flag, void* stream);

/* xgb_sage_prepare reading Q/K/V straight from a received PHAA FP8 wire
 * (the payload fp8_all_to_all_many exchanges, x_base/x_base/phaa/
 * fp8_transport.py:85-144, before its decode): per source peer p the Q, K
 * and V sections of rows [s < seq, batch, head] (128 e4m3 bytes + fp32
 * scale each), then peer_padding bytes. Attention row g < valid_seq is row
 * g % seq of peer g / seq; each value is read as bf16(e4m3 * scale), the
 * decode's result, so the outputs equal decode + xgb_sage_prepare on
 * [batch, heads, valid_seq, 128]. workspace: xgb_sage_prepare_workspace(
 * batch, heads, valid_seq) bytes; payload 4-byte aligned. */
int xgb_sage_prepare_wire(const uint8_t* payload, int64_t peers, int64_t seq, int64_t batch,
                          int64_t heads, int64_t valid_seq, int64_t peer_padding, float sm_scale,
                          int8_t* q8, float* q_scale, int8_t* k8, float* k_scale, uint8_t* v8,
                          float* v_scale, void* workspace, int64_t workspace_bytes, int* error_flag,
                          void* stream);

/* Non-causal attention over xgb_sage_prepare's outputs: INT8 Q.K^T
 * (tcgen05 kind::i8), fp32 online softmax in the exp2 domain, e4m3 P.V
 * (kind::f8f6f4), fp32 accumulation; writes bf16 out[b, h, s, :] at element
 * strides out_strides (b, h, s, d = 1). error_flag (device int, may be
 * NULL) receives a non-zero code if a bounded wait inside the kernel gave
 * up. Replaces `sageattn(q, k, v, tensor_layout="HND", is_causal=False)`,
 * x_base/x_base/operator/attention.py:363-375, via H3SageCUDA.__call__,
 * x_base/x_base/operator/h3_sage_cuda.py:21-25. */
int xgb_attention_sage(const int8_t* q8, const float* q_scale, const int8_t* k8,
                       const float* k_scale, const uint8_t* v8, const float* v_scale,
                       int64_t batch, int64_t heads, int64_t seq, void* out,
                       const int64_t* out_strides, void* split_workspace,
                       int64_t split_workspace_bytes, int* error_flag, void* stream);

/* Both attention entry points take an optional tail-split workspace
 * (xgb_attention_split_workspace_bytes() bytes, zeroed once by the caller;
 * NULL or smaller disables the split). A launch runs one CTA per (batch*
 * head, 256 query rows), one CTA per SM; the items of the last, partial
 * wave are split along the key range across the idle SMs and merged by the
 * last part to finish, so that wave costs a fraction of a full one. The
 * workspace is used stream-ordered: launches that share it must not overlap. */
int64_t xgb_attention_split_workspace_bytes(void);

/* ---- Sage quantisation before the SP exchange ("INT8 on the wire") ---- */

/* Per (peer, batch, head) of the rank's local rows, viewed like the FP8 wire
 * sources as [peers, seq, batch, heads] rows of 128 bf16 channels (element
 * strides *_strides[0..3], channel stride 1): channel sums of K after the
 * partial RoPE (rotary channels, cos/sin [seq, rotary] fp32, rotary a
 * multiple of 16 or 0) into ksum, and channel abs-maxima of V into vmax,
 * both [peers*batch*heads][128] fp32, in a fixed order. The caller
 * all-reduces them over the SP group (SUM, MAX) for sequence-wide values.
 * Part of the B200 "INT8 on the wire" exchange that replaces the FP8 wire
 * (x_base/x_base/phaa/fp8_transport.py:85-144) plus the attention-side
 * Sage quantisation. */
int64_t xgb_sage_wire_stats_workspace(int64_t peers, int64_t seq, int64_t batch, int64_t heads);
int xgb_sage_wire_stats(const void* k, const int64_t* k_strides, const void* v,
                        const int64_t* v_strides, int64_t peers, int64_t seq, int64_t batch,
                        int64_t heads, const float* cos, const float* sin, int64_t rotary,
                        float* ksum, float* vmax, void* workspace, int64_t workspace_bytes,
                        void* stream);

/* Quantise the rank's rows for the exchange (seq a multiple of 16): Q after
 * RoPE times sm_scale*log2(e) and K after RoPE minus ksum/seq_real, int8
 * per (head, group of 16 rows) with scale amax/127; V e4m3 per channel with
 * scale max(vmax/448, FLT_MIN). Writes q8/k8/v8 [peers][seq][batch][heads]
 * [128], qk_scale [peers][seq/16][batch][heads][2] (Q, K) and v_scale
 * [peers*batch*heads][128]; after an A2A over the peer dimension the
 * receiver passes them to xgb_attention_sage_strided unchanged. */
int xgb_sage_wire_encode(const void* q, const int64_t* q_strides, const void* k,
                         const int64_t* k_strides, const void* v, const int64_t* v_strides,
                         int64_t peers, int64_t seq, int64_t batch, int64_t heads,
                         const float* cos, const float* sin, int64_t rotary, float sm_scale,
                         const float* ksum, const float* vmax, int64_t seq_real, int8_t* q8,
                         int8_t* k8, uint8_t* v8, float* qk_scale, float* v_scale, void* stream);

/* xgb_attention_sage over quantised tensors in place: q8/k8/v8 rows of
 * (b, h, s) at byte offsets b*st[0] + h*st[1] + s*st[2] (multiples of 16),
 * Q/K scales per group of 16 rows at element offsets b*sst[0] + h*sst[1] +
 * (s/16)*sst[2], V scale rows at b*vst[0] + h*vst[1]; scale_rows (>= seq, a
 * multiple of 16) rows exist behind every (b, h); keys >= seq are masked.
 * Output and split workspace as xgb_attention_sage. */
int xgb_attention_sage_strided(const int8_t* q8, const int64_t* q_strides, const float* q_scale,
                               const int64_t* q_scale_strides, const int8_t* k8,
                               const int64_t* k_strides, const float* k_scale,
                               const int64_t* k_scale_strides, const uint8_t* v8,
                               const int64_t* v_strides, const float* v_scale,
                               const int64_t* v_scale_strides, int64_t batch, int64_t heads,
                               int64_t seq, int64_t scale_rows, void* out,
                               const int64_t* out_strides, void* split_workspace,
                               int64_t split_workspace_bytes, int* error_flag, void* stream);

/* Non-causal BF16 attention (tcgen05 kind::f16, fp32 accumulation) reading
 * q [b, h, seq_q, 128] and k/v [b, h, seq_kv, 128] views in place through
 * TMA (strides in elements, multiples of 8, d stride 1), scale sm_scale.
 * Replaces cuDNN SDPA in H3DenseCUDA.__call__,
 * x_base/x_base/operator/h3_dense_cuda.py:11-15. */
int xgb_attention_bf16(const void* q, const int64_t* q_strides, const void* k,
                       const int64_t* k_strides, const void* v, const int64_t* v_strides,
                       int64_t batch, int64_t heads, int64_t seq_q, int64_t seq_kv,
                       float sm_scale, void* out, const int64_t* out_strides,
                       void* split_workspace, int64_t split_workspace_bytes, int* error_flag,
                       void* stream);

#ifdef __cplusplus
}
#endif

#endif /* XGB_H_ */
