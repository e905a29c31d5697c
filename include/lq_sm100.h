/*
 * lq_sm100.h -- C ABI of liblq_sm100.so, the B200 (sm_100a) kernels behind the
 * llm_quant quantization hot path.
 *
 * Conventions
 *   - Every pointer is a device pointer (or a host pointer where named
 *     "host_"), every size is in elements unless the name says bytes.
 *   - The caller allocates every output and every workspace; the library
 *     never allocates device memory.  Its only mutable global state is the
 *     launch counter (lq_launch_count, atomic) and the fixed scratch array of
 *     lq_tensor_qparams_noalloc; every other entry point is re-entrant.
 *   - All work is enqueued on `stream` (a cudaStream_t, NULL = legacy default
 *     stream); no call synchronizes the host.
 *   - Every entry point returns an lq_status (0 = success).  On failure
 *     lq_last_error() gives a message for the calling host thread.
 *   - Floating-point semantics follow the reference's PyTorch CPU code: each
 *     elementwise op computes in fp32 and rounds (round-to-nearest-even) to
 *     the op's result dtype; reductions propagate NaN.
 *
 * Each entry point names the reference function (file:line of the
 * MindIntels/llm_quant source tree) whose behaviour it implements.
 */
#ifndef LQ_SM100_H_
#define LQ_SM100_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- element types ------------------------------------------------------ */
typedef enum {
  LQ_F32 = 0,
  LQ_F16 = 1,
  LQ_BF16 = 2,
  LQ_I8 = 3,
  LQ_I16 = 4,
  LQ_I32 = 5,
  LQ_I64 = 6,
  LQ_U8 = 7,
  LQ_U4X2 = 8 /* two 4-bit codes per byte, element 2i in the low nibble */
} lq_dtype;

/* ---- status codes --------------------------------------------------------- */
typedef enum {
  LQ_OK = 0,
  LQ_EINVAL = -1,   /* bad argument: shape, size, null pointer, bit width   */
  LQ_EDTYPE = -2,   /* unsupported dtype combination                        */
  LQ_ECUDA = -3,    /* a CUDA launch or runtime call failed                 */
  LQ_ETIMEOUT = -4, /* a bounded device-side wait ran out                   */
  LQ_EALIGN = -5,   /* pointer alignment the kernel requires is not met     */
  LQ_ERANGE = -6    /* size above a documented maximum                      */
} lq_status;

/* ---- modes of the fused quantization kernels ----------------------------- */
typedef enum {
  LQ_MODE_QPARAMS = 0, /* write scale / zero_point only                      */
  LQ_MODE_FAKE = 1,    /* quantize -> dequantize (fake_quantize value)       */
  LQ_MODE_CODES = 2    /* integer codes (round, clamp) + scale / zero_point  */
} lq_mode;

const char* lq_last_error(void);
const char* lq_status_string(int status);
int lq_version(void);
/* Number of kernels this library has enqueued from this process (all threads). */
uint64_t lq_launch_count(void);
/* Failure detection (the reference has no device code; its counterpart is the
 * bounded-wait requirement on every device-side spin-wait): probe of the
 * bounded mbarrier wait that the pipelined kernels use.  One warp waits on an
 * mbarrier that gets its arrival (arrive != 0) or never does, for at most
 * limit_ns (<= 10 s).  Writes out[0] = LQ_OK (the phase completed) or
 * LQ_ETIMEOUT (the wait gave up), out[1] = the wait's duration in ns
 * (out: 2 device int64).  The context stays usable after a timeout. */
int lq_wait_probe(int64_t limit_ns, int arrive, int64_t* out, void* stream);

/* ---- group / row quantization ---------------------------------------------
 * x is [rows, cols] row-major.  Each row is cut into ceil(cols/group)
 * groups of `group` columns; a ragged last group is padded with zeros that
 * take part in its min/max (core/quantizer.py:89-95).  group == cols gives
 * one group per row (PER_CHANNEL with channel_dim 0, per-token KV).
 *   scale, zero_point: [rows, n_groups] in x's dtype (n_groups = ceil(cols/group)).
 *   out (FAKE): [rows, cols] in x's dtype, value of fake_quantize
 *               (core/quantizer.py:143-185, STE rounding semantics).
 *   out (CODES): [rows, cols] codes = round(x/scale + zp).clamp(qmin, qmax)
 *               (core/quantizer.py:115-131 / kv_cache_quant.py:186-193) in
 *               out_dtype: LQ_I8, LQ_I16 or x's float dtype.
 * Replaces compute_qparams PER_GROUP / PER_CHANNEL (core/quantizer.py:41-108),
 * QuantizedLinear.quantize_weights (core/quantizer.py:231-260),
 * KVCacheQuantizer.quantize PER_TOKEN (kv_cache_quant.py:168-193). */
int lq_group_quant(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t group,
                   int n_bits, int symmetric, int mode, void* out, int out_dtype,
                   void* scale, void* zero_point, void* stream);

/* ---- fake_quantize backward ------------------------------------------------
 * grad_x of fake_quantize under autograd (core/quantizer.py:143-185 with
 * ste_round, core/quantizer.py:32-34): straight-through round, the clamp
 * mask, and the gradient through the group's scale (min / max, or max |x|,
 * distributed evenly over tied extrema; zero point has no gradient since it
 * comes from round).  Groups as in lq_group_quant (rows x cols, groups of
 * `group` columns, zero padding); PER_TENSOR is rows = 1, cols = group = n. */
int lq_fake_quant_backward(const void* x, const void* grad_out, int dtype, int64_t rows,
                           int64_t cols, int64_t group, int n_bits, int symmetric, void* grad_x,
                           void* stream);

/* ---- token-group (column) quantization --------------------------------------
 * x is [P, T, D] row-major; for every (p, d) the T tokens are cut into
 * ceil(T/tgroup) groups of `tgroup` tokens, zero-padded at the end
 * (kv_cache_quant.py:141-166).  tgroup >= T gives PER_CHANNEL
 * (kv_cache_quant.py:119-122).
 *   scale, zero_point: [P, n_tgroups, D] in x's dtype.
 *   out (CODES): [P, T, D] in LQ_I8 / LQ_I16 / x's dtype.
 *   out (FAKE):  [P, T, D] fp32 = (codes - zp) * scale computed in fp32
 *                (KVCacheQuantizer.fake_quantize, kv_cache_quant.py:269-276).
 * Replaces KVCacheQuantizer.quantize PER_CHANNEL / PER_GROUP
 * (kv_cache_quant.py:168-219). */
int lq_token_group_quant(const void* x, int x_dtype, int64_t P, int64_t T, int64_t D,
                         int64_t tgroup, int n_bits, int symmetric, int mode, void* out,
                         int out_dtype, void* scale, void* zero_point, void* stream);

/* ---- KV dequantization -------------------------------------------------------
 * out[p, t, d] = (float(codes[p, t, d]) - zp) * scale, computed in fp32
 * (KVCacheQuantizer.dequantize, kv_cache_quant.py:221-267).
 * codes: [P, T, D] with row pitch `codes_pitch_t` tokens per p (>= T, for a
 * cache stored with spare capacity); int8 or int16.
 * granularity 0 = per-token: scale/zp [P, sz_pitch_t] (one per token),
 *             1 = per-channel: scale/zp [P, D],
 *             2 = per-group: scale/zp [P, ceil(T/tgroup) pitch sz_pitch_t, D].
 * scale / zero_point dtype: s_dtype (f32/f16/bf16).  out: fp32 [P, T, D]. */
int lq_kv_dequant(const void* codes, int code_dtype, int64_t P, int64_t T, int64_t D,
                  int64_t codes_pitch_t, int granularity, int64_t tgroup, const void* scale,
                  const void* zero_point, int s_dtype, int64_t sz_pitch, float* out,
                  void* stream);

/* ---- KV-cache append ----------------------------------------------------------
 * The append half of QuantizedKVCache.update (kv_cache_quant.py:354-377) in
 * one pass: quantize the new chunk x [P, Tn, D] with the given granularity
 * (0 per-token, 1 per-channel, 2 per-group of `tgroup` tokens) and write its
 * codes (LQ_I8 / LQ_I16) into cache storage with spare capacity,
 * codes [P, codes_pitch_t, D] at token offset t_offset.  Scales / zero points
 * (x's dtype) go to
 *   per-token   [P, sz_pitch] at offset sz_offset,
 *   per-channel [P, D]: written when merge == 0, or max-merged into the stored
 *               values when merge == 1 (torch.maximum, as _cat_scales does,
 *               kv_cache_quant.py:395-402; old codes are not requantized),
 *   per-group   [P, sz_pitch, D] at group offset sz_offset. */
int lq_kv_append(const void* x, int x_dtype, int64_t P, int64_t Tn, int64_t D, int granularity,
                 int64_t tgroup, int n_bits, int symmetric, void* codes, int code_dtype,
                 int64_t codes_pitch_t, int64_t t_offset, void* scale, void* zero_point,
                 int64_t sz_pitch, int64_t sz_offset, int merge, void* stream);

/* ---- decode attention over the quantized cache ---------------------------------
 * out[b, hq, i, :] = softmax(q[b, hq, i, :] . K^T * sm_scale) V with K, V the
 * fp32 dequantization (code - zero) * scale of the cache storage above
 * (kv_cache_quant.py:221-267; the reference returns the whole dequantized
 * cache from update(), kv_cache_quant.py:379-382, and leaves attention to the
 * caller).  The codes are read in place; K / V are never materialized.
 *   q, out   [B, Hq, Sq, D] contiguous, q_dtype (f32 / f16 / bf16); query
 *            head hq reads kv head hq / (Hq / H).
 *   codes    [B*H, cap, D] (LQ_I8, or LQ_I16 with codes <= 1024), T tokens
 *            valid, cap a multiple of 16.
 *   *_gran   0 per-token: scale/zp [B*H, pitch] (pitch >= cap, pitch * size
 *              of s_dtype a multiple of 16 bytes),
 *            1 per-channel: scale/zp [B*H, D],
 *            2 per-group: scale/zp [B*H, pitch, D], *_group tokens per row
 *              (a multiple of 16).
 *   causal   1: query position i sees tokens t <= T - Sq + i.
 * Codes, scales and zero points must be 16-byte aligned.  When the work is
 * split along the tokens the call needs lq_kv_attention_workspace_bytes()
 * bytes of workspace (0 = none needed).  D = 64 or 128. */
size_t lq_kv_attention_workspace_bytes(int64_t B, int64_t Hq, int64_t H, int64_t Sq, int64_t D,
                                       int64_t T);
int lq_kv_attention(const void* q, int q_dtype, int64_t B, int64_t Hq, int64_t H, int64_t Sq,
                    int64_t D, int64_t T, int64_t cap, int code_dtype, const void* k_codes,
                    int k_gran, int64_t k_group, const void* k_scale, const void* k_zp,
                    int64_t k_pitch, const void* v_codes, int v_gran, int64_t v_group,
                    const void* v_scale, const void* v_zp, int64_t v_pitch, int s_dtype,
                    float sm_scale, int causal, void* out, void* workspace,
                    size_t workspace_bytes, void* stream);

/* ---- per-tensor qparams -------------------------------------------------------
 * compute_qparams PER_TENSOR (core/quantizer.py:63-72): scale = 0-dim,
 * zero_point = [1] (sym) or 0-dim (asym), both in x's dtype.  x is n
 * contiguous elements.  Needs a caller-provided workspace of at least
 * lq_tensor_qparams_workspace_size() bytes (16-byte aligned). */
size_t lq_tensor_qparams_workspace_size(int64_t n);
int lq_tensor_qparams(const void* x, int x_dtype, int64_t n, int n_bits, int symmetric,
                      void* scale, void* zero_point, void* workspace, size_t workspace_bytes,
                      void* stream);

/* lq_tensor_qparams without a workspace argument -- no counterpart in the
 * reference (which has no C interface); it exists for callers that cannot
 * allocate device memory (an FFI host that is handed tensor pointers by
 * another runtime and has no device allocator, or an application whose
 * device memory is all reserved by a framework allocator).  Same results as
 * lq_tensor_qparams.  Its partial results live in a fixed 128 KB array in
 * this library's device memory (held by every GPU that loads the library),
 * which limits n to 64 Mi elements (larger n: LQ_ERANGE).  All calls share
 * that array: calls whose kernels overlap on the GPU race.  The first call on
 * a device looks up the array's address (cudaGetSymbolAddress), so make it
 * before any stream capture.  The address is kept for the life of the
 * process: after a cudaDeviceReset of that device the array may move, so do
 * not call this entry point again in that process.  Allocates nothing. */
int lq_tensor_qparams_noalloc(const void* x, int x_dtype, int64_t n, int n_bits, int symmetric,
                              void* scale, void* zero_point, void* stream);

/* ---- per-channel reduction along an inner axis ---------------------------------
 * compute_qparams PER_CHANNEL with channel_dim != 0 (core/quantizer.py:74-85):
 * x is [outer, C, inner]; scale/zp [C] reduce over outer and inner.
 * Needs a workspace of lq_channel_qparams_workspace_size() bytes. */
size_t lq_channel_qparams_workspace_size(int64_t outer, int64_t C, int64_t inner);
int lq_channel_qparams(const void* x, int x_dtype, int64_t outer, int64_t C, int64_t inner,
                       int n_bits, int symmetric, void* scale, void* zero_point,
                       void* workspace, size_t workspace_bytes, void* stream);

/* ---- broadcast affine ops --------------------------------------------------------
 * Elementwise over a broadcast shape of `ndim` (<= 6) dims with per-operand
 * element strides (0 = broadcast).  op_dtypes[i] is the result dtype of the
 * i-th torch op (type promotion is resolved by the caller):
 *   LQ_AFFINE_QUANT   (quantize_tensor, core/quantizer.py:115-131):
 *       t = x / s  [op_dtypes[0]];  t = t + zp  [op_dtypes[1]];
 *       out = round(t).clamp(qmin, qmax)
 *   LQ_AFFINE_DEQUANT (dequantize_tensor, core/quantizer.py:134-140):
 *       t = x - zp [op_dtypes[0]];  out = t * s [op_dtypes[1]]
 *   LQ_AFFINE_FAKE    (fake_quantize with given qparams, core/quantizer.py:177-185):
 *       QUANT with STE rounding, then t = q - zp [op_dtypes[1]]; out = t * s [op_dtypes[1]]
 * x may be any lq_dtype except LQ_U4X2; out is a float dtype or LQ_I8/LQ_I16. */
typedef enum { LQ_AFFINE_QUANT = 0, LQ_AFFINE_DEQUANT = 1, LQ_AFFINE_FAKE = 2 } lq_affine_op;

/* ste_round forward value (core/quantizer.py:32-34): round half to even,
 * zero results as +0.0, +-inf -> NaN.  n contiguous elements. */
int lq_ste_round(const void* x, int dtype, int64_t n, void* out, void* stream);
int lq_affine(int op, int ndim, const int64_t* host_shape, const void* x, int x_dtype,
              const int64_t* host_x_strides, const void* scale, int s_dtype,
              const int64_t* host_s_strides, const void* zero_point, int z_dtype,
              const int64_t* host_z_strides, const int* host_op_dtypes, int n_bits,
              int symmetric, void* out, int out_dtype, void* stream);

/* ---- NF4 (qlora.py) ----------------------------------------------------------------
 * x: n contiguous elements grouped in blocks of `group` over the flattened
 * tensor, last block zero-padded (qlora.py:84-93).
 * lq_nf4_quantize: scales[n_groups] (x's dtype) = absmax.clamp(1e-12);
 *   codes = first argmin_i |x/scale - NF4_TABLE[i]| in fp32 (qlora.py:66-110);
 *   code_dtype LQ_I64 (the API's LongTensor), LQ_U8 or LQ_U4X2 (packed).
 * lq_nf4_dequantize: out = NF4_TABLE.to(s_dtype)[codes] * scales (qlora.py:113-157).
 * lq_double_quantize / lq_double_dequantize: qlora.py:164-196 / 199-223.
 * lq_nf4_pack: QLoRALinear.pack_base (qlora.py:281-292) in one pass:
 *   packed codes (LQ_U4X2, n/2 bytes), nf4 scales, and when dq_group > 0
 *   the double-quantized q_scales [n_groups] and dq_scales [ceil(n_groups/dq_group)].
 * lq_nf4_unpack: QLoRALinear._dequantize_base (qlora.py:294-304) in one pass:
 *   restores scales through double_dequantize when q_scales != NULL. */
int lq_nf4_quantize(const void* x, int x_dtype, int64_t n, int64_t group, void* codes,
                    int code_dtype, void* scales, void* stream);
int lq_nf4_dequantize(const void* codes, int code_dtype, int64_t n, int64_t group,
                      const void* scales, int s_dtype, void* out, void* stream);
int lq_double_quantize(const void* scales, int dtype, int64_t n, int64_t dq_group,
                       void* q_scales, void* dq_scales, void* stream);
int lq_double_dequantize(const void* q_scales, const void* dq_scales, int dtype, int64_t n,
                         int64_t dq_group, void* out, void* stream);
/* Convert n NF4 codes between containers (LQ_I64, LQ_U8, LQ_U4X2), e.g. the
 * int64 nf4_codes buffer of QLoRALinear's state_dict (qlora.py:264) and the
 * packed storage used on the device. */
int lq_codes_convert(const void* src, int src_dtype, int64_t n, void* dst, int dst_dtype,
                     void* stream);
int lq_nf4_pack(const void* x, int x_dtype, int64_t n, int64_t group, int64_t dq_group,
                uint8_t* packed_codes, void* scales, void* q_scales, void* dq_scales,
                void* stream);
int lq_nf4_unpack(const uint8_t* packed_codes, int64_t n, int64_t group, int64_t dq_group,
                  const void* scales, const void* q_scales, const void* dq_scales, int s_dtype,
                  void* out, void* stream);

/* ---- Walsh-Hadamard transform (core/rotation.py:130-147) ------------------------------
 * out = x @ hadamard_matrix(d, dtype) for x [rows, d], d a power of two
 * (2 <= d <= 32768), computed as an in-register/shared-memory butterfly in
 * fp32 and scaled by the dtype-rounded 1/sqrt(d) entry (core/rotation.py:30-43).
 * lq_hadamard_fake_quant additionally applies per-row fake quantization
 * (fake_quantize PER_CHANNEL on the [rows, d] result, core/quantizer.py:143-185)
 * to the dtype-rounded transform, as QuaRot.rotate_activation followed by
 * fake_quantize does (quarot.py:168-170). scale/zp may be NULL. */
int lq_hadamard(const void* x, int dtype, int64_t rows, int64_t d, void* out, void* stream);
int lq_hadamard_fake_quant(const void* x, int dtype, int64_t rows, int64_t d, int n_bits,
                           int symmetric, void* out, void* scale, void* zero_point,
                           void* stream);

/* ---- W4A16 QuantizedLinear forward (core/quantizer.py:262-280) ------------------------
 * Weights: QuantizedLinear's int8 codes [N, K] (n_bits <= 4: asymmetric codes
 * 0..15 or symmetric -8..7) with per-group scale / zero_point [N, K/group]
 * (f32 / f16 / bf16).  lq_w4a16_pack builds the kernel's packed operand
 * (lq_w4a16_packed_bytes() bytes, 16-byte aligned): 4-bit codes in 128-row x
 * 64-column tiles followed by per-(row, group) (zero + magic, scale) pairs in
 * the activation dtype.
 * lq_w4a16_linear: y[M, N] = x[M, K] @ dequant(W)^T + bias, x / y in act_dtype
 * (LQ_F16 or LQ_BF16), bias fp32 [N] or NULL, fp32 accumulation on the tensor
 * cores (M > 8: tcgen05.mma, A = weights dequantized into tensor memory, B =
 * activations by TMA; M <= 8: a weight-streaming mma.sync kernel).
 * Requires N % 128 == 0, K % 64 == 0, group % 64 == 0.
 * err (device int, may be NULL) receives a non-zero code if a bounded
 * device-side wait ran out (the kernel then returns early). */
size_t lq_w4a16_packed_bytes(int64_t N, int64_t K, int64_t group);
int lq_w4a16_pack(const int8_t* weight_int, const void* scale, const void* zero_point,
                  int s_dtype, int64_t N, int64_t K, int64_t group, int symmetric,
                  int act_dtype, void* packed, void* stream);
int lq_w4a16_linear(const void* x, int act_dtype, int64_t M, int64_t N, int64_t K,
                    int64_t group, const void* packed, const float* bias, void* y, int* err,
                    void* stream);

/* ---- NF4 linear (replaces QLoRALinear.forward's base path, qlora.py:306-312) --
 * The reference dequantizes the whole NF4 base weight (_dequantize_base,
 * qlora.py:294-304) and calls F.linear; here the table lookup and the block
 * scale are fused into the same GEMM kernels as lq_w4a16_linear.
 * lq_nf4_linear_pack builds the operand (lq_nf4_linear_packed_bytes() bytes,
 * 16-byte aligned) from the module's packed codes (LQ_U4X2 layout of the
 * flattened [N, K] weight) and its block scales: either `scales` [N*K/group],
 * or q_scales [N*K/group] + dq_scales [.. / dq_group] (the double
 * quantization, restored as round(round(q/127) * dq) in s_dtype, exactly as
 * _dequantize_base does).  Requires N % 128 == 0, K % 64 == 0,
 * group % 64 == 0 and K % group == 0.
 * lq_nf4_linear: y[M, N] = x[M, K] @ W^T + bias with W = round_T(NF4[code] *
 * scale), x / y in act_dtype (LQ_F16 or LQ_BF16), bias fp32 [N] or NULL, fp32
 * accumulation; err as for lq_w4a16_linear. */
size_t lq_nf4_linear_packed_bytes(int64_t N, int64_t K);
/* lq_nf4_linear_lora: QLoRALinear.forward whole (qlora.py:306-312): y =
 * x @ W^T + bias + u @ lora_b^T, the LoRA term in the same kernel (the
 * tensor-core path runs it as one more K step with lora_B's rows as the A
 * operand, the weight-streaming path as one more MMA pass per 16-row slab).
 * u = scaling * x @ lora_A^T [M, 64] in act_dtype (columns rank..63 zero),
 * lora_b [N, rank] in act_dtype; rank even, <= 16 for M > 8 and <= 64 for
 * M <= 8. */
int lq_nf4_linear_lora(const void* x, int act_dtype, int64_t M, int64_t N, int64_t K,
                       const void* packed, const float* bias, const void* lora_u,
                       const void* lora_b, int64_t rank, void* y, int* err, void* stream);
/* lq_nf4_qlora_forward: QLoRALinear.forward whole (qlora.py:306-312) in two
 * launches: lq_lora_u (u = scaling * x @ lora_a^T into the caller's u
 * workspace, [M, 64] act_dtype) and the fused kernel of lq_nf4_linear_lora,
 * which runs as a programmatic dependent of the first: its base product
 * starts while u is computed, only the LoRA step waits for u.  lora_a in
 * LQ_F32 or act_dtype, lora_b [N, rank] act_dtype; limits as for
 * lq_nf4_linear_lora. */
int lq_nf4_qlora_forward(const void* x, int act_dtype, int64_t M, int64_t N, int64_t K,
                         const void* packed, const float* bias, const void* lora_a, int a_dtype,
                         const void* lora_b, int64_t rank, float scaling, void* u, void* y, int* err,
                         void* stream);

/* lq_lora_u: the LoRA down-projection of QLoRALinear.forward (qlora.py:311,
 * F.linear(x, lora_A) * scaling) as the u operand of lq_nf4_linear_lora:
 * u[M, 64] (act_dtype) = scaling * x[M, K] @ lora_a[rank, K]^T in columns
 * 0..rank-1 and zeros in rank..63; fp32 accumulation on the tensor cores,
 * rounded once to act_dtype.  lora_a in LQ_F32 or act_dtype; K % 64 == 0,
 * 1 <= rank <= 64; x and lora_a 16-byte aligned.  Launched as a programmatic
 * dependent of the kernel ahead of it on the stream: it waits for that
 * kernel to complete before its first memory access, so stream order holds
 * as for an ordinary launch. */
int lq_lora_u(const void* x, int act_dtype, int64_t M, int64_t K, const void* lora_a, int a_dtype,
              int64_t rank, float scaling, void* u, void* stream);

/* lq_nf4_merge_lora: QLoRALinear.merge_lora (qlora.py:314-317) in one pass:
 * out [N, K] = W_base + scaling * lora_b @ lora_a with W_base exactly
 * _dequantize_base's (scales / double-quantized scales as in lq_nf4_unpack,
 * s_dtype), lora_a [rank, K] and lora_b [N, rank] in p_dtype, each op rounded
 * as torch rounds it; out_dtype = promote(s_dtype, p_dtype).  K % 8 == 0,
 * 1 <= rank <= 64. */
int lq_nf4_merge_lora(const uint8_t* packed_codes, int64_t N, int64_t K, int64_t group,
                      int64_t dq_group, const void* scales, const void* q_scales,
                      const void* dq_scales, int s_dtype, const void* lora_a,
                      const void* lora_b, int p_dtype, int64_t rank, float scaling, void* out,
                      int out_dtype, void* stream);
int lq_nf4_linear_pack(const void* codes, const void* scales, const void* q_scales,
                       const void* dq_scales, int s_dtype, int64_t N, int64_t K, int64_t group,
                       int64_t dq_group, int act_dtype, void* packed, void* stream);
int lq_nf4_linear(const void* x, int act_dtype, int64_t M, int64_t N, int64_t K,
                  const void* packed, const float* bias, void* y, int* err, void* stream);

/* ---- SpQR outliers (replaces the outlier restore of SpQRLinear.forward, spqr.py:191-193)
 * With the int part of the weight done by lq_w4a16_linear, the fp outliers are a
 * sparse correction C (outlier minus dequantized int weight at each masked
 * position) stored by rows: row_ids[n_rows] (int32), row_ptr[n_rows + 1]
 * (int32), cols[nnz] (int32), vals[nnz] (fp32).  lq_sparse_row_add adds it:
 * y[m, row_ids[r]] += sum_j x[m, cols[j]] * vals[j] over j in
 * [row_ptr[r], row_ptr[r+1]), summed in fp32 and rounded once into y.
 * x [M, K] and y [M, N] row-major in dtype (LQ_F32 / LQ_F16 / LQ_BF16). */
int lq_sparse_row_add(const void* x, int dtype, int64_t M, int64_t K, int64_t N,
                      const int32_t* row_ptr, const int32_t* row_ids, int64_t n_rows,
                      const int32_t* cols, const float* vals, void* y, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* LQ_SM100_H_ */
