/*
 * faquant_b200.h -- C ABI of libfaquant_b200.so, the B200 (sm_100a) kernels behind
 * FAQUANT's two HiF4 hot paths: the W4A4 quantized Linear and the HiF4 QK/PV
 * flash attention.
 *
 * Conventions (every entry point):
 *  - returns FAQ_OK (0) or a FAQ_ERR_* code; faq_last_error() gives the message
 *    of the calling thread's last failure;
 *  - all pointers are device pointers unless stated, sizes and strides are in
 *    ELEMENTS, the innermost dimension is contiguous;
 *  - `stream` is a cudaStream_t (NULL = legacy default stream); work is
 *    stream-ordered, the calls are thread-safe across streams and never
 *    synchronize the device;
 *  - the library allocates no device memory: every output is caller-owned;
 *  - arguments are validated on the host; a device-side wait that exceeds its
 *    time limit records FAQ_STATUS_TIMEOUT in a status word read by
 *    faq_device_status() (kernels never trap).
 *
 * Packed HiF4 storage format (this project's own; the reference stores only
 * bf16 dequantized values plus fp32/int8 metadata, qad_checkpoint.py:43-48):
 *  - codes: uint8 [rows, K64/2], K64 = K rounded up to 64. Value 2i is the low
 *    nibble and value 2i+1 the high nibble of byte i; nibble = sign<<3 | m with
 *    sign = (x < 0) and m in 0..7 the element magnitude in quarters;
 *  - meta:  uint32 [rows, K64/64], one word per 64-value block:
 *      bits  0-7 : E6M2 scale code, (e + 48) << 2 | t, scale = (1 + t/4) * 2^e;
 *      bits  8-15: lv2 exponent bit of each 8-value sub-block;
 *      bits 16-31: lv3 exponent bit of each 4-value sub-block;
 *  - value = (-1)^sign * (m / 4) * scale * 2^(lv2 + lv3).
 */
#ifndef FAQUANT_B200_H_
#define FAQUANT_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define FAQ_OK 0
#define FAQ_ERR_ARG 1         /* invalid argument (shape, stride, alignment, null) */
#define FAQ_ERR_CUDA 2        /* a CUDA runtime/driver call failed */
#define FAQ_ERR_UNSUPPORTED 3 /* valid for the reference, not supported by these kernels */
#define FAQ_ERR_TIMEOUT 4     /* a device-side wait ran out (see faq_device_status) */

/* device status word bits */
#define FAQ_STATUS_TIMEOUT 1u

/* element types */
#define FAQ_BF16 0
#define FAQ_F32 1

/* HiF4 scale-level variants (src/faquant/hif4.py:13-43) */
#define FAQ_LEVELS_123 123
#define FAQ_LEVELS_12 12
#define FAQ_LEVELS_13 13

/* activations fused into faq_hif4_quantize_act */
#define FAQ_ACT_NONE 0
#define FAQ_ACT_SWIGLU 1    /* x [rows, 2k] = gate | up: bf16(bf16(silu(gate)) * up) (Qwen3MLP) */
#define FAQ_ACT_GELU_TANH 2 /* x [rows, k]: the tanh GELU rounded to bf16 (the DiT FFN) */

/* Version of the library as major*10000 + minor*100 + patch. */
int faq_version(void);

/* Copy the calling thread's last error message into buf (NUL-terminated). */
int faq_last_error(char* buf, size_t len);

/* Read the device status word of the current device into *status; clear it
 * when `reset` is non-zero. Synchronizes with the legacy default stream. */
int faq_device_status(unsigned int* status, int reset);

/*
 * K1 -- activation rotation + HiF4 quantization, rows of x [rows, k] (row stride ldx).
 *
 * Replaces the input path of FakeQuantLinear.forward (src/faquant/quantization.py:200-221
 * and :267-274): optional per-channel input_scale multiplied in x's dtype
 * (:200-201); when `signs` is given, x*signs in fp32 (int8 [k]), a gather by
 * `perm` (int64 [k], NULL = identity), an fp32 Walsh-Hadamard over consecutive
 * blocks of `rot_block` (a power of two 1..1024 dividing k; 0 = no Hadamard)
 * normalized by 1/sqrt(rot_block) (rotation.py:14-29, 117-135) and one rounding
 * to x's dtype; then HiF4 quantization along k in blocks of 64 with a
 * zero-padded tail (hif4.py:376-390), `levels` in {123, 12, 13}.
 * Outputs (any may be NULL, not all): packed `codes`/`meta` (format above) and
 * the dequantized values `qdq` [rows, ldq] in x's dtype (bit-exact with the
 * reference's fake_quantize output).
 */
int faq_hif4_quantize(const void* x, int x_dtype, int64_t rows, int64_t k, int64_t ldx,
                      const void* input_scale, const int8_t* signs, const int64_t* perm,
                      int rot_block, int levels, uint8_t* codes, uint32_t* meta, void* qdq,
                      int64_t ldq, void* stream);
/*
 * K1 with the decoder layer's RMSNorm fused in front (the "per norm" HiSQ readers of a
 * Qwen3 layer: input_layernorm -> q/k/v, post_attention_layernorm -> gate/up): each row
 * x [rows, k] bf16 is normalized as faq_rms_norm does, bf16(w * bf16(x * rsqrt(mean(x^2)
 * + eps))) with the same fp32 summation order, so the same bits, then (optionally
 * times input_scale, rounded) rotated with signs / perm / rot_block and HiF4-quantized
 * exactly as faq_hif4_quantize. The normalized tensor never goes to memory. Replaces the
 * pair Qwen3RMSNorm (modeling_qwen3 as the reference's models use it) then the input
 * path of FakeQuantLinear.forward (src/faquant/quantization.py:200-221). bf16 only.
 * Outputs as faq_hif4_quantize's (any may be NULL, not both codes and qdq): packed
 * `codes` [rows, k/2] (16-byte aligned, row stride k/2), `meta` [rows, k/64] and the
 * dequantized `qdq` [rows, ldq]; codes alone are what a sequence-parallel caller
 * all-gathers (0.5625 bytes per value instead of 2). FAQ_ERR_UNSUPPORTED unless
 * k % 1024 == 0, k <= 16384 and 32 <= rot_block <= 1024.
 */
int faq_hif4_quantize_rms_norm(const void* x, int64_t rows, int64_t k, int64_t ldx, const void* norm_weight,
                               float eps, const void* input_scale, const int8_t* signs, const int64_t* perm,
                               int rot_block, int levels, uint8_t* codes, uint32_t* meta, void* qdq, int64_t ldq,
                               void* stream);
/*
 * The same with the Wan DiT block's affine-free LayerNorm in front (norm1 -> qkv, norm2
 * -> ffn.0; the rbhn_r64 readers): bf16((x - mean) * rsqrt(var + eps)), biased
 * variance, summed in faq_layer_norm's order, so the same bits as faq_layer_norm then
 * faq_hif4_quantize. Replaces WanLayerNorm (the reference's Wan checkout, elementwise_affine
 * False) then HiF4Linear's input quantization (src/faquant/wan22_hif4.py:81-92). Same
 * limits as faq_hif4_quantize_rms_norm.
 */
int faq_hif4_quantize_layer_norm(const void* x, int64_t rows, int64_t k, int64_t ldx, float eps,
                                 const void* input_scale, const int8_t* signs, const int64_t* perm, int rot_block,
                                 int levels, uint8_t* codes, uint32_t* meta, void* qdq, int64_t ldq, void* stream);

/*
 * faq_hif4_quantize of an activation's output, the activation fused into the load: `act`
 * FAQ_ACT_SWIGLU reads x [rows, 2k] (gate in columns 0..k-1, up in k..2k-1) and quantizes
 * bf16(bf16(silu(gate)) * up); FAQ_ACT_GELU_TANH reads x [rows, k] and quantizes its tanh
 * GELU rounded to bf16 -- the same values faq_silu_mul / faq_gelu_tanh write, so the
 * outputs are those of the activation followed by faq_hif4_quantize, without the
 * activation's [rows, k] tensor in HBM. bf16 only, signs-only rotations (`signs`, 8-byte
 * aligned, with rot_block 8..256) -- the row-parallel down_proj / ffn.2 inputs; k % 64 == 0,
 * 16-byte aligned rows. No counterpart in the reference (separate passes there).
 */
int faq_hif4_quantize_act(const void* x, int act, int64_t rows, int64_t k, int64_t ldx,
                          const void* input_scale, const int8_t* signs, int rot_block, int levels,
                          uint8_t* codes, uint32_t* meta, void* qdq, int64_t ldq, void* stream);

/* Dequantize packed HiF4 rows back to out [rows, ldo] (bf16 or fp32).
 * The inverse of the packing above; replaces expand_hif4_parameters +
 * quantize_hif4_with_parameters (hif4.py:222-271) for stored codes. */
int faq_hif4_dequantize(const uint8_t* codes, const uint32_t* meta, int64_t rows, int64_t k,
                        void* out, int out_dtype, int64_t ldo, void* stream);

/*
 * K2 -- pack HiF4-grid weights w [n, k] (bf16 or fp32, row stride ldw) into codes/meta.
 * With `scale` (fp32 [n, k/64]), `lv2` (int8 [n, k/64, 8]) and `lv3` (int8 [n, k/64, 16])
 * -- the compact metadata GPTQ records (gptq.py:411-423, 562-570) -- codes are
 * round(|w| / dequant_scale * 4) clamped to 0..7 (hif4.py:311). Without them the
 * metadata is fitted from w as the RTN quantizer does (FakeQuantLinear.__init__,
 * quantization.py:169-184), so w must be the source (unquantized) weight: RTN is
 * not idempotent, re-fitting an already quantized block can pick another scale.
 * Every value that the packed form does not reproduce exactly increments
 * *mismatches (device int64, caller-zeroed; may be NULL): zero for an on-grid
 * weight with its metadata, the number of changed values for an RTN source.
 */
int faq_hif4_pack_weight(const void* w, int w_dtype, int64_t n, int64_t k, int64_t ldw,
                         const float* scale, const int8_t* lv2, const int8_t* lv3, int levels,
                         uint8_t* codes, uint32_t* meta, unsigned long long* mismatches,
                         void* stream);

/*
 * K3 -- y [m, n] = a [m, k] . b [n, k]^T (+ bias [n]); bf16 operands and output,
 * fp32 accumulation on tcgen05 tensor cores (TMEM accumulators, TMA loads).
 * Replaces F.linear(x_qdq, weight, bias) (quantization.py:277, wan22_hif4.py:88)
 * on exactly-dequantized HiF4 operands. Needs lda, ldb multiples of 8, 16-byte
 * aligned a/b and k a multiple of 8. Shapes with m >= 256 and n >= 256 run on clusters
 * of two CTAs (tcgen05.mma.cta_group::2, 256 x 256 tiles), smaller ones on one CTA per
 * SM; both give the same bits (FAQ_GEMM_ONE_SM=1 in the environment keeps the latter).
 */
int faq_gemm_bf16_tn(const void* a, int64_t lda, const void* b, int64_t ldb, int64_t m,
                     int64_t n, int64_t k, const void* bias, void* y, int64_t ldy, void* stream);
/*
 * faq_gemm_bf16_tn with the residual add of a decoder layer in the epilogue:
 * y = bf16(bf16(a . b^T + bias) + residual), residual [m, n] bf16 with leading dimension
 * ldr -- the same bits as the GEMM followed by the eager bf16 add
 * `hidden = residual + o_proj(x)` of Qwen3DecoderLayer (and Wan's x + attn / x + ffn).
 * residual may be null (then it is faq_gemm_bf16_tn). No counterpart in the reference,
 * which adds in a separate elementwise pass.
 */
int faq_gemm_bf16_tn_residual(const void* a, int64_t lda, const void* b, int64_t ldb, int64_t m,
                              int64_t n, int64_t k, const void* bias, const void* residual, int64_t ldr,
                              void* y, int64_t ldy, void* stream);
/*
 * The number of SMs the persistent GEMMs (faq_gemm_bf16_tn*, faq_w4a4_gemm*) size their
 * grids for, from the next launch on (0, the default: every SM of the device; values
 * above the SM count mean every SM). Process-wide and read on the host at launch, not
 * stream-ordered. For callers that run collectives (NCCL) beside the GEMMs on another
 * stream: a GEMM grid over every SM leaves no SM for the collective's kernels until the
 * GEMM drains. The result bits do not depend on it. The counterpart of cuBLAS's
 * cublasSetSmCountTarget; no counterpart in the reference.
 */
int faq_set_gemm_sm_target(int sms);

/*
 * K3p -- the W4A4 GEMM on packed HiF4 operands: y [m, n] = deq(a) . deq(b)^T (+ bias [n])
 * (+ residual [m, n], ldr), bf16 output, where a [m, k] and b [n, k] are in the packed
 * format above (codes uint8 [rows, k/2] and meta uint32 [rows, k/64], rows contiguous)
 * -- K1's `codes`/`meta` for the activations, K2's
 * for the weights. The tensor cores read bf16 tiles expanded from the packed bytes in
 * shared memory, so HBM holds and moves 4.5 bits per operand value; the result is
 * bit-identical to faq_gemm_bf16_tn(_residual) on the dequantized operands, which is
 * F.linear on the reference's fake-quantized tensors (src/faquant/quantization.py:277 with
 * hif4.py:254-271 for both operands). k must be a multiple of 256 (the meta rows are
 * loaded by TMA, which needs 16-byte rows; FAQ_ERR_UNSUPPORTED otherwise), codes and meta
 * 16-byte aligned. Replaces, with
 * faq_hif4_quantize writing codes, FakeQuantLinear.forward's quantize-then-F.linear
 * (quantization.py:267-277).
 */
int faq_w4a4_gemm(const uint8_t* a_codes, const uint32_t* a_meta, const uint8_t* b_codes,
                  const uint32_t* b_meta, int64_t m, int64_t n, int64_t k, const void* bias,
                  const void* residual, int64_t ldr, void* y, int64_t ldy, void* stream);
/*
 * faq_w4a4_gemm with the activation operand given as its exact bf16 dequantization
 * a [m, lda] (faq_hif4_quantize's `qdq` output; lda >= k, a multiple of 8, 16-byte aligned)
 * and the weight packed: for callers that keep the QDQ activation (the same bits as
 * faq_w4a4_gemm on the activation's codes). For m <= 16 (decode) it runs a small-row kernel
 * that streams the packed weight into register-fragment MMAs, split over K inside each
 * CTA and summed in a fixed order: deterministic, equal to the tiled GEMM up to fp32
 * rounding of the sums (another summation order), not bit for bit.
 */
int faq_w4a4_gemm_qdq_a(const void* a, int64_t lda, const uint8_t* b_codes, const uint32_t* b_meta,
                        int64_t m, int64_t n, int64_t k, const void* bias, const void* residual,
                        int64_t ldr, void* y, int64_t ldy, void* stream);

/*
 * K4 -- attention operand preparation for one of Q, K or V.
 * x is [batch, heads, seq, d] with element strides (sb, sh, ss) and d contiguous,
 * bf16 or fp32. Replaces the post-RoPE block of qwen3._attention_forward
 * (src/faquant/qwen3.py:101-130), Wan's self_forward/rotate_heads
 * (wan22_attention.py:186-192, 257-259) and the operand QDQ of the simulator
 * (simulated_flash_attention.py:588-619): in fp32, x - offset (fp32 [heads, d],
 * K only), then x * smooth (smooth_mode 1, Q) or x / smooth (smooth_mode 2, K)
 * with smooth fp32 [d] (smooth_head_stride 0) or [heads, d]; a normalized
 * Hadamard over d when `rotate` (d a power of two <= 128); one rounding to bf16;
 * then, when `levels` != 0, HiF4 quantization along d. Output bf16 with strides
 * (ob, oh, os); optional packed codes/meta for the rows in (b, h, s) order.
 */
int faq_qk_prep(const void* x, int x_dtype, int64_t batch, int64_t heads, int64_t seq, int d,
                int64_t sb, int64_t sh, int64_t ss, const float* offset, const float* smooth,
                int64_t smooth_head_stride, int smooth_mode, int rotate, int levels, void* out,
                int64_t ob, int64_t oh, int64_t os, uint8_t* codes, uint32_t* meta, void* stream);

/*
 * K4 with Qwen3's pre-RoPE steps in front: the per-head RMSNorm of q_norm/k_norm
 * (HF Qwen3RMSNorm over d: fp32 mean of squares, rsqrt, bf16, times the bf16
 * `norm_weight` [d], bf16; skipped when null) and RoPE as HF apply_rotary_pos_emb
 * computes it in bf16 (x cos + rotate_half(x) sin, each product and the sum rounded)
 * with bf16 tables cos/sin [seq, rope_ld] indexed by the sequence position (skipped
 * when null), then everything faq_qk_prep does. Replaces the q_norm/k_norm + RoPE +
 * post-RoPE transform of qwen3._attention_forward (src/faquant/qwen3.py:87-130) in one
 * HBM pass.
 */
int faq_qk_norm_rope_prep(const void* x, int x_dtype, int64_t batch, int64_t heads, int64_t seq, int d,
                          int64_t sb, int64_t sh, int64_t ss, const void* norm_weight, float eps,
                          const void* cos, const void* sin, int64_t rope_ld, const float* offset,
                          const float* smooth, int64_t smooth_head_stride, int smooth_mode, int rotate,
                          int levels, void* out, int64_t ob, int64_t oh, int64_t os, uint8_t* codes,
                          uint32_t* meta, void* stream);

/*
 * K4 for Wan2.2's self-attention q/k (wan22_attention.py:250-258: norm_q/norm_k, Wan's
 * rope_apply, the optional faquant_qk_smooth_scale, then make_flash_attention's
 * rotate_heads and input_qdq): x bf16 [batch, heads, seq, d] with element strides.
 * head_ss holds the per-head sums of squares of all heads_total heads of the layer
 * (faq_row_sumsq with seg_cols = d; on a head shard all-gathered over the ranks): head
 * g of token t at head_ss[(g / heads_per_block) * ss_block_stride + t * ss_token_stride
 * + g % heads_per_block]. They are added in a fixed order, so the norm does not depend
 * on the sharding. norm_weight fp32 [heads, d] this shard's weight; pair_cos/pair_sin
 * fp64 [seq, d/2] (or null) the 3-axis RoPE table. v = bf16(x * rsqrt(sum / (heads_total
 * d) + eps)) * w, the RoPE in fp64 rounded to fp32, smooth (as faq_qk_prep), Hadamard,
 * one bf16 rounding, HiF4.
 */
int faq_wan_qk_prep(const void* x, int64_t batch, int64_t heads, int64_t seq, int d, int64_t sb, int64_t sh,
                    int64_t ss, const float* head_ss, int64_t heads_total, int64_t heads_per_block,
                    int64_t ss_token_stride, int64_t ss_block_stride, const float* norm_weight, float eps,
                    const double* pair_cos, const double* pair_sin, const float* smooth,
                    int64_t smooth_head_stride, int smooth_mode, int rotate, int levels, void* out, int64_t ob,
                    int64_t oh, int64_t os, void* stream);

/*
 * Decoder glue, one HBM pass each (bf16, 16-byte aligned rows, strides in elements):
 * faq_rms_norm: out = bf16(w * bf16(x * rsqrt(mean(x^2) + eps))) per row of k, as HF
 *   Qwen3RMSNorm (the input_layernorm/post_attention_layernorm the reference's Qwen3
 *   decoder layers apply before the projections K1 quantizes);
 * faq_silu_mul: out[:, j] = bf16(bf16(silu(gu[:, j])) * gu[:, f + j]) for a gate|up
 *   tensor of 2f columns, as Qwen3MLP's act_fn(gate) * up;
 * faq_layer_norm: out = bf16((x - mean) * rsqrt(var + eps)) per row of k (biased
 *   variance, no affine), as the Wan DiT block's WanLayerNorm norm1/norm2 in fp32;
 * faq_gelu_tanh: out = bf16(0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))), the
 *   Wan FFN's GELU(approximate="tanh");
 * faq_row_sumsq: out[r * segments + s] = sum of x[r, s * seg_cols + c]^2 over c, fp32,
 *   for `segments` adjacent column segments (the q and k heads of a fused qkv projection).
 */
int faq_rms_norm(const void* x, int64_t rows, int64_t k, int64_t ldx, const void* weight, float eps,
                 void* out, int64_t ldo, void* stream);
int faq_silu_mul(const void* gate_up, int64_t rows, int64_t f, int64_t ld, void* out, int64_t ldo,
                 void* stream);
int faq_layer_norm(const void* x, int64_t rows, int64_t k, int64_t ldx, float eps, void* out, int64_t ldo,
                   void* stream);
int faq_gelu_tanh(const void* x, int64_t rows, int64_t cols, int64_t ld, void* out, int64_t ldo, void* stream);
int faq_row_sumsq(const void* x, int64_t rows, int64_t segments, int64_t seg_cols, int64_t ld, float* out,
                  void* stream);

/*
 * K5 -- HiF4 QK/PV flash attention on pre-quantized bf16 operands (output of K4).
 * q [batch, hq, sq, 128], k/v [batch, hkv, sk, 128] with element strides, d contiguous;
 * out [batch, sq, hq, 128] bf16 with element strides (ob, os, oh).
 * Replaces simulated_flash_attention_forward (simulated_flash_attention.py:457-909,
 * no mask) and Wan's hif4_attention (wan22_attention.py:165-183): scores
 * q.k^T * scale in fp32, bottom-right causal mask when `causal`, online softmax
 * over key tiles of 128 against the running max, HiF4 quantization of
 * P = exp(s - max) along each tile's keys in groups of 64 (`p_levels`, 0 = no P
 * quantization), the denominator from the quantized P when
 * `normalizer_quantized` (P-Reordering) else from the unquantized P, fp32 PV
 * accumulation, out = acc / denominator. GQA maps q head h to kv head
 * h / (hq / hkv) (simulated_flash_attention.py:231-240).
 */
int faq_hif4_attention(const void* q, const void* k, const void* v, int64_t batch, int64_t hq,
                       int64_t hkv, int64_t sq, int64_t sk, int d, int64_t qb, int64_t qh,
                       int64_t qs, int64_t kb, int64_t kh, int64_t ks, int64_t vb, int64_t vh,
                       int64_t vs, float scale, int causal, int p_levels, int normalizer_quantized,
                       void* out, int64_t ob, int64_t os, int64_t oh, void* stream);

/*
 * K6 -- HiF4 attention decode: sq (<= 32 / (hq / hkv)) new query positions against a
 * cache of sk keys, the queries being the last sq positions (bottom-right causal).
 * Same semantics and operand contract as faq_hif4_attention (pre-quantized bf16 Q/K/V;
 * out [batch, sq, hq, 128]), the decode call of simulated_flash_attention_forward
 * (simulated_flash_attention.py:457-909 with a growing cache). The keys are split over
 * the GPU in three kernels (scores and per-tile row maxima; P and P.V per split of 2-16
 * key tiles starting from the exact running max before the split, so every tile's HiF4 P
 * is the sequential one; the join of the splits). `workspace` is a caller-owned device
 * buffer of at least faq_hif4_decode_workspace_bytes(...) bytes (scores, tile maxima and
 * per-split partial results); it needs no initialization.
 */
size_t faq_hif4_decode_workspace_bytes(int64_t batch, int64_t hq, int64_t hkv, int64_t sq, int64_t sk, int d);
int faq_hif4_decode_attention(const void* q, const void* k, const void* v, int64_t batch, int64_t hq,
                              int64_t hkv, int64_t sq, int64_t sk, int d, int64_t qb, int64_t qh,
                              int64_t qs, int64_t kb, int64_t kh, int64_t ks, int64_t vb, int64_t vh,
                              int64_t vs, float scale, int p_levels, int normalizer_quantized, void* out,
                              int64_t ob, int64_t os, int64_t oh, void* workspace, size_t workspace_bytes,
                              void* stream);

/*
 * faq_hif4_decode_attention without a workspace argument, for callers that cannot
 * allocate device memory (a runtime that plans all of its memory at start-up and forbids
 * allocations while serving; a host hot path where cudaMalloc would synchronize the
 * device). No counterpart in the reference: it is this library's allocation-free variant.
 * Its scratch is one file-scope device array of FAQ_DECODE_STATIC_SCRATCH_BYTES that
 * every GPU loading the library holds until exit; problems whose
 * faq_hif4_decode_workspace_bytes(...) exceeds it are rejected with FAQ_ERR_ARG. The
 * array's address is looked up on the first call on each device (make that call before
 * any stream capture). Under lazy module loading (the CUDA default) that first call is
 * also when the driver loads the library's module onto the device, which is what places
 * the array in device memory: make it at start-up. `stream` must belong to the current
 * device (FAQ_ERR_ARG otherwise) and to its primary context. Nothing in the array must
 * start at zero; calls that may overlap on one GPU share the array and race -- order them.
 */
#define FAQ_DECODE_STATIC_SCRATCH_BYTES ((size_t)16 << 20)
int faq_hif4_decode_attention_static(const void* q, const void* k, const void* v, int64_t batch,
                                     int64_t hq, int64_t hkv, int64_t sq, int64_t sk, int d,
                                     int64_t qb, int64_t qh, int64_t qs, int64_t kb, int64_t kh,
                                     int64_t ks, int64_t vb, int64_t vh, int64_t vs, float scale,
                                     int p_levels, int normalizer_quantized, void* out, int64_t ob,
                                     int64_t os, int64_t oh, void* stream);

/*
 * GPTQ with HiF4 grids (offline weight production): the per-column loop of one block of
 * `cols` (64 or 128) columns for every row of w, as GPTQ.quantize does it
 * (src/faquant/gptq.py:417-548; block-diagonal form :197-298). w [rows, ldw] fp32 holds
 * the block's current values at column b * cols for block b < nblocks (nblocks > 1: the
 * independent groups of the block-diagonal form); hinv: block b's [cols x cols] upper
 * inverse Cholesky factor at hinv + b * hinv_stride, row stride ldh. At each 64-column
 * group start the HiF4 metadata is fitted from the group's current values
 * (fit_hif4_compact_parameters, `levels`) and written to scale/rec ([rows,
 * groups_per_row] fp32, the block's first group at column b * cols / 64), lv2 ([.., 8]) and
 * lv3 ([.., 16]) int8; then per column: q = the HiF4 value, e = (w - q) / hinv[c][c],
 * w[j] -= e * hinv[c][j] for j >= c, each step one fp32 rounding as in the reference.
 * Writes the quantized values to q and the errors to err (same layout as w); w is not
 * modified. The caller applies the lazy update of later columns, w[:, stop:] -= err @
 * H^-1[block, stop:], with any fp32 GEMM.
 */
int faq_gptq_hif4_block(const float* w, int64_t ldw, int64_t rows, int cols, int64_t nblocks,
                        const float* hinv, int64_t ldh, int64_t hinv_stride, int levels, float* q,
                        int64_t ldq, float* err, int64_t lde, float* scale, float* rec, int8_t* lv2,
                        int8_t* lv3, int64_t groups_per_row, void* stream);

/* Diagnostics: copy up to max_records records of the waits that gave up (3 words
 * each: site | tile << 8, blockIdx.x | blockIdx.y << 16, blockIdx.z) into `records`
 * (host memory); returns the number of timeouts recorded (>= 0) or -FAQ_ERR_*.
 * Clears the record count when `reset` is non-zero. */
int faq_device_trace(unsigned int* records, int max_records, int reset);

/* Diagnostics: launch one CTA that waits on an mbarrier nothing arrives at, for
 * at most `limit_ns` nanoseconds, then records FAQ_STATUS_TIMEOUT and returns.
 * Exercises the bounded-wait path of the kernels without faulting the GPU. */
int faq_selftest_wait_timeout(int64_t limit_ns, void* stream);

/* Diagnostics (no counterpart in the reference): evaluates ex2.approx.ftz on every
 * float in [-inf, 1] in increasing order and stores in *violations the number of
 * consecutive pairs whose results decrease. K5 takes the HiF4 scale of each 64-key group
 * of P from the group's largest score, which equals the largest P only when this is 0. */
int faq_selftest_ex2_monotone(uint64_t* violations, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FAQUANT_B200_H_ */
