// K4 -- attention operand preparation: (offset) -> Smooth-QK -> Hadamard over
// head_dim -> one bf16 rounding -> HiF4 along head_dim, for Q, K or V.
//
// Reference: qwen3._attention_forward (src/faquant/qwen3.py:101-130) computes, in one
// fp32 excursion, k - offset, q * s, k / s (true division), hadamard_transform over
// head_dim (rotation.py:14-29, whose final `/ sqrt(128)` is a correctly rounded fp32
// divide), and a single cast to bf16; the simulator then fake-quantizes Q/K/V along
// head_dim (simulated_flash_attention.py:588-619). Wan does the same
// (wan22_attention.py:186-192, 221, 257-259).
//
// faq_wan_qk_prep does the same for Wan's self-attention (wan22_attention.py:250-258
// with Wan's WanRMSNorm and rope_apply): the RMSNorm over all heads of a token from
// per-head sums of squares, the 3-D RoPE in fp64 rounded to fp32, then the steps above.
//
// The fused entry point faq_qk_norm_rope_prep puts Qwen3's own steps in front
// (qwen3.py:87-100 with HF Qwen3Attention): the per-head RMSNorm over head_dim
// (Qwen3RMSNorm: fp32 mean of squares, rsqrt, cast to bf16, times the bf16 weight, cast)
// and RoPE in bf16 as HF's apply_rotary_pos_emb does it (bf16(q cos) + bf16(rotate_half(q)
// sin), rounded; rotate_half's partner channel is d/2 away, i.e. d/16 lanes).
//
// Mapping: d/8 lanes per (b, h, s) row, 8 consecutive channels per lane, so the
// Hadamard strides 1, 2, 4 are inside a lane and 8 .. d/2 are lane shuffles, and
// the HiF4 64-blocks are 8 aligned lanes (hif4_quant8). HBM-bound: one read and
// one write of the operand.
#include "common.cuh"
#include "hif4.cuh"

namespace faq {

struct QkPrepParams {
  const void* x;
  int64_t batch, heads, seq;
  int64_t sb, sh, ss;
  const float* offset;  // [heads, d] or null
  const float* smooth;  // [d] or [heads, d] or null
  int64_t smooth_head_stride;
  int smooth_mode;  // 0 none, 1 multiply, 2 divide
  int rotate;
  int levels;  // 0 = no quantization
  __nv_bfloat16* out;
  int64_t ob, oh, os;
  uint8_t* codes;
  uint32_t* meta;
  bool x_vec, out_vec;
  const __nv_bfloat16* norm_w;  // [d] or null: per-head RMSNorm first
  float eps;
  const __nv_bfloat16* cos;     // [seq, rope_ld] or null: RoPE after the norm
  const __nv_bfloat16* sin;
  int64_t rope_ld;
  // Wan's self-attention glue: WanRMSNorm over a token's whole row of heads_total * d
  // channels, bf16(x * rsqrt(mean + eps)) times the weight w[head * d + c] in fp32. The
  // row's sum of squares is the sum, in a fixed order, of per-head sums: head g of token
  // t at head_ss[(g / heads_per_block) * ss_block_stride + t * ss_token_stride + g %
  // heads_per_block] (blocks = ranks of a head-sharded layer), so the sum is the same
  // for every sharding. Then rope_apply's 3-D RoPE on channel pairs (2i, 2i+1) as
  // complex numbers: fp64 products with fp64 tables [seq, d/2], rounded to fp32.
  const float* head_ss;         // or null
  int64_t heads_total, heads_per_block, ss_token_stride, ss_block_stride;
  const float* tok_w;           // [heads, d]
  const double* pair_cos;       // [seq, d/2] or null
  const double* pair_sin;
};

template <typename T, int D>
__global__ void __launch_bounds__(256) qk_prep_kernel(QkPrepParams p) {
  constexpr int LANES = D / 8;           // lanes per row
  constexpr int ROWS_PER_WARP = 32 / LANES;
  const int lane = threadIdx.x & 31;
  const int sub = lane % LANES;          // position of the lane inside its row
  const int64_t rows = p.batch * p.heads * p.seq;
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t warp_id = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  for (int64_t base = warp_id * ROWS_PER_WARP; base < rows; base += warps_total * ROWS_PER_WARP) {
    const int64_t r = base + lane / LANES;
    const bool live = r < rows;
    const int64_t rr = live ? r : 0;
    const int64_t s = rr % p.seq, h = (rr / p.seq) % p.heads, b = rr / (p.seq * p.heads);
    const T* src = static_cast<const T*>(p.x) + b * p.sb + h * p.sh + s * p.ss + sub * 8;
    float v[8];
    if (p.x_vec) {
      if constexpr (sizeof(T) == 2) {
        const uint4 u = *reinterpret_cast<const uint4*>(src);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          v[2 * i] = __uint_as_float(w[i] << 16);
          v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        }
      } else {
        const float4 a = reinterpret_cast<const float4*>(src)[0];
        const float4 c = reinterpret_cast<const float4*>(src)[1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if constexpr (sizeof(T) == 2)
          v[i] = __bfloat162float(src[i]);
        else
          v[i] = src[i];
      }
    }
    if (p.norm_w != nullptr) {
      // Qwen3RMSNorm over the row: sum of squares across the row's lanes
      float ss = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));  // h.pow(2), summed
#pragma unroll
      for (int ls = 1; ls < LANES; ls <<= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, ls));
      const float r = rsqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(D)), p.eps));
      const uint4 wu = *reinterpret_cast<const uint4*>(p.norm_w + sub * 8);
      const uint32_t ww[4] = {wu.x, wu.y, wu.z, wu.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float w = __uint_as_float(i & 1 ? ww[i >> 1] & 0xFFFF0000u : ww[i >> 1] << 16);
        v[i] = bf16_round(__fmul_rn(w, bf16_round(__fmul_rn(v[i], r))));
      }
    }
    if (p.head_ss != nullptr) {
      // lane `sub` adds heads sub, sub + LANES, ..., then a butterfly over the row's lanes
      const int64_t t = b * p.seq + s;
      float ss = 0.0f;
      for (int64_t g = sub; g < p.heads_total; g += LANES)
        ss = __fadd_rn(ss, p.head_ss[(g / p.heads_per_block) * p.ss_block_stride + t * p.ss_token_stride +
                                     g % p.heads_per_block]);
#pragma unroll
      for (int ls = 1; ls < LANES; ls <<= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, ls));
      const float r = rsqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(p.heads_total * D)), p.eps));
      const float* w = p.tok_w + h * D + sub * 8;
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(bf16_round(__fmul_rn(v[i], r)), w[i]);
    }
    if (p.pair_cos != nullptr) {
      // four complex pairs per lane; the fp32 result stays unrounded into the Hadamard
      const double* cr = p.pair_cos + s * (D / 2) + sub * 4;
      const double* sr = p.pair_sin + s * (D / 2) + sub * 4;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const double re = v[2 * i], im = v[2 * i + 1], c = cr[i], sn = sr[i];
        v[2 * i] = __double2float_rn(__dsub_rn(__dmul_rn(re, c), __dmul_rn(im, sn)));
        v[2 * i + 1] = __double2float_rn(__dadd_rn(__dmul_rn(re, sn), __dmul_rn(im, c)));
      }
    }
    if (p.cos != nullptr) {
      // HF rotate_half: channel j pairs with j + d/2 (negated) below d/2, with j - d/2 above
      constexpr int HALF_LANES = LANES / 2;
      const __nv_bfloat16* cr = p.cos + s * p.rope_ld + sub * 8;
      const __nv_bfloat16* sr = p.sin + s * p.rope_ld + sub * 8;
      const uint4 cu = *reinterpret_cast<const uint4*>(cr);
      const uint4 su = *reinterpret_cast<const uint4*>(sr);
      const uint32_t cw[4] = {cu.x, cu.y, cu.z, cu.w}, sw[4] = {su.x, su.y, su.z, su.w};
      const bool low = sub < HALF_LANES;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float partner = __shfl_xor_sync(0xffffffffu, v[i], HALF_LANES);
        const float rot = low ? -partner : partner;
        const float c = __uint_as_float(i & 1 ? cw[i >> 1] & 0xFFFF0000u : cw[i >> 1] << 16);
        const float sn = __uint_as_float(i & 1 ? sw[i >> 1] & 0xFFFF0000u : sw[i >> 1] << 16);
        v[i] = bf16_round(__fadd_rn(bf16_round(__fmul_rn(v[i], c)), bf16_round(__fmul_rn(rot, sn))));
      }
    }
    if (p.offset != nullptr) {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __fsub_rn(v[i], p.offset[h * D + sub * 8 + i]);
    }
    if (p.smooth_mode != 0) {
      const float* sm = p.smooth + h * p.smooth_head_stride + sub * 8;
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = p.smooth_mode == 1 ? __fmul_rn(v[i], sm[i]) : __fdiv_rn(v[i], sm[i]);
    }
    if (p.rotate) {
      // strides 1, 2, 4 inside the lane
#pragma unroll
      for (int st = 1; st < 8; st <<= 1) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if ((i & st) == 0) {
            const float l = v[i], rgt = v[i + st];
            v[i] = __fadd_rn(l, rgt);
            v[i + st] = __fsub_rn(l, rgt);
          }
        }
      }
      // strides 8 .. D/2 across the lanes of the row
#pragma unroll
      for (int ls = 1; ls < LANES; ls <<= 1) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float other = __shfl_xor_sync(0xffffffffu, v[i], ls);
          v[i] = (sub & ls) ? __fsub_rn(other, v[i]) : __fadd_rn(v[i], other);
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if constexpr (D == 128)
          v[i] = __fdiv_rn(v[i], 11.313708498984761f);  // fp32(sqrt(128)), correctly rounded divide
        else
          v[i] = __fmul_rn(v[i], 0.125f);  // 1/sqrt(64), exact
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = bf16_round(v[i]);
    float q[8];
    uint32_t nib = 0, meta_word = 0;
    if (p.levels != 0) {
      nib = hif4_quant8(v, p.levels, q, meta_word);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) q[i] = v[i];
    }
    if (!live) continue;
    __nv_bfloat16* dst = p.out + b * p.ob + h * p.oh + s * p.os + sub * 8;
    if (p.out_vec) {
      uint4 u;
      u.x = exact_bf16_bits(q[0]) | (exact_bf16_bits(q[1]) << 16);
      u.y = exact_bf16_bits(q[2]) | (exact_bf16_bits(q[3]) << 16);
      u.z = exact_bf16_bits(q[4]) | (exact_bf16_bits(q[5]) << 16);
      u.w = exact_bf16_bits(q[6]) | (exact_bf16_bits(q[7]) << 16);
      *reinterpret_cast<uint4*>(dst) = u;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) dst[i] = __ushort_as_bfloat16(static_cast<unsigned short>(exact_bf16_bits(q[i])));
    }
    if (p.levels != 0) {
      if (p.codes) reinterpret_cast<uint32_t*>(p.codes + r * (D / 2))[sub] = nib;
      if (p.meta && (lane & 7) == 0) p.meta[r * (D / 64) + sub / 8] = meta_word;
    }
  }
}

}  // namespace faq

namespace faq {
static int qk_prep_launch(QkPrepParams& p, int x_dtype, int d, void* stream) {
  const int64_t vec_elems = x_dtype == FAQ_BF16 ? 8 : 4;
  const uint64_t xa = reinterpret_cast<uintptr_t>(p.x), oa = reinterpret_cast<uintptr_t>(p.out);
  p.x_vec = (xa & 15) == 0 && p.sb % vec_elems == 0 && p.sh % vec_elems == 0 && p.ss % vec_elems == 0;
  p.out_vec = (oa & 15) == 0 && p.ob % 8 == 0 && p.oh % 8 == 0 && p.os % 8 == 0;
  const int64_t rows = p.batch * p.heads * p.seq;
  const int rows_per_block = 8 * (32 / (d / 8));
  const int64_t blocks = std::min<int64_t>((rows + rows_per_block - 1) / rows_per_block,
                                           static_cast<int64_t>(num_sms()) * 16);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned g = static_cast<unsigned>(blocks);
  if (x_dtype == FAQ_BF16) {
    if (d == 128)
      qk_prep_kernel<__nv_bfloat16, 128><<<g, 256, 0, st>>>(p);
    else
      qk_prep_kernel<__nv_bfloat16, 64><<<g, 256, 0, st>>>(p);
  } else {
    if (d == 128)
      qk_prep_kernel<float, 128><<<g, 256, 0, st>>>(p);
    else
      qk_prep_kernel<float, 64><<<g, 256, 0, st>>>(p);
  }
  return launch_status("qk_prep_kernel");
}
}  // namespace faq

namespace faq {
static int qk_prep_checked(const void* x, int x_dtype, int64_t batch, int64_t heads, int64_t seq, int d, int64_t sb,
                           int64_t sh, int64_t ss, const float* offset, const float* smooth,
                           int64_t smooth_head_stride, int smooth_mode, int rotate, int levels, void* out, int64_t ob,
                           int64_t oh, int64_t os, uint8_t* codes, uint32_t* meta, const void* norm_w, float eps,
                           const void* cos, const void* sin, int64_t rope_ld, void* stream) {
  FAQ_CHECK_ARG(x && out, "null pointer");
  FAQ_CHECK_ARG(x_dtype == FAQ_BF16 || x_dtype == FAQ_F32, "x_dtype must be FAQ_BF16 or FAQ_F32");
  FAQ_CHECK_ARG(batch >= 0 && heads > 0 && seq >= 0, "bad shape");
  if (d != 64 && d != 128) return fail(FAQ_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  FAQ_CHECK_ARG(smooth_mode >= 0 && smooth_mode <= 2, "smooth_mode must be 0, 1 or 2");
  FAQ_CHECK_ARG(smooth_mode == 0 || smooth != nullptr, "smooth_mode needs smooth");
  FAQ_CHECK_ARG(levels == 0 || levels == 123 || levels == 12 || levels == 13, "levels must be 0, 123, 12 or 13");
  FAQ_CHECK_ARG(levels != 0 || (codes == nullptr && meta == nullptr), "codes/meta need levels");
  FAQ_CHECK_ARG(!codes || (reinterpret_cast<uintptr_t>(codes) & 3) == 0, "codes must be 4-byte aligned");
  FAQ_CHECK_ARG(!norm_w || aligned16(norm_w), "norm_weight must be 16-byte aligned");
  FAQ_CHECK_ARG(!norm_w || eps >= 0.0f, "eps must be non-negative");
  FAQ_CHECK_ARG((cos == nullptr) == (sin == nullptr), "cos and sin come together");
  FAQ_CHECK_ARG(!cos || (aligned16(cos) && aligned16(sin) && rope_ld >= d && rope_ld % 8 == 0),
                "cos/sin must be 16-byte aligned [seq, rope_ld >= d] tables with rope_ld % 8 == 0");
  if (batch == 0 || seq == 0) return FAQ_OK;
  QkPrepParams p;
  p.x = x;
  p.batch = batch;
  p.heads = heads;
  p.seq = seq;
  p.sb = sb;
  p.sh = sh;
  p.ss = ss;
  p.offset = offset;
  p.smooth = smooth;
  p.smooth_head_stride = smooth_head_stride;
  p.smooth_mode = smooth_mode;
  p.rotate = rotate;
  p.levels = levels;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ob = ob;
  p.oh = oh;
  p.os = os;
  p.codes = codes;
  p.meta = meta;
  p.norm_w = static_cast<const __nv_bfloat16*>(norm_w);
  p.eps = eps;
  p.cos = static_cast<const __nv_bfloat16*>(cos);
  p.sin = static_cast<const __nv_bfloat16*>(sin);
  p.rope_ld = rope_ld;
  p.head_ss = nullptr;
  p.heads_total = p.heads_per_block = 1;
  p.ss_token_stride = p.ss_block_stride = 0;
  p.tok_w = nullptr;
  p.pair_cos = nullptr;
  p.pair_sin = nullptr;
  return qk_prep_launch(p, x_dtype, d, stream);
}
}  // namespace faq

extern "C" int faq_qk_prep(const void* x, int x_dtype, int64_t batch, int64_t heads, int64_t seq, int d, int64_t sb,
                           int64_t sh, int64_t ss, const float* offset, const float* smooth, int64_t smooth_head_stride,
                           int smooth_mode, int rotate, int levels, void* out, int64_t ob, int64_t oh, int64_t os,
                           uint8_t* codes, uint32_t* meta, void* stream) {
  return faq::qk_prep_checked(x, x_dtype, batch, heads, seq, d, sb, sh, ss, offset, smooth, smooth_head_stride,
                              smooth_mode, rotate, levels, out, ob, oh, os, codes, meta, nullptr, 0.0f, nullptr,
                              nullptr, 0, stream);
}

extern "C" int faq_qk_norm_rope_prep(const void* x, int x_dtype, int64_t batch, int64_t heads, int64_t seq, int d,
                                     int64_t sb, int64_t sh, int64_t ss, const void* norm_weight, float eps,
                                     const void* cos, const void* sin, int64_t rope_ld, const float* offset,
                                     const float* smooth, int64_t smooth_head_stride, int smooth_mode, int rotate,
                                     int levels, void* out, int64_t ob, int64_t oh, int64_t os, uint8_t* codes,
                                     uint32_t* meta, void* stream) {
  return faq::qk_prep_checked(x, x_dtype, batch, heads, seq, d, sb, sh, ss, offset, smooth, smooth_head_stride,
                              smooth_mode, rotate, levels, out, ob, oh, os, codes, meta, norm_weight, eps, cos, sin,
                              rope_ld, stream);
}

extern "C" int faq_wan_qk_prep(const void* x, int64_t batch, int64_t heads, int64_t seq, int d, int64_t sb,
                               int64_t sh, int64_t ss, const float* head_ss, int64_t heads_total,
                               int64_t heads_per_block, int64_t ss_token_stride, int64_t ss_block_stride,
                               const float* norm_weight, float eps, const double* pair_cos, const double* pair_sin, const float* smooth,
                               int64_t smooth_head_stride, int smooth_mode, int rotate, int levels, void* out,
                               int64_t ob, int64_t oh, int64_t os, void* stream) {
  using namespace faq;
  FAQ_CHECK_ARG(batch >= 0 && heads > 0 && seq >= 0, "bad shape");
  if (d != 64 && d != 128) return fail(FAQ_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  FAQ_CHECK_ARG(levels == 0 || levels == 123 || levels == 12 || levels == 13, "levels must be 0, 123, 12 or 13");
  FAQ_CHECK_ARG((pair_cos == nullptr) == (pair_sin == nullptr), "pair_cos and pair_sin come together");
  FAQ_CHECK_ARG(heads_total > 0 && heads_per_block > 0 && eps >= 0.0f,
                "heads_total and heads_per_block must be positive and eps non-negative");
  FAQ_CHECK_ARG(smooth_mode >= 0 && smooth_mode <= 2, "smooth_mode must be 0, 1 or 2");
  FAQ_CHECK_ARG(smooth_mode == 0 || smooth != nullptr, "smooth_mode needs smooth");
  if (batch == 0 || seq == 0) return FAQ_OK;
  FAQ_CHECK_ARG(x && out && head_ss && norm_weight, "null pointer");
  QkPrepParams p;
  p.x = x;
  p.batch = batch;
  p.heads = heads;
  p.seq = seq;
  p.sb = sb;
  p.sh = sh;
  p.ss = ss;
  p.offset = nullptr;
  p.smooth = smooth;
  p.smooth_head_stride = smooth_head_stride;
  p.smooth_mode = smooth_mode;
  p.rotate = rotate;
  p.levels = levels;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ob = ob;
  p.oh = oh;
  p.os = os;
  p.codes = nullptr;
  p.meta = nullptr;
  p.norm_w = nullptr;
  p.eps = eps;
  p.cos = nullptr;
  p.sin = nullptr;
  p.rope_ld = 0;
  p.head_ss = head_ss;
  p.heads_total = heads_total;
  p.heads_per_block = heads_per_block;
  p.ss_token_stride = ss_token_stride;
  p.ss_block_stride = ss_block_stride;
  p.tok_w = norm_weight;
  p.pair_cos = pair_cos;
  p.pair_sin = pair_sin;
  return qk_prep_launch(p, FAQ_BF16, d, stream);
}
