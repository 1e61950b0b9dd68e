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
  int hpw, groups;              // heads per work item, items per token (set by the launch)
  bool passthrough;             // bf16 input that no stage changes (set by the launch)
};

// bf16(fp32(x / c)) for c = fp32(sqrt(128)), the last step of the head_dim Hadamard:
// returns a value whose bf16 rounding is that of the correctly rounded quotient.
// q = fl(x * fl(1/c)) is within |x/c| * 2^-23 (1 + 2^-25) of x/c, i.e. within 5 units of
// the quotient's bit pattern even next to a power of two; when the low 16 bits of q's
// pattern are 8 or more away from 0 and 0x8000 (the bf16 boundaries) the two round to the
// same bf16. Otherwise -- and for zero, tiny, infinite or NaN q -- the division is done.
__device__ __forceinline__ float div_sqrt128_for_bf16(float x) {
  const float q = __fmul_rn(x, __uint_as_float(0x3DB504F3u));  // fl(1 / fp32(sqrt(128)))
  const uint32_t bits = __float_as_uint(q);
  const bool safe = ((bits & 0x7FFFu) - 8u) <= 0x7FF0u && (bits & 0x7F800000u) >= (27u << 23);
  return safe ? q : __fdiv_rn(x, 11.313708498984761f);
}

// Work item = (token, group of hpw heads): the index arithmetic and the token's data
// (Wan's row norm, the RoPE table rows) are set up once per item, and the heads of the
// group -- neighbours in a [.., S, H, D] projection output -- go RPW per warp iteration.
// codes/meta rows are in [b, h, s] order. MODE 0: offset/smooth only; MODE 1: Qwen3's
// per-head RMSNorm and RoPE in front; MODE 2: Wan's row RMSNorm and 3-D RoPE in front.
template <typename T, int D, int MODE>
__global__ void __launch_bounds__(256, 4) qk_prep_kernel(QkPrepParams p) {
  constexpr int LANES = D / 8;           // lanes per row
  constexpr int RPW = 32 / LANES;        // rows per warp iteration
  const int lane = threadIdx.x & 31;
  const int sub = lane % LANES;          // position of the lane inside its row
  const int slot = lane / LANES;
  const int64_t items = p.batch * p.seq * p.groups;
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t warp_id = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  uint32_t nw[4] = {0, 0, 0, 0};
  if (MODE == 1 && p.norm_w != nullptr) {
    const uint4 u = *reinterpret_cast<const uint4*>(p.norm_w + sub * 8);
    nw[0] = u.x; nw[1] = u.y; nw[2] = u.z; nw[3] = u.w;
  }
  for (int64_t item = warp_id; item < items; item += warps_total) {
    const int64_t t = item / p.groups;
    const int h_begin = static_cast<int>(item - t * p.groups) * p.hpw;
    const int h_end = min(h_begin + p.hpw, static_cast<int>(p.heads));
    const int64_t b = t / p.seq, s = t - b * p.seq;
    float tok_r = 0.0f;
    if (MODE == 2) {
      // lane l adds heads l, l + 32, ..., then a butterfly: an order fixed by heads_total
      float ss = 0.0f;
      for (int64_t g = lane; g < p.heads_total; g += 32)
        ss = __fadd_rn(ss, p.head_ss[(g / p.heads_per_block) * p.ss_block_stride + t * p.ss_token_stride +
                                     g % p.heads_per_block]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
      tok_r = rsqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(p.heads_total * D)), p.eps));
    }
    double pc[4] = {0, 0, 0, 0}, ps[4] = {0, 0, 0, 0};
    if (MODE == 2 && p.pair_cos != nullptr) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        pc[i] = p.pair_cos[s * (D / 2) + sub * 4 + i];
        ps[i] = p.pair_sin[s * (D / 2) + sub * 4 + i];
      }
    }
    for (int h0 = h_begin; h0 < h_end; h0 += RPW) {
      const bool live = h0 + slot < h_end;
      const int64_t h = live ? h0 + slot : h_begin;  // idle slots redo a live row, unstored
      const T* src = static_cast<const T*>(p.x) + b * p.sb + h * p.sh + s * p.ss + sub * 8;
      float v[8];
      uint4 raw = make_uint4(0, 0, 0, 0);
      if (p.x_vec) {
        if constexpr (sizeof(T) == 2) {
          const uint4 u = __ldcs(reinterpret_cast<const uint4*>(src));
          raw = u;
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            v[2 * i] = __uint_as_float(w[i] << 16);
            v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
          }
        } else {
          const float4 a = __ldcs(reinterpret_cast<const float4*>(src));
          const float4 c = __ldcs(reinterpret_cast<const float4*>(src) + 1);
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
      if (MODE == 1 && p.norm_w != nullptr) {
        // Qwen3RMSNorm over the row: sum of squares across the row's lanes
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));  // h.pow(2), summed
#pragma unroll
        for (int ls = 1; ls < LANES; ls <<= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, ls));
        const float r = rsqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(D)), p.eps));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float w = __uint_as_float(i & 1 ? nw[i >> 1] & 0xFFFF0000u : nw[i >> 1] << 16);
          v[i] = bf16_round(__fmul_rn(w, bf16_round(__fmul_rn(v[i], r))));
        }
      }
      if (MODE == 2) {
        const float4* w4 = reinterpret_cast<const float4*>(p.tok_w + h * D + sub * 8);
        const float4 wa = w4[0], wb = w4[1];
        const float w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(bf16_round(__fmul_rn(v[i], tok_r)), w[i]);
      }
      if (MODE == 2 && p.pair_cos != nullptr) {
        // four complex pairs per lane; the fp32 result stays unrounded into the Hadamard
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const double re = v[2 * i], im = v[2 * i + 1];
          v[2 * i] = __double2float_rn(__dsub_rn(__dmul_rn(re, pc[i]), __dmul_rn(im, ps[i])));
          v[2 * i + 1] = __double2float_rn(__dadd_rn(__dmul_rn(re, ps[i]), __dmul_rn(im, pc[i])));
        }
      }
      if (MODE == 1 && p.cos != nullptr) {
        // HF rotate_half: channel j pairs with j + d/2 (negated) below d/2, with j - d/2 above
        constexpr int HALF_LANES = LANES / 2;
        const bool low = sub < HALF_LANES;
        // the token's table row, re-read per head from L1 (holding it would spill)
        const uint4 cu = *reinterpret_cast<const uint4*>(p.cos + s * p.rope_ld + sub * 8);
        const uint4 su = *reinterpret_cast<const uint4*>(p.sin + s * p.rope_ld + sub * 8);
        const uint32_t cw[4] = {cu.x, cu.y, cu.z, cu.w}, sw[4] = {su.x, su.y, su.z, su.w};
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
      float2 f[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) f[i] = make_float2(v[2 * i], v[2 * i + 1]);
      if (p.rotate) {
        // stride 1 inside each pair, 2 and 4 between the lane's pairs
#pragma unroll
        for (int i = 0; i < 4; ++i) f[i] = make_float2(__fadd_rn(f[i].x, f[i].y), __fsub_rn(f[i].x, f[i].y));
#pragma unroll
        for (int d = 1; d < 4; d <<= 1) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if ((i & d) == 0) {
              const float2 l = f[i], r = f[i + d];
              f[i] = __fadd2_rn(l, r);
              f[i + d] = __ffma2_rn(r, make_float2(-1.0f, -1.0f), l);  // l - r, one rounding
            }
          }
        }
        // strides 8 .. D/2 across the lanes of the row: the upper lane of a pair takes
        // other - own, the lower own + other, both as one FMA with a +-1 factor
#pragma unroll
        for (int ls = 1; ls < LANES; ls <<= 1) {
          const float sg = (sub & ls) ? -1.0f : 1.0f;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 other = make_float2(__shfl_xor_sync(0xffffffffu, f[i].x, ls),
                                             __shfl_xor_sync(0xffffffffu, f[i].y, ls));
            f[i] = __ffma2_rn(f[i], make_float2(sg, sg), other);
          }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if constexpr (D == 128)
            f[i] = make_float2(div_sqrt128_for_bf16(f[i].x), div_sqrt128_for_bf16(f[i].y));
          else
            f[i] = __fmul2_rn(f[i], make_float2(0.125f, 0.125f));  // 1/sqrt(64), exact
        }
      }
      uint32_t w[4];
      if (sizeof(T) == 2 && p.x_vec && p.passthrough) {
        w[0] = raw.x; w[1] = raw.y; w[2] = raw.z; w[3] = raw.w;  // no stage changed the bf16 values
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const __nv_bfloat162 b2 = __float22bfloat162_rn(f[i]);
          w[i] = static_cast<uint32_t>(__bfloat16_as_ushort(b2.x)) |
                 (static_cast<uint32_t>(__bfloat16_as_ushort(b2.y)) << 16);
        }
      }
      uint32_t nib = 0, meta_word = 0;
      const uint4 o = p.levels != 0 ? hif4_quant8_bits(w, p.levels, p.codes != nullptr || p.meta != nullptr, nib, meta_word)
                                    : make_uint4(w[0], w[1], w[2], w[3]);
      if (!live) continue;
      __nv_bfloat16* dst = p.out + b * p.ob + h * p.oh + s * p.os + sub * 8;
      if (p.out_vec) {
        __stcs(reinterpret_cast<uint4*>(dst), o);
      } else {
        const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
        for (int i = 0; i < 8; ++i)
          dst[i] = __ushort_as_bfloat16(static_cast<unsigned short>(i & 1 ? ow[i >> 1] >> 16 : ow[i >> 1] & 0xFFFFu));
      }
      if (p.levels != 0) {
        const int64_t canon = (b * p.heads + h) * p.seq + s;
        if (p.codes) reinterpret_cast<uint32_t*>(p.codes + canon * (D / 2))[sub] = nib;
        if (p.meta && (lane & 7) == 0) p.meta[canon * (D / 64) + sub / 8] = meta_word;
      }
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
  // heads per work item: whole tokens when there are enough of them to fill the resident
  // warps (4 blocks of 8 per SM), fewer heads per item (down to one warp iteration) else
  const int rpw = 32 / (d / 8);
  const int64_t tokens = p.batch * p.seq, resident = static_cast<int64_t>(num_sms()) * 32;
  const int64_t iters_all = (p.heads + rpw - 1) / rpw;
  const int64_t iters = std::max<int64_t>(1, std::min<int64_t>(iters_all, tokens * iters_all / resident));
  p.hpw = static_cast<int>(iters * rpw);
  p.groups = static_cast<int>((p.heads + p.hpw - 1) / p.hpw);
  const int64_t items = tokens * p.groups;
  p.passthrough = x_dtype == FAQ_BF16 && p.head_ss == nullptr && p.norm_w == nullptr && p.cos == nullptr &&
                  p.offset == nullptr && p.smooth_mode == 0 && !p.rotate;
  // one resident wave: every warp loops over items with the grid's stride
  const int64_t blocks = std::min<int64_t>((items + 7) / 8, static_cast<int64_t>(num_sms()) * 4);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const unsigned g = static_cast<unsigned>(blocks);
  const int mode = p.head_ss != nullptr ? 2 : (p.norm_w != nullptr || p.cos != nullptr) ? 1 : 0;
  if (x_dtype == FAQ_BF16) {
    if (mode == 2) {
      if (d == 128)
        qk_prep_kernel<__nv_bfloat16, 128, 2><<<g, 256, 0, st>>>(p);
      else
        qk_prep_kernel<__nv_bfloat16, 64, 2><<<g, 256, 0, st>>>(p);
    } else if (mode == 1) {
      if (d == 128)
        qk_prep_kernel<__nv_bfloat16, 128, 1><<<g, 256, 0, st>>>(p);
      else
        qk_prep_kernel<__nv_bfloat16, 64, 1><<<g, 256, 0, st>>>(p);
    } else {
      if (d == 128)
        qk_prep_kernel<__nv_bfloat16, 128, 0><<<g, 256, 0, st>>>(p);
      else
        qk_prep_kernel<__nv_bfloat16, 64, 0><<<g, 256, 0, st>>>(p);
    }
  } else {
    if (mode == 1) {  // fp32 input with Qwen's norm/RoPE
      if (d == 128)
        qk_prep_kernel<float, 128, 1><<<g, 256, 0, st>>>(p);
      else
        qk_prep_kernel<float, 64, 1><<<g, 256, 0, st>>>(p);
    } else {
      if (d == 128)
        qk_prep_kernel<float, 128, 0><<<g, 256, 0, st>>>(p);
      else
        qk_prep_kernel<float, 64, 0><<<g, 256, 0, st>>>(p);
    }
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
