// HiF4 S1P2 quantization on the device, bit-exact with src/faquant/hif4.py.
//
// Arithmetic of the reference, step by step (each step is one IEEE fp32 op with
// round-to-nearest-even, so every intermediate matches the CPU reference):
//   s   = bf16(max64 * bf16(1/d))  d = 7 (levels 123) or 3.5 (12, 13)   hif4.py:102-103
//   s   = clamp(s, 2^-48, 49152)                                          hif4.py:104
//   s   = rint(s * 2^(2-e)) * 2^(e-2), e = floor(log2 s)  (E6M2 grid)     hif4.py:108-113
//   rec = bf16(1 / s)   (correctly rounded fp32 divide, then bf16)        hif4.py:114
//   lv2 = [max8 * rec >= 4]          (123)  | [max8 * rec >= 2] (12)      hif4.py:200-209
//   lv3 = [max4 * rec / 2^lv2 >= 2]  (123)  | [max4 * rec >= 2] (13)      hif4.py:205-213
//   qm  = rec / 2^lv2 / 2^lv3,  ds = s * 2^lv2 * 2^lv3   (exact)          hif4.py:236-239
//   m   = min(floor(|x| * qm * 4 + 0.5), 7)                               hif4.py:268-269
//   y   = sign(x) * m/4 * ds  (exact; sign(-0.0) = +0)                    hif4.py:270
// The multiplies and adds use __fmul_rn/__fadd_rn so the compiler never fuses
// them into an FMA, which would skip an intermediate rounding.
#pragma once

#include "common.cuh"

namespace faq {

__device__ __forceinline__ float divisor_reciprocal(int levels) {
  // bf16(fp32(1/7)) = 0x3E12 = 0.142578125, bf16(fp32(1/3.5)) = 0x3E92 = 0.28515625
  return levels == 123 ? 0.142578125f : 0.28515625f;
}

struct Hif4Scale {
  float s;    // E6M2 scale
  float rec;  // bf16 reciprocal
  uint32_t code;  // (e + 48) << 2 | t
};

// The E6M2 rounding and the reciprocal work on the bit pattern of the clamped scale
// (a positive normal float, low 16 bits zero after the bf16 rounding):
//  * rint(s * 2^(2-e)) * 2^(e-2) keeps two mantissa bits with round-half-to-even; an
//    integer add of 2^20 - 1 + (bit 21) followed by clearing bits 0..20 does exactly
//    that, and a carry out of the mantissa is the reference's move to the next octave.
//  * s = m * 2^e with m in {1, 1.25, 1.5, 1.75}, so bf16(fp32(1/s)) = bf16(fp32(1/m)) *
//    2^-e exactly (both roundings commute with power-of-two scaling in the normal range,
//    and 1/s stays in [2^-16, 2^48]). bf16(fp32(1/m)) for the four mantissas is
//    0x3F80 (1), 0x3F4D (fp32 0x3F4CCCCD rounded up), 0x3F2B (0x3F2AAAAB up) and
//    0x3F12 (0x3F124925 down); the exponent is then lowered by e.
//  * the E6M2 code (e + 48) << 2 | t is the top bits of the pattern minus (127-48) << 2.
__device__ __forceinline__ Hif4Scale hif4_scale(float max64, int levels) {
  float s = bf16_round(__fmul_rn(max64, divisor_reciprocal(levels)));
  s = fminf(fmaxf(s, 3.552713678800501e-15f), 49152.0f);  // [2^-48, 49152]
  uint32_t b = __float_as_uint(s);
  b = (b + 0x000FFFFFu + ((b >> 21) & 1u)) & 0xFFE00000u;
  const uint32_t t = (b >> 21) & 3u;
  // bytes 2t, 2t+1 of the table {0x3F123F2B : 0x3F4D3F80} are bf16(fp32(1/m_t))
  const uint32_t rb = __byte_perm(0x3F4D3F80u, 0x3F123F2Bu, 34u * t + 16u) << 16;
  Hif4Scale r;
  r.s = __uint_as_float(b);
  r.rec = __uint_as_float(rb - (b & 0x7F800000u) + 0x3F800000u);
  r.code = (b >> 21) - ((127u - 48u) << 2);
  return r;
}

// The lv2/lv3 shifts of one 8-value sub-block from the products of its two quarter
// maxima with the reciprocal, ra = fl(m3a * rec) and rb = fl(m3b * rec). The comparisons
// fl(m2 * rec) >= 4 (or 2) and fl(m3 * rec) >= thr of the three level variants are tests
// of exponent fields -- x >= 2^k is one for a non-negative float, and fl(m2 * rec) =
// max(ra, rb) because rounding is monotone -- and for 123, lv2 + [e(ra) >= 1 + lv2] =
// max(e(ra), lv2) since e(ra) <= e(max(ra, rb)) <= 2. A NaN product counts as 0 (max(NaN,
// 0) is 0 on the GPU), as it does in the comparisons, and every shift is clamped to its
// range, so infinite or large products give the comparisons' answers. The equivalence
// was checked against the comparisons for every exponent field with edge mantissas, zero,
// infinities and NaNs, in each variant. Returns lv2 (0 or 1); ea and eb receive
// (lv2 + lv3) << 23 of the two quarters.
__device__ __forceinline__ uint32_t hif4_level_shifts(float ra, float rb, int levels, uint32_t& ea, uint32_t& eb) {
  const int fa = static_cast<int>(__float_as_uint(fmaxf(ra, 0.0f)) & 0x7F800000u);
  const int fb = static_cast<int>(__float_as_uint(fmaxf(rb, 0.0f)) & 0x7F800000u);
  if (levels == 123) {
    const int lv = min(max(max(fa, fb) - (128 << 23), 0), 1 << 23);
    ea = static_cast<uint32_t>(min(max(fa - (127 << 23), lv), 2 << 23));
    eb = static_cast<uint32_t>(min(max(fb - (127 << 23), lv), 2 << 23));
    return static_cast<uint32_t>(lv) >> 23;
  }
  if (levels == 12) {
    ea = eb = static_cast<uint32_t>(min(max(max(fa, fb) - (127 << 23), 0), 1 << 23));
    return ea >> 23;
  }
  ea = static_cast<uint32_t>(min(max(fa - (127 << 23), 0), 1 << 23));
  eb = static_cast<uint32_t>(min(max(fb - (127 << 23), 0), 1 << 23));
  return 0;
}

// Element code from |x| and qm4 = 4 * qm (exact): min(floor(fl(fl(|x| * qm4) + 0.5)), 7).
// fl(|x| * qm) * 4 == fl(|x| * 4qm) because scaling by 4 is exact, so one multiply
// reproduces the reference's two. floor(t) of 0 <= t < 2^23 is taken on the FP32
// adder: t + 2^23 rounded toward zero is exactly 2^23 + floor(t).
__device__ __forceinline__ float hif4_code4(float a, float qm4) {
  const float t = __fadd_rn(__fmul_rn(a, qm4), 0.5f);
  const float f = __fsub_rn(__fadd_rz(t, 8388608.0f), 8388608.0f);
  return fminf(f, 7.0f);
}
__device__ __forceinline__ float hif4_code(float a, float qm) { return hif4_code4(a, __fmul_rn(qm, 4.0f)); }

// Quantize the 8 consecutive values v[0..7] of one lv2 sub-block. The 8 lanes of
// an aligned lane group (lanes 8g .. 8g+7) together hold one 64-value block in
// order. Writes the dequantized values to out[], returns this thread's 8 packed
// nibbles (value i at bits 4i..4i+3) and, in lane 8g, the block's meta word.
// All 32 lanes of the warp must call it (shuffles use the full mask).
__device__ __forceinline__ uint32_t hif4_quant8(const float (&v)[8], int levels, float (&out)[8],
                                               uint32_t& meta_word) {
  float a[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) a[i] = fabsf(v[i]);
  const float m3_0 = fmaxf(fmaxf(a[0], a[1]), fmaxf(a[2], a[3]));
  const float m3_1 = fmaxf(fmaxf(a[4], a[5]), fmaxf(a[6], a[7]));
  const float m2 = fmaxf(m3_0, m3_1);
  float m1 = m2;
  m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 1));
  m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 2));
  m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 4));
  const Hif4Scale sc = hif4_scale(m1, levels);
  uint32_t e0, e1;
  const uint32_t lv2 = hif4_level_shifts(__fmul_rn(m3_0, sc.rec), __fmul_rn(m3_1, sc.rec), levels, e0, e1);
  const uint32_t lv3_0 = (e0 >> 23) - lv2, lv3_1 = (e1 >> 23) - lv2;
  const float qm0 = __fmul_rn(sc.rec, pow2f(2 - static_cast<int>(lv2 + lv3_0)));  // 4 * qm
  const float qm1 = __fmul_rn(sc.rec, pow2f(2 - static_cast<int>(lv2 + lv3_1)));
  const float ds0 = __fmul_rn(sc.s, pow2f(static_cast<int>(lv2 + lv3_0)));
  const float ds1 = __fmul_rn(sc.s, pow2f(static_cast<int>(lv2 + lv3_1)));
  uint32_t nibbles = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float m = hif4_code4(a[i], i < 4 ? qm0 : qm1);
    const float mag = __fmul_rn(__fmul_rn(m, 0.25f), i < 4 ? ds0 : ds1);
    const bool neg = v[i] < 0.0f;
    out[i] = neg ? -mag : mag;
    nibbles |= ((static_cast<uint32_t>(m) | (static_cast<uint32_t>(neg) << 3)) << (4 * i));
  }
  const int pos = threadIdx.x & 7;
  uint32_t bits = (lv2 << (8 + pos)) | (lv3_0 << (16 + 2 * pos)) | (lv3_1 << (17 + 2 * pos));
  bits |= __shfl_xor_sync(0xffffffffu, bits, 1);
  bits |= __shfl_xor_sync(0xffffffffu, bits, 2);
  bits |= __shfl_xor_sync(0xffffffffu, bits, 4);
  meta_word = bits | sc.code;
  return nibbles;
}

// hif4_quant8 on bf16 input held as four pair words (value 2i in the low half of w[i]),
// with the arithmetic moved off the conversion units: |x| and the sign come from the bit
// pattern (the sign is dropped on a zero half, sign(-0.0) = +0), 4 qm and ds / 4 are exponent
// field moves of rec and s (both normal, and they stay normal), and per pair
//   t   = min(fl(fl(|x| 4qm) + 0.5), 7.5)   (== clamping the code to 7 after the floor)
//   r   = t + 2^23 rounded toward zero       (== 2^23 + floor(t); the code is r's low bits)
//   mag = r * ds/4 - 2^23 * ds/4             (one FMA, exact: code * ds/4 has <= 6 bits)
// so the dequantized value is the top half of mag's pattern with the sign put back.
// Returns the four dequantized pair words; nib and meta_word as hif4_quant8 when
// want_codes (which must be the same in all lanes of the warp), else left 0.
__device__ __forceinline__ uint4 hif4_quant8_bits(const uint32_t (&w)[4], int levels, bool want_codes,
                                                  uint32_t& nib, uint32_t& meta_word) {
  uint32_t sgn[4];
  float2 a[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t m = w[i] & 0x7FFF7FFFu;
    // bit 15 of each half of m + 0x7FFF is set iff that half's magnitude is nonzero
    sgn[i] = w[i] & (m + 0x7FFF7FFFu) & 0x80008000u;
    a[i] = make_float2(__uint_as_float(m << 16), __uint_as_float(m & 0xFFFF0000u));
  }
  const float m3_0 = fmaxf(fmaxf(a[0].x, a[0].y), fmaxf(a[1].x, a[1].y));
  const float m3_1 = fmaxf(fmaxf(a[2].x, a[2].y), fmaxf(a[3].x, a[3].y));
  const float m2 = fmaxf(m3_0, m3_1);
  float m1 = m2;
  m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 1));
  m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 2));
  m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 4));
  const Hif4Scale sc = hif4_scale(m1, levels);
  // the float comparisons here (not hif4_level_shifts): K4, the caller, sits at its
  // 64-register budget, which the integer form's live values would exceed
  uint32_t lv2 = 0, lv3_0 = 0, lv3_1 = 0;
  if (levels == 123) {
    lv2 = __fmul_rn(m2, sc.rec) >= 4.0f;
    const float thr = lv2 ? 4.0f : 2.0f;
    lv3_0 = __fmul_rn(m3_0, sc.rec) >= thr;
    lv3_1 = __fmul_rn(m3_1, sc.rec) >= thr;
  } else if (levels == 12) {
    lv2 = __fmul_rn(m2, sc.rec) >= 2.0f;
  } else {
    lv3_0 = __fmul_rn(m3_0, sc.rec) >= 2.0f;
    lv3_1 = __fmul_rn(m3_1, sc.rec) >= 2.0f;
  }
  const uint32_t rec_q = __float_as_uint(sc.rec) + (2u << 23), s_d = __float_as_uint(sc.s) - (2u << 23);
  const uint32_t e0 = (lv2 + lv3_0) << 23, e1 = (lv2 + lv3_1) << 23;
  const float qm[2] = {__uint_as_float(rec_q - e0), __uint_as_float(rec_q - e1)};
  const float ds[2] = {__uint_as_float(s_d + e0), __uint_as_float(s_d + e1)};
  const float off[2] = {__uint_as_float(s_d + e0 + 0x8B800000u), __uint_as_float(s_d + e1 + 0x8B800000u)};
  uint32_t out[4];
  nib = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int qq = i >> 1;  // pairs 0, 1: first quarter; 2, 3: second
    float2 t = __fadd2_rn(__fmul2_rn(a[i], make_float2(qm[qq], qm[qq])), make_float2(0.5f, 0.5f));
    t = make_float2(fminf(t.x, 7.5f), fminf(t.y, 7.5f));
    const float2 r = __fadd2_rz(t, make_float2(8388608.0f, 8388608.0f));
    const float2 mag = __ffma2_rn(r, make_float2(ds[qq], ds[qq]), make_float2(off[qq], off[qq]));
    out[i] = __byte_perm(__float_as_uint(mag.x), __float_as_uint(mag.y), 0x7632) | sgn[i];
    if (want_codes) {
      const uint32_t na = (__float_as_uint(r.x) & 7u) | ((sgn[i] >> 12) & 8u);
      const uint32_t nb = (__float_as_uint(r.y) & 7u) | ((sgn[i] >> 28) & 8u);
      nib |= (na | (nb << 4)) << (8 * i);
    }
  }
  meta_word = 0;
  if (!want_codes) return make_uint4(out[0], out[1], out[2], out[3]);
  const int pos = threadIdx.x & 7;
  uint32_t bits = (lv2 << (8 + pos)) | (lv3_0 << (16 + 2 * pos)) | (lv3_1 << (17 + 2 * pos));
  bits |= __shfl_xor_sync(0xffffffffu, bits, 1);
  bits |= __shfl_xor_sync(0xffffffffu, bits, 2);
  bits |= __shfl_xor_sync(0xffffffffu, bits, 4);
  meta_word = bits | sc.code;
  return make_uint4(out[0], out[1], out[2], out[3]);
}

// Packed HiF4 -> bf16 for 32 consecutive values (half `half` of a 64-value block): `codes`
// their 16 code bytes (two sign-magnitude nibbles per byte, value 2i in the low nibble of
// byte i), `meta` the block's word (E6M2 code | lv2 bits << 8 | lv3 bits << 16). out[q]
// receives values 2q (low half) and 2q + 1 as bf16 bits, exactly hif4_decode's values
// (-0.0 for a negative zero code). Per pair of values: one byte permute gathers
// [m0 | s0 at bit 15 | m1 | s1 at bit 31] from the code word and its 4-bit rotation, the
// bf16 pair (128 + m0, 128 + m1) = (x & 0x00070007) | 0x43004300 is exact, one
// fma.rn.bf16x2 with (c, -128 c), c = scale * 2^(lv2 + lv3 - 2) (exact, by exponent
// arithmetic on the E6M2 code), gives m * c exactly, and an xor restores the sign.
__device__ __forceinline__ uint32_t hfma2_bf16(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ void hif4_expand32_bf16(const uint4& codes, uint32_t meta, int half, uint32_t (&out)[16]) {
  const uint32_t code = meta & 0xFFu;
  // bf16 bits of c0 = scale * 2^-2 and of -128 c0, duplicated in both halves; a micro
  // exponent e adds e to both exponents (e <= 2 stays far from the field's ends: the
  // scale's exponent lies in [-48, 15])
  const uint32_t sb = code << 5;  // (e + 48) << 7 | t << 5: the scale's bf16 bits minus 79 << 7
  const uint32_t base_c = (sb + (77u << 7)) * 0x00010001u;
  const uint32_t base_n = ((sb + (84u << 7)) | 0x8000u) * 0x00010001u;
  const uint32_t l2 = meta >> (8 + 4 * half);   // bit i: lv2 of code word i
  const uint32_t l3 = meta >> (16 + 8 * half);  // bits 2i, 2i + 1: lv3 of word i's two groups
  const uint32_t words[4] = {codes.x, codes.y, codes.z, codes.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t w = words[i];
    const uint32_t r = __funnelshift_l(w, w, 4);
    const uint32_t e2 = (l2 >> i) & 1u;
    const uint32_t ea = (e2 + ((l3 >> (2 * i)) & 1u)) * 0x00800080u;
    const uint32_t eb = (e2 + ((l3 >> (2 * i + 1)) & 1u)) * 0x00800080u;
    const uint32_t ca = base_c + ea, na = base_n + ea;
    const uint32_t cb = base_c + eb, nb = base_n + eb;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      // bytes: [w.j (m0), r.j (s0 in bit 7), r.(j+1) (m1), w.j (s1 in bit 7)]
      const uint32_t sel = static_cast<uint32_t>(j) | (static_cast<uint32_t>(4 + j) << 4) |
                           (static_cast<uint32_t>(4 + ((j + 1) & 3)) << 8) | (static_cast<uint32_t>(j) << 12);
      const uint32_t x = __byte_perm(w, r, sel);
      const uint32_t magic = (x & 0x00070007u) | 0x43004300u;  // (128 + m0, 128 + m1)
      const uint32_t v = hfma2_bf16(magic, j < 2 ? ca : cb, j < 2 ? na : nb);
      out[4 * i + j] = v ^ (x & 0x80008000u);
    }
  }
}

// Decode one packed nibble with its block's meta word (inverse of the packing).
__device__ __forceinline__ float hif4_decode(uint32_t nibble, uint32_t meta, int index_in_block) {
  const uint32_t code = meta & 0xFFu;
  const int e = static_cast<int>(code >> 2) - 48;
  const float s = __fmul_rn(1.0f + 0.25f * static_cast<float>(code & 3u), pow2f(e));
  const int sub8 = index_in_block >> 3, sub4 = index_in_block >> 2;
  const int shift = static_cast<int>((meta >> (8 + sub8)) & 1u) + static_cast<int>((meta >> (16 + sub4)) & 1u);
  const float mag = __fmul_rn(__fmul_rn(static_cast<float>(nibble & 7u), 0.25f), __fmul_rn(s, pow2f(shift)));
  return (nibble & 8u) ? -mag : mag;
}

}  // namespace faq
