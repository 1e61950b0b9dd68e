// GPTQ's column loop with HiF4 grids on the device: the inner, per-column part of
// GPTQ.quantize (src/faquant/gptq.py:417-548, full Hessian) and of its block-diagonal form
// (:197-298), for one block of 64 or 128 columns of every weight row.
//
// Rows are independent in GPTQ (they share only H^-1), so one warp owns one row: lane l
// holds the block's columns l, l + 32, ... in registers, and the CTA's warps share the
// block of the upper inverse Cholesky factor H^-1 in shared memory. Per column c, in the
// reference's order and with its single roundings:
//   at a group start (c % 64 == 0): the HiF4 fit of the group's 64 current values
//     (fit_hif4_compact_parameters, hif4.py:142-219): warp shuffles give the per-4 and
//     per-8 maxima and the group maximum, hif4.cuh's exact helpers the E6M2 scale, the
//     bf16 reciprocal and the lv2/lv3 exponents, which are also written out as the
//     reference's compact metadata;
//   q = sign(w) * min(floor(fl(|w| * qm) * 4 + 0.5), 7) / 4 * ds   (hif4.py:254-271);
//   e = fl(fl(w - q) / hinv[c][c]);
//   w_j = fl(w_j - fl(e * hinv[c][j])) for j >= c   (the rank-1 update of :545-547).
// The caller does the lazy update of the later columns (weight[:, stop:] -= E @ H^-1,
// :552), a plain fp32 GEMM.
#include "common.cuh"
#include "hif4.cuh"

namespace faq {
namespace gptq {

constexpr int WARPS = 8;  // rows per CTA

struct Params {
  const float* w;   // block 0 of row 0; row stride ldw; block b at column b * cols
  int64_t ldw;
  int rows;
  int nblocks;
  const float* hinv;  // block b's [cols x cols] at hinv + b * hinv_stride, row stride ldh
  int64_t ldh, hinv_stride;
  int levels;
  float* q;  // quantized values, like w
  int64_t ldq;
  float* err;  // GPTQ errors, like w
  int64_t lde;
  float* scale;  // [rows, groups_per_row] (+ the block's first group)
  float* rec;
  int8_t* lv2;   // [rows, groups_per_row, 8]
  int8_t* lv3;   // [rows, groups_per_row, 16]
  int64_t groups_per_row;
};

// One value's quantization with its parameters qm4 = 4 qm and ds4 = ds / 4 (hif4.py:266-270):
// the code is min(floor(fl(|w| qm4) + 0.5), 7) (hif4_code4), the magnitude code * ds4 is exact,
// and the sign is sign(w) with sign(+-0) = 0, so only negative w give a negative result.
__device__ __forceinline__ float quant_value(float w, float qm4, float ds4) {
  const float mag = __fmul_rn(hif4_code4(fabsf(w), qm4), ds4);
  return w < 0.0f ? -mag : mag;
}

template <int COLS>
__global__ void __launch_bounds__(WARPS * 32) gptq_hif4_block_kernel(const __grid_constant__ Params p) {
  constexpr int NI = COLS / 32;  // values per lane
  extern __shared__ float hs[];  // [COLS][COLS] of this block's H^-1
  const int b = blockIdx.y;
  const float* hsrc = p.hinv + static_cast<int64_t>(b) * p.hinv_stride;
  for (int idx = threadIdx.x; idx < COLS * COLS; idx += blockDim.x)
    hs[idx] = hsrc[static_cast<int64_t>(idx / COLS) * p.ldh + idx % COLS];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * WARPS + warp;
  if (row >= p.rows) return;  // no barrier follows: a warp with no row simply ends
  const int64_t col0 = static_cast<int64_t>(b) * COLS;
  const float* wrow = p.w + row * p.ldw + col0;
  float v[NI], qv[NI], ev[NI];
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    v[i] = wrow[32 * i + lane];
    qv[i] = 0.0f;
    ev[i] = 0.0f;
  }
#pragma unroll
  for (int g = 0; g < COLS / 64; ++g) {
    // ---- HiF4 fit of the group's current values: columns 64g + lane (v[2g]) and
    // 64g + 32 + lane (v[2g + 1]); a 4-column quarter is 4 consecutive lanes
    float m3[2], qm4[2], ds4[2];
    float m1 = 0.0f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float a = fabsf(v[2 * g + h]);
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
      m3[h] = a;
      m1 = fmaxf(m1, a);
    }
#pragma unroll
    for (int s = 4; s < 32; s <<= 1) m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, s));
    const Hif4Scale sc = hif4_scale(m1, p.levels);
    const int64_t grp = row * p.groups_per_row + (col0 / 64 + g);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      // this lane's quarter and the other quarter of its 8-column sub-block
      const float other = __shfl_xor_sync(0xffffffffu, m3[h], 4);
      const bool first = (lane & 4) == 0;
      uint32_t ea, eb;
      const uint32_t lv2 = hif4_level_shifts(__fmul_rn(first ? m3[h] : other, sc.rec),
                                             __fmul_rn(first ? other : m3[h], sc.rec), p.levels, ea, eb);
      const int sh = static_cast<int>((first ? ea : eb) >> 23);  // lv2 + lv3 of this quarter
      qm4[h] = __fmul_rn(sc.rec, pow2f(2 - sh));
      ds4[h] = __fmul_rn(sc.s, pow2f(sh - 2));
      if ((lane & 3) == 0) p.lv3[grp * 16 + 8 * h + (lane >> 2)] = static_cast<int8_t>(sh - static_cast<int>(lv2));
      if ((lane & 7) == 0) p.lv2[grp * 8 + 4 * h + (lane >> 3)] = static_cast<int8_t>(lv2);
    }
    if (lane == 0) {
      p.scale[grp] = sc.s;
      p.rec[grp] = sc.rec;
    }
    // ---- the group's 64 columns in order
#pragma unroll 1
    for (int ci = 0; ci < 64; ++ci) {
      const int c = 64 * g + ci;
      const int hsel = ci >> 5, owner = ci & 31;
      const float mine = hsel ? v[2 * g + 1] : v[2 * g];
      const float q = quant_value(mine, hsel ? qm4[1] : qm4[0], hsel ? ds4[1] : ds4[0]);
      const float e_mine = __fdiv_rn(__fsub_rn(mine, q), hs[c * COLS + c]);
      const float e = __shfl_sync(0xffffffffu, e_mine, owner);
      if (lane == owner) {
        if (hsel) {
          qv[2 * g + 1] = q;
          ev[2 * g + 1] = e;
        } else {
          qv[2 * g] = q;
          ev[2 * g] = e;
        }
      }
      const float* hrow = hs + c * COLS;
#pragma unroll
      for (int i = 0; i < NI; ++i) {
        const int j = 32 * i + lane;
        if (j >= c) v[i] = __fsub_rn(v[i], __fmul_rn(e, hrow[j]));
      }
    }
  }
  float* qrow = p.q + row * p.ldq + col0;
  float* erow = p.err + row * p.lde + col0;
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    qrow[32 * i + lane] = qv[i];
    erow[32 * i + lane] = ev[i];
  }
}

}  // namespace gptq
}  // namespace faq

extern "C" int faq_gptq_hif4_block(const float* w, int64_t ldw, int64_t rows, int cols, int64_t nblocks,
                                   const float* hinv, int64_t ldh, int64_t hinv_stride, int levels, float* q,
                                   int64_t ldq, float* err, int64_t lde, float* scale, float* rec, int8_t* lv2,
                                   int8_t* lv3, int64_t groups_per_row, void* stream) {
  using namespace faq;
  FAQ_CHECK_ARG(cols == 64 || cols == 128, "cols (the GPTQ block) must be 64 or 128");
  FAQ_CHECK_ARG(levels == 123 || levels == 12 || levels == 13, "levels must be 123, 12 or 13");
  FAQ_CHECK_ARG(rows >= 0 && rows < (int64_t(1) << 31) && nblocks >= 1 && nblocks < 65536, "bad rows or nblocks");
  FAQ_CHECK_ARG(w && hinv && q && err && scale && rec && lv2 && lv3, "null pointer");
  FAQ_CHECK_ARG(ldw >= nblocks * cols && ldq >= nblocks * cols && lde >= nblocks * cols, "leading dimension too small");
  FAQ_CHECK_ARG(ldh >= cols && (nblocks == 1 || hinv_stride >= static_cast<int64_t>(cols) * ldh),
                "bad H^-1 layout");
  FAQ_CHECK_ARG(groups_per_row >= nblocks * cols / 64, "groups_per_row too small");
  if (rows == 0) return FAQ_OK;
  gptq::Params p{w, ldw, static_cast<int>(rows), static_cast<int>(nblocks), hinv, ldh, hinv_stride, levels,
                 q, ldq, err, lde, scale, rec, lv2, lv3, groups_per_row};
  const dim3 grid(static_cast<unsigned>((rows + gptq::WARPS - 1) / gptq::WARPS), static_cast<unsigned>(nblocks));
  const size_t smem = static_cast<size_t>(cols) * cols * sizeof(float);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cols == 128) {
    FAQ_CUDA(cudaFuncSetAttribute(gptq::gptq_hif4_block_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(smem)));
    gptq::gptq_hif4_block_kernel<128><<<grid, gptq::WARPS * 32, smem, s>>>(p);
  } else {
    gptq::gptq_hif4_block_kernel<64><<<grid, gptq::WARPS * 32, smem, s>>>(p);
  }
  return launch_status("gptq_hif4_block_kernel");
}
