// Decoder-layer glue around the two hot paths, fused to one HBM pass each:
//   faq_rms_norm   Qwen3RMSNorm over the last axis (modeling_qwen3.Qwen3RMSNorm as the
//                  reference's Qwen3 models use it): h = fp32(x), h * rsqrt(mean(h^2) +
//                  eps), rounded to bf16, times the bf16 weight, rounded.
//   faq_silu_mul   the SwiGLU gate of Qwen3MLP on one [rows, 2f] gate|up tensor:
//                  bf16(bf16(silu(g)) * u), silu(g) = g / (1 + exp(-g)) in fp32.
//   faq_layer_norm WanLayerNorm without affine (the DiT block's norm1/norm2: LayerNorm of
//                  fp32(x), cast back): mean, biased variance, (x - mean) * rsqrt(var + eps).
//   faq_gelu_tanh  the tanh GELU of the DiT FFN in fp32, rounded once:
//                  0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))).
//   faq_row_sumsq  per-row fp32 sums of squares of column segments, row-major (one per
//                  head for Wan's q/k RMSNorm over all heads: a head-sharded layer
//                  all-gathers them and K4 adds them up in a fixed order).
// torch runs each as 4-8 elementwise kernels with fp32 temporaries; here one read and
// one write of the tensor. Rounding points are torch's; the fp32 sums are not in
// torch's order (tolerance, not bit-exactness, for these).
#include "common.cuh"

namespace faq {

__device__ __forceinline__ void unpack8(const uint4 u, float (&v)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {  // values already bf16-exact
  return make_uint4(exact_bf16_bits(v[0]) | (exact_bf16_bits(v[1]) << 16),
                    exact_bf16_bits(v[2]) | (exact_bf16_bits(v[3]) << 16),
                    exact_bf16_bits(v[4]) | (exact_bf16_bits(v[5]) << 16),
                    exact_bf16_bits(v[6]) | (exact_bf16_bits(v[7]) << 16));
}

// One CTA per row, warp w owning the 1024-channel chunks w, w + W, ...; the row's packed
// bf16 values stay in registers between the reduction and the scaling. The fp32 sum of
// squares has a fixed order that the fused norm of K1 (faq_hif4_quantize_rms_norm)
// repeats bit for bit: lane l of chunk c sums the squares of channels 1024 c + 32 l ..
// + 31 -- its four 8-channel units in the order u = (i + ((l >> 1) & 3)) & 3, i = 0..3
// (the order in which K1 reads them from shared memory without bank conflicts), the even
// and the odd channels in two running sums added at the end; the lanes' sums meet in an
// xor tree (16, 8, 4, 2, 1); the chunks' sums are added in chunk order.
template <int CH>
__global__ void __launch_bounds__(256) rms_norm_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows, int k,
                                                      int64_t ldx, const __nv_bfloat16* __restrict__ w, float eps,
                                                      __nv_bfloat16* __restrict__ out, int64_t ldo) {
  __shared__ float partial[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
  const int nchunks = (k + 1023) / 1024, rot = (lane >> 1) & 3;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    uint4 v[CH][4];
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int chunk = warp + c * W;
      float2 ss2 = make_float2(0.0f, 0.0f);  // even and odd channels, each in turn
#pragma unroll
      for (int u = 0; u < 4; ++u) {  // slot u holds unit (u + rot) & 3
        const int col = chunk * 1024 + 32 * lane + 8 * ((u + rot) & 3);
        v[c][u] = chunk < nchunks && col < k ? *reinterpret_cast<const uint4*>(x + row * ldx + col)
                                             : make_uint4(0, 0, 0, 0);
        float f[8];
        unpack8(v[c][u], f);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 ab = make_float2(f[2 * i], f[2 * i + 1]);
          ss2 = __fadd2_rn(ss2, __fmul2_rn(ab, ab));
        }
      }
      float ss = __fadd_rn(ss2.x, ss2.y);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
      if (lane == 0 && chunk < nchunks) partial[chunk] = ss;
    }
    __syncthreads();
    float total = 0.0f;
    for (int c = 0; c < nchunks; ++c) total = __fadd_rn(total, partial[c]);
    __syncthreads();  // partial[] is rewritten by the next row
    const float r = rsqrtf(__fadd_rn(__fdiv_rn(total, static_cast<float>(k)), eps));
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int chunk = warp + c * W;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int col = chunk * 1024 + 32 * lane + 8 * ((u + rot) & 3);
        if (chunk < nchunks && col < k) {
          float f[8], wv[8], y[8];
          unpack8(v[c][u], f);
          unpack8(*reinterpret_cast<const uint4*>(w + col), wv);
#pragma unroll
          for (int i = 0; i < 8; ++i) y[i] = bf16_round(__fmul_rn(wv[i], bf16_round(__fmul_rn(f[i], r))));
          *reinterpret_cast<uint4*>(out + row * ldo + col) = pack8(y);
        }
      }
    }
  }
}

__global__ void __launch_bounds__(256) silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, int64_t rows, int64_t f,
                                                       int64_t ld, __nv_bfloat16* __restrict__ out, int64_t ldo) {
  const int64_t per_row = f / 8, total = rows * per_row;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / per_row, col = (i % per_row) * 8;
    float g[8], u[8], y[8];
    unpack8(*reinterpret_cast<const uint4*>(gu + row * ld + col), g);
    unpack8(*reinterpret_cast<const uint4*>(gu + row * ld + f + col), u);
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = swiglu_bf16(g[j], u[j]);
    *reinterpret_cast<uint4*>(out + row * ldo + col) = pack8(y);
  }
}

// One CTA per row, warp w owning the 1024-channel chunks w, w + W, ...: the mean, then the
// biased variance around it, each summed in the order faq_rms_norm uses (lane units
// (i + ((l >> 1) & 3)) & 3, even and odd channels in two running sums, an xor tree over
// the lanes, the chunks in order), which the fused norm of K1
// (faq_hif4_quantize_layer_norm) repeats bit for bit.
template <int CH>
__global__ void __launch_bounds__(256) layer_norm_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows, int k,
                                                        int64_t ldx, float eps, __nv_bfloat16* __restrict__ out,
                                                        int64_t ldo) {
  __shared__ float partial[2][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
  const int nchunks = (k + 1023) / 1024, rot = (lane >> 1) & 3;
  const float inv_k = __fdiv_rn(1.0f, static_cast<float>(k));
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    uint4 v[CH][4];
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int chunk = warp + c * W;
      float2 s2 = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int u = 0; u < 4; ++u) {  // slot u holds unit (u + rot) & 3
        const int col = chunk * 1024 + 32 * lane + 8 * ((u + rot) & 3);
        v[c][u] = chunk < nchunks && col < k ? *reinterpret_cast<const uint4*>(x + row * ldx + col)
                                             : make_uint4(0, 0, 0, 0);
        float f[8];
        unpack8(v[c][u], f);
#pragma unroll
        for (int i = 0; i < 4; ++i) s2 = __fadd2_rn(s2, make_float2(f[2 * i], f[2 * i + 1]));
      }
      float sum = __fadd_rn(s2.x, s2.y);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
      if (lane == 0 && chunk < nchunks) partial[0][chunk] = sum;
    }
    __syncthreads();
    float total = 0.0f;
    for (int c = 0; c < nchunks; ++c) total = __fadd_rn(total, partial[0][c]);
    const float mean = __fmul_rn(total, inv_k);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int chunk = warp + c * W;
      float2 d2 = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int col = chunk * 1024 + 32 * lane + 8 * ((u + rot) & 3);
        if (chunk < nchunks && col < k) {
          float f[8];
          unpack8(v[c][u], f);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 e = __ffma2_rn(make_float2(mean, mean), make_float2(-1.0f, -1.0f),
                                        make_float2(f[2 * i], f[2 * i + 1]));
            d2 = __fadd2_rn(d2, __fmul2_rn(e, e));
          }
        }
      }
      float dev = __fadd_rn(d2.x, d2.y);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dev = __fadd_rn(dev, __shfl_xor_sync(0xffffffffu, dev, o));
      if (lane == 0 && chunk < nchunks) partial[1][chunk] = dev;
    }
    __syncthreads();
    float var = 0.0f;
    for (int c = 0; c < nchunks; ++c) var = __fadd_rn(var, partial[1][c]);
    __syncthreads();  // partial[] is rewritten by the next row
    const float r = rsqrtf(__fadd_rn(__fmul_rn(var, inv_k), eps));
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const int chunk = warp + c * W;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int col = chunk * 1024 + 32 * lane + 8 * ((u + rot) & 3);
        if (chunk < nchunks && col < k) {
          float f[8], y[8];
          unpack8(v[c][u], f);
#pragma unroll
          for (int i = 0; i < 8; ++i) y[i] = bf16_round(__fmul_rn(__fsub_rn(f[i], mean), r));
          *reinterpret_cast<uint4*>(out + row * ldo + col) = pack8(y);
        }
      }
    }
  }
}


__global__ void __launch_bounds__(256) gelu_tanh_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows,
                                                        int64_t cols, int64_t ld, __nv_bfloat16* __restrict__ out,
                                                        int64_t ldo) {
  const int64_t per_row = cols / 8, total = rows * per_row;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / per_row, col = (i % per_row) * 8;
    float v[8], y[8];
    unpack8(*reinterpret_cast<const uint4*>(x + row * ld + col), v);
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = gelu_tanh_bf16(v[j]);
    *reinterpret_cast<uint4*>(out + row * ldo + col) = pack8(y);
  }
}

// GROUP lanes (16 or 32) per (row, segment) item, consecutive items on consecutive
// groups; the lanes stride the segment's 8-value chunks, then a butterfly. The order of
// the additions depends only on seg_cols.
template <int GROUP>
__global__ void __launch_bounds__(256) row_sumsq_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows,
                                                        int64_t segments, int64_t seg_cols, int64_t ld,
                                                        float* __restrict__ out) {
  const int lane = threadIdx.x & 31, sub = lane % GROUP;
  const int64_t items = rows * segments, chunks = seg_cols / 8;
  const int64_t groups = static_cast<int64_t>(gridDim.x) * (blockDim.x / GROUP);
  const int64_t first = static_cast<int64_t>(blockIdx.x) * (blockDim.x / GROUP) + threadIdx.x / GROUP;
  // every lane of a warp runs the same number of iterations (the butterfly is warp-wide)
  const int64_t warp_first = first - lane / GROUP;
  for (int64_t base = warp_first; base < items; base += groups) {
    const int64_t it = base + lane / GROUP;
    float ss = 0.0f;
    if (it < items) {
      const int64_t row = it / segments, seg = it % segments;
      const __nv_bfloat16* src = x + row * ld + seg * seg_cols;
      for (int64_t ch = sub; ch < chunks; ch += GROUP) {
        float v[8];
        unpack8(*reinterpret_cast<const uint4*>(src + ch * 8), v);
#pragma unroll
        for (int i = 0; i < 8; ++i) ss = __fadd_rn(ss, __fmul_rn(v[i], v[i]));
      }
    }
#pragma unroll
    for (int o = 1; o < GROUP; o <<= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    if (sub == 0 && it < items) out[it] = ss;
  }
}

}  // namespace faq

extern "C" int faq_rms_norm(const void* x, int64_t rows, int64_t k, int64_t ldx, const void* weight, float eps,
                            void* out, int64_t ldo, void* stream) {
  using namespace faq;
  FAQ_CHECK_ARG(rows >= 0 && k > 0 && k % 8 == 0 && k <= 32768, "k must be a positive multiple of 8, at most 32768");
  if (rows == 0) return FAQ_OK;  // an empty tensor may have no storage
  FAQ_CHECK_ARG(x && weight && out, "null pointer");
  FAQ_CHECK_ARG(ldx >= k && ldo >= k && ldx % 8 == 0 && ldo % 8 == 0, "row strides must be >= k and multiples of 8");
  FAQ_CHECK_ARG(aligned16(x) && aligned16(weight) && aligned16(out), "tensors must be 16-byte aligned");
  FAQ_CHECK_ARG(eps >= 0.0f, "eps must be non-negative");
  const auto* xp = static_cast<const __nv_bfloat16*>(x);
  const auto* wp = static_cast<const __nv_bfloat16*>(weight);
  auto* op = static_cast<__nv_bfloat16*>(out);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nchunks = static_cast<int>((k + 1023) / 1024);  // <= 32
  const int W = std::min(nchunks, 8), per_warp = (nchunks + W - 1) / W;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(rows, static_cast<int64_t>(num_sms()) * 16));
  if (per_warp == 1)
    rms_norm_kernel<1><<<grid, 32 * W, 0, st>>>(xp, rows, static_cast<int>(k), ldx, wp, eps, op, ldo);
  else if (per_warp == 2)
    rms_norm_kernel<2><<<grid, 32 * W, 0, st>>>(xp, rows, static_cast<int>(k), ldx, wp, eps, op, ldo);
  else
    rms_norm_kernel<4><<<grid, 32 * W, 0, st>>>(xp, rows, static_cast<int>(k), ldx, wp, eps, op, ldo);
  return launch_status("rms_norm_kernel");
}

extern "C" int faq_silu_mul(const void* gate_up, int64_t rows, int64_t f, int64_t ld, void* out, int64_t ldo,
                            void* stream) {
  using namespace faq;
  FAQ_CHECK_ARG(rows >= 0 && f > 0 && f % 8 == 0, "f must be a positive multiple of 8");
  if (rows == 0) return FAQ_OK;  // an empty tensor may have no storage
  FAQ_CHECK_ARG(gate_up && out, "null pointer");
  FAQ_CHECK_ARG(ld >= 2 * f && ldo >= f && ld % 8 == 0 && ldo % 8 == 0, "bad row strides");
  FAQ_CHECK_ARG(aligned16(gate_up) && aligned16(out), "tensors must be 16-byte aligned");
  const int64_t total = rows * (f / 8);
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, static_cast<int64_t>(num_sms()) * 16));
  silu_mul_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const __nv_bfloat16*>(gate_up),
                                                                        rows, f, ld, static_cast<__nv_bfloat16*>(out),
                                                                        ldo);
  return launch_status("silu_mul_kernel");
}

extern "C" int faq_layer_norm(const void* x, int64_t rows, int64_t k, int64_t ldx, float eps, void* out, int64_t ldo,
                              void* stream) {
  using namespace faq;
  FAQ_CHECK_ARG(rows >= 0 && k > 0 && k % 8 == 0 && k <= 32768, "k must be a positive multiple of 8, at most 32768");
  if (rows == 0) return FAQ_OK;  // an empty tensor may have no storage
  FAQ_CHECK_ARG(x && out, "null pointer");
  FAQ_CHECK_ARG(ldx >= k && ldo >= k && ldx % 8 == 0 && ldo % 8 == 0, "row strides must be >= k and multiples of 8");
  FAQ_CHECK_ARG(aligned16(x) && aligned16(out), "tensors must be 16-byte aligned");
  FAQ_CHECK_ARG(eps >= 0.0f, "eps must be non-negative");
  const auto* xp = static_cast<const __nv_bfloat16*>(x);
  auto* op = static_cast<__nv_bfloat16*>(out);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nchunks = static_cast<int>((k + 1023) / 1024);  // <= 32
  const int W = std::min(nchunks, 8), per_warp = (nchunks + W - 1) / W;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>(rows, static_cast<int64_t>(num_sms()) * 16));
  const int kk = static_cast<int>(k);
  if (per_warp == 1)
    layer_norm_kernel<1><<<grid, 32 * W, 0, st>>>(xp, rows, kk, ldx, eps, op, ldo);
  else if (per_warp == 2)
    layer_norm_kernel<2><<<grid, 32 * W, 0, st>>>(xp, rows, kk, ldx, eps, op, ldo);
  else
    layer_norm_kernel<4><<<grid, 32 * W, 0, st>>>(xp, rows, kk, ldx, eps, op, ldo);
  return launch_status("layer_norm_kernel");
}

extern "C" int faq_gelu_tanh(const void* x, int64_t rows, int64_t cols, int64_t ld, void* out, int64_t ldo,
                             void* stream) {
  using namespace faq;
  FAQ_CHECK_ARG(rows >= 0 && cols > 0 && cols % 8 == 0, "cols must be a positive multiple of 8");
  if (rows == 0) return FAQ_OK;  // an empty tensor may have no storage
  FAQ_CHECK_ARG(x && out, "null pointer");
  FAQ_CHECK_ARG(ld >= cols && ldo >= cols && ld % 8 == 0 && ldo % 8 == 0, "bad row strides");
  FAQ_CHECK_ARG(aligned16(x) && aligned16(out), "tensors must be 16-byte aligned");
  const int64_t total = rows * (cols / 8);
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, static_cast<int64_t>(num_sms()) * 16));
  gelu_tanh_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), rows, cols, ld, static_cast<__nv_bfloat16*>(out), ldo);
  return launch_status("gelu_tanh_kernel");
}

extern "C" int faq_row_sumsq(const void* x, int64_t rows, int64_t segments, int64_t seg_cols, int64_t ld, float* out,
                             void* stream) {
  using namespace faq;
  FAQ_CHECK_ARG(rows >= 0 && segments > 0 && seg_cols > 0 && seg_cols % 8 == 0,
                "segments must be positive and seg_cols a positive multiple of 8");
  if (rows == 0) return FAQ_OK;  // an empty tensor may have no storage
  FAQ_CHECK_ARG(x && out, "null pointer");
  FAQ_CHECK_ARG(ld >= segments * seg_cols && ld % 8 == 0, "ld must be >= segments * seg_cols and a multiple of 8");
  FAQ_CHECK_ARG(aligned16(x), "x must be 16-byte aligned");
  const int64_t items = rows * segments;
  const int group = seg_cols <= 128 ? 16 : 32;
  const int64_t per_block = 256 / group;
  const unsigned grid = static_cast<unsigned>(
      std::min<int64_t>((items + per_block - 1) / per_block, static_cast<int64_t>(num_sms()) * 16));
  const auto* xp = static_cast<const __nv_bfloat16*>(x);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (group == 16)
    row_sumsq_kernel<16><<<grid, 256, 0, st>>>(xp, rows, segments, seg_cols, ld, out);
  else
    row_sumsq_kernel<32><<<grid, 256, 0, st>>>(xp, rows, segments, seg_cols, ld, out);
  return launch_status("row_sumsq_kernel");
}
