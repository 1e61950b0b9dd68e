// K1 (activation rotation + HiF4 quantization), HiF4 dequantization and K2 (weight
// packing). All three are HBM-bound streaming kernels: one pass over the input,
// 16-byte vector accesses, outputs written once.
//
// K1 with a rotation works on whole rows staged in shared memory, because the
// HiSQ permutation gathers from anywhere in the row (hisq_rotation.py:50-71):
//   1. the row is loaded into shared memory (x dtype; input_scale applied);
//   2. each warp takes segments of 32*E consecutive output channels (E = max(1,
//      block/32)); lane l holds channels seg + 32 i + l, i < E, gathered through
//      the permutation with the sign applied in fp32 (quantization.py:212-213);
//      the Walsh-Hadamard butterflies run in the reference's stage order (stride
//      1, 2, ..., block/2, each (l + r, l - r), rotation.py:22-28): strides < 32
//      across lanes with shuffles, larger strides inside a lane;
//   3. normalization by 1/sqrt(block): an exact power-of-two multiply when
//      log2(block) is even, else a correctly rounded divide by fp32(sqrt(block))
//      (torch's CPU `x / math.sqrt(n)`), then one rounding to x's dtype;
//   4. HiF4 quantization: 8 values per thread, 8 lanes per 64-block (hif4.cuh).
#include <cmath>

#include "common.cuh"
#include "hif4.cuh"

namespace faq {

// number of valid values (0..8) in an 8-value chunk with `left` values left in the row
__device__ __forceinline__ int valid8(int64_t left) { return left <= 0 ? 0 : (left >= 8 ? 8 : static_cast<int>(left)); }

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ float round_to(float v);
template <>
__device__ __forceinline__ float round_to<float>(float v) { return v; }
template <>
__device__ __forceinline__ float round_to<__nv_bfloat16>(float v) { return bf16_round(v); }

// Load 8 consecutive elements of type T starting at p (16-byte vectors when `vec`).
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8], bool vec, int valid) {
  if (vec && valid >= 8) {
    if constexpr (sizeof(T) == 2) {
      const uint4 u = *reinterpret_cast<const uint4*>(p);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
      }
    } else {
      const float4 a = reinterpret_cast<const float4*>(p)[0];
      const float4 b = reinterpret_cast<const float4*>(p)[1];
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = i < valid ? to_f32<T>(p[i]) : 0.0f;
  }
}

// Store 8 values (exactly representable in T) at p.
template <typename T>
__device__ __forceinline__ void store8(T* p, const float (&v)[8], bool vec, int valid) {
  if (vec && valid >= 8) {
    if constexpr (sizeof(T) == 2) {
      uint4 u;
      u.x = exact_bf16_bits(v[0]) | (exact_bf16_bits(v[1]) << 16);
      u.y = exact_bf16_bits(v[2]) | (exact_bf16_bits(v[3]) << 16);
      u.z = exact_bf16_bits(v[4]) | (exact_bf16_bits(v[5]) << 16);
      u.w = exact_bf16_bits(v[6]) | (exact_bf16_bits(v[7]) << 16);
      *reinterpret_cast<uint4*>(p) = u;
    } else {
      reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
      reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
  } else {
    for (int i = 0; i < 8 && i < valid; ++i) {
      if constexpr (sizeof(T) == 2)
        p[i] = __ushort_as_bfloat16(static_cast<unsigned short>(exact_bf16_bits(v[i])));
      else
        p[i] = v[i];
    }
  }
}

struct QuantOut {
  uint8_t* codes;   // [rows, k64/2] or null
  uint32_t* meta;   // [rows, k64/64] or null
  void* qdq;        // [rows, ldq] or null
  int64_t ldq;
  bool qdq_vec;
};

// Quantize the 8 values of chunk `c` (columns 8c..8c+7) of row `row` and write outputs.
template <typename T>
__device__ __forceinline__ void quantize_and_store(const float (&v)[8], int64_t row, int64_t c, int64_t k,
                                                   int64_t k64, int levels, const QuantOut& o) {
  float q[8];
  uint32_t meta_word;
  const uint32_t nib = hif4_quant8(v, levels, q, meta_word);
  if (o.codes) reinterpret_cast<uint32_t*>(o.codes + row * (k64 / 2))[c] = nib;
  if (o.meta && (threadIdx.x & 7) == 0) o.meta[row * (k64 / 64) + c / 8] = meta_word;
  if (o.qdq) {
    const int64_t col = c * 8;
    const int valid = valid8(k - col);
    if (valid > 0) store8<T>(static_cast<T*>(o.qdq) + row * o.ldq + col, q, o.qdq_vec, valid);
  }
}

// ---------------------------------------------------------------- K1, no rotation
// One thread per 8 values; threads of a row are consecutive so that each 64-block
// is held by 8 aligned lanes. Rows are padded to k64 with zeros.
template <typename T>
__global__ void __launch_bounds__(256) hif4_quantize_direct_kernel(const T* __restrict__ x, int64_t rows, int64_t k,
                                                                   int64_t ldx, const T* __restrict__ input_scale,
                                                                   bool x_vec, int levels, QuantOut o) {
  const int64_t k64 = (k + 63) / 64 * 64;
  const int64_t chunks_per_row = k64 / 8;
  const int64_t total = rows * chunks_per_row;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  // every lane of a warp runs the same number of iterations (the shuffles need
  // all 32): the loop bound is rounded up to a whole warp.
  const int64_t total_warps = (total + 31) / 32 * 32;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx - threadIdx.x % 32 < total_warps;
       idx += stride) {
    const bool live = idx < total;
    const int64_t row = live ? idx / chunks_per_row : 0;
    const int64_t c = live ? idx % chunks_per_row : 0;
    const int64_t col = c * 8;
    const int valid = live ? valid8(k - col) : 0;
    float v[8];
    load8<T>(x + row * ldx + col, v, x_vec, valid);
    if (input_scale != nullptr) {
      float s[8];
      load8<T>(input_scale + col, s, x_vec, valid);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = round_to<T>(__fmul_rn(v[i], s[i]));
    }
    float q[8];
    uint32_t meta_word;
    const uint32_t nib = hif4_quant8(v, levels, q, meta_word);
    if (!live) continue;
    if (o.codes) reinterpret_cast<uint32_t*>(o.codes + row * (k64 / 2))[c] = nib;
    if (o.meta && (threadIdx.x & 7) == 0) o.meta[row * (k64 / 64) + c / 8] = meta_word;
    if (o.qdq && valid > 0) store8<T>(static_cast<T*>(o.qdq) + row * o.ldq + col, q, o.qdq_vec, valid);
  }
}

// ---------------------------------------------------------------- K1, signs-only rotation
// A rotation without a permutation (the reference's "signs" construction, hisq_rotation.py:
// 156-167) mixes channels only inside each block of B = 2^LOG2B <= 256 consecutive
// channels, so no row needs staging: it streams like the direct kernel. A thread holds
// 8 consecutive channels; the B/8 lanes of a block are consecutive lanes of one warp
// (k is a multiple of max(64, B), so blocks never straddle a warp or a row). Element
// pipeline as in the staged kernel below (after the activation of ACT, if any, on the
// loaded values -- faq_hif4_quantize_act): input_scale rounded to x's dtype, the sign as
// an exact fp32 negation, butterflies in the reference's stage order (strides 1, 2, 4
// inside the thread, 8 .. B/2 across lanes), the normalization, one rounding to x's
// dtype, then HiF4 on the 8-lane 64-blocks.
template <typename T, int LOG2B, int ACT = 0>
__global__ void __launch_bounds__(256) hif4_rotate_signs_kernel(const T* __restrict__ x, int64_t rows, int64_t k,
                                                                int64_t ldx, const T* __restrict__ input_scale,
                                                                const int8_t* __restrict__ signs, int levels,
                                                                QuantOut o) {
  static_assert(LOG2B >= 3 && LOG2B <= 8, "blocks of 8 .. 256 channels");
  const int64_t chunks_per_row = k / 8;
  const int64_t total = rows * chunks_per_row;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int lane = threadIdx.x & 31;
  const int64_t total_warps = (total + 31) / 32 * 32;  // whole warps: every lane shuffles
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx - lane < total_warps;
       idx += stride) {
    const bool live = idx < total;
    const int64_t row = live ? idx / chunks_per_row : 0;
    const int64_t c = live ? idx % chunks_per_row : 0;
    const int64_t col = c * 8;
    float v[8];
    if constexpr (ACT == FAQ_ACT_SWIGLU) {  // x is [rows, 2k]: gate | up, the product is bf16
      float u[8];
      load8<T>(x + row * ldx + col, v, true, live ? 8 : 0);
      load8<T>(x + row * ldx + k + col, u, true, live ? 8 : 0);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = swiglu_bf16(v[i], u[i]);
    } else {
      load8<T>(x + row * ldx + col, v, true, live ? 8 : 0);
      if constexpr (ACT == FAQ_ACT_GELU_TANH) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = gelu_tanh_bf16(v[i]);
      }
    }
    if (input_scale != nullptr) {
      float sc[8];
      load8<T>(input_scale + col, sc, true, live ? 8 : 0);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = round_to<T>(__fmul_rn(v[i], sc[i]));
    }
    const uint2 sg = live ? *reinterpret_cast<const uint2*>(signs + col) : make_uint2(0, 0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t byte = ((i < 4 ? sg.x : sg.y) >> (8 * (i & 3))) & 0xFFu;
      if (byte & 0x80u) v[i] = -v[i];  // int8 sign < 0: x * (-1), exact
    }
#pragma unroll
    for (int st = 1; st < 8; st <<= 1) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if ((i & st) == 0) {
          const float l = v[i], r = v[i + st];
          v[i] = __fadd_rn(l, r);
          v[i + st] = __fsub_rn(l, r);
        }
      }
    }
#pragma unroll
    for (int st = 1; st < (1 << (LOG2B - 3)); st <<= 1) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float other = __shfl_xor_sync(0xffffffffu, v[i], st);
        v[i] = (lane & st) ? __fsub_rn(other, v[i]) : __fadd_rn(v[i], other);
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float r;
      if constexpr ((LOG2B & 1) == 0)
        r = __fmul_rn(v[i], pow2f(-(LOG2B / 2)));
      else
        r = __fdiv_rn(v[i], static_cast<float>(LOG2B == 3 ? 2.8284271247461903 : LOG2B == 5 ? 5.656854249492381
                                                                                          : 11.313708498984761));
      v[i] = round_to<T>(r);
    }
    float q[8];
    uint32_t meta_word;
    const uint32_t nib = hif4_quant8(v, levels, q, meta_word);
    if (!live) continue;
    const int64_t k64 = k;  // k is a multiple of 64 here
    if (o.codes) reinterpret_cast<uint32_t*>(o.codes + row * (k64 / 2))[c] = nib;
    if (o.meta && (threadIdx.x & 7) == 0) o.meta[row * (k64 / 64) + c / 8] = meta_word;
    if (o.qdq) store8<T>(static_cast<T*>(o.qdq) + row * o.ldq + col, q, o.qdq_vec, 8);
  }
}

// ---------------------------------------------------------------- K1, rotation
template <typename T, int LOG2B>
__global__ void __launch_bounds__(256) hif4_quantize_rotate_kernel(const T* __restrict__ x, int64_t rows, int64_t k,
                                                                   int64_t ldx, const T* __restrict__ input_scale,
                                                                   const int8_t* __restrict__ signs,
                                                                   const int64_t* __restrict__ perm, bool x_vec,
                                                                   int levels, QuantOut o) {
  constexpr int B = 1 << LOG2B;
  constexpr int E = B >= 32 ? B / 32 : 1;  // elements per lane in a segment
  constexpr int SEG = 32 * E;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int64_t k64 = (k + 63) / 64 * 64;
  // layout: src index | sign bit (int32 [k]) ; row in x dtype [k64] ; rotated row [k64]
  int32_t* s_map = reinterpret_cast<int32_t*>(smem_raw);
  T* s_in = reinterpret_cast<T*>(smem_raw + ((k * 4 + 15) / 16) * 16);
  T* s_rot = s_in + k64;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;

  for (int64_t j = tid; j < k; j += blockDim.x) {
    const int64_t src = perm ? perm[j] : j;
    s_map[j] = static_cast<int32_t>(src << 1) | (signs[src] < 0 ? 1 : 0);
  }
  __syncthreads();

  const int64_t nseg = (k + SEG - 1) / SEG;
  const int64_t chunks = k64 / 8;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    // 1. stage the row (input_scale applied in x's dtype)
    for (int64_t c = tid; c < chunks; c += blockDim.x) {
      const int64_t col = c * 8;
      const int valid = valid8(k - col);
      float v[8];
      load8<T>(x + row * ldx + col, v, x_vec, valid);
      if (input_scale != nullptr) {
        float s[8];
        load8<T>(input_scale + col, s, x_vec, valid);
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = round_to<T>(__fmul_rn(v[i], s[i]));
      }
      store8<T>(s_in + col, v, true, 8);
    }
    __syncthreads();
    // 2-3. gather, butterflies, normalization, rounding
    for (int64_t seg = warp; seg < nseg; seg += nwarps) {
      float v[E];
#pragma unroll
      for (int i = 0; i < E; ++i) {
        const int64_t j = seg * SEG + i * 32 + lane;
        float val = 0.0f;
        if (j < k) {
          const int32_t m = s_map[j];
          val = to_f32<T>(s_in[m >> 1]);
          if (m & 1) val = -val;  // x * (-1) in fp32 is exact
        }
        v[i] = val;
      }
#pragma unroll
      for (int st = 1; st < B; st <<= 1) {
        if (st < 32) {
#pragma unroll
          for (int i = 0; i < E; ++i) {
            const float other = __shfl_xor_sync(0xffffffffu, v[i], st);
            v[i] = (lane & st) ? __fsub_rn(other, v[i]) : __fadd_rn(v[i], other);
          }
        } else {
          const int d = st >> 5;
#pragma unroll
          for (int i = 0; i < E; ++i) {
            if ((i & d) == 0) {
              const float l = v[i], r = v[i + d];
              v[i] = __fadd_rn(l, r);
              v[i + d] = __fsub_rn(l, r);
            }
          }
        }
      }
#pragma unroll
      for (int i = 0; i < E; ++i) {
        float r;
        if constexpr ((LOG2B & 1) == 0) {
          r = __fmul_rn(v[i], pow2f(-(LOG2B / 2)));
        } else {
          r = __fdiv_rn(v[i], static_cast<float>(LOG2B == 1 ? 1.4142135623730951 : LOG2B == 3 ? 2.8284271247461903
                                                : LOG2B == 5 ? 5.656854249492381 : LOG2B == 7 ? 11.313708498984761
                                                : 22.627416997969522));
        }
        const int64_t j = seg * SEG + i * 32 + lane;
        if (j < k64) {
          if constexpr (sizeof(T) == 2)
            s_rot[j] = __float2bfloat16_rn(r);
          else
            s_rot[j] = r;
        }
      }
    }
    __syncthreads();
    // 4. quantize the rotated row
    for (int64_t c0 = 0; c0 < chunks; c0 += blockDim.x) {
      const int64_t c = c0 + tid;
      float v[8];
      const int64_t col = c * 8;
      const int valid = c < chunks ? valid8(k - col) : 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = i < valid ? to_f32<T>(s_rot[col + i]) : 0.0f;
      float q[8];
      uint32_t meta_word;
      const uint32_t nib = hif4_quant8(v, levels, q, meta_word);
      if (c < chunks) {
        if (o.codes) reinterpret_cast<uint32_t*>(o.codes + row * (k64 / 2))[c] = nib;
        if (o.meta && (tid & 7) == 0) o.meta[row * (k64 / 64) + c / 8] = meta_word;
        if (o.qdq && valid > 0) store8<T>(static_cast<T*>(o.qdq) + row * o.ldq + col, q, o.qdq_vec, valid);
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------- K1 v2, rotation, bf16 rows
// The fast path for bf16 rows with k % 64 == 0, k <= 32768 and 16-byte aligned rows:
//   - persistent CTAs; each row arrives by a TMA bulk copy (cp.async.bulk) into one
//     of two shared-memory buffers, issued one row ahead, so the load of row r+1
//     overlaps the arithmetic of row r;
//   - the permutation and the sign share one 16-bit word per channel (index | sign << 15);
//   - butterflies of stride < min(block, 512) run in registers, one warp per
//     segment of min(block, 512) channels (16 values per lane at most), and write
//     fp32 to shared memory; for block 1024 the last butterfly (stride 512) runs in
//     the quantization pass, which reads both halves -- the stages keep the
//     reference's order (rotation.py:22-28);
//   - the quantization pass normalizes, rounds to bf16 and quantizes 8 values per
//     thread (hif4_quant8).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
               : "memory");
}

template <int LOG2B>
__global__ void __launch_bounds__(512) hif4_rotate_bf16_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows,
                                                               int k, int64_t ldx,
                                                               const __nv_bfloat16* __restrict__ input_scale,
                                                               const int8_t* __restrict__ signs,
                                                               const int64_t* __restrict__ perm, int levels,
                                                               QuantOut o) {
  constexpr int B = 1 << LOG2B;
  constexpr int HALF = B > 512 ? 512 : B;           // butterflies done in registers
  constexpr int E = HALF >= 32 ? HALF / 32 : 1;     // values per lane
  constexpr int SEG = 32 * E;
  constexpr bool SPLIT = B > 512;                   // last stage in the quantization pass
  extern __shared__ __align__(16) unsigned char smem_raw[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw);                 // 2 barriers
  uint16_t* s_map = reinterpret_cast<uint16_t*>(smem_raw + 64);           // [k]
  const size_t map_bytes = (static_cast<size_t>(k) * 2 + 127) / 128 * 128;
  __nv_bfloat16* s_in = reinterpret_cast<__nv_bfloat16*>(smem_raw + 64 + map_bytes);  // [2][k]
  float* s_mid = reinterpret_cast<float*>(smem_raw + 64 + map_bytes + static_cast<size_t>(k) * 4);  // [k]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const uint32_t row_bytes = static_cast<uint32_t>(k) * 2;

  if (tid == 0) {
    mbar_init(smem_addr(&bars[0]), 1);
    mbar_init(smem_addr(&bars[1]), 1);
    fence_barrier_init();
  }
  for (int j = tid; j < k; j += blockDim.x) {
    const int src = perm ? static_cast<int>(perm[j]) : j;
    s_map[j] = static_cast<uint16_t>(src | ((signs[src] < 0) ? 0x8000 : 0));
  }
  __syncthreads();
  const int64_t first = blockIdx.x;
  if (tid == 0) {
    for (int b = 0; b < 2; ++b) {
      const int64_t r = first + static_cast<int64_t>(b) * gridDim.x;
      if (r < rows) {
        mbar_arrive_expect_tx(smem_addr(&bars[b]), row_bytes);
        bulk_load(smem_addr(s_in + b * k), x + r * ldx, row_bytes, smem_addr(&bars[b]));
      }
    }
  }
  const int nseg = k / SEG;
  const int chunks = k / 8;
  int it = 0;
  for (int64_t row = first; row < rows; row += gridDim.x, ++it) {
    const int buf = it & 1;
    const __nv_bfloat16* in = s_in + buf * k;
    // CTA-uniform decision: a barrier follows, so no warp may leave the loop alone
    if (!__syncthreads_and(mbar_wait(smem_addr(&bars[buf]), (it >> 1) & 1))) {
      if (tid == 0) {
        trace_timeout(30, it);
        // bounded drain of the copies still in flight into either buffer
        for (int b = 0; b < 2; ++b) {
          const int64_t r = row + static_cast<int64_t>(b) * gridDim.x;
          if (r < rows) mbar_wait(smem_addr(&bars[(it + b) & 1]), ((it + b) >> 1) & 1);
        }
      }
      break;
    }
    // gather + butterflies in registers
    for (int seg = warp; seg < nseg; seg += nwarps) {
      float v[E];
#pragma unroll
      for (int i = 0; i < E; ++i) {
        const int j = seg * SEG + i * 32 + lane;
        const uint32_t m = s_map[j];
        const int src = static_cast<int>(m & 0x7FFFu);
        float val = __bfloat162float(in[src]);
        if (input_scale != nullptr) val = bf16_round(__fmul_rn(val, __bfloat162float(input_scale[src])));
        v[i] = (m & 0x8000u) ? -val : val;
      }
#pragma unroll
      for (int st = 1; st < HALF; st <<= 1) {
        if (st < 32) {
#pragma unroll
          for (int i = 0; i < E; ++i) {
            const float other = __shfl_xor_sync(0xffffffffu, v[i], st);
            v[i] = (lane & st) ? __fsub_rn(other, v[i]) : __fadd_rn(v[i], other);
          }
        } else {
          const int d = st >> 5;
#pragma unroll
          for (int i = 0; i < E; ++i) {
            if ((i & d) == 0) {
              const float l = v[i], r = v[i + d];
              v[i] = __fadd_rn(l, r);
              v[i + d] = __fsub_rn(l, r);
            }
          }
        }
      }
#pragma unroll
      for (int i = 0; i < E; ++i) {
        float r = v[i];
        if constexpr (!SPLIT) {
          if constexpr ((LOG2B & 1) == 0)
            r = __fmul_rn(r, pow2f(-(LOG2B / 2)));
          else
            r = __fdiv_rn(r, static_cast<float>(LOG2B == 1 ? 1.4142135623730951 : LOG2B == 3 ? 2.8284271247461903
                                                : LOG2B == 5 ? 5.656854249492381 : LOG2B == 7 ? 11.313708498984761
                                                : 22.627416997969522));
          r = bf16_round(r);
        }
        s_mid[seg * SEG + i * 32 + lane] = r;
      }
    }
    __syncthreads();
    // the input buffer is free again: prefetch the row after next into it
    if (tid == 0) {
      const int64_t r2 = row + 2 * static_cast<int64_t>(gridDim.x);
      if (r2 < rows) {
        mbar_arrive_expect_tx(smem_addr(&bars[buf]), row_bytes);
        bulk_load(smem_addr(s_in + buf * k), x + r2 * ldx, row_bytes, smem_addr(&bars[buf]));
      }
    }
    // quantization pass (with the last butterfly for block 1024)
    for (int c0 = 0; c0 < chunks; c0 += blockDim.x) {
      const int c = c0 + tid;
      const bool live = c < chunks;
      const int col = live ? c * 8 : 0;
      float v[8];
      {
        const float4 a0 = *reinterpret_cast<const float4*>(s_mid + col);
        const float4 a1 = *reinterpret_cast<const float4*>(s_mid + col + 4);
        v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w;
        v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
      }
      if constexpr (SPLIT) {
        const int partner = col ^ 512;
        const float4 b0 = *reinterpret_cast<const float4*>(s_mid + partner);
        const float4 b1 = *reinterpret_cast<const float4*>(s_mid + partner + 4);
        const float w[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
        const bool lower = (col & 512) == 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float r = lower ? __fadd_rn(v[i], w[i]) : __fsub_rn(w[i], v[i]);
          v[i] = bf16_round(__fmul_rn(r, 0.03125f));  // 1/sqrt(1024), exact
        }
      }
      float q[8];
      uint32_t meta_word;
      const uint32_t nib = hif4_quant8(v, levels, q, meta_word);
      if (live) {
        if (o.codes) reinterpret_cast<uint32_t*>(o.codes + row * (k / 2))[c] = nib;
        if (o.meta && (tid & 7) == 0) o.meta[row * (k / 64) + c / 8] = meta_word;
        if (o.qdq) store8<__nv_bfloat16>(static_cast<__nv_bfloat16*>(o.qdq) + row * o.ldq + col, q, o.qdq_vec, 8);
      }
    }
    __syncthreads();
  }
}

__device__ __forceinline__ float2 f2add(float2 a, float2 b) { return __fadd2_rn(a, b); }
// a - b as one packed FMA: b * -1 + a, a single rounding of the exact difference
__device__ __forceinline__ float2 f2sub(float2 a, float2 b) { return __ffma2_rn(b, make_float2(-1.0f, -1.0f), a); }

// ---------------------------------------------------------------- 32 values per lane
// HiF4 of 32 consecutive bf16 values held by one lane as 16 pair words in channel order
// (value 2q in the low half of w[q]): half of a 64-block whose other half the partner
// lane (lane ^ 1, the even lane holding the lower half) holds; both lanes call it
// together (one shuffle for the block maximum, one for the meta word).
//   - sign bits from the bf16 pattern, cleared where the magnitude is zero: a -0.0
//     quantizes to +0 as the reference's sign(-0.0) == 0 does;
//   - per-4 / per-8 maxima in registers, the E6M2 scale and its reciprocal
//     (hif4_scale), the level shifts (hif4_level_shifts), then per pair on FP32x2
//       t = min(fl(fl(|x| 4qm) + 0.5), 7.5)  (== clamping the code to 7 after the floor)
//       r = t + 2^23 rounded toward zero    (== 2^23 + floor(t))
//       mag = r * ds/4 - 2^23 * ds/4        (one FMA, exact: code * ds/4 has <= 6 bits)
//     with 4 qm = rec 2^(2 - sh), ds / 4 = s 2^(sh - 2) and -2^23 ds / 4 as exponent-field
//     moves of rec and s (both normal, and they stay normal).
// Outputs: the dequantized pair words q[16], the nibbles nib[4] (codes, when CODES) and
// the block's meta word (in both lanes).
template <bool CODES>
__device__ __forceinline__ void hif4_quant32_lane(const uint32_t (&w)[16], int levels, uint32_t (&q)[16],
                                                  uint32_t (&nib)[4], uint32_t& meta) {
  uint32_t sgn[16];  // sign bits of each bf16 pair, clear on a zero half
  float2 a[16];      // |x| pairs
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const uint32_t m = w[i] & 0x7FFF7FFFu;
    // bit 15 of each half of m + 0x7FFF is set iff that half's magnitude is nonzero
    // (no carry crosses the halves: 0x7FFF + 0x7FFF < 2^16)
    sgn[i] = w[i] & (m + 0x7FFF7FFFu) & 0x80008000u;
    a[i] = make_float2(__uint_as_float(m << 16), __uint_as_float(m & 0xFFFF0000u));
  }
  float m3[8], m2[4];
#pragma unroll
  for (int i = 0; i < 8; ++i) m3[i] = fmaxf(fmaxf(a[2 * i].x, a[2 * i].y), fmaxf(a[2 * i + 1].x, a[2 * i + 1].y));
#pragma unroll
  for (int i = 0; i < 4; ++i) m2[i] = fmaxf(m3[2 * i], m3[2 * i + 1]);
  float m1 = fmaxf(fmaxf(m2[0], m2[1]), fmaxf(m2[2], m2[3]));
  m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 1));
  const Hif4Scale sc = hif4_scale(m1, levels);
  uint32_t lvbits = 0;  // bit s: lv2 of sub-block s, bit 4+j: lv3 of quarter j
  const uint32_t rec_q0 = __float_as_uint(sc.rec) + (2u << 23);  // 4 * rec
  const uint32_t s_d0 = __float_as_uint(sc.s) - (2u << 23);      // s / 4
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    nib[s] = 0;
    const float2 rab = __fmul2_rn(make_float2(m3[2 * s], m3[2 * s + 1]), make_float2(sc.rec, sc.rec));
    uint32_t ea, eb;  // (lv2 + lv3) << 23 of the two quarters
    const uint32_t lv2 = hif4_level_shifts(rab.x, rab.y, levels, ea, eb);
    const uint32_t la = (ea >> 23) - lv2, lb = (eb >> 23) - lv2;
    lvbits |= (lv2 << s) | (la << (4 + 2 * s)) | (lb << (5 + 2 * s));
    const float2 qm_a = make_float2(__uint_as_float(rec_q0 - ea), __uint_as_float(rec_q0 - ea));
    const float2 qm_b = make_float2(__uint_as_float(rec_q0 - eb), __uint_as_float(rec_q0 - eb));
    const float2 ds_a = make_float2(__uint_as_float(s_d0 + ea), __uint_as_float(s_d0 + ea));
    const float2 ds_b = make_float2(__uint_as_float(s_d0 + eb), __uint_as_float(s_d0 + eb));
    const float2 of_a = make_float2(__uint_as_float(s_d0 + ea + 0x8B800000u), __uint_as_float(s_d0 + ea + 0x8B800000u));
    const float2 of_b = make_float2(__uint_as_float(s_d0 + eb + 0x8B800000u), __uint_as_float(s_d0 + eb + 0x8B800000u));
#pragma unroll
    for (int h = 0; h < 4; ++h) {  // pair 4 s + h, in quarter h / 2 of sub-block s
      const int i = 4 * s + h;
      float2 t = __fadd2_rn(__fmul2_rn(a[i], h < 2 ? qm_a : qm_b), make_float2(0.5f, 0.5f));
      t = make_float2(fminf(t.x, 7.5f), fminf(t.y, 7.5f));
      const float2 r = __fadd2_rz(t, make_float2(8388608.0f, 8388608.0f));
      const float2 mag = __ffma2_rn(r, h < 2 ? ds_a : ds_b, h < 2 ? of_a : of_b);
      q[i] = __byte_perm(__float_as_uint(mag.x), __float_as_uint(mag.y), 0x7632) | sgn[i];
      if constexpr (CODES) {
        const uint32_t na = (__float_as_uint(r.x) & 7u) | ((sgn[i] >> 12) & 8u);  // r = 2^23 + code
        const uint32_t nb = (__float_as_uint(r.y) & 7u) | ((sgn[i] >> 28) & 8u);
        nib[s] |= (na | (nb << 4)) << (8 * h);
      }
    }
  }
  const int half = threadIdx.x & 1;
  uint32_t mb = ((lvbits & 0xFu) << (8 + 4 * half)) | (((lvbits >> 4) & 0xFFu) << (16 + 8 * half));
  mb |= __shfl_xor_sync(0xffffffffu, mb, 1);
  meta = mb | sc.code;
}

// Stores of hif4_quant32_lane's outputs for channels col .. col + 31 of `row` (k % 64 == 0,
// 16-byte aligned qdq rows and codes).
__device__ __forceinline__ void store_quant32(const QuantOut& o, int64_t row, int64_t k, int64_t col,
                                              const uint32_t (&q)[16], const uint32_t (&nib)[4], uint32_t meta,
                                              bool codes) {
  if (o.qdq) {
    uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(o.qdq) + row * o.ldq + col);
#pragma unroll
    for (int s = 0; s < 4; ++s) dst[s] = make_uint4(q[4 * s], q[4 * s + 1], q[4 * s + 2], q[4 * s + 3]);
  }
  if (codes && o.codes)
    *reinterpret_cast<uint4*>(o.codes + row * (k / 2) + col / 2) = make_uint4(nib[0], nib[1], nib[2], nib[3]);
  if (o.meta && (threadIdx.x & 1) == 0) o.meta[row * (k / 64) + col / 64] = meta;
}

// ---------------------------------------------------------------- K1, signs-only, 64-channel blocks
// The row-parallel inputs (the reference's "signs" construction with 64-channel blocks,
// bf16): a lane holds 32 consecutive channels, half of a block, and its partner lane
// (lane ^ 1) the other half. Strides 1..16 run inside the lane on FP32x2 pairs, stride 32
// with one exchange between the partners (the reference's stage order), then the
// normalization by 1/8 (exact), one rounding to bf16 and hif4_quant32_lane -- the
// arithmetic of hif4_rotate_signs_kernel with a quarter of its exchanges. Work items
// (row, half block) run halves fastest, so a warp reads 2 KB of a row in 16-byte loads.
// ACT fuses the activation into the load as in hif4_rotate_signs_kernel.
template <int ACT, bool CODES>
__global__ void __launch_bounds__(256) hif4_rotate_signs64_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows,
                                                                  int64_t k, int64_t ldx,
                                                                  const __nv_bfloat16* __restrict__ input_scale,
                                                                  const int8_t* __restrict__ signs, int levels,
                                                                  QuantOut o) {
  const int64_t halves = k / 32;
  const int64_t total = rows * halves;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int lane = threadIdx.x & 31;
  const int64_t total_warps = (total + 31) / 32 * 32;  // whole warps: partners exchange
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx - lane < total_warps;
       idx += stride) {
    const bool live = idx < total;
    const int64_t row = live ? idx / halves : 0, col = live ? (idx % halves) * 32 : 0;
    const __nv_bfloat16* xr = x + row * ldx + col;
    uint32_t w[16];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint4 v = live ? __ldg(reinterpret_cast<const uint4*>(xr) + u) : make_uint4(0, 0, 0, 0);
      w[4 * u] = v.x; w[4 * u + 1] = v.y; w[4 * u + 2] = v.z; w[4 * u + 3] = v.w;
    }
    float2 p[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) p[i] = make_float2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xFFFF0000u));
    if constexpr (ACT == FAQ_ACT_SWIGLU) {  // x is [rows, 2k]: gate | up
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint4 v = live ? __ldg(reinterpret_cast<const uint4*>(xr + k) + u) : make_uint4(0, 0, 0, 0);
        const uint32_t up[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          float2& g = p[4 * u + h];
          g = make_float2(swiglu_bf16(g.x, __uint_as_float(up[h] << 16)),
                          swiglu_bf16(g.y, __uint_as_float(up[h] & 0xFFFF0000u)));
        }
      }
    } else if constexpr (ACT == FAQ_ACT_GELU_TANH) {
#pragma unroll
      for (int i = 0; i < 16; ++i) p[i] = make_float2(gelu_tanh_bf16(p[i].x), gelu_tanh_bf16(p[i].y));
    }
    if (input_scale != nullptr) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint4 v = live ? __ldg(reinterpret_cast<const uint4*>(input_scale + col) + u) : make_uint4(0, 0, 0, 0);
        const uint32_t sc[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          float2& e = p[4 * u + h];
          e = make_float2(bf16_round(__fmul_rn(e.x, __uint_as_float(sc[h] << 16))),
                          bf16_round(__fmul_rn(e.y, __uint_as_float(sc[h] & 0xFFFF0000u))));
        }
      }
    }
    // int8 signs: a negative one flips the sign bit (x * -1, exact)
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const uint4 v = live ? __ldg(reinterpret_cast<const uint4*>(signs + col) + u) : make_uint4(0, 0, 0, 0);
      const uint32_t sg[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        // bytes 4h .. 4h + 3 of this 16-byte run: values 16 u + 4 h .. + 3, pairs 8 u + 2 h, + 1
        float2& a = p[8 * u + 2 * h];
        float2& b = p[8 * u + 2 * h + 1];
        a.x = __uint_as_float(__float_as_uint(a.x) ^ ((sg[h] << 24) & 0x80000000u));
        a.y = __uint_as_float(__float_as_uint(a.y) ^ ((sg[h] << 16) & 0x80000000u));
        b.x = __uint_as_float(__float_as_uint(b.x) ^ ((sg[h] << 8) & 0x80000000u));
        b.y = __uint_as_float(__float_as_uint(b.y) ^ (sg[h] & 0x80000000u));
      }
    }
    // stride 1 inside each pair, strides 2 .. 16 between pairs (distance d = stride / 2)
#pragma unroll
    for (int i = 0; i < 16; ++i) p[i] = make_float2(__fadd_rn(p[i].x, p[i].y), __fsub_rn(p[i].x, p[i].y));
#pragma unroll
    for (int d = 1; d < 16; d <<= 1) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        if ((i & d) == 0) {
          const float2 l = p[i], r = p[i + d];
          p[i] = f2add(l, r);
          p[i + d] = f2sub(l, r);
        }
      }
    }
    // stride 32: the lower half (even lane) keeps a + b, the upper b's lane a - b
    const bool upper = lane & 1;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float ox = __shfl_xor_sync(0xffffffffu, p[i].x, 1);
      const float oy = __shfl_xor_sync(0xffffffffu, p[i].y, 1);
      p[i] = upper ? make_float2(__fsub_rn(ox, p[i].x), __fsub_rn(oy, p[i].y))
                   : make_float2(__fadd_rn(p[i].x, ox), __fadd_rn(p[i].y, oy));
    }
    // / sqrt(64) = * 2^-3 (exact), one rounding to bf16, as pair words
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const __nv_bfloat162 b2 = __float22bfloat162_rn(__fmul2_rn(p[i], make_float2(0.125f, 0.125f)));
      w[i] = *reinterpret_cast<const uint32_t*>(&b2);
    }
    uint32_t q[16], nib[4], meta;
    hif4_quant32_lane<CODES>(w, levels, q, nib, meta);
    if (live) store_quant32(o, row, k, col, q, nib, meta, CODES);
  }
}

// ---------------------------------------------------------------- K1 v4, rotation, bf16 rows
// Throughput path for bf16 rows with k % 1024 == 0, k <= 16384 and 32 <= block <= 1024
// (all HiSQ and r64 shapes of the BASELINE configurations). It is issue-bound (a
// 1024-point Hadamard is 10 adds per value before any quantization), so the work is
// counted per element:
//   - one warp per 1024-channel chunk; lane l gathers output channels 32l .. 32l+31 of its
//     chunk through a 16-bit map entry (byte offset | sign << 15), stored lane-transposed
//     so that one 16-byte load brings 8 entries without bank conflicts; the sign is one
//     XOR of the sign bit (x * -1 is exact);
//   - butterflies (the reference's stage order, rotation.py:22-28): stride 1 inside a
//     float2, strides 2..16 on float2 pairs (packed FP32x2 adds), a 32x34 shared-memory
//     transpose, then strides 32..block/2 the same way;
//   - normalization by an exact power of two as one ffma2(v, 2^-k, +0) per pair: the
//     reference's correctly rounded division, subnormals included, up to the sign of a
//     zero, which the quantization below does not look at;
//   - the quantization pass takes sign bits from the bf16 pattern, cleared where the
//     magnitude is zero: a -0.0 (an input zero, an underflow of the scaling, or a tiny
//     negative value rounded to zero in bf16) quantizes to +0 as the reference's
//     sign(-0.0) == 0 does;
//   - quantization: one lane per 32 values (half a 64-block), one shuffle for the block
//     maximum, per-4/per-8 maxima in registers, the element code on FP32x2.
// A CTA owns one row at a time (the permutation gathers from anywhere in the row), but
// its warps meet only at the two row buffers:
//   - full[b] completes when the row in buffer b has landed (cp.async.bulk, complete_tx);
//   - empty[b] completes when every warp has gathered its chunk out of buffer b;
//   - lane 0 of warp 0 refills buffer b with the row after next once empty[b] has
//     completed, at the end of its own row.
// Each warp stages its rotated chunk in its own transpose scratch and quantizes it from
// there (the 64-blocks of a chunk never cross chunks), so no CTA-wide barrier is left in
// the row loop and the warps of a CTA drift freely over a row. The launch bounds hold
// every width class to the registers of 20 resident warps per SM (the shared memory of a
// 4-warp CTA allows 5).

// map entry w = ((chunk * 4 + t8) * 32 + lane) * 8 + e8 describes output channel
// chunk * 1024 + 32 lane + 8 t8 + e8
__device__ __forceinline__ int v4_map_channel(int w) {
  return (w & ~1023) + 32 * ((w >> 3) & 31) + 8 * ((w >> 8) & 3) + (w & 7);
}

__device__ __forceinline__ float v4_gathered(const unsigned char* in, uint32_t off, uint32_t sign,
                                             const __nv_bfloat16* __restrict__ input_scale) {
  uint32_t bits = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(in + off)) << 16;
  if (input_scale != nullptr)
    bits = __float_as_uint(bf16_round(__fmul_rn(__uint_as_float(bits), __bfloat162float(input_scale[off >> 1]))));
  return __uint_as_float(bits ^ sign);
}

// fused norms of K1 v4
constexpr int kNormNone = 0, kNormRms = 1, kNormLayer = 2;

// the two channels of one map word (low entry -> .x); NORM == kNormRms applies the RMSNorm
// first, bf16(gamma * bf16(x * rn)), NORM == kNormLayer the affine-free LayerNorm,
// bf16((x - mu) * rn), on the pair (cvt.rn.bf16x2 rounds each half as bf16_round does)
template <int NORM>
__device__ __forceinline__ float2 v4_gathered2(const unsigned char* in, const unsigned char* gam, float rn, float mu,
                                               uint32_t m, const __nv_bfloat16* __restrict__ input_scale) {
  const uint32_t oa = m & 0x7FFFu, ob = (m >> 16) & 0x7FFFu;
  const uint32_t sa = (m << 16) & 0x80000000u, sb = m & 0x80000000u;
  if constexpr (NORM == kNormNone) {
    return make_float2(v4_gathered(in, oa, sa, input_scale), v4_gathered(in, ob, sb, input_scale));
  } else {
    const float2 xv = make_float2(__uint_as_float(static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(in + oa)) << 16),
                                  __uint_as_float(static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(in + ob)) << 16));
    [[maybe_unused]] const float2 gv = make_float2(__uint_as_float(static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(gam + oa)) << 16),
                                  __uint_as_float(static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(gam + ob)) << 16));
    __nv_bfloat162 t;
    uint32_t tb;
    if constexpr (NORM == kNormRms) {
      t = __float22bfloat162_rn(__fmul2_rn(xv, make_float2(rn, rn)));
      tb = *reinterpret_cast<const uint32_t*>(&t);
      t = __float22bfloat162_rn(__fmul2_rn(gv, make_float2(__uint_as_float(tb << 16), __uint_as_float(tb & 0xFFFF0000u))));
    } else {  // x - mu as one rounding of the exact difference, then the scale
      t = __float22bfloat162_rn(__fmul2_rn(__ffma2_rn(make_float2(mu, mu), make_float2(-1.0f, -1.0f), xv),
                                           make_float2(rn, rn)));
    }
    tb = *reinterpret_cast<const uint32_t*>(&t);
    uint32_t ba = tb << 16, bb = tb & 0xFFFF0000u;
    if (input_scale != nullptr) {
      ba = __float_as_uint(bf16_round(__fmul_rn(__uint_as_float(ba), __bfloat162float(input_scale[oa >> 1]))));
      bb = __float_as_uint(bf16_round(__fmul_rn(__uint_as_float(bb), __bfloat162float(input_scale[ob >> 1]))));
    }
    return make_float2(__uint_as_float(ba ^ sa), __uint_as_float(bb ^ sb));
  }
}

constexpr int kK1Warps = 20;  // resident warps per SM the launch bounds size registers for

// dynamic shared memory of K1 v4: barriers, map (2 B per channel), two row buffers, one
// 32 x 34 float transpose scratch per warp; with the norm, its weight and the partial sums
inline size_t v4_smem_bytes(int64_t k, int norm) {
  const size_t w = static_cast<size_t>(k / 1024);
  return 64 + static_cast<size_t>(k) * 2 + static_cast<size_t>(k) * 4 + w * 32 * 34 * 4 +
         (norm == kNormRms ? static_cast<size_t>(k) * 2 + 128 : norm == kNormLayer ? 256 : 0);
}

template <int LOG2B, bool CODES, int MAXW, int NORM = kNormNone>
__global__ void __launch_bounds__(MAXW * 32, kK1Warps / MAXW > 0 ? kK1Warps / MAXW : 1) hif4_rotate_v4_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t rows, int k, int64_t ldx,
    const __nv_bfloat16* __restrict__ input_scale, const int8_t* __restrict__ signs,
    const int64_t* __restrict__ perm, int levels, QuantOut o, const __nv_bfloat16* __restrict__ gamma, float eps) {
  constexpr int B = 1 << LOG2B;
  static_assert(B >= 32 && B <= 1024, "v4 handles blocks 32..1024");
  constexpr int TS = 34;  // transpose row stride (floats): 64-bit stores and column loads conflict-free
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int W = blockDim.x >> 5;  // == k / 1024
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);
  uint64_t* empty = full + 2;
  uint64_t* normbar = full + 4;  // NORM, [kind][2] by row parity: every warp's partial sum is in s_part
  unsigned char* s_map = smem_raw + 64;
  unsigned char* s_in = s_map + static_cast<size_t>(k) * 2;                    // [2][k] bf16
  float* s_tr = reinterpret_cast<float*>(s_in + static_cast<size_t>(k) * 4);  // [W][32 * TS]
  unsigned char* s_gamma = reinterpret_cast<unsigned char*>(s_tr + W * 32 * TS);  // NORM: [k] bf16
  float* s_part = reinterpret_cast<float*>(s_gamma + (NORM == kNormRms ? static_cast<size_t>(k) * 2 : 0));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t row_bytes = static_cast<uint32_t>(k) * 2;
  const int64_t G = gridDim.x;
  const int64_t first = blockIdx.x;
  const bool loader = tid == 0;
  uint32_t pending = 0;  // loader: bit b set while a load into buffer b is in flight unconsumed

  if (loader) {
    mbar_init(smem_addr(&full[0]), 1);
    mbar_init(smem_addr(&full[1]), 1);
    mbar_init(smem_addr(&empty[0]), W);
    mbar_init(smem_addr(&empty[1]), W);
    if constexpr (NORM != kNormNone) {
      for (int b = 0; b < (NORM == kNormLayer ? 4 : 2); ++b) mbar_init(smem_addr(&normbar[b]), W);
    }
    fence_barrier_init();
    for (int b = 0; b < 2; ++b) {
      const int64_t r = first + b * G;
      if (r < rows) {
        mbar_arrive_expect_tx(smem_addr(&full[b]), row_bytes);
        bulk_load(smem_addr(s_in + b * row_bytes), x + r * ldx, row_bytes, smem_addr(&full[b]));
        pending |= 1u << b;
      }
    }
  }
  // the map, built while the first rows load: all permutation reads of a batch are in
  // flight together, then all sign reads
  {
    constexpr int U = 16;
    for (int w0 = tid; w0 < k; w0 += U * static_cast<int>(blockDim.x)) {
      int src[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int w = w0 + u * static_cast<int>(blockDim.x);
        const int j = v4_map_channel(w);
        src[u] = w < k ? (perm ? static_cast<int>(perm[j]) : j) : 0;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int w = w0 + u * static_cast<int>(blockDim.x);
        if (w < k) {
          const bool neg = signs[src[u]] < 0;
          reinterpret_cast<uint16_t*>(s_map)[w] = static_cast<uint16_t>((src[u] * 2) | (neg ? 0x8000 : 0));
        }
      }
    }
  }
  if constexpr (NORM == kNormRms) {  // the norm weight in channel order (k % 1024 == 0: whole 16-byte units)
    for (int i = tid; i < k / 8; i += static_cast<int>(blockDim.x))
      reinterpret_cast<uint4*>(s_gamma)[i] = __ldg(reinterpret_cast<const uint4*>(gamma) + i);
  }
  __syncthreads();

  const int ch = warp;
  float* tr = s_tr + warp * (32 * TS);
  uint16_t* s_outw = reinterpret_cast<uint16_t*>(tr);  // this warp's rotated chunk, 1024 bf16
  const uint4* mrow = reinterpret_cast<const uint4*>(s_map) + (ch << 7) + lane;
  const int rot = (lane >> 1) & 3;  // rotation of this lane's staged row, see below
  int it = 0;
  for (int64_t row = first; row < rows; row += G, ++it) {
    const int buf = it & 1;
    if (!mbar_wait_warp(smem_addr(&full[buf]), (it >> 1) & 1, 31, it)) break;
    if (loader) pending &= ~(1u << buf);
    const unsigned char* in = s_in + buf * row_bytes;
    float rn = 0.0f, mu = 0.0f;  // NORM: the row's rsqrt(... + eps) and (LayerNorm) mean
    if constexpr (NORM == kNormRms) {
      // the sum of squares in the order of faq_rms_norm: lane l of chunk c takes its four
      // 8-channel units u = (i + rot) & 3, i = 0..3 (conflict-free 16-byte reads), even and
      // odd channels in two running sums added at the end, then an xor tree over the lanes,
      // then the chunks in order after every warp has published
      const uint4* src = reinterpret_cast<const uint4*>(in + static_cast<size_t>(ch) * 2048 + 64 * lane);
      float2 ss2 = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 v = src[(i + rot) & 3];
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float2 ab = make_float2(__uint_as_float(wv[h] << 16), __uint_as_float(wv[h] & 0xFFFF0000u));
          ss2 = __fadd2_rn(ss2, __fmul2_rn(ab, ab));
        }
      }
      float ss = __fadd_rn(ss2.x, ss2.y);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
      float* part = s_part + 16 * (it & 1);
      if (lane == 0) {
        part[ch] = ss;
        mbar_arrive(smem_addr(&normbar[it & 1]));  // release: the partial is visible to the waiters
      }
      // a warp can be at most one row ahead of another here (it needs every warp's arrival
      // for the next row), so the parity of each barrier is unambiguous
      if (!mbar_wait_warp(smem_addr(&normbar[it & 1]), (it >> 1) & 1, 33, it)) break;
      float total = 0.0f;
      for (int c = 0; c < W; ++c) total = __fadd_rn(total, part[c]);
      rn = rsqrtf(__fadd_rn(__fdiv_rn(total, static_cast<float>(k)), eps));
    } else if constexpr (NORM == kNormLayer) {
      // mean, then the biased variance around it, in the order of faq_layer_norm: per lane
      // the four units u = (i + rot) & 3, even and odd channels in two running sums, an
      // xor tree over the lanes, the chunks in order, each sum published and awaited
      const uint4* src = reinterpret_cast<const uint4*>(in + static_cast<size_t>(ch) * 2048 + 64 * lane);
      float2 xv[16];
      float2 s2 = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 v = src[(i + rot) & 3];
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          xv[4 * i + h] = make_float2(__uint_as_float(wv[h] << 16), __uint_as_float(wv[h] & 0xFFFF0000u));
          s2 = __fadd2_rn(s2, xv[4 * i + h]);
        }
      }
      const float inv_k = __fdiv_rn(1.0f, static_cast<float>(k));
      float* part = s_part + 32 * (it & 1);
      float sum = __fadd_rn(s2.x, s2.y);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, off));
      if (lane == 0) {
        part[ch] = sum;
        mbar_arrive(smem_addr(&normbar[it & 1]));
      }
      if (!mbar_wait_warp(smem_addr(&normbar[it & 1]), (it >> 1) & 1, 33, it)) break;
      float total = 0.0f;
      for (int c = 0; c < W; ++c) total = __fadd_rn(total, part[c]);
      mu = __fmul_rn(total, inv_k);
      float2 d2 = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float2 e = __ffma2_rn(make_float2(mu, mu), make_float2(-1.0f, -1.0f), xv[i]);
        d2 = __fadd2_rn(d2, __fmul2_rn(e, e));
      }
      float dev = __fadd_rn(d2.x, d2.y);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) dev = __fadd_rn(dev, __shfl_xor_sync(0xffffffffu, dev, off));
      if (lane == 0) {
        part[16 + ch] = dev;
        mbar_arrive(smem_addr(&normbar[2 + (it & 1)]));
      }
      if (!mbar_wait_warp(smem_addr(&normbar[2 + (it & 1)]), (it >> 1) & 1, 34, it)) break;
      float var = 0.0f;
      for (int c = 0; c < W; ++c) var = __fadd_rn(var, part[16 + c]);
      rn = rsqrtf(__fadd_rn(__fmul_rn(var, inv_k), eps));
    }
    float2 p[16];
#pragma unroll
    for (int t8 = 0; t8 < 4; ++t8) {
      const uint4 m4 = mrow[t8 * 32];
      const uint32_t m[4] = {m4.x, m4.y, m4.z, m4.w};
#pragma unroll
      for (int h = 0; h < 4; ++h)
        p[4 * t8 + h] = v4_gathered2<NORM>(in, s_gamma, rn, mu, m[h], input_scale);
    }
    // stride 1: inside each float2 (the gathered values are consumed here)
#pragma unroll
    for (int q = 0; q < 16; ++q) p[q] = make_float2(__fadd_rn(p[q].x, p[q].y), __fsub_rn(p[q].x, p[q].y));
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_addr(&empty[buf]));  // this warp is done with the buffer
    // strides 2 .. 16 (and < B): float2 index distance d = stride / 2
#pragma unroll
    for (int d = 1; d < 16 && 2 * d < B; d <<= 1) {
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        if ((q & d) == 0) {
          const float2 l = p[q], r = p[q + d];
          p[q] = f2add(l, r);
          p[q + d] = f2sub(l, r);
        }
      }
    }
    // transpose through the warp's scratch: lane c then holds channels c + 32 i
#pragma unroll
    for (int q = 0; q < 16; ++q) *reinterpret_cast<float2*>(tr + lane * TS + 2 * q) = p[q];
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 16; ++q) p[q] = make_float2(tr[(2 * q) * TS + lane], tr[(2 * q + 1) * TS + lane]);
    __syncwarp();
    // strides 32 .. B/2: i xor 1 inside the float2, then float2 distance d
    if constexpr (B >= 64) {
#pragma unroll
      for (int q = 0; q < 16; ++q) p[q] = make_float2(__fadd_rn(p[q].x, p[q].y), __fsub_rn(p[q].x, p[q].y));
    }
#pragma unroll
    for (int d = 1; 64 * d < B; d <<= 1) {
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        if ((q & d) == 0) {
          const float2 l = p[q], r = p[q + d];
          p[q] = f2add(l, r);
          p[q + d] = f2sub(l, r);
        }
      }
    }
    // Stage the rotated chunk as bf16, 32-value row i = channels 32 i .. 32 i + 31, with
    // the 16-byte unit u of row i at (u + (i >> 1)) & 3: lane writes stay one 64-byte
    // span per instruction, and the quantization below (lane i reads row i's units in
    // the order u = 0..3, each from its rotated place) hits 8 different 16-byte bank
    // groups in every quarter-warp. For lane c, element i sits in unit c >> 3 of row i.
    {
      uint16_t* out = s_outw + (lane & 7);
      int rot8[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) rot8[r] = 8 * (((lane >> 3) + r) & 3);
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        float2 r;
        if constexpr ((LOG2B & 1) == 0) {
          const float c = pow2f(-(LOG2B / 2));
          r = __ffma2_rn(p[q], make_float2(c, c), make_float2(0.0f, 0.0f));  // == p / 2^(LOG2B/2)
        } else {
          const float sq = static_cast<float>(LOG2B == 5 ? 5.656854249492381 : LOG2B == 7 ? 11.313708498984761
                                                : 22.627416997969522);
          r = make_float2(__fadd_rn(__fdiv_rn(p[q].x, sq), 0.0f), __fadd_rn(__fdiv_rn(p[q].y, sq), 0.0f));
        }
        const __nv_bfloat162 b2 = __float22bfloat162_rn(r);
        // elements i = 2q and 2q + 1: both have i >> 1 == q
        out[(2 * q) * 32 + rot8[q & 3]] = __bfloat16_as_ushort(b2.x);
        out[(2 * q + 1) * 32 + rot8[q & 3]] = __bfloat16_as_ushort(b2.y);
      }
    }
    __syncwarp();
    // quantization: lane l = channels 32 l .. 32 l + 31 of the chunk (half a 64-block; the
    // partner lane l ^ 1 holds the other half)
    {
      const int col = (ch << 10) + 32 * lane;
      uint32_t w[16];
      {
        const uint4* src = reinterpret_cast<const uint4*>(s_outw + 32 * lane);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint4 v = src[(u + rot) & 3];
          w[4 * u] = v.x; w[4 * u + 1] = v.y; w[4 * u + 2] = v.z; w[4 * u + 3] = v.w;
        }
      }
      __syncwarp();  // the scratch is free for the next row's transpose
      uint32_t q[16], nib[4], meta;
      hif4_quant32_lane<CODES>(w, levels, q, nib, meta);
      store_quant32(o, row, k, col, q, nib, meta, CODES);
    }
    // refill this buffer with the row after next once every warp has gathered from it
    if (loader) {
      const int64_t r2 = row + 2 * G;
      if (r2 < rows && mbar_wait_site(smem_addr(&empty[buf]), (it >> 1) & 1, 32, it)) {
        mbar_arrive_expect_tx(smem_addr(&full[buf]), row_bytes);
        bulk_load(smem_addr(s_in + buf * row_bytes), x + r2 * ldx, row_bytes, smem_addr(&full[buf]));
        pending |= 1u << buf;
      }
    }
  }
  // a wait that gave up leaves loads in flight: let them land (bounded) before exiting.
  // Buffer b has completed (it - b + 1) / 2 phases by iteration `it`.
  if (loader) {
    for (int b = 0; b < 2; ++b)
      if ((pending >> b) & 1u) mbar_wait(smem_addr(&full[b]), static_cast<uint32_t>((it - b + 1) >> 1) & 1u);
  }
}

// ---------------------------------------------------------------- dequantize
template <typename T>
__global__ void __launch_bounds__(256) hif4_dequantize_kernel(const uint8_t* __restrict__ codes,
                                                              const uint32_t* __restrict__ meta, int64_t rows,
                                                              int64_t k, T* __restrict__ out, int64_t ldo, bool vec) {
  const int64_t k64 = (k + 63) / 64 * 64;
  const int64_t chunks_per_row = k64 / 8;
  const int64_t total = rows * chunks_per_row;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = idx / chunks_per_row, c = idx % chunks_per_row;
    const int64_t col = c * 8;
    const int valid = valid8(k - col);
    if (valid == 0) continue;
    const uint32_t nib = reinterpret_cast<const uint32_t*>(codes + row * (k64 / 2))[c];
    const uint32_t m = meta[row * (k64 / 64) + c / 8];
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = hif4_decode((nib >> (4 * i)) & 0xFu, m, static_cast<int>((col & 63) + i));
    store8<T>(out + row * ldo + col, v, vec, valid);
  }
}

// bf16 output of whole 64-value blocks (k % 64 == 0, 16-byte aligned output rows): one
// thread per 32 values -- a 16-byte code load, the block's meta word,
// hif4_expand32_bf16, four 16-byte stores -- on a grid of as many threads as items, so
// the pass runs near the speed of its bytes (0.5625 read + 2 written per value): the form
// in which packed weights feed the bf16 GEMM at prefill sizes. (A grid of one wave with
// two items per thread in flight measured 3.5 TB/s against 4.1 on the config-2 weights.)
// Item indices fit 32 bits (checked by the caller).
__global__ void __launch_bounds__(256) hif4_expand_bf16_kernel(const uint8_t* __restrict__ codes,
                                                               const uint32_t* __restrict__ meta, uint32_t rows,
                                                               uint32_t k, __nv_bfloat16* __restrict__ out,
                                                               int64_t ldo) {
  const uint32_t halves = k / 32;  // items per row
  const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * halves) return;
  const uint32_t row = idx / halves, h = idx - row * halves;
  const uint4 c = __ldg(reinterpret_cast<const uint4*>(codes + static_cast<uint64_t>(row) * (k / 2)) + h);
  const uint32_t m = __ldg(meta + static_cast<uint64_t>(row) * (k / 64) + (h >> 1));
  uint32_t o[16];
  hif4_expand32_bf16(c, m, static_cast<int>(h & 1u), o);
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * ldo + 32 * static_cast<int64_t>(h));
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[i] = make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
}

// ---------------------------------------------------------------- K2: pack weights
// With GPTQ metadata: code = clamp(round(|w| / ds * 4), 0, 7) (hif4.py:311, torch.round
// is half-to-even = rintf); without it, the RTN fit of the quantizer applied to w,
// which must then be the SOURCE weight: RTN is not idempotent (a quantized block
// has a smaller maximum and can fit another E6M2 scale), which is why the reference
// fits weight metadata from the source (quantization.py:329-345). Values the packed
// form does not reproduce exactly are counted in *mismatches.
template <typename T>
__global__ void __launch_bounds__(256) hif4_pack_kernel(const T* __restrict__ w, int64_t n, int64_t k, int64_t ldw,
                                                        const float* __restrict__ scale, const int8_t* __restrict__ lv2,
                                                        const int8_t* __restrict__ lv3, bool w_vec, int levels,
                                                        uint8_t* __restrict__ codes, uint32_t* __restrict__ meta,
                                                        unsigned long long* mismatches) {
  const int64_t k64 = (k + 63) / 64 * 64;
  const int64_t chunks_per_row = k64 / 8;
  const int64_t total = n * chunks_per_row;
  const int64_t total_warps = (total + 31) / 32 * 32;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx - threadIdx.x % 32 < total_warps;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const bool live = idx < total;
    const int64_t row = live ? idx / chunks_per_row : 0, c = live ? idx % chunks_per_row : 0;
    const int64_t col = c * 8;
    const int valid = live ? valid8(k - col) : 0;
    float v[8];
    load8<T>(w + row * ldw + col, v, w_vec, valid);
    uint32_t nib = 0, meta_word = 0;
    float q[8];
    if (scale == nullptr) {
      nib = hif4_quant8(v, levels, q, meta_word);
    } else if (live) {
      const int64_t blk = row * (k64 / 64) + c / 8;
      const int pos = static_cast<int>(c & 7);
      const float s = scale[blk];
      const int e2 = lv2[blk * 8 + pos];
      const int e3a = lv3[blk * 16 + 2 * pos], e3b = lv3[blk * 16 + 2 * pos + 1];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float ds = __fmul_rn(s, pow2f(e2 + (i < 4 ? e3a : e3b)));
        const float m = fminf(fmaxf(rintf(__fmul_rn(__fdiv_rn(fabsf(v[i]), ds), 4.0f)), 0.0f), 7.0f);
        const bool neg = v[i] < 0.0f;
        const float mag = __fmul_rn(__fmul_rn(m, 0.25f), ds);
        q[i] = neg ? -mag : mag;
        nib |= (static_cast<uint32_t>(m) | (static_cast<uint32_t>(neg) << 3)) << (4 * i);
      }
      const int e = exponent_of(s);
      meta_word = (static_cast<uint32_t>(e + 48) << 2) | (static_cast<uint32_t>(__fmul_rn(s, pow2f(2 - e))) - 4u);
      uint32_t bits = (static_cast<uint32_t>(e2) << (8 + pos)) | (static_cast<uint32_t>(e3a) << (16 + 2 * pos)) |
                      (static_cast<uint32_t>(e3b) << (17 + 2 * pos));
      meta_word |= bits;
    }
    if (scale != nullptr) {
      // gather the lv bits of the 8 lanes of the block
      uint32_t bits = meta_word & 0xFFFFFF00u;
      bits |= __shfl_xor_sync(0xffffffffu, bits, 1);
      bits |= __shfl_xor_sync(0xffffffffu, bits, 2);
      bits |= __shfl_xor_sync(0xffffffffu, bits, 4);
      meta_word = (meta_word & 0xFFu) | bits;
    }
    if (!live) continue;
    int bad = 0;
    for (int i = 0; i < valid; ++i) bad += (__float_as_uint(q[i]) != __float_as_uint(v[i])) && !(q[i] == 0.0f && v[i] == 0.0f);
    if (bad && mismatches) atomicAdd(mismatches, static_cast<unsigned long long>(bad));
    reinterpret_cast<uint32_t*>(codes + row * (k64 / 2))[c] = nib;
    if ((threadIdx.x & 7) == 0) meta[row * (k64 / 64) + c / 8] = meta_word;
  }
}

// ---------------------------------------------------------------- host launchers
static bool valid_levels(int levels) { return levels == 123 || levels == 12 || levels == 13; }

template <typename T>
static int launch_quantize(const void* x, int64_t rows, int64_t k, int64_t ldx, const void* input_scale,
                           const int8_t* signs, const int64_t* perm, int rot_block, int levels, const QuantOut& o,
                           cudaStream_t stream) {
  const bool x_vec = aligned16(x) && (ldx * static_cast<int64_t>(sizeof(T))) % 16 == 0 &&
                     (input_scale == nullptr || aligned16(input_scale));
  const int sms = num_sms();
  if (signs == nullptr) {
    const int64_t k64 = (k + 63) / 64 * 64;
    const int64_t threads = rows * (k64 / 8);
    const int64_t blocks = std::min<int64_t>((threads + 255) / 256, static_cast<int64_t>(sms) * 16);
    hif4_quantize_direct_kernel<T><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        static_cast<const T*>(x), rows, k, ldx, static_cast<const T*>(input_scale), x_vec, levels, o);
    return launch_status("hif4_quantize_direct_kernel");
  }
  int block = rot_block == 0 ? 1 : rot_block;
  int log2b = 0;
  while ((1 << log2b) < block) ++log2b;
  // signs without a permutation in 64-channel blocks, bf16: two lanes per block
  if constexpr (sizeof(T) == 2) {
    if (perm == nullptr && log2b == 6 && k % 64 == 0 && x_vec && (o.qdq == nullptr || o.qdq_vec) &&
        aligned16(signs) && (o.codes == nullptr || aligned16(o.codes))) {
      const int64_t threads = rows * (k / 32);
      const int64_t blocks = std::min<int64_t>((threads + 255) / 256, static_cast<int64_t>(sms) * 8);
      if (blocks == 0) return FAQ_OK;
      const auto* xb = static_cast<const __nv_bfloat16*>(x);
      const auto* sc = static_cast<const __nv_bfloat16*>(input_scale);
      if (o.codes != nullptr)
        hif4_rotate_signs64_kernel<FAQ_ACT_NONE, true><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
            xb, rows, k, ldx, sc, signs, levels, o);
      else
        hif4_rotate_signs64_kernel<FAQ_ACT_NONE, false><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
            xb, rows, k, ldx, sc, signs, levels, o);
      return launch_status("hif4_rotate_signs64_kernel");
    }
  }
  // signs without a permutation: blocks are independent, the row streams (no staging)
  if (perm == nullptr && log2b >= 3 && log2b <= 8 && k % 64 == 0 && k % block == 0 && x_vec &&
      (o.qdq == nullptr || o.qdq_vec) &&
      (reinterpret_cast<uintptr_t>(signs) & 7) == 0 &&
      (o.codes == nullptr || (reinterpret_cast<uintptr_t>(o.codes) & 3) == 0)) {
    const int64_t threads = rows * (k / 8);
    const int64_t blocks = std::min<int64_t>((threads + 255) / 256, static_cast<int64_t>(sms) * 16);
    if (blocks == 0) return FAQ_OK;
#define FAQ_ROTS_CASE(L)                                                                                       \
  case L:                                                                                                      \
    hif4_rotate_signs_kernel<T, L><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(                          \
        static_cast<const T*>(x), rows, k, ldx, static_cast<const T*>(input_scale), signs, levels, o);          \
    return launch_status("hif4_rotate_signs_kernel");
    switch (log2b) {
      FAQ_ROTS_CASE(3)
      FAQ_ROTS_CASE(4)
      FAQ_ROTS_CASE(5)
      FAQ_ROTS_CASE(6)
      FAQ_ROTS_CASE(7)
      FAQ_ROTS_CASE(8)
      default:
        break;
    }
#undef FAQ_ROTS_CASE
  }
  if constexpr (sizeof(T) == 2) {
    const bool v4 = k % 1024 == 0 && k <= 16384 && x_vec && block >= 32 && block <= 1024 &&
                    (o.qdq == nullptr || (o.qdq_vec && o.ldq % 8 == 0)) &&
                    (o.codes == nullptr || aligned16(o.codes));
    if (v4) {
      // one warp per 1024-chunk: barriers, map (2 B per channel), two row buffers, one
      // 32 x 34 float transpose scratch per warp
      const int W = static_cast<int>(k / 1024);
      const size_t smem4 = v4_smem_bytes(k, kNormNone);
      if (smem4 <= 200 * 1024) {
        const int per_sm = std::max(1, std::min(16, static_cast<int>((227 * 1024) / (smem4 + 1024))));
        const int64_t blocks4 = std::min<int64_t>(rows, static_cast<int64_t>(sms) * per_sm);
        const bool codes = o.codes != nullptr;
        const int wclass = W <= 4 ? 4 : W <= 8 ? 8 : W <= 12 ? 12 : 16;
#define FAQ_ROT4_LAUNCH(L, MW)                                                                                     \
  {                                                                                                                \
    auto kern = codes ? hif4_rotate_v4_kernel<L, true, MW> : hif4_rotate_v4_kernel<L, false, MW>;                 \
    FAQ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem4)));   \
    kern<<<static_cast<unsigned>(blocks4), W * 32, smem4, stream>>>(                                               \
        static_cast<const __nv_bfloat16*>(x), rows, static_cast<int>(k), ldx,                                       \
        static_cast<const __nv_bfloat16*>(input_scale), signs, perm, levels, o, nullptr, 0.0f);                     \
    return launch_status("hif4_rotate_v4_kernel");                                                                \
  }
#define FAQ_ROT4_CASE(L)                 \
  case L:                                \
    if (wclass == 4) FAQ_ROT4_LAUNCH(L, 4)   \
    if (wclass == 8) FAQ_ROT4_LAUNCH(L, 8)   \
    if (wclass == 12) FAQ_ROT4_LAUNCH(L, 12) \
    FAQ_ROT4_LAUNCH(L, 16)
        switch (log2b) {
          FAQ_ROT4_CASE(5)
          FAQ_ROT4_CASE(6)
          FAQ_ROT4_CASE(7)
          FAQ_ROT4_CASE(8)
          FAQ_ROT4_CASE(9)
          FAQ_ROT4_CASE(10)
          default:
            break;
        }
#undef FAQ_ROT4_CASE
#undef FAQ_ROT4_LAUNCH
      }
    }
    const bool v2 = k % 64 == 0 && k <= 32768 && x_vec && (block >= 32 || k % 32 == 0) && block <= 1024;
    if (v2) {
      const size_t smem2 = 64 + (static_cast<size_t>(k) * 2 + 127) / 128 * 128 + static_cast<size_t>(k) * 4 +
                           static_cast<size_t>(k) * 4;
      if (smem2 <= 200 * 1024) {
        const int threads = k >= 8192 ? 512 : 256;
        const int per_sm = std::max(1, std::min(4, static_cast<int>((220 * 1024) / (smem2 + 1024))));
        const int64_t blocks2 = std::min<int64_t>(rows, static_cast<int64_t>(sms) * per_sm);
#define FAQ_ROT2_CASE(L)                                                                                          \
  case L: {                                                                                                       \
    auto kern = hif4_rotate_bf16_kernel<L>;                                                                       \
    FAQ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem2)));  \
    kern<<<static_cast<unsigned>(blocks2), threads, smem2, stream>>>(                                             \
        static_cast<const __nv_bfloat16*>(x), rows, static_cast<int>(k), ldx,                                      \
        static_cast<const __nv_bfloat16*>(input_scale), signs, perm, levels, o);                                   \
    return launch_status("hif4_rotate_bf16_kernel");                                                             \
  }
        switch (log2b) {
          FAQ_ROT2_CASE(0)
          FAQ_ROT2_CASE(1)
          FAQ_ROT2_CASE(2)
          FAQ_ROT2_CASE(3)
          FAQ_ROT2_CASE(4)
          FAQ_ROT2_CASE(5)
          FAQ_ROT2_CASE(6)
          FAQ_ROT2_CASE(7)
          FAQ_ROT2_CASE(8)
          FAQ_ROT2_CASE(9)
          FAQ_ROT2_CASE(10)
          default:
            break;
        }
#undef FAQ_ROT2_CASE
      }
    }
  }
  const int64_t k64 = (k + 63) / 64 * 64;
  const size_t smem = static_cast<size_t>((k * 4 + 15) / 16 * 16) + 2 * static_cast<size_t>(k64) * sizeof(T);
  if (smem > 220 * 1024)
    return fail(FAQ_ERR_UNSUPPORTED, "rotated row of k=" + std::to_string(k) + " does not fit in shared memory");
  const int per_sm = std::max(1, static_cast<int>((228 * 1024) / (smem + 1024)));
  const int64_t blocks = std::min<int64_t>(rows, static_cast<int64_t>(sms) * std::min(per_sm, 8));
  if (blocks == 0) return FAQ_OK;
#define FAQ_ROT_CASE(L)                                                                                         \
  case L: {                                                                                                     \
    auto kern = hif4_quantize_rotate_kernel<T, L>;                                                              \
    FAQ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem))); \
    kern<<<static_cast<unsigned>(blocks), 256, smem, stream>>>(static_cast<const T*>(x), rows, k, ldx,           \
                                                               static_cast<const T*>(input_scale), signs, perm, \
                                                               x_vec, levels, o);                               \
    return launch_status("hif4_quantize_rotate_kernel");                                                       \
  }
  switch (log2b) {
    FAQ_ROT_CASE(0)
    FAQ_ROT_CASE(1)
    FAQ_ROT_CASE(2)
    FAQ_ROT_CASE(3)
    FAQ_ROT_CASE(4)
    FAQ_ROT_CASE(5)
    FAQ_ROT_CASE(6)
    FAQ_ROT_CASE(7)
    FAQ_ROT_CASE(8)
    FAQ_ROT_CASE(9)
    FAQ_ROT_CASE(10)
    default:
      return fail(FAQ_ERR_UNSUPPORTED, "rotation block " + std::to_string(rot_block) + " > 1024");
  }
#undef FAQ_ROT_CASE
}

}  // namespace faq

using namespace faq;

extern "C" int faq_hif4_quantize(const void* x, int x_dtype, int64_t rows, int64_t k, int64_t ldx,
                                 const void* input_scale, const int8_t* signs, const int64_t* perm, int rot_block,
                                 int levels, uint8_t* codes, uint32_t* meta, void* qdq, int64_t ldq, void* stream) {
  FAQ_CHECK_ARG(x_dtype == FAQ_BF16 || x_dtype == FAQ_F32, "x_dtype must be FAQ_BF16 or FAQ_F32");
  FAQ_CHECK_ARG(rows >= 0 && k > 0, "need rows >= 0 and k > 0 (HiF4 does not support an empty axis)");
  FAQ_CHECK_ARG(x != nullptr || rows == 0, "x is null");
  FAQ_CHECK_ARG(ldx >= k, "ldx < k");
  FAQ_CHECK_ARG(valid_levels(levels), "levels must be 123, 12 or 13");
  FAQ_CHECK_ARG(codes || meta || qdq || rows == 0, "all outputs are null");
  FAQ_CHECK_ARG(qdq == nullptr || ldq >= k, "ldq < k");
  FAQ_CHECK_ARG(!codes || (reinterpret_cast<uintptr_t>(codes) & 3) == 0, "codes must be 4-byte aligned");
  FAQ_CHECK_ARG(!meta || (reinterpret_cast<uintptr_t>(meta) & 3) == 0, "meta must be 4-byte aligned");
  FAQ_CHECK_ARG(perm == nullptr || signs != nullptr, "a permutation needs signs (pass all-ones signs)");
  if (signs != nullptr) {
    FAQ_CHECK_ARG(rot_block >= 0 && (rot_block & (rot_block - 1)) == 0, "rot_block must be 0 or a power of two");
    FAQ_CHECK_ARG(rot_block == 0 || k % rot_block == 0, "k must be divisible by rot_block");
    FAQ_CHECK_ARG(k < (int64_t(1) << 30), "k too large");
  }
  if (rows == 0) return FAQ_OK;
  QuantOut o{codes, meta, qdq, ldq, false};
  const size_t es = x_dtype == FAQ_BF16 ? 2 : 4;
  o.qdq_vec = qdq && aligned16(qdq) && (ldq * static_cast<int64_t>(es)) % 16 == 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (x_dtype == FAQ_BF16)
    return launch_quantize<__nv_bfloat16>(x, rows, k, ldx, input_scale, signs, perm, rot_block, levels, o, s);
  return launch_quantize<float>(x, rows, k, ldx, input_scale, signs, perm, rot_block, levels, o, s);
}

namespace faq {
// K1 v4 behind a fused norm (kNormRms with its weight, kNormLayer without one)
template <int NORM>
int quantize_norm(const void* x, int64_t rows, int64_t k, int64_t ldx, const void* norm_weight, float eps,
                  const void* input_scale, const int8_t* signs, const int64_t* perm, int rot_block, int levels,
                  uint8_t* codes, uint32_t* meta, void* qdq, int64_t ldq, void* stream) {
  FAQ_CHECK_ARG(rows >= 0 && k > 0, "need rows >= 0 and k > 0");
  FAQ_CHECK_ARG(x != nullptr || rows == 0, "x is null");
  FAQ_CHECK_ARG(NORM != kNormRms || (norm_weight != nullptr && aligned16(norm_weight)),
                "norm_weight must be non-null and 16-byte aligned");
  FAQ_CHECK_ARG(eps >= 0.0f, "eps must be non-negative");
  FAQ_CHECK_ARG(valid_levels(levels), "levels must be 123, 12 or 13");
  FAQ_CHECK_ARG(qdq != nullptr || codes != nullptr || rows == 0, "qdq and codes are both null");
  FAQ_CHECK_ARG(qdq == nullptr || (ldq >= k && ldq % 8 == 0 && aligned16(qdq)),
                "qdq must be 16-byte aligned with ldq >= k, a multiple of 8");
  FAQ_CHECK_ARG(codes == nullptr || aligned16(codes), "codes must be 16-byte aligned");
  FAQ_CHECK_ARG(!meta || (reinterpret_cast<uintptr_t>(meta) & 3) == 0, "meta must be 4-byte aligned");
  FAQ_CHECK_ARG(signs != nullptr, "the fused norm feeds a rotation: signs are required");
  FAQ_CHECK_ARG((x == nullptr || aligned16(x)) && ldx >= k && ldx % 8 == 0 &&
                    (input_scale == nullptr || aligned16(input_scale)),
                "x must be 16-byte aligned with ldx >= k, a multiple of 8");
  FAQ_CHECK_ARG(rot_block >= 32 && rot_block <= 1024 && (rot_block & (rot_block - 1)) == 0,
                "rot_block must be a power of two in 32..1024");
  if (k % 1024 != 0 || k > 16384)
    return fail(FAQ_ERR_UNSUPPORTED, "the fused norm needs k a multiple of 1024, at most 16384");
  if (rows == 0) return FAQ_OK;
  const size_t smem = v4_smem_bytes(k, NORM);
  if (smem > 200 * 1024) return fail(FAQ_ERR_UNSUPPORTED, "row too long for the fused norm's shared memory");
  int log2b = 0;
  while ((1 << log2b) < rot_block) ++log2b;
  QuantOut o{codes, meta, qdq, ldq, true};
  const int W = static_cast<int>(k / 1024);
  const int per_sm = std::max(1, std::min(16, static_cast<int>((227 * 1024) / (smem + 1024))));
  const int64_t grid = std::min<int64_t>(rows, static_cast<int64_t>(num_sms()) * per_sm);
  const int wclass = W <= 4 ? 4 : W <= 8 ? 8 : W <= 12 ? 12 : 16;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define FAQ_ROTN_LAUNCH(L, MW)                                                                                       \
  {                                                                                                                \
    auto kern = codes ? hif4_rotate_v4_kernel<L, true, MW, NORM> : hif4_rotate_v4_kernel<L, false, MW, NORM>;       \
    FAQ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));    \
    kern<<<static_cast<unsigned>(grid), W * 32, smem, st>>>(                                                       \
        static_cast<const __nv_bfloat16*>(x), rows, static_cast<int>(k), ldx,                                       \
        static_cast<const __nv_bfloat16*>(input_scale), signs, perm, levels, o,                                     \
        static_cast<const __nv_bfloat16*>(norm_weight), eps);                                                       \
    return launch_status("hif4_rotate_v4_kernel (fused norm)");                                                 \
  }
#define FAQ_ROTN_CASE(L)                   \
  case L:                                  \
    if (wclass == 4) FAQ_ROTN_LAUNCH(L, 4)   \
    if (wclass == 8) FAQ_ROTN_LAUNCH(L, 8)   \
    if (wclass == 12) FAQ_ROTN_LAUNCH(L, 12) \
    FAQ_ROTN_LAUNCH(L, 16)
  switch (log2b) {
    FAQ_ROTN_CASE(5)
    FAQ_ROTN_CASE(6)
    FAQ_ROTN_CASE(7)
    FAQ_ROTN_CASE(8)
    FAQ_ROTN_CASE(9)
    FAQ_ROTN_CASE(10)
    default:
      break;
  }
#undef FAQ_ROTN_CASE
#undef FAQ_ROTN_LAUNCH
  return fail(FAQ_ERR_UNSUPPORTED, "rot_block outside 32..1024");
}
}  // namespace faq

extern "C" int faq_hif4_quantize_rms_norm(const void* x, int64_t rows, int64_t k, int64_t ldx, const void* norm_weight,
                                          float eps, const void* input_scale, const int8_t* signs,
                                          const int64_t* perm, int rot_block, int levels, uint8_t* codes,
                                          uint32_t* meta, void* qdq, int64_t ldq, void* stream) {
  return faq::quantize_norm<faq::kNormRms>(x, rows, k, ldx, norm_weight, eps, input_scale, signs, perm, rot_block,
                                           levels, codes, meta, qdq, ldq, stream);
}

extern "C" int faq_hif4_quantize_layer_norm(const void* x, int64_t rows, int64_t k, int64_t ldx, float eps,
                                            const void* input_scale, const int8_t* signs, const int64_t* perm,
                                            int rot_block, int levels, uint8_t* codes, uint32_t* meta, void* qdq,
                                            int64_t ldq, void* stream) {
  return faq::quantize_norm<faq::kNormLayer>(x, rows, k, ldx, nullptr, eps, input_scale, signs, perm, rot_block,
                                             levels, codes, meta, qdq, ldq, stream);
}

extern "C" int faq_hif4_quantize_act(const void* x, int act, int64_t rows, int64_t k, int64_t ldx,
                                     const void* input_scale, const int8_t* signs, int rot_block, int levels,
                                     uint8_t* codes, uint32_t* meta, void* qdq, int64_t ldq, void* stream) {
  FAQ_CHECK_ARG(act == FAQ_ACT_SWIGLU || act == FAQ_ACT_GELU_TANH, "act must be FAQ_ACT_SWIGLU or FAQ_ACT_GELU_TANH");
  FAQ_CHECK_ARG(rows >= 0 && k > 0 && k % 64 == 0, "need rows >= 0 and k a positive multiple of 64");
  FAQ_CHECK_ARG(x != nullptr || rows == 0, "x is null");
  FAQ_CHECK_ARG(ldx >= (act == FAQ_ACT_SWIGLU ? 2 * k : k), "ldx too small for the activation's input");
  FAQ_CHECK_ARG(valid_levels(levels), "levels must be 123, 12 or 13");
  FAQ_CHECK_ARG(codes || meta || qdq || rows == 0, "all outputs are null");
  FAQ_CHECK_ARG(qdq == nullptr || ldq >= k, "ldq < k");
  FAQ_CHECK_ARG(!codes || (reinterpret_cast<uintptr_t>(codes) & 3) == 0, "codes must be 4-byte aligned");
  FAQ_CHECK_ARG(!meta || (reinterpret_cast<uintptr_t>(meta) & 3) == 0, "meta must be 4-byte aligned");
  FAQ_CHECK_ARG(signs != nullptr && (reinterpret_cast<uintptr_t>(signs) & 7) == 0,
                "the fused activation path needs 8-byte aligned signs (a signs-only rotation)");
  FAQ_CHECK_ARG(rot_block >= 8 && rot_block <= 256 && (rot_block & (rot_block - 1)) == 0 && k % rot_block == 0,
                "rot_block must be a power of two in 8..256 dividing k");
  FAQ_CHECK_ARG((x == nullptr || aligned16(x)) && ldx % 8 == 0 && (input_scale == nullptr || aligned16(input_scale)),
                "x must be 16-byte aligned with ldx a multiple of 8");
  QuantOut o{codes, meta, qdq, ldq, false};
  o.qdq_vec = qdq && aligned16(qdq) && ldq % 8 == 0;
  FAQ_CHECK_ARG(qdq == nullptr || o.qdq_vec, "qdq must be 16-byte aligned with ldq a multiple of 8");
  if (rows == 0) return FAQ_OK;
  int log2b = 0;
  while ((1 << log2b) < rot_block) ++log2b;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  const auto* sc = static_cast<const __nv_bfloat16*>(input_scale);
  if (log2b == 6 && aligned16(signs) && (codes == nullptr || aligned16(codes))) {  // two lanes per block
    const int64_t blocks64 = std::min<int64_t>((rows * (k / 32) + 255) / 256, static_cast<int64_t>(num_sms()) * 8);
    const bool cd = codes != nullptr;
    if (act == FAQ_ACT_SWIGLU) {
      auto kern = cd ? hif4_rotate_signs64_kernel<FAQ_ACT_SWIGLU, true> : hif4_rotate_signs64_kernel<FAQ_ACT_SWIGLU, false>;
      kern<<<static_cast<unsigned>(blocks64), 256, 0, st>>>(xb, rows, k, ldx, sc, signs, levels, o);
    } else {
      auto kern = cd ? hif4_rotate_signs64_kernel<FAQ_ACT_GELU_TANH, true>
                     : hif4_rotate_signs64_kernel<FAQ_ACT_GELU_TANH, false>;
      kern<<<static_cast<unsigned>(blocks64), 256, 0, st>>>(xb, rows, k, ldx, sc, signs, levels, o);
    }
    return launch_status("hif4_rotate_signs64_kernel (fused activation)");
  }
  const int64_t blocks = std::min<int64_t>((rows * (k / 8) + 255) / 256, static_cast<int64_t>(num_sms()) * 16);
#define FAQ_ACT_CASE(L)                                                                                              \
  case L:                                                                                                            \
    if (act == FAQ_ACT_SWIGLU)                                                                                       \
      hif4_rotate_signs_kernel<__nv_bfloat16, L, FAQ_ACT_SWIGLU>                                                     \
          <<<static_cast<unsigned>(blocks), 256, 0, st>>>(xb, rows, k, ldx, sc, signs, levels, o);                   \
    else                                                                                                             \
      hif4_rotate_signs_kernel<__nv_bfloat16, L, FAQ_ACT_GELU_TANH>                                                  \
          <<<static_cast<unsigned>(blocks), 256, 0, st>>>(xb, rows, k, ldx, sc, signs, levels, o);                   \
    return launch_status("hif4_rotate_signs_kernel (fused activation)");
  switch (log2b) {
    FAQ_ACT_CASE(3)
    FAQ_ACT_CASE(4)
    FAQ_ACT_CASE(5)
    FAQ_ACT_CASE(6)
    FAQ_ACT_CASE(7)
    FAQ_ACT_CASE(8)
    default:
      break;
  }
#undef FAQ_ACT_CASE
  return fail(FAQ_ERR_UNSUPPORTED, "rot_block");
}

extern "C" int faq_hif4_dequantize(const uint8_t* codes, const uint32_t* meta, int64_t rows, int64_t k, void* out,
                                   int out_dtype, int64_t ldo, void* stream) {
  FAQ_CHECK_ARG(codes && meta && out, "null pointer");
  FAQ_CHECK_ARG(out_dtype == FAQ_BF16 || out_dtype == FAQ_F32, "out_dtype must be FAQ_BF16 or FAQ_F32");
  FAQ_CHECK_ARG(rows >= 0 && k > 0 && ldo >= k, "bad shape");
  FAQ_CHECK_ARG((reinterpret_cast<uintptr_t>(codes) & 3) == 0, "codes must be 4-byte aligned");
  if (rows == 0) return FAQ_OK;
  const int64_t k64 = (k + 63) / 64 * 64;
  const int64_t blocks = std::min<int64_t>((rows * (k64 / 8) + 255) / 256, static_cast<int64_t>(num_sms()) * 16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t es = out_dtype == FAQ_BF16 ? 2 : 4;
  const bool vec = aligned16(out) && (ldo * static_cast<int64_t>(es)) % 16 == 0;
  if (out_dtype == FAQ_BF16 && k % 64 == 0 && vec && rows * (k / 32) < (int64_t(1) << 31) &&
      (reinterpret_cast<uintptr_t>(codes) & 15) == 0 && (reinterpret_cast<uintptr_t>(meta) & 3) == 0) {
    const int64_t items = rows * (k / 32);
    const int64_t grid = (items + 255) / 256;
    hif4_expand_bf16_kernel<<<static_cast<unsigned>(grid), 256, 0, s>>>(
        codes, meta, static_cast<uint32_t>(rows), static_cast<uint32_t>(k), static_cast<__nv_bfloat16*>(out), ldo);
    return launch_status("hif4_expand_bf16_kernel");
  }
  if (out_dtype == FAQ_BF16)
    hif4_dequantize_kernel<__nv_bfloat16><<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        codes, meta, rows, k, static_cast<__nv_bfloat16*>(out), ldo, vec);
  else
    hif4_dequantize_kernel<float><<<static_cast<unsigned>(blocks), 256, 0, s>>>(codes, meta, rows, k,
                                                                                static_cast<float*>(out), ldo, vec);
  return launch_status("hif4_dequantize_kernel");
}

extern "C" int faq_hif4_pack_weight(const void* w, int w_dtype, int64_t n, int64_t k, int64_t ldw,
                                    const float* scale, const int8_t* lv2, const int8_t* lv3, int levels,
                                    uint8_t* codes, uint32_t* meta, unsigned long long* mismatches, void* stream) {
  FAQ_CHECK_ARG(w && codes && meta, "null pointer");
  FAQ_CHECK_ARG(w_dtype == FAQ_BF16 || w_dtype == FAQ_F32, "w_dtype must be FAQ_BF16 or FAQ_F32");
  FAQ_CHECK_ARG(n >= 0 && k > 0 && ldw >= k, "bad shape");
  FAQ_CHECK_ARG(valid_levels(levels), "levels must be 123, 12 or 13");
  FAQ_CHECK_ARG((scale == nullptr) == (lv2 == nullptr) && (scale == nullptr) == (lv3 == nullptr),
                "scale, lv2 and lv3 come together");
  FAQ_CHECK_ARG(scale == nullptr || k % 64 == 0, "GPTQ metadata needs k % 64 == 0");
  FAQ_CHECK_ARG((reinterpret_cast<uintptr_t>(codes) & 3) == 0 && (reinterpret_cast<uintptr_t>(meta) & 3) == 0,
                "codes/meta must be 4-byte aligned");
  if (n == 0) return FAQ_OK;
  const int64_t k64 = (k + 63) / 64 * 64;
  const int64_t blocks = std::min<int64_t>((n * (k64 / 8) + 255) / 256, static_cast<int64_t>(num_sms()) * 16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t es = w_dtype == FAQ_BF16 ? 2 : 4;
  const bool vec = aligned16(w) && (ldw * static_cast<int64_t>(es)) % 16 == 0;
  if (w_dtype == FAQ_BF16)
    hif4_pack_kernel<__nv_bfloat16><<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(w), n, k, ldw, scale, lv2, lv3, vec, levels, codes, meta, mismatches);
  else
    hif4_pack_kernel<float><<<static_cast<unsigned>(blocks), 256, 0, s>>>(
        static_cast<const float*>(w), n, k, ldw, scale, lv2, lv3, vec, levels, codes, meta, mismatches);
  return launch_status("hif4_pack_kernel");
}
