// K3s -- the W4A4 product for a few rows (decode, small batches): y[m, n] = A[m, :] . W[n, :]
// + bias (+ residual) with W in the packed HiF4 format of include/faquant_b200.h and A the
// activation's bf16 QDQ, m <= 16; faq_w4a4_gemm_qdq_a runs it for such m.
//
// A decode step reads every weight once for a handful of rows, so the weight bytes bound
// it: here W streams in its 4.5-bit form (0.5625 bytes per value against 2 for bf16) and
// is expanded in registers right before the tensor cores use it.
//   - One CTA per R = 8 or 16 weight rows: thread 0 copies the rows' codes and meta words
//     into shared memory with one cp.async.bulk per row (all of them in flight at once),
//     then eight warps split K, each over whole 64-value blocks.
//   - Products on mma.sync m16n8k16 (bf16 in, fp32 accumulate; the rows past m are zero).
//     Inside every 16-value step the reduction index is permuted so that lane (g, t) holds,
//     for weight row g, the four consecutive values 4t .. 4t + 3 -- one quarter of a
//     64-value block, so one scale word, and two code bytes -- and, for activation rows g
//     and g + 8, the same four columns (one 8-byte load each). Any permutation of the
//     reduction index applied to both operands leaves the sum unchanged.
//   - The expansion is the packed GEMM's (hif4_expand32_bf16): a byte permute gathers
//     [m0 | s0 at bit 15 | m1 | s1 at bit 31], (128 + m) as bf16 is exact, one bf16x2 FMA
//     with (c, -128 c) gives m c exactly, an xor restores the sign.
//   - The eight warps' partial sums meet in shared memory, added in warp order (a fixed
//     order: the same bits on every run), then bias, residual and the bf16 store as K3's
//     epilogue does them.
// The products are summed in another order than K3's tcgen05 tiles, so the result equals
// the bf16 GEMM on the dequantized operands up to fp32 rounding of the sums, not bit for bit.
#include "common.cuh"
#include "hif4.cuh"

namespace faq {
namespace w4s {

constexpr int WARPS = 8;
constexpr int THREADS = WARPS * 32;
constexpr int MAX_M = 16;

struct Params {
  const __nv_bfloat16* a;  // [m, lda], the QDQ activation (exact HiF4 values)
  int64_t lda;
  const uint8_t* codes;    // [n, k / 2]
  const uint32_t* meta;    // [n, k / 64]
  int m, n, k;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* residual;
  int64_t ldr;
  __nv_bfloat16* y;
  int64_t ldy;
};

// shared memory: codes [R][k/2 + 16] bytes, meta [R][k/64 + 4] words (rows padded by 16
// bytes, so the eight rows a warp reads at one offset fall on different banks; the rows stay
// 16-byte aligned for the bulk copies), partial sums [WARPS][R/8][32 lanes][4] floats, the
// copies' mbarrier
template <int R>
constexpr size_t partial_floats() {
  return static_cast<size_t>(WARPS) * (R / 8) * 32 * 4;
}
template <int R>
inline size_t smem_bytes(int k) {
  return static_cast<size_t>(R) * (k / 2 + 16) + static_cast<size_t>(R) * (k / 16 + 16) + partial_floats<R>() * 4 + 16;
}
constexpr size_t MAX_SMEM = 232448;  // the opt-in maximum per CTA

// The four values of one quarter (two code bytes in the low half of h) as two bf16 pairs,
// with c / nc the bf16x2 words of (scale 2^(lv2 + lv3 - 2), -128 times it).
__device__ __forceinline__ void expand_quarter(uint32_t h, uint32_t c, uint32_t nc, uint32_t& b0, uint32_t& b1) {
  const uint32_t r = __funnelshift_l(h, h, 4);
  const uint32_t x0 = __byte_perm(h, r, 0x0540);  // byte 0: [h.0, r.0, r.1, h.0]
  const uint32_t x1 = __byte_perm(h, r, 0x1651);  // byte 1: [h.1, r.1, r.2, h.1]
  b0 = hfma2_bf16((x0 & 0x00070007u) | 0x43004300u, c, nc) ^ (x0 & 0x80008000u);
  b1 = hfma2_bf16((x1 & 0x00070007u) | 0x43004300u, c, nc) ^ (x1 & 0x80008000u);
}

template <int R>
__global__ void __launch_bounds__(THREADS) w4a4_small_m_kernel(const __grid_constant__ Params p) {
  constexpr int NB = R / 8;  // n-blocks of 8 weight rows
  extern __shared__ __align__(16) unsigned char smem[];
  const int kc = p.k / 2, km = p.k / 64;
  const int kcs = kc + 16, kms = km + 4;  // padded row strides (bytes, words)
  unsigned char* s_codes = smem;
  uint32_t* s_meta = reinterpret_cast<uint32_t*>(smem + static_cast<size_t>(R) * kcs);
  float* s_part = reinterpret_cast<float*>(s_meta + static_cast<size_t>(R) * kms);
  uint64_t* bar = reinterpret_cast<uint64_t*>(s_part + partial_floats<R>());
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n0 = blockIdx.x * R;
  const int rows = min(R, p.n - n0);
  if (tid == 0) {
    mbar_init(smem_addr(bar), 1);
    fence_barrier_init();
    const uint32_t bytes = static_cast<uint32_t>(rows) * static_cast<uint32_t>(kc + 4 * km);
    mbar_arrive_expect_tx(smem_addr(bar), bytes);
    for (int r = 0; r < rows; ++r) {
      bulk_load(smem_addr(s_codes + static_cast<size_t>(r) * kcs), p.codes + static_cast<int64_t>(n0 + r) * kc,
                static_cast<uint32_t>(kc), smem_addr(bar));
      bulk_load(smem_addr(s_meta + static_cast<size_t>(r) * kms), p.meta + static_cast<int64_t>(n0 + r) * km,
                static_cast<uint32_t>(4 * km), smem_addr(bar));
    }
  }
  __syncthreads();
  const bool landed = __syncthreads_and(mbar_wait(smem_addr(bar), 0));
  if (!landed) {  // the status records the timeout; let the copies land (bounded) before leaving
    if (tid == 0) {
      trace_timeout(50, blockIdx.x);
      mbar_wait(smem_addr(bar), 0);
    }
    return;
  }
  const int g = lane >> 2, t = lane & 3;
  const int b0 = warp * km / WARPS, b1 = (warp + 1) * km / WARPS;  // this warp's 64-value blocks
  const __nv_bfloat16* a_lo = g < p.m ? p.a + static_cast<int64_t>(g) * p.lda : nullptr;
  const __nv_bfloat16* a_hi = g + 8 < p.m ? p.a + static_cast<int64_t>(g + 8) * p.lda : nullptr;
  float acc[NB][4];
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[nb][c] = 0.0f;
  // the activation fragments of a block (rows g and g + 8, four 16-value steps), loaded one
  // block ahead so that their L2 round trip overlaps the current block's products
  auto load_a = [&](int blk, uint2 (&lo)[4], uint2 (&hi)[4]) {
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const int col = 64 * blk + 16 * s + 4 * t;
      lo[s] = a_lo ? __ldg(reinterpret_cast<const uint2*>(a_lo + col)) : make_uint2(0u, 0u);
      hi[s] = a_hi ? __ldg(reinterpret_cast<const uint2*>(a_hi + col)) : make_uint2(0u, 0u);
    }
  };
  uint2 alo[4], ahi[4];
  if (b0 < b1) load_a(b0, alo, ahi);
  for (int blk = b0; blk < b1; ++blk) {
    uint2 nlo[4], nhi[4];
    if (blk + 1 < b1) load_a(blk + 1, nlo, nhi);
    uint32_t base_c[NB], base_n[NB], mw[NB];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      mw[nb] = s_meta[(nb * 8 + g) * kms + blk];
      const uint32_t sb = (mw[nb] & 0xFFu) << 5;  // the E6M2 code as bf16 exponent and mantissa bits, see hif4.cuh
      base_c[nb] = (sb + (77u << 7)) * 0x00010001u;
      base_n[nb] = ((sb + (84u << 7)) | 0x8000u) * 0x00010001u;
    }
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const uint32_t af[4] = {alo[s].x, ahi[s].x, alo[s].y, ahi[s].y};
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
        const uint32_t h =
            *reinterpret_cast<const uint16_t*>(s_codes + static_cast<size_t>(nb * 8 + g) * kcs + 32 * blk + 8 * s + 2 * t);
        const uint32_t e = ((mw[nb] >> (8 + 2 * s + (t >> 1))) & 1u) + ((mw[nb] >> (16 + 4 * s + t)) & 1u);
        uint32_t w0, w1;
        expand_quarter(h, base_c[nb] + e * 0x00800080u, base_n[nb] + e * 0x00800080u, w0, w1);
        mma_bf16_16816(acc[nb], af, w0, w1);
      }
    }
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      alo[s] = nlo[s];
      ahi[s] = nhi[s];
    }
  }
  // partial sums: [warp][nb][lane][fragment]
#pragma unroll
  for (int nb = 0; nb < NB; ++nb)
#pragma unroll
    for (int c = 0; c < 4; ++c) s_part[((warp * NB + nb) * 32 + lane) * 4 + c] = acc[nb][c];
  __syncthreads();
  // output (m, column j of this CTA's rows): fragment c holds row g (c < 2) or g + 8, column 2t + (c & 1)
  if (tid < MAX_M * R) {
    const int m = tid / R, j = tid % R;
    const int nb = j / 8, nn = j % 8;
    const int src_lane = (m & 7) * 4 + (nn >> 1), c = (nn & 1) + (m >= 8 ? 2 : 0);
    float sum = 0.0f;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) sum += s_part[((w * NB + nb) * 32 + src_lane) * 4 + c];
    const int n = n0 + j;
    if (m < p.m && j < rows) {
      float v = sum + (p.bias != nullptr ? __bfloat162float(p.bias[n]) : 0.0f);
      if (p.residual != nullptr) v = bf16_round(v) + __bfloat162float(p.residual[static_cast<int64_t>(m) * p.ldr + n]);
      p.y[static_cast<int64_t>(m) * p.ldy + n] = __float2bfloat16_rn(v);
    }
  }
}

// Whether the kernel takes this shape: m <= MAX_M and 8 weight rows fit in shared memory.
inline bool small_m_fits(int64_t m, int64_t k) { return m <= MAX_M && smem_bytes<8>(static_cast<int>(k)) <= MAX_SMEM; }

// Launch for small_m_fits shapes (the caller validated the operands as for the packed
// GEMM: k % 256 == 0, 16-byte aligned codes and meta, lda % 8 == 0).
static int launch_small_m(const Params& p, void* stream) {
  const bool wide = p.k <= 12288;  // 16 rows per CTA while their codes and meta fit twice per SM
  const size_t smem = wide ? smem_bytes<16>(p.k) : smem_bytes<8>(p.k);
  const int rows = wide ? 16 : 8;
  const unsigned grid = static_cast<unsigned>((p.n + rows - 1) / rows);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (wide) {
    FAQ_CUDA(cudaFuncSetAttribute(w4a4_small_m_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(smem)));
    w4a4_small_m_kernel<16><<<grid, THREADS, smem, s>>>(p);
  } else {
    FAQ_CUDA(cudaFuncSetAttribute(w4a4_small_m_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(smem)));
    w4a4_small_m_kernel<8><<<grid, THREADS, smem, s>>>(p);
  }
  return launch_status("w4a4_small_m_kernel");
}

}  // namespace w4s
}  // namespace faq
