// K6 -- HiF4 attention decode (a few new query positions against a long K/V cache).
//
// Semantics are the prefill kernel's (K5) and the reference simulator's
// (simulated_flash_attention.py:623-884 with query_length <= 16): key tiles of 128 from
// key 0 in order, the running max including the current tile, P = exp(s - max)
// HiF4-quantized (unsigned) in groups of 64 keys inside each tile, the denominator from
// the quantized P (P-Reordering) or the raw P, O = alpha O + P V, out = O / denominator;
// the queries are the last sq positions of the sequence (bottom-right causal).
//
// A decode step reads the whole cache for very little arithmetic, so it must spread the
// keys over the GPU. The running max makes a plain split-K inexact -- P of a tile is
// quantized relative to the max through that tile, not a split's local max. Here the max
// is known before any P is formed:
//   pass 1  (grid: key tiles x (batch, kv head)) raw scores q.k for the G = hq / hkv query
//           heads x sq positions of the group (R rows) and each tile's per-row max, into
//           the workspace;
//   pass 2  (grid: splits of SPLIT_TILES tiles x (batch, kv head)) every split starts from
//           the exact running max before its first tile (a max over the pass-1 tile maxima),
//           so each tile's P, its HiF4 codes and its alpha are the sequential ones; the
//           split's O and denominator are carried exactly as the sequential loop carries
//           them, from the split's first tile;
//   pass 3  (grid: (batch, kv head)) joins the splits: O = sum_s O_s exp2(m_s - m_end), the
//           same for the denominator (what the sequential alphas multiply to, up to fp32
//           rounding order), out = O / denominator in bf16.
// All three are CUDA-core kernels: R <= 32 rows is far from a tensor-core tile, and the
// cache bytes, not the FLOPs, bound a decode step.
#include "common.cuh"
#include "hif4.cuh"

namespace faq {
namespace dec {

constexpr int D = 128;
constexpr int TILE = 128;        // keys per tile (the reference's key chunk)
constexpr int SPLIT_TILES = 8;   // tiles per pass-2 split
constexpr int MAX_ROWS = 32;     // G * sq
constexpr int THREADS = 256;

struct Params {
  const __nv_bfloat16 *q, *k, *v;
  int64_t qb, qh, qs, kb, kh, ks, vb, vh, vs;
  int batch, hq, hkv, group, sq, sk, rows, ntiles, nsplits;
  float scale_log2;  // scale * log2(e)
  int p_levels;      // 0: P not quantized
  int raw_normalizer;
  __nv_bfloat16* out;
  int64_t ob, os, oh;
  float* scores;     // [B*hkv][rows][ntiles*TILE] raw q.k
  float* tmax;       // [B*hkv][rows][ntiles] raw per-tile row max (-inf: fully masked)
  float* part_o;     // [B*hkv][nsplits][rows][D]
  float* part_l;     // [B*hkv][nsplits][rows]
  float* part_m;     // [B*hkv][nsplits][rows] log2-domain running max after the split
};

// workspace sections, each rounded up to 16 floats (64 bytes) so every section starts aligned
__host__ __device__ inline int64_t round16(int64_t n) { return (n + 15) / 16 * 16; }
__host__ __device__ inline size_t workspace_floats(int64_t bh, int64_t rows, int64_t ntiles, int64_t nsplits) {
  return static_cast<size_t>(round16(bh * rows * ntiles * TILE) + round16(bh * rows * ntiles) +
                             round16(bh * nsplits * rows * D) + 2 * round16(bh * nsplits * rows));
}

// row r of a group: query head g = r / sq, query position i = r % sq; its last visible key
__device__ __forceinline__ int last_key(const Params& p, int r) { return p.sk - p.sq + (r % p.sq); }

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem)), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all_but_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ---------------------------------------------------------------- pass 1
// A half-warp per key (16 lanes x 8 channels), two keys per warp step; the R query rows
// of the group sit in shared memory as fp32.
constexpr int KS = D + 8;  // staged K row stride (elements): 16 bytes of padding per row
                           // puts neighbouring keys on different banks
// Scores of rows r0 .. r0 + RC - 1 for the whole tile: a half-warp per key (8 channels
// per lane, keys from the staged tile), the rows' q channels in registers. The RC partial
// dot products of a lane are reduced over the 16 lanes by a transposed butterfly -- each
// exchange keeps half of the rows and sends the other half (8 rows: 4 + 2 + 1 + 1
// shuffles instead of 8 x 4; 4 rows: 2 + 1 + 1 + 1) -- and lane (16 / RC) j ends with
// row j's total. Rows past p.rows read zero q rows and are not stored.
template <int RC>
__device__ __forceinline__ void score_rows(const Params& p, const __nv_bfloat16* s_k, const float* s_q, float* s_s,
                                           int tile, int warp, int half, int sub, int r0) {
  constexpr int STEPS = TILE / (2 * (THREADS / 32));
  float qr[RC][8];
#pragma unroll
  for (int j = 0; j < RC; ++j) {
    const float4 qa = *reinterpret_cast<const float4*>(s_q + (r0 + j) * D + sub * 8);
    const float4 qc = *reinterpret_cast<const float4*>(s_q + (r0 + j) * D + sub * 8 + 4);
    qr[j][0] = qa.x; qr[j][1] = qa.y; qr[j][2] = qa.z; qr[j][3] = qa.w;
    qr[j][4] = qc.x; qr[j][5] = qc.y; qr[j][6] = qc.z; qr[j][7] = qc.w;
  }
#pragma unroll 2
  for (int step = 0; step < STEPS; ++step) {
    const int kk = step * 2 * (THREADS / 32) + warp * 2 + half;
    const int key = tile * TILE + kk;
    const uint4 kcur = *reinterpret_cast<const uint4*>(s_k + kk * KS + sub * 8);
    const uint32_t w[4] = {kcur.x, kcur.y, kcur.z, kcur.w};
    float kv[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      kv[2 * i] = __uint_as_float(w[i] << 16);
      kv[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
    float v[RC];
#pragma unroll
    for (int j = 0; j < RC; ++j) {
      float acc = __fmul_rn(qr[j][0], kv[0]);
#pragma unroll
      for (int c = 1; c < 8; ++c) acc = __fmaf_rn(qr[j][c], kv[c], acc);
      v[j] = acc;
    }
    const bool b3 = sub & 8, b2 = sub & 4, b1 = sub & 2;
    float tot;
    int r;
    if constexpr (RC == 8) {
      float u4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float send = b3 ? v[i] : v[i + 4];
        const float keep = b3 ? v[i + 4] : v[i];
        u4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
      }
      float u2[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float send = b2 ? u4[i] : u4[i + 2];
        const float keep = b2 ? u4[i + 2] : u4[i];
        u2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
      }
      const float send = b1 ? u2[0] : u2[1];
      const float keep = b1 ? u2[1] : u2[0];
      tot = keep + __shfl_xor_sync(0xffffffffu, send, 2);
      tot += __shfl_xor_sync(0xffffffffu, tot, 1);
      r = r0 + (b3 ? 4 : 0) + (b2 ? 2 : 0) + (b1 ? 1 : 0);
    } else {
      float u2[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float send = b3 ? v[i] : v[i + 2];
        const float keep = b3 ? v[i + 2] : v[i];
        u2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
      }
      const float send = b2 ? u2[0] : u2[1];
      const float keep = b2 ? u2[1] : u2[0];
      tot = keep + __shfl_xor_sync(0xffffffffu, send, 4);
      tot += __shfl_xor_sync(0xffffffffu, tot, 2);
      tot += __shfl_xor_sync(0xffffffffu, tot, 1);
      r = r0 + (b3 ? 2 : 0) + (b2 ? 1 : 0);
    }
    const bool writer = (sub & (16 / RC - 1)) == 0;
    if (writer && r < p.rows) s_s[r * TILE + kk] = (key <= last_key(p, r)) ? tot : -INFINITY;
  }
}

// Dynamic shared memory: the K tile (staged by cp.async, all of it in flight at once),
// the group's q rows in fp32, the tile's scores.
constexpr size_t SCORES_SMEM = TILE * KS * 2 + MAX_ROWS * D * 4 + MAX_ROWS * TILE * 4;

__global__ void __launch_bounds__(THREADS, 2) decode_scores_kernel(Params p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* s_k = reinterpret_cast<__nv_bfloat16*>(smem_raw);   // [TILE][D]
  float* s_q = reinterpret_cast<float*>(s_k + TILE * KS);             // [MAX_ROWS][D]
  float* s_s = s_q + MAX_ROWS * D;                                    // [MAX_ROWS][TILE]
  const int tile = blockIdx.x, bh = blockIdx.y;
  const int b = bh / p.hkv, hk = bh % p.hkv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  {
    const __nv_bfloat16* kbase = p.k + b * p.kb + hk * p.kh;
    for (int i = tid; i < TILE * D / 8; i += THREADS) {
      const int key = tile * TILE + i / (D / 8), c8 = i % (D / 8);
      __nv_bfloat16* dst = s_k + (i / (D / 8)) * KS + c8 * 8;
      if (key < p.sk)
        cp_async16(dst, kbase + static_cast<int64_t>(key) * p.ks + c8 * 8);
      else
        *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
    cp_async_commit();
  }
  const int rows8 = (p.rows + 7) / 8 * 8;
  for (int i = tid; i < rows8 * (D / 8); i += THREADS) {  // 8 channels per thread, 16-byte loads
    const int r = i / (D / 8), c8 = i % (D / 8);
    float4 lo = make_float4(0.f, 0.f, 0.f, 0.f), hi = lo;
    if (r < p.rows) {
      const int g = r / p.sq, pos = r % p.sq;  // query head in the group, position in q
      const uint4 u = *reinterpret_cast<const uint4*>(p.q + b * p.qb + static_cast<int64_t>(hk * p.group + g) * p.qh +
                                                      static_cast<int64_t>(pos) * p.qs + c8 * 8);
      lo = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u), __uint_as_float(u.y << 16),
                       __uint_as_float(u.y & 0xFFFF0000u));
      hi = make_float4(__uint_as_float(u.z << 16), __uint_as_float(u.z & 0xFFFF0000u), __uint_as_float(u.w << 16),
                       __uint_as_float(u.w & 0xFFFF0000u));
    }
    *reinterpret_cast<float4*>(s_q + r * D + c8 * 8) = lo;
    *reinterpret_cast<float4*>(s_q + r * D + c8 * 8 + 4) = hi;
  }
  cp_async_wait_all();
  __syncthreads();
  const int half = lane >> 4, sub = lane & 15;
  if (p.rows <= 4)
    score_rows<4>(p, s_k, s_q, s_s, tile, warp, half, sub, 0);
  else
    for (int r0 = 0; r0 < p.rows; r0 += 8) score_rows<8>(p, s_k, s_q, s_s, tile, warp, half, sub, r0);
  __syncthreads();
  float* dst = p.scores + (static_cast<int64_t>(bh) * p.rows) * (p.ntiles * TILE) + static_cast<int64_t>(tile) * TILE;
  for (int i = tid; i < p.rows * TILE; i += THREADS) {
    const int r = i / TILE, kk = i % TILE;
    dst[static_cast<int64_t>(r) * (p.ntiles * TILE) + kk] = s_s[i];
  }
  // per-row tile max: one warp per row
  for (int r = warp; r < p.rows; r += THREADS / 32) {
    float m = -INFINITY;
    for (int kk = lane; kk < TILE; kk += 32) m = fmaxf(m, s_s[r * TILE + kk]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) p.tmax[(static_cast<int64_t>(bh) * p.rows + r) * p.ntiles + tile] = m;
  }
}

// ---------------------------------------------------------------- pass 2
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}


// Dynamic shared memory: two V tiles (the next one arrives by cp.async while this one is
// multiplied), P of the tile in bf16, the two key halves' partial O, per-row scalars.
constexpr size_t PV_SMEM = 2 * TILE * D * 2 + MAX_ROWS * TILE * 2 + 2 * MAX_ROWS * D * 4 + 3 * MAX_ROWS * 4;

__global__ void __launch_bounds__(THREADS) decode_pv_kernel(Params p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* s_vbuf = reinterpret_cast<__nv_bfloat16*>(smem_raw);                     // [2][TILE][D]
  __nv_bfloat16* s_p = s_vbuf + 2 * TILE * D;                                              // [MAX_ROWS][TILE]
  float* s_o = reinterpret_cast<float*>(s_p + MAX_ROWS * TILE);                            // [2][MAX_ROWS][D]
  float* s_m = s_o + 2 * MAX_ROWS * D;
  float* s_alpha = s_m + MAX_ROWS;
  float* s_sum = s_alpha + MAX_ROWS;
  const int split = blockIdx.x, bh = blockIdx.y;
  const int b = bh / p.hkv, hk = bh % p.hkv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t0 = split * SPLIT_TILES, t1 = min(p.ntiles, t0 + SPLIT_TILES);
  const float* tmax = p.tmax + static_cast<int64_t>(bh) * p.rows * p.ntiles;
  const __nv_bfloat16* vbase = p.v + b * p.vb + hk * p.vh;
  auto prefetch_v = [&](int t, int buf) {
    __nv_bfloat16* dst = s_vbuf + buf * TILE * D;
    for (int i = tid; i < TILE * D / 8; i += THREADS) {
      const int key = t * TILE + i / (D / 8), c8 = i % (D / 8);
      if (key < p.sk)
        cp_async16(dst + i * 8, vbase + static_cast<int64_t>(key) * p.vs + c8 * 8);
      else
        *reinterpret_cast<uint4*>(dst + i * 8) = make_uint4(0, 0, 0, 0);
    }
    cp_async_commit();
  };
  prefetch_v(t0, 0);
  // running max before the split (log2 domain): max over the earlier tiles' maxima
  for (int r = warp; r < p.rows; r += THREADS / 32) {
    float m = -INFINITY;
    for (int t = lane; t < t0; t += 32) m = fmaxf(m, tmax[r * p.ntiles + t]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) s_m[r] = m == -INFINITY ? -INFINITY : __fmul_rn(m, p.scale_log2);
  }
  // P.V work split: warp = (key half kh, row group rg); rows rg*rpw .. rg*rpw + rpw - 1,
  // keys 64 kh .. 64 kh + 63 of each tile; lane = 4 channels
  const int kh = warp & 1, rg = warp >> 1;
  const int rpw = (p.rows + 3) / 4;  // <= 8
  float acc[8][4];
  float l_run[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    l_run[j] = 0.0f;
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[j][c] = 0.0f;
  }
  __syncthreads();
  const float* sc = p.scores + static_cast<int64_t>(bh) * p.rows * (p.ntiles * TILE);
  for (int t = t0; t < t1; ++t) {
    const int buf = (t - t0) & 1;
    if (t + 1 < t1) {
      prefetch_v(t + 1, buf ^ 1);
    } else {
      cp_async_commit();  // an empty group keeps the wait count uniform
    }
    // new running max and alpha per row (the reference's order: max includes this tile)
    if (tid < p.rows) {
      const float tm = tmax[tid * p.ntiles + t];
      const float m_old = s_m[tid];
      const float m_new = fmaxf(m_old, tm == -INFINITY ? -INFINITY : __fmul_rn(tm, p.scale_log2));
      const float m_use = m_new == -INFINITY ? 0.0f : m_new;
      s_alpha[tid] = m_old == -INFINITY ? 0.0f : ex2(__fsub_rn(m_old, m_use));
      s_m[tid] = m_new;
      s_sum[tid] = 0.0f;
    }
    __syncthreads();
    // P = exp2(s c - m), HiF4 per 64 keys: 8 lanes x 8 keys per group, four groups per warp
    const int ngroups = p.rows * (TILE / 64);
    for (int g0 = warp * 4; g0 < ngroups; g0 += 4 * (THREADS / 32)) {  // warp-uniform bound
      const int grp = g0 + (lane >> 3);
      const bool live = grp < ngroups;
      const int r = live ? grp / (TILE / 64) : 0, half = grp % (TILE / 64);
      const int kk0 = half * 64 + (lane & 7) * 8;
      const float m = s_m[r];
      const float m_use = m == -INFINITY ? 0.0f : m;
      float v8[8];
      const float* srow = sc + static_cast<int64_t>(r) * (p.ntiles * TILE) + t * TILE + kk0;
      const float4 sa = live ? *reinterpret_cast<const float4*>(srow) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      const float4 sb = live ? *reinterpret_cast<const float4*>(srow + 4) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      const float sv[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) v8[i] = sv[i] == -INFINITY ? 0.0f : ex2(__fmaf_rn(sv[i], p.scale_log2, -m_use));
      float raw = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) raw = __fadd_rn(raw, v8[i]);
      float q8[8];
      if (p.p_levels != 0) {
        uint32_t meta;
        hif4_quant8(v8, p.p_levels, q8, meta);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) q8[i] = bf16_round(v8[i]);  // P enters the PV product as bf16
      }
      float qs = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) qs = __fadd_rn(qs, q8[i]);
      float contrib = (p.raw_normalizer || p.p_levels == 0) ? raw : qs;
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) contrib = __fadd_rn(contrib, __shfl_xor_sync(0xffffffffu, contrib, o));
      if (live) {
#pragma unroll
        for (int i = 0; i < 8; ++i) s_p[r * TILE + kk0 + i] = __float2bfloat16_rn(q8[i]);  // exact for HiF4
        if ((lane & 7) == 0) atomicAdd(&s_sum[r], contrib);
      }
    }
    cp_async_wait_all_but_one();  // this tile's V landed (the next one may still be in flight)
    __syncthreads();
    // O = alpha O + P V over this warp's key half; l = alpha l + sum (key half 0 keeps l)
    const __nv_bfloat16* vt = s_vbuf + buf * TILE * D;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int r = rg * rpw + j;
      if (j < rpw && r < p.rows) {
        const float a = s_alpha[r];
        float o0 = acc[j][0] * a, o1 = acc[j][1] * a, o2 = acc[j][2] * a, o3 = acc[j][3] * a;
        const __nv_bfloat16* pr = s_p + r * TILE + kh * 64;
        const __nv_bfloat16* vr = vt + (kh * 64) * D + lane * 4;
#pragma unroll 4
        for (int kk = 0; kk < 64; ++kk) {
          const float pv = __bfloat162float(pr[kk]);
          const uint2 u = *reinterpret_cast<const uint2*>(vr + kk * D);
          o0 = __fmaf_rn(pv, __uint_as_float(u.x << 16), o0);
          o1 = __fmaf_rn(pv, __uint_as_float(u.x & 0xFFFF0000u), o1);
          o2 = __fmaf_rn(pv, __uint_as_float(u.y << 16), o2);
          o3 = __fmaf_rn(pv, __uint_as_float(u.y & 0xFFFF0000u), o3);
        }
        acc[j][0] = o0;
        acc[j][1] = o1;
        acc[j][2] = o2;
        acc[j][3] = o3;
        l_run[j] = __fadd_rn(__fmul_rn(a, l_run[j]), s_sum[r]);
      }
    }
    __syncthreads();  // P, the scalars and this V buffer are rewritten next tile
  }
  cp_async_wait_all_but_one();
  asm volatile("cp.async.wait_all;" ::: "memory");
  // join the two key halves, write the split's partial state
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int r = rg * rpw + j;
    if (j < rpw && r < p.rows)
      *reinterpret_cast<float4*>(s_o + (kh * MAX_ROWS + r) * D + lane * 4) =
          make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
  }
  __syncthreads();
  const int64_t base = (static_cast<int64_t>(bh) * p.nsplits + split) * p.rows;
  for (int i = tid; i < p.rows * D; i += THREADS) {
    const int r = i / D, dd = i % D;
    p.part_o[(base + r) * D + dd] = __fadd_rn(s_o[r * D + dd], s_o[(MAX_ROWS + r) * D + dd]);
  }
  if (kh == 0) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int r = rg * rpw + j;
      if (j < rpw && r < p.rows && lane == 0) {
        p.part_l[base + r] = l_run[j];
        p.part_m[base + r] = s_m[r];
      }
    }
  }
}

// ---------------------------------------------------------------- pass 3
__global__ void __launch_bounds__(D) decode_combine_kernel(Params p) {
  const int bh = blockIdx.x, r = blockIdx.y, dd = threadIdx.x;  // one CTA per (batch, kv head, row)
  const int b = bh / p.hkv, hk = bh % p.hkv;
  {
    const int64_t base = static_cast<int64_t>(bh) * p.nsplits * p.rows;
    const float m_end = p.part_m[base + static_cast<int64_t>(p.nsplits - 1) * p.rows + r];
    const float m_use = m_end == -INFINITY ? 0.0f : m_end;
    float o = 0.0f, l = 0.0f;
#pragma unroll 8
    for (int s = 0; s < p.nsplits; ++s) {  // unrolled: the splits' loads are independent
      const float ms = p.part_m[base + static_cast<int64_t>(s) * p.rows + r];
      const float f = ms == -INFINITY ? 0.0f : ex2(__fsub_rn(ms, m_use));
      o = __fmaf_rn(p.part_o[(base + static_cast<int64_t>(s) * p.rows + r) * D + dd], f, o);
      l = __fmaf_rn(p.part_l[base + static_cast<int64_t>(s) * p.rows + r], f, l);
    }
    const float y = l > 0.0f ? __fdiv_rn(o, l) : 0.0f;
    const int g = r / p.sq, i_pos = r % p.sq;
    p.out[b * p.ob + static_cast<int64_t>(i_pos) * p.os + static_cast<int64_t>(hk * p.group + g) * p.oh + dd] =
        __float2bfloat16_rn(y);
  }
}

}  // namespace dec
}  // namespace faq

namespace faq {
static int decode_setup(dec::Params& p, const void* q, const void* k, const void* v, int64_t batch, int64_t hq,
                        int64_t hkv, int64_t sq, int64_t sk, int d, int64_t qb, int64_t qh, int64_t qs, int64_t kb,
                        int64_t kh, int64_t ks, int64_t vb, int64_t vh, int64_t vs, float scale, int p_levels,
                        int normalizer_quantized, void* out, int64_t ob, int64_t os, int64_t oh) {
  FAQ_CHECK_ARG(q && k && v && out, "null pointer");
  FAQ_CHECK_ARG(batch > 0 && hq > 0 && hkv > 0 && sq > 0 && sk >= sq, "bad shape (need sk >= sq > 0)");
  FAQ_CHECK_ARG(hq % hkv == 0, "query heads must be divisible by key/value heads");
  if (d != dec::D) return fail(FAQ_ERR_UNSUPPORTED, "head_dim must be 128");
  FAQ_CHECK_ARG((hq / hkv) * sq <= dec::MAX_ROWS, "decode handles at most 32 rows per kv head ((hq / hkv) * sq)");
  FAQ_CHECK_ARG(sk < (int64_t(1) << 30), "cache too long");
  FAQ_CHECK_ARG(p_levels == 0 || p_levels == 123 || p_levels == 12 || p_levels == 13, "p_levels must be 0/123/12/13");
  FAQ_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && qb % 8 == 0 && qh % 8 == 0 && qs % 8 == 0 &&
                    kb % 8 == 0 && kh % 8 == 0 && ks % 8 == 0 && vb % 8 == 0 && vh % 8 == 0 && vs % 8 == 0,
                "Q/K/V must be 16-byte aligned with strides multiple of 8");
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.qb = qb; p.qh = qh; p.qs = qs; p.kb = kb; p.kh = kh; p.ks = ks; p.vb = vb; p.vh = vh; p.vs = vs;
  p.batch = static_cast<int>(batch);
  p.hq = static_cast<int>(hq);
  p.hkv = static_cast<int>(hkv);
  p.group = static_cast<int>(hq / hkv);
  p.sq = static_cast<int>(sq);
  p.sk = static_cast<int>(sk);
  p.rows = p.group * p.sq;
  p.ntiles = static_cast<int>((sk + dec::TILE - 1) / dec::TILE);
  p.nsplits = (p.ntiles + dec::SPLIT_TILES - 1) / dec::SPLIT_TILES;
  p.scale_log2 = static_cast<float>(static_cast<double>(scale) * 1.4426950408889634);
  p.p_levels = p_levels;
  p.raw_normalizer = !normalizer_quantized;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ob = ob; p.os = os; p.oh = oh;
  return FAQ_OK;
}

static int decode_launch(dec::Params& p, float* ws, void* stream) {
  const int64_t bh = static_cast<int64_t>(p.batch) * p.hkv;
  p.scores = ws;
  p.tmax = p.scores + dec::round16(bh * p.rows * p.ntiles * dec::TILE);
  p.part_o = p.tmax + dec::round16(bh * p.rows * p.ntiles);
  p.part_l = p.part_o + dec::round16(bh * p.nsplits * p.rows * dec::D);
  p.part_m = p.part_l + dec::round16(bh * p.nsplits * p.rows);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  FAQ_CHECK_ARG(bh <= 65535, "batch * kv heads must be <= 65535");
  FAQ_CUDA(cudaFuncSetAttribute(dec::decode_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(dec::SCORES_SMEM)));
  dec::decode_scores_kernel<<<dim3(p.ntiles, static_cast<unsigned>(bh)), dec::THREADS, dec::SCORES_SMEM, st>>>(p);
  FAQ_CUDA(cudaFuncSetAttribute(dec::decode_pv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(dec::PV_SMEM)));
  dec::decode_pv_kernel<<<dim3(p.nsplits, static_cast<unsigned>(bh)), dec::THREADS, dec::PV_SMEM, st>>>(p);
  dec::decode_combine_kernel<<<dim3(static_cast<unsigned>(bh), static_cast<unsigned>(p.rows)), dec::D, 0, st>>>(p);
  return launch_status("hif4 decode kernels");
}
}  // namespace faq

extern "C" size_t faq_hif4_decode_workspace_bytes(int64_t batch, int64_t hq, int64_t hkv, int64_t sq, int64_t sk,
                                                  int d) {
  using namespace faq;
  if (batch <= 0 || hkv <= 0 || hq <= 0 || sq <= 0 || sk <= 0 || d != dec::D || hq % hkv) return 0;
  const int64_t rows = (hq / hkv) * sq, ntiles = (sk + dec::TILE - 1) / dec::TILE;
  const int64_t nsplits = (ntiles + dec::SPLIT_TILES - 1) / dec::SPLIT_TILES;
  return dec::workspace_floats(batch * hkv, rows, ntiles, nsplits) * sizeof(float);
}

extern "C" int faq_hif4_decode_attention(const void* q, const void* k, const void* v, int64_t batch, int64_t hq,
                                         int64_t hkv, int64_t sq, int64_t sk, int d, int64_t qb, int64_t qh,
                                         int64_t qs, int64_t kb, int64_t kh, int64_t ks, int64_t vb, int64_t vh,
                                         int64_t vs, float scale, int p_levels, int normalizer_quantized, void* out,
                                         int64_t ob, int64_t os, int64_t oh, void* workspace, size_t workspace_bytes,
                                         void* stream) {
  using namespace faq;
  dec::Params p;
  int rc = decode_setup(p, q, k, v, batch, hq, hkv, sq, sk, d, qb, qh, qs, kb, kh, ks, vb, vh, vs, scale, p_levels,
                        normalizer_quantized, out, ob, os, oh);
  if (rc) return rc;
  const size_t need = faq_hif4_decode_workspace_bytes(batch, hq, hkv, sq, sk, d);
  FAQ_CHECK_ARG(workspace != nullptr && aligned16(workspace), "workspace must be a 16-byte aligned device buffer");
  FAQ_CHECK_ARG(workspace_bytes >= need, "workspace too small: faq_hif4_decode_workspace_bytes() bytes needed");
  return decode_launch(p, static_cast<float*>(workspace), stream);
}

// ---------------------------------------------------------------- allocation-free decode
// A decode call for callers that cannot allocate device memory: a serving runtime that
// plans all of its memory at start-up and forbids allocations while it serves, or a host
// hot path where cudaMalloc would synchronize the device. Instead of a caller workspace
// the three passes use one file-scope scratch array of FAQ_DECODE_STATIC_SCRATCH_BYTES
// (16 MiB), which every GPU that loads this library holds until the process exits.
//   - The kernels write every scratch word they read within the same call (scores and
//     tile maxima in pass 1, partial results in pass 2), so nothing has to start at zero.
//   - All calls on a device share the one array: calls that may overlap on that GPU
//     (different streams without ordering between them) race; order them on one stream.
//   - The array's device address is looked up (cudaGetSymbolAddress) on the first call on
//     each device, with that device current, and cached; make that first call before
//     any stream capture. No call allocates.
namespace faq {
namespace dec {
constexpr size_t STATIC_SCRATCH_BYTES = size_t(16) << 20;
static __device__ __align__(256) float g_static_scratch[STATIC_SCRATCH_BYTES / sizeof(float)];
constexpr int MAX_DEVICES = 64;
static float* g_static_scratch_ptr[MAX_DEVICES] = {};
static std::mutex g_static_scratch_mutex;

static int static_scratch(float** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice");
  if (dev < 0 || dev >= MAX_DEVICES) return fail(FAQ_ERR_UNSUPPORTED, "device ordinal beyond 63");
  std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
  if (g_static_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_static_scratch);
    if (err != cudaSuccess) return cuda_fail(err, "cudaGetSymbolAddress(decode scratch)");
    g_static_scratch_ptr[dev] = static_cast<float*>(ptr);
  }
  *out = g_static_scratch_ptr[dev];
  return FAQ_OK;
}
}  // namespace dec
}  // namespace faq

extern "C" int faq_hif4_decode_attention_static(const void* q, const void* k, const void* v, int64_t batch,
                                                int64_t hq, int64_t hkv, int64_t sq, int64_t sk, int d, int64_t qb,
                                                int64_t qh, int64_t qs, int64_t kb, int64_t kh, int64_t ks,
                                                int64_t vb, int64_t vh, int64_t vs, float scale, int p_levels,
                                                int normalizer_quantized, void* out, int64_t ob, int64_t os,
                                                int64_t oh, void* stream) {
  using namespace faq;
  dec::Params p;
  int rc = decode_setup(p, q, k, v, batch, hq, hkv, sq, sk, d, qb, qh, qs, kb, kh, ks, vb, vh, vs, scale, p_levels,
                        normalizer_quantized, out, ob, os, oh);
  if (rc) return rc;
  const size_t need = faq_hif4_decode_workspace_bytes(batch, hq, hkv, sq, sk, d);
  if (need > dec::STATIC_SCRATCH_BYTES)
    return fail(FAQ_ERR_ARG, "decode needs " + std::to_string(need) +
                                 " bytes of scratch, more than the 16 MiB static array of "
                                 "faq_hif4_decode_attention_static; use faq_hif4_decode_attention with a workspace");
  float* scratch = nullptr;
  rc = dec::static_scratch(&scratch);
  if (rc) return rc;
  return decode_launch(p, scratch, stream);
}
