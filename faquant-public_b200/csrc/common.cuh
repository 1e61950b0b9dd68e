// Shared device helpers for the sm_100a kernels: error reporting, the device
// status word, bf16 bit helpers, bounded mbarrier waits and the PTX wrappers for
// TMA (cp.async.bulk.tensor) and the 5th-generation tensor cores (tcgen05).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/faquant_b200.h"

namespace faq {

// ---------------------------------------------------------------- host errors
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t err, const char* what);

#define FAQ_CHECK_ARG(cond, msg)                            \
  do {                                                      \
    if (!(cond)) return ::faq::fail(FAQ_ERR_ARG, (msg));    \
  } while (0)

#define FAQ_CUDA(call)                                      \
  do {                                                      \
    cudaError_t err_ = (call);                              \
    if (err_ != cudaSuccess) return ::faq::cuda_fail(err_, #call); \
  } while (0)

inline int launch_status(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return cuda_fail(err, what);
  return FAQ_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int num_sms();

// ---------------------------------------------------------------- status word
// One word per device, set when a bounded wait runs out. The library is a single
// translation unit (faquant_b200.cu includes every kernel file), so this header
// defines it exactly once.
__device__ unsigned int g_status = 0;

// Where waits gave up: up to kTraceSlots records of (site | tile << 8, block x | block y << 16, block z),
// read by faq_device_trace(). Written only on a timeout.
constexpr int kTraceSlots = 32;
__device__ unsigned int g_trace_count = 0;
__device__ unsigned int g_trace[kTraceSlots * 3];

__device__ __forceinline__ void report_timeout() { atomicOr(&g_status, FAQ_STATUS_TIMEOUT); }

__device__ __forceinline__ void trace_timeout(int site, int tile) {
  const unsigned int slot = atomicAdd(&g_trace_count, 1u);
  if (slot < kTraceSlots) {
    g_trace[slot * 3 + 0] = static_cast<unsigned int>(site) | (static_cast<unsigned int>(tile) << 8);
    g_trace[slot * 3 + 1] = blockIdx.x | (blockIdx.y << 16);
    g_trace[slot * 3 + 2] = blockIdx.z;
  }
}

// Default wait limit of the kernels' spin loops: 2 s of %globaltimer.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- bf16 bits
__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}
// fp32 value already exactly representable in bf16 -> its bf16 bits
__device__ __forceinline__ uint32_t exact_bf16_bits(float x) { return __float_as_uint(x) >> 16; }

// ---------------------------------------------------------------- activations (bf16 results)
// SwiGLU of Qwen3MLP: bf16(bf16(silu(g)) * u), silu(g) = g / (1 + exp(-g)) in fp32.
__device__ __forceinline__ float swiglu_bf16(float g, float u) {
  const float s = bf16_round(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))));
  return bf16_round(__fmul_rn(s, u));
}
// The DiT FFN's tanh GELU in fp32, rounded once: 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))).
__device__ __forceinline__ float gelu_tanh_bf16(float x) {
  const float beta = 0.7978845608028654f;  // sqrt(2 / pi)
  const float cube = __fmul_rn(__fmul_rn(x, x), x);
  const float inner = __fmul_rn(beta, __fadd_rn(x, __fmul_rn(0.044715f, cube)));
  return bf16_round(__fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner))));
}

__device__ __forceinline__ float pow2f(int e) {  // 2^e for -126 <= e <= 127
  return __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
}
__device__ __forceinline__ int exponent_of(float x) {  // floor(log2 x), x positive normal
  return static_cast<int>((__float_as_uint(x) >> 23) & 0xFF) - 127;
}

// ---------------------------------------------------------------- register-fragment MMA
// mma.sync m16n8k16, bf16 operands, fp32 accumulate in place: for products too small for a
// tcgen05 tile (decode rows, a few query rows per KV head).
__device__ __forceinline__ void mma_bf16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------- smem / mbarrier
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1; }" ::"r"(bar),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}
// try_wait that lets the hardware suspend the thread for up to `suspend_ns` while the
// phase is incomplete (it resumes when the phase completes): for warps that wait often and
// long, so that their polling does not take issue slots from the warps doing work.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint32_t bar, uint32_t parity, uint32_t suspend_ns) {
  uint32_t done;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
      : "=r"(done)
      : "r"(bar), "r"(parity), "r"(suspend_ns)
      : "memory");
  return done != 0;
}
// Warp-uniform bounded wait (as mbar_wait_warp) built on mbar_try_wait_suspend.
__device__ __forceinline__ bool mbar_wait_warp_suspend(uint32_t bar, uint32_t parity, uint32_t suspend_ns, int site,
                                                       int tile) {
  bool ok = mbar_try_wait_suspend(bar, parity, suspend_ns);
  if (!__all_sync(0xffffffffu, ok)) {
    const uint64_t start = globaltimer();
    while (!ok) {
      ok = mbar_try_wait_suspend(bar, parity, suspend_ns);
      if (!ok && globaltimer() - start > kWaitLimitNs) break;
    }
    if (!ok) report_timeout();
    ok = __all_sync(0xffffffffu, ok);
    if (!ok && (threadIdx.x & 31) == 0) trace_timeout(site, tile);
  }
  return ok;
}

// try_wait with acquire at cluster scope: for phases completed by arrivals from the other
// CTA of a pair (release.cluster), whose shared-memory writes the waiter then relies on.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster_site(uint32_t bar, uint32_t parity, int site, int tile) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t start = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait_cluster(bar, parity)) return true;
    if (globaltimer() - start > kWaitLimitNs) {
      report_timeout();
      trace_timeout(site, tile);
      return false;
    }
  }
}

// Wait for the phase of parity `parity` to complete, for at most `limit_ns`.
// Returns false (and records FAQ_STATUS_TIMEOUT) when the limit runs out.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity,
                                          uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - start > limit_ns) {
      report_timeout();
      return false;
    }
  }
}

// Bounded wait for a barrier that a whole warp waits on together. Every lane polls
// (bounded), then the lanes agree: the result is warp-uniform, so a timeout can
// never leave part of the warp inside a loop of .sync.aligned instructions.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, int site = 0, int tile = 0,
                                               uint64_t limit_ns = kWaitLimitNs) {
  const bool ok = __all_sync(0xffffffffu, mbar_wait(bar, parity, limit_ns));
  if (!ok && (threadIdx.x & 31) == 0) trace_timeout(site, tile);
  return ok;
}
// Single-lane variant that records the site on a timeout.
__device__ __forceinline__ bool mbar_wait_site(uint32_t bar, uint32_t parity, int site, int tile) {
  const bool ok = mbar_wait(bar, parity);
  if (!ok) trace_timeout(site, tile);
  return ok;
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, uint32_t bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* tmap, uint32_t bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
// Order this thread's generic-proxy shared-memory writes before later async-proxy
// (tensor core / TMA) reads of the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- programmatic dependent launch
// A kernel launched with the programmatic-stream-serialization attribute may start while
// the previous kernel of the stream is still running, once every CTA of that kernel has
// called allow_dependent_launch() (or exited). Before grid_dependency_wait() it may only
// touch memory the previous kernel neither writes nor reads; grid_dependency_wait()
// returns when the previous kernel has completed and its writes are visible (at once,
// for a kernel launched without the attribute).
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_dependent_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] . B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulate), one CTA.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] . B[smem]^T, kind::f16: A (M=128 rows in the TMEM lanes, 16-bit K
// values packed two per 32-bit column, even K in the low half) comes from tensor memory.
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p; }" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// ---------------------------------------------------------------- CTA pairs (cta_group::2)
// A cluster of two CTAs on the two SMs of a TPC: one tcgen05.mma.cta_group::2 issued by
// the pair's leader (rank 0) reads A rows 0..M/2-1 and B columns 0..N/2-1 from the
// leader's shared memory and the other halves from the peer's, at the same offsets, and
// writes D rows 0..M/2-1 to the leader's tensor memory and the rest to the peer's.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of this CTA's shared-memory location `saddr` in CTA `rank`
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// every thread of both CTAs; orders the mbarrier initializations before any remote use
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// arrive on an mbarrier of any CTA of the cluster (a shared::cluster address)
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Both CTAs of the pair allocate (the same warp index in each); the column address is the
// same in both.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem of both CTAs] (+)= A . B^T over the pair, kind::f16; issued by the leader only
__device__ __forceinline__ void tc_mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive, once the pair's previously issued MMAs complete, on the mbarrier at this
// shared-memory offset in every CTA of `cta_mask`.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar, uint16_t cta_mask) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::
                   "r"(bar), "h"(cta_mask)
               : "memory");
}
// TMA tile load into this CTA's shared memory whose bytes are counted on an mbarrier in
// either CTA of the pair (`bar_cluster`, a shared::cluster address): the leader's barrier
// counts both CTAs' operand tiles. Not a multicast load.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void* tmap, uint32_t bar_cluster, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bit, 32 consecutive columns: thread i of the warp reads TMEM lane
// (warp quarter * 32 + i), columns [col, col + 32). The load is asynchronous: the
// registers are valid only after tc_wait_ld() followed by reg_fence32() on them.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// The same load into floats (f[0..31] of the caller's array).
__device__ __forceinline__ void tmem_ld32f(uint32_t taddr, float* f) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=f"(f[0]), "=f"(f[1]), "=f"(f[2]), "=f"(f[3]), "=f"(f[4]), "=f"(f[5]), "=f"(f[6]), "=f"(f[7]), "=f"(f[8]),
        "=f"(f[9]), "=f"(f[10]), "=f"(f[11]), "=f"(f[12]), "=f"(f[13]), "=f"(f[14]), "=f"(f[15]), "=f"(f[16]),
        "=f"(f[17]), "=f"(f[18]), "=f"(f[19]), "=f"(f[20]), "=f"(f[21]), "=f"(f[22]), "=f"(f[23]), "=f"(f[24]),
        "=f"(f[25]), "=f"(f[26]), "=f"(f[27]), "=f"(f[28]), "=f"(f[29]), "=f"(f[30]), "=f"(f[31])
      : "r"(taddr));
}
__device__ __forceinline__ void reg_fence32f(float* f) {
  asm volatile("" : "+f"(f[0]), "+f"(f[1]), "+f"(f[2]), "+f"(f[3]), "+f"(f[4]), "+f"(f[5]), "+f"(f[6]), "+f"(f[7]),
               "+f"(f[8]), "+f"(f[9]), "+f"(f[10]), "+f"(f[11]), "+f"(f[12]), "+f"(f[13]), "+f"(f[14]), "+f"(f[15]),
               "+f"(f[16]), "+f"(f[17]), "+f"(f[18]), "+f"(f[19]), "+f"(f[20]), "+f"(f[21]), "+f"(f[22]),
               "+f"(f[23]), "+f"(f[24]), "+f"(f[25]), "+f"(f[26]), "+f"(f[27]), "+f"(f[28]), "+f"(f[29]),
               "+f"(f[30]), "+f"(f[31]));
}
__device__ __forceinline__ void tmem_st32f(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]),
      "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]), "f"(v[18]),
      "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]),
      "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
}
// Orders every later use of r after the preceding tc_wait_ld(): both are volatile
// asm statements, so the compiler keeps them in program order, and the "+r"
// operands make the uses depend on this one.
__device__ __forceinline__ void reg_fence32(uint32_t (&r)[32]) {
  asm volatile("" : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31]));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile stored in the
// 128-byte swizzled layout TMA writes (rows of 128 B, 8-row atoms of 1024 B).
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);  // start address
  d |= static_cast<uint64_t>(1) << 16;                  // leading byte offset (unused for SW128 K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;          // stride byte offset: next 8-row atom
  d |= static_cast<uint64_t>(1) << 46;                  // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                  // SWIZZLE_128B
  return d;
}
// Same layout seen as an MN-major operand (e.g. V as the B operand of P.V): the
// contiguous 128-byte rows run along N; `lbo` is the byte distance between
// 64-element column chunks along N, 1024 B between 8-row groups along K.
__device__ __forceinline__ uint64_t sw128_mnmajor_desc(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}
// The upper 32 bits of every 128-byte-swizzled descriptor above (stride byte offset
// 1024, version, layout); the lower 32 bits hold the start address and the leading
// byte offset.
constexpr uint32_t SW128_DESC_HI = (1024u >> 4) | (1u << (46 - 32)) | (2u << (61 - 32));
__device__ __forceinline__ uint32_t sw128_desc_lo(uint32_t saddr, uint32_t lbo) {
  return ((saddr >> 4) & 0x3FFFu) | (((lbo >> 4) & 0x3FFFu) << 16);
}
// tcgen05.mma forms taking the low descriptor words only (the upper words are
// SW128_DESC_HI): fewer registers for an issuer that keeps many descriptors live.
__device__ __forceinline__ void tc_mma_f16_lo(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; .reg .b64 ad, bd; setp.ne.b32 p, %4, 0;\n"
      "mov.b64 ad, {%1, %5}; mov.b64 bd, {%2, %5};\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %3, p; }" ::"r"(d_tmem),
      "r"(a_lo), "r"(b_lo), "r"(idesc), "r"(accumulate), "n"(SW128_DESC_HI)
      : "memory");
}
// tcgen05.mma.cta_group::2 form taking the low descriptor words (see tc_mma_f16_lo)
__device__ __forceinline__ void tc_mma_f16_pair_lo(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo, uint32_t idesc,
                                                   uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; .reg .b64 ad, bd; setp.ne.b32 p, %4, 0;\n"
      "mov.b64 ad, {%1, %5}; mov.b64 bd, {%2, %5};\n"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], ad, bd, %3, p; }" ::"r"(d_tmem),
      "r"(a_lo), "r"(b_lo), "r"(idesc), "r"(accumulate), "n"(SW128_DESC_HI)
      : "memory");
}
__device__ __forceinline__ void tc_mma_f16_ts_lo(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; .reg .b64 bd; setp.ne.b32 p, %4, 0;\n"
      "mov.b64 bd, {%2, %5};\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], bd, %3, p; }" ::"r"(d_tmem),
      "r"(a_tmem), "r"(b_lo), "r"(idesc), "r"(accumulate), "n"(SW128_DESC_HI)
      : "memory");
}
// Instruction descriptor: kind::f16 with bf16 A/B, fp32 D, dense.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                                  // D format: F32
         | (1u << 7)                                // A format: BF16
         | (1u << 10)                               // B format: BF16
         | (static_cast<uint32_t>(a_mn_major) << 15)  // A major
         | (static_cast<uint32_t>(b_mn_major) << 16)  // B major
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

__device__ __forceinline__ bool elect_one_sync() {
  uint32_t pred = 0;
  asm volatile(
      "{ .reg .b32 r; .reg .pred p; elect.sync r|p, 0xffffffff; selp.u32 %0, 1, 0, p; }"
      : "=r"(pred));
  return pred != 0;
}

}  // namespace faq
