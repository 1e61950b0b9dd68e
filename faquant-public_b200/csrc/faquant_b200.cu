// libfaquant_b200.so -- the single translation unit of the library.
//
// The kernels live in the component files included below; compiling them as one
// unit keeps the device status word (g_status) a single device symbol without
// relocatable device code. This file also holds the host-side glue of the C ABI
// declared in include/faquant_b200.h: error messages, device properties, TMA
// tensor-map encoding and the diagnostics entry points.
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "tma.h"

namespace faq {

static thread_local std::string t_last_error;

void set_error(const std::string& msg) { t_last_error = msg; }

int fail(int code, const std::string& msg) {
  set_error(msg);
  return code;
}

int cuda_fail(cudaError_t err, const char* what) {
  return fail(FAQ_ERR_CUDA, std::string(what) + ": " + cudaGetErrorName(err) + " (" + cudaGetErrorString(err) + ")");
}

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
              const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(FAQ_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], e[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    e[i] = 1;
    if (i + 1 < rank) {
      s[i] = strides_bytes[i];
      if (s[i] % 16 != 0) return fail(FAQ_ERR_ARG, "TMA strides must be multiples of 16 bytes");
    }
  }
  const CUresult r = fn(map, dtype, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, s, b, e,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FAQ_ERR_ARG, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(r));
  return FAQ_OK;
}

// Waits on an mbarrier that nothing arrives at; the bounded wait gives up after
// `limit_ns` and records FAQ_STATUS_TIMEOUT.
__global__ void selftest_wait_kernel(uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(smem_addr(&bar), 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(smem_addr(&bar), 0, limit_ns);
}

}  // namespace faq

#include "quantize.cu"
#include "gemm_sm100.cu"
#include "gemm_w4_small.cu"
#include "gemm_w4a4.cu"
#include "qk_prep.cu"
#include "attention_sm100.cu"
#include "glue.cu"
#include "decode.cu"
#include "gptq.cu"

extern "C" int faq_version(void) { return 100; }

extern "C" int faq_last_error(char* buf, size_t len) {
  if (buf == nullptr || len == 0) return FAQ_ERR_ARG;
  const std::string& m = faq::t_last_error;
  const size_t n = std::min(len - 1, m.size());
  std::memcpy(buf, m.data(), n);
  buf[n] = '\0';
  return FAQ_OK;
}

extern "C" int faq_device_status(unsigned int* status, int reset) {
  FAQ_CHECK_ARG(status != nullptr, "status is null");
  FAQ_CUDA(cudaMemcpyFromSymbol(status, faq::g_status, sizeof(unsigned int)));
  if (reset) {
    const unsigned int zero = 0;
    FAQ_CUDA(cudaMemcpyToSymbol(faq::g_status, &zero, sizeof(unsigned int)));
  }
  return FAQ_OK;
}

extern "C" int faq_device_trace(unsigned int* records, int max_records, int reset) {
  FAQ_CHECK_ARG(records != nullptr && max_records >= 0, "bad arguments");
  unsigned int count = 0;
  FAQ_CUDA(cudaMemcpyFromSymbol(&count, faq::g_trace_count, sizeof(count)));
  const int n = static_cast<int>(std::min<unsigned int>(count, std::min<unsigned int>(max_records, faq::kTraceSlots)));
  if (n > 0) FAQ_CUDA(cudaMemcpyFromSymbol(records, faq::g_trace, sizeof(unsigned int) * 3 * n));
  if (reset) {
    const unsigned int zero = 0;
    FAQ_CUDA(cudaMemcpyToSymbol(faq::g_trace_count, &zero, sizeof(zero)));
  }
  return static_cast<int>(count);
}

extern "C" int faq_selftest_wait_timeout(int64_t limit_ns, void* stream) {
  FAQ_CHECK_ARG(limit_ns > 0 && limit_ns <= 5000000000ll, "limit_ns must be in (0, 5 s]");
  faq::selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint64_t>(limit_ns));
  return faq::launch_status("selftest_wait_kernel");
}
