// ltxb_dq_gemm_noalloc: the int8 grouped-128 linear for callers that cannot
// allocate device memory (their allocator owns the GPU, or they must not
// allocate while running). The bf16 expansion of the weights goes to a fixed
// scratch array compiled into the library instead of a caller workspace.
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace ltxb {

// Holds the bf16 expansion of one int8 weight matrix (N * K * 2 bytes).
// Part of the library image: every GPU that loads the library holds it until
// the process exits. Shared by all calls; each call overwrites what it reads.
static __device__ __align__(256) uint8_t g_noalloc_scratch[LTXB_NOALLOC_SCRATCH_BYTES];

// Device address of the scratch per device. A __device__ symbol named in host
// code is only a host-side stand-in, so the address is looked up once per
// device, with that device current.
static void* g_noalloc_ptr[64];
static std::mutex g_noalloc_mu;

static int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_cuda_error(e, "no-alloc scratch: cudaGetDevice");
  if (dev < 0 || dev >= 64) return set_error(LTXB_EINVAL, "no-alloc scratch: device %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) return set_cuda_error(e, "no-alloc scratch: cudaGetSymbolAddress");
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return LTXB_OK;
}

}  // namespace ltxb

using namespace ltxb;

extern "C" int ltxb_dq_gemm_noalloc(const void* A, const void* Wq, const void* scales, int scale_dtype,
                                    const void* bias, void* out, int M, int N, int K, void* stream) {
  if (scale_dtype != LTXB_DT_F32 && scale_dtype != LTXB_DT_BF16)
    return set_error(LTXB_EINVAL, "dq_gemm_noalloc: scale dtype must be LTXB_DT_F32 or LTXB_DT_BF16");
  if (M <= 0 || N <= 0 || K <= 0) return set_error(LTXB_EINVAL, "dq_gemm_noalloc: empty shape");
  if ((uint64_t)N * (uint64_t)K * 2u > (uint64_t)LTXB_NOALLOC_SCRATCH_BYTES)
    return set_error(LTXB_EINVAL,
                     "dq_gemm_noalloc: N * K = %llu weights need %llu scratch bytes; the built-in scratch holds %u "
                     "(N * K <= %u)",
                     (unsigned long long)N * K, (unsigned long long)N * K * 2, (unsigned)LTXB_NOALLOC_SCRATCH_BYTES,
                     (unsigned)(LTXB_NOALLOC_SCRATCH_BYTES / 2));
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  GemmArgs g{};
  g.A = A;
  g.lda = K;
  g.B = scratch;
  g.ldb = K;
  g.M = M;
  g.N = N;
  g.K = K;
  g.epi = EPI_BF16;
  g.bias = bias;
  g.out = out;
  g.ldo = N;
  // every argument check runs before the first launch: a rejected call
  // leaves the shared scratch untouched
  if ((rc = gemm_check(g, nullptr))) return rc;
  if ((reinterpret_cast<uintptr_t>(Wq) & 15) || (reinterpret_cast<uintptr_t>(scales) & (scale_dtype == LTXB_DT_BF16 ? 1 : 3)))
    return set_error(LTXB_EINVAL, "dq_gemm_noalloc: weights must be 16-byte aligned, scales element-aligned");
  rc = dequant_weights(static_cast<const int8_t*>(Wq), scales, scale_dtype == LTXB_DT_BF16, N, K, scratch, st);
  if (rc) return rc;
  return gemm_tc(g, st);
}
