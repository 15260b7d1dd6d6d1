// Device-side structural statistics of an f32 tensor: the reference's
// statsOf (ltx/core_parts.zig:183-193), which lets a host check a
// production-length output with a 12-byte readback instead of the whole
// tensor (ltx/e2e_prod.zig:444-468).
//
//   out[0] = number of NaN values (v != v, as the reference counts them)
//   out[1] = sum of v^2 (accumulated in f64, rounded once to f32)
//   out[2] = max |v| over the non-NaN values
//
// Two launches with a fixed grid and a fixed reduction order, so the result
// is the same on every run: each of STATS_BLOCKS CTAs reduces a grid-strided
// share into its own slot of the caller's workspace, then one CTA folds the
// slots in index order.
#include "common.cuh"
#include "kernels.h"

namespace ltxb {

constexpr int STATS_BLOCKS = 2 * 148;
constexpr int STATS_THREADS = 512;

struct StatsPart {
  double ss;
  float nan;
  float maxa;
};

__device__ __forceinline__ void stats_reduce(double& ss, float& nan, float& maxa) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
    nan += __shfl_xor_sync(0xffffffffu, nan, o);
    maxa = fmaxf(maxa, __shfl_xor_sync(0xffffffffu, maxa, o));
  }
  __shared__ double s_ss[32];
  __shared__ float s_nan[32], s_max[32];
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) {
    s_ss[w] = ss;
    s_nan[w] = nan;
    s_max[w] = maxa;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    ss = 0.0;
    nan = 0.f;
    maxa = 0.f;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) {
      ss += s_ss[i];
      nan += s_nan[i];
      maxa = fmaxf(maxa, s_max[i]);
    }
  }
}

__global__ void __launch_bounds__(STATS_THREADS) stats_partial_kernel(const float* __restrict__ v, uint64_t n,
                                                                      StatsPart* __restrict__ part) {
  double ss = 0.0;
  float nan = 0.f, maxa = 0.f;
  const uint64_t n4 = ((reinterpret_cast<uintptr_t>(v) & 15) == 0) ? n / 4 : 0;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  auto one = [&](float x) {
    if (x != x) {
      nan += 1.f;
    } else {
      ss = fma((double)x, (double)x, ss);
      maxa = fmaxf(maxa, fabsf(x));
    }
  };
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 q = __ldg(reinterpret_cast<const float4*>(v) + i);
    one(q.x);
    one(q.y);
    one(q.z);
    one(q.w);
  }
  for (uint64_t i = n4 * 4 + blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += stride) one(__ldg(v + i));
  stats_reduce(ss, nan, maxa);
  if (threadIdx.x == 0) part[blockIdx.x] = StatsPart{ss, nan, maxa};
}

__global__ void stats_final_kernel(const StatsPart* __restrict__ part, int nparts, float* __restrict__ out) {
  if (threadIdx.x != 0) return;
  double ss = 0.0, nan = 0.0;
  float maxa = 0.f;
  for (int i = 0; i < nparts; ++i) {
    ss += part[i].ss;
    nan += part[i].nan;
    maxa = fmaxf(maxa, part[i].maxa);
  }
  out[0] = (float)nan;
  out[1] = (float)ss;
  out[2] = maxa;
}

}  // namespace ltxb

using namespace ltxb;

extern "C" {

uint64_t ltxb_stats_workspace_bytes(void) { return (uint64_t)STATS_BLOCKS * sizeof(StatsPart); }

int ltxb_stats(const float* v, uint64_t n, float* out, void* workspace, uint64_t workspace_bytes, void* stream) {
  if (!out) return set_error(LTXB_EINVAL, "stats: out is null");
  if (n > 0 && !v) return set_error(LTXB_EINVAL, "stats: v is null");
  if (!workspace || workspace_bytes < ltxb_stats_workspace_bytes())
    return set_error(LTXB_EINVAL, "stats: workspace of %llu bytes is smaller than the %llu required",
                     (unsigned long long)workspace_bytes, (unsigned long long)ltxb_stats_workspace_bytes());
  if ((reinterpret_cast<uintptr_t>(workspace) & 15) || (reinterpret_cast<uintptr_t>(v) & 3) ||
      (reinterpret_cast<uintptr_t>(out) & 3))
    return set_error(LTXB_EINVAL, "stats: workspace must be 16-byte aligned, v and out 4-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  StatsPart* part = static_cast<StatsPart*>(workspace);
  stats_partial_kernel<<<STATS_BLOCKS, STATS_THREADS, 0, st>>>(v, n, part);
  launched();
  stats_final_kernel<<<1, 32, 0, st>>>(part, STATS_BLOCKS, out);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "stats");
}

}  // extern "C"
