// The f32 conformance path (LTXB_MODE_F32): the reference `Block` computes in
// f32 with bf16 weights upcast (ltx/block.zig:22-26) and is gated at rel-RMS
// <= 1e-5 against f64, a bar bf16 tensor-core inputs cannot meet. These SIMT
// FFMA kernels keep every operand in f32: a tiled GEMM with the block's
// epilogues, and a blockwise online-softmax attention (whileSdpa,
// ltx/block.zig:105-154). They serve the 1k-token conformance config and
// full-size cross-checks of the tensor-core path; throughput is not their job.
#include <atomic>

#include "common.cuh"
#include "kernels.h"

namespace ltxb {

// ---------------------------------------------------------------------------
// GEMM: C[M, N] = A[M, K] . W[N, K]^T, A f32, W bf16 or int8 with grouped-128
// scales (dequantised as the reference's dq4 does, ltx/block.zig:462-471: the
// int8 value converted to f32 times its group's scale, one f32 multiply).
// Tile 128 x 128 x 16, 256 threads, 8 x 8 outputs per thread.
// ---------------------------------------------------------------------------
constexpr int FB_M = 128, FB_N = 128, FB_K = 16;

__device__ __forceinline__ float w_elem(const __nv_bfloat16* W, const int8_t* wq, const void* scales, int scale_bf16,
                                        int gn, int k, int K) {
  if (!wq) return __bfloat162float(W[(size_t)gn * K + k]);
  const size_t si = (size_t)gn * (K / 128) + (k >> 7);
  const float sc = scale_bf16 ? __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(scales)[si] << 16)
                              : reinterpret_cast<const float*>(scales)[si];
  return (float)wq[(size_t)gn * K + k] * sc;
}

__global__ void __launch_bounds__(256) gemm_f32_kernel(const float* __restrict__ A, int lda,
                                                       const __nv_bfloat16* __restrict__ W,
                                                       const int8_t* __restrict__ wq, const void* __restrict__ scales,
                                                       int scale_bf16, int M, int N, int K,
                                                       const __nv_bfloat16* __restrict__ bias, int epi,
                                                       float* __restrict__ out, int ldo, const float* __restrict__ xres,
                                                       const float* __restrict__ sst, const float* __restrict__ tstab,
                                                       const int* __restrict__ tidx, int tk, int ada_row) {
  __shared__ float sa[FB_K][FB_M + 4];
  __shared__ float sw[FB_K][FB_N + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * FB_M, n0 = blockIdx.x * FB_N;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  for (int k0 = 0; k0 < K; k0 += FB_K) {
    // 128 x 16 of A and W: 2048 elements each, 8 per thread
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int e = u * 256 + threadIdx.x;
      const int r = e >> 4, c = e & 15;
      const int gm = m0 + r, gn = n0 + r;
      sa[c][r] = (gm < M) ? A[(size_t)gm * lda + k0 + c] : 0.f;
      sw[c][r] = (gn < N) ? w_elem(W, wq, scales, scale_bf16, gn, k0 + c, K) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < FB_K; ++kk) {
      float a[8], b[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = sa[kk][ty * 4 + i];
        a[4 + i] = sa[kk][64 + ty * 4 + i];
        b[i] = sw[kk][tx * 4 + i];
        b[4 + i] = sw[kk][64 + tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int gm = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (gm >= M) continue;
    const int trow = epi == EPI_RESID_F32 ? table_row(tidx, gm, tk) : 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int gn = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (gn >= N) continue;
      float v = acc[i][j];
      if (bias) v += __bfloat162float(bias[gn]);
      if (epi == EPI_GELU_BF16) {
        // GELU tanh approximation in f32 (accurate tanhf for the f32 path)
        const float u = 0.7978845608028654f * (v + 0.044715f * v * v * v);
        v = 0.5f * v * (1.0f + tanhf(u));
      } else if (epi == EPI_GATE2SIG_F32) {
        v = 2.0f / (1.0f + expf(-v));
      } else if (epi == EPI_RESID_F32) {
        const float g = tstab[((size_t)trow * 9 + ada_row) * N + gn] + sst[(size_t)ada_row * N + gn];
        v = (xres ? xres[(size_t)gm * ldo + gn] : 0.f) + v * g;
      }
      out[(size_t)gm * ldo + gn] = v;
    }
  }
}

int gemm_f32(const float* A, int lda, const void* W, int M, int N, int K, const void* bias, int epi, float* out,
             int ldo, float* /*ssq*/, int /*ssq_ld*/, const float* xres, const float* sst, const float* tstab,
             const int* tidx, int tk, int ada_row, cudaStream_t st, const int8_t* wq, const void* scales,
             int scale_bf16) {
  if (M <= 0 || N <= 0) return LTXB_OK;
  if (K % FB_K) return set_error(LTXB_EINVAL, "gemm_f32: K %% 16");
  if (wq && (K % 128 || !scales)) return set_error(LTXB_EINVAL, "gemm_f32: int8 weights need K %% 128 and scales");
  if (!wq && !W) return set_error(LTXB_EINVAL, "gemm_f32: no weights");
  dim3 grid((N + FB_N - 1) / FB_N, (M + FB_M - 1) / FB_M);
  gemm_f32_kernel<<<grid, 256, 0, st>>>(A, lda, reinterpret_cast<const __nv_bfloat16*>(W), wq, scales, scale_bf16, M,
                                        N, K,
                                        reinterpret_cast<const __nv_bfloat16*>(bias), epi, out, ldo, xres, sst, tstab,
                                        tidx, tk, ada_row);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "gemm_f32");
}

// ---------------------------------------------------------------------------
// attention: CTA = 64 query rows x 1 head, K/V tiles of 64, online softmax.
// ---------------------------------------------------------------------------
constexpr int FA_Q = 64, FA_K = 64, FA_D = 128;

__global__ void __launch_bounds__(256) attention_f32_kernel(const float* __restrict__ q, int ldq,
                                                            const float* __restrict__ k, int ldk,
                                                            const float* __restrict__ v, int ldv,
                                                            float* __restrict__ out, const float* __restrict__ gate,
                                                            int ldg, int Tq, int Tkv, int H, float scale) {
  extern __shared__ float fsm[];
  float* sq = fsm;                      // [64][128]
  float* sk = sq + FA_Q * FA_D;         // [64][129] (padded)
  float* sv = sk + FA_K * (FA_D + 1);   // [64][128]
  float* sp = sv + FA_K * FA_D;         // [64][65]
  float* scorr = sp + FA_Q * (FA_K + 1);  // [64]
  float* sl = scorr + FA_Q;               // [64]
  const int h = blockIdx.y, q0 = blockIdx.x * FA_Q;
  const int tid = threadIdx.x;
  const size_t ld = (size_t)H * FA_D;

  for (int e = tid; e < FA_Q * FA_D; e += 256) {
    const int r = e >> 7, c = e & 127;
    sq[e] = (q0 + r < Tq) ? q[(size_t)(q0 + r) * ldq + h * FA_D + c] : 0.f;
  }
  // softmax ownership: 4 threads per row, 16 columns each
  const int srow = tid >> 2, sg = tid & 3;
  float m_run = -3.402823466e38f, l_run = 0.f;
  // O ownership: row = tid / 4, dims d = sg*4 + 16*kk + e
  float o[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) o[i] = 0.f;

  for (int k0 = 0; k0 < Tkv; k0 += FA_K) {
    __syncthreads();
    for (int e = tid; e < FA_K * FA_D; e += 256) {
      const int r = e >> 7, c = e & 127;
      const bool ok = k0 + r < Tkv;
      sk[r * (FA_D + 1) + c] = ok ? k[(size_t)(k0 + r) * ldk + h * FA_D + c] : 0.f;
      sv[e] = ok ? v[(size_t)(k0 + r) * ldv + h * FA_D + c] : 0.f;
    }
    __syncthreads();
    // S = q . k^T * scale: thread -> rows (tid/16)*4 .. +4, cols (tid%16)*4 .. +4
    {
      const int r0 = (tid >> 4) * 4, c0 = (tid & 15) * 4;
      float s[4][4] = {};
      for (int d = 0; d < FA_D; ++d) {
        float a[4], b[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          a[i] = sq[(r0 + i) * FA_D + d];
          b[i] = sk[(c0 + i) * (FA_D + 1) + d];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) s[i][j] = fmaf(a[i], b[j], s[i][j]);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          sp[(r0 + i) * (FA_K + 1) + c0 + j] = (k0 + c0 + j < Tkv) ? s[i][j] * scale : -INFINITY;
    }
    __syncthreads();
    {
      float mx = -INFINITY;
      for (int j = sg * 16; j < sg * 16 + 16; ++j) mx = fmaxf(mx, sp[srow * (FA_K + 1) + j]);
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run, mx);
      const float corr = expf(m_run - m_new);
      float sum = 0.f;
      for (int j = sg * 16; j < sg * 16 + 16; ++j) {
        const float p = expf(sp[srow * (FA_K + 1) + j] - m_new);
        sp[srow * (FA_K + 1) + j] = p;
        sum += p;
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      l_run = l_run * corr + sum;
      m_run = m_new;
      if (sg == 0) {
        scorr[srow] = corr;
        sl[srow] = l_run;
      }
    }
    __syncthreads();
    {
      const int r = tid >> 2;
      const float c = scorr[r];
#pragma unroll
      for (int i = 0; i < 32; ++i) o[i] *= c;
      for (int j = 0; j < FA_K; ++j) {
        const float p = sp[r * (FA_K + 1) + j];
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const float4 vv = *reinterpret_cast<const float4*>(sv + j * FA_D + kk * 16 + sg * 4);
          o[kk * 4 + 0] = fmaf(p, vv.x, o[kk * 4 + 0]);
          o[kk * 4 + 1] = fmaf(p, vv.y, o[kk * 4 + 1]);
          o[kk * 4 + 2] = fmaf(p, vv.z, o[kk * 4 + 2]);
          o[kk * 4 + 3] = fmaf(p, vv.w, o[kk * 4 + 3]);
        }
      }
    }
  }
  __syncthreads();
  const int r = tid >> 2;
  if (q0 + r < Tq) {
    const float inv = 1.0f / sl[r];
    const float g = gate ? gate[(size_t)(q0 + r) * ldg + h] : 1.0f;
    float* op = out + (q0 + r) * ld + h * FA_D;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
#pragma unroll
      for (int e = 0; e < 4; ++e) op[kk * 16 + sg * 4 + e] = o[kk * 4 + e] * inv * g;
  }
}

int attention_f32(const float* q, int ldq, const float* k, int ldk, const float* v, int ldv, float* out,
                  const float* gate, int ldg, int Tq, int Tkv, int H, float scale, cudaStream_t st) {
  if (Tq <= 0) return LTXB_OK;
  if (Tkv <= 0) return set_error(LTXB_EINVAL, "attention_f32: empty K/V");
  const size_t smem =
      sizeof(float) * (FA_Q * FA_D + FA_K * (FA_D + 1) + FA_K * FA_D + FA_Q * (FA_K + 1) + 2 * FA_Q);
  static std::atomic<bool> attr[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return set_error(LTXB_EINVAL, "attention_f32: device %d out of range", dev);
  if (!attr[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(attention_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_cuda_error(e, "attention_f32 attr");
    attr[dev].store(true, std::memory_order_release);
  }
  dim3 grid((Tq + FA_Q - 1) / FA_Q, H);
  attention_f32_kernel<<<grid, 256, smem, st>>>(q, ldq, k, ldk, v, ldv, out, gate, ldg, Tq, Tkv, H, scale);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "attention_f32");
}

}  // namespace ltxb
