// Bandwidth-bound kernels of the block: RMSNorm + AdaLN modulation, q/k norm
// with split-half RoPE, prompt K/V modulation, weight dequantisation, casts.
//
// Reference ops (ltx/block.zig): rmsNoW/rmsW :28-34, modulate :36-38,
// adaVal :47-67, rope :71-77 (view at :221-226), caOut's K/V modulation
// :298-301, dq4 :462-471.
//
// One CTA per token row for the row-wise kernels: a [D] f32 row is 16 KB at
// D = 4096, read once with 16-byte loads, reduced in registers + one
// shared-memory pass, written once.
#include "common.cuh"
#include "kernels.h"

namespace ltxb {

constexpr float kEps = 1e-6f;
constexpr int ROW_THREADS = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  const int nw = blockDim.x >> 5;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}

// ada value for (token row t, table row r, column c): tstab[tidx[t], r, c] + sst[r, c]
// (ltx/block.zig:47-67: the gathered per-token row plus the per-block row)
__device__ __forceinline__ float4 ada4(const float* sst, const float* tstab, int trow, int r, int D, int c) {
  const float4 tv = __ldg(reinterpret_cast<const float4*>(tstab + ((size_t)trow * 9 + r) * D + c));
  const float4 sv = __ldg(reinterpret_cast<const float4*>(sst + (size_t)r * D + c));
  return make_float4(tv.x + sv.x, tv.y + sv.y, tv.z + sv.z, tv.w + sv.w);
}

// n = x * rsqrt(mean(x^2) + eps); out = n * (1 + ada(r_scale)) + ada(r_shift)
__global__ void __launch_bounds__(ROW_THREADS) norm_modulate_kernel(const float* __restrict__ x, int D,
                                                                    const float* __restrict__ sst,
                                                                    const float* __restrict__ tstab,
                                                                    const int* __restrict__ tidx, int tk, int r_shift,
                                                                    int r_scale, void* __restrict__ out, int out_f32,
                                                                    float* __restrict__ rms_copy) {
  __shared__ float red[32];
  const int t = blockIdx.x;
  const float* xr = x + (size_t)t * D;
  const int nv = D / 4;  // float4 per row
  float ss = 0.f;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    float4 v = reinterpret_cast<const float4*>(xr)[i];
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
  }
  ss = block_sum(ss, red);
  const float r = rsqrtf(ss / (float)D + kEps);
  const int trow = table_row(tidx, t, tk);
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    const int c = i * 4;
    float4 v = reinterpret_cast<const float4*>(xr)[i];
    float4 n = make_float4(v.x * r, v.y * r, v.z * r, v.w * r);
    if (rms_copy) reinterpret_cast<float4*>(rms_copy + (size_t)t * D)[i] = n;
    if (r_shift < 0) {
      if (out_f32)
        reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (size_t)t * D)[i] = n;
      else
        reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(out) + (size_t)t * D)[i] =
            make_uint2(pack_bf16x2(n.x, n.y), pack_bf16x2(n.z, n.w));
      continue;
    }
    const float4 sc = ada4(sst, tstab, trow, r_scale, D, c);
    const float4 sh = ada4(sst, tstab, trow, r_shift, D, c);
    float4 o;
    o.x = n.x * (sc.x + 1.0f) + sh.x;
    o.y = n.y * (sc.y + 1.0f) + sh.y;
    o.z = n.z * (sc.z + 1.0f) + sh.z;
    o.w = n.w * (sc.w + 1.0f) + sh.w;
    if (out_f32)
      reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (size_t)t * D)[i] = o;
    else
      reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(out) + (size_t)t * D)[i] =
          make_uint2(pack_bf16x2(o.x, o.y), pack_bf16x2(o.z, o.w));
  }
}

// The same function with the row held in registers: V float4 per thread
// (D <= V * 4 * ROW_THREADS), so x is read from HBM once, the sum of squares
// needs one barrier, and at <= 32 registers a thread eight rows are in flight
// per SM (the two-pass kernel above is register-limited to four and reads
// each row twice).
template <int V>
__global__ void __launch_bounds__(ROW_THREADS, 8) norm_modulate_reg_kernel(
    const float* __restrict__ x, int D, const float* __restrict__ sst, const float* __restrict__ tstab,
    const int* __restrict__ tidx, int tk, int r_shift, int r_scale, void* __restrict__ out, int out_f32) {
  __shared__ float red[ROW_THREADS / 32];
  const int t = blockIdx.x;
  const int nv = D >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)t * D);
  float4 v[V];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int i = threadIdx.x + j * ROW_THREADS;
    v[j] = i < nv ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int j = 0; j < V; ++j) {
    ss = fmaf(v[j].x, v[j].x, ss);
    ss = fmaf(v[j].y, v[j].y, ss);
    ss = fmaf(v[j].z, v[j].z, ss);
    ss = fmaf(v[j].w, v[j].w, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  ss = 0.f;
#pragma unroll
  for (int i = 0; i < ROW_THREADS / 32; ++i) ss += red[i];
  const float r = rsqrtf(ss / (float)D + kEps);
  const int trow = table_row(tidx, t, tk);
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int i = threadIdx.x + j * ROW_THREADS;
    if (i >= nv) break;
    const int c = i * 4;
    const float4 sc = ada4(sst, tstab, trow, r_scale, D, c);
    const float4 sh = ada4(sst, tstab, trow, r_shift, D, c);
    float4 o;
    o.x = v[j].x * r * (sc.x + 1.0f) + sh.x;
    o.y = v[j].y * r * (sc.y + 1.0f) + sh.y;
    o.z = v[j].z * r * (sc.z + 1.0f) + sh.z;
    o.w = v[j].w * r * (sc.w + 1.0f) + sh.w;
    if (out_f32)
      reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (size_t)t * D)[i] = o;
    else
      reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(out) + (size_t)t * D)[i] =
          make_uint2(pack_bf16x2(o.x, o.y), pack_bf16x2(o.z, o.w));
  }
}

// The modulation rows of up to three norm-modulate calls, combined once per
// block call: tab[n][k][0] = (sst[scale_n] + tstab[k, scale_n]) + 1 and
// tab[n][k][1] = sst[shift_n] + tstab[k, shift_n], the same f32 operations
// norm_modulate does per element, so results are bit-identical.
struct ModRows {
  int shift[3], scale[3];
};
__global__ void mod_tables_kernel(const float* __restrict__ sst, const float* __restrict__ tstab, int tk, int D,
                                  ModRows rows, int n, float* __restrict__ tab) {
  const size_t total = (size_t)n * tk * D;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % D);
    const int k = (int)((i / D) % tk);
    const int m = (int)(i / ((size_t)tk * D));
    const int rs = rows.scale[m], rh = rows.shift[m];
    float* o = tab + (((size_t)m * tk + k) * 2) * D + c;
    o[0] = (tstab[((size_t)k * 9 + rs) * D + c] + sst[(size_t)rs * D + c]) + 1.0f;
    o[D] = tstab[((size_t)k * 9 + rh) * D + c] + sst[(size_t)rh * D + c];
  }
}

int mod_tables(const float* sst, const float* tstab, int tk, int D, const int* shifts, const int* scales, int n,
               float* tab, cudaStream_t st) {
  if (n < 1 || n > 3 || tk < 1) return set_error(LTXB_EINVAL, "mod_tables: 1..3 tables, tk >= 1");
  ModRows r{};
  for (int i = 0; i < n; ++i) {
    r.shift[i] = shifts[i];
    r.scale[i] = scales[i];
  }
  const size_t total = (size_t)n * tk * D;
  int grid = (int)((total + 255) / 256);
  if (grid > 4 * sm_count()) grid = 4 * sm_count();
  mod_tables_kernel<<<grid, 256, 0, st>>>(sst, tstab, tk, D, r, n, tab);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_error(LTXB_ECUDA, "mod_tables: %s", cudaGetErrorString(e));
}

// norm_modulate_reg_kernel with the modulation rows read from a combined
// table (two loads per four columns instead of four).
template <int V>
__global__ void __launch_bounds__(ROW_THREADS, 8) norm_modulate_tab_kernel(
    const float* __restrict__ x, int D, const float* __restrict__ tab, const int* __restrict__ tidx, int tk,
    void* __restrict__ out, int out_f32) {
  __shared__ float red[ROW_THREADS / 32];
  const int t = blockIdx.x;
  const int nv = D >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)t * D);
  float4 v[V];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int i = threadIdx.x + j * ROW_THREADS;
    v[j] = i < nv ? xr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int j = 0; j < V; ++j) {
    ss = fmaf(v[j].x, v[j].x, ss);
    ss = fmaf(v[j].y, v[j].y, ss);
    ss = fmaf(v[j].z, v[j].z, ss);
    ss = fmaf(v[j].w, v[j].w, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  ss = 0.f;
#pragma unroll
  for (int i = 0; i < ROW_THREADS / 32; ++i) ss += red[i];
  const float r = rsqrtf(ss / (float)D + kEps);
  const int trow = table_row(tidx, t, tk);
  const float4* sc4 = reinterpret_cast<const float4*>(tab + (size_t)trow * 2 * D);
  const float4* sh4 = sc4 + nv;
#pragma unroll
  for (int j = 0; j < V; ++j) {
    const int i = threadIdx.x + j * ROW_THREADS;
    if (i >= nv) break;
    const float4 sc = __ldg(sc4 + i), sh = __ldg(sh4 + i);
    float4 o;
    o.x = v[j].x * r * sc.x + sh.x;
    o.y = v[j].y * r * sc.y + sh.y;
    o.z = v[j].z * r * sc.z + sh.z;
    o.w = v[j].w * r * sc.w + sh.w;
    if (out_f32)
      reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (size_t)t * D)[i] = o;
    else
      reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(out) + (size_t)t * D)[i] =
          make_uint2(pack_bf16x2(o.x, o.y), pack_bf16x2(o.z, o.w));
  }
}

int norm_modulate_tab(const float* x, int T, int D, const float* tab, const int* tidx, int tk, void* out, int out_f32,
                      cudaStream_t st) {
  if (T <= 0) return LTXB_OK;
  const int v = (D / 4 + ROW_THREADS - 1) / ROW_THREADS;
  if (D % 4 || v > 4) return set_error(LTXB_EINVAL, "norm_modulate_tab: D must be a multiple of 4, at most 4096");
  switch (v) {
    case 1: norm_modulate_tab_kernel<1><<<T, ROW_THREADS, 0, st>>>(x, D, tab, tidx, tk, out, out_f32); break;
    case 2: norm_modulate_tab_kernel<2><<<T, ROW_THREADS, 0, st>>>(x, D, tab, tidx, tk, out, out_f32); break;
    case 3: norm_modulate_tab_kernel<3><<<T, ROW_THREADS, 0, st>>>(x, D, tab, tidx, tk, out, out_f32); break;
    default: norm_modulate_tab_kernel<4><<<T, ROW_THREADS, 0, st>>>(x, D, tab, tidx, tk, out, out_f32); break;
  }
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "norm_modulate_tab");
}

int norm_modulate(const float* x, int T, int D, const float* sst, const float* tstab, const int* tidx, int tk, int r_shift,
                  int r_scale, void* out, int out_f32, float* rms_copy, cudaStream_t st) {
  if (T <= 0) return LTXB_OK;
  if (D % 4) return set_error(LTXB_EINVAL, "norm_modulate: D %% 4");
  const int v = (D / 4 + ROW_THREADS - 1) / ROW_THREADS;
  if (!rms_copy && r_shift >= 0 && v <= 4) {
    switch (v) {
      case 1: norm_modulate_reg_kernel<1><<<T, ROW_THREADS, 0, st>>>(x, D, sst, tstab, tidx, tk, r_shift, r_scale, out, out_f32); break;
      case 2: norm_modulate_reg_kernel<2><<<T, ROW_THREADS, 0, st>>>(x, D, sst, tstab, tidx, tk, r_shift, r_scale, out, out_f32); break;
      case 3: norm_modulate_reg_kernel<3><<<T, ROW_THREADS, 0, st>>>(x, D, sst, tstab, tidx, tk, r_shift, r_scale, out, out_f32); break;
      default: norm_modulate_reg_kernel<4><<<T, ROW_THREADS, 0, st>>>(x, D, sst, tstab, tidx, tk, r_shift, r_scale, out, out_f32); break;
    }
    launched();
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "norm_modulate");
  }
  norm_modulate_kernel<<<T, ROW_THREADS, 0, st>>>(x, D, sst, tstab, tidx, tk, r_shift, r_scale, out, out_f32, rms_copy);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "norm_modulate");
}

int rms_rows(const float* x, int T, int D, float* out, cudaStream_t st) {
  return norm_modulate(x, T, D, nullptr, nullptr, nullptr, 0, -1, -1, out, 1, nullptr, st);
}

// q/k norm over the full D from bf16 raw projections and per-N-tile sums of
// squares computed by the GEMM epilogue, then split-half RoPE per head:
//   y = raw * rsqrt(sum(ssq[t, :]) / D + eps) * w
//   (a, b) = (y[h*128 + i], y[h*128 + 64 + i]) -> (a c - b s, b c + a s)
// Thread layout: 8 threads per head, each owning 8 consecutive pair indices.
// Up to two tensors (q and k) share one pass over the cos/sin tables.
struct QkSide {
  const __nv_bfloat16* raw;
  int ld_raw;
  const float* ssq;  // [T, ssq_ld], n_ssq partials; null -> compute from raw
  int ssq_ld;
  const __nv_bfloat16* w;
  __nv_bfloat16* out_bf16;
  float* out_f32;
};

__device__ __forceinline__ void unpack8(uint4 u, float* f) {
  f[0] = bf16_lo(u.x); f[1] = bf16_hi(u.x); f[2] = bf16_lo(u.y); f[3] = bf16_hi(u.y);
  f[4] = bf16_lo(u.z); f[5] = bf16_hi(u.z); f[6] = bf16_lo(u.w); f[7] = bf16_hi(u.w);
}

__device__ __forceinline__ void qk_side_row(const QkSide& s, int n_ssq, const float* cos, const float* sin, int t,
                                            int D, float* red) {
  const int H = D / 128;
  const __nv_bfloat16* raw = s.raw + (size_t)t * s.ld_raw;
  float ss;
  if (s.ssq) {
    ss = 0.f;
    for (int i = 0; i < n_ssq; ++i) ss += s.ssq[(size_t)t * s.ssq_ld + i];
  } else {
    float p = 0.f;
    for (int c = threadIdx.x * 8; c < D; c += blockDim.x * 8) {
      float f[8];
      unpack8(*reinterpret_cast<const uint4*>(raw + c), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) p = fmaf(f[j], f[j], p);
    }
    ss = block_sum(p, red);
  }
  const float r = rsqrtf(ss / (float)D + kEps);
  for (int u = threadIdx.x; u < H * 8; u += blockDim.x) {
    const int h = u >> 3, i0 = (u & 7) * 8;
    const int ca = h * 128 + i0, cb = ca + 64;
    float a[8], b[8], wa[8], wb[8];
    unpack8(*reinterpret_cast<const uint4*>(raw + ca), a);
    unpack8(*reinterpret_cast<const uint4*>(raw + cb), b);
    unpack8(__ldg(reinterpret_cast<const uint4*>(s.w + ca)), wa);
    unpack8(__ldg(reinterpret_cast<const uint4*>(s.w + cb)), wb);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      a[j] = a[j] * r * wa[j];
      b[j] = b[j] * r * wb[j];
    }
    if (cos) {
      const float* cp = cos + ((size_t)t * H + h) * 64 + i0;
      const float* sp = sin + ((size_t)t * H + h) * 64 + i0;
      float c8[8], s8[8];
      *reinterpret_cast<float4*>(c8) = __ldg(reinterpret_cast<const float4*>(cp));
      *reinterpret_cast<float4*>(c8 + 4) = __ldg(reinterpret_cast<const float4*>(cp + 4));
      *reinterpret_cast<float4*>(s8) = __ldg(reinterpret_cast<const float4*>(sp));
      *reinterpret_cast<float4*>(s8 + 4) = __ldg(reinterpret_cast<const float4*>(sp + 4));
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float ra = a[j] * c8[j] - b[j] * s8[j];
        const float rb = b[j] * c8[j] + a[j] * s8[j];
        a[j] = ra;
        b[j] = rb;
      }
    }
    if (s.out_bf16) {
      __nv_bfloat16* o = s.out_bf16 + (size_t)t * D;
      *reinterpret_cast<uint4*>(o + ca) =
          make_uint4(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]), pack_bf16x2(a[4], a[5]), pack_bf16x2(a[6], a[7]));
      *reinterpret_cast<uint4*>(o + cb) =
          make_uint4(pack_bf16x2(b[0], b[1]), pack_bf16x2(b[2], b[3]), pack_bf16x2(b[4], b[5]), pack_bf16x2(b[6], b[7]));
    }
    if (s.out_f32) {
      float* o = s.out_f32 + (size_t)t * D;
      *reinterpret_cast<float4*>(o + ca) = make_float4(a[0], a[1], a[2], a[3]);
      *reinterpret_cast<float4*>(o + ca + 4) = make_float4(a[4], a[5], a[6], a[7]);
      *reinterpret_cast<float4*>(o + cb) = make_float4(b[0], b[1], b[2], b[3]);
      *reinterpret_cast<float4*>(o + cb + 4) = make_float4(b[4], b[5], b[6], b[7]);
    }
  }
}

__global__ void __launch_bounds__(ROW_THREADS) qk_norm_rope_kernel(QkSide s0, QkSide s1, int nsides, int n_ssq,
                                                                   const float* __restrict__ cos,
                                                                   const float* __restrict__ sin, int D) {
  __shared__ float red[32];
  const int t = blockIdx.x;
  qk_side_row(s0, n_ssq, cos, sin, t, D, red);
  if (nsides > 1) qk_side_row(s1, n_ssq, cos, sin, t, D, red);
}

int qk_norm_rope(const void* raw, int ld_raw, const float* ssq, int ssq_ld, int n_ssq, const void* w_bf16,
                 const float* cos, const float* sin, int T, int D, void* out_bf16, float* out_f32, cudaStream_t st) {
  if (T <= 0) return LTXB_OK;
  QkSide s{reinterpret_cast<const __nv_bfloat16*>(raw), ld_raw, ssq, ssq_ld,
           reinterpret_cast<const __nv_bfloat16*>(w_bf16), reinterpret_cast<__nv_bfloat16*>(out_bf16), out_f32};
  qk_norm_rope_kernel<<<T, ROW_THREADS, 0, st>>>(s, s, 1, n_ssq, cos, sin, D);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "qk_norm_rope");
}

// q and k of self-attention in one pass (shared cos/sin reads).
int qk_norm_rope2(const void* raw_q, const void* raw_k, int ld_raw, const float* ssq_q, const float* ssq_k,
                  int ssq_ld, int n_ssq, const void* wq, const void* wk, const float* cos, const float* sin, int T,
                  int D, void* out_q, void* out_k, cudaStream_t st) {
  if (T <= 0) return LTXB_OK;
  QkSide a{reinterpret_cast<const __nv_bfloat16*>(raw_q), ld_raw, ssq_q, ssq_ld,
           reinterpret_cast<const __nv_bfloat16*>(wq), reinterpret_cast<__nv_bfloat16*>(out_q), nullptr};
  QkSide b{reinterpret_cast<const __nv_bfloat16*>(raw_k), ld_raw, ssq_k, ssq_ld,
           reinterpret_cast<const __nv_bfloat16*>(wk), reinterpret_cast<__nv_bfloat16*>(out_k), nullptr};
  qk_norm_rope_kernel<<<T, ROW_THREADS, 0, st>>>(a, b, 2, n_ssq, cos, sin, D);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "qk_norm_rope2");
}

// ---- f32 variant: raw projections in f32, weights bf16, sum of squares in-kernel
__global__ void __launch_bounds__(ROW_THREADS) qk_norm_rope_f32_kernel(const float* __restrict__ raw, int ld_raw,
                                                                       const __nv_bfloat16* __restrict__ w,
                                                                       const float* __restrict__ cos,
                                                                       const float* __restrict__ sin, int D,
                                                                       float* __restrict__ out,
                                                                       __nv_bfloat16* __restrict__ out_bf16) {
  __shared__ float red[32];
  const int t = blockIdx.x, H = D / 128;
  const float* rr = raw + (size_t)t * ld_raw;
  float p = 0.f;
  for (int c = threadIdx.x * 4; c < D; c += blockDim.x * 4) {
    float4 v = *reinterpret_cast<const float4*>(rr + c);
    p = fmaf(v.x, v.x, p);
    p = fmaf(v.y, v.y, p);
    p = fmaf(v.z, v.z, p);
    p = fmaf(v.w, v.w, p);
  }
  const float ss = block_sum(p, red);
  const float r = rsqrtf(ss / (float)D + kEps);
  for (int u = threadIdx.x; u < H * 64; u += blockDim.x) {
    const int h = u >> 6, i = u & 63;
    const int ca = h * 128 + i, cb = ca + 64;
    float a = rr[ca] * r * __bfloat162float(w[ca]);
    float b = rr[cb] * r * __bfloat162float(w[cb]);
    if (cos) {
      const float c = cos[((size_t)t * H + h) * 64 + i], s = sin[((size_t)t * H + h) * 64 + i];
      const float ra = a * c - b * s, rb = b * c + a * s;
      a = ra;
      b = rb;
    }
    if (out) {
      out[(size_t)t * D + ca] = a;
      out[(size_t)t * D + cb] = b;
    } else {
      out_bf16[(size_t)t * D + ca] = __float2bfloat16_rn(a);
      out_bf16[(size_t)t * D + cb] = __float2bfloat16_rn(b);
    }
  }
}

int qk_norm_rope_f32(const float* raw, int ld_raw, const void* w_bf16, const float* cos, const float* sin, int T,
                     int D, float* out, cudaStream_t st, void* out_bf16) {
  if (T <= 0) return LTXB_OK;
  if (!out && !out_bf16) return set_error(LTXB_EINVAL, "qk_norm_rope_f32: no output");
  qk_norm_rope_f32_kernel<<<T, ROW_THREADS, 0, st>>>(raw, ld_raw, reinterpret_cast<const __nv_bfloat16*>(w_bf16),
                                                     cos, sin, D, out, reinterpret_cast<__nv_bfloat16*>(out_bf16));
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "qk_norm_rope_f32");
}

// enc = ctx * (1 + psst[1] + pts2[1]) + (psst[0] + pts2[0])   (ltx/block.zig:298-301)
__global__ void ctx_modulate_kernel(const float* __restrict__ ctx, int S, int D, const float* __restrict__ psst,
                                    const float* __restrict__ pts2, __nv_bfloat16* __restrict__ ob,
                                    float* __restrict__ of) {
  const size_t n = (size_t)S * D;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int c = (int)(i % D);
    const float shift = psst[c] + pts2[c];
    const float scale = psst[D + c] + pts2[D + c];
    const float v = ctx[i] * (scale + 1.0f) + shift;
    if (ob) ob[i] = __float2bfloat16_rn(v);
    if (of) of[i] = v;
  }
}

int ctx_modulate(const float* ctx, int S, int D, const float* psst, const float* pts2, void* out_bf16,
                 float* out_f32, cudaStream_t st) {
  if (S <= 0) return LTXB_OK;
  const size_t n = (size_t)S * D;
  int grid = (int)((n + 255) / 256);
  if (grid > 4 * sm_count()) grid = 4 * sm_count();
  ctx_modulate_kernel<<<grid, 256, 0, st>>>(ctx, S, D, psst, pts2, reinterpret_cast<__nv_bfloat16*>(out_bf16),
                                            out_f32);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "ctx_modulate");
}

// int8 [N, K] x scale[N, K/128] -> bf16 [N, K]; 16 weights per chunk, four
// chunks per thread in flight (their loads issued before any arithmetic).
__device__ __forceinline__ float dq_scale(const void* scales, int scale_bf16, size_t si) {
  return scale_bf16 ? __uint_as_float((uint32_t)__ldg(reinterpret_cast<const uint16_t*>(scales) + si) << 16)
                    : __ldg(reinterpret_cast<const float*>(scales) + si);
}

__device__ __forceinline__ void dq_store16(uint4 v, float s, __nv_bfloat16* out) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  uint32_t o[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int8_t b0 = (int8_t)(w[j] & 0xFF), b1 = (int8_t)((w[j] >> 8) & 0xFF);
    const int8_t b2 = (int8_t)((w[j] >> 16) & 0xFF), b3 = (int8_t)(w[j] >> 24);
    o[2 * j] = pack_bf16x2((float)b0 * s, (float)b1 * s);
    o[2 * j + 1] = pack_bf16x2((float)b2 * s, (float)b3 * s);
  }
  uint4* op = reinterpret_cast<uint4*>(out);
  op[0] = make_uint4(o[0], o[1], o[2], o[3]);
  op[1] = make_uint4(o[4], o[5], o[6], o[7]);
}

__global__ void __launch_bounds__(256, 4) dequant_weights_kernel(const int8_t* __restrict__ q,
                                                              const void* __restrict__ scales, int scale_bf16, int N,
                                                              int K, __nv_bfloat16* __restrict__ out) {
  const size_t n16 = (size_t)N * K / 16;
  const int G = K / 128, c16 = K / 16;  // chunks per row
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  for (; i + 3 * stride < n16; i += 4 * stride) {
    uint4 v[4];
    float sc[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const size_t c = i + u * stride;
      v[u] = __ldg(reinterpret_cast<const uint4*>(q) + c);
      sc[u] = dq_scale(scales, scale_bf16, (c / c16) * G + ((c % c16) >> 3));
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) dq_store16(v[u], sc[u], out + (i + u * stride) * 16);
  }
  for (; i < n16; i += stride)
    dq_store16(__ldg(reinterpret_cast<const uint4*>(q) + i), dq_scale(scales, scale_bf16, (i / c16) * G + ((i % c16) >> 3)),
               out + i * 16);
}

int dequant_weights(const int8_t* q, const void* scales, int scale_bf16, int N, int K, void* out, cudaStream_t st) {
  if ((size_t)N * K == 0) return LTXB_OK;
  if (K % 128) return set_error(LTXB_EINVAL, "dequant: K %% 128");
  if ((reinterpret_cast<uintptr_t>(q) & 15) || (reinterpret_cast<uintptr_t>(out) & 15) ||
      (reinterpret_cast<uintptr_t>(scales) & (scale_bf16 ? 1 : 3)))
    return set_error(LTXB_EINVAL, "dequant: weights and output must be 16-byte aligned, scales element-aligned");
  const size_t n16 = (size_t)N * K / 16;
  int grid = (int)((n16 + 255) / 256);
  if (grid > 8 * sm_count()) grid = 8 * sm_count();
  dequant_weights_kernel<<<grid, 256, 0, st>>>(q, scales, scale_bf16, N, K, reinterpret_cast<__nv_bfloat16*>(out));
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "dequant_weights");
}

// (w_hi | w_lo) rows from int8 + scales, 8 weights per thread step
__global__ void dequant_split_kernel(const int8_t* __restrict__ q, const void* __restrict__ scales, int scale_bf16,
                                     int N, int K, __nv_bfloat16* __restrict__ out) {
  const size_t n8 = (size_t)N * K / 8;
  const int G = K / 128;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n8; i += (size_t)gridDim.x * blockDim.x) {
    const size_t e0 = i * 8;
    const size_t row = e0 / K, col = e0 % K;
    const int g = (int)(col >> 7);
    const float s = scale_bf16
                        ? __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(scales)[row * G + g] << 16)
                        : reinterpret_cast<const float*>(scales)[row * G + g];
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(q) + i);
    const uint32_t w[2] = {v.x, v.y};
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
#pragma unroll
      for (int b = 0; b < 4; b += 2) {
        const float f0 = (float)(int8_t)((w[j] >> (8 * b)) & 0xFF) * s;
        const float f1 = (float)(int8_t)((w[j] >> (8 * b + 8)) & 0xFF) * s;
        const uint32_t h = pack_bf16x2(f0, f1);
        hi[2 * j + b / 2] = h;
        lo[2 * j + b / 2] = pack_bf16x2(f0 - bf16_lo(h), f1 - bf16_hi(h));
      }
    }
    __nv_bfloat16* o = out + row * (size_t)(2 * K) + col;
    *reinterpret_cast<uint4*>(o) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *reinterpret_cast<uint4*>(o + K) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
}

int dequant_split(const int8_t* q, const void* scales, int scale_bf16, int N, int K, void* out, cudaStream_t st) {
  if ((size_t)N * K == 0) return LTXB_OK;
  if (K % 128) return set_error(LTXB_EINVAL, "dequant_split: K %% 128");
  if ((reinterpret_cast<uintptr_t>(q) & 7) || (reinterpret_cast<uintptr_t>(out) & 15))
    return set_error(LTXB_EINVAL, "dequant_split: weights 8-byte and output 16-byte aligned");
  const size_t n8 = (size_t)N * K / 8;
  int grid = (int)((n8 + 255) / 256);
  if (grid > 8 * sm_count()) grid = 8 * sm_count();
  dequant_split_kernel<<<grid, 256, 0, st>>>(q, scales, scale_bf16, N, K, reinterpret_cast<__nv_bfloat16*>(out));
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "dequant_split");
}

// Head-group regrouping for the sequence-parallel exchange. The columns of
// a [T, D] matrix split into N rank groups of D/N, each into SG sub-groups of
// Dg = D / (N SG). sp_regroup: up to three token-major bf16 matrices (row
// strides ld[x]) -> [SG][x][N][T][Dg], so that every (sub-group, tensor,
// rank) block is contiguous; sp_ungroup: [SG][N][T][Dg] -> [T, D] (row stride
// ld_out). 16-byte moves.
struct RegroupSrc {
  const __nv_bfloat16* p[3];
  int ld[3];
};

__global__ void sp_regroup_kernel(RegroupSrc src, int nsrc, int T, int D, int N, int SG,
                                  __nv_bfloat16* __restrict__ dst) {
  const int Dn = D / N, Dg = Dn / SG, c8 = Dg / 8;
  const size_t blk8 = (size_t)T * c8;  // 16-byte units per block
  const size_t n = (size_t)SG * nsrc * N * blk8;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t b = i / blk8, k = i % blk8;  // block index = (g nsrc + x) N + p
    const int p = (int)(b % N), x = (int)((b / N) % nsrc), g = (int)(b / ((size_t)N * nsrc));
    const int t = (int)(k / c8), c = (int)(k % c8) * 8;
    const uint4 v = *reinterpret_cast<const uint4*>(src.p[x] + (size_t)t * src.ld[x] + p * Dn + g * Dg + c);
    *reinterpret_cast<uint4*>(dst + (b * T + t) * Dg + c) = v;
  }
}

__global__ void sp_ungroup_kernel(const __nv_bfloat16* __restrict__ src, int T, int D, int N, int SG,
                                  __nv_bfloat16* __restrict__ out, int ld_out) {
  const int Dn = D / N, Dg = Dn / SG, c8 = Dg / 8;
  const size_t blk8 = (size_t)T * c8;
  const size_t n = (size_t)SG * N * blk8;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t b = i / blk8, k = i % blk8;  // block index = g N + p
    const int p = (int)(b % N), g = (int)(b / N);
    const int t = (int)(k / c8), c = (int)(k % c8) * 8;
    *reinterpret_cast<uint4*>(out + (size_t)t * ld_out + p * Dn + g * Dg + c) =
        *reinterpret_cast<const uint4*>(src + (b * T + t) * Dg + c);
  }
}

int sp_regroup(const void* const* srcs, const int* lds, int nsrc, int T, int D, int N, int SG, void* dst,
               cudaStream_t st) {
  if (nsrc < 1 || nsrc > 3 || N < 1 || SG < 1 || D % (8 * N * SG))
    return set_error(LTXB_EINVAL, "sp_regroup: D must split into 16-byte groups");
  RegroupSrc s{};
  for (int x = 0; x < nsrc; ++x) {
    s.p[x] = static_cast<const __nv_bfloat16*>(srcs[x]);
    s.ld[x] = lds[x];
    if ((reinterpret_cast<uintptr_t>(srcs[x]) & 15) || lds[x] % 8) return set_error(LTXB_EINVAL, "sp_regroup: alignment");
  }
  const size_t n = (size_t)nsrc * T * (D / 8);
  if (n == 0) return LTXB_OK;
  int grid = (int)((n + 255) / 256);
  if (grid > 8 * sm_count()) grid = 8 * sm_count();
  sp_regroup_kernel<<<grid, 256, 0, st>>>(s, nsrc, T, D, N, SG, static_cast<__nv_bfloat16*>(dst));
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "sp_regroup");
}

int sp_ungroup(const void* src, int T, int D, int N, int SG, void* out, int ld_out, cudaStream_t st) {
  if (N < 1 || SG < 1 || D % (8 * N * SG) || ld_out % 8)
    return set_error(LTXB_EINVAL, "sp_ungroup: D must split into 16-byte groups");
  const size_t n = (size_t)T * (D / 8);
  if (n == 0) return LTXB_OK;
  int grid = (int)((n + 255) / 256);
  if (grid > 8 * sm_count()) grid = 8 * sm_count();
  sp_ungroup_kernel<<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(src), T, D, N, SG,
                                          static_cast<__nv_bfloat16*>(out), ld_out);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "sp_ungroup");
}

__global__ void cast_f32_bf16_kernel(const float* __restrict__ in, __nv_bfloat16* __restrict__ out, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n / 4; i += (size_t)gridDim.x * blockDim.x) {
    float4 v = reinterpret_cast<const float4*>(in)[i];
    reinterpret_cast<uint2*>(out)[i] = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
  }
}

int cast_f32_bf16(const float* in, void* out, size_t n, cudaStream_t st) {
  if (n == 0) return LTXB_OK;
  if (n % 4) return set_error(LTXB_EINVAL, "cast: n %% 4");
  int grid = (int)((n / 4 + 255) / 256);
  if (grid > 8 * sm_count()) grid = 8 * sm_count();
  cast_f32_bf16_kernel<<<grid, 256, 0, st>>>(in, reinterpret_cast<__nv_bfloat16*>(out), n);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "cast_f32_bf16");
}

__global__ void split_f32_bf16_kernel(const float* __restrict__ in, int rows, int cols, int parts,
                                      __nv_bfloat16* __restrict__ out) {
  const size_t n = (size_t)rows * cols;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / cols, c = i % cols;
    const float x = in[i];
    const __nv_bfloat16 hi = __float2bfloat16_rn(x);
    const __nv_bfloat16 lo = __float2bfloat16_rn(x - __bfloat162float(hi));
    __nv_bfloat16* o = out + r * (size_t)parts * cols + c;
    o[0] = hi;
    if (parts == 2) o[cols] = lo;
    if (parts == 3) {
      o[cols] = hi;
      o[2 * (size_t)cols] = lo;
    }
  }
}

int split_f32_bf16(const float* in, int rows, int cols, int parts, void* out, cudaStream_t st) {
  const size_t n = (size_t)rows * cols;
  if (n == 0) return LTXB_OK;
  if (parts < 2 || parts > 3) return set_error(LTXB_EINVAL, "split_f32_bf16: 2 or 3 parts");
  int grid = (int)((n + 255) / 256);
  if (grid > 8 * sm_count()) grid = 8 * sm_count();
  split_f32_bf16_kernel<<<grid, 256, 0, st>>>(in, rows, cols, parts, reinterpret_cast<__nv_bfloat16*>(out));
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "split_f32_bf16");
}

__global__ void cast_rows_f32_bf16_kernel(const float* __restrict__ in, int ld_in, __nv_bfloat16* __restrict__ out,
                                          int ld_out, int rows, int cols) {
  const size_t n = (size_t)rows * cols;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / cols, c = i % cols;
    out[r * ld_out + c] = __float2bfloat16_rn(in[r * ld_in + c]);
  }
}

int cast_rows_f32_bf16(const float* in, int ld_in, void* out, int ld_out, int rows, int cols, cudaStream_t st) {
  const size_t n = (size_t)rows * cols;
  if (n == 0) return LTXB_OK;
  int grid = (int)((n + 255) / 256);
  if (grid > 8 * sm_count()) grid = 8 * sm_count();
  cast_rows_f32_bf16_kernel<<<grid, 256, 0, st>>>(in, ld_in, reinterpret_cast<__nv_bfloat16*>(out), ld_out, rows, cols);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "cast_rows_f32_bf16");
}

__global__ void cast_bf16_f32_kernel(const __nv_bfloat16* __restrict__ in, float* __restrict__ out, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    out[i] = __bfloat162float(in[i]);
}

int cast_bf16_f32(const void* in, float* out, size_t n, cudaStream_t st) {
  if (n == 0) return LTXB_OK;
  int grid = (int)((n + 255) / 256);
  if (grid > 8 * sm_count()) grid = 8 * sm_count();
  cast_bf16_f32_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(in), out, n);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "cast_bf16_f32");
}

}  // namespace ltxb
