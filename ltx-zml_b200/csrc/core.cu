// Device-side steps either side of the block:
//
// * the core parts of ltx/core_parts.zig (adaln MLPs -> embedded_timestep
//   and the block's ts9 table, prompt adaln -> pts2, patchify_proj, and the
//   output tail LayerNorm -> modulate -> proj_out), in f32 with bf16
//   weights like the reference's traced model: the linears run on the f32
//   SIMT GEMM (they are < 0.2 % of a step's FLOPs), the sinusoid, SiLU and
//   the LayerNorm-modulate pass are kernels here;
// * the distilled scheduler of ltx/scheduler.zig, bit-exact in f32: the
//   rounding of every reference operation is reproduced with _rn
//   intrinsics (no contraction into FMA), and torch.lerp's fused
//   multiply-add with __fmaf_rn;
//
// * RoPE tables in the block's cos/sin layout [T, H, 64] f32, generated on
//   the GPU instead of host-built 0.9 GB tables at 28k tokens:
//     - LTX layout (ltx/block_conformance.zig:87-127): frequency grid
//       theta^(k/(NF-1)) * pi/2 in f64 rounded to f32 (NF = H*128/6), token
//       position = midpoint of its (start, end) grid cell per axis, scaled
//       to [-1, 1] by max_pos (20, 2048, 2048); table slot j = h*64 + f:
//       j < 2 is the identity (1, 0), else frequency (j-2)/3 of axis
//       (j-2)%3. Angles, cos and sin in f64, rounded to f32 at the end —
//       the reference's host generator.
//     - per-axis split (44, 42, 42) of each head's 128 dims from integer
//       (frame, row, col) positions, the same table for every head:
//       inv_k = theta^(-2k/dims) in f64.
//   The small frequency tables are computed on the host in f64 exactly as
//   the reference computes them and passed by value.
#include <math.h>
#include <string.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "upload.h"

namespace ltxb {

constexpr int kRopeMaxNF = 700;  // H*128/6 for H <= 32

struct RopeTab {
  double axes_inv[64];     // per-axis split: inverse frequencies per pair
  int axes_axis[64];       // axis of each pair
  float ltx_f[kRopeMaxNF];  // LTX layout: f32-rounded frequency grid
};

__global__ void rope_ltx_kernel(const float* __restrict__ grid, int T, int H, const __grid_constant__ RopeTab tab,
                                float* __restrict__ cos_out, float* __restrict__ sin_out) {
  const size_t n = (size_t)T * H * 64;
  const double maxpos[3] = {20.0, 2048.0, 2048.0};
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / ((size_t)H * 64));
    const int j = (int)(i % ((size_t)H * 64));
    double c = 1.0, s = 0.0;
    if (j >= 2) {
      const int q = j - 2, k = q / 3, ax = q % 3;
      const double s0 = grid[((size_t)ax * T + t) * 2], s1 = grid[((size_t)ax * T + t) * 2 + 1];
      const double mid = __dadd_rn(s0, s1) / 2.0;
      const double arg = __dadd_rn(__dmul_rn(mid / maxpos[ax], 2.0), -1.0);
      sincos(__dmul_rn((double)tab.ltx_f[k], arg), &s, &c);
    }
    cos_out[i] = (float)c;
    sin_out[i] = (float)s;
  }
}

__global__ void rope_axes_kernel(const float* __restrict__ pos, int T, int H, const __grid_constant__ RopeTab tab,
                                 float* __restrict__ cos_out, float* __restrict__ sin_out) {
  const size_t n = (size_t)T * 64;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / 64), f = (int)(i % 64);
    double s, c;
    sincos(__dmul_rn((double)pos[(size_t)t * 3 + tab.axes_axis[f]], tab.axes_inv[f]), &s, &c);
    const float cf = (float)c, sf = (float)s;
    for (int h = 0; h < H; ++h) {
      cos_out[((size_t)t * H + h) * 64 + f] = cf;
      sin_out[((size_t)t * H + h) * 64 + f] = sf;
    }
  }
}

int rope_tables(int kind, const float* pos, int T, int H, double theta, float* cos_out, float* sin_out,
                cudaStream_t st) {
  if (T <= 0) return LTXB_OK;
  if (H <= 0 || !pos || !cos_out || !sin_out) return set_error(LTXB_EINVAL, "rope: bad arguments");
  RopeTab tab;
  memset(&tab, 0, sizeof(tab));
  int grid = 0;
  if (kind == LTXB_ROPE_LTX) {
    const int nf = H * 128 / 6;
    if (nf < 2 || nf > kRopeMaxNF || (H * 64 - 3) / 3 >= nf)
      return set_error(LTXB_EUNSUPPORTED, "rope: LTX layout supports up to %d frequencies (H <= 32)", kRopeMaxNF);
    for (int k = 0; k < nf; ++k) {
      const double x = (double)k / (double)(nf - 1 > 0 ? nf - 1 : 1);
      tab.ltx_f[k] = (float)(pow(theta, x) * (M_PI / 2.0));
    }
    const size_t n = (size_t)T * H * 64;
    grid = (int)std::min<size_t>((n + 255) / 256, (size_t)sm_count() * 16);
    rope_ltx_kernel<<<grid, 256, 0, st>>>(pos, T, H, tab, cos_out, sin_out);
  } else if (kind == LTXB_ROPE_AXES) {
    const int split[3] = {44, 42, 42};
    int f = 0;
    for (int ax = 0; ax < 3; ++ax)
      for (int k = 0; k < split[ax] / 2; ++k, ++f) {
        tab.axes_inv[f] = pow(theta, -2.0 * k / split[ax]);
        tab.axes_axis[f] = ax;
      }
    const size_t n = (size_t)T * 64;
    grid = (int)std::min<size_t>((n + 255) / 256, (size_t)sm_count() * 16);
    rope_axes_kernel<<<grid, 256, 0, st>>>(pos, T, H, tab, cos_out, sin_out);
  } else {
    return set_error(LTXB_EINVAL, "rope: unknown table kind %d", kind);
  }
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "rope tables");
}


// ---------------------------------------------------------------------------
// core parts
// ---------------------------------------------------------------------------

// out [K, 256]: cos(t*1000*f_i) | sin(t*1000*f_i), f_i = exp(i * (-ln(1e4)/128))
// in f32 (ltx/core_parts.zig:42-49)
__global__ void sinusoid_kernel(const float* __restrict__ t, int K, float* __restrict__ out) {
  const int n = K * 128;
  const float c = (float)(-9.210340371976184 / 128.0);  // -ln(1e4)/128 as an f32 constant
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int k = i / 128, f = i % 128;
    const float freq = expf(__fmul_rn((float)f, c));
    const float arg = __fmul_rn(__fmul_rn(t[k], 1000.0f), freq);
    float sn, cs;
    sincosf(arg, &sn, &cs);
    out[(size_t)k * 256 + f] = cs;
    out[(size_t)k * 256 + 128 + f] = sn;
  }
}

// y = x * sigmoid(x)
__global__ void silu_kernel(const float* __restrict__ x, float* __restrict__ y, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    y[i] = v / (1.0f + expf(-v));
  }
}

// out = LayerNorm(x) * (1 + fsst[1] + e) + (fsst[0] + e), LayerNorm mean-
// subtracting with biased variance and eps 1e-6 (ltx/core_parts.zig:30-35,
// :148-152); e = emb[row] with row = tidx[t] chosen as the block's
// modulation-table row (table_row: out-of-range reads row 0), or emb[t]
// without tidx. One CTA per row.
__global__ void __launch_bounds__(256) tail_norm_kernel(const float* __restrict__ x, const float* __restrict__ emb,
                                                        int K, const int* __restrict__ tidx,
                                                        const float* __restrict__ fsst,
                                                        int D, float* __restrict__ out) {
  __shared__ float red[8];
  const int t = blockIdx.x;
  const float* xr = x + (size_t)t * D;
  const float* er = emb + (size_t)(tidx ? table_row(tidx, t, K) : t) * D;
  auto block_sum = [&](float v) {
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = 0.f;
    for (int w = 0; w < 8; ++w) s += red[w];
    return s;
  };
  float s = 0.f;
  for (int i = threadIdx.x; i < D; i += 256) s += xr[i];
  const float mean = block_sum(s) / (float)D;
  float v = 0.f;
  for (int i = threadIdx.x; i < D; i += 256) {
    const float d = xr[i] - mean;
    v += d * d;
  }
  const float rstd = rsqrtf(block_sum(v) / (float)D + 1e-6f);
  for (int i = threadIdx.x; i < D; i += 256) {
    const float n = (xr[i] - mean) * rstd;
    const float scale = fsst[D + i] + er[i], shift = fsst[i] + er[i];
    out[(size_t)t * D + i] = n * (1.0f + scale) + shift;
  }
}

static int grid_for(size_t n) { return (int)std::min<size_t>((n + 255) / 256, (size_t)sm_count() * 16); }

int sinusoid(const float* t, int K, float* out, cudaStream_t st) {
  if (K <= 0) return LTXB_OK;
  sinusoid_kernel<<<grid_for((size_t)K * 128), 256, 0, st>>>(t, K, out);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "sinusoid");
}

static int silu(const float* x, float* y, size_t n, cudaStream_t st) {
  if (!n) return LTXB_OK;
  silu_kernel<<<grid_for(n), 256, 0, st>>>(x, y, n);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "silu");
}

__global__ void fill_kernel(float* p, int n, float v) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) p[i] = v;
}

// ---------------------------------------------------------------------------
// scheduler
// ---------------------------------------------------------------------------

// torch.lerp: |w| < 0.5 -> a + w (b - a), else b - (b - a)(1 - w), each a single
// fused multiply-add (ltx/scheduler.zig:20-35)
__device__ __forceinline__ float lerp_t(float a, float b, float w) {
  const float d = __fsub_rn(b, a);
  if (fabsf(w) < 0.5f) return __fmaf_rn(w, d, a);
  return __fmaf_rn(-d, __fsub_rn(1.0f, w), b);
}

__global__ void noise_init_kernel(const float* __restrict__ clean, const float* __restrict__ noise,
                                  const float* __restrict__ mask, size_t n, int C, float noise_scale,
                                  float* __restrict__ out) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float c = clean[i];
    out[i] = lerp_t(c, lerp_t(c, noise[i], noise_scale), mask[i / C]);
  }
}

__global__ void timesteps_kernel(const float* __restrict__ mask, int T, float sigma, float* __restrict__ ts) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < T; i += gridDim.x * blockDim.x) ts[i] = __fmul_rn(mask[i], sigma);
}

// to_denoised -> post_process -> Euler step (ltx/scheduler.zig:54-80), fused
// per element with every reference rounding kept
__global__ void sched_step_kernel(const float* __restrict__ x, const float* __restrict__ vel,
                                  const float* __restrict__ ts, const float* __restrict__ clean,
                                  const float* __restrict__ mask, size_t n, int C, float sigma, float dt,
                                  float* __restrict__ out) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t t = i / C;
    const float xi = x[i];
    const float den = __fsub_rn(xi, __fmul_rn(vel[i], ts[t]));
    const float m = mask[t];
    const float post = __fadd_rn(__fmul_rn(den, m), __fmul_rn(clean[i], __fsub_rn(1.0f, m)));
    const float v = __fdiv_rn(__fsub_rn(xi, post), sigma);
    out[i] = __fadd_rn(xi, __fmul_rn(v, dt));
  }
}

}  // namespace ltxb

using namespace ltxb;

struct ltxb_core {
  int device = 0, D = 0;
  Lin ada1, ada2, ada_out, pada1, pada2, pada_out, pat, po;
  const float* fsst = nullptr;
  std::vector<void*> allocs;
  uint64_t bytes = 0;
};

// DISTILLED_SIGMA_VALUES and its stage-2 tail (ltx/scheduler.zig:11-18): each
// decimal is parsed to f64 and then cast to f32, as the reference does.
static const float kSigmasStage1[] = {(float)1.0,      (float)0.99375, (float)0.9875,   (float)0.98125, (float)0.975,
                                      (float)0.909375, (float)0.725,   (float)0.421875, (float)0.0};
static const float kSigmasStage2[] = {(float)0.909375, (float)0.725, (float)0.421875, (float)0.0};

extern "C" {

void ltxb_core_free(ltxb_core* c) {
  if (!c) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(c->device);
  for (void* p : c->allocs) cudaFree(p);
  cudaSetDevice(prev);
  delete c;
}

int ltxb_core_upload(int device, const void* blob, uint64_t blob_bytes, const ltxb_entry* entries, int n_entries,
                     int hidden, ltxb_core** out) {
  if (!out || !blob || !entries || n_entries <= 0) return set_error(LTXB_EINVAL, "core upload: null argument");
  if (hidden <= 0 || hidden % 128) return set_error(LTXB_EINVAL, "core upload: hidden must be a multiple of 128");
  *out = nullptr;
  if (int rc0 = check_entries(entries, n_entries, blob_bytes)) return rc0;
  cudaError_t ce = cudaSetDevice(device);
  if (ce != cudaSuccess) return set_cuda_error(ce, "cudaSetDevice");
  auto* c = new ltxb_core();
  c->device = device;
  c->D = hidden;
  const int D = hidden;
  Uploader u{&c->allocs, &c->bytes, static_cast<const uint8_t*>(blob), blob_bytes, entries, n_entries, -1};
  int rc = u.linear(c->ada1, {"adaln_single_emb_timestep_embedder_linear_1"}, D, 256, true, false);
  if (!rc) rc = u.linear(c->ada2, {"adaln_single_emb_timestep_embedder_linear_2"}, D, D, true, false);
  if (!rc) rc = u.linear(c->ada_out, {"adaln_single_linear"}, 9 * D, D, true, false);
  if (!rc) rc = u.linear(c->pada1, {"prompt_adaln_single_emb_timestep_embedder_linear_1"}, D, 256, true, false);
  if (!rc) rc = u.linear(c->pada2, {"prompt_adaln_single_emb_timestep_embedder_linear_2"}, D, D, true, false);
  if (!rc) rc = u.linear(c->pada_out, {"prompt_adaln_single_linear"}, 2 * D, D, true, false);
  if (!rc) rc = u.linear(c->pat, {"patchify_proj"}, D, 128, true, false);
  if (!rc) rc = u.linear(c->po, {"proj_out"}, 128, D, true, false);
  const void* fsst = nullptr;
  if (!rc) rc = u.tensor("scale_shift_table", LTXB_DT_F32, 2, D, &fsst);
  if (rc) {
    ltxb_core_free(c);
    return rc;
  }
  c->fsst = static_cast<const float*>(fsst);
  *out = c;
  return LTXB_OK;
}

static uint64_t up256(uint64_t x) { return (x + 255) & ~uint64_t(255); }

static uint64_t adaln_ws(int D, int K) { return up256((uint64_t)K * 256 * 4) + 2 * up256((uint64_t)K * D * 4); }

uint64_t ltxb_core_workspace_bytes(const ltxb_core* c, int T, int K) {
  if (!c) return 0;
  const uint64_t a = adaln_ws(c->D, K > 1 ? K : 1), t = up256((uint64_t)(T > 0 ? T : 0) * c->D * 4);
  return a > t ? a : t;
}

int ltxb_core_sinusoid(const float* t, int K, float* out, void* stream) {
  if (K > 0 && (!t || !out)) return set_error(LTXB_EINVAL, "sinusoid: null argument");
  return sinusoid(t, K, out, static_cast<cudaStream_t>(stream));
}

// [K, 256] sinusoid -> linear_1 -> SiLU -> linear_2 (= emb) -> SiLU -> out linear
static int adaln_mlp(const ltxb_core* c, const Lin& l1, const Lin& l2, const Lin& lo, const float* t, int K,
                     float* emb, float* out, void* ws, uint64_t ws_bytes, cudaStream_t st) {
  const int D = c->D;
  if (!ws || ws_bytes < adaln_ws(D, K))
    return set_error(LTXB_EINVAL, "core: workspace of %llu bytes is smaller than the %llu required",
                     (unsigned long long)ws_bytes, (unsigned long long)adaln_ws(D, K));
  uint8_t* w = static_cast<uint8_t*>(ws);
  float* sn = reinterpret_cast<float*>(w);
  float* h = reinterpret_cast<float*>(w + up256((uint64_t)K * 256 * 4));
  float* e2 = reinterpret_cast<float*>(w + up256((uint64_t)K * 256 * 4) + up256((uint64_t)K * D * 4));
  int rc = sinusoid(t, K, sn, st);
  if (!rc) rc = gemm_f32(sn, 256, l1.w, K, D, 256, l1.b, EPI_F32, h, D, nullptr, 0, nullptr, nullptr, nullptr, nullptr, 0, 0, st);
  if (!rc) rc = silu(h, h, (size_t)K * D, st);
  float* e = emb ? emb : e2;
  if (!rc) rc = gemm_f32(h, D, l2.w, K, D, D, l2.b, EPI_F32, e, D, nullptr, 0, nullptr, nullptr, nullptr, nullptr, 0, 0, st);
  if (!rc) rc = silu(e, e2, (size_t)K * D, st);
  if (!rc) rc = gemm_f32(e2, D, lo.w, K, lo.N, D, lo.b, EPI_F32, out, lo.N, nullptr, 0, nullptr, nullptr, nullptr, nullptr, 0, 0, st);
  return rc;
}

int ltxb_core_adaln(const ltxb_core* c, const float* t, int K, float* emb, float* ts9, void* workspace,
                    uint64_t workspace_bytes, void* stream) {
  if (!c || !t || !ts9) return set_error(LTXB_EINVAL, "core adaln: null argument");
  if (K <= 0) return LTXB_OK;
  if (int rc = check_device(c->device, "core adaln")) return rc;
  return adaln_mlp(c, c->ada1, c->ada2, c->ada_out, t, K, emb, ts9, workspace, workspace_bytes,
                   static_cast<cudaStream_t>(stream));
}

int ltxb_core_pts2(const ltxb_core* c, const float* sigma, float* pts2, void* workspace, uint64_t workspace_bytes,
                   void* stream) {
  if (!c || !sigma || !pts2) return set_error(LTXB_EINVAL, "core pts2: null argument");
  if (int rc = check_device(c->device, "core pts2")) return rc;
  return adaln_mlp(c, c->pada1, c->pada2, c->pada_out, sigma, 1, nullptr, pts2, workspace, workspace_bytes,
                   static_cast<cudaStream_t>(stream));
}

int ltxb_core_patchify(const ltxb_core* c, const float* latent, int T, float* x, void* stream) {
  if (!c || (T > 0 && (!latent || !x))) return set_error(LTXB_EINVAL, "core patchify: null argument");
  if (T > 0)
    if (int rc = check_device(c->device, "core patchify")) return rc;
  return gemm_f32(latent, 128, c->pat.w, T, c->D, 128, c->pat.b, EPI_F32, x, c->D, nullptr, 0, nullptr, nullptr,
                  nullptr, nullptr, 0, 0, static_cast<cudaStream_t>(stream));
}

int ltxb_core_tail(const ltxb_core* c, const float* x, const float* emb, int K, const int* tidx, int T, float* velocity,
                   void* workspace, uint64_t workspace_bytes, void* stream) {
  if (!c || (T > 0 && (!x || !emb || !velocity))) return set_error(LTXB_EINVAL, "core tail: null argument");
  if (T <= 0) return LTXB_OK;
  if (int rc = check_device(c->device, "core tail")) return rc;
  if (tidx && K <= 0) return set_error(LTXB_EINVAL, "core tail: K must be positive with tidx");
  const uint64_t need = up256((uint64_t)T * c->D * 4);
  if (!workspace || workspace_bytes < need)
    return set_error(LTXB_EINVAL, "core tail: workspace of %llu bytes is smaller than the %llu required",
                     (unsigned long long)workspace_bytes, (unsigned long long)need);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* n = static_cast<float*>(workspace);
  tail_norm_kernel<<<T, 256, 0, st>>>(x, emb, K, tidx, c->fsst, c->D, n);
  launched();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "tail norm");
  return gemm_f32(n, c->D, c->po.w, T, 128, c->D, c->po.b, EPI_F32, velocity, 128, nullptr, 0, nullptr, nullptr,
                  nullptr, nullptr, 0, 0, st);
}

int ltxb_sched_sigmas(int stage, float* out, int capacity) {
  const float* s = stage == 1 ? kSigmasStage1 : stage == 2 ? kSigmasStage2 : nullptr;
  const int n = stage == 1 ? 9 : stage == 2 ? 4 : 0;
  if (!s) return set_error(LTXB_EINVAL, "sigmas: stage must be 1 or 2");
  if (out) {
    if (capacity < n) return set_error(LTXB_EINVAL, "sigmas: capacity %d < %d", capacity, n);
    memcpy(out, s, n * sizeof(float));
  }
  return n;
}

int ltxb_sched_noise_init(const float* clean, const float* noise, const float* mask, int T, int C, float noise_scale,
                          float* out, void* stream) {
  if (T <= 0) return LTXB_OK;
  if (!clean || !noise || !mask || !out || C <= 0) return set_error(LTXB_EINVAL, "noise init: bad arguments");
  const size_t n = (size_t)T * C;
  noise_init_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(clean, noise, mask, n, C, noise_scale,
                                                                              out);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "noise init");
}

int ltxb_sched_timesteps(const float* mask, int T, float sigma, float* ts, void* stream) {
  if (T <= 0) return LTXB_OK;
  if (!mask || !ts) return set_error(LTXB_EINVAL, "timesteps: null argument");
  timesteps_kernel<<<grid_for((size_t)T), 256, 0, static_cast<cudaStream_t>(stream)>>>(mask, T, sigma, ts);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "timesteps");
}

int ltxb_sched_step(const float* x, const float* velocity, const float* ts, const float* clean, const float* mask,
                    int T, int C, float sigma, float sigma_next, float* out, void* stream) {
  if (T <= 0) return LTXB_OK;
  if (!x || !velocity || !ts || !clean || !mask || !out || C <= 0) return set_error(LTXB_EINVAL, "step: bad arguments");
  const size_t n = (size_t)T * C;
  const float dt = sigma_next - sigma;  // one f32 subtraction, as the reference's host
  sched_step_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, velocity, ts, clean, mask, n, C,
                                                                              sigma, dt, out);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "scheduler step");
}

// ---------------------------------------------------------------------------
// denoising loop
// ---------------------------------------------------------------------------

struct DenoiseWs {
  uint8_t* block;  // the blocks' workspace
  float *x, *emb, *ts9, *pts2, *vel, *ts, *tk, *sig, *core;
  uint64_t block_bytes, core_bytes, total;
};

static DenoiseWs denoise_layout(const ltxb_core* c, const ltxb_weights* blk, const ltxb_config* cfg, uint8_t* base) {
  DenoiseWs w{};
  const uint64_t T = cfg->T, K = cfg->K, D = c->D;
  uint64_t off = 0;
  auto take = [&](uint64_t bytes) {
    uint8_t* p = base ? base + off : nullptr;
    off += up256(bytes);
    return p;
  };
  w.block_bytes = ltxb_block_workspace_bytes(blk, cfg);
  w.core_bytes = ltxb_core_workspace_bytes(c, cfg->T, cfg->K);
  w.block = take(w.block_bytes);
  w.x = reinterpret_cast<float*>(take(T * D * 4));
  w.emb = reinterpret_cast<float*>(take(K * D * 4));
  w.ts9 = reinterpret_cast<float*>(take(K * 9 * D * 4));
  w.pts2 = reinterpret_cast<float*>(take(2 * D * 4));
  w.vel = reinterpret_cast<float*>(take(T * 128 * 4));
  w.ts = reinterpret_cast<float*>(take(T * 4));
  w.tk = reinterpret_cast<float*>(take(K * 4));
  w.sig = reinterpret_cast<float*>(take(4));
  w.core = reinterpret_cast<float*>(take(w.core_bytes));
  w.total = off;
  return w;
}

uint64_t ltxb_denoise_workspace_bytes(const ltxb_core* core, const ltxb_weights* block, const ltxb_config* cfg) {
  if (!core || !block || !cfg) return 0;
  return denoise_layout(core, block, cfg, nullptr).total;
}

int ltxb_denoise_run(const ltxb_core* core, const ltxb_weights* const* blocks, int n_blocks, const float* sigmas,
                     int n_steps, const ltxb_denoise_io* io, const ltxb_config* cfg, void* stream) {
  if (!core || !blocks || n_blocks <= 0 || !sigmas || n_steps < 0 || !io || !cfg)
    return set_error(LTXB_EINVAL, "denoise: null argument");
  if (!io->latent || !io->clean || !io->mask || !io->mask_values || !io->tidx || !io->ctx || !io->cos || !io->sin)
    return set_error(LTXB_EINVAL, "denoise: null tensor");
  if (cfg->T <= 0 || cfg->K <= 0 || cfg->S <= 0) return set_error(LTXB_EINVAL, "denoise: T, K and S must be positive");
  for (int b = 0; b < n_blocks; ++b)
    if (!blocks[b]) return set_error(LTXB_EINVAL, "denoise: block %d is null", b);
  if (int rc = check_device(core->device, "denoise")) return rc;
  const DenoiseWs need = denoise_layout(core, blocks[0], cfg, nullptr);
  if (!io->workspace || io->workspace_bytes < need.total)
    return set_error(LTXB_EINVAL, "denoise: workspace of %llu bytes is smaller than the %llu required",
                     (unsigned long long)io->workspace_bytes, (unsigned long long)need.total);
  if (reinterpret_cast<uintptr_t>(io->workspace) & 255) return set_error(LTXB_EINVAL, "workspace must be 256-byte aligned");
  const DenoiseWs w = denoise_layout(core, blocks[0], cfg, static_cast<uint8_t*>(io->workspace));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int T = cfg->T, K = cfg->K;
  ltxb_block_io bio{};
  bio.x = w.x;
  bio.out = w.x;  // the block allows out == x
  bio.tstab = w.ts9;
  bio.tidx = io->tidx;
  bio.ctx = io->ctx;
  bio.pts2 = w.pts2;
  bio.cos = io->cos;
  bio.sin = io->sin;
  bio.workspace = w.block;
  bio.workspace_bytes = w.block_bytes;
  int rc;
  for (int s = 0; s < n_steps; ++s) {
    const float sigma = sigmas[s], sigma_next = sigmas[s + 1];
    // conditioning: per-token ts, per-mask-value t_k (the same f32 products)
    if ((rc = ltxb_sched_timesteps(io->mask, T, sigma, w.ts, st))) return rc;
    if ((rc = ltxb_sched_timesteps(io->mask_values, K, sigma, w.tk, st))) return rc;
    fill_kernel<<<1, 32, 0, st>>>(w.sig, 1, sigma);  // sigma as a device scalar for pts2
    launched();
    if ((rc = ltxb_core_adaln(core, w.tk, K, w.emb, w.ts9, w.core, w.core_bytes, st))) return rc;
    if ((rc = ltxb_core_pts2(core, w.sig, w.pts2, w.core, w.core_bytes, st))) return rc;
    if ((rc = ltxb_core_patchify(core, io->latent, T, w.x, st))) return rc;
    for (int b = 0; b < n_blocks; ++b)
      if ((rc = ltxb_block_forward(blocks[b], &bio, cfg, st))) return rc;
    if ((rc = ltxb_core_tail(core, w.x, w.emb, K, io->tidx, T, w.vel, w.core, w.core_bytes, st))) return rc;
    if ((rc = ltxb_sched_step(io->latent, w.vel, w.ts, io->clean, io->mask, T, 128, sigma, sigma_next, io->latent, st)))
      return rc;
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "denoise loop");
}

}  // extern "C"
