// Flash attention on tcgen05 for 128-dim heads: the blockwise online softmax
// of the reference's whileSdpa (ltx/block.zig:105-154) and the dense
// zml.nn.sdpa it agrees with (ltx/block.zig:234, gate ltx/block_conformance.zig:406).
//
// CTA = one 128-row query tile of one head, 256 threads:
//   warp 0      TMA producer: Q once, then K_j / V_j tiles (128 x 128) into a
//               2-stage ring (separate K and V barriers)
//   warp 1      TMEM owner + single-thread MMA issuer:
//                 S_j = Q K_j^T  -> TMEM (two S buffers, 128 columns each)
//                 O  += P_j V_j  -> TMEM (128 columns), P_j from shared memory
//   warps 4..7  softmax: thread i owns query row i (TMEM lane i); reads S_j,
//               keeps (m, l) in log2 units, writes P_j (bf16, 128B-swizzled
//               K-major) and, only when a row max grows by more than 2^8,
//               rescales that warp's O rows in TMEM; finally normalises O and
//               applies the per-head gate (2*sigmoid logits) in the epilogue.
//   warps 2..3  idle (keep the softmax warps on TMEM lane quarters 0..3)
//
// K/V rows past Tkv are zero-filled by TMA and masked to -inf before the
// softmax; query rows past Tq are computed and dropped.
//
// Ring attention: with MERGE, the kernel processes one K/V shard and merges
// its (m, l, O) into an f32 running state instead of writing the output.
#include "common.cuh"
#include "kernels.h"

namespace ltxb {

constexpr int AT_BM = 128, AT_BN = 128, AT_D = 128;
constexpr int AT_STAGES = 2;
constexpr int AT_TILE = AT_BM * AT_D * 2;  // 32 KB: one 128 x 128 bf16 tile (two 64-col halves)
constexpr int AT_HALF = AT_TILE / 2;
constexpr int AT_SMEM = 1024 + AT_TILE /*Q*/ + 2 * AT_STAGES * AT_TILE /*K,V*/ + AT_TILE /*P*/ + 256;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale only when the max grows by > 2^8

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <bool MERGE>
__global__ void __launch_bounds__(256, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const AttnArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + AT_TILE;
  uint8_t* sV = sK + AT_STAGES * AT_TILE;
  uint8_t* sP = sV + AT_STAGES * AT_TILE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + AT_TILE);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;              // [2]
  uint64_t* v_full = bars + 3;              // [2]
  uint64_t* kv_empty = bars + 5;            // [2]
  uint64_t* s_full = bars + 7;              // [2]
  uint64_t* s_free = bars + 9;              // [2]
  uint64_t* p_full = bars + 11;
  uint64_t* pv_done = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);

  const int warp = warp_id(), lane = lane_id();
  const int q0 = blockIdx.x * AT_BM, h = blockIdx.y;
  const int H = args.H, Tq = args.Tq, Tkv = args.Tkv;
  const int nkv = (Tkv + AT_BN - 1) / AT_BN;
  const int col0 = h * AT_D;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(pv_done, 1);
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS0 = tmem, tO = tmem + 256;

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, AT_TILE);
      tma_load_2d(sQ, &tmQ, q_full, col0, q0);
      tma_load_2d(sQ + AT_HALF, &tmQ, q_full, col0 + 64, q0);
      for (int j = 0; j < nkv; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&kv_empty[st], ph ^ 1, 0x201)) goto done;
        uint8_t* k = sK + st * AT_TILE;
        uint8_t* v = sV + st * AT_TILE;
        mbar_arrive_expect_tx(&k_full[st], AT_TILE);
        tma_load_2d(k, &tmK, &k_full[st], col0, j * AT_BN);
        tma_load_2d(k + AT_HALF, &tmK, &k_full[st], col0 + 64, j * AT_BN);
        mbar_arrive_expect_tx(&v_full[st], AT_TILE);
        tma_load_2d(v, &tmV, &v_full[st], col0, j * AT_BN);
        tma_load_2d(v + AT_HALF, &tmV, &v_full[st], col0 + 64, j * AT_BN);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(AT_BM, AT_BN, 0, 0);
      constexpr uint32_t idesc_o = idesc_bf16_f32(AT_BM, AT_D, 0, 1);
      const uint32_t qa = smem_u32(sQ);
      if (!mbar_wait(q_full, 0, 0x202)) goto done;
      // S_0
      if (!mbar_wait(&k_full[0], 0, 0x203)) goto done;
      tc_fence_after();
      {
        const uint32_t ka = smem_u32(sK);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * AT_HALF + (kk & 3) * 32;
          umma_ss(tS0, sdesc_kmajor_sw128(qa + off), sdesc_kmajor_sw128(ka + off), idesc_s, kk > 0);
        }
        umma_commit(&s_full[0]);
      }
      for (int j = 0; j < nkv; ++j) {
        const int st = j & 1;
        if (j + 1 < nkv) {
          const int sn = (j + 1) & 1;
          const uint32_t use = (uint32_t)((j + 1) >> 1);  // uses of S buffer sn so far
          if (!mbar_wait(&s_free[sn], (use & 1) ^ 1, 0x204)) goto done;
          if (!mbar_wait(&k_full[sn], ((j + 1) >> 1) & 1, 0x205)) goto done;
          tc_fence_after();
          const uint32_t ka = smem_u32(sK + sn * AT_TILE);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = (kk >> 2) * AT_HALF + (kk & 3) * 32;
            umma_ss(tS0 + sn * AT_BN, sdesc_kmajor_sw128(qa + off), sdesc_kmajor_sw128(ka + off), idesc_s, kk > 0);
          }
          umma_commit(&s_full[sn]);
        }
        if (!mbar_wait(p_full, j & 1, 0x206)) goto done;
        if (!mbar_wait(&v_full[st], (j >> 1) & 1, 0x207)) goto done;
        tc_fence_after();
        const uint32_t pa = smem_u32(sP), va = smem_u32(sV + st * AT_TILE);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t adesc = sdesc_kmajor_sw128(pa + (kk >> 2) * AT_HALF + (kk & 3) * 32);
          const uint64_t bdesc = sdesc_mnmajor_sw128(va + kk * 2048, AT_HALF);
          umma_ss(tO, adesc, bdesc, idesc_o, (j | kk) != 0);
        }
        umma_commit(pv_done);
        umma_commit(&kv_empty[st]);
      }
    }
  } else if (warp >= 4) {
    // ---------------- softmax / correction / epilogue ----------------
    const int qw = warp & 3;
    const int r = qw * 32 + lane;                  // row within the tile == TMEM lane
    const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
    const float c = args.scale * 1.4426950408889634f;  // scores -> log2 units
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv && ok; ++j) {
      const int sb = j & 1;
      if (!warp_wait(&s_full[sb], (j >> 1) & 1, 0x208)) { ok = false; break; }
      tc_fence_after();
      float s[128];
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t u[32];
        tmem_ld32(tS0 + sb * AT_BN + lane_off + cc * 32, u);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) s[cc * 32 + e] = __uint_as_float(u[e]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[sb]);
      const int valid = Tkv - j * AT_BN;  // columns < valid are real keys
      float mx = -INFINITY;
#pragma unroll
      for (int e = 0; e < 128; ++e) {
        s[e] = (e < valid) ? s[e] * c : -INFINITY;
        mx = fmaxf(mx, s[e]);
      }
      // previous P_{j-1} must be consumed (and O_{j-1} final) before we touch
      // the P buffer or O
      if (j > 0 && !warp_wait(pv_done, (j - 1) & 1, 0x209)) { ok = false; break; }
      const bool need = mx > m_ref + kRescaleThreshold;
      if (j == 0) {
        m_ref = mx;
      } else if (__any_sync(0xffffffffu, need)) {
        const float m_new = need ? mx : m_ref;
        const float corr = ex2(m_ref - m_new);
        l *= corr;
        m_ref = m_new;
        tc_fence_after();
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t u[32];
          tmem_ld32(tO + lane_off + cc * 32, u);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) u[e] = __float_as_uint(__uint_as_float(u[e]) * corr);
          tmem_st32(tO + lane_off + cc * 32, u);
        }
        tmem_wait_st();
      }
      float sum = 0.f;
      uint8_t* prow = sP + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
      for (int ch = 0; ch < 16; ++ch) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p0 = ex2(s[ch * 8 + 2 * e] - m_ref);
          const float p1 = ex2(s[ch * 8 + 2 * e + 1] - m_ref);
          sum += p0 + p1;
          w[e] = pack_bf16x2(p0, p1);
        }
        const int half = ch >> 3, lc = ch & 7;
        *reinterpret_cast<uint4*>(prow + half * AT_HALF + ((lc ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      l += sum;
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    // ---------------- epilogue ----------------
    if (ok && warp_wait(pv_done, (nkv - 1) & 1, 0x20A)) {
      tc_fence_after();
      const int row = q0 + r;
      const bool row_ok = row < Tq;
      const size_t obase = ((size_t)row * H + h) * AT_D;
      if (!MERGE) {
        const float g = (row_ok && args.gate) ? args.gate[(size_t)row * args.ldg + h] : 1.0f;
        const float inv = g / l;
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t u[32];
          tmem_ld32(tO + lane_off + cc * 32, u);
          tmem_wait_ld();
          if (row_ok) {
            uint4* op = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(args.out) + obase + cc * 32);
#pragma unroll
            for (int e = 0; e < 4; ++e)
              op[e] = make_uint4(pack_bf16x2(__uint_as_float(u[8 * e + 0]) * inv, __uint_as_float(u[8 * e + 1]) * inv),
                                 pack_bf16x2(__uint_as_float(u[8 * e + 2]) * inv, __uint_as_float(u[8 * e + 3]) * inv),
                                 pack_bf16x2(__uint_as_float(u[8 * e + 4]) * inv, __uint_as_float(u[8 * e + 5]) * inv),
                                 pack_bf16x2(__uint_as_float(u[8 * e + 6]) * inv, __uint_as_float(u[8 * e + 7]) * inv));
          }
        }
      } else {
        // merge (m_ref, l, O) into the running state (m, l in log2 units)
        float a = 0.f, b = 1.f;
        const size_t si = (size_t)h * Tq + row;
        if (row_ok) {
          if (args.first) {
            args.m_state[si] = m_ref;
            args.l_state[si] = l;
          } else {
            const float ms = args.m_state[si], ls = args.l_state[si];
            const float mn = fmaxf(ms, m_ref);
            a = ex2(ms - mn);
            b = ex2(m_ref - mn);
            args.m_state[si] = mn;
            args.l_state[si] = ls * a + l * b;
          }
        }
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t u[32];
          tmem_ld32(tO + lane_off + cc * 32, u);
          tmem_wait_ld();
          if (row_ok) {
            float4* op = reinterpret_cast<float4*>(args.o_acc + obase + cc * 32);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              float4 o = make_float4(__uint_as_float(u[4 * e]) * b, __uint_as_float(u[4 * e + 1]) * b,
                                     __uint_as_float(u[4 * e + 2]) * b, __uint_as_float(u[4 * e + 3]) * b);
              if (!args.first) {
                const float4 pv = op[e];
                o.x = fmaf(pv.x, a, o.x);
                o.y = fmaf(pv.y, a, o.y);
                o.z = fmaf(pv.z, a, o.z);
                o.w = fmaf(pv.w, a, o.w);
              }
              op[e] = o;
            }
          }
        }
      }
    }
  }
done:
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// out = o_acc / l * gate (bf16), after the last ring step
__global__ void attn_finalize_kernel(const float* __restrict__ o_acc, const float* __restrict__ l_state,
                                     const float* __restrict__ gate, int ldg, int Tq, int H,
                                     __nv_bfloat16* __restrict__ out) {
  const size_t n = (size_t)Tq * H * (AT_D / 8);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t e0 = i * 8;
    const int row = (int)(e0 / ((size_t)H * AT_D));
    const int h = (int)((e0 / AT_D) % H);
    const float g = gate ? gate[(size_t)row * ldg + h] : 1.0f;
    const float inv = g / l_state[(size_t)h * Tq + row];
    const float4 a = reinterpret_cast<const float4*>(o_acc + e0)[0];
    const float4 b = reinterpret_cast<const float4*>(o_acc + e0)[1];
    reinterpret_cast<uint4*>(out + e0)[0] = make_uint4(pack_bf16x2(a.x * inv, a.y * inv), pack_bf16x2(a.z * inv, a.w * inv),
                                                       pack_bf16x2(b.x * inv, b.y * inv), pack_bf16x2(b.z * inv, b.w * inv));
  }
}

template <bool MERGE>
static int launch_attn(const AttnArgs& a, cudaStream_t st) {
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<MERGE>, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM);
    if (e != cudaSuccess) return set_cuda_error(e, "attention: cudaFuncSetAttribute");
    attr[dev & 63] = true;
  }
  const int w = a.H * AT_D;
  CUtensorMap tq, tk, tv;
  int rc = make_tmap_2d(&tq, a.q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, a.Tq, a.ldq, 64, AT_BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = make_tmap_2d(&tk, a.k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, a.Tkv, a.ldk, 64, AT_BN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = make_tmap_2d(&tv, a.v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, a.Tkv, a.ldv, 64, AT_BN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  dim3 grid((a.Tq + AT_BM - 1) / AT_BM, a.H);
  attn_tc_kernel<MERGE><<<grid, 256, AT_SMEM, st>>>(tq, tk, tv, a);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "attention launch");
}

int attention_tc(const AttnArgs& a, cudaStream_t st) {
  if (a.Tq <= 0) return LTXB_OK;
  if (a.Tkv <= 0) return set_error(LTXB_EINVAL, "attention: empty K/V");
  if (a.H <= 0) return set_error(LTXB_EINVAL, "attention: H must be positive");
  if ((reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) | reinterpret_cast<uintptr_t>(a.v) |
       reinterpret_cast<uintptr_t>(a.out)) & 15)
    return set_error(LTXB_EINVAL, "attention: q/k/v/out must be 16-byte aligned");
  if (a.o_acc) return launch_attn<true>(a, st);
  return launch_attn<false>(a, st);
}

int attention_finalize(const AttnArgs& a, cudaStream_t st) {
  const size_t n = (size_t)a.Tq * a.H * (AT_D / 8);
  if (n == 0) return LTXB_OK;
  int grid = (int)((n + 255) / 256);
  if (grid > 8 * sm_count()) grid = 8 * sm_count();
  attn_finalize_kernel<<<grid, 256, 0, st>>>(a.o_acc, a.l_state, a.gate, a.ldg, a.Tq, a.H,
                                             reinterpret_cast<__nv_bfloat16*>(a.out));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "attention finalize");
}

}  // namespace ltxb
