// Flash attention on tcgen05 for 128-dim heads: the blockwise online softmax
// of the reference's whileSdpa (ltx/block.zig:105-154) and the dense
// zml.nn.sdpa it agrees with (ltx/block.zig:234, gate ltx/block_conformance.zig:406).
//
// CTA = two 128-row query tiles (A, B) of one head sharing every K/V tile,
// 576 threads:
//   warps 0..7   softmax of tile A: query row i lives in TMEM lane i and is
//                served by two warps, one per 64-column half of the scores
//   warps 8..15  softmax of tile B
//   warp 16      TMA producer: Q_A, Q_B once, then K_j / V_j (128 x 128 bf16)
//                into a 2-stage ring with separate K and V barriers
//   warp 17      TMEM owner + tcgen05.mma issuer (one elected lane)
// TMEM (512 columns): S_A [0,128) S_B [128,256) O_A [256,384) O_B [384,512).
// The softmax writes P_X (bf16 pairs) back over the first 64 columns of S_X,
// and O_X += P_X V_j reads its A operand straight from TMEM.
//
// MMA issue order: S_A0 S_B0 | PV_A0 S_A1 | PV_B0 S_B1 | PV_A1 S_A2 | ...
// so the softmax of one tile runs while the tensor core works on the other.
// tcgen05 MMAs from one thread complete in order, so the commit that
// signals S_X(j) also covers PV_X(j-1): once S_X(j) is visible, P_X(j-1)'s
// columns and O_X are free to overwrite / rescale.
//
// Softmax per row: scores in log2 units, a running reference max that only
// moves (with an O rescale in TMEM) when the tile max exceeds it by more than
// 2^8, exp2 split between the MUFU unit and a degree-3 polynomial on the FMA
// pipe (1 of 8 pairs), row sums in f32; the per-pair arithmetic uses the
// two-wide f32 instructions (fma/add .f32x2, 3-input max). The two warps of a
// row exchange their partial maxima once per K/V tile; the first 32 columns
// of P are computed with the current reference max while that exchange
// completes (and redone from S in the rare rescale case), then handed to the
// MMA warp on their own (p_half) so PV starts before the second half is done.
// K/V rows past Tkv are zero-filled by TMA and masked; query rows past Tq are
// computed and dropped.
//
// MERGE: the kernel writes an f32 (m, l, O) state instead of the output --
// one state per K/V range with split-K/V (grid z = kv_splits), or merged
// into a running state across the shards of the ring alternative of
// sequence parallelism; attn_combine_kernel turns the states into the output.
#define LTXB_LOCAL_STATUS 1  // whole-program device code (no -rdc): own status word
#include <atomic>

#include "common.cuh"
#include "kernels.h"

namespace ltxb {

constexpr int AT_BM = 128, AT_BN = 128, AT_D = 128;
constexpr int AT_STAGES = 2;
constexpr int AT_TILE = AT_BM * AT_D * 2;  // 32 KB: one 128 x 128 bf16 tile (two 64-col halves)
constexpr int AT_HALF = AT_TILE / 2;
constexpr int AT_THREADS = 576;  // 16 softmax warps + TMA warp + MMA warp
constexpr int AT_SMEM = 1024 + 2 * AT_TILE /*Q_A,Q_B*/ + 2 * AT_STAGES * AT_TILE /*K,V*/ + 256 +
                        (2 * 2 * 2 + 2 * 2) * AT_BM * 4 /*row-max (x2 buffers) and row-sum exchange*/;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale only when the max grows by > 2^8

// How many of the 16 exponential pairs of a 32-column chunk run as the
// polynomial on the FMA pipe (the rest on MUFU), spread evenly over the
// chunk. A build-time parameter: the best split depends on whether the
// kernel runs at full clock or at the board's power limit.
#ifndef LTXB_EXP_POLY_PAIRS
#define LTXB_EXP_POLY_PAIRS 2
#endif
// bit e set: pair e of the chunk on the polynomial (1, 2, 3, 4, 6, 8 or 16 pairs)
__host__ __device__ constexpr uint32_t poly_pair_mask(int n) {
  return n <= 0 ? 0u
       : n == 1 ? 0x0020u
       : n == 2 ? 0x2020u
       : n == 3 ? 0x2084u
       : n == 4 ? 0x2222u
       : n == 6 ? 0x2A2Au
       : n == 8 ? 0xAAAAu
                : 0xFFFFu;
}
constexpr uint32_t kPolyMask = poly_pair_mask(LTXB_EXP_POLY_PAIRS);

__device__ __forceinline__ float ex2_mufu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA pipe: x = n + f with n = rint(x) (via the 1.5 * 2^23
// rounding constant), f in [-1/2, 1/2]; 2^f by a degree-3 polynomial fitted by
// least squares on Chebyshev nodes of [-1/2, 1/2] (max relative error
// 7.8e-5); 2^n is added to the exponent field. x is clamped to >= -120, which
// keeps the exponent arithmetic in range (2^-120 is negligible next to a
// row sum >= 1).
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -120.0f);
  const float magic = 12582912.0f;  // 1.5 * 2^23
  const float t = x + magic;
  const float n = t - magic;
  const float f = x - n;
  float p = fmaf(0.05508868396282196f, f, 0.24260404706001282f);
  p = fmaf(p, f, 0.6932762265205383f);
  p = fmaf(p, f, 0.9999289512634277f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// Two-wide f32 SIMD (sm_100 `*.f32x2`) on register pairs.
__device__ __forceinline__ uint64_t pk2(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void up2(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// MMA issue with the shared-memory descriptors passed as their low words: the
// high word of every 128-byte-swizzle descriptor here is the same constant
// (SBO 1024 B, descriptor version 1, layout SWIZZLE_128B), and the low word
// (start address >> 4, LBO) is stepped by plain 32-bit adds.
constexpr uint32_t kDescHi = (1024u >> 4) | (1u << 14) | (2u << 29);
__device__ __forceinline__ uint32_t desc_lo(uint32_t saddr, uint32_t lbo_field) {
  return ((saddr >> 4) & 0x3FFFu) | (lbo_field << 16);
}
__device__ __forceinline__ void mma_ss_lo(uint32_t d, uint32_t alo, uint32_t blo, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .b64 da, db;\n\t.reg .pred p;\n\t"
      "mov.b64 da, {%1, %5};\n\tmov.b64 db, {%2, %5};\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, p;\n\t}" ::"r"(d),
      "r"(alo), "r"(blo), "r"(idesc), "r"(acc), "r"(kDescHi)
      : "memory");
}
__device__ __forceinline__ void mma_ts_lo(uint32_t d, uint32_t a_tmem, uint32_t blo, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .b64 db;\n\t.reg .pred p;\n\t"
      "mov.b64 db, {%2, %5};\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %3, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "r"(blo), "r"(idesc), "r"(acc), "r"(kDescHi)
      : "memory");
}

// ex2_poly for a pair, the range reduction and polynomial in f32x2.
__device__ __forceinline__ void ex2_poly2(float x0, float x1, float& p0, float& p1) {
  x0 = fmaxf(x0, -120.0f);
  x1 = fmaxf(x1, -120.0f);
  const uint64_t x2 = pk2(x0, x1);
  const uint64_t t2 = add2(x2, pk2(12582912.0f, 12582912.0f));
  const uint64_t n2 = add2(t2, pk2(-12582912.0f, -12582912.0f));
  const uint64_t f2 = fma2(n2, pk2(-1.0f, -1.0f), x2);
  uint64_t q2 = fma2(pk2(0.05508868396282196f, 0.05508868396282196f), f2,
                     pk2(0.24260404706001282f, 0.24260404706001282f));
  q2 = fma2(q2, f2, pk2(0.6932762265205383f, 0.6932762265205383f));
  q2 = fma2(q2, f2, pk2(0.9999289512634277f, 0.9999289512634277f));
  float t0, t1;
  up2(q2, p0, p1);
  up2(t2, t0, t1);
  p0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  p1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}

template <bool MERGE>
__global__ void __launch_bounds__(AT_THREADS, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const AttnArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                        // Q_A, Q_B
  uint8_t* sK = sQ + 2 * AT_TILE;            // [stage]
  uint8_t* sV = sK + AT_STAGES * AT_TILE;    // [stage]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + AT_STAGES * AT_TILE);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* v_full = bars + 3;    // [2]
  uint64_t* k_empty = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;    // [tile]
  uint64_t* p_full = bars + 11;   // [tile]
  uint64_t* o_done = bars + 13;   // [tile]
  uint64_t* p_half = bars + 15;   // [tile]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  float* xmax = reinterpret_cast<float*>(bars + 32);  // [2 bufs][2 tiles][2 halves][128]
  float* xsum = xmax + 2 * 2 * 2 * AT_BM;             // [2 tiles][2 halves][128]

  const int warp = warp_id(), lane = lane_id();
  const int q0 = blockIdx.x * (2 * AT_BM), h = blockIdx.y;
  const int H = args.H, Tq = args.Tq, Tkv = args.Tkv;
  const size_t ldo = args.ldo > 0 ? (size_t)args.ldo : (size_t)H * AT_D;  // output row stride (elements)
  // this CTA's K/V tiles: [t0, t0 + nkv) of the nkv_all tiles (one split of
  // kv_splits; the whole range without splitting)
  const int nkv_all = (Tkv + AT_BN - 1) / AT_BN;
  const int nsplit = MERGE && args.kv_splits > 1 ? args.kv_splits : 1;
  const int t0 = (int)(((long long)blockIdx.z * nkv_all) / nsplit);
  const int nkv = (int)(((long long)(blockIdx.z + 1) * nkv_all) / nsplit) - t0;
  // Each CTA walks the K/V tiles starting from its own offset (step i reads
  // tile (i + kv0) mod nkv): the CTAs resident at one time then stream
  // different tiles instead of all requesting the same lines of L2 at once.
  // Online softmax is order-independent; the order is fixed per CTA, so
  // results stay deterministic.
  const int kv0 = (int)(((long long)blockIdx.x * nkv) / gridDim.x);
  auto kv_tile = [&](int i) { const int t = i + kv0; return t0 + (t >= nkv ? t - nkv : t); };
  const int col0 = h * AT_D;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 8);
      mbar_init(&p_half[i], 8);
      mbar_init(&o_done[i], 1);
    }
    fence_mbar_init();
  }
  if (warp == 16 && lane == 0) {
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 17) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Warps 16 and 17 run their loops with all 32 lanes (warp-uniform control
  // flow and operands, so descriptors and addresses stay in uniform
  // registers) and let one elected lane issue each copy / MMA / commit.
  if (warp == 16) {
    // ---------------- TMA producer ----------------
    if (elect_one()) {
      mbar_arrive_expect_tx(q_full, 2 * AT_TILE);
      tma_load_2d(sQ, &tmQ, q_full, col0, q0);
      tma_load_2d(sQ + AT_HALF, &tmQ, q_full, col0 + 64, q0);
      tma_load_2d(sQ + AT_TILE, &tmQ, q_full, col0, q0 + AT_BM);
      tma_load_2d(sQ + AT_TILE + AT_HALF, &tmQ, q_full, col0 + 64, q0 + AT_BM);
    }
    __syncwarp();
    for (int j = 0; j < nkv; ++j) {
      // K_j and V_j have separate free signals: K's stage frees once both
      // S MMAs of step j-2 are done, V's once both PV MMAs are, so each
      // load starts about one and a half steps before its first use.
      const int st = j & 1;
      uint8_t* k = sK + st * AT_TILE;
      uint8_t* v = sV + st * AT_TILE;
      const int krow = kv_tile(j) * AT_BN;
      if (!warp_wait(&k_empty[st], ((j >> 1) & 1) ^ 1, 0x201)) goto done;
      if (elect_one()) {
        mbar_arrive_expect_tx(&k_full[st], AT_TILE);
        tma_load_2d(k, &tmK, &k_full[st], col0, krow);
        tma_load_2d(k + AT_HALF, &tmK, &k_full[st], col0 + 64, krow);
      }
      __syncwarp();
      if (!warp_wait(&v_empty[st], ((j >> 1) & 1) ^ 1, 0x20a)) goto done;
      if (elect_one()) {
        mbar_arrive_expect_tx(&v_full[st], AT_TILE);
        tma_load_2d(v, &tmV, &v_full[st], col0, krow);
        tma_load_2d(v + AT_HALF, &tmV, &v_full[st], col0 + 64, krow);
      }
      __syncwarp();
    }
  } else if (warp == 17) {
    // ---------------- MMA issuer ----------------
    constexpr uint32_t idesc_s = idesc_bf16_f32(AT_BM, AT_BN, 0, 0);
    constexpr uint32_t idesc_o = idesc_bf16_f32(AT_BM, AT_D, 0, 1);
    const uint32_t qa = smem_u32(sQ);
    auto issue_s = [&](int tile, int j) {
      const uint32_t klo = desc_lo(smem_u32(sK + (j & 1) * AT_TILE), 1);
      const uint32_t qlo = desc_lo(qa + tile * AT_TILE, 1);
      const uint32_t d = tmem + tile * 128;
      if (elect_one()) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = ((kk >> 2) * AT_HALF + (kk & 3) * 32) >> 4;
          mma_ss_lo(d, qlo + off, klo + off, idesc_s, kk > 0);
        }
        umma_commit(&s_full[tile]);
      }
      __syncwarp();
    };
    // PV in two halves of the K (key) steps: part 0 = steps 0, 1, 4, 5 (the
    // P chunks the softmax warps hand over first), part 1 = steps 2, 3, 6, 7.
    auto issue_pv = [&](int tile, int j, int part) {
      const uint32_t vlo = desc_lo(smem_u32(sV + (j & 1) * AT_TILE), AT_HALF >> 4);
      const uint32_t d = tmem + 256 + tile * 128, pa = tmem + tile * 128;
      if (elect_one()) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int kk = (i & 1) + (i >> 1) * 4 + part * 2;
          mma_ts_lo(d, pa + kk * 8, vlo + kk * (2048 >> 4), idesc_o, (j | part | i) != 0);
        }
      }
      __syncwarp();
    };
    auto commit = [&](uint64_t* bar) {
      if (elect_one()) umma_commit(bar);
      __syncwarp();
    };
    if (!warp_wait(q_full, 0, 0x202)) goto done;
    if (!warp_wait(&k_full[0], 0, 0x203)) goto done;
    tc_fence_after();
    issue_s(0, 0);
    issue_s(1, 0);
    commit(&k_empty[0]);  // K_0 consumed by both S MMAs
    for (int j = 0; j < nkv; ++j) {
      const int st = j & 1;
      const bool more = j + 1 < nkv;
      // tile A: O_A += P_A V_j, then S_A(j+1)
      if (!warp_wait(&v_full[st], (j >> 1) & 1, 0x205)) goto done;  // normally long ready
      if (!warp_wait(&p_half[0], j & 1, 0x20b)) goto done;
      tc_fence_after();
      issue_pv(0, j, 0);
      if (!warp_wait(&p_full[0], j & 1, 0x204)) goto done;
      tc_fence_after();
      issue_pv(0, j, 1);
      if (more) {
        if (!warp_wait(&k_full[st ^ 1], ((j + 1) >> 1) & 1, 0x206)) goto done;
        tc_fence_after();
        issue_s(0, j + 1);
      } else {
        commit(&o_done[0]);
      }
      // tile B
      if (!warp_wait(&p_half[1], j & 1, 0x20c)) goto done;
      tc_fence_after();
      issue_pv(1, j, 0);
      if (!warp_wait(&p_full[1], j & 1, 0x207)) goto done;
      tc_fence_after();
      issue_pv(1, j, 1);
      commit(&v_empty[st]);  // V_j consumed by both PV MMAs
      if (more) {
        issue_s(1, j + 1);
        commit(&k_empty[st ^ 1]);  // K_{j+1} consumed by both S MMAs
      } else {
        commit(&o_done[1]);
      }
    }
  } else if (warp < 16) {
    // ---------------- softmax / correction / epilogue (warps 0..15) ----------------
    // Two warps per query row: warp w serves tile w / 8, TMEM lane quarter
    // w % 4 and score columns [64 hf, 64 hf + 64) with hf = (w / 4) % 2. The
    // pair exchanges its partial row maxima through shared memory once per
    // iteration (named barrier 1 + 4 tile + quarter, 64 threads), so both
    // halves move the reference max together.
    const int tile = warp >> 3;  // 0 = A, 1 = B
    const int hf = (warp >> 2) & 1;
    const int qw = warp & 3;
    const int r = qw * 32 + lane;
    const uint32_t bar_id = 1 + tile * 4 + qw;
    const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
    const uint32_t tS = tmem + tile * 128 + lane_off;
    const uint32_t tO = tmem + 256 + tile * 128 + lane_off + hf * 64;
    const float c = args.scale * 1.4426950408889634f;  // scores -> log2 units
    float m_ref = -INFINITY, l = 0.f;  // m_ref in log2 units, l over this warp's columns
    bool ok = true;
    auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory"); };
    // Every warp of a pair passes the same pair barriers (one per iteration,
    // one in the epilogue) even after a timed-out wait, so that a failure in
    // one warp can never leave its partner blocked on the named barrier.
    for (int j = 0; j < nkv; ++j) {
      if (ok && !warp_wait(&s_full[tile], j & 1, 0x208)) ok = false;
      float* xm = xmax + (((j & 1) * 2 + tile) * 2) * AT_BM;
      if (!ok) {
        xm[hf * AT_BM + r] = -INFINITY;
        pair_sync();
        continue;
      }
      tc_fence_after();
      uint32_t c0[32], c1[32];
      tmem_ld32(tS + hf * 64, c0);
      tmem_ld32(tS + hf * 64 + 32, c1);
      tmem_wait_ld();
      const int valid = Tkv - kv_tile(j) * AT_BN - hf * 64;  // this warp's columns < valid are real keys
      if (valid < 64) {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          if (e >= valid) c0[e] = __float_as_uint(-INFINITY);
          if (32 + e >= valid) c1[e] = __float_as_uint(-INFINITY);
        }
      }
      float m4[4] = {__uint_as_float(c0[0]), __uint_as_float(c0[1]), __uint_as_float(c1[0]), __uint_as_float(c1[1])};
#pragma unroll
      for (int e = 1; e < 16; ++e) {
        m4[(2 * e) & 3] = max3(m4[(2 * e) & 3], __uint_as_float(c0[2 * e]), __uint_as_float(c0[2 * e + 1]));
        m4[(2 * e + 1) & 3] = max3(m4[(2 * e + 1) & 3], __uint_as_float(c1[2 * e]), __uint_as_float(c1[2 * e + 1]));
      }
      const float pm = max3(m4[0], m4[1], fmaxf(m4[2], m4[3]));
      xm[hf * AT_BM + r] = pm;
      // p = 2^(s c - m) -> bf16 pairs over S columns [32 hf, 32 hf + 32)
      // (keys 64 hf .. 64 hf + 63). Chunk 0 (keys 64 hf .. 64 hf + 31) is
      // computed speculatively with the current reference max while the
      // pair's max exchange completes; only when the exchange asks for a
      // rescale (rare: the max grew by more than 2^8) is it recomputed. It is
      // handed to the MMA warp on its own (p_half), so the PV K-steps over
      // keys 0-31 and 64-95 run while chunk 1 is computed.
      const uint64_t c2 = pk2(c, c);
      uint64_t acc2[2];
      uint32_t pk[16];
      auto exp_chunk = [&](const uint32_t* cv) {
        const uint64_t nm2 = pk2(-m_ref, -m_ref);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float a0, a1, p0, p1;
          up2(fma2(pk2(__uint_as_float(cv[2 * e]), __uint_as_float(cv[2 * e + 1])), c2, nm2), a0, a1);
          // 1 of every 8 pairs on the FMA pipe (packed polynomial), the rest on
          // MUFU: the best balance measured under the board's power limit
          if ((kPolyMask >> e) & 1u) {
            ex2_poly2(a0, a1, p0, p1);
          } else {
            p0 = ex2_mufu(a0);
            p1 = ex2_mufu(a1);
          }
          acc2[e & 1] = add2(acc2[e & 1], pk2(p0, p1));
          pk[e] = pack_bf16x2(p0, p1);
        }
      };
      auto hand_over = [&](int ch) {
        tmem_st16(tS + hf * 32 + ch * 16, pk);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(ch == 0 ? &p_half[tile] : &p_full[tile]);
      };
      acc2[0] = acc2[1] = pk2(0.f, 0.f);
      exp_chunk(c0);  // speculative (at j = 0 always redone: m_ref is -inf)
      pair_sync();    // both halves' S loads are complete and their maxima published
      const float cm = fmaxf(pm, xm[(hf ^ 1) * AT_BM + r]) * c;
      const bool need = cm > m_ref + kRescaleThreshold;
      if (__any_sync(0xffffffffu, need)) {  // same rows in both warps: same branch
        const float m_new = need ? cm : m_ref;
        const float corr = ex2_mufu(m_ref - m_new);  // 0 on the first iteration
        m_ref = m_new;
        l *= corr;
        if (j > 0) {  // this warp's half of O (complete: S(j) committed after PV(j-1))
#pragma unroll 1
          for (int cc = 0; cc < 4; ++cc) {
            uint32_t u[16];
            tmem_ld16(tO + cc * 16, u);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) u[e] = __float_as_uint(__uint_as_float(u[e]) * corr);
            tmem_st16(tO + cc * 16, u);
          }
        }
        // redo chunk 0 from S, still intact in TMEM: no P of this pair is
        // stored before the exchange, and the partner's P never covers these
        // columns
        uint32_t r0[32];
        tmem_ld32(tS + hf * 64, r0);
        tmem_wait_ld();
        if (valid < 32) {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            if (e >= valid) r0[e] = __float_as_uint(-INFINITY);
        }
        acc2[0] = acc2[1] = pk2(0.f, 0.f);
        exp_chunk(r0);
      }
      hand_over(0);
      exp_chunk(c1);
      hand_over(1);
      {
        float s0, s1, s2, s3;
        up2(acc2[0], s0, s1);
        up2(acc2[1], s2, s3);
        l += (s0 + s1) + (s2 + s3);
      }
    }
    // ---------------- epilogue: this warp's 64 output columns ----------------
    const bool eok = ok && warp_wait(&o_done[tile], 0, 0x209);
    const int row = q0 + tile * AT_BM + r;
    const bool row_ok = row < Tq;
    // ring merge: both halves read the old (m, l) state before the pair
    // barrier, half 0 writes the new one after it
    float ms = 0.f, ls = 0.f;
    const size_t si = (size_t)blockIdx.z * H * Tq + (size_t)h * Tq + row;
    if (MERGE && eok && row_ok && !args.first) {
      ms = args.m_state[si];
      ls = args.l_state[si];
    }
    float* xs = xsum + tile * 2 * AT_BM;
    xs[hf * AT_BM + r] = l;
    pair_sync();
    if (eok) {
      tc_fence_after();
      const float lt = l + xs[(hf ^ 1) * AT_BM + r];  // full row sum
      const size_t obase = ((size_t)row * H + h) * AT_D + hf * 64;
      if (!MERGE) {
        const float g = (row_ok && args.gate) ? args.gate[(size_t)row * args.ldg + h] : 1.0f;
        const float inv = g / lt;
        // this row's output: here, or (peer exchange) in the window of the
        // rank that holds the row's token
        __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(args.out);
        size_t orow_off = (size_t)row * ldo;
        if (args.out_tab && row_ok) {
          const int p = row / args.peer_rows;
          orow = reinterpret_cast<__nv_bfloat16*>(args.out_tab[p]);
          orow_off = (size_t)(row - p * args.peer_rows) * ldo + args.out_col0;
        }
#pragma unroll 1
        for (int cc = 0; cc < 2; ++cc) {
          uint32_t u[32];
          tmem_ld32(tO + cc * 32, u);
          tmem_wait_ld();
          if (row_ok) {
            uint4* op = reinterpret_cast<uint4*>(orow + orow_off + h * AT_D + hf * 64 + cc * 32);
#pragma unroll
            for (int e = 0; e < 4; ++e)
              op[e] = make_uint4(pack_bf16x2(__uint_as_float(u[8 * e + 0]) * inv, __uint_as_float(u[8 * e + 1]) * inv),
                                 pack_bf16x2(__uint_as_float(u[8 * e + 2]) * inv, __uint_as_float(u[8 * e + 3]) * inv),
                                 pack_bf16x2(__uint_as_float(u[8 * e + 4]) * inv, __uint_as_float(u[8 * e + 5]) * inv),
                                 pack_bf16x2(__uint_as_float(u[8 * e + 6]) * inv, __uint_as_float(u[8 * e + 7]) * inv));
          }
        }
      } else {
        // merge (m_ref, lt, O) into the running state (m, l in log2 units)
        float a = 0.f, b = 1.f;
        if (row_ok) {
          if (args.first) {
            if (hf == 0) {
              args.m_state[si] = m_ref;
              args.l_state[si] = lt;
            }
          } else {
            const float mn = fmaxf(ms, m_ref);
            a = ex2_mufu(ms - mn);
            b = ex2_mufu(m_ref - mn);
            if (hf == 0) {
              args.m_state[si] = mn;
              args.l_state[si] = ls * a + lt * b;
            }
          }
        }
#pragma unroll 1
        for (int cc = 0; cc < 2; ++cc) {
          uint32_t u[32];
          tmem_ld32(tO + cc * 32, u);
          tmem_wait_ld();
          if (row_ok) {
            float4* op = reinterpret_cast<float4*>(args.o_acc + (size_t)blockIdx.z * Tq * H * AT_D + obase + cc * 32);
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
  if (warp == 17) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  // peer exchange: the last CTA tells every rank that its rows have landed
  // (also after a timed-out wait, so that no rank waits for this one in vain)
  if (!MERGE && args.sig_counter) last_cta_signal(args.sig_counter, args.sig_tab, args.sig_n, args.sig_epoch);
}

// out = sum_z O_z 2^(m_z - m) / sum_z l_z 2^(m_z - m) * gate (bf16), m = max_z m_z:
// the merge of `nsplit` partial states (m, l in log2 units), or with one state
// the normalisation after the last ring step.
__global__ void attn_combine_kernel(const float* __restrict__ o_acc, const float* __restrict__ m_state,
                                    const float* __restrict__ l_state, int nsplit, const float* __restrict__ gate,
                                    int ldg, int Tq, int H, __nv_bfloat16* __restrict__ out, size_t ldo) {
  const size_t n = (size_t)Tq * H * (AT_D / 8);
  const size_t ostride = (size_t)Tq * H * AT_D, sstride = (size_t)H * Tq;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t e0 = i * 8;
    const int row = (int)(e0 / ((size_t)H * AT_D));
    const int h = (int)((e0 / AT_D) % H);
    const size_t si = (size_t)h * Tq + row;
    float m = m_state[si];
    for (int z = 1; z < nsplit; ++z) m = fmaxf(m, m_state[z * sstride + si]);
    float l = 0.f, o[8] = {};
    for (int z = 0; z < nsplit; ++z) {
      const float w = nsplit > 1 ? ex2_mufu(m_state[z * sstride + si] - m) : 1.0f;
      l = fmaf(l_state[z * sstride + si], w, l);
      const float4 a = reinterpret_cast<const float4*>(o_acc + z * ostride + e0)[0];
      const float4 b = reinterpret_cast<const float4*>(o_acc + z * ostride + e0)[1];
      o[0] = fmaf(a.x, w, o[0]); o[1] = fmaf(a.y, w, o[1]); o[2] = fmaf(a.z, w, o[2]); o[3] = fmaf(a.w, w, o[3]);
      o[4] = fmaf(b.x, w, o[4]); o[5] = fmaf(b.y, w, o[5]); o[6] = fmaf(b.z, w, o[6]); o[7] = fmaf(b.w, w, o[7]);
    }
    const float g = gate ? gate[(size_t)row * ldg + h] : 1.0f;
    const float inv = g / l;
    reinterpret_cast<uint4*>(out + (size_t)row * ldo + (e0 - (size_t)row * H * AT_D))[0] = make_uint4(pack_bf16x2(o[0] * inv, o[1] * inv), pack_bf16x2(o[2] * inv, o[3] * inv),
                                                       pack_bf16x2(o[4] * inv, o[5] * inv), pack_bf16x2(o[6] * inv, o[7] * inv));
  }
}

template <bool MERGE>
static int launch_attn(const AttnArgs& a, cudaStream_t st) {
  static std::atomic<bool> attr[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return set_error(LTXB_EINVAL, "attention: device %d out of range", dev);
  if (!attr[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel<MERGE>, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_SMEM);
    if (e != cudaSuccess) return set_cuda_error(e, "attention: cudaFuncSetAttribute");
    attr[dev].store(true, std::memory_order_release);
  }
  const int w = a.H * AT_D;
  CUtensorMap tq, tk, tv;
  int rc = make_tmap_2d(&tq, a.q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, a.Tq, a.ldq, 64, AT_BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = make_tmap_2d(&tk, a.k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, a.Tkv, a.ldk, 64, AT_BN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (!rc) rc = make_tmap_2d(&tv, a.v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, a.Tkv, a.ldv, 64, AT_BN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  dim3 grid((a.Tq + 2 * AT_BM - 1) / (2 * AT_BM), a.H, MERGE && a.kv_splits > 1 ? a.kv_splits : 1);
  attn_tc_kernel<MERGE><<<grid, AT_THREADS, AT_SMEM, st>>>(tq, tk, tv, a);
  launched();
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

cudaError_t attn_status(uint32_t* v, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(v, g_status, sizeof(*v));
  if (e == cudaSuccess && clear && *v) {
    const uint32_t z = 0;
    e = cudaMemcpyToSymbol(g_status, &z, sizeof(z));
  }
  return e;
}

int attention_combine(const AttnArgs& a, cudaStream_t st) {
  const size_t n = (size_t)a.Tq * a.H * (AT_D / 8);
  if (n == 0) return LTXB_OK;
  int grid = (int)((n + 255) / 256);
  if (grid > 8 * sm_count()) grid = 8 * sm_count();
  attn_combine_kernel<<<grid, 256, 0, st>>>(a.o_acc, a.m_state, a.l_state, a.kv_splits > 1 ? a.kv_splits : 1, a.gate,
                                            a.ldg, a.Tq, a.H, reinterpret_cast<__nv_bfloat16*>(a.out),
                                            a.ldo > 0 ? (size_t)a.ldo : (size_t)a.H * AT_D);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "attention combine");
}

int attention_kv_splits(int Tq, int Tkv, int H, int max_splits) {
  // time ~ waves x tiles per split; a split adds one partial state to write
  // and read back (about 3 % of a tile-sweep per split here)
  const long long units = (long long)((Tq + 2 * AT_BM - 1) / (2 * AT_BM)) * H;
  const int nkv = (Tkv + AT_BN - 1) / AT_BN, sms = sm_count();
  int best = 1;
  double best_t = 0;
  for (int s = 1; s <= max_splits && s <= nkv; ++s) {
    const double waves = (double)((units * s + sms - 1) / sms);
    const double t = waves * ((nkv + s - 1) / s) * (1.0 + 0.03 * (s - 1));
    if (s == 1 || t < best_t) {
      best = s;
      best_t = t;
    }
  }
  return best;
}

int attention_split(AttnArgs a, int splits, cudaStream_t st) {
  if (splits <= 1) {  // one range: the direct kernel writes the output itself
    a.o_acc = a.m_state = a.l_state = nullptr;
    a.kv_splits = 0;
    return attention_tc(a, st);
  }
  if (!a.o_acc || !a.m_state || !a.l_state) return set_error(LTXB_EINVAL, "attention split: state buffers missing");
  a.kv_splits = splits;
  a.first = 1;
  int rc = attention_tc(a, st);
  if (rc) return rc;
  return attention_combine(a, st);
}

}  // namespace ltxb
