// tcgen05 GEMM for the block's linears: D[M, N] = A[M, K] . B[N, K]^T with
// bf16 A (activations, token-major) and B either bf16 or int8 + grouped-128
// scales (weights, [out, in] row-major as stored in the checkpoint), f32
// accumulation in TMEM, and the block's elementwise tails fused into the
// epilogue (bias, q/k-norm sum of squares, GELU, 2*sigmoid gate, gated f32
// residual).
//
// Replaces the reference's `lin` / `linQ` (ltx/block.zig:22-26, :462-477),
// which upcast the weights to f32 per call and run f32 dots.
//
// Structure (one CTA per SM, persistent over output tiles 128 x BN):
//   warp 0      TMA producer: A tile [128 x 64] and B tile [BN x 64] per stage
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..5  epilogue: tcgen05.ld of the accumulator, fused tail, stores
//   warps 6..9  (int8 B only) dequantisers: int8 tile + per-group scale ->
//               bf16 tile in the 128B-swizzled K-major layout the MMA reads
// Two TMEM accumulators (2 x BN columns) let the epilogue of tile i overlap
// the main loop of tile i+1.
#include <atomic>

#include "common.cuh"
#include "kernels.h"

namespace ltxb {

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_GROUP_M = 16;  // M tiles walked together for L2 reuse

// XBUF: the gated-residual epilogue's two [128 x 32] f32 chunk buffers (the
// residual input arrives there by TMA, the output leaves by TMA store).
template <int BN, bool BQ8, bool XBUF = false>
struct GemmCfg {
  static constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;   // 16 KB
  static constexpr int B_BYTES = BN * GEMM_BK * 2;        // bf16 tile
  static constexpr int BQ_BYTES = BQ8 ? BN * GEMM_BK : 0; // int8 tile
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + BQ_BYTES;
  static constexpr int XCHUNK = GEMM_BM * 32 * 4;         // 16 KB
  static constexpr int XBUF_BYTES = XBUF ? 2 * XCHUNK : 0;
  static constexpr int STAGES_RAW = ((XBUF ? 192 : 200) * 1024) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static constexpr int NUM_THREADS = BQ8 ? 320 : 192;
  static constexpr int TMEM_COLS = (2 * BN < 32) ? 32 : 2 * BN;
  static constexpr int BAR_BYTES = 8 * (3 * STAGES + 4 + 2) + 16;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + XBUF_BYTES + BAR_BYTES;
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
  static_assert((TMEM_COLS & (TMEM_COLS - 1)) == 0, "TMEM columns must be a power of two");
  static_assert(SMEM_BYTES <= 232448, "shared memory");
};

__device__ __forceinline__ float gelu_tanh_f(float x) {
  // 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), hardware tanh approximation
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  float u = k0 * fmaf(k1 * x, x * x, x);
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
  return 0.5f * x * (1.0f + t);
}

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& m, int& n) {
  const int per_group = GEMM_GROUP_M * num_n;
  const int g = tile / per_group;
  const int first_m = g * GEMM_GROUP_M;
  const int gm = min(GEMM_GROUP_M, num_m - first_m);
  const int idx = tile - g * per_group;
  m = first_m + idx % gm;
  n = idx / gm;
}

// int8 x 8 -> bf16 x 8 with one scale: x in [-128, 127] is rebuilt exactly as
// a float from the magic constant 2^23 (0x4B000000 | (x + 128)) minus
// (2^23 + 128), scaled in f32 and rounded once to bf16.
__device__ __forceinline__ uint4 dequant8(uint2 q, float s) {
  const uint32_t w0 = q.x ^ 0x80808080u, w1 = q.y ^ 0x80808080u;
  const float bias = 8388736.0f;  // 2^23 + 128
  float f[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t b0, b1;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(b0) : "r"(w0), "r"(0x4B000000u), "r"(0x7650u | (uint32_t)i));
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(b1) : "r"(w1), "r"(0x4B000000u), "r"(0x7650u | (uint32_t)i));
    f[i] = (__uint_as_float(b0) - bias) * s;
    f[4 + i] = (__uint_as_float(b1) - bias) * s;
  }

  uint4 o;
  o.x = pack_bf16x2(f[0], f[1]);
  o.y = pack_bf16x2(f[2], f[3]);
  o.z = pack_bf16x2(f[4], f[5]);
  o.w = pack_bf16x2(f[6], f[7]);
  return o;
}

// Work units of a launch: tiles [0, dp) whole, then the ks_tiles trailing
// tiles in ks pieces of their K loop each (piece i = (tile - dp) ks + s).
struct Unit {
  int tile, kb0, kb1, piece;  // piece < 0: a whole tile
};
__device__ __forceinline__ Unit unit_of(int u, int num_tiles, int nkb, const GemmArgs& a) {
  const int dp = num_tiles - a.ks_tiles;
  if (u < dp) return Unit{u, 0, nkb, -1};
  const int i = u - dp, s = i % a.ks;
  return Unit{dp + i / a.ks, (int)((long long)s * nkb / a.ks), (int)((long long)(s + 1) * nkb / a.ks), i};
}

// The fused tail of the generic epilogue for 32 accumulator columns
// [col0, col0 + 32) of one row: bias, then the epilogue's transform and
// store; EPI_BF16_SSQ also accumulates the row's sum of squares (in column
// order). Shared by the GEMM and its split-K fix-up, so both produce the
// same bits from the same accumulator values.
template <int EPI>
__device__ __forceinline__ void epi_chunk(const GemmArgs& args, float (&v)[32], int row, int col0, int trow,
                                          float& ssq) {
  if (args.bias != nullptr) {
    const uint4* bp = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(args.bias) + col0);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 b = __ldg(bp + j);
      v[8 * j + 0] += bf16_lo(b.x); v[8 * j + 1] += bf16_hi(b.x);
      v[8 * j + 2] += bf16_lo(b.y); v[8 * j + 3] += bf16_hi(b.y);
      v[8 * j + 4] += bf16_lo(b.z); v[8 * j + 5] += bf16_hi(b.z);
      v[8 * j + 6] += bf16_lo(b.w); v[8 * j + 7] += bf16_hi(b.w);
    }
  }
  if (EPI == EPI_BF16 || EPI == EPI_BF16_SSQ || EPI == EPI_GELU_BF16) {
    if (EPI == EPI_GELU_BF16) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = gelu_tanh_f(v[j]);
    }
    if (EPI == EPI_BF16_SSQ) {
#pragma unroll
      for (int j = 0; j < 32; ++j) ssq = fmaf(v[j], v[j], ssq);
    }
    uint4* op = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(args.out) + (size_t)row * args.ldo + col0);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 o;
      o.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
      o.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
      o.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
      o.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
      op[j] = o;
    }
  } else if (EPI == EPI_RESID_F32) {
    // out = xres + y * (sst[r] + tstab[tidx[row], r])
    const float4* xp =
        args.xres ? reinterpret_cast<const float4*>(args.xres + (size_t)row * args.ldx + col0) : nullptr;
    const float4* sp = reinterpret_cast<const float4*>(args.sst + (size_t)args.ada_row * args.ada_d + col0);
    const float4* tp =
        reinterpret_cast<const float4*>(args.tstab + ((size_t)trow * 9 + args.ada_row) * args.ada_d + col0);
    float4* op = reinterpret_cast<float4*>(reinterpret_cast<float*>(args.out) + (size_t)row * args.ldo + col0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float4 xv = xp ? xp[j] : make_float4(0.f, 0.f, 0.f, 0.f), sv = __ldg(sp + j), tv = __ldg(tp + j), o;
      o.x = xv.x + v[4 * j + 0] * (tv.x + sv.x);
      o.y = xv.y + v[4 * j + 1] * (tv.y + sv.y);
      o.z = xv.z + v[4 * j + 2] * (tv.z + sv.z);
      o.w = xv.w + v[4 * j + 3] * (tv.w + sv.w);
      op[j] = o;
    }
  } else {  // EPI_F32 / EPI_GATE2SIG_F32
    float4* op = reinterpret_cast<float4*>(reinterpret_cast<float*>(args.out) + (size_t)row * args.ldo + col0);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float4 o = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      if (EPI == EPI_GATE2SIG_F32) {
        o.x = 2.0f / (1.0f + __expf(-o.x));
        o.y = 2.0f / (1.0f + __expf(-o.y));
        o.z = 2.0f / (1.0f + __expf(-o.z));
        o.w = 2.0f / (1.0f + __expf(-o.w));
      }
      op[j] = o;
    }
  }
}

// A split piece's accumulator rows, raw, into its [128 x BN] f32 partial.
template <int BN>
__device__ __forceinline__ void dump_partial(const GemmArgs& args, uint32_t tbase, int piece, int row_local) {
  float* dst = args.part + ((size_t)piece * GEMM_BM + row_local) * BN;
#pragma unroll 1
  for (int cc = 0; cc < BN / 32; ++cc) {
    uint32_t r[32];
    tmem_ld32(tbase + cc * 32, r);
    tmem_wait_ld();
    float4* d4 = reinterpret_cast<float4*>(dst + cc * 32);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      d4[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]), __uint_as_float(r[4 * j + 2]),
                          __uint_as_float(r[4 * j + 3]));
  }
}

template <int BN, bool BQ8, int EPI>
__global__ void __launch_bounds__(GemmCfg<BN, BQ8>::NUM_THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmO,
                   const GemmArgs args) {
  constexpr bool XB = EPI == EPI_RESID_F32;
  using C = GemmCfg<BN, BQ8, XB>;
  constexpr int S = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + S * C::A_BYTES;
  uint8_t* sBq = sB + S * C::B_BYTES;
  uint8_t* xbuf = sBq + S * C::BQ_BYTES;  // [2][128 rows][128 B], 128B-swizzled (XB only)
  uint64_t* bars = reinterpret_cast<uint64_t*>(xbuf + C::XBUF_BYTES);
  uint64_t* full = bars;            // TMA -> (dequant | MMA)
  uint64_t* deq = bars + S;         // dequant -> MMA
  uint64_t* empty = bars + 2 * S;   // MMA -> TMA
  uint64_t* tfull = bars + 3 * S;   // MMA -> epilogue, 2 accumulators
  uint64_t* tempty = tfull + 2;     // epilogue -> MMA
  uint64_t* xfull = tempty + 2;     // residual chunk landed (XB), 2 buffers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xfull + 2);

  const int warp = warp_id(), lane = lane_id();
  const int M = args.M, N = args.N, K = args.K;
  const int num_m = (M + GEMM_BM - 1) / GEMM_BM, num_n = N / BN, nkb = K / GEMM_BK;
  const int num_tiles = num_m * num_n;
  const int num_units = num_tiles - args.ks_tiles + args.ks_tiles * args.ks;
  const int dp = num_tiles - args.ks_tiles;  // units below dp are whole tiles
  const int kw = args.b_kwrap > 0 ? args.b_kwrap : K;  // B's own K (columns repeat with this period)

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&deq[i], 4);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 4);
      mbar_init(&xfull[i], 1);
    }
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (XB && args.xres) {
      prefetch_tmap(&tmX);
      prefetch_tmap(&tmO);
    }
  }
  if (warp == 1) tmem_alloc(tmem_slot, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      const uint32_t bytes = C::A_BYTES + (BQ8 ? C::BQ_BYTES : C::B_BYTES);
      for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
        const Unit un = unit_of(u, num_tiles, nkb, args);
        int m, n;
        tile_coords(un.tile, num_m, num_n, m, n);
        for (int kb = un.kb0; kb < un.kb1; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, 0x101)) goto done;
          mbar_arrive_expect_tx(&full[s], bytes);
          tma_load_2d(sA + s * C::A_BYTES, &tmA, &full[s], kb * GEMM_BK, m * GEMM_BM);
          const int bx = (kb * GEMM_BK) % kw;
          if (BQ8)
            tma_load_2d(sBq + s * C::BQ_BYTES, &tmB, &full[s], bx, n * BN);
          else
            tma_load_2d(sB + s * C::B_BYTES, &tmB, &full[s], bx, n * BN);
          if (++s == S) { s = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(GEMM_BM, BN);
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++it) {
        const Unit un = unit_of(u, num_tiles, nkb, args);
        const int acc = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], aph ^ 1, 0x102)) goto done;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = un.kb0; kb < un.kb1; ++kb) {
          if (!mbar_wait(BQ8 ? &deq[s] : &full[s], ph, 0x103)) goto done;
          tc_fence_after();
          const uint64_t da = sdesc_kmajor_sw128(smem_u32(sA + s * C::A_BYTES));
          const uint64_t db = sdesc_kmajor_sw128(smem_u32(sB + s * C::B_BYTES));
#pragma unroll
          for (int k = 0; k < GEMM_BK / 16; ++k)
            umma_ss(d_tmem, da + 2 * k, db + 2 * k, idesc, (kb != un.kb0 || k != 0));
          umma_commit(&empty[s]);
          if (++s == S) { s = 0; ph ^= 1; }
        }
        umma_commit(&tfull[acc]);
      }
    }
  } else if (warp < 6 && XB && args.xres != nullptr) {
    // ---------------- gated-residual epilogue through shared memory ----------------
    // out = xres + y * ada, 32 columns at a time: the [128 x 32] f32 chunk of
    // xres arrives by TMA one chunk ahead, each thread (one row) combines it
    // with its accumulator row in place, and one TMA store writes the chunk
    // back as whole rows. Thread 64 (warp 2, lane 0) issues the copies; two
    // buffers alternate, a buffer is reloaded only once the store that last
    // read it is done reading (wait_group.read), and all 128 threads pass
    // every named barrier together (failures are OR-reduced across them).
    const int q = warp & 3;
    const int row_local = q * 32 + lane;
    const bool leader = threadIdx.x == 64;
    constexpr int NCH = BN / 32;
    uint32_t issued = 0, g = 0;  // residual chunks requested / consumed
    auto load_chunk = [&](int tile, int cc) {
      int m, n;
      tile_coords(tile, num_m, num_n, m, n);
      const int b = issued & 1;
      mbar_arrive_expect_tx(&xfull[b], C::XCHUNK);
      tma_load_2d(xbuf + b * C::XCHUNK, &tmX, &xfull[b], n * BN + cc * 32, m * GEMM_BM);
      ++issued;
    };
    if (leader && (int)blockIdx.x < dp) load_chunk(blockIdx.x, 0);
    int it = 0;
    bool failed = false;
    for (int u = blockIdx.x; u < num_units && !failed; u += gridDim.x, ++it) {
      const int tile = u;  // whole tiles come first (u < dp)
      const int acc = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      const bool tok = warp_wait(&tfull[acc], aph, 0x104);
      if (named_bar_any(1, 128, !tok)) break;
      tc_fence_after();
      if (u >= dp) {  // a split piece: its raw partial, the fix-up kernel applies the epilogue
        const Unit un = unit_of(u, num_tiles, nkb, args);
        dump_partial<BN>(args, tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN, un.piece, row_local);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        continue;
      }
      int m, n;
      tile_coords(tile, num_m, num_n, m, n);
      const int row = m * GEMM_BM + row_local;
      const int trow = row < M ? table_row(args.tidx, row, args.tk) : 0;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
#pragma unroll 1
      for (int cc = 0; cc < NCH; ++cc, ++g) {
        uint32_t r[32];
        tmem_ld32(tbase + cc * 32, r);
        tmem_wait_ld();
        const int col0 = n * BN + cc * 32;
        const int b = g & 1;
        const bool ok = warp_wait(&xfull[b], (g >> 1) & 1, 0x106);
        if (ok) {
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          if (args.bias != nullptr) {
            const uint4* bp = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(args.bias) + col0);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              uint4 bb = __ldg(bp + j);
              v[8 * j + 0] += bf16_lo(bb.x); v[8 * j + 1] += bf16_hi(bb.x);
              v[8 * j + 2] += bf16_lo(bb.y); v[8 * j + 3] += bf16_hi(bb.y);
              v[8 * j + 4] += bf16_lo(bb.z); v[8 * j + 5] += bf16_hi(bb.z);
              v[8 * j + 6] += bf16_lo(bb.w); v[8 * j + 7] += bf16_hi(bb.w);
            }
          }
          const float4* sp = reinterpret_cast<const float4*>(args.sst + (size_t)args.ada_row * args.ada_d + col0);
          const float4* tp = reinterpret_cast<const float4*>(
              args.tstab + ((size_t)trow * 9 + args.ada_row) * args.ada_d + col0);
          uint8_t* rowp = xbuf + b * C::XCHUNK + row_local * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float4* slot = reinterpret_cast<float4*>(rowp + ((j ^ (row_local & 7)) << 4));
            const float4 xv = *slot, sv = __ldg(sp + j), tv = __ldg(tp + j);
            float4 o;
            o.x = xv.x + v[4 * j + 0] * (tv.x + sv.x);
            o.y = xv.y + v[4 * j + 1] * (tv.y + sv.y);
            o.z = xv.z + v[4 * j + 2] * (tv.z + sv.z);
            o.w = xv.w + v[4 * j + 3] * (tv.w + sv.w);
            *slot = o;
          }
          fence_proxy_async_smem();
        }
        if (named_bar_any(1, 128, !ok)) {
          failed = true;
          break;
        }
        if (leader) {
          tma_store_2d(&tmO, xbuf + b * C::XCHUNK, col0, m * GEMM_BM);
          bulk_commit();
          const int ntile = cc + 1 < NCH ? tile : tile + (int)gridDim.x;
          if (ntile < dp) {
            bulk_wait_read<1>();  // the store that last read the other buffer is done with it
            load_chunk(ntile, cc + 1 < NCH ? cc + 1 : 0);
          }
        }
      }
      if (failed) break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
    if (leader) {
      bulk_wait_all();
      // a residual chunk requested but never consumed (only after a failed
      // wait): let it land before the CTA's shared memory is released
      if (issued > g) mbar_wait(&xfull[(issued - 1) & 1], ((issued - 1) >> 1) & 1, 0x107);
    }
  } else if (warp < 6) {
    // ---------------- epilogue ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_local = q * 32 + lane;
    int it = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++it) {
      const Unit un = unit_of(u, num_tiles, nkb, args);
      const int acc = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      if (!warp_wait(&tfull[acc], aph, 0x104)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      if (un.piece >= 0) {  // a split piece: its raw partial, the fix-up kernel applies the epilogue
        dump_partial<BN>(args, tbase, un.piece, row_local);
      } else {
        int m, n;
        tile_coords(un.tile, num_m, num_n, m, n);
        const int row = m * GEMM_BM + row_local;
        const bool row_ok = row < M;
        float ssq = 0.f;
        const int trow = (EPI == EPI_RESID_F32 && row_ok) ? table_row(args.tidx, row, args.tk) : 0;
#pragma unroll 1
        for (int cc = 0; cc < BN / 32; ++cc) {
          uint32_t r[32];
          tmem_ld32(tbase + cc * 32, r);
          tmem_wait_ld();
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          if (row_ok) epi_chunk<EPI>(args, v, row, n * BN + cc * 32, trow, ssq);
        }
        if (EPI == EPI_BF16_SSQ && row_ok && n * BN < args.ssq_cols)
          args.ssq[(size_t)row * args.ssq_ld + n] = ssq;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  } else if (BQ8) {
    // ---------------- dequantisers (warps 6..9) ----------------
    const int td = threadIdx.x - 192;  // 0..127
    int s = 0;
    uint32_t ph = 0;
    const int ngroups = kw / 128;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x) {
      const Unit un = unit_of(u, num_tiles, nkb, args);
      int m, n;
      tile_coords(un.tile, num_m, num_n, m, n);
      for (int kb = un.kb0; kb < un.kb1; ++kb) {
        if (!warp_wait(&full[s], ph, 0x105)) goto done;
        const uint8_t* src = sBq + s * C::BQ_BYTES;
        uint8_t* dst = sB + s * C::B_BYTES;
        const int g = ((kb * GEMM_BK) % kw) >> 7;
#pragma unroll 4
        for (int j = 0; j < BN * 8 / 128; ++j) {
          const int id = j * 128 + td;
          const int r = id >> 3, c = id & 7;
          const size_t si = (size_t)(n * BN + r) * ngroups + g;
          const float sc = args.scale_bf16
                               ? __uint_as_float((uint32_t)__ldg(reinterpret_cast<const uint16_t*>(args.scales) + si) << 16)
                               : __ldg(reinterpret_cast<const float*>(args.scales) + si);
          const uint2 qv = *reinterpret_cast<const uint2*>(src + r * 64 + c * 8);
          *reinterpret_cast<uint4*>(dst + (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4)) = dequant8(qv, sc);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&deq[s]);
        if (++s == S) { s = 0; ph ^= 1; }
      }
    }
  }
done:
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// Split-K fix-up: one CTA per (split tile, group of 32 rows), one warp per
// 32-column chunk, one thread per row: sums the tile's ks partials in piece
// order (so the result does not depend on which CTA ran which piece) and
// applies the whole-tile path's epilogue. The sum of squares of a row
// (EPI_BF16_SSQ) adds the chunks' sums in chunk order.
constexpr int FIX_ROWS = 32;
template <int BN, int EPI>
__global__ void __launch_bounds__(FIX_ROWS * (BN / 32)) gemm_fixup_kernel(const GemmArgs args) {
  __shared__ float red[BN / 32][FIX_ROWS];
  const int num_m = (args.M + GEMM_BM - 1) / GEMM_BM, num_n = args.N / BN;
  const int groups = GEMM_BM / FIX_ROWS;
  const int ti = blockIdx.x / groups, rg = blockIdx.x % groups;
  const int tile = num_m * num_n - args.ks_tiles + ti;
  int m, n;
  tile_coords(tile, num_m, num_n, m, n);
  const int rl = rg * FIX_ROWS + (threadIdx.x % FIX_ROWS), cc = threadIdx.x / FIX_ROWS;
  const int row = m * GEMM_BM + rl;
  const bool row_ok = row < args.M;
  float ssq = 0.f;
  if (row_ok) {
    const int trow = EPI == EPI_RESID_F32 ? table_row(args.tidx, row, args.tk) : 0;
    const float4* src = reinterpret_cast<const float4*>(
        args.part + ((size_t)ti * args.ks * GEMM_BM + rl) * BN + cc * 32);
    const size_t pstride = (size_t)GEMM_BM * BN / 4;  // float4 between consecutive pieces
    float v[32];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 a = src[j];
      v[4 * j] = a.x;
      v[4 * j + 1] = a.y;
      v[4 * j + 2] = a.z;
      v[4 * j + 3] = a.w;
    }
    for (int s = 1; s < args.ks; ++s) {
      float4 a[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] = src[s * pstride + j];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[4 * j] += a[j].x;
        v[4 * j + 1] += a[j].y;
        v[4 * j + 2] += a[j].z;
        v[4 * j + 3] += a[j].w;
      }
    }
    epi_chunk<EPI>(args, v, row, n * BN + cc * 32, trow, ssq);
  }
  if (EPI == EPI_BF16_SSQ) {
    red[cc][threadIdx.x % FIX_ROWS] = ssq;
    __syncthreads();
    if (cc == 0 && row_ok && n * BN < args.ssq_cols) {
      float t = red[0][threadIdx.x];
#pragma unroll
      for (int c = 1; c < BN / 32; ++c) t += red[c][threadIdx.x];
      args.ssq[(size_t)row * args.ssq_ld + n] = t;
    }
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

size_t gemm_part_floats() { return (size_t)sm_count() * GEMM_BM * 256; }

template <int BN, bool BQ8, int EPI>
static int launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tx, const CUtensorMap& to,
                      const GemmArgs& a, cudaStream_t st) {
  using C = GemmCfg<BN, BQ8, EPI == EPI_RESID_F32>;
  auto kern = gemm_tc_kernel<BN, BQ8, EPI>;
  // per device and instance: the shared-memory opt-in, set once (host threads
  // may race to set it; the call is idempotent and the flag is atomic)
  static std::atomic<bool> attr_set[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) return set_error(LTXB_EINVAL, "gemm: device %d out of range", dev);
  if (!attr_set[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    if (e != cudaSuccess) return set_cuda_error(e, "gemm: cudaFuncSetAttribute");
    attr_set[dev].store(true, std::memory_order_release);
  }
  const int num_tiles = ((a.M + GEMM_BM - 1) / GEMM_BM) * (a.N / BN);
  const int num_units = num_tiles - a.ks_tiles + a.ks_tiles * a.ks;
  const int grid = num_units < sm_count() ? num_units : sm_count();
  kern<<<grid, C::NUM_THREADS, C::SMEM_BYTES, st>>>(ta, tb, tx, to, a);
  launched();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e, "gemm launch");
  if (a.ks_tiles > 0) {
    gemm_fixup_kernel<BN, EPI><<<a.ks_tiles * (GEMM_BM / FIX_ROWS), FIX_ROWS * (BN / 32), 0, st>>>(a);
    launched();
    e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error(e, "gemm split-K fix-up launch");
  }
  return LTXB_OK;
}

// Which tiles to split (see GemmArgs::part): the tiles of a last wave that
// would fill at most a quarter of the SMs (or every tile with ksplit_all),
// each into as many K pieces as fill the SMs, at most 8 and at least 2
// K blocks of 64 per piece. Sets a.ks_tiles / a.ks (0 / 1: no split).
static void plan_split(GemmArgs& a, int bn) {
  a.ks_tiles = 0;
  a.ks = 1;
  if (!a.part || a.b_int8) return;
  const int P = sm_count(), nkb = a.K / GEMM_BK;
  const int tiles = ((a.M + GEMM_BM - 1) / GEMM_BM) * (a.N / bn);
  int r = 0;
  if (a.ksplit_all)
    r = tiles;
  else if (tiles > P && tiles % P != 0 && (tiles % P) * 4 <= P)
    r = tiles % P;
  if (r == 0 || r > P) return;
  int ks = P / r;
  if (ks > 8) ks = 8;
  if (ks > nkb / 2) ks = nkb / 2;
  if (ks < 2) return;
  a.ks_tiles = r;
  a.ks = ks;
}

template <int BN, bool BQ8>
static int dispatch_epi(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tx, const CUtensorMap& to,
                        const GemmArgs& a, cudaStream_t st) {
  switch (a.epi) {
    case EPI_BF16: return launch_one<BN, BQ8, EPI_BF16>(ta, tb, tx, to, a, st);
    case EPI_BF16_SSQ: return launch_one<BN, BQ8, EPI_BF16_SSQ>(ta, tb, tx, to, a, st);
    case EPI_GELU_BF16: return launch_one<BN, BQ8, EPI_GELU_BF16>(ta, tb, tx, to, a, st);
    case EPI_RESID_F32: return launch_one<BN, BQ8, EPI_RESID_F32>(ta, tb, tx, to, a, st);
    case EPI_GATE2SIG_F32: return launch_one<BN, BQ8, EPI_GATE2SIG_F32>(ta, tb, tx, to, a, st);
    case EPI_F32: return launch_one<BN, BQ8, EPI_F32>(ta, tb, tx, to, a, st);
  }
  return set_error(LTXB_EINVAL, "gemm: unknown epilogue");
}

int gemm_check(const GemmArgs& a, int* bn_out) {
  if (a.M <= 0 || a.N <= 0 || a.K <= 0) return set_error(LTXB_EINVAL, "gemm: empty shape");
  if (a.K % GEMM_BK) return set_error(LTXB_EINVAL, "gemm: K must be a multiple of 64");
  if (a.b_int8 && (a.K % 128)) return set_error(LTXB_EINVAL, "gemm: int8 weights need K % 128 == 0");
  int bn = a.bn;
  if (bn == 0) bn = (a.N % 256 == 0) ? 256 : (a.N % 128 == 0) ? 128 : (a.N % 32 == 0 ? 32 : 0);
  if (bn == 0 || a.N % bn) return set_error(LTXB_EINVAL, "gemm: N must be a multiple of 32");
  if (a.b_int8 && bn == 32) return set_error(LTXB_EINVAL, "gemm: int8 weights need N % 128 == 0");
  // a K block of 64 (int8: a scale group of 128) never straddles B's column period
  if (a.b_kwrap < 0 || (a.b_kwrap > 0 && a.b_kwrap % (a.b_int8 ? 128 : GEMM_BK)))
    return set_error(LTXB_EINVAL, "gemm: B's column period must be whole 64 (int8: 128) column blocks");
  if ((reinterpret_cast<uintptr_t>(a.A) & 15) || (reinterpret_cast<uintptr_t>(a.B) & 15) || (a.lda % 8) ||
      (a.ldb % (a.b_int8 ? 16 : 8)) || (a.ldo % 8))
    return set_error(LTXB_EINVAL, "gemm: operands must be 16-byte aligned with 16-byte row strides");
  // the epilogue moves 16-byte vectors of out, bias and the residual input
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!a16(a.out) || !a16(a.bias) || !a16(a.xres) || !a16(a.part) || (a.xres && a.ldx % 4))
    return set_error(LTXB_EINVAL, "gemm: out, bias and residual must be 16-byte aligned");
  if (bn_out) *bn_out = bn;
  return LTXB_OK;
}

int gemm_tc(const GemmArgs& a_in, cudaStream_t st) {
  int bn = 0;
  if (int rc = gemm_check(a_in, &bn)) return rc;
  GemmArgs a = a_in;
  plan_split(a, bn);
  CUtensorMap ta, tb;
  int rc = make_tmap_2d(&ta, a.A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.K, a.M, a.lda, GEMM_BK, GEMM_BM,
                        CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  const int kw = a.b_kwrap > 0 ? a.b_kwrap : a.K;
  if (a.b_int8)
    rc = make_tmap_2d(&tb, a.B, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, kw, a.N, a.ldb, GEMM_BK, bn,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
  else
    rc = make_tmap_2d(&tb, a.B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, kw, a.N, a.ldb, GEMM_BK, bn,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  // the gated-residual epilogue moves [128 x 32] f32 chunks of the residual
  // input and the output by TMA (128-byte rows, 128B swizzle)
  CUtensorMap tx = ta, to = ta;
  if (a.epi == EPI_RESID_F32 && a.xres) {
    rc = make_tmap_2d(&tx, a.xres, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a.N, a.M, a.ldx, 32, GEMM_BM,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc)
      rc = make_tmap_2d(&to, a.out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a.N, a.M, a.ldo, 32, GEMM_BM,
                        CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  if (a.b_int8) {
    if (bn == 256) return dispatch_epi<256, true>(ta, tb, tx, to, a, st);
    return dispatch_epi<128, true>(ta, tb, tx, to, a, st);
  }
  if (bn == 256) return dispatch_epi<256, false>(ta, tb, tx, to, a, st);
  if (bn == 128) return dispatch_epi<128, false>(ta, tb, tx, to, a, st);
  return dispatch_epi<32, false>(ta, tb, tx, to, a, st);
}

}  // namespace ltxb
