// Internal interfaces between the C-ABI layer (ltxb.cu, block.cu) and the
// kernels. Host-side only types; nothing here crosses the public boundary.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/ltxb.h"

namespace ltxb {

// ---- errors (thread-local message, see ltxb_last_error) ----
int set_error(int code, const char* fmt, ...);
int set_cuda_error(cudaError_t e, const char* what);
// LTXB_EINVAL unless `device` (where a handle's buffers live) is the current device
int check_device(int device, const char* what);
int sm_count();
// per-device caches are indexed by device ordinal below this bound
constexpr int kMaxDevices = 64;

// ---- launch accounting and per-phase profiling ----
// Every kernel launcher calls launched() after a successful launch, so
// ltxb_launch_count() counts this library's kernels.
void launched();
// RAII phase marker: with profiling on, records CUDA events on `st` around
// the scope and attributes the elapsed device time to `name`.
struct Phase {
  Phase(const char* name, cudaStream_t st);
  ~Phase();
  const char* name;
  cudaStream_t st;
  int slot;
};

// ---- TMA descriptors ----
// 2-D tensor map of a row-major [rows, cols] matrix with row stride `ld`
// elements; box [box_rows, box_cols]. x = column (innermost), y = row.
int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, int cols, int rows,
                 int ld, int box_cols, int box_rows, CUtensorMapSwizzle swz);

// ---- tcgen05 GEMM ----
enum Epi : int {
  EPI_BF16 = 0,          // out bf16 = acc (+ bias)
  EPI_BF16_SSQ = 1,      // EPI_BF16 + per-(row, N tile) sum of squares for columns < ssq_cols
  EPI_GELU_BF16 = 2,     // out bf16 = gelu_tanh(acc (+ bias))
  EPI_RESID_F32 = 3,     // out f32 = xres + (acc + bias) * ada(ada_row)
  EPI_GATE2SIG_F32 = 4,  // out f32 = 2 * sigmoid(acc + bias)
  EPI_F32 = 5,           // out f32 = acc (+ bias)
};

struct GemmArgs {
  const void* A;  // bf16 [M, K], row stride lda
  int lda;
  const void* B;  // bf16 or int8 [N, K], row stride ldb
  int ldb;
  int b_int8;
  const void* scales;  // [N, K/128] f32 or bf16
  int scale_bf16;
  int M, N, K;
  int bn;  // N tile (0 = auto)
  int epi;
  const void* bias;  // bf16 [N] or null
  void* out;
  int ldo;
  // EPI_BF16_SSQ
  float* ssq;
  int ssq_cols;
  int ssq_ld;
  // EPI_RESID_F32
  const float* xres;
  int ldx;
  const float* sst;    // [9, D]
  const float* tstab;  // [K, 9, D]
  const int* tidx;     // [M]
  int tk;              // rows of tstab
  int ada_row;
  int ada_d;
  // split-precision products (the f32-exact prompt K/V): B's columns repeat
  // with period b_kwrap (its real K; 0 = no repeat)
  int b_kwrap;
  // split-K of trailing tiles (deterministic): with `part` set (f32 scratch
  // of gemm_part_floats() floats), gemm_tc splits the K loop of the tiles
  // of a last wave that would leave most SMs idle (or of every tile with
  // ksplit_all) into pieces that write f32 partials, and a fix-up kernel sums
  // them in a fixed order and applies the epilogue. ks_tiles / ks are set
  // by gemm_tc (the split tiles, pieces per tile).
  float* part;
  int ksplit_all;
  int ks_tiles, ks;
};
// floats of split-K scratch gemm_tc may use (one [128 x 256] tile per SM)
size_t gemm_part_floats();
// Shape, alignment and tile checks of gemm_tc, on the host, launching
// nothing; *bn_out receives the N tile gemm_tc will use.
int gemm_check(const GemmArgs& a, int* bn_out);
int gemm_tc(const GemmArgs& a, cudaStream_t st);

// ---- flash attention (tcgen05) ----
struct AttnArgs {
  const void* q;  // bf16 [Tq, H, 128], row stride ldq elements
  const void* k;  // bf16 [Tkv, H, 128], row stride ldk
  const void* v;  // bf16 [Tkv, H, 128], row stride ldv
  int ldq, ldk, ldv;
  void* out;           // bf16 [Tq, H, 128], row stride ldo elements (0: H * 128)
  int ldo;
  const float* gate;   // f32 [Tq, ldg], column h = head h; or null
  int ldg;
  int Tq, Tkv, H;
  float scale;
  // ring-attention partial state (f32); when o_acc != null the kernel
  // merges into (o_acc [Tq, H, 128], m [H, Tq], l [H, Tq]) instead of
  // writing `out`, and `finalize` writes out = o_acc / l * gate.
  float* o_acc;
  float* m_state;
  float* l_state;
  int first;  // state starts empty
  // split-K/V: with kv_splits = s > 1 (and `first`), split z of s covers K/V
  // tiles [z n / s, (z + 1) n / s) and writes its own state at o_acc + z Tq H
  // 128, m/l + z H Tq; attention_combine merges the s states into `out`.
  int kv_splits;
  // Output into other ranks' memory (head-parallel exchange, peer.cu): with
  // out_tab set, output row i goes to out_tab[i / peer_rows] (a device
  // array of pointers) at row i % peer_rows, columns out_col0 + h 128 ..,
  // row stride ldo; `out` is unused. With sig_counter set, the last CTA to
  // finish publishes sig_epoch at *sig_tab[p] for p < sig_n (device array).
  void* const* out_tab;
  int peer_rows;
  int out_col0;
  uint32_t* sig_counter;
  uint32_t* const* sig_tab;
  int sig_n;
  uint32_t sig_epoch;
};
int attention_tc(const AttnArgs& a, cudaStream_t st);
// out = (merged state of a.kv_splits splits, 1 for a ring's accumulated state) / l * gate
int attention_combine(const AttnArgs& a, cudaStream_t st);
// split count that best fills the GPU's SMs for this shape (1 = no split)
int attention_kv_splits(int Tq, int Tkv, int H, int max_splits);
// whole split-K/V attention: partial states in (o_acc, m_state, l_state), sized for
// attention_kv_splits(...) splits, then the combine into `out`
int attention_split(AttnArgs a, int splits, cudaStream_t st);
// RoPE tables (core.cu)
int rope_tables(int kind, const float* pos, int T, int H, double theta, float* cos_out, float* sin_out,
                cudaStream_t st);
// status word of the attention unit (compiled separately, see common.cuh)
cudaError_t attn_status(uint32_t* v, bool clear);

// ---- elementwise / normalisation kernels ----
// n = rms(x) * (1 + ada(r_scale)) + ada(r_shift) -> bf16 or f32 [T, D]; tstab has tk rows
int norm_modulate(const float* x, int T, int D, const float* sst, const float* tstab, const int* tidx, int tk, int r_shift,
                  int r_scale, void* out, int out_f32, float* rms_copy, cudaStream_t st);
// combined modulation rows of n (<= 3) norm-modulate calls: tab [n][tk][2][D]
// = ((sst + tstab)[scale] + 1, (sst + tstab)[shift]) per table row
int mod_tables(const float* sst, const float* tstab, int tk, int D, const int* shifts, const int* scales, int n,
               float* tab, cudaStream_t st);
// norm_modulate from one table of mod_tables (tab points at its [tk][2][D])
int norm_modulate_tab(const float* x, int T, int D, const float* tab, const int* tidx, int tk, void* out, int out_f32,
                      cudaStream_t st);
// weightless rms only (s4_normed stage), f32 out
int rms_rows(const float* x, int T, int D, float* out, cudaStream_t st);
// q/k norm (+ optional RoPE) from raw bf16 projections and per-tile sums of squares
int qk_norm_rope(const void* raw, int ld_raw, const float* ssq, int ssq_ld, int n_ssq, const void* w_bf16,
                 const float* cos, const float* sin, int T, int D, void* out_bf16, float* out_f32, cudaStream_t st);
// enc = ctx * (1 + (psst[1] + pts2[1])) + (psst[0] + pts2[0]) -> bf16 and/or f32
int ctx_modulate(const float* ctx, int S, int D, const float* psst, const float* pts2, void* out_bf16,
                 float* out_f32, cudaStream_t st);
// int8 [N, K] + scales -> bf16 [N, K]
int dequant_weights(const int8_t* q, const void* scales, int scale_bf16, int N, int K, void* out, cudaStream_t st);
// f32 -> bf16 / bf16 -> f32 copies
int cast_f32_bf16(const float* in, void* out, size_t n, cudaStream_t st);
int cast_bf16_f32(const void* in, float* out, size_t n, cudaStream_t st);
// q and k of self-attention normalised (+RoPE) in one pass sharing cos/sin
int qk_norm_rope2(const void* raw_q, const void* raw_k, int ld_raw, const float* ssq_q, const float* ssq_k,
                  int ssq_ld, int n_ssq, const void* wq, const void* wk, const float* cos, const float* sin, int T,
                  int D, void* out_q, void* out_k, cudaStream_t st);

// ---- f32 SIMT path (LTXB_MODE_F32) ----
// C[M, N] = A[M, K] (f32) . W[N, K]^T + bias, epilogues as Epi; W bf16
// (upcast) or, with wq set, int8 [N, K] times grouped-128 scales in f32
int gemm_f32(const float* A, int lda, const void* W, int M, int N, int K, const void* bias, int epi, float* out,
             int ldo, float* ssq, int ssq_ld, const float* xres, const float* sst, const float* tstab,
             const int* tidx, int tk, int ada_row, cudaStream_t st, const int8_t* wq = nullptr,
             const void* scales = nullptr, int scale_bf16 = 0);
// f32 attention: q/k/v f32 [T, H, 128] (row strides ld*) -> out f32 [Tq, H*128],
// with optional gate [Tq, ldg]
int attention_f32(const float* q, int ldq, const float* k, int ldk, const float* v, int ldv, float* out,
                  const float* gate, int ldg, int Tq, int Tkv, int H, float scale, cudaStream_t st);
// q/k norm (+RoPE) on f32 raw projections (ssq computed in-kernel); f32
// output, or bf16 (one rounding) into out_bf16 when out is null
int qk_norm_rope_f32(const float* raw, int ld_raw, const void* w_bf16, const float* cos, const float* sin, int T,
                     int D, float* out, cudaStream_t st, void* out_bf16 = nullptr);
// x f32 [rows, cols] -> [rows, parts * cols] bf16: parts 2 = (hi | lo),
// parts 3 = (hi | hi | lo), with hi = bf16(x), lo = bf16(x - hi), so that
// x = hi + lo to ~2^-16
int split_f32_bf16(const float* in, int rows, int cols, int parts, void* out, cudaStream_t st);
// int8 [N, K] + grouped-128 scales -> bf16 [N, 2K] = (w_hi | w_lo) with
// w_hi = bf16(q s) and w_lo = bf16(q s - w_hi): q s has at most 15
// significant bits (bf16 scales), so w_hi + w_lo = q s exactly
int dequant_split(const int8_t* q, const void* scales, int scale_bf16, int N, int K, void* out, cudaStream_t st);
// sequence-parallel head-group layout (rank groups of D/N columns, each in
// SG sub-groups of Dg = D/(N SG)): nsrc (<= 3) bf16 [T, D] matrices with row
// strides lds -> dst [SG][nsrc][N][T][Dg]; and [SG][N][T][Dg] -> out [T, D]
int sp_regroup(const void* const* srcs, const int* lds, int nsrc, int T, int D, int N, int SG, void* dst,
               cudaStream_t st);
int sp_ungroup(const void* src, int T, int D, int N, int SG, void* out, int ld_out, cudaStream_t st);
// ---- head-parallel exchange over peer memory (peer.cu) ----
constexpr int kMaxPeers = 8;
struct PeerScatterArgs {
  const __nv_bfloat16* src[3];  // q, k, v of this rank's tokens, [T, >= D], row strides ld
  int ld[3];
  const float* gate;            // [T, G] f32 or null
  int G;
  __nv_bfloat16* rx[kMaxPeers]; // per owner rank p: its receive buffer [3][N][T][D/N] (peer address)
  float* gall[kMaxPeers];       // per rank p: its gate buffer [N T][G] (peer address)
  uint32_t* flag[kMaxPeers];    // per rank p: the arrival flag of this rank in p's window
  uint32_t* counter;            // this rank's CTA counter (zero between launches)
  uint32_t epoch;
  int N, r, T, D;
};
int peer_scatter(const PeerScatterArgs& a, cudaStream_t st);
// bounded wait until flags[p] has reached `epoch` for every p != r
int peer_wait(const uint32_t* flags, int N, int r, uint32_t epoch, uint32_t site, cudaStream_t st);
// rows x cols f32 (row stride ld_in) -> bf16 (row stride ld_out)
int cast_rows_f32_bf16(const float* in, int ld_in, void* out, int ld_out, int rows, int cols, cudaStream_t st);

}  // namespace ltxb
