// The LTX-2.5 DiT block behind the C ABI: device-resident weight upload from
// the reference's blob format, workspace layout, and the launch sequence of
// one block forward (ltx/block.zig:340-353 `wBlockOut`, :544-574
// `qBlockOutAll`), single-GPU or sequence-parallel.
//
// Launch sequence (bf16 / int8 modes; f32 mode runs the same graph on the
// SIMT f32 kernels):
//   1  n    = rms(x) (1 + ada1) + ada0                      norm_modulate
//   2  qkv  = n . [Wq;Wk;Wv]^T + b  (+ row sum-of-squares)   gemm  N = 3D
//   3  gate = 2 sigmoid(n . Wg^T + bg)                       gemm  N = 32
//   4  q,k  = rope(rms_w(q_raw)), rope(rms_w(k_raw))         qk_norm_rope2
//   5  o    = softmax(q k^T / sqrt(128)) v * gate            attention (ring for SP)
//   6  x_sa = x + (o . Wo^T + bo) * ada2                      gemm  (resid epilogue)
//   7  a    = rms(x_sa) (1 + ada7) + ada6                     norm_modulate
//   8  enc  = ctx (1 + kv1) + kv0;  [k2;v2] = enc . W^T + b    ctx_modulate, split, gemm (M = S,
//      k2 = rms_w(k2) -> bf16, v2 -> bf16                       f32-exact), f32 q/k norm, cast
//   9  q2   = a . Wq2^T + b;  gate2                           gemm x2
//  10  q2   = rms_w(.)                                        qk_norm_rope (no RoPE)
//  11  o2   = cross attention * gate2                          attention (T_kv = S)
//  12  x_ca = x_sa + (o2 . Wo2^T + b) * ada8                  gemm
//  13  f    = rms(x_ca) (1 + ada4) + ada3                      norm_modulate
//  14  h    = gelu(f . W1^T)                                  gemm  N = FF
//  15  out  = x_ca + (h . W2^T) * ada5                        gemm  K = FF
#include <nccl.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include <algorithm>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "upload.h"

struct ltxb_weights {
  int device = 0, mode = 0, qset = 0, D = 0, FF = 0, H = 0, G = 0;
  ltxb::Lin qkv1, g1, o1, q2, g2, kv2, o2, ff1, ff2;
  const void *qn1 = nullptr, *kn1 = nullptr, *qn2 = nullptr, *kn2 = nullptr;
  const float *sst = nullptr, *psst = nullptr;
  std::vector<void*> allocs;
  uint64_t bytes = 0;
};

// Peer window: device memory of this rank that every other rank of the
// communicator has mapped (CUDA IPC), for the head-parallel exchange over
// peer memory (peer.cu). Offsets are identical on every rank:
//   [0, kWinHdr)  header: arrival flags [2 kinds][kMaxPeers] u32 at 0 (kind
//                 0: q/k/v and gates, 1: attention output; entry p written
//                 by rank p), CTA counters [2] at 256, and from kWinTab the
//                 device pointer tables the kernels index, as this process
//                 maps them: [table][2 parities][kMaxPeers] (orx: every
//                 rank's output buffer; flago: this rank's kind-1 flag in
//                 every window)
//   rx[2]         [3][N][T][D/N] bf16: q, k, v of the owned heads, all tokens
//   orx[2]        [T][D] bf16: this rank's attention output, all heads
//   gall[2]       [N T][G] f32: every rank's gate logits
struct PeerWin {
  uint8_t* local = nullptr;
  size_t bytes = 0;
  std::vector<uint8_t*> base;  // every rank's window as mapped in this process
  std::vector<char> opened;    // base[p] came from cudaIpcOpenMemHandle
  size_t off_rx[2] = {}, off_orx[2] = {}, off_gall[2] = {};
  int T = 0, D = 0, G = 0;     // the shapes the layout was made for
  uint32_t epoch = 0;          // block calls through the window since it was made
};
constexpr size_t kWinHdr = 4096, kWinTab = 1024;
enum WinTable { TAB_ORX = 0, TAB_FLAGO = 1 };

struct ltxb_comm {
  ncclComm_t nccl = nullptr;
  int rank = 0, nranks = 1, device = 0;
  cudaStream_t comm_stream = nullptr;
  std::vector<cudaEvent_t> ev;  // pool of events for cross-stream ordering
  bool peer_ok = false;         // every rank mapped every other rank's window
  PeerWin win;
  void* xbuf = nullptr;         // [nranks][128] bytes: handle exchange
};

namespace ltxb {


// ---------------------------------------------------------------------------
// workspace layout
// ---------------------------------------------------------------------------
struct Ws {
  size_t off = 0;
  uint8_t* base = nullptr;
  template <class T>
  T* take(size_t count, size_t elem = sizeof(T)) {
    off = (off + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += count * elem;
    return p;
  }
};

struct Bufs {
  // activations: bf16 in tensor-core modes, f32 in f32 mode (`act` elem size)
  void* n = nullptr;      // [T, D]   norm-modulate output (reused: attn_in, ff_in)
  float* mod = nullptr;   // [3][K][2][D] combined modulation rows of the three norms (small K)
  void* qkv = nullptr;    // [T, 3D]
  float* ssq = nullptr;   // [T, 32]  q/k row sums of squares per N tile
  void* q = nullptr;      // [T, D]
  void* k = nullptr;      // [T_total, D]  (gathered for SP)
  void* v = nullptr;      // [T_total, D]  (SP only)
  float* gate = nullptr;  // [T, G]
  void* o = nullptr;      // [T, D]   attention output (merged heads)
  float* x_sa = nullptr;  // [T, D]
  void* enc = nullptr;    // [S, D]
  void* kv2 = nullptr;    // [S, 2D]
  float* ssq2 = nullptr;  // [S, 32]
  void* k2 = nullptr;     // [S, D]
  float* enc32 = nullptr; // [S, D]   f32 prompt K/V input (tensor-core modes)
  void* enc_split = nullptr; // [S, 3D] bf16 parts of enc32 (hi | lo | hi)
  float* kv2_32 = nullptr;// [S, 2D]  f32 prompt K/V projections (tensor-core modes)
  float* x_ca = nullptr;  // [T, D]
  void* h = nullptr;      // [T, FF]
  float* part = nullptr;  // split-K partials of the GEMMs' trailing tiles (gemm_part_floats())
  void* deq = nullptr;    // bf16: the int8 weights of one linear expanded (unfused int8 path)
  size_t deq_elems = 0;   // its capacity in elements
  float* o_acc = nullptr; // [T, D]  ring state
  float* m_st = nullptr;  // [H, T]
  float* l_st = nullptr;  // [H, T]
  // head-parallel exchange (SP_ALLTOALL)
  void* a2a_send = nullptr;  // [3][N][T][D/N] bf16: q, k, v by head group
  void* a2a_recv = nullptr;  // [3][N T][D/N]: this rank's heads over all tokens
  void* a2a_o = nullptr;     // [N T][D/N]: their attention output
  void* a2a_orecv = nullptr; // [N][T][D/N]: this rank's tokens, every head group
  float* gate_all = nullptr; // [N T][G]
};

static bool g_fused_dequant = false;  // int8 GEMMs: dequantise in smem (true) or expand first (false)
// modulation tables with at most this many rows get combined once per call
constexpr int kModTableRows = 64;

// Sequence-parallel self-attention, three exchanges:
//   SP_ALLTOALL  head-parallel: q/k/v go to the rank that owns their heads
//                (H/N heads per rank, all tokens), the outputs come back;
//                the default when the heads divide evenly over the ranks
//   SP_ALLGATHER every rank gathers all K/V, head group by head group, and
//                attends its own tokens (LTXB_SP=allgather)
//   SP_RING      K/V shards passed around a ring (LTXB_SP=ring or
//                LTXB_SP_RING=1), kept for comparison
//   SP_PEER      head-parallel like SP_ALLTOALL, the exchange written as
//                stores into the other ranks' memory (peer.cu): the default
//                when the heads divide evenly and every rank mapped every
//                other rank's window (LTXB_SP=alltoall forces the NCCL form)
enum SpAlgo { SP_ALLTOALL = 0, SP_ALLGATHER = 1, SP_RING = 2, SP_PEER = 3 };
static int sp_env_algo() {
  static const int a = [] {
    const char* r = getenv("LTXB_SP_RING");
    if (r && r[0] == '1') return (int)SP_RING;
    const char* e = getenv("LTXB_SP");
    if (e && !strcmp(e, "ring")) return (int)SP_RING;
    if (e && !strcmp(e, "allgather")) return (int)SP_ALLGATHER;
    if (e && !strcmp(e, "alltoall")) return (int)SP_ALLTOALL;
    if (e && !strcmp(e, "peer")) return (int)SP_PEER;
    return -1;
  }();
  return a;
}
static SpAlgo sp_algo(const ltxb_weights* w, const ltxb_config* c) {
  const int n = c->sp_size > 1 ? c->sp_size : 1;
  const bool a2a_ok = w->H % n == 0;
  const int e = sp_env_algo();
  if (e == SP_RING || e == SP_ALLGATHER) return static_cast<SpAlgo>(e);
  if (e == SP_PEER) return SP_PEER;  // the forward call reports it if the windows are missing
  if (e == SP_ALLTOALL) return a2a_ok ? SP_ALLTOALL : SP_ALLGATHER;
  const bool peer_ok = a2a_ok && n <= kMaxPeers && c->comm && c->comm->peer_ok;
  return peer_ok ? SP_PEER : a2a_ok ? SP_ALLTOALL : SP_ALLGATHER;
}
static bool sp_use_ring(const ltxb_weights* w, const ltxb_config* c) { return sp_algo(w, c) == SP_RING; }
// K/V splits of the gathered attention (1 for the ring, whose steps merge
// into one state)
// Head groups of the all-gather path: K/V travel and are attended group by
// group, so that group g's attention overlaps the gathers of groups > g.
static int sp_groups(const ltxb_weights* w) { return w->H % 4 == 0 ? 4 : 1; }
static int sp_kv_splits(const ltxb_weights* w, const ltxb_config* c) {
  if (sp_use_ring(w, c)) return 1;
  return attention_kv_splits(c->T, c->T * c->sp_size, w->H / sp_groups(w), 8);
}

static size_t layout(const ltxb_weights* w, const ltxb_config* c, uint8_t* base, Bufs& b) {
  Ws ws;
  ws.base = base;
  const size_t T = c->T, S = c->S, D = w->D, FF = w->FF;
  const size_t Tt = (size_t)c->T * (c->sp_size > 1 ? c->sp_size : 1);
  const size_t act = (w->mode == LTXB_MODE_F32) ? 4 : 2;
  b.n = ws.take<uint8_t>(T * D, act);
  if (c->K <= kModTableRows) b.mod = ws.take<float>((size_t)3 * c->K * 2 * D);
  b.qkv = ws.take<uint8_t>(T * 3 * D, act);
  b.ssq = ws.take<float>(T * 32);
  const bool sp = c->sp_size > 1;
  const SpAlgo alg = sp_algo(w, c);
  const bool a2a = sp && alg == SP_ALLTOALL;
  const bool headpar = a2a || (sp && alg == SP_PEER);  // K of this rank's tokens only
  b.q = ws.take<uint8_t>(T * D, act);
  b.k = ws.take<uint8_t>((headpar ? T : Tt) * D, act);
  if (sp && !headpar) b.v = ws.take<uint8_t>(Tt * D, act);
  b.gate = ws.take<float>(T * w->G);
  b.o = ws.take<uint8_t>(T * D, act);
  b.x_sa = ws.take<float>(T * D);
  b.enc = ws.take<uint8_t>(S * D, act);
  b.kv2 = ws.take<uint8_t>(S * 2 * D, act);
  b.ssq2 = ws.take<float>(S * 32);
  b.k2 = ws.take<uint8_t>(S * D, act);
  if (w->mode != LTXB_MODE_F32) {
    b.enc32 = ws.take<float>(S * D);
    b.enc_split = ws.take<uint8_t>(S * 3 * D, 2);
    b.kv2_32 = ws.take<float>(S * 2 * D);
  }
  b.x_ca = ws.take<float>(T * D);
  b.h = ws.take<uint8_t>(T * FF, act);
  if (w->mode != LTXB_MODE_F32) b.part = ws.take<float>(gemm_part_floats());
  if (w->mode == LTXB_MODE_INT8 && !g_fused_dequant) {
    // the largest int8 matrix expanded at once: the fused q/k/v [3D, D], an
    // FFN one [FF, D], or the prompt K/V's (hi | lo) split [2D, 2D]
    b.deq_elems = std::max({FF * D, 3 * D * D, 4 * D * D});
    b.deq = ws.take<uint8_t>(b.deq_elems, 2);
  }
  if (sp && !headpar) {
    // split states of one head group (the ring: one state of all heads)
    const size_t ns = sp_kv_splits(w, c), gh = alg == SP_RING ? w->H : w->H / sp_groups(w);
    b.o_acc = ws.take<float>(ns * T * gh * 128);
    b.m_st = ws.take<float>(ns * gh * T);
    b.l_st = ws.take<float>(ns * gh * T);
  }
  if (a2a) {
    b.a2a_send = ws.take<uint8_t>(3 * T * D, 2);
    b.a2a_recv = ws.take<uint8_t>(3 * T * D, 2);
    b.a2a_o = ws.take<uint8_t>(T * D, 2);
    b.a2a_orecv = ws.take<uint8_t>(T * D, 2);
    b.gate_all = ws.take<float>(Tt * w->G);
  }
  return (ws.off + 255) & ~size_t(255);
}

// ---------------------------------------------------------------------------
// linears
// ---------------------------------------------------------------------------
struct LinCall {
  const ltxb_weights* w;
  Bufs* b;
  cudaStream_t st;
  int tk;  // rows of the modulation table (cfg K)
};

// y = A . L^T with epilogue `epi`; tensor-core modes take bf16 A.
static int run_lin(const LinCall& lc, const Lin& L, const void* A, int lda, int M, int epi, void* out, int ldo,
                   float* ssq = nullptr, int ssq_cols = 0, const float* xres = nullptr, const float* tstab = nullptr,
                   const int* tidx = nullptr, int ada_row = 0) {
  const ltxb_weights* w = lc.w;
  if (M <= 0) return LTXB_OK;
  if (w->mode == LTXB_MODE_F32)
    return gemm_f32(static_cast<const float*>(A), lda, L.w, M, L.N, L.K, L.b, epi, static_cast<float*>(out), ldo,
                    ssq, 32, xres, w->sst, tstab, tidx, lc.tk, ada_row, lc.st);
  GemmArgs g{};
  g.A = A;
  g.lda = lda;
  g.M = M;
  g.N = L.N;
  g.K = L.K;
  g.epi = epi;
  g.bias = L.b;
  g.out = out;
  g.ldo = ldo;
  g.ssq = ssq;
  g.ssq_cols = ssq_cols;
  g.ssq_ld = 32;
  g.xres = xres;
  g.ldx = ldo;
  g.sst = w->sst;
  g.tstab = tstab;
  g.tidx = tidx;
  g.tk = lc.tk;
  g.ada_row = ada_row;
  g.ada_d = w->D;
  g.part = lc.b->part;
  if (L.wq) {
    if (g_fused_dequant) {
      g.B = L.wq;
      g.ldb = L.K;
      g.b_int8 = 1;
      g.scales = L.sc;
      g.scale_bf16 = L.sc_bf16;
    } else {
      if ((size_t)L.N * L.K > lc.b->deq_elems)
        return set_error(LTXB_EINVAL, "int8 linear [%d, %d] exceeds the expansion buffer", L.N, L.K);
      g.B = lc.b->deq;
      g.ldb = L.K;
      if (int rc = gemm_check(g, nullptr)) return rc;
      int rc = dequant_weights(L.wq, L.sc, L.sc_bf16, L.N, L.K, lc.b->deq, lc.st);
      if (rc) return rc;
    }
  } else {
    g.B = L.w;
    g.ldb = L.K;
  }
  return gemm_tc(g, lc.st);
}

static int attn(const ltxb_weights* w, const void* q, int ldq, const void* k, int ldk, const void* v, int ldv, void* out,
                const float* gate, int Tq, int Tkv, cudaStream_t st) {
  const float scale = 0.08838834764831845f;  // 1/sqrt(128)
  if (w->mode == LTXB_MODE_F32)
    return attention_f32(static_cast<const float*>(q), ldq, static_cast<const float*>(k), ldk,
                         static_cast<const float*>(v), ldv, static_cast<float*>(out), gate, w->G, Tq, Tkv, w->H, scale,
                         st);
  AttnArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.ldq = ldq;
  a.ldk = ldk;
  a.ldv = ldv;
  a.out = out;
  a.gate = gate;
  a.ldg = w->G;
  a.Tq = Tq;
  a.Tkv = Tkv;
  a.H = w->H;
  a.scale = scale;
  return attention_tc(a, st);
}

struct RingStep {
  int compute, recv, next, prev;
};

static RingStep ring_step(int r, int N, int s) {
  RingStep x;
  x.compute = ((r - s) % N + N) % N;
  x.recv = (s + 1 < N) ? ((r - s - 1) % N + N) % N : -1;
  x.next = (r + 1) % N;
  x.prev = (r - 1 + N) % N;
  return x;
}

// sequence-parallel self-attention: ring of K/V shards over NCCL, merging
// (m, l, O) per shard; compute of shard s overlaps the receive of shard s+1.
static int ring_attention(const ltxb_weights* w, const ltxb_config* c, Bufs& b, const void* q, const void* v_local,
                          int ldv_local, const float* gate, cudaStream_t st) {
  ltxb_comm* cm = c->comm;
  const int N = c->sp_size, r = c->sp_rank, T = c->T, D = w->D;
  const size_t chunk = (size_t)T * D * 2;
  uint8_t* kb = static_cast<uint8_t*>(b.k);
  uint8_t* vb = static_cast<uint8_t*>(b.v);
  // local V into its slot of the gathered buffer (K was written there by qk-norm)
  cudaError_t e = cudaMemcpy2DAsync(vb + (size_t)r * chunk, (size_t)D * 2, v_local, (size_t)ldv_local * 2,
                                    (size_t)D * 2, T, cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) return set_cuda_error(e, "ring: local V copy");
  if ((int)cm->ev.size() < 2 * N + 2) return set_error(LTXB_EINVAL, "ring: communicator event pool too small");
  // comm stream starts after this rank's K/V are ready
  cudaEventRecord(cm->ev[0], st);
  cudaStreamWaitEvent(cm->comm_stream, cm->ev[0], 0);
  AttnArgs a{};
  a.q = q;
  a.ldq = D;
  a.ldk = D;
  a.ldv = D;
  a.gate = gate;
  a.ldg = w->G;
  a.Tq = T;
  a.Tkv = T;
  a.H = w->H;
  a.scale = 0.08838834764831845f;
  a.o_acc = b.o_acc;
  a.m_state = b.m_st;
  a.l_state = b.l_st;
  a.out = b.o;
  for (int s = 0; s < N; ++s) {
    const RingStep rs = ring_step(r, N, s);
    const int cur = rs.compute;  // shard held at step s
    const int nxt = rs.recv;     // shard arriving during step s
    if (s + 1 < N) {
      ncclGroupStart();
      ncclSend(kb + (size_t)cur * chunk, chunk, ncclUint8, rs.next, cm->nccl, cm->comm_stream);
      ncclRecv(kb + (size_t)nxt * chunk, chunk, ncclUint8, rs.prev, cm->nccl, cm->comm_stream);
      ncclSend(vb + (size_t)cur * chunk, chunk, ncclUint8, rs.next, cm->nccl, cm->comm_stream);
      ncclRecv(vb + (size_t)nxt * chunk, chunk, ncclUint8, rs.prev, cm->nccl, cm->comm_stream);
      ncclResult_t nr = ncclGroupEnd();
      if (nr != ncclSuccess) return set_error(LTXB_ENCCL, "ring step %d: %s", s, ncclGetErrorString(nr));
      cudaEventRecord(cm->ev[1 + s], cm->comm_stream);
    }
    if (s > 0) cudaStreamWaitEvent(st, cm->ev[s], 0);  // shard `cur` has landed
    a.k = kb + (size_t)cur * chunk;
    a.v = vb + (size_t)cur * chunk;
    a.first = (s == 0);
    int rc = attention_tc(a, st);
    if (rc) return rc;
    // No other cross-stream edge is needed: every remote slot is received
    // exactly once and before it is read, the local slot is never received
    // into, and the send of step s+1 reads the slot the recv of step s wrote
    // (same stream). The last compute step waits on the last group, so the
    // comm stream is idle when the caller's stream is.
  }
  return attention_combine(a, st);
}

// All-gather variant. The local K (in the attention-output buffer) and V
// (in the fused q/k/v buffer) are regrouped into head-group-major gathered
// buffers, [G][N T][D / G], so that each group's slice of every rank is one
// contiguous block. Group by group, an in-place ncclAllGather on the
// (high-priority) comm stream fills in the other ranks' K and V, and the
// compute stream runs that group's split-K/V attention as soon as its gather
// has landed: the gathers of later groups overlap the attention of earlier
// ones.
// Head-parallel (all-to-all) variant. Rank r owns heads [r H/N, (r+1) H/N),
// processed in SG sub-groups of 4 heads (a sub-group's attention over all
// tokens is 4 x 110 query-tile pairs at T 28,160: whole waves on 148 SMs).
// 1. q, k (this rank's tokens, already normalised and rotated) and v are
//    regrouped into [SG][x][N][T][Dg] (Dg = 4 x 128), so that every
//    (sub-group, tensor, rank) block is contiguous. Per sub-group, one NCCL
//    group sends block p to rank p and receives rank p's block for this
//    rank's heads; rank p's tokens are tokens [p T, (p+1) T), so the
//    received blocks stack into [N T][Dg] in token order. The gate logits
//    [T, G] are all-gathered first.
// 2. Per sub-group, attention over all N T queries and keys for its heads
//    (the single-GPU kernel), as soon as that sub-group has arrived: it
//    overlaps the transfer of the later sub-groups.
// 3. Per sub-group, a group returns rows [p T, (p+1) T) of its output to
//    rank p while the next sub-group computes; the received
//    [SG][N][T][Dg] blocks are placed into the [T, D] attention output.
// The caller's stream waits on the comm stream after the last exchange, so
// the comm stream is idle whenever the caller's stream is.
// a2a_start enqueues step 1 (the caller's stream only records an event the
// comm stream waits on); a2a_finish runs steps 2-3. Work that needs neither
// can run on the caller's stream in between.
static int a2a_subgroups(const ltxb_weights* w, const ltxb_config* c) {
  const int hn = w->H / c->sp_size;
  return hn % 4 == 0 ? hn / 4 : 1;
}

static int a2a_start(const ltxb_weights* w, const ltxb_config* c, Bufs& b, const void* q, const void* k,
                     const void* v_local, int ldv_local, const float* gate, cudaStream_t st) {
  ltxb_comm* cm = c->comm;
  const int N = c->sp_size, r = c->sp_rank, T = c->T, D = w->D, SG = a2a_subgroups(w, c);
  const int Dg = D / N / SG;
  if ((int)cm->ev.size() < 1 + 3 * SG) return set_error(LTXB_EINVAL, "sp: communicator event pool too small");
  const size_t blk = (size_t)T * Dg * 2;  // bytes of one [T][Dg] block
  uint8_t* send = static_cast<uint8_t*>(b.a2a_send);
  uint8_t* recv = static_cast<uint8_t*>(b.a2a_recv);
  const void* srcs[3] = {q, k, v_local};
  const int lds[3] = {D, D, ldv_local};
  if (int rc = sp_regroup(srcs, lds, 3, T, D, N, SG, send, st)) return rc;
  cudaEventRecord(cm->ev[0], st);
  cudaStreamWaitEvent(cm->comm_stream, cm->ev[0], 0);
  if (gate) {
    ncclResult_t gr = ncclAllGather(gate, b.gate_all, (size_t)T * w->G, ncclFloat, cm->nccl, cm->comm_stream);
    if (gr != ncclSuccess) return set_error(LTXB_ENCCL, "gate all-gather: %s", ncclGetErrorString(gr));
  }
  for (int g = 0; g < SG; ++g) {
    ncclGroupStart();
    for (int x = 0; x < 3; ++x)
      for (int p = 0; p < N; ++p) {
        if (p == r) continue;
        const size_t off = (((size_t)g * 3 + x) * N + p) * blk;
        ncclSend(send + off, blk, ncclUint8, p, cm->nccl, cm->comm_stream);
        ncclRecv(recv + off, blk, ncclUint8, p, cm->nccl, cm->comm_stream);
      }
    ncclResult_t nr = ncclGroupEnd();
    if (nr != ncclSuccess) return set_error(LTXB_ENCCL, "q/k/v all-to-all: %s", ncclGetErrorString(nr));
    for (int x = 0; x < 3; ++x) {  // this rank's own block
      const size_t off = (((size_t)g * 3 + x) * N + r) * blk;
      cudaError_t e = cudaMemcpyAsync(recv + off, send + off, blk, cudaMemcpyDeviceToDevice, cm->comm_stream);
      if (e != cudaSuccess) return set_cuda_error(e, "sp: local block");
    }
    cudaEventRecord(cm->ev[1 + g], cm->comm_stream);
  }
  return LTXB_OK;
}

static int a2a_finish(const ltxb_weights* w, const ltxb_config* c, Bufs& b, const float* gate, cudaStream_t st) {
  ltxb_comm* cm = c->comm;
  const int N = c->sp_size, r = c->sp_rank, T = c->T, D = w->D, Hn = w->H / N, SG = a2a_subgroups(w, c);
  const int Dg = D / N / SG, hg = Hn / SG;
  const size_t blk = (size_t)T * Dg * 2;
  uint8_t* recv = static_cast<uint8_t*>(b.a2a_recv);
  uint8_t* o = static_cast<uint8_t*>(b.a2a_o);
  uint8_t* orecv = static_cast<uint8_t*>(b.a2a_orecv);
  for (int g = 0; g < SG; ++g) {
    cudaStreamWaitEvent(st, cm->ev[1 + g], 0);
    AttnArgs a{};
    a.q = recv + ((size_t)g * 3 + 0) * N * blk;
    a.k = recv + ((size_t)g * 3 + 1) * N * blk;
    a.v = recv + ((size_t)g * 3 + 2) * N * blk;
    a.ldq = a.ldk = a.ldv = Dg;
    a.out = o + (size_t)g * N * blk;
    a.ldo = Dg;
    a.gate = gate ? b.gate_all + (size_t)r * Hn + (size_t)g * hg : nullptr;
    a.ldg = w->G;
    a.Tq = N * T;
    a.Tkv = N * T;
    a.H = hg;
    a.scale = 0.08838834764831845f;
    if (int rc = attention_tc(a, st)) return rc;
    cudaEventRecord(cm->ev[1 + SG + g], st);
    cudaStreamWaitEvent(cm->comm_stream, cm->ev[1 + SG + g], 0);
    ncclGroupStart();
    for (int p = 0; p < N; ++p) {
      if (p == r) continue;
      const size_t off = ((size_t)g * N + p) * blk;
      ncclSend(o + off, blk, ncclUint8, p, cm->nccl, cm->comm_stream);
      ncclRecv(orecv + off, blk, ncclUint8, p, cm->nccl, cm->comm_stream);
    }
    ncclResult_t nr = ncclGroupEnd();
    if (nr != ncclSuccess) return set_error(LTXB_ENCCL, "attention output all-to-all: %s", ncclGetErrorString(nr));
    const size_t off = ((size_t)g * N + r) * blk;
    cudaError_t e = cudaMemcpyAsync(orecv + off, o + off, blk, cudaMemcpyDeviceToDevice, cm->comm_stream);
    if (e != cudaSuccess) return set_cuda_error(e, "sp: local output block");
  }
  cudaEventRecord(cm->ev[1 + 2 * SG], cm->comm_stream);
  cudaStreamWaitEvent(st, cm->ev[1 + 2 * SG], 0);
  return sp_ungroup(orecv, T, D, N, SG, b.o, D, st);
}

// ---- peer window (SP_PEER) ----
// Closes the other ranks' windows and frees this one (no waiting on peers).
static void win_release(ltxb_comm* c) {
  PeerWin& W = c->win;
  for (size_t p = 0; p < W.base.size(); ++p)
    if (W.opened[p]) cudaIpcCloseMemHandle(W.base[p]);
  if (W.local) cudaFree(W.local);
  W = PeerWin{};
}

struct WinXchg {
  cudaIpcMemHandle_t h;
  uint64_t pid;
  uint64_t ok;
};
static_assert(sizeof(WinXchg) <= 128, "exchange record");

// Collective: every rank allocates a window of `bytes`, the ranks exchange
// IPC handles through NCCL and map each other's windows. Any earlier window
// is released first, after a barrier that ends every rank's use of it.
// Synchronous (the host waits); fails on every rank if any rank failed. The
// header (flags, counters) starts zeroed and the epoch restarts.
static int win_setup(ltxb_comm* c, size_t bytes) {
  const int N = c->nranks, r = c->rank;
  cudaStream_t cs = c->comm_stream;
  uint8_t* xb = static_cast<uint8_t*>(c->xbuf);
  auto fail = [&](int code, const char* what) { return set_error(code, "peer window: %s", what); };
  cudaDeviceSynchronize();
  if (c->win.local) {
    // barrier: every rank's kernels that could still write this window are done
    if (ncclAllReduce(xb, xb, 1, ncclUint8, ncclMax, c->nccl, cs) != ncclSuccess ||
        cudaStreamSynchronize(cs) != cudaSuccess)
      return fail(LTXB_ENCCL, "barrier before release");
    win_release(c);
  }
  WinXchg mine{};
  mine.pid = (uint64_t)getpid();
  uint8_t* local = nullptr;
  bool ok = cudaMalloc(&local, bytes) == cudaSuccess;
  if (ok) ok = cudaMemset(local, 0, kWinHdr) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
  if (ok) ok = cudaIpcGetMemHandle(&mine.h, local) == cudaSuccess;
  cudaGetLastError();
  mine.ok = ok ? 1 : 0;
  // every transfer of the exchange runs on the comm stream, in order
  std::vector<uint8_t> all_raw((size_t)N * 128);
  if (cudaMemcpyAsync(xb + (size_t)r * 128, &mine, sizeof(mine), cudaMemcpyHostToDevice, cs) != cudaSuccess ||
      ncclAllGather(xb + (size_t)r * 128, xb, 128, ncclUint8, c->nccl, cs) != ncclSuccess ||
      cudaMemcpyAsync(all_raw.data(), xb, all_raw.size(), cudaMemcpyDeviceToHost, cs) != cudaSuccess ||
      cudaStreamSynchronize(cs) != cudaSuccess) {
    if (local) cudaFree(local);
    return fail(LTXB_ENCCL, "handle exchange");
  }
  std::vector<WinXchg> all(N);
  for (int p = 0; p < N; ++p) memcpy(&all[p], all_raw.data() + (size_t)p * 128, sizeof(WinXchg));
  PeerWin& W = c->win;
  W.local = local;
  W.bytes = bytes;
  W.base.assign(N, nullptr);
  W.opened.assign(N, 0);
  W.base[r] = local;
  for (int p = 0; p < N && ok; ++p) {
    if (p == r) continue;
    // ranks in one process cannot open each other's handles: the window
    // exchange needs one process per rank
    if (!all[p].ok || all[p].pid == mine.pid) {
      ok = false;
      break;
    }
    void* m = nullptr;
    if (cudaIpcOpenMemHandle(&m, all[p].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      ok = false;
      break;
    }
    W.base[p] = static_cast<uint8_t*>(m);
    W.opened[p] = 1;
  }
  // every rank learns whether all ranks mapped every window
  uint8_t okb = ok ? 1 : 0;
  if (cudaMemcpyAsync(xb, &okb, 1, cudaMemcpyHostToDevice, cs) != cudaSuccess ||
      ncclAllReduce(xb, xb, 1, ncclUint8, ncclMin, c->nccl, cs) != ncclSuccess ||
      cudaMemcpyAsync(&okb, xb, 1, cudaMemcpyDeviceToHost, cs) != cudaSuccess ||
      cudaStreamSynchronize(cs) != cudaSuccess)
    okb = 0;
  if (!okb) {
    win_release(c);
    return fail(LTXB_EUNSUPPORTED, "a rank could not map the other ranks' memory");
  }
  return LTXB_OK;
}

// Makes the window fit a block call of T tokens per rank (collective and
// synchronous when the shapes change, otherwise free) and writes the device
// pointer tables the kernels index.
static int win_prepare(ltxb_comm* c, int T, int D, int G) {
  PeerWin& W = c->win;
  if (W.local && W.T == T && W.D == D && W.G == G) return LTXB_OK;
  const int N = c->nranks, r = c->rank;
  auto al = [](size_t v) { return (v + 255) & ~size_t(255); };
  size_t off = kWinHdr, o_rx[2], o_orx[2], o_gall[2];
  for (int i = 0; i < 2; ++i) { o_rx[i] = off; off += al((size_t)3 * N * T * (D / N) * 2); }
  for (int i = 0; i < 2; ++i) { o_orx[i] = off; off += al((size_t)T * D * 2); }
  for (int i = 0; i < 2; ++i) { o_gall[i] = off; off += al((size_t)N * T * G * 4); }
  if (int rc = win_setup(c, off)) return rc;
  for (int i = 0; i < 2; ++i) {
    W.off_rx[i] = o_rx[i];
    W.off_orx[i] = o_orx[i];
    W.off_gall[i] = o_gall[i];
  }
  W.T = T;
  W.D = D;
  W.G = G;
  uint64_t tab[2][2][kMaxPeers] = {};
  for (int i = 0; i < 2; ++i)
    for (int p = 0; p < N; ++p) {
      tab[TAB_ORX][i][p] = reinterpret_cast<uint64_t>(W.base[p] + o_orx[i]);
      tab[TAB_FLAGO][i][p] = reinterpret_cast<uint64_t>(W.base[p] + (size_t)(1 * kMaxPeers + r) * 4);
    }
  if (cudaMemcpyAsync(W.local + kWinTab, tab, sizeof(tab), cudaMemcpyHostToDevice, c->comm_stream) != cudaSuccess ||
      cudaStreamSynchronize(c->comm_stream) != cudaSuccess)
    return set_error(LTXB_ECUDA, "peer window: tables");
  return LTXB_OK;
}

// SP_PEER, step 1 (before the prompt K/V): this rank's q, k, v and gate
// logits into the owners' windows, on the comm stream; returns the epoch of
// this call.
static int peer_start(const ltxb_weights* w, const ltxb_config* c, const void* q, const void* k, const void* v,
                      int ldv, const float* gate, cudaStream_t st, uint32_t* epoch) {
  ltxb_comm* cm = c->comm;
  if (!cm->peer_ok)
    return set_error(LTXB_EUNSUPPORTED, "peer exchange: the ranks could not map each other's memory");
  if (c->sp_size > kMaxPeers || w->H % c->sp_size)
    return set_error(LTXB_EUNSUPPORTED, "peer exchange: %d ranks, %d heads", c->sp_size, w->H);
  if (int rc = win_prepare(cm, c->T, w->D, w->G)) return rc;
  PeerWin& W = cm->win;
  const uint32_t e = ++W.epoch;
  const int par = e & 1, N = c->sp_size, r = c->sp_rank;
  PeerScatterArgs a{};
  a.src[0] = static_cast<const __nv_bfloat16*>(q);
  a.src[1] = static_cast<const __nv_bfloat16*>(k);
  a.src[2] = static_cast<const __nv_bfloat16*>(v);
  a.ld[0] = a.ld[1] = w->D;
  a.ld[2] = ldv;
  a.gate = gate;
  a.G = w->G;
  for (int p = 0; p < N; ++p) {
    a.rx[p] = reinterpret_cast<__nv_bfloat16*>(W.base[p] + W.off_rx[par]);
    a.gall[p] = reinterpret_cast<float*>(W.base[p] + W.off_gall[par]);
    a.flag[p] = reinterpret_cast<uint32_t*>(W.base[p] + (size_t)(0 * kMaxPeers + r) * 4);
  }
  a.counter = reinterpret_cast<uint32_t*>(W.local + 256);
  a.epoch = e;
  a.N = N;
  a.r = r;
  a.T = c->T;
  a.D = w->D;
  cudaEventRecord(cm->ev[0], st);
  cudaStreamWaitEvent(cm->comm_stream, cm->ev[0], 0);
  if (int rc = peer_scatter(a, cm->comm_stream)) return rc;
  cudaEventRecord(cm->ev[1], cm->comm_stream);
  *epoch = e;
  return LTXB_OK;
}

// SP_PEER, step 2: wait for every rank's q/k/v, attend all N T tokens of the
// owned heads with the output rows stored straight into their ranks'
// windows, wait for every rank's output rows. Returns this rank's [T, D]
// attention output (in its window).
static int peer_finish(const ltxb_weights* w, const ltxb_config* c, uint32_t e, bool gated, cudaStream_t st,
                       void** o_out) {
  ltxb_comm* cm = c->comm;
  PeerWin& W = cm->win;
  const int par = e & 1, N = c->sp_size, r = c->sp_rank, T = c->T, D = w->D, Dn = D / N;
  const uint32_t* flags = reinterpret_cast<const uint32_t*>(W.local);
  cudaStreamWaitEvent(st, cm->ev[1], 0);  // this rank's own slice is written by its scatter
  if (int rc = peer_wait(flags, N, r, e, 0x301, st)) return rc;
  const uint8_t* rx = W.local + W.off_rx[par];
  const size_t blk = (size_t)N * T * Dn * 2;
  AttnArgs a{};
  a.q = rx;
  a.k = rx + blk;
  a.v = rx + 2 * blk;
  a.ldq = a.ldk = a.ldv = Dn;
  a.gate = gated ? reinterpret_cast<const float*>(W.local + W.off_gall[par]) + (size_t)r * (w->H / N) : nullptr;
  a.ldg = w->G;
  a.Tq = N * T;
  a.Tkv = N * T;
  a.H = w->H / N;
  a.scale = 0.08838834764831845f;
  a.ldo = D;
  a.out_tab = reinterpret_cast<void* const*>(W.local + kWinTab + (size_t)(TAB_ORX * 2 + par) * kMaxPeers * 8);
  a.peer_rows = T;
  a.out_col0 = r * Dn;
  a.sig_counter = reinterpret_cast<uint32_t*>(W.local + 256 + 4);
  a.sig_tab = reinterpret_cast<uint32_t* const*>(W.local + kWinTab + (size_t)(TAB_FLAGO * 2 + par) * kMaxPeers * 8);
  a.sig_n = N;
  a.sig_epoch = e;
  if (int rc = attention_tc(a, st)) return rc;
  if (int rc = peer_wait(flags + kMaxPeers, N, r, e, 0x302, st)) return rc;
  *o_out = W.local + W.off_orx[par];
  return LTXB_OK;
}

static int sp_attention(const ltxb_weights* w, const ltxb_config* c, Bufs& b, const void* q, const void* v_local,
                        int ldv_local, const float* gate, cudaStream_t st) {
  const SpAlgo alg = sp_algo(w, c);
  if (alg == SP_ALLTOALL) {
    if (int rc = a2a_start(w, c, b, q, b.k, v_local, ldv_local, gate, st)) return rc;
    return a2a_finish(w, c, b, gate, st);
  }
  if (alg == SP_RING) return ring_attention(w, c, b, q, v_local, ldv_local, gate, st);
  ltxb_comm* cm = c->comm;
  const int N = c->sp_size, r = c->sp_rank, T = c->T, D = w->D;
  const int G = sp_groups(w), Dg = D / G, Hg = w->H / G;
  if ((int)cm->ev.size() < G + 1) return set_error(LTXB_EINVAL, "sp: communicator event pool too small");
  const size_t gbytes = (size_t)N * T * Dg * 2, sbytes = (size_t)T * Dg * 2;  // one group; one rank's slice
  uint8_t* kb = static_cast<uint8_t*>(b.k);
  uint8_t* vb = static_cast<uint8_t*>(b.v);
  const uint8_t* kl = static_cast<const uint8_t*>(b.o);
  const uint8_t* vl = static_cast<const uint8_t*>(v_local);
  for (int g = 0; g < G; ++g) {
    cudaError_t e = cudaMemcpy2DAsync(kb + g * gbytes + r * sbytes, (size_t)Dg * 2, kl + (size_t)g * Dg * 2,
                                      (size_t)D * 2, (size_t)Dg * 2, T, cudaMemcpyDeviceToDevice, st);
    if (e == cudaSuccess)
      e = cudaMemcpy2DAsync(vb + g * gbytes + r * sbytes, (size_t)Dg * 2, vl + (size_t)g * Dg * 2,
                            (size_t)ldv_local * 2, (size_t)Dg * 2, T, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return set_cuda_error(e, "sp: regroup local K/V");
  }
  cudaEventRecord(cm->ev[0], st);
  cudaStreamWaitEvent(cm->comm_stream, cm->ev[0], 0);
  for (int g = 0; g < G; ++g) {
    ncclGroupStart();
    ncclAllGather(kb + g * gbytes + r * sbytes, kb + g * gbytes, sbytes, ncclUint8, cm->nccl, cm->comm_stream);
    ncclAllGather(vb + g * gbytes + r * sbytes, vb + g * gbytes, sbytes, ncclUint8, cm->nccl, cm->comm_stream);
    ncclResult_t nr = ncclGroupEnd();
    if (nr != ncclSuccess) return set_error(LTXB_ENCCL, "K/V all-gather, group %d: %s", g, ncclGetErrorString(nr));
    cudaEventRecord(cm->ev[1 + g], cm->comm_stream);
  }
  const int ns = sp_kv_splits(w, c);
  for (int g = 0; g < G; ++g) {
    cudaStreamWaitEvent(st, cm->ev[1 + g], 0);
    AttnArgs a{};
    a.q = static_cast<const uint8_t*>(q) + (size_t)g * Dg * 2;
    a.ldq = D;
    a.k = kb + g * gbytes;
    a.v = vb + g * gbytes;
    a.ldk = a.ldv = Dg;
    a.out = static_cast<uint8_t*>(b.o) + (size_t)g * Dg * 2;
    a.ldo = D;
    a.gate = gate ? gate + (size_t)g * Hg : nullptr;
    a.ldg = w->G;
    a.Tq = T;
    a.Tkv = T * N;
    a.H = Hg;
    a.scale = 0.08838834764831845f;
    a.o_acc = b.o_acc;  // states reused group after group (stream order)
    a.m_state = b.m_st;
    a.l_state = b.l_st;
    int rc = attention_split(a, ns, st);
    if (rc) return rc;
  }
  return LTXB_OK;
}

// The block, up to `stage` (LTXB_STAGE_BLOCK_OUT = whole block).
static int run_block(const ltxb_weights* w, const ltxb_block_io* io, const ltxb_config* c, int stage,
                     float* stage_out, cudaStream_t st) {
  if (!w || !io || !c) return set_error(LTXB_EINVAL, "null argument");
  if (c->mode != w->mode) return set_error(LTXB_EINVAL, "config mode %d != weights mode %d", c->mode, w->mode);
  if (c->T <= 0 || c->S <= 0 || c->K <= 0) return set_error(LTXB_EINVAL, "T, S and K must be positive");
  {
    // the kernels read rows of these tensors as 16-byte vectors
    const void* v16[] = {io->x, io->out, io->tstab, io->ctx, io->pts2, io->cos, io->sin};
    for (const void* p : v16)
      if (!p || (reinterpret_cast<uintptr_t>(p) & 15))
        return set_error(LTXB_EINVAL, "block io: x, out, tstab, ctx, pts2, cos and sin must be non-null and 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(io->tidx) & 3) return set_error(LTXB_EINVAL, "block io: tidx must be 4-byte aligned");
    if (reinterpret_cast<uintptr_t>(stage_out) & 15) return set_error(LTXB_EINVAL, "stage_out must be 16-byte aligned");
  }
  if (int rc = check_device(w->device, "block")) return rc;
  const bool sp = c->sp_size > 1;
  if (sp && (!c->comm || c->comm->nranks != c->sp_size || c->comm->rank != c->sp_rank))
    return set_error(LTXB_EINVAL, "sp_size > 1 needs a communicator matching sp_rank/sp_size");
  if (sp && w->mode == LTXB_MODE_F32) return set_error(LTXB_EUNSUPPORTED, "sequence parallelism runs bf16/int8 modes");
  if (sp && stage != LTXB_STAGE_BLOCK_OUT) return set_error(LTXB_EINVAL, "stages are single-rank");
  Bufs b;
  const size_t need = layout(w, c, nullptr, b);
  if (!io->workspace || io->workspace_bytes < need)
    return set_error(LTXB_EINVAL, "workspace of %llu bytes is smaller than the %llu required",
                     (unsigned long long)io->workspace_bytes, (unsigned long long)need);
  if (reinterpret_cast<uintptr_t>(io->workspace) & 255) return set_error(LTXB_EINVAL, "workspace must be 256-byte aligned");
  layout(w, c, static_cast<uint8_t*>(io->workspace), b);
  const int T = c->T, S = c->S, D = w->D, FF = w->FF;
  const bool f32 = w->mode == LTXB_MODE_F32;
  const size_t act = f32 ? 4 : 2;
  LinCall lc{w, &b, st, c->K};
  int rc;
#define CK(x)            \
  do {                   \
    if ((rc = (x))) return rc; \
  } while (0)
  auto col = [&](void* p, size_t c0) { return static_cast<void*>(static_cast<uint8_t*>(p) + c0 * act); };

  // 1. n = modulate(rms(x), ada1, ada0)
  if (stage == LTXB_STAGE_S1_NORM_MSA)
    return norm_modulate(io->x, T, D, w->sst, io->tstab, io->tidx, c->K, 0, 1, stage_out, 1, nullptr, st);
  // the three norms' modulation rows, combined once: (0, 1) attention input,
  // (6, 7) cross-attention query input, (3, 4) FFN input
  const size_t mod_stride = (size_t)c->K * 2 * D;
  if (b.mod) {
    const int shifts[3] = {0, 6, 3}, scales[3] = {1, 7, 4};
    CK(mod_tables(w->sst, io->tstab, c->K, D, shifts, scales, 3, b.mod, st));
  }
  auto norm = [&](const float* xin, int which, int r_shift, int r_scale) {
    if (b.mod) return norm_modulate_tab(xin, T, D, b.mod + which * mod_stride, io->tidx, c->K, b.n, f32, st);
    return norm_modulate(xin, T, D, w->sst, io->tstab, io->tidx, c->K, r_shift, r_scale, b.n, f32, nullptr, st);
  };
  {
    Phase p("norm_msa", st);
    CK(norm(io->x, 0, 0, 1));
  }
  // 2. fused q/k/v projection (+ q/k sums of squares)
  {
    Phase p("gemm_qkv1", st);
    CK(run_lin(lc, w->qkv1, b.n, D, T, f32 ? EPI_F32 : EPI_BF16_SSQ, b.qkv, 3 * D, b.ssq, 2 * D));
  }
  const int n_ssq = D / 256;  // N tiles per q (or k) part at BN = 256
  if (stage == LTXB_STAGE_S1B_QNORM) {
    if (f32) return qk_norm_rope_f32(static_cast<const float*>(b.qkv), 3 * D, w->qn1, nullptr, nullptr, T, D, stage_out, st);
    return qk_norm_rope(b.qkv, 3 * D, b.ssq, 32, n_ssq, w->qn1, nullptr, nullptr, T, D, nullptr, stage_out, st);
  }
  // 3. gate logits
  const bool gated = stage != LTXB_STAGE_S2_ATTN1_NOGATE;
  if (gated) {
    Phase p("gemm_gate1", st);
    CK(run_lin(lc, w->g1, b.n, D, T, EPI_GATE2SIG_F32, b.gate, w->G));
  }
  // 4. q/k norm + RoPE (K goes to its slot of the gathered buffer under SP)
  // (the all-gather path regroups K from the attention-output buffer, which
  // is free until the attention writes it)
  const SpAlgo alg = sp_algo(w, c);
  void* k_dst = !sp ? b.k
                : alg == SP_RING ? col(b.k, (size_t)c->sp_rank * T * D)
                : alg == SP_ALLGATHER ? b.o : b.k;
  {
  Phase p("qk_norm_rope", st);
  if (f32) {
    CK(qk_norm_rope_f32(static_cast<const float*>(b.qkv), 3 * D, w->qn1, io->cos, io->sin, T, D,
                        static_cast<float*>(b.q), st));
    CK(qk_norm_rope_f32(static_cast<const float*>(b.qkv) + D, 3 * D, w->kn1, io->cos, io->sin, T, D,
                        static_cast<float*>(k_dst), st));
  } else {
    CK(qk_norm_rope2(b.qkv, col(b.qkv, D), 3 * D, b.ssq, b.ssq + n_ssq, 32, n_ssq, w->qn1, w->kn1, io->cos, io->sin,
                     T, D, b.q, k_dst, st));
  }
  }
  // 8. prompt K/V. The 128 text tokens are computed to f32 accuracy in every
  // mode, as the reference computes them (ltx/block.zig:298-304 with the f32
  // `lin` and dq4 of :22-26, :462-471): enc in f32, the projection exact to
  // ~2^-16 on the tensor cores by splitting both operands into bf16 parts
  // (enc = e_hi + e_lo; an int8 weight q s = w_hi + w_lo exactly, since q s
  // has at most 15 significant bits): [e_hi | e_hi | e_lo] . [w_hi | w_lo |
  // w_hi]^T, one GEMM with K = 3D over the expansion (w_hi | w_lo) whose
  // columns wrap with period 2D (bf16 weights are exact:
  // [e_hi | e_lo] . [w | w]^T); the k norm in f32; k2 / v2 rounded to bf16
  // once, as attention operands.
  auto prompt_kv = [&]() -> int {
    Phase p("prompt_kv", st);
    if (f32) {
      CK(ctx_modulate(io->ctx, S, D, w->psst, io->pts2, nullptr, static_cast<float*>(b.enc), st));
      CK(run_lin(lc, w->kv2, b.enc, D, S, EPI_F32, b.kv2, 2 * D, b.ssq2, D));
    } else {
      const Lin& L = w->kv2;
      const int parts = L.wq ? 3 : 2;
      CK(ctx_modulate(io->ctx, S, D, w->psst, io->pts2, nullptr, b.enc32, st));
      CK(split_f32_bf16(b.enc32, S, D, parts, b.enc_split, st));
      GemmArgs g{};
      g.A = b.enc_split;
      g.lda = parts * D;
      g.M = S;
      g.N = 2 * D;
      g.K = parts * D;
      g.bn = 128;  // 64 CTAs for the 128 text tokens instead of 32
      // one M tile: its K loop, not its width, sets the time, so it is split
      // in K -- except under the peer exchange, whose scatter shares the SMs
      // with it then (8 GPUs: 0.197 ms unsplit, 0.229 ms split)
      g.part = b.part;
      g.ksplit_all = !(sp && alg == SP_PEER);
      g.epi = EPI_F32;
      g.bias = L.b;
      g.out = b.kv2_32;
      g.ldo = 2 * D;
      if (L.wq) {
        if ((size_t)2 * D * 2 * D > b.deq_elems)
          return set_error(LTXB_EINVAL, "prompt K/V: split expansion exceeds the expansion buffer");
        g.B = b.deq;
        g.ldb = 2 * D;
        g.b_kwrap = 2 * D;
        CK(gemm_check(g, nullptr));
        CK(dequant_split(L.wq, L.sc, L.sc_bf16, 2 * D, D, b.deq, st));
      } else {
        g.B = L.w;
        g.ldb = D;
        g.b_kwrap = D;
      }
      CK(gemm_tc(g, st));
      CK(qk_norm_rope_f32(b.kv2_32, 2 * D, w->kn2, nullptr, nullptr, S, D, nullptr, st, b.k2));
      CK(cast_rows_f32_bf16(b.kv2_32 + D, 2 * D, col(b.kv2, D), 2 * D, S, D, st));
    }
    return LTXB_OK;
  };

  // 5. self-attention
  const float* g1 = gated ? b.gate : nullptr;
  void* o_self = b.o;  // self-attention output [T, D]
  if (sp && alg == SP_PEER) {
    // q/k/v go into the owners' memory on the comm stream while the prompt
    // K/V runs here; the attention stores its rows into their ranks' memory
    uint32_t e = 0;
    {
      Phase p("sp_send", st);
      CK(peer_start(w, c, b.q, b.k, col(b.qkv, 2 * D), 3 * D, g1, st, &e));
    }
    CK(prompt_kv());
    Phase p("attn_self", st);
    CK(peer_finish(w, c, e, gated, st, &o_self));
  } else if (sp && alg == SP_ALLTOALL) {
    // the q/k/v exchange runs on the comm stream while the prompt K/V runs here
    {
      Phase p("sp_send", st);
      CK(a2a_start(w, c, b, b.q, b.k, col(b.qkv, 2 * D), 3 * D, g1, st));
    }
    CK(prompt_kv());
    Phase p("attn_self", st);
    CK(a2a_finish(w, c, b, g1, st));
  } else {
    if (sp) CK(prompt_kv());
    Phase p("attn_self", st);
    if (sp)
      CK(sp_attention(w, c, b, b.q, col(b.qkv, 2 * D), 3 * D, g1, st));
    else
      CK(attn(w, b.q, D, b.k, D, col(b.qkv, 2 * D), 3 * D, b.o, g1, T, T, st));
  }
  if (stage == LTXB_STAGE_S2_ATTN1_NOGATE || stage == LTXB_STAGE_S3_ATTN1)
    return run_lin(lc, w->o1, o_self, D, T, EPI_F32, stage_out, D);
  // 6. x_sa = x + (o Wo^T + bo) * ada2
  {
    Phase p("gemm_o1", st);
    CK(run_lin(lc, w->o1, o_self, D, T, EPI_RESID_F32, b.x_sa, D, nullptr, 0, io->x, io->tstab, io->tidx, 2));
  }
  if (stage == LTXB_STAGE_S4_AFTER_SA)
    return cudaMemcpyAsync(stage_out, b.x_sa, (size_t)T * D * 4, cudaMemcpyDeviceToDevice, st) == cudaSuccess
               ? LTXB_OK
               : set_error(LTXB_ECUDA, "stage copy");
  if (stage == LTXB_STAGE_S4_NORMED) return rms_rows(b.x_sa, T, D, stage_out, st);
  // 7. cross-attention query input
  {
    Phase p("norm_ca", st);
    CK(norm(b.x_sa, 1, 6, 7));
  }
  // 8. prompt K/V (computed before self-attention under sequence
  // parallelism, where it overlaps the q/k/v exchange; it reads neither x
  // nor the attention)
  if (!sp) CK(prompt_kv());
  // 9. q2 and gate2
  {
    Phase p("gemm_q2", st);
    CK(run_lin(lc, w->q2, b.n, D, T, f32 ? EPI_F32 : EPI_BF16_SSQ, b.qkv, D, b.ssq, D));
  }
  {
    Phase p("gemm_gate2", st);
    CK(run_lin(lc, w->g2, b.n, D, T, EPI_GATE2SIG_F32, b.gate, w->G));
  }
  // 10. q2 / k2 norms (no RoPE in cross-attention, ltx/block.zig:304)
  {
  Phase p("qk_norm2", st);
  if (f32) {
    CK(qk_norm_rope_f32(static_cast<const float*>(b.qkv), D, w->qn2, nullptr, nullptr, T, D, static_cast<float*>(b.q), st));
    CK(qk_norm_rope_f32(static_cast<const float*>(b.kv2), 2 * D, w->kn2, nullptr, nullptr, S, D,
                        static_cast<float*>(b.k2), st));
  } else {
    CK(qk_norm_rope(b.qkv, D, b.ssq, 32, n_ssq, w->qn2, nullptr, nullptr, T, D, b.q, nullptr, st));
  }
  }
  // 11. cross-attention
  {
    Phase p("attn_cross", st);
    CK(attn(w, b.q, D, b.k2, D, col(b.kv2, D), 2 * D, b.o, b.gate, T, S, st));
  }
  // 12. x_ca = x_sa + (o2 Wo2^T + b) * ada8
  if (stage == LTXB_STAGE_S5_CA_OUT)
    return run_lin(lc, w->o2, b.o, D, T, EPI_RESID_F32, stage_out, D, nullptr, 0, nullptr, io->tstab, io->tidx, 8);
  {
    Phase p("gemm_o2", st);
    CK(run_lin(lc, w->o2, b.o, D, T, EPI_RESID_F32, b.x_ca, D, nullptr, 0, b.x_sa, io->tstab, io->tidx, 8));
  }
  // 13. FFN input
  if (stage == LTXB_STAGE_S6_FF_IN)
    return norm_modulate(b.x_ca, T, D, w->sst, io->tstab, io->tidx, c->K, 3, 4, stage_out, 1, nullptr, st);
  {
    Phase p("norm_mlp", st);
    CK(norm(b.x_ca, 2, 3, 4));
  }
  // 14. h = gelu(f W1^T)
  {
    Phase p("gemm_ff1", st);
    CK(run_lin(lc, w->ff1, b.n, D, T, EPI_GELU_BF16, b.h, FF));
  }
  // 15. out = x_ca + (h W2^T) * ada5
  if (stage == LTXB_STAGE_S7_FF_OUT) return run_lin(lc, w->ff2, b.h, FF, T, EPI_F32, stage_out, D);
  {
    Phase p("gemm_ff2", st);
    CK(run_lin(lc, w->ff2, b.h, FF, T, EPI_RESID_F32, io->out, D, nullptr, 0, b.x_ca, io->tstab, io->tidx, 5));
  }
#undef CK
  return LTXB_OK;
}

}  // namespace ltxb

using namespace ltxb;

extern "C" {

int ltxb_ring_step(int rank, int nranks, int step, int* compute_shard, int* recv_shard, int* next_rank,
                   int* prev_rank) {
  if (nranks < 1 || rank < 0 || rank >= nranks || step < 0 || step >= nranks)
    return set_error(LTXB_EINVAL, "ring step: rank %d / %d, step %d", rank, nranks, step);
  const RingStep x = ring_step(rank, nranks, step);
  if (compute_shard) *compute_shard = x.compute;
  if (recv_shard) *recv_shard = x.recv;
  if (next_rank) *next_rank = x.next;
  if (prev_rank) *prev_rank = x.prev;
  return LTXB_OK;
}

void ltxb_weights_free(ltxb_weights* w) {
  if (!w) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(w->device);
  for (void* p : w->allocs) cudaFree(p);
  cudaSetDevice(prev);
  delete w;
}

uint64_t ltxb_weights_bytes(const ltxb_weights* w) { return w ? w->bytes : 0; }

int ltxb_weights_upload(int device, const void* blob, uint64_t blob_bytes, const ltxb_entry* entries, int n_entries,
                        int block_idx, int mode, int qset, int hidden, int ff, ltxb_weights** out) {
  if (!out) return set_error(LTXB_EINVAL, "out is null");
  *out = nullptr;
  if (!blob || !entries || n_entries <= 0) return set_error(LTXB_EINVAL, "empty blob");
  if (mode < LTXB_MODE_F32 || mode > LTXB_MODE_INT8) return set_error(LTXB_EINVAL, "unknown mode %d", mode);
  if (mode == LTXB_MODE_INT8 && qset != LTXB_QSET_REF && qset != LTXB_QSET_EXT && qset != LTXB_QSET_QKV)
    return set_error(LTXB_EINVAL, "unknown quant set %d", qset);
  if (hidden <= 0 || hidden % 256 || ff <= 0 || ff % 256)
    return set_error(LTXB_EINVAL, "hidden (%d) and ff (%d) must be positive multiples of 256", hidden, ff);
  int rc = check_entries(entries, n_entries, blob_bytes);
  if (rc) return rc;
  rc = ltxb_init(device);
  if (rc) return rc;
  auto* w = new ltxb_weights();
  w->device = device;
  w->mode = mode;
  w->qset = qset;
  w->D = hidden;
  w->FF = ff;
  w->H = hidden / 128;
  w->G = (w->H + 31) / 32 * 32;
  Uploader u{&w->allocs, &w->bytes, static_cast<const uint8_t*>(blob), blob_bytes, entries, n_entries, block_idx};
  const int D = hidden, H = w->H;
  const bool q8 = mode == LTXB_MODE_INT8;
  const bool qo = q8 && qset == LTXB_QSET_EXT;
  const bool qf = q8 && qset != LTXB_QSET_QKV;
  rc = u.linear(w->qkv1, {"attn1_to_q", "attn1_to_k", "attn1_to_v"}, D, D, true, q8);
  if (!rc) rc = u.linear(w->g1, {"attn1_to_gate_logits"}, H, D, true, false, w->G - H);
  if (!rc) rc = u.linear(w->o1, {"attn1_to_out_0"}, D, D, true, qo);
  if (!rc) rc = u.linear(w->q2, {"attn2_to_q"}, D, D, true, q8);
  if (!rc) rc = u.linear(w->g2, {"attn2_to_gate_logits"}, H, D, true, false, w->G - H);
  if (!rc) rc = u.linear(w->kv2, {"attn2_to_k", "attn2_to_v"}, D, D, true, q8);
  if (!rc) rc = u.linear(w->o2, {"attn2_to_out_0"}, D, D, true, qo);
  if (!rc) rc = u.linear(w->ff1, {"ff_net_0_proj"}, ff, D, false, qf);
  if (!rc) rc = u.linear(w->ff2, {"ff_net_2"}, D, ff, false, qf);
  if (!rc) rc = u.tensor("attn1_q_norm_weight", LTXB_DT_BF16, D, 0, &w->qn1);
  if (!rc) rc = u.tensor("attn1_k_norm_weight", LTXB_DT_BF16, D, 0, &w->kn1);
  if (!rc) rc = u.tensor("attn2_q_norm_weight", LTXB_DT_BF16, D, 0, &w->qn2);
  if (!rc) rc = u.tensor("attn2_k_norm_weight", LTXB_DT_BF16, D, 0, &w->kn2);
  const void *sst = nullptr, *psst = nullptr;
  if (!rc) rc = u.tensor("scale_shift_table", LTXB_DT_F32, 9, D, &sst);
  if (!rc) rc = u.tensor("prompt_scale_shift_table", LTXB_DT_F32, 2, D, &psst);
  if (rc) {
    ltxb_weights_free(w);
    return rc;
  }
  w->sst = static_cast<const float*>(sst);
  w->psst = static_cast<const float*>(psst);
  *out = w;
  return LTXB_OK;
}

uint64_t ltxb_block_workspace_bytes(const ltxb_weights* w, const ltxb_config* cfg) {
  if (!w || !cfg) return 0;
  Bufs b;
  return layout(w, cfg, nullptr, b);
}

int ltxb_block_forward(const ltxb_weights* w, const ltxb_block_io* io, const ltxb_config* cfg, void* stream) {
  return run_block(w, io, cfg, LTXB_STAGE_BLOCK_OUT, nullptr, static_cast<cudaStream_t>(stream));
}

int ltxb_block_stage(const ltxb_weights* w, const ltxb_block_io* io, const ltxb_config* cfg, int stage,
                     float* stage_out, void* stream) {
  if (stage < 0 || stage > LTXB_STAGE_BLOCK_OUT) return set_error(LTXB_EINVAL, "unknown stage %d", stage);
  if (stage != LTXB_STAGE_BLOCK_OUT && !stage_out) return set_error(LTXB_EINVAL, "stage_out is null");
  if (stage == LTXB_STAGE_BLOCK_OUT) {
    int rc = run_block(w, io, cfg, stage, nullptr, static_cast<cudaStream_t>(stream));
    if (rc || !stage_out || stage_out == io->out) return rc;
    cudaError_t e = cudaMemcpyAsync(stage_out, io->out, (size_t)cfg->T * w->D * 4, cudaMemcpyDeviceToDevice,
                                    static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "stage copy");
  }
  return run_block(w, io, cfg, stage, stage_out, static_cast<cudaStream_t>(stream));
}

// ---- host-buffer pipeline ----
}  // extern "C"

struct ltxb_host_pipe {
  const ltxb_weights* w = nullptr;
  ltxb_config cfg{};
  ltxb_block_io io{};
  int device = 0;
  size_t bytes = 0;
  float* x_dev[2] = {nullptr, nullptr};
  float* out_dev[2] = {nullptr, nullptr};
  cudaStream_t h2d = nullptr, d2h = nullptr;
  cudaEvent_t h2d_done[2] = {}, comp_done[2] = {}, d2h_done[2] = {}, start = nullptr;
  int64_t calls = 0;
  bool fresh = true;
};

extern "C" {

void ltxb_host_pipe_free(ltxb_host_pipe* p) {
  if (!p) return;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(p->device);
  if (p->h2d) cudaStreamSynchronize(p->h2d);
  if (p->d2h) cudaStreamSynchronize(p->d2h);
  for (int i = 0; i < 2; ++i) {
    if (p->x_dev[i]) cudaFree(p->x_dev[i]);
    if (p->out_dev[i]) cudaFree(p->out_dev[i]);
    if (p->h2d_done[i]) cudaEventDestroy(p->h2d_done[i]);
    if (p->comp_done[i]) cudaEventDestroy(p->comp_done[i]);
    if (p->d2h_done[i]) cudaEventDestroy(p->d2h_done[i]);
  }
  if (p->start) cudaEventDestroy(p->start);
  if (p->h2d) cudaStreamDestroy(p->h2d);
  if (p->d2h) cudaStreamDestroy(p->d2h);
  cudaSetDevice(prev);
  delete p;
}

int ltxb_host_pipe_create(const ltxb_weights* w, const ltxb_config* cfg, const ltxb_block_io* tables,
                          ltxb_host_pipe** out) {
  if (!out) return set_error(LTXB_EINVAL, "out is null");
  *out = nullptr;
  if (!w || !cfg || !tables) return set_error(LTXB_EINVAL, "null argument");
  if (cfg->T <= 0) return set_error(LTXB_EINVAL, "T must be positive");
  auto* p = new ltxb_host_pipe();
  p->w = w;
  p->cfg = *cfg;
  p->io = *tables;
  p->device = w->device;
  p->bytes = (size_t)cfg->T * w->D * sizeof(float);
  cudaSetDevice(w->device);
  bool ok = true;
  for (int i = 0; i < 2 && ok; ++i) {
    ok = cudaMalloc(&p->x_dev[i], p->bytes) == cudaSuccess && cudaMalloc(&p->out_dev[i], p->bytes) == cudaSuccess &&
         cudaEventCreateWithFlags(&p->h2d_done[i], cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&p->comp_done[i], cudaEventDisableTiming) == cudaSuccess &&
         cudaEventCreateWithFlags(&p->d2h_done[i], cudaEventDisableTiming) == cudaSuccess;
  }
  ok = ok && cudaEventCreateWithFlags(&p->start, cudaEventDisableTiming) == cudaSuccess &&
       cudaStreamCreateWithFlags(&p->h2d, cudaStreamNonBlocking) == cudaSuccess &&
       cudaStreamCreateWithFlags(&p->d2h, cudaStreamNonBlocking) == cudaSuccess;
  if (!ok) {
    ltxb_host_pipe_free(p);
    return set_error(LTXB_ENOMEM, "host pipe: staging allocation failed");
  }
  *out = p;
  return LTXB_OK;
}

int ltxb_block_forward_host(ltxb_host_pipe* p, const float* x_host, float* out_host, void* stream) {
  if (!p || !x_host || !out_host) return set_error(LTXB_EINVAL, "null argument");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int b = (int)(p->calls & 1);
  if (p->fresh) {  // the first copy of a run starts after the caller's earlier work
    cudaEventRecord(p->start, st);
    cudaStreamWaitEvent(p->h2d, p->start, 0);
    p->fresh = false;
  }
  // x_dev[b] was last read by the compute of call k-2
  if (p->calls >= 2) cudaStreamWaitEvent(p->h2d, p->comp_done[b], 0);
  cudaError_t e = cudaMemcpyAsync(p->x_dev[b], x_host, p->bytes, cudaMemcpyHostToDevice, p->h2d);
  if (e != cudaSuccess) return set_cuda_error(e, "host pipe: H2D");
  cudaEventRecord(p->h2d_done[b], p->h2d);
  cudaStreamWaitEvent(st, p->h2d_done[b], 0);
  // out_dev[b] was last copied out by the D2H of call k-2
  if (p->calls >= 2) cudaStreamWaitEvent(st, p->d2h_done[b], 0);
  ltxb_block_io io = p->io;
  io.x = p->x_dev[b];
  io.out = p->out_dev[b];
  int rc = run_block(p->w, &io, &p->cfg, LTXB_STAGE_BLOCK_OUT, nullptr, st);
  if (rc) return rc;
  cudaEventRecord(p->comp_done[b], st);
  cudaStreamWaitEvent(p->d2h, p->comp_done[b], 0);
  e = cudaMemcpyAsync(out_host, p->out_dev[b], p->bytes, cudaMemcpyDeviceToHost, p->d2h);
  if (e != cudaSuccess) return set_cuda_error(e, "host pipe: D2H");
  cudaEventRecord(p->d2h_done[b], p->d2h);
  p->calls += 1;
  return LTXB_OK;
}

int ltxb_host_pipe_join(ltxb_host_pipe* p, void* stream) {
  if (!p) return set_error(LTXB_EINVAL, "null pipe");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int i = 0; i < 2 && i < p->calls; ++i) {
    cudaStreamWaitEvent(st, p->d2h_done[i], 0);
    cudaStreamWaitEvent(st, p->h2d_done[i], 0);
  }
  p->fresh = true;
  return LTXB_OK;
}

// ---- communicator ----
int ltxb_comm_id_bytes(void) { return (int)sizeof(ncclUniqueId); }

int ltxb_comm_get_id(void* id) {
  if (!id) return set_error(LTXB_EINVAL, "id is null");
  ncclResult_t r = ncclGetUniqueId(static_cast<ncclUniqueId*>(id));
  return r == ncclSuccess ? LTXB_OK : set_error(LTXB_ENCCL, "ncclGetUniqueId: %s", ncclGetErrorString(r));
}

int ltxb_comm_init(const void* id, int rank, int nranks, int device, ltxb_comm** out) {
  if (!id || !out || nranks < 1 || rank < 0 || rank >= nranks) return set_error(LTXB_EINVAL, "bad communicator args");
  *out = nullptr;
  int rc = ltxb_init(device);
  if (rc) return rc;
  auto* c = new ltxb_comm();
  c->rank = rank;
  c->nranks = nranks;
  c->device = device;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclResult_t r = ncclCommInitRank(&c->nccl, nranks, uid, rank);
  if (r != ncclSuccess) {
    delete c;
    return set_error(LTXB_ENCCL, "ncclCommInitRank: %s", ncclGetErrorString(r));
  }
  int prio_lo = 0, prio_hi = 0;  // collectives get SMs ahead of queued compute blocks
  cudaDeviceGetStreamPriorityRange(&prio_lo, &prio_hi);
  if (cudaStreamCreateWithPriority(&c->comm_stream, cudaStreamNonBlocking, prio_hi) != cudaSuccess) {
    ncclCommDestroy(c->nccl);
    delete c;
    return set_error(LTXB_ECUDA, "comm stream");
  }
  c->ev.resize(std::max(2 * nranks + 2, 32));
  for (auto& e : c->ev) cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
  // the peer-memory exchange: map a header-sized window of every rank now,
  // so that every rank knows before the first block call (and before any
  // workspace query) whether the exchange is available; it grows on first use
  if (nranks > 1 && nranks <= kMaxPeers && cudaMalloc(&c->xbuf, (size_t)nranks * 128) == cudaSuccess)
    c->peer_ok = win_setup(c, kWinHdr) == LTXB_OK;  // if not, the NCCL exchanges remain
  cudaGetLastError();
  *out = c;
  return LTXB_OK;
}

int ltxb_comm_peer_mapped(const ltxb_comm* c) { return c && c->peer_ok ? 1 : 0; }

void ltxb_comm_free(ltxb_comm* c) {
  if (!c) return;
  if (c->comm_stream) cudaStreamSynchronize(c->comm_stream);
  cudaDeviceSynchronize();  // this rank's kernels that use the peer windows are done
  win_release(c);
  if (c->xbuf) cudaFree(c->xbuf);
  for (auto& e : c->ev) cudaEventDestroy(e);
  if (c->nccl) ncclCommDestroy(c->nccl);
  if (c->comm_stream) cudaStreamDestroy(c->comm_stream);
  delete c;
}

int ltxb_comm_check(ltxb_comm* c) {
  if (!c || !c->nccl) return set_error(LTXB_EINVAL, "comm check: null communicator");
  ncclResult_t async = ncclSuccess;
  ncclResult_t r = ncclCommGetAsyncError(c->nccl, &async);
  if (r != ncclSuccess) return set_error(LTXB_ENCCL, "ncclCommGetAsyncError: %s", ncclGetErrorString(r));
  if (async != ncclSuccess && async != ncclInProgress)
    return set_error(LTXB_ENCCL, "communicator error: %s", ncclGetErrorString(async));
  return LTXB_OK;
}

void ltxb_comm_abort(ltxb_comm* c) {
  if (!c) return;
  // abort first: it ends the NCCL kernels still waiting for peers, so the
  // streams and events below no longer depend on a rank that is gone
  if (c->nccl) ncclCommAbort(c->nccl);
  win_release(c);  // waits only for this rank's kernels, whose peer waits are bounded
  if (c->xbuf) cudaFree(c->xbuf);
  for (auto& e : c->ev) cudaEventDestroy(e);
  if (c->comm_stream) cudaStreamDestroy(c->comm_stream);  // releases once its work has ended
  delete c;
}

// ---- standalone operators ----
int ltxb_attention(const void* q, const void* k, const void* v, void* out, const float* gate, int Tq, int Tkv, int H,
                   float scale, void* stream) {
  AttnArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.ldq = a.ldk = a.ldv = H * 128;
  a.out = out;
  a.gate = gate;
  a.ldg = H;
  a.Tq = Tq;
  a.Tkv = Tkv;
  a.H = H;
  a.scale = scale;
  return attention_tc(a, static_cast<cudaStream_t>(stream));
}

int ltxb_rope_tables(int kind, const float* pos, int T, int H, double theta, float* cos, float* sin, void* stream) {
  return rope_tables(kind, pos, T, H, theta, cos, sin, static_cast<cudaStream_t>(stream));
}

static int split_count(int Tq, int Tkv, int H, int splits) {
  const int nkv = (Tkv + 127) / 128;
  if (splits <= 0) return attention_kv_splits(Tq, Tkv, H, 8);
  return splits < nkv ? splits : nkv;
}

static uint64_t split_ws(int Tq, int H, int ns, size_t* o_off, size_t* m_off, size_t* l_off) {
  auto up = [](uint64_t x) { return (x + 255) & ~uint64_t(255); };
  const uint64_t ob = up((uint64_t)ns * Tq * H * 128 * 4), sb = up((uint64_t)ns * H * Tq * 4);
  if (o_off) *o_off = 0;
  if (m_off) *m_off = ob;
  if (l_off) *l_off = ob + sb;
  return ob + 2 * sb;
}

uint64_t ltxb_attention_split_workspace_bytes(int Tq, int Tkv, int H, int splits) {
  if (Tq <= 0 || Tkv <= 0 || H <= 0) return 0;
  return split_ws(Tq, H, split_count(Tq, Tkv, H, splits), nullptr, nullptr, nullptr);
}

int ltxb_attention_split(const void* q, const void* k, const void* v, void* out, const float* gate, int Tq, int Tkv,
                         int H, float scale, int splits, void* workspace, uint64_t workspace_bytes, void* stream) {
  if (Tq <= 0) return LTXB_OK;
  if (Tkv <= 0 || H <= 0) return set_error(LTXB_EINVAL, "attention split: empty K/V or no heads");
  if (splits < 0) return set_error(LTXB_EINVAL, "attention split: negative split count");
  const int ns = split_count(Tq, Tkv, H, splits);
  size_t oo, mo, lo;
  const uint64_t need = split_ws(Tq, H, ns, &oo, &mo, &lo);
  if (!workspace || workspace_bytes < need)
    return set_error(LTXB_EINVAL, "attention split: workspace of %llu bytes is smaller than the %llu required",
                     (unsigned long long)workspace_bytes, (unsigned long long)need);
  if (reinterpret_cast<uintptr_t>(workspace) & 255) return set_error(LTXB_EINVAL, "workspace must be 256-byte aligned");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  AttnArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.ldq = a.ldk = a.ldv = H * 128;
  a.out = out;
  a.gate = gate;
  a.ldg = H;
  a.Tq = Tq;
  a.Tkv = Tkv;
  a.H = H;
  a.scale = scale;
  a.o_acc = reinterpret_cast<float*>(ws + oo);
  a.m_state = reinterpret_cast<float*>(ws + mo);
  a.l_state = reinterpret_cast<float*>(ws + lo);
  return attention_split(a, ns, static_cast<cudaStream_t>(stream));
}

int ltxb_dq_gemm(const void* A, const void* Wq, const void* scales, int scale_dtype, const void* bias, void* out, int M,
                 int N, int K, int fused, void* workspace, uint64_t workspace_bytes, void* stream) {
  if (scale_dtype != LTXB_DT_F32 && scale_dtype != LTXB_DT_BF16) return set_error(LTXB_EINVAL, "scale dtype");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  GemmArgs g{};
  g.A = A;
  g.lda = K;
  g.M = M;
  g.N = N;
  g.K = K;
  g.epi = EPI_BF16;
  g.bias = bias;
  g.out = out;
  g.ldo = N;
  if (fused) {
    g.B = Wq;
    g.ldb = K;
    g.b_int8 = 1;
    g.scales = scales;
    g.scale_bf16 = scale_dtype == LTXB_DT_BF16;
  } else {
    if (!workspace || workspace_bytes < (uint64_t)N * K * 2)
      return set_error(LTXB_EINVAL, "dq_gemm: unfused path needs N*K*2 workspace bytes");
    g.B = workspace;
    g.ldb = K;
    // all checks before the expansion launch
    if (int rc = gemm_check(g, nullptr)) return rc;
    if ((reinterpret_cast<uintptr_t>(Wq) & 15) ||
        (reinterpret_cast<uintptr_t>(scales) & (scale_dtype == LTXB_DT_BF16 ? 1 : 3)))
      return set_error(LTXB_EINVAL, "dq_gemm: weights must be 16-byte aligned, scales element-aligned");
    int rc = dequant_weights(static_cast<const int8_t*>(Wq), scales, scale_dtype == LTXB_DT_BF16, N, K, workspace, st);
    if (rc) return rc;
  }
  return gemm_tc(g, st);
}

int ltxb_gemm_bf16(const void* A, const void* W, const void* bias, void* out, int M, int N, int K, void* stream) {
  GemmArgs g{};
  g.A = A;
  g.lda = K;
  g.B = W;
  g.ldb = K;
  g.M = M;
  g.N = N;
  g.K = K;
  g.epi = EPI_BF16;
  g.bias = bias;
  g.out = out;
  g.ldo = N;
  return gemm_tc(g, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
