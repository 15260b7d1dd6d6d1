/*
 * ltxb.h -- C ABI of libltxb.so, a B200-native (sm_100a) LTX-2.5 DiT block.
 *
 * The library replaces the reference's traced block executable
 * (ABSatVPS/ltx-zml, ltx/block.zig) and its device upload path
 * (ltx/loader.zig) behind a plain extern-C boundary: plain pointers and
 * sizes, opaque handles, status codes. No torch or CUDA C++ types appear in
 * the signatures; `stream` is a cudaStream_t passed as void*.
 *
 * Conventions
 *  - Every function returns LTXB_OK (0) or a negative LTXB_E* code; the
 *    message of the last failure on the calling thread is ltxb_last_error().
 *    (The reference's boundary uses Zig error unions, ltx/loader.zig:63-128,
 *    and the in-repo C-ABI precedent coli-zml/coli/abi.zig:1-10 returns
 *    1/0; negative codes keep the error kind.)
 *  - All device memory passed in is caller-owned and stream-ordered. Compute
 *    entry points enqueue work on `stream` and return without a host sync;
 *    device-side failures of bounded waits surface through
 *    ltxb_device_status().
 *  - Compute entry points run on the calling thread's current device, which
 *    must be the device a weights / core handle was uploaded to (LTXB_EINVAL
 *    otherwise, before anything is launched).
 *  - Layouts are row-major. Activations are token-major [T, D] with D = H*128
 *    and heads concatenated (head h occupies columns [128h, 128h+128)).
 *  - Weights are [out, in] row-major as in the checkpoint; int8 weights carry
 *    grouped-128 scales [out, in/128] (f32 as the reference stores them,
 *    tools/quantize_block.py:70-73, or bf16 as the BASELINE configs ask).
 */
#ifndef LTXB_H
#define LTXB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define LTXB_OK 0
#define LTXB_EINVAL (-1)      /* bad argument / shape / alignment */
#define LTXB_ECUDA (-2)       /* a CUDA runtime or driver call failed */
#define LTXB_ENOMEM (-3)      /* device or host allocation failed */
#define LTXB_ELAYOUT (-4)     /* blob layout: Misaligned / LayoutGap / TrailingBytes */
#define LTXB_EMISSING (-5)    /* blob has no entry of a required name */
#define LTXB_EDTYPE (-6)      /* blob entry has the wrong dtype or shape */
#define LTXB_ENCCL (-7)       /* an NCCL call failed */
#define LTXB_ETIMEOUT (-8)    /* a bounded device wait expired */
#define LTXB_EUNSUPPORTED (-9)/* valid request this build does not implement */

/* ---- enums ------------------------------------------------------------- */
#define LTXB_DT_BF16 0
#define LTXB_DT_F32 1
#define LTXB_DT_I8 2

/* Precision modes of a block (ltxb_weights_upload / ltxb_config.mode). */
#define LTXB_MODE_F32 0   /* reference `Block`: bf16 weights upcast, f32 math     */
#define LTXB_MODE_BF16 1  /* bf16 weights, bf16 activations on tcgen05, f32 accum */
#define LTXB_MODE_INT8 2  /* reference `QBlock`: int8 g128 q/k/v (x2) + FFN       */

/* Which linears LTXB_MODE_INT8 takes int8 (ltx/loader.zig:147-156 for the
 * reference set; BASELINE config 3 also quantises the output projections;
 * QBlock.qBlockOut, ltx/block.zig:577-611, keeps the FFN unquantised). */
#define LTXB_QSET_REF 0   /* q1,k1,v1,q2,k2,v2,ff1,ff2 (qBlockOutAll)            */
#define LTXB_QSET_EXT 1   /* LTXB_QSET_REF + o1,o2                               */
#define LTXB_QSET_QKV 2   /* q1,k1,v1,q2,k2,v2; FFN bf16 (qBlockOut)             */

/* Stage selectors for ltxb_block_stage (ltx/block_conformance.zig:311-322). */
#define LTXB_STAGE_S1_NORM_MSA 0
#define LTXB_STAGE_S1B_QNORM 1
#define LTXB_STAGE_S2_ATTN1_NOGATE 2
#define LTXB_STAGE_S3_ATTN1 3
#define LTXB_STAGE_S4_AFTER_SA 4
#define LTXB_STAGE_S4_NORMED 5
#define LTXB_STAGE_S5_CA_OUT 6
#define LTXB_STAGE_S6_FF_IN 7
#define LTXB_STAGE_S7_FF_OUT 8
#define LTXB_STAGE_BLOCK_OUT 9

/* ---- library ----------------------------------------------------------- */

/* Initialise the library on one CUDA device (sets it current on the calling
 * thread, resolves the TMA encoder). Replaces `Platform.auto`
 * (ltx/e2e_prod.zig:187-189). Idempotent. */
int ltxb_init(int device);

/* Message for the last failure on the calling thread ("" if none). */
const char* ltxb_last_error(void);

/* Library version string. */
const char* ltxb_version(void);

/* Read (and, if clear != 0, reset) the device status word of the current
 * device: LTXB_OK, or LTXB_ETIMEOUT when a kernel's bounded mbarrier/peer
 * wait expired; *site (optional) receives the failing wait's site code.
 * Synchronises the device. */
int ltxb_device_status(int clear, uint32_t* site);

/* Failure-detection self-test: one kernel waits, bounded by limit_us
 * (1 us .. 2 s), on an mbarrier that nothing arrives on -- the path every
 * kernel's waits take when a producer is lost. Afterwards
 * ltxb_device_status reports LTXB_ETIMEOUT with site LTXB_SELFTEST_SITE;
 * the context stays usable once the status is cleared (no fault, no hang). */
#define LTXB_SELFTEST_SITE 0x7E0
int ltxb_selftest_wait(uint32_t limit_us, void* stream);

/* ---- measurement -------------------------------------------------------- */

/* Kernels this library has launched in this process (all devices). */
uint64_t ltxb_launch_count(void);

/* Per-phase device timing of the block's launch sequence (CUDA events around
 * each phase on the caller's stream). Off by default; the reference's
 * equivalent is host wall-clock around synchronised calls
 * (ltx/smoke.zig:243-254). */
int ltxb_profile_enable(int on);

/* Synchronise the recorded events and accumulate them per phase name.
 * Writes up to max_phases rows: names (name_stride bytes each), total device
 * milliseconds, kernel launches, and calls; returns the number of phases
 * (or a negative error). reset != 0 clears the accumulators afterwards. */
int ltxb_profile_collect(int max_phases, char* names, int name_stride, double* total_ms, uint64_t* launches,
                         int* calls, int reset);

/* ---- weights (ltx/loader.zig:133-172) ---------------------------------- */

/* One entry of a packed block blob, in the format of tools/pack_block.py:
 * `name` is the checkpoint name ("transformer_blocks.{i}.attn1.to_q.weight",
 * companions "...::q8" / "...::q8scale"), matched after the reference's
 * normalisation ('.' and '::' -> '_', ltx/loader.zig:102-129). */
typedef struct {
  const char* name;
  int32_t dtype;       /* LTXB_DT_* */
  int32_t ndim;        /* 1 or 2 */
  int64_t shape[2];
  uint64_t offset;     /* bytes from the blob start */
  uint64_t nbytes;
} ltxb_entry;

typedef struct ltxb_weights ltxb_weights;

/* Check the blob layout (ltx/loader.zig:73-82: 64-byte aligned offsets, gaps
 * only alignment fill, no trailing bytes) without uploading anything.
 * Returns LTXB_ELAYOUT with the reference's error name in the message. */
int ltxb_blob_check_layout(const ltxb_entry* entries, int n_entries, uint64_t blob_bytes, uint32_t align);

/* ---- native blob reader (tools/pack_block.py's format) ----
 * ltxb_blob_open reads <dir>/blob_manifest.json and maps <dir>/blob.bin
 * read-only, as Blob.open does (ltx/loader.zig:50-69): blob.bin's size must
 * equal total_bytes (ELAYOUT "BlobSizeMismatch"), the layout must pass
 * ltxb_blob_check_layout, and `verify` selects SHA-256 checks: the whole
 * blob against blob_sha256 (the loader's first-touch check,
 * ltx/loader.zig:270-276) and/or every entry against its own digest (ELAYOUT
 * "BlobDigestMismatch"). Missing files: EMISSING. Entry dtypes other than
 * BF16 / F32 / I8 read as -1; shape[] holds the first two dimensions. */
typedef struct ltxb_blob ltxb_blob;
#define LTXB_VERIFY_BLOB 1
#define LTXB_VERIFY_ENTRIES 2
int ltxb_blob_open(const char* dir, int verify, ltxb_blob** out);
void ltxb_blob_close(ltxb_blob* blob);
/* The mapped bytes and the manifest's entries, valid until ltxb_blob_close:
 * what ltxb_weights_upload / ltxb_core_upload take. Any output may be NULL. */
int ltxb_blob_view(const ltxb_blob* blob, const void** data, uint64_t* bytes, const ltxb_entry** entries,
                   int* n_entries, uint32_t* align, int64_t* block);
/* findEntry (ltx/loader.zig:122-129): the entry whose normalised name
 * ('.' and '::' -> '_') is `name`; EMISSING otherwise. */
int ltxb_blob_find(const ltxb_blob* blob, const char* name, const ltxb_entry** out);
/* The digest checks of ltxb_blob_open on an open blob. */
int ltxb_blob_verify(const ltxb_blob* blob, int verify);
/* SHA-256 (FIPS 180-4) of a host buffer: 64 lowercase hex digits + NUL. */
void ltxb_sha256_hex(const void* data, uint64_t bytes, char hex[65]);
/* Which SHA-256 code runs: portable_only != 0 forces the portable C++ path;
 * 0 uses the x86 SHA extensions when the CPU has them. Returns 1 when the
 * extensions are in use. For tests that compare the two. */
int ltxb_sha256_impl(int portable_only);

/* ---- streaming staging of blobs (ltx/loader.zig:176-321) ----
 * Two host slots (page-locked when pinned != 0, so device copies from them
 * run at the link's full rate) and a reader thread: for schedule position
 * pos = 0, 1, ... the thread waits for a free slot, checks the blob's digest
 * on its first touch (verify != 0), and copies blobs[schedule[pos]] into the
 * slot while the caller uploads from the other one. The caller takes the
 * positions in order: ltxb_stage_acquire (bounded by timeout_ms:
 * LTXB_ETIMEOUT), upload, ltxb_stage_release -- or ltxb_stage_upload, which
 * does the three for a block's weights. Slots move free -> filling -> ready
 * -> in_use -> free; any other move is LTXB_EINVAL. Checked before any I/O:
 * every schedule entry names a blob ("ScheduleOutOfRange") and fits a slot
 * ("SlotTooSmall"). A reader failure (e.g. "BlobDigestMismatch") is returned
 * by every acquire of a position not staged before it; after
 * ltxb_stage_abort acquire returns "RingShutdown". The blobs must stay open
 * while the stage exists. */
typedef struct ltxb_stage ltxb_stage;
typedef struct {
  uint64_t reader_parks;    /* reader waits for a free slot   */
  uint64_t consumer_parks;  /* acquire waits for a ready slot */
  uint64_t copy_ns;         /* reader time copying into slots */
  uint64_t verify_ns;       /* reader time hashing blobs      */
  uint64_t staged_bytes;
} ltxb_stage_stats;
int ltxb_stage_create(const ltxb_blob* const* blobs, int n_blobs, const int* schedule, int n_schedule,
                      uint64_t slot_bytes, int pinned, int verify, ltxb_stage** out);
int ltxb_stage_acquire(ltxb_stage* stage, int pos, const void** data, uint64_t* bytes, uint32_t timeout_ms);
int ltxb_stage_release(ltxb_stage* stage, int pos);
int ltxb_stage_upload(ltxb_stage* stage, int pos, int device, int block_idx, int mode, int qset, int hidden, int ff,
                      uint32_t timeout_ms, ltxb_weights** out);
int ltxb_stage_get_stats(ltxb_stage* stage, ltxb_stage_stats* out);
void ltxb_stage_abort(ltxb_stage* stage);
void ltxb_stage_free(ltxb_stage* stage);

/* Upload one block's weights from a host blob into device-resident buffers
 * on `device` (replaces buildBlockBufs + buildQuantBufs, ltx/loader.zig:
 * 133-172). mode LTXB_MODE_F32/BF16 uploads the 28 base tensors; mode
 * LTXB_MODE_INT8 uploads the int8/scale pairs of `qset` instead of those
 * matrices' bf16 copies. `hidden` (D) and `ff` (FF) give the geometry
 * (4096 / 16384 for LTX-2.5; D a multiple of 256, FF of 256). The device
 * allocations are owned by the returned handle. Synchronous. */
int ltxb_weights_upload(int device, const void* blob, uint64_t blob_bytes, const ltxb_entry* entries,
                        int n_entries, int block_idx, int mode, int qset, int hidden, int ff,
                        ltxb_weights** out);

/* Device bytes held by a weights handle. */
uint64_t ltxb_weights_bytes(const ltxb_weights* w);

/* Free a weights handle (and its device buffers). NULL is a no-op. */
void ltxb_weights_free(ltxb_weights* w);

/* ---- sequence-parallel communicator ------------------------------------ */

typedef struct ltxb_comm ltxb_comm;

/* Size of the opaque unique id rank 0 creates and every rank receives. */
int ltxb_comm_id_bytes(void);
/* Rank 0: fill `id` (ltxb_comm_id_bytes() bytes). */
int ltxb_comm_get_id(void* id);
/* Every rank: join the group (NCCL over NVLink; one rank per GPU). With
 * 2..8 ranks in separate processes it also maps a window of device memory of
 * every other rank (CUDA IPC) for the head-parallel exchange over peer
 * memory; the windows grow, collectively and synchronously, on the first
 * block call of a new shape. */
int ltxb_comm_init(const void* id, int rank, int nranks, int device, ltxb_comm** out);
/* 1 when every rank mapped every other rank's window, so that
 * sequence-parallel block calls can exchange q/k/v and attention rows by
 * stores into peer memory; 0 when only the NCCL exchanges are available. No
 * counterpart in the reference (single device). */
int ltxb_comm_peer_mapped(const ltxb_comm* c);
/* Waits for the communicator's queued transfers, then frees it. */
void ltxb_comm_free(ltxb_comm* c);
/* The error NCCL has recorded on the communicator, if any
 * (ncclCommGetAsyncError): LTXB_OK or LTXB_ENCCL with NCCL's message. A host
 * watchdog polls it while block calls are in flight. */
int ltxb_comm_check(ltxb_comm* c);
/* Frees the communicator without waiting (ncclCommAbort): for a host that
 * knows a peer rank is gone. Collectives in flight on it end without
 * completing; the block calls that used it must be treated as failed and
 * their outputs discarded. */
void ltxb_comm_abort(ltxb_comm* c);

/* Ring schedule of the sequence-parallel self-attention (host-side, no GPU):
 * at step s (0 <= s < nranks) rank r computes against K/V shard
 * *compute_shard while sending that shard to *next_rank and receiving
 * *recv_shard from *prev_rank (recv_shard = -1 on the last step). Shard i
 * holds tokens [i T, (i+1) T). Pure function; the block's ring follows it. */
int ltxb_ring_step(int rank, int nranks, int step, int* compute_shard, int* recv_shard, int* next_rank,
                   int* prev_rank);

/* ---- the block (ltx/block.zig:340-353, :544-574) ----------------------- */

typedef struct {
  int32_t T;          /* video tokens held by this rank (T_total / sp_size) */
  int32_t S;          /* text (context) tokens                              */
  int32_t K;          /* rows of the timestep table tstab                   */
  int32_t mode;       /* LTXB_MODE_*; must match the weights' mode          */
  int32_t sp_rank;    /* sequence-parallel rank (0 when sp_size == 1)       */
  int32_t sp_size;    /* ranks sharing the T_total tokens                   */
  ltxb_comm* comm;    /* required when sp_size > 1                          */
} ltxb_config;

/* Per-call tensors (device pointers). Shapes for one rank:
 *   x, out   [T, D] f32   (out may alias x)
 *   tstab    [K, 9, D] f32, tidx [T] int32   -- ada rows (ltx/block.zig:47-67); token t
 *            reads row tidx[t], or row 0 when tidx[t] is outside [0, K) (the
 *            reference's select chain)
 *   ctx      [S, D] f32, pts2 [2, D] f32     -- cross-attention K/V modulation
 *   cos, sin [T, H, 64] f32                  -- split-half RoPE tables
 *   workspace: ltxb_block_workspace_bytes(cfg) bytes, 256-byte aligned.
 * The f32 tensors must be 16-byte aligned (the kernels move 16-byte vectors)
 * and tidx 4-byte aligned; a NULL tidx reads row 0 for every token. */
typedef struct {
  const float* x;
  float* out;
  const float* tstab;
  const int32_t* tidx;
  const float* ctx;
  const float* pts2;
  const float* cos;
  const float* sin;
  void* workspace;
  uint64_t workspace_bytes;
} ltxb_block_io;

/* Workspace the block needs for `cfg` on weights `w`. */
uint64_t ltxb_block_workspace_bytes(const ltxb_weights* w, const ltxb_config* cfg);

/* out = block(x): the whole block, blockwise (flash) self-attention. The
 * equivalent of exe.call on `wBlockOut` / `qBlockOutAll`
 * (ltx/e2e_prod.zig:377-395). With sp_size > 1 the ranks exchange K/V
 * over NVLink (a head-group pipelined all-gather; the send/recv ring with
 * the environment variable LTXB_SP_RING=1); each rank holds its token slice. */
int ltxb_block_forward(const ltxb_weights* w, const ltxb_block_io* io, const ltxb_config* cfg, void* stream);

/* One conformance stage (LTXB_STAGE_*) of the block, written to stage_out
 * [T, D] f32 -- the staged methods s1NormMsa ... blockOut
 * (ltx/block.zig:248-353, gated by ltx/block_conformance.zig:311-350).
 * Single rank only. */
int ltxb_block_stage(const ltxb_weights* w, const ltxb_block_io* io, const ltxb_config* cfg, int stage,
                     float* stage_out, void* stream);

/* ---- host-buffer pipeline ---------------------------------------------- */

/* For callers whose activations live in host memory (the reference uploads
 * x from the host with zml.Buffer.fromBytes and reads the block output back
 * with toSliceAlloc, ltx/e2e_prod.zig:377-395): a pipe owns two device
 * staging pairs (x, out) and two copy streams, so consecutive
 * ltxb_block_forward_host calls overlap the host->device copy of call k and
 * the device->host copy of call k-1 with the compute of call k. Every call
 * still copies its whole input in and its whole result out. */
typedef struct ltxb_host_pipe ltxb_host_pipe;

/* `tables` supplies the per-call device tensors other than x/out (tstab,
 * tidx, ctx, pts2, cos, sin) and the workspace; they must outlive the pipe.
 * The pipe allocates 4 * T * D * 4 bytes of staging memory. */
int ltxb_host_pipe_create(const ltxb_weights* w, const ltxb_config* cfg, const ltxb_block_io* tables,
                          ltxb_host_pipe** out);

/* Enqueue one block call: x_host [T, D] f32 -> out_host [T, D] f32 (pinned
 * host memory gives full copy bandwidth). Compute runs on `stream`. x_host
 * must stay unchanged and out_host unread until ltxb_host_pipe_join(). */
int ltxb_block_forward_host(ltxb_host_pipe* p, const float* x_host, float* out_host, void* stream);

/* Make `stream` wait for every copy the pipe has enqueued, so synchronising
 * `stream` (or an event recorded on it afterwards) covers all results. */
int ltxb_host_pipe_join(ltxb_host_pipe* p, void* stream);

void ltxb_host_pipe_free(ltxb_host_pipe* p);

/* ---- standalone operators (BASELINE configs 1 and 2) ------------------- */

/* Non-causal softmax attention, softmax(q k^T * scale) v, for H heads of
 * 128 dims: q [Tq, H, 128], k/v [Tkv, H, 128], out [Tq, H, 128], all bf16
 * (token-major, the block's layout). Blockwise online softmax (the
 * reference's whileSdpa, ltx/block.zig:105-154; dense zml.nn.sdpa at
 * ltx/block.zig:234 is the same function). `gate` (optional, f32 [Tq, H])
 * multiplies each head's output (the block's 2*sigmoid gate). */
int ltxb_attention(const void* q, const void* k, const void* v, void* out, const float* gate, int Tq, int Tkv,
                   int H, float scale, void* stream);

/* Split-K/V form of ltxb_attention for short query sequences (a
 * sequence-parallel rank's shard against the whole sequence): the K/V tiles
 * are divided into `splits` ranges (0 = the count that best fills the GPU),
 * each computed into its own f32 partial state (m, l, O) in `workspace`,
 * then merged into `out`, so that the grid covers the SMs evenly. The merge
 * is the online-softmax combine of the reference's whileSdpa carries
 * (ltx/block.zig:105-154). Same arguments and results as ltxb_attention
 * otherwise; `workspace` (256-byte aligned) holds
 * ltxb_attention_split_workspace_bytes(Tq, Tkv, H, splits) bytes. */
uint64_t ltxb_attention_split_workspace_bytes(int Tq, int Tkv, int H, int splits);
int ltxb_attention_split(const void* q, const void* k, const void* v, void* out, const float* gate, int Tq, int Tkv,
                         int H, float scale, int splits, void* workspace, uint64_t workspace_bytes, void* stream);

/* out[M, N] (bf16) = A[M, K] (bf16) . dequant(Wq[N, K] int8, scales[N, K/128])^T
 * (+ bias[N] bf16, optional): the int8 grouped-128 dequant linear `linQ`
 * (ltx/block.zig:462-477). scale_dtype LTXB_DT_F32 or LTXB_DT_BF16.
 * fused != 0 dequantises tiles in shared memory inside the GEMM;
 * fused == 0 expands the weights into `workspace` (N*K*2 bytes) with a
 * bandwidth-bound pass and runs the bf16 GEMM. Shapes: K a multiple of 128,
 * N of 128 (fused) or 32. A, Wq, bias, out and workspace 16-byte aligned (TMA and the
 * epilogue's 16-byte vectors); scales aligned to their element size.
 * Misaligned pointers or unsupported shapes return LTXB_EINVAL before
 * anything is launched. */
int ltxb_dq_gemm(const void* A, const void* Wq, const void* scales, int scale_dtype, const void* bias, void* out,
                 int M, int N, int K, int fused, void* workspace, uint64_t workspace_bytes, void* stream);

/* RoPE tables on the device, in the block's cos/sin layout [T, H, 64] f32.
 *  LTXB_ROPE_LTX: the reference's LTX layout (ltx/block_conformance.zig:87-127,
 *    which replaces the host tables the harnesses load): pos = grid [3, T, 2]
 *    f32 (start, end) per axis; frequencies theta^(k/(NF-1)) * pi/2 rounded
 *    to f32, NF = H*128/6 (H <= 32); midpoint positions scaled to [-1, 1]
 *    by max_pos (20, 2048, 2048); slot j = h*64 + f: j < 2 identity (1, 0),
 *    else frequency (j-2)/3 of axis (j-2)%3.
 *  LTXB_ROPE_AXES: the BASELINE configs' split of each head's 128 dims
 *    into (44, 42, 42) per (frame, row, col) axis from integer positions
 *    pos [T, 3] f32, the same table for every head.
 * Angles and trigonometry in f64, rounded to f32 (as the reference's host
 * generator; its gate allows 1-ulp stragglers in 0.01% of the values). */
#define LTXB_ROPE_LTX 0
#define LTXB_ROPE_AXES 1
int ltxb_rope_tables(int kind, const float* pos, int T, int H, double theta, float* cos, float* sin, void* stream);

/* ---- core parts: the steps either side of the blocks (ltx/core_parts.zig) ----
 * f32 arithmetic with bf16 weights, like the reference's traced CoreParts.
 * Weights come from a blob with the checkpoint's names (ltx/core_parts.zig:52-70):
 * adaln_single.emb.timestep_embedder.linear_{1,2}.{weight,bias},
 * adaln_single.linear.{weight,bias}, the same under prompt_adaln_single,
 * patchify_proj.{weight,bias}, proj_out.{weight,bias} (bf16) and
 * scale_shift_table [2, D] (f32). */
typedef struct ltxb_core ltxb_core;
int ltxb_core_upload(int device, const void* blob, uint64_t blob_bytes, const ltxb_entry* entries, int n_entries,
                     int hidden, ltxb_core** out);
void ltxb_core_free(ltxb_core* core);
/* scratch for ltxb_core_adaln (K timesteps), ltxb_core_pts2 and ltxb_core_tail (T tokens) */
uint64_t ltxb_core_workspace_bytes(const ltxb_core* core, int T, int K);
/* out [K, 256] = cos | sin of t*1000*exp(i*(-ln 1e4)/128), f32 (core_parts.zig:42-49) */
int ltxb_core_sinusoid(const float* t, int K, float* out, void* stream);
/* t [K] -> embedded_timestep emb [K, D] (optional) and the block's ts9 table
 * [K, 9, D] (CoreParts.emb / ts9r, core_parts.zig:117-137) */
int ltxb_core_adaln(const ltxb_core* core, const float* t, int K, float* emb, float* ts9, void* workspace,
                    uint64_t workspace_bytes, void* stream);
/* sigma (one device float) -> pts2 [2, D] (CoreParts.pts2r, core_parts.zig:127-142) */
int ltxb_core_pts2(const ltxb_core* core, const float* sigma, float* pts2, void* workspace, uint64_t workspace_bytes,
                   void* stream);
/* latent [T, 128] -> x [T, D] (patchify_proj, core_parts.zig:144-146) */
int ltxb_core_patchify(const ltxb_core* core, const float* latent, int T, float* x, void* stream);
/* velocity [T, 128] = proj_out(LayerNorm(x) * (1 + sst[1] + e) + sst[0] + e), e the RAW
 * embedded_timestep of each token: emb[tidx[t]] (emb [K, D]; a tidx outside [0, K)
 * reads row 0, as the block's table select does), or emb [T, D] per token when tidx
 * is NULL (K ignored) (CoreParts.tailFromEmb, core_parts.zig:148-170) */
int ltxb_core_tail(const ltxb_core* core, const float* x, const float* emb, int K, const int* tidx, int T, float* velocity,
                   void* workspace, uint64_t workspace_bytes, void* stream);

/* ---- scheduler: the distilled LTX-2.5 sampler (ltx/scheduler.zig), bit-exact f32 ----
 * Latents are [T, C] (C = 128 channels) with one mask / timestep value per token. */
/* copies the sigma list of stage 1 (9 values) or 2 (4 values) into out (if not NULL);
 * returns the count, or a negative status */
int ltxb_sched_sigmas(int stage, float* out, int capacity);
/* out = lerp(clean, lerp(clean, noise, noise_scale), mask) with torch.lerp's fused
 * two-branch arithmetic (scheduler.zig:20-46) */
int ltxb_sched_noise_init(const float* clean, const float* noise, const float* mask, int T, int C, float noise_scale,
                          float* out, void* stream);
/* ts = mask * sigma (scheduler.zig:49-51) */
int ltxb_sched_timesteps(const float* mask, int T, float sigma, float* ts, void* stream);
/* out = Euler step of x towards post_process(to_denoised(x, velocity, ts), clean, mask)
 * from sigma to sigma_next (scheduler.zig:54-80, the host march of e2e_denoise.zig:320-325) */
int ltxb_sched_step(const float* x, const float* velocity, const float* ts, const float* clean, const float* mask,
                    int T, int C, float sigma, float sigma_next, float* out, void* stream);

/* ---- the denoising loop (ltx/e2e_denoise.zig:218-336) on the device ----
 * Per step s (sigma = sigmas[s], sigma_next = sigmas[s+1]): ts = mask*sigma;
 * t_k = mask_values[k]*sigma -> embedded_timestep [K, D] and ts9 [K, 9, D];
 * pts2 from sigma; x = patchify(latent); x = block_b(x) for every block;
 * velocity = tail(x, embedded_timestep[tidx]); latent = Euler step of
 * latent towards post_process(to_denoised(latent, velocity, ts)). Latents,
 * tables and activations stay on the device; nothing synchronises the host.
 * cfg.T is this rank's tokens, cfg.K the number of distinct mask values;
 * with cfg.sp_size > 1 each rank passes its token slice (latent, clean, mask,
 * tidx, cos, sin) and the blocks exchange K/V as in ltxb_block_forward. */
typedef struct {
  float* latent;             /* [T, 128] f32: the noised initial latent in, the final latent out */
  const float* clean;        /* [T, 128] clean latent (the post-process blend)                     */
  const float* mask;         /* [T] denoise mask                                                   */
  const float* mask_values;  /* [K] its distinct values                                            */
  const int32_t* tidx;       /* [T] index of each token's mask value in mask_values                */
  const float* ctx;          /* [S, D] text context                                                */
  const float* cos;          /* [T, H, 64] RoPE tables                                             */
  const float* sin;
  void* workspace;           /* ltxb_denoise_workspace_bytes, 256-byte aligned                     */
  uint64_t workspace_bytes;
} ltxb_denoise_io;
uint64_t ltxb_denoise_workspace_bytes(const ltxb_core* core, const ltxb_weights* block, const ltxb_config* cfg);
/* sigmas: host array of n_steps + 1 values (e.g. ltxb_sched_sigmas(1, ...): 8 steps) */
int ltxb_denoise_run(const ltxb_core* core, const ltxb_weights* const* blocks, int n_blocks, const float* sigmas,
                     int n_steps, const ltxb_denoise_io* io, const ltxb_config* cfg, void* stream);

/* ---- structural statistics (statsOf, ltx/core_parts.zig:183-193) ----
 * out (3 device floats) = [NaN count (v != v), sum of v^2, max |v| over the
 * non-NaN values] of the n f32 values at v, so a host checks a full-length
 * output (the production pass's velocity, ltx/e2e_prod.zig:444-468) with a
 * 12-byte readback. Sum of squares in f64, rounded once; a fixed grid and
 * reduction order make the result identical run to run. workspace: at least
 * ltxb_stats_workspace_bytes() bytes of device memory, 16-byte aligned. */
uint64_t ltxb_stats_workspace_bytes(void);
int ltxb_stats(const float* v, uint64_t n, float* out, void* workspace, uint64_t workspace_bytes, void* stream);

/* Size of the scratch ltxb_dq_gemm_noalloc keeps in the library image. */
#define LTXB_NOALLOC_SCRATCH_BYTES (32u << 20)

/* The int8 grouped-128 linear of ltxb_dq_gemm (expand-then-GEMM path) for
 * callers that cannot call cudaMalloc: hosts whose device memory belongs to
 * another allocator (a Zig host with a fixed arena, a serving process with
 * its own caching allocator) or code that must not allocate while it runs.
 * No counterpart in the reference: its ZML runtime always allocates. The
 * bf16 expansion of Wq lives in a fixed LTXB_NOALLOC_SCRATCH_BYTES array
 * inside the library (held on every GPU that loads the library until the
 * process exits), so N * K * 2 must not exceed it (N * K <= 16,777,216, e.g.
 * 4096 x 4096); larger requests return LTXB_EINVAL. The caller passes A, the
 * weights, scales, bias and out as for ltxb_dq_gemm. The first call on a
 * device looks up the scratch address for that device; make that first call
 * before any stream capture. All calls share the one scratch array: calls
 * whose work overlaps on the GPU (different streams) race on it. Nothing in
 * it needs to start at zero -- each call overwrites the part it reads. */
int ltxb_dq_gemm_noalloc(const void* A, const void* Wq, const void* scales, int scale_dtype, const void* bias,
                         void* out, int M, int N, int K, void* stream);

/* out[M, N] (bf16) = A[M, K] (bf16) . W[N, K] (bf16)^T (+ bias): the plain
 * bf16 `lin` on tcgen05. K a multiple of 64, N of 32; pointers 16-byte
 * aligned (LTXB_EINVAL otherwise, before anything is launched). */
int ltxb_gemm_bf16(const void* A, const void* W, const void* bias, void* out, int M, int N, int K, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LTXB_H */
