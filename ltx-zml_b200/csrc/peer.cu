// Head-parallel sequence parallelism over peer memory: the exchange around
// self-attention written as stores into the other GPUs' memory instead of
// collective calls.
//
// Every rank owns a window of device memory that the other ranks of the
// communicator have mapped (CUDA IPC over NVLink / NVSwitch). Rank r owns
// heads [r H/N, (r+1) H/N) (Dn = D/N columns) for all N T tokens:
//
//   peer_scatter   reads this rank's q, k (normalised, rotated), v and gate
//                  logits and stores every (tensor, owner) slice straight
//                  into the owner's receive buffer: rx[x][r][t][0:Dn] of
//                  rank p gets columns [p Dn, (p+1) Dn) of token t of tensor
//                  x; the gate rows go to every rank. The last CTA to finish
//                  raises this rank's arrival flag in every window.
//   peer_wait      one warp spins (bounded) on the flags the other ranks
//                  raise in this rank's window.
//   attention      (attn_tc.cu) over all N T queries and keys of the owned
//                  heads; its epilogue stores output row i into the window of
//                  rank i / T, and its last CTA raises the output flags.
//
// Flags carry a call counter (epoch) instead of a boolean, so they are never
// reset; the receive buffers alternate by the epoch's parity, which makes
// reuse safe without a second handshake. Rank q writes rank p's buffer e % 2
// in call e; p last read it in call e-2. q's call-e scatter comes after q
// saw p's call-(e-1) arrival flag, which p raised after its call e-2 had
// finished (stream order); q's call-e attention output comes after q saw
// p's call-e arrival, raised after p's call e-1 had finished.
//
// Memory ordering: each CTA's stores are followed by a system-scope fence
// before it counts itself done (atomic on a per-kernel counter); the last CTA
// fences again and publishes the epoch with st.release.sys; the waiter reads
// it with ld.acquire.sys. Kernels that read the data run after the waiter on
// the same stream.
#include "common.cuh"
#include "kernels.h"

namespace ltxb {

__global__ void __launch_bounds__(256) peer_scatter_kernel(const PeerScatterArgs a) {
  const int Dn = a.D / a.N, c16 = Dn / 8;  // 16-byte units per row slice
  const int tid = blockIdx.x * blockDim.x + threadIdx.x, nthr = gridDim.x * blockDim.x;
  // q / k / v: 16-byte units of the (tensor, owner, token) row slices of Dn
  // columns, consecutive threads on consecutive units of a slice; four units
  // per thread are loaded before any is stored
  const int units = 3 * a.N * a.T * c16;
  for (int u0 = tid; u0 < units; u0 += 4 * nthr) {
    uint4 v[4];
    uint4* d[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int u = u0 + j * nthr;
      d[j] = nullptr;
      v[j] = make_uint4(0, 0, 0, 0);
      if (u < units) {
        const int c = u % c16, row = u / c16;
        const int t = row % a.T, xp = row / a.T, p = xp % a.N, x = xp / a.N;
        v[j] = reinterpret_cast<const uint4*>(a.src[x] + (size_t)t * a.ld[x] + (size_t)p * Dn)[c];
        d[j] = reinterpret_cast<uint4*>(a.rx[p] + (((size_t)x * a.N + a.r) * a.T + t) * Dn) + c;
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (d[j]) *d[j] = v[j];
  }
  // gate logits [T, G] f32 to every rank's [N T, G] at rows [r T, (r+1) T)
  if (a.gate) {
    const int g4 = a.G / 4, gunits = a.N * a.T * g4;
    for (int i = tid; i < gunits; i += nthr) {
      const int c = i % g4, pt = i / g4, t = pt % a.T, p = pt / a.T;
      reinterpret_cast<float4*>(a.gall[p] + ((size_t)a.r * a.T + t) * a.G)[c] =
          reinterpret_cast<const float4*>(a.gate + (size_t)t * a.G)[c];
    }
  }
  last_cta_signal(a.counter, a.flag, a.N, a.epoch);
}

// Wait until every other rank has published `epoch` in flags[p] (this
// rank's window). Bounded: after kWaitLimitNs the site is recorded in the
// device status word and the kernel returns.
__global__ void peer_wait_kernel(const uint32_t* flags, int N, int r, uint32_t epoch, uint32_t site) {
  const int p = threadIdx.x;
  if (p < N && p != r) {
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while ((int)(ld_acquire_sys(flags + p) - epoch) < 0) {
      if ((++spins & 63u) == 0) {
        if (*(volatile uint32_t*)&g_status != 0u) break;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          report_timeout(site);
          break;
        }
      }
      __nanosleep(128);
    }
  }
  __threadfence_system();
}

int peer_scatter(const PeerScatterArgs& a, cudaStream_t st) {
  if (a.N < 2 || a.N > kMaxPeers || a.r < 0 || a.r >= a.N || a.T < 1 || a.D % a.N || (a.D / a.N) % 8 || a.G % 4)
    return set_error(LTXB_EINVAL, "peer scatter: %d ranks, T %d, D %d, G %d", a.N, a.T, a.D, a.G);
  if ((size_t)3 * a.N * a.T * (a.D / a.N / 8) + (size_t)4 * sm_count() * 256 >= (1u << 31) ||
      (size_t)a.N * a.T * (a.G / 4) + (size_t)sm_count() * 256 >= (1u << 31))
    return set_error(LTXB_EINVAL, "peer scatter: too many rows");
  // a third of the SMs: enough stores in flight for the links, the rest stay
  // free for the work that overlaps the exchange
  int grid = sm_count() / 3;
  if (grid < 8) grid = 8;
  peer_scatter_kernel<<<grid, 256, 0, st>>>(a);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "peer scatter");
}

int peer_wait(const uint32_t* flags, int N, int r, uint32_t epoch, uint32_t site, cudaStream_t st) {
  if (N < 2 || N > kMaxPeers) return set_error(LTXB_EINVAL, "peer wait: %d ranks", N);
  peer_wait_kernel<<<1, 32, 0, st>>>(flags, N, r, epoch, site);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "peer wait");
}

}  // namespace ltxb
