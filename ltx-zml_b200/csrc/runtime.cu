// Library runtime: error reporting, device init, the TMA descriptor encoder
// (resolved from the driver at init, so the library links no libcuda), and
// the device status word that bounded waits write on expiry.
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "kernels.h"

namespace ltxb {

__device__ uint32_t g_status = 0;

static thread_local char t_err[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
  return code;
}

int set_cuda_error(cudaError_t e, const char* what) {
  return set_error(LTXB_ECUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

static std::atomic<int> g_sms[kMaxDevices];

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  const bool cached = dev >= 0 && dev < kMaxDevices;
  int n = cached ? g_sms[dev].load(std::memory_order_relaxed) : 0;
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    if (cached) g_sms[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// ---- launch accounting / profiling ----
static std::atomic<uint64_t> g_launches{0};
void launched() { g_launches.fetch_add(1, std::memory_order_relaxed); }

namespace {
struct ProfRec {
  std::string name;
  cudaEvent_t a, b;
  uint64_t launches;
};
struct ProfState {
  std::mutex mu;
  bool on = false;
  std::vector<cudaEvent_t> pool;
  std::vector<ProfRec> pending;
  std::vector<std::string> names;
  std::vector<double> ms;
  std::vector<uint64_t> launches;
  std::vector<int> count;
};
ProfState g_prof;

cudaEvent_t prof_event() {
  if (!g_prof.pool.empty()) {
    cudaEvent_t e = g_prof.pool.back();
    g_prof.pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}
}  // namespace

Phase::Phase(const char* n, cudaStream_t s) : name(n), st(s), slot(-1) {
  std::lock_guard<std::mutex> lk(g_prof.mu);
  if (!g_prof.on) return;
  ProfRec r{n, prof_event(), prof_event(), g_launches.load()};
  cudaEventRecord(r.a, st);
  g_prof.pending.push_back(r);
  slot = (int)g_prof.pending.size() - 1;
}

Phase::~Phase() {
  std::lock_guard<std::mutex> lk(g_prof.mu);
  if (slot < 0 || slot >= (int)g_prof.pending.size()) return;
  ProfRec& r = g_prof.pending[slot];
  cudaEventRecord(r.b, st);
  r.launches = g_launches.load() - r.launches;
}

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

static int resolve_encoder() {
  std::call_once(g_encode_once, [] {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) return set_error(LTXB_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  return LTXB_OK;
}

int make_tmap_2d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, int cols, int rows,
                 int ld, int box_cols, int box_rows, CUtensorMapSwizzle swz) {
  int rc = resolve_encoder();
  if (rc) return rc;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((size_t)ld * elem_bytes) % 16)
    return set_error(LTXB_EINVAL, "TMA: base must be 16-byte aligned and the row stride a multiple of 16 bytes");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * elem_bytes};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(LTXB_ECUDA, "cuTensorMapEncodeTiled failed (%d): %d x %d, ld %d, box %d x %d", (int)r, rows,
                     cols, ld, box_rows, box_cols);
  return LTXB_OK;
}

int check_device(int device, const char* what) {
  int cur = -1;
  cudaError_t e = cudaGetDevice(&cur);
  if (e != cudaSuccess) return set_cuda_error(e, what);
  if (cur != device)
    return set_error(LTXB_EINVAL, "%s: the weights live on device %d but device %d is current", what, device, cur);
  return LTXB_OK;
}

}  // namespace ltxb

using namespace ltxb;

extern "C" {

const char* ltxb_last_error(void) { return t_err; }

const char* ltxb_version(void) { return "ltxb 0.1 (sm_100a)"; }

int ltxb_init(int device) {
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaSetDevice");
  e = cudaFree(nullptr);  // create / bind the primary context
  if (e != cudaSuccess) return set_cuda_error(e, "context init");
  cudaDeviceProp p;
  e = cudaGetDeviceProperties(&p, device);
  if (e != cudaSuccess) return set_cuda_error(e, "cudaGetDeviceProperties");
  if (p.major != 10 || p.minor != 0)
    return set_error(LTXB_EUNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a (B200)", device, p.major,
                     p.minor);
  sm_count();
  return resolve_encoder();
}

uint64_t ltxb_launch_count(void) { return g_launches.load(); }

int ltxb_profile_enable(int on) {
  std::lock_guard<std::mutex> lk(g_prof.mu);
  g_prof.on = on != 0;
  return LTXB_OK;
}

int ltxb_profile_collect(int max_phases, char* names, int name_stride, double* total_ms, uint64_t* launches,
                         int* calls, int reset) {
  std::lock_guard<std::mutex> lk(g_prof.mu);
  for (ProfRec& r : g_prof.pending) {
    float ms = 0.f;
    cudaError_t e = cudaEventSynchronize(r.b);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, r.a, r.b);
    if (e != cudaSuccess) return set_cuda_error(e, "profile events");
    size_t i = 0;
    while (i < g_prof.names.size() && g_prof.names[i] != r.name) ++i;
    if (i == g_prof.names.size()) {
      g_prof.names.push_back(r.name);
      g_prof.ms.push_back(0.0);
      g_prof.launches.push_back(0);
      g_prof.count.push_back(0);
    }
    g_prof.ms[i] += ms;
    g_prof.launches[i] += r.launches;
    g_prof.count[i] += 1;
    g_prof.pool.push_back(r.a);
    g_prof.pool.push_back(r.b);
  }
  g_prof.pending.clear();
  const int n = (int)g_prof.names.size();
  for (int i = 0; i < n && i < max_phases; ++i) {
    if (names && name_stride > 0) snprintf(names + (size_t)i * name_stride, name_stride, "%s", g_prof.names[i].c_str());
    if (total_ms) total_ms[i] = g_prof.ms[i];
    if (launches) launches[i] = g_prof.launches[i];
    if (calls) calls[i] = g_prof.count[i];
  }
  if (reset) {
    g_prof.names.clear();
    g_prof.ms.clear();
    g_prof.launches.clear();
    g_prof.count.clear();
  }
  return n;
}

// One warp waits (bounded, limit_us) on an mbarrier that nothing arrives on:
// the expiry path every kernel wait takes, exercised without a fault or a
// hang. Lane 0 of the other warp of the block only initialises the barrier.
__global__ void selftest_wait_kernel(uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x < 32) warp_wait_limit(&bar, 0, LTXB_SELFTEST_SITE, limit_ns);
}

int ltxb_selftest_wait(uint32_t limit_us, void* stream) {
  if (limit_us == 0 || limit_us > 2000000) return set_error(LTXB_EINVAL, "self-test wait: limit must be 1 us .. 2 s");
  selftest_wait_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>((uint64_t)limit_us * 1000);
  launched();
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? LTXB_OK : set_cuda_error(e, "self-test wait");
}

int ltxb_device_status(int clear, uint32_t* site) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return set_cuda_error(e, "cudaDeviceSynchronize");
  uint32_t v = 0;
  e = cudaMemcpyFromSymbol(&v, g_status, sizeof(v));
  if (e != cudaSuccess) return set_cuda_error(e, "read status");
  if (clear && v) {
    uint32_t z = 0;
    e = cudaMemcpyToSymbol(g_status, &z, sizeof(z));
    if (e != cudaSuccess) return set_cuda_error(e, "clear status");
  }
  uint32_t va = 0;
  e = ltxb::attn_status(&va, clear != 0);
  if (e != cudaSuccess) return set_cuda_error(e, "read attention status");
  if (!v) v = va;
  if (site) *site = v >> 8;
  if ((v & 0xFF) == STATUS_TIMEOUT) return set_error(LTXB_ETIMEOUT, "device wait expired at site 0x%x", v >> 8);
  return LTXB_OK;
}

}  // extern "C"
