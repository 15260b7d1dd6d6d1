// Library runtime: error reporting, device init, the TMA descriptor encoder
// (resolved from the driver at init, so the library links no libcuda), and
// the device status word that bounded waits write on expiry.
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>

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

static int g_sms[64];

int sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 63;
  if (g_sms[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sms[dev] = n;
  }
  return g_sms[dev];
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
  if (site) *site = v >> 8;
  if ((v & 0xFF) == STATUS_TIMEOUT) return set_error(LTXB_ETIMEOUT, "device wait expired at site 0x%x", v >> 8);
  return LTXB_OK;
}

}  // extern "C"
