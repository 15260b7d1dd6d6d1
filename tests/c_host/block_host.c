/* A plain-C host that runs one block end to end through libltxb.so, as a Zig
 * or C caller without Python would: it reads a packed blob, fills the entry
 * table from a text manifest, uploads the weights, allocates its own device
 * buffers with the CUDA driver API (the library allocates nothing for the
 * caller), runs ltxb_block_forward and writes the output.
 *
 *   block_host <dir>
 *
 * <dir>/manifest.txt  one entry per line: name dtype ndim d0 d1 offset nbytes
 * <dir>/dims.txt      T S K D FF mode qset
 * <dir>/blob.bin      the packed blob
 * <dir>/inputs.bin    x [T,D] f32 | tstab [K,9,D] f32 | tidx [T] i32 |
 *                     ctx [S,D] f32 | pts2 [2,D] f32 | cos [T,H,64] f32 | sin
 * <dir>/out.bin       written: the block output [T,D] f32
 *
 * Exit status 0 on success; every failure prints the library's message. */
#include <cuda.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "ltxb.h"

#define MAX_ENTRIES 256

static void* read_file(const char* dir, const char* name, size_t* size) {
  char path[1024];
  snprintf(path, sizeof path, "%s/%s", dir, name);
  FILE* f = fopen(path, "rb");
  if (!f) return NULL;
  fseek(f, 0, SEEK_END);
  long n = ftell(f);
  fseek(f, 0, SEEK_SET);
  void* p = malloc(n > 0 ? (size_t)n : 1);
  if (p && n > 0 && fread(p, 1, (size_t)n, f) != (size_t)n) {
    free(p);
    p = NULL;
  }
  fclose(f);
  if (size) *size = (size_t)n;
  return p;
}

static int cu_ok(CUresult r, const char* what) {
  if (r == CUDA_SUCCESS) return 1;
  const char* msg = NULL;
  cuGetErrorString(r, &msg);
  fprintf(stderr, "%s: %s\n", what, msg ? msg : "?");
  return 0;
}

static int ltxb_ok(int rc, const char* what) {
  if (rc == LTXB_OK) return 1;
  fprintf(stderr, "%s: status %d: %s\n", what, rc, ltxb_last_error());
  return 0;
}

/* a device buffer of `bytes`, filled from `host` unless it is NULL */
static CUdeviceptr upload(const void* host, size_t bytes) {
  CUdeviceptr d = 0;
  if (!cu_ok(cuMemAlloc(&d, bytes ? bytes : 4), "cuMemAlloc")) return 0;
  if (host && bytes && !cu_ok(cuMemcpyHtoD(d, host, bytes), "cuMemcpyHtoD")) return 0;
  return d;
}

int main(int argc, char** argv) {
  if (argc != 2) {
    fprintf(stderr, "usage: block_host <dir>\n");
    return 2;
  }
  const char* dir = argv[1];
  int T, S, K, D, FF, mode, qset;
  {
    char* dims = read_file(dir, "dims.txt", NULL);
    if (!dims || sscanf(dims, "%d %d %d %d %d %d %d", &T, &S, &K, &D, &FF, &mode, &qset) != 7) {
      fprintf(stderr, "bad dims.txt\n");
      return 1;
    }
    free(dims);
  }
  const int H = D / 128;

  /* entries from the manifest */
  static ltxb_entry ent[MAX_ENTRIES];
  static char names[MAX_ENTRIES][256];
  int n = 0;
  {
    char path[1024];
    snprintf(path, sizeof path, "%s/manifest.txt", dir);
    FILE* f = fopen(path, "r");
    if (!f) {
      fprintf(stderr, "no manifest.txt\n");
      return 1;
    }
    long long d0, d1;
    unsigned long long off, nb;
    int dt, nd;
    while (n < MAX_ENTRIES &&
           fscanf(f, "%255s %d %d %lld %lld %llu %llu", names[n], &dt, &nd, &d0, &d1, &off, &nb) == 7) {
      ent[n].name = names[n];
      ent[n].dtype = dt;
      ent[n].ndim = nd;
      ent[n].shape[0] = d0;
      ent[n].shape[1] = d1;
      ent[n].offset = off;
      ent[n].nbytes = nb;
      ++n;
    }
    fclose(f);
  }
  size_t blob_bytes = 0;
  void* blob = read_file(dir, "blob.bin", &blob_bytes);
  if (!blob) {
    fprintf(stderr, "no blob.bin\n");
    return 1;
  }
  if (!ltxb_ok(ltxb_blob_check_layout(ent, n, blob_bytes, 64), "ltxb_blob_check_layout")) return 1;

  /* the caller's CUDA context: the device's primary context, which the
   * library's runtime shares */
  CUdevice dev;
  CUcontext ctx;
  if (!cu_ok(cuInit(0), "cuInit") || !cu_ok(cuDeviceGet(&dev, 0), "cuDeviceGet") ||
      !cu_ok(cuDevicePrimaryCtxRetain(&ctx, dev), "cuDevicePrimaryCtxRetain") ||
      !cu_ok(cuCtxSetCurrent(ctx), "cuCtxSetCurrent"))
    return 1;
  if (!ltxb_ok(ltxb_init(0), "ltxb_init")) return 1;

  ltxb_weights* w = NULL;
  if (!ltxb_ok(ltxb_weights_upload(0, blob, blob_bytes, ent, n, 0, mode, qset, D, FF, &w), "ltxb_weights_upload"))
    return 1;

  size_t in_bytes = 0;
  char* in = read_file(dir, "inputs.bin", &in_bytes);
  const size_t sx = (size_t)T * D * 4, st = (size_t)K * 9 * D * 4, si = (size_t)T * 4, sc = (size_t)S * D * 4,
               sp = (size_t)2 * D * 4, sr = (size_t)T * H * 64 * 4;
  if (!in || in_bytes != sx + st + si + sc + sp + 2 * sr) {
    fprintf(stderr, "inputs.bin has %zu bytes, expected %zu\n", in_bytes, sx + st + si + sc + sp + 2 * sr);
    return 1;
  }
  size_t o = 0;
  CUdeviceptr x = upload(in + o, sx);
  o += sx;
  CUdeviceptr tstab = upload(in + o, st);
  o += st;
  CUdeviceptr tidx = upload(in + o, si);
  o += si;
  CUdeviceptr cctx = upload(in + o, sc);
  o += sc;
  CUdeviceptr pts2 = upload(in + o, sp);
  o += sp;
  CUdeviceptr cosd = upload(in + o, sr);
  o += sr;
  CUdeviceptr sind = upload(in + o, sr);
  CUdeviceptr out = upload(NULL, sx);
  if (!x || !tstab || !tidx || !cctx || !pts2 || !cosd || !sind || !out) return 1;

  ltxb_config cfg;
  memset(&cfg, 0, sizeof cfg);
  cfg.T = T;
  cfg.S = S;
  cfg.K = K;
  cfg.mode = mode;
  cfg.sp_size = 1;
  const uint64_t ws_bytes = ltxb_block_workspace_bytes(w, &cfg);
  CUdeviceptr ws = upload(NULL, ws_bytes + 256);
  if (!ws) return 1;

  ltxb_block_io io;
  memset(&io, 0, sizeof io);
  io.x = (const float*)(uintptr_t)x;
  io.out = (float*)(uintptr_t)out;
  io.tstab = (const float*)(uintptr_t)tstab;
  io.tidx = (const int32_t*)(uintptr_t)tidx;
  io.ctx = (const float*)(uintptr_t)cctx;
  io.pts2 = (const float*)(uintptr_t)pts2;
  io.cos = (const float*)(uintptr_t)cosd;
  io.sin = (const float*)(uintptr_t)sind;
  io.workspace = (void*)(uintptr_t)((ws + 255) & ~(CUdeviceptr)255);
  io.workspace_bytes = ws_bytes;
  if (!ltxb_ok(ltxb_block_forward(w, &io, &cfg, NULL), "ltxb_block_forward")) return 1;
  if (!ltxb_ok(ltxb_device_status(1, NULL), "ltxb_device_status")) return 1;

  float* host_out = malloc(sx);
  if (!host_out || !cu_ok(cuMemcpyDtoH(host_out, out, sx), "cuMemcpyDtoH")) return 1;
  char path[1024];
  snprintf(path, sizeof path, "%s/out.bin", dir);
  FILE* f = fopen(path, "wb");
  if (!f || fwrite(host_out, 1, sx, f) != sx) {
    fprintf(stderr, "cannot write out.bin\n");
    return 1;
  }
  fclose(f);

  ltxb_weights_free(w);
  cuMemFree(x);
  cuMemFree(tstab);
  cuMemFree(tidx);
  cuMemFree(cctx);
  cuMemFree(pts2);
  cuMemFree(cosd);
  cuMemFree(sind);
  cuMemFree(out);
  cuMemFree(ws);
  free(host_out);
  free(in);
  free(blob);
  cuDevicePrimaryCtxRelease(dev);
  printf("block_host: T=%d D=%d mode=%d ok\n", T, D, mode);
  return 0;
}
