// Host-side weight upload from a packed blob (shared by the block and the
// core parts).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include <initializer_list>
#include <string>
#include <vector>

#include "kernels.h"

namespace ltxb {

struct Lin {
  int N = 0, K = 0;
  const void* w = nullptr;     // bf16 [N, K]
  const int8_t* wq = nullptr;  // int8 [N, K]
  const void* sc = nullptr;    // [N, K/128]
  int sc_bf16 = 0;
  const void* b = nullptr;     // bf16 [N] or null
};

// Checkpoint names: '.' and '::' become '_' (the reference's blob keys,
// ltx/loader.zig:138).
inline std::string norm_name(const char* n) {
  std::string s;
  for (const char* p = n; *p; ++p) {
    if (p[0] == ':' && p[1] == ':') {
      s.push_back('_');
      ++p;
    } else if (*p == '.') {
      s.push_back('_');
    } else {
      s.push_back(*p);
    }
  }
  return s;
}

// Every caller-supplied entry must lie inside the blob: offset + nbytes <=
// blob_bytes, checked in a form no 64-bit sum can wrap. Runs on the host
// before any device call, so a bad table is rejected without touching a GPU.
inline int check_entries(const ltxb_entry* e, int n, uint64_t blob_bytes) {
  for (int i = 0; i < n; ++i)
    if (e[i].nbytes > blob_bytes || e[i].offset > blob_bytes - e[i].nbytes)
      return set_error(LTXB_ELAYOUT, "entry %d (%s): %llu bytes at %llu run past the %llu-byte blob", i,
                       e[i].name ? e[i].name : "?", (unsigned long long)e[i].nbytes,
                       (unsigned long long)e[i].offset, (unsigned long long)blob_bytes);
  return LTXB_OK;
}

// Finds, checks and uploads the tensors of one weight set from a host blob:
// entries are named `<prefix><stem>` (prefix "transformer_blocks_<i>_" for a
// block, empty for the core parts); every allocation is recorded in `allocs`
// and counted in `total`.
struct Uploader {
  std::vector<void*>* allocs;
  uint64_t* total;
  const uint8_t* blob;
  uint64_t blob_bytes;
  const ltxb_entry* e;
  int n;
  int block;

  const ltxb_entry* find(const char* stem) {
    char want[512];
    if (block >= 0)
      snprintf(want, sizeof(want), "transformer_blocks_%d_%s", block, stem);
    else
      snprintf(want, sizeof(want), "%s", stem);
    for (int i = 0; i < n; ++i)
      if (norm_name(e[i].name) == want) return &e[i];
    return nullptr;
  }

  int missing(const char* stem) {
    if (block >= 0)
      return set_error(LTXB_EMISSING, "blob %d: no entry named transformer_blocks_%d_%s", block, block, stem);
    return set_error(LTXB_EMISSING, "blob: no entry named %s", stem);
  }

  int require(const char* stem, int dtype, int64_t r, int64_t c, const ltxb_entry** out) {
    const ltxb_entry* x = find(stem);
    if (!x) return missing(stem);
    const int64_t cols = (x->ndim == 2) ? x->shape[1] : 1;
    const int64_t rows = x->shape[0];
    const bool shape_ok = (c == 0) ? (x->ndim == 1 && rows == r) : (x->ndim == 2 && rows == r && cols == c);
    if (x->dtype != dtype || !shape_ok)
      return set_error(LTXB_EDTYPE, "entry %s: dtype %d shape [%lld, %lld], expected dtype %d [%lld, %lld]", x->name,
                       x->dtype, (long long)rows, (long long)cols, dtype, (long long)r, (long long)c);
    const int esz = dtype == LTXB_DT_F32 ? 4 : dtype == LTXB_DT_BF16 ? 2 : 1;
    const uint64_t need = (uint64_t)r * (c ? c : 1) * esz;
    // written so that no sum can wrap: offset + nbytes <= blob_bytes
    if (x->nbytes != need || x->nbytes > blob_bytes || x->offset > blob_bytes - x->nbytes)
      return set_error(LTXB_ELAYOUT, "entry %s: %llu bytes at %llu does not fit (need %llu, blob %llu)", x->name,
                       (unsigned long long)x->nbytes, (unsigned long long)x->offset, (unsigned long long)need,
                       (unsigned long long)blob_bytes);
    *out = x;
    return LTXB_OK;
  }

  int alloc(size_t bytes, void** p) {
    cudaError_t err = cudaMalloc(p, bytes < 256 ? 256 : bytes);
    if (err != cudaSuccess) return set_error(LTXB_ENOMEM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(err));
    allocs->push_back(*p);
    *total += bytes;
    return LTXB_OK;
  }

  // copy `x` to dst + offset
  int put(const ltxb_entry* x, void* dst, size_t off) {
    cudaError_t err = cudaMemcpy(static_cast<uint8_t*>(dst) + off, blob + x->offset, x->nbytes, cudaMemcpyHostToDevice);
    return err == cudaSuccess ? LTXB_OK : set_cuda_error(err, "weights H2D");
  }

  // one tensor, uploaded as is
  int tensor(const char* stem, int dtype, int64_t r, int64_t c, const void** out) {
    const ltxb_entry* x;
    int rc = require(stem, dtype, r, c, &x);
    if (rc) return rc;
    void* p;
    if ((rc = alloc(x->nbytes, &p))) return rc;
    if ((rc = put(x, p, 0))) return rc;
    *out = p;
    return LTXB_OK;
  }

  // A linear made of 1..3 stacked checkpoint matrices [r_i, K] (bf16 or int8)
  int linear(Lin& L, std::initializer_list<const char*> stems, int rows_each, int K, bool has_bias, bool quant,
             int pad_rows = 0) {
    const int parts = (int)stems.size();
    const int N = parts * rows_each + pad_rows;
    L.N = N;
    L.K = K;
    int rc;
    if (quant) {
      void *wq, *sc;
      const ltxb_entry* first_sc = nullptr;
      if ((rc = alloc((size_t)N * K, &wq))) return rc;
      int i = 0;
      for (const char* s : stems) {
        char nm[256];
        snprintf(nm, sizeof(nm), "%s_weight_q8", s);
        const ltxb_entry* x;
        if ((rc = require(nm, LTXB_DT_I8, rows_each, K, &x))) return rc;
        if ((rc = put(x, wq, (size_t)i * rows_each * K))) return rc;
        snprintf(nm, sizeof(nm), "%s_weight_q8scale", s);
        const ltxb_entry* xs = find(nm);
        if (!xs) return missing(nm);
        if (!first_sc) {
          first_sc = xs;
          L.sc_bf16 = xs->dtype == LTXB_DT_BF16;
          if ((rc = alloc((size_t)N * (K / 128) * (L.sc_bf16 ? 2 : 4), &sc))) return rc;
        }
        if ((rc = require(nm, L.sc_bf16 ? LTXB_DT_BF16 : LTXB_DT_F32, rows_each, K / 128, &xs))) return rc;
        if ((rc = put(xs, sc, (size_t)i * rows_each * (K / 128) * (L.sc_bf16 ? 2 : 4)))) return rc;
        ++i;
      }
      L.wq = static_cast<const int8_t*>(wq);
      L.sc = sc;
    } else {
      void* wb;
      if ((rc = alloc((size_t)N * K * 2, &wb))) return rc;
      if (pad_rows && cudaMemset(wb, 0, (size_t)N * K * 2) != cudaSuccess)
        return set_error(LTXB_ECUDA, "memset");
      int i = 0;
      for (const char* s : stems) {
        char nm[256];
        snprintf(nm, sizeof(nm), "%s_weight", s);
        const ltxb_entry* x;
        if ((rc = require(nm, LTXB_DT_BF16, rows_each, K, &x))) return rc;
        if ((rc = put(x, wb, (size_t)i * rows_each * K * 2))) return rc;
        ++i;
      }
      L.w = wb;
    }
    if (has_bias) {
      void* bb;
      if ((rc = alloc((size_t)N * 2, &bb))) return rc;
      if (pad_rows && cudaMemset(bb, 0, (size_t)N * 2) != cudaSuccess) return set_error(LTXB_ECUDA, "memset");
      int i = 0;
      for (const char* s : stems) {
        char nm[256];
        snprintf(nm, sizeof(nm), "%s_bias", s);
        const ltxb_entry* x;
        if ((rc = require(nm, LTXB_DT_BF16, rows_each, 0, &x))) return rc;
        if ((rc = put(x, bb, (size_t)i * rows_each * 2))) return rc;
        ++i;
      }
      L.b = bb;
    }
    return LTXB_OK;
  }
};

}  // namespace ltxb
