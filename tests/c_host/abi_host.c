/* A plain-C host of libltxb.so: what a Zig (or any C-ABI) caller sees. It
 * exercises the host-side entry points that need no GPU -- the blob layout
 * check with the loader's error cases, the native blob reader on a packed
 * blob directory given as the first argument, the ring schedule, the
 * scheduler's sigma lists, error reporting -- and prints one line per check
 * for the pytest driver (tests/test_c_host.py), which compiles it with gcc
 * against include/ltxb.h. Exit status 0 when every check passes. */
#include <stdio.h>
#include <string.h>

#include "ltxb.h"

static int failures = 0;

static void check(int ok, const char* what) {
  printf("%s %s\n", ok ? "ok" : "FAIL", what);
  if (!ok) ++failures;
}

/* Blob.open + checkLayout + findEntry + the digest check (ltx/loader.zig:
 * 50-129, :270-276) through the native reader */
static void blob_checks(const char* dir) {
  ltxb_blob* b = NULL;
  check(ltxb_blob_open(dir, LTXB_VERIFY_BLOB | LTXB_VERIFY_ENTRIES, &b) == LTXB_OK && b != NULL,
        "blob: open with both digest checks");
  if (!b) return;
  const void* data = NULL;
  uint64_t bytes = 0;
  const ltxb_entry* ents = NULL;
  int n = 0;
  uint32_t align = 0;
  int64_t block = -1;
  check(ltxb_blob_view(b, &data, &bytes, &ents, &n, &align, &block) == LTXB_OK && data && bytes > 0 && n > 0 &&
            align == 64 && block == 0,
        "blob: view");
  check(ltxb_blob_check_layout(ents, n, bytes, align) == LTXB_OK, "blob: entries pass the layout check");
  const ltxb_entry* e = NULL;
  check(ltxb_blob_find(b, "transformer_blocks_0_attn1_to_q_weight_q8", &e) == LTXB_OK && e &&
            e->dtype == LTXB_DT_I8 && e->ndim == 2 && e->offset + e->nbytes <= bytes,
        "blob: findEntry");
  check(ltxb_blob_find(b, "transformer_blocks_0_missing", &e) == LTXB_EMISSING &&
            strstr(ltxb_last_error(), "no entry named") != NULL,
        "blob: MissingEntry");
  char hex[65];
  ltxb_sha256_hex("abc", 3, hex);
  check(strlen(hex) == 64, "sha256 hex digest");

  /* the staging ring over the same blob, three times, host-memory slots */
  const ltxb_blob* list[1] = {b};
  const int schedule[3] = {0, 0, 0};
  ltxb_stage* st = NULL;
  check(ltxb_stage_create(list, 1, schedule, 3, bytes, 0, 1, &st) == LTXB_OK && st != NULL, "stage: create");
  int same = st != NULL;
  for (int pos = 0; st && pos < 3; ++pos) {
    const void* slot = NULL;
    uint64_t got = 0;
    if (ltxb_stage_acquire(st, pos, &slot, &got, 10000) != LTXB_OK || got != bytes || memcmp(slot, data, bytes))
      same = 0;
    if (ltxb_stage_release(st, pos) != LTXB_OK) same = 0;
  }
  check(same, "stage: every position holds the blob's bytes");
  ltxb_stage_stats ss;
  check(st && ltxb_stage_get_stats(st, &ss) == LTXB_OK && ss.staged_bytes == 3 * bytes, "stage: stats");
  ltxb_stage_free(st);
  check(ltxb_stage_create(list, 1, schedule, 3, bytes - 1, 0, 0, &st) == LTXB_EINVAL &&
            strstr(ltxb_last_error(), "SlotTooSmall") != NULL,
        "stage: SlotTooSmall");
  ltxb_blob_close(b);
  check(ltxb_blob_open("/nonexistent-blob-dir", 0, &b) == LTXB_EMISSING && b == NULL, "blob: missing directory");
}

int main(int argc, char** argv) {
  check(ltxb_version() != NULL && strlen(ltxb_version()) > 0, "version string");
  if (argc > 1) blob_checks(argv[1]);

  /* blob layout (ltx/loader.zig:73-82): 64-byte aligned, no gap, no tail */
  ltxb_entry e[2];
  memset(e, 0, sizeof e);
  e[0].name = "a";
  e[0].dtype = LTXB_DT_BF16;
  e[0].ndim = 1;
  e[0].shape[0] = 16;
  e[0].offset = 0;
  e[0].nbytes = 32;
  e[1].name = "b";
  e[1].dtype = LTXB_DT_F32;
  e[1].ndim = 2;
  e[1].shape[0] = 2;
  e[1].shape[1] = 4;
  e[1].offset = 64;
  e[1].nbytes = 32;
  check(ltxb_blob_check_layout(e, 2, 96, 64) == LTXB_OK, "layout: valid");
  e[1].offset = 40;
  check(ltxb_blob_check_layout(e, 2, 72, 64) == LTXB_ELAYOUT && strstr(ltxb_last_error(), "Misaligned") != NULL,
        "layout: Misaligned");
  e[1].offset = 128;
  check(ltxb_blob_check_layout(e, 2, 160, 64) == LTXB_ELAYOUT && strstr(ltxb_last_error(), "LayoutGap") != NULL,
        "layout: LayoutGap");
  e[1].offset = 64;
  check(ltxb_blob_check_layout(e, 2, 160, 64) == LTXB_ELAYOUT && strstr(ltxb_last_error(), "TrailingBytes") != NULL,
        "layout: TrailingBytes");

  /* ring schedule: every rank computes every shard exactly once */
  int ok = 1;
  for (int n = 1; n <= 8; n *= 2)
    for (int r = 0; r < n; ++r) {
      int seen[8] = {0};
      for (int s = 0; s < n; ++s) {
        int cur, rcv, nxt, prv;
        if (ltxb_ring_step(r, n, s, &cur, &rcv, &nxt, &prv) != LTXB_OK || cur < 0 || cur >= n) ok = 0;
        else ++seen[cur];
        if (s == n - 1 && rcv != -1) ok = 0;
      }
      for (int i = 0; i < n; ++i)
        if (seen[i] != 1) ok = 0;
    }
  check(ok, "ring schedule covers every shard once");
  int cur, rcv, nxt, prv;
  check(ltxb_ring_step(2, 2, 0, &cur, &rcv, &nxt, &prv) == LTXB_EINVAL, "ring schedule rejects a bad rank");

  /* the distilled sigma lists (ltx/scheduler.zig:11-18) */
  float sg[9];
  check(ltxb_sched_sigmas(1, sg, 9) == 9 && sg[0] == 1.0f && sg[5] == (float)0.909375 && sg[8] == 0.0f,
        "stage-1 sigmas");
  check(ltxb_sched_sigmas(2, sg, 4) == 4 && sg[0] == (float)0.909375, "stage-2 sigmas");
  check(ltxb_sched_sigmas(3, sg, 9) == LTXB_EINVAL && ltxb_last_error()[0] != '\0', "unknown stage is an error");
  check(ltxb_sched_sigmas(1, sg, 4) == LTXB_EINVAL, "short output buffer is an error");

  printf("%d failure(s)\n", failures);
  return failures ? 1 : 0;
}
