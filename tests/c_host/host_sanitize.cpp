// Sanitizer driver for the library's host-only C++ (csrc/blob.cpp,
// csrc/stage.cpp), compiled together with those two files by
// tests/test_c_host.py under AddressSanitizer + UBSan and under
// ThreadSanitizer. No GPU code is involved: the error-string functions the
// two files call come from this driver instead of the CUDA runtime part of
// the library.
//
//   host_sanitize fuzz  <blob dir> <work dir> <iterations>
//       mutated copies of the directory's manifest (byte edits, deletions,
//       insertions, truncations) through ltxb_blob_open, half of them with
//       both digest checks
//   host_sanitize stage <blob dir>...
//       the staging ring over the given blobs: 20 rounds of a 200-entry
//       schedule, some ended early, some aborted, all freed with the reader
//       in any state
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <random>
#include <sstream>
#include <string>
#include <vector>

#include "ltxb.h"

namespace ltxb {
static thread_local char g_msg[512];
int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof g_msg, fmt, ap);
  va_end(ap);
  return code;
}
}  // namespace ltxb
extern "C" const char* ltxb_last_error(void) { return ltxb::g_msg; }
// the staging ring's device upload is not exercised here
extern "C" int ltxb_weights_upload(int, const void*, uint64_t, const ltxb_entry*, int, int, int, int, int, int,
                                   ltxb_weights**) {
  return LTXB_EUNSUPPORTED;
}

static std::string slurp(const std::string& path) {
  std::ifstream f(path, std::ios::binary);
  std::stringstream ss;
  ss << f.rdbuf();
  return ss.str();
}

static int fuzz(const char* dir, const char* work, int iterations) {
  const std::string manifest = slurp(std::string(dir) + "/blob_manifest.json");
  const std::string blob = slurp(std::string(dir) + "/blob.bin");
  if (manifest.empty()) return fprintf(stderr, "no manifest\n"), 1;
  { std::ofstream(std::string(work) + "/blob.bin", std::ios::binary) << blob; }
  std::mt19937 rng(1);
  const char alpha[] = "{}[]\":,\\u0123456789eE+-.tfnrl \n";
  int opened = 0, rejected = 0;
  for (int it = 0; it < iterations; ++it) {
    std::string m = manifest;
    for (int k = 1 + (int)(rng() % 4); k > 0; --k) {
      const size_t p = rng() % m.size();
      switch (rng() % 4) {
        case 0: m[p] = alpha[rng() % (sizeof alpha - 1)]; break;
        case 1: m.erase(p, 1 + rng() % 8); break;
        case 2: m.insert(p, 1, alpha[rng() % (sizeof alpha - 1)]); break;
        default: m.resize(p); break;
      }
      if (m.empty()) m = "{";
    }
    { std::ofstream(std::string(work) + "/blob_manifest.json", std::ios::binary) << m; }
    ltxb_blob* b = nullptr;
    if (ltxb_blob_open(work, (it & 1) ? LTXB_VERIFY_BLOB | LTXB_VERIFY_ENTRIES : 0, &b) == LTXB_OK) {
      const ltxb_entry* e = nullptr;
      ltxb_blob_find(b, "transformer_blocks_0_attn1_to_q_weight", &e);
      ltxb_blob_close(b);
      ++opened;
    } else {
      ++rejected;
    }
  }
  printf("fuzz: %d opened, %d rejected\n", opened, rejected);
  return 0;
}

static int stage(int n, char** dirs) {
  std::vector<ltxb_blob*> blobs;
  uint64_t largest = 0;
  for (int i = 0; i < n; ++i) {
    ltxb_blob* b = nullptr;
    if (ltxb_blob_open(dirs[i], LTXB_VERIFY_BLOB, &b) != LTXB_OK) return fprintf(stderr, "%s\n", ltxb_last_error()), 1;
    uint64_t bytes = 0;
    ltxb_blob_view(b, nullptr, &bytes, nullptr, nullptr, nullptr, nullptr);
    if (bytes > largest) largest = bytes;
    blobs.push_back(b);
  }
  std::vector<int> schedule;
  for (int p = 0; p < 200; ++p) schedule.push_back(p % n);
  for (int round = 0; round < 20; ++round) {
    ltxb_stage* st = nullptr;
    if (ltxb_stage_create(blobs.data(), n, schedule.data(), (int)schedule.size(), largest, 0, 1, &st) != LTXB_OK)
      return fprintf(stderr, "%s\n", ltxb_last_error()), 1;
    const int last = round % 3 == 0 ? 50 : (int)schedule.size();
    for (int p = 0; p < last; ++p) {
      const void* d = nullptr;
      uint64_t bytes = 0;
      if (ltxb_stage_acquire(st, p, &d, &bytes, 10000) != LTXB_OK) return fprintf(stderr, "%s\n", ltxb_last_error()), 1;
      volatile uint8_t touch = static_cast<const uint8_t*>(d)[bytes / 2];
      (void)touch;
      ltxb_stage_release(st, p);
    }
    if (round % 3 == 1) ltxb_stage_abort(st);
    ltxb_stage_free(st);
  }
  for (ltxb_blob* b : blobs) ltxb_blob_close(b);
  printf("stage: ok\n");
  return 0;
}

int main(int argc, char** argv) {
  if (argc >= 5 && !strcmp(argv[1], "fuzz")) return fuzz(argv[2], argv[3], atoi(argv[4]));
  if (argc >= 3 && !strcmp(argv[1], "stage")) return stage(argc - 2, argv + 2);
  fprintf(stderr, "usage: host_sanitize fuzz <dir> <work> <n> | stage <dir>...\n");
  return 2;
}
