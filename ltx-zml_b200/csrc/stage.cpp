// Streaming weight staging: the host side of uploading a schedule of packed
// blobs (the reference's Ring, ltx/loader.zig:176-321, rebuilt for B200).
//
// Two host slots (page-locked when asked, so device copies from them run at
// the link's full rate). A reader thread walks the schedule in order; for
// each position it waits for a free slot, verifies the blob's digest on its
// first touch (optional), and copies the mapped blob into the slot. The
// consumer takes positions in order (acquire), uploads from the slot and
// gives it back (release), so reading blob k+1 from the page cache overlaps
// the device copies of blob k. Slot states move free -> filling -> ready ->
// in_use -> free and every transition is checked. Waits are bounded: acquire
// gives up after its timeout (LTXB_ETIMEOUT); abort() retires the reader at
// its next wait. The schedule is checked before any I/O: every index names a
// blob (ScheduleOutOfRange) and every blob fits a slot (SlotTooSmall).
#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "kernels.h"

using ltxb::set_error;

namespace {

enum SlotState { kFree, kFilling, kReady, kInUse };

bool legal(SlotState from, SlotState to) {
  switch (from) {
    case kFree: return to == kFilling;
    case kFilling: return to == kReady;
    case kReady: return to == kInUse;
    case kInUse: return to == kFree;
  }
  return false;
}

struct Slot {
  uint8_t* mem = nullptr;
  SlotState state = kFree;
  int pos = -1;          // schedule position held (state != kFree)
  uint64_t bytes = 0;    // bytes staged
};

uint64_t now_ns() {
  return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

}  // namespace

struct ltxb_stage {
  std::vector<const ltxb_blob*> blobs;
  std::vector<int> schedule;
  uint64_t slot_bytes = 0;
  bool pinned = false;
  bool verify = false;
  Slot slots[2];
  std::vector<char> verified;  // per blob: digest checked

  std::mutex mu;
  std::condition_variable cv;
  bool shutdown = false;
  int reader_code = LTXB_OK;   // the reader's failure, reported to the consumer
  std::string reader_msg;
  ltxb_stage_stats stats{};
  std::thread reader;

  // under mu
  int move(Slot& s, SlotState to) {
    if (!legal(s.state, to)) {
      return set_error(LTXB_EINVAL, "stage: illegal slot transition %d -> %d", (int)s.state, (int)to);
    }
    s.state = to;
    return LTXB_OK;
  }

  void fail_reader(int code, const std::string& msg) {
    std::lock_guard<std::mutex> lk(mu);
    if (reader_code == LTXB_OK) {
      reader_code = code;
      reader_msg = msg;
    }
    cv.notify_all();
  }

  void reader_main() {
    for (size_t pos = 0; pos < schedule.size(); ++pos) {
      const int bi = schedule[pos];
      Slot* slot = nullptr;
      {
        std::unique_lock<std::mutex> lk(mu);
        for (;;) {
          if (shutdown) return;
          for (Slot& s : slots)
            if (s.state == kFree) {
              slot = &s;
              break;
            }
          if (slot) break;
          ++stats.reader_parks;
          cv.wait(lk);
        }
        if (move(*slot, kFilling)) {
          reader_code = LTXB_EINVAL;
          reader_msg = "stage: illegal slot transition in the reader";
          cv.notify_all();
          return;
        }
        slot->pos = (int)pos;
      }
      const void* data = nullptr;
      uint64_t bytes = 0;
      ltxb_blob_view(blobs[bi], &data, &bytes, nullptr, nullptr, nullptr, nullptr);
      if (verify && !verified[bi]) {
        const uint64_t t0 = now_ns();
        if (ltxb_blob_verify(blobs[bi], LTXB_VERIFY_BLOB) != LTXB_OK) {
          fail_reader(LTXB_ELAYOUT, std::string("stage: blob ") + std::to_string(bi) + ": " + ltxb_last_error());
          return;
        }
        verified[bi] = 1;
        std::lock_guard<std::mutex> lk(mu);
        stats.verify_ns += now_ns() - t0;
      }
      const uint64_t t0 = now_ns();
      if (bytes) memcpy(slot->mem, data, (size_t)bytes);
      const uint64_t dt = now_ns() - t0;
      {
        std::lock_guard<std::mutex> lk(mu);
        slot->bytes = bytes;
        stats.copy_ns += dt;
        stats.staged_bytes += bytes;
        if (move(*slot, kReady)) {
          reader_code = LTXB_EINVAL;
          reader_msg = "stage: illegal slot transition in the reader";
          cv.notify_all();
          return;
        }
      }
      cv.notify_all();
    }
  }

  void stop() {
    {
      std::lock_guard<std::mutex> lk(mu);
      shutdown = true;
    }
    cv.notify_all();
    if (reader.joinable()) reader.join();
  }

  ~ltxb_stage() {
    stop();
    for (Slot& s : slots) {
      if (!s.mem) continue;
      if (pinned) cudaFreeHost(s.mem);
      else free(s.mem);
    }
  }
};

extern "C" {

int ltxb_stage_create(const ltxb_blob* const* blobs, int n_blobs, const int* schedule, int n_schedule,
                      uint64_t slot_bytes, int pinned, int verify, ltxb_stage** out) {
  if (!out) return set_error(LTXB_EINVAL, "stage: out is null");
  *out = nullptr;
  if (n_blobs <= 0 || !blobs || n_schedule < 0 || (n_schedule > 0 && !schedule))
    return set_error(LTXB_EINVAL, "stage: no blobs or no schedule");
  std::vector<uint64_t> sizes(n_blobs);
  for (int i = 0; i < n_blobs; ++i) {
    if (!blobs[i]) return set_error(LTXB_EINVAL, "stage: blob %d is null", i);
    ltxb_blob_view(blobs[i], nullptr, &sizes[i], nullptr, nullptr, nullptr, nullptr);
  }
  // the static check before any I/O (ltx/loader.zig:225-235)
  for (int p = 0; p < n_schedule; ++p) {
    if (schedule[p] < 0 || schedule[p] >= n_blobs)
      return set_error(LTXB_EINVAL, "ScheduleOutOfRange: position %d names blob %d of %d", p, schedule[p], n_blobs);
    if (sizes[schedule[p]] > slot_bytes)
      return set_error(LTXB_EINVAL, "SlotTooSmall: blob %d has %llu bytes, a slot %llu", schedule[p],
                       (unsigned long long)sizes[schedule[p]], (unsigned long long)slot_bytes);
  }
  auto* s = new ltxb_stage();
  s->blobs.assign(blobs, blobs + n_blobs);
  s->schedule.assign(schedule, schedule + n_schedule);
  s->slot_bytes = slot_bytes;
  s->pinned = pinned != 0;
  s->verify = verify != 0;
  s->verified.assign(n_blobs, 0);
  const size_t cap = (size_t)(slot_bytes ? slot_bytes : 1);
  for (Slot& sl : s->slots) {
    if (s->pinned) {
      void* p = nullptr;
      cudaError_t e = cudaHostAlloc(&p, cap, cudaHostAllocPortable);
      if (e != cudaSuccess) {
        delete s;
        return set_error(LTXB_ENOMEM, "stage: cudaHostAlloc(%zu): %s", cap, cudaGetErrorString(e));
      }
      sl.mem = static_cast<uint8_t*>(p);
    } else {
      sl.mem = static_cast<uint8_t*>(aligned_alloc(4096, (cap + 4095) / 4096 * 4096));
      if (!sl.mem) {
        delete s;
        return set_error(LTXB_ENOMEM, "stage: host allocation of %zu bytes", cap);
      }
    }
  }
  s->reader = std::thread([s] { s->reader_main(); });
  *out = s;
  return LTXB_OK;
}

int ltxb_stage_acquire(ltxb_stage* s, int pos, const void** data, uint64_t* bytes, uint32_t timeout_ms) {
  if (!s) return set_error(LTXB_EINVAL, "stage: null");
  if (pos < 0 || pos >= (int)s->schedule.size())
    return set_error(LTXB_EINVAL, "stage: position %d outside the %zu-entry schedule", pos, s->schedule.size());
  std::unique_lock<std::mutex> lk(s->mu);
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
  for (;;) {
    if (s->shutdown) return set_error(LTXB_EINVAL, "RingShutdown: the stage was aborted");
    // positions staged before a reader failure stay available
    for (Slot& sl : s->slots)
      if (sl.state == kReady && sl.pos == pos) {
        int rc = s->move(sl, kInUse);
        if (rc) return rc;
        if (data) *data = sl.mem;
        if (bytes) *bytes = sl.bytes;
        return LTXB_OK;
      }
    if (s->reader_code != LTXB_OK) return set_error(s->reader_code, "%s", s->reader_msg.c_str());
    ++s->stats.consumer_parks;
    if (s->cv.wait_until(lk, deadline) == std::cv_status::timeout) {
      // one last look: the slot may have become ready as the wait ended
      for (Slot& sl : s->slots)
        if (sl.state == kReady && sl.pos == pos) {
          int rc = s->move(sl, kInUse);
          if (rc) return rc;
          if (data) *data = sl.mem;
          if (bytes) *bytes = sl.bytes;
          return LTXB_OK;
        }
      return set_error(LTXB_ETIMEOUT, "stage: position %d not staged within %u ms", pos, timeout_ms);
    }
  }
}

int ltxb_stage_release(ltxb_stage* s, int pos) {
  if (!s) return set_error(LTXB_EINVAL, "stage: null");
  {
    std::lock_guard<std::mutex> lk(s->mu);
    Slot* held = nullptr;
    for (Slot& sl : s->slots)
      if (sl.state == kInUse && sl.pos == pos) held = &sl;
    if (!held) return set_error(LTXB_EINVAL, "stage: position %d is not held", pos);
    int rc = s->move(*held, kFree);
    if (rc) return rc;
    held->pos = -1;
    held->bytes = 0;
  }
  s->cv.notify_all();
  return LTXB_OK;
}

int ltxb_stage_upload(ltxb_stage* s, int pos, int device, int block_idx, int mode, int qset, int hidden, int ff,
                      uint32_t timeout_ms, ltxb_weights** out) {
  if (!s || !out) return set_error(LTXB_EINVAL, "stage upload: null argument");
  *out = nullptr;
  if (pos < 0 || pos >= (int)s->schedule.size())
    return set_error(LTXB_EINVAL, "stage: position %d outside the %zu-entry schedule", pos, s->schedule.size());
  const ltxb_entry* entries = nullptr;
  int n = 0;
  ltxb_blob_view(s->blobs[s->schedule[pos]], nullptr, nullptr, &entries, &n, nullptr, nullptr);
  const void* data = nullptr;
  uint64_t bytes = 0;
  int rc = ltxb_stage_acquire(s, pos, &data, &bytes, timeout_ms);
  if (rc) return rc;
  rc = ltxb_weights_upload(device, data, bytes, entries, n, block_idx, mode, qset, hidden, ff, out);
  // the upload's copies have completed when it returns: the slot is free again
  const int rc2 = ltxb_stage_release(s, pos);
  return rc ? rc : rc2;
}

int ltxb_stage_get_stats(ltxb_stage* s, ltxb_stage_stats* out) {
  if (!s || !out) return set_error(LTXB_EINVAL, "stage stats: null argument");
  std::lock_guard<std::mutex> lk(s->mu);
  *out = s->stats;
  return LTXB_OK;
}

void ltxb_stage_abort(ltxb_stage* s) {
  if (!s) return;
  {
    std::lock_guard<std::mutex> lk(s->mu);
    s->shutdown = true;
  }
  s->cv.notify_all();
}

void ltxb_stage_free(ltxb_stage* s) { delete s; }

}  // extern "C"
