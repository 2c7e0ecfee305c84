// Frozen-block streaming: pinned-host masters of frozen transformer blocks, copied on demand
// into a small set of device staging slots on a caller-owned copy stream.
//
// The reference keeps this state machine in Python (training/memory.py:92-360): per slot a
// resident block index, a generation counter, a lease flag and two events - `ready` (the H2D
// copy finished) and `reusable` (the last kernel that read the slot finished). Here the same
// rules run natively, and the copy is one copy-engine transfer of the block's packed master:
//   * select  : the slot that already holds the block, else an empty slot, else the first
//               slot that is neither leased nor protected (the running block and the block
//               being prefetched);
//   * stage   : the copy stream waits for the slot's `reusable` event, copies the master into
//               the slot and records `ready`; the generation advances;
//   * lease   : the compute stream waits for `ready`; a leased slot is never overwritten;
//   * hold    : a checkpoint recomputation keeps the lease until the block's backward is done;
//   * release : records `reusable` on the stream that used the slot and drops the lease
//               (optionally checking that the slot still holds the same block generation).
// Slot memory is supplied by the caller (device allocations it owns), so views of a slot stay
// valid for as long as the caller keeps them.
#include <algorithm>
#include <mutex>
#include <vector>

#include "errors.cuh"

namespace moss {
namespace {

struct DeviceGuard {
  int prev = 0;
  bool ok = false;
  explicit DeviceGuard(int device) {
    if (cudaGetDevice(&prev) == cudaSuccess) ok = cudaSetDevice(device) == cudaSuccess;
  }
  ~DeviceGuard() { cudaSetDevice(prev); }
};

struct MasterBlock {
  const void* host = nullptr;
  size_t bytes = 0;
};

struct Slot {
  void* device = nullptr;
  size_t capacity = 0;
  int64_t block = -1;
  uint64_t generation = 0;
  bool leased = false;
  bool has_reusable = false;
  cudaEvent_t ready = nullptr;
  cudaEvent_t reusable = nullptr;
};

struct TimedCopy {
  cudaEvent_t start = nullptr;
  cudaEvent_t end = nullptr;
  size_t bytes = 0;
};

struct Stager {
  std::mutex mu;
  int device = 0;
  cudaStream_t copy = nullptr;
  std::vector<MasterBlock> blocks;
  std::vector<Slot> slots;
  std::vector<TimedCopy> pending;       // timing pairs of copies not yet accounted
  std::vector<TimedCopy> spare;         // recycled timing pairs
  uint64_t copies = 0;
  uint64_t bytes = 0;
  uint64_t timed_bytes = 0;
  double copy_ms = 0.0;
  int peak_resident = 0;
};

constexpr size_t kMaxPendingTimings = 64;

int resident_count(const Stager& s) {
  int n = 0;
  for (const Slot& slot : s.slots) n += slot.block >= 0;
  return n;
}

// Fold finished timing pairs into the totals; with `wait`, wait for all of them first.
int account_timings(Stager& s, bool wait) {
  std::vector<TimedCopy> still;
  for (TimedCopy& t : s.pending) {
    cudaError_t e = wait ? cudaEventSynchronize(t.end) : cudaEventQuery(t.end);
    if (e == cudaErrorNotReady) {
      still.push_back(t);
      continue;
    }
    if (e != cudaSuccess) return check_cuda(e, "block stager copy timing");
    float ms = 0.f;
    MOSS_CUDA_TRY(cudaEventElapsedTime(&ms, t.start, t.end));
    s.copy_ms += ms;
    s.timed_bytes += t.bytes;
    s.spare.push_back(t);
  }
  s.pending.swap(still);
  return MOSS_OK;
}

int timing_pair(Stager& s, TimedCopy* out) {
  if (!s.spare.empty()) {
    *out = s.spare.back();
    s.spare.pop_back();
    return MOSS_OK;
  }
  TimedCopy t;
  MOSS_CUDA_TRY(cudaEventCreate(&t.start));
  cudaError_t e = cudaEventCreate(&t.end);
  if (e != cudaSuccess) {
    cudaEventDestroy(t.start);
    return check_cuda(e, "cudaEventCreate");
  }
  *out = t;
  return MOSS_OK;
}

int check_slot(const Stager& s, int slot) {
  if (slot < 0 || slot >= static_cast<int>(s.slots.size()))
    return fail(MOSS_ERR_INVALID_ARGUMENT, "staging slot %d out of range [0, %zu)", slot, s.slots.size());
  return MOSS_OK;
}

void destroy_events(Stager& s) {
  for (Slot& slot : s.slots) {
    if (slot.ready) cudaEventDestroy(slot.ready);
    if (slot.reusable) cudaEventDestroy(slot.reusable);
    slot.ready = slot.reusable = nullptr;
  }
  for (auto* list : {&s.pending, &s.spare}) {
    for (TimedCopy& t : *list) {
      cudaEventDestroy(t.start);
      cudaEventDestroy(t.end);
    }
    list->clear();
  }
}

}  // namespace
}  // namespace moss

using moss::Stager;

extern "C" int moss_block_stager_create(int device, int num_slots, moss_stream_t copy, void** stager) {
  using namespace moss;
  if (stager == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null stager out-pointer");
  *stager = nullptr;
  if (num_slots < 1 || num_slots > 64) return fail(MOSS_ERR_INVALID_ARGUMENT, "num_slots must be in [1, 64]");
  if (copy == nullptr)
    return fail(MOSS_ERR_INVALID_ARGUMENT, "the block stager needs a dedicated (non-default) copy stream");
  Stager* s = new Stager();
  s->device = device;
  s->copy = reinterpret_cast<cudaStream_t>(copy);
  s->slots.resize(static_cast<size_t>(num_slots));
  DeviceGuard guard(device);
  cudaError_t e = guard.ok ? cudaSuccess : cudaErrorInvalidDevice;
  for (Slot& slot : s->slots) {
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&slot.ready, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&slot.reusable, cudaEventDisableTiming);
  }
  if (e != cudaSuccess) {
    destroy_events(*s);
    delete s;
    return check_cuda(e, "block stager setup");
  }
  *stager = s;
  return clear_ok();
}

extern "C" int moss_block_stager_destroy(void* stager, int force) {
  using namespace moss;
  if (stager == nullptr) return clear_ok();
  Stager* s = static_cast<Stager*>(stager);
  cudaError_t e = cudaSuccess;
  {
    std::lock_guard<std::mutex> lock(s->mu);
    if (!force && std::any_of(s->slots.begin(), s->slots.end(), [](const Slot& slot) { return slot.leased; }))
      return fail(MOSS_ERR_BUSY, "a staging slot is still leased by a running block or a pending backward");
    DeviceGuard guard(s->device);
    e = cudaStreamSynchronize(s->copy);
    for (Slot& slot : s->slots) {
      cudaError_t w = slot.has_reusable ? cudaEventSynchronize(slot.reusable) : cudaSuccess;
      if (e == cudaSuccess) e = w;
    }
    destroy_events(*s);
  }
  delete s;
  const int rc = check_cuda(e, "block stager teardown");
  return rc == MOSS_OK ? clear_ok() : rc;
}

extern "C" int moss_block_stager_add_block(void* stager, const void* host, size_t nbytes, int64_t* block) {
  using namespace moss;
  if (stager == nullptr || block == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null stager or block pointer");
  if (nbytes > 0) {
    if (host == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null block master");
    cudaPointerAttributes attr{};
    const cudaError_t e = cudaPointerGetAttributes(&attr, host);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return check_cuda(e, "block master attributes");
    }
    if (attr.type != cudaMemoryTypeHost)
      return fail(MOSS_ERR_INVALID_ARGUMENT, "block masters must be page-locked (pinned) host memory");
  }
  Stager& s = *static_cast<Stager*>(stager);
  std::lock_guard<std::mutex> lock(s.mu);
  *block = static_cast<int64_t>(s.blocks.size());
  s.blocks.push_back({host, nbytes});
  return clear_ok();
}

extern "C" int moss_block_stager_set_slot(void* stager, int slot, void* device, size_t capacity) {
  using namespace moss;
  if (stager == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null stager");
  if (capacity > 0 && device == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null slot memory");
  Stager& s = *static_cast<Stager*>(stager);
  std::lock_guard<std::mutex> lock(s.mu);
  if (int rc = check_slot(s, slot)) return rc;
  Slot& target = s.slots[slot];
  if (target.leased) return fail(MOSS_ERR_BUSY, "staging slot %d is leased", slot);
  if (target.block >= 0 && capacity < s.blocks[target.block].bytes)
    return fail(MOSS_ERR_INVALID_ARGUMENT, "slot memory smaller than its resident block");
  target.device = device;
  target.capacity = capacity;
  return clear_ok();
}

extern "C" int moss_block_stager_select(void* stager, int64_t block, const int64_t* protected_blocks, int n_protected,
                                        int* slot) {
  using namespace moss;
  if (stager == nullptr || slot == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null stager or slot pointer");
  if (n_protected < 0 || (n_protected > 0 && protected_blocks == nullptr))
    return fail(MOSS_ERR_INVALID_ARGUMENT, "bad protected block list");
  Stager& s = *static_cast<Stager*>(stager);
  std::lock_guard<std::mutex> lock(s.mu);
  if (block < 0 || block >= static_cast<int64_t>(s.blocks.size()))
    return fail(MOSS_ERR_NOT_FOUND, "block %lld is not registered", static_cast<long long>(block));
  const int n = static_cast<int>(s.slots.size());
  for (int i = 0; i < n; ++i)
    if (s.slots[i].block == block) {
      *slot = i;
      return clear_ok();
    }
  for (int i = 0; i < n; ++i)
    if (s.slots[i].block < 0) {
      *slot = i;
      return clear_ok();
    }
  for (int i = 0; i < n; ++i) {
    const Slot& candidate = s.slots[i];
    const bool is_protected =
        std::find(protected_blocks, protected_blocks + n_protected, candidate.block) != protected_blocks + n_protected;
    if (!candidate.leased && !is_protected) {
      *slot = i;
      return clear_ok();
    }
  }
  return fail(MOSS_ERR_BUSY, "every staging slot is leased or protected");
}

extern "C" int moss_block_stager_stage(void* stager, int64_t block, int slot, uint64_t* generation) {
  using namespace moss;
  if (stager == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null stager");
  Stager& s = *static_cast<Stager*>(stager);
  std::lock_guard<std::mutex> lock(s.mu);
  if (int rc = check_slot(s, slot)) return rc;
  if (block < 0 || block >= static_cast<int64_t>(s.blocks.size()))
    return fail(MOSS_ERR_NOT_FOUND, "block %lld is not registered", static_cast<long long>(block));
  Slot& target = s.slots[slot];
  if (target.block != block) {
    const MasterBlock& master = s.blocks[block];
    if (target.leased) return fail(MOSS_ERR_BUSY, "staging slot %d is leased", slot);
    if (target.capacity < master.bytes)
      return fail(MOSS_ERR_INVALID_ARGUMENT, "staging slot %d holds %zu bytes, block %lld needs %zu", slot,
                  target.capacity, static_cast<long long>(block), master.bytes);
    DeviceGuard guard(s.device);
    if (target.has_reusable) MOSS_CUDA_TRY(cudaStreamWaitEvent(s.copy, target.reusable, 0));
    if (master.bytes > 0) {
      if (s.pending.size() >= kMaxPendingTimings)
        if (int rc = account_timings(s, false)) return rc;
      TimedCopy t{};
      const bool timed = s.pending.size() < kMaxPendingTimings && timing_pair(s, &t) == MOSS_OK;
      if (timed) MOSS_CUDA_TRY(cudaEventRecord(t.start, s.copy));
      MOSS_CUDA_TRY(cudaMemcpyAsync(target.device, master.host, master.bytes, cudaMemcpyHostToDevice, s.copy));
      if (timed) {
        MOSS_CUDA_TRY(cudaEventRecord(t.end, s.copy));
        t.bytes = master.bytes;
        s.pending.push_back(t);
      }
    }
    MOSS_CUDA_TRY(cudaEventRecord(target.ready, s.copy));
    // later copies into this slot are ordered behind this one on the copy stream
    target.has_reusable = false;
    target.block = block;
    target.generation += 1;
    s.copies += 1;
    s.bytes += master.bytes;
    s.peak_resident = std::max(s.peak_resident, resident_count(s));
  }
  if (generation != nullptr) *generation = target.generation;
  return clear_ok();
}

extern "C" int moss_block_stager_lease(void* stager, int slot, moss_stream_t compute, uint64_t* generation) {
  using namespace moss;
  if (stager == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null stager");
  Stager& s = *static_cast<Stager*>(stager);
  std::lock_guard<std::mutex> lock(s.mu);
  if (int rc = check_slot(s, slot)) return rc;
  Slot& target = s.slots[slot];
  if (target.block < 0) return fail(MOSS_ERR_NOT_FOUND, "staging slot %d holds no block", slot);
  if (target.leased) return fail(MOSS_ERR_BUSY, "staging slot %d is already leased", slot);
  DeviceGuard guard(s.device);
  MOSS_CUDA_TRY(cudaStreamWaitEvent(reinterpret_cast<cudaStream_t>(compute), target.ready, 0));
  target.leased = true;
  if (generation != nullptr) *generation = target.generation;
  return clear_ok();
}

extern "C" int moss_block_stager_hold(void* stager, int slot) {
  using namespace moss;
  if (stager == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null stager");
  Stager& s = *static_cast<Stager*>(stager);
  std::lock_guard<std::mutex> lock(s.mu);
  if (int rc = check_slot(s, slot)) return rc;
  Slot& target = s.slots[slot];
  if (!target.leased) return fail(MOSS_ERR_INVALID_ARGUMENT, "staging slot %d is not leased", slot);
  target.has_reusable = false;
  return clear_ok();
}

extern "C" int moss_block_stager_release(void* stager, int slot, int64_t block, uint64_t generation,
                                         moss_stream_t stream) {
  using namespace moss;
  if (stager == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null stager");
  Stager& s = *static_cast<Stager*>(stager);
  std::lock_guard<std::mutex> lock(s.mu);
  if (int rc = check_slot(s, slot)) return rc;
  Slot& target = s.slots[slot];
  if (block >= 0 && (target.block != block || target.generation != generation))
    return fail(MOSS_ERR_NOT_FOUND, "staging slot %d changed before its user finished", slot);
  DeviceGuard guard(s.device);
  MOSS_CUDA_TRY(cudaEventRecord(target.reusable, reinterpret_cast<cudaStream_t>(stream)));
  target.has_reusable = true;
  target.leased = false;
  return clear_ok();
}

extern "C" int moss_block_stager_slot_info(void* stager, int slot, int64_t* block, uint64_t* generation,
                                           int* leased) {
  using namespace moss;
  if (stager == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null stager");
  Stager& s = *static_cast<Stager*>(stager);
  std::lock_guard<std::mutex> lock(s.mu);
  if (int rc = check_slot(s, slot)) return rc;
  const Slot& target = s.slots[slot];
  if (block != nullptr) *block = target.block;
  if (generation != nullptr) *generation = target.generation;
  if (leased != nullptr) *leased = target.leased ? 1 : 0;
  return clear_ok();
}

extern "C" int moss_block_stager_stats(void* stager, uint64_t* copies, uint64_t* bytes, int* peak_resident,
                                       double* copy_ms, uint64_t* timed_bytes) {
  using namespace moss;
  if (stager == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null stager");
  Stager& s = *static_cast<Stager*>(stager);
  std::lock_guard<std::mutex> lock(s.mu);
  if (copy_ms != nullptr || timed_bytes != nullptr) {
    DeviceGuard guard(s.device);
    if (int rc = account_timings(s, true)) return rc;
  }
  if (copies != nullptr) *copies = s.copies;
  if (bytes != nullptr) *bytes = s.bytes;
  if (peak_resident != nullptr) *peak_resident = s.peak_resident;
  if (copy_ms != nullptr) *copy_ms = s.copy_ms;
  if (timed_bytes != nullptr) *timed_bytes = s.timed_bytes;
  return clear_ok();
}
