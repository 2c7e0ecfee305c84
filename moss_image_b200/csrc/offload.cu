// Saved-activation offload: strided gather/scatter kernels and the pinned-host ring.
//
// The reference (training/activation_offload.py:116-147) allocates pinned memory per saved
// tensor and issues the D2H copy on the compute stream, and issues the H2D copy on demand
// when autograd unpacks. Here:
//   * one pinned arena made of cudaHostAlloc segments, bump-allocated per saved tensor and
//     rewound when no ticket is live (segments are kept for the next step);
//   * D2H copies on a dedicated stream, ordered after the producing kernels by an event
//     recorded on the compute stream; H2D copies on a second dedicated stream, ordered
//     after the ticket's D2H; the compute stream waits on the ticket's H2D event only when
//     autograd actually needs the tensor, so restores can be issued ahead (prefetch);
//   * non-contiguous payload views are first gathered on the GPU into one dense buffer so
//     each saved tensor is a single copy-engine transfer (and scattered back on restore).
#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "errors.cuh"

namespace moss {

constexpr int kMaxDims = 8;

struct StridedDesc {
  int ndim;
  int64_t sizes[kMaxDims];
  int64_t strides[kMaxDims];
};

// dense index i (row-major over sizes) -> element offset in the strided view
__device__ __forceinline__ int64_t strided_offset(const StridedDesc& d, int64_t i) {
  int64_t off = 0;
  for (int k = d.ndim - 1; k >= 0; --k) {
    const int64_t sz = d.sizes[k];
    const int64_t idx = i % sz;
    i /= sz;
    off += idx * d.strides[k];
  }
  return off;
}

template <typename T, bool kGather>
__global__ void strided_copy_kernel(const T* __restrict__ src, T* __restrict__ dst, StridedDesc d, int64_t total) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t off = strided_offset(d, i);
    if (kGather)
      dst[i] = src[off];
    else
      dst[off] = src[i];
  }
}

template <bool kGather>
static int strided_copy(const void* src, int64_t elem_size, int ndim, const int64_t* sizes, const int64_t* strides,
                        void* dst, cudaStream_t stream) {
  if (ndim < 0 || ndim > kMaxDims) return fail(MOSS_ERR_INVALID_ARGUMENT, "ndim must be in [0, %d]", kMaxDims);
  if (ndim > 0 && (sizes == nullptr || strides == nullptr))
    return fail(MOSS_ERR_INVALID_ARGUMENT, "null sizes/strides");
  StridedDesc d{};
  d.ndim = ndim;
  int64_t total = 1;
  for (int i = 0; i < ndim; ++i) {
    if (sizes[i] < 0 || strides[i] < 0) return fail(MOSS_ERR_INVALID_ARGUMENT, "negative size or stride");
    d.sizes[i] = sizes[i];
    d.strides[i] = strides[i];
    total *= sizes[i];
  }
  if (total == 0) return clear_ok();
  if (src == nullptr || dst == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null pointer");
  if (ndim == 0) d.ndim = 0;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 148 * 16));
  switch (elem_size) {
    case 1:
      strided_copy_kernel<uint8_t, kGather><<<grid, 256, 0, stream>>>(static_cast<const uint8_t*>(src),
                                                                     static_cast<uint8_t*>(dst), d, total);
      break;
    case 2:
      strided_copy_kernel<uint16_t, kGather><<<grid, 256, 0, stream>>>(static_cast<const uint16_t*>(src),
                                                                      static_cast<uint16_t*>(dst), d, total);
      break;
    case 4:
      strided_copy_kernel<uint32_t, kGather><<<grid, 256, 0, stream>>>(static_cast<const uint32_t*>(src),
                                                                      static_cast<uint32_t*>(dst), d, total);
      break;
    case 8:
      strided_copy_kernel<uint64_t, kGather><<<grid, 256, 0, stream>>>(static_cast<const uint64_t*>(src),
                                                                      static_cast<uint64_t*>(dst), d, total);
      break;
    default:
      return fail(MOSS_ERR_UNSUPPORTED, "element size %lld is not 1, 2, 4 or 8", (long long)elem_size);
  }
  MOSS_CUDA_TRY(cudaGetLastError());
  return clear_ok();
}

// ------------------------------------------------------------------------------------ ring
struct Segment {
  uint8_t* host = nullptr;
  size_t bytes = 0;
};

struct Ticket {
  bool live = false;
  int seg = 0;
  size_t off = 0;
  size_t bytes = 0;
  cudaEvent_t d2h_done = nullptr;
  cudaEvent_t h2d_done = nullptr;
  bool h2d_issued = false;
};

struct OffloadRing {
  int device = 0;
  size_t segment_bytes = 0;
  size_t max_bytes = 0;
  cudaStream_t d2h = nullptr;
  cudaStream_t h2d = nullptr;
  std::vector<Segment> segments;
  size_t reserved = 0;
  int cur_seg = 0;
  size_t cur_off = 0;
  std::vector<Ticket> tickets;
  std::vector<int64_t> free_slots;
  int64_t live = 0;
  cudaEvent_t rewind_fence = nullptr;  // last H2D before a rewind
  bool fence_pending = false;
  uint64_t d2h_bytes = 0, h2d_bytes = 0;
  // Optional copy-engine timing (moss_offload_set_timing): an event pair around each copy.
  bool timing = false;
  struct TimedCopy {
    cudaEvent_t start = nullptr, end = nullptr;
    size_t bytes = 0;
    bool h2d = false;
  };
  std::vector<TimedCopy> pending;     // recorded, not yet harvested
  std::vector<TimedCopy> event_pool;  // harvested pairs, reused
  double d2h_ms = 0.0, h2d_ms = 0.0;
  uint64_t d2h_timed_bytes = 0, h2d_timed_bytes = 0;
  std::mutex mu;
};

// Event pair for one timed copy (from the pool, or new).
static int timed_copy_begin(OffloadRing& r, bool h2d, size_t bytes, cudaStream_t stream, OffloadRing::TimedCopy* out) {
  OffloadRing::TimedCopy c;
  if (!r.event_pool.empty()) {
    c = r.event_pool.back();
    r.event_pool.pop_back();
  } else {
    MOSS_CUDA_TRY(cudaEventCreate(&c.start));
    MOSS_CUDA_TRY(cudaEventCreate(&c.end));
  }
  c.bytes = bytes;
  c.h2d = h2d;
  MOSS_CUDA_TRY(cudaEventRecord(c.start, stream));
  *out = c;
  return MOSS_OK;
}

// Accumulate the copies whose end event has completed (all of them when `wait` is set).
static void harvest(OffloadRing& r, bool wait) {
  size_t keep = 0;
  for (size_t i = 0; i < r.pending.size(); ++i) {
    OffloadRing::TimedCopy& c = r.pending[i];
    if (wait) cudaEventSynchronize(c.end);
    float ms = 0.0f;
    if (cudaEventQuery(c.end) == cudaSuccess && cudaEventElapsedTime(&ms, c.start, c.end) == cudaSuccess) {
      if (c.h2d) {
        r.h2d_ms += ms;
        r.h2d_timed_bytes += c.bytes;
      } else {
        r.d2h_ms += ms;
        r.d2h_timed_bytes += c.bytes;
      }
      r.event_pool.push_back(c);
    } else {
      cudaGetLastError();
      r.pending[keep++] = c;
    }
  }
  r.pending.resize(keep);
}

static constexpr size_t kAlign = 256;

static int ensure_events(Ticket& t) {
  if (t.d2h_done == nullptr) MOSS_CUDA_TRY(cudaEventCreateWithFlags(&t.d2h_done, cudaEventDisableTiming));
  if (t.h2d_done == nullptr) MOSS_CUDA_TRY(cudaEventCreateWithFlags(&t.h2d_done, cudaEventDisableTiming));
  return MOSS_OK;
}

// Reserve `bytes` of pinned space (growing the arena when allowed).
static int reserve(OffloadRing& r, size_t bytes, int* seg_out, size_t* off_out) {
  const size_t need = (bytes + kAlign - 1) / kAlign * kAlign;
  while (true) {
    if (r.cur_seg < static_cast<int>(r.segments.size())) {
      Segment& s = r.segments[r.cur_seg];
      if (r.cur_off + need <= s.bytes) {
        *seg_out = r.cur_seg;
        *off_out = r.cur_off;
        r.cur_off += need;
        return MOSS_OK;
      }
      ++r.cur_seg;
      r.cur_off = 0;
      continue;
    }
    const size_t seg_bytes = std::max(r.segment_bytes, need);
    if (r.reserved + seg_bytes > r.max_bytes)
      return fail(MOSS_ERR_RING_FULL, "offload ring full: %zu bytes reserved, %zu more needed, limit %zu", r.reserved,
                  seg_bytes, r.max_bytes);
    Segment s;
    void* p = nullptr;
    MOSS_CUDA_TRY(cudaHostAlloc(&p, seg_bytes, cudaHostAllocPortable));
    s.host = static_cast<uint8_t*>(p);
    s.bytes = seg_bytes;
    r.segments.push_back(s);
    r.reserved += seg_bytes;
    // loop picks up the new segment at r.cur_seg
  }
}

static Ticket* lookup(OffloadRing& r, int64_t ticket) {
  if (ticket < 0 || ticket >= static_cast<int64_t>(r.tickets.size())) return nullptr;
  Ticket& t = r.tickets[ticket];
  return t.live ? &t : nullptr;
}

}  // namespace moss

using namespace moss;

extern "C" int moss_strided_gather(const void* src, int64_t elem_size, int ndim, const int64_t* sizes,
                                   const int64_t* strides, void* dst, moss_stream_t stream) {
  return strided_copy<true>(src, elem_size, ndim, sizes, strides, dst, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int moss_strided_scatter(const void* src, int64_t elem_size, int ndim, const int64_t* sizes,
                                    const int64_t* strides, void* dst, moss_stream_t stream) {
  return strided_copy<false>(src, elem_size, ndim, sizes, strides, dst, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int moss_offload_ring_create(int device, size_t segment_bytes, size_t max_bytes, moss_stream_t d2h,
                                        moss_stream_t h2d, void** ring) {
  if (ring == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null ring out-pointer");
  if (d2h == nullptr || h2d == nullptr)
    return fail(MOSS_ERR_INVALID_ARGUMENT, "the offload ring needs two dedicated (non-default) streams");
  if (segment_bytes == 0 || max_bytes < segment_bytes)
    return fail(MOSS_ERR_INVALID_ARGUMENT, "segment_bytes must be > 0 and <= max_bytes");
  OffloadRing* r = new OffloadRing();
  r->device = device;
  r->segment_bytes = segment_bytes;
  r->max_bytes = max_bytes;
  r->d2h = reinterpret_cast<cudaStream_t>(d2h);
  r->h2d = reinterpret_cast<cudaStream_t>(h2d);
  int prev = 0;
  cudaGetDevice(&prev);
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&r->rewind_fence, cudaEventDisableTiming);
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    delete r;
    return check_cuda(e, "offload ring setup");
  }
  *ring = r;
  return clear_ok();
}

extern "C" int moss_offload_ring_destroy(void* ring) {
  if (ring == nullptr) return clear_ok();
  OffloadRing* r = static_cast<OffloadRing*>(ring);
  {
    std::lock_guard<std::mutex> lock(r->mu);
    cudaStreamSynchronize(r->d2h);
    cudaStreamSynchronize(r->h2d);
    for (Ticket& t : r->tickets) {
      if (t.d2h_done) cudaEventDestroy(t.d2h_done);
      if (t.h2d_done) cudaEventDestroy(t.h2d_done);
    }
    for (auto& c : r->pending) {
      cudaEventDestroy(c.start);
      cudaEventDestroy(c.end);
    }
    for (auto& c : r->event_pool) {
      cudaEventDestroy(c.start);
      cudaEventDestroy(c.end);
    }
    for (Segment& s : r->segments) cudaFreeHost(s.host);
    if (r->rewind_fence) cudaEventDestroy(r->rewind_fence);
  }
  delete r;
  return clear_ok();
}

extern "C" int moss_offload_pack(void* ring, const void* src, size_t nbytes, moss_stream_t compute, int64_t* ticket) {
  if (ring == nullptr || ticket == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null ring or ticket pointer");
  if (nbytes > 0 && src == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null source");
  OffloadRing& r = *static_cast<OffloadRing*>(ring);
  std::lock_guard<std::mutex> lock(r.mu);
  int seg = 0;
  size_t off = 0;
  int rc = reserve(r, nbytes, &seg, &off);
  if (rc != MOSS_OK) return rc;
  int64_t id;
  if (!r.free_slots.empty()) {
    id = r.free_slots.back();
    r.free_slots.pop_back();
  } else {
    id = static_cast<int64_t>(r.tickets.size());
    r.tickets.emplace_back();
  }
  Ticket& t = r.tickets[id];
  rc = ensure_events(t);
  if (rc != MOSS_OK) return rc;
  t.live = true;
  t.seg = seg;
  t.off = off;
  t.bytes = nbytes;
  t.h2d_issued = false;
  ++r.live;
  // The D2H stream first waits for the producing kernels (recorded on `compute`) and, after
  // a rewind, for the H2D copies that still read the region being reused.
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(compute);
  MOSS_CUDA_TRY(cudaEventRecord(t.d2h_done, cs));
  MOSS_CUDA_TRY(cudaStreamWaitEvent(r.d2h, t.d2h_done, 0));
  if (r.fence_pending) {
    MOSS_CUDA_TRY(cudaStreamWaitEvent(r.d2h, r.rewind_fence, 0));
    r.fence_pending = false;
  }
  if (nbytes > 0) {
    OffloadRing::TimedCopy tc;
    if (r.timing) {
      rc = timed_copy_begin(r, false, nbytes, r.d2h, &tc);
      if (rc != MOSS_OK) return rc;
    }
    MOSS_CUDA_TRY(cudaMemcpyAsync(r.segments[seg].host + off, src, nbytes, cudaMemcpyDeviceToHost, r.d2h));
    if (r.timing) {
      MOSS_CUDA_TRY(cudaEventRecord(tc.end, r.d2h));
      r.pending.push_back(tc);
      if (r.pending.size() > 4096) harvest(r, false);
    }
  }
  MOSS_CUDA_TRY(cudaEventRecord(t.d2h_done, r.d2h));
  r.d2h_bytes += nbytes;
  *ticket = id;
  return clear_ok();
}

extern "C" int moss_offload_prefetch(void* ring, int64_t ticket, void* dst) {
  if (ring == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null ring");
  OffloadRing& r = *static_cast<OffloadRing*>(ring);
  std::lock_guard<std::mutex> lock(r.mu);
  Ticket* t = lookup(r, ticket);
  if (t == nullptr) return fail(MOSS_ERR_NOT_FOUND, "unknown or released offload ticket %lld", (long long)ticket);
  if (t->bytes > 0 && dst == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null destination");
  MOSS_CUDA_TRY(cudaStreamWaitEvent(r.h2d, t->d2h_done, 0));
  if (t->bytes > 0) {
    OffloadRing::TimedCopy tc;
    if (r.timing) {
      const int rc = timed_copy_begin(r, true, t->bytes, r.h2d, &tc);
      if (rc != MOSS_OK) return rc;
    }
    MOSS_CUDA_TRY(cudaMemcpyAsync(dst, r.segments[t->seg].host + t->off, t->bytes, cudaMemcpyHostToDevice, r.h2d));
    if (r.timing) {
      MOSS_CUDA_TRY(cudaEventRecord(tc.end, r.h2d));
      r.pending.push_back(tc);
      if (r.pending.size() > 4096) harvest(r, false);
    }
  }
  MOSS_CUDA_TRY(cudaEventRecord(t->h2d_done, r.h2d));
  t->h2d_issued = true;
  r.h2d_bytes += t->bytes;
  return clear_ok();
}

extern "C" int moss_offload_wait(void* ring, int64_t ticket, moss_stream_t compute) {
  if (ring == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null ring");
  OffloadRing& r = *static_cast<OffloadRing*>(ring);
  std::lock_guard<std::mutex> lock(r.mu);
  Ticket* t = lookup(r, ticket);
  if (t == nullptr) return fail(MOSS_ERR_NOT_FOUND, "unknown or released offload ticket %lld", (long long)ticket);
  if (!t->h2d_issued) return fail(MOSS_ERR_INVALID_ARGUMENT, "ticket %lld has no restore in flight", (long long)ticket);
  MOSS_CUDA_TRY(cudaStreamWaitEvent(reinterpret_cast<cudaStream_t>(compute), t->h2d_done, 0));
  return clear_ok();
}

extern "C" int moss_offload_release(void* ring, int64_t ticket) {
  if (ring == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null ring");
  OffloadRing& r = *static_cast<OffloadRing*>(ring);
  std::lock_guard<std::mutex> lock(r.mu);
  Ticket* t = lookup(r, ticket);
  if (t == nullptr) return fail(MOSS_ERR_NOT_FOUND, "unknown or released offload ticket %lld", (long long)ticket);
  // Space is only reused after a rewind; the rewind fence below orders later D2H writes
  // after every H2D read issued so far, and D2H copies are ordered among themselves.
  t->live = false;
  r.free_slots.push_back(ticket);
  if (--r.live == 0) {
    // Rewind: every later D2H must wait for all H2D copies issued so far.
    MOSS_CUDA_TRY(cudaEventRecord(r.rewind_fence, r.h2d));
    r.fence_pending = true;
    r.cur_seg = 0;
    r.cur_off = 0;
  }
  return clear_ok();
}

extern "C" int moss_offload_host_ptr(void* ring, int64_t ticket, void** host) {
  if (ring == nullptr || host == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null argument");
  OffloadRing& r = *static_cast<OffloadRing*>(ring);
  std::lock_guard<std::mutex> lock(r.mu);
  Ticket* t = lookup(r, ticket);
  if (t == nullptr) return fail(MOSS_ERR_NOT_FOUND, "unknown or released offload ticket %lld", (long long)ticket);
  *host = r.segments[t->seg].host + t->off;
  return clear_ok();
}

extern "C" int moss_offload_stats(void* ring, uint64_t* d2h_bytes, uint64_t* h2d_bytes, int64_t* live,
                                  uint64_t* pinned_bytes) {
  if (ring == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null ring");
  OffloadRing& r = *static_cast<OffloadRing*>(ring);
  std::lock_guard<std::mutex> lock(r.mu);
  if (d2h_bytes) *d2h_bytes = r.d2h_bytes;
  if (h2d_bytes) *h2d_bytes = r.h2d_bytes;
  if (live) *live = r.live;
  if (pinned_bytes) *pinned_bytes = r.reserved;
  return clear_ok();
}

extern "C" int moss_offload_set_timing(void* ring, int enable) {
  if (ring == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null ring");
  OffloadRing& r = *static_cast<OffloadRing*>(ring);
  std::lock_guard<std::mutex> lock(r.mu);
  r.timing = enable != 0;
  return clear_ok();
}

extern "C" int moss_offload_copy_time(void* ring, double* d2h_ms, double* h2d_ms, uint64_t* d2h_timed_bytes,
                                      uint64_t* h2d_timed_bytes) {
  if (ring == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null ring");
  OffloadRing& r = *static_cast<OffloadRing*>(ring);
  std::lock_guard<std::mutex> lock(r.mu);
  harvest(r, true);
  if (d2h_ms) *d2h_ms = r.d2h_ms;
  if (h2d_ms) *h2d_ms = r.h2d_ms;
  if (d2h_timed_bytes) *d2h_timed_bytes = r.d2h_timed_bytes;
  if (h2d_timed_bytes) *h2d_timed_bytes = r.h2d_timed_bytes;
  return clear_ok();
}
