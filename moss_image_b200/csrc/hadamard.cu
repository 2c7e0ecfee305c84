// Grouped normalised Hadamard rotation for ConvRot-quantised linears (sm_100a).
//
// ConvRot stores W·H in int8 and computes (x·H)·(W·H)^T; the input gradient is H·(dY·dec(W·H)).
// H is block-diagonal with `group`-sized blocks (a power of two) built from the regular H4
// (and one H2 factor for odd log2(group)). The reference runs one elementwise kernel per stage
// through a scratch tensor, storing every stage in the tensor's dtype
// (training/quant_kernels.py:231-277, :376-426). Here one CTA stages a tile of rows x one group
// in shared memory (f32) and runs every stage there: one HBM read and one write in total,
// with the same per-stage arithmetic and rounding, so the result is bit-identical:
//   radix 4 (strides 1, 4, 16, ...): total = ((a + b) + c) + d;
//                                   out[digit] = (total - 2 * {d, c, b, a}[digit]) * 0.5
//   radix 2 (last, odd log2(group)):  (a + b) * 0.70710678f, (a - b) * 0.70710678f
// Explicit round-to-nearest intrinsics keep the compiler from contracting or reassociating.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "errors.cuh"

namespace moss {
namespace {

constexpr int kThreads = 256;
constexpr int kTileFloats = 8192;  // 32 KB of shared memory per tile
constexpr int64_t kMaxGroup = kTileFloats;

// Round an f32 to the storage kind and back (round to nearest even). The bf16 case uses
// integer arithmetic, which is cheaper than a scalar conversion round trip.
__device__ __forceinline__ float round_stage(float x, int kind) {
  if (kind == kBF16) {
    uint32_t u = __float_as_uint(x);
    if ((u & 0x7fffffffu) > 0x7f800000u) return __uint_as_float((u | 0x00400000u) & 0xffff0000u);  // NaN stays NaN
    u += 0x7fffu + ((u >> 16) & 1u);
    return __uint_as_float(u & 0xffff0000u);
  }
  if (kind == kF16) return __half2float(__float2half_rn(x));
  return x;
}

__global__ void __launch_bounds__(kThreads)
    hadamard_kernel(const void* x, void* y, int kind, int64_t rows, int64_t cols, int group, int rows_per_tile) {
  extern __shared__ float tile[];
  const int64_t groups_per_row = cols / group;
  const int64_t row_tiles = (rows + rows_per_tile - 1) / rows_per_tile;
  const int64_t tiles = row_tiles * groups_per_row;
  const int esize = kind == kF32 ? 4 : 2;
  const bool vec = (group % 8 == 0) && (cols % 8 == 0) && esize == 2 &&
                   (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0;
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int64_t row0 = (t / groups_per_row) * rows_per_tile;
    const int64_t col0 = (t % groups_per_row) * group;
    const int nrows = static_cast<int>(std::min<int64_t>(rows_per_tile, rows - row0));
    const int count = nrows * group;
    // load (16 bytes per thread when possible)
    if (vec) {
      for (int i = threadIdx.x * 8; i < count; i += kThreads * 8) {
        const int r = i / group, c = i - r * group;
        const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + (row0 + r) * cols + col0 + c);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (kind == kBF16) {
            tile[i + 2 * j] = __uint_as_float(w[j] << 16);
            tile[i + 2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
          } else {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
            tile[i + 2 * j] = f.x;
            tile[i + 2 * j + 1] = f.y;
          }
        }
      }
    } else {
      for (int i = threadIdx.x; i < count; i += kThreads) {
        const int r = i / group, c = i - r * group;
        tile[i] = load_as_float(x, kind, (row0 + r) * cols + col0 + c);
      }
    }
    __syncthreads();
    int stride = 1;
    while (stride * 4 <= group) {
      const int quads = count / 4;
      const int per_row = group / 4;
      for (int qd = threadIdx.x; qd < quads; qd += kThreads) {
        const int r = qd / per_row, qq = qd - r * per_row;
        const int blk = qq / stride, pos = qq - blk * stride;
        float* v = tile + r * group + blk * 4 * stride + pos;
        const float a = v[0], b = v[stride], c = v[2 * stride], d = v[3 * stride];
        const float total = __fadd_rn(__fadd_rn(__fadd_rn(a, b), c), d);
        v[0] = round_stage(__fmul_rn(__fsub_rn(total, __fmul_rn(2.0f, d)), 0.5f), kind);
        v[stride] = round_stage(__fmul_rn(__fsub_rn(total, __fmul_rn(2.0f, c)), 0.5f), kind);
        v[2 * stride] = round_stage(__fmul_rn(__fsub_rn(total, __fmul_rn(2.0f, b)), 0.5f), kind);
        v[3 * stride] = round_stage(__fmul_rn(__fsub_rn(total, __fmul_rn(2.0f, a)), 0.5f), kind);
      }
      __syncthreads();
      stride *= 4;
    }
    if (stride < group) {
      const float h = 0.7071067811865476f;
      const int pairs = count / 2;
      const int per_row = group / 2;
      for (int pr = threadIdx.x; pr < pairs; pr += kThreads) {
        const int r = pr / per_row, pp = pr - r * per_row;
        const int blk = pp / stride, pos = pp - blk * stride;
        float* v = tile + r * group + blk * 2 * stride + pos;
        const float a = v[0], b = v[stride];
        v[0] = round_stage(__fmul_rn(__fadd_rn(a, b), h), kind);
        v[stride] = round_stage(__fmul_rn(__fsub_rn(a, b), h), kind);
      }
      __syncthreads();
    }
    // store (the values are already rounded to the storage kind)
    if (vec) {
      for (int i = threadIdx.x * 8; i < count; i += kThreads * 8) {
        const int r = i / group, c = i - r * group;
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if (kind == kBF16) {
            w[j] = (__float_as_uint(tile[i + 2 * j]) >> 16) | (__float_as_uint(tile[i + 2 * j + 1]) & 0xffff0000u);
          } else {
            __half2 h2 = __floats2half2_rn(tile[i + 2 * j], tile[i + 2 * j + 1]);
            w[j] = *reinterpret_cast<uint32_t*>(&h2);
          }
        }
        *reinterpret_cast<uint4*>(static_cast<uint16_t*>(y) + (row0 + r) * cols + col0 + c) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    } else {
      for (int i = threadIdx.x; i < count; i += kThreads) {
        const int r = i / group, c = i - r * group;
        store_from_float(y, kind, (row0 + r) * cols + col0 + c, tile[i]);
      }
    }
    __syncthreads();  // the next tile reuses the shared memory
  }
}

// ---------------------------------------------------------------------------------------------
// Register-resident variant for 16 <= group <= 4096 with 16-bit storage and 16-byte aligned rows.
// The group's index bits are processed in phases of 4: in phase p a thread owns the 16
// elements whose index differs only in bits [4p, 4p + 4), applies the radix-4 stages of those
// two bit pairs (and the final radix-2 stage on an odd top bit) in registers, and exchanges
// through shared memory between phases. Pairing, order and rounding are the staged
// transform's, so the result is identical to the general kernel above.
constexpr int kFastTile = 4096;  // elements per tile: 16 per thread
// one pad float per 16: a warp writing 16 consecutive floats per lane, or reading one float per
// lane at any power-of-two stride >= 16, hits 32 distinct banks
__device__ __forceinline__ int padded(int e) { return e + (e >> 4); }

// Round 2N values to the 16-bit storage type and back (exact for every representable value):
// one packed conversion per pair, the halves widened with integer ops.
template <int kKind, int N>
__device__ __forceinline__ void round_all(float (&v)[16]) {
  if constexpr (kKind == kF32) return;
#pragma unroll
  for (int i = 0; i < N; i += 2) {
    if constexpr (kKind == kBF16) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[i], v[i + 1]);
      uint32_t w;
      memcpy(&w, &h, sizeof(w));
      v[i] = __uint_as_float(w << 16);
      v[i + 1] = __uint_as_float(w & 0xffff0000u);
    } else {
      const float2 f = __half22float2(__floats2half2_rn(v[i], v[i + 1]));
      v[i] = f.x;
      v[i + 1] = f.y;
    }
  }
}

// Radix-4 stage on register index bits (2b, 2b + 1) of N registers: quads {j, j + s, j + 2s,
// j + 3s} with s = 4^b. The staged transform's (total - 2 x) * 0.5 is computed as
// total * 0.5 - x: halving is exact and commutes with the rounding, so every value whose
// magnitude stays in the normal range is identical, with one operation per output less.
template <int kStride, int N>
__device__ __forceinline__ void radix4(float (&v)[16]) {
#pragma unroll
  for (int j = 0; j < N; ++j) {
    if ((j / kStride) % 4 != 0) continue;
    const float a = v[j], b = v[j + kStride], c = v[j + 2 * kStride], d = v[j + 3 * kStride];
    const float half = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(a, b), c), d), 0.5f);
    v[j] = __fsub_rn(half, d);
    v[j + kStride] = __fsub_rn(half, c);
    v[j + 2 * kStride] = __fsub_rn(half, b);
    v[j + 3 * kStride] = __fsub_rn(half, a);
  }
}
template <int kStride, int N>
__device__ __forceinline__ void radix2(float (&v)[16]) {
  const float h = 0.7071067811865476f;
#pragma unroll
  for (int j = 0; j < N; ++j) {
    if ((j / kStride) % 2 != 0) continue;
    const float a = v[j], b = v[j + kStride];
    v[j] = __fmul_rn(__fadd_rn(a, b), h);
    v[j + kStride] = __fmul_rn(__fsub_rn(a, b), h);
  }
}

// All stages of one phase with NB (1..4) index bits in register bits [0, NB).
template <int kKind, int NB>
__device__ __forceinline__ void phase_stages(float (&v)[16]) {
  constexpr int N = 1 << NB;
  if constexpr (NB >= 2) {
    radix4<1, N>(v);
    round_all<kKind, N>(v);
  }
  if constexpr (NB == 4) {
    radix4<4, N>(v);
    round_all<kKind, N>(v);
  } else if constexpr (NB == 3) {
    radix2<4, N>(v);
    round_all<kKind, N>(v);
  } else if constexpr (NB == 1) {
    radix2<1, N>(v);
    round_all<kKind, N>(v);
  }
}

// Phase P (>= 1) of a tile held in shared memory: lines fix every index bit outside
// [4P, 4P + NB); lanes vary the low bits so a warp touches distinct banks.
template <int kKind, int LOG2G, int P>
__device__ __forceinline__ void smem_phase(float* tile, int nrows) {
  constexpr int kLow = 4 * P;
  constexpr int kNB = (LOG2G - kLow) < 4 ? (LOG2G - kLow) : 4;
  constexpr int kHiBits = LOG2G - kLow - kNB;
  constexpr int kN = 1 << kNB;
  const int lines = (nrows << LOG2G) >> kNB;
  for (int line = threadIdx.x; line < lines; line += kThreads) {
    const int lo = line & ((1 << kLow) - 1);
    const int rest = line >> kLow;  // (row, high bits)
    const int hi = rest & ((1 << kHiBits) - 1);
    const int row = rest >> kHiBits;
    const int base = (row << LOG2G) + lo + (hi << (kLow + kNB));
    float w[16];
#pragma unroll
    for (int i = 0; i < kN; ++i) w[i] = tile[padded(base + (i << kLow))];
    phase_stages<kKind, kNB>(w);
#pragma unroll
    for (int i = 0; i < kN; ++i) tile[padded(base + (i << kLow))] = w[i];
  }
  __syncthreads();
}

// The last phase of a tile: as smem_phase, but each thread stores its 16 outputs (already
// rounded to the storage kind) straight to global memory instead of back to shared memory.
// For a fixed i the 16 lanes of a half-warp store 16 consecutive elements (32 bytes).
template <int kKind>
__device__ __forceinline__ uint16_t storage_bits(float v) {
  if constexpr (kKind == kBF16) {
    return static_cast<uint16_t>(__float_as_uint(v) >> 16);
  } else {
    return __half_as_ushort(__float2half_rn(v));
  }
}
template <int kKind, int LOG2G, int P>
__device__ __forceinline__ void smem_phase_store(const float* tile, int nrows, uint16_t* y_tile) {
  constexpr int kLow = 4 * P;
  constexpr int kNB = (LOG2G - kLow) < 4 ? (LOG2G - kLow) : 4;
  constexpr int kHiBits = LOG2G - kLow - kNB;
  constexpr int kN = 1 << kNB;
  const int lines = (nrows << LOG2G) >> kNB;
  for (int line = threadIdx.x; line < lines; line += kThreads) {
    const int lo = line & ((1 << kLow) - 1);
    const int rest = line >> kLow;
    const int hi = rest & ((1 << kHiBits) - 1);
    const int row = rest >> kHiBits;
    const int base = (row << LOG2G) + lo + (hi << (kLow + kNB));
    float w[16];
#pragma unroll
    for (int i = 0; i < kN; ++i) w[i] = tile[padded(base + (i << kLow))];
    phase_stages<kKind, kNB>(w);
#pragma unroll
    for (int i = 0; i < kN; ++i) y_tile[base + (i << kLow)] = storage_bits<kKind>(w[i]);
  }
}

// The tensor is contiguous [rows, cols] with cols a multiple of the group, so its flat view is
// a sequence of whole groups: a tile is kFastTile consecutive elements (kFastTile / group
// groups), and the last tile holds the remaining whole groups. Each thread owns 16 consecutive
// elements of a tile (32 bytes). The input is prefetched kPipe - 1 tiles ahead with cp.async
// into a per-thread slot of a shared ring (a thread reads back only what it copied, so the ring
// needs no barrier), keeping 2 x 8 KB per CTA in flight while the current tile is rotated.
constexpr int kPipe = 3;

template <int kKind, int LOG2G>
__global__ void __launch_bounds__(kThreads, 5)
    hadamard_fast_kernel(const uint16_t* x, uint16_t* y, int64_t total) {
  constexpr int kPhases = (LOG2G + 3) / 4;
  __shared__ float tile[kPhases > 1 ? kFastTile + kFastTile / 16 : 1];
  __shared__ __align__(16) uint4 ring[kPipe][kThreads * 2];
  const int64_t tiles = (total + kFastTile - 1) / kFastTile;
  const int t = threadIdx.x;
  const int e0 = t * 16;  // element index within the tile (row-major groups)
  // copy this thread's 32 bytes of the j-th tile of this CTA into ring slot j % kPipe
  auto prefetch = [&](int64_t j) {
    const int64_t tix = blockIdx.x + j * gridDim.x;
    if (tix < tiles && tix * kFastTile + e0 < total) {
      const uint16_t* src = x + tix * kFastTile + e0;
      const uint32_t dst = smem_u32(&ring[j % kPipe][2 * t]);
      cp_async16(dst, src);
      cp_async16(dst + 16, src + 8);
    }
    cp_async_commit();  // empty groups keep the group count uniform
  };
#pragma unroll
  for (int j = 0; j < kPipe - 1; ++j) prefetch(j);
  int64_t j = 0;
  for (int64_t tix = blockIdx.x; tix < tiles; tix += gridDim.x, ++j) {
    prefetch(j + kPipe - 1);  // into the slot read in the previous iteration
    cp_async_wait<kPipe - 1>();
    const int64_t base = tix * kFastTile;
    const int count = static_cast<int>(std::min<int64_t>(kFastTile, total - base));  // whole groups
    const int nrows = count >> LOG2G;
    // phase 0: the thread's 16 contiguous elements, from its ring slot
    float v[16];
    const bool live = e0 < count;
    if (live) {
      const uint4 u0 = ring[j % kPipe][2 * t], u1 = ring[j % kPipe][2 * t + 1];
      const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if constexpr (kKind == kBF16) {
          v[2 * k] = __uint_as_float(w[k] << 16);
          v[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
        } else {
          __half2 h2;
          memcpy(&h2, &w[k], sizeof(h2));
          const float2 f = __half22float2(h2);
          v[2 * k] = f.x;
          v[2 * k + 1] = f.y;
        }
      }
      phase_stages<kKind, (LOG2G < 4 ? LOG2G : 4)>(v);
    }
    if constexpr (kPhases > 1) {
      if (live) {
#pragma unroll
        for (int i = 0; i < 16; ++i) tile[padded(e0 + i)] = v[i];
      }
      __syncthreads();
      if constexpr (kPhases > 2) {
        smem_phase<kKind, LOG2G, 1>(tile, nrows);
        smem_phase_store<kKind, LOG2G, 2>(tile, nrows, y + base);
      } else {
        smem_phase_store<kKind, LOG2G, 1>(tile, nrows, y + base);
      }
    } else if (live) {
      uint32_t w[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if constexpr (kKind == kBF16) {
          w[k] = (__float_as_uint(v[2 * k]) >> 16) | (__float_as_uint(v[2 * k + 1]) & 0xffff0000u);
        } else {
          const __half2 h2 = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
          memcpy(&w[k], &h2, sizeof(uint32_t));
        }
      }
      uint4* dst = reinterpret_cast<uint4*>(y + base + e0);
      dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
      dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
    if constexpr (kPhases > 1) __syncthreads();  // the next tile reuses the shared memory
  }
  cp_async_wait<0>();  // no copy outlives the CTA (the trailing groups are empty)
}

template <int kKind>
void launch_fast(const void* x, void* y, int64_t total, int log2g, unsigned grid, cudaStream_t s) {
  const uint16_t* xi = static_cast<const uint16_t*>(x);
  uint16_t* yi = static_cast<uint16_t*>(y);
  switch (log2g) {
    case 4: hadamard_fast_kernel<kKind, 4><<<grid, kThreads, 0, s>>>(xi, yi, total); break;
    case 5: hadamard_fast_kernel<kKind, 5><<<grid, kThreads, 0, s>>>(xi, yi, total); break;
    case 6: hadamard_fast_kernel<kKind, 6><<<grid, kThreads, 0, s>>>(xi, yi, total); break;
    case 7: hadamard_fast_kernel<kKind, 7><<<grid, kThreads, 0, s>>>(xi, yi, total); break;
    case 8: hadamard_fast_kernel<kKind, 8><<<grid, kThreads, 0, s>>>(xi, yi, total); break;
    case 9: hadamard_fast_kernel<kKind, 9><<<grid, kThreads, 0, s>>>(xi, yi, total); break;
    case 10: hadamard_fast_kernel<kKind, 10><<<grid, kThreads, 0, s>>>(xi, yi, total); break;
    case 11: hadamard_fast_kernel<kKind, 11><<<grid, kThreads, 0, s>>>(xi, yi, total); break;
    default: hadamard_fast_kernel<kKind, 12><<<grid, kThreads, 0, s>>>(xi, yi, total); break;
  }
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

}  // namespace
}  // namespace moss

using namespace moss;

extern "C" int moss_hadamard_rotate(const void* x, int dtype, int64_t rows, int64_t cols, int64_t group, void* y,
                                    moss_stream_t stream) {
  if (!is_float_kind(dtype)) return fail(MOSS_ERR_UNSUPPORTED, "unsupported dtype code %d", dtype);
  if (rows < 0 || cols < 0) return fail(MOSS_ERR_INVALID_ARGUMENT, "negative shape");
  if (group < 1 || (group & (group - 1)) != 0)
    return fail(MOSS_ERR_INVALID_ARGUMENT, "Hadamard group size must be a positive power of two (got %lld)",
                static_cast<long long>(group));
  if (cols % group != 0)
    return fail(MOSS_ERR_INVALID_ARGUMENT, "Input width must be divisible by Hadamard group size (%lld %% %lld)",
                static_cast<long long>(cols), static_cast<long long>(group));
  if (group > kMaxGroup)
    return fail(MOSS_ERR_UNSUPPORTED, "Hadamard group size %lld exceeds %lld", static_cast<long long>(group),
                static_cast<long long>(kMaxGroup));
  if (rows == 0 || cols == 0) return clear_ok();
  if (x == nullptr || y == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null tensor pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int esize = dtype == kF32 ? 4 : 2;
  if (group == 1) {
    if (x != y) MOSS_CUDA_TRY(cudaMemcpyAsync(y, x, static_cast<size_t>(rows * cols * esize), cudaMemcpyDeviceToDevice, s));
    return clear_ok();
  }
  const bool fast_ok = dtype != kF32 && group >= 16 && group <= kFastTile && cols % 8 == 0 &&
                       (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0;
  if (fast_ok) {
    int log2g = 0;
    while ((int64_t{1} << log2g) < group) ++log2g;
    const int64_t total = rows * cols;
    const int64_t tiles = (total + kFastTile - 1) / kFastTile;
    const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(tiles, 5LL * sm_count())));
    if (dtype == kBF16)
      launch_fast<kBF16>(x, y, total, log2g, grid, s);
    else
      launch_fast<kF16>(x, y, total, log2g, grid, s);
    MOSS_CUDA_TRY(cudaGetLastError());
    return clear_ok();
  }
  const int rows_per_tile = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(rows, kTileFloats / group)));
  const int64_t tiles = (rows + rows_per_tile - 1) / rows_per_tile * (cols / group);
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(tiles, 8LL * sm_count())));
  const size_t smem = static_cast<size_t>(rows_per_tile) * group * sizeof(float);
  hadamard_kernel<<<grid, kThreads, smem, s>>>(x, y, dtype, rows, cols, static_cast<int>(group), rows_per_tile);
  MOSS_CUDA_TRY(cudaGetLastError());
  return clear_ok();
}
