// Per-sequence conditioning of a packed token stream: adaLN modulation and gated residuals.
//
// A packed batch concatenates the tokens of several samples into one [rows, dim] stream with
// cumulative boundaries `offsets` [segments + 1]; each sample has its own modulation rows.
// The reference expands every condition to a [rows, dim] tensor with index_select and then
// runs separate elementwise ops (training/model.py:288-312, :752-771). Here one pass reads
// each token once, finds its segment from the offsets, and applies the condition row of that
// segment from cache:
//   modulate  y = round(round(x * round(1 + scale[s])) + shift[s])
//   gate      y = round(x + round(u * gate[s]))
// Every product and sum is rounded to the result dtype in the reference's order, with
// __fmul_rn/__fadd_rn so the compiler cannot contract them into an FMA - the outputs are
// bit-identical to the reference's eager ops. The backward passes also reduce the condition
// gradients per segment (f32 sums, block-reduced in shared memory, one atomic per column and
// segment per CTA).
//
// Tiling: a CTA covers 256 columns (32 lanes x 8 contiguous elements) of kRowsPerCta rows;
// its 8 warps take interleaved rows. All accesses are 16-byte vectors when the pointers and
// row strides allow, else element accesses with the same arithmetic.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "errors.cuh"

namespace moss {
namespace {

constexpr int kSegThreads = 256;
constexpr int kSegWarps = kSegThreads / 32;
constexpr int kColsPerCta = 256;
constexpr int kRowsPerCta = 64;

__host__ __device__ constexpr int promote_kind(int a, int b) { return a == b ? a : kF32; }

template <int K>
__device__ __forceinline__ float rnd(float v) {
  if constexpr (K == kBF16) return __bfloat162float(__float2bfloat16_rn(v));
  if constexpr (K == kF16) return __half2float(__float2half_rn(v));
  return v;
}

template <int K>
__device__ __forceinline__ float ld1(const void* p, int64_t i) {
  if constexpr (K == kBF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  if constexpr (K == kF16) return __half2float(static_cast<const __half*>(p)[i]);
  return static_cast<const float*>(p)[i];
}

template <int K>
__device__ __forceinline__ void st1(void* p, int64_t i, float v) {
  if constexpr (K == kBF16) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else if constexpr (K == kF16) static_cast<__half*>(p)[i] = __float2half_rn(v);
  else static_cast<float*>(p)[i] = v;
}

// 8 consecutive elements starting at element i (i % 8 == 0 on the vector path)
template <int K, bool kVec>
__device__ __forceinline__ void ld8(const void* p, int64_t i, int n, float (&f)[8]) {
  if constexpr (kVec) {
    if constexpr (K == kF32) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p) + i));
      const float4 b = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p) + i) + 1);
      f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
    } else {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p) + i));
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if constexpr (K == kBF16) {
          const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[j]));
          f[2 * j] = t.x;
          f[2 * j + 1] = t.y;
        } else {
          const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
          f[2 * j] = t.x;
          f[2 * j + 1] = t.y;
        }
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = j < n ? ld1<K>(p, i + j) : 0.f;
  }
}

template <int K, bool kVec>
__device__ __forceinline__ void st8(void* p, int64_t i, int n, const float (&f)[8]) {
  if constexpr (kVec) {
    if constexpr (K == kF32) {
      float4* q = reinterpret_cast<float4*>(static_cast<float*>(p) + i);
      q[0] = make_float4(f[0], f[1], f[2], f[3]);
      q[1] = make_float4(f[4], f[5], f[6], f[7]);
    } else {
      uint32_t w[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if constexpr (K == kBF16) {
          const __nv_bfloat162 t = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
          w[j] = *reinterpret_cast<const uint32_t*>(&t);
        } else {
          const __half2 t = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
          w[j] = *reinterpret_cast<const uint32_t*>(&t);
        }
      }
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p) + i) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (j < n) st1<K>(p, i + j, f[j]);
  }
}

// segment of `row`: the s with offsets[s] <= row < offsets[s + 1], clamped to [0, segments)
__device__ __forceinline__ int segment_of(const int64_t* __restrict__ offsets, int segments, int64_t row) {
  int lo = 0, hi = segments - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(offsets + mid) <= row)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

struct SegArgs {
  const void* x;       // tokens (modulate: normalised hidden; gate: residual stream)
  const void* u;       // gate: the branch output multiplied by the gate
  const void* dy;      // backward: gradient of the output
  const void* c0;      // modulate: scale; gate: gate
  const void* c1;      // modulate: shift
  int64_t c_stride;    // elements between consecutive segment rows of c0 / c1
  const int64_t* offsets;
  int segments;
  int64_t rows;
  int64_t dim;
  void* out;           // forward: y; backward: grad of x (modulate) or of u (gate)
  float* acc0;         // backward: f32 [segments, dim] sums (dscale or dgate), may be null
  float* acc1;         // backward: f32 [segments, dim] sums (dshift), may be null
};

template <int KX, int KC, bool kGate, bool kVec>
__global__ void __launch_bounds__(kSegThreads) segment_fwd_kernel(SegArgs a) {
  constexpr int KO = promote_kind(KX, KC);
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t col = static_cast<int64_t>(blockIdx.x) * kColsPerCta + lane * 8;
  if (col >= a.dim) return;
  const int n = static_cast<int>(a.dim - col < 8 ? a.dim - col : 8);
  const int64_t row0 = static_cast<int64_t>(blockIdx.y) * kRowsPerCta;
  const int64_t row_end = row0 + kRowsPerCta < a.rows ? row0 + kRowsPerCta : a.rows;
  int seg = -1;
  float c0[8], c1[8];
  for (int64_t row = row0 + warp; row < row_end; row += kSegWarps) {
    const int s = segment_of(a.offsets, a.segments, row);
    if (s != seg) {
      seg = s;
      ld8<KC, kVec>(a.c0, seg * a.c_stride + col, n, c0);
      if constexpr (!kGate) {
        ld8<KC, kVec>(a.c1, seg * a.c_stride + col, n, c1);
#pragma unroll
        for (int j = 0; j < 8; ++j) c0[j] = rnd<KC>(__fadd_rn(1.0f, c0[j]));
      }
    }
    float x[8], y[8];
    ld8<KX, kVec>(a.x, row * a.dim + col, n, x);
    if constexpr (kGate) {
      float u[8];
      ld8<KX, kVec>(a.u, row * a.dim + col, n, u);
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = rnd<KO>(__fadd_rn(x[j], rnd<KO>(__fmul_rn(u[j], c0[j]))));
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = rnd<KO>(__fadd_rn(rnd<KO>(__fmul_rn(x[j], c0[j])), c1[j]));
    }
    st8<KO, kVec>(a.out, row * a.dim + col, n, y);
  }
}

// Shared-memory column sums of one segment across the CTA's warps, then one atomic per column.
__device__ __forceinline__ void flush_segment(float (*red)[kColsPerCta], const float (&part)[8], int warp, int lane,
                                              float* acc, int64_t seg_base, int64_t col0, int64_t dim) {
#pragma unroll
  for (int j = 0; j < 8; ++j) red[warp][lane * 8 + j] = part[j];
  __syncthreads();
  const int c = threadIdx.x;  // kSegThreads == kColsPerCta
  float sum = 0.f;
#pragma unroll
  for (int w = 0; w < kSegWarps; ++w) sum += red[w][c];
  if (col0 + c < dim) atomicAdd(acc + seg_base + col0 + c, sum);
  __syncthreads();
}

template <int KX, int KC, bool kGate, bool kVec>
__global__ void __launch_bounds__(kSegThreads) segment_bwd_kernel(SegArgs a) {
  constexpr int KO = promote_kind(KX, KC);
  __shared__ float red[kSegWarps][kColsPerCta];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t col0 = static_cast<int64_t>(blockIdx.x) * kColsPerCta;
  const int64_t col = col0 + lane * 8;
  const bool active = col < a.dim;
  const int n = active ? static_cast<int>(a.dim - col < 8 ? a.dim - col : 8) : 0;
  const int64_t row0 = static_cast<int64_t>(blockIdx.y) * kRowsPerCta;
  const int64_t row_end = row0 + kRowsPerCta < a.rows ? row0 + kRowsPerCta : a.rows;
  const bool reduce = a.acc0 != nullptr || a.acc1 != nullptr;
  // the segments present in this CTA's rows, walked in order (usually one)
  int seg = segment_of(a.offsets, a.segments, row0);
  const int seg_last = segment_of(a.offsets, a.segments, row_end - 1);
  for (; seg <= seg_last; ++seg) {
    int64_t lo = __ldg(a.offsets + seg), hi = __ldg(a.offsets + seg + 1);
    if (seg == 0) lo = 0;
    if (seg == a.segments - 1) hi = a.rows;
    lo = lo > row0 ? lo : row0;
    hi = hi < row_end ? hi : row_end;
    float c0[8];
    if (active) {
      ld8<KC, kVec>(a.c0, seg * a.c_stride + col, n, c0);
      if constexpr (!kGate) {
#pragma unroll
        for (int j = 0; j < 8; ++j) c0[j] = rnd<KC>(__fadd_rn(1.0f, c0[j]));
      }
    }
    float p0[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float p1[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    // rows of this segment owned by this warp: the first row >= lo congruent to row0 + warp
    int64_t first = row0 + warp;
    if (first < lo) first += ((lo - first + kSegWarps - 1) / kSegWarps) * kSegWarps;
    for (int64_t row = first; active && row < hi; row += kSegWarps) {
      float dy[8], v[8], g[8];
      ld8<KO, kVec>(a.dy, row * a.dim + col, n, dy);
      ld8<KX, kVec>(kGate ? a.u : a.x, row * a.dim + col, n, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        g[j] = rnd<KX>(rnd<KO>(__fmul_rn(dy[j], c0[j])));
        p0[j] += rnd<KC>(rnd<KO>(__fmul_rn(dy[j], v[j])));
        if constexpr (!kGate) p1[j] += rnd<KC>(dy[j]);
      }
      st8<KX, kVec>(a.out, row * a.dim + col, n, g);
    }
    if (reduce) {  // uniform across the CTA
      if (a.acc0 != nullptr) flush_segment(red, p0, warp, lane, a.acc0, seg * a.dim, col0, a.dim);
      if (!kGate && a.acc1 != nullptr) flush_segment(red, p1, warp, lane, a.acc1, seg * a.dim, col0, a.dim);
    }
  }
}

bool aligned16(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <int KX, int KC, bool kGate, bool kBwd>
void launch_kinds(const SegArgs& a, bool vec, cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned>((a.dim + kColsPerCta - 1) / kColsPerCta),
                  static_cast<unsigned>((a.rows + kRowsPerCta - 1) / kRowsPerCta));
  if constexpr (kBwd) {
    if (vec)
      segment_bwd_kernel<KX, KC, kGate, true><<<grid, kSegThreads, 0, stream>>>(a);
    else
      segment_bwd_kernel<KX, KC, kGate, false><<<grid, kSegThreads, 0, stream>>>(a);
  } else {
    if (vec)
      segment_fwd_kernel<KX, KC, kGate, true><<<grid, kSegThreads, 0, stream>>>(a);
    else
      segment_fwd_kernel<KX, KC, kGate, false><<<grid, kSegThreads, 0, stream>>>(a);
  }
}

template <bool kGate, bool kBwd, int KX>
void launch_cond(const SegArgs& a, int kc, bool vec, cudaStream_t stream) {
  if (kc == kBF16) launch_kinds<KX, kBF16, kGate, kBwd>(a, vec, stream);
  else if (kc == kF16) launch_kinds<KX, kF16, kGate, kBwd>(a, vec, stream);
  else launch_kinds<KX, kF32, kGate, kBwd>(a, vec, stream);
}

template <bool kGate, bool kBwd>
int run(const SegArgs& a, int kx, int kc, moss_stream_t stream, const char* what) {
  if (!is_float_kind(kx) || !is_float_kind(kc)) return fail(MOSS_ERR_UNSUPPORTED, "%s: unsupported dtype code", what);
  if (a.rows < 0 || a.dim < 1 || a.segments < 1 || a.c_stride < a.dim)
    return fail(MOSS_ERR_INVALID_ARGUMENT, "%s: need rows >= 0, dim >= 1, segments >= 1, cond_stride >= dim", what);
  if (a.rows == 0) return clear_ok();
  if (a.rows > (int64_t{65535} * kRowsPerCta))
    return fail(MOSS_ERR_UNSUPPORTED, "%s: more than %lld rows", what, static_cast<long long>(65535LL * kRowsPerCta));
  if (a.offsets == nullptr || a.c0 == nullptr || a.out == nullptr || (!kGate && !kBwd && a.c1 == nullptr) ||
      (kBwd ? a.dy == nullptr : a.x == nullptr) || ((kGate || kBwd) && (kGate ? a.u : a.x) == nullptr))
    return fail(MOSS_ERR_INVALID_ARGUMENT, "%s: null pointer", what);
  const bool vec = a.dim % 8 == 0 && a.c_stride % 8 == 0 && aligned16(a.x) && aligned16(a.u) && aligned16(a.dy) &&
                   aligned16(a.c0) && aligned16(a.c1) && aligned16(a.out);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (kx == kBF16) launch_cond<kGate, kBwd, kBF16>(a, kc, vec, s);
  else if (kx == kF16) launch_cond<kGate, kBwd, kF16>(a, kc, vec, s);
  else launch_cond<kGate, kBwd, kF32>(a, kc, vec, s);
  return check_cuda(cudaGetLastError(), what) == MOSS_OK ? clear_ok() : MOSS_ERR_CUDA;
}

}  // namespace
}  // namespace moss

using moss::SegArgs;

extern "C" int moss_segment_modulate(const void* x, int x_dtype, int64_t rows, int64_t dim, const void* scale,
                                     const void* shift, int cond_dtype, int64_t cond_stride, const int64_t* offsets,
                                     int64_t segments, void* y, moss_stream_t stream) {
  SegArgs a{x, nullptr, nullptr, scale, shift, cond_stride, offsets, static_cast<int>(segments), rows, dim, y,
            nullptr, nullptr};
  if (segments > (1 << 30)) return moss::fail(MOSS_ERR_UNSUPPORTED, "too many segments");
  return moss::run<false, false>(a, x_dtype, cond_dtype, stream, "moss_segment_modulate");
}

extern "C" int moss_segment_modulate_bwd(const void* dy, const void* x, int x_dtype, int64_t rows, int64_t dim,
                                         const void* scale, int cond_dtype, int64_t cond_stride,
                                         const int64_t* offsets, int64_t segments, void* dx, float* dscale,
                                         float* dshift, moss_stream_t stream) {
  SegArgs a{x, nullptr, dy, scale, nullptr, cond_stride, offsets, static_cast<int>(segments), rows, dim, dx,
            dscale, dshift};
  if (segments > (1 << 30)) return moss::fail(MOSS_ERR_UNSUPPORTED, "too many segments");
  return moss::run<false, true>(a, x_dtype, cond_dtype, stream, "moss_segment_modulate_bwd");
}

extern "C" int moss_segment_gate(const void* x, const void* update, int x_dtype, int64_t rows, int64_t dim,
                                 const void* gate, int cond_dtype, int64_t cond_stride, const int64_t* offsets,
                                 int64_t segments, void* y, moss_stream_t stream) {
  SegArgs a{x, update, nullptr, gate, nullptr, cond_stride, offsets, static_cast<int>(segments), rows, dim, y,
            nullptr, nullptr};
  if (segments > (1 << 30)) return moss::fail(MOSS_ERR_UNSUPPORTED, "too many segments");
  return moss::run<true, false>(a, x_dtype, cond_dtype, stream, "moss_segment_gate");
}

extern "C" int moss_segment_gate_bwd(const void* dy, const void* update, int x_dtype, int64_t rows, int64_t dim,
                                     const void* gate, int cond_dtype, int64_t cond_stride, const int64_t* offsets,
                                     int64_t segments, void* dupdate, float* dgate, moss_stream_t stream) {
  SegArgs a{nullptr, update, dy, gate, nullptr, cond_stride, offsets, static_cast<int>(segments), rows, dim, dupdate,
            dgate, nullptr};
  if (segments > (1 << 30)) return moss::fail(MOSS_ERR_UNSUPPORTED, "too many segments");
  return moss::run<true, true>(a, x_dtype, cond_dtype, stream, "moss_segment_gate_bwd");
}
