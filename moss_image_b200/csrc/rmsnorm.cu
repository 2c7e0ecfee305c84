// RMSNorm over the last dimension with the reference's rounding points
// (training/model.py:154-172):
//   n = round_x(x * rsqrt(mean(x^2) + eps))      statistics in f32, one cast to x's dtype
//   y = round_y(n * w)                            y's dtype = promote(x, w)
// and its input gradient (the weight is frozen on this path):
//   dn = round_x(round_y(dy * w))
//   dx = round_x(r * dn - x * r^3 * sum(dn * x) / dim)        in f32, r saved per row
//
// Each thread moves 16-byte chunks of 8 elements and keeps up to a few of them in registers
// between the two passes. Rows of up to 128 chunks (1024 elements) belong to a group of L
// lanes (L = chunks / 4 rounded up to a power of two), so a warp holds several short rows -
// the per-head q/k norms (128 elements) put 8 rows in a warp, 4 chunks per lane - with the
// sums reduced by shuffles inside the group. Longer rows (3072) belong to a CTA of 128
// threads with a shared-memory reduction.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "errors.cuh"

namespace moss {
namespace {

constexpr int kNormThreads = 256;

__host__ __device__ constexpr int promote(int a, int b) { return a == b ? a : kF32; }

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

// Raw 16-byte chunk (8 elements of a 16-bit type, or two float4 for f32).
template <int K>
struct Chunk {
  uint4 a, b;  // b used by f32 only
};

template <int K>
__device__ __forceinline__ Chunk<K> ldc(const void* p, int64_t i) {
  Chunk<K> c;
  if constexpr (K == kF32) {
    const uint4* q = reinterpret_cast<const uint4*>(static_cast<const float*>(p) + i);
    c.a = __ldg(q);
    c.b = __ldg(q + 1);
  } else {
    c.a = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p) + i));
    c.b = make_uint4(0, 0, 0, 0);
  }
  return c;
}

// two packed 16-bit values (low half first) to f32, exactly
template <int K>
__device__ __forceinline__ void unpack2(uint32_t w, float& lo, float& hi) {
  if constexpr (K == kBF16) {
    lo = __uint_as_float(w << 16);
    hi = __uint_as_float(w & 0xffff0000u);
  } else {
    __half2 h;
    memcpy(&h, &w, sizeof(h));
    const float2 t = __half22float2(h);
    lo = t.x;
    hi = t.y;
  }
}

template <int K>
__device__ __forceinline__ void unpack(const Chunk<K>& c, float (&f)[8]) {
  if constexpr (K == kF32) {
    f[0] = __uint_as_float(c.a.x); f[1] = __uint_as_float(c.a.y);
    f[2] = __uint_as_float(c.a.z); f[3] = __uint_as_float(c.a.w);
    f[4] = __uint_as_float(c.b.x); f[5] = __uint_as_float(c.b.y);
    f[6] = __uint_as_float(c.b.z); f[7] = __uint_as_float(c.b.w);
  } else {
    const uint32_t w0 = c.a.x, w1 = c.a.y, w2 = c.a.z, w3 = c.a.w;
    unpack2<K>(w0, f[0], f[1]);
    unpack2<K>(w1, f[2], f[3]);
    unpack2<K>(w2, f[4], f[5]);
    unpack2<K>(w3, f[6], f[7]);
  }
}

// two f32 values rounded to the 16-bit type and packed (low half first)
template <int K>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  uint32_t w;
  if constexpr (K == kBF16) {
    const __nv_bfloat162 t = __floats2bfloat162_rn(lo, hi);
    memcpy(&w, &t, sizeof(w));
  } else {
    const __half2 t = __floats2half2_rn(lo, hi);
    memcpy(&w, &t, sizeof(w));
  }
  return w;
}

template <int K>
__device__ __forceinline__ void st8(void* p, int64_t i, const float (&f)[8]) {
  if constexpr (K == kF32) {
    float4* q = reinterpret_cast<float4*>(static_cast<float*>(p) + i);
    q[0] = make_float4(f[0], f[1], f[2], f[3]);
    q[1] = make_float4(f[4], f[5], f[6], f[7]);
  } else {
    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(p) + i) =
        make_uint4(pack2<K>(f[0], f[1]), pack2<K>(f[2], f[3]), pack2<K>(f[4], f[5]), pack2<K>(f[6], f[7]));
  }
}

template <int L>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int off = L / 2; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

struct NormArgs {
  const void* x;
  const void* w;
  const void* dy;
  const float* rstd_in;
  void* out;         // forward: y; backward: dx
  float* rstd_out;   // forward, optional
  int64_t rows;
  int64_t dim;
  float eps;
};

// ---------------------------------------------------------------- vector path (dim % 8 == 0)
// L lanes per row (32 / L rows per warp), C chunks per lane held in registers; chunks beyond
// C * L (rows longer than the register budget) are re-read in the second pass. The loops run
// per warp row so every lane takes part in the group shuffles; rows past the end only skip
// their loads and stores.
template <int KX, int KW>
__device__ __forceinline__ void norm_emit(const void* wp, void* out, int64_t base, int c, float r,
                                          const float (&f)[8]) {
  constexpr int KY = promote(KX, KW);
  float w[8], y[8];
  unpack<KW>(ldc<KW>(wp, c * 8), w);
#pragma unroll
  for (int j = 0; j < 8; ++j) y[j] = rnd<KY>(__fmul_rn(rnd<KX>(__fmul_rn(f[j], r)), w[j]));
  st8<KY>(out, base + c * 8, y);
}

// dn = round_x(round_y(dy * w)) for chunk c
template <int KX, int KW>
__device__ __forceinline__ void norm_dn(const void* dy, const void* wp, int64_t base, int c, float (&dn)[8]) {
  constexpr int KY = promote(KX, KW);
  float d[8], w[8];
  unpack<KY>(ldc<KY>(dy, base + c * 8), d);
  unpack<KW>(ldc<KW>(wp, c * 8), w);
#pragma unroll
  for (int j = 0; j < 8; ++j) dn[j] = rnd<KX>(rnd<KY>(__fmul_rn(d[j], w[j])));
}

template <int KX, int KW>
__device__ __forceinline__ void norm_emit_dx(const void* dy, const void* wp, void* out, int64_t base, int c, float r,
                                             float coef, const float (&x)[8]) {
  float dn[8], dx[8];
  norm_dn<KX, KW>(dy, wp, base, c, dn);
#pragma unroll
  for (int j = 0; j < 8; ++j) dx[j] = rnd<KX>(__fsub_rn(__fmul_rn(dn[j], r), __fmul_rn(x[j], coef)));
  st8<KX>(out, base + c * 8, dx);
}

template <int KX>
__device__ __forceinline__ float sum_squares(const float (&f)[8], float ss) {
#pragma unroll
  for (int j = 0; j < 8; ++j) ss = __fadd_rn(ss, __fmul_rn(f[j], f[j]));
  return ss;
}

// Rows of at most C * L chunks (every chunk of a row is held by its group). Each warp loads
// the next rows it owns while it reduces and writes the current ones, so its loads stay in
// flight across iterations.
template <int KX, int KW, int L, int C>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_fwd_kernel(NormArgs a) {
  constexpr int G = 32 / L;  // rows per warp
  const void* const w = a.w;
  void* const out = a.out;
  const int lane = threadIdx.x & (L - 1);
  const int g = (threadIdx.x & 31) / L;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kNormThreads + threadIdx.x) / 32;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kNormThreads / 32 * G;
  const int chunks = static_cast<int>(a.dim / 8);
  const float inv_dim = 1.0f / static_cast<float>(a.dim);
  Chunk<KX> next[C];
  int64_t first = warp * G;
#pragma unroll
  for (int i = 0; i < C; ++i) {
    const int c = lane + i * L;
    if (first + g < a.rows && c < chunks) next[i] = ldc<KX>(a.x, (first + g) * a.dim + c * 8);
  }
  for (; first < a.rows; first += stride) {
    const int64_t row = first + g;
    const bool live = row < a.rows;
    const int64_t base = row * a.dim;
    Chunk<KX> held[C];
#pragma unroll
    for (int i = 0; i < C; ++i) held[i] = next[i];
    const int64_t ahead = row + stride;
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int c = lane + i * L;
      if (ahead < a.rows && c < chunks) next[i] = ldc<KX>(a.x, ahead * a.dim + c * 8);
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int c = lane + i * L;
      if (live && c < chunks) {
        float f[8];
        unpack<KX>(held[i], f);
        ss = sum_squares<KX>(f, ss);
      }
    }
    ss = group_sum<L>(ss);
    if (!live) continue;
    const float r = rsqrtf(__fadd_rn(__fmul_rn(ss, inv_dim), a.eps));
    if (a.rstd_out != nullptr && lane == 0) a.rstd_out[row] = r;
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int c = lane + i * L;
      if (c < chunks) {
        float f[8];
        unpack<KX>(held[i], f);
        norm_emit<KX, KW>(w, out, base, c, r, f);
      }
    }
  }
}

// Holds x and dy between the passes. Unlike the forward it does not load the next rows ahead:
// holding both rows of both tensors took 97 registers (2 CTAs per SM), and without it the
// kernel uses 64 and is faster (221184 x 128: 49.1 -> 45.2 us).
template <int KX, int KW, int L, int C>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_bwd_kernel(NormArgs a) {
  constexpr int KY = promote(KX, KW);
  constexpr int G = 32 / L;
  const void* const wp = a.w;
  void* const out = a.out;
  const int lane = threadIdx.x & (L - 1);
  const int g = (threadIdx.x & 31) / L;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kNormThreads + threadIdx.x) / 32;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kNormThreads / 32 * G;
  const int chunks = static_cast<int>(a.dim / 8);
  const float inv_dim = 1.0f / static_cast<float>(a.dim);
  int64_t first = warp * G;
  for (; first < a.rows; first += stride) {
    const int64_t row = first + g;
    const bool live = row < a.rows;
    const int64_t base = row * a.dim;
    const float r = live ? __ldg(a.rstd_in + row) : 0.f;
    Chunk<KX> hx[C];
    Chunk<KY> hdy[C];
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int c = lane + i * L;
      if (live && c < chunks) {
        hx[i] = ldc<KX>(a.x, base + c * 8);
        hdy[i] = ldc<KY>(a.dy, base + c * 8);
      }
    }
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int c = lane + i * L;
      if (live && c < chunks) {
        float x[8], d[8], wv[8];
        unpack<KX>(hx[i], x);
        unpack<KY>(hdy[i], d);
        unpack<KW>(ldc<KW>(wp, c * 8), wv);
#pragma unroll
        for (int j = 0; j < 8; ++j) dot = __fadd_rn(dot, __fmul_rn(rnd<KX>(rnd<KY>(__fmul_rn(d[j], wv[j]))), x[j]));
      }
    }
    dot = group_sum<L>(dot);
    if (!live) continue;
    const float coef = __fmul_rn(__fmul_rn(__fmul_rn(r, r), r), __fmul_rn(dot, inv_dim));
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int c = lane + i * L;
      if (c < chunks) {
        float x[8], d[8], wv[8], dx[8];
        unpack<KX>(hx[i], x);
        unpack<KY>(hdy[i], d);
        unpack<KW>(ldc<KW>(wp, c * 8), wv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float dn = rnd<KX>(rnd<KY>(__fmul_rn(d[j], wv[j])));
          dx[j] = rnd<KX>(__fsub_rn(__fmul_rn(dn, r), __fmul_rn(x[j], coef)));
        }
        st8<KX>(out, base + c * 8, dx);
      }
    }
  }
}

// ---------------------------------------------------------------- long rows: one CTA per row
// kRowThreads threads share a row (C chunks each in registers, the rest re-read), the sums are
// reduced through shared memory, and many rows stay in flight per SM.
constexpr int kRowThreads = 128;

__device__ __forceinline__ float cta_sum(float v, float* red) {
  v = group_sum<32>(v);
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int w = 0; w < kRowThreads / 32; ++w) total += red[w];
  __syncthreads();  // red is reused by the next row
  return total;
}

template <int KX, int KW, int C>
__global__ void __launch_bounds__(kRowThreads) rmsnorm_row_fwd_kernel(NormArgs a) {
  __shared__ float red[kRowThreads / 32];
  const void* const w = a.w;
  void* const out = a.out;
  const int t = threadIdx.x;
  const int chunks = static_cast<int>(a.dim / 8);
  const float inv_dim = 1.0f / static_cast<float>(a.dim);
  // the CTA's next row is loaded while the current one is reduced and written
  Chunk<KX> next[C];
  int64_t row = blockIdx.x;
#pragma unroll
  for (int i = 0; i < C; ++i) {
    const int c = t + i * kRowThreads;
    if (row < a.rows && c < chunks) next[i] = ldc<KX>(a.x, row * a.dim + c * 8);
  }
  for (; row < a.rows; row += gridDim.x) {
    const int64_t base = row * a.dim;
    Chunk<KX> held[C];
#pragma unroll
    for (int i = 0; i < C; ++i) held[i] = next[i];
    const int64_t ahead = row + gridDim.x;
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int c = t + i * kRowThreads;
      if (ahead < a.rows && c < chunks) next[i] = ldc<KX>(a.x, ahead * a.dim + c * 8);
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int c = t + i * kRowThreads;
      if (c < chunks) {
        float f[8];
        unpack<KX>(held[i], f);
        ss = sum_squares<KX>(f, ss);
      }
    }
    for (int c = t + C * kRowThreads; c < chunks; c += kRowThreads) {
      float f[8];
      unpack<KX>(ldc<KX>(a.x, base + c * 8), f);
      ss = sum_squares<KX>(f, ss);
    }
    ss = cta_sum(ss, red);
    const float r = rsqrtf(__fadd_rn(__fmul_rn(ss, inv_dim), a.eps));
    if (a.rstd_out != nullptr && t == 0) a.rstd_out[row] = r;
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int c = t + i * kRowThreads;
      if (c < chunks) {
        float f[8];
        unpack<KX>(held[i], f);
        norm_emit<KX, KW>(w, out, base, c, r, f);
      }
    }
    for (int c = t + C * kRowThreads; c < chunks; c += kRowThreads) {
      float f[8];
      unpack<KX>(ldc<KX>(a.x, base + c * 8), f);
      norm_emit<KX, KW>(w, out, base, c, r, f);
    }
  }
}

// Holds x of its chunks between the passes and re-reads dy (an L2 hit) in the second. Holding
// dy and prefetching the next row as the forward does raised the registers to 80 and made
// 9216 x 3072 slower (45 -> 49 us).
template <int KX, int KW, int C>
__global__ void __launch_bounds__(kRowThreads) rmsnorm_row_bwd_kernel(NormArgs a) {
  __shared__ float red[kRowThreads / 32];
  const void* const w = a.w;
  const void* const dy = a.dy;
  void* const out = a.out;
  const int t = threadIdx.x;
  const int chunks = static_cast<int>(a.dim / 8);
  const float inv_dim = 1.0f / static_cast<float>(a.dim);
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const int64_t base = row * a.dim;
    const float r = __ldg(a.rstd_in + row);
    Chunk<KX> hx[C];
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int c = t + i * kRowThreads;
      if (c < chunks) {
        hx[i] = ldc<KX>(a.x, base + c * 8);
        float x[8], dn[8];
        unpack<KX>(hx[i], x);
        norm_dn<KX, KW>(dy, w, base, c, dn);
#pragma unroll
        for (int j = 0; j < 8; ++j) dot = __fadd_rn(dot, __fmul_rn(dn[j], x[j]));
      }
    }
    for (int c = t + C * kRowThreads; c < chunks; c += kRowThreads) {
      float x[8], dn[8];
      unpack<KX>(ldc<KX>(a.x, base + c * 8), x);
      norm_dn<KX, KW>(dy, w, base, c, dn);
#pragma unroll
      for (int j = 0; j < 8; ++j) dot = __fadd_rn(dot, __fmul_rn(dn[j], x[j]));
    }
    dot = cta_sum(dot, red);
    const float coef = __fmul_rn(__fmul_rn(__fmul_rn(r, r), r), __fmul_rn(dot, inv_dim));
#pragma unroll
    for (int i = 0; i < C; ++i) {
      const int c = t + i * kRowThreads;
      if (c < chunks) {
        float x[8];
        unpack<KX>(hx[i], x);
        norm_emit_dx<KX, KW>(dy, w, out, base, c, r, coef, x);
      }
    }
    for (int c = t + C * kRowThreads; c < chunks; c += kRowThreads) {
      float x[8];
      unpack<KX>(ldc<KX>(a.x, base + c * 8), x);
      norm_emit_dx<KX, KW>(dy, w, out, base, c, r, coef, x);
    }
  }
}

// ---------------------------------------------------------------- element path (any dim)
template <int KX, int KW>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_generic_kernel(NormArgs a, bool backward) {
  constexpr int KY = promote(KX, KW);
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kNormThreads + threadIdx.x) / 32;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * kNormThreads / 32;
  const float inv_dim = 1.0f / static_cast<float>(a.dim);
  for (int64_t row = warp; row < a.rows; row += warps) {
    const int64_t base = row * a.dim;
    if (!backward) {
      float ss = 0.f;
      for (int64_t k = lane; k < a.dim; k += 32) {
        const float f = ld1<KX>(a.x, base + k);
        ss = __fadd_rn(ss, __fmul_rn(f, f));
      }
      ss = group_sum<32>(ss);
      const float r = rsqrtf(__fadd_rn(__fmul_rn(ss, inv_dim), a.eps));
      if (a.rstd_out != nullptr && lane == 0) a.rstd_out[row] = r;
      for (int64_t k = lane; k < a.dim; k += 32)
        st1<KY>(a.out, base + k, rnd<KY>(__fmul_rn(rnd<KX>(__fmul_rn(ld1<KX>(a.x, base + k), r)), ld1<KW>(a.w, k))));
    } else {
      const float r = a.rstd_in[row];
      float dot = 0.f;
      for (int64_t k = lane; k < a.dim; k += 32) {
        const float dn = rnd<KX>(rnd<KY>(__fmul_rn(ld1<KY>(a.dy, base + k), ld1<KW>(a.w, k))));
        dot = __fadd_rn(dot, __fmul_rn(dn, ld1<KX>(a.x, base + k)));
      }
      dot = group_sum<32>(dot);
      const float coef = __fmul_rn(__fmul_rn(__fmul_rn(r, r), r), __fmul_rn(dot, inv_dim));
      for (int64_t k = lane; k < a.dim; k += 32) {
        const float dn = rnd<KX>(rnd<KY>(__fmul_rn(ld1<KY>(a.dy, base + k), ld1<KW>(a.w, k))));
        st1<KX>(a.out, base + k, rnd<KX>(__fsub_rn(__fmul_rn(dn, r), __fmul_rn(ld1<KX>(a.x, base + k), coef))));
      }
    }
  }
}

bool aligned16(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int grid_for(int64_t rows, int rows_per_cta) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = (rows + rows_per_cta - 1) / rows_per_cta;
  const int64_t cap = static_cast<int64_t>(sms) * 8;  // 8 CTAs of 256 threads per SM, grid-stride beyond
  return static_cast<int>(want < cap ? (want > 0 ? want : 1) : cap);
}

template <int KX, int KW, bool kBwd, int L>
void launch_group(const NormArgs& a, cudaStream_t s) {
  const int grid = grid_for(a.rows, kNormThreads / L);
  if constexpr (kBwd)
    rmsnorm_bwd_kernel<KX, KW, L, 4><<<grid, kNormThreads, 0, s>>>(a);
  else
    rmsnorm_fwd_kernel<KX, KW, L, 4><<<grid, kNormThreads, 0, s>>>(a);
}

template <int KX, int KW, bool kBwd, int C>
void launch_row(const NormArgs& a, cudaStream_t s) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if constexpr (kBwd) {
    const int grid = static_cast<int>(std::min<int64_t>(a.rows, static_cast<int64_t>(sms) * 16));
    rmsnorm_row_bwd_kernel<KX, KW, C><<<grid, kRowThreads, 0, s>>>(a);
  } else {
    // One wave of resident CTAs, each walking rows with its next row in flight.
    static int per_sm = 0;
    static std::once_flag once;
    std::call_once(once, [] {
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rmsnorm_row_fwd_kernel<KX, KW, C>, kRowThreads, 0) !=
              cudaSuccess ||
          per_sm < 1) {
        cudaGetLastError();
        per_sm = 8;
      }
    });
    const int grid = static_cast<int>(std::min<int64_t>(a.rows, static_cast<int64_t>(sms) * per_sm));
    rmsnorm_row_fwd_kernel<KX, KW, C><<<grid, kRowThreads, 0, s>>>(a);
  }
}

// Rows of up to 128 chunks: a group of L lanes per row with up to 4 chunks per lane, so each
// warp keeps 32 x 4 chunks (2 KB of bf16) of one or more rows in flight. Longer rows: one CTA
// of 128 threads per row.
template <int KX, int KW, bool kBwd>
void launch_kinds(const NormArgs& a, bool vec, cudaStream_t s) {
  if (!vec) {
    rmsnorm_generic_kernel<KX, KW><<<grid_for(a.rows, kNormThreads / 32), kNormThreads, 0, s>>>(a, kBwd);
    return;
  }
  const int64_t chunks = a.dim / 8;
  if (chunks <= 4) return launch_group<KX, KW, kBwd, 1>(a, s);
  if (chunks <= 8) return launch_group<KX, KW, kBwd, 2>(a, s);
  if (chunks <= 16) return launch_group<KX, KW, kBwd, 4>(a, s);
  if (chunks <= 32) return launch_group<KX, KW, kBwd, 8>(a, s);
  if (chunks <= 64) return launch_group<KX, KW, kBwd, 16>(a, s);
  if (chunks <= 128) return launch_group<KX, KW, kBwd, 32>(a, s);
  if (chunks <= 2 * kRowThreads) return launch_row<KX, KW, kBwd, 2>(a, s);
  if (chunks <= 3 * kRowThreads) return launch_row<KX, KW, kBwd, 3>(a, s);  // 3072-wide rows
  // Longer rows hold 4 chunks a thread and re-read the rest in the second pass (8 chunks plus
  // the forward's prefetched next row would take 123-168 registers a thread).
  launch_row<KX, KW, kBwd, 4>(a, s);
}

template <bool kBwd, int KX>
void launch_w(const NormArgs& a, int kw, bool vec, cudaStream_t s) {
  if (kw == kBF16) launch_kinds<KX, kBF16, kBwd>(a, vec, s);
  else if (kw == kF16) launch_kinds<KX, kF16, kBwd>(a, vec, s);
  else launch_kinds<KX, kF32, kBwd>(a, vec, s);
}

template <bool kBwd>
int run(const NormArgs& a, int kx, int kw, moss_stream_t stream, const char* what) {
  if (!is_float_kind(kx) || !is_float_kind(kw)) return fail(MOSS_ERR_UNSUPPORTED, "%s: unsupported dtype code", what);
  if (a.rows < 0 || a.dim < 1) return fail(MOSS_ERR_INVALID_ARGUMENT, "%s: need rows >= 0 and dim >= 1", what);
  if (a.rows == 0) return clear_ok();
  if (a.x == nullptr || a.w == nullptr || a.out == nullptr || (kBwd && (a.dy == nullptr || a.rstd_in == nullptr)))
    return fail(MOSS_ERR_INVALID_ARGUMENT, "%s: null pointer", what);
  const bool vec = a.dim % 8 == 0 && a.dim / 8 <= static_cast<int64_t>(1) << 30 && aligned16(a.x) && aligned16(a.w) &&
                   aligned16(a.dy) && aligned16(a.out);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (kx == kBF16) launch_w<kBwd, kBF16>(a, kw, vec, s);
  else if (kx == kF16) launch_w<kBwd, kF16>(a, kw, vec, s);
  else launch_w<kBwd, kF32>(a, kw, vec, s);
  return check_cuda(cudaGetLastError(), what) == MOSS_OK ? clear_ok() : MOSS_ERR_CUDA;
}

}  // namespace
}  // namespace moss

extern "C" int moss_rmsnorm_fwd(const void* x, int x_dtype, int64_t rows, int64_t dim, const void* weight,
                                int w_dtype, float eps, void* y, float* rstd, moss_stream_t stream) {
  moss::NormArgs a{x, weight, nullptr, nullptr, y, rstd, rows, dim, eps};
  return moss::run<false>(a, x_dtype, w_dtype, stream, "moss_rmsnorm_fwd");
}

extern "C" int moss_rmsnorm_bwd(const void* dy, const void* x, int x_dtype, int64_t rows, int64_t dim,
                                const void* weight, int w_dtype, const float* rstd, void* dx, moss_stream_t stream) {
  moss::NormArgs a{x, weight, dy, rstd, dx, nullptr, rows, dim, 0.0f};
  return moss::run<true>(a, x_dtype, w_dtype, stream, "moss_rmsnorm_bwd");
}
