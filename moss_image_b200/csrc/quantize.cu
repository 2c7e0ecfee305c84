// Per-output-channel symmetric int8 quantiser and decoder.
//
// Quantiser (training/quantization.py:87-91): one warp per output row.
//   pass 1: absmax over the row in f32 (exact), finiteness check;
//   s = amax / 127 with IEEE round-to-nearest division (never a reciprocal multiply);
//   s == 0 -> 1;
//   pass 2: q = clamp(rint(w / s), -127, 127) with IEEE division and round-half-even.
// Every operation is correctly rounded, so codes and scales are bit-identical to the
// reference's torch CPU arithmetic.
#include "common.cuh"
#include "errors.cuh"

namespace moss {

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const T* __restrict__ w, int64_t n, int64_t k,
                                                            int8_t* __restrict__ q,
                                                            float* __restrict__ scale, int* status) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= n) return;
  const T* wr = w + row * k;
  float amax = 0.f;
  bool finite = true;
  for (int64_t i = lane; i < k; i += 32) {
    const float v = to_f32<T>(wr[i]);
    finite = finite && isfinite(v);
    amax = fmaxf(amax, fabsf(v));
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  const bool all_finite = __all_sync(0xffffffffu, finite);
  float s = __fdiv_rn(amax, 127.0f);
  if (s == 0.0f) s = 1.0f;
  if (lane == 0) {
    scale[row] = s;
    if (!all_finite) report_status(status, MOSS_STATUS_NONFINITE_WEIGHT);
  }
  int8_t* qr = q + row * k;
  for (int64_t i = lane; i < k; i += 32) {
    float r = rintf(__fdiv_rn(to_f32<T>(wr[i]), s));
    r = fminf(fmaxf(r, -127.0f), 127.0f);
    qr[i] = static_cast<int8_t>(static_cast<int>(r));
  }
}

// out[n,k] = round_w(q * round_w(s)) in the requested float kind (training/quantization.py:23-24).
template <typename T>
__global__ void dequantize_kernel(const int8_t* __restrict__ q, const float* __restrict__ scale, int64_t n,
                                  int64_t k, T* __restrict__ out, int kind) {
  const int64_t total = n * k;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / k;
    const float s = round_to_kind(scale[row], kind);
    const float v = round_to_kind(static_cast<float>(q[i]) * s, kind);
    store_from_float(out, kind, i, v);
  }
}

}  // namespace moss

using namespace moss;

extern "C" int moss_w8_quantize(const void* w, int w_dtype, int64_t n, int64_t k, int8_t* q, float* scale,
                                int* status, moss_stream_t stream) {
  if (n < 0 || k < 0) return fail(MOSS_ERR_INVALID_ARGUMENT, "negative weight shape (%lld, %lld)",
                                  (long long)n, (long long)k);
  if (!is_float_kind(w_dtype)) return fail(MOSS_ERR_UNSUPPORTED, "unsupported weight dtype code %d", w_dtype);
  if (n == 0) return clear_ok();
  if (w == nullptr || q == nullptr || scale == nullptr)
    return fail(MOSS_ERR_INVALID_ARGUMENT, "null pointer passed to moss_w8_quantize");
  const int warps = 8;
  const unsigned grid = static_cast<unsigned>((n + warps - 1) / warps);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (w_dtype == MOSS_DTYPE_F32)
    quantize_rows_kernel<float><<<grid, warps * 32, 0, s>>>(static_cast<const float*>(w), n, k, q, scale, status);
  else if (w_dtype == MOSS_DTYPE_BF16)
    quantize_rows_kernel<__nv_bfloat16>
        <<<grid, warps * 32, 0, s>>>(static_cast<const __nv_bfloat16*>(w), n, k, q, scale, status);
  else
    quantize_rows_kernel<__half><<<grid, warps * 32, 0, s>>>(static_cast<const __half*>(w), n, k, q, scale, status);
  MOSS_CUDA_TRY(cudaGetLastError());
  return clear_ok();
}

extern "C" int moss_w8_dequantize(const int8_t* q, const float* scale, int64_t n, int64_t k, int out_dtype,
                                  void* out, moss_stream_t stream) {
  if (n < 0 || k < 0) return fail(MOSS_ERR_INVALID_ARGUMENT, "negative weight shape");
  if (!is_float_kind(out_dtype)) return fail(MOSS_ERR_UNSUPPORTED, "unsupported dtype code %d", out_dtype);
  if (n == 0 || k == 0) return clear_ok();
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t total = n * k;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 148 * 32));
  if (out_dtype == MOSS_DTYPE_F32)
    dequantize_kernel<float><<<grid, 256, 0, s>>>(q, scale, n, k, static_cast<float*>(out), out_dtype);
  else if (out_dtype == MOSS_DTYPE_BF16)
    dequantize_kernel<__nv_bfloat16>
        <<<grid, 256, 0, s>>>(q, scale, n, k, static_cast<__nv_bfloat16*>(out), out_dtype);
  else
    dequantize_kernel<__half><<<grid, 256, 0, s>>>(q, scale, n, k, static_cast<__half*>(out), out_dtype);
  MOSS_CUDA_TRY(cudaGetLastError());
  return clear_ok();
}
