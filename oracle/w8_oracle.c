/*
 * CPU restatement of the MOSS-Image int8 hot path - TEST INFRASTRUCTURE ONLY.
 *
 * This file is the parity checker for libmoss_w8.so. Only the tests, the smoke check and
 * the CPU-baseline leg of the benchmark load it; no product code path calls it.
 * Each function follows the reference line it cites (paths relative to the MOSS-Image
 * repository). Floating-point rounding is spelled out (round-to-nearest-even helpers), so
 * the results do not depend on the host compiler's default conversions.
 */
#include <math.h>
#include <stddef.h>
#include <stdlib.h>
#include <stdint.h>
#include <string.h>

#define KIND_F16 0
#define KIND_BF16 1
#define KIND_F32 2

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* f32 -> bf16 bits, round to nearest even (NaN kept quiet). */
uint16_t oracle_f32_to_bf16(float f) {
  uint32_t u = f2u(f);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
float oracle_bf16_to_f32(uint16_t h) { return u2f(((uint32_t)h) << 16); }

uint16_t oracle_f32_to_f16(float f) {
  _Float16 h = (_Float16)f; /* IEEE conversion: round to nearest even */
  uint16_t b;
  memcpy(&b, &h, 2);
  return b;
}
float oracle_f16_to_f32(uint16_t b) {
  _Float16 h;
  memcpy(&h, &b, 2);
  return (float)h;
}

/* Round an f32 to the given kind and back. */
float oracle_round(float x, int kind) {
  if (kind == KIND_BF16) return oracle_bf16_to_f32(oracle_f32_to_bf16(x));
  if (kind == KIND_F16) return oracle_f16_to_f32(oracle_f32_to_f16(x));
  return x;
}

/*
 * Per-output-channel symmetric quantiser.
 * training/quantization.py:87  weight = linear.weight.detach().float()
 * training/quantization.py:88  scale = weight.abs().amax(dim=1) / 127
 * training/quantization.py:89  scale = where(scale == 0, 1, scale)
 * training/quantization.py:90  (weight / scale[:, None]).round().clamp(-127, 127).to(int8)
 * round() is half-to-even (rintf under the default rounding mode); all divisions are
 * correctly rounded f32 divisions. Returns 1 if a non-finite weight was seen
 * (training/quantization.py:82-83 rejects those), else 0.
 */
int oracle_quantize(const float* w, int64_t n, int64_t k, int8_t* q, float* scale) {
  int nonfinite = 0;
  for (int64_t r = 0; r < n; ++r) {
    const float* row = w + r * k;
    float amax = 0.0f;
    for (int64_t c = 0; c < k; ++c) {
      float v = row[c];
      if (!isfinite(v)) nonfinite = 1;
      float a = fabsf(v);
      if (a > amax) amax = a;
    }
    volatile float s = amax / 127.0f;
    float sv = s;
    if (sv == 0.0f) sv = 1.0f;
    scale[r] = sv;
    for (int64_t c = 0; c < k; ++c) {
      volatile float d = row[c] / sv;
      float t = rintf(d);
      if (t > 127.0f) t = 127.0f;
      if (t < -127.0f) t = -127.0f;
      q[r * k + c] = (int8_t)t;
    }
  }
  return nonfinite;
}

/*
 * Decoded weight element, training/quantization.py:23-24 (eager) and
 * training/quant_kernels.py:138-149 (tile decode):
 *   dec_w = round_w(float(q) * round_w(s)); the GEMM then consumes round_v(dec_w).
 */
float oracle_decode(int8_t q, float s, int w_kind, int v_kind) {
  float dw = oracle_round((float)q * oracle_round(s, w_kind), w_kind);
  return oracle_round(dw, v_kind);
}

/* out[n,k] = dec_w(q, s) as f32 values (no compute-dtype rounding). */
void oracle_dequantize(const int8_t* q, const float* s, int64_t n, int64_t k, int w_kind, float* out) {
  for (int64_t r = 0; r < n; ++r) {
    float sw = oracle_round(s[r], w_kind);
    for (int64_t c = 0; c < k; ++c) out[r * k + c] = oracle_round((float)q[r * k + c] * sw, w_kind);
  }
}

/*
 * Forward, training/quant_kernels.py:125-162 / training/quantization.py:43:
 *   y[m,n] = sum_k round_v(x[m,k]) * dec(q[n,k]) + round_v(bias[n])
 *            (+ lora_scale * sum_j xa[m,j] * b[n,j])
 * accumulated in double; written unrounded (y_acc) so tests can round or compare either way.
 * x: f32 values already in the compute dtype; bias may be NULL; xa/b may be NULL.
 */
void oracle_gemm_fwd(const float* x, int64_t m, int64_t k, const int8_t* q, const float* s, int64_t n,
                     int w_kind, int v_kind, const float* bias, const float* xa, const float* b, int64_t r,
                     float lora_scale, double* y_acc) {
  float* dec = (float*)malloc(sizeof(float) * (size_t)(n * k > 0 ? n * k : 1));
  for (int64_t j = 0; j < n; ++j)
    for (int64_t c = 0; c < k; ++c) dec[j * k + c] = oracle_decode(q[j * k + c], s[j], w_kind, v_kind);
  for (int64_t i = 0; i < m; ++i) {
    const float* xr = x + i * k;
    for (int64_t j = 0; j < n; ++j) {
      const float* dr = dec + j * k;
      double acc = 0.0;
      for (int64_t c = 0; c < k; ++c) acc += (double)xr[c] * (double)dr[c];
      if (xa != NULL) {
        double l = 0.0;
        for (int64_t t = 0; t < r; ++t) l += (double)xa[i * r + t] * (double)b[j * r + t];
        acc += (double)lora_scale * l;
      }
      y_acc[i * n + j] = acc + (bias ? (double)oracle_round(bias[j], v_kind) : 0.0);
    }
  }
  free(dec);
}

/*
 * Input gradient, training/quant_kernels.py:193-218 / training/quantization.py:61-64:
 *   dx[m,k] = sum_n dy[m,n] * dec(q[n,k]) (+ lora_scale * sum_j dyb[m,j] * a[j,k])
 */
void oracle_gemm_dx(const float* dy, int64_t m, int64_t n, const int8_t* q, const float* s, int64_t k,
                    int w_kind, int v_kind, const float* dyb, const float* a, int64_t r, float lora_scale,
                    double* dx_acc) {
  double* row = (double*)malloc(sizeof(double) * (size_t)(k > 0 ? k : 1));
  float* dec = (float*)malloc(sizeof(float) * (size_t)(n * k > 0 ? n * k : 1));
  for (int64_t j = 0; j < n; ++j)
    for (int64_t c = 0; c < k; ++c) dec[j * k + c] = oracle_decode(q[j * k + c], s[j], w_kind, v_kind);
  for (int64_t i = 0; i < m; ++i) {
    for (int64_t c = 0; c < k; ++c) row[c] = 0.0;
    for (int64_t j = 0; j < n; ++j) {
      const double g = (double)dy[i * n + j];
      const float* dr = dec + j * k;
      for (int64_t c = 0; c < k; ++c) row[c] += g * (double)dr[c];
    }
    if (dyb != NULL) {
      for (int64_t t = 0; t < r; ++t) {
        const double g = (double)lora_scale * (double)dyb[i * r + t];
        for (int64_t c = 0; c < k; ++c) row[c] += g * (double)a[t * k + c];
      }
    }
    for (int64_t c = 0; c < k; ++c) dx_acc[i * k + c] = row[c];
  }
  free(dec);
  free(row);
}

/*
 * Payload view of a saved tensor, training/activation_offload.py:32-61.
 * Writes the payload shape; returns 0 if the tensor can be offloaded, 1 if it must stay
 * resident (negative stride or overlapping elements).
 */
int oracle_offload_view(int ndim, const int64_t* shape, const int64_t* stride, int64_t* payload_shape) {
  for (int d = 0; d < ndim; ++d) {
    if (stride[d] < 0) return 1;
    payload_shape[d] = (stride[d] == 0 && shape[d] > 1) ? 1 : shape[d];
  }
  /* sort (stride, size) pairs of dims with size > 1 by stride, then size */
  int64_t st[16], sz[16];
  int cnt = 0;
  for (int d = 0; d < ndim && cnt < 16; ++d) {
    if (payload_shape[d] > 1) {
      st[cnt] = stride[d];
      sz[cnt] = payload_shape[d];
      ++cnt;
    }
  }
  for (int i = 1; i < cnt; ++i) {
    int64_t a = st[i], b = sz[i];
    int j = i - 1;
    while (j >= 0 && (st[j] > a || (st[j] == a && sz[j] > b))) {
      st[j + 1] = st[j];
      sz[j + 1] = sz[j];
      --j;
    }
    st[j + 1] = a;
    sz[j + 1] = b;
  }
  int64_t extent = 1;
  for (int i = 0; i < cnt; ++i) {
    if (st[i] < extent) return 1;
    extent += (sz[i] - 1) * st[i];
  }
  return 0;
}

/* Dense row-major gather of a strided view (element size esize bytes): the payload bytes
 * that pack() copies to the host (training/activation_offload.py:119-124). */
void oracle_gather(const uint8_t* src, int64_t esize, int ndim, const int64_t* shape, const int64_t* stride,
                   uint8_t* dst) {
  int64_t total = 1;
  for (int d = 0; d < ndim; ++d) total *= shape[d];
  for (int64_t i = 0; i < total; ++i) {
    int64_t rem = i, off = 0;
    for (int d = ndim - 1; d >= 0; --d) {
      int64_t idx = rem % shape[d];
      rem /= shape[d];
      off += idx * stride[d];
    }
    memcpy(dst + i * esize, src + off * esize, (size_t)esize);
  }
}

/*
 * Grouped normalised Hadamard rotation (ConvRot), as the reference's staged transform
 * computes it (training/quant_kernels.py:231-277 for one stage, :376-426 for the stage
 * order): radix-4 stages at strides 1, 4, 16, ... while 4 * stride <= group, then one radix-2
 * stage if log2(group) is odd. Each stage reads the previous stage's values, computes in f32
 *   radix 4: total = ((a + b) + c) + d; out[digit] = (total - 2 * {d, c, b, a}[digit]) * 0.5
 *   radix 2: out = (a + b) * 0.70710678f, (a - b) * 0.70710678f
 * and rounds to `kind` (the reference stores every stage in the tensor's dtype).
 * In place is allowed (y == x).
 */
void oracle_hadamard(const float* x, int64_t rows, int64_t cols, int64_t group, int kind, float* y) {
  if (y != x) memcpy(y, x, (size_t)(rows * cols) * sizeof(float));
  if (group <= 1) return;
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t g0 = 0; g0 < cols; g0 += group) {
      float* v = y + r * cols + g0;
      int64_t stride = 1;
      while (stride * 4 <= group) {
        for (int64_t base = 0; base < group; base += 4 * stride) {
          for (int64_t p = 0; p < stride; ++p) {
            const float a = v[base + p], b = v[base + p + stride];
            const float c = v[base + p + 2 * stride], d = v[base + p + 3 * stride];
            const float total = ((a + b) + c) + d;
            v[base + p] = oracle_round((total - 2.0f * d) * 0.5f, kind);
            v[base + p + stride] = oracle_round((total - 2.0f * c) * 0.5f, kind);
            v[base + p + 2 * stride] = oracle_round((total - 2.0f * b) * 0.5f, kind);
            v[base + p + 3 * stride] = oracle_round((total - 2.0f * a) * 0.5f, kind);
          }
        }
        stride *= 4;
      }
      if (stride < group) {
        const float h = 0.7071067811865476f;
        for (int64_t base = 0; base < group; base += 2 * stride) {
          for (int64_t p = 0; p < stride; ++p) {
            const float a = v[base + p], b = v[base + p + stride];
            v[base + p] = oracle_round((a + b) * h, kind);
            v[base + p + stride] = oracle_round((a - b) * h, kind);
          }
        }
      }
    }
  }
}
