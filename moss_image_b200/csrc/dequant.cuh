// int8 -> 16-bit operand decode shared by the GEMM kernels, plus small shared-memory helpers.
//
// Decode rounding follows training/quant_kernels.py:138-149 (and the eager
// training/quantization.py:23-24): dec = round_v(round_w(q * round_w(s))), with v the compute
// dtype and w the module (weight) dtype.
#pragma once

#include "common.cuh"

namespace moss {
namespace gemm {

// int8 -> 16-bit decode of one 32-bit word (4 codes) into two packed pairs.
//
// bf16: for a code q with raw byte b, A = bf16 bits 0x4300 | (b & 0x7F) = 128 + (b & 127) and
// C = 0x4300 | (b & 0x80) = 128 or 256. A - C = q exactly (two's complement), then one
// round-to-nearest bf16 multiply by bf16(s) gives bf16(q * bf16(s)) exactly as the reference.
__device__ __forceinline__ void dequant_word_bf16(uint32_t w, __nv_bfloat162 s2, uint32_t& lo, uint32_t& hi) {
  const uint32_t t01 = prmt(w, 0x43u, 0x4140u);  // 0x43 b1 0x43 b0
  const uint32_t t23 = prmt(w, 0x43u, 0x4342u);
  const uint32_t a01 = t01 & 0xFF7FFF7Fu, c01 = t01 & 0xFF80FF80u;
  const uint32_t a23 = t23 & 0xFF7FFF7Fu, c23 = t23 & 0xFF80FF80u;
  __nv_bfloat162 x01 = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&a01),
                               *reinterpret_cast<const __nv_bfloat162*>(&c01));
  __nv_bfloat162 x23 = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&a23),
                               *reinterpret_cast<const __nv_bfloat162*>(&c23));
  x01 = __hmul2(x01, s2);
  x23 = __hmul2(x23, s2);
  lo = *reinterpret_cast<uint32_t*>(&x01);
  hi = *reinterpret_cast<uint32_t*>(&x23);
}

// f16: 0x6400 | (b ^ 0x80) is the half 1024 + q + 128 exactly; subtracting 1152 gives q.
__device__ __forceinline__ void dequant_word_f16(uint32_t w, __half2 s2, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  const uint32_t t01 = prmt(u, 0x64u, 0x4140u);
  const uint32_t t23 = prmt(u, 0x64u, 0x4342u);
  const __half2 magic = __half2half2(__ushort_as_half(0x6480));  // 1152
  __half2 x01 = __hsub2(*reinterpret_cast<const __half2*>(&t01), magic);
  __half2 x23 = __hsub2(*reinterpret_cast<const __half2*>(&t23), magic);
  x01 = __hmul2(x01, s2);
  x23 = __hmul2(x23, s2);
  lo = *reinterpret_cast<uint32_t*>(&x01);
  hi = *reinterpret_cast<uint32_t*>(&x23);
}

__device__ __forceinline__ uint32_t pack2(float a, float b, int v_kind) {
  if (v_kind == kBF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Two f32 values -> one packed pair of the 16-bit compute kind, each rounded to nearest even
// by a single packed conversion. (A scalar round-trip through the 16-bit type per element is
// several times more expensive in the epilogue and rounds identically.)
template <int kV>
__device__ __forceinline__ uint32_t pack2_kind(float a, float b) {
  if constexpr (kV == kBF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// Bias of 32 consecutive output columns as f32 values rounded to the compute kind (the
// reference adds round_v(bias) to the f32 accumulator, training/quant_kernels.py:160-163).
// A 16-bit bias of the compute kind is exact in f32 and is read as packed words.
template <int kV>
__device__ __forceinline__ void load_bias32(const void* bias, int bias_kind, int col0, int ncols, float (&b)[32]) {
  const uint16_t* b16 = static_cast<const uint16_t*>(bias) + col0;
  if (bias_kind == kV && col0 + 32 <= ncols && (reinterpret_cast<uintptr_t>(b16) & 15) == 0) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(b16) + i);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if constexpr (kV == kBF16) {
          b[8 * i + 2 * k] = __uint_as_float(w[k] << 16);
          b[8 * i + 2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
        } else {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
          b[8 * i + 2 * k] = f.x;
          b[8 * i + 2 * k + 1] = f.y;
        }
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      b[j] = col0 + j < ncols ? round_to_kind(load_as_float(bias, bias_kind, col0 + j), kV) : 0.0f;
  }
}

// 16 f32 values times s -> two 16-byte chunks of the 16-bit operand (LoRA factor blocks).
__device__ __forceinline__ void pack16_scaled(const float (&f)[16], float s, int v_kind, uint4& o0, uint4& o1) {
  o0 = make_uint4(pack2(f[0] * s, f[1] * s, v_kind), pack2(f[2] * s, f[3] * s, v_kind),
                  pack2(f[4] * s, f[5] * s, v_kind), pack2(f[6] * s, f[7] * s, v_kind));
  o1 = make_uint4(pack2(f[8] * s, f[9] * s, v_kind), pack2(f[10] * s, f[11] * s, v_kind),
                  pack2(f[12] * s, f[13] * s, v_kind), pack2(f[14] * s, f[15] * s, v_kind));
}

// Load 16 consecutive values of a float-kind row as f32, zero past `ncols` (LoRA factors).
__device__ __forceinline__ void load16_f32(const void* base, int kind, int64_t row_off, int col0, int ncols,
                                           float (&v)[16]) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int c = col0 + i;
    v[i] = (c < ncols) ? load_as_float(base, kind, row_off + c) : 0.0f;
  }
}

// Generic decode (weight dtype differs from the compute dtype): f32 arithmetic.
__device__ __forceinline__ void dequant_word_generic(uint32_t w, float s_w, int w_kind, int v_kind,
                                                     uint32_t& lo, uint32_t& hi) {
  float d[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float q = static_cast<float>(static_cast<int8_t>((w >> (8 * i)) & 0xFF));
    d[i] = round_to_kind(q * s_w, w_kind);
  }
  lo = pack2(d[0], d[1], v_kind);
  hi = pack2(d[2], d[3], v_kind);
}

// Per-row decode context (scale in the right representation for each path).
template <int kV, bool kFast>
struct Dec {
  uint32_t s2;   // packed pair of round_v(s) for the fast paths
  float s_w;     // round_w(s) for the generic path
  __device__ __forceinline__ void set(float s, int w_kind) {
    if constexpr (kFast) {
      if constexpr (kV == kBF16) {
        __nv_bfloat162 h = __bfloat162bfloat162(__float2bfloat16_rn(s));
        s2 = *reinterpret_cast<uint32_t*>(&h);
      } else {
        __half2 h = __half2half2(__float2half_rn(s));
        s2 = *reinterpret_cast<uint32_t*>(&h);
      }
    } else {
      s_w = round_to_kind(s, w_kind);
    }
  }
  __device__ __forceinline__ void word(uint32_t w, int w_kind, uint32_t& lo, uint32_t& hi) const {
    if constexpr (kFast) {
      if constexpr (kV == kBF16) {
        dequant_word_bf16(w, *reinterpret_cast<const __nv_bfloat162*>(&s2), lo, hi);
      } else {
        dequant_word_f16(w, *reinterpret_cast<const __half2*>(&s2), lo, hi);
      }
    } else {
      dequant_word_generic(w, s_w, w_kind, kV, lo, hi);
    }
  }
  // 8 codes -> 16 bytes of 16-bit operand
  __device__ __forceinline__ uint4 chunk8(uint2 q, int w_kind) const {
    uint4 o;
    word(q.x, w_kind, o.x, o.y);
    word(q.y, w_kind, o.z, o.w);
    return o;
  }
  // 16 codes -> 32 bytes of 16-bit operand
  __device__ __forceinline__ void chunk(uint4 q, int w_kind, uint4& o0, uint4& o1) const {
    word(q.x, w_kind, o0.x, o0.y);
    word(q.y, w_kind, o0.z, o0.w);
    word(q.z, w_kind, o1.x, o1.y);
    word(q.w, w_kind, o1.z, o1.w);
  }
};

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr) : "memory");
  return v;
}
// 8 consecutive values of a float-kind row as f32 (zero past `ncols`), times s, packed.
__device__ __forceinline__ uint4 load8_scaled(const void* base, int kind, int64_t row_off, int col0, int ncols, float s,
                                              int v_kind) {
  float f[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = col0 + i;
    f[i] = (c < ncols) ? load_as_float(base, kind, row_off + c) * s : 0.0f;
  }
  return make_uint4(pack2(f[0], f[1], v_kind), pack2(f[2], f[3], v_kind), pack2(f[4], f[5], v_kind),
                    pack2(f[6], f[7], v_kind));
}
// 256-bit global store (one full 32-byte sector; address 32-byte aligned).
__device__ __forceinline__ void stg256(void* p, const uint32_t (&v)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(v[0]), "r"(v[1]), "r"(v[2]),
               "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}


}  // namespace gemm
}  // namespace moss
