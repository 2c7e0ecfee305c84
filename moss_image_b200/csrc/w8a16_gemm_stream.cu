// Few-row weight-streaming variant of the weight-only int8 GEMM for sm_100a (M <= 16 rows).
//
// With a handful of activation rows (the per-block adaLN modulation rows, single samples,
// decode-like calls) every int8 weight byte is used at most 16 times, so the GEMM is a read of
// the weight at HBM speed plus its decode. This kernel keeps no shared-memory pipeline at all:
// every lane streams its own 16-byte slices of the weight with non-allocating global loads,
// several slabs ahead, decodes them in registers with the shared exact decode (dequant.cuh)
// and feeds them to warp-level m16n8k16 MMAs (f32 accumulation) whose other operand is the
// handful of activation rows, read through L1. The tensor work is tiny (at most two n8 tiles);
// what matters is that enough weight bytes are in flight per SM, which the register-resident
// batches of 16-byte loads provide without barriers between producer and consumer.
//
//   forward:    Y^T[N, M]  = dec(W)[N, K] * X^T[K, M]       (MMA M = 16 output features)
//   grad-input: dX^T[K, M] = dec(W)^T[K, N] * dY^T[N, M]    (MMA M = 16 output columns)
//
// Because the reduction is a sum, the k (forward) and n (grad-input) positions inside an MMA
// are relabelled freely, as long as both operands use the same relabelling. Forward: lane
// (g, t) loads 16 consecutive codes of rows g and g + 8 at k0 + 16 t; MMA step j uses codes
// 4 j .. 4 j + 3 of that slice, and the same four activations. Grad-input: lane (g, t) loads
// 16 consecutive codes (output columns k0 + 16 g ..) of the four reduction rows n0 + 4 t .. + 3;
// MMA tile j takes columns 2 j and 2 j + 1 of the slice (byte-interleaved across two rows with
// one prmt), and the same four dY values per lane serve all eight tiles.
//
// A CTA of 8 warps owns 16 output features (forward) or 128 output columns (grad-input) and a
// range of the reduction; its warps take interleaved slabs of that range and add their
// partial sums in shared memory at the end. When the output alone cannot occupy the GPU the
// reduction is also split across CTAs: f32 partials go to the caller's workspace and the
// split-K reduction kernel adds them in split order (deterministic), with the bias.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "dequant.cuh"
#include "errors.cuh"
#include "gemm_args.cuh"

namespace moss {
namespace gemm {
namespace stream {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kFwdRows = 16;     // output features per forward CTA
constexpr int kFwdSlab = 64;     // reduction elements per forward slab (16 codes per lane x 4 lanes)
constexpr int kDxCols = 128;     // output columns per grad-input CTA
constexpr int kDxSlab = 16;      // reduction rows per grad-input slab
// Weight loads in flight per warp: the forward keeps kFwdBatch slabs of 1 KB in rotating
// register slots (a slot is refilled as soon as its last word is decoded, so the count never
// drains between batches); the grad-input issues batches of kDxBatch slabs of 2 KB. The
// forward's 64-register budget fits four CTAs (32 warps) per SM. Measured on the forward
// shapes (CUDA-graph timed, 2 x 3072 -> 18432): rotating 2 slots 14.75 us, 3 slots 15.5,
// 4 slots at 3 CTAs per SM 16.9; batches that drain before the next refill: 3 x 4
// CTAs 14.7-14.8 us, 4 x 3 16.5, 2 x 5 15.9, 6 x 2 19.2; a per-warp cp.async ring of 4-8 slabs
// in shared memory 16.5-17.3 us. At 16 rows the rotating slots are 8% faster (21.1 vs 23.0 us).
#ifndef MOSS_STREAM_FWD_BATCH
#define MOSS_STREAM_FWD_BATCH 2
#endif
#ifndef MOSS_STREAM_CTAS_PER_SM
#define MOSS_STREAM_CTAS_PER_SM 2
#endif
constexpr int kFwdBatch = MOSS_STREAM_FWD_BATCH;
constexpr int kDxBatch = 2;
#ifndef MOSS_STREAM_MIN_CTAS
#define MOSS_STREAM_MIN_CTAS 4
#endif
constexpr int kMinCtasPerSm = MOSS_STREAM_MIN_CTAS;  // register budget: 65536 / (4 x 256) = 64 per thread

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ldg16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ldg8(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// D (16 x 8, f32) += A (16 x 16) * B (16 x 8), 16-bit operands of kind kV.
template <int kV>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  if constexpr (kV == kBF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

// Decode of a byte-interleaved word [a0, b0, a1, b1] (codes of rows a and b) with row scales
// sa and sb: lo = (dec a0, dec b0), hi = (dec a1, dec b1). Same rounding as Dec::word.
template <int kV, bool kFast>
struct PairDec {
  uint32_t s2;
  float sa, sb;
  __device__ __forceinline__ void set(float a, float b, int w_kind) {
    if constexpr (kFast) {
      if constexpr (kV == kBF16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        s2 = *reinterpret_cast<uint32_t*>(&h);
      } else {
        __half2 h = __floats2half2_rn(a, b);
        s2 = *reinterpret_cast<uint32_t*>(&h);
      }
    } else {
      sa = round_to_kind(a, w_kind);
      sb = round_to_kind(b, w_kind);
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
      float d[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float q = static_cast<float>(static_cast<int8_t>((w >> (8 * i)) & 0xFF));
        d[i] = round_to_kind(q * ((i & 1) ? sb : sa), w_kind);
      }
      lo = pack2(d[0], d[1], kV);
      hi = pack2(d[2], d[3], kV);
    }
  }
};

// ------------------------------------------------------------------------------- forward
// grid = ceil(N / 16) * splits; block = 256. CTA b: row group b / splits, reduction split
// b % splits (slabs [split * per_split, ...) of 64 elements).
template <int kV, bool kFast, int kMT>
__global__ void __launch_bounds__(kThreads, kMT == 1 ? kMinCtasPerSm : 2) w8_stream_fwd_kernel(const Args a, int splits, int per_split) {
  __shared__ float red[kWarps][kFwdRows][16 + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int group = blockIdx.x / splits, split = blockIdx.x - group * splits;
  const int n0 = group * kFwdRows;
  const int slabs = a.Kr / kFwdSlab;
  const int sl0 = split * per_split, sl1 = min(slabs, sl0 + per_split);

  // rows past N are clamped for the loads and dropped at the store
  const int ra = min(n0 + g, a.Nc - 1), rb = min(n0 + g + 8, a.Nc - 1);
  Dec<kV, kFast> da, db;
  da.set(__ldg(a.scale + ra), a.w_kind);
  db.set(__ldg(a.scale + rb), a.w_kind);
  const int8_t* wa = a.w + static_cast<int64_t>(ra) * a.ldw + 16 * t;
  const int8_t* wb = a.w + static_cast<int64_t>(rb) * a.ldw + 16 * t;
  const uint16_t* xr[kMT];
  bool xv[kMT];
#pragma unroll
  for (int mt = 0; mt < kMT; ++mt) {
    const int m = 8 * mt + g;
    xv[mt] = m < a.M;
    xr[mt] = static_cast<const uint16_t*>(a.a) + static_cast<int64_t>(xv[mt] ? m : 0) * a.lda + 16 * t;
  }

  float acc[kMT][4];
#pragma unroll
  for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[mt][i] = 0.0f;

  // Rotating slots: slot u holds the slab kFwdBatch positions ahead of the one being decoded;
  // it is refilled as soon as its last word is decoded, so every warp keeps kFwdBatch slabs
  // of weight loads in flight instead of draining to none at the end of each batch.
  uint4 qa[kFwdBatch], qb[kFwdBatch];
#pragma unroll
  for (int u = 0; u < kFwdBatch; ++u) {
    const int slab = sl0 + warp + kWarps * u;
    if (slab < sl1) {
      qa[u] = ldg_stream(wa + slab * kFwdSlab);
      qb[u] = ldg_stream(wb + slab * kFwdSlab);
    }
  }
  for (int sl = sl0 + warp; sl < sl1; sl += kWarps * kFwdBatch) {
#pragma unroll
    for (int u = 0; u < kFwdBatch; ++u) {
      const int slab = sl + kWarps * u;
      if (slab >= sl1) break;
      const int k0 = slab * kFwdSlab;
      const int next = slab + kWarps * kFwdBatch;
      uint4 xs[kMT][2];
#pragma unroll
      for (int mt = 0; mt < kMT; ++mt) {
        if (xv[mt]) {
          xs[mt][0] = ldg16(xr[mt] + k0);
          xs[mt][1] = ldg16(xr[mt] + k0 + 8);
        } else {
          xs[mt][0] = make_uint4(0, 0, 0, 0);
          xs[mt][1] = make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t r0, r1, r2, r3;
        da.word(word_of(qa[u], j), a.w_kind, r0, r2);
        db.word(word_of(qb[u], j), a.w_kind, r1, r3);
        if (j == 3 && next < sl1) {
          qa[u] = ldg_stream(wa + next * kFwdSlab);
          qb[u] = ldg_stream(wb + next * kFwdSlab);
        }
#pragma unroll
        for (int mt = 0; mt < kMT; ++mt) {
          const uint4& xw = xs[mt][j >> 1];
          const uint32_t b0 = (j & 1) ? xw.z : xw.x;
          const uint32_t b1 = (j & 1) ? xw.w : xw.y;
          mma16816<kV>(acc[mt], r0, r1, r2, r3, b0, b1);
        }
      }
    }
  }

  // D fragment: (feature g, tokens 2t, 2t+1) and (feature g + 8, same tokens) per n8 tile
#pragma unroll
  for (int mt = 0; mt < kMT; ++mt) {
    red[warp][g][8 * mt + 2 * t] = acc[mt][0];
    red[warp][g][8 * mt + 2 * t + 1] = acc[mt][1];
    red[warp][g + 8][8 * mt + 2 * t] = acc[mt][2];
    red[warp][g + 8][8 * mt + 2 * t + 1] = acc[mt][3];
  }
  __syncthreads();
  // thread i: token m = i / 16, feature n0 + i % 16 (consecutive threads: consecutive features)
  const int m = threadIdx.x >> 4, nl = threadIdx.x & 15;
  const int n = n0 + nl;
  if (m < a.M && n < a.Nc) {
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += red[w][nl][m];
    if (splits > 1) {
      a.partial[(static_cast<int64_t>(split) * a.M + m) * a.Nc + n] = v;
    } else {
      if (a.bias != nullptr) v += round_to_kind(load_as_float(a.bias, a.bias_kind, n), kV);
      store_from_float(a.out, a.out_kind, static_cast<int64_t>(m) * a.ldo + n, round_to_kind(v, kV));
    }
  }
}

// ------------------------------------------------------------------------------- grad-input
// grid = (Nc / 128) * splits; block = 256; dynamic shared memory = red. CTA b: one output strip
// (128 columns of dX) and one reduction split (slabs of 16 weight rows), ordered as below.
template <int kV, bool kFast, int kMT>
__global__ void __launch_bounds__(kThreads) w8_stream_dx_kernel(const Args a, int splits, int per_split) {
  constexpr int kRedStride = kDxCols + 1;
  extern __shared__ float red_dyn[];  // [kWarps][8 * kMT][kRedStride]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  // With up to 8 rows consecutive CTAs take the strips of one reduction range, so CTAs resident
  // together read whole weight rows (every 128-byte strip of them) rather than one strip of many
  // rows: 1-5% faster at 1-8 rows, 20% slower at 16 rows, which keep split-major order
  // (CUDA-graph timed, 3072-18432 wide).
  int strip, split;
  if constexpr (kMT == 1) {
    const int strips = a.Nc / kDxCols;
    split = blockIdx.x / strips;
    strip = blockIdx.x - split * strips;
  } else {
    strip = blockIdx.x / splits;
    split = blockIdx.x - strip * splits;
  }
  const int k0 = strip * kDxCols;  // first output column of the strip
  const int slabs = a.w_rows / kDxSlab;
  const int sl0 = split * per_split, sl1 = min(slabs, sl0 + per_split);

  const int8_t* wcol = a.w + k0 + 16 * g;  // this lane's 16 output columns
  const uint16_t* dyr[kMT];
  bool dv[kMT];
#pragma unroll
  for (int mt = 0; mt < kMT; ++mt) {
    const int m = 8 * mt + g;
    dv[mt] = m < a.M;
    dyr[mt] = static_cast<const uint16_t*>(a.a) + static_cast<int64_t>(dv[mt] ? m : 0) * a.lda + 4 * t;
  }

  float acc[kMT][8][4];
#pragma unroll
  for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[mt][j][i] = 0.0f;

  // With 9-16 rows (two n8 tiles) each slab carries twice the MMA work, and rotating slots
  // (a slot refilled with the slab two positions ahead as soon as its last word is decoded)
  // were 10% faster at 16 rows; with up to 8 rows they were 4-9% slower than batches of
  // kDxBatch slabs that drain before the next refill (CUDA-graph timed, 3072-18432 wide).
  if constexpr (kMT == 2) {
    uint4 q[kDxBatch][4];
    float sc[kDxBatch][4];
    auto load_slab = [&](int u, int slab) {
      const int r0 = slab * kDxSlab + 4 * t;  // this lane's four reduction rows
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        q[u][i] = ldg_stream(wcol + static_cast<int64_t>(r0 + i) * a.ldw);
        sc[u][i] = __ldg(a.scale + r0 + i);
      }
    };
#pragma unroll
    for (int u = 0; u < kDxBatch; ++u)
      if (sl0 + warp + kWarps * u < sl1) load_slab(u, sl0 + warp + kWarps * u);
    for (int sl = sl0 + warp; sl < sl1; sl += kWarps * kDxBatch) {
#pragma unroll
      for (int u = 0; u < kDxBatch; ++u) {
        const int slab = sl + kWarps * u;
        if (slab >= sl1) break;
        const int next = slab + kWarps * kDxBatch;
        uint2 dy[kMT];
#pragma unroll
        for (int mt = 0; mt < kMT; ++mt) dy[mt] = dv[mt] ? ldg8(dyr[mt] + slab * kDxSlab) : make_uint2(0, 0);
        PairDec<kV, kFast> d01, d23;
        d01.set(sc[u][0], sc[u][1], a.w_kind);
        d23.set(sc[u][2], sc[u][3], a.w_kind);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t sel = (j & 1) ? 0x7362u : 0x5140u;  // bytes (2j, 2j+1) of two rows, interleaved
          const uint32_t u01 = prmt(word_of(q[u][0], j >> 1), word_of(q[u][1], j >> 1), sel);
          const uint32_t u23 = prmt(word_of(q[u][2], j >> 1), word_of(q[u][3], j >> 1), sel);
          uint32_t r0, r1, r2, r3;
          d01.word(u01, a.w_kind, r0, r1);
          d23.word(u23, a.w_kind, r2, r3);
          if (j == 7 && next < sl1) load_slab(u, next);
#pragma unroll
          for (int mt = 0; mt < kMT; ++mt) mma16816<kV>(acc[mt][j], r0, r1, r2, r3, dy[mt].x, dy[mt].y);
        }
      }
    }
  } else {
    for (int sl = sl0 + warp; sl < sl1; sl += kWarps * kDxBatch) {
      uint4 q[kDxBatch][4];
      float sc[kDxBatch][4];
#pragma unroll
      for (int u = 0; u < kDxBatch; ++u) {
        const int slab = sl + kWarps * u;
        if (slab < sl1) {
          const int r0 = slab * kDxSlab + 4 * t;  // this lane's four reduction rows
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            q[u][i] = ldg_stream(wcol + static_cast<int64_t>(r0 + i) * a.ldw);
            sc[u][i] = __ldg(a.scale + r0 + i);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kDxBatch; ++u) {
        const int slab = sl + kWarps * u;
        if (slab >= sl1) break;
        uint2 dy[kMT];
#pragma unroll
        for (int mt = 0; mt < kMT; ++mt) dy[mt] = dv[mt] ? ldg8(dyr[mt] + slab * kDxSlab) : make_uint2(0, 0);
        PairDec<kV, kFast> d01, d23;
        d01.set(sc[u][0], sc[u][1], a.w_kind);
        d23.set(sc[u][2], sc[u][3], a.w_kind);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint32_t sel = (j & 1) ? 0x7362u : 0x5140u;  // bytes (2j, 2j+1) of two rows, interleaved
          const uint32_t u01 = prmt(word_of(q[u][0], j >> 1), word_of(q[u][1], j >> 1), sel);
          const uint32_t u23 = prmt(word_of(q[u][2], j >> 1), word_of(q[u][3], j >> 1), sel);
          uint32_t r0, r1, r2, r3;
          d01.word(u01, a.w_kind, r0, r1);
          d23.word(u23, a.w_kind, r2, r3);
#pragma unroll
          for (int mt = 0; mt < kMT; ++mt) mma16816<kV>(acc[mt][j], r0, r1, r2, r3, dy[mt].x, dy[mt].y);
        }
      }
    }

  }

  // D fragment of tile j: (column 16 g + 2 j, tokens 2t, 2t+1), (column 16 g + 2 j + 1, same)
#pragma unroll
  for (int mt = 0; mt < kMT; ++mt) {
    float* base = red_dyn + static_cast<int64_t>(warp * 8 * kMT + 8 * mt + 2 * t) * kRedStride + 16 * g;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      base[2 * j] = acc[mt][j][0];
      base[kRedStride + 2 * j] = acc[mt][j][1];
      base[2 * j + 1] = acc[mt][j][2];
      base[kRedStride + 2 * j + 1] = acc[mt][j][3];
    }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < a.M * kDxCols; idx += kThreads) {
    const int m = idx / kDxCols, cl = idx - m * kDxCols;
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += red_dyn[static_cast<int64_t>(w * 8 * kMT + m) * kRedStride + cl];
    const int col = k0 + cl;
    if (splits > 1) {
      a.partial[(static_cast<int64_t>(split) * a.M + m) * a.Nc + col] = v;
    } else {
      store_from_float(a.out, a.out_kind, static_cast<int64_t>(m) * a.ldo + col, round_to_kind(v, kV));
    }
  }
}

template <bool kDX, int kV, bool kFast, int kMT>
static int launch_typed(const Args& a, const StreamPlan& p, cudaStream_t stream) {
  if constexpr (!kDX) {
    w8_stream_fwd_kernel<kV, kFast, kMT><<<p.ctas, kThreads, 0, stream>>>(a, p.splits, p.per_split);
  } else {
    constexpr int smem = kWarps * 8 * kMT * (kDxCols + 1) * static_cast<int>(sizeof(float));
    auto kern = w8_stream_dx_kernel<kV, kFast, kMT>;
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [&] { attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); });
    MOSS_CUDA_TRY(attr_err);
    kern<<<p.ctas, kThreads, smem, stream>>>(a, p.splits, p.per_split);
  }
  MOSS_CUDA_TRY(cudaGetLastError());
  if (p.splits > 1)
    return launch_splitk_reduce(kV, a.partial, p.splits, a.M, a.Nc, kDX ? nullptr : a.bias, a.bias_kind, a.out,
                                a.out_kind, a.ldo, stream);
  return MOSS_OK;
}

template <bool kDX, int kV, bool kFast>
static int launch_mt(const Args& a, const StreamPlan& p, cudaStream_t s) {
  return a.M <= 8 ? launch_typed<kDX, kV, kFast, 1>(a, p, s) : launch_typed<kDX, kV, kFast, 2>(a, p, s);
}

}  // namespace stream

// The reduction is split across CTAs only as far as the output tiles leave SMs idle: about two
// CTAs of 8 warps per SM keep ~64 KB of weight loads in flight per SM, enough to cover the HBM
// latency, and each warp keeps at least one slab per split.
StreamPlan plan_stream(bool dx, int64_t M, int64_t Nc, int64_t Kr, int sms) {
  using namespace stream;
  StreamPlan p;
  if (M <= 0 || M > kStreamMaxRows || Nc <= 0 || Kr <= 0 || Nc > INT32_MAX || Kr > INT32_MAX) return p;
  int64_t tiles, slabs;
  if (!dx) {
    if (Kr % kFwdSlab != 0) return p;
    tiles = (Nc + kFwdRows - 1) / kFwdRows;
    slabs = Kr / kFwdSlab;
  } else {
    if (Nc % kDxCols != 0 || Kr % kDxSlab != 0) return p;
    tiles = Nc / kDxCols;
    slabs = Kr / kDxSlab;
  }
  const int64_t target = static_cast<int64_t>(MOSS_STREAM_CTAS_PER_SM) * sms;
  int64_t splits = std::min<int64_t>((target + tiles - 1) / tiles, std::max<int64_t>(1, slabs / kWarps));
  splits = std::max<int64_t>(1, splits);
  const int64_t per = (slabs + splits - 1) / splits;
  splits = (slabs + per - 1) / per;
  if (tiles * splits > INT32_MAX) return p;
  p.usable = true;
  p.splits = static_cast<int>(splits);
  p.per_split = static_cast<int>(per);
  p.ctas = static_cast<int>(tiles * splits);
  p.partial_bytes = splits > 1 ? (static_cast<size_t>(splits) * M * Nc * 4 + 255) / 256 * 256 : 0;
  return p;
}

StreamPlan unsplit(StreamPlan p) {
  if (!p.usable || p.splits == 1) return p;
  const int tiles = p.ctas / p.splits;
  p.per_split = p.per_split * p.splits;
  p.splits = 1;
  p.ctas = tiles;
  p.partial_bytes = 0;
  return p;
}

int launch_stream(bool dx, int v_kind, bool fast, const Args& a, const StreamPlan& p, cudaStream_t s) {
  using namespace stream;
  if (!p.usable || a.ext_r > 0) return MOSS_ERR_UNSUPPORTED;
  // 16-byte vector loads of weight rows and activation rows; 8-byte loads of dY in the grad-input
  if ((reinterpret_cast<uintptr_t>(a.w) & 15) != 0 || (a.ldw & 15) != 0) return MOSS_ERR_UNSUPPORTED;
  if (!dx && ((reinterpret_cast<uintptr_t>(a.a) & 15) != 0 || (a.lda & 7) != 0)) return MOSS_ERR_UNSUPPORTED;
  if (dx && ((reinterpret_cast<uintptr_t>(a.a) & 7) != 0 || (a.lda & 3) != 0)) return MOSS_ERR_UNSUPPORTED;
  if (p.splits > 1 && a.partial == nullptr) return MOSS_ERR_UNSUPPORTED;
  if (dx) {
    if (v_kind == kBF16) return fast ? launch_mt<true, kBF16, true>(a, p, s) : launch_mt<true, kBF16, false>(a, p, s);
    return fast ? launch_mt<true, kF16, true>(a, p, s) : launch_mt<true, kF16, false>(a, p, s);
  }
  if (v_kind == kBF16) return fast ? launch_mt<false, kBF16, true>(a, p, s) : launch_mt<false, kBF16, false>(a, p, s);
  return fast ? launch_mt<false, kF16, true>(a, p, s) : launch_mt<false, kF16, false>(a, p, s);
}

}  // namespace gemm
}  // namespace moss
