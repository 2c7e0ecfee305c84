// Weight-only int8 GEMM for sm_100a: TMA -> shared-memory dequant -> tcgen05.mma -> TMEM.
//
// One kernel template covers both directions of the frozen int8 linear:
//   forward (kDX = false): C[M, N] = X[M, K] * dec(W)[N, K]^T   (B operand K-major)
//   grad-in (kDX = true):  C[M, K] = dY[M, N] * dec(W)[N, K]     (B operand MN-major)
// In both cases the int8 weight is read in its [N, K] storage order; for the grad-input the
// transpose lives only in the UMMA shared-memory descriptor (MN-major, 128B swizzle).
//
// Persistent, warp-specialised CTA (512 threads, one CTA per SM):
//   warp 0      TMA producer: bf16 A tile (128 x 64) + int8 W tile per stage
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer (M=128, N=256, K=16)
//   warps 4-7   epilogue: tcgen05.ld of the accumulator, bias, rounding, global stores
//   warps 8-15  converters: int8 -> f16/bf16 with the per-channel scale, written straight
//               into the canonical SW128 operand layout the MMA reads
// Accumulators are double-buffered in TMEM (2 x 256 f32 columns) so the epilogue of tile
// i overlaps the main loop of tile i+1.
//
// Decode rounding follows training/quant_kernels.py:138-149 (and the eager
// training/quantization.py:23-24): dec = round_v(round_w(q * round_w(s))), with v the
// compute dtype and w the module (weight) dtype. For v == w the converter uses an exact
// integer trick (see dequant_word_bf16/_f16); the rare v != w case decodes in f32.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "dequant.cuh"
#include "errors.cuh"
#include "gemm_args.cuh"

namespace moss {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int kStages = 4;   // A + int8 W stages
constexpr int kBStages = 2;  // converted 16-bit B stages
constexpr int kConvWarps = 8;
constexpr int kEpiWarp0 = 4;
constexpr int kConvWarp0 = 8;
constexpr int kThreads = 16 * 32;
constexpr uint32_t kABytes = BM * BK * 2;  // 16 KB
constexpr uint32_t kWBytes = BN * BK;      // 16 KB
constexpr uint32_t kBBytes = BN * BK * 2;  // 32 KB
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kDataBytes = kStages * (kABytes + kWBytes) + kBStages * kBBytes;
constexpr uint32_t kSmemBytes = kDataBytes + 1024 + 256;
// Problems with more rows than this use the CTA-pair kernel (256-row tiles) when TMA can
// describe them; smaller ones keep 128-row tiles.
constexpr int64_t kPairMinRows = 128;
// Split-K (f32 partials through the caller's workspace) is used up to this many rows.
constexpr int64_t kSplitMaxRows = 32;

struct Barriers {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t b_full[kBStages];
  uint64_t b_empty[kBStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(Barriers) <= 256, "barrier block too large");

// Byte offset of element (row, col) of a 16-bit K-major SW128 tile (rows of 64 elements).
__device__ __forceinline__ uint32_t sw128_kmajor_off16(int row, int col) {
  return static_cast<uint32_t>((row >> 3) * 1024 + (row & 7) * 128 + ((((col >> 3) ^ (row & 7)) & 7) << 4) +
                               (col & 7) * 2);
}

// --------------------------------------------------------------------------------------------
template <bool kDX, int kV, bool kFast>
__global__ void __launch_bounds__(kThreads, 1)
    w8_gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w,
                   const __grid_constant__ CUtensorMap tm_ext, const Args args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* const base_ptr = smem_raw + (base - raw_base);
  const uint32_t a_smem = base;
  const uint32_t w_smem = base + kStages * kABytes;
  const uint32_t b_smem = w_smem + kStages * kWBytes;
  Barriers* bars = reinterpret_cast<Barriers*>(base_ptr + kDataBytes);
  auto bar = [&](uint64_t& b) { return smem_u32(&b); };
  volatile int* abort_flag = &bars->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = args.tiles_m * args.tiles_n;
  const int num_units = num_tiles * args.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(bars->full[s]), 1);
      mbar_init(bar(bars->empty[s]), 1 + kConvWarps);
    }
    for (int s = 0; s < kBStages; ++s) {
      mbar_init(bar(bars->b_full[s]), kConvWarps);
      mbar_init(bar(bars->b_empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(bars->acc_full[s]), 1);
      mbar_init(bar(bars->acc_empty[s]), 4);
    }
    mbar_init(bar(bars->drain), 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&bars->tmem_base), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    if (!args.manual && lane == 0) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_w);
      if (args.ext_r > 0) tma_prefetch_desc(&tm_ext);
    }
    int stage = 0;
    uint32_t phase = 0;
    uint32_t used_mask = 0;        // stages that received a TMA copy
    uint32_t last_phase_mask = 0;  // phase bit of the last copy per stage
    bool ok = true;
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
      const int t = u / args.splits;
      const UnitRange ur = unit_range(args, u - t * args.splits);
      int m_blk, n_blk;
      tile_coords(t, args.tiles_m, args.tiles_n, m_blk, n_blk);
      const int m0 = m_blk * BM;
      const int n0 = n_blk * BN;
      for (int i = 0; i < ur.n_iter; ++i) {
        const int kb = ur.kb(i, args.main_kb);
        if (!mbar_wait(bar(bars->empty[stage]), phase ^ 1u, abort_flag, args.status, MOSS_STATUS_TIMEOUT_LOAD)) {
          ok = false;
          break;
        }
        const bool ext = kb >= args.main_kb;
        const uint32_t a_dst = a_smem + stage * kABytes;
        const uint32_t w_dst = w_smem + stage * kWBytes;
        if (!args.manual) {
          if (lane == 0) {
            const uint32_t fb = bar(bars->full[stage]);
            if (!ext) {
              mbar_arrive_expect_tx(fb, kABytes + kWBytes);
              tma_load_2d(a_dst, &tm_a, fb, kb * BK, m0);
              if constexpr (!kDX) {
                tma_load_2d(w_dst, &tm_w, fb, kb * BK, n0);
              } else {
                tma_load_2d(w_dst, &tm_w, fb, n0, kb * BK);
                tma_load_2d(w_dst + kWBytes / 2, &tm_w, fb, n0 + 128, kb * BK);
              }
            } else {
              mbar_arrive_expect_tx(fb, kABytes);
              tma_load_2d(a_dst, &tm_ext, fb, (kb - args.main_kb) * BK, m0);
            }
            used_mask |= 1u << stage;
            last_phase_mask = (last_phase_mask & ~(1u << stage)) | (phase << stage);
          }
        } else {
          // Plain loads into the exact layouts TMA would have produced.
          const uint16_t* asrc = static_cast<const uint16_t*>(ext ? args.ext_a : args.a);
          const int64_t lda = ext ? args.ld_ext_a : args.lda;
          const int acols = ext ? args.ext_r : args.Kr;
          const int k0 = (ext ? (kb - args.main_kb) : kb) * BK;
          uint8_t* a_ptr = base_ptr + (a_dst - base);
          for (int idx = lane; idx < BM * BK; idx += 32) {
            const int r = idx / BK, c = idx % BK;
            const int gm = m0 + r, gk = k0 + c;
            const uint16_t v = (gm < args.M && gk < acols) ? asrc[static_cast<int64_t>(gm) * lda + gk] : 0;
            *reinterpret_cast<uint16_t*>(a_ptr + sw128_kmajor_off16(r, c)) = v;
          }
          if (!ext) {
            uint8_t* w_ptr = base_ptr + (w_dst - base);
            if constexpr (!kDX) {
              for (int idx = lane; idx < BN * BK; idx += 32) {
                const int r = idx / BK, c = idx % BK;
                const int gn = n0 + r, gk = kb * BK + c;
                w_ptr[r * BK + c] = (gn < args.w_rows && gk < args.w_cols)
                                        ? static_cast<uint8_t>(args.w[static_cast<int64_t>(gn) * args.ldw + gk])
                                        : 0;
              }
            } else {
              for (int idx = lane; idx < BK * BN; idx += 32) {
                const int r = idx / BN, c = idx % BN;  // r: reduction row (n), c: output col (k)
                const int gn = kb * BK + r, gk = n0 + c;
                const uint8_t v = (gn < args.w_rows && gk < args.w_cols)
                                      ? static_cast<uint8_t>(args.w[static_cast<int64_t>(gn) * args.ldw + gk])
                                      : 0;
                const int box = c >> 7, c8 = (c & 127) >> 4;
                w_ptr[box * (kWBytes / 2) + r * 128 + (((c8 ^ (r & 7)) & 7) << 4) + (c & 15)] = v;
              }
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(bars->full[stage]));
        }
        __syncwarp();
        if (++stage == kStages) { stage = 0; phase ^= 1u; }
      }
    }
    // Drain: never leave with our own TMA copies still writing into shared memory.
    if (!args.manual && lane == 0) {
      for (int s = 0; s < kStages; ++s) {
        if (!((used_mask >> s) & 1u)) continue;
        const long long start = clock64();
        while (!mbar_try_wait(bar(bars->full[s]), (last_phase_mask >> s) & 1u)) {
          if (clock64() - start > kWaitBudgetCycles) {
            report_status(args.status, MOSS_STATUS_TIMEOUT_DRAIN);
            break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = umma_idesc_f16(kV == kBF16 ? 1u : 0u, kDX, BM, BN);
    int stage = 0, bstage = 0;
    uint32_t phase = 0, bphase = 0;
    int it = 0;
    bool ok = true;
    bool issued_any = false;
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++it) {
      const UnitRange ur = unit_range(args, u % args.splits);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(bar(bars->acc_empty[acc]), acc_phase ^ 1u, abort_flag, args.status, MOSS_STATUS_TIMEOUT_MMA)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
      for (int i = 0; i < ur.n_iter; ++i) {
        if (!mbar_wait(bar(bars->full[stage]), phase, abort_flag, args.status, MOSS_STATUS_TIMEOUT_MMA) ||
            !mbar_wait(bar(bars->b_full[bstage]), bphase, abort_flag, args.status, MOSS_STATUS_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_base = a_smem + stage * kABytes;
          const uint32_t b_base = b_smem + bstage * kBBytes;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t adesc = umma_desc_sw128(a_base + kk * 32, 16, 1024);
            uint64_t bdesc;
            if constexpr (!kDX) {
              bdesc = umma_desc_sw128(b_base + kk * 32, 16, 1024);
            } else {
              bdesc = umma_desc_sw128(b_base + kk * 2048, 8192, 1024);
            }
            umma_f16(d_tmem, adesc, bdesc, idesc, (i | kk) != 0 ? 1u : 0u);
          }
          umma_commit(bar(bars->empty[stage]));
          umma_commit(bar(bars->b_empty[bstage]));
          issued_any = true;
        }
        __syncwarp();
        if (++stage == kStages) { stage = 0; phase ^= 1u; }
        if (++bstage == kBStages) { bstage = 0; bphase ^= 1u; }
      }
      if (!ok) break;
      if (lane == 0) umma_commit(bar(bars->acc_full[acc]));
      __syncwarp();
    }
    // Drain: all issued MMAs must retire before TMEM is released.
    if (lane == 0 && issued_any) {
      umma_commit(bar(bars->drain));
      const long long start = clock64();
      while (!mbar_try_wait(bar(bars->drain), 0)) {
        if (clock64() - start > kWaitBudgetCycles) {
          report_status(args.status, MOSS_STATUS_TIMEOUT_DRAIN);
          break;
        }
      }
    }
    __syncwarp();
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int it = 0;
    for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++it) {
      const int t = u / args.splits;
      const int split = u - t * args.splits;
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(bar(bars->acc_full[acc]), acc_phase, abort_flag, args.status, MOSS_STATUS_TIMEOUT_EPILOGUE))
        break;
      tc_fence_after();
      int m_blk, n_blk;
      tile_coords(t, args.tiles_m, args.tiles_n, m_blk, n_blk);
      const int m0 = m_blk * BM;
      const int n0 = n_blk * BN;
      const int row = m0 + q * 32 + lane;
      const bool row_ok = row < args.M;
      const bool vec_ok = (args.out_kind != kF32) && ((args.ldo & 7) == 0) &&
                          ((reinterpret_cast<uintptr_t>(args.out) & 15) == 0);
      const bool split_k = args.splits > 1;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN + c * 32), r);
        tmem_wait_ld();
        if (c == BN / 32 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(bars->acc_empty[acc]));
        }
        const int col0 = n0 + c * 32;
        if (col0 >= args.Nc) continue;
        if (split_k) {
          // partial f32 sums of this split; reduced below by the tile's last split
          if (!row_ok) continue;
          float* dst = args.partial + (static_cast<int64_t>(split) * args.M + row) * args.Nc + col0;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col0 + j < args.Nc) dst[j] = __uint_as_float(r[j]);
          continue;
        }
        if (!row_ok) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if constexpr (!kDX) {
          if (args.bias != nullptr) {
            float b[32];
            load_bias32<kV>(args.bias, args.bias_kind, col0, args.Nc, b);
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] += b[j];
          }
        }
        const int64_t off = static_cast<int64_t>(row) * args.ldo + col0;
        if (args.out_kind == kV && vec_ok && col0 + 32 <= args.Nc) {
          uint32_t p[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) p[j] = pack2_kind<kV>(v[2 * j], v[2 * j + 1]);
          uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(args.out) + off);
#pragma unroll
          for (int j = 0; j < 4; ++j) dst[j] = make_uint4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col0 + j < args.Nc) store_from_float(args.out, args.out_kind, off + j, round_to_kind(v[j], kV));
        }
      }
      if (!split_k) continue;
      // Per 32-row slice (one epilogue warp): the last split to finish reduces all partials of
      // the slice in split order (deterministic). Warps never wait on each other here.
      __threadfence();
      __syncwarp();
      int done = 0;
      if (lane == 0) done = atomicAdd(args.counters + t * 4 + q, 1);
      done = __shfl_sync(0xffffffffu, done, 0);
      if (done != args.splits - 1) continue;
      __threadfence();
      if (row_ok) {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          const int col0 = n0 + c * 32;
          if (col0 >= args.Nc) break;
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0.0f;
          for (int sp = 0; sp < args.splits; ++sp) {
            const float* src = args.partial + (static_cast<int64_t>(sp) * args.M + row) * args.Nc + col0;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < args.Nc) v[j] += __ldcg(src + j);
          }
          const int64_t off = static_cast<int64_t>(row) * args.ldo + col0;
          if constexpr (!kDX) {
            if (args.bias != nullptr) {
              float b[32];
              load_bias32<kV>(args.bias, args.bias_kind, col0, args.Nc, b);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] += b[j];
            }
          }
          if (args.out_kind == kV && vec_ok && col0 + 32 <= args.Nc) {
            uint32_t p[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) p[j] = pack2_kind<kV>(v[2 * j], v[2 * j + 1]);
            uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(args.out) + off);
#pragma unroll
            for (int j = 0; j < 4; ++j) dst[j] = make_uint4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < args.Nc) store_from_float(args.out, args.out_kind, off + j, round_to_kind(v[j], kV));
          }
        }
      }
      __syncwarp();
      if (lane == 0) args.counters[t * 4 + q] = 0;  // ready for the next call
    }
  } else if (warp >= kConvWarp0) {
    // ------------------------------------------------------------------ converters
    const int ct = threadIdx.x - kConvWarp0 * 32;  // 0..255
    int stage = 0, bstage = 0;
    uint32_t phase = 0, bphase = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
      const int t = u / args.splits;
      const UnitRange ur = unit_range(args, u - t * args.splits);
      int m_blk, n_blk;
      tile_coords(t, args.tiles_m, args.tiles_n, m_blk, n_blk);
      const int n0 = n_blk * BN;
      // forward: this thread always handles tile rows (ct >> 2) + 64 j, j = 0..3
      Dec<kV, kFast> dec_f[4];
      if constexpr (!kDX) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int gn = n0 + (ct >> 2) + 64 * j;
          dec_f[j].set(gn < args.w_rows ? args.scale[gn] : 0.0f, args.w_kind);
        }
      }
      for (int i = 0; i < ur.n_iter; ++i) {
        const int kb = ur.kb(i, args.main_kb);
        if (!mbar_wait(bar(bars->full[stage]), phase, abort_flag, args.status, MOSS_STATUS_TIMEOUT_CONVERT) ||
            !mbar_wait(bar(bars->b_empty[bstage]), bphase ^ 1u, abort_flag, args.status, MOSS_STATUS_TIMEOUT_CONVERT)) {
          ok = false;
          break;
        }
        const uint32_t w_base = w_smem + stage * kWBytes;
        const uint32_t b_base = b_smem + bstage * kBBytes;
        const bool ext = kb >= args.main_kb;
        if constexpr (!kDX) {
          const int c = ct & 3;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int row = (ct >> 2) + 64 * j;
            uint4 o0, o1;
            if (!ext) {
              const uint4 qv = lds128(w_base + row * 64 + c * 16);
              dec_f[j].chunk(qv, args.w_kind, o0, o1);
            } else {
              float f[16];
              const int gn = n0 + row;
              if (gn < args.Nc) {
                load16_f32(args.ext_b, args.ext_b_kind, static_cast<int64_t>(gn) * args.ld_ext_b,
                           (kb - args.main_kb) * BK + c * 16, args.ext_r, f);
              } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) f[i] = 0.0f;
              }
              pack16_scaled(f, args.ext_scale, kV, o0, o1);
            }
            const uint32_t rbase = b_base + (row >> 3) * 1024 + (row & 7) * 128;
            sts128(rbase + ((((2 * c) ^ (row & 7)) & 7) << 4), o0);
            sts128(rbase + ((((2 * c + 1) ^ (row & 7)) & 7) << 4), o1);
          }
        } else {
          // grad-input: rows are reduction indices; this thread owns one row per stage.
          const int cw = ct >> 5;
          const int ph = lane >> 3;
          const int hi = (lane >> 2) & 1;
          const int qd = lane & 3;
          const int r_in = hi ? (ph ^ 5) : ph;  // row pairs (0,5) (1,4) (2,7) (3,6)
          const int row = cw * 8 + r_in;
          Dec<kV, kFast> dec;
          if (!ext) {
            const int gn = kb * BK + row;
            dec.set(gn < args.w_rows ? args.scale[gn] : 0.0f, args.w_kind);
          }
#pragma unroll
          for (int a = 0; a < 4; ++a) {
            const int c16 = 4 * a + qd;
            uint4 o0, o1;
            if (!ext) {
              const int box = a >> 1, c8 = 4 * (a & 1) + qd;
              const uint4 qv = lds128(w_base + box * (kWBytes / 2) + row * 128 + (((c8 ^ r_in) & 7) << 4));
              dec.chunk(qv, args.w_kind, o0, o1);
            } else {
              float f[16];
              const int gj = (kb - args.main_kb) * BK + row;
              if (gj < args.ext_r) {
                load16_f32(args.ext_b, args.ext_b_kind, static_cast<int64_t>(gj) * args.ld_ext_b, n0 + c16 * 16,
                           args.Nc, f);
              } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) f[i] = 0.0f;
              }
              pack16_scaled(f, args.ext_scale, kV, o0, o1);
            }
            const uint32_t rbase = b_base + a * (kBBytes / 4) + row * 128;
            sts128(rbase + ((((2 * qd) ^ r_in) & 7) << 4), o0);
            sts128(rbase + ((((2 * qd + 1) ^ r_in) & 7) << 4), o1);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(bar(bars->b_full[bstage]));
          mbar_arrive(bar(bars->empty[stage]));
        }
        if (++stage == kStages) { stage = 0; phase ^= 1u; }
        if (++bstage == kBStages) { bstage = 0; bphase ^= 1u; }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// K == 0: the product is empty, y = round(bias) (or zeros).
__global__ void fill_bias_kernel(int M, int N, const void* bias, int bias_kind, int v_kind, void* out, int out_kind,
                                 int64_t ldo) {
  const int64_t total = static_cast<int64_t>(M) * N;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / N, c = i % N;
    const float b = bias ? round_to_kind(load_as_float(bias, bias_kind, c), v_kind) : 0.0f;
    store_from_float(out, out_kind, r * ldo + c, round_to_kind(b, v_kind));
  }
}

// --------------------------------------------------------------------------------------------
// host side

static int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

template <bool kDX, int kV, bool kFast>
static int launch_typed(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& te, const Args& a,
                        cudaStream_t stream) {
  auto kern = w8_gemm_kernel<kDX, kV, kFast>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  });
  MOSS_CUDA_TRY(attr_err);
  const int units = a.tiles_m * a.tiles_n * a.splits;
  const int grid = std::min(units, sm_count());
  kern<<<grid, kThreads, kSmemBytes, stream>>>(ta, tw, te, a);
  MOSS_CUDA_TRY(cudaGetLastError());
  return MOSS_OK;
}

template <bool kDX>
static int dispatch(int v_kind, bool fast, const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& te,
                    const Args& a, cudaStream_t s) {
  if (v_kind == kBF16) {
    return fast ? launch_typed<kDX, kBF16, true>(ta, tw, te, a, s) : launch_typed<kDX, kBF16, false>(ta, tw, te, a, s);
  }
  return fast ? launch_typed<kDX, kF16, true>(ta, tw, te, a, s) : launch_typed<kDX, kF16, false>(ta, tw, te, a, s);
}

// Split-K plan of the 1-CTA kernel (small M: too few output tiles to occupy the GPU).
struct SplitPlan {
  int splits = 1;
  int kb_per_split = 0;
  size_t partial_bytes = 0;
  size_t counter_bytes = 0;
  size_t total() const { return splits > 1 ? partial_bytes + counter_bytes : 0; }
};

static bool use_pair(int64_t M, int64_t Nc, int sms) {
  if (M <= kPairMinRows) return false;
  const int64_t pair_tiles = ((M + 255) / 256) * ((Nc + 255) / 256);
  return pair_tiles * 4 >= sms;  // the pair grid fills at least half of the SMs
}

static SplitPlan plan_split(int64_t M, int64_t Nc, int64_t Kr, int sms) {
  SplitPlan p;
  const int64_t tiles = ((M + BM - 1) / BM) * ((Nc + BN - 1) / BN);
  const int64_t main_kb = (Kr + BK - 1) / BK;
  // Only for a few rows: the f32 partials then cost far less than the weight bytes.
  if (M > kSplitMaxRows || tiles <= 0 || tiles * 2 >= sms || main_kb < 8) return p;
  int64_t want = std::min<int64_t>((sms + tiles - 1) / tiles, std::min<int64_t>(main_kb / 4, 32));
  if (want < 2) return p;
  const int64_t kps = (main_kb + want - 1) / want;
  p.splits = static_cast<int>((main_kb + kps - 1) / kps);
  p.kb_per_split = static_cast<int>(kps);
  if (p.splits < 2) return SplitPlan{};
  p.partial_bytes = (static_cast<size_t>(p.splits) * M * Nc * 4 + 255) / 256 * 256;
  p.counter_bytes = (static_cast<size_t>(tiles) * 4 * 4 + 255) / 256 * 256;
  return p;
}

// Shared driver for both directions.
//   A: [M, Kr] in v_kind (x or dy); weight q: [w_rows, w_cols]; C: [M, Nc]
//   rot_group > 1 (grad-input only): ask the CTA-pair kernel to apply the ConvRot rotation in its
//   epilogue; *rotated reports whether it did (otherwise the caller rotates the output).
static int run(bool dx, const void* a_ptr, int v_kind, int64_t M, int64_t Kr, int64_t Nc, const int8_t* q,
               const float* scale, int w_kind, int64_t w_rows, int64_t w_cols, const void* bias, int bias_kind,
               const void* ext_a, const void* ext_b, int ext_b_kind, int64_t ext_r, float ext_scale, void* out,
               int out_kind, void* workspace, size_t workspace_bytes, int* status, cudaStream_t stream,
               int64_t rot_group = 0, bool* rotated = nullptr) {
  if (rotated != nullptr) *rotated = false;
  if (M < 0 || Kr < 0 || Nc < 0) return fail(MOSS_ERR_INVALID_ARGUMENT, "negative GEMM shape");
  if (v_kind != kBF16 && v_kind != kF16)
    return fail(MOSS_ERR_UNSUPPORTED, "compute dtype must be float16 or bfloat16 (got code %d)", v_kind);
  if (!is_float_kind(w_kind) || !is_float_kind(out_kind))
    return fail(MOSS_ERR_UNSUPPORTED, "unsupported weight/output dtype code");
  if (bias != nullptr && !is_float_kind(bias_kind)) return fail(MOSS_ERR_UNSUPPORTED, "unsupported bias dtype code");
  if (M > INT32_MAX || Kr > INT32_MAX || Nc > INT32_MAX) return fail(MOSS_ERR_INVALID_ARGUMENT, "GEMM dimension too large");
  if (ext_a != nullptr) {
    if (ext_b == nullptr || ext_r <= 0 || ext_r > 256 || !is_float_kind(ext_b_kind))
      return fail(MOSS_ERR_INVALID_ARGUMENT, "LoRA operands need rank in [1, 256] and both factors");
  }
  if (M == 0 || Nc == 0) return clear_ok();
  if (out == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null output pointer");
  if (Kr == 0 && ext_a == nullptr) {
    const int64_t total = M * Nc;
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 4096));
    fill_bias_kernel<<<grid, 256, 0, stream>>>(static_cast<int>(M), static_cast<int>(Nc), dx ? nullptr : bias,
                                               bias_kind, v_kind, out, out_kind, Nc);
    MOSS_CUDA_TRY(cudaGetLastError());
    return clear_ok();
  }
  if (Kr > 0 && (a_ptr == nullptr || q == nullptr || scale == nullptr))
    return fail(MOSS_ERR_INVALID_ARGUMENT, "null input, weight or scale pointer");

  Args a{};
  a.M = static_cast<int>(M);
  a.Nc = static_cast<int>(Nc);
  a.Kr = static_cast<int>(Kr);
  a.tiles_m = static_cast<int>((M + BM - 1) / BM);
  a.tiles_n = static_cast<int>((Nc + BN - 1) / BN);
  a.main_kb = static_cast<int>((Kr + BK - 1) / BK);
  const int ext_kb = ext_a ? static_cast<int>((ext_r + BK - 1) / BK) : 0;
  a.num_kb = a.main_kb + ext_kb;
  a.a = a_ptr;
  a.lda = Kr;
  a.w = q;
  a.ldw = w_cols;
  a.w_rows = static_cast<int>(w_rows);
  a.w_cols = static_cast<int>(w_cols);
  a.scale = scale;
  a.w_kind = w_kind;
  a.bias = dx ? nullptr : bias;
  a.bias_kind = bias_kind;
  a.out = out;
  a.out_kind = out_kind;
  a.ldo = Nc;
  a.ext_a = ext_a;
  a.ld_ext_a = ext_r;
  a.ext_b = ext_b;
  a.ext_b_kind = ext_b_kind;
  a.ld_ext_b = dx ? Nc : ext_r;
  a.ext_r = ext_a ? static_cast<int>(ext_r) : 0;
  a.ext_scale = ext_scale;
  a.status = StatusSink{status, status_mirror_for_current_device()};
  a.debug_stall = take_debug_stall() ? 1 : 0;
  a.splits = 1;
  a.kb_per_split = a.main_kb;
  a.partial = nullptr;
  a.counters = nullptr;
  a.tail_first = a.tiles_m * a.tiles_n;  // the CTA-pair kernel's last-round split: none
  a.tail_splits = 1;
  a.rot_group = 0;
  a.group_m = kGroupM;

  CUtensorMap ta, tw, te;
  memset(&ta, 0, sizeof(ta));
  memset(&tw, 0, sizeof(tw));
  memset(&te, 0, sizeof(te));
  const CUtensorMapDataType v_dt = v_kind == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  bool tma = make_map(&ta, v_dt, 2, a_ptr, Kr, M, Kr * 2, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (tma) {
    if (!dx)
      tma = make_map(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, q, w_cols, w_rows, w_cols, BK, BN,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
    else
      tma = make_map(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, q, w_cols, w_rows, w_cols, 128, BK,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (tma && ext_a != nullptr)
    tma = make_map(&te, v_dt, 2, ext_a, ext_r, M, ext_r * 2, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B);
  a.manual = tma ? 0 : 1;
  const bool fast = (w_kind == v_kind);
  const int sms = sm_count();
  if (dx && rot_group > 1 && tma && ext_a == nullptr && use_pair(M, Nc, sms)) {
    // ConvRot grad-input with the rotation in the CTA-pair epilogue (whole tiles, no split)
    Args a2 = a;
    a2.tiles_m = static_cast<int>((M + 255) / 256);
    a2.tiles_n = static_cast<int>((Nc + 255) / 256);
    a2.tail_first = a2.tiles_m * a2.tiles_n;
    a2.tail_splits = 1;
    a2.rot_group = static_cast<int>(rot_group);
    const int rc = launch_pair(dx, v_kind, fast, a2, stream);
    if (rc != MOSS_ERR_UNSUPPORTED) {
      if (rc == MOSS_OK && rotated != nullptr) *rotated = true;
      return rc;
    }
  }
  if (ext_a == nullptr && M <= kStreamMaxRows) {
    // A handful of rows: stream the weight at HBM speed, decode in registers, warp-level MMAs.
    StreamPlan sp = plan_stream(dx, M, Nc, Kr, sms);
    if (sp.usable) {
      Args s = a;
      if (sp.splits > 1 && workspace != nullptr && workspace_bytes >= sp.total() &&
          (reinterpret_cast<uintptr_t>(workspace) & 255) == 0) {
        s.partial = static_cast<float*>(workspace);
      } else {
        sp = unsplit(sp);
      }
      const int rc = launch_stream(dx, v_kind, fast, s, sp, stream);
      if (rc != MOSS_ERR_UNSUPPORTED) return rc;
    }
  }
  if (tma && ext_a == nullptr && !use_pair(M, Nc, sms)) {
    // Too few rows for the CTA-pair tiles: operand-swapped kernel that streams the weight over
    // all SMs (split over K when needed).
    const SkinnyPlan sp = plan_skinny(M, Nc, Kr, sms);
    if (sp.usable) {
      Args s = a;
      s.tiles_m = sp.tiles_m;
      s.tiles_n = sp.tiles_n;
      if (sp.splits > 1 && workspace != nullptr && workspace_bytes >= sp.total() &&
          (reinterpret_cast<uintptr_t>(workspace) & 255) == 0) {
        s.splits = sp.splits;
        s.kb_per_split = sp.kb_per_split;
        s.partial = static_cast<float*>(workspace);
        s.counters = nullptr;
      }
      const int rc = launch_skinny(dx, v_kind, fast, sp.nt, s, stream);
      if (rc != MOSS_ERR_UNSUPPORTED) return rc;
    }
  }
  if (tma && use_pair(M, Nc, sms)) {
    // CTA-pair kernel: 256 x 256 tiles, multi-k-block TMA boxes; falls through when the
    // shapes do not fit its boxes.
    Args a2 = a;
    a2.tiles_m = static_cast<int>((M + 255) / 256);
    a2.tiles_n = static_cast<int>((Nc + 255) / 256);
    a2.tail_first = a2.tiles_m * a2.tiles_n;
    a2.tail_splits = 1;
    const PairTailPlan tp = plan_pair_tail(M, Nc, Kr, sms);
    if (tp.splits > 1 && workspace != nullptr && workspace_bytes >= tp.total() &&
        (reinterpret_cast<uintptr_t>(workspace) & 255) == 0) {
      a2.tail_first = tp.tail_first;
      a2.tail_splits = tp.splits;
      a2.partial = static_cast<float*>(workspace);
    }
    const int rc = launch_pair(dx, v_kind, fast, a2, stream);
    if (rc != MOSS_ERR_UNSUPPORTED) return rc;
  }
  const SplitPlan plan = plan_split(M, Nc, Kr, sms);
  if (plan.splits > 1 && workspace != nullptr && workspace_bytes >= plan.total() &&
      (reinterpret_cast<uintptr_t>(workspace) & 255) == 0) {
    a.splits = plan.splits;
    a.kb_per_split = plan.kb_per_split;
    a.partial = static_cast<float*>(workspace);
    a.counters = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + plan.partial_bytes);
    MOSS_CUDA_TRY(cudaMemsetAsync(a.counters, 0, plan.counter_bytes, stream));
  }
  return dx ? dispatch<true>(v_kind, fast, ta, tw, te, a, stream) : dispatch<false>(v_kind, fast, ta, tw, te, a, stream);
}

}  // namespace gemm
}  // namespace moss

using namespace moss;

extern "C" int moss_w8a16_gemm_workspace_bytes(int64_t m, int64_t n_out, int64_t k_red, size_t* bytes) {
  if (bytes == nullptr) return fail(MOSS_ERR_INVALID_ARGUMENT, "null bytes pointer");
  *bytes = 0;
  if (m <= 0 || n_out <= 0 || k_red <= 0) return clear_ok();
  const int sms = gemm::sm_count();
  if (gemm::use_pair(m, n_out, sms)) {
    // the CTA-pair kernel's split of its last, partly empty round of tiles
    *bytes = gemm::plan_pair_tail(m, n_out, k_red, sms).total();
    return clear_ok();
  }
  // Enough for whichever kernel the call picks: the few-row kernel (no LoRA term) or the
  // 1-CTA kernel's split-K (with one).
  size_t need = gemm::plan_split(m, n_out, k_red, sms).total();
  const gemm::SkinnyPlan sp = gemm::plan_skinny(m, n_out, k_red, sms);
  if (sp.usable) need = std::max(need, sp.total());
  // the few-row streaming kernel (either direction: the query does not say which)
  need = std::max(need, gemm::plan_stream(false, m, n_out, k_red, sms).total());
  need = std::max(need, gemm::plan_stream(true, m, n_out, k_red, sms).total());
  *bytes = need;
  return clear_ok();
}

extern "C" int moss_w8a16_gemm_fwd(const void* x, int x_dtype, int64_t m, int64_t k, const int8_t* q,
                                   const float* scale, int weight_dtype, int64_t n, const void* bias, int bias_dtype,
                                   const void* lora_xa, const void* lora_b, int lora_b_dtype, int64_t lora_rank,
                                   float lora_scale, void* y, int y_dtype, void* workspace, size_t workspace_bytes,
                                   int* status, moss_stream_t stream) {
  const int rc = gemm::run(false, x, x_dtype, m, k, n, q, scale, weight_dtype, n, k, bias, bias_dtype, lora_xa, lora_b,
                           lora_b_dtype, lora_rank, lora_scale, y, y_dtype, workspace, workspace_bytes, status,
                           reinterpret_cast<cudaStream_t>(stream));
  return rc == MOSS_OK ? clear_ok() : rc;
}

extern "C" int moss_w8a16_gemm_dx(const void* dy, int dy_dtype, int64_t m, int64_t n, const int8_t* q,
                                  const float* scale, int weight_dtype, int64_t k, const void* lora_dyb,
                                  const void* lora_a, int lora_a_dtype, int64_t lora_rank, float lora_scale, void* dx,
                                  int dx_dtype, void* workspace, size_t workspace_bytes, int* status,
                                  moss_stream_t stream) {
  const int rc = gemm::run(true, dy, dy_dtype, m, n, k, q, scale, weight_dtype, n, k, nullptr, 0, lora_dyb, lora_a,
                           lora_a_dtype, lora_rank, lora_scale, dx, dx_dtype, workspace, workspace_bytes, status,
                           reinterpret_cast<cudaStream_t>(stream));
  return rc == MOSS_OK ? clear_ok() : rc;
}

extern "C" int moss_w8a16_gemm_dx_rotated(const void* dy, int dy_dtype, int64_t m, int64_t n, const int8_t* q,
                                          const float* scale, int weight_dtype, int64_t k, int64_t group, void* dx,
                                          int dx_dtype, void* workspace, size_t workspace_bytes, int* status,
                                          moss_stream_t stream) {
  if (group < 1 || (group & (group - 1)) != 0 || group > 8192 || (k > 0 && k % group != 0))
    return fail(MOSS_ERR_INVALID_ARGUMENT, "rotation group %lld must be a power of two <= 8192 dividing k=%lld",
                static_cast<long long>(group), static_cast<long long>(k));
  bool rotated = false;
  int rc = gemm::run(true, dy, dy_dtype, m, n, k, q, scale, weight_dtype, n, k, nullptr, 0, nullptr, nullptr, 0, 0, 1.0f,
                     dx, dx_dtype, workspace, workspace_bytes, status, reinterpret_cast<cudaStream_t>(stream), group,
                     &rotated);
  if (rc != MOSS_OK) return rc;
  if (!rotated && group > 1 && m > 0 && k > 0) rc = moss_hadamard_rotate(dx, dx_dtype, m, k, group, dx, stream);
  return rc == MOSS_OK ? clear_ok() : rc;
}

// -----------------------------------------------------------------------------------------
// Allocation-free forward GEMM (moss_w8a16_gemm_fwd_noalloc).
//
// For callers that cannot allocate device memory on this path: a host whose HBM is owned by
// another allocator (a caching pool that has already reserved the free memory, so a side
// cudaMalloc fails or makes the pool give memory back), or an FFI caller (cgo, JNI, plain
// ctypes) that has no device allocator of its own to hand out a workspace. The split-K
// scratch then lives in one fixed array compiled into this library instead of a caller
// workspace; nothing here calls cudaMalloc, cudaFree or any allocating routine.
namespace moss {
namespace gemm {

constexpr size_t kNoAllocScratchBytes = MOSS_W8A16_NOALLOC_SCRATCH_BYTES;
constexpr int kNoAllocMaxDevices = 64;

// One copy per device that loads this library, held until the process exits. In host code
// this name is only a stand-in for the device symbol, never an address: the device address
// comes from cudaGetSymbolAddress in noalloc_scratch().
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device, looked up on the first call
// per device (with that device current) and cached afterwards.
static int noalloc_scratch(void** out) {
  static std::mutex mu;
  static void* addr[kNoAllocMaxDevices] = {};
  int device = -1;
  MOSS_CUDA_TRY(cudaGetDevice(&device));
  if (device < 0 || device >= kNoAllocMaxDevices)
    return fail(MOSS_ERR_UNSUPPORTED, "device ordinal %d is beyond the %d devices the static scratch covers", device,
                kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(mu);
  if (addr[device] == nullptr) {
    void* p = nullptr;
    MOSS_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    if (p == nullptr || (reinterpret_cast<uintptr_t>(p) & 255) != 0)
      return fail(MOSS_ERR_CUDA, "static split-K scratch has no 256-byte aligned device address");
    addr[device] = p;
  }
  *out = addr[device];
  return MOSS_OK;
}

}  // namespace gemm
}  // namespace moss

extern "C" int moss_w8a16_gemm_fwd_noalloc(const void* x, int x_dtype, int64_t m, int64_t k, const int8_t* q,
                                           const float* scale, int weight_dtype, int64_t n, const void* bias,
                                           int bias_dtype, const void* lora_xa, const void* lora_b,
                                           int lora_b_dtype, int64_t lora_rank, float lora_scale, void* y,
                                           int y_dtype, int* status, moss_stream_t stream) {
  void* scratch = nullptr;
  int rc = gemm::noalloc_scratch(&scratch);
  if (rc != MOSS_OK) return rc;
  size_t need = 0;
  rc = moss_w8a16_gemm_workspace_bytes(m, n, k, &need);
  if (rc != MOSS_OK) return rc;
  if (need > gemm::kNoAllocScratchBytes && gemm::use_pair(m, n, gemm::sm_count()))
    need = 0;  // the CTA-pair kernel then runs without splitting its last round of tiles
  if (need > gemm::kNoAllocScratchBytes)
    return fail(MOSS_ERR_INVALID_ARGUMENT,
                "moss_w8a16_gemm_fwd_noalloc: m=%lld n=%lld k=%lld needs %zu bytes of split-K scratch, more than "
                "the %zu-byte static array; call moss_w8a16_gemm_fwd with a workspace instead",
                static_cast<long long>(m), static_cast<long long>(n), static_cast<long long>(k), need,
                gemm::kNoAllocScratchBytes);
  // The split-K counters are cleared on the stream inside run() before the kernel; the f32
  // partials are always written before they are read, so stale contents are harmless.
  rc = gemm::run(false, x, x_dtype, m, k, n, q, scale, weight_dtype, n, k, bias, bias_dtype, lora_xa, lora_b,
                 lora_b_dtype, lora_rank, lora_scale, y, y_dtype, need > 0 ? scratch : nullptr, need, status,
                 reinterpret_cast<cudaStream_t>(stream));
  return rc == MOSS_OK ? clear_ok() : rc;
}
