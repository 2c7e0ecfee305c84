// Operand-swapped ("skinny") variant of the weight-only int8 GEMM for sm_100a, used when the
// activation rows are too few for the CTA-pair kernel to occupy the GPU: adaLN modulation rows,
// small batches and decode-like calls up to a few thousand rows.
//
// With few rows the problem streams the weight: every int8 byte is used M times, so the
// time is the weight read plus its dequantisation. The 128-row tiles of the other kernels
// would spend most of each MMA on padding rows, so this kernel swaps the operands and
// computes the transposed product
//   forward:    Y^T[N, M]  = dec(W)[N, K]   * X^T[K, M]
//   grad-input: dX^T[K, M] = dec(W)^T[K, N] * dY^T[N, M]
// The dequantised weight tile is the 128-row MMA operand A (shared memory; K-major for the
// forward, MN-major for the grad-input, the same canonical layouts the CTA-pair kernel builds
// for its B operand) and a tile of kNT = 16 .. 256 activation rows is the B operand:
// tcgen05.mma M = 128, N = kNT. Each accumulator is a kNT-column slice of TMEM whose lane is the
// output feature. Per MMA flop it dequantises half as much weight as a 128-row activation tile
// with 256 features would.
//
// Work is split over (token tile, 128-feature tile) pairs and, when those are too few to occupy
// the GPU, over K: each split writes f32 partials to the caller's workspace and a second, fully
// parallel kernel adds them in split order (so the result does not depend on timing), adds the
// bias and rounds. A per-tile "last split reduces" scheme would put up to splits x 256 x 128
// partials on four warps of one CTA.
//
// Warp roles (768 threads, one CTA per SM):
//   warp 0       TMA producer of the int8 weight stages (kSub k-blocks per box)
//   warp 1       TMEM owner + single-thread MMA issuer
//   warp 2       TMA producer of the activation stages (kXSub k-blocks per box)
//   warps 4-7    epilogue, one TMEM lane quarter each
//   warps 8-23   converters: kGroups groups of 4 warps; group g dequantises k-block g of
//                every weight stage, so kGroups k-blocks are converted concurrently (one group
//                is bound by the latency of its per-block chain, not by issue bandwidth)
// Decode rounding is the shared one (dequant.cuh): dec = round_v(round_w(q * round_w(s))).
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "dequant.cuh"
#include "errors.cuh"
#include "gemm_args.cuh"

namespace moss {
namespace gemm {
namespace skinny {

constexpr int BM = 128;  // output features per tile (MMA M)
constexpr int BK = 64;
constexpr int kSub = 4;  // k-blocks per weight / activation stage
constexpr int kGroups = kSub;
constexpr int kGroupWarps = 4;
constexpr int kConvWarps = kGroups * kGroupWarps;
constexpr int kEpiWarp0 = 4;
constexpr int kConvWarp0 = 8;
constexpr int kThreads = (kConvWarp0 + kConvWarps) * 32;
constexpr uint32_t kWBlock = BM * BK;          // 8 KB of int8 per k-block (both directions)
constexpr uint32_t kWStage = kSub * kWBlock;   // 32 KB
constexpr uint32_t kCBlock = BM * BK * 2;      // 16 KB converted operand per k-block
constexpr int kMaxCStages = 7;
constexpr int kMaxWStages = 4;
constexpr int kMaxXStages = 4;

// Shared-memory budget per token-tile width: narrow tiles fetch kSub activation k-blocks per
// copy (a tensor copy costs a roughly fixed ~500 cycles), wide ones one k-block per copy.
template <int kNT>
struct Cfg {
  static constexpr int kXSub = kNT <= 64 ? kSub : 1;
  static constexpr int kWStages = kNT <= 32 ? 3 : 2;
  static constexpr int kXStages = kNT == 128 ? 4 : 2;
  // More converted stages than converter groups: a group then never waits for the MMA of its
  // own previous k-block before converting the next one.
  static constexpr int kCStages = kNT == 16 ? 7 : 6;
  static constexpr uint32_t kXBlock = kNT * BK * 2;  // one k-block of kNT activation rows
  static constexpr uint32_t kXStage = kXSub * kXBlock;
  static constexpr uint32_t kDataBytes = kWStages * kWStage + kXStages * kXStage + kCStages * kCBlock;
  static constexpr uint32_t kSmemBytes = kDataBytes + 1024 + 512;
  static constexpr uint32_t kTmemCols = 2 * kNT < 32 ? 32 : 2 * kNT;  // two accumulators
  static_assert(kSmemBytes <= 232448, "shared memory budget");
  static_assert(kWStages <= kMaxWStages && kXStages <= kMaxXStages && kCStages <= kMaxCStages, "barrier arrays");
};

struct Barriers {
  uint64_t w_full[kMaxWStages];
  uint64_t w_empty[kMaxWStages];
  uint64_t x_full[kMaxXStages];
  uint64_t x_empty[kMaxXStages];
  uint64_t c_full[kMaxCStages];
  uint64_t c_empty[kMaxCStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(Barriers) <= 512, "barrier block too large");

// Work unit u -> tile t = (token tile m_blk, feature tile n_blk), K split s, weight k-blocks
// [kb0, kb1). Token tiles vary fastest, so the tiles that share a weight tile run together
// and re-read it from L2.
struct Unit {
  int t, m_blk, n_blk, s, kb0, kb1;
};
__device__ __forceinline__ Unit unit_of(const Args& a, int u) {
  Unit r;
  r.t = u / a.splits;
  r.s = u - r.t * a.splits;
  r.n_blk = r.t / a.tiles_m;
  r.m_blk = r.t - r.n_blk * a.tiles_m;
  r.kb0 = r.s * a.kb_per_split;
  r.kb1 = min(a.main_kb, r.kb0 + a.kb_per_split);
  return r;
}

__device__ __forceinline__ void tma_load_3d(uint32_t smem_dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Store 16 token values (tokens tok0 + m0 .. tok0 + m0 + 15, those with m < `mrows`) of one
// output feature, i.e. of column `row` of the row-major output. Pairs of tokens share one packed
// conversion.
template <int kV>
__device__ __forceinline__ void store_tokens16(const Args& a, int row, const float (&v)[16], int tok0, int m0,
                                               int mrows) {
  if (a.out_kind == kV) {
    uint16_t* out = static_cast<uint16_t*>(a.out) + static_cast<int64_t>(tok0) * a.ldo + row;
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      const int m = m0 + j;
      if (m < mrows) {
        const uint32_t p = pack2_kind<kV>(v[j], v[j + 1]);
        out[static_cast<int64_t>(m) * a.ldo] = static_cast<uint16_t>(p & 0xFFFFu);
        if (m + 1 < mrows) out[static_cast<int64_t>(m + 1) * a.ldo] = static_cast<uint16_t>(p >> 16);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j)
      if (m0 + j < mrows)
        store_from_float(a.out, a.out_kind, static_cast<int64_t>(tok0 + m0 + j) * a.ldo + row, round_to_kind(v[j], kV));
  }
}

template <bool kDX, int kV, bool kFast, int kNT>
__global__ void __launch_bounds__(kThreads, 1)
    w8_gemm_skinny_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                          const Args args) {
  using C = Cfg<kNT>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* const base_ptr = smem_raw + (base - raw_base);
  const uint32_t w_smem = base;
  const uint32_t x_smem = w_smem + C::kWStages * kWStage;
  const uint32_t c_smem = x_smem + C::kXStages * C::kXStage;
  Barriers* bars = reinterpret_cast<Barriers*>(base_ptr + C::kDataBytes);
  auto bar = [&](uint64_t& b) { return smem_u32(&b); };
  volatile int* abort_flag = &bars->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_units = args.tiles_m * args.tiles_n * args.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kWStages; ++s) {
      mbar_init(bar(bars->w_full[s]), 1);
      mbar_init(bar(bars->w_empty[s]), kConvWarps);
    }
    for (int s = 0; s < C::kXStages; ++s) {
      mbar_init(bar(bars->x_full[s]), 1);
      mbar_init(bar(bars->x_empty[s]), 1);
    }
    for (int s = 0; s < C::kCStages; ++s) {
      mbar_init(bar(bars->c_full[s]), kGroupWarps);
      mbar_init(bar(bars->c_empty[s]), 1);
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
    tmem_alloc(smem_u32(&bars->tmem_base), C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp == 0 || warp == 2) {
    // ------------------------------------------------------------------ producers
    // warp 0 streams the int8 weight ring, warp 2 the activation ring.
    const bool w_role = warp == 0;
    const int nst = w_role ? C::kWStages : C::kXStages;
    const int per = w_role ? kSub : C::kXSub;  // k-blocks per copy
    if (lane == 0) tma_prefetch_desc(w_role ? &tm_w : &tm_x);
    int stage = 0;
    uint32_t phase = 0;
    uint32_t used_mask = 0, last_phase_mask = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
      const Unit U = unit_of(args, u);
      for (int kb = U.kb0; kb < U.kb1; kb += per) {
        const uint32_t empty_bar = w_role ? bar(bars->w_empty[stage]) : bar(bars->x_empty[stage]);
        if (!mbar_wait(empty_bar, phase ^ 1u, abort_flag, args.status, MOSS_STATUS_TIMEOUT_LOAD)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          if (w_role) {
            const uint32_t dst = w_smem + stage * kWStage;
            const uint32_t fb = bar(bars->w_full[stage]);
            mbar_arrive_expect_tx(fb, kWStage);
            if constexpr (!kDX) {
              tma_load_3d(dst, &tm_w, fb, 0, U.n_blk * BM, kb);  // [kSub][128 rows][64 B]
            } else {
              tma_load_2d(dst, &tm_w, fb, U.n_blk * BM, kb * BK);  // [kSub * 64 rows][128 B], 128B swizzle
            }
          } else {
            const uint32_t dst = x_smem + stage * C::kXStage;
            const uint32_t fb = bar(bars->x_full[stage]);
            mbar_arrive_expect_tx(fb, C::kXStage);
            tma_load_3d(dst, &tm_x, fb, 0, U.m_blk * kNT, kb);  // [kXSub][kNT rows][128 B], rows past M zero
          }
          used_mask |= 1u << stage;
          last_phase_mask = (last_phase_mask & ~(1u << stage)) | (phase << stage);
        }
        __syncwarp();
        if (++stage == nst) { stage = 0; phase ^= 1u; }
      }
    }
    // Drain: never leave with our own TMA copies still writing into shared memory.
    if (lane == 0) {
      for (int s = 0; s < nst; ++s) {
        if (!((used_mask >> s) & 1u)) continue;
        const uint32_t fb = w_role ? bar(bars->w_full[s]) : bar(bars->x_full[s]);
        const long long start = clock64();
        while (!mbar_try_wait(fb, (last_phase_mask >> s) & 1u)) {
          if (clock64() - start > kWaitBudgetCycles) {
            report_status(args.status, MOSS_STATUS_TIMEOUT_DRAIN);
            break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = umma_idesc_f16_ab(kV == kBF16 ? 1u : 0u, kDX, false, BM, kNT);
    int xstage = 0, cstage = 0;
    uint32_t xphase = 0, cphase = 0;
    int it = 0;
    bool ok = true;
    bool issued_any = false;
    if (args.debug_stall) {
      // Test hook (moss_debug_stall_next_gemm): nothing arrives on the drain barrier before an
      // MMA is issued, so this bounded wait runs out, raises the abort flag and reports
      // MOSS_STATUS_TIMEOUT_MMA; every role then leaves and the copies in flight are drained.
      mbar_wait(bar(bars->drain), 0, abort_flag, args.status, MOSS_STATUS_TIMEOUT_MMA);
      ok = false;
    }
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++it) {
      const Unit U = unit_of(args, u);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(bar(bars->acc_empty[acc]), acc_phase ^ 1u, abort_flag, args.status, MOSS_STATUS_TIMEOUT_MMA)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kNT);
      bool first = true;
      for (int kb = U.kb0; kb < U.kb1 && ok; ++kb) {
        const int xsub = (kb - U.kb0) % C::kXSub;  // position in the activation stage
        if (xsub == 0 &&
            !mbar_wait(bar(bars->x_full[xstage]), xphase, abort_flag, args.status, MOSS_STATUS_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        if (!mbar_wait(bar(bars->c_full[cstage]), cphase, abort_flag, args.status, MOSS_STATUS_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t c_base = c_smem + cstage * kCBlock;
          const uint32_t x_base = x_smem + xstage * C::kXStage + xsub * C::kXBlock;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            uint64_t adesc;
            if constexpr (!kDX) {
              adesc = umma_desc_sw128(c_base + kk * 32, 16, 1024);
            } else {
              adesc = umma_desc_sw128(c_base + kk * 2048, 8192, 1024);
            }
            const uint64_t bdesc = umma_desc_sw128(x_base + kk * 32, 16, 1024);
            umma_f16(d_tmem, adesc, bdesc, idesc, (first && kk == 0) ? 0u : 1u);
          }
          umma_commit(bar(bars->c_empty[cstage]));
          issued_any = true;
        }
        first = false;
        __syncwarp();
        if (++cstage == C::kCStages) { cstage = 0; cphase ^= 1u; }
        if (xsub == C::kXSub - 1 || kb == U.kb1 - 1) {
          if (lane == 0) umma_commit(bar(bars->x_empty[xstage]));
          __syncwarp();
          if (++xstage == C::kXStages) { xstage = 0; xphase ^= 1u; }
        }
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
      const Unit U = unit_of(args, u);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(bar(bars->acc_full[acc]), acc_phase, abort_flag, args.status, MOSS_STATUS_TIMEOUT_EPILOGUE))
        break;
      tc_fence_after();
      const int row = U.n_blk * BM + q * 32 + lane;  // output feature
      const int tok0 = U.m_blk * kNT;                // first token (activation row) of the tile
      const int mrows = min(kNT, args.M - tok0);
      const bool row_ok = row < args.Nc;
      float b = 0.0f;
      if constexpr (!kDX) {
        if (args.bias != nullptr && row_ok) b = round_to_kind(load_as_float(args.bias, args.bias_kind, row), kV);
      }
      // 16 token columns at a time; the accumulator is released after the last TMEM load
#pragma unroll 1
      for (int j = 0; j < kNT / 16; ++j) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * kNT + 16 * j), r);
        tmem_wait_ld();
        if (j == kNT / 16 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar(bars->acc_empty[acc]));
        }
        if (!row_ok || 16 * j >= mrows) continue;
        if (args.splits == 1) {
          float v[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]) + b;
          store_tokens16<kV>(args, row, v, tok0, 16 * j, mrows);
        } else {
          // partial f32 sums of this split, [split][M][Nc]; lanes write consecutive features
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (16 * j + i < mrows)
              args.partial[(static_cast<int64_t>(U.s) * args.M + tok0 + 16 * j + i) * args.Nc + row] = __uint_as_float(r[i]);
        }
      }
    }
  } else if (warp >= kConvWarp0) {
    // ------------------------------------------------------------------ converters
    const int group = (warp - kConvWarp0) / kGroupWarps;  // the k-block of each stage it converts
    const int gw = (warp - kConvWarp0) % kGroupWarps;
    // Conflict-free mapping: the 8 lanes of each quarter-warp cover one 128-byte operand row;
    // lane (l % 8) converts 8 codes into one 16-byte chunk. Forward task i of a thread is
    // weight row crow + 16 i; grad-input task i is reduction row crow + 16 (i % 4) of atom i / 4.
    const int crow = gw * 4 + (lane >> 3);  // 0..15
    const int cch = lane & 7;
    int stage = 0, cstage = 0;
    uint32_t phase = 0, cphase = 0;
    bool ok = true;
    // forward: the row scales of the next unit are requested while this one is converted
    float next_scale[8];
    auto load_unit_scales = [&](int u_next) {
      if constexpr (!kDX) {
        const int base_n = u_next < num_units ? unit_of(args, u_next).n_blk * BM : 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int gn = base_n + crow + 16 * i;
          next_scale[i] = (u_next < num_units && gn < args.w_rows) ? __ldg(args.scale + gn) : 0.0f;
        }
      }
    };
    load_unit_scales(blockIdx.x);
    for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
      const Unit U = unit_of(args, u);
      Dec<kV, kFast> dec_f[8];
      if constexpr (!kDX) {
#pragma unroll
        for (int i = 0; i < 8; ++i) dec_f[i].set(next_scale[i], args.w_kind);
        load_unit_scales(u + gridDim.x);
      }
      for (int kb = U.kb0; kb < U.kb1 && ok; kb += kSub) {
        const int nsub = min(kSub, U.kb1 - kb);
        // grad-input: request this group's row scales before the waits (they depend only on
        // the k-block index), not inside the conversion chain
        float dx_scale[4];
        if constexpr (kDX) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int gn = (kb + group) * BK + crow + 16 * j;
            dx_scale[j] = (group < nsub && gn < args.w_rows) ? __ldg(args.scale + gn) : 0.0f;
          }
        }
        if (!mbar_wait(bar(bars->w_full[stage]), phase, abort_flag, args.status, MOSS_STATUS_TIMEOUT_CONVERT)) {
          ok = false;
          break;
        }
        // Each warp releases the int8 stage as soon as its k-block is in registers, so the
        // producer refills it while the decode, stores and fence are still running; warps with
        // no k-block in a short final stage release it after the stage has landed.
        bool released = false;
        for (int sub = 0; sub < nsub; ++sub) {
          if (sub == group) {
            if (!mbar_wait(bar(bars->c_empty[cstage]), cphase ^ 1u, abort_flag, args.status,
                           MOSS_STATUS_TIMEOUT_CONVERT)) {
              ok = false;
              break;
            }
            const uint32_t c_base = c_smem + cstage * kCBlock;
            const uint32_t w_base = w_smem + stage * kWStage;
            uint4 o[8];
            if constexpr (!kDX) {
              // forward: K-major A [128 features][64 k]; the stage holds [kSub][128 rows][64 B]
              uint2 qv[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) qv[i] = lds64(w_base + sub * kWBlock + (crow + 16 * i) * 64 + cch * 8);
              __syncwarp();
              if (lane == 0) mbar_arrive(bar(bars->w_empty[stage]));  // int8 bytes are in registers
              released = true;
#pragma unroll
              for (int i = 0; i < 8; ++i) o[i] = dec_f[i].chunk8(qv[i], args.w_kind);
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int row = crow + 16 * i;
                sts128(c_base + (row >> 3) * 1024 + (row & 7) * 128 + (((cch ^ (row & 7)) & 7) << 4), o[i]);
              }
            } else {
              // grad-input: MN-major A = 2 atoms x [64 reduction rows][64 output features];
              // the stage holds kSub * 64 reduction rows of 128 bytes (128B swizzle).
              Dec<kV, kFast> dec[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) dec[j].set(dx_scale[j], args.w_kind);
              uint2 qv[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int a = i >> 2, r = crow + 16 * (i & 3);
                const int q16 = 4 * a + (cch >> 1);
                qv[i] = lds64(w_base + (sub * BK + r) * 128 + (((q16 ^ (r & 7)) & 7) << 4) + (cch & 1) * 8);
              }
              __syncwarp();
              if (lane == 0) mbar_arrive(bar(bars->w_empty[stage]));  // int8 bytes are in registers
              released = true;
#pragma unroll
              for (int i = 0; i < 8; ++i) o[i] = dec[i & 3].chunk8(qv[i], args.w_kind);
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int a = i >> 2, r = crow + 16 * (i & 3);
                sts128(c_base + a * (kCBlock / 2) + r * 128 + (((cch ^ (r & 7)) & 7) << 4), o[i]);
              }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(bars->c_full[cstage]));
          }
          // every group walks every converted stage, so the ring positions stay in step
          if (++cstage == C::kCStages) { cstage = 0; cphase ^= 1u; }
        }
        if (!ok) break;
        if (!released && lane == 0) mbar_arrive(bar(bars->w_empty[stage]));
        if (++stage == C::kWStages) { stage = 0; phase ^= 1u; }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// Split-K epilogue: out[m, n] = round_v(sum_s partial[s, m, n] + round_v(bias[n])), the splits
// added in order. A thread produces 8 consecutive features of one row: two 16-byte loads per
// split and one 16-byte store, so every access is coalesced.
template <int kV>
__global__ void __launch_bounds__(256)
    splitk_reduce_kernel(const float* __restrict__ partial, int splits, int M, int Nc, const void* bias, int bias_kind,
                         void* out, int out_kind, int64_t ldo) {
  const int groups = (Nc + 7) / 8;
  const int64_t total = static_cast<int64_t>(M) * groups;
  const int64_t split_stride = static_cast<int64_t>(M) * Nc;
  const bool vec_in = (Nc & 3) == 0;  // rows of 16-byte aligned float4s (the workspace is 256-byte aligned)
  const bool vec_out = out_kind == kV && (ldo & 7) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int m = static_cast<int>(i / groups);
    const int n0 = static_cast<int>(i - static_cast<int64_t>(m) * groups) * 8;
    const bool full = n0 + 8 <= Nc;
    const float* src = partial + static_cast<int64_t>(m) * Nc + n0;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = 0.0f;
    if (full && vec_in) {
#pragma unroll 4
      for (int sp = 0; sp < splits; ++sp) {
        const float4 a = __ldcs(reinterpret_cast<const float4*>(src + sp * split_stride));
        const float4 b = __ldcs(reinterpret_cast<const float4*>(src + sp * split_stride) + 1);
        v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w;
        v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
      }
    } else {
      for (int sp = 0; sp < splits; ++sp) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (n0 + j < Nc) v[j] += __ldcs(src + sp * split_stride + j);
      }
    }
    if (bias != nullptr) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (n0 + j < Nc) v[j] += round_to_kind(load_as_float(bias, bias_kind, n0 + j), kV);
    }
    const int64_t off = static_cast<int64_t>(m) * ldo + n0;
    if (full && vec_out) {
      const uint4 o = make_uint4(pack2_kind<kV>(v[0], v[1]), pack2_kind<kV>(v[2], v[3]), pack2_kind<kV>(v[4], v[5]),
                                 pack2_kind<kV>(v[6], v[7]));
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + off) = o;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (n0 + j < Nc) store_from_float(out, out_kind, off + j, round_to_kind(v[j], kV));
    }
  }
}

static int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

template <bool kDX, int kV, bool kFast, int kNT>
static int launch_typed(const CUtensorMap& tx, const CUtensorMap& tw, const Args& a, cudaStream_t stream) {
  using C = Cfg<kNT>;
  auto kern = w8_gemm_skinny_kernel<kDX, kV, kFast, kNT>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] { attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes); });
  MOSS_CUDA_TRY(attr_err);
  const int units = a.tiles_m * a.tiles_n * a.splits;
  const unsigned grid = static_cast<unsigned>(std::max(1, std::min(units, sm_count())));
  kern<<<grid, kThreads, C::kSmemBytes, stream>>>(tx, tw, a);
  MOSS_CUDA_TRY(cudaGetLastError());
  if (a.splits > 1) {
    const int64_t total = static_cast<int64_t>(a.M) * ((a.Nc + 7) / 8);
    const unsigned rgrid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, 8 * sm_count())));
    splitk_reduce_kernel<kV><<<rgrid, 256, 0, stream>>>(a.partial, a.splits, a.M, a.Nc, kDX ? nullptr : a.bias, a.bias_kind,
                                                        a.out, a.out_kind, a.ldo);
    MOSS_CUDA_TRY(cudaGetLastError());
  }
  return MOSS_OK;
}

template <bool kDX, int kV, bool kFast>
static int launch_nt(int nt, const CUtensorMap& tx, const CUtensorMap& tw, const Args& a, cudaStream_t s) {
  switch (nt) {
    case 16: return launch_typed<kDX, kV, kFast, 16>(tx, tw, a, s);
    case 32: return launch_typed<kDX, kV, kFast, 32>(tx, tw, a, s);
    case 64: return launch_typed<kDX, kV, kFast, 64>(tx, tw, a, s);
    case 128: return launch_typed<kDX, kV, kFast, 128>(tx, tw, a, s);
    default: return launch_typed<kDX, kV, kFast, 256>(tx, tw, a, s);
  }
}

}  // namespace skinny

int launch_splitk_reduce(int v_kind, const float* partial, int splits, int M, int Nc, const void* bias, int bias_kind,
                         void* out, int out_kind, int64_t ldo, cudaStream_t stream) {
  const int64_t total = static_cast<int64_t>(M) * ((Nc + 7) / 8);
  const unsigned grid =
      static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, 8 * skinny::sm_count())));
  if (v_kind == kBF16)
    skinny::splitk_reduce_kernel<kBF16><<<grid, 256, 0, stream>>>(partial, splits, M, Nc, bias, bias_kind, out, out_kind, ldo);
  else
    skinny::splitk_reduce_kernel<kF16><<<grid, 256, 0, stream>>>(partial, splits, M, Nc, bias, bias_kind, out, out_kind, ldo);
  MOSS_CUDA_TRY(cudaGetLastError());
  return MOSS_OK;
}

SkinnyPlan plan_skinny(int64_t M, int64_t Nc, int64_t Kr, int sms) {
  using namespace skinny;
  SkinnyPlan p;
  if (M <= 0 || Nc <= 0 || Kr <= 0 || M > INT32_MAX) return p;
  const int64_t tiles_n = (Nc + BM - 1) / BM;
  const int64_t main_kb = (Kr + BK - 1) / BK;
  if (((M + 15) / 16) * tiles_n > INT32_MAX / 64) return p;
  // Token tile and K split from a time model fitted to B200 measurements of this kernel (both
  // directions, 3072-18432 wide weights, 16-1024 tokens, single launches on a cold L2; median
  // error 2-3%): each wave of CTAs costs kb x 0.43 us per k-block for token tiles up to 128
  // (0.66 us at 256, whose MMA takes longer than the conversion), and a split adds ~4 us
  // for the reduction launch plus its f32 partials written and read back at ~5.5 TB/s.
  // Everything else (launch, pipeline fill, the cold weight stream) is the same for every
  // choice and left out.
  double best = -1.0;
  for (int nt : {16, 32, 64, 128, 256}) {
    if (nt > 16 && nt / 2 >= M) continue;  // a tile at least twice the token count buys nothing
    const double t_kb = nt == 256 ? 0.66 : 0.43;
    const int64_t tiles = ((M + nt - 1) / nt) * tiles_n;
    const int64_t max_splits = std::min<int64_t>((main_kb + kSub - 1) / kSub, 64);
    for (int64_t want = 1; want <= std::max<int64_t>(max_splits, 1); ++want) {
      int64_t kps = main_kb, splits = 1;
      if (want > 1) {
        kps = (main_kb + want - 1) / want;
        kps = (kps + kSub - 1) / kSub * kSub;
        splits = (main_kb + kps - 1) / kps;
        if (splits != want) continue;
      }
      const int64_t waves = (tiles * splits + sms - 1) / sms;
      double cost = static_cast<double>(waves * kps) * t_kb;
      if (splits > 1) cost += 4.0 + 0.18 * 2.0 * static_cast<double>(splits) * M * Nc * 4.0 / 1.0e6;
      if (best < 0.0 || cost < best - 1e-9) {
        best = cost;
        p.nt = nt;
        p.tiles_m = static_cast<int>((M + nt - 1) / nt);
        p.splits = static_cast<int>(splits);
        p.kb_per_split = static_cast<int>(kps);
      }
    }
  }
  p.usable = true;
  p.tiles_n = static_cast<int>(tiles_n);
  p.partial_bytes = p.splits > 1 ? (static_cast<size_t>(p.splits) * M * Nc * 4 + 255) / 256 * 256 : 0;
  return p;
}

int launch_skinny(bool dx, int v_kind, bool fast, int nt, const Args& a, cudaStream_t s) {
  using namespace skinny;
  if (a.Kr % BK != 0 || a.ext_r > 0) return MOSS_ERR_UNSUPPORTED;
  const CUtensorMapDataType v_dt = v_kind == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap tx, tw;
  memset(&tx, 0, sizeof(tx));
  memset(&tw, 0, sizeof(tw));
  {
    // activations [M, Kr] viewed as {64, M, Kr / 64}: one box = kSub (nt <= 64) or 1 k-blocks of nt rows
    const uint64_t dims[3] = {BK, static_cast<uint64_t>(a.M), static_cast<uint64_t>(a.Kr / BK)};
    const uint64_t strides[2] = {static_cast<uint64_t>(a.lda) * 2, BK * 2};
    const uint32_t box[3] = {BK, static_cast<uint32_t>(nt), nt <= 64 ? static_cast<uint32_t>(kSub) : 1u};
    if (!make_map_nd(&tx, v_dt, 2, a.a, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return MOSS_ERR_UNSUPPORTED;
  }
  if (!dx) {
    // weight [N, K] int8 viewed as {64, N, K / 64}: [kSub][128 rows][64 B] per box
    if (a.w_cols % BK != 0) return MOSS_ERR_UNSUPPORTED;
    const uint64_t dims[3] = {BK, static_cast<uint64_t>(a.w_rows), static_cast<uint64_t>(a.w_cols / BK)};
    const uint64_t strides[2] = {static_cast<uint64_t>(a.ldw), BK};
    const uint32_t box[3] = {BK, BM, kSub};
    if (!make_map_nd(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.w, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE))
      return MOSS_ERR_UNSUPPORTED;
  } else {
    // weight rows are reduction indices: one box = kSub * 64 rows x 128 output features
    if (!make_map(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.w, a.w_cols, a.w_rows, a.ldw, BM, BK * kSub,
                  CU_TENSOR_MAP_SWIZZLE_128B))
      return MOSS_ERR_UNSUPPORTED;
  }
  if (dx) {
    if (v_kind == kBF16) return fast ? launch_nt<true, kBF16, true>(nt, tx, tw, a, s) : launch_nt<true, kBF16, false>(nt, tx, tw, a, s);
    return fast ? launch_nt<true, kF16, true>(nt, tx, tw, a, s) : launch_nt<true, kF16, false>(nt, tx, tw, a, s);
  }
  if (v_kind == kBF16) return fast ? launch_nt<false, kBF16, true>(nt, tx, tw, a, s) : launch_nt<false, kBF16, false>(nt, tx, tw, a, s);
  return fast ? launch_nt<false, kF16, true>(nt, tx, tw, a, s) : launch_nt<false, kF16, false>(nt, tx, tw, a, s);
}

}  // namespace gemm
}  // namespace moss
