// CTA-pair (cta_group::2) variant of the weight-only int8 GEMM for sm_100a.
//
// A cluster of two CTAs on two SMs computes one 256 x 256 output tile with 2-SM UMMAs
// (tcgen05.mma.cta_group::2, M = 256, N = 256, K = 16):
//   * each CTA TMA-loads its 128 rows of the bf16/f16 A tile into its own shared memory;
//   * each CTA TMA-loads its 128-row half of the int8 weight tile into its own shared
//     memory and its converter warps dequantise that half into the canonical SW128 layout;
//     once both halves of a stage (A rows and converted B columns) are in place they signal
//     the leader (remote mbarrier arrive through mapa);
//   * the leader's single MMA thread issues the 2-SM MMAs; the hardware reads the A rows and
//     B columns held by each CTA at the same shared-memory offsets, and each CTA's TMEM holds
//     its 128 accumulator rows; completion is committed to both CTAs (multicast commit);
//   * each CTA's epilogue warps drain their own TMEM half and release it to the leader.
// Compared with the 1-CTA kernel this halves the dequant work per SM and lowers the operand
// bytes per FLOP (each SM loads half of the int8 tile).
// The decode rounding is identical (dequant.cuh).
#include <algorithm>
#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "dequant.cuh"
#include "errors.cuh"
#include "gemm_args.cuh"

namespace moss {
namespace gemm {
namespace pair {

constexpr int BK = 64;
constexpr int kHalf = 128;  // rows of A (M) and of B (N) held by each CTA
constexpr int kTileM = 256;
constexpr int kTileN = 256;
// TMA cost on this part is dominated by a per-operation overhead (about two tensor ops in
// flight per SM), so each load stage fetches kSub k-blocks with one 3-D box per operand.
constexpr int kSub = 2;
// Separate rings: an A stage lives until the MMAs that read it retire; an int8 stage only
// until it is dequantised, so fewer int8 stages are needed. A converted entry holds the kSub
// k-blocks of one load step, so the MMA issuer waits and commits once per step rather than
// once per k-block (about 8% on the 9216 x 3072 x 3072 forward against per-k-block entries).
constexpr int kAStages = 3;
constexpr int kWStages = 2;
constexpr int kBStages = 3;
constexpr int kConvWarps = 8;
// The converter warps form kSub groups; group g dequantises k-block g of every weight stage,
// so kSub k-blocks are converted concurrently. A single group working through the k-blocks
// one at a time is bound by the latency of its per-block chain (shared loads, decode, stores,
// proxy fence, remote arrive), not by issue bandwidth.
constexpr int kGroupWarps = kConvWarps / kSub;
constexpr int kEpiWarp0 = 4;
constexpr int kConvWarp0 = 8;
constexpr int kThreads = 16 * 32;
constexpr uint32_t kABlock = kHalf * BK * 2;  // 16 KB: one k-block of this CTA's A rows
constexpr uint32_t kWBlock = kHalf * BK;      // 8 KB: one k-block of this CTA's int8 half
constexpr uint32_t kAStage = kSub * kABlock;
constexpr uint32_t kWStage = kSub * kWBlock;
constexpr uint32_t kBBytes = kHalf * BK * 2;  // 16 KB converted operand per k-block
constexpr uint32_t kBEntry = kSub * kBBytes;  // one converted entry per load step
constexpr uint32_t kTmemCols = 512;           // two 256-column accumulators
constexpr uint32_t kDataBytes = kAStages * kAStage + kWStages * kWStage + kBStages * kBEntry;
constexpr uint32_t kSmemBytes = kDataBytes + 1024 + 512;
// Last-round split (plan_pair_tail): at most this many units per tile, and only when it saves
// at least this many load steps of the tail round.
constexpr int64_t kMaxTailSplits = 16;
constexpr int64_t kMinTailGainSteps = 8;
static_assert(kSmemBytes <= 227 * 1024, "rings exceed the 227 KB of shared memory a CTA may use");
// Budget of the final wait for the peer CTA. Every other wait of either CTA is bounded: after
// a failure a role gives up its pipeline wait within kWaitBudgetCycles (or at once, when the
// abort flag is raised), and the drains of its own copies and MMAs take at most kAStages more
// budgets. The peer therefore reaches the exit barrier within about 4 budgets of any failure,
// and this wait outlasts that by a factor of two: a CTA that gives up here has a peer that can
// no longer run at all, so freeing TMEM cannot race the peer's MMAs or remote arrivals.
constexpr long long kExitBudgetCycles = 8 * kWaitBudgetCycles;

// Load schedule of one tile: main steps of up to kSub weight k-blocks, then one step per
// LoRA k-block. Every role walks the same sequence. Tiles in flight at the same time walk K
// in the same order, so the A rows and weight columns they share are read from L2 while hot.
struct Step {
  bool ext;
  int first_kb;  // weight k-block (main) or LoRA block index (ext)
  int nsub;
};
__device__ __forceinline__ Step step_of(int s, int main_kb) {
  const int main_steps = (main_kb + kSub - 1) / kSub;
  Step st;
  if (s < main_steps) {
    st.ext = false;
    st.first_kb = s * kSub;
    st.nsub = min(kSub, main_kb - st.first_kb);
  } else {
    st.ext = true;
    st.first_kb = s - main_steps;
    st.nsub = 1;
  }
  return st;
}
__device__ __forceinline__ int steps_per_tile(const Args& a) {
  return (a.main_kb + kSub - 1) / kSub + (a.num_kb - a.main_kb);
}

// Work unit of the persistent loop: whole tiles first, then the tiles of the last partial
// round, each cut into `tail_splits` ranges of load steps. Every role walks the same units.
struct Unit {
  int tile;
  int s0, s1;  // load steps [s0, s1)
  int tail;    // index among the split tiles; -1 for a whole tile
  int split;
};
__device__ __forceinline__ int units_of(const Args& a) {
  return a.tail_first + (a.tiles_m * a.tiles_n - a.tail_first) * a.tail_splits;
}
__device__ __forceinline__ Unit unit_of(const Args& a, int u, int nsteps) {
  Unit w;
  if (u < a.tail_first) {
    w.tile = u;
    w.s0 = 0;
    w.s1 = nsteps;
    w.tail = -1;
    w.split = 0;
  } else {
    const int v = u - a.tail_first;
    w.tail = v / a.tail_splits;
    w.split = v - w.tail * a.tail_splits;
    w.tile = a.tail_first + w.tail;
    w.s0 = w.split * nsteps / a.tail_splits;
    w.s1 = (w.split + 1) * nsteps / a.tail_splits;
  }
  return w;
}

__device__ __forceinline__ void tma_load_3d(uint32_t smem_dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// f32 partial of a split tile: [tail tile][split][256 tile rows][256 tile columns].
__device__ __forceinline__ float* partial_at(const Args& a, int tail, int split, int lrow, int lcol) {
  return a.partial + ((static_cast<int64_t>(tail) * a.tail_splits + split) * kTileM + lrow) * kTileN + lcol;
}

// L2 policy for the output stores: evict first. The outputs are written once and read by the
// next operation, while the A rows and weight columns are re-read by later tiles; without the
// hint a 12288-wide output streaming through L2 evicts the weight between row groups.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}
__device__ __forceinline__ void stg256_evict_first(void* p, const uint32_t (&v)[8], uint64_t policy) {
  asm volatile("st.global.L2::cache_hint.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8}, %9;" ::"l"(p), "r"(v[0]), "r"(v[1]),
               "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "l"(policy)
               : "memory");
}

// Bias (forward) and the rounded store of 32 consecutive outputs of one row.
template <bool kDX, int kV>
__device__ __forceinline__ void store_out32(const Args& args, float (&v)[32], int row, int col0, bool vec_ok) {
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
    // 64 contiguous bytes per thread as two full 32-byte sectors
    uint32_t p0[8], p1[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      p0[j] = pack2_kind<kV>(v[2 * j], v[2 * j + 1]);
      p1[j] = pack2_kind<kV>(v[16 + 2 * j], v[16 + 2 * j + 1]);
    }
    uint16_t* dst = static_cast<uint16_t*>(args.out) + off;
    const uint64_t policy = l2_evict_first_policy();
    stg256_evict_first(dst, p0, policy);
    stg256_evict_first(dst + 16, p1, policy);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (col0 + j < args.Nc) store_from_float(args.out, args.out_kind, off + j, round_to_kind(v[j], kV));
  }
}

// Finishes the split tiles of the last round: the units' f32 partials summed in split order
// (so the result does not depend on which unit ran first), plus the bias, rounded to the
// output kind. One thread per 4 consecutive columns of a tile row; a warp covers 512
// contiguous bytes of one partial row, so every load is coalesced.
template <bool kDX, int kV>
__global__ void __launch_bounds__(256) pair_tail_reduce_kernel(const Args args) {
  constexpr int kQuads = kTileN / 4;
  const int64_t total = static_cast<int64_t>(args.tiles_m * args.tiles_n - args.tail_first) * kTileM * kQuads;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int quad = static_cast<int>(i % kQuads);
    const int lrow = static_cast<int>((i / kQuads) % kTileM);
    const int tail = static_cast<int>(i / (static_cast<int64_t>(kQuads) * kTileM));
    int m_blk, n_blk;
    tile_coords(args.tail_first + tail, args.tiles_m, args.tiles_n, m_blk, n_blk, args.group_m);
    const int row = m_blk * kTileM + lrow;
    const int col = n_blk * kTileN + quad * 4;
    if (row >= args.M || col >= args.Nc) continue;
    float4 acc = __ldcg(reinterpret_cast<const float4*>(partial_at(args, tail, 0, lrow, quad * 4)));
    for (int sp = 1; sp < args.tail_splits; ++sp) {
      const float4 f = __ldcg(reinterpret_cast<const float4*>(partial_at(args, tail, sp, lrow, quad * 4)));
      acc.x += f.x;
      acc.y += f.y;
      acc.z += f.z;
      acc.w += f.w;
    }
    float v[4] = {acc.x, acc.y, acc.z, acc.w};
    if constexpr (!kDX) {
      if (args.bias != nullptr) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (col + j < args.Nc) v[j] += round_to_kind(load_as_float(args.bias, args.bias_kind, col + j), kV);
      }
    }
    const int64_t off = static_cast<int64_t>(row) * args.ldo + col;
    if (args.out_kind == kV && col + 4 <= args.Nc && (off & 3) == 0 &&
        (reinterpret_cast<uintptr_t>(args.out) & 7) == 0) {
      const uint2 p = make_uint2(pack2_kind<kV>(v[0], v[1]), pack2_kind<kV>(v[2], v[3]));
      *reinterpret_cast<uint2*>(static_cast<uint16_t*>(args.out) + off) = p;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (col + j < args.Nc) store_from_float(args.out, args.out_kind, off + j, round_to_kind(v[j], kV));
    }
  }
}

// ConvRot grad-input epilogue: the grouped Hadamard rotation (group 256 = one tile width) of
// one output row, with the arithmetic and the per-stage rounding of the standalone rotation
// kernel for 16-bit data (hadamard.cu, reference training/quant_kernels.py:231-277), so
// GEMM-then-rotate and the fused epilogue agree bit for bit: the row is first rounded to the
// compute kind (the GEMM output), every radix-4 stage (total * 0.5 - x, in f32) is rounded to it
// again. The fused path is used only when the output kind is the compute kind.
constexpr int kRotGroup = 256;
template <int kV>
__device__ __forceinline__ void rot_round_pair(float& a, float& b) {
  const uint32_t p = pack2_kind<kV>(a, b);
  if constexpr (kV == kBF16) {
    a = __uint_as_float(p << 16);
    b = __uint_as_float(p & 0xffff0000u);
  } else {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&p));
    a = f.x;
    b = f.y;
  }
}
__device__ __forceinline__ void rot_radix4(float& a, float& b, float& c, float& d) {
  const float half = __fmul_rn(__fadd_rn(__fadd_rn(__fadd_rn(a, b), c), d), 0.5f);
  const float na = __fsub_rn(half, d), nb = __fsub_rn(half, c), nc = __fsub_rn(half, b), nd = __fsub_rn(half, a);
  a = na;
  b = nb;
  c = nc;
  d = nd;
}
template <int kV, int N>
__device__ __forceinline__ void rot_round_all(float (&v)[N]) {
#pragma unroll
  for (int i = 0; i < N; i += 2) rot_round_pair<kV>(v[i], v[i + 1]);
}

// Rotates the 256 accumulator columns of this thread's TMEM row in place (radix-4 stages of
// stride 1, 4 and 16 inside each 64-column window, through registers), then applies the
// stride-64 stage on four 16-column slices at a time and stores the rounded outputs.
template <int kV>
__device__ __forceinline__ void rotate_store_row(const Args& args, uint32_t tacc, int row, int col0, bool row_ok,
                                                 bool vec_ok) {
#pragma unroll 1
  for (int w = 0; w < 4; ++w) {
    uint32_t r[64];
    tmem_ld_32x32b_x32(tacc + w * 64, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
    tmem_ld_32x32b_x32(tacc + w * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
    tmem_wait_ld();
    float v[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
    rot_round_all<kV>(v);
#pragma unroll
    for (int b = 0; b < 16; ++b) rot_radix4(v[4 * b], v[4 * b + 1], v[4 * b + 2], v[4 * b + 3]);
    rot_round_all<kV>(v);
#pragma unroll
    for (int b = 0; b < 4; ++b)
#pragma unroll
      for (int p = 0; p < 4; ++p) rot_radix4(v[16 * b + p], v[16 * b + p + 4], v[16 * b + p + 8], v[16 * b + p + 12]);
    rot_round_all<kV>(v);
#pragma unroll
    for (int p = 0; p < 16; ++p) rot_radix4(v[p], v[p + 16], v[p + 32], v[p + 48]);
    rot_round_all<kV>(v);
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      uint32_t o[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(v[16 * h + i]);
      tmem_st_32x32b_x16(tacc + w * 64 + 16 * h, o);
    }
    tmem_wait_st();
  }
#pragma unroll 1
  for (int j0 = 0; j0 < 64; j0 += 16) {
    uint32_t r[4][16];
#pragma unroll
    for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x16(tacc + c * 64 + j0, r[c]);
    tmem_wait_ld();
    uint32_t p[4][8];
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      float v0[2], v1[2], v2[2], v3[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        v0[e] = __uint_as_float(r[0][i + e]);
        v1[e] = __uint_as_float(r[1][i + e]);
        v2[e] = __uint_as_float(r[2][i + e]);
        v3[e] = __uint_as_float(r[3][i + e]);
        rot_radix4(v0[e], v1[e], v2[e], v3[e]);
      }
      p[0][i / 2] = pack2_kind<kV>(v0[0], v0[1]);
      p[1][i / 2] = pack2_kind<kV>(v1[0], v1[1]);
      p[2][i / 2] = pack2_kind<kV>(v2[0], v2[1]);
      p[3][i / 2] = pack2_kind<kV>(v3[0], v3[1]);
    }
    if (!row_ok) continue;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int64_t off = static_cast<int64_t>(row) * args.ldo + col0 + c * 64 + j0;
      uint16_t* dst = static_cast<uint16_t*>(args.out) + off;
      if (vec_ok) {
        stg256(dst, p[c]);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          dst[2 * e] = static_cast<uint16_t>(p[c][e] & 0xFFFFu);
          dst[2 * e + 1] = static_cast<uint16_t>(p[c][e] >> 16);
        }
      }
    }
  }
}

struct Barriers {
  uint64_t a_full[kAStages];   // local: this CTA's A half landed
  uint64_t a_empty[kAStages];  // local: A stage free (MMA commit)
  uint64_t w_full[kWStages];   // local: this CTA's int8 half landed
  uint64_t w_empty[kWStages];  // local: int8 stage free (local converters)
  uint64_t b_full[kBStages];   // leader: both CTAs' converted halves written (one group each)
  uint64_t b_empty[kBStages];  // local: converted stage free (MMA commit)
  uint64_t acc_full[2];        // local: accumulator ready (MMA commit)
  uint64_t acc_empty[2];       // leader: both CTAs drained the accumulator
  uint64_t drain;              // leader: all MMAs retired
  uint64_t exit_bar;           // local: peer finished
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(Barriers) <= 512, "barrier block too large");

template <bool kDX, int kV, bool kFast, bool kRot>
__global__ void __launch_bounds__(kThreads, 1)
    w8_gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_w,
                        const __grid_constant__ CUtensorMap tm_ext, const Args args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_base = smem_u32(smem_raw);
  const uint32_t base = (raw_base + 1023u) & ~1023u;
  uint8_t* const base_ptr = smem_raw + (base - raw_base);
  const uint32_t a_smem = base;
  const uint32_t w_smem = base + kAStages * kAStage;
  const uint32_t b_smem = w_smem + kWStages * kWStage;
  Barriers* bars = reinterpret_cast<Barriers*>(base_ptr + kDataBytes);
  auto bar = [&](uint64_t& b) { return smem_u32(&b); };
  volatile int* abort_flag = &bars->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair_id = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;
  const int num_units = units_of(args);
  const int nsteps = steps_per_tile(args);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(bar(bars->a_full[s]), 1);
      mbar_init(bar(bars->a_empty[s]), 1);
    }
    for (int s = 0; s < kWStages; ++s) {
      mbar_init(bar(bars->w_full[s]), 1);
      mbar_init(bar(bars->w_empty[s]), kConvWarps);
    }
    for (int s = 0; s < kBStages; ++s) {
      mbar_init(bar(bars->b_full[s]), 2 * kConvWarps);
      mbar_init(bar(bars->b_empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar(bars->acc_full[s]), 1);
      mbar_init(bar(bars->acc_empty[s]), 8);
    }
    mbar_init(bar(bars->drain), 1);
    mbar_init(bar(bars->exit_bar), 1);
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(&bars->tmem_base), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  // Both CTAs' barriers must be initialised before any cross-CTA arrival.
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_base;

  if (warp == 0 || warp == 2) {
    // ------------------------------------------------------------------ producers (both CTAs)
    // warp 0 streams the A ring, warp 2 the int8 ring; each waits only on its own ring.
    const bool a_role = warp == 0;
    if (lane == 0) {
      if (a_role) {
        tma_prefetch_desc(&tm_a);
        if (args.ext_r > 0) tma_prefetch_desc(&tm_ext);
      } else {
        tma_prefetch_desc(&tm_w);
      }
    }
    const int nst = a_role ? kAStages : kWStages;
    int stage = 0;
    uint32_t phase = 0;
    uint32_t used_mask = 0, last_phase_mask = 0;
    bool ok = true;
    for (int u = pair_id; u < num_units && ok; u += num_pairs) {
      const Unit w = unit_of(args, u, nsteps);
      int m_blk, n_blk;
      tile_coords(w.tile, args.tiles_m, args.tiles_n, m_blk, n_blk, args.group_m);
      const int m0 = m_blk * kTileM + static_cast<int>(rank) * kHalf;
      const int n0 = n_blk * kTileN + static_cast<int>(rank) * kHalf;
      for (int si = w.s0; si < w.s1; ++si) {
        const Step st = step_of(si, args.main_kb);
        const uint32_t empty_bar = a_role ? bar(bars->a_empty[stage]) : bar(bars->w_empty[stage]);
        if (!mbar_wait_cluster(empty_bar, phase ^ 1u, abort_flag, args.status, MOSS_STATUS_TIMEOUT_LOAD)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          if (a_role) {
            const uint32_t a_dst = a_smem + stage * kAStage;
            const uint32_t a_bar = bar(bars->a_full[stage]);
            if (!st.ext) {
              // one op for kSub k-blocks (chunks past K are zero-filled)
              mbar_arrive_expect_tx(a_bar, kAStage);
              tma_load_3d(a_dst, &tm_a, a_bar, 0, m0, st.first_kb);
            } else {
              mbar_arrive_expect_tx(a_bar, kABlock);
              tma_load_2d(a_dst, &tm_ext, a_bar, st.first_kb * BK, m0);
            }
          } else {
            const uint32_t w_dst = w_smem + stage * kWStage;
            const uint32_t w_bar = bar(bars->w_full[stage]);
            if (!st.ext) {
              mbar_arrive_expect_tx(w_bar, kWStage);
              if constexpr (!kDX) {
                tma_load_3d(w_dst, &tm_w, w_bar, 0, n0, st.first_kb);
              } else {
                tma_load_2d(w_dst, &tm_w, w_bar, n0, st.first_kb * BK);
              }
            } else {
              mbar_arrive(w_bar);  // LoRA block: no int8 data, keep the phase
            }
          }
          used_mask |= 1u << stage;
          last_phase_mask = (last_phase_mask & ~(1u << stage)) | (phase << stage);
        }
        __syncwarp();
        if (++stage == nst) { stage = 0; phase ^= 1u; }
      }
    }
    // Drain our own copies before leaving.
    if (lane == 0) {
      for (int s2 = 0; s2 < nst; ++s2) {
        if (!((used_mask >> s2) & 1u)) continue;
        const uint32_t ph = (last_phase_mask >> s2) & 1u;
        const uint32_t fb = a_role ? bar(bars->a_full[s2]) : bar(bars->w_full[s2]);
        const long long start = clock64();
        while (!mbar_try_wait(fb, ph)) {
          if (clock64() - start > kWaitBudgetCycles) {
            report_status(args.status, MOSS_STATUS_TIMEOUT_DRAIN);
            break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (leader)
    if (leader) {
      constexpr uint32_t idesc = umma_idesc_f16(kV == kBF16 ? 1u : 0u, kDX, kTileM, kTileN);
      int stage = 0, bstage = 0;
      uint32_t phase = 0, bphase = 0;
      int it = 0;
      bool ok = true;
      bool issued_any = false;
      for (int u = pair_id; u < num_units && ok; u += num_pairs, ++it) {
        const Unit w = unit_of(args, u, nsteps);
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait_cluster(bar(bars->acc_empty[acc]), acc_phase ^ 1u, abort_flag, args.status,
                               MOSS_STATUS_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kTileN);
        bool first = true;
        for (int si = w.s0; si < w.s1 && ok; ++si) {
          const Step st = step_of(si, args.main_kb);
          if (!mbar_wait_cluster(bar(bars->a_full[stage]), phase, abort_flag, args.status, MOSS_STATUS_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          if (!mbar_wait_cluster(bar(bars->b_full[bstage]), bphase, abort_flag, args.status,
                                 MOSS_STATUS_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int sub = 0; sub < st.nsub; ++sub) {
            if (lane == 0) {
              const uint32_t a_base = a_smem + stage * kAStage + sub * kABlock;
              const uint32_t b_base = b_smem + bstage * kBEntry + sub * kBBytes;
#pragma unroll
              for (int kk = 0; kk < BK / 16; ++kk) {
                const uint64_t adesc = umma_desc_sw128(a_base + kk * 32, 16, 1024);
                uint64_t bdesc;
                if constexpr (!kDX) {
                  bdesc = umma_desc_sw128(b_base + kk * 32, 16, 1024);
                } else {
                  bdesc = umma_desc_sw128(b_base + kk * 2048, 8192, 1024);
                }
                umma_f16_pair(d_tmem, adesc, bdesc, idesc, (first && kk == 0) ? 0u : 1u);
              }
              issued_any = true;
            }
            first = false;
          }
          if (lane == 0) umma_commit_pair_mc(bar(bars->b_empty[bstage]), 0x3);
          __syncwarp();
          if (++bstage == kBStages) { bstage = 0; bphase ^= 1u; }
          if (lane == 0) umma_commit_pair_mc(bar(bars->a_empty[stage]), 0x3);
          __syncwarp();
          if (++stage == kAStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        if (lane == 0) umma_commit_pair_mc(bar(bars->acc_full[acc]), 0x3);
        __syncwarp();
      }
      if (lane == 0 && issued_any) {
        umma_commit_pair(bar(bars->drain));
        const long long start = clock64();
        while (!mbar_try_wait(bar(bars->drain), 0)) {
          if (clock64() - start > kWaitBudgetCycles) {
            report_status(args.status, MOSS_STATUS_TIMEOUT_DRAIN);
            break;
          }
        }
      }
      __syncwarp();
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {
    // ------------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    int it = 0;
    for (int u = pair_id; u < num_units; u += num_pairs, ++it) {
      const Unit w = unit_of(args, u, nsteps);
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait_cluster(bar(bars->acc_full[acc]), acc_phase, abort_flag, args.status,
                             MOSS_STATUS_TIMEOUT_EPILOGUE))
        break;
      tc_fence_after();
      int m_blk, n_blk;
      tile_coords(w.tile, args.tiles_m, args.tiles_n, m_blk, n_blk, args.group_m);
      const int lrow = static_cast<int>(rank) * kHalf + q * 32 + lane;  // row within the tile
      const int row = m_blk * kTileM + lrow;
      const int n0 = n_blk * kTileN;
      const bool row_ok = row < args.M;
      const bool vec_ok = (args.out_kind != kF32) && ((args.ldo & 15) == 0) &&
                          ((reinterpret_cast<uintptr_t>(args.out) & 31) == 0);
      if constexpr (kRot) {
        // whole tiles only (the host disables the last-round split and needs Nc % 256 == 0)
        rotate_store_row<kV>(args, tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * kTileN),
                             row, n0, row_ok, vec_ok);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          const uint32_t eb = bar(bars->acc_empty[acc]);
          if (leader)
            mbar_arrive(eb);
          else
            mbar_arrive_cluster(mapa_shared(eb, 0));
        }
        continue;
      }
#pragma unroll 1
      for (int c = 0; c < kTileN / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                               static_cast<uint32_t>(acc * kTileN + c * 32),
                           r);
        tmem_wait_ld();
        if (c == kTileN / 32 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
            const uint32_t eb = bar(bars->acc_empty[acc]);
            if (leader)
              mbar_arrive(eb);
            else
              mbar_arrive_cluster(mapa_shared(eb, 0));
          }
        }
        const int col0 = n0 + c * 32;
        if (col0 >= args.Nc || !row_ok) continue;
        if (w.tail >= 0) {
          // split tile: this unit's f32 partial, summed by pair_tail_reduce_kernel
          float* dst = partial_at(args, w.tail, w.split, lrow, c * 32);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            uint32_t p[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) p[e] = r[8 * j + e];
            stg256(dst + 8 * j, p);
          }
          continue;
        }
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        store_out32<kDX, kV>(args, v, row, col0, vec_ok);
      }
    }
  } else if (warp >= kConvWarp0) {
    // ------------------------------------------------------------------ converters (both CTAs)
    const int group = (warp - kConvWarp0) / kGroupWarps;  // the k-block of each stage it converts
    const int gw = (warp - kConvWarp0) % kGroupWarps;
    // Conflict-free mapping: the 8 lanes of each quarter-warp cover one 128-byte operand row;
    // lane (l % 8) converts 8 codes into one 16-byte chunk. Forward task i of a thread is
    // weight row crow + 16 i; grad-input task i is reduction row crow + 16 (i % 4) of atom i / 4.
    const int crow = gw * 4 + (lane >> 3);  // 0..15
    const int cch = lane & 7;
    int stage = 0, bstage = 0, astage = 0;
    uint32_t phase = 0, bphase = 0, aphase = 0;
    bool ok = true;
    // forward: the row scales of the next tile are requested while this one is converted
    float next_scale[8];
    auto load_unit_scales = [&](int u_next) {
      if constexpr (!kDX) {
        const bool valid = u_next < num_units;
        int mb = 0, nb = 0;
        if (valid) tile_coords(unit_of(args, u_next, nsteps).tile, args.tiles_m, args.tiles_n, mb, nb, args.group_m);
        const int base_n = nb * kTileN + static_cast<int>(rank) * kHalf;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int gn = base_n + crow + 16 * i;
          next_scale[i] = (valid && gn < args.w_rows) ? __ldg(args.scale + gn) : 0.0f;
        }
      }
    };
    load_unit_scales(pair_id);
    for (int u = pair_id; u < num_units && ok; u += num_pairs) {
      const Unit w = unit_of(args, u, nsteps);
      int m_blk, n_blk;
      tile_coords(w.tile, args.tiles_m, args.tiles_n, m_blk, n_blk, args.group_m);
      const int n0 = n_blk * kTileN + static_cast<int>(rank) * kHalf;
      Dec<kV, kFast> dec_f[8];
      if constexpr (!kDX) {
#pragma unroll
        for (int i = 0; i < 8; ++i) dec_f[i].set(next_scale[i], args.w_kind);
        load_unit_scales(u + num_pairs);
      }
      for (int si = w.s0; si < w.s1 && ok; ++si) {
        const Step st = step_of(si, args.main_kb);
        // grad-input: the row scales of this group's k-block depend only on the k-block index,
        // so they are requested before the waits instead of inside the conversion chain
        float dx_scale[4];
        if constexpr (kDX) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int gn = (st.first_kb + group) * BK + crow + 16 * j;
            dx_scale[j] = (!st.ext && group < st.nsub && gn < args.w_rows) ? __ldg(args.scale + gn) : 0.0f;
          }
        }
        if (!mbar_wait(bar(bars->w_full[stage]), phase, abort_flag, args.status, MOSS_STATUS_TIMEOUT_CONVERT)) {
          ok = false;
          break;
        }
        // One converted entry per step: group g fills k-block g of it. Every converter warp of
        // both CTAs arrives on the leader's b_full, idle groups of a one-block step included.
        if (!mbar_wait_cluster(bar(bars->b_empty[bstage]), bphase ^ 1u, abort_flag, args.status,
                               MOSS_STATUS_TIMEOUT_CONVERT)) {
          ok = false;
          break;
        }
        if (group < st.nsub) {
          const int sub = group;
          const uint32_t b_base = b_smem + bstage * kBEntry + sub * kBBytes;
          uint4 o[8];
          if constexpr (!kDX) {
            // forward: K-major B half [128 n][64 k], int8 stage rows of 64 bytes
            const uint32_t w_base = w_smem + stage * kWStage + sub * kWBlock;
            if (!st.ext) {
              uint2 qv[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) qv[i] = lds64(w_base + (crow + 16 * i) * 64 + cch * 8);
#pragma unroll
              for (int i = 0; i < 8; ++i) o[i] = dec_f[i].chunk8(qv[i], args.w_kind);
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int gn = n0 + crow + 16 * i;
                o[i] = gn < args.Nc ? load8_scaled(args.ext_b, args.ext_b_kind,
                                                   static_cast<int64_t>(gn) * args.ld_ext_b, st.first_kb * BK + cch * 8,
                                                   args.ext_r, args.ext_scale, kV)
                                    : make_uint4(0, 0, 0, 0);
              }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int row = crow + 16 * i;
              sts128(b_base + (row >> 3) * 1024 + (row & 7) * 128 + (((cch ^ (row & 7)) & 7) << 4), o[i]);
            }
          } else {
            // grad-input: MN-major B half = 2 atoms x [64 n][64 k]; the int8 stage holds
            // kSub * 64 reduction rows of 128 bytes (128B swizzle).
            if (!st.ext) {
              Dec<kV, kFast> dec[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) dec[j].set(dx_scale[j], args.w_kind);
              uint2 qv[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int a = i >> 2, r = crow + 16 * (i & 3);
                const int q16 = 4 * a + (cch >> 1);
                qv[i] = lds64(w_smem + stage * kWStage + (sub * BK + r) * 128 + (((q16 ^ (r & 7)) & 7) << 4) +
                              (cch & 1) * 8);
              }
#pragma unroll
              for (int i = 0; i < 8; ++i) o[i] = dec[i & 3].chunk8(qv[i], args.w_kind);
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int a = i >> 2, r = crow + 16 * (i & 3);
                const int gj = st.first_kb * BK + r;
                o[i] = gj < args.ext_r ? load8_scaled(args.ext_b, args.ext_b_kind,
                                                      static_cast<int64_t>(gj) * args.ld_ext_b, n0 + a * 64 + cch * 8,
                                                      args.Nc, args.ext_scale, kV)
                                       : make_uint4(0, 0, 0, 0);
              }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const int a = i >> 2, r = crow + 16 * (i & 3);
              sts128(b_base + a * (kBBytes / 2) + r * 128 + (((cch ^ (r & 7)) & 7) << 4), o[i]);
            }
          }
        }
        // b_full also certifies this CTA's A rows: the leader's MMA reads both CTAs' halves
        if (group == 0 &&
            !mbar_wait(bar(bars->a_full[astage]), aphase, abort_flag, args.status, MOSS_STATUS_TIMEOUT_CONVERT)) {
          ok = false;
          break;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const uint32_t fb = bar(bars->b_full[bstage]);
          if (leader)
            mbar_arrive(fb);
          else
            mbar_arrive_cluster(mapa_shared(fb, 0));
        }
        if (++bstage == kBStages) { bstage = 0; bphase ^= 1u; }
        if (!ok) break;
        if (lane == 0) mbar_arrive(bar(bars->w_empty[stage]));
        if (++stage == kWStages) { stage = 0; phase ^= 1u; }
        if (++astage == kAStages) { astage = 0; aphase ^= 1u; }
      }
    }
  }

  // Leave together: the leader's MMAs read the peer's shared memory and write its TMEM, and
  // the peer arrives on the leader's barriers, so neither CTA may exit or free TMEM first.
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    // A failure in this CTA ends the peer's loops too (it would otherwise wait out its own
    // budgets on barriers this CTA no longer feeds). The peer is still resident: it cannot
    // pass its exit wait before the arrival below.
    if (*abort_flag) st_shared_cluster_u32(mapa_shared(smem_u32(&bars->abort_flag), rank ^ 1u), 1u);
    mbar_arrive_cluster(mapa_shared(bar(bars->exit_bar), rank ^ 1u));
    const long long start = clock64();
    while (!mbar_try_wait_cluster(bar(bars->exit_bar), 0)) {
      if (clock64() - start > kExitBudgetCycles) {
        report_status(args.status, MOSS_STATUS_TIMEOUT_DRAIN);
        break;
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

static int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

template <bool kDX, int kV, bool kFast, bool kRot = false>
static int launch_typed(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& te, const Args& a,
                        cudaStream_t stream) {
  auto kern = w8_gemm_pair_kernel<kDX, kV, kFast, kRot>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  static int max_pairs = 0;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (attr_err != cudaSuccess) return;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * (sm_count() / 2));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters <= 0) {
      cudaGetLastError();
      clusters = sm_count() / 2;
    }
    max_pairs = clusters;
  });
  MOSS_CUDA_TRY(attr_err);
  const int units = a.tail_first + (a.tiles_m * a.tiles_n - a.tail_first) * a.tail_splits;
  const int pairs = std::max(1, std::min(units, max_pairs));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  MOSS_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, ta, tw, te, a));
  if (a.tail_splits > 1) {
    const int64_t quads = static_cast<int64_t>(a.tiles_m * a.tiles_n - a.tail_first) * kTileM * (kTileN / 4);
    const int blocks = static_cast<int>(std::min<int64_t>((quads + 255) / 256, 8LL * sm_count()));
    pair_tail_reduce_kernel<kDX, kV><<<blocks, 256, 0, stream>>>(a);
    MOSS_CUDA_TRY(cudaGetLastError());
  }
  return MOSS_OK;
}

}  // namespace pair

PairTailPlan plan_pair_tail(int64_t M, int64_t Nc, int64_t Kr, int sms) {
  using namespace pair;
  PairTailPlan p;
  const int64_t tiles = ((M + kTileM - 1) / kTileM) * ((Nc + kTileN - 1) / kTileN);
  p.tail_first = static_cast<int>(std::min<int64_t>(tiles, INT32_MAX));
  const int64_t pairs = sms / 2;
  const int64_t steps = ((Kr + BK - 1) / BK + kSub - 1) / kSub;
  if (tiles <= 0 || pairs <= 0 || tiles > INT32_MAX) return p;
  const int64_t tail = tiles % pairs;
  if (tail == 0) return p;
  // As many splits as the idle pairs of the last round allow, each at least one load step.
  const int64_t splits = std::min<int64_t>(pairs / tail, std::min<int64_t>(steps, kMaxTailSplits));
  if (splits < 2) return p;
  // The split must save more load steps (about 1 us each on a 256 x 256 tile) than the
  // partials' round trip through L2 and the reduction launch cost.
  if (steps - (steps + splits - 1) / splits < kMinTailGainSteps) return p;
  p.tail_first = static_cast<int>(tiles - tail);
  p.splits = static_cast<int>(splits);
  p.partial_bytes = static_cast<size_t>(tail * splits) * kTileM * kTileN * sizeof(float);
  return p;
}

int launch_pair(bool dx, int v_kind, bool fast, const Args& a_in, cudaStream_t s) {
  using namespace pair;
  Args a = a_in;
  // Rasterisation: groups of row tiles x all column tiles. With few column tiles, a group of 8
  // rows spans more than one round of the persistent grid, and the tiles of the next round
  // stream the same A rows from DRAM again (2.9x the A bytes at K = 12288, N = 3072); a group
  // of at most one round's worth of tiles keeps each A row block within one round.
  {
    const int pairs = std::max(1, sm_count() / 2);
    a.group_m = a.tiles_n < pairs ? std::max(1, std::min(kGroupM, pairs / a.tiles_n)) : kGroupM;
  }
  // A: [M, Kr] viewed as {64, M, Kr / 64} so one box carries kSub k-blocks of 128 rows.
  if (a.Kr % BK != 0) return MOSS_ERR_UNSUPPORTED;
  const CUtensorMapDataType v_dt = v_kind == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tw, te;
  memset(&ta, 0, sizeof(ta));
  memset(&tw, 0, sizeof(tw));
  memset(&te, 0, sizeof(te));
  {
    const uint64_t dims[3] = {BK, static_cast<uint64_t>(a.M), static_cast<uint64_t>(a.Kr / BK)};
    const uint64_t strides[2] = {static_cast<uint64_t>(a.lda) * 2, BK * 2};
    const uint32_t box[3] = {BK, kHalf, kSub};
    if (!make_map_nd(&ta, v_dt, 2, a.a, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B)) return MOSS_ERR_UNSUPPORTED;
  }
  if (!dx) {
    // weight [N, K] int8 viewed as {64, N, K / 64}: [kSub][128 rows][64 B] per box
    if (a.w_cols % BK != 0) return MOSS_ERR_UNSUPPORTED;
    const uint64_t dims[3] = {BK, static_cast<uint64_t>(a.w_rows), static_cast<uint64_t>(a.w_cols / BK)};
    const uint64_t strides[2] = {static_cast<uint64_t>(a.ldw), BK};
    const uint32_t box[3] = {BK, kHalf, kSub};
    if (!make_map_nd(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.w, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE))
      return MOSS_ERR_UNSUPPORTED;
  } else {
    // weight rows are reduction indices: one box = kSub * 64 rows x 128 output columns
    if (!make_map(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.w, a.w_cols, a.w_rows, a.ldw, 128, BK * kSub,
                  CU_TENSOR_MAP_SWIZZLE_128B))
      return MOSS_ERR_UNSUPPORTED;
  }
  if (a.ext_r > 0 && !make_map(&te, v_dt, 2, a.ext_a, a.ext_r, a.M, a.ld_ext_a * 2, BK, kHalf,
                               CU_TENSOR_MAP_SWIZZLE_128B))
    return MOSS_ERR_UNSUPPORTED;
  if (a.rot_group != 0) {
    // ConvRot grad-input rotated in the epilogue: whole 256-column tiles, no last-round split
    if (!dx || a.rot_group != kRotGroup || a.Nc % kTileN != 0 || a.tail_splits != 1 || a.ext_r > 0 ||
        a.out_kind != v_kind)
      return MOSS_ERR_UNSUPPORTED;
    if (v_kind == kBF16)
      return fast ? launch_typed<true, kBF16, true, true>(ta, tw, te, a, s)
                  : launch_typed<true, kBF16, false, true>(ta, tw, te, a, s);
    return fast ? launch_typed<true, kF16, true, true>(ta, tw, te, a, s)
                : launch_typed<true, kF16, false, true>(ta, tw, te, a, s);
  }
  if (dx) {
    if (v_kind == kBF16)
      return fast ? launch_typed<true, kBF16, true>(ta, tw, te, a, s) : launch_typed<true, kBF16, false>(ta, tw, te, a, s);
    return fast ? launch_typed<true, kF16, true>(ta, tw, te, a, s) : launch_typed<true, kF16, false>(ta, tw, te, a, s);
  }
  if (v_kind == kBF16)
    return fast ? launch_typed<false, kBF16, true>(ta, tw, te, a, s) : launch_typed<false, kBF16, false>(ta, tw, te, a, s);
  return fast ? launch_typed<false, kF16, true>(ta, tw, te, a, s) : launch_typed<false, kF16, false>(ta, tw, te, a, s);
}

}  // namespace gemm
}  // namespace moss
