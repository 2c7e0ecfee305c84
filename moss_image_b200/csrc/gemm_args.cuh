// Launch arguments shared by the int8 GEMM kernels (1-CTA and CTA-pair variants).
#pragma once

#include <cstring>
#include <mutex>

#include "common.cuh"

namespace moss {
namespace gemm {

struct Args {
  int M, Nc, Kr;            // C[M, Nc] = A[M, Kr] * B[Kr, Nc]
  int tiles_m, tiles_n;
  int main_kb, num_kb;      // k-blocks from the int8 weight, total (incl. LoRA extension)
  int manual;               // 1: producer uses plain loads (shapes TMA cannot describe)
  const void* a; int64_t lda;
  const int8_t* w; int64_t ldw; int w_rows, w_cols;
  const float* scale;
  int w_kind;
  const void* bias; int bias_kind;
  void* out; int out_kind; int64_t ldo;
  const void* ext_a; int64_t ld_ext_a;             // LoRA: [M, r] (value dtype)
  const void* ext_b; int ext_b_kind; int64_t ld_ext_b; int ext_r;  // fwd [Nc, r]; dx [r, Nc]
  float ext_scale;
  StatusSink status;        // failure bits: the caller's device word (+ the host-visible copy)
  // Test hook (moss_debug_stall_next_gemm): the operand-swapped kernel's MMA issuer waits on a
  // barrier nothing arrives on, so its bounded wait runs out; 0 in every ordinary launch.
  int debug_stall;
  // split-K (1-CTA kernel): work units are (tile, split); split s covers weight k-blocks
  // [s * kb_per_split, (s + 1) * kb_per_split) and the last split also the LoRA blocks.
  // Partial f32 tiles go to `partial` [splits][M][Nc]; `counters` [tiles] count arrivals.
  int splits, kb_per_split;
  float* partial;
  int* counters;
  // CTA-pair kernel, last partial wave: tiles [tail_first, tiles) are split along K into
  // tail_splits units each, whose f32 partials go to `partial` [tail tile][split][256][256]
  // and are summed by a reduction kernel after the GEMM. tail_first = tiles: no split.
  int tail_first, tail_splits;
  // ConvRot grad-input (CTA-pair kernel only): rotate each output row by the grouped Hadamard
  // transform of this group size in the epilogue; 0 = no rotation.
  int rot_group;
  // CTA-pair kernel: row tiles per rasterisation group (tile_coords)
  int group_m;
};

// k-block schedule of one work unit: iteration i -> weight k-block or LoRA block.
struct UnitRange {
  int kb0, main_count, n_iter;
  __device__ __forceinline__ int kb(int i, int main_kb) const { return i < main_count ? kb0 + i : main_kb + (i - main_count); }
};
__device__ __forceinline__ UnitRange unit_range(const Args& a, int split) {
  UnitRange r;
  r.kb0 = split * a.kb_per_split;
  const int kb1 = min(a.main_kb, r.kb0 + a.kb_per_split);
  r.main_count = max(0, kb1 - r.kb0);
  r.n_iter = r.main_count + (split == a.splits - 1 ? a.num_kb - a.main_kb : 0);
  return r;
}

// ------------------------------------------------------------------ host: TMA descriptors
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Tiled tensor map of `rank` (2 or 3) dimensions: dims/box innermost first, strides in bytes
// for dimensions 1.. . Returns false (no map) when TMA cannot describe the view.
inline bool make_map_nd(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* ptr, int rank,
                        const uint64_t* dims, const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr || rank < 2 || rank > 3) return false;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0) return false;
  if ((static_cast<uint64_t>(box[0]) * esize) % 16 != 0) return false;
  cuuint64_t d[3];
  cuuint64_t st[2];
  cuuint32_t bx[3];
  cuuint32_t es[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    if (dims[i] == 0 || box[i] == 0 || box[i] > 256) return false;
    d[i] = dims[i];
    bx[i] = box[i];
  }
  for (int i = 0; i < rank - 1; ++i) {
    if (strides[i] % 16 != 0) return false;
    st[i] = strides[i];
  }
  return fn(map, dt, rank, const_cast<void*>(ptr), d, st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline bool make_map(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* ptr, uint64_t inner,
                     uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  const uint64_t dims[2] = {inner, outer};
  const uint64_t strides[1] = {row_bytes};
  const uint32_t box[2] = {box_inner, box_outer};
  return make_map_nd(map, dt, esize, ptr, 2, dims, strides, box, swz);
}

// Grouped tile rasterisation: tiles are walked in groups of kGroupM row blocks x all column
// blocks, so the tiles in flight at one time (one per CTA or CTA pair) cover a compact
// block of the output and reuse their A rows and weight columns from L2.
constexpr int kGroupM = 8;
__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& m_blk, int& n_blk,
                                            int group_m = kGroupM) {
  const int per_group = group_m * tiles_n;
  const int group = t / per_group;
  const int first_m = group * group_m;
  const int gsm = min(tiles_m - first_m, group_m);
  const int r = t - group * per_group;
  m_blk = first_m + r % gsm;
  n_blk = r / gsm;
}

// CTA-pair (cta_group::2) launcher, defined in w8a16_gemm_2sm.cu. Builds its own tensor maps;
// returns MOSS_ERR_UNSUPPORTED (without launching) when the shapes do not fit it.
int launch_pair(bool dx, int v_kind, bool fast, const Args& a, cudaStream_t stream);

// Split of the CTA-pair kernel's last partial wave (defined in w8a16_gemm_2sm.cu). When the
// 256 x 256 tiles leave the final round of the persistent grid partly empty, that round's
// tiles are cut along K so every pair gets a share; the planner depends only on the shape
// (not on a LoRA term), so the workspace query and the launch agree.
struct PairTailPlan {
  int tail_first = 0;  // first split tile (= number of tiles when nothing is split)
  int splits = 1;
  size_t partial_bytes = 0;
  size_t total() const { return splits > 1 ? partial_bytes : 0; }
};
PairTailPlan plan_pair_tail(int64_t M, int64_t Nc, int64_t Kr, int sms);

// Operand-swapped kernel (w8a16_gemm_skinny.cu): any M without a LoRA term, used when the
// CTA-pair kernel would leave SMs idle.
struct SkinnyPlan {
  bool usable = false;
  int nt = 16;                   // token tile width = MMA N (16, 32, 64, 128 or 256)
  int tiles_m = 0, tiles_n = 0;  // token tiles x 128-feature tiles
  int splits = 1;                // K splits (> 1 needs the workspace for the f32 partials)
  int kb_per_split = 0;          // weight k-blocks per split (a multiple of the stage depth)
  size_t partial_bytes = 0;
  size_t total() const { return splits > 1 ? partial_bytes : 0; }
};
SkinnyPlan plan_skinny(int64_t M, int64_t Nc, int64_t Kr, int sms);
int launch_skinny(bool dx, int v_kind, bool fast, int nt, const Args& a, cudaStream_t stream);

// Split-K epilogue shared by the few-row kernels (w8a16_gemm_skinny.cu):
// out[m, n] = round_v(sum_s partial[s, m, n] + round_v(bias[n])), splits added in order.
int launch_splitk_reduce(int v_kind, const float* partial, int splits, int M, int Nc, const void* bias, int bias_kind,
                         void* out, int out_kind, int64_t ldo, cudaStream_t stream);

// Weight-streaming kernel for at most kStreamMaxRows activation rows without a LoRA term
// (w8a16_gemm_stream.cu): 16 output features (forward) or 128 output columns (grad-input) per
// CTA, the reduction split across CTAs when those alone leave SMs idle.
constexpr int64_t kStreamMaxRows = 16;
struct StreamPlan {
  bool usable = false;
  int splits = 1;     // reduction splits (> 1 needs the workspace for the f32 partials)
  int per_split = 0;  // slabs per split
  int ctas = 0;
  size_t partial_bytes = 0;
  size_t total() const { return splits > 1 ? partial_bytes : 0; }
};
StreamPlan plan_stream(bool dx, int64_t M, int64_t Nc, int64_t Kr, int sms);
StreamPlan unsplit(StreamPlan p);  // the same plan with the reduction in one CTA per tile
int launch_stream(bool dx, int v_kind, bool fast, const Args& a, const StreamPlan& p, cudaStream_t stream);

}  // namespace gemm
}  // namespace moss
