// C ABI of the B200 fused FFN (declarations and reference citations in include/ffn_b200.h).
//
// Host responsibilities, all without device allocation:
//   * planning   -- tile shape, swap-AB choice, Stream-K split, scratch sizes
//                   (reference: ops/host/tiling.py:58-74, ops/host/dispatch.py:42-66);
//   * preparing  -- device / block_num checks and TMA tensor-map encoding
//                   (reference: ops/api.py:48-89, ops/host/dispatch.py:97-116);
//   * running    -- one cooperative launch of the persistent fused kernel per call
//                   (reference: ops/api.py:37-45).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>

#include "../../include/ffn_b200.h"
#include "ffn_kernel.cuh"
#include "ffn_rowblock.cuh"
#include "ffn_hslice.cuh"

namespace ffnb200 {
const int32_t* internal_pair_owner_map(int device, int grid, int smem);  // ffn_placement.cu
}  // namespace ffnb200

namespace {

using ffnb200::Params;
using ffnb200::PhaseSched;
using KernelFn = void (*)(const Params);

struct Variant {
  int bn, stages;
  bool swap, pair;
  int ksub;       // 64-wide K sub-blocks per pipeline stage
  int epi;        // epilogue warps (4, or 8 = two per TMEM sub-partition for short tiles)
  bool rowblock;  // hidden-resident row-block kernel (down_impl full_load_a); bn = Y width
  bool w8;        // fp8 weights widened on chip by 4 converter warps (decode tiles)
  int hslice;     // hidden-slice decode kernel: cluster size (CTAs sharing a hidden super-block)
};
// 0: prefill tiles 128x256 (one CTA), 1: 128x128 for small grids, 2/3: swap-AB decode
// tiles (16 / 64 tokens), 4: prefill tiles 256x256 computed by a CTA pair (cta_group::2),
// 5/6: swap-AB decode tiles with 256/128-wide K stages (longer contiguous weight reads),
// 7/8/9: hidden-resident row blocks with a 64/128/256-column Y accumulator,
// 10/11: swap-AB decode tiles (16 / 64 tokens) with fp8 weights, 12: hidden-slice decode
// (16 tokens; clusters of 2, 4 or 8 CTAs -- the plan's row_split -- each CTA owning 128
// hidden rows, ffn_hslice.cuh).
constexpr int kSliceVariant = 12;
constexpr Variant kVariants[] = {
    {256, 4, false, false, 1, 4, false, false}, {128, 4, false, false, 1, 8, false, false},
    {16, 8, true, false, 1, 8, false, false},   {64, 8, true, false, 1, 8, false, false},
    {256, 6, false, true, 1, 4, false, false},  {16, 3, true, false, 4, 8, false, false},
    {64, 4, true, false, 2, 8, false, false},   {64, 4, false, false, 1, 16, true, false},
    {128, 4, false, false, 1, 16, true, false}, {256, 4, false, false, 1, 16, true, false},
    {16, 6, true, false, 2, 8, false, true},    {64, 4, true, false, 2, 8, false, true},
    {16, ffnb200::SliceLayout<4>::kStages, true, false, 1, 4, false, false, 4}};
constexpr int kNumVariants = 13;
constexpr int kFirstRowblock = 7;

template <int BN, int ST, bool SW, bool PR, int KS, int EP, bool W8, bool B16>
KernelFn pick_kernel_act(int act) {
  using namespace ffnb200;
  if (act == 3) return ffn_fused_kernel<BN, ST, SW, PR, KS, EP, B16, 3, W8>;
  if (act == 2) return ffn_fused_kernel<BN, ST, SW, PR, KS, EP, B16, 2, W8>;
  if (act == 1) return ffn_fused_kernel<BN, ST, SW, PR, KS, EP, B16, 1, W8>;
  return ffn_fused_kernel<BN, ST, SW, PR, KS, EP, B16, 0, W8>;
}
template <int BN, int ST, bool SW, bool PR, int KS, int EP, bool W8>
KernelFn pick_kernel(int bf16, int act) {
  return bf16 ? pick_kernel_act<BN, ST, SW, PR, KS, EP, W8, true>(act) : pick_kernel_act<BN, ST, SW, PR, KS, EP, W8, false>(act);
}
#define FFN_B200_VARIANTS(X)                  \
  X(0, 256, 4, false, false, 1, 4, false)     \
  X(1, 128, 4, false, false, 1, 8, false)     \
  X(2, 16, 8, true, false, 1, 8, false)       \
  X(3, 64, 8, true, false, 1, 8, false)       \
  X(4, 256, 6, false, true, 1, 4, false)      \
  X(5, 16, 3, true, false, 4, 8, false)       \
  X(6, 64, 4, true, false, 2, 8, false)       \
  X(10, 16, 6, true, false, 2, 8, true)       \
  X(11, 64, 4, true, false, 2, 8, true)
template <int NY>
KernelFn pick_rowblock(int bf16, int act) {
  using namespace ffnb200;
  if (bf16) {
    if (act == 3) return ffn_rowblock_kernel<NY, 4, true, 3>;
    return act == 2 ? ffn_rowblock_kernel<NY, 4, true, 2>
                    : (act == 1 ? ffn_rowblock_kernel<NY, 4, true, 1> : ffn_rowblock_kernel<NY, 4, true, 0>);
  }
  if (act == 3) return ffn_rowblock_kernel<NY, 4, false, 3>;
  return act == 2 ? ffn_rowblock_kernel<NY, 4, false, 2>
                  : (act == 1 ? ffn_rowblock_kernel<NY, 4, false, 1> : ffn_rowblock_kernel<NY, 4, false, 0>);
}
template <int S>
KernelFn pick_hslice_s(int bf16, int act) {
  using namespace ffnb200;
  if (bf16) {
    return act == 2 ? ffn_hslice_kernel<S, true, 2>
                    : (act == 1 ? ffn_hslice_kernel<S, true, 1> : ffn_hslice_kernel<S, true, 0>);
  }
  return act == 2 ? ffn_hslice_kernel<S, false, 2>
                  : (act == 1 ? ffn_hslice_kernel<S, false, 1> : ffn_hslice_kernel<S, false, 0>);
}
// Hidden-slice kernels by cluster size S (the plan's row_split); SwiGLU has none.
KernelFn pick_hslice(int S, int bf16, int act) {
  if (act == FFN_B200_SWIGLU) return nullptr;
  return S == 8 ? pick_hslice_s<8>(bf16, act) : (S == 4 ? pick_hslice_s<4>(bf16, act) : pick_hslice_s<2>(bf16, act));
}
int hslice_smem(int S) {
  return S == 8 ? ffnb200::SliceLayout<8>::kSmem
                : (S == 4 ? ffnb200::SliceLayout<4>::kSmem : ffnb200::SliceLayout<2>::kSmem);
}
int hslice_ring_bytes(int S) {
  return S == 8 ? ffnb200::SliceLayout<8>::kStages * ffnb200::SliceLayout<8>::kStage
                : (S == 4 ? ffnb200::SliceLayout<4>::kStages * ffnb200::SliceLayout<4>::kStage
                          : ffnb200::SliceLayout<2>::kStages * ffnb200::SliceLayout<2>::kStage);
}
KernelFn kernel_for(int variant, int bf16, int gelu) {
  switch (variant) {
#define X(id, bn, st, sw, pr, ks, ep, w8) \
  case id: return pick_kernel<bn, st, sw, pr, ks, ep, w8>(bf16, gelu);
    FFN_B200_VARIANTS(X)
#undef X
    case 7: return pick_rowblock<64>(bf16, gelu);
    case 8: return pick_rowblock<128>(bf16, gelu);
    case 9: return pick_rowblock<256>(bf16, gelu);
    case kSliceVariant: return pick_hslice(kVariants[kSliceVariant].hslice, bf16, gelu);
  }
  return nullptr;
}
int smem_for(int variant) {
  switch (variant) {
#define X(id, bn, st, sw, pr, ks, ep, w8) \
  case id: return ffnb200::Layout<bn, st, sw, pr, ks, ep, w8>::kSmem;
    FFN_B200_VARIANTS(X)
#undef X
    case 7: return ffnb200::RowLayout<64, 4>::kSmem;
    case 8: return ffnb200::RowLayout<128, 4>::kSmem;
    case 9: return ffnb200::RowLayout<256, 4>::kSmem;
    case kSliceVariant: return hslice_smem(kVariants[kSliceVariant].hslice);
  }
  return 0;
}
int threads_for(int variant) {
  return ffnb200::kCtrlThreads + 32 * (kVariants[variant].epi + (kVariants[variant].w8 ? 12 : 0));
}
int tmem_cols_for(int variant) {
  switch (variant) {
#define X(id, bn, st, sw, pr, ks, ep, w8) \
  case id: return ffnb200::Layout<bn, st, sw, pr, ks, ep, w8>::kTmemCols;
    FFN_B200_VARIANTS(X)
#undef X
  }
  return 512;  // row-block and hidden-slice variants
}

int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

constexpr int kMinSplitKBlocks = 32;  // see make_plan: the up phase splits only tiles this long
constexpr int kMinSegment = 16;       // minimum K steps of one CTA's Stream-K share

struct PhaseInput {
  int64_t rows, cols, depth;
};

// Fills one phase's schedule.  split=true applies the Stream-K tail split of the reference
// (ops/kernel/ffn.py:642-665): sk = T mod C tail tiles, their sk*L k-blocks spread as
// q = floor(sk*L / C) per CTA with the first (sk*L mod C) CTAs taking one more.
int phase_plan(const PhaseInput& in, int tile_m, int bn, int tile_k, int C, bool split, int group,
               ffn_b200_phase_plan* out) {
  const int64_t tr = cdiv(in.rows, tile_m);
  const int64_t tq = cdiv(in.cols, bn);
  const int64_t T = tr * tq;
  const int64_t L = cdiv(in.depth, tile_k);
  if (T >= (int64_t(1) << 31) || tr >= (int64_t(1) << 31)) return FFN_B200_ERR_TOO_LARGE;
  out->tiles_r = static_cast<int32_t>(tr);
  out->tiles_q = static_cast<int32_t>(tq);
  out->tiles = static_cast<int32_t>(T);
  out->k_blocks = static_cast<int32_t>(L);
  out->group = static_cast<int32_t>(group < 1 ? 1 : (group > tr ? tr : group));
  if (split) {
    const int64_t sk = T % C;
    const int64_t iters = sk * L;
    // Each share gets at least kMinSegment K steps: short tails go to fewer CTAs, so an
    // owner never waits for, and reads, more partials than the split saves.
    int64_t ctas = iters / kMinSegment;
    ctas = ctas < 1 ? 1 : (ctas > C ? C : ctas);
    out->sk_tiles = static_cast<int32_t>(sk);
    out->dp_tiles = static_cast<int32_t>(T - sk);
    out->sk_ctas = static_cast<int32_t>(ctas);
    out->sk_iters = static_cast<int32_t>(iters / ctas);
    out->sk_rem = static_cast<int32_t>(iters % ctas);
  } else {
    out->sk_tiles = 0;
    out->dp_tiles = static_cast<int32_t>(T);
    out->sk_ctas = 0;
    out->sk_iters = 0;
    out->sk_rem = 0;
  }
  return FFN_B200_OK;
}

// down_impl full_load_a: hidden-resident row blocks (ffn_rowblock.cuh).  One CTA per row
// block of 128 tokens, up to `grid` CTAs; the Y row block lives in TMEM next to the two up
// accumulators, at most 256 columns of it, so it applies when N <= 512 (as the reference's
// full-load tiling applies only when the operand fits on chip): above 256 columns each row
// block is computed as two units, one per half of Y, each recomputing the hidden chunks.
int plan_rowblock(const ffn_b200_problem& pr, int grid, ffn_b200_plan* out) {
  if (pr.n > 512) return FFN_B200_ERR_NOT_APPLICABLE;
  int variant = pr.n <= 64 ? kFirstRowblock : (pr.n <= 128 ? kFirstRowblock + 1 : kFirstRowblock + 2);
  if (pr.tile_variant > 0) {
    const int forced = pr.tile_variant - 1;
    if (!kVariants[forced].rowblock || 2 * kVariants[forced].bn < pr.n) return FFN_B200_ERR_INVALID;
    variant = forced;
  }
  const Variant& v = kVariants[variant];
  const int64_t rows = cdiv(pr.m, ffnb200::kBM);
  const int64_t parts = cdiv(pr.n, v.bn);  // Y column parts (1 or 2), one unit each per row block
  const int64_t units = rows * parts;
  // 128-row chunks of W1: H/128, or for SwiGLU's packed W1 (64 gate + 64 up rows) H/64.
  const int64_t chunks = pr.gelu == FFN_B200_SWIGLU ? cdiv(pr.h, 64) : cdiv(pr.h, 128);
  if (units * chunks >= (int64_t(1) << 31)) return FFN_B200_ERR_TOO_LARGE;
  // Few units: clusters of S CTAs split each unit's H chunks (S = 2, 4 or 8 while S*units
  // CTAs fit the grid and every CTA keeps at least one chunk); one unit per cluster.
  int S = 1;
  while (S < 8 && units * S * 2 <= grid && chunks >= S * 2) S *= 2;
  const int C = static_cast<int>(S > 1 ? units * S : (units < grid ? units : grid));
  auto fill = [&](ffn_b200_phase_plan* ph, int64_t tq, int64_t depth) {
    ph->tiles_r = static_cast<int32_t>(rows);
    ph->tiles_q = static_cast<int32_t>(tq);
    ph->tiles = static_cast<int32_t>(rows * tq);
    ph->k_blocks = static_cast<int32_t>(cdiv(depth, ffnb200::kBK));
    ph->dp_tiles = ph->tiles;
    ph->group = 1;
  };
  fill(&out->up, chunks, pr.k);
  fill(&out->down, 1, pr.h);
  out->variant = variant;
  out->tile_m = ffnb200::kBM;
  out->tile_n = v.bn;
  out->tile_k = ffnb200::kBK;
  out->stages = v.stages;
  out->block_num = C;
  out->tmem_cols = tmem_cols_for(variant);
  out->smem_bytes = smem_for(variant);
  out->workspace_floats = 4;
  out->counter_words = ffnb200::kClaimWords + 2;
  out->flag_words = 2;
  out->status_words = 4;
  out->schedule = 1;
  out->row_split = S;
  return FFN_B200_OK;
}

// Hidden-slice decode plan (ffn_hslice.cuh): M <= 16 tokens; clusters of S CTAs, CTA r of a
// cluster owning hidden rows [(sb*S + r)*128, +128) of each super-block sb the cluster takes
// (super-block sb goes to cluster sb mod CL) and Y rows of n-blocks [r*NBR, (r+1)*NBR).
// Every cluster must be resident at once (the final reduction waits on all of them).  With
// one CTA per SM a B200 (148 SMs) holds at most 74 / 33 / 15 clusters of 2 / 4 / 8 CTAs
// (cudaOccupancyMaxActiveClusters, measured; ffn_b200_prepare checks the actual device), so
// the planner takes the largest S whose super-blocks fit one wave of clusters, else the S
// with the most even share.  `forced`: chosen through tile_variant; otherwise only when the
// clusters get equal shares of super-blocks (within 15 %) and there are at least two.
int plan_hslice(const ffn_b200_problem& pr, int grid, bool forced, ffn_b200_plan* out) {
  if (pr.m > 16 || pr.gelu == FFN_B200_SWIGLU || pr.weight_format != FFN_B200_WEIGHTS_NATIVE)
    return FFN_B200_ERR_NOT_APPLICABLE;
  const int64_t nhb = cdiv(pr.h, ffnb200::kBM);
  const int64_t nnb = cdiv(pr.n, ffnb200::kBM);
  const int sm = pr.sm_count > 0 ? pr.sm_count : 148;
  int best_s = 0;
  int64_t best_cl = 0;
  double best_bal = -1.0;
  for (int S : {8, 4, 2}) {
    const int64_t cap = (S == 8 ? 15 : (S == 4 ? 33 : 74)) * static_cast<int64_t>(sm) / 148;
    const int64_t cl_max = std::min<int64_t>(cap, grid / S);
    const int64_t sb = cdiv(nhb, S);
    const int64_t nbr = cdiv(nnb, S);
    if (cl_max < 1) continue;
    const int64_t cl = std::min(sb, cl_max);
    if (nbr * 16 > 448) continue;  // down accumulators beside the up one in TMEM
    const int64_t waves = cdiv(sb, cl);
    const double bal = static_cast<double>(sb) / static_cast<double>(waves * cl);
    if (waves == 1) {  // the largest cluster whose super-blocks fit one wave
      best_s = S; best_cl = cl; best_bal = 1.0;
      break;
    }
    if (bal > best_bal + 1e-9) { best_s = S; best_cl = cl; best_bal = bal; }
  }
  if (best_s == 0) return FFN_B200_ERR_NOT_APPLICABLE;
  const int S = best_s;
  const int64_t sb = cdiv(nhb, S);
  const int64_t nbr = cdiv(nnb, S);
  const int64_t cl = best_cl;
  if (!forced && (sb < 2 || best_bal < 0.85)) return FFN_B200_ERR_NOT_APPLICABLE;
  auto fill = [](ffn_b200_phase_plan* ph, int64_t tiles, int64_t depth) {
    ph->tiles_r = static_cast<int32_t>(tiles);
    ph->tiles_q = 1;
    ph->tiles = static_cast<int32_t>(tiles);
    ph->k_blocks = static_cast<int32_t>(cdiv(depth, ffnb200::kBK));
    ph->dp_tiles = ph->tiles;
    ph->sk_tiles = 0;
    ph->sk_iters = 0;
    ph->sk_rem = 0;
    ph->group = 1;
    ph->sk_ctas = 0;
  };
  fill(&out->up, nhb, pr.k);
  fill(&out->down, nnb, pr.h);
  out->variant = kSliceVariant;
  out->swap_ab = 1;
  out->cta_pair = 0;
  out->tile_m = ffnb200::kBM;
  out->tile_n = kVariants[kSliceVariant].bn;
  out->tile_k = ffnb200::kBK;
  out->stages = hslice_ring_bytes(S) / ffnb200::SliceLayout<4>::kStage;
  out->block_num = static_cast<int32_t>(cl * S);
  out->tmem_cols = tmem_cols_for(kSliceVariant);
  out->smem_bytes = hslice_smem(S);
  out->workspace_floats = cl * S * nbr * ffnb200::kBM * 16;  // one fp32 [S*NBR*128 x 16] partial per cluster
  out->counter_words = ffnb200::kClaimWords + S;              // one count per cluster rank
  out->flag_words = 2;
  out->status_words = 4;
  out->schedule = 1;
  out->row_split = S;
  return FFN_B200_OK;
}

int query_sm_count(int* sm) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FFN_B200_ERR_CUDA;
  if (cudaDeviceGetAttribute(sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return FFN_B200_ERR_CUDA;
  return FFN_B200_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int get_encode() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode ? FFN_B200_OK : FFN_B200_ERR_CUDA;
}

// 2-D row-major tensor [outer, inner] with `pitch` elements per row; 128B-swizzled boxes.
int encode_2d(CUtensorMap* tm, const void* base, int dtype, int64_t inner, int64_t outer, int64_t pitch,
              uint32_t box_inner, uint32_t box_outer) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch) * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt =
      dtype == FFN_B200_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = g_encode(tm, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FFN_B200_OK : FFN_B200_ERR_CUDA;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 2-D row-major fp32 tensor [outer, inner], pitch in elements; boxes of 32 x box_outer
// (128-byte rows, 128B-swizzled): the fp32 staging of the fused reduce-scatter.
int encode_2d_f32(CUtensorMap* tm, const void* base, int64_t inner, int64_t outer, int64_t pitch, uint32_t box_outer) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch) * 4};
  cuuint32_t box[2] = {32, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FFN_B200_OK : FFN_B200_ERR_CUDA;
}

// 2-D row-major tensor of fp8 codes [outer, inner] (inner even), pitch in bytes, described to
// the TMA as pairs of codes (16-bit elements: the copy engine's work follows the element
// count, and the bytes and their swizzled placement are the same); box_inner in bytes; the
// swizzle spans the box row (64- or 128-byte rows).
int encode_2d_u8(CUtensorMap* tm, const void* base, int64_t inner, int64_t outer, int64_t pitch, uint32_t box_inner,
                 uint32_t box_outer) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner / 2), static_cast<cuuint64_t>(outer)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch)};
  cuuint32_t box[2] = {box_inner / 2, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(tm, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        box_inner >= 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FFN_B200_OK : FFN_B200_ERR_CUDA;
}

}  // namespace

struct ffn_b200_handle {
  ffn_b200_problem prob;
  ffn_b200_plan plan;
  ffn_b200_buffers buf;
  int device;
  KernelFn kernel;
  Params params;
  int overlap;  // launch with programmatic stream serialisation (ffn_b200_set_launch_overlap)
};

extern "C" {

int ffn_b200_abi_version(void) { return FFN_B200_ABI_VERSION; }

const char* ffn_b200_strerror(int code) {
  switch (code) {
    case FFN_B200_OK: return "ok";
    case FFN_B200_ERR_INVALID: return "invalid argument";
    case FFN_B200_ERR_NOT_APPLICABLE: return "Stream-K candidate has no remainder tiles or fewer than two K tiles";
    case FFN_B200_ERR_UNAVAILABLE: return "implementation not available (full_load_b)";
    case FFN_B200_ERR_DEVICE: return "device is not sm_100 or block_num exceeds the SM count";
    case FFN_B200_ERR_CUDA: return "CUDA call failed";
    case FFN_B200_ERR_ALIGNMENT: return "buffer base not 16-byte aligned or pitch not a multiple of 8 elements";
    case FFN_B200_ERR_TOO_LARGE: return "problem does not fit one launch";
    case FFN_B200_ERR_SCRATCH:
      return "problem needs more scratch than the 32 MiB that ffn_b200_run_noalloc holds; use ffn_b200_prepare";
  }
  return "unknown error";
}

int ffn_b200_device_info(int device, int* sm_count, int* cc_major, int* cc_minor) {
  if (!sm_count || !cc_major || !cc_minor) return FFN_B200_ERR_INVALID;
  if (cudaDeviceGetAttribute(sm_count, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
      cudaDeviceGetAttribute(cc_major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess ||
      cudaDeviceGetAttribute(cc_minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess) {
    cudaGetLastError();
    return FFN_B200_ERR_CUDA;
  }
  return FFN_B200_OK;
}

int64_t ffn_b200_swiglu_rows(int64_t h, int32_t swap_ab) {
  if (h <= 0) return 0;
  return swap_ab ? 2 * h : 128 * ((h + 63) / 64);
}

int ffn_b200_make_plan(const ffn_b200_problem* pr, ffn_b200_plan* out) {
  if (!pr || !out) return FFN_B200_ERR_INVALID;
  // Shape contract of ops/host/inputs.py:38-53.
  if (pr->m <= 0 || pr->k <= 0 || pr->h <= 0 || pr->n <= 0) return FFN_B200_ERR_INVALID;
  if (pr->k > 65535 || pr->h > 65535 || pr->n > 65535 || pr->m > (int64_t(1) << 31) - 16)
    return FFN_B200_ERR_INVALID;
  if (pr->dtype != FFN_B200_F16 && pr->dtype != FFN_B200_BF16) return FFN_B200_ERR_INVALID;
  if (pr->gelu < FFN_B200_GELU_RATIONAL || pr->gelu > FFN_B200_SWIGLU) return FFN_B200_ERR_INVALID;
  if (pr->down_impl < 0 || pr->down_impl > 3) return FFN_B200_ERR_INVALID;
  if (pr->down_impl == FFN_B200_DOWN_FULL_LOAD_B) return FFN_B200_ERR_UNAVAILABLE;
  int sm = pr->sm_count;
  if (sm <= 0) {
    const int rc = query_sm_count(&sm);
    if (rc) return rc;
  }
  const int grid = pr->block_num > 0 ? pr->block_num : sm;
  if (grid < 1 || grid > 65535 || pr->block_num < 0) return FFN_B200_ERR_INVALID;
  if (pr->tile_variant < 0 || pr->tile_variant > kNumVariants) return FFN_B200_ERR_INVALID;
  if (pr->raster_group < 0 || pr->l2_policy < 0 || pr->l2_policy > 4) return FFN_B200_ERR_INVALID;
  if (pr->schedule < 0 || pr->schedule > 3) return FFN_B200_ERR_INVALID;
  if (pr->weight_format != FFN_B200_WEIGHTS_NATIVE && pr->weight_format != FFN_B200_WEIGHTS_FP8_ROWS)
    return FFN_B200_ERR_INVALID;
  const bool fp8w = pr->weight_format == FFN_B200_WEIGHTS_FP8_ROWS;

  std::memset(out, 0, sizeof(*out));
  if (pr->down_impl == FFN_B200_DOWN_FULL_LOAD_A) {
    if (fp8w) return FFN_B200_ERR_NOT_APPLICABLE;
    return plan_rowblock(*pr, grid, out);
  }
  if (pr->tile_variant > 0 && kVariants[pr->tile_variant - 1].rowblock) return FFN_B200_ERR_INVALID;
  if (pr->tile_variant > 0 && kVariants[pr->tile_variant - 1].w8 != fp8w) return FFN_B200_ERR_INVALID;
  // fp8 weights are widened on chip by the decode tiles only (the weight-streaming,
  // HBM-bound regime where halving the weight bytes matters).
  if (fp8w && pr->tile_variant == 0 && pr->m > 64) return FFN_B200_ERR_NOT_APPLICABLE;
  if (fp8w && ((pr->k & 1) || (pr->h & 1))) return FFN_B200_ERR_NOT_APPLICABLE;  // code pairs per TMA element
  const bool slice_forced = pr->tile_variant == kSliceVariant + 1;
  int variant;
  if (slice_forced) {
    variant = 2;  // the swap-AB plan's applicability rules come first
    if (pr->m > 16) return FFN_B200_ERR_INVALID;
  } else if (pr->tile_variant > 0) {
    variant = pr->tile_variant - 1;
    if (kVariants[variant].swap && pr->m > kVariants[variant].bn) return FFN_B200_ERR_INVALID;
    if (kVariants[variant].pair && grid < 2) return FFN_B200_ERR_INVALID;
  } else if (fp8w) {
    variant = pr->m <= 16 ? 10 : 11;
  } else if (pr->m <= 16) {
    variant = 2;
  } else if (pr->m <= 64) {
    variant = 3;
  } else {
    // Long prefill runs (at least 8 waves of 256x256 tiles): CTA pairs, whose halved
    // shared-memory traffic per FLOP and deeper ring run the tensor pipe busier at the same
    // power (cfg4: 90 % vs 87 % tensor-pipe activity; cfg5: 1280 vs 1231 TFLOP/s on one box).
    const int64_t t256 = cdiv(pr->m, 128) * cdiv(pr->h, 256);
    const int64_t p256 = cdiv(pr->m, 256) * cdiv(pr->h, 256);
    if (grid >= 2 && (grid % 2) == 0 && p256 >= 8 * static_cast<int64_t>(grid / 2)) variant = 4;
    else variant = t256 >= 2 * static_cast<int64_t>(grid) ? 0 : 1;
  }
  const Variant& v = kVariants[variant];
  const int ncta = v.pair ? 2 : 1;
  const int tile_m = ffnb200::kBM * ncta;
  const int C = grid / ncta;  // work-list owners (CTAs, or CTA pairs)
  // SwiGLU: the up GEMM runs over the packed gate/up rows of W1 (ffn_b200_swiglu_rows).
  const int64_t up_rows = pr->gelu == FFN_B200_SWIGLU ? ffn_b200_swiglu_rows(pr->h, v.swap ? 1 : 0) : pr->h;
  const PhaseInput up = v.swap ? PhaseInput{up_rows, pr->m, pr->k} : PhaseInput{pr->m, up_rows, pr->k};
  const PhaseInput dn = v.swap ? PhaseInput{pr->n, pr->m, pr->h} : PhaseInput{pr->m, pr->n, pr->h};
  // Raster group: a wave of C concurrent tiles spans `group` tile rows x C/group tile columns;
  // balancing their operand bytes (group*tile_m = (C/group)*tile_n) minimises the K-slices a
  // wave pulls through L2.
  int group = pr->raster_group;
  if (group <= 0) {
    // (CTA pairs: half the balanced height -- measured on cfg5, 4 pair rows beat 8 by 1-4 %
    // and 16 loses 6 %.)
    const double balanced = std::sqrt(static_cast<double>(C) * v.bn / tile_m) / (v.pair ? 2.0 : 1.0);
    group = static_cast<int>(std::lround(balanced));
    // Prefer a nearby divisor of the tile-row count so no group is a ragged remainder
    // (measured on cfg5: 16 rows of 128 beat 17 by 2 %).
    const int64_t rows = cdiv(v.swap ? pr->h : pr->m, tile_m);
    for (int d = 0; d <= static_cast<int>(0.3 * balanced); ++d) {
      if (group - d >= 1 && rows % (group - d) == 0) { group -= d; break; }
      if (rows % (group + d) == 0) { group += d; break; }
    }
  }

  // Up phase: data-parallel, with the tail wave split along K when whole tiles would leave
  // more than a tenth of the CTAs idle in the last wave (a schedule choice only).
  ffn_b200_phase_plan probe;
  const int tile_k = ffnb200::kBK * v.ksub;
  int rc = phase_plan(up, tile_m, v.bn, tile_k, C, false, group, &probe);
  if (rc) return rc;
  // Splitting only pays when a tile's mainloop outlasts the partial exchange and fixup
  // (measured ~5-10 us): short tiles (fewer than kMinSplitKBlocks stages) stay whole even
  // if the last wave leaves SMs idle.
  const int64_t waves = cdiv(probe.tiles, C);
  const bool up_split = (probe.tiles % C) != 0 && probe.k_blocks >= kMinSplitKBlocks &&
                        static_cast<double>(probe.tiles) < 0.9 * static_cast<double>(waves * C);
  rc = phase_plan(up, tile_m, v.bn, tile_k, C, up_split, group, &out->up);
  if (rc) return rc;

  const bool streamk = pr->down_impl == FFN_B200_DOWN_STREAMK;
  rc = phase_plan(dn, tile_m, v.bn, tile_k, C, streamk, group, &out->down);
  if (rc) return rc;
  if (streamk && (out->down.tiles % C == 0 || out->down.k_blocks < 2)) return FFN_B200_ERR_NOT_APPLICABLE;
  if (static_cast<int64_t>(out->up.sk_tiles) * out->up.k_blocks >= (int64_t(1) << 31) ||
      static_cast<int64_t>(out->down.sk_tiles) * out->down.k_blocks >= (int64_t(1) << 31))
    return FFN_B200_ERR_TOO_LARGE;

  out->variant = variant;
  out->swap_ab = v.swap ? 1 : 0;
  out->cta_pair = v.pair ? 1 : 0;
  out->tile_m = tile_m;
  out->tile_n = v.bn;
  out->tile_k = tile_k;
  out->stages = v.stages;
  out->block_num = C * ncta;
  out->tmem_cols = tmem_cols_for(variant);
  out->smem_bytes = smem_for(variant);
  out->workspace_floats = 2ll * C * ncta * ffnb200::kBM * v.bn;
  out->counter_words = ffnb200::kClaimWords + (v.swap ? out->up.tiles_q : out->up.tiles_r);
  out->flag_words = 2ll * C * ncta;
  out->status_words = 4;
  // Automatic: the wave-synchronised static order for CTA-pair plans, whose pairs drift apart
  // under the plain static order (cfg5: 773 us of spread at the phase change, 189 GB of DRAM
  // reads) and lose their placement under dynamic claims (cfg5: 1253-1263 TFLOP/s dynamic,
  // 1279-1283 synced); static for one-CTA tiles, whose cooperative launch keeps GPC-major
  // placement and little drift (cfg5: 52 GB static against 64 GB dynamic) and for decode
  // grids of one or two waves, where a claim would only add its latency.
  out->schedule = pr->schedule ? pr->schedule : (v.pair ? 3 : 1);
  out->row_split = 1;
  // Decode (M <= 16): the hidden-slice kernel where its clusters share the work evenly.
  if (slice_forced || (pr->tile_variant == 0 && variant == 2)) {
    ffn_b200_plan sl;
    std::memset(&sl, 0, sizeof(sl));
    const int rs = plan_hslice(*pr, grid, slice_forced, &sl);
    if (rs == FFN_B200_OK) *out = sl;
    else if (slice_forced) return rs == FFN_B200_ERR_NOT_APPLICABLE ? FFN_B200_ERR_INVALID : rs;
  }
  return FFN_B200_OK;
}

int ffn_b200_prepare(const ffn_b200_problem* pr, const ffn_b200_buffers* b, int device, ffn_b200_handle** out) {
  if (!pr || !b || !out) return FFN_B200_ERR_INVALID;
  *out = nullptr;
  int sm = 0, ccmaj = 0, ccmin = 0;
  int rc = ffn_b200_device_info(device, &sm, &ccmaj, &ccmin);
  if (rc) return rc;
  if (ccmaj != 10 || ccmin != 0) return FFN_B200_ERR_DEVICE;
  ffn_b200_problem prob = *pr;
  if (prob.sm_count <= 0) prob.sm_count = sm;
  if (prob.block_num > sm) return FFN_B200_ERR_DEVICE;  // co-residency (ops/api.py:63-64)
  ffn_b200_plan plan;
  rc = ffn_b200_make_plan(&prob, &plan);
  if (rc) return rc;
  if (plan.block_num > sm) return FFN_B200_ERR_DEVICE;

  // Buffers: TMA needs 16-byte aligned bases and pitches.  The row-block kernel keeps the
  // hidden activations on chip and ignores `hidden` / `ldh`.
  const bool rowblock = kVariants[plan.variant].rowblock;
  const void* bases[] = {b->x, b->w1, b->w2, b->y, b->workspace, rowblock ? b->y : b->hidden};
  for (const void* p : bases)
    if (!p) return FFN_B200_ERR_INVALID;
  for (const void* p : bases)
    if (!aligned16(p)) return FFN_B200_ERR_ALIGNMENT;
  if (!b->counters || !b->flags || !b->status) return FFN_B200_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(b->counters) & 7u) return FFN_B200_ERR_ALIGNMENT;
  if ((b->bias1 && !aligned16(b->bias1)) || (b->bias2 && !aligned16(b->bias2))) return FFN_B200_ERR_ALIGNMENT;
  if (b->bias1 && pr->gelu == FFN_B200_SWIGLU) return FFN_B200_ERR_INVALID;  // no gate/up bias
  const int64_t pitches[] = {b->ldx, b->ldw1, b->ldw2, rowblock ? b->ldy : b->ldh, b->ldy};
  for (int64_t p : pitches)
    if (p <= 0 || (p % 8) != 0) return FFN_B200_ERR_ALIGNMENT;
  const bool w8 = kVariants[plan.variant].w8;
  if (w8) {  // fp8 codes: 1-byte elements, so 16-byte pitches are multiples of 16 elements
    if ((b->ldw1 % 16) != 0 || (b->ldw2 % 16) != 0) return FFN_B200_ERR_ALIGNMENT;
    if (!b->w1_scale || !b->w2_scale) return FFN_B200_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(b->w1_scale) & 3u) || (reinterpret_cast<uintptr_t>(b->w2_scale) & 3u))
      return FFN_B200_ERR_ALIGNMENT;
  }
  if (b->ldx < prob.k || b->ldw1 < prob.k || b->ldw2 < prob.h || (!rowblock && b->ldh < prob.h) || b->ldy < prob.n)
    return FFN_B200_ERR_INVALID;

  rc = get_encode();
  if (rc) return rc;

  auto* h = new (std::nothrow) ffn_b200_handle();
  if (!h) return FFN_B200_ERR_INVALID;
  h->prob = prob;
  h->plan = plan;
  h->buf = *b;
  h->device = device;
  h->kernel = kVariants[plan.variant].hslice ? pick_hslice(plan.row_split, prob.dtype == FFN_B200_BF16, prob.gelu)
                                             : kernel_for(plan.variant, prob.dtype == FFN_B200_BF16, prob.gelu);

  Params& P = h->params;
  std::memset(&P, 0, sizeof(P));
  // Rows of W1 as stored: the gate/up-packed rows for SwiGLU.
  const int64_t w1_rows = prob.gelu == FFN_B200_SWIGLU ? ffn_b200_swiglu_rows(prob.h, plan.swap_ab) : prob.h;
  // B boxes: each CTA of a pair loads half of the tile's B rows.
  const uint32_t bn = static_cast<uint32_t>(plan.tile_n / (plan.cta_pair ? 2 : 1));
  const int dt = prob.dtype;
  const bool sw = plan.swap_ab != 0;
  // Up:   normal A = X [M,K] (128-row boxes), B = W1 [H,K] (bn-row boxes); swap exchanges them.
  // Down: normal A = hidden [M,H], B = W2 [N,H]; swap exchanges them.
  if (rowblock) {
    // X [M,K] and W1 [H,K] in 128-row boxes, W2 [N,H] in one box of tile_n rows, Y stores.
    rc = encode_2d(&P.tm_a_up, b->x, dt, prob.k, prob.m, b->ldx, 64, 128);
    if (!rc) rc = encode_2d(&P.tm_b_up, b->w1, dt, prob.k, w1_rows, b->ldw1, 64, 128);
    if (!rc) rc = encode_2d(&P.tm_b_dn, b->w2, dt, prob.h, prob.n, b->ldw2, 64, static_cast<uint32_t>(plan.tile_n));
    if (!rc) rc = encode_2d(&P.tm_st_y, b->y, dt, prob.n, prob.m, b->ldy, 64, ffnb200::kStoreRows);
  } else if (!sw) {
    rc = encode_2d(&P.tm_a_up, b->x, dt, prob.k, prob.m, b->ldx, 64, 128);
    if (!rc) rc = encode_2d(&P.tm_b_up, b->w1, dt, prob.k, w1_rows, b->ldw1, 64, bn);
    if (!rc) rc = encode_2d(&P.tm_a_dn, b->hidden, dt, prob.h, prob.m, b->ldh, 64, 128);
    if (!rc) rc = encode_2d(&P.tm_b_dn, b->w2, dt, prob.h, prob.n, b->ldw2, 64, bn);
    if (!rc) rc = encode_2d(&P.tm_st_hid, b->hidden, dt, prob.h, prob.m, b->ldh, 64, ffnb200::kStoreRows);
    if (!rc) rc = encode_2d(&P.tm_st_y, b->y, dt, prob.n, prob.m, b->ldy, 64, ffnb200::kStoreRows);
  } else if (w8) {
    // fp8 weight k-blocks: 128 rows x 64 one-byte codes, 64-byte swizzle (the converter
    // warps read them bank-conflict free); the token operands as in the 16-bit decode tiles.
    const uint32_t wbox = static_cast<uint32_t>(64 * kVariants[plan.variant].ksub);  // bytes of a weight row per load
    rc = encode_2d_u8(&P.tm_a_up, b->w1, prob.k, w1_rows, b->ldw1, wbox, 128);
    if (!rc) rc = encode_2d(&P.tm_b_up, b->x, dt, prob.k, prob.m, b->ldx, 64, bn);
    if (!rc) rc = encode_2d_u8(&P.tm_a_dn, b->w2, prob.h, prob.n, b->ldw2, wbox, 128);
    if (!rc) rc = encode_2d(&P.tm_b_dn, b->hidden, dt, prob.h, prob.m, b->ldh, 64, bn);
    P.w1_scale = b->w1_scale;
    P.w2_scale = b->w2_scale;
  } else {
    rc = encode_2d(&P.tm_a_up, b->w1, dt, prob.k, w1_rows, b->ldw1, 64, 128);
    if (!rc) rc = encode_2d(&P.tm_b_up, b->x, dt, prob.k, prob.m, b->ldx, 64, bn);
    if (!rc) rc = encode_2d(&P.tm_a_dn, b->w2, dt, prob.h, prob.n, b->ldw2, 64, 128);
    if (!rc) rc = encode_2d(&P.tm_b_dn, b->hidden, dt, prob.h, prob.m, b->ldh, 64, bn);
  }
  if (rc) {
    delete h;
    return rc;
  }
  P.bias1 = static_cast<const uint16_t*>(b->bias1);
  P.bias2 = static_cast<const uint16_t*>(b->bias2);
  P.hidden = b->hidden;
  P.y = b->y;
  P.ldh = b->ldh;
  P.ldy = b->ldy;
  P.ws = b->workspace;
  P.claims = reinterpret_cast<unsigned long long*>(b->counters);
  P.launches = reinterpret_cast<unsigned long long*>(b->counters + 4);
  P.counters = b->counters + ffnb200::kClaimWords;
  P.dyn = plan.schedule == 2 ? 1 : 0;
  P.flags = b->flags;
  P.status = b->status;
  auto to_sched = [](const ffn_b200_phase_plan& pp) {
    PhaseSched s;
    s.tiles_r = pp.tiles_r; s.tiles_q = pp.tiles_q; s.T = pp.tiles; s.L = pp.k_blocks;
    s.dp = pp.dp_tiles; s.sk = pp.sk_tiles; s.q = pp.sk_iters; s.rem = pp.sk_rem; s.group = pp.group;
    s.skc = pp.sk_ctas;
    return s;
  };
  P.up = to_sched(plan.up);
  P.dn = to_sched(plan.down);
  P.M = static_cast<int>(prob.m);
  P.H = static_cast<int>(prob.h);
  P.N = static_cast<int>(prob.n);
  const int ncta = plan.cta_pair ? 2 : 1;
  P.C = plan.block_num / ncta;
  P.rb_split = plan.row_split;
  // Serpentine K order for the prefill tiles (cfg5: DRAM reads 60.6 -> 53.2 GB per call, +1 %
  // TFLOP/s at a 2 % higher clock under the power cap); decode tiles stream weights once.
  P.kserp = plan.swap_ab ? 0 : 1;
  P.wave_sync = plan.schedule == 3 ? 1 : 0;
  if (kVariants[plan.variant].hslice) {
    const int S = plan.row_split;
    P.hs_superblocks = static_cast<int>(cdiv(plan.up.tiles_r, S));
    P.hs_nbr = static_cast<int>(cdiv(plan.down.tiles_r, S));
  }
  P.wait_limit_ns = 4000000000ull;
  P.inject = 0;
  P.l2_hints = prob.l2_policy == 2 ? 1 : (prob.l2_policy == 3 ? 2 : (prob.l2_policy == 4 ? 3 : 0));
  // The launch epoch lives on the device (Params::launches, in the counters buffer): readiness
  // counters gain epi * ncta * (up tiles per row block) per launch and flags epi per launch,
  // compared modulo 2^32, so nothing here counts launches and a captured launch replays.

  int cur = 0;
  cudaGetDevice(&cur);
  if (cur != device) cudaSetDevice(device);
  const cudaError_t e =
      cudaFuncSetAttribute(h->kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(plan.smem_bytes));
  int rc2 = e == cudaSuccess ? FFN_B200_OK : FFN_B200_ERR_CUDA;
  const int wait_cluster = plan.cta_pair ? 2 : (kVariants[plan.variant].hslice ? plan.row_split : 1);
  if (!rc2 && wait_cluster > 1) {
    // Every cluster of the grid must be resident at once (pairs: the down phase waits on up
    // tiles of other pairs; hidden slices: the final reduction waits on every cluster): the
    // grid may not exceed the co-resident cluster count.
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(static_cast<unsigned>(plan.block_num), 1, 1);
    cfg.blockDim = dim3(static_cast<unsigned>(threads_for(plan.variant)), 1, 1);
    cfg.dynamicSmemBytes = static_cast<size_t>(plan.smem_bytes);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(wait_cluster);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, h->kernel, &cfg) != cudaSuccess) {
      cudaGetLastError();
      rc2 = FFN_B200_ERR_CUDA;
    } else if (plan.block_num > wait_cluster * clusters) {
      rc2 = FFN_B200_ERR_DEVICE;
    }
  }
  // Pair plans over the whole GPU: renumber the pairs so that neighbouring work-list owners
  // share a GPC (see ffn_placement.cu); null keeps launch order.
  if (!rc2 && plan.cta_pair)
    P.owner_map = ffnb200::internal_pair_owner_map(device, plan.block_num, static_cast<int>(plan.smem_bytes));
  if (cur != device) cudaSetDevice(cur);
  if (rc2) {
    cudaGetLastError();
    delete h;
    return rc2;
  }
  *out = h;
  return FFN_B200_OK;
}

int ffn_b200_reset(ffn_b200_handle* h, void* stream) {
  if (!h) return FFN_B200_ERR_INVALID;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const ffn_b200_buffers& b = h->buf;
  if (cudaMemsetAsync(b.counters, 0, sizeof(uint32_t) * h->plan.counter_words, st) != cudaSuccess ||
      cudaMemsetAsync(b.flags, 0, sizeof(uint32_t) * h->plan.flag_words, st) != cudaSuccess ||
      cudaMemsetAsync(b.status, 0, sizeof(int32_t) * h->plan.status_words, st) != cudaSuccess) {
    cudaGetLastError();
    return FFN_B200_ERR_CUDA;
  }
  if (h->params.rs_world > 1) {
    const size_t band = static_cast<size_t>(h->params.rs_band_tiles) * h->plan.down.tiles_q;
    if (cudaMemsetAsync(h->params.rs_flags[h->params.rs_rank], 0, 4 * band * h->params.rs_world, st) !=
        cudaSuccess) {
      cudaGetLastError();
      return FFN_B200_ERR_CUDA;
    }
  }
  return FFN_B200_OK;
}

int ffn_b200_run(ffn_b200_handle* h, void* stream) {
  if (!h) return FFN_B200_ERR_INVALID;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(static_cast<unsigned>(h->plan.block_num), 1, 1);
  cfg.blockDim = dim3(static_cast<unsigned>(threads_for(h->plan.variant)), 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(h->plan.smem_bytes);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  unsigned n_attr = 0;
  if (h->plan.cta_pair || h->plan.row_split > 1) {  // CTA pairs; split row blocks
    attr[n_attr].id = cudaLaunchAttributeClusterDimension;
    attr[n_attr].val.clusterDim.x = h->plan.cta_pair ? 2 : static_cast<unsigned>(h->plan.row_split);
    attr[n_attr].val.clusterDim.y = 1;
    attr[n_attr].val.clusterDim.z = 1;
    ++n_attr;
  } else if (!kVariants[h->plan.variant].rowblock && !h->overlap) {
    // Row-block plans have no waits between CTAs: no co-residency needed.  An overlapped
    // launch is a plain one too: a cooperative grid starts only once the previous grid has
    // left every SM, which would void the overlap.  Its CTAs (one per SM, grid <= SMs) all
    // become resident as the previous kernel's CTAs exit; the bounded waits report, rather
    // than hang, if another stream's kernel kept SMs from them for longer than the limit.
    attr[n_attr].id = cudaLaunchAttributeCooperative;
    attr[n_attr].val.cooperative = 1;
    ++n_attr;
  }
  if (h->overlap) {
    attr[n_attr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n_attr].val.programmaticStreamSerializationAllowed = 1;
    ++n_attr;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n_attr;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, h->kernel, h->params);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return FFN_B200_ERR_CUDA;
  }
  return FFN_B200_OK;
}

int ffn_b200_rebind_io(ffn_b200_handle* h, const void* x, void* y) {
  if (!h || !x || !y) return FFN_B200_ERR_INVALID;
  if (!aligned16(x) || !aligned16(y)) return FFN_B200_ERR_ALIGNMENT;
  const ffn_b200_problem& pr = h->prob;
  const int dt = pr.dtype;
  const uint32_t bn = static_cast<uint32_t>(h->plan.tile_n);
  Params P = h->params;
  int rc;
  if (!h->plan.swap_ab) {
    rc = encode_2d(&P.tm_a_up, x, dt, pr.k, pr.m, h->buf.ldx, 64, 128);
    if (!rc) rc = encode_2d(&P.tm_st_y, y, dt, pr.n, pr.m, h->buf.ldy, 64, ffnb200::kStoreRows);
  } else {
    rc = encode_2d(&P.tm_b_up, x, dt, pr.k, pr.m, h->buf.ldx, 64, bn);
  }
  if (rc) return rc;
  P.y = y;
  h->params = P;
  h->buf.x = x;
  h->buf.y = y;
  return FFN_B200_OK;
}

int ffn_b200_set_wait_limit(ffn_b200_handle* h, uint64_t ns) {
  if (!h || ns == 0) return FFN_B200_ERR_INVALID;
  h->params.wait_limit_ns = ns;
  return FFN_B200_OK;
}

int ffn_b200_set_fault_injection(ffn_b200_handle* h, int mode) {
  if (!h || mode < 0 || mode > 1) return FFN_B200_ERR_INVALID;
  h->params.inject = mode;
  return FFN_B200_OK;
}

// ---- multi-GPU: peer-visible buffers and the fused reduce-scatter ----------------------
int ffn_b200_peer_alloc(uint64_t bytes, void** dev_ptr, void* ipc_handle) {
  if (!dev_ptr || !ipc_handle || bytes == 0) return FFN_B200_ERR_INVALID;
  void* ptr = nullptr;
  if (cudaMalloc(&ptr, bytes) != cudaSuccess) {
    cudaGetLastError();
    return FFN_B200_ERR_CUDA;
  }
  cudaIpcMemHandle_t hd;
  if (cudaMemset(ptr, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&hd, ptr) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(ptr);
    return FFN_B200_ERR_CUDA;
  }
  std::memcpy(ipc_handle, &hd, sizeof(hd));
  *dev_ptr = ptr;
  return FFN_B200_OK;
}

int ffn_b200_peer_open(const void* ipc_handle, void** dev_ptr) {
  if (!ipc_handle || !dev_ptr) return FFN_B200_ERR_INVALID;
  cudaIpcMemHandle_t hd;
  std::memcpy(&hd, ipc_handle, sizeof(hd));
  if (cudaIpcOpenMemHandle(dev_ptr, hd, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return FFN_B200_ERR_CUDA;
  }
  return FFN_B200_OK;
}

int ffn_b200_peer_close(void* dev_ptr) {
  if (!dev_ptr) return FFN_B200_ERR_INVALID;
  if (cudaIpcCloseMemHandle(dev_ptr) != cudaSuccess) {
    cudaGetLastError();
    return FFN_B200_ERR_CUDA;
  }
  return FFN_B200_OK;
}

int ffn_b200_peer_free(void* dev_ptr) {
  if (!dev_ptr) return FFN_B200_ERR_INVALID;
  if (cudaFree(dev_ptr) != cudaSuccess) {
    cudaGetLastError();
    return FFN_B200_ERR_CUDA;
  }
  return FFN_B200_OK;
}

int ffn_b200_reduce_scatter_bytes(const ffn_b200_handle* h, int world, int32_t partial, uint64_t* stage_bytes,
                                  uint64_t* flag_bytes) {
  if (!h || !stage_bytes || !flag_bytes || world < 2 || world > ffnb200::kMaxRanks) return FFN_B200_ERR_INVALID;
  if (partial != FFN_B200_PARTIAL_F32 && partial != FFN_B200_PARTIAL_INPUT && partial != FFN_B200_PARTIAL_F24)
    return FFN_B200_ERR_INVALID;
  const ffn_b200_plan& pl = h->plan;
  if (pl.swap_ab || pl.cta_pair || pl.down.tiles_r % world) return FFN_B200_ERR_INVALID;
  const uint64_t band = static_cast<uint64_t>(pl.down.tiles_r / world) * pl.down.tiles_q;
  const uint64_t esize = partial == FFN_B200_PARTIAL_F32 ? 4 : (partial == FFN_B200_PARTIAL_F24 ? 3 : 2);
  *stage_bytes = 2ull * world * band * ffnb200::kBM * pl.tile_n * esize;
  *flag_bytes = 4ull * world * band;
  return FFN_B200_OK;
}

int ffn_b200_set_reduce_scatter(ffn_b200_handle* h, int world, int rank, int32_t partial, void* const* stage_ptrs,
                                void* const* flag_ptrs, void* y_local, int64_t ldy_local) {
  if (!h || world < 2 || world > ffnb200::kMaxRanks || rank < 0 || rank >= world || !stage_ptrs || !flag_ptrs ||
      !y_local)
    return FFN_B200_ERR_INVALID;
  if (partial != FFN_B200_PARTIAL_F32 && partial != FFN_B200_PARTIAL_INPUT && partial != FFN_B200_PARTIAL_F24)
    return FFN_B200_ERR_INVALID;
  const ffn_b200_plan& pl = h->plan;
  if (pl.swap_ab || pl.cta_pair || pl.down.tiles_r % world) return FFN_B200_ERR_INVALID;
  if (h->prob.m % (static_cast<int64_t>(world) * pl.tile_m) != 0) return FFN_B200_ERR_INVALID;
  if (!aligned16(y_local) || ldy_local < h->prob.n || (ldy_local % 8) != 0) return FFN_B200_ERR_ALIGNMENT;
  for (int r = 0; r < world; ++r)
    if (!stage_ptrs[r] || !flag_ptrs[r] || !aligned16(stage_ptrs[r])) return FFN_B200_ERR_INVALID;
  const int rc = encode_2d(&h->params.tm_st_y, y_local, h->prob.dtype, h->prob.n, h->prob.m / world, ldy_local, 64,
                           ffnb200::kStoreRows);
  if (rc) return rc;
  Params& P = h->params;
  P.rs_world = world;
  P.rs_rank = rank;
  P.rs_band_tiles = pl.down.tiles_r / world;
  P.rs_format = partial == FFN_B200_PARTIAL_F32 ? 1 : (partial == FFN_B200_PARTIAL_F24 ? 2 : 0);
  const int64_t stage_rows = 2ll * world * (pl.down.tiles_r / world) * pl.down.tiles_q * ffnb200::kBM;
  P.rs_lo_off = stage_rows * pl.tile_n * 2;  // format 2: the byte plane follows the 16-bit plane
  for (int r = 0; r < world; ++r) {
    P.rs_stage[r] = stage_ptrs[r];
    P.rs_flags[r] = static_cast<unsigned*>(flag_ptrs[r]);
    // Bulk-store maps over rank r's staging buffer ([rows][tile_n], no multicast).
    int e = P.rs_format == 1 ? encode_2d_f32(&P.tm_rs[r], stage_ptrs[r], pl.tile_n, stage_rows, pl.tile_n,
                                             ffnb200::kStoreRows)
                             : encode_2d(&P.tm_rs[r], stage_ptrs[r], h->prob.dtype, pl.tile_n, stage_rows, pl.tile_n,
                                         64, ffnb200::kStoreRows);
    if (!e && P.rs_format == 2)  // the byte plane: 64-byte rows of a 64-column chunk
      e = encode_2d_u8(&P.tm_rs_lo[r], static_cast<const uint8_t*>(stage_ptrs[r]) + P.rs_lo_off, pl.tile_n,
                       stage_rows, pl.tile_n, 64, ffnb200::kStoreRows);
    if (e) return e;
  }
  return FFN_B200_OK;
}

int ffn_b200_set_launch_overlap(ffn_b200_handle* h, int32_t enable) {
  if (!h || (enable != 0 && enable != 1)) return FFN_B200_ERR_INVALID;
  h->overlap = enable;
  return FFN_B200_OK;
}

int ffn_b200_set_trace(ffn_b200_handle* h, uint64_t* device_stamps) {
  if (!h) return FFN_B200_ERR_INVALID;
  if (device_stamps && (reinterpret_cast<uintptr_t>(device_stamps) & 7u)) return FFN_B200_ERR_ALIGNMENT;
  h->params.trace = reinterpret_cast<unsigned long long*>(device_stamps);
  return FFN_B200_OK;
}

int ffn_b200_set_owner_map(ffn_b200_handle* h, const int32_t* device_map) {
  if (!h) return FFN_B200_ERR_INVALID;
  if (device_map && (reinterpret_cast<uintptr_t>(device_map) & 3u)) return FFN_B200_ERR_ALIGNMENT;
  h->params.owner_map = device_map;
  return FFN_B200_OK;
}

int ffn_b200_get_owner_map(const ffn_b200_handle* h, int32_t* host_out, int32_t capacity, int32_t* count) {
  if (!h || !count || capacity < 0 || (capacity > 0 && !host_out)) return FFN_B200_ERR_INVALID;
  const int owners = h->plan.block_num / (h->plan.cta_pair ? 2 : 1);
  *count = h->params.owner_map ? owners : 0;
  if (!h->params.owner_map || capacity == 0) return FFN_B200_OK;
  const int n = owners < capacity ? owners : capacity;
  if (cudaMemcpy(host_out, h->params.owner_map, sizeof(int32_t) * n, cudaMemcpyDeviceToHost) != cudaSuccess) {
    cudaGetLastError();
    return FFN_B200_ERR_CUDA;
  }
  return FFN_B200_OK;
}

int ffn_b200_get_plan(const ffn_b200_handle* h, ffn_b200_plan* plan) {
  if (!h || !plan) return FFN_B200_ERR_INVALID;
  *plan = h->plan;
  return FFN_B200_OK;
}

int ffn_b200_destroy(ffn_b200_handle* h) {
  delete h;
  return FFN_B200_OK;
}

int ffn_b200_launch(const ffn_b200_problem* pr, const ffn_b200_buffers* b, void* stream) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FFN_B200_ERR_CUDA;
  ffn_b200_handle* h = nullptr;
  int rc = ffn_b200_prepare(pr, b, dev, &h);
  if (rc) return rc;
  rc = ffn_b200_reset(h, stream);
  if (!rc) rc = ffn_b200_run(h, stream);
  ffn_b200_destroy(h);
  return rc;
}

}  // extern "C"

// Internal accessors used by the allocation-free entry point in ffn_noalloc.cu; not exported.
namespace ffnb200 {
bool internal_is_rowblock(int variant) { return variant >= 0 && variant < kNumVariants && kVariants[variant].rowblock; }
bool internal_is_hslice(int variant) { return variant >= 0 && variant < kNumVariants && kVariants[variant].hslice > 0; }
void (*internal_kernel_for(int variant, int bf16, int gelu))(const Params) {
  return kernel_for(variant, bf16, gelu);
}
int internal_threads_for(int variant) { return threads_for(variant); }
int internal_encode_2d(CUtensorMap* tm, const void* base, int dtype, int64_t inner, int64_t outer, int64_t pitch,
                       uint32_t box_inner, uint32_t box_outer) {
  const int rc = get_encode();
  if (rc) return rc;
  return encode_2d(tm, base, dtype, inner, outer, pitch, box_inner, box_outer);
}
}  // namespace ffnb200
