// Allocation-free entry point ffn_b200_run_noalloc (declared in include/ffn_b200.h).
//
// For callers that must not allocate device memory while they run the FFN -- an inference
// engine that gives its plugins a fixed memory budget and calls them on its execution path
// (where cudaMalloc is refused, or synchronises the whole device and stalls every other
// stream), or a serving loop that reserves all of its memory up front.  Such a caller passes
// X, W1, W2 and Y; everything else the fused kernel needs -- the hidden activations, the
// Stream-K fp32 partials, the readiness counters, flags and status words -- lives in one
// statically sized device array owned by this file.
//
// Limits and rules:
//   * the array holds FFN_B200_NOALLOC_SCRATCH_BYTES (32 MiB) on every GPU that loads this
//     code, until the process exits; a problem whose scratch does not fit is rejected with
//     FFN_B200_ERR_SCRATCH before anything is launched;
//   * the array's device address is looked up once per device (cudaGetSymbolAddress, with
//     that device current) by the first call made on that device -- make that first call
//     before any stream capture;
//   * every call clears the counters, flags and status words on its stream, launches once
//     with launch epoch 1 and leaves the array as the kernel left it; calls share the one
//     array, so calls that overlap on the GPU race and must be serialised by the caller;
//   * nothing here calls cudaMalloc, cudaFree or any allocating routine.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/ffn_b200.h"
#include "ffn_kernel.cuh"

namespace ffnb200 {
void (*internal_kernel_for(int variant, int bf16, int gelu))(const Params);
int internal_encode_2d(CUtensorMap* tm, const void* base, int dtype, int64_t inner, int64_t outer, int64_t pitch,
                       uint32_t box_inner, uint32_t box_outer);
int internal_threads_for(int variant);
bool internal_is_rowblock(int variant);
bool internal_is_hslice(int variant);
}  // namespace ffnb200

// The scratch.  In host code this name is only a stand-in for the symbol; the device address
// comes from cudaGetSymbolAddress below and is what the kernel receives.
static __device__ __align__(256) unsigned char g_noalloc_scratch[FFN_B200_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
std::once_flag g_setup_once[kMaxDevices];
unsigned char* g_scratch[kMaxDevices];
int g_setup_rc[kMaxDevices];

int64_t round_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Once per device, with that device current: the array's device address.
int scratch_for_device(int dev, unsigned char** out) {
  if (dev < 0 || dev >= kMaxDevices) return FFN_B200_ERR_DEVICE;
  std::call_once(g_setup_once[dev], [dev] {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr) {
      cudaGetLastError();
      g_setup_rc[dev] = FFN_B200_ERR_CUDA;
      return;
    }
    g_scratch[dev] = static_cast<unsigned char*>(ptr);
    g_setup_rc[dev] = FFN_B200_OK;
  });
  *out = g_scratch[dev];
  return g_setup_rc[dev];
}

}  // namespace

extern "C" int ffn_b200_run_noalloc(const ffn_b200_problem* problem, const void* x, int64_t ldx, const void* w1,
                                    int64_t ldw1, const void* w2, int64_t ldw2, void* y, int64_t ldy,
                                    int32_t* status, void* stream) {
  using namespace ffnb200;
  if (!problem || !x || !w1 || !w2 || !y) return FFN_B200_ERR_INVALID;
  if (!aligned16(x) || !aligned16(w1) || !aligned16(w2) || !aligned16(y)) return FFN_B200_ERR_ALIGNMENT;
  if (status && (reinterpret_cast<uintptr_t>(status) & 3u)) return FFN_B200_ERR_ALIGNMENT;
  const int64_t lds[] = {ldx, ldw1, ldw2, ldy};
  for (int64_t v : lds)
    if (v <= 0 || (v % 8) != 0) return FFN_B200_ERR_ALIGNMENT;
  if (ldx < problem->k || ldw1 < problem->k || ldw2 < problem->h || ldy < problem->n) return FFN_B200_ERR_INVALID;

  int dev = 0, sm = 0, ccmaj = 0, ccmin = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FFN_B200_ERR_CUDA;
  int rc = ffn_b200_device_info(dev, &sm, &ccmaj, &ccmin);
  if (rc) return rc;
  if (ccmaj != 10 || ccmin != 0) return FFN_B200_ERR_DEVICE;
  ffn_b200_problem prob = *problem;
  prob.sm_count = sm;
  if (prob.block_num > sm) return FFN_B200_ERR_DEVICE;
  if (prob.tile_variant == 5 || prob.tile_variant == 13) return FFN_B200_ERR_INVALID;  // cluster-launched tiles
  if (prob.weight_format != FFN_B200_WEIGHTS_NATIVE) return FFN_B200_ERR_INVALID;  // no scale arguments here
  // SwiGLU's W1 row order depends on the chosen tiles, which this entry point may change.
  if (prob.gelu == FFN_B200_SWIGLU) return FFN_B200_ERR_INVALID;
  ffn_b200_plan plan;
  rc = ffn_b200_make_plan(&prob, &plan);
  if (rc) return rc;
  if (plan.cta_pair) {  // automatic choice of CTA-pair tiles: use the one-CTA 128x256 tiles here
    prob.tile_variant = 1;
    rc = ffn_b200_make_plan(&prob, &plan);
    if (rc) return rc;
  }
  if (internal_is_hslice(plan.variant)) {  // automatic hidden-slice decode: the swap-AB 16-token tiles here
    prob.tile_variant = 3;
    rc = ffn_b200_make_plan(&prob, &plan);
    if (rc) return rc;
  }

  // Scratch layout: hidden [M, ldh] | fp32 partials | counters | flags | status, 256-B aligned.
  // The row-block kernel (full_load_a) keeps hidden on chip and needs no hidden scratch.
  const bool rowblock = internal_is_rowblock(plan.variant);
  const int64_t ldh = round_up(prob.h, 8);
  const int64_t off_ws = rowblock ? 0 : round_up(prob.m * ldh * 2, 256);
  const int64_t off_cnt = off_ws + round_up(plan.workspace_floats * 4, 256);
  const int64_t off_flg = off_cnt + round_up(plan.counter_words * 4, 256);
  const int64_t off_st = off_flg + round_up(plan.flag_words * 4, 256);
  const int64_t total = off_st + 256;
  if (total > FFN_B200_NOALLOC_SCRATCH_BYTES) return FFN_B200_ERR_SCRATCH;

  unsigned char* base = nullptr;
  rc = scratch_for_device(dev, &base);
  if (rc) return rc;
  void* hidden = base;
  float* ws = reinterpret_cast<float*>(base + off_ws);
  unsigned* counters = reinterpret_cast<unsigned*>(base + off_cnt);
  unsigned* flags = reinterpret_cast<unsigned*>(base + off_flg);
  int* st = status ? status : reinterpret_cast<int*>(base + off_st);

  Params P;
  std::memset(&P, 0, sizeof(P));
  const int dt = prob.dtype;
  const uint32_t bn = static_cast<uint32_t>(plan.tile_n);
  if (rowblock) {
    rc = internal_encode_2d(&P.tm_a_up, x, dt, prob.k, prob.m, ldx, 64, 128);
    if (!rc) rc = internal_encode_2d(&P.tm_b_up, w1, dt, prob.k, prob.h, ldw1, 64, 128);
    if (!rc) rc = internal_encode_2d(&P.tm_b_dn, w2, dt, prob.h, prob.n, ldw2, 64, bn);
    if (!rc) rc = internal_encode_2d(&P.tm_st_y, y, dt, prob.n, prob.m, ldy, 64, kStoreRows);
  } else if (!plan.swap_ab) {
    rc = internal_encode_2d(&P.tm_a_up, x, dt, prob.k, prob.m, ldx, 64, 128);
    if (!rc) rc = internal_encode_2d(&P.tm_b_up, w1, dt, prob.k, prob.h, ldw1, 64, bn);
    if (!rc) rc = internal_encode_2d(&P.tm_a_dn, hidden, dt, prob.h, prob.m, ldh, 64, 128);
    if (!rc) rc = internal_encode_2d(&P.tm_b_dn, w2, dt, prob.h, prob.n, ldw2, 64, bn);
    if (!rc) rc = internal_encode_2d(&P.tm_st_hid, hidden, dt, prob.h, prob.m, ldh, 64, kStoreRows);
    if (!rc) rc = internal_encode_2d(&P.tm_st_y, y, dt, prob.n, prob.m, ldy, 64, kStoreRows);
  } else {
    rc = internal_encode_2d(&P.tm_a_up, w1, dt, prob.k, prob.h, ldw1, 64, 128);
    if (!rc) rc = internal_encode_2d(&P.tm_b_up, x, dt, prob.k, prob.m, ldx, 64, bn);
    if (!rc) rc = internal_encode_2d(&P.tm_a_dn, w2, dt, prob.h, prob.n, ldw2, 64, 128);
    if (!rc) rc = internal_encode_2d(&P.tm_b_dn, hidden, dt, prob.h, prob.m, ldh, 64, bn);
  }
  if (rc) return rc;
  auto to_sched = [](const ffn_b200_phase_plan& pp) {
    PhaseSched s;
    s.tiles_r = pp.tiles_r; s.tiles_q = pp.tiles_q; s.T = pp.tiles; s.L = pp.k_blocks;
    s.dp = pp.dp_tiles; s.sk = pp.sk_tiles; s.q = pp.sk_iters; s.rem = pp.sk_rem; s.group = pp.group;
    s.skc = pp.sk_ctas;
    return s;
  };
  P.hidden = hidden;
  P.y = y;
  P.ldh = ldh;
  P.ldy = ldy;
  P.ws = ws;
  P.claims = reinterpret_cast<unsigned long long*>(counters);
  P.launches = reinterpret_cast<unsigned long long*>(counters + 4);
  P.counters = counters + ffnb200::kClaimWords;
  P.dyn = plan.schedule == 2 ? 1 : 0;
  P.flags = flags;
  P.status = st;
  P.up = to_sched(plan.up);
  P.dn = to_sched(plan.down);
  P.rb_split = plan.row_split;
  P.kserp = plan.swap_ab ? 0 : 1;  // the same K order as a prepared handle
  P.M = static_cast<int>(prob.m);
  P.H = static_cast<int>(prob.h);
  P.N = static_cast<int>(prob.n);
  P.C = plan.block_num;
  P.wait_limit_ns = 4000000000ull;
  P.inject = 0;
  P.l2_hints = prob.l2_policy == 2 ? 1 : (prob.l2_policy == 3 ? 2 : (prob.l2_policy == 4 ? 3 : 0));

  cudaStream_t sh = static_cast<cudaStream_t>(stream);
  // Everything the kernel counts from zero starts at zero: counters, flags, status.
  if (cudaMemsetAsync(counters, 0, static_cast<size_t>(off_st - off_cnt), sh) != cudaSuccess ||
      cudaMemsetAsync(st, 0, 4 * sizeof(int), sh) != cudaSuccess) {
    cudaGetLastError();
    return FFN_B200_ERR_CUDA;
  }
  void (*kernel)(const Params) = internal_kernel_for(plan.variant, dt == FFN_B200_BF16, prob.gelu);
  if (!kernel) return FFN_B200_ERR_INVALID;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(plan.smem_bytes)) !=
      cudaSuccess) {
    cudaGetLastError();
    return FFN_B200_ERR_CUDA;
  }
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(static_cast<unsigned>(plan.block_num), 1, 1);
  cfg.blockDim = dim3(static_cast<unsigned>(internal_threads_for(plan.variant)), 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(plan.smem_bytes);
  cfg.stream = sh;
  cudaLaunchAttribute attr[1];
  if (rowblock && plan.row_split > 1) {  // a cluster per split row block
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(plan.row_split);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
  } else {
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, kernel, P) != cudaSuccess) {
    cudaGetLastError();
    return FFN_B200_ERR_CUDA;
  }
  return FFN_B200_OK;
}
