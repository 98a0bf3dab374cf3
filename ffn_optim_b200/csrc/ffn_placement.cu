// Work-list placement for CTA-pair plans.
//
// The persistent kernel hands tile t of a wave to work-list owner t mod C, and the raster
// makes owners with neighbouring indices share operand strips (the tiles of one B column
// run on `group` consecutive owners).  Which SMs those owners run on depends on how the
// block scheduler places the launch:
//   * a cooperative one-CTA launch fills the GPU GPC by GPC, so consecutive CTAs sit in the
//     same GPC (and die);
//   * a launch with 2-CTA clusters places cluster k on the k-th TPC in SM-id order, which
//     on B200 walks round-robin over the GPCs of both dies.
// With launch-order owners, the CTA-pair kernel therefore spread every B column over all
// GPCs and read 2.5x the DRAM bytes of the one-CTA kernel for the same tiles (L2 hit rate
// of SM reads 71% vs 89%).  Renumbering the pairs in the cooperative launch's GPC-major
// order restores the one-CTA kernel's locality.
//
// The order is measured, not assumed: once per device two probe kernels with the fused
// kernel's launch shape (one CTA per SM through its shared-memory size) record %smid per
// CTA, one launched cooperatively and one with 2-CTA clusters.  Pair k gets the rank of
// its leader's TPC in the cooperative order.  The result is always a permutation of the
// owners, so a placement that differs at run time (another kernel holding SMs) only costs
// locality, never correctness.  The map lives in a static device array (no allocation).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>
#include <numeric>
#include <vector>

namespace ffnb200 {
namespace {

constexpr int kMaxPlacementCtas = 1024;
constexpr int kMaxDevices = 64;

__device__ int32_t g_pair_owner_map[kMaxPlacementCtas / 2];
__device__ int32_t g_probe_smid[2][kMaxPlacementCtas];

__global__ void ffn_placement_probe(int32_t* smids) {
  if (threadIdx.x == 0) {
    uint32_t s;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(s));
    smids[blockIdx.x] = static_cast<int32_t>(s);
  }
}

struct DevicePlacement {
  std::once_flag once;
  const int32_t* map = nullptr;  // device address of g_pair_owner_map, or null
  int grid = 0;
};
DevicePlacement g_placement[kMaxDevices];

// Launches both probes on a private stream and returns the per-CTA SM ids, or an empty
// vector on any CUDA error (cleared).
bool probe_placement(int grid, int smem, std::vector<int32_t>& coop, std::vector<int32_t>& pair) {
  void* base = nullptr;
  if (cudaGetSymbolAddress(&base, g_probe_smid) != cudaSuccess) return false;
  int32_t* s_coop = static_cast<int32_t*>(base);
  int32_t* s_pair = s_coop + kMaxPlacementCtas;
  if (cudaFuncSetAttribute(ffn_placement_probe, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return false;
  cudaStream_t st;
  if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) return false;
  bool ok = cudaMemsetAsync(base, 0xff, sizeof(int32_t) * 2 * kMaxPlacementCtas, st) == cudaSuccess;
  if (ok) {
    void* args[] = {&s_coop};
    ok = cudaLaunchCooperativeKernel(reinterpret_cast<void*>(ffn_placement_probe), dim3(grid), dim3(32), args,
                                     static_cast<size_t>(smem), st) == cudaSuccess;
  }
  if (ok) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
    cfg.blockDim = dim3(32, 1, 1);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ok = cudaLaunchKernelEx(&cfg, ffn_placement_probe, s_pair) == cudaSuccess;
  }
  coop.assign(grid, -1);
  pair.assign(grid, -1);
  if (ok) ok = cudaMemcpyAsync(coop.data(), s_coop, sizeof(int32_t) * grid, cudaMemcpyDeviceToHost, st) == cudaSuccess;
  if (ok) ok = cudaMemcpyAsync(pair.data(), s_pair, sizeof(int32_t) * grid, cudaMemcpyDeviceToHost, st) == cudaSuccess;
  if (cudaStreamSynchronize(st) != cudaSuccess) ok = false;
  cudaStreamDestroy(st);
  return ok;
}

}  // namespace

// Pair k -> work-list owner, from the two probe placements.  Pairs whose TPC the
// cooperative launch did not use keep their launch order after all others.
std::vector<int32_t> pair_owner_order(const std::vector<int32_t>& coop, const std::vector<int32_t>& pair) {
  const int pairs = static_cast<int>(pair.size()) / 2;
  std::vector<int> tpc_rank;
  int next = 0;
  for (int32_t s : coop) {
    if (s < 0) continue;
    const int tpc = s / 2;
    if (tpc >= static_cast<int>(tpc_rank.size())) tpc_rank.resize(tpc + 1, -1);
    if (tpc_rank[tpc] < 0) tpc_rank[tpc] = next++;
  }
  std::vector<long long> key(pairs);
  for (int k = 0; k < pairs; ++k) {
    const int s = pair[2 * k];
    const int tpc = s < 0 ? -1 : s / 2;
    const bool known = tpc >= 0 && tpc < static_cast<int>(tpc_rank.size()) && tpc_rank[tpc] >= 0;
    key[k] = known ? tpc_rank[tpc] : static_cast<long long>(next) + k;
  }
  std::vector<int32_t> by_key(pairs);
  std::iota(by_key.begin(), by_key.end(), 0);
  std::stable_sort(by_key.begin(), by_key.end(), [&](int a, int b) { return key[a] < key[b]; });
  std::vector<int32_t> owner(pairs);
  for (int pos = 0; pos < pairs; ++pos) owner[by_key[pos]] = pos;
  return owner;
}

// Device address of the pair owner map for a full-GPU pair grid on `device` (the current
// device), or null when the grid is not one CTA per SM or probing failed.
const int32_t* internal_pair_owner_map(int device, int grid, int smem) {
  if (device < 0 || device >= kMaxDevices || grid <= 0 || grid > kMaxPlacementCtas || (grid & 1)) return nullptr;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms != grid) {
    cudaGetLastError();
    return nullptr;
  }
  DevicePlacement& dp = g_placement[device];
  std::call_once(dp.once, [&] {
    std::vector<int32_t> coop, pair;
    if (!probe_placement(grid, smem, coop, pair)) {
      cudaGetLastError();
      return;
    }
    const std::vector<int32_t> owner = pair_owner_order(coop, pair);
    void* addr = nullptr;
    if (cudaGetSymbolAddress(&addr, g_pair_owner_map) != cudaSuccess ||
        cudaMemcpyToSymbol(g_pair_owner_map, owner.data(), sizeof(int32_t) * owner.size()) != cudaSuccess) {
      cudaGetLastError();
      return;
    }
    dp.map = static_cast<const int32_t*>(addr);
    dp.grid = grid;
  });
  return dp.grid == grid ? dp.map : nullptr;
}

}  // namespace ffnb200
