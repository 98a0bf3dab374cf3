// Fused FFN kernel for sm_100a:  hidden = GELU(X . W1^T) ;  Y = hidden . W2^T  -- one launch.
//
// Replaces the two Ascend kernels of the reference (ops/kernel/ffn.py:55-585 "basic" and
// ops/kernel/ffn.py:588-1423 "streamk").  Same arithmetic contract: fp16/bf16 operands,
// fp32 accumulation, GELU in fp32 rounded once to the input dtype for the hidden tensor,
// down-projection accumulated in fp32 and rounded once to the input dtype.
//
// Design (one persistent CTA per SM, 6 warps, warp-specialised):
//   warp 0      TMA producer: 128B-swizzled A/B tiles into an S-stage shared-memory ring.
//   warp 1      MMA issuer: tcgen05.mma (kind::f16, cta_group::1, M=128) into one of two
//               TMEM accumulators; owns the TMEM allocation.
//   warps 2..5  epilogue: tcgen05.ld TMEM -> registers -> (Stream-K fixup) -> GELU / cast ->
//               swizzled shared staging -> TMA store (or direct stores in swap mode).
//
// Work list of each CTA (static, identical for all three roles):
//   up DP tiles, up Stream-K parts, down DP tiles, down Stream-K parts.
// A down tile may start only when every up tile of its hidden row block has been stored:
// the reference's global AIC/AIV rendezvous (ops/kernel/ffn.py:373-376, 582-585) becomes a
// per-row-block readiness counter (release/acquire at GPU scope, bounded spin).  Counters
// grow monotonically with the launch epoch, so they are never cleared between launches.
//
// Stream-K (reference ops/kernel/ffn.py:642-665 split, 1240-1422 fixup): the T mod C tail
// tiles of a phase have their k-blocks split evenly over all C CTAs.  The CTA that owns a
// tile's k = 0 block keeps its partial in TMEM, waits for the other contributors' fp32
// partials and adds them in ascending CTA order (the reference sums in ascending core
// order), then runs the normal epilogue.  The reduction order is fixed, so results are
// deterministic run to run.
//
// "Swap" mode (M <= 64, decode): the weight rows become the 128-row MMA operand and the
// tokens the MMA N dimension (16 or 64), so the kernel streams weights from HBM on all SMs.
//
// Every wait is bounded by a wall-clock limit (globaltimer); on expiry the kernel records
// an error in status[], raises a CTA-local abort flag, drains its in-flight copies, frees
// TMEM and returns.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace ffnb200 {

constexpr int kBM = 128;          // MMA M (rows of the A operand per tile)
constexpr int kBK = 64;           // K per pipeline stage = one 128-byte swizzle atom of 16-bit data
constexpr int kCtrlThreads = 64;  // warp 0 (TMA producer) + warp 1 (MMA issuer); epilogue warps follow
constexpr int kABytes = kBM * kBK * 2;
constexpr int kStoreRows = 32;    // rows per epilogue warp (one TMEM sub-partition)
constexpr int kStageBufBytes = kStoreRows * 128;  // 32 rows x 64 x 16-bit, 128B-swizzled
constexpr int kMaxRanks = 8;                      // GPUs of one fused reduce-scatter

enum : int { kRoleFull = 0, kRoleOwner = 1, kRoleContrib = 2 };

struct PhaseSched {
  int tiles_r, tiles_q, T, L;  // tile grid, tiles, k-blocks per tile
  int dp, sk, q, rem;          // data-parallel tiles, Stream-K tiles, k-blocks per CTA (+1 if c < rem)
  int group;                   // raster group height in tile rows
  int skc;                     // CTAs sharing the Stream-K tail (the first skc)
};

struct Params {
  CUtensorMap tm_a_up;   // up A operand  (X rows, or W1 rows in swap mode)
  CUtensorMap tm_b_up;   // up B operand  (W1 rows, or X rows in swap mode)
  CUtensorMap tm_a_dn;   // down A operand (hidden rows, or W2 rows in swap mode)
  CUtensorMap tm_b_dn;   // down B operand (W2 rows, or hidden rows in swap mode)
  CUtensorMap tm_st_hid; // hidden store map (normal mode)
  CUtensorMap tm_st_y;   // Y store map (normal mode)
  void* hidden;
  void* y;
  long long ldh, ldy;    // pitches in elements
  float* ws;             // [2][C][ncta][kBM][BN] fp32 partials (one slot per CTA)
  unsigned* counters;    // readiness per token block
  unsigned* flags;       // [2][C][ncta] partial-ready counts (4 per launch)
  int* status;           // [0] code, [1] CTA, [2] aux
  PhaseSched up, dn;
  int M, H, N;
  int C;
  // Launch epoch, kept on the device so that a launch captured in a CUDA graph replays
  // correctly: every CTA adds 1 to `launches` (a u64 that only a reset zeroes), so the CTAs
  // of launch e read (e-1)*grid .. e*grid-1 and all compute e = old / grid + 1.  Counters and
  // flags grow by a fixed amount per launch; their waits compare modulo 2^32 against e.
  unsigned long long* launches;
  unsigned long long wait_limit_ns;
  int inject;
  int l2_hints;          // 1: evict-last on A (row operand), evict-first on B; 2: evict-normal on
                         // both; 3: evict-last on A only
  unsigned long long* trace;  // optional [grid][16]: TraceSlot stamps, then kTrSmid; null = off
  const int* owner_map;       // optional [C]: work-list owner of each CTA (pair), a permutation of
                              // 0..C-1; null = launch order
  unsigned long long* claims;  // [2] per-phase counters of claimed data-parallel tiles; every
                               // launch adds exactly dp + C (one failed claim per owner)
  int dyn;                     // 1: data-parallel tiles are claimed from `claims` in raster order;
                               // 0: owner c takes tiles c, c + C, ...
  const float* w1_scale;       // fp8 weights: per-row fp32 scales of W1 [H] and W2 [N]
  const float* w2_scale;
  const uint16_t* bias1;       // optional [H] / [N] biases in the input dtype, added in fp32 to
  const uint16_t* bias2;       // the hidden sums before the activation / to Y before rounding
  // Fused reduce-scatter of the down phase across `rs_world` GPUs (tensor parallel over H):
  // rank b owns the Y rows of tile rows [b*rs_band_tiles, (b+1)*rs_band_tiles).  A down tile
  // of another rank's band is pushed as a partial (rs_format: 1 fp32; 2 fp32 rounded to 24
  // bits; 0 rounded to the input dtype) into that rank's staging buffer over NVLink; an
  // owner sums the partials of its band in ascending rank order.
  int rb_split;          // row-block kernel: CTAs (a cluster) sharing one row block's H chunks
  int kserp;             // 1: serpentine K order over the waves of data-parallel tiles (see the producer)
  int wave_sync;         // static schedule: wave lag of the bounded-drift order (0 = off, 1 = schedule 3)
  int hs_superblocks;    // hidden-slice decode kernel: super-blocks of (cluster size) x 128 hidden rows
  int hs_nbr;            // hidden-slice decode kernel: 128-row blocks of Y per cluster rank
  int rs_world, rs_rank, rs_band_tiles;
  int rs_format;                   // staged partials: 0 input dtype, 1 fp32, 2 fp32 rounded to 24 bits
  long long rs_lo_off;             // format 2: byte offset of the low-byte plane in a staging buffer
  void* rs_stage[kMaxRanks];       // per rank: [2 parity][world][band tiles][kBM][BN] partials
  unsigned* rs_flags[kMaxRanks];   // per rank: [world][band tiles] push counts (4 per launch)
  CUtensorMap tm_rs[kMaxRanks];    // store maps over each rank's staging, viewed as [rows][BN]
  CUtensorMap tm_rs_lo[kMaxRanks]; // format 2: store maps over the low-byte planes ([rows][BN] bytes)
};

static_assert(sizeof(Params) <= 4096, "kernel parameters must fit the 4 KB parameter space");

// u32 words at the start of the counters buffer: the two u64 tile-claim counters, then the
// u64 launch counter (Params::launches).
constexpr int kClaimWords = 6;

// Per-CTA trace stamps (ns, %globaltimer) written when Params::trace is set.
enum TraceSlot : int {
  kTrStart = 0,       // setup done (barriers, TMEM)
  kTrFirstLoad = 1,   // producer issued its first TMA load
  kTrDownReady = 2,   // producer saw its first down tile's hidden rows ready
  kTrLastLoad = 3,    // producer issued its last load
  kTrLastMma = 4,     // MMA thread committed its last accumulator
  kTrUpStored = 5,    // first epilogue warp finished its last up-phase unit
  kTrFirstDown = 6,   // first epilogue warp got its first down-phase accumulator
  kTrEnd = 7,         // teardown reached
  kTrSmid = 8,        // not a stamp: the SM (%smid) the CTA ran on
  kTrAux1 = 9,        // kernel-specific stamps (hidden-slice kernel: all partials released,
  kTrAux2 = 10,       // reduction pieces landed, Y written)
  kTrAux3 = 11,
  kTrWords = 16       // words per CTA
};

// ------------------------------------------------------------------------------------------
// PTX wrappers
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void fence_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void fence_acq_rel_gpu() {
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_sys_add(unsigned* p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release(unsigned* p, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Programmatic dependent launch: a kernel launched with programmatic stream serialisation
// may start while the previous kernel of the stream is finishing; `griddepcontrol.wait`
// blocks until that kernel has completed and its memory is visible (it returns at once in a
// kernel launched without the attribute).  `launch_dependents` lets the next such kernel be
// scheduled (as SMs free up) before this one ends.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* tm) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}
// TMA tiled load into this CTA's shared memory (no multicast), completion on an mbarrier.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* tm, int c0, int c1,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}
// Same with an L2 eviction-priority policy (from createpolicy).
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const CUtensorMap* tm, int c0, int c1, uint32_t bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(bar), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* tm, uint32_t src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
               ::"l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(src)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Waits until at most `keep` of this thread's newest bulk groups are pending (2, 4 or 8;
// any other count waits for all of them).
__device__ __forceinline__ void bulk_wait_keep(int keep) {
  if (keep == 8) asm volatile("cp.async.bulk.wait_group 8;" ::: "memory");
  else if (keep == 4) asm volatile("cp.async.bulk.wait_group 4;" ::: "memory");
  else if (keep == 2) asm volatile("cp.async.bulk.wait_group 2;" ::: "memory");
  else bulk_wait_all();
}

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem] (+)= A[smem] . B[smem]^T, both K-major, fp32 accumulate.
__device__ __forceinline__ void umma_f16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
      ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(accum)
      : "memory");
}
// Same with the A operand in tensor memory (lane i = row i, two 16-bit K values per
// 32-bit column; K = 16 spans 8 columns).
__device__ __forceinline__ void umma_f16_ta(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n"
      ::"r"(d), "r"(a_tmem), "l"(b), "r"(idesc), "r"(accum)
      : "memory");
}
// Arrive on an mbarrier once every tcgen05 op issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// ---- CTA-pair (cluster of 2, tcgen05 cta_group::2) forms --------------------------------
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Parity wait with acquire at cluster scope: for data that the other CTA of the pair wrote
// into this CTA's shared memory (or read from it) before its release-arrive.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// 8 words to / from a shared-memory slot of this CTA, or (cluster address) of the peer CTA.
__device__ __forceinline__ void st_shared_8(uint32_t addr, const int* v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3])
               : "memory");
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr + 16), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}
__device__ __forceinline__ float4 ld_cluster_f4(uint32_t cluster_addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(cluster_addr)
               : "memory");
  return v;
}
__device__ __forceinline__ void st_cluster_8(uint32_t cluster_addr, const int* v) {
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_addr), "r"(v[0]), "r"(v[1]),
               "r"(v[2]), "r"(v[3])
               : "memory");
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_addr + 16), "r"(v[4]), "r"(v[5]),
               "r"(v[6]), "r"(v[7])
               : "memory");
}
__device__ __forceinline__ void ld_shared_8(uint32_t addr, int* v) {
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]) : "r"(addr)
               : "memory");
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(addr + 16)
               : "memory");
}
// TMA load into this CTA's shared memory whose completion is counted on an mbarrier of
// either CTA of the pair (here: the leader's), no multicast.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* tm, int c0, int c1,
                                                 uint32_t cluster_bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(cluster_bar)
      : "memory");
}
__device__ __forceinline__ void tma_load_2d_pair_hint(uint32_t dst, const CUtensorMap* tm, int c0, int c1,
                                                      uint32_t cluster_bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(cluster_bar), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem of both CTAs] (+)= A[256 rows: 128 in each CTA] . B[N rows: N/2 in each CTA]^T.
__device__ __forceinline__ void umma_f16_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
      ::"r"(d), "l"(a), "l"(b), "r"(idesc), "r"(accum)
      : "memory");
}
// Arrive once on this CTA's mbarrier when the pair MMAs issued so far complete.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// Same, arriving on the mbarrier at this shared-memory offset in both CTAs of the pair
// (tcgen05.commit signal fan-out; this is not a data load and reads no memory).
__device__ __forceinline__ void umma_commit_pair_both(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
               ::"r"(bar), "h"(static_cast<uint16_t>(0x3))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns; the wait is in the same asm block so the
// outputs are never consumed before the load has landed.
// 32 consecutive 32-bit columns of this warp's 32 TMEM lanes from registers; returns after
// the stores are complete (tcgen05.wait::st).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n\t"
      "tcgen05.wait::st.sync.aligned;"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 64 consecutive 32-bit columns of this warp's 32 lanes, with the wait in the same asm block.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* v) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
      "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}
// Two 16-column loads at different column addresses, one wait (in the same asm block, so the
// outputs are never consumed before they have landed).
__device__ __forceinline__ void tmem_ld16x2(uint32_t ta, uint32_t tb, float* va, float* vb) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%32];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%33];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(ta), "r"(tb)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    va[i] = __uint_as_float(r[i]);
    vb[i] = __uint_as_float(r[16 + i]);
  }
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor: K-major tile of 128-byte rows, 128B swizzle, 8-row
// swizzle atoms 1024 B apart (SBO), descriptor version 1 (sm_100).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}
// Instruction descriptor for kind::f16: D fp32, A/B fp16 or bf16, both K-major, M x N.
template <bool BF16, int N, int M>
__host__ __device__ constexpr uint32_t make_idesc() {
  return (1u << 4) | ((BF16 ? 1u : 0u) << 7) | ((BF16 ? 1u : 0u) << 10) |
         (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// ------------------------------------------------------------------------------------------
// Epilogue arithmetic
// ------------------------------------------------------------------------------------------
// The reference kernel's GELU: 0.5 z (1 + erf~(clip(z/sqrt2, +-3.92))), erf~ = t P(t^2) / Q(t^2)
// with degree-5 P and Q.  Coefficients as in ops/kernel/ffn.py:556-566 and
// validation/reference.py:5-13 (the reference's own published approximation).
__device__ __forceinline__ float gelu_rational(float z) {
  float t = fminf(fmaxf(z * 0.70710678118654752f, -3.92f), 3.92f);
  float t2 = t * t;
  float p = fmaf(t2, 0.053443748819f, 7.5517016694f);
  p = fmaf(p, t2, 101.62808918f);
  p = fmaf(p, t2, 1393.8061484f);
  p = fmaf(p, t2, 5063.7915060f);
  p = fmaf(p, t2, 29639.384698f);
  p *= t;
  float q = t2 + 31.212858877f;
  q = fmaf(q, t2, 398.56963806f);
  q = fmaf(q, t2, 3023.1248150f);
  q = fmaf(q, t2, 13243.365831f);
  q = fmaf(q, t2, 26267.224157f);
  return 0.5f * z * (1.0f + __fdividef(p, q));
}
__device__ __forceinline__ float gelu_erf(float z) {
  return 0.5f * z * (1.0f + erff(z * 0.70710678118654752f));
}
// SiLU (the swish activation): z * sigmoid(z) with CUDA's __expf and __fdividef.
__device__ __forceinline__ float silu(float z) { return __fdividef(z, 1.0f + __expf(-z)); }
// Activation of the hidden layer: 0 the rational GELU, 1 the exact-erf GELU, 2 SiLU;
// 3 is SwiGLU (SiLU(gate) * up over a gate/up-packed W1), handled in the epilogues.
template <int GELU>
__device__ __forceinline__ float gelu(float z) {
  if constexpr (GELU == 0) return gelu_rational(z);
  else if constexpr (GELU == 1) return gelu_erf(z);
  else return silu(z);
}
// Packed fp32 pairs (sm_100 fma/mul/add .f32x2): each lane is one IEEE fp32 operation
// rounded to nearest, so a pair evaluates exactly what two scalar operations would.
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t r, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_splat(float c) { return f2_pack(c, c); }
// gelu_rational on two values at once: the same operations in the same order (the clip
// and the division per lane), with the Horner steps and products packed.
__device__ __forceinline__ void gelu_rational2(float& z0, float& z1) {
  const uint64_t z = f2_pack(z0, z1);
  float t0, t1;
  f2_unpack(f2_mul(z, f2_splat(0.70710678118654752f)), t0, t1);
  t0 = fminf(fmaxf(t0, -3.92f), 3.92f);
  t1 = fminf(fmaxf(t1, -3.92f), 3.92f);
  const uint64_t t = f2_pack(t0, t1);
  const uint64_t t2 = f2_mul(t, t);
  uint64_t p = f2_fma(t2, f2_splat(0.053443748819f), f2_splat(7.5517016694f));
  p = f2_fma(p, t2, f2_splat(101.62808918f));
  p = f2_fma(p, t2, f2_splat(1393.8061484f));
  p = f2_fma(p, t2, f2_splat(5063.7915060f));
  p = f2_fma(p, t2, f2_splat(29639.384698f));
  p = f2_mul(p, t);
  uint64_t q = f2_add(t2, f2_splat(31.212858877f));
  q = f2_fma(q, t2, f2_splat(398.56963806f));
  q = f2_fma(q, t2, f2_splat(3023.1248150f));
  q = f2_fma(q, t2, f2_splat(13243.365831f));
  q = f2_fma(q, t2, f2_splat(26267.224157f));
  float p0, p1, q0, q1;
  f2_unpack(p, p0, p1);
  f2_unpack(q, q0, q1);
  const uint64_t r = f2_pack(1.0f + __fdividef(p0, q0), 1.0f + __fdividef(p1, q1));
  f2_unpack(f2_mul(f2_mul(f2_splat(0.5f), z), r), z0, z1);
}
template <int GELU>
__device__ __forceinline__ void gelu2(float& a, float& b) {
  if constexpr (GELU == 0) {
    gelu_rational2(a, b);
  } else {
    a = gelu<GELU>(a);
    b = gelu<GELU>(b);
  }
}

// Two e4m3 codes (low byte: the lower-addressed element) -> two fp16 (exact) or bf16 (exact:
// every e4m3 value is a normal fp16 and a bf16) in one 32-bit word, low half first.
template <bool BF16>
__device__ __forceinline__ uint32_t e4m3x2_to_16x2(uint32_t two) {
  uint32_t h;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(static_cast<unsigned short>(two & 0xFFFFu)));
  if constexpr (BF16) {
    const __half2 hh = *reinterpret_cast<const __half2*>(&h);
    const float2 f = __half22float2(hh);
    const __nv_bfloat162 b = __floats2bfloat162_rn(f.x, f.y);
    return *reinterpret_cast<const uint32_t*>(&b);
  }
  return h;
}
template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}
template <bool BF16>
__device__ __forceinline__ float unpack_lo(uint32_t w) {
  if constexpr (BF16) return __uint_as_float(w << 16);
  else return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFFu)));
}
template <bool BF16>
__device__ __forceinline__ float unpack_hi(uint32_t w) {
  if constexpr (BF16) return __uint_as_float(w & 0xFFFF0000u);
  else return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
}
template <bool BF16>
__device__ __forceinline__ uint16_t cvt1(float a) {
  if constexpr (BF16) {
    __nv_bfloat16 h = __float2bfloat16_rn(a);
    return *reinterpret_cast<uint16_t*>(&h);
  } else {
    __half h = __float2half_rn(a);
    return *reinterpret_cast<uint16_t*>(&h);
  }
}
// Bias of W consecutive features starting at `c0` (16-bit values, widened to fp32), added to
// v; features at or beyond `count` get none (ragged tiles).  Vector loads when the whole run
// is inside (c0 is a multiple of 64 and the bias 16-byte aligned).
template <bool BF16, int W>
__device__ __forceinline__ void add_bias(float* v, const uint16_t* bias, int c0, int count) {
  if (c0 + W <= count) {
#pragma unroll
    for (int q = 0; q < W / 8; ++q) {
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(bias + c0) + q);
      const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        v[8 * q + 2 * e] += unpack_lo<BF16>(wv[e]);
        v[8 * q + 2 * e + 1] += unpack_hi<BF16>(wv[e]);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < W; ++j)
      if (c0 + j < count) v[j] += unpack_lo<BF16>(static_cast<uint32_t>(__ldg(bias + c0 + j)));
  }
}

// ------------------------------------------------------------------------------------------
// Schedule
// ------------------------------------------------------------------------------------------
struct Unit {
  int phase;     // 0 up, 1 down
  int tile;      // raster index in [0, T)
  int kb0, kb1;  // k-block range
  int role;      // kRoleFull / kRoleOwner / kRoleContrib
  int c_first, c_last;  // contributors whose partials an owner adds (ascending)
  int rev;       // 1: the producer loads the k-blocks in descending order
};

__device__ __forceinline__ int sk_start(const PhaseSched& s, int c) { return c * s.q + min(c, s.rem); }
__device__ __forceinline__ int sk_cta_of(const PhaseSched& s, int i) {
  const int big = s.rem * (s.q + 1);
  if (i < big) return i / (s.q + 1);
  return s.rem + (i - big) / s.q;
}
// Grouped raster: within a group of `group` tile rows, walk rows fastest then columns.
__device__ __forceinline__ void tile_coords(const PhaseSched& s, int t, int& tr, int& tq) {
  const int per_group = s.group * s.tiles_q;
  const int g = t / per_group;
  const int rem = t - g * per_group;
  const int r0 = g * s.group;
  const int gs = min(s.group, s.tiles_r - r0);
  tr = r0 + rem % gs;
  tq = rem / gs;
}
// Tile coordinates of a unit.  Under the fused reduce-scatter every rank visits the down
// phase's bands of tile rows starting after its own band, so pushes to the other ranks go
// out first and its own band, which waits for their partials, comes last.
__device__ __forceinline__ void unit_coords(const Params& p, const Unit& u, int& tr, int& tq) {
  const PhaseSched& s = u.phase ? p.dn : p.up;
  tile_coords(s, u.tile, tr, tq);
  if (u.phase == 1 && p.rs_world > 1) tr = (tr + (p.rs_rank + 1) * p.rs_band_tiles) % s.tiles_r;
}

// Data-parallel tile t of a phase: the whole K range in one unit.
__device__ __forceinline__ void dp_unit(const PhaseSched& s, int ph, int t, Unit& u) {
  u.phase = ph; u.tile = t; u.kb0 = 0; u.kb1 = s.L;
  u.role = kRoleFull; u.c_first = 1; u.c_last = 0; u.rev = 0;
}
// Stream-K part `idx` of owner c in a phase (static split of the tail tiles' K blocks).
__device__ __forceinline__ bool sk_unit(const PhaseSched& s, int ph, int c, int idx, Unit& u) {
  if (s.sk <= 0 || c >= s.skc) return false;
  const int st = sk_start(s, c);
  const int en = sk_start(s, c + 1);
  if (en <= st) return false;
  const int n_sk = (en - 1) / s.L - st / s.L + 1;
  if (idx >= n_sk) return false;
  const int trel = st / s.L + idx;
  const int tb = trel * s.L, te = tb + s.L;
  const int a = max(st, tb), b = min(en, te);
  u.phase = ph; u.tile = s.dp + trel; u.kb0 = a - tb; u.kb1 = b - tb; u.rev = 0;
  if (a == tb) {
    u.role = kRoleOwner; u.c_first = c + 1; u.c_last = sk_cta_of(s, te - 1);
  } else {
    u.role = kRoleContrib; u.c_first = 1; u.c_last = 0;
  }
  return true;
}
// A unit as the 8 words of a unit-ring slot; word 7 = 1 + rev for a unit, 0 for end of work.
__device__ __forceinline__ void pack_unit(const Unit& u, int* w) {
  w[0] = u.phase; w[1] = u.tile; w[2] = u.kb0; w[3] = u.kb1;
  w[4] = u.role; w[5] = u.c_first; w[6] = u.c_last; w[7] = 1 + u.rev;
}
__device__ __forceinline__ void unpack_unit(const int* w, Unit& u) {
  u.phase = w[0]; u.tile = w[1]; u.kb0 = w[2]; u.kb1 = w[3];
  u.role = w[4]; u.c_first = w[5]; u.c_last = w[6]; u.rev = w[7] - 1;
}

__device__ __forceinline__ void trace_mark(const Params& p, int slot) {
  if (p.trace) p.trace[static_cast<size_t>(blockIdx.x) * kTrWords + slot] = gtimer();
}

__device__ __forceinline__ void report(const Params& p, int code, int aux) {
  if (atomicCAS(p.status, 0, code) == 0) {
    p.status[1] = static_cast<int>(blockIdx.x);
    p.status[2] = aux;
  }
}

// Bounded mbarrier wait.  Returns false when the CTA aborts (timeout here or elsewhere).
// On-chip pipeline waits get twice the limit of the cross-CTA waits below: when a readiness
// counter or Stream-K flag never arrives, that wait (the cause) expires and reports first,
// not the pipeline stages stalled behind it.
template <bool CL = false>
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                         const Params& p, int aux) {
  auto try_wait = [&]() { return CL ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity); };
  if (try_wait()) return true;
  const uint64_t t0 = gtimer();
  uint32_t n = 0;
#pragma unroll 1
  while (true) {
    if (try_wait()) return true;
    if ((++n & 15u) == 0) {
      if (*abort_flag) return false;
      if (gtimer() - t0 > 2 * p.wait_limit_ns) {
        report(p, 1, aux);
        *abort_flag = 1;
        return false;
      }
    }
  }
}
// Bounded wait until *word >= target (wrapping compare).  Acquire at GPU scope, or at
// system scope (SYS) for words written by peer GPUs.
template <bool SYS = false>
__device__ __forceinline__ bool wait_word_ge(const unsigned* word, unsigned target, volatile int* abort_flag,
                                             const Params& p, int code, int aux) {
  auto load = [&]() { return SYS ? ld_acquire_sys(word) : ld_acquire(word); };
  if (static_cast<int>(load() - target) >= 0) return true;
  const uint64_t t0 = gtimer();
#pragma unroll 1
  while (true) {
    __nanosleep(64);
    if (static_cast<int>(load() - target) >= 0) return true;
    if (*abort_flag) return false;
    if (gtimer() - t0 > p.wait_limit_ns) {
      report(p, code, aux);
      *abort_flag = 1;
      return false;
    }
  }
}

// ------------------------------------------------------------------------------------------
// The kernel
// ------------------------------------------------------------------------------------------
template <int BN, int STAGES, bool SWAP, bool PAIR = false, int KSUB = 1, int EPI = 4, bool W8 = false>
struct Layout {
  static constexpr int kEpiWarps = EPI;             // 4, or 8 = two warps per TMEM sub-partition
  // fp8 -> 16-bit weight converters: kCvtGroups groups of 4 warps (one per SMSP) take the
  // k-blocks in turn, so that many k-blocks are in conversion at once.
  static constexpr int kCvtGroups = W8 ? 3 : 0;
  static constexpr int kCvtWarps = 4 * kCvtGroups;
  static constexpr int kThreads = kCtrlThreads + 32 * (EPI + kCvtWarps);
  static constexpr int kQStage = W8 ? KSUB * kBM * kBK : 0;  // one fp8 weight k-block (128 rows x 64*KSUB bytes)
  static constexpr int kNcta = PAIR ? 2 : 1;       // CTAs per tile (cluster size)
  static constexpr int kBRows = BN / kNcta;         // B rows each CTA loads per stage
  static constexpr int kBSub = kBRows * kBK * 2;    // one 64-wide K sub-block of B
  static constexpr int kAStage = KSUB * kABytes;    // a stage holds KSUB adjacent K sub-blocks
  static constexpr int kBStage = KSUB * kBSub;
  // W8: the widened weight tiles (A) live in TMEM and B in its own ring: no smem stages.
  static constexpr int kStageBytes = W8 ? 0 : kAStage + kBStage;
  static constexpr int kEpiBytes = SWAP ? 0 : EPI * 2 * kStageBufBytes;
  static constexpr int kBarBytes = W8 ? 1024 : 256;
  // Unit ring: the leader's producer publishes each unit it takes (a claimed or static tile)
  // for the MMA issuer, the epilogue warps and, in a pair, the peer CTA.  Deep enough that
  // the producer (at most STAGES k-blocks ahead of the MMA, which is at most two
  // accumulators ahead of the epilogue) never waits on it in steady state.
  static constexpr int kRing = 16;
  static constexpr int kRingBytes = kRing * 32 + 2 * kRing * 8;  // slots, full and empty barriers
  // MMA + epilogue warps (+ peer's producer and epilogue, + converter warps)
  static constexpr int kRingConsumers = (PAIR ? 2 + 2 * EPI : 1 + EPI) + kCvtWarps;
  // W8: a ring of fp8 weight k-blocks deeper than the MMA stages (the bytes in flight set the
  // HBM rate of the weight stream), 1024-aligned after the barriers and the unit ring.
  // The token operand (B) then has its own ring of the same depth, read by the MMA in place,
  // so the MMA stages hold only the widened weights and no memory latency sits in their cycle.
  // (a converter's slot waits stay unambiguous while kQSlots >= STAGES + kCvtGroups + 1)
  static constexpr int kQSlots = W8 ? (BN <= 16 ? 10 : 9) : 0;
  static constexpr int kBSlots = W8 ? (BN <= 16 ? 10 : 4) : 0;  // (one producer, one in-order consumer)
  static constexpr int kQOffset = (kBarBytes + kRingBytes + 1023) / 1024 * 1024;  // from the barrier area
  static constexpr int kBRingOffset = kQOffset + kQSlots * kQStage;
  static constexpr int kSmem = 1024 /*align slack*/ + STAGES * kStageBytes + kEpiBytes +
                               (W8 ? kBRingOffset + kBSlots * kBStage : kBarBytes + kRingBytes);
  static_assert(kSmem <= 232448, "dynamic shared memory per CTA");
  // W8: two accumulators then STAGES weight tiles of 32 columns (128 rows x 64 16-bit K).
  // Decode (swap-AB) tiles have N = 16 or 64: one MMA does little work, and MMAs that add
  // into the same accumulator run one after the other, so their latency, not the tensor
  // pipe, would set the pace.  K-step i therefore adds into chain i mod kChains, an
  // accumulator of its own; the epilogue sums the chains in a fixed order.
  static constexpr int kChains = SWAP ? (BN <= 16 ? 4 : 2) : 1;
  static constexpr int kAccCols = kChains * BN;  // one accumulator buffer
  static constexpr int kTmemCols = W8 ? 512 : (2 * kAccCols < 32 ? 32 : 2 * kAccCols);
  static constexpr int kTmemA = 32 * KSUB;  // W8: TMEM columns of one widened weight k-block
  static_assert(!W8 || 2 * kAccCols + kTmemA * STAGES <= 512, "TMEM: accumulators and weight stages");
  static_assert(kChains <= 4 * KSUB, "every chain gets a K step from each k-block");
  static_assert(!W8 || (kQSlots >= STAGES + kCvtGroups + 1 && kCvtGroups <= STAGES), "ring depths");
  static_assert((kBSub % 1024) == 0, "B tile must be whole swizzle atoms");
  // (the last 16 bytes hold the epoch barrier and the launch epoch)
  static_assert((W8 ? 2 * STAGES + 6 + 2 * kQSlots + 2 * kBSlots : 2 * STAGES + 5) * 8 + 8 <= kBarBytes - 16,
                "barrier area");
  static_assert(!W8 || (SWAP && !PAIR && (KSUB == 1 || KSUB == 2)), "fp8 weights: swap-AB decode tiles");
  static_assert(!PAIR || !SWAP, "CTA pairs are used for prefill tiles only");
  static_assert(EPI == 4 || EPI == 8, "epilogue warps: one or two per TMEM sub-partition");
};

// PAIR = true: a cluster of two CTAs computes one 256 x BN tile with tcgen05 cta_group::2.
// Each CTA loads 128 rows of A and BN/2 rows of B into its own shared memory (plain TMA
// loads, no multicast) and completes the transaction bytes on the leader's (rank 0) full
// barrier; the leader's MMA thread issues the pair MMAs, whose D lands 128 rows in each
// CTA's TMEM, and its tcgen05.commit arrives on the empty / tmem-full barriers of both CTAs;
// each CTA's epilogue stores its own 128 rows and releases the accumulator on the leader.
template <int BN, int STAGES, bool SWAP, bool PAIR, int KSUB, int EPI, bool BF16, int GELU, bool W8 = false>
__global__ void __launch_bounds__(kCtrlThreads + 32 * (EPI + (W8 ? 12 : 0)), 1)
    ffn_fused_kernel(const __grid_constant__ Params p) {
  using LY = Layout<BN, STAGES, SWAP, PAIR, KSUB, EPI, W8>;
  constexpr int kParts = EPI / 4;  // epilogue warps per TMEM sub-partition, each takes a column share
  // Swap mode reads TMEM in chunks of kCW token columns; normal mode in 64-column chunks.
  constexpr int kCW = SWAP ? (BN / kParts < 16 ? BN / kParts : 16) : 64;
  constexpr int kChunks = BN / kCW;
  static_assert(kChunks % kParts == 0, "column chunks split evenly over the warps of a sub-partition");
  constexpr int kNcta = LY::kNcta;
  constexpr int kTileM = kBM * kNcta;
  // W8 multiplies fp16 x fp16: the widened weights are exact in fp16 and the token tiles
  // (16-bit activations) are moved to fp16 in shared memory (bf16 -> fp16 is exact inside
  // fp16's range; a value beyond it is reported as kernel error 6).
  constexpr uint32_t kIdesc = make_idesc<BF16 && !W8, BN, kTileM>();
  static_assert(SWAP || (BN % 64) == 0, "normal mode stores 64-column chunks");
  static_assert(!SWAP || (BN % 16) == 0, "swap mode loads 16-column chunks");

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sA = base;
  const uint32_t sB = sA + STAGES * LY::kAStage;
  const uint32_t sE = W8 ? sA : sB + STAGES * LY::kBStage;  // (W8: no smem stages)
  const uint32_t sBar = sE + LY::kEpiBytes;
  auto full_bar = [&](int s) { return sBar + 8u * s; };
  auto empty_bar = [&](int s) { return sBar + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return sBar + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return sBar + 8u * (2 * STAGES + 2 + a); };
  const uint32_t drain_bar = sBar + 8u * (2 * STAGES + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + (sBar - base) + 8 * (2 * STAGES + 5));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // The launch epoch: published once by the first epilogue warp (one atomic per CTA), read
  // by the roles that wait on counters or flags when they first need it.
  const uint32_t epoch_bar = sBar + LY::kBarBytes - 16;
  volatile unsigned long long* epoch_val =
      reinterpret_cast<volatile unsigned long long*>(gbase + (sBar - base) + LY::kBarBytes - 8);
  auto fetch_epoch = [&](unsigned long long& e) -> bool {
    if (!wait_bar(epoch_bar, 0u, abort_flag, p, 700)) return false;
    e = *epoch_val;
    return true;
  };
  const uint32_t sRing = sBar + LY::kBarBytes;
  const uint32_t sQ = sBar + LY::kQOffset;      // fp8 weight k-blocks (W8), 1024-aligned
  const uint32_t sBR = sBar + LY::kBRingOffset;  // token-operand k-blocks (W8), 1024-aligned
  auto qfull_bar = [&](int j) { return sBar + 8u * (2 * STAGES + 6 + j); };
  auto qempty_bar = [&](int j) { return sBar + 8u * (2 * STAGES + 6 + LY::kQSlots + j); };
  auto bfull_bar = [&](int j) { return sBar + 8u * (2 * STAGES + 6 + 2 * LY::kQSlots + j); };
  auto bempty_bar = [&](int j) { return sBar + 8u * (2 * STAGES + 6 + 2 * LY::kQSlots + LY::kBSlots + j); };
  auto ring_slot = [&](int i) { return sRing + 32u * i; };
  auto ring_full = [&](int i) { return sRing + 32u * LY::kRing + 8u * i; };
  auto ring_empty = [&](int i) { return sRing + 32u * LY::kRing + 8u * (LY::kRing + i); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const bool leader = rank == 0;
  const int slot_base = static_cast<int>(rank);          // partial / flag slot = (phase*C + cta)*kNcta + rank

  if (threadIdx.x == 0) {
#pragma unroll 1
    for (int s = 0; s < STAGES; ++s) {
      // W8: one arrival per warp of the converter group that owns the k-block.
      mbar_init(full_bar(s), W8 ? 4 : 1);
      mbar_init(empty_bar(s), 1);
    }
    if constexpr (W8) {
#pragma unroll 1
      for (int j = 0; j < LY::kQSlots; ++j) {
        mbar_init(qfull_bar(j), 1);
        mbar_init(qempty_bar(j), 4);
      }
#pragma unroll 1
      for (int j = 0; j < LY::kBSlots; ++j) {
        mbar_init(bfull_bar(j), 1);
        mbar_init(bempty_bar(j), 1);
      }
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 32 * EPI * kNcta);
    }
    mbar_init(drain_bar, 1);
    mbar_init(epoch_bar, 1);
#pragma unroll 1
    for (int i = 0; i < LY::kRing; ++i) {
      mbar_init(ring_full(i), 1);
      mbar_init(ring_empty(i), LY::kRingConsumers);
    }
    *abort_flag = 0;
    fence_barrier_init();
    fence_async_shared();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&p.tm_a_up); prefetch_tmap(&p.tm_b_up);
    prefetch_tmap(&p.tm_a_dn); prefetch_tmap(&p.tm_b_dn);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(smem_u32(tmem_slot), LY::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(tmem_slot), LY::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // peer barriers initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Everything above touches on-chip state only; with an overlapped launch it runs while
  // the previous kernel finishes.  Every global access (operands, hidden, counters, flags,
  // partials, status) comes after this wait, so consecutive calls stay ordered.
  if (threadIdx.x == 0) grid_dep_launch();
  grid_dep_wait();
  // Work-list owner (one per tile-sized group of CTAs).
  const int cta = p.owner_map ? p.owner_map[blockIdx.x / kNcta] : static_cast<int>(blockIdx.x) / kNcta;
  if (threadIdx.x == 0) {
    trace_mark(p, kTrStart);
    if (p.trace) {
      uint32_t smid;
      asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
      p.trace[static_cast<size_t>(blockIdx.x) * kTrWords + kTrSmid] = smid;
    }
  }

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      int ready_blk = -1;
      const unsigned per_blk = static_cast<unsigned>(EPI * kNcta) * static_cast<unsigned>(SWAP ? p.up.tiles_r : p.up.tiles_q);
      unsigned long long epoch = 0;  // fetched when first needed (readiness waits, claims)
      unsigned target = 0;
      bool have_epoch = false;
      auto need_epoch = [&]() -> bool {
        if (have_epoch) return true;
        if (!fetch_epoch(epoch)) return false;
        target = static_cast<unsigned>(epoch) * per_blk + (p.inject ? 1u : 0u);
        have_epoch = true;
        return true;
      };
      // Optional L2 policy (off by default: on cfg5 it raised DRAM reads from 62 GB to 430 GB).
      const uint64_t pol_a = p.l2_hints == 2 ? policy_evict_normal() : policy_evict_last();
      const uint64_t pol_b = p.l2_hints == 2 ? policy_evict_normal() : policy_evict_first();
      const bool hints = p.l2_hints != 0 && !SWAP;
      const bool hint_b = p.l2_hints != 3;  // policy 3: hint only the row operand (A)
      // Issues the TMA loads of one unit; false when the CTA aborts.
      auto do_loads = [&](const Unit& u) -> bool {
        int tr, tq;
        unit_coords(p, u, tr, tq);
        const CUtensorMap* ta = u.phase ? &p.tm_a_dn : &p.tm_a_up;
        const CUtensorMap* tb = u.phase ? &p.tm_b_dn : &p.tm_b_up;
        if constexpr (W8) {
          // K-block n: fp8 weights to q slot n mod Q (for the converters), tokens to B slot
          // n mod QB (read by the MMA in place), ahead of the MMA by up to the ring depths.  A
          // down unit's tokens (hidden rows) wait for the rows to be ready; its weights never
          // wait.  One k-block is KSUB x 64 K: 64*KSUB bytes of each weight row per load.
          const int wrow = tr * kTileM;
#pragma unroll 1
          for (int kb = u.kb0; kb < u.kb1; ++kb) {
            const int j = static_cast<int>(issued % LY::kQSlots);
            const uint32_t rpar = static_cast<uint32_t>((issued / LY::kQSlots) & 1);
            if (!wait_bar(qempty_bar(j), rpar ^ 1u, abort_flag, p, 150 + j)) return false;
            mbar_expect_tx(qfull_bar(j), LY::kQStage);
            tma_load_2d(sQ + j * LY::kQStage, ta, kb * kBK * KSUB / 2, wrow, qfull_bar(j));  // (code pairs)
            const int jb = static_cast<int>(issued % LY::kBSlots);
            const uint32_t bpar = static_cast<uint32_t>((issued / LY::kBSlots) & 1);
            if (!wait_bar(bempty_bar(jb), bpar ^ 1u, abort_flag, p, 170 + jb)) return false;
            if (u.phase == 1 && tq != ready_blk) {  // swap mode: the row block is a token block
              if (!need_epoch() || !wait_word_ge(p.counters + tq, target, abort_flag, p, 2, tq)) return false;
              fence_async_global();
              if (ready_blk < 0) trace_mark(p, kTrDownReady);
              ready_blk = tq;
            }
            mbar_expect_tx(bfull_bar(jb), LY::kBStage);
#pragma unroll
            for (int jj = 0; jj < KSUB; ++jj)
              tma_load_2d(sBR + jb * LY::kBStage + jj * LY::kBSub, tb, (kb * KSUB + jj) * kBK, tq * BN, bfull_bar(jb));
            if (issued == 0) trace_mark(p, kTrFirstLoad);
            ++issued;
          }
          return true;
        }
        const int arow = tr * kTileM + static_cast<int>(rank) * kBM;
        const int brow = tq * BN + static_cast<int>(rank) * LY::kBRows;
        // One operand load into stage `st` (which = 0: A, 1: B), with the chosen L2 policy.
        auto load = [&](int which, int st, int kb) {
          const CUtensorMap* tm = which == 0 ? ta : tb;
          const int row = which == 0 ? arow : brow;
#pragma unroll
          for (int j = 0; j < KSUB; ++j) {
            const uint32_t dst = which == 0 ? sA + st * LY::kAStage + j * kABytes : sB + st * LY::kBStage + j * LY::kBSub;
            const int kx = (kb * KSUB + j) * kBK;
            const bool hinted = hints && (which == 0 || hint_b);
            if constexpr (PAIR) {
              const uint32_t fb = map_to_rank(full_bar(st), 0);
              if (hinted) tma_load_2d_pair_hint(dst, tm, kx, row, fb, which == 0 ? pol_a : pol_b);
              else tma_load_2d_pair(dst, tm, kx, row, fb);
            } else {
              if (hinted) tma_load_2d_hint(dst, tm, kx, row, full_bar(st), which == 0 ? pol_a : pol_b);
              else tma_load_2d(dst, tm, kx, row, full_bar(st));
            }
          }
        };
        auto arm = [&](int st) {  // expect both operands' bytes of this stage
          if constexpr (PAIR) {
            if (leader) mbar_expect_tx(full_bar(st), kNcta * LY::kStageBytes);
          } else {
            mbar_expect_tx(full_bar(st), LY::kStageBytes);
          }
        };
        // K-block of step j: ascending, or descending for a reversed unit (the MMA adds the
        // stages in the order they arrive; it never reads the k-block index).
        auto kb_at = [&](int j) { return u.rev ? u.kb1 - 1 - j : u.kb0 + j; };
        const int nk = u.kb1 - u.kb0;
        int j0 = 0;
        if (u.phase == 1) {
          const int blk = SWAP ? tq : tr;
          if (blk != ready_blk) {
            // The hidden rows of this tile are not known to be ready.  The weight operand
            // (W2: A in swap mode, B otherwise) does not depend on them: fill up to STAGES
            // ring slots with it, then wait for the rows and complete those stages with the
            // hidden operand.  (An extra L2 prefetch of W2 here was measured neutral on the
            // bandwidth-bound decode shape: it only moved bytes from the down to the up phase.)
            const int wop = SWAP ? 0 : 1;
            const int n_pre = min(STAGES, nk);
            const int st0 = stage;
            int pre = 0;
            for (; pre < n_pre; ++pre) {
              if (!wait_bar(empty_bar(stage), phase ^ 1u, abort_flag, p, 100 + stage)) return false;
              arm(stage);
              load(wop, stage, kb_at(pre));
              if (issued == 0) trace_mark(p, kTrFirstLoad);
              ++issued;
              if (++stage == STAGES) { stage = 0; phase ^= 1u; }
            }
            if (!need_epoch() || !wait_word_ge(p.counters + blk, target, abort_flag, p, 2, blk)) return false;
            fence_async_global();
            if (ready_blk < 0) trace_mark(p, kTrDownReady);
            ready_blk = blk;
            for (int j = 0; j < pre; ++j) load(1 - wop, (st0 + j) % STAGES, kb_at(j));
            j0 = pre;
          }
        }
#pragma unroll 1
        for (int j = j0; j < nk; ++j) {
          if (!wait_bar(empty_bar(stage), phase ^ 1u, abort_flag, p, 100 + stage)) return false;
          arm(stage);
          load(0, stage, kb_at(j));
          load(1, stage, kb_at(j));
          if (issued == 0) trace_mark(p, kTrFirstLoad);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        return true;
      };
      bool ok = true;
      int seq = 0;  // units published (leader) or taken from the ring (peer)
      if (leader) {
        // Publish a unit (8 words) in this CTA's ring slot and, in a pair, the peer's.
        auto publish = [&](const int* w) -> bool {
          const int slot = seq % LY::kRing;
          const uint32_t par = static_cast<uint32_t>((seq / LY::kRing) & 1);
          if (!wait_bar<PAIR>(ring_empty(slot), par ^ 1u, abort_flag, p, 500 + slot)) return false;
          st_shared_8(ring_slot(slot), w);
          if constexpr (PAIR) {
            st_cluster_8(map_to_rank(ring_slot(slot), 1), w);
            mbar_arrive_cluster(map_to_rank(ring_full(slot), 1));
          }
          mbar_arrive(ring_full(slot));
          ++seq;
          return true;
        };
#pragma unroll 1
        for (int ph = 0; ph < 2 && ok; ++ph) {
          const PhaseSched& s = ph ? p.dn : p.up;
          // Data-parallel tiles.  Owner c's first tile is tile c; under the dynamic schedule
          // every later one is claimed (tile C + claim index) so that the tiles in flight
          // stay a contiguous stretch of the raster however far the owners drift apart.
          // Every owner ends with one failed claim, so each launch advances the counter by
          // exactly max(dp - C, 0) + C.  The next claim is in flight during the loads.
          const long long span = max(s.dp - p.C, 0) + p.C;
          const long long t_end = max(s.dp, p.C) + p.C;  // claimed tiles lie in [C, t_end)
          auto claimed = [&](unsigned long long raw) {  // (after need_epoch)
            return p.C + static_cast<long long>(raw - (epoch - 1ull) * static_cast<unsigned long long>(span));
          };
          long long t = cta;
          bool from_claim = false;
          if (p.dyn && t >= s.dp) {
            const unsigned long long raw = atomicAdd(p.claims + ph, 1ull);
            if (!need_epoch()) { ok = false; break; }
            t = claimed(raw);
            from_claim = true;
          }
#pragma unroll 1
          while (true) {
            if (from_claim && (t < p.C || t >= t_end)) {  // counters not reset after an error
              report(p, 5, ph);
              *abort_flag = 1;
              ok = false;
              break;
            }
            if (t >= s.dp) break;
            if (p.wave_sync > 0 && !p.dyn) {
              // Static order with bounded drift: start wave i = t / C only once every owner has
              // started its tile of wave i - wave_sync (claims[ph] counts started tiles; it
              // grows by exactly dp per launch).  (Lags of 2 and 4 waves measured 7 % and 10 %
              // slower on cfg5 CTA pairs, and synchronising within tiles -- every 16 to 64
              // k-steps -- 15-17 % slower: owners then wait on the slowest at every step.)
              if (!need_epoch()) { ok = false; break; }
              const long long wave = t / p.C;
              if (wave >= p.wave_sync) {
                const unsigned long long want = (epoch - 1ull) * static_cast<unsigned long long>(s.dp) +
                                                static_cast<unsigned long long>((wave - p.wave_sync + 1) * p.C);
                const uint64_t t0 = gtimer();
                uint32_t n = 0;
#pragma unroll 1
                while (static_cast<long long>(*reinterpret_cast<volatile unsigned long long*>(p.claims + ph) - want) < 0) {
                  __nanosleep(128);
                  if ((++n & 15u) == 0) {
                    if (*abort_flag) { ok = false; break; }
                    if (gtimer() - t0 > p.wait_limit_ns) {
                      report(p, 2, 1000 + ph);
                      *abort_flag = 1;
                      ok = false;
                      break;
                    }
                  }
                }
                if (!ok) break;
              }
              atomicAdd(p.claims + ph, 1ull);
            }
            Unit u;
            dp_unit(s, ph, static_cast<int>(t), u);
            // Serpentine K order: the data-parallel tiles of every other wave walk K backwards,
            // so a wave starts on the K-slices the previous wave (the same rows) left in L2.
            u.rev = p.kserp && ((t / p.C) & 1) ? 1 : 0;
            int w[8];
            pack_unit(u, w);
            if (!publish(w)) { ok = false; break; }
            unsigned long long next = 0;
            if (p.dyn) next = atomicAdd(p.claims + ph, 1ull);
            if (!do_loads(u)) { ok = false; break; }
            if (p.dyn) {
              if (!need_epoch()) { ok = false; break; }
              t = claimed(next);
              from_claim = true;
            } else {
              t += p.C;
            }
          }
          // Stream-K parts of this owner.
#pragma unroll 1
          for (int i = 0; ok; ++i) {
            Unit u;
            if (!sk_unit(s, ph, cta, i, u)) break;
            int w[8];
            pack_unit(u, w);
            if (!publish(w) || !do_loads(u)) ok = false;
          }
        }
        if (ok) {
          const int w[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // end of work
          ok = publish(w);
        }
      } else {
        // The peer of a pair loads its halves of the units its leader publishes.
#pragma unroll 1
        while (ok) {
          const int slot = seq % LY::kRing;
          const uint32_t par = static_cast<uint32_t>((seq / LY::kRing) & 1);
          if (!wait_bar<PAIR>(ring_full(slot), par, abort_flag, p, 600 + slot)) { ok = false; break; }
          int w[8];
          ld_shared_8(ring_slot(slot), w);
          mbar_arrive_cluster(map_to_rank(ring_empty(slot), 0));
          ++seq;
          if (!w[7]) break;
          Unit u;
          unpack_unit(w, u);
          if (!do_loads(u)) ok = false;
        }
      }
      trace_mark(p, kTrLastLoad);
      // Drain: every issued load must land before the CTA may exit.  In a pair the
      // transaction bytes land on the leader's barriers, so the leader drains for both.
      // One deadline for the whole drain: after an abort, stages armed for both operands
      // but given only the weight operand never complete, and must not each wait the limit.
      if constexpr (W8) {  // the token loads of the last kBSlots k-blocks land too
        const long long firstb = issued > LY::kBSlots ? issued - LY::kBSlots : 0;
        const uint64_t tb0 = gtimer();
#pragma unroll 1
        for (long long i = firstb; i < issued; ++i) {
          const int jb = static_cast<int>(i % LY::kBSlots);
          const uint32_t par = static_cast<uint32_t>((i / LY::kBSlots) & 1);
          bool late = false;
          while (!mbar_try_wait(bfull_bar(jb), par)) {
            if (gtimer() - tb0 > p.wait_limit_ns) { late = true; break; }
          }
          if (late) break;
        }
      }
      if (leader) {
        // (W8: the producer's own loads are the fp8 k-blocks of the q ring.)
        constexpr int kRingDepth = W8 ? LY::kQSlots : STAGES;
        const long long first = issued > kRingDepth ? issued - kRingDepth : 0;
        const uint64_t t0 = gtimer();
        bool late = false;
#pragma unroll 1
        for (long long i = first; i < issued && !late; ++i) {
          const int s = static_cast<int>(i % kRingDepth);
          const uint32_t par = static_cast<uint32_t>((i / kRingDepth) & 1);
          while (!mbar_try_wait(W8 ? qfull_bar(s) : full_bar(s), par)) {
            if (gtimer() - t0 > p.wait_limit_ns) { late = true; break; }
          }

        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer (leader)
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      long long kn = 0;  // W8: k-blocks consumed (token-operand ring position)
      bool ok = true;
#pragma unroll 1
      for (int seq = 0; ok; ++seq) {
        const int slot = seq % LY::kRing;
        if (!wait_bar<PAIR>(ring_full(slot), static_cast<uint32_t>((seq / LY::kRing) & 1), abort_flag, p,
                            600 + slot))
          break;
        int w[8];
        ld_shared_8(ring_slot(slot), w);
        mbar_arrive(ring_empty(slot));
        if (!w[7]) break;
        Unit u;
        unpack_unit(w, u);
        if (!wait_bar(tempty_bar(acc), acc_phase ^ 1u, abort_flag, p, 200 + acc)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * LY::kAccCols);
#pragma unroll 1
        for (int kb = u.kb0; kb < u.kb1; ++kb) {
          if (!wait_bar(full_bar(stage), phase, abort_flag, p, 300 + stage)) { ok = false; break; }
          uint32_t sbk = sB + stage * LY::kBStage;  // this k-block's B tile
          int bslot = 0;
          if constexpr (W8) {  // the token tile waits in its own ring slot
            bslot = static_cast<int>(kn % LY::kBSlots);
            const uint32_t bpar = static_cast<uint32_t>((kn / LY::kBSlots) & 1);
            if (!wait_bar(bfull_bar(bslot), bpar, abort_flag, p, 320 + bslot)) { ok = false; break; }
            sbk = sBR + bslot * LY::kBStage;
            ++kn;
          }
          tc_fence_after();
#pragma unroll
          for (int j = 0; j < KSUB; ++j) {
            const uint64_t da = sw128_desc(sA + stage * LY::kAStage + j * kABytes);
            const uint64_t db = sw128_desc(sbk + j * LY::kBSub);
            const uint32_t ta =
                tmem_base + static_cast<uint32_t>(2 * LY::kAccCols + LY::kTmemA * stage + 32 * j);  // W8: A in TMEM
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k) {
              // +32 bytes along K inside the 128-byte swizzle atom = +2 in the 16-byte address field
              const int ks = (j * (kBK / 16) + k);  // K step within the k-block
              const uint32_t dc = d + static_cast<uint32_t>((ks % LY::kChains) * BN);
              const uint32_t accum = (kb > u.kb0 || ks >= LY::kChains) ? 1u : 0u;
              if constexpr (PAIR) umma_f16_pair(dc, da + 2 * k, db + 2 * k, kIdesc, accum);
              else if constexpr (W8) umma_f16_ta(dc, ta + 8 * k, db + 2 * k, kIdesc, accum);
              else umma_f16(dc, da + 2 * k, db + 2 * k, kIdesc, accum);
            }
          }
          if constexpr (PAIR) {
            umma_commit_pair_both(empty_bar(stage));
          } else {
            umma_commit(empty_bar(stage));
            if constexpr (W8) umma_commit(bempty_bar(bslot));
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        if constexpr (PAIR) {
          umma_commit_pair_both(tfull_bar(acc));
        } else {
          umma_commit(tfull_bar(acc));
        }
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
      trace_mark(p, kTrLastMma);
      // Drain: all issued MMAs complete before TMEM is released.
      if constexpr (PAIR) umma_commit_pair(drain_bar);
      else umma_commit(drain_bar);
      const uint64_t t0 = gtimer();
      while (!mbar_try_wait(drain_bar, 0)) {
        if (gtimer() - t0 > p.wait_limit_ns) break;
      }
    }
  } else if (warp >= kCtrlThreads / 32 + EPI) {
    // ---------------------------------------------------------------- fp8 weight converters (W8)
    // Group g takes k-blocks g, g + G, g + 2G, ... of the CTA's sequence (k-block n: q slot
    // n mod Q, MMA stage n mod STAGES).  For each, its 4 warps wait for the fp8 k-block; each
    // warp widens the 64 fp8 codes of the 32 weight rows of its TMEM sub-partition to the
    // problem's 16-bit type, frees the q slot, waits for the stage's TMEM columns to be free
    // and stores the rows there (the MMA's A operand in tensor memory), then arrives.
    if constexpr (W8) {
      const int cw = warp - (kCtrlThreads / 32 + EPI);
      const int group = cw >> 2;
      const int r = (warp & 3) * 32 + lane;  // row of the A tile = TMEM lane of this warp
      const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
      long long n = 0;  // k-blocks of this CTA seen so far
      int ok = 1;
#pragma unroll 1
      for (int seq = 0; ok; ++seq) {
        const int slot = seq % LY::kRing;
        const uint32_t rpar = static_cast<uint32_t>((seq / LY::kRing) & 1);
        if (lane == 0) ok = wait_bar(ring_full(slot), rpar, abort_flag, p, 600 + slot) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        if (lane != 0) (void)mbar_try_wait(ring_full(slot), rpar);
        int w[8];
        ld_shared_8(ring_slot(slot), w);
        __syncwarp();
        if (lane == 0) mbar_arrive(ring_empty(slot));
        if (!w[7]) break;
        const int nkb = w[3] - w[2];
#pragma unroll 1
        for (int i = 0; i < nkb; ++i, ++n) {
          if (n % LY::kCvtGroups != group) continue;  // another group's k-block
          const int j = static_cast<int>(n % LY::kQSlots);
          const uint32_t qpar = static_cast<uint32_t>((n / LY::kQSlots) & 1);
          const int st = static_cast<int>(n % STAGES);
          const uint32_t spar = static_cast<uint32_t>((n / STAGES) & 1);
          if (lane == 0) ok = wait_bar(qfull_bar(j), qpar, abort_flag, p, 700 + j) ? 1 : 0;
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) break;
          if (lane != 0) (void)mbar_try_wait(qfull_bar(j), qpar);
          // Row r of the q slot: 64*KSUB codes.  The box carries the TMA's swizzle: with
          // 64-byte rows (KSUB 1) 16-byte chunk c sits at c ^ ((r >> 1) & 3), with 128-byte rows
          // (KSUB 2) at c ^ (r & 7); either way 8 consecutive rows cover all banks.
          const uint32_t src = sQ + static_cast<uint32_t>(j * LY::kQStage + r * 64 * KSUB);
          uint32_t q[16 * KSUB];
#pragma unroll
          for (int c = 0; c < 4 * KSUB; ++c) {
            const int pc = KSUB == 2 ? (c ^ (r & 7)) : (c ^ ((r >> 1) & 3));
            asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(q[4 * c]), "=r"(q[4 * c + 1]), "=r"(q[4 * c + 2]), "=r"(q[4 * c + 3])
                         : "r"(src + (pc << 4))
                         : "memory");
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(qempty_bar(j));  // the codes are in registers
          if constexpr (BF16) {
            // The token tile of this k-block (B ring slot n mod QB, landed by TMA): bf16 ->
            // fp16 in place, 128B-swizzled positions unchanged.  The 4 warps of the group split
            // it; each thread converts 8-element (16-byte) pieces.
            const int jb = static_cast<int>(n % LY::kBSlots);
            const uint32_t bpar = static_cast<uint32_t>((n / LY::kBSlots) & 1);
            if (lane == 0) ok = wait_bar(bfull_bar(jb), bpar, abort_flag, p, 720 + jb) ? 1 : 0;
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
            if (lane != 0) (void)mbar_try_wait(bfull_bar(jb), bpar);
            constexpr int kPieces = LY::kBStage / 16;  // 16-byte pieces of the tile
            const uint32_t bbase = sBR + static_cast<uint32_t>(jb * LY::kBStage);
            bool range_ok = true;
#pragma unroll 1
            for (int piece = (warp & 3) * 32 + lane; piece < kPieces; piece += 128) {
              uint32_t v[4];
              asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                           : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                           : "r"(bbase + piece * 16)
                           : "memory");
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float lo = __uint_as_float(v[e] << 16), hi = __uint_as_float(v[e] & 0xFFFF0000u);
                range_ok = range_ok && fabsf(lo) <= 65504.0f && fabsf(hi) <= 65504.0f;
                const __half2 h = __floats2half2_rn(lo, hi);
                v[e] = *reinterpret_cast<const uint32_t*>(&h);
              }
              asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(bbase + piece * 16), "r"(v[0]), "r"(v[1]),
                           "r"(v[2]), "r"(v[3])
                           : "memory");
            }
            if (!range_ok) report(p, 6, static_cast<int>(n));  // recorded, the results are not valid
            fence_async_shared();
          }
          if (lane == 0) ok = wait_bar(empty_bar(st), spar ^ 1u, abort_flag, p, 100 + st) ? 1 : 0;
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (!ok) break;
          tc_fence_after();  // the MMAs that read these columns have completed
#pragma unroll
          for (int jj = 0; jj < KSUB; ++jj) {
            uint32_t o[32];
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              o[2 * k] = e4m3x2_to_16x2<false>(q[16 * jj + k]);
              o[2 * k + 1] = e4m3x2_to_16x2<false>(q[16 * jj + k] >> 16);
            }
            tmem_st32(tmem_base + lane_off + static_cast<uint32_t>(2 * LY::kAccCols + LY::kTmemA * st + 32 * jj), o);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(full_bar(st));
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5)
    const int ew = warp - 2;            // staging-buffer owner index
    const int sub = warp & 3;           // TMEM lane sub-partition this warp may access
    const int part = ew >> 2;           // which share of the columns this warp handles
    const int row = sub * 32 + lane;    // row inside this CTA's 128 rows of the tile
    constexpr int kMyChunks = kChunks / kParts;
    const int ch0 = part * kMyChunks;
    int acc = 0;
    uint32_t acc_phase = 0;
    int sbuf = 0;
    bool seen_down = false;
    if (ew == 0 && lane == 0) {  // this CTA's share of the launch count -> the launch epoch
      const unsigned long long old = atomicAdd(p.launches, 1ull);
      *epoch_val = old / gridDim.x + 1ull;
      mbar_arrive(epoch_bar);
    }
    unsigned long long epoch = 0;  // fetched before the first flag wait or staging slot
    bool have_epoch = false;
    // Fused reduce-scatter: the owner's count of the last pushed tile, released one tile
    // late (lane 0) -- once the next tile's stores are issued and this one's have completed
    // -- so the warp does not sit out an NVLink round trip per tile.  Flushed before any
    // unit that waits on other ranks and at the end.
    unsigned* rs_pending = nullptr;
    auto rs_flush = [&]() {
      if (lane == 0 && rs_pending) {
        bulk_wait_all();
        fence_async_global();
        red_release_sys_add(rs_pending, 1u);
        rs_pending = nullptr;
      }
    };
#pragma unroll 1
    for (int seq = 0;; ++seq) {
      // Next unit from the ring: lane 0 waits, the warp reads the slot, lane 0 frees it.
      const int slot = seq % LY::kRing;
      int ok = 1;
      if (lane == 0)
        ok = wait_bar<PAIR>(ring_full(slot), static_cast<uint32_t>((seq / LY::kRing) & 1), abort_flag, p, 600 + slot)
                 ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      if (lane != 0) {  // the phase is complete (the slot is not freed yet): acquire for this lane too
        const uint32_t par = static_cast<uint32_t>((seq / LY::kRing) & 1);
        (void)(PAIR ? mbar_try_wait_cluster(ring_full(slot), par) : mbar_try_wait(ring_full(slot), par));
      }
      int w[8];
      ld_shared_8(ring_slot(slot), w);
      __syncwarp();
      if (lane == 0) {
        if constexpr (PAIR) mbar_arrive_cluster(map_to_rank(ring_empty(slot), 0));
        else mbar_arrive(ring_empty(slot));
      }
      if (!w[7]) break;
      Unit u;
      unpack_unit(w, u);
      int tr, tq;
      unit_coords(p, u, tr, tq);
      if (lane == 0) ok = wait_bar(tfull_bar(acc), acc_phase, abort_flag, p, 400 + acc) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      if (ew == 0 && lane == 0 && u.phase == 1 && !seen_down) trace_mark(p, kTrFirstDown);
      if (u.phase == 1) seen_down = true;
      if (!have_epoch && (u.role == kRoleOwner || p.rs_world > 1)) {
        if (lane == 0) ok = fetch_epoch(epoch) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        epoch = __shfl_sync(0xffffffffu, epoch, 0);
        have_epoch = true;
      }
      // Stream-K owner: wait for every contributor's partial of this tile (same pair rank).
      // Lane i acquires contributor c_first + i's flag, so the ~5 flags of a decode tile are
      // polled at once rather than one L2 round trip after another; the warp barrier then
      // orders every lane's reads of the partials after all of those acquires.
      if (u.role == kRoleOwner && u.c_first <= u.c_last) {
        for (int c0 = u.c_first; c0 <= u.c_last && ok; c0 += 32) {
          const int c2 = c0 + lane;
          int mine = 1;
          if (c2 <= u.c_last)
            mine = wait_word_ge(p.flags + (u.phase * p.C + c2) * kNcta + slot_base,
                                EPI * static_cast<unsigned>(epoch), abort_flag, p, 3, c2) ? 1 : 0;
          ok = __all_sync(0xffffffffu, mine);
        }
        __syncwarp();
        if (!ok) break;
      }
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(sub * 32) << 16) + static_cast<uint32_t>(acc * LY::kAccCols);
      // Stream-K partial slot of CTA c (kBM x BN fp32), stored as [BN/4 column groups][kBM rows]
      // float4: the 32 lanes of a warp (consecutive rows) write and read 512 contiguous bytes
      // per access.  This thread's float4 of column group g:
      auto ws_f4 = [&](int c, int g) {
        return reinterpret_cast<float4*>(p.ws) +
               (static_cast<size_t>((u.phase * p.C + c) * kNcta + slot_base) * (BN / 4) + g) * kBM + row;
      };

      // Fused reduce-scatter (down phase, tile finalised here): push to the owning rank, or
      // (own band) wait for every other rank's partial of this tile.
      bool rs_push = false, rs_reduce = false;
      int rs_owner = 0;
      size_t rs_tile = 0;
      if constexpr (!SWAP && !PAIR) {
        if (p.rs_world > 1 && u.phase == 1 && u.role != kRoleContrib) {
          rs_owner = tr / p.rs_band_tiles;
          rs_tile = static_cast<size_t>(tr - rs_owner * p.rs_band_tiles) * p.dn.tiles_q + tq;
          rs_push = rs_owner != p.rs_rank;
          rs_reduce = !rs_push;
          if (rs_reduce) {
            rs_flush();  // (other ranks' own bands may wait on it)
            // Lane `src` acquires rank src's flag (all ranks at once); the warp barrier orders
            // every lane's reads of the staged partials after those acquires.
            const size_t band = static_cast<size_t>(p.rs_band_tiles) * p.dn.tiles_q;
            int mine = 1;
            if (lane < p.rs_world && lane != p.rs_rank)
              mine = wait_word_ge<true>(p.rs_flags[p.rs_rank] + lane * band + rs_tile,
                                        EPI * static_cast<unsigned>(epoch), abort_flag, p, 4, lane) ? 1 : 0;
            ok = __all_sync(0xffffffffu, mine);
            __syncwarp();
            if (!ok) break;
          }
        }
      }
      auto rs_row = [&](int src) {  // element offset of this thread's row in a staging slot
        const size_t band = static_cast<size_t>(p.rs_band_tiles) * p.dn.tiles_q;
        const size_t slot = ((static_cast<size_t>(epoch & 1u) * p.rs_world + src) * band + rs_tile) * kBM + row;
        return slot * BN;
      };

      if constexpr (!SWAP) {
        // Normal mode: tile rows are tokens, columns are features (H for up, N for down).
        const CUtensorMap* tms = u.phase ? &p.tm_st_y : &p.tm_st_hid;
        const int orow = (rs_reduce ? (tr - p.rs_rank * p.rs_band_tiles) : tr) * kTileM +
                         static_cast<int>(rank) * kBM + sub * 32;
#pragma unroll 1
        for (int ch = ch0; ch < ch0 + kMyChunks; ++ch) {
          if constexpr (GELU == 3) {  // SwiGLU up values: consumed with their gate chunk
            if (u.phase == 0 && (ch & 1) && u.role != kRoleContrib) continue;
          }
          float v[64];
          tmem_ld32(tbase + ch * 64, v);
          tmem_ld32(tbase + ch * 64 + 32, v + 32);
          if (u.role == kRoleContrib) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              *ws_f4(cta, ch * 16 + j) = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            continue;
          }
          if (u.role == kRoleOwner) {
#pragma unroll 1
            for (int c2 = u.c_first; c2 <= u.c_last; ++c2) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const float4 t = __ldcg(ws_f4(c2, ch * 16 + j));
                v[4 * j] += t.x; v[4 * j + 1] += t.y; v[4 * j + 2] += t.z; v[4 * j + 3] += t.w;
              }
            }
          }
          int hcol = tq * BN + ch * 64;  // hidden column of this chunk (up phase)
          if constexpr (GELU == 3) {
            // SwiGLU: W1 rows come in blocks of 64 gate rows then the matching 64 up rows, so
            // chunk ch (even) holds gates and chunk ch + 1 the up values of 64 hidden columns.
            if (u.phase == 0) {
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {  // up values 32 at a time (register pressure)
                float w[32];
                tmem_ld32(tbase + (ch + 1) * 64 + hh * 32, w);
                if (u.role == kRoleOwner) {
#pragma unroll 1
                  for (int c2 = u.c_first; c2 <= u.c_last; ++c2) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                      const float4 t = __ldcg(ws_f4(c2, (ch + 1) * 16 + hh * 8 + j));
                      w[4 * j] += t.x; w[4 * j + 1] += t.y; w[4 * j + 2] += t.z; w[4 * j + 3] += t.w;
                    }
                  }
                }
#pragma unroll
                for (int j = 0; j < 32; ++j) v[hh * 32 + j] = silu(v[hh * 32 + j]) * w[j];
              }
              hcol = tq * (BN / 2) + (ch / 2) * 64;
            }
          } else if (u.phase == 0) {
            if (p.bias1) add_bias<BF16, 64>(v, p.bias1, tq * BN + ch * 64, p.H);
#pragma unroll
            for (int j = 0; j < 64; j += 2) gelu2<GELU>(v[j], v[j + 1]);
          }
          if (u.phase == 1 && p.bias2 && !rs_push && !rs_reduce) add_bias<BF16, 64>(v, p.bias2, tq * BN + ch * 64, p.N);
          if (rs_reduce) {
            // Ascending rank order: sum = p_0 + p_1 + ... (this rank's fp32 partial in place),
            // 16 columns at a time to keep the register peak of the chunk loop.
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float acc[16];
#pragma unroll 1
              for (int src = 0; src < p.rs_world; ++src) {
                if (src == p.rs_rank) {
#pragma unroll
                  for (int j = 0; j < 16; ++j) acc[j] = src == 0 ? v[16 * q + j] : acc[j] + v[16 * q + j];
                } else if (p.rs_format == 1) {
                  const float4* sp = reinterpret_cast<const float4*>(static_cast<const float*>(p.rs_stage[p.rs_rank]) +
                                                                     rs_row(src) + ch * 64 + 16 * q);
                  float4 w[4];
#pragma unroll
                  for (int j = 0; j < 4; ++j) w[j] = __ldcg(sp + j);
#pragma unroll
                  for (int j = 0; j < 4; ++j) {
                    acc[4 * j] = src == 0 ? w[j].x : acc[4 * j] + w[j].x;
                    acc[4 * j + 1] = src == 0 ? w[j].y : acc[4 * j + 1] + w[j].y;
                    acc[4 * j + 2] = src == 0 ? w[j].z : acc[4 * j + 2] + w[j].z;
                    acc[4 * j + 3] = src == 0 ? w[j].w : acc[4 * j + 3] + w[j].w;
                  }
                } else if (p.rs_format == 2) {
                  // 24-bit partial: the high 16 bits of the rounded fp32 word from the u16
                  // plane, the next 8 from the byte plane (low 8 bits zero).
                  const size_t e0 = rs_row(src) + ch * 64 + 16 * q;
                  const uint4* hp = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.rs_stage[p.rs_rank]) + e0);
                  const uint4 lw = __ldcg(reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(p.rs_stage[p.rs_rank]) +
                                                                         p.rs_lo_off + e0));
                  const uint32_t lv[4] = {lw.x, lw.y, lw.z, lw.w};
#pragma unroll
                  for (int j = 0; j < 2; ++j) {
                    const uint4 w = __ldcg(hp + j);
                    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                      const int c = 8 * j + 2 * e;  // column of the low element of this pair
                      const uint32_t b0 = (lv[c >> 2] >> (8 * (c & 3))) & 0xFFu;
                      const uint32_t b1 = (lv[(c + 1) >> 2] >> (8 * ((c + 1) & 3))) & 0xFFu;
                      const float lo = __uint_as_float((wv[e] << 16) | (b0 << 8));
                      const float hi = __uint_as_float((wv[e] & 0xFFFF0000u) | (b1 << 8));
                      acc[c] = src == 0 ? lo : acc[c] + lo;
                      acc[c + 1] = src == 0 ? hi : acc[c + 1] + hi;
                    }
                  }
                } else {
                  const uint4* sp = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.rs_stage[p.rs_rank]) +
                                                                   rs_row(src) + ch * 64 + 16 * q);
#pragma unroll
                  for (int j = 0; j < 2; ++j) {
                    const uint4 w = __ldcg(sp + j);
                    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                      const float lo = unpack_lo<BF16>(wv[e]), hi = unpack_hi<BF16>(wv[e]);
                      acc[8 * j + 2 * e] = src == 0 ? lo : acc[8 * j + 2 * e] + lo;
                      acc[8 * j + 2 * e + 1] = src == 0 ? hi : acc[8 * j + 2 * e + 1] + hi;
                    }
                  }
                }
              }
#pragma unroll
              for (int j = 0; j < 16; ++j) v[16 * q + j] = acc[j];
            }
            // (the band owner adds the bias once, to the sum of all ranks' partials)
            if (p.bias2) add_bias<BF16, 64>(v, p.bias2, tq * BN + ch * 64, p.N);
          }
          if (rs_push && p.rs_format == 2) {
            // 24-bit partial for the owning GPU: each fp32 word rounded to nearest (ties to
            // even) at bit 8, its high 16 bits sent as a u16 tile and the next 8 as a byte
            // tile (two bulk stores per chunk and warp; 3/4 of the fp32 bytes over NVLink).
            const size_t band = static_cast<size_t>(p.rs_band_tiles) * p.dn.tiles_q;
            const int srow = static_cast<int>(((static_cast<size_t>(epoch & 1u) * p.rs_world + p.rs_rank) * band +
                                               rs_tile) * kBM) + sub * 32;
            uint32_t hi2[32], lo4[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) lo4[j] = 0u;
#pragma unroll
            for (int j = 0; j < 64; ++j) {
              const uint32_t b = __float_as_uint(v[j]);
              const uint32_t r24 = b + 0x7Fu + ((b >> 8) & 1u);
              const uint32_t h16 = r24 >> 16;
              if (j & 1) hi2[j >> 1] |= h16 << 16;
              else hi2[j >> 1] = h16;
              lo4[j >> 2] |= ((r24 >> 8) & 0xFFu) << (8 * (j & 3));
            }
#pragma unroll
            for (int pl = 0; pl < 2; ++pl) {
              const uint32_t sb = sE + static_cast<uint32_t>((ew * 2 + sbuf) * kStageBufBytes);
              if (lane == 0) bulk_wait_read1();
              __syncwarp();
              if (pl == 0) {  // 32 rows x 128 B, 128B-swizzled
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  const uint32_t addr = sb + lane * 128 + ((j ^ (lane & 7)) << 4);
                  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(hi2[4 * j]),
                               "r"(hi2[4 * j + 1]), "r"(hi2[4 * j + 2]), "r"(hi2[4 * j + 3])
                               : "memory");
                }
              } else {  // 32 rows x 64 B, 64B-swizzled: 16-byte chunk c of row r at c ^ ((r >> 1) & 3)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const uint32_t addr = sb + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4);
                  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(lo4[4 * j]),
                               "r"(lo4[4 * j + 1]), "r"(lo4[4 * j + 2]), "r"(lo4[4 * j + 3])
                               : "memory");
                }
              }
              fence_async_shared();
              __syncwarp();
              if (lane == 0) {
                if (pl == 0) tma_store_2d(&p.tm_rs[rs_owner], sb, ch * 64, srow);
                else tma_store_2d(&p.tm_rs_lo[rs_owner], sb, ch * 32, srow);  // (byte pairs: x in units of 2 bytes)
                bulk_commit();
              }
              sbuf ^= 1;
            }
            continue;
          }
          if (rs_push && p.rs_format == 1) {
            // fp32 partial for the owning GPU: two 32-column halves (128-byte rows), each
            // staged 128B-swizzled in one of this warp's buffers and sent as one 4 KB bulk
            // store over NVLink, so the owner's sum sees the unrounded partial.
            const size_t band = static_cast<size_t>(p.rs_band_tiles) * p.dn.tiles_q;
            const int srow = static_cast<int>(((static_cast<size_t>(epoch & 1u) * p.rs_world + p.rs_rank) * band +
                                               rs_tile) * kBM) + sub * 32;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const uint32_t sb = sE + static_cast<uint32_t>((ew * 2 + sbuf) * kStageBufBytes);
              if (lane == 0) bulk_wait_read1();
              __syncwarp();
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const uint32_t addr = sb + lane * 128 + ((j ^ (lane & 7)) << 4);
                asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v[32 * hh + 4 * j]),
                             "f"(v[32 * hh + 4 * j + 1]), "f"(v[32 * hh + 4 * j + 2]), "f"(v[32 * hh + 4 * j + 3])
                             : "memory");
              }
              fence_async_shared();
              __syncwarp();
              if (lane == 0) {
                tma_store_2d(&p.tm_rs[rs_owner], sb, ch * 64 + 32 * hh, srow);
                bulk_commit();
              }
              sbuf ^= 1;
            }
            continue;
          }
          uint32_t pk[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) pk[j] = pack2<BF16>(v[2 * j], v[2 * j + 1]);
          // Staging buffer (32 rows x 128 B, 128B-swizzled) owned by this warp.
          const uint32_t sb = sE + static_cast<uint32_t>((ew * 2 + sbuf) * kStageBufBytes);
          if (lane == 0) bulk_wait_read1();
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t addr = sb + lane * 128 + ((j ^ (lane & 7)) << 4);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(pk[4 * j]),
                         "r"(pk[4 * j + 1]), "r"(pk[4 * j + 2]), "r"(pk[4 * j + 3])
                         : "memory");
          }
          fence_async_shared();
          __syncwarp();
          if (lane == 0) {
            if (rs_push) {
              // The owner's staging slot (this rank's partial of the tile): one 4 KB bulk
              // store over NVLink per chunk and warp.
              const size_t band = static_cast<size_t>(p.rs_band_tiles) * p.dn.tiles_q;
              const int srow = static_cast<int>(((static_cast<size_t>(epoch & 1u) * p.rs_world + p.rs_rank) * band +
                                                 rs_tile) * kBM) + sub * 32;
              tma_store_2d(&p.tm_rs[rs_owner], sb, ch * 64, srow);
            } else {
              tma_store_2d(tms, sb, u.phase ? tq * BN + ch * 64 : hcol, orow);
            }
            bulk_commit();
          }
          sbuf ^= 1;
        }
      } else {
        // Swap mode: tile rows are features (H for up, N for down), columns are tokens.
        const int feat = tr * kBM + row;
        const int F = u.phase ? p.N : (GELU == 3 ? 2 * p.H : p.H);  // feature rows (SwiGLU: gate/up pairs)
        uint16_t* out = reinterpret_cast<uint16_t*>(u.phase ? p.y : p.hidden);
        const long long ld = u.phase ? p.ldy : p.ldh;
#pragma unroll 1
        for (int ch = ch0; ch < ch0 + kMyChunks; ++ch) {
          float v[kCW];
          if constexpr (kCW == 16) tmem_ld16(tbase + ch * kCW, v);
          else tmem_ld8(tbase + ch * kCW, v);
#pragma unroll
          for (int c = 1; c < LY::kChains; ++c) {  // the other K chains, in order
            float w[kCW];
            if constexpr (kCW == 16) tmem_ld16(tbase + c * BN + ch * kCW, w);
            else tmem_ld8(tbase + c * BN + ch * kCW, w);
#pragma unroll
            for (int j = 0; j < kCW; ++j) v[j] += w[j];
          }
          if (u.role == kRoleContrib) {
#pragma unroll
            for (int j = 0; j < kCW / 4; ++j)
              *ws_f4(cta, ch * (kCW / 4) + j) = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            continue;
          }
          if (u.role == kRoleOwner) {
            // The contributors' partials, several float4 loads in flight (a decode tile has
            // ~5 contributors: one L2 round trip per batch instead of one per contributor),
            // added in contributor order as before, so the sum is the same bit for bit.  The
            // fp8 tiles run 22 warps and have fewer registers per thread for the batch.
            constexpr int kF4 = kCW / 4;
            constexpr int kBatch = W8 ? (kF4 <= 2 ? 4 : 1) : 16 / kF4;
#pragma unroll 1
            for (int c0 = u.c_first; c0 <= u.c_last; c0 += kBatch) {
              float4 t[kBatch][kF4];
#pragma unroll
              for (int b = 0; b < kBatch; ++b) {
                if (c0 + b <= u.c_last) {
#pragma unroll
                  for (int j = 0; j < kF4; ++j) t[b][j] = __ldcg(ws_f4(c0 + b, ch * kF4 + j));
                }
              }
#pragma unroll
              for (int b = 0; b < kBatch; ++b) {
                if (c0 + b <= u.c_last) {
#pragma unroll
                  for (int j = 0; j < kF4; ++j) {
                    v[4 * j] += t[b][j].x; v[4 * j + 1] += t[b][j].y; v[4 * j + 2] += t[b][j].z; v[4 * j + 3] += t[b][j].w;
                  }
                }
              }
            }
          }
          if constexpr (W8) {  // fp8 weights: the row's scale factors out of the K sum
            if (feat < F) {
              const float sc = __ldg((u.phase ? p.w2_scale : p.w1_scale) + feat);
#pragma unroll
              for (int j = 0; j < kCW; ++j) v[j] *= sc;
            }
          }
          {
            const uint16_t* bias = u.phase ? p.bias2 : p.bias1;
            if (bias && feat < F) {  // rows are features here: one bias value per row
              const float b = unpack_lo<BF16>(static_cast<uint32_t>(__ldg(bias + feat)));
#pragma unroll
              for (int j = 0; j < kCW; ++j) v[j] += b;
            }
          }
          if constexpr (GELU == 3) {
            // SwiGLU in the decode tiles: W1 rows alternate gate, up (rows 2i, 2i + 1 give
            // hidden feature i), so the up value sits in the neighbouring lane.
            if (u.phase == 0) {
#pragma unroll
              for (int j = 0; j < kCW; ++j) {
                const float up = __shfl_xor_sync(0xffffffffu, v[j], 1);
                v[j] = silu(v[j]) * up;
              }
              const int hfeat = feat >> 1;
              if ((row & 1) == 0 && hfeat < p.H) {
#pragma unroll
                for (int j = 0; j < kCW; ++j) {
                  const int m = tq * BN + ch * kCW + j;
                  if (m < p.M) out[static_cast<long long>(m) * ld + hfeat] = cvt1<BF16>(v[j]);
                }
              }
              continue;
            }
          }
          if (feat < F) {
#pragma unroll
            for (int j = 0; j < kCW; ++j) {
              const int m = tq * BN + ch * kCW + j;
              if (m < p.M) {
                const float val = u.phase == 0 ? gelu<GELU>(v[j]) : v[j];
                out[static_cast<long long>(m) * ld + feat] = cvt1<BF16>(val);
              }
            }
          }
        }
      }
      // Release the TMEM accumulator to the (leader's) MMA warp.
      tc_fence_before();
      if constexpr (PAIR) mbar_arrive_cluster(map_to_rank(tempty_bar(acc), 0));
      else mbar_arrive(tempty_bar(acc));
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }

      if (rs_push) {
        // Publish this warp's 32 rows to the owning GPU, one tile late: the previous pushed
        // tile's bulk stores complete (all but this tile's groups), the async proxy is
        // ordered before the generic one, then one system-scope release per warp on that
        // owner's count for (this rank, tile).
        const size_t band = static_cast<size_t>(p.rs_band_tiles) * p.dn.tiles_q;
        if (lane == 0) {
          if (rs_pending) {
            bulk_wait_keep((p.rs_format == 0 ? 1 : 2) * kMyChunks);  // bulk groups of this tile
            fence_async_global();
            red_release_sys_add(rs_pending, 1u);
          }
          rs_pending = p.rs_flags[rs_owner] + p.rs_rank * band + rs_tile;
        }
        __syncwarp();
      }
      if (u.role == kRoleContrib) {
        // Publish this warp's 32 rows of the partial: one release per warp, so the owner
        // waits for 4 signals per launch and no CTA-wide barrier is involved.
        __threadfence();
        __syncwarp();
        if (lane == 0) red_release_add(p.flags + (u.phase * p.C + cta) * kNcta + slot_base, 1u);
      } else if (u.phase == 0) {
        // Hidden tile stored: signal the row block (one signal per warp).
        const int blk = SWAP ? tq : tr;
        if constexpr (!SWAP) {
          if (lane == 0) {
            bulk_wait_all();
            fence_async_global();
            red_release_add(p.counters + blk, 1u);
          }
          __syncwarp();
        } else {
          __threadfence();
          __syncwarp();
          if (lane == 0) red_release_add(p.counters + blk, 1u);
        }
        if (ew == 0 && lane == 0) trace_mark(p, kTrUpStored);
      }
    }
    rs_flush();
    if constexpr (!SWAP) {
      if (lane == 0) bulk_wait_all();
      __syncwarp();
    }
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // no CTA leaves while its peer may still signal it
  tc_fence_after();
  if (threadIdx.x == 0) trace_mark(p, kTrEnd);
  if (warp == 1) {
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, LY::kTmemCols);
    else tmem_dealloc(tmem_base, LY::kTmemCols);
  }
}

}  // namespace ffnb200
