// Decode FFN (M <= 16 tokens) with the hidden dimension split over the CTAs of a cluster:
// no hidden tensor in global memory and no grid-wide wait between the two GEMMs.
//
// The decode shapes stream both weight matrices once from HBM; the two-phase kernel must
// finish every up tile before any down tile can start (each output needs the whole hidden
// row), and both phases end in Stream-K fixups.  Here each CTA owns 128 hidden rows and a
// cluster of S CTAs owns S*128 of them (a "hidden super-block"):
//
//   up:      hidT[128 x 16]  = W1[h0 : h0+128, :] . X^T            (TMEM, 4 K chains)
//   slice:   GELU, round to the input dtype, write the 16 x 128 slice K-major into this
//            CTA's slot of the cluster hidden buffer and copy it into every peer's slot
//            (shared-memory to shared-memory bulk copies, completion on the peer's mbarrier)
//   down:    YT[n-block] += W2[n-block, cluster's S*128 hidden columns] . hid^T
//            for the N/S rows of Y this CTA's cluster rank owns   (TMEM, kept over super-blocks)
//   partial: the fp32 [N/S x 16] partial of each cluster goes to global memory, and
//   reduce:  Y rows of rank r are summed over the clusters (ascending cluster order) by the
//            rank-r CTAs of all clusters, each taking an equal share of those rows (coalesced
//            L2 loads, 32 clusters' partials in flight per thread).
//
// Every CTA streams 128 rows of W1 and 128 hidden columns' worth of W2 (S*128 columns for
// N/S rows): equal bytes, one pass over HBM, and the only cross-cluster wait is the final
// reduction of (cluster count) partials per output, read from L2.  The weight tiles are the
// MMA's 128-row A operand and the 16 token rows its N dimension, as in the swap-AB tiles.
//
// Arithmetic: fp32 accumulation over K (4 chains summed in a fixed order), activation of
// the fp32 sum, hidden rounded once to the input dtype, fp32 accumulation over H (per
// cluster in k-block order, then over clusters in ascending order), one rounding of Y.  The
// order of every sum is fixed by the plan, so results are identical run to run.
//
// Every wait is bounded (globaltimer); on expiry the CTA records an error in status[],
// raises its abort flag and falls through to the teardown, where the cluster barrier keeps
// each CTA resident until its peers no longer touch its shared memory.
#pragma once

#include <type_traits>

#include "ffn_kernel.cuh"

namespace ffnb200 {

template <int S>
struct SliceLayout {
  static constexpr int kT = 16;                           // token columns (MMA N)
  static constexpr int kWBytes = kBM * kBK * 2;           // one weight k-block: 128 rows x 64
  static constexpr int kXBytes = kT * kBK * 2;            // one token k-block: 16 rows x 64
  static constexpr int kStage = kWBytes + kXBytes;        // 18 KB, a multiple of 1024
  static constexpr int kKbBytes = kT * 128;               // one hidden k-block: 16 rows x 128 B
  static constexpr int kSlice = 2 * kKbBytes;             // one CTA's 128 hidden columns
  static constexpr int kHidBuf = S * kSlice;              // the cluster's S*128 hidden columns
  static constexpr int kBarBytes = 512;
  static constexpr int kStages = (232448 - 1024 - 2 * kHidBuf - kBarBytes) / kStage;
  static constexpr int kSmem = 1024 + kStages * kStage + 2 * kHidBuf + kBarBytes;
  static constexpr int kEpiWarps = 4;
  static constexpr int kThreads = kCtrlThreads + 32 * kEpiWarps;
  static constexpr int kUpChains = 4;                     // K chains of the up accumulator
  static constexpr int kUpCols = kUpChains * kT;          // TMEM columns 0 .. 63
  static constexpr int kTmemCols = 512;                   // down accumulators from column 64
  static_assert(S == 2 || S == 4 || S == 8, "cluster size");
  static_assert(kStages >= 4, "operand ring depth");
  static_assert((2 * kStages + 11) * 8 <= kBarBytes, "barrier area");
  static_assert(kSmem <= 232448, "dynamic shared memory per CTA");
};

// Down-phase K chains for `nbr` n-blocks per CTA: as many as fit next to the up accumulator.
__host__ __device__ constexpr int slice_down_chains(int nbr) {
  return nbr * 4 * 16 <= 448 ? 4 : (nbr * 2 * 16 <= 448 ? 2 : 1);
}

// Shared-memory to shared-memory bulk copy into a peer CTA of the cluster; the bytes complete
// on the peer's mbarrier (cluster addresses from mapa).
__device__ __forceinline__ void bulk_copy_to_peer(uint32_t dst_cluster, uint32_t src, uint32_t bytes,
                                                  uint32_t bar_cluster) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(dst_cluster), "r"(src), "r"(bytes), "r"(bar_cluster)
               : "memory");
}

template <int S, bool BF16, int GELU>
__global__ void __launch_bounds__(kCtrlThreads + 32 * 4, 1) ffn_hslice_kernel(const __grid_constant__ Params p) {
  using LY = SliceLayout<S>;
  constexpr int kT = LY::kT;
  constexpr int ST = LY::kStages;
  constexpr uint32_t kIdesc = make_idesc<BF16, kT, kBM>();

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sS = base;                        // operand ring: weight k-block + token k-block
  const uint32_t sH = sS + ST * LY::kStage;        // two cluster hidden buffers
  const uint32_t sBar = sH + 2 * LY::kHidBuf;
  auto full_bar = [&](int s) { return sBar + 8u * s; };
  auto empty_bar = [&](int s) { return sBar + 8u * (ST + s); };
  const uint32_t ufull = sBar + 8u * (2 * ST);
  const uint32_t uempty = sBar + 8u * (2 * ST + 1);
  auto hfull = [&](int b) { return sBar + 8u * (2 * ST + 2 + b); };
  const uint32_t dfull = sBar + 8u * (2 * ST + 4);
  const uint32_t drain_bar = sBar + 8u * (2 * ST + 5);
  const uint32_t epoch_bar = sBar + 8u * (2 * ST + 6);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + (sBar - base) + 8 * (2 * ST + 7));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile unsigned long long* epoch_val =
      reinterpret_cast<volatile unsigned long long*>(gbase + (sBar - base) + 8 * (2 * ST + 8));
  // The 4 epilogue warps wrote their parts of the slice in hidden buffer b (one barrier per
  // buffer: a warp can start the next super-block's slice before the others finish this one).
  auto sdone = [&](int b) { return sBar + 8u * (2 * ST + 9 + b); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t r = cluster_rank();               // rank in the cluster
  const int cl = static_cast<int>(blockIdx.x) / S;  // cluster index
  const int CL = static_cast<int>(gridDim.x) / S;   // clusters launched
  const int SB = p.hs_superblocks;                  // hidden super-blocks of S*128 rows
  const int NBR = p.hs_nbr;                         // 128-row n-blocks of Y per cluster rank
  const int KB = p.up.L;                            // 64-wide k-blocks of K
  const int DC = slice_down_chains(NBR);
  const int n_sb = cl < SB ? (SB - 1 - cl) / CL + 1 : 0;  // super-blocks of this cluster

  if (threadIdx.x == 0) {
#pragma unroll 1
    for (int s = 0; s < ST; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(ufull, 1);
    mbar_init(uempty, LY::kEpiWarps);
    mbar_init(hfull(0), 1);
    mbar_init(hfull(1), 1);
    mbar_init(dfull, 1);
    mbar_init(drain_bar, 1);
    mbar_init(epoch_bar, 1);
    mbar_init(sdone(0), LY::kEpiWarps);
    mbar_init(sdone(1), LY::kEpiWarps);
    *abort_flag = 0;
    fence_barrier_init();
    fence_async_shared();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&p.tm_a_up);
    prefetch_tmap(&p.tm_b_up);
    prefetch_tmap(&p.tm_a_dn);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), LY::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // every peer's barriers are initialised before any copy lands on them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) grid_dep_launch();
  grid_dep_wait();
  if (threadIdx.x == 0) trace_mark(p, kTrStart);

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      auto next = [&](uint32_t bytes) -> bool {
        if (!wait_bar(empty_bar(stage), phase ^ 1u, abort_flag, p, 100 + stage)) return false;
        mbar_expect_tx(full_bar(stage), bytes);
        return true;
      };
      auto advance = [&]() {
        if (issued == 0) trace_mark(p, kTrFirstLoad);
        ++issued;
        if (++stage == ST) { stage = 0; phase ^= 1u; }
      };
#pragma unroll 1
      for (int i = 0; i < n_sb && ok; ++i) {
        const int sb = cl + i * CL;
        const int h0 = (sb * S + static_cast<int>(r)) * kBM;  // this CTA's hidden rows
#pragma unroll 1
        for (int kb = 0; kb < KB; ++kb) {  // up: W1 rows h0.. and the 16 token rows
          if (!next(LY::kStage)) { ok = false; break; }
          const uint32_t st = sS + stage * LY::kStage;
          tma_load_2d(st, &p.tm_a_up, kb * kBK, h0, full_bar(stage));
          tma_load_2d(st + LY::kWBytes, &p.tm_b_up, kb * kBK, 0, full_bar(stage));
          advance();
        }
        const int hc0 = sb * S * kBM;  // the cluster's hidden columns
#pragma unroll 1
        for (int nb = 0; nb < NBR && ok; ++nb) {  // down: W2 tiles of this rank's n-blocks
          const int n0 = (static_cast<int>(r) * NBR + nb) * kBM;
#pragma unroll 1
          for (int kb = 0; kb < 2 * S; ++kb) {
            if (!next(LY::kWBytes)) { ok = false; break; }
            tma_load_2d(sS + stage * LY::kStage, &p.tm_a_dn, hc0 + kb * kBK, n0, full_bar(stage));
            advance();
          }
        }
      }
      trace_mark(p, kTrLastLoad);
      const long long first = issued > ST ? issued - ST : 0;
      const uint64_t t0 = gtimer();
      bool late = false;
#pragma unroll 1
      for (long long i = first; i < issued && !late; ++i) {
        const int s = static_cast<int>(i % ST);
        const uint32_t par = static_cast<uint32_t>((i / ST) & 1);
        while (!mbar_try_wait(full_bar(s), par)) {
          if (gtimer() - t0 > p.wait_limit_ns) { late = true; break; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const uint32_t d_up = tmem_base;
      const uint32_t d_dn = tmem_base + static_cast<uint32_t>(LY::kUpCols);
#pragma unroll 1
      for (int i = 0; i < n_sb && ok; ++i) {
        if (!wait_bar(uempty, (i & 1) ^ 1u, abort_flag, p, 200)) { ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int kb = 0; kb < KB; ++kb) {
          if (!wait_bar(full_bar(stage), phase, abort_flag, p, 300 + stage)) { ok = false; break; }
          tc_fence_after();
          const uint32_t st = sS + stage * LY::kStage;
          const uint64_t da = sw128_desc(st);
          const uint64_t db = sw128_desc(st + LY::kWBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            const int ks = kb * (kBK / 16) + k;
            umma_f16(d_up + static_cast<uint32_t>((ks % LY::kUpChains) * kT), da + 2 * k, db + 2 * k, kIdesc,
                     ks >= LY::kUpChains ? 1u : 0u);
          }
          umma_commit(empty_bar(stage));
          if (++stage == ST) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit(ufull);
        // The cluster's hidden columns: this CTA's slice and its peers' copies.
        const int b = i & 1;
        if (!wait_bar<true>(hfull(b), static_cast<uint32_t>((i >> 1) & 1), abort_flag, p, 220 + b)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t hb = sH + static_cast<uint32_t>(b * LY::kHidBuf);
#pragma unroll 1
        for (int nb = 0; nb < NBR && ok; ++nb) {
#pragma unroll 1
          for (int kb = 0; kb < 2 * S; ++kb) {
            if (!wait_bar(full_bar(stage), phase, abort_flag, p, 300 + stage)) { ok = false; break; }
            tc_fence_after();
            const uint64_t da = sw128_desc(sS + stage * LY::kStage);
            const uint64_t db = sw128_desc(hb + static_cast<uint32_t>(kb * LY::kKbBytes));
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k) {
              const int ks = kb * (kBK / 16) + k;
              const uint32_t d = d_dn + static_cast<uint32_t>((nb * DC + ks % DC) * kT);
              umma_f16(d, da + 2 * k, db + 2 * k, kIdesc, (i > 0 || ks >= DC) ? 1u : 0u);
            }
            umma_commit(empty_bar(stage));
            if (++stage == ST) { stage = 0; phase ^= 1u; }
          }
        }
      }
      if (ok) umma_commit(dfull);
      trace_mark(p, kTrLastMma);
      umma_commit(drain_bar);
      const uint64_t t0 = gtimer();
      while (!mbar_try_wait(drain_bar, 0)) {
        if (gtimer() - t0 > p.wait_limit_ns) break;
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5)
    const int ew = warp - kCtrlThreads / 32;  // 0..3
    const int sub = warp & 3;                 // TMEM lane sub-partition of this warp
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const int hl = sub * 32 + lane;           // hidden row of this CTA's slice (TMEM lane)
    if (ew == 0 && lane == 0) {  // this CTA's share of the launch count -> the launch epoch
      const unsigned long long old = atomicAdd(p.launches, 1ull);
      *epoch_val = old / gridDim.x + 1ull;
      mbar_arrive(epoch_bar);
    }
    auto warp_wait = [&](uint32_t bar, uint32_t par, int aux) {
      int v = 1;
      if (lane == 0) v = wait_bar(bar, par, abort_flag, p, aux) ? 1 : 0;
      return __shfl_sync(0xffffffffu, v, 0);
    };
    int ok = 1;
    int i = 0;
#pragma unroll 1
    for (; i < n_sb && ok; ++i) {
      const int sb = cl + i * CL;
      ok = warp_wait(ufull, i & 1, 400);
      if (!ok) break;
      tc_fence_after();
      float v[kT];
      {  // the 4 K chains, two per TMEM round trip, summed in chain order
        static_assert(LY::kUpChains == 4, "up chains");
        float w[kT], a[kT], b[kT];
        tmem_ld16x2(tmem_base + lane_off, tmem_base + lane_off + kT, v, w);
        tmem_ld16x2(tmem_base + lane_off + 2 * kT, tmem_base + lane_off + 3 * kT, a, b);
#pragma unroll
        for (int j = 0; j < kT; ++j) v[j] = ((v[j] + w[j]) + a[j]) + b[j];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(uempty);
      const int h = (sb * S + static_cast<int>(r)) * kBM + hl;
      if (p.bias1 && h < p.H) {
        const float bv = unpack_lo<BF16>(static_cast<uint32_t>(__ldg(p.bias1 + h)));
#pragma unroll
        for (int j = 0; j < kT; ++j) v[j] += bv;
      }
      // This CTA's slot of hidden buffer b: k-block hl/64 of the slice, token row t, the
      // 16-byte chunk (hl%64)/8 (128B-swizzled by t) and the element hl%8 inside it.
      const int b = i & 1;
      const uint32_t slot = sH + static_cast<uint32_t>(b * LY::kHidBuf + static_cast<int>(r) * LY::kSlice);
      const uint32_t kbase = slot + static_cast<uint32_t>((hl >> 6) * LY::kKbBytes + (hl & 7) * 2);
      const int chunk = (hl & 63) >> 3;
#pragma unroll
      for (int t = 0; t < kT; ++t) {
        const uint16_t hv = cvt1<BF16>(gelu<GELU>(v[t]));
        const uint32_t addr = kbase + static_cast<uint32_t>(t * 128 + ((chunk ^ (t & 7)) << 4));
        asm volatile("st.shared.b16 [%0], %1;" ::"r"(addr), "h"(hv) : "memory");
      }
      fence_async_shared();  // generic stores, then the async proxy (MMA, bulk copies) reads them
      __syncwarp();
      if (lane == 0) mbar_arrive(sdone(b));
      if (ew == 0) {
        // Once all 4 warps' parts are written: own arrival with the peers' bytes to come, then
        // this slice into every peer's slot.  (An mbarrier with a bounded wait, not a named
        // barrier: a warp that aborted never arrives, and the wait then ends.)
        ok = warp_wait(sdone(b), static_cast<uint32_t>((i >> 1) & 1), 450);
        if (!ok) break;
        if (lane == 0) {
          asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(hfull(b)),
                       "r"(static_cast<uint32_t>((S - 1) * LY::kSlice))
                       : "memory");
#pragma unroll 1
          for (int q = 1; q < S; ++q) {
            const uint32_t peer = (r + static_cast<uint32_t>(q)) % S;
            bulk_copy_to_peer(map_to_rank(slot, peer), slot, LY::kSlice, map_to_rank(hfull(b), peer));
          }
        }
        __syncwarp();
      }
    }
    if (ew == 0 && lane == 0) trace_mark(p, kTrUpStored);  // this CTA's slices are out
    unsigned long long epoch = 0;
    if (ok) {
      // Down accumulators: rows n of this rank's n-blocks, 16 token columns, DC chains each.
      ok = warp_wait(dfull, 0, 440);
      if (ok) {
        if (ew == 0 && lane == 0) trace_mark(p, kTrFirstDown);  // down accumulators complete
        tc_fence_after();
        const size_t npad = static_cast<size_t>(S) * NBR * kBM;  // partial rows per cluster
        // Partial layout: [cluster][token quad q][row n][4 tokens] fp32, so the 32 lanes of a
        // warp (consecutive rows) store 512 contiguous bytes per token quad.
        float4* part = reinterpret_cast<float4*>(p.ws) + static_cast<size_t>(cl) * 4 * npad;
        // The down accumulators are TMEM columns [64, 64 + NBR*DC*16): 64 columns (64/(DC*16)
        // n-blocks, DC chains each) per round trip; the chains are summed in chain order.
        auto drain = [&](auto dc_tag) {
          constexpr int kDC = decltype(dc_tag)::value;
          constexpr int kPer = 64 / (kDC * kT);
#pragma unroll 1
          for (int nb0 = 0; nb0 < NBR; nb0 += kPer) {
            float v64[64];
            tmem_ld64(tmem_base + lane_off + static_cast<uint32_t>(LY::kUpCols + nb0 * kDC * kT), v64);
#pragma unroll
            for (int k = 0; k < kPer; ++k) {
              if (nb0 + k >= NBR) break;
              float v[kT];
#pragma unroll
              for (int j = 0; j < kT; ++j) {
                float a = v64[k * kDC * kT + j];
#pragma unroll
                for (int c = 1; c < kDC; ++c) a += v64[(k * kDC + c) * kT + j];
                v[j] = n_sb == 0 ? 0.0f : a;  // (a cluster without a super-block: none is launched)
              }
              const size_t n = static_cast<size_t>((static_cast<int>(r) * NBR + nb0 + k) * kBM + hl);
#pragma unroll
              for (int q = 0; q < kT / 4; ++q)
                part[static_cast<size_t>(q) * npad + n] =
                    make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            }
          }
        };
        if (DC == 4) drain(std::integral_constant<int, 4>{});
        else if (DC == 2) drain(std::integral_constant<int, 2>{});
        else drain(std::integral_constant<int, 1>{});
        if (ew == 0 && lane == 0) trace_mark(p, 14);
        // The warp barrier orders every lane's stores before lane 0's release (cumulative at
        // GPU scope); readers acquire the count, then fence the async proxy before their bulk
        // copies of the partials.
        __syncwarp();
        if (lane == 0) red_release_add(p.counters + r, 1u);
        if (ew == 0 && lane == 0) trace_mark(p, kTrDownReady);  // this CTA's partial released
        // Reduction of this rank's Y rows: every rank-r CTA of the CL clusters takes an equal
        // share [row0, row0 + nrows).  Work item (token quad q, row): the CL partial float4s
        // (one per cluster; a warp's 32 rows are 512 contiguous bytes of each) are loaded 32 at
        // a time, then summed in ascending cluster order.
        const int rows_r = NBR * kBM;              // Y rows of rank r
        const int share = (rows_r + CL - 1) / CL;  // rows per rank-r CTA
        const int row0 = static_cast<int>(r) * rows_r + cl * share;
        const int nrows = max(0, min(share, rows_r - cl * share));
        if (lane == 0) {
          ok = wait_bar(epoch_bar, 0u, abort_flag, p, 700) ? 1 : 0;
          if (ok) epoch = *epoch_val;
          if (ok)
            ok = wait_word_ge(p.counters + r,
                              static_cast<unsigned>(LY::kEpiWarps * CL) * static_cast<unsigned>(epoch) +
                                  (p.inject ? 1u : 0u),  // (fault injection: a count that never arrives)
                              abort_flag, p, 3, static_cast<int>(r))
                     ? 1 : 0;
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        __syncwarp();  // (orders every lane's loads after lane 0's acquire)
        if (ok && ew == 0 && lane == 0) trace_mark(p, kTrAux1);  // every cluster's partial of rank r released
        if (ok && nrows > 0) {
          uint16_t* y = reinterpret_cast<uint16_t*>(p.y);
          const float4* base4 = reinterpret_cast<const float4*>(p.ws);
#pragma unroll 1
          for (int it = ew * 32 + lane; it < nrows * (kT / 4); it += 32 * LY::kEpiWarps) {
            const int q = it / nrows;
            const int n = row0 + (it - q * nrows);
            const float4* src = base4 + static_cast<size_t>(q) * npad + n;  // cluster 0's float4
            const size_t cstride = 4 * npad;                                 // next cluster
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            constexpr int kBatch = 32;  // (32 clusters' float4s in flight per thread: one L2 round trip for cfg3)
#pragma unroll 1
            for (int c0 = 0; c0 < CL; c0 += kBatch) {
              float4 t[kBatch];
#pragma unroll
              for (int b = 0; b < kBatch; ++b)
                if (c0 + b < CL) t[b] = __ldcg(src + static_cast<size_t>(c0 + b) * cstride);
#pragma unroll
              for (int b = 0; b < kBatch; ++b)
                if (c0 + b < CL) {
                  if (c0 + b == 0) {
                    acc = t[b];
                  } else {
                    acc.x += t[b].x; acc.y += t[b].y; acc.z += t[b].z; acc.w += t[b].w;
                  }
                }
            }
            if (n < p.N) {
              float vals[4] = {acc.x, acc.y, acc.z, acc.w};
              const float bv = p.bias2 ? unpack_lo<BF16>(static_cast<uint32_t>(__ldg(p.bias2 + n))) : 0.0f;
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int t = 4 * q + e;
                if (t < p.M) y[static_cast<long long>(t) * p.ldy + n] = cvt1<BF16>(vals[e] + bv);
              }
            }
          }
        }
        if (ok && ew == 0 && lane == 0) trace_mark(p, kTrAux2);
      }
    }
    if (ok && ew == 0 && lane == 0) trace_mark(p, kTrAux3);  // this CTA's Y rows written
    // Every slice copied into this CTA lands before the CTA may leave (bounded, one deadline):
    // the hidden buffers' phases this CTA's MMA did not wait for (abort paths).
    if (lane == 0 && ew == 0 && !ok) {
      const uint64_t t0 = gtimer();
#pragma unroll 1
      for (int j = 0; j < n_sb; ++j) {
        while (!mbar_try_wait_cluster(hfull(j & 1), static_cast<uint32_t>((j >> 1) & 1))) {
          if (gtimer() - t0 > p.wait_limit_ns) break;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while a peer may still copy into it or read its partials' flags
  tc_fence_after();
  if (threadIdx.x == 0) trace_mark(p, kTrEnd);
  if (warp == 1) tmem_dealloc(tmem_base, LY::kTmemCols);
}

}  // namespace ffnb200
