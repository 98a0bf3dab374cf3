// Row-block FFN with the hidden activations resident on chip: the B200 form of the
// reference's down_impl "full_load_a" (the down GEMM's A operand -- the hidden row block --
// fully loaded on chip instead of streamed from global memory; ops/host/dispatch.py:15,
// spec/v1_spec.md:156).
//
// One CTA owns 128 tokens (a row block) at a time and walks H in chunks of 128 columns:
//
//   up(j):   D_up[j%2]  = X[rb, :] . W1[128j : 128j+128, :]^T      (TMEM, fp32, 128 cols)
//   epi(j):  hid[j%2]   = RN(GELU(D_up[j%2]))                       (shared memory, 128B-swizzled
//                                                                    K-major: the A operand)
//   down(j): D_y       += hid[j%2] . W2[:, 128j : 128j+128]^T       (TMEM, fp32, NY cols)
//
// and after the last chunk stores D_y as Y[rb, :N].  The MMA issuer runs up(j+1) while the
// epilogue converts chunk j, so the tensor core alternates up and down chunks:
// up(0) up(1) down(0) up(2) down(1) ... down(J-1).  Hidden never reaches global memory and
// no CTA waits on another, so the launch needs no co-residency.  TMEM holds both up
// accumulators (256 columns) and the Y accumulator (NY <= 256 columns): the variant
// applies when N <= 2 * NY (see the Y column parts below).
//
// Y wider than the accumulator (NY < N <= 2*NY): the Y columns are split into NS = ceil(N/NY)
// parts, and a row unit (row block, part) computes Y[rb, part*NY : part*NY + NY]; each part
// recomputes the row block's hidden chunks (the up work is done NS times), which keeps both
// parts free of any exchange.  Units are dealt to CTAs (or clusters) like row blocks.
//
// Arithmetic is that of the two-phase kernel: fp32 accumulation over K, GELU of the fp32
// sum, hidden rounded once to the input dtype, fp32 accumulation over H, one rounding of
// Y.  Only the order of the H summation differs (chunks of 128 in ascending order, inside
// one accumulator).
//
// Few row blocks (M <= 128 * SMs / 2): a cluster of S = Params::rb_split CTAs (2, 4 or 8)
// shares each row block, CTA s taking H chunks [s*J/S, (s+1)*J/S), so S times as many SMs work and
// each walks 1/S of the chain.  At the end every CTA leaves the fp32 Y partials of the
// column chunks it does not finalise in its own (then idle) operand ring; Y column chunk yc is finalised by CTA yc % S, which after
// a cluster barrier reads the other CTAs' partials of it over distributed shared memory and
// sums all S in rank order (fixed, so the result is the same on every run); a second
// barrier keeps every CTA resident until the others have read its partials.
#pragma once

#include "ffn_kernel.cuh"

namespace ffnb200 {

template <int NY, int STAGES>
struct RowLayout {
  static constexpr int kEpiWarps = 16;                  // four per TMEM sub-partition
  static constexpr int kThreads = kCtrlThreads + 32 * kEpiWarps;
  static constexpr int kChunk = 128;                    // H columns per up chunk
  static constexpr int kStage = 32768;                  // X + W1 k-block, or one W2 k-block
  static constexpr int kHidBuf = kChunk * kBM * 2;      // one hidden chunk: 2 k-blocks of 16 KB
  static constexpr int kBarBytes = 256;
  static constexpr int kSmem = 1024 + STAGES * kStage + 2 * kHidBuf + kBarBytes;
  static constexpr int kTmemCols = 512;                 // up accumulators 0..255, Y 256..256+NY
  static_assert(NY == 64 || NY == 128 || NY == 256, "Y accumulator width");
  static_assert(NY * kBK * 2 <= kStage, "W2 k-block fits a stage");
  static_assert((2 * STAGES + 12) * 8 + 8 <= kBarBytes, "barrier area");
  static_assert(kSmem <= 232448, "dynamic shared memory per CTA");
  // A split row block's Y partial (kBM x 256 fp32) lives in the operand ring at the end.
  static_assert(STAGES * kStage >= kBM * 256 * 4, "Y partial fits the operand ring");
};

template <int NY, int STAGES, bool BF16, int GELU>
__global__ void __launch_bounds__(kCtrlThreads + 32 * 16, 1) ffn_rowblock_kernel(const __grid_constant__ Params p) {
  using LY = RowLayout<NY, STAGES>;
  constexpr uint32_t kIdescUp = make_idesc<BF16, LY::kChunk, kBM>();
  constexpr uint32_t kIdescDn = make_idesc<BF16, NY, kBM>();
  constexpr uint32_t kUpBytes = 2 * kABytes;           // X k-block + W1 k-block (128 rows each)
  constexpr uint32_t kDnBytes = NY * kBK * 2;          // W2 k-block
  // SwiGLU (GELU == 3): a 128-row chunk of the packed W1 holds 64 gate rows then the matching
  // 64 up rows, so each chunk yields 64 hidden columns: one k-block of the down GEMM.
  constexpr bool kGlu = GELU == 3;
  constexpr int kHidKb = kGlu ? 1 : 2;                 // down k-blocks per chunk

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t sS = base;                             // operand ring
  const uint32_t sH = sS + STAGES * LY::kStage;         // two hidden chunk buffers
  const uint32_t sBar = sH + 2 * LY::kHidBuf;
  auto full_bar = [&](int s) { return sBar + 8u * s; };
  auto empty_bar = [&](int s) { return sBar + 8u * (STAGES + s); };
  auto ufull = [&](int a) { return sBar + 8u * (2 * STAGES + a); };
  auto uempty = [&](int a) { return sBar + 8u * (2 * STAGES + 2 + a); };
  auto hfull = [&](int b) { return sBar + 8u * (2 * STAGES + 4 + b); };
  auto hempty = [&](int b) { return sBar + 8u * (2 * STAGES + 6 + b); };
  const uint32_t yfull = sBar + 8u * (2 * STAGES + 8);
  const uint32_t yempty = sBar + 8u * (2 * STAGES + 9);
  const uint32_t drain_bar = sBar + 8u * (2 * STAGES + 10);
  const uint32_t ystage_free = sBar + 8u * (2 * STAGES + 11);  // Y staging read by its TMA stores
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + (sBar - base) + 8 * (2 * STAGES + 12));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int RB = p.up.tiles_r;   // row blocks
  const int NS = (p.N + NY - 1) / NY;  // Y column parts
  const int units = RB * NS;     // (row block, Y part) units
  const int J = p.up.tiles_q;    // H chunks
  const int KB = p.up.L;         // 64-wide k-blocks of K
  // H split: CTA `srank` of a cluster of S takes chunks [j0, j0 + Js) of its row block.
  const int S = p.rb_split > 1 ? p.rb_split : 1;
  const int srank = S > 1 ? static_cast<int>(cluster_rank()) : 0;
  const int j0 = srank * J / S;
  const int Js = (srank + 1) * J / S - j0;
  const int un_first = static_cast<int>(blockIdx.x) / S;
  const int un_step = static_cast<int>(gridDim.x) / S;

  if (threadIdx.x == 0) {
#pragma unroll 1
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(ufull(a), 1);
      mbar_init(uempty(a), LY::kEpiWarps);
      mbar_init(hfull(a), LY::kEpiWarps);
      mbar_init(hempty(a), 1);
    }
    mbar_init(yfull, 1);
    mbar_init(yempty, LY::kEpiWarps);
    mbar_init(drain_bar, 1);
    mbar_init(ystage_free, LY::kEpiWarps);
    *abort_flag = 0;
    fence_barrier_init();
    fence_async_shared();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&p.tm_a_up);
    prefetch_tmap(&p.tm_b_up);
    prefetch_tmap(&p.tm_b_dn);
    prefetch_tmap(&p.tm_st_y);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), LY::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // On-chip setup above; every global access below (overlapped launches, see grid_dep_wait).
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
      auto next_stage = [&]() -> bool {
        if (!wait_bar(empty_bar(stage), phase ^ 1u, abort_flag, p, 100 + stage)) return false;
        return true;
      };
      auto advance = [&]() {
        ++issued;
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      };
#pragma unroll 1
      for (int un = un_first; un < units && ok; un += un_step) {
        const int rb = un / NS;
        const int ycol0 = (un % NS) * NY;
#pragma unroll 1
        for (int jj = 0; jj <= Js && ok; ++jj) {
          const int j = j0 + jj;
          if (jj < Js) {  // up(j): X and W1 k-blocks
#pragma unroll 1
            for (int kb = 0; kb < KB; ++kb) {
              if (!next_stage()) { ok = false; break; }
              const uint32_t st = sS + stage * LY::kStage;
              mbar_expect_tx(full_bar(stage), kUpBytes);
              tma_load_2d(st, &p.tm_a_up, kb * kBK, rb * kBM, full_bar(stage));
              tma_load_2d(st + kABytes, &p.tm_b_up, kb * kBK, j * LY::kChunk, full_bar(stage));
              if (issued == 0) trace_mark(p, kTrFirstLoad);
              advance();
            }
          }
          if (ok && jj >= 1) {  // down(j-1): the two W2 k-blocks of chunk j-1
#pragma unroll 1
            for (int kk = 0; kk < kHidKb; ++kk) {
              if (!next_stage()) { ok = false; break; }
              mbar_expect_tx(full_bar(stage), kDnBytes);
              tma_load_2d(sS + stage * LY::kStage, &p.tm_b_dn, ((j - 1) * kHidKb + kk) * kBK, ycol0, full_bar(stage));
              advance();
            }
          }
        }
      }
      trace_mark(p, kTrLastLoad);
      // Every issued load lands before the CTA may exit (one deadline for the drain).
      const long long first = issued > STAGES ? issued - STAGES : 0;
      const uint64_t t0 = gtimer();
      bool late = false;
#pragma unroll 1
      for (long long i = first; i < issued && !late; ++i) {
        const int s = static_cast<int>(i % STAGES);
        const uint32_t par = static_cast<uint32_t>((i / STAGES) & 1);
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
      int ucnt = 0, dcnt = 0, rcnt = 0;
      bool ok = true;
      auto up_chunk = [&]() -> bool {
        const int a = ucnt & 1;
        if (!wait_bar(uempty(a), ((ucnt >> 1) & 1) ^ 1u, abort_flag, p, 200 + a)) return false;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(a * LY::kChunk);
#pragma unroll 1
        for (int kb = 0; kb < KB; ++kb) {
          if (!wait_bar(full_bar(stage), phase, abort_flag, p, 300 + stage)) return false;
          tc_fence_after();
          const uint32_t st = sS + stage * LY::kStage;
          const uint64_t da = sw128_desc(st);
          const uint64_t db = sw128_desc(st + kABytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_f16(d, da + 2 * k, db + 2 * k, kIdescUp, (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(empty_bar(stage));
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        umma_commit(ufull(a));
        ++ucnt;
        return true;
      };
      auto down_chunk = [&](bool first) -> bool {
        const int b = dcnt & 1;
        if (!wait_bar(hfull(b), (dcnt >> 1) & 1, abort_flag, p, 220 + b)) return false;
        if (first && !wait_bar(yempty, (rcnt & 1) ^ 1u, abort_flag, p, 240)) return false;
        tc_fence_after();
        const uint32_t d = tmem_base + 256u;
#pragma unroll 1
        for (int kk = 0; kk < kHidKb; ++kk) {
          if (!wait_bar(full_bar(stage), phase, abort_flag, p, 300 + stage)) return false;
          tc_fence_after();
          const uint64_t da = sw128_desc(sH + b * LY::kHidBuf + kk * kABytes);
          const uint64_t db = sw128_desc(sS + stage * LY::kStage);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_f16(d, da + 2 * k, db + 2 * k, kIdescDn, (!first || kk > 0 || k > 0) ? 1u : 0u);
          umma_commit(empty_bar(stage));
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        umma_commit(hempty(b));
        ++dcnt;
        return true;
      };
#pragma unroll 1
      for (int un = un_first; un < units && ok; un += un_step) {
#pragma unroll 1
        for (int jj = 0; jj <= Js && ok; ++jj) {
          if (jj < Js && !up_chunk()) ok = false;
          if (ok && jj >= 1 && !down_chunk(jj == 1)) ok = false;
        }
        if (!ok) break;
        umma_commit(yfull);
        ++rcnt;
      }
      trace_mark(p, kTrLastMma);
      umma_commit(drain_bar);
      const uint64_t t0 = gtimer();
      while (!mbar_try_wait(drain_bar, 0)) {
        if (gtimer() - t0 > p.wait_limit_ns) break;
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..17)
    // Four warps per TMEM sub-partition; warp `part` of a sub-partition converts columns
    // part*32 .. part*32+31 of each 128-column chunk for its 32 rows.
    const int ew = warp - kCtrlThreads / 32;  // 0..15
    const int sub = warp & 3;                 // TMEM lane sub-partition this warp may access
    const int part = ew >> 2;                 // 32-column quarter of a chunk
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const int row = sub * 32 + lane;          // row of the block
    // This warp's 64-byte half rows of hidden buffer b: k-block part/2, 16-byte chunks
    // (part&1)*4 .. +3 of row `row` (128B-swizzled, the MMA's K-major A layout).
    auto hid_row = [&](int b) {
      return sH + static_cast<uint32_t>(b * LY::kHidBuf + (part >> 1) * kABytes + row * 128);
    };
    // Y staging: 4 KB per warp (32 rows x 128 B) over the idle hidden buffers.
    const uint32_t ystage = sH + static_cast<uint32_t>(ew * 4096);
    int ucnt = 0, hcnt = 0, rcnt = 0;
    bool y_staged = false;  // this CTA's last Y staging may still be read by TMA stores
    int ok = 1;
    auto warp_wait = [&](uint32_t bar, uint32_t par, int aux) {
      int r = 1;
      if (lane == 0) r = wait_bar(bar, par, abort_flag, p, aux) ? 1 : 0;
      return __shfl_sync(0xffffffffu, r, 0);
    };
    // 16 packed words = 32 columns as four swizzled 16-byte chunks c0..c0+3 of a 128-byte row.
    auto store_quarter = [&](uint32_t row_addr, int swz_row, int c0, const uint32_t* pk) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint32_t addr = row_addr + (((c0 + c) ^ (swz_row & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(pk[4 * c]), "r"(pk[4 * c + 1]),
                     "r"(pk[4 * c + 2]), "r"(pk[4 * c + 3])
                     : "memory");
      }
    };
#pragma unroll 1
    for (int un = un_first; un < units && ok; un += un_step) {
      const int rb = un / NS;
      const int ycol0 = (un % NS) * NY;
#pragma unroll 1
      for (int jj = 0; jj < Js && ok; ++jj) {
        const int j = j0 + jj;
        const int a = ucnt & 1;
        ok = warp_wait(ufull(a), (ucnt >> 1) & 1, 400 + a);
        if (!ok) break;
        tc_fence_after();
        float v[32];
        if constexpr (kGlu) {  // gate and up sums of hidden columns part*16 .. part*16+15
          tmem_ld16(tmem_base + lane_off + static_cast<uint32_t>(a * LY::kChunk + part * 16), v);
          tmem_ld16(tmem_base + lane_off + static_cast<uint32_t>(a * LY::kChunk + 64 + part * 16), v + 16);
        } else {
          tmem_ld32(tmem_base + lane_off + static_cast<uint32_t>(a * LY::kChunk + part * 32), v);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(uempty(a));
        ++ucnt;
        uint32_t pk[16];
        if constexpr (kGlu) {
#pragma unroll
          for (int i = 0; i < 8; ++i)
            pk[i] = pack2<BF16>(silu(v[2 * i]) * v[16 + 2 * i], silu(v[2 * i + 1]) * v[16 + 2 * i + 1]);
        } else {
          if (p.bias1) add_bias<BF16, 32>(v, p.bias1, j * LY::kChunk + part * 32, p.H);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            gelu2<GELU>(v[2 * i], v[2 * i + 1]);
            pk[i] = pack2<BF16>(v[2 * i], v[2 * i + 1]);
          }
        }
        const int b = hcnt & 1;
        ok = warp_wait(hempty(b), ((hcnt >> 1) & 1) ^ 1u, 420 + b);
        if (ok && y_staged) {  // every warp's Y stores have read the staging this write overlaps
          ok = warp_wait(ystage_free, (rcnt - 1) & 1, 460);
          y_staged = false;
        }
        if (!ok) break;
        if constexpr (kGlu) {  // 16 columns = 16-byte chunks part*2, part*2+1 of k-block 0
          const uint32_t row_addr = sH + static_cast<uint32_t>(b * LY::kHidBuf + row * 128);
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const uint32_t addr = row_addr + (((part * 2 + c) ^ (row & 7)) << 4);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(pk[4 * c]), "r"(pk[4 * c + 1]),
                         "r"(pk[4 * c + 2]), "r"(pk[4 * c + 3])
                         : "memory");
          }
        } else {
          store_quarter(hid_row(b), row, (part & 1) * 4, pk);
        }
        fence_async_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive(hfull(b));
        ++hcnt;
      }
      if (!ok) break;
      // Y of the row block: 64-column chunks, one per warp of a sub-partition (NY <= 256).
      ok = warp_wait(yfull, rcnt & 1, 440);
      if (!ok) break;
      if (ew == 0 && lane == 0) trace_mark(p, kTrFirstDown);  // (the last unit's stamp stays)
      tc_fence_after();
      const int yc = part;
      const bool mine = yc < NY / 64 && ycol0 + yc * 64 < p.N;
      if (S > 1) {  // split row block (one per cluster): combined after the loop
        ++rcnt;
        break;
      }
      if (mine) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float v[32];
          tmem_ld32(tmem_base + lane_off + 256u + static_cast<uint32_t>(yc * 64 + h * 32), v);
          if (p.bias2) add_bias<BF16, 32>(v, p.bias2, ycol0 + yc * 64 + h * 32, p.N);
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) pk[i] = pack2<BF16>(v[2 * i], v[2 * i + 1]);
          store_quarter(ystage + lane * 128, lane, h * 4, pk);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(yempty);
      if (mine) {
        fence_async_shared();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&p.tm_st_y, ystage, ycol0 + yc * 64, rb * kBM + sub * 32);
          bulk_commit();
        }
      }
      if (lane == 0) {
        bulk_wait_read0();
        mbar_arrive(ystage_free);
      }
      __syncwarp();
      y_staged = true;
      ++rcnt;
    }
    if (lane == 0) bulk_wait_read0();  // staging read; the stores complete with the grid
    __syncwarp();
  }

  if (S > 1) {
    // Split row block: Y columns [g*GW, (g+1)*GW) of the unit (GW = NY/S, in 8-column units)
    // are finalised by CTA g of the cluster.  (1) Once every CTA's MMAs are done, the operand
    // rings are idle; each CTA stores the fp32 partial of every other CTA's columns straight
    // into that CTA's ring (slot = sender rank; [8-column unit][2 float4][128 rows]), (2) then
    // each finaliser adds the S partials in rank order (its own from TMEM) and stores Y.
    constexpr int kUnits = NY / 8;           // 8-column units of the Y accumulator
    const int gw_units = kUnits / S;          // units per finalising CTA
    tc_fence_before();
    cluster_sync();  // (1) every CTA of the cluster has its final Y partial in TMEM
    tc_fence_after();
    if (threadIdx.x == 0) trace_mark(p, kTrAux1);
    const int un = un_first;  // one unit per cluster
    const int rb = un / NS;
    const int ycol0 = (un % NS) * NY;
    const int ew = warp - kCtrlThreads / 32;
    const bool epi = warp >= kCtrlThreads / 32 && un < units && !*abort_flag;
    const int sub = warp & 3;
    const int part = ew >> 2;
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const int row = sub * 32 + lane;
    auto slot_addr = [&](int sender, int u_local, int half) {  // in the finaliser's ring
      return sS + static_cast<uint32_t>((((sender * gw_units + u_local) * 2 + half) * kBM + row) * 16);
    };
    if (epi) {
      // Part `part` of the epilogue warps pushes the contiguous units [part*kQ, (part+1)*kQ)
      // of its 32 rows, read from TMEM in one round trip.
      constexpr int kQ = kUnits / 4;
      float v[kQ * 8];
      const uint32_t tcol = tmem_base + lane_off + 256u + static_cast<uint32_t>(part * kQ * 8);
      if constexpr (kQ == 8) tmem_ld64(tcol, v);
      else if constexpr (kQ == 4) tmem_ld32(tcol, v);
      else tmem_ld16(tcol, v);
      if (threadIdx.x == kCtrlThreads) trace_mark(p, 12);
#pragma unroll
      for (int k = 0; k < kQ; ++k) {
        const int u = part * kQ + k;
        const int g = u / gw_units;
        if (g == srank || ycol0 + u * 8 >= p.N) continue;
        const uint32_t dst = map_to_rank(slot_addr(srank, u - g * gw_units, 0), static_cast<uint32_t>(g));
        asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "f"(v[8 * k]), "f"(v[8 * k + 1]),
                     "f"(v[8 * k + 2]), "f"(v[8 * k + 3])
                     : "memory");
        asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(dst + kBM * 16), "f"(v[8 * k + 4]),
                     "f"(v[8 * k + 5]), "f"(v[8 * k + 6]), "f"(v[8 * k + 7])
                     : "memory");
      }
    }
    tc_fence_before();
    cluster_sync();  // (2) every partial is in its finaliser's shared memory; no more remote stores
    tc_fence_after();
    if (threadIdx.x == 0) trace_mark(p, kTrAux2);
    // Finalisation: this CTA's units [srank*gw, (srank+1)*gw), `per` contiguous units per part
    // (its own partial read from TMEM in one round trip), summed with the S-1 pushed partials
    // in rank order.
    const int per = gw_units >= 4 ? gw_units / 4 : 1;
    const int ul0 = part * per;
    if (epi && ul0 < gw_units) {
      uint16_t* y = reinterpret_cast<uint16_t*>(p.y);
      const long long grow = static_cast<long long>(rb) * kBM + row;  // token row of Y
      float own[32];
      const uint32_t tcol = tmem_base + lane_off + 256u + static_cast<uint32_t>((srank * gw_units + ul0) * 8);
      if (per >= 4) tmem_ld32(tcol, own);
      else if (per == 2) tmem_ld16(tcol, own);
      else tmem_ld8(tcol, own);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (k >= per) break;
        const int ul = ul0 + k;
        const int u = srank * gw_units + ul;
        const int col = ycol0 + u * 8;
        if (col >= p.N) continue;
        float v[8];
#pragma unroll 1
        for (int s2 = 0; s2 < S; ++s2) {  // partials summed in rank order
          float t[8];
          if (s2 == srank) {
#pragma unroll
            for (int i = 0; i < 8; ++i) t[i] = own[8 * k + i];
          } else {
            const uint32_t a = slot_addr(s2, ul, 0);
            asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(t[0]), "=f"(t[1]), "=f"(t[2]), "=f"(t[3]) : "r"(a)
                         : "memory");
            asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                         : "=f"(t[4]), "=f"(t[5]), "=f"(t[6]), "=f"(t[7])
                         : "r"(a + kBM * 16)
                         : "memory");
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = s2 == 0 ? t[i] : v[i] + t[i];
        }
        if (threadIdx.x == kCtrlThreads) trace_mark(p, 13);
        if (p.bias2) add_bias<BF16, 8>(v, p.bias2, col, p.N);
        if (grow < p.M) {
          uint16_t* dst = y + grow * p.ldy + col;
          if (col + 8 <= p.N) {
            uint4 w;
            w.x = pack2<BF16>(v[0], v[1]); w.y = pack2<BF16>(v[2], v[3]);
            w.z = pack2<BF16>(v[4], v[5]); w.w = pack2<BF16>(v[6], v[7]);
            *reinterpret_cast<uint4*>(dst) = w;
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              if (col + i < p.N) dst[i] = cvt1<BF16>(v[i]);
          }
        }
      }
    }
  }
  if (threadIdx.x == kCtrlThreads) trace_mark(p, kTrAux3);  // first epilogue warp done
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0) trace_mark(p, kTrEnd);
  if (warp == 1) tmem_dealloc(tmem_base, LY::kTmemCols);
}

}  // namespace ffnb200
