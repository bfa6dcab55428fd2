// Persistent grouped NVFP4 GEMM for sm_100a: TMA-fed shared-memory pipeline, tcgen05 block-scaled MMA
// (kind::mxf4nvf4, ue4m3 scale per 16 elements applied inside the MMA), fp32 accumulator in TMEM, fused epilogues.
//
//   D[m, n] = alpha[g] * sum_k (a[m, k] * sfa[m, k/16]) * (b[g*N + n, k] * sfb[g*N + n, k/16])
//
// Roles (448 threads, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: per k-block first the stage's scale atoms (plain bulk copies, on the stage's sf_full
//               barrier), then the A tile 128 x 256 (e2m1, 128-byte swizzle) and the B tile BN x 256 (on its full
//               barrier); STAGES-deep ring of shared-memory stages freed through the empty barriers.
//   warp 1      TMEM owner and MMA issuer (one thread): per k-block, once the stage's operands landed and its scales
//               are in TMEM, 4 MMAs of K = 64; tcgen05.commit frees the stage and, after the tile's last k-block,
//               signals the accumulator full.
//   warps 2, 11-13  scale writers, one per TMEM lane quarter (warp % 4): per k-block each reads the stage's scale
//               atoms from shared memory and writes with tcgen05.st exactly the words its quarter's MMA datapath
//               reads (the scale of row m sits in lane m % 32 of every quarter, column m / 32: the A scales of the
//               quarter's own 32 rows, the B scales of all BN rows), then arrives on the stage's sf barrier. This
//               replaces 4 + 4 * BN / 128 tcgen05.cp copies per k-block, each of which held the tensor pipe about
//               55 cycles beside 512 cycles of MMAs; the scales are loaded first so that the writers finish while
//               the operand tiles are still landing.
//   warps 3-10  epilogue: two warps per TMEM lane quadrant (32 rows), each owning half of the tile's columns; a warp
//               copies its accumulator share to registers (tcgen05.ld), releases the accumulator so the MMAs of the
//               next tile start, then runs the output stage from registers, overlapping the next mainloop. The bf16
//               output goes through a per-warp shared-memory buffer in the 128-byte swizzle layout and leaves by TMA
//               tensor stores (32 rows x 64 columns each), so the warp moves on while the copy engine writes.
// Tiles are M-major over N tiles (consecutive CTAs share the A row block and walk one expert's weights), so an
// expert's weights stay in L2 while its row blocks are in flight.
// CTA pairs (PAIR; the grouped down projection over a pair table, dense bf16 GEMMs over row blocks 2p, 2p + 1): a
// cluster of two CTAs computes 256 rows x BN with tcgen05.mma.cta_group::2 issued by the leader (rank 0). Each CTA
// TMA-loads its own 128 A rows and half of the B tile into its own shared memory, both completing on the leader's
// full barrier, which the leader arms for both; each CTA's scale writers fill its own TMEM (its A rows, all BN B
// rows) and arrive on the leader's sf barrier; the leader's commits signal the empty / accumulator barriers of both CTAs; each CTA's
// epilogue drains its own 128 rows and releases the accumulator on the leader's barrier. A stage is then 38 KB
// instead of 54, so five fit. Cross-CTA arrives use the default (CTA-scope release) form: a cluster-scope release
// measured ~1,400 cycles each.
// Every wait is bounded (common.cuh); on expiry all roles leave, in-flight copies and MMAs are drained with bounded
// waits, TMEM is freed and the status word holds kErrTimeout.

#include "common.cuh"
#include "ops.h"

namespace ssb {

namespace {

constexpr int kBM = 128;
constexpr int kBKBytes = 128;   // one k-block: 256 e2m1 elements = 128 bytes = one 128-byte swizzle row
constexpr int kThreads = 448;   // warp 0 TMA, warp 1 MMA, warps 2 and 11-13 scale writers, warps 3-10 epilogue
constexpr int kEpiWarp0 = 3;
constexpr int kEpiWarps = 8;
constexpr int kOutStage = 4096; // bf16 epilogue: per-warp staging buffer, 32 rows x 64 columns

template <int BN, int EPI, bool PAIR>
struct Cfg {
  // PAIR: the two CTAs of a cluster share each MMA (cta_group::2, M = 256): each holds its own 128 A rows and half of
  // the BN B rows, so a stage is 38 KB instead of 54 and five fit. Otherwise the bf16 epilogue's staging buffers take
  // the room of one stage.
  static constexpr int STAGES = PAIR ? 5 : BN == 256 ? (EPI == kEpiBF16 ? 3 : 4) : 6;
  static constexpr int A_BYTES = kBM * kBKBytes;               // 16 KB
  static constexpr int B_BYTES = (PAIR ? BN / 2 : BN) * kBKBytes;
  static constexpr int SFA_BYTES = 2048;                        // 4 atoms (128 rows x 64 K each)
  static constexpr int SFB_BYTES = (BN / 128) * 2048;
  static constexpr int AB_TX = A_BYTES + B_BYTES;               // one CTA's operand bytes per stage
  static constexpr int SF_TX = SFA_BYTES + SFB_BYTES;
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + STAGES * A_BYTES;
  static constexpr int OFF_SFA = OFF_B + STAGES * B_BYTES;
  static constexpr int OFF_SFB = OFF_SFA + STAGES * SFA_BYTES;
  static constexpr int OFF_OUT = OFF_SFB + STAGES * SFB_BYTES;
  static constexpr int OUT_BYTES = EPI == kEpiBF16 ? kEpiWarps * kOutStage : 0;
  // full[S], sf_full[S], sf[S], empty[S], acc_full, acc_empty, drain
  static constexpr int OFF_BAR = OFF_OUT + OUT_BYTES;
  static constexpr int OFF_MISC = OFF_BAR + (4 * STAGES + 3) * 8;
  static constexpr int SMEM = OFF_MISC + 16 + 1024;             // + alignment slack
  static_assert(SMEM <= 232448, "shared memory per block");
  // TMEM columns: accumulator [0, BN); per stage s, at BN + s * SF_STRIDE: A scales 16 columns (4 per MMA),
  // B scales BN / 8 columns (BN / 32 per MMA)
  static constexpr int SF_STRIDE = 16 + BN / 8;
  static constexpr int SFA_COL = BN;
  static constexpr int TMEM_COLS = (BN + STAGES * SF_STRIDE) <= 256 ? 256 : 512;
  static_assert(BN + STAGES * SF_STRIDE <= 512, "TMEM columns");
};

// shared -> global tensor-map store of one box, tracked by the issuing thread's bulk groups
SSB_DEVICE void tma_store_2d(const CUtensorMap* m, uint32_t src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
SSB_DEVICE void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// ---- CTA pairs (cluster of 2, cta_group::2) ----
SSB_DEVICE uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of this CTA's shared-memory location `a` in cluster CTA `rank`
SSB_DEVICE uint32_t map_to_rank(uint32_t a, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}
SSB_DEVICE void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
SSB_DEVICE bool mbar_try_wait_cl(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait on a barrier that the other CTA of the pair arrives on (cluster-scope acquire)
SSB_DEVICE bool mbar_wait_cl(uint32_t bar, uint32_t parity, volatile int32_t* abort_flag, int32_t* status) {
  if (mbar_try_wait_cl(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (mbar_try_wait_cl(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > kWaitNs) {
      *abort_flag = 1;
      raise_status(status, kErrTimeout);
      return false;
    }
  }
}
template <bool PAIR>
SSB_DEVICE void release_acc(uint32_t bar) {
  if constexpr (PAIR) mbar_arrive_remote(bar);
  else mbar_arrive(bar);
}
template <bool PAIR>
SSB_DEVICE bool wait_bar(uint32_t bar, uint32_t parity, volatile int32_t* abort_flag, int32_t* status) {
  if constexpr (PAIR) return mbar_wait_cl(bar, parity, abort_flag, status);
  else return mbar_wait(bar, parity, abort_flag, status);
}
// TMA tile load into this CTA's shared memory whose completion is counted on `bar` in either CTA of the pair (each
// CTA loads its own tiles)
SSB_DEVICE void tma_load_2d_pair(uint32_t dst, const CUtensorMap* m, int32_t x, int32_t y, uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}
// D (+)= A x B over both CTAs: A rows 0-127 and B rows 0-BN/2 from the leader's shared memory, the rest from the
// peer's at the same offsets; each CTA's TMEM holds its own 128 rows of D and their scales
SSB_DEVICE void tc_mma_nvf4_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate,
                                 uint32_t sfa_tmem, uint32_t sfb_tmem) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
SSB_DEVICE void tc_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
               : "memory");
}
SSB_DEVICE void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

SSB_DEVICE void tmem_st_x16(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

struct TileInfo {
  int group, row0, rows, nt;
};

SSB_DEVICE bool tile_info(const GemmArgs& a, int t, int n_tiles, TileInfo& ti) {
  const int mt = t / n_tiles;
  ti.nt = t - mt * n_tiles;
  if (a.mtiles == nullptr) {
    ti.group = 0;
    ti.row0 = mt * kBM;
    ti.rows = min(kBM, a.M - ti.row0);
  } else {
    const int4 e = reinterpret_cast<const int4*>(a.mtiles)[mt];
    ti.group = e.x;
    ti.row0 = e.y;
    ti.rows = e.z;
  }
  return ti.rows > 0;
}

SSB_DEVICE int total_tiles(const GemmArgs& a, int n_tiles) {
  int num_m;
  if (a.mtiles == nullptr) {
    num_m = (a.M + kBM - 1) / kBM;
  } else {
    num_m = min(*a.num_mtiles, a.mtile_cap);
  }
  return num_m * n_tiles;
}

// The CTA's t-th output tile. PAIR: t indexes pair tiles x N tiles, a pair tile being {group, first row, leader rows,
// peer rows} from `mpairs`, or (dense, no tables) row blocks 2 p and 2 p + 1; the leader (rank 0) takes rows
// [first, +128), the peer the next 128 (its rows may be 0 or fewer: it still feeds the MMA, and its epilogue stores
// nothing). Returns false for a tile to skip (no rows).
template <bool PAIR>
SSB_DEVICE bool step_tile(const GemmArgs& a, int t, int n_tiles, uint32_t rank, TileInfo& ti) {
  if constexpr (!PAIR) {
    return tile_info(a, t, n_tiles, ti);
  } else {
    const int mp = t / n_tiles;
    ti.nt = t - mp * n_tiles;
    if (a.mpairs == nullptr) {
      const int lead0 = 2 * mp * kBM;
      ti.group = 0;
      ti.row0 = lead0 + (rank != 0 ? kBM : 0);
      ti.rows = min(kBM, a.M - ti.row0);
      return a.M - lead0 > 0;
    }
    const int4 e = reinterpret_cast<const int4*>(a.mpairs)[mp];
    ti.group = e.x;
    ti.row0 = e.y + (rank != 0 ? kBM : 0);
    ti.rows = rank != 0 ? e.w : e.z;
    return e.z > 0;
  }
}

template <bool PAIR>
SSB_DEVICE int total_steps(const GemmArgs& a, int n_tiles) {
  if constexpr (!PAIR) return total_tiles(a, n_tiles);
  else if (a.mpairs == nullptr) return ((a.M + 2 * kBM - 1) / (2 * kBM)) * n_tiles;
  else return min(*a.num_mpairs, a.mpair_cap) * n_tiles;
}

// Bounded wait that ignores the abort flag: used only to drain copies / MMAs already in flight before exit.
SSB_DEVICE void drain_wait(uint32_t bar, uint32_t parity) {
  const unsigned long long t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > kWaitNs) break;
  }
}

template <int BN, int EPI, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_nvfp4_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmO, const GemmArgs args) {
  using C = Cfg<BN, EPI, PAIR>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_full = sbase + C::OFF_BAR;                 // operand tiles landed (TMA)
  const uint32_t bar_sf_full = bar_full + C::STAGES * 8;        // scale atoms landed (bulk copies)
  const uint32_t bar_sf = bar_sf_full + C::STAGES * 8;          // scales written to TMEM (4 writer warps)
  const uint32_t bar_empty = bar_sf + C::STAGES * 8;            // the stage's MMAs completed
  const uint32_t bar_acc_full = bar_empty + C::STAGES * 8;
  const uint32_t bar_acc_empty = bar_acc_full + 8;
  const uint32_t bar_drain = bar_acc_empty + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_MISC);
  volatile int32_t* abort_flag = reinterpret_cast<volatile int32_t*>(smem + C::OFF_MISC + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // PAIR: rank 0 (the leader) issues the MMAs of both CTAs and owns the full / sf / acc_empty barriers they use
  const uint32_t rank = PAIR ? cluster_rank() : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_sf_full + 8 * s, 1);
      mbar_init(bar_sf + 8 * s, PAIR ? 8 : 4);          // one arrive per scale-writer warp
      mbar_init(bar_empty + 8 * s, 1);
    }
    mbar_init(bar_acc_full, 1);
    mbar_init(bar_acc_empty, PAIR ? 2 * kEpiWarps : kEpiWarps);
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                   "r"(C::TMEM_COLS));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();               // both CTAs' barriers initialized before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int n_tiles = EPI == kEpiF32 ? (args.N + BN - 1) / BN : args.N / BN;
  const int num_kb = (args.K + 255) / 256;
  const int total = total_steps<PAIR>(args, n_tiles);
  const int first = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int stride = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int t = first; ok && t < total; t += stride) {
        TileInfo ti;
        if (!step_tile<PAIR>(args, t, n_tiles, rank, ti)) continue;
        const int brow0 = ti.group * args.N + ti.nt * BN;
        // a peer tile without rows reads the leader's scale rows (it may lie past the scale buffer's end)
        const int srow0 = ti.rows > 0 ? ti.row0 : ti.row0 - kBM;
        const uint8_t* sfa = args.sfa + (int64_t)(srow0 / kBM) * args.ncb_k * 512;
        const uint8_t* sfb = args.sfb + (int64_t)(brow0 / kBM) * args.ncb_k * 512;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!wait_bar<PAIR>(bar_empty + 8 * stage, phase ^ 1, abort_flag, args.status)) {
            ok = false;
            break;
          }
          const uint32_t sb = bar_sf_full + 8 * stage;
          mbar_arrive_expect_tx(sb, C::SF_TX);
          bulk_load(sbase + C::OFF_SFA + stage * C::SFA_BYTES, sfa + (int64_t)kb * 2048, 2048, sb);
#pragma unroll
          for (int j = 0; j < BN / 128; ++j)
            bulk_load(sbase + C::OFF_SFB + stage * C::SFB_BYTES + j * 2048,
                      sfb + ((int64_t)j * args.ncb_k + kb * 4) * 512, 2048, sb);
          const uint32_t fb = bar_full + 8 * stage;
          if constexpr (PAIR) {
            // both CTAs' operand bytes complete on the leader's full barrier, which the leader arms for both
            const uint32_t fbl = map_to_rank(fb, 0);
            if (rank == 0) mbar_arrive_expect_tx(fb, 2 * C::AB_TX);
            tma_load_2d_pair(sbase + C::OFF_A + stage * C::A_BYTES, &tmA, kb * kBKBytes, ti.row0, fbl);
            tma_load_2d_pair(sbase + C::OFF_B + stage * C::B_BYTES, &tmB, kb * kBKBytes,
                             brow0 + static_cast<int>(rank) * (BN / 2), fbl);
          } else {
            mbar_arrive_expect_tx(fb, C::AB_TX);
            tma_load_2d(sbase + C::OFF_A + stage * C::A_BYTES, &tmA, kb * kBKBytes, ti.row0, fb);
            tma_load_2d(sbase + C::OFF_B + stage * C::B_BYTES, &tmB, kb * kBKBytes, brow0, fb);
          }
          ++issued;
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // drain: the last min(issued, STAGES) loads may still be landing in shared memory
        int s = stage;
        uint32_t p = phase;
        for (int i = 0; i < min(issued, C::STAGES); ++i) {
          if (--s < 0) {
            s = C::STAGES - 1;
            p ^= 1;
          }
          drain_wait(bar_sf_full + 8 * s, p);
          if (rank == 0) drain_wait(bar_full + 8 * s, p);     // PAIR: counts the peer's bytes too
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------- MMA issuer (PAIR: the leader's, for both CTAs) ----------------
      constexpr uint32_t idesc = idesc_nvf4(PAIR ? 2 * kBM : kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t iter = 0;
      bool ok = true;
      bool any_mma = false;
      for (int t = first; ok && t < total; t += stride) {
        TileInfo ti;
        if (!step_tile<PAIR>(args, t, n_tiles, rank, ti)) continue;
        if (!wait_bar<PAIR>(bar_acc_empty, (iter & 1) ^ 1, abort_flag, args.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!wait_bar<PAIR>(bar_full + 8 * stage, phase, abort_flag, args.status) ||
              !wait_bar<PAIR>(bar_sf + 8 * stage, phase, abort_flag, args.status)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = sbase + C::OFF_A + stage * C::A_BYTES;
          const uint32_t sb = sbase + C::OFF_B + stage * C::B_BYTES;
          const uint32_t sfo = stage * C::SF_STRIDE;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint64_t ad = smem_desc(sa + i * 32, 0, 1024, 2);
            const uint64_t bd = smem_desc(sb + i * 32, 0, 1024, 2);
            if constexpr (PAIR)
              tc_mma_nvf4_pair(tmem, ad, bd, idesc, (kb | i) != 0 ? 1u : 0u, tmem + sfo + C::SFA_COL + 4 * i,
                               tmem + sfo + C::SFA_COL + 16 + (BN / 32) * i);
            else
              tc_mma_nvf4(tmem, ad, bd, idesc, (kb | i) != 0 ? 1u : 0u, tmem + sfo + C::SFA_COL + 4 * i,
                          tmem + sfo + C::SFA_COL + 16 + (BN / 32) * i);
          }
          any_mma = true;
          if constexpr (PAIR) {
            tc_commit_pair(map_to_rank(bar_empty + 8 * stage, 0));
            tc_commit_pair(map_to_rank(bar_empty + 8 * stage, 1));
          } else {
            tc_commit(bar_empty + 8 * stage);
          }
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if constexpr (PAIR) {
          tc_commit_pair(map_to_rank(bar_acc_full, 0));
          tc_commit_pair(map_to_rank(bar_acc_full, 1));
        } else {
          tc_commit(bar_acc_full);
        }
        ++iter;
      }
      if (!ok && any_mma) {
        if constexpr (PAIR) tc_commit_pair(map_to_rank(bar_drain, 0));
        else tc_commit(bar_drain);
        drain_wait(bar_drain, 0);
      }
    }
  } else if (warp == 2 || warp >= kEpiWarp0 + kEpiWarps) {
    // ---------------- scale writers (warps 2, 11, 12, 13: TMEM lane quarters 2, 3, 0, 1) ----------------
    // Per stage, TMEM columns [SFA_COL, +16): A scales, 4 columns per MMA, every column of a group holding the
    // quarter's own rows' word (the datapath of quarter q reads column q of the group); [SFA_COL + 16, + BN / 8): B
    // scales, BN / 32 columns per MMA, column c holding rows 32 c + lane of the B tile, the same in every quarter.
    // Source: the 128x4 atoms of the stage, whose 16-byte row l holds rows l, l + 32, l + 64, l + 96.
    const int q = warp & 3;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = first; ok && t < total; t += stride) {
      TileInfo ti;
      if (!step_tile<PAIR>(args, t, n_tiles, rank, ti)) continue;
      for (int kb = 0; kb < num_kb; ++kb) {
        // the stage's previous MMAs completed before its scale copies were issued, so its columns are free
        if (!mbar_wait(bar_sf_full + 8 * stage, phase, abort_flag, args.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint8_t* ssfa = smem + C::OFF_SFA + stage * C::SFA_BYTES + 16 * lane;
        const uint8_t* ssfb = smem + C::OFF_SFB + stage * C::SFB_BYTES + 16 * lane;
        uint32_t w[16 + BN / 8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 v = *reinterpret_cast<const uint4*>(ssfa + i * 512);
          const uint32_t a = q == 0 ? v.x : q == 1 ? v.y : q == 2 ? v.z : v.w;
          w[4 * i] = a;
          w[4 * i + 1] = a;
          w[4 * i + 2] = a;
          w[4 * i + 3] = a;
#pragma unroll
          for (int j = 0; j < BN / 128; ++j) {
            const uint4 b = *reinterpret_cast<const uint4*>(ssfb + j * 2048 + i * 512);
            w[16 + (BN / 32) * i + 4 * j] = b.x;
            w[16 + (BN / 32) * i + 4 * j + 1] = b.y;
            w[16 + (BN / 32) * i + 4 * j + 2] = b.z;
            w[16 + (BN / 32) * i + 4 * j + 3] = b.w;
          }
        }
        const uint32_t ta = tmem + (static_cast<uint32_t>(q * 32) << 16) + stage * C::SF_STRIDE + C::SFA_COL;
#pragma unroll
        for (int c = 0; c < (16 + BN / 8) / 16; ++c) tmem_st_x16(ta + 16 * c, w + 16 * c);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (PAIR) mbar_arrive_remote(map_to_rank(bar_sf + 8 * stage, 0));
          else mbar_arrive(bar_sf + 8 * stage);
        }
        if (++stage == C::STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else {
    // ---------------- epilogue (warps 3..10) ----------------
    const int quad = warp & 3;
    const int half = (warp - kEpiWarp0) >> 2;                      // which half of the tile's columns this warp owns
    const int rl = quad * 32 + lane;                       // row inside the tile = TMEM lane
    const uint32_t tq = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    uint32_t iter = 0;
    // PAIR: the accumulator is released on the leader's barrier
    const uint32_t acc_empty = PAIR ? map_to_rank(bar_acc_empty, 0) : bar_acc_empty;
    for (int t = first; t < total; t += stride) {
      TileInfo ti;
      if (!step_tile<PAIR>(args, t, n_tiles, rank, ti)) continue;
      if (!wait_bar<PAIR>(bar_acc_full, iter & 1, abort_flag, args.status)) break;
      tc_fence_after();
      const float alpha = args.alpha != nullptr ? args.alpha[ti.group] : args.alpha_scalar;
      const bool valid = rl < ti.rows;
      const int64_t row = (int64_t)ti.row0 + rl;
      if constexpr (EPI == kEpiSwiGLU) {
        // columns [64 half, +64) of the gate block and the same of the up block (tile columns 128 + ...)
        float g[64], u[64];
        tmem_ld_32x32b_x32(tq + 64 * half, *reinterpret_cast<float(*)[32]>(g));
        tmem_ld_32x32b_x32(tq + 64 * half + 32, *reinterpret_cast<float(*)[32]>(g + 32));
        tmem_ld_32x32b_x32(tq + 128 + 64 * half, *reinterpret_cast<float(*)[32]>(u));
        tmem_ld_32x32b_x32(tq + 128 + 64 * half + 32, *reinterpret_cast<float(*)[32]>(u + 32));
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) release_acc<PAIR>(acc_empty);
        uint8_t* codes = reinterpret_cast<uint8_t*>(args.out);
        uint32_t pk[8], sfw = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float h[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float gv = g[16 * q + i] * alpha;
            const float uv = u[16 * q + i] * alpha;
            h[i] = __fdividef(gv, 1.0f + __expf(-gv)) * uv;
          }
          uint32_t p2[2];
          sfw |= nvfp4_quant16(h, args.out_gs, p2) << (8 * q);
          pk[2 * q] = p2[0];
          pk[2 * q + 1] = p2[1];
        }
        if (valid) {
          const int col = ti.nt * 128 + 64 * half;          // first h column of this warp's share
          uint4* dst = reinterpret_cast<uint4*>(codes + row * args.ldo + col / 2);
          dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          *reinterpret_cast<uint32_t*>(args.out_sf + sf_atom_offset(row, col / 16, args.out_ncb)) = sfw;
        }
      } else if constexpr (EPI == kEpiBF16) {
        // columns [128 half, +128), 64 per tcgen05.ld round: to bf16 pairs, into this warp's staging buffer (row r's
        // 16-byte chunk c at chunk c ^ (r & 7), the 128-byte swizzle of the output map; conflict-free), then one TMA
        // store of the 32 x 64 box. Rows past the tile's valid rows are the group's padding rows (or past the map's
        // rows, where the store is clipped).
        const uint32_t stg = sbase + C::OFF_OUT + (warp - kEpiWarp0) * kOutStage;
        const int y0 = ti.row0 + quad * 32;
        const int x0 = ti.nt * BN + 128 * half;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float v[64];
          tmem_ld_32x32b_x32(tq + 128 * half + 64 * h, *reinterpret_cast<float(*)[32]>(v));
          tmem_ld_32x32b_x32(tq + 128 * half + 64 * h + 32, *reinterpret_cast<float(*)[32]>(v + 32));
          tmem_ld_wait();
          if (h == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) release_acc<PAIR>(acc_empty);
          }
          uint32_t pk[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            __nv_bfloat162 b2 = __floats2bfloat162_rn(v[2 * j] * alpha, v[2 * j + 1] * alpha);
            pk[j] = *reinterpret_cast<uint32_t*>(&b2);
          }
          if (lane == 0) bulk_wait_read0();             // the previous store has read the buffer
          __syncwarp();
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint32_t a = stg + lane * 128 + ((c ^ (lane & 7)) << 4);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(pk[4 * c]), "r"(pk[4 * c + 1]),
                         "r"(pk[4 * c + 2]), "r"(pk[4 * c + 3])
                         : "memory");
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && ti.rows > 0) {                // a PAIR peer tile without rows stores nothing
            tma_store_2d(&tmO, stg, x0 + 64 * h, y0);
            bulk_commit();
          }
        }
      } else {
        // columns [64 half, +64) of a 128-wide tile
        float v[64];
        tmem_ld_32x32b_x32(tq + 64 * half, *reinterpret_cast<float(*)[32]>(v));
        tmem_ld_32x32b_x32(tq + 64 * half + 32, *reinterpret_cast<float(*)[32]>(v + 32));
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) release_acc<PAIR>(acc_empty);
        if (valid) {
          float* out = reinterpret_cast<float*>(args.out);
          const int col0 = ti.nt * BN + 64 * half;
          if (col0 + 64 <= args.N) {
            float4* dst = reinterpret_cast<float4*>(out + row * args.ldo + col0);
#pragma unroll
            for (int i = 0; i < 16; ++i)
              dst[i] = make_float4(v[4 * i] * alpha, v[4 * i + 1] * alpha, v[4 * i + 2] * alpha, v[4 * i + 3] * alpha);
          } else {
#pragma unroll
            for (int i = 0; i < 64; ++i)
              if (col0 + i < args.N) out[row * args.ldo + col0 + i] = v[i] * alpha;
          }
        }
      }
      ++iter;
    }
    if constexpr (EPI == kEpiBF16) {
      if (lane == 0) bulk_wait0();                     // the output stores completed before the CTA exits
    }
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync_all();              // no CTA leaves while its peer may still signal it
  tc_fence_after();
  if (warp == 1) {
    if constexpr (PAIR)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS));
    else
      tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ---- host side ------------------------------------------------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2D uint8 map over [rows, width bytes] with row pitch `ld` bytes; box = 128 bytes x box_rows, 128-byte swizzle.
int make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t width, int64_t ld, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return kErrNoDriver;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld & 15) || width <= 0 || rows <= 0) return kErrArgs;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBKBytes), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kErrArgs;
}

template <int BN, int EPI, bool PAIR>
int launch(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mo, const GemmArgs& args, int grid,
           cudaStream_t stream) {
  using Cf = Cfg<BN, EPI, PAIR>;
  auto kern = gemm_nvfp4_kernel<BN, EPI, PAIR>;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::SMEM) != cudaSuccess)
      return kErrCuda;
    attr_set = true;
  }
  if constexpr (PAIR) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid & ~1);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = Cf::SMEM;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, ma, mb, mo, args) != cudaSuccess) return kErrCuda;
  } else {
    kern<<<grid, kThreads, Cf::SMEM, stream>>>(ma, mb, mo, args);
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace

int make_map_2d_swizzled(CUtensorMap* m, const void* base, int64_t rows, int64_t width, int64_t ld_bytes,
                         int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return kErrNoDriver;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld_bytes & 15) || width <= 0 || rows <= 0) return kErrArgs;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld_bytes)};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kErrArgs;
}

int make_map_2d_ex(CUtensorMap* m, int dtype, const void* base, int64_t rows, int64_t width, int64_t ld_bytes,
                   int box_cols, int box_rows, int swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return kErrNoDriver;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld_bytes & 15) || width <= 0 || rows <= 0) return kErrArgs;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, static_cast<CUtensorMapDataType>(dtype), 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, static_cast<CUtensorMapSwizzle>(swizzle),
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kErrArgs;
}

int make_map_2d(CUtensorMap* m, int dtype, const void* base, int64_t rows, int64_t width, int64_t ld_bytes,
                int box_cols, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return kErrNoDriver;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld_bytes & 15) || width <= 0 || rows <= 0) return kErrArgs;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, static_cast<CUtensorMapDataType>(dtype), 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kErrArgs;
}

int device_sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

int launch_gemm_nvfp4(int epilogue, const uint8_t* a, int64_t a_rows, int64_t lda, const uint8_t* b, int64_t b_rows,
                      int64_t ldb, const GemmArgs& args, int num_sms, cudaStream_t stream) {
  if (args.K <= 0 || args.K % 64 != 0 || args.N <= 0) return kErrArgs;
  if (args.ncb_k != sf_atom_cols(args.K)) return kErrArgs;
  if ((reinterpret_cast<uintptr_t>(args.sfa) & 15) || (reinterpret_cast<uintptr_t>(args.sfb) & 15)) return kErrArgs;
  const int BN = epilogue == kEpiF32 ? 128 : 256;
  if (epilogue != kEpiF32 && args.N % BN != 0) return kErrArgs;
  if (epilogue == kEpiSwiGLU && (args.ldo % 16 != 0 || args.out_ncb != sf_atom_cols(args.N / 2))) return kErrArgs;
  if (epilogue == kEpiBF16 && args.ldo % 8 != 0) return kErrArgs;
  if (args.mtiles == nullptr && args.M <= 0) return kOk;
  // CTA pairs: the grouped 256-wide epilogues when the caller gives a pair table; dense bf16 GEMMs of more than one
  // row block (their 3-stage single-CTA ring leaves the MMAs waiting for operands)
  const bool pair = num_sms >= 2 && ((args.mpairs != nullptr && epilogue != kEpiF32) ||
                                     (args.mtiles == nullptr && epilogue == kEpiBF16 && args.M > kBM));
  if (args.mpairs != nullptr && (args.num_mpairs == nullptr || args.mpair_cap <= 0)) return kErrArgs;
  CUtensorMap ma, mb;
  int rc = make_map(&ma, a, a_rows, args.K / 2, lda, kBM);
  if (rc != kOk) return rc;
  rc = make_map(&mb, b, b_rows, args.K / 2, ldb, pair ? BN / 2 : BN);
  if (rc != kOk) return rc;
  int grid = num_sms;
  if (args.mtiles == nullptr) {
    const int n_tiles = (args.N + BN - 1) / BN;
    const int m_units = pair ? 2 * ((args.M + 2 * kBM - 1) / (2 * kBM)) : (args.M + kBM - 1) / kBM;
    const int tiles = m_units * n_tiles;
    grid = tiles < num_sms ? tiles : num_sms;
  }
  switch (epilogue) {
    case kEpiF32:
      return launch<128, kEpiF32, false>(ma, mb, ma, args, grid, stream);
    case kEpiBF16: {
      // output map: [a_rows, N] bf16 rows of pitch ldo, box 64 columns x 32 rows, 128-byte swizzle
      CUtensorMap mo;
      rc = make_map_2d_swizzled(&mo, args.out, a_rows, args.N, args.ldo * 2, 32);
      if (rc != kOk) return rc;
      return pair ? launch<256, kEpiBF16, true>(ma, mb, mo, args, grid, stream)
                  : launch<256, kEpiBF16, false>(ma, mb, mo, args, grid, stream);
    }
    case kEpiSwiGLU:
      return pair ? launch<256, kEpiSwiGLU, true>(ma, mb, ma, args, grid, stream)
                  : launch<256, kEpiSwiGLU, false>(ma, mb, ma, args, grid, stream);
    default:
      return kErrArgs;
  }
}

}  // namespace ssb
