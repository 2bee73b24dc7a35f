// Tensor-core (tcgen05) backward score kernel with staggered token tiles, D <= 64, 2-SM.
//
// The same work as bwd_scores_kernel (tc_bwd.cu) -- per 256-row vocabulary tile of the chunk
// and 128-token tile: S^T = W h^T (recompute), dP^T = E dO^T, P, dS = P (dP - delta), db,
// dE += P^T dO, dS^T * s stored for the GEMMs -- with the S recompute fed at the gemm
// kernel's bytes per MMA cycle.  Two token tiles of a unit are in flight at every stage and
// read the same W K-block: tile i of a unit owns the unit's stages [i H, i H + KB)
// (H = ceil(KB / 2), KB 128-wide K-blocks per tile) and reads K-block (stage mod KB) there, so
// its K loop starts half a loop after tile i-1's and wraps around.  A stage holds one W
// K-block (32 KB per CTA) and the two tiles' h K-blocks (16 KB each): 64 KB per 1024 MMA
// cycles, against 56 KB per 768 cycles for single 192-token tiles; the MMA thread waits on
// one barrier per 16 MMAs.  Only a unit's first and last H stages carry one tile.
//
// Tensor memory (512 columns per CTA): three S^T regions of 128 columns (global tile g in
// region g mod 3), dP^T (64 columns) and dE (64).  When a tile's last stage has been issued,
// its S region is committed to the gradient warps and the tile's two 64-token dP^T chunks,
// its gradient pass and its dE follow while the next tiles stream: the MMA thread issues
// them between stages as soon as non-blocking barrier tests pass, and blocks for them only
// before a region is reused (tile g + 3 starts), oldest tile first (a tile's dE before the
// next tile's dP: the gO / E producer loads a tile's K-major gO and E only after the previous
// tile's MN-major gO, whose buffer that dE frees).  P overwrites the S columns the gradient
// pass has read, 16 packed columns per 32, and is the A operand of dE from tensor memory.
//
// Warp roles: warp 0 loads W and h (both CTAs), warp 2 loads E, the K-major gO of each
// tile (dP^T operand) and its MN-major gO (dE operand) (both CTAs), warp 1 (one thread of the
// even CTA) issues every MMA, warps 4-7 run the gradient pass (one thread per vocabulary
// row).  All MMAs are tcgen05.mma.cta_group::2; each CTA's TMA loads complete on the leader's
// barrier; commits multicast to both CTAs.  Every wait is bounded (error word, clean exit).
// The K order of a tile's S accumulation starts at K-block (i H mod KB), so S (and, rarely,
// a rounded dS) can differ in the last bits from a kernel that starts every tile at K-block 0.
//
// Replaces the reference's per-chunk recompute GEMM + Triton _bwd_chunk_kernel
// (swvr/chunked.py:120-131, swvr/triton_kernels.py:76-118) for D <= 64.
#include "ptx.cuh"
#include "tc.cuh"

namespace swvr {
namespace tc {

template <int NS>
struct StaggerCfg {
  static constexpr int BN = 128;                        // tokens per tile (64 staged per CTA)
  static constexpr int DPC = 64;                        // tokens per dP^T chunk
  static constexpr int NCH = BN / DPC;                  // dP^T chunks per tile
  static constexpr int WBOX = 128 * 128;                // 128 W rows x 64 K (16-bit)
  static constexpr int HBOX = (BN / 2) * 128;           // this CTA's 64 h rows x 64 K
  static constexpr int W_BYTES = 2 * WBOX;              // one 128-wide K-block of W
  static constexpr int H_BYTES = 2 * HBOX;              // one 128-wide K-block of a tile's h
  static constexpr int STAGE = W_BYTES + 2 * H_BYTES;   // W + the h slots of two tiles
  static constexpr int E_BYTES = WBOX;                  // this CTA's 128 E rows x 64
  static constexpr int GOK_CBOX = (DPC / 2) * 128;      // a chunk's 32 tokens (this CTA) x 64, K-major
  static constexpr int GOK_BYTES = NCH * GOK_CBOX;
  static constexpr int GOM_ROW = 64;                    // 32 embedding columns (this CTA's half of N)
  static constexpr int GOM_BYTES = BN * GOM_ROW;        // all BN tokens, MN-major, 64-byte swizzle
  static constexpr int SMEM_STAGE = 0;
  static constexpr int SMEM_E = SMEM_STAGE + NS * STAGE;
  static constexpr int SMEM_GOK = SMEM_E + E_BYTES;
  static constexpr int SMEM_GOM = SMEM_GOK + GOK_BYTES;
  static constexpr int SMEM_LSE = SMEM_GOM + GOM_BYTES;
  static constexpr int SMEM_DELTA = SMEM_LSE + BN * 4;
  static constexpr int SMEM_BAR = SMEM_DELTA + BN * 4;
  static constexpr int NBAR = 2 * NS + 17;
  static constexpr int SMEM_TOTAL = SMEM_BAR + NBAR * 8 + 16;
  static constexpr int SMEM_ALLOC = SMEM_TOTAL + 1024;
  static constexpr uint32_t DP_COL = 3 * BN, DE_COL = DP_COL + DPC;
  static_assert(DE_COL + 64 <= 512, "TMEM budget");
  static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
  static_assert(STAGE % 1024 == 0 && HBOX % 1024 == 0 && GOK_CBOX % 1024 == 0 && GOM_BYTES % 1024 == 0,
                "1024-byte alignment");
};

// Per-tile bookkeeping of the MMA thread for the (at most three) tiles with deferred work.
struct StaggerTile {
  uint32_t unit;  // the pair's unit counter
  bool first, last;
};

template <bool kBF16, int NS>
__global__ void __launch_bounds__(256, 1)
    bwd_scores_stagger_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_h,
                              const __grid_constant__ CUtensorMap tm_e, const __grid_constant__ CUtensorMap tm_gok,
                              const __grid_constant__ CUtensorMap tm_gom, const BwdScoresParams p) {
  using Cfg = StaggerCfg<NS>;
  constexpr int BN = Cfg::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::SMEM_BAR);
  uint64_t* full = bars;               // [NS] leader: both CTAs' bytes
  uint64_t* empty = bars + NS;         // [NS] both (multicast commit)
  uint64_t* s_full = bars + 2 * NS;    // [3] both: one phase per use of an S region
  uint64_t* p_ready = s_full + 3;      // [3] leader: one arrival per CTA per use
  uint64_t* dp_full = p_ready + 3;     // both: one phase per dP chunk
  uint64_t* dp_free = dp_full + 1;     // leader: one arrival per CTA per dP chunk
  uint64_t* e_full = dp_free + 1;      // leader: both CTAs' bytes, one phase per unit
  uint64_t* e_empty = e_full + 1;      // both
  uint64_t* gok_full = e_empty + 1;    // leader: one phase per tile
  uint64_t* gok_empty = gok_full + 1;  // both
  uint64_t* gom_full = gok_empty + 1;  // leader: one phase per tile
  uint64_t* gom_empty = gom_full + 1;  // both
  uint64_t* de_full = gom_empty + 1;   // both: one phase per unit
  uint64_t* de_free = de_full + 1;     // leader: one arrival per CTA per unit
  uint64_t* spare = de_free + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + Cfg::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* lse_s = reinterpret_cast<float*>(smem + Cfg::SMEM_LSE);
  float* delta_s = reinterpret_cast<float*>(smem + Cfg::SMEM_DELTA);

  const bool need_ds = p.ds != nullptr, need_de = p.part_de != nullptr, need_db = p.part_db != nullptr;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int r = 0; r < 3; ++r) {
      mbar_init(&s_full[r], 1);
      mbar_init(&p_ready[r], 2);
    }
    mbar_init(dp_full, 1);
    mbar_init(dp_free, 2);
    mbar_init(e_full, 1);
    mbar_init(e_empty, 1);
    mbar_init(gok_full, 1);
    mbar_init(gok_empty, 1);
    mbar_init(gom_full, 1);
    mbar_init(gom_empty, 1);
    mbar_init(de_full, 1);
    mbar_init(de_free, 2);
    mbar_init(spare, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_h);
    tma_prefetch_desc(&tm_e);
    tma_prefetch_desc(&tm_gok);
    tma_prefetch_desc(&tm_gom);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  if (threadIdx.x == 0) pdl_trigger();
  const int KB = (p.K + 127) / 128;  // 128-wide K-blocks per tile
  const int H = (KB + 1) / 2;        // stage offset between consecutive tiles of a unit

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ W / h producer (both CTAs)
      uint32_t stage = 0, sphase = 0;
      for (int u = pair; u < p.units; u += npairs) {
        const int vt = u / p.TS, ts = u % p.TS;
        const int it0 = ts * p.per_t, n = min(it0 + p.per_t, p.NT) - it0;
        if (n <= 0) continue;
        const int vrow0 = p.v_begin + vt * 256 + static_cast<int>(rank) * 128;
        const int S = (n - 1) * H + KB;
        for (int s = 0; s < S; ++s) {
          const int kw = s % KB, i1 = s / H, i0 = i1 - 1;
          const bool a1 = i1 < n;
          const bool a0 = i0 >= 0 && i0 < n && s < i0 * H + KB;
          if (!mbar_wait(&empty[stage], sphase ^ 1u, abort_flag, kErrBwdScores | 2)) goto done;
          if (leader)
            mbar_arrive_expect_tx(&full[stage], 2 * (Cfg::W_BYTES + (int(a0) + int(a1)) * Cfg::H_BYTES));
          const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
          uint8_t* sb = smem + Cfg::SMEM_STAGE + stage * Cfg::STAGE;
#pragma unroll
          for (int hk = 0; hk < 2; ++hk) {
            const int k0 = (kw * 2 + hk) * 64;  // past K the boxes read zero fill
            tma_load_2d_pair(sb + hk * Cfg::WBOX, &tm_w, fb, k0, vrow0);
            if (a0)
              tma_load_2d_pair(sb + Cfg::W_BYTES + (i0 & 1) * Cfg::H_BYTES + hk * Cfg::HBOX, &tm_h, fb, k0,
                               (it0 + i0) * BN + static_cast<int>(rank) * (BN / 2));
            if (a1)
              tma_load_2d_pair(sb + Cfg::W_BYTES + (i1 & 1) * Cfg::H_BYTES + hk * Cfg::HBOX, &tm_h, fb, k0,
                               (it0 + i1) * BN + static_cast<int>(rank) * (BN / 2));
          }
          if (++stage == NS) {
            stage = 0;
            sphase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 2) {
    if (lane == 0) {
      // ------------------------------------------------------------ gO / E producer (both CTAs)
      // Per tile, in the MMA thread's order: the unit's E (first tile), the tile's K-major gO
      // (after the previous tile's dP chunks) and MN-major gO (after the previous tile's dE).
      uint32_t g = 0, uc = 0;
      for (int u = pair; u < p.units; u += npairs) {
        const int vt = u / p.TS, ts = u % p.TS;
        const int it0 = ts * p.per_t, it1 = min(it0 + p.per_t, p.NT);
        if (it1 <= it0) continue;
        const int vrow0 = p.v_begin + vt * 256 + static_cast<int>(rank) * 128;
        for (int it = it0; it < it1; ++it, ++g) {
          if (it == it0) {
            if (!mbar_wait(e_empty, (uc & 1u) ^ 1u, abort_flag, kErrBwdScores | 1)) goto done;
            if (leader) mbar_arrive_expect_tx(e_full, 2 * Cfg::E_BYTES);
            tma_load_2d_pair(smem + Cfg::SMEM_E, &tm_e, mapa_shared(smem_u32(e_full), 0), 0, vrow0);
          }
          if (!mbar_wait(gok_empty, (g & 1u) ^ 1u, abort_flag, kErrBwdScores | 3)) goto done;
          if (leader) mbar_arrive_expect_tx(gok_full, 2 * Cfg::GOK_BYTES);
#pragma unroll
          for (int jj = 0; jj < Cfg::NCH; ++jj)
            tma_load_2d_pair(smem + Cfg::SMEM_GOK + jj * Cfg::GOK_CBOX, &tm_gok, mapa_shared(smem_u32(gok_full), 0), 0,
                             it * BN + jj * Cfg::DPC + static_cast<int>(rank) * (Cfg::DPC / 2));
          if (!mbar_wait(gom_empty, (g & 1u) ^ 1u, abort_flag, kErrBwdScores | 4)) goto done;
          if (leader) mbar_arrive_expect_tx(gom_full, 2 * Cfg::GOM_BYTES);
          tma_load_2d_pair(smem + Cfg::SMEM_GOM, &tm_gom, mapa_shared(smem_u32(gom_full), 0),
                           static_cast<int>(rank) * 32, it * BN);
        }
        ++uc;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------------------ MMA issuer (leader only)
      const uint32_t idS = idesc_f16(kBF16, 256, BN, false, false);
      const uint32_t idDP = idesc_f16(kBF16, 256, Cfg::DPC, false, false);
      const uint32_t idDE = idesc_f16(kBF16, 256, 64, false, true);
      const uint32_t ebase = smem_u32(smem + Cfg::SMEM_E);
      const uint32_t gokbase = smem_u32(smem + Cfg::SMEM_GOK);
      const uint32_t gombase = smem_u32(smem + Cfg::SMEM_GOM);
      // stage-0 descriptors of W and of h slot 0; a stage / slot / K half / 16-wide K step adds
      // (byte offset >> 4)
      const uint64_t dw0 = sdesc_sw128(smem_u32(smem + Cfg::SMEM_STAGE), 16, 1024);
      const uint64_t dh0 = sdesc_sw128(smem_u32(smem + Cfg::SMEM_STAGE + Cfg::W_BYTES), 16, 1024);
      uint32_t stage = 0, sphase = 0;
      uint32_t q = 0;                                // dP chunks issued
      uint32_t completed = 0;                        // tiles whose S has been committed
      uint32_t dp_tile = 0, dp_jj = 0, de_tile = 0;  // next deferred dP chunk / dE
      StaggerTile meta[4];                           // tiles g with completed - 4 < g, by g & 3

      // The oldest deferred dP chunk: 1 issued, 0 a test failed (non-blocking), -1 abort.
      auto try_dp = [&](bool block) -> int {
        const uint32_t gt = dp_tile;
        if (q > 0) {
          if (block) {
            if (!mbar_wait(dp_free, (q - 1u) & 1u, abort_flag, kErrBwdScores | 6)) return -1;
          } else if (!mbar_test(dp_free, (q - 1u) & 1u)) {
            return 0;
          }
        }
        const StaggerTile& m = meta[gt & 3u];
        if (dp_jj == 0) {
          if (block) {
            if (!mbar_wait(e_full, m.unit & 1u, abort_flag, kErrBwdScores | 6)) return -1;
            if (!mbar_wait(gok_full, gt & 1u, abort_flag, kErrBwdScores | 7)) return -1;
          } else if (!mbar_test(e_full, m.unit & 1u) || !mbar_test(gok_full, gt & 1u)) {
            return 0;
          }
        }
        tc_fence_after();
        const uint32_t gk = gokbase + dp_jj * Cfg::GOK_CBOX;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          umma2_ss(tmem + Cfg::DP_COL, sdesc_sw128(ebase + ks * 32, 16, 1024), sdesc_sw128(gk + ks * 32, 16, 1024),
                   idDP, ks ? 1u : 0u);
        if (dp_jj == Cfg::NCH - 1) {
          umma2_commit_mc(gok_empty, 3);
          if (m.last) umma2_commit_mc(e_empty, 3);
        }
        umma2_commit_mc(dp_full, 3);
        ++q;
        if (++dp_jj == Cfg::NCH) {
          dp_jj = 0;
          ++dp_tile;
        }
        return 1;
      };
      // The oldest deferred dE (its tile's dP chunks all issued).
      auto try_de = [&](bool block) -> int {
        const uint32_t gt = de_tile, rg = gt % 3u;
        const StaggerTile& m = meta[gt & 3u];
        const bool wait_free = need_de && m.first && m.unit > 0;
        if (block) {
          if (!mbar_wait(&p_ready[rg], (gt / 3u) & 1u, abort_flag, kErrBwdScores | 8)) return -1;
          if (!mbar_wait(gom_full, gt & 1u, abort_flag, kErrBwdScores | 9)) return -1;
          if (wait_free && !mbar_wait(de_free, (m.unit - 1u) & 1u, abort_flag, kErrBwdScores | 9)) return -1;
        } else if (!mbar_test(&p_ready[rg], (gt / 3u) & 1u) || !mbar_test(gom_full, gt & 1u) ||
                   (wait_free && !mbar_test(de_free, (m.unit - 1u) & 1u))) {
          return 0;
        }
        if (need_de) {
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < BN / 16; ++ks)
            umma2_ts(tmem + Cfg::DE_COL, tmem + rg * BN + ks * 8, sdesc_sw64(gombase + ks * 16 * 64, Cfg::GOM_BYTES, 512),
                     idDE, (m.first && ks == 0) ? 0u : 1u);
        }
        umma2_commit_mc(gom_empty, 3);
        if (need_de && m.last) umma2_commit_mc(de_full, 3);
        ++de_tile;
        return 1;
      };
      // Blocking: every deferred dP chunk and dE of tiles up to gt, oldest tile first.
      auto flush_through = [&](uint32_t gt) -> bool {
        while (de_tile <= gt && de_tile < completed) {
          const int r = de_tile < dp_tile ? try_de(true) : try_dp(true);
          if (r < 0) return false;
        }
        return true;
      };
      // Non-blocking: deferred work whose barriers have already completed, in order.
      auto side_work = [&]() -> bool {
        while (dp_tile < completed) {
          const int r = try_dp(false);
          if (r < 0) return false;
          if (r == 0) break;
        }
        while (de_tile < dp_tile) {
          const int r = try_de(false);
          if (r < 0) return false;
          if (r == 0) break;
        }
        return true;
      };

      uint32_t g0 = 0, uc = 0;  // global index of the unit's first tile; unit counter
      for (int u = pair; u < p.units; u += npairs) {
        const int ts = u % p.TS;
        const int it0 = ts * p.per_t, n = min(it0 + p.per_t, p.NT) - it0;
        if (n <= 0) continue;
        const int S = (n - 1) * H + KB;
        for (int s = 0; s < S; ++s) {
          const int i1 = s / H, i0 = i1 - 1;
          const bool a1 = i1 < n;
          const bool a0 = i0 >= 0 && i0 < n && s < i0 * H + KB;
          if (a1 && s == i1 * H) {
            // tile g starts: its region's previous tile (g - 3) must be finished
            const uint32_t g = g0 + i1;
            if (g >= 3 && !flush_through(g - 3)) goto done;
            meta[g & 3u] = StaggerTile{uc, i1 == 0, i1 == n - 1};  // tile g - 4's entry is no longer read
          }
          if (!mbar_wait(&full[stage], sphase, abort_flag, kErrBwdScores | 5)) goto done;
          const uint64_t so = static_cast<uint64_t>(stage * (Cfg::STAGE >> 4));
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const bool act = t == 0 ? a0 : a1;
            if (!act) continue;
            const int i = t == 0 ? i0 : i1;
            const uint32_t dcol = tmem + ((g0 + static_cast<uint32_t>(i)) % 3u) * BN;
            const uint64_t hs = so + static_cast<uint64_t>((i & 1) * (Cfg::H_BYTES >> 4));
            const bool first = s == i * H;
#pragma unroll
            for (int k8 = 0; k8 < 8; ++k8)
              umma2_ss(dcol, dw0 + so + (k8 >> 2) * (Cfg::WBOX >> 4) + (k8 & 3) * 2,
                       dh0 + hs + (k8 >> 2) * (Cfg::HBOX >> 4) + (k8 & 3) * 2, idS, (first && k8 == 0) ? 0u : 1u);
          }
          umma2_commit_mc(&empty[stage], 3);
          if (a0 && s == i0 * H + KB - 1) {
            umma2_commit_mc(&s_full[(g0 + i0) % 3u], 3);
            ++completed;
          }
          if (a1 && s == i1 * H + KB - 1) {
            umma2_commit_mc(&s_full[(g0 + i1) % 3u], 3);
            ++completed;
          }
          if (++stage == NS) {
            stage = 0;
            sphase ^= 1u;
          }
          if (!side_work()) goto done;
        }
        g0 += n;
        ++uc;
      }
      if (g0 > 0 && !flush_through(g0 - 1)) goto done;
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------------- gradient warps (both CTAs)
    // lse_s holds -LSE*log2e and delta_s holds -delta for the current token tile; each thread
    // stores its row of dS*s (128 tokens, contiguous) with 16-byte stores, one dP chunk at a
    // time, and writes P over the S columns it has read.
    const int r = threadIdx.x - 128;
    const uint32_t trow = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const float2 sc2v = make_float2(p.sc2, p.sc2), scalev = make_float2(p.scale, p.scale);
    const uint32_t p_ready_leader = mapa_shared(smem_u32(p_ready), 0);
    const uint32_t dp_free_leader = mapa_shared(smem_u32(dp_free), 0);
    const uint32_t de_free_leader = mapa_shared(smem_u32(de_free), 0);
    // The loads and MMAs above read inputs only; the dS buffer and the partial slots written
    // here are still read by the previous chunk's kernels until they complete.
    pdl_wait();
    uint32_t g = 0, uc = 0, q = 0;
    for (int u = pair; u < p.units; u += npairs) {
      const int vt = u / p.TS, ts = u % p.TS;
      const int it0 = ts * p.per_t, it1 = min(it0 + p.per_t, p.NT);
      if (it1 <= it0) continue;
      const int local_row0 = vt * 256 + static_cast<int>(rank) * 128;  // within the chunk
      const int vrow = p.v_begin + local_row0 + r;
      const bool vvalid = vrow < p.v_end;
      const float b2 = (p.bias != nullptr && vvalid) ? load_f(p.bias, p.bias_dt, vrow) * kLog2e : 0.f;
      const float2 b2v = make_float2(b2, b2);
      float2 db = make_float2(0.f, 0.f);
      for (int it = it0; it < it1; ++it, ++g) {
        const int t0 = it * BN;
        named_bar_sync(1, 128);
        {
          const int t = t0 + r;  // 128 threads, 128 tokens
          lse_s[r] = t < p.N ? -p.lse[t] * kLog2e : -INFINITY;
          delta_s[r] = t < p.N ? -p.delta[t] : 0.f;
        }
        named_bar_sync(1, 128);
        const uint32_t rg = g % 3u;
        if (!warp_wait(&s_full[rg], (g / 3u) & 1u, abort_flag, kErrBwdScores | 10)) goto done;
        const uint32_t sbase = trow + rg * BN;
#pragma unroll 1
        for (int jj = 0; jj < Cfg::NCH; ++jj, ++q) {
          if (!warp_wait(dp_full, q & 1u, abort_flag, kErrBwdScores | 11)) goto done;
          tc_fence_after();
#pragma unroll 1
          for (int c2 = 0; c2 < Cfg::DPC / 32; ++c2) {
            const int c = jj * (Cfg::DPC / 32) + c2;  // 32-token column block of the tile
            uint32_t s[32], dp[32];
            tmem_ld32(sbase + c * 32, s);
            tmem_ld32(trow + Cfg::DP_COL + c2 * 32, dp);
            tmem_wait_ld();
            uint32_t pk_p[16], pk_ds[16];
            const float4* L4 = reinterpret_cast<const float4*>(lse_s + c * 32);
            const float4* D4 = reinterpret_cast<const float4*>(delta_s + c * 32);
#pragma unroll
            for (int qq = 0; qq < 8; ++qq) {
              const float4 nl = L4[qq], nd = D4[qq];
#pragma unroll
              for (int hh = 0; hh < 2; ++hh) {
                const int i = 4 * qq + 2 * hh;
                const float2 sv = make_float2(__uint_as_float(s[i]), __uint_as_float(s[i + 1]));
                const float2 dpv = make_float2(__uint_as_float(dp[i]), __uint_as_float(dp[i + 1]));
                const float2 bl = fadd2(b2v, hh ? make_float2(nl.z, nl.w) : make_float2(nl.x, nl.y));
                const float2 x = ffma2(sv, sc2v, bl);
                const float2 pv = make_float2(ex2(x.x), ex2(x.y));
                const float2 d = fmul2(pv, fadd2(dpv, hh ? make_float2(nd.z, nd.w) : make_float2(nd.x, nd.y)));
                db = fadd2(db, d);
                const float2 dsv = fmul2(d, scalev);
                pk_ds[i / 2] = pack2<kBF16>(dsv.x, dsv.y);
                pk_p[i / 2] = pack2<kBF16>(pv.x, pv.y);
              }
            }
            if (need_ds && vvalid) {
              // 64 contiguous bytes of row r: tokens [t0 + 32c, t0 + 32c + 32)
              uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.ds) +
                                                    static_cast<int64_t>(local_row0 + r) * p.ld_ds + t0 + c * 32);
#pragma unroll
              for (int k = 0; k < 4; ++k)
                dst[k] = make_uint4(pk_ds[4 * k], pk_ds[4 * k + 1], pk_ds[4 * k + 2], pk_ds[4 * k + 3]);
            }
            // P overwrites S columns that have been read: block c's 16 packed columns start at 16c
            if (need_de) tmem_st16(sbase + c * 16, pk_p);
          }
          const bool last = jj == Cfg::NCH - 1;
          if (last && need_de) tmem_wait_st();
          tc_fence_before();
          named_bar_sync(1, 128);
          if (r == 0) {
            mbar_arrive_cluster_relaxed(dp_free_leader);
            if (last) mbar_arrive_cluster_relaxed(p_ready_leader + rg * 8);
          }
        }
      }
      const int64_t slot = static_cast<int64_t>(u) * 256 + static_cast<int>(rank) * 128 + r;
      if (need_de) {
        if (!warp_wait(de_full, uc & 1u, abort_flag, kErrBwdScores | 12)) goto done;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t o[32];
          tmem_ld32(trow + Cfg::DE_COL + c * 32, o);
          tmem_wait_ld();
          if (vvalid) store_row32(p.part_de + slot * p.D, c * 32, p.D, o);
        }
        tc_fence_before();
        named_bar_sync(1, 128);
        if (r == 0) mbar_arrive_cluster_relaxed(de_free_leader);
      }
      if (need_db && vvalid) p.part_db[slot] = db.x + db.y;
      ++uc;
    }
  }
done:
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) drain_after_abort_pair(warp == 1 && lane == 0 && leader, spare);
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

template <bool kBF16, int NS>
static cudaError_t launch_stagger(const BwdScoresMaps& m, const BwdScoresParams& prm, int max_pairs, bool pdl,
                                  cudaStream_t st) {
  using Cfg = StaggerCfg<NS>;
  auto kern = bwd_scores_stagger_kernel<kBF16, NS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_ALLOC);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.blockDim = dim3(256, 1, 1);
  cfg.dynamicSmemBytes = Cfg::SMEM_ALLOC;
  cfg.stream = st;
  cfg.gridDim = dim3(2 * 74, 1, 1);
  int clusters = 0;
  e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
  if (e != cudaSuccess) return e;
  int pairs = std::min(std::min(clusters, max_pairs), prm.units);
  if (pairs < 1) pairs = 1;
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  if (pdl) {  // may start while the previous kernel in the stream drains (see pdl_wait in the kernel)
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 2;
  }
  return cudaLaunchKernelEx(&cfg, kern, m.w, m.h, m.e, m.gok, m.gom, prm);
}

cudaError_t launch_bwd_scores_stagger_kernel(bool bf16, const BwdScoresMaps& maps, const BwdScoresParams& prm,
                                             int max_pairs, bool pdl, cudaStream_t st) {
  return bf16 ? launch_stagger<true, 3>(maps, prm, max_pairs, pdl, st)
              : launch_stagger<false, 3>(maps, prm, max_pairs, pdl, st);
}

}  // namespace tc
}  // namespace swvr
