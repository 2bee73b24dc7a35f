// Tensor-core (tcgen05) backward score kernel on sm_100a, vocabulary-major, 2-SM.
//
// A CTA pair (cluster of 2) owns a 256-row vocabulary tile of the current chunk (the MMA M
// dimension: 128 rows, TMEM lanes and threads per CTA) and walks a range of BN-token tiles:
//   S^T  = W_tile . h_tile^T                 (K = hidden; recompute of the forward scores)
//   dP^T = E_tile . dO_tile^T                (K = D)
//   P    = 2^(S*s*log2e + b*log2e - LSE*log2e),   dS = P * (dP - delta)
//   db  += rowsum(dS)                        (thread-local: the thread owns the row)
//   dE  += P^T . dO_tile                     (A = P read from TMEM, D in TMEM)
//   dS^T * s is stored in the compute dtype for the dh / dW GEMMs (tc_gemm.cu).
// All three products are tcgen05.mma.cta_group::2 issued by the even CTA: each CTA stages
// its own 128 W rows and half of the h tile (BN/2 tokens) per 64-wide K-block.
//
// Token tiles.  The S recompute streams W and h from L2 at (128 + BN/2) * 128 bytes per CTA
// per 2*BN MMA cycles, so the tile width sets the L2 feed the kernel needs: 96 B/cycle/SM at
// BN = 128, 75 at BN = 192 (the forward kernel's operand shape).  S is double-buffered
// (2 x BN TMEM columns) so a tile's gradient pass runs under the next tile's MMAs.
//  * BN = 128 (any D): S 2 x 128, dP 128, dE 64/128 columns; 4 stages of 128-wide K-blocks
//    for D <= 64, 3 for D <= 128.  For D <= 256 dE is N = 256 and takes 256 columns, so S is
//    single-buffered (2 stages): a tile's gradient pass and its dE run before the next tile's
//    S MMAs, and the MN-major gO is loaded with the tile's own K-major copy.
//  * BN = 192 (D <= 64, long K): S 2 x 192 and dE 64 leave 64 columns for dP, so dP^T is
//    computed in three 64-token chunks.  The MMA thread issues the first right after the
//    tile's S; the next ones while it streams the following tile's S K-loop, each as soon as
//    both CTAs' gradient passes have read the previous chunk (a non-blocking barrier test
//    between K stages).  The K-major gO copy is double-buffered, because the last chunk of a
//    tile is issued during the next tile's loads.  3 stages.
// With two S buffers the pair's tiles form one sequence across its units: tile g's S loop
// runs while the gradient warps process tile g-1, also when g-1 closes the previous unit
// (its remaining dP chunks are issued during g's S loop and its dE after it), so no unit
// boundary drains the pipeline.  E is single-buffered: a unit's E is loaded at the last
// stage of its first tile, after the previous unit's last dP chunk has completed.
// gO is staged twice per token tile: the CTA's half of each dP chunk's tokens, K-major, as
// the B operand of dP^T (loaded during the tile's S K-loop), and the CTA's half of the
// embedding columns of all BN tokens, MN-major, as the B operand of dE (single-buffered,
// loaded one tile later, after the previous dE).  For D <= 64 dE is N = 64 and the MN-major
// copy is 32 columns wide with a 64-byte swizzle; for D <= 128 it is N = 128 with a 128-byte
// swizzle.
// dE and db of a unit go to a partial slot; reduce_de_db_kernel (small.cu) sums the token
// splits of a vocabulary row in a fixed order, so the result is deterministic.
// From the second chunk on, the launch may overlap the previous chunk's GEMM (programmatic
// dependent launch): loads and MMAs read inputs only, and the gradient warps wait for the
// predecessors (pdl_wait) before their first dS or partial-slot store.
//
// Replaces the reference's per-chunk recompute GEMM + Triton _bwd_chunk_kernel
// (swvr/chunked.py:120-131, swvr/triton_kernels.py:76-118).
#include <cstdlib>

#include "ptx.cuh"
#include "tc.cuh"

namespace swvr {
namespace tc {

// KH: 64-wide K halves per pipeline stage (8 MMAs per barrier round trip of the single
// MMA-issuing thread).
template <bool kBF16, int DP, int BN, int NS, int KH>
struct BwdCfg {
  static constexpr int BOX = 128 * 128;         // 128 rows x 128 bytes (64 16-bit elements)
  static constexpr int HBOX = (BN / 2) * 128;   // this CTA's BN/2 h rows x 128 bytes
  static constexpr int A_BYTES = KH * BOX;      // this CTA's 128 W rows x 64*KH K
  static constexpr int B_BYTES = KH * HBOX;     // this CTA's BN/2 h rows x 64*KH K
  // D padded to 256: dE needs 256 TMEM columns, so S is single-buffered (the gradient pass
  // then runs between a tile's S MMAs and the next tile's instead of under them)
  static constexpr bool kSingleS = DP == 256;
  static constexpr int DPC = bwd_dp_chunk(BN);   // tokens per dP^T chunk
  static constexpr int NCH = BN / DPC;           // dP^T chunks per tile
  static constexpr int DEN = DP == 64 ? 64 : (DP == 128 ? 128 : 256);  // dE MMA N (padded)
  static constexpr int GOM_W = DEN / 2;                // embedding columns of gO this CTA stages for dE
  static constexpr int GOM_BW = GOM_W < 64 ? GOM_W : 64;  // columns per box (one swizzle atom)
  static constexpr int GOM_NB = GOM_W / GOM_BW;        // boxes
  static constexpr int GOM_ROW = GOM_BW * 2;           // bytes per token row of a box (64 or 128)
  static constexpr int GOM_BOX = BN * GOM_ROW;         // BN tokens, MN-major
  static constexpr int GOM_BYTES = GOM_NB * GOM_BOX;
  static constexpr int E_BYTES = (DP / 64) * BOX;      // this CTA's 128 E rows x DP
  static constexpr int GOK_CBOX = (DPC / 2) * 128;     // one 64-column box of a chunk: DPC/2 tokens
  static constexpr int GOK_CH = (DP / 64) * GOK_CBOX;  // one chunk (K-major)
  static constexpr int GOK_BYTES = NCH * GOK_CH;       // one tile
  static constexpr int GOK_NB = NCH > 1 ? 2 : 1;       // tile buffers
  static constexpr int SMEM_A = 0;
  static constexpr int SMEM_B = SMEM_A + NS * A_BYTES;
  static constexpr int SMEM_GOM = SMEM_B + NS * B_BYTES;  // operand reads stay below SMEM_E
  static constexpr int SMEM_GOK = SMEM_GOM + GOM_BYTES;
  static constexpr int SMEM_E = SMEM_GOK + GOK_NB * GOK_BYTES;
  static constexpr int SMEM_LSE = SMEM_E + E_BYTES;
  static constexpr int SMEM_DELTA = SMEM_LSE + BN * 4;
  static constexpr int SMEM_BAR = SMEM_DELTA + BN * 4;
  static constexpr int NBAR = 2 * NS + 18;
  static constexpr int SMEM_TOTAL = SMEM_BAR + NBAR * 8 + 16;
  static constexpr int SMEM_ALLOC = SMEM_TOTAL + 1024;
  static constexpr uint32_t S_COL = 0, DP_COL = (kSingleS ? 1 : 2) * BN, DE_COL = DP_COL + DPC;
  static_assert(DE_COL + DEN <= 512, "TMEM budget");
  static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
  static_assert(DP == 64 || DP == 128 || DP == 256, "D padding");
  static_assert(BN == 128 || (BN == 192 && DP == 64), "token tile");
  static_assert(DPC % 32 == 0 && BN % DPC == 0 && (kSingleS ? NCH == 1 : true), "dP chunks");
  static_assert(GOM_BYTES % 1024 == 0 && GOK_CBOX % 1024 == 0 && HBOX % 1024 == 0, "1024-byte alignment");
};

template <bool kBF16, int DP, int BN, int NS, int KH>
__global__ void __launch_bounds__(256, 1)
    bwd_scores_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_h,
                      const __grid_constant__ CUtensorMap tm_e, const __grid_constant__ CUtensorMap tm_gok,
                      const __grid_constant__ CUtensorMap tm_gom, const BwdScoresParams p) {
  using Cfg = BwdCfg<kBF16, DP, BN, NS, KH>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::SMEM_BAR);
  uint64_t* full = bars;               // [NS] leader: both CTAs' bytes
  uint64_t* empty = bars + NS;         // [NS] both (multicast commit)
  uint64_t* e_full = bars + 2 * NS;    // leader: both CTAs' bytes
  uint64_t* e_empty = e_full + 1;      // both
  uint64_t* gok_full = e_empty + 1;    // [2] leader: both CTAs' bytes
  uint64_t* gok_empty = gok_full + 2;  // [2] both
  uint64_t* gom_full = gok_empty + 2;  // leader: both CTAs' bytes
  uint64_t* gom_empty = gom_full + 1;  // both
  uint64_t* s_full = gom_empty + 1;    // [2] both
  uint64_t* dp_full = s_full + 2;      // both: one phase per dP chunk
  uint64_t* dp_free = dp_full + 1;     // leader: one arrival per CTA per dP chunk
  uint64_t* p_ready = dp_free + 1;     // [2] leader: one arrival per CTA
  uint64_t* de_full = p_ready + 2;     // both
  uint64_t* de_free = de_full + 1;     // leader: one arrival per CTA
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
    mbar_init(e_full, 1);
    mbar_init(e_empty, 1);
    mbar_init(gom_full, 1);
    mbar_init(gom_empty, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&gok_full[b], 1);
      mbar_init(&gok_empty[b], 1);
      mbar_init(&s_full[b], 1);
      mbar_init(&p_ready[b], 2);
    }
    mbar_init(dp_full, 1);
    mbar_init(dp_free, 2);
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
  const int KB = (p.K + 64 * KH - 1) / (64 * KH);  // pipeline stages per S tile
  const int kx = min(NS, KB - 1);                  // stage after which a tile's gO loads are issued

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer (both CTAs)
      // gO (K-major) of tile i and gO (MN-major) of the tile before it are loaded after stage
      // kx of tile i's W / h loads: by then the MMAs that last read those buffers have
      // completed (in-order MMA execution), so the waits below do not stall the W / h stream.
      uint32_t stage = 0, sphase = 0, g = 0, uc = 0;
      int prev_it = 0;  // token tile of the previous tile of this pair (double-buffered S)
      for (int u = pair; u < p.units; u += npairs) {
        int vt, ts;
        bwd_unit(p, u, &vt, &ts);
        const int it0 = ts * p.per_t, it1 = min(it0 + p.per_t, p.NT);
        if (it1 <= it0) continue;
        const int vrow0 = p.v_begin + vt * 256 + static_cast<int>(rank) * 128;
        for (int it = it0; it < it1; ++it, ++g) {
          const int trow = it * BN + static_cast<int>(rank) * (BN / 2);
          for (int kb = 0; kb < KB; ++kb) {
            if (!mbar_wait(&empty[stage], sphase ^ 1u, abort_flag, kErrBwdScores | 2)) goto done;
            if (leader) mbar_arrive_expect_tx(&full[stage], 2 * (Cfg::A_BYTES + Cfg::B_BYTES));
            const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
#pragma unroll
            for (int hk = 0; hk < KH; ++hk) {
              const int k0 = (kb * KH + hk) * 64;  // past K the boxes read zero fill
              tma_load_2d_pair(smem + Cfg::SMEM_A + stage * Cfg::A_BYTES + hk * Cfg::BOX, &tm_w, fb, k0, vrow0);
              tma_load_2d_pair(smem + Cfg::SMEM_B + stage * Cfg::B_BYTES + hk * Cfg::HBOX, &tm_h, fb, k0, trow);
            }
            if (++stage == NS) {
              stage = 0;
              sphase ^= 1u;
            }
            if (kb == kx && !p.aux_loads) {
              {
                // gO, K-major: this CTA's DPC/2 tokens of each dP chunk
                const uint32_t kbuf = g % Cfg::GOK_NB;
                if (!mbar_wait(&gok_empty[kbuf], ((g / Cfg::GOK_NB) & 1u) ^ 1u, abort_flag, kErrBwdScores | 3))
                  goto done;
                if (leader) mbar_arrive_expect_tx(&gok_full[kbuf], 2 * Cfg::GOK_BYTES);
                const uint32_t gb = mapa_shared(smem_u32(&gok_full[kbuf]), 0);
#pragma unroll
                for (int jj = 0; jj < Cfg::NCH; ++jj)
#pragma unroll
                  for (int c = 0; c < DP / 64; ++c)
                    tma_load_2d_pair(smem + Cfg::SMEM_GOK + kbuf * Cfg::GOK_BYTES + jj * Cfg::GOK_CH + c * Cfg::GOK_CBOX,
                                     &tm_gok, gb, c * 64,
                                     it * BN + jj * Cfg::DPC + static_cast<int>(rank) * (Cfg::DPC / 2));
              }
              // MN-major gO of the tile whose dE comes next: with single-buffered S this tile
              // (its dE runs before the next S); otherwise the previous tile of the pair,
              // which may belong to the previous unit
              const bool gom_now = Cfg::kSingleS || g > 0;
              if (gom_now) {
                const uint32_t fill = Cfg::kSingleS ? g : g - 1u;  // one MN-major fill per tile
                const int gom_tile = Cfg::kSingleS ? it : prev_it;
                if (!mbar_wait(gom_empty, (fill & 1u) ^ 1u, abort_flag, kErrBwdScores | 4)) goto done;
                if (leader) mbar_arrive_expect_tx(gom_full, 2 * Cfg::GOM_BYTES);
                const uint32_t mb = mapa_shared(smem_u32(gom_full), 0);
#pragma unroll
                for (int c = 0; c < Cfg::GOM_NB; ++c)
                  tma_load_2d_pair(smem + Cfg::SMEM_GOM + c * Cfg::GOM_BOX, &tm_gom, mb,
                                   static_cast<int>(rank) * Cfg::GOM_W + c * Cfg::GOM_BW, gom_tile * BN);
              }
            }
            if (!p.aux_loads && it == it0 && kb == (Cfg::kSingleS ? kx : KB - 1)) {
              // E of this unit.  With double-buffered S the previous unit's last dP chunks
              // may still be issued during this tile's S loop, so E is replaced at its end.
              if (!mbar_wait(e_empty, (uc & 1u) ^ 1u, abort_flag, kErrBwdScores | 1)) goto done;
              if (leader) mbar_arrive_expect_tx(e_full, 2 * Cfg::E_BYTES);
              const uint32_t eb = mapa_shared(smem_u32(e_full), 0);
#pragma unroll
              for (int c = 0; c < DP / 64; ++c)
                tma_load_2d_pair(smem + Cfg::SMEM_E + c * Cfg::BOX, &tm_e, eb, c * 64, vrow0);
            }
          }
          prev_it = it;
        }
        ++uc;
      }
      if (!p.aux_loads && !Cfg::kSingleS && g > 0) {
        // the pair's last tile: its MN-major gO, once the previous tile's dE has read the buffer
        if (!mbar_wait(gom_empty, ((g - 1u) & 1u) ^ 1u, abort_flag, kErrBwdScores | 4)) goto done;
        if (leader) mbar_arrive_expect_tx(gom_full, 2 * Cfg::GOM_BYTES);
        const uint32_t mb = mapa_shared(smem_u32(gom_full), 0);
#pragma unroll
        for (int c = 0; c < Cfg::GOM_NB; ++c)
          tma_load_2d_pair(smem + Cfg::SMEM_GOM + c * Cfg::GOM_BOX, &tm_gom, mb,
                           static_cast<int>(rank) * Cfg::GOM_W + c * Cfg::GOM_BW, prev_it * BN);
      }
    }
  } else if (warp == 2) {
    if (lane == 0 && p.aux_loads) {
      // ------------------------------------------------ gO / E producer (both CTAs, aux_loads)
      // The same loads, waits and buffers as the interleaved path above, in the order the MMA
      // thread consumes them: per tile, the unit's E (first tile), the tile's K-major gO, and
      // the MN-major gO of the tile whose dE comes next.  The W / h stream of warp 0 then
      // never waits on these buffers.
      uint32_t g = 0, uc = 0;
      int prev_it = 0;
      for (int u = pair; u < p.units; u += npairs) {
        int vt, ts;
        bwd_unit(p, u, &vt, &ts);
        const int it0 = ts * p.per_t, it1 = min(it0 + p.per_t, p.NT);
        if (it1 <= it0) continue;
        const int vrow0 = p.v_begin + vt * 256 + static_cast<int>(rank) * 128;
        for (int it = it0; it < it1; ++it, ++g) {
          if (it == it0) {
            if (!mbar_wait(e_empty, (uc & 1u) ^ 1u, abort_flag, kErrBwdScores | 1)) goto done;
            if (leader) mbar_arrive_expect_tx(e_full, 2 * Cfg::E_BYTES);
            const uint32_t eb = mapa_shared(smem_u32(e_full), 0);
#pragma unroll
            for (int c = 0; c < DP / 64; ++c)
              tma_load_2d_pair(smem + Cfg::SMEM_E + c * Cfg::BOX, &tm_e, eb, c * 64, vrow0);
          }
          {
            const uint32_t kbuf = g % Cfg::GOK_NB;
            if (!mbar_wait(&gok_empty[kbuf], ((g / Cfg::GOK_NB) & 1u) ^ 1u, abort_flag, kErrBwdScores | 3))
              goto done;
            if (leader) mbar_arrive_expect_tx(&gok_full[kbuf], 2 * Cfg::GOK_BYTES);
            const uint32_t gb = mapa_shared(smem_u32(&gok_full[kbuf]), 0);
#pragma unroll
            for (int jj = 0; jj < Cfg::NCH; ++jj)
#pragma unroll
              for (int c = 0; c < DP / 64; ++c)
                tma_load_2d_pair(smem + Cfg::SMEM_GOK + kbuf * Cfg::GOK_BYTES + jj * Cfg::GOK_CH + c * Cfg::GOK_CBOX,
                                 &tm_gok, gb, c * 64,
                                 it * BN + jj * Cfg::DPC + static_cast<int>(rank) * (Cfg::DPC / 2));
          }
          if (Cfg::kSingleS || g > 0) {
            const uint32_t fill = Cfg::kSingleS ? g : g - 1u;
            const int gom_tile = Cfg::kSingleS ? it : prev_it;
            if (!mbar_wait(gom_empty, (fill & 1u) ^ 1u, abort_flag, kErrBwdScores | 4)) goto done;
            if (leader) mbar_arrive_expect_tx(gom_full, 2 * Cfg::GOM_BYTES);
            const uint32_t mb = mapa_shared(smem_u32(gom_full), 0);
#pragma unroll
            for (int c = 0; c < Cfg::GOM_NB; ++c)
              tma_load_2d_pair(smem + Cfg::SMEM_GOM + c * Cfg::GOM_BOX, &tm_gom, mb,
                               static_cast<int>(rank) * Cfg::GOM_W + c * Cfg::GOM_BW, gom_tile * BN);
          }
          prev_it = it;
        }
        ++uc;
      }
      if (!Cfg::kSingleS && g > 0) {
        if (!mbar_wait(gom_empty, ((g - 1u) & 1u) ^ 1u, abort_flag, kErrBwdScores | 4)) goto done;
        if (leader) mbar_arrive_expect_tx(gom_full, 2 * Cfg::GOM_BYTES);
        const uint32_t mb = mapa_shared(smem_u32(gom_full), 0);
#pragma unroll
        for (int c = 0; c < Cfg::GOM_NB; ++c)
          tma_load_2d_pair(smem + Cfg::SMEM_GOM + c * Cfg::GOM_BOX, &tm_gom, mb,
                           static_cast<int>(rank) * Cfg::GOM_W + c * Cfg::GOM_BW, prev_it * BN);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------------------ MMA issuer (leader only)
      const uint32_t idS = idesc_f16(kBF16, 256, BN, false, false);
      const uint32_t idDP = idesc_f16(kBF16, 256, Cfg::DPC, false, false);
      const uint32_t idDE = idesc_f16(kBF16, 256, Cfg::DEN, false, true);
      // q counts the dP chunks issued so far; before chunk q is written into the single dP
      // buffer, both CTAs' gradient passes must have read chunk q-1 (dp_free phase q-1).
      uint32_t stage = 0, sphase = 0, g = 0, uc = 0, q = 0;
      const uint32_t ebase = smem_u32(smem + Cfg::SMEM_E);
      const uint32_t gokbase = smem_u32(smem + Cfg::SMEM_GOK);
      const uint32_t gombase = smem_u32(smem + Cfg::SMEM_GOM);
      // stage-0 descriptors; a stage / K half / 16-wide K step adds (byte offset >> 4)
      const uint64_t da0 = sdesc_sw128(smem_u32(smem + Cfg::SMEM_A), 16, 1024);
      const uint64_t db0 = sdesc_sw128(smem_u32(smem + Cfg::SMEM_B), 16, 1024);
      // S^T of tile g (global tile counter) into S buffer b: the unit's K loop
      auto issue_s = [&](uint32_t b, uint32_t kb) {
        const uint64_t sa = static_cast<uint64_t>(stage * (Cfg::A_BYTES >> 4));
        const uint64_t sb = static_cast<uint64_t>(stage * (Cfg::B_BYTES >> 4));
#pragma unroll
        for (int k8 = 0; k8 < 4 * KH; ++k8)
          umma2_ss(tmem + Cfg::S_COL + b * BN, da0 + sa + (k8 >> 2) * (Cfg::BOX >> 4) + (k8 & 3) * 2,
                   db0 + sb + (k8 >> 2) * (Cfg::HBOX >> 4) + (k8 & 3) * 2, idS, (kb | k8) ? 1u : 0u);
        umma2_commit_mc(&empty[stage], 3);
        if (++stage == NS) {
          stage = 0;
          sphase ^= 1u;
        }
      };
      // dP^T chunk jj of tile gt: E . gO_chunk^T into the dP buffer.  After the last chunk of
      // a unit's last tile the unit's E may be replaced.
      auto issue_dp = [&](uint32_t gt, int jj, bool unit_last) {
        const uint32_t kbuf = gt % Cfg::GOK_NB;
        const uint32_t gk = gokbase + kbuf * Cfg::GOK_BYTES + jj * Cfg::GOK_CH;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < DP / 16; ++ks)
          umma2_ss(tmem + Cfg::DP_COL, sdesc_sw128(ebase + (ks >> 2) * Cfg::BOX + (ks & 3) * 32, 16, 1024),
                   sdesc_sw128(gk + (ks >> 2) * Cfg::GOK_CBOX + (ks & 3) * 32, 16, 1024), idDP, ks ? 1u : 0u);
        if (jj == Cfg::NCH - 1) {
          umma2_commit_mc(&gok_empty[kbuf], 3);
          if (unit_last) umma2_commit_mc(e_empty, 3);
        }
        umma2_commit_mc(dp_full, 3);
      };
      // dE += P^T . gO of tile gt (S buffer sb), once both CTAs' gradient passes have written
      // P; the first tile of a unit overwrites dE, after the previous unit's dE was read out.
      auto issue_de = [&](uint32_t gt, uint32_t sb, bool unit_first, bool unit_last, uint32_t guc) -> bool {
        if (!mbar_wait(gom_full, gt & 1u, abort_flag, kErrBwdScores | 9)) return false;
        if (need_de) {
          if (unit_first && guc > 0 && !mbar_wait(de_free, (guc - 1u) & 1u, abort_flag, kErrBwdScores | 9))
            return false;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < BN / 16; ++ks) {
            const uint64_t bdesc = Cfg::GOM_ROW == 64 ? sdesc_sw64(gombase + ks * 16 * 64, Cfg::GOM_BOX, 512)
                                                      : sdesc_sw128(gombase + ks * 16 * 128, Cfg::GOM_BOX, 1024);
            umma2_ts(tmem + Cfg::DE_COL, tmem + Cfg::S_COL + sb * BN + ks * 8, bdesc, idDE,
                     (unit_first && ks == 0) ? 0u : 1u);
          }
        }
        umma2_commit_mc(gom_empty, 3);
        if (need_de && unit_last) umma2_commit_mc(de_full, 3);
        return true;
      };
      if constexpr (Cfg::kSingleS) {
        // one S buffer: each tile's S, dP, gradient pass and dE before the next tile's S
        for (int u = pair; u < p.units; u += npairs) {
          int vt, ts;
          bwd_unit(p, u, &vt, &ts);
          const int it0 = ts * p.per_t, it1 = min(it0 + p.per_t, p.NT);
          const int n = it1 - it0;
          if (n <= 0) continue;
          for (int j = 0; j < n; ++j, ++g) {
            for (int kb = 0; kb < KB; ++kb) {
              if (!mbar_wait(&full[stage], sphase, abort_flag, kErrBwdScores | 5)) goto done;
              issue_s(0u, kb);
            }
            umma2_commit_mc(&s_full[0], 3);
            if (q > 0 && !mbar_wait(dp_free, (q - 1u) & 1u, abort_flag, kErrBwdScores | 6)) goto done;
            if (j == 0 && !mbar_wait(e_full, uc & 1u, abort_flag, kErrBwdScores | 6)) goto done;
            if (!mbar_wait(&gok_full[0], g & 1u, abort_flag, kErrBwdScores | 7)) goto done;
            issue_dp(g, 0, j == n - 1);
            ++q;
            if (!mbar_wait(&p_ready[0], g & 1u, abort_flag, kErrBwdScores | 8)) goto done;
            if (!issue_de(g, 0u, j == 0, j == n - 1, uc)) goto done;
          }
          ++uc;
        }
      } else {
        // Two S buffers: tile g's S loop runs while the gradient warps process tile g-1; the
        // pair's tiles form one sequence across units, so a unit's last tile is finished
        // (remaining dP chunks, dE) during the next unit's first S loop.
        int pj = Cfg::NCH;  // next dP chunk of the previous tile (NCH: none left)
        bool prev_first = false, prev_last = false;  // the previous tile opens / closes its unit
        uint32_t prev_uc = 0;                        // and its unit
        for (int u = pair; u < p.units; u += npairs) {
          int vt, ts;
          bwd_unit(p, u, &vt, &ts);
          const int it0 = ts * p.per_t, it1 = min(it0 + p.per_t, p.NT);
          const int n = it1 - it0;
          if (n <= 0) continue;
          for (int j = 0; j < n; ++j, ++g) {
            const uint32_t b = g & 1u;
            for (int kb = 0; kb < KB; ++kb) {
              if (!mbar_wait(&full[stage], sphase, abort_flag, kErrBwdScores | 5)) goto done;
              issue_s(b, kb);
              if constexpr (Cfg::NCH > 1) {
                // the previous tile's next dP chunk, once its gradient passes have read the last
                if (pj < Cfg::NCH && mbar_test(dp_free, (q - 1u) & 1u)) {
                  issue_dp(g - 1u, pj, prev_last);
                  ++pj;
                  ++q;
                }
              }
            }
            umma2_commit_mc(&s_full[b], 3);
            // the previous tile's remaining dP chunks
            while (pj < Cfg::NCH) {
              if (!mbar_wait(dp_free, (q - 1u) & 1u, abort_flag, kErrBwdScores | 13)) goto done;
              issue_dp(g - 1u, pj, prev_last);
              ++pj;
              ++q;
            }
            const bool have_prev = g > 0;
            if (have_prev) {
              if (!mbar_wait(&p_ready[(g - 1u) & 1u], ((g - 1u) >> 1) & 1u, abort_flag, kErrBwdScores | 8)) goto done;
              // across a unit boundary the previous unit's dE goes first: this tile's first dP
              // chunk waits for the new E, which the producer loads at the end of this S loop
              if (prev_last && !issue_de(g - 1u, (g - 1u) & 1u, prev_first, true, prev_uc)) goto done;
            }
            // this tile's first dP chunk, once both CTAs' gradient passes have read the last one
            if (q > 0 && !mbar_wait(dp_free, (q - 1u) & 1u, abort_flag, kErrBwdScores | 6)) goto done;
            if (j == 0 && !mbar_wait(e_full, uc & 1u, abort_flag, kErrBwdScores | 6)) goto done;
            if (!mbar_wait(&gok_full[g % Cfg::GOK_NB], (g / Cfg::GOK_NB) & 1u, abort_flag, kErrBwdScores | 7))
              goto done;
            issue_dp(g, 0, j == n - 1);
            ++q;
            pj = 1;
            if (have_prev && !prev_last && !issue_de(g - 1u, (g - 1u) & 1u, prev_first, false, prev_uc)) goto done;
            prev_first = j == 0;
            prev_last = j == n - 1;
            prev_uc = uc;
          }
          ++uc;
        }
        if (g > 0) {
          // the pair's last tile
          while (pj < Cfg::NCH) {
            if (!mbar_wait(dp_free, (q - 1u) & 1u, abort_flag, kErrBwdScores | 13)) goto done;
            issue_dp(g - 1u, pj, prev_last);
            ++pj;
            ++q;
          }
          if (!mbar_wait(&p_ready[(g - 1u) & 1u], ((g - 1u) >> 1) & 1u, abort_flag, kErrBwdScores | 8)) goto done;
          if (!issue_de(g - 1u, (g - 1u) & 1u, prev_first, true, prev_uc)) goto done;
        }
      }
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------------- gradient warps (both CTAs)
    // lse_s holds -LSE*log2e and delta_s holds -delta for the current token tile, so each
    // pair of tokens costs a handful of packed f32x2 ops.  Each thread stores its row of
    // dS*s (BN tokens, contiguous) with 16-byte stores, one dP chunk at a time.
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
      int vt, ts;
      bwd_unit(p, u, &vt, &ts);
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
#pragma unroll
        for (int i = r; i < BN; i += 128) {
          const int t = t0 + i;
          lse_s[i] = t < p.N ? -p.lse[t] * kLog2e : -INFINITY;
          delta_s[i] = t < p.N ? -p.delta[t] : 0.f;
        }
        named_bar_sync(1, 128);
        const uint32_t b = Cfg::kSingleS ? 0u : (g & 1u);
        const uint32_t s_par = Cfg::kSingleS ? (g & 1u) : ((g >> 1) & 1u);
        if (!warp_wait(&s_full[b], s_par, abort_flag, kErrBwdScores | 10)) goto done;
        const uint32_t sbase = trow + Cfg::S_COL + b * BN;
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
            if (last) mbar_arrive_cluster_relaxed(p_ready_leader + b * 8);
          }
        }
      }
      const int64_t slot = static_cast<int64_t>(vt * p.TS + ts) * 256 + static_cast<int>(rank) * 128 + r;
      if (need_de) {
        if (!warp_wait(de_full, uc & 1u, abort_flag, kErrBwdScores | 12)) goto done;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < DP / 32; ++c) {
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

template <bool kBF16, int DP, int BN, int NS, int KH>
static cudaError_t launch_bwd(const BwdScoresMaps& m, const BwdScoresParams& prm, int max_pairs, bool pdl,
                              cudaStream_t st) {
  using Cfg = BwdCfg<kBF16, DP, BN, NS, KH>;
  auto kern = bwd_scores_kernel<kBF16, DP, BN, NS, KH>;
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

int bwd_gom_width(int DP) { return DP == 64 ? 32 : 64; }  // columns per box (DP 256: two boxes per CTA)

int bwd_token_tile(int DP, int64_t K) {
  // 192-token tiles need a K loop long enough to cover the dP chunk round trips under the
  // next tile's S MMAs; SWVR_BWD_TOKEN_TILE (128 or 192) overrides the choice.
  int bn = (DP == 64 && K >= 1024) ? 192 : 128;
  if (const char* s = std::getenv("SWVR_BWD_TOKEN_TILE")) {
    const int v = std::atoi(s);
    if (v == 128 || (v == 192 && DP == 64)) bn = v;
  }
  return bn;
}

cudaError_t launch_bwd_scores_kernel(bool bf16, int DP, int BN, const BwdScoresMaps& maps,
                                     const BwdScoresParams& prm, int max_pairs, bool pdl, cudaStream_t st) {
  if (DP == 64 && BN == 192)
    return bf16 ? launch_bwd<true, 64, 192, 3, 2>(maps, prm, max_pairs, pdl, st)
                : launch_bwd<false, 64, 192, 3, 2>(maps, prm, max_pairs, pdl, st);
  if (BN != 128) return cudaErrorInvalidValue;
  if (DP == 64)
    return bf16 ? launch_bwd<true, 64, 128, 4, 2>(maps, prm, max_pairs, pdl, st)
                : launch_bwd<false, 64, 128, 4, 2>(maps, prm, max_pairs, pdl, st);
  if (DP == 128)
    return bf16 ? launch_bwd<true, 128, 128, 3, 2>(maps, prm, max_pairs, pdl, st)
                : launch_bwd<false, 128, 128, 3, 2>(maps, prm, max_pairs, pdl, st);
  return bf16 ? launch_bwd<true, 256, 128, 2, 2>(maps, prm, max_pairs, pdl, st)
              : launch_bwd<false, 256, 128, 2, 2>(maps, prm, max_pairs, pdl, st);
}

}  // namespace tc
}  // namespace swvr
