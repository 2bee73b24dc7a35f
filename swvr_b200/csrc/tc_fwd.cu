// Tensor-core (tcgen05) forward of the softmax readout on sm_100a, 2-SM.
//
// A CTA pair (cluster of 2) walks work units (a 256-token tile x a contiguous range of
// vocabulary tiles of BV rows: 192 for D <= 128, 128 for D <= 256).  Each CTA owns 128 of the
// tokens (TMEM lanes = token rows).
// Per vocabulary tile j, with tcgen05.mma.cta_group::2 issued by the even CTA:
//   S_j  = h_tile . W_j^T            M = 256 tokens, N = BV rows; each CTA stages its own
//                                    128 h rows and half of the W rows per K-block
//   P_j  = 2^(S_j*s*log2e + b*log2e - m_ref), rounded to bf16/fp16 and stored back into
//          TMEM over S_j (one thread per token row: row max / row sum are thread-local)
//   O   += P_j . E_j                 A = P from TMEM; B = E_j, N = 128 or 256 (each CTA stages
//                                    half of the embedding columns; past D the boxes read
//                                    zero fill)
// so neither S nor P ever leaves the SM.  A pair moves 28 KB per CTA per 64-wide K-block
// for 2*256*192*64 FLOP, against 40 KB for a single-CTA 128x192 tile: the L2->SMEM feed,
// which bounds the single-CTA kernel, drops below the MMA rate.  Warp roles: warp 0 issues
// TMA loads, warp 1 (one thread, even CTA) issues MMAs, warps 4-7 run the online softmax.
// S is double-buffered in TMEM (2 x BV columns, O in the last 128 or 256), so the MMAs of tile
// j+1 overlap the softmax of tile j.  The running reference m_ref (log2 units) is only raised
// when a tile's max exceeds it by more than kEmergency octaves (exact either way because l and
// O share m_ref), and then to that max before any P of the tile is written: only l and O (fp32)
// are rescaled, so every 16-bit P value carries one rounding.
//
// Each unit writes its per-row state (m_ref in log2 units, l, O-accumulator) to a partial
// slot; combine_kernel (small.cu) merges the slots of a row in a fixed order.
//
// This replaces the reference's per-chunk cuBLAS S GEMM + Triton _fwd_chunk_kernel
// (swvr/chunked.py:89-95, swvr/triton_kernels.py:37-73) with one fused kernel.
#include "ptx.cuh"
#include "tc.cuh"

namespace swvr {
namespace tc {

// KH: 64-wide K halves per pipeline stage (8 MMAs per barrier round trip of the MMA thread).
// BV: vocabulary rows per tile (the S MMA's N); OW: the O MMA's N (embedding columns padded
// to 128 or 256; each CTA stages OW / 2 of them as 64-column boxes).  Two S buffers and O
// share the 512 TMEM columns: (192, 128) for D <= 128, (128, 256) for D <= 256.
template <bool kBF16, int NS, int KH, int BV_, int OW>
struct FwdCfg {
  static constexpr int BV = BV_;
  static constexpr int HBV = BV / 2;         // W rows staged by each CTA
  static constexpr int BOXA = 128 * 128;     // 128 h rows x 64 K
  static constexpr int BOXB = HBV * 128;     // HBV W rows x 64 K
  static constexpr int A_BYTES = KH * BOXA;
  static constexpr int B_BYTES = KH * BOXB;
  static constexpr int EB = OW / 128;        // 64-column E boxes per CTA
  static constexpr int E_BOX = BV * 128;     // BV vocabulary rows x 64 embedding columns
  static constexpr int E_BYTES = EB * E_BOX;
  static constexpr int SMEM_A = 0;
  static constexpr int SMEM_B = SMEM_A + NS * A_BYTES;
  static constexpr int SMEM_E = SMEM_B + NS * B_BYTES;
  static constexpr int SMEM_BIAS = SMEM_E + 2 * E_BYTES;  // 2 x 256 floats: bias*log2e, -inf past V
  static constexpr int SMEM_BAR = SMEM_BIAS + 2 * 256 * 4;
  static constexpr int NBAR = 2 * NS + 12;
  static constexpr float kEmergency = kBF16 ? 64.f : 8.f;  // max P = 2^kEmergency stays finite in 16 bits
  static constexpr int SMEM_TOTAL = SMEM_BAR + NBAR * 8 + 16;
  static constexpr int SMEM_ALLOC = SMEM_TOTAL + 1024;
  static constexpr uint32_t O_COL = 2 * BV;
  static_assert(O_COL + OW <= 512, "TMEM budget");
  static_assert(OW == 128 || OW == 256, "O width");
  static_assert(BV % 32 == 0 && HBV % 8 == 0, "vocabulary tile");
  static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
  static_assert(BOXA % 1024 == 0 && BOXB % 1024 == 0 && E_BYTES % 1024 == 0, "1024-byte alignment");
};

template <bool kBF16, int NS, int KH, int BV_, int OW>
__global__ void __launch_bounds__(256, 1)
    fwd_kernel(const __grid_constant__ CUtensorMap tm_h, const __grid_constant__ CUtensorMap tm_w,
               const __grid_constant__ CUtensorMap tm_e, const FwdParams p) {
  using Cfg = FwdCfg<kBF16, NS, KH, BV_, OW>;
  constexpr int BV = Cfg::BV;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::SMEM_BAR);
  uint64_t* full = bars;              // [NS] leader: both CTAs' bytes
  uint64_t* empty = bars + NS;        // [NS] both (multicast commit)
  uint64_t* s_full = bars + 2 * NS;   // [2] both
  uint64_t* p_ready = s_full + 2;     // [2] leader: one arrival per CTA
  uint64_t* e_full = p_ready + 2;     // [2] leader: both CTAs' bytes
  uint64_t* e_empty = e_full + 2;     // [2] both
  uint64_t* pe_done = e_empty + 2;    // both
  uint64_t* o_free = pe_done + 1;     // leader: one arrival per CTA
  uint64_t* spare = o_free + 1;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + Cfg::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_ready[b], 2);
      mbar_init(&e_full[b], 1);
      mbar_init(&e_empty[b], 1);
    }
    mbar_init(pe_done, 1);
    mbar_init(o_free, 2);
    mbar_init(spare, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_h);
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_e);
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
  if (threadIdx.x == 0) pdl_trigger();  // the combine may launch early; it waits for this grid
  const int KB = (p.K + 64 * KH - 1) / (64 * KH);  // pipeline stages per S tile

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer (both CTAs)
      uint32_t stage = 0, sphase = 0, g = 0;
      for (int u = pair; u < p.units; u += npairs) {
        int mt, sp;
        fwd_unit(p, u, &mt, &sp);
        const int vt0 = sp * p.per, vt1 = min(vt0 + p.per, p.VT);
        const int hrow = mt * 256 + static_cast<int>(rank) * 128;
        for (int vt = vt0; vt < vt1; ++vt, ++g) {
          const int wrow = vt * BV + static_cast<int>(rank) * Cfg::HBV;
          for (int kb = 0; kb < KB; ++kb) {
            if (!mbar_wait(&empty[stage], sphase ^ 1u, abort_flag, kErrFwd | 1)) goto done;
            if (leader) mbar_arrive_expect_tx(&full[stage], 2 * (Cfg::A_BYTES + Cfg::B_BYTES));
            const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
#pragma unroll
            for (int hk = 0; hk < KH; ++hk) {
              const int k0 = (kb * KH + hk) * 64;  // past K the boxes read zero fill
              tma_load_2d_pair(smem + Cfg::SMEM_A + stage * Cfg::A_BYTES + hk * Cfg::BOXA, &tm_h, fb, k0, hrow);
              tma_load_2d_pair(smem + Cfg::SMEM_B + stage * Cfg::B_BYTES + hk * Cfg::BOXB, &tm_w, fb, k0, wrow);
            }
            if (++stage == NS) {
              stage = 0;
              sphase ^= 1u;
            }
          }
          const uint32_t eb = g & 1u, use = g >> 1;
          if (!mbar_wait(&e_empty[eb], (use & 1u) ^ 1u, abort_flag, kErrFwd | 2)) goto done;
          if (leader) mbar_arrive_expect_tx(&e_full[eb], 2 * Cfg::E_BYTES);
#pragma unroll
          for (int c = 0; c < Cfg::EB; ++c)
            tma_load_2d_pair(smem + Cfg::SMEM_E + eb * Cfg::E_BYTES + c * Cfg::E_BOX, &tm_e,
                             mapa_shared(smem_u32(&e_full[eb]), 0), static_cast<int>(rank) * (OW / 2) + c * 64,
                             vt * BV);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------------------ MMA issuer (leader only)
      const uint32_t idS = idesc_f16(kBF16, 256, BV, false, false);
      const uint32_t idPE = idesc_f16(kBF16, 256, OW, false, true);
      // stage-0 descriptors; a stage / K half / 16-wide K step adds (byte offset >> 4)
      const uint64_t da0 = sdesc_sw128(smem_u32(smem + Cfg::SMEM_A), 16, 1024);
      const uint64_t db0 = sdesc_sw128(smem_u32(smem + Cfg::SMEM_B), 16, 1024);
      uint32_t stage = 0, sphase = 0, g = 0, uc = 0;
      for (int u = pair; u < p.units; u += npairs) {
        int mt, sp;
        fwd_unit(p, u, &mt, &sp);
        const int vt0 = sp * p.per, vt1 = min(vt0 + p.per, p.VT);
        const int ntiles = vt1 - vt0;
        if (ntiles <= 0) continue;
        for (int j = 0; j <= ntiles; ++j) {
          if (j < ntiles) {
            const uint32_t b = g & 1u;
            for (int kb = 0; kb < KB; ++kb) {
              if (!mbar_wait(&full[stage], sphase, abort_flag, kErrFwd | 3)) goto done;
              const uint64_t sa = static_cast<uint64_t>(stage * (Cfg::A_BYTES >> 4));
              const uint64_t sb = static_cast<uint64_t>(stage * (Cfg::B_BYTES >> 4));
#pragma unroll
              for (int k8 = 0; k8 < 4 * KH; ++k8)
                umma2_ss(tmem + b * BV, da0 + sa + (k8 >> 2) * (Cfg::BOXA >> 4) + (k8 & 3) * 2,
                         db0 + sb + (k8 >> 2) * (Cfg::BOXB >> 4) + (k8 & 3) * 2, idS, (kb | k8) ? 1u : 0u);
              umma2_commit_mc(&empty[stage], 3);
              if (++stage == NS) {
                stage = 0;
                sphase ^= 1u;
              }
            }
            umma2_commit_mc(&s_full[b], 3);
            ++g;
          }
          if (j > 0) {
            // O += P . E for the previous tile (its softmax overlapped the MMAs just issued)
            const uint32_t gg = g - 1u - (j < ntiles ? 1u : 0u);
            const uint32_t bb = gg & 1u, use = gg >> 1;
            const bool first = (j == 1);
            if (!mbar_wait(&p_ready[bb], use & 1u, abort_flag, kErrFwd | 4)) goto done;
            if (!mbar_wait(&e_full[bb], use & 1u, abort_flag, kErrFwd | 5)) goto done;
            if (first && uc > 0 && !mbar_wait(o_free, (uc - 1u) & 1u, abort_flag, kErrFwd | 6)) goto done;
            tc_fence_after();
            const uint32_t ebase = smem_u32(smem + Cfg::SMEM_E + bb * Cfg::E_BYTES);
#pragma unroll
            for (int ks = 0; ks < BV / 16; ++ks)
              umma2_ts(tmem + Cfg::O_COL, tmem + bb * BV + ks * 8, sdesc_sw128(ebase + ks * 2048, Cfg::E_BOX, 1024),
                       idPE, (first && ks == 0) ? 0u : 1u);
            umma2_commit_mc(pe_done, 3);
            umma2_commit_mc(&e_empty[bb], 3);
          }
        }
        ++uc;
      }
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------------- softmax warps (both CTAs)
    // One pass per tile.  P = 2^(t - ref) with t = S*s*log2e + b*log2e and ref the running
    // reference.  Two passes over the tile's S in TMEM: the first finds the tile's max tm of t;
    // if tm exceeds ref + kEmergency, ref becomes tm and l and (after the previous P.E
    // completed) O are rescaled by 2^(old - new) in fp32; the second writes P.  P values are
    // bounded by 2^kEmergency, finite in 16 bits, and never rescaled.
    const int r = threadIdx.x - 128;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t trow = tmem + lane_base;
    float* bias_s = reinterpret_cast<float*>(smem + Cfg::SMEM_BIAS);
    const uint32_t p_ready_leader = mapa_shared(smem_u32(p_ready), 0);
    const uint32_t o_free_leader = mapa_shared(smem_u32(o_free), 0);
    uint32_t g = 0;
    for (int u = pair; u < p.units; u += npairs) {
      int mt, sp;
        fwd_unit(p, u, &mt, &sp);
      const int vt0 = sp * p.per, vt1 = min(vt0 + p.per, p.VT);
      if (vt1 <= vt0) continue;
      const int n = mt * 256 + static_cast<int>(rank) * 128 + r;
      float ref = -INFINITY, l = 0.f;
      for (int vt = vt0; vt < vt1; ++vt, ++g) {
        const uint32_t b = g & 1u;
        const bool not_first = vt > vt0;
        const int v0 = vt * BV;
        // stage this tile's bias (log2 units); columns past V get -inf, which masks them
        float* bt = bias_s + b * 256;
        for (int c = r; c < BV; c += 128) {
          const int col = v0 + c;
          bt[c] = col < p.V ? (p.bias ? load_f(p.bias, p.bias_dt, col) * kLog2e : 0.f) : -INFINITY;
        }
        named_bar_sync(1, 128);
        if (!warp_wait(&s_full[b], (g >> 1) & 1u, abort_flag, kErrFwd | 7)) goto done;
        tc_fence_after();
        const uint32_t sbase = trow + b * BV;
        // pass 1: the tile's max of t.  The reference moves at most once per tile, before any P
        // of the tile is written, so no P value is ever rescaled (each keeps one 16-bit rounding)
        float tm = -INFINITY;
#pragma unroll 1
        for (int c = 0; c < BV / 32; ++c) {
          uint32_t x[32];
          tmem_ld32(sbase + c * 32, x);
          tmem_wait_ld();
          const float4* b4 = reinterpret_cast<const float4*>(bt + c * 32);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 bb = b4[q];
            const float2 t0 = ffma2(make_float2(__uint_as_float(x[4 * q]), __uint_as_float(x[4 * q + 1])),
                                    make_float2(p.sc2, p.sc2), make_float2(bb.x, bb.y));
            const float2 t1 = ffma2(make_float2(__uint_as_float(x[4 * q + 2]), __uint_as_float(x[4 * q + 3])),
                                    make_float2(p.sc2, p.sc2), make_float2(bb.z, bb.w));
            tm = fmaxf(tm, fmaxf(fmaxf(t0.x, t0.y), fmaxf(t1.x, t1.y)));
          }
        }
        // a tile whose max exceeds ref + kEmergency sets ref to that max: l now, O below
        const float ref_start = ref;
        float alpha = 1.f;
        if (tm > ref + Cfg::kEmergency) {
          alpha = ref == -INFINITY ? 0.f : ex2(ref - tm);
          ref = tm;
          l *= alpha;
        }
        const float refe = ref == -INFINITY ? 0.f : ref;
        // pass 2: P = 2^(t - ref), summed unrounded into l and stored rounded over S
        float2 lsum = make_float2(0.f, 0.f);
#pragma unroll 1
        for (int c = 0; c < BV / 32; ++c) {
          uint32_t x[32];
          tmem_ld32(sbase + c * 32, x);
          tmem_wait_ld();
          const float4* b4 = reinterpret_cast<const float4*>(bt + c * 32);
          uint32_t pk[16];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 bb = b4[q];
            const float2 t0 = ffma2(make_float2(__uint_as_float(x[4 * q]), __uint_as_float(x[4 * q + 1])),
                                    make_float2(p.sc2, p.sc2), make_float2(bb.x, bb.y));
            const float2 t1 = ffma2(make_float2(__uint_as_float(x[4 * q + 2]), __uint_as_float(x[4 * q + 3])),
                                    make_float2(p.sc2, p.sc2), make_float2(bb.z, bb.w));
            const float2 p0 = make_float2(ex2(t0.x - refe), ex2(t0.y - refe));
            const float2 p1 = make_float2(ex2(t1.x - refe), ex2(t1.y - refe));
            lsum = fadd2(lsum, fadd2(p0, p1));
            pk[2 * q] = pack2<kBF16>(p0.x, p0.y);
            pk[2 * q + 1] = pack2<kBF16>(p1.x, p1.y);
          }
          tmem_st16(sbase + c * 16, pk);
        }
        l += lsum.x + lsum.y;
        // the previous tile's P.E must be done before O is rescaled (consumes one completion)
        if (not_first) {
          if (!warp_wait(pe_done, (g - 1u) & 1u, abort_flag, kErrFwd | 8)) goto done;
          tc_fence_after();
          if (__any_sync(0xffffffffu, ref != ref_start)) {
#pragma unroll 1
            for (int c = 0; c < p.D; c += 32) {
              uint32_t o[32];
              tmem_ld32(trow + Cfg::O_COL + c, o);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
              tmem_st32(trow + Cfg::O_COL + c, o);
            }
          }
        }
        tmem_wait_st();
        tc_fence_before();
        named_bar_sync(1, 128);
        if (r == 0) mbar_arrive_cluster_relaxed(p_ready_leader + b * 8);
      }
      // unit end: wait for the last P.E, then write this unit's partial state
      if (!warp_wait(pe_done, (g - 1u) & 1u, abort_flag, kErrFwd | 9)) goto done;
      tc_fence_after();
      {
        const int64_t slot = static_cast<int64_t>(mt * p.splits + sp) * 256 + static_cast<int>(rank) * 128 + r;
#pragma unroll 1
        for (int c = 0; c < p.D; c += 32) {
          uint32_t o[32];
          tmem_ld32(trow + Cfg::O_COL + c, o);
          tmem_wait_ld();
          if (n < p.N) store_row32(p.part_acc + slot * p.D, c, p.D, o);
        }
        tc_fence_before();
        named_bar_sync(1, 128);
        if (r == 0) mbar_arrive_cluster_relaxed(o_free_leader);
        if (n < p.N) {
          p.part_m2[slot] = ref;
          p.part_l[slot] = l;
        }
      }
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

// ------------------------------------------------------------------------------------- host
template <bool kBF16, int NS, int KH, int BV, int OW>
static cudaError_t launch_fwd(const FwdMaps& m, const FwdParams& prm, int max_pairs, cudaStream_t st) {
  using Cfg = FwdCfg<kBF16, NS, KH, BV, OW>;
  auto kern = fwd_kernel<kBF16, NS, KH, BV, OW>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_ALLOC);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
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
  return cudaLaunchKernelEx(&cfg, kern, m.h, m.w, m.e, prm);
}

int fwd_vocab_tile(int DP) { return DP <= 128 ? 192 : 128; }
int fwd_o_width(int DP) { return DP <= 128 ? 128 : 256; }

cudaError_t launch_fwd_kernel(bool bf16, int DP, const FwdMaps& maps, const FwdParams& prm, int max_pairs,
                              cudaStream_t st) {
  if (DP <= 128)
    return bf16 ? launch_fwd<true, 3, 2, 192, 128>(maps, prm, max_pairs, st)
                : launch_fwd<false, 3, 2, 192, 128>(maps, prm, max_pairs, st);
  return bf16 ? launch_fwd<true, 3, 2, 128, 256>(maps, prm, max_pairs, st)
              : launch_fwd<false, 3, 2, 128, 256>(maps, prm, max_pairs, st);
}

}  // namespace tc
}  // namespace swvr
