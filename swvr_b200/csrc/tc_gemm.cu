// Tensor-core (tcgen05) GEMMs of the backward on sm_100a: for one vocabulary chunk,
//   dW_c = dS_c^T . h        (M = chunk rows, N = hidden, K = tokens)    -> gW rows
//   dh  += dS_c   . W_c      (M = tokens, N = hidden, K = chunk rows)    -> fp32 accumulator
// from the dS^T chunk that bwd_scores_kernel wrote.
//
// 2-SM design: CTA pairs (clusters of 2) compute 256 x 256 output tiles with
// tcgen05.mma.cta_group::2.  Each CTA of a pair stages its own 128 rows of A and its own
// 128-column half of B (128 FLOP per staged byte, against 85 for a single-CTA 128 x 256
// tile).  K-blocks are 128 wide (8 MMAs per pipeline stage): the single MMA-issuing
// thread pays its barrier wait and loop overhead once per 8 MMAs, which the shallow MMA
// issue queue would otherwise expose as tensor-pipe bubbles.  The even CTA (the leader)
// issues every MMA; its commits arrive on the barriers of both CTAs, and both CTAs' TMA
// loads count their bytes on the leader's barrier.  Each CTA's epilogue reads its own 128
// rows from its TMEM and writes them with TMA: a store for dW (cast to the W dtype) and an
// element-wise TMA add-reduction into the fp32 dh accumulator.  Both problems share one
// persistent launch (dW tiles first); chunks run in order, so dh's accumulation order is
// fixed.  The launch may overlap the previous kernel's tail (programmatic dependent launch):
// setup runs at once and the producer waits for the predecessors (pdl_wait) before its
// first dS load.
//
// Replaces the reference's cuBLAS calls gH += mm_acc(gS, W_c) and gW[v0:v1] = mm_acc(gS^T, h)
// (swvr/chunked.py:146-150).
#include <cstdio>
#include <cstdlib>

#include "ptx.cuh"
#include "tc.cuh"

namespace swvr {
namespace tc {

template <int NS>
struct GemmCfg {
  static constexpr int HALF = 128 * 128;     // one 64-wide K half: 128 rows (A) or columns (B)
  static constexpr int A_BYTES = 2 * HALF;   // this CTA's 128 rows x 128 16-bit elements
  static constexpr int B_BYTES = 2 * HALF;   // this CTA's 128 columns x 128 K
  static constexpr int BOX64 = 64 * 128;     // one 64 x 64 box
  static constexpr int STG_BYTES = 128 * 128;
  static constexpr int SMEM_A = 0;
  static constexpr int SMEM_B = NS * A_BYTES;
  static constexpr int SMEM_STG = SMEM_B + NS * B_BYTES;
  static constexpr int SMEM_BAR = SMEM_STG + 2 * STG_BYTES;
  static constexpr int NBAR = 2 * NS + 5;
  static constexpr int SMEM_TOTAL = SMEM_BAR + NBAR * 8 + 16;
  static constexpr int SMEM_ALLOC = SMEM_TOTAL + 1024;
  static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
};

struct TileInfo {
  bool dw;
  int mb, nb, kblocks;
};

// Pair tiles: dW tiles first (mb over 256-row blocks of the chunk), then dh tiles.
__device__ __forceinline__ TileInfo decode_tile(const GemmParams& p, int t) {
  TileInfo ti;
  if (t < p.dw_tiles) {
    ti.dw = true;
    ti.mb = t / p.dw_nt;
    ti.nb = t % p.dw_nt;
    ti.kblocks = (p.dw_kb + 1) / 2;  // 128-wide K-blocks
  } else {
    t -= p.dw_tiles;
    ti.dw = false;
    ti.mb = t / p.dh_nt;
    ti.nb = t % p.dh_nt;
    ti.kblocks = (p.dh_kb + 1) / 2;
  }
  return ti;
}

// Write one thread's 128-byte row into a 128B-swizzled staging slab (TMA SWIZZLE_128B layout).
__device__ __forceinline__ void stage_row(uint8_t* stg, int r, const uint32_t (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    uint4 q = make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    *reinterpret_cast<uint4*>(stg + r * 128 + ((j ^ (r & 7)) << 4)) = q;
  }
}

template <bool kBF16, int NS>
__global__ void __launch_bounds__(256, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_ds_k, const __grid_constant__ CUtensorMap tm_ds_mn,
                const __grid_constant__ CUtensorMap tm_h_mn, const __grid_constant__ CUtensorMap tm_w_mn,
                const __grid_constant__ CUtensorMap tm_gw, const __grid_constant__ CUtensorMap tm_dh,
                const GemmParams p) {
  using Cfg = GemmCfg<NS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::SMEM_BAR);
  uint64_t* full = bars;               // [NS] leader's copy counts both CTAs' bytes
  uint64_t* empty = bars + NS;         // [NS] both CTAs (multicast commit)
  uint64_t* acc_full = bars + 2 * NS;  // [2]  both CTAs (multicast commit)
  uint64_t* acc_empty = acc_full + 2;  // [2]  leader's copy: one arrival per CTA
  uint64_t* spare = acc_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + Cfg::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int ntiles = p.dw_tiles + p.dh_tiles;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2);
    }
    mbar_init(spare, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_ds_k);
    tma_prefetch_desc(&tm_ds_mn);
    tma_prefetch_desc(&tm_h_mn);
    tma_prefetch_desc(&tm_w_mn);
    tma_prefetch_desc(&tm_gw);
    tma_prefetch_desc(&tm_dh);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer's barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  if (threadIdx.x == 0) pdl_trigger();  // the next chunk's score kernel may take SMs as they free up

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer (both CTAs)
      pdl_wait();  // dS of this chunk comes from the kernels before this one
      uint32_t stage = 0, sphase = 0;
      for (int t = pair; t < ntiles; t += npairs) {
        const TileInfo ti = decode_tile(p, t);
        const int row = ti.mb * 256 + static_cast<int>(rank) * 128;
        const int col = ti.nb * 256 + static_cast<int>(rank) * 128;
        for (int kb = 0; kb < ti.kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], sphase ^ 1u, abort_flag, kErrGemm | 1)) goto done;
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * (Cfg::A_BYTES + Cfg::B_BYTES));
          const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
#pragma unroll
          for (int hk = 0; hk < 2; ++hk) {
            const int k0 = (2 * kb + hk) * 64;  // past K the boxes read zero fill
            uint8_t* a = smem + Cfg::SMEM_A + stage * Cfg::A_BYTES + hk * Cfg::HALF;
            uint8_t* b = smem + Cfg::SMEM_B + stage * Cfg::B_BYTES + hk * Cfg::HALF;
            if (ti.dw) {
              tma_load_2d_pair(a, &tm_ds_k, fb, k0, row);
              tma_load_2d_pair(b, &tm_h_mn, fb, col, k0);
              tma_load_2d_pair(b + Cfg::BOX64, &tm_h_mn, fb, col + 64, k0);
            } else {
              tma_load_2d_pair(a, &tm_ds_mn, fb, row, k0);
              tma_load_2d_pair(a + Cfg::BOX64, &tm_ds_mn, fb, row + 64, k0);
              tma_load_2d_pair(b, &tm_w_mn, fb, col, p.v_begin + k0);
              tma_load_2d_pair(b + Cfg::BOX64, &tm_w_mn, fb, col + 64, p.v_begin + k0);
            }
          }
          if (++stage == NS) {
            stage = 0;
            sphase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ------------------------------------------------------------ MMA issuer (leader only)
      const uint32_t id_dw = idesc_f16(kBF16, 256, 256, false, true);
      const uint32_t id_dh = idesc_f16(kBF16, 256, 256, true, true);
      // descriptors of stage 0; a stage / K-half / 16-wide K step adds a byte offset >> 4
      const uint64_t da_k = sdesc_sw128(smem_u32(smem + Cfg::SMEM_A), 16, 1024);           // K-major A (dW)
      const uint64_t da_mn = sdesc_sw128(smem_u32(smem + Cfg::SMEM_A), Cfg::BOX64, 1024);  // MN-major A (dh)
      const uint64_t db_mn = sdesc_sw128(smem_u32(smem + Cfg::SMEM_B), Cfg::BOX64, 1024);  // MN-major B
      uint32_t stage = 0, sphase = 0, tc = 0;
      for (int t = pair; t < ntiles; t += npairs, ++tc) {
        const TileInfo ti = decode_tile(p, t);
        const uint32_t ab = tc & 1u;
        if (!mbar_wait(&acc_empty[ab], ((tc >> 1) & 1u) ^ 1u, abort_flag, kErrGemm | 2)) goto done;
        tc_fence_after();
        const uint32_t dcol = tmem + ab * 256;
        const uint64_t da = ti.dw ? da_k : da_mn;
        const uint32_t id = ti.dw ? id_dw : id_dh;
        const uint32_t a_step = ti.dw ? (32u >> 4) : (2048u >> 4);  // one 16-wide K step of A
        for (int kb = 0; kb < ti.kblocks; ++kb) {
          if (!mbar_wait(&full[stage], sphase, abort_flag, kErrGemm | 3)) goto done;
          const uint64_t so = static_cast<uint64_t>(stage * (Cfg::A_BYTES >> 4));  // A and B stages are equal
#pragma unroll
          for (int k8 = 0; k8 < 8; ++k8) {
            const uint64_t half = static_cast<uint64_t>((k8 >> 2) * (Cfg::HALF >> 4));
            umma2_ss(dcol, da + so + half + (k8 & 3) * a_step, db_mn + so + half + (k8 & 3) * (2048u >> 4), id,
                     (kb | k8) ? 1u : 0u);
          }
          umma2_commit_mc(&empty[stage], 3);
          if (++stage == NS) {
            stage = 0;
            sphase ^= 1u;
          }
        }
        umma2_commit_mc(&acc_full[ab], 3);
      }
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------------- epilogue warps (both CTAs)
    const int r = threadIdx.x - 128;
    const bool ep_leader = (r == 0);
    const uint32_t trow = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    uint32_t tc = 0, sl = 0;
    for (int t = pair; t < ntiles; t += npairs, ++tc) {
      const TileInfo ti = decode_tile(p, t);
      const uint32_t ab = tc & 1u;
      const int row = ti.mb * 256 + static_cast<int>(rank) * 128;
      if (!warp_wait(&acc_full[ab], (tc >> 1) & 1u, abort_flag, kErrGemm | 4)) goto done;
      tc_fence_after();
      const uint32_t acol = trow + ab * 256;
      const bool f16out = ti.dw && !p.gw_f32;
      const int nslab = f16out ? 4 : 8;
#pragma unroll 1
      for (int s = 0; s < nslab; ++s, ++sl) {
        uint32_t v[32];
        if (f16out) {
          uint32_t x0[32], x1[32];
          tmem_ld32(acol + s * 64, x0);
          tmem_ld32(acol + s * 64 + 32, x1);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            v[i] = pack2<kBF16>(__uint_as_float(x0[2 * i]), __uint_as_float(x0[2 * i + 1]));
            v[16 + i] = pack2<kBF16>(__uint_as_float(x1[2 * i]), __uint_as_float(x1[2 * i + 1]));
          }
        } else {
          tmem_ld32(acol + s * 32, v);
          tmem_wait_ld();
        }
        uint8_t* stg = smem + Cfg::SMEM_STG + (sl & 1u) * Cfg::STG_BYTES;
        if (ep_leader) tma_store_wait_read<1>();  // the store issued from this slab two steps ago has read it
        named_bar_sync(1, 128);
        stage_row(stg, r, v);
        fence_proxy_async_smem();
        named_bar_sync(1, 128);
        if (ep_leader) {
          if (ti.dw)
            tma_store_2d(&tm_gw, stg, ti.nb * 256 + s * (f16out ? 64 : 32), p.v_begin + row);
          else
            tma_reduce_add_2d(&tm_dh, stg, ti.nb * 256 + s * 32, row);
          tma_store_commit();
        }
      }
      // every thread of this CTA has read its accumulator rows: release them to the leader
      tc_fence_before();
      named_bar_sync(1, 128);
      if (ep_leader) mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[ab]), 0));
    }
    if (ep_leader) tma_store_wait_all<0>();
  }
done:
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) drain_after_abort_pair(warp == 1 && lane == 0 && leader, spare);
  cluster_sync_all();  // neither CTA releases TMEM / shared memory while its peer may use them
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

template <bool kBF16, int NS>
static cudaError_t launch(const GemmMaps& m, const GemmParams& prm, int max_pairs, bool pdl, cudaStream_t st) {
  using Cfg = GemmCfg<NS>;
  auto kern = gemm_kernel<kBF16, NS>;
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
  const int tiles = prm.dw_tiles + prm.dh_tiles;
  int pairs = std::min(std::min(clusters, max_pairs), tiles);
  if (pairs < 1) pairs = 1;
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  if (pdl) {  // may start while the previous kernel in the stream drains (see pdl_wait in the kernel)
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 2;
  }
  static bool reported = false;
  if (!reported && getenv("SWVR_DEBUG")) {
    fprintf(stderr, "[swvr] gemm_kernel: %d co-resident 2-CTA clusters, launching %d pairs for %d tiles\n", clusters,
            pairs, tiles);
    reported = true;
  }
  return cudaLaunchKernelEx(&cfg, kern, m.ds_k, m.ds_mn, m.h_mn, m.w_mn, m.gw, m.dh, prm);
}

cudaError_t launch_gemm_kernel(bool bf16, const GemmMaps& maps, const GemmParams& prm, int max_pairs, bool pdl,
                               cudaStream_t st) {
  return bf16 ? launch<true, 3>(maps, prm, max_pairs, pdl, st) : launch<false, 3>(maps, prm, max_pairs, pdl, st);
}

}  // namespace tc
}  // namespace swvr
