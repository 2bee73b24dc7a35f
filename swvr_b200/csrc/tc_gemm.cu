// Tensor-core (tcgen05) GEMMs of the backward on sm_100a: for one vocabulary chunk,
//   dW_c = dS_c^T . h        (M = chunk rows, N = hidden, K = tokens)    -> gW rows
//   dh  += dS_c   . W_c      (M = tokens, N = hidden, K = chunk rows)    -> fp32 accumulator
// from the dS^T chunk that bwd_scores_kernel wrote.  Both problems share one persistent
// launch (dW tiles first, then dh tiles; each CTA takes tiles round-robin) with 128 x 256
// output tiles, a 4-stage TMA ring of 128B-swizzled tiles, and two TMEM accumulators so the
// epilogue of one tile overlaps the main loop of the next.  The epilogue stages 128-byte
// row slabs in shared memory and writes them with TMA: a store for dW (cast to the W
// dtype) and an element-wise TMA add-reduction into the fp32 dh accumulator, so dh is
// never read back into the SM.  Chunks run in order, so dh's accumulation order is fixed.
//
// Replaces the reference's cuBLAS calls gH += mm_acc(gS, W_c) and gW[v0:v1] = mm_acc(gS^T, h)
// (swvr/chunked.py:146-150).
#include "ptx.cuh"
#include "tc.cuh"

namespace swvr {
namespace tc {

template <int NS>
struct GemmCfg {
  static constexpr int A_BYTES = 128 * 128;  // 128 rows x 64 16-bit elements
  static constexpr int B_BYTES = 256 * 128;  // 4 boxes of 64 rows x 64 elements
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

__device__ __forceinline__ TileInfo decode_tile(const GemmParams& p, int t) {
  TileInfo ti;
  if (t < p.dw_tiles) {
    ti.dw = true;
    ti.mb = t / p.dw_nt;
    ti.nb = t % p.dw_nt;
    ti.kblocks = p.dw_kb;
  } else {
    t -= p.dw_tiles;
    ti.dw = false;
    ti.mb = t / p.dh_nt;
    ti.nb = t % p.dh_nt;
    ti.kblocks = p.dh_kb;
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
  uint64_t* full = bars;
  uint64_t* empty = bars + NS;
  uint64_t* acc_full = bars + 2 * NS;  // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint64_t* spare = acc_empty + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + Cfg::NBAR);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int ntiles = p.dw_tiles + p.dh_tiles;
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
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
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      uint32_t stage = 0, sphase = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const TileInfo ti = decode_tile(p, t);
        for (int kb = 0; kb < ti.kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], sphase ^ 1u, abort_flag, kErrGemm | 1)) goto done;
          mbar_arrive_expect_tx(&full[stage], Cfg::A_BYTES + Cfg::B_BYTES);
          uint8_t* a = smem + Cfg::SMEM_A + stage * Cfg::A_BYTES;
          uint8_t* b = smem + Cfg::SMEM_B + stage * Cfg::B_BYTES;
          if (ti.dw) {
            tma_load_2d(a, &tm_ds_k, &full[stage], kb * 64, ti.mb * 128);
#pragma unroll
            for (int c = 0; c < 4; ++c)
              tma_load_2d(b + c * Cfg::BOX64, &tm_h_mn, &full[stage], ti.nb * 256 + c * 64, kb * 64);
          } else {
#pragma unroll
            for (int c = 0; c < 2; ++c)
              tma_load_2d(a + c * Cfg::BOX64, &tm_ds_mn, &full[stage], ti.mb * 128 + c * 64, kb * 64);
#pragma unroll
            for (int c = 0; c < 4; ++c)
              tma_load_2d(b + c * Cfg::BOX64, &tm_w_mn, &full[stage], ti.nb * 256 + c * 64, p.v_begin + kb * 64);
          }
          if (++stage == NS) {
            stage = 0;
            sphase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      const uint32_t id_dw = idesc_f16(kBF16, 128, 256, false, true);
      const uint32_t id_dh = idesc_f16(kBF16, 128, 256, true, true);
      uint32_t stage = 0, sphase = 0, tc = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++tc) {
        const TileInfo ti = decode_tile(p, t);
        const uint32_t ab = tc & 1u;
        if (!mbar_wait(&acc_empty[ab], ((tc >> 1) & 1u) ^ 1u, abort_flag, kErrGemm | 2)) goto done;
        tc_fence_after();
        const uint32_t dcol = tmem + ab * 256;
        for (int kb = 0; kb < ti.kblocks; ++kb) {
          if (!mbar_wait(&full[stage], sphase, abort_flag, kErrGemm | 3)) goto done;
          tc_fence_after();
          const uint32_t abase = smem_u32(smem + Cfg::SMEM_A + stage * Cfg::A_BYTES);
          const uint32_t bbase = smem_u32(smem + Cfg::SMEM_B + stage * Cfg::B_BYTES);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint64_t bdesc = sdesc_sw128(bbase + ks * 2048, Cfg::BOX64, 1024);
            if (ti.dw)
              umma_ss(dcol, sdesc_sw128(abase + ks * 32, 16, 1024), bdesc, id_dw, (kb | ks) ? 1u : 0u);
            else
              umma_ss(dcol, sdesc_sw128(abase + ks * 2048, Cfg::BOX64, 1024), bdesc, id_dh, (kb | ks) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == NS) {
            stage = 0;
            sphase ^= 1u;
          }
        }
        umma_commit(&acc_full[ab]);
      }
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------------- epilogue warps
    const int r = threadIdx.x - 128;
    const bool leader = (r == 0);
    const uint32_t trow = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    uint32_t tc = 0, sl = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++tc) {
      const TileInfo ti = decode_tile(p, t);
      const uint32_t ab = tc & 1u;
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
        if (leader) tma_store_wait_read<1>();  // the store issued from this slab two steps ago has read it
        named_bar_sync(1, 128);
        stage_row(stg, r, v);
        fence_proxy_async_smem();
        named_bar_sync(1, 128);
        if (leader) {
          if (ti.dw)
            tma_store_2d(&tm_gw, stg, ti.nb * 256 + s * (f16out ? 64 : 32), p.v_begin + ti.mb * 128);
          else
            tma_reduce_add_2d(&tm_dh, stg, ti.nb * 256 + s * 32, ti.mb * 128);
          tma_store_commit();
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[ab]);
    }
    if (leader) tma_store_wait_all<0>();
  }
done:
  tc_fence_before();
  __syncthreads();
  if (*abort_flag) drain_after_abort(warp == 1 && lane == 0, spare);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <bool kBF16, int NS>
static cudaError_t launch(const GemmMaps& m, const GemmParams& prm, int grid, cudaStream_t st) {
  using Cfg = GemmCfg<NS>;
  auto kern = gemm_kernel<kBF16, NS>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_ALLOC);
  if (e != cudaSuccess) return e;
  kern<<<grid, 256, Cfg::SMEM_ALLOC, st>>>(m.ds_k, m.ds_mn, m.h_mn, m.w_mn, m.gw, m.dh, prm);
  return cudaGetLastError();
}

cudaError_t launch_gemm_kernel(bool bf16, const GemmMaps& maps, const GemmParams& prm, int grid, cudaStream_t st) {
  return bf16 ? launch<true, 4>(maps, prm, grid, st) : launch<false, 4>(maps, prm, grid, st);
}

}  // namespace tc
}  // namespace swvr
