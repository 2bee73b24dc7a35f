// Host/device declarations shared by the tcgen05 (tensor-core) kernels.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace swvr {
namespace tc {

// ------------------------------------------------------------------ forward
struct FwdParams {
  int N, K, V, D;
  float sc2;  // logit_scale * log2(e)
  const void* bias;
  int bias_dt;
  int MT, VT;             // 256-token pair tiles, vocabulary tiles
  int splits, per, units; // vocabulary splits per token tile, tiles per split, MT * splits
  int gm;                 // unit order: groups of gm token tiles walk the splits split-major
  float* part_m2;         // [units * 256]
  float* part_l;          // [units * 256]
  float* part_acc;        // [units * 256 * D]
};

constexpr int kFwdTokenTile = 256;  // tokens per work unit (a CTA pair, 128 per CTA)

// Work unit u -> (token tile mt, vocabulary split sp).  Consecutive units run at the same time
// on consecutive pairs, so the order decides which W slices are streamed together: groups of
// gm token tiles take the splits one after another (gm = 1: every split of a token tile in a
// row; gm >= MT: one split for all token tiles).  The partial-state slot of a unit is
// mt * splits + sp whatever the order.
__host__ __device__ inline void fwd_unit(const FwdParams& p, int u, int* mt, int* sp) {
  const int gsize = p.gm * p.splits;
  const int grp = u / gsize, r = u % gsize;
  const int rows = min(p.gm, p.MT - grp * p.gm);  // token tiles in this (possibly last, short) group
  *sp = r / rows;
  *mt = grp * p.gm + r % rows;
}

int fwd_vocab_tile(int DP);  // vocabulary rows per tile: 192 (DP <= 128) or 128 (DP 256)
int fwd_o_width(int DP);     // the O MMA's N: 128 or 256; each CTA stages half of it

struct FwdMaps {
  CUtensorMap h;  // h, box {64, 128}
  CUtensorMap w;  // W, box {64, fwd_vocab_tile / 2} (half a vocabulary tile)
  CUtensorMap e;  // E, box {64, fwd_vocab_tile}
};

// Launches clusters of 2 CTAs (at most max_pairs pairs, and no more than can be co-resident).
cudaError_t launch_fwd_kernel(bool bf16, int DP, const FwdMaps& maps, const FwdParams& prm, int max_pairs,
                              cudaStream_t st);

// ------------------------------------------------------------------ backward: scores tile kernel
struct BwdScoresParams {
  int N, K, D;
  int v_begin, v_end;  // this chunk's vocabulary rows
  float scale, sc2;    // logit_scale, logit_scale * log2(e)
  const void* bias;
  int bias_dt;
  const float* lse;    // [N]
  const float* delta;  // [N]
  int NT, VT;          // BN-token tiles, 256-row vocabulary pair tiles of the chunk
  int TS, per_t, units;  // token splits, token tiles per split, VT * TS
  int gv;              // unit order: groups of gv vocabulary tiles walk the token splits split-major
  void* ds;            // dS^T [chunk rows, ld_ds] in the compute dtype, or null (ld_ds >= NT*BN)
  int64_t ld_ds;
  float* part_de;      // [units * 256 * D] or null
  float* part_db;      // [units * 256] or null
  int aux_loads;       // 1: warp 2 loads gO and E, so the W / h stream never waits on their buffers
};

// Work unit u -> (256-row vocabulary tile vt, token split ts).  Consecutive units run at the
// same time on consecutive pairs: groups of gv vocabulary tiles take the token splits one
// after another, so about 74 / gv splits of h and gv W tiles stream together (gv = 1: every
// split of a vocabulary tile in a row, so all of h streams in each round of units).  The
// partial dE / db slot of a unit is vt * TS + ts whatever the order.
__host__ __device__ inline void bwd_unit(const BwdScoresParams& p, int u, int* vt, int* ts) {
  const int gsize = p.gv * p.TS;
  const int grp = u / gsize, r = u % gsize;
  const int rows = min(p.gv, p.VT - grp * p.gv);  // vocabulary tiles in this (possibly last, short) group
  *ts = r / rows;
  *vt = grp * p.gv + r % rows;
}

struct BwdScoresMaps {
  CUtensorMap w;    // W, box {64, 128}
  CUtensorMap h;    // h, box {64, BN / 2} (half a token tile)
  CUtensorMap e;    // E, box {64, 128}
  CUtensorMap gok;  // gO in the compute dtype [Npad, DP], box {64, bwd_dp_chunk(BN) / 2}, 128-byte swizzle
  CUtensorMap gom;  // the same, box {bwd_gom_width(DP), BN}, 64-byte (DP 64) or 128-byte swizzle;
                    // each CTA stages one box of its half of the columns (two for DP 256)
};

// Tokens per score tile (BN): 192 for DP 64 with K >= 1024, else 128 (the environment
// variable SWVR_BWD_TOKEN_TILE = 128 or 192 overrides it where that tile exists).
int bwd_token_tile(int DP, int64_t K);

// Tokens per dP^T chunk: 64 for 192-token tiles (the TMEM left beside two S buffers and
// dE), else the whole tile.
__host__ __device__ constexpr int bwd_dp_chunk(int BN) { return BN == 192 ? 64 : BN; }

// Embedding columns per box of gO as the MN-major dE operand (each CTA stages half the dE
// MMA's N: one box, or two for DP 256).
int bwd_gom_width(int DP);

// Launches clusters of 2 CTAs (at most max_pairs pairs, and no more than can be co-resident).
// pdl: launch with programmatic stream serialization (the previous kernel in the stream is
// one of ours whose reads of dS / the partial slots this kernel's stores wait for).
cudaError_t launch_bwd_scores_kernel(bool bf16, int DP, int BN, const BwdScoresMaps& maps,
                                     const BwdScoresParams& prm, int max_pairs, bool pdl, cudaStream_t st);

// ------------------------------------------------------------------ backward: dW / dh GEMMs
struct GemmParams {
  int dw_tiles, dh_tiles;    // number of 256x256 pair tiles of each problem
  int dw_mt, dw_nt, dw_kb;   // dW: row tiles (chunk rows / 256), column tiles (K / 256), k-blocks (tokens / 64)
  int dh_mt, dh_nt, dh_kb;   // dh: row tiles (tokens / 256), column tiles, k-blocks (chunk rows / 64)
  int v_begin;               // first vocabulary row of the chunk
  int gw_f32;                // dW output is fp32 (else the 16-bit compute dtype)
};

struct GemmMaps {
  CUtensorMap ds_k;   // dS^T as a K-major A operand (dW), box {64, 128}
  CUtensorMap ds_mn;  // dS^T as an MN-major A operand (dh), box {64, 64}
  CUtensorMap h_mn;   // h as an MN-major B operand (dW), box {64, 64}
  CUtensorMap w_mn;   // W as an MN-major B operand (dh), box {64, 64}
  CUtensorMap gw;     // dW output (TMA store), box {64 or 32, 128}
  CUtensorMap dh;     // fp32 dh accumulator (TMA reduce-add), box {32, 128}
};

// Launches clusters of 2 CTAs (at most max_pairs pairs, and no more than can be co-resident).
cudaError_t launch_gemm_kernel(bool bf16, const GemmMaps& maps, const GemmParams& prm, int max_pairs, bool pdl,
                               cudaStream_t st);

}  // namespace tc
}  // namespace swvr
