// Shared pieces of the tile-streaming projection kernels (MoE experts, dense packed GEMM).
//
// Each warp owns a ring of shared-memory stages. Lane 0 fills a stage with 1-D bulk
// copies (cp.async.bulk, TMA engine, no multicast) that complete on the stage's
// mbarrier; the warp waits on the barrier (bounded), decodes the tile into BF16 MMA
// fragments in registers and multiplies it with up to 4 column blocks of 8 activation
// rows (m16n8k16, FP32 accumulate). The stage is refilled only after every lane has
// decoded it (the decode consumes the loaded words, so the shared-memory reads are done).
#pragma once

#include "tiles.cuh"

namespace qk {

constexpr int kWarps = 8;                // warps per CTA of the projection kernels
constexpr int kRingBytes = 226 * 1024;   // shared-memory ring per CTA (one CTA per SM)
constexpr int kChunk = 32;               // activation rows per pass (4 MMA column blocks)

template <QType QT, bool kGateUp>
struct ProjCfg {
  static constexpr int kTile = Tile<QT>::kBytes;
  static constexpr int kStage = kGateUp ? 2 * kTile : kTile;
  static constexpr int kStages = kRingBytes / (kWarps * kStage);
  static constexpr size_t kSmem = static_cast<size_t>(kWarps) * kStages * kStage +
                                  static_cast<size_t>(kWarps) * kStages * 8;
};


// B fragments of 8 consecutive permuted positions starting at `col` for J column blocks.
// kSafe: rows may be unaligned / ragged (K % 8 != 0 or a partial last block): element-wise
// loads, positions >= K read as zero.
template <int J, bool kSafe>
__device__ __forceinline__ void load_b(const uint16_t* const (&rows)[4], int col, int K,
                                       uint4 (&xb)[4]) {
#pragma unroll
  for (int j = 0; j < J; ++j) {
    if (!rows[j]) {
      xb[j] = make_uint4(0, 0, 0, 0);
    } else if (!kSafe) {
      xb[j] = ld_nc_v4(rows[j] + col);
    } else {
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t lo = col + 2 * i < K ? rows[j][col + 2 * i] : 0u;
        const uint32_t hi = col + 2 * i + 1 < K ? rows[j][col + 2 * i + 1] : 0u;
        w[i] = lo | (hi << 16);
      }
      xb[j] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// Decode one stage (a tile pair when kPair) and run the MMAs for J column blocks.
template <QType QT, bool kPair, int J, bool kSafe>
__device__ __forceinline__ void proj_stage(const uint8_t* stage, int lane, int kcol, int K,
                                           const uint16_t* const (&rows)[4],
                                           float (&acc_a)[4][4], float (&acc_b)[4][4]) {
  using T = Tile<QT>;
  const int c = lane & 3;
  typename T::Regs ra, rb;
  T::load(ra, stage, lane);
  if (kPair) T::load(rb, stage + T::kBytes, lane);
  ScaleState<QT> sa, sb;
#pragma unroll
  for (int s2 = 0; s2 < 8; ++s2) {
    uint4 xb[4];
    load_b<J, kSafe>(rows, kcol + T::p0(c, 2 * s2), K, xb);
#pragma unroll
    for (int sub = 0; sub < 2; ++sub) {
      const int s = 2 * s2 + sub;
      sa.update(ra, c, s);
      uint32_t fa[4];
      tile_fragment<QT>(ra, sa, s, fa);
      uint32_t fb[4];
      if (kPair) {
        sb.update(rb, c, s);
        tile_fragment<QT>(rb, sb, s, fb);
      }
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const uint32_t b0 = sub ? xb[j].z : xb[j].x, b1 = sub ? xb[j].w : xb[j].y;
        mma_bf16(acc_a[j], fa, b0, b1);
        if (kPair) mma_bf16(acc_b[j], fb, b0, b1);
      }
    }
  }
}

}  // namespace qk
