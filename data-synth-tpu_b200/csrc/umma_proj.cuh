// Packed-weight projection on the 5th-generation tensor core (tcgen05), decode regime.
//
// Work item: one token chunk (<= kMaxTok routed rows of one expert, or of x) times one
// 128-row MMA tile of the weight matrix, over the item's K blocks. The 128-row A operand
// is two 64-row weight tiles with interleaved rows: TMEM lane L holds row L >> 1 of tile
// L & 1. For gate/up the two tiles are the gate and up rows of the same 64 rows of I, so
// the SwiGLU partners sit in neighbouring lanes; for down / dense they are rows
// 128p .. 128p + 63 and 128p + 64 .. 128p + 127.
//
// One persistent CTA per SM, 25 warps:
//   warps 0-15  decode, in two groups of 8 that take alternate K-block stages (group g =
//               warp / 8 decodes stage counter sc with sc % 2 == g into A buffer g). In a
//               group, warp w decodes half h = (w / 4) % 2 of the block for TMEM lanes
//               32 (w % 4) .. + 31: it reads its row's half block from the shared-memory
//               stage, frees the stage, decodes 128 values into BF16 and stores them with
//               tcgen05.st into its lane (64 columns).
//   warp 16     producer: one lane streams each stage's two weight tiles and the chunk's
//               activation tile (already in the 128-byte-swizzled K-major layout) into a
//               shared-memory ring with 1-D bulk copies (TMA engine, no multicast).
//   warps 17-20 MMA: lane 0 of issuer i issues, per stage, the 4 tcgen05.mma kind::f16
//               (M = 128, N = chunk tokens rounded to 16, K = 16) of K atom i (values
//               64i .. 64i + 63 of the block) with A from TMEM and B from shared memory
//               into its own FP32 accumulator, and signals with tcgen05.commit. One thread
//               issues an MMA only every ~60 cycles whatever N is, so four issuers (one
//               per scheduler) keep the tensor core fed at N = 16.
//   warps 21-24 epilogue: read the four accumulators (tcgen05.ld), release them, add
//               them, and write h = SwiGLU (gate/up), y (down) or the FP32 output (dense).
// TMEM: A buffers [0, 256) (2 x 128 columns = 256 BF16 of K per lane), accumulators
// [256, 512) (2 buffers x 4 issuers x kMaxTok columns). Every wait is bounded; on
// give-up the CTA records QK_ERR_TIMEOUT in `status` and leaves its loops.
#pragma once

#include "rowtile.cuh"
#include "umma.cuh"

namespace qk {

constexpr int kDecodeWarps = 16;
constexpr int kProducerWarp = 16;
constexpr int kMmaWarp0 = 17;
constexpr int kMmaIssuers = 4;  // one per 64-value K atom of a block
constexpr int kEpilogueWarp0 = kMmaWarp0 + kMmaIssuers;
constexpr int kUmmaThreads = (kEpilogueWarp0 + 4) * 32;
constexpr int kMaxTok = 32;                   // tokens per chunk (MMA N <= 32)
constexpr int kXtStageBytes = kMaxTok * 512;  // activation tile of one K block
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kAccCol = 256;

enum { kModeGateUp = 0, kModeDown = 1, kModeDense = 2 };

template <QType QT>
struct UCfg {
  static constexpr int kTile = HalfTile<QT>::kBytes;
  // The second tile starts 64 bytes past a 128-byte boundary, so the two 16-row halves a
  // warp reads (even lanes tile 0, odd lanes tile 1) fall on different banks.
  static constexpr int kTile1 = (kTile + 127) / 128 * 128 + 64;
  static constexpr int kWBytes = (kTile1 + kTile + 1023) / 1024 * 1024;
  static constexpr int kStageBytes = kWBytes + kXtStageBytes;
  static constexpr int kStages = (225 * 1024) / kStageBytes;  // 5 (Q6_K), 6 (Q4_K)
  static constexpr size_t kSmem = 1024 + static_cast<size_t>(kStages) * kStageBytes + 512;
};

struct UArgs {
  const uint8_t* wa;       // tiles of gate (gate/up), down, or the dense matrix
  const uint8_t* wb;       // tiles of up (gate/up only)
  int64_t expert_bytes;    // tiled bytes of one expert's matrix
  int nkb;                 // K blocks of 256 values
  int tiles64;             // 64-row tiles of one expert's matrix
  int items_per_chunk;     // 128-row MMA tiles per token chunk
  const uint8_t* xt;       // activation tiles of this pass
  // chunk tables (MoE) or the dense token count
  const int32_t* n_chunks_p;
  int n_chunks_dense;
  int m_dense;
  const int32_t* chunk_off;  // [n_active + 1]
  const int32_t* row_off;    // [n_active + 1]
  const int32_t* active;
  const int32_t* counts;
  const int32_t* offsets;
  const int32_t* n_active_p;
  // outputs
  uint8_t* ht;       // gate/up: activation tiles of the down pass
  int nkb_out;       // gate/up: K blocks of the down pass
  uint16_t* y;       // down: y [entries, nrows]
  float* out;        // dense: out [M, nrows], or with ksplit the block partials [nkb, M, nrows]
  int nrows;         // output rows of the matrix (I, H or N)
  int ksplit;        // dense: one work item per K block (partial sums, reduced in K order)
  int32_t* status;
};

struct ChunkInfo {
  int e;          // local expert (0 for dense)
  int ntok;       // tokens in the chunk
  int r16;        // ntok rounded up to 16 (MMA N, rows of the activation tile)
  int entry0;     // first entry (MoE) or first row of x (dense)
  int64_t xrow;   // first activation-tile row of the chunk
};

template <int MODE>
__device__ __forceinline__ ChunkInfo chunk_info(const UArgs& A, int ci) {
  ChunkInfo c;
  if (MODE == kModeDense) {
    c.e = 0;
    c.entry0 = kMaxTok * ci;
    c.xrow = kMaxTok * ci;
    c.ntok = min(kMaxTok, A.m_dense - kMaxTok * ci);
  } else {
    int lo = 0, hi = *A.n_active_p;  // largest a with chunk_off[a] <= ci
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (A.chunk_off[mid] <= ci) lo = mid;
      else hi = mid;
    }
    const int ch = ci - A.chunk_off[lo];
    c.e = A.active[lo];
    c.ntok = min(kMaxTok, A.counts[c.e] - kMaxTok * ch);
    c.entry0 = A.offsets[c.e] + kMaxTok * ch;
    c.xrow = A.row_off[lo] + kMaxTok * ch;
  }
  c.r16 = (c.ntok + 15) & ~15;
  return c;
}

// Work item -> (token chunk, MMA tile p, K-block range).
struct ItemInfo {
  int ci, p, kb0, kb1;
};

__device__ __forceinline__ ItemInfo item_info(const UArgs& A, int item) {
  ItemInfo it;
  if (A.ksplit) {
    it.kb0 = item % A.nkb;
    it.kb1 = it.kb0 + 1;
    item /= A.nkb;
  } else {
    it.kb0 = 0;
    it.kb1 = A.nkb;
  }
  it.ci = item / A.items_per_chunk;
  it.p = item % A.items_per_chunk;
  return it;
}

// The two 64-row tiles of MMA tile p: gate/up -> gate and up tile p; down / dense ->
// tiles 2p and 2p + 1 (the second may not exist). Returns the number of tiles.
template <int MODE>
__device__ __forceinline__ int item_tiles(const UArgs& A, int e, int p, const uint8_t*& w0,
                                          const uint8_t*& w1, int& rt0, int& rt1) {
  const uint8_t* base = A.wa + static_cast<int64_t>(e) * A.expert_bytes;
  if (MODE == kModeGateUp) {
    w0 = base;
    w1 = A.wb + static_cast<int64_t>(e) * A.expert_bytes;
    rt0 = rt1 = p;
    return 2;
  }
  w0 = w1 = base;
  rt0 = 2 * p;
  rt1 = 2 * p + 1;
  return rt1 < A.tiles64 ? 2 : 1;
}

template <QType QT, int MODE>
__global__ void __launch_bounds__(kUmmaThreads, 1) umma_proj_kernel(const UArgs A) {
  using Cfg = UCfg<QT>;
  using HT = HalfTile<QT>;
  constexpr int S = Cfg::kStages;
  constexpr int TB = Cfg::kTile;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(S) * Cfg::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* afull = empty + S;
  uint64_t* aempty = afull + 2;
  uint64_t* dfull = aempty + 2;
  uint64_t* dempty = dfull + 2;
  uint32_t* tmem_sh = reinterpret_cast<uint32_t*>(dempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_chunks = MODE == kModeDense ? A.n_chunks_dense : *A.n_chunks_p;
  const int n_items = n_chunks * A.items_per_chunk * (A.ksplit ? A.nkb : 1);
  if (static_cast<int>(blockIdx.x) >= n_items) return;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDecodeWarps / 2 + kMmaIssuers);  // the stage's decode group + the MMA commits
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&afull[i], kDecodeWarps / 2);
      mbar_init(&aempty[i], kMmaIssuers);
      mbar_init(&dfull[i], kMmaIssuers);
      mbar_init(&dempty[i], 4);
    }
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tmem_sh, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_sh;
  bool ok = true;

  if (warp == kProducerWarp) {
    if (lane == 0) {
      uint32_t sc = 0;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const ItemInfo it = item_info(A, item);
        const ChunkInfo c = chunk_info<MODE>(A, it.ci);
        const uint8_t *w0, *w1;
        int rt0, rt1;
        const int nt = item_tiles<MODE>(A, c.e, it.p, w0, w1, rt0, rt1);
        const uint32_t xbytes = static_cast<uint32_t>(c.r16) * 512u;
        const uint8_t* xsrc = A.xt + c.xrow * 512 * A.nkb;
        for (int kb = it.kb0; kb < it.kb1; ++kb, ++sc) {
          const int s = sc % S;
          if (sc >= S && !mbar_wait_bounded(&empty[s], ((sc / S) - 1) & 1)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + static_cast<size_t>(s) * Cfg::kStageBytes;
          mbar_expect_tx(&full[s], static_cast<uint32_t>(TB * nt) + xbytes);
          bulk_g2s(st, w0 + (static_cast<int64_t>(rt0) * A.nkb + kb) * TB, TB, &full[s]);
          if (nt == 2) bulk_g2s(st + Cfg::kTile1, w1 + (static_cast<int64_t>(rt1) * A.nkb + kb) * TB, TB, &full[s]);
          bulk_g2s(st + Cfg::kWBytes, xsrc + static_cast<int64_t>(kb) * xbytes, xbytes, &full[s]);
        }
      }
    }
  } else if (warp >= kMmaWarp0 && warp < kEpilogueWarp0) {
    if (lane == 0) {
      const uint32_t atom_i = static_cast<uint32_t>(warp - kMmaWarp0);
      uint32_t sc = 0, ic = 0;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const ItemInfo it = item_info(A, item);
        const ChunkInfo c = chunk_info<MODE>(A, it.ci);
        const uint32_t idesc = idesc_bf16_m128(static_cast<uint32_t>(c.r16));
        const uint32_t atom = static_cast<uint32_t>(c.r16 >> 3) * 1024u;  // bytes per 64-value K atom
        const uint32_t d = ic & 1;
        const uint32_t dcol = tbase + kAccCol + (d * kMmaIssuers + atom_i) * kMaxTok;
        if (ic >= 2 && !mbar_wait_bounded(&dempty[d], ((ic >> 1) - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = it.kb0; kb < it.kb1; ++kb, ++sc) {
          const int s = sc % S;
          const uint32_t g = sc & 1;
          if (!mbar_wait_bounded(&full[s], (sc / S) & 1) || !mbar_wait_bounded(&afull[g], (sc >> 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t b0 = sdesc_sw128(
              smem_addr(smem + static_cast<size_t>(s) * Cfg::kStageBytes + Cfg::kWBytes + atom_i * atom), 1024u);
          const uint32_t acol = tbase + g * 128 + atom_i * 32;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            umma_ts(dcol, acol + ks * 8, b0 + ks * 2, idesc, (kb != it.kb0) || (ks != 0));
          umma_commit(&aempty[g]);
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&dfull[d]);
        ++ic;
      }
    }
  } else if (warp >= kEpilogueWarp0) {
    // ---------------- epilogue ----------------
    const int q = warp & 3, L = 32 * q + lane;
    uint32_t ic = 0;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++ic) {
      const ItemInfo it = item_info(A, item);
      const ChunkInfo c = chunk_info<MODE>(A, it.ci);
      const uint32_t d = ic & 1;
      if (!mbar_wait_bounded(&dfull[d], (ic >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // Eight token columns at a time: acc = ((D0 + D1) + D2) + D3 over the four issuers'
      // accumulators, then the mode's output for those columns.
      const uint32_t dcol = tbase + (static_cast<uint32_t>(32 * q) << 16) + kAccCol + d * kMmaIssuers * kMaxTok;
      const int t = L & 1, r = L >> 1;
      const int R = MODE == kModeGateUp ? 64 * it.p + r : 128 * it.p + 64 * t + r;
      uint8_t* hbase = MODE == kModeGateUp
                           ? A.ht + c.xrow * 512 * A.nkb_out + static_cast<int64_t>(R >> 8) * c.r16 * 512
                           : nullptr;
      float* obase = MODE == kModeDense
                         ? (A.ksplit ? A.out + static_cast<int64_t>(it.kb0) * A.m_dense * A.nrows : A.out)
                         : nullptr;
#pragma unroll
      for (int cg = 0; cg < kMaxTok / 8; ++cg) {
        if (8 * cg >= c.r16) break;
        uint32_t v[kMmaIssuers][8];
#pragma unroll
        for (int i = 0; i < kMmaIssuers; ++i) tmem_ld8(dcol + i * kMaxTok + 8 * cg, v[i]);
        tmem_wait_ld();
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          acc[j] = __uint_as_float(v[0][j]);
#pragma unroll
          for (int i = 1; i < kMmaIssuers; ++i) acc[j] = __fadd_rn(acc[j], __uint_as_float(v[i][j]));
        }
        if (MODE == kModeGateUp) {
          // lane pair (gate row r, up row r): the even lane takes the first half of the
          // token columns, the odd lane the second; each gets its partner's value by shuffle.
          const int half = c.r16 >> 1;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int col = 8 * cg + j;
            const float other = __shfl_xor_sync(0xffffffffu, acc[j], 1);
            if ((col < half) == (t == 0)) {
              const float gb = bf16_round(t == 0 ? acc[j] : other);
              const float ub = bf16_round(t == 0 ? other : acc[j]);
              const float act = bf16_round(__fmul_rn(gb, sigmoid_ref(gb)));  // silu, math.py:19-20
              *reinterpret_cast<uint16_t*>(hbase + xt_offset(c.r16, col, R & 255)) = bf16_bits_rne(__fmul_rn(act, ub));
            }
          }
        } else if (R < A.nrows) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int col = 8 * cg + j;
            if (col >= c.ntok) break;
            const int64_t orow = c.entry0 + col;
            if (MODE == kModeDown) A.y[orow * A.nrows + R] = bf16_bits_rne(acc[j]);
            else obase[orow * A.nrows + R] = acc[j];
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dempty[d]);
    }
  } else {
    // ---------------- decode warps ----------------
    const int g = warp >> 3, q = warp & 3, L = 32 * q + lane;
    const int t = L & 1, r = L >> 1;
    auto run = [&](auto hc) {
      constexpr int h = decltype(hc)::value;
      uint32_t sc = 0, j = 0;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const ItemInfo it = item_info(A, item);
        const ChunkInfo c = chunk_info<MODE>(A, it.ci);
        const uint8_t *w0, *w1;
        int rt0, rt1;
        const bool mine = t < item_tiles<MODE>(A, c.e, it.p, w0, w1, rt0, rt1);
        for (int kb = it.kb0; kb < it.kb1; ++kb, ++sc) {
          if ((sc & 1) != static_cast<uint32_t>(g)) continue;
          const int s = sc % S;
          if (!mbar_wait_bounded(&full[s], (sc / S) & 1)) {
            ok = false;
            break;
          }
          // Lanes of a missing second tile (odd lanes when the matrix ends inside the MMA
          // tile) decode zeros: tcgen05.st / wait::st are warp-collective, so every lane
          // of the warp must run them.
          typename HT::Regs regs;
          if (mine) HT::template load<h>(regs, smem + static_cast<size_t>(s) * Cfg::kStageBytes + t * Cfg::kTile1, r);
          else HT::clear(regs);
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
          if (j >= 1 && !mbar_wait_bounded(&aempty[g], (j - 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t col0 = tbase + (static_cast<uint32_t>(32 * q) << 16) + g * 128 + h * 64;
          HT::template decode<false, h>(regs, [&](int col, const uint32_t(&o)[8]) { tmem_st8(col0 + col, o); });
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&afull[g]);
          ++j;
        }
      }
    };
    if (((warp >> 2) & 1) == 0) run(std::integral_constant<int, 0>{});
    else run(std::integral_constant<int, 1>{});
  }

  if (!ok && lane == 0 && A.status) atomicExch(A.status, QK_ERR_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

template <QType QT, int MODE>
int launch_umma(const UArgs& A, int grid, cudaStream_t st) {
  using Cfg = UCfg<QT>;
  int rc = allow_smem(reinterpret_cast<const void*>(umma_proj_kernel<QT, MODE>), Cfg::kSmem);
  if (rc) return rc;
  umma_proj_kernel<QT, MODE><<<grid, kUmmaThreads, Cfg::kSmem, st>>>(A);
  QK_LAUNCHED("umma_proj_kernel");
  return QK_OK;
}

}  // namespace qk
