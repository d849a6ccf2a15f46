// Packed-weight projection on the 5th-generation tensor core (tcgen05), decode regime.
//
// One persistent CTA per SM, 10 warps:
//   warps 0-7  decode: thread r of warps 4t..4t+3 owns row r of weight tile t (two tiles of
//              128 rows per work item). Per K block it reads its row's packed bytes from the
//              shared-memory stage, decodes 128 values per half block into BF16 and stores
//              them with tcgen05.st into its TMEM lane (the A operand); after the last K
//              block it reads the FP32 accumulators back (tcgen05.ld) for the epilogue.
//   warp 8     producer: one lane streams each K block's two weight tiles and the activation
//              tile (already in the 128-byte-swizzled K-major layout, see xt_offset) into a
//              shared-memory ring with 1-D bulk copies (TMA engine, no multicast).
//   warp 9     MMA: one lane issues tcgen05.mma kind::f16 (M = 128 rows, N = tokens of the
//              chunk, K = 16) with A from TMEM and B from shared memory, D (FP32) in TMEM, and
//              signals completion with tcgen05.commit.
// TMEM (512 columns): A double buffer [0, 256) = 2 x (2 tiles x 64 columns = 128 values),
// D double buffer [256, 512) = 2 x (2 tiles x 64 columns = up to 64 tokens).
// Every wait is bounded; on give-up the CTA records QK_ERR_TIMEOUT in `status`.
#pragma once

#include "rowtile.cuh"
#include "umma.cuh"

namespace qk {

constexpr int kDecodeWarps = 8;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kUmmaThreads = 320;
constexpr int kMaxTok = 64;                  // tokens per chunk (MMA N <= 64)
constexpr int kXtStageBytes = kMaxTok * 512;  // activation tile of one K block
constexpr uint32_t kTmemCols = 512;

enum { kModeGateUp = 0, kModeDown = 1, kModeDense = 2 };

template <QType QT>
struct UCfg {
  static constexpr int kTile = RowTile<QT>::kBytes;
  static constexpr int kWBytes = (2 * kTile + 1023) / 1024 * 1024;
  static constexpr int kStageBytes = kWBytes + kXtStageBytes;
  static constexpr int kStages = (220 * 1024) / kStageBytes;  // 2 (Q6_K), 3 (Q4_K)
  static constexpr size_t kSmem = 1024 + static_cast<size_t>(kStages) * kStageBytes + 256;
};

struct UArgs {
  const uint8_t* wa;       // tiles of gate (gate/up), down, or the dense matrix
  const uint8_t* wb;       // tiles of up (gate/up only)
  int64_t expert_bytes;    // tiled bytes of one expert's matrix
  int nkb;                 // K blocks of 256 values
  int rowtiles;            // 128-row tiles of one expert's matrix
  int pairs;               // work items per token chunk
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

// The (one or two) weight tiles of item pair p: gate/up -> gate row tile p and up row tile p;
// down / dense -> row tiles 2p and 2p + 1 (the second may not exist).
template <int MODE>
__device__ __forceinline__ int item_tiles(const UArgs& A, int e, int p, const uint8_t*& w0,
                                          const uint8_t*& w1, int& rt0) {
  constexpr int TB = 0;
  (void)TB;
  const uint8_t* base = A.wa + static_cast<int64_t>(e) * A.expert_bytes;
  if (MODE == kModeGateUp) {
    rt0 = p;
    w0 = base;
    w1 = A.wb + static_cast<int64_t>(e) * A.expert_bytes;
    return 2;
  }
  rt0 = 2 * p;
  w0 = base;
  w1 = base;
  return (2 * p + 1 < A.rowtiles) ? 2 : 1;
}

// Work item -> (token chunk, tile pair, K-block range).
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
  it.ci = item / A.pairs;
  it.p = item % A.pairs;
  return it;
}

template <QType QT, int MODE>
__global__ void __launch_bounds__(kUmmaThreads, 1) umma_proj_kernel(const UArgs A) {
  using Cfg = UCfg<QT>;
  using RT = RowTile<QT>;
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
  const int n_items = n_chunks * A.pairs * (A.ksplit ? A.nkb : 1);
  if (static_cast<int>(blockIdx.x) >= n_items) return;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDecodeWarps + 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&afull[i], kDecodeWarps);
      mbar_init(&aempty[i], 1);
      mbar_init(&dfull[i], 1);
      mbar_init(&dempty[i], kDecodeWarps);
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
        int rt0;
        const int nt = item_tiles<MODE>(A, c.e, it.p, w0, w1, rt0);
        const int rtb = MODE == kModeGateUp ? rt0 : rt0 + 1;
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
          if (nt == 2) bulk_g2s(st + TB, w1 + (static_cast<int64_t>(rtb) * A.nkb + kb) * TB, TB, &full[s]);
          bulk_g2s(st + Cfg::kWBytes, xsrc + static_cast<int64_t>(kb) * xbytes, xbytes, &full[s]);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      uint32_t sc = 0, ac = 0, ic = 0;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const ItemInfo it = item_info(A, item);
        const ChunkInfo c = chunk_info<MODE>(A, it.ci);
        const uint8_t *w0, *w1;
        int rt0;
        const int nt = item_tiles<MODE>(A, c.e, it.p, w0, w1, rt0);
        const uint32_t idesc = idesc_bf16_m128(static_cast<uint32_t>(c.r16));
        const uint32_t d = ic & 1;
        if (ic >= 2 && !mbar_wait_bounded(&dempty[d], ((ic >> 1) - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = it.kb0; kb < it.kb1 && ok; ++kb, ++sc) {
          const int s = sc % S;
          if (!mbar_wait_bounded(&full[s], (sc / S) & 1)) {
            ok = false;
            break;
          }
          const uint32_t xs = smem_addr(smem + static_cast<size_t>(s) * Cfg::kStageBytes + Cfg::kWBytes);
          for (int h = 0; h < 2; ++h, ++ac) {
            const uint32_t aa = ac & 1;
            if (!mbar_wait_bounded(&afull[aa], (ac >> 1) & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            for (int t = 0; t < nt; ++t) {
#pragma unroll
              for (int ks = 0; ks < 8; ++ks) {
                const uint32_t k = h * 128 + ks * 16;
                const uint64_t desc =
                    sdesc_sw128(xs + (k >> 6) * (static_cast<uint32_t>(c.r16) >> 3) * 1024u + (k & 63) * 2u, 1024u);
                umma_ts(tbase + 256 + d * 128 + t * 64, tbase + aa * 128 + t * 64 + ks * 8, desc, idesc,
                        ((kb - it.kb0) | h | ks) != 0);
              }
            }
            umma_commit(&aempty[aa]);
          }
          umma_commit(&empty[s]);
        }
        if (!ok) break;
        umma_commit(&dfull[d]);
        ++ic;
      }
    }
  } else {
    // ---------------- decode + epilogue warps ----------------
    const int t = warp >> 2, q = warp & 3, row = 32 * q + lane;
    uint32_t sc = 0, ac = 0, ic = 0;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      const ItemInfo it = item_info(A, item);
      const ChunkInfo c = chunk_info<MODE>(A, it.ci);
      const uint8_t *w0, *w1;
      int rt0;
      const int nt = item_tiles<MODE>(A, c.e, it.p, w0, w1, rt0);
      const bool mine = t < nt;
      for (int kb = it.kb0; kb < it.kb1 && ok; ++kb, ++sc) {
        const int s = sc % S;
        if (!mbar_wait_bounded(&full[s], (sc / S) & 1)) {
          ok = false;
          break;
        }
        typename RT::Regs r;
        if (mine) RT::load(r, smem + static_cast<size_t>(s) * Cfg::kStageBytes + t * TB, row);
        // The two half blocks; h is a template constant so the row's words stay in registers.
        auto half = [&](auto hc) {
          constexpr int h = decltype(hc)::value;
          const uint32_t aa = ac & 1;
          if (ac >= 2 && !mbar_wait_bounded(&aempty[aa], ((ac >> 1) - 1) & 1)) {
            ok = false;
            return;
          }
          if (mine) {
            const uint32_t col0 = aa * 128 + t * 64;
            RT::template decode_half<false, h>(r, [&](int col, const uint32_t(&o)[8]) {
              tmem_st8(tmem_addr(tbase, 32 * q, col0 + col), o);
            });
            tmem_wait_st();
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&afull[aa]);
          ++ac;
        };
        half(std::integral_constant<int, 0>{});
        if (ok) half(std::integral_constant<int, 1>{});
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      if (!ok) break;
      // ---------------- epilogue ----------------
      const uint32_t d = ic & 1;
      if (!mbar_wait_bounded(&dfull[d], (ic >> 1) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t dcol = 256 + d * 128;
      if (MODE == kModeGateUp) {
        // warps w and w + 4 share TMEM lanes 32q..; they split the token columns
        const int half = warp >> 2, cols = c.r16 >> 1;
        const int R = rt0 * 128 + row;  // row of h = K index of the down pass
        uint8_t* hbase = A.ht + c.xrow * 512 * A.nkb_out + static_cast<int64_t>(R >> 8) * c.r16 * 512;
        for (int c0 = half * cols; c0 < (half + 1) * cols; c0 += 8) {
          uint32_t g[8], u[8];
          tmem_ld8(tmem_addr(tbase, 32 * q, dcol + c0), g);
          tmem_ld8(tmem_addr(tbase, 32 * q, dcol + 64 + c0), u);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float gb = bf16_round(__uint_as_float(g[j]));
            const float ub = bf16_round(__uint_as_float(u[j]));
            const float act = bf16_round(__fmul_rn(gb, sigmoid_ref(gb)));  // silu, math.py:19-20
            const uint16_t hv = bf16_bits_rne(__fmul_rn(act, ub));
            *reinterpret_cast<uint16_t*>(hbase + xt_offset(c.r16, c0 + j, R & 255)) = hv;
          }
        }
      } else if (mine) {
        const int R = (rt0 + t) * 128 + row;
        for (int c0 = 0; c0 < c.r16; c0 += 8) {
          uint32_t v[8];
          tmem_ld8(tmem_addr(tbase, 32 * q, dcol + t * 64 + c0), v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int col = c0 + j;
            if (col >= c.ntok) break;
            const int64_t orow = c.entry0 + col;
            if (MODE == kModeDown) {
              A.y[orow * A.nrows + R] = bf16_bits_rne(__uint_as_float(v[j]));
            } else if (R < A.nrows) {
              float* o = A.ksplit ? A.out + static_cast<int64_t>(it.kb0) * A.m_dense * A.nrows : A.out;
              o[orow * A.nrows + R] = __uint_as_float(v[j]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dempty[d]);
      ++ic;
    }
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
