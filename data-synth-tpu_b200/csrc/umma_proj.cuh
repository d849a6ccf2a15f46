// Packed-weight projection on the 5th-generation tensor core (tcgen05), decode regime.
//
// Work item: one token chunk (<= 32 routed rows of one expert, <= 128 in the wide form, or
// up to 32 rows of x) times one 128-row MMA tile of the weight matrix, over the item's K
// blocks. The 128-row A operand
// is two 64-row weight tiles with interleaved rows: TMEM lane L holds row L >> 1 of tile
// L & 1. For gate/up the two tiles are the gate and up rows of the same 64 rows of I, so
// the SwiGLU partners sit in neighbouring lanes; for down / dense they are rows
// 128p .. 128p + 63 and 128p + 64 .. 128p + 127.
//
// One persistent CTA per SM, 25 warps:
//   warps 0-15  decode, in two groups of 8 that take alternate K-block stages (group g =
//               warp / 8 decodes the stages sc with sc % 2 == g, into A buffer sc % 3). In a
//               group, warp w decodes half h = (w / 4) % 2 of the block for TMEM lanes
//               32 (w % 4) .. + 31: it reads its row's half block from the shared-memory
//               weight ring into registers, frees the slot, decodes 128 values into BF16
//               and stores them with tcgen05.st into its lane (64 columns).
//               Each weight slot has a full barrier per group. With an odd number of slots
//               the uses of a slot alternate between the groups, and a group's previous wait
//               on one shared barrier would be two phases back: the copy of the other
//               group's use can still be in flight (copies land out of order), and a parity
//               wait would then take that incomplete phase for its own completed one. (With
//               three A buffers only a three-slot ring reaches that: the A-buffer waits order
//               the other group's use of a five- or seven-slot ring first.) On its own barrier
//               a group waits on every phase in order, whatever the A buffers order.
//   warp 16     producer: one lane issues, per stage, the activation tile (already in the
//               128-byte-swizzled K-major layout) and then the two weight tiles as 1-D bulk
//               copies (TMA engine, no multicast). Issued together they land together: the
//               SM's copy queue is kept deep by the weight stream, and an activation tile
//               requested later would arrive microseconds after the decoded weights.
//               Weight slots are freed by the decode (right after its register load), so
//               the stream runs ahead by the whole weight ring; activation tiles live in a
//               64 KB ring of 8 KB granules (16 tokens x one K block each) until their MMAs
//               complete.
//   warps 17-20 MMA: lane 0 of issuer i issues, per stage, the 4 tcgen05.mma kind::f16
//               (M = 128, N = chunk tokens rounded to 16, K = 16) of K atom i (values
//               64i .. 64i + 63 of the block) with A from TMEM and B from shared memory
//               into its own FP32 accumulator, and signals with tcgen05.commit. One thread
//               issues an MMA only every ~60 cycles (more when the decode warps saturate
//               the schedulers) whatever N is, so four issuers - one per scheduler - share
//               the stage.
//   warps 21-24 epilogue: read the four accumulators (tcgen05.ld), add them, release them,
//               and write h = SwiGLU (gate/up), y (down) or the FP32 output (dense).
// TMEM: A buffers [0, 384) (3 x 128 columns = 256 BF16 of K per lane; three, so a decode
// group never waits for the MMA of the stage it decoded last; each half of a buffer - values
// 0..127 and 128..255 of the block - has its own full/empty barrier pair, so the issuers of
// K atoms 0-1 start when the 4 warps of half 0 are done and half 0's warps reuse the buffer
// as soon as those issuers' MMAs complete), accumulators [384, 512)
// (4 issuers x 32 columns; the wide form: 1 issuer x 128 columns, the epilogue reading them
// 32 columns at a time). Every wait is bounded; on give-up the CTA records QK_ERR_TIMEOUT in
// `status` and leaves its loops.
#pragma once

#include "rowtile.cuh"
#include "umma.cuh"

namespace qk {

// TMEM split (overridable when building: -DQK_UMMA_ISSUERS=.. -DQK_UMMA_ABUF=.. -DQK_UMMA_DBUF=..)
#ifndef QK_UMMA_ISSUERS
#define QK_UMMA_ISSUERS 4
#endif
#ifndef QK_UMMA_ABUF
#define QK_UMMA_ABUF 3
#endif
#ifndef QK_UMMA_DBUF
#define QK_UMMA_DBUF 1
#endif
// Decode order: 0 = load a stage's codes into registers, release the weight slot, then wait
// for the A buffer and decode; 1 = wait for the A buffer, then load and decode in one
// stretch and release the slot after the decode.
#ifndef QK_LATE_RELEASE
#define QK_LATE_RELEASE 0
#endif
#ifndef QK_TMEM_ST32
#define QK_TMEM_ST32 1
#endif
constexpr int kDecodeWarps = 16;
constexpr int kProducerWarp = 16;
constexpr int kMmaWarp0 = 17;
constexpr int kMmaIssuers = QK_UMMA_ISSUERS;  // each takes 16 / kMmaIssuers of a block's 16 K steps
constexpr int kABuffers = QK_UMMA_ABUF;
constexpr int kDBuffers = QK_UMMA_DBUF;
constexpr int kMaxTok = 32;           // tokens per chunk of the narrow (decode) form (MMA N <= 32)
constexpr int kWideTok = 128;         // tokens per chunk of the wide (many tokens per expert) form
constexpr int kXGranule = 16 * 512;   // activation tile of 16 tokens x one K block
constexpr int kXSlots = 8;            // stages that can hold activation granules at once
constexpr uint32_t kTmemCols = 512;

enum { kModeGateUp = 0, kModeDown = 1, kModeDense = 2 };

// The two forms of the pass. Narrow: chunks of <= 32 tokens, kMmaIssuers MMA-issuing warps
// (one per scheduler; small-N MMAs are issue-bound), a 64 KB activation ring. Wide: chunks
// of <= 128 tokens, so an expert's weights are decoded once per 128 tokens instead of once
// per 32, one issuer (an M=128, N=128 MMA keeps the tensor pipe busy for its issue time),
// and a 128 KB activation ring (two stages of 128 tokens).
// The down pass of the narrow form: 2 MMA issuers (one per half block) and two accumulator
// buffers, so the MMAs of the next item do not wait for the epilogue to read the last one
// (an item has only I / 256 K blocks there; 43.3 vs 44.9 us at M = 16, 128 experts).
#ifndef QK_DOWN_ISSUERS
#define QK_DOWN_ISSUERS 2
#endif
#ifndef QK_DOWN_DBUF
#define QK_DOWN_DBUF 2
#endif
template <bool W, int MODE = kModeGateUp>
struct Form {
  static constexpr bool kDown = MODE == kModeDown;
  static constexpr int kTok = W ? kWideTok : kMaxTok;
  static constexpr int kIssuers = W ? 1 : kDown ? QK_DOWN_ISSUERS : kMmaIssuers;
  static constexpr int kXGranules = W ? 16 : 8;
  // TMEM: A buffers of 128 columns, then the accumulators. (Two A and two accumulator
  // buffers for the wide form measured the same as three and one.)
  static constexpr int kABuf = W ? 3 : kABuffers;
  static constexpr int kDBuf = W ? 1 : kDown ? QK_DOWN_DBUF : kDBuffers;
  static constexpr uint32_t kAccCol = kABuf * 128;
  static constexpr int kEpilogueWarp0 = kMmaWarp0 + kIssuers;
  static constexpr int kThreads = (kEpilogueWarp0 + 4) * 32;
  static_assert(16 % kIssuers == 0 && 16 / kIssuers >= 4, "issuers take whole 64-value K atoms");
  static_assert(kABuf * 128 + kDBuf * kIssuers * kTok <= 512, "TMEM columns");
};

template <QType QT, bool W = false>
struct UCfg {
  static constexpr int kTile = HalfTile<QT>::kBytes;
  // The second tile starts 64 bytes past a 128-byte boundary, so the two 16-row halves a
  // warp reads (even lanes tile 0, odd lanes tile 1) fall on different banks.
  static constexpr int kTile1 = (kTile + 127) / 128 * 128 + 64;
  static constexpr int kWStageBytes = (kTile1 + kTile + 127) / 128 * 128;
  // Activation ring (1024-aligned granules at the start) and weight ring. The weight ring
  // gets the rest: at ~2.7 us loaded HBM latency an SM needs ~130 KB of weights in flight
  // to take its share of the HBM bandwidth, besides the two stages being decoded.
  static constexpr int kXBytes = Form<W>::kXGranules * kXGranule;
  static constexpr int kWStages = (223 * 1024 - kXBytes) / kWStageBytes;  // narrow 6 (Q6_K), 8 (Q4_K)
  static constexpr size_t kWOff = kXBytes;
  static constexpr size_t kBarOff = kWOff + static_cast<size_t>(kWStages) * kWStageBytes;
  static constexpr size_t kEpiOff = kBarOff + 512;  // output staging of the 4 epilogue warps
  static constexpr size_t kSmem = 1024 + kEpiOff + 4 * 512;
  static_assert(kSmem <= 232448, "shared memory");
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
  const int4* chunk_rec;     // [n_chunks] {expert, tokens, first entry, first tile row}
  const int32_t* row_off;    // [n_active + 1]
  const int32_t* active;
  const int32_t* counts;
  const int32_t* offsets;
  const int32_t* n_active_p;
  // outputs
  uint8_t* ht;       // gate/up: activation tiles of the down pass
  int nkb_out;       // gate/up: K blocks of the down pass
  uint16_t* y;       // down: y [entries, nrows]
  float* yr;         // down, tensor parallel: FP32 y of each entry's route [B * top_k, nrows]
  const int32_t* entry_route;  // down: route b * top_k + j of each entry
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
    const int4 rec = A.chunk_rec[ci];
    c.e = rec.x;
    c.ntok = rec.y;
    c.entry0 = rec.z;
    c.xrow = rec.w;
  }
  c.r16 = (c.ntok + 15) & ~15;
  return c;
}

// Work item -> (token chunk, MMA tile p, K-block range). The items of one chunk run on
// neighbouring CTAs at the same time; each walks its K blocks starting at a different one
// (block kb0 + (i + p) % n at step i), so they do not all fetch the same activation tile
// from the same L2 lines at once. The FP32 accumulation order over K blocks is the only
// thing that changes.
struct ItemInfo {
  int ci, p, kb0, kb1;
  __device__ __forceinline__ int kblock(int i) const {
    const int n = kb1 - kb0;
    return kb0 + (i + p) % n;
  }
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

// SwiGLU of one 16-token group held by a gate/up lane pair, written as 16-byte chunks of the
// down pass's activation tiles. Lane `lane` of the warp holds, in acc[i], the accumulator of
// token first + i for row r = lane >> 1 of the warp's 16 consecutive I rows (K positions
// k0 .. k0 + 15 of the down pass, k0 a multiple of 16 inside one 256-value block): the gate
// row on even lanes, the up row on odd ones. The pair exchanges values by shuffle; lane t of
// the pair computes h = bf16(bf16(silu(bf16 g)) * bf16 u) (experts.py:103-107,
// math.py:10-20) for tokens 8t .. 8t + 7, all lanes on the same path. The 16 x 16 BF16
// results pass through `stage` (512 B of this warp's shared memory) so that each lane then
// stores one 16-byte chunk (8 K positions of one token): wide stores instead of 2-byte ones,
// which the L2 takes at a fraction of the rate. Rows at or past `rows` (zero-padded tile rows)
// are not written.
__device__ __forceinline__ void swiglu_group16(const float (&acc)[16], int lane, uint16_t* stage, uint8_t* hbase,
                                               int r16, int first, int k0, int row0, int rows) {
  const int t = lane & 1, r = lane >> 1;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float mine = t == 0 ? acc[j] : acc[8 + j];
    const float send = t == 0 ? acc[8 + j] : acc[j];
    const float other = __shfl_xor_sync(0xffffffffu, send, 1);
    const float gb = bf16_round_hw(t == 0 ? mine : other);
    const float ub = bf16_round_hw(t == 0 ? other : mine);
    const float act = bf16_round_hw(__fmul_rn(gb, sigmoid_ref(gb)));
    stage[(8 * t + j) * 16 + r] = bf16_bits_hw(__fmul_rn(act, ub));
  }
  __syncwarp();
  const int T = lane >> 1, c = lane & 1;
  const uint4 v = *reinterpret_cast<const uint4*>(stage + T * 16 + 8 * c);
  if (row0 + 8 * c < rows)
    *reinterpret_cast<uint4*>(hbase + xt_offset(r16, first + T, k0 + 8 * c)) = v;
  __syncwarp();
}

// BF16 y of 8 tokens for the warp's 32 rows, stored as 16-byte chunks of the [entries, rows]
// output. Lane `lane` holds acc[i] = the FP32 result of token first + i for its row
// rowbase[lane] (two runs of 16 consecutive rows: lanes 2i -> run 0 row i, 2i + 1 -> run 1
// row i when `interleaved`; otherwise one run of 32 rows, lane i -> row i). `stage` is 512 B
// of this warp's shared memory. Tokens at or past ntok are not written.
__device__ __forceinline__ void store_y8(const float (&acc)[8], int lane, uint16_t* stage, uint16_t* y, int64_t entry0,
                                         int first, int ntok, int nrows, int row_a, int row_b, bool interleaved) {
  // position of this lane's row inside the 32-row staging line: run 0 then run 1
  const int pos = interleaved ? ((lane & 1) * 16 + (lane >> 1)) : lane;
#pragma unroll
  for (int j = 0; j < 8; ++j) stage[j * 32 + pos] = bf16_bits_hw(acc[j]);
  __syncwarp();
  const int T = lane >> 2, part = lane & 3;  // token, 8-row piece of its 32 rows
  const int row = part < 2 ? row_a + 8 * part : row_b + 8 * (part - 2);
  if (first + T < ntok && row < nrows) {
    const uint4 v = *reinterpret_cast<const uint4*>(stage + T * 32 + 8 * part);
    *reinterpret_cast<uint4*>(y + (entry0 + first + T) * nrows + row) = v;
  }
  __syncwarp();
}

// Phase of stage sc on its group's full barrier wfull[2 (sc % SW) + sc % 2]: the number of
// earlier stages of the same slot and group. With SW even every use of a slot is one group's
// (use u = sc / SW); with SW odd the uses alternate, and the group's own are every other one.
template <int SW>
__device__ __forceinline__ uint32_t wfull_phase(uint32_t sc) {
  return SW % 2 == 0 ? sc / SW : (sc / SW) >> 1;
}

template <QType QT, int MODE, bool W = false>
__global__ void __launch_bounds__(Form<W, MODE>::kThreads, 1) umma_proj_kernel(const UArgs A) {
  using Cfg = UCfg<QT, W>;
  using HT = HalfTile<QT>;
  constexpr int SW = Cfg::kWStages;
  constexpr int NI = Form<W, MODE>::kIssuers;       // MMA-issuing warps
  constexpr int TOK = Form<W, MODE>::kTok;          // tokens per chunk (accumulator columns per issuer)
  constexpr int XG = Form<W, MODE>::kXGranules;     // activation ring granules
  constexpr int EW0 = Form<W, MODE>::kEpilogueWarp0;
  constexpr int AB = Form<W, MODE>::kABuf;          // A buffers
  constexpr int DB = Form<W, MODE>::kDBuf;          // accumulator buffers
  constexpr uint32_t kAccCol = Form<W, MODE>::kAccCol;
  constexpr int TB = Cfg::kTile;
  static_assert((3 * SW + 2 * kXSlots + 4 * AB + 2 * DB) * 8 + kXSlots * 4 + 4 <= 512, "barrier region");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xring = smem;
  uint8_t* wring = smem + Cfg::kWOff;
  // weight slot s: wfull[2 s + g] when the copies of a stage of decode group g have landed
  // (stage sc is group sc % 2's), wempty[s] when its group has taken it into registers
  uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOff);
  uint64_t* wempty = wfull + 2 * SW;
  uint64_t* xfull = wempty + SW;
  uint64_t* xempty = xfull + kXSlots;
  // A buffer b, half h (values 128 h .. 128 h + 127 of the block): afull[2 b + h] when its
  // 4 decode warps have stored it, aempty[2 b + h] when the MMAs reading it have completed.
  uint64_t* afull = xempty + kXSlots;
  uint64_t* aempty = afull + 2 * AB;
  uint64_t* dfull = aempty + 2 * AB;
  uint64_t* dempty = dfull + DB;
  volatile uint32_t* xoff = reinterpret_cast<volatile uint32_t*>(dempty + DB);  // [kXSlots] granule of each stage
  uint32_t* tmem_sh = const_cast<uint32_t*>(xoff + kXSlots);
  // 512 B of output staging per epilogue warp
  uint16_t* estage = reinterpret_cast<uint16_t*>(smem + Cfg::kEpiOff) + (threadIdx.x / 32 - EW0) * 256;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();  // the next pass may be launched now; its CTAs start as these ones leave

  if (threadIdx.x == 0) {
    for (int s = 0; s < SW; ++s) {
      mbar_init(&wfull[2 * s], 1);
      mbar_init(&wfull[2 * s + 1], 1);
      mbar_init(&wempty[s], kDecodeWarps / 2);  // the stage's decode group
    }
    for (int s = 0; s < kXSlots; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], NI);  // the MMA commits
    }
    for (int i = 0; i < AB; ++i) {
      for (int h = 0; h < 2; ++h) {
        mbar_init(&afull[2 * i + h], kDecodeWarps / 4);
        mbar_init(&aempty[2 * i + h], NI >= 2 ? NI / 2 : 1);
      }
    }
    for (int i = 0; i < DB; ++i) {
      mbar_init(&dfull[i], NI);
      mbar_init(&dempty[i], 4);
    }
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tmem_sh, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_sh;
  pdl_wait();  // everything above is this CTA's own set-up; from here on, earlier kernels' data
  const int n_chunks = MODE == kModeDense ? A.n_chunks_dense : *A.n_chunks_p;
  const int n_items = n_chunks * A.items_per_chunk * (A.ksplit ? A.nkb : 1);
  bool ok = true;
  const bool idle = static_cast<int>(blockIdx.x) >= n_items;  // no item for this CTA

  if (idle) {
    // nothing to do: fall through to the teardown
  } else if (warp == kProducerWarp) {
    if (lane == 0) {
      const uint64_t wpol = l2_evict_first_policy(), xpol = l2_evict_last_policy();
      uint32_t sc = 0;
      uint32_t xlo = 0, xused = 0, xhead = 0;  // granule ring: oldest live stage, granules held,
      uint64_t xcnt = 0;                         // next free granule, 8-bit counts per stage slot
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const ItemInfo it = item_info(A, item);
        const ChunkInfo c = chunk_info<MODE>(A, it.ci);
        const uint8_t *w0, *w1;
        int rt0, rt1;
        const int nt = item_tiles<MODE>(A, c.e, it.p, w0, w1, rt0, rt1);
        const uint32_t g = static_cast<uint32_t>(c.r16) / 16;  // granules per activation tile
        const uint32_t xbytes = g * kXGranule;
        const uint8_t* xsrc = A.xt + c.xrow * 512 * A.nkb;
        for (int i = 0; i < it.kb1 - it.kb0 && ok; ++i, ++sc) {
          const int kb = it.kblock(i);
          // activation granules: contiguous, skipping a tail granule too short for the tile
          const uint32_t off = xhead + g > XG ? 0u : xhead;
          const uint32_t need = g + (off == 0u && xhead != 0u ? XG - xhead : 0u);
          while (xused + need > XG || sc - xlo >= kXSlots) {
            if (!mbar_wait_bounded(&xempty[xlo % kXSlots], (xlo / kXSlots) & 1)) {
              ok = false;
              break;
            }
            xused -= static_cast<uint32_t>(xcnt >> (8 * (xlo % kXSlots))) & 255u;
            ++xlo;
          }
          const int s = sc % SW;
          if (!ok || (sc >= SW && !mbar_wait_bounded(&wempty[s], ((sc / SW) - 1) & 1))) {
            ok = false;
            break;
          }
          const uint32_t j = sc % kXSlots;
          xcnt = (xcnt & ~(uint64_t{255} << (8 * j))) | (static_cast<uint64_t>(need) << (8 * j));
          xused += need;
          xhead = (off + g) % XG;
          xoff[j] = off;
          mbar_expect_tx(&xfull[j], xbytes);
          bulk_g2s_hint(xring + off * kXGranule, xsrc + static_cast<int64_t>(kb) * xbytes, xbytes, &xfull[j], xpol);
          uint8_t* st = wring + static_cast<size_t>(s) * Cfg::kWStageBytes;
          uint64_t* wf = &wfull[2 * s + (sc & 1)];
          mbar_expect_tx(wf, static_cast<uint32_t>(TB * nt));
          bulk_g2s_hint(st, w0 + (static_cast<int64_t>(rt0) * A.nkb + kb) * TB, TB, wf, wpol);
          if (nt == 2)
            bulk_g2s_hint(st + Cfg::kTile1, w1 + (static_cast<int64_t>(rt1) * A.nkb + kb) * TB, TB, wf, wpol);
        }
      }
      // Every copy issued must have landed before the CTA leaves: instant when the consumers
      // took them all, and otherwise (another role gave up a wait) a bounded wait for the last
      // phase of each slot, so that no copy writes into the shared memory of a CTA that ended.
      // (Only a slot's last use can be in flight: the one before it was decoded before the
      // slot was refilled.)
      for (uint32_t t = 0; t < SW && t < sc; ++t) {
        const uint32_t last = t + (sc - 1 - t) / SW * SW;
        mbar_wait_bounded(&wfull[2 * t + (last & 1)], wfull_phase<SW>(last) & 1);
      }
      for (uint32_t t = 0; t < kXSlots && t < sc; ++t)
        mbar_wait_bounded(&xfull[t], ((sc - t + kXSlots - 1) / kXSlots - 1) & 1);
    }
  } else if (warp >= kMmaWarp0 && warp < EW0) {
    if (lane == 0) {
      const uint32_t mi = static_cast<uint32_t>(warp - kMmaWarp0);
      uint32_t sc = 0, ic = 0;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const ItemInfo it = item_info(A, item);
        const ChunkInfo c = chunk_info<MODE>(A, it.ci);
        const uint32_t idesc = idesc_bf16_m128(static_cast<uint32_t>(c.r16));
        const uint32_t atom = static_cast<uint32_t>(c.r16 >> 3) * 1024u;  // bytes per 64-value K atom
        const uint32_t d = ic % DB;
        const uint32_t dcol = tbase + kAccCol + (d * NI + mi) * TOK;
        if (ic >= DB && !mbar_wait_bounded(&dempty[d], ((ic / DB) - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int i = 0; i < it.kb1 - it.kb0; ++i, ++sc) {
          const uint32_t j = sc % kXSlots, b = sc % AB;
          // the halves of the block this issuer's K atoms lie in
          constexpr int kAtoms = 16 / NI / 4;
          const uint32_t h0 = (mi * kAtoms) / 2, h1 = (mi * kAtoms + kAtoms - 1) / 2;
          if (!mbar_wait_bounded(&xfull[j], (sc / kXSlots) & 1) || !mbar_wait_bounded(&afull[2 * b + h0], (sc / AB) & 1) ||
              (h1 != h0 && !mbar_wait_bounded(&afull[2 * b + h1], (sc / AB) & 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
          constexpr int kSteps = 16 / NI;  // K steps of 16 values per issuer
          const uint32_t xs = smem_addr(xring + xoff[j] * kXGranule);
          const uint64_t bd = sdesc_sw128(xs + (mi * kSteps / 4) * atom, 1024u);
          const uint32_t acol = tbase + b * 128 + mi * kSteps * 8;
#pragma unroll
          for (int ks = 0; ks < kSteps; ++ks)
            umma_ts(dcol, acol + ks * 8, bd + (((ks >> 2) * atom) >> 4) + (ks & 3) * 2, idesc, (i != 0) || (ks != 0));
          umma_commit(&aempty[2 * b + h0]);
          if (h1 != h0) umma_commit(&aempty[2 * b + h1]);
          umma_commit(&xempty[j]);
        }
        if (!ok) break;
        umma_commit(&dfull[d]);
        ++ic;
      }
    }
  } else if (warp >= EW0) {
    // ---------------- epilogue ----------------
    const int q = warp & 3, L = 32 * q + lane;
    uint32_t ic = 0;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++ic) {
      const ItemInfo it = item_info(A, item);
      const ChunkInfo c = chunk_info<MODE>(A, it.ci);
      const uint32_t d = ic % DB;
      if (!mbar_wait_bounded(&dfull[d], (ic / DB) & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // acc = ((D0 + D1) + D2) + D3 over the issuers' accumulators, in groups of 32 token
      // columns (one group in the narrow form), eight columns at a time; the accumulators are
      // released once the last group is in registers, before its outputs are computed.
      const uint32_t dcol = tbase + (static_cast<uint32_t>(32 * q) << 16) + kAccCol + d * NI * TOK;
      const int t = L & 1, r = L >> 1;
      const int c_end = W ? c.r16 : 1;  // the narrow form has one group (r16 <= 32)
      for (int c0 = 0; c0 < c_end; c0 += 32) {
        const int gcols = W ? min(32, c.r16 - c0) : c.r16;  // a multiple of 16
        float acc[32];
#pragma unroll
        for (int cg = 0; cg < 4; ++cg) {
          if (8 * cg >= gcols) break;
          uint32_t v[NI][8];
#pragma unroll
          for (int i = 0; i < NI; ++i) tmem_ld8(dcol + i * TOK + c0 + 8 * cg, v[i]);
          tmem_wait_ld();
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            float a = __uint_as_float(v[0][jj]);
#pragma unroll
            for (int i = 1; i < NI; ++i) a = __fadd_rn(a, __uint_as_float(v[i][jj]));
            acc[8 * cg + jj] = a;
          }
        }
        if (!W || c0 + 32 >= c.r16) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&dempty[d]);
        }
        if (MODE == kModeGateUp) {
          // lane pair (gate row r, up row r): in each group of 16 token columns the even lane
          // writes the first 8, the odd lane the last 8, every lane on its own token at each
          // step (no divergence); each gets its partner's value by shuffle. Rows past I are
          // zero-padded tile rows and are not written.
          const int R0 = 64 * it.p + 16 * q;  // the warp's first row of I = K index of the down pass
          uint8_t* hbase = A.ht + c.xrow * 512 * A.nkb_out + static_cast<int64_t>(R0 >> 8) * c.r16 * 512;
          float lo[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) lo[i] = acc[i];
          swiglu_group16(lo, lane, estage, hbase, c.r16, c0, R0 & 255, R0, A.nrows);
          if (gcols > 16) {
            float hi[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) hi[i] = acc[16 + i];
            swiglu_group16(hi, lane, estage, hbase, c.r16, c0 + 16, R0 & 255, R0, A.nrows);
          }
        } else if (MODE == kModeDown && !A.yr) {
          // rows 128p + 16q + i (even lanes) and 128p + 64 + 16q + i (odd lanes), 8 tokens at a time
          const int ra = 128 * it.p + 16 * q, rb = ra + 64;
#pragma unroll
          for (int g8 = 0; g8 < 4; ++g8) {
            if (8 * g8 >= gcols) break;
            float a8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) a8[i] = acc[8 * g8 + i];
            store_y8(a8, lane, estage, A.y, c.entry0, c0 + 8 * g8, c.ntok, A.nrows, ra, rb, true);
          }
        } else {
          const int R = 128 * it.p + 64 * t + r;
          if (R < A.nrows) {
            float* obase = MODE == kModeDense
                               ? (A.ksplit ? A.out + static_cast<int64_t>(it.kb0) * A.m_dense * A.nrows : A.out)
                               : nullptr;
#pragma unroll
            for (int col = 0; col < 32; ++col) {
              if (c0 + col >= c.ntok) break;
              const int64_t orow = c.entry0 + c0 + col;
              if (MODE == kModeDown) {
                if (A.yr) A.yr[static_cast<int64_t>(A.entry_route[orow]) * A.nrows + R] = acc[col];
                else A.y[orow * A.nrows + R] = bf16_bits_rne(acc[col]);
              } else {
                obase[orow * A.nrows + R] = acc[col];
              }
            }
          }
        }
      }
    }
  } else {
    // ---------------- decode warps ----------------
    const int g = warp >> 3, q = warp & 3, L = 32 * q + lane;
    const int t = L & 1, r = L >> 1;
    // One copy of the loop for both halves (h a run-time value): a copy per half doubled the
    // decode warps' code, and the instruction-cache misses of that showed as no_instruction stalls.
    auto run = [&](int h) {
      uint32_t sc = 0;
#ifdef QK_STAGGER_NS
      if (g == 1) __nanosleep(QK_STAGGER_NS);  // start the second decode group half a stage later
#endif
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        // The decode needs no chunk metadata: only whether its tile exists.
        const ItemInfo it = item_info(A, item);
        const bool mine = MODE == kModeGateUp || t == 0 || 2 * it.p + 1 < A.tiles64;
        for (int i = 0; i < it.kb1 - it.kb0; ++i, ++sc) {
          if ((sc & 1) != static_cast<uint32_t>(g)) continue;
          const int s = sc % SW;
          if (!mbar_wait_bounded(&wfull[2 * s + g], wfull_phase<SW>(sc) & 1)) {
            ok = false;
            break;
          }
          // Lanes of a missing second tile (odd lanes when the matrix ends inside the MMA
          // tile) decode zeros: tcgen05.st / wait::st are warp-collective, so every lane
          // of the warp must run them.
          const uint32_t b = sc % AB;
#if QK_LATE_RELEASE
          // wait for the A buffer first, then load and decode in one stretch (the shared-memory
          // loads of later sub-blocks overlap the decode of earlier ones); the weight slot is
          // released after the decode
          if (sc >= AB && !mbar_wait_bounded(&aempty[2 * b + h], ((sc / AB) - 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          typename HT::Regs regs;
          if (mine) HT::load(regs, wring + static_cast<size_t>(s) * Cfg::kWStageBytes + t * Cfg::kTile1, r, h);
          else HT::clear(regs);
#else
          typename HT::Regs regs;
          if (mine) HT::load(regs, wring + static_cast<size_t>(s) * Cfg::kWStageBytes + t * Cfg::kTile1, r, h);
          else HT::clear(regs);
          __syncwarp();
          if (lane == 0) mbar_arrive(&wempty[s]);
          if (sc >= AB && !mbar_wait_bounded(&aempty[2 * b + h], ((sc / AB) - 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
#endif
          const uint32_t col0 = tbase + (static_cast<uint32_t>(32 * q) << 16) + b * 128 + h * 64;
#if QK_TMEM_ST32
          // 32 columns per TMEM store: four decode steps land in distinct registers, and one
          // tcgen05.st takes them (the registers of an 8-column store are not free for the next
          // step's results until the store has read them)
          uint32_t sbuf[32];
          HT::template decode<false>(regs, h, [&](int col, const uint32_t(&o)[8]) {
#pragma unroll
            for (int i = 0; i < 8; ++i) sbuf[(col & 31) + i] = o[i];
            if ((col & 31) == 24) tmem_st32(col0 + (col & ~31), sbuf);
          });
#else
          HT::template decode<false>(regs, h, [&](int col, const uint32_t(&o)[8]) { tmem_st8(col0 + col, o); });
#endif
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
#if QK_LATE_RELEASE
            mbar_arrive(&wempty[s]);
#endif
            mbar_arrive(&afull[2 * b + h]);
          }
        }
      }
    };
    run((warp >> 2) & 1);
  }

  if (!ok && lane == 0 && A.status) atomicExch(A.status, QK_ERR_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

template <QType QT, int MODE, bool W = false>
int launch_umma(const UArgs& A, int grid, cudaStream_t st) {
  using Cfg = UCfg<QT, W>;
  int rc = allow_smem(reinterpret_cast<const void*>(umma_proj_kernel<QT, MODE, W>), Cfg::kSmem);
  if (rc) return rc;
  const cudaError_t e = launch_dependent(umma_proj_kernel<QT, MODE, W>, dim3(grid), dim3(Form<W, MODE>::kThreads), Cfg::kSmem,
                                         st, A);
  if (e != cudaSuccess) return cuda_error(e, "umma_proj_kernel");
  count_launch(1);
  return QK_OK;
}

}  // namespace qk
