// Packed-weight expert projection for many tokens per expert (prefill): tcgen05 MMAs with
// both operands in shared memory and all 512 TMEM columns as accumulators.
//
// The decode-regime kernel (umma_proj.cuh) decodes each weight tile into TMEM once per token
// chunk of <= 32 (or 128) tokens, so with hundreds of tokens per expert the decode, not the
// tensor core, bounds it. Here a work item is (token chunk of <= 256 tokens of one expert,
// weight pair p), and each weight value is decoded once per 256 tokens:
//   gate/up: pair p = I rows [128p, 128p + 128): MMA tile 0 is gate tile 2p and up tile 2p
//            with interleaved rows (A row r = row r >> 1 of gate (r even) or up (r odd)), MMA
//            tile 1 the same for tiles 2p + 1, so SwiGLU partners sit in neighbouring TMEM
//            lanes; the epilogue writes h = bf16(silu(bf16 g) * bf16 u) as the down pass's
//            activation tiles.
//   down:    pair p = H rows [256p, 256p + 256): MMA tile t is rows 256p + 128t .. + 127
//            (weight tiles 4p + 2t, 4p + 2t + 1); the epilogue writes y = bf16(h Wd^T).
// TMEM: MMA tile t accumulates into columns [256t, 256t + 256) (one column per token).
//
// The K loop runs over 64-value K atoms. Per atom, 8 decode warps (a group; the two groups
// take alternate atoms) turn one quarter block of each of the item's 256 weight rows into the
// BF16 A operand (2 x [128 rows x 128 B], 128-byte-swizzled K-major) in shared memory. The
// producer streams each K block of the item's 4 weight tiles (one 1-D bulk copy per tile:
// a copy costs its SM ~0.3 us up to ~16 KB, so copies must be large) and each activation atom
// ([tokens x 128 B], the layout the dispatch / gate-up epilogue wrote; 32 KB at 256 tokens),
// no multicast. The weight stage is single: every decode warp takes its two quarters of the
// block into registers first and releases the stage, so the next block's copies overlap the
// block's four atoms. One thread issues 2 x 4 MMAs (M = 128, N = chunk tokens rounded to 16,
// K = 16) per atom. Warps: 0-15 decode, 16 producer, 17 MMA, 18-25 epilogue (two per TMEM
// lane quadrant, each taking half of the token columns). Every wait is bounded; on give-up
// the CTA records QK_ERR_TIMEOUT in `status` and leaves its loops.
#pragma once

#include "rowtile.cuh"
#include "umma.cuh"
#include "umma_proj.cuh"

namespace qk {

constexpr int kPTok = 256;  // tokens per chunk of the prefill form (MMA N <= 256)
constexpr int kPDecodeWarps = 16;
constexpr int kPProducerWarp = 16;
constexpr int kPMmaWarp = 17;
constexpr int kPEpilogueWarp0 = 18;
constexpr int kPEpilogueWarps = 8;
constexpr int kPThreads = (kPEpilogueWarp0 + kPEpilogueWarps) * 32;  // 832
constexpr int kPAtomA = 2 * 128 * 128;                                // A operand of one atom: 32 KB
constexpr int kPAtomB = kPTok * 128;                                  // B operand of one atom: 32 KB

// Decode of one weight row's quarter blocks (64 values = one K atom) from a K-block stage of
// its 64-row tile (the tile's whole block, as one bulk copy). Decode group g handles the
// atoms g and g + 2 of every K block, i.e. quarter g of both halves: `load` reads their
// bytes into registers once per K block (so the stage can be refilled while the group
// decodes), `decode<h>` then produces quarter g of half h.
template <QType QT>
struct QuarterRegs;

template <>
struct QuarterRegs<QType::Q6_K> {
  uint32_t w[2][12];  // re-packed codes of sub-blocks 8h + 4g .. + 3 (three words each)
  uint32_t sc[2];     // their int8 sub-scales
  float d;
  __device__ __forceinline__ void load(const uint8_t* tile, int row, int g) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        const uint4 v = lds128(tile + ((6 * h + 3 * g + c) * kTileRows + row) * 16);
        w[h][4 * c] = v.x;
        w[h][4 * c + 1] = v.y;
        w[h][4 * c + 2] = v.z;
        w[h][4 * c + 3] = v.w;
      }
      sc[h] = *reinterpret_cast<const uint32_t*>(tile + (12 * kTileRows + row) * 16 + 8 * h + 4 * g);
    }
    d = f16_to_f32(*reinterpret_cast<const uint16_t*>(tile + HalfTile<QType::Q6_K>::kScaleOff + row * 2));
  }
  __device__ __forceinline__ void clear() {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int i = 0; i < 12; ++i) w[h][i] = 0;
      sc[h] = 0;
    }
    d = 0.f;
  }
  // emit(k0, out[8]): 16 values at K positions k0 .. k0 + 15 of the atom
  template <int h, typename Emit>
  __device__ __forceinline__ void decode(int g, Emit&& emit) const {
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const float ds = __fmul_rn(d, static_cast<float>(static_cast<int8_t>((sc[h] >> (8 * jj)) & 0xffu)));
      const uint32_t w0 = w[h][3 * jj], w1 = w[h][3 * jj + 1], w2 = w[h][3 * jj + 2];
      const uint32_t c3 = ((w0 >> 6) & 0x03030303u) | ((w1 >> 4) & 0x0c0c0c0cu) | ((w2 >> 2) & 0x30303030u);
      uint32_t out[8];
      code4<false, false>(w0 & 0x3f3f3f3fu, ds, 32.f, 0.f, out[0], out[1]);
      code4<false, false>(w1 & 0x3f3f3f3fu, ds, 32.f, 0.f, out[2], out[3]);
      code4<false, false>(w2 & 0x3f3f3f3fu, ds, 32.f, 0.f, out[4], out[5]);
      code4<false, false>(c3, ds, 32.f, 0.f, out[6], out[7]);
      emit(16 * jj, out);
    }
  }
};

template <>
struct QuarterRegs<QType::Q4_K> {
  uint32_t hd[4];     // d | dmin << 16, then the 12 packed scale bytes
  uint32_t w[2][8];   // quant bytes of sub-blocks 4h + 2g and 4h + 2g + 1 (32 bytes)
  __device__ __forceinline__ void load(const uint8_t* tile, int row, int g) {
    const uint4 v = lds128(tile + row * 16);
    hd[0] = v.x;
    hd[1] = v.y;
    hd[2] = v.z;
    hd[3] = v.w;
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint4 u = lds128(tile + ((1 + 4 * h + 2 * g + c) * kTileRows + row) * 16);
        w[h][4 * c] = u.x;
        w[h][4 * c + 1] = u.y;
        w[h][4 * c + 2] = u.z;
        w[h][4 * c + 3] = u.w;
      }
  }
  __device__ __forceinline__ void clear() {
#pragma unroll
    for (int i = 0; i < 4; ++i) hd[i] = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int i = 0; i < 8; ++i) w[h][i] = 0;
  }
  __device__ __forceinline__ int scale_byte(int i) const {
    return static_cast<int>((hd[1 + (i >> 2)] >> (8 * (i & 3))) & 0xffu);
  }
  template <int h, typename Emit>
  __device__ __forceinline__ void decode(int g, Emit&& emit) const {
    const float d = f16_to_f32(static_cast<uint16_t>(hd[0] & 0xffffu));
    const float dmin = f16_to_f32(static_cast<uint16_t>(hd[0] >> 16));
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int j = 4 * h + 2 * g + s;  // sub-block of 32 values (gguf_quant.py:118-135)
      int sc, m;
      if (j < 4) {
        sc = scale_byte(j) & 63;
        m = scale_byte(j + 4) & 63;
      } else {
        sc = (scale_byte(j + 4) & 15) | ((scale_byte(j - 4) >> 6) << 4);
        m = (scale_byte(j + 4) >> 4) | ((scale_byte(j) >> 6) << 4);
      }
      const float ds = __fmul_rn(d, static_cast<float>(sc));
      const float dm = __fmul_rn(dmin, static_cast<float>(m));
#pragma unroll
      for (int half16 = 0; half16 < 2; ++half16) {
        uint32_t out[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t code = (w[h][4 * half16 + i] >> (4 * s)) & 0x0f0f0f0fu;
          code4<false, true>(code, ds, 0.f, dm, out[2 * i], out[2 * i + 1]);
        }
        emit(32 * s + 16 * half16, out);
      }
    }
  }
};

template <>
struct QuarterRegs<QType::Q8_0> {
  uint32_t dw[2];      // FP16 scales of GGUF blocks 4h + 2g, 4h + 2g + 1
  uint32_t w[2][16];   // their 64 codes
  __device__ __forceinline__ void load(const uint8_t* tile, int row, int g) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      dw[h] = *reinterpret_cast<const uint32_t*>(tile + row * 16 + 8 * h + 4 * g);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 v = lds128(tile + ((1 + 8 * h + 4 * g + c) * kTileRows + row) * 16);
        w[h][4 * c] = v.x;
        w[h][4 * c + 1] = v.y;
        w[h][4 * c + 2] = v.z;
        w[h][4 * c + 3] = v.w;
      }
    }
  }
  __device__ __forceinline__ void clear() {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      dw[h] = 0;
#pragma unroll
      for (int i = 0; i < 16; ++i) w[h][i] = 0;
    }
  }
  template <int h, typename Emit>
  __device__ __forceinline__ void decode(int g, Emit&& emit) const {
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const float d = f16_to_f32(static_cast<uint16_t>(dw[h] >> (16 * s)));
#pragma unroll
      for (int half16 = 0; half16 < 2; ++half16) {
        uint32_t out[8];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          code4<false, false>(w[h][8 * s + 4 * half16 + i] ^ 0x80808080u, d, 128.f, 0.f, out[2 * i], out[2 * i + 1]);
        emit(32 * s + 16 * half16, out);
      }
    }
  }
};

template <>
struct QuarterRegs<QType::Q5_K> {
  uint32_t hd[4];     // d | dmin << 16, then the 12 packed scale bytes
  uint32_t qh[8];     // the 32 high-bit bytes
  uint32_t w[2][8];   // nibble bytes of sub-blocks 4h + 2g and 4h + 2g + 1 (32 bytes)
  __device__ __forceinline__ void load(const uint8_t* tile, int row, int g) {
    const uint4 v = lds128(tile + row * 16);
    hd[0] = v.x;
    hd[1] = v.y;
    hd[2] = v.z;
    hd[3] = v.w;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const uint4 u = lds128(tile + ((1 + c) * kTileRows + row) * 16);
      qh[4 * c] = u.x;
      qh[4 * c + 1] = u.y;
      qh[4 * c + 2] = u.z;
      qh[4 * c + 3] = u.w;
    }
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint4 u = lds128(tile + ((3 + 4 * h + 2 * g + c) * kTileRows + row) * 16);
        w[h][4 * c] = u.x;
        w[h][4 * c + 1] = u.y;
        w[h][4 * c + 2] = u.z;
        w[h][4 * c + 3] = u.w;
      }
  }
  __device__ __forceinline__ void clear() {
#pragma unroll
    for (int i = 0; i < 4; ++i) hd[i] = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) qh[i] = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int i = 0; i < 8; ++i) w[h][i] = 0;
  }
  __device__ __forceinline__ int scale_byte(int i) const {
    return static_cast<int>((hd[1 + (i >> 2)] >> (8 * (i & 3))) & 0xffu);
  }
  template <int h, typename Emit>
  __device__ __forceinline__ void decode(int g, Emit&& emit) const {
    const float d = f16_to_f32(static_cast<uint16_t>(hd[0] & 0xffffu));
    const float dmin = f16_to_f32(static_cast<uint16_t>(hd[0] >> 16));
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int j = 4 * h + 2 * g + s;  // sub-block of 32 values (gguf_quant.py:118-151)
      int sc, m;
      if (j < 4) {
        sc = scale_byte(j) & 63;
        m = scale_byte(j + 4) & 63;
      } else {
        sc = (scale_byte(j + 4) & 15) | ((scale_byte(j - 4) >> 6) << 4);
        m = (scale_byte(j + 4) >> 4) | ((scale_byte(j) >> 6) << 4);
      }
      const float ds = __fmul_rn(d, static_cast<float>(sc));
      const float dm = __fmul_rn(dmin, static_cast<float>(m));
#pragma unroll
      for (int half16 = 0; half16 < 2; ++half16) {
        uint32_t out[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int wi = 4 * half16 + i;
          const uint32_t lo = (w[h][wi] >> (4 * s)) & 0x0f0f0f0fu;
          const uint32_t hi = ((qh[wi] >> j) & 0x01010101u) << 4;
          code4<false, true>(lo | hi, ds, 0.f, dm, out[2 * i], out[2 * i + 1]);
        }
        emit(32 * s + 16 * half16, out);
      }
    }
  }
};

template <>
struct QuarterRegs<QType::Q5_1> {
  uint32_t dm[2][2];   // d | m << 16 of GGUF blocks 4h + 2g, 4h + 2g + 1
  uint32_t qh[2][2];   // their high-bit words
  uint32_t w[2][8];    // their nibble bytes
  __device__ __forceinline__ void load(const uint8_t* tile, int row, int g) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint2 a = *reinterpret_cast<const uint2*>(tile + (h * kTileRows + row) * 16 + 8 * g);
      const uint2 b = *reinterpret_cast<const uint2*>(tile + ((2 + h) * kTileRows + row) * 16 + 8 * g);
      dm[h][0] = a.x;
      dm[h][1] = a.y;
      qh[h][0] = b.x;
      qh[h][1] = b.y;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const uint4 u = lds128(tile + ((4 + 4 * h + 2 * g + c) * kTileRows + row) * 16);
        w[h][4 * c] = u.x;
        w[h][4 * c + 1] = u.y;
        w[h][4 * c + 2] = u.z;
        w[h][4 * c + 3] = u.w;
      }
    }
  }
  __device__ __forceinline__ void clear() {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      dm[h][0] = dm[h][1] = qh[h][0] = qh[h][1] = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) w[h][i] = 0;
    }
  }
  template <int h, typename Emit>
  __device__ __forceinline__ void decode(int g, Emit&& emit) const {
#pragma unroll
    for (int s = 0; s < 2; ++s) {  // GGUF block 4h + 2g + s (quant.py:31-55)
      const float d = f16_to_f32(static_cast<uint16_t>(dm[h][s] & 0xffffu));
      const float m = f16_to_f32(static_cast<uint16_t>(dm[h][s] >> 16));
#pragma unroll
      for (int half16 = 0; half16 < 2; ++half16) {
        uint32_t out[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t lo = (w[h][4 * s + i] >> (4 * half16)) & 0x0f0f0f0fu;
          code4<false, true>(lo | HalfTile<QType::Q5_1>::high4(qh[h][s], 16 * half16 + 4 * i), d, 0.f, -m,
                             out[2 * i], out[2 * i + 1]);
        }
        emit(32 * s + 16 * half16, out);
      }
    }
  }
};

template <QType QT>
struct PCfg {
  static constexpr int kTile = HalfTile<QT>::kBytes;   // one 64-row tile of one K block
  static constexpr int kTileStride = kTile + 64;       // neighbouring tiles on other banks
  static constexpr int kStageBytes = 4 * kTileStride;  // one K block of the item's 4 tiles
  static constexpr int kBBufs = QT == QType::Q8_0 ? 2 : 3;
  static constexpr size_t kAOff = 0;
  static constexpr size_t kBOff = kAOff + 2 * kPAtomA;
  static constexpr size_t kRawOff = kBOff + static_cast<size_t>(kBBufs) * kPAtomB;
  static constexpr size_t kBarOff = kRawOff + kStageBytes;
  static constexpr size_t kEpiOff = kBarOff + 256;  // output staging of the 8 epilogue warps
  static constexpr size_t kSmem = 1024 + kEpiOff + kPEpilogueWarps * 512;
  static_assert(kSmem <= 232448, "shared memory of the prefill form");
};

// A operand byte offset of (row, K position) inside one MMA tile's [128 rows x 64] atom.
__device__ __forceinline__ uint32_t a_offset(uint32_t row, uint32_t k) {
  const uint32_t chunk = k >> 3;
  return (row >> 3) * 1024u + (row & 7) * 128u + ((chunk ^ (row & 7)) << 4) + (k & 7) * 2u;
}

template <QType QT, int MODE>
__global__ void __launch_bounds__(kPThreads, 1) umma_prefill_kernel(const UArgs A) {
  using Cfg = PCfg<QT>;
  using QR = QuarterRegs<QT>;
  constexpr int NB = Cfg::kBBufs;
  constexpr int TB = Cfg::kTile;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* abuf = smem + Cfg::kAOff;
  uint8_t* bbuf = smem + Cfg::kBOff;
  uint8_t* raw = smem + Cfg::kRawOff;
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(smem + Cfg::kBarOff);
  uint64_t* raw_empty = raw_full + 1;
  uint64_t* b_full = raw_empty + 1;
  uint64_t* b_empty = b_full + NB;
  uint64_t* a_full = b_empty + NB;
  uint64_t* a_empty = a_full + 2;
  uint64_t* acc_full = a_empty + 2;
  uint64_t* acc_empty = acc_full + 1;
  uint32_t* tmem_sh = reinterpret_cast<uint32_t*>(acc_empty + 1);
  // 512 B of output staging per epilogue warp
  uint16_t* estage = reinterpret_cast<uint16_t*>(smem + Cfg::kEpiOff) + (threadIdx.x / 32 - kPEpilogueWarp0) * 256;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();

  if (threadIdx.x == 0) {
    mbar_init(raw_full, 1);
    mbar_init(raw_empty, kPDecodeWarps);  // every decode warp loads its registers from each stage
    for (int s = 0; s < NB; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&a_full[s], kPDecodeWarps / 2);
      mbar_init(&a_empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, kPEpilogueWarps);
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tmem_sh, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_sh;
  pdl_wait();
  const int n_chunks = *A.n_chunks_p;
  const int n_items = n_chunks * A.items_per_chunk;
  const int n_atoms = 4 * A.nkb;  // K atoms of 64 values per item
  bool ok = true;
  const bool idle = static_cast<int>(blockIdx.x) >= n_items;

  // weight tile w (0..3) of pair p: gate/up -> gate 2p, up 2p, gate 2p+1, up 2p+1;
  // down -> 4p .. 4p + 3. nullptr when the tile lies past the matrix.
  auto tile_ptr = [&](int e, int p, int w, int kb) -> const uint8_t* {
    int rt;
    const uint8_t* base;
    if (MODE == kModeGateUp) {
      rt = 2 * p + (w >> 1);
      base = ((w & 1) ? A.wb : A.wa) + static_cast<int64_t>(e) * A.expert_bytes;
    } else {
      rt = 4 * p + w;
      base = A.wa + static_cast<int64_t>(e) * A.expert_bytes;
    }
    if (rt >= A.tiles64) return nullptr;
    return base + (static_cast<int64_t>(rt) * A.nkb + kb) * TB;
  };

  if (idle) {
  } else if (warp == kPProducerWarp) {
    if (lane == 0) {
      const uint64_t wpol = l2_evict_first_policy(), xpol = l2_evict_last_policy();
      uint32_t kc = 0, ac = 0;  // K-block stages and atoms issued so far
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const int ci = item / A.items_per_chunk, p = item % A.items_per_chunk;
        const ChunkInfo c = chunk_info<MODE>(A, ci);
        const uint8_t* xsrc = A.xt + c.xrow * 512 * A.nkb;
        const uint32_t xatom = static_cast<uint32_t>(c.r16) * 128u;
        for (int kb = 0; kb < A.nkb && ok; ++kb, ++kc) {
          // the item's 4 weight tiles of this K block: one copy each, once every decode warp
          // has taken the previous block into its registers
          if (kc >= 1 && !mbar_wait_bounded(raw_empty, (kc - 1) & 1)) {
            ok = false;
            break;
          }
          const uint8_t* tp[4];
          uint32_t bytes = 0;
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            tp[w] = tile_ptr(c.e, p, w, kb);
            if (tp[w]) bytes += TB;
          }
          mbar_expect_tx(raw_full, bytes);
#pragma unroll
          for (int w = 0; w < 4; ++w)
            if (tp[w]) bulk_g2s_hint(raw + w * Cfg::kTileStride, tp[w], TB, raw_full, wpol);
          for (int a4 = 0; a4 < 4; ++a4, ++ac) {
            const int bsl = ac % NB;
            if (ac >= NB && !mbar_wait_bounded(&b_empty[bsl], ((ac / NB) - 1) & 1)) {
              ok = false;
              break;
            }
            mbar_expect_tx(&b_full[bsl], xatom);
            bulk_g2s_hint(bbuf + static_cast<size_t>(bsl) * kPAtomB,
                          xsrc + static_cast<int64_t>(kb) * c.r16 * 512 + a4 * xatom, xatom, &b_full[bsl], xpol);
          }
        }
      }
      // every copy issued must have landed before the CTA leaves (instant unless another role
      // gave up a wait; bounded otherwise)
      if (kc > 0) mbar_wait_bounded(raw_full, (kc - 1) & 1);
      for (uint32_t t = 0; t < static_cast<uint32_t>(NB) && t < ac; ++t)
        mbar_wait_bounded(&b_full[t], ((ac - t + NB - 1) / NB - 1) & 1);
    }
  } else if (warp == kPMmaWarp) {
    if (lane == 0) {
      uint32_t ac = 0, ic = 0;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++ic) {
        const int ci = item / A.items_per_chunk;
        const ChunkInfo c = chunk_info<MODE>(A, ci);
        const uint32_t idesc = idesc_bf16_m128(static_cast<uint32_t>(c.r16));
        if (ic >= 1 && !mbar_wait_bounded(acc_empty, (ic - 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int at = 0; at < n_atoms; ++at, ++ac) {
          const int ab = ac & 1, bsl = ac % NB;
          if (!mbar_wait_bounded(&a_full[ab], (ac >> 1) & 1) || !mbar_wait_bounded(&b_full[bsl], (ac / NB) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t as = smem_addr(abuf + ab * kPAtomA), bs = smem_addr(bbuf + static_cast<size_t>(bsl) * kPAtomB);
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const uint64_t ad = sdesc_sw128(as + t * (kPAtomA / 2), 1024u);
            const uint64_t bd = sdesc_sw128(bs, 1024u);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              umma_ss(tbase + 256u * t, ad + ks * 2, bd + ks * 2, idesc, (at != 0) || (ks != 0));
          }
          umma_commit(&a_empty[ab]);
          umma_commit(&b_empty[bsl]);
        }
        if (!ok) break;
        umma_commit(acc_full);
      }
    }
  } else if (warp >= kPEpilogueWarp0) {
    const int ew = warp - kPEpilogueWarp0;
    const int q = warp & 3, L = 32 * q + lane;  // TMEM lane quadrant of this warp
    const int half = ew >> 2;                    // token columns [128 half, 128 half + 128)
    uint32_t ic = 0;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++ic) {
      const int ci = item / A.items_per_chunk, p = item % A.items_per_chunk;
      const ChunkInfo c = chunk_info<MODE>(A, ci);
      if (!mbar_wait_bounded(acc_full, ic & 1)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int c_lo = 128 * half, c_hi = min(c.r16, c_lo + 128);
#pragma unroll 1
      for (int t = 0; t < 2; ++t) {
        const uint32_t tcol = tbase + (static_cast<uint32_t>(32 * q) << 16) + 256u * t;
#pragma unroll 1
        for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
          float acc[16];
#pragma unroll
          for (int cg = 0; cg < 2; ++cg) {
            uint32_t v[8];
            tmem_ld8(tcol + c0 + 8 * cg, v);
            tmem_wait_ld();
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) acc[8 * cg + jj] = __uint_as_float(v[jj]);
          }
          if (MODE == kModeGateUp) {
            // lane pair (gate row r, up row r) of weight tile pair (2p + t): the even lane writes
            // tokens c0 .. c0 + 7 of the group, the odd lane c0 + 8 .. c0 + 15. Every lane works
            // on its own token at each step (no divergence, eight independent chains).
            const int R0 = 64 * (2 * p + t) + 16 * q;  // the warp's first row of I
            uint8_t* hbase = A.ht + c.xrow * 512 * A.nkb_out + static_cast<int64_t>(R0 >> 8) * c.r16 * 512;
            swiglu_group16(acc, lane, estage, hbase, c.r16, c0, R0 & 255, R0, A.nrows);
          } else if (!A.yr) {
            const int R0 = 256 * p + 128 * t + 32 * q;  // the warp's 32 consecutive rows of H
#pragma unroll
            for (int g8 = 0; g8 < 2; ++g8) {
              float a8[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) a8[i] = acc[8 * g8 + i];
              store_y8(a8, lane, estage, A.y, c.entry0, c0 + 8 * g8, c.ntok, A.nrows, R0, R0 + 16, false);
            }
          } else {
            const int R = 256 * p + 128 * t + L;  // row of H
            if (R < A.nrows) {
#pragma unroll
              for (int col = 0; col < 16; ++col) {
                if (c0 + col >= c.ntok) break;
                const int64_t orow = c.entry0 + c0 + col;
                if (A.yr) A.yr[static_cast<int64_t>(A.entry_route[orow]) * A.nrows + R] = acc[col];
                else A.y[orow * A.nrows + R] = bf16_bits_rne(acc[col]);
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
    }
  } else {
    // ---- decode warps: group g takes atoms g and g + 2 of every K block (ac % 2 == g) ----
    const int g = warp >> 3, ar = 32 * (warp & 7) + lane;  // A row 0..255 of the atom
    const int t = ar >> 7, r = ar & 127;                   // MMA tile, row inside it
    // weight tile (0..3 of the item) and its row: gate/up interleave gate and up rows
    const int wt = MODE == kModeGateUp ? 2 * t + (r & 1) : 2 * t + (r >> 6);
    const int wrow = MODE == kModeGateUp ? (r >> 1) : (r & 63);
    uint8_t* dst0 = abuf + g * kPAtomA + t * (kPAtomA / 2);
    uint32_t kc = 0, ac = static_cast<uint32_t>(g);  // this group's atoms: g, g + 2, g + 4, ...
    auto store = [&](int k0, const uint32_t(&o)[8]) {
      *reinterpret_cast<uint4*>(dst0 + a_offset(r, k0)) = make_uint4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<uint4*>(dst0 + a_offset(r, k0 + 8)) = make_uint4(o[4], o[5], o[6], o[7]);
    };
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      const int p = item % A.items_per_chunk;
      const int rt = MODE == kModeGateUp ? 2 * p + (wt >> 1) : 4 * p + wt;
      const bool mine = rt < A.tiles64;
      for (int kb = 0; kb < A.nkb && ok; ++kb, ++kc) {
        if (!mbar_wait_bounded(raw_full, kc & 1)) {
          ok = false;
          break;
        }
        QR regs;
        if (mine) regs.load(raw + wt * Cfg::kTileStride, wrow, g);
        else regs.clear();
        __syncwarp();
        if (lane == 0) mbar_arrive(raw_empty);
#pragma unroll
        for (int h = 0; h < 2; ++h, ac += 2) {  // atoms 2h + g of this K block
          if (ac >= 2 && !mbar_wait_bounded(&a_empty[g], ((ac >> 1) - 1) & 1)) {
            ok = false;
            break;
          }
          if (h == 0) regs.template decode<0>(g, store);
          else regs.template decode<1>(g, store);
          fence_proxy_async_smem();  // the generic-proxy stores must be visible to the MMA
          __syncwarp();
          if (lane == 0) mbar_arrive(&a_full[g]);
        }
      }
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
int launch_prefill(const UArgs& A, int grid, cudaStream_t st) {
  using Cfg = PCfg<QT>;
  int rc = allow_smem(reinterpret_cast<const void*>(umma_prefill_kernel<QT, MODE>), Cfg::kSmem);
  if (rc) return rc;
  const cudaError_t e = launch_dependent(umma_prefill_kernel<QT, MODE>, dim3(grid), dim3(kPThreads), Cfg::kSmem, st, A);
  if (e != cudaSuccess) return cuda_error(e, "umma_prefill_kernel");
  count_launch(1);
  return QK_OK;
}

}  // namespace qk
