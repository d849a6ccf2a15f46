// 64-row weight tiles and their half-block decode into BF16 TMEM columns.
//
// Layout of one matrix W[rows, K] (rows zero-padded to a multiple of 64): tiles of 64 rows x
// one 256-value GGUF block, ordered [row tile][k block]. Inside a tile the first 16 * C
// bytes of every row's block are stored as [chunk c][row r][16 B] (C = 13 for Q6_K, C = 9
// for Q4_K); Q6_K then holds the rows' FP16 scale d as [row][2 B]. A decode thread owning
// row r reads chunk c at (c * 64 + r) * 16 - consecutive rows are consecutive 16-byte
// words, so the shared-memory reads of a warp are conflict free.
//
// Each block is decoded as two halves (values 0..127 and 128..255) by two different
// threads; a half needs only its own chunks:
//   Q6_K half h: code chunks 6h .. 6h + 5, the sub-scale chunk 12 (8 bytes of it) and d;
//   Q4_K half h: chunk 0 (d, dmin, packed scales) and quant chunks 1 + 4h .. 4 + 4h.
//
// Q4_K rows keep the GGUF block bytes. Q6_K rows re-pack the 6-bit codes (a lossless bit
// permutation, still 192 bytes per block): sub-block j (values 16j .. 16j + 15, one int8
// sub-scale) is three words W0, W1, W2 at bytes 12j .. 12j + 11, where byte i of Wn holds
// code 4n + i in bits 0..5 and bits 2n..2n+1 of code 12 + i in bits 6..7. Codes 0..11
// then need one AND per four codes, codes 12..15 a shift-and-or of the three words.
// Bytes 192..207 are the int8 sub-scales and the FP16 d follows in the scale plane.
//
// Values: the reference decodes (d * sc) * q (Q6_K) and (d * sc) * q - dmin * m (Q4_K)
// in FP32 and rounds to BF16 (glm53_offload/gguf_quant.py:154-157,171). The products are
// exact in FP32 (d * sc needs at most 18 significant bits, the code 6), so one fused
// multiply-add per element reproduces them (see code4):
//   Q6_K: w = fma(1024 + code, ds, -1056 ds) = (code - 32) ds   (1056 ds is exact);
//   Q4_K: w = fma(1024 + code, ds, -1024 ds) - dmin m.
// The fused form turns a (d * sc) * 0 of negative sign into +0, which no dot product can
// see; kExact (the dequantisation entry points) subtracts before multiplying and so
// reproduces the reference bit for bit, signed zeros included.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace qk {

enum class QType { Q6_K = 14, Q4_K = 12, Q8_0 = 8, Q5_K = 13, Q5_1 = 7 };

constexpr int kTileRows = 64;

// Two codes (bytes 2P and 2P + 1 of `codes`) as FP32 1024 + code, via an FP16 pair.
template <int P>
__device__ __forceinline__ float2 magic1024(uint32_t codes) {
  const uint32_t h2 = __byte_perm(codes, 0x6464u, P == 0 ? 0x5140u : 0x5342u);
  return __half22float2(*reinterpret_cast<const __half2*>(&h2));
}

// Code byte I of `codes` (a value below 128) as the FP32 number 0.5 + code / 256.
template <int I>
__device__ __forceinline__ float half_plus_code(uint32_t codes) {
  return __uint_as_float(__byte_perm(codes, 0x3F000000u, 0x7044u | (I << 8)));
}

// Four codes (bytes of `code`) -> two packed BF16 pairs: w = (code - off) * ds [- dm].
// The fused forms (kExact false) build the code as a float with byte permutes and apply
// the scale in one multiply-add; the offsets below keep every product exact:
//   kDecodeViaHalf: u = 1024 + code via an FP16 pair (one permute per two codes, the
//                   FP16 -> FP32 conversions run on the FMA pipe): w = fma(u, ds, -(1024 + off) ds);
//   otherwise:      f = 0.5 + code / 256 (one permute per code): w = fma(f, 256 ds, -(128 + off) ds).
// Both constants are exact: (1024 + off) and (128 + off) have at most 6 significant bits.
constexpr bool kDecodeViaHalf = true;

template <bool kExact, bool kMin>
__device__ __forceinline__ void code4(uint32_t code, float ds, float off, float dm, uint32_t& lo,
                                      uint32_t& hi) {
  float2 w01, w23;
  if (kExact) {
    const float2 u01 = magic1024<0>(code), u23 = magic1024<1>(code);
    const float2 o = make_float2(-(1024.f + off), -(1024.f + off));
    const float2 s = make_float2(ds, ds);
    w01 = __fmul2_rn(__fadd2_rn(u01, o), s);
    w23 = __fmul2_rn(__fadd2_rn(u23, o), s);
  } else if (kDecodeViaHalf) {
    const float k = __fmul_rn(ds, -(1024.f + off));
    const float2 s2 = make_float2(ds, ds), k2 = make_float2(k, k);
    w01 = __ffma2_rn(magic1024<0>(code), s2, k2);
    w23 = __ffma2_rn(magic1024<1>(code), s2, k2);
  } else {
    const float s256 = __fmul_rn(ds, 256.f), k = __fmul_rn(ds, -(128.f + off));
    const float2 s2 = make_float2(s256, s256), k2 = make_float2(k, k);
    w01 = __ffma2_rn(make_float2(half_plus_code<0>(code), half_plus_code<1>(code)), s2, k2);
    w23 = __ffma2_rn(make_float2(half_plus_code<2>(code), half_plus_code<3>(code)), s2, k2);
  }
  if (kMin) {
    const float2 m = make_float2(-dm, -dm);
    w01 = __fadd2_rn(w01, m);
    w23 = __fadd2_rn(w23, m);
  }
  lo = pack_bf16x2(w01.x, w01.y);
  hi = pack_bf16x2(w23.x, w23.y);
}

__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

template <QType QT>
struct HalfTile;

template <>
struct HalfTile<QType::Q6_K> {
  static constexpr int kBlockBytes = 210;
  static constexpr int kChunks = 13;
  static constexpr int kBytes = kTileRows * kBlockBytes;  // 13440
  static constexpr int kScaleOff = kChunks * kTileRows * 16;

  struct Regs {
    uint32_t w[24];  // re-packed codes of sub-blocks 8h .. 8h + 7
    uint32_t sc[2];  // their int8 sub-scales
    float d;
  };

  // A row that does not exist: decodes to zeros.
  __device__ __forceinline__ static void clear(Regs& r) {
#pragma unroll
    for (int i = 0; i < 24; ++i) r.w[i] = 0;
    r.sc[0] = r.sc[1] = 0;
    r.d = 0.f;
  }

  __device__ __forceinline__ static void load(Regs& r, const uint8_t* tile, int row, int h) {
#pragma unroll
    for (int c = 0; c < 6; ++c) {
      const uint4 v = lds128(tile + ((6 * h + c) * kTileRows + row) * 16);
      r.w[4 * c] = v.x;
      r.w[4 * c + 1] = v.y;
      r.w[4 * c + 2] = v.z;
      r.w[4 * c + 3] = v.w;
    }
    const uint2 s = *reinterpret_cast<const uint2*>(tile + (12 * kTileRows + row) * 16 + 8 * h);
    r.sc[0] = s.x;
    r.sc[1] = s.y;
    r.d = f16_to_f32(*reinterpret_cast<const uint16_t*>(tile + kScaleOff + row * 2));
  }

  // emit(col, regs[8]) receives the 8 packed BF16 pairs of the 16 positions starting at
  // column `col` of the half (column = position / 2 inside the half).
  template <bool kExact, typename Emit>
  __device__ __forceinline__ static void decode(const Regs& r, int h, Emit&& emit) {
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      const int sc = static_cast<int8_t>((r.sc[jj >> 2] >> (8 * (jj & 3))) & 0xffu);
      const float ds = __fmul_rn(r.d, static_cast<float>(sc));
      const uint32_t w0 = r.w[3 * jj], w1 = r.w[3 * jj + 1], w2 = r.w[3 * jj + 2];
      const uint32_t c3 = ((w0 >> 6) & 0x03030303u) | ((w1 >> 4) & 0x0c0c0c0cu) | ((w2 >> 2) & 0x30303030u);
      uint32_t out[8];
      code4<kExact, false>(w0 & 0x3f3f3f3fu, ds, 32.f, 0.f, out[0], out[1]);
      code4<kExact, false>(w1 & 0x3f3f3f3fu, ds, 32.f, 0.f, out[2], out[3]);
      code4<kExact, false>(w2 & 0x3f3f3f3fu, ds, 32.f, 0.f, out[4], out[5]);
      code4<kExact, false>(c3, ds, 32.f, 0.f, out[6], out[7]);
      emit(jj * 8, out);
    }
  }
};

template <>
struct HalfTile<QType::Q4_K> {
  static constexpr int kBlockBytes = 144;
  static constexpr int kChunks = 9;
  static constexpr int kBytes = kTileRows * kBlockBytes;  // 9216

  struct Regs {
    uint32_t hd[4];  // d | dmin << 16, then the 12 packed scale bytes
    uint32_t w[16];  // quant bytes of sub-blocks 4h .. 4h + 3
  };

  // A row that does not exist: decodes to zeros.
  __device__ __forceinline__ static void clear(Regs& r) {
#pragma unroll
    for (int i = 0; i < 4; ++i) r.hd[i] = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) r.w[i] = 0;
  }

  __device__ __forceinline__ static void load(Regs& r, const uint8_t* tile, int row, int h) {
    const uint4 v = lds128(tile + row * 16);
    r.hd[0] = v.x;
    r.hd[1] = v.y;
    r.hd[2] = v.z;
    r.hd[3] = v.w;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 u = lds128(tile + ((1 + 4 * h + c) * kTileRows + row) * 16);
      r.w[4 * c] = u.x;
      r.w[4 * c + 1] = u.y;
      r.w[4 * c + 2] = u.z;
      r.w[4 * c + 3] = u.w;
    }
  }

  __device__ __forceinline__ static int scale_byte(const Regs& r, int i) {
    return static_cast<int>((r.hd[1 + (i >> 2)] >> (8 * (i & 3))) & 0xffu);
  }

  // 6-bit scale and min of sub-block j = 4 h + jj (jj a compile-time index, h the half, which
  // may be a run-time value: the register indices stay constant either way).
  __device__ __forceinline__ static void scales_of(const Regs& r, int h, int jj, int& sc, int& m) {
    const int b0 = scale_byte(r, jj), b4 = scale_byte(r, jj + 4), b8 = scale_byte(r, jj + 8);
    if (h == 0) {
      sc = b0 & 63;
      m = b4 & 63;
    } else {
      sc = (b8 & 15) | ((b0 >> 6) << 4);
      m = (b8 >> 4) | ((b4 >> 6) << 4);
    }
  }

  template <bool kExact, typename Emit>
  __device__ __forceinline__ static void decode(const Regs& r, int h, Emit&& emit) {
    const float d = f16_to_f32(static_cast<uint16_t>(r.hd[0] & 0xffffu));
    const float dmin = f16_to_f32(static_cast<uint16_t>(r.hd[0] >> 16));
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int j = 4 * h + jj;  // sub-block of 32 positions (gguf_quant.py:118-135)
      int sc, m;
      scales_of(r, h, jj, sc, m);
      const float ds = __fmul_rn(d, static_cast<float>(sc));
      const float dm = __fmul_rn(dmin, static_cast<float>(m));
#pragma unroll
      for (int half16 = 0; half16 < 2; ++half16) {
        uint32_t out[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t word = r.w[8 * (jj >> 1) + 4 * half16 + i];
          const uint32_t code = (word >> (4 * (j & 1))) & 0x0f0f0f0fu;
          code4<kExact, true>(code, ds, 0.f, dm, out[2 * i], out[2 * i + 1]);
        }
        emit(jj * 16 + half16 * 8, out);
      }
    }
  }
};

// Q8_0 (gguf_quant.py:111-114: v = f32(d) * q, 32 values per 34-byte block) in super-blocks
// of 256 values = 8 GGUF blocks, 272 bytes per row: chunk 0 holds the 8 FP16 scales, chunks
// 1 .. 16 the 256 int8 codes (16 per chunk). A row whose width is not a multiple of 256 is
// padded with zero blocks (d = 0, codes 0), which decode to zeros.
// Half h: scale bytes 8h .. 8h + 7 of chunk 0 and code chunks 1 + 8h .. 8 + 8h.
template <>
struct HalfTile<QType::Q8_0> {
  static constexpr int kBlockBytes = 272;
  static constexpr int kChunks = 17;
  static constexpr int kBytes = kTileRows * kBlockBytes;  // 17408

  struct Regs {
    uint32_t d[2];   // the 4 FP16 scales of the half
    uint32_t w[32];  // its 128 codes
  };

  __device__ __forceinline__ static void clear(Regs& r) {
    r.d[0] = r.d[1] = 0;
#pragma unroll
    for (int i = 0; i < 32; ++i) r.w[i] = 0;
  }

  __device__ __forceinline__ static void load(Regs& r, const uint8_t* tile, int row, int h) {
    const uint2 s = *reinterpret_cast<const uint2*>(tile + row * 16 + 8 * h);
    r.d[0] = s.x;
    r.d[1] = s.y;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 v = lds128(tile + ((1 + 8 * h + c) * kTileRows + row) * 16);
      r.w[4 * c] = v.x;
      r.w[4 * c + 1] = v.y;
      r.w[4 * c + 2] = v.z;
      r.w[4 * c + 3] = v.w;
    }
  }

  // Codes are signed; flipping their sign bits gives code + 128 in [1, 255], decoded with
  // offset 128: (1024 + code + 128) d - 1152 d = code d, exact in FP32 (19 significant bits).
  template <bool kExact, typename Emit>
  __device__ __forceinline__ static void decode(const Regs& r, int h, Emit&& emit) {
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {  // GGUF block 4h + jj of the super-block
      const float d = f16_to_f32(static_cast<uint16_t>(r.d[jj >> 1] >> (16 * (jj & 1))));
#pragma unroll
      for (int half16 = 0; half16 < 2; ++half16) {
        uint32_t out[8];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          code4<kExact, false>(r.w[8 * jj + 4 * half16 + i] ^ 0x80808080u, d, 128.f, 0.f, out[2 * i], out[2 * i + 1]);
        emit(jj * 16 + half16 * 8, out);
      }
    }
  }
};

// Q5_K (gguf_quant.py:115-157: v = (d * sc) * q - dmin * m, q = low nibble | high bit << 4):
// the GGUF block bytes unchanged, as [chunk][row][16 B] - chunk 0 holds d, dmin and the 12
// packed scale bytes (as Q4_K), chunks 1-2 the 32 high-bit bytes (bit j of byte l is the fifth
// bit of value 32 j + l), chunks 3-10 the 128 nibble bytes (value 32 j + l in byte
// 32 (j / 2) + l, nibble j % 2). Half h: chunk 0, chunks 1-2 and nibble chunks 3 + 4h .. 6 + 4h.
template <>
struct HalfTile<QType::Q5_K> {
  static constexpr int kBlockBytes = 176;
  static constexpr int kChunks = 11;
  static constexpr int kBytes = kTileRows * kBlockBytes;  // 11264

  struct Regs {
    uint32_t hd[4];  // d | dmin << 16, then the 12 packed scale bytes
    uint32_t qh[8];  // the 32 high-bit bytes
    uint32_t w[16];  // nibble bytes of sub-blocks 4h .. 4h + 3
  };

  __device__ __forceinline__ static void clear(Regs& r) {
#pragma unroll
    for (int i = 0; i < 4; ++i) r.hd[i] = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) r.qh[i] = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) r.w[i] = 0;
  }

  __device__ __forceinline__ static void load(Regs& r, const uint8_t* tile, int row, int h) {
    const uint4 v = lds128(tile + row * 16);
    r.hd[0] = v.x;
    r.hd[1] = v.y;
    r.hd[2] = v.z;
    r.hd[3] = v.w;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const uint4 u = lds128(tile + ((1 + c) * kTileRows + row) * 16);
      r.qh[4 * c] = u.x;
      r.qh[4 * c + 1] = u.y;
      r.qh[4 * c + 2] = u.z;
      r.qh[4 * c + 3] = u.w;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 u = lds128(tile + ((3 + 4 * h + c) * kTileRows + row) * 16);
      r.w[4 * c] = u.x;
      r.w[4 * c + 1] = u.y;
      r.w[4 * c + 2] = u.z;
      r.w[4 * c + 3] = u.w;
    }
  }

  __device__ __forceinline__ static int scale_byte(const Regs& r, int i) {
    return static_cast<int>((r.hd[1 + (i >> 2)] >> (8 * (i & 3))) & 0xffu);
  }

  // 6-bit scale and min of sub-block j = 4 h + jj (jj a compile-time index, h the half, which
  // may be a run-time value: the register indices stay constant either way).
  __device__ __forceinline__ static void scales_of(const Regs& r, int h, int jj, int& sc, int& m) {
    const int b0 = scale_byte(r, jj), b4 = scale_byte(r, jj + 4), b8 = scale_byte(r, jj + 8);
    if (h == 0) {
      sc = b0 & 63;
      m = b4 & 63;
    } else {
      sc = (b8 & 15) | ((b0 >> 6) << 4);
      m = (b8 >> 4) | ((b4 >> 6) << 4);
    }
  }

  template <bool kExact, typename Emit>
  __device__ __forceinline__ static void decode(const Regs& r, int h, Emit&& emit) {
    const float d = f16_to_f32(static_cast<uint16_t>(r.hd[0] & 0xffffu));
    const float dmin = f16_to_f32(static_cast<uint16_t>(r.hd[0] >> 16));
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int j = 4 * h + jj;  // sub-block of 32 values
      int sc, m;
      scales_of(r, h, jj, sc, m);
      const float ds = __fmul_rn(d, static_cast<float>(sc));
      const float dm = __fmul_rn(dmin, static_cast<float>(m));
#pragma unroll
      for (int half16 = 0; half16 < 2; ++half16) {
        uint32_t out[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int wi = 4 * half16 + i;  // bytes 4 wi .. 4 wi + 3 of the sub-block's 32
          const uint32_t lo = (r.w[8 * (jj >> 1) + wi] >> (4 * (j & 1))) & 0x0f0f0f0fu;
          const uint32_t hi = ((r.qh[wi] >> j) & 0x01010101u) << 4;
          code4<kExact, true>(lo | hi, ds, 0.f, dm, out[2 * i], out[2 * i + 1]);
        }
        emit(jj * 16 + half16 * 8, out);
      }
    }
  }
};

// Q5_1 (quant.py:31-55: v = d * q + m, q = low nibble | high bit << 4, 32 values per 24-byte
// block) in super-blocks of 256 values = 8 GGUF blocks, 192 bytes per row: chunk h holds the
// (d, m) FP16 pairs of blocks 4h .. 4h + 3, chunk 2 + h their 32-bit high-bit words, chunks
// 4 .. 11 the 16 nibble bytes of blocks 0 .. 7 (value p < 16 in the low nibble of byte p,
// value 16 + p in its high nibble). Blocks past the row's end are zero and decode to zeros.
// Half h: chunks h, 2 + h and 4 + 4h .. 7 + 4h.
template <>
struct HalfTile<QType::Q5_1> {
  static constexpr int kBlockBytes = 192;
  static constexpr int kChunks = 12;
  static constexpr int kBytes = kTileRows * kBlockBytes;  // 12288

  struct Regs {
    uint32_t dm[4];  // d | m << 16 of the half's 4 blocks
    uint32_t qh[4];  // their high-bit words
    uint32_t w[16];  // their nibble bytes
  };

  __device__ __forceinline__ static void clear(Regs& r) {
#pragma unroll
    for (int i = 0; i < 4; ++i) r.dm[i] = r.qh[i] = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) r.w[i] = 0;
  }

  __device__ __forceinline__ static void load(Regs& r, const uint8_t* tile, int row, int h) {
    const uint4 a = lds128(tile + (h * kTileRows + row) * 16);
    const uint4 b = lds128(tile + ((2 + h) * kTileRows + row) * 16);
    r.dm[0] = a.x;
    r.dm[1] = a.y;
    r.dm[2] = a.z;
    r.dm[3] = a.w;
    r.qh[0] = b.x;
    r.qh[1] = b.y;
    r.qh[2] = b.z;
    r.qh[3] = b.w;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 u = lds128(tile + ((4 + 4 * h + c) * kTileRows + row) * 16);
      r.w[4 * c] = u.x;
      r.w[4 * c + 1] = u.y;
      r.w[4 * c + 2] = u.z;
      r.w[4 * c + 3] = u.w;
    }
  }

  // The 4 high bits (bits n .. n + 3 of `qh`) of four codes, one per byte, at bit 4: the
  // multiply spreads bit i of the nibble to bit 8 i + 4 (the partial products do not overlap).
  __device__ __forceinline__ static uint32_t high4(uint32_t qh, int n) {
    return (((qh >> n) & 15u) * 0x02040810u) & 0x10101010u;
  }

  // v = d * q + m: fma(1024 + q, d, -1024 d) is d * q exactly (both factors have at most 11
  // significant bits), then one FP32 addition of m, as the reference rounds it.
  template <bool kExact, typename Emit>
  __device__ __forceinline__ static void decode(const Regs& r, int h, Emit&& emit) {
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {  // GGUF block 4h + jj of the super-block
      const float d = f16_to_f32(static_cast<uint16_t>(r.dm[jj] & 0xffffu));
      const float m = f16_to_f32(static_cast<uint16_t>(r.dm[jj] >> 16));
#pragma unroll
      for (int half16 = 0; half16 < 2; ++half16) {  // values 16 half16 .. + 15 of the block
        uint32_t out[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t lo = (r.w[4 * jj + i] >> (4 * half16)) & 0x0f0f0f0fu;
          code4<kExact, true>(lo | high4(r.qh[jj], 16 * half16 + 4 * i), d, 0.f, -m, out[2 * i], out[2 * i + 1]);
        }
        emit(jj * 16 + half16 * 8, out);
      }
    }
  }
};

}  // namespace qk
