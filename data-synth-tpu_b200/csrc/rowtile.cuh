// 128-row weight tiles and their thread-per-row decode into BF16 TMEM columns.
//
// Layout of one matrix W[rows, K] (rows zero-padded to a multiple of 128): tiles of 128
// rows x one 256-value GGUF block, ordered [row tile][k block]. Inside a tile the first
// 16 * C bytes of every row's block are stored as [chunk c][row r][16 B] (C = 13 for Q6_K,
// C = 9 for Q4_K); Q6_K then holds the rows' FP16 scale d as [row][2 B]. Thread r of the
// decode warps reads chunk c of its row at (c * 128 + r) * 16 - consecutive rows are
// consecutive 16-byte words, so the shared-memory reads are conflict free - and decodes
// the row in natural K order.
//
// Q4_K rows keep the GGUF block bytes. Q6_K rows re-pack the 6-bit codes (a lossless bit
// permutation, still 192 bytes per block): sub-block j (values 16j .. 16j + 15, one int8
// sub-scale) is three words W0, W1, W2 at bytes 12j .. 12j + 11, where byte i of Wn holds
// code 4n + i in bits 0..5 and bits 2m..2m+1 of code 12 + i in bits 6..7 (m = n). Codes
// 0..11 then need one AND per four codes, codes 12..15 a shift-and-or of the three words.
// Bytes 192..207 are the int8 sub-scales and the FP16 d follows in the scale plane.
//
// Values: the reference decodes (d * sc) * q (Q6_K) and (d * sc) * q - dmin * m (Q4_K)
// in FP32 and rounds to BF16 (glm53_offload/gguf_quant.py:154-157,171). The products are
// exact in FP32, so one fused multiply-add per element reproduces them:
//   code -> FP16 1024 + code (byte permute, two codes per instruction) -> FP32;
//   Q6_K: w = fma(v, ds, -1056 ds) = (code - 32) ds (1056 ds is exact: 33 ds needs <= 24 bits);
//   Q4_K: w = fma(v, ds, -1024 ds) - dmin m.
// The fused form turns a (d * sc) * 0 of negative sign into +0, which no dot product can
// see; kExact (the dequantisation entry points) subtracts before multiplying and so
// reproduces the reference bit for bit, signed zeros included.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace qk {

enum class QType { Q6_K = 14, Q4_K = 12 };

// Two codes (bytes 2P and 2P + 1 of `codes`) as FP32 1024 + code, via an FP16 pair.
template <int P>
__device__ __forceinline__ float2 magic1024(uint32_t codes) {
  const uint32_t h2 = __byte_perm(codes, 0x6464u, P == 0 ? 0x5140u : 0x5342u);
  return __half22float2(*reinterpret_cast<const __half2*>(&h2));
}

// Four codes (bytes of `code`) -> two packed BF16 pairs: w = (code - off) * ds [- dm].
template <bool kExact, bool kMin>
__device__ __forceinline__ void code4(uint32_t code, float ds, float nk, float off, float dm,
                                      uint32_t& lo, uint32_t& hi) {
  const float2 u01 = magic1024<0>(code), u23 = magic1024<1>(code);
  const float2 s = make_float2(ds, ds);
  float2 w01, w23;
  if (kExact) {
    const float2 o = make_float2(-off, -off);
    w01 = __fmul2_rn(__fadd2_rn(u01, o), s);
    w23 = __fmul2_rn(__fadd2_rn(u23, o), s);
  } else {
    const float2 k = make_float2(nk, nk);
    w01 = __ffma2_rn(u01, s, k);
    w23 = __ffma2_rn(u23, s, k);
  }
  if (kMin) {
    const float2 m = make_float2(-dm, -dm);
    w01 = __fadd2_rn(w01, m);
    w23 = __fadd2_rn(w23, m);
  }
  lo = pack_bf16x2(w01.x, w01.y);
  hi = pack_bf16x2(w23.x, w23.y);
}

template <QType QT>
struct RowTile;

template <>
struct RowTile<QType::Q6_K> {
  static constexpr int kBlockBytes = 210;
  static constexpr int kChunks = 13;
  static constexpr int kBytes = 128 * kBlockBytes;  // 26880

  struct Regs {
    uint32_t w[52];  // block bytes 0..207: re-packed codes (words 0..47), sub-scales (48..51)
    float d;
  };

  __device__ __forceinline__ static void load(Regs& r, const uint8_t* tile, int row) {
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      const uint4 v = *reinterpret_cast<const uint4*>(tile + (c * 128 + row) * 16);
      r.w[4 * c] = v.x;
      r.w[4 * c + 1] = v.y;
      r.w[4 * c + 2] = v.z;
      r.w[4 * c + 3] = v.w;
    }
    r.d = f16_to_f32(*reinterpret_cast<const uint16_t*>(tile + kChunks * 128 * 16 + row * 2));
  }

  // Decode positions 128 h .. 128 h + 127 of the block (h compile-time, so the word
  // indices are constants and the row stays in registers); emit(col, regs[8]) receives the
  // 8 packed BF16 pairs of the 16 positions starting at column `col` (= position / 2
  // inside the half).
  template <bool kExact, int h, typename Emit>
  __device__ __forceinline__ static void decode_half(const Regs& r, Emit&& emit) {
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) {
      const int j = 8 * h + jj;  // sub-block of 16 positions
      const int sc = static_cast<int8_t>((r.w[48 + (j >> 2)] >> (8 * (j & 3))) & 0xffu);
      const float ds = __fmul_rn(r.d, static_cast<float>(sc));
      const float nk = __fmul_rn(ds, -1056.f);
      const uint32_t w0 = r.w[3 * j], w1 = r.w[3 * j + 1], w2 = r.w[3 * j + 2];
      const uint32_t c3 = ((w0 >> 6) & 0x03030303u) | ((w1 >> 4) & 0x0c0c0c0cu) | ((w2 >> 2) & 0x30303030u);
      uint32_t out[8];
      code4<kExact, false>(w0 & 0x3f3f3f3fu, ds, nk, 1056.f, 0.f, out[0], out[1]);
      code4<kExact, false>(w1 & 0x3f3f3f3fu, ds, nk, 1056.f, 0.f, out[2], out[3]);
      code4<kExact, false>(w2 & 0x3f3f3f3fu, ds, nk, 1056.f, 0.f, out[4], out[5]);
      code4<kExact, false>(c3, ds, nk, 1056.f, 0.f, out[6], out[7]);
      emit(jj * 8, out);
    }
  }
};

template <>
struct RowTile<QType::Q4_K> {
  static constexpr int kBlockBytes = 144;
  static constexpr int kChunks = 9;
  static constexpr int kBytes = 128 * kBlockBytes;  // 18432

  struct Regs {
    uint32_t w[36];  // d | dmin << 16 (word 0), 12 scale bytes (1..3), qs (4..35)
  };

  __device__ __forceinline__ static void load(Regs& r, const uint8_t* tile, int row) {
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
      const uint4 v = *reinterpret_cast<const uint4*>(tile + (c * 128 + row) * 16);
      r.w[4 * c] = v.x;
      r.w[4 * c + 1] = v.y;
      r.w[4 * c + 2] = v.z;
      r.w[4 * c + 3] = v.w;
    }
  }

  __device__ __forceinline__ static int scale_byte(const Regs& r, int i) {
    return static_cast<int>((r.w[1 + (i >> 2)] >> (8 * (i & 3))) & 0xffu);
  }

  template <bool kExact, int h, typename Emit>
  __device__ __forceinline__ static void decode_half(const Regs& r, Emit&& emit) {
    const float d = f16_to_f32(static_cast<uint16_t>(r.w[0] & 0xffffu));
    const float dmin = f16_to_f32(static_cast<uint16_t>(r.w[0] >> 16));
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int j = 4 * h + jj;  // sub-block of 32 positions (gguf_quant.py:118-135)
      int sc, m;
      if (j < 4) {
        sc = scale_byte(r, j) & 63;
        m = scale_byte(r, j + 4) & 63;
      } else {
        sc = (scale_byte(r, j + 4) & 15) | ((scale_byte(r, j - 4) >> 6) << 4);
        m = (scale_byte(r, j + 4) >> 4) | ((scale_byte(r, j) >> 6) << 4);
      }
      const float ds = __fmul_rn(d, static_cast<float>(sc));
      const float nk = __fmul_rn(ds, -1024.f);
      const float dm = __fmul_rn(dmin, static_cast<float>(m));
#pragma unroll
      for (int half16 = 0; half16 < 2; ++half16) {
        uint32_t out[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t word = r.w[4 + 8 * (j >> 1) + 4 * half16 + i];
          const uint32_t code = (word >> (4 * (j & 1))) & 0x0f0f0f0fu;
          code4<kExact, true>(code, ds, nk, 1024.f, dm, out[2 * i], out[2 * i + 1]);
        }
        emit(jj * 16 + half16 * 8, out);
      }
    }
  }
};

}  // namespace qk
