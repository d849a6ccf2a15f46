// 128-row weight tiles and their thread-per-row decode into BF16 TMEM columns.
//
// Layout of one matrix W[rows, K] (rows zero-padded to a multiple of 128): tiles of 128
// rows x one 256-value GGUF block, ordered [row tile][k block]. Inside a tile the first
// 16 * C bytes of every row's block are stored as [chunk c][row r][16 B] (C = 13 for Q6_K,
// covering block bytes 0..207; C = 9 for Q4_K, the whole 144-byte block); Q6_K then holds
// the rows' FP16 scale d as [row][2 B]. Thread r of the decode warps reads chunk c of its
// row at (c * 128 + r) * 16 - consecutive rows are consecutive 16-byte words, so the
// shared-memory reads are conflict free - and decodes the row in natural K order.
//
// Values: the reference decodes (d * sc) * q (Q6_K) and (d * sc) * q - dmin * m (Q4_K)
// in FP32 and rounds to BF16 (glm53_offload/gguf_quant.py:154-157,171). The products are
// exact in FP32, so one fused multiply-add per element reproduces them:
//   Q6_K: u = 128 + code (byte permute into FP32 bits 0x43000000 | code << 16),
//         w = fma(u, ds, -160 ds) = (code - 32) ds;
//   Q4_K: w = fma(u, ds, -128 ds) - dmin m.
// The fused form turns a (d * sc) * 0 of negative sign into +0, which no dot product can
// see; kExact (the dequantisation entry points) subtracts before multiplying and so
// reproduces the reference bit for bit, signed zeros included.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace qk {

enum class QType { Q6_K = 14, Q4_K = 12 };

// 128 + byte I of `codes` as FP32.
template <int I>
__device__ __forceinline__ float magic128(uint32_t codes) {
  return __uint_as_float(__byte_perm(codes, 0x43u, 0x4055u | (I << 8)));
}

// Four codes (bytes of `code`) -> two packed BF16 pairs.
template <bool kExact>
__device__ __forceinline__ void code4_q6(uint32_t code, float ds, float nk, uint32_t& lo, uint32_t& hi) {
  const float2 u01 = make_float2(magic128<0>(code), magic128<1>(code));
  const float2 u23 = make_float2(magic128<2>(code), magic128<3>(code));
  const float2 s = make_float2(ds, ds);
  float2 w01, w23;
  if (kExact) {
    const float2 off = make_float2(-160.f, -160.f);
    w01 = __fmul2_rn(__fadd2_rn(u01, off), s);
    w23 = __fmul2_rn(__fadd2_rn(u23, off), s);
  } else {
    const float2 k = make_float2(nk, nk);
    w01 = __ffma2_rn(u01, s, k);
    w23 = __ffma2_rn(u23, s, k);
  }
  lo = pack_bf16x2(w01.x, w01.y);
  hi = pack_bf16x2(w23.x, w23.y);
}

template <bool kExact>
__device__ __forceinline__ void code4_q4(uint32_t code, float ds, float nk, float dm, uint32_t& lo,
                                         uint32_t& hi) {
  const float2 u01 = make_float2(magic128<0>(code), magic128<1>(code));
  const float2 u23 = make_float2(magic128<2>(code), magic128<3>(code));
  const float2 s = make_float2(ds, ds), m = make_float2(-dm, -dm);
  float2 w01, w23;
  if (kExact) {
    const float2 off = make_float2(-128.f, -128.f);
    w01 = __fmul2_rn(__fadd2_rn(u01, off), s);
    w23 = __fmul2_rn(__fadd2_rn(u23, off), s);
  } else {
    const float2 k = make_float2(nk, nk);
    w01 = __ffma2_rn(u01, s, k);
    w23 = __ffma2_rn(u23, s, k);
  }
  w01 = __fadd2_rn(w01, m);
  w23 = __fadd2_rn(w23, m);
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
    uint32_t w[52];  // block bytes 0..207: ql (words 0..31), qh (32..47), sub-scales (48..51)
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
    for (int lg = 0; lg < 2; ++lg) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int j = 8 * h + 2 * q + lg;  // sub-block of 16 positions
        const int sc = static_cast<int8_t>((r.w[48 + (j >> 2)] >> (8 * (j & 3))) & 0xffu);
        const float ds = __fmul_rn(r.d, static_cast<float>(sc));
        const float nk = __fmul_rn(ds, -160.f);
        uint32_t out[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t ql = r.w[16 * h + 8 * (q & 1) + 4 * lg + i];
          const uint32_t qh = r.w[32 + 8 * h + 4 * lg + i];
          const uint32_t code = ((ql >> (4 * (q >> 1))) & 0x0f0f0f0fu) | (((qh >> (2 * q)) & 0x03030303u) << 4);
          code4_q6<kExact>(code, ds, nk, out[2 * i], out[2 * i + 1]);
        }
        emit(q * 16 + lg * 8, out);
      }
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
      const float nk = __fmul_rn(ds, -128.f);
      const float dm = __fmul_rn(dmin, static_cast<float>(m));
#pragma unroll
      for (int half16 = 0; half16 < 2; ++half16) {
        uint32_t out[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t word = r.w[4 + 8 * (j >> 1) + 4 * half16 + i];
          const uint32_t code = (word >> (4 * (j & 1))) & 0x0f0f0f0fu;
          code4_q4<kExact>(code, ds, nk, dm, out[2 * i], out[2 * i + 1]);
        }
        emit(jj * 16 + half16 * 8, out);
      }
    }
  }
};

}  // namespace qk
