// Tiled Q6_K / Q4_K weight layout and its in-register decode into BF16 MMA fragments.
//
// A tile is 16 weight rows x one 256-value GGUF block. Tiles of one matrix are ordered
// [row_strip][k_block]; rows are zero-padded to a multiple of 16 (a zero FP16 scale
// decodes to zero). Lane l = 4*g + c of a warp owns rows g and g+8 of the tile (the
// two row halves rh = 0, 1 of the m16n8k16 A fragment) and a fixed quarter of each
// row's 256 positions. The k order inside an MMA is a permutation of the block's
// positions; the activation (B) fragment is loaded with the same permutation, so the
// dot product is unchanged. k-step s (0..15) of lane c covers 4 consecutive positions
// p0(c, s) .. p0 + 3: A regs {a0, a2} hold row g's pairs (p0, p0+1), (p0+2, p0+3),
// {a1, a3} the same for row g+8, and the B regs hold x[p0..p0+3] of token column g.
//
// Values: the reference decodes Q6_K as (d * sc) * q and Q4_K as (d * sc) * q - dmin * m
// in FP32 (glm53_offload/gguf_quant.py:154-157,171), then rounds to BF16. Every product
// there is exact in FP32 (d: 11 significant bits, sc <= 8, q <= 6), so the only rounding
// is the final BF16 RNE (and, for Q4_K, the FP32 subtraction). The decoders below form
// the same exact FP32 values with one fused multiply-add per element:
//   Q6_K: u = 128 + code (built by byte permute into FP32 bits 0x43000000 | code << 16),
//         w = fma(u, ds, -160 * ds) = (code - 32) * ds, exact;
//   Q4_K: w = fma(u, ds, -128 * ds) - dm, the multiply exact, one rounding in the sub.
// These fused forms give +0 where the reference's (d * sc) * 0 keeps the sign of d * sc;
// a signed zero cannot change a dot product, so the GEMM kernels use them. The kExact
// variant (qk_dequantize_tiled) subtracts first and then multiplies, which reproduces
// the reference bit for bit, signed zeros included: w = (u - 160) * ds for Q6_K and
// w = (u - 128) * ds - dm for Q4_K.
#pragma once

#include "common.cuh"

namespace qk {

enum class QType { Q6_K = 14, Q4_K = 12 };

template <QType QT>
struct Tile;

// Builds 128 + byte_i of `codes` as an FP32 value (byte i in bits 16..23 under 0x43).
template <int I>
__device__ __forceinline__ float magic128(uint32_t codes) {
  return __uint_as_float(__byte_perm(codes, 0x43u, 0x4055u | (I << 8)));
}

// ---------------------------------------------------------------------------------
// Q6_K: 3360-byte tile (layout written out in oracle/layout.py and repack.cu)
// ---------------------------------------------------------------------------------
template <>
struct Tile<QType::Q6_K> {
  static constexpr int kBytes = 3360;
  static constexpr int kBlockBytes = 210;

  struct Regs {
    uint4 ql[2][2];  // [rh][part]
    uint4 qh[2];     // [rh]
    uint2 sc;        // rh0: sc for quarters 0..3, rh1: same
    uint32_t d;      // d(row g) | d(row g+8) << 16
  };

  __device__ __forceinline__ static void load(Regs& r, const uint8_t* t, int lane) {
    r.ql[0][0] = lds_v4(t + 0 * 512 + lane * 16);
    r.ql[0][1] = lds_v4(t + 1 * 512 + lane * 16);
    r.ql[1][0] = lds_v4(t + 2 * 512 + lane * 16);
    r.ql[1][1] = lds_v4(t + 3 * 512 + lane * 16);
    r.qh[0] = lds_v4(t + 2048 + lane * 16);
    r.qh[1] = lds_v4(t + 2560 + lane * 16);
    r.sc = *reinterpret_cast<const uint2*>(t + 3072 + lane * 8);
    r.d = *reinterpret_cast<const uint32_t*>(t + 3328 + (lane >> 2) * 4);
  }

  // Position of the first of the 4 values of k-step s for lane quarter c.
  __device__ __forceinline__ static int p0(int c, int s) {
    return (c >> 1) * 128 + (s >> 2) * 32 + (c & 1) * 16 + (s & 3) * 4;
  }

  // Scale of sub-block (rh, quarter q) and the matching -160 * scale.
  __device__ __forceinline__ static float2 scale(const Regs& r, int rh, int q) {
    const float d = f16_to_f32(static_cast<uint16_t>(rh ? (r.d >> 16) : (r.d & 0xffffu)));
    const uint32_t w = rh ? r.sc.y : r.sc.x;
    const int sc = static_cast<int8_t>((w >> (8 * q)) & 0xffu);
    const float ds = __fmul_rn(d, static_cast<float>(sc));
    return make_float2(ds, __fmul_rn(ds, -160.f));
  }

  // Four BF16 values of row half rh at k-step s -> two packed pairs.
  // s must fold to a constant (callers fully unroll their k-step loops).
  template <bool kExact>
  __device__ __forceinline__ static void pairs(const Regs& r, int rh, float2 sc, int s,
                                               uint32_t& lo, uint32_t& hi) {
    const int Q = s >> 2, J4 = s & 3;
    const uint32_t l = (word(r.ql[rh][Q & 1], J4) >> (4 * (Q >> 1))) & 0x0f0f0f0fu;
    const uint32_t h = (word(r.qh[rh], J4) >> (2 * Q)) & 0x03030303u;
    const uint32_t code = l | (h << 4);
    const float2 ds = make_float2(sc.x, sc.x);
    const float2 u01 = make_float2(magic128<0>(code), magic128<1>(code));
    const float2 u23 = make_float2(magic128<2>(code), magic128<3>(code));
    float2 w01, w23;
    if (kExact) {
      const float2 off = make_float2(-160.f, -160.f);
      w01 = __fmul2_rn(__fadd2_rn(u01, off), ds);
      w23 = __fmul2_rn(__fadd2_rn(u23, off), ds);
    } else {
      const float2 nk = make_float2(sc.y, sc.y);
      w01 = __ffma2_rn(u01, ds, nk);
      w23 = __ffma2_rn(u23, ds, nk);
    }
    lo = pack_bf16x2(w01.x, w01.y);
    hi = pack_bf16x2(w23.x, w23.y);
  }

  // A fragment of k-step s. `sc[rh]` must hold scale(r, rh, s >> 2).
  template <bool kExact = false>
  __device__ __forceinline__ static void fragment(const Regs& r, const float2 (&sc)[2], int s,
                                                  uint32_t (&a)[4]) {
    pairs<kExact>(r, 0, sc[0], s, a[0], a[2]);
    pairs<kExact>(r, 1, sc[1], s, a[1], a[3]);
  }

};

// ---------------------------------------------------------------------------------
// Q4_K: 2304-byte tile
// ---------------------------------------------------------------------------------
template <>
struct Tile<QType::Q4_K> {
  static constexpr int kBytes = 2304;
  static constexpr int kBlockBytes = 144;

  struct Regs {
    uint4 qs[2][2];  // [rh][half]
    uint4 head[2];   // [rh]: d, dmin, 12 scale bytes
  };

  __device__ __forceinline__ static void load(Regs& r, const uint8_t* t, int lane) {
    r.qs[0][0] = lds_v4(t + 0 * 512 + lane * 16);
    r.qs[0][1] = lds_v4(t + 1 * 512 + lane * 16);
    r.qs[1][0] = lds_v4(t + 2 * 512 + lane * 16);
    r.qs[1][1] = lds_v4(t + 3 * 512 + lane * 16);
    const int g = lane >> 2;
    r.head[0] = lds_v4(t + 2048 + g * 16);
    r.head[1] = lds_v4(t + 2048 + (g + 8) * 16);
  }

  // k-step s: sub-block 2c + (s >> 3), 16-byte half (s >> 2) & 1, word s & 3.
  __device__ __forceinline__ static int p0(int c, int s) {
    return (2 * c + (s >> 3)) * 32 + ((s >> 2) & 1) * 16 + (s & 3) * 4;
  }

  // 6-bit scale and min of sub-block j (gguf_quant.py:118-135).
  __device__ __forceinline__ static void sub(const uint4& h, int j, int& sc, int& m) {
    auto byte = [&](int i) -> int {  // scale bytes start at block byte 4 (= head.y)
      const uint32_t w = i < 4 ? h.y : i < 8 ? h.z : h.w;
      return static_cast<int>((w >> (8 * (i & 3))) & 0xffu);
    };
    if (j < 4) {
      sc = byte(j) & 63;
      m = byte(j + 4) & 63;
    } else {
      sc = (byte(j + 4) & 15) | ((byte(j - 4) >> 6) << 4);
      m = (byte(j + 4) >> 4) | ((byte(j) >> 6) << 4);
    }
  }

  // (d * sc, -128 * d * sc, dmin * m) for row half rh and sub-block j.
  __device__ __forceinline__ static float4 scale(const Regs& r, int rh, int j) {
    const uint4& h = r.head[rh];
    const float d = f16_to_f32(static_cast<uint16_t>(h.x & 0xffffu));
    const float dmin = f16_to_f32(static_cast<uint16_t>(h.x >> 16));
    int sc, m;
    sub(h, j, sc, m);
    const float ds = __fmul_rn(d, static_cast<float>(sc));
    return make_float4(ds, __fmul_rn(ds, -128.f), __fmul_rn(dmin, static_cast<float>(m)), 0.f);
  }

  template <bool kExact>
  __device__ __forceinline__ static void pairs(const Regs& r, int rh, float4 sc, int s,
                                               uint32_t& lo, uint32_t& hi) {
    const int NIB = s >> 3, HALF = (s >> 2) & 1, J4 = s & 3;
    const uint32_t code = (word(r.qs[rh][HALF], J4) >> (4 * NIB)) & 0x0f0f0f0fu;
    const float2 ds = make_float2(sc.x, sc.x);
    const float2 dm = make_float2(-sc.z, -sc.z);
    const float2 u01 = make_float2(magic128<0>(code), magic128<1>(code));
    const float2 u23 = make_float2(magic128<2>(code), magic128<3>(code));
    float2 w01, w23;
    if (kExact) {
      const float2 off = make_float2(-128.f, -128.f);
      w01 = __fmul2_rn(__fadd2_rn(u01, off), ds);
      w23 = __fmul2_rn(__fadd2_rn(u23, off), ds);
    } else {
      const float2 nk = make_float2(sc.y, sc.y);
      w01 = __ffma2_rn(u01, ds, nk);
      w23 = __ffma2_rn(u23, ds, nk);
    }
    w01 = __fadd2_rn(w01, dm);
    w23 = __fadd2_rn(w23, dm);
    lo = pack_bf16x2(w01.x, w01.y);
    hi = pack_bf16x2(w23.x, w23.y);
  }

  template <bool kExact = false>
  __device__ __forceinline__ static void fragment(const Regs& r, const float4 (&sc)[2], int s,
                                                  uint32_t (&a)[4]) {
    pairs<kExact>(r, 0, sc[0], s, a[0], a[2]);
    pairs<kExact>(r, 1, sc[1], s, a[1], a[3]);
  }
};

// Scale state carried across k-steps: float2 per row half for Q6_K, float4 for Q4_K.
template <QType QT>
struct ScaleState;
template <>
struct ScaleState<QType::Q6_K> {
  float2 v[2];
  __device__ __forceinline__ void update(const Tile<QType::Q6_K>::Regs& r, int c, int s) {
    (void)c;
    if ((s & 3) == 0) {
      v[0] = Tile<QType::Q6_K>::scale(r, 0, s >> 2);
      v[1] = Tile<QType::Q6_K>::scale(r, 1, s >> 2);
    }
  }
};
template <>
struct ScaleState<QType::Q4_K> {
  float4 v[2];
  __device__ __forceinline__ void update(const Tile<QType::Q4_K>::Regs& r, int c, int s) {
    if ((s & 7) == 0) {
      v[0] = Tile<QType::Q4_K>::scale(r, 0, 2 * c + (s >> 3));
      v[1] = Tile<QType::Q4_K>::scale(r, 1, 2 * c + (s >> 3));
    }
  }
};

// Decode the A fragment of k-step s with a scale state already updated for s.
template <QType QT, bool kExact = false>
__device__ __forceinline__ void tile_fragment(const typename Tile<QT>::Regs& r,
                                              const ScaleState<QT>& st, int s, uint32_t (&a)[4]) {
  Tile<QT>::template fragment<kExact>(r, st.v, s, a);
}

}  // namespace qk
