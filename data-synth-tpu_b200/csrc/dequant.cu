// GGUF block decode (raw and tiled layouts) and the lossless raw <-> tiled repack.
//
// qk_dequantize_rows restates glm53_offload/gguf_quant.py:63-177 (Q4_K, Q5_K, Q6_K,
// Q8_0, F16, BF16, F32) and qwen38_tpu/quant.py:15-55 (Q4_0, Q4_1, Q5_0, Q5_1,
// IQ4_NL) one output value per thread. FP32 operations are written with explicit
// round-to-nearest intrinsics so no multiply-add is contracted.
#include "common.cuh"
#include "rowtile.cuh"

namespace qk {
namespace {

__device__ __constant__ float kIq4Values[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                                1,    13,   25,  38,  53,  69,  89,  113};

struct BlockShape {
  int values;
  int bytes;
};

__host__ __device__ inline BlockShape block_shape(int qtype) {
  switch (qtype) {
    case QK_TYPE_F32: return {1, 4};
    case QK_TYPE_F16: return {1, 2};
    case QK_TYPE_BF16: return {1, 2};
    case QK_TYPE_Q4_0: return {32, 18};
    case QK_TYPE_Q4_1: return {32, 20};
    case QK_TYPE_Q5_0: return {32, 22};
    case QK_TYPE_Q5_1: return {32, 24};
    case QK_TYPE_Q8_0: return {32, 34};
    case QK_TYPE_IQ4_NL: return {32, 18};
    case QK_TYPE_Q4_K: return {256, 144};
    case QK_TYPE_Q5_K: return {256, 176};
    case QK_TYPE_Q6_K: return {256, 210};
    default: return {0, 0};
  }
}

__device__ __forceinline__ float f16_at(const uint8_t* b) {
  return f16_to_f32(static_cast<uint16_t>(b[0] | (b[1] << 8)));
}

__device__ __forceinline__ void k_scale_min(const uint8_t* blk, int j, int& sc, int& m) {
  const uint8_t* s = blk + 4;
  if (j < 4) {
    sc = s[j] & 63;
    m = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
    m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

// Value p of one GGUF block.
__device__ float decode_value(const uint8_t* blk, int qtype, int p) {
  switch (qtype) {
    case QK_TYPE_F32: {
      uint32_t bits = blk[0] | (blk[1] << 8) | (blk[2] << 16) | (static_cast<uint32_t>(blk[3]) << 24);
      return __uint_as_float(bits);
    }
    case QK_TYPE_F16: return f16_at(blk);
    case QK_TYPE_BF16: return bf16_to_f32(static_cast<uint16_t>(blk[0] | (blk[1] << 8)));
    case QK_TYPE_Q8_0:
      return __fmul_rn(f16_at(blk), static_cast<float>(static_cast<int8_t>(blk[2 + p])));
    case QK_TYPE_Q4_0:
    case QK_TYPE_Q4_1:
    case QK_TYPE_Q5_0:
    case QK_TYPE_Q5_1:
    case QK_TYPE_IQ4_NL: {  // quant.py:31-55
      const bool affine = qtype == QK_TYPE_Q4_1 || qtype == QK_TYPE_Q5_1;
      const bool five = qtype == QK_TYPE_Q5_0 || qtype == QK_TYPE_Q5_1;
      const int base = affine ? 4 : 2;
      const uint8_t byte = blk[base + (five ? 4 : 0) + (p & 15)];
      int q = p < 16 ? (byte & 15) : (byte >> 4);
      if (five) {
        const uint8_t* h = blk + base;
        const uint32_t bits = h[0] | (h[1] << 8) | (h[2] << 16) | (static_cast<uint32_t>(h[3]) << 24);
        q |= static_cast<int>((bits >> p) & 1u) << 4;
      }
      const float d = f16_at(blk);
      float v;
      if (qtype == QK_TYPE_IQ4_NL) v = __fmul_rn(d, kIq4Values[q]);
      else if (affine) v = __fmul_rn(d, static_cast<float>(q));
      else v = __fmul_rn(d, static_cast<float>(q - (five ? 16 : 8)));
      if (affine) v = __fadd_rn(v, f16_at(blk + 2));
      return v;
    }
    case QK_TYPE_Q4_K:
    case QK_TYPE_Q5_K: {  // gguf_quant.py:115-157
      const int j = p >> 5, i = p & 31;
      int q;
      if (qtype == QK_TYPE_Q4_K) {
        q = (blk[16 + (j >> 1) * 32 + i] >> (4 * (j & 1))) & 15;
      } else {
        q = ((blk[48 + (j >> 1) * 32 + i] >> (4 * (j & 1))) & 15) | (((blk[16 + i] >> j) & 1) << 4);
      }
      int sc, m;
      k_scale_min(blk, j, sc, m);
      const float a = __fmul_rn(__fmul_rn(f16_at(blk), static_cast<float>(sc)), static_cast<float>(q));
      return __fsub_rn(a, __fmul_rn(f16_at(blk + 2), static_cast<float>(m)));
    }
    case QK_TYPE_Q6_K: {  // gguf_quant.py:158-173, packed_q6/reference.py:21-30
      const int half = p >> 7, quarter = (p & 127) >> 5, lane = p & 31;
      const int lo = (blk[half * 64 + (quarter & 1) * 32 + lane] >> (4 * (quarter >> 1))) & 15;
      const int hi = (blk[128 + half * 32 + lane] >> (2 * quarter)) & 3;
      const int q = (lo | (hi << 4)) - 32;
      const float ds = __fmul_rn(f16_at(blk + 208), static_cast<float>(static_cast<int8_t>(blk[192 + (p >> 4)])));
      return __fmul_rn(ds, static_cast<float>(q));
    }
    default: return 0.f;
  }
}

__global__ void dequant_rows_kernel(const uint8_t* __restrict__ raw, int qtype, int64_t rows,
                                    int64_t width, int64_t nblk, BlockShape shape, int out_bf16,
                                    void* __restrict__ out) {
  const int64_t total = rows * width;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / width, col = i % width;
    const int64_t b = col / shape.values;
    const uint8_t* blk = raw + (row * nblk + b) * shape.bytes;
    const float v = decode_value(blk, qtype, static_cast<int>(col % shape.values));
    if (out_bf16) static_cast<uint16_t*>(out)[i] = bf16_bits_rne(v);
    else static_cast<float*>(out)[i] = v;
  }
}

// ---- tiled layout (the format is stated in oracle/layout.py and rowtile.cuh) ----

inline int tile_bytes(int qtype) {
  return qtype == QK_TYPE_Q6_K   ? HalfTile<QType::Q6_K>::kBytes
         : qtype == QK_TYPE_Q4_K ? HalfTile<QType::Q4_K>::kBytes
         : qtype == QK_TYPE_Q8_0 ? HalfTile<QType::Q8_0>::kBytes
         : qtype == QK_TYPE_Q5_K ? HalfTile<QType::Q5_K>::kBytes
         : qtype == QK_TYPE_Q5_1 ? HalfTile<QType::Q5_1>::kBytes
                                 : 0;
}

// Byte offset, inside a 64-row tile, of 32-bit word w of row r.
__device__ __forceinline__ int tile_word(int r, int w) { return ((w >> 2) * kTileRows + r) * 16 + (w & 3) * 4; }

// Q6_K code of position p of a GGUF block (packed_q6/reference.py:21-27 position rule).
__device__ __forceinline__ uint32_t q6_code(const uint8_t* blk, int p) {
  const int half = p >> 7, quarter = (p & 127) >> 5, lane = p & 31;
  const uint32_t lo = (blk[half * 64 + (quarter & 1) * 32 + lane] >> (4 * (quarter >> 1))) & 15u;
  const uint32_t hi = (blk[128 + half * 32 + lane] >> (2 * quarter)) & 3u;
  return lo | (hi << 4);
}

// One thread per (tile row, sub-block j) - 16 codes -> 3 words; j == 16 copies the
// sub-scale words and d. kPack: raw -> tiled, else tiled -> raw.
template <bool kPack>
__global__ void __launch_bounds__(kTileRows) repack_q6_kernel(const uint8_t* __restrict__ in, uint8_t* __restrict__ out,
                                                              int64_t rows, int64_t nblk, int32_t* bad_scales) {
  constexpr int TB = HalfTile<QType::Q6_K>::kBytes;
  constexpr int kScaleOff = HalfTile<QType::Q6_K>::kScaleOff;
  const int64_t tile = blockIdx.x;
  const int64_t strip = tile / nblk, kb = tile % nblk;
  const int r = threadIdx.x;
  const int64_t row = strip * kTileRows + r;
  const bool real = row < rows;
  uint8_t* traw_out = nullptr;
  const uint8_t* blk = nullptr;
  uint8_t* t = nullptr;
  const uint8_t* tin = nullptr;
  if (kPack) {
    blk = real ? in + (row * nblk + kb) * 210 : nullptr;
    t = out + tile * TB;
  } else {
    tin = in + tile * TB;
    traw_out = real ? out + (row * nblk + kb) * 210 : nullptr;
  }
  if (kPack) {
    for (int j = 0; j < 16; ++j) {
      uint32_t u[16];
      for (int i = 0; i < 16; ++i) u[i] = real ? q6_code(blk, 16 * j + i) : 0u;
      uint32_t w[3] = {0, 0, 0};
      for (int n = 0; n < 3; ++n)
        for (int i = 0; i < 4; ++i)
          w[n] |= (u[4 * n + i] | (((u[12 + i] >> (2 * n)) & 3u) << 6)) << (8 * i);
      for (int n = 0; n < 3; ++n) *reinterpret_cast<uint32_t*>(t + tile_word(r, 3 * j + n)) = w[n];
    }
    for (int n = 0; n < 4; ++n) {  // sub-scales: block bytes 192..207
      uint32_t v = 0;
      if (real)
        for (int i = 0; i < 4; ++i) v |= static_cast<uint32_t>(blk[192 + 4 * n + i]) << (8 * i);
      *reinterpret_cast<uint32_t*>(t + tile_word(r, 48 + n)) = v;
    }
    const uint16_t d = real ? static_cast<uint16_t>(blk[208] | (blk[209] << 8)) : 0;
    *reinterpret_cast<uint16_t*>(t + kScaleOff + r * 2) = d;
    if (bad_scales && (d & 0x7c00) == 0x7c00) atomicAdd(bad_scales, 1);
  } else if (real) {
    uint8_t b[208];
    for (int i = 0; i < 192; ++i) b[i] = 0;
    for (int j = 0; j < 16; ++j) {
      uint32_t w[3];
      for (int n = 0; n < 3; ++n) w[n] = *reinterpret_cast<const uint32_t*>(tin + tile_word(r, 3 * j + n));
      for (int i = 0; i < 16; ++i) {
        uint32_t u;
        if (i < 12) {
          u = (w[i >> 2] >> (8 * (i & 3))) & 63u;
        } else {
          const int m = i - 12;
          u = 0;
          for (int n = 0; n < 3; ++n) u |= ((w[n] >> (8 * m + 6)) & 3u) << (2 * n);
        }
        const int p = 16 * j + i, half = p >> 7, quarter = (p & 127) >> 5, lane = p & 31;
        b[half * 64 + (quarter & 1) * 32 + lane] |= static_cast<uint8_t>((u & 15u) << (4 * (quarter >> 1)));
        b[128 + half * 32 + lane] |= static_cast<uint8_t>((u >> 4) << (2 * quarter));
      }
    }
    for (int n = 0; n < 4; ++n) {
      const uint32_t v = *reinterpret_cast<const uint32_t*>(tin + tile_word(r, 48 + n));
      for (int i = 0; i < 4; ++i) b[192 + 4 * n + i] = static_cast<uint8_t>(v >> (8 * i));
    }
    for (int i = 0; i < 208; ++i) traw_out[i] = b[i];
    const uint16_t d = *reinterpret_cast<const uint16_t*>(tin + kScaleOff + r * 2);
    traw_out[208] = static_cast<uint8_t>(d & 0xff);
    traw_out[209] = static_cast<uint8_t>(d >> 8);
  }
}

// Q4_K and Q5_K: a byte transpose of the GGUF block bytes. One CTA per tile; byte `off` of
// the tile is chunk off / 1024, row (off % 1024) / 16, byte off % 16 of the chunk, i.e. block
// byte 16 * chunk + off % 16. tiled[...] <- raw[...] (or the reverse).
template <bool kPack, int kBlockBytes>
__global__ void repack_k_kernel(const uint8_t* __restrict__ in, uint8_t* __restrict__ out, int64_t rows,
                                int64_t nblk, int32_t* bad_scales) {
  constexpr int TB = kTileRows * kBlockBytes;
  const int64_t tile = blockIdx.x;
  const int64_t strip = tile / nblk, kb = tile % nblk;
  for (int off = threadIdx.x; off < TB; off += blockDim.x) {
    const int r = (off & 1023) >> 4, src = (off >> 10) * 16 + (off & 15);
    const int64_t row = strip * kTileRows + r;
    const int64_t raw_off = (row * nblk + kb) * kBlockBytes + src;
    const int64_t tiled_off = tile * TB + off;
    if (kPack) {
      uint8_t v = 0;
      if (row < rows) {
        v = in[raw_off];
        if (bad_scales && (src == 1 || src == 3) && (v & 0x7c) == 0x7c) atomicAdd(bad_scales, 1);
      }
      out[tiled_off] = v;
    } else if (row < rows) {
      out[raw_off] = in[tiled_off];
    }
  }
}

// Q5_1: super-blocks of 8 GGUF blocks of 24 bytes (rowtile.cuh). One CTA per tile; chunk c,
// row r, byte b of the tile hold, for c < 2, byte b % 4 of block 4c + b / 4 (d, m); for
// c in {2, 3}, byte 4 + b % 4 of block 4 (c - 2) + b / 4 (the high-bit word); for c >= 4,
// byte 8 + b of block c - 4 (the nibbles). Raw rows have nblk32 blocks; super-block blocks
// past them are zero.
template <bool kPack>
__global__ void repack_q51_kernel(const uint8_t* __restrict__ in, uint8_t* __restrict__ out, int64_t rows,
                                  int64_t nblk, int64_t nblk32, int32_t* bad_scales) {
  constexpr int TB = HalfTile<QType::Q5_1>::kBytes;
  const int64_t tile = blockIdx.x;
  const int64_t strip = tile / nblk, kb = tile % nblk;
  for (int off = threadIdx.x; off < TB; off += blockDim.x) {
    const int c = off >> 10, r = (off & 1023) >> 4, byte = off & 15;
    const int64_t row = strip * kTileRows + r;
    int j, src;
    if (c < 2) {
      j = 4 * c + (byte >> 2);
      src = byte & 3;
    } else if (c < 4) {
      j = 4 * (c - 2) + (byte >> 2);
      src = 4 + (byte & 3);
    } else {
      j = c - 4;
      src = 8 + byte;
    }
    const int64_t blk = kb * 8 + j;
    const bool exists = row < rows && blk < nblk32;
    const int64_t raw_off = (row * nblk32 + blk) * 24 + src;
    const int64_t tiled_off = tile * TB + off;
    if (kPack) {
      uint8_t v = 0;
      if (exists) {
        v = in[raw_off];
        if (bad_scales && src == 1 && (v & 0x7c) == 0x7c) atomicAdd(bad_scales, 1);
      }
      out[tiled_off] = v;
    } else if (exists) {
      out[raw_off] = in[tiled_off];
    }
  }
}

// Q8_0: super-blocks of 8 GGUF blocks (rowtile.cuh). One CTA per tile; byte `off` of the
// tile is chunk off / 1024, row (off % 1024) / 16, byte off % 16 of the chunk. Raw rows have
// nblk32 blocks of 34 bytes; super-block blocks past them are zero.
template <bool kPack>
__global__ void repack_q8_kernel(const uint8_t* __restrict__ in, uint8_t* __restrict__ out, int64_t rows,
                                 int64_t nblk, int64_t nblk32, int32_t* bad_scales) {
  constexpr int TB = HalfTile<QType::Q8_0>::kBytes;
  const int64_t tile = blockIdx.x;
  const int64_t strip = tile / nblk, kb = tile % nblk;
  for (int off = threadIdx.x; off < TB; off += blockDim.x) {
    const int c = off >> 10, r = (off & 1023) >> 4, byte = off & 15;
    const int64_t row = strip * kTileRows + r;
    int j, src;  // GGUF block of the super-block and byte of it
    if (c == 0) {
      j = byte >> 1;
      src = byte & 1;
    } else {
      const int code = (c - 1) * 16 + byte;
      j = code >> 5;
      src = 2 + (code & 31);
    }
    const int64_t blk = kb * 8 + j;
    const bool exists = row < rows && blk < nblk32;
    const int64_t raw_off = (row * nblk32 + blk) * 34 + src;
    const int64_t tiled_off = tile * TB + off;
    if (kPack) {
      uint8_t v = 0;
      if (exists) {
        v = in[raw_off];
        if (bad_scales && c == 0 && src == 1 && (v & 0x7c) == 0x7c) atomicAdd(bad_scales, 1);
      }
      out[tiled_off] = v;
    } else if (exists) {
      out[raw_off] = in[tiled_off];
    }
  }
}

// Decode of the tiled layout through the half-block decoders of the tensor-core kernels:
// kExact selects the reference-exact form (signed zeros included), otherwise the fused
// form the kernels run (equal values; a zero may carry the other sign). One thread per
// (tile row, half block).
template <QType QT, bool kExact>
__global__ void __launch_bounds__(2 * kTileRows) dequant_tiled_kernel(const uint8_t* __restrict__ tiled, int64_t rows,
                                                                      int64_t width, int64_t nblk, int out_bf16,
                                                                      void* __restrict__ out) {
  using HT = HalfTile<QT>;
  const int64_t tile = blockIdx.x;
  const int64_t strip = tile / nblk, kb = tile % nblk;
  const int r = threadIdx.x % kTileRows, h = threadIdx.x / kTileRows;
  const int64_t row = strip * kTileRows + r;
  if (row >= rows) return;
  const uint8_t* t = tiled + tile * HT::kBytes;
  auto store = [&](int64_t k0, const uint32_t(&o)[8]) {
    for (int i = 0; i < 16; ++i) {
      const int64_t k = k0 + i;
      if (k >= width) break;
      const uint16_t bits = static_cast<uint16_t>(o[i >> 1] >> (16 * (i & 1)));
      if (out_bf16) static_cast<uint16_t*>(out)[row * width + k] = bits;
      else static_cast<float*>(out)[row * width + k] = bf16_to_f32(bits);
    }
  };
  typename HT::Regs regs;
  if (h == 0) {
    HT::load(regs, t, r, 0);
    HT::template decode<kExact>(regs, 0, [&](int col, const uint32_t(&o)[8]) { store(kb * 256 + 2 * col, o); });
  } else {
    HT::load(regs, t, r, 1);
    HT::template decode<kExact>(regs, 1, [&](int col, const uint32_t(&o)[8]) { store(kb * 256 + 128 + 2 * col, o); });
  }
}

// The reference's TPU input form of a Q6_K projection (packed_q6/layout.py:49-91, PackedQ6):
// per (64-row output tile, K block) one 13,312-byte data tile holding the rows' GGUF bytes
// [0, 128) as [row][128], then [128, 192) as [row][64], then [192, 208) as [row][16], and a
// separate scale plane holding the rows' FP16 `d` bytes [208, 210) as [tile][block][row][2].
// This kernel restores the GGUF rows [rows, blocks, 210] from the two planes (the inverse,
// unpack_q6, is layout.py:93-108); rows past `rows` in the last tile are padding and skipped.
// One CTA per (tile, block); each thread writes bytes of the tile's rows in order.
__global__ void q6_soa_to_rows_kernel(const uint8_t* __restrict__ data, const uint8_t* __restrict__ scales,
                                      int64_t rows, int64_t blocks, uint8_t* __restrict__ raw) {
  constexpr int kRows = 64, kBlock = 210, kDataTile = kRows * 208;
  const int64_t tb = blockIdx.x;  // tile * blocks + block
  const int64_t tile = tb / blocks, blk = tb % blocks;
  const uint8_t* src = data + tb * kDataTile;
  const uint8_t* sc = scales + tb * (kRows * 2);
  for (int i = threadIdx.x; i < kRows * kBlock; i += blockDim.x) {
    const int r = i / kBlock, b = i % kBlock;
    const int64_t row = tile * kRows + r;
    if (row >= rows) break;
    uint8_t v;
    if (b < 128) v = src[r * 128 + b];
    else if (b < 192) v = src[kRows * 128 + r * 64 + (b - 128)];
    else if (b < 208) v = src[kRows * 192 + r * 16 + (b - 192)];
    else v = sc[r * 2 + (b - 208)];
    raw[(row * blocks + blk) * kBlock + b] = v;
  }
}

int grid_for(int64_t total, int block) {
  int64_t g = (total + block - 1) / block;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 32;
  return static_cast<int>(g < 1 ? 1 : (g > cap ? cap : g));
}

}  // namespace
}  // namespace qk

using namespace qk;

extern "C" {

int qk_dequantize_rows(const uint8_t* raw, int qtype, int64_t rows, int64_t row_width,
                       int out_dtype, void* out, qk_stream_t stream) {
  const BlockShape shape = block_shape(qtype);
  if (shape.values == 0) return set_error(QK_ERR_UNSUPPORTED_TYPE, "unsupported GGUF quantization type: %d", qtype);
  QK_REQUIRE(rows >= 0 && row_width > 0, "row_width must be a positive integer");
  QK_REQUIRE(out_dtype == QK_OUT_F32 || out_dtype == QK_OUT_BF16, "out_dtype must be F32 or BF16");
  if (rows == 0) return QK_OK;
  QK_REQUIRE(raw && out, "null pointer");
  const int64_t nblk = (row_width + shape.values - 1) / shape.values;
  dequant_rows_kernel<<<grid_for(rows * row_width, 256), 256, 0, as_stream(stream)>>>(
      raw, qtype, rows, row_width, nblk, shape, out_dtype == QK_OUT_BF16, out);
  QK_LAUNCHED("dequant_rows_kernel");
  return QK_OK;
}

int64_t qk_tiled_bytes(int qtype, int64_t rows, int64_t row_width) {
  const int tb = tile_bytes(qtype);
  if (tb == 0 || rows < 0 || row_width <= 0) return -1;
  return (rows + kTileRows - 1) / kTileRows * ((row_width + 255) / 256) * tb;
}

static int repack_common(const uint8_t* in, int qtype, int64_t rows, int64_t row_width,
                         uint8_t* out, int32_t* bad, qk_stream_t stream, bool pack) {
  const int tb = tile_bytes(qtype);
  if (tb == 0)
    return set_error(QK_ERR_UNSUPPORTED_TYPE, "tiled layout supports Q6_K, Q4_K, Q5_K, Q8_0 and Q5_1; got %d", qtype);
  QK_REQUIRE(rows > 0 && row_width > 0, "Expected [output_features, ceil(input_features / block), bytes]");
  QK_REQUIRE(in && out, "null pointer");
  const int64_t nblk = (row_width + 255) / 256;
  const int64_t tiles = (rows + kTileRows - 1) / kTileRows * nblk;
  QK_REQUIRE(tiles < (1ll << 31), "too many tiles");
  const unsigned g = static_cast<unsigned>(tiles);
  cudaStream_t st = as_stream(stream);
  if (qtype == QK_TYPE_Q6_K) {
    if (pack) repack_q6_kernel<true><<<g, kTileRows, 0, st>>>(in, out, rows, nblk, bad);
    else repack_q6_kernel<false><<<g, kTileRows, 0, st>>>(in, out, rows, nblk, nullptr);
  } else if (qtype == QK_TYPE_Q8_0) {
    const int64_t nblk32 = (row_width + 31) / 32;
    if (pack) repack_q8_kernel<true><<<g, 256, 0, st>>>(in, out, rows, nblk, nblk32, bad);
    else repack_q8_kernel<false><<<g, 256, 0, st>>>(in, out, rows, nblk, nblk32, nullptr);
  } else if (qtype == QK_TYPE_Q5_1) {
    const int64_t nblk32 = (row_width + 31) / 32;
    if (pack) repack_q51_kernel<true><<<g, 256, 0, st>>>(in, out, rows, nblk, nblk32, bad);
    else repack_q51_kernel<false><<<g, 256, 0, st>>>(in, out, rows, nblk, nblk32, nullptr);
  } else if (qtype == QK_TYPE_Q5_K) {
    if (pack) repack_k_kernel<true, 176><<<g, 256, 0, st>>>(in, out, rows, nblk, bad);
    else repack_k_kernel<false, 176><<<g, 256, 0, st>>>(in, out, rows, nblk, nullptr);
  } else {
    if (pack) repack_k_kernel<true, 144><<<g, 256, 0, st>>>(in, out, rows, nblk, bad);
    else repack_k_kernel<false, 144><<<g, 256, 0, st>>>(in, out, rows, nblk, nullptr);
  }
  QK_LAUNCHED("repack_kernel");
  return QK_OK;
}

int qk_repack_rows(const uint8_t* raw, int qtype, int64_t rows, int64_t row_width,
                   uint8_t* tiled, int32_t* bad_scales, qk_stream_t stream) {
  return repack_common(raw, qtype, rows, row_width, tiled, bad_scales, stream, true);
}

int qk_unpack_rows(const uint8_t* tiled, int qtype, int64_t rows, int64_t row_width, uint8_t* raw,
                   qk_stream_t stream) {
  return repack_common(tiled, qtype, rows, row_width, raw, nullptr, stream, false);
}

int qk_dequantize_tiled(const uint8_t* tiled, int qtype, int64_t rows, int64_t row_width,
                        int out_dtype, void* out, qk_stream_t stream) {
  if (tile_bytes(qtype) == 0)
    return set_error(QK_ERR_UNSUPPORTED_TYPE, "tiled layout supports Q6_K, Q4_K, Q5_K, Q8_0 and Q5_1; got %d", qtype);
  QK_REQUIRE(rows > 0 && row_width > 0, "rows and row_width must be positive");
  const bool fused = (out_dtype & QK_DECODE_FUSED) != 0;
  out_dtype &= ~QK_DECODE_FUSED;
  QK_REQUIRE(out_dtype == QK_OUT_F32 || out_dtype == QK_OUT_BF16, "out_dtype must be F32 or BF16");
  QK_REQUIRE(tiled && out, "null pointer");
  const int64_t nblk = (row_width + 255) / 256;
  const int64_t tiles = (rows + kTileRows - 1) / kTileRows * nblk;
  QK_REQUIRE(tiles < (1ll << 31), "too many tiles");
  const unsigned grid = static_cast<unsigned>(tiles);
  const int bf = out_dtype == QK_OUT_BF16;
  cudaStream_t st = as_stream(stream);
  if (qtype == QK_TYPE_Q6_K) {
    if (fused) dequant_tiled_kernel<QType::Q6_K, false><<<grid, 2 * kTileRows, 0, st>>>(tiled, rows, row_width, nblk, bf, out);
    else dequant_tiled_kernel<QType::Q6_K, true><<<grid, 2 * kTileRows, 0, st>>>(tiled, rows, row_width, nblk, bf, out);
  } else if (qtype == QK_TYPE_Q8_0) {
    if (fused) dequant_tiled_kernel<QType::Q8_0, false><<<grid, 2 * kTileRows, 0, st>>>(tiled, rows, row_width, nblk, bf, out);
    else dequant_tiled_kernel<QType::Q8_0, true><<<grid, 2 * kTileRows, 0, st>>>(tiled, rows, row_width, nblk, bf, out);
  } else if (qtype == QK_TYPE_Q5_K) {
    if (fused) dequant_tiled_kernel<QType::Q5_K, false><<<grid, 2 * kTileRows, 0, st>>>(tiled, rows, row_width, nblk, bf, out);
    else dequant_tiled_kernel<QType::Q5_K, true><<<grid, 2 * kTileRows, 0, st>>>(tiled, rows, row_width, nblk, bf, out);
  } else if (qtype == QK_TYPE_Q5_1) {
    if (fused) dequant_tiled_kernel<QType::Q5_1, false><<<grid, 2 * kTileRows, 0, st>>>(tiled, rows, row_width, nblk, bf, out);
    else dequant_tiled_kernel<QType::Q5_1, true><<<grid, 2 * kTileRows, 0, st>>>(tiled, rows, row_width, nblk, bf, out);
  } else {
    if (fused) dequant_tiled_kernel<QType::Q4_K, false><<<grid, 2 * kTileRows, 0, st>>>(tiled, rows, row_width, nblk, bf, out);
    else dequant_tiled_kernel<QType::Q4_K, true><<<grid, 2 * kTileRows, 0, st>>>(tiled, rows, row_width, nblk, bf, out);
  }
  QK_LAUNCHED("dequant_tiled_kernel");
  return QK_OK;
}

int qk_q6_soa_to_rows(const uint8_t* data, const uint8_t* scales, int64_t rows, int64_t input_features,
                      uint8_t* raw, qk_stream_t stream) {
  QK_REQUIRE(rows > 0 && input_features > 0, "rows and input_features must be positive");
  QK_REQUIRE(data && scales && raw, "null pointer");
  const int64_t blocks = (input_features + 255) / 256;
  const int64_t tiles = (rows + 63) / 64;
  QK_REQUIRE(tiles * blocks < (1ll << 31), "too many tiles");
  q6_soa_to_rows_kernel<<<static_cast<unsigned>(tiles * blocks), 256, 0, as_stream(stream)>>>(
      data, scales, rows, blocks, raw);
  QK_LAUNCHED("q6_soa_to_rows_kernel");
  return QK_OK;
}

}  // extern "C"
