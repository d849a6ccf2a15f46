// W8A8 down projection of the int8_q8 expert policy on the 5th-generation tensor core
// (tcgen05 kind::i8): the integer dot of qwen38_tpu/compute.py:20-34 (q8_matmul) for a Q8_0
// down projection, as qwen38_tpu/experts.py:85-107 runs it under compute="int8_q8".
//
// Arithmetic (compute.py:52-65, numpy_q8_matmul): per token and 32-value group g of h,
// act_scale = max|h| / 127 and codes = clip(rint(h / act_scale), -127, 127) (a zero scale
// divides by 1); partial[g] = sum of codes x weight codes over the group, exact in int32;
// y = bf16(sum over g in order of (f32(partial[g]) * act_scale[g]) * weight_scale[g]).
//
// Two kernels (also the dense W8A8 projection qk_q8_matmul, compute.py:20-34, with x in
// chunks of 32 rows):
//  * moe_quant_h_kernel - one warp per (token row of a chunk, 256-value K block) of the
//    gate/up pass's h tiles: the activation codes, written as the B operand of the integer
//    MMA (K-major, no swizzle: [16-byte K chunk][token row][16 B] per K block), and the FP32
//    scales ([K block][group][token row]).
//  * umma_i8_down_kernel - one persistent CTA per SM, 6 warps. Work item: one token chunk
//    (<= 32 tokens) x 128 rows of H (weight tiles 2p and 2p + 1). Per K block the producer
//    (warp 0) loads the two 64-row Q8_0 tiles with one 5-D tensor copy that interleaves them
//    per 16-byte chunk ([chunk][tile][row][16 B], so the 128 rows of a chunk are one
//    canonical K-major operand), the chunk's activation codes and scales with two bulk
//    copies (no multicast). The MMA warp (warp 1) issues one M = 128, N = tokens, K = 32
//    integer MMA per group - the weight codes straight from shared memory, no decode - into
//    its own int32 accumulator (8 groups x 32 columns; two buffers). The four epilogue warps
//    (warps 2-5, one TMEM lane quadrant each, lane = row) read the eight accumulators, scale
//    and add them in group order into FP32 sums per token, and after the last K block store
//    y = bf16(sum) (or, tensor parallel, the FP32 sum per route).
// Every wait is bounded; on give-up the CTA records QK_ERR_TIMEOUT and leaves its loops.
#pragma once

#include <cuda.h>  // CUtensorMap

#include <cstring>

#include "rowtile.cuh"
#include "umma.cuh"

namespace qk {
namespace {  // each translation unit that launches these kernels holds its own copy

constexpr int kI8Stages = 4;
constexpr int kI8Tok = 32;             // tokens per chunk (the narrow chunks)
constexpr int kI8Threads = 6 * 32;
constexpr int kI8W = 2 * HalfTile<QType::Q8_0>::kBytes;  // two tiles: [17 chunks][2][64 rows][16 B]
constexpr int kI8X = 256 * kI8Tok;                       // codes of one K block: [16][32 rows][16 B]
constexpr int kI8S = 8 * kI8Tok * 4;                     // scales of one K block: [8 groups][32 rows] FP32
constexpr int kI8Stage = kI8W + kI8X + kI8S;             // 44032, a multiple of 1024
constexpr size_t kI8Smem = 1024 + static_cast<size_t>(kI8Stages) * kI8Stage + 256;
static_assert(kI8Stage % 1024 == 0, "stage alignment");

// Each thread of the warp reads 32 consecutive 32-bit columns of its own lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// Shared-memory matrix descriptor, K-major, no swizzle: 8-row x 16-byte core matrices, row
// groups `sbo` bytes apart, the two 16-byte K halves of the 32-byte K step `lbo` bytes apart.
__device__ __forceinline__ uint64_t sdesc_none(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3fffu) | (static_cast<uint64_t>((lbo >> 4) & 0x3fffu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46);
}

// Instruction descriptor of kind::i8: signed 8-bit A and B, int32 D, both K-major, M = 128, N.
__device__ __forceinline__ uint32_t idesc_s8_m128(uint32_t n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}

// D[tmem] = A[smem] * B[smem] (int32), M = 128, N from the descriptor, K = 32. One thread.
__device__ __forceinline__ void umma_s8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, 0, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc)
      : "memory");
}

// 5-D tensor copy (no multicast) of one box into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3, int c4,
                                            uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(smem_addr(bar)),
      "l"(policy)
      : "memory");
}

struct I8Args {
  const uint8_t* ht;         // h tiles of the gate/up pass (BF16, the down pass's activation tiles)
  int8_t* qx;                // activation codes [rows][nkb][16][16 B] per chunk (see the kernels)
  float* qs;                 // activation scales [rows / r16][nkb][8][r16] per chunk
  int nkb;                   // K blocks of the down pass (ceil(I / 256))
  int ngroups;               // 32-value groups of I (I / 32)
  int items_per_chunk;       // 128-row tiles of H
  int tiles64;               // 64-row tiles of one expert's down matrix
  const int32_t* n_chunks_p;
  const int4* chunk_rec;     // {expert, tokens, first entry, first tile row}
  uint16_t* y;               // [entries, H] BF16
  float* yr;                 // tensor parallel: FP32 [B * top_k, H] per route, or null
  const int32_t* entry_route;
  int nrows;                 // H (MoE) or N (dense)
  int32_t* status;
  // dense form (qk_q8_matmul): x of dense_m rows in chunks of 32 (entry = row), the FP32 or
  // BF16 output [dense_m, nrows] in `out`; 0 for the MoE form
  int dense_m;
  void* out;
  int out_bf16;
};

__device__ __forceinline__ int i8_chunks(const I8Args& a) {
  return a.dense_m ? (a.dense_m + kI8Tok - 1) / kI8Tok : *a.n_chunks_p;
}
// {expert, tokens, first entry, first tile row} of chunk ci
__device__ __forceinline__ int4 i8_chunk(const I8Args& a, int ci) {
  if (a.dense_m) return make_int4(0, min(kI8Tok, a.dense_m - kI8Tok * ci), kI8Tok * ci, kI8Tok * ci);
  return a.chunk_rec[ci];
}

// Activation codes and scales of the chunks' h rows (compute.py:25-31).
__global__ void __launch_bounds__(256) moe_quant_h_kernel(const I8Args a, int ctok) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  const int n = i8_chunks(a) * ctok * a.nkb;
  for (int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < n; w += warps) {
    const int kb = w % a.nkb, rc = w / a.nkb, ci = rc / ctok, rr = rc % ctok;
    const int4 rec = i8_chunk(a, ci);
    const int r16 = (rec.y + 15) & ~15;
    if (rr >= r16) continue;
    const int64_t xrow = rec.w;
    // values 8 lane .. 8 lane + 7 of the K block: one 16-byte piece of the swizzled BF16 tile
    const uint8_t* tile = a.ht + xrow * 512 * a.nkb + static_cast<int64_t>(kb) * r16 * 512;
    const uint4 v = *reinterpret_cast<const uint4*>(tile + xt_offset(static_cast<uint32_t>(r16), rr, 8 * lane));
    const uint32_t p[4] = {v.x, v.y, v.z, v.w};
    float x[8], m = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      x[i] = bf16_to_f32(static_cast<uint16_t>(p[i >> 1] >> (16 * (i & 1))));
      m = fmaxf(m, fabsf(x[i]));
    }
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));  // the 4 lanes of a 32-value group
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    const float s = __fdiv_rn(m, 127.f);
    const float div = s == 0.f ? 1.f : s;
    uint32_t q[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int c = __float2int_rn(__fdiv_rn(x[i], div));  // rint: ties to even
      c = c < -127 ? -127 : (c > 127 ? 127 : c);
      q[i >> 2] |= (static_cast<uint32_t>(c) & 0xffu) << (8 * (i & 3));
    }
    int8_t* codes = a.qx + xrow * 256 * a.nkb + static_cast<int64_t>(kb) * 256 * r16;
    *reinterpret_cast<uint2*>(codes + (lane >> 1) * (r16 * 16) + rr * 16 + (lane & 1) * 8) = make_uint2(q[0], q[1]);
    if ((lane & 3) == 0) a.qs[xrow * 8 * a.nkb + (static_cast<int64_t>(kb) * 8 + (lane >> 2)) * r16 + rr] = s;
  }
  pdl_trigger();
}

__global__ void __launch_bounds__(kI8Threads, 1) umma_i8_down_kernel(const __grid_constant__ CUtensorMap tm_w,
                                                                     const I8Args A) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kI8Stages * kI8Stage);
  uint64_t* empty = full + kI8Stages;
  uint64_t* dfull = empty + kI8Stages;
  uint64_t* dempty = dfull + 2;
  uint32_t* tmem_sh = reinterpret_cast<uint32_t*>(dempty + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_trigger();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kI8Stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 5);  // the MMA commit and the four epilogue warps (they read the scales)
    }
    for (int d = 0; d < 2; ++d) {
      mbar_init(&dfull[d], 1);
      mbar_init(&dempty[d], 4);
    }
    fence_mbar_init();
  }
  if (warp == 0) tmem_alloc(tmem_sh, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_sh;
  pdl_wait();
  const int n_items = i8_chunks(A) * A.items_per_chunk;
  const int nkb = A.nkb;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      uint32_t sc = 0;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const int ci = item / A.items_per_chunk, p = item % A.items_per_chunk;
        const int4 rec = i8_chunk(A, ci);
        const int r16 = (rec.y + 15) & ~15;
        const int t0 = rec.x * A.tiles64 + 2 * p;
        const int8_t* xsrc = A.qx + static_cast<int64_t>(rec.w) * 256 * nkb;
        const float* ssrc = A.qs + static_cast<int64_t>(rec.w) * 8 * nkb;
        for (int kb = 0; kb < nkb; ++kb, ++sc) {
          const int s = sc % kI8Stages;
          if (sc >= kI8Stages && !mbar_wait_bounded(&empty[s], ((sc / kI8Stages) - 1) & 1)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + s * kI8Stage;
          mbar_expect_tx(&full[s], static_cast<uint32_t>(kI8W + 256 * r16 + 32 * r16));
          tma_load_5d(st, &tm_w, 0, 0, t0, 0, kb, &full[s], pol);
          bulk_g2s(st + kI8W, xsrc + static_cast<int64_t>(kb) * 256 * r16, static_cast<uint32_t>(256 * r16), &full[s]);
          bulk_g2s(st + kI8W + kI8X, ssrc + static_cast<int64_t>(kb) * 8 * r16, static_cast<uint32_t>(32 * r16),
                   &full[s]);
        }
      }
      // every copy issued must have landed before the CTA leaves: instant when the consumers
      // took them all, bounded after a give-up here or in another role
      for (uint32_t i = sc > kI8Stages ? sc - kI8Stages : 0; i < sc; ++i)
          mbar_wait_bounded(&full[i % kI8Stages], (i / kI8Stages) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      uint32_t sc = 0;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const int ci = item / A.items_per_chunk;
        const int r16 = (i8_chunk(A, ci).y + 15) & ~15;
        const uint32_t idesc = idesc_s8_m128(static_cast<uint32_t>(r16));
        for (int kb = 0; kb < nkb; ++kb, ++sc) {
          const int s = sc % kI8Stages;
          const uint32_t d = sc & 1;
          if (!mbar_wait_bounded(&full[s], (sc / kI8Stages) & 1) ||
              (sc >= 2 && !mbar_wait_bounded(&dempty[d], ((sc >> 1) - 1) & 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t ws = smem_addr(smem + s * kI8Stage), xs = ws + kI8W;
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            // weight codes of group g: chunks 1 + 2g, 2 + 2g (2048 bytes apart); 128 rows at 128 B
            const uint64_t ad = sdesc_none(ws + (1 + 2 * g) * 2048u, 2048u, 128u);
            // activation codes of group g: chunks 2g, 2g + 1 (r16 * 16 bytes apart)
            const uint64_t bd = sdesc_none(xs + static_cast<uint32_t>(2 * g * r16 * 16), static_cast<uint32_t>(r16 * 16), 128u);
            umma_s8_ss(tbase + d * 256 + g * 32, ad, bd, idesc);
          }
          umma_commit(&dfull[d]);
          umma_commit(&empty[s]);
        }
      }
    }
  } else {
    // ---------------- epilogue: warps 2..5, TMEM lane quadrant warp % 4 ----------------
    const int quad = warp & 3, row = 32 * quad + lane;  // MMA row: tile row / 64, row % 64
    const int tile = row >> 6, trow = row & 63;
    uint32_t sc = 0;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      const int ci = item / A.items_per_chunk, p = item % A.items_per_chunk;
      const int4 rec = i8_chunk(A, ci);
      const int ntok = rec.y, r16 = (ntok + 15) & ~15;
      float acc[kI8Tok];
#pragma unroll
      for (int j = 0; j < kI8Tok; ++j) acc[j] = 0.f;
      for (int kb = 0; kb < nkb; ++kb, ++sc) {
        const int s = sc % kI8Stages;
        const uint32_t d = sc & 1;
        if (!mbar_wait_bounded(&dfull[d], (sc >> 1) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint8_t* st = smem + s * kI8Stage;
        const float* xsc = reinterpret_cast<const float*>(st + kI8W + kI8X);
        const int ngr = min(8, A.ngroups - 8 * kb);
        for (int g = 0; g < ngr; ++g) {
          uint32_t v[32];
          tmem_ld32(tbase + (static_cast<uint32_t>(32 * quad) << 16) + d * 256 + g * 32, v);
          tmem_wait_ld();
          // this row's FP16 weight scale of block 8 kb + g: chunk 0 of its tile
          const float sw = f16_to_f32(*reinterpret_cast<const uint16_t*>(st + tile * 1024 + trow * 16 + 2 * g));
#pragma unroll
          for (int j = 0; j < kI8Tok; ++j)
            if (j < ntok)
              acc[j] = __fadd_rn(acc[j], __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int32_t>(v[j])),
                                                             xsc[g * r16 + j]),
                                                   sw));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&dempty[d]);
          mbar_arrive(&empty[s]);
        }
      }
      if (!ok) break;
      const int R = 128 * p + row;
      if (R < A.nrows) {
#pragma unroll
        for (int j = 0; j < kI8Tok; ++j) {
          if (j >= ntok) break;
          const int64_t e = rec.z + j;
          if (A.dense_m) {
            if (A.out_bf16) static_cast<uint16_t*>(A.out)[e * A.nrows + R] = bf16_bits_rne(acc[j]);
            else static_cast<float*>(A.out)[e * A.nrows + R] = acc[j];
          } else if (A.yr) {
            A.yr[static_cast<int64_t>(A.entry_route[e]) * A.nrows + R] = acc[j];
          } else {
            A.y[e * A.nrows + R] = bf16_bits_rne(acc[j]);
          }
        }
      }
    }
  }

  if (!ok && lane == 0 && A.status) atomicExch(A.status, QK_ERR_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The W8A8 pass over `a`: activation codes and scales, then the integer-MMA projection.
// `w` is the tiled Q8_0 matrix of `ntiles` 64-row tiles, viewed as 5 dimensions - 16 bytes,
// 64 rows, tile (stride one tile row of blocks), chunk (1024 B), K block (one tile) - so that
// one box of 16 x 64 x 2 x 17 x 1 lands as [chunk][tile][row][16 B]: the two tiles of a
// 128-row MMA operand interleaved per 16-byte chunk. A box reaching past the last tile reads
// zeros.
int launch_w8a8(const I8Args& a, const uint8_t* w, int64_t ntiles, int sms, cudaStream_t st) {
  EncodeTiledFn enc = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!enc) return set_error(QK_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  constexpr int TB = HalfTile<QType::Q8_0>::kBytes;
  const cuuint64_t dims[5] = {16, 64, static_cast<cuuint64_t>(ntiles), 17, static_cast<cuuint64_t>(a.nkb)};
  const cuuint64_t strides[4] = {16, static_cast<cuuint64_t>(a.nkb) * TB, 1024, TB};
  const cuuint32_t box[5] = {16, 64, 2, 17, 1};
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUtensorMap map;
  memset(&map, 0, sizeof(map));
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 5, const_cast<uint8_t*>(w), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return set_error(QK_ERR_CUDA, "cuTensorMapEncodeTiled refused the Q8_0 tile map");
  cudaError_t e = launch_dependent(moe_quant_h_kernel, dim3(static_cast<unsigned>(sms * 8)), dim3(256), 0, st, a,
                                   static_cast<int>(kI8Tok));
  if (e != cudaSuccess) return cuda_error(e, "moe_quant_h_kernel");
  count_launch(1);
  int rc = allow_smem(reinterpret_cast<const void*>(umma_i8_down_kernel), kI8Smem);
  if (rc) return rc;
  e = launch_dependent(umma_i8_down_kernel, dim3(sms), dim3(kI8Threads), kI8Smem, st, map, a);
  if (e != cudaSuccess) return cuda_error(e, "umma_i8_down_kernel");
  count_launch(1);
  return QK_OK;
}

}  // namespace
}  // namespace qk
