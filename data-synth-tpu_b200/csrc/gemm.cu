// Packed-weight projection: out[M, N] (FP32) = bf16 x[M, K] @ bf16(decode(W))[N, K]^T.
//
// Replaces packed_q6/kernel.py:98-148 (q6_matmul) and its XLA baseline
// packed_q6/baselines.py:33-39. The weights stay packed in HBM (64-row Q6_K / Q4_K tiles);
// the tcgen05 pass of umma_proj.cuh decodes them into TMEM and multiplies with FP32
// accumulation. x is first packed into the tensor core's activation-tile layout (chunks of
// 32 rows, zero padding for ragged M and K, as the reference zero-pads, kernel.py:139-140);
// rows at or beyond N are not stored.
#include "common.cuh"
#include "umma_i8.cuh"
#include "umma_proj.cuh"

namespace qk {
namespace {

__host__ __device__ inline int64_t dense_tile_rows(int64_t M) {
  const int64_t full = M / kMaxTok, rest = M % kMaxTok;
  return full * kMaxTok + ((rest + 15) & ~int64_t(15));
}

// x [M, K] (any K, any alignment) -> activation tiles [chunk][kb][r16 x 512 B].
__global__ void __launch_bounds__(256) pack_x_kernel(const uint16_t* __restrict__ x, int M, int K,
                                                     int nkb, uint8_t* __restrict__ xt) {
  pdl_trigger();
  const int64_t rows = dense_tile_rows(M);
  const int cpr = nkb * 32;  // 16-byte chunks of one padded row
  const int64_t total = rows * cpr;
  const bool aligned = (K & 7) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t g = i / cpr;
    const int j = static_cast<int>(i % cpr);
    const int ch = static_cast<int>(g / kMaxTok), rr = static_cast<int>(g % kMaxTok);
    const int ntok = min(kMaxTok, M - kMaxTok * ch), r16 = (ntok + 15) & ~15;
    const int k = j * 8;
    uint32_t w[4] = {0, 0, 0, 0};
    if (rr < ntok) {
      const uint16_t* src = x + g * K;
      if (aligned && k + 8 <= K) {
        const uint4 v = ld_nc_v4(src + k);
        w[0] = v.x, w[1] = v.y, w[2] = v.z, w[3] = v.w;
      } else {
        for (int e = 0; e < 8; ++e)
          if (k + e < K) w[e >> 1] |= static_cast<uint32_t>(src[k + e]) << (16 * (e & 1));
      }
    }
    uint8_t* dst = xt + static_cast<int64_t>(kMaxTok) * ch * 512 * nkb +
                   static_cast<int64_t>(k >> 8) * r16 * 512 + xt_offset(r16, rr, k & 255);
    *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// out[m, n] = sum over K blocks, in K order, of the block partials [nkb, M, N].
__global__ void reduce_blocks_kernel(const float* __restrict__ part, int64_t mn, int nkb, float* __restrict__ out) {
  pdl_wait();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < mn;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float acc = part[i];
    for (int kb = 1; kb < nkb; ++kb) acc = __fadd_rn(acc, part[kb * mn + i]);
    out[i] = acc;
  }
}

size_t xt_bytes(int64_t M, int64_t K) {
  return static_cast<size_t>(dense_tile_rows(M)) * 512 * static_cast<size_t>((K + 255) / 256);
}

}  // namespace
}  // namespace qk

using namespace qk;

extern "C" {

size_t qk_quant_gemm_workspace_bytes(int64_t M, int64_t K, int64_t N) {
  if (M <= 0 || K <= 0 || N <= 0) return 0;
  const int64_t nkb = (K + 255) / 256;
  return xt_bytes(M, K) + (nkb > 1 ? static_cast<size_t>(nkb * M * N) * 4 : 0);
}

int qk_quant_gemm(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w_tiled, int qtype,
                  int64_t N, float* out, void* workspace, size_t workspace_bytes, qk_stream_t stream) {
  if (qtype != QK_TYPE_Q6_K && qtype != QK_TYPE_Q4_K && qtype != QK_TYPE_Q8_0 && qtype != QK_TYPE_Q5_K &&
      qtype != QK_TYPE_Q5_1)
    return set_error(QK_ERR_UNSUPPORTED_TYPE, "packed projection supports Q6_K, Q4_K, Q5_K, Q8_0 and Q5_1; got %d",
                     qtype);
  QK_REQUIRE(M >= 0 && K > 0 && N > 0, "x must be a nonempty [M,K] BF16 array");
  QK_REQUIRE(M < (1 << 30) && K < (1 << 30) && N < (1 << 30), "dimension too large");
  if (M == 0) return QK_OK;
  QK_REQUIRE(x && w_tiled && out, "null pointer");
  const size_t need = qk_quant_gemm_workspace_bytes(M, K, N);
  if (!workspace || workspace_bytes < need)
    return set_error(QK_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", need, workspace_bytes);
  cudaStream_t st = as_stream(stream);
  const int nkb = static_cast<int>((K + 255) / 256);
  const int sms = sm_count();
  int64_t pgrid = (dense_tile_rows(M) * nkb * 32 + 255) / 256;
  if (pgrid > sms * 16) pgrid = sms * 16;
  pack_x_kernel<<<static_cast<unsigned>(pgrid), 256, 0, st>>>(x, static_cast<int>(M), static_cast<int>(K), nkb,
                                                              static_cast<uint8_t*>(workspace));
  QK_LAUNCHED("pack_x_kernel");

  UArgs a{};
  a.wa = w_tiled;
  a.expert_bytes = 0;
  a.nkb = nkb;
  a.tiles64 = static_cast<int>((N + kTileRows - 1) / kTileRows);
  a.items_per_chunk = static_cast<int>((N + 2 * kTileRows - 1) / (2 * kTileRows));
  a.xt = static_cast<const uint8_t*>(workspace);
  a.n_chunks_dense = static_cast<int>((M + kMaxTok - 1) / kMaxTok);
  a.m_dense = static_cast<int>(M);
  a.nrows = static_cast<int>(N);
  // Split K: one item per 256-value block writes its FP32 partial sum; the partials are
  // then added in K order (the per-block accumulation of packed_q6/kernel.py:95-107).
  a.ksplit = nkb > 1;
  a.out = a.ksplit ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + xt_bytes(M, K)) : out;
  const int64_t items = static_cast<int64_t>(a.n_chunks_dense) * a.items_per_chunk * (a.ksplit ? nkb : 1);
  const int grid = static_cast<int>(items < sms ? items : sms);
  int rc = qtype == QK_TYPE_Q6_K   ? launch_umma<QType::Q6_K, kModeDense>(a, grid, st)
           : qtype == QK_TYPE_Q4_K ? launch_umma<QType::Q4_K, kModeDense>(a, grid, st)
           : qtype == QK_TYPE_Q5_K ? launch_umma<QType::Q5_K, kModeDense>(a, grid, st)
           : qtype == QK_TYPE_Q5_1 ? launch_umma<QType::Q5_1, kModeDense>(a, grid, st)
                                   : launch_umma<QType::Q8_0, kModeDense>(a, grid, st);
  if (rc || !a.ksplit) return rc;
  const int64_t mn = M * N;
  int64_t rgrid = (mn + 255) / 256;
  if (rgrid > sms * 8) rgrid = sms * 8;
  const cudaError_t e = launch_dependent(reduce_blocks_kernel, dim3(static_cast<unsigned>(rgrid)), dim3(256), 0, st,
                                         static_cast<const float*>(a.out), mn, nkb, out);
  if (e != cudaSuccess) return cuda_error(e, "reduce_blocks_kernel");
  count_launch(1);
  return QK_OK;
}

// ---- W8A8 projection (qwen38_tpu/compute.py:20-34, q8_matmul) ----
// Workspace: the BF16 activation tiles of x, the int8 codes [chunks x 32 rows x K256] and the
// FP32 scales [chunks x 32 rows x K256 / 32] (K256: K rounded up to 256).
static size_t q8mm_parts(int64_t M, int64_t K, size_t* codes_off, size_t* scales_off) {
  const int64_t rows = (M + kMaxTok - 1) / kMaxTok * kMaxTok, k256 = (K + 255) / 256 * 256;
  const size_t xt = (xt_bytes(M, K) + 255) & ~size_t(255);
  const size_t codes = (static_cast<size_t>(rows * k256) + 255) & ~size_t(255);
  *codes_off = xt;
  *scales_off = xt + codes;
  return xt + codes + static_cast<size_t>(rows * (k256 / 32)) * 4;
}

size_t qk_q8_matmul_workspace_bytes(int64_t M, int64_t K, int64_t N) {
  if (M <= 0 || K <= 0 || N <= 0) return 0;
  size_t c, s;
  return q8mm_parts(M, K, &c, &s);
}

int qk_q8_matmul(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w_tiled, int64_t N, int out_dtype,
                 void* out, void* workspace, size_t workspace_bytes, qk_stream_t stream) {
  QK_REQUIRE(M >= 0 && K > 0 && N > 0, "x must be a nonempty [M,K] BF16 array");
  QK_REQUIRE(K % 32 == 0, "Q8_0 input features must be a multiple of 32");
  QK_REQUIRE(M < (1 << 30) && K < (1 << 20) && N < (1 << 24), "dimension too large");
  QK_REQUIRE(out_dtype == QK_OUT_F32 || out_dtype == QK_OUT_BF16, "out_dtype must be F32 or BF16");
  if (M == 0) return QK_OK;
  QK_REQUIRE(x && w_tiled && out, "null pointer");
  size_t codes_off, scales_off;
  const size_t need = q8mm_parts(M, K, &codes_off, &scales_off);
  if (!workspace || workspace_bytes < need)
    return set_error(QK_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", need, workspace_bytes);
  QK_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, "workspace must be 256-byte aligned");
  QK_REQUIRE((reinterpret_cast<uintptr_t>(w_tiled) & 15) == 0, "tiled weights must be 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  const int sms = sm_count();
  const int nkb = static_cast<int>((K + 255) / 256);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  {
    const int64_t total = dense_tile_rows(M) * nkb * 32;
    int64_t g = (total + 255) / 256;
    if (g > sms * 8) g = sms * 8;
    pack_x_kernel<<<static_cast<unsigned>(g), 256, 0, st>>>(x, static_cast<int>(M), static_cast<int>(K), nkb, ws);
    QK_LAUNCHED("pack_x_kernel");
  }
  I8Args a{};
  a.ht = ws;
  a.qx = reinterpret_cast<int8_t*>(ws + codes_off);
  a.qs = reinterpret_cast<float*>(ws + scales_off);
  a.nkb = nkb;
  a.ngroups = static_cast<int>(K / 32);
  a.items_per_chunk = static_cast<int>((N + 127) / 128);
  a.tiles64 = 0;  // one matrix: tile 2p of item p
  a.nrows = static_cast<int>(N);
  a.dense_m = static_cast<int>(M);
  a.out = out;
  a.out_bf16 = out_dtype == QK_OUT_BF16;
  return launch_w8a8(a, w_tiled, (N + kTileRows - 1) / kTileRows, sms, st);
}

}  // extern "C"
