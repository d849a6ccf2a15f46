// Packed-weight projection: out[M, N] (FP32) = bf16 x[M, K] @ bf16(decode(W))[N, K]^T.
//
// Replaces packed_q6/kernel.py:98-148 (q6_matmul) and its XLA baseline
// packed_q6/baselines.py:33-39: weights stay packed in HBM (tiled Q6_K or Q4_K), each
// warp streams its 16-row strip's tiles through a shared-memory ring (bulk copies) and
// decodes them into BF16 MMA fragments in registers; FP32 accumulation. Ragged M, N
// and K are handled like the reference (zero-padded x, cropped output): positions at
// or beyond K read x as zero, rows at or beyond N / M are not stored.
#include "common.cuh"
#include "proj.cuh"

namespace qk {
namespace {

template <QType QT>
__global__ void __launch_bounds__(kWarps * 32, 1) quant_gemm_kernel(const uint16_t* __restrict__ x,
                                                                   int M, int K,
                                                                   const uint8_t* __restrict__ w,
                                                                   int N, float* __restrict__ out,
                                                                   int32_t* status) {
  using Cfg = ProjCfg<QT, false>;
  constexpr int TB = Tile<QT>::kBytes, R = Cfg::kStages;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  uint8_t* ring = smem + static_cast<size_t>(warp) * R * Cfg::kStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(kWarps) * R * Cfg::kStage) + warp * R;

  const int strips = (N + 15) / 16, nkb = (K + 255) / 256, mchunks = (M + kChunk - 1) / kChunk;
  const int n_items = strips * mchunks;
  const int total = gridDim.x * kWarps;
  const int first = blockIdx.x * kWarps + warp;
  if (first >= n_items) return;
  if (lane == 0) {
    for (int i = 0; i < R; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  __syncwarp();

  // Tile stream: items first, first + total, ...; each item = nkb tiles of one strip.
  int p_item = first, p_kb = 0;
  uint32_t tp = 0, tc = 0;
  auto issue = [&]() {
    if (lane == 0) {
      const uint32_t slot = tp % R;
      const int strip = p_item % strips;
      mbar_expect_tx(&bars[slot], TB);
      bulk_g2s(ring + slot * Cfg::kStage, w + (static_cast<int64_t>(strip) * nkb + p_kb) * TB, TB, &bars[slot]);
    }
    ++tp;
    if (++p_kb == nkb) {
      p_kb = 0;
      p_item += total;
    }
  };
  for (int i = 0; i < R && p_item < n_items; ++i) issue();

  const bool ragged = (K % 256) != 0;
  bool ok = true;
  for (int item = first; item < n_items && ok; item += total) {
    const int strip = item % strips, chunk = item / strips;
    const int ntok = min(kChunk, M - chunk * kChunk);
    const int J = (ntok + 7) / 8;
    const uint16_t* rows[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int m = chunk * kChunk + 8 * j + g;
      rows[j] = (8 * j + g < ntok) ? x + static_cast<int64_t>(m) * K : nullptr;
    }
    // One fresh FP32 partial sum per 256-value block, added to the running total: keeps
    // the accumulator small while the MMAs sum, as the reference's per-block dot does.
    float acc[4][4] = {}, unused[4][4];
    for (int kb = 0; kb < nkb; ++kb) {
      float blk[4][4] = {};
      const uint32_t slot = tc % R;
      if (!mbar_wait_bounded(&bars[slot], (tc / R) & 1)) {
        ok = false;
        break;
      }
      const uint8_t* stage = ring + slot * Cfg::kStage;
      const bool safe = ragged && kb == nkb - 1;
      if (safe || (K & 7)) {
        if (J == 1) proj_stage<QT, false, 1, true>(stage, lane, kb * 256, K, rows, blk, unused);
        else if (J == 2) proj_stage<QT, false, 2, true>(stage, lane, kb * 256, K, rows, blk, unused);
        else proj_stage<QT, false, 4, true>(stage, lane, kb * 256, K, rows, blk, unused);
      } else {
        if (J == 1) proj_stage<QT, false, 1, false>(stage, lane, kb * 256, K, rows, blk, unused);
        else if (J == 2) proj_stage<QT, false, 2, false>(stage, lane, kb * 256, K, rows, blk, unused);
        else proj_stage<QT, false, 4, false>(stage, lane, kb * 256, K, rows, blk, unused);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[j][i] = __fadd_rn(acc[j][i], blk[j][i]);
      ++tc;
      __syncwarp();
      if (lane == 0) fence_proxy_async_smem();
      if (p_item < n_items) issue();
    }
    if (!ok) break;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j >= J) break;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int col = 8 * j + 2 * c + (i & 1);
        const int n = strip * 16 + g + (i >> 1) * 8;
        if (col < ntok && n < N) out[static_cast<int64_t>(chunk * kChunk + col) * N + n] = acc[j][i];
      }
    }
  }
  if (!ok) {
    if (lane == 0 && status) atomicExch(status, QK_ERR_TIMEOUT);
    while (tc < tp) {
      mbar_wait_bounded(&bars[tc % R], (tc / R) & 1);
      ++tc;
    }
  }
}

}  // namespace
}  // namespace qk

using namespace qk;

extern "C" int qk_quant_gemm(const uint16_t* x, int64_t M, int64_t K, const uint8_t* w_tiled,
                             int qtype, int64_t N, float* out, qk_stream_t stream) {
  if (qtype != QK_TYPE_Q6_K && qtype != QK_TYPE_Q4_K)
    return set_error(QK_ERR_UNSUPPORTED_TYPE, "packed projection supports Q6_K and Q4_K; got %d", qtype);
  QK_REQUIRE(M >= 0 && K > 0 && N > 0, "x must be a nonempty [M,K] BF16 array");
  QK_REQUIRE(M < (1 << 30) && K < (1 << 30) && N < (1 << 30), "dimension too large");
  if (M == 0) return QK_OK;
  QK_REQUIRE(x && w_tiled && out, "null pointer");
  QK_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15) == 0 || (K & 7), "x must be 16-byte aligned");
  const int64_t items = (N + 15) / 16 * ((M + kChunk - 1) / kChunk);
  const int sms = sm_count();
  int grid = static_cast<int>((items + kWarps - 1) / kWarps);
  grid = grid > sms ? sms : grid;
  cudaStream_t st = as_stream(stream);
  int rc;
  if (qtype == QK_TYPE_Q6_K) {
    using Cfg = ProjCfg<QType::Q6_K, false>;
    if ((rc = allow_smem(reinterpret_cast<const void*>(quant_gemm_kernel<QType::Q6_K>), Cfg::kSmem))) return rc;
    quant_gemm_kernel<QType::Q6_K><<<grid, kWarps * 32, Cfg::kSmem, st>>>(x, (int)M, (int)K, w_tiled, (int)N, out, nullptr);
  } else {
    using Cfg = ProjCfg<QType::Q4_K, false>;
    if ((rc = allow_smem(reinterpret_cast<const void*>(quant_gemm_kernel<QType::Q4_K>), Cfg::kSmem))) return rc;
    quant_gemm_kernel<QType::Q4_K><<<grid, kWarps * 32, Cfg::kSmem, st>>>(x, (int)M, (int)K, w_tiled, (int)N, out, nullptr);
  }
  QK_LAUNCHED("quant_gemm_kernel");
  return QK_OK;
}
