// Elementwise FP32 numerics of the kernels, evaluated on the GPU for validation.
//
// The reference pins its FP32 nonlinear arithmetic (qwen38_tpu/numerics.py:13-51: exp,
// divide, sigmoid, softmax) against an FP64 host oracle with a 5e-7 per-element relative
// budget (numerics_validation.py:12-74). The kernels here compute the same functions with
// the device helpers of common.cuh; qk_numerics runs exactly those helpers over caller
// buffers so that a test can hold them to the same budget:
//   QK_NUM_EXP       out = exp_ref(a)                       (router, attention, sigmoid)
//   QK_NUM_SIGMOID   out = sigmoid_ref(a)                   (SwiGLU, shared-expert gate)
//   QK_NUM_DIVIDE    out = a / b, IEEE round-to-nearest     (router renormalisation)
//   QK_NUM_SOFTMAX   rows of `row_len` values of a          (the router's softmax_row_warp)
//   QK_NUM_SILU_BF16 out = bf16(bf16(a) * sigmoid(bf16(a)))  (the SwiGLU epilogue's activation)
#include "common.cuh"

namespace qk {
namespace {

__global__ void numerics_elementwise_kernel(int op, const float* __restrict__ a, const float* __restrict__ b,
                                            float* __restrict__ out, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float x = a[i];
    float y;
    switch (op) {
      case QK_NUM_EXP: y = exp_ref(x); break;
      case QK_NUM_SIGMOID: y = sigmoid_ref(x); break;
      case QK_NUM_DIVIDE: y = __fdiv_rn(x, b[i]); break;
      default: {  // QK_NUM_SILU_BF16, as the gate/up epilogue computes it
        const float g = bf16_round(x);
        y = bf16_round(__fmul_rn(g, sigmoid_ref(g)));
      }
    }
    out[i] = y;
  }
}

// One warp per row: the row is copied to `out` and normalised there in place.
__global__ void numerics_softmax_kernel(const float* __restrict__ a, float* __restrict__ out, int64_t rows,
                                        int row_len) {
  const int lane = threadIdx.x & 31;
  const int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (r >= rows) return;
  float* row = out + r * row_len;
  for (int e = lane; e < row_len; e += 32) row[e] = a[r * row_len + e];
  __syncwarp();
  softmax_row_warp(row, row_len, lane);
}

}  // namespace
}  // namespace qk

using namespace qk;

extern "C" {

int qk_numerics(int op, const float* a, const float* b, float* out, int64_t n, int row_len, qk_stream_t stream) {
  QK_REQUIRE(op >= QK_NUM_EXP && op <= QK_NUM_SILU_BF16, "unknown numerics op %d", op);
  QK_REQUIRE(n >= 0, "n must be non-negative");
  if (n == 0) return QK_OK;
  QK_REQUIRE(a && out && (op != QK_NUM_DIVIDE || b), "null pointer");
  cudaStream_t st = as_stream(stream);
  if (op == QK_NUM_SOFTMAX) {
    QK_REQUIRE(row_len > 0 && n % row_len == 0, "softmax rows: n must be a multiple of row_len > 0");
    const int64_t rows = n / row_len;
    numerics_softmax_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, st>>>(a, out, rows, row_len);
    QK_LAUNCHED("numerics_softmax_kernel");
    return QK_OK;
  }
  int64_t grid = (n + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  numerics_elementwise_kernel<<<static_cast<unsigned>(grid > cap ? cap : grid), 256, 0, st>>>(op, a, b, out, n);
  QK_LAUNCHED("numerics_elementwise_kernel");
  return QK_OK;
}

}  // extern "C"
