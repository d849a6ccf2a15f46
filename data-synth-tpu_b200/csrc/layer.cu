// The small per-token operations on either side of the routed-expert FFN and the Q8 decode
// attention in a decoder layer (qwen38_tpu/math.py, attention_cache.py:128-150,
// math.py:277-284): RMSNorm, the per-head q/k RMSNorm + rotary embedding of the attention
// step, the shared expert's route, and the residual add. Each is one launch over all rows,
// so a decode step of many layers is not bound by launches of tiny elementwise kernels.
// These are latency-bound (a few KB per row); one block per row (or row x head).
#include "common.cuh"

namespace qk {
namespace {

constexpr int kRowThreads = 256;

static_assert(kRowThreads == kRowBlock, "the row kernels use the common row layout");

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int t = 0; t < 4; ++t)
    w[t] = static_cast<uint32_t>(bf16_bits_rne(f[2 * t])) | (static_cast<uint32_t>(bf16_bits_rne(f[2 * t + 1])) << 16);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// out = bf16(v * r * gamma) for the row's chunks held in registers, r = rsqrt(mean(v^2) + eps)
// from the threads' sums of squares `ss` (math.py:27-31).
__device__ __forceinline__ void rms_finish(const uint4 (&v)[kRowChunks], float ss, float* red, const uint16_t* gamma,
                                           int width, float eps, uint16_t* orow) {
  const int nch = width / 8;
  const float r = rsqrtf(__fadd_rn(__fdiv_rn(block_sum(ss, red), static_cast<float>(width)), eps));
  uint4 g[kRowChunks];
#pragma unroll
  for (int c = 0; c < kRowChunks; ++c) {
    const int i = threadIdx.x + c * kRowThreads;
    g[c] = i < nch ? reinterpret_cast<const uint4*>(gamma)[i] : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int c = 0; c < kRowChunks; ++c) {
    const int i = threadIdx.x + c * kRowThreads;
    if (i >= nch) break;
    float f[8], gf[8];
    unpack8(v[c], f);
    unpack8(g[c], gf);
#pragma unroll
    for (int t = 0; t < 8; ++t) f[t] = __fmul_rn(__fmul_rn(f[t], r), gf[t]);
    reinterpret_cast<uint4*>(orow)[i] = pack8(f);
  }
}

// math.py:27-31 rms: bf16(xf * rsqrt(mean(xf^2) + eps) * gamma), one block per row, the row
// held in registers (one round of loads instead of one per 256 values).
__global__ void __launch_bounds__(kRowThreads) rms_norm_kernel(const uint16_t* __restrict__ x,
                                                               const uint16_t* __restrict__ gamma, int width,
                                                               float eps, uint16_t* __restrict__ out) {
  pdl_wait();  // launched as a programmatic dependent: the previous kernel's outputs first
  pdl_trigger();
  __shared__ float red[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * width);
  const int nch = width / 8;
  uint4 v[kRowChunks];
#pragma unroll
  for (int c = 0; c < kRowChunks; ++c) {
    const int i = threadIdx.x + c * kRowThreads;
    v[c] = i < nch ? xr[i] : make_uint4(0, 0, 0, 0);
  }
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kRowChunks; ++c) {
    if (threadIdx.x + c * kRowThreads >= nch) break;
    float f[8];
    unpack8(v[c], f);
#pragma unroll
    for (int t = 0; t < 8; ++t) ss = fmaf(f[t], f[t], ss);
  }
  rms_finish(v, ss, red, gamma, width, eps, out + row * width);
}

// The residual add and the RMSNorm that follows it, one block per row: xo = bf16(x + y)
// (stored; xo may alias x), then out = rms(xo) as rms_norm_kernel computes it (the same
// chunk layout and reduction over the BF16 sums), so one launch gives the bits of
// qk_residual_add + qk_rms_norm.
__global__ void __launch_bounds__(kRowThreads) residual_rms_norm_kernel(const uint16_t* x, const uint16_t* __restrict__ y,
                                                                        const uint16_t* __restrict__ gamma, int width,
                                                                        float eps, uint16_t* xo,
                                                                        uint16_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[kRowThreads / 32];
  const int64_t row = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * width);
  const uint4* yr = reinterpret_cast<const uint4*>(y + row * width);
  const int nch = width / 8;
  uint4 v[kRowChunks], u[kRowChunks];
#pragma unroll
  for (int c = 0; c < kRowChunks; ++c) {
    const int i = threadIdx.x + c * kRowThreads;
    v[c] = i < nch ? xr[i] : make_uint4(0, 0, 0, 0);
    u[c] = i < nch ? yr[i] : make_uint4(0, 0, 0, 0);
  }
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < kRowChunks; ++c) {
    const int i = threadIdx.x + c * kRowThreads;
    if (i >= nch) break;
    float f[8], g[8];
    unpack8(v[c], f);
    unpack8(u[c], g);
#pragma unroll
    for (int t = 0; t < 8; ++t) f[t] = __fadd_rn(f[t], g[t]);
    v[c] = pack8(f);  // the BF16 sum: stored, and the RMSNorm's input
    reinterpret_cast<uint4*>(xo + row * width)[i] = v[c];
    unpack8(v[c], f);
#pragma unroll
    for (int t = 0; t < 8; ++t) ss = fmaf(f[t], f[t], ss);
  }
  rms_finish(v, ss, red, gamma, width, eps, out + row * width);
}

// attention_cache.py:129-135: the fused projection output of one row is
// [hq x (q hd | gate hd)] [kv x k hd] [kv x v hd] (BF16). Block (row, head slot):
// slots < hq are query heads (rms with q_norm, rotary, and the gate copied out), the
// next kv slots are key heads (rms with k_norm, rotary) with their value heads copied out.
// Rotary (math.py:231-243 with one position for every section): dims i < half and
// i + half of the first `rotary` dims rotate by angle position * inv_freq[i], with the
// cosine and sine rounded to BF16; the rest pass through.
__global__ void __launch_bounds__(kRowThreads) qk_norm_rope_kernel(
    const uint16_t* __restrict__ qkv, const uint16_t* __restrict__ q_norm, const uint16_t* __restrict__ k_norm,
    const float* __restrict__ inv_freq, const int32_t* __restrict__ positions, int hq, int kv, int hd, int rotary,
    float eps, uint16_t* __restrict__ q_out, uint16_t* __restrict__ gate_out, uint16_t* __restrict__ k_out,
    uint16_t* __restrict__ v_out) {
  pdl_wait();  // launched as a programmatic dependent: the previous kernel's outputs first
  pdl_trigger();
  __shared__ float red[kRowThreads / 32];
  __shared__ float normed[512];
  const int64_t b = blockIdx.x;
  const int slot = blockIdx.y, d = threadIdx.x;
  const int64_t width = static_cast<int64_t>(2 * hq + 2 * kv) * hd;
  const uint16_t* row = qkv + b * width;
  const bool query = slot < hq;
  const uint16_t* src = query ? row + static_cast<int64_t>(slot) * 2 * hd : row + static_cast<int64_t>(2 * hq + slot - hq) * hd;
  const uint16_t* gamma = query ? q_norm : k_norm;
  const float v = d < hd ? bf16_to_f32(src[d]) : 0.f;
  const float r = rsqrtf(__fadd_rn(__fdiv_rn(block_sum(v * v, red), static_cast<float>(hd)), eps));
  if (d < hd) normed[d] = bf16_round(__fmul_rn(__fmul_rn(v, r), bf16_to_f32(gamma[d])));
  __syncthreads();
  if (d >= hd) return;
  float o = normed[d];
  const int half = rotary / 2;
  if (d < rotary) {
    const int i = d < half ? d : d - half;
    const float angle = __fmul_rn(static_cast<float>(positions[b]), inv_freq[i]);
    const float cs = bf16_round(cosf(angle)), sn = bf16_round(sinf(angle));
    const float a = normed[i], c = normed[i + half];
    o = d < half ? __fsub_rn(__fmul_rn(a, cs), __fmul_rn(c, sn)) : __fadd_rn(__fmul_rn(c, cs), __fmul_rn(a, sn));
  }
  if (query) {
    const int64_t oi = (b * hq + slot) * hd + d;
    q_out[oi] = bf16_bits_rne(o);
    gate_out[oi] = src[hd + d];
  } else {
    const int h = slot - hq;
    const int64_t oi = (b * kv + h) * hd + d;
    k_out[oi] = bf16_bits_rne(o);
    v_out[oi] = row[static_cast<int64_t>(2 * hq + kv + h) * hd + d];
  }
}

// out = bf16(f32(x) + f32(y)) over n values (out may alias x).
__global__ void residual_add_kernel(const uint16_t* x, const uint16_t* __restrict__ y, int64_t n, uint16_t* out) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = bf16_bits_rne(__fadd_rn(bf16_to_f32(x[i]), bf16_to_f32(y[i])));
}

// Routes of each row plus one route to the shared expert: ids_out[b] = ids[b] ++ shared_id,
// w_out[b] = w[b] ++ bf16(sigmoid(bf16(h[b] . wsr))) (math.py:282-283, the shared expert's
// sigmoid gate). One block per row.
// per > 0 (expert parallel): routed expert e is renumbered (e / per) * (per + 1) + e % per, so
// each rank's slice of `per` routed experts is followed by one more local slot (its copy of
// the shared expert); shared_id is then the caller's own slot.
__global__ void __launch_bounds__(kRowThreads) append_shared_route_kernel(
    const int32_t* __restrict__ ids, const uint16_t* __restrict__ w, int k, const uint16_t* __restrict__ h,
    const uint16_t* __restrict__ wsr, int H, int shared_id, int per, int32_t* __restrict__ ids_out,
    uint16_t* __restrict__ w_out) {
  pdl_wait();  // launched as a programmatic dependent: the previous kernel's outputs first
  pdl_trigger();
  __shared__ float red[kRowThreads / 32];
  const int64_t b = blockIdx.x;
  const float dot = row_dot_bf16(h + b * H, wsr, H, red);
  if (threadIdx.x < k) {
    const int e = ids[b * k + threadIdx.x];
    ids_out[b * (k + 1) + threadIdx.x] = per > 0 && e >= 0 ? (e / per) * (per + 1) + e % per : e;
    w_out[b * (k + 1) + threadIdx.x] = w[b * k + threadIdx.x];
  }
  if (threadIdx.x == 0) {
    ids_out[b * (k + 1) + k] = shared_id;
    w_out[b * (k + 1) + k] = bf16_bits_rne(sigmoid_ref(dot));
  }
}

}  // namespace
}  // namespace qk

using namespace qk;

extern "C" {

int qk_rms_norm(const uint16_t* x, const uint16_t* gamma, int rows, int width, float eps, uint16_t* out,
                qk_stream_t stream) {
  QK_REQUIRE(rows >= 0 && width > 0 && width % 8 == 0 && width <= kMaxRowWidth,
             "rms width must be a positive multiple of 8 up to %d", kMaxRowWidth);
  if (rows == 0) return QK_OK;
  QK_REQUIRE(x && gamma && out, "null pointer");
  QK_REQUIRE(((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(out)) & 15) == 0,
             "x, gamma and out must be 16-byte aligned");
  const cudaError_t e = launch_dependent(rms_norm_kernel, dim3(rows), dim3(kRowThreads), 0, as_stream(stream), x, gamma,
                                         width, eps, out);
  if (e != cudaSuccess) return cuda_error(e, "rms_norm_kernel");
  count_launch();
  return QK_OK;
}

int qk_residual_rms_norm(const uint16_t* x, const uint16_t* y, const uint16_t* gamma, int rows, int width, float eps,
                         uint16_t* x_out, uint16_t* out, qk_stream_t stream) {
  QK_REQUIRE(rows >= 0 && width > 0 && width % 8 == 0 && width <= kMaxRowWidth,
             "rms width must be a positive multiple of 8 up to %d", kMaxRowWidth);
  if (rows == 0) return QK_OK;
  QK_REQUIRE(x && y && gamma && x_out && out, "null pointer");
  QK_REQUIRE(((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(gamma) |
               reinterpret_cast<uintptr_t>(x_out) | reinterpret_cast<uintptr_t>(out)) & 15) == 0,
             "x, y, gamma, x_out and out must be 16-byte aligned");
  const cudaError_t e = launch_dependent(residual_rms_norm_kernel, dim3(rows), dim3(kRowThreads), 0, as_stream(stream),
                                         x, y, gamma, width, eps, x_out, out);
  if (e != cudaSuccess) return cuda_error(e, "residual_rms_norm_kernel");
  count_launch();
  return QK_OK;
}

int qk_qk_norm_rope(const uint16_t* qkv, const uint16_t* q_norm, const uint16_t* k_norm, const float* inv_freq,
                    const int32_t* positions, int B, int hq, int kv, int head_dim, int rotary_dim, float eps,
                    uint16_t* q_out, uint16_t* gate_out, uint16_t* k_out, uint16_t* v_out, qk_stream_t stream) {
  QK_REQUIRE(B >= 0 && hq > 0 && kv > 0, "invalid head geometry");
  QK_REQUIRE(head_dim > 0 && head_dim <= kRowThreads, "head_dim must be in [1, %d]", kRowThreads);
  QK_REQUIRE(rotary_dim >= 0 && rotary_dim <= head_dim && rotary_dim % 2 == 0, "rotary_dim must be even and <= head_dim");
  if (B == 0) return QK_OK;
  QK_REQUIRE(qkv && q_norm && k_norm && positions && q_out && gate_out && k_out && v_out, "null pointer");
  QK_REQUIRE(inv_freq || rotary_dim == 0, "inv_freq is required when rotary_dim > 0");
  const cudaError_t e = launch_dependent(qk_norm_rope_kernel, dim3(B, hq + kv), dim3(kRowThreads), 0, as_stream(stream),
                                         qkv, q_norm, k_norm, inv_freq, positions, hq, kv, head_dim, rotary_dim, eps,
                                         q_out, gate_out, k_out, v_out);
  if (e != cudaSuccess) return cuda_error(e, "qk_norm_rope_kernel");
  count_launch();
  return QK_OK;
}

int qk_residual_add(const uint16_t* x, const uint16_t* y, int64_t n, uint16_t* out, qk_stream_t stream) {
  QK_REQUIRE(n >= 0, "invalid size");
  if (n == 0) return QK_OK;
  QK_REQUIRE(x && y && out, "null pointer");
  const int64_t blocks = (n + 255) / 256;
  const cudaError_t e = launch_dependent(residual_add_kernel, dim3(static_cast<unsigned>(blocks < 4 * 148 ? blocks : 4 * 148)),
                                         dim3(256), 0, as_stream(stream), x, y, n, out);
  if (e != cudaSuccess) return cuda_error(e, "residual_add_kernel");
  count_launch();
  return QK_OK;
}

int qk_append_shared_route(const int32_t* ids, const uint16_t* weights, int B, int k, const uint16_t* h,
                           const uint16_t* shared_router, int H, int shared_id, int32_t* ids_out,
                           uint16_t* weights_out, qk_stream_t stream) {
  QK_REQUIRE(B >= 0 && k > 0 && k < kRowThreads && H > 0 && H % 8 == 0 && H <= kMaxRowWidth,
             "invalid route geometry");
  if (B == 0) return QK_OK;
  QK_REQUIRE(ids && weights && h && shared_router && ids_out && weights_out, "null pointer");
  QK_REQUIRE(((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(shared_router)) & 15) == 0,
             "h and shared_router must be 16-byte aligned");
  const cudaError_t e = launch_dependent(append_shared_route_kernel, dim3(B), dim3(kRowThreads), 0, as_stream(stream),
                                         ids, weights, k, h, shared_router, H, shared_id, 0, ids_out, weights_out);
  if (e != cudaSuccess) return cuda_error(e, "append_shared_route_kernel");
  count_launch();
  return QK_OK;
}

int qk_append_shared_route_ep(const int32_t* ids, const uint16_t* weights, int B, int k, const uint16_t* h,
                              const uint16_t* shared_router, int H, int experts_per_rank, int rank,
                              int32_t* ids_out, uint16_t* weights_out, qk_stream_t stream) {
  QK_REQUIRE(B >= 0 && k > 0 && k < kRowThreads && H > 0 && H % 8 == 0 && H <= kMaxRowWidth,
             "invalid route geometry");
  QK_REQUIRE(experts_per_rank > 0 && rank >= 0, "invalid expert partition");
  if (B == 0) return QK_OK;
  QK_REQUIRE(ids && weights && h && shared_router && ids_out && weights_out, "null pointer");
  QK_REQUIRE(((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(shared_router)) & 15) == 0,
             "h and shared_router must be 16-byte aligned");
  const int shared_id = rank * (experts_per_rank + 1) + experts_per_rank;
  const cudaError_t e = launch_dependent(append_shared_route_kernel, dim3(B), dim3(kRowThreads), 0, as_stream(stream),
                                         ids, weights, k, h, shared_router, H, shared_id, experts_per_rank, ids_out,
                                         weights_out);
  if (e != cudaSuccess) return cuda_error(e, "append_shared_route_kernel");
  count_launch();
  return QK_OK;
}

}  // extern "C"

// ---- greedy sampling with a non-finite check (qwen38_tpu/run.py:46-55 checked_argmax) ----
namespace qk {
namespace {

constexpr int kArgThreads = 1024;

// (value, index) pair order of jnp.argmax: NaN above everything, then larger value, then the
// lower index.
__device__ __forceinline__ bool arg_better(float a, int ia, float b, int ib) {
  const bool na = a != a, nb = b != b;
  if (na || nb) return na && (!nb || ia < ib);
  return a > b || (a == b && ia < ib);
}

template <typename T>
__device__ __forceinline__ float logit_at(const T* row, int64_t i);
template <>
__device__ __forceinline__ float logit_at<uint16_t>(const uint16_t* row, int64_t i) {
  return bf16_to_f32(row[i]);
}
template <>
__device__ __forceinline__ float logit_at<float>(const float* row, int64_t i) {
  return row[i];
}

template <typename T>
__global__ void __launch_bounds__(kArgThreads) checked_argmax_kernel(const T* __restrict__ logits, int64_t V,
                                                                     int32_t* __restrict__ out) {
  __shared__ float sv[32];
  __shared__ int si[32], sc[32];
  pdl_wait();
  const int64_t b = blockIdx.x;
  const T* row = logits + b * V;
  float best = -INFINITY;
  int bi = 0x7fffffff, bad = 0;
  for (int64_t i = threadIdx.x; i < V; i += kArgThreads) {
    const float v = logit_at<T>(row, i);
    bad += !isfinite(v);
    if (arg_better(v, static_cast<int>(i), best, bi)) {
      best = v;
      bi = static_cast<int>(i);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    bad += __shfl_xor_sync(0xffffffffu, bad, o);
    if (arg_better(ov, oi, best, bi)) {
      best = ov;
      bi = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
    sc[warp] = bad;
  }
  __syncthreads();
  if (warp == 0) {
    best = sv[lane];
    bi = si[lane];
    bad = sc[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      bad += __shfl_xor_sync(0xffffffffu, bad, o);
      if (arg_better(ov, oi, best, bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      out[2 * b] = bi;
      out[2 * b + 1] = bad;
    }
  }
}

}  // namespace
}  // namespace qk

extern "C" int qk_checked_argmax(const void* logits, int in_dtype, int B, int64_t V, int32_t* out,
                                 qk_stream_t stream) {
  using namespace qk;
  QK_REQUIRE(B >= 0 && V > 0 && V < (int64_t{1} << 31), "invalid logits geometry");
  QK_REQUIRE(in_dtype == QK_OUT_F32 || in_dtype == QK_OUT_BF16, "logits must be FP32 or BF16");
  if (B == 0) return QK_OK;
  QK_REQUIRE(logits && out, "null pointer");
  const cudaError_t e =
      in_dtype == QK_OUT_BF16
          ? launch_dependent(checked_argmax_kernel<uint16_t>, dim3(B), dim3(kArgThreads), 0, as_stream(stream),
                             static_cast<const uint16_t*>(logits), V, out)
          : launch_dependent(checked_argmax_kernel<float>, dim3(B), dim3(kArgThreads), 0, as_stream(stream),
                             static_cast<const float*>(logits), V, out);
  if (e != cudaSuccess) return cuda_error(e, "checked_argmax_kernel");
  count_launch();
  return QK_OK;
}
