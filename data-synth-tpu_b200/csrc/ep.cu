// Expert-parallel token exchange: route planning, row gather and the route-weighted
// combine of expert outputs returned by the owning ranks.
//
// The expert-parallel layer with token dispatch (each rank holds a contiguous range of
// experts, as parallel.py:64-87 places them, and its own tokens):
//   1. qk_ep_plan       - per token, merge routes naming the same expert into one route of
//                         weight bf16(sum) and drop zero-weight routes (experts.py:66-76),
//                         then counting-sort the routes by the rank that owns the expert;
//   2. qk_gather_rows   - the token rows of the send slots, rank-major, for an all-to-all;
//   3. (all-to-all of rows and expert ids; the owning rank runs qk_moe_forward with top_k 1
//       and route weight 1, which returns bf16(h Wd^T) per row; all-to-all back);
//   4. qk_ep_combine    - per token, the FP32 sum of f32(y) * f32(w) over its routes in
//                         ascending expert order (experts.py:129), then BF16 - the same
//                         arithmetic as the single-device combine.
#include "common.cuh"

namespace qk {
namespace {

constexpr int kMaxRanks = 1024;
constexpr int kMaxRoutes = 32;

// Merged weight of route (b, j): 0 when the route is dropped (a later slot of a repeated
// expert, an expert outside [0, n_experts), or a zero merged weight).
__device__ float merged_weight(const int32_t* ids, const uint16_t* weights, int b, int k, int j,
                               int n_experts) {
  const int e = ids[b * k + j];
  if (e < 0 || e >= n_experts) return 0.f;
  for (int jj = 0; jj < j; ++jj)
    if (ids[b * k + jj] == e) return 0.f;
  float w = 0.f;
  for (int jj = j; jj < k; ++jj)
    if (ids[b * k + jj] == e) w = __fadd_rn(w, bf16_to_f32(weights[b * k + jj]));
  return bf16_round(w);
}

__global__ void __launch_bounds__(1024) ep_plan_kernel(const int32_t* __restrict__ ids,
                                                       const uint16_t* __restrict__ weights, int B,
                                                       int k, int experts_per_rank, int world,
                                                       int32_t* send_counts, int32_t* send_rows,
                                                       int32_t* send_expert, int32_t* route_slot,
                                                       float* route_weight) {
  extern __shared__ int32_t sh[];
  int32_t* counts = sh;          // [world]
  int32_t* cursor = sh + world;  // [world]
  const int tid = threadIdx.x, nt = blockDim.x;
  const int n_experts = experts_per_rank * world;
  for (int r = tid; r < world; r += nt) counts[r] = cursor[r] = 0;
  __syncthreads();
  for (int i = tid; i < B * k; i += nt) {
    const int b = i / k, j = i % k;
    const float w = merged_weight(ids, weights, b, k, j, n_experts);
    route_weight[i] = w;
    if (w != 0.f) atomicAdd(&counts[ids[i] / experts_per_rank], 1);
  }
  __syncthreads();
  if (tid == 0) {  // exclusive scan over ranks (world is small)
    int run = 0;
    for (int r = 0; r < world; ++r) {
      const int c = counts[r];
      send_counts[r] = c;
      cursor[r] = run;
      run += c;
    }
  }
  __syncthreads();
  for (int i = tid; i < B * k; i += nt) {
    int slot = -1;
    if (route_weight[i] != 0.f) {
      const int e = ids[i];
      slot = atomicAdd(&cursor[e / experts_per_rank], 1);
      send_rows[slot] = i / k;
      send_expert[slot] = e;
    }
    route_slot[i] = slot;
  }
}

__global__ void gather_rows_kernel(const uint4* __restrict__ src, const int32_t* __restrict__ rows,
                                   int64_t n, int64_t w16, uint4* __restrict__ dst) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n * w16;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / w16, c = i % w16;
    dst[i] = ld_nc_v4(src + static_cast<int64_t>(rows[r]) * w16 + c);
  }
}

// One warp per token; lane j holds route j. Ranks by expert id give the ascending-expert
// order; each lane sums 8 columns per 256-column block in FP32.
__global__ void __launch_bounds__(256) ep_combine_kernel(const uint16_t* __restrict__ y,
                                                         const int32_t* __restrict__ route_slot,
                                                         const int32_t* __restrict__ ids,
                                                         const float* __restrict__ route_weight, int B,
                                                         int k, int H, int out_bf16, void* out) {
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (b >= B) return;
  const int slot = lane < k ? route_slot[b * k + lane] : -1;
  const int eid = slot >= 0 ? ids[b * k + lane] : 0x7fffffff;
  const float w = slot >= 0 ? route_weight[b * k + lane] : 0.f;
  int rank = 0, n = 0;
  for (int j = 0; j < k; ++j) {
    const int ej = __shfl_sync(0xffffffffu, eid, j);
    const int vj = __shfl_sync(0xffffffffu, slot, j) >= 0;
    n += vj;
    rank += vj && (ej < eid);
  }
  for (int c0 = lane * 8; c0 < H; c0 += 256) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int i = 0; i < n; ++i) {
      const unsigned who = __ballot_sync(0xffffffffu, slot >= 0 && rank == i);
      const int src = __ffs(who) - 1;
      const int s = __shfl_sync(0xffffffffu, slot, src);
      const float wi = __shfl_sync(0xffffffffu, w, src);
      const uint4 v = ld_nc_v4(y + static_cast<int64_t>(s) * H + c0);
      const uint32_t p[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const float yv = bf16_to_f32(static_cast<uint16_t>(p[t >> 1] >> (16 * (t & 1))));
        acc[t] = __fadd_rn(acc[t], __fmul_rn(yv, wi));
      }
    }
    const int64_t o = static_cast<int64_t>(b) * H + c0;
    if (out_bf16) {
      uint32_t q[4];
#pragma unroll
      for (int t = 0; t < 4; ++t)
        q[t] = static_cast<uint32_t>(bf16_bits_rne(acc[2 * t])) | (static_cast<uint32_t>(bf16_bits_rne(acc[2 * t + 1])) << 16);
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + o) = make_uint4(q[0], q[1], q[2], q[3]);
    } else {
      float4* f = reinterpret_cast<float4*>(static_cast<float*>(out) + o);
      f[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      f[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
}

}  // namespace
}  // namespace qk

using namespace qk;

extern "C" {

int qk_ep_plan(const int32_t* ids, const uint16_t* weights, int B, int k, int experts_per_rank,
               int world, int32_t* send_counts, int32_t* send_rows, int32_t* send_expert,
               int32_t* route_slot, float* route_weight, qk_stream_t stream) {
  QK_REQUIRE(B >= 0 && k > 0 && k <= kMaxRoutes, "top_k must be in [1, %d]", kMaxRoutes);
  QK_REQUIRE(experts_per_rank > 0 && world > 0 && world <= kMaxRanks, "invalid expert placement");
  QK_REQUIRE(send_counts, "null pointer");
  cudaStream_t st = as_stream(stream);
  if (B == 0) {
    const cudaError_t e = cudaMemsetAsync(send_counts, 0, sizeof(int32_t) * world, st);
    return e == cudaSuccess ? QK_OK : cuda_error(e, "qk_ep_plan");
  }
  QK_REQUIRE(ids && weights && send_rows && send_expert && route_slot && route_weight, "null pointer");
  ep_plan_kernel<<<1, 1024, 2 * world * sizeof(int32_t), st>>>(ids, weights, B, k, experts_per_rank, world,
                                                                send_counts, send_rows, send_expert, route_slot,
                                                                route_weight);
  QK_LAUNCHED("ep_plan_kernel");
  return QK_OK;
}

int qk_gather_rows(const uint16_t* src, const int32_t* rows, int64_t n, int64_t width, uint16_t* dst,
                   qk_stream_t stream) {
  QK_REQUIRE(n >= 0 && width > 0 && width % 8 == 0, "width must be a positive multiple of 8");
  if (n == 0) return QK_OK;
  QK_REQUIRE(src && rows && dst, "null pointer");
  QK_REQUIRE((reinterpret_cast<uintptr_t>(src) & 15) == 0 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0,
             "rows must be 16-byte aligned");
  const int64_t w16 = width / 8;
  int64_t grid = (n * w16 + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  gather_rows_kernel<<<static_cast<unsigned>(grid > cap ? cap : grid), 256, 0, as_stream(stream)>>>(
      reinterpret_cast<const uint4*>(src), rows, n, w16, reinterpret_cast<uint4*>(dst));
  QK_LAUNCHED("gather_rows_kernel");
  return QK_OK;
}

int qk_ep_combine(const uint16_t* y, const int32_t* route_slot, const int32_t* ids,
                  const float* route_weight, int B, int k, int H, int out_dtype, void* out,
                  qk_stream_t stream) {
  QK_REQUIRE(B >= 0 && k > 0 && k <= kMaxRoutes, "top_k must be in [1, %d]", kMaxRoutes);
  QK_REQUIRE(H > 0 && H % 256 == 0, "hidden must be a positive multiple of 256");
  QK_REQUIRE(out_dtype == QK_OUT_F32 || out_dtype == QK_OUT_BF16, "out_dtype must be F32 or BF16");
  if (B == 0) return QK_OK;
  QK_REQUIRE(route_slot && ids && route_weight && out, "null pointer");
  ep_combine_kernel<<<(B + 7) / 8, 256, 0, as_stream(stream)>>>(y, route_slot, ids, route_weight, B, k, H,
                                                                out_dtype == QK_OUT_BF16, out);
  QK_LAUNCHED("ep_combine_kernel");
  return QK_OK;
}

}  // extern "C"
