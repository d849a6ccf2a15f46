// Router top-k: FP32 logits, softmax, top-k (ties to the lower index), renormalise, BF16.
//
// Replaces the router of qwen38_tpu/math.py:277-281 (routes_and_shared):
//   probs = numerics.softmax(linear(f32(x), f32(Wr)))      (HIGHEST: FP32 dot)
//   w, ids = lax.top_k(probs, k); w = numerics.divide(w, sum(w))
//   w = compute_cast(where(active, w, 0), bf16)
// A thread-block cluster of kCluster CTAs handles up to 8 tokens. Each CTA stages the
// tokens' x rows in shared memory and computes the logits of its slice of the experts (one
// warp per expert row, fixed-order reductions; each router row is read once per cluster),
// storing them into the first CTA's shared memory (distributed shared memory). After the
// cluster barrier the first CTA's warp t runs softmax and the k selection rounds for token
// t. Divisions are IEEE; exp is exp_ref (expf).
//
// The same result in two launches, for callers that own a logits buffer (the decoder stack):
// router_logits_kernel spreads the experts over many CTAs (4 router rows per CTA, so the
// FP32 router matrix is read by ~E / 4 SMs instead of the cluster's 8) with the same
// per-lane accumulation order and reduction, and router_select_kernel runs the softmax and
// the selection, one warp per token.
#include <cooperative_groups.h>

#include "common.cuh"

namespace cg = cooperative_groups;

namespace qk {
namespace {

constexpr int kTok = 8;
constexpr int kCluster = 8;
constexpr int kWarps = 16;  // warps per CTA (each takes two router rows at a time)

// Softmax, top-k (ties to the lower index) and renormalisation of token t's logits `row`
// (E floats in shared memory, overwritten), by one warp. Route j goes to ids / weights
// [t * stride + j]; with per > 0 expert e is written as (e / per) * (per + 1) + e % per (the
// expert-parallel numbering with one shared-expert slot after each rank's `per` experts).
__device__ __forceinline__ void select_row(float* row, int t, int E, int k, int lane, const uint8_t* __restrict__ active,
                                           int32_t* __restrict__ ids, uint16_t* __restrict__ weights,
                                           float* __restrict__ probs_out, int stride, int per) {
  // softmax (numerics.py:48-51)
  softmax_row_warp(row, E, lane);
  if (probs_out)
    for (int e = lane; e < E; e += 32) probs_out[static_cast<int64_t>(t) * E + e] = row[e];

  // top-k: k rounds of a warp argmax; ties go to the lower expert index (lax.top_k). Each
  // lane keeps the best of its own entries e = lane + 32 i. A round takes the warp's maximum
  // with two reductions (probabilities are >= 0, so their bit patterns order like their
  // values; taken entries are -1), and only the lane that held the winner rescans.
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  auto lane_best = [&]() {
    bv = -INFINITY;
    bi = 0x7fffffff;
    for (int e = lane; e < E; e += 32) {
      const float v = row[e];
      if (v > bv || (v == bv && e < bi)) {
        bv = v;
        bi = e;
      }
    }
  };
  lane_best();
  float mine = 0.f;  // lane j keeps the j-th selected probability
  int mine_id = 0;
  for (int j = 0; j < k; ++j) {
    const bool cand = bv >= 0.f;
    const uint32_t key = cand ? __float_as_uint(bv) : 0u;
    const uint32_t top = __reduce_max_sync(0xffffffffu, key);
    const uint32_t id = __reduce_min_sync(0xffffffffu, cand && key == top ? static_cast<uint32_t>(bi) : 0xffffffffu);
    if (lane == j) {
      mine = __uint_as_float(top);
      mine_id = static_cast<int>(id);
    }
    if (id < static_cast<uint32_t>(E) && lane == static_cast<int>(id & 31)) {
      row[id] = -1.f;  // excluded from later rounds
      lane_best();
    }
  }
  __syncwarp();
  // renormalise with a sequential FP32 sum over j (the oracle uses the same order)
  float total = 0.f;
  for (int j = 0; j < k; ++j) total = __fadd_rn(total, __shfl_sync(0xffffffffu, mine, j));
  if (lane < k) {
    const bool on = active ? active[t] != 0 : true;
    const float wv = on ? __fdiv_rn(mine, total) : 0.f;
    ids[static_cast<int64_t>(t) * stride + lane] = per > 0 ? (mine_id / per) * (per + 1) + mine_id % per : mine_id;
    weights[static_cast<int64_t>(t) * stride + lane] = bf16_bits_rne(wv);
  }
}

__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kWarps * 32)
    router_kernel(const uint16_t* __restrict__ x, const float* __restrict__ w,
                  const uint8_t* __restrict__ active, int T, int H, int E, int k, int32_t* __restrict__ ids,
                  uint16_t* __restrict__ weights, float* __restrict__ probs_out) {
  extern __shared__ __align__(16) float lg[];  // [kTok][E], then x rows [kTok][H] (BF16)
  uint16_t* xs = reinterpret_cast<uint16_t*>(lg + kTok * E);
  pdl_wait();  // launched as a programmatic dependent: the previous kernel's outputs first
  pdl_trigger();
  cg::cluster_group cluster = cg::this_cluster();
  const unsigned crank = cluster.block_rank();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = (blockIdx.x / kCluster) * kTok;
  const int nt = min(kTok, T - t0);

  {
    const int pieces = nt * H / 8;  // 16-byte pieces of the token rows
    for (int i = threadIdx.x; i < pieces; i += blockDim.x)
      reinterpret_cast<uint4*>(xs)[i] = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(t0) * H)[i];
    __syncthreads();
    float* lg0 = cluster.map_shared_rank(lg, 0);
    const int per = (E + kCluster - 1) / kCluster, e0 = static_cast<int>(crank) * per;
    const int e1 = min(E, e0 + per);
    // Each warp takes two router rows at a time and keeps kU 16-byte loads per row in flight
    // (the loads are issued before the FMAs that use them); every lane still adds its
    // columns h = 4 lane + 128 i in increasing i, so the logits do not depend on kU.
    constexpr int kU = 8;
    for (int ea = e0 + warp; ea < e1; ea += 2 * kWarps) {
      const int eb = ea + kWarps;
      const bool has_b = eb < e1;
      float acc[2][kTok];
#pragma unroll
      for (int t = 0; t < kTok; ++t) acc[0][t] = acc[1][t] = 0.f;
      const float* wa = w + static_cast<int64_t>(ea) * H;
      const float* wb = w + static_cast<int64_t>(has_b ? eb : ea) * H;
      for (int h0 = lane * 4; h0 < H; h0 += 128 * kU) {
        float4 va[kU], vb[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int h = h0 + 128 * u;
          va[u] = h < H ? *reinterpret_cast<const float4*>(wa + h) : make_float4(0.f, 0.f, 0.f, 0.f);
          vb[u] = h < H && has_b ? *reinterpret_cast<const float4*>(wb + h) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int h = h0 + 128 * u;
          if (h >= H) break;
#pragma unroll
          for (int t = 0; t < kTok; ++t) {
            if (t >= nt) break;
            const uint2 xv = *reinterpret_cast<const uint2*>(xs + t * H + h);
            const float x0 = bf16_to_f32(static_cast<uint16_t>(xv.x & 0xffffu));
            const float x1 = bf16_to_f32(static_cast<uint16_t>(xv.x >> 16));
            const float x2 = bf16_to_f32(static_cast<uint16_t>(xv.y & 0xffffu));
            const float x3 = bf16_to_f32(static_cast<uint16_t>(xv.y >> 16));
            acc[0][t] = fmaf(va[u].x, x0, acc[0][t]);
            acc[0][t] = fmaf(va[u].y, x1, acc[0][t]);
            acc[0][t] = fmaf(va[u].z, x2, acc[0][t]);
            acc[0][t] = fmaf(va[u].w, x3, acc[0][t]);
            acc[1][t] = fmaf(vb[u].x, x0, acc[1][t]);
            acc[1][t] = fmaf(vb[u].y, x1, acc[1][t]);
            acc[1][t] = fmaf(vb[u].z, x2, acc[1][t]);
            acc[1][t] = fmaf(vb[u].w, x3, acc[1][t]);
          }
        }
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
#pragma unroll
        for (int t = 0; t < kTok; ++t) {
          float v = acc[r][t];
          for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          if (lane == 0 && t < nt && (r == 0 || has_b)) lg0[t * E + (r == 0 ? ea : eb)] = v;
        }
      }
    }
  }
  cluster.sync();  // every CTA's logits are in the first CTA's shared memory
  if (crank != 0) return;
  __syncthreads();
  if (warp >= nt) return;
  const int t = t0 + warp;
  float* row = lg + warp * E;

  select_row(row, t, E, k, lane, active, ids, weights, probs_out, k, 0);
}


// Logits only: CTA (blockIdx.x, blockIdx.y) computes the logits of router rows
// [kLogitRows * blockIdx.x, + kLogitRows) for tokens [kTok * blockIdx.y, + kTok), one warp
// per row, with the per-lane order and the butterfly of router_kernel (identical values).
constexpr int kLogitRows = 4;

__global__ void __launch_bounds__(kLogitRows * 32)
    router_logits_kernel(const uint16_t* __restrict__ x, const float* __restrict__ w, int T, int H, int E,
                         float* __restrict__ logits) {
  extern __shared__ __align__(16) uint16_t xs_l[];  // x rows [kTok][H] (BF16)
  constexpr int kU = 16;  // a whole 2048-value row's loads in flight per lane (the order of the sums is the same)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * kLogitRows + warp;
  const float* wr = w + static_cast<int64_t>(e < E ? e : 0) * H;
  float4 v[kU];
  auto load_w = [&](int h0) {
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int h = h0 + 128 * u;
      v[u] = h < H ? *reinterpret_cast<const float4*>(wr + h) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  // The router matrix is no earlier kernel's output: its first loads go out before the wait.
  load_w(lane * 4);
  pdl_wait();
  pdl_trigger();
  const int t0 = blockIdx.y * kTok, nt = min(kTok, T - t0);
  {
    // the token rows, 8 loads per thread in flight before the stores
    const int pieces = nt * H / 8;
    const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(t0) * H);
    for (int i0 = 0; i0 < pieces; i0 += kLogitRows * 32 * 8) {
      uint4 xv[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = i0 + threadIdx.x + kLogitRows * 32 * j;
        xv[j] = i < pieces ? src[i] : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = i0 + threadIdx.x + kLogitRows * 32 * j;
        if (i < pieces) reinterpret_cast<uint4*>(xs_l)[i] = xv[j];
      }
    }
  }
  __syncthreads();
  if (e >= E) return;
  float acc[kTok];
#pragma unroll
  for (int t = 0; t < kTok; ++t) acc[t] = 0.f;
  for (int h0 = lane * 4; h0 < H; h0 += 128 * kU) {
    if (h0 != lane * 4) load_w(h0);
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int h = h0 + 128 * u;
      if (h >= H) break;
#pragma unroll
      for (int t = 0; t < kTok; ++t) {
        if (t >= nt) break;
        const uint2 xv = *reinterpret_cast<const uint2*>(xs_l + t * H + h);
        acc[t] = fmaf(v[u].x, bf16_to_f32(static_cast<uint16_t>(xv.x & 0xffffu)), acc[t]);
        acc[t] = fmaf(v[u].y, bf16_to_f32(static_cast<uint16_t>(xv.x >> 16)), acc[t]);
        acc[t] = fmaf(v[u].z, bf16_to_f32(static_cast<uint16_t>(xv.y & 0xffffu)), acc[t]);
        acc[t] = fmaf(v[u].w, bf16_to_f32(static_cast<uint16_t>(xv.y >> 16)), acc[t]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kTok; ++t) {
    float v = acc[t];
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0 && t < nt) logits[static_cast<int64_t>(t0 + t) * E + e] = v;
  }
}

// Token t's logits row into shared memory by one warp: all its 16-byte loads are issued
// before the stores when the row is 16-byte aligned (E % 4 == 0), else one float at a time.
__device__ __forceinline__ void stage_row(float* row, const float* __restrict__ logits, int t, int E, int lane) {
  const float* src = logits + static_cast<int64_t>(t) * E;
  if ((E & 3) == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
    const int n4 = E / 4;
    for (int i0 = 0; i0 < n4; i0 += 32 * 8) {
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = i0 + lane + 32 * j;
        v[j] = i < n4 ? reinterpret_cast<const float4*>(src)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = i0 + lane + 32 * j;
        if (i < n4) reinterpret_cast<float4*>(row)[i] = v[j];
      }
    }
  } else {
    for (int e = lane; e < E; e += 32) row[e] = src[e];
  }
}

// Selection from FP32 logits [T, E]: one warp per token, its row staged in shared memory.
constexpr int kSelectWarps = 8;

__global__ void __launch_bounds__(kSelectWarps * 32)
    router_select_kernel(const float* __restrict__ logits, const uint8_t* __restrict__ active, int T, int E, int k,
                         int32_t* __restrict__ ids, uint16_t* __restrict__ weights, float* __restrict__ probs_out) {
  extern __shared__ __align__(16) float rows[];  // [kSelectWarps][E]
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * kSelectWarps + warp;
  if (t >= T) return;
  float* row = rows + warp * E;
  stage_row(row, logits, t, E, lane);
  __syncwarp();
  select_row(row, t, E, k, lane, active, ids, weights, probs_out, k, 0);
}

// Selection plus the shared expert's route (math.py:282-283), one 256-thread CTA per token:
// ids_out / w_out [T, k + 1] hold the k routes and then (shared_id, bf16(sigmoid(bf16(h . wsr)))).
// The dot product is qk_append_shared_route's (row_dot_bf16), so this launch replaces
// qk_router_topk_logits + qk_append_shared_route with the same bits.
constexpr int kSharedThreads = kRowBlock;

__global__ void __launch_bounds__(kSharedThreads)
    router_select_shared_kernel(const float* __restrict__ logits, const uint8_t* __restrict__ active, int E, int k,
                                const uint16_t* __restrict__ h, const uint16_t* __restrict__ wsr, int H,
                                int shared_id, int per, int32_t* __restrict__ ids_out, uint16_t* __restrict__ w_out) {
  extern __shared__ __align__(16) float row_s[];  // [E]
  __shared__ float red[kSharedThreads / 32];
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x, lane = threadIdx.x & 31;
  // the shared-expert dot's loads are in flight while warp 0 selects
  RowDot rd;
  row_dot_load(rd, h + static_cast<int64_t>(t) * H, wsr, H);
  if (threadIdx.x < 32) {
    stage_row(row_s, logits, t, E, lane);
    __syncwarp();
    select_row(row_s, t, E, k, lane, active, ids_out, w_out, nullptr, k + 1, per);
  }
  const float dot = row_dot_finish(rd, H, red);
  if (threadIdx.x == 0) {
    ids_out[static_cast<int64_t>(t) * (k + 1) + k] = shared_id;
    w_out[static_cast<int64_t>(t) * (k + 1) + k] = bf16_bits_rne(sigmoid_ref(dot));
  }
}

}  // namespace
}  // namespace qk

using namespace qk;

static int router_launch(const uint16_t* x, const float* w, const uint8_t* active, int T, int H, int E, int k,
                         int32_t* ids, uint16_t* weights, float* probs, qk_stream_t stream) {
  QK_REQUIRE(T >= 0 && E > 0 && k > 0 && k <= E && k <= 32, "Invalid expert top-k");
  if (T == 0) return QK_OK;
  QK_REQUIRE(ids && weights, "null pointer");
  const size_t smem = static_cast<size_t>(kTok) * E * 4 + static_cast<size_t>(kTok) * H * 2;
  QK_REQUIRE(smem <= 200 * 1024, "too many experts or too wide a hidden size for the router kernel "
             "(8 * (4 E + 2 H) bytes must stay within 200 KB)");
  int rc = allow_smem(reinterpret_cast<const void*>(router_kernel), smem);
  if (rc) return rc;
  const int blocks = (T + kTok - 1) / kTok;
  const cudaError_t e = launch_dependent(router_kernel, dim3(blocks * kCluster), dim3(kWarps * 32), smem, as_stream(stream), x, w,
                                         active, T, H, E, k, ids, weights, probs);
  if (e != cudaSuccess) return cuda_error(e, "router_kernel");
  count_launch();
  return QK_OK;
}

extern "C" {

int qk_router_topk(const uint16_t* x, const float* router_w, const uint8_t* active, int T, int H,
                   int E, int k, int32_t* ids, uint16_t* weights, float* probs, qk_stream_t stream) {
  QK_REQUIRE(H > 0 && H % 8 == 0, "hidden must be a positive multiple of 8");
  QK_REQUIRE(T == 0 || (x && router_w), "null pointer");
  QK_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(router_w) & 15) == 0,
             "x and router_w must be 16-byte aligned");
  return router_launch(x, router_w, active, T, H, E, k, ids, weights, probs, stream);
}

int qk_router_logits(const uint16_t* x, const float* router_w, int T, int H, int E, float* logits,
                     qk_stream_t stream) {
  QK_REQUIRE(T >= 0 && E > 0, "invalid router geometry");
  QK_REQUIRE(H > 0 && H % 8 == 0, "hidden must be a positive multiple of 8");
  if (T == 0) return QK_OK;
  QK_REQUIRE(x && router_w && logits, "null pointer");
  QK_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(router_w) & 15) == 0,
             "x and router_w must be 16-byte aligned");
  const size_t smem = static_cast<size_t>(kTok) * H * 2;
  QK_REQUIRE(smem <= 200 * 1024, "too wide a hidden size for the router logits kernel (16 H bytes within 200 KB)");
  int rc = allow_smem(reinterpret_cast<const void*>(router_logits_kernel), smem);
  if (rc) return rc;
  const dim3 grid((E + kLogitRows - 1) / kLogitRows, (T + kTok - 1) / kTok);
  const cudaError_t e = launch_dependent(router_logits_kernel, grid, dim3(kLogitRows * 32), smem, as_stream(stream), x,
                                         router_w, T, H, E, logits);
  if (e != cudaSuccess) return cuda_error(e, "router_logits_kernel");
  count_launch();
  return QK_OK;
}

int qk_router_topk_logits(const float* logits, const uint8_t* active, int T, int E, int k,
                          int32_t* ids, uint16_t* weights, float* probs, qk_stream_t stream) {
  QK_REQUIRE(T >= 0 && E > 0 && k > 0 && k <= E && k <= 32, "Invalid expert top-k");
  if (T == 0) return QK_OK;
  QK_REQUIRE(logits && ids && weights, "null pointer");
  const size_t smem = static_cast<size_t>(kSelectWarps) * E * 4;
  QK_REQUIRE(smem <= 200 * 1024, "too many experts for the router selection kernel (32 E bytes within 200 KB)");
  int rc = allow_smem(reinterpret_cast<const void*>(router_select_kernel), smem);
  if (rc) return rc;
  const cudaError_t e = launch_dependent(router_select_kernel, dim3((T + kSelectWarps - 1) / kSelectWarps),
                                         dim3(kSelectWarps * 32), smem, as_stream(stream), logits, active, T, E, k,
                                         ids, weights, probs);
  if (e != cudaSuccess) return cuda_error(e, "router_select_kernel");
  count_launch();
  return QK_OK;
}

int qk_router_select_shared(const float* logits, const uint8_t* active, int T, int E, int k, const uint16_t* h,
                            const uint16_t* shared_router, int H, int shared_id, int experts_per_rank,
                            int32_t* ids_out, uint16_t* weights_out, qk_stream_t stream) {
  QK_REQUIRE(T >= 0 && E > 0 && k > 0 && k <= E && k <= 32, "Invalid expert top-k");
  QK_REQUIRE(H > 0 && H % 8 == 0 && H <= kMaxRowWidth && experts_per_rank >= 0, "invalid route geometry");
  if (T == 0) return QK_OK;
  QK_REQUIRE(logits && h && shared_router && ids_out && weights_out, "null pointer");
  QK_REQUIRE(((reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(shared_router)) & 15) == 0,
             "h and shared_router must be 16-byte aligned");
  const size_t smem = static_cast<size_t>(E) * 4;
  QK_REQUIRE(smem <= 200 * 1024, "too many experts for the router selection kernel (4 E bytes within 200 KB)");
  int rc = allow_smem(reinterpret_cast<const void*>(router_select_shared_kernel), smem);
  if (rc) return rc;
  const cudaError_t e = launch_dependent(router_select_shared_kernel, dim3(T), dim3(kSharedThreads), smem,
                                         as_stream(stream), logits, active, E, k, h, shared_router, H, shared_id,
                                         experts_per_rank, ids_out, weights_out);
  if (e != cudaSuccess) return cuda_error(e, "router_select_shared_kernel");
  count_launch();
  return QK_OK;
}

}  // extern "C"
