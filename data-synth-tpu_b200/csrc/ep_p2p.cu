// Expert-parallel token exchange over peer memory (NVLink / NVSwitch), with no host
// synchronisation and no data-dependent sizes on the host.
//
// The reference's expert-parallel layer (qwen38_tpu/experts.py:61-131) gives every device
// its experts' share of the routed FFN and adds the devices' partial outputs with a psum
// over the "expert" axis (experts.py:130-131). Here each rank keeps its own tokens; a step
// is three stream-ordered calls per rank:
//
//   qk_ep_p2p_dispatch  this rank's token row b goes, once, to every rank that owns one of its
//                       routed experts: x[b] and the routes that name that rank's experts are
//                       stored straight into slot [this rank][b] of the owner's region
//                       (other slots of the row list -1). The last CTA to finish raises
//                       recv_flag[this rank] in every owner's region (even where it sent no
//                       row), so an owner always knows when a source is complete.
//   qk_ep_p2p_expert    (moe.cu) waits for every source's flag, runs the routed FFN of its
//                       experts over the [world * max_tokens] received slots, and writes each
//                       sent slot's FP32 partial sum over its experts (ascending expert order)
//                       straight into the source's ret[this rank][b]; the last CTA raises
//                       ret_flag[this rank] at every source.
//   qk_ep_p2p_combine   waits for every owner's flag and adds, per token, the partials of the
//                       ranks it routed to in ascending rank (= expert) order, then rounds
//                       once to BF16: the reference's local sum + psum, experts.py:128-131.
//
// Slots are indexed by the source's token index, so no rank needs another's counts. Reuse is
// safe without extra back-pressure: a rank dispatches step t + 1 only after its combine of
// step t saw every owner's ret_flag for t, which each owner raises after its expert pass of t
// has read all received rows; an owner returns step t + 1 only after its own dispatch of
// t + 1 (so after its combine of t read its ret slots). Epochs: every rank counts its steps
// in ctrl.epoch; flags carry the step's epoch. Every wait is bounded (a few seconds); on
// give-up the kernel stores QK_ERR_TIMEOUT in ctrl.status and returns.
#include <cstring>

#include "ep_p2p.cuh"

namespace qk {
namespace {

__global__ void __launch_bounds__(512) ep_dispatch_kernel(uint8_t* const* __restrict__ peers, uint8_t* own, EpLayout L,
                                                          int rank, int experts_per_rank,
                                                          const uint16_t* __restrict__ x,
                                                          const int32_t* __restrict__ ids,
                                                          const uint16_t* __restrict__ w, int B) {
  pdl_wait();
  EpCtrl* ctrl = reinterpret_cast<EpCtrl*>(own);
  const uint32_t epoch = ctrl->epoch + 1;  // every CTA reads it before the last one advances it
  const int lane = threadIdx.x & 31, k = L.top_k, H = L.hidden, T = L.max_tokens;
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  for (int g = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); g < L.world * T; g += nwarps) {
    const int dst = g / T, b = g - dst * T;
    uint8_t* pb = peers[dst];
    const size_t slot = static_cast<size_t>(rank) * T + b;
    int id = -1;
    uint16_t wt = 0;
    if (b < B && lane < k) {
      const int e = ids[static_cast<int64_t>(b) * k + lane];
      const uint16_t v = w[static_cast<int64_t>(b) * k + lane];
      if (e >= dst * experts_per_rank && e < (dst + 1) * experts_per_rank && (v & 0x7fffu) != 0) {
        id = e;
        wt = v;
      }
    }
    const bool routed = __any_sync(0xffffffffu, id >= 0);
    if (lane < k) {
      reinterpret_cast<int32_t*>(pb + L.recv_ids)[slot * k + lane] = id;
      reinterpret_cast<uint16_t*>(pb + L.recv_w)[slot * k + lane] = wt;
    }
    if (routed) {
      // the row's 16-byte pieces, eight per lane in flight before they are stored
      constexpr int kU = 8;
      const uint4* src = reinterpret_cast<const uint4*>(x + static_cast<int64_t>(b) * H);
      uint4* dstp = reinterpret_cast<uint4*>(pb + L.recv_x + slot * H * 2);
      for (int c0 = lane; c0 < H / 8; c0 += 32 * kU) {
        uint4 v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u)
          if (c0 + 32 * u < H / 8) v[u] = ld_nc_v4(src + c0 + 32 * u);
#pragma unroll
        for (int u = 0; u < kU; ++u)
          if (c0 + 32 * u < H / 8) dstp[c0 + 32 * u] = v[u];
      }
    }
  }
  if (ep_last_cta(&ctrl->dispatch_arrivals)) {
    for (int t = threadIdx.x; t < L.world; t += blockDim.x)
      ep_store_release(&reinterpret_cast<EpCtrl*>(peers[t])->recv_flag[rank], epoch);
    __syncthreads();
    if (threadIdx.x == 0) ctrl->epoch = epoch;
  }
}

// Per token: the FP32 sum of the returned partials of the ranks it routed to, in ascending
// rank order, rounded once to BF16. One warp per (token, 256 columns).
__global__ void __launch_bounds__(256) ep_final_kernel(uint8_t* own, EpLayout L, int experts_per_rank,
                                                       const int32_t* __restrict__ ids,
                                                       const uint16_t* __restrict__ w, int B,
                                                       uint16_t* __restrict__ out) {
  pdl_wait();
  EpCtrl* ctrl = reinterpret_cast<EpCtrl*>(own);
  const uint32_t epoch = ctrl->epoch;
  __shared__ int ok;
  if (threadIdx.x == 0) ok = 1;
  __syncthreads();
  for (int t = threadIdx.x; t < L.world; t += blockDim.x)
    if (!ep_wait_flag(&ctrl->ret_flag[t], epoch)) {
      ok = 0;
      atomicExch(&ctrl->status, QK_ERR_TIMEOUT);
    }
  __syncthreads();
  if (!ok) return;
  const int lane = threadIdx.x & 31, k = L.top_k, H = L.hidden, T = L.max_tokens;
  const int blocks = H / 256;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (gw >= B * blocks) return;
  const int b = gw / blocks, c0 = (gw - b * blocks) * 256 + lane * 8;
  uint64_t mask = 0;
  if (lane < k) {
    const int e = ids[static_cast<int64_t>(b) * k + lane];
    const uint16_t v = w[static_cast<int64_t>(b) * k + lane];
    if (e >= 0 && e < L.world * experts_per_rank && (v & 0x7fffu) != 0) mask = 1ull << (e / experts_per_rank);
  }
  for (int o = 16; o > 0; o >>= 1) mask |= __shfl_xor_sync(0xffffffffu, mask, o);
  float acc[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) acc[t] = 0.f;
  const float* ret = reinterpret_cast<const float*>(own + L.ret);
  while (mask) {
    const int r = __ffsll(static_cast<long long>(mask)) - 1;
    mask &= mask - 1;
    const float* p = ret + (static_cast<size_t>(r) * T + b) * H + c0;
    const float4 a = *reinterpret_cast<const float4*>(p), c = *reinterpret_cast<const float4*>(p + 4);
    const float v[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
#pragma unroll
    for (int t = 0; t < 8; ++t) acc[t] = __fadd_rn(acc[t], v[t]);
  }
  uint32_t q[4];
#pragma unroll
  for (int t = 0; t < 4; ++t)
    q[t] = static_cast<uint32_t>(bf16_bits_rne(acc[2 * t])) | (static_cast<uint32_t>(bf16_bits_rne(acc[2 * t + 1])) << 16);
  *reinterpret_cast<uint4*>(out + static_cast<int64_t>(b) * H + c0) = make_uint4(q[0], q[1], q[2], q[3]);
}

int check_layout(int world, int rank, int max_tokens, int hidden, int top_k, int experts_per_rank) {
  QK_REQUIRE(world >= 1 && world <= kEpMaxRanks, "world must be in [1, %d]", kEpMaxRanks);
  QK_REQUIRE(rank >= 0 && rank < world, "rank must be in [0, world)");
  QK_REQUIRE(max_tokens >= 1, "max_tokens must be positive");
  QK_REQUIRE(hidden > 0 && hidden % 256 == 0, "hidden must be a positive multiple of 256");
  QK_REQUIRE(top_k >= 1 && top_k <= 32, "top_k must be in [1, 32]");
  QK_REQUIRE(experts_per_rank >= 1, "experts_per_rank must be positive");
  return QK_OK;
}

}  // namespace
}  // namespace qk

using namespace qk;

extern "C" {

size_t qk_ep_p2p_bytes(int world, int max_tokens, int hidden, int top_k) {
  if (world < 1 || world > kEpMaxRanks || max_tokens < 1 || hidden <= 0 || top_k < 1) return 0;
  return ep_layout(world, max_tokens, hidden, top_k).total;
}

int qk_ep_p2p_reset(void* region, qk_stream_t stream) {
  QK_REQUIRE(region && (reinterpret_cast<uintptr_t>(region) & 255) == 0, "region must be 256-byte aligned");
  const cudaError_t e = cudaMemsetAsync(region, 0, sizeof(EpCtrl), as_stream(stream));
  if (e != cudaSuccess) return cuda_error(e, "qk_ep_p2p_reset");
  return QK_OK;
}

int qk_ep_p2p_status(const void* region, qk_stream_t stream) {
  QK_REQUIRE(region, "null region");
  int32_t status = 0;
  const EpCtrl* ctrl = static_cast<const EpCtrl*>(region);
  cudaError_t e = cudaMemcpyAsync(&status, &ctrl->status, 4, cudaMemcpyDeviceToHost, as_stream(stream));
  if (e == cudaSuccess) e = cudaStreamSynchronize(as_stream(stream));
  if (e != cudaSuccess) return cuda_error(e, "qk_ep_p2p_status");
  if (status) return set_error(status, "a bounded wait of the expert-parallel exchange gave up (a peer did not signal)");
  return QK_OK;
}

int qk_ep_p2p_dispatch(void* const* peers, void* region, int world, int rank, int max_tokens, int hidden,
                       int top_k, int experts_per_rank, const uint16_t* x, const int32_t* ids,
                       const uint16_t* weights, int B, qk_stream_t stream) {
  int rc = check_layout(world, rank, max_tokens, hidden, top_k, experts_per_rank);
  if (rc) return rc;
  QK_REQUIRE(peers && region, "null pointer");
  QK_REQUIRE(B >= 0 && B <= max_tokens, "batch must be in [0, max_tokens]");
  QK_REQUIRE(B == 0 || (x && ids && weights), "null pointer");
  const EpLayout L = ep_layout(world, max_tokens, hidden, top_k);
  const int64_t warps = static_cast<int64_t>(world) * max_tokens;
  int64_t grid = (warps + 15) / 16;
  const int64_t cap = static_cast<int64_t>(sm_count());  // few CTAs: one system-scope fence each
  if (grid > cap) grid = cap;
  const cudaError_t e = launch_dependent(ep_dispatch_kernel, dim3(static_cast<unsigned>(grid)), dim3(512), 0,
                                         as_stream(stream), reinterpret_cast<uint8_t* const*>(peers),
                                         static_cast<uint8_t*>(region), L, rank, experts_per_rank, x, ids, weights, B);
  if (e != cudaSuccess) return cuda_error(e, "ep_dispatch_kernel");
  count_launch(1);
  return QK_OK;
}

int qk_ep_p2p_combine(void* region, int world, int rank, int max_tokens, int hidden, int top_k,
                      int experts_per_rank, const int32_t* ids, const uint16_t* weights, int B,
                      uint16_t* out, qk_stream_t stream) {
  int rc = check_layout(world, rank, max_tokens, hidden, top_k, experts_per_rank);
  if (rc) return rc;
  QK_REQUIRE(region, "null region");
  QK_REQUIRE(B >= 0 && B <= max_tokens, "batch must be in [0, max_tokens]");
  QK_REQUIRE(B == 0 || (ids && weights && out), "null pointer");
  QK_REQUIRE((reinterpret_cast<uintptr_t>(out) & 15) == 0, "out must be 16-byte aligned");
  const EpLayout L = ep_layout(world, max_tokens, hidden, top_k);
  // at least one CTA, so the step's flags are consumed even for an empty batch
  const int64_t warps = static_cast<int64_t>(B) * (hidden / 256);
  const int64_t grid = warps > 0 ? (warps + 7) / 8 : 1;
  const cudaError_t e = launch_dependent(ep_final_kernel, dim3(static_cast<unsigned>(grid)), dim3(256), 0,
                                         as_stream(stream), static_cast<uint8_t*>(region), L, experts_per_rank, ids,
                                         weights, B, out);
  if (e != cudaSuccess) return cuda_error(e, "ep_final_kernel");
  count_launch(1);
  return QK_OK;
}

// ---- device memory that other processes can map (CUDA IPC) -----------------------------

int qk_device_alloc(size_t bytes, void** ptr) {
  QK_REQUIRE(ptr && bytes > 0, "bad allocation request");
  const cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return cuda_error(e, "qk_device_alloc");
  return QK_OK;
}

int qk_device_free(void* ptr) {
  if (!ptr) return QK_OK;
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return cuda_error(e, "qk_device_free");
  return QK_OK;
}

int qk_ipc_get_handle(void* ptr, uint8_t* handle64) {
  QK_REQUIRE(ptr && handle64, "null pointer");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) return cuda_error(e, "qk_ipc_get_handle");
  memcpy(handle64, &h, 64);
  return QK_OK;
}

int qk_ipc_open_handle(const uint8_t* handle64, void** ptr) {
  QK_REQUIRE(ptr && handle64, "null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, 64);
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_error(e, "qk_ipc_open_handle");
  return QK_OK;
}

int qk_ipc_close_handle(void* ptr) {
  if (!ptr) return QK_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return cuda_error(e, "qk_ipc_close_handle");
  return QK_OK;
}

}  // extern "C"
