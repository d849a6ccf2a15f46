// Layout of the per-rank exchange region of the peer-to-peer expert-parallel layer.
//
// Every rank of the group allocates one region of the same size (qk_ep_p2p_bytes) and maps
// every other rank's region into its address space (CUDA IPC over NVLink / NVSwitch). A
// rank writes only into the slots that belong to it in another rank's region, so no two
// ranks ever write the same bytes:
//
//   ctrl      control words (below)
//   recv_ids  int32 [world][max_tokens][top_k]  expert ids of the rows source s sent here
//   recv_w    bf16  [world][max_tokens][top_k]  their route weights
//   recv_x    bf16  [world][max_tokens][hidden] the rows themselves (slot = source token index)
//   ret       f32   [world][max_tokens][hidden] owner w's partial sum for this rank's token b
//
// Control words (uint32): recv_flag[s] = epoch of the last rows source s finished sending;
// ret_flag[w] = epoch of the last partials owner w finished returning; two arrival counters
// (one per signalling kernel); the epoch of this rank's current step; a status word.
#pragma once

#include "common.cuh"

namespace qk {

constexpr int kEpMaxRanks = 64;

struct EpCtrl {
  uint32_t recv_flag[kEpMaxRanks];
  uint32_t ret_flag[kEpMaxRanks];
  uint32_t dispatch_arrivals;
  uint32_t combine_arrivals;
  uint32_t epoch;
  int32_t status;
  uint32_t reserved[60];
};

struct EpLayout {
  int world, max_tokens, hidden, top_k;
  size_t recv_ids, recv_w, recv_x, ret, total;
};

inline size_t ep_align(size_t n) { return (n + 255) & ~size_t(255); }

inline EpLayout ep_layout(int world, int max_tokens, int hidden, int top_k) {
  EpLayout L;
  L.world = world;
  L.max_tokens = max_tokens;
  L.hidden = hidden;
  L.top_k = top_k;
  const size_t rows = static_cast<size_t>(world) * max_tokens;
  size_t off = ep_align(sizeof(EpCtrl));
  L.recv_ids = off;
  off += ep_align(rows * top_k * 4);
  L.recv_w = off;
  off += ep_align(rows * top_k * 2);
  L.recv_x = off;
  off += ep_align(rows * hidden * 2);
  L.ret = off;
  off += ep_align(rows * hidden * 4);
  L.total = off;
  return L;
}

// Bounded acquire poll of a control word until it equals `want`: about four seconds at most.
__device__ __forceinline__ bool ep_wait_flag(const uint32_t* flag, uint32_t want) {
  for (uint32_t i = 0; i < (1u << 22); ++i) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
    if (v == want) return true;
    __nanosleep(i < 64 ? 32 : 1000);
  }
  return false;
}

__device__ __forceinline__ void ep_store_release(uint32_t* flag, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(v) : "memory");
}

// The calling CTA has finished its writes. Returns true in exactly one CTA of the grid (the
// last to arrive), after every CTA's writes are visible system-wide; that CTA resets the
// counter for the next step. Call with every thread of the CTA.
__device__ __forceinline__ bool ep_last_cta(uint32_t* counter) {
  __shared__ uint32_t last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(counter, 1u);
    last = prev == gridDim.x - 1;
    if (last) {
      __threadfence_system();
      atomicExch(counter, 0u);
    }
  }
  __syncthreads();
  return last != 0;
}

}  // namespace qk
