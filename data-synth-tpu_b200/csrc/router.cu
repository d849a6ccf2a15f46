// Router top-k: FP32 logits, softmax, top-k (ties to the lower index), renormalise, BF16.
//
// Replaces the router of qwen38_tpu/math.py:277-281 (routes_and_shared):
//   probs = numerics.softmax(linear(f32(x), f32(Wr)))      (HIGHEST: FP32 dot)
//   w, ids = lax.top_k(probs, k); w = numerics.divide(w, sum(w))
//   w = compute_cast(where(active, w, 0), bf16)
// One CTA handles up to 8 tokens: its 8 warps compute the logits of all experts for the
// CTA's tokens (each router row is read once per CTA; fixed-order reductions), then warp t
// runs softmax and the k selection rounds for token t. Divisions are IEEE; exp is expf.
#include "common.cuh"

namespace qk {
namespace {

constexpr int kTok = 8;

__global__ void __launch_bounds__(256) router_kernel(const uint16_t* __restrict__ x,
                                                     const float* __restrict__ w,
                                                     const float* __restrict__ logits_in,
                                                     const uint8_t* __restrict__ active, int T,
                                                     int H, int E, int k, int32_t* __restrict__ ids,
                                                     uint16_t* __restrict__ weights,
                                                     float* __restrict__ probs_out) {
  extern __shared__ float lg[];  // [kTok][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * kTok;
  const int nt = min(kTok, T - t0);

  if (logits_in) {
    for (int i = threadIdx.x; i < nt * E; i += blockDim.x)
      lg[i] = logits_in[static_cast<int64_t>(t0) * E + i];
  } else {
    for (int e = warp; e < E; e += 8) {
      float acc[kTok];
#pragma unroll
      for (int t = 0; t < kTok; ++t) acc[t] = 0.f;
      const float* wr = w + static_cast<int64_t>(e) * H;
      for (int h = lane * 4; h < H; h += 128) {
        const float4 wv = *reinterpret_cast<const float4*>(wr + h);
#pragma unroll
        for (int t = 0; t < kTok; ++t) {
          if (t >= nt) break;
          const uint2 xv = *reinterpret_cast<const uint2*>(x + static_cast<int64_t>(t0 + t) * H + h);
          acc[t] = fmaf(wv.x, bf16_to_f32(static_cast<uint16_t>(xv.x & 0xffffu)), acc[t]);
          acc[t] = fmaf(wv.y, bf16_to_f32(static_cast<uint16_t>(xv.x >> 16)), acc[t]);
          acc[t] = fmaf(wv.z, bf16_to_f32(static_cast<uint16_t>(xv.y & 0xffffu)), acc[t]);
          acc[t] = fmaf(wv.w, bf16_to_f32(static_cast<uint16_t>(xv.y >> 16)), acc[t]);
        }
      }
#pragma unroll
      for (int t = 0; t < kTok; ++t) {
        float v = acc[t];
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0 && t < nt) lg[t * E + e] = v;
      }
    }
  }
  __syncthreads();
  if (warp >= nt) return;
  const int t = t0 + warp;
  float* row = lg + warp * E;

  // softmax (numerics.py:48-51)
  float mx = -INFINITY;
  for (int e = lane; e < E; e += 32) mx = fmaxf(mx, row[e]);
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
  for (int e = lane; e < E; e += 32) {
    const float ex = expf(row[e] - mx);
    row[e] = ex;
    sum = __fadd_rn(sum, ex);
  }
  for (int o = 16; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
  for (int e = lane; e < E; e += 32) {
    row[e] = __fdiv_rn(row[e], sum);
    if (probs_out) probs_out[static_cast<int64_t>(t) * E + e] = row[e];
  }
  __syncwarp();

  // top-k: k rounds of warp argmax; ties go to the lower expert index (lax.top_k).
  float mine = 0.f;  // lane j keeps the j-th selected probability
  int mine_id = 0;
  for (int j = 0; j < k; ++j) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int e = lane; e < E; e += 32) {
      const float v = row[e];
      if (v > bv || (v == bv && e < bi)) {
        bv = v;
        bi = e;
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == j) {
      mine = bv;
      mine_id = bi;
    }
    if (lane == (bi & 31)) row[bi] = -1.f;  // probabilities are >= 0: excluded from later rounds
    __syncwarp();
  }
  // renormalise with a sequential FP32 sum over j (the oracle uses the same order)
  float total = 0.f;
  for (int j = 0; j < k; ++j) total = __fadd_rn(total, __shfl_sync(0xffffffffu, mine, j));
  if (lane < k) {
    const bool on = active ? active[t] != 0 : true;
    const float wv = on ? __fdiv_rn(mine, total) : 0.f;
    ids[static_cast<int64_t>(t) * k + lane] = mine_id;
    weights[static_cast<int64_t>(t) * k + lane] = bf16_bits_rne(wv);
  }
}

}  // namespace
}  // namespace qk

using namespace qk;

static int router_launch(const uint16_t* x, const float* w, const float* logits,
                         const uint8_t* active, int T, int H, int E, int k, int32_t* ids,
                         uint16_t* weights, float* probs, qk_stream_t stream) {
  QK_REQUIRE(T >= 0 && E > 0 && k > 0 && k <= E && k <= 32, "Invalid expert top-k");
  if (T == 0) return QK_OK;
  QK_REQUIRE(ids && weights, "null pointer");
  const size_t smem = static_cast<size_t>(kTok) * E * 4;
  QK_REQUIRE(smem <= 200 * 1024, "too many experts for the router kernel (E <= 6400)");
  int rc = allow_smem(reinterpret_cast<const void*>(router_kernel), smem);
  if (rc) return rc;
  router_kernel<<<(T + kTok - 1) / kTok, 256, smem, as_stream(stream)>>>(x, w, logits, active, T, H, E, k, ids, weights, probs);
  QK_LAUNCHED("router_kernel");
  return QK_OK;
}

extern "C" {

int qk_router_topk(const uint16_t* x, const float* router_w, const uint8_t* active, int T, int H,
                   int E, int k, int32_t* ids, uint16_t* weights, float* probs, qk_stream_t stream) {
  QK_REQUIRE(H > 0 && H % 4 == 0, "hidden must be a positive multiple of 4");
  QK_REQUIRE(T == 0 || (x && router_w), "null pointer");
  QK_REQUIRE((reinterpret_cast<uintptr_t>(x) & 7) == 0 && (reinterpret_cast<uintptr_t>(router_w) & 15) == 0,
             "x must be 8-byte and router_w 16-byte aligned");
  return router_launch(x, router_w, nullptr, active, T, H, E, k, ids, weights, probs, stream);
}

int qk_router_topk_logits(const float* logits, const uint8_t* active, int T, int E, int k,
                          int32_t* ids, uint16_t* weights, float* probs, qk_stream_t stream) {
  QK_REQUIRE(T == 0 || logits, "null pointer");
  return router_launch(nullptr, nullptr, logits, active, T, 0, E, k, ids, weights, probs, stream);
}

}  // extern "C"
