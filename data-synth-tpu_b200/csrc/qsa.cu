// Sparse-attention token selection (QSA indexer) feeding the Q8 KV decode attention.
//
// Replaces the selection half of qwen38_tpu/attention_cache.py:84-125 (select_tokens), after
// the block keys are up to date:
//   scores[b, t] = sum_h relu(q[b, h] . keys[b, t]) / sqrt(dim)   (FP32, :100-112)
//   scores[b, t] = -inf for t >= count, count = (lengths[b] + 1) // ratio   (:113-114)
//   selected = lax.top_k(scores, K), K = min(budget // ratio, blocks)      (:115-116)
//   indices = [selected * ratio + r for r < ratio] ++ [count * ratio + j for j < ratio - 1]
//   valid   = [selected < count] * ratio ++ [j < (lengths + 1) % ratio]   (:117-122)
//   indices = where(valid, indices, 0)                                      (:123-124)
//
// qsa_scores_kernel: HBM-bound pass over the block keys (dim BF16 values per block); a warp
// takes four blocks at a time, its lanes split the dimension, and the query heads live in
// shared memory. qsa_select_kernel: one CTA per row; radix select (4 passes of 8 bits over
// an order-preserving key of the FP32 score) finds the K-th largest score, a block-wide scan
// keeps every larger score and the lowest-index equal ones (lax.top_k's tie rule), and a
// bitonic sort orders the K blocks by (score descending, index ascending), top_k's order.
#include <algorithm>
#include <cmath>

#include "common.cuh"

namespace qk {
namespace {

constexpr int kScoreWarps = 8;
constexpr int kBlocksPerWarp = 4;  // blocks a warp scores at once (loads in flight)
constexpr int kSelThreads = 1024;
constexpr int kMaxHeads = 8, kMaxDim = 256, kMaxK = 1024, kMaxBlocks = 16384;

// PER = dim / 32 values of each block's key per lane (2, 4 or 8: dim 64, 128 or 256).
template <int PER>
__global__ void __launch_bounds__(kScoreWarps * 32) qsa_scores_kernel(const uint16_t* __restrict__ query,
                                                                      const uint16_t* __restrict__ keys,
                                                                      const int32_t* __restrict__ lengths, int heads,
                                                                      int blocks, int ratio, float root,
                                                                      float* __restrict__ scores) {
  constexpr int dim = PER * 32;
  __shared__ float qs[kMaxHeads * kMaxDim];
  const int b = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < heads * dim; i += blockDim.x)
    qs[i] = bf16_to_f32(query[static_cast<int64_t>(b) * heads * dim + i]);
  __syncthreads();
  const int count = (lengths[b] + 1) / ratio;
  const int t0 = (blockIdx.x * kScoreWarps + warp) * kBlocksPerWarp;
  const uint16_t* kb = keys + static_cast<int64_t>(b) * blocks * dim;
  uint32_t raw[kBlocksPerWarp][PER / 2];  // the lane's PER BF16 values of each block
#pragma unroll
  for (int u = 0; u < kBlocksPerWarp; ++u) {
    const int t = t0 + u;
    const uint16_t* row = kb + static_cast<int64_t>(t < blocks ? t : 0) * dim + lane * PER;
    if constexpr (PER == 8) {
      const uint4 v = t < blocks ? *reinterpret_cast<const uint4*>(row) : make_uint4(0, 0, 0, 0);
      raw[u][0] = v.x;
      raw[u][1] = v.y;
      raw[u][2] = v.z;
      raw[u][3] = v.w;
    } else if constexpr (PER == 4) {
      const uint2 v = t < blocks ? *reinterpret_cast<const uint2*>(row) : make_uint2(0, 0);
      raw[u][0] = v.x;
      raw[u][1] = v.y;
    } else {
      raw[u][0] = t < blocks ? *reinterpret_cast<const uint32_t*>(row) : 0u;
    }
  }
#pragma unroll
  for (int u = 0; u < kBlocksPerWarp; ++u) {
    const int t = t0 + u;
    float score = 0.f;
    for (int h = 0; h < heads; ++h) {
      const float* q = qs + h * dim + lane * PER;
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < PER; ++j)
        dot = fmaf(q[j], bf16_to_f32(static_cast<uint16_t>(raw[u][j / 2] >> (16 * (j & 1)))), dot);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      score = __fadd_rn(score, fmaxf(dot, 0.f));
    }
    if (lane == 0 && t < blocks)
      scores[static_cast<int64_t>(b) * blocks + t] = t < count ? __fdiv_rn(score, root) : -INFINITY;
  }
}

// Order-preserving map of an FP32 score to an unsigned key (larger score, larger key).
__device__ __forceinline__ uint32_t score_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Exclusive block-wide scan of one int per thread (kSelThreads threads); returns the total.
__device__ __forceinline__ int block_scan(int v, int* warp_sums, int* excl) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  __syncthreads();  // warp_sums may still be read by a previous scan
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int s = warp_sums[lane];
    int si = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, si, o);
      if (lane >= o) si += n;
    }
    warp_sums[lane] = si - s;  // exclusive prefix of the warp totals
    if (lane == 31) warp_sums[32] = si;
  }
  __syncthreads();
  *excl = warp_sums[warp] + incl - v;
  return warp_sums[32];
}

__global__ void __launch_bounds__(kSelThreads) qsa_select_kernel(const float* __restrict__ scores,
                                                                 const int32_t* __restrict__ lengths, int blocks,
                                                                 int ratio, int K, int width,
                                                                 int32_t* __restrict__ indices,
                                                                 uint8_t* __restrict__ valid) {
  extern __shared__ uint32_t keys[];                        // [blocks]
  __shared__ uint32_t sel_key[kMaxK];
  __shared__ int32_t sel_idx[kMaxK];
  __shared__ int hist[256];
  __shared__ int warp_sums[33];
  __shared__ uint32_t s_prefix;
  __shared__ int s_remaining;
  const int b = blockIdx.x, tid = threadIdx.x;
  const float* row = scores + static_cast<int64_t>(b) * blocks;
  for (int i = tid; i < blocks; i += kSelThreads) keys[i] = score_key(row[i]);
  if (tid == 0) {
    s_prefix = 0;
    s_remaining = K;
  }
  __syncthreads();

  // radix select of the K-th largest key, 8 bits at a time from the top
  uint32_t mask = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += kSelThreads) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix;
    // one shared-memory atomic per distinct bin of a warp (scores that share their top bits
    // would otherwise serialise on one counter)
    for (int i = tid; i < blocks; i += kSelThreads) {
      const uint32_t k = keys[i];
      const uint32_t bin = (k & mask) == prefix ? (k >> shift) & 255u : 256u;
      const unsigned peers = __match_any_sync(__activemask(), bin);
      if (bin < 256u && (tid & 31) == __ffs(peers) - 1) atomicAdd(&hist[bin], __popc(peers));
    }
    __syncthreads();
    if (tid < 32) {
      // warp 0 finds the bin holding the need-th largest key: lane l sums bins 8l .. 8l + 7,
      // a suffix scan gives the count above each lane's bins, and the lane whose bins
      // reach `need` walks them from the top
      const int lane = tid, need = s_remaining;
      int mine = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) mine += hist[8 * lane + j];
      int suffix = mine;  // keys in the bins of this lane and every higher lane
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_down_sync(0xffffffffu, suffix, o);
        if (lane + o < 32) suffix += n;
      }
      const int above = suffix - mine;  // keys in the bins of higher lanes
      const bool here = above < need && suffix >= need;  // exactly one lane
      if (here) {
        int acc = above, bin = 8 * lane + 7;
        for (; bin > 8 * lane; --bin) {
          if (acc + hist[bin] >= need) break;
          acc += hist[bin];
        }
        s_remaining = need - acc;  // how many keys of this bin (and prefix) still to take
        s_prefix = prefix | (static_cast<uint32_t>(bin) << shift);
      }
    }
    mask |= 255u << shift;
    __syncthreads();
  }
  const uint32_t T = s_prefix;
  const int take_equal = s_remaining;  // keys equal to T to keep, lowest block index first

  // keep every key > T and the first take_equal keys == T (in block order): each thread
  // scans a contiguous chunk of blocks
  const int per = (blocks + kSelThreads - 1) / kSelThreads;
  const int lo = min(blocks, tid * per), hi = min(blocks, lo + per);
  int n_eq = 0;
  for (int i = lo; i < hi; ++i) n_eq += keys[i] == T;
  int eq_before = 0;
  block_scan(n_eq, warp_sums, &eq_before);
  int n_take = 0;
  {
    int e = eq_before;
    for (int i = lo; i < hi; ++i) {
      const uint32_t k = keys[i];
      if (k > T) ++n_take;
      else if (k == T) n_take += e++ < take_equal;
    }
  }
  int pos = 0;
  block_scan(n_take, warp_sums, &pos);
  {
    int e = eq_before;
    for (int i = lo; i < hi; ++i) {
      const uint32_t k = keys[i];
      const bool take = k > T || (k == T && e++ < take_equal);
      if (take && pos < K) {
        sel_key[pos] = k;
        sel_idx[pos] = i;
        ++pos;
      }
    }
  }
  __syncthreads();
  // sort the K kept blocks by (key descending, index ascending): thread t holds element t of
  // a 1024-entry bitonic network as one 64-bit value key << 32 | ~index (padding sorts last);
  // strides below 32 exchange by warp shuffle, larger ones through shared memory
  uint64_t v = tid < K ? (static_cast<uint64_t>(sel_key[tid]) << 32) | (0xffffffffu - static_cast<uint32_t>(sel_idx[tid]))
                       : 0ull;
  uint64_t* xch = reinterpret_cast<uint64_t*>(keys);  // the keys are no longer needed
  for (int size = 2; size <= kSelThreads; size <<= 1) {
    const bool desc = (tid & size) == 0;
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      uint64_t other;
      if (stride >= 32) {
        __syncthreads();
        xch[tid] = v;
        __syncthreads();
        other = xch[tid ^ stride];
      } else {
        other = __shfl_xor_sync(0xffffffffu, v, stride);
      }
      const bool lower = (tid & stride) == 0;
      v = (lower == desc) ? (v > other ? v : other) : (v < other ? v : other);
    }
  }
  __syncthreads();
  if (tid < K) sel_idx[tid] = static_cast<int32_t>(0xffffffffu - static_cast<uint32_t>(v));
  __syncthreads();
  // expand to token indices and flags
  const int len1 = lengths[b] + 1, count = len1 / ratio;
  int32_t* out_i = indices + static_cast<int64_t>(b) * width;
  uint8_t* out_v = valid + static_cast<int64_t>(b) * width;
  for (int i = tid; i < K * ratio; i += kSelThreads) {
    const int blk = sel_idx[i / ratio];
    const bool ok = blk < count;
    out_i[i] = ok ? blk * ratio + i % ratio : 0;
    out_v[i] = ok;
  }
  for (int j = tid; j < ratio - 1; j += kSelThreads) {
    const bool ok = j < len1 % ratio;
    out_i[K * ratio + j] = ok ? count * ratio + j : 0;
    out_v[K * ratio + j] = ok;
  }
}

// ---- the key-maintenance half of select_tokens (attention_cache.py:86-99) ----

struct QsaRope {
  const float* inv_freq;  // [rotary / 2]: theta^(-2i / rotary)
  const int32_t* axis;    // [rotary / 2]: which of the 3 position components rotates pair i
  int rotary;
};

// In place on v[0 .. dim) of one thread block (thread d owns v[d]; dim <= blockDim.x):
// math.py:27-31 rms with gamma, then math.py:231-243 rope at positions pos[3] (the
// rotary cosine and sine rounded to BF16). Returns this thread's BF16 result.
__device__ float rms_rope(float v, int d, int dim, const uint16_t* gamma, float eps, const int32_t* pos,
                          const QsaRope& rp, float* red, float* row) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  float ss = d < dim ? v * v : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  __syncthreads();
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < nw; ++w) tot += red[w];
  const float r = rsqrtf(__fadd_rn(__fdiv_rn(tot, static_cast<float>(dim)), eps));
  if (d < dim) row[d] = bf16_round(__fmul_rn(__fmul_rn(v, r), bf16_to_f32(gamma[d])));
  __syncthreads();
  if (d >= dim) return 0.f;
  float o = row[d];
  const int half = rp.rotary / 2;
  if (d < rp.rotary) {
    const int i = d < half ? d : d - half;
    const float angle = __fmul_rn(static_cast<float>(pos[rp.axis[i]]), rp.inv_freq[i]);
    const float cs = bf16_round(cosf(angle)), sn = bf16_round(sinf(angle));
    const float a = row[i], c = row[i + half];
    o = bf16_round(d < half ? __fsub_rn(__fmul_rn(a, cs), __fmul_rn(c, sn)) : __fadd_rn(__fmul_rn(c, cs), __fmul_rn(a, sn)));
  }
  return o;
}

// One block per row b (thread d = channel d): write this step's raw key into the tail at
// slot lengths % ratio (active rows), note the block start on slot 0, pool the tail (FP32
// mean, BF16), rms + rope it at the block start and, on the block's last slot, store it as
// key lengths / ratio.
__global__ void qsa_update_keys_kernel(const uint16_t* __restrict__ raw_k, const int32_t* __restrict__ lengths,
                                       const int32_t* __restrict__ positions, const uint8_t* __restrict__ active,
                                       const uint16_t* __restrict__ k_norm, float eps, QsaRope rp, int ratio, int dim,
                                       int blocks, uint16_t* tail, int32_t* starts, uint16_t* keys) {
  __shared__ float red[32];
  __shared__ float row[kMaxDim];
  const int b = blockIdx.x, d = threadIdx.x;
  const bool on = active ? active[b] != 0 : true;
  const int len = lengths[b], slot = len % ratio;
  uint16_t* tb = tail + static_cast<int64_t>(b) * ratio * dim;
  if (on && d < dim) tb[slot * dim + d] = raw_k[static_cast<int64_t>(b) * dim + d];
  __syncthreads();
  if (on && slot == 0 && d < 3) starts[b * 3 + d] = positions[b * 3 + d];
  float sum = 0.f;
  if (d < dim)
    for (int j = 0; j < ratio; ++j) sum = __fadd_rn(sum, bf16_to_f32(tb[j * dim + d]));
  const float pooled = bf16_round(__fdiv_rn(sum, static_cast<float>(ratio)));
  __syncthreads();  // every thread has read starts[] written above before rms_rope reads it
  int32_t st[3];
  for (int c = 0; c < 3; ++c) st[c] = starts[b * 3 + c];
  const float key = rms_rope(pooled, d, dim, k_norm, eps, st, rp, red, row);
  const int blk = len / ratio;
  if (on && slot == ratio - 1 && d < dim && blk < blocks)
    keys[(static_cast<int64_t>(b) * blocks + blk) * dim + d] = bf16_bits_rne(key);
}

// Block (row b, head h): rms + rope of the query head at positions[b] (attention_cache.py:98-99).
__global__ void qsa_query_kernel(const uint16_t* __restrict__ raw_q, const int32_t* __restrict__ positions,
                                 const uint16_t* __restrict__ q_norm, float eps, QsaRope rp, int heads, int dim,
                                 uint16_t* __restrict__ query) {
  __shared__ float red[32];
  __shared__ float row[kMaxDim];
  const int b = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const int64_t base = (static_cast<int64_t>(b) * heads + h) * dim;
  const float v = d < dim ? bf16_to_f32(raw_q[base + d]) : 0.f;
  int32_t pos[3];
  for (int c = 0; c < 3; ++c) pos[c] = positions[b * 3 + c];
  const float o = rms_rope(v, d, dim, q_norm, eps, pos, rp, red, row);
  if (d < dim) query[base + d] = bf16_bits_rne(o);
}

}  // namespace
}  // namespace qk

using namespace qk;

extern "C" {

int qk_qsa_update_keys(const uint16_t* raw_k, const int32_t* lengths, const int32_t* positions,
                       const uint8_t* active, const uint16_t* k_norm, float eps, const float* inv_freq,
                       const int32_t* axis, int rotary, int B, int ratio, int dim, int blocks, uint16_t* tail,
                       int32_t* starts, uint16_t* keys, qk_stream_t stream) {
  QK_REQUIRE(B >= 0 && ratio >= 2 && blocks > 0, "invalid indexer geometry");
  QK_REQUIRE(dim > 0 && dim <= kMaxDim && rotary >= 0 && rotary <= dim && rotary % 2 == 0, "invalid indexer dim");
  if (B == 0) return QK_OK;
  QK_REQUIRE(raw_k && lengths && positions && k_norm && tail && starts && keys, "null pointer");
  QK_REQUIRE(rotary == 0 || (inv_freq && axis), "inv_freq and axis are required");
  const int threads = (dim + 31) / 32 * 32;
  qsa_update_keys_kernel<<<B, threads, 0, as_stream(stream)>>>(raw_k, lengths, positions, active, k_norm, eps,
                                                               QsaRope{inv_freq, axis, rotary}, ratio, dim, blocks,
                                                               tail, starts, keys);
  QK_LAUNCHED("qsa_update_keys_kernel");
  return QK_OK;
}

int qk_qsa_query(const uint16_t* raw_q, const int32_t* positions, const uint16_t* q_norm, float eps,
                 const float* inv_freq, const int32_t* axis, int rotary, int B, int heads, int dim, uint16_t* query,
                 qk_stream_t stream) {
  QK_REQUIRE(B >= 0 && heads > 0, "invalid indexer geometry");
  QK_REQUIRE(dim > 0 && dim <= kMaxDim && rotary >= 0 && rotary <= dim && rotary % 2 == 0, "invalid indexer dim");
  if (B == 0) return QK_OK;
  QK_REQUIRE(raw_q && positions && q_norm && query, "null pointer");
  QK_REQUIRE(rotary == 0 || (inv_freq && axis), "inv_freq and axis are required");
  const int threads = (dim + 31) / 32 * 32;
  qsa_query_kernel<<<dim3(B, heads), threads, 0, as_stream(stream)>>>(raw_q, positions, q_norm, eps,
                                                                      QsaRope{inv_freq, axis, rotary}, heads, dim,
                                                                      query);
  QK_LAUNCHED("qsa_query_kernel");
  return QK_OK;
}

int qk_qsa_block_scores(const uint16_t* query, const uint16_t* keys, const int32_t* lengths, int B, int heads,
                        int dim, int blocks, int ratio, float* scores, qk_stream_t stream) {
  QK_REQUIRE(B >= 0 && blocks > 0 && ratio >= 2, "invalid indexer geometry");
  QK_REQUIRE(heads >= 1 && heads <= kMaxHeads, "indexer heads must be in [1, %d]", kMaxHeads);
  QK_REQUIRE(dim == 64 || dim == 128 || dim == 256, "indexer dim must be 64, 128 or 256");
  if (B == 0) return QK_OK;
  QK_REQUIRE(query && keys && lengths && scores, "null pointer");
  const int per_cta = kScoreWarps * kBlocksPerWarp;
  const dim3 grid((blocks + per_cta - 1) / per_cta, B);
  QK_REQUIRE((reinterpret_cast<uintptr_t>(keys) & 15) == 0, "keys must be 16-byte aligned");
  const float root = static_cast<float>(std::sqrt(static_cast<double>(dim)));
  const cudaStream_t st = as_stream(stream);
  if (dim == 64)
    qsa_scores_kernel<2><<<grid, kScoreWarps * 32, 0, st>>>(query, keys, lengths, heads, blocks, ratio, root, scores);
  else if (dim == 128)
    qsa_scores_kernel<4><<<grid, kScoreWarps * 32, 0, st>>>(query, keys, lengths, heads, blocks, ratio, root, scores);
  else
    qsa_scores_kernel<8><<<grid, kScoreWarps * 32, 0, st>>>(query, keys, lengths, heads, blocks, ratio, root, scores);
  QK_LAUNCHED("qsa_scores_kernel");
  return QK_OK;
}

int qk_qsa_select(const float* scores, const int32_t* lengths, int B, int blocks, int ratio, int budget,
                  int32_t* indices, uint8_t* valid, qk_stream_t stream) {
  QK_REQUIRE(B >= 0 && blocks > 0 && ratio >= 2, "invalid indexer geometry");
  QK_REQUIRE(blocks <= kMaxBlocks, "at most %d index blocks per row", kMaxBlocks);
  QK_REQUIRE(budget >= ratio && budget % ratio == 0, "Invalid sparse attention indexer dimensions or budget");
  const int K = min(budget / ratio, blocks);
  QK_REQUIRE(K <= kMaxK, "at most %d selected blocks", kMaxK);
  if (B == 0) return QK_OK;
  QK_REQUIRE(scores && lengths && indices && valid, "null pointer");
  const int width = K * ratio + ratio - 1;
  // keys [blocks] (4 B each), reused as the sort's 1024 x 8 B exchange buffer
  const size_t smem = std::max(static_cast<size_t>(blocks) * 4, static_cast<size_t>(kSelThreads) * 8);
  if (int rc = allow_smem(reinterpret_cast<const void*>(qsa_select_kernel), smem)) return rc;
  qsa_select_kernel<<<B, kSelThreads, smem, as_stream(stream)>>>(scores, lengths, blocks, ratio, K, width, indices,
                                                                 valid);
  QK_LAUNCHED("qsa_select_kernel");
  return QK_OK;
}

}  // extern "C"
