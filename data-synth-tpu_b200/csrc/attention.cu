// Split-KV decode attention over the Q8 KV cache (reference cache layout).
//
// Replaces the attention core of qwen38_tpu/attention_cache.py:152-170 (step, after the
// cache write): per batch row b and KV head h, the r = hq / kv query heads of the group
// attend over S gathered slots. Per 16-slot tile one warp
//   - gathers the int8 K rows of its 16 slots through `indices` (plain 16-byte loads),
//     dequantises them in registers to bf16(code * scale) (read_quantized, :71-81; the
//     product is exact so the only rounding is BF16 RNE) and runs QK^T as m16n8k16 MMAs
//     (16 slots x 8 heads, FP32 accumulate);
//   - forms score = bf16(bf16(qk) / sqrt(hd)) (:160-165), masks, and updates an online
//     softmax (running max / sum per head, FP32);
//   - gathers V, dequantises it into the transposed A operand and accumulates
//     O^T[d, head] += V^T P^T with P = bf16(exp(score - running max)).
// A CTA's warps take tiles of one split of the slot range; the CTA merges its warps with
// the log-sum-exp rule, and a second kernel merges the splits in split order, divides by
// the sum and applies bf16(bf16(o) * bf16(sigmoid(gate))) (:170).
// Deviation from the reference, inside the 1e-2 layer tolerance: the reference rounds the
// normalised probability to BF16 before PV; here the unnormalised exp(score - max) is
// rounded (normalisation happens after the FP32 sum).
#include "common.cuh"

namespace qk {
namespace {

constexpr int kAttnWarps = 4;
constexpr int kHeads = 8;  // query heads per KV head handled by the MMA column block

struct AttnArgs {
  const uint16_t* q;
  const int8_t* k_codes;
  const int8_t* v_codes;
  const uint16_t* k_scale;
  const uint16_t* v_scale;
  const int32_t* indices;
  const uint8_t* valid;
  const int32_t* lengths;
  const uint16_t* gate;
  uint16_t* out;
  float* part_m;  // [B, kv, splits, 8]
  float* part_l;  // [B, kv, splits, 8]
  float* part_o;  // [B, kv, splits, 8, hd]
  int B, S, T, hq, kv, r, splits, tiles_per_split;
  float div;      // f32(sqrt(hd))
};

__device__ __forceinline__ int wrap_clamp(int t, int T) {
  if (t < 0) t += T;
  return t < 0 ? 0 : (t >= T ? T - 1 : t);
}

// Signed int8 byte i of `w` as FP32 (exact), via 2^23 + (byte ^ 0x80) - (2^23 + 128).
template <int I>
__device__ __forceinline__ float s8_at(uint32_t wx) {
  return __uint_as_float(__byte_perm(wx, 0x4bu, 0x4550u | I));
}

__device__ __forceinline__ uint32_t dq_pair(float c0, float c1, float s0, float s1) {
  const float2 code = __fadd2_rn(make_float2(c0, c1), make_float2(-8388736.f, -8388736.f));
  const float2 v = __fmul2_rn(code, make_float2(s0, s1));
  return pack_bf16x2(v.x, v.y);
}

__device__ __forceinline__ float output_value(float o, const uint16_t* gate, int64_t gi) {
  float v = bf16_round(o);
  if (gate) v = bf16_round(__fmul_rn(v, bf16_round(sigmoid_ref(bf16_to_f32(gate[gi])))));
  return v;
}

template <int HD>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_split_kernel(AttnArgs a) {
  constexpr int KSTEPS = HD / 16;      // QK k-steps over d
  constexpr int KB = HD / 4;           // K bytes per lane per token row
  constexpr int KV4 = KB / 16;         // uint4 per K row
  constexpr int VB = HD / 8;           // V bytes per lane per token
  constexpr int VV4 = VB / 16 > 0 ? VB / 16 : 1;
  constexpr int MT = HD / 16;          // PV m-tiles over d
  static_assert(HD == 128 || HD == 256, "head_dim 128 or 256");

  __shared__ __align__(16) uint16_t q_s[kHeads * HD];
  __shared__ float m_s[kAttnWarps][kHeads], l_s[kAttnWarps][kHeads];
  __shared__ float o_s[kAttnWarps][kHeads][HD];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int G = a.kv * HD / 32;

  for (int i = threadIdx.x; i < kHeads * HD; i += blockDim.x) {
    const int r = i / HD, d = i % HD;
    q_s[i] = r < a.r ? a.q[(static_cast<int64_t>(b) * a.hq + h * a.r + r) * HD + d] : 0;
  }
  __syncthreads();

  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float o_acc[MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) o_acc[mt][0] = o_acc[mt][1] = o_acc[mt][2] = o_acc[mt][3] = 0.f;

  const int ntiles = (a.S + 15) / 16;
  const int t_begin = split * a.tiles_per_split;
  const int t_end = min(ntiles, t_begin + a.tiles_per_split);
  const int len = a.lengths ? a.lengths[b] : a.S;

  for (int tile = t_begin + warp; tile < t_end; tile += kAttnWarps) {
    const int s0 = tile * 16;
    // ---- K: rows g, g+8 of the tile; lane quarter c holds d in [c*KB, (c+1)*KB) ----
    int tk[2];
    bool vk[2];
#pragma unroll
    for (int rh = 0; rh < 2; ++rh) {
      const int s = s0 + g + 8 * rh;
      const bool in = s < a.S;
      tk[rh] = in ? wrap_clamp(a.indices[static_cast<int64_t>(b) * a.S + s], a.T) : 0;
      vk[rh] = in && (a.valid ? a.valid[static_cast<int64_t>(b) * a.S + s] != 0 : s <= len);
    }
    uint4 kw[2][KV4];
    float ks[2][2];
#pragma unroll
    for (int rh = 0; rh < 2; ++rh) {
      const int8_t* row = a.k_codes + ((static_cast<int64_t>(b) * a.T + tk[rh]) * a.kv + h) * HD + c * KB;
#pragma unroll
      for (int i = 0; i < KV4; ++i) kw[rh][i] = ld_nc_v4(row + 16 * i);
      const int grp0 = h * (HD / 32) + (c * KB) / 32;
#pragma unroll
      for (int i = 0; i < (KB >= 32 ? KB / 32 : 1); ++i)
        ks[rh][i] = bf16_to_f32(a.k_scale[(static_cast<int64_t>(b) * G + grp0 + i) * a.T + tk[rh]]);
    }
    float sacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int st = 0; st < KSTEPS; ++st) {
      const int gi = (st * 4) / 32;  // scale group inside this lane's K bytes
      uint32_t af[4];
#pragma unroll
      for (int rh = 0; rh < 2; ++rh) {
        const uint32_t wx = word(kw[rh][st / 4], st % 4) ^ 0x80808080u;
        const float sc = ks[rh][KB >= 32 ? gi : 0];
        af[rh] = dq_pair(s8_at<0>(wx), s8_at<1>(wx), sc, sc);
        af[2 + rh] = dq_pair(s8_at<2>(wx), s8_at<3>(wx), sc, sc);
      }
      const uint2 qb = *reinterpret_cast<const uint2*>(&q_s[g * HD + c * KB + st * 4]);
      mma_bf16(sacc, af, qb.x, qb.y);
    }
    // ---- V loads (tokens 2c, 2c+1, 2c+8, 2c+9; d in [g*VB, (g+1)*VB)) issued early ----
    uint4 vw[4][VV4];
    float vs[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int s = s0 + 2 * c + (i & 1) + 8 * (i >> 1);
      const int t = s < a.S ? wrap_clamp(a.indices[static_cast<int64_t>(b) * a.S + s], a.T) : 0;
      const int8_t* row = a.v_codes + ((static_cast<int64_t>(b) * a.T + t) * a.kv + h) * HD + g * VB;
#pragma unroll
      for (int j = 0; j < VV4; ++j) vw[i][j] = ld_nc_v4(row + 16 * j);
      vs[i] = bf16_to_f32(a.v_scale[(static_cast<int64_t>(b) * G + h * (HD / 32) + (g * VB) / 32) * a.T + t]);
    }
    // ---- scores, online softmax (heads 2c, 2c+1; tokens g, g+8) ----
    float p[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const bool valid = vk[i >> 1];
      const float raw = bf16_round(sacc[i]);
      p[i] = valid ? bf16_round(__fdiv_rn(raw, a.div)) : -INFINITY;
    }
    float alpha[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float mt = fmaxf(p[hh], p[2 + hh]);
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
      mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
      const float m_new = fmaxf(m_run[hh], mt);
      if (m_new == -INFINITY) {
        alpha[hh] = 1.f;
        p[hh] = p[2 + hh] = 0.f;
      } else {
        alpha[hh] = expf(m_run[hh] - m_new);
        p[hh] = expf(p[hh] - m_new);
        p[2 + hh] = expf(p[2 + hh] - m_new);
      }
      m_run[hh] = m_new;
    }
    // P in BF16 (the MMA operand); the running sum uses the same rounded values.
    const uint32_t P0 = pack_bf16x2(p[0], p[1]), P1 = pack_bf16x2(p[2], p[3]);
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float ps = __fadd_rn(bf16_to_f32(static_cast<uint16_t>(P0 >> (16 * hh))),
                           bf16_to_f32(static_cast<uint16_t>(P1 >> (16 * hh))));
      ps += __shfl_xor_sync(0xffffffffu, ps, 4);
      ps += __shfl_xor_sync(0xffffffffu, ps, 8);
      ps += __shfl_xor_sync(0xffffffffu, ps, 16);
      l_run[hh] = __fadd_rn(__fmul_rn(l_run[hh], alpha[hh]), ps);
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      o_acc[mt][0] *= alpha[0];
      o_acc[mt][1] *= alpha[1];
      o_acc[mt][2] *= alpha[0];
      o_acc[mt][3] *= alpha[1];
    }
    const uint32_t b0 = movmatrix_trans(P0), b1 = movmatrix_trans(P1);
    // ---- PV: O^T[d, head] += V^T[d, tok] P^T[tok, head]; d0 = g*VB + 2 mt, d1 = d0 + 1 ----
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int byte = 2 * mt;                 // inside this lane's VB bytes
      const int wi = (byte / 4) % 4, vi = byte / 16;
      uint32_t af[4];
      uint32_t wx[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) wx[i] = word(vw[i][vi], wi) ^ 0x80808080u;
      const int lo = byte & 3;  // 0 or 2
      if (lo == 0) {
        af[0] = dq_pair(s8_at<0>(wx[0]), s8_at<0>(wx[1]), vs[0], vs[1]);
        af[1] = dq_pair(s8_at<1>(wx[0]), s8_at<1>(wx[1]), vs[0], vs[1]);
        af[2] = dq_pair(s8_at<0>(wx[2]), s8_at<0>(wx[3]), vs[2], vs[3]);
        af[3] = dq_pair(s8_at<1>(wx[2]), s8_at<1>(wx[3]), vs[2], vs[3]);
      } else {
        af[0] = dq_pair(s8_at<2>(wx[0]), s8_at<2>(wx[1]), vs[0], vs[1]);
        af[1] = dq_pair(s8_at<3>(wx[0]), s8_at<3>(wx[1]), vs[0], vs[1]);
        af[2] = dq_pair(s8_at<2>(wx[2]), s8_at<2>(wx[3]), vs[2], vs[3]);
        af[3] = dq_pair(s8_at<3>(wx[2]), s8_at<3>(wx[3]), vs[2], vs[3]);
      }
      mma_bf16(o_acc[mt], af, b0, b1);
    }
  }

  // ---- merge the CTA's warps (log-sum-exp), write the split partial or the output ----
  if (g == 0) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      m_s[warp][2 * c + hh] = m_run[hh];
      l_s[warp][2 * c + hh] = l_run[hh];
    }
  }
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const int d0 = g * VB + 2 * mt;
    o_s[warp][2 * c][d0] = o_acc[mt][0];
    o_s[warp][2 * c + 1][d0] = o_acc[mt][1];
    o_s[warp][2 * c][d0 + 1] = o_acc[mt][2];
    o_s[warp][2 * c + 1][d0 + 1] = o_acc[mt][3];
  }
  __syncthreads();
  const int64_t pbase = (static_cast<int64_t>(b) * a.kv + h) * a.splits + split;
  for (int i = threadIdx.x; i < kHeads * HD; i += blockDim.x) {
    const int r = i / HD, d = i % HD;
    float M = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, m_s[w][r]);
    float L = 0.f, O = 0.f;
    for (int w = 0; w < kAttnWarps; ++w) {
      const float f = m_s[w][r] == -INFINITY ? 0.f : expf(m_s[w][r] - M);
      L = __fadd_rn(L, __fmul_rn(l_s[w][r], f));
      O = __fadd_rn(O, __fmul_rn(o_s[w][r][d], f));
    }
    if (a.splits == 1) {
      if (r < a.r) {
        const int64_t oi = (static_cast<int64_t>(b) * a.hq + h * a.r + r) * HD + d;
        a.out[oi] = bf16_bits_rne(output_value(__fdiv_rn(O, L), a.gate, oi));
      }
    } else {
      a.part_o[pbase * kHeads * HD + i] = O;
      if (d == 0) {
        a.part_m[pbase * kHeads + r] = M;
        a.part_l[pbase * kHeads + r] = L;
      }
    }
  }
}

template <int HD>
__global__ void attn_merge_kernel(AttnArgs a) {
  const int h = blockIdx.x, b = blockIdx.y;
  const int64_t base = (static_cast<int64_t>(b) * a.kv + h) * a.splits;
  for (int i = threadIdx.x; i < a.r * HD; i += blockDim.x) {
    const int r = i / HD, d = i % HD;
    float M = -INFINITY;
    for (int s = 0; s < a.splits; ++s) M = fmaxf(M, a.part_m[(base + s) * kHeads + r]);
    float L = 0.f, O = 0.f;
    for (int s = 0; s < a.splits; ++s) {
      const float ms = a.part_m[(base + s) * kHeads + r];
      const float f = ms == -INFINITY ? 0.f : expf(ms - M);
      L = __fadd_rn(L, __fmul_rn(a.part_l[(base + s) * kHeads + r], f));
      O = __fadd_rn(O, __fmul_rn(a.part_o[((base + s) * kHeads + r) * HD + d], f));
    }
    const int64_t oi = (static_cast<int64_t>(b) * a.hq + h * a.r + r) * HD + d;
    a.out[oi] = bf16_bits_rne(output_value(__fdiv_rn(O, L), a.gate, oi));
  }
}

int choose_splits(int B, int kv, int S) {
  const int ntiles = (S + 15) / 16;
  const int target = sm_count() * 3;                 // CTAs in flight
  int splits = (target + B * kv - 1) / (B * kv);
  const int max_splits = (ntiles + kAttnWarps - 1) / kAttnWarps;  // >= one tile per warp
  if (splits > max_splits) splits = max_splits;
  return splits < 1 ? 1 : splits;
}

size_t part_bytes(int B, int kv, int splits, int hd) {
  const size_t n = static_cast<size_t>(B) * kv * splits * kHeads;
  return n * 4 * 2 + n * hd * 4 + 256;
}

}  // namespace
}  // namespace qk

using namespace qk;

extern "C" {

size_t qk_kv_q8_attention_workspace_bytes(int B, int S, int hq, int kv_heads, int head_dim) {
  if (B <= 0 || S <= 0 || kv_heads <= 0 || head_dim <= 0) return 0;
  (void)hq;
  const int splits = choose_splits(B, kv_heads, S);
  return splits > 1 ? part_bytes(B, kv_heads, splits, head_dim) : 0;
}

int qk_kv_q8_decode_attention(const uint16_t* q, const int8_t* k_codes, const int8_t* v_codes,
                              const uint16_t* k_scale, const uint16_t* v_scale,
                              const int32_t* indices, const uint8_t* valid, const int32_t* lengths,
                              const uint16_t* gate, int B, int S, int T, int hq, int kv_heads,
                              int head_dim, uint16_t* out, void* workspace, size_t workspace_bytes,
                              qk_stream_t stream) {
  QK_REQUIRE(B >= 0 && S > 0 && T > 0 && hq > 0 && kv_heads > 0, "invalid attention geometry");
  QK_REQUIRE(hq % kv_heads == 0, "Head counts must have integer repetition factors");
  QK_REQUIRE(hq / kv_heads <= kHeads, "at most %d query heads per KV head", kHeads);
  QK_REQUIRE(head_dim == 128 || head_dim == 256, "head_dim must be 128 or 256");
  QK_REQUIRE(valid || lengths, "either valid or lengths is required");
  if (B == 0) return QK_OK;
  QK_REQUIRE(q && k_codes && v_codes && k_scale && v_scale && indices && out, "null pointer");
  AttnArgs a{};
  a.q = q; a.k_codes = k_codes; a.v_codes = v_codes; a.k_scale = k_scale; a.v_scale = v_scale;
  a.indices = indices; a.valid = valid; a.lengths = valid ? nullptr : lengths; a.gate = gate; a.out = out;
  a.B = B; a.S = S; a.T = T; a.hq = hq; a.kv = kv_heads; a.r = hq / kv_heads;
  a.splits = choose_splits(B, kv_heads, S);
  const int ntiles = (S + 15) / 16;
  a.tiles_per_split = (ntiles + a.splits - 1) / a.splits;
  a.splits = (ntiles + a.tiles_per_split - 1) / a.tiles_per_split;
  a.div = sqrtf(static_cast<float>(head_dim));
  if (a.splits > 1) {
    const size_t need = part_bytes(B, kv_heads, a.splits, head_dim);
    if (!workspace || workspace_bytes < need)
      return set_error(QK_ERR_WORKSPACE, "attention workspace needs %zu bytes, got %zu", need, workspace_bytes);
    const size_t n = static_cast<size_t>(B) * kv_heads * a.splits * kHeads;
    a.part_m = static_cast<float*>(workspace);
    a.part_l = a.part_m + n;
    a.part_o = a.part_l + n;
  }
  cudaStream_t st = as_stream(stream);
  dim3 grid(a.splits, kv_heads, B);
  if (head_dim == 256) attn_split_kernel<256><<<grid, kAttnWarps * 32, 0, st>>>(a);
  else attn_split_kernel<128><<<grid, kAttnWarps * 32, 0, st>>>(a);
  QK_LAUNCHED("attn_split_kernel");
  if (a.splits > 1) {
    if (head_dim == 256) attn_merge_kernel<256><<<dim3(kv_heads, B), 256, 0, st>>>(a);
    else attn_merge_kernel<128><<<dim3(kv_heads, B), 256, 0, st>>>(a);
    QK_LAUNCHED("attn_merge_kernel");
  }
  return QK_OK;
}

}  // extern "C"
