// Split-KV decode attention over the Q8 KV cache (reference cache layout).
//
// Replaces the attention core of qwen38_tpu/attention_cache.py:152-170 (step, after the
// cache write): per batch row b and KV head h (a "pair"), the r = hq / kv query heads of
// the group attend over S gathered slots.
//
// Work split (stream-K): a pair's slots form tiles of 16; the B * kv * ceil(S/16) tiles of
// all pairs are cut into one contiguous, equal range per CTA (one CTA per SM), so the
// grid is balanced whatever B and S are. A CTA walks the pairs its range touches in order;
// its warps take the tiles of that range round robin. Per tile a warp
//   - gathers the int8 K and V rows of its 16 slots through `indices` with cp.async into a
//     three-stage ring of its own in shared memory (two tiles in flight while it computes
//     the third; XOR-swizzled so the fragment loads below are free of bank conflicts),
//     and the BF16 scales: two 16-byte copies per group when the tile's cache times are
//     16 consecutive, 8-aligned times (any page table of 16-multiple pages), else one
//     load per scale;
//   - dequantises K in registers to bf16(code * scale) (read_quantized, :71-81; the product
//     is exact so the only rounding is BF16 RNE) and runs QK^T as m16n8k16 MMAs (16 slots x
//     8 heads, FP32 accumulate);
//   - forms score = bf16(bf16(qk) / sqrt(hd)) (:160-165), masks, and updates an online
//     softmax (running max / sum per head, FP32);
//   - dequantises V into the transposed A operand and accumulates O^T[d, head] += V^T P^T
//     with P = bf16(exp(score - running max)).
// At the end of each pair the CTA merges its warps with the log-sum-exp rule. A pair that
// lies inside one CTA's range is finished there: divide by the sum, then
// bf16(bf16(o) * bf16(sigmoid(gate))) (:170). A pair cut by CTA boundaries leaves one
// partial (max, sum, out) per CTA in the workspace, and the merge kernel (launched as a
// programmatic dependent of the split kernel, so it is resident when the split kernel
// ends) combines them in CTA order.
// Deviation from the reference, inside the 1e-2 layer tolerance: the reference rounds the
// normalised probability to BF16 before PV; here the unnormalised exp(score - max) is
// rounded (normalisation happens after the FP32 sum).
#include "common.cuh"

namespace qk {
namespace {

constexpr int kAttnWarps = 8;   // warps per CTA (one CTA per SM)
constexpr int kHeads = 8;       // query heads per KV head handled by the MMA column block
constexpr int kStages = 3;      // per-warp copy ring depth
constexpr int kMinTilesPerCta = 2 * kAttnWarps;
constexpr int kMergeThreads = 256;

template <int HD>
struct Geo {
  static constexpr int kGroups = HD / 32;                 // scale groups per slot row
  static constexpr int kChunks = HD / 16;                 // 16-byte chunks per slot row
  static constexpr int kTile = 16 * HD;                   // bytes of one K (or V) code tile
  static constexpr int kScale = kGroups * 16 * 2;         // bytes of one scale tile [group][slot]
  static constexpr int kStage = 2 * kTile + 2 * kScale;   // K codes, V codes, K scales, V scales
  static constexpr int kRing = kStages * kStage;          // one warp's ring
  static constexpr int kOOff = kAttnWarps * kRing;        // float o_s[kHeads][HD]
  static constexpr int kMOff = kOOff + kHeads * HD * 4;   // float m_s[warps][kHeads], l_s[..]
  static constexpr int kHOff = kMOff + 2 * kAttnWarps * kHeads * 4;  // float head M, L
  static constexpr int kMaskOff = kHOff + 2 * kHeads * 4;            // uint32 [warps][stages]
  static constexpr int kSmem = kMaskOff + kAttnWarps * kStages * 4;
  static constexpr int kSlotFloats = 2 * kHeads + kHeads * HD;       // partial: m, l, o
};

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
  float* part;       // [2 * ctas][kSlotFloats]: slot 2c = CTA c's first pair, 2c + 1 = its last
  long long units;   // B * kv * nt tiles
  int B, S, T, hq, kv, r, nt, ctas, fast_scales;
  float div;         // f32(sqrt(hd))
};

__host__ __device__ __forceinline__ long long cta_start(long long c, long long units, int ctas) {
  return c * units / ctas;
}
// The CTA whose range holds tile u: the largest c with cta_start(c) <= u.
__device__ __forceinline__ int cta_of(long long u, long long units, int ctas) {
  return static_cast<int>(((u + 1) * ctas - 1) / units);
}

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

// 16-byte cp.async that writes zeros when `bytes` is 0 (slots past the end of the pair).
__device__ __forceinline__ void cp_async16_fill(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
               "r"(bytes)
               : "memory");
}

// Raw per-lane metadata of one tile, loaded one tile before its copies are issued so the
// loads' latency hides behind a tile of compute. Lane l (and l + 16) describe slot l.
struct Meta {
  int t;    // indices[b, s] (0 when s >= S)
  int v;    // valid[b, s], or 0
  int len;  // lengths[b], or 0
};

__device__ __forceinline__ Meta load_meta(const AttnArgs& a, long long u, int lane) {
  const int p = static_cast<int>(u / a.nt);
  const int tile = static_cast<int>(u - static_cast<long long>(p) * a.nt);
  const int b = p / a.kv;
  const int s = tile * 16 + (lane & 15);
  Meta m{0, 0, 0};
  if (s < a.S) {
    const int64_t i = static_cast<int64_t>(b) * a.S + s;
    m.t = a.indices[i];
    if (a.valid) m.v = a.valid[i];
  }
  if (!a.valid) m.len = a.lengths[b];
  return m;
}

// Issue the copies of tile u into `stage` and record its valid-slot mask.
template <int HD>
__device__ __forceinline__ void issue_tile(const AttnArgs& a, uint8_t* stage, uint32_t* mask_slot,
                                           long long u, const Meta& meta, int lane) {
  using G = Geo<HD>;
  const int p = static_cast<int>(u / a.nt);
  const int tile = static_cast<int>(u - static_cast<long long>(p) * a.nt);
  const int b = p / a.kv, h = p - b * a.kv;
  const int s = tile * 16 + (lane & 15);
  const bool in = s < a.S;
  const int t = in ? wrap_clamp(meta.t, a.T) : 0;
  const bool valid = in && (a.valid ? meta.v != 0 : s <= meta.len);
  const uint32_t vmask = __ballot_sync(0xffffffffu, valid) & 0xffffu;
  const uint32_t inmask = __ballot_sync(0xffffffffu, in) & 0xffffu;
  if (lane == 0) *mask_slot = vmask;

  const int64_t row_stride = static_cast<int64_t>(a.kv) * HD;
  const int64_t pair_off = static_cast<int64_t>(b) * a.T * row_stride + static_cast<int64_t>(h) * HD;
  const int8_t* kb = a.k_codes + pair_off;
  const int8_t* vb = a.v_codes + pair_off;
  uint8_t* ks = stage;
  uint8_t* vs = stage + G::kTile;
#pragma unroll
  for (int k = 0; k < G::kChunks / 2; ++k) {
    const int q = lane + 32 * k;
    const int row = q / G::kChunks, col = q % G::kChunks;
    const int trow = __shfl_sync(0xffffffffu, t, row);
    const uint32_t bytes = (inmask >> row) & 1u ? 16u : 0u;
    const int64_t off = static_cast<int64_t>(trow) * row_stride + col * 16;
    cp_async16_fill(ks + row * HD + ((col ^ (row & 7)) << 4), kb + off, bytes);
    cp_async16_fill(vs + row * HD + ((col ^ ((row >> 1) & 3)) << 4), vb + off, bytes);
  }

  // scales: [group][slot] bf16 tiles
  const int t0 = __shfl_sync(0xffffffffu, t, 0);
  const bool run = __ballot_sync(0xffffffffu, lane >= 16 || t == t0 + lane) == 0xffffffffu;
  const int64_t grp0 = (static_cast<int64_t>(b) * a.kv + h) * G::kGroups;  // first scale row of the pair
  uint8_t* kss = stage + 2 * G::kTile;
  uint8_t* vss = kss + G::kScale;
  if (a.fast_scales && run && inmask == 0xffffu && (t0 & 7) == 0) {
    if (lane < 4 * G::kGroups) {
      const int which = lane / (2 * G::kGroups), gi = (lane >> 1) % G::kGroups, half = lane & 1;
      const uint16_t* plane = which ? a.v_scale : a.k_scale;
      cp_async16(stage + 2 * G::kTile + which * G::kScale + gi * 32 + half * 16,
                 plane + (grp0 + gi) * a.T + t0 + 8 * half);
    }
  } else {
    const int slot = lane & 15;
#pragma unroll
    for (int m = 0; m < G::kGroups / 2; ++m) {
      const int gi = (lane >> 4) + 2 * m;
      uint16_t kv_k = 0, kv_v = 0;
      if (in) {
        kv_k = a.k_scale[(grp0 + gi) * a.T + t];
        kv_v = a.v_scale[(grp0 + gi) * a.T + t];
      }
      reinterpret_cast<uint16_t*>(kss)[gi * 16 + slot] = kv_k;
      reinterpret_cast<uint16_t*>(vss)[gi * 16 + slot] = kv_v;
    }
  }
}

template <int HD>
__global__ void __launch_bounds__(kAttnWarps * 32, 1) attn_stream_kernel(AttnArgs a) {
  using G = Geo<HD>;
  constexpr int KSTEPS = HD / 16;      // QK k-steps over d
  constexpr int KB = HD / 4;           // K bytes per lane per slot row
  constexpr int KV4 = KB / 16;         // 16-byte chunks per lane per K row
  constexpr int VB = HD / 8;           // V bytes per lane per slot row
  constexpr int VV4 = VB / 16 > 0 ? VB / 16 : 1;
  constexpr int MT = HD / 16;          // PV m-tiles over d
  constexpr int KG = KB / 32;          // scale groups per lane per K row
  static_assert(HD == 128 || HD == 256, "head_dim 128 or 256");

  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  uint8_t* ring = smem + warp * G::kRing;
  float* o_s = reinterpret_cast<float*>(smem + G::kOOff);
  float* m_s = reinterpret_cast<float*>(smem + G::kMOff);
  float* l_s = m_s + kAttnWarps * kHeads;
  float* hm_s = reinterpret_cast<float*>(smem + G::kHOff);
  float* hl_s = hm_s + kHeads;
  uint32_t* mask_s = reinterpret_cast<uint32_t*>(smem + G::kMaskOff) + warp * kStages;

  pdl_trigger();  // the merge kernel may take its place now; it waits for this grid to end

  const int cta = blockIdx.x;
  const long long u0 = cta_start(cta, a.units, a.ctas), u1 = cta_start(cta + 1, a.units, a.ctas);
  const int n_mine = u1 - u0 > warp ? static_cast<int>((u1 - u0 - warp + kAttnWarps - 1) / kAttnWarps) : 0;
  auto unit_of = [&](int j) { return u0 + warp + static_cast<long long>(kAttnWarps) * j; };

  // prologue: the first kStages - 1 tiles in flight, metadata of the next one loaded
  Meta meta{0, 0, 0};
  if (n_mine > 0) meta = load_meta(a, unit_of(0), lane);
#pragma unroll
  for (int k = 0; k < kStages - 1; ++k) {
    if (k < n_mine) {
      issue_tile<HD>(a, ring + k * G::kStage, mask_s + k, unit_of(k), meta, lane);
      if (k + 1 < n_mine) meta = load_meta(a, unit_of(k + 1), lane);
    }
    cp_async_commit();
  }

  const long long p_first = u0 / a.nt, p_last = (u1 - 1) / a.nt;
  int j = 0;
  for (long long p = p_first; p <= p_last; ++p) {
    const int b = static_cast<int>(p / a.kv), h = static_cast<int>(p - static_cast<long long>(b) * a.kv);
    // query fragments of head g: d = c*KB + 4*st .. +3 for k-step st
    uint2 qf[KSTEPS];
    {
      const bool mine = g < a.r;
      const uint16_t* qrow = a.q + (static_cast<int64_t>(b) * a.hq + h * a.r + (mine ? g : 0)) * HD + c * KB;
#pragma unroll
      for (int st = 0; st < KSTEPS; ++st)
        qf[st] = mine ? *reinterpret_cast<const uint2*>(qrow + 4 * st) : make_uint2(0u, 0u);
    }
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    float o_acc[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) o_acc[mt][0] = o_acc[mt][1] = o_acc[mt][2] = o_acc[mt][3] = 0.f;

    for (; j < n_mine && unit_of(j) / a.nt == p; ++j) {
      const int nxt = j + kStages - 1;
      if (nxt < n_mine) {
        issue_tile<HD>(a, ring + (nxt % kStages) * G::kStage, mask_s + nxt % kStages, unit_of(nxt), meta, lane);
        if (nxt + 1 < n_mine) meta = load_meta(a, unit_of(nxt + 1), lane);
      }
      cp_async_commit();
      cp_async_wait<kStages - 1>();
      __syncwarp();

      const int sidx = j % kStages;
      const uint8_t* stage = ring + sidx * G::kStage;
      const uint8_t* kt = stage;
      const uint8_t* vt = stage + G::kTile;
      const uint16_t* kss = reinterpret_cast<const uint16_t*>(stage + 2 * G::kTile);
      const uint16_t* vss = kss + G::kScale / 2;
      const uint32_t vmask = mask_s[sidx];

      // ---- QK^T: rows g, g+8 of the tile; lane quarter c holds d in [c*KB, (c+1)*KB) ----
      float sacc[4] = {0.f, 0.f, 0.f, 0.f};
      {
        uint4 kw[2][KV4];
        float ks[2][KG];
#pragma unroll
        for (int rh = 0; rh < 2; ++rh) {
          const int row = g + 8 * rh;
#pragma unroll
          for (int i = 0; i < KV4; ++i)
            kw[rh][i] = lds_v4(kt + row * HD + (((c * KV4 + i) ^ (row & 7)) << 4));
#pragma unroll
          for (int i = 0; i < KG; ++i) ks[rh][i] = bf16_to_f32(kss[(c * KG + i) * 16 + row]);
        }
#pragma unroll
        for (int st = 0; st < KSTEPS; ++st) {
          const int gi = (st * 4) / 32;
          uint32_t af[4];
#pragma unroll
          for (int rh = 0; rh < 2; ++rh) {
            const uint32_t wx = word(kw[rh][st / 4], st % 4) ^ 0x80808080u;
            const float sc = ks[rh][gi];
            af[rh] = dq_pair(s8_at<0>(wx), s8_at<1>(wx), sc, sc);
            af[2 + rh] = dq_pair(s8_at<2>(wx), s8_at<3>(wx), sc, sc);
          }
          mma_bf16(sacc, af, qf[st].x, qf[st].y);
        }
      }
      // ---- V fragments (slots 2c, 2c+1, 2c+8, 2c+9; d in [g*VB, (g+1)*VB)) ----
      uint4 vw[4][VV4];
      float vsc[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = 2 * c + (i & 1) + 8 * (i >> 1);
#pragma unroll
        for (int jj = 0; jj < VV4; ++jj)
          vw[i][jj] = lds_v4(vt + row * HD + (((g * VV4 + jj) ^ ((row >> 1) & 3)) << 4));
        vsc[i] = bf16_to_f32(vss[((g * VB) / 32) * 16 + row]);
      }
      // ---- scores, online softmax (heads 2c, 2c+1; slots g, g+8) ----
      float pr[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const bool ok = (vmask >> (g + 8 * (i >> 1))) & 1u;
        const float raw = bf16_round(sacc[i]);
        const float sc = HD == 256 ? __fmul_rn(raw, 0.0625f) : __fdiv_rn(raw, a.div);
        pr[i] = ok ? bf16_round(sc) : -INFINITY;
      }
      float alpha[2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float mt = fmaxf(pr[hh], pr[2 + hh]);
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
        const float m_new = fmaxf(m_run[hh], mt);
        if (m_new == -INFINITY) {
          alpha[hh] = 1.f;
          pr[hh] = pr[2 + hh] = 0.f;
        } else {
          alpha[hh] = expf(m_run[hh] - m_new);
          pr[hh] = expf(pr[hh] - m_new);
          pr[2 + hh] = expf(pr[2 + hh] - m_new);
        }
        m_run[hh] = m_new;
      }
      // P in BF16 (the MMA operand); the running sum uses the same rounded values.
      const uint32_t P0 = pack_bf16x2(pr[0], pr[1]), P1 = pack_bf16x2(pr[2], pr[3]);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float ps = __fadd_rn(bf16_to_f32(static_cast<uint16_t>(P0 >> (16 * hh))),
                             bf16_to_f32(static_cast<uint16_t>(P1 >> (16 * hh))));
        ps += __shfl_xor_sync(0xffffffffu, ps, 4);
        ps += __shfl_xor_sync(0xffffffffu, ps, 8);
        ps += __shfl_xor_sync(0xffffffffu, ps, 16);
        l_run[hh] = __fadd_rn(__fmul_rn(l_run[hh], alpha[hh]), ps);
      }
      if (!__all_sync(0xffffffffu, alpha[0] == 1.f && alpha[1] == 1.f)) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          o_acc[mt][0] *= alpha[0];
          o_acc[mt][1] *= alpha[1];
          o_acc[mt][2] *= alpha[0];
          o_acc[mt][3] *= alpha[1];
        }
      }
      const uint32_t b0 = movmatrix_trans(P0), b1 = movmatrix_trans(P1);
      // ---- PV: O^T[d, head] += V^T[d, slot] P^T[slot, head]; d0 = g*VB + 2 mt, d1 = d0 + 1 ----
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int byte = 2 * mt;  // inside this lane's VB bytes
        const int wi = (byte / 4) % 4, vi = byte / 16;
        uint32_t af[4];
        uint32_t wx[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) wx[i] = word(vw[i][vi], wi) ^ 0x80808080u;
        if ((byte & 3) == 0) {
          af[0] = dq_pair(s8_at<0>(wx[0]), s8_at<0>(wx[1]), vsc[0], vsc[1]);
          af[1] = dq_pair(s8_at<1>(wx[0]), s8_at<1>(wx[1]), vsc[0], vsc[1]);
          af[2] = dq_pair(s8_at<0>(wx[2]), s8_at<0>(wx[3]), vsc[2], vsc[3]);
          af[3] = dq_pair(s8_at<1>(wx[2]), s8_at<1>(wx[3]), vsc[2], vsc[3]);
        } else {
          af[0] = dq_pair(s8_at<2>(wx[0]), s8_at<2>(wx[1]), vsc[0], vsc[1]);
          af[1] = dq_pair(s8_at<3>(wx[0]), s8_at<3>(wx[1]), vsc[0], vsc[1]);
          af[2] = dq_pair(s8_at<2>(wx[2]), s8_at<2>(wx[3]), vsc[2], vsc[3]);
          af[3] = dq_pair(s8_at<3>(wx[2]), s8_at<3>(wx[3]), vsc[2], vsc[3]);
        }
        mma_bf16(o_acc[mt], af, b0, b1);
      }
      __syncwarp();  // every lane is done with this stage before it is refilled
    }

    // ---- end of pair p: merge the warps (log-sum-exp, warp order), finish or leave a partial ----
    if (g == 0) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        m_s[warp * kHeads + 2 * c + hh] = m_run[hh];
        l_s[warp * kHeads + 2 * c + hh] = l_run[hh];
      }
    }
    __syncthreads();
    float f[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      float M = -INFINITY;
      for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, m_s[w * kHeads + 2 * c + hh]);
      f[hh] = m_run[hh] == -INFINITY ? 0.f : expf(m_run[hh] - M);
    }
    if (threadIdx.x < kHeads) {
      const int r = threadIdx.x;
      float M = -INFINITY;
      for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, m_s[w * kHeads + r]);
      float L = 0.f;
      for (int w = 0; w < kAttnWarps; ++w) {
        const float mw = m_s[w * kHeads + r];
        L = __fadd_rn(L, __fmul_rn(l_s[w * kHeads + r], mw == -INFINITY ? 0.f : expf(mw - M)));
      }
      hm_s[r] = M;
      hl_s[r] = L;
    }
    for (int w = 0; w < kAttnWarps; ++w) {
      if (warp == w) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          const int d0 = g * VB + 2 * mt;
          float* r0 = o_s + (2 * c) * HD + d0;
          float* r1 = o_s + (2 * c + 1) * HD + d0;
          const float x0 = __fmul_rn(o_acc[mt][0], f[0]), x1 = __fmul_rn(o_acc[mt][1], f[1]);
          const float x2 = __fmul_rn(o_acc[mt][2], f[0]), x3 = __fmul_rn(o_acc[mt][3], f[1]);
          if (w == 0) {
            r0[0] = x0; r1[0] = x1; r0[1] = x2; r1[1] = x3;
          } else {
            r0[0] = __fadd_rn(r0[0], x0); r1[0] = __fadd_rn(r1[0], x1);
            r0[1] = __fadd_rn(r0[1], x2); r1[1] = __fadd_rn(r1[1], x3);
          }
        }
      }
      __syncthreads();
    }
    const bool whole = p * a.nt >= u0 && (p + 1) * a.nt <= u1;
    if (whole) {
      for (int i = threadIdx.x; i < a.r * HD; i += blockDim.x) {
        const int r = i / HD;
        const int64_t oi = (static_cast<int64_t>(b) * a.hq + h * a.r) * HD + i;
        a.out[oi] = bf16_bits_rne(output_value(__fdiv_rn(o_s[i], hl_s[r]), a.gate, oi));
      }
    } else {
      float* slot = a.part + static_cast<int64_t>(2 * cta + (p == p_first ? 0 : 1)) * G::kSlotFloats;
      for (int i = threadIdx.x; i < a.r * HD; i += blockDim.x) slot[2 * kHeads + i] = o_s[i];
      if (threadIdx.x < kHeads) {
        slot[threadIdx.x] = hm_s[threadIdx.x];
        slot[kHeads + threadIdx.x] = hl_s[threadIdx.x];
      }
    }
    __syncthreads();  // o_s, m_s and the head statistics are reused by the next pair
  }
}

// Combine the partials of pairs cut by CTA boundaries: block (pair, head, d slice);
// thread = 8 consecutive d of one CTA subset; subsets are merged in CTA order.
template <int HD>
__global__ void __launch_bounds__(kMergeThreads) attn_merge_kernel(AttnArgs a, int dslices) {
  using G = Geo<HD>;
  __shared__ float sm_m[kMergeThreads], sm_l[kMergeThreads];
  __shared__ __align__(16) float sm_o[kMergeThreads * 8];
  pdl_wait();
  const int p = blockIdx.x, r = blockIdx.y;
  if (r >= a.r) return;
  const long long lo = static_cast<long long>(p) * a.nt;
  const int c0 = cta_of(lo, a.units, a.ctas), c1 = cta_of(lo + a.nt - 1, a.units, a.ctas);
  if (c0 == c1) return;  // finished by the split kernel
  const int n = c1 - c0 + 1;
  const int width = HD / dslices, dthreads = width / 8, groups = kMergeThreads / dthreads;
  const int tid = threadIdx.x, dt = tid % dthreads, grp = tid / dthreads;
  const int d0 = blockIdx.z * width + dt * 8;
  float m = -INFINITY, l = 0.f, o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = 0.f;
  for (int k0 = grp; k0 < n; k0 += 4 * groups) {
    float pm[4], pl[4];
    float4 x[4][2];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int k = k0 + u * groups;
      pm[u] = -INFINITY;
      pl[u] = 0.f;
      x[u][0] = x[u][1] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (k < n) {
        const int cc = c0 + k;
        const int first = static_cast<int>(cta_start(cc, a.units, a.ctas) / a.nt);
        const float* s = a.part + static_cast<int64_t>(2 * cc + (first == p ? 0 : 1)) * G::kSlotFloats;
        pm[u] = s[r];
        pl[u] = s[kHeads + r];
        const float4* so = reinterpret_cast<const float4*>(s + 2 * kHeads + r * HD + d0);
        x[u][0] = so[0];
        x[u][1] = so[1];
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float M = fmaxf(m, pm[u]);
      if (M == -INFINITY) continue;
      const float fo = m == -INFINITY ? 0.f : expf(m - M);
      const float fn = pm[u] == -INFINITY ? 0.f : expf(pm[u] - M);
      l = __fadd_rn(__fmul_rn(l, fo), __fmul_rn(pl[u], fn));
      const float xs[8] = {x[u][0].x, x[u][0].y, x[u][0].z, x[u][0].w,
                           x[u][1].x, x[u][1].y, x[u][1].z, x[u][1].w};
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = __fadd_rn(__fmul_rn(o[i], fo), __fmul_rn(xs[i], fn));
      m = M;
    }
  }
  sm_m[tid] = m;
  sm_l[tid] = l;
#pragma unroll
  for (int i = 0; i < 8; ++i) sm_o[tid * 8 + i] = o[i];
  __syncthreads();
  if (grp != 0) return;
  float M = -INFINITY;
  for (int k = 0; k < groups; ++k) M = fmaxf(M, sm_m[k * dthreads + dt]);
  float L = 0.f, O[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) O[i] = 0.f;
  for (int k = 0; k < groups; ++k) {
    const int t = k * dthreads + dt;
    const float fk = sm_m[t] == -INFINITY ? 0.f : expf(sm_m[t] - M);
    L = __fadd_rn(L, __fmul_rn(sm_l[t], fk));
#pragma unroll
    for (int i = 0; i < 8; ++i) O[i] = __fadd_rn(O[i], __fmul_rn(sm_o[t * 8 + i], fk));
  }
  const int b = p / a.kv, h = p - b * a.kv;
  const int64_t oi = ((static_cast<int64_t>(b) * a.hq + h * a.r + r) * HD) + d0;
#pragma unroll
  for (int i = 0; i < 8; ++i) a.out[oi + i] = bf16_bits_rne(output_value(__fdiv_rn(O[i], L), a.gate, oi + i));
}

// CTAs of the split kernel for B pairs-of-tiles `units` (one per SM, at least two tiles
// per warp).
int choose_ctas(long long units) {
  long long c = units / kMinTilesPerCta;
  const long long cap = sm_count();
  if (c > cap) c = cap;
  return c < 1 ? 1 : static_cast<int>(c);
}

size_t slot_bytes(int hd) { return static_cast<size_t>(2 * kHeads + kHeads * hd) * sizeof(float); }

}  // namespace
}  // namespace qk

using namespace qk;

extern "C" {

size_t qk_kv_q8_attention_workspace_bytes(int B, int S, int hq, int kv_heads, int head_dim) {
  if (B <= 0 || S <= 0 || kv_heads <= 0 || head_dim <= 0) return 0;
  (void)hq;
  const long long units = static_cast<long long>(B) * kv_heads * ((S + 15) / 16);
  const int ctas = choose_ctas(units);
  return ctas > 1 ? 2 * static_cast<size_t>(ctas) * slot_bytes(head_dim) : 0;
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
  QK_REQUIRE((reinterpret_cast<uintptr_t>(k_codes) & 15) == 0 && (reinterpret_cast<uintptr_t>(v_codes) & 15) == 0,
             "K/V code planes must be 16-byte aligned");
  QK_REQUIRE((reinterpret_cast<uintptr_t>(q) & 7) == 0, "q must be 8-byte aligned");
  AttnArgs a{};
  a.q = q; a.k_codes = k_codes; a.v_codes = v_codes; a.k_scale = k_scale; a.v_scale = v_scale;
  a.indices = indices; a.valid = valid; a.lengths = valid ? nullptr : lengths; a.gate = gate; a.out = out;
  a.B = B; a.S = S; a.T = T; a.hq = hq; a.kv = kv_heads; a.r = hq / kv_heads;
  a.nt = (S + 15) / 16;
  a.units = static_cast<long long>(B) * kv_heads * a.nt;
  a.ctas = choose_ctas(a.units);
  a.fast_scales = (T % 8) == 0 && (reinterpret_cast<uintptr_t>(k_scale) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(v_scale) & 15) == 0;
  a.div = sqrtf(static_cast<float>(head_dim));
  if (a.ctas > 1) {
    const size_t need = 2 * static_cast<size_t>(a.ctas) * slot_bytes(head_dim);
    if (!workspace || workspace_bytes < need)
      return set_error(QK_ERR_WORKSPACE, "attention workspace needs %zu bytes, got %zu", need, workspace_bytes);
    QK_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 15) == 0, "workspace must be 16-byte aligned");
    a.part = static_cast<float*>(workspace);
  }
  cudaStream_t st = as_stream(stream);
  const int smem = head_dim == 256 ? Geo<256>::kSmem : Geo<128>::kSmem;
  const void* kern = head_dim == 256 ? reinterpret_cast<const void*>(attn_stream_kernel<256>)
                                     : reinterpret_cast<const void*>(attn_stream_kernel<128>);
  if (int rc = allow_smem(kern, smem)) return rc;
  if (head_dim == 256) attn_stream_kernel<256><<<a.ctas, kAttnWarps * 32, smem, st>>>(a);
  else attn_stream_kernel<128><<<a.ctas, kAttnWarps * 32, smem, st>>>(a);
  QK_LAUNCHED("attn_stream_kernel");
  if (a.ctas > 1) {
    // partials per cut pair: about nt / (units / ctas) + 1; wider merges split d further
    const long long per = a.units / a.ctas;
    const long long n = (a.nt + per - 1) / per + 1;
    const int dslices = n > 32 ? 4 : (n > 8 ? 2 : 1);
    const dim3 grid(static_cast<unsigned>(static_cast<long long>(B) * kv_heads), kHeads, dslices);
    const cudaError_t e = head_dim == 256
                              ? launch_dependent(attn_merge_kernel<256>, grid, dim3(kMergeThreads), 0, st, a, dslices)
                              : launch_dependent(attn_merge_kernel<128>, grid, dim3(kMergeThreads), 0, st, a, dslices);
    if (e != cudaSuccess) return cuda_error(e, "attn_merge_kernel");
    QK_LAUNCHED("attn_merge_kernel");
  }
  return QK_OK;
}

}  // extern "C"
