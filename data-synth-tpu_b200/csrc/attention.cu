// Split-KV decode attention over the Q8 KV cache (reference cache layout).
//
// Replaces the attention core of qwen38_tpu/attention_cache.py:152-170 (step, after the
// cache write): per batch row b and KV head h (a "pair"), the r = hq / kv query heads of
// the group attend over S gathered slots.
//
// Work split (stream-K): a pair's slots form tiles of 16. The B * kv * ceil(S/16) tiles of
// all pairs are ordered (b, tile, h) when kv divides the CTA's 8 warps (else (b, h, tile))
// and cut into one contiguous, equal range per CTA, one CTA per SM, so the grid is
// balanced whatever B and S are. The 8 warps take the tiles of their CTA's range round
// robin; with the (b, tile, h) order each warp keeps one KV head, and the warps of the
// different heads fetch the same cache rows at the same moment (a row holds all heads).
// Per tile, a warp
//   - has the tile's cache times (indices) copied by cp.async into a small ring several
//     tiles ahead, so address generation never waits on a load;
//   - copies its K and V codes into a two-stage ring completing on one mbarrier per stage:
//     when the 16 times are consecutive, as 2D tensor copies (TMA) of 16 rows x 128 bytes
//     with the 128-byte shared-memory swizzle (two boxes per plane at head_dim 256), and
//     the BF16 scale tiles as 2D tensor copies when the first time is 8-aligned; else one
//     bulk copy per 128-byte row piece and one load per scale;
//   - loads the tile's K and V fragments into registers and refills the stage with the
//     tile two ahead, so two tiles stay in flight while it computes;
//   - dequantises K in registers to bf16(code * scale) (read_quantized, :71-81; the
//     product is exact so the only rounding is BF16 RNE) for QK^T as m16n8k16 MMAs (16
//     slots x 8 heads, FP32 accumulate); score = bf16(bf16(qk) / sqrt(hd)) (:160-165),
//     masked, feeds an online softmax (running max / sum per head, FP32); V is dequantised
//     into the transposed A operand for O^T[d, head] += V^T P^T with
//     P = bf16(exp(score - running max)).
// At the end of each batch row (or pair) the CTA merges the warps of each KV head with the
// log-sum-exp rule in warp order. A pair that lies inside one CTA's range is finished
// there: divide by the sum, then bf16(bf16(o) * bf16(sigmoid(gate))) (:170). A pair cut by
// CTA boundaries leaves one partial (max, sum, out) per CTA in the workspace, and the merge
// kernel (launched as a programmatic dependent of the split kernel, so it is resident when
// the split kernel ends) combines them in CTA order.
// Deviation from the reference, inside the 1e-2 layer tolerance: the reference rounds the
// normalised probability to BF16 before PV; here the unnormalised exp(score - max) is
// rounded (normalisation happens after the FP32 sum).
#include <cuda.h>  // CUtensorMap and its enums; the encoder is looked up at run time

#include "common.cuh"

namespace qk {
namespace {

constexpr int kAttnWarps = 8;   // warps per CTA (one CTA per SM)
constexpr int kHeads = 8;       // query heads per KV head handled by the MMA column block
constexpr int kStages = 2;      // per-warp copy ring depth (the stage is refilled on read)
constexpr int kMetaLead = 3;    // tiles between a tile's index copy and its code copies
constexpr int kMetaSlots = 6;   // index ring slots per warp (> kStages + kMetaLead)
constexpr int kMinTilesPerCta = 2 * kAttnWarps;
constexpr int kMergeThreads = 256;
constexpr int kBox = 128;       // bytes of one tensor-copy box row (the 128-byte swizzle span)

template <int HD>
struct Geo {
  static constexpr int kGroups = HD / 32;                 // scale groups per slot row
  static constexpr int kBoxes = HD / kBox;                // boxes per 16-row code tile
  static constexpr int kTile = 16 * HD;                   // one plane's codes: [box][16 rows][128 B]
  static constexpr int kScale = kGroups * 16 * 2;         // one scale tile [group][slot] BF16
  static constexpr int kStage = (2 * kTile + 2 * kScale + 1023) / 1024 * 1024;  // swizzle atoms stay aligned
  static constexpr int kRing = kStages * kStage;
  static constexpr int kOP = HD == 256 ? 274 : 146;       // o_buf row (floats): conflict-free writes
  static constexpr int kMeta = 16 * 4 + 16;               // index ring slot: 16 times, 16 valid flags
  static constexpr int kOOff = kAttnWarps * kRing;        // float o_buf[warps][kHeads][kOP]
  static constexpr int kMOff = kOOff + kAttnWarps * kHeads * kOP * 4;  // float m_s, l_s, f_s [warps][kHeads]
  static constexpr int kIdxOff = kMOff + 3 * kAttnWarps * kHeads * 4;  // [warps][kMetaSlots][kMeta]
  static constexpr int kFlagOff = kIdxOff + kAttnWarps * kMetaSlots * kMeta;  // uint32 [warps][stages]
  static constexpr int kBarOff = kFlagOff + kAttnWarps * kStages * 4;         // uint64 [warps][stages]
  static constexpr int kQOff = kBarOff + kAttnWarps * kStages * 8;  // bf16 q_s[heads][kHeads][HD], then L
  static constexpr int kSlotFloats = 2 * kHeads + kHeads * HD;      // partial: m, l, o
  // dynamic shared memory for `nh` KV heads per segment (plus slack to align to 1024)
  static constexpr size_t smem(int nh) { return kQOff + static_cast<size_t>(nh) * kHeads * (HD * 2 + 4) + 1024; }
  // byte of (row, 16-byte chunk) in a plane tile; swizzled when written by a tensor copy
  __device__ static int at(int row, int chunk, bool swz) {
    return (chunk >> 3) * (16 * kBox) + row * kBox + (((chunk & 7) ^ (swz ? (row & 7) : 0)) << 4);
  }
  // o_buf column of output dim d (a gap every 32 floats)
  __device__ static int oc(int d) { return d + d / 32; }
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
  float* part;       // [2 * ctas][kv][kSlotFloats]: CTA c's first (2c) and last (2c + 1) segment
  long long units;   // B * kv * nt tiles
  int B, S, T, hq, kv, r, nt, ctas;
  int hfast;         // tiles ordered (b, tile, h); else (b, h, tile)
  int seg_units;     // tiles per segment: nt * kv (a batch row) or nt (a pair)
  int tma_codes;     // code tiles of consecutive times use the tensor maps
  int tma_scales;    // ... and the scale tiles too (T % 8 == 0, aligned planes)
  int idx16;         // indices rows start 16-byte aligned (S % 4 == 0): 4-index copies
  int flag16;        // valid rows start 16-byte aligned (S % 16 == 0): 16-flag copies
  float div;         // f32(sqrt(hd))
};

// Set when a bounded wait of the split kernel gives up; read and cleared by
// qk_kv_q8_attention_check.
__device__ int g_attn_status;

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

// 2D tensor copy (no multicast) of one box into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// cp.async of 4 bytes (L1-allocating form; the 16-byte form is cp_async16).
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}

// A warp's position in its tile sequence, advanced by kAttnWarps tiles without divisions.
struct Cursor {
  int b, h, tile;
  __device__ void init(long long u, const AttnArgs& a) {
    const long long per_b = static_cast<long long>(a.nt) * a.kv;
    b = static_cast<int>(u / per_b);
    const int rem = static_cast<int>(u - b * per_b);
    if (a.hfast) {
      tile = rem / a.kv;
      h = rem - tile * a.kv;
    } else {
      h = rem / a.nt;
      tile = rem - h * a.nt;
    }
  }
  __device__ void advance(const AttnArgs& a) {
    if (a.hfast) {  // kv divides kAttnWarps: the head stays
      tile += kAttnWarps / a.kv;
      while (tile >= a.nt) {
        tile -= a.nt;
        ++b;
      }
    } else {
      tile += kAttnWarps;
      while (tile >= a.nt) {
        tile -= a.nt;
        if (++h == a.kv) {
          h = 0;
          ++b;
        }
      }
    }
  }
  __device__ int seg(const AttnArgs& a) const { return a.hfast ? b : b * a.kv + h; }
};

// Copy the cache times (and valid flags) of the tile at `at` into index ring slot `slot`.
// Times of slots past S are not read; their entries are never used.
__device__ __forceinline__ void copy_meta(const AttnArgs& a, uint8_t* slot, const Cursor& at, int lane) {
  const int s0 = at.tile * 16;
  const int64_t row = static_cast<int64_t>(at.b) * a.S + s0;
  const bool full = s0 + 16 <= a.S;
  if (a.idx16 && full) {
    if (lane < 4) cp_async16(slot + 16 * lane, a.indices + row + 4 * lane);
  } else if (lane < 16 && s0 + lane < a.S) {
    cp_async4(slot + 4 * lane, a.indices + row + lane);
  }
  if (a.valid && a.flag16 && full && lane == 16) cp_async16(slot + 64, a.valid + row);
}

// Issue the code and scale copies of the tile at `at` into `stage`, completing on `bar`,
// and record in *flag whether the code tiles are swizzled (tensor copies).
template <int HD>
__device__ __forceinline__ void issue_tile(const AttnArgs& a, const CUtensorMap* tm_k, const CUtensorMap* tm_v,
                                           const CUtensorMap* tm_ks, const CUtensorMap* tm_vs, uint8_t* stage,
                                           uint64_t* bar, uint32_t* flag, const int32_t* times, const Cursor& at,
                                           int lane, uint64_t pol) {
  using G = Geo<HD>;
  const int slot = lane & 15;
  const bool in = at.tile * 16 + slot < a.S;
  const int t = in ? wrap_clamp(times[slot], a.T) : 0;
  const uint32_t inmask = __ballot_sync(0xffffffffu, in) & 0xffffu;
  const int t0 = __shfl_sync(0xffffffffu, t, 0);
  const bool run = __ballot_sync(0xffffffffu, lane >= 16 || t == t0 + lane) == 0xffffffffu;
  const bool tma = a.tma_codes && run && inmask == 0xffffu;  // times t0 .. t0+15, all < T
  const bool tma_s = tma && a.tma_scales && (t0 & 7) == 0;
  const uint32_t bytes = (tma ? 2u * G::kTile : __popc(inmask) * 2u * HD) + (tma_s ? 2u * G::kScale : 0u);
  if (lane == 0) {
    *flag = tma ? 1u : 0u;
    mbar_expect_tx(bar, bytes);
  }
  __syncwarp();

  bool generic = false;
  if (tma) {
    if (lane < 2 * G::kBoxes) {
      const int plane = lane / G::kBoxes, e = lane % G::kBoxes;
      tma_load_2d(stage + plane * G::kTile + e * 16 * kBox, plane ? tm_v : tm_k, at.h * HD + e * kBox,
                  at.b * a.T + t0, bar, pol);
    }
  } else {
    // lane l: plane l >> 4 (K, V), row l & 15, as kBoxes linear 128-byte pieces
    const int plane = lane >> 4;
    uint8_t* dst = stage + plane * G::kTile + slot * kBox;
    if (in) {
      const int64_t off = (static_cast<int64_t>(at.b) * a.T + t) * a.kv * HD + static_cast<int64_t>(at.h) * HD;
      const int8_t* src = (plane ? a.v_codes : a.k_codes) + off;
#pragma unroll
      for (int e = 0; e < G::kBoxes; ++e) bulk_g2s_hint(dst + e * 16 * kBox, src + e * kBox, kBox, bar, pol);
    } else {  // past the end of the pair: zero codes (and zero scales below)
#pragma unroll
      for (int e = 0; e < G::kBoxes; ++e)
#pragma unroll
        for (int i = 0; i < kBox / 16; ++i)
          reinterpret_cast<uint4*>(dst + e * 16 * kBox)[i] = make_uint4(0u, 0u, 0u, 0u);
      generic = true;
    }
  }
  uint8_t* kss = stage + 2 * G::kTile;
  const int grp0 = (at.b * a.kv + at.h) * G::kGroups;  // first scale row of the pair
  if (tma_s) {
    if (lane < 2) tma_load_2d(kss + lane * G::kScale, lane ? tm_vs : tm_ks, t0, grp0, bar, pol);
  } else {
#pragma unroll
    for (int m = 0; m < G::kGroups / 2; ++m) {
      const int gi = (lane >> 4) + 2 * m;
      uint16_t sk = 0, sv = 0;
      if (in) {
        sk = a.k_scale[static_cast<int64_t>(grp0 + gi) * a.T + t];
        sv = a.v_scale[static_cast<int64_t>(grp0 + gi) * a.T + t];
      }
      reinterpret_cast<uint16_t*>(kss)[gi * 16 + slot] = sk;
      reinterpret_cast<uint16_t*>(kss + G::kScale)[gi * 16 + slot] = sv;
    }
    generic = true;
  }
  // generic stores into the stage come before any later asynchronous copy into it
  if (__any_sync(0xffffffffu, generic)) fence_proxy_async_smem();
}

template <int HD>
__global__ void __launch_bounds__(kAttnWarps * 32, 1)
    attn_stream_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                       const __grid_constant__ CUtensorMap tm_ks, const __grid_constant__ CUtensorMap tm_vs,
                       AttnArgs a) {
  using G = Geo<HD>;
  constexpr int KSTEPS = HD / 16;      // QK k-steps over d
  constexpr int KB = HD / 4;           // K bytes per lane per slot row
  constexpr int KV4 = KB / 16;         // 16-byte chunks per lane per K row
  constexpr int VB = HD / 8;           // V bytes per lane per slot row (chunks g, g + 8)
  constexpr int VV4 = VB / 16;
  constexpr int MT = HD / 16;          // PV m-tiles over d
  constexpr int KG = KB / 32;          // scale groups per lane per K row
  static_assert(HD == 128 || HD == 256, "head_dim 128 or 256");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int tid = threadIdx.x;
  uint8_t* ring = smem + warp * G::kRing;
  float* o_buf = reinterpret_cast<float*>(smem + G::kOOff);
  float* m_s = reinterpret_cast<float*>(smem + G::kMOff);
  float* l_s = m_s + kAttnWarps * kHeads;
  float* f_s = l_s + kAttnWarps * kHeads;
  uint8_t* meta = smem + G::kIdxOff + warp * kMetaSlots * G::kMeta;
  uint32_t* flags = reinterpret_cast<uint32_t*>(smem + G::kFlagOff) + warp * kStages;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::kBarOff) + warp * kStages;
  uint16_t* q_s = reinterpret_cast<uint16_t*>(smem + G::kQOff);
  const int nh_max = a.hfast ? a.kv : 1;
  float* hl_s = reinterpret_cast<float*>(smem + G::kQOff + nh_max * kHeads * HD * 2);  // [nh][kHeads]

  if (lane == 0)
    for (int i = 0; i < kStages; ++i) mbar_init(bars + i, 1);
  fence_mbar_init();
  __syncthreads();
  pdl_trigger();  // the merge kernel may take its place now; it waits for this grid to end

  const int cta = blockIdx.x;
  const long long u0 = cta_start(cta, a.units, a.ctas), u1 = cta_start(cta + 1, a.units, a.ctas);
  const int n_mine = u1 - u0 > warp ? static_cast<int>((u1 - u0 - warp + kAttnWarps - 1) / kAttnWarps) : 0;
  const uint64_t pol = l2_evict_first_policy();
  // hfast: warp w keeps head (u0 + w) % kv; heads_of[h] = bit mask of those warps
  const int h0 = a.hfast ? static_cast<int>(u0 % a.kv) : 0;
  const int warp_h = a.hfast ? (h0 + warp) % a.kv : 0;

  // cursors over this warp's tiles: `cons` computed, `iss` next code copy, `mc` next index copy
  Cursor cons, iss, mc;
  cons.init(u0 + warp, a);
  iss = cons;
  mc = cons;
  // prologue: index copies of the first kStages + kMetaLead tiles (one group each), then
  // the code copies of the first kStages tiles
  int metas = 0;
  for (; metas < kStages + kMetaLead; ++metas) {
    if (metas < n_mine) {
      copy_meta(a, meta + (metas % kMetaSlots) * G::kMeta, mc, lane);
      mc.advance(a);
    }
    cp_async_commit();
  }
  cp_async_wait<0>();
  __syncwarp();
  int issued = 0;
  for (; issued < kStages && issued < n_mine; ++issued) {
    issue_tile<HD>(a, &tm_k, &tm_v, &tm_ks, &tm_vs, ring + issued * G::kStage, bars + issued, flags + issued,
                   reinterpret_cast<const int32_t*>(meta + (issued % kMetaSlots) * G::kMeta), iss, lane, pol);
    iss.advance(a);
  }

  bool ok = true;
  int drain_from = 0;
  const int s_first = static_cast<int>(u0 / a.seg_units), s_last = static_cast<int>((u1 - 1) / a.seg_units);
  int j = 0;
  for (int sg = s_first; sg <= s_last; ++sg) {
    const int b = a.hfast ? sg : sg / a.kv;
    const int h_lo = a.hfast ? 0 : sg - b * a.kv, nh = a.hfast ? a.kv : 1;
    // q of the segment's heads: q_s[hl][r][d], zero rows for r >= a.r
    for (int i = tid; i < nh * kHeads * HD; i += blockDim.x) {
      const int hl = i / (kHeads * HD), r = (i / HD) % kHeads, d = i % HD;
      q_s[i] = r < a.r ? a.q[(static_cast<int64_t>(b) * a.hq + (h_lo + hl) * a.r + r) * HD + d] : 0;
    }
    const int len = a.valid ? 0 : a.lengths[b];
    __syncthreads();
    const int hw = a.hfast ? warp_h : 0;  // this warp's head, relative to h_lo
    const uint16_t* qh = q_s + hw * kHeads * HD;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    float o_acc[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) o_acc[mt][0] = o_acc[mt][1] = o_acc[mt][2] = o_acc[mt][3] = 0.f;

    for (; j < n_mine && cons.seg(a) == sg; ++j, cons.advance(a)) {
      const int sidx = j % kStages;
      uint8_t* stage = ring + sidx * G::kStage;
      const bool got = ok && mbar_wait_bounded(bars + sidx, (j / kStages) & 1);
      if (!__all_sync(0xffffffffu, got)) {  // a wait gave up: record it, stop issuing and computing
        if (ok) {
          if (lane == 0) atomicExch(&g_attn_status, QK_ERR_TIMEOUT);
          drain_from = j;
        }
        ok = false;
        continue;
      }
      // ---- fragments of this tile into registers; the stage is then refilled ----
      uint4 kw[2][KV4];
      float ks[2][KG];
      uint4 vw[4][VV4];
      float vsc[VV4][4];  // V scale of chunk jj (d in [128 jj + 16 g, +16): group g / 2 + 4 jj)
      {
        const bool swz = flags[sidx] != 0;
        const uint8_t* kt = stage;
        const uint8_t* vt = stage + G::kTile;
        const uint16_t* kss = reinterpret_cast<const uint16_t*>(stage + 2 * G::kTile);
        const uint16_t* vss = kss + G::kScale / 2;
#pragma unroll
        for (int rh = 0; rh < 2; ++rh) {
          const int row = g + 8 * rh;
#pragma unroll
          for (int i = 0; i < KV4; ++i) kw[rh][i] = lds_v4(kt + G::at(row, c * KV4 + i, swz));
#pragma unroll
          for (int i = 0; i < KG; ++i) ks[rh][i] = bf16_to_f32(kss[(c * KG + i) * 16 + row]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = 2 * c + (i & 1) + 8 * (i >> 1);
#pragma unroll
          for (int jj = 0; jj < VV4; ++jj) {
            vw[i][jj] = lds_v4(vt + G::at(row, g + 8 * jj, swz));
            vsc[jj][i] = bf16_to_f32(vss[(g / 2 + 4 * jj) * 16 + row]);
          }
        }
      }
      // valid slots g and g + 8 of this tile
      bool okv[2];
      {
        const uint8_t* mslot = meta + (j % kMetaSlots) * G::kMeta;
#pragma unroll
        for (int rh = 0; rh < 2; ++rh) {
          const int s = cons.tile * 16 + g + 8 * rh;
          bool v = s < a.S;
          if (v) {
            if (!a.valid) v = s <= len;
            else if (a.flag16 && cons.tile * 16 + 16 <= a.S) v = mslot[64 + g + 8 * rh] != 0;
            else v = a.valid[static_cast<int64_t>(b) * a.S + s] != 0;
          }
          okv[rh] = v;
        }
      }
      __syncwarp();  // every lane has its fragments and flags: stage and index slot may be refilled
      if (issued < n_mine) {
        cp_async_wait<kMetaLead - 1>();  // the index copy of tile `issued`
        __syncwarp();
        issue_tile<HD>(a, &tm_k, &tm_v, &tm_ks, &tm_vs, stage, bars + sidx, flags + sidx,
                       reinterpret_cast<const int32_t*>(meta + (issued % kMetaSlots) * G::kMeta), iss, lane, pol);
        iss.advance(a);
        ++issued;
      }
      if (metas < n_mine) {
        copy_meta(a, meta + (metas % kMetaSlots) * G::kMeta, mc, lane);
        mc.advance(a);
        ++metas;
      }
      cp_async_commit();

      // ---- QK^T: rows g, g+8 of the tile; lane quarter c holds d in [c*KB, (c+1)*KB) ----
      float sa[4] = {0.f, 0.f, 0.f, 0.f}, sb[4] = {0.f, 0.f, 0.f, 0.f};
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
        const uint2 qb = *reinterpret_cast<const uint2*>(qh + g * HD + c * KB + 4 * st);
        if (st & 1) mma_bf16(sb, af, qb.x, qb.y);
        else mma_bf16(sa, af, qb.x, qb.y);
      }
      // ---- scores, online softmax (heads 2c, 2c+1; slots g, g+8) ----
      float pr[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float raw = bf16_round(sa[i] + sb[i]);
        const float sc = HD == 256 ? __fmul_rn(raw, 0.0625f) : __fdiv_rn(raw, a.div);
        pr[i] = okv[i >> 1] ? bf16_round(sc) : -INFINITY;
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
      // ---- PV: O^T[d, head] += V^T[d, slot] P^T[slot, head]; lane g holds d0, d0 + 1 of
      // m-tile mt with d0 = 128 (mt / 8) + 16 g + 2 (mt % 8) ----
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int byte = 2 * mt;  // inside this lane's VB bytes
        const int wi = (byte / 4) % 4, vi = byte / 16;
        uint32_t af[4];
        uint32_t wx[4];
        const float(&vs)[4] = vsc[vi];
#pragma unroll
        for (int i = 0; i < 4; ++i) wx[i] = word(vw[i][vi], wi) ^ 0x80808080u;
        if ((byte & 3) == 0) {
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

    // ---- end of segment: per KV head, merge its warps (log-sum-exp, warp order) ----
    if (g == 0) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        m_s[warp * kHeads + 2 * c + hh] = m_run[hh];
        l_s[warp * kHeads + 2 * c + hh] = l_run[hh];
      }
    }
    __syncthreads();
    {
      float f[2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float M = -INFINITY;
        for (int w = 0; w < kAttnWarps; ++w)
          if (!a.hfast || (h0 + w) % a.kv == warp_h) M = fmaxf(M, m_s[w * kHeads + 2 * c + hh]);
        f[hh] = m_run[hh] == -INFINITY ? 0.f : expf(m_run[hh] - M);
        if (g == 0) f_s[warp * kHeads + 2 * c + hh] = f[hh];
      }
      float* ob = o_buf + warp * kHeads * G::kOP;
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int d0 = 128 * (mt / 8) + 16 * g + 2 * (mt % 8);
        float* r0 = ob + (2 * c) * G::kOP;
        float* r1 = ob + (2 * c + 1) * G::kOP;
        r0[G::oc(d0)] = __fmul_rn(o_acc[mt][0], f[0]);
        r1[G::oc(d0)] = __fmul_rn(o_acc[mt][1], f[1]);
        r0[G::oc(d0 + 1)] = __fmul_rn(o_acc[mt][2], f[0]);
        r1[G::oc(d0 + 1)] = __fmul_rn(o_acc[mt][3], f[1]);
      }
    }
    __syncthreads();
    if (tid < nh * kHeads) {  // per (head, query head): the sum L
      const int hl = tid / kHeads, r = tid % kHeads;
      float L = 0.f;
      for (int w = 0; w < kAttnWarps; ++w)
        if (!a.hfast || (h0 + w) % a.kv == hl) L = __fadd_rn(L, __fmul_rn(l_s[w * kHeads + r], f_s[w * kHeads + r]));
      hl_s[tid] = L;
    }
    __syncthreads();
    const long long lo = static_cast<long long>(sg) * a.seg_units;
    const bool whole = lo >= u0 && lo + a.seg_units <= u1;
    const int last = sg == s_first ? 0 : 1;
    for (int i = tid; i < nh * a.r * HD; i += blockDim.x) {
      const int hl = i / (a.r * HD), r = (i / HD) % a.r, d = i % HD;
      // the warps of head hl: w = hl - h0 (mod kv), then every kv-th (all warps unless hfast)
      const int step = a.hfast ? a.kv : 1;
      const int w0 = a.hfast ? (hl - h0 + a.kv) % a.kv : 0;
      float O = 0.f;
      for (int w = w0; w < kAttnWarps; w += step) O = __fadd_rn(O, o_buf[(w * kHeads + r) * G::kOP + G::oc(d)]);
      const int h = h_lo + hl;
      if (whole) {
        const int64_t oi = (static_cast<int64_t>(b) * a.hq + h * a.r + r) * HD + d;
        a.out[oi] = bf16_bits_rne(output_value(__fdiv_rn(O, hl_s[hl * kHeads + r]), a.gate, oi));
      } else {
        float* part = a.part + (static_cast<int64_t>(2 * cta + last) * a.kv + h) * G::kSlotFloats;
        part[2 * kHeads + r * HD + d] = O;
      }
    }
    if (!whole && tid < nh * kHeads) {
      const int hl = tid / kHeads, r = tid % kHeads;
      float M = -INFINITY;
      for (int w = 0; w < kAttnWarps; ++w)
        if (!a.hfast || (h0 + w) % a.kv == hl) M = fmaxf(M, m_s[w * kHeads + r]);
      float* part = a.part + (static_cast<int64_t>(2 * cta + last) * a.kv + h_lo + hl) * G::kSlotFloats;
      part[r] = M;
      part[kHeads + r] = hl_s[tid];
    }
    __syncthreads();  // q_s, o_buf and the statistics are rewritten by the next segment
  }
  // after a timeout, wait (bounded) for the copies still in flight before leaving
  if (!ok)
    for (int n = drain_from; n < issued; ++n) mbar_wait_bounded(bars + n % kStages, (n / kStages) & 1);
  cp_async_wait<0>();
}

// Combine the partials of pairs cut by CTA boundaries: block (pair, query head, d slice);
// thread = 8 consecutive d of one CTA subset; subsets are merged in CTA order.
template <int HD>
__global__ void __launch_bounds__(kMergeThreads) attn_merge_kernel(AttnArgs a, int dslices) {
  using G = Geo<HD>;
  __shared__ float sm_m[kMergeThreads], sm_l[kMergeThreads];
  __shared__ __align__(16) float sm_o[kMergeThreads * 8];
  pdl_wait();
  const int p = blockIdx.x, r = blockIdx.y;
  if (r >= a.r) return;
  const int b = p / a.kv, h = p - b * a.kv;
  const int sg = a.hfast ? b : p;
  const long long lo = static_cast<long long>(sg) * a.seg_units;
  const int c0 = cta_of(lo, a.units, a.ctas), c1 = cta_of(lo + a.seg_units - 1, a.units, a.ctas);
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
        const int first = static_cast<int>(cta_start(cc, a.units, a.ctas) / a.seg_units);
        const float* s = a.part + (static_cast<int64_t>(2 * cc + (first == sg ? 0 : 1)) * a.kv + h) * G::kSlotFloats;
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
  const int64_t oi = ((static_cast<int64_t>(b) * a.hq + h * a.r + r) * HD) + d0;
#pragma unroll
  for (int i = 0; i < 8; ++i) a.out[oi + i] = bf16_bits_rne(output_value(__fdiv_rn(O[i], L), a.gate, oi + i));
}

// CTAs of the split kernel for `units` tiles (one per SM, at least two tiles per warp).
int choose_ctas(long long units) {
  long long c = units / kMinTilesPerCta;
  const long long cap = sm_count();
  if (c > cap) c = cap;
  return c < 1 ? 1 : static_cast<int>(c);
}

size_t slot_bytes(int hd) { return static_cast<size_t>(2 * kHeads + kHeads * hd) * sizeof(float); }

size_t workspace_for(int B, int S, int kv, int hd) {
  const long long units = static_cast<long long>(B) * kv * ((S + 15) / 16);
  const int ctas = choose_ctas(units);
  return ctas > 1 ? 2 * static_cast<size_t>(ctas) * kv * slot_bytes(hd) : 0;
}

// ---- tensor maps (the driver's encoder, looked up once through the runtime) ----
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

// 2D map over `rows` x `cols` elements (row pitch `pitch` bytes), box `box_cols` x
// `box_rows`. False when the encoder is missing or refuses.
bool encode_2d(CUtensorMap* map, const void* base, CUtensorMapDataType type, uint64_t cols, uint64_t rows,
               uint64_t pitch, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encoder();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {pitch};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace
}  // namespace qk

using namespace qk;

extern "C" {

size_t qk_kv_q8_attention_workspace_bytes(int B, int S, int hq, int kv_heads, int head_dim) {
  if (B <= 0 || S <= 0 || kv_heads <= 0 || head_dim <= 0) return 0;
  (void)hq;
  return workspace_for(B, S, kv_heads, head_dim);
}

int qk_kv_q8_attention_check(qk_stream_t stream) {
  int status = 0;
  cudaStream_t st = as_stream(stream);
  cudaError_t e = cudaMemcpyFromSymbolAsync(&status, g_attn_status, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && status) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_attn_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  }
  if (e != cudaSuccess) return cuda_error(e, "qk_kv_q8_attention_check");
  if (status) return set_error(status, "a bounded device wait in the attention kernel gave up");
  return QK_OK;
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
  QK_REQUIRE(static_cast<long long>(B) * T < (1ll << 31) && static_cast<long long>(B) * S < (1ll << 31),
             "B * T and B * S must stay below 2^31");
  AttnArgs a{};
  a.q = q; a.k_codes = k_codes; a.v_codes = v_codes; a.k_scale = k_scale; a.v_scale = v_scale;
  a.indices = indices; a.valid = valid; a.lengths = valid ? nullptr : lengths; a.gate = gate; a.out = out;
  a.B = B; a.S = S; a.T = T; a.hq = hq; a.kv = kv_heads; a.r = hq / kv_heads;
  a.nt = (S + 15) / 16;
  a.units = static_cast<long long>(B) * kv_heads * a.nt;
  a.ctas = choose_ctas(a.units);
  const size_t smem_limit = 227 * 1024;
  const auto smem_of = [&](int nh) { return head_dim == 256 ? Geo<256>::smem(nh) : Geo<128>::smem(nh); };
  a.hfast = kAttnWarps % kv_heads == 0 && smem_of(kv_heads) <= smem_limit;
  QK_REQUIRE(smem_of(a.hfast ? kv_heads : 1) <= smem_limit, "attention geometry exceeds shared memory");
  a.seg_units = a.hfast ? a.nt * kv_heads : a.nt;
  a.idx16 = (S % 4) == 0 && (reinterpret_cast<uintptr_t>(indices) & 15) == 0;
  a.flag16 = valid && (S % 16) == 0 && (reinterpret_cast<uintptr_t>(valid) & 15) == 0;
  a.div = sqrtf(static_cast<float>(head_dim));

  CUtensorMap maps[4];
  memset(maps, 0, sizeof(maps));
  const uint64_t rows = static_cast<uint64_t>(B) * T, width = static_cast<uint64_t>(kv_heads) * head_dim;
  a.tma_codes = encode_2d(&maps[0], k_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, width, rows, width, kBox, 16,
                          CU_TENSOR_MAP_SWIZZLE_128B) &&
                encode_2d(&maps[1], v_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, width, rows, width, kBox, 16,
                          CU_TENSOR_MAP_SWIZZLE_128B);
  const uint64_t planes = static_cast<uint64_t>(B) * kv_heads * (head_dim / 32);
  a.tma_scales = a.tma_codes && (T % 8) == 0 && (reinterpret_cast<uintptr_t>(k_scale) & 15) == 0 &&
                 (reinterpret_cast<uintptr_t>(v_scale) & 15) == 0 &&
                 encode_2d(&maps[2], k_scale, CU_TENSOR_MAP_DATA_TYPE_UINT16, T, planes,
                           static_cast<uint64_t>(T) * 2, 16, head_dim / 32, CU_TENSOR_MAP_SWIZZLE_NONE) &&
                 encode_2d(&maps[3], v_scale, CU_TENSOR_MAP_DATA_TYPE_UINT16, T, planes,
                           static_cast<uint64_t>(T) * 2, 16, head_dim / 32, CU_TENSOR_MAP_SWIZZLE_NONE);

  if (a.ctas > 1) {
    const size_t need = workspace_for(B, S, kv_heads, head_dim);
    if (!workspace || workspace_bytes < need)
      return set_error(QK_ERR_WORKSPACE, "attention workspace needs %zu bytes, got %zu", need, workspace_bytes);
    QK_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 15) == 0, "workspace must be 16-byte aligned");
    a.part = static_cast<float*>(workspace);
  }
  cudaStream_t st = as_stream(stream);
  const size_t smem = smem_of(a.hfast ? kv_heads : 1);
  const void* kern = head_dim == 256 ? reinterpret_cast<const void*>(attn_stream_kernel<256>)
                                     : reinterpret_cast<const void*>(attn_stream_kernel<128>);
  if (int rc = allow_smem(kern, smem)) return rc;
  if (head_dim == 256)
    attn_stream_kernel<256><<<a.ctas, kAttnWarps * 32, smem, st>>>(maps[0], maps[1], maps[2], maps[3], a);
  else
    attn_stream_kernel<128><<<a.ctas, kAttnWarps * 32, smem, st>>>(maps[0], maps[1], maps[2], maps[3], a);
  QK_LAUNCHED("attn_stream_kernel");
  if (a.ctas > 1) {
    // partials per cut segment: about seg_units / (units / ctas) + 1; wider merges split d further
    const long long per = a.units / a.ctas;
    const long long n = (a.seg_units + per - 1) / per + 1;
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
