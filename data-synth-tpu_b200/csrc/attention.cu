// Split-KV decode attention over the Q8 KV cache (reference cache layout).
//
// Replaces the attention core of qwen38_tpu/attention_cache.py:152-170 (step, after the
// cache write): per batch row b and KV head h (a "pair"), the r = hq / kv query heads of
// the group attend over S gathered slots.
//
// Work unit: 128 / kg consecutive slots of one batch row for a group of kg KV heads (kg the
// largest power of two dividing kv, at most 2 at head_dim 256 and 8 at head_dim 128), i.e.
// eight (16-slot tile, KV head) items - one per warp of the CTA. When the unit's cache
// times are consecutive (any page table of 128-slot-multiple pages), its K and V codes
// arrive as 2D tensor copies (TMA) of [unit rows x 128 bytes] boxes with the 128-byte
// shared-memory swizzle (each box 8 KB at head_dim 256, large enough that the copy engine
// streams at HBM speed) and its BF16 scales as one 2D box per plane; otherwise as one bulk
// copy per 128-byte row piece and one load per scale. The units of all batch rows and head
// groups are cut into one contiguous, equal range per CTA (stream-K, one CTA per SM).
//
// Pipeline: the CTA has a two-stage ring of units and a four-slot ring of cache times and
// valid flags, filled by one producer warp (its warpgroup gives registers to the eight
// consumer warps through setmaxnreg). Each consumer warp waits for the stage, loads its
// item's K and V fragments into registers and arrives on the stage's "empty" barrier; the
// producer, once all eight have arrived, starts the time copy of unit k + 4 and the code
// and scale copies of unit k + 2 (it checks that unit's cache times, landed two units
// earlier, for a consecutive run). Units are stepped through with cursors (no divisions).
// Then each warp
//   - dequantises K in registers to bf16(code * scale) (read_quantized, :71-81; the
//     product is exact so the only rounding is BF16 RNE) for QK^T as m16n8k16 MMAs (16
//     slots x 8 query heads, FP32 accumulate); score = bf16(bf16(qk) / sqrt(hd))
//     (:160-165), masked, feeds an online softmax (running max / sum per head, FP32);
//   - dequantises V into the transposed A operand for O^T[d, head] += V^T P^T with
//     P = bf16(exp(score - running max)).
// At the end of a (batch row, head group) segment the CTA merges the warps of each KV head
// with the log-sum-exp rule in warp order. A pair that lies inside one CTA's range is
// finished there: divide by the sum, then bf16(bf16(o) * bf16(sigmoid(gate))) (:170). A
// pair cut by CTA boundaries leaves one partial (max, sum, out) per CTA in the workspace,
// and the merge kernel (launched as a programmatic dependent of the split kernel, so it is
// resident when the split kernel ends) combines them in CTA order.
// Deviation from the reference, inside the 1e-2 layer tolerance: the reference rounds the
// normalised probability to BF16 before PV; here the unnormalised exp(score - max) is
// rounded (normalisation happens after the FP32 sum).
#include <cuda.h>  // CUtensorMap and its enums; the encoder is looked up at run time

#include "common.cuh"

namespace qk {
namespace {

constexpr int kAttnWarps = 8;   // consumer warps per CTA (one CTA per SM); one (tile, head) item each
constexpr int kProducerWarps = 4;  // one warpgroup: its first warp issues the copies, the others leave
constexpr int kThreads = (kAttnWarps + kProducerWarps) * 32;
// setmaxnreg split of the launch's kThreads x 168 registers: consumers grow, producers shrink
constexpr int kLaunchRegs = 168, kConsumerRegs = 232, kProducerRegs = 40;
static_assert(kAttnWarps * 32 * kConsumerRegs + kProducerWarps * 32 * kProducerRegs <= kThreads * kLaunchRegs,
              "register split exceeds the launch's registers");
constexpr int kHeads = 8;       // query heads per KV head handled by the MMA column block
constexpr int kStages = 2;      // unit ring depth
constexpr int kMetaSlots = 4;   // cache-time ring: unit n's times are copied at unit n-4's release
constexpr int kUnitRows = 128;  // slots x heads of a unit (16 slots x 8 warps)
constexpr int kMergeThreads = 256;
constexpr int kBox = 128;       // bytes of one tensor-copy box row (the 128-byte swizzle span)
constexpr int kMetaBytes = kUnitRows * 4 + kUnitRows;  // cache times (int32), valid flags (uint8)

template <int HD>
struct Geo {
  static constexpr int kGroups = HD / 32;                 // scale groups per head row
  static constexpr int kCodes = kUnitRows * HD;           // one plane of a unit: [box][rows][128 B]
  static constexpr int kKgMax = HD == 256 ? 2 : 8;        // KV heads per unit at most
  // one scale plane: [kg * groups][rows + 8] BF16 (the 8-time pad staggers the groups over
  // the shared-memory banks), sized for the largest kg
  static constexpr int kScales = 8 * HD + kKgMax * HD / 2;
  static constexpr int kStage = (2 * kCodes + 2 * kScales + 1023) / 1024 * 1024;  // swizzle atoms
  static constexpr int kQP = HD + 16;                     // q_s row (bf16): 4 blocks of HD / 4, each + 4
  static constexpr int kOP = HD == 256 ? 274 : 146;       // o_buf row (floats): conflict-free writes
  static constexpr int kOOff = kStages * kStage;          // float o_buf[warps][kHeads][kOP]
  static constexpr int kMOff = kOOff + kAttnWarps * kHeads * kOP * 4;  // float m_s, l_s, f_s [warps][kHeads]
  static constexpr int kIdxOff = kMOff + 3 * kAttnWarps * kHeads * 4;  // [kMetaSlots][kMetaBytes]
  static constexpr int kBarOff = kIdxOff + kMetaSlots * kMetaBytes;    // uint64 full[stages], meta[slots], empty[stages]
  static constexpr int kCtlOff = kBarOff + (2 * kStages + kMetaSlots) * 8; // uint32 swz[stages], abort
  static constexpr int kQOff = kCtlOff + 64;                           // bf16 q_s[kg][kHeads][kQP], then float L
  static constexpr int kSlotFloats = 2 * kHeads + kHeads * HD;         // partial: m, l, o
  static_assert(kStage % 1024 == 0, "stage size");
  // dynamic shared memory for kg KV heads per unit (plus slack to align to 1024)
  static constexpr size_t smem(int kg) { return kQOff + static_cast<size_t>(kg) * kHeads * (kQP * 2 + 4) + 1024; }
  // q_s element of (head row, d): blocks of HD / 4 (one lane quarter's K bytes) 8 bytes apart
  __device__ static int qi(int hrow, int d) { return hrow * kQP + (d / (HD / 4)) * (HD / 4 + 4) + d % (HD / 4); }
  // byte offset of (row, 16-byte chunk of the kg-head row) in a code plane of `rows` rows
  __device__ static int at(int rows, int row, int chunk, bool swz) {
    return (chunk >> 3) * (rows * kBox) + row * kBox + (((chunk & 7) ^ (swz ? (row & 7) : 0)) << 4);
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
  float* po;         // partial mode (time-sharded callers): FP32 [B, hq, HD] unnormalised output
  float* pst;        // ... and FP32 [B, hq, 2] (max, sum) of it, in place of out
  float* part;       // [2 * ctas][kv][kSlotFloats]: CTA c's first (2c) and last (2c + 1) segment
  long long units;   // B * groups * nch
  int B, S, T, hq, kv, r, ctas;
  int kg;            // KV heads per unit
  int rows;          // slots per unit = kUnitRows / kg
  int groups;        // kv / kg head groups
  int nch;           // units per segment (batch row, head group) = ceil(S / rows)
  int tma_codes;     // code tiles of consecutive times use the tensor maps
  int code3d;        // ... one 3D box per plane (else one 2D box per 128-byte column block)
  int tma_scales;    // ... and the scale tiles too (T % 8 == 0, aligned planes)
  int idx16;         // cache-time rows 16-byte aligned (S % 4 == 0): the time ring is used
  int flag16;        // valid rows 16-byte aligned (S % 16 == 0): flags ride in the time ring
  float div;         // f32(sqrt(hd))
};

// Set when a bounded wait of the split kernel gives up; read and cleared by
// qk_kv_q8_attention_check.
__device__ int g_attn_status;

__host__ __device__ __forceinline__ long long cta_start(long long c, long long units, int ctas) {
  return c * units / ctas;
}
// The CTA whose range holds unit u: the largest c with cta_start(c) <= u.
__device__ __forceinline__ int cta_of(long long u, long long units, int ctas) {
  return static_cast<int>(((u + 1) * ctas - 1) / units);
}

__device__ __forceinline__ int wrap_clamp(int t, int T) {
  if (t < 0) t += T;
  return t < 0 ? 0 : (t >= T ? T - 1 : t);
}

// Byte I of `wx` (a code byte with its sign bit flipped, u = code + 128) as the FP32
// number 2^15 + u: bit pattern 0x47 | 0x00 | u | 0x00, one byte permute.
template <int I>
__device__ __forceinline__ float s8_at(uint32_t wx) {
  return __uint_as_float(__byte_perm(wx, 0x4700u, 0x5404u | (I << 4)));
}

// bf16(code * s) for two codes given as 2^15 + u: fma(2^15 + u, s, k) with k = -(2^15 + 128) s
// is exactly code * s before the one rounding to FP32 (code * s has at most 16 significant
// bits and k at most 17, so both are exact), then BF16 RNE as in read_quantized.
__device__ __forceinline__ float dq_bias(float s) { return __fmul_rn(s, -32896.f); }
__device__ __forceinline__ uint32_t dq_pair(float c0, float c1, float s0, float s1, float k0, float k1) {
  const float2 v = __ffma2_rn(make_float2(c0, c1), make_float2(s0, s1), make_float2(k0, k1));
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

// 3D tensor copy (no multicast): one box of a [col block][time row][128 bytes] view.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Expected transaction bytes without an arrival, and a plain arrival (release): the
// issuing warp registers the copies' bytes, issues them, makes its own stores, then arrives.
__device__ __forceinline__ void mbar_expect_only(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive_release(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// Bounded wait that also gives up at once when another warp has aborted (*abort != 0).
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile uint32_t* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (*abort) return false;
    if (mbar_try_wait_suspend(bar, parity, kWaitHintNs)) return true;
  }
  return false;
}

// A unit of the CTA order: segment (batch row b, head group hg) and chunk ch of `rows`
// slots. Decoded from the unit number once; cursors then step through consecutive units
// without divisions.
struct Unit {
  int b, hg, ch;
  __device__ Unit(long long n, const AttnArgs& a) {
    const int seg = static_cast<int>(n / a.nch);
    ch = static_cast<int>(n - static_cast<long long>(seg) * a.nch);
    b = seg / a.groups;
    hg = seg - b * a.groups;
  }
  __device__ void next(const AttnArgs& a) {
    if (++ch == a.nch) {
      ch = 0;
      if (++hg == a.groups) {
        hg = 0;
        ++b;
      }
    }
  }
  __device__ int s0(const AttnArgs& a) const { return ch * a.rows; }
  __device__ int nvalid(const AttnArgs& a) const { return min(a.rows, a.S - ch * a.rows); }
};

// Start the copy of unit n's cache times (and valid flags) into a time-ring slot (one
// thread; only when the rows are 16-byte aligned).
__device__ __forceinline__ void issue_meta(const AttnArgs& a, uint8_t* slot, uint64_t* bar, const Unit& u) {
  const int nvalid = u.nvalid(a);
  const int64_t row = static_cast<int64_t>(u.b) * a.S + u.s0(a);
  const uint32_t flags = a.flag16 ? static_cast<uint32_t>(nvalid) : 0u;
  mbar_expect_tx(bar, static_cast<uint32_t>(nvalid) * 4u + flags);
  bulk_g2s(slot, a.indices + row, static_cast<uint32_t>(nvalid) * 4u, bar);
  if (flags) bulk_g2s(slot + kUnitRows * 4, a.valid + row, flags, bar);
}

// Issue unit n's code and scale copies into `stage` (one warp), completing on `full`.
// `swz` records whether the code planes are swizzled (tensor copies). Returns false when
// the wait for the unit's cache times gave up.
template <int HD>
__device__ __forceinline__ bool issue_unit(const AttnArgs& a, const CUtensorMap* tm_k, const CUtensorMap* tm_v,
                                           const CUtensorMap* tm_ks, const CUtensorMap* tm_vs, uint8_t* stage,
                                           uint64_t* full, uint32_t* swz, const uint8_t* mslot, uint64_t* mbar,
                                           uint32_t mparity, volatile uint32_t* abort, const Unit& u, int lane,
                                           uint64_t pol) {
  using G = Geo<HD>;
  const int rows = a.rows, kg = a.kg;
  const int nvalid = u.nvalid(a);
  const int32_t* times = reinterpret_cast<const int32_t*>(mslot);
  const int64_t trow = static_cast<int64_t>(u.b) * a.S + u.s0(a);
  int t0;
  bool run;
  {
    bool ok = true;
    if (a.idx16) ok = wait_or_abort(mbar, mparity, abort);
    if (!__all_sync(0xffffffffu, ok)) return false;
    // lane l holds the times of slots l, l + 32, ... (rows <= 128)
    int t[kUnitRows / 32];
    run = true;
#pragma unroll
    for (int q = 0; q < kUnitRows / 32; ++q) t[q] = 0;
    if (a.idx16) {
#pragma unroll
      for (int q = 0; q < kUnitRows / 32; ++q) {
        const int s = lane + 32 * q;
        if (s < nvalid) t[q] = wrap_clamp(times[s], a.T);
      }
    } else {
#pragma unroll
      for (int q = 0; q < kUnitRows / 32; ++q) {
        const int s = lane + 32 * q;
        if (s < nvalid) t[q] = wrap_clamp(a.indices[trow + s], a.T);
      }
    }
    t0 = __shfl_sync(0xffffffffu, t[0], 0);
#pragma unroll
    for (int q = 0; q < kUnitRows / 32; ++q) {
      const int s = lane + 32 * q;
      if (s < nvalid && t[q] != t0 + s) run = false;
    }
    run = __all_sync(0xffffffffu, run) && nvalid == rows;
  }
  const bool tma = a.tma_codes && run;  // times t0 .. t0 + rows - 1, all < T
  const bool tma_s = tma && a.tma_scales && (t0 & 7) == 0;
  const int nbox = kg * HD / kBox;
  const int sp = rows + 8;  // scale plane pitch (times)
  const uint32_t bytes = (tma ? 2u * G::kCodes : static_cast<uint32_t>(nvalid) * 2u * kg * HD) +
                         (tma_s ? 4u * kg * G::kGroups * sp : 0u);
  if (lane == 0) {
    *swz = tma ? 1u : 0u;
    mbar_expect_only(full, bytes);
  }
  __syncwarp();

  bool generic = false;
  const int col0 = u.hg * kg * HD;  // first code byte of the head group in a cache row
  if (tma && a.code3d) {
    if (lane < 2) tma_load_3d(stage + lane * G::kCodes, lane ? tm_v : tm_k, 0, u.b * a.T + t0, col0 / kBox, full, pol);
  } else if (tma) {
    if (lane < 2 * nbox) {
      const int plane = lane / nbox, e = lane % nbox;
      tma_load_2d(stage + plane * G::kCodes + e * rows * kBox, plane ? tm_v : tm_k, col0 + e * kBox,
                  u.b * a.T + t0, full, pol);
    }
  } else {
    // one bulk copy per (row, plane, 128-byte piece); rows past S are zero
    for (int item = lane; item < rows * 2 * nbox; item += 32) {
      const int s = item % rows, pe = item / rows, plane = pe / nbox, e = pe % nbox;
      uint8_t* dst = stage + plane * G::kCodes + e * rows * kBox + s * kBox;
      if (s < nvalid) {
        const int ts = wrap_clamp(a.idx16 ? times[s] : a.indices[trow + s], a.T);
        const int64_t off = (static_cast<int64_t>(u.b) * a.T + ts) * a.kv * HD + col0 + e * kBox;
        bulk_g2s_hint(dst, (plane ? a.v_codes : a.k_codes) + off, kBox, full, pol);
      } else {
#pragma unroll
        for (int i = 0; i < kBox / 16; ++i) reinterpret_cast<uint4*>(dst)[i] = make_uint4(0u, 0u, 0u, 0u);
        generic = true;
      }
    }
  }
  uint8_t* sc = stage + 2 * G::kCodes;
  const int grp0 = (u.b * a.kv + u.hg * kg) * G::kGroups;  // first scale row of the head group
  if (tma_s) {
    if (lane < 2) tma_load_2d(sc + lane * G::kScales, lane ? tm_vs : tm_ks, t0, grp0, full, pol);
  } else {
    // [kg * groups][rows + 8] per plane; rows past S are zero
    for (int item = lane; item < rows * kg * G::kGroups * 2; item += 32) {
      const int s = item % rows, rg = (item / rows) % (kg * G::kGroups), plane = item / (rows * kg * G::kGroups);
      uint16_t v = 0;
      if (s < nvalid) {
        const int ts = wrap_clamp(a.idx16 ? times[s] : a.indices[trow + s], a.T);
        v = (plane ? a.v_scale : a.k_scale)[static_cast<int64_t>(grp0 + rg) * a.T + ts];
      }
      reinterpret_cast<uint16_t*>(sc + plane * G::kScales)[rg * sp + s] = v;
    }
    generic = true;
  }
  // generic stores into the stage come before any later asynchronous copy into it
  if (__any_sync(0xffffffffu, generic)) fence_proxy_async_smem();
  __syncwarp();
  // the stage's one arrival, after every lane's stores (the phase completes once the
  // copies' bytes have landed as well)
  if (lane == 0) mbar_arrive_release(full);
  return true;
}

// Barrier over the consumer warps only (the producer warpgroup never joins).
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kAttnWarps * 32) : "memory");
}

template <int N>
__device__ __forceinline__ void regs_grow() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_shrink() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// The producer warp: for each unit of the CTA's range, wait until the consumers are done
// with the unit two places back (its stage and time slot), start the time copy of the unit
// two places ahead and the code / scale copies of this unit. Returns false on a timeout.
template <int HD>
__device__ __forceinline__ bool attn_produce(const AttnArgs& a, const CUtensorMap* tm_k, const CUtensorMap* tm_v,
                                          const CUtensorMap* tm_ks, const CUtensorMap* tm_vs, uint8_t* smem,
                                          long long u0, int nk, int lane) {
  using G = Geo<HD>;
  uint8_t* meta = smem + G::kIdxOff;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + G::kBarOff);
  uint64_t* mbar = full + kStages;
  uint64_t* empty = mbar + kMetaSlots;
  uint32_t* swz = reinterpret_cast<uint32_t*>(smem + G::kCtlOff);
  volatile uint32_t* abort = swz + kStages;
  const uint64_t pol = l2_evict_first_policy();
  Unit iss(u0, a), met(u0, a);
  for (int m = 0; m < 2; ++m) {
    if (a.idx16 && lane == 0 && m < nk) issue_meta(a, meta + m * kMetaBytes, mbar + m, met);
    met.next(a);
  }
  for (int n = 0; n < nk; ++n) {
    const int st = n % kStages;
    if (n >= kStages && !__all_sync(0xffffffffu, wait_or_abort(empty + st, (n / kStages - 1) & 1, abort)))
      return false;
    const int nm = n + 2;  // its time slot held unit n - 2
    if (a.idx16 && lane == 0 && nm < nk)
      issue_meta(a, meta + (nm % kMetaSlots) * kMetaBytes, mbar + nm % kMetaSlots, met);
    met.next(a);
    if (!issue_unit<HD>(a, tm_k, tm_v, tm_ks, tm_vs, smem + st * G::kStage, full + st, swz + st,
                        meta + (n % kMetaSlots) * kMetaBytes, mbar + n % kMetaSlots, (n / kMetaSlots) & 1, abort,
                        iss, lane, pol))
      return false;
    iss.next(a);
  }
  return true;
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
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
  float* o_buf = reinterpret_cast<float*>(smem + G::kOOff);
  float* m_s = reinterpret_cast<float*>(smem + G::kMOff);
  float* l_s = m_s + kAttnWarps * kHeads;
  float* f_s = l_s + kAttnWarps * kHeads;
  uint8_t* meta = smem + G::kIdxOff;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + G::kBarOff);
  uint64_t* mbar = full + kStages;
  uint64_t* empty = mbar + kMetaSlots;
  uint32_t* swz = reinterpret_cast<uint32_t*>(smem + G::kCtlOff);
  volatile uint32_t* abort = swz + kStages;
  uint16_t* q_s = reinterpret_cast<uint16_t*>(smem + G::kQOff);
  float* hl_s = reinterpret_cast<float*>(smem + G::kQOff + a.kg * kHeads * G::kQP * 2);  // [kg][kHeads]

  const int kg = a.kg, rows = a.rows;
  const int item_tile = warp / kg, hl_w = warp % kg;  // this warp's (tile, head) in every unit

  if (tid == 0) {
    for (int i = 0; i < kStages + kMetaSlots; ++i) mbar_init(full + i, 1);
    for (int i = 0; i < kStages; ++i) mbar_init(empty + i, kAttnWarps);
    *abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // Launched as a programmatic dependent: the set-up above overlaps the previous kernel (the
  // cache append); the cache, q and the lengths are read only after it has finished.
  pdl_wait();
  pdl_trigger();  // the merge kernel may take its place now; it waits for this grid to end

  const int cta = blockIdx.x;
  const long long u0 = cta_start(cta, a.units, a.ctas), u1 = cta_start(cta + 1, a.units, a.ctas);
  const int nk = static_cast<int>(u1 - u0);

  if (warp >= kAttnWarps) {  // the producer warpgroup
    regs_shrink<kProducerRegs>();
    if (warp == kAttnWarps) {
      if (!attn_produce<HD>(a, &tm_k, &tm_v, &tm_ks, &tm_vs, smem, u0, nk, lane) && lane == 0) {
        atomicExch(&g_attn_status, QK_ERR_TIMEOUT);
        *abort = 1;
      }
      // after an abort, wait (bounded) for copies that may still be in flight before leaving
      if (*abort && lane == 0) {
        for (int i = 0; i < kStages; ++i) {
          mbar_wait_bounded(full + i, 0);
          mbar_wait_bounded(full + i, 1);
        }
      }
    }
    return;
  }
  regs_grow<kConsumerRegs>();
  bool ok = true;
  Unit cur(u0, a);

  const int s_first = static_cast<int>(u0 / a.nch), s_last = static_cast<int>((u1 - 1) / a.nch);
  int k = 0;
  for (int sg = s_first; sg <= s_last; ++sg) {
    const int b = sg / a.groups, hg = sg - b * a.groups;
    // q of the segment's heads: q_s[hl][r][d] (padded blocks), zero rows for r >= a.r. With
    // an aligned q every thread issues its 16-byte loads (at most 4) before storing any: a
    // 2-byte load per store put one global round trip per 256 values on every segment start.
    if ((reinterpret_cast<uintptr_t>(a.q) & 15) == 0) {
      constexpr int kQChunks = (Geo<HD>::kKgMax * kHeads * HD / 8 + kAttnWarps * 32 - 1) / (kAttnWarps * 32);
      const int nq = kg * kHeads * HD / 8;
      uint4 qv[kQChunks];
#pragma unroll
      for (int c = 0; c < kQChunks; ++c) {
        const int i = tid + c * kAttnWarps * 32, e = 8 * i;
        const int hl = e / (kHeads * HD), r = (e / HD) % kHeads, d = e % HD;
        qv[c] = i < nq && r < a.r ? *reinterpret_cast<const uint4*>(
                                        a.q + (static_cast<int64_t>(b) * a.hq + (hg * kg + hl) * a.r + r) * HD + d)
                                  : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int c = 0; c < kQChunks; ++c) {
        const int i = tid + c * kAttnWarps * 32, e = 8 * i;
        if (i >= nq) break;
        const int hl = e / (kHeads * HD), r = (e / HD) % kHeads, d = e % HD;
        uint2* dst = reinterpret_cast<uint2*>(q_s + G::qi(hl * kHeads + r, d));  // 8-byte aligned
        dst[0] = make_uint2(qv[c].x, qv[c].y);
        dst[1] = make_uint2(qv[c].z, qv[c].w);
      }
    } else {
      for (int i = tid; i < kg * kHeads * HD; i += kAttnWarps * 32) {
        const int hl = i / (kHeads * HD), r = (i / HD) % kHeads, d = i % HD;
        q_s[G::qi(hl * kHeads + r, d)] =
            r < a.r ? a.q[(static_cast<int64_t>(b) * a.hq + (hg * kg + hl) * a.r + r) * HD + d] : 0;
      }
    }
    const int len = a.valid ? 0 : a.lengths[b];
    consumer_sync();
    const uint16_t* qh = q_s + hl_w * kHeads * G::kQP;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    float o_acc[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) o_acc[mt][0] = o_acc[mt][1] = o_acc[mt][2] = o_acc[mt][3] = 0.f;

    for (; k < nk && cur.b == b && cur.hg == hg; ++k, cur.next(a)) {
      const int sidx = k % kStages;
      const uint8_t* stage = smem + sidx * G::kStage;
      const bool got = ok && wait_or_abort(full + sidx, (k / kStages) & 1, abort);
      if (!__all_sync(0xffffffffu, got) && ok) {
        if (lane == 0) {
          atomicExch(&g_attn_status, QK_ERR_TIMEOUT);
          *abort = 1;
        }
        ok = false;
      }
      const int s0 = cur.s0(a);
      const int r0 = item_tile * 16;  // this warp's first row in the unit
      // ---- fragments of this item into registers, then release the stage ----
      uint4 kw[2][KV4];
      float ks[2][KG];            // K scales
      uint4 vw[4][VV4];           // V code words, sign bits flipped
      float vsc[VV4][4];  // V scale of chunk jj (d in [128 jj + 16 g, +16): group g / 2 + 4 jj)
      bool okv[2];
      {
        const bool sw = swz[sidx] != 0;
        const uint8_t* kt = stage;
        const uint8_t* vt = stage + G::kCodes;
        const int sp = rows + 8;  // scale plane pitch
        const uint16_t* kss = reinterpret_cast<const uint16_t*>(stage + 2 * G::kCodes) + hl_w * G::kGroups * sp;
        const uint16_t* vss = kss + G::kScales / 2;
        const int ch0 = hl_w * (HD / 16);  // this head's first 16-byte chunk in a kg-head row
#pragma unroll
        for (int rh = 0; rh < 2; ++rh) {
          const int row = r0 + g + 8 * rh;
#pragma unroll
          for (int i = 0; i < KV4; ++i) kw[rh][i] = lds_v4(kt + G::at(rows, row, ch0 + c * KV4 + i, sw));
#pragma unroll
          for (int i = 0; i < KG; ++i) ks[rh][i] = bf16_to_f32(kss[(c * KG + i) * sp + row]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int row = r0 + 2 * c + (i & 1) + 8 * (i >> 1);
#pragma unroll
          for (int jj = 0; jj < VV4; ++jj) {
            vw[i][jj] = lds_v4(vt + G::at(rows, row, ch0 + g + 8 * jj, sw));
            vw[i][jj].x ^= 0x80808080u;
            vw[i][jj].y ^= 0x80808080u;
            vw[i][jj].z ^= 0x80808080u;
            vw[i][jj].w ^= 0x80808080u;
            vsc[jj][i] = bf16_to_f32(vss[(g / 2 + 4 * jj) * sp + row]);
          }
        }
        const uint8_t* mslot = meta + (k % kMetaSlots) * kMetaBytes;
#pragma unroll
        for (int rh = 0; rh < 2; ++rh) {
          const int s = s0 + r0 + g + 8 * rh;
          bool v = s < a.S;
          if (v) {
            if (!a.valid) v = s <= len;
            else if (a.flag16) v = mslot[kUnitRows * 4 + r0 + g + 8 * rh] != 0;
            else v = a.valid[static_cast<int64_t>(b) * a.S + s] != 0;
          }
          okv[rh] = v;
        }
      }
      // this warp is done with the stage and the unit's time slot (release: every lane's
      // reads come first); the producer refills them once all eight warps have arrived
      __syncwarp();
      if (lane == 0) mbar_arrive_release(empty + sidx);
      if (!ok) continue;

      // ---- QK^T: rows g, g+8 of the tile; lane quarter c holds d in [c*KB, (c+1)*KB) ----
      float sacc[4][4];  // four independent MMA chains over the k-steps
#pragma unroll
      for (int i = 0; i < 4; ++i) sacc[i][0] = sacc[i][1] = sacc[i][2] = sacc[i][3] = 0.f;
#pragma unroll
      for (int st = 0; st < KSTEPS; ++st) {
        const int j = st / 4;  // the lane's 16-byte chunk
        uint32_t af[4];
#pragma unroll
        for (int rh = 0; rh < 2; ++rh) {
          const uint32_t wx = word(kw[rh][st / 4], st % 4) ^ 0x80808080u;
          const float sc = ks[rh][j >> 1], kc = dq_bias(sc);
          af[rh] = dq_pair(s8_at<0>(wx), s8_at<1>(wx), sc, sc, kc, kc);
          af[2 + rh] = dq_pair(s8_at<2>(wx), s8_at<3>(wx), sc, sc, kc, kc);
        }
        const uint2 qb = *reinterpret_cast<const uint2*>(qh + G::qi(g, c * KB + 16 * j + 4 * (st % 4)));
        mma_bf16(sacc[st & 3], af, qb.x, qb.y);
      }
      // ---- scores, online softmax (heads 2c, 2c+1; slots g, g+8) ----
      float pr[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float raw = bf16_round((sacc[0][i] + sacc[1][i]) + (sacc[2][i] + sacc[3][i]));
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
          alpha[hh] = exp_ref(m_run[hh] - m_new);
          pr[hh] = exp_ref(pr[hh] - m_new);
          pr[2 + hh] = exp_ref(pr[2 + hh] - m_new);
        }
        m_run[hh] = m_new;
      }
      // P in BF16 (the MMA operand); the running sum uses the same rounded values. Each lane
      // keeps the sum of its own slots (the lanes of a head are added at the segment's end).
      const uint32_t P0 = pack_bf16x2(pr[0], pr[1]), P1 = pack_bf16x2(pr[2], pr[3]);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const float ps = __fadd_rn(bf16_to_f32(static_cast<uint16_t>(P0 >> (16 * hh))),
                                   bf16_to_f32(static_cast<uint16_t>(P1 >> (16 * hh))));
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
        const float vb[4] = {dq_bias(vs[0]), dq_bias(vs[1]), dq_bias(vs[2]), dq_bias(vs[3])};
#pragma unroll
        for (int i = 0; i < 4; ++i) wx[i] = word(vw[i][vi], wi);
        if ((byte & 3) == 0) {
          af[0] = dq_pair(s8_at<0>(wx[0]), s8_at<0>(wx[1]), vs[0], vs[1], vb[0], vb[1]);
          af[1] = dq_pair(s8_at<1>(wx[0]), s8_at<1>(wx[1]), vs[0], vs[1], vb[0], vb[1]);
          af[2] = dq_pair(s8_at<0>(wx[2]), s8_at<0>(wx[3]), vs[2], vs[3], vb[2], vb[3]);
          af[3] = dq_pair(s8_at<1>(wx[2]), s8_at<1>(wx[3]), vs[2], vs[3], vb[2], vb[3]);
        } else {
          af[0] = dq_pair(s8_at<2>(wx[0]), s8_at<2>(wx[1]), vs[0], vs[1], vb[0], vb[1]);
          af[1] = dq_pair(s8_at<3>(wx[0]), s8_at<3>(wx[1]), vs[0], vs[1], vb[0], vb[1]);
          af[2] = dq_pair(s8_at<2>(wx[2]), s8_at<2>(wx[3]), vs[2], vs[3], vb[2], vb[3]);
          af[3] = dq_pair(s8_at<3>(wx[2]), s8_at<3>(wx[3]), vs[2], vs[3], vb[2], vb[3]);
        }
        mma_bf16(o_acc[mt], af, b0, b1);
      }
    }

    // ---- end of segment: per KV head, merge its warps (log-sum-exp, warp order) ----
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {  // the lanes' partial sums of a head
      l_run[hh] += __shfl_xor_sync(0xffffffffu, l_run[hh], 4);
      l_run[hh] += __shfl_xor_sync(0xffffffffu, l_run[hh], 8);
      l_run[hh] += __shfl_xor_sync(0xffffffffu, l_run[hh], 16);
    }
    if (g == 0) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        m_s[warp * kHeads + 2 * c + hh] = m_run[hh];
        l_s[warp * kHeads + 2 * c + hh] = l_run[hh];
      }
    }
    consumer_sync();
    {
      float f[2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float M = -INFINITY;
        for (int w = hl_w; w < kAttnWarps; w += kg) M = fmaxf(M, m_s[w * kHeads + 2 * c + hh]);
        f[hh] = m_run[hh] == -INFINITY ? 0.f : exp_ref(m_run[hh] - M);
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
    consumer_sync();
    if (tid < kg * kHeads) {  // per (head, query head): the sum L
      const int hl = tid / kHeads, r = tid % kHeads;
      float L = 0.f;
      for (int w = hl; w < kAttnWarps; w += kg) L = __fadd_rn(L, __fmul_rn(l_s[w * kHeads + r], f_s[w * kHeads + r]));
      hl_s[tid] = L;
    }
    consumer_sync();
    const long long lo = static_cast<long long>(sg) * a.nch;
    const bool whole = lo >= u0 && lo + a.nch <= u1;
    const int last = sg == s_first ? 0 : 1;
    for (int i = tid; i < kg * a.r * HD; i += kAttnWarps * 32) {
      const int hl = i / (a.r * HD), r = (i / HD) % a.r, d = i % HD;
      float O = 0.f;
      for (int w = hl; w < kAttnWarps; w += kg) O = __fadd_rn(O, o_buf[(w * kHeads + r) * G::kOP + G::oc(d)]);
      const int h = hg * kg + hl;
      if (whole) {
        const int64_t oi = (static_cast<int64_t>(b) * a.hq + h * a.r + r) * HD + d;
        if (a.po)
          a.po[oi] = O;
        else
          a.out[oi] = bf16_bits_rne(output_value(__fdiv_rn(O, hl_s[hl * kHeads + r]), a.gate, oi));
      } else {
        float* part = a.part + (static_cast<int64_t>(2 * cta + last) * a.kv + h) * G::kSlotFloats;
        part[2 * kHeads + r * HD + d] = O;
      }
    }
    if ((!whole || a.po) && tid < kg * kHeads) {
      const int hl = tid / kHeads, r = tid % kHeads;
      float M = -INFINITY;
      for (int w = hl; w < kAttnWarps; w += kg) M = fmaxf(M, m_s[w * kHeads + r]);
      if (!whole) {
        float* part = a.part + (static_cast<int64_t>(2 * cta + last) * a.kv + hg * kg + hl) * G::kSlotFloats;
        part[r] = M;
        part[kHeads + r] = hl_s[tid];
      } else if (r < a.r) {
        const int64_t si = (static_cast<int64_t>(b) * a.hq + (hg * kg + hl) * a.r + r) * 2;
        a.pst[si] = M;
        a.pst[si + 1] = hl_s[tid];
      }
    }
    consumer_sync();  // q_s, o_buf and the statistics are rewritten by the next segment
  }
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
  const int sg = b * a.groups + h / a.kg;
  const long long lo = static_cast<long long>(sg) * a.nch;
  const int c0 = cta_of(lo, a.units, a.ctas), c1 = cta_of(lo + a.nch - 1, a.units, a.ctas);
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
        const int first = static_cast<int>(cta_start(cc, a.units, a.ctas) / a.nch);
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
      const float fo = m == -INFINITY ? 0.f : exp_ref(m - M);
      const float fn = pm[u] == -INFINITY ? 0.f : exp_ref(pm[u] - M);
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
    const float fk = sm_m[t] == -INFINITY ? 0.f : exp_ref(sm_m[t] - M);
    L = __fadd_rn(L, __fmul_rn(sm_l[t], fk));
#pragma unroll
    for (int i = 0; i < 8; ++i) O[i] = __fadd_rn(O[i], __fmul_rn(sm_o[t * 8 + i], fk));
  }
  const int64_t oi = ((static_cast<int64_t>(b) * a.hq + h * a.r + r) * HD) + d0;
  if (a.po) {  // partial mode: the unnormalised output and its (max, sum)
#pragma unroll
    for (int i = 0; i < 8; ++i) a.po[oi + i] = O[i];
    if (d0 == 0) {
      const int64_t si = (static_cast<int64_t>(b) * a.hq + h * a.r + r) * 2;
      a.pst[si] = M;
      a.pst[si + 1] = L;
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) a.out[oi + i] = bf16_bits_rne(output_value(__fdiv_rn(O[i], L), a.gate, oi + i));
}

// Log-sum-exp combine of R partial (output, max, sum) sets in set order (the time shards of
// one decode step, all-gathered across ranks): out = bf16(gate(sum_r o_r e^(m_r - M) /
// sum_r l_r e^(m_r - M))). A set is rows * hd outputs followed by rows (max, sum) pairs.
// Block = one (batch row, query head); thread = consecutive d.
__global__ void __launch_bounds__(256) attn_combine_kernel(const float* __restrict__ parts, int R, long long rows,
                                                           int hd, const uint16_t* gate, uint16_t* out) {
  const long long row = blockIdx.x;
  const long long set = rows * (hd + 2);
  float M = -INFINITY;
  for (int k = 0; k < R; ++k) M = fmaxf(M, parts[k * set + rows * hd + row * 2]);
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float L = 0.f, O = 0.f;
    for (int k = 0; k < R; ++k) {
      const float* st = parts + k * set + rows * hd + row * 2;
      const float f = st[0] == -INFINITY ? 0.f : exp_ref(st[0] - M);
      L = __fadd_rn(L, __fmul_rn(st[1], f));
      O = __fadd_rn(O, __fmul_rn(parts[k * set + row * hd + d], f));
    }
    const int64_t oi = row * hd + d;
    out[oi] = bf16_bits_rne(output_value(__fdiv_rn(O, L), gate, oi));
  }
}

// KV heads per unit: the largest power of two dividing kv, at most 2 at head_dim 256 (the
// query tile of more KV heads would not fit beside the ring) and 8 at head_dim 128.
int heads_per_unit(int kv, int hd) {
  int kg = 1;
  while (kg * 2 <= (hd == 256 ? 2 : 8) && kv % (kg * 2) == 0) kg *= 2;
  return kg;
}

// CTAs of the split kernel: one per SM, at most one per unit.
int choose_ctas(long long units) {
  const long long cap = sm_count();
  return static_cast<int>(units < cap ? (units < 1 ? 1 : units) : cap);
}

long long units_for(int B, int S, int kv, int hd) {
  const int kg = heads_per_unit(kv, hd), rows = kUnitRows / kg;
  return static_cast<long long>(B) * (kv / kg) * ((S + rows - 1) / rows);
}

size_t slot_bytes(int hd) { return static_cast<size_t>(2 * kHeads + kHeads * hd) * sizeof(float); }

size_t workspace_for(int B, int S, int kv, int hd) {
  const int ctas = choose_ctas(units_for(B, S, kv, hd));
  return ctas > 1 ? 2 * static_cast<size_t>(ctas) * kv * slot_bytes(hd) : 0;
}

// ---- tensor maps (the driver's encoder, looked up once through the runtime) ----
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() { return reinterpret_cast<EncodeTiledFn>(tensor_map_encoder()); }

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

// 3D map over a [rows][cols] byte plane viewed as [cols / 128][rows][128] (column blocks
// outermost, so a box lands in shared memory as [block][row][128 bytes], the 2D boxes'
// layout), box 128 x box_rows x box_blocks with the 128-byte swizzle.
bool encode_blocks_3d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint32_t box_rows,
                      uint32_t box_blocks) {
  EncodeTiledFn fn = encoder();
  if (!fn || cols % kBox) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kBox), rows, cols / kBox};
  const cuuint64_t strides[2] = {cols, static_cast<cuuint64_t>(kBox)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(kBox), box_rows, box_blocks};
  const cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
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

}  // extern "C"

namespace {

// The split and merge launches of one decode attention call: the final BF16 output into
// `out`, or (po != NULL) the unnormalised FP32 output and its (max, sum) statistics.
int launch_attention(const uint16_t* q, const int8_t* k_codes, const int8_t* v_codes, const uint16_t* k_scale,
                     const uint16_t* v_scale, const int32_t* indices, const uint8_t* valid, const int32_t* lengths,
                     const uint16_t* gate, int B, int S, int T, int hq, int kv_heads, int head_dim, uint16_t* out,
                     float* po, float* pst, void* workspace, size_t workspace_bytes, qk_stream_t stream) {
  QK_REQUIRE(B >= 0 && S > 0 && T > 0 && hq > 0 && kv_heads > 0, "invalid attention geometry");
  QK_REQUIRE(hq % kv_heads == 0, "Head counts must have integer repetition factors");
  QK_REQUIRE(hq / kv_heads <= kHeads, "at most %d query heads per KV head", kHeads);
  QK_REQUIRE(head_dim == 128 || head_dim == 256, "head_dim must be 128 or 256");
  QK_REQUIRE(valid || lengths, "either valid or lengths is required");
  if (B == 0) return QK_OK;
  QK_REQUIRE(q && k_codes && v_codes && k_scale && v_scale && indices && (po ? pst != nullptr : out != nullptr),
             "null pointer");
  QK_REQUIRE((reinterpret_cast<uintptr_t>(k_codes) & 15) == 0 && (reinterpret_cast<uintptr_t>(v_codes) & 15) == 0,
             "K/V code planes must be 16-byte aligned");
  QK_REQUIRE(static_cast<long long>(B) * T < (1ll << 31) && static_cast<long long>(B) * S < (1ll << 31),
             "B * T and B * S must stay below 2^31");
  AttnArgs a{};
  a.q = q; a.k_codes = k_codes; a.v_codes = v_codes; a.k_scale = k_scale; a.v_scale = v_scale;
  a.indices = indices; a.valid = valid; a.lengths = valid ? nullptr : lengths; a.gate = gate; a.out = out;
  a.po = po; a.pst = pst;
  a.B = B; a.S = S; a.T = T; a.hq = hq; a.kv = kv_heads; a.r = hq / kv_heads;
  a.kg = heads_per_unit(kv_heads, head_dim);
  a.rows = kUnitRows / a.kg;
  a.groups = kv_heads / a.kg;
  a.nch = (S + a.rows - 1) / a.rows;
  a.units = units_for(B, S, kv_heads, head_dim);
  a.ctas = choose_ctas(a.units);
  a.idx16 = (S % 4) == 0 && (reinterpret_cast<uintptr_t>(indices) & 15) == 0;
  a.flag16 = a.idx16 && valid && (S % 16) == 0 && (reinterpret_cast<uintptr_t>(valid) & 15) == 0;
  a.div = sqrtf(static_cast<float>(head_dim));

  CUtensorMap maps[4];
  memset(maps, 0, sizeof(maps));
  const uint64_t nrows = static_cast<uint64_t>(B) * T, width = static_cast<uint64_t>(kv_heads) * head_dim;
  const uint32_t nblk = static_cast<uint32_t>(a.kg * head_dim / kBox);  // column blocks of a unit row
  a.code3d = encode_blocks_3d(&maps[0], k_codes, width, nrows, a.rows, nblk) &&
             encode_blocks_3d(&maps[1], v_codes, width, nrows, a.rows, nblk);
  a.tma_codes = a.code3d ||
                (encode_2d(&maps[0], k_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, width, nrows, width, kBox, a.rows,
                           CU_TENSOR_MAP_SWIZZLE_128B) &&
                 encode_2d(&maps[1], v_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, width, nrows, width, kBox, a.rows,
                           CU_TENSOR_MAP_SWIZZLE_128B));
  const uint64_t planes = static_cast<uint64_t>(B) * kv_heads * (head_dim / 32);
  // scale boxes: rows + 8 times (the padded plane pitch; times past T read as zero) x kg * groups
  const uint32_t scale_rows = static_cast<uint32_t>(a.kg * (head_dim / 32));
  a.tma_scales = a.tma_codes && (T % 8) == 0 && (reinterpret_cast<uintptr_t>(k_scale) & 15) == 0 &&
                 (reinterpret_cast<uintptr_t>(v_scale) & 15) == 0 &&
                 encode_2d(&maps[2], k_scale, CU_TENSOR_MAP_DATA_TYPE_UINT16, T, planes,
                           static_cast<uint64_t>(T) * 2, a.rows + 8, scale_rows, CU_TENSOR_MAP_SWIZZLE_NONE) &&
                 encode_2d(&maps[3], v_scale, CU_TENSOR_MAP_DATA_TYPE_UINT16, T, planes,
                           static_cast<uint64_t>(T) * 2, a.rows + 8, scale_rows, CU_TENSOR_MAP_SWIZZLE_NONE);

  if (a.ctas > 1) {
    const size_t need = workspace_for(B, S, kv_heads, head_dim);
    if (!workspace || workspace_bytes < need)
      return set_error(QK_ERR_WORKSPACE, "attention workspace needs %zu bytes, got %zu", need, workspace_bytes);
    QK_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 15) == 0, "workspace must be 16-byte aligned");
    a.part = static_cast<float*>(workspace);
  }
  cudaStream_t st = as_stream(stream);
  const size_t smem = head_dim == 256 ? Geo<256>::smem(a.kg) : Geo<128>::smem(a.kg);
  const void* kern = head_dim == 256 ? reinterpret_cast<const void*>(attn_stream_kernel<256>)
                                     : reinterpret_cast<const void*>(attn_stream_kernel<128>);
  if (int rc = allow_smem(kern, smem)) return rc;
  // the consumers' setmaxnreg.inc waits until the producers' registers are free: launch only
  // with at least the registers the split adds up to (it would wait for ever otherwise)
  static int regs[2] = {-1, -1};
  int& nregs = regs[head_dim == 256 ? 1 : 0];
  if (nregs < 0) {
    cudaFuncAttributes attr{};
    const cudaError_t e = cudaFuncGetAttributes(&attr, kern);
    if (e != cudaSuccess) return cuda_error(e, "attn_stream_kernel attributes");
    nregs = attr.numRegs;
  }
  if (nregs < kLaunchRegs)
    return set_error(QK_ERR_CUDA, "attention kernel built with %d registers per thread, the split needs %d",
                     nregs, kLaunchRegs);
  {
    const cudaError_t e =
        head_dim == 256
            ? launch_dependent(attn_stream_kernel<256>, dim3(a.ctas), dim3(kThreads), smem, st, maps[0], maps[1], maps[2],
                               maps[3], a)
            : launch_dependent(attn_stream_kernel<128>, dim3(a.ctas), dim3(kThreads), smem, st, maps[0], maps[1], maps[2],
                               maps[3], a);
    if (e != cudaSuccess) return cuda_error(e, "attn_stream_kernel");
    count_launch();
  }
  if (a.ctas > 1) {
    // partials per cut segment: about nch / (units / ctas) + 1; wider merges split d further
    const long long per = a.units / a.ctas;
    const long long n = (a.nch + per - 1) / per + 1;
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

}  // namespace

extern "C" {

int qk_kv_q8_decode_attention(const uint16_t* q, const int8_t* k_codes, const int8_t* v_codes,
                              const uint16_t* k_scale, const uint16_t* v_scale,
                              const int32_t* indices, const uint8_t* valid, const int32_t* lengths,
                              const uint16_t* gate, int B, int S, int T, int hq, int kv_heads,
                              int head_dim, uint16_t* out, void* workspace, size_t workspace_bytes,
                              qk_stream_t stream) {
  return launch_attention(q, k_codes, v_codes, k_scale, v_scale, indices, valid, lengths, gate, B, S, T, hq,
                          kv_heads, head_dim, out, nullptr, nullptr, workspace, workspace_bytes, stream);
}

int qk_kv_q8_decode_attention_partial(const uint16_t* q, const int8_t* k_codes, const int8_t* v_codes,
                                      const uint16_t* k_scale, const uint16_t* v_scale,
                                      const int32_t* indices, const uint8_t* valid,
                                      const int32_t* lengths, int B, int S, int T, int hq,
                                      int kv_heads, int head_dim, float* partial, void* workspace,
                                      size_t workspace_bytes, qk_stream_t stream) {
  QK_REQUIRE(partial, "partial is required");
  QK_REQUIRE((reinterpret_cast<uintptr_t>(partial) & 15) == 0, "partial must be 16-byte aligned");
  float* stats = partial + static_cast<int64_t>(B) * hq * head_dim;
  return launch_attention(q, k_codes, v_codes, k_scale, v_scale, indices, valid, lengths, nullptr, B, S, T, hq,
                          kv_heads, head_dim, nullptr, partial, stats, workspace, workspace_bytes, stream);
}

int qk_kv_q8_attention_combine(const float* parts, int R, int B, int hq, int head_dim, const uint16_t* gate,
                               uint16_t* out, qk_stream_t stream) {
  QK_REQUIRE(R > 0 && B >= 0 && hq > 0 && head_dim > 0, "invalid combine geometry");
  if (B == 0) return QK_OK;
  QK_REQUIRE(parts && out, "null pointer");
  const long long rows = static_cast<long long>(B) * hq;
  QK_REQUIRE(rows < (1ll << 31), "B * hq must stay below 2^31");
  cudaStream_t st = as_stream(stream);
  attn_combine_kernel<<<static_cast<unsigned>(rows), 256, 0, st>>>(parts, R, rows, head_dim, gate, out);
  QK_LAUNCHED("attn_combine_kernel");
  return QK_OK;
}

}  // extern "C"
