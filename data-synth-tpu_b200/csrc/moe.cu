// Routed-expert SwiGLU FFN over tiled Q6_K / Q4_K expert weights (decode regime).
//
// Replaces the routed FFN of qwen38_tpu/experts.py:61-131 (and grouped_experts.py:185-292
// at tp = 1) for the experts one rank holds. Five launches on one stream:
//
//  1. route    - one CTA turns ids/weights [B, k] into per-expert entry lists (expert-
//                sorted), merging duplicate routes of a token into one entry whose weight
//                is bf16(sum) (experts.py:66-73) and dropping zero-weight routes (their
//                contribution is zero in the reference, experts.py:74-76); it also lays
//                out the token chunks (<= 64 entries of one expert) of the next passes.
//  2. dispatch - copies each entry's x row into the activation tiles of its chunk (BF16,
//                128-byte-swizzled K-major: the tensor core's shared-memory operand layout).
//  3. gate/up  - tcgen05 pass (umma_proj.cuh): per (chunk, 64 rows of I), gate and up
//                rows decoded into one 128-lane TMEM operand, FP32 accumulators; epilogue
//                h = bf16(silu(bf16(x Wg^T)) * bf16(x Wu^T)) (experts.py:103-107,
//                math.py:10-20) written as the activation tiles of the down pass.
//  4. down     - tcgen05 pass, per (chunk, 128 rows of H): y = bf16(h Wd^T).
//  5. combine  - per token, FP32 sum of f32(y) * f32(route) over its experts in ascending
//                expert order (the reference's accumulation order, experts.py:129), then
//                BF16 (experts.py:131), or the FP32 partial sum for an EP all-reduce.
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "ep_p2p.cuh"
#include "umma_i8.cuh"
#include "umma_prefill.cuh"
#include "umma_proj.cuh"

namespace qk {
namespace {

struct MoeMeta {
  int32_t n_active;
  int32_t n_entries;
  int32_t status;
  int32_t n_chunks;
  int32_t row_total;
  int32_t reserved[3];
};

struct Workspace {
  MoeMeta* meta;
  int32_t* counts;        // [E]
  int32_t* offsets;       // [E + 1]
  int32_t* active;        // [E]   active expert ids (local), ascending
  int32_t* chunk_off;     // [E + 1] first chunk of each active slot
  int4* chunk_rec;        // [chunks_max] per chunk: {expert, tokens, first entry, first tile row}
  int32_t* row_off;       // [E + 1] first activation-tile row of each active slot
  int32_t* entry_token;   // [B k] token of each entry (expert-sorted)
  float* entry_weight;    // [B k] bf16-valued route weight of each entry
  int32_t* route_entry;   // [B k] entry of route (b, j), -1 if none
  int32_t* entry_route;   // [B k] route b * k + j that owns each entry
  uint8_t* xt;            // gate/up activation tiles [rows_max x H bf16]
  uint8_t* ht;            // down activation tiles [rows_max x I bf16]
  uint16_t* y;            // [B k, H]
  int32_t* hist;          // [kRouteCtas][E] entries per (route CTA, expert), many-route calls only
  int8_t* qx;             // int8_q8 down: activation codes [rows_max x I] (W8A8 calls only)
  float* qs;              // int8_q8 down: activation scales [rows_max x I / 32]
};

inline size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

constexpr int kStagedRoutes = 4096;
// Above this many routes the metadata is built by three kernels over many CTAs (count,
// tables, place) instead of one CTA.
constexpr int kManyRoutes = 16384;
constexpr int kRouteCtas = 256;         // CTAs of the count / place kernels at most
constexpr int kRouteThreads = 512;

// Activation-tile rows: each active expert's entries rounded up to 16 per chunk.
// Token chunks: each active expert's entries in runs of kMaxTok (or of kWideTok; the
// narrow chunks bound both).
inline size_t chunks_bound(const qk_moe_desc& d, int max_tokens) {
  const size_t R = static_cast<size_t>(max_tokens) * d.top_k;
  const size_t E = static_cast<size_t>(d.num_experts);
  return (R + kMaxTok - 1) / kMaxTok + (E < R ? E : R);
}

inline size_t rows_bound(const qk_moe_desc& d, int max_tokens) {
  const size_t R = static_cast<size_t>(max_tokens) * d.top_k;
  const size_t E = static_cast<size_t>(d.num_experts);
  return R + 15 * (E < R ? E : R);
}

size_t layout(const qk_moe_desc& d, int max_tokens, uint8_t* base, Workspace* ws) {
  const size_t E = d.num_experts, R = static_cast<size_t>(max_tokens) * d.top_k;
  const size_t rows = rows_bound(d, max_tokens);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    uint8_t* p = base ? base + off : nullptr;
    off += align256(bytes);
    return p;
  };
  uint8_t* meta = take(sizeof(MoeMeta));
  uint8_t* counts = take(E * 4);
  uint8_t* offsets = take((E + 1) * 4);
  uint8_t* active = take(E * 4);
  uint8_t* chunk_off = take((E + 1) * 4);
  uint8_t* chunk_rec = take(chunks_bound(d, max_tokens) * sizeof(int4));
  uint8_t* row_off = take((E + 1) * 4);
  uint8_t* et = take(R * 4);
  uint8_t* ew = take(R * 4);
  uint8_t* re = take(R * 4);
  uint8_t* er = take(R * 4);
  uint8_t* xt = take(rows * d.hidden * 2);
  uint8_t* ht = take(rows * ((d.intermediate + 255) / 256 * 256) * 2);  // whole 256-value K blocks
  uint8_t* y = take(R * d.hidden * 2);
  uint8_t* hist = take(R > kManyRoutes ? kRouteCtas * E * 4 : 0);
  const bool w8a8 = d.compute == QK_COMPUTE_INT8_Q8 && d.down_type == QK_TYPE_Q8_0;
  const size_t ipad = (d.intermediate + 255) / 256 * 256;
  uint8_t* qx = take(w8a8 ? rows * ipad : 0);
  uint8_t* qs = take(w8a8 ? rows * (ipad / 32) * 4 : 0);
  if (ws) {
    ws->meta = reinterpret_cast<MoeMeta*>(meta);
    ws->counts = reinterpret_cast<int32_t*>(counts);
    ws->offsets = reinterpret_cast<int32_t*>(offsets);
    ws->active = reinterpret_cast<int32_t*>(active);
    ws->chunk_off = reinterpret_cast<int32_t*>(chunk_off);
    ws->chunk_rec = reinterpret_cast<int4*>(chunk_rec);
    ws->row_off = reinterpret_cast<int32_t*>(row_off);
    ws->entry_token = reinterpret_cast<int32_t*>(et);
    ws->entry_weight = reinterpret_cast<float*>(ew);
    ws->route_entry = reinterpret_cast<int32_t*>(re);
    ws->entry_route = reinterpret_cast<int32_t*>(er);
    ws->xt = xt;
    ws->ht = ht;
    ws->y = reinterpret_cast<uint16_t*>(y);
    ws->hist = reinterpret_cast<int32_t*>(hist);
    ws->qx = reinterpret_cast<int8_t*>(qx);
    ws->qs = reinterpret_cast<float*>(qs);
  }
  return off;
}

// ------------------------------------------------------------------------------------
// 1. routing metadata
// ------------------------------------------------------------------------------------

// Route (b, j)'s entry: the first slot j of a token that names local expert e owns the
// merged entry; its weight is bf16 of the FP32 sum over all slots naming e, in slot order
// (experts.py:66-73). Zero-weight entries are dropped (experts.py:74-76). Returns the local
// expert, or -1 when the route owns no entry.
__device__ __forceinline__ int route_owner(const int32_t* ids, const uint16_t* weights, int b, int j, int k, int E,
                                           int first, float& w) {
  const int e = ids[b * k + j] - first;
  int own = e >= 0 && e < E;
  for (int jj = 0; own && jj < j; ++jj) own = ids[b * k + jj] - first != e;
  w = 0.f;
  if (own) {
    for (int jj = j; jj < k; ++jj)
      if (ids[b * k + jj] - first == e) w = __fadd_rn(w, bf16_to_f32(weights[b * k + jj]));
    w = bf16_round(w);
    own = w != 0.f;
  }
  return own ? e : -1;
}

// The tables every later pass reads, from the entry counts per expert (`counts`, shared
// memory, [E]): exclusive offsets (`offsets`, shared memory, [E + 1], and ws.offsets),
// ws.counts, the ascending active-expert list, and the token chunks (<= ctok entries of
// one expert) with their activation-tile rows (each chunk padded to a multiple of 16 rows)
// and one record per chunk. Run by a whole CTA: warp 0 scans into shared memory (`tab`,
// [3 E + 2] ints: active list, chunk offsets, row offsets), then every thread copies the
// tables out and writes the chunk records, so no thread waits on a global read.
__device__ void route_tables(const int32_t* counts, int32_t* offsets, int32_t* tab, int E, int ctok,
                             const Workspace& ws) {
  __shared__ int32_t base[2][33], n_act_sh;
  int32_t* active = tab;                // [E]
  int32_t* chunk_off = tab + E;         // [E + 1]
  int32_t* row_off = tab + 2 * E + 1;   // [E + 1]
  const int tid = threadIdx.x, nt = blockDim.x;
  if (tid < 32) {
    const int per = (E + 31) / 32, lo = min(E, tid * per), hi = min(E, lo + per);
    int sum = 0, act = 0;
    for (int e = lo; e < hi; ++e) {
      sum += counts[e];
      act += counts[e] > 0;
    }
    int incl = sum, iact = act;
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o), a = __shfl_up_sync(0xffffffffu, iact, o);
      if (tid >= o) {
        incl += v;
        iact += a;
      }
    }
    int run = incl - sum, arun = iact - act;
    for (int e = lo; e < hi; ++e) {
      offsets[e] = run;
      run += counts[e];
      if (counts[e] > 0) active[arun++] = e;
    }
    const int total = __shfl_sync(0xffffffffu, incl, 31), n_act = __shfl_sync(0xffffffffu, iact, 31);
    if (tid == 31) {
      offsets[E] = total;
      n_act_sh = n_act;
      ws.meta->n_entries = total;
      ws.meta->n_active = n_act;
      ws.meta->status = 0;
    }
    __syncwarp();
    const int per2 = (n_act + 31) / 32, lo2 = min(n_act, tid * per2), hi2 = min(n_act, lo2 + per2);
    int ch_sum = 0, row_sum = 0;
    for (int a = lo2; a < hi2; ++a) {
      const int m = counts[active[a]], nch = (m + ctok - 1) / ctok;
      ch_sum += nch;
      row_sum += ctok * (nch - 1) + (((m - ctok * (nch - 1)) + 15) & ~15);
    }
    int ch_incl = ch_sum, row_incl = row_sum;
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, ch_incl, o), w = __shfl_up_sync(0xffffffffu, row_incl, o);
      if (tid >= o) {
        ch_incl += v;
        row_incl += w;
      }
    }
    int cb = ch_incl - ch_sum, rb = row_incl - row_sum;
    for (int a = lo2; a < hi2; ++a) {
      const int m = counts[active[a]], nch = (m + ctok - 1) / ctok;
      chunk_off[a] = cb;
      row_off[a] = rb;
      cb += nch;
      rb += ctok * (nch - 1) + (((m - ctok * (nch - 1)) + 15) & ~15);
    }
    if (tid == 31) {
      chunk_off[n_act] = ch_incl;
      row_off[n_act] = row_incl;
      ws.meta->n_chunks = ch_incl;
      ws.meta->row_total = row_incl;
    }
  }
  __syncthreads();

  // Copies of the tables for the later passes, and one record per token chunk (the
  // tensor-core passes read one record per chunk instead of searching the chunk tables).
  const int n_act = n_act_sh;
  for (int e = tid; e <= E; e += nt) {
    ws.offsets[e] = offsets[e];
    if (e < E) ws.counts[e] = counts[e];
  }
  for (int a = tid; a <= n_act; a += nt) {
    ws.chunk_off[a] = chunk_off[a];
    ws.row_off[a] = row_off[a];
    if (a == n_act) break;
    const int e = active[a], m = counts[e], nch = (m + ctok - 1) / ctok;
    ws.active[a] = e;
    const int c0 = chunk_off[a], r0 = row_off[a], e0 = offsets[e];
    for (int ch = 0; ch < nch; ++ch)
      ws.chunk_rec[c0 + ch] = make_int4(e, min(ctok, m - ctok * ch), e0 + ctok * ch, r0 + ctok * ch);
  }
}

// One CTA builds everything (B * k <= kManyRoutes).
__global__ void __launch_bounds__(1024) moe_route_kernel(const int32_t* ids, const uint16_t* weights,
                                                         int B, int k, int E, int first, int ctok,
                                                         Workspace ws) {
  extern __shared__ int32_t sh[];
  pdl_wait();     // launched as a programmatic dependent: the routes' producer first
  pdl_trigger();  // the dispatch may launch now (it waits for this kernel before reading)
  int32_t* counts = sh;            // [E]
  int32_t* cursor = sh + E;        // [E]
  int32_t* offsets = sh + 2 * E;   // [E + 1]
  int32_t* tab = sh + 3 * E + 1;   // [3 E + 2] route_tables' scratch
  const int tid = threadIdx.x, nt = blockDim.x;
  // The routes staged in shared memory when they fit (kStagedRoutes): both passes read
  // every route of a token k times.
  const bool staged = B * k <= kStagedRoutes;
  int32_t* s_ids = sh + 6 * E + 3;                                                   // [B k]
  uint16_t* s_w = reinterpret_cast<uint16_t*>(s_ids + (staged ? B * k : 0));          // [B k]
  for (int e = tid; e < E; e += nt) counts[e] = cursor[e] = 0;
  if (staged) {
    for (int i = tid; i < B * k; i += nt) {
      s_ids[i] = ids[i];
      s_w[i] = weights[i];
    }
    ids = s_ids;
    weights = s_w;
  }
  __syncthreads();

  // Pass 1: entries per expert, one thread per route (b, j).
  for (int route = tid; route < B * k; route += nt) {
    const int b = route / k, j = route - b * k;
    float w;
    const int e = route_owner(ids, weights, b, j, k, E, first, w);
    if (e >= 0) atomicAdd(&counts[e], 1);
  }
  __syncthreads();
  route_tables(counts, offsets, tab, E, ctok, ws);

  // Pass 2: place entries (one thread per route).
  for (int route = tid; route < B * k; route += nt) {
    const int b = route / k, j = route - b * k;
    float w;
    const int e = route_owner(ids, weights, b, j, k, E, first, w);
    int slot = -1;
    if (e >= 0) {
      slot = offsets[e] + atomicAdd(&cursor[e], 1);
      ws.entry_token[slot] = b;
      ws.entry_weight[slot] = w;
      ws.entry_route[slot] = b * k + j;
    }
    ws.route_entry[b * k + j] = slot;
  }
}

// Many routes (B * k > kManyRoutes): CTA g of the count and place kernels takes the tokens
// [g B / G, (g + 1) B / G). The count kernel writes the CTA's entries per expert to
// ws.hist[g][E]; the tables kernel turns each expert's column into exclusive prefixes over
// the CTAs and builds the tables from the column sums; the place kernel puts CTA g's
// entries of expert e at offsets[e] + hist[g][e] onwards. Inside one CTA the order of an
// expert's entries is free (each entry is one independent token column of the projections).
__global__ void __launch_bounds__(kRouteThreads) moe_route_count_kernel(const int32_t* ids, const uint16_t* weights,
                                                                        int B, int k, int E, int first, Workspace ws) {
  extern __shared__ int32_t sh[];  // [E]
  pdl_wait();
  pdl_trigger();
  const int G = gridDim.x, g = blockIdx.x;
  for (int e = threadIdx.x; e < E; e += blockDim.x) sh[e] = 0;
  __syncthreads();
  const int b0 = static_cast<int>(static_cast<int64_t>(g) * B / G), b1 = static_cast<int>(static_cast<int64_t>(g + 1) * B / G);
  for (int route = b0 * k + threadIdx.x; route < b1 * k; route += blockDim.x) {
    const int b = route / k, j = route - b * k;
    float w;
    const int e = route_owner(ids, weights, b, j, k, E, first, w);
    if (e >= 0) atomicAdd(&sh[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) ws.hist[static_cast<int64_t>(g) * E + e] = sh[e];
}

__global__ void __launch_bounds__(1024) moe_route_tables_kernel(int G, int E, int ctok, Workspace ws) {
  extern __shared__ int32_t sh[];
  int32_t* counts = sh;       // [E]
  int32_t* offsets = sh + E;  // [E + 1]
  int32_t* tab = sh + 2 * E + 1;  // [3 E + 2]
  pdl_wait();
  pdl_trigger();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int g = 0; g < G; ++g) {
      const int64_t i = static_cast<int64_t>(g) * E + e;
      const int v = ws.hist[i];
      ws.hist[i] = run;
      run += v;
    }
    counts[e] = run;
  }
  __syncthreads();
  route_tables(counts, offsets, tab, E, ctok, ws);
}

__global__ void __launch_bounds__(kRouteThreads) moe_route_place_kernel(const int32_t* ids, const uint16_t* weights,
                                                                        int B, int k, int E, int first, Workspace ws) {
  extern __shared__ int32_t sh[];  // [E] next slot of each expert
  pdl_wait();
  pdl_trigger();
  const int G = gridDim.x, g = blockIdx.x;
  for (int e = threadIdx.x; e < E; e += blockDim.x) sh[e] = ws.offsets[e] + ws.hist[static_cast<int64_t>(g) * E + e];
  __syncthreads();
  const int b0 = static_cast<int>(static_cast<int64_t>(g) * B / G), b1 = static_cast<int>(static_cast<int64_t>(g + 1) * B / G);
  for (int route = b0 * k + threadIdx.x; route < b1 * k; route += blockDim.x) {
    const int b = route / k, j = route - b * k;
    float w;
    const int e = route_owner(ids, weights, b, j, k, E, first, w);
    int slot = -1;
    if (e >= 0) {
      slot = atomicAdd(&sh[e], 1);
      ws.entry_token[slot] = b;
      ws.entry_weight[slot] = w;
      ws.entry_route[slot] = b * k + j;
    }
    ws.route_entry[b * k + j] = slot;
  }
}

// ------------------------------------------------------------------------------------
// 2. dispatch: x rows of every chunk into the swizzled activation tiles (zero padding rows)
// ------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) moe_dispatch_kernel(const uint16_t* __restrict__ x, int H, int ctok,
                                                           Workspace ws) {
  // One warp per (token chunk, tile row): the chunk's record gives the row's place; the
  // lanes load the row's 16-byte pieces (H / 8 of them) eight at a time before storing them
  // into the swizzled tile. Rows past the chunk's tokens (up to the 16-row padding) are zero.
  constexpr int kU = 8;
  pdl_wait();
  const int n_rows = ws.meta->n_chunks * ctok;
  const int lane = threadIdx.x & 31, cpr = H / 8, nkb = H / 256;
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int g = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); g < n_rows; g += warps) {
    const int ci = g / ctok, rr = g % ctok;
    const int4 rec = ws.chunk_rec[ci];  // {expert, tokens, first entry, first tile row}
    const int ntok = rec.y, r16 = (ntok + 15) & ~15;
    if (rr >= r16) continue;
    const uint16_t* src = rr < ntok ? x + static_cast<int64_t>(ws.entry_token[rec.z + rr]) * H : nullptr;
    uint8_t* base = ws.xt + static_cast<int64_t>(rec.w) * 512 * nkb;
    for (int j0 = lane; j0 < cpr; j0 += 32 * kU) {
      uint4 v[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int j = j0 + 32 * u;
        v[u] = src && j < cpr ? ld_nc_v4(src + j * 8) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int j = j0 + 32 * u, k = j * 8;
        if (j < cpr)
          *reinterpret_cast<uint4*>(base + static_cast<int64_t>(k >> 8) * r16 * 512 + xt_offset(r16, rr, k & 255)) = v[u];
      }
    }
  }
  // Only now may the projection be launched: its CTAs take a whole SM each and would
  // otherwise crowd out the rest of this grid.
  pdl_trigger();
}

// ------------------------------------------------------------------------------------
// 5. combine
// ------------------------------------------------------------------------------------
constexpr int kMaxTopK = 32;

// One warp per (token, group of KG 256-column blocks): lane j < k holds route j's entry, and
// its rank among the token's entries by expert id gives the reference's ascending-expert
// accumulation order (experts.py:129); lane i then learns which lane holds rank i. Each lane
// owns 8 columns of each block of the group: for KR routes at a time it loads all KR x KG of
// its 16-byte pieces before adding them, in rank order, into FP32 sums, so the loads of a warp
// are in flight together. Many tokens: KG = 4, KR = 2 (the route metadata is read twice per
// token at H = 2048); few tokens (a decode batch): KG = 1, KR = 8, so the warps of a small
// batch are eight times as many and each waits for fewer rounds of loads. The sums do not
// depend on KG or KR.
// With `yr` (tensor parallel: the FP32 down projection of each route, summed over the tensor
// ranks) the expert output of route (b, j) is bf16(yr[b * k + j]) (grouped_experts.py:
// 113-119: psum before the BF16 rounding); otherwise the entry's BF16 y.
template <int kG, int kR>
__global__ void __launch_bounds__(256) moe_combine_kernel(const int32_t* __restrict__ ids, int B,
                                                          int k, int H, int out_bf16, void* out,
                                                          const float* __restrict__ yr, Workspace ws) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int blocks = H / 256, ngroups = (blocks + kG - 1) / kG;
  const int wi_ = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (wi_ >= B * ngroups) return;
  const int b = wi_ / ngroups, g0 = (wi_ - b * ngroups) * kG;
  const int entry = lane < k ? ws.route_entry[b * k + lane] : -1;
  const int eid = entry >= 0 ? ids[b * k + lane] : 0x7fffffff;
  const float w = entry >= 0 ? ws.entry_weight[entry] : 0.f;
  int rank = 0, n = 0, src_of_rank = 0;
  for (int j = 0; j < k; ++j) {
    const int ej = __shfl_sync(0xffffffffu, eid, j);
    const int vj = __shfl_sync(0xffffffffu, entry, j) >= 0;
    n += vj;
    rank += vj && (ej < eid);  // entries of a token name distinct experts
  }
  for (int j = 0; j < k; ++j) {
    const int rj = __shfl_sync(0xffffffffu, rank, j);
    const int vj = __shfl_sync(0xffffffffu, entry, j) >= 0;
    if (vj && rj == lane) src_of_rank = j;
  }
  {
    float acc[kG][8];
#pragma unroll
    for (int q = 0; q < kG; ++q)
#pragma unroll
      for (int t = 0; t < 8; ++t) acc[q][t] = 0.f;
    for (int i0 = 0; i0 < n; i0 += kR) {
      uint4 v[kR][kG];
      float wi[kR];
#pragma unroll
      for (int u = 0; u < kR; ++u) {
        const int i = i0 + u;
        const int src = __shfl_sync(0xffffffffu, src_of_rank, i < n ? i : 0);
        const int ent = __shfl_sync(0xffffffffu, entry, src);
        wi[u] = __shfl_sync(0xffffffffu, w, src);
#pragma unroll
        for (int q = 0; q < kG; ++q) {
          v[u][q] = make_uint4(0, 0, 0, 0);
          const int c0 = (g0 + q) * 256 + lane * 8;
          if (i >= n || g0 + q >= blocks) continue;
          if (yr) {
            const float* f = yr + (static_cast<int64_t>(b) * k + src) * H + c0;
            const float4 f0 = *reinterpret_cast<const float4*>(f), f1 = *reinterpret_cast<const float4*>(f + 4);
            v[u][q] = make_uint4(bf16_bits_rne(f0.x) | (static_cast<uint32_t>(bf16_bits_rne(f0.y)) << 16),
                                 bf16_bits_rne(f0.z) | (static_cast<uint32_t>(bf16_bits_rne(f0.w)) << 16),
                                 bf16_bits_rne(f1.x) | (static_cast<uint32_t>(bf16_bits_rne(f1.y)) << 16),
                                 bf16_bits_rne(f1.z) | (static_cast<uint32_t>(bf16_bits_rne(f1.w)) << 16));
          } else {
            v[u][q] = ld_nc_v4(ws.y + static_cast<int64_t>(ent) * H + c0);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kR; ++u) {
        if (i0 + u >= n) break;
#pragma unroll
        for (int q = 0; q < kG; ++q) {
          const uint32_t p[4] = {v[u][q].x, v[u][q].y, v[u][q].z, v[u][q].w};
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            const float y = bf16_to_f32(static_cast<uint16_t>(p[t >> 1] >> (16 * (t & 1))));
            acc[q][t] = __fadd_rn(acc[q][t], __fmul_rn(y, wi[u]));
          }
        }
      }
    }
#pragma unroll
    for (int q = 0; q < kG; ++q) {
      if (g0 + q >= blocks) break;
      const int64_t o = static_cast<int64_t>(b) * H + (g0 + q) * 256 + lane * 8;
      if (out_bf16) {
        uint32_t r[4];
#pragma unroll
        for (int t = 0; t < 4; ++t)
          r[t] = static_cast<uint32_t>(bf16_bits_rne(acc[q][2 * t])) |
                 (static_cast<uint32_t>(bf16_bits_rne(acc[q][2 * t + 1])) << 16);
        *reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + o) = make_uint4(r[0], r[1], r[2], r[3]);
      } else {
        float4* f = reinterpret_cast<float4*>(static_cast<float*>(out) + o);
        f[0] = make_float4(acc[q][0], acc[q][1], acc[q][2], acc[q][3]);
        f[1] = make_float4(acc[q][4], acc[q][5], acc[q][6], acc[q][7]);
      }
    }
  }
}

// The combine's form: a warp per (token, 4 blocks) with 2 routes in flight for many tokens,
// a warp per (token, block) with 8 routes in flight for a decode batch.
template <typename... Args>
cudaError_t launch_combine(int B, int H, cudaStream_t st, Args... args) {
  const int blocks = H / 256;
  if (static_cast<int64_t>(B) * blocks <= 2048) {
    const int warps = B * blocks;
    return launch_dependent(moe_combine_kernel<1, 8>, dim3((warps + 7) / 8), dim3(256), 0, st, args...);
  }
  const int warps = B * ((blocks + 3) / 4);
  return launch_dependent(moe_combine_kernel<4, 2>, dim3((warps + 7) / 8), dim3(256), 0, st, args...);
}

__global__ void cast_kernel(const float* __restrict__ in, uint16_t* __restrict__ out, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = bf16_bits_rne(in[i]);
}

// Expert-parallel form of the combine (qk_ep_p2p_expert): the rows are the received slots
// [source s][token b] of this rank's exchange region. Each slot that its source sent (some
// route names one of this rank's experts) gets the FP32 sum of f32(y) * f32(route) over its
// entries in ascending expert order, stored straight into the source's region at
// ret[this rank][b] (over NVLink for another rank). Unsent slots are not written. The last
// CTA raises ret_flag[this rank] in every source's region.
__global__ void __launch_bounds__(512) moe_combine_push_kernel(const int32_t* __restrict__ ids, int Bp, int k, int H,
                                                               Workspace ws, uint8_t* const* __restrict__ peers,
                                                               uint8_t* own, EpLayout L, int rank) {
  pdl_wait();
  EpCtrl* ctrl = reinterpret_cast<EpCtrl*>(own);
  const uint32_t epoch = ctrl->epoch;
  const int lane = threadIdx.x & 31;
  const int blocks = H / 256;
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  // One CTA per SM walks all received slots, a warp per slot: the system-scope fence and the
  // arrival at the end of the kernel cost about as much per CTA as a slot's work, so the grid
  // is kept small. A warp reads the slot's route metadata once; then, per entry, its lanes
  // load all their 256-column pieces of the y row at once, so the loads are in flight
  // together before the FP32 partial is stored into the source's region.
  constexpr int kSplit = 1;  // warps per slot
  for (int gwi = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); gwi < Bp * kSplit; gwi += nwarps) {
    const int b = gwi / kSplit, part = gwi - b * kSplit;
    const int cb_lo = blocks * part / kSplit, cb_hi = blocks * (part + 1) / kSplit;
    const int id = lane < k ? ids[b * k + lane] : -1;
    if (!__any_sync(0xffffffffu, id >= 0)) continue;
    const int entry = lane < k ? ws.route_entry[b * k + lane] : -1;
    const int eid = entry >= 0 ? id : 0x7fffffff;
    const float w = entry >= 0 ? ws.entry_weight[entry] : 0.f;
    int rank_in = 0, n = 0;
    for (int j = 0; j < k; ++j) {
      const int ej = __shfl_sync(0xffffffffu, eid, j);
      const int vj = __shfl_sync(0xffffffffu, entry, j) >= 0;
      n += vj;
      rank_in += vj && (ej < eid);
    }
    const int src_rank = b / L.max_tokens, tok = b - src_rank * L.max_tokens;
    float* dst = reinterpret_cast<float*>(peers[src_rank] + L.ret) + (static_cast<size_t>(rank) * L.max_tokens + tok) * H;
    for (int cb0 = cb_lo; cb0 < cb_hi; cb0 += 8) {  // up to 8 pieces of 256 columns at a time
      float acc[8][8];
#pragma unroll
      for (int cc = 0; cc < 8; ++cc)
#pragma unroll
        for (int t = 0; t < 8; ++t) acc[cc][t] = 0.f;
      for (int i = 0; i < n; ++i) {
        const unsigned who = __ballot_sync(0xffffffffu, entry >= 0 && rank_in == i);
        const int src = __ffs(who) - 1;
        const int ent = __shfl_sync(0xffffffffu, entry, src);
        const float wi = __shfl_sync(0xffffffffu, w, src);
        uint4 v[8];
#pragma unroll
        for (int cc = 0; cc < 8; ++cc)
          if (cb0 + cc < cb_hi) v[cc] = ld_nc_v4(ws.y + static_cast<int64_t>(ent) * H + (cb0 + cc) * 256 + lane * 8);
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          if (cb0 + cc >= cb_hi) break;
          const uint32_t p[4] = {v[cc].x, v[cc].y, v[cc].z, v[cc].w};
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            const float y = bf16_to_f32(static_cast<uint16_t>(p[t >> 1] >> (16 * (t & 1))));
            acc[cc][t] = __fadd_rn(acc[cc][t], __fmul_rn(y, wi));
          }
        }
      }
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        if (cb0 + cc >= cb_hi) break;
        float4* o = reinterpret_cast<float4*>(dst + (cb0 + cc) * 256 + lane * 8);
        o[0] = make_float4(acc[cc][0], acc[cc][1], acc[cc][2], acc[cc][3]);
        o[1] = make_float4(acc[cc][4], acc[cc][5], acc[cc][6], acc[cc][7]);
      }
    }
  }
  if (ep_last_cta(&ctrl->combine_arrivals)) {
    for (int t = threadIdx.x; t < L.world; t += blockDim.x)
      ep_store_release(&reinterpret_cast<EpCtrl*>(peers[t])->ret_flag[rank], epoch);
  }
}

// Waits until every source has raised its recv_flag for this rank's current epoch.
__global__ void ep_wait_sources_kernel(uint8_t* own, int world) {
  EpCtrl* ctrl = reinterpret_cast<EpCtrl*>(own);
  const uint32_t epoch = ctrl->epoch;
  for (int t = threadIdx.x; t < world; t += blockDim.x)
    if (!ep_wait_flag(&ctrl->recv_flag[t], epoch)) atomicExch(&ctrl->status, QK_ERR_TIMEOUT);
  __syncthreads();
  pdl_trigger();
}

// Gate and up: Q6_K, Q4_K or Q5_K (the Q4 checkpoint's gate/up types, checkpoints/q4.json).
bool supported(int t) { return t == QK_TYPE_Q6_K || t == QK_TYPE_Q4_K || t == QK_TYPE_Q5_K; }
// Down: those k-quants but Q5_K, Q8_0 (the Q6 checkpoint's down type, checkpoints/q6.json) or
// Q5_1 (the Q4 checkpoint's, checkpoints/q4.json).
bool supported_down(int t) {
  return t == QK_TYPE_Q6_K || t == QK_TYPE_Q4_K || t == QK_TYPE_Q8_0 || t == QK_TYPE_Q5_1;
}

// One projection pass of `form` (0 narrow, 1 wide, 2 prefill) for weight type qtype.
template <int MODE>
int launch_pass(int qtype, int form, const UArgs& a, int sms, cudaStream_t st) {
  auto go = [&](auto q) -> int {
    constexpr QType Q = decltype(q)::value;
    if (form == 2) return launch_prefill<Q, MODE>(a, sms, st);
    if (form == 1) return launch_umma<Q, MODE, true>(a, sms, st);
    return launch_umma<Q, MODE>(a, sms, st);
  };
  switch (qtype) {
    case QK_TYPE_Q6_K: return go(std::integral_constant<QType, QType::Q6_K>{});
    case QK_TYPE_Q4_K: return go(std::integral_constant<QType, QType::Q4_K>{});
    case QK_TYPE_Q5_K:
      if constexpr (MODE == kModeGateUp) return go(std::integral_constant<QType, QType::Q5_K>{});
      break;
    case QK_TYPE_Q8_0:
      if constexpr (MODE == kModeDown) return go(std::integral_constant<QType, QType::Q8_0>{});
      break;
    case QK_TYPE_Q5_1:
      if constexpr (MODE == kModeDown) return go(std::integral_constant<QType, QType::Q5_1>{});
      break;
  }
  return set_error(QK_ERR_UNSUPPORTED_TYPE, "no projection pass for type %d", qtype);
}

// The int8_q8 down pass (umma_i8.cuh): `dn` carries the chunk tables and outputs of the BF16
// down pass it replaces.
int launch_w8a8_down(const qk_moe_desc& d, const UArgs& dn, const Workspace& ws, const uint8_t* down, int sms,
                     cudaStream_t st) {
  I8Args a{};
  a.ht = dn.xt;
  a.qx = ws.qx;
  a.qs = ws.qs;
  a.nkb = dn.nkb;
  a.ngroups = d.intermediate / 32;
  a.items_per_chunk = d.hidden / 128;
  a.tiles64 = dn.tiles64;
  a.n_chunks_p = dn.n_chunks_p;
  a.chunk_rec = dn.chunk_rec;
  a.y = dn.y;
  a.yr = dn.yr;
  a.entry_route = dn.entry_route;
  a.nrows = d.hidden;
  a.status = dn.status;
  return launch_w8a8(a, down, static_cast<int64_t>(d.num_experts) * dn.tiles64, sms, st);
}

}  // namespace
}  // namespace qk

using namespace qk;

extern "C" {

size_t qk_moe_workspace_bytes(const qk_moe_desc* desc, int max_tokens) {
  if (!desc || max_tokens < 0) return 0;
  return layout(*desc, max_tokens, nullptr, nullptr);
}

// phase kFull: all five launches; kPartial: route .. down with the FP32 down projection of
// every route written to `yr` [B * top_k, hidden] (no combine); kCombine: only the combine,
// from `yr` and the routing metadata a kPartial call left in the same workspace.
enum { kFull = 0, kPartial = 1, kCombine = 2, kPush = 3 };

// The exchange region of the expert-parallel form (phase kPush).
struct PushArgs {
  uint8_t* const* peers;
  uint8_t* own;
  EpLayout L;
  int rank;
};

static int moe_forward_impl(const qk_moe_desc* desc, const uint8_t* gate, const uint8_t* up,
                            const uint8_t* down, const uint16_t* x, const int32_t* ids,
                            const uint16_t* weights, int B, int out_dtype, void* out,
                            void* workspace, size_t workspace_bytes, qk_stream_t stream,
                            void* const* events, float* yr = nullptr, int phase = kFull,
                            const PushArgs* push = nullptr) {
  QK_REQUIRE(desc, "null descriptor");
  const qk_moe_desc& d = *desc;
  if (!supported(d.gate_type) || d.gate_type != d.up_type || !supported_down(d.down_type))
    return set_error(QK_ERR_UNSUPPORTED_TYPE,
                     "expert types: gate and up both Q6_K, Q4_K or Q5_K, down Q6_K, Q4_K, Q8_0 or Q5_1 (got %d/%d/%d)",
                     d.gate_type, d.up_type, d.down_type);
  QK_REQUIRE(d.hidden > 0 && d.hidden % 256 == 0, "hidden must be a positive multiple of 256");
  // The gate/up tiles zero-pad their rows to 64; the down projection reads whole GGUF blocks
  // of intermediate (256 values for the k-quants, 32 for Q8_0).
  const bool down32 = d.down_type == QK_TYPE_Q8_0 || d.down_type == QK_TYPE_Q5_1;  // 32-value blocks
  QK_REQUIRE(d.intermediate > 0 && d.intermediate % (down32 ? 32 : 256) == 0,
             "intermediate must be a positive multiple of the down type's block (256, or 32 for Q8_0 and Q5_1)");
  QK_REQUIRE(d.num_experts > 0 && d.num_experts <= 4096, "num_experts must be in [1, 4096]");
  QK_REQUIRE(d.top_k > 0 && d.top_k <= kMaxTopK, "top_k must be in [1, %d]", kMaxTopK);
  QK_REQUIRE(d.compute == QK_COMPUTE_BF16 || d.compute == QK_COMPUTE_INT8_Q8, "Unknown expert compute policy");
  QK_REQUIRE(B >= 0, "batch must be non-negative");
  QK_REQUIRE(out_dtype == QK_OUT_F32 || out_dtype == QK_OUT_BF16, "out_dtype must be F32 or BF16");
  if (B == 0) return QK_OK;
  if (phase == kCombine)
    QK_REQUIRE(ids && yr && out, "null pointer");
  else
    QK_REQUIRE(gate && up && down && x && ids && weights &&
                   (phase == kPartial ? yr != nullptr : phase == kPush ? push != nullptr : out != nullptr),
               "null pointer");
  if (yr) QK_REQUIRE((reinterpret_cast<uintptr_t>(yr) & 15) == 0, "y_routes must be 16-byte aligned");
  const size_t need = layout(d, B, nullptr, nullptr);
  if (!workspace || workspace_bytes < need)
    return set_error(QK_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", need, workspace_bytes);
  Workspace ws;
  layout(d, B, static_cast<uint8_t*>(workspace), &ws);
  cudaStream_t st = as_stream(stream);
  auto mark = [&](int i) {
    if (events && events[i]) cudaEventRecord(static_cast<cudaEvent_t>(events[i]), st);
  };

  if (phase == kCombine) {
    const cudaError_t e = launch_combine(B, d.hidden, st, ids, B, d.top_k,
                                           d.hidden, static_cast<int>(out_dtype == QK_OUT_BF16), out,
                                           static_cast<const float*>(yr), ws);
    if (e != cudaSuccess) return cuda_error(e, "moe_combine_kernel");
    count_launch(1);
    return QK_OK;
  }
  mark(0);
  if (d.intermediate % 256) {
    // The down pass reads whole 256-value K blocks of h; the padded channels must be zero
    // (their decoded weights are zero, and 0 * NaN would not be).
    const size_t bytes = rows_bound(d, B) * ((d.intermediate + 255) / 256 * 256) * 2;
    const cudaError_t e = cudaMemsetAsync(ws.ht, 0, bytes, st);
    if (e != cudaSuccess) return cuda_error(e, "clearing the padded activation tiles");
  }
  // The expert-parallel form receives [world x max_tokens] slots of which about max_tokens
  // carry routes for this rank when the experts are evenly loaded: the form follows that.
  const size_t routes = static_cast<size_t>(phase == kPush ? push->L.max_tokens : B) * d.top_k;
  // The wide form (128-token chunks) when the routes average at least 64 tokens per expert
  // the rank holds (prefill-sized batches); the narrow form (32-token chunks) otherwise.
#ifndef QK_WIDE_MIN_TOKENS
#define QK_WIDE_MIN_TOKENS 64
#endif
  // The prefill form (256-token chunks, each weight decoded once per 256 tokens into shared
  // memory, all of TMEM as accumulators) from QK_PREFILL_MIN_TOKENS routes per expert.
#ifndef QK_PREFILL_MIN_TOKENS
#define QK_PREFILL_MIN_TOKENS 192
#endif
  // The int8_q8 policy's W8A8 down pass takes token chunks of at most 32 (the narrow form).
  const bool w8a8 = d.compute == QK_COMPUTE_INT8_Q8 && d.down_type == QK_TYPE_Q8_0;
  const bool prefill = !w8a8 && routes >= QK_PREFILL_MIN_TOKENS * static_cast<size_t>(d.num_experts);
  const bool wide = !w8a8 && !prefill && routes >= QK_WIDE_MIN_TOKENS * static_cast<size_t>(d.num_experts);
  const int ctok = prefill ? kPTok : wide ? kWideTok : kMaxTok;
  const size_t all_routes = static_cast<size_t>(B) * d.top_k;
  const int E = d.num_experts;
  int rc;
  if (all_routes <= static_cast<size_t>(kManyRoutes)) {
    // one CTA; it stages all B * top_k routes in shared memory when they fit
    const size_t route_smem = (6 * static_cast<size_t>(E) + 3) * 4 + (all_routes <= kStagedRoutes ? all_routes * 6 : 0);
    rc = allow_smem(reinterpret_cast<const void*>(moe_route_kernel), route_smem);
    if (rc) return rc;
    const cudaError_t e = launch_dependent(moe_route_kernel, dim3(1), dim3(1024), route_smem, st, ids, weights, B,
                                           d.top_k, E, d.first_expert, ctok, ws);
    if (e != cudaSuccess) return cuda_error(e, "moe_route_kernel");
    count_launch(1);
  } else {
    // count, tables, place: about 4096 routes per CTA of the count and place kernels
    int G = static_cast<int>((all_routes + 4095) / 4096);
    if (G > kRouteCtas) G = kRouteCtas;
    if (G > B) G = B;
    const size_t hsmem = static_cast<size_t>(E) * 4, tsmem = (5 * static_cast<size_t>(E) + 3) * 4;
    rc = allow_smem(reinterpret_cast<const void*>(moe_route_count_kernel), hsmem);
    if (!rc) rc = allow_smem(reinterpret_cast<const void*>(moe_route_tables_kernel), tsmem);
    if (!rc) rc = allow_smem(reinterpret_cast<const void*>(moe_route_place_kernel), hsmem);
    if (rc) return rc;
    cudaError_t e = launch_dependent(moe_route_count_kernel, dim3(G), dim3(kRouteThreads), hsmem, st, ids, weights, B,
                                     d.top_k, E, d.first_expert, ws);
    if (e != cudaSuccess) return cuda_error(e, "moe_route_count_kernel");
    e = launch_dependent(moe_route_tables_kernel, dim3(1), dim3(1024), tsmem, st, G, E, ctok, ws);
    if (e != cudaSuccess) return cuda_error(e, "moe_route_tables_kernel");
    e = launch_dependent(moe_route_place_kernel, dim3(G), dim3(kRouteThreads), hsmem, st, ids, weights, B, d.top_k, E,
                         d.first_expert, ws);
    if (e != cudaSuccess) return cuda_error(e, "moe_route_place_kernel");
    count_launch(3);
  }

  const int sms = sm_count();
  const int64_t rows_max = static_cast<int64_t>(chunks_bound(d, B)) * kMaxTok;
  int64_t dgrid = (rows_max + 7) / 8;  // 8 rows (warps) per CTA
  if (dgrid > sms * 8) dgrid = sms * 8;
  {
    const cudaError_t e = launch_dependent(moe_dispatch_kernel, dim3(static_cast<unsigned>(dgrid)), dim3(256), 0, st,
                                           x, d.hidden, ctok, ws);
    if (e != cudaSuccess) return cuda_error(e, "moe_dispatch_kernel");
    count_launch(1);
  }

  UArgs gu{};
  gu.wa = gate;
  gu.wb = up;
  gu.expert_bytes = qk_tiled_bytes(d.gate_type, d.intermediate, d.hidden);
  gu.nkb = d.hidden / 256;
  gu.tiles64 = (d.intermediate + kTileRows - 1) / kTileRows;
  gu.items_per_chunk = gu.tiles64;  // 64 rows of I (gate + up) per MMA tile
  gu.xt = ws.xt;
  gu.n_chunks_p = &ws.meta->n_chunks;
  gu.chunk_off = ws.chunk_off;
  gu.chunk_rec = ws.chunk_rec;
  gu.row_off = ws.row_off;
  gu.active = ws.active;
  gu.counts = ws.counts;
  gu.offsets = ws.offsets;
  gu.n_active_p = &ws.meta->n_active;
  gu.ht = ws.ht;
  gu.nkb_out = (d.intermediate + 255) / 256;
  gu.nrows = d.intermediate;
  gu.status = &ws.meta->status;
  UArgs dn = gu;
  dn.wa = down;
  dn.wb = nullptr;
  dn.expert_bytes = qk_tiled_bytes(d.down_type, d.hidden, d.intermediate);
  dn.nkb = (d.intermediate + 255) / 256;
  dn.tiles64 = d.hidden / kTileRows;
  dn.items_per_chunk = d.hidden / (2 * kTileRows);
  dn.xt = ws.ht;
  dn.ht = nullptr;
  dn.y = ws.y;
  dn.yr = phase == kPartial ? yr : nullptr;
  dn.entry_route = ws.entry_route;
  dn.nrows = d.hidden;
  mark(1);
  const int form = prefill ? 2 : wide ? 1 : 0;
  if (prefill) {
    gu.items_per_chunk = (gu.tiles64 + 1) / 2;  // 128 rows of I (gate and up) per item
    dn.items_per_chunk = (dn.tiles64 + 3) / 4;  // 256 rows of H per item
  }
  rc = launch_pass<kModeGateUp>(d.gate_type, form, gu, sms, st);
  if (rc) return rc;
  mark(2);
  rc = w8a8 ? launch_w8a8_down(d, dn, ws, down, sms, st) : launch_pass<kModeDown>(d.down_type, form, dn, sms, st);
  if (rc) return rc;
  mark(3);
  if (phase == kPartial) return QK_OK;
  if (phase == kPush) {
    int64_t pgrid = (static_cast<int64_t>(B) + 15) / 16;
    if (pgrid > sms) pgrid = sms;
    const cudaError_t e = launch_dependent(moe_combine_push_kernel, dim3(static_cast<unsigned>(pgrid)), dim3(512), 0,
                                           st, ids, B, d.top_k, d.hidden, ws, push->peers, push->own, push->L,
                                           push->rank);
    if (e != cudaSuccess) return cuda_error(e, "moe_combine_push_kernel");
    count_launch(1);
    mark(4);
    return QK_OK;
  }
  {
    const cudaError_t e = launch_combine(B, d.hidden, st, ids, B, d.top_k,
                                           d.hidden, static_cast<int>(out_dtype == QK_OUT_BF16), out,
                                           static_cast<const float*>(nullptr), ws);
    if (e != cudaSuccess) return cuda_error(e, "moe_combine_kernel");
    count_launch(1);
  }
  mark(4);
  return QK_OK;
}

int qk_moe_forward(const qk_moe_desc* desc, const uint8_t* gate, const uint8_t* up,
                   const uint8_t* down, const uint16_t* x, const int32_t* ids,
                   const uint16_t* weights, int B, int out_dtype, void* out, void* workspace,
                   size_t workspace_bytes, qk_stream_t stream) {
  return moe_forward_impl(desc, gate, up, down, x, ids, weights, B, out_dtype, out, workspace,
                          workspace_bytes, stream, nullptr);
}

int qk_moe_forward_profiled(const qk_moe_desc* desc, const uint8_t* gate, const uint8_t* up,
                            const uint8_t* down, const uint16_t* x, const int32_t* ids,
                            const uint16_t* weights, int B, int out_dtype, void* out,
                            void* workspace, size_t workspace_bytes, qk_stream_t stream,
                            void* const* events) {
  return moe_forward_impl(desc, gate, up, down, x, ids, weights, B, out_dtype, out, workspace,
                          workspace_bytes, stream, events);
}

int qk_moe_forward_tp_partial(const qk_moe_desc* desc, const uint8_t* gate, const uint8_t* up,
                              const uint8_t* down, const uint16_t* x, const int32_t* ids,
                              const uint16_t* weights, int B, float* y_routes, void* workspace,
                              size_t workspace_bytes, qk_stream_t stream) {
  return moe_forward_impl(desc, gate, up, down, x, ids, weights, B, QK_OUT_F32, nullptr, workspace,
                          workspace_bytes, stream, nullptr, y_routes, kPartial);
}

int qk_moe_forward_tp_combine(const qk_moe_desc* desc, const float* y_routes, const int32_t* ids, int B,
                              int out_dtype, void* out, void* workspace, size_t workspace_bytes,
                              qk_stream_t stream) {
  return moe_forward_impl(desc, nullptr, nullptr, nullptr, nullptr, ids, nullptr, B, out_dtype, out, workspace,
                          workspace_bytes, stream, nullptr, const_cast<float*>(y_routes), kCombine);
}

static int ep_p2p_expert_impl(const qk_moe_desc* desc, const uint8_t* gate, const uint8_t* up, const uint8_t* down,
                              void* const* peers, void* region, int world, int rank, int max_tokens, void* workspace,
                              size_t workspace_bytes, qk_stream_t stream, void* const* events);

int qk_ep_p2p_expert(const qk_moe_desc* desc, const uint8_t* gate, const uint8_t* up, const uint8_t* down,
                     void* const* peers, void* region, int world, int rank, int max_tokens, void* workspace,
                     size_t workspace_bytes, qk_stream_t stream) {
  return ep_p2p_expert_impl(desc, gate, up, down, peers, region, world, rank, max_tokens, workspace,
                            workspace_bytes, stream, nullptr);
}

int qk_ep_p2p_expert_profiled(const qk_moe_desc* desc, const uint8_t* gate, const uint8_t* up,
                              const uint8_t* down, void* const* peers, void* region, int world, int rank,
                              int max_tokens, void* workspace, size_t workspace_bytes, qk_stream_t stream,
                              void* const* events) {
  return ep_p2p_expert_impl(desc, gate, up, down, peers, region, world, rank, max_tokens, workspace,
                            workspace_bytes, stream, events);
}

static int ep_p2p_expert_impl(const qk_moe_desc* desc, const uint8_t* gate, const uint8_t* up, const uint8_t* down,
                              void* const* peers, void* region, int world, int rank, int max_tokens, void* workspace,
                              size_t workspace_bytes, qk_stream_t stream, void* const* events) {
  QK_REQUIRE(desc && peers && region, "null pointer");
  QK_REQUIRE(world >= 1 && world <= kEpMaxRanks && rank >= 0 && rank < world, "bad rank or world");
  QK_REQUIRE(max_tokens >= 1, "max_tokens must be positive");
  QK_REQUIRE(desc->first_expert == rank * desc->num_experts,
             "first_expert must be rank * num_experts (contiguous expert ranges, parallel.py:64-87)");
  const EpLayout L = ep_layout(world, max_tokens, desc->hidden, desc->top_k);
  uint8_t* own = static_cast<uint8_t*>(region);
  ep_wait_sources_kernel<<<1, 64, 0, as_stream(stream)>>>(own, world);
  QK_LAUNCHED("ep_wait_sources_kernel");
  PushArgs push{reinterpret_cast<uint8_t* const*>(peers), own, L, rank};
  return moe_forward_impl(desc, gate, up, down, reinterpret_cast<const uint16_t*>(own + L.recv_x),
                          reinterpret_cast<const int32_t*>(own + L.recv_ids),
                          reinterpret_cast<const uint16_t*>(own + L.recv_w), world * max_tokens, QK_OUT_F32,
                          nullptr, workspace, workspace_bytes, stream, events, nullptr, kPush, &push);
}

int qk_cast_f32_bf16(const float* in, uint16_t* out, int64_t n, qk_stream_t stream) {
  QK_REQUIRE(n >= 0, "n must be non-negative");
  if (n == 0) return QK_OK;
  QK_REQUIRE(in && out, "null pointer");
  int64_t grid = (n + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  cast_kernel<<<static_cast<unsigned>(grid > cap ? cap : grid), 256, 0, as_stream(stream)>>>(in, out, n);
  QK_LAUNCHED("cast_kernel");
  return QK_OK;
}

int qk_moe_check(const void* workspace, qk_stream_t stream) {
  QK_REQUIRE(workspace, "null workspace");
  int32_t status = 0;
  const MoeMeta* meta = static_cast<const MoeMeta*>(workspace);
  cudaError_t e = cudaMemcpyAsync(&status, &meta->status, 4, cudaMemcpyDeviceToHost, as_stream(stream));
  if (e == cudaSuccess) e = cudaStreamSynchronize(as_stream(stream));
  if (e != cudaSuccess) return cuda_error(e, "qk_moe_check");
  if (status) return set_error(status, "a bounded device wait in the expert kernels gave up");
  return QK_OK;
}

}  // extern "C"
