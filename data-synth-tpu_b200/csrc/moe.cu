// Routed-expert SwiGLU FFN over tiled Q6_K / Q4_K expert weights (decode regime).
//
// Replaces the routed FFN of qwen38_tpu/experts.py:61-131 (and grouped_experts.py:185-292
// at tp = 1) for the experts one rank holds. Four launches on one stream:
//
//  1. route   - one CTA turns ids/weights [B, k] into per-expert entry lists (expert-
//               sorted), merging duplicate routes of a token into one entry whose weight
//               is bf16(sum) (experts.py:66-73) and dropping zero-weight routes (their
//               contribution is zero in the reference, experts.py:74-76).
//  2. gate/up - per (active expert, 16-row strip of I): h = bf16(silu(bf16(x Wg^T)) *
//               bf16(x Wu^T)) for every entry of the expert (experts.py:103-107,
//               math.py:10-20). Weight tiles stream HBM -> shared memory with 1-D bulk
//               copies (TMA engine) into a per-warp ring; each warp decodes its tile into
//               BF16 MMA fragments in registers and runs m16n8k16 MMAs with FP32 accumulate.
//  3. down    - per (active expert, 16-row strip of H): y = bf16(h Wd^T).
//  4. combine - per token, FP32 sum of f32(y) * f32(route) over its experts in ascending
//               expert order (the reference's accumulation order, experts.py:129), then
//               BF16 (experts.py:131), or the FP32 partial sum for an EP all-reduce.
#include "common.cuh"
#include "proj.cuh"

namespace qk {
namespace {

struct MoeMeta {
  int32_t n_active;
  int32_t n_entries;
  int32_t status;
  int32_t reserved;
};

struct Workspace {
  MoeMeta* meta;
  int32_t* counts;        // [E]
  int32_t* offsets;       // [E + 1]
  int32_t* active;        // [E]   active expert ids (local), ascending
  int32_t* entry_token;   // [B k] token of each entry (expert-sorted)
  float* entry_weight;    // [B k] bf16-valued route weight of each entry
  int32_t* route_entry;   // [B k] entry of route (b, j), -1 if none
  uint16_t* h;            // [B k, I]
  uint16_t* y;            // [B k, H]
};

inline size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

size_t layout(const qk_moe_desc& d, int max_tokens, uint8_t* base, Workspace* ws) {
  const size_t E = d.num_experts, R = static_cast<size_t>(max_tokens) * d.top_k;
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
  uint8_t* et = take(R * 4);
  uint8_t* ew = take(R * 4);
  uint8_t* re = take(R * 4);
  uint8_t* h = take(R * d.intermediate * 2);
  uint8_t* y = take(R * d.hidden * 2);
  if (ws) {
    ws->meta = reinterpret_cast<MoeMeta*>(meta);
    ws->counts = reinterpret_cast<int32_t*>(counts);
    ws->offsets = reinterpret_cast<int32_t*>(offsets);
    ws->active = reinterpret_cast<int32_t*>(active);
    ws->entry_token = reinterpret_cast<int32_t*>(et);
    ws->entry_weight = reinterpret_cast<float*>(ew);
    ws->route_entry = reinterpret_cast<int32_t*>(re);
    ws->h = reinterpret_cast<uint16_t*>(h);
    ws->y = reinterpret_cast<uint16_t*>(y);
  }
  return off;
}

// ------------------------------------------------------------------------------------
// 1. routing metadata (one CTA)
// ------------------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) moe_route_kernel(const int32_t* __restrict__ ids,
                                                         const uint16_t* __restrict__ weights,
                                                         int B, int k, int E, int first,
                                                         Workspace ws) {
  extern __shared__ int32_t sh[];
  int32_t* counts = sh;            // [E]
  int32_t* cursor = sh + E;        // [E]
  int32_t* offsets = sh + 2 * E;   // [E + 1]
  __shared__ int32_t chunk_base[33], active_base[33];
  const int tid = threadIdx.x, nt = blockDim.x;
  for (int e = tid; e < E; e += nt) counts[e] = cursor[e] = 0;
  __syncthreads();

  // Pass 1: entries per expert. The first slot j of a token that names expert e owns
  // the merged entry; its weight is bf16 of the FP32 sum over all slots naming e.
  for (int b = tid; b < B; b += nt) {
    for (int j = 0; j < k; ++j) {
      const int e = ids[b * k + j] - first;
      int own = e >= 0 && e < E;
      for (int jj = 0; own && jj < j; ++jj) own = ids[b * k + jj] - first != e;
      float w = 0.f;
      if (own) {
        for (int jj = j; jj < k; ++jj)
          if (ids[b * k + jj] - first == e) w = __fadd_rn(w, bf16_to_f32(weights[b * k + jj]));
        w = bf16_round(w);
        own = w != 0.f;
      }
      if (own) atomicAdd(&counts[e], 1);
    }
  }
  __syncthreads();

  // Exclusive scan over experts (warp 0, contiguous chunks per lane) + active list.
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
    chunk_base[tid] = incl - sum;
    active_base[tid] = iact - act;
    if (tid == 31) {
      chunk_base[32] = incl;
      active_base[32] = iact;
    }
    __syncwarp();
    int run = chunk_base[tid], arun = active_base[tid];
    for (int e = lo; e < hi; ++e) {
      offsets[e] = run;
      ws.offsets[e] = run;
      ws.counts[e] = counts[e];
      run += counts[e];
      if (counts[e] > 0) ws.active[arun++] = e;
    }
    if (tid == 31) {
      offsets[E] = chunk_base[32];
      ws.offsets[E] = chunk_base[32];
      ws.meta->n_entries = chunk_base[32];
      ws.meta->n_active = active_base[32];
      ws.meta->status = 0;
    }
  }
  __syncthreads();

  // Pass 2: place entries.
  for (int b = tid; b < B; b += nt) {
    for (int j = 0; j < k; ++j) {
      const int e = ids[b * k + j] - first;
      int own = e >= 0 && e < E;
      for (int jj = 0; own && jj < j; ++jj) own = ids[b * k + jj] - first != e;
      float w = 0.f;
      if (own) {
        for (int jj = j; jj < k; ++jj)
          if (ids[b * k + jj] - first == e) w = __fadd_rn(w, bf16_to_f32(weights[b * k + jj]));
        w = bf16_round(w);
        own = w != 0.f;
      }
      int slot = -1;
      if (own) {
        slot = offsets[e] + atomicAdd(&cursor[e], 1);
        ws.entry_token[slot] = b;
        ws.entry_weight[slot] = w;
      }
      ws.route_entry[b * k + j] = slot;
    }
  }
}

// ------------------------------------------------------------------------------------
// 2./3. projection kernels
// ------------------------------------------------------------------------------------

struct ProjArgs {
  const uint8_t* wa;      // gate (gate/up) or down tiles, expert-major
  const uint8_t* wb;      // up tiles (gate/up only)
  int64_t expert_bytes;   // tiled bytes per expert of one projection
  const uint16_t* act;    // x [B, H] (gate/up) or h [entries, I] (down)
  int K;                  // reduction width (H or I)
  int N;                  // output rows (I or H)
  Workspace ws;
};

// Position of (item, chunk, kb) in a warp's tile stream.
struct Cursor {
  int item, chunk, kb, chunks;
  __device__ __forceinline__ bool valid(int n_items) const { return item < n_items; }
};

template <QType QT, bool kGateUp>
__device__ __forceinline__ int chunks_of(const ProjArgs& a, int item, int strips) {
  const int e = a.ws.active[item / strips];
  return (a.ws.counts[e] + kChunk - 1) / kChunk;
}

template <QType QT, bool kGateUp>
__global__ void __launch_bounds__(kWarps * 32, 1) moe_proj_kernel(ProjArgs a) {
  using Cfg = ProjCfg<QT, kGateUp>;
  constexpr int TB = Tile<QT>::kBytes, R = Cfg::kStages;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  uint8_t* ring = smem + static_cast<size_t>(warp) * R * Cfg::kStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(kWarps) * R * Cfg::kStage) + warp * R;

  const int strips = a.N / 16, nkb = a.K / 256;
  const int n_items = a.ws.meta->n_active * strips;
  const int total = gridDim.x * kWarps;
  const int first = blockIdx.x * kWarps + warp;
  if (first >= n_items) return;

  if (lane == 0) {
    for (int i = 0; i < R; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  __syncwarp();

  auto tile_src = [&](const uint8_t* base, const Cursor& cur) {
    const int e = a.ws.active[cur.item / strips];
    const int strip = cur.item % strips;
    return base + e * a.expert_bytes + (static_cast<int64_t>(strip) * nkb + cur.kb) * TB;
  };
  auto advance = [&](Cursor& cur) {
    if (++cur.kb == nkb) {
      cur.kb = 0;
      if (++cur.chunk == cur.chunks) {
        cur.chunk = 0;
        cur.item += total;
        cur.chunks = cur.item < n_items ? chunks_of<QT, kGateUp>(a, cur.item, strips) : 0;
      }
    }
  };

  Cursor prod{first, 0, 0, chunks_of<QT, kGateUp>(a, first, strips)};
  Cursor cons = prod;
  uint32_t tp = 0, tc = 0;
  auto issue = [&]() {
    if (lane == 0) {
      const uint32_t slot = tp % R;
      uint8_t* dst = ring + slot * Cfg::kStage;
      mbar_expect_tx(&bars[slot], Cfg::kStage);
      bulk_g2s(dst, tile_src(a.wa, prod), TB, &bars[slot]);
      if (kGateUp) bulk_g2s(dst + TB, tile_src(a.wb, prod), TB, &bars[slot]);
    }
    ++tp;
    advance(prod);
  };
  for (int i = 0; i < R && prod.valid(n_items); ++i) issue();

  bool ok = true;
  while (cons.valid(n_items) && ok) {
    const int e = a.ws.active[cons.item / strips];
    const int strip = cons.item % strips;
    const int base = a.ws.offsets[e] + cons.chunk * kChunk;
    const int ntok = min(kChunk, a.ws.counts[e] - cons.chunk * kChunk);
    const int J = (ntok + 7) / 8;
    // B-fragment source rows of token columns 8j + g.
    const uint16_t* rows[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int col = 8 * j + g;
      rows[j] = nullptr;
      if (col < ntok) {
        const int src = kGateUp ? a.ws.entry_token[base + col] : base + col;
        rows[j] = a.act + static_cast<int64_t>(src) * a.K;
      }
    }
    float acc_a[4][4] = {}, acc_b[4][4] = {};
    for (int kb = 0; kb < nkb; ++kb) {
      const uint32_t slot = tc % R;
      if (!mbar_wait_bounded(&bars[slot], (tc / R) & 1)) {
        ok = false;
        break;
      }
      const uint8_t* stage = ring + slot * Cfg::kStage;
      if (J == 1) proj_stage<QT, kGateUp, 1, false>(stage, lane, kb * 256, a.K, rows, acc_a, acc_b);
      else if (J == 2) proj_stage<QT, kGateUp, 2, false>(stage, lane, kb * 256, a.K, rows, acc_a, acc_b);
      else proj_stage<QT, kGateUp, 4, false>(stage, lane, kb * 256, a.K, rows, acc_a, acc_b);
      ++tc;
      // Every lane has consumed (decoded) its shared-memory words: refill the slot.
      __syncwarp();
      if (lane == 0) fence_proxy_async_smem();
      if (prod.valid(n_items)) issue();
    }
    if (!ok) break;
    // Epilogue: rows strip*16 + g (+8), token columns 8j + 2c (+1).
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j >= J) break;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int col = 8 * j + 2 * c + (i & 1);
        const int row = strip * 16 + g + (i >> 1) * 8;
        if (col >= ntok) continue;
        const int entry = base + col;
        if (kGateUp) {
          const float gb = bf16_round(acc_a[j][i]);
          const float ub = bf16_round(acc_b[j][i]);
          const float act = bf16_round(__fmul_rn(gb, sigmoid_ref(gb)));  // silu, math.py:19-20
          a.ws.h[static_cast<int64_t>(entry) * a.N + row] = bf16_bits_rne(__fmul_rn(act, ub));
        } else {
          a.ws.y[static_cast<int64_t>(entry) * a.N + row] = bf16_bits_rne(acc_a[j][i]);
        }
      }
    }
    // advance consumer to the next (item, chunk)
    cons.kb = nkb - 1;
    advance(cons);
  }
  if (!ok) {
    if (lane == 0) atomicExch(&a.ws.meta->status, QK_ERR_TIMEOUT);
    // Drain copies still in flight into this warp's ring before leaving.
    while (tc < tp) {
      mbar_wait_bounded(&bars[tc % R], (tc / R) & 1);
      ++tc;
    }
  }
}

// ------------------------------------------------------------------------------------
// 4. combine
// ------------------------------------------------------------------------------------
constexpr int kMaxTopK = 32;

__global__ void __launch_bounds__(256) moe_combine_kernel(const int32_t* __restrict__ ids, int B,
                                                          int k, int H, int out_bf16, void* out,
                                                          Workspace ws) {
  const int b = blockIdx.x;
  int ent[kMaxTopK], eid[kMaxTopK];
  int n = 0;
  for (int j = 0; j < k; ++j) {
    const int entry = ws.route_entry[b * k + j];
    if (entry < 0) continue;
    const int e = ids[b * k + j];
    int pos = n++;
    while (pos > 0 && eid[pos - 1] > e) {  // insertion sort by expert id
      eid[pos] = eid[pos - 1];
      ent[pos] = ent[pos - 1];
      --pos;
    }
    eid[pos] = e;
    ent[pos] = entry;
  }
  for (int col = threadIdx.x; col < H; col += blockDim.x) {
    float acc = 0.f;
    for (int i = 0; i < n; ++i) {
      const float y = bf16_to_f32(ws.y[static_cast<int64_t>(ent[i]) * H + col]);
      acc = __fadd_rn(acc, __fmul_rn(y, ws.entry_weight[ent[i]]));
    }
    if (out_bf16) static_cast<uint16_t*>(out)[static_cast<int64_t>(b) * H + col] = bf16_bits_rne(acc);
    else static_cast<float*>(out)[static_cast<int64_t>(b) * H + col] = acc;
  }
}

__global__ void cast_kernel(const float* __restrict__ in, uint16_t* __restrict__ out, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    out[i] = bf16_bits_rne(in[i]);
}

bool supported(int t) { return t == QK_TYPE_Q6_K || t == QK_TYPE_Q4_K; }

template <QType QT>
int launch_proj(const ProjArgs& a, int max_items, cudaStream_t st, bool gateup) {
  const int sms = sm_count();
  int grid = (max_items + kWarps - 1) / kWarps;
  grid = grid < 1 ? 1 : (grid > sms ? sms : grid);
  if (gateup) {
    using Cfg = ProjCfg<QT, true>;
    int rc = allow_smem(reinterpret_cast<const void*>(moe_proj_kernel<QT, true>), Cfg::kSmem);
    if (rc) return rc;
    moe_proj_kernel<QT, true><<<grid, kWarps * 32, Cfg::kSmem, st>>>(a);
  } else {
    using Cfg = ProjCfg<QT, false>;
    int rc = allow_smem(reinterpret_cast<const void*>(moe_proj_kernel<QT, false>), Cfg::kSmem);
    if (rc) return rc;
    moe_proj_kernel<QT, false><<<grid, kWarps * 32, Cfg::kSmem, st>>>(a);
  }
  QK_LAUNCHED("moe_proj_kernel");
  return QK_OK;
}

}  // namespace
}  // namespace qk

using namespace qk;

extern "C" {

size_t qk_moe_workspace_bytes(const qk_moe_desc* desc, int max_tokens) {
  if (!desc || max_tokens < 0) return 0;
  return layout(*desc, max_tokens, nullptr, nullptr);
}

static int moe_forward_impl(const qk_moe_desc* desc, const uint8_t* gate, const uint8_t* up,
                            const uint8_t* down, const uint16_t* x, const int32_t* ids,
                            const uint16_t* weights, int B, int out_dtype, void* out,
                            void* workspace, size_t workspace_bytes, qk_stream_t stream,
                            void* const* events) {
  QK_REQUIRE(desc, "null descriptor");
  const qk_moe_desc& d = *desc;
  if (!supported(d.gate_type) || d.gate_type != d.up_type || d.gate_type != d.down_type)
    return set_error(QK_ERR_UNSUPPORTED_TYPE, "expert types must all be Q6_K or all Q4_K (got %d/%d/%d)", d.gate_type, d.up_type, d.down_type);
  QK_REQUIRE(d.hidden > 0 && d.hidden % 256 == 0, "hidden must be a positive multiple of 256");
  QK_REQUIRE(d.intermediate > 0 && d.intermediate % 256 == 0, "intermediate must be a positive multiple of 256");
  QK_REQUIRE(d.num_experts > 0 && d.num_experts <= 4096, "num_experts must be in [1, 4096]");
  QK_REQUIRE(d.top_k > 0 && d.top_k <= kMaxTopK, "top_k must be in [1, %d]", kMaxTopK);
  QK_REQUIRE(B >= 0, "batch must be non-negative");
  QK_REQUIRE(out_dtype == QK_OUT_F32 || out_dtype == QK_OUT_BF16, "out_dtype must be F32 or BF16");
  if (B == 0) return QK_OK;
  QK_REQUIRE(gate && up && down && x && ids && weights && out, "null pointer");
  const size_t need = layout(d, B, nullptr, nullptr);
  if (!workspace || workspace_bytes < need)
    return set_error(QK_ERR_WORKSPACE, "workspace needs %zu bytes, got %zu", need, workspace_bytes);
  Workspace ws;
  layout(d, B, static_cast<uint8_t*>(workspace), &ws);
  cudaStream_t st = as_stream(stream);
  auto mark = [&](int i) {
    if (events && events[i]) cudaEventRecord(static_cast<cudaEvent_t>(events[i]), st);
  };

  mark(0);
  const size_t route_smem = (3 * static_cast<size_t>(d.num_experts) + 1) * 4;
  int rc = allow_smem(reinterpret_cast<const void*>(moe_route_kernel), route_smem);
  if (rc) return rc;
  moe_route_kernel<<<1, 1024, route_smem, st>>>(ids, weights, B, d.top_k, d.num_experts, d.first_expert, ws);
  QK_LAUNCHED("moe_route_kernel");

  const int max_active = d.num_experts < B * d.top_k ? d.num_experts : B * d.top_k;
  ProjArgs gu{gate, up, qk_tiled_bytes(d.gate_type, d.intermediate, d.hidden), x, d.hidden, d.intermediate, ws};
  ProjArgs dn{down, nullptr, qk_tiled_bytes(d.down_type, d.hidden, d.intermediate), ws.h, d.intermediate, d.hidden, ws};
  const bool q6 = d.gate_type == QK_TYPE_Q6_K;
  mark(1);
  rc = q6 ? launch_proj<QType::Q6_K>(gu, max_active * (d.intermediate / 16), st, true)
          : launch_proj<QType::Q4_K>(gu, max_active * (d.intermediate / 16), st, true);
  if (rc) return rc;
  mark(2);
  rc = q6 ? launch_proj<QType::Q6_K>(dn, max_active * (d.hidden / 16), st, false)
          : launch_proj<QType::Q4_K>(dn, max_active * (d.hidden / 16), st, false);
  if (rc) return rc;
  mark(3);
  moe_combine_kernel<<<B, 256, 0, st>>>(ids, B, d.top_k, d.hidden, out_dtype == QK_OUT_BF16, out, ws);
  QK_LAUNCHED("moe_combine_kernel");
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
