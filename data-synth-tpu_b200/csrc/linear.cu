// Dense BF16 projection for decode-sized batches on the tcgen05 tensor core:
//   y[M, N] = bf16(x[M, K] @ W[N, K]^T) with FP32 accumulation,
// the reference's linear (qwen38_tpu/math.py:10-16: BF16 operands, preferred_element_type
// FP32, compute_cast to BF16). It serves the decoder stack's attention projections
// (attention_cache.py:131-134 q|gate, k, v and :171 out) at M = decode batch <= 256, where
// the pass is bound by streaming W from HBM once.
//
// Work item: 128 rows of W (one M = 128 MMA tile, i.e. 128 output columns) times a slice of
// the K dimension. A row tile is cut into `splits` K slices so that about every SM streams
// W; the slices leave FP32 partials in the workspace and the last CTA of the tile to finish
// (a counter per tile, reset by that CTA) adds them in slice order and writes BF16, so the
// result does not depend on which CTA ends last. With one slice the epilogue writes BF16
// directly.
//
// Warps: 0 producer - per 64-value K atom one 2D tensor copy of the W box [128 rows x
// 128 B] and one of the x box [M16 rows x 128 B] (rows past M read as zeros), both landing
// with the 128-byte swizzle that the MMA's K-major descriptors read; 1 MMA issuer - 4
// tcgen05.mma kind::f16 (M = 128, N = M16, K = 16) per atom, A = W and B = x from shared
// memory, the FP32 accumulator in TMEM; 2-5 epilogue - tcgen05.ld of their TMEM lane quarter.
// Launched as a programmatic dependent: the W boxes of the first stages are requested before
// griddepcontrol.wait (no earlier kernel writes W), the x boxes after it. No multicast. Every
// wait is bounded; on give-up the CTA records QK_ERR_TIMEOUT in the workspace status word.
//
// Up to kGemvMaxM rows of x (a decode step of one to four sequences) take linear_gemv_kernel
// instead: a warp per output column, the row of W streamed with 16-byte loads (eight per lane
// in flight) against x held in shared memory, FP32 fused multiply-adds and a warp butterfly.
// An MMA of N = 16 tokens would waste 15/16 of its columns there, and the per-CTA MMA chain,
// the split-K partials and their ordered sum were most of that pass's time.
#include <cuda.h>  // CUtensorMap and its enums; the encoder is looked up at run time

#include "umma.cuh"

namespace qk {
namespace {

constexpr int kLinThreads = 6 * 32;
constexpr int kLinStagesMax = 8;
constexpr int kLinMaxM = 256;
constexpr uint32_t kWBox = 128 * 128;  // bytes of one W box (128 rows x 64 BF16)
constexpr size_t kLinSmemBudget = 200 * 1024;

struct LinArgs {
  int M, N, m16, splits, atoms, stages;
  uint32_t tcols;
  uint16_t* y;
  float* part;      // [splits][M][N] FP32 partials (splits > 1)
  int* counters;    // [tiles]
  int* status;
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void epilogue_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

constexpr int kGemvMaxM = 4;
constexpr int kGemvThreads = 256;
constexpr int kGemvChunks = 8;  // 16-byte chunks of a W row per lane per pass (256 per warp)

// y[m, n] = bf16(sum_k x[m, k] w[n, k]) for m < MM: warp per column n (grid-strided), lane l
// adding the chunks l, l + 32, ... of the row in order, then a butterfly over the lanes.
template <int MM>
__global__ void __launch_bounds__(kGemvThreads) linear_gemv_kernel(const uint16_t* x, const uint16_t* __restrict__ w,
                                                                   int N, int K, uint16_t* __restrict__ y) {
  extern __shared__ uint4 xs[];  // x [MM][K / 8 chunks]
  const int lane = threadIdx.x & 31;
  const int nw = gridDim.x * (kGemvThreads / 32);
  const int kc = K / 8;
  const uint4* w4 = reinterpret_cast<const uint4*>(w);
  uint4 wv[kGemvChunks];
  auto load_pass = [&](int r, int c0) {
#pragma unroll
    for (int j = 0; j < kGemvChunks; ++j) {
      const int c = c0 + lane + 32 * j;
      wv[j] = c < kc ? w4[static_cast<int64_t>(r) * kc + c] : make_uint4(0, 0, 0, 0);
    }
  };
  int row = blockIdx.x * (kGemvThreads / 32) + (threadIdx.x >> 5);
  if (row < N) load_pass(row, 0);  // W is no earlier kernel's output: fetched before the wait
  pdl_wait();
  pdl_trigger();
  for (int i = threadIdx.x; i < MM * kc; i += kGemvThreads) xs[i] = reinterpret_cast<const uint4*>(x)[i];
  __syncthreads();
  for (; row < N; row += nw) {
    float acc[MM];
#pragma unroll
    for (int m = 0; m < MM; ++m) acc[m] = 0.f;
    for (int c0 = 0; c0 < kc; c0 += 32 * kGemvChunks) {
      if (c0 > 0) load_pass(row, c0);
#pragma unroll
      for (int j = 0; j < kGemvChunks; ++j) {
        const int c = c0 + lane + 32 * j;
        if (c >= kc) break;
        float f[8];
        unpack8(wv[j], f);
#pragma unroll
        for (int m = 0; m < MM; ++m) {
          float g[8];
          unpack8(xs[m * kc + c], g);
#pragma unroll
          for (int t = 0; t < 8; ++t) acc[m] = fmaf(f[t], g[t], acc[m]);
        }
      }
    }
    if (row + nw < N) load_pass(row + nw, 0);  // the next column's loads overlap this one's sums
#pragma unroll
    for (int m = 0; m < MM; ++m) {
      float v = acc[m];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) y[static_cast<int64_t>(m) * N + row] = bf16_bits_rne(v);
    }
  }
}

template <int MM>
cudaError_t launch_gemv(const uint16_t* x, const uint16_t* w, int N, int K, uint16_t* y, cudaStream_t st) {
  const size_t smem = static_cast<size_t>(MM) * K * 2;
  int rc = allow_smem(reinterpret_cast<const void*>(linear_gemv_kernel<MM>), smem);
  if (rc) return cudaErrorInvalidValue;
  int64_t grid = (static_cast<int64_t>(N) + kGemvThreads / 32 - 1) / (kGemvThreads / 32);
  if (grid > 4 * sm_count()) grid = 4 * sm_count();
  return launch_dependent(linear_gemv_kernel<MM>, dim3(static_cast<unsigned>(grid)), dim3(kGemvThreads), smem, st, x, w,
                          N, K, y);
}

__global__ void __launch_bounds__(kLinThreads, 1)
    linear_bf16_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx, LinArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stages = a.stages;
  const uint32_t xbytes = static_cast<uint32_t>(a.m16) * 128u, stage_bytes = kWBox + xbytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(stages) * stage_bytes);
  uint64_t* empty = full + kLinStagesMax;
  uint64_t* done = empty + kLinStagesMax;
  uint32_t* tmem_sh = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* last_flag = reinterpret_cast<volatile int*>(tmem_sh + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = static_cast<int>(blockIdx.x) / a.splits, split = static_cast<int>(blockIdx.x) % a.splits;
  const int a0 = split * a.atoms / a.splits, a1 = (split + 1) * a.atoms / a.splits;
  const int n = a1 - a0;  // >= 1: splits <= atoms

  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(done, 1);
    *last_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_sh, a.tcols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_sh;
  pdl_trigger();
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t wpol = l2_evict_first_policy(), xpol = l2_evict_last_policy();
      const int pre = min(stages, n);
      for (int i = 0; i < pre; ++i) {
        mbar_expect_tx(&full[i], stage_bytes);
        tma_load_2d(smem + static_cast<size_t>(i) * stage_bytes, &tw, (a0 + i) * 64, tile * 128, &full[i], wpol);
      }
      pdl_wait();  // x is the previous kernel's output
      for (int i = 0; i < pre; ++i)
        tma_load_2d(smem + static_cast<size_t>(i) * stage_bytes + kWBox, &tx, (a0 + i) * 64, 0, &full[i], xpol);
      int issued = pre;
      for (int i = pre; i < n; ++i) {
        const int s = i % stages;
        if (!mbar_wait_bounded(&empty[s], ((i / stages) - 1) & 1)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + static_cast<size_t>(s) * stage_bytes;
        mbar_expect_tx(&full[s], stage_bytes);
        tma_load_2d(st, &tw, (a0 + i) * 64, tile * 128, &full[s], wpol);
        tma_load_2d(st + kWBox, &tx, (a0 + i) * 64, 0, &full[s], xpol);
        issued = i + 1;
      }
      // every copy issued must have landed before the CTA leaves (instant when the MMA
      // consumed them all; bounded otherwise)
      for (int s = 0; s < min(stages, issued); ++s) {
        const int loads = (issued - s + stages - 1) / stages;  // copies into stage s
        mbar_wait_bounded(&full[s], (loads - 1) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16_m128(static_cast<uint32_t>(a.m16));
      for (int i = 0; i < n; ++i) {
        const int s = i % stages;
        if (!mbar_wait_bounded(&full[s], (i / stages) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sw = smem_addr(smem + static_cast<size_t>(s) * stage_bytes);
        const uint64_t ad = sdesc_sw128(sw, 1024u), bd = sdesc_sw128(sw + kWBox, 1024u);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) umma_ss(tbase, ad + ks * 2, bd + ks * 2, idesc, (i != 0) || (ks != 0));
        umma_commit(&empty[s]);
      }
      umma_commit(done);
    }
  } else {
    // epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 = rows r of the W tile
    const int q = warp & 3, r = 32 * q + lane, row = tile * 128 + r;
    const bool have = mbar_wait_bounded(done, 0);
    if (!have) ok = false;
    tc_fence_after();
    const bool direct = a.splits == 1;
    for (int c0 = 0; c0 < a.m16; c0 += 8) {
      uint32_t v[8];
      tmem_ld8(tbase + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(c0), v);
      tmem_wait_ld();
      if (!have || row >= a.N) continue;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int m = c0 + j;
        if (m >= a.M) break;
        const float f = __uint_as_float(v[j]);
        if (direct) a.y[static_cast<int64_t>(m) * a.N + row] = bf16_bits_rne(f);
        else a.part[(static_cast<int64_t>(split) * a.M + m) * a.N + row] = f;
      }
    }
    if (!direct) {
      __threadfence();  // this CTA's partials are visible before its arrival is counted
      epilogue_sync();
      if (threadIdx.x == 2 * 32) *last_flag = atomicAdd(&a.counters[tile], 1) == a.splits - 1;
    }
  }

  if (!ok && lane == 0) atomicExch(a.status, QK_ERR_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, a.tcols);
  }
  if (*last_flag) {
    // the last CTA of the tile: every thread adds the slices' partials of (token, 4 columns)
    // items in slice order (loads of several slices in flight), then BF16
    __threadfence();
    const int n0 = tile * 128;
    const int64_t sstride = static_cast<int64_t>(a.M) * a.N;
    const bool vec = (a.N & 3) == 0;
    for (int it = threadIdx.x; it < a.M * 32; it += blockDim.x) {
      const int m = it >> 5, col = n0 + (it & 31) * 4;
      if (col >= a.N) continue;
      const float* p = a.part + static_cast<int64_t>(m) * a.N + col;
      uint16_t* yo = a.y + static_cast<int64_t>(m) * a.N + col;
      if (vec) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
        for (int sp = 0; sp < a.splits; ++sp) {
          const float4 v = __ldcg(reinterpret_cast<const float4*>(p + sp * sstride));
          acc.x = __fadd_rn(acc.x, v.x);
          acc.y = __fadd_rn(acc.y, v.y);
          acc.z = __fadd_rn(acc.z, v.z);
          acc.w = __fadd_rn(acc.w, v.w);
        }
        *reinterpret_cast<uint2*>(yo) =
            make_uint2(bf16_bits_rne(acc.x) | (static_cast<uint32_t>(bf16_bits_rne(acc.y)) << 16),
                       bf16_bits_rne(acc.z) | (static_cast<uint32_t>(bf16_bits_rne(acc.w)) << 16));
      } else {
        for (int j = 0; j < 4 && col + j < a.N; ++j) {
          float acc = 0.f;
          for (int sp = 0; sp < a.splits; ++sp) acc = __fadd_rn(acc, __ldcg(p + sp * sstride + j));
          yo[j] = bf16_bits_rne(acc);
        }
      }
    }
    if (threadIdx.x == 0) a.counters[tile] = 0;  // ready for the next call
  }
}

// K slices per 128-row tile: enough CTAs for the SMs, each slice at least one atom, the
// partials (written and read once, 8 M bytes per K slice per output column) at most about a
// quarter of the W bytes of the slice (2 K bytes per column), and at most 256 KB of partials
// per tile for its last CTA to add.
int splits_for(int64_t M, int64_t K, int64_t N) {
  const int64_t tiles = (N + 127) / 128, atoms = K / 64;
  int64_t s = sm_count() / tiles;
  const int64_t cap = K / (8 * M) < 65536 / (128 * M) ? K / (8 * M) : 65536 / (128 * M);
  if (s > cap) s = cap;
  if (s > atoms) s = atoms;
  return static_cast<int>(s < 1 ? 1 : s);
}

size_t header_bytes(int64_t N) {
  const int64_t tiles = (N + 127) / 128;
  return (256 + static_cast<size_t>(tiles) * 4 + 255) / 256 * 256;
}

size_t workspace_need(int64_t M, int64_t K, int64_t N) {
  const int s = splits_for(M, K, N);
  return header_bytes(N) + (s > 1 ? static_cast<size_t>(s) * M * N * 4 : 0);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// 2D map over a row-major BF16 [rows, K] matrix, box 64 x box_rows, 128-byte swizzle.
bool encode_rows(CUtensorMap* map, const void* base, uint64_t K, uint64_t rows, uint32_t box_rows) {
  EncodeTiledFn fn = reinterpret_cast<EncodeTiledFn>(tensor_map_encoder());
  if (!fn) return false;
  const cuuint64_t dims[2] = {K, rows};
  const cuuint64_t strides[1] = {K * 2};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace
}  // namespace qk

using namespace qk;

extern "C" {

size_t qk_linear_bf16_workspace_bytes(int64_t M, int64_t K, int64_t N) {
  if (M <= 0 || M > kLinMaxM || K <= 0 || K % 64 || N <= 0) return 0;
  return workspace_need(M, K, N);
}

int qk_linear_bf16(const uint16_t* x, int64_t M, int64_t K, const uint16_t* w, int64_t N, uint16_t* y,
                   void* workspace, size_t workspace_bytes, qk_stream_t stream) {
  QK_REQUIRE(M >= 0 && M <= kLinMaxM, "M must be in [0, %d] (decode batches; larger M is a library GEMM's)",
             kLinMaxM);
  QK_REQUIRE(K > 0 && K % 64 == 0, "K must be a positive multiple of 64");
  QK_REQUIRE(N > 0 && N < (1ll << 31) && K < (1ll << 31), "invalid N or K");
  if (M == 0) return QK_OK;
  QK_REQUIRE(x && w && y, "null pointer");
  QK_REQUIRE((reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0,
             "x and w must be 16-byte aligned");
  const size_t need = workspace_need(M, K, N);
  if (!workspace || workspace_bytes < need)
    return set_error(QK_ERR_WORKSPACE, "linear workspace needs %zu bytes, got %zu", need, workspace_bytes);
  QK_REQUIRE((reinterpret_cast<uintptr_t>(workspace) & 255) == 0, "workspace must be 256-byte aligned");
  if (M <= kGemvMaxM && K <= 16384) {
    cudaStream_t st = as_stream(stream);
    const int n = static_cast<int>(N), k = static_cast<int>(K);
    const cudaError_t e = M == 1   ? launch_gemv<1>(x, w, n, k, y, st)
                          : M == 2 ? launch_gemv<2>(x, w, n, k, y, st)
                          : M == 3 ? launch_gemv<3>(x, w, n, k, y, st)
                                   : launch_gemv<4>(x, w, n, k, y, st);
    if (e != cudaSuccess) return cuda_error(e, "linear_gemv_kernel");
    count_launch();
    return QK_OK;
  }
  LinArgs a{};
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.m16 = static_cast<int>((M + 15) / 16 * 16);
  a.splits = splits_for(M, K, N);
  a.atoms = static_cast<int>(K / 64);
  const size_t stage_bytes = kWBox + static_cast<size_t>(a.m16) * 128;
  a.stages = static_cast<int>(kLinSmemBudget / stage_bytes);
  if (a.stages > kLinStagesMax) a.stages = kLinStagesMax;
  a.tcols = 32;
  while (a.tcols < static_cast<uint32_t>(a.m16)) a.tcols *= 2;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  a.status = reinterpret_cast<int*>(ws);
  a.counters = reinterpret_cast<int*>(ws + 256);
  a.part = reinterpret_cast<float*>(ws + header_bytes(N));
  a.y = y;
  CUtensorMap maps[2];
  memset(maps, 0, sizeof(maps));
  if (!encode_rows(&maps[0], w, static_cast<uint64_t>(K), static_cast<uint64_t>(N), 128) ||
      !encode_rows(&maps[1], x, static_cast<uint64_t>(K), static_cast<uint64_t>(M), static_cast<uint32_t>(a.m16)))
    return set_error(QK_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable or refused the linear operands");
  const size_t smem = 1024 + static_cast<size_t>(a.stages) * stage_bytes + (2 * kLinStagesMax + 1) * 8 + 8;
  int rc = allow_smem(reinterpret_cast<const void*>(linear_bf16_kernel), smem);
  if (rc) return rc;
  const int tiles = static_cast<int>((N + 127) / 128);
  const cudaError_t e = launch_dependent(linear_bf16_kernel, dim3(tiles * a.splits), dim3(kLinThreads), smem,
                                         as_stream(stream), maps[0], maps[1], a);
  if (e != cudaSuccess) return cuda_error(e, "linear_bf16_kernel");
  count_launch();
  return QK_OK;
}

int qk_linear_bf16_check(const void* workspace, qk_stream_t stream) {
  QK_REQUIRE(workspace, "null pointer");
  int status = 0;
  cudaStream_t st = as_stream(stream);
  cudaError_t e = cudaMemcpyAsync(&status, workspace, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && status) {
    e = cudaMemsetAsync(const_cast<void*>(workspace), 0, sizeof(int), st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  }
  if (e != cudaSuccess) return cuda_error(e, "qk_linear_bf16_check");
  if (status) return set_error(status, "a bounded device wait in the linear kernel gave up");
  return QK_OK;
}

}  // extern "C"
