// Shared device helpers for the qk_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "qk_b200.h"

namespace qk {

// ---------------------------------------------------------------------------------
// host-side status plumbing
// ---------------------------------------------------------------------------------

int set_error(int status, const char* fmt, ...);
int cuda_error(cudaError_t err, const char* where);
void count_launch(int n = 1);

#define QK_REQUIRE(cond, ...)                                        \
  do {                                                               \
    if (!(cond)) return ::qk::set_error(QK_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
  } while (0)

#define QK_LAUNCHED(where)                                           \
  do {                                                               \
    cudaError_t e_ = cudaGetLastError();                             \
    if (e_ != cudaSuccess) return ::qk::cuda_error(e_, where);       \
    ::qk::count_launch();                                            \
  } while (0)

inline cudaStream_t as_stream(qk_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Programmatic dependent launch: a kernel started with launch_dependent may begin (and run
// its prologue) while the previous kernel of the stream is still running; it must call
// pdl_wait() before touching anything that kernel (or an earlier one) writes or reads.
// pdl_trigger() lets the next dependent kernel be launched early. Both are no-ops when the
// kernel was launched normally.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                             Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

int sm_count();  // SMs of the current device (cached per device)
// The driver's cuTensorMapEncodeTiled, looked up once through the runtime (NULL if absent).
void* tensor_map_encoder();
// Opt a kernel into `bytes` of dynamic shared memory on the current device (once).
int allow_smem(const void* kernel, size_t bytes);

// ---------------------------------------------------------------------------------
// numeric boundaries
// ---------------------------------------------------------------------------------

// BF16 storage bits of x rounded to nearest even; NaN quieted by setting bit 22
// (the integer rule of the reference's rounded_bf16_float32).
__host__ __device__ __forceinline__ uint16_t bf16_bits_rne(float x) {
#ifdef __CUDA_ARCH__
  uint32_t b = __float_as_uint(x);
#else
  uint32_t b;
  __builtin_memcpy(&b, &x, 4);
#endif
  if ((b & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((b | 0x00400000u) >> 16);
  return static_cast<uint16_t>((b + 0x7fffu + ((b >> 16) & 1u)) >> 16);
}

__device__ __forceinline__ float bf16_round(float x) {
  return __uint_as_float(static_cast<uint32_t>(bf16_bits_rne(x)) << 16);
}

// bf16_round by the hardware conversion (cvt.rn.bf16.f32): the same result for finite and
// infinite values; a NaN comes out as the canonical quiet NaN instead of the quieted payload.
__device__ __forceinline__ uint16_t bf16_bits_hw(float x) {
  uint16_t r;
  asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float bf16_round_hw(float x) {
  return __uint_as_float(static_cast<uint32_t>(bf16_bits_hw(x)) << 16);
}

__device__ __forceinline__ float bf16_to_f32(uint16_t bits) {
  return __uint_as_float(static_cast<uint32_t>(bits) << 16);
}

// Exact FP16 -> FP32 expansion (subnormals and signed zero included).
__device__ __forceinline__ float f16_to_f32(uint16_t bits) {
  return __half2float(__ushort_as_half(bits));
}

// Two FP32 values -> packed BF16x2 (low half = a), hardware RNE (cvt.rn.bf16x2.f32).
// Used only on finite values, where it equals the integer rule above.
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));
  return r;
}

// numerics.py:13-14 accurate FP32 exp (AccuracyMode.HIGHEST): CUDA's expf, whose documented
// maximum error is 2 ulp, inside the reference's 5e-7 relative budget
// (numerics_validation.py:40). Every exponential of the kernels goes through it; qk_numerics
// evaluates it for the FP64 check.
__device__ __forceinline__ float exp_ref(float x) { return expf(x); }

// numerics.py:42-45 sigmoid: divide(x >= 0 ? 1 : e, 1 + e), e = exp(-|x|), IEEE divide.
__device__ __forceinline__ float sigmoid_ref(float x) {
  float e = exp_ref(-fabsf(x));
  return __fdiv_rn(x >= 0.f ? 1.f : e, __fadd_rn(1.f, e));
}

// numerics.py:48-51 softmax of one row of n values, in place, by one warp: the maximum,
// exp(x - max), a lane-strided FP32 sum folded by an XOR butterfly, then an IEEE divide.
// The router uses it for its probabilities; qk_numerics exposes it for the FP64 check.
__device__ __forceinline__ void softmax_row_warp(float* row, int n, int lane) {
  float mx = -INFINITY;
  for (int e = lane; e < n; e += 32) mx = fmaxf(mx, row[e]);
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
  for (int e = lane; e < n; e += 32) {
    const float ex = exp_ref(row[e] - mx);
    row[e] = ex;
    sum = __fadd_rn(sum, ex);
  }
  for (int o = 16; o > 0; o >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, o));
  for (int e = lane; e < n; e += 32) row[e] = __fdiv_rn(row[e], sum);
  __syncwarp();
}

// ---------------------------------------------------------------------------------
// tensor core: legacy warp MMA, used for the HBM-bound small-M paths
// ---------------------------------------------------------------------------------

// D[16x8] += A[16x16] * B[16x8], BF16 operands, FP32 accumulate.
// a[0]=(r g, k 2c..2c+1) a[1]=(r g+8, k 2c..) a[2]=(r g, k 2c+8..) a[3]=(r g+8, k 2c+8..)
// b[0]=(k 2c..2c+1, n g) b[1]=(k 2c+8.., n g); d[0..1]=(r g, n 2c..2c+1) d[2..3]=(r g+8, ..)
// with g = lane / 4 and c = lane % 4.
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Transpose of an 8x8 b16 matrix held in the mma fragment layout.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t r;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}

// ---------------------------------------------------------------------------------
// async bulk copies (TMA engine, 1-D, no multicast) and mbarriers
// ---------------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// Global -> shared bulk copy completing on `bar`. dst, src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// 16-byte asynchronous global -> shared copy (LSU path, L2 only), and its group control.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
// Arrive on `bar` (without adding to its expected count) once every cp.async this thread
// issued so far has completed.
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// L2 eviction-priority policies for bulk copies: data streamed once (weights) is evicted
// first, data that other CTAs read again soon (activation tiles) last.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// bulk_g2s with an L2 cache policy.
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, "
      "p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that may suspend the thread until the phase completes or `hint_ns` passes, so
// a waiting warp takes no issue slots from the warps doing work.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, "
      "p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after `limit` polls (each suspends for at most kWaitHintNs, so
// the wait ends within about four seconds) and returns false; the caller records
// QK_ERR_TIMEOUT and stops issuing work.
constexpr uint32_t kWaitLimit = 1u << 22;
constexpr uint32_t kWaitHintNs = 1000;

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  // Not unrolled: the loop is inlined at every wait of a kernel, and unrolled copies of it
  // made the projection kernels' code several times larger than their hot loops (a kernel
  // whose warps run different roles then misses in the instruction cache).
#pragma unroll 1
  for (uint32_t i = 0; i < kWaitLimit; ++i)
    if (mbar_try_wait_suspend(bar, parity, kWaitHintNs)) return true;
  return false;
}

// ---------------------------------------------------------------------------------
// small loads
// ---------------------------------------------------------------------------------

// Block-wide FP32 sum (all threads get the result): a warp butterfly, then the warps' sums
// added in warp order. `red` holds blockDim.x / 32 floats.
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();  // `red` may still be read by a previous call
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
  for (int w = 0; w < nw; ++w) s += red[w];
  return s;
}

// One-block-per-row kernels (256 threads) hold a BF16 row of up to kRowChunks x 256 x 8
// values in registers, 8 values per 16-byte chunk: thread t takes chunks t, t + 256, ...,
// issues all its loads before using them and accumulates chunk by chunk in value order;
// block_sum then adds the threads. Kernels that share this layout give the same bits.
constexpr int kRowBlock = 256;
constexpr int kRowChunks = 4;
constexpr int kMaxRowWidth = kRowChunks * kRowBlock * 8;  // 8192 values

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    f[2 * t] = __uint_as_float(w[t] << 16);
    f[2 * t + 1] = __uint_as_float(w[t] & 0xffff0000u);
  }
}

// Dot product of a BF16 row of H values with a BF16 vector in the row layout (FP32 fused
// multiply-adds), rounded to BF16: the shared expert's gate logit bf16(h . wsr)
// (math.py:282-283). Every thread of the 256-thread block calls it, or row_dot_load and
// later row_dot_finish (the loads in flight meanwhile).
struct RowDot {
  uint4 a[kRowChunks], b[kRowChunks];
};

__device__ __forceinline__ void row_dot_load(RowDot& r, const uint16_t* hrow, const uint16_t* wsr, int H) {
  const int nch = H / 8;
#pragma unroll
  for (int c = 0; c < kRowChunks; ++c) {
    const int i = threadIdx.x + c * kRowBlock;
    r.a[c] = i < nch ? reinterpret_cast<const uint4*>(hrow)[i] : make_uint4(0, 0, 0, 0);
    r.b[c] = i < nch ? reinterpret_cast<const uint4*>(wsr)[i] : make_uint4(0, 0, 0, 0);
  }
}

__device__ __forceinline__ float row_dot_finish(const RowDot& r, int H, float* red) {
  const int nch = H / 8;
  float s = 0.f;
#pragma unroll
  for (int c = 0; c < kRowChunks; ++c) {
    if (threadIdx.x + c * kRowBlock >= nch) break;
    float f[8], g[8];
    unpack8(r.a[c], f);
    unpack8(r.b[c], g);
#pragma unroll
    for (int t = 0; t < 8; ++t) s = fmaf(f[t], g[t], s);
  }
  return bf16_round(block_sum(s, red));
}

__device__ __forceinline__ float row_dot_bf16(const uint16_t* hrow, const uint16_t* wsr, int H, float* red) {
  RowDot r;
  row_dot_load(r, hrow, wsr, H);
  return row_dot_finish(r, H, red);
}

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 r;
  asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint4 lds_v4(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}

__device__ __forceinline__ uint32_t word(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

}  // namespace qk
