// Q8 KV cache codec, append and gathers (reference cache layout).
//
// Codec: qwen38_tpu/attention_cache.py:15-23 (quantize): per `group` channels
//   scale = bf16(max|x| / 127), codes = clip(rint(x / (scale == 0 ? 1 : scale)), +-127).
// The division is IEEE (the reference's own oracle, validation.py:44-48, divides with
// NumPy); rintf rounds half to even like jnp.rint.
// Layout: codes int8 [B, T, kv*hd]; scale planes BF16 [B*G, T], G = kv*hd/group
// (attention_cache.py:26-43, engine.py:350-369). Time index rule of gathers: negative
// indices wrap once, then clamp to [0, T-1] (tests/test_qwen38_kv_gather.py:22-32).
#include "common.cuh"

namespace qk {
namespace {

__device__ __forceinline__ float load_in(const void* p, int64_t i, int bf16) {
  return bf16 ? bf16_to_f32(static_cast<const uint16_t*>(p)[i]) : static_cast<const float*>(p)[i];
}

// Quantise one element whose group occupies `group` consecutive lanes of the warp.
// All 32 lanes must call (inactive lanes pass x = 0).
__device__ __forceinline__ void quantize_lane(float x, int group, int8_t& code, uint16_t& scale_bits) {
  float amax = fabsf(x);
  for (int o = group >> 1; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = bf16_round(__fdiv_rn(amax, 127.f));
  const float divisor = scale == 0.f ? 1.f : scale;
  const float q = fminf(fmaxf(rintf(__fdiv_rn(x, divisor)), -127.f), 127.f);
  code = static_cast<int8_t>(q);
  scale_bits = bf16_bits_rne(scale);
}

__device__ __forceinline__ int wrap_clamp(int t, int T) {
  if (t < 0) t += T;
  return t < 0 ? 0 : (t >= T ? T - 1 : t);
}

__global__ void quantize_kernel(const void* __restrict__ x, int in_bf16, int64_t total, int width,
                                int group, int8_t* __restrict__ codes, uint16_t* __restrict__ scales) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x; base < total; base += stride) {
    const int64_t i = base + threadIdx.x;  // warps never straddle a group: group | 32, width % group == 0
    const bool in = i < total;
    int8_t code;
    uint16_t sb;
    quantize_lane(in ? load_in(x, i, in_bf16) : 0.f, group, code, sb);
    if (in) {
      codes[i] = code;
      if (i % group == 0) scales[i / group] = sb;
    }
  }
}

// write_quantized: one thread per (input row, tensor k/v, channel). With W > 1 (a prompt
// chunk) input row r is token r % W of cache row r / W, written at time time[r / W] + r % W.
__global__ void append_kernel(const void* __restrict__ key, const void* __restrict__ value, int in_bf16,
                              const int32_t* __restrict__ time, const uint8_t* __restrict__ active,
                              int8_t* k_codes, int8_t* v_codes, uint16_t* k_scale, uint16_t* v_scale,
                              int B, int T, int D, int group, int W = 1) {
  pdl_wait();  // launched as a programmatic dependent: the keys' and values' producer first
  pdl_trigger();
  const int64_t total = static_cast<int64_t>(B) * W * 2 * D;
  const int G = D / group;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x; base < total; base += stride) {
    const int64_t i = base + threadIdx.x;
    const bool in = i < total;
    const int b = in ? static_cast<int>(i / (2 * D)) : 0;
    const int which = in ? static_cast<int>((i / D) & 1) : 0;
    const int col = in ? static_cast<int>(i % D) : 0;
    const void* src = which ? value : key;
    int8_t code;
    uint16_t sb;
    quantize_lane(in ? load_in(src, static_cast<int64_t>(b) * D + col, in_bf16) : 0.f, group, code, sb);
    const int row = b / W, tok = b - row * W;  // cache row and token of the chunk
    if (!in || (active && !active[row])) continue;
    int t = time[row];
    if (t < 0) t += T;
    t += tok;
    if (t < 0 || t >= T) continue;  // out-of-range scatter updates are dropped
    int8_t* codes = which ? v_codes : k_codes;
    uint16_t* plane = which ? v_scale : k_scale;
    codes[(static_cast<int64_t>(row) * T + t) * D + col] = code;
    if (col % group == 0) plane[(static_cast<int64_t>(row) * G + col / group) * T + t] = sb;
  }
}

__global__ void gather_scales_kernel(const uint16_t* __restrict__ plane, const int32_t* __restrict__ idx,
                                     int B, int S, int G, int T, uint16_t* __restrict__ out) {
  const int64_t total = static_cast<int64_t>(B) * S * G;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int g = static_cast<int>(i % G);
    const int64_t bs = i / G;
    const int b = static_cast<int>(bs / S);
    const int t = wrap_clamp(idx[bs], T);
    out[i] = plane[(static_cast<int64_t>(b) * G + g) * T + t];
  }
}

__global__ void read_kernel(const int8_t* __restrict__ codes, const uint16_t* __restrict__ plane,
                            const int32_t* __restrict__ idx, int B, int S, int T, int D, int group,
                            int out_bf16, void* __restrict__ out) {
  const int64_t total = static_cast<int64_t>(B) * S * D;
  const int G = D / group;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int col = static_cast<int>(i % D);
    const int64_t bs = i / D;
    const int b = static_cast<int>(bs / S);
    const int t = wrap_clamp(idx[bs], T);
    const float code = static_cast<float>(codes[(static_cast<int64_t>(b) * T + t) * D + col]);
    const float scale = bf16_to_f32(plane[(static_cast<int64_t>(b) * G + col / group) * T + t]);
    const float v = __fmul_rn(code, scale);  // exact: 8-bit code x 8-bit scale
    if (out_bf16) static_cast<uint16_t*>(out)[i] = bf16_bits_rne(v);
    else static_cast<float*>(out)[i] = v;
  }
}

int grid_for(int64_t total, int block) {
  int64_t g = (total + block - 1) / block;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  return static_cast<int>(g < 1 ? 1 : (g > cap ? cap : g));
}

bool pow2_le32(int g) { return g >= 1 && g <= 32 && (g & (g - 1)) == 0; }

}  // namespace
}  // namespace qk

using namespace qk;

extern "C" {

int qk_kv_q8_quantize(const void* x, int in_dtype, int64_t rows, int width, int group, int8_t* codes,
                      uint16_t* scales, qk_stream_t stream) {
  QK_REQUIRE(in_dtype == QK_OUT_F32 || in_dtype == QK_OUT_BF16, "in_dtype must be F32 or BF16");
  QK_REQUIRE(pow2_le32(group) && width > 0 && width % group == 0, "width must divide into groups of a power of two <= 32");
  QK_REQUIRE(rows >= 0, "rows must be non-negative");
  if (rows == 0) return QK_OK;
  QK_REQUIRE(x && codes && scales, "null pointer");
  const int64_t total = rows * width;
  quantize_kernel<<<grid_for(total, 256), 256, 0, as_stream(stream)>>>(x, in_dtype == QK_OUT_BF16, total, width, group, codes, scales);
  QK_LAUNCHED("quantize_kernel");
  return QK_OK;
}

int qk_kv_q8_append(const void* key, const void* value, int in_dtype, const int32_t* time,
                    const uint8_t* active, int8_t* k_codes, int8_t* v_codes, uint16_t* k_scale,
                    uint16_t* v_scale, int B, int T, int kv_heads, int head_dim, qk_stream_t stream) {
  QK_REQUIRE(in_dtype == QK_OUT_F32 || in_dtype == QK_OUT_BF16, "in_dtype must be F32 or BF16");
  QK_REQUIRE(B >= 0 && T > 0 && kv_heads > 0 && head_dim > 0, "invalid cache geometry");
  const int group = head_dim < 32 ? head_dim : 32;  // config.py:91-93
  QK_REQUIRE(pow2_le32(group) && head_dim % group == 0, "KV head dimension must divide into cache quantization groups");
  if (B == 0) return QK_OK;
  QK_REQUIRE(key && value && time && k_codes && v_codes && k_scale && v_scale, "null pointer");
  const int D = kv_heads * head_dim;
  const cudaError_t e = launch_dependent(append_kernel, dim3(grid_for(static_cast<int64_t>(B) * 2 * D, 256)), dim3(256),
                                         0, as_stream(stream), key, value, static_cast<int>(in_dtype == QK_OUT_BF16),
                                         time, active, k_codes, v_codes, k_scale, v_scale, B, T, D, group, 1);
  if (e != cudaSuccess) return cuda_error(e, "append_kernel");
  count_launch();
  return QK_OK;
}

int qk_kv_q8_append_chunk(const void* key, const void* value, int in_dtype, const int32_t* start,
                          const uint8_t* active, int8_t* k_codes, int8_t* v_codes, uint16_t* k_scale,
                          uint16_t* v_scale, int B, int W, int T, int kv_heads, int head_dim,
                          qk_stream_t stream) {
  QK_REQUIRE(in_dtype == QK_OUT_F32 || in_dtype == QK_OUT_BF16, "in_dtype must be F32 or BF16");
  QK_REQUIRE(B >= 0 && W >= 1 && T > 0 && kv_heads > 0 && head_dim > 0, "invalid cache geometry");
  const int group = head_dim < 32 ? head_dim : 32;  // config.py:91-93
  QK_REQUIRE(pow2_le32(group) && head_dim % group == 0, "KV head dimension must divide into cache quantization groups");
  if (B == 0) return QK_OK;
  QK_REQUIRE(key && value && start && k_codes && v_codes && k_scale && v_scale, "null pointer");
  const int D = kv_heads * head_dim;
  append_kernel<<<grid_for(static_cast<int64_t>(B) * W * 2 * D, 256), 256, 0, as_stream(stream)>>>(
      key, value, in_dtype == QK_OUT_BF16, start, active, k_codes, v_codes, k_scale, v_scale, B, T, D, group, W);
  QK_LAUNCHED("append_kernel");
  return QK_OK;
}

int qk_kv_q8_gather_scales(const uint16_t* plane, const int32_t* indices, int B, int S, int groups,
                           int T, uint16_t* out, qk_stream_t stream) {
  QK_REQUIRE(B >= 0 && S >= 0 && groups > 0 && T > 0, "Scale plane must be [batch * groups, time] for [batch, selected] indices");
  if (B == 0 || S == 0) return QK_OK;
  QK_REQUIRE(plane && indices && out, "null pointer");
  gather_scales_kernel<<<grid_for(static_cast<int64_t>(B) * S * groups, 256), 256, 0, as_stream(stream)>>>(plane, indices, B, S, groups, T, out);
  QK_LAUNCHED("gather_scales_kernel");
  return QK_OK;
}

int qk_kv_q8_read(const int8_t* codes, const uint16_t* plane, const int32_t* indices, int B, int S,
                  int T, int kv_heads, int head_dim, int out_dtype, void* out, qk_stream_t stream) {
  QK_REQUIRE(out_dtype == QK_OUT_F32 || out_dtype == QK_OUT_BF16, "out_dtype must be F32 or BF16");
  QK_REQUIRE(B >= 0 && S >= 0 && T > 0 && kv_heads > 0 && head_dim > 0, "invalid cache geometry");
  const int group = head_dim < 32 ? head_dim : 32;
  QK_REQUIRE(head_dim % group == 0, "KV head dimension must divide into cache quantization groups");
  if (B == 0 || S == 0) return QK_OK;
  QK_REQUIRE(codes && plane && indices && out, "null pointer");
  const int D = kv_heads * head_dim;
  read_kernel<<<grid_for(static_cast<int64_t>(B) * S * D, 256), 256, 0, as_stream(stream)>>>(
      codes, plane, indices, B, S, T, D, group, out_dtype == QK_OUT_BF16, out);
  QK_LAUNCHED("read_kernel");
  return QK_OK;
}

}  // extern "C"
