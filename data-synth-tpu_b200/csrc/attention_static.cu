// Q8 decode attention whose split-KV scratch lives in a fixed array of the library's own
// device image, so the call needs no workspace from its caller.
//
// Why it exists: some embedders cannot give a kernel library device memory at the point
// of the call. One example is a foreign-function handler that receives only its operand
// and result buffers. Another is a serving loop whose device memory is sized and frozen
// before it starts. The regular entry point, qk_kv_q8_decode_attention, needs a
// caller-owned workspace of qk_kv_q8_attention_workspace_bytes() for the per-split
// partial (max, sum, output) rows. This entry point takes that scratch from
// `g_attn_scratch` instead.
//
// Limit: kStaticScratchBytes (16 MiB). The split kernel runs one CTA per SM and each CTA
// leaves at most two partial rows per KV head, so the workspace query never exceeds
// 2 * SMs * kv_heads * (16 + 8 * head_dim) * 4 bytes whatever B and S are: 4.9 MB for 2 KV
// heads at head_dim 256 and 9.9 MB for 8 KV heads at head_dim 128 on a 148-SM B200. On a
// 148-SM B200 the bound exceeds the array once kv_heads * head_dim reaches 2048 (8 KV heads
// of 256, 16 of 128: about 19.5-19.7 MB); such a geometry, or any whose query exceeds the
// array, is refused with QK_ERR_WORKSPACE before anything runs.
//
// Set-up: the first call on each device (the device current on the calling thread) looks
// up the array's device address with cudaGetSymbolAddress and caches it. That first call
// should therefore come before any stream capture. The cached address belongs to the
// device's primary context: after cudaDeviceReset (or any teardown of that context) the
// library must be reloaded before this entry point is called again. Nothing in the scratch
// has to start at zero: the split kernel writes every partial row before the merge kernel
// reads it.
//
// The scratch is one array per device. Two calls that can overlap on the same device (on
// different streams, or from different host threads) race on it. Calls issued in order on
// one stream are safe.
#include <atomic>

#include "common.cuh"

namespace qk {
namespace {

constexpr size_t kStaticScratchBytes = size_t(16) << 20;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_attn_scratch[kStaticScratchBytes];

std::atomic<void*> g_scratch_addr[kMaxDevices];

// Device address of g_attn_scratch on the current device (looked up once per device).
int static_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "qk_kv_q8_decode_attention_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(QK_ERR_INVALID_ARGUMENT, "device ordinal %d out of range", dev);
  void* p = g_scratch_addr[dev].load(std::memory_order_acquire);
  if (!p) {
    e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess)
      return cuda_error(e, "qk_kv_q8_decode_attention_noalloc: cudaGetSymbolAddress");
    g_scratch_addr[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return QK_OK;
}

}  // namespace
}  // namespace qk

using namespace qk;

extern "C" {

int qk_kv_q8_decode_attention_noalloc(const uint16_t* q, const int8_t* k_codes,
                                      const int8_t* v_codes, const uint16_t* k_scale,
                                      const uint16_t* v_scale, const int32_t* indices,
                                      const uint8_t* valid, const int32_t* lengths,
                                      const uint16_t* gate, int B, int S, int T, int hq,
                                      int kv_heads, int head_dim, uint16_t* out,
                                      qk_stream_t stream) {
  const size_t need = qk_kv_q8_attention_workspace_bytes(B, S, hq, kv_heads, head_dim);
  if (need > kStaticScratchBytes)
    return set_error(QK_ERR_WORKSPACE,
                     "qk_kv_q8_decode_attention_noalloc: this geometry needs %zu bytes of split "
                     "scratch, above the fixed %zu; call qk_kv_q8_decode_attention with a workspace",
                     need, kStaticScratchBytes);
  void* scratch = nullptr;
  if (need > 0) {
    const int rc = static_scratch(&scratch);
    if (rc) return rc;
  }
  return qk_kv_q8_decode_attention(q, k_codes, v_codes, k_scale, v_scale, indices, valid, lengths,
                                   gate, B, S, T, hq, kv_heads, head_dim, out, scratch,
                                   need > 0 ? kStaticScratchBytes : 0, stream);
}

}  // extern "C"
