// Library-level C ABI: version, last-error text, launch counter.
#include <atomic>
#include <cstdarg>
#include <cstdio>

#include "common.cuh"

namespace qk {

namespace {
thread_local char g_last_error[512] = "";
std::atomic<uint64_t> g_launches{0};
int g_sm_count[64] = {0};
}  // namespace

int set_error(int status, const char* fmt, ...) {
  va_list args;
  va_start(args, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, args);
  va_end(args);
  return status;
}

int cuda_error(cudaError_t err, const char* where) {
  return set_error(QK_ERR_CUDA, "%s: %s", where, cudaGetErrorString(err));
}

void count_launch(int n) { g_launches.fetch_add(static_cast<uint64_t>(n)); }

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

int allow_smem(const void* kernel, size_t bytes) {
  // The attribute is per (kernel, device) and is a ceiling: remember the largest value
  // set so far and raise it when a launch needs more (never lower it).
  static thread_local const void* done_kernel[256];
  static thread_local int done_dev[256];
  static thread_local size_t done_bytes[256];
  static thread_local int n_done = 0;
  if (bytes <= 48 * 1024) return QK_OK;  // below the default limit: nothing to opt into
  int dev = 0;
  cudaGetDevice(&dev);
  int slot = -1;
  for (int i = 0; i < n_done; ++i)
    if (done_kernel[i] == kernel && done_dev[i] == dev) {
      if (done_bytes[i] >= bytes) return QK_OK;
      slot = i;
    }
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(bytes));
  if (e != cudaSuccess) return cuda_error(e, "cudaFuncSetAttribute");
  if (slot < 0 && n_done < 256) slot = n_done++;
  if (slot >= 0) {
    done_kernel[slot] = kernel;
    done_dev[slot] = dev;
    done_bytes[slot] = bytes;
  }
  return QK_OK;
}

void* tensor_map_encoder() {
  static void* fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return p;
  }();
  return fn;
}

}  // namespace qk

extern "C" {

const char* qk_version(void) { return "qk_b200 0.1 sm_100a"; }

const char* qk_last_error(void) { return qk::g_last_error; }

uint64_t qk_launch_count(void) { return qk::g_launches.load(); }

}  // extern "C"
