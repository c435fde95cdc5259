// Host-side runtime pieces shared by every entry point: the thread-local error
// slot, the launch counter, status strings and the SM-count cache.
//
// The reference reports failures as candle_core::Error::Msg strings
// (worker_w8a16.rs:369-378, :410-416, :465-467); across this C ABI the same
// information is a dial_status plus the message returned by dial_last_error().
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "common.cuh"

namespace dial {

namespace {
thread_local char g_msg[512] = {0};
std::atomic<uint64_t> g_launches{0};
std::mutex g_sm_mu;
int g_sm_count[64] = {0};
}  // namespace

void clear_error() { g_msg[0] = 0; }

dial_status fail(dial_status s, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return s;
}

dial_status cuda_fail(cudaError_t e, const char* what) {
  return fail(DIAL_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

dial_status check_launch(const char* kernel_name) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, kernel_name);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return DIAL_OK;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("DIAL_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lk(g_sm_mu);
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

}  // namespace dial

extern "C" {

const char* dial_status_string(dial_status s) {
  switch (s) {
    case DIAL_OK: return "ok";
    case DIAL_ERR_INVALID_ARG: return "invalid argument";
    case DIAL_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype";
    case DIAL_ERR_MISALIGNED: return "misaligned pointer or stride";
    case DIAL_ERR_SHAPE: return "unsupported shape";
    case DIAL_ERR_CUDA: return "CUDA error";
    case DIAL_ERR_NCCL: return "NCCL error";
    case DIAL_ERR_TIMEOUT: return "timeout";
    case DIAL_ERR_NO_DEVICE: return "no sm_100 device";
    default: return "unknown status";
  }
}

const char* dial_last_error(void) { return dial::g_msg; }

int dial_abi_version(void) { return DIAL_ABI_VERSION; }

uint64_t dial_launch_count(void) { return dial::g_launches.load(std::memory_order_relaxed); }

}  // extern "C"
