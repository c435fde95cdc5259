// dial_check_bounded_wait: a self-test of the bounded-wait error path that
// every pipelined kernel of this library relies on (include/dial_cuda.h).
//
// The kernel runs the same helpers the GEMV and GEMM kernels use: it starts a
// real bulk copy into shared memory on one mbarrier, then waits (tma::mbar_wait,
// limit tma::kWaitNs = 1 s on %globaltimer) on a second mbarrier that nothing
// ever signals.  The wait gives up, records DIAL_ERR_TIMEOUT in the device error
// flag, and the kernel drains the copy still tracked by the first barrier
// (tma::mbar_drain, bounded as well) before it returns -- the order a kernel
// that gives up follows.  The context stays usable: nothing faults, traps or
// spins without a limit.  One CTA of 32 threads, 256 bytes of shared memory.
#include "common.cuh"
#include "tma.cuh"

namespace dial {

int* device_error_ptr();

namespace {

__global__ void bounded_wait_selftest_kernel(const uint4* __restrict__ src, int* err,
                                             int* __restrict__ result) {
  __shared__ __align__(128) uint4 buf[16];
  __shared__ __align__(8) unsigned long long bars[2];
  const uint32_t copy_bar = tma::smem_u32(&bars[0]), idle_bar = tma::smem_u32(&bars[1]);
  if (threadIdx.x == 0) {
    tma::mbar_init(copy_bar, 1);
    tma::mbar_init(idle_bar, 1);  // one arrival expected; none will come
    tma::fence_barrier_init();
    tma::mbar_expect_tx(copy_bar, sizeof(buf));
    tma::load_1d(tma::smem_u32(buf), src, sizeof(buf), copy_bar);
  }
  __syncwarp();
  const bool ok = __all_sync(0xffffffffu, tma::mbar_wait(idle_bar, 0, err));
  if (threadIdx.x == 0) {
    // drain the copy that is still tracked, as a kernel that gives up does
    const unsigned long long deadline = tma::global_ns() + tma::kWaitNs;
    const bool drained = tma::mbar_drain(copy_bar, 0, deadline);
    result[0] = ok ? 1 : 0;        // the wait must not have succeeded
    result[1] = drained ? 1 : 0;   // and the copy must have landed
    result[2] = drained ? (int)buf[3].x : -1;
  }
}

}  // namespace
}  // namespace dial

using namespace dial;

extern "C" dial_status dial_check_bounded_wait(const void* src, int* result, dial_stream stream) {
  clear_error();
  if (!src || !result) return fail(DIAL_ERR_INVALID_ARG, "null pointer");
  if (!aligned16(src)) return fail(DIAL_ERR_MISALIGNED, "src must be 16-byte aligned");
  int* err = device_error_ptr();
  if (!err) return fail(DIAL_ERR_CUDA, "device error flag is unavailable");
  bounded_wait_selftest_kernel<<<1, 32, 0, as_stream(stream)>>>(static_cast<const uint4*>(src), err,
                                                               result);
  return check_launch("bounded_wait_selftest_kernel");
}
