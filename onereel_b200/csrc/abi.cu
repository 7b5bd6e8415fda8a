// Library-wide C entry points: version and error strings.
#include <cstdio>
#include <cstring>

#include "orl_common.h"
#include "ptx.cuh"

extern "C" const char* orl_version(void) { return "onereel_b200 0.1.0 (sm_100a)"; }

extern "C" const char* orl_error_string(int code) {
  switch (code) {
    case ORL_OK: return "ok";
    case ORL_ERR_ARG: return "invalid argument";
    case ORL_ERR_ALIGN: return "pointer, offset or size not 16-byte aligned";
    case ORL_ERR_UNSUPPORTED: return "unsupported head_dim (64 or 128)";
    case ORL_ERR_DRIVER: return "cuTensorMapEncodeTiled unavailable from the driver";
    case ORL_ERR_TENSOR_MAP: return "the driver rejected a TMA tensor map";
    case ORL_ERR_LAUNCH: return "kernel launch failed";
    case ORL_ERR_CAPACITY: return "caller buffer too small";
    case ORL_ERR_COMM: return "NCCL error (communicator aborted after a failed wait)";
    case ORL_ERR_TIMEOUT: return "collective wait timed out (communicator aborted)";
    default: return "unknown error";
  }
}

extern "C" int orl_error_bits_describe(int bits, char* buf, int cap) {
  if (buf == nullptr || cap <= 0) return ORL_ERR_ARG;
  buf[0] = 0;
  const struct { int bit; const char* what; } names[] = {
      {orl::kErrTimeoutLoad, "producer timed out waiting for a free K/V stage"},
      {orl::kErrTimeoutMma, "MMA warp timed out waiting for a tile or for P"},
      {orl::kErrTimeoutSoftmax, "softmax warps timed out waiting for S or O"},
      {orl::kErrTimeoutDrain, "wind-down timed out waiting for in-flight copies"},
      {orl::kErrTimeoutPack, "pack kernel timed out waiting for a bulk copy"},
      {orl::kErrPlan, "cu_seqlens rejected on the device (decreasing or outside the tensors): nothing computed"},
      {orl::kErrPeerTimeout, "a peer GPU did not reach the device barrier in time"},
  };
  int n = 0;
  for (const auto& e : names)
    if (bits & e.bit) n += snprintf(buf + n, n < cap ? cap - n : 0, "%s%s", n ? "; " : "", e.what);
  return ORL_OK;
}

// Failure-path self test: one CTA initialises an mbarrier that nothing arrives at and waits on it with the kernel's
// bounded wait shortened to limit_ns; the wait gives up, the kernel records the timeout bit and returns. The host
// reads the status: a pipeline wait that runs out ends the kernel with an error word, never a hang or a trap.
namespace {
__global__ void selftest_timeout_kernel(int* status, unsigned long long limit_ns) {
  __shared__ __align__(8) unsigned long long bar;
  if (threadIdx.x != 0) return;
  const uint32_t b = orl::smem_u32(&bar);
  orl::mbar_init(b, 1);
  orl::fence_mbar_init();
  const unsigned long long t0 = orl::global_ns();
  int bits = 0;
  while (!orl::mbar_try_wait(b, 0)) {
    if (orl::global_ns() - t0 > limit_ns) {
      bits |= orl::kErrTimeoutSoftmax;
      break;
    }
  }
  *status = bits;
}
}  // namespace

extern "C" int orl_selftest_timeout(int* status_dev, unsigned long long limit_ns, void* stream) {
  if (status_dev == nullptr || limit_ns == 0 || limit_ns > orl::kWaitLimitNs) return ORL_ERR_ARG;
  selftest_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status_dev, limit_ns);
  return cudaGetLastError() == cudaSuccess ? ORL_OK : ORL_ERR_LAUNCH;
}
