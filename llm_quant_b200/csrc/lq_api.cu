// lq_api.cu -- status strings, per-thread error messages, launch counter,
// and the probe of the kernels' bounded device-side wait.
#include <cstdarg>

#include "lq_common.cuh"
#include "lq_tma.cuh"

namespace lq {

std::atomic<uint64_t> g_launches{0};

namespace {
thread_local char t_err[512] = "";
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err, sizeof(t_err), fmt, ap);
  va_end(ap);
}

}  // namespace lq

extern "C" const char* lq_last_error(void) { return lq::t_err; }

extern "C" const char* lq_status_string(int status) {
  switch (status) {
    case LQ_OK: return "ok";
    case LQ_EINVAL: return "invalid argument";
    case LQ_EDTYPE: return "unsupported dtype";
    case LQ_ECUDA: return "CUDA error";
    case LQ_ETIMEOUT: return "device wait timed out";
    case LQ_EALIGN: return "misaligned pointer";
    case LQ_ERANGE: return "size above supported maximum";
    default: return "unknown status";
  }
}

extern "C" int lq_version(void) { return 100; }

extern "C" uint64_t lq_launch_count(void) { return lq::g_launches.load(std::memory_order_relaxed); }

// ---------------------------------------------------------------------------
// Probe of the bounded wait every pipelined kernel uses on its mbarriers
// (mbar_wait_for in lq_tma.cuh): one warp initialises an mbarrier that
// expects one arrival, arrives on it or not, and waits with the given limit.
// out[0] = LQ_OK when the wait returned because the phase completed,
// LQ_ETIMEOUT when it gave up; out[1] = the nanoseconds the wait took.  A
// wait that never completes therefore ends the kernel with a status instead
// of a hang, and the context stays usable.
// ---------------------------------------------------------------------------
namespace lq {
namespace {
__global__ void wait_probe_kernel(int64_t limit_ns, int arrive, int64_t* out) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  if (arrive && threadIdx.x == 0) mbar_arrive(&bar);
  __syncwarp();
  const uint64_t t0 = global_ns();
  const bool ok = mbar_wait_for(&bar, 0, (uint64_t)limit_ns);
  const uint64_t t1 = global_ns();
  if (threadIdx.x == 0) {
    out[0] = ok ? LQ_OK : LQ_ETIMEOUT;
    out[1] = (int64_t)(t1 - t0);
  }
}
}  // namespace
}  // namespace lq

extern "C" int lq_wait_probe(int64_t limit_ns, int arrive, int64_t* out, void* stream) {
  using namespace lq;
  LQ_REQUIRE(out, LQ_EINVAL, "NULL pointer");
  LQ_REQUIRE(limit_ns >= 0 && limit_ns <= 10000000000LL, LQ_ERANGE,
             "wait limit %lld ns outside [0, 10 s]", (long long)limit_ns);
  wait_probe_kernel<<<1, 32, 0, as_stream(stream)>>>(limit_ns, arrive, out);
  return launched("wait_probe_kernel");
}
