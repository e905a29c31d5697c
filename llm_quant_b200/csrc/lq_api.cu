// lq_api.cu -- status strings, per-thread error messages, launch counter.
#include <cstdarg>

#include "lq_common.cuh"

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
