// lq_common.cuh -- shared device helpers for liblq_sm100.so.
//
// Numeric model (matches the reference's PyTorch CPU kernels): every
// elementwise op computes in fp32 with IEEE round-to-nearest-even
// (explicit __f*_rn intrinsics, so no FMA contraction can merge two ops) and
// rounds once to the op's result dtype.  Reductions are exact; NaN anywhere in
// a reduction makes the result NaN (torch.amin / amax semantics).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstdio>
#include <string>
#include <utility>

#include "../../include/lq_sm100.h"

namespace lq {

// ---------------------------------------------------------------------------
// host-side status plumbing
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
extern std::atomic<uint64_t> g_launches;

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Check the launch that was just enqueued; count it.
inline int launched(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
    return LQ_ECUDA;
  }
  return LQ_OK;
}

#define LQ_REQUIRE(cond, code, ...) \
  do {                              \
    if (!(cond)) {                  \
      ::lq::set_error(__VA_ARGS__); \
      return (code);                \
    }                               \
  } while (0)

// Programmatic dependent launch.  A kernel launched with launch_pdl() may be
// scheduled before the kernel ahead of it in the stream has finished;
// pdl_wait() blocks until that kernel has completed and its memory writes are
// visible (a no-op after an ordinary launch), so a kernel calls it before its
// first global-memory access -- the stream-ordered allocator may have handed
// it memory the previous kernel still uses.  pdl_trigger() lets the next
// kernel's blocks launch before this one has finished.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
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
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Return the status of a helper that failed (it has already set the error).
#define LQ_TRY(expr)                  \
  do {                                \
    const int lq_rc_ = (expr);        \
    if (lq_rc_ != LQ_OK) return lq_rc_; \
  } while (0)

inline bool is_float_dtype(int dt) { return dt == LQ_F32 || dt == LQ_F16 || dt == LQ_BF16; }
inline int dtype_size(int dt) {
  switch (dt) {
    case LQ_F32: case LQ_I32: return 4;
    case LQ_F16: case LQ_BF16: case LQ_I16: return 2;
    case LQ_I8: case LQ_U8: return 1;
    case LQ_I64: return 8;
    default: return 0;
  }
}
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

inline int qmin_of(int n_bits, int sym) { return sym ? -(1 << (n_bits - 1)) : 0; }
inline int qmax_of(int n_bits, int sym) { return sym ? (1 << (n_bits - 1)) - 1 : (1 << n_bits) - 1; }

// ---------------------------------------------------------------------------
// storage types
// ---------------------------------------------------------------------------
template <typename T> struct Ty;
template <> struct Ty<float> {
  static constexpr int code = LQ_F32;
  __device__ __forceinline__ static float to_f(float v) { return v; }
  __device__ __forceinline__ static float from_f(float v) { return v; }
  __device__ __forceinline__ static float round(float v) { return v; }
};
template <> struct Ty<__half> {
  static constexpr int code = LQ_F16;
  __device__ __forceinline__ static float to_f(__half v) { return __half2float(v); }
  __device__ __forceinline__ static __half from_f(float v) { return __float2half_rn(v); }
  __device__ __forceinline__ static float round(float v) { return __half2float(__float2half_rn(v)); }
};
// bf16 -> fp32 is a 16-bit shift (exact, one ALU op); fp32 -> bf16 rounding
// uses the hardware round-to-nearest-even conversion.
template <> struct Ty<__nv_bfloat16> {
  static constexpr int code = LQ_BF16;
  __device__ __forceinline__ static float to_f(__nv_bfloat16 v) {
    return __uint_as_float((uint32_t)__bfloat16_as_ushort(v) << 16);
  }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  __device__ __forceinline__ static float round(float v) {
    return __uint_as_float((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v)) << 16);
  }
};

// Round an fp32 value to the dtype named by a runtime code.
__device__ __forceinline__ float round_to(int dt, float v) {
  if (dt == LQ_F16) return Ty<__half>::round(v);
  if (dt == LQ_BF16) return Ty<__nv_bfloat16>::round(v);
  return v;
}

// One torch op in dtype T: fp32 IEEE op, then round to T.
template <typename T> __device__ __forceinline__ float tdiv(float a, float b) {
  return Ty<T>::round(__fdiv_rn(a, b));
}
template <typename T> __device__ __forceinline__ float tadd(float a, float b) {
  return Ty<T>::round(__fadd_rn(a, b));
}
template <typename T> __device__ __forceinline__ float tsub(float a, float b) {
  return Ty<T>::round(__fsub_rn(a, b));
}
template <typename T> __device__ __forceinline__ float tmul(float a, float b) {
  return Ty<T>::round(__fmul_rn(a, b));
}

// NF4_TABLE as float32 (qlora.py:50-55).
static __device__ __constant__ float kNF4[16] = {
    -1.0f, -0.6962f, -0.5251f, -0.3949f, -0.2844f, -0.1848f, -0.0911f, 0.0f,
    0.0796f, 0.1609f, 0.2461f, 0.3379f, 0.4407f, 0.5626f, 0.7230f, 1.0f};

// torch.clamp(v, lo, hi): NaN passes, -0.0 is kept.
__device__ __forceinline__ float tclamp(float v, float lo, float hi) {
  v = (v < lo) ? lo : v;
  return (v > hi) ? hi : v;
}

// torch.clamp(t, lo, hi) on a tensor of dtype T: the scalar bounds are
// converted to T first, so a bound T cannot hold acts as its rounded value
// (qmax = 4095 clamps to 4096 in bf16).
template <typename T>
__device__ __forceinline__ float tclamp_t(float v, float lo, float hi) {
  return tclamp(v, Ty<T>::round(lo), Ty<T>::round(hi));
}

// torch.round: half to even, sign of zero kept.
__device__ __forceinline__ float trint(float v) { return rintf(v); }

// Value of ste_round(t) = t + (round(t) - t): round(t) with zero results
// turned into +0.0 and +-inf turned into NaN (core/quantizer.py:32-34).
__device__ __forceinline__ float tste(float t) {
  float r = rintf(t);
  float d = __fsub_rn(r, t);
  return __fadd_rn(t, d);
}

// float -> intN the way torch's CPU cast does: truncation through int32,
// NaN / inf -> INT32_MIN, then the low bits.
__device__ __forceinline__ int32_t tcast_i32(float v) {
  if (!(fabsf(v) < 2147483648.0f)) return INT32_MIN;  // NaN, inf, out of range
  return static_cast<int32_t>(v);
}

// NaN-propagating min / max (PTX min.NaN / max.NaN: a NaN operand gives NaN),
// the semantics of torch.amin / torch.amax.
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float fmin_nan(float a, float b) {
  float r;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// Min / max accumulator; NaN anywhere makes both NaN.  For symmetric
// quantization only mx is used (fed |x|), so its shuffles skip mn.
struct MinMax {
  float mn, mx;
  __device__ __forceinline__ void init() {
    mn = __int_as_float(0x7f800000);
    mx = __int_as_float(0xff800000);
  }
  __device__ __forceinline__ void add(float v) {
    mn = fmin_nan(mn, v);
    mx = fmax_nan(mx, v);
  }
  // v must be >= 0 or NaN with a clear sign bit (callers pass fabsf(x)):
  // then the integer order of the bit patterns is the float order and any
  // NaN is above +inf, so an integer max propagates NaN like torch.amax.
  __device__ __forceinline__ void add_max(float v) {
    mx = __int_as_float(max(__float_as_int(mx), __float_as_int(v)));
  }
  __device__ __forceinline__ void merge(const MinMax& o) {
    mn = fmin_nan(mn, o.mn);
    mx = fmax_nan(mx, o.mx);
  }
  __device__ __forceinline__ void shfl_xor_merge(int mask, bool max_only = false) {
    if (!max_only) mn = fmin_nan(mn, __shfl_xor_sync(0xffffffffu, mn, mask));
    mx = fmax_nan(mx, __shfl_xor_sync(0xffffffffu, mx, mask));
  }
  __device__ __forceinline__ bool has_nan() const { return (mn != mn) || (mx != mx); }
};

// Scale / zero point from a group's reduction (core/quantizer.py:64-104,
// kv_cache_quant.py:129-137).  For symmetric quantization only mx is used
// and it must hold max |x|.
template <typename T>
__device__ __forceinline__ void qparams_from(const MinMax& r, bool sym, float qmin, float qmax,
                                             float lo_T, float& scale, float& zp) {
  if (sym) {
    float amax = r.mx;
    amax = (amax < lo_T) ? lo_T : amax;  // clamp(min=1e-12) in T; NaN passes
    scale = tdiv<T>(amax, qmax);
    zp = 0.0f;
  } else {
    const float mn = r.mn, mx = r.mx;  // both NaN if the group holds a NaN
    float rng = tsub<T>(mx, mn);
    rng = (rng < lo_T) ? lo_T : rng;
    scale = tdiv<T>(rng, qmax - qmin);
    zp = tclamp_t<T>(trint(tdiv<T>(-mn, scale)), qmin, qmax);
  }
}

// 1e-12 converted to T (the scalar of clamp(min=1e-12)): 0 in fp16.
template <typename T> inline float lo_clamp_value();
template <> inline float lo_clamp_value<float>() { return 1e-12f; }
template <> inline float lo_clamp_value<__half>() { return __half2float(__float2half_rn(1e-12f)); }
template <> inline float lo_clamp_value<__nv_bfloat16>() {
  return __bfloat162float(__float2bfloat16_rn(1e-12f));
}

// 16-byte vector of T.
template <typename T> struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
  union {
    uint4 u;
    T v[N];
  };
};

__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
// 32 bytes (one whole sector) per thread; p must be 32-byte aligned
__device__ __forceinline__ void ld_nc_v8(const void* p, uint4& a, uint4& b) {
  asm volatile("ld.global.nc.L1::no_allocate.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(a.x), "=r"(a.y), "=r"(a.z), "=r"(a.w), "=r"(b.x), "=r"(b.y), "=r"(b.z), "=r"(b.w)
               : "l"(p));
}
__device__ __forceinline__ void st_v4(void* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// lq_group.cu: group quantization with output-row remapping (see GroupArgs).
int group_quant_remap(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t group,
                      int n_bits, int symmetric, int mode, void* out, int out_dtype, void* scale,
                      void* zero_point, void* stream, int64_t rpp, int64_t opitch, int64_t ooff,
                      int64_t spitch, int64_t soff);

inline int num_sms() {
  static int n = [] {
    int dev = 0, v = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    return v > 0 ? v : 148;
  }();
  return n;
}

// Grid of at most one wave of resident blocks of `kernel` (grid-stride
// kernels then share their work evenly; a second, partly filled wave would run
// at lower occupancy), and at most `want` blocks.
template <typename K>
inline int resident_grid(K kernel, int threads, size_t smem, int64_t want) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess ||
      per_sm < 1) {
    cudaGetLastError();
    per_sm = 1;
  }
  const int64_t cap = (int64_t)num_sms() * per_sm;
  return (int)(want < 1 ? 1 : (want < cap ? want : cap));
}

// lq_lora_u for at most 16 tokens runs as one cluster of this many blocks
// (each a share of K); a kernel launched behind it leaves them their SMs.
constexpr int kLoraUSplitBlocks = 8;

}  // namespace lq
