// lq_affine.cu -- broadcast elementwise quantize / dequantize / fake-quant with
// caller-given qparams, and the whole-tensor / per-channel qparams reductions.
//
// quantize_tensor and dequantize_tensor (core/quantizer.py:115-140) accept
// any broadcastable scale / zero point and follow torch type promotion; the
// caller passes each op's result dtype, the kernel does fp32 math and rounds
// after every op.  Operands are addressed through per-dim element strides
// over a broadcast shape of up to 6 dims (stride 0 = broadcast); the common
// contiguous / scalar-qparams cases skip the index arithmetic.
#include "lq_common.cuh"

namespace lq {
namespace {

constexpr int kMaxDims = 6;

struct AffArgs {
  int64_t numel;
  int ndim;
  int64_t shape[kMaxDims];
  int64_t xs[kMaxDims], ss[kMaxDims], zs[kMaxDims];
  int xdt, sdt, zdt, odt;
  int d0, d1;  // result dtypes of the two ops (QUANT: div, add; DEQUANT: sub, mul)
  float qmin, qmax;
  int x_contig, s_scalar, z_scalar;
};

__device__ __forceinline__ float load_any(const void* p, int dt, int64_t i) {
  switch (dt) {
    case LQ_F32: return static_cast<const float*>(p)[i];
    case LQ_F16: return __half2float(static_cast<const __half*>(p)[i]);
    case LQ_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
    case LQ_I8: return (float)static_cast<const int8_t*>(p)[i];
    case LQ_I16: return (float)static_cast<const int16_t*>(p)[i];
    case LQ_I32: return (float)static_cast<const int32_t*>(p)[i];
    case LQ_I64: return (float)static_cast<const int64_t*>(p)[i];
    case LQ_U8: return (float)static_cast<const uint8_t*>(p)[i];
  }
  return 0.0f;
}

__device__ __forceinline__ void store_any(void* p, int dt, int64_t i, float v) {
  switch (dt) {
    case LQ_F32: static_cast<float*>(p)[i] = v; break;
    case LQ_F16: static_cast<__half*>(p)[i] = __float2half_rn(v); break;
    case LQ_BF16: static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v); break;
    case LQ_I8: static_cast<int8_t*>(p)[i] = (int8_t)tcast_i32(v); break;
    case LQ_I16: static_cast<int16_t*>(p)[i] = (int16_t)tcast_i32(v); break;
  }
}

template <int OP>
__global__ void __launch_bounds__(256) affine_kernel(const void* __restrict__ x,
                                                     const void* __restrict__ s,
                                                     const void* __restrict__ z, AffArgs a,
                                                     void* __restrict__ out) {
  const float s0 = a.s_scalar ? load_any(s, a.sdt, 0) : 0.0f;
  const float z0 = a.z_scalar ? load_any(z, a.zdt, 0) : 0.0f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < a.numel;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t xo = i, so = 0, zo = 0;
    if (!(a.x_contig && a.s_scalar && a.z_scalar)) {
      xo = 0;
      int64_t rem = i;
      for (int d = a.ndim - 1; d >= 0; --d) {
        const int64_t idx = rem % a.shape[d];
        rem /= a.shape[d];
        xo += idx * a.xs[d];
        so += idx * a.ss[d];
        zo += idx * a.zs[d];
      }
    }
    const float xv = load_any(x, a.xdt, xo);
    const float sv = a.s_scalar ? s0 : load_any(s, a.sdt, so);
    const float zv = a.z_scalar ? z0 : load_any(z, a.zdt, zo);
    float o;
    if constexpr (OP == LQ_AFFINE_DEQUANT) {
      o = round_to(a.d1, __fmul_rn(round_to(a.d0, __fsub_rn(xv, zv)), sv));
    } else {
      const float t = round_to(a.d1, __fadd_rn(round_to(a.d0, __fdiv_rn(xv, sv)), zv));
      if constexpr (OP == LQ_AFFINE_QUANT) {
        // the clamp bounds act in the result dtype (4095 -> 4096 in bf16)
        o = tclamp(trint(t), round_to(a.d1, a.qmin), round_to(a.d1, a.qmax));
      } else {
        const float q = tclamp(tste(t), round_to(a.d1, a.qmin), round_to(a.d1, a.qmax));
        o = round_to(a.d1, __fmul_rn(round_to(a.d1, __fsub_rn(q, zv)), sv));
      }
    }
    store_any(out, a.odt, i, o);
  }
}

// ---------------------------------------------------------------------------
// Whole-tensor min/max: per-block partials into the workspace, then one block
// finalises scale / zero point (core/quantizer.py:63-72).
// ---------------------------------------------------------------------------
constexpr int kTensorBlocks = 1024;

// ste_round forward value (core/quantizer.py:32-34), elementwise in T.
template <typename T>
__global__ void __launch_bounds__(256) ste_round_kernel(const T* __restrict__ x, int64_t n,
                                                        T* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = Ty<T>::from_f(tste(Ty<T>::to_f(x[i])));
}

template <typename T>
int ste_t(const void* x, int64_t n, void* out, cudaStream_t st) {
  int64_t want = (n + 255) / 256;
  int grid = (int)(want < (int64_t)num_sms() * 16 ? want : (int64_t)num_sms() * 16);
  ste_round_kernel<T><<<grid, 256, 0, st>>>(static_cast<const T*>(x), n, static_cast<T*>(out));
  return launched("ste_round_kernel");
}

template <typename T>
__global__ void __launch_bounds__(256) tensor_minmax_kernel(const T* __restrict__ x, int64_t n,
                                                            MinMax* __restrict__ part) {
  __shared__ MinMax red[8];
  MinMax r;
  r.init();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    r.add(Ty<T>::to_f(x[i]));
  for (int m = 16; m >= 1; m >>= 1) r.shfl_xor_merge(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = r;
  __syncthreads();
  if (threadIdx.x == 0) {
    MinMax t = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) t.merge(red[w]);
    part[blockIdx.x] = t;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) tensor_qparams_kernel(const MinMax* __restrict__ part,
                                                             int nparts, int sym, float qmin,
                                                             float qmax, float lo,
                                                             T* __restrict__ scale,
                                                             T* __restrict__ zp) {
  __shared__ MinMax red[8];
  MinMax r;
  r.init();
  for (int i = threadIdx.x; i < nparts; i += blockDim.x) r.merge(part[i]);
  for (int m = 16; m >= 1; m >>= 1) r.shfl_xor_merge(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = r;
  __syncthreads();
  if (threadIdx.x == 0) {
    MinMax t = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) t.merge(red[w]);
    if (sym) t.mx = fmaxf(-t.mn, t.mx);  // max |x|
    float s, z;
    qparams_from<T>(t, sym, qmin, qmax, lo, s, z);
    scale[0] = Ty<T>::from_f(s);
    zp[0] = Ty<T>::from_f(z);
  }
}

template <typename T>
int tensor_qparams_t(const void* x, int64_t n, int n_bits, int sym, void* scale, void* zp,
                     void* ws, cudaStream_t st) {
  int64_t want = (n + 256 * 8 - 1) / (256 * 8);
  int nb = (int)(want < kTensorBlocks ? (want > 0 ? want : 1) : kTensorBlocks);
  MinMax* part = static_cast<MinMax*>(ws);
  tensor_minmax_kernel<T><<<nb, 256, 0, st>>>(static_cast<const T*>(x), n, part);
  int rc = launched("tensor_minmax_kernel");
  if (rc) return rc;
  tensor_qparams_kernel<T><<<1, 256, 0, st>>>(part, nb, sym, (float)qmin_of(n_bits, sym),
                                              (float)qmax_of(n_bits, sym), lo_clamp_value<T>(),
                                              static_cast<T*>(scale), static_cast<T*>(zp));
  return launched("tensor_qparams_kernel");
}

// ---------------------------------------------------------------------------
// Per-channel qparams with the channel in the middle: x [outer, C, inner],
// reduce over outer and inner for every c (core/quantizer.py:74-85).
// Partials per (c, chunk of outer) go to the workspace, then one pass per c.
// ---------------------------------------------------------------------------
constexpr int kChanChunks = 64;

template <typename T>
__global__ void __launch_bounds__(256) channel_minmax_kernel(const T* __restrict__ x,
                                                             int64_t outer, int64_t C,
                                                             int64_t inner, int chunks,
                                                             MinMax* __restrict__ part) {
  __shared__ MinMax red[8];
  for (int64_t job = blockIdx.x; job < C * chunks; job += gridDim.x) {
    const int64_t c = job / chunks;
    const int ch = (int)(job % chunks);
    const int64_t o0 = outer * ch / chunks, o1 = outer * (ch + 1) / chunks;
    const int64_t cnt = (o1 - o0) * inner;
    MinMax r;
    r.init();
    for (int64_t k = threadIdx.x; k < cnt; k += blockDim.x) {
      const int64_t o = o0 + k / inner, i = k % inner;
      r.add(Ty<T>::to_f(x[(o * C + c) * inner + i]));
    }
    for (int m = 16; m >= 1; m >>= 1) r.shfl_xor_merge(m);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = r;
    __syncthreads();
    if (threadIdx.x == 0) {
      MinMax t = red[0];
      for (int w = 1; w < (int)(blockDim.x >> 5); ++w) t.merge(red[w]);
      part[job] = t;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) channel_qparams_kernel(const MinMax* __restrict__ part,
                                                              int64_t C, int chunks, int sym,
                                                              float qmin, float qmax, float lo,
                                                              T* __restrict__ scale,
                                                              T* __restrict__ zp) {
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < C;
       c += (int64_t)gridDim.x * blockDim.x) {
    MinMax t = part[c * chunks];
    for (int k = 1; k < chunks; ++k) t.merge(part[c * chunks + k]);
    if (sym) t.mx = fmaxf(-t.mn, t.mx);
    float s, z;
    qparams_from<T>(t, sym, qmin, qmax, lo, s, z);
    scale[c] = Ty<T>::from_f(s);
    zp[c] = Ty<T>::from_f(z);
  }
}

template <typename T>
int channel_qparams_t(const void* x, int64_t outer, int64_t C, int64_t inner, int n_bits,
                      int sym, void* scale, void* zp, void* ws, cudaStream_t st) {
  const int chunks = (int)(outer < kChanChunks ? outer : kChanChunks);
  MinMax* part = static_cast<MinMax*>(ws);
  int64_t jobs = C * chunks;
  int grid = (int)(jobs < (int64_t)num_sms() * 8 ? jobs : (int64_t)num_sms() * 8);
  channel_minmax_kernel<T><<<grid, 256, 0, st>>>(static_cast<const T*>(x), outer, C, inner, chunks, part);
  int rc = launched("channel_minmax_kernel");
  if (rc) return rc;
  int g2 = (int)((C + 255) / 256);
  if (g2 > num_sms() * 8) g2 = num_sms() * 8;
  channel_qparams_kernel<T><<<g2, 256, 0, st>>>(part, C, chunks, sym, (float)qmin_of(n_bits, sym),
                                                (float)qmax_of(n_bits, sym), lo_clamp_value<T>(),
                                                static_cast<T*>(scale), static_cast<T*>(zp));
  return launched("channel_qparams_kernel");
}

}  // namespace
}  // namespace lq

using namespace lq;

extern "C" int lq_affine(int op, int ndim, const int64_t* shape, const void* x, int x_dtype,
                         const int64_t* x_strides, const void* scale, int s_dtype,
                         const int64_t* s_strides, const void* zero_point, int z_dtype,
                         const int64_t* z_strides, const int* op_dtypes, int n_bits,
                         int symmetric, void* out, int out_dtype, void* stream) {
  LQ_REQUIRE(op >= 0 && op <= 2, LQ_EINVAL, "bad op %d", op);
  LQ_REQUIRE(ndim >= 0 && ndim <= kMaxDims, LQ_ERANGE, "ndim %d above %d", ndim, kMaxDims);
  LQ_REQUIRE(dtype_size(x_dtype) > 0, LQ_EDTYPE, "bad x dtype %d", x_dtype);
  LQ_REQUIRE(is_float_dtype(s_dtype) && is_float_dtype(z_dtype), LQ_EDTYPE, "qparams must be float");
  LQ_REQUIRE(is_float_dtype(out_dtype) || out_dtype == LQ_I8 || out_dtype == LQ_I16, LQ_EDTYPE, "bad out dtype");
  LQ_REQUIRE(is_float_dtype(op_dtypes[0]) && is_float_dtype(op_dtypes[1]), LQ_EDTYPE, "bad op dtypes");
  LQ_REQUIRE(n_bits >= 1 && n_bits <= 16, LQ_EINVAL, "n_bits out of range");
  AffArgs a;
  a.ndim = ndim;
  a.numel = 1;
  bool xc = true, sc = true, zc = true;
  int64_t expect = 1;
  for (int d = ndim - 1; d >= 0; --d) {
    LQ_REQUIRE(shape[d] >= 0, LQ_EINVAL, "negative dim");
    a.shape[d] = shape[d];
    a.xs[d] = x_strides[d];
    a.ss[d] = s_strides[d];
    a.zs[d] = z_strides[d];
    if (shape[d] != 1) {
      if (x_strides[d] != expect) xc = false;
      if (s_strides[d] != 0) sc = false;
      if (z_strides[d] != 0) zc = false;
    }
    expect *= shape[d];
    a.numel *= shape[d];
  }
  if (a.numel == 0) return LQ_OK;
  LQ_REQUIRE(x && scale && zero_point && out, LQ_EINVAL, "NULL pointer");
  a.x_contig = xc;
  a.s_scalar = sc;
  a.z_scalar = zc;
  a.xdt = x_dtype;
  a.sdt = s_dtype;
  a.zdt = z_dtype;
  a.odt = out_dtype;
  a.d0 = op_dtypes[0];
  a.d1 = op_dtypes[1];
  a.qmin = (float)qmin_of(n_bits, symmetric);
  a.qmax = (float)qmax_of(n_bits, symmetric);
  cudaStream_t st = as_stream(stream);
  int64_t want = (a.numel + 255) / 256;
  int grid = (int)(want < (int64_t)num_sms() * 16 ? want : (int64_t)num_sms() * 16);
  switch (op) {
    case LQ_AFFINE_QUANT: affine_kernel<LQ_AFFINE_QUANT><<<grid, 256, 0, st>>>(x, scale, zero_point, a, out); break;
    case LQ_AFFINE_DEQUANT: affine_kernel<LQ_AFFINE_DEQUANT><<<grid, 256, 0, st>>>(x, scale, zero_point, a, out); break;
    default: affine_kernel<LQ_AFFINE_FAKE><<<grid, 256, 0, st>>>(x, scale, zero_point, a, out); break;
  }
  return launched("affine_kernel");
}

extern "C" size_t lq_tensor_qparams_workspace_size(int64_t n) {
  (void)n;
  return (size_t)kTensorBlocks * sizeof(MinMax);
}

extern "C" int lq_tensor_qparams(const void* x, int x_dtype, int64_t n, int n_bits, int symmetric,
                                 void* scale, void* zero_point, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  LQ_REQUIRE(n >= 1, LQ_EINVAL, "per-tensor qparams of an empty tensor");
  LQ_REQUIRE(n_bits >= 1 && n_bits <= 16, LQ_EINVAL, "n_bits out of range");
  LQ_REQUIRE(x && scale && zero_point && workspace, LQ_EINVAL, "NULL pointer");
  LQ_REQUIRE(workspace_bytes >= lq_tensor_qparams_workspace_size(n), LQ_EINVAL, "workspace too small");
  LQ_REQUIRE(aligned16(workspace), LQ_EALIGN, "workspace must be 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  switch (x_dtype) {
    case LQ_F32: return tensor_qparams_t<float>(x, n, n_bits, symmetric, scale, zero_point, workspace, st);
    case LQ_F16: return tensor_qparams_t<__half>(x, n, n_bits, symmetric, scale, zero_point, workspace, st);
    case LQ_BF16: return tensor_qparams_t<__nv_bfloat16>(x, n, n_bits, symmetric, scale, zero_point, workspace, st);
    default: set_error("unsupported dtype %d", x_dtype); return LQ_EDTYPE;
  }
}

extern "C" size_t lq_channel_qparams_workspace_size(int64_t outer, int64_t C, int64_t inner) {
  (void)inner;
  int64_t chunks = outer < kChanChunks ? outer : kChanChunks;
  if (chunks < 1) chunks = 1;
  return (size_t)(C * chunks) * sizeof(MinMax);
}

extern "C" int lq_channel_qparams(const void* x, int x_dtype, int64_t outer, int64_t C,
                                  int64_t inner, int n_bits, int symmetric, void* scale,
                                  void* zero_point, void* workspace, size_t workspace_bytes,
                                  void* stream) {
  LQ_REQUIRE(outer >= 1 && C >= 1 && inner >= 1, LQ_EINVAL, "per-channel qparams of an empty tensor");
  LQ_REQUIRE(n_bits >= 1 && n_bits <= 16, LQ_EINVAL, "n_bits out of range");
  LQ_REQUIRE(x && scale && zero_point && workspace, LQ_EINVAL, "NULL pointer");
  LQ_REQUIRE(workspace_bytes >= lq_channel_qparams_workspace_size(outer, C, inner), LQ_EINVAL, "workspace too small");
  cudaStream_t st = as_stream(stream);
  switch (x_dtype) {
    case LQ_F32: return channel_qparams_t<float>(x, outer, C, inner, n_bits, symmetric, scale, zero_point, workspace, st);
    case LQ_F16: return channel_qparams_t<__half>(x, outer, C, inner, n_bits, symmetric, scale, zero_point, workspace, st);
    case LQ_BF16: return channel_qparams_t<__nv_bfloat16>(x, outer, C, inner, n_bits, symmetric, scale, zero_point, workspace, st);
    default: set_error("unsupported dtype %d", x_dtype); return LQ_EDTYPE;
  }
}

extern "C" int lq_ste_round(const void* x, int dtype, int64_t n, void* out, void* stream) {
  LQ_REQUIRE(n >= 0, LQ_EINVAL, "bad size");
  if (n == 0) return LQ_OK;
  LQ_REQUIRE(x && out, LQ_EINVAL, "NULL pointer");
  cudaStream_t st = as_stream(stream);
  switch (dtype) {
    case LQ_F32: return ste_t<float>(x, n, out, st);
    case LQ_F16: return ste_t<__half>(x, n, out, st);
    case LQ_BF16: return ste_t<__nv_bfloat16>(x, n, out, st);
    default: set_error("unsupported dtype %d", dtype); return LQ_EDTYPE;
  }
}

// ---------------------------------------------------------------------------
// Per-tensor qparams without a caller-provided workspace.
//
// For callers that cannot allocate device memory themselves -- a host
// program that reaches this library only through its C ABI (an FFI binding
// that is handed tensor pointers owned by another runtime and has no device
// allocator of its own), or an application whose device memory is entirely
// reserved by a framework allocator it cannot call into -- this variant keeps
// its per-block partial results in a fixed array in this library's own
// device memory instead of a workspace argument.
//
// Limits and behaviour:
//   * the array holds kNoAllocParts partials of one 4096-element block each,
//     so n is limited to kNoAllocParts * 4096 = 64 Mi elements (every GPU
//     that loads the library holds the 128 KB array until the process exits);
//   * every call on a device shares the array: calls whose kernels overlap on
//     the GPU (different streams without ordering) race and give wrong
//     results; calls ordered on one stream are safe.  Each call writes every
//     partial it later reads, so nothing has to be cleared between calls;
//   * the first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (once per device, with that device current), so
//     make that first call before any stream capture.  The address is cached
//     for the life of the process; a cudaDeviceReset of the device may move
//     the array, so the entry point must not be called after one;
//   * the call allocates nothing: no cudaMalloc, no cudaFree, no library
//     routine that allocates.
// ---------------------------------------------------------------------------
namespace lq {
namespace {

constexpr int64_t kNoAllocParts = 16384;
constexpr int64_t kNoAllocBlockElems = 256 * 16;

static __device__ __align__(256) MinMax g_noalloc_partials[kNoAllocParts];

MinMax* noalloc_partials_for_current_device() {
  static std::atomic<MinMax*> slots[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  MinMax* p = slots[dev].load(std::memory_order_acquire);
  if (p) return p;
  void* addr = nullptr;
  // the host-side name of the array is only a stand-in: ask the runtime for
  // its address on this device
  if (cudaGetSymbolAddress(&addr, g_noalloc_partials) != cudaSuccess || addr == nullptr) return nullptr;
  p = static_cast<MinMax*>(addr);
  slots[dev].store(p, std::memory_order_release);
  return p;
}

template <typename T>
int tensor_qparams_noalloc_t(const void* x, int64_t n, int n_bits, int sym, void* scale, void* zp,
                             MinMax* part, cudaStream_t st) {
  const int nb = (int)((n + kNoAllocBlockElems - 1) / kNoAllocBlockElems);
  tensor_minmax_kernel<T><<<nb, 256, 0, st>>>(static_cast<const T*>(x), n, part);
  int rc = launched("tensor_minmax_kernel");
  if (rc) return rc;
  tensor_qparams_kernel<T><<<1, 256, 0, st>>>(part, nb, sym, (float)qmin_of(n_bits, sym),
                                              (float)qmax_of(n_bits, sym), lo_clamp_value<T>(),
                                              static_cast<T*>(scale), static_cast<T*>(zp));
  return launched("tensor_qparams_kernel");
}

}  // namespace
}  // namespace lq

extern "C" int lq_tensor_qparams_noalloc(const void* x, int x_dtype, int64_t n, int n_bits,
                                         int symmetric, void* scale, void* zero_point,
                                         void* stream) {
  using namespace lq;
  LQ_REQUIRE(n >= 1, LQ_EINVAL, "per-tensor qparams of an empty tensor");
  LQ_REQUIRE(n <= kNoAllocParts * kNoAllocBlockElems, LQ_ERANGE,
             "lq_tensor_qparams_noalloc: n = %lld is above its maximum of %lld elements "
             "(use lq_tensor_qparams with a workspace)",
             (long long)n, (long long)(kNoAllocParts * kNoAllocBlockElems));
  LQ_REQUIRE(n_bits >= 1 && n_bits <= 16, LQ_EINVAL, "n_bits out of range");
  LQ_REQUIRE(x && scale && zero_point, LQ_EINVAL, "NULL pointer");
  MinMax* part = noalloc_partials_for_current_device();
  LQ_REQUIRE(part != nullptr, LQ_ECUDA, "cudaGetSymbolAddress of the scratch array failed");
  cudaStream_t st = as_stream(stream);
  switch (x_dtype) {
    case LQ_F32: return tensor_qparams_noalloc_t<float>(x, n, n_bits, symmetric, scale, zero_point, part, st);
    case LQ_F16: return tensor_qparams_noalloc_t<__half>(x, n, n_bits, symmetric, scale, zero_point, part, st);
    case LQ_BF16: return tensor_qparams_noalloc_t<__nv_bfloat16>(x, n, n_bits, symmetric, scale, zero_point, part, st);
    default: set_error("unsupported dtype %d", x_dtype); return LQ_EDTYPE;
  }
}
