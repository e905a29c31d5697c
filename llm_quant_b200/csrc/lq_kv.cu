// lq_kv.cu -- KV-cache quantization along the token axis and KV dequantization.
//
// Token-group quantization: x is [P, T, D] (P = batch*heads).  For every
// (p, d) the tokens are cut into groups of `tgroup` tokens (zero-padded at the
// end, kv_cache_quant.py:141-166), or taken whole for PER_CHANNEL
// (kv_cache_quant.py:119-122).  One block owns one (p, token-group,
// column-tile) slab: threads are laid out [TY token rows x TX columns], each
// column thread moving 16-byte vectors.  Pass 1 reduces min/max per column,
// pass 2 re-reads the slab (an L2 hit for slabs of a few hundred KB) and
// writes codes or fp32 fake-quant values.
#include "lq_common.cuh"

namespace lq {
namespace {

template <typename OutT> struct CodeCast;
template <> struct CodeCast<int8_t> {
  __device__ __forceinline__ static int8_t cv(float v) { return (int8_t)tcast_i32(v); }
};
template <> struct CodeCast<int16_t> {
  __device__ __forceinline__ static int16_t cv(float v) { return (int16_t)tcast_i32(v); }
};
template <> struct CodeCast<float> {  // FAKE output (already a value)
  __device__ __forceinline__ static float cv(float v) { return v; }
};
template <> struct CodeCast<__half> {
  __device__ __forceinline__ static __half cv(float v) { return __float2half_rn(v); }
};
template <> struct CodeCast<__nv_bfloat16> {
  __device__ __forceinline__ static __nv_bfloat16 cv(float v) { return __float2bfloat16_rn(v); }
};

struct TokArgs {
  int64_t P, T, D, S;  // S = tokens per group (== T for per-channel)
  int64_t ngt;         // token groups
  int64_t ntile;       // column tiles of CW elements
  int CW;              // column tile width in elements
  int pad;             // 1: the last group is zero-padded to S tokens
  float qmin, qmax, lo;
  int sym;
  // output placement (KV append into capacity storage): codes of token t of
  // slab p go to row p * out_pitch_t + out_t_off + t; the scales of token
  // group g to row p * s_pitch_g + s_off_g + g.  merge = 1 folds the new
  // scale / zero point into the stored ones with torch.maximum
  // (QuantizedKVCache._cat_scales PER_CHANNEL, kv_cache_quant.py:395-402).
  int64_t out_pitch_t, out_t_off, s_pitch_g, s_off_g;
  int merge;
};

// torch.maximum: NaN if either operand is NaN.
__device__ __forceinline__ float tmaximum(float a, float b) {
  if (a != a || b != b) return __int_as_float(0x7fc00000);
  return (a < b) ? b : a;
}

// MODE 0 = QPARAMS, 1 = FAKE (fp32 out), 2 = CODES
template <typename T, int MODE, typename OutT, bool VEC>
__global__ void __launch_bounds__(256) token_group_kernel(const T* __restrict__ x, TokArgs a,
                                                          OutT* __restrict__ out,
                                                          T* __restrict__ scale_out,
                                                          T* __restrict__ zp_out) {
  constexpr int V = VEC ? 16 / sizeof(T) : 1;
  extern __shared__ unsigned char smraw[];
  MinMax* sm = reinterpret_cast<MinMax*>(smraw);  // [TY][CW]
  const int TX = a.CW / V;
  const int TY = blockDim.x / TX;
  const int tx = threadIdx.x % TX, ty = threadIdx.x / TX;
  const int64_t nslab = a.P * a.ngt * a.ntile;
  for (int64_t slab = blockIdx.x; slab < nslab; slab += gridDim.x) {
    const int64_t tile = slab % a.ntile;
    const int64_t gt = (slab / a.ntile) % a.ngt;
    const int64_t p = slab / (a.ntile * a.ngt);
    const int64_t t0 = gt * a.S;
    const int64_t t1 = min(t0 + a.S, a.T);
    const int64_t c0 = tile * a.CW + (int64_t)tx * V;
    const bool col_ok = (ty < TY) && (c0 < a.D);
    const T* xb = x + p * a.T * a.D;
    MinMax r[V];
#pragma unroll
    for (int i = 0; i < V; ++i) r[i].init();
    if (col_ok) {
#pragma unroll 8
      for (int64_t t = t0 + ty; t < t1; t += TY) {  // unrolled: 8 token rows' loads in flight
        const T* src = xb + t * a.D + c0;
        if constexpr (VEC) {
          Vec16<T> u;
          u.u = ld_nc_v4(src);
#pragma unroll
          for (int i = 0; i < V; ++i) {
            float v = Ty<T>::to_f(u.v[i]);
            if (a.sym) r[i].add_max(fabsf(v));
            else r[i].add(v);
          }
        } else {
          float v = Ty<T>::to_f(*src);
          if (a.sym) r[0].add_max(fabsf(v));
          else r[0].add(v);
        }
      }
      // zero padding of the last token group takes part in min/max
      if (a.pad && t1 - t0 < a.S && ty == 0) {
#pragma unroll
        for (int i = 0; i < V; ++i) r[i].add(0.0f);
      }
    }
    __syncthreads();
    if (ty < TY) {
#pragma unroll
      for (int i = 0; i < V; ++i) sm[ty * a.CW + tx * V + i] = r[i];
    }
    __syncthreads();
    // column finalisation: thread c (< CW) reduces the TY partials of column c
    for (int c = threadIdx.x; c < a.CW; c += blockDim.x) {
      MinMax m = sm[c];
      for (int y = 1; y < TY; ++y) m.merge(sm[y * a.CW + c]);
      float s, z;
      qparams_from<T>(m, a.sym, a.qmin, a.qmax, a.lo, s, z);
      sm[c].mn = s;  // reuse row 0 as (scale, zp) storage
      sm[c].mx = z;
      const int64_t col = tile * a.CW + c;
      if (col < a.D && scale_out) {
        const int64_t o = (p * a.s_pitch_g + a.s_off_g + gt) * a.D + col;
        if (a.merge) {
          scale_out[o] = Ty<T>::from_f(tmaximum(Ty<T>::to_f(scale_out[o]), s));
          zp_out[o] = Ty<T>::from_f(tmaximum(Ty<T>::to_f(zp_out[o]), z));
        } else {
          scale_out[o] = Ty<T>::from_f(s);
          zp_out[o] = Ty<T>::from_f(z);
        }
      }
    }
    __syncthreads();
    if constexpr (MODE != 0) {
      if (col_ok) {
        float sc[V], zz[V];
#pragma unroll
        for (int i = 0; i < V; ++i) {
          sc[i] = sm[tx * V + i].mn;
          zz[i] = sm[tx * V + i].mx;
        }
        OutT* ob = out + (p * a.out_pitch_t + a.out_t_off) * a.D;
#pragma unroll 4
        for (int64_t t = t0 + ty; t < t1; t += TY) {
          const T* src = xb + t * a.D + c0;
          float v[V];
          if constexpr (VEC) {
            Vec16<T> u;
            u.u = ld_nc_v4(src);
#pragma unroll
            for (int i = 0; i < V; ++i) v[i] = Ty<T>::to_f(u.v[i]);
          } else {
            v[0] = Ty<T>::to_f(*src);
          }
          constexpr int BYTES = V * sizeof(OutT);
          union {
            OutT o[V];
            uint4 q4[(BYTES + 15) / 16];
            uint2 q2;
            uint32_t q1;
          } ov;
#pragma unroll
          for (int i = 0; i < V; ++i) {
            float q = tclamp_t<T>(trint(tadd<T>(tdiv<T>(v[i], sc[i]), zz[i])), a.qmin, a.qmax);
            if constexpr (MODE == 1) {
              // KVCacheQuantizer.fake_quantize: codes are cast to intN first
              // (NaN -> 0), then (q.float() - zp) * scale in fp32.
              float qi = (float)(a.sym ? (int8_t)tcast_i32(q) : (int16_t)tcast_i32(q));
              ov.o[i] = CodeCast<OutT>::cv(__fmul_rn(__fsub_rn(qi, zz[i]), sc[i]));
            } else {
              ov.o[i] = CodeCast<OutT>::cv(q);
            }
          }
          OutT* dst = ob + t * a.D + c0;
          if constexpr (VEC) {
            if constexpr (BYTES >= 16) {
#pragma unroll
              for (int k = 0; k < BYTES / 16; ++k) st_v4(reinterpret_cast<uint4*>(dst) + k, ov.q4[k]);
            } else if constexpr (BYTES == 8) {
              *reinterpret_cast<uint2*>(dst) = ov.q2;
            } else {
              *reinterpret_cast<uint32_t*>(dst) = ov.q1;
            }
          } else {
            *dst = ov.o[0];
          }
        }
      }
    }
    __syncthreads();
  }
}

template <typename T, int MODE, typename OutT>
int launch_tok(const T* x, TokArgs a, OutT* out, T* s, T* z, bool vec, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  const int threads = 256;
  a.CW = (int)(a.D < 256 ? a.D : 256);
  if (vec) {
    // column tile: a multiple of V, at most 256 elements (32 vector threads
    // for fp32), narrowed (down to 4 vector threads) until there are slabs
    // for two per SM -- a per-channel chunk of few (batch, head) pairs would
    // otherwise leave most SMs idle
    while (a.P * a.ngt * ((a.D + a.CW - 1) / a.CW) < 2 * (int64_t)num_sms() && a.CW / V > 4 &&
           (a.CW / 2) % V == 0)
      a.CW /= 2;
  }
  a.ntile = (a.D + a.CW - 1) / a.CW;
  const int TX = vec ? a.CW / V : a.CW;
  const int TY = threads / TX;
  size_t smem = (size_t)TY * a.CW * sizeof(MinMax);
  int64_t nslab = a.P * a.ngt * a.ntile;
  int grid = (int)(nslab < (int64_t)num_sms() * 8 ? nslab : (int64_t)num_sms() * 8);
  if (grid < 1) grid = 1;
  if (vec) {
    token_group_kernel<T, MODE, OutT, true><<<grid, threads, smem, st>>>(x, a, out, s, z);
  } else {
    token_group_kernel<T, MODE, OutT, false><<<grid, threads, smem, st>>>(x, a, out, s, z);
  }
  return launched("token_group_kernel");
}

template <typename T>
int token_group_t(const void* xv, int64_t P, int64_t T_, int64_t D, int64_t tgroup, int n_bits,
                  int sym, int mode, void* out, int out_dtype, void* scale, void* zp,
                  cudaStream_t st, int64_t out_pitch_t = -1, int64_t out_t_off = 0,
                  int64_t s_pitch_g = -1, int64_t s_off_g = 0, int merge = 0) {
  const T* x = static_cast<const T*>(xv);
  TokArgs a;
  a.out_pitch_t = out_pitch_t >= 0 ? out_pitch_t : T_;
  a.out_t_off = out_t_off;
  a.merge = merge;
  a.P = P;
  a.T = T_;
  a.D = D;
  a.pad = tgroup > 0;
  a.S = tgroup > 0 ? tgroup : T_;
  a.ngt = (T_ + a.S - 1) / a.S;
  a.s_pitch_g = s_pitch_g >= 0 ? s_pitch_g : a.ngt;
  a.s_off_g = s_off_g;
  a.qmin = (float)qmin_of(n_bits, sym);
  a.qmax = (float)qmax_of(n_bits, sym);
  a.lo = lo_clamp_value<T>();
  a.sym = sym;
  constexpr int V = 16 / sizeof(T);
  const int osz = mode == LQ_MODE_QPARAMS ? 1 : (mode == LQ_MODE_FAKE ? 4 : dtype_size(out_dtype));
  bool vec = (D % V == 0) && (D <= 256 ? true : (256 % V == 0)) && aligned16(x) &&
             (mode == LQ_MODE_QPARAMS || (reinterpret_cast<uintptr_t>(out) % (V * osz) == 0));
  T* s = static_cast<T*>(scale);
  T* z = static_cast<T*>(zp);
  if (mode == LQ_MODE_QPARAMS) return launch_tok<T, 0, float>(x, a, nullptr, s, z, vec, st);
  if (mode == LQ_MODE_FAKE) {
    LQ_REQUIRE(out_dtype == LQ_F32, LQ_EDTYPE, "token-group fake-quant writes fp32");
    LQ_REQUIRE(n_bits <= 8 || !sym, LQ_EINVAL, "symmetric codes are int8: n_bits <= 8");
    return launch_tok<T, 1, float>(x, a, static_cast<float*>(out), s, z, vec, st);
  }
  if (out_dtype == LQ_I8) return launch_tok<T, 2, int8_t>(x, a, static_cast<int8_t*>(out), s, z, vec, st);
  if (out_dtype == LQ_I16) return launch_tok<T, 2, int16_t>(x, a, static_cast<int16_t*>(out), s, z, vec, st);
  if (out_dtype == Ty<T>::code) return launch_tok<T, 2, T>(x, a, static_cast<T*>(out), s, z, vec, st);
  set_error("unsupported code dtype %d", out_dtype);
  return LQ_EDTYPE;
}

// ---------------------------------------------------------------------------
// KV dequantization: out = (float(q) - zp) * scale in fp32.
// Thread = 4 consecutive elements of one token row (16 bytes of fp32 out).
// ---------------------------------------------------------------------------
struct DqArgs {
  int64_t P, T, D, cpitch, S, szpitch;
  int gran;
};

template <typename CT, typename ST>
__global__ void __launch_bounds__(256) kv_dequant_kernel(const CT* __restrict__ codes, DqArgs a,
                                                         const ST* __restrict__ scale,
                                                         const ST* __restrict__ zp,
                                                         float* __restrict__ out, int vec4) {
  const int64_t per_row = vec4 ? a.D / 4 : a.D;
  const int64_t total = a.P * a.T * per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / per_row;  // (p, t)
    const int64_t c = (i % per_row) * (vec4 ? 4 : 1);
    const int64_t p = r / a.T, t = r % a.T;
    const CT* q = codes + (p * a.cpitch + t) * a.D + c;
    const int n = vec4 ? 4 : 1;
    float o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (k >= n) break;
      int64_t si;
      if (a.gran == 0) si = p * a.szpitch + t;
      else if (a.gran == 1) si = p * a.D + c + k;
      else si = (p * a.szpitch + t / a.S) * a.D + c + k;
      const float s = Ty<ST>::to_f(scale[si]);
      const float z = Ty<ST>::to_f(zp[si]);
      o[k] = __fmul_rn(__fsub_rn((float)q[k], z), s);
    }
    float* dst = out + r * a.D + c;
    if (vec4) st_v4(dst, make_uint4(__float_as_uint(o[0]), __float_as_uint(o[1]), __float_as_uint(o[2]), __float_as_uint(o[3])));
    else dst[0] = o[0];
  }
}

// Segment path (D % 4 == 0): a warp takes 512 consecutive elements of one
// (p) slice -- T*D elements, contiguous in the output and in the code buffer
// -- and lane l the 4-element chunks 4l + 128k, k = 0..3, so every load and
// store instruction of the warp covers one contiguous span (128 or 256 bytes
// of codes, 512 bytes of fp32).  float(q) is formed exactly as
// (1.5 * 2^23 + q) - 1.5 * 2^23.
template <typename CT> struct Codes4;
template <> struct Codes4<int8_t> {
  using W = uint32_t;
  __device__ __forceinline__ static int get(W w, int i) { return (int)(int8_t)(w >> (8 * i)); }
};
template <> struct Codes4<int16_t> {
  using W = uint2;
  __device__ __forceinline__ static int get(W w, int i) {
    return (int)(int16_t)((i < 2 ? w.x : w.y) >> (16 * (i & 1)));
  }
};

template <typename CT, typename ST>
__global__ void __launch_bounds__(256) kv_dequant_seg_kernel(const CT* __restrict__ codes, DqArgs a,
                                                             const ST* __restrict__ scale,
                                                             const ST* __restrict__ zp,
                                                             float* __restrict__ out,
                                                             int64_t segs_per_p, int d_shift) {
  using W = typename Codes4<CT>::W;
  const int lane = threadIdx.x & 31;
  const int64_t slice = a.T * a.D;
  const int64_t nseg = a.P * segs_per_p;
  const int64_t warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t g = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; g < nseg; g += warps) {
    const int64_t p = g / segs_per_p;
    const int64_t e0 = (g - p * segs_per_p) * 512 + 4 * lane;
    const CT* qp = codes + p * a.cpitch * a.D;
    float* op = out + p * slice;
    W w[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int64_t e = e0 + 128 * k;
      if (e < slice) w[k] = *reinterpret_cast<const W*>(qp + e);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int64_t e = e0 + 128 * k;
      if (e >= slice) break;
      const int64_t t = d_shift >= 0 ? (e >> d_shift) : e / a.D;
      const int64_t c = e - t * a.D;
      float sv[4], zv[4];
      if (a.gran == 0) {
        const int64_t si = p * a.szpitch + t;
        const float s0 = Ty<ST>::to_f(scale[si]), z0 = Ty<ST>::to_f(zp[si]);
#pragma unroll
        for (int i = 0; i < 4; ++i) { sv[i] = s0; zv[i] = z0; }
      } else {
        const int64_t base = (a.gran == 1) ? p * a.D + c : (p * a.szpitch + t / a.S) * a.D + c;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          sv[i] = Ty<ST>::to_f(scale[base + i]);
          zv[i] = Ty<ST>::to_f(zp[base + i]);
        }
      }
      float o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float qf = __fsub_rn(__int_as_float(0x4B400000 + Codes4<CT>::get(w[k], i)), 12582912.0f);
        o[i] = __fmul_rn(__fsub_rn(qf, zv[i]), sv[i]);
      }
      st_v4(op + e, make_uint4(__float_as_uint(o[0]), __float_as_uint(o[1]), __float_as_uint(o[2]),
                               __float_as_uint(o[3])));
    }
  }
}

template <typename CT, typename ST>
int kv_dequant_t(const void* codes, const DqArgs& a, const void* s, const void* z, float* out,
                 cudaStream_t st) {
  if (a.D % 4 == 0 && aligned16(out) && reinterpret_cast<uintptr_t>(codes) % (4 * sizeof(CT)) == 0) {
    const int64_t segs_per_p = (a.T * a.D + 511) / 512;
    const int64_t warps_needed = a.P * segs_per_p;
    const int grid = resident_grid(kv_dequant_seg_kernel<CT, ST>, 256, 0, (warps_needed + 7) / 8);
    int d_shift = -1;
    if ((a.D & (a.D - 1)) == 0) {
      d_shift = 0;
      while ((int64_t(1) << d_shift) < a.D) ++d_shift;
    }
    kv_dequant_seg_kernel<CT, ST><<<grid, 256, 0, st>>>(static_cast<const CT*>(codes), a,
                                                        static_cast<const ST*>(s),
                                                        static_cast<const ST*>(z), out, segs_per_p,
                                                        d_shift);
    return launched("kv_dequant_seg_kernel");
  }
  int vec4 = (a.D % 4 == 0) && aligned16(out) &&
             (reinterpret_cast<uintptr_t>(codes) % (4 * sizeof(CT)) == 0);
  const int64_t per_row = vec4 ? a.D / 4 : a.D;
  const int64_t total = a.P * a.T * per_row;
  int64_t want = (total + 255) / 256;
  int grid = (int)(want < (int64_t)num_sms() * 16 ? (want > 0 ? want : 1) : (int64_t)num_sms() * 16);
  kv_dequant_kernel<CT, ST><<<grid, 256, 0, st>>>(static_cast<const CT*>(codes), a,
                                                  static_cast<const ST*>(s),
                                                  static_cast<const ST*>(z), out, vec4);
  return launched("kv_dequant_kernel");
}

template <typename CT>
int kv_dequant_c(const void* codes, const DqArgs& a, const void* s, const void* z, int sdt,
                 float* out, cudaStream_t st) {
  switch (sdt) {
    case LQ_F32: return kv_dequant_t<CT, float>(codes, a, s, z, out, st);
    case LQ_F16: return kv_dequant_t<CT, __half>(codes, a, s, z, out, st);
    case LQ_BF16: return kv_dequant_t<CT, __nv_bfloat16>(codes, a, s, z, out, st);
    default: set_error("unsupported scale dtype %d", sdt); return LQ_EDTYPE;
  }
}

}  // namespace
}  // namespace lq

extern "C" int lq_token_group_quant(const void* x, int x_dtype, int64_t P, int64_t T, int64_t D,
                                    int64_t tgroup, int n_bits, int symmetric, int mode,
                                    void* out, int out_dtype, void* scale, void* zero_point,
                                    void* stream) {
  using namespace lq;
  LQ_REQUIRE(P >= 0 && T >= 0 && D >= 0 && tgroup >= 0, LQ_EINVAL, "bad shape");
  LQ_REQUIRE(n_bits >= 1 && n_bits <= 16, LQ_EINVAL, "n_bits %d out of range", n_bits);
  LQ_REQUIRE(mode >= 0 && mode <= 2, LQ_EINVAL, "bad mode %d", mode);
  if (P * T * D == 0) return LQ_OK;
  LQ_REQUIRE(x, LQ_EINVAL, "x is NULL");
  LQ_REQUIRE(mode == LQ_MODE_QPARAMS || out, LQ_EINVAL, "out is NULL");
  LQ_REQUIRE((scale == nullptr) == (zero_point == nullptr), LQ_EINVAL, "scale and zero_point must both be given");
  LQ_REQUIRE(mode != LQ_MODE_QPARAMS || scale, LQ_EINVAL, "QPARAMS mode needs scale/zero_point");
  cudaStream_t st = as_stream(stream);
  switch (x_dtype) {
    case LQ_F32: return token_group_t<float>(x, P, T, D, tgroup, n_bits, symmetric, mode, out, out_dtype, scale, zero_point, st);
    case LQ_F16: return token_group_t<__half>(x, P, T, D, tgroup, n_bits, symmetric, mode, out, out_dtype, scale, zero_point, st);
    case LQ_BF16: return token_group_t<__nv_bfloat16>(x, P, T, D, tgroup, n_bits, symmetric, mode, out, out_dtype, scale, zero_point, st);
    default: set_error("unsupported x dtype %d", x_dtype); return LQ_EDTYPE;
  }
}

extern "C" int lq_kv_dequant(const void* codes, int code_dtype, int64_t P, int64_t T, int64_t D,
                             int64_t codes_pitch_t, int granularity, int64_t tgroup,
                             const void* scale, const void* zero_point, int s_dtype,
                             int64_t sz_pitch, float* out, void* stream) {
  using namespace lq;
  LQ_REQUIRE(P >= 0 && T >= 0 && D >= 0, LQ_EINVAL, "bad shape");
  LQ_REQUIRE(codes_pitch_t >= T, LQ_EINVAL, "codes pitch %lld < T %lld", (long long)codes_pitch_t, (long long)T);
  LQ_REQUIRE(granularity >= 0 && granularity <= 2, LQ_EINVAL, "bad granularity %d", granularity);
  LQ_REQUIRE(granularity != 2 || tgroup > 0, LQ_EINVAL, "per-group needs tgroup > 0");
  if (P * T * D == 0) return LQ_OK;
  LQ_REQUIRE(codes && scale && zero_point && out, LQ_EINVAL, "NULL pointer");
  DqArgs a;
  a.P = P; a.T = T; a.D = D; a.cpitch = codes_pitch_t; a.gran = granularity;
  a.S = tgroup > 0 ? tgroup : 1;
  a.szpitch = sz_pitch;
  if (granularity == 0) LQ_REQUIRE(sz_pitch >= T, LQ_EINVAL, "per-token scale pitch < T");
  if (granularity == 2) LQ_REQUIRE(sz_pitch >= (T + tgroup - 1) / tgroup, LQ_EINVAL, "per-group scale pitch too small");
  cudaStream_t st = as_stream(stream);
  if (code_dtype == LQ_I8) return kv_dequant_c<int8_t>(codes, a, scale, zero_point, s_dtype, out, st);
  if (code_dtype == LQ_I16) return kv_dequant_c<int16_t>(codes, a, scale, zero_point, s_dtype, out, st);
  set_error("unsupported code dtype %d", code_dtype);
  return LQ_EDTYPE;
}

// QuantizedKVCache.update, append half (kv_cache_quant.py:354-377): quantize
// the new chunk x [P, Tn, D] and write its codes straight into the cache's
// capacity storage at token offset t_offset (codes [P, codes_pitch_t, D]);
// scales / zero points go to:
//   per-token   [P, sz_pitch] at token offset sz_offset (= t_offset),
//   per-channel [P, D], written (merge = 0) or max-merged (merge = 1),
//   per-group   [P, sz_pitch, D] at group offset sz_offset.
extern "C" int lq_kv_append(const void* x, int x_dtype, int64_t P, int64_t Tn, int64_t D,
                            int granularity, int64_t tgroup, int n_bits, int symmetric,
                            void* codes, int code_dtype, int64_t codes_pitch_t, int64_t t_offset,
                            void* scale, void* zero_point, int64_t sz_pitch, int64_t sz_offset,
                            int merge, void* stream) {
  using namespace lq;
  LQ_REQUIRE(P >= 0 && Tn >= 0 && D >= 0 && t_offset >= 0 && sz_offset >= 0, LQ_EINVAL, "bad shape");
  LQ_REQUIRE(granularity >= 0 && granularity <= 2, LQ_EINVAL, "bad granularity %d", granularity);
  LQ_REQUIRE(n_bits >= 1 && n_bits <= 16, LQ_EINVAL, "n_bits out of range");
  LQ_REQUIRE(code_dtype == LQ_I8 || code_dtype == LQ_I16, LQ_EDTYPE, "codes must be int8/int16");
  LQ_REQUIRE(codes_pitch_t >= t_offset + Tn, LQ_ERANGE, "cache capacity %lld < %lld tokens",
             (long long)codes_pitch_t, (long long)(t_offset + Tn));
  if (P * Tn * D == 0) return LQ_OK;
  LQ_REQUIRE(x && codes && scale && zero_point, LQ_EINVAL, "NULL pointer");
  if (granularity == 0) {
    LQ_REQUIRE(sz_pitch >= sz_offset + Tn, LQ_ERANGE, "scale capacity too small");
    return group_quant_remap(x, x_dtype, P * Tn, D, D, n_bits, symmetric, LQ_MODE_CODES, codes,
                             code_dtype, scale, zero_point, stream, Tn, codes_pitch_t, t_offset,
                             sz_pitch, sz_offset);
  }
  const int64_t tg = granularity == 1 ? 0 : tgroup;
  LQ_REQUIRE(granularity == 1 || tgroup > 0, LQ_EINVAL, "per-group needs tgroup > 0");
  if (granularity == 2)
    LQ_REQUIRE(sz_pitch >= sz_offset + (Tn + tgroup - 1) / tgroup, LQ_ERANGE, "scale capacity too small");
  const int64_t spitch = granularity == 1 ? 1 : sz_pitch;
  const int64_t soff = granularity == 1 ? 0 : sz_offset;
  cudaStream_t st = as_stream(stream);
  switch (x_dtype) {
    case LQ_F32: return token_group_t<float>(x, P, Tn, D, tg, n_bits, symmetric, LQ_MODE_CODES, codes, code_dtype, scale, zero_point, st, codes_pitch_t, t_offset, spitch, soff, merge);
    case LQ_F16: return token_group_t<__half>(x, P, Tn, D, tg, n_bits, symmetric, LQ_MODE_CODES, codes, code_dtype, scale, zero_point, st, codes_pitch_t, t_offset, spitch, soff, merge);
    case LQ_BF16: return token_group_t<__nv_bfloat16>(x, P, Tn, D, tg, n_bits, symmetric, LQ_MODE_CODES, codes, code_dtype, scale, zero_point, st, codes_pitch_t, t_offset, spitch, soff, merge);
    default: set_error("unsupported x dtype %d", x_dtype); return LQ_EDTYPE;
  }
}
