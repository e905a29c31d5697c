// lq_nf4.cu -- NF4 blockwise quantization (qlora.py).
//
// Encoding.  The reference picks code = first argmin_i |x_norm - NF4_TABLE[i]|
// with the differences computed in fp32 (qlora.py:103-104), where
// x_norm = round_T(x / scale).  For x_norm in [-1, 1] the fp32 differences on
// either side of x_norm are monotone, so the code is a non-decreasing step
// function of x_norm, and since round_T is monotone too, of the unrounded
// quotient p = x / scale: code = #{i : p >= kTheta[T][i]}, where kTheta[T][i]
// is the smallest fp32 value whose reference code is > i (found by exhaustive
// bisection over fp32 bit patterns; the CPU tests re-derive the fp32 set).
// The thresholds are >= 0.08 apart, so a 65-bucket table over [-1, 1]
// (bucket width 1/32, at most one threshold per bucket) turns the count into
// one FFMA (bucket index), one shared-memory load and one compare.  A NaN
// quotient gets code 0, as torch.argmin gives for an all-NaN row.
//
// Layout.  The tensor is flattened and cut into groups of G elements, the
// last one zero-padded (qlora.py:84-93).  A team of G/(V*NVT) lanes owns one
// group (V elements = 16 bytes per vector, NVT vectors per lane) and keeps
// four groups in flight; a block walks "super-groups" of DG consecutive
// groups so the double quantization of their DG scales (qlora.py:164-196) is
// done in shared memory in the same pass.
#include <type_traits>

#include "lq_common.cuh"
#include "lq_tma.cuh"

namespace lq {
namespace {


// Decision thresholds on the unrounded quotient, per input dtype
// (row 0: fp32, 1: fp16, 2: bf16).
__device__ __constant__ float kTheta[3][15] = {
    {-0x1.b23a28p-1f, -0x1.38a71cp-1f, -0x1.d70a3cp-2f, -0x1.5bcd34p-2f, -0x1.e075f4p-3f,
     -0x1.1a8586p-3f, -0x1.752544p-5f, 0x1.460aa8p-5f, 0x1.ec8b44p-4f, 0x1.a0c49cp-3f,
     0x1.2b020ep-2f, 0x1.8ea4aap-2f, 0x1.00d846p-1f, 0x1.491d16p-1f, 0x1.b91688p-1f},
    {-0x1.b22p-1f, -0x1.38ap-1f, -0x1.d72p-2f, -0x1.5bdffep-2f, -0x1.e05ffep-3f,
     -0x1.1aap-3f, -0x1.752p-5f, 0x1.462002p-5f, 0x1.eca002p-4f, 0x1.a0ep-3f,
     0x1.2b2002p-2f, 0x1.8ea002p-2f, 0x1.00ep-1f, 0x1.492002p-1f, 0x1.b92002p-1f},
    {-0x1.b2fffep-1f, -0x1.39p-1f, -0x1.d6fffep-2f, -0x1.5afffep-2f, -0x1.e1p-3f,
     -0x1.1afffep-3f, -0x1.75p-5f, 0x1.47p-5f, 0x1.ed0002p-4f, 0x1.a10002p-3f,
     0x1.2bp-2f, 0x1.8fp-2f, 0x1.010002p-1f, 0x1.490002p-1f, 0x1.b90002p-1f}};

template <typename T> struct ThetaRow;
template <> struct ThetaRow<float> { static constexpr int row = 0; };
template <> struct ThetaRow<__half> { static constexpr int row = 1; };
template <> struct ThetaRow<__nv_bfloat16> { static constexpr int row = 2; };

constexpr int kLut = 128;  // 65 buckets used; the rest catch NaN bucket indices

// lut[b] = (bits of the threshold inside bucket b or +inf, code at the bucket's
// left edge); bucket b covers quotients p with rint(32 p) = b - 32.
template <typename T>
__device__ __forceinline__ void build_lut(int2* lut) {
  for (int b = threadIdx.x; b < kLut; b += blockDim.x) {
    int code = 0;
    float th = __int_as_float(0x7f800000);
    if (b <= 64) {
      const float left = (float)(2 * b - 65) / 64.0f, right = (float)(2 * b - 63) / 64.0f;
      for (int i = 0; i < 15; ++i) {
        const float t = kTheta[ThetaRow<T>::row][i];
        code += (t <= left);
        if (t > left && t <= right) th = t;
      }
    }
    lut[b] = make_int2(__float_as_int(th), code);
  }
}

__device__ __forceinline__ int nf4_encode(float p, const int2* lut) {
  const float f = fmaf(p, 32.0f, 12582944.0f);  // 1.5 * 2^23 + 32: rint(32 p) + 32 in the low bits
  const int2 e = lut[__float_as_int(f) & (kLut - 1)];
  const int c = e.y + (p >= __int_as_float(e.x) ? 1 : 0);
  return (p == p) ? c : 0;
}

// The unrounded quotient p compared against kTheta[T].  For bf16 operands
// x * rcp_rn(scale) rounds to the same bf16 value as x / scale whenever the
// product is a normal number: a quotient of two 8-bit significands is either
// exact or at least 2^-17 (relative) away from every bf16 rounding midpoint
// (a midpoint needs a 9-bit odd significand), while x * rcp is within 2^-23
// of the quotient; tiny (subnormal) products lie far inside the code-7
// interval either way.  Other dtypes divide.
template <typename T>
__device__ __forceinline__ float nf4_quotient(float x, float scale, float rcp) {
  if constexpr (sizeof(T) == 2 && Ty<T>::code == LQ_BF16) return __fmul_rn(x, rcp);
  return __fdiv_rn(x, scale);
}

struct NfArgs {
  int64_t n, G, DG, n_groups, n_super;
  float lo;
  int g_shift;   // log2(G) when G is a power of two, else -1
  int dg_shift;  // log2(DG) when DG is a power of two, else -1
};

inline int log2_exact(int64_t v) {
  if (v <= 0 || (v & (v - 1))) return -1;
  int k = 0;
  while ((int64_t(1) << k) < v) ++k;
  return k;
}

// Write V (4 or 8) codes of elements e..e+V-1.
template <int V, int CODE_DT>
__device__ __forceinline__ void store_codes(void* codes, int64_t e, const int* c, int64_t n) {
  if constexpr (CODE_DT == LQ_U4X2) {
    uint8_t* p = static_cast<uint8_t*>(codes) + e / 2;
    if (e + V <= n) {
      uint32_t w = 0;
#pragma unroll
      for (int i = 0; i < V; ++i) w |= (uint32_t)c[i] << (4 * i);
      if constexpr (V == 8) *reinterpret_cast<uint32_t*>(p) = w;
      else *reinterpret_cast<uint16_t*>(p) = (uint16_t)w;
    } else {
      for (int i = 0; i < V; i += 2) {
        if (e + i >= n) break;
        int hi = (e + i + 1 < n) ? c[i + 1] : 0;
        p[i / 2] = (uint8_t)(c[i] | (hi << 4));
      }
    }
  } else if constexpr (CODE_DT == LQ_U8) {
    uint8_t* p = static_cast<uint8_t*>(codes) + e;
    for (int i = 0; i < V; ++i)
      if (e + i < n) p[i] = (uint8_t)c[i];
  } else {
    int64_t* p = static_cast<int64_t*>(codes) + e;
    if (e + V <= n) {
#pragma unroll
      for (int i = 0; i < V; i += 2)
        *reinterpret_cast<longlong2*>(p + i) = make_longlong2(c[i], c[i + 1]);
    } else {
      for (int i = 0; i < V; ++i)
        if (e + i < n) p[i] = c[i];
    }
  }
}

// Quantize kernel.  blockDim.x = 256; a team of `tps` lanes holds a group of
// G = tps*NVT*V elements (vector path, G % V == 0) in registers; every team
// keeps U groups in flight (loads of all U issued before any reduction).
template <typename T, int NVT, int CODE_DT, bool DQ>
__global__ void __launch_bounds__(256) nf4_quant_kernel(const T* __restrict__ x, NfArgs a,
                                                        int tps, void* __restrict__ codes,
                                                        T* __restrict__ scales,
                                                        T* __restrict__ q_scales,
                                                        T* __restrict__ dq_scales) {
  constexpr int V = 16 / sizeof(T);
  constexpr int U = 4;
  extern __shared__ float s_scale[];  // [DG] (double quant only)
  __shared__ MinMax red[8];
  __shared__ int2 lut[kLut];
  build_lut<T>(lut);
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t = lane & (tps - 1);
  const int teams_per_block = blockDim.x / tps;
  const int team = threadIdx.x / tps;
  for (int64_t sg = blockIdx.x; sg < a.n_super; sg += gridDim.x) {
    const int64_t g_begin = sg * a.DG;
    const int64_t g_end = min(g_begin + a.DG, a.n_groups);
    // all warps iterate the same number of times
    for (int64_t gb = g_begin; gb < g_end; gb += (int64_t)teams_per_block * U) {
      float v[U][NVT * V];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t g = gb + team + (int64_t)u * teams_per_block;
        const bool live = g < g_end;
        const int64_t e0 = g * a.G;
#pragma unroll
        for (int k = 0; k < NVT; ++k) {
          const int64_t e = e0 + (int64_t)(k * tps + t) * V;
          if (live && e + V <= a.n) {
            Vec16<T> w;
            w.u = ld_nc_v4(x + e);
#pragma unroll
            for (int i = 0; i < V; ++i) v[u][k * V + i] = Ty<T>::to_f(w.v[i]);
          } else {
#pragma unroll
            for (int i = 0; i < V; ++i)
              v[u][k * V + i] = (live && e + i < a.n) ? Ty<T>::to_f(x[e + i]) : 0.0f;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t g = gb + team + (int64_t)u * teams_per_block;
        const bool live = g < g_end;
        // absmax as an integer max of |x| bit patterns (NaN bits exceed +inf)
        int amb = 0;
#pragma unroll
        for (int i = 0; i < NVT * V; ++i) amb = max(amb, __float_as_int(v[u][i]) & 0x7FFFFFFF);
        for (int m = 1; m < tps; m <<= 1) amb = max(amb, __shfl_xor_sync(0xffffffffu, amb, m));
        const float am = __int_as_float(amb);
        if (!live) continue;
        const float s = (am < a.lo) ? a.lo : am;  // clamp(min=1e-12) in T; NaN passes
        if (t == 0) {
          scales[g] = Ty<T>::from_f(s);
          if constexpr (DQ) s_scale[g - g_begin] = s;
        }
        const float rcp = __frcp_rn(s);
        const int64_t e0 = g * a.G;
#pragma unroll
        for (int k = 0; k < NVT; ++k) {
          const int64_t e = e0 + (int64_t)(k * tps + t) * V;
          if (e >= a.n) continue;
          int c[V];
#pragma unroll
          for (int i = 0; i < V; ++i) c[i] = nf4_encode(nf4_quotient<T>(v[u][k * V + i], s, rcp), lut);
          store_codes<V, CODE_DT>(codes, e, c, a.n);
        }
      }
    }
    if constexpr (DQ) {
      __syncthreads();
      // dq_scale = absmax over the DG scales (zero-padded), clamp(1e-12) in T
      const int cnt = (int)(g_end - g_begin);
      MinMax r;
      r.init();
      for (int j = threadIdx.x; j < cnt; j += blockDim.x) r.add_max(fabsf(s_scale[j]));
      for (int m = 16; m >= 1; m >>= 1) r.shfl_xor_merge(m, true);
      if (lane == 0) red[warp] = r;
      __syncthreads();
      MinMax tot = red[0];
      for (int w = 1; w < (int)(blockDim.x >> 5); ++w) tot.merge(red[w]);
      float dq = fmax_nan(tot.mx, 0.0f);  // zero padding of a partial super-group
      dq = (dq < a.lo) ? a.lo : dq;
      if (threadIdx.x == 0) dq_scales[sg] = Ty<T>::from_f(dq);
      for (int j = threadIdx.x; j < cnt; j += blockDim.x) {
        float sn = tdiv<T>(s_scale[j], dq);
        float q = tclamp(trint(tmul<T>(sn, 127.0f)), -127.0f, 127.0f);
        q_scales[g_begin + j] = Ty<T>::from_f(q);
      }
      __syncthreads();
    }
  }
}

// bf16 input, packed 4-bit codes (QLoRALinear.pack_base): the same algorithm
// as nf4_quant_kernel on raw 32-bit words (two bf16 each).
//   absmax: |w| = w & 0x7FFF7FFF and an unsigned 16-bit-pair max; for
//           non-negative bf16 bit patterns the integer order is the float
//           order and NaN patterns lie above +inf, so NaN propagates;
//   quotient: x * rcp_rn(scale) (see nf4_quotient), one shift per element to
//           widen bf16 to fp32;
//   NaN: a quotient can only be NaN when the scale is not finite, so the
//           per-element NaN test runs only for such groups;
//   packing: codes folded into nibbles with integer multiply-adds.
__device__ __forceinline__ int nf4_encode_finite(float p, const int2* lut) {
  const float f = fmaf(p, 32.0f, 12582944.0f);
  const int2 e = lut[__float_as_int(f) & (kLut - 1)];
  return e.y + (p >= __int_as_float(e.x) ? 1 : 0);
}

__device__ __forceinline__ uint32_t nf4_pack8_bf16(const uint4& w, float rcp, bool finite,
                                                   const int2* lut) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
  int c[8];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float lo = __uint_as_float(ws[j] << 16), hi = __uint_as_float(ws[j] & 0xFFFF0000u);
    const float plo = __fmul_rn(lo, rcp), phi = __fmul_rn(hi, rcp);
    c[2 * j] = nf4_encode_finite(plo, lut);
    c[2 * j + 1] = nf4_encode_finite(phi, lut);
    if (!finite) {
      c[2 * j] = (plo == plo) ? c[2 * j] : 0;
      c[2 * j + 1] = (phi == phi) ? c[2 * j + 1] : 0;
    }
  }
  uint32_t acc = (uint32_t)c[7];
#pragma unroll
  for (int i = 6; i >= 0; --i) acc = acc * 16u + (uint32_t)c[i];
  return acc;
}

template <int NVT, bool DQ>
__global__ void __launch_bounds__(256) nf4_pack_bf16_kernel(const __nv_bfloat16* __restrict__ x,
                                                            NfArgs a, int tps,
                                                            uint8_t* __restrict__ codes,
                                                            __nv_bfloat16* __restrict__ scales,
                                                            __nv_bfloat16* __restrict__ q_scales,
                                                            __nv_bfloat16* __restrict__ dq_scales) {
  using T = __nv_bfloat16;
  constexpr int V = 8;
  constexpr int U = 4;
  extern __shared__ float s_scale[];  // [DG] (double quant only)
  __shared__ MinMax red[8];
  __shared__ int2 lut[kLut];
  build_lut<T>(lut);
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t = lane & (tps - 1);
  const int teams_per_block = blockDim.x / tps;
  const int team = threadIdx.x / tps;
  for (int64_t sg = blockIdx.x; sg < a.n_super; sg += gridDim.x) {
    const int64_t g_begin = sg * a.DG;
    const int64_t g_end = min(g_begin + a.DG, a.n_groups);
    for (int64_t gb = g_begin; gb < g_end; gb += (int64_t)teams_per_block * U) {
      uint4 w[U][NVT];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t g = gb + team + (int64_t)u * teams_per_block;
        const bool live = g < g_end;
#pragma unroll
        for (int k = 0; k < NVT; ++k) {
          const int64_t e = g * a.G + (int64_t)(k * tps + t) * V;
          if (live && e + V <= a.n) {
            w[u][k] = ld_nc_v4(x + e);
          } else {
            uint16_t hv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) hv[i] = (live && e + i < a.n) ? __bfloat16_as_ushort(x[e + i]) : 0;
            w[u][k] = make_uint4(hv[0] | (uint32_t)hv[1] << 16, hv[2] | (uint32_t)hv[3] << 16,
                                 hv[4] | (uint32_t)hv[5] << 16, hv[6] | (uint32_t)hv[7] << 16);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t g = gb + team + (int64_t)u * teams_per_block;
        const bool live = g < g_end;
        uint32_t m2 = 0;
#pragma unroll
        for (int k = 0; k < NVT; ++k) {
          m2 = __vmaxu2(m2, w[u][k].x & 0x7FFF7FFFu);
          m2 = __vmaxu2(m2, w[u][k].y & 0x7FFF7FFFu);
          m2 = __vmaxu2(m2, w[u][k].z & 0x7FFF7FFFu);
          m2 = __vmaxu2(m2, w[u][k].w & 0x7FFF7FFFu);
        }
        uint32_t m16 = max(m2 & 0xFFFFu, m2 >> 16);
        for (int m = 1; m < tps; m <<= 1) m16 = max(m16, __shfl_xor_sync(0xffffffffu, m16, m));
        if (!live) continue;
        const float am = __uint_as_float(m16 << 16);
        const float s = (am < a.lo) ? a.lo : am;  // clamp(min=1e-12) in bf16; NaN passes
        if (t == 0) {
          scales[g] = __float2bfloat16_rn(s);
          if constexpr (DQ) s_scale[g - g_begin] = s;
        }
        const float rcp = __frcp_rn(s);
        const bool finite = s <= 3.40282347e38f;
#pragma unroll
        for (int k = 0; k < NVT; ++k) {
          const int64_t e = g * a.G + (int64_t)(k * tps + t) * V;
          if (e >= a.n) continue;
          const uint32_t pk = nf4_pack8_bf16(w[u][k], rcp, finite, lut);
          if (e + V <= a.n) {
            *reinterpret_cast<uint32_t*>(codes + e / 2) = pk;
          } else {
            for (int i = 0; i < V; i += 2)
              if (e + i < a.n) codes[(e + i) / 2] = (uint8_t)((pk >> (4 * i)) & (e + i + 1 < a.n ? 0xFF : 0x0F));
          }
        }
      }
    }
    if constexpr (DQ) {
      __syncthreads();
      const int cnt = (int)(g_end - g_begin);
      MinMax r;
      r.init();
      for (int j = threadIdx.x; j < cnt; j += blockDim.x) r.add_max(fabsf(s_scale[j]));
      for (int m = 16; m >= 1; m >>= 1) r.shfl_xor_merge(m, true);
      if (lane == 0) red[warp] = r;
      __syncthreads();
      MinMax tot = red[0];
      for (int w2 = 1; w2 < (int)(blockDim.x >> 5); ++w2) tot.merge(red[w2]);
      float dq = fmax_nan(tot.mx, 0.0f);
      dq = (dq < a.lo) ? a.lo : dq;
      if (threadIdx.x == 0) dq_scales[sg] = __float2bfloat16_rn(dq);
      for (int j = threadIdx.x; j < cnt; j += blockDim.x) {
        float sn = tdiv<T>(s_scale[j], dq);
        float q = tclamp(trint(tmul<T>(sn, 127.0f)), -127.0f, 127.0f);
        q_scales[g_begin + j] = __float2bfloat16_rn(q);
      }
      __syncthreads();
    }
  }
}

// bf16 input, G = 64, packed codes, n % 64 == 0 (the QLoRA default): one
// thread per group, so the absmax, the reciprocal and the group's 32 code
// bytes stay in one thread, and a 256-thread block covers exactly one
// double-quantization super-group of DG = 256 scales.
//   bucket: f = fmaf(p, 4096, 1.5*2^23 + 4608) holds rint(4096 p) + 4608 in
//           its low mantissa bits, so bits(f) & 0x3F80 = 128 k with bucket
//           k = (rint(4096 p) + 4608) >> 7 in [4, 68] for p in [-1, 1]
//           (width 1/32, at most one threshold inside);
//   table:  16 copies of the 128-entry (threshold, code) table, entry k of
//           copy r at byte 128 k + 8 r; lane l reads copy l % 16, so the 16
//           lanes of a half-warp never share a bank: the byte offset of an
//           element's entry is one LOP3, (bits(f) & 0x3F80) | 8 (l % 16).
constexpr int kG64Rep = 16;
constexpr float kG64Magic = 12582912.0f + 4608.0f;

// Bucket k holds the quotients with rint(4096 p) in [128 k - 4608,
// 128 k - 4481], i.e. p in [(256 k - 9217) / 8192, (256 k - 8961) / 8192].
__device__ __forceinline__ void build_lut_g64(int2* lut) {
  for (int k = threadIdx.x; k < 128; k += blockDim.x) {
    const float left = (float)(256 * k - 9217) / 8192.0f, right = (float)(256 * k - 8961) / 8192.0f;
    int code = 0;
    float th = __int_as_float(0x7f800000);
    for (int i = 0; i < 15; ++i) {
      const float t = kTheta[ThetaRow<__nv_bfloat16>::row][i];
      code += (t <= left);
      if (t > left && t <= right) th = t;
    }
    const int2 e = make_int2(__float_as_int(th), code);
#pragma unroll
    for (int r = 0; r < kG64Rep; ++r) lut[k * kG64Rep + r] = e;
  }
}

// Codes of the 64 elements in w (element 8k + i at bits 4i of out[k]).
// CHECK: the scale is not finite, so quotients may be NaN (code 0).
template <bool CHECK>
__device__ __forceinline__ void nf4_encode_g64(const uint4 (&w)[8], float rcp, const char* lutb,
                                               uint32_t rep, uint32_t (&out)[8]) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t ws[4] = {w[k].x, w[k].y, w[k].z, w[k].w};
    uint32_t acc = 0;
#pragma unroll
    for (int j = 3; j >= 0; --j) {
#pragma unroll
      for (int h = 1; h >= 0; --h) {
        const float x = __uint_as_float(h ? (ws[j] & 0xFFFF0000u) : (ws[j] << 16));
        const float p = __fmul_rn(x, rcp);
        const float f = fmaf(p, 4096.0f, kG64Magic);
        const int2 e = *reinterpret_cast<const int2*>(lutb + ((__float_as_uint(f) & 0x3F80u) | rep));
        int c = e.y + (p >= __int_as_float(e.x) ? 1 : 0);
        if (CHECK) c = (p == p) ? c : 0;
        acc = acc * 16u + (uint32_t)c;
      }
    }
    out[k] = acc;
  }
}

struct G64Out {
  uint4* codes;
  __nv_bfloat16* scales;
  __nv_bfloat16* q_scales;
  __nv_bfloat16* dq_scales;
  int64_t n_groups;
  float lo;
};

// One super-group (256 groups, one per thread of the block), first half:
// scale and codes of the thread's group, and (DQ) the warp's largest scale in
// wmax[warp].  Returns the group's scale.
__device__ __forceinline__ float g64_group(const uint4 (&w)[8], int64_t sg, const G64Out& o,
                                           const char* lutb, uint32_t rep, uint32_t* wmax) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t g = sg * 256 + threadIdx.x;
  const bool live = g < o.n_groups;
  // |x| as unsigned bf16 pairs; the pair max keeps NaN (its pattern is above +inf)
  uint32_t m2 = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    m2 = __vimax3_u16x2(m2, w[k].x & 0x7FFF7FFFu, w[k].y & 0x7FFF7FFFu);
    m2 = __vimax3_u16x2(m2, w[k].z & 0x7FFF7FFFu, w[k].w & 0x7FFF7FFFu);
  }
  const float am = __uint_as_float(max(m2 & 0xFFFFu, m2 >> 16) << 16);
  const float s = (am < o.lo) ? o.lo : am;  // clamp(min=1e-12) in bf16; NaN passes
  const float rcp = __frcp_rn(s);
  uint32_t out[8];
  if (s <= 3.40282347e38f) nf4_encode_g64<false>(w, rcp, lutb, rep, out);
  else nf4_encode_g64<true>(w, rcp, lutb, rep, out);
  if (live) {
    o.scales[g] = __float2bfloat16_rn(s);
    o.codes[2 * g] = make_uint4(out[0], out[1], out[2], out[3]);
    o.codes[2 * g + 1] = make_uint4(out[4], out[5], out[6], out[7]);
  }
  if (wmax) {
    // absmax of the warp's scales (s >= 0 or +NaN: integer order is float order)
    const uint32_t mb = __reduce_max_sync(0xffffffffu, live ? __float_as_uint(s) : 0u);
    if (lane == 0) wmax[warp] = mb;
  }
  return s;
}

// Second half (DQ), after a block barrier has made the 8 warp maxima
// visible: the super-group's dq scale and the thread's quantized scale.
__device__ __forceinline__ void g64_double_quant(float s, int64_t sg, const G64Out& o, const uint32_t* wmax) {
  using T = __nv_bfloat16;
  const int64_t g = sg * 256 + threadIdx.x;
  uint32_t tot = wmax[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) tot = max(tot, wmax[i]);
  float dq = __uint_as_float(tot);
  dq = (dq < o.lo) ? o.lo : dq;
  if (threadIdx.x == 0) o.dq_scales[sg] = __float2bfloat16_rn(dq);
  if (g < o.n_groups) {
    const float sn = tdiv<T>(s, dq);
    const float q = tclamp(trint(tmul<T>(sn, 127.0f)), -127.0f, 127.0f);
    o.q_scales[g] = __float2bfloat16_rn(q);
  }
}

// Input staging: the weight, viewed as [n_groups][128 bytes], is read by TMA
// one super-group (256 rows = 32 KB) per copy with the 128-byte swizzle, into
// a ring of kG64Stages shared-memory stages; row r's 16-byte chunk c lands at
// chunk c ^ (r % 8), so thread t reads its group as chunks k ^ (t % 8) and
// the 8 lanes of each quarter-warp hit 8 different bank groups.  Thread 0
// issues the copies; a stage is refilled (with the super-group kG64Stages
// iterations ahead) once every thread has read it.  Waits are bounded: a copy
// that has not landed after 2 s ends the block, whose current super-group
// then gets NaN scales.
constexpr int kG64Stages = 2;
constexpr int kG64StageBytes = 256 * 128;
constexpr int kG64LutBytes = 128 * kG64Rep * 8;
// dynamic shared memory: the stages, the barriers and the 1024-byte alignment
// slack; the code table is a static __shared__ array (kG64LutBytes)
constexpr int kG64SmemBytes = kG64Stages * kG64StageBytes + 64 + 1024;

template <bool DQ>
__global__ void __launch_bounds__(256, 2) nf4_pack_g64_kernel(const __grid_constant__ CUtensorMap tmap,
                                                              int64_t n_super, G64Out o) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // The code table is a static __shared__ array so that its per-element
  // lookups compile to shared-window loads with 32-bit addresses (a pointer
  // into the dynamic area above, aligned through an integer, is a generic
  // pointer: 64-bit address arithmetic per lookup; measured 9 % slower).
  __shared__ __align__(128) int2 lut[128 * kG64Rep];
  static_assert(sizeof(lut) == kG64LutBytes, "table size");
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kG64Stages * kG64StageBytes);
  __shared__ uint32_t red[2][8];  // warp maxima, by iteration parity
  __shared__ int s_fail;
  const int t = threadIdx.x;
  const int64_t step = gridDim.x;
  if (t == 0) {
    s_fail = 0;
    for (int i = 0; i < kG64Stages; ++i) mbar_init(&bars[i], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  build_lut_g64(lut);
  __syncthreads();
  pdl_wait();     // the previous kernel in the stream is done (its memory may be reused here)
  pdl_trigger();  // the next kernel may launch (it waits for this one the same way)
  if (t == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap)) : "memory");
    for (int j = 0; j < kG64Stages; ++j) {
      const int64_t sj = blockIdx.x + j * step;
      if (sj < n_super) {
        mbar_expect_tx(&bars[j], kG64StageBytes);
        tma_load_2d(smem + j * kG64StageBytes, &tmap, 0, (int)(sj * 256), &bars[j]);
      }
    }
  }
  const char* lutb = reinterpret_cast<const char*>(lut);
  const uint32_t rep = (t & 15) * 8;
  int it = 0;
  int64_t sg = blockIdx.x;
  for (; sg < n_super; sg += step, ++it) {
    const int s = it % kG64Stages;
    if (!mbar_wait(&bars[s], (it / kG64Stages) & 1)) s_fail = 1;
    uint4 w[8];
    const uint32_t row = smem_u32(smem) + s * kG64StageBytes + t * 128;
#pragma unroll
    for (int k = 0; k < 8; ++k) w[k] = lds_v4(row + ((k ^ (t & 7)) << 4));
    const float sc = g64_group(w, sg, o, lutb, rep, DQ ? red[it & 1] : nullptr);
    // one barrier per super-group: stage s has been read by every thread and
    // the warp maxima of this super-group are visible (red is double-buffered
    // by iteration parity, so the next super-group cannot overwrite them)
    __syncthreads();
    if (s_fail) break;
    if (t == 0) {
      const int64_t nsg = sg + kG64Stages * step;
      if (nsg < n_super) {
        mbar_expect_tx(&bars[s], kG64StageBytes);
        tma_load_2d(smem + s * kG64StageBytes, &tmap, 0, (int)(nsg * 256), &bars[s]);
      }
    }
    if constexpr (DQ) g64_double_quant(sc, sg, o, red[it & 1]);
  }
  if (sg < n_super) {  // a copy timed out: mark this super-group, wait out the copies still in flight
    const int64_t g = sg * 256 + t;
    if (g < o.n_groups) o.scales[g] = __float2bfloat16_rn(__int_as_float(0x7fc00000));
    if (t == 0) {
      for (int j = 0; j < kG64Stages; ++j) {  // the timed-out copy and the ones issued after it
        const int jt = it + j;
        if (sg + j * step < n_super) mbar_wait(&bars[jt % kG64Stages], (jt / kG64Stages) & 1);
      }
    }
  }
}

// Generic scalar path (any G): pass 1 writes the group scales (one block per
// group), pass 2 writes codes for pairs of flat elements, so packed bytes are
// always written whole even when a pair straddles two groups.
template <typename T>
__global__ void __launch_bounds__(256) nf4_scales_kernel(const T* __restrict__ x, NfArgs a,
                                                         T* __restrict__ scales) {
  __shared__ MinMax red[8];
  for (int64_t g = blockIdx.x; g < a.n_groups; g += gridDim.x) {
    const int64_t e0 = g * a.G;
    MinMax r;
    r.init();
    for (int64_t i = threadIdx.x; i < a.G; i += blockDim.x) {
      float v = (e0 + i < a.n) ? Ty<T>::to_f(x[e0 + i]) : 0.0f;
      r.add(fabsf(v));
    }
    for (int m = 16; m >= 1; m >>= 1) r.shfl_xor_merge(m);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = r;
    __syncthreads();
    MinMax tot = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) tot.merge(red[w]);
    float s = fmax_nan(tot.mx, 0.0f);
    s = (s < a.lo) ? a.lo : s;
    if (threadIdx.x == 0) scales[g] = Ty<T>::from_f(s);
  }
}

template <typename T, int CODE_DT>
__global__ void __launch_bounds__(256) nf4_codes_kernel(const T* __restrict__ x, NfArgs a,
                                                        const T* __restrict__ scales,
                                                        void* __restrict__ codes) {
  __shared__ int2 lut[kLut];
  build_lut<T>(lut);
  __syncthreads();
  const int64_t npair = (a.n + 1) / 2;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < npair;
       i += (int64_t)gridDim.x * blockDim.x) {
    int c[2] = {0, 0};
    for (int k = 0; k < 2; ++k) {
      const int64_t e = 2 * i + k;
      if (e < a.n) c[k] = nf4_encode(__fdiv_rn(Ty<T>::to_f(x[e]), Ty<T>::to_f(scales[e / a.G])), lut);
    }
    if constexpr (CODE_DT == LQ_U4X2) {
      static_cast<uint8_t*>(codes)[i] = (uint8_t)(c[0] | (c[1] << 4));
    } else if constexpr (CODE_DT == LQ_U8) {
      for (int k = 0; k < 2; ++k)
        if (2 * i + k < a.n) static_cast<uint8_t*>(codes)[2 * i + k] = (uint8_t)c[k];
    } else {
      for (int k = 0; k < 2; ++k)
        if (2 * i + k < a.n) static_cast<int64_t*>(codes)[2 * i + k] = c[k];
    }
  }
}

// ---------------------------------------------------------------------------
// Dequantize: out[e] = table_T[code[e]] * scale[e / G] in T.  When q_scales
// is given the scale is first restored as (q / 127) * dq (qlora.py:199-223).
// Thread = 8 consecutive elements.
// ---------------------------------------------------------------------------
template <typename T, int CODE_DT>
__global__ void __launch_bounds__(256) nf4_dequant_kernel(const void* __restrict__ codes, NfArgs a,
                                                          const T* __restrict__ scales,
                                                          const T* __restrict__ q_scales,
                                                          const T* __restrict__ dq_scales,
                                                          T* __restrict__ out, int vec,
                                                          int64_t e_begin) {
  __shared__ float tab[16];
  if (threadIdx.x < 16) tab[threadIdx.x] = Ty<T>::round(kNF4[threadIdx.x]);
  __syncthreads();
  const int64_t nthr = (a.n - e_begin + 7) / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nthr;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e0 = e_begin + i * 8;
    int c[8];
    if (CODE_DT == LQ_U4X2 && vec && e0 + 8 <= a.n && (e0 & 7) == 0) {
      uint32_t w = *reinterpret_cast<const uint32_t*>(static_cast<const uint8_t*>(codes) + e0 / 2);
#pragma unroll
      for (int k = 0; k < 8; ++k) c[k] = (w >> (4 * k)) & 15;
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        int64_t e = e0 + k;
        int cv = 0;
        if (e < a.n) {
          if constexpr (CODE_DT == LQ_U4X2) cv = (static_cast<const uint8_t*>(codes)[e / 2] >> (4 * (e & 1))) & 15;
          else if constexpr (CODE_DT == LQ_U8) cv = static_cast<const uint8_t*>(codes)[e];
          else cv = (int)static_cast<const int64_t*>(codes)[e];
        }
        c[k] = cv;
      }
    }
    float o[8];
    int64_t glast = -1;
    float s = 0.0f;
    const bool one_group = (a.G & 7) == 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int64_t g = one_group ? (k == 0 ? (a.g_shift >= 0 ? (e0 >> a.g_shift) : e0 / a.G) : glast)
                                  : (e0 + k) / a.G;
      if (g != glast && e0 + k < a.n) {
        glast = g;
        if (q_scales) {
          s = tmul<T>(tdiv<T>(Ty<T>::to_f(q_scales[g]), 127.0f), Ty<T>::to_f(dq_scales[g / a.DG]));
        } else {
          s = Ty<T>::to_f(scales[g]);
        }
      }
      // torch indexing of an out-of-range code would raise; codes are 0..15 here
      o[k] = tmul<T>(tab[c[k] & 15], s);
    }
    if (vec && e0 + 8 <= a.n) {
      if constexpr (sizeof(T) == 2) {
        Vec16<T> u;
#pragma unroll
        for (int k = 0; k < 8; ++k) u.v[k] = Ty<T>::from_f(o[k]);
        st_v4(out + e0, u.u);
      } else {
        st_v4(out + e0, make_uint4(__float_as_uint(o[0]), __float_as_uint(o[1]), __float_as_uint(o[2]), __float_as_uint(o[3])));
        st_v4(out + e0 + 4, make_uint4(__float_as_uint(o[4]), __float_as_uint(o[5]), __float_as_uint(o[6]), __float_as_uint(o[7])));
      }
    } else {
      for (int k = 0; k < 8; ++k)
        if (e0 + k < a.n) out[e0 + k] = Ty<T>::from_f(o[k]);
    }
  }
}

// Vectorized dequantize of packed codes for 2-byte T (G % 8 == 0): a chunk is
// 8 elements (4 code bytes, 16 output bytes) inside one group, and lane l of a
// warp takes chunks base + 32 k + l, so every load and store instruction of
// the warp covers one contiguous span (128 bytes of codes, 512 of output).
// pair[b] holds round_T(NF4_TABLE) of both nibbles of code byte b; the
// product with the scale is __hmul2, whose correctly rounded result equals
// round_T(fp32 product) because the product of two 8- or 11-bit significands
// is exact in fp32.  The 256-entry table is stored 32 times, entry b of copy
// r at word 32 b + r, and lane l reads copy l: no bank conflicts.
constexpr int kUnpackK = 8;  // chunks per lane per warp iteration

template <typename T>
__global__ void __launch_bounds__(256) nf4_unpack_vec_kernel(const uint32_t* __restrict__ codes,
                                                             NfArgs a,
                                                             const T* __restrict__ scales,
                                                             const T* __restrict__ q_scales,
                                                             const T* __restrict__ dq_scales,
                                                             uint4* __restrict__ out, int64_t nchunk) {
  __shared__ __align__(16) uint32_t pair[256 * 32];
  __shared__ uint32_t pair1[256];
  {
    const int b = threadIdx.x;  // blockDim.x == 256
    union {
      T h[2];
      uint32_t u;
    } pr;
    pr.h[0] = Ty<T>::from_f(Ty<T>::round(kNF4[b & 15]));
    pr.h[1] = Ty<T>::from_f(Ty<T>::round(kNF4[b >> 4]));
    pair1[b] = pr.u;
  }
  __syncthreads();
  // replicate: thread t fills words 4t..4t+3 of each 4 KB slice (copies of
  // entry t/8 + 32j), so the 8 lanes of a quarter-warp store 128 contiguous bytes
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t v = pair1[(threadIdx.x >> 3) + 32 * j];
    reinterpret_cast<uint4*>(pair)[threadIdx.x + 256 * j] = make_uint4(v, v, v, v);
  }
  __syncthreads();
  pdl_wait();     // the previous kernel in the stream (the packing) is done
  pdl_trigger();
  const char* pb = reinterpret_cast<const char*>(pair);
  const int lane = threadIdx.x & 31;
  const uint32_t lane4 = (uint32_t)lane * 4;
  const int c_shift = a.g_shift >= 3 ? a.g_shift - 3 : -1;  // chunk -> group
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t span = 32 * kUnpackK;
  for (int64_t base = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * span; base < nchunk;
       base += warps * span) {
    // every load of the iteration (codes and scales) is issued before any use
    uint32_t w[kUnpackK];
    T sq[kUnpackK], sd[kUnpackK];
#pragma unroll
    for (int k = 0; k < kUnpackK; ++k) {
      const int64_t c = base + 32 * k + lane;
      const bool live = c < nchunk;
      const int64_t g = !live ? 0 : (c_shift >= 0 ? (c >> c_shift) : (c * 8) / a.G);
      w[k] = live ? __ldg(codes + c) : 0u;
      if (q_scales) {
        sq[k] = q_scales[g];
        sd[k] = dq_scales[a.dg_shift >= 0 ? (g >> a.dg_shift) : g / a.DG];
      } else {
        sq[k] = scales[g];
      }
    }
#pragma unroll
    for (int k = 0; k < kUnpackK; ++k) {
      const int64_t c = base + 32 * k + lane;
      if (c >= nchunk) break;
      float s;
      if (q_scales) s = tmul<T>(tdiv<T>(Ty<T>::to_f(sq[k]), 127.0f), Ty<T>::to_f(sd[k]));
      else s = Ty<T>::to_f(sq[k]);
      union {
        T h[2];
        uint32_t u;
      } s2;
      s2.h[0] = s2.h[1] = Ty<T>::from_f(s);
      uint32_t o[4];
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t off = (b == 0 ? (w[k] << 7) : (w[k] >> (8 * b - 7))) & 0x7F80u;
        uint32_t pv = *reinterpret_cast<const uint32_t*>(pb + (off | lane4));
        if constexpr (Ty<T>::code == LQ_BF16) {
          __nv_bfloat162 r = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&pv),
                                     *reinterpret_cast<__nv_bfloat162*>(&s2.u));
          o[b] = *reinterpret_cast<uint32_t*>(&r);
        } else {
          __half2 r = __hmul2(*reinterpret_cast<__half2*>(&pv), *reinterpret_cast<__half2*>(&s2.u));
          o[b] = *reinterpret_cast<uint32_t*>(&r);
        }
      }
      st_v4(out + c, make_uint4(o[0], o[1], o[2], o[3]));
    }
  }
}

// Code container conversion (I64 / U8 / U4X2): pairs of elements per thread so
// packed bytes are written whole.
__device__ __forceinline__ int load_code(const void* p, int dt, int64_t e) {
  if (dt == LQ_U4X2) return (static_cast<const uint8_t*>(p)[e >> 1] >> (4 * (e & 1))) & 15;
  if (dt == LQ_U8) return static_cast<const uint8_t*>(p)[e];
  return (int)static_cast<const int64_t*>(p)[e];
}

__global__ void __launch_bounds__(256) codes_convert_kernel(const void* __restrict__ src, int sdt,
                                                            int64_t n, void* __restrict__ dst,
                                                            int ddt) {
  const int64_t npair = (n + 1) / 2;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < npair;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = 2 * i;
    const int c0 = load_code(src, sdt, e);
    const int c1 = (e + 1 < n) ? load_code(src, sdt, e + 1) : 0;
    if (ddt == LQ_U4X2) {
      static_cast<uint8_t*>(dst)[i] = (uint8_t)((c0 & 15) | ((c1 & 15) << 4));
    } else if (ddt == LQ_U8) {
      static_cast<uint8_t*>(dst)[e] = (uint8_t)c0;
      if (e + 1 < n) static_cast<uint8_t*>(dst)[e + 1] = (uint8_t)c1;
    } else {
      static_cast<int64_t*>(dst)[e] = c0;
      if (e + 1 < n) static_cast<int64_t*>(dst)[e + 1] = c1;
    }
  }
}

// double_quantize / double_dequantize on a scale vector (qlora.py:164-223).
template <typename T>
__global__ void __launch_bounds__(256) double_quant_kernel(const T* __restrict__ s, int64_t n,
                                                           int64_t DG, float lo,
                                                           T* __restrict__ q,
                                                           T* __restrict__ dq) {
  __shared__ MinMax red[8];
  const int64_t nd = (n + DG - 1) / DG;
  for (int64_t d = blockIdx.x; d < nd; d += gridDim.x) {
    const int64_t b = d * DG, e = min(b + DG, n);
    MinMax r;
    r.init();
    for (int64_t j = b + threadIdx.x; j < e; j += blockDim.x) r.add(fabsf(Ty<T>::to_f(s[j])));
    for (int m = 16; m >= 1; m >>= 1) r.shfl_xor_merge(m);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = r;
    __syncthreads();
    MinMax tot = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) tot.merge(red[w]);
    float m = fmax_nan(tot.mx, 0.0f);  // padding zeros
    m = (m < lo) ? lo : m;
    if (threadIdx.x == 0) dq[d] = Ty<T>::from_f(m);
    for (int64_t j = b + threadIdx.x; j < e; j += blockDim.x) {
      float sn = tdiv<T>(Ty<T>::to_f(s[j]), m);
      q[j] = Ty<T>::from_f(tclamp(trint(tmul<T>(sn, 127.0f)), -127.0f, 127.0f));
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) double_dequant_kernel(const T* __restrict__ q,
                                                             const T* __restrict__ dq, int64_t n,
                                                             int64_t DG, T* __restrict__ out) {
  for (int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; j < n;
       j += (int64_t)gridDim.x * blockDim.x)
    out[j] = Ty<T>::from_f(tmul<T>(tdiv<T>(Ty<T>::to_f(q[j]), 127.0f), Ty<T>::to_f(dq[j / DG])));
}

int grid_cap(int64_t want, int per_sm = 8) {
  int64_t cap = (int64_t)num_sms() * per_sm;
  return (int)(want < 1 ? 1 : (want < cap ? want : cap));
}

// TMA view of a bf16 weight as [n_groups][64 elements] (128-byte rows),
// boxes of 256 rows, 128-byte swizzle; false when the driver entry point is
// missing or rejects the map (the caller then uses the register path).
bool g64_tensor_map(CUtensorMap* map, const void* x, int64_t n_groups) {
  EncodeTiledFn enc = encode_fn();
  if (enc == nullptr || n_groups >= (int64_t(1) << 31)) return false;
  cuuint64_t dims[2] = {64, (cuuint64_t)n_groups};
  cuuint64_t strides[1] = {128};
  cuuint32_t box[2] = {64, 256};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T, int CODE_DT, bool DQ>
int nf4_quant_launch(const T* x, NfArgs a, void* codes, T* scales, T* qs, T* dqs, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  const bool vec = (a.G % V == 0) && aligned16(x) && (a.G / V) <= 32 * 4 &&
                   (CODE_DT != LQ_U4X2 || (a.G * 4) % 8 == 0) &&
                   (reinterpret_cast<uintptr_t>(codes) % (CODE_DT == LQ_I64 ? 16 : 4) == 0);
  // the fused one-pass kernels hold a group in a team of tps lanes x nvt
  // vectors; other group sizes (and unaligned buffers) take the scalar path:
  // scales, then codes, then (double quantization) the scales' second level
  const int64_t nv = a.G / V;
  int tps = 1, nvt = 1;
  bool fused = vec;
  if (fused && nv <= 32) {
    while (tps < nv) tps <<= 1;
    fused = (tps == nv);
  } else if (fused) {
    tps = 32;
    nvt = (int)(nv / 32);
    fused = (nv % 32 == 0) && (nvt == 2 || nvt == 4);
  }
  if (!fused) {
    nf4_scales_kernel<T><<<grid_cap(a.n_groups, 16), 256, 0, st>>>(x, a, scales);
    int rc = launched("nf4_scales_kernel");
    if (rc != LQ_OK) return rc;
    nf4_codes_kernel<T, CODE_DT><<<grid_cap((a.n + 511) / 512, 16), 256, 0, st>>>(x, a, scales, codes);
    rc = launched("nf4_codes_kernel");
    if (rc != LQ_OK || !DQ) return rc;
    double_quant_kernel<T><<<grid_cap(a.n_super, 16), 256, 0, st>>>(scales, a.n_groups, a.DG, a.lo, qs, dqs);
    return launched("double_quant_kernel");
  }
  if (!DQ) {
    a.DG = 256 / tps * 8;  // super-group = a few block iterations
    a.n_super = (a.n_groups + a.DG - 1) / a.DG;
  }
  size_t smem = DQ ? (size_t)a.DG * sizeof(float) : 0;
  int grid = grid_cap(a.n_super, 8);
  if constexpr (std::is_same<T, __nv_bfloat16>::value && CODE_DT == LQ_U4X2) {
    uint8_t* cp = static_cast<uint8_t*>(codes);
    if (a.G == 64 && a.n % 64 == 0 && aligned16(codes) && (!DQ || a.DG == 256)) {
      const int64_t n_chunks = (a.n_groups + 255) / 256;
      CUtensorMap map;
      if (g64_tensor_map(&map, x, a.n_groups)) {
        G64Out o;
        o.codes = reinterpret_cast<uint4*>(cp);
        o.scales = scales;
        o.q_scales = qs;
        o.dq_scales = dqs;
        o.n_groups = a.n_groups;
        o.lo = a.lo;
        auto kern = nf4_pack_g64_kernel<DQ>;
        static std::atomic<uint64_t> attr_done{0};  // one bit per device
        int dev = 0;
        cudaGetDevice(&dev);
        const uint64_t bit = 1ull << (dev & 63);
        if (!(attr_done.load() & bit)) {
          cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kG64SmemBytes);
          LQ_REQUIRE(e == cudaSuccess, LQ_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
          attr_done.fetch_or(bit);
        }
        launch_pdl(kern, dim3((unsigned)grid_cap(n_chunks, 2)), dim3(256), kG64SmemBytes, st, map, n_chunks, o);
        return launched("nf4_pack_g64_kernel");
      }
    }
    if (nvt == 1) nf4_pack_bf16_kernel<1, DQ><<<grid, 256, smem, st>>>(x, a, tps, cp, scales, qs, dqs);
    else if (nvt == 2) nf4_pack_bf16_kernel<2, DQ><<<grid, 256, smem, st>>>(x, a, tps, cp, scales, qs, dqs);
    else nf4_pack_bf16_kernel<4, DQ><<<grid, 256, smem, st>>>(x, a, tps, cp, scales, qs, dqs);
    return launched("nf4_pack_bf16_kernel");
  }
  if (nvt == 1) nf4_quant_kernel<T, 1, CODE_DT, DQ><<<grid, 256, smem, st>>>(x, a, tps, codes, scales, qs, dqs);
  else if (nvt == 2) nf4_quant_kernel<T, 2, CODE_DT, DQ><<<grid, 256, smem, st>>>(x, a, tps, codes, scales, qs, dqs);
  else nf4_quant_kernel<T, 4, CODE_DT, DQ><<<grid, 256, smem, st>>>(x, a, tps, codes, scales, qs, dqs);
  return launched("nf4_quant_kernel");
}

template <typename T>
int nf4_quant_t(const void* x, int64_t n, int64_t G, int64_t DG, void* codes, int cdt,
                void* scales, void* qs, void* dqs, cudaStream_t st) {
  NfArgs a;
  a.n = n;
  a.G = G;
  a.n_groups = (n + G - 1) / G;
  a.DG = DG > 0 ? DG : 1;
  a.n_super = (a.n_groups + a.DG - 1) / a.DG;
  a.lo = lo_clamp_value<T>();
  a.g_shift = log2_exact(G);
  a.dg_shift = log2_exact(a.DG);
  const T* xp = static_cast<const T*>(x);
  T* sp = static_cast<T*>(scales);
  if (DG > 0) {
    LQ_REQUIRE(DG <= 8192, LQ_ERANGE, "dq_group %lld above 8192", (long long)DG);
    switch (cdt) {
      case LQ_U4X2: return nf4_quant_launch<T, LQ_U4X2, true>(xp, a, codes, sp, (T*)qs, (T*)dqs, st);
      case LQ_U8: return nf4_quant_launch<T, LQ_U8, true>(xp, a, codes, sp, (T*)qs, (T*)dqs, st);
      case LQ_I64: return nf4_quant_launch<T, LQ_I64, true>(xp, a, codes, sp, (T*)qs, (T*)dqs, st);
    }
  } else {
    switch (cdt) {
      case LQ_U4X2: return nf4_quant_launch<T, LQ_U4X2, false>(xp, a, codes, sp, nullptr, nullptr, st);
      case LQ_U8: return nf4_quant_launch<T, LQ_U8, false>(xp, a, codes, sp, nullptr, nullptr, st);
      case LQ_I64: return nf4_quant_launch<T, LQ_I64, false>(xp, a, codes, sp, nullptr, nullptr, st);
    }
  }
  set_error("unsupported code dtype %d", cdt);
  return LQ_EDTYPE;
}

template <typename T>
int nf4_dequant_t(const void* codes, int cdt, int64_t n, int64_t G, int64_t DG, const void* s,
                  const void* qs, const void* dqs, void* out, cudaStream_t st) {
  NfArgs a;
  a.n = n;
  a.G = G;
  a.DG = DG > 0 ? DG : 1;
  a.n_groups = (n + G - 1) / G;
  a.n_super = 0;
  a.lo = 0;
  a.g_shift = log2_exact(G);
  a.dg_shift = log2_exact(a.DG);
  const T* sp = static_cast<const T*>(s);
  const T* q = static_cast<const T*>(qs);
  const T* d = static_cast<const T*>(dqs);
  T* o = static_cast<T*>(out);
  int64_t done = 0;
  if (sizeof(T) == 2 && cdt == LQ_U4X2 && G % 8 == 0 && reinterpret_cast<uintptr_t>(codes) % 4 == 0 &&
      aligned16(out)) {
    const int64_t nchunk = n / 8;
    if (nchunk > 0) {
      const int grid = resident_grid(nf4_unpack_vec_kernel<T>, 256, 0, (nchunk + 256 * kUnpackK - 1) / (256 * kUnpackK));
      launch_pdl(nf4_unpack_vec_kernel<T>, dim3(grid), dim3(256), 0, st, static_cast<const uint32_t*>(codes), a,
                 sp, q, d, reinterpret_cast<uint4*>(o), nchunk);
      int rc = launched("nf4_unpack_vec_kernel");
      if (rc) return rc;
      done = nchunk * 8;
    }
    if (done == n) return LQ_OK;
  }
  int vec = aligned16(out) && (reinterpret_cast<uintptr_t>(codes) % 4 == 0);
  int grid = grid_cap((n - done + 8 * 256 - 1) / (8 * 256), 16);
  switch (cdt) {
    case LQ_U4X2: nf4_dequant_kernel<T, LQ_U4X2><<<grid, 256, 0, st>>>(codes, a, sp, q, d, o, vec, done); break;
    case LQ_U8: nf4_dequant_kernel<T, LQ_U8><<<grid, 256, 0, st>>>(codes, a, sp, q, d, o, vec, done); break;
    case LQ_I64: nf4_dequant_kernel<T, LQ_I64><<<grid, 256, 0, st>>>(codes, a, sp, q, d, o, vec, done); break;
    default: set_error("unsupported code dtype %d", cdt); return LQ_EDTYPE;
  }
  return launched("nf4_dequant_kernel");
}

#define LQ_DISPATCH_FLOAT(dt, FN, ...)                                   \
  switch (dt) {                                                          \
    case LQ_F32: return FN<float>(__VA_ARGS__);                          \
    case LQ_F16: return FN<__half>(__VA_ARGS__);                         \
    case LQ_BF16: return FN<__nv_bfloat16>(__VA_ARGS__);                 \
    default: ::lq::set_error("unsupported dtype %d", (int)(dt)); return LQ_EDTYPE; \
  }

template <typename T>
int dq_t(const void* s, int64_t n, int64_t DG, void* q, void* dq, cudaStream_t st) {
  const int64_t nd = (n + DG - 1) / DG;
  double_quant_kernel<T><<<grid_cap(nd, 16), 256, 0, st>>>(static_cast<const T*>(s), n, DG, lo_clamp_value<T>(), static_cast<T*>(q), static_cast<T*>(dq));
  return launched("double_quant_kernel");
}
template <typename T>
int ddq_t(const void* q, const void* dq, int64_t n, int64_t DG, void* out, cudaStream_t st) {
  double_dequant_kernel<T><<<grid_cap((n + 255) / 256, 16), 256, 0, st>>>(static_cast<const T*>(q), static_cast<const T*>(dq), n, DG, static_cast<T*>(out));
  return launched("double_dequant_kernel");
}

}  // namespace
}  // namespace lq

using namespace lq;

extern "C" int lq_nf4_quantize(const void* x, int x_dtype, int64_t n, int64_t group, void* codes,
                               int code_dtype, void* scales, void* stream) {
  LQ_REQUIRE(n >= 0 && group >= 1, LQ_EINVAL, "bad size n=%lld group=%lld", (long long)n, (long long)group);
  if (n == 0) return LQ_OK;
  LQ_REQUIRE(x && codes && scales, LQ_EINVAL, "NULL pointer");
  LQ_DISPATCH_FLOAT(x_dtype, nf4_quant_t, x, n, group, 0, codes, code_dtype, scales, nullptr, nullptr, as_stream(stream));
}

extern "C" int lq_nf4_dequantize(const void* codes, int code_dtype, int64_t n, int64_t group,
                                 const void* scales, int s_dtype, void* out, void* stream) {
  LQ_REQUIRE(n >= 0 && group >= 1, LQ_EINVAL, "bad size");
  if (n == 0) return LQ_OK;
  LQ_REQUIRE(codes && scales && out, LQ_EINVAL, "NULL pointer");
  LQ_DISPATCH_FLOAT(s_dtype, nf4_dequant_t, codes, code_dtype, n, group, 0, scales, nullptr, nullptr, out, as_stream(stream));
}

extern "C" int lq_double_quantize(const void* scales, int dtype, int64_t n, int64_t dq_group,
                                  void* q_scales, void* dq_scales, void* stream) {
  LQ_REQUIRE(n >= 0 && dq_group >= 1, LQ_EINVAL, "bad size");
  if (n == 0) return LQ_OK;
  LQ_REQUIRE(scales && q_scales && dq_scales, LQ_EINVAL, "NULL pointer");
  LQ_DISPATCH_FLOAT(dtype, dq_t, scales, n, dq_group, q_scales, dq_scales, as_stream(stream));
}

extern "C" int lq_double_dequantize(const void* q_scales, const void* dq_scales, int dtype,
                                    int64_t n, int64_t dq_group, void* out, void* stream) {
  LQ_REQUIRE(n >= 0 && dq_group >= 1, LQ_EINVAL, "bad size");
  if (n == 0) return LQ_OK;
  LQ_REQUIRE(q_scales && dq_scales && out, LQ_EINVAL, "NULL pointer");
  LQ_DISPATCH_FLOAT(dtype, ddq_t, q_scales, dq_scales, n, dq_group, out, as_stream(stream));
}

extern "C" int lq_nf4_pack(const void* x, int x_dtype, int64_t n, int64_t group, int64_t dq_group,
                           uint8_t* packed_codes, void* scales, void* q_scales, void* dq_scales,
                           void* stream) {
  LQ_REQUIRE(n >= 0 && group >= 1 && dq_group >= 0, LQ_EINVAL, "bad size");
  if (n == 0) return LQ_OK;
  LQ_REQUIRE(x && packed_codes && scales, LQ_EINVAL, "NULL pointer");
  LQ_REQUIRE(dq_group == 0 || (q_scales && dq_scales), LQ_EINVAL, "double quantization needs q_scales/dq_scales");
  LQ_DISPATCH_FLOAT(x_dtype, nf4_quant_t, x, n, group, dq_group, packed_codes, LQ_U4X2, scales, q_scales, dq_scales, as_stream(stream));
}

extern "C" int lq_nf4_unpack(const uint8_t* packed_codes, int64_t n, int64_t group, int64_t dq_group,
                             const void* scales, const void* q_scales, const void* dq_scales,
                             int s_dtype, void* out, void* stream) {
  LQ_REQUIRE(n >= 0 && group >= 1, LQ_EINVAL, "bad size");
  if (n == 0) return LQ_OK;
  LQ_REQUIRE(packed_codes && out && (scales || q_scales), LQ_EINVAL, "NULL pointer");
  LQ_REQUIRE(!q_scales || (dq_scales && dq_group > 0), LQ_EINVAL, "double dequantization needs dq_scales and dq_group");
  LQ_DISPATCH_FLOAT(s_dtype, nf4_dequant_t, packed_codes, LQ_U4X2, n, group, dq_group, scales, q_scales, dq_scales, out, as_stream(stream));
}

extern "C" int lq_codes_convert(const void* src, int src_dtype, int64_t n, void* dst, int dst_dtype,
                                void* stream) {
  LQ_REQUIRE(n >= 0, LQ_EINVAL, "bad size");
  auto ok = [](int d) { return d == LQ_I64 || d == LQ_U8 || d == LQ_U4X2; };
  LQ_REQUIRE(ok(src_dtype) && ok(dst_dtype), LQ_EDTYPE, "code containers are I64, U8 or U4X2");
  if (n == 0) return LQ_OK;
  LQ_REQUIRE(src && dst, LQ_EINVAL, "NULL pointer");
  codes_convert_kernel<<<grid_cap(((n + 1) / 2 + 255) / 256, 16), 256, 0, as_stream(stream)>>>(src, src_dtype, n, dst, dst_dtype);
  return launched("codes_convert_kernel");
}

// ---------------------------------------------------------------------------
// QLoRALinear.merge_lora (qlora.py:314-317) in one pass:
//   out[n, k] = W_base[n, k] + scaling * (lora_B @ lora_A)[n, k]
// W_base is _dequantize_base's weight, bit for bit (NF4 table value rounded
// to the scales' dtype S times the block's scale, restored through double
// dequantization when q_scales is given); each torch op's rounding is kept:
// t = sum_j B[n, j] A[j, k] (fp32 accumulation, rounded to the LoRA dtype P),
// t = round_P(scaling * t), out = round_O(W + t) with O = promote(S, P).  The
// rank-r product is the only arithmetic that differs from the reference's
// (its summation order is BLAS's).
// Tile of a block: 32 rows x 128 columns; thread = 2 rows x 8 columns, the
// tile's lora_A columns (r x 128) and lora_B rows (32 x r) in shared memory
// as fp32.  HBM-bound: 0.5 byte of codes in, sizeof(O) out per element.
// ---------------------------------------------------------------------------
namespace lq {
namespace {

constexpr int kMrRows = 32, kMrCols = 128, kMrMaxRank = 64;

template <typename S, typename P, typename O>
__global__ void __launch_bounds__(256) nf4_merge_lora_kernel(
    const uint8_t* __restrict__ codes, const S* __restrict__ scales, const S* __restrict__ q_scales,
    const S* __restrict__ dq_scales, int64_t group, int64_t dq_group, const P* __restrict__ lora_a,
    const P* __restrict__ lora_b, int r, float scaling, int N, int K, O* __restrict__ out) {
  __shared__ float sa[kMrMaxRank][kMrCols];   // lora_A[j, k0 + c]
  __shared__ float sb[kMrRows][kMrMaxRank];   // lora_B[n0 + i, j]
  __shared__ float tab[16];
  const int n0 = blockIdx.y * kMrRows, k0 = blockIdx.x * kMrCols;
  if (threadIdx.x < 16) tab[threadIdx.x] = Ty<S>::round(kNF4[threadIdx.x]);
  for (int i = threadIdx.x; i < r * kMrCols; i += blockDim.x) {
    const int j = i / kMrCols, c = i % kMrCols;
    sa[j][c] = (k0 + c < K) ? Ty<P>::to_f(lora_a[(int64_t)j * K + k0 + c]) : 0.0f;
  }
  for (int i = threadIdx.x; i < kMrRows * r; i += blockDim.x) {
    const int rr = i / r, j = i % r;
    sb[rr][j] = (n0 + rr < N) ? Ty<P>::to_f(lora_b[(int64_t)(n0 + rr) * r + j]) : 0.0f;
  }
  __syncthreads();
  const int cl = (threadIdx.x & 15) * 8;  // first of the thread's 8 columns in the tile
  const int rl = (threadIdx.x >> 4) * 2;  // first of its 2 rows
  if (k0 + cl >= K) return;
  float acc[2][8];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[i][c] = 0.0f;
  for (int j = 0; j < r; ++j) {
    float av[8], bv[2];
#pragma unroll
    for (int c = 0; c < 8; ++c) av[c] = sa[j][cl + c];
#pragma unroll
    for (int i = 0; i < 2; ++i) bv[i] = sb[rl + i][j];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int c = 0; c < 8; ++c) acc[i][c] = fmaf(bv[i], av[c], acc[i][c]);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int n = n0 + rl + i;
    if (n >= N) break;
    const int64_t e0 = (int64_t)n * K + k0 + cl;  // 8 consecutive flat elements (K % 8 == 0)
    const uint32_t cw = *reinterpret_cast<const uint32_t*>(codes + e0 / 2);
    int64_t glast = -1;
    float s = 0.0f;
    float o[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int64_t g = (e0 + c) / group;
      if (g != glast) {
        glast = g;
        s = q_scales ? tmul<S>(tdiv<S>(Ty<S>::to_f(q_scales[g]), 127.0f), Ty<S>::to_f(dq_scales[g / dq_group]))
                     : Ty<S>::to_f(scales[g]);
      }
      const float w = tmul<S>(tab[(cw >> (4 * c)) & 15], s);
      const float t = tmul<P>(scaling, Ty<P>::round(acc[i][c]));
      o[c] = tadd<O>(w, t);
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) out[e0 + c] = Ty<O>::from_f(o[c]);
  }
}

template <typename S, typename P>
int merge_lora_sp(const uint8_t* codes, const void* s, const void* qs, const void* dqs, int64_t group,
                  int64_t dq_group, const void* la, const void* lb, int r, float scaling, int N, int K,
                  void* out, int out_dtype, cudaStream_t st) {
  dim3 grid((unsigned)((K + kMrCols - 1) / kMrCols), (unsigned)((N + kMrRows - 1) / kMrRows));
  const S* sp = static_cast<const S*>(s);
  const S* qp = static_cast<const S*>(qs);
  const S* dp = static_cast<const S*>(dqs);
  const P* ap = static_cast<const P*>(la);
  const P* bp = static_cast<const P*>(lb);
  // O = promote(S, P): float32 if either is, else S (== P)
  if (out_dtype == LQ_F32)
    nf4_merge_lora_kernel<S, P, float><<<grid, 256, 0, st>>>(codes, sp, qp, dp, group, dq_group, ap, bp, r, scaling, N, K, static_cast<float*>(out));
  else
    nf4_merge_lora_kernel<S, P, S><<<grid, 256, 0, st>>>(codes, sp, qp, dp, group, dq_group, ap, bp, r, scaling, N, K, static_cast<S*>(out));
  return launched("nf4_merge_lora_kernel");
}

template <typename S>
int merge_lora_s(int p_dtype, const uint8_t* codes, const void* s, const void* qs, const void* dqs,
                 int64_t group, int64_t dq_group, const void* la, const void* lb, int r, float scaling,
                 int N, int K, void* out, int out_dtype, cudaStream_t st) {
  switch (p_dtype) {
    case LQ_F32: return merge_lora_sp<S, float>(codes, s, qs, dqs, group, dq_group, la, lb, r, scaling, N, K, out, out_dtype, st);
    case LQ_F16: return merge_lora_sp<S, __half>(codes, s, qs, dqs, group, dq_group, la, lb, r, scaling, N, K, out, out_dtype, st);
    case LQ_BF16: return merge_lora_sp<S, __nv_bfloat16>(codes, s, qs, dqs, group, dq_group, la, lb, r, scaling, N, K, out, out_dtype, st);
    default: set_error("unsupported LoRA dtype %d", p_dtype); return LQ_EDTYPE;
  }
}

}  // namespace
}  // namespace lq

extern "C" int lq_nf4_merge_lora(const uint8_t* packed_codes, int64_t N, int64_t K, int64_t group,
                                 int64_t dq_group, const void* scales, const void* q_scales,
                                 const void* dq_scales, int s_dtype, const void* lora_a,
                                 const void* lora_b, int p_dtype, int64_t rank, float scaling,
                                 void* out, int out_dtype, void* stream) {
  using namespace lq;
  LQ_REQUIRE(N >= 0 && K >= 0 && group >= 1, LQ_EINVAL, "bad size");
  if (N == 0 || K == 0) return LQ_OK;
  LQ_REQUIRE(K % 8 == 0, LQ_EINVAL, "merge_lora needs in_features %% 8 == 0 (got %lld)", (long long)K);
  LQ_REQUIRE(N < (1LL << 31) && K < (1LL << 31), LQ_ERANGE, "shape too large");
  LQ_REQUIRE(rank >= 1 && rank <= kMrMaxRank, LQ_ERANGE, "LoRA rank %lld outside [1, %d]", (long long)rank, kMrMaxRank);
  LQ_REQUIRE(packed_codes && out && lora_a && lora_b && (scales || q_scales), LQ_EINVAL, "NULL pointer");
  LQ_REQUIRE(!q_scales || (dq_scales && dq_group > 0), LQ_EINVAL, "double dequantization needs dq_scales and dq_group");
  LQ_REQUIRE(reinterpret_cast<uintptr_t>(packed_codes) % 4 == 0, LQ_EALIGN, "codes must be 4-byte aligned");
  const bool f32 = s_dtype == LQ_F32 || p_dtype == LQ_F32;
  LQ_REQUIRE(f32 ? out_dtype == LQ_F32 : (s_dtype == p_dtype && out_dtype == s_dtype), LQ_EDTYPE,
             "merge_lora output dtype must be the promotion of the scales' and LoRA dtypes");
  cudaStream_t st = as_stream(stream);
  const uint8_t* c = packed_codes;
  switch (s_dtype) {
    case LQ_F32: return merge_lora_s<float>(p_dtype, c, scales, q_scales, dq_scales, group, dq_group, lora_a, lora_b, (int)rank, scaling, (int)N, (int)K, out, out_dtype, st);
    case LQ_F16: return merge_lora_s<__half>(p_dtype, c, scales, q_scales, dq_scales, group, dq_group, lora_a, lora_b, (int)rank, scaling, (int)N, (int)K, out, out_dtype, st);
    case LQ_BF16: return merge_lora_s<__nv_bfloat16>(p_dtype, c, scales, q_scales, dq_scales, group, dq_group, lora_a, lora_b, (int)rank, scaling, (int)N, (int)K, out, out_dtype, st);
    default: set_error("unsupported scale dtype %d", s_dtype); return LQ_EDTYPE;
  }
}
