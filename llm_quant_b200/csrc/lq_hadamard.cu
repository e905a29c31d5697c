// lq_hadamard.cu -- Walsh-Hadamard transform along the last dim, optionally
// fused with per-row fake quantization.
//
// The reference computes x @ hadamard_matrix(d, x.dtype) as a dense d x d
// matmul (core/rotation.py:130-147), O(d^2) per row.  Here it is the
// O(d log d) butterfly of the same Sylvester matrix: for h = 1, 2, 4, ...
// every index pair (i, i + h) with bit h clear becomes (a + b, a - b), then
// the result is scaled by the matrix entry round_T(1 / sqrt(d))
// (core/rotation.py:30-43), once, and rounded to T.
//
// Row mapping: a team of NT = d / E threads owns one row, thread t holding
// elements [t*E, t*E + E) (contiguous 16/32-byte vector loads).  Stages
// h < E run in registers, stages E <= h < 32E through warp shuffles, and the
// remaining log2(NT/32) stages after one shared-memory transpose in which
// every thread takes the NT/32 elements that differ only in the warp bits.
#include "lq_common.cuh"

namespace lq {
namespace {

struct FhtArgs {
  int64_t rows;
  int d, E, log2d;
  float entry;  // round_T(1 / sqrt(d))
  // fused quantization
  float qmin, qmax, lo;
  int sym;
  int al32;  // x is 32-byte aligned: rows are read with whole-sector loads
};

template <typename T, int E>
__device__ __forceinline__ void load_row_chunk(const T* __restrict__ src, float* v, bool vec) {
  if (vec) {
    constexpr int V = 16 / sizeof(T);
#pragma unroll
    for (int k = 0; k < E / V; ++k) {
      Vec16<T> u;
      u.u = ld_nc_v4(src + k * V);
#pragma unroll
      for (int i = 0; i < V; ++i) v[k * V + i] = Ty<T>::to_f(u.v[i]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < E; ++i) v[i] = Ty<T>::to_f(src[i]);
  }
}

template <typename T, int E>
__device__ __forceinline__ void store_row_chunk(T* __restrict__ dst, const float* v, bool vec) {
  if (vec) {
    constexpr int V = 16 / sizeof(T);
#pragma unroll
    for (int k = 0; k < E / V; ++k) {
      Vec16<T> u;
#pragma unroll
      for (int i = 0; i < V; ++i) u.v[i] = Ty<T>::from_f(v[k * V + i]);
      st_v4(dst + k * V, u.u);
    }
  } else {
#pragma unroll
    for (int i = 0; i < E; ++i) dst[i] = Ty<T>::from_f(v[i]);
  }
}

template <int E>
__device__ __forceinline__ void butterfly_regs(float* v) {
#pragma unroll
  for (int h = 1; h < E; h <<= 1) {
#pragma unroll
    for (int i = 0; i < E; ++i) {
      if ((i & h) == 0) {
        float a = v[i], b = v[i + h];
        v[i] = __fadd_rn(a, b);
        v[i + h] = __fsub_rn(a, b);
      }
    }
  }
}

// Shuffle stages over lane bits [0, log2(tps)): the lower lane of a pair
// keeps a + b, the upper one a - b, both as one exact fma(v, +-1, partner).
template <int E>
__device__ __forceinline__ void butterfly_lanes(float* v, int tps, int lane_in_team) {
  for (int m = 1; m < tps; m <<= 1) {
    const float sgn = (lane_in_team & m) ? -1.0f : 1.0f;
#pragma unroll
    for (int i = 0; i < E; ++i) {
      const float p = __shfl_xor_sync(0xffffffffu, v[i], m);
      v[i] = fmaf(v[i], sgn, p);
    }
  }
}

template <typename T, int E, bool QUANT>
__device__ __forceinline__ void finish_and_quant(float* v, const FhtArgs& a, MinMax& r) {
  // y = round_T(acc * entry)
#pragma unroll
  for (int i = 0; i < E; ++i) v[i] = Ty<T>::round(__fmul_rn(v[i], a.entry));
  if constexpr (QUANT) {
    r.init();
#pragma unroll
    for (int i = 0; i < E; ++i) {
      if (a.sym) r.add_max(fabsf(v[i]));
      else r.add(v[i]);
    }
  }
}

// fake_quantize of T-rounded values with the row's scale / zero point.  For
// bf16, round_T(v / scale) is computed as round_T(v * rcp_rn(scale)): a
// quotient of two 8-bit significands is either exact or at least 2^-17
// (relative) away from every bf16 rounding midpoint, while v * rcp is within
// 2^-23 of it, so both round to the same bf16 value when the product is a
// normal number (otherwise the IEEE division is used).
template <typename T, int E>
__device__ __forceinline__ void fake_quant_vals(float* v, const FhtArgs& a, float scale, float zp) {
  constexpr bool kBf16 = Ty<T>::code == LQ_BF16;
  const float rcp = __frcp_rn(scale);
  const bool rcp_ok = kBf16 && scale >= 0x1p-126f && scale <= 0x1p126f;
#pragma unroll
  for (int i = 0; i < E; ++i) {
    float qv;
    if (kBf16) {
      const float pr = __fmul_rn(v[i], rcp);
      qv = (rcp_ok && (fabsf(pr) >= 0x1p-126f || pr == 0.0f)) ? Ty<T>::round(pr) : tdiv<T>(v[i], scale);
    } else {
      qv = tdiv<T>(v[i], scale);
    }
    // symmetric: zp is +0.0 and both zero-point ops are exact no-ops here
    const float t = a.sym ? qv : tadd<T>(qv, zp);
    const float q = tclamp_t<T>(tste(t), a.qmin, a.qmax);
    v[i] = tmul<T>(a.sym ? q : tsub<T>(q, zp), scale);
  }
}

// Teams of tps = d/E <= 32 lanes; several rows per warp.
template <typename T, int E, bool QUANT>
__global__ void __launch_bounds__(256) fht_warp_kernel(const T* __restrict__ x, FhtArgs a,
                                                       T* __restrict__ out,
                                                       T* __restrict__ scale_out,
                                                       T* __restrict__ zp_out, int vec) {
  pdl_wait();  // launched as a programmatic dependent: the previous kernel is done
  pdl_trigger();
  const int tps = a.d / E;
  const int lane = threadIdx.x & 31;
  const int t = lane & (tps - 1);
  const int64_t team = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / tps;
  const int64_t nteams = ((int64_t)gridDim.x * blockDim.x) / tps;
  const int64_t team0 = team - lane / tps;
  for (int64_t r0 = team0; r0 < a.rows; r0 += nteams) {
    const int64_t row = r0 + lane / tps;
    const bool live = row < a.rows;
    float v[E];
    if (live) load_row_chunk<T, E>(x + row * a.d + (int64_t)t * E, v, vec);
    else {
#pragma unroll
      for (int i = 0; i < E; ++i) v[i] = 0.0f;
    }
    butterfly_regs<E>(v);
    butterfly_lanes<E>(v, tps, t);
    MinMax r;
    finish_and_quant<T, E, QUANT>(v, a, r);
    if constexpr (QUANT) {
      for (int m = 1; m < tps; m <<= 1) r.shfl_xor_merge(m, a.sym);
      float scale, zp;
      qparams_from<T>(r, a.sym, a.qmin, a.qmax, a.lo, scale, zp);
      if (live && t == 0 && scale_out) {
        scale_out[row] = Ty<T>::from_f(scale);
        zp_out[row] = Ty<T>::from_f(zp);
      }
      fake_quant_vals<T, E>(v, a, scale, zp);
    }
    if (live) store_row_chunk<T, E>(out + row * a.d + (int64_t)t * E, v, vec);
  }
}

// One block of NT = 32*W threads (d = NT*E, W <= E) per row.
template <typename T, int E, int W, bool QUANT>
__global__ void __launch_bounds__(1024) fht_block_kernel(const T* __restrict__ x, FhtArgs a,
                                                         T* __restrict__ out,
                                                         T* __restrict__ scale_out,
                                                         T* __restrict__ zp_out, int vec) {
  pdl_wait();  // launched as a programmatic dependent: the previous kernel is done
  pdl_trigger();
  extern __shared__ float sm[];  // [d]
  __shared__ MinMax red[32];
  const int t = threadIdx.x, lane = t & 31;
  constexpr int span = 32 * E;  // elements covered by one warp
  constexpr int cpt = E / W;    // (lane, reg) combos per thread in phase 2
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    float v[E];
    load_row_chunk<T, E>(x + row * a.d + (int64_t)t * E, v, vec);
    butterfly_regs<E>(v);
    butterfly_lanes<E>(v, 32, lane);
    __syncthreads();  // previous row's readers are done with sm
#pragma unroll
    for (int i = 0; i < E; ++i) sm[t * E + i] = v[i];
    __syncthreads();
    // phase 2: thread owns combos c = t*cpt + m (c in [0, span)), each with W
    // elements at c + w*span; butterfly over w in registers (reusing v).
    float* u = v;
#pragma unroll
    for (int m = 0; m < cpt; ++m) {
      const int c = t * cpt + m;
#pragma unroll
      for (int w = 0; w < W; ++w) u[m * W + w] = sm[c + w * span];
    }
#pragma unroll
    for (int h = 1; h < W; h <<= 1) {
#pragma unroll
      for (int m = 0; m < cpt; ++m) {
#pragma unroll
        for (int w = 0; w < W; ++w) {
          if ((w & h) == 0) {
            float p = u[m * W + w], q = u[m * W + w + h];
            u[m * W + w] = __fadd_rn(p, q);
            u[m * W + w + h] = __fsub_rn(p, q);
          }
        }
      }
    }
    MinMax r;
    finish_and_quant<T, E, QUANT>(u, a, r);
    __syncthreads();
#pragma unroll
    for (int m = 0; m < cpt; ++m) {
      const int c = t * cpt + m;
#pragma unroll
      for (int w = 0; w < W; ++w) sm[c + w * span] = u[m * W + w];
    }
    float scale = 0.f, zp = 0.f;
    if constexpr (QUANT) {
      for (int mm = 16; mm >= 1; mm >>= 1) r.shfl_xor_merge(mm, a.sym);
      if (lane == 0) red[t >> 5] = r;
    }
    __syncthreads();
    if constexpr (QUANT) {
      MinMax tot = red[0];
      for (int i = 1; i < W; ++i) tot.merge(red[i]);
      qparams_from<T>(tot, a.sym, a.qmin, a.qmax, a.lo, scale, zp);
      if (t == 0 && scale_out) {
        scale_out[row] = Ty<T>::from_f(scale);
        zp_out[row] = Ty<T>::from_f(zp);
      }
    }
#pragma unroll
    for (int i = 0; i < E; ++i) v[i] = sm[t * E + i];
    if constexpr (QUANT) fake_quant_vals<T, E>(v, a, scale, zp);
    store_row_chunk<T, E>(out + row * a.d + (int64_t)t * E, v, vec);
  }
}

// ---------------------------------------------------------------------------
// d = 2^L, L in {11, 12, 13}: one block of NT = d/32 threads per row, 32
// elements per thread held as 16 float2 (elements 2j, 2j+1 = "pair" j), in
// three register phases joined by two shared-memory transposes:
//   phase 1  thread t holds pairs 16t..16t+15 (elements 32t..32t+31, read
//            from global memory): stage of element bit 0 inside each float2,
//            then pair bits 0..3;
//   phase 2  thread t holds pairs (t % 16) + 16k + 256(t / 16), k = 0..15:
//            pair bits 4..7;
//   phase 3  thread t holds pairs f + NF t + 256 k3 (NF = 2^(13-L) "filler"
//            values f, k3 over the remaining pair bits 8..L-2): those bits,
//            then the row is finished in registers and stored, NF pairs
//            (2 NF contiguous elements) per store.
// Stages run in the order of the element bits (0, 1, ..., L-1) like the
// other kernels; between float2 registers they are packed f32x2 operations
// (a + b, and a - b as the exact fma(b, -1, a)).  Shared-memory layout: pair
// j at float2 slot j + j/16 (one pad slot per 16), which keeps the 16 lanes
// of every 64-bit access of all three phases on distinct banks.
//
// Fused fake quantization, bf16: the row's values y = round_bf16(acc *
// entry) are kept as bf16x2 words.  When the scale lies in [2^-126, 2^126]
// and every |t| (quotient plus zero point) is below 63, each pair is
//   t = round_bf16(y * rcp_rn(scale)) (+ zp),  q = (t + 192) - 192,
//   q = clamp(q, qmin, qmax) (- zp),  out = round_bf16(q * scale)
// in bf16x2 arithmetic: t + 192 lands in [128, 256) where the bf16 spacing
// is 1, so the pair of adds is round-half-even to an integer with a zero
// result of +0, which is what ste_round gives for finite t; the sums,
// differences and products of these small integers and bf16 values are exact
// before their one rounding.  Other rows, and fp16 / fp32, use the scalar
// fake_quant_vals.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void bfly2(float2& a, float2& b) {
  const float2 s = __fadd2_rn(a, b);
  b = __ffma2_rn(b, make_float2(-1.0f, -1.0f), a);
  a = s;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ __nv_bfloat162 as_bf2(uint32_t u) { return *reinterpret_cast<__nv_bfloat162*>(&u); }
__device__ __forceinline__ uint32_t as_u32(__nv_bfloat162 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Store NW 32-bit words (NW in {1, 2, 4}) at dst (aligned to 4 NW bytes).
template <int NW>
__device__ __forceinline__ void store_words(void* dst, const uint32_t* w) {
  if constexpr (NW == 1) *reinterpret_cast<uint32_t*>(dst) = w[0];
  else if constexpr (NW == 2) *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
  else st_v4(dst, make_uint4(w[0], w[1], w[2], w[3]));
}

// Store NF consecutive float2 (2 NF elements, rounded to T) at dst.
template <typename T, int NF>
__device__ __forceinline__ void store_pairs(T* dst, const float2* v) {
  if constexpr (sizeof(T) == 4) {
    if constexpr (NF == 1) {
      *reinterpret_cast<float2*>(dst) = v[0];
    } else {
#pragma unroll
      for (int f = 0; f < NF; f += 2)
        st_v4(dst + 2 * f, make_uint4(__float_as_uint(v[f].x), __float_as_uint(v[f].y),
                                      __float_as_uint(v[f + 1].x), __float_as_uint(v[f + 1].y)));
    }
  } else {
    uint32_t w[NF];
#pragma unroll
    for (int f = 0; f < NF; ++f)
      w[f] = Ty<T>::code == LQ_BF16 ? pack_bf16x2(v[f].x, v[f].y) : pack_f16x2(v[f].x, v[f].y);
    store_words<NF>(dst, w);
  }
}

template <typename T, int L, bool QUANT>
__global__ void __launch_bounds__((1 << L) / 32) fht3_kernel(const T* __restrict__ x, FhtArgs a,
                                                            T* __restrict__ out,
                                                            T* __restrict__ scale_out,
                                                            T* __restrict__ zp_out) {
  pdl_wait();  // launched as a programmatic dependent: the previous kernel is done
  pdl_trigger();
  constexpr int D = 1 << L, NT = D / 32, C3 = L - 9, NF = 1 << (4 - C3), NK3 = 1 << C3;
  constexpr bool kBf16 = Ty<T>::code == LQ_BF16;
  __shared__ float2 sm[(D / 2) + (D / 32)];
  __shared__ MinMax red[NT / 32];
  const int t = threadIdx.x, lane = t & 31;
  const int base2 = (t & 15) + 272 * (t >> 4);
  const int base3 = NF * t + ((NF * t) >> 4);
  constexpr int V = 16 / sizeof(T);
  // this thread's 32 input elements of the current row; the next row's are
  // loaded as soon as these are in registers, so the load overlaps the row
  uint4 raw[32 / V];
  // a thread's 32 elements are 64 (bf16) or 128 (fp32) contiguous bytes:
  // 32-byte loads take whole sectors (16-byte loads at a 64-byte lane stride
  // would fetch every sector twice)
  auto load_row = [&](int64_t r) {
    const T* src = x + r * D + (int64_t)t * 32;
    if (a.al32) {
#pragma unroll
      for (int k = 0; k < 32 / V; k += 2) ld_nc_v8(src + k * V, raw[k], raw[k + 1]);
    } else {
#pragma unroll
      for (int k = 0; k < 32 / V; ++k) raw[k] = ld_nc_v4(src + k * V);
    }
  };
  if (blockIdx.x < a.rows) load_row(blockIdx.x);
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    float2 v[16];
    {  // phase 1
#pragma unroll
      for (int k = 0; k < 32 / V; ++k) {
        Vec16<T> u;
        u.u = raw[k];
#pragma unroll
        for (int i = 0; i < V; i += 2)
          v[(k * V + i) / 2] = make_float2(Ty<T>::to_f(u.v[i]), Ty<T>::to_f(u.v[i + 1]));
      }
      const int64_t nrow = row + gridDim.x;
      if (nrow < a.rows) load_row(nrow);
    }
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      const float p = v[m].x, q = v[m].y;
      v[m] = make_float2(__fadd_rn(p, q), __fsub_rn(p, q));
    }
#pragma unroll
    for (int h = 1; h < 16; h <<= 1)
#pragma unroll
      for (int m = 0; m < 16; ++m)
        if ((m & h) == 0) bfly2(v[m], v[m + h]);
    __syncthreads();  // the previous row's phase-3 reads are done
#pragma unroll
    for (int m = 0; m < 16; ++m) sm[17 * t + m] = v[m];
    __syncthreads();
    // phase 2
#pragma unroll
    for (int k = 0; k < 16; ++k) v[k] = sm[base2 + 17 * k];
#pragma unroll
    for (int h = 1; h < 16; h <<= 1)
#pragma unroll
      for (int k = 0; k < 16; ++k)
        if ((k & h) == 0) bfly2(v[k], v[k + h]);
#pragma unroll
    for (int k = 0; k < 16; ++k) sm[base2 + 17 * k] = v[k];
    __syncthreads();
    // phase 3: register r = f + NF * k3
#pragma unroll
    for (int k3 = 0; k3 < NK3; ++k3)
#pragma unroll
      for (int f = 0; f < NF; ++f) v[f + NF * k3] = sm[base3 + f + 272 * k3];
#pragma unroll
    for (int h = NF; h < 16; h <<= 1)
#pragma unroll
      for (int r = 0; r < 16; ++r)
        if ((r & h) == 0) bfly2(v[r], v[r + h]);
    // finish: y = round_T(acc * entry)
    const float2 e2 = make_float2(a.entry, a.entry);
#pragma unroll
    for (int r = 0; r < 16; ++r) v[r] = __fmul2_rn(v[r], e2);
    T* dst = out + row * D + 2 * NF * (int64_t)t;
    if constexpr (!QUANT) {
#pragma unroll
      for (int k3 = 0; k3 < NK3; ++k3) store_pairs<T, NF>(dst + 512 * k3, v + NF * k3);
    } else if constexpr (kBf16) {
      uint32_t y[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) y[r] = pack_bf16x2(v[r].x, v[r].y);
      MinMax mm;
      mm.init();
      if (a.sym) {
        uint32_t m2 = 0;
#pragma unroll
        for (int r = 0; r < 16; r += 2) m2 = __vimax3_u16x2(m2, y[r] & 0x7FFF7FFFu, y[r + 1] & 0x7FFF7FFFu);
        mm.mx = __uint_as_float(max(m2 & 0xFFFFu, m2 >> 16) << 16);
      } else {
        __nv_bfloat162 lo2 = as_bf2(y[0]), hi2 = lo2;
#pragma unroll
        for (int r = 1; r < 16; ++r) {
          lo2 = __hmin2_nan(lo2, as_bf2(y[r]));
          hi2 = __hmax2_nan(hi2, as_bf2(y[r]));
        }
        mm.mn = fmin_nan(__low2float(lo2), __high2float(lo2));
        mm.mx = fmax_nan(__low2float(hi2), __high2float(hi2));
      }
      for (int s = 16; s >= 1; s >>= 1) mm.shfl_xor_merge(s, a.sym);
      if (lane == 0) red[t >> 5] = mm;
      __syncthreads();
      MinMax tot = red[0];
#pragma unroll
      for (int i = 1; i < NT / 32; ++i) tot.merge(red[i]);
      float scale, zp;
      qparams_from<T>(tot, a.sym, a.qmin, a.qmax, a.lo, scale, zp);
      if (t == 0 && scale_out) {
        scale_out[row] = Ty<T>::from_f(scale);
        zp_out[row] = Ty<T>::from_f(zp);
      }
      const float rcp = __frcp_rn(scale);
      const float bound = a.sym ? tot.mx * rcp : fmaxf(fabsf(tot.mn), fabsf(tot.mx)) * rcp + fabsf(zp);
      const bool fast = scale >= 0x1p-126f && scale <= 0x1p126f && bound < 63.0f;
      uint32_t o[16];
      if (fast) {
        const float2 r2 = make_float2(rcp, rcp);
        const __nv_bfloat162 magic = __float2bfloat162_rn(192.0f);
        const __nv_bfloat162 qlo = __float2bfloat162_rn(a.qmin), qhi = __float2bfloat162_rn(a.qmax);
        const __nv_bfloat162 z2 = __float2bfloat162_rn(zp), s2 = __float2bfloat162_rn(scale);
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          const float2 p = __fmul2_rn(make_float2(__uint_as_float(y[r] << 16), __uint_as_float(y[r] & 0xFFFF0000u)), r2);
          __nv_bfloat162 q = as_bf2(pack_bf16x2(p.x, p.y));
          if (!a.sym) q = __hadd2(q, z2);
          q = __hsub2(__hadd2(q, magic), magic);
          q = __hmin2(__hmax2(q, qlo), qhi);
          if (!a.sym) q = __hsub2(q, z2);
          o[r] = as_u32(__hmul2(q, s2));
        }
      } else {
        float f[32];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          f[2 * r] = __uint_as_float(y[r] << 16);
          f[2 * r + 1] = __uint_as_float(y[r] & 0xFFFF0000u);
        }
        fake_quant_vals<T, 32>(f, a, scale, zp);
#pragma unroll
        for (int r = 0; r < 16; ++r) o[r] = pack_bf16x2(f[2 * r], f[2 * r + 1]);
      }
#pragma unroll
      for (int k3 = 0; k3 < NK3; ++k3) store_words<NF>(dst + 512 * k3, o + NF * k3);
    } else {
      float* f = reinterpret_cast<float*>(v);
#pragma unroll
      for (int i = 0; i < 32; ++i) f[i] = Ty<T>::round(f[i]);
      MinMax mm;
      mm.init();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (a.sym) mm.add_max(fabsf(f[i]));
        else mm.add(f[i]);
      }
      for (int s = 16; s >= 1; s >>= 1) mm.shfl_xor_merge(s, a.sym);
      if (lane == 0) red[t >> 5] = mm;
      __syncthreads();
      MinMax tot = red[0];
#pragma unroll
      for (int i = 1; i < NT / 32; ++i) tot.merge(red[i]);
      float scale, zp;
      qparams_from<T>(tot, a.sym, a.qmin, a.qmax, a.lo, scale, zp);
      if (t == 0 && scale_out) {
        scale_out[row] = Ty<T>::from_f(scale);
        zp_out[row] = Ty<T>::from_f(zp);
      }
      fake_quant_vals<T, 32>(f, a, scale, zp);
#pragma unroll
      for (int k3 = 0; k3 < NK3; ++k3) store_pairs<T, NF>(dst + 512 * k3, v + NF * k3);
    }
  }
}

template <typename T> float entry_of(int d) {
  float c = 1.0f / (float)sqrt((double)d);
  if (Ty<T>::code == LQ_BF16) return __bfloat162float(__float2bfloat16_rn(c));
  if (Ty<T>::code == LQ_F16) return __half2float(__float2half_rn(c));
  return c;
}

template <typename T, bool QUANT>
int fht_launch(const T* x, FhtArgs a, T* out, T* s, T* z, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  const int d = a.d;
  auto vec_for = [&](int E) {
    return (E % V == 0) && aligned16(x) && aligned16(out) && ((int64_t)d * sizeof(T)) % 16 == 0;
  };
  int E_warp = d <= 32 * V ? V : (d <= 32 * 16 ? 16 : 32);
  if (d <= 32 * E_warp) {
    int E = d < E_warp ? d : E_warp;
    int tps = d / E;
    int64_t threads_needed = a.rows * tps;
    int grid = (int)((threads_needed + 255) / 256);
    int cap = num_sms() * 16;
    grid = grid < 1 ? 1 : (grid > cap ? cap : grid);
    int vec = vec_for(E);
    switch (E) {
      case 1: launch_pdl(fht_warp_kernel<T, 1, QUANT>, dim3((unsigned)(grid)), dim3((unsigned)(256)), 0, st, x, a, out, s, z, 0); break;
      case 2: launch_pdl(fht_warp_kernel<T, 2, QUANT>, dim3((unsigned)(grid)), dim3((unsigned)(256)), 0, st, x, a, out, s, z, 0); break;
      case 4: launch_pdl(fht_warp_kernel<T, 4, QUANT>, dim3((unsigned)(grid)), dim3((unsigned)(256)), 0, st, x, a, out, s, z, vec); break;
      case 8: launch_pdl(fht_warp_kernel<T, 8, QUANT>, dim3((unsigned)(grid)), dim3((unsigned)(256)), 0, st, x, a, out, s, z, vec); break;
      case 16: launch_pdl(fht_warp_kernel<T, 16, QUANT>, dim3((unsigned)(grid)), dim3((unsigned)(256)), 0, st, x, a, out, s, z, vec); break;
      case 32: launch_pdl(fht_warp_kernel<T, 32, QUANT>, dim3((unsigned)(grid)), dim3((unsigned)(256)), 0, st, x, a, out, s, z, vec); break;
      default: set_error("internal: bad E %d", E); return LQ_EINVAL;
    }
    return launched("fht_warp_kernel");
  }
  if ((d == 2048 || d == 4096 || d == 8192) && aligned16(x) && aligned16(out)) {
    void (*k3)(const T*, FhtArgs, T*, T*, T*) =
        d == 2048 ? fht3_kernel<T, 11, QUANT> : (d == 4096 ? fht3_kernel<T, 12, QUANT> : fht3_kernel<T, 13, QUANT>);
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k3, d / 32, 0);
    LQ_REQUIRE(e == cudaSuccess && per_sm > 0, LQ_ECUDA, "occupancy query: %s", cudaGetErrorString(e));
    const int64_t cap = (int64_t)num_sms() * per_sm;
    const int grid = (int)(a.rows < cap ? a.rows : cap);
    FhtArgs a3 = a;
    a3.al32 = (reinterpret_cast<uintptr_t>(x) & 31) == 0;
    launch_pdl(k3, dim3((unsigned)(grid)), dim3((unsigned)(d / 32)), 0, st, x, a3, out, s, z);
    return launched("fht3_kernel");
  }
  int E = (d <= 8192) ? 16 : 32;
  int NT = d / E;
  LQ_REQUIRE(NT <= 1024 && NT / 32 <= E, LQ_ERANGE, "hadamard d=%d too large", d);
  size_t smem = (size_t)d * sizeof(float);
  int grid = (int)(a.rows < (int64_t)num_sms() * 4 ? a.rows : (int64_t)num_sms() * 4);
  int vec = vec_for(E);
  void (*k)(const T*, FhtArgs, T*, T*, T*, int) = nullptr;
  const int W = NT / 32;
  if (E == 16 && W == 4) k = fht_block_kernel<T, 16, 4, QUANT>;
  else if (E == 16 && W == 8) k = fht_block_kernel<T, 16, 8, QUANT>;
  else if (E == 16 && W == 16) k = fht_block_kernel<T, 16, 16, QUANT>;
  else if (E == 32 && W == 16) k = fht_block_kernel<T, 32, 16, QUANT>;
  else if (E == 32 && W == 32) k = fht_block_kernel<T, 32, 32, QUANT>;
  LQ_REQUIRE(k != nullptr, LQ_EINVAL, "internal: no block shape for d=%d", d);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    LQ_REQUIRE(e == cudaSuccess, LQ_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  }
  launch_pdl(k, dim3((unsigned)(grid)), dim3((unsigned)(NT)), smem, st, x, a, out, s, z, vec);
  return launched("fht_block_kernel");
}

template <typename T, bool QUANT>
int fht_t(const void* x, int64_t rows, int64_t d, int n_bits, int sym, void* out, void* s,
          void* z, cudaStream_t st) {
  FhtArgs a;
  a.rows = rows;
  a.d = (int)d;
  a.E = 0;
  a.al32 = 0;
  a.log2d = 0;
  while ((1 << a.log2d) < d) ++a.log2d;
  a.entry = entry_of<T>((int)d);
  a.qmin = (float)qmin_of(n_bits, sym);
  a.qmax = (float)qmax_of(n_bits, sym);
  a.lo = lo_clamp_value<T>();
  a.sym = sym;
  return fht_launch<T, QUANT>(static_cast<const T*>(x), a, static_cast<T*>(out),
                              static_cast<T*>(s), static_cast<T*>(z), st);
}

}  // namespace
}  // namespace lq

using namespace lq;

static int check_fht(int64_t rows, int64_t d) {
  LQ_REQUIRE(rows >= 0, LQ_EINVAL, "bad rows");
  LQ_REQUIRE(d >= 1 && (d & (d - 1)) == 0, LQ_EINVAL, "last dim must be power of 2 (got %lld)", (long long)d);
  LQ_REQUIRE(d <= 32768, LQ_ERANGE, "d=%lld above 32768", (long long)d);
  return LQ_OK;
}

extern "C" int lq_hadamard(const void* x, int dtype, int64_t rows, int64_t d, void* out,
                           void* stream) {
  int rc = check_fht(rows, d);
  if (rc) return rc;
  if (rows == 0) return LQ_OK;
  LQ_REQUIRE(x && out, LQ_EINVAL, "NULL pointer");
  cudaStream_t st = as_stream(stream);
  switch (dtype) {
    case LQ_F32: return fht_t<float, false>(x, rows, d, 8, 1, out, nullptr, nullptr, st);
    case LQ_F16: return fht_t<__half, false>(x, rows, d, 8, 1, out, nullptr, nullptr, st);
    case LQ_BF16: return fht_t<__nv_bfloat16, false>(x, rows, d, 8, 1, out, nullptr, nullptr, st);
    default: set_error("unsupported dtype %d", dtype); return LQ_EDTYPE;
  }
}

extern "C" int lq_hadamard_fake_quant(const void* x, int dtype, int64_t rows, int64_t d,
                                      int n_bits, int symmetric, void* out, void* scale,
                                      void* zero_point, void* stream) {
  int rc = check_fht(rows, d);
  if (rc) return rc;
  LQ_REQUIRE(n_bits >= 1 && n_bits <= 16, LQ_EINVAL, "n_bits out of range");
  LQ_REQUIRE((scale == nullptr) == (zero_point == nullptr), LQ_EINVAL, "scale and zero_point must both be given");
  if (rows == 0) return LQ_OK;
  LQ_REQUIRE(x && out, LQ_EINVAL, "NULL pointer");
  cudaStream_t st = as_stream(stream);
  switch (dtype) {
    case LQ_F32: return fht_t<float, true>(x, rows, d, n_bits, symmetric, out, scale, zero_point, st);
    case LQ_F16: return fht_t<__half, true>(x, rows, d, n_bits, symmetric, out, scale, zero_point, st);
    case LQ_BF16: return fht_t<__nv_bfloat16, true>(x, rows, d, n_bits, symmetric, out, scale, zero_point, st);
    default: set_error("unsupported dtype %d", dtype); return LQ_EDTYPE;
  }
}
