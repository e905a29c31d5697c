// lq_group.cu -- group / row quantization (min/max or absmax per group,
// scale + zero point, round-half-even, clamp, fake-quant or integer codes).
//
// Layout: x is [rows, cols] row-major; every row is cut into groups of G
// columns, the last one zero-padded (core/quantizer.py:89-95).  One "team" of
// threads owns one group at a time and keeps it in registers, so x is read
// from HBM exactly once and the output written once:
//   * warp teams (1..32 lanes) for groups up to 32 x NVT x 16 bytes,
//   * block teams (up to 1024 threads) for longer groups (per-token rows),
//   * a streaming block path (two passes, the second from L2) beyond that.
// The vector path moves 16 bytes per load/store (ld.global.nc.v4); it needs
// G*sizeof(T) % 16 == 0, cols % G == 0 and 16-byte aligned pointers.
#include <type_traits>

#include "lq_common.cuh"

namespace lq {
namespace {

enum { MODE_QPARAMS = 0, MODE_FAKE = 1, MODE_CODES = 2 };

template <typename OutT, typename T> struct Store;
template <typename T> struct Store<int8_t, T> {
  __device__ __forceinline__ static int8_t cv(float v) { return (int8_t)tcast_i32(v); }
};
template <typename T> struct Store<int16_t, T> {
  __device__ __forceinline__ static int16_t cv(float v) { return (int16_t)tcast_i32(v); }
};
template <typename T> struct Store<T, T> {
  __device__ __forceinline__ static T cv(float v) { return Ty<T>::from_f(v); }
};

// Store V consecutive outputs (V * sizeof(OutT) bytes, naturally aligned).
template <typename OutT, typename T, int V>
__device__ __forceinline__ void store_vec(OutT* p, const float* vals) {
  constexpr int BYTES = V * sizeof(OutT);
  union {
    OutT o[V];
    uint32_t w[(BYTES + 3) / 4];
    uint16_t h;
    uint8_t b;
  } u;
#pragma unroll
  for (int i = 0; i < V; ++i) u.o[i] = Store<OutT, T>::cv(vals[i]);
  if constexpr (BYTES == 16) {
    st_v4(p, make_uint4(u.w[0], u.w[1], u.w[2], u.w[3]));
  } else if constexpr (BYTES == 8) {
    *reinterpret_cast<uint2*>(p) = make_uint2(u.w[0], u.w[1]);
  } else if constexpr (BYTES == 4) {
    *reinterpret_cast<uint32_t*>(p) = u.w[0];
  } else if constexpr (BYTES == 2) {
    *reinterpret_cast<uint16_t*>(p) = u.h;
  } else {
    *reinterpret_cast<uint8_t*>(p) = u.b;
  }
}

struct GroupArgs {
  int64_t rows, cols, G, groups_per_row, total_groups;
  float qmin, qmax, lo;
  int sym;
  // Output row remapping (KV append into a cache with spare capacity):
  // input row r = (p, t) with t = r % rpp lands on output row
  // p * opitch + ooff + t, and its scales on row p * spitch + soff + t.
  int64_t rpp, opitch, ooff, spitch, soff;
  __device__ __forceinline__ int64_t out_row(int64_t r) const {
    return (r / rpp) * opitch + ooff + r % rpp;
  }
  __device__ __forceinline__ int64_t sc_index(int64_t g) const {
    const int64_t r = g / groups_per_row;
    return ((r / rpp) * spitch + soff + r % rpp) * groups_per_row + g % groups_per_row;
  }
};

// Per-element output of the fused modes.  A zero point of +0.0 (symmetric
// quantization) is skipped: t + 0 only turns a -0.0 into +0.0, which ste_round
// and the code casts treat alike, and q - 0 is exact for integer q.
// The quotient stage of apply_q, t = round_T(x / scale) (+ zp), without an
// IEEE division per element where that provably gives the same result, from
// the group's reciprocal rcp = rcp_rn(scale):
//   bf16: round_bf16(x * rcp) == round_bf16(fl32(x / scale)) whenever the
//         product is a normal fp32 number (both operands have 8-bit
//         significands: their quotient is exactly representable or at least
//         2^-17 away from every bf16 rounding midpoint, x * rcp is within
//         2^-23 of it); zero, subnormal and non-finite products divide.
//   fp32, when only rint(t + zp) reaches the outputs (integer codes, and fake
//         quantization through ste_round, whose zero is +0.0 either way; not
//         float codes, which keep the sign of a zero): t0 = x * rcp is within 2^-22 |t0| of fl32(x / scale),
//         so t0 + zp is within 2^-22 |t0| + 2^-23 |t| of the reference's
//         t; when it lies more than 2^-20 (|t0| + |t|) from every
//         half-integer, both round to the same integer and t0 + zp stands in
//         for t.  The window tested is wg = tie_window(...) >= 2^-20 (|t0| +
//         |t|) for every element of the group.  Otherwise (ties, values near
//         a tie, non-finite) it divides.
//   fp16: divides.
template <typename T, bool RINT_ONLY>
__device__ __forceinline__ float quotient_zp(float v, float scale, float rcp, float zp, bool zp0, float wg) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    const float p = __fmul_rn(v, rcp);
    float t = (fabsf(p) >= 1.17549435e-38f || v == 0.0f) ? Ty<T>::round(p) : tdiv<T>(v, scale);
    return zp0 ? t : tadd<T>(t, zp);
  } else if constexpr (std::is_same<T, float>::value && RINT_ONLY) {
    const float t0 = __fmul_rn(v, rcp);
    const float t = zp0 ? t0 : __fadd_rn(t0, zp);
    if (__fsub_rn(0.5f, fabsf(__fsub_rn(t, rintf(t)))) > wg) return t;
    const float e = tdiv<T>(v, scale);
    return zp0 ? e : tadd<T>(e, zp);
  } else {
    const float t = tdiv<T>(v, scale);
    return zp0 ? t : tadd<T>(t, zp);
  }
}

// A bound, over a group, of the window 2^-20 (|t0| + |t|) that quotient_zp
// tests against: |t0| = fl(|x| |rcp|) <= fl(amax |rcp|) and |t| <=
// fl(|t0| + |zp|), and rounding is monotone, so every element's own window is
// at most this.  NaN when the group holds a NaN or an infinity (amax or rcp
// gives NaN): then every element divides.
__device__ __forceinline__ float tie_window(const MinMax& r, bool sym, float rcp, float zp) {
  const float amax = sym ? r.mx : fmax_nan(fabsf(r.mn), fabsf(r.mx));
  const float a = __fmul_rn(amax, fabsf(rcp));
  const float t = __fadd_rn(a, fabsf(zp));
  return __fmul_rn(__fadd_rn(a, t), 9.5367431640625e-07f);  // 2^-20
}

template <typename T, int MODE, bool RINT_ONLY>
__device__ __forceinline__ float apply_q(float v, float scale, float rcp, float zp, float qmin,
                                         float qmax, bool zp0, float wg) {
  const float t = quotient_zp<T, RINT_ONLY>(v, scale, rcp, zp, zp0, wg);
  if constexpr (MODE == MODE_FAKE) {
    float q = tclamp_t<T>(tste(t), qmin, qmax);
    return tmul<T>(zp0 ? q : tsub<T>(q, zp), scale);
  } else {
    return tclamp_t<T>(trint(t), qmin, qmax);
  }
}

// Outputs that depend on the quotient only through its rint: fake
// quantization and integer codes.
template <int MODE, typename OutT, typename T>
__host__ __device__ constexpr bool rint_only() {
  return MODE == MODE_FAKE || !std::is_same<OutT, T>::value;
}

// The symmetric skip is exact for fake quantization and integer codes; a
// float code output keeps the +0.0 add (it can turn a -0.0 code into +0.0).
template <int MODE, typename OutT, typename T>
__device__ __forceinline__ bool zp0_ok(const GroupArgs& a) {
  return a.sym && (MODE == MODE_FAKE || !std::is_same<OutT, T>::value);
}

// ---------------------------------------------------------------------------
// Register-resident group processing shared by warp teams and block teams.
// Slot k of thread t holds elements e = (k*TPS + t)*V + i (VEC) or
// e = k*TPS + t (scalar, V == 1).
// ---------------------------------------------------------------------------
template <typename T, int NVT, bool VEC>
struct Tile {
  static constexpr int V = VEC ? (16 / sizeof(T)) : 1;
  float v[NVT * V];
  unsigned inb;  // bit k: slot k belongs to the group (e < G)

  __device__ __forceinline__ void load(const T* __restrict__ x, int64_t row, int64_t gcol0,
                                       const GroupArgs& a, int t, int tps) {
    inb = 0;
    const T* base = x + row * a.cols + gcol0;
#pragma unroll
    for (int k = 0; k < NVT; ++k) {
      int64_t e = (int64_t)(k * tps + t) * V;
      bool in = e < a.G;
      inb |= (in ? 1u : 0u) << k;
      if constexpr (VEC) {
        Vec16<T> u;
        if (in) u.u = ld_nc_v4(base + e);
        else u.u = make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int i = 0; i < V; ++i) v[k * V + i] = Ty<T>::to_f(u.v[i]);
      } else {
        // columns past `cols` are the zero padding of the last group
        bool valid = in && (gcol0 + e < a.cols);
        v[k] = valid ? Ty<T>::to_f(base[e]) : 0.0f;
      }
    }
  }

  __device__ __forceinline__ void reduce_local(MinMax& r, bool sym) const {
    r.init();
#pragma unroll
    for (int k = 0; k < NVT; ++k) {
      if (inb & (1u << k)) {
#pragma unroll
        for (int i = 0; i < V; ++i) {
          if (sym) r.add_max(fabsf(v[k * V + i]));
          else r.add(v[k * V + i]);
        }
      }
    }
  }

  template <int MODE, typename OutT>
  __device__ __forceinline__ void emit(OutT* __restrict__ out, int64_t row, int64_t gcol0,
                                       const GroupArgs& a, int t, int tps, float scale,
                                       float zp, const MinMax& r) {
    OutT* base = out + a.out_row(row) * a.cols + gcol0;
    const float rcp = __frcp_rn(scale);
    const float wg = tie_window(r, a.sym, rcp, zp);
    constexpr bool kFast = std::is_same<T, float>::value && rint_only<MODE, OutT, T>();
    const bool zp0 = zp0_ok<MODE, OutT, T>(a);
    auto put = [&](int k, const float* o) {
      const int64_t e = (int64_t)(k * tps + t) * V;
      if constexpr (VEC) {
        store_vec<OutT, T, V>(base + e, o);
      } else {
        if (gcol0 + e < a.cols) base[e] = Store<OutT, T>::cv(o[0]);
      }
    };
    bool slow = !kFast;
    if constexpr (kFast) {
      // fp32 codes / fake quantization from the product quotient.  Where
      // t = x rcp (+ zp) is finite and more than wg from a half-integer (the
      // test of quotient_zp), r = rint(t) is the nearest integer and r - t is
      // exact (Sterbenz for |t| >= 0.5, -t below), so ste_round(t) =
      // t + (r - t) = r with a zero made +0.0 (r + 0.0), and clamp on a finite
      // value is min / max.  A thread with any other element rewrites its
      // outputs through apply_q below (ties, values within wg of one,
      // non-finite groups).  (Testing rint(x rcp) and clamping it to
      // [qmin - zp, qmax - zp] instead saves two adds per element but
      // measured 3 % slower.)
#pragma unroll
      for (int k = 0; k < NVT; ++k) {
        if (!(inb & (1u << k))) continue;
        float o[V];
#pragma unroll
        for (int i = 0; i < V; ++i) {
          const float t0 = __fmul_rn(v[k * V + i], rcp);
          const float tq = zp0 ? t0 : __fadd_rn(t0, zp);
          const float rq = rintf(tq);
          slow |= !(__fsub_rn(0.5f, fabsf(__fsub_rn(tq, rq))) > wg);
          if constexpr (MODE == MODE_FAKE) {
            const float q = fminf(fmaxf(__fadd_rn(rq, 0.0f), a.qmin), a.qmax);
            o[i] = __fmul_rn(zp0 ? q : __fsub_rn(q, zp), scale);
          } else {
            o[i] = fminf(fmaxf(rq, a.qmin), a.qmax);
          }
        }
        put(k, o);
      }
    }
    if (slow) {
#pragma unroll
      for (int k = 0; k < NVT; ++k) {
        if (!(inb & (1u << k))) continue;
        float o[V];
#pragma unroll
        for (int i = 0; i < V; ++i)
          o[i] = apply_q<T, MODE, rint_only<MODE, OutT, T>()>(v[k * V + i], scale, rcp, zp, a.qmin, a.qmax, zp0, wg);
        put(k, o);
      }
    }
  }
};

// Warp teams: `tps` lanes (power of two <= 32) per group.
template <typename T, int MODE, typename OutT, int NVT, bool VEC>
__global__ void __launch_bounds__(256) group_warp_kernel(const T* __restrict__ x, GroupArgs a,
                                                         int tps, OutT* __restrict__ out,
                                                         T* __restrict__ scale_out,
                                                         T* __restrict__ zp_out) {
  const int lane = threadIdx.x & 31;
  const int t = lane & (tps - 1);
  const int64_t team = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) / tps;
  const int64_t nteams = ((int64_t)gridDim.x * blockDim.x) / tps;
  // all lanes of a warp iterate the same number of times (shuffles below)
  const int64_t warp_team0 = team - (lane / tps);
  // the team's next group is loaded before the current one is reduced and
  // written, so its loads are in flight meanwhile
  auto fetch = [&](Tile<T, NVT, VEC>& tl, int64_t g) {
    if (g < a.total_groups) tl.load(x, g / a.groups_per_row, (g % a.groups_per_row) * a.G, a, t, tps);
    else tl.inb = 0;
  };
  Tile<T, NVT, VEC> tile;
  fetch(tile, warp_team0 + lane / tps);
  for (int64_t g0 = warp_team0; g0 < a.total_groups; g0 += nteams) {
    const int64_t g = g0 + lane / tps;
    const bool live = g < a.total_groups;
    Tile<T, NVT, VEC> next;
    fetch(next, g + nteams);
    MinMax r;
    tile.reduce_local(r, a.sym);
    for (int m = 1; m < tps; m <<= 1) r.shfl_xor_merge(m, a.sym);
    if (live) {
      const int64_t row = g / a.groups_per_row;
      const int64_t gcol0 = (g % a.groups_per_row) * a.G;
      float scale, zp;
      qparams_from<T>(r, a.sym, a.qmin, a.qmax, a.lo, scale, zp);
      if (t == 0 && scale_out) {
        const int64_t si = a.sc_index(g);
        scale_out[si] = Ty<T>::from_f(scale);
        zp_out[si] = Ty<T>::from_f(zp);
      }
      if constexpr (MODE != MODE_QPARAMS) tile.template emit<MODE>(out, row, gcol0, a, t, tps, scale, zp, r);
    }
    tile = next;
  }
}

// Block-wide NaN-aware min/max reduction; result broadcast to all threads.
__device__ __forceinline__ MinMax block_reduce(MinMax r, MinMax* sm, bool sym) {
  for (int m = 16; m >= 1; m >>= 1) r.shfl_xor_merge(m, sym);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();  // sm may still be read from the previous group
  if ((threadIdx.x & 31) == 0) sm[w] = r;
  __syncthreads();
  MinMax t = sm[0];
  for (int i = 1; i < nw; ++i) t.merge(sm[i]);
  return t;
}

// Block teams: one block (blockDim.x threads) per group.
template <typename T, int MODE, typename OutT, int NVT, bool VEC>
__global__ void __launch_bounds__(1024) group_block_kernel(const T* __restrict__ x, GroupArgs a,
                                                           OutT* __restrict__ out,
                                                           T* __restrict__ scale_out,
                                                           T* __restrict__ zp_out) {
  __shared__ MinMax sm[32];
  const int t = threadIdx.x, tps = blockDim.x;
  for (int64_t g = blockIdx.x; g < a.total_groups; g += gridDim.x) {
    const int64_t row = g / a.groups_per_row;
    const int64_t gcol0 = (g % a.groups_per_row) * a.G;
    Tile<T, NVT, VEC> tile;
    tile.load(x, row, gcol0, a, t, tps);
    MinMax r;
    tile.reduce_local(r, a.sym);
    r = block_reduce(r, sm, a.sym);
    float scale, zp;
    qparams_from<T>(r, a.sym, a.qmin, a.qmax, a.lo, scale, zp);
    if (t == 0 && scale_out) {
      const int64_t si = a.sc_index(g);
      scale_out[si] = Ty<T>::from_f(scale);
      zp_out[si] = Ty<T>::from_f(zp);
    }
    if constexpr (MODE != MODE_QPARAMS) tile.template emit<MODE>(out, row, gcol0, a, t, tps, scale, zp, r);
  }
}

// Streaming block path for groups too long for registers: pass 1 reduces,
// pass 2 re-reads (from L2) and writes.  Scalar, coalesced.
template <typename T, int MODE, typename OutT>
__global__ void __launch_bounds__(1024) group_stream_kernel(const T* __restrict__ x, GroupArgs a,
                                                            OutT* __restrict__ out,
                                                            T* __restrict__ scale_out,
                                                            T* __restrict__ zp_out) {
  __shared__ MinMax sm[32];
  for (int64_t g = blockIdx.x; g < a.total_groups; g += gridDim.x) {
    const int64_t row = g / a.groups_per_row;
    const int64_t gcol0 = (g % a.groups_per_row) * a.G;
    const T* base = x + row * a.cols + gcol0;
    MinMax r;
    r.init();
    for (int64_t e = threadIdx.x; e < a.G; e += blockDim.x) {
      float v = (gcol0 + e < a.cols) ? Ty<T>::to_f(base[e]) : 0.0f;
      if (a.sym) r.add_max(fabsf(v));
      else r.add(v);
    }
    r = block_reduce(r, sm, a.sym);
    float scale, zp;
    qparams_from<T>(r, a.sym, a.qmin, a.qmax, a.lo, scale, zp);
    if (threadIdx.x == 0 && scale_out) {
      const int64_t si = a.sc_index(g);
      scale_out[si] = Ty<T>::from_f(scale);
      zp_out[si] = Ty<T>::from_f(zp);
    }
    if constexpr (MODE != MODE_QPARAMS) {
      OutT* ob = out + a.out_row(row) * a.cols + gcol0;
      const float rcp = __frcp_rn(scale);
      const float wg = tie_window(r, a.sym, rcp, zp);
      for (int64_t e = threadIdx.x; e < a.G && gcol0 + e < a.cols; e += blockDim.x)
        ob[e] = Store<OutT, T>::cv(apply_q<T, MODE, rint_only<MODE, OutT, T>()>(Ty<T>::to_f(base[e]), scale, rcp, zp, a.qmin, a.qmax, zp0_ok<MODE, OutT, T>(a), wg));
    }
  }
}

int grid_for(int64_t units, int per_block) {
  int64_t want = (units + per_block - 1) / per_block;
  int64_t cap = (int64_t)num_sms() * 16;
  return (int)(want < cap ? (want > 0 ? want : 1) : cap);
}

template <typename T, int MODE, typename OutT, int NVT, bool VEC>
int launch_warp(const T* x, const GroupArgs& a, int tps, OutT* out, T* s, T* z, cudaStream_t st) {
  const int threads = 256;
  const int grid = resident_grid(group_warp_kernel<T, MODE, OutT, NVT, VEC>, threads, 0,
                                 (a.total_groups * tps + threads - 1) / threads);
  group_warp_kernel<T, MODE, OutT, NVT, VEC><<<grid, threads, 0, st>>>(x, a, tps, out, s, z);
  return launched("group_warp_kernel");
}

template <typename T, int MODE, typename OutT, int NVT, bool VEC>
int launch_block(const T* x, const GroupArgs& a, int threads, OutT* out, T* s, T* z,
                 cudaStream_t st) {
  int grid = grid_for(a.total_groups, 1);
  group_block_kernel<T, MODE, OutT, NVT, VEC><<<grid, threads, 0, st>>>(x, a, out, s, z);
  return launched("group_block_kernel");
}

// Pick a team shape for a group of G elements and launch.
template <typename T, int MODE, typename OutT>
int dispatch(const T* x, const GroupArgs& a, OutT* out, T* s, T* z, bool vec_ok,
             cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  const int64_t G = a.G;
  if (vec_ok) {
    const int64_t nv = G / V;  // vectors per group
    // up to 8 vectors (128 bytes) in flight per lane, teams of <= 32 lanes
    int nvt = 1;
    while (nvt < 8 && nvt * 2 <= nv) nvt *= 2;
    int64_t need = (nv + nvt - 1) / nvt;
    if (need > 32) {
      nvt = 8;
      need = (nv + 7) / 8;
    }
    if (need <= 32) {
      int tps = 1;
      while (tps < need) tps <<= 1;
      switch (nvt) {
        case 1: return launch_warp<T, MODE, OutT, 1, true>(x, a, tps, out, s, z, st);
        case 2: return launch_warp<T, MODE, OutT, 2, true>(x, a, tps, out, s, z, st);
        case 4: return launch_warp<T, MODE, OutT, 4, true>(x, a, tps, out, s, z, st);
        default: return launch_warp<T, MODE, OutT, 8, true>(x, a, tps, out, s, z, st);
      }
    }
    // block teams: up to 1024 threads x 2 vectors in registers
    for (int threads = 128; threads <= 1024; threads *= 2) {
      if (nv <= (int64_t)threads * 2) {
        if (nv <= threads) return launch_block<T, MODE, OutT, 1, true>(x, a, threads, out, s, z, st);
        return launch_block<T, MODE, OutT, 2, true>(x, a, threads, out, s, z, st);
      }
    }
  } else {
    if (G <= 32) {
      int tps = 1;
      while (tps < G) tps <<= 1;
      return launch_warp<T, MODE, OutT, 1, false>(x, a, tps, out, s, z, st);
    }
    if (G <= 128) return launch_warp<T, MODE, OutT, 4, false>(x, a, 32, out, s, z, st);
    if (G <= 512) return launch_warp<T, MODE, OutT, 16, false>(x, a, 32, out, s, z, st);
    if (G <= 8192) return launch_block<T, MODE, OutT, 8, false>(x, a, 1024, out, s, z, st);
  }
  int grid = grid_for(a.total_groups, 1);
  group_stream_kernel<T, MODE, OutT><<<grid, 1024, 0, st>>>(x, a, out, s, z);
  return launched("group_stream_kernel");
}

template <typename T>
int group_quant_t(const void* xv, int64_t rows, int64_t cols, int64_t G, int n_bits, int sym,
                  int mode, void* out, int out_dtype, void* scale, void* zp, cudaStream_t st,
                  int64_t rpp, int64_t opitch, int64_t ooff, int64_t spitch, int64_t soff) {
  const T* x = static_cast<const T*>(xv);
  GroupArgs a;
  a.rpp = rpp;
  a.opitch = opitch;
  a.ooff = ooff;
  a.spitch = spitch;
  a.soff = soff;
  a.rows = rows;
  a.cols = cols;
  a.G = G;
  a.groups_per_row = (cols + G - 1) / G;
  a.total_groups = rows * a.groups_per_row;
  a.qmin = (float)qmin_of(n_bits, sym);
  a.qmax = (float)qmax_of(n_bits, sym);
  a.lo = lo_clamp_value<T>();
  a.sym = sym;
  constexpr int V = 16 / sizeof(T);
  int osz = mode == MODE_QPARAMS ? 1 : dtype_size(out_dtype);
  bool vec_ok = (G % V == 0) && (cols % G == 0) && aligned16(x) &&
                (mode == MODE_QPARAMS || (reinterpret_cast<uintptr_t>(out) % (V * osz) == 0));
  T* s = static_cast<T*>(scale);
  T* z = static_cast<T*>(zp);
  if (mode == MODE_QPARAMS) return dispatch<T, MODE_QPARAMS, T>(x, a, nullptr, s, z, vec_ok, st);
  if (mode == MODE_FAKE) {
    LQ_REQUIRE(out_dtype == Ty<T>::code, LQ_EDTYPE, "fake-quant output dtype must equal input dtype");
    return dispatch<T, MODE_FAKE, T>(x, a, static_cast<T*>(out), s, z, vec_ok, st);
  }
  if (out_dtype == LQ_I8) return dispatch<T, MODE_CODES, int8_t>(x, a, static_cast<int8_t*>(out), s, z, vec_ok, st);
  if (out_dtype == LQ_I16) return dispatch<T, MODE_CODES, int16_t>(x, a, static_cast<int16_t*>(out), s, z, vec_ok, st);
  if (out_dtype == Ty<T>::code) return dispatch<T, MODE_CODES, T>(x, a, static_cast<T*>(out), s, z, vec_ok, st);
  set_error("unsupported code dtype %d", out_dtype);
  return LQ_EDTYPE;
}

}  // namespace

// Shared with lq_kv.cu (KV append into capacity storage).
int group_quant_remap(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t group,
                      int n_bits, int symmetric, int mode, void* out, int out_dtype, void* scale,
                      void* zero_point, void* stream, int64_t rpp, int64_t opitch, int64_t ooff,
                      int64_t spitch, int64_t soff) {
  cudaStream_t st = as_stream(stream);
  switch (x_dtype) {
    case LQ_F32: return group_quant_t<float>(x, rows, cols, group, n_bits, symmetric, mode, out, out_dtype, scale, zero_point, st, rpp, opitch, ooff, spitch, soff);
    case LQ_F16: return group_quant_t<__half>(x, rows, cols, group, n_bits, symmetric, mode, out, out_dtype, scale, zero_point, st, rpp, opitch, ooff, spitch, soff);
    case LQ_BF16: return group_quant_t<__nv_bfloat16>(x, rows, cols, group, n_bits, symmetric, mode, out, out_dtype, scale, zero_point, st, rpp, opitch, ooff, spitch, soff);
    default: set_error("unsupported x dtype %d", x_dtype); return LQ_EDTYPE;
  }
}

}  // namespace lq

extern "C" int lq_group_quant(const void* x, int x_dtype, int64_t rows, int64_t cols,
                              int64_t group, int n_bits, int symmetric, int mode, void* out,
                              int out_dtype, void* scale, void* zero_point, void* stream) {
  using namespace lq;
  LQ_REQUIRE(rows >= 0 && cols >= 0 && group >= 1, LQ_EINVAL, "bad shape rows=%lld cols=%lld group=%lld",
             (long long)rows, (long long)cols, (long long)group);
  LQ_REQUIRE(n_bits >= 1 && n_bits <= 16, LQ_EINVAL, "n_bits %d out of range", n_bits);
  LQ_REQUIRE(mode >= 0 && mode <= 2, LQ_EINVAL, "bad mode %d", mode);
  if (rows == 0 || cols == 0) return LQ_OK;
  LQ_REQUIRE(x, LQ_EINVAL, "x is NULL");
  LQ_REQUIRE(mode == LQ_MODE_QPARAMS || out, LQ_EINVAL, "out is NULL");
  LQ_REQUIRE((scale == nullptr) == (zero_point == nullptr), LQ_EINVAL, "scale and zero_point must both be given");
  LQ_REQUIRE(mode != LQ_MODE_QPARAMS || scale, LQ_EINVAL, "QPARAMS mode needs scale/zero_point");
  return lq::group_quant_remap(x, x_dtype, rows, cols, group, n_bits, symmetric, mode, out,
                               out_dtype, scale, zero_point, stream, rows, rows, 0, rows, 0);
}

// ---------------------------------------------------------------------------
// fake_quantize backward (core/quantizer.py:143-185 under autograd).
// Per group (zero padding included in the reductions, its gradient dropped):
//   y = (clamp(ste(x/s + zp)) - zp) * s,  s = clamp_min(mx - mn, lo) / (qmax - qmin)
//   (symmetric: s = clamp_min(max|x|, lo) / qmax, zp = 0); zp has no gradient
//   (it comes from round).  With m_i the clamp mask and c_i the clamped code:
//   direct_i = (g_i * s) * m_i / s
//   ds       = sum_i g_i * (c_i - zp)  +  sum_i -(g_i * s * m_i) * ((x_i / s) / s)
//   d_rng    = ds / (qmax - qmin) if mx - mn >= lo else 0   (symmetric: / qmax)
//   dx_i     = direct_i + [x_i == mx] d_rng / #max - [x_i == mn] d_rng / #min
//              (symmetric: + sign(x_i) [|x_i| == max|x|] d_rng / #max)
// Each elementwise op rounds to T as torch does; sums accumulate in fp32.
// One block per group, three passes over the group (L2-resident).
// ---------------------------------------------------------------------------
namespace lq {
namespace {

template <typename T>
__global__ void __launch_bounds__(256) fq_backward_kernel(const T* __restrict__ x,
                                                          const T* __restrict__ g, GroupArgs a,
                                                          T* __restrict__ dx) {
  __shared__ MinMax sm[32];
  __shared__ float red[3][32];
  for (int64_t grp = blockIdx.x; grp < a.total_groups; grp += gridDim.x) {
    const int64_t row = grp / a.groups_per_row;
    const int64_t c0 = (grp % a.groups_per_row) * a.G;
    const T* xb = x + row * a.cols + c0;
    const T* gb = g + row * a.cols + c0;
    T* db = dx + row * a.cols + c0;
    const int64_t valid = min(a.G, a.cols - c0);
    // pass 1: min / max (padding zeros included)
    MinMax r;
    r.init();
    for (int64_t e = threadIdx.x; e < a.G; e += blockDim.x) {
      const float v = e < valid ? Ty<T>::to_f(xb[e]) : 0.0f;
      if (a.sym) r.add_max(fabsf(v));
      else r.add(v);
    }
    r = block_reduce(r, sm, a.sym);
    float s, zp;
    qparams_from<T>(r, a.sym, a.qmin, a.qmax, a.lo, s, zp);
    // pass 2: tie counts and the two sums of the scale gradient
    float cmax = 0.f, cmin = 0.f, s1 = 0.f, s2 = 0.f;
    for (int64_t e = threadIdx.x; e < a.G; e += blockDim.x) {
      const bool in = e < valid;
      const float v = in ? Ty<T>::to_f(xb[e]) : 0.0f;
      const float gv = in ? Ty<T>::to_f(gb[e]) : 0.0f;
      if (a.sym) {
        cmax += (fabsf(v) == r.mx) ? 1.f : 0.f;
      } else {
        cmax += (v == r.mx) ? 1.f : 0.f;
        cmin += (v == r.mn) ? 1.f : 0.f;
      }
      const float t = tadd<T>(tdiv<T>(v, s), zp);
      const float q = tste(t);
      const bool m = (q >= Ty<T>::round(a.qmin)) && (q <= Ty<T>::round(a.qmax));
      const float c = tclamp_t<T>(q, a.qmin, a.qmax);
      s1 += tmul<T>(gv, tsub<T>(c, zp));
      const float du = m ? tmul<T>(gv, s) : 0.0f;
      s2 += tmul<T>(-du, tdiv<T>(tdiv<T>(v, s), s));
    }
    float vals[3] = {cmax, cmin, __fadd_rn(s1, s2)};
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      for (int o = 16; o >= 1; o >>= 1) vals[k] += __shfl_xor_sync(0xffffffffu, vals[k], o);
    }
    __syncthreads();
    if ((threadIdx.x & 31) == 0) {
      red[0][threadIdx.x >> 5] = vals[0];
      red[1][threadIdx.x >> 5] = vals[1];
      red[2][threadIdx.x >> 5] = vals[2];
    }
    __syncthreads();
    float tot[3] = {0.f, 0.f, 0.f};
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
      tot[0] += red[0][w];
      tot[1] += red[1][w];
      tot[2] += red[2][w];
    }
    const float ds = Ty<T>::round(tot[2]);
    float drng;
    if (a.sym) {
      const bool pass = r.mx >= a.lo;  // clamp_min backward mask
      drng = pass ? tdiv<T>(ds, a.qmax) : 0.0f;
    } else {
      const bool pass = tsub<T>(r.mx, r.mn) >= a.lo;
      drng = pass ? tdiv<T>(ds, a.qmax - a.qmin) : 0.0f;
    }
    const float dmax = tdiv<T>(drng, tot[0]);
    const float dmin = a.sym ? 0.0f : tdiv<T>(-drng, tot[1]);
    // pass 3: the gradient of every real (non-padding) element
    for (int64_t e = threadIdx.x; e < valid; e += blockDim.x) {
      const float v = Ty<T>::to_f(xb[e]);
      const float gv = Ty<T>::to_f(gb[e]);
      const float t = tadd<T>(tdiv<T>(v, s), zp);
      const float q = tste(t);
      const bool m = (q >= Ty<T>::round(a.qmin)) && (q <= Ty<T>::round(a.qmax));
      float d = m ? tdiv<T>(tmul<T>(gv, s), s) : 0.0f;
      if (a.sym) {
        if (fabsf(v) == r.mx) d = tadd<T>(d, tmul<T>(dmax, v > 0.f ? 1.f : (v < 0.f ? -1.f : 0.f)));
      } else {
        if (v == r.mx) d = tadd<T>(d, dmax);
        if (v == r.mn) d = tadd<T>(d, dmin);
      }
      db[e] = Ty<T>::from_f(d);
    }
    __syncthreads();
  }
}

template <typename T>
int fq_backward_t(const void* x, const void* g, int64_t rows, int64_t cols, int64_t G, int n_bits,
                  int sym, void* dx, cudaStream_t st) {
  GroupArgs a;
  a.rows = rows;
  a.cols = cols;
  a.G = G;
  a.groups_per_row = (cols + G - 1) / G;
  a.total_groups = rows * a.groups_per_row;
  a.qmin = (float)qmin_of(n_bits, sym);
  a.qmax = (float)qmax_of(n_bits, sym);
  a.lo = lo_clamp_value<T>();
  a.sym = sym;
  a.rpp = a.opitch = a.spitch = rows;
  a.ooff = a.soff = 0;
  int64_t want = a.total_groups;
  int grid = (int)(want < (int64_t)num_sms() * 16 ? want : (int64_t)num_sms() * 16);
  fq_backward_kernel<T><<<grid, 256, 0, st>>>(static_cast<const T*>(x), static_cast<const T*>(g),
                                              a, static_cast<T*>(dx));
  return launched("fq_backward_kernel");
}

}  // namespace
}  // namespace lq

extern "C" int lq_fake_quant_backward(const void* x, const void* grad_out, int dtype, int64_t rows,
                                      int64_t cols, int64_t group, int n_bits, int symmetric,
                                      void* grad_x, void* stream) {
  using namespace lq;
  LQ_REQUIRE(rows >= 0 && cols >= 0 && group >= 1, LQ_EINVAL, "bad shape");
  LQ_REQUIRE(n_bits >= 1 && n_bits <= 16, LQ_EINVAL, "n_bits out of range");
  if (rows == 0 || cols == 0) return LQ_OK;
  LQ_REQUIRE(x && grad_out && grad_x, LQ_EINVAL, "NULL pointer");
  cudaStream_t st = as_stream(stream);
  switch (dtype) {
    case LQ_F32: return fq_backward_t<float>(x, grad_out, rows, cols, group, n_bits, symmetric, grad_x, st);
    case LQ_F16: return fq_backward_t<__half>(x, grad_out, rows, cols, group, n_bits, symmetric, grad_x, st);
    case LQ_BF16: return fq_backward_t<__nv_bfloat16>(x, grad_out, rows, cols, group, n_bits, symmetric, grad_x, st);
    default: set_error("unsupported dtype %d", dtype); return LQ_EDTYPE;
  }
}
