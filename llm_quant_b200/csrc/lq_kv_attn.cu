// lq_kv_attn.cu -- decode attention read straight from the quantized KV cache.
//
// out[b, hq, i, :] = softmax(q[b, hq, i, :] . K^T * sm_scale) V, where K and V
// are the fp32 dequantization (code - zero) * scale of QuantizedKVCache's
// storage (kv_cache_quant.py:221-267).  The reference rebuilds the whole fp32
// K and V on every update (kv_cache_quant.py:379-382) and leaves attention to
// the caller; here the codes are read once and never widened in memory.
//
// Grouped-query layout: q head hq uses kv head hq / (Hq / H).  The G * Sq
// query rows of one kv head ("rows", G = Hq / H) share every K / V tile.
// causal = 1 aligns the queries to the end of the cache: row position i
// (0..Sq-1) sees tokens t <= T - Sq + i.
//
// Work split (flash-decoding): grid = (token splits, B * H, row blocks of
// 8 * NQ rows).  A block's 4 warps take its 16-token tiles round robin; each
// warp streams its tiles (codes, and per-token / per-group scales) with
// 16-byte cp.async into its own ring of shared-memory stages, XOR-swizzled by
// 16-byte chunk so the fragment reads below are free of bank conflicts.
//
// Tensor cores (mma.sync.m16n8k16, f16 in, fp32 accumulate):
//   S = K q'^T : A = 16 tokens x 16 d of codes, converted exactly to the f16
//       integers (code - zero) (magic-exponent trick: 1024 + u is exact for
//       u < 1024); B = 8 query rows of q' (f16).  d is permuted inside each
//       16-wide k block (lane c owns d in [c D/4, (c+1) D/4)), identically
//       for A and B, so a lane's A words are whole 32-bit code words.
//   O += V^T P'^T : A = 16 d x 16 tokens of V codes (code - zero), B = P'
//       (8 query rows), obtained from the S accumulator by movmatrix.trans.
// Scales stay in fp32 outside the MMA where they can: a per-token K scale
// multiplies S, a per-channel V scale multiplies O at the end, a per-group V
// scale multiplies each tile's O contribution.  Where a scale has to enter an
// f16 operand (per-channel / per-group K scale into q', per-token V scale
// into P') the operand is normalised (q' by the row's largest scale; P' by
// folding log2 of the scale into the softmax exponent, so P' <= 1) and split
// into hi + lo f16 halves (two MMAs), which keeps ~22 significant bits.
// Online softmax in the exp2 domain; per-split partials (unnormalised O,
// running max, running sum) are merged by kv_attn_combine_kernel.
#include "lq_common.cuh"

namespace lq {
namespace {

constexpr int kAttnWarps = 4;

// The combine kernel is a programmatic dependent launch (launch_pdl): its
// blocks may be scheduled once every attention block has passed
// pdl_trigger() (after its token loop), and its first statement, pdl_wait(),
// blocks until the attention kernel's partials are complete and visible.  The
// combine's launch and block scheduling overlap the attention kernel's merge
// and tail instead of following them.
constexpr int kTile = 16;  // tokens per tile

struct KvSide {
  const uint8_t* codes;  // [B*H, cap, D] int8 / int16
  const uint8_t* scale;  // per-token [B*H, pitch]; per-channel [B*H, D]; per-group [B*H, pitch, D]
  const uint8_t* zp;     // same layout as scale
  int64_t pitch;         // scale rows per (b, h)
  int gran;              // 0 per-token, 1 per-channel, 2 per-group
  int group;             // tokens per scale row (per-group)
  int off_s, off_z;      // byte offsets of the tile's scale / zero rows inside a stage
  int bytes;             // bytes of one of those rows (0: nothing staged)
};

struct AttnArgs {
  const uint8_t* q;
  int q_dtype, s_dtype, ses;
  int Hq, H, Sq, G, rows;
  int T, cap;
  float sm_log2;  // softmax scale * log2(e)
  int causal, qlo;
  int n_tiles, n_split, tiles_per_split;
  int stage_bytes;
  KvSide k, v;
  uint8_t* out;  // [B, Hq, Sq, D] in q_dtype (n_split == 1)
  float* ws;     // [B*H, n_split, rows, D + 2] partials (n_split > 1)
};

template <int D, int CES>
struct AttnCfg {
  static constexpr int RB = D * CES;        // bytes of one token row of codes
  static constexpr int CPR = RB / 16;       // 16-byte chunks per row
  static constexpr int KB = kTile * RB;     // bytes of a tile of K (or of V)
  static constexpr int STAGES = CES == 1 ? 3 : 2;
  static constexpr int NKB = D / 16;        // k blocks of S = K q'^T; d blocks of O
  static constexpr int LKC = D * CES / 64;  // K chunks a lane reads per row (D/4 codes)
  static constexpr int VB = D * CES / 8;    // V bytes a lane reads per row (D/8 codes)
  static constexpr int QS = D + 16;         // q' row stride (floats) in shared memory
  static constexpr int QC = D / 4 + 4;      // stride of a lane's d range inside a row
};

// 16-byte chunk j of token row r is stored at chunk j ^ swz(r)
template <int CPR>
__device__ __forceinline__ int swz(int r) {
  return CPR >= 8 ? (r & 7) : ((r >> 1) & (CPR - 1));
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ float ld_f(const uint8_t* p, int64_t i, int dt) {
  if (dt == LQ_F32) return reinterpret_cast<const float*>(p)[i];
  if (dt == LQ_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
}
// scale / zero-point load: compile-time dtype STC (LQ_F32 / LQ_F16 / LQ_BF16),
// or the runtime dtype dt when STC < 0
template <int STC>
__device__ __forceinline__ float lds(const uint8_t* p, int64_t i, int dt) {
  if constexpr (STC == LQ_F32) return reinterpret_cast<const float*>(p)[i];
  else if constexpr (STC == LQ_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  else if constexpr (STC == LQ_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  else return ld_f(p, i, dt);
}
__device__ __forceinline__ float ex2(float x) {  // 2^x (PTX ex2.approx; -inf -> 0)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float lg2(float x) {  // log2 x (PTX lg2.approx; 0 -> -inf)
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void st_f(uint8_t* p, int64_t i, int dt, float v) {
  if (dt == LQ_F32) reinterpret_cast<float*>(p)[i] = v;
  else if (dt == LQ_F16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ float2 unpack_h2(uint32_t v) {
  return __half22float2(*reinterpret_cast<__half2*>(&v));
}
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
  __half2 h = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&h);
}
// (lo, hi) -> f16 pair hi and the f16 pair of the remainders
__device__ __forceinline__ void split_h2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  hi = pack_h2(x0, x1);
  const float2 f = unpack_h2(hi);
  lo = pack_h2(x0 - f.x, x1 - f.y);
}
__device__ __forceinline__ void mma_f16(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t trans8x8(uint32_t x) {
  uint32_t r;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}

// f16 pair of the magic-biased codes: int8 bytes (b0, b1) of w at byte
// offset 2*hh -> (1152 + c0, 1152 + c1); int16 word -> (1024 + u0, 1024 + u1)
template <int CES>
struct Codes;
template <>
struct Codes<1> {
  static constexpr float bias = 1152.0f;
  __device__ __forceinline__ static uint32_t pair(uint32_t w, int hh) {  // w already ^ 0x80808080
    return __byte_perm(w, 0x64646464u, hh ? 0x4342 : 0x4140);
  }
};
template <>
struct Codes<2> {
  static constexpr float bias = 1024.0f;
  __device__ __forceinline__ static uint32_t pair(uint32_t w) { return w | 0x64006400u; }
};

__device__ __forceinline__ uint32_t zpair(float za, float zb, float bias) { return pack_h2(bias + za, bias + zb); }

// the 8-row per-token variants are held to 128 registers (4 blocks per SM)
template <int D, int CES, int NQ, bool GEN, bool QLO, int STC>
__global__ void __launch_bounds__(32 * kAttnWarps, (NQ == 1 && !GEN) ? 4 : 1) kv_attn_kernel(AttnArgs a) {
  using C = AttnCfg<D, CES>;
  constexpr int NR = 8 * NQ;     // query rows of the block
  constexpr int NKB = C::NKB;
  extern __shared__ __align__(16) uint8_t sm[];
  float* qs = reinterpret_cast<float*>(sm);  // raw q rows [NR][QS]
  uint8_t* ring = reinterpret_cast<uint8_t*>(qs + NR * C::QS + 8);  // warps' stage rings
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int split = blockIdx.x, bh = blockIdx.y, zb = blockIdx.z;
  const int b = bh / a.H, h = bh % a.H;
  const int tile_lo = split * a.tiles_per_split;
  const int tile_hi = min(a.n_tiles, tile_lo + a.tiles_per_split);
  const int dk0 = c * (D / 4);   // lane's d range in S = K q'^T
  const int dv0 = g * (D / 8);   // lane's d range in O
  const float bias = Codes<CES>::bias;

  // ---- prologue: raw q rows ---------------------------------------------
#pragma unroll
  for (int idx = threadIdx.x; idx < NR * D; idx += 32 * kAttnWarps) {
    const int r = idx / D, d = idx % D, qr = zb * NR + r;
    float v = 0.0f;
    if (qr < a.rows) {
      const int hq = h * a.G + qr / a.Sq, i = qr % a.Sq;
      v = ld_f(a.q, (((int64_t)b * a.Hq + hq) * a.Sq + i) * D + d, a.q_dtype);
    }
    qs[r * C::QS + (d / (D / 4)) * C::QC + d % (D / 4)] = v;
  }
  __syncthreads();

  // per-channel sides: the lane's scales / zero pairs, once
  uint32_t zkp[GEN ? NKB : 1][2];   // K zero pairs of (d0, d0+1), (d0+2, d0+3) of k block j
  uint32_t zvp[GEN ? NKB : 1][2];   // V zero pairs of d = dv0 + 2e (both tokens), d + 1
  float vsd[GEN ? NKB : 1][2];      // V scales of d, d + 1
  float sigma_k = 1.0f;
  auto fill_k_rows = [&](const uint8_t* sp, const uint8_t* zp, int64_t base, bool shared_row) {
    // sp/zp: scale / zero rows of D values (global rows at element base, or a stage row)
    float m = 0.0f;
#pragma unroll
    for (int j = 0; j < (GEN ? NKB : 0); ++j) {
      const int d0 = dk0 + 4 * j;
      float z[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        z[u] = lds<STC>(zp, base + d0 + u, a.s_dtype);
        m = fmaxf(m, fabsf(lds<STC>(sp, base + d0 + u, a.s_dtype)));
      }
      zkp[j][0] = zpair(z[0], z[1], bias);
      zkp[j][1] = zpair(z[2], z[3], bias);
    }
    (void)shared_row;
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    sigma_k = (m > 0.0f && m < INFINITY) ? m : 1.0f;
  };
  auto fill_v_rows = [&](const uint8_t* sp, const uint8_t* zp, int64_t base) {
#pragma unroll
    for (int e = 0; e < (GEN ? NKB : 0); ++e) {
      const int d = dv0 + 2 * e;
      const float z0 = lds<STC>(zp, base + d, a.s_dtype), z1 = lds<STC>(zp, base + d + 1, a.s_dtype);
      zvp[e][0] = zpair(z0, z0, bias);
      zvp[e][1] = zpair(z1, z1, bias);
      vsd[e][0] = lds<STC>(sp, base + d, a.s_dtype);
      vsd[e][1] = lds<STC>(sp, base + d + 1, a.s_dtype);
    }
  };
  if constexpr (GEN) {
    if (a.k.gran == 1) fill_k_rows(a.k.scale, a.k.zp, (int64_t)bh * D, false);
    if (a.v.gran == 1) fill_v_rows(a.v.scale, a.v.zp, (int64_t)bh * D);
  }

  // q' = q (* scale_d / sigma_k for a per-channel / per-group K) as f16 hi / lo
  uint32_t bq[NQ][NKB][2], bql[QLO ? NQ : 1][QLO ? NKB : 1][2];
  auto make_q = [&](const uint8_t* sp, int64_t base, bool scaled) {
    const float inv = 1.0f / sigma_k;
#pragma unroll
    for (int nq = 0; nq < NQ; ++nq) {
      const float* qr = qs + (8 * nq + g) * C::QS + c * C::QC;
#pragma unroll
      for (int j = 0; j < NKB; ++j) {
        const float4 v4 = *reinterpret_cast<const float4*>(qr + 4 * j);
        float x[4] = {v4.x, v4.y, v4.z, v4.w};
        if (GEN && scaled) {
#pragma unroll
          for (int u = 0; u < 4; ++u) x[u] *= lds<STC>(sp, base + dk0 + 4 * j + u, a.s_dtype) * inv;
        }
        if constexpr (QLO) {
          split_h2(x[0], x[1], bq[nq][j][0], bql[nq][j][0]);
          split_h2(x[2], x[3], bq[nq][j][1], bql[nq][j][1]);
        } else {
          bq[nq][j][0] = pack_h2(x[0], x[1]);
          bq[nq][j][1] = pack_h2(x[2], x[3]);
        }
      }
    }
  };
  if (!GEN || a.k.gran != 2) make_q(a.k.scale, (int64_t)bh * D, GEN && a.k.gran == 1);

  // running softmax state of the lane's query columns (2c, 2c+1 of each n tile)
  float mrun[NQ][2], lrun[NQ][2], O[NQ][NKB][4];
  int lim[NQ][2];
#pragma unroll
  for (int nq = 0; nq < NQ; ++nq)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      mrun[nq][e] = -INFINITY;
      lrun[nq][e] = 0.0f;
      const int qr = zb * NR + 8 * nq + 2 * c + e;
      lim[nq][e] = (a.causal && qr < a.rows) ? a.T - a.Sq + qr % a.Sq : a.T - 1;
    }
#pragma unroll
  for (int nq = 0; nq < NQ; ++nq)
#pragma unroll
    for (int e = 0; e < NKB; ++e)
#pragma unroll
      for (int u = 0; u < 4; ++u) O[nq][e][u] = 0.0f;

  // ---- main loop over this warp's tiles ----------------------------------
  // stage layout: K tile, V tile, then K scale / zero and V scale / zero rows;
  // compile-time on the all-per-token path (16 tokens x the scale size each)
  constexpr int SES = STC == LQ_F32 ? 4 : 2;
  const int SB = GEN ? a.stage_bytes : 2 * C::KB + 64 * SES;
  const int kso = GEN ? a.k.off_s : 2 * C::KB, kzo = GEN ? a.k.off_z : 2 * C::KB + 16 * SES;
  const int vso = GEN ? a.v.off_s : 2 * C::KB + 32 * SES, vzo = GEN ? a.v.off_z : 2 * C::KB + 48 * SES;
  uint8_t* ring_w = ring + (size_t)warp * C::STAGES * SB;
  // lane-constant byte offsets inside a stage: K rows g (g + 8: + 8 rows,
  // same swizzle), V rows 2c, 2c+1 (2c+8, 2c+9: + 8 rows)
  int koff[C::LKC];
#pragma unroll
  for (int i = 0; i < C::LKC; ++i) koff[i] = g * C::RB + (((c * C::LKC + i) ^ swz<C::CPR>(g)) << 4);
  constexpr int NVC = C::VB >= 16 ? C::VB / 16 : 1;
  int voff[2][NVC];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int r = 2 * c + e, byte0 = dv0 * CES;
#pragma unroll
    for (int i = 0; i < NVC; ++i)
      voff[e][i] = C::KB + r * C::RB + (((byte0 / 16 + i) ^ swz<C::CPR>(r)) << 4) + (C::VB >= 16 ? 0 : (byte0 & 15));
  }
  const int n_my = tile_hi > tile_lo + warp ? (tile_hi - tile_lo - warp + kAttnWarps - 1) / kAttnWarps : 0;
  // per-(b, h) bases of the codes and scale rows; per tile only t0 moves
  const uint8_t* kbase = a.k.codes + (int64_t)bh * a.cap * C::RB;
  const uint8_t* vbase = a.v.codes + (int64_t)bh * a.cap * C::RB;
  const int64_t ksrow = (int64_t)bh * a.k.pitch * (a.k.gran == 0 ? a.ses : D * a.ses);
  const int64_t vsrow = (int64_t)bh * a.v.pitch * (a.v.gran == 0 ? a.ses : D * a.ses);
  const int lr = lane / C::CPR, lj = lane % C::CPR;  // row / chunk of the lane's first chunk
  int ioff[kTile * C::CPR / 32];  // stage offsets of the lane's chunks lane + 32 i
#pragma unroll
  for (int i = 0; i < kTile * C::CPR / 32; ++i) {
    const int r = lr + i * (32 / C::CPR);
    ioff[i] = r * C::RB + ((lj ^ swz<C::CPR>(r)) << 4);
  }
  auto issue = [&](int tb, uint8_t* st) {
    const int t0 = tb * kTile;
    const uint8_t* kc = kbase + t0 * C::RB + lane * 16;
    const uint8_t* vc = vbase + t0 * C::RB + lane * 16;
#pragma unroll
    for (int i = 0; i < kTile * C::CPR / 32; ++i) {
      cp16(st + ioff[i], kc + 512 * i);
      cp16(st + C::KB + ioff[i], vc + 512 * i);
    }
    auto side = [&](const KvSide& s, int64_t base, int so, int zo) {
      if (s.bytes == 0) return;
      const int64_t row = base + (s.gran == 0 ? (int64_t)t0 * a.ses : (int64_t)(t0 / s.group) * D * a.ses);
      if (lane < s.bytes / 16) {  // at most 32 chunks per row
        cp16(st + so + lane * 16, s.scale + row + lane * 16);
        cp16(st + zo + lane * 16, s.zp + row + lane * 16);
      }
    };
    side(a.k, ksrow, kso, kzo);
    side(a.v, vsrow, vso, vzo);
  };
#pragma unroll
  for (int s = 0; s < C::STAGES; ++s) {
    if (s < n_my) issue(tile_lo + warp + kAttnWarps * s, ring_w + s * SB);
    cp_commit();
  }
  int slot = 0;
  for (int it = 0; it < n_my; ++it) {
    const int tb = tile_lo + warp + kAttnWarps * it;
    const int t0 = tb * kTile;
    uint8_t* st = ring_w + slot * SB;
    slot = slot + 1 == C::STAGES ? 0 : slot + 1;
    cp_wait<C::STAGES - 1>();
    __syncwarp();
    const bool full_tile = t0 + kTile <= a.T;
    const int tg = t0 + g, tg8 = t0 + g + 8;

    // per-tile scale rows (per-group) / per-token scalars
    float ks_g = 1.0f, ks_g8 = 1.0f;
    uint32_t zk_g = 0, zk_g8 = 0;
    if (!GEN || a.k.gran == 0) {
      const uint8_t* ksp = st + kso;
      const uint8_t* kzp = st + kzo;
      ks_g = lds<STC>(ksp, g, a.s_dtype);
      ks_g8 = lds<STC>(ksp, g + 8, a.s_dtype);
      const float z0 = tg < a.T ? lds<STC>(kzp, g, a.s_dtype) : 0.0f;
      const float z1 = tg8 < a.T ? lds<STC>(kzp, g + 8, a.s_dtype) : 0.0f;
      zk_g = zpair(z0, z0, bias);
      zk_g8 = zpair(z1, z1, bias);
    } else if (GEN && a.k.gran == 2) {
      fill_k_rows(st + kso, st + kzo, 0, true);
      make_q(st + kso, 0, true);
    }
    if (GEN && a.v.gran == 2) fill_v_rows(st + vso, st + vzo, 0);

    // ---- S = K q'^T ----
    float S[NQ][4], S1[NQ][4];  // even / odd k blocks: two MMA chains
#pragma unroll
    for (int nq = 0; nq < NQ; ++nq)
#pragma unroll
      for (int u = 0; u < 4; ++u) S[nq][u] = S1[nq][u] = 0.0f;
    uint32_t kw[2][C::LKC * 4];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
#pragma unroll
      for (int i = 0; i < C::LKC; ++i) {
        const uint4 w = *reinterpret_cast<const uint4*>(st + koff[i] + 8 * C::RB * rr);
        kw[rr][4 * i] = w.x;
        kw[rr][4 * i + 1] = w.y;
        kw[rr][4 * i + 2] = w.z;
        kw[rr][4 * i + 3] = w.w;
      }
    }
#pragma unroll
    for (int j = 0; j < NKB; ++j) {
      uint32_t ka[4];
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        uint32_t lo, hi;
        if constexpr (CES == 1) {
          const uint32_t w = kw[rr][j] ^ 0x80808080u;
          lo = Codes<1>::pair(w, 0);
          hi = Codes<1>::pair(w, 1);
        } else {
          lo = Codes<2>::pair(kw[rr][2 * j]);
          hi = Codes<2>::pair(kw[rr][2 * j + 1]);
        }
        if (!GEN || a.k.gran == 0) {
          const uint32_t z = rr ? zk_g8 : zk_g;
          ka[rr] = hsub2(lo, z);
          ka[2 + rr] = hsub2(hi, z);
        } else {
          ka[rr] = hsub2(lo, zkp[GEN ? j : 0][0]);
          ka[2 + rr] = hsub2(hi, zkp[GEN ? j : 0][1]);
        }
      }
#pragma unroll
      for (int nq = 0; nq < NQ; ++nq) {
        float* acc = (j & 1) ? S1[nq] : S[nq];
        mma_f16(acc, ka, bq[nq][j][0], bq[nq][j][1]);
        if constexpr (QLO) mma_f16(acc, ka, bql[nq][j][0], bql[nq][j][1]);
      }
    }
#pragma unroll
    for (int nq = 0; nq < NQ; ++nq)
#pragma unroll
      for (int u = 0; u < 4; ++u) S[nq][u] += S1[nq][u];

    // ---- scale, mask, online softmax ----
    float fk0, fk1;
    if (!GEN || a.k.gran == 0) {
      fk0 = ks_g * a.sm_log2;
      fk1 = ks_g8 * a.sm_log2;
    } else {
      fk0 = fk1 = sigma_k * a.sm_log2;
    }
    // per-token V: P' = P * vs_t, taken as exp2(s + log2(vs_t) - m') with the
    // running max m' over s + log2(vs_t), so P' <= 1 fits the f16 operand;
    // the softmax denominator sums exp2(s - m') separately
    const bool vtok = !GEN || a.v.gran == 0;
    float lv0 = 0.0f, lv1 = 0.0f;
    if (vtok) {
      lv0 = tg < a.T ? lg2(lds<STC>(st + vso, g, a.s_dtype)) : 0.0f;
      lv1 = tg8 < a.T ? lg2(lds<STC>(st + vso, g + 8, a.s_dtype)) : 0.0f;
    }
    uint32_t pb[NQ][2], pbl[NQ][2];
#pragma unroll
    for (int nq = 0; nq < NQ; ++nq) {
      float p[4], alpha[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float s0 = tg <= lim[nq][e] ? S[nq][e] * fk0 : -INFINITY;
        const float s1 = tg8 <= lim[nq][e] ? S[nq][2 + e] * fk1 : -INFINITY;
        const float w0 = s0 + lv0, w1 = s1 + lv1;
        float mt = fmaxf(w0, w1);
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
        mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
        const float mnew = fmaxf(mrun[nq][e], mt);
        const float mref = mnew == -INFINITY ? 0.0f : mnew;
        alpha[e] = mnew > mrun[nq][e] ? ex2(mrun[nq][e] - mref) : 1.0f;
        p[e] = ex2(w0 - mref);
        p[2 + e] = ex2(w1 - mref);
        const float den = vtok ? ex2(s0 - mref) + ex2(s1 - mref) : p[e] + p[2 + e];
        lrun[nq][e] = lrun[nq][e] * alpha[e] + den;
        mrun[nq][e] = mnew;
      }
      // rescale O only when a running max of the warp's columns grew
      if (__any_sync(0xffffffffu, alpha[0] != 1.0f || alpha[1] != 1.0f)) {
#pragma unroll
        for (int d = 0; d < NKB; ++d) {
          O[nq][d][0] *= alpha[0];
          O[nq][d][1] *= alpha[1];
          O[nq][d][2] *= alpha[0];
          O[nq][d][3] *= alpha[1];
        }
      }
      // P' rows t = g (tokens 0-7 block) and t = g + 8, columns 2c, 2c+1
      uint32_t x0, x1, l0, l1;
      split_h2(p[0], p[1], x0, l0);
      split_h2(p[2], p[3], x1, l1);
      pb[nq][0] = trans8x8(x0);
      pb[nq][1] = trans8x8(x1);
      pbl[nq][0] = trans8x8(l0);
      pbl[nq][1] = trans8x8(l1);
    }

    // ---- O += V^T P'^T ----
    // lane rows 2c, 2c+1, 2c+8, 2c+9; bytes [dv0 * CES, +VB)
    constexpr int VWORDS = C::VB / 4;
    uint32_t vw[4][VWORDS];
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) {
      const int r = 2 * c + (q4 & 1) + 8 * (q4 >> 1);
      const uint8_t* vp = st + 8 * C::RB * (q4 >> 1);
      if constexpr (C::VB >= 16) {
#pragma unroll
        for (int i = 0; i < C::VB / 16; ++i) {
          const uint4 w = *reinterpret_cast<const uint4*>(vp + voff[q4 & 1][i]);
          vw[q4][4 * i] = w.x;
          vw[q4][4 * i + 1] = w.y;
          vw[q4][4 * i + 2] = w.z;
          vw[q4][4 * i + 3] = w.w;
        }
      } else {  // 8 bytes: half of a chunk
        const uint2 w = *reinterpret_cast<const uint2*>(vp + voff[q4 & 1][0]);
        vw[q4][0] = w.x;
        vw[q4][1] = w.y;
      }
      if (!full_tile && t0 + r >= a.T) {  // past the end: unwritten codes -> 0
#pragma unroll
        for (int i = 0; i < VWORDS; ++i) vw[q4][i] = 0u;
      }
    }
    uint32_t zv_a = 0, zv_b = 0;  // per-token V zero pairs of rows (2c, 2c+1), (2c+8, 2c+9)
    if (!GEN || a.v.gran == 0) {
      const uint8_t* vzp = st + vzo;
      const int ra = 2 * c, rb = 2 * c + 8;
      const float z0 = t0 + ra < a.T ? lds<STC>(vzp, ra, a.s_dtype) : 0.0f;
      const float z1 = t0 + ra + 1 < a.T ? lds<STC>(vzp, ra + 1, a.s_dtype) : 0.0f;
      const float z2 = t0 + rb < a.T ? lds<STC>(vzp, rb, a.s_dtype) : 0.0f;
      const float z3 = t0 + rb + 1 < a.T ? lds<STC>(vzp, rb + 1, a.s_dtype) : 0.0f;
      zv_a = zpair(z0, z1, bias);
      zv_b = zpair(z2, z3, bias);
    }
    float Ot[GEN ? NQ : 1][GEN ? NKB : 1][4];
    if constexpr (GEN) {
#pragma unroll
      for (int nq = 0; nq < NQ; ++nq)
#pragma unroll
        for (int e = 0; e < NKB; ++e)
#pragma unroll
          for (int u = 0; u < 4; ++u) Ot[nq][e][u] = 0.0f;
    }
    const bool vgroup = GEN && a.v.gran == 2;
#pragma unroll
    for (int e = 0; e < NKB; ++e) {
      // d = dv0 + 2e (A row g) and d + 1 (A row g + 8); tokens (2c, 2c+1) | (2c+8, 2c+9)
      uint32_t av[4];
#pragma unroll
      for (int half = 0; half < 2; ++half) {  // half 0: rows 2c, 2c+1; half 1: rows 2c+8, 2c+9
        const int qa = 2 * half, qb = 2 * half + 1;
        uint32_t p0, p1;  // (V[a][d], V[b][d]), (V[a][d+1], V[b][d+1])
        if constexpr (CES == 1) {
          const int w = e >> 1, hh = e & 1;  // word w of the lane's bytes, pair (2hh, 2hh+1)
          const uint32_t wa = vw[qa][w] ^ 0x80808080u, wb = vw[qb][w] ^ 0x80808080u;
          const uint32_t x = __byte_perm(wa, wb, hh ? 0x7362 : 0x5140);  // (a_d, b_d, a_d1, b_d1)
          p0 = Codes<1>::pair(x, 0);
          p1 = Codes<1>::pair(x, 1);
        } else {
          const uint32_t wa = vw[qa][e], wb = vw[qb][e];  // codes (d, d+1) of rows a, b
          p0 = Codes<2>::pair(__byte_perm(wa, wb, 0x5410));
          p1 = Codes<2>::pair(__byte_perm(wa, wb, 0x7632));
        }
        if (!GEN || a.v.gran == 0) {
          const uint32_t z = half ? zv_b : zv_a;
          av[2 * half] = hsub2(p0, z);
          av[2 * half + 1] = hsub2(p1, z);
        } else {
          av[2 * half] = hsub2(p0, zvp[GEN ? e : 0][0]);
          av[2 * half + 1] = hsub2(p1, zvp[GEN ? e : 0][1]);
        }
      }
      // A fragment order: a0 = (row g, k 2c..), a1 = (row g+8, k 2c..), a2 = (row g, k 2c+8..), a3
      const uint32_t afr[4] = {av[0], av[1], av[2], av[3]};
#pragma unroll
      for (int nq = 0; nq < NQ; ++nq) {
        float* acc = O[nq][e];
        if constexpr (GEN) {
          if (vgroup) acc = Ot[nq][e];
        }
        mma_f16(acc, afr, pb[nq][0], pb[nq][1]);
        mma_f16(acc, afr, pbl[nq][0], pbl[nq][1]);
      }
    }
    if constexpr (GEN) {
      if (vgroup) {
#pragma unroll
        for (int nq = 0; nq < NQ; ++nq)
#pragma unroll
          for (int e = 0; e < NKB; ++e) {
            O[nq][e][0] = fmaf(vsd[e][0], Ot[nq][e][0], O[nq][e][0]);
            O[nq][e][1] = fmaf(vsd[e][0], Ot[nq][e][1], O[nq][e][1]);
            O[nq][e][2] = fmaf(vsd[e][1], Ot[nq][e][2], O[nq][e][2]);
            O[nq][e][3] = fmaf(vsd[e][1], Ot[nq][e][3], O[nq][e][3]);
          }
      }
    }
    __syncwarp();  // every lane has read the stage before it is refilled
    if (it + C::STAGES < n_my) issue(tb + kAttnWarps * C::STAGES, st);
    cp_commit();
  }
  cp_wait<0>();

  // ---- final V scale, row sums ----
#pragma unroll
  for (int nq = 0; nq < NQ; ++nq) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      float l = lrun[nq][e];
      l += __shfl_xor_sync(0xffffffffu, l, 4);
      l += __shfl_xor_sync(0xffffffffu, l, 8);
      l += __shfl_xor_sync(0xffffffffu, l, 16);
      lrun[nq][e] = l;
    }
#pragma unroll
    for (int e = 0; e < NKB; ++e) {
      float f0 = 1.0f, f1 = 1.0f;
      if (GEN && a.v.gran == 1) {
        f0 = vsd[GEN ? e : 0][0];
        f1 = vsd[GEN ? e : 0][1];
      }
      O[nq][e][0] *= f0;
      O[nq][e][1] *= f0;
      O[nq][e][2] *= f1;
      O[nq][e][3] *= f1;
    }
  }

  // ---- merge the 4 warps in shared memory (the ring is free now) ----
  if (threadIdx.x == 0) pdl_trigger();  // token loop done: the combine's blocks may launch
  __syncthreads();
  float* mb = reinterpret_cast<float*>(ring);  // [warps][NR]
  float* lb = mb + kAttnWarps * NR;            // [warps][NR]
  float* ob = lb + kAttnWarps * NR;            // [warps][NR][D]
  if (g == 0) {
#pragma unroll
    for (int nq = 0; nq < NQ; ++nq)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        mb[warp * NR + 8 * nq + 2 * c + e] = mrun[nq][e];
        lb[warp * NR + 8 * nq + 2 * c + e] = lrun[nq][e];
      }
  }
#pragma unroll
  for (int nq = 0; nq < NQ; ++nq)
#pragma unroll
    for (int e = 0; e < NKB; ++e)
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int col = 8 * nq + 2 * c + (u & 1);
        const int d = dv0 + 2 * e + (u >> 1);
        ob[(warp * NR + col) * D + d] = O[nq][e][u];
      }
  __syncthreads();
  for (int idx = threadIdx.x; idx < NR * D; idx += blockDim.x) {
    const int r = idx / D, d = idx % D, qr = zb * NR + r;
    if (qr >= a.rows) continue;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, mb[w * NR + r]);
    float o = 0.0f, L = 0.0f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w) {
        const float f = ex2(mb[w * NR + r] - M);
        o = fmaf(f, ob[(w * NR + r) * D + d], o);
        L = fmaf(f, lb[w * NR + r], L);
      }
    }
    if (a.n_split == 1) {
      const int hq = h * a.G + qr / a.Sq, i = qr % a.Sq;
      st_f(a.out, (((int64_t)b * a.Hq + hq) * a.Sq + i) * D + d, a.q_dtype, o / L);
    } else {
      float* p = a.ws + (((int64_t)bh * a.n_split + split) * a.rows + qr) * (D + 2);
      p[d] = o;
      if (d == 0) {
        p[D] = M;
        p[D + 1] = L;
      }
    }
  }
}

// One thread per output element (b, h, row, d): merge the splits' (O, max,
// sum) partials; the (max, sum) pairs of a row are read by all its threads
// (L1 broadcast).
__global__ void __launch_bounds__(128) kv_attn_combine_kernel(const float* __restrict__ ws, int n_split,
                                                              int rows, int D, int H, int Hq, int Sq,
                                                              int G, int64_t n_items, uint8_t* out,
                                                              int out_dtype) {
  pdl_wait();  // the attention kernel's partials are complete and visible
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n_items * D) return;
  const int64_t item = e / D;
  const int d = (int)(e % D);
  const int64_t bh = item / rows;
  const int qr = (int)(item % rows);
  const float* base = ws + (bh * n_split * rows + qr) * (int64_t)(D + 2);
  const int64_t sstride = (int64_t)rows * (D + 2);
  float M = -INFINITY;
#pragma unroll 8
  for (int s = 0; s < n_split; ++s) M = fmaxf(M, __ldg(base + s * sstride + D));
  float o = 0.0f, L = 0.0f;
  if (M != -INFINITY) {
#pragma unroll 8
    for (int s = 0; s < n_split; ++s) {
      const float* p = base + s * sstride;
      const float f = ex2(__ldg(p + D) - M);
      o = fmaf(f, __ldg(p + d), o);
      L = fmaf(f, __ldg(p + D + 1), L);
    }
  }
  const int b = (int)(bh / H), h = (int)(bh % H);
  const int hq = h * G + qr / Sq, i = qr % Sq;
  st_f(out, (((int64_t)b * Hq + hq) * Sq + i) * D + d, out_dtype, o / L);
}

// SMs of the current device (148 on B200; 148 when there is none, for the
// workspace query on a host without a GPU).
int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return 148;
  }
  if (!cached[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = 148;
    }
    cached[dev] = n;
  }
  return cached[dev];
}

// Token splits: one wave of blocks (4 resident per SM for the per-token
// variants), each as long as possible -- the pipeline fill, the q prologue
// and the warp merge are paid once per block -- with at least 4 tiles (one
// per warp) per split.
struct SplitPlan {
  int n_tiles, n_split, tiles_per_split;
};
SplitPlan plan_split(int64_t BH, int64_t row_blocks, int64_t T) {
  SplitPlan p;
  p.n_tiles = (int)((T + kTile - 1) / kTile);
  const int64_t slots = (int64_t)sm_count() * 4;
  int64_t ns = std::max<int64_t>(1, slots / (BH * row_blocks));
  ns = std::min<int64_t>(ns, std::max(1, p.n_tiles / kAttnWarps));
  p.tiles_per_split = (int)((p.n_tiles + ns - 1) / ns);
  p.n_split = (p.n_tiles + p.tiles_per_split - 1) / p.tiles_per_split;
  return p;
}

template <int D, int CES, int NQ, bool GEN, bool QLO, int STC>
int launch_attn(const AttnArgs& a, int B, int row_blocks, int combine_items, cudaStream_t st) {
  using C = AttnCfg<D, CES>;
  constexpr int NR = 8 * NQ;
  const size_t ring = (size_t)kAttnWarps * C::STAGES * a.stage_bytes;
  const size_t merge = (size_t)kAttnWarps * NR * (D + 2) * 4;
  const size_t smem = (size_t)NR * C::QS * 4 + 32 + std::max(ring, merge);
  auto kern = kv_attn_kernel<D, CES, NQ, GEN, QLO, STC>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return launched("kv_attn_kernel (attribute)");
  dim3 grid(a.n_split, B * a.H, row_blocks);
  kern<<<grid, 32 * kAttnWarps, smem, st>>>(a);
  int rc = launched("kv_attn_kernel");
  if (rc != LQ_OK || a.n_split == 1) return rc;
  launch_pdl(kv_attn_combine_kernel, dim3((unsigned)((combine_items * D + 127) / 128)), dim3(128), 0, st,
             (const float*)a.ws, a.n_split, a.rows, D, a.H, a.Hq, a.Sq, a.G, (int64_t)combine_items, a.out,
             a.q_dtype);
  return launched("kv_attn_combine_kernel");
}

template <int D, int CES, int NQ>
int attn_dispatch_nq(const AttnArgs& a, int B, bool gen, int row_blocks, int items, cudaStream_t st) {
  // a per-token K with an f16 / bf16 query needs no lo half of q'
  // the all-per-token path is compiled per scale dtype; the general one reads
  // scales with a runtime dtype switch
  if (gen) return launch_attn<D, CES, NQ, true, true, -1>(a, B, row_blocks, items, st);
  switch (a.s_dtype) {
    case LQ_F32:
      return a.qlo ? launch_attn<D, CES, NQ, false, true, LQ_F32>(a, B, row_blocks, items, st)
                   : launch_attn<D, CES, NQ, false, false, LQ_F32>(a, B, row_blocks, items, st);
    case LQ_F16:
      return a.qlo ? launch_attn<D, CES, NQ, false, true, LQ_F16>(a, B, row_blocks, items, st)
                   : launch_attn<D, CES, NQ, false, false, LQ_F16>(a, B, row_blocks, items, st);
    default:
      return a.qlo ? launch_attn<D, CES, NQ, false, true, LQ_BF16>(a, B, row_blocks, items, st)
                   : launch_attn<D, CES, NQ, false, false, LQ_BF16>(a, B, row_blocks, items, st);
  }
}

template <int D, int CES>
int attn_dispatch(const AttnArgs& a, int B, int nq, bool gen, int row_blocks, int items, cudaStream_t st) {
  return nq == 1 ? attn_dispatch_nq<D, CES, 1>(a, B, gen, row_blocks, items, st)
                 : attn_dispatch_nq<D, CES, 2>(a, B, gen, row_blocks, items, st);
}

}  // namespace
}  // namespace lq

extern "C" size_t lq_kv_attention_workspace_bytes(int64_t B, int64_t Hq, int64_t H, int64_t Sq,
                                                  int64_t D, int64_t T) {
  using namespace lq;
  if (B <= 0 || H <= 0 || Hq <= 0 || Sq <= 0 || D <= 0 || T <= 0 || Hq % H) return 0;
  const int64_t rows = Hq / H * Sq;
  const int64_t nr = rows <= 8 ? 8 : 16;
  const SplitPlan p = plan_split(B * H, (rows + nr - 1) / nr, T);
  if (p.n_split == 1) return 0;
  return (size_t)(B * H) * p.n_split * rows * (D + 2) * sizeof(float);
}

extern "C" int lq_kv_attention(const void* q, int q_dtype, int64_t B, int64_t Hq, int64_t H,
                               int64_t Sq, int64_t D, int64_t T, int64_t cap, int code_dtype,
                               const void* k_codes, int k_gran, int64_t k_group, const void* k_scale,
                               const void* k_zp, int64_t k_pitch, const void* v_codes, int v_gran,
                               int64_t v_group, const void* v_scale, const void* v_zp,
                               int64_t v_pitch, int s_dtype, float sm_scale, int causal, void* out,
                               void* workspace, size_t workspace_bytes, void* stream) {
  using namespace lq;
  LQ_REQUIRE(B >= 0 && H > 0 && Hq > 0 && Sq >= 0 && T >= 0, LQ_EINVAL, "bad shape");
  LQ_REQUIRE(Hq % H == 0, LQ_EINVAL, "query heads %lld not a multiple of kv heads %lld", (long long)Hq,
             (long long)H);
  LQ_REQUIRE(D == 64 || D == 128, LQ_EINVAL, "head dim %lld: 64 or 128 supported", (long long)D);
  LQ_REQUIRE(code_dtype == LQ_I8 || code_dtype == LQ_I16, LQ_EDTYPE, "codes must be int8 / int16");
  LQ_REQUIRE(is_float_dtype(q_dtype) && is_float_dtype(s_dtype), LQ_EDTYPE, "float q / scales required");
  LQ_REQUIRE(k_gran >= 0 && k_gran <= 2 && v_gran >= 0 && v_gran <= 2, LQ_EINVAL, "bad granularity");
  LQ_REQUIRE(cap % kTile == 0 && cap >= T, LQ_EINVAL, "capacity %lld must be a multiple of %d and >= T",
             (long long)cap, kTile);
  LQ_REQUIRE(k_gran != 2 || (k_group > 0 && k_group % kTile == 0), LQ_EINVAL,
             "per-group K needs a group size that is a multiple of %d", kTile);
  LQ_REQUIRE(v_gran != 2 || (v_group > 0 && v_group % kTile == 0), LQ_EINVAL,
             "per-group V needs a group size that is a multiple of %d", kTile);
  LQ_REQUIRE(k_gran != 0 || k_pitch >= cap, LQ_EINVAL, "per-token K scale pitch < capacity");
  LQ_REQUIRE(v_gran != 0 || v_pitch >= cap, LQ_EINVAL, "per-token V scale pitch < capacity");
  LQ_REQUIRE(k_gran != 2 || k_pitch * k_group >= T, LQ_EINVAL, "per-group K scale rows too few");
  LQ_REQUIRE(v_gran != 2 || v_pitch * v_group >= T, LQ_EINVAL, "per-group V scale rows too few");
  if (B * Hq * Sq * D == 0) return LQ_OK;
  LQ_REQUIRE(T > 0, LQ_EINVAL, "empty cache");
  LQ_REQUIRE(q && out && k_codes && v_codes && k_scale && k_zp && v_scale && v_zp, LQ_EINVAL, "NULL pointer");
  LQ_REQUIRE(aligned16(k_codes) && aligned16(v_codes) && aligned16(k_scale) && aligned16(k_zp) &&
                 aligned16(v_scale) && aligned16(v_zp),
             LQ_EALIGN, "codes / scales must be 16-byte aligned");
  const int ses = dtype_size(s_dtype);
  LQ_REQUIRE((k_gran != 0 || (k_pitch * ses) % 16 == 0) && (v_gran != 0 || (v_pitch * ses) % 16 == 0),
             LQ_EALIGN, "per-token scale pitch must be a multiple of 16 bytes");
  const int64_t rows = Hq / H * Sq;
  const int nq = rows <= 8 ? 1 : 2;
  const int64_t row_blocks = (rows + 8 * nq - 1) / (8 * nq);
  LQ_REQUIRE(B * H <= 65535 && row_blocks <= 65535, LQ_ERANGE, "too many heads / rows");
  const SplitPlan p = plan_split(B * H, row_blocks, T);
  if (p.n_split > 1) {
    const size_t need = (size_t)(B * H) * p.n_split * rows * (D + 2) * sizeof(float);
    LQ_REQUIRE(workspace && workspace_bytes >= need, LQ_EINVAL, "workspace of %zu bytes needed", need);
  }
  const int ces = code_dtype == LQ_I8 ? 1 : 2;
  AttnArgs a;
  a.q = static_cast<const uint8_t*>(q);
  a.q_dtype = q_dtype;
  a.s_dtype = s_dtype;
  a.ses = ses;
  a.Hq = (int)Hq;
  a.H = (int)H;
  a.Sq = (int)Sq;
  a.G = (int)(Hq / H);
  a.rows = (int)rows;
  a.T = (int)T;
  a.cap = (int)cap;
  a.sm_log2 = sm_scale * 1.4426950408889634f;
  a.causal = causal ? 1 : 0;
  a.qlo = (q_dtype == LQ_F32 || k_gran != 0) ? 1 : 0;
  a.n_tiles = p.n_tiles;
  a.n_split = p.n_split;
  a.tiles_per_split = p.tiles_per_split;
  auto side = [&](KvSide& s, const void* codes, int gran, int64_t group, const void* sc, const void* zp,
                  int64_t pitch) {
    s.codes = static_cast<const uint8_t*>(codes);
    s.scale = static_cast<const uint8_t*>(sc);
    s.zp = static_cast<const uint8_t*>(zp);
    s.pitch = pitch;
    s.gran = gran;
    s.group = (int)(gran == 2 ? group : 1);
    s.bytes = gran == 0 ? kTile * ses : gran == 2 ? (int)D * ses : 0;
  };
  side(a.k, k_codes, k_gran, k_group, k_scale, k_zp, k_pitch);
  side(a.v, v_codes, v_gran, v_group, v_scale, v_zp, v_pitch);
  int off = 2 * kTile * (int)D * ces;
  a.k.off_s = off;
  off += a.k.bytes;
  a.k.off_z = off;
  off += a.k.bytes;
  a.v.off_s = off;
  off += a.v.bytes;
  a.v.off_z = off;
  off += a.v.bytes;
  a.stage_bytes = (off + 15) / 16 * 16;
  a.out = static_cast<uint8_t*>(out);
  a.ws = static_cast<float*>(workspace);
  const bool gen = k_gran != 0 || v_gran != 0;
  const int items = (int)(B * H * rows);
  cudaStream_t st = as_stream(stream);
  if (D == 64)
    return ces == 1 ? attn_dispatch<64, 1>(a, (int)B, nq, gen, (int)row_blocks, items, st)
                    : attn_dispatch<64, 2>(a, (int)B, nq, gen, (int)row_blocks, items, st);
  return ces == 1 ? attn_dispatch<128, 1>(a, (int)B, nq, gen, (int)row_blocks, items, st)
                  : attn_dispatch<128, 2>(a, (int)B, nq, gen, (int)row_blocks, items, st);
}
