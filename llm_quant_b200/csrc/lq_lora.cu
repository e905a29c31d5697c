// lq_lora.cu -- the LoRA down-projection of QLoRALinear.forward
// (qlora.py:311: F.linear(x, lora_A) * scaling), written straight into the
// zero-padded [M, 64] activation-dtype operand that the fused NF4 kernels take
// as u.  One launch replaces a memset, a dtype cast of lora_A and a cuBLAS
// call with a 16-column output.
//
// A block owns a 16-token tile of x; its 16 warps take the K steps (64 wide)
// w, w + 16, ... (a few each, their loads in flight together) and run mma.sync.m16n8k16 (fp32 accumulate) with x as A and
// lora_A^T as B, one 8-column B tile per 8 ranks.  A lane reads the 16
// contiguous halves 16c .. 16c+15 of each step for its two token rows and its
// rank row (the k slots of the four MMAs of a step are a fixed permutation of
// those 16, the same on both operands, so each lane needs two 16-byte loads
// per row and no shuffles).  The warps' partial sums are added in shared
// memory; the block writes scaling * sum rounded to the activation dtype, and
// zeros in columns rank .. 63.  (Splitting K over a cluster of blocks, summed
// through distributed shared memory, measured slower: 12.1 against 7.9 us at
// M = 1024, K = 4096, rank 16.)  Up to 16 tokens there is only one tile, and
// one block reading all of lora_A is the whole cost: there the K split over a
// cluster of eight small blocks (lora_u_split_kernel) is used, 4.2 -> 3.2 us.
#include <type_traits>

#include "lq_common.cuh"

namespace lq {
namespace {

constexpr int kLuWarps = 16;
constexpr int kLuPitch = 64;  // u row pitch (the fused kernels' LoRA K step)

template <typename T> struct LuMma;
template <> struct LuMma<__half> {
  __device__ __forceinline__ static void mma(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
};
template <> struct LuMma<__nv_bfloat16> {
  __device__ __forceinline__ static void mma(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
};

__device__ __forceinline__ uint32_t lu_word(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// 16 k values of rank row `row` (zero past the rank) as 8 words of T pairs
template <typename T, typename AT>
__device__ __forceinline__ void lu_load_a(const AT* a, int row, int rank, int64_t K, int64_t k, uint4 (&w)[2]) {
  if (row >= rank) {
    w[0] = w[1] = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  if constexpr (std::is_same<AT, float>::value) {
    const float4* p = reinterpret_cast<const float4*>(a + (size_t)row * K + k);
    float4 f[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = __ldg(p + i);
    w[0] = make_uint4(LuMma<T>::pack(f[0].x, f[0].y), LuMma<T>::pack(f[0].z, f[0].w), LuMma<T>::pack(f[1].x, f[1].y),
                      LuMma<T>::pack(f[1].z, f[1].w));
    w[1] = make_uint4(LuMma<T>::pack(f[2].x, f[2].y), LuMma<T>::pack(f[2].z, f[2].w), LuMma<T>::pack(f[3].x, f[3].y),
                      LuMma<T>::pack(f[3].z, f[3].w));
  } else {
    const uint4* p = reinterpret_cast<const uint4*>(a + (size_t)row * K + k);
    w[0] = __ldg(p);
    w[1] = __ldg(p + 1);
  }
}

template <typename T, typename AT, int NTL>
__global__ void __launch_bounds__(32 * kLuWarps) lora_u_kernel(const T* __restrict__ x, const AT* __restrict__ a,
                                                               T* __restrict__ u, int64_t M, int64_t K, int rank,
                                                               float scaling) {
  constexpr int H = kLuWarps / 2;
  __shared__ float red[H][NTL][32][4];
  // launched as a programmatic dependent: wait for the kernel ahead of it (which
  // may write x) before the first global access, and only then let the fused
  // linear that consumes u start -- it reads x and the weights at once and
  // waits for this grid only before it reads u
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int64_t n_tiles = (M + 15) / 16;
  for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
  const int64_t m0 = tile * 16;
  // token rows of this lane (rows past M read row M - 1; never stored)
  const int64_t r0 = min(m0 + g, M - 1), r1 = min(m0 + g + 8, M - 1);
  float d[NTL][4];
#pragma unroll
  for (int nt = 0; nt < NTL; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) d[nt][e] = 0.0f;
  const int64_t n_steps = K / 64;
  constexpr int UNR = NTL <= 2 ? 4 : NTL <= 4 ? 2 : 1;
#pragma unroll UNR
  for (int64_t s = warp; s < n_steps; s += kLuWarps) {
    const int64_t k = s * 64 + 16 * c;
    const uint4* p0 = reinterpret_cast<const uint4*>(x + r0 * K + k);
    const uint4* p1 = reinterpret_cast<const uint4*>(x + r1 * K + k);
    const uint4 x0[2] = {__ldg(p0), __ldg(p0 + 1)};
    const uint4 x1[2] = {__ldg(p1), __ldg(p1 + 1)};
    uint4 av[NTL][2];
#pragma unroll
    for (int nt = 0; nt < NTL; ++nt) lu_load_a<T, AT>(a, nt * 8 + g, rank, K, k, av[nt]);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int h = t >> 1, w0 = 2 * (t & 1);
#pragma unroll
      for (int nt = 0; nt < NTL; ++nt)
        LuMma<T>::mma(d[nt], lu_word(x0[h], w0), lu_word(x1[h], w0), lu_word(x0[h], w0 + 1), lu_word(x1[h], w0 + 1),
                      lu_word(av[nt][h], w0), lu_word(av[nt][h], w0 + 1));
    }
  }
  // warps w and w + 8 share a slot of the partial sums
  if (warp >= H) {
#pragma unroll
    for (int nt = 0; nt < NTL; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) red[warp - H][nt][lane][e] = d[nt][e];
  }
  __syncthreads();
  if (warp < H) {
#pragma unroll
    for (int nt = 0; nt < NTL; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) red[warp][nt][lane][e] += d[nt][e];
  }
  __syncthreads();
  // 16 rows x 32 column pairs of the padded output
  for (int i = threadIdx.x; i < 16 * (kLuPitch / 2); i += blockDim.x) {
    const int row = i / (kLuPitch / 2), pr = i % (kLuPitch / 2);
    if (m0 + row >= M) continue;
    const int nt = pr / 4, cc = pr % 4, ln = (row % 8) * 4 + cc, e = row >= 8 ? 2 : 0;
    float v0 = 0.0f, v1 = 0.0f;
    if (nt < NTL && 2 * pr < rank) {
#pragma unroll
      for (int w = 0; w < H; ++w) {
        v0 += red[w][nt][ln][e];
        v1 += red[w][nt][ln][e + 1];
      }
      v0 *= scaling;
      v1 = 2 * pr + 1 < rank ? v1 * scaling : 0.0f;
    }
    reinterpret_cast<uint32_t*>(u + (m0 + row) * kLuPitch)[pr] = LuMma<T>::pack(v0, v1);
  }
  __syncthreads();  // red is rewritten by the next tile
  }
}

// At most 16 tokens (one token tile): the K steps are split over a cluster
// of kLoraUSplitBlocks blocks of 4 warps (block r takes steps [r S / B,
// (r + 1) S / B), its warps those steps round robin), so that the 128 KB of a
// rank-16 lora_A are read by eight SMs instead of one.  Each block adds its
// warps' partial sums in shared memory; after a cluster barrier block r adds
// the blocks' sums, in block order, for its share of the 16 x 64 outputs
// through distributed shared memory, and a second barrier keeps every
// block's shared memory alive until those reads are done.
constexpr int kLsWarps = 4;

__device__ __forceinline__ float ld_cluster_f32(const float* p, uint32_t rank) {
  uint32_t ra;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
  return v;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

template <typename T, typename AT, int NTL>
__global__ void __launch_bounds__(32 * kLsWarps) lora_u_split_kernel(const T* __restrict__ x, const AT* __restrict__ a,
                                                                    T* __restrict__ u, int M, int64_t K, int rank,
                                                                    float scaling) {
  constexpr int B = kLoraUSplitBlocks;
  __shared__ float part[kLsWarps][NTL][32][4];
  __shared__ float sum[NTL][32][4];
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int blk = (int)blockIdx.x;  // the cluster is the whole grid: rank = blockIdx.x
  const int64_t r0 = min(g, M - 1), r1 = min(g + 8, M - 1);
  float d[NTL][4];
#pragma unroll
  for (int nt = 0; nt < NTL; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) d[nt][e] = 0.0f;
  const int64_t n_steps = K / 64;
  const int64_t s_lo = n_steps * blk / B, s_hi = n_steps * (blk + 1) / B;
#pragma unroll 2
  for (int64_t s = s_lo + warp; s < s_hi; s += kLsWarps) {
    const int64_t k = s * 64 + 16 * c;
    const uint4* p0 = reinterpret_cast<const uint4*>(x + r0 * K + k);
    const uint4* p1 = reinterpret_cast<const uint4*>(x + r1 * K + k);
    const uint4 x0[2] = {__ldg(p0), __ldg(p0 + 1)};
    const uint4 x1[2] = {__ldg(p1), __ldg(p1 + 1)};
    uint4 av[NTL][2];
#pragma unroll
    for (int nt = 0; nt < NTL; ++nt) lu_load_a<T, AT>(a, nt * 8 + g, rank, K, k, av[nt]);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int h = t >> 1, w0 = 2 * (t & 1);
#pragma unroll
      for (int nt = 0; nt < NTL; ++nt)
        LuMma<T>::mma(d[nt], lu_word(x0[h], w0), lu_word(x1[h], w0), lu_word(x0[h], w0 + 1), lu_word(x1[h], w0 + 1),
                      lu_word(av[nt][h], w0), lu_word(av[nt][h], w0 + 1));
    }
  }
#pragma unroll
  for (int nt = 0; nt < NTL; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) part[warp][nt][lane][e] = d[nt][e];
  __syncthreads();
  for (int i = threadIdx.x; i < NTL * 32 * 4; i += blockDim.x) {
    float v = 0.0f;
#pragma unroll
    for (int w = 0; w < kLsWarps; ++w) v += (&part[w][0][0][0])[i];
    (&sum[0][0][0])[i] = v;
  }
  cluster_sync_all();
  // block blk writes outputs (row, column pair) i = blk, blk + B, ... of the
  // 16 x 32 column pairs of u (zeros past the rank)
  for (int i = blk * blockDim.x + threadIdx.x; i < 16 * (kLuPitch / 2); i += B * blockDim.x) {
    const int row = i / (kLuPitch / 2), pr = i % (kLuPitch / 2);
    if (row >= M) continue;
    const int nt = pr / 4, cc = pr % 4, ln = (row % 8) * 4 + cc, e = row >= 8 ? 2 : 0;
    float v0 = 0.0f, v1 = 0.0f;
    if (nt < NTL && 2 * pr < rank) {
#pragma unroll
      for (int r = 0; r < B; ++r) {
        v0 += ld_cluster_f32(&sum[nt][ln][e], (uint32_t)r);
        v1 += ld_cluster_f32(&sum[nt][ln][e + 1], (uint32_t)r);
      }
      v0 *= scaling;
      v1 = 2 * pr + 1 < rank ? v1 * scaling : 0.0f;
    }
    reinterpret_cast<uint32_t*>(u + (int64_t)row * kLuPitch)[pr] = LuMma<T>::pack(v0, v1);
  }
  cluster_sync_all();  // no block leaves while others may still read its sums
}

template <typename T, typename AT>
int lora_u_split_t(const void* x, int64_t M, int64_t K, const void* a, int rank, float scaling, void* u,
                   cudaStream_t st) {
  auto kern = rank <= 16 ? lora_u_split_kernel<T, AT, 2>
                         : rank <= 32 ? lora_u_split_kernel<T, AT, 4> : lora_u_split_kernel<T, AT, 8>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kLoraUSplitBlocks);
  cfg.blockDim = dim3(32 * kLsWarps);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kLoraUSplitBlocks;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<const T*>(x), static_cast<const AT*>(a),
                                           static_cast<T*>(u), (int)M, K, rank, scaling);
  LQ_REQUIRE(e == cudaSuccess, LQ_ECUDA, "lora_u_split_kernel launch: %s", cudaGetErrorString(e));
  return launched("lora_u_split_kernel");
}

template <typename T, typename AT>
int lora_u_t(const void* x, int64_t M, int64_t K, const void* a, int rank, float scaling, void* u, cudaStream_t st,
             int max_blocks) {
  if (M <= 16) return lora_u_split_t<T, AT>(x, M, K, a, rank, scaling, u, st);
  const int64_t tiles = (M + 15) / 16;
  const dim3 grid((unsigned)(max_blocks > 0 && max_blocks < tiles ? max_blocks : tiles));
  const T* xp = static_cast<const T*>(x);
  const AT* ap = static_cast<const AT*>(a);
  T* up = static_cast<T*>(u);
  auto kern = rank <= 16 ? lora_u_kernel<T, AT, 2> : rank <= 32 ? lora_u_kernel<T, AT, 4> : lora_u_kernel<T, AT, 8>;
  const cudaError_t e = launch_pdl(kern, grid, dim3(32 * kLuWarps), 0, st, xp, ap, up, M, K, rank, scaling);
  LQ_REQUIRE(e == cudaSuccess, LQ_ECUDA, "lora_u_kernel launch: %s", cudaGetErrorString(e));
  return launched("lora_u_kernel");
}

}  // namespace

// lq_lora_u on at most max_blocks blocks (<= 0: one per 16-token tile), each
// looping over its tiles.  A kernel queued behind it cannot share an SM with
// these blocks when it takes a whole SM's shared memory; on fewer SMs the
// down-projection takes longer but leaves the rest of the machine to that
// kernel's first tiles.
int lora_u_launch(const void* x, int act_dtype, int64_t M, int64_t K, const void* lora_a, int a_dtype, int64_t rank,
                  float scaling, void* u, void* stream, int max_blocks) {
  LQ_REQUIRE(M >= 0 && M < (1LL << 31) && K >= 0 && K < (1LL << 31), LQ_EINVAL, "bad size");
  if (M == 0) return LQ_OK;
  LQ_REQUIRE(K % 64 == 0 && K > 0, LQ_EINVAL, "lora_u needs in_features %% 64 == 0 (got %lld)", (long long)K);
  LQ_REQUIRE(rank >= 1 && rank <= kLuPitch, LQ_ERANGE, "LoRA rank %lld outside [1, 64]", (long long)rank);
  LQ_REQUIRE(x && lora_a && u, LQ_EINVAL, "NULL pointer");
  LQ_REQUIRE(aligned16(x) && aligned16(lora_a) && reinterpret_cast<uintptr_t>(u) % 4 == 0, LQ_EALIGN,
             "x and lora_a must be 16-byte aligned, u 4-byte aligned");
  LQ_REQUIRE(a_dtype == LQ_F32 || a_dtype == act_dtype, LQ_EDTYPE, "lora_A must be fp32 or the activation dtype");
  cudaStream_t st = as_stream(stream);
  if (act_dtype == LQ_F16)
    return a_dtype == LQ_F32 ? lora_u_t<__half, float>(x, M, K, lora_a, (int)rank, scaling, u, st, max_blocks)
                             : lora_u_t<__half, __half>(x, M, K, lora_a, (int)rank, scaling, u, st, max_blocks);
  if (act_dtype == LQ_BF16)
    return a_dtype == LQ_F32 ? lora_u_t<__nv_bfloat16, float>(x, M, K, lora_a, (int)rank, scaling, u, st, max_blocks)
                             : lora_u_t<__nv_bfloat16, __nv_bfloat16>(x, M, K, lora_a, (int)rank, scaling, u, st, max_blocks);
  set_error("lora_u: activations must be fp16 or bf16 (got dtype %d)", act_dtype);
  return LQ_EDTYPE;
}

}  // namespace lq

extern "C" int lq_lora_u(const void* x, int act_dtype, int64_t M, int64_t K, const void* lora_a, int a_dtype,
                         int64_t rank, float scaling, void* u, void* stream) {
  return lq::lora_u_launch(x, act_dtype, M, K, lora_a, a_dtype, rank, scaling, u, stream, 0);
}
