// lq_w4a16.cu -- QuantizedLinear W4A16 forward on the 5th-generation tensor cores.
//
// y[M, N] = x[M, K] @ W^T + bias, W = (q - zero) * scale per group of the K
// dim (core/quantizer.py:262-280 dequantizes the whole weight to fp32 and
// calls F.linear; here the dequantization is fused into the GEMM).
//
// Tile = 128 weight rows x BT tokens ("swap AB"): the dequantized weights are
// the MMA's A operand and live in tensor memory, the activations are the B
// operand (TMA, 128-byte swizzle, K-major), the fp32 accumulator D[128, BT]
// is in tensor memory.  Warp roles (608 threads):
//   warp 0       activation producer: one TMA tile per stage into the
//                activation ring (S stages, refilled when the stage's MMAs
//                have completed);
//   warp 18      weight producer: packed 4-bit weight tile + (zero, scale)
//                pairs per stage into the weight ring (SW >= S stages,
//                refilled once the dequant warps have read the slot);
//   warp 1       allocates tensor memory, one lane issues tcgen05.mma
//                (4 x K=16 per 64-wide K step) and tcgen05.commit;
//   warps 2..17  dequantize, in two groups of eight taking alternate stages:
//                thread = one weight row and half of the K step, 32 codes
//                per 64-wide half -> 16 packed fp16/bf16 pairs -> tcgen05.st
//                into its half of the stage's A slot; afterwards all sixteen
//                are the epilogue (tcgen05.ld of the accumulator, + bias,
//                convert, store y).
// Warp w may only touch tensor-memory lanes 32*(w%4)..+31, so in each group
// warps 2..5 (10..13) and 6..9 (14..17) own weight rows 64..95, 96..127,
// 0..31, 32..63 of the tile.
//
// Every mbarrier wait is bounded; on timeout the kernel records an error
// code in *err (when given), drains its outstanding copies (bounded), frees
// its tensor memory and returns.
#include "lq_common.cuh"
#include "lq_tma.cuh"

#include <initializer_list>

namespace lq {
// lq_lora.cu: lq_lora_u on at most max_blocks blocks (<= 0: no limit)
int lora_u_launch(const void* x, int act_dtype, int64_t M, int64_t K, const void* lora_a, int a_dtype, int64_t rank,
                  float scaling, void* u, void* stream, int max_blocks);
}  // namespace lq

namespace lq {
namespace {

constexpr int kBK = 64;           // K per stage (128 bytes of fp16)
constexpr int kRows = 128;        // weight rows per tile (UMMA M)
constexpr int kWStage = kRows * kBK / 2;  // packed codes per stage: 4 KB
constexpr int kSStage = kRows * 4;        // (zero, scale) pairs per stage: 512 B
constexpr int kAcol = 256;        // first TMEM column of the A slots
constexpr uint32_t kTmemCols = 512;

// ---- tensor-core PTX wrappers ----------------------------------------------
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* b) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(b))
               : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t addr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(addr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t addr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(addr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory descriptor of a K-major, 128-byte-swizzled tile (rows of 128
// bytes, 8-row groups 1024 bytes apart), sm100 format.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);  // start address
  d |= (uint64_t)1 << 16;                   // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;         // stride byte offset
  d |= (uint64_t)1 << 46;                   // descriptor version (sm100)
  d |= (uint64_t)2 << 61;                   // SWIZZLE_128B
  return d;
}

// kind::f16 instruction descriptor: D fp32, A/B fp16 (fmt 0) or bf16 (fmt 1),
// both K-major, M = 128, N = BT.
__host__ __device__ constexpr uint32_t make_idesc(int fmt, int bt) {
  return (1u << 4) | ((uint32_t)fmt << 7) | ((uint32_t)fmt << 10) | ((uint32_t)(bt >> 3) << 17) |
         ((uint32_t)(kRows >> 4) << 24);
}

template <typename T> struct Act;
template <> struct Act<__half> {
  static constexpr int fmt = 0;
  static constexpr uint32_t magic = 0x64006400u;  // fp16 1024.0 in both halves
  __device__ __forceinline__ static uint32_t mul2(uint32_t v, uint32_t s) {
    __half2 h = __hmul2(*reinterpret_cast<__half2*>(&v), *reinterpret_cast<__half2*>(&s));
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static uint32_t sub_mul(uint32_t v, uint32_t zb, uint32_t s) {
    __half2 h = __hsub2(*reinterpret_cast<__half2*>(&v), *reinterpret_cast<__half2*>(&zb));
    h = __hmul2(h, *reinterpret_cast<__half2*>(&s));
    return *reinterpret_cast<uint32_t*>(&h);
  }
};
template <> struct Act<__nv_bfloat16> {
  static constexpr int fmt = 1;
  static constexpr uint32_t magic = 0x43004300u;  // bf16 128.0 in both halves
  __device__ __forceinline__ static uint32_t mul2(uint32_t v, uint32_t s) {
    __nv_bfloat162 h = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&v), *reinterpret_cast<__nv_bfloat162*>(&s));
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static uint32_t sub_mul(uint32_t v, uint32_t zb, uint32_t s) {
    __nv_bfloat162 h = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&v), *reinterpret_cast<__nv_bfloat162*>(&zb));
    h = __hmul2(h, *reinterpret_cast<__nv_bfloat162*>(&s));
    return *reinterpret_cast<uint32_t*>(&h);
  }
};

struct W4Args {
  int M, N, K, group, n_kb, n_groups;
  int kb_shift;  // log2(group / kBK) when that is a power of two, else -1
  // 1: launched right behind the kernel that writes u (lq_nf4_qlora_forward),
  // so only u's load waits for it; 0: every thread waits before its first
  // global access (any predecessor)
  int u_only_wait;
};

// The LoRA term of QLoRALinear.forward fused into the base product
// (qlora.py:306-312): y += u @ b^T with u = scaling * x @ lora_A^T [M, r]
// (computed by the caller; padded to 64 columns of zeros for the tensor-core
// path) and b = lora_B [N, r], both in the activation dtype.  r = 0: none.
struct LoraArgs {
  const void* u = nullptr;
  const void* b = nullptr;
  int r = 0;
  int u_only_wait = 0;  // see W4Args
};

inline int kb_shift_of(int group) {
  const int r = group / kBK;
  return (r & (r - 1)) == 0 ? __builtin_ctz(r) : -1;
}

// group index of K step kb (group is a multiple of kBK)
__device__ __forceinline__ int group_of(const W4Args& a, int kb) {
  return a.kb_shift >= 0 ? kb >> a.kb_shift : (kb * kBK) / a.group;
}

// NF4 weights (QLoRALinear): code byte b = elements 2i (low nibble) and
// 2i+1 (high nibble) -> the pair (round_T(NF4[lo]), round_T(NF4[hi])).  The
// 256-entry table is stored C times (C = 32 or 16), entry b of copy r at word
// C b + r; lane l reads copy l % C, so with 32 copies 32 independent lookups
// never share a bank (with 16, lanes l and l + 16 meet when their entries
// differ and have equal parity, for half the table's size).  tmp holds the
// 256 pairs while the copies are written.  Every thread of the block calls
// this (it synchronizes).
constexpr int kPairLutWords = 256 * 32;
template <typename T, int C = 32>
__device__ __forceinline__ void build_pair_lut(uint32_t* lut, uint32_t* tmp) {
  for (int b = threadIdx.x; b < 256; b += blockDim.x) {
    union {
      T h[2];
      uint32_t u;
    } pr;
    pr.h[0] = Ty<T>::from_f(Ty<T>::round(kNF4[b & 15]));
    pr.h[1] = Ty<T>::from_f(Ty<T>::round(kNF4[b >> 4]));
    tmp[b] = pr.u;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 256 * C / 4; i += blockDim.x) {
    const uint32_t v = tmp[(4 * i) / C];  // words 4i..4i+3 are copies of entry 4i / C
    reinterpret_cast<uint4*>(lut)[i] = make_uint4(v, v, v, v);
  }
}

// Byte offset of the table word for byte b (0..3) of w, in copy lane4 / 4
// (lane4 = 4 * (lane % C)).
template <int C = 32>
__device__ __forceinline__ uint32_t pair_lut_off(uint32_t w, int b, uint32_t lane4) {
  constexpr int SH = C == 32 ? 7 : 6;  // log2 of the entry stride in bytes
  constexpr uint32_t MASK = 255u << SH;
  const uint32_t off = (b == 0 ? (w << SH) : (w >> (8 * b - SH))) & MASK;
  return off | lane4;
}

// Block: activation producer warp, MMA warp, kDG groups of 8 dequant /
// epilogue warps, weight producer warp.  Group g dequantizes the stages g,
// g + kDG, ...: one warp's per-stage chain (barrier waits, shared loads,
// conversion, tcgen05.st and its wait, arrive) is latency- not issue-bound,
// so two groups keep two stages in flight.
constexpr int kDG = 2;
constexpr int kW4Threads = 64 + 256 * kDG + 32;
constexpr int kWProdWarp = kW4Threads / 32 - 1;

// A stage holds WK 64-wide K halves (WK = 2: 128 K per stage), so the
// per-stage barrier round trips and MMA-thread bookkeeping -- which pace the
// pipeline, not the tensor cores -- are paid once per 128 K.
// The weights (packed codes + (zero, scale) pairs) have a ring of their own,
// SW stages deep (what shared memory leaves, at most 8): a slot is refilled
// once the dequant warps are done with it, not when the MMA that used the
// stage completes, so a stage's weights are requested up to SW stages before
// its dequantization instead of S - 1 MMA steps before (with the weights
// arriving late, the dequant warps waited on them: 17 % of the kernel time).
template <typename T, int BT, int S, bool NF, int WK>
struct Smem {
  static constexpr int kXh = BT * kBK * 2;  // activation bytes of one 64-wide half
  static constexpr int kX = WK * kXh;       // activation tile bytes per stage
  static constexpr int kWS = WK * (kWStage + kSStage);  // weight + pair bytes per stage
  // NF4 table copies: 16 for the wide tiles with 128-wide stages (room for
  // three stages), 32 otherwise
  static constexpr int kLutC = (NF && BT > 128 && WK == 2) ? 16 : 32;
  static constexpr int kLutBytes = NF ? 256 * kLutC * 4 : 0;
  static constexpr int kRest = (NF ? kLutBytes + 1024 : 0) + 2048;  // table, barriers, slack
  // 226 KB: a block's opt-in limit is 1 KB under the SM's 227 KB (a
  // 231648-byte layout failed cudaFuncSetAttribute, 231168 bytes launched)
  static constexpr int kBudget = 226 * 1024;
  static constexpr int kFit = (kBudget - S * kX - kRest) / kWS;
  static constexpr int SW = kFit > 8 ? 8 : kFit;
  static constexpr int off_x = 0;
  static constexpr int off_w = off_x + S * kX;                  // [SW][WK] weight halves
  static constexpr int off_s = off_w + SW * WK * kWStage;       // [SW][WK] pair halves
  static constexpr int off_lut = off_s + SW * WK * kSStage;     // NF4 pair table (NF only)
  static constexpr int off_tmp = off_lut + kLutBytes;
  static constexpr int off_bar = off_tmp + (NF ? 1024 : 0);
  // barriers: full_x[S], a_full[S], empty[S], full_w[SW], w_empty[SW], acc_full
  static constexpr int n_bar = 3 * S + 2 * SW + 1;
  static constexpr int off_tmem = off_bar + n_bar * 8;
  static constexpr int bytes = off_tmem + 16 + 1024;  // + alignment slack
};

template <typename T, int BT, int S, bool NF, int WK>
__global__ void __launch_bounds__(kW4Threads, 1) w4a16_kernel(const __grid_constant__ CUtensorMap tmap_x,
                                                       const __grid_constant__ CUtensorMap tmap_u,
                                                       const uint8_t* __restrict__ packed,
                                                       const float* __restrict__ bias,
                                                       T* __restrict__ y, W4Args a,
                                                       const T* __restrict__ lora_b, int lora_r,
                                                       int* __restrict__ err) {
  using L = Smem<T, BT, S, NF, WK>;
  constexpr int SC = WK * (kBK / 2);  // tensor-memory columns of one stage's A slot
  constexpr int SW = L::SW;           // weight-ring stages
  static_assert(BT % 16 == 0 && BT <= kAcol && kAcol + S * SC <= (int)kTmemCols,
                "accumulator and A slots must fit tensor memory without overlap");
  static_assert(L::bytes <= L::kBudget, "shared memory per CTA");
  static_assert(SW >= S, "the weight ring is at least as deep as the activation ring");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::off_bar);
  uint64_t* full_x = bars;
  uint64_t* a_full = bars + S;
  uint64_t* empty = bars + 2 * S;
  uint64_t* full_w = bars + 3 * S;
  uint64_t* w_empty = bars + 3 * S + SW;
  uint64_t* acc_full = bars + 3 * S + 2 * SW;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::off_tmem);
  __shared__ int s_err;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = blockIdx.x;       // weight-row tile
  const int m0 = blockIdx.y * BT;  // first token of the tile
  // the base product's K steps, then (LoRA) one more whose A operand is
  // lora_B's 128 rows of the tile and whose B operand is u (zero past r)
  const int n_main = a.n_kb / WK;
  const int n_steps = n_main + (lora_r > 0 ? 1 : 0);
  const uint8_t* wtile = packed + (size_t)nt * a.n_kb * kWStage;
  const uint8_t* stile = packed + (size_t)(a.N / kRows) * a.n_kb * kWStage +
                         (size_t)nt * a.n_groups * kSStage;

  if (threadIdx.x == 0) {
    s_err = 0;
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_x[i], 1);
      mbar_init(&a_full[i], 8);  // one arrival per dequant warp
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < SW; ++i) {
      mbar_init(&full_w[i], 1);
      mbar_init(&w_empty[i], 8);  // one arrival per dequant warp, once it has read the slot
    }
    mbar_init(acc_full, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if constexpr (NF) {
    build_pair_lut<T, L::kLutC>(reinterpret_cast<uint32_t*>(smem + L::off_lut), reinterpret_cast<uint32_t*>(smem + L::off_tmp));
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // With the LoRA term the kernel is launched as a programmatic dependent of
  // the u kernel: the set-up above overlaps that kernel's tail, and no thread
  // touches global memory before the previous kernel is complete (a no-op
  // after an ordinary launch) -- or, right behind lq_lora_u, whose only
  // output is u, just the load of u waits (the base product runs meanwhile).
  if (!a.u_only_wait) pdl_wait();

  if (warp == 0) {
    // ---------------- activation producer ----------------
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_x)) : "memory");
      if (lora_r > 0) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_u)) : "memory");
      int issued = 0;
      for (int i = 0; i < n_steps; ++i) {
        const int s = i % S;
        if (i >= S && !mbar_wait(&empty[s], ((i / S) - 1) & 1)) { s_err = 1; break; }
        if (s_err) break;
        mbar_expect_tx(&full_x[s], L::kX);
#pragma unroll
        for (int hk = 0; hk < WK; ++hk) {
          if (i < n_main)
            tma_load_2d(smem + L::off_x + s * L::kX + hk * L::kXh, &tmap_x, (i * WK + hk) * kBK, m0, &full_x[s]);
          else {  // u has 64 columns: the second half of a 128-wide stage is all fill (zeros)
            if (hk == 0 && a.u_only_wait) pdl_wait();
            tma_load_2d(smem + L::off_x + s * L::kX + hk * L::kXh, &tmap_u, hk * kBK, m0, &full_x[s]);
          }
        }
        issued = i + 1;
      }
      if (s_err) {
        // drain: wait (bounded) for every stage this thread may still have in flight
        for (int i = (issued > S ? issued - S : 0); i < issued; ++i) mbar_wait(&full_x[i % S], (i / S) & 1);
      }
    }
  } else if (warp == kWProdWarp) {
    // ---------------- weight producer ----------------
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < n_steps; ++i) {
        const int sw = i % SW;
        if (i >= SW && !mbar_wait(&w_empty[sw], ((i / SW) - 1) & 1)) { s_err = 5; break; }
        if (s_err) break;
        if (i == n_main) {
          // LoRA step: the tile's 128 rows of lora_B (r values each) into the code slot
          const uint32_t nb = (uint32_t)(kRows * lora_r * (int)sizeof(T));
          mbar_expect_tx(&full_w[sw], nb);
          bulk_load(smem + L::off_w + sw * WK * kWStage, lora_b + (size_t)nt * kRows * lora_r, nb, &full_w[sw]);
          issued = i + 1;
          continue;
        }
        mbar_expect_tx(&full_w[sw], WK * (kWStage + kSStage));
        // the WK weight halves of a step are adjacent in the packed layout
        bulk_load(smem + L::off_w + sw * WK * kWStage, wtile + (size_t)i * WK * kWStage, WK * kWStage, &full_w[sw]);
#pragma unroll
        for (int hk = 0; hk < WK; ++hk) {
          const int g = group_of(a, i * WK + hk);
          bulk_load(smem + L::off_s + (sw * WK + hk) * kSStage, stile + (size_t)g * kSStage, kSStage, &full_w[sw]);
        }
        issued = i + 1;
      }
      if (s_err) {
        for (int i = (issued > SW ? issued - SW : 0); i < issued; ++i) mbar_wait(&full_w[i % SW], (i / SW) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    // 128-wide stages: one wait per stage, a_full completes only after the
    // dequant warps have written the A slot AND (warp 2 waits on it first) the
    // activations landed; 64-wide stages wait on the activations directly
    bool issued_any = false;
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc(Act<T>::fmt, BT);
      for (int i = 0; i < n_steps; ++i) {
        const int s = i % S;
        const uint32_t ph = (i / S) & 1;
        if ((WK == 1 && !mbar_wait(&full_x[s], ph)) || !mbar_wait(&a_full[s], ph)) { s_err = 2; break; }
        tc_fence_after();
        const uint32_t xs = smem_u32(smem + L::off_x + s * L::kX);
        const uint32_t acol0 = tmem + kAcol + s * SC;
#pragma unroll
        for (int kk = 0; kk < WK * (kBK / 16); ++kk) {
          const uint64_t bdesc = sw128_desc(xs + (kk >> 2) * L::kXh + (kk & 3) * 32);
          tc_mma(tmem, acol0 + kk * 8, bdesc, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(&empty[s]);  // frees the activation stage and the A slot
        issued_any = true;
      }
      if (issued_any) tc_commit(acc_full);
      if (s_err && issued_any) mbar_wait(acc_full, 0);  // MMAs in flight must finish before dealloc
    }
    __syncwarp();
  } else {
    // ---------------- dequantization (warps 2..), then epilogue ----------------
    // kDG groups of 8 warps; group grp takes the stages grp, grp + kDG, ...
    const int dw = warp - 2;
    const int grp = dw >> 3, wi = dw & 7;
    const int q = warp & 3;          // tensor-memory lane quarter
    const int h = wi >> 2;           // half of each 64-wide K half (A slot columns 16h..16h+15)
    const int row = q * 32 + lane;   // weight row within the tile
    // the row's bias, requested now and added in the epilogue
    const float b = bias ? __ldg(&bias[nt * kRows + row]) : 0.0f;
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
    const uint32_t sbase = smem_u32(smem);
    bool ok = true;
    for (int i = grp; i < n_steps && ok; i += kDG) {
      const int s = i % S;
      const uint32_t ph = (i / S) & 1;
      const int sw = i % SW;
      if (!mbar_wait_warp(&full_w[sw], (i / SW) & 1)) { ok = false; break; }
      if (i >= S && !mbar_wait_warp(&empty[s], ph ^ 1)) { ok = false; break; }
      if (i == n_main) {
        // LoRA step: A = lora_B[row, hk*64 + 32h + 0..31] (zero past r)
        const uint32_t brow = sbase + L::off_w + sw * WK * kWStage + (uint32_t)(row * lora_r * (int)sizeof(T));
#pragma unroll
        for (int hk = 0; hk < WK; ++hk) {
          uint32_t r[16];
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const int col = hk * kBK + 32 * h + 2 * c;
            r[c] = col < lora_r ? lds_b32(brow + col * (int)sizeof(T)) : 0u;
          }
          tmem_st16(lane_base + kAcol + s * SC + hk * (kBK / 2) + 16 * h, r);
        }
      } else {
#pragma unroll
      for (int hk = 0; hk < WK; ++hk) {
        // this warp's half of the row's codes: words 4h..4h+3 (k = 32h..32h+31)
        const uint4 cw = lds_v4(sbase + L::off_w + (sw * WK + hk) * kWStage + row * 32 + 16 * h);
        const uint32_t zs = lds_b32(sbase + L::off_s + (sw * WK + hk) * kSStage + row * 4);
        // zs = (zero_b, scale) as a T pair; broadcast each half to both halves
        const uint32_t zb = __byte_perm(zs, zs, 0x1010);
        const uint32_t sc = __byte_perm(zs, zs, 0x3232);
        const uint32_t w[4] = {cw.x, cw.y, cw.z, cw.w};
        uint32_t r[16];
        if constexpr (NF) {
          // byte c = k pair (2c, 2c+1) -> table pair * scale = round_T(NF4 * scale)
          const uint32_t lb = sbase + L::off_lut;
          const uint32_t l4 = (uint32_t)(lane % L::kLutC) << 2;
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const uint32_t pv = lds_b32(lb + pair_lut_off<L::kLutC>(w[c >> 2], c & 3, l4));
            r[c] = Act<T>::mul2(pv, sc);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
#pragma unroll
            for (int p = 0; p < 4; ++p) {
              // nibbles (4p, 16+4p) of word j are k = 8j+2p (low half), 8j+2p+1 (high half)
              const uint32_t v = ((w[j] >> (4 * p)) & 0x000F000Fu) | Act<T>::magic;
              r[j * 4 + p] = Act<T>::sub_mul(v, zb, sc);
            }
          }
        }
        tmem_st16(lane_base + kAcol + s * SC + hk * (kBK / 2) + 16 * h, r);
      }
      }
      tmem_wait_st();
      tc_fence_before();
      // 128-wide stages: warp 2 also waits for the stage's activations, so
      // a_full stands for both and the MMA thread waits once per stage
      if (WK == 2 && wi == 0 && !mbar_wait_warp(&full_x[s], ph)) { ok = false; break; }
      // one elected arrival per warp once every lane's store has landed; the
      // warp has read its weights too, so the weight slot (needed again SW >= S
      // stages later) is released in the same step
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&w_empty[sw]);
        mbar_arrive(&a_full[s]);
      }
    }
    if (!ok) s_err = 3;
    // epilogue: accumulator rows = weight rows (this thread's row), columns = tokens
    if (ok && mbar_wait_warp(acc_full, 0)) {
      tc_fence_after();
      const int n = nt * kRows + row;
#pragma unroll 1
      for (int c = 32 * (dw >> 2); c < BT; c += 64 * kDG) {
        uint32_t v[32];
        tmem_ld32(lane_base + c, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int m = m0 + c + j;
          if (m < a.M) y[(size_t)m * a.N + n] = Ty<T>::from_f(__fadd_rn(__uint_as_float(v[j]), b));
        }
      }
    } else if (ok) {
      s_err = 4;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
  if (threadIdx.x == 0 && s_err && err) atomicExch(err, s_err);
}

// ---------------------------------------------------------------------------
// Small M (M <= 8 tokens): the forward is a weight-streaming GEMV, bound by
// HBM; a 128 x BT tensor-memory tile would sit mostly idle.  It runs
// mma.sync.m16n8k16 (f32 accumulate) with the weights as the A operand and
// one 8-token B tile, on a layout of the codes of its own that the pack
// kernels append to the operand ("GEMV records", gv_record_bytes):
//
//   [N/16 slabs][groups][steps of the group: 32 lanes x 4 words][16 pairs],
//   lane L = 4 g + c owns the 16 bytes of its A fragments: word t holds rows
//   (g, g + 8) x k (4t .. 4t+3) of the lane's 16-wide k range 16c .. 16c+15
//   of the 64-wide step, as
//     INT4: bits 0-3 / 16-19   row g,   k 4t, 4t+1     (a0)
//           bits 4-7 / 20-23   row g+8, k 4t, 4t+1     (a1)
//           bits 8-11 / 24-27  row g,   k 4t+2, 4t+3   (a2)
//           bits 12-15 / 28-31 row g+8, k 4t+2, 4t+3   (a3)
//     NF4:  byte b = the (low, high) nibble pair of fragment a_b;
//   then the slab's 16 (magic + zero, scale) pairs (NF4: (0, block scale)).
//   The MMA's k slots (2c, 2c+1, 2c+8, 2c+9) of step t are these k values,
//   for the weights and the activations alike, so each lane's activations are
//   16 contiguous halves (two 16-byte loads) and each lane reads exactly its
//   16 bytes of codes (one shared load, no broadcast).
//
// INT4: a fragment is (code | magic) with one LOP3 -- 1024 + q (fp16, bits
// 0-3), 1024 + 16 q (fp16, bits 4-7: rows g + 8), 128 + q (bf16, after a
// shift) -- and the zero point is not subtracted per weight: with S = sum of
// the group's activations (formed once per block), the group contributes
// s * (f D - (o + z) S) to the output, (f, o) = (1, magic) or (1/16, 64),
// D = the MMA sum of the fragments over the group's steps.  NF4: the
// fragment is the table pair of the code byte, the block scale multiplies D.
// The kernel itself (w4a16_gemv_kernel) is described at its definition.
// ---------------------------------------------------------------------------
template <typename T> struct MmaOp;
template <> struct MmaOp<__half> {
  __device__ __forceinline__ static void mma(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t sub2(uint32_t v, uint32_t z) {
    __half2 h = __hsub2(*reinterpret_cast<__half2*>(&v), *reinterpret_cast<__half2*>(&z));
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static float hi_f(uint32_t pair) {
    return __half2float(__ushort_as_half((unsigned short)(pair >> 16)));
  }
  __device__ __forceinline__ static float lo_f(uint32_t pair) {
    return __half2float(__ushort_as_half((unsigned short)(pair & 0xFFFFu)));
  }
};
template <> struct MmaOp<__nv_bfloat16> {
  __device__ __forceinline__ static void mma(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t sub2(uint32_t v, uint32_t z) {
    __nv_bfloat162 h = __hsub2(*reinterpret_cast<__nv_bfloat162*>(&v), *reinterpret_cast<__nv_bfloat162*>(&z));
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static float hi_f(uint32_t pair) { return __uint_as_float(pair & 0xFFFF0000u); }
  __device__ __forceinline__ static float lo_f(uint32_t pair) { return __uint_as_float(pair << 16); }
};



// Byte offset of the GEMV records in the packed operand (after the tile codes
// and the (zero, scale) pairs of n_pairs groups per row).
__host__ __device__ inline int64_t gemv_codes_off(int64_t N, int64_t K, int64_t pairs_per_row) {
  return N * K / 2 + N * pairs_per_row * 4;
}
// GEMV record of one (16-row slab, group): the group's K steps of codes (512
// bytes each, lane-major) followed by the slab's 16 (zero, scale) pairs
// (64 bytes).  Records are stored slab-major ([slab][group]): a slab's whole
// K range is one run of memory, fetched in a few large bulk copies.  (NF4:
// 64-wide groups.)
__host__ __device__ inline int64_t gv_record_bytes(int64_t group) { return group / kBK * 512 + 64; }

// word i (0..3, a compile-time constant after unrolling) of v
__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

template <typename T> struct GvInt4;
template <> struct GvInt4<__half> {
  // fragments a0..a3 of one code word
  __device__ __forceinline__ static void frag(uint32_t w, uint32_t (&a)[4]) {
    const uint32_t w8 = w >> 8;
    a[0] = (w & 0x000F000Fu) | 0x64006400u;   // 1024 + q
    a[1] = (w & 0x00F000F0u) | 0x64006400u;   // 1024 + 16 q
    a[2] = (w8 & 0x000F000Fu) | 0x64006400u;
    a[3] = (w8 & 0x00F000F0u) | 0x64006400u;
  }
  // (f, -(o + z)) of rows g and g + 8 from zb = magic + z
  __device__ __forceinline__ static void fold(float zb, bool hi_row, float& f, float& c) {
    f = hi_row ? 0.0625f : 1.0f;
    c = hi_row ? -(zb - 960.0f) : -zb;
  }
};
template <> struct GvInt4<__nv_bfloat16> {
  __device__ __forceinline__ static void frag(uint32_t w, uint32_t (&a)[4]) {
    a[0] = (w & 0x000F000Fu) | 0x43004300u;   // 128 + q
    a[1] = ((w >> 4) & 0x000F000Fu) | 0x43004300u;
    a[2] = ((w >> 8) & 0x000F000Fu) | 0x43004300u;
    a[3] = ((w >> 12) & 0x000F000Fu) | 0x43004300u;
  }
  __device__ __forceinline__ static void fold(float zb, bool, float& f, float& c) {
    f = 1.0f;
    c = -zb;
  }
};

// Set a kernel's dynamic shared-memory limit once per device.
template <typename Kern>
int set_smem_once(Kern kern, int smem_bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = 1ull << (dev & 63);  // one bit per device
  if (!(done.load() & bit)) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    LQ_REQUIRE(e == cudaSuccess, LQ_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    done.fetch_or(bit);
  }
  return LQ_OK;
}

// Persistent streaming GEMV.  One block per SM owns the slabs b, b + grid,
// ...; their records stream through a STAGES-deep shared-memory ring in
// chunks of CG groups: one bulk copy of ~32 KB per chunk, issued by a
// producer warp that refills a slot once every consumer warp has released
// it (full / empty mbarriers per slot), so up to ~200 KB per SM are in
// flight.  The 16 consumer warps split each chunk's groups and never wait
// for one another: a warp stores its share of a slab (fp32, in one of two
// buffers by slab parity) and the last of the 16 to do so adds the shares
// and writes the slab's outputs.  With XS the activations (M rows of K
// halves, at most 136 KB) are copied once into shared memory; otherwise the
// lanes read them from global memory (L2).  For INT4 the block first forms S[group][token] =
// the group's activation sums (fp32), which fold the zero points: a group adds
// s (f D - (o + z) S) to its rows' outputs, D the MMA sum of the (o + q)
// fragments.  The LoRA term is one more MMA pass per slab, lora_B's rows as A
// and u as B.
constexpr int kGvWarps = 16;      // consumer warps; one producer warp more
constexpr int kGvMaxStages = 16;
constexpr int kGvSmemMax = 227 * 1024;
constexpr int kGvXsMax = 136 * 1024;
__host__ __device__ inline int gv_xpitch_bytes(int K) { return 2 * K + 16; }

struct GvArgs {
  int G, cg, stages;
};

template <typename T, bool NF, int NT, bool XS, int SPG>
__global__ void __launch_bounds__(32 * (kGvWarps + 1), 1) w4a16_gemv_kernel(const T* __restrict__ x,
                                                    const uint8_t* __restrict__ packed,
                                                    const float* __restrict__ bias,
                                                    T* __restrict__ y, W4Args a, GvArgs v, int* err,
                                                    const T* __restrict__ lora_u,
                                                    const T* __restrict__ lora_b, int lora_r) {
  constexpr int CH = (NT == 2 && !XS) ? 1 : 2;  // MMA chains per group and B tile
  constexpr int GP = (NF && NT == 2) ? 1 : 2;    // groups per pass
  const int G = v.G, cg = v.cg, stages = v.stages;
  const int rb = (int)gv_record_bytes(G);
  const int spg = SPG > 0 ? SPG : G / kBK;  // K steps per group
  const int n_grp = a.K / G;
  const int n_chunk = (n_grp + cg - 1) / cg;
  const int n_slab = a.N / 16;
  const int chunk_bytes = cg * rb;
  extern __shared__ __align__(128) uint8_t gv_smem[];
  uint8_t* p = gv_smem;
  uint32_t* lut = reinterpret_cast<uint32_t*>(p);  // NF: pair table (+1 KB build space)
  if (NF) p += kPairLutWords * 4 + 1024;
  float* red = reinterpret_cast<float*>(p);  // [2][warps][NT * 128] slab shares, fragment order
  p += 2 * kGvWarps * NT * 512;
  int* cnt = reinterpret_cast<int*>(p);  // [2] warps done with the buffer's slab
  int* gen = cnt + 2;                    // [2] slabs written out of the buffer
  p += 128;
  uint64_t* full = reinterpret_cast<uint64_t*>(p);  // [kGvMaxStages]
  uint64_t* empty = full + kGvMaxStages;            // [kGvMaxStages]
  uint64_t* xbar = empty + kGvMaxStages;
  p += 2 * kGvMaxStages * 8 + 128;
  float* S = reinterpret_cast<float*>(p);  // INT4: [n_grp][16 tokens]
  if (!NF) p += ((n_grp * 64 + 127) / 128) * 128;
  uint8_t* xs = p;  // XS: [M][K] halves at pitch 2 K + 16 bytes
  if (XS) p += ((a.M * gv_xpitch_bytes(a.K) + 127) / 128) * 128;
  uint8_t* ring = p;  // [stages][chunk_bytes]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool producer = warp == kGvWarps;
  const uint8_t* recs = packed + gemv_codes_off(a.N, a.K, NF ? a.n_kb : a.n_groups);
  // this block's units, in order: (slab blockIdx.x + i grid, chunk j) = unit i n_chunk + j
  const int my_slabs = blockIdx.x < n_slab ? (n_slab - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int n_units = my_slabs * n_chunk;
  auto issue = [&](int u) {
    const int slab = blockIdx.x + (u / n_chunk) * gridDim.x, ch = u % n_chunk;
    const uint32_t nb = (uint32_t)(min(cg, n_grp - ch * cg) * rb);
    const int sl = u % stages;
    mbar_expect_tx(&full[sl], nb);
    bulk_load(ring + (size_t)sl * chunk_bytes, recs + ((size_t)slab * n_grp + (size_t)ch * cg) * rb, nb, &full[sl]);
  };
  if (threadIdx.x < 4) cnt[threadIdx.x] = 0;  // and gen
  if (producer && lane == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kGvWarps);
    }
    mbar_init(xbar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (XS) {
      mbar_expect_tx(xbar, (uint32_t)(a.M * a.K * 2));
      for (int row = 0; row < a.M; ++row)
        bulk_load(xs + row * gv_xpitch_bytes(a.K), x + (size_t)row * a.K, (uint32_t)(a.K * 2), xbar);
    }
    for (int u = 0; u < stages && u < n_units; ++u) issue(u);
  }
  if constexpr (NF) build_pair_lut<T>(lut, reinterpret_cast<uint32_t*>(gv_smem + kPairLutWords * 4));
  __syncthreads();
  bool ok = XS ? mbar_wait(xbar, 0) : true;
  if constexpr (!NF) {
    // group sums of the activations: eight lanes per (group, token), each
    // adding G / 8 halves, then three shuffles (tokens past M are not read)
    const int n_items = n_grp * a.M, part = threadIdx.x & 7, per = G / 8;
    for (int base = 0; base < n_items; base += blockDim.x / 8) {
      const int it = base + (int)(threadIdx.x >> 3);
      float sum = 0.0f;
      if (it < n_items && ok) {
        const int gi = it / a.M, tok = it % a.M;
        const T* xr = XS ? reinterpret_cast<const T*>(xs + tok * gv_xpitch_bytes(a.K)) + gi * G + part * per
                         : x + (size_t)tok * a.K + gi * G + part * per;
        for (int k = 0; k < per; k += 8) {
          const uint4 q = XS ? *reinterpret_cast<const uint4*>(xr + k) : __ldg(reinterpret_cast<const uint4*>(xr + k));
          const T* h = reinterpret_cast<const T*>(&q);
#pragma unroll
          for (int e = 0; e < 8; ++e) sum += Ty<T>::to_f(h[e]);
        }
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      sum += __shfl_xor_sync(0xffffffffu, sum, 4);
      if (it < n_items && part == 0) S[(it / a.M) * 16 + it % a.M] = sum;
    }
  }
  __syncthreads();
  if (producer) {
    // refill slot u % stages for unit u once the 16 consumers released unit u - stages
    int u = stages;
    if (lane == 0) {
      for (; ok && u < n_units; ++u) {
        if (!mbar_wait(&empty[u % stages], (uint32_t)(u / stages - 1) & 1u)) {
          atomicExch(err, 5);
          break;
        }
        issue(u);
      }
      // before the block exits, every copy it issued has landed (bounded)
      const int issued = min(u, n_units);
      for (int w = max(0, issued - stages); w < issued; ++w) mbar_wait(&full[w % stages], (uint32_t)(w / stages) & 1u);
    }
    return;
  }
  const int g = lane >> 2, c = lane & 3;
  // activations of lane (g, c) in B tile j: token 8 j + g (token 0 for
  // columns past M, which are never stored), halves 16 c .. 16 c + 15 of each
  // 64-wide step
  const uint32_t xs_a = smem_u32(xs), ring_a = smem_u32(ring), lut_a = smem_u32(lut);
  uint32_t xoff[NT];  // XS: byte offset in the shared copy
  int64_t xoffg[NT];  // else: byte offset in x
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int tok = 8 * j + g < a.M ? 8 * j + g : 0;
    xoff[j] = (uint32_t)(tok * gv_xpitch_bytes(a.K) + 32 * c);
    xoffg[j] = (int64_t)tok * a.K * 2 + 32 * c;
  }
  const uint32_t lane4 = (uint32_t)lane << 2;  // NF4: the lane's copy of the pair table
  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[j][e] = 0.0f;
  int sl = 0, ch = 0, si = 0;
  uint32_t par = 0;
  float bias_r[2] = {0.0f, 0.0f};  // bias of the lane's rows of the current slab
  // LoRA: warp w < rank / 16 adds rank columns 16 w .. 16 w + 15 of every slab
  // (u . lora_B^T, one MMA per token tile).  Its lora_B fragment is requested
  // at the slab's start; u is the same for every slab and read once, at the
  // first slab's end -- right behind lq_lora_u (a.u_only_wait) only after
  // griddepcontrol.wait, so the weights stream while u is computed.
  const bool lora_w = lora_r > 0 && warp * 16 < lora_r;
  uint32_t lb_r[4] = {0u, 0u, 0u, 0u};
  uint32_t u_r[NT][2];
  bool u_ready = false;
  for (int u = 0; u < n_units; ++u) {
    if (ch == 0 && bias) {
      // requested at the slab's start, used when (if) this warp writes it out
      const int row = (blockIdx.x + si * gridDim.x) * 16 + (lane >> 2);
      bias_r[0] = __ldg(&bias[row]);
      bias_r[1] = __ldg(&bias[row + 8]);
    }
    if (ch == 0 && lora_w) {
      // A fragment: rows g, g + 8 of the slab x rank columns 2c, 2c + 8 (+1) of
      // this warp's tile (0 past the rank)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int row = (blockIdx.x + si * gridDim.x) * 16 + g + (q & 1) * 8;
        const int col = 16 * warp + 2 * c + (q >> 1) * 8;
        lb_r[q] = col < lora_r ? __ldg(reinterpret_cast<const unsigned int*>(lora_b + (size_t)row * lora_r + col)) : 0u;
      }
    }
    if (!(ok && mbar_wait(&full[sl], par))) {
      if (lane == 0) atomicExch(err, 5);
      break;
    }
    const int ng = min(cg, n_grp - ch * cg);
    const uint32_t st = ring_a + (uint32_t)(sl * chunk_bytes);
    // warp w takes the chunk's groups w, w + 16, ..., GP at a time (gl and
    // gl + 16): their MMA chains are independent, so their latencies overlap
    for (int gl = warp; gl < ng; gl += GP * kGvWarps) {
      const bool two = GP == 2 && gl + kGvWarps < ng;
      const int grp[2] = {ch * cg + gl, ch * cg + gl + (two ? kGvWarps : 0)};
      const uint32_t rec[2] = {st + (uint32_t)(gl * rb), st + (uint32_t)((gl + (two ? kGvWarps : 0)) * rb)};
      float dc[GP][NT][CH][4];
#pragma unroll
      for (int q = 0; q < GP; ++q)
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
          for (int h = 0; h < CH; ++h)
#pragma unroll
            for (int e = 0; e < 4; ++e) dc[q][j][h][e] = 0.0f;
#pragma unroll
      for (int ks = 0; ks < (SPG > 0 ? SPG : 1); ++ks)
        for (int kr = ks; kr < (SPG > 0 ? ks + 1 : spg); ++kr) {
          uint4 cw[GP];
          uint4 xv[GP][NT][2];
#pragma unroll
          for (int q = 0; q < GP; ++q) {
            cw[q] = lds_v4(rec[q] + kr * 512 + lane * 16);
            const uint32_t xk = (uint32_t)(grp[q] * G + kr * kBK) * 2u;
#pragma unroll
            for (int j = 0; j < NT; ++j) {
              if constexpr (XS) {
                xv[q][j][0] = lds_v4(xs_a + xoff[j] + xk);
                xv[q][j][1] = lds_v4(xs_a + xoff[j] + xk + 16);
              } else {
                const uint4* xp = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(x) + xoffg[j] + xk);
                xv[q][j][0] = __ldg(xp);
                xv[q][j][1] = __ldg(xp + 1);
              }
            }
          }
#pragma unroll
          for (int t = 0; t < 4; ++t)
#pragma unroll
            for (int q = 0; q < GP; ++q) {
              uint32_t af[4];
              if constexpr (NF) {
#pragma unroll
                for (int b = 0; b < 4; ++b) af[b] = lds_b32(lut_a + pair_lut_off(word_of(cw[q], t), b, lane4));
              } else {
                GvInt4<T>::frag(word_of(cw[q], t), af);
              }
#pragma unroll
              for (int j = 0; j < NT; ++j)
                MmaOp<T>::mma(dc[q][j][t % CH], af, word_of(xv[q][j][t >> 1], 2 * (t & 1)),
                              word_of(xv[q][j][t >> 1], 2 * (t & 1) + 1));
            }
        }
#pragma unroll
      for (int q = 0; q < GP; ++q) {
        if (q == 1 && !two) break;
        float d[NT][4];
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float sum = dc[q][j][0][e];
#pragma unroll
            for (int h = 1; h < CH; ++h) sum += dc[q][j][h][e];
            d[j][e] = sum;
          }
        // fold the group in: the slab's 16 (zero, scale) pairs follow its codes
        const uint32_t zs0 = lds_b32(rec[q] + spg * 512 + 4 * g);
        const uint32_t zs1 = lds_b32(rec[q] + spg * 512 + 4 * (g + 8));
        const float s0 = MmaOp<T>::hi_f(zs0), s1 = MmaOp<T>::hi_f(zs1);
        if constexpr (NF) {
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            acc[j][0] = fmaf(d[j][0], s0, acc[j][0]);
            acc[j][1] = fmaf(d[j][1], s0, acc[j][1]);
            acc[j][2] = fmaf(d[j][2], s1, acc[j][2]);
            acc[j][3] = fmaf(d[j][3], s1, acc[j][3]);
          }
        } else {
          float f0, c0, f1, c1;
          GvInt4<T>::fold(MmaOp<T>::lo_f(zs0), false, f0, c0);
          GvInt4<T>::fold(MmaOp<T>::lo_f(zs1), true, f1, c1);
          const float sf0 = s0 * f0, sc0 = s0 * c0, sf1 = s1 * f1, sc1 = s1 * c1;
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            // rows g, g + 8 x tokens 8 j + 2 c, 8 j + 2 c + 1
            const float2 sv = *reinterpret_cast<const float2*>(&S[grp[q] * 16 + 8 * j + 2 * c]);
            acc[j][0] = fmaf(d[j][0], sf0, fmaf(sv.x, sc0, acc[j][0]));
            acc[j][1] = fmaf(d[j][1], sf0, fmaf(sv.y, sc0, acc[j][1]));
            acc[j][2] = fmaf(d[j][2], sf1, fmaf(sv.x, sc1, acc[j][2]));
            acc[j][3] = fmaf(d[j][3], sf1, fmaf(sv.y, sc1, acc[j][3]));
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[sl]);  // the slot may be refilled
    if (ch == n_chunk - 1) {
      const int slab = blockIdx.x + si * gridDim.x;
      if (lora_w) {
        if (!u_ready) {
          if (a.u_only_wait) pdl_wait();
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            const T* ur = lora_u + (size_t)(8 * j + g < a.M ? 8 * j + g : 0) * kBK + 16 * warp + 2 * c;
            u_r[j][0] = *reinterpret_cast<const uint32_t*>(ur);
            u_r[j][1] = *reinterpret_cast<const uint32_t*>(ur + 8);
          }
          u_ready = true;
        }
#pragma unroll
        for (int j = 0; j < NT; ++j) MmaOp<T>::mma(acc[j], lb_r, u_r[j][0], u_r[j][1]);
      }
      // this warp's share of the slab into its slot of buffer si % 2 (free
      // once slab si - 2 is written out); the last of the 16 adds the slots
      // and writes the outputs
      const int r = si & 1;
      float* rbuf = red + r * (kGvWarps * NT * 128);
      if (si >= 2 && *reinterpret_cast<volatile int*>(&gen[r]) < (si >> 1)) {
        const uint64_t t0 = global_ns();
        for (uint32_t i = 0; *reinterpret_cast<volatile int*>(&gen[r]) < (si >> 1); ++i)
          if ((i & 63) == 63 && global_ns() - t0 > kWaitNs) {
            if (lane == 0) atomicExch(err, 5);
            break;
          }
      }
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        *reinterpret_cast<float4*>(&rbuf[(warp * NT + j) * 128 + lane * 4]) = make_float4(acc[j][0], acc[j][1], acc[j][2], acc[j][3]);
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[j][e] = 0.0f;
      }
      __threadfence_block();
      __syncwarp();
      int last = 0;
      if (lane == 0) last = atomicAdd(&cnt[r], 1) == kGvWarps - 1;
      last = __shfl_sync(0xffffffffu, last, 0);
      if (last) {
        __threadfence_block();
#pragma unroll
        for (int j = 0; j < NT; ++j) {
          float4 sum = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll 4
          for (int w = 0; w < kGvWarps; ++w) {
            const uint4 q = lds_v4(smem_u32(&rbuf[(w * NT + j) * 128 + lane * 4]));
            sum.x += __uint_as_float(q.x);
            sum.y += __uint_as_float(q.y);
            sum.z += __uint_as_float(q.z);
            sum.w += __uint_as_float(q.w);
          }
          const float vals[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int tok = 8 * j + 2 * (lane & 3) + (e & 1);
            if (tok >= a.M) continue;
            const int row = slab * 16 + (lane >> 2) + (e >= 2 ? 8 : 0);
            y[(size_t)tok * a.N + row] = Ty<T>::from_f(bias ? __fadd_rn(vals[e], bias_r[e >> 1]) : vals[e]);
          }
        }
        __syncwarp();
        if (lane == 0) {
          cnt[r] = 0;
          __threadfence_block();
          *reinterpret_cast<volatile int*>(&gen[r]) = (si >> 1) + 1;
        }
      }
      ++si;
    }
    if (++ch == n_chunk) ch = 0;
    if (++sl == stages) {
      sl = 0;
      par ^= 1u;
    }
  }
}

// Shared memory of the streaming GEMV before its ring: table (NF4), slab
// shares and counters, barriers, group sums (INT4), activations (XS).
inline int gv_fixed_smem(bool nf, bool xs, int NT, int M, int K, int G) {
  const int n_grp = K / G;
  return (nf ? kPairLutWords * 4 + 1024 : 0) + 2 * kGvWarps * NT * 512 + 128 +
         2 * kGvMaxStages * 8 + 128 + (nf ? 0 : ((n_grp * 64 + 127) / 128) * 128) +
         (xs ? ((M * gv_xpitch_bytes(K) + 127) / 128) * 128 : 0);
}

template <typename T, bool NF, int NT, bool XS, int SPG>
int launch_gemv_nt(const W4Args& a, const void* x, const void* packed, const float* bias, void* y,
                   int* err, cudaStream_t st, const LoraArgs& lo) {
  static std::atomic<uint64_t> attr_done{0};
  GvArgs v;
  v.G = NF ? kBK : a.group;
  const int rb = (int)gv_record_bytes(v.G);
  const int n_grp = a.K / v.G;
  // chunks of ~32 KB (whole groups, a multiple of the warp count), smaller
  // when that leaves under three stages
  const int fixed = gv_fixed_smem(NF, XS, NT, a.M, a.K, v.G);
  const int avail = kGvSmemMax - fixed;
  int cg = ((32768 + rb - 1) / rb + kGvWarps - 1) / kGvWarps * kGvWarps;
  if (3 * cg * rb > avail) {
    cg = avail / 3 / rb;
    if (cg >= kGvWarps) cg = cg / kGvWarps * kGvWarps;
    if (cg < 1) return 1;
  }
  if (cg > n_grp) cg = n_grp;
  v.cg = cg;
  v.stages = avail / (cg * rb);
  if (v.stages > kGvMaxStages) v.stages = kGvMaxStages;
  if (v.stages < 2) return 1;
  const int smem = fixed + v.stages * cg * rb;
  auto kern = w4a16_gemv_kernel<T, NF, NT, XS, SPG>;
  LQ_TRY(set_smem_once(kern, kGvSmemMax, attr_done));
  const int n_slab = a.N / 16;
  if (a.u_only_wait) {
    // right behind lq_lora_u (one cluster of kLoraUSplitBlocks blocks for these
    // token counts): a programmatic dependent on the SMs those leave free,
    // started before u is done
    const int sms = num_sms() - kLoraUSplitBlocks;
    const int grid = n_slab < sms ? n_slab : sms;
    const cudaError_t e = launch_pdl(kern, dim3((unsigned)grid), dim3(32 * (kGvWarps + 1)), (size_t)smem, st,
                                     static_cast<const T*>(x), static_cast<const uint8_t*>(packed), bias,
                                     static_cast<T*>(y), a, v, err, static_cast<const T*>(lo.u),
                                     static_cast<const T*>(lo.b), lo.r);
    LQ_REQUIRE(e == cudaSuccess, LQ_ECUDA, "w4a16_gemv_kernel launch: %s", cudaGetErrorString(e));
    return launched("w4a16_gemv_kernel");
  }
  const int grid = n_slab < num_sms() ? n_slab : num_sms();
  kern<<<grid, 32 * (kGvWarps + 1), smem, st>>>(static_cast<const T*>(x), static_cast<const uint8_t*>(packed), bias,
                                               static_cast<T*>(y), a, v, err, static_cast<const T*>(lo.u),
                                               static_cast<const T*>(lo.b), lo.r);
  return launched("w4a16_gemv_kernel");
}

template <typename T, bool NF, int SPG>
int launch_gemv_m(const W4Args& a, const void* x, const void* packed, const float* bias, void* y, int* err,
                  cudaStream_t st, const LoraArgs& lo, bool xs) {
  return xs ? launch_gemv_nt<T, NF, 1, true, SPG>(a, x, packed, bias, y, err, st, lo)
            : launch_gemv_nt<T, NF, 1, false, SPG>(a, x, packed, bias, y, err, st, lo);
}

// 0 = launched (or a launch error), 1 = not applicable here (more than 8
// tokens -- from 9 on the 32-token tensor-core tile measured faster --,
// groups above 256, or the shared memory leaves fewer than two ring stages)
template <typename T, bool NF>
int launch_gemv(const void* x, int M, int N, int K, int group, const void* packed, const float* bias,
                void* y, int* err, cudaStream_t st, const LoraArgs& lo) {
  W4Args a;
  a.M = M;
  a.N = N;
  a.K = K;
  a.group = group;
  a.n_kb = K / kBK;
  a.n_groups = K / group;
  a.kb_shift = kb_shift_of(group);
  a.u_only_wait = lo.r > 0 ? lo.u_only_wait : 0;
  if (M > 8 || (!NF && group > 4 * kBK)) return 1;
  // the activations are copied to shared memory when they fit and their rows
  // start on 16-byte boundaries (K is a multiple of 64)
  const bool xs = (int64_t)M * gv_xpitch_bytes(K) <= kGvXsMax && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  // K steps per group as a compile-time constant for the common groups
  // (NF4: 64; INT4: 64, 128), looped otherwise
  const int spg = NF ? 1 : group / kBK;
  if (spg == 1) return launch_gemv_m<T, NF, 1>(a, x, packed, bias, y, err, st, lo, xs);
  if constexpr (!NF) {
    if (spg == 2) return launch_gemv_m<T, NF, 2>(a, x, packed, bias, y, err, st, lo, xs);
    return launch_gemv_m<T, NF, 0>(a, x, packed, bias, y, err, st, lo, xs);
  }
  return 1;
}

// ---------------------------------------------------------------------------
// Packing: QuantizedLinear int8 codes + (scale, zero) -> kernel operand.
//   codes: [N/128][K/64][128 rows][8 words]; word j of a row holds
//          k = 8j..8j+7 with k = 8j+2p at bits 4p and k = 8j+2p+1 at bits 16+4p;
//          symmetric codes are stored biased by +8.
//   pairs: [N/128][K/group][128 rows] (zero_b, scale) in the activation type,
//          zero_b = magic + zero (+8 symmetric), magic = 1024 (fp16) / 128 (bf16).
// ---------------------------------------------------------------------------
template <typename ST>
__device__ __forceinline__ float ld_s(const void* p, int64_t i) {
  return Ty<ST>::to_f(static_cast<const ST*>(p)[i]);
}

template <typename T, typename ST>
__global__ void __launch_bounds__(256) w4a16_pack_kernel(const int8_t* __restrict__ wi,
                                                         const void* __restrict__ sc,
                                                         const void* __restrict__ zp, int N, int K,
                                                         int group, int sym,
                                                         uint8_t* __restrict__ packed) {
  const int n_kb = K / kBK, ng = K / group;
  const int64_t words = (int64_t)N * K / 8;
  uint32_t* out = reinterpret_cast<uint32_t*>(packed);
  const int bias8 = sym ? 8 : 0;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < words;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(t & 7);
    const int64_t r0 = t >> 3;  // (nt, kb, row)
    const int row = (int)(r0 % kRows);
    const int64_t r1 = r0 / kRows;
    const int kb = (int)(r1 % n_kb);
    const int nt = (int)(r1 / n_kb);
    const int n = nt * kRows + row;
    const int k0 = kb * kBK + j * 8;
    const int8_t* src = wi + (int64_t)n * K + k0;
    uint32_t w = 0;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      w |= (uint32_t)((src[2 * p] + bias8) & 15) << (4 * p);
      w |= (uint32_t)((src[2 * p + 1] + bias8) & 15) << (16 + 4 * p);
    }
    out[t] = w;
  }
  const int64_t pairs = (int64_t)N * ng;
  uint32_t* pout = reinterpret_cast<uint32_t*>(packed + (int64_t)N * K / 2);
  const float magic = (Ty<T>::code == LQ_F16) ? 1024.0f : 128.0f;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < pairs;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(t % kRows);
    const int64_t r1 = t / kRows;
    const int g = (int)(r1 % ng);
    const int nt = (int)(r1 / ng);
    const int n = nt * kRows + row;
    const float z = ld_s<ST>(zp, (int64_t)n * ng + g) + (float)bias8;
    const float s = ld_s<ST>(sc, (int64_t)n * ng + g);
    union {
      T h[2];
      uint32_t u;
    } pr;
    pr.h[0] = Ty<T>::from_f(magic + z);
    pr.h[1] = Ty<T>::from_f(s);
    pout[t] = pr.u;
  }
  // GEMV records (see gv_record_bytes): code word (slab, kb, lane 4g + c, t)
  // -> rows (16 slab + g, + 8), k = 64 kb + 16 c + 4 t + 0..3, nibble
  // positions as the GEMV reads them; then the group's 16 (zero_b, scale) pairs
  uint8_t* gbase = packed + gemv_codes_off(N, K, ng);
  const int spg = group / kBK;
  const int64_t rb = gv_record_bytes(group);
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < words;
       u += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(u & 3), L = (int)((u >> 2) & 31);
    const int64_t rest = u >> 7;
    const int kb = (int)(rest % n_kb);
    const int64_t slab = rest / n_kb;
    const int64_t n0 = slab * 16 + (L >> 2);
    const int k0 = kb * kBK + 16 * (L & 3) + 4 * t;
    const int8_t* p0 = wi + n0 * K + k0;
    const int8_t* p1 = p0 + 8 * (int64_t)K;
    auto q = [&](const int8_t* p, int i) { return (uint32_t)((p[i] + bias8) & 15); };
    uint8_t* rec = gbase + (slab * ng + kb / spg) * rb + (kb % spg) * 512;
    reinterpret_cast<uint32_t*>(rec)[L * 4 + t] =
        q(p0, 0) | (q(p0, 1) << 16) | (q(p1, 0) << 4) | (q(p1, 1) << 20) | (q(p0, 2) << 8) |
        (q(p0, 3) << 24) | (q(p1, 2) << 12) | (q(p1, 3) << 28);
  }
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < pairs;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = t / ng;
    const int g = (int)(t % ng);
    const float z = ld_s<ST>(zp, n * ng + g) + (float)bias8;
    const float sv = ld_s<ST>(sc, n * ng + g);
    union {
      T h[2];
      uint32_t u;
    } pr;
    pr.h[0] = Ty<T>::from_f(magic + z);
    pr.h[1] = Ty<T>::from_f(sv);
    reinterpret_cast<uint32_t*>(gbase + ((n / 16) * ng + g) * rb + spg * 512)[n % 16] = pr.u;
  }
}

// ---------------------------------------------------------------------------
// NF4 linear operand (QLoRALinear base weight) from the module's packed codes
// (flattened weight, element 2i in the low nibble of byte i) and its block
// scales:
//   codes: [N/128][K/64][128 rows][32 bytes] in that natural nibble order, so
//          byte c of a row's K step is the k pair (2c, 2c+1);
//   pairs: [N/128][K/64][128 rows] (0, scale) in the activation type: the
//          scale of the block holding the row's 64-element K step, restored
//          from the double quantization when given (round(round(q/127)*dq) in
//          the scales' dtype, as _dequantize_base computes it).
// ---------------------------------------------------------------------------
template <typename T, typename ST>
__global__ void __launch_bounds__(256) nf4lin_pack_kernel(const uint32_t* __restrict__ codes,
                                                          const ST* __restrict__ scales,
                                                          const ST* __restrict__ q_scales,
                                                          const ST* __restrict__ dq_scales,
                                                          int64_t dq_group, int N, int K, int group,
                                                          uint8_t* __restrict__ packed) {
  const int n_kb = K / kBK;
  const int64_t words = (int64_t)N * K / 8;
  uint32_t* out = reinterpret_cast<uint32_t*>(packed);
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < words;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(t & 7);
    const int64_t r0 = t >> 3;  // (nt, kb, row)
    const int row = (int)(r0 % kRows);
    const int64_t r1 = r0 / kRows;
    const int kb = (int)(r1 % n_kb);
    const int nt = (int)(r1 / n_kb);
    const int64_t n = (int64_t)nt * kRows + row;
    out[t] = codes[(n * K + kb * kBK + j * 8) / 8];
  }
  const int64_t pairs = (int64_t)N * n_kb;
  uint32_t* pout = reinterpret_cast<uint32_t*>(packed + (int64_t)N * K / 2);
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < pairs;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(t % kRows);
    const int64_t r1 = t / kRows;
    const int kb = (int)(r1 % n_kb);
    const int nt = (int)(r1 / n_kb);
    const int64_t n = (int64_t)nt * kRows + row;
    const int64_t g = (n * K + (int64_t)kb * kBK) / group;
    const float sv = q_scales ? tmul<ST>(tdiv<ST>(Ty<ST>::to_f(q_scales[g]), 127.0f), Ty<ST>::to_f(dq_scales[g / dq_group]))
                              : Ty<ST>::to_f(scales[g]);
    union {
      T h[2];
      uint32_t u;
    } pr;
    pr.h[0] = Ty<T>::from_f(0.0f);
    pr.h[1] = Ty<T>::from_f(sv);
    pout[t] = pr.u;
  }
  // GEMV records (64-wide groups, see gv_record_bytes): byte b of word (slab,
  // kb, lane 4g + c, t) = the code byte of fragment a_b (rows 16 slab + g, + 8;
  // k = 64 kb + 16 c + 4 t (+2)); then the step's 16 (0, scale) pairs
  const uint8_t* cb = reinterpret_cast<const uint8_t*>(codes);
  uint8_t* gbase = packed + gemv_codes_off(N, K, n_kb);
  const int64_t rb = gv_record_bytes(kBK);
  for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < words;
       u += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(u & 3), L = (int)((u >> 2) & 31);
    const int64_t rest = u >> 7;
    const int kb = (int)(rest % n_kb);
    const int64_t slab = rest / n_kb;
    const int64_t n0 = slab * 16 + (L >> 2);
    const int64_t e0 = (n0 * K + kb * kBK + 16 * (L & 3) + 4 * t) / 2;  // byte of (row g, k0, k0 + 1)
    const int64_t e1 = e0 + 4 * (int64_t)K;                                // row g + 8
    reinterpret_cast<uint32_t*>(gbase + (slab * n_kb + kb) * rb)[L * 4 + t] =
        (uint32_t)cb[e0] | ((uint32_t)cb[e1] << 8) | ((uint32_t)cb[e0 + 1] << 16) | ((uint32_t)cb[e1 + 1] << 24);
  }
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < pairs;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t n = t / n_kb;
    const int kb = (int)(t % n_kb);
    const int64_t g = (n * K + (int64_t)kb * kBK) / group;
    const float sv = q_scales ? tmul<ST>(tdiv<ST>(Ty<ST>::to_f(q_scales[g]), 127.0f), Ty<ST>::to_f(dq_scales[g / dq_group]))
                              : Ty<ST>::to_f(scales[g]);
    union {
      T h[2];
      uint32_t u;
    } pr;
    pr.h[0] = Ty<T>::from_f(0.0f);
    pr.h[1] = Ty<T>::from_f(sv);
    reinterpret_cast<uint32_t*>(gbase + ((n / 16) * n_kb + kb) * rb + 512)[n % 16] = pr.u;
  }
}

// ---- host side ---------------------------------------------------------------
// Activation tensor map: [M, K] row-major, box kBK x BT, 128-byte swizzle.
template <typename T>
int encode_x_map(CUtensorMap* map, const void* x, int M, int K, int BT) {
  EncodeTiledFn enc = encode_fn();
  LQ_REQUIRE(enc != nullptr, LQ_ECUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)BT};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, Act<T>::fmt == 0 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                   2, const_cast<void*>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  LQ_REQUIRE(r == CUDA_SUCCESS, LQ_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return LQ_OK;
}

inline W4Args w4_args(int M, int N, int K, int group) {
  W4Args a;
  a.M = M;
  a.N = N;
  a.K = K;
  a.group = group;
  a.n_kb = K / kBK;
  a.n_groups = K / group;
  a.kb_shift = kb_shift_of(group);
  a.u_only_wait = 0;
  return a;
}

template <typename T, int BT, int S, bool NF, int WK>
int launch_w4(const void* x, int M, int N, int K, int group, const void* packed, const float* bias,
              void* y, int* err, cudaStream_t st, const LoraArgs& lo) {
  using L = Smem<T, BT, S, NF, WK>;
  CUtensorMap map, umap;
  LQ_TRY(encode_x_map<T>(&map, x, M, K, BT));
  if (lo.r > 0) {
    LQ_TRY(encode_x_map<T>(&umap, lo.u, M, kBK, BT));  // u padded to 64 columns
  } else {
    umap = map;  // unused
  }
  W4Args a = w4_args(M, N, K, group);
  a.u_only_wait = lo.r > 0 ? lo.u_only_wait : 0;
  auto kern = w4a16_kernel<T, BT, S, NF, WK>;
  const int smem_bytes = L::bytes > 117 * 1024 ? L::bytes : 117 * 1024;
  static std::atomic<uint64_t> attr_done{0};
  LQ_TRY(set_smem_once(kern, smem_bytes, attr_done));
  dim3 grid(N / kRows, (M + BT - 1) / BT);
  if (lo.r > 0) {
    const cudaError_t e = launch_pdl(kern, grid, dim3(kW4Threads), smem_bytes, st, map, umap,
                                     static_cast<const uint8_t*>(packed), bias, static_cast<T*>(y), a,
                                     static_cast<const T*>(lo.b), lo.r, err);
    LQ_REQUIRE(e == cudaSuccess, LQ_ECUDA, "w4a16_kernel launch: %s", cudaGetErrorString(e));
  } else {
    kern<<<grid, kW4Threads, smem_bytes, st>>>(map, umap, static_cast<const uint8_t*>(packed), bias,
                                      static_cast<T*>(y), a, static_cast<const T*>(lo.b), lo.r, err);
  }
  return launched("w4a16_kernel");
}

// Token-tile width for M > 128: one CTA per SM runs one 128 x BT tile at a
// time, so a launch costs ceil(tiles / SMs) waves of one tile's time.  With
// 128-wide stages a tile's time grows with BT plus a part that does not (the
// weight side: loads, dequantization, pipeline fill and epilogue), measured at
// about 170 columns' worth for K = 4096 (M = 2048, N = 14336: 24.8, 26.4,
// 29.4, 32.0 us per wave at BT = 160, 192, 224, 256): take the candidate with
// the least waves x (BT + 170).  With 64-wide stages a step's cost hardly
// depends on BT (the MMA thread's bookkeeping paces it): take the widest tile
// among those with the fewest waves.
inline int pick_bt(int M, int N, std::initializer_list<int> cands, bool tensor_bound) {
  const int sms = num_sms();
  int best = *cands.begin();
  int64_t best_cost = INT64_MAX;
  for (int bt : cands) {
    const int64_t tiles = (int64_t)(N / kRows) * ((M + bt - 1) / bt);
    const int64_t waves = (tiles + sms - 1) / sms;
    const int64_t cost = tensor_bound ? waves * (bt + 170) : waves;
    if (cost < best_cost) { best_cost = cost; best = bt; }
  }
  return best;
}

// K multiple of 128: 128-wide stages (WK = 2), as many as shared and tensor
// memory allow (3 for the wide tiles, 4 up to BT = 128).  Otherwise 64-wide
// stages.
template <typename T, bool NF>
int w4_dispatch(const void* x, int M, int N, int K, int group, const void* packed,
                const float* bias, void* y, int* err, cudaStream_t st, const LoraArgs& lo = LoraArgs()) {
  if (M <= 16) {
    const int rc = launch_gemv<T, NF>(x, M, N, K, group, packed, bias, y, err, st, lo);
    if (rc != 1) return rc;
    // 9 - 16 tokens (or a group too large for the GEMV): 32-token tensor-core tiles
    if (K % (2 * kBK) == 0) return launch_w4<T, 32, 4, NF, 2>(x, M, N, K, group, packed, bias, y, err, st, lo);
    return launch_w4<T, 32, 8, NF, 1>(x, M, N, K, group, packed, bias, y, err, st, lo);
  }
  if (K % (2 * kBK) == 0) {
    if (M <= 32) return launch_w4<T, 32, 4, NF, 2>(x, M, N, K, group, packed, bias, y, err, st, lo);
    if (M <= 64) return launch_w4<T, 64, 4, NF, 2>(x, M, N, K, group, packed, bias, y, err, st, lo);
    if (M <= 128) return launch_w4<T, 128, 4, NF, 2>(x, M, N, K, group, packed, bias, y, err, st, lo);
    if constexpr (!NF) {
      switch (pick_bt(M, N, {256, 224, 192, 160}, true)) {
        case 224: return launch_w4<T, 224, 3, NF, 2>(x, M, N, K, group, packed, bias, y, err, st, lo);
        case 192: return launch_w4<T, 192, 3, NF, 2>(x, M, N, K, group, packed, bias, y, err, st, lo);
        case 160: return launch_w4<T, 160, 3, NF, 2>(x, M, N, K, group, packed, bias, y, err, st, lo);
        default: return launch_w4<T, 256, 3, NF, 2>(x, M, N, K, group, packed, bias, y, err, st, lo);
      }
    } else {
      // NF4 past M = 128: with the 16-copy pair table three 128-wide stages
      // fit up to BT = 224 (not 256: the weight ring would be one deep)
      switch (pick_bt(M, N, {224, 192, 160}, true)) {
        case 192: return launch_w4<T, 192, 3, NF, 2>(x, M, N, K, group, packed, bias, y, err, st, lo);
        case 160: return launch_w4<T, 160, 3, NF, 2>(x, M, N, K, group, packed, bias, y, err, st, lo);
        default: return launch_w4<T, 224, 3, NF, 2>(x, M, N, K, group, packed, bias, y, err, st, lo);
      }
    }
  }
  if (M <= 32) return launch_w4<T, 32, 8, NF, 1>(x, M, N, K, group, packed, bias, y, err, st, lo);
  if (M <= 64) return launch_w4<T, 64, 8, NF, 1>(x, M, N, K, group, packed, bias, y, err, st, lo);
  if (M <= 128) return launch_w4<T, 128, 8, NF, 1>(x, M, N, K, group, packed, bias, y, err, st, lo);
  constexpr int S = NF ? 5 : 6;
  switch (pick_bt(M, N, {256, 224, 192}, false)) {
    case 224: return launch_w4<T, 224, S, NF, 1>(x, M, N, K, group, packed, bias, y, err, st, lo);
    case 192: return launch_w4<T, 192, S, NF, 1>(x, M, N, K, group, packed, bias, y, err, st, lo);
    default: return launch_w4<T, 256, S, NF, 1>(x, M, N, K, group, packed, bias, y, err, st, lo);
  }
}

// The token-tile width w4_dispatch launches for M > 16 tokens.
inline int w4_token_tile(bool nf, int M, int N, int K) {
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  if (K % (2 * kBK) == 0) return nf ? pick_bt(M, N, {224, 192, 160}, true) : pick_bt(M, N, {256, 224, 192, 160}, true);
  return pick_bt(M, N, {256, 224, 192}, false);
}

template <typename T, typename ST>
int pack_t(const int8_t* wi, const void* s, const void* z, int N, int K, int group, int sym,
           void* packed, cudaStream_t st) {
  int64_t work = (int64_t)N * K / 8;
  int grid = (int)((work + 255) / 256);
  if (grid > num_sms() * 16) grid = num_sms() * 16;
  w4a16_pack_kernel<T, ST><<<grid, 256, 0, st>>>(wi, s, z, N, K, group, sym,
                                                 static_cast<uint8_t*>(packed));
  return launched("w4a16_pack_kernel");
}

template <typename T>
int pack_s(const int8_t* wi, const void* s, const void* z, int sdt, int N, int K, int group,
           int sym, void* packed, cudaStream_t st) {
  switch (sdt) {
    case LQ_F32: return pack_t<T, float>(wi, s, z, N, K, group, sym, packed, st);
    case LQ_F16: return pack_t<T, __half>(wi, s, z, N, K, group, sym, packed, st);
    case LQ_BF16: return pack_t<T, __nv_bfloat16>(wi, s, z, N, K, group, sym, packed, st);
    default: set_error("unsupported scale dtype %d", sdt); return LQ_EDTYPE;
  }
}

int check_shape(int64_t N, int64_t K, int64_t group) {
  LQ_REQUIRE(N > 0 && K > 0 && group > 0, LQ_EINVAL, "bad shape");
  LQ_REQUIRE(N % kRows == 0, LQ_EINVAL, "W4A16 needs out_features %% 128 == 0 (got %lld)", (long long)N);
  LQ_REQUIRE(K % kBK == 0, LQ_EINVAL, "W4A16 needs in_features %% 64 == 0 (got %lld)", (long long)K);
  LQ_REQUIRE(group % kBK == 0 && K % group == 0, LQ_EINVAL,
             "W4A16 needs group_size %% 64 == 0 dividing in_features (got %lld)", (long long)group);
  LQ_REQUIRE(N < (1LL << 31) && K < (1LL << 31), LQ_ERANGE, "shape too large");
  return LQ_OK;
}

template <typename T, typename ST>
int nf4lin_pack_t(const void* codes, const void* s, const void* qs, const void* dqs, int64_t dq_group,
                  int N, int K, int group, void* packed, cudaStream_t st) {
  int64_t work = (int64_t)N * K / 8;
  int grid = (int)((work + 255) / 256);
  if (grid > num_sms() * 16) grid = num_sms() * 16;
  nf4lin_pack_kernel<T, ST><<<grid, 256, 0, st>>>(static_cast<const uint32_t*>(codes), static_cast<const ST*>(s),
                                                  static_cast<const ST*>(qs), static_cast<const ST*>(dqs),
                                                  dq_group, N, K, group, static_cast<uint8_t*>(packed));
  return launched("nf4lin_pack_kernel");
}

template <typename T>
int nf4lin_pack_s(const void* codes, const void* s, const void* qs, const void* dqs, int sdt,
                  int64_t dq_group, int N, int K, int group, void* packed, cudaStream_t st) {
  switch (sdt) {
    case LQ_F32: return nf4lin_pack_t<T, float>(codes, s, qs, dqs, dq_group, N, K, group, packed, st);
    case LQ_F16: return nf4lin_pack_t<T, __half>(codes, s, qs, dqs, dq_group, N, K, group, packed, st);
    case LQ_BF16: return nf4lin_pack_t<T, __nv_bfloat16>(codes, s, qs, dqs, dq_group, N, K, group, packed, st);
    default: set_error("unsupported scale dtype %d", sdt); return LQ_EDTYPE;
  }
}

}  // namespace
}  // namespace lq

using namespace lq;

extern "C" size_t lq_nf4_linear_packed_bytes(int64_t N, int64_t K) {
  if (N <= 0 || K <= 0) return 0;
  return (size_t)(gemv_codes_off(N, K, K / kBK) + N / 16 * (K / kBK) * gv_record_bytes(kBK));
}

extern "C" int lq_nf4_linear_pack(const void* codes, const void* scales, const void* q_scales,
                                  const void* dq_scales, int s_dtype, int64_t N, int64_t K,
                                  int64_t group, int64_t dq_group, int act_dtype, void* packed,
                                  void* stream) {
  int rc = check_shape(N, K, group);
  if (rc) return rc;
  LQ_REQUIRE(codes && packed, LQ_EINVAL, "NULL pointer");
  LQ_REQUIRE(scales || (q_scales && dq_scales && dq_group > 0), LQ_EINVAL,
             "need the block scales, or q_scales + dq_scales + dq_group");
  LQ_REQUIRE(reinterpret_cast<uintptr_t>(codes) % 4 == 0 && aligned16(packed), LQ_EALIGN,
             "codes must be 4-byte and packed 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  const void* s = q_scales ? nullptr : scales;
  const void* qs = q_scales ? q_scales : nullptr;
  const void* dqs = q_scales ? dq_scales : nullptr;
  if (act_dtype == LQ_F16) return nf4lin_pack_s<__half>(codes, s, qs, dqs, s_dtype, dq_group, (int)N, (int)K, (int)group, packed, st);
  if (act_dtype == LQ_BF16) return nf4lin_pack_s<__nv_bfloat16>(codes, s, qs, dqs, s_dtype, dq_group, (int)N, (int)K, (int)group, packed, st);
  set_error("NF4 linear activations must be fp16 or bf16 (got dtype %d)", act_dtype);
  return LQ_EDTYPE;
}

extern "C" int lq_nf4_linear(const void* x, int act_dtype, int64_t M, int64_t N, int64_t K,
                             const void* packed, const float* bias, void* y, int* err, void* stream) {
  int rc = check_shape(N, K, kBK);
  if (rc) return rc;
  LQ_REQUIRE(M >= 0 && M < (1LL << 31), LQ_EINVAL, "bad M");
  if (M == 0) return LQ_OK;
  LQ_REQUIRE(x && packed && y, LQ_EINVAL, "NULL pointer");
  LQ_REQUIRE(aligned16(x) && aligned16(packed), LQ_EALIGN, "x and packed must be 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  if (act_dtype == LQ_F16) return w4_dispatch<__half, true>(x, (int)M, (int)N, (int)K, kBK, packed, bias, y, err, st);
  if (act_dtype == LQ_BF16) return w4_dispatch<__nv_bfloat16, true>(x, (int)M, (int)N, (int)K, kBK, packed, bias, y, err, st);
  set_error("NF4 linear activations must be fp16 or bf16 (got dtype %d)", act_dtype);
  return LQ_EDTYPE;
}

extern "C" int lq_nf4_linear_lora(const void* x, int act_dtype, int64_t M, int64_t N, int64_t K,
                                  const void* packed, const float* bias, const void* lora_u,
                                  const void* lora_b, int64_t rank, void* y, int* err, void* stream) {
  int rc = check_shape(N, K, kBK);
  if (rc) return rc;
  LQ_REQUIRE(M >= 0 && M < (1LL << 31), LQ_EINVAL, "bad M");
  if (M == 0) return LQ_OK;
  LQ_REQUIRE(x && packed && y && lora_u && lora_b, LQ_EINVAL, "NULL pointer");
  LQ_REQUIRE(aligned16(x) && aligned16(packed) && aligned16(lora_u) && aligned16(lora_b), LQ_EALIGN,
             "x, packed, lora_u and lora_b must be 16-byte aligned");
  LQ_REQUIRE(rank >= 2 && rank % 2 == 0 && rank <= (M <= 8 ? kBK : 16), LQ_ERANGE,
             "fused LoRA needs an even rank <= %d at M = %lld (got %lld)", M <= 8 ? kBK : 16,
             (long long)M, (long long)rank);
  LoraArgs lo;
  lo.u = lora_u;
  lo.b = lora_b;
  lo.r = (int)rank;
  cudaStream_t st = as_stream(stream);
  if (act_dtype == LQ_F16) return w4_dispatch<__half, true>(x, (int)M, (int)N, (int)K, kBK, packed, bias, y, err, st, lo);
  if (act_dtype == LQ_BF16) return w4_dispatch<__nv_bfloat16, true>(x, (int)M, (int)N, (int)K, kBK, packed, bias, y, err, st, lo);
  set_error("NF4 linear activations must be fp16 or bf16 (got dtype %d)", act_dtype);
  return LQ_EDTYPE;
}

extern "C" int lq_nf4_qlora_forward(const void* x, int act_dtype, int64_t M, int64_t N, int64_t K,
                                    const void* packed, const float* bias, const void* lora_a, int a_dtype,
                                    const void* lora_b, int64_t rank, float scaling, void* u, void* y,
                                    int* err, void* stream) {
  int rc = check_shape(N, K, kBK);
  if (rc) return rc;
  LQ_REQUIRE(M >= 0 && M < (1LL << 31), LQ_EINVAL, "bad M");
  if (M == 0) return LQ_OK;
  LQ_REQUIRE(x && packed && y && lora_a && lora_b && u, LQ_EINVAL, "NULL pointer");
  LQ_REQUIRE(aligned16(x) && aligned16(packed) && aligned16(u) && aligned16(lora_b), LQ_EALIGN,
             "x, packed, u and lora_b must be 16-byte aligned");
  LQ_REQUIRE(rank >= 2 && rank % 2 == 0 && rank <= (M <= 8 ? kBK : 16), LQ_ERANGE,
             "fused LoRA needs an even rank <= %d at M = %lld (got %lld)", M <= 8 ? kBK : 16,
             (long long)M, (long long)rank);
  LQ_REQUIRE(act_dtype == LQ_F16 || act_dtype == LQ_BF16, LQ_EDTYPE,
             "NF4 linear activations must be fp16 or bf16 (got dtype %d)", act_dtype);
  // The fused kernel takes a whole SM per tile, so it starts on the SMs that
  // the down-projection leaves free.  When its last wave of tiles leaves
  // SMs idle, the down-projection runs on that many (at most 4 token tiles
  // each; a block's tiles run one after another, about 3 us apiece): the
  // other SMs start the base product at once and the ones it delays have a
  // tile fewer to run (M = 1024, N = 14336: 32 blocks, 116.5 -> 113.9 us).
  int lu_blocks = 0;
  if (M > 16) {
    const int sms = num_sms(), bt = w4_token_tile(true, (int)M, (int)N, (int)K);
    const int64_t tiles = (N / kRows) * ((M + bt - 1) / bt);
    const int idle = (int)(tiles % sms == 0 ? 0 : sms - tiles % sms);
    if ((int64_t)idle * 4 >= (M + 15) / 16) lu_blocks = idle;
  }
  rc = lora_u_launch(x, act_dtype, M, K, lora_a, a_dtype, rank, scaling, u, stream, lu_blocks);
  if (rc) return rc;
  LoraArgs lo;
  lo.u = u;
  lo.b = lora_b;
  lo.r = (int)rank;
  lo.u_only_wait = 1;  // the kernel ahead of it in the stream is lq_lora_u, which writes only u
  cudaStream_t st = as_stream(stream);
  if (act_dtype == LQ_F16) return w4_dispatch<__half, true>(x, (int)M, (int)N, (int)K, kBK, packed, bias, y, err, st, lo);
  return w4_dispatch<__nv_bfloat16, true>(x, (int)M, (int)N, (int)K, kBK, packed, bias, y, err, st, lo);
}

extern "C" size_t lq_w4a16_packed_bytes(int64_t N, int64_t K, int64_t group) {
  if (N <= 0 || K <= 0 || group <= 0) return 0;
  return (size_t)(gemv_codes_off(N, K, K / group) + N / 16 * (K / group) * gv_record_bytes(group));
}

extern "C" int lq_w4a16_pack(const int8_t* weight_int, const void* scale, const void* zero_point,
                             int s_dtype, int64_t N, int64_t K, int64_t group, int symmetric,
                             int act_dtype, void* packed, void* stream) {
  int rc = check_shape(N, K, group);
  if (rc) return rc;
  LQ_REQUIRE(weight_int && scale && zero_point && packed, LQ_EINVAL, "NULL pointer");
  LQ_REQUIRE(aligned16(packed), LQ_EALIGN, "packed buffer must be 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  if (act_dtype == LQ_F16) return pack_s<__half>(weight_int, scale, zero_point, s_dtype, (int)N, (int)K, (int)group, symmetric, packed, st);
  if (act_dtype == LQ_BF16) return pack_s<__nv_bfloat16>(weight_int, scale, zero_point, s_dtype, (int)N, (int)K, (int)group, symmetric, packed, st);
  set_error("W4A16 activations must be fp16 or bf16 (got dtype %d)", act_dtype);
  return LQ_EDTYPE;
}

extern "C" int lq_w4a16_linear(const void* x, int act_dtype, int64_t M, int64_t N, int64_t K,
                               int64_t group, const void* packed, const float* bias, void* y,
                               int* err, void* stream) {
  int rc = check_shape(N, K, group);
  if (rc) return rc;
  LQ_REQUIRE(M >= 0 && M < (1LL << 31), LQ_EINVAL, "bad M");
  if (M == 0) return LQ_OK;
  LQ_REQUIRE(x && packed && y, LQ_EINVAL, "NULL pointer");
  LQ_REQUIRE(aligned16(x) && aligned16(packed), LQ_EALIGN, "x and packed must be 16-byte aligned");
  cudaStream_t st = as_stream(stream);
  if (act_dtype == LQ_F16) return w4_dispatch<__half, false>(x, (int)M, (int)N, (int)K, (int)group, packed, bias, y, err, st);
  if (act_dtype == LQ_BF16) return w4_dispatch<__nv_bfloat16, false>(x, (int)M, (int)N, (int)K, (int)group, packed, bias, y, err, st);
  set_error("W4A16 activations must be fp16 or bf16 (got dtype %d)", act_dtype);
  return LQ_EDTYPE;
}
