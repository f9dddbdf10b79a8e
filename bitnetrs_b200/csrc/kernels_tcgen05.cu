// kernels_tcgen05.cu — weight-streaming GEMMs on the 5th-generation tensor
// cores (tcgen05.mma, accumulator in tensor memory) for many activation rows:
//   * the ternary x int8 matmul (kind::i8) for M > 1 rows (batched decode
//     and prefill);
//   * the int8 lm_head for many rows (kind::f16): every int8 weight is exact
//     in bf16 and the f32 hidden state is the sum of three bf16 terms
//     (h1 | h2 | h3, concatenated along K), so each product the tensor core
//     forms is exact and only the f32 summation order differs from the
//     reference's FMA chains (the AUTO numerics of the lm_head).
//
// Ternary: the same integer identity as the other matmul kernels (gemv.rs:299-308):
//     sum_k (1 - c_k) x_k = rowsum(x) - sum_k c_k x_k,   c_k in {0,1,2},
// so the tensor core multiplies unsigned 2-bit codes widened to u8 by the
// signed int8 activations, exact in int32; the epilogue applies the
// reference's `acc as f32 * (weight_scale * act_absmax / 127)`.
//
// Weight-stationary tiling: the weight matrix is the large, streamed operand,
// so 128 weight rows are the MMA's M (one TMEM lane per output feature) and up
// to 256 activation rows are its N. One CTA computes 128 features x nb rows:
//   * warp 4 issues every TMA load (one lane): packed 2-bit words in groups of
//     four k-steps (128 bytes per weight row, 128-byte swizzled) and the
//     activation tile of each k-step (nb rows x 128 bytes, 128-byte swizzled,
//     rows past M read as zero);
//   * warps 0-3 widen the packed words of their own weight row into u8 codes
//     and store them straight into tensor memory (lane = weight row, four
//     codes per 32-bit column), then run the epilogue;
//   * warp 5 issues four 128 x nb x 32 MMAs per k-step (one lane), A from
//     tensor memory and B from shared memory, and commits them to the
//     mbarriers that release the stages.
// A k-step stage is one activation tile in shared memory plus 32 columns of
// widened weights in tensor memory (the accumulator uses columns 0-255). Its
// `full` mbarrier completes when the activation bytes have landed and all four
// widen warps have arrived; one tcgen05.commit on its `empty` mbarrier
// releases both halves. The MMA warp waits for step i+1 while the MMAs of
// step i execute, so the handshake stays off the tensor pipe's critical path.
// The epilogue thread of feature n reads its TMEM lane; for each activation
// row the 32 lanes of a warp store 32 consecutive features (128 bytes).
//
// Split-K: when the feature tiles alone leave SMs idle, `splits` CTAs of a
// thread-block cluster take consecutive k ranges of the same tile, stage their
// int32 partials in their own shared memory, and each reduces one slice of the
// tile's activation rows across the cluster through distributed shared memory.
// Integer sums make the result independent of the split.
//
// Every mbarrier wait is bounded; a CTA that gives up records
// kStatusWaitTimeout, waits (bounded) for the loads and MMAs it issued, still
// meets its cluster barriers and frees its tensor memory.
#include "kernels.cuh"

#include <cudaTypedefs.h>

#include <mutex>

namespace bitnet {

namespace {

constexpr int kTcRows = 128;    // weight rows per CTA: MMA M, TMEM lanes
constexpr int kTcBK = 128;      // codes per k-step (128 bytes of u8 per row)
constexpr int kTcMaxNb = 256;   // activation rows per CTA: MMA N
constexpr int kTcPG = 4;        // packed-weight ring (groups)
constexpr int kTcMaxSB = 8;     // k-step stages (activation tile + widened weights; fewer for wide tiles)
constexpr int kTcThreads = 192; // warps 0-3 widen + epilogue, warp 4 loads, warp 5 MMA
constexpr int kTcPacked = kTcRows * 32 * 4;  // 16 KiB: 32 words per row
constexpr uint32_t kTcTmemCols = 512;        // accumulator + widened stages
constexpr uint32_t kTcTmemA = 256;           // first column of the widened stages (32 columns each)
constexpr int kTcCombStride = kTcMaxNb + 4;
constexpr int kTcMaxSplits = 4;
constexpr int kTcDynBudget = 220 * 1024;     // dynamic shared memory cap per CTA
constexpr long long kTcWaitCycles = 2000000000LL;
constexpr long long kTcDrainCycles = 4000000LL;  // a load lands within microseconds

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool tc_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __noinline__ bool tc_wait_slow(uint32_t bar, uint32_t parity, const volatile int* abort_flag) {
  const long long t0 = clock64();
  for (;;) {
    if (tc_try_wait(bar, parity)) return true;
    if (abort_flag && *abort_flag) return false;
    if (clock64() - t0 > kTcWaitCycles) return false;
  }
}
__device__ __forceinline__ bool tc_wait(uint32_t bar, uint32_t parity, const volatile int* abort_flag) {
  return tc_try_wait(bar, parity) || tc_wait_slow(bar, parity, abort_flag);
}
__device__ __noinline__ bool tc_wait_for(uint32_t bar, uint32_t parity, long long cycles) {
  const long long t0 = clock64();
  while (!tc_try_wait(bar, parity))
    if (clock64() - t0 > cycles) return false;
  return true;
}
__device__ __forceinline__ void tc_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar,
                                           uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];\n" ::"r"(dst),
      "l"((uint64_t)map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

// Shared-memory matrix descriptor: K-major operand, rows of 128 bytes,
// 128-byte swizzle, 8-row groups 1024 bytes apart (sm_100 descriptor v1).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);  // start address
  d |= (uint64_t)1 << 16;                            // leading byte offset (unused with swizzle)
  d |= (uint64_t)(1024 >> 4) << 32;                  // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                            // descriptor version
  d |= (uint64_t)2 << 61;                            // SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

// 32 consecutive 32-bit columns of this warp's 32 lanes from registers.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}

// Epilogue for one output feature over `cnt` (<= R) consecutive activation
// rows: out[m] = acc * comb[m] (Store) or out[m] + acc * comb[m] (Residual),
// the reference's rounding order. Residual reads every old value before the
// first store so the loads overlap.
template <int R>
__device__ __forceinline__ void store_rows(float* __restrict__ p, int ldo, const int32_t (&a)[R],
                                           const float* comb, int cnt, Epi epi) {
  float v[R];
#pragma unroll
  for (int j = 0; j < R; ++j) v[j] = __fmul_rn((float)a[j], comb[j]);
  if (epi == Epi::Residual) {
    float old[R];
#pragma unroll
    for (int j = 0; j < R; ++j) old[j] = j < cnt ? p[(size_t)j * ldo] : 0.0f;
#pragma unroll
    for (int j = 0; j < R; ++j)
      if (j < cnt) p[(size_t)j * ldo] = __fadd_rn(old[j], v[j]);
  } else {
#pragma unroll
    for (int j = 0; j < R; ++j)
      if (j < cnt) p[(size_t)j * ldo] = v[j];
  }
}

// int8 (sign-extended) -> float, exactly, on the full-rate pipes: the bit
// pattern 0x4B400000 + v is the float 1.5 * 2^23 + v for |v| < 2^22.
__device__ __forceinline__ float i8_exact_f32(int32_t v) {
  return __fsub_rn(__int_as_float(0x4B400000 + v), 12582912.0f);
}
// Four int8 of a word (lowest byte first) -> two bf16x2 words; a float holding
// an integer of at most 8 significant bits has its bf16 in the top half.
__device__ __forceinline__ uint2 i8x4_to_bf16x4(uint32_t w) {
  const float f0 = i8_exact_f32((int32_t)(w << 24) >> 24), f1 = i8_exact_f32((int32_t)(w << 16) >> 24);
  const float f2 = i8_exact_f32((int32_t)(w << 8) >> 24), f3 = i8_exact_f32((int32_t)w >> 24);
  return make_uint2((__float_as_uint(f0) >> 16) | (__float_as_uint(f1) & 0xffff0000u),
                    (__float_as_uint(f2) >> 16) | (__float_as_uint(f3) & 0xffff0000u));
}

}  // namespace

enum class TcKind : int { Ternary = 0, LmHead = 1 };

// Per-kind pieces of the kernel. A weight load brings 128 bytes of each of the
// tile's 128 rows (128-byte swizzled); a k-step fills 32 TMEM columns.
template <TcKind K>
struct TcTraits;
template <>
struct TcTraits<TcKind::Ternary> {
  static constexpr int kGroupSteps = 4;  // 4 x 32 bytes of packed codes per load
  static constexpr int kActCols = 128;   // int8 activation elements per k-step
  // D s32, A u8 (codes), B s8 (activations), both K-major, M = 128, N = nb.
  static __device__ __forceinline__ uint32_t idesc(int nb) {
    return (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(nb >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
  }
  // step q of the group: chunks 2q, 2q+1 of the row's packed line. Word c holds
  // codes 16c..16c+15; column 4c+e receives codes 16c+4e..16c+4e+3.
  static __device__ __forceinline__ void widen(const uint8_t* prow, int q, int row, uint32_t (&col)[32]) {
    const uint4 p0 = *reinterpret_cast<const uint4*>(prow + (((2 * q) ^ (row & 7)) << 4));
    const uint4 p1 = *reinterpret_cast<const uint4*>(prow + (((2 * q + 1) ^ (row & 7)) << 4));
    const uint32_t words[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
    for (int c = 0; c < 8; ++c) {
#pragma unroll
      for (int e = 0; e < 4; ++e) col[4 * c + e] = (words[c] >> (2 * e)) & 0x03030303u;
    }
  }
};
template <>
struct TcTraits<TcKind::LmHead> {
  static constexpr int kGroupSteps = 2;  // 2 x 64 int8 weights per load
  static constexpr int kActCols = 64;    // bf16 activation elements per k-step
  // D f32, A bf16 (widened weights), B bf16 (activation terms), K-major, M = 128, N = nb.
  static __device__ __forceinline__ uint32_t idesc(int nb) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(nb >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
  }
  // step q of the group: chunks 4q..4q+3 (64 int8); column c receives
  // elements 2c, 2c+1 as bf16x2.
  static __device__ __forceinline__ void widen(const uint8_t* prow, int q, int row, uint32_t (&col)[32]) {
#pragma unroll
    for (int cc = 0; cc < 4; ++cc) {
      const uint4 p = *reinterpret_cast<const uint4*>(prow + (((4 * q + cc) ^ (row & 7)) << 4));
      const uint32_t w[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint2 b = i8x4_to_bf16x4(w[j]);
        col[8 * cc + 2 * j] = b.x;
        col[8 * cc + 2 * j + 1] = b.y;
      }
    }
  }
};

struct TcShape {
  int nb, sb, splits, per;  // activation rows per CTA, activation stages, k splits, k-steps per split
};

// nk k-steps in all; the lm_head runs three passes of kpass k-steps over the
// same weights (one per bf16 term of the activations), the ternary matmul one.
template <TcKind KIND>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap, int N, int nk,
                   int kpass, int M, TcShape sh, const float* __restrict__ amax, const int32_t* __restrict__ rowsum,
                   Segments seg, const float* __restrict__ vscale, Epi epi, float* __restrict__ out, int ldo,
                   int32_t* __restrict__ acc_out, int32_t* __restrict__ status) {
  using Tr = TcTraits<KIND>;
  constexpr int kGroup = Tr::kGroupSteps;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t pk_full[kTcPG], pk_empty[kTcPG];
  __shared__ __align__(8) uint64_t full[kTcMaxSB], empty[kTcMaxSB];
  __shared__ __align__(8) uint64_t acc_full;
  __shared__ float comb_s[3][kTcCombStride];  // (scale_seg * absmax[m]) / 127 per segment and row
  __shared__ int32_t rs_s[kTcMaxNb];          // rowsum[m]
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  // the warp index through a shuffle: the compiler then treats role branches
  // and the loop counters inside them as warp-uniform, which keeps the
  // tcgen05/mbarrier operands in uniform registers
  const int tid = threadIdx.x, warp = __shfl_sync(0xffffffffu, tid >> 5, 0), lane = tid & 31;
  const int nb = sh.nb, sb = sh.sb, splits = sh.splits;
  const int n0 = blockIdx.x * kTcRows, m0 = blockIdx.y * nb;
  uint32_t rank = 0;
  if (splits > 1) asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(rank));
  const int kb = (int)rank * sh.per;
  const int steps = max(0, min(nk, kb + sh.per) - kb);
  // shared layout (1024-aligned): activation stages | weight ring
  const uint32_t raw = su32(smem_raw);
  uint8_t* base = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  const int act_bytes = nb * kTcBK;
  uint8_t* sAct = base;
  uint8_t* sPk = sAct + sb * act_bytes;
  const uint32_t sAct32 = su32(sAct), sPk32 = su32(sPk);

  if (tid == 0) {
    for (int s = 0; s < kTcPG; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(su32(&pk_full[s])), "r"(1) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(su32(&pk_empty[s])), "r"(4) : "memory");
    }
    for (int s = 0; s < kTcMaxSB; ++s) {
      // producer's expect_tx arrival + one arrival per widen warp
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(su32(&full[s])), "r"(5) : "memory");
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(su32(&empty[s])), "r"(1) : "memory");
    }
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(su32(&acc_full)), "r"(1) : "memory");
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(su32(&tmem_slot)),
                 "r"(kTcTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
  const uint32_t tmem = tmem_slot;
  volatile int* abort_p = &abort_flag;
  auto fail = [&]() {
    if (!*abort_p) {
      *abort_p = 1;
      atomicOr(status, kStatusWaitTimeout);
    }
  };

  if (warp == 4) {
    // ---------------- loads: the whole warp runs the loop, lane 0 issues ----------------
    int g_issued = 0, a_issued = 0;
    bool stop = false;
    int s = 0, wrap = 0;  // stage of step i; completed passes over the ring
    for (int i = 0; i < steps; ++i) {
      if (__any_sync(0xffffffffu, *abort_p != 0)) break;
      if ((i & (kGroup - 1)) == 0) {
        const int g = i / kGroup, sp = g % kTcPG;
        if (g >= kTcPG && !__all_sync(0xffffffffu, tc_wait(su32(&pk_empty[sp]), ((g / kTcPG) - 1) & 1, abort_p))) {
          stop = true;
          break;
        }
        // x of the group's first k-step: packed words (ternary) or weight bytes within the pass
        const int wx = KIND == TcKind::Ternary ? (kb + i) * 8 : ((kb + i) % kpass) * 64;
        if (lane == 0) tc_load_2d(sPk32 + sp * kTcPacked, &wmap, wx, n0, su32(&pk_full[sp]), kTcPacked);
        __syncwarp();
        g_issued = g + 1;
      }
      if (wrap > 0 && !__all_sync(0xffffffffu, tc_wait(su32(&empty[s]), (wrap - 1) & 1, abort_p))) {
        stop = true;
        break;
      }
      if (lane == 0)
        tc_load_2d(sAct32 + s * act_bytes, &xmap, (kb + i) * Tr::kActCols, m0, su32(&full[s]), (uint32_t)act_bytes);
      __syncwarp();
      a_issued = i + 1;
      if (++s == sb) {
        s = 0;
        ++wrap;
      }
    }
    if (stop) fail();
    if (__any_sync(0xffffffffu, *abort_p != 0)) {
      // let the loads still in flight land before this CTA may exit; a stage
      // whose widen arrivals are missing never completes, so these waits are
      // short-bounded
      for (int g = max(0, g_issued - kTcPG); g < g_issued; ++g)
        tc_wait_for(su32(&pk_full[g % kTcPG]), (g / kTcPG) & 1, kTcDrainCycles);
      for (int i = max(0, a_issued - sb); i < a_issued; ++i)
        tc_wait_for(su32(&full[i % sb]), (i / sb) & 1, kTcDrainCycles);
    }
  } else if (warp == 5) {
    // ---------------- MMA issue: the whole warp runs the loop, lane 0 issues ----------------
    const uint32_t idesc = Tr::idesc(nb);
    int s = 0;
    uint32_t parity = 0;
    bool ok = steps > 0 && tc_wait(su32(&full[0]), 0, abort_p);
    for (int i = 0; i < steps; ++i) {
      if (!__all_sync(0xffffffffu, ok)) {
        fail();
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
      if (lane == 0) {
        const uint32_t a_tmem = tmem + kTcTmemA + (uint32_t)(s * (kTcBK / 4));
        const uint32_t b_addr = sAct32 + s * act_bytes;
#pragma unroll
        for (int kk = 0; kk < kTcBK / 32; ++kk) {
          const uint64_t bd = sw128_desc(b_addr + 32 * kk);
          const uint32_t accumulate = (i > 0 || kk > 0) ? 1u : 0u;
          if constexpr (KIND == TcKind::Ternary)
            asm volatile(
                "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                " tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem),
                "r"(a_tmem + 8u * kk), "l"(bd), "r"(idesc), "r"(accumulate)
                : "memory");
          else  // bf16 x bf16 -> f32 (A and B of one type)
            asm volatile(
                "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem),
                "r"(a_tmem + 8u * kk), "l"(bd), "r"(idesc), "r"(accumulate)
                : "memory");
        }
      }
      __syncwarp();
      // operands of step i+1, while the MMAs of step i run
      const int ns = s + 1 == sb ? 0 : s + 1;
      const uint32_t nparity = ns == 0 ? parity ^ 1u : parity;
      if (i + 1 < steps) ok = tc_wait(su32(&full[ns]), nparity, abort_p);
      if (lane == 0) tc_commit(su32(&empty[s]));
      __syncwarp();
      s = ns;
      parity = nparity;
    }
    if (lane == 0) tc_commit(su32(&acc_full));  // tracks every MMA lane 0 issued
    __syncwarp();
  } else {
    // epilogue constants, read after the named barrier that precedes the
    // epilogue; their loads overlap the first weight loads
    if constexpr (KIND == TcKind::Ternary) {
      for (int c = tid; c < kTcMaxNb; c += 128) {
        const int m = m0 + c;
        const bool valid = c < nb && m < M;
        const float am = valid ? amax[m] : 0.0f;
        rs_s[c] = valid ? rowsum[m] : 0;
#pragma unroll
        for (int q = 0; q < 3; ++q) comb_s[q][c] = __fdiv_rn(__fmul_rn(seg.scale[q], am), 127.0f);
      }
    }
    // ---------------- widen: thread tid owns weight row n0 + tid (TMEM lane tid) ----------------
    const uint32_t wlane = tmem + ((uint32_t)(32 * warp) << 16) + kTcTmemA;
    int s = 0, wrap = 0;
    for (int i = 0; i < steps; ++i) {
      const int g = i / kGroup, q = i & (kGroup - 1), sp = g % kTcPG;
      bool ok = true;
      if (q == 0) ok = tc_wait(su32(&pk_full[sp]), (g / kTcPG) & 1, abort_p);
      if (ok && wrap > 0) ok = tc_wait(su32(&empty[s]), (wrap - 1) & 1, abort_p);
      if (!__all_sync(0xffffffffu, ok)) {
        fail();
        break;
      }
      // this row's 128-byte weight line, stored 128-byte swizzled
      uint32_t col[32];
      Tr::widen(sPk + sp * kTcPacked + tid * 128, q, tid, col);
      if (q == kGroup - 1 || i == steps - 1) {
        __syncwarp();
        if (lane == 0) tc_arrive(su32(&pk_empty[sp]));
      }
      asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");  // after the empty wait
      tmem_st32(wlane + (uint32_t)(s * (kTcBK / 4)), col);
      asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
      __syncwarp();
      if (lane == 0) tc_arrive(su32(&full[s]));
      if (++s == sb) {
        s = 0;
        ++wrap;
      }
    }

    // ---------------- epilogue ----------------
    const bool done = tc_wait(su32(&acc_full), 0, nullptr);
    if (!__all_sync(0xffffffffu, done)) fail();
    asm volatile("bar.sync 1, 128;\n" ::: "memory");
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    const bool ok = __shfl_sync(0xffffffffu, *abort_p == 0 ? 1 : 0, 0) != 0;
    const int n = n0 + tid;
    const int sidx = n < seg.end[0] ? 0 : (n < seg.end[1] ? 1 : 2);
    const float* comb = comb_s[sidx];
    const uint32_t trow = tmem + ((uint32_t)(32 * warp) << 16);
    if constexpr (KIND == TcKind::LmHead) {
      // logits[m][n] = acc * scale[n]
      const bool live = ok && n < N;
      const float vs = live ? vscale[n] : 0.0f;
      const int rows = min(nb, M - m0);
#pragma unroll 1
      for (int c0 = 0; c0 < nb; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(trow + (uint32_t)c0, r);
        const int cnt = min(32, rows - c0);
        if (live && cnt > 0) {
          float* p = out + (size_t)(m0 + c0) * ldo + n;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (j < cnt) p[(size_t)j * ldo] = __fmul_rn(__uint_as_float(r[j]), vs);
        }
      }
    } else if (splits == 1) {
      const bool live = ok && n < N;
      const int rows = min(nb, M - m0);  // valid activation rows of this tile
#pragma unroll 1
      for (int c0 = 0; c0 < nb; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(trow + (uint32_t)c0, r);
        const int cnt = min(32, rows - c0);  // uniform across the CTA
        if (live && cnt > 0) {
          int32_t a[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) a[j] = rs_s[c0 + j] - (int32_t)r[j];
          store_rows(out + (size_t)(m0 + c0) * ldo + n, ldo, a, comb + c0, cnt, epi);
          if (acc_out) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < cnt) acc_out[(size_t)(m0 + c0 + j) * N + n] = a[j];
          }
        }
      }
    } else {
      // stage this CTA's int32 partial in groups of four activation rows:
      // 16-byte unit (c / 4) * 128 + tid holds rows c..c+3 of feature tid, so
      // each warp access below (local or remote) covers 512 contiguous bytes
      uint4* stage = reinterpret_cast<uint4*>(base) + tid;
#pragma unroll 1
      for (int c0 = 0; c0 < nb; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(trow + (uint32_t)c0, r);
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          if (c0 + j < nb) stage[((c0 + j) >> 2) * kTcRows] = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
      }
    }
  }

  if (KIND == TcKind::Ternary && splits > 1) {
    // every thread of every CTA of the cluster meets both barriers
    cluster_sync_all();
    if (tid < 128) {
      const bool ok = *abort_p == 0;
      const int n = n0 + tid;
      const int sidx = n < seg.end[0] ? 0 : (n < seg.end[1] ? 1 : 2);
      const float* comb = comb_s[sidx];
      const int cs = nb / splits, c_lo = (int)rank * cs;
      const uint32_t my = su32(base) + (uint32_t)tid * 16u;
      uint32_t peer[kTcMaxSplits];
#pragma unroll
      for (int q = 0; q < kTcMaxSplits; ++q) {
        peer[q] = my;
        if (q < splits) asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(peer[q]) : "r"(my), "r"(q));
      }
      const int rows = min(nb, M - m0);
      // blocks of 8 activation rows: two coalesced 16-byte loads from each CTA of the cluster
#pragma unroll 1
      for (int c = c_lo; c < c_lo + cs; c += 8) {
        uint32_t v[kTcMaxSplits][8];
#pragma unroll
        for (int q = 0; q < kTcMaxSplits; ++q) {
          if (q < splits) {
#pragma unroll
            for (int h = 0; h < 2; ++h)
              asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];\n"
                           : "=r"(v[q][4 * h]), "=r"(v[q][4 * h + 1]), "=r"(v[q][4 * h + 2]), "=r"(v[q][4 * h + 3])
                           : "r"(peer[q] + (uint32_t)(((c >> 2) + h) * kTcRows) * 16u));
          }
        }
        int32_t a[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          int32_t sum = 0;
#pragma unroll
          for (int q = 0; q < kTcMaxSplits; ++q)
            if (q < splits) sum += (int32_t)v[q][e];
          a[e] = rs_s[c + e] - sum;
        }
        const int cnt = min(min(8, rows - c), c_lo + cs - c);  // this CTA's slice only
        if (ok && n < N && cnt > 0) {
          store_rows(out + (size_t)(m0 + c) * ldo + n, ldo, a, comb + c, cnt, epi);
          if (acc_out) {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (e < cnt) acc_out[(size_t)(m0 + c + e) * N + n] = a[e];
          }
        }
      }
    }
    cluster_sync_all();  // peers have finished reading this CTA's partial
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
  __syncthreads();
  if (warp == 5)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTcTmemCols)
                 : "memory");
}

namespace {
PFN_cuTensorMapEncodeTiled_v12000 tc_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

size_t tc_dyn_smem(int nb, int sb) { return 1024 + (size_t)sb * nb * kTcBK + (size_t)kTcPG * kTcPacked; }

int g_sm_count = 148;
}  // namespace

int ternary_tc_prepare() {
  if (!tc_encoder()) return 1;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&g_sm_count, cudaDevAttrMultiProcessorCount, dev);
  if (cudaFuncSetAttribute(tc_gemm_kernel<TcKind::Ternary>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kTcDynBudget) != cudaSuccess)
    return 1;
  return cudaFuncSetAttribute(tc_gemm_kernel<TcKind::LmHead>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              kTcDynBudget) == cudaSuccess
             ? 0
             : 1;
}

int ternary_tc_plan(int N, int K, int M, int* nb_out, int* sb_out, int* splits_out, int* per_out) {
  if (M < 1 || N < 1 || K < 1) return 1;
  const int kw = (int)words_per_row(K);
  const int nk = (kw + 7) / 8;
  const int tiles_m = (M + kTcMaxNb - 1) / kTcMaxNb;
  const int nb = ((M + tiles_m - 1) / tiles_m + 15) / 16 * 16;
  int sb = kTcMaxSB;
  while (sb > 2 && tc_dyn_smem(nb, sb) > (size_t)kTcDynBudget) --sb;
  const int tiles = ((N + kTcRows - 1) / kTcRows) * tiles_m;
  int splits = 1;
  // doubling keeps each CTA's reduction slice (nb / splits rows) a multiple of 8
  while (splits < kTcMaxSplits && tiles * splits * 2 <= g_sm_count && nk >= splits * 4 &&
         nb % (16 * splits) == 0)
    splits *= 2;
  int per = (nk + splits - 1) / splits;
  while (splits > 1 && (splits - 1) * per >= nk) {
    splits /= 2;
    per = (nk + splits - 1) / splits;
  }
  *nb_out = nb;
  *sb_out = sb;
  *splits_out = splits;
  *per_out = per;
  return 0;
}

int launch_ternary_tc(const uint32_t* W, int N, int K, const int8_t* xq, int ldq, const float* act_absmax,
                      const int32_t* row_sum, int M, const Segments& seg, Epi epi, float* out, int ldo, int32_t* acc,
                      int32_t* status, cudaStream_t st) {
  auto enc = tc_encoder();
  if (!enc || !status) return 1;
  const int kw = (int)words_per_row(K);
  if ((reinterpret_cast<uintptr_t>(xq) & 15) || (ldq % 16) || (reinterpret_cast<uintptr_t>(W) & 15) || (kw % 4))
    return 1;
  TcShape sh;
  if (ternary_tc_plan(N, K, M, &sh.nb, &sh.sb, &sh.splits, &sh.per) != 0) return 1;
  CUtensorMap xmap, wmap;
  {
    const cuuint64_t dims[2] = {(cuuint64_t)ldq, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)ldq};
    const cuuint32_t box[2] = {(cuuint32_t)kTcBK, (cuuint32_t)sh.nb};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&xmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(xq), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return 1;
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)kw, (cuuint64_t)N};
    const cuuint64_t strides[1] = {(cuuint64_t)kw * 4};
    const cuuint32_t box[2] = {32, (cuuint32_t)kTcRows};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(W), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return 1;
  }
  const int nk = (kw + 7) / 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ceil_div(N, kTcRows), (unsigned)ceil_div(M, sh.nb), (unsigned)sh.splits);
  cfg.blockDim = dim3(kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = tc_dyn_smem(sh.nb, sh.sb);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = (unsigned)sh.splits;
  cfg.attrs = attr;
  cfg.numAttrs = sh.splits > 1 ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, tc_gemm_kernel<TcKind::Ternary>, wmap, xmap, N, nk, nk, M, sh, act_absmax, row_sum,
                         seg, static_cast<const float*>(nullptr), epi, out, ldo, acc, status) != cudaSuccess) {
    (void)cudaGetLastError();  // the caller falls back to another kernel; do not leave the error pending
    return 1;
  }
  count_launch();
  return 0;
}

bool lm_head_tc_supported(int H) { return H > 0 && H % 128 == 0; }

int launch_lm_head_tc(const uint16_t* a3, int M, int V, int H, const int8_t* W, const float* scales, float* out,
                      int ldo, int32_t* status, cudaStream_t st) {
  auto enc = tc_encoder();
  if (!enc || !status || !lm_head_tc_supported(H) || M < 1 || V < 1) return 1;
  if ((reinterpret_cast<uintptr_t>(a3) & 15) || (reinterpret_cast<uintptr_t>(W) & 15)) return 1;
  TcShape sh;
  // rows per CTA and stages as for the ternary matmul of the same M; no k split
  if (ternary_tc_plan(V, 16, M, &sh.nb, &sh.sb, &sh.splits, &sh.per) != 0) return 1;
  const int kpass = H / 64, nk = 3 * kpass;
  sh.splits = 1;
  sh.per = nk;
  CUtensorMap xmap, wmap;
  {
    const cuuint64_t dims[2] = {(cuuint64_t)(3 * H), (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)(3 * H) * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)sh.nb};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(a3), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return 1;
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)H, (cuuint64_t)V};
    const cuuint64_t strides[1] = {(cuuint64_t)H};
    const cuuint32_t box[2] = {128, (cuuint32_t)kTcRows};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(W), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return 1;
  }
  Segments seg;
  dim3 grid((unsigned)ceil_div(V, kTcRows), (unsigned)ceil_div(M, sh.nb), 1);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = tc_dyn_smem(sh.nb, sh.sb);
  cfg.stream = st;
  if (cudaLaunchKernelEx(&cfg, tc_gemm_kernel<TcKind::LmHead>, wmap, xmap, V, nk, kpass, M, sh,
                         static_cast<const float*>(nullptr), static_cast<const int32_t*>(nullptr), seg, scales,
                         Epi::Store, out, ldo, static_cast<int32_t*>(nullptr), status) != cudaSuccess) {
    (void)cudaGetLastError();  // the caller falls back to the mma.sync kernel
    return 1;
  }
  count_launch();
  return 0;
}

}  // namespace bitnet
