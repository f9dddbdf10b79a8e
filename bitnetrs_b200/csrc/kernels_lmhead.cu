// kernels_lmhead.cu — lm_head matmuls and greedy argmax.
//
// The reference computes every logit as one AVX2 dot product
// (dot_f32_i8w_avx2 / dot_f32_bf16w_avx2 / dot_f32_f32_avx2, simd.rs):
// eight FMA chains over groups of 8 columns, hsum_f32_avx2, then a scalar
// tail (mul + add).  Here thread (row r, chain j) of a block runs chain j of
// row r for a group of tokens, and the eight chain threads of a row combine
// with the same hsum tree, so each logit is bit-identical to the reference.
#include "kernels.cuh"

namespace bitnet {

template <LmW WT>
struct WTraits;
template <>
struct WTraits<LmW::I8> {
  using T = int8_t;
  static constexpr int ROWS = 32;
  static constexpr int COLS = 512;
  __device__ static float cvt(T w) { return (float)w; }
};
template <>
struct WTraits<LmW::BF16> {
  using T = uint16_t;
  static constexpr int ROWS = 32;
  static constexpr int COLS = 256;
  __device__ static float cvt(T w) { return bf16_bits_to_f32(w); }
};
template <>
struct WTraits<LmW::F32> {
  using T = float;
  static constexpr int ROWS = 32;
  static constexpr int COLS = 128;
  __device__ static float cvt(T w) { return w; }
};

template <LmW WT, int TM>
__global__ void __launch_bounds__(256) lm_head_kernel(const typename WTraits<WT>::T* __restrict__ W,
                                                      const float* __restrict__ scales, const float* __restrict__ h,
                                                      int ldh, int M, int V, int H, float* __restrict__ out, int ldo) {
  using T = typename WTraits<WT>::T;
  constexpr int ROWS = WTraits<WT>::ROWS;
  constexpr int kLmCols = WTraits<WT>::COLS;  // columns staged per chunk (multiple of 8)
  constexpr int WPAD = 16 / sizeof(T);  // 16-byte row pad
  constexpr int WSTR = kLmCols + WPAD;
  __shared__ __align__(16) T wsm[ROWS * WSTR];
  __shared__ __align__(16) float hsm[kLmCols * TM];

  const int tid = threadIdx.x;
  const int r = tid >> 3, j = tid & 7;
  const int v0 = blockIdx.x * ROWS;
  const int v = v0 + r;
  const int Hm = (H / 8) * 8;

  for (int g0 = 0; g0 < M; g0 += TM) {
    const int tm = min(TM, M - g0);
    float acc[TM];
#pragma unroll
    for (int m = 0; m < TM; ++m) acc[m] = 0.0f;
    for (int c0 = 0; c0 < Hm; c0 += kLmCols) {
      const int nc = min(kLmCols, Hm - c0);
      __syncthreads();
      // Stage W[v0 .. v0+ROWS)[c0 .. c0+nc) (16-byte vectors where aligned).
      constexpr int VEC = 16 / sizeof(T);
      const int vec_per_row = nc / VEC;
      const bool vec_ok = ((size_t)H * sizeof(T)) % 16 == 0 && (c0 * sizeof(T)) % 16 == 0 && nc % VEC == 0;
      if (vec_ok) {
        for (int i = tid; i < ROWS * vec_per_row; i += 256) {
          int rr = i / vec_per_row, cc = (i % vec_per_row) * VEC;
          uint4 val = make_uint4(0, 0, 0, 0);
          if (v0 + rr < V) val = __ldcs(reinterpret_cast<const uint4*>(W + (size_t)(v0 + rr) * H + c0 + cc));
          *reinterpret_cast<uint4*>(&wsm[rr * WSTR + cc]) = val;
        }
      } else {
        for (int i = tid; i < ROWS * nc; i += 256) {
          int rr = i / nc, cc = i % nc;
          wsm[rr * WSTR + cc] = (v0 + rr < V) ? W[(size_t)(v0 + rr) * H + c0 + cc] : (T)0;
        }
      }
      for (int i = tid; i < TM * nc; i += 256) {
        int m = i / nc, cc = i % nc;
        hsm[cc * TM + m] = (m < tm) ? h[(size_t)(g0 + m) * ldh + c0 + cc] : 0.0f;
      }
      __syncthreads();
      const T* wr = wsm + r * WSTR;
      for (int i = 0; i < nc / 8; ++i) {
        float w = WTraits<WT>::cvt(wr[8 * i + j]);
        const float* hv = hsm + (8 * i + j) * TM;
#pragma unroll
        for (int m = 0; m < TM; ++m) acc[m] = __fmaf_rn(w, hv[m], acc[m]);
      }
    }
    // hsum tree across the eight chain threads of each row (lanes 8k..8k+7).
#pragma unroll
    for (int m = 0; m < TM; ++m) {
      float a = acc[m];
      float s = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 4));   // j<4: a_j + a_{j+4}
      float u = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, 1));   // j=0: s0+s1, j=2: s2+s3
      float res = __fadd_rn(u, __shfl_xor_sync(0xffffffffu, u, 2)); // j=0: (s0+s1)+(s2+s3)
      if (j == 0 && m < tm && v < V) {
        const float* hrow = h + (size_t)(g0 + m) * ldh;
        for (int c = Hm; c < H; ++c)
          res = __fadd_rn(res, __fmul_rn(WTraits<WT>::cvt(W[(size_t)v * H + c]), hrow[c]));
        if (WT == LmW::I8) res = __fmul_rn(res, scales[v]);
        out[(size_t)(g0 + m) * ldo + v] = res;
      }
    }
  }
}

template <LmW WT>
static void run_lm(const void* W, const float* scales, const float* h, int ldh, int M, int V, int H, float* out,
                   int ldo, cudaStream_t st) {
  using T = typename WTraits<WT>::T;
  dim3 grid((unsigned)ceil_div(V, WTraits<WT>::ROWS));
  if (M == 1)
    lm_head_kernel<WT, 1><<<grid, 256, 0, st>>>((const T*)W, scales, h, ldh, M, V, H, out, ldo);
  else if (M <= 4)
    lm_head_kernel<WT, 4><<<grid, 256, 0, st>>>((const T*)W, scales, h, ldh, M, V, H, out, ldo);
  else
    lm_head_kernel<WT, 8><<<grid, 256, 0, st>>>((const T*)W, scales, h, ldh, M, V, H, out, ldo);
  count_launch();
}

void launch_lm_head(const void* W, LmW wt, const float* scales, const float* h, int ldh, int M, int V, int H,
                    float* out, int ldo, cudaStream_t st) {
  if (M <= 0 || V <= 0) return;
  switch (wt) {
    case LmW::I8: run_lm<LmW::I8>(W, scales, h, ldh, M, V, H, out, ldo, st); break;
    case LmW::BF16: run_lm<LmW::BF16>(W, scales, h, ldh, M, V, H, out, ldo, st); break;
    case LmW::F32: run_lm<LmW::F32>(W, scales, h, ldh, M, V, H, out, ldo, st); break;
  }
}

// ---------------------------------------------------------------------------
// Tensor-core lm_head for many tokens: logits = (W_i8 . h) * scale.
// h (f32) is split into three bf16 terms h1 + h2 + h3 (h1 = bf16(h),
// h2 = bf16(h - h1), h3 = bf16(h - h1 - h2)), which represent h to 2^-27
// relative; int8 weights are exact in bf16, so every product the tensor core
// forms is exact and only the f32 accumulation order differs from the
// reference's FMA chains.  A' = [h1 | h2 | h3] is [M][3H] bf16.
// ---------------------------------------------------------------------------
__global__ void split_bf16x3_kernel(const float* __restrict__ h, int H, uint16_t* __restrict__ a3) {
  const int m = blockIdx.x;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float x = h[(size_t)m * H + i];
    uint16_t b1 = f32_to_bf16_bits(x);
    float r1 = x - bf16_bits_to_f32(b1);
    uint16_t b2 = f32_to_bf16_bits(r1);
    float r2 = r1 - bf16_bits_to_f32(b2);
    uint16_t b3 = f32_to_bf16_bits(r2);
    uint16_t* row = a3 + (size_t)m * 3 * H;
    row[i] = b1;
    row[H + i] = b2;
    row[2 * H + i] = b3;
  }
}

__device__ __forceinline__ void cpa16(void* smem_dst, const void* gsrc, int bytes) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gsrc), "r"(bytes));
}
__device__ __forceinline__ void ldsm4(uint32_t r[4], const void* p) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}
__device__ __forceinline__ void mma16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Two int8 (consecutive bytes of a 16-bit word) -> packed bf16x2 (exact).
__device__ __forceinline__ uint32_t i8x2_to_bf16x2(uint32_t w16) {
  float lo = (float)(int8_t)(w16 & 0xff), hi = (float)(int8_t)((w16 >> 8) & 0xff);
  return (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xffff0000u);
}

// Block tile 64 tokens x 128 vocab rows x 64 k; 8 warps as 2 (M) x 4 (N), warp tile 32 x 32.
constexpr int kLmBM = 64, kLmBN = 128, kLmBK = 64, kLmStages = 3;
constexpr int kLmAS = kLmBK * 2 + 16;  // A smem row: 64 bf16 + 16 B pad
constexpr int kLmWS = kLmBK + 16;      // W smem row: 64 int8 + 16 B pad

__global__ void __launch_bounds__(256) lm_head_mma_kernel(const uint16_t* __restrict__ a3, const int8_t* __restrict__ W,
                                                          const float* __restrict__ scales, int M, int V, int H,
                                                          float* __restrict__ out, int ldo) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* as = smem;                                    // [stages][BM][kLmAS]
  uint8_t* ws = smem + kLmStages * kLmBM * kLmAS;       // [stages][BN][kLmWS]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int wm = warp >> 2, wn = warp & 3;
  const int m0 = blockIdx.x * kLmBM, n0 = blockIdx.y * kLmBN;
  const int K3 = 3 * H;
  const int ktiles = K3 / kLmBK;  // H % 64 == 0 (checked by the launcher)

  auto load = [&](int stage, int kt) {
    const int k = kt * kLmBK;
    // A': 64 rows x 128 B
    for (int c = threadIdx.x; c < kLmBM * 8; c += 256) {
      int r = c >> 3, sg = c & 7;
      int gm = m0 + r;
      const uint16_t* src = a3 + (size_t)min(gm, M - 1) * K3 + k + sg * 8;
      cpa16(as + (stage * kLmBM + r) * kLmAS + sg * 16, src, gm < M ? 16 : 0);
    }
    // W: 128 rows x 64 B (k mod H)
    const int kw = k % H;
    for (int c = threadIdx.x; c < kLmBN * 4; c += 256) {
      int r = c >> 2, sg = c & 3;
      int gv = n0 + r;
      const int8_t* src = W + (size_t)min(gv, V - 1) * H + kw + sg * 16;
      cpa16(ws + (stage * kLmBN + r) * kLmWS + sg * 16, src, gv < V ? 16 : 0);
    }
  };

  float acc[2][4][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = acc[i][j][2] = acc[i][j][3] = 0.0f;

#pragma unroll
  for (int s = 0; s < kLmStages - 1; ++s) {
    if (s < ktiles) load(s, s);
    asm volatile("cp.async.commit_group;\n" ::);
  }
  for (int kt = 0; kt < ktiles; ++kt) {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(kLmStages - 2));
    __syncthreads();
    if (kt + kLmStages - 1 < ktiles) load((kt + kLmStages - 1) % kLmStages, kt + kLmStages - 1);
    asm volatile("cp.async.commit_group;\n" ::);
    const uint8_t* ast = as + (kt % kLmStages) * kLmBM * kLmAS;
    const uint8_t* wst = ws + (kt % kLmStages) * kLmBN * kLmWS;
#pragma unroll
    for (int ks = 0; ks < kLmBK / 16; ++ks) {
      uint32_t a[2][4];
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        int row = wm * 32 + mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        ldsm4(a[mt], ast + row * kLmAS + ks * 32 + (lane >> 4) * 16);
      }
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const uint8_t* wr = wst + (wn * 32 + nt * 8 + (lane >> 2)) * kLmWS + ks * 16 + 2 * (lane & 3);
        uint32_t b0 = i8x2_to_bf16x2(*reinterpret_cast<const uint16_t*>(wr));
        uint32_t b1 = i8x2_to_bf16x2(*reinterpret_cast<const uint16_t*>(wr + 8));
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) mma16816(acc[mt][nt], a[mt], b0, b1);
      }
    }
  }
  asm volatile("cp.async.wait_group 0;\n" ::);
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      int m = m0 + wm * 32 + mt * 16 + (lane >> 2) + 8 * half;
      if (m >= M) continue;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          int v = n0 + wn * 32 + nt * 8 + 2 * (lane & 3) + e;
          if (v < V) out[(size_t)m * ldo + v] = acc[mt][nt][2 * half + e] * scales[v];
        }
    }
}

bool lm_head_mma_supported(int H) { return H % kLmBK == 0; }

int lm_head_mma_prepare() {
  int smem = kLmStages * (kLmBM * kLmAS + kLmBN * kLmWS);
  return cudaFuncSetAttribute(lm_head_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) == cudaSuccess
             ? 0
             : 1;
}

void launch_lm_head_mma(const float* h, int M, int V, int H, const int8_t* W, const float* scales, uint16_t* a3,
                        float* out, int ldo, cudaStream_t st, int32_t* status) {
  if (M <= 0 || V <= 0) return;
  split_bf16x3_kernel<<<M, 256, 0, st>>>(h, H, a3);
  // tcgen05 kernel (same exact products, f32 sums in the tensor core's order)
  if (status && ternary_tc_ready() && lm_head_tc_supported(H) &&
      launch_lm_head_tc(a3, M, V, H, W, scales, out, ldo, status, st) == 0) {
    count_launch();  // the split kernel
    return;
  }
  int smem = kLmStages * (kLmBM * kLmAS + kLmBN * kLmWS);
  dim3 grid((unsigned)ceil_div(M, kLmBM), (unsigned)ceil_div(V, kLmBN));
  lm_head_mma_kernel<<<grid, 256, smem, st>>>(a3, W, scales, M, V, H, out, ldo);
  count_launch(2);
}

// ---------------------------------------------------------------------------
// Greedy argmax with Iterator::max_by(partial_cmp) semantics
// (inference/lib.rs:263-274): a NaN compares Equal, so the fold restarts
// after the last NaN; among the rest the last maximal index wins.
// State of a contiguous segment: last NaN index (-1: none) and the best
// (value, index) of the suffix after it (index -1: empty suffix).
// ---------------------------------------------------------------------------
struct ArgState {
  int nan_idx;
  int best_idx;
  float best_val;
};

__device__ __forceinline__ ArgState arg_combine(const ArgState& a, const ArgState& b) {  // a precedes b
  if (b.nan_idx >= 0) return b;
  ArgState r;
  r.nan_idx = a.nan_idx;
  if (b.best_idx < 0) {
    r.best_idx = a.best_idx;
    r.best_val = a.best_val;
  } else if (a.best_idx < 0 || !(a.best_val > b.best_val)) {
    r.best_idx = b.best_idx;
    r.best_val = b.best_val;
  } else {
    r.best_idx = a.best_idx;
    r.best_val = a.best_val;
  }
  return r;
}

__global__ void argmax_kernel(const float* __restrict__ logits, int ldl, int V, uint32_t* __restrict__ out) {
  __shared__ ArgState sm[32];
  const int m = blockIdx.x;
  const float* x = logits + (size_t)m * ldl;
  const int per = (V + blockDim.x - 1) / blockDim.x;
  const int b = threadIdx.x * per, e = min(V, b + per);
  ArgState s{-1, -1, 0.0f};
  for (int i = b; i < e; ++i) {
    float v = x[i];
    if (isnan(v)) {
      s.nan_idx = i;
      s.best_idx = -1;
    } else if (s.best_idx < 0 || !(s.best_val > v)) {
      s.best_idx = i;
      s.best_val = v;
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 1; o < 32; o <<= 1) {
    ArgState t;
    t.nan_idx = __shfl_down_sync(0xffffffffu, s.nan_idx, o);
    t.best_idx = __shfl_down_sync(0xffffffffu, s.best_idx, o);
    t.best_val = __shfl_down_sync(0xffffffffu, s.best_val, o);
    if ((lane & (2 * o - 1)) == 0 && lane + o < 32) s = arg_combine(s, t);
  }
  if (lane == 0) sm[warp] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    ArgState r = sm[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) r = arg_combine(r, sm[w]);
    uint32_t tok = r.best_idx >= 0 ? (uint32_t)r.best_idx : (r.nan_idx >= 0 ? (uint32_t)r.nan_idx : 0u);
    out[m] = tok;
  }
}

void launch_argmax(const float* logits, int ldl, int M, int V, uint32_t* out, cudaStream_t st) {
  if (M <= 0) return;
  argmax_kernel<<<M, 1024, 0, st>>>(logits, ldl, V, out);
  count_launch();
}

// ---------------------------------------------------------------------------
// One-row int8 lm_head with the greedy argmax folded in (decode at batch 1).
// Lane l of warp w owns vocabulary row v = 128 * block + 32 w + l and runs all
// eight of the reference's FMA chains of that row (dot_f32_i8w_avx2: chain j
// takes columns 8 i + j, i = 0, 1, ... in order), then hsum_f32_avx2 and the
// scale, as lm_head_kernel does.  The warp's 32 rows stream through three
// 4 KiB TMA stages (32 rows x 128 columns, 128-byte swizzle), so each lane
// reads its row's 16-byte chunks conflict-free.  int8 -> f32 is exact: the
// byte + 128 is placed in the mantissa of 2^23 and 2^23 + 128 subtracted.
// Each block leaves the ordered argmax state of its 128 rows; argmax1_kernel
// combines the blocks in order (same ties and NaN rule as argmax_kernel).
// ---------------------------------------------------------------------------
namespace {
constexpr int kL1Warps = 4;
constexpr int kL1Rows = 32 * kL1Warps;  // rows per block
constexpr int kL1Stages = 3;  // 3 x 4 warps x 4 KiB + the row: three blocks per SM
constexpr int kL1Tile = 32 * 128;       // bytes per stage: 32 rows x 128 columns
constexpr long long kL1WaitCycles = 2000000000LL;

__device__ __forceinline__ uint32_t l1_smem(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ bool l1_wait(uint32_t bar, uint32_t parity) {
  const long long t0 = clock64();
  for (;;) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
    if (clock64() - t0 > kL1WaitCycles) return false;
  }
}
__device__ __forceinline__ float i8_to_f32(uint32_t u, int k) {  // u = word ^ 0x80808080
  return __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540u | (uint32_t)k)), 8388736.0f);
}
}  // namespace

__global__ void __launch_bounds__(kL1Warps * 32) lm_head_m1_kernel(const __grid_constant__ CUtensorMap tmap,
                                                                   const float* __restrict__ h,
                                                                   const float* __restrict__ scales, int V, int H,
                                                                   float* __restrict__ out, ArgState* __restrict__ part,
                                                                   int32_t* status) {
  extern __shared__ uint8_t l1_raw[];
  __shared__ __align__(8) uint64_t bar[kL1Warps][kL1Stages];
  __shared__ ArgState wst[kL1Warps];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t raw = l1_smem(l1_raw);
  uint8_t* base = l1_raw + ((1024u - (raw & 1023u)) & 1023u);  // 1024-aligned (128-byte swizzle)
  float* hs = reinterpret_cast<float*>(base + kL1Warps * kL1Stages * kL1Tile);
  const int v0 = blockIdx.x * kL1Rows + warp * 32, nst = H / 128;
  if (lane == 0) {
    for (int s = 0; s < kL1Stages; ++s)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(l1_smem(&bar[warp][s])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  for (int i = tid; i < (H >> 2); i += kL1Warps * 32) reinterpret_cast<float4*>(hs)[i] = reinterpret_cast<const float4*>(h)[i];
  __syncthreads();
  const uint32_t tiles = l1_smem(base) + (uint32_t)(warp * kL1Stages * kL1Tile);
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(pol));
  int issued = 0;  // lane 0: stages issued
  auto issue = [&](int s) {
    const uint32_t b = l1_smem(&bar[warp][s % kL1Stages]);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(b), "r"(kL1Tile) : "memory");
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;\n" ::"r"(tiles + (uint32_t)((s % kL1Stages) * kL1Tile)),
        "l"((uint64_t)&tmap), "r"(128 * s), "r"(v0), "r"(b), "l"(pol)
        : "memory");
    ++issued;
  };
  if (lane == 0)
    for (int s = 0; s < min(kL1Stages, nst); ++s) issue(s);
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
  bool ok = true;
  const uint32_t hs_s = l1_smem(hs);
  for (int s = 0; s < nst; ++s) {
    ok = __all_sync(0xffffffffu, l1_wait(l1_smem(&bar[warp][s % kL1Stages]), (uint32_t)(s / kL1Stages) & 1u));
    if (!ok) break;
    const uint32_t tb = tiles + (uint32_t)((s % kL1Stages) * kL1Tile) + (uint32_t)lane * 128u;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint4 w;
      asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];\n"
                   : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w)
                   : "r"(tb + ((uint32_t)(c ^ (lane & 7)) << 4)));
      const uint32_t ww[4] = {w.x ^ 0x80808080u, w.y ^ 0x80808080u, w.z ^ 0x80808080u, w.w ^ 0x80808080u};
      // groups 16 s + 2 c (words 0, 1) and 16 s + 2 c + 1 (words 2, 3)
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        float4 h0, h1;
        const uint32_t ha = hs_s + (uint32_t)((128 * s + 16 * c + 8 * g) * 4);
        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];\n" : "=f"(h0.x), "=f"(h0.y), "=f"(h0.z), "=f"(h0.w) : "r"(ha));
        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];\n" : "=f"(h1.x), "=f"(h1.y), "=f"(h1.z), "=f"(h1.w) : "r"(ha + 16));
        const float hv[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = __fmaf_rn(i8_to_f32(ww[2 * g + (j >> 2)], j & 3), hv[j], acc[j]);
      }
    }
    __syncwarp();  // every lane has read the stage before it is refilled
    if (lane == 0 && s + kL1Stages < nst) issue(s + kL1Stages);
  }
  if (!ok) {
    if (lane == 0) {
      atomicOr(status, kStatusWaitTimeout);
      for (int s = 0; s < issued; ++s)  // let issued copies land (bounded) before the CTA exits
        if (!l1_wait(l1_smem(&bar[warp][s % kL1Stages]), (uint32_t)(s / kL1Stages) & 1u)) break;
    }
    return;
  }
  const int v = v0 + lane;
  ArgState st{-1, -1, 0.0f};
  if (v < V) {
    const float res = __fmul_rn(hsum8(acc), scales[v]);
    out[v] = res;
    if (isnan(res))
      st.nan_idx = v;
    else {
      st.best_idx = v;
      st.best_val = res;
    }
  }
  for (int o = 1; o < 32; o <<= 1) {
    ArgState t;
    t.nan_idx = __shfl_down_sync(0xffffffffu, st.nan_idx, o);
    t.best_idx = __shfl_down_sync(0xffffffffu, st.best_idx, o);
    t.best_val = __shfl_down_sync(0xffffffffu, st.best_val, o);
    if ((lane & (2 * o - 1)) == 0 && lane + o < 32) st = arg_combine(st, t);
  }
  if (lane == 0) wst[warp] = st;
  __syncthreads();
  if (tid == 0) {
    ArgState r = wst[0];
    for (int w = 1; w < kL1Warps; ++w) r = arg_combine(r, wst[w]);
    part[blockIdx.x] = r;
  }
}

// The argmax of the blocks' states, combined in block order.
__global__ void argmax1_kernel(const ArgState* __restrict__ part, int n, uint32_t* __restrict__ out) {
  __shared__ ArgState sm[32];
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int b = threadIdx.x * per, e = min(n, b + per);
  ArgState s{-1, -1, 0.0f};
  for (int i = b; i < e; ++i) s = arg_combine(s, part[i]);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int o = 1; o < 32; o <<= 1) {
    ArgState t;
    t.nan_idx = __shfl_down_sync(0xffffffffu, s.nan_idx, o);
    t.best_idx = __shfl_down_sync(0xffffffffu, s.best_idx, o);
    t.best_val = __shfl_down_sync(0xffffffffu, s.best_val, o);
    if ((lane & (2 * o - 1)) == 0 && lane + o < 32) s = arg_combine(s, t);
  }
  if (lane == 0) sm[warp] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    ArgState r = sm[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) r = arg_combine(r, sm[w]);
    out[0] = r.best_idx >= 0 ? (uint32_t)r.best_idx : (r.nan_idx >= 0 ? (uint32_t)r.nan_idx : 0u);
  }
}

bool lm_head_m1_supported(int H, int V) { return H > 0 && H % 128 == 0 && H <= 16384 && V > 0; }
size_t lm_head_m1_parts(int V) { return (size_t)ceil_div((size_t)V, (size_t)kL1Rows); }
size_t lm_head_m1_part_bytes(int V) { return lm_head_m1_parts(V) * sizeof(ArgState); }
static size_t lm_head_m1_smem(int H) { return 1024 + (size_t)kL1Warps * kL1Stages * kL1Tile + (size_t)H * 4; }

int lm_head_m1_prepare(int H) {
  return cudaFuncSetAttribute(lm_head_m1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lm_head_m1_smem(H)) ==
                 cudaSuccess
             ? 0
             : 1;
}

// The int8 table [V][H] as a 2-D tensor: x = column (H), y = row (V); a box
// of 128 x 32 is one stage.
int lm_head_m1_make_tmap(const int8_t* W, int V, int H, CUtensorMap* map) {
  if (!lm_head_m1_supported(H, V) || reinterpret_cast<uintptr_t>(W) % 16) return 1;
  auto enc = tensor_map_encoder();
  if (!enc) return 1;
  const cuuint64_t dims[2] = {(cuuint64_t)H, (cuuint64_t)V};
  const cuuint64_t strides[1] = {(cuuint64_t)H};
  const cuuint32_t box[2] = {128, 32};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(W), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : 1;
}

void launch_lm_head_m1(const CUtensorMap& map, const float* h, const float* scales, int V, int H, float* out,
                       void* part, uint32_t* next, int32_t* status, cudaStream_t st) {
  const unsigned blocks = (unsigned)lm_head_m1_parts(V);
  lm_head_m1_kernel<<<blocks, kL1Warps * 32, lm_head_m1_smem(H), st>>>(map, h, scales, V, H, out,
                                                                        reinterpret_cast<ArgState*>(part), status);
  argmax1_kernel<<<1, 1024, 0, st>>>(reinterpret_cast<const ArgState*>(part), (int)blocks, next);
  count_launch(2);
}

}  // namespace bitnet
