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

}  // namespace bitnet
