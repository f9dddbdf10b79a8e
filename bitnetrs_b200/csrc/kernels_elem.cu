// kernels_elem.cu — weight repack, activation quantisation, RMSNorm and the
// elementwise ops of the bitnetrs hot path.
#include "kernels.cuh"

#include <atomic>

namespace bitnet {

static std::atomic<uint64_t> g_launches{0};
void count_launch(uint64_t n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
void uncount_launch(uint64_t n) { g_launches.fetch_sub(n, std::memory_order_relaxed); }
uint64_t launches_total() { return g_launches.load(std::memory_order_relaxed); }

// ---------------------------------------------------------------------------
// Repack (one thread per 32-bit output word).
// ---------------------------------------------------------------------------
__global__ void repack_ternary_kernel(const uint8_t* __restrict__ src, uint32_t* __restrict__ dst, int rows, int cols,
                                      int pc, int kw) {
  size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (size_t)rows * kw) return;
  int r = (int)(idx / kw), g = (int)(idx % kw);
  uint32_t word = 0;
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    int k = 16 * g + e;
    uint32_t code = 1;  // padding columns: weight 0
    if (k < cols) {
      code = (src[(size_t)r * pc + (k >> 2)] >> (2 * (k & 3))) & 3u;
      if (code == 3) code = 1;  // DECODE_LUT maps the invalid code to 0
    }
    word |= code << (8 * (e & 3) + 2 * (e >> 2));
  }
  dst[idx] = word;
}

void launch_repack_ternary(const uint8_t* src, uint32_t* dst, int rows, int cols, cudaStream_t st) {
  int pc = (cols + 3) / 4, kw = (int)words_per_row(cols);
  size_t n = (size_t)rows * kw;
  repack_ternary_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(src, dst, rows, cols, pc, kw);
  count_launch();
}

// ---------------------------------------------------------------------------
// absmax quantisation of one row held in shared memory (absmax.rs:127-165).
// Called by the whole block; y is the row (length d).
// ---------------------------------------------------------------------------
__device__ void quantize_row_smem(const float* y, int d, int8_t* xq_row, int ldq, float* act_absmax, float* scale_out,
                                  int32_t* row_sum, int32_t* status, float* red_f, int* red_i) {
  float mx = 0.0f;
  int bad = 0;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    float v = y[i];
    if (!isfinite(v)) bad = 1;
    mx = fmaxf(mx, fabsf(v));
  }
  mx = block_reduce(mx, [](float a, float b) { return fmaxf(a, b); }, red_f);
  bad = block_reduce(bad, [](int a, int b) { return a | b; }, red_i);
  float mc = fmaxf(mx, 1e-5f);
  float scale = __fdiv_rn(mc, 127.0f);
  float inv = __fdiv_rn(127.0f, mc);
  int sum = 0;
  for (int i = threadIdx.x; i < ldq; i += blockDim.x) {
    int8_t q = 0;
    if (i < d) q = quant_i8(y[i], inv);
    xq_row[i] = q;
    sum += q;
  }
  sum = block_reduce(sum, [](int a, int b) { return a + b; }, red_i);
  if (threadIdx.x == 0) {
    if (act_absmax) *act_absmax = __fmul_rn(scale, 127.0f);
    if (scale_out) *scale_out = scale;
    if (row_sum) *row_sum = sum;
    if (bad && status) atomicOr(status, 1);
  }
}

template <bool BF16>
__global__ void quantize_rows_kernel(const void* __restrict__ xv, int ldx, int K, int8_t* __restrict__ xq, int ldq,
                                     float* act_absmax, float* scale, int32_t* row_sum, int32_t* status) {
  extern __shared__ float row[];
  __shared__ float red_f[32];
  __shared__ int red_i[32];
  int m = blockIdx.x;
  for (int i = threadIdx.x; i < K; i += blockDim.x) {
    if (BF16)
      row[i] = bf16_bits_to_f32(((const uint16_t*)xv)[(size_t)m * ldx + i]);
    else
      row[i] = ((const float*)xv)[(size_t)m * ldx + i];
  }
  __syncthreads();
  quantize_row_smem(row, K, xq + (size_t)m * ldq, ldq, act_absmax ? act_absmax + m : nullptr,
                    scale ? scale + m : nullptr, row_sum ? row_sum + m : nullptr, status, red_f, red_i);
}

void launch_quantize_rows(const void* x, bool x_bf16, int ldx, int M, int K, int8_t* xq, int ldq, float* act_absmax,
                          float* scale, int32_t* row_sum, int32_t* status, cudaStream_t st) {
  if (M <= 0) return;
  size_t smem = (size_t)K * sizeof(float);
  if (x_bf16)
    quantize_rows_kernel<true><<<M, 256, smem, st>>>(x, ldx, K, xq, ldq, act_absmax, scale, row_sum, status);
  else
    quantize_rows_kernel<false><<<M, 256, smem, st>>>(x, ldx, K, xq, ldq, act_absmax, scale, row_sum, status);
  count_launch();
}

// ---------------------------------------------------------------------------
// RMSNorm, reference order (norm.rs:113-137, simd.rs:802-826):
//   sum_sq = hsum8(8 FMA chains over chunks of 8) + sequential scalar tail
//   inv = 1 / sqrt(sum_sq / d + eps);  out = (x * inv) * w
// Lanes 0..7 of warp 0 run the eight chains; the result is broadcast.
// ---------------------------------------------------------------------------
__device__ float rms_inv_exact(const float* x, int d, float eps, float* bcast) {
  if (threadIdx.x < 32) {
    int lane = threadIdx.x;
    int chunks = d >> 3;
    float acc = 0.0f;
    if (lane < 8) {
      int i = 0;
      for (; i + 16 <= chunks; i += 16) {
        float v[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) v[u] = x[8 * (i + u) + lane];
#pragma unroll
        for (int u = 0; u < 16; ++u) acc = __fmaf_rn(v[u], v[u], acc);
      }
      for (; i < chunks; ++i) {
        float a = x[8 * i + lane];
        acc = __fmaf_rn(a, a, acc);
      }
    }
    float a[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] = __shfl_sync(0xffffffffu, acc, j);
    if (lane == 0) {
      float ss = hsum8(a);
      for (int i = chunks * 8; i < d; ++i) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
      float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)d), eps));
      *bcast = __fdiv_rn(1.0f, rms);
    }
  }
  __syncthreads();
  return *bcast;
}

__global__ void rms_norm_kernel(const float* __restrict__ x, int ldx, const float* __restrict__ w, int d, float eps,
                                float* __restrict__ out, int ldo) {
  extern __shared__ float row[];
  __shared__ float bc;
  int m = blockIdx.x;
  for (int i = threadIdx.x; i < d; i += blockDim.x) row[i] = x[(size_t)m * ldx + i];
  __syncthreads();
  float inv = rms_inv_exact(row, d, eps, &bc);
  for (int i = threadIdx.x; i < d; i += blockDim.x) out[(size_t)m * ldo + i] = __fmul_rn(__fmul_rn(row[i], inv), w[i]);
}

void launch_rms_norm(const float* x, int ldx, const float* w, int d, float eps, float* out, int ldo, int M,
                     cudaStream_t st) {
  if (M <= 0 || d <= 0) return;
  rms_norm_kernel<<<M, 256, (size_t)d * sizeof(float), st>>>(x, ldx, w, d, eps, out, ldo);
  count_launch();
}

// One block per row: the row (or sqrelu(gate)*up) is staged in shared
// memory by all threads, lanes 0..7 of warp 0 run the reference's eight FMA
// chains from there, then the block forms y = (x * inv) * w, its absmax and
// the int8 row (absmax.rs:127-165).
template <bool GATE_UP>
__global__ void __launch_bounds__(256) norm_quant_kernel(const float* __restrict__ x, const float* __restrict__ x2,
                                                         int ldx, const float* __restrict__ w, int d, float eps,
                                                         int8_t* __restrict__ xq, int ldq, float* __restrict__ act_absmax,
                                                         int32_t* __restrict__ row_sum, int32_t* status) {
  extern __shared__ float row[];
  __shared__ float bc;
  __shared__ float red_f[32];
  __shared__ int red_i[32];
  pdl_launch_dependents();
  pdl_wait();
  x = after_wait(x);
  if (GATE_UP) x2 = after_wait(x2);
  const int m = blockIdx.x;
  const float* xr = x + (size_t)m * ldx;
  const bool vec = (d & 3) == 0 && (ldx & 3) == 0 && ((uintptr_t)x & 15) == 0 && (!GATE_UP || ((uintptr_t)x2 & 15) == 0);
  if (vec) {
    const float4* x4 = reinterpret_cast<const float4*>(xr);
    const float4* y4 = GATE_UP ? reinterpret_cast<const float4*>(x2 + (size_t)m * ldx) : nullptr;
    for (int i = threadIdx.x; i < d / 4; i += blockDim.x) {
      float4 v = x4[i];
      if (GATE_UP) {
        float4 u = y4[i];
        float r0 = fmaxf(v.x, 0.0f), r1 = fmaxf(v.y, 0.0f), r2 = fmaxf(v.z, 0.0f), r3 = fmaxf(v.w, 0.0f);
        v = make_float4(__fmul_rn(__fmul_rn(r0, r0), u.x), __fmul_rn(__fmul_rn(r1, r1), u.y),
                        __fmul_rn(__fmul_rn(r2, r2), u.z), __fmul_rn(__fmul_rn(r3, r3), u.w));
      }
      reinterpret_cast<float4*>(row)[i] = v;
    }
  } else {
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
      float v = xr[i];
      if (GATE_UP) {
        float r = fmaxf(v, 0.0f);  // f32::max(0.0): NaN -> 0
        v = __fmul_rn(__fmul_rn(r, r), x2[(size_t)m * ldx + i]);
      }
      row[i] = v;
    }
  }
  __syncthreads();
  float inv = rms_inv_exact(row, d, eps, &bc);
  for (int i = threadIdx.x; i < d; i += blockDim.x) row[i] = __fmul_rn(__fmul_rn(row[i], inv), w[i]);
  __syncthreads();
  quantize_row_smem(row, d, xq + (size_t)m * ldq, ldq, act_absmax + m, nullptr, row_sum + m, status, red_f, red_i);
}

// Register-resident variant for rows of at most 8192 values with 256 threads
// or 16384 with 512 (d % 4 == 0): thread t holds float4 groups t, t + NT, ...
// of the row. The norm weights
// (no kernel writes them) are loaded before griddepcontrol.wait; lanes 0..7 of
// warp 0 run the eight FMA chains from a shared copy of the row, their
// shared-memory loads issued one block of 16 ahead; the rest of the block then
// normalises, takes the absmax and quantises from registers. Same operations
// and order as norm_quant_kernel.
template <bool GATE_UP, int U, int NT>
__global__ void __launch_bounds__(NT) norm_quant_reg_kernel(const float* __restrict__ x, const float* __restrict__ x2,
                                                             int ldx, const float* __restrict__ w, int d, float eps,
                                                             int8_t* __restrict__ xq, int ldq,
                                                             float* __restrict__ act_absmax,
                                                             int32_t* __restrict__ row_sum, int32_t* status) {
  extern __shared__ float4 row4[];  // the row, d / 4 float4
  __shared__ float bc;
  constexpr int NW = NT / 32;
  __shared__ float red_f[NW];
  __shared__ int red_i[NW], red_b[NW];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int m = blockIdx.x, n4 = d >> 2;
  pdl_launch_dependents();
  float4 wv[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int j = t + NT * u;
    wv[u] = j < n4 ? reinterpret_cast<const float4*>(w)[j] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
  pdl_wait();
  x = after_wait(x);
  if (GATE_UP) x2 = after_wait(x2);
  const float4* x4 = reinterpret_cast<const float4*>(x + (size_t)m * ldx);
  const float4* y4 = GATE_UP ? reinterpret_cast<const float4*>(x2 + (size_t)m * ldx) : nullptr;
  float4 v[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int j = t + NT * u;
    v[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (j < n4) {
      float4 a = x4[j];
      if (GATE_UP) {
        const float4 b = y4[j];
        const float r0 = fmaxf(a.x, 0.0f), r1 = fmaxf(a.y, 0.0f), r2 = fmaxf(a.z, 0.0f), r3 = fmaxf(a.w, 0.0f);
        a = make_float4(__fmul_rn(__fmul_rn(r0, r0), b.x), __fmul_rn(__fmul_rn(r1, r1), b.y),
                        __fmul_rn(__fmul_rn(r2, r2), b.z), __fmul_rn(__fmul_rn(r3, r3), b.w));
      }
      v[u] = a;
      row4[j] = a;
    }
  }
  __syncthreads();
  if (warp == 0) {
    const float* row = reinterpret_cast<const float*>(row4);
    const int chunks = d >> 3;
    float acc = 0.0f;
    if (lane < 8) {
      // two 16-element register blocks in turn: one block's loads are in
      // flight while the other's FMAs run, with no register copies in the loop
      const int full = chunks & ~31;
      float ba[16], bb[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) ba[k] = full ? row[8 * k + lane] : 0.0f;
      int i = 0;
      for (; i < full; i += 32) {
#pragma unroll
        for (int k = 0; k < 16; ++k) bb[k] = row[8 * (i + 16 + k) + lane];
#pragma unroll
        for (int k = 0; k < 16; ++k) acc = __fmaf_rn(ba[k], ba[k], acc);
        const int ni = i + 32 < full ? i + 32 : i;
#pragma unroll
        for (int k = 0; k < 16; ++k) ba[k] = row[8 * (ni + k) + lane];
#pragma unroll
        for (int k = 0; k < 16; ++k) acc = __fmaf_rn(bb[k], bb[k], acc);
      }
      for (; i < chunks; ++i) {
        const float a = row[8 * i + lane];
        acc = __fmaf_rn(a, a, acc);
      }
    }
    float a[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] = __shfl_sync(0xffffffffu, acc, j);
    if (lane == 0) {
      float ss = hsum8(a);
      for (int i = chunks * 8; i < d; ++i) ss = __fadd_rn(ss, __fmul_rn(row[i], row[i]));
      const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)d), eps));
      bc = __fdiv_rn(1.0f, rms);
    }
  }
  __syncthreads();
  const float inv = bc;
  float mx = 0.0f;
  int bad = 0;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    if (t + NT * u < n4) {
      float4 a = v[u];
      a.x = __fmul_rn(__fmul_rn(a.x, inv), wv[u].x);
      a.y = __fmul_rn(__fmul_rn(a.y, inv), wv[u].y);
      a.z = __fmul_rn(__fmul_rn(a.z, inv), wv[u].z);
      a.w = __fmul_rn(__fmul_rn(a.w, inv), wv[u].w);
      v[u] = a;
      bad |= !isfinite(a.x) || !isfinite(a.y) || !isfinite(a.z) || !isfinite(a.w);
      mx = fmaxf(fmaxf(fmaxf(mx, fabsf(a.x)), fmaxf(fabsf(a.y), fabsf(a.z))), fabsf(a.w));
    }
  }
  mx = warp_max(mx);
  bad = __any_sync(0xffffffffu, bad);
  if (lane == 0) {
    red_f[warp] = mx;
    red_b[warp] = bad;
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < NW; ++k) {
    mx = fmaxf(mx, red_f[k]);
    bad |= red_b[k];
  }
  const float mc = fmaxf(mx, 1e-5f);
  const float scale = __fdiv_rn(mc, 127.0f), qinv = __fdiv_rn(127.0f, mc);
  int8_t* q = xq + (size_t)m * ldq;
  int sum = 0;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int j = t + NT * u;
    if (j < n4) {
      const int8_t c0 = quant_i8(v[u].x, qinv), c1 = quant_i8(v[u].y, qinv), c2 = quant_i8(v[u].z, qinv),
                   c3 = quant_i8(v[u].w, qinv);
      sum += (int)c0 + (int)c1 + (int)c2 + (int)c3;
      reinterpret_cast<char4*>(q)[j] = make_char4(c0, c1, c2, c3);
    }
  }
  for (int i = d + t; i < ldq; i += NT) q[i] = 0;  // K padding of the int8 row
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) red_i[warp] = sum;
  __syncthreads();
  if (t == 0) {
    int total = 0;
#pragma unroll
    for (int k = 0; k < NW; ++k) total += red_i[k];
    act_absmax[m] = __fmul_rn(scale, 127.0f);
    row_sum[m] = total;
    if (bad && status) atomicOr(status, 1);
  }
}

template <bool GATE_UP>
static bool launch_norm_quant_reg(const float* x, const float* x2, int ldx, const float* w, int d, float eps,
                                  int8_t* xq, int ldq, float* act_absmax, int32_t* row_sum, int32_t* status, int M,
                                  cudaStream_t st) {
  const int n4 = d / 4, U = (n4 + 255) / 256, U2 = (n4 + 511) / 512;
  const bool ok = d % 4 == 0 && ldx % 4 == 0 && ldq % 4 == 0 && U >= 1 && U2 <= 8 &&
                  ((uintptr_t)x & 15) == 0 && (!GATE_UP || ((uintptr_t)x2 & 15) == 0) && ((uintptr_t)w & 15) == 0 &&
                  ((uintptr_t)xq & 3) == 0;
  if (!ok) return false;
  const size_t smem = (size_t)d * sizeof(float);
#define BN_NQ(UU, NTT)                                                                                 \
  case UU:                                                                                             \
    norm_quant_reg_kernel<GATE_UP, UU, NTT><<<M, NTT, smem, st>>>(x, x2, ldx, w, d, eps, xq, ldq,        \
                                                                 act_absmax, row_sum, status);         \
    break;
  if (U <= 8) {
    switch (U) {
      BN_NQ(1, 256)
      BN_NQ(2, 256)
      BN_NQ(3, 256)
      BN_NQ(4, 256)
      BN_NQ(5, 256)
      BN_NQ(6, 256)
      BN_NQ(7, 256)
      BN_NQ(8, 256)
    }
  } else {
    switch (U2) {  // rows of 8193 .. 16384 values: 512 threads
      BN_NQ(5, 512)
      BN_NQ(6, 512)
      BN_NQ(7, 512)
      BN_NQ(8, 512)
    }
  }
#undef BN_NQ
  return true;
}

int row_kernels_prepare() {
  const int bytes = kMaxRowFloats * (int)sizeof(float);
  int bad = 0;
  bad |= cudaFuncSetAttribute(quantize_rows_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess;
  bad |= cudaFuncSetAttribute(quantize_rows_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess;
  bad |= cudaFuncSetAttribute(rms_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess;
  bad |= cudaFuncSetAttribute(norm_quant_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess;
  bad |= cudaFuncSetAttribute(norm_quant_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess;
  // the 512-thread register variants hold rows of up to 16384 floats in shared memory too
  const int big = 16384 * (int)sizeof(float);
  bad |= cudaFuncSetAttribute(norm_quant_reg_kernel<true, 5, 512>, cudaFuncAttributeMaxDynamicSharedMemorySize, big) != cudaSuccess;
  bad |= cudaFuncSetAttribute(norm_quant_reg_kernel<true, 6, 512>, cudaFuncAttributeMaxDynamicSharedMemorySize, big) != cudaSuccess;
  bad |= cudaFuncSetAttribute(norm_quant_reg_kernel<true, 7, 512>, cudaFuncAttributeMaxDynamicSharedMemorySize, big) != cudaSuccess;
  bad |= cudaFuncSetAttribute(norm_quant_reg_kernel<true, 8, 512>, cudaFuncAttributeMaxDynamicSharedMemorySize, big) != cudaSuccess;
  bad |= cudaFuncSetAttribute(norm_quant_reg_kernel<false, 5, 512>, cudaFuncAttributeMaxDynamicSharedMemorySize, big) != cudaSuccess;
  bad |= cudaFuncSetAttribute(norm_quant_reg_kernel<false, 6, 512>, cudaFuncAttributeMaxDynamicSharedMemorySize, big) != cudaSuccess;
  bad |= cudaFuncSetAttribute(norm_quant_reg_kernel<false, 7, 512>, cudaFuncAttributeMaxDynamicSharedMemorySize, big) != cudaSuccess;
  bad |= cudaFuncSetAttribute(norm_quant_reg_kernel<false, 8, 512>, cudaFuncAttributeMaxDynamicSharedMemorySize, big) != cudaSuccess;
  return bad;
}

void launch_norm_quant(const float* x, const float* x2, int ldx, const float* w, int d, float eps, int8_t* xq, int ldq,
                       float* act_absmax, int32_t* row_sum, int32_t* status, int M, cudaStream_t st) {
  if (M <= 0) return;
  count_launch();
  if (x2 ? launch_norm_quant_reg<true>(x, x2, ldx, w, d, eps, xq, ldq, act_absmax, row_sum, status, M, st)
         : launch_norm_quant_reg<false>(x, x2, ldx, w, d, eps, xq, ldq, act_absmax, row_sum, status, M, st))
    return;
  size_t smem = (size_t)d * sizeof(float);
  if (x2)
    norm_quant_kernel<true><<<M, 256, smem, st>>>(x, x2, ldx, w, d, eps, xq, ldq, act_absmax, row_sum, status);
  else
    norm_quant_kernel<false><<<M, 256, smem, st>>>(x, x2, ldx, w, d, eps, xq, ldq, act_absmax, row_sum, status);
}

// ---------------------------------------------------------------------------
// Elementwise ops.
// ---------------------------------------------------------------------------
__global__ void squared_relu_kernel(float* x, size_t n) {
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    float r = fmaxf(x[i], 0.0f);
    x[i] = __fmul_rn(r, r);
  }
}
void launch_squared_relu(float* x, size_t n, cudaStream_t st) {
  if (!n) return;
  squared_relu_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(x, n);
  count_launch();
}

__global__ void sqrelu_gate_kernel(const float* g, const float* u, float* o, size_t n) {
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    float r = fmaxf(g[i], 0.0f);
    o[i] = __fmul_rn(__fmul_rn(r, r), u[i]);
  }
}
void launch_sqrelu_gate(const float* g, const float* u, float* out, size_t n, cudaStream_t st) {
  if (!n) return;
  sqrelu_gate_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(g, u, out, n);
  count_launch();
}

__global__ void elementwise_mul_kernel(const float* a, const float* b, float* o, size_t n) {
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) o[i] = __fmul_rn(a[i], b[i]);
}
void launch_elementwise_mul(const float* a, const float* b, float* out, size_t n, cudaStream_t st) {
  if (!n) return;
  elementwise_mul_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(a, b, out, n);
  count_launch();
}

// softmax (activation.rs:230-255): max, exp(x - max), sequential sum, * 1/sum.
__global__ void softmax_max_exp_kernel(float* x, size_t n, float* out_max, ExpTable et) {
  __shared__ float red[32];
  float m = -INFINITY;
  for (size_t i = threadIdx.x; i < n; i += blockDim.x) m = fmaxf(m, x[i]);
  m = block_reduce(m, [](float a, float b) { return fmaxf(a, b); }, red);
  for (size_t i = threadIdx.x; i < n; i += blockDim.x) x[i] = exp_host_libm(__fsub_rn(x[i], m), et);
  if (threadIdx.x == 0) *out_max = m;
}
__global__ void softmax_sum_kernel(const float* x, size_t n, float* out_inv) {
  float s = 0.0f;
  for (size_t i = 0; i < n; ++i) s = __fadd_rn(s, x[i]);
  *out_inv = __fdiv_rn(1.0f, s);
}
__global__ void softmax_scale_kernel(float* x, size_t n, const float* inv) {
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) x[i] = __fmul_rn(x[i], *inv);
}
void launch_softmax(float* x, size_t n, float* scratch, const ExpTable& et, cudaStream_t st) {
  if (!n) return;
  softmax_max_exp_kernel<<<1, 1024, 0, st>>>(x, n, scratch, et);
  softmax_sum_kernel<<<1, 1, 0, st>>>(x, n, scratch + 1);
  softmax_scale_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(x, n, scratch + 1);
  count_launch(3);
}

__global__ void embed_kernel(const uint16_t* __restrict__ embed, const uint32_t* __restrict__ tokens, int H,
                             float* __restrict__ h, int32_t* status, int vocab) {
  int t = blockIdx.x;
  uint32_t tok = tokens[t];
  if (tok >= (uint32_t)vocab) {
    if (threadIdx.x == 0) atomicOr(status, 2);
    tok = 0;
  }
  const uint16_t* row = embed + (size_t)tok * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) h[(size_t)t * H + i] = bf16_bits_to_f32(row[i]);
}
void launch_embed(const uint16_t* embed, const uint32_t* tokens, int T, int H, float* h, int32_t* status, int vocab,
                  cudaStream_t st) {
  if (T <= 0) return;
  embed_kernel<<<T, 256, 0, st>>>(embed, tokens, H, h, status, vocab);
  count_launch();
}

__global__ void gather_rows_kernel(const float* __restrict__ src, int ld, const int32_t* __restrict__ rows,
                                   float* __restrict__ dst) {
  const float* s = src + (size_t)rows[blockIdx.x] * ld;
  for (int i = threadIdx.x; i < ld; i += blockDim.x) dst[(size_t)blockIdx.x * ld + i] = s[i];
}
void launch_gather_rows(const float* src, int ld, const int32_t* rows, int n, float* dst, cudaStream_t st) {
  if (n <= 0) return;
  gather_rows_kernel<<<n, 256, 0, st>>>(src, ld, rows, dst);
  count_launch();
}

__global__ void exp_candidates_kernel(uint32_t lo, uint32_t hi, uint2* out, uint32_t cap, uint32_t* count,
                                      ExpTable et) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i <= (uint64_t)(hi - lo);
       i += (uint64_t)gridDim.x * blockDim.x) {
    uint32_t u = lo + (uint32_t)i;
    float x = __uint_as_float(u);
    float f;
    if (exp_candidate(x, et, &f)) {
      uint32_t slot = atomicAdd(count, 1u);
      if (slot < cap) out[slot] = make_uint2(u, __float_as_uint(f));
    }
  }
}

void launch_exp_candidates(uint32_t lo, uint32_t hi, uint2* out, uint32_t cap, uint32_t* count, const ExpTable& et,
                           cudaStream_t st) {
  exp_candidates_kernel<<<148 * 16, 256, 0, st>>>(lo, hi, out, cap, count, et);
  count_launch();
}

}  // namespace bitnet
