// common.cuh — shared helpers for the bitnetrs B200 backend.
//
// Numerics: every translation unit is compiled with -fmad=false, so a*b+c is
// two IEEE roundings unless __fmaf_rn is written explicitly.  This is what
// makes the kernels bit-identical to the reference's CPU code, where scalar
// Rust never contracts and FMA only appears through _mm256_fmadd_ps.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/bitnet_cuda.h"

namespace bitnet {

// ---------------------------------------------------------------------------
// Host-side error reporting (thread-local last error, BitNetError codes).
// ---------------------------------------------------------------------------
void set_error(int code, const char* fmt, ...);
int shape_error(const std::string& expected, const std::string& got);
int quant_error(const std::string& msg);
int config_error(const std::string& msg);
int backend_error(const std::string& msg);
int cuda_error(cudaError_t e, const char* what);

#define BN_CUDA(call)                                  \
  do {                                                 \
    cudaError_t _e = (call);                           \
    if (_e != cudaSuccess) return cuda_error(_e, #call); \
  } while (0)

#define BN_TRY(call)          \
  do {                        \
    int _rc = (call);         \
    if (_rc != BITNET_OK) return _rc; \
  } while (0)

inline size_t round_up(size_t x, size_t m) { return (x + m - 1) / m * m; }
inline size_t ceil_div(size_t a, size_t b) { return (a + b - 1) / b; }

// Device layout of one ternary tensor [rows, cols]: each row is padded to a
// multiple of 64 columns (16 bytes) and stored as 32-bit words of 16 codes.
// Code c in {0,1,2} stands for the weight 1-c (+1, 0, -1), as in the
// reference format (ternary.rs:266-285); the reference's invalid code 3 is
// rewritten to 1 (zero) at upload, matching DECODE_LUT (simd.rs:390-405).
// Inside a word, element e = 4*i + j of the 16 lives in byte j, bits 2i..2i+1,
// so (word >> 2i) & 0x03030303 yields the codes of elements 4i..4i+3 as four
// consecutive bytes — ready for dp4a / int8 MMA without a lookup table.
inline size_t padded_cols(size_t cols) { return round_up(cols, 64); }
inline size_t words_per_row(size_t cols) { return padded_cols(cols) / 16; }

// ---------------------------------------------------------------------------
// Device helpers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// half::bf16::from_f32: round to nearest even, NaN kept quiet.
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u | 0x00400000u) >> 16);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

// The reference's hsum_f32_avx2 (simd.rs:292-307) over eight lane sums:
// ((a0+a4) + (a1+a5)) + ((a2+a6) + (a3+a7)).
__device__ __forceinline__ float hsum8(const float a[8]) {
  float s0 = __fadd_rn(a[0], a[4]);
  float s1 = __fadd_rn(a[1], a[5]);
  float s2 = __fadd_rn(a[2], a[6]);
  float s3 = __fadd_rn(a[3], a[7]);
  return __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide reductions for blockDim.x a multiple of 32 (<= 1024).
template <class T, class Op>
__device__ __forceinline__ T block_reduce(T v, Op op, T* smem32) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) smem32[warp] = v;
  __syncthreads();
  T r = smem32[0];
  for (int i = 1; i < nw; ++i) r = op(r, smem32[i]);
  return r;
}

// exp for the reference's softmax (ops.rs:206-227), which calls f32::exp ->
// the host libm's expf.  exp is evaluated in double and rounded to float,
// which is the correctly rounded result except when the double lands within
// 2^-20 ulp of a rounding boundary; the host libm itself is within 0.502 ulp
// of the exact value, so the two can only disagree when the exact value is
// within 0.002 ulp of a float midpoint.  Inputs whose double result lies that
// close (|position| > 0.497 ulp from the rounded value, ~0.15% of inputs) are
// looked up in a table of the host libm's results that differ from the
// double-rounded one (measured once per device, see ensure_exp_table); all
// other inputs already agree.  The table covers x in [-112, 0], the range of
// the softmax's x - max (below -112 both give 0).  It is held twice: sorted
// (keys/vals, binary search) and as an open-addressing hash of (key, value)
// pairs (linear probing, at most hash_probes slots per lookup, key 0 = empty
// since +0.0 is never an entry).
struct ExpTable {
  const uint32_t* keys = nullptr;  // float bit patterns, ascending
  const float* vals = nullptr;     // the host libm's expf of each key
  int n = 0;
  const uint2* hash = nullptr;     // (key, value bits) slots
  uint32_t hash_shift = 32;        // slot = (key * kExpHashMul) >> hash_shift
  uint32_t hash_mask = 0;          // slots - 1
  int hash_probes = 0;             // longest probe sequence in the table
};
constexpr uint32_t kExpHashMul = 0x9E3779B1u;

__device__ __forceinline__ double exp_round_position(double d, float f) {
  uint32_t fb = __float_as_uint(f);
  double nb = (double)__uint_as_float(d >= (double)f ? fb + 1 : fb - 1);
  double ulp = fabs(nb - (double)f);
  return fabs(d - (double)f) / ulp;
}

// exp in double for the softmax: Cody-Waite reduction x = k ln2 + r (ln2 in
// two parts, the first with 21 trailing zero bits so k * ln2_hi is exact),
// the Taylor polynomial of exp(r) to degree 11 for |r| <= ln2/2 (Horner,
// coefficients 1/n! rounded to double), then the exact scaling by 2^k.
// Relative error below 1e-14 on [-150, 100] (a CPU mirror checked it on
// every seventh float of [-112, 0] against long double expl): 1.5e-7 of a
// float ulp, far inside the 0.003-ulp margin of the table rule.  Below -150
// the result is 0 (exp(-150) < 2^-149); NaN stays NaN.
__device__ __forceinline__ double exp_f64(float xf) {
  const double x = (double)xf;
  if (!(x > -150.0)) return x != x ? x : 0.0;
  if (x > 100.0) return __longlong_as_double(0x7ff0000000000000LL);
  const double k = rint(x * 0x1.71547652b82fep+0);  // x / ln2
  double r = __fma_rn(-k, 0x1.62e42fee00000p-1, x);
  r = __fma_rn(-k, 0x1.a39ef35793c76p-33, r);
  double p = 0x1.ae64567f544e4p-26;  // 1/11!
  p = __fma_rn(p, r, 0x1.27e4fb7789f5cp-22);
  p = __fma_rn(p, r, 0x1.71de3a556c734p-19);
  p = __fma_rn(p, r, 0x1.a01a01a01a01ap-16);
  p = __fma_rn(p, r, 0x1.a01a01a01a01ap-13);
  p = __fma_rn(p, r, 0x1.6c16c16c16c17p-10);
  p = __fma_rn(p, r, 0x1.1111111111111p-7);
  p = __fma_rn(p, r, 0x1.5555555555555p-5);
  p = __fma_rn(p, r, 0x1.5555555555555p-3);
  p = __fma_rn(p, r, 0x1.0000000000000p-1);
  p = __fma_rn(p, r, 1.0);
  p = __fma_rn(p, r, 1.0);
  return __dmul_rn(p, __longlong_as_double((long long)((long long)k + 1023) << 52));
}

// True when the float rounding of d = exp_f64(x) (f its rounded value) lies
// more than 0.497 ulp from f, i.e. within 0.003 ulp of a midpoint.  For a
// result in the float normal range the position is read from the 29
// mantissa bits the rounding discards; smaller results use the division.
__device__ __forceinline__ bool exp_near_midpoint(double d, float f) {
  if (d >= 0x1p-126) {
    const int r = (int)((unsigned long long)__double_as_longlong(d) & 0x1FFFFFFFull) - (1 << 28);
    return (r < 0 ? -r : r) <= 1610612;  // |r - 2^28| <= 0.003 * 2^29
  }
  return exp_round_position(d, f) > 0.497;
}

// First half of exp_host_libm: the double-rounded value, and whether the
// input needs the table (returns true; the caller resolves it later).
__device__ __forceinline__ bool exp_needs_table(float x, const ExpTable& t, float* out) {
  const double d = exp_f64(x);
  const float f = (float)d;
  *out = f;
  if (t.n == 0 || !(f > 0.0f) || isinf(f)) return false;
  return exp_near_midpoint(d, f);
}

// Second half: the host libm's value for a table candidate `key` whose
// double-rounded value is f.
__device__ __forceinline__ float exp_table_lookup(uint32_t key, float f, const ExpTable& t) {
  if (t.hash) {
    uint32_t i = (key * kExpHashMul) >> t.hash_shift;
    for (int k = 0; k <= t.hash_probes; ++k) {
      const uint2 e = t.hash[(i + k) & t.hash_mask];
      if (e.x == key) return __uint_as_float(e.y);
      if (e.x == 0u) return f;
    }
    return f;
  }
  int lo = 0, hi = t.n - 1;
  while (lo <= hi) {
    int mid = (lo + hi) >> 1;
    uint32_t k = t.keys[mid];
    if (k == key) return t.vals[mid];
    if (k < key)
      lo = mid + 1;
    else
      hi = mid - 1;
  }
  return f;
}

__device__ __forceinline__ float exp_host_libm(float x, const ExpTable& t) {
  float f;
  if (!exp_needs_table(x, t, &f)) return f;
  return exp_table_lookup(__float_as_uint(x), f, t);
}

// Programmatic dependent launch (griddepcontrol, sm_90+).  A kernel launched
// with launch_pdl may begin while the previous kernel in the stream is still
// running; it must call pdl_wait() before it reads anything an earlier kernel
// writes or writes anything an earlier kernel reads (pdl_wait returns once
// the previous grid has completed and its memory is visible).  Only loads of
// data no kernel writes (weights) may precede it.  pdl_launch_dependents()
// allows the next kernel to start its own prologue.  Both are no-ops for a
// kernel launched without the attribute.  Measured on the 2B decode step,
// only the M = 1 GEMV gains from being launched this way (its weight stream
// starts under the previous kernel); the decode-chain kernels before it call
// pdl_launch_dependents so that it can. Launching the norm, RoPE and attention
// kernels this way as well was slower at batch 1 (517 vs 600 tokens/s) and at
// batch 256.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
// A pointer to data an earlier kernel writes, made opaque after pdl_wait():
// loads through it depend on an instruction that follows the wait, so the
// compiler cannot schedule them before it (it may move loads through
// const __restrict__ pointers across a plain memory clobber).
template <typename T>
__device__ __forceinline__ T* after_wait(T* p) {
  asm volatile("" : "+l"(p)::"memory");
  return p;
}
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

// Rust f32::round: half away from zero (roundf), then clamp, then cast.
__device__ __forceinline__ int8_t quant_i8(float x, float inv) {
  float s = roundf(__fmul_rn(x, inv));
  s = fminf(fmaxf(s, -128.0f), 127.0f);
  return (int8_t)(int)s;
}

}  // namespace bitnet
