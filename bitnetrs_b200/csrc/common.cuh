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

// Code dot products without shifts.  Masking a packed word in place leaves
// the codes of elements 4i..4i+3 in bits 2i..2i+1 of each byte, i.e. scaled
// by 4^i; dp4a with unsigned bytes (the scaled code is at most 2 << 6 = 128)
// and signed int8 activations accumulates 4^i * sum(c * x) exactly into
// acc[i].  codes_sum() undoes the scale: every term of acc[i] is a multiple of
// 4^i, so the arithmetic shift is exact (|acc[3]| < 2^31 for rows of up to
// 2^21 codes).  Two logic ops fewer per word than shift-and-mask.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// acc[i] += 4^i * sum_j code(element 4i + j of w) * byte j of x_i
__device__ __forceinline__ void dp4a_word_scaled(uint32_t w, const uint4& x, int (&acc)[4]) {
  acc[0] = dp4a_us(w & 0x03030303u, (int)x.x, acc[0]);
  acc[1] = dp4a_us(w & 0x0C0C0C0Cu, (int)x.y, acc[1]);
  acc[2] = dp4a_us(w & 0x30303030u, (int)x.z, acc[2]);
  acc[3] = dp4a_us(w & 0xC0C0C0C0u, (int)x.w, acc[3]);
}
__device__ __forceinline__ int codes_sum(const int (&acc)[4]) {
  return acc[0] + (acc[1] >> 2) + (acc[2] >> 4) + (acc[3] >> 6);
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
// the host libm's expf.  The device computes exp far more precisely than a
// float (exp_pair; exp_f64 outside [-87, 0]) and rounds; that agrees with
// the host libm except where the exact value lies very close to a float
// midpoint (the host libm's own disagreements with the correctly rounded
// value all lie within 0.00165 ulp of one, measured over every float of
// [-87, 0]).  Inputs whose value lies within 0.003 ulp of a midpoint
// (position > 0.497 ulp from the rounded value, ~0.15% of inputs) are table
// candidates; the table holds the host libm's value for each candidate of
// [-112, -0] where it differs from the device's rounded value (built once
// per device by ensure_exp_table from the device's own candidates), and
// every other input already agrees.  Below -112 both give 0.  The table is
// held sorted (keys/vals, binary search) and as a two-choice bucketed hash:
// buckets of 8 (key, value bits) slots, 64 bytes each, the key in the less
// full of buckets h1(key) and h2(key), so a lookup loads both buckets at
// once (one memory round trip); key 0 marks an empty slot (+0.0 is never a
// key).
struct ExpTable {
  const uint32_t* keys = nullptr;  // float bit patterns, ascending
  const float* vals = nullptr;     // the host libm's expf of each key
  int n = 0;
  const uint4* buckets = nullptr;  // [nbuckets][4] uint4 = 8 (key, value bits) slots each
  uint32_t bucket_shift = 32;      // bucket = (key * multiplier) >> bucket_shift
  // float-pair tables of exp_pair: en[k] = (hi, lo, S as int bits, 0) with
  // hi + lo = exp(-k) * 2^S (k < 88, S = round(k / ln2)); fj[j] = (hi, lo) =
  // exp(-j/128)
  const float4* en = nullptr;
  const float2* fj = nullptr;
};
constexpr uint32_t kExpHashMul = 0x9E3779B1u;   // h1
constexpr uint32_t kExpHashMul2 = 0x85EBCA77u;  // h2
constexpr int kExpBucketSlots = 8;

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

// exp for x in [-87, 0] in single-precision pairs (the softmax's x - max),
// to far better than float precision: the reduction x = n + j/128 + r (n =
// ceil(x), j = ceil(128 (x - n)), r in (-1/128, 0]) is exact; exp(r) = 1 +
// r + r^2 (1/2 + r (1/6 + r (1/24 + r/120))) with 1 + r kept as an exact
// pair; exp(n) (scaled by 2^S into [0.7, 1.4]) and exp(j/128) come from the
// pair tables; two pair products and a renormalisation give hi + lo, within
// 1e-4 float ulp of exp(x) * 2^S.  f = hi * 2^-S is the rounded value, and
// the input is a table candidate when lo lies more than 0.497 ulp from hi
// (toward lo: the grid below a power of two is twice as fine).  A CPU mirror
// of these exact operations was checked against the host libm's expf on
// every float of [-87, 0]: every non-candidate agrees bit for bit.
// Returns -1 outside [-87, 0] (the caller falls back to exp_f64), else
// whether x is a candidate, with f in *out.
__device__ __forceinline__ int exp_pair(float x, const ExpTable& t, float* out) {
  if (!(x >= -87.0f && x <= 0.0f) || t.en == nullptr) return -1;
  // ceil(v) for |v| < 2^22: v + 1.5 * 2^23 rounded up is an integer whose
  // value sits in the low mantissa bits (no conversion instruction needed)
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  const float nm = __fadd_ru(x, kMagic);
  const float n = __fsub_rn(nm, kMagic);  // ceil(x)
  const float fr = __fsub_rn(x, n);
  const float jm = __fadd_ru(__fmul_rn(fr, 128.0f), kMagic);
  const float jf = __fsub_rn(jm, kMagic);  // ceil(128 fr)
  const float r = __fsub_rn(fr, __fmul_rn(jf, 0.0078125f));
  float q = __fmaf_rn(r, 0x1.111112p-7f, 0x1.555556p-5f);  // 1/120, 1/24
  q = __fmaf_rn(q, r, 0x1.555556p-3f);                     // 1/6
  q = __fmaf_rn(q, r, 0.5f);
  q = __fmul_rn(q, __fmul_rn(r, r));
  const float a_hi = __fadd_rn(1.0f, r);
  const float a_lo = __fadd_rn(__fsub_rn(r, __fsub_rn(a_hi, 1.0f)), q);
  const int k = __float_as_int(kMagic) - __float_as_int(nm);  // -n
  const int j = __float_as_int(kMagic) - __float_as_int(jm);  // -ceil(128 fr)
  const float4 E = __ldg(t.en + k);
  const float2 F = __ldg(t.fj + j);
  const float p = __fmul_rn(E.x, F.x);
  float pe = __fmaf_rn(E.x, F.x, -p);
  pe = __fmaf_rn(E.x, F.y, pe);
  pe = __fmaf_rn(E.y, F.x, pe);
  const float y = __fmul_rn(p, a_hi);
  float ye = __fmaf_rn(p, a_hi, -y);
  ye = __fmaf_rn(p, a_lo, ye);
  ye = __fmaf_rn(pe, a_hi, ye);
  const float hi = __fadd_rn(y, ye);
  const float lo = __fsub_rn(ye, __fsub_rn(hi, y));
  const int S = __float_as_int(E.z);
  const uint32_t hb = __float_as_uint(hi);
  if ((int)((hb >> 23) & 0xffu) - S <= 0) return -1;  // not reached for x >= -87
  *out = __uint_as_float(hb - ((uint32_t)S << 23));
  float ulp = __uint_as_float((hb & 0x7f800000u) - (23u << 23));
  if (lo < 0.0f && (hb & 0x7fffffu) == 0u) ulp = __fmul_rn(ulp, 0.5f);
  return fabsf(lo) > __fmul_rn(0.497f, ulp) ? 1 : 0;
}

// The value exp_host_libm starts from (*out) and whether it lies within
// 0.003 ulp of a rounding midpoint (a table candidate): exp_pair, or exp_f64
// outside its range.
__device__ __forceinline__ bool exp_candidate(float x, const ExpTable& t, float* out) {
  const int c = exp_pair(x, t, out);
  if (c >= 0) return c != 0;
  const double d = exp_f64(x);
  const float f = (float)d;
  *out = f;
  if (!(f > 0.0f) || isinf(f)) return false;
  return exp_near_midpoint(d, f);
}

// First half of exp_host_libm: the starting value, and whether the input
// needs the table (returns true; the caller resolves it later).
__device__ __forceinline__ bool exp_needs_table(float x, const ExpTable& t, float* out) {
  const bool c = exp_candidate(x, t, out);
  return t.n != 0 && c;
}

// Second half: the host libm's value for a table candidate `key` whose
// device-rounded value is f.
__device__ __forceinline__ float exp_table_lookup(uint32_t key, float f, const ExpTable& t) {
  if (t.buckets) {
    const uint4* b1 = t.buckets + 4 * (size_t)((key * kExpHashMul) >> t.bucket_shift);
    const uint4* b2 = t.buckets + 4 * (size_t)((key * kExpHashMul2) >> t.bucket_shift);
    uint4 v[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[i] = __ldg(b1 + i);
      v[4 + i] = __ldg(b2 + i);
    }
    float r = f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (v[i].x == key) r = __uint_as_float(v[i].y);
      if (v[i].z == key) r = __uint_as_float(v[i].w);
    }
    return r;
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
