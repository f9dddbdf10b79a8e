// kernels_decode1.cu — the layer stack of a one-token decode step as one
// persistent kernel (bf16 paged KV cache, head_dim 128).
//
// At batch 1 every per-layer kernel of the step is a few microseconds of
// latency on a GPU that is mostly idle, and the launch boundaries (about ten
// per layer) dominate the token time.  This kernel runs all layers of
// BitNetModel::forward (bitnet-model/src/lib.rs:559-860) for the single new
// token with the same operations in the same order as the per-layer kernels
// (and so as the reference), one CTA per SM, cooperative launch:
//
// * CTAs [0, nh / HPC) are attention CTAs, each serving HPC query heads of
//   one kv head (attention.rs:165-206, ops.rs:172-227); HPC is the smallest
//   divisor of the GQA group that keeps them to kD1MaxAttn CTAs, one query
//   head per CTA for the 2B model.  The K and V pages of the kv head (4 KiB
//   TMA tiles, 128-byte swizzle) stream through a ring of shared-memory
//   slots that runs ahead into the next layer, so a short context is
//   resident before the layer's q arrives.
// * The other CTAs are matmul CTAs.  Each owns a fixed slice of the rows of the
//   four projections (qkv, o, gate/up, down) and keeps one shared-memory slot
//   per projection; the slot of a projection is refilled with the next layer's
//   rows (one bulk copy) as soon as this layer's product has read it, so the
//   weight stream runs a whole layer ahead of the arithmetic.  Every matmul CTA
//   computes each RMSNorm + absmax quantisation (absmax.rs:127-165) of the
//   full row itself, so no grid barrier separates a norm from its matmul.
//
// Per layer the grid meets at five counters in global memory: qkv written
// (attention CTAs wait), attention written, o-projection added to h, gate/up
// written, down-projection added to h (matmul CTAs wait).  A counter is a
// release-add by each producer CTA and an acquire spin by the consumers;
// every spin and every mbarrier wait is bounded (kAsyncWaitCycles).  A CTA
// whose wait runs out raises the launch's abort word and records
// kStatusWaitTimeout; every CTA then lets its own copies land (bounded) and
// returns.  Data other CTAs wrote in this launch is read with ld.global.cg.
#include "async.cuh"

namespace bitnet {

namespace {

constexpr int kD1Threads = 512;
constexpr int kD1Warps = kD1Threads / 32;
constexpr int kD1Page = 4096;        // one page of one kv head: [16 rows][2 halves][64] bf16, 128-byte swizzle
constexpr int kD1MaxRing = 64;       // ring slots (mbarriers) of an attention CTA
constexpr int kD1MinRing = 8;        // fewest ring slots a plan may leave
constexpr int kD1MaxAttn = 32;       // most attention CTAs
constexpr int kD1SyncStride = 32;    // 32-bit words between counters (one 128-byte line each)
enum { kCtrQkv = 0, kCtrAttn = 1, kCtrO = 2, kCtrGu = 3, kCtrDown = 4, kCtrAbort = 5 };

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

// Slot and phase parity of one item of an attention CTA's ring of S slots
// (item A sits in slot A % S and completes phase (A / S) & 1 of its
// barrier), advanced without integer division.
struct RingPos {
  int slot;
  uint32_t par;
};
__device__ __forceinline__ RingPos ring_add(RingPos p, int k, int S) {  // 0 <= k <= S
  p.slot += k;
  if (p.slot >= S) {
    p.slot -= S;
    p.par ^= 1u;
  }
  return p;
}
__device__ __forceinline__ RingPos ring_advance(RingPos p, int k, int S) {  // any k >= 0
  while (k > S) {
    p = ring_add(p, S, S);
    k -= S;
  }
  return ring_add(p, k, S);
}
__device__ __forceinline__ uint16_t lds16(uint32_t a) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];\n" : "=h"(v) : "r"(a));
  return v;
}

// Raises the launch's abort word (once) and records the timeout for the host.
__device__ __forceinline__ void grid_abort(uint32_t* sync, int32_t* status) {
  if (atomicExch(sync + kCtrAbort * kD1SyncStride, 1u) == 0u) atomicOr(status, kStatusWaitTimeout);
}

// This CTA's writes so far are published: one release-add to counter `which`.
__device__ __forceinline__ void grid_arrive(uint32_t* sync, int which) {
  __syncthreads();
  if (threadIdx.x == 0) red_release_add(sync + which * kD1SyncStride, 1u);
}

// Waits until counter `which` reaches `target`; false (in every thread) when
// the launch is aborting or the wait ran out.
__device__ __forceinline__ bool grid_wait(uint32_t* sync, int which, uint32_t target, int32_t* status) {
  int ok = 1;
  if (threadIdx.x == 0) {
    const uint32_t* ctr = sync + which * kD1SyncStride;
    if (ld_acquire_u32(ctr) < target) {
      const volatile uint32_t* ab = sync + kCtrAbort * kD1SyncStride;
      const long long t0 = clock64();
      for (;;) {
        if (ld_acquire_u32(ctr) >= target) break;
        if (*ab) {
          ok = 0;
          break;
        }
        if (clock64() - t0 > kAsyncWaitCycles) {
          grid_abort(sync, status);
          ok = 0;
          break;
        }
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

// Waits (every thread) for phase `parity` of a shared-memory copy barrier.
__device__ __forceinline__ bool copy_wait(uint32_t bar, uint32_t parity, uint32_t* sync, int32_t* status) {
  const int ok = __syncthreads_and(mbar_wait(bar, parity, nullptr) ? 1 : 0);
  if (!ok && threadIdx.x == 0) grid_abort(sync, status);
  return ok != 0;
}

// ---------------------------------------------------------------------------
// RMSNorm + absmax quantisation of one row (absmax.rs:127-165) with the
// operations of norm_quant_reg_kernel.  Thread t holds float4 groups
// t + 512 u of the row (v) and of the gains (wv, loaded ahead of time: no
// kernel writes them); the row is also in shared memory, from where lanes
// 0..7 of warp 0 run the eight FMA chains of the sum of squares (then
// hsum_f32_avx2), their loads issued 16 elements ahead.  Then y = (x * inv)
// * w in registers, its absmax and the int8 row, zero-padded to kpad and
// stored chunk-transposed: 16-byte word q (elements 16 q .. 16 q + 15) of
// 64-element chunk c sits at word q * (kpad / 64) + c, so that lanes reading
// chunks l + 32 j of x touch consecutive words.  The code sum of the row is
// taken by the matmul warps themselves (d1_gemv).
// ---------------------------------------------------------------------------
constexpr int kD1U = 4;  // float4 per thread: rows of up to 4 * 4 * 512 = 8192 floats

__device__ __forceinline__ void norm_gains(float4 (&wv)[kD1U], const float* w, int d) {
  const float4* w4 = reinterpret_cast<const float4*>(w);
#pragma unroll
  for (int u = 0; u < kD1U; ++u) {
    const int j = (int)threadIdx.x + kD1Threads * u;
    wv[u] = j < (d >> 2) ? __ldg(w4 + j) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
}

// A row other CTAs wrote in this launch, into registers and the shared row
// (every load is issued before the first store, so they overlap).
__device__ __forceinline__ void load_row(float4 (&v)[kD1U], float* row, const float* src, int d) {
  const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
  for (int u = 0; u < kD1U; ++u) {
    const int j = (int)threadIdx.x + kD1Threads * u;
    if (j < (d >> 2)) v[u] = __ldcg(s4 + j);
  }
#pragma unroll
  for (int u = 0; u < kD1U; ++u) {
    const int j = (int)threadIdx.x + kD1Threads * u;
    if (j < (d >> 2)) reinterpret_cast<float4*>(row)[j] = v[u];
  }
}

// sqrelu(gate) * up (f32::max(0), then r * r * u) into registers and the shared row.
__device__ __forceinline__ void load_gate_up(float4 (&v)[kD1U], float* row, const float* gu, int F) {
  const float4* g4 = reinterpret_cast<const float4*>(gu);
  const float4* u4 = reinterpret_cast<const float4*>(gu + F);
  float4 b4[kD1U];
#pragma unroll
  for (int u = 0; u < kD1U; ++u) {
    const int j = (int)threadIdx.x + kD1Threads * u;
    if (j < (F >> 2)) {
      v[u] = __ldcg(g4 + j);
      b4[u] = __ldcg(u4 + j);
    }
  }
#pragma unroll
  for (int u = 0; u < kD1U; ++u) {
    const int j = (int)threadIdx.x + kD1Threads * u;
    if (j < (F >> 2)) {
      const float4 a = v[u], b = b4[u];
      const float r0 = fmaxf(a.x, 0.0f), r1 = fmaxf(a.y, 0.0f), r2 = fmaxf(a.z, 0.0f), r3 = fmaxf(a.w, 0.0f);
      v[u] = make_float4(__fmul_rn(__fmul_rn(r0, r0), b.x), __fmul_rn(__fmul_rn(r1, r1), b.y),
                         __fmul_rn(__fmul_rn(r2, r2), b.z), __fmul_rn(__fmul_rn(r3, r3), b.w));
      reinterpret_cast<float4*>(row)[j] = v[u];
    }
  }
}

__device__ __forceinline__ float lds32f(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];\n" : "=f"(v) : "r"(a));
  return v;
}

// Returns act_absmax; the int8 row is complete when it returns.
__device__ float d1_norm_quant(float4 (&v)[kD1U], const float4 (&wv)[kD1U], const float* row, int d, float eps,
                               int8_t* xq, int kpad, float* s_bc, float* red_f, int* red_b, int32_t* status) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5, n4 = d >> 2;
  __syncthreads();  // the shared row is complete
  if (warp == 0) {
    const int chunks = d >> 3;
    float acc = 0.0f;
    if (lane < 8) {
      // element 8 i + lane of the row at byte 32 i + 4 lane
      const uint32_t rs = smem_u32(row) + 4u * (uint32_t)lane;
      // two 16-element register blocks in turn: one block's loads are in
      // flight while the other's FMAs run, with no register copies in the loop
      const int full = chunks & ~31;
      float ba[16], bb[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) ba[k] = full ? lds32f(rs + 32u * (uint32_t)k) : 0.0f;
      int i = 0;
      for (; i < full; i += 32) {
#pragma unroll
        for (int k = 0; k < 16; ++k) bb[k] = lds32f(rs + 32u * (uint32_t)(i + 16 + k));
#pragma unroll
        for (int k = 0; k < 16; ++k) acc = __fmaf_rn(ba[k], ba[k], acc);
        const int ni = i + 32 < full ? i + 32 : i;
#pragma unroll
        for (int k = 0; k < 16; ++k) ba[k] = lds32f(rs + 32u * (uint32_t)(ni + k));
#pragma unroll
        for (int k = 0; k < 16; ++k) acc = __fmaf_rn(bb[k], bb[k], acc);
      }
      for (; i < chunks; ++i) {
        const float a = lds32f(rs + 32u * (uint32_t)i);
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
      *s_bc = __fdiv_rn(1.0f, rms);
    }
  }
  __syncthreads();
  const float inv = *s_bc;
  float mx = 0.0f;
  int bad = 0;
#pragma unroll
  for (int u = 0; u < kD1U; ++u) {
    if (t + kD1Threads * u < n4) {
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
  mx = 0.0f;
  bad = 0;
#pragma unroll
  for (int k = 0; k < kD1Warps; ++k) {
    mx = fmaxf(mx, red_f[k]);
    bad |= red_b[k];
  }
  const float mc = fmaxf(mx, 1e-5f);
  const float scale = __fdiv_rn(mc, 127.0f), qinv = __fdiv_rn(127.0f, mc);
  const int nc = kpad >> 6;  // 64-element chunks
#pragma unroll
  for (int u = 0; u < kD1U; ++u) {
    const int j = t + kD1Threads * u;  // elements 4 j .. 4 j + 3
    if (j < n4) {
      const int8_t c0 = quant_i8(v[u].x, qinv), c1 = quant_i8(v[u].y, qinv), c2 = quant_i8(v[u].z, qinv),
                   c3 = quant_i8(v[u].w, qinv);
      *reinterpret_cast<char4*>(xq + ((((j >> 2) & 3) * nc + (j >> 4)) << 4) + ((j & 3) << 2)) =
          make_char4(c0, c1, c2, c3);
    }
  }
  for (int e = d + t; e < kpad; e += kD1Threads) xq[((((e >> 4) & 3) * nc + (e >> 6)) << 4) + (e & 15)] = 0;
  if (bad && t == 0) atomicOr(status, kStatusNonFinite);
  __syncthreads();
  return __fmul_rn(scale, 127.0f);
}

// 1 / rms of a row in shared memory (rms_inv_exact: the eight FMA chains by
// lanes 0..7 of warp 0, hsum_f32_avx2, the tail, sqrt(ss / d + eps)), for the
// final norm.  The caller has synchronised after filling the row.
__device__ __noinline__ float d1_rms_inv(const float* row, int d, float eps, float* s_bc) {
  const int lane = threadIdx.x & 31;
  if (threadIdx.x < 32) {
    const int chunks = d >> 3;
    float acc = 0.0f;
    if (lane < 8)
      for (int i = 0; i < chunks; ++i) {
        const float a = row[8 * i + lane];
        acc = __fmaf_rn(a, a, acc);
      }
    float a[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] = __shfl_sync(0xffffffffu, acc, j);
    if (lane == 0) {
      float ss = hsum8(a);
      for (int i = chunks * 8; i < d; ++i) ss = __fadd_rn(ss, __fmul_rn(row[i], row[i]));
      const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)d), eps));
      *s_bc = __fdiv_rn(1.0f, rms);
    }
  }
  __syncthreads();
  return *s_bc;
}

// ---------------------------------------------------------------------------
// The CTA's rows of one projection, from its shared-memory slot: the exact
// int32 sum of the rowsum identity of gemv_m1_kernel, then the reference's
// dequantisation acc as f32 * (ws * act_absmax / 127) with the combined
// scale of each output segment formed once.  A warp takes rows r and r + 16
// together; lane l multiplies 16-byte chunks l + 32 j of both with the
// matching 64 bytes of x, which it keeps in registers, into two partial sums
// per row (integer sums: any order is exact).  With `hown` (the CTA's rows of
// the residual stream h, kept in shared memory) the result is added to h.
// ---------------------------------------------------------------------------
struct D1Epi {
  float comb[3];
  int end0, end1;
};

__device__ __forceinline__ D1Epi d1_epi(float s0, float s1, float s2, int end0, int end1, float amax) {
  D1Epi e;
  e.comb[0] = __fdiv_rn(__fmul_rn(s0, amax), 127.0f);
  e.comb[1] = __fdiv_rn(__fmul_rn(s1, amax), 127.0f);
  e.comb[2] = __fdiv_rn(__fmul_rn(s2, amax), 127.0f);
  e.end0 = end0;
  e.end1 = end1;
  return e;
}

__device__ __forceinline__ void d1_put(int r, int s, int xsum, const D1Epi& ep, int n0, float* out, float* hown) {
  const int n = n0 + r;
  const float comb = n < ep.end0 ? ep.comb[0] : (n < ep.end1 ? ep.comb[1] : ep.comb[2]);
  const float v = __fmul_rn((float)(xsum - s), comb);
  if (hown) {
    const float hv = __fadd_rn(hown[r], v);  // axpy_f32_fast(1.0, o, h) == h + o
    hown[r] = hv;
    out[n] = hv;
  } else {
    out[n] = v;
  }
}

template <int CH>
__device__ __forceinline__ void d1_gemv(uint32_t ws, int nrows, int kw4, const uint4* xs, const D1Epi ep, int n0,
                                        float* out, float* hown) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint4 xr[CH][4];
  int xsum = 0;  // the code sum of the int8 row, taken by every warp
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const int c = lane + 32 * j;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      xr[j][q] = c < kw4 ? xs[q * kw4 + c] : make_uint4(0, 0, 0, 0);
      xsum = __dp4a((int)xr[j][q].x, 0x01010101, xsum);
      xsum = __dp4a((int)xr[j][q].y, 0x01010101, xsum);
      xsum = __dp4a((int)xr[j][q].z, 0x01010101, xsum);
      xsum = __dp4a((int)xr[j][q].w, 0x01010101, xsum);
    }
  }
  xsum = warp_sum_i(xsum);
  for (int r = warp; r < nrows; r += 2 * kD1Warps) {
    const int r2 = r + kD1Warps;
    const bool two = r2 < nrows;
    int a[4] = {0, 0, 0, 0}, b[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < CH; ++j) {
      const int c = lane + 32 * j;
      if (c < kw4) {
        const uint4 w = lds128(ws + (uint32_t)(r * kw4 + c) * 16u);
        const uint4 w2 = two ? lds128(ws + (uint32_t)(r2 * kw4 + c) * 16u) : make_uint4(0, 0, 0, 0);
        dp4a_word_scaled(w.x, xr[j][0], a);
        dp4a_word_scaled(w2.x, xr[j][0], b);
        dp4a_word_scaled(w.y, xr[j][1], a);
        dp4a_word_scaled(w2.y, xr[j][1], b);
        dp4a_word_scaled(w.z, xr[j][2], a);
        dp4a_word_scaled(w2.z, xr[j][2], b);
        dp4a_word_scaled(w.w, xr[j][3], a);
        dp4a_word_scaled(w2.w, xr[j][3], b);
      }
    }
    const int s = warp_sum_i(codes_sum(a)), s2 = warp_sum_i(codes_sum(b));
    if (lane == 0) {
      d1_put(r, s, xsum, ep, n0, out, hown);
      if (two) d1_put(r2, s2, xsum, ep, n0, out, hown);
    }
  }
}

__device__ __forceinline__ void d1_gemv_any(uint32_t ws, int nrows, int kw4, const uint4* xs, const D1Epi ep,
                                            int n0, float* out, float* hown) {
  if (kw4 <= 32)
    d1_gemv<1>(ws, nrows, kw4, xs, ep, n0, out, hown);
  else if (kw4 <= 64)
    d1_gemv<2>(ws, nrows, kw4, xs, ep, n0, out, hown);
  else
    d1_gemv<4>(ws, nrows, kw4, xs, ep, n0, out, hown);
}

// The 16 V values of one page at the lane's dimension (row offsets voff).
__device__ __forceinline__ void d1_load_v(float (&vv)[kPage], uint32_t vb, const uint32_t (&voff)[4]) {
#pragma unroll
  for (int rr = 0; rr < kPage; ++rr) vv[rr] = bf16_bits_to_f32(lds16(vb + (uint32_t)rr * 256u + voff[rr & 3]));
}

// Rotates (lo, hi) = (x[p], x[p + 64]) of one head (rope.rs:414-431, half split).
__device__ __forceinline__ float2 rope_pair(float lo, float hi, float c, float s) {
  return make_float2(__fsub_rn(__fmul_rn(lo, c), __fmul_rn(hi, s)), __fadd_rn(__fmul_rn(hi, c), __fmul_rn(lo, s)));
}

}  // namespace

// ---------------------------------------------------------------------------
// The kernel.  HPC = query heads per attention CTA (1, 2, 4 or 8; a divisor
// of the GQA group).
// ---------------------------------------------------------------------------
template <int HPC>
__global__ void __launch_bounds__(kD1Threads, 1)
    decode1_kernel(const __grid_constant__ D1Params P, const __grid_constant__ CUtensorMap tmap) {
  extern __shared__ uint8_t d1_smem_raw[];
  __shared__ __align__(8) uint64_t bar[kD1MaxRing];  // matmul CTAs: [0, 4) weight slots; attention CTAs: ring
  __shared__ __align__(16) float qs[HPC * 128];      // the CTA's rotated query rows
  __shared__ __align__(16) uint16_t kn[128], vn[128];  // the new position's k (rotated) and v, bf16 bits
  __shared__ float red_f[kD1Warps * HPC];
  __shared__ int red_b[kD1Warps];
  __shared__ float s_bc, s_m[HPC], s_inv[HPC];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t raw = smem_u32(d1_smem_raw);
  uint8_t* sm = d1_smem_raw + ((1024u - (raw & 1023u)) & 1023u);  // 1024-aligned (TMA swizzle)
  const uint32_t sm_s = smem_u32(sm);
  uint32_t* sync = P.sync;
  int32_t* status = P.status;
  const int L = P.L, H = P.H, F = P.F;
  const int qd = P.nh * 128, kvd = P.nkv * 128, nqkv = qd + 2 * kvd;
  const uint64_t pol = evict_first_policy();
  const int n_attn = P.nh / HPC, G = (int)gridDim.x - n_attn;
  const int pos = __ldg(P.tok_pos), seq = __ldg(P.tok_seq);
  const int32_t* pt = P.page_table + (size_t)seq * P.g.max_pages_per_seq;

  if ((int)blockIdx.x < n_attn) {
    // ============ attention CTA: query heads [head0, head0 + HPC) of kv head kvh ============
    const int as = (P.nh / P.nkv) / HPC;  // attention CTAs per kv head
    const int kvh = (int)blockIdx.x / as, head0 = (int)blockIdx.x * HPC;
    const bool leader = (int)blockIdx.x % as == 0;  // stores the new k and v
    const int S = P.ring_slots;
    const int ctx = pos + 1, np = (ctx + kPage - 1) / kPage;
    const int RP = min(2 * kD1Warps, S & ~1);  // pages per round
    const int total = L * 2 * np;              // ring items of the launch: per layer K pages then V pages
    float* sc = reinterpret_cast<float*>(sm + P.sc_off);  // [ctx][HPC] scores, then e, then p
    if (tid == 0) {
      for (int s = 0; s < S; ++s) mbar_init(smem_u32(&bar[s]), 1);
      asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncthreads();
    if (ctx > P.cap || S < kD1MinRing) {  // the host plans for the context; uniform over the CTA
      if (tid == 0) {
        atomicOr(status, kStatusBadContext);
        atomicExch(sync + kCtrAbort * kD1SyncStride, 1u);
      }
      return;
    }
    int issued = 0;  // thread 0: items issued so far
    auto issue_upto = [&](int limit) {
      if (tid != 0) return;
      limit = min(limit, total);
      if (issued < limit) fence_proxy_async();
      for (; issued < limit; ++issued) {
        const int l = issued / (2 * np), i = issued % (2 * np);
        const int kind = i < np ? 0 : 1, page = i < np ? i : i - np;
        const int s = issued % S;
        const uint32_t b = smem_u32(&bar[s]);
        mbar_expect_tx(b, kD1Page);
        tma_page(sm_s + (uint32_t)s * kD1Page, &tmap, (kvh * 2 + kind) * kPage, l * P.g.pages + __ldg(pt + page), b,
                 pol);
      }
    };
    auto item_wait = [&](int A) { return mbar_wait(smem_u32(&bar[A % S]), (uint32_t)(A / S) & 1u, nullptr); };
    auto ring_wait = [&](RingPos a) { return mbar_wait(smem_u32(&bar[a.slot]), a.par, nullptr); };
    RingPos lpos = {0, 0u};  // ring position of the first item of layer l
    int consumed = 0;  // items every thread has finished reading
    issue_upto(S);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(128.0f));
    const uint32_t qs_s = smem_u32(qs);
    // PV: lane (warp < 4) owns dimension 32 warp + lane; byte offset of its
    // value in row rr of a V tile is rr * 256 + voff[rr & 3] (128-byte swizzle)
    uint32_t voff[4];
    {
      const int dd = 32 * warp + lane, half = (dd >> 6) & 1;
      const uint32_t cw = (uint32_t)((dd & 63) >> 3), bo = (uint32_t)(dd & 7) * 2;
#pragma unroll
      for (int k = 0; k < 4; ++k) voff[k] = (uint32_t)half * 128u + ((cw ^ (uint32_t)(2 * k + half)) << 4) + bo;
    }
    bool alive = true;
    for (int l = 0; l < L && alive; ++l) {
      const int base = l * 2 * np;
      if (!grid_wait(sync, kCtrQkv, (uint32_t)((l + 1) * G), status)) {
        alive = false;
        break;
      }
      // the CTA's query rows and the kv head's k, rotated at this position, and v
      {
        const float* qkv = P.qkv;
        const float* rc = P.rope_cos + (size_t)pos * 64;
        const float* rs = P.rope_sin + (size_t)pos * 64;
        for (int i = tid; i < HPC * 64 + 64 + 128; i += kD1Threads) {
          if (i < HPC * 64) {
            const int hh = i >> 6, p = i & 63;
            const float* x = qkv + (size_t)(head0 + hh) * 128;
            const float2 r = rope_pair(__ldcg(x + p), __ldcg(x + p + 64), __ldg(rc + p), __ldg(rs + p));
            qs[hh * 128 + p] = r.x;
            qs[hh * 128 + p + 64] = r.y;
          } else if (i < HPC * 64 + 64) {
            const int p = i - HPC * 64;
            const float* x = qkv + qd + (size_t)kvh * 128;
            const float2 r = rope_pair(__ldcg(x + p), __ldcg(x + p + 64), __ldg(rc + p), __ldg(rs + p));
            kn[p] = f32_to_bf16_bits(r.x);
            kn[p + 64] = f32_to_bf16_bits(r.y);
          } else {
            const int d = i - HPC * 64 - 64;
            vn[d] = f32_to_bf16_bits(__ldcg(qkv + qd + kvd + (size_t)kvh * 128 + d));
          }
        }
      }
      __syncthreads();
      if (leader && tid < 256) {  // KVCache::store_kv of this layer, kv head and position
        const int kind = tid >> 7, d = tid & 127;
        const size_t off = ((((size_t)l * P.g.pages + __ldg(pt + pos / kPage)) * P.g.kv_heads + kvh) * 2 + kind) *
                               (size_t)(kPage * 128) +
                           (size_t)(pos % kPage) * 128 + d;
        reinterpret_cast<uint16_t*>(P.g.pool)[off] = kind ? vn[d] : kn[d];
      }
      // ---- scores of positions < pos: lane = one row of page p0 + 2 warp + (lane >> 4) ----
      float mx[HPC];
#pragma unroll
      for (int h = 0; h < HPC; ++h) mx[h] = -INFINITY;
      {
        const int r = lane & 15, hp = lane >> 4;
        const uint32_t xo0 = (uint32_t)((2 * r) & 7) << 4, xo1 = (uint32_t)((2 * r + 1) & 7) << 4;
        RingPos rp = lpos;  // item base + p0
        for (int p0 = 0; p0 < np; p0 += RP) {
          const int pend = min(np, p0 + RP), pw = p0 + 2 * warp;
          int ok = 1;
          if (pw < pend) {
            const RingPos ia = ring_add(rp, 2 * warp, S), ib = ring_add(ia, 1, S);
            ok = ring_wait(ia) && (pw + 1 >= pend || ring_wait(ib));
            const int pa = pw + hp;
            if (ok && pa < pend) {
              const uint32_t ba = sm_s + (uint32_t)(hp ? ib.slot : ia.slot) * kD1Page + (uint32_t)(2 * r) * 128;
              const uint32_t c0 = ba | xo0, c1 = (ba + 128) | xo1;
              float acc[HPC][8];
#pragma unroll
              for (int h = 0; h < HPC; ++h)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[h][j] = 0.0f;
#pragma unroll
              for (int c = 0; c < 16; ++c) {
                const uint4 k4 = lds128((c < 8 ? c0 : c1) ^ ((uint32_t)(c & 7) << 4));
                const float kf[8] = {bf_lo(k4.x), bf_hi(k4.x), bf_lo(k4.y), bf_hi(k4.y),
                                     bf_lo(k4.z), bf_hi(k4.z), bf_lo(k4.w), bf_hi(k4.w)};
#pragma unroll
                for (int h = 0; h < HPC; ++h) {
                  const float4 q0 = lds128f(qs_s + (uint32_t)(h * 128 + 8 * c) * 4);
                  const float4 q1 = lds128f(qs_s + (uint32_t)(h * 128 + 8 * c + 4) * 4);
                  const float qq[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                  for (int j = 0; j < 8; ++j) acc[h][j] = __fmaf_rn(qq[j], kf[j], acc[h][j]);
                }
              }
              const int position = pa * kPage + r;
              if (position < pos) {
#pragma unroll
                for (int h = 0; h < HPC; ++h) {
                  const float sv = __fmul_rn(hsum8(acc[h]), scale);
                  sc[position * HPC + h] = sv;
                  mx[h] = fmaxf(mx[h], sv);
                }
              }
            }
          }
          if (!__syncthreads_and(ok)) {
            if (tid == 0) grid_abort(sync, status);
            alive = false;
            break;
          }
          consumed = base + pend;
          issue_upto(min(consumed + S, base + 2 * np));  // this layer's pages first
          rp = ring_add(rp, pend - p0, S);
        }
      }
      if (!alive) break;
      // ---- the new position's scores, from kn ----
      // (lane j of each group of eight runs FMA chain j of one head; the
      // group's first lane combines the chains in hsum_f32_avx2 order)
      if (warp * 32 < 8 * HPC) {
        const int j = lane & 7, h = min(tid >> 3, HPC - 1);
        float acc = 0.0f;
#pragma unroll
        for (int c = 0; c < 16; ++c) acc = __fmaf_rn(qs[h * 128 + 8 * c + j], bf16_bits_to_f32(kn[8 * c + j]), acc);
        float a[8];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) a[jj] = __shfl_sync(0xffffffffu, acc, (lane & ~7) + jj);
        if (j == 0 && tid < 8 * HPC) {
          const float sv = __fmul_rn(hsum8(a), scale);
          sc[pos * HPC + h] = sv;
#pragma unroll
          for (int hh = 0; hh < HPC; ++hh)
            if (hh == h) mx[hh] = fmaxf(mx[hh], sv);
        }
      }
#pragma unroll
      for (int h = 0; h < HPC; ++h) {
        const float mv = warp_max(mx[h]);
        if (lane == 0) red_f[warp * HPC + h] = mv;
      }
      __syncthreads();
      if (tid < HPC) {
        float m = red_f[tid];
        for (int w = 1; w < kD1Warps; ++w) m = fmaxf(m, red_f[w * HPC + tid]);
        s_m[tid] = m;
      }
      __syncthreads();
      // ---- softmax_f32 (ops.rs:206-227): e = exp(x - max), serial sum, p = e * (1 / sum) ----
      for (int i = tid; i < ctx * HPC; i += kD1Threads)
        sc[i] = exp_host_libm(__fsub_rn(sc[i], s_m[i & (HPC - 1)]), P.et);
      __syncthreads();
      if (tid < HPC) {
        const float* e = sc + tid;
        const int full = ctx & ~15;
        float sum = 0.0f;
        int i = 0;
        for (; i < full; i += 16) {
          float a[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) a[k] = e[HPC * (i + k)];
#pragma unroll
          for (int k = 0; k < 16; ++k) sum = __fadd_rn(sum, a[k]);
        }
        if (i < ctx) {
          float a[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) a[k] = i + k < ctx ? e[HPC * (i + k)] : 0.0f;
#pragma unroll
          for (int k = 0; k < 16; ++k)
            if (i + k < ctx) sum = __fadd_rn(sum, a[k]);
        }
        s_inv[tid] = __fdiv_rn(1.0f, sum);
      }
      __syncthreads();
      for (int i = tid; i < ctx * HPC; i += kD1Threads) sc[i] = __fmul_rn(sc[i], s_inv[i & (HPC - 1)]);
      __syncthreads();
      // ---- out[h][d] = fma(p_t, V[t][d], out[h][d]) over t (axpy_f32): warps 0..3, lane = dim ----
      //      (the next page's V values are loaded while this page's FMAs run)
      float o[HPC];
#pragma unroll
      for (int h = 0; h < HPC; ++h) o[h] = 0.0f;
      const int d = 32 * warp + lane;
      RingPos vp = ring_advance(lpos, np, S);  // item base + np + P0
      for (int P0 = 0; P0 < np; P0 += RP) {
        const int pend = min(np, P0 + RP);
        int ok = 1;
        if (warp < 4) {
          RingPos cur = vp;
          float vv[kPage];
          ok = ring_wait(cur);
          if (ok) d1_load_v(vv, sm_s + (uint32_t)cur.slot * kD1Page, voff);
          for (int pg = P0; pg < pend && ok; ++pg) {
            const int rows = min(kPage, pos - pg * kPage);  // positions < pos of this page
            // the page's p rows [16][HPC] into registers first (HPC <= 2: 4 HPC
            // 16-byte loads; rows past pos read scores of this page, unused)
            constexpr int kPr = HPC <= 2 ? kPage * HPC : 1;
            float pr[kPr];
            const float* pp = sc + pg * kPage * HPC;
            if constexpr (HPC <= 2) {
              const uint32_t pa = smem_u32(pp);
#pragma unroll
              for (int q = 0; q < kPr / 4; ++q) {
                const float4 t4 = lds128f(pa + 16u * (uint32_t)q);
                pr[4 * q] = t4.x;
                pr[4 * q + 1] = t4.y;
                pr[4 * q + 2] = t4.z;
                pr[4 * q + 3] = t4.w;
              }
            }
            const RingPos nx = ring_add(cur, 1, S);
            float vnx[kPage];
            if (pg + 1 < pend) {
              ok = ring_wait(nx);
              if (ok) d1_load_v(vnx, sm_s + (uint32_t)nx.slot * kD1Page, voff);
            }
#pragma unroll
            for (int rr = 0; rr < kPage; ++rr)
              if (rr < rows)
#pragma unroll
                for (int h = 0; h < HPC; ++h) {
                  const float pv = HPC <= 2 ? pr[(rr * HPC + h) % kPr] : pp[rr * HPC + h];
                  o[h] = __fmaf_rn(pv, vv[rr], o[h]);
                }
#pragma unroll
            for (int rr = 0; rr < kPage; ++rr) vv[rr] = vnx[rr];
            cur = nx;
          }
        }
        if (!__syncthreads_and(ok)) {
          if (tid == 0) grid_abort(sync, status);
          alive = false;
          break;
        }
        consumed = base + np + pend;
        issue_upto(min(consumed + S, base + 2 * np));
        vp = ring_add(vp, pend - P0, S);
      }
      if (!alive) break;
      if (warp < 4) {
        const float vf = bf16_bits_to_f32(vn[d]);
#pragma unroll
        for (int h = 0; h < HPC; ++h) {
          o[h] = __fmaf_rn(sc[pos * HPC + h], vf, o[h]);
          P.attn[(size_t)(head0 + h) * 128 + d] = o[h];
        }
      }
      grid_arrive(sync, kCtrAttn);
      issue_upto(consumed + S);  // the ring runs on into the next layer's pages while the grid works
      lpos = ring_advance(lpos, 2 * np, S);
    }
    if (!alive && tid == 0) {
      // let the copies this CTA issued land before it exits (bounded)
      for (int A = consumed; A < issued; ++A)
        if (!item_wait(A)) break;
    }
    return;
  }

  // ===================== matmul CTA gi of G =====================
  const int gi = (int)blockIdx.x - n_attn;
  const int Nr[4] = {nqkv, H, 2 * F, H}, Kc[4] = {H, qd, H, F};
  int r0[4], nr[4], kw4[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    r0[p] = (int)((long long)gi * Nr[p] / G);
    nr[p] = (int)((long long)(gi + 1) * Nr[p] / G) - r0[p];
    kw4[p] = (Kc[p] + 63) / 64;
  }
  float* row = reinterpret_cast<float*>(sm + P.row_off);
  int8_t* xq = reinterpret_cast<int8_t*>(sm + P.xq_off);
  float* hown = reinterpret_cast<float*>(sm + P.hown_off);  // h[r0[1] + i]: o and down share the row split
  const uint4* xs = reinterpret_cast<const uint4*>(xq);
  if (tid == 0) {
    for (int p = 0; p < 4; ++p) mbar_init(smem_u32(&bar[p]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();
  int pend[4] = {-1, -1, -1, -1};  // thread 0: layer of a copy into the slot not yet waited for
  auto issue = [&](int p, int l) {
    if (tid != 0 || l >= L || nr[p] == 0) return;
    const uint32_t bytes = (uint32_t)nr[p] * (uint32_t)kw4[p] * 16u;
    const uint8_t* src = reinterpret_cast<const uint8_t*>(P.layers[l].w[p]) + (size_t)r0[p] * kw4[p] * 16;
    fence_proxy_async();
    mbar_expect_tx(smem_u32(&bar[p]), bytes);
    bulk_copy(sm_s + P.slot_off[p], src, bytes, smem_u32(&bar[p]), pol);
    pend[p] = l;
  };
  auto slot_wait = [&](int p, int l) {
    if (nr[p] == 0) return true;
    const bool ok = copy_wait(smem_u32(&bar[p]), (uint32_t)l & 1u, sync, status);
    if (tid == 0) pend[p] = -1;
    return ok;
  };
#pragma unroll
  for (int p = 0; p < 4; ++p) issue(p, 0);
  float4 v[kD1U], wv[kD1U];
  norm_gains(wv, P.layers[0].norm[0], H);
  // embedding row (bf16 -> f32); this CTA's rows of h, which only it adds to
  {
    uint32_t tok = __ldg(P.token);
    if (tok >= (uint32_t)P.V) {
      if (tid == 0) atomicOr(status, kStatusBadToken);
      tok = 0;
    }
    const uint2* er = reinterpret_cast<const uint2*>(P.embed + (size_t)tok * H);
    uint2 e[kD1U];
#pragma unroll
    for (int u = 0; u < kD1U; ++u) {
      const int j = tid + kD1Threads * u;
      if (j < (H >> 2)) e[u] = __ldg(er + j);
    }
#pragma unroll
    for (int u = 0; u < kD1U; ++u) {
      const int j = tid + kD1Threads * u;
      if (j < (H >> 2)) {
        v[u] = make_float4(bf_lo(e[u].x), bf_hi(e[u].x), bf_lo(e[u].y), bf_hi(e[u].y));
        reinterpret_cast<float4*>(row)[j] = v[u];
      }
    }
    __syncthreads();
    for (int i = tid; i < nr[1]; i += kD1Threads) {
      hown[i] = row[r0[1] + i];
      P.h[r0[1] + i] = hown[i];
    }
  }
  int l = 0;
  for (; l < L; ++l) {
    const D1Layer& Lw = P.layers[l];
    // the layer's scales, loaded ahead of the norms that precede their use
    const float l_sq = __ldg(&Lw.sq), l_sk = __ldg(&Lw.sk), l_sv = __ldg(&Lw.sv), l_so = __ldg(&Lw.so),
                l_sg = __ldg(&Lw.sg), l_su = __ldg(&Lw.su), l_sd = __ldg(&Lw.sd);
    // ---- attention block ----
    if (l > 0) load_row(v, row, P.h, H);
    float am = d1_norm_quant(v, wv, row, H, P.eps, xq, kw4[0] * 64, &s_bc, red_f, red_b, status);
    {
      const D1Epi ep = d1_epi(l_sq, l_sk, l_sv, qd, qd + kvd, am);
      if (!slot_wait(0, l)) break;
      d1_gemv_any(sm_s + P.slot_off[0], nr[0], kw4[0], xs, ep, r0[0], P.qkv, nullptr);
    }
    grid_arrive(sync, kCtrQkv);  // (its __syncthreads also ends every read of the slot)
    issue(0, l + 1);
    norm_gains(wv, Lw.norm[1], qd);
    if (!grid_wait(sync, kCtrAttn, (uint32_t)((l + 1) * n_attn), status)) break;
    load_row(v, row, P.attn, qd);
    am = d1_norm_quant(v, wv, row, qd, P.eps, xq, kw4[1] * 64, &s_bc, red_f, red_b, status);
    {
      const D1Epi ep = d1_epi(l_so, l_so, l_so, H, H, am);
      if (!slot_wait(1, l)) break;
      d1_gemv_any(sm_s + P.slot_off[1], nr[1], kw4[1], xs, ep, r0[1], P.h, hown);
    }
    grid_arrive(sync, kCtrO);
    issue(1, l + 1);
    norm_gains(wv, Lw.norm[2], H);
    if (!grid_wait(sync, kCtrO, (uint32_t)((l + 1) * G), status)) break;
    // ---- FFN block ----
    load_row(v, row, P.h, H);
    am = d1_norm_quant(v, wv, row, H, P.eps, xq, kw4[2] * 64, &s_bc, red_f, red_b, status);
    {
      const D1Epi ep = d1_epi(l_sg, l_su, l_su, F, 2 * F, am);
      if (!slot_wait(2, l)) break;
      d1_gemv_any(sm_s + P.slot_off[2], nr[2], kw4[2], xs, ep, r0[2], P.gu, nullptr);
    }
    grid_arrive(sync, kCtrGu);
    issue(2, l + 1);
    norm_gains(wv, Lw.norm[3], F);
    if (!grid_wait(sync, kCtrGu, (uint32_t)((l + 1) * G), status)) break;
    load_gate_up(v, row, P.gu, F);
    am = d1_norm_quant(v, wv, row, F, P.eps, xq, kw4[3] * 64, &s_bc, red_f, red_b, status);
    {
      const D1Epi ep = d1_epi(l_sd, l_sd, l_sd, H, H, am);
      if (!slot_wait(3, l)) break;
      d1_gemv_any(sm_s + P.slot_off[3], nr[3], kw4[3], xs, ep, r0[3], P.h, hown);
    }
    grid_arrive(sync, kCtrDown);
    issue(3, l + 1);
    if (l + 1 < L) {
      norm_gains(wv, P.layers[l + 1].norm[0], H);
      if (!grid_wait(sync, kCtrDown, (uint32_t)((l + 1) * G), status)) break;
    }
  }
  // the final RMSNorm of h (rms_norm_kernel's operations) by the first matmul CTA once every down-projection is in
  if (l == L && gi == 0 && P.hn && grid_wait(sync, kCtrDown, (uint32_t)(L * G), status)) {
    norm_gains(wv, P.final_norm, H);
    load_row(v, row, P.h, H);
    __syncthreads();
    const float inv = d1_rms_inv(row, H, P.eps, &s_bc);
#pragma unroll
    for (int u = 0; u < kD1U; ++u) {
      const int j = tid + kD1Threads * u;
      if (j < (H >> 2))
        reinterpret_cast<float4*>(P.hn)[j] =
            make_float4(__fmul_rn(__fmul_rn(v[u].x, inv), wv[u].x), __fmul_rn(__fmul_rn(v[u].y, inv), wv[u].y),
                        __fmul_rn(__fmul_rn(v[u].z, inv), wv[u].z), __fmul_rn(__fmul_rn(v[u].w, inv), wv[u].w));
    }
  }
  if (tid == 0)  // normally nothing is in flight here; after an abort, issued copies land first (bounded)
    for (int p = 0; p < 4; ++p)
      if (pend[p] >= 0 && !mbar_wait(smem_u32(&bar[p]), (uint32_t)pend[p] & 1u, nullptr)) break;
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
namespace {

template <int HPC>
void* d1_fn() {
  return reinterpret_cast<void*>(&decode1_kernel<HPC>);
}
void* d1_kernel_for(int hpc) {
  switch (hpc) {
    case 1: return d1_fn<1>();
    case 2: return d1_fn<2>();
    case 4: return d1_fn<4>();
    case 8: return d1_fn<8>();
  }
  return nullptr;
}

}  // namespace

int decode1_hpc(int nh, int nkv) {
  if (nkv <= 0 || nh % nkv != 0) return 0;
  const int gq = nh / nkv;
  if (gq != 1 && gq != 2 && gq != 4 && gq != 8) return 0;
  int hpc = 1;
  while (nh / hpc > kD1MaxAttn && hpc < gq) hpc *= 2;
  return hpc;
}

bool decode1_supported(int nh, int nkv, int H, int F, const KvGeom& g) {
  if (!g.bf16 || g.hd != 128 || decode1_hpc(nh, nkv) == 0) return false;
  const int qd = nh * 128, dmax = std::max(std::max(H, qd), F);
  return H % 8 == 0 && F % 8 == 0 && H > 0 && F > 0 && dmax <= kD1U * 4 * kD1Threads;
}

size_t decode1_plan(D1Params* P, int sms, int cap, size_t smem_limit) {
  P->hpc = decode1_hpc(P->nh, P->nkv);
  if (!P->hpc) return 0;
  const int G = sms - P->nh / P->hpc;
  if (G < 1 || cap < 1) return 0;
  const int qd = P->nh * 128, kvd = P->nkv * 128, nqkv = qd + 2 * kvd;
  const int N[4] = {nqkv, P->H, 2 * P->F, P->H}, K[4] = {P->H, qd, P->H, P->F};
  size_t off = 0;
  for (int p = 0; p < 4; ++p) {
    const size_t bytes = round_up(ceil_div((size_t)N[p], (size_t)G) * (padded_cols((size_t)K[p]) / 4), 128);
    if (bytes >= (1u << 20)) return 0;  // an mbarrier transaction count
    P->slot_off[p] = (uint32_t)off;
    P->slot_bytes[p] = (uint32_t)bytes;
    off += bytes;
  }
  const size_t dmax = std::max(std::max((size_t)P->H, (size_t)qd), (size_t)P->F);
  P->row_off = (uint32_t)off;
  off += round_up(dmax * 4, 128);
  P->xq_off = (uint32_t)off;
  off += round_up(padded_cols(dmax), 128);
  P->hown_off = (uint32_t)off;
  off += round_up(ceil_div((size_t)P->H, (size_t)G) * 4, 128);
  const size_t scb = round_up((size_t)cap * (size_t)P->hpc * 4, 128);
  const size_t need = std::max(off, (size_t)kD1MinRing * kD1Page + scb);
  const int S = (int)std::min<size_t>((size_t)kD1MaxRing, (need - scb) / kD1Page);
  P->ring_slots = S;
  P->sc_off = (uint32_t)((size_t)S * kD1Page);
  P->cap = cap;
  const size_t dyn = std::max(need, (size_t)S * kD1Page + scb) + 1024;  // + alignment of the base to 1024
  return dyn <= smem_limit ? dyn : 0;
}

size_t decode1_smem_limit(int hpc) {
  void* fn = d1_kernel_for(hpc);
  int dev = 0, optin = 0;
  cudaFuncAttributes fa{};
  if (!fn || cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
      cudaFuncGetAttributes(&fa, fn) != cudaSuccess)
    return 0;
  const size_t lim = (size_t)optin > fa.sharedSizeBytes ? (size_t)optin - fa.sharedSizeBytes : 0;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lim) != cudaSuccess) return 0;
  return lim;
}

bool decode1_fits(int hpc, int grid, size_t smem) {
  void* fn = d1_kernel_for(hpc);
  int dev = 0, sms = 0, per_sm = 0;
  if (!fn || cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kD1Threads, smem) != cudaSuccess)
    return false;
  return per_sm >= 1 && grid <= per_sm * sms;
}

int launch_decode1(const D1Params& P, const CUtensorMap& tmap, int grid, size_t smem, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kD1Threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the grid counters need it
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaErrorInvalidValue;
  switch (P.hpc) {
    case 1: e = cudaLaunchKernelEx(&cfg, decode1_kernel<1>, P, tmap); break;
    case 2: e = cudaLaunchKernelEx(&cfg, decode1_kernel<2>, P, tmap); break;
    case 4: e = cudaLaunchKernelEx(&cfg, decode1_kernel<4>, P, tmap); break;
    case 8: e = cudaLaunchKernelEx(&cfg, decode1_kernel<8>, P, tmap); break;
  }
  count_launch();
  return e == cudaSuccess ? 0 : (int)e;
}

size_t decode1_sync_bytes() { return (size_t)(kCtrAbort + 1) * kD1SyncStride * sizeof(uint32_t); }

}  // namespace bitnet
