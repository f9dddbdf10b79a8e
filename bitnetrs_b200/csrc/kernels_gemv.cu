// kernels_gemv.cu — ternary (2-bit) x int8 matmul for the bitnetrs hot path.
//
// All variants compute the exact int32 sum of the reference
// (gemv.rs:299-308, `dot_packed_ternary_i8_fast`) via the identity
//     sum_k (1 - c_k) x_k = rowsum(x) - sum_k c_k x_k,   c_k in {0,1,2}
// so the device only ever multiplies unsigned 2-bit codes by int8
// activations: the codes come out of the packed word with one shift and one
// mask, with no decode table and no sign handling (the -128 x -1 edge of
// simd.rs:1569-1590 is exact by construction).  The f32 epilogue is the
// reference's `acc as f32 * (weight_scale * act_absmax / 127)`.
#include "kernels.cuh"

namespace bitnet {

// ---------------------------------------------------------------------------
// PTX helpers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc, int src_bytes) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gsrc), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}
__device__ __forceinline__ void ldmatrix_x4(uint32_t r[4], const void* smem_row) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(smem_row);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}
// D += A(s8, 16x32 row) * B(u8, 32x8 col), int32 accumulate.
__device__ __forceinline__ void mma_s8u8(int32_t c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void epilogue_store(float* out, int ldo, int m, int n, float v, Epi epi) {
  float* p = out + (size_t)m * ldo + n;
  if (epi == Epi::Residual)
    *p = __fadd_rn(*p, v);  // axpy_f32_fast(1.0, o, h): fma(1, o, h) == h + o
  else
    *p = v;
}

// ---------------------------------------------------------------------------
// M = 1 GEMV (decode).  A warp owns R consecutive rows.  Every lane first
// issues its 16-byte streaming loads of those rows (chunk lane + 32 j of each
// row, j < CH), then the block stages x in shared memory and sums it while
// the weight loads are in flight, then each lane multiplies its codes by x
// with dp4a and the warp reduces.  One DRAM round trip per block, every load
// 128-bit and coalesced.
// ---------------------------------------------------------------------------
template <int R, int CH>
__global__ void __launch_bounds__(256) gemv_m1_kernel(const uint32_t* __restrict__ W, int N, int kw,
                                                      const int8_t* __restrict__ xq, const float* __restrict__ amax,
                                                      Segments seg, Epi epi, float* __restrict__ out,
                                                      int32_t* __restrict__ acc_out) {
  extern __shared__ uint4 xs4[];  // kw*16 bytes of x
  __shared__ int red[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int kw4 = kw >> 2;  // 16-byte chunks per row
  const int row0 = (blockIdx.x * 8 + warp) * R;
  const uint4* W4 = reinterpret_cast<const uint4*>(W);
  pdl_launch_dependents();
  uint4 w[R][CH];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int j = 0; j < CH; ++j) {
      const int c = lane + 32 * j;
      w[r][j] = (row0 + r < N && c < kw4) ? __ldcs(W4 + (size_t)(row0 + r) * kw4 + c) : make_uint4(0, 0, 0, 0);
    }
  pdl_wait();  // weights are constant; x and out belong to the previous kernels
  xq = after_wait(xq);
  amax = after_wait(amax);
  out = after_wait(out);
  int xsum = 0;
  const uint4* xg = reinterpret_cast<const uint4*>(xq);
  for (int i = threadIdx.x; i < kw; i += 256) {
    const uint4 v = xg[i];
    xs4[i] = v;
    xsum = __dp4a((int)v.x, 0x01010101, xsum);
    xsum = __dp4a((int)v.y, 0x01010101, xsum);
    xsum = __dp4a((int)v.z, 0x01010101, xsum);
    xsum = __dp4a((int)v.w, 0x01010101, xsum);
  }
  xsum = warp_sum_i(xsum);
  if (lane == 0) red[warp] = xsum;
  __syncthreads();
  xsum = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) xsum += red[k];
  if (row0 >= N) return;
  int acc[R][4];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[r][i] = 0;
#pragma unroll
  for (int j = 0; j < CH; ++j) {
    const int c = lane + 32 * j;
    if (c < kw4) {
      const uint4* x = xs4 + 4 * c;
      const uint4 xv[4] = {x[0], x[1], x[2], x[3]};
#pragma unroll
      for (int r = 0; r < R; ++r) {
        dp4a_word_scaled(w[r][j].x, xv[0], acc[r]);
        dp4a_word_scaled(w[r][j].y, xv[1], acc[r]);
        dp4a_word_scaled(w[r][j].z, xv[2], acc[r]);
        dp4a_word_scaled(w[r][j].w, xv[3], acc[r]);
      }
    }
  }
  const float am = amax[0];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int s = warp_sum_i(codes_sum(acc[r]));
    if (lane == 0 && row0 + r < N) {
      const int n = row0 + r;
      const int32_t a = xsum - s;
      if (acc_out) acc_out[n] = a;
      epilogue_store(out, 0, 0, n, dequant(a, seg_scale(seg, n), am), epi);
    }
  }
}

// M = 1 for rows longer than 8192 codes: each warp streams R rows as one
// run of 16-byte chunks.
template <int R>
__global__ void __launch_bounds__(128) gemv_m1_long_kernel(const uint32_t* __restrict__ W, int N, int kw,
                                                      const int8_t* __restrict__ xq, const float* __restrict__ amax,
                                                      Segments seg, Epi epi, float* __restrict__ out,
                                                      int32_t* __restrict__ acc_out) {
  extern __shared__ uint4 xs4[];  // kw*16 bytes of x
  __shared__ int red[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int kw4 = kw >> 2;  // uint4 chunks per row
  int xsum = 0;
  const uint4* xg = reinterpret_cast<const uint4*>(xq);
  for (int i = threadIdx.x; i < kw; i += blockDim.x) {
    uint4 v = xg[i];
    xs4[i] = v;
    xsum = __dp4a((int)v.x, 0x01010101, xsum);
    xsum = __dp4a((int)v.y, 0x01010101, xsum);
    xsum = __dp4a((int)v.z, 0x01010101, xsum);
    xsum = __dp4a((int)v.w, 0x01010101, xsum);
  }
  xsum = block_reduce(xsum, [](int a, int b) { return a + b; }, red);  // includes __syncthreads

  const int row0 = (blockIdx.x * (blockDim.x >> 5) + warp) * R;
  if (row0 >= N) return;
  const int nrows = min(R, N - row0);
  const uint4* wp = reinterpret_cast<const uint4*>(W + (size_t)row0 * kw);
  const int total = nrows * kw4;
  int acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0;
  for (int i = lane; i < total; i += 32) {
    uint4 w = __ldcs(wp + i);  // streamed once: evict-first
    int r = i / kw4, c = i - r * kw4;
    const uint4* x = xs4 + 4 * c;
    int dd[4] = {0, 0, 0, 0};
    dp4a_word_scaled(w.x, x[0], dd);
    dp4a_word_scaled(w.y, x[1], dd);
    dp4a_word_scaled(w.z, x[2], dd);
    dp4a_word_scaled(w.w, x[3], dd);
    const int d = codes_sum(dd);
#pragma unroll
    for (int rr = 0; rr < R; ++rr)
      if (r == rr) acc[rr] += d;
  }
  const float am = amax[0];
#pragma unroll
  for (int rr = 0; rr < R; ++rr) {
    int s = warp_sum_i(acc[rr]);
    if (lane == 0 && rr < nrows) {
      int n = row0 + rr;
      int32_t a = xsum - s;
      if (acc_out) acc_out[n] = a;
      epilogue_store(out, 0, 0, n, dequant(a, seg_scale(seg, n), am), epi);
    }
  }
}

// ---------------------------------------------------------------------------
// M > 1: tensor-core GEMM (mma.sync m16n8k32, s8 activations x u8 codes).
// A 128-column k-tile of W is 32 packed bytes per row; codes are expanded in
// registers straight into the B fragment (thread t of a quad needs element
// group 4t..4t+3 of each 16-column word = one shift + mask).
// ---------------------------------------------------------------------------
template <int BM, int BN, int WARPS_M, int WARPS_N>
__global__ void __launch_bounds__(WARPS_M* WARPS_N * 32)
    ternary_mma_kernel(const uint32_t* __restrict__ W, int N, int kw, const int8_t* __restrict__ X, int ldq, int M,
                       const float* __restrict__ amax, const int32_t* __restrict__ rowsum, Segments seg, Epi epi,
                       float* __restrict__ out, int ldo, int32_t* __restrict__ acc_out) {
  constexpr int BK = 128;
  constexpr int XS = BK + 16;  // conflict-free ldmatrix rows
  constexpr int WS = 48;       // 32 data bytes + 16 pad
  constexpr int STAGES = 3;
  constexpr int NTH = WARPS_M * WARPS_N * 32;
  constexpr int WTM = BM / WARPS_M, WTN = BN / WARPS_N;
  constexpr int MT = WTM / 16, NT = WTN / 8;
  extern __shared__ __align__(16) uint8_t smem[];
  uint8_t* xs = smem;
  uint8_t* wsm = smem + STAGES * BM * XS;
  pdl_launch_dependents();
  pdl_wait();
  X = after_wait(X);
  amax = after_wait(amax);
  rowsum = after_wait(rowsum);
  out = after_wait(out);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int wm = warp / WARPS_N, wn = warp % WARPS_N;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int Kpad = kw * 16;
  const int ktiles = (Kpad + BK - 1) / BK;

  auto load_tile = [&](int stage, int kt) {
    const int kb = kt * BK;
    for (int c = threadIdx.x; c < BM * 8; c += NTH) {
      int r = c >> 3, sg = c & 7;
      int gm = m0 + r, k = kb + sg * 16;
      bool ok = gm < M && k < Kpad;
      const int8_t* src = ok ? X + (size_t)gm * ldq + k : X;
      cp_async16(xs + (stage * BM + r) * XS + sg * 16, src, ok ? 16 : 0);
    }
    for (int c = threadIdx.x; c < BN * 2; c += NTH) {
      int r = c >> 1, sg = c & 1;
      int gn = n0 + r, wd = kt * 8 + sg * 4;
      bool ok = gn < N && wd < kw;
      const uint32_t* src = ok ? W + (size_t)gn * kw + wd : W;
      cp_async16(wsm + (stage * BN + r) * WS + sg * 16, src, ok ? 16 : 0);
    }
  };

  int32_t acc[MT][NT][4];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[i][j][q] = 0;

#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < ktiles) load_tile(s, s);
    cp_async_commit();
  }
  for (int kt = 0; kt < ktiles; ++kt) {
    cp_async_wait<STAGES - 2>();
    __syncthreads();
    int nk = kt + STAGES - 1;
    if (nk < ktiles) load_tile(nk % STAGES, nk);
    cp_async_commit();
    const int stage = kt % STAGES;
    const uint8_t* xst = xs + stage * BM * XS;
    const uint8_t* wst = wsm + stage * BN * WS;
#pragma unroll
    for (int ks = 0; ks < BK / 32; ++ks) {
      uint32_t a[MT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        int row = wm * WTM + mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        ldmatrix_x4(a[mt], xst + row * XS + ks * 32 + (lane >> 4) * 16);
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        int row = wn * WTN + nt * 8 + (lane >> 2);
        uint2 wv = *reinterpret_cast<const uint2*>(wst + row * WS + ks * 8);
        int sh = 2 * (lane & 3);
        uint32_t b0 = (wv.x >> sh) & 0x03030303u, b1 = (wv.y >> sh) & 0x03030303u;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) mma_s8u8(acc[mt][nt], a[mt], b0, b1);
      }
    }
  }
  cp_async_wait<0>();

#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      int m = m0 + wm * WTM + mt * 16 + (lane >> 2) + half * 8;
      if (m >= M) continue;
      float am = amax[m];
      int32_t rs = rowsum[m];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          int n = n0 + wn * WTN + nt * 8 + 2 * (lane & 3) + e;
          if (n >= N) continue;
          int32_t a = rs - acc[mt][nt][half * 2 + e];
          if (acc_out) acc_out[(size_t)m * N + n] = a;
          epilogue_store(out, ldo, m, n, dequant(a, seg_scale(seg, n), am), epi);
        }
      }
    }
  }
}

template <int BM, int BN, int WM, int WN>
static void run_mma(const uint32_t* W, int N, int kw, const int8_t* xq, int ldq, int M, const float* amax,
                    const int32_t* rowsum, const Segments& seg, Epi epi, float* out, int ldo, int32_t* acc,
                    cudaStream_t st) {
  constexpr int smem = 3 * (BM * (128 + 16) + BN * 48);
  static_assert(smem <= 48 * 1024, "dynamic shared memory above the default limit");
  dim3 grid((unsigned)ceil_div(N, BN), (unsigned)ceil_div(M, BM));
  ternary_mma_kernel<BM, BN, WM, WN><<<grid, WM * WN * 32, smem, st>>>(W, N, kw, xq, ldq, M, amax, rowsum, seg, epi,
                                                                      out, ldo, acc);
  count_launch();
}

// cudaFuncAttributes::binaryVersion of a kernel of this library on the current
// device (the SASS architecture the driver loaded, major * 10 + minor).
int kernel_binary_version(int* v) {
  cudaFuncAttributes fa{};
  const cudaError_t e = cudaFuncGetAttributes(&fa, gemv_m1_kernel<1, 2>);
  if (e != cudaSuccess) return (int)e;
  *v = fa.binaryVersion;
  return 0;
}

static bool g_tc_ready = false;  // ternary_tc_prepare succeeded on every device set up so far
void set_ternary_tc_ready(bool ready) { g_tc_ready = ready; }
bool ternary_tc_ready() { return g_tc_ready; }

void launch_ternary_matmul(const uint32_t* W, int N, int K, const int8_t* xq, int ldq, const float* act_absmax,
                           const int32_t* row_sum, int M, const Segments& seg, Epi epi, float* out, int ldo,
                           int32_t* acc, cudaStream_t st, int32_t* status) {
  const int kw = (int)words_per_row(K);
  if (M <= 0 || N <= 0) return;
  // every multi-row product runs on the tensor cores when they are set up (measured faster than the
  // mma.sync kernels from M = 8 up, and never slower below)
  if (M > 1 && status && g_tc_ready &&
      launch_ternary_tc(W, N, K, xq, ldq, act_absmax, row_sum, M, seg, epi, out, ldo, acc, status, st) == 0)
    return;
  if (M == 1) {
    const int kw4 = kw / 4;
    const size_t smem = (size_t)kw * 16;
    if (kw4 > 32 * 8 || smem > 48 * 1024) {
      constexpr int R = 2;
      gemv_m1_long_kernel<R><<<(unsigned)ceil_div(N, 4 * R), 128, smem, st>>>(W, N, kw, xq, act_absmax, seg, epi,
                                                                              out, acc);
      count_launch();
      return;
    }
    // rows per warp: keep at least ~2 blocks of 8 warps per SM
    const int R = N >= 9472 ? 4 : (N >= 4736 ? 2 : 1);
    const unsigned grid = (unsigned)ceil_div(N, 8 * R);
#define BN_GEMV(RR, CC) \
  launch_pdl(gemv_m1_kernel<RR, CC>, dim3(grid), dim3(256), smem, st, W, N, kw, xq, act_absmax, seg, epi, out, acc)
#define BN_GEMV_R(CC) \
  do {                \
    if (R == 4)       \
      BN_GEMV(4, CC); \
    else if (R == 2)  \
      BN_GEMV(2, CC); \
    else              \
      BN_GEMV(1, CC); \
  } while (0)
    if (kw4 <= 32)
      BN_GEMV_R(1);
    else if (kw4 <= 64)
      BN_GEMV_R(2);
    else if (kw4 <= 128)
      BN_GEMV_R(4);
    else
      BN_GEMV_R(8);
#undef BN_GEMV_R
#undef BN_GEMV
    count_launch();
    return;
  }
  if (M <= 16)
    run_mma<16, 64, 1, 4>(W, N, kw, xq, ldq, M, act_absmax, row_sum, seg, epi, out, ldo, acc, st);
  else if (M <= 64)
    run_mma<64, 64, 2, 2>(W, N, kw, xq, ldq, M, act_absmax, row_sum, seg, epi, out, ldo, acc, st);
  else
    run_mma<64, 128, 2, 4>(W, N, kw, xq, ldq, M, act_absmax, row_sum, seg, epi, out, ldo, acc, st);
}

__global__ void row_sum_kernel(const int8_t* __restrict__ xq, int ldq, int K, int32_t* __restrict__ out) {
  __shared__ int red[32];
  int m = blockIdx.x, s = 0;
  for (int i = threadIdx.x; i < K; i += blockDim.x) s += xq[(size_t)m * ldq + i];
  s = block_reduce(s, [](int a, int b) { return a + b; }, red);
  if (threadIdx.x == 0) out[m] = s;
}
void launch_row_sum(const int8_t* xq, int ldq, int M, int K, int32_t* row_sum, cudaStream_t st) {
  if (M <= 0) return;
  row_sum_kernel<<<M, 256, 0, st>>>(xq, ldq, K, row_sum);
  count_launch();
}

// ---------------------------------------------------------------------------
// ternary_gemv_f32 (gemv.rs:108-165 -> simd.rs:572-610 + 190-262).  One warp
// per row; lane c computes 32-element chunk sums exactly like
// dot_ternary_f32_avx2 (8 lanes, mul, w==0 lanes forced to +0, add, hsum);
// lane 0 then adds the chunk sums in order and runs the scalar tail.
// ---------------------------------------------------------------------------
__global__ void gemv_f32_kernel(const uint8_t* __restrict__ packed, int N, int K, float ws,
                                const float* __restrict__ x, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= N) return;
  const int pc = (K + 3) / 4;
  const uint8_t* wr = packed + (size_t)row * pc;
  const int full = K / 32, rem = K % 32;
  float total = 0.0f;
  for (int base = 0; base < full; base += 32) {
    int c = base + lane;
    float cs = 0.0f;
    if (c < full) {
      float a[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] = 0.0f;
#pragma unroll
      for (int sub = 0; sub < 4; ++sub) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          int e = 32 * c + 8 * sub + j;
          int code = (wr[e >> 2] >> (2 * (e & 3))) & 3;
          float w = code == 0 ? 1.0f : (code == 2 ? -1.0f : 0.0f);
          float p = (w == 0.0f) ? 0.0f : __fmul_rn(w, x[e]);
          a[j] = __fadd_rn(a[j], p);
        }
      }
      cs = hsum8(a);
    }
    int cnt = min(32, full - base);
    for (int i = 0; i < cnt; ++i) {
      float v = __shfl_sync(0xffffffffu, cs, i);
      total = __fadd_rn(total, v);
    }
  }
  if (lane == 0) {
    for (int i = 0; i < rem; ++i) {
      int e = full * 32 + i;
      int code = (wr[e >> 2] >> (2 * (e & 3))) & 3;
      float w = code == 0 ? 1.0f : (code == 2 ? -1.0f : 0.0f);
      total = __fadd_rn(total, __fmul_rn(w, x[e]));
    }
    out[row] = __fmul_rn(total, ws);
  }
}

void launch_ternary_gemv_f32(const uint8_t* packed, int N, int K, float ws, const float* x, float* out,
                             cudaStream_t st) {
  if (N <= 0) return;
  gemv_f32_kernel<<<(unsigned)ceil_div(N, 4), 128, 0, st>>>(packed, N, K, ws, x, out);
  count_launch();
}

}  // namespace bitnet
