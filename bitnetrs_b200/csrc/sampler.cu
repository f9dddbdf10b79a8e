// sampler.cu — sample_next_token (crates/bitnet-inference/src/lib.rs:236-390)
// on the GPU, in the reference's arithmetic order, one CTA per call:
//   1. repetition penalty: logits[t] /= penalty once per occurrence of t in
//      the history (occurrences counted with atomics, the first occurrence
//      applies the divisions; the count table is left at zero);
//   2. temperature: logits *= 1/t when |t - 1| > 1e-6;
//   3. top_k == 1: greedy argmax (ties to the later index);
//   4. top-k: the k-th largest value by an exact radix select on the
//      order-preserving bits of the logits; smaller logits become -inf;
//   5. top-p: softmax over the finite logits (max, exp, sequential sum in
//      index order, * 1/sum), indices ordered by probability (descending,
//      equal probabilities in ascending index order: the reference's
//      sort_unstable leaves that order unspecified), the smallest prefix whose
//      sequential cumulative probability reaches p kept, the rest -inf;
//   6. softmax over the finite logits, one LCG step (seed + history length),
//      and the inverse-CDF draw in index order; argmax fallback.
// Sums over the finite logits skip the others, whose terms are exactly +0.
// The finite logits are gathered in index order into shared memory when
// there are at most kMaxCand of them; a larger set is supported without
// top-p (the sums then stream over the vocabulary through shared memory)
// and reported as unsupported with top-p.
#include "internal.h"

namespace bitnet {

namespace {

constexpr int kThreads = 1024;
constexpr int kMaxCand = 4096;  // finite logits held in shared memory
constexpr int kChunk = 4096;    // streamed values per serial-sum chunk (large path)
constexpr int kSampleUnsupported = 1;

__device__ __forceinline__ uint32_t order_key(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Block-wide max of v (all threads call; result for every thread).
__device__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
  for (int i = 1; i < kThreads / 32; ++i) r = fmaxf(r, red[i]);
  return r;
}

// Block-wide argmax as Iterator::max_by with partial_cmp: the largest value,
// ties to the larger index (NaN compares equal; the logits are NaN-free).
__device__ void argmax_merge(float& bv, uint32_t& bi, float v, uint32_t i) {
  if (v > bv || (v == bv && i > bi)) {
    bv = v;
    bi = i;
  }
}
__device__ uint32_t block_argmax(float v, uint32_t i, float* redv, uint32_t* redi) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) argmax_merge(v, i, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, i, o));
  __syncthreads();
  if (lane == 0) {
    redv[warp] = v;
    redi[warp] = i;
  }
  __syncthreads();
  float bv = redv[0];
  uint32_t bi = redi[0];
  for (int w = 1; w < kThreads / 32; ++w) argmax_merge(bv, bi, redv[w], redi[w]);
  return bi;
}

// Exclusive prefix of `flag` over the block in thread order; *total gets the sum.
__device__ int block_rank(int flag, int* warp_cnt, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t b = __ballot_sync(0xffffffffu, flag);
  const int in_warp = __popc(b & ((1u << lane) - 1u));
  __syncthreads();
  if (lane == 0) warp_cnt[warp] = __popc(b);
  __syncthreads();
  int before = 0, all = 0;
  for (int w = 0; w < kThreads / 32; ++w) {
    const int c = warp_cnt[w];
    if (w < warp) before += c;
    all += c;
  }
  *total = all;
  return before + in_warp;
}

}  // namespace

// counts: [V] int32, zero on entry and on exit; escratch: [V] floats (the
// streamed path); out: the token; status |= kSampleUnsupported when top-p
// meets more than kMaxCand finite logits.  Dynamic shared memory:
// kMaxCand * (4 + 4 + 4 + 8) bytes.
__global__ void __launch_bounds__(kThreads) sample_kernel(float* __restrict__ logits, uint32_t V, float temperature,
                                                        float top_p, uint32_t top_k, float penalty, uint64_t seed,
                                                        const uint32_t* __restrict__ past, uint32_t n_past,
                                                        int32_t* __restrict__ counts, float* __restrict__ escratch,
                                                        uint32_t* __restrict__ out, int32_t* __restrict__ status,
                                                        ExpTable et) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint32_t* cidx = reinterpret_cast<uint32_t*>(smem);                  // finite logits' indices, ascending
  float* cval = reinterpret_cast<float*>(cidx + kMaxCand);             // their logits
  float* cprob = cval + kMaxCand;                                      // their probabilities
  unsigned long long* skey = reinterpret_cast<unsigned long long*>(cprob + kMaxCand);  // sort keys / stream chunk
  __shared__ float redv[32];
  __shared__ uint32_t redi[32];
  __shared__ int wcnt[32];
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_u[2];
  __shared__ float s_f[2];
  __shared__ int s_i[2];
  const int tid = threadIdx.x;
  const float ninf = -INFINITY;

  // 1. repetition penalty (lib.rs:246-253)
  if (penalty != 1.0f && n_past > 0) {
    for (uint32_t i = tid; i < n_past; i += kThreads)
      if (past[i] < V) atomicAdd(&counts[past[i]], 1);
    __syncthreads();
    for (uint32_t i = tid; i < n_past; i += kThreads) {
      const uint32_t t = past[i];
      if (t >= V) continue;
      const int c = atomicExch(&counts[t], 0);
      if (c > 0) {
        float x = logits[t];
        for (int k = 0; k < c; ++k) x = __fdiv_rn(x, penalty);
        logits[t] = x;
      }
    }
    __syncthreads();
  }
  // 2. temperature (lib.rs:256-261)
  if (fabsf(__fsub_rn(temperature, 1.0f)) > 1e-6f) {
    const float inv = __fdiv_rn(1.0f, temperature);
    for (uint32_t v = tid; v < V; v += kThreads) logits[v] = __fmul_rn(logits[v], inv);
  }
  __syncthreads();
  // 3. greedy shortcut (lib.rs:264-271)
  if (top_k == 1) {
    float bv = ninf;
    uint32_t bi = 0;
    for (uint32_t v = tid; v < V; v += kThreads) argmax_merge(bv, bi, logits[v], v);
    const uint32_t t = block_argmax(bv, bi, redv, redi);
    if (tid == 0) *out = t;
    return;
  }
  // 4. top-k (lib.rs:274-291): radix select of the k-th largest, 8 bits a pass
  if (top_k > 0 && top_k < V) {
    uint32_t prefix = 0, mask = 0, remaining = top_k;
    for (int shift = 24; shift >= 0; shift -= 8) {
      if (tid < 256) hist[tid] = 0;
      __syncthreads();
      for (uint32_t v = tid; v < V; v += kThreads) {
        const uint32_t key = order_key(logits[v]);
        if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xffu], 1u);
      }
      __syncthreads();
      if (tid == 0) {
        uint32_t cum = 0;
        for (int b = 255; b >= 0; --b) {
          if (cum + hist[b] >= remaining) {
            s_u[0] = prefix | ((uint32_t)b << shift);
            s_u[1] = remaining - cum;
            break;
          }
          cum += hist[b];
        }
      }
      __syncthreads();
      prefix = s_u[0];
      remaining = s_u[1];
      mask |= 0xffu << shift;
    }
    const float thr = key_value(prefix);
    for (uint32_t v = tid; v < V; v += kThreads)
      if (logits[v] < thr) logits[v] = ninf;
    __syncthreads();
  }
  // gather the finite logits in index order
  int n = 0;
  for (uint32_t base = 0; base < V; base += kThreads) {
    const uint32_t v = base + tid;
    const float x = v < V ? logits[v] : ninf;
    const int fin = v < V && isfinite(x);
    int total;
    const int r = block_rank(fin, wcnt, &total);
    if (fin && n + r < kMaxCand) {
      cidx[n + r] = v;
      cval[n + r] = x;
    }
    n += total;
  }
  __syncthreads();
  const uint64_t st = (seed + (uint64_t)n_past) * 6364136223846793005ULL + 1442695040888963407ULL;
  const float rf = __fdiv_rn(__ull2float_rn(st >> 11), 9007199254740992.0f);  // lib.rs:380-386
  if (n > kMaxCand) {
    if (top_p < 1.0f) {
      if (tid == 0) {
        atomicOr(status, kSampleUnsupported);
        *out = 0;
      }
      return;
    }
    // 6 over the whole vocabulary, streamed: e = exp(x - max) to escratch,
    // the sequential sum over chunks staged in shared memory
    float m = ninf;
    for (uint32_t v = tid; v < V; v += kThreads) {
      const float x = logits[v];
      if (isfinite(x)) m = fmaxf(m, x);
    }
    m = block_max(m, redv);
    float* chunk = reinterpret_cast<float*>(skey);
    float sum = 0.0f;
    for (uint32_t c0 = 0; c0 < V; c0 += kChunk) {
      const uint32_t len = min((uint32_t)kChunk, V - c0);
      for (uint32_t i = tid; i < len; i += kThreads) {
        const float x = logits[c0 + i];
        const float e = isfinite(x) ? exp_host_libm(__fsub_rn(x, m), et) : 0.0f;
        escratch[c0 + i] = e;
        chunk[i] = e;
      }
      __syncthreads();
      if (tid == 0)
        for (uint32_t i = 0; i < len; ++i) sum = __fadd_rn(sum, chunk[i]);
      __syncthreads();
    }
    if (tid == 0) s_f[0] = sum > 0.0f ? __fdiv_rn(1.0f, sum) : 1.0f;
    __syncthreads();
    const float inv = s_f[0];
    if (tid == 0) s_i[0] = -1;
    if (!(rf > 0.0f)) {
      if (tid == 0) *out = 0;
      return;
    }
    float cum = 0.0f;
    for (uint32_t c0 = 0; c0 < V; c0 += kChunk) {
      const uint32_t len = min((uint32_t)kChunk, V - c0);
      for (uint32_t i = tid; i < len; i += kThreads) chunk[i] = __fmul_rn(escratch[c0 + i], inv);
      __syncthreads();
      if (tid == 0)
        for (uint32_t i = 0; i < len; ++i) {
          cum = __fadd_rn(cum, chunk[i]);
          if (rf <= cum) {
            s_i[0] = (int)(c0 + i);
            break;
          }
        }
      __syncthreads();
      if (s_i[0] >= 0) break;
    }
    if (s_i[0] >= 0) {
      if (tid == 0) *out = (uint32_t)s_i[0];
      return;
    }
    float bv = ninf;
    uint32_t bi = 0;
    for (uint32_t v = tid; v < V; v += kThreads) argmax_merge(bv, bi, __fmul_rn(escratch[v], inv), v);
    const uint32_t t = block_argmax(bv, bi, redv, redi);
    if (tid == 0) *out = t;
    return;
  }
  // ---- at most kMaxCand finite logits, in shared memory, index order ----
  if (top_p < 1.0f && n > 0) {
    // 5. top-p (lib.rs:294-353): probabilities over the finite logits
    float m = ninf;
    for (int i = tid; i < n; i += kThreads) m = fmaxf(m, cval[i]);
    m = block_max(m, redv);
    for (int i = tid; i < n; i += kThreads) cprob[i] = exp_host_libm(__fsub_rn(cval[i], m), et);
    __syncthreads();
    if (tid == 0) {
      float sum = 0.0f;
      for (int i = 0; i < n; ++i) sum = __fadd_rn(sum, cprob[i]);
      s_f[0] = sum > 0.0f ? __fdiv_rn(1.0f, sum) : 1.0f;
    }
    __syncthreads();
    const float inv = s_f[0];
    // sort keys, ascending: larger probability first, then smaller index
    int P = 1;
    while (P < n) P <<= 1;
    for (int i = tid; i < P; i += kThreads) {
      if (i < n) {
        const float pr = __fmul_rn(cprob[i], inv);
        cprob[i] = pr;
        skey[i] = ~((((unsigned long long)__float_as_uint(pr)) << 32) | (unsigned long long)(0xffffffffu - cidx[i]));
      } else {
        skey[i] = ~0ull;
      }
    }
    __syncthreads();
    for (int k = 2; k <= P; k <<= 1)
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = tid; i < P; i += kThreads) {
          const int l = i ^ j;
          if (l > i) {
            const unsigned long long a = skey[i], b = skey[l];
            if (((i & k) == 0) ? a > b : a < b) {
              skey[i] = b;
              skey[l] = a;
            }
          }
        }
        __syncthreads();
      }
    if (tid == 0) {
      // the smallest prefix whose cumulative probability reaches top_p
      float cum = 0.0f;
      int cut = n;
      for (int r = 0; r < n; ++r) {
        cum = __fadd_rn(cum, __uint_as_float((uint32_t)(~skey[r] >> 32)));
        if (cum >= top_p) {
          cut = r + 1;
          break;
        }
      }
      s_i[0] = cut;
    }
    __syncthreads();
    const int cut = s_i[0];
    // every index past the cut leaves the finite set (and becomes -inf, as the
    // reference writes it into the logits)
    for (int r = cut + tid; r < n; r += kThreads) {
      const uint32_t v = 0xffffffffu - (uint32_t)(~skey[r]);
      logits[v] = ninf;
      int lo = 0, hi = n - 1;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (cidx[mid] < v)
          lo = mid + 1;
        else
          hi = mid;
      }
      cval[lo] = ninf;
    }
    __syncthreads();
    // compact the remaining finite logits, still in index order
    uint32_t* tidx = reinterpret_cast<uint32_t*>(skey);
    float* tval = cprob;
    int n2 = 0;
    for (int base = 0; base < n; base += kThreads) {
      const int i = base + tid;
      const int keep = i < n && isfinite(cval[i]);
      int total;
      const int r = block_rank(keep, wcnt, &total);
      if (keep) {
        tidx[n2 + r] = cidx[i];
        tval[n2 + r] = cval[i];
      }
      n2 += total;
    }
    __syncthreads();
    for (int i = tid; i < n2; i += kThreads) {
      cidx[i] = tidx[i];
      cval[i] = tval[i];
    }
    n = n2;
    __syncthreads();
  }
  // 6. softmax over the finite logits and the inverse-CDF draw (lib.rs:356-397)
  if (n == 0) {
    // no finite logit: every probability is 0; the draw takes index 0 when
    // the uniform is 0, else max_by falls back to the last index
    if (tid == 0) *out = rf > 0.0f ? V - 1 : 0;
    return;
  }
  float m = ninf;
  for (int i = tid; i < n; i += kThreads) m = fmaxf(m, cval[i]);
  m = block_max(m, redv);
  for (int i = tid; i < n; i += kThreads) cprob[i] = exp_host_libm(__fsub_rn(cval[i], m), et);
  __syncthreads();
  if (tid == 0) {
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) sum = __fadd_rn(sum, cprob[i]);
    s_f[0] = sum > 0.0f ? __fdiv_rn(1.0f, sum) : 1.0f;
  }
  __syncthreads();
  const float inv = s_f[0];
  for (int i = tid; i < n; i += kThreads) cprob[i] = __fmul_rn(cprob[i], inv);
  __syncthreads();
  if (tid == 0) {
    int tok = -1;
    if (!(rf > 0.0f)) {
      tok = 0;
    } else {
      float cum = 0.0f;
      for (int i = 0; i < n; ++i) {
        cum = __fadd_rn(cum, cprob[i]);
        if (rf <= cum) {
          tok = (int)cidx[i];
          break;
        }
      }
    }
    s_i[1] = tok;
  }
  __syncthreads();
  if (s_i[1] >= 0) {
    if (tid == 0) *out = (uint32_t)s_i[1];
    return;
  }
  float bv = ninf;
  uint32_t bi = 0;
  for (int i = tid; i < n; i += kThreads) argmax_merge(bv, bi, cprob[i], cidx[i]);
  const uint32_t t = block_argmax(bv, bi, redv, redi);
  if (tid == 0) *out = t;
}

size_t sampler_smem() { return (size_t)kMaxCand * (4 + 4 + 4 + 8); }

int sampler_prepare() {
  return cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sampler_smem()) ==
                 cudaSuccess
             ? 0
             : 1;
}

void launch_sample(float* logits, uint32_t V, const bitnet_cuda_sampling& c, const uint32_t* past, uint32_t n_past,
                   int32_t* counts, float* escratch, uint32_t* out, int32_t* status, const ExpTable& et,
                   cudaStream_t st) {
  sample_kernel<<<1, kThreads, sampler_smem(), st>>>(logits, V, c.temperature, c.top_p, c.top_k, c.repetition_penalty,
                                                     c.seed, past, n_past, counts, escratch, out, status, et);
  count_launch();
}

}  // namespace bitnet
