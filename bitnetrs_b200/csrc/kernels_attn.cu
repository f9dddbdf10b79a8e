// kernels_attn.cu — RoPE + paged KV store and GQA attention.
#include "kernels.cuh"

namespace bitnet {

__device__ __forceinline__ float exp_ref(float x) { return (float)exp((double)x); }

// ---------------------------------------------------------------------------
// Backend::masked_attention on the reference's head-major cache
// (attention.rs:97-209), in the reference's operation order:
//   score[t] = dot_f32_f32(q_h, K[t]) * (1/sqrt(hd))   (8 FMA chains + hsum + tail)
//   softmax_f32: max, exp(s - max), sequential sum, * (1/sum)
//   out = 0; for t: out = fma(p_t, V[t], out)          (axpy; tail dims mul+add)
// One block per query head.  `scratch` holds nh * seq_len floats.
// ---------------------------------------------------------------------------
__device__ float dot_ref(const float* a, const float* b, int n) {
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
  int chunks = n >> 3;
  for (int i = 0; i < chunks; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = __fmaf_rn(a[8 * i + j], b[8 * i + j], acc[j]);
  float r = hsum8(acc);
  for (int i = chunks * 8; i < n; ++i) r = __fadd_rn(r, __fmul_rn(a[i], b[i]));
  return r;
}

__global__ void masked_attention_headmajor_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                                  const float* __restrict__ vc, float* __restrict__ out, int nh,
                                                  int nkv, int hd, int stride, int seq_len, float* scratch) {
  __shared__ float red[32];
  __shared__ float bc[2];
  const int h = blockIdx.x;
  const int kvh = h / (nh / nkv);
  const float* qh = q + (size_t)h * hd;
  const float* kb = kc + (size_t)kvh * stride;
  const float* vb = vc + (size_t)kvh * stride;
  float* s = scratch + (size_t)h * seq_len;
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  for (int t = threadIdx.x; t < seq_len; t += blockDim.x) s[t] = __fmul_rn(dot_ref(qh, kb + (size_t)t * hd, hd), scale);
  __syncthreads();
  float m = -INFINITY;
  for (int t = threadIdx.x; t < seq_len; t += blockDim.x) m = fmaxf(m, s[t]);
  m = block_reduce(m, [](float a, float b) { return fmaxf(a, b); }, red);
  for (int t = threadIdx.x; t < seq_len; t += blockDim.x) s[t] = exp_ref(__fsub_rn(s[t], m));
  __syncthreads();
  if (threadIdx.x == 0) {
    float sum = 0.0f;
    for (int t = 0; t < seq_len; ++t) sum = __fadd_rn(sum, s[t]);
    bc[0] = __fdiv_rn(1.0f, sum);
  }
  __syncthreads();
  const float inv = bc[0];
  for (int t = threadIdx.x; t < seq_len; t += blockDim.x) s[t] = __fmul_rn(s[t], inv);
  __syncthreads();
  const int fma_dims = (hd / 8) * 8;
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float o = 0.0f;
    if (d < fma_dims) {
      for (int t = 0; t < seq_len; ++t) o = __fmaf_rn(s[t], vb[(size_t)t * hd + d], o);
    } else {
      for (int t = 0; t < seq_len; ++t) o = __fadd_rn(o, __fmul_rn(s[t], vb[(size_t)t * hd + d]));
    }
    out[(size_t)h * hd + d] = o;
  }
}

void launch_masked_attention_headmajor(const float* q, const float* kc, const float* vc, float* out, int nh, int nkv,
                                       int hd, int stride, int seq_len, float* scratch, cudaStream_t st) {
  masked_attention_headmajor_kernel<<<nh, 128, 0, st>>>(q, kc, vc, out, nh, nkv, hd, stride, seq_len, scratch);
  count_launch();
}

// ---------------------------------------------------------------------------
// Paged cache addressing: pool[layer][page][kv_head][kind][slot][hd].
// ---------------------------------------------------------------------------
__device__ __forceinline__ size_t kv_off(const KvGeom& g, int layer, int page, int kvh, int kind, int slot) {
  return ((((size_t)layer * g.pages + page) * g.kv_heads + kvh) * 2 + kind) * (size_t)(kPage * g.hd) +
         (size_t)slot * g.hd;
}
__device__ __forceinline__ float kv_load(const KvGeom& g, size_t off) {
  return g.bf16 ? bf16_bits_to_f32(((const uint16_t*)g.pool)[off]) : ((const float*)g.pool)[off];
}
__device__ __forceinline__ void kv_store(const KvGeom& g, size_t off, float v) {
  if (g.bf16)
    ((uint16_t*)g.pool)[off] = f32_to_bf16_bits(v);
  else
    ((float*)g.pool)[off] = v;
}

// ---------------------------------------------------------------------------
// RoPE (rope.rs:414-431, half-split) + KVCache::store_kv.
// ---------------------------------------------------------------------------
__global__ void rope_kv_store_kernel(const float* __restrict__ qkv, int ldqkv, int nh, int nkv, int hd,
                                     const float* __restrict__ rcos, const float* __restrict__ rsin,
                                     const int32_t* __restrict__ tok_pos, const int32_t* __restrict__ tok_seq,
                                     const int32_t* __restrict__ page_table, KvGeom g, int layer,
                                     float* __restrict__ q_out) {
  const int t = blockIdx.x;
  const int pos = tok_pos[t], seq = tok_seq[t];
  const int half = hd / 2;
  const float* row = qkv + (size_t)t * ldqkv;
  const float* c = rcos + (size_t)pos * half;
  const float* s = rsin + (size_t)pos * half;
  const int page = page_table[(size_t)seq * g.max_pages_per_seq + pos / kPage];
  const int slot = pos % kPage;
  const int nq = nh * half, nk = nkv * half;
  for (int i = threadIdx.x; i < nq + nk; i += blockDim.x) {
    int head = i < nq ? i / half : (i - nq) / half;
    int p = i < nq ? i % half : (i - nq) % half;
    const float* x = row + (i < nq ? 0 : nh * hd) + head * hd;
    float lo = x[p], hi = x[p + half];
    float cc = c[p], ss = s[p];
    float nlo = __fsub_rn(__fmul_rn(lo, cc), __fmul_rn(hi, ss));
    float nhi = __fadd_rn(__fmul_rn(hi, cc), __fmul_rn(lo, ss));
    if (i < nq) {
      q_out[(size_t)t * nh * hd + head * hd + p] = nlo;
      q_out[(size_t)t * nh * hd + head * hd + p + half] = nhi;
    } else {
      size_t off = kv_off(g, layer, page, head, 0, slot);
      kv_store(g, off + p, nlo);
      kv_store(g, off + p + half, nhi);
    }
  }
  const float* vrow = row + (nh + nkv) * hd;
  for (int i = threadIdx.x; i < nkv * hd; i += blockDim.x) {
    int head = i / hd, d = i % hd;
    kv_store(g, kv_off(g, layer, page, head, 1, slot) + d, vrow[i]);
  }
}

void launch_rope_kv_store(const float* qkv, int ldqkv, int T, int nh, int nkv, int hd, const float* rope_cos,
                          const float* rope_sin, const int32_t* tok_pos, const int32_t* tok_seq,
                          const int32_t* page_table, const KvGeom& kv, int layer, float* q_out, cudaStream_t st) {
  if (T <= 0) return;
  rope_kv_store_kernel<<<T, 256, 0, st>>>(qkv, ldqkv, nh, nkv, hd, rope_cos, rope_sin, tok_pos, tok_seq, page_table,
                                          kv, layer, q_out);
  count_launch();
}

__global__ void rope_apply_kernel(const float* __restrict__ qk, int heads, int hd, const float* __restrict__ c,
                                  const float* __restrict__ s, float* __restrict__ out) {
  const int half = hd / 2;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < heads * half; i += gridDim.x * blockDim.x) {
    int head = i / half, p = i % half;
    const float* x = qk + (size_t)head * hd;
    float lo = x[p], hi = x[p + half];
    out[(size_t)head * hd + p] = __fsub_rn(__fmul_rn(lo, c[p]), __fmul_rn(hi, s[p]));
    out[(size_t)head * hd + p + half] = __fadd_rn(__fmul_rn(hi, c[p]), __fmul_rn(lo, s[p]));
  }
}

void launch_rope_apply(const float* qk, int nh, int nkv, int hd, const float* cos_table, const float* sin_table,
                       size_t pos, float* out, cudaStream_t st) {
  int heads = nh + nkv, half = hd / 2;
  int n = heads * half;
  if (n <= 0) return;
  rope_apply_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(qk, heads, hd, cos_table + pos * half,
                                                                sin_table + pos * half, out);
  count_launch();
}

// ---------------------------------------------------------------------------
// Paged GQA attention, split over the context (flash-decoding).  One block per
// (query token, kv head, split); one warp per query head of the group; lane l
// owns dims l, l+32, ...  Online softmax in f32.
// ---------------------------------------------------------------------------
constexpr int kSplit = 512;  // context positions per split

template <int DPL>
__global__ void __launch_bounds__(256) paged_attention_kernel(const float* __restrict__ q, int nh,
                                                              const int32_t* __restrict__ tok_pos,
                                                              const int32_t* __restrict__ tok_seq,
                                                              const int32_t* __restrict__ page_table, KvGeom g,
                                                              int layer, int max_splits, float* __restrict__ out,
                                                              float* __restrict__ partial) {
  const int t = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int ctx = tok_pos[t] + 1;
  const int nsplit = (ctx + kSplit - 1) / kSplit;
  if (split >= nsplit) return;
  const int group = nh / g.kv_heads;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int hd = g.hd;
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  const int seq = tok_seq[t];
  const int32_t* pt = page_table + (size_t)seq * g.max_pages_per_seq;
  const int t0 = split * kSplit, t1 = min(ctx, t0 + kSplit);
  for (int hh = warp; hh < group; hh += nwarps) {
    const int h = kvh * group + hh;
    const float* qh = q + ((size_t)t * nh + h) * hd;
    float qv[DPL], o[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) {
      int d = lane + 32 * i;
      qv[i] = d < hd ? qh[d] : 0.0f;
      o[i] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;
    for (int p = t0; p < t1; ++p) {
      const int page = pt[p / kPage], slot = p % kPage;
      const size_t koff = kv_off(g, layer, page, kvh, 0, slot);
      const size_t voff = koff + (size_t)kPage * hd;
      float part = 0.0f;
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        int d = lane + 32 * i;
        if (d < hd) part = __fmaf_rn(qv[i], kv_load(g, koff + d), part);
      }
      float sc = __fmul_rn(warp_sum(part), scale);
      float mn = fmaxf(m, sc);
      float corr = expf(m - mn);
      float pw = expf(sc - mn);
      l = __fmaf_rn(l, corr, pw);
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        int d = lane + 32 * i;
        float vv = d < hd ? kv_load(g, voff + d) : 0.0f;
        o[i] = __fmaf_rn(o[i], corr, __fmul_rn(pw, vv));
      }
      m = mn;
    }
    if (nsplit == 1) {
      float inv = __fdiv_rn(1.0f, l);
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        int d = lane + 32 * i;
        if (d < hd) out[((size_t)t * nh + h) * hd + d] = __fmul_rn(o[i], inv);
      }
    } else {
      float* pp = partial + (((size_t)t * nh + h) * max_splits + split) * (hd + 2);
      if (lane == 0) {
        pp[0] = m;
        pp[1] = l;
      }
#pragma unroll
      for (int i = 0; i < DPL; ++i) {
        int d = lane + 32 * i;
        if (d < hd) pp[2 + d] = o[i];
      }
    }
  }
}

__global__ void attention_combine_kernel(const int32_t* __restrict__ tok_pos, int nh, int hd, int max_splits,
                                         const float* __restrict__ partial, float* __restrict__ out) {
  const int t = blockIdx.x, h = blockIdx.y;
  const int ctx = tok_pos[t] + 1;
  const int nsplit = (ctx + kSplit - 1) / kSplit;
  if (nsplit == 1) return;
  const float* pp = partial + ((size_t)t * nh + h) * max_splits * (hd + 2);
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, pp[s * (hd + 2)]);
  float L = 0.0f;
  for (int s = 0; s < nsplit; ++s) L = __fmaf_rn(pp[s * (hd + 2) + 1], expf(pp[s * (hd + 2)] - M), L);
  float invL = __fdiv_rn(1.0f, L);
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float acc = 0.0f;
    for (int s = 0; s < nsplit; ++s) acc = __fmaf_rn(pp[s * (hd + 2) + 2 + d], expf(pp[s * (hd + 2)] - M), acc);
    out[((size_t)t * nh + h) * hd + d] = __fmul_rn(acc, invL);
  }
}

size_t paged_attention_partial_floats(int T, int nh, int hd, int max_ctx) {
  int ms = (max_ctx + kSplit - 1) / kSplit;
  return (size_t)T * nh * ms * (hd + 2);
}

void launch_paged_attention(const float* q, int T, int nh, const int32_t* tok_pos, const int32_t* tok_seq,
                            const int32_t* page_table, const KvGeom& kv, int layer, int max_ctx, float* out,
                            float* partial, size_t partial_floats, cudaStream_t st) {
  if (T <= 0) return;
  int ms = (max_ctx + kSplit - 1) / kSplit;
  (void)partial_floats;
  int group = nh / kv.kv_heads;
  int threads = 32 * min(group, 8);
  dim3 grid(T, kv.kv_heads, ms);
  int dpl = (kv.hd + 31) / 32;
  if (dpl <= 1)
    paged_attention_kernel<1><<<grid, threads, 0, st>>>(q, nh, tok_pos, tok_seq, page_table, kv, layer, ms, out, partial);
  else if (dpl <= 2)
    paged_attention_kernel<2><<<grid, threads, 0, st>>>(q, nh, tok_pos, tok_seq, page_table, kv, layer, ms, out, partial);
  else if (dpl <= 4)
    paged_attention_kernel<4><<<grid, threads, 0, st>>>(q, nh, tok_pos, tok_seq, page_table, kv, layer, ms, out, partial);
  else
    paged_attention_kernel<8><<<grid, threads, 0, st>>>(q, nh, tok_pos, tok_seq, page_table, kv, layer, ms, out, partial);
  count_launch();
  if (ms > 1) {
    attention_combine_kernel<<<dim3(T, nh), 128, 0, st>>>(tok_pos, nh, kv.hd, ms, partial, out);
    count_launch();
  }
}

// ---------------------------------------------------------------------------
// KV seeding: counter-based N(0,1) (SplitMix64 -> Box-Muller in double).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}

__global__ void kv_fill_random_kernel(KvGeom g, const int32_t* __restrict__ page_row, int n, uint64_t seed,
                                      uint32_t seq) {
  // One block per (position, layer); threads over (kv_head, kind, element pair).
  // Same draws as synth_kv_normal: single-precision Box-Muller on one 64-bit
  // draw per element pair (cosine branch -> even element, sine -> odd).
  const int layer = blockIdx.y, pos = blockIdx.x;
  if (pos >= n) return;
  const int page = page_row[pos / kPage], slot = pos % kPage;
  const int half = g.hd / 2;
  const int per = g.kv_heads * 2 * half;
  for (int i = threadIdx.x; i < per; i += blockDim.x) {
    int kvh = i / (2 * half), kind = (i / half) % 2, j = i % half;
    uint64_t key = mix64(seed ^ mix64(((uint64_t)seq << 40) ^ ((uint64_t)layer << 24) ^ ((uint64_t)kind << 20) ^
                                       ((uint64_t)kvh << 16) ^ 0x5eedULL));
    uint64_t pair = ((uint64_t)pos * g.hd) / 2 + j;
    uint64_t a = mix64(key + pair * 0x9e3779b97f4a7c15ULL);
    float u1 = (float)((a >> 40) + 1) * (1.0f / 16777216.0f);
    float u2 = (float)(a & 0xffffffu) * (1.0f / 16777216.0f);
    float r = sqrtf(__fmul_rn(-2.0f, logf(u1)));
    float t = __fmul_rn(6.28318530717958647692f, u2);
    size_t off = kv_off(g, layer, page, kvh, kind, slot) + 2 * j;
    kv_store(g, off, __fmul_rn(r, cosf(t)));
    kv_store(g, off + 1, __fmul_rn(r, sinf(t)));
  }
}

void launch_kv_fill_random(const KvGeom& kv, const int32_t* page_row, int n, uint64_t seed, uint32_t seq,
                           cudaStream_t st) {
  if (n <= 0) return;
  kv_fill_random_kernel<<<dim3(n, kv.layers), 256, 0, st>>>(kv, page_row, n, seed, seq);
  count_launch();
}

__global__ void kv_copy_kernel(KvGeom g, const int32_t* __restrict__ page_row, int n, float* ks, float* vs,
                               int to_cache) {
  const int layer = blockIdx.y, pos = blockIdx.x;
  const int page = page_row[pos / kPage], slot = pos % kPage;
  const int row = g.kv_heads * g.hd;
  for (int i = threadIdx.x; i < row; i += blockDim.x) {
    int kvh = i / g.hd, d = i % g.hd;
    size_t so = ((size_t)layer * n + pos) * row + i;
    size_t ko = kv_off(g, layer, page, kvh, 0, slot) + d, vo = kv_off(g, layer, page, kvh, 1, slot) + d;
    if (to_cache) {
      kv_store(g, ko, ks[so]);
      kv_store(g, vo, vs[so]);
    } else {
      ks[so] = kv_load(g, ko);
      vs[so] = kv_load(g, vo);
    }
  }
}

void launch_kv_copy(const KvGeom& kv, const int32_t* page_row, int n, float* k_stage, float* v_stage, bool to_cache,
                    cudaStream_t st) {
  if (n <= 0) return;
  kv_copy_kernel<<<dim3(n, kv.layers), 128, 0, st>>>(kv, page_row, n, k_stage, v_stage, to_cache ? 1 : 0);
  count_launch();
}

}  // namespace bitnet
