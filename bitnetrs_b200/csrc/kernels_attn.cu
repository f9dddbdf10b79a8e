// kernels_attn.cu — RoPE + paged KV store and GQA attention.
#include "kernels.cuh"

#include <algorithm>

namespace bitnet {


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
                                                  int nkv, int hd, int stride, int seq_len, float* scratch,
                                                  ExpTable et) {
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
  for (int t = threadIdx.x; t < seq_len; t += blockDim.x) s[t] = exp_host_libm(__fsub_rn(s[t], m), et);
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
                                       int hd, int stride, int seq_len, float* scratch, const ExpTable& et,
                                       cudaStream_t st) {
  masked_attention_headmajor_kernel<<<nh, 128, 0, st>>>(q, kc, vc, out, nh, nkv, hd, stride, seq_len, scratch, et);
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
  pdl_launch_dependents();
  pdl_wait();
  qkv = after_wait(qkv);
  tok_pos = after_wait(tok_pos);
  tok_seq = after_wait(tok_seq);
  page_table = after_wait(page_table);
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
// Paged attention in the reference's operation order (attention.rs:165-206):
// one block per (query token, kv head) serves the G query heads of the group.
//   1. score[g][t] = dot_f32_f32(q_g, K[t]) * scale    (8 FMA chains + hsum + tail)
//   2. m_g = max_t score;  e = exp(score - m_g)
//   3. sum_g = ((e_0 + e_1) + e_2) + ...               (one thread per head)
//   4. p = e * (1 / sum_g)
//   5. out[g][d] = fma chain over t of p[g][t] * V[t][d] (mul+add for dims past hd/8*8)
// Every step but exp reproduces the reference bit for bit; exp is evaluated
// in double and rounded, i.e. correctly rounded, which glibc's expf matches
// except when the exact value lies within ~1e-3 ulp of a rounding boundary.
// Scores live in shared memory (G * ctx floats) or, for long contexts, in
// the global `scratch` ([T][nh][max_ctx] floats).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(512) paged_attention_exact_kernel(
    const float* __restrict__ q, int nh, const int32_t* __restrict__ tok_pos, const int32_t* __restrict__ tok_seq,
    const int32_t* __restrict__ page_table, KvGeom g, int layer, int max_ctx, int scores_in_smem,
    float* __restrict__ scratch, float* __restrict__ out, ExpTable et) {
  extern __shared__ float sm[];
  __shared__ float red[32][8];
  __shared__ float head_max[8], head_inv[8];
  const int t = blockIdx.x, kvh = blockIdx.y;
  const int ctx = tok_pos[t] + 1;
  const int G = nh / g.kv_heads, hd = g.hd;
  const int32_t* pt = page_table + (size_t)tok_seq[t] * g.max_pages_per_seq;
  float* qs = sm;  // [G][hd]
  float* sc = scores_in_smem ? sm + G * hd : scratch + ((size_t)t * nh + (size_t)kvh * G) * max_ctx;
  for (int i = threadIdx.x; i < G * hd; i += blockDim.x)
    qs[i] = q[((size_t)t * nh + (size_t)kvh * G) * hd + i];
  __syncthreads();
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)hd));
  const int chunks = hd >> 3;
  // 1. scores, thread per (head, position)
  for (int i = threadIdx.x; i < G * ctx; i += blockDim.x) {
    const int gg = i % G, p = i / G;
    const size_t koff = kv_off(g, layer, pt[p / kPage], kvh, 0, p % kPage);
    const float* qv = qs + gg * hd;
    float a[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] = 0.0f;
    if ((hd & 7) != 0) {
      for (int c = 0; c < chunks; ++c)
#pragma unroll
        for (int j = 0; j < 8; ++j) a[j] = __fmaf_rn(qv[8 * c + j], kv_load(g, koff + 8 * c + j), a[j]);
    } else if (g.bf16) {
      const uint16_t* kr = (const uint16_t*)g.pool + koff;
      for (int c = 0; c < chunks; ++c) {
        uint4 w = *reinterpret_cast<const uint4*>(kr + 8 * c);
        const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          a[2 * j] = __fmaf_rn(qv[8 * c + 2 * j], __uint_as_float(wv[j] << 16), a[2 * j]);
          a[2 * j + 1] = __fmaf_rn(qv[8 * c + 2 * j + 1], __uint_as_float(wv[j] & 0xffff0000u), a[2 * j + 1]);
        }
      }
    } else {
      const float* kr = (const float*)g.pool + koff;
      for (int c = 0; c < chunks; ++c) {
        float4 k0 = *reinterpret_cast<const float4*>(kr + 8 * c);
        float4 k1 = *reinterpret_cast<const float4*>(kr + 8 * c + 4);
        a[0] = __fmaf_rn(qv[8 * c + 0], k0.x, a[0]);
        a[1] = __fmaf_rn(qv[8 * c + 1], k0.y, a[1]);
        a[2] = __fmaf_rn(qv[8 * c + 2], k0.z, a[2]);
        a[3] = __fmaf_rn(qv[8 * c + 3], k0.w, a[3]);
        a[4] = __fmaf_rn(qv[8 * c + 4], k1.x, a[4]);
        a[5] = __fmaf_rn(qv[8 * c + 5], k1.y, a[5]);
        a[6] = __fmaf_rn(qv[8 * c + 6], k1.z, a[6]);
        a[7] = __fmaf_rn(qv[8 * c + 7], k1.w, a[7]);
      }
    }
    float r = hsum8(a);
    for (int d = chunks * 8; d < hd; ++d) r = __fadd_rn(r, __fmul_rn(qv[d], kv_load(g, koff + d)));
    sc[gg * ctx + p] = __fmul_rn(r, scale);
  }
  __syncthreads();
  // 2. per-head max (order-free), then exp
  {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int gg = 0; gg < G; ++gg) {
      float m = -INFINITY;
      for (int p = threadIdx.x; p < ctx; p += blockDim.x) m = fmaxf(m, sc[gg * ctx + p]);
      m = warp_max(m);
      if (lane == 0) red[warp][gg & 7] = m;
      __syncthreads();
      if (threadIdx.x == 0) {
        float mm = red[0][gg & 7];
        for (int w = 1; w < nw; ++w) mm = fmaxf(mm, red[w][gg & 7]);
        head_max[gg & 7] = mm;
      }
      __syncthreads();
      const float hm = head_max[gg & 7];
      for (int p = threadIdx.x; p < ctx; p += blockDim.x)
        sc[gg * ctx + p] = exp_host_libm(__fsub_rn(sc[gg * ctx + p], hm), et);
      __syncthreads();
    }
  }
  // 3. sequential sum, one thread per head
  for (int gg = threadIdx.x; gg < G; gg += blockDim.x) {
    float s = 0.0f;
    const float* e = sc + gg * ctx;
    for (int p = 0; p < ctx; ++p) s = __fadd_rn(s, e[p]);
    head_inv[gg & 7] = __fdiv_rn(1.0f, s);
  }
  __syncthreads();
  // 4. normalise
  for (int i = threadIdx.x; i < G * ctx; i += blockDim.x) sc[i] = __fmul_rn(sc[i], head_inv[(i / ctx) & 7]);
  __syncthreads();
  // 5. output, thread per (head, dim), FMA chain over positions
  const int fma_dims = chunks * 8;
  for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
    const int gg = i / hd, d = i % hd;
    const float* pr = sc + gg * ctx;
    float o = 0.0f;
    int p = 0;
    if (d < fma_dims) {
      for (; p + 4 <= ctx; p += 4) {
        float v0 = kv_load(g, kv_off(g, layer, pt[(p + 0) / kPage], kvh, 1, (p + 0) % kPage) + d);
        float v1 = kv_load(g, kv_off(g, layer, pt[(p + 1) / kPage], kvh, 1, (p + 1) % kPage) + d);
        float v2 = kv_load(g, kv_off(g, layer, pt[(p + 2) / kPage], kvh, 1, (p + 2) % kPage) + d);
        float v3 = kv_load(g, kv_off(g, layer, pt[(p + 3) / kPage], kvh, 1, (p + 3) % kPage) + d);
        o = __fmaf_rn(pr[p + 0], v0, o);
        o = __fmaf_rn(pr[p + 1], v1, o);
        o = __fmaf_rn(pr[p + 2], v2, o);
        o = __fmaf_rn(pr[p + 3], v3, o);
      }
      for (; p < ctx; ++p) o = __fmaf_rn(pr[p], kv_load(g, kv_off(g, layer, pt[p / kPage], kvh, 1, p % kPage) + d), o);
    } else {
      for (; p < ctx; ++p)
        o = __fadd_rn(o, __fmul_rn(pr[p], kv_load(g, kv_off(g, layer, pt[p / kPage], kvh, 1, p % kPage) + d)));
    }
    out[((size_t)t * nh + (size_t)kvh * G + gg) * hd + d] = o;
  }
}

// ---------------------------------------------------------------------------
// The same reference-order attention, specialised for a bf16 cache with
// head_dim 128 and GQA group 4 (the 2B and scaled shapes), organised for
// throughput: one 256-thread block per (query token, kv head).
//   phase 1: K blocks of 4 pages (64 positions) stream through a 2-stage
//            ring with cp.async (16-byte chunk c of row r at c ^ (r & 15));
//            thread (head g, position p) forms one score with the eight FMA
//            chains of dot_f32_f32 and hsum8.
//   phase 2: per-head max, exp (correctly rounded), sequential sum by one
//            thread per head, p = e * (1/sum) — all in shared memory.
//   phase 3: V blocks stream the same way; thread (head g, dims 2j, 2j+1)
//            runs the two FMA chains over positions in order.
// Every step matches the reference operation for operation.
// ---------------------------------------------------------------------------
constexpr int kX2Pages = 4;                      // pages per round
constexpr int kX2Ring = 2 * kX2Pages * 4096;     // two rounds of K or V blocks (bytes)

__global__ void __launch_bounds__(256) paged_attention_exact2_kernel(
    const float* __restrict__ q, int nh, const int32_t* __restrict__ tok_pos, const int32_t* __restrict__ tok_seq,
    const int32_t* __restrict__ page_table, KvGeom g, int layer, int cap, float* __restrict__ out, ExpTable et) {
  extern __shared__ __align__(128) uint8_t smem[];
  float* qs = reinterpret_cast<float*>(smem);                  // [4][128]
  uint8_t* ring = smem + 4 * 128 * 4;                          // kX2Ring bytes
  float* sc = reinterpret_cast<float*>(ring + kX2Ring);        // [4][cap]
  __shared__ float red[8][4];
  __shared__ float hmax[4], hinv[4];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int t = blockIdx.x, kvh = blockIdx.y;
  const int ctx = tok_pos[t] + 1;
  const int32_t* pt = page_table + (size_t)tok_seq[t] * g.max_pages_per_seq;
  const size_t page_stride = (size_t)g.kv_heads * 2 * kPage * 128;
  const uint16_t* kvbase =
      (const uint16_t*)g.pool + (size_t)layer * g.pages * page_stride + (size_t)kvh * 2 * kPage * 128;
  for (int i = tid; i < 4 * 128; i += 256) qs[i] = q[((size_t)t * nh + (size_t)kvh * 4) * 128 + i];
  const int npages = (ctx + kPage - 1) / kPage;
  const int rounds = (npages + kX2Pages - 1) / kX2Pages;

  // Stage round r of the K (kind 0) or V (kind 1) blocks into ring half r & 1.
  auto stage = [&](int r, int kind) {
    if (r < rounds) {
      uint8_t* dst = ring + (r & 1) * (kX2Pages * 4096);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        int c = tid + 256 * k;  // 1024 chunks: [page][row][16]
        int pg = c >> 8, row = (c >> 4) & 15, ch = c & 15;
        int page_idx = r * kX2Pages + pg;
        int pos = page_idx * kPage + row;
        const uint16_t* src = kvbase + (page_idx < npages ? (size_t)pt[page_idx] * page_stride : 0) +
                              (size_t)kind * kPage * 128 + row * 128 + ch * 8;
        uint32_t sd = (uint32_t)__cvta_generic_to_shared(dst + pg * 4096 + row * 256 + ((ch ^ row) << 4));
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(sd), "l"(src),
                     "r"(pos < ctx ? 16 : 0));
      }
    }
    asm volatile("cp.async.commit_group;\n" ::);
  };

  // ---- phase 1: scores ----
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(128.0f));
  const int g1 = tid >> 6, p1 = tid & 63;  // head, position within the round
  stage(0, 0);
  for (int r = 0; r < rounds; ++r) {
    stage(r + 1, 0);
    asm volatile("cp.async.wait_group 1;\n" ::);
    __syncthreads();
    const int pos = r * 64 + p1;
    if (pos < ctx) {
      const uint8_t* kr = ring + (r & 1) * (kX2Pages * 4096) + (p1 >> 4) * 4096 + (p1 & 15) * 256;
      const float* qv = qs + g1 * 128;
      float a[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] = 0.0f;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        uint4 w = *reinterpret_cast<const uint4*>(kr + ((c ^ (p1 & 15)) << 4));
        float4 q0 = *reinterpret_cast<const float4*>(qv + 8 * c);
        float4 q1 = *reinterpret_cast<const float4*>(qv + 8 * c + 4);
        a[0] = __fmaf_rn(q0.x, __uint_as_float(w.x << 16), a[0]);
        a[1] = __fmaf_rn(q0.y, __uint_as_float(w.x & 0xffff0000u), a[1]);
        a[2] = __fmaf_rn(q0.z, __uint_as_float(w.y << 16), a[2]);
        a[3] = __fmaf_rn(q0.w, __uint_as_float(w.y & 0xffff0000u), a[3]);
        a[4] = __fmaf_rn(q1.x, __uint_as_float(w.z << 16), a[4]);
        a[5] = __fmaf_rn(q1.y, __uint_as_float(w.z & 0xffff0000u), a[5]);
        a[6] = __fmaf_rn(q1.z, __uint_as_float(w.w << 16), a[6]);
        a[7] = __fmaf_rn(q1.w, __uint_as_float(w.w & 0xffff0000u), a[7]);
      }
      sc[g1 * cap + pos] = __fmul_rn(hsum8(a), scale);
    }
    __syncthreads();
  }
  // prefetch the first V round while the softmax runs
  stage(0, 1);
  // ---- phase 2: softmax ----
  {
    float mx = -INFINITY;
    for (int p = p1; p < ctx; p += 64) mx = fmaxf(mx, sc[g1 * cap + p]);
    mx = warp_max(mx);
    if (lane == 0) red[warp][0] = mx;
    __syncthreads();
    if (tid < 4) hmax[tid] = fmaxf(red[2 * tid][0], red[2 * tid + 1][0]);
    __syncthreads();
    const float hm = hmax[g1];
    for (int p = p1; p < ctx; p += 64) sc[g1 * cap + p] = exp_host_libm(__fsub_rn(sc[g1 * cap + p], hm), et);
    __syncthreads();
    if (tid < 4) {
      const float* e = sc + tid * cap;
      float sum = 0.0f;
      int p = 0;
      for (; p + 8 <= ctx; p += 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = e[p + u];
#pragma unroll
        for (int u = 0; u < 8; ++u) sum = __fadd_rn(sum, v[u]);
      }
      for (; p < ctx; ++p) sum = __fadd_rn(sum, e[p]);
      hinv[tid] = __fdiv_rn(1.0f, sum);
    }
    __syncthreads();
    const float hi = hinv[g1];
    for (int p = p1; p < ctx; p += 64) sc[g1 * cap + p] = __fmul_rn(sc[g1 * cap + p], hi);
  }
  // ---- phase 3: out[g][d] = fma chain over positions ----
  const int g3 = tid >> 6, j3 = tid & 63;  // head, dim pair
  const float* pr = sc + g3 * cap;
  float o0 = 0.0f, o1 = 0.0f;
  for (int r = 0; r < rounds; ++r) {
    stage(r + 1, 1);
    asm volatile("cp.async.wait_group 1;\n" ::);
    __syncthreads();
    const uint8_t* vb = ring + (r & 1) * (kX2Pages * 4096);
    const int ch = j3 >> 2, within = (j3 & 3) * 4;  // 16-byte chunk holding dims 2*j3, 2*j3+1
    const int pend = min(64, ctx - r * 64);
#pragma unroll 4
    for (int pp = 0; pp < pend; ++pp) {
      uint32_t w = *reinterpret_cast<const uint32_t*>(vb + (pp >> 4) * 4096 + (pp & 15) * 256 +
                                                      ((ch ^ (pp & 15)) << 4) + within);
      const float p = pr[r * 64 + pp];
      o0 = __fmaf_rn(p, __uint_as_float(w << 16), o0);
      o1 = __fmaf_rn(p, __uint_as_float(w & 0xffff0000u), o1);
    }
    __syncthreads();
  }
  asm volatile("cp.async.wait_group 0;\n" ::);
  *reinterpret_cast<float2*>(out + ((size_t)t * nh + (size_t)kvh * 4 + g3) * 128 + 2 * j3) = make_float2(o0, o1);
}

bool exact2_supported(const KvGeom& kv, int nh) { return kv.bf16 && kv.hd == 128 && nh == 4 * kv.kv_heads; }

size_t exact2_smem(int max_ctx) {
  int cap = (max_ctx + 63) / 64 * 64;
  return 4 * 128 * 4 + kX2Ring + (size_t)4 * cap * 4;
}

int exact2_prepare(size_t smem) {
  return cudaFuncSetAttribute(paged_attention_exact2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ==
                 cudaSuccess
             ? 0
             : 1;
}

void launch_paged_attention_exact2(const float* q, int T, int nh, const int32_t* tok_pos, const int32_t* tok_seq,
                                   const int32_t* page_table, const KvGeom& kv, int layer, int max_ctx, float* out,
                                   const ExpTable& et, cudaStream_t st) {
  if (T <= 0) return;
  const int cap = (max_ctx + 63) / 64 * 64;
  paged_attention_exact2_kernel<<<dim3(T, kv.kv_heads), 256, exact2_smem(max_ctx), st>>>(
      q, nh, tok_pos, tok_seq, page_table, kv, layer, cap, out, et);
  count_launch();
}

size_t paged_attention_exact_smem(int nh, int kv_heads, int hd, int max_ctx) {
  int G = nh / kv_heads;
  return (size_t)G * hd * 4 + (size_t)G * max_ctx * 4;
}

int paged_attention_exact_prepare(size_t smem) {
  if (smem > 48 * 1024)
    if (cudaFuncSetAttribute(paged_attention_exact_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return 1;
  return 0;
}

void launch_paged_attention_exact(const float* q, int T, int nh, const int32_t* tok_pos, const int32_t* tok_seq,
                                  const int32_t* page_table, const KvGeom& kv, int layer, int max_ctx, float* out,
                                  float* scratch, bool scores_in_smem, const ExpTable& et, cudaStream_t st) {
  if (T <= 0) return;
  const int G = nh / kv.kv_heads;
  int threads = std::min(512, std::max(64, ((G * kv.hd + 31) / 32) * 32));
  size_t smem = scores_in_smem ? paged_attention_exact_smem(nh, kv.kv_heads, kv.hd, max_ctx)
                               : (size_t)G * kv.hd * 4;
  paged_attention_exact_kernel<<<dim3(T, kv.kv_heads), threads, smem, st>>>(
      q, nh, tok_pos, tok_seq, page_table, kv, layer, max_ctx, scores_in_smem ? 1 : 0, scratch, out, et);
  count_launch();
}

// ---------------------------------------------------------------------------
// Tensor-core decode attention for a bf16 cache (head_dim 128, GQA group <= 4).
// One warp per (query token, kv head, split of kMmaSplit positions); four
// warps per block take consecutive splits.  Pages (16 positions: K block then
// V block, 8 KB contiguous per kv head) stream through a per-warp ring in
// shared memory with cp.async; 16-byte chunk c of row r is stored at chunk
// c ^ (r & 7) so ldmatrix rows never share banks.
//   S = Q K^T : mma m16n8k16, A rows 0-3 = bf16(q) of the group's heads,
//               rows 4-7 = bf16(q - bf16(q)); the two halves are summed in f32.
//   O = P V   : A rows 0-3 = bf16(p), rows 4-7 = bf16(p - bf16(p)).
// K and V are exact in bf16 and products accumulate in f32, so the result
// matches f32 attention to ~1e-5 relative.  Online softmax, f32 state.
// ---------------------------------------------------------------------------
constexpr int kMmaSplit = 256;
constexpr int kMmaStages = 3;
constexpr int kMmaWarps = 4;

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
}
__device__ __forceinline__ float bf16r(float x) { return bf16_bits_to_f32(f32_to_bf16_bits(x)); }

__device__ __forceinline__ void mma_bf16(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t r[4], const void* p) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t r[4], const void* p) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s));
}
__device__ __forceinline__ void cp_async16_zfill(void* smem_dst, const void* gsrc, int bytes) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(smem_dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gsrc), "r"(bytes));
}

__global__ void __launch_bounds__(kMmaWarps * 32) flash_decode_mma_kernel(
    const float* __restrict__ q, int nh, const int32_t* __restrict__ tok_pos, const int32_t* __restrict__ tok_seq,
    const int32_t* __restrict__ page_table, KvGeom g, int layer, int max_splits, float* __restrict__ out,
    float* __restrict__ partial) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t = blockIdx.x, kvh = blockIdx.y;
  const int split = blockIdx.z * kMmaWarps + warp;
  const int ctx = tok_pos[t] + 1;
  const int nsplit = (ctx + kMmaSplit - 1) / kMmaSplit;
  if (split >= nsplit) return;
  const int G = nh / g.kv_heads;  // <= 4
  const int gq = lane >> 2, tq = lane & 3;
  const int32_t* pt = page_table + (size_t)tok_seq[t] * g.max_pages_per_seq;
  uint8_t* ring = smem + (size_t)warp * kMmaStages * 8192;
  const int p0 = split * kMmaSplit, p1 = min(ctx, p0 + kMmaSplit);
  const int npages = (p1 - p0 + kPage - 1) / kPage;
  const size_t page_stride = (size_t)g.kv_heads * 2 * kPage * 128;  // bf16 elements per (layer, page)
  const uint16_t* kvbase = (const uint16_t*)g.pool + (size_t)layer * g.pages * page_stride + (size_t)kvh * 2 * kPage * 128;

  auto load_page = [&](int i) {
    if (i < npages) {
      const int pos0 = p0 + i * kPage;
      const uint16_t* src = kvbase + (size_t)pt[pos0 / kPage] * page_stride;
      uint8_t* dst = ring + (i % kMmaStages) * 8192;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        int c = lane + 32 * k;  // 512 chunks: [kind][row][16 chunks]
        int kind = c >> 8, row = (c >> 4) & 15, ch = c & 15;
        int bytes = (pos0 + row < ctx) ? 16 : 0;  // rows past the context are zero-filled
        cp_async16_zfill(dst + kind * 4096 + row * 256 + ((ch ^ (row & 7)) << 4), src + (size_t)c * 8, bytes);
      }
    }
    asm volatile("cp.async.commit_group;\n" ::);
  };

  // Q fragments (A operand): row r<4 -> bf16 hi of head r, 4<=r<8 -> lo of head r-4, rows 8-15 zero.
  uint32_t qa[8][2];
  {
    const int hh = gq & 3;
    const bool valid = hh < G;
    const float* qh = q + ((size_t)t * nh + (size_t)kvh * G + (valid ? hh : 0)) * 128;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        int d = 16 * ks + 8 * half + 2 * tq;
        float x0 = valid ? qh[d] : 0.0f, x1 = valid ? qh[d + 1] : 0.0f;
        if (gq >= 4) {
          x0 = x0 - bf16r(x0);
          x1 = x1 - bf16r(x1);
        }
        qa[ks][half] = pack_bf16x2(x0, x1);
      }
    }
  }
  const float scale_log2 = __fdiv_rn(1.0f, __fsqrt_rn(128.0f)) * 1.4426950408889634f;
  float m = -INFINITY, l = 0.0f;  // per head (row gq & 3), natural-log units scaled by log2(e)
  float o[16][2];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = 0.0f;

#pragma unroll
  for (int i = 0; i < kMmaStages - 1; ++i) load_page(i);
  for (int i = 0; i < npages; ++i) {
    load_page(i + kMmaStages - 1);
    asm volatile("cp.async.wait_group %0;\n" ::"n"(kMmaStages - 1));
    __syncwarp();
    const uint8_t* kb = ring + (i % kMmaStages) * 8192;
    const uint8_t* vb = kb + 4096;
    // ---- scores for 16 positions ----
    float sc[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.0f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t b[4];
      const int mat = lane >> 3;
      const int row = 8 * (mat >> 1) + (lane & 7);
      const int ch = 2 * ks + (mat & 1);
      ldsm_x4(b, kb + row * 256 + ((ch ^ (row & 7)) << 4));
      const uint32_t a[4] = {qa[ks][0], 0u, qa[ks][1], 0u};
      mma_bf16(sc[0], a, b[0], b[1]);
      mma_bf16(sc[1], a, b[2], b[3]);
    }
    // combine hi + lo rows (lanes l and l^16), scale, mask
    float s4[4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float v = sc[nt][e] + __shfl_xor_sync(0xffffffffu, sc[nt][e], 16);
        int pos = p0 + i * kPage + 8 * nt + 2 * tq + e;
        s4[2 * nt + e] = pos < ctx ? v * scale_log2 : -INFINITY;
      }
    float mx = fmaxf(fmaxf(s4[0], s4[1]), fmaxf(s4[2], s4[3]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mn = fmaxf(m, mx);
    const float corr = exp2f(m - mn);
    float pr[4], rs = 0.0f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      pr[e] = exp2f(s4[e] - mn);
      rs += pr[e];
    }
    rs += __shfl_xor_sync(0xffffffffu, rs, 1);
    rs += __shfl_xor_sync(0xffffffffu, rs, 2);
    l = l * corr + rs;
    m = mn;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= corr;
      o[j][1] *= corr;
    }
    // P as the A operand: lanes 0-15 hi parts, lanes 16-31 lo parts.
    float pv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) pv[e] = gq >= 4 ? pr[e] - bf16r(pr[e]) : pr[e];
    const uint32_t pa[4] = {pack_bf16x2(pv[0], pv[1]), 0u, pack_bf16x2(pv[2], pv[3]), 0u};
    // ---- O += P V over 128 dims ----
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      uint32_t b[4];
      const int mat = lane >> 3;
      const int row = 8 * (mat & 1) + (lane & 7);
      const int ch = j + (mat >> 1);
      ldsm_x4_t(b, vb + row * 256 + ((ch ^ (row & 7)) << 4));
      float c0[4] = {o[j][0], o[j][1], 0.0f, 0.0f};
      float c1[4] = {o[j + 1][0], o[j + 1][1], 0.0f, 0.0f};
      mma_bf16(c0, pa, b[0], b[1]);
      mma_bf16(c1, pa, b[2], b[3]);
      o[j][0] = c0[0];
      o[j][1] = c0[1];
      o[j + 1][0] = c1[0];
      o[j + 1][1] = c1[1];
    }
    __syncwarp();
  }
  asm volatile("cp.async.wait_group 0;\n" ::);
  // hi + lo halves of O
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    o[j][0] += __shfl_xor_sync(0xffffffffu, o[j][0], 16);
    o[j][1] += __shfl_xor_sync(0xffffffffu, o[j][1], 16);
  }
  const int hh = gq;
  if (lane < 16 && hh < G) {
    const int h = kvh * G + hh;
    if (nsplit == 1) {
      const float inv = 1.0f / l;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float2 v = make_float2(o[j][0] * inv, o[j][1] * inv);
        *reinterpret_cast<float2*>(out + ((size_t)t * nh + h) * 128 + 8 * j + 2 * tq) = v;
      }
    } else {
      float* pp = partial + (((size_t)t * nh + h) * max_splits + split) * (128 + 2);
      if (tq == 0) {
        pp[0] = m * 0.6931471805599453f;  // back to natural-log units for the combine
        pp[1] = l;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        pp[2 + 8 * j + 2 * tq] = o[j][0];
        pp[2 + 8 * j + 2 * tq + 1] = o[j][1];
      }
    }
  }
}

__global__ void mma_combine_kernel(const int32_t* __restrict__ tok_pos, int nh, int max_splits,
                                   const float* __restrict__ partial, float* __restrict__ out) {
  const int t = blockIdx.x, h = blockIdx.y;
  const int ctx = tok_pos[t] + 1;
  const int nsplit = (ctx + kMmaSplit - 1) / kMmaSplit;
  if (nsplit == 1) return;
  const float* pp = partial + ((size_t)t * nh + h) * max_splits * 130;
  float M = -INFINITY;
  for (int s = 0; s < nsplit; ++s) M = fmaxf(M, pp[s * 130]);
  float L = 0.0f;
  for (int s = 0; s < nsplit; ++s) L += pp[s * 130 + 1] * expf(pp[s * 130] - M);
  const float invL = 1.0f / L;
  for (int d = threadIdx.x; d < 128; d += blockDim.x) {
    float acc = 0.0f;
    for (int s = 0; s < nsplit; ++s) acc += pp[s * 130 + 2 + d] * expf(pp[s * 130] - M);
    out[((size_t)t * nh + h) * 128 + d] = acc * invL;
  }
}

bool flash_decode_mma_supported(const KvGeom& kv, int nh) {
  return kv.bf16 && kv.hd == 128 && nh % kv.kv_heads == 0 && nh / kv.kv_heads <= 4;
}

size_t flash_decode_mma_partial_floats(int T, int nh, int max_ctx) {
  int ms = (max_ctx + kMmaSplit - 1) / kMmaSplit;
  return (size_t)T * nh * ms * 130;
}

int flash_decode_mma_prepare() {
  int smem = kMmaWarps * kMmaStages * 8192;
  return cudaFuncSetAttribute(flash_decode_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) ==
                 cudaSuccess
             ? 0
             : 1;
}

void launch_flash_decode_mma(const float* q, int T, int nh, const int32_t* tok_pos, const int32_t* tok_seq,
                             const int32_t* page_table, const KvGeom& kv, int layer, int max_ctx, float* out,
                             float* partial, cudaStream_t st) {
  if (T <= 0) return;
  const int ms = (max_ctx + kMmaSplit - 1) / kMmaSplit;
  dim3 grid(T, kv.kv_heads, (ms + kMmaWarps - 1) / kMmaWarps);
  flash_decode_mma_kernel<<<grid, kMmaWarps * 32, kMmaWarps * kMmaStages * 8192, st>>>(
      q, nh, tok_pos, tok_seq, page_table, kv, layer, ms, out, partial);
  count_launch();
  if (ms > 1) {
    mma_combine_kernel<<<dim3(T, nh), 128, 0, st>>>(tok_pos, nh, ms, partial, out);
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
