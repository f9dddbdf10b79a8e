// kernels_attn_x4.cu — reference-order paged decode attention for a bf16 cache
// with head_dim 128 and GQA group 4, as two streaming kernels per layer.
//
// Each (query token, kv head) serves the four query heads of the group and
// computes, bit for bit, what the reference's masked_attention does for each
// head (attention.rs:165-206):
//   score[g][t] = dot_f32_f32(q_g, K[t]) * (1/sqrt(128))   8 FMA chains over
//                 16 chunks of 8 dims, then hsum_f32_avx2 (simd.rs:292-307)
//   softmax_f32 (ops.rs:206-227): m = max_t score, e = exp(score - m),
//                sum = ((e_0 + e_1) + e_2) + ...,  p = e * (1/sum)
//   out[g][d]  = fma(p_t, V[t][d], out[g][d]) for t = 0, 1, ...   (axpy_f32)
//
// The QK dot products of different positions are independent, while each
// output dimension of PV is one FMA chain over all positions; a single CTA
// that does both phases leaves most of its warps idle in turn.  So:
//
// attn_qk_softmax_kernel (one CTA per (token, kv head), 4 compute warps + a
//   loader warp, three CTAs per SM): K pages stream through a 16-slot ring of
//   4 KiB TMA tiles (one page of one kv head, 128-byte swizzle) that holds two
//   rounds of every warp's pages, so a warp's next pages land while it
//   computes.  Every lane owns one position and runs all 32 chains (8 per
//   head) of it, so one broadcast load of q serves 32 positions and each K
//   element is converted once for four FMAs.  Raw scores go to a global
//   scratch row [cap][4].  The same CTA then finishes the softmax: max from
//   the lanes' running maxima,
//   e = exp(x - m) into shared memory (the ring, reused), the four serial sums
//   (one thread per head, reference order), and p = e * (1/sum) written back
//   over the scores.
//
// attn_pv_kernel (one CTA per (token, kv head), 2 PV warps + a loader warp,
//   many CTAs per SM): each page brings its V tile (TMA) and the page's 16 p
//   rows (a 256-byte bulk copy) into one ring slot; lane l of PV warp w owns
//   dims 64w + 2l and 64w + 2l + 1 of all four heads (8 chains), reading one
//   32-bit word of V and one broadcast float4 of p per position.
//
// Both kernels visit tokens in the order `order` gives (longest context first,
// so the last CTAs to start are the shortest).  TMA loads carry an L2
// evict-first policy: K and V are read once, the score rows are read again.
// Every mbarrier wait is bounded; a CTA that gives up records
// kStatusWaitTimeout, lets its issued copies land (bounded) and returns.
#include "async.cuh"

namespace bitnet {

namespace {

constexpr int kSlotBytes = 4096;                         // one page of one kv head: [16 rows][2 halves][64] bf16
constexpr int kQkWarps = 4;                              // compute warps of the QK kernel
constexpr int kQkThreads = (kQkWarps + 1) * 32;          // + the loader warp
constexpr int kQkSlots = 16;                             // ring pages: two rounds of the four warps
constexpr int kQkRoundPages = 2 * kQkWarps;              // pages per round: two per warp (one row per lane)
constexpr int kEChunk = kQkSlots * kSlotBytes / 16;      // exp values (float4 per position) the ring holds
constexpr int kMaxCand = 256;                            // queued host-libm table lookups per chunk (~100 expected)
constexpr int kPvWarps = 2;                              // PV warps
constexpr int kPvThreads = (kPvWarps + 1) * 32;          // + the loader warp
constexpr int kPvSlots = 8;                              // ring pages
constexpr int kPvSlotBytes = kSlotBytes + kPage * 16;    // V tile + the page's p rows

}  // namespace

// One CTA per (token order[blockIdx.x / kv_heads], kv head blockIdx.x % kv_heads): the scores of the
// group's four heads over the token's context, then its softmax; p[t][pos]
// (float4 over the four heads) is left in sp[(t * kv_heads + kvh) * cap + pos].
__global__ void __launch_bounds__(kQkThreads, 3) attn_qk_softmax_kernel(
    const float* __restrict__ q, int nh, const int32_t* __restrict__ tok_pos, const int32_t* __restrict__ tok_seq,
    const int32_t* __restrict__ order, const int32_t* __restrict__ page_table, KvGeom g, int layer, int cap,
    float4* __restrict__ sp, ExpTable et, int32_t* __restrict__ status, const __grid_constant__ CUtensorMap tmap) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kQkSlots];
  __shared__ __align__(8) uint64_t empty_bar[kQkSlots];
  __shared__ __align__(16) float qs[4 * 128];  // the group's four query rows
  __shared__ float red[kQkWarps + 1][4];
  __shared__ float hstat[4];
  __shared__ int last_page[kQkSlots];  // last page issued into each slot (-1: none)
  __shared__ uint2 cand[kMaxCand];     // exp inputs that need the host-libm table: (float index in e_sm, x bits)
  __shared__ int abort_flag, ncand;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kvh = (int)(blockIdx.x % (unsigned)g.kv_heads), oi = (int)(blockIdx.x / (unsigned)g.kv_heads);
  pdl_launch_dependents();
  pdl_wait();
  q = after_wait(q);
  tok_pos = after_wait(tok_pos);
  tok_seq = after_wait(tok_seq);
  order = after_wait(order);
  page_table = after_wait(page_table);
  const int t = order ? order[oi] : oi;
  const int ctx = tok_pos[t] + 1;
  if (ctx > cap || ctx <= 0) {  // uniform over the block
    if (tid == 0) atomicOr(status, kStatusBadContext);
    return;
  }
  const int n = (ctx + kPage - 1) / kPage;
  const size_t row = ((size_t)t * g.kv_heads + kvh) * (size_t)cap;
  // dynamic shared memory: [ring (1024-aligned) | page z coordinates]
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* ring = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  int32_t* pages = reinterpret_cast<int32_t*>(ring + kQkSlots * kSlotBytes);
  {
    const int32_t* pt = page_table + (size_t)tok_seq[t] * g.max_pages_per_seq;
    for (int i = tid; i < n; i += kQkThreads) pages[i] = layer * g.pages + pt[i];
    const float4* qg = reinterpret_cast<const float4*>(q + ((size_t)t * nh + (size_t)kvh * 4) * 128);
    if (tid < 128) reinterpret_cast<float4*>(qs)[tid] = qg[tid];
  }
  if (tid < kQkSlots) last_page[tid] = -1;
  if (tid == 0) {
    for (int s = 0; s < kQkSlots; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();
  volatile int* abort_p = &abort_flag;

  if (warp == kQkWarps) {
    // ---------------- loader: K page i into slot i % kQkSlots ----------------
    const uint64_t pol = evict_first_policy();
    auto issue = [&](int i) {
      const int s = i % kQkSlots;
      const uint32_t bar = smem_u32(&full_bar[s]);
      mbar_expect_tx(bar, kSlotBytes);
      tma_page(smem_u32(ring + s * kSlotBytes), &tmap, (kvh * 2 + 0) * kPage, pages[i], bar, pol);
      last_page[s] = i;
    };
    int i = min(n, kQkSlots);
    if (lane < i) issue(lane);
    // page k reuses the slot of page k - kQkSlots once its warp has read it
    // (the slot's empty barrier completes phase k / kQkSlots - 1); a warp
    // frees its two pages together, so they are refilled two at a time
    while (i < n && !*abort_p) {
      const int nb = min(2, n - i);
      if (lane < nb) {
        const int k = i + lane;
        if (mbar_wait(smem_u32(&empty_bar[k % kQkSlots]), ((k / kQkSlots) - 1) & 1, abort_p))
          issue(k);
        else
          give_up(abort_p, status);
      }
      __syncwarp();
      i += nb;
    }
    if (lane < 4) red[kQkWarps][lane] = -INFINITY;
  } else {
    // ---------------- QK: warp w reads pages 8j + 2w and 8j + 2w + 1 of round j ----------------
    // The ring holds two rounds, so a warp's next pages land while it
    // computes; lane l owns row l & 15 of page 8j + 2w + (l >> 4).
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(128.0f));
    const uint32_t ring_s = smem_u32(ring), qs_s = smem_u32(qs);
    const int r = lane & 15, hp = lane >> 4;
    // 16-byte chunk c of row r sits in 128-byte unit u = 2r + (c >> 3) at
    // chunk (c & 7) ^ (u & 7); a unit's base has no bits in 4..6, so the
    // address is (base_u | ((u & 7) << 4)) ^ ((c & 7) << 4)
    const uint32_t xo0 = (uint32_t)((2 * r) & 7) << 4, xo1 = (uint32_t)((2 * r + 1) & 7) << 4;
    float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    for (int p0 = warp * 2; p0 < n; p0 += kQkRoundPages) {
      bool ok = mbar_wait(smem_u32(&full_bar[p0 % kQkSlots]), (p0 / kQkSlots) & 1, abort_p);
      if (ok && p0 + 1 < n) ok = mbar_wait(smem_u32(&full_bar[(p0 + 1) % kQkSlots]), ((p0 + 1) / kQkSlots) & 1, abort_p);
      if (!ok) {
        give_up(abort_p, status);
        break;
      }
      const int pa = p0 + hp;  // this lane's page (past the context when pa >= n: not loaded, masked)
      const uint32_t ba = ring_s + (uint32_t)(pa % kQkSlots) * kSlotBytes + (uint32_t)(2 * r) * 128;
      const uint32_t c0 = ba | xo0, c1 = (ba + 128) | xo1;
      float acc[4][8];
#pragma unroll
      for (int h = 0; h < 4; ++h)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[h][j] = 0.0f;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint4 k4 = lds128((c < 8 ? c0 : c1) ^ ((uint32_t)(c & 7) << 4));
        const float kf[8] = {bf_lo(k4.x), bf_hi(k4.x), bf_lo(k4.y), bf_hi(k4.y),
                             bf_lo(k4.z), bf_hi(k4.z), bf_lo(k4.w), bf_hi(k4.w)};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float4 q0 = lds128f(qs_s + (uint32_t)(h * 128 + 8 * c) * 4);
          const float4 q1 = lds128f(qs_s + (uint32_t)(h * 128 + 8 * c + 4) * 4);
          const float qq[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[h][j] = __fmaf_rn(qq[j], kf[j], acc[h][j]);
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(smem_u32(&empty_bar[p0 % kQkSlots]));
        if (p0 + 1 < n) mbar_arrive(smem_u32(&empty_bar[(p0 + 1) % kQkSlots]));
      }
      const int pos = pa * kPage + r;
      float sc[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) sc[h] = __fmul_rn(hsum8(acc[h]), scale);
      if (pos < ctx) {
        sp[row + pos] = make_float4(sc[0], sc[1], sc[2], sc[3]);
#pragma unroll
        for (int h = 0; h < 4; ++h) mx[h] = fmaxf(mx[h], sc[h]);
      }
    }
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float v = warp_max(mx[h]);
      if (lane == 0) red[warp][h] = v;
    }
  }
  __syncthreads();
  if (!abort_flag) {
    // ---------------- softmax over [0, ctx), chunks of kEChunk positions through the ring ----------------
    if (tid < 4) {
      float m = red[0][tid];
      for (int w = 1; w <= kQkWarps; ++w) m = fmaxf(m, red[w][tid]);
      hstat[tid] = m;
    }
    __syncthreads();
    const float m0 = hstat[0], m1 = hstat[1], m2 = hstat[2], m3 = hstat[3];
    float4* e_sm = reinterpret_cast<float4*>(ring);
    const int nchunks = (ctx + kEChunk - 1) / kEChunk;
    float sum = 0.0f;  // thread h < 4: the running sum of head h
    for (int c0 = 0; c0 < ctx; c0 += kEChunk) {
      const int len = min(kEChunk, ctx - c0);
      // e = exp(x - m) of the chunk.  The few inputs whose value needs the
      // host-libm table are queued and looked up together afterwards (a
      // lookup is a dependent global load), and each thread's next score row
      // is loaded while the current one is computed.
      if (tid == 0) ncand = 0;
      __syncthreads();
      float4 xn = tid < len ? sp[row + c0 + tid] : make_float4(0.f, 0.f, 0.f, 0.f);
      for (int i = tid; i < len; i += kQkThreads) {
        const float4 x = xn;
        if (i + kQkThreads < len) xn = sp[row + c0 + i + kQkThreads];
        const float xs[4] = {__fsub_rn(x.x, m0), __fsub_rn(x.y, m1), __fsub_rn(x.z, m2), __fsub_rn(x.w, m3)};
        float e[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          if (exp_needs_table(xs[h], et, &e[h])) {
            const int k = atomicAdd(&ncand, 1);
            if (k < kMaxCand)
              cand[k] = make_uint2((uint32_t)(4 * i + h), __float_as_uint(xs[h]));
            else
              e[h] = exp_table_lookup(__float_as_uint(xs[h]), e[h], et);
          }
        }
        e_sm[i] = make_float4(e[0], e[1], e[2], e[3]);
      }
      __syncthreads();
      {
        float* ef = reinterpret_cast<float*>(e_sm);
        const int nc = min(ncand, kMaxCand);
        for (int k = tid; k < nc; k += kQkThreads) ef[cand[k].x] = exp_table_lookup(cand[k].y, ef[cand[k].x], et);
      }
      __syncthreads();
      if (nchunks > 1)
        for (int i = tid; i < len; i += kQkThreads) sp[row + c0 + i] = e_sm[i];
      if (tid < 4) {
        // sum = ((e_0 + e_1) + e_2) + ... of head tid, loads issued a block ahead
        const float* e = reinterpret_cast<const float*>(e_sm) + tid;
        const int full = len & ~15;
        int i = 0;
        for (; i < full; i += 16) {
          float a[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) a[k] = e[4 * (i + k)];
#pragma unroll
          for (int k = 0; k < 16; ++k) sum = __fadd_rn(sum, a[k]);
        }
        for (; i < len; ++i) sum = __fadd_rn(sum, e[4 * i]);
      }
      __syncthreads();
    }
    if (tid < 4) hstat[tid] = __fdiv_rn(1.0f, sum);
    __syncthreads();
    const float i0 = hstat[0], i1 = hstat[1], i2 = hstat[2], i3 = hstat[3];
    const int last0 = (nchunks - 1) * kEChunk;
    for (int i = tid; i < ctx; i += kQkThreads) {
      const float4 e = i >= last0 ? e_sm[i - last0] : sp[row + i];
      sp[row + i] = make_float4(__fmul_rn(e.x, i0), __fmul_rn(e.y, i1), __fmul_rn(e.z, i2), __fmul_rn(e.w, i3));
    }
  } else if (tid == 0) {
    // after a failed wait, copies may still be landing in the ring: wait (again
    // bounded) for the last one issued into each slot before the CTA exits
    for (int s = 0; s < kQkSlots; ++s)
      if (last_page[s] >= 0) mbar_wait(smem_u32(&full_bar[s]), (last_page[s] / kQkSlots) & 1, nullptr);
  }
}

// One CTA per (token order[blockIdx.x / kv_heads], kv head blockIdx.x % kv_heads): out = sum_t p_t V_t
// for the group's four heads, p from the QK kernel's rows of sp.
__global__ void __launch_bounds__(kPvThreads, 6) attn_pv_kernel(
    const int32_t* __restrict__ tok_pos, const int32_t* __restrict__ tok_seq, const int32_t* __restrict__ order,
    const int32_t* __restrict__ page_table, KvGeom g, int layer, int cap, int nh, const float4* __restrict__ sp,
    float* __restrict__ out, int32_t* __restrict__ status, const __grid_constant__ CUtensorMap tmap) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kPvSlots];
  __shared__ __align__(8) uint64_t empty_bar[kPvSlots];
  __shared__ int last_page[kPvSlots];
  __shared__ int abort_flag;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kvh = (int)(blockIdx.x % (unsigned)g.kv_heads), oi = (int)(blockIdx.x / (unsigned)g.kv_heads);
  pdl_launch_dependents();
  pdl_wait();
  tok_pos = after_wait(tok_pos);
  tok_seq = after_wait(tok_seq);
  order = after_wait(order);
  page_table = after_wait(page_table);
  sp = after_wait(sp);
  const int t = order ? order[oi] : oi;
  const int ctx = tok_pos[t] + 1;
  if (ctx > cap || ctx <= 0) {
    if (tid == 0) atomicOr(status, kStatusBadContext);
    return;
  }
  const int n = (ctx + kPage - 1) / kPage;
  const size_t row = ((size_t)t * g.kv_heads + kvh) * (size_t)cap;
  // dynamic shared memory: [V tiles (1024-aligned) | p rows | page z coordinates]
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* vring = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  uint8_t* pring = vring + kPvSlots * kSlotBytes;
  int32_t* pages = reinterpret_cast<int32_t*>(pring + kPvSlots * kPage * 16);
  {
    const int32_t* pt = page_table + (size_t)tok_seq[t] * g.max_pages_per_seq;
    for (int i = tid; i < n; i += kPvThreads) pages[i] = layer * g.pages + pt[i];
  }
  if (tid < kPvSlots) last_page[tid] = -1;
  if (tid == 0) {
    for (int s = 0; s < kPvSlots; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), kPvWarps);
    }
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();
  volatile int* abort_p = &abort_flag;

  if (warp == kPvWarps) {
    // ---------------- loader: V page i and its p rows into slot i % kPvSlots ----------------
    const uint64_t pol = evict_first_policy();
    auto issue = [&](int i) {
      const int s = i % kPvSlots;
      const uint32_t bar = smem_u32(&full_bar[s]);
      mbar_expect_tx(bar, kPvSlotBytes);
      tma_page(smem_u32(vring + s * kSlotBytes), &tmap, (kvh * 2 + 1) * kPage, pages[i], bar, pol);
      bulk_copy(smem_u32(pring + s * kPage * 16), sp + row + (size_t)i * kPage, kPage * 16, bar, pol);
      last_page[s] = i;
    };
    int i = min(n, kPvSlots);
    if (lane < i) issue(lane);
    while (i < n && !*abort_p) {
      const int nb = min(2, n - i);
      if (lane < nb) {
        const int k = i + lane;
        if (mbar_wait(smem_u32(&empty_bar[k % kPvSlots]), ((k / kPvSlots) - 1) & 1, abort_p))
          issue(k);
        else
          give_up(abort_p, status);
      }
      __syncwarp();
      i += nb;
    }
  } else {
    // ---------------- PV: lane l of warp w owns dims 64w + 2l, 64w + 2l + 1 of the four heads ----------------
    // row rr of the V tile: the lane's word sits in unit u = 2 rr + w at chunk
    // (l >> 2) ^ (u & 7), byte 4 (l & 3); the swizzle repeats every 4 rows
    uint32_t vo[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      vo[k] = (uint32_t)(warp * 128 + ((((lane >> 2) ^ ((2 * k + warp) & 7))) << 4) + (lane & 3) * 4);
    const uint32_t vring_s = smem_u32(vring), pring_s = smem_u32(pring);
    float o[4][2];
#pragma unroll
    for (int h = 0; h < 4; ++h) o[h][0] = o[h][1] = 0.0f;
    for (int P = 0; P < n; ++P) {
      const int s = P % kPvSlots;
      if (!mbar_wait(smem_u32(&full_bar[s]), (P / kPvSlots) & 1, abort_p)) {
        give_up(abort_p, status);
        break;
      }
      const uint32_t vb = vring_s + (uint32_t)s * kSlotBytes, pb = pring_s + (uint32_t)s * kPage * 16;
      const int rows = min(kPage, ctx - P * kPage);
      if (rows == kPage) {
        uint32_t v[kPage];
#pragma unroll
        for (int rr = 0; rr < kPage; ++rr) v[rr] = lds32(vb + 256u * rr + vo[rr & 3]);
        // p of the next four rows is loaded while the current four are used
        float4 pa[4], pn[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) pa[k] = lds128f(pb + 16u * k);
#pragma unroll
        for (int g4 = 0; g4 < 4; ++g4) {
          if (g4 < 3) {
#pragma unroll
            for (int k = 0; k < 4; ++k) pn[k] = lds128f(pb + 16u * (4 * (g4 + 1) + k));
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint32_t w = v[4 * g4 + k];
            const float x0 = bf_lo(w), x1 = bf_hi(w);
            o[0][0] = __fmaf_rn(pa[k].x, x0, o[0][0]);
            o[0][1] = __fmaf_rn(pa[k].x, x1, o[0][1]);
            o[1][0] = __fmaf_rn(pa[k].y, x0, o[1][0]);
            o[1][1] = __fmaf_rn(pa[k].y, x1, o[1][1]);
            o[2][0] = __fmaf_rn(pa[k].z, x0, o[2][0]);
            o[2][1] = __fmaf_rn(pa[k].z, x1, o[2][1]);
            o[3][0] = __fmaf_rn(pa[k].w, x0, o[3][0]);
            o[3][1] = __fmaf_rn(pa[k].w, x1, o[3][1]);
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) pa[k] = pn[k];
        }
      } else {
        for (int rr = 0; rr < rows; ++rr) {
          const uint32_t w = lds32(vb + 256u * rr + vo[rr & 3]);
          const float4 pp = lds128f(pb + 16u * rr);
          const float x0 = bf_lo(w), x1 = bf_hi(w);
          o[0][0] = __fmaf_rn(pp.x, x0, o[0][0]);
          o[0][1] = __fmaf_rn(pp.x, x1, o[0][1]);
          o[1][0] = __fmaf_rn(pp.y, x0, o[1][0]);
          o[1][1] = __fmaf_rn(pp.y, x1, o[1][1]);
          o[2][0] = __fmaf_rn(pp.z, x0, o[2][0]);
          o[2][1] = __fmaf_rn(pp.z, x1, o[2][1]);
          o[3][0] = __fmaf_rn(pp.w, x0, o[3][0]);
          o[3][1] = __fmaf_rn(pp.w, x1, o[3][1]);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&empty_bar[s]));
    }
    float* ob = out + ((size_t)t * nh + (size_t)kvh * 4) * 128 + 64 * warp + 2 * lane;
#pragma unroll
    for (int h = 0; h < 4; ++h) *reinterpret_cast<float2*>(ob + h * 128) = make_float2(o[h][0], o[h][1]);
  }
  __syncthreads();
  if (abort_flag && tid == 0)
    for (int s = 0; s < kPvSlots; ++s)
      if (last_page[s] >= 0) mbar_wait(smem_u32(&full_bar[s]), (last_page[s] / kPvSlots) & 1, nullptr);
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
bool attn_x4_supported(const KvGeom& kv, int nh) { return kv.bf16 && kv.hd == 128 && nh == 4 * kv.kv_heads; }

int attn_x4_cap(int max_ctx) { return (max_ctx + 63) / 64 * 64; }

size_t attn_x4_scratch_floats(int T, int kv_heads, int max_ctx) {
  return (size_t)T * kv_heads * attn_x4_cap(max_ctx) * 4;
}

static size_t qk_smem(int cap) { return 1024 + (size_t)kQkSlots * kSlotBytes + (size_t)(cap / kPage) * 4; }
static size_t pv_smem(int cap) {
  return 1024 + (size_t)kPvSlots * (kSlotBytes + kPage * 16) + (size_t)(cap / kPage) * 4;
}

size_t attn_x4_smem(int max_ctx) { return qk_smem(attn_x4_cap(max_ctx)); }

int attn_x4_prepare(int max_ctx) {
  const int cap = attn_x4_cap(max_ctx);
  if (cudaFuncSetAttribute(attn_qk_softmax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)qk_smem(cap)) !=
      cudaSuccess)
    return 1;
  if (cudaFuncSetAttribute(attn_pv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pv_smem(cap)) !=
      cudaSuccess)
    return 1;
  return 0;
}

void launch_attn_x4(const float* q, int T, int nh, const int32_t* tok_pos, const int32_t* tok_seq,
                    const int32_t* order, const int32_t* page_table, const KvGeom& kv, const CUtensorMap& map,
                    int layer, int max_ctx, float* out, float* scratch, const ExpTable& et, int32_t* status,
                    cudaStream_t st) {
  if (T <= 0) return;
  const int cap = attn_x4_cap(max_ctx);
  float4* sp = reinterpret_cast<float4*>(scratch);
  attn_qk_softmax_kernel<<<(unsigned)(T * kv.kv_heads), kQkThreads, qk_smem(cap), st>>>(q, nh, tok_pos, tok_seq, order,
                                                                                 page_table, kv, layer, cap, sp, et,
                                                                                 status, map);
  count_launch();
  attn_pv_kernel<<<(unsigned)(T * kv.kv_heads), kPvThreads, pv_smem(cap), st>>>(tok_pos, tok_seq, order, page_table, kv,
                                                                         layer, cap, nh, sp, out, status, map);
  count_launch();
}

}  // namespace bitnet
