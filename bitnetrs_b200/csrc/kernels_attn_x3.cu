// kernels_attn_x3.cu — reference-order paged attention for a bf16 cache with
// head_dim 128 and GQA group 4, fed by TMA.
//
// One CTA per (query token, kv head) serves the four query heads of the group
// and computes, bit for bit, what the reference's masked_attention does for
// each head (attention.rs:165-206):
//   score[g][t] = dot_f32_f32(q_g, K[t]) * (1/sqrt(128))   8 FMA chains over
//                 16 chunks of 8 dims, then hsum_f32_avx2 (simd.rs:292-307)
//   softmax_f32: m = max_t score, e = exp(score - m),
//                sum = ((e_0 + e_1) + e_2) + ...,  p = e * (1/sum)
//   out[g][d]  = fma(p_t, V[t][d], out[g][d]) for t = 0, 1, ...
//
// Organisation (288 threads = 9 warps, two CTAs per SM):
//   * The context streams through a ring of kX3Slots page slots, one 4-D TMA
//     tile load per page (128-byte swizzle; slot layout [16 rows][2 halves]
//     [64 bf16], the 16-byte chunk c of 128-byte unit u = 2*row + half
//     stored at chunk c ^ (u & 7)): first the K blocks of every page, then
//     the V blocks.  Warp 8 issues the loads, kX3Batch at a time from
//     separate lanes (issuing a bulk copy holds the issuing thread for ~150
//     cycles, so it stays off the compute warps).
//     A slot's "full" mbarrier counts the TMA bytes; its "empty" signal is
//     named barrier 1 + slot: the four warps that read the slot bar.arrive,
//     the loader warp bar.syncs before refilling it.
//   * QK: warps 4g..4g+3 take pages g, g+2, ... (4 positions each); eight
//     lanes per position, lane (jq, hp) runs FMA chains 2jq and 2jq+1 of heads
//     2hp and 2hp+1 (fmaf, one rounding each, as _mm256_fmadd_ps); two
//     shuffles then combine the chains in hsum order.
//   * Softmax in shared memory: exp inputs that need the host-libm table are
//     queued and resolved together; lanes 0-3 of warp 0 run the four
//     sequential sums.
//   * PV: warps 0-3, lane l of warp w owns dim 32w + l of all four heads
//     (each V element converted once), each chain running over positions in
//     order.
#include "kernels.cuh"

#include <cudaTypedefs.h>

#include <mutex>

namespace bitnet {

namespace {

constexpr int kX3Slots = 8;            // ring depth (pages of K or V)
constexpr int kX3SlotBytes = 4096;     // [16 rows][2 halves][64 bf16], 128-byte swizzled
constexpr int kX3Warps = 8;            // compute warps: QK (four per page), softmax, PV (warps 0-3)
constexpr int kX3Threads = (kX3Warps + 1) * 32;  // + the loader warp
constexpr int kX3Batch = 2;            // loads the loader issues per step, one lane each
constexpr int kX3ComputeThreads = kX3Warps * 32;
constexpr int kX3SlotBar = 160;        // threads meeting at a slot's named barrier (4 readers + loader)
constexpr int kX3MaxCand = 256;        // queued exp-table lookups per CTA
constexpr long long kX3WaitCycles = 2000000000LL;  // ~1 s at the boost clock

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for the phase of `parity` to complete.  Returns false when it has not
// completed within kX3WaitCycles, or (when abort_flag is given) as soon as
// another warp of the CTA has given up.
__device__ __noinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, const volatile int* abort_flag) {
  const long long t0 = clock64();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort_flag && *abort_flag) return false;
    if (clock64() - t0 > kX3WaitCycles) return false;
  }
}
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const volatile int* abort_flag) {
  return mbar_try_wait(bar, parity) || mbar_wait_slow(bar, parity, abort_flag);
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %2, %3, %4}], "
      "[%5];\n" ::"r"(dst),
      "l"((uint64_t)map), "r"(0), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

// Named barriers: 0 = __syncthreads, 1..kX3Slots = slot s is free again,
// kX3Slots + 1 = the compute warps.
template <int ID>
__device__ __forceinline__ void bar_arrive_id() {
  asm volatile("bar.arrive %0, %1;\n" ::"n"(ID), "n"(kX3SlotBar) : "memory");
}
template <int ID>
__device__ __forceinline__ void bar_sync_id() {
  asm volatile("bar.sync %0, %1;\n" ::"n"(ID), "n"(kX3SlotBar) : "memory");
}
// Immediate barrier ids (a register id costs uniform-datapath moves per use).
__device__ __forceinline__ void slot_release(int s) {
  switch (s) {
    case 0: bar_arrive_id<1>(); break;
    case 1: bar_arrive_id<2>(); break;
    case 2: bar_arrive_id<3>(); break;
    case 3: bar_arrive_id<4>(); break;
    case 4: bar_arrive_id<5>(); break;
    case 5: bar_arrive_id<6>(); break;
    case 6: bar_arrive_id<7>(); break;
    default: bar_arrive_id<8>(); break;
  }
}
__device__ __forceinline__ void slot_wait_free(int s) {
  switch (s) {
    case 0: bar_sync_id<1>(); break;
    case 1: bar_sync_id<2>(); break;
    case 2: bar_sync_id<3>(); break;
    case 3: bar_sync_id<4>(); break;
    case 4: bar_sync_id<5>(); break;
    case 5: bar_sync_id<6>(); break;
    case 6: bar_sync_id<7>(); break;
    default: bar_sync_id<8>(); break;
  }
}
static_assert(kX3Slots == 8, "slot barriers are spelled out for 8 slots");
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];\n" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];\n" : "=h"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ void compute_bar() {
  asm volatile("bar.sync %0, %1;\n" ::"n"(kX3Slots + 1), "n"(kX3ComputeThreads) : "memory");
}

}  // namespace

__global__ void __launch_bounds__(kX3Threads, 2) paged_attention_exact3_kernel(
    const float* __restrict__ q, int nh, const int32_t* __restrict__ tok_pos, const int32_t* __restrict__ tok_seq,
    const int32_t* __restrict__ page_table, KvGeom g, int layer, int cap, float* __restrict__ out, ExpTable et,
    int32_t* __restrict__ status, const __grid_constant__ CUtensorMap tmap) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kX3Slots];
  __shared__ __align__(16) float4 qs[16 * 8];  // [chunk][jq][hp]: q[2hp][8c+2jq..+1], q[2hp+1][8c+2jq..+1]
  __shared__ int issued_sh;                    // loads issued (0 .. issued_sh-1)
  __shared__ uint2 cand[kX3MaxCand];           // (float index into the scores, exp input bits)
  __shared__ float red[kX3Warps][4];
  __shared__ float hmax[4], hinv[4];
  __shared__ int abort_flag, ncand;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t = blockIdx.x, kvh = blockIdx.y;
  pdl_launch_dependents();
  pdl_wait();
  q = after_wait(q);
  tok_pos = after_wait(tok_pos);
  tok_seq = after_wait(tok_seq);
  page_table = after_wait(page_table);
  const int ctx = tok_pos[t] + 1;
  if (ctx > cap || ctx <= 0) {  // uniform over the block
    if (tid == 0) atomicOr(status, kStatusBadContext);
    return;
  }
  const int n = (ctx + kPage - 1) / kPage;
  const int total = 2 * n;  // K blocks, then V blocks
  // shared layout: [ring (1024-aligned)][page z coordinates cap/16][scores cap x float4]
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* ring = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  int32_t* pages = reinterpret_cast<int32_t*>(ring + kX3Slots * kX3SlotBytes);
  float4* sc = reinterpret_cast<float4*>(pages + cap / kPage);
  {
    const int32_t* pt = page_table + (size_t)tok_seq[t] * g.max_pages_per_seq;
    for (int i = tid; i < n; i += kX3Threads) pages[i] = layer * g.pages + pt[i];
    const float* qg = q + ((size_t)t * nh + (size_t)kvh * 4) * 128;
    if (tid < 128) {
      const int c = tid >> 3, jq = (tid >> 1) & 3, hp = tid & 1;
      const float2 a = *reinterpret_cast<const float2*>(qg + (2 * hp) * 128 + 8 * c + 2 * jq);
      const float2 b = *reinterpret_cast<const float2*>(qg + (2 * hp + 1) * 128 + 8 * c + 2 * jq);
      qs[tid] = make_float4(a.x, a.y, b.x, b.y);
    }
  }
  if (tid == 0) {
    for (int s = 0; s < kX3Slots; ++s) mbar_init(smem_u32(&full_bar[s]), 1);
    abort_flag = 0;
    ncand = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();
  volatile int* abort_p = &abort_flag;

  if (warp == kX3Warps) {
    // ---------------- loader: load i (K page i, or V page i - n) into slot i % kX3Slots ----------------
    // Each step frees kX3Batch slots (named barriers) and lanes 0..kX3Batch-1 issue
    // one load each: issuing holds a thread for ~150 cycles, and a single thread
    // issuing page by page falls behind the QK warps.
    auto issue = [&](int i) {
      const int s = i % kX3Slots, kind = i < n ? 0 : 1;
      const uint32_t bar = smem_u32(&full_bar[s]);
      mbar_expect_tx(bar, kX3SlotBytes);
      tma_load_4d(smem_u32(ring + s * kX3SlotBytes), &tmap, (kvh * 2 + kind) * kPage, pages[kind ? i - n : i], bar);
    };
    // Invariant: the readers of loads [0, i - kX3Slots) have been waited for,
    // each exactly once (the readers arrive once per load, issued or not).
    int i = min(total, kX3Slots), issued = i;
    if (lane < i) issue(lane);
    while (i < total) {
      const int nb = min(kX3Batch, total - i);
      for (int b = 0; b < nb; ++b) slot_wait_free((i + b) % kX3Slots);  // readers of load i+b-kX3Slots are done
      i += nb;
      if (*abort_p) break;
      if (lane < nb) issue(i - nb + lane);
      issued = i;
      __syncwarp();
    }
    if (lane == 0) issued_sh = issued;
    // wait for the readers of loads [i - kX3Slots, total), so that no named
    // barrier is left with pending arrivals
    for (int k = max(i, kX3Slots); k < total + kX3Slots; ++k) slot_wait_free(k % kX3Slots);
  } else {
    auto wait_full = [&](int i) {
      if (!mbar_wait(smem_u32(&full_bar[i % kX3Slots]), (i / kX3Slots) & 1, abort_p) && !*abort_p) {
        *abort_p = 1;
        atomicOr(status, kStatusWaitTimeout);
      }
    };
    // ---------------- QK ----------------
    {
      const float scale = __fdiv_rn(1.0f, __fsqrt_rn(128.0f));
      const int jq = lane & 3;          // chains 2jq, 2jq+1
      const int hp = (lane >> 2) & 1;   // heads 2hp, 2hp+1
      const int r = (warp & 3) * 4 + (lane >> 3);  // row (position) within the page
      const float4* qv = qs + jq * 2 + hp;
      // chunk c of row r sits in unit u = 2r + (c >> 3) at chunk (c & 7) ^ (u & 7);
      // the unit's base has no bits in 4..6, so the offset is base_u ^ ((c & 7) << 4)
      const uint32_t kb0 = (uint32_t)((2 * r) * 128 + (((2 * r) & 7) << 4) + jq * 4);
      const uint32_t kb1 = (uint32_t)((2 * r + 1) * 128 + (((2 * r + 1) & 7) << 4) + jq * 4);
      const uint32_t ring_s = smem_u32(ring);
      for (int P = warp >> 2; P < n; P += 2) {
        wait_full(P);
        const int s = P % kX3Slots;
        const uint32_t ka0 = ring_s + s * kX3SlotBytes + kb0, ka1 = ring_s + s * kX3SlotBytes + kb1;
        uint32_t w[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) w[c] = lds_u32((c < 8 ? ka0 : ka1) ^ ((c & 7) << 4));
        slot_release(s);
        // chains 2jq, 2jq+1 of head 2hp (a0, a1) and of head 2hp+1 (b0, b1)
        float a0 = 0.0f, a1 = 0.0f, b0 = 0.0f, b1 = 0.0f;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const float klo = __uint_as_float(w[c] << 16), khi = __uint_as_float(w[c] & 0xffff0000u);
          const float4 qq = qv[8 * c];
          a0 = __fmaf_rn(qq.x, klo, a0);
          a1 = __fmaf_rn(qq.y, khi, a1);
          b0 = __fmaf_rn(qq.z, klo, b0);
          b1 = __fmaf_rn(qq.w, khi, b1);
        }
        // hsum8: lane jq=0 holds chains (0,1), jq=1 (2,3), jq=2 (4,5), jq=3 (6,7);
        // xor 2 pairs chain j with j+4: (s0,s1) on jq=0, (s2,s3) on jq=1
        const float sa0 = __fadd_rn(a0, __shfl_xor_sync(0xffffffffu, a0, 2));
        const float sa1 = __fadd_rn(a1, __shfl_xor_sync(0xffffffffu, a1, 2));
        const float sb0 = __fadd_rn(b0, __shfl_xor_sync(0xffffffffu, b0, 2));
        const float sb1 = __fadd_rn(b1, __shfl_xor_sync(0xffffffffu, b1, 2));
        const float t0 = __fadd_rn(sa0, sa1), t1 = __fadd_rn(sb0, sb1);
        const float u0 = __fadd_rn(t0, __shfl_xor_sync(0xffffffffu, t0, 1));
        const float u1 = __fadd_rn(t1, __shfl_xor_sync(0xffffffffu, t1, 1));
        const int pos = P * kPage + r;
        if (jq == 0 && pos < ctx)
          reinterpret_cast<float2*>(sc + pos)[hp] = make_float2(__fmul_rn(u0, scale), __fmul_rn(u1, scale));
      }
    }
    compute_bar();
    // ---------------- softmax ----------------
    {
      float4 m4 = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      for (int p = tid; p < ctx; p += kX3ComputeThreads) {
        const float4 v = sc[p];
        m4.x = fmaxf(m4.x, v.x);
        m4.y = fmaxf(m4.y, v.y);
        m4.z = fmaxf(m4.z, v.z);
        m4.w = fmaxf(m4.w, v.w);
      }
      m4.x = warp_max(m4.x);
      m4.y = warp_max(m4.y);
      m4.z = warp_max(m4.z);
      m4.w = warp_max(m4.w);
      if (lane == 0) {
        red[warp][0] = m4.x;
        red[warp][1] = m4.y;
        red[warp][2] = m4.z;
        red[warp][3] = m4.w;
      }
      compute_bar();
      if (tid < 4) {
        float m = red[0][tid];
        for (int w = 1; w < kX3Warps; ++w) m = fmaxf(m, red[w][tid]);
        hmax[tid] = m;
      }
      compute_bar();
      const float hm[4] = {hmax[0], hmax[1], hmax[2], hmax[3]};
      for (int p = tid; p < ctx; p += kX3ComputeThreads) {
        float v[4];
        *reinterpret_cast<float4*>(v) = sc[p];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float x = __fsub_rn(v[c], hm[c]);
          float f;
          if (exp_needs_table(x, et, &f)) {
            const int i = atomicAdd(&ncand, 1);
            if (i < kX3MaxCand)
              cand[i] = make_uint2((uint32_t)(4 * p + c), __float_as_uint(x));
            else
              f = exp_table_lookup(__float_as_uint(x), f, et);
          }
          v[c] = f;
        }
        sc[p] = *reinterpret_cast<const float4*>(v);
      }
      compute_bar();
      {
        float* scf = reinterpret_cast<float*>(sc);
        const int nc = min(ncand, kX3MaxCand);
        for (int i = tid; i < nc; i += kX3ComputeThreads)
          scf[cand[i].x] = exp_table_lookup(cand[i].y, scf[cand[i].x], et);
      }
      compute_bar();
      if (tid < 4) {
        // sequential sum of head tid with loads issued a block ahead
        const float* e = reinterpret_cast<const float*>(sc) + tid;
        float sum = 0.0f;
        const int full = ctx & ~15;
        float a[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) a[k] = full ? e[4 * k] : 0.0f;
        for (int p = 0; p < full; p += 16) {
          float b[16];
          const int nx = p + 16 < full ? p + 16 : p;
#pragma unroll
          for (int k = 0; k < 16; ++k) b[k] = e[4 * (nx + k)];
#pragma unroll
          for (int k = 0; k < 16; ++k) sum = __fadd_rn(sum, a[k]);
#pragma unroll
          for (int k = 0; k < 16; ++k) a[k] = b[k];
        }
        for (int p = full; p < ctx; ++p) sum = __fadd_rn(sum, e[4 * p]);
        hinv[tid] = __fdiv_rn(1.0f, sum);
      }
      compute_bar();
      const float i0 = hinv[0], i1 = hinv[1], i2 = hinv[2], i3 = hinv[3];
      for (int p = tid; p < ctx; p += kX3ComputeThreads) {
        float4 v = sc[p];
        v.x = __fmul_rn(v.x, i0);
        v.y = __fmul_rn(v.y, i1);
        v.z = __fmul_rn(v.z, i2);
        v.w = __fmul_rn(v.w, i3);
        sc[p] = v;
      }
      compute_bar();
    }
    // ---------------- PV (warps 0-3) ----------------
    if (warp < 4) {
      const int d = 32 * warp + lane;                        // dim of this lane, all four heads
      // row rr of the lane's dim: unit u = 2rr + h (h = d >> 6), chunk ((d >> 3) & 7) ^ (u & 7),
      // byte 2 (d & 7); the swizzle repeats every 4 rows: offset = 256 rr + vo[rr & 3]
      // with vo[k] the offset of row k less 256 k
      uint32_t vo[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int u = 2 * k + (d >> 6);  // unit of row k; row rr = k + 4m sits 1024 m (= 256 (rr - k)) further
        vo[k] = (uint32_t)((d >> 6) * 128 + ((((d >> 3) & 7) ^ (u & 7)) << 4) + (d & 7) * 2);
      }
      const uint32_t ring_s = smem_u32(ring);
      float o0 = 0.0f, o1 = 0.0f, o2 = 0.0f, o3 = 0.0f;
      for (int P = 0; P < n; ++P) {
        const int i = n + P, s = i % kX3Slots;
        wait_full(i);
        const uint32_t sb = ring_s + s * kX3SlotBytes;
        const int rows = min(kPage, ctx - P * kPage);
        const float4* pp = sc + P * kPage;
        uint32_t v[kPage];
#pragma unroll
        for (int rr = 0; rr < kPage; ++rr) v[rr] = lds_u16(sb + vo[rr & 3] + 256 * rr);
        slot_release(s);
        if (rows == kPage) {
          // p of the next four rows is loaded while the current four are used
          float4 pa[4], pb[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) pa[k] = pp[k];
#pragma unroll
          for (int g4 = 0; g4 < 4; ++g4) {
            if (g4 < 3) {
#pragma unroll
              for (int k = 0; k < 4; ++k) pb[k] = pp[4 * (g4 + 1) + k];
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float x = __uint_as_float(v[4 * g4 + k] << 16);
              o0 = __fmaf_rn(pa[k].x, x, o0);
              o1 = __fmaf_rn(pa[k].y, x, o1);
              o2 = __fmaf_rn(pa[k].z, x, o2);
              o3 = __fmaf_rn(pa[k].w, x, o3);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) pa[k] = pb[k];
          }
        } else {
#pragma unroll
          for (int rr = 0; rr < kPage; ++rr) {
            if (rr >= rows) break;
            const float4 p = pp[rr];
            const float x = __uint_as_float(v[rr] << 16);
            o0 = __fmaf_rn(p.x, x, o0);
            o1 = __fmaf_rn(p.y, x, o1);
            o2 = __fmaf_rn(p.z, x, o2);
            o3 = __fmaf_rn(p.w, x, o3);
          }
        }
      }
      float* o = out + ((size_t)t * nh + (size_t)kvh * 4) * 128 + d;
      o[0] = o0;
      o[128] = o1;
      o[256] = o2;
      o[384] = o3;
    }
  }
  __syncthreads();
  // After a failed wait, loads may still be landing in the ring: wait (again
  // bounded) for the last load issued into each slot before the CTA exits.
  if (abort_flag && tid == 0)
    for (int k = max(0, issued_sh - kX3Slots); k < issued_sh; ++k)
      mbar_wait(smem_u32(&full_bar[k % kX3Slots]), (k / kX3Slots) & 1, nullptr);
}

}  // namespace bitnet

namespace bitnet {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool exact3_supported(const KvGeom& kv, int nh) { return kv.bf16 && kv.hd == 128 && nh == 4 * kv.kv_heads; }

int exact3_cap(int max_ctx) { return (max_ctx + 63) / 64 * 64; }

size_t exact3_smem(int max_ctx) {
  const int cap = exact3_cap(max_ctx);
  return 1024 + (size_t)kX3Slots * kX3SlotBytes + (size_t)(cap / kPage) * 4 + (size_t)cap * 16;
}

int exact3_prepare(size_t smem) {
  return cudaFuncSetAttribute(paged_attention_exact3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ==
                 cudaSuccess
             ? 0
             : 1;
}

// The pool viewed as a 4-D tensor of bf16: x = dim within a half row (64),
// h = half (2), y = row within a page block of all kv heads and both kinds
// (kv_heads * 2 * 16), z = layer * pages + page.  A box of 64 x 2 x 16 x 1 is
// one K or V page of one kv head (4 KiB).
int exact3_make_tmap(const KvGeom& kv, CUtensorMap* map) {
  if (!kv.bf16 || kv.hd != 128) return 1;
  if ((uint64_t)kv.layers * (uint64_t)kv.pages >= (1ull << 31)) return 1;
  if (reinterpret_cast<uintptr_t>(kv.pool) % 16) return 1;
  auto enc = tensor_map_encoder();
  if (!enc) return 1;
  const cuuint64_t dims[4] = {64, 2, (cuuint64_t)kv.kv_heads * 2 * kPage, (cuuint64_t)kv.layers * kv.pages};
  const cuuint64_t strides[3] = {64 * 2, 128 * 2, (cuuint64_t)kv.kv_heads * 2 * kPage * 128 * 2};
  const cuuint32_t box[4] = {64, 2, kPage, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, kv.pool, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : 1;
}

void launch_paged_attention_exact3(const float* q, int T, int nh, const int32_t* tok_pos, const int32_t* tok_seq,
                                   const int32_t* page_table, const KvGeom& kv, const CUtensorMap& map, int layer,
                                   int max_ctx, float* out, const ExpTable& et, int32_t* status, cudaStream_t st) {
  if (T <= 0) return;
  paged_attention_exact3_kernel<<<dim3(T, kv.kv_heads), kX3Threads, exact3_smem(max_ctx), st>>>(
      q, nh, tok_pos, tok_seq, page_table, kv, layer, exact3_cap(max_ctx), out, et, status, map);
  count_launch();
}

}  // namespace bitnet
