// tp.cu — tensor-parallel support: NCCL loaded at run time, the unique-id
// entry point, and the kernels around the model's per-layer collectives
// (gate of the local FFN slice, re-layout of all-gathered rows, epilogue of
// all-reduced int32 accumulators).
#include <dlfcn.h>

#include <cstdlib>
#include <cstring>
#include <mutex>

#include "internal.h"
#include "tp.cuh"

static_assert(sizeof(ncclUniqueId) == BITNET_TP_ID_BYTES, "NCCL unique id size");

namespace bitnet {

namespace {

std::once_flag g_nccl_once;
NcclApi g_nccl{};
bool g_nccl_ok = false;
std::string g_nccl_why;

template <class F>
bool resolve(void* h, const char* name, F* out) {
  *out = reinterpret_cast<F>(dlsym(h, name));
  if (!*out) g_nccl_why = std::string("NCCL symbol ") + name + " not found";
  return *out != nullptr;
}

void load_nccl() {
  const char* env = std::getenv("BITNET_NCCL_LIBRARY");
  const char* name = env && *env ? env : "libnccl.so.2";
  void* h = dlopen(name, RTLD_NOW | RTLD_GLOBAL);
  if (!h) {
    const char* e = dlerror();
    g_nccl_why = std::string("cannot load ") + name + (e ? std::string(": ") + e : std::string());
    return;
  }
  g_nccl_ok = resolve(h, "ncclGetUniqueId", &g_nccl.get_unique_id) &&
              resolve(h, "ncclCommInitRank", &g_nccl.comm_init_rank) &&
              resolve(h, "ncclCommInitRankConfig", &g_nccl.comm_init_rank_config) &&
              resolve(h, "ncclCommGetAsyncError", &g_nccl.comm_get_async_error) &&
              resolve(h, "ncclCommAbort", &g_nccl.comm_abort) &&
              resolve(h, "ncclCommDestroy", &g_nccl.comm_destroy) &&
              resolve(h, "ncclAllReduce", &g_nccl.all_reduce) && resolve(h, "ncclAllGather", &g_nccl.all_gather) &&
              resolve(h, "ncclGetErrorString", &g_nccl.error_string);
}

}  // namespace

const NcclApi* nccl_api(std::string* why) {
  std::call_once(g_nccl_once, load_nccl);
  if (!g_nccl_ok && why) *why = g_nccl_why;
  return g_nccl_ok ? &g_nccl : nullptr;
}

// ---------------------------------------------------------------------------
// Kernels. One thread per float4; every size is a multiple of 4 floats.
// ---------------------------------------------------------------------------
__global__ void tp_gate_rows_kernel(const float4* __restrict__ gu, int T, int F4, float4* __restrict__ out) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)T * F4) return;
  const size_t t = i / F4, j = i % F4;
  const float4 g = gu[t * 2 * F4 + j], u = gu[t * 2 * F4 + F4 + j];
  // sqrelu_gate: r = max(g, 0) (NaN -> 0), out = (r * r) * u
  const float r0 = fmaxf(g.x, 0.0f), r1 = fmaxf(g.y, 0.0f), r2 = fmaxf(g.z, 0.0f), r3 = fmaxf(g.w, 0.0f);
  out[i] = make_float4(__fmul_rn(__fmul_rn(r0, r0), u.x), __fmul_rn(__fmul_rn(r1, r1), u.y),
                       __fmul_rn(__fmul_rn(r2, r2), u.z), __fmul_rn(__fmul_rn(r3, r3), u.w));
}

void launch_tp_gate_rows(const float* gu, int T, int Fr, float* out, cudaStream_t st) {
  const size_t n = (size_t)T * (Fr / 4);
  if (!n) return;
  tp_gate_rows_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(reinterpret_cast<const float4*>(gu), T, Fr / 4,
                                                                  reinterpret_cast<float4*>(out));
  count_launch();
}

__global__ void tp_unchunk_kernel(const float4* __restrict__ src, int G, int T, int C4, float4* __restrict__ dst) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)G * T * C4) return;
  const size_t c = i % C4, r = i / C4;
  const size_t t = r % T, g = r / T;
  dst[t * (size_t)G * C4 + g * C4 + c] = src[i];
}

void launch_tp_unchunk(const float* src, int G, int T, int C, float* dst, cudaStream_t st) {
  const size_t n = (size_t)G * T * (C / 4);
  if (!n) return;
  tp_unchunk_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(reinterpret_cast<const float4*>(src), G, T, C / 4,
                                                               reinterpret_cast<float4*>(dst));
  count_launch();
}

__global__ void acc_epilogue_kernel(const int32_t* __restrict__ acc, int M, int N, float ws,
                                    const float* __restrict__ amax, int residual, float* __restrict__ out, int ldo) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)M * N) return;
  const size_t m = i / N, n = i % N;
  // acc as f32 * (weight_scale * act_absmax / 127) (gemv.rs:299-308)
  const float combined = __fdiv_rn(__fmul_rn(ws, amax[m]), 127.0f);
  const float v = __fmul_rn((float)acc[i], combined);
  float* p = out + m * (size_t)ldo + n;
  *p = residual ? __fadd_rn(*p, v) : v;  // residual: axpy_f32_fast(1.0, o, h) == h + o
}

void launch_acc_epilogue(const int32_t* acc, int M, int N, float ws, const float* amax, Epi epi, float* out, int ldo,
                         cudaStream_t st) {
  const size_t n = (size_t)M * N;
  if (!n) return;
  acc_epilogue_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, st>>>(acc, M, N, ws, amax, epi == Epi::Residual ? 1 : 0,
                                                                  out, ldo);
  count_launch();
}

__device__ __forceinline__ void pair_merge(float& bv, uint32_t& bi, float v, uint32_t i) {
  if (v > bv || (v == bv && i > bi)) {
    bv = v;
    bi = i;
  }
}

__global__ void argmax_pairs_kernel(const float* __restrict__ logits, int ld, int V, uint32_t offset,
                                    uint2* __restrict__ pairs) {
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  const int m = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* row = logits + (size_t)m * ld;
  float bv = -INFINITY;
  uint32_t bi = 0;
  for (int v = threadIdx.x; v < V; v += blockDim.x) pair_merge(bv, bi, row[v], (uint32_t)v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
    pair_merge(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) pair_merge(bv, bi, sv[w], si[w]);
    pairs[m] = make_uint2(__float_as_uint(bv), bi + offset);
  }
}

void launch_argmax_pairs(const float* logits, int ld, int M, int V, uint32_t offset, uint2* pairs, cudaStream_t st) {
  if (M <= 0) return;
  argmax_pairs_kernel<<<M, 1024, 0, st>>>(logits, ld, V, offset, pairs);
  count_launch();
}

__global__ void argmax_combine_kernel(const uint2* __restrict__ all, int G, int M, uint32_t* __restrict__ out) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= M) return;
  float bv = -INFINITY;
  uint32_t bi = 0;
  for (int g = 0; g < G; ++g) {
    const uint2 p = all[(size_t)g * M + m];
    pair_merge(bv, bi, __uint_as_float(p.x), p.y);
  }
  out[m] = bi;
}

void launch_argmax_combine(const uint2* all, int G, int M, uint32_t* out, cudaStream_t st) {
  if (M <= 0) return;
  argmax_combine_kernel<<<(unsigned)ceil_div(M, 256), 256, 0, st>>>(all, G, M, out);
  count_launch();
}

}  // namespace bitnet

using namespace bitnet;

extern "C" int bitnet_cuda_tp_unique_id(uint8_t* id, size_t id_len) {
  if (!id) return shape_error("non-null id buffer", "null");
  if (id_len < sizeof(ncclUniqueId))
    return shape_error("id_len >= " + std::to_string(sizeof(ncclUniqueId)), std::to_string(id_len));
  std::string why;
  const NcclApi* nc = nccl_api(&why);
  if (!nc) return backend_error(why);
  ncclUniqueId u;
  ncclResult_t r = nc->get_unique_id(&u);
  if (r != ncclSuccess) return backend_error(std::string("ncclGetUniqueId: ") + nc->error_string(r));
  std::memcpy(id, &u, sizeof u);
  return BITNET_OK;
}
