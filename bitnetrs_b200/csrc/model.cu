// model.cu — device-resident BitNet model, paged KV cache and the forward,
// batched decode, ragged prefill and greedy generate entry points.
//
// Orchestration follows BitNetModel::forward / forward_into
// (crates/bitnet-model/src/lib.rs:559-862, 931-1163) with the per-token GEMVs
// batched into matmuls over all tokens of a step, the shared activation
// quantisation fused into the preceding RMSNorm, the residual adds fused into
// the o_proj / down_proj epilogues, and q/k/v (gate/up) projections fused into
// one matmul each.  Every fused step computes the same f32 values as the
// reference's separate calls.
#include <algorithm>
#include <chrono>
#include <thread>
#include <tuple>
#include <cmath>
#include <cstring>

#include "internal.h"
#include "tp.cuh"

using namespace bitnet;

namespace {

struct Layer {
  uint32_t *wqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wdown = nullptr;
  float sq, sk, sv, so, sg, su, sd;
  float *attn_norm = nullptr, *attn_sub_norm = nullptr, *ffn_norm = nullptr, *ffn_sub_norm = nullptr;
};

std::string sz(size_t v) { return std::to_string(v); }

}  // namespace

struct bitnet_cuda_model {
  std::atomic<int> refs{1};  // the user handle + one per KV cache
  bitnet_cuda_ctx* ctx = nullptr;
  bitnet_cuda_config cfg{};
  int H = 0, hd = 0, nh = 0, nkv = 0, qd = 0, kvd = 0, F = 0, V = 0, L = 0, Tmax = 0;
  int ldq = 0;  // row stride of the quantised activation buffer
  bool exact_smem_ok = false;  // shared-memory limit of the exact attention kernel raised
  size_t exact_smem_max = 0;
  bool mma_attn_ok = false;  // shared-memory limit of the tensor-core attention kernel raised
  bool lm_mma_ok = false;    // tensor-core lm_head usable (hidden % 64 == 0, smem limit raised)
  bool exact2_ok = false;    // shared-memory limit of the bf16/hd128 reference-order attention raised
  size_t exact2_smem_max = 0;
  bool exact3_ok = false;    // same for the TMA-fed variant
  size_t exact3_smem_max = 0;
  bool x4_ok = false;        // same for the two-kernel (QK + softmax, PV) variant
  size_t x4_smem_max = 0;
  uint16_t* a3 = nullptr;    // [R][3H] bf16 split of the final-normed rows
  int numerics = BITNET_NUMERICS_AUTO;
  std::vector<Layer> layers;
  std::vector<void*> allocs;
  uint16_t* embed = nullptr;
  int8_t* lm_i8 = nullptr;
  float* lm_scales = nullptr;
  float* final_norm = nullptr;
  float *rope_cos = nullptr, *rope_sin = nullptr;
  // activations
  float *h = nullptr, *qkv = nullptr, *qrot = nullptr, *attn = nullptr, *gu = nullptr, *hn = nullptr, *logits = nullptr;
  int8_t* xq = nullptr;
  float* amax = nullptr;
  int32_t* rowsum = nullptr;
  uint32_t *tokens = nullptr, *next = nullptr;
  uint32_t* hist = nullptr;  // [max_position_embeddings] tokens of the sequence being sampled
  int32_t *tok_pos = nullptr, *tok_seq = nullptr, *last_row = nullptr, *order = nullptr, *status = nullptr;
  DevBuf partial;
  // pinned staging
  int32_t* h_meta = nullptr;  // [4 * Tmax]: pos, seq, last_row, order (tokens by descending position)
  uint32_t* h_tokens = nullptr;
  // captured decode graphs, keyed by (kv, batch, timed), with their kernel
  // counts and (when timed) the event pairs recorded around each launch
  struct Graph {
    cudaGraphExec_t exec;
    uint64_t kernels;
    std::vector<std::tuple<int, cudaEvent_t, cudaEvent_t>> marks;
  };
  std::map<std::tuple<void*, int, int>, Graph> graphs;
  bool timing = false;
  const Graph* last_timed = nullptr;
  std::vector<std::tuple<int, cudaEvent_t, cudaEvent_t>>* marks = nullptr;  // set while capturing a timed graph
  // tensor parallelism (bitnet_cuda_model_create_tp): nh, nkv, qd, kvd and F
  // above are this rank's share; qd_all and F_all the full widths
  bool tp = false;
  int tp_rank = 0, tp_world = 1, qd_all = 0, F_all = 0;
  const NcclApi* nc = nullptr;
  ncclComm_t comm = nullptr;
  ncclResult_t nccl_rc = ncclSuccess;  // first failed collective since the last check
  float *tp_gath = nullptr, *tp_full = nullptr;  // [world][T][C] all-gather, [T][world*C] full rows
  int32_t *tp_acc = nullptr, *tp_rowsum = nullptr;  // [T][H] partial then total accumulators; slice row sums
  // vocabulary slice of the lm_head: rows [v0, v0 + Vloc) of the table, Vs
  // columns per rank in `logits` (the last rank's slice may be shorter)
  int v0 = 0, Vloc = 0, Vs = 0;
  uint2 *tp_pairs = nullptr, *tp_pairs_all = nullptr;  // [R] this rank's (value, index) argmax, [G][R] all ranks'
  float *tp_lgath = nullptr, *tp_logits = nullptr;     // [G][R][Vs] all-gathered slices, [R][G*Vs] full rows
  bool tp_dead = false;  // the communicator was aborted; every later call fails
  int tp_timeout_ms = 300000;
  // one-token decode steps as one persistent kernel (kernels_decode1.cu)
  D1Layer* d1_layers = nullptr;  // device copy of the per-layer pointers and scales
  uint32_t* d1_sync = nullptr;   // the kernel's grid counters
  size_t d1_limit = 0;           // dynamic shared memory the kernel may use (0: unavailable)
  int d1_sms = 0;
  bool d1_enabled = true;        // bitnet_cuda_model_set_fused_decode
  int d1_cap = 0;                // context capacity of the cached plan (0: none)
  size_t d1_smem = 0;            // its dynamic shared memory (0: the plan does not fit)
  D1Params d1_plan;
  // one-row int8 lm_head with the argmax folded in (launch_lm_head_m1)
  bool lm1_ok = false;
  CUtensorMap lm1_tmap{};
  void* lm1_part = nullptr;

  template <class T>
  int alloc(T** p, size_t n) {
    void* q = nullptr;
    cudaError_t e = cudaMalloc(&q, std::max<size_t>(n * sizeof(T), 16));
    if (e != cudaSuccess) return cuda_error(e, "cudaMalloc");
    allocs.push_back(q);
    *p = (T*)q;
    return BITNET_OK;
  }
};

struct bitnet_cuda_kv {
  bitnet_cuda_model* model = nullptr;
  KvGeom g;
  int max_seqs = 0;
  std::vector<int32_t> free_pages;
  std::vector<std::vector<int32_t>> seq_pages;
  std::vector<size_t> seq_len;
  std::vector<int32_t> h_table;
  int32_t* d_table = nullptr;
  CUtensorMap tmap{};     // the pool as a tensor for TMA (bf16, head_dim 128)
  bool tmap_ok = false;
  size_t capacity() const { return (size_t)g.max_pages_per_seq * kPage; }
};

static void model_release(bitnet_cuda_model* m);

namespace {

// ModelConfig::validate (config.rs:110-150).
int validate_config(const bitnet_cuda_config& c) {
  if (c.hidden_size == 0) return config_error("hidden_size must be > 0");
  if (c.num_attention_heads == 0) return config_error("num_attention_heads must be > 0");
  if (c.num_key_value_heads == 0) return config_error("num_key_value_heads must be > 0");
  if (c.hidden_size % c.num_attention_heads != 0)
    return config_error("hidden_size (" + sz(c.hidden_size) + ") must be divisible by num_attention_heads (" +
                        sz(c.num_attention_heads) + ")");
  if (c.num_attention_heads % c.num_key_value_heads != 0)
    return config_error("num_attention_heads (" + sz(c.num_attention_heads) +
                        ") must be divisible by num_key_value_heads (" + sz(c.num_key_value_heads) + ")");
  if (c.vocab_size == 0) return config_error("vocab_size must be > 0");
  if (c.num_hidden_layers == 0) return config_error("num_hidden_layers must be > 0");
  if (c.intermediate_size == 0) return config_error("intermediate_size must be > 0");
  if (c.max_position_embeddings == 0) return config_error("max_position_embeddings must be > 0");
  if (c.hidden_size > (uint32_t)kMaxRowFloats || c.intermediate_size > (uint32_t)kMaxRowFloats)
    return config_error("hidden_size and intermediate_size must be <= " + sz(kMaxRowFloats) +
                        " (rows staged in shared memory)");
  if (!(c.rope_theta > 0.0f)) return config_error("rope_theta must be > 0");
  if (!(c.rms_norm_eps > 0.0f)) return config_error("rms_norm_eps must be > 0");
  return BITNET_OK;
}

// Upload `rows` rows of a reference-format ternary tensor and repack them
// into dst (device words) starting at row `row0`.
int put_ternary(bitnet_cuda_model* m, const uint8_t* src, int rows, int cols, uint32_t* dst, int row0, DevBuf& tmp) {
  if (!src) return shape_error("non-null ternary weight pointer", "null");
  size_t pc = (size_t)(cols + 3) / 4;
  BN_TRY(tmp.ensure((size_t)rows * pc));
  BN_CUDA(cudaMemcpyAsync(tmp.p, src, (size_t)rows * pc, cudaMemcpyHostToDevice, m->ctx->stream));
  launch_repack_ternary(tmp.as<uint8_t>(), dst + (size_t)row0 * words_per_row(cols), rows, cols, m->ctx->stream);
  BN_CUDA(cudaStreamSynchronize(m->ctx->stream));  // tmp is reused by the next tensor
  return BITNET_OK;
}

template <class T>
int put(bitnet_cuda_model* m, T** dst, const T* src, size_t n) {
  if (!src) return shape_error("non-null weight pointer", "null");
  BN_TRY(m->alloc(dst, n));
  BN_CUDA(cudaMemcpyAsync(*dst, src, n * sizeof(T), cudaMemcpyHostToDevice, m->ctx->stream));
  return BITNET_OK;
}

int check_scale(float s, const char* what) {
  if (!(s > 0.0f) || !std::isfinite(s)) return quant_error(std::string(what) + " scale must be finite and > 0");
  return BITNET_OK;
}

int model_wait(bitnet_cuda_model* m, cudaStream_t st);

// Ensure sequence `seq` has pages for positions [0, end); update the device table.
int kv_reserve(bitnet_cuda_kv* kv, uint32_t seq, size_t end, cudaStream_t st) {
  if (end > kv->capacity())
    return shape_error("position < kv capacity (" + sz(kv->capacity()) + ")", "position = " + sz(end - 1));
  auto& pages = kv->seq_pages[seq];
  size_t need = (end + kPage - 1) / kPage;
  if (need <= pages.size()) return BITNET_OK;
  if (need - pages.size() > kv->free_pages.size()) return backend_error("paged KV cache is out of free pages");
  size_t first = pages.size();
  while (pages.size() < need) {
    int32_t p = kv->free_pages.back();
    kv->free_pages.pop_back();
    kv->h_table[(size_t)seq * kv->g.max_pages_per_seq + pages.size()] = p;
    pages.push_back(p);
  }
  int32_t* src = &kv->h_table[(size_t)seq * kv->g.max_pages_per_seq + first];
  BN_CUDA(cudaMemcpyAsync(kv->d_table + (size_t)seq * kv->g.max_pages_per_seq + first, src,
                          (need - first) * sizeof(int32_t), cudaMemcpyHostToDevice, st));
  // the host table entries stay valid until the pages are freed; the copy
  // must finish before they can change
  return model_wait(kv->model, st);
}

// Attention policy: the reference-order kernel serves decode steps and
// short prefills (each query token streams its own context); long packed
// prefills use the split-context kernel.
constexpr int kExactMaxTokens = 1024;
constexpr int kSmallStepTokens = 16;
constexpr size_t kExactMaxSmem = 200 * 1024;

// Kernel choice (bitnet_cuda_model_set_numerics):
//  - attention feeds the next int8 quantisation, so outside FAST mode it
//    always runs in the reference's operation order;
//  - the lm_head feeds nothing back: AUTO runs the tensor-core kernel for
//    steps with more than kSmallStepTokens output rows.
bool use_exact_attention(const bitnet_cuda_model* m, int T) {
  return m->numerics != BITNET_NUMERICS_FAST && T <= kExactMaxTokens && m->nh / m->nkv <= 8;
}
bool use_mma_attention(const bitnet_cuda_model* m, const bitnet_cuda_kv* kv, int T) {
  return !use_exact_attention(m, T) && m->mma_attn_ok && flash_decode_mma_supported(kv->g, m->nh);
}
bool use_exact2_attention(const bitnet_cuda_model* m, const bitnet_cuda_kv* kv, int max_ctx) {
  return m->exact2_ok && exact2_supported(kv->g, m->nh) && exact2_smem(max_ctx) <= m->exact2_smem_max;
}
bool use_x4_attention(const bitnet_cuda_model* m, const bitnet_cuda_kv* kv, int max_ctx) {
  return m->x4_ok && kv->tmap_ok && attn_x4_supported(kv->g, m->nh) && attn_x4_smem(max_ctx) <= m->x4_smem_max;
}
bool use_exact3_attention(const bitnet_cuda_model* m, const bitnet_cuda_kv* kv, int max_ctx) {
  return m->exact3_ok && kv->tmap_ok && exact3_supported(kv->g, m->nh) && exact3_smem(max_ctx) <= m->exact3_smem_max;
}
// The one-token step runs as decode1_kernel when the model and cache fit it
// (not tensor-parallel, bf16 cache with its tensor map, head_dim 128, GQA
// group 1/2/4/8) outside FAST numerics, and d1_prepare planned its shared
// memory for this context capacity.
constexpr int kD1CapStep = 256;
bool decode1_eligible(const bitnet_cuda_model* m, const bitnet_cuda_kv* kv, int T) {
  return T == 1 && m->d1_enabled && !m->tp && m->numerics != BITNET_NUMERICS_FAST && m->d1_layers && m->d1_limit &&
         kv->tmap_ok && decode1_supported(m->nh, m->nkv, m->H, m->F, kv->g);
}
bool use_decode1(const bitnet_cuda_model* m, const bitnet_cuda_kv* kv, int T, int max_ctx) {
  return decode1_eligible(m, kv, T) && m->d1_cap == (int)round_up((size_t)max_ctx, kD1CapStep) && m->d1_smem > 0;
}
// Plans (and caches) the kernel's shared memory for contexts up to max_ctx;
// outside graph capture.
void d1_prepare(bitnet_cuda_model* m, const bitnet_cuda_kv* kv, int T, int max_ctx) {
  if (!decode1_eligible(m, kv, T)) return;
  const int cap = (int)round_up((size_t)max_ctx, kD1CapStep);
  if (cap == m->d1_cap) return;
  D1Params P;
  P.L = m->L;
  P.H = m->H;
  P.nh = m->nh;
  P.nkv = m->nkv;
  P.F = m->F;
  P.V = m->V;
  P.eps = m->cfg.rms_norm_eps;
  size_t smem = decode1_plan(&P, m->d1_sms, cap, m->d1_limit);
  if (smem && !decode1_fits(P.hpc, m->d1_sms, smem)) smem = 0;
  m->d1_cap = cap;
  m->d1_smem = smem;
  m->d1_plan = P;
}
void launch_decode1_step(bitnet_cuda_model* m, bitnet_cuda_kv* kv, cudaStream_t st) {
  D1Params P = m->d1_plan;
  P.layers = m->d1_layers;
  P.embed = m->embed;
  P.token = m->tokens;
  P.tok_pos = m->tok_pos;
  P.tok_seq = m->tok_seq;
  P.page_table = kv->d_table;
  P.g = kv->g;
  P.rope_cos = m->rope_cos;
  P.rope_sin = m->rope_sin;
  P.et = m->ctx->exp_table;
  P.h = m->h;
  P.qkv = m->qkv;
  P.attn = m->attn;
  P.gu = m->gu;
  P.status = m->status;
  P.sync = m->d1_sync;
  P.final_norm = m->final_norm;
  P.hn = m->hn;
  cudaMemsetAsync(m->d1_sync, 0, decode1_sync_bytes(), st);
  launch_decode1(P, kv->tmap, m->d1_sms, m->d1_smem, st);
}
bool use_fast_lm_head(const bitnet_cuda_model* m, int n_out) {
  if (!m->lm_mma_ok || m->numerics == BITNET_NUMERICS_EXACT) return false;
  return m->numerics == BITNET_NUMERICS_FAST || n_out > kSmallStepTokens;
}
bool exact_scores_in_smem(const bitnet_cuda_model* m, int max_ctx) {
  return m->exact_smem_ok && paged_attention_exact_smem(m->nh, m->nkv, m->hd, max_ctx) <= m->exact_smem_max;
}

// Kernel classes for the per-step timing of device-resident decode graphs.
enum KClass { kAttn = 0, kMatmul = 1, kNormQuant = 2, kRopeKv = 3, kLmHead = 4, kOther = 5, kLayers = 6, kClasses = 7 };

// Records an event pair around `launch` when the graph being captured is timed.
template <class F>
void timed(bitnet_cuda_model* m, int cls, cudaStream_t st, F launch) {
  if (!m->marks) {
    launch();
    return;
  }
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  // external records become event-record nodes of the captured graph
  cudaEventRecordWithFlags(a, st, cudaEventRecordExternal);
  launch();
  cudaEventRecordWithFlags(b, st, cudaEventRecordExternal);
  m->marks->emplace_back(cls, a, b);
}

void nccl_note(bitnet_cuda_model* m, ncclResult_t r) {
  // a nonblocking communicator may still be enqueueing the call
  if (r == ncclInProgress) {
    const auto t0 = std::chrono::steady_clock::now();
    do {
      m->nc->comm_get_async_error(m->comm, &r);
      if (r != ncclInProgress) break;
      std::this_thread::yield();
    } while (std::chrono::steady_clock::now() - t0 < std::chrono::milliseconds(m->tp_timeout_ms));
  }
  if (r != ncclSuccess && m->nccl_rc == ncclSuccess) m->nccl_rc = r;
}

// Aborts the communicator of a tensor-parallel model: its pending
// collectives return, and every later call on the model fails.
void tp_abort(bitnet_cuda_model* m) {
  if (m->comm) m->nc->comm_abort(m->comm);
  m->comm = nullptr;
  m->tp_dead = true;
}

// Waits for st.  For a tensor-parallel model the wait also watches the
// communicator: an asynchronous NCCL error, or no completion within
// tp_timeout_ms (a peer that left or stopped), aborts the communicator.
int model_wait(bitnet_cuda_model* m, cudaStream_t st) {
  if (!m->tp) {
    BN_CUDA(cudaStreamSynchronize(st));
    return BITNET_OK;
  }
  if (m->tp_dead) return backend_error("the tensor-parallel communicator was aborted after an earlier failure");
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t e = cudaStreamQuery(st);
    if (e == cudaSuccess) return BITNET_OK;
    if (e != cudaErrorNotReady) return cuda_error(e, "cudaStreamQuery");
    ncclResult_t ae = ncclSuccess;
    m->nc->comm_get_async_error(m->comm, &ae);
    const bool late = std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(m->tp_timeout_ms);
    if ((ae != ncclSuccess && ae != ncclInProgress) || late) {
      std::string why = late ? "no completion within " + std::to_string(m->tp_timeout_ms) + " ms"
                             : std::string("NCCL error: ") + m->nc->error_string(ae);
      tp_abort(m);
      // the aborted collectives should now return; the wait for them is
      // bounded too, since a collective that does not observe the abort
      // would keep the stream busy until the process exits
      const auto t1 = std::chrono::steady_clock::now();
      while (cudaStreamQuery(st) == cudaErrorNotReady &&
             std::chrono::steady_clock::now() - t1 < std::chrono::milliseconds(m->tp_timeout_ms))
        std::this_thread::sleep_for(std::chrono::microseconds(200));
      const bool idle = cudaStreamQuery(st) != cudaErrorNotReady;
      cudaGetLastError();
      return backend_error("tensor-parallel step failed (" + why + "); communicator aborted" +
                           (idle ? std::string() : std::string("; its stream is still busy: end the process")));
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// Tensor parallelism: all-gather this rank's [T][C] chunk (already in its
// slot of tp_gath) and lay the result out as full rows [T][world*C] in tp_full.
void tp_gather_rows(bitnet_cuda_model* m, int T, int C, cudaStream_t st) {
  const size_t cnt = (size_t)T * C;
  nccl_note(m, m->nc->all_gather(m->tp_gath + (size_t)m->tp_rank * cnt, m->tp_gath, cnt, ncclFloat32, m->comm, st));
  launch_tp_unchunk(m->tp_gath, m->tp_world, T, C, m->tp_full, st);
}

// Tensor parallelism, row-split projection (o_proj, down_proj): this rank's K
// input columns of W against its slice of the quantised full rows, the int32
// accumulators summed over ranks (exact), then the reference epilogue with
// the residual add into h on every rank.
void tp_row_split(bitnet_cuda_model* m, const uint32_t* W, int K, float ws, int T, cudaStream_t st) {
  const int H = m->H;
  const int8_t* xs = m->xq + (size_t)m->tp_rank * K;
  launch_row_sum(xs, m->ldq, T, K, m->tp_rowsum, st);
  Segments s;
  s.end[0] = s.end[1] = s.end[2] = H;
  s.scale[0] = s.scale[1] = s.scale[2] = ws;
  launch_ternary_matmul(W, H, K, xs, m->ldq, m->amax, m->tp_rowsum, T, s, Epi::Store, m->qrot, H, m->tp_acc, st,
                        m->status);
  nccl_note(m, m->nc->all_reduce(m->tp_acc, m->tp_acc, (size_t)T * H, ncclInt32, ncclSum, m->comm, st));
  launch_acc_epilogue(m->tp_acc, T, H, ws, m->amax, Epi::Residual, m->h, H, st);
}

// Run the transformer over T tokens whose metadata (tokens, tok_pos, tok_seq,
// last_row) is already on the device.  n_out rows of final hidden state
// (selected by last_row) go through final norm, lm_head and argmax.
void run_forward(bitnet_cuda_model* m, bitnet_cuda_kv* kv, int T, int n_out, int max_ctx, cudaStream_t st) {
  const int H = m->H, qd = m->qd, kvd = m->kvd, F = m->F;
  const float eps = m->cfg.rms_norm_eps;
  const int nqkv = qd + 2 * kvd;
  const bool fused = use_decode1(m, kv, T, max_ctx);
  if (fused) timed(m, kLayers, st, [&] { launch_decode1_step(m, kv, st); });
  else
    timed(m, kOther, st, [&] {
      launch_embed(m->embed, m->tokens, T, H, m->h, m->status, m->V, st);
    });
  for (int l = 0; l < (fused ? 0 : m->L); ++l) {
    const Layer& Lw = m->layers[l];
    // attention block
    timed(m, kNormQuant, st, [&] {
      launch_norm_quant(m->h, nullptr, H, Lw.attn_norm, H, eps, m->xq, m->ldq, m->amax, m->rowsum, m->status, T, st);
    });
    Segments sqkv;
    sqkv.n = 3;
    sqkv.end[0] = qd;
    sqkv.end[1] = qd + kvd;
    sqkv.end[2] = nqkv;
    sqkv.scale[0] = Lw.sq;
    sqkv.scale[1] = Lw.sk;
    sqkv.scale[2] = Lw.sv;
    timed(m, kMatmul, st, [&] {
      launch_ternary_matmul(Lw.wqkv, nqkv, H, m->xq, m->ldq, m->amax, m->rowsum, T, sqkv, Epi::Store, m->qkv, nqkv,
                            nullptr, st, m->status);
    });
    timed(m, kRopeKv, st, [&] {
      launch_rope_kv_store(m->qkv, nqkv, T, m->nh, m->nkv, m->hd, m->rope_cos, m->rope_sin, m->tok_pos, m->tok_seq,
                           kv->d_table, kv->g, l, m->qrot, st);
    });
    // a tensor-parallel rank writes its heads straight into its all-gather slot
    float* attn_out = m->tp ? m->tp_gath + (size_t)m->tp_rank * T * qd : m->attn;
    timed(m, kAttn, st, [&] {
      if (use_exact_attention(m, T) && use_x4_attention(m, kv, max_ctx))
        launch_attn_x4(m->qrot, T, m->nh, m->tok_pos, m->tok_seq, m->order, kv->d_table, kv->g, kv->tmap, l, max_ctx,
                       attn_out, m->partial.as<float>(), m->ctx->exp_table, m->status, st);
      else if (use_exact_attention(m, T) && use_exact3_attention(m, kv, max_ctx))
        launch_paged_attention_exact3(m->qrot, T, m->nh, m->tok_pos, m->tok_seq, kv->d_table, kv->g, kv->tmap, l,
                                      max_ctx, attn_out, m->ctx->exp_table, m->status, st);
      else if (use_exact_attention(m, T) && use_exact2_attention(m, kv, max_ctx))
        launch_paged_attention_exact2(m->qrot, T, m->nh, m->tok_pos, m->tok_seq, kv->d_table, kv->g, l, max_ctx,
                                      attn_out, m->ctx->exp_table, st);
      else if (use_exact_attention(m, T))
        launch_paged_attention_exact(m->qrot, T, m->nh, m->tok_pos, m->tok_seq, kv->d_table, kv->g, l, max_ctx,
                                     attn_out, m->partial.as<float>(), exact_scores_in_smem(m, max_ctx),
                                     m->ctx->exp_table, st);
      else if (use_mma_attention(m, kv, T))
        launch_flash_decode_mma(m->qrot, T, m->nh, m->tok_pos, m->tok_seq, kv->d_table, kv->g, l, max_ctx, attn_out,
                                m->partial.as<float>(), st);
      else
        launch_paged_attention(m->qrot, T, m->nh, m->tok_pos, m->tok_seq, kv->d_table, kv->g, l, max_ctx, attn_out,
                               m->partial.as<float>(), m->partial.cap / 4, st);
    });
    if (m->tp) {
      timed(m, kOther, st, [&] { tp_gather_rows(m, T, qd, st); });
      timed(m, kNormQuant, st, [&] {
        launch_norm_quant(m->tp_full, nullptr, m->qd_all, Lw.attn_sub_norm, m->qd_all, eps, m->xq, m->ldq, m->amax,
                          m->rowsum, m->status, T, st);
      });
      timed(m, kMatmul, st, [&] { tp_row_split(m, Lw.wo, qd, Lw.so, T, st); });
    } else {
      timed(m, kNormQuant, st, [&] {
        launch_norm_quant(m->attn, nullptr, qd, Lw.attn_sub_norm, qd, eps, m->xq, m->ldq, m->amax, m->rowsum,
                          m->status, T, st);
      });
      Segments so;
      so.end[0] = so.end[1] = so.end[2] = H;
      so.scale[0] = so.scale[1] = so.scale[2] = Lw.so;
      timed(m, kMatmul, st, [&] {
        launch_ternary_matmul(Lw.wo, H, qd, m->xq, m->ldq, m->amax, m->rowsum, T, so, Epi::Residual, m->h, H, nullptr,
                              st, m->status);
      });
    }
    // FFN block
    timed(m, kNormQuant, st, [&] {
      launch_norm_quant(m->h, nullptr, H, Lw.ffn_norm, H, eps, m->xq, m->ldq, m->amax, m->rowsum, m->status, T, st);
    });
    Segments sgu;
    sgu.n = 2;
    sgu.end[0] = F;
    sgu.end[1] = sgu.end[2] = 2 * F;
    sgu.scale[0] = Lw.sg;
    sgu.scale[1] = sgu.scale[2] = Lw.su;
    timed(m, kMatmul, st, [&] {
      launch_ternary_matmul(Lw.wgu, 2 * F, H, m->xq, m->ldq, m->amax, m->rowsum, T, sgu, Epi::Store, m->gu, 2 * F,
                            nullptr, st, m->status);
    });
    if (m->tp) {
      timed(m, kOther, st, [&] {
        launch_tp_gate_rows(m->gu, T, F, m->tp_gath + (size_t)m->tp_rank * T * F, st);
        tp_gather_rows(m, T, F, st);
      });
      timed(m, kNormQuant, st, [&] {
        launch_norm_quant(m->tp_full, nullptr, m->F_all, Lw.ffn_sub_norm, m->F_all, eps, m->xq, m->ldq, m->amax,
                          m->rowsum, m->status, T, st);
      });
      timed(m, kMatmul, st, [&] { tp_row_split(m, Lw.wdown, F, Lw.sd, T, st); });
    } else {
      timed(m, kNormQuant, st, [&] {
        launch_norm_quant(m->gu, m->gu + F, 2 * F, Lw.ffn_sub_norm, F, eps, m->xq, m->ldq, m->amax, m->rowsum,
                          m->status, T, st);
      });
      Segments sd;
      sd.end[0] = sd.end[1] = sd.end[2] = H;
      sd.scale[0] = sd.scale[1] = sd.scale[2] = Lw.sd;
      timed(m, kMatmul, st, [&] {
        launch_ternary_matmul(Lw.wdown, H, F, m->xq, m->ldq, m->amax, m->rowsum, T, sd, Epi::Residual, m->h, H,
                              nullptr, st, m->status);
      });
    }
  }
  // final norm on the selected rows (the fused layer kernel writes it itself), lm_head, greedy argmax
  if (!fused) {
    timed(m, kOther, st, [&] {
      launch_gather_rows(m->h, H, m->last_row, n_out, m->qrot, st);
    });
    timed(m, kOther, st, [&] {
      launch_rms_norm(m->qrot, H, m->final_norm, H, eps, m->hn, H, n_out, st);
    });
  }
  if (n_out == 1 && m->lm1_ok && !m->tp && !use_fast_lm_head(m, n_out)) {
    timed(m, kLmHead, st, [&] {
      launch_lm_head_m1(m->lm1_tmap, m->hn, m->lm_scales, m->Vloc, H, m->logits, m->lm1_part, m->next, m->status,
                        st);
    });
    return;
  }
  // this rank's vocabulary slice (the whole vocabulary without tensor parallelism)
  timed(m, kLmHead, st, [&] {
    if (use_fast_lm_head(m, n_out))
      launch_lm_head_mma(m->hn, n_out, m->Vloc, H, m->lm_i8, m->lm_scales, m->a3, m->logits, m->Vs, st, m->status);
    else
      launch_lm_head(m->lm_i8, LmW::I8, m->lm_scales, m->hn, H, n_out, m->Vloc, H, m->logits, m->Vs, st);
  });
  timed(m, kOther, st, [&] {
    if (m->tp) {
      // each rank's best (value, index), all-gathered, the best of those
      launch_argmax_pairs(m->logits, m->Vs, n_out, m->Vloc, (uint32_t)m->v0, m->tp_pairs, st);
      nccl_note(m, m->nc->all_gather(m->tp_pairs, m->tp_pairs_all, (size_t)n_out * 2, ncclUint32, m->comm, st));
      launch_argmax_combine(m->tp_pairs_all, m->tp_world, n_out, m->next, st);
    } else {
      launch_argmax(m->logits, m->V, n_out, m->V, m->next, st);
    }
  });
}

// Full logits rows [n_out][V] of the last forward: the model's own buffer, or
// for a tensor-parallel model the all-gather of every rank's slice (a
// collective: every rank must ask for logits in the same call).  *ld gets
// the row stride.
const float* full_logits(bitnet_cuda_model* m, int n_out, size_t* ld, cudaStream_t st) {
  if (!m->tp) {
    *ld = (size_t)m->V;
    return m->logits;
  }
  const size_t cnt = (size_t)n_out * m->Vs;
  nccl_note(m, m->nc->all_gather(m->logits, m->tp_lgath, cnt, ncclFloat32, m->comm, st));
  launch_tp_unchunk(m->tp_lgath, m->tp_world, n_out, m->Vs, m->tp_logits, st);
  *ld = (size_t)m->tp_world * m->Vs;
  return m->tp_logits;
}

// Copies n_out rows of full logits to dst (row length V).
int copy_logits(bitnet_cuda_model* m, int n_out, float* dst, cudaMemcpyKind kind, cudaStream_t st) {
  size_t ld = 0;
  const float* src = full_logits(m, n_out, &ld, st);
  BN_CUDA(cudaMemcpy2DAsync(dst, (size_t)m->V * 4, src, ld * 4, (size_t)m->V * 4, (size_t)n_out, kind, st));
  return BITNET_OK;
}

// Name of the attention kernel run_forward launches for T tokens (same tests).
const char* attention_kernel_name(const bitnet_cuda_model* m, const bitnet_cuda_kv* kv, int T, int max_ctx) {
  if (use_decode1(m, kv, T, max_ctx)) return "decode1_kernel";
  if (use_exact_attention(m, T) && use_x4_attention(m, kv, max_ctx)) return "attn_qk_softmax_kernel+attn_pv_kernel";
  if (use_exact_attention(m, T) && use_exact3_attention(m, kv, max_ctx)) return "paged_attention_exact3_kernel";
  if (use_exact_attention(m, T) && use_exact2_attention(m, kv, max_ctx)) return "paged_attention_exact2_kernel";
  if (use_exact_attention(m, T)) return "paged_attention_exact_kernel";
  if (use_mma_attention(m, kv, T)) return "flash_decode_mma_kernel";
  return "paged_attention_kernel";
}

// Reads (and clears) the device status word; synchronises the stream.
int check_status(bitnet_cuda_model* m) {
  int32_t s = 0;
  BN_CUDA(cudaMemcpyAsync(&s, m->status, 4, cudaMemcpyDeviceToHost, m->ctx->stream));
  BN_TRY(model_wait(m, m->ctx->stream));
  if (s) {
    BN_CUDA(cudaMemsetAsync(m->status, 0, 4, m->ctx->stream));
    BN_CUDA(cudaStreamSynchronize(m->ctx->stream));
  }
  if (m->nccl_rc != ncclSuccess) {
    ncclResult_t r = m->nccl_rc;
    m->nccl_rc = ncclSuccess;
    return backend_error(std::string("NCCL collective failed: ") + m->nc->error_string(r));
  }
  if (s & kStatusWaitTimeout) return backend_error("a device-side wait timed out (attention pipeline)");
  if (s & kStatusBadContext) return backend_error("a token's context exceeds the attention kernel's capacity");
  if (s & kStatusBadToken) return shape_error("token id < vocab_size", "out-of-range token id");
  if (s & kStatusNonFinite) return quant_error("non-finite activation value in the forward pass");
  return BITNET_OK;
}

// Host-side bookkeeping for a batch of (seq, n_tokens) appended at each
// sequence's current length: reserve pages, fill the pinned metadata.
int prepare_batch(bitnet_cuda_model* m, bitnet_cuda_kv* kv, size_t n_seqs, const uint32_t* seq_ids,
                  const uint32_t* counts, int* T_out, int* max_ctx_out, cudaStream_t st) {
  size_t T = 0;
  for (size_t i = 0; i < n_seqs; ++i) {
    if (seq_ids[i] >= (uint32_t)kv->max_seqs)
      return shape_error("seq id < max_seqs (" + sz(kv->max_seqs) + ")", "seq id " + sz(seq_ids[i]));
    for (size_t j = 0; j < i; ++j)
      if (seq_ids[j] == seq_ids[i]) return shape_error("distinct sequence ids in one batch", "duplicate " + sz(seq_ids[i]));
    if (counts[i] == 0) return shape_error("tokens.len() > 0", "0 tokens for a sequence");
    T += counts[i];
  }
  if (T > (size_t)m->Tmax) return shape_error("batch tokens <= " + sz(m->Tmax), sz(T));
  int max_ctx = 1;
  size_t t = 0;
  for (size_t i = 0; i < n_seqs; ++i) {
    uint32_t s = seq_ids[i];
    size_t start = kv->seq_len[s], end = start + counts[i];
    if (end > m->cfg.max_position_embeddings)
      return shape_error("sequence position <= max_position_embeddings " + sz(m->cfg.max_position_embeddings),
                         "position " + sz(end));
    BN_TRY(kv_reserve(kv, s, end, st));
    for (size_t j = 0; j < counts[i]; ++j, ++t) {
      m->h_meta[t] = (int32_t)(start + j);
      m->h_meta[m->Tmax + t] = (int32_t)s;
    }
    m->h_meta[2 * m->Tmax + i] = (int32_t)(t - 1);
    max_ctx = std::max<int>(max_ctx, (int)end);
  }
  // attention CTAs start in this order: the longest contexts first
  int32_t* order = m->h_meta + 3 * m->Tmax;
  for (size_t i = 0; i < T; ++i) order[i] = (int32_t)i;
  std::stable_sort(order, order + T, [&](int32_t a, int32_t b) { return m->h_meta[a] > m->h_meta[b]; });
  *T_out = (int)T;
  *max_ctx_out = max_ctx;
  return BITNET_OK;
}

int upload_meta(bitnet_cuda_model* m, int T, int n_out, cudaStream_t st) {
  BN_CUDA(cudaMemcpyAsync(m->tok_pos, m->h_meta, T * 4, cudaMemcpyHostToDevice, st));
  BN_CUDA(cudaMemcpyAsync(m->tok_seq, m->h_meta + m->Tmax, T * 4, cudaMemcpyHostToDevice, st));
  BN_CUDA(cudaMemcpyAsync(m->last_row, m->h_meta + 2 * m->Tmax, n_out * 4, cudaMemcpyHostToDevice, st));
  BN_CUDA(cudaMemcpyAsync(m->order, m->h_meta + 3 * m->Tmax, T * 4, cudaMemcpyHostToDevice, st));
  return BITNET_OK;
}

void destroy_graph(bitnet_cuda_model::Graph& g) {
  cudaGraphExecDestroy(g.exec);
  for (auto& t : g.marks) {
    cudaEventDestroy(std::get<1>(t));
    cudaEventDestroy(std::get<2>(t));
  }
}

void drop_graphs(bitnet_cuda_model* m) {
  for (auto& kvp : m->graphs) destroy_graph(kvp.second);
  m->graphs.clear();
  m->last_timed = nullptr;
}

int ensure_partial(bitnet_cuda_model* m, const bitnet_cuda_kv* kv, int T, int max_ctx) {
  d1_prepare(m, kv, T, max_ctx);
  size_t floats = use_exact_attention(m, T)
                      ? (use_x4_attention(m, kv, max_ctx) ? attn_x4_scratch_floats(T, m->nkv, max_ctx)
                         : (use_exact3_attention(m, kv, max_ctx) || use_exact2_attention(m, kv, max_ctx) ||
                          exact_scores_in_smem(m, max_ctx))
                             ? 0
                             : (size_t)T * m->nh * max_ctx)
                      : (use_mma_attention(m, kv, T) ? flash_decode_mma_partial_floats(T, m->nh, max_ctx)
                                                     : paged_attention_partial_floats(T, m->nh, m->hd, max_ctx));
  size_t bytes = std::max<size_t>(floats, 16) * sizeof(float);
  if (bytes <= m->partial.cap) return BITNET_OK;
  // captured graphs hold the old address
  BN_TRY(model_wait(m, m->ctx->stream));
  drop_graphs(m);
  return m->partial.ensure(bytes);
}

}  // namespace

static void model_release(bitnet_cuda_model* m) {
  if (m->refs.fetch_sub(1) != 1) return;
  bitnet_cuda_ctx* c = m->ctx;
  cudaSetDevice(c->device);
  if (m->tp && model_wait(m, c->stream) != BITNET_OK) cudaGetLastError();
  if (m->tp_dead && cudaStreamQuery(c->stream) == cudaErrorNotReady) {
    // an aborted collective never returned: freeing would wait for it
    // forever, so the device memory stays with the process, which must end
    cudaGetLastError();
    delete m;
    return;
  }
  cudaStreamSynchronize(c->stream);
  // graphs that hold NCCL calls go before their communicator
  drop_graphs(m);
  if (m->comm) m->nc->comm_destroy(m->comm);
  for (void* p : m->allocs) cudaFree(p);
  if (m->h_meta) cudaFreeHost(m->h_meta);
  if (m->h_tokens) cudaFreeHost(m->h_tokens);
  m->partial.release();
  delete m;
  ctx_release(c);
}

namespace {

// Uploads the share of rank `rank` of `world`; without an NCCL id the whole
// model on one device with no collectives.
int model_create_impl(bitnet_cuda_ctx* ctx, const bitnet_cuda_config* cfg, const bitnet_cuda_weights* w,
                      uint32_t max_batch_tokens, uint32_t rank, uint32_t world, const uint8_t* nccl_id,
                      bitnet_cuda_model** out) {
  if (!out || !cfg || !w || !ctx) return shape_error("non-null arguments", "null");
  *out = nullptr;
  BN_TRY(validate_config(*cfg));
  if (max_batch_tokens == 0) return shape_error("max_batch_tokens > 0", "0");
  if (!w->layers) return shape_error("non-null layers", "null");
  const bool tp = nccl_id != nullptr;
  const NcclApi* nc = nullptr;
  if (tp) {
    const uint32_t nh = cfg->num_attention_heads, nkv = cfg->num_key_value_heads;
    const size_t qd_all = (size_t)(cfg->hidden_size / nh) * nh;
    if (world == 0 || rank >= world) return config_error("tensor-parallel rank must be < world (world > 0)");
    if (nh % world != 0 || nkv % world != 0)
      return config_error("num_attention_heads (" + sz(nh) + ") and num_key_value_heads (" + sz(nkv) +
                          ") must be divisible by the tensor-parallel world (" + sz(world) + ")");
    if (cfg->intermediate_size % world != 0 || (qd_all / world) % 64 != 0 || (cfg->intermediate_size / world) % 64 != 0)
      return config_error("per-rank attention width (" + sz(qd_all / world) + ") and intermediate slice (" +
                          sz(cfg->intermediate_size / world) + ") must be multiples of 64");
    std::string why;
    nc = nccl_api(&why);
    if (!nc) return backend_error("tensor parallelism needs NCCL: " + why);
  }
  std::lock_guard<std::mutex> lk(ctx->mu);
  cudaSetDevice(ctx->device);
  auto* m = new bitnet_cuda_model();
  m->ctx = ctx;
  ctx_retain(ctx);
  m->cfg = *cfg;
  const int G = tp ? (int)world : 1, rk = tp ? (int)rank : 0;
  m->tp = tp;
  m->tp_rank = rk;
  m->tp_world = G;
  m->nc = nc;
  m->H = (int)cfg->hidden_size;
  m->hd = m->H / (int)cfg->num_attention_heads;
  m->nh = (int)cfg->num_attention_heads / G;
  m->nkv = (int)cfg->num_key_value_heads / G;
  m->qd = m->nh * m->hd;
  m->kvd = m->nkv * m->hd;
  m->qd_all = m->qd * G;
  m->F_all = (int)cfg->intermediate_size;
  m->F = m->F_all / G;
  m->V = (int)cfg->vocab_size;
  m->L = (int)cfg->num_hidden_layers;
  m->Tmax = (int)max_batch_tokens;
  m->ldq = (int)std::max({padded_cols(m->H), padded_cols(m->qd_all), padded_cols(m->F_all)});
  auto fail = [&](int rc) {
    model_release(m);
    return rc;
  };
  int rc;
  if (tp) {
    // collective: every rank rendezvouses here before any upload
    ncclUniqueId id;
    std::memcpy(&id, nccl_id, sizeof id);
    // nonblocking init, bounded: a peer that never joins ends it with an error
    if (const char* t = std::getenv("BITNET_TP_TIMEOUT_MS")) m->tp_timeout_ms = std::max(1, std::atoi(t));
    ncclConfig_t nc_cfg = NCCL_CONFIG_INITIALIZER;
    nc_cfg.blocking = 0;
    ncclResult_t r = nc->comm_init_rank_config(&m->comm, G, id, rk, &nc_cfg);
    const auto t0 = std::chrono::steady_clock::now();
    while (r == ncclInProgress && m->comm) {
      if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(m->tp_timeout_ms)) break;
      std::this_thread::sleep_for(std::chrono::milliseconds(1));
      nc->comm_get_async_error(m->comm, &r);
    }
    if (r != ncclSuccess) {
      const std::string why = r == ncclInProgress ? "peers did not join within " + std::to_string(m->tp_timeout_ms) +
                                                        " ms"
                                                  : std::string(nc->error_string(r));
      if (m->comm) nc->comm_abort(m->comm);
      m->comm = nullptr;
      return fail(backend_error("ncclCommInitRankConfig: " + why));
    }
  }
  DevBuf tmp;
  const int H = m->H, qd = m->qd, kvd = m->kvd, F = m->F;
  const size_t pcH = ((size_t)H + 3) / 4;
  // input columns [rk*k, (rk+1)*k) of a [H][K] reference-format tensor, k % 4 == 0
  std::vector<uint8_t> cols;
  auto col_slice = [&](const uint8_t* src, int K, int k) -> const uint8_t* {
    if (!src || G == 1) return src;
    const size_t pc = ((size_t)K + 3) / 4, pk = (size_t)k / 4;
    cols.resize((size_t)H * pk);
    for (int i = 0; i < H; ++i) std::memcpy(&cols[(size_t)i * pk], src + (size_t)i * pc + (size_t)rk * pk, pk);
    return cols.data();
  };
  auto row_slice = [&](const uint8_t* src, int rows) -> const uint8_t* {
    return src ? src + (size_t)rk * rows * pcH : src;
  };
  for (int l = 0; l < m->L; ++l) {
    const bitnet_cuda_layer_weights& s = w->layers[l];
    Layer Lw;
    Lw.sq = s.q_scale;
    Lw.sk = s.k_scale;
    Lw.sv = s.v_scale;
    Lw.so = s.o_scale;
    Lw.sg = s.gate_scale;
    Lw.su = s.up_scale;
    Lw.sd = s.down_scale;
    for (float sc : {s.q_scale, s.k_scale, s.v_scale, s.o_scale, s.gate_scale, s.up_scale, s.down_scale})
      if ((rc = check_scale(sc, "projection"))) return fail(rc);
    if ((rc = m->alloc(&Lw.wqkv, (size_t)(qd + 2 * kvd) * words_per_row(H)))) return fail(rc);
    if ((rc = m->alloc(&Lw.wo, (size_t)H * words_per_row(qd)))) return fail(rc);
    if ((rc = m->alloc(&Lw.wgu, (size_t)2 * F * words_per_row(H)))) return fail(rc);
    if ((rc = m->alloc(&Lw.wdown, (size_t)H * words_per_row(F)))) return fail(rc);
    // column-split projections keep this rank's output rows; row-split ones
    // (o, down) its input columns; the sub-norms act on full rows
    if ((rc = put_ternary(m, row_slice(s.q_proj, qd), qd, H, Lw.wqkv, 0, tmp))) return fail(rc);
    if ((rc = put_ternary(m, row_slice(s.k_proj, kvd), kvd, H, Lw.wqkv, qd, tmp))) return fail(rc);
    if ((rc = put_ternary(m, row_slice(s.v_proj, kvd), kvd, H, Lw.wqkv, qd + kvd, tmp))) return fail(rc);
    if ((rc = put_ternary(m, col_slice(s.o_proj, m->qd_all, qd), H, qd, Lw.wo, 0, tmp))) return fail(rc);
    if ((rc = put_ternary(m, row_slice(s.gate_proj, F), F, H, Lw.wgu, 0, tmp))) return fail(rc);
    if ((rc = put_ternary(m, row_slice(s.up_proj, F), F, H, Lw.wgu, F, tmp))) return fail(rc);
    if ((rc = put_ternary(m, col_slice(s.down_proj, m->F_all, F), H, F, Lw.wdown, 0, tmp))) return fail(rc);
    if ((rc = put(m, &Lw.attn_norm, s.attention_norm, H))) return fail(rc);
    if ((rc = put(m, &Lw.attn_sub_norm, s.attn_sub_norm, m->qd_all))) return fail(rc);
    if ((rc = put(m, &Lw.ffn_norm, s.ffn_norm, H))) return fail(rc);
    if ((rc = put(m, &Lw.ffn_sub_norm, s.ffn_sub_norm, m->F_all))) return fail(rc);
    m->layers.push_back(Lw);
  }
  const size_t V = m->V;
  if ((rc = put(m, &m->embed, w->embed_tokens, V * H))) return fail(rc);
  // lm_head rows: a tensor-parallel rank keeps a slice of 128-row multiples
  m->Vs = tp ? (int)round_up(ceil_div(V, (size_t)G), 128) : (int)V;
  m->v0 = tp ? std::min<int>(rk * m->Vs, (int)V) : 0;
  m->Vloc = tp ? std::min<int>(m->Vs, (int)V - m->v0) : (int)V;
  if (m->Vloc <= 0) return fail(config_error("vocab_size is too small for the tensor-parallel world"));
  if (!w->lm_head_i8 || !w->lm_head_scales) return fail(shape_error("non-null lm_head table and scales", "null"));
  if ((rc = put(m, &m->lm_i8, w->lm_head_i8 + (size_t)m->v0 * H, (size_t)m->Vloc * H))) return fail(rc);
  if ((rc = put(m, &m->lm_scales, w->lm_head_scales + m->v0, (size_t)m->Vloc))) return fail(rc);
  if ((rc = put(m, &m->final_norm, w->final_norm, H))) return fail(rc);
  if (!tp && lm_head_m1_supported(H, m->Vloc) && lm_head_m1_prepare(H) == 0 &&
      lm_head_m1_make_tmap(m->lm_i8, m->Vloc, H, &m->lm1_tmap) == 0) {
    uint8_t* part = nullptr;
    if ((rc = m->alloc(&part, lm_head_m1_part_bytes(m->Vloc)))) return fail(rc);
    m->lm1_part = part;
    m->lm1_ok = true;
  }
  {
    KvGeom g16;
    g16.bf16 = 1;
    g16.hd = 128;
    if (!tp && m->hd == 128 && decode1_supported(m->nh, m->nkv, H, F, g16)) {
      std::vector<D1Layer> dl(m->L);
      for (int l = 0; l < m->L; ++l) {
        const Layer& a = m->layers[l];
        D1Layer& b = dl[l];
        b.w[0] = a.wqkv;
        b.w[1] = a.wo;
        b.w[2] = a.wgu;
        b.w[3] = a.wdown;
        b.norm[0] = a.attn_norm;
        b.norm[1] = a.attn_sub_norm;
        b.norm[2] = a.ffn_norm;
        b.norm[3] = a.ffn_sub_norm;
        b.sq = a.sq;
        b.sk = a.sk;
        b.sv = a.sv;
        b.so = a.so;
        b.sg = a.sg;
        b.su = a.su;
        b.sd = a.sd;
        b.pad = 0.0f;
      }
      if ((rc = put(m, &m->d1_layers, dl.data(), dl.size()))) return fail(rc);
      if ((rc = m->alloc(&m->d1_sync, decode1_sync_bytes() / 4))) return fail(rc);
      cudaDeviceGetAttribute(&m->d1_sms, cudaDevAttrMultiProcessorCount, ctx->device);
      const int hpc = decode1_hpc(m->nh, m->nkv);
      m->d1_limit = m->d1_sms > m->nh / hpc ? decode1_smem_limit(hpc) : 0;
    }
  }
  {
    size_t smem = paged_attention_exact_smem(m->nh, m->nkv, m->hd, (int)round_up(cfg->max_position_embeddings, kPage));
    if (smem <= kExactMaxSmem && paged_attention_exact_prepare(smem) == 0) {
      m->exact_smem_ok = true;
      m->exact_smem_max = smem;
    }
  }
  if ((rc = ensure_exp_table(ctx))) return fail(rc);
  m->mma_attn_ok = flash_decode_mma_prepare() == 0;
  m->lm_mma_ok = lm_head_mma_supported(m->H) && lm_head_mma_prepare() == 0;
  {
    size_t smem = exact2_smem((int)round_up(cfg->max_position_embeddings, kPage));
    if (smem <= kExactMaxSmem && exact2_prepare(smem) == 0) {
      m->exact2_ok = true;
      m->exact2_smem_max = smem;
    }
  }
  {
    size_t smem = exact3_smem((int)round_up(cfg->max_position_embeddings, kPage));
    if (smem <= kExactMaxSmem && exact3_prepare(smem) == 0) {
      m->exact3_ok = true;
      m->exact3_smem_max = smem;
    }
  }
  {
    const int max_ctx = (int)round_up(cfg->max_position_embeddings, kPage);
    size_t smem = attn_x4_smem(max_ctx);
    if (smem <= kExactMaxSmem && attn_x4_prepare(max_ctx) == 0) {
      m->x4_ok = true;
      m->x4_smem_max = smem;
    }
  }
  // RoPE table for every position the model accepts (rope.rs:100-147).
  std::vector<float> cs, sn;
  if ((rc = build_rope_host(cfg->max_position_embeddings, m->hd, cfg->rope_theta, cs, sn))) return fail(rc);
  if ((rc = put(m, &m->rope_cos, cs.data(), cs.size()))) return fail(rc);
  if ((rc = put(m, &m->rope_sin, sn.data(), sn.size()))) return fail(rc);
  // activations
  const size_t T = m->Tmax;
  const size_t R = std::min<size_t>(T, 1024);  // logits rows per forward
  if ((rc = m->alloc(&m->h, T * H))) return fail(rc);
  if ((rc = m->alloc(&m->qkv, T * (qd + 2 * kvd)))) return fail(rc);
  if ((rc = m->alloc(&m->qrot, T * std::max(qd, H)))) return fail(rc);
  if ((rc = m->alloc(&m->attn, T * qd))) return fail(rc);
  if ((rc = m->alloc(&m->gu, T * 2 * F))) return fail(rc);
  if ((rc = m->alloc(&m->hn, R * H))) return fail(rc);
  if ((rc = m->alloc(&m->logits, R * m->Vs))) return fail(rc);
  if ((rc = m->alloc(&m->a3, R * 3 * H))) return fail(rc);
  if ((rc = m->alloc(&m->xq, T * m->ldq))) return fail(rc);
  if ((rc = m->alloc(&m->amax, T))) return fail(rc);
  if ((rc = m->alloc(&m->rowsum, T))) return fail(rc);
  if ((rc = m->alloc(&m->tokens, T))) return fail(rc);
  if ((rc = m->alloc(&m->next, T))) return fail(rc);
  if ((rc = m->alloc(&m->tok_pos, T))) return fail(rc);
  if ((rc = m->alloc(&m->tok_seq, T))) return fail(rc);
  if ((rc = m->alloc(&m->last_row, T))) return fail(rc);
  if ((rc = m->alloc(&m->order, T))) return fail(rc);
  if ((rc = m->alloc(&m->hist, cfg->max_position_embeddings))) return fail(rc);
  if ((rc = m->alloc(&m->status, 16))) return fail(rc);
  if (tp) {
    const size_t wide = (size_t)std::max(m->qd_all, m->F_all);
    if ((rc = m->alloc(&m->tp_gath, T * wide))) return fail(rc);
    if ((rc = m->alloc(&m->tp_full, T * wide))) return fail(rc);
    if ((rc = m->alloc(&m->tp_acc, T * H))) return fail(rc);
    if ((rc = m->alloc(&m->tp_rowsum, T))) return fail(rc);
    if ((rc = m->alloc(&m->tp_pairs, R))) return fail(rc);
    if ((rc = m->alloc(&m->tp_pairs_all, R * G))) return fail(rc);
    if ((rc = m->alloc(&m->tp_lgath, R * G * m->Vs))) return fail(rc);
    if ((rc = m->alloc(&m->tp_logits, R * G * m->Vs))) return fail(rc);
  }
  cudaError_t e = cudaMallocHost(&m->h_meta, 4 * T * sizeof(int32_t));
  if (e != cudaSuccess) return fail(cuda_error(e, "cudaMallocHost"));
  e = cudaMallocHost(&m->h_tokens, T * sizeof(uint32_t));
  if (e != cudaSuccess) return fail(cuda_error(e, "cudaMallocHost"));
  e = cudaMemsetAsync(m->status, 0, 64, ctx->stream);
  if (e != cudaSuccess) return fail(cuda_error(e, "cudaMemset"));
  e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return fail(cuda_error(e, "model upload"));
  *out = m;
  return BITNET_OK;
}

}  // namespace

extern "C" {

int bitnet_cuda_model_create(bitnet_cuda_ctx* ctx, const bitnet_cuda_config* cfg, const bitnet_cuda_weights* w,
                             uint32_t max_batch_tokens, bitnet_cuda_model** out) {
  return model_create_impl(ctx, cfg, w, max_batch_tokens, 0, 1, nullptr, out);
}

int bitnet_cuda_model_create_tp(bitnet_cuda_ctx* ctx, const bitnet_cuda_config* cfg, const bitnet_cuda_weights* w,
                                uint32_t max_batch_tokens, uint32_t rank, uint32_t world, const uint8_t* nccl_id,
                                size_t id_len, bitnet_cuda_model** out) {
  if (out) *out = nullptr;
  if (!nccl_id) return shape_error("non-null NCCL id", "null");
  if (id_len < sizeof(ncclUniqueId))
    return shape_error("id_len >= " + sz(sizeof(ncclUniqueId)), sz(id_len));
  return model_create_impl(ctx, cfg, w, max_batch_tokens, rank, world, nccl_id, out);
}

void bitnet_cuda_model_destroy(bitnet_cuda_model* m) {
  if (m) model_release(m);
}

// ---- KV cache -----------------------------------------------------------------
int bitnet_cuda_kv_create(bitnet_cuda_model* m, uint32_t num_pages, uint32_t max_seqs, int kv_dtype,
                          bitnet_cuda_kv** out) {
  if (!out || !m) return shape_error("non-null arguments", "null");
  *out = nullptr;
  if (num_pages == 0 || max_seqs == 0) return shape_error("num_pages > 0 and max_seqs > 0", "0");
  if (kv_dtype != BITNET_KV_F32 && kv_dtype != BITNET_KV_BF16) return config_error("kv_dtype must be F32 or BF16");
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  cudaSetDevice(m->ctx->device);
  auto* kv = new bitnet_cuda_kv();
  kv->model = m;
  kv->g.bf16 = kv_dtype == BITNET_KV_BF16;
  kv->g.pages = (int)num_pages;
  kv->g.kv_heads = m->nkv;
  kv->g.hd = m->hd;
  kv->g.layers = m->L;
  kv->g.max_pages_per_seq = (int)ceil_div(m->cfg.max_position_embeddings, kPage);
  kv->max_seqs = (int)max_seqs;
  size_t elem = kv->g.bf16 ? 2 : 4;
  size_t bytes = (size_t)m->L * num_pages * m->nkv * 2 * kPage * m->hd * elem;
  cudaError_t e = cudaMalloc(&kv->g.pool, bytes);
  if (e != cudaSuccess) {
    delete kv;
    return cuda_error(e, "cudaMalloc(kv pool)");
  }
  size_t tbl = (size_t)max_seqs * kv->g.max_pages_per_seq;
  e = cudaMalloc(&kv->d_table, tbl * sizeof(int32_t));
  if (e != cudaSuccess) {
    cudaFree(kv->g.pool);
    delete kv;
    return cuda_error(e, "cudaMalloc(page table)");
  }
  cudaMemsetAsync(kv->d_table, 0, tbl * sizeof(int32_t), m->ctx->stream);
  cudaStreamSynchronize(m->ctx->stream);
  kv->h_table.assign(tbl, 0);
  kv->tmap_ok = exact3_make_tmap(kv->g, &kv->tmap) == 0;
  kv->free_pages.resize(num_pages);
  for (uint32_t i = 0; i < num_pages; ++i) kv->free_pages[i] = (int32_t)(num_pages - 1 - i);
  kv->seq_pages.assign(max_seqs, {});
  kv->seq_len.assign(max_seqs, 0);
  m->refs.fetch_add(1);
  *out = kv;
  return BITNET_OK;
}

void bitnet_cuda_kv_destroy(bitnet_cuda_kv* kv) {
  if (!kv) return;
  bitnet_cuda_model* m = kv->model;
  cudaSetDevice(m->ctx->device);
  cudaStreamSynchronize(m->ctx->stream);
  for (auto it = m->graphs.begin(); it != m->graphs.end();) {
    if (std::get<0>(it->first) == (void*)kv) {
      if (m->last_timed == &it->second) m->last_timed = nullptr;
      destroy_graph(it->second);
      it = m->graphs.erase(it);
    } else {
      ++it;
    }
  }
  cudaFree(kv->g.pool);
  cudaFree(kv->d_table);
  delete kv;
  model_release(m);
}

int bitnet_cuda_kv_seq_reset(bitnet_cuda_kv* kv, uint32_t seq) {
  if (seq >= (uint32_t)kv->max_seqs) return shape_error("seq < max_seqs", sz(seq));
  for (int32_t p : kv->seq_pages[seq]) kv->free_pages.push_back(p);
  kv->seq_pages[seq].clear();
  kv->seq_len[seq] = 0;
  return BITNET_OK;
}

int bitnet_cuda_kv_seq_len(bitnet_cuda_kv* kv, uint32_t seq, size_t* len) {
  if (seq >= (uint32_t)kv->max_seqs) return shape_error("seq < max_seqs", sz(seq));
  *len = kv->seq_len[seq];
  return BITNET_OK;
}

int bitnet_cuda_kv_free_pages(bitnet_cuda_kv* kv, size_t* n) {
  *n = kv->free_pages.size();
  return BITNET_OK;
}

int bitnet_cuda_kv_seq_reserve(bitnet_cuda_kv* kv, uint32_t seq, size_t len) {
  if (seq >= (uint32_t)kv->max_seqs) return shape_error("seq < max_seqs", sz(seq));
  std::lock_guard<std::mutex> lk(kv->model->ctx->mu);
  cudaSetDevice(kv->model->ctx->device);
  return kv_reserve(kv, seq, len, kv->model->ctx->stream);
}

static int kv_seq_copy(bitnet_cuda_kv* kv, uint32_t seq, size_t n, const float* k, float* kout, const float* v,
                       float* vout, bool to_cache) {
  if (seq >= (uint32_t)kv->max_seqs) return shape_error("seq < max_seqs", sz(seq));
  bitnet_cuda_model* m = kv->model;
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  cudaSetDevice(m->ctx->device);
  cudaStream_t st = m->ctx->stream;
  if (!to_cache && n > kv->seq_len[seq]) return shape_error("n <= sequence length " + sz(kv->seq_len[seq]), sz(n));
  if (to_cache) BN_TRY(kv_reserve(kv, seq, n, st));
  if (n == 0) {
    if (to_cache) kv->seq_len[seq] = 0;
    return BITNET_OK;
  }
  size_t elems = (size_t)m->L * n * m->kvd;
  DevBuf ks, vs;
  BN_TRY(ks.ensure(elems * 4));
  BN_TRY(vs.ensure(elems * 4));
  const int32_t* row = kv->d_table + (size_t)seq * kv->g.max_pages_per_seq;
  if (to_cache) {
    BN_CUDA(cudaMemcpyAsync(ks.p, k, elems * 4, cudaMemcpyHostToDevice, st));
    BN_CUDA(cudaMemcpyAsync(vs.p, v, elems * 4, cudaMemcpyHostToDevice, st));
    launch_kv_copy(kv->g, row, (int)n, ks.as<float>(), vs.as<float>(), true, st);
    kv->seq_len[seq] = n;
  } else {
    launch_kv_copy(kv->g, row, (int)n, ks.as<float>(), vs.as<float>(), false, st);
    BN_CUDA(cudaMemcpyAsync(kout, ks.p, elems * 4, cudaMemcpyDeviceToHost, st));
    BN_CUDA(cudaMemcpyAsync(vout, vs.p, elems * 4, cudaMemcpyDeviceToHost, st));
  }
  BN_CUDA(cudaGetLastError());
  BN_CUDA(cudaStreamSynchronize(st));
  return BITNET_OK;
}

int bitnet_cuda_kv_seq_write(bitnet_cuda_kv* kv, uint32_t seq, size_t n, const float* k, const float* v) {
  return kv_seq_copy(kv, seq, n, k, nullptr, v, nullptr, true);
}

int bitnet_cuda_kv_seq_read(bitnet_cuda_kv* kv, uint32_t seq, size_t n, float* k, float* v) {
  return kv_seq_copy(kv, seq, n, nullptr, k, nullptr, v, false);
}

int bitnet_cuda_kv_seq_fill_random(bitnet_cuda_kv* kv, uint32_t seq, size_t n, uint64_t seed) {
  if (seq >= (uint32_t)kv->max_seqs) return shape_error("seq < max_seqs", sz(seq));
  bitnet_cuda_model* m = kv->model;
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  cudaSetDevice(m->ctx->device);
  cudaStream_t st = m->ctx->stream;
  BN_TRY(kv_reserve(kv, seq, n, st));
  launch_kv_fill_random(kv->g, kv->d_table + (size_t)seq * kv->g.max_pages_per_seq, (int)n, seed, seq, st);
  BN_CUDA(cudaGetLastError());
  BN_CUDA(cudaStreamSynchronize(st));
  kv->seq_len[seq] = n;
  return BITNET_OK;
}

// ---- forward / decode / prefill ------------------------------------------------------
static int forward_common(bitnet_cuda_model* m, bitnet_cuda_kv* kv, size_t n_seqs, const uint32_t* seq_ids,
                          const uint32_t* counts, const uint32_t* tokens, float* logits, uint32_t* next) {
  cudaStream_t st = m->ctx->stream;
  int T = 0, max_ctx = 1;
  BN_TRY(prepare_batch(m, kv, n_seqs, seq_ids, counts, &T, &max_ctx, st));
  if (n_seqs > 1024) return shape_error("<= 1024 sequences per call", sz(n_seqs));
  BN_TRY(ensure_partial(m, kv, T, max_ctx));
  std::memcpy(m->h_tokens, tokens, (size_t)T * 4);
  BN_CUDA(cudaMemcpyAsync(m->tokens, m->h_tokens, (size_t)T * 4, cudaMemcpyHostToDevice, st));
  BN_TRY(upload_meta(m, T, (int)n_seqs, st));
  run_forward(m, kv, T, (int)n_seqs, max_ctx, st);
  BN_CUDA(cudaGetLastError());
  if (logits) BN_TRY(copy_logits(m, (int)n_seqs, logits, cudaMemcpyDeviceToHost, st));
  if (next) BN_CUDA(cudaMemcpyAsync(next, m->next, n_seqs * 4, cudaMemcpyDeviceToHost, st));
  BN_TRY(check_status(m));
  for (size_t i = 0; i < n_seqs; ++i) kv->seq_len[seq_ids[i]] += counts[i];
  return BITNET_OK;
}

int bitnet_cuda_forward(bitnet_cuda_model* m, bitnet_cuda_kv* kv, uint32_t seq, const uint32_t* tokens, size_t n,
                        size_t start_pos, float* logits) {
  if (!m || !kv) return shape_error("non-null model and kv", "null");
  if (n == 0) return shape_error("tokens must not be empty", "0 tokens");
  if (seq >= (uint32_t)kv->max_seqs) return shape_error("seq < max_seqs", sz(seq));
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  cudaSetDevice(m->ctx->device);
  size_t len = kv->seq_len[seq];
  if (start_pos > len) return shape_error("start_pos <= cached positions (" + sz(len) + ")", "start_pos = " + sz(start_pos));
  kv->seq_len[seq] = start_pos;  // positions >= start_pos are overwritten
  // chunk long inputs by the model's token capacity (same per-token math)
  size_t done = 0;
  while (done < n) {
    uint32_t cnt = (uint32_t)std::min<size_t>(n - done, (size_t)m->Tmax);
    bool last = done + cnt == n;
    BN_TRY(forward_common(m, kv, 1, &seq, &cnt, tokens + done, last ? logits : nullptr, nullptr));
    done += cnt;
  }
  return BITNET_OK;
}

int bitnet_cuda_prefill(bitnet_cuda_model* m, bitnet_cuda_kv* kv, size_t n_seqs, const uint32_t* seq_ids,
                        const uint32_t* tokens, const uint32_t* cu_seqlens, float* logits, uint32_t* next_tokens) {
  if (!m || !kv) return shape_error("non-null model and kv", "null");
  if (n_seqs == 0) return BITNET_OK;
  std::vector<uint32_t> counts(n_seqs);
  for (size_t i = 0; i < n_seqs; ++i) {
    if (cu_seqlens[i + 1] < cu_seqlens[i]) return shape_error("non-decreasing cu_seqlens", "decreasing");
    counts[i] = cu_seqlens[i + 1] - cu_seqlens[i];
  }
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  cudaSetDevice(m->ctx->device);
  return forward_common(m, kv, n_seqs, seq_ids, counts.data(), tokens + cu_seqlens[0], logits, next_tokens);
}

// One decode step as a CUDA graph: tokens come from `src` (host or device),
// next tokens / logits stay in the model's device buffers.
static int decode_graph(bitnet_cuda_model* m, bitnet_cuda_kv* kv, size_t batch, const uint32_t* seq_ids,
                        const uint32_t* src, bool src_on_host, cudaStream_t st) {
  if (batch > 1024) return shape_error("batch <= 1024", sz(batch));
  std::vector<uint32_t> ones(batch, 1);
  int T = 0, max_ctx = 1;
  BN_TRY(prepare_batch(m, kv, batch, seq_ids, ones.data(), &T, &max_ctx, st));
  // The graph is sized for the cache capacity so it can be replayed as
  // contexts grow; splits past a token's context exit immediately.
  const int cap_ctx = (int)kv->capacity();
  BN_TRY(ensure_partial(m, kv, T, cap_ctx));
  BN_TRY(upload_meta(m, T, T, st));
  if (src_on_host) {
    std::memcpy(m->h_tokens, src, (size_t)T * 4);
    BN_CUDA(cudaMemcpyAsync(m->tokens, m->h_tokens, (size_t)T * 4, cudaMemcpyHostToDevice, st));
  } else {
    BN_CUDA(cudaMemcpyAsync(m->tokens, src, (size_t)T * 4, cudaMemcpyDeviceToDevice, st));
  }
  if (m->tp_dead) return backend_error("the tensor-parallel communicator was aborted after an earlier failure");
  auto key = std::make_tuple((void*)kv, T, m->timing ? 1 : 0);
  auto it = m->graphs.find(key);
  if (it == m->graphs.end()) {
    bitnet_cuda_model::Graph gr{};
    cudaGraph_t g;
    uint64_t before = launches_total();
    if (m->timing) m->marks = &gr.marks;
    cudaError_t e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
    if (e == cudaSuccess) {
      run_forward(m, kv, T, T, cap_ctx, st);
      e = cudaStreamEndCapture(st, &g);
    }
    m->marks = nullptr;
    gr.kernels = launches_total() - before;
    uncount_launch(gr.kernels);  // captured, not launched: replays count them
    if (e != cudaSuccess) {
      destroy_graph(gr);
      return cuda_error(e, "CUDA graph capture");
    }
    e = cudaGraphInstantiate(&gr.exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_error(e, "cudaGraphInstantiate");
    it = m->graphs.emplace(key, std::move(gr)).first;
  }
  BN_CUDA(cudaGraphLaunch(it->second.exec, st));
  count_launch(it->second.kernels);
  if (m->timing) m->last_timed = &it->second;
  for (size_t i = 0; i < batch; ++i) kv->seq_len[seq_ids[i]] += 1;
  return BITNET_OK;
}

int bitnet_cuda_decode_step(bitnet_cuda_model* m, bitnet_cuda_kv* kv, size_t batch, const uint32_t* seq_ids,
                            const uint32_t* tokens, float* logits, uint32_t* next_tokens) {
  if (!m || !kv) return shape_error("non-null model and kv", "null");
  if (batch == 0) return BITNET_OK;
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  cudaSetDevice(m->ctx->device);
  cudaStream_t st = m->ctx->stream;
  BN_TRY(decode_graph(m, kv, batch, seq_ids, tokens, true, st));
  if (logits) BN_TRY(copy_logits(m, (int)batch, logits, cudaMemcpyDeviceToHost, st));
  if (next_tokens) BN_CUDA(cudaMemcpyAsync(next_tokens, m->next, batch * 4, cudaMemcpyDeviceToHost, st));
  return check_status(m);  // synchronises
}

int bitnet_cuda_decode_step_device(bitnet_cuda_model* m, bitnet_cuda_kv* kv, size_t batch, const uint32_t* seq_ids,
                                   const uint32_t* d_tokens, uint32_t* d_next, float* d_logits, void* stream) {
  if (!m || !kv) return shape_error("non-null model and kv", "null");
  if (batch == 0) return BITNET_OK;
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  cudaSetDevice(m->ctx->device);
  cudaStream_t st = stream ? (cudaStream_t)stream : m->ctx->stream;
  BN_TRY(decode_graph(m, kv, batch, seq_ids, d_tokens, false, st));
  BN_CUDA(cudaMemcpyAsync(d_next, m->next, batch * 4, cudaMemcpyDeviceToDevice, st));
  if (d_logits) BN_TRY(copy_logits(m, (int)batch, d_logits, cudaMemcpyDeviceToDevice, st));
  return BITNET_OK;
}

int bitnet_cuda_model_set_numerics(bitnet_cuda_model* m, int mode) {
  if (!m) return shape_error("non-null model", "null");
  if (mode != BITNET_NUMERICS_AUTO && mode != BITNET_NUMERICS_EXACT && mode != BITNET_NUMERICS_FAST)
    return config_error("numerics mode must be AUTO, EXACT or FAST");
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  cudaSetDevice(m->ctx->device);
  cudaStreamSynchronize(m->ctx->stream);
  m->numerics = mode;
  drop_graphs(m);  // captured graphs embed the previous kernel choice
  return BITNET_OK;
}

int bitnet_cuda_model_set_fused_decode(bitnet_cuda_model* m, int enable) {
  if (!m) return shape_error("non-null model", "null");
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  cudaSetDevice(m->ctx->device);
  cudaStreamSynchronize(m->ctx->stream);
  m->d1_enabled = enable != 0;
  drop_graphs(m);  // captured graphs embed the previous kernel choice
  return BITNET_OK;
}

int bitnet_cuda_model_attention_kernel(bitnet_cuda_model* m, bitnet_cuda_kv* kv, uint32_t tokens, char* name,
                                       size_t name_len) {
  if (!m || !kv || !name || name_len == 0) return shape_error("non-null arguments", "null");
  if (tokens == 0) return shape_error("tokens > 0", "0");
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  cudaSetDevice(m->ctx->device);
  d1_prepare(m, kv, (int)tokens, (int)kv->capacity());
  const char* k = attention_kernel_name(m, kv, (int)tokens, (int)kv->capacity());
  std::snprintf(name, name_len, "%s", k);
  return BITNET_OK;
}

int bitnet_cuda_model_set_kernel_timing(bitnet_cuda_model* m, int enable) {
  if (!m) return shape_error("non-null model", "null");
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  m->timing = enable != 0;
  return BITNET_OK;
}

int bitnet_cuda_model_kernel_times(bitnet_cuda_model* m, float* ms, int32_t* launches) {
  if (!m || !ms || !launches) return shape_error("non-null arguments", "null");
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  cudaSetDevice(m->ctx->device);
  for (int c = 0; c < kClasses; ++c) {
    ms[c] = 0.0f;
    launches[c] = 0;
  }
  if (!m->last_timed) return backend_error("no timed decode step has run");
  for (const auto& t : m->last_timed->marks) {
    BN_CUDA(cudaEventSynchronize(std::get<2>(t)));
    float e = 0.0f;
    BN_CUDA(cudaEventElapsedTime(&e, std::get<1>(t), std::get<2>(t)));
    ms[std::get<0>(t)] += e;
    launches[std::get<0>(t)] += 1;
  }
  return BITNET_OK;
}

int bitnet_cuda_model_check(bitnet_cuda_model* m) {
  if (!m) return shape_error("non-null model", "null");
  std::lock_guard<std::mutex> lk(m->ctx->mu);
  cudaSetDevice(m->ctx->device);
  return check_status(m);
}

int bitnet_cuda_generate(bitnet_cuda_model* m, bitnet_cuda_kv* kv, uint32_t seq, const uint32_t* prompt,
                         size_t n_prompt, size_t max_new, uint32_t eos0, uint32_t eos1, uint32_t* out_tokens,
                         size_t* n_out) {
  if (!n_out) return shape_error("non-null n_out", "null");
  *n_out = 0;
  if (n_prompt == 0) return BITNET_OK;
  BN_TRY(bitnet_cuda_kv_seq_reset(kv, seq));
  uint32_t next = 0;
  {
    std::lock_guard<std::mutex> lk(m->ctx->mu);
    cudaSetDevice(m->ctx->device);
    size_t done = 0;
    while (done < n_prompt) {
      uint32_t cnt = (uint32_t)std::min<size_t>(n_prompt - done, (size_t)m->Tmax);
      BN_TRY(forward_common(m, kv, 1, &seq, &cnt, prompt + done, nullptr, &next));
      done += cnt;
    }
  }
  for (size_t step = 0; step < max_new; ++step) {
    if (next == eos0 || next == eos1) break;
    out_tokens[(*n_out)++] = next;
    BN_TRY(bitnet_cuda_decode_step(m, kv, 1, &seq, &next, nullptr, &next));
  }
  return BITNET_OK;
}

int bitnet_cuda_generate_sampled(bitnet_cuda_model* m, bitnet_cuda_kv* kv, uint32_t seq, const uint32_t* prompt,
                                 size_t n_prompt, size_t max_new, const bitnet_cuda_sampling* cfg, uint32_t eos0,
                                 uint32_t eos1, uint32_t* out_tokens, size_t* n_out) {
  if (!n_out || !cfg || !m || !kv) return shape_error("non-null model, kv, config and n_out", "null");
  *n_out = 0;
  BN_TRY(validate_sampling(*cfg, max_new));  // generate_from_tokens_streaming, lib.rs:706
  if (n_prompt == 0) return BITNET_OK;
  if (n_prompt + max_new > m->cfg.max_position_embeddings)
    return shape_error("prompt + max_new <= max_position_embeddings " + sz(m->cfg.max_position_embeddings),
                       sz(n_prompt + max_new));
  BN_TRY(bitnet_cuda_kv_seq_reset(kv, seq));
  size_t n_hist = n_prompt;
  uint32_t next = 0;
  {
    std::lock_guard<std::mutex> lk(m->ctx->mu);
    cudaSetDevice(m->ctx->device);
    cudaStream_t st = m->ctx->stream;
    BN_CUDA(cudaMemcpyAsync(m->hist, prompt, n_prompt * 4, cudaMemcpyHostToDevice, st));
    size_t done = 0;
    while (done < n_prompt) {
      uint32_t cnt = (uint32_t)std::min<size_t>(n_prompt - done, (size_t)m->Tmax);
      BN_TRY(forward_common(m, kv, 1, &seq, &cnt, prompt + done, nullptr, nullptr));
      done += cnt;
    }
    size_t ld = 0;
    float* lg = const_cast<float*>(full_logits(m, 1, &ld, st));
    BN_TRY(sample_device(m->ctx, lg, (size_t)m->V, *cfg, m->hist, n_hist, &next, st));
  }
  for (size_t step = 0; step < max_new; ++step) {
    if (next == eos0 || next == eos1) break;
    out_tokens[(*n_out)++] = next;
    // the decode step leaves this token's logits in the model's row 0
    BN_TRY(bitnet_cuda_decode_step(m, kv, 1, &seq, &next, nullptr, nullptr));
    std::lock_guard<std::mutex> lk(m->ctx->mu);
    cudaSetDevice(m->ctx->device);
    cudaStream_t st = m->ctx->stream;
    BN_CUDA(cudaMemcpyAsync(m->hist + n_hist, &next, 4, cudaMemcpyHostToDevice, st));
    ++n_hist;
    if (step + 1 < max_new) {
      size_t ld = 0;
      float* lg = const_cast<float*>(full_logits(m, 1, &ld, st));
      BN_TRY(sample_device(m->ctx, lg, (size_t)m->V, *cfg, m->hist, n_hist, &next, st));
    }
  }
  return BITNET_OK;
}

}  // extern "C"
