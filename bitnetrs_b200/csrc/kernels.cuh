// kernels.cuh — launchers for the device kernels (all asynchronous on `st`).
#pragma once

#include "common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

namespace bitnet {

// Bits of the device status word (read and cleared by the host after a step).
constexpr int kStatusNonFinite = 1;    // non-finite activation met by a quantiser
constexpr int kStatusBadToken = 2;     // token id >= vocab_size
constexpr int kStatusBadContext = 4;   // a token's context exceeds the kernel's capacity
constexpr int kStatusWaitTimeout = 8;  // a bounded device-side wait gave up

// Launch with programmatic stream serialisation (the kernel must follow the
// pdl_wait rule of common.cuh).
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Per-launch kernel counter (reported by bitnet_cuda_kernel_launches).
void count_launch(uint64_t n = 1);
void uncount_launch(uint64_t n);
uint64_t launches_total();

// ---- weight layout ----------------------------------------------------------
// Reference 2-bit rows [rows][ceil(cols/4)] -> device words [rows][words_per_row(cols)].
void launch_repack_ternary(const uint8_t* src, uint32_t* dst, int rows, int cols, cudaStream_t st);

// ---- activation quantisation / norms ---------------------------------------
// absmax_quantize_row_into per row.  x: [M][ldx] (f32, or bf16 bits when x_bf16).
// xq: [M][ldq] zero padded to ldq; act_absmax[m] = (mc/127)*127; scale[m] = mc/127
// (either may be null); row_sum[m] = sum of xq; status |= 1 on non-finite input.
void launch_quantize_rows(const void* x, bool x_bf16, int ldx, int M, int K, int8_t* xq, int ldq, float* act_absmax,
                          float* scale, int32_t* row_sum, int32_t* status, cudaStream_t st);

// The row kernels below stage one row of up to kMaxRowFloats f32 in shared
// memory; row_kernels_prepare raises their limit above the 48 KiB default on
// the current device (call outside graph capture; 0 on success).
constexpr int kMaxRowFloats = 56 * 1024;
int row_kernels_prepare();

// rms_norm in the reference order (norm.rs:113-137): out[m] = (x*inv)*w.
void launch_rms_norm(const float* x, int ldx, const float* w, int d, float eps, float* out, int ldo, int M,
                     cudaStream_t st);

// rms_norm followed by absmax quantisation of the normalised row (the model's
// rms_norm -> absmax_quantize_row_into pairs, model/src/lib.rs:952-962 etc.).
// When `gate_up` is set, the row is first formed as sqrelu(gate)*up
// (simd.rs:1135-1184) from x (gate) and x2 (up).
void launch_norm_quant(const float* x, const float* x2, int ldx, const float* w, int d, float eps, int8_t* xq, int ldq,
                       float* act_absmax, int32_t* row_sum, int32_t* status, int M, cudaStream_t st);

// ---- elementwise -------------------------------------------------------------
void launch_squared_relu(float* x, size_t n, cudaStream_t st);
void launch_sqrelu_gate(const float* g, const float* u, float* out, size_t n, cudaStream_t st);
void launch_elementwise_mul(const float* a, const float* b, float* out, size_t n, cudaStream_t st);
// activation::softmax in place over one vector (sequential sum order).
void launch_softmax(float* x, size_t n, float* scratch_max, const ExpTable& et, cudaStream_t st);
// bf16 embedding rows -> f32 hidden rows.
void launch_embed(const uint16_t* embed, const uint32_t* tokens, int T, int H, float* h, int32_t* status, int vocab,
                  cudaStream_t st);

// dst[r] = src[rows[r]] for r < n (rows of length ld).
void launch_gather_rows(const float* src, int ld, const int32_t* rows, int n, float* dst, cudaStream_t st);

// ---- ternary matmul ------------------------------------------------------------
// Output segments: rows [seg_end[s-1], seg_end[s]) use scale seg_scale[s].
struct Segments {
  int n = 1;
  int end[3] = {0, 0, 0};
  float scale[3] = {0.f, 0.f, 0.f};
};
enum class Epi : int { Store = 0, Residual = 1 };
__device__ __forceinline__ float seg_scale(const Segments& s, int n) {
  return n < s.end[0] ? s.scale[0] : (n < s.end[1] ? s.scale[1] : s.scale[2]);
}
// The reference's dequantisation (bitnet-cpu/src/gemv.rs:297-307): acc as f32 * (ws * act_absmax / 127).
__device__ __forceinline__ float dequant(int32_t acc, float ws, float amax) {
  float combined = __fdiv_rn(__fmul_rn(ws, amax), 127.0f);
  return __fmul_rn((float)acc, combined);
}
// out[m][n] = (sum_k W[n,k] x[m][k]) * ((seg_scale*act_absmax[m])/127); Residual: out += that.
// acc (optional) receives the int32 sums [M][N] (row stride N).
// `status` (optional) receives kStatusWaitTimeout if the tensor-core kernel
// (used for M > 1 when ternary_tc_prepare succeeded) gives up a wait.
void launch_ternary_matmul(const uint32_t* W, int N, int K, const int8_t* xq, int ldq, const float* act_absmax,
                           const int32_t* row_sum, int M, const Segments& seg, Epi epi, float* out, int ldo,
                           int32_t* acc, cudaStream_t st, int32_t* status = nullptr);
// tcgen05 ternary GEMM (kernels_tcgen05.cu): 128 weight rows x up to 256
// activation rows per CTA, TMEM accumulator, optional cluster split-K.
int ternary_tc_prepare();  // per device, outside graph capture; 0 on success
// Tile plan for an M x N x K product: activation rows per CTA, activation
// stages, k splits (cluster size) and k-steps per split. 0 on success.
int ternary_tc_plan(int N, int K, int M, int* nb, int* stages, int* splits, int* per);
int launch_ternary_tc(const uint32_t* W, int N, int K, const int8_t* xq, int ldq, const float* act_absmax,
                      const int32_t* row_sum, int M, const Segments& seg, Epi epi, float* out, int ldo, int32_t* acc,
                      int32_t* status, cudaStream_t st);  // 0 on success
int kernel_binary_version(int* v);  // binaryVersion of a library kernel; 0 on success
void set_ternary_tc_ready(bool ready);
bool ternary_tc_ready();
// Tensor-core lm_head (kernels_tcgen05.cu): a3 = [M][3H] bf16 terms of h.
bool lm_head_tc_supported(int H);
int launch_lm_head_tc(const uint16_t* a3, int M, int V, int H, const int8_t* W, const float* scales, float* out,
                      int ldo, int32_t* status, cudaStream_t st);  // 0 on success
// row_sum for callers that quantised elsewhere.
void launch_row_sum(const int8_t* xq, int ldq, int M, int K, int32_t* row_sum, cudaStream_t st);

// ternary_gemv_f32 (gemv.rs:108-165) in the reference's f32 summation order.
void launch_ternary_gemv_f32(const uint8_t* packed, int N, int K, float ws, const float* x, float* out,
                             cudaStream_t st);

// ---- lm_head -------------------------------------------------------------------
enum class LmW : int { I8 = 0, BF16 = 1, F32 = 2 };
// out[m][v] = dot(W[v], h[m]) (* scales[v] for I8), reference FMA order.
void launch_lm_head(const void* W, LmW wt, const float* scales, const float* h, int ldh, int M, int V, int H,
                    float* out, int ldo, cudaStream_t st);
// Tensor-core i8 lm_head for many tokens (h split into three bf16 terms);
// a3 is scratch of M*3*H bf16.  Requires H % 64 == 0.
bool lm_head_mma_supported(int H);
int lm_head_mma_prepare();  // outside graph capture; 0 on success
void launch_lm_head_mma(const float* h, int M, int V, int H, const int8_t* W, const float* scales, uint16_t* a3,
                        float* out, int ldo, cudaStream_t st, int32_t* status = nullptr);
// sample_next_token on one row of logits (sampler.cu): counts is [V] int32
// kept at zero between calls, escratch [V] floats; status |= 1 when top-p
// meets more than 4096 finite logits.
size_t sampler_smem();
int sampler_prepare();  // outside graph capture; 0 on success
void launch_sample(float* logits, uint32_t V, const bitnet_cuda_sampling& c, const uint32_t* past, uint32_t n_past,
                   int32_t* counts, float* escratch, uint32_t* out, int32_t* status, const ExpTable& et,
                   cudaStream_t st);
// greedy argmax per row (ties -> last index, NaN compares Equal).
void launch_argmax(const float* logits, int ldl, int M, int V, uint32_t* out, cudaStream_t st);

// ---- attention -------------------------------------------------------------------
// Backend::masked_attention on a head-major cache (attention.rs:97-209).
void launch_masked_attention_headmajor(const float* q, const float* kc, const float* vc, float* out, int nh, int nkv,
                                       int hd, int stride, int seq_len, float* scratch, const ExpTable& et,
                                       cudaStream_t st);

// Backend::rope_embed on one row [q (nh*hd) | k (nkv*hd)] -> out (same layout).
void launch_rope_apply(const float* qk, int nh, int nkv, int hd, const float* cos_table, const float* sin_table,
                       size_t pos, float* out, cudaStream_t st);

// Paged KV cache geometry.
struct KvGeom {
  void* pool = nullptr;       // [layers][pages][kv_heads][2][16][hd]
  int bf16 = 1;               // element type
  int pages = 0, kv_heads = 0, hd = 0, layers = 0;
  int max_pages_per_seq = 0;  // page table row length
};
constexpr int kPage = 16;

// Rotate q/k of T tokens (qkv rows [q | k | v]) with the rope table
// [max_pos][hd/2] (cos, sin), write rotated q into q_out [T][q_dim] and k/v
// into the paged cache of `layer` at each token's position.
void launch_rope_kv_store(const float* qkv, int ldqkv, int T, int nh, int nkv, int hd, const float* rope_cos,
                          const float* rope_sin, const int32_t* tok_pos, const int32_t* tok_seq,
                          const int32_t* page_table, const KvGeom& kv, int layer, float* q_out, cudaStream_t st);

// Decode / prefill attention for T query tokens over the paged cache: token t
// attends to positions [0, tok_pos[t]] of its sequence.
void launch_paged_attention(const float* q, int T, int nh, const int32_t* tok_pos, const int32_t* tok_seq,
                            const int32_t* page_table, const KvGeom& kv, int layer, int max_ctx, float* out,
                            float* partial, size_t partial_floats, cudaStream_t st);
size_t paged_attention_partial_floats(int T, int nh, int hd, int max_ctx);

// Same attention in the reference's exact operation order (see kernels_attn.cu).
// Scores take G*max_ctx floats of shared memory (scores_in_smem) or
// T*nh*max_ctx floats of global scratch.
void launch_paged_attention_exact(const float* q, int T, int nh, const int32_t* tok_pos, const int32_t* tok_seq,
                                  const int32_t* page_table, const KvGeom& kv, int layer, int max_ctx, float* out,
                                  float* scratch, bool scores_in_smem, const ExpTable& et, cudaStream_t st);
size_t paged_attention_exact_smem(int nh, int kv_heads, int hd, int max_ctx);
// Raises the kernel's dynamic shared memory limit (call outside graph capture); 0 on success.
int paged_attention_exact_prepare(size_t smem);

// Reference-order attention for a bf16 cache with head_dim 128 and group 4,
// organised for throughput (scores in shared memory: exact2_smem bytes).
bool exact2_supported(const KvGeom& kv, int nh);
size_t exact2_smem(int max_ctx);
int exact2_prepare(size_t smem);  // outside graph capture; 0 on success
void launch_paged_attention_exact2(const float* q, int T, int nh, const int32_t* tok_pos, const int32_t* tok_seq,
                                   const int32_t* page_table, const KvGeom& kv, int layer, int max_ctx, float* out,
                                   const ExpTable& et, cudaStream_t st);
// The same computation fed by TMA (2-D tiles, 128-byte swizzle) through a
// ring of page slots; needs a tensor map of the pool (exact3_make_tmap).
bool exact3_supported(const KvGeom& kv, int nh);
size_t exact3_smem(int max_ctx);
int exact3_prepare(size_t smem);  // outside graph capture; 0 on success
int exact3_make_tmap(const KvGeom& kv, CUtensorMap* map);  // 0 on success
void launch_paged_attention_exact3(const float* q, int T, int nh, const int32_t* tok_pos, const int32_t* tok_seq,
                                   const int32_t* page_table, const KvGeom& kv, const CUtensorMap& map, int layer,
                                   int max_ctx, float* out, const ExpTable& et, int32_t* status, cudaStream_t st);
// The same computation as two streaming kernels per layer (kernels_attn_x4.cu):
// QK + softmax per (token, kv head), then PV per (token, kv head), through
// `scratch` (attn_x4_scratch_floats floats).  `order` (T entries, may be
// null) lists the tokens in the order their CTAs start (longest context
// first).  Uses the pool's tensor map (exact3_make_tmap).
bool attn_x4_supported(const KvGeom& kv, int nh);
size_t attn_x4_scratch_floats(int T, int kv_heads, int max_ctx);
size_t attn_x4_smem(int max_ctx);
int attn_x4_prepare(int max_ctx);  // outside graph capture; 0 on success
void launch_attn_x4(const float* q, int T, int nh, const int32_t* tok_pos, const int32_t* tok_seq,
                    const int32_t* order, const int32_t* page_table, const KvGeom& kv, const CUtensorMap& map,
                    int layer, int max_ctx, float* out, float* scratch, const ExpTable& et, int32_t* status,
                    cudaStream_t st);
// Candidates for the exp exception table: bit patterns u in [lo, hi] whose
// exp (exp_candidate, with et's pair tables) lands within 0.003 ulp of a
// float rounding midpoint; writes (u, starting value) pairs and counts them.
void launch_exp_candidates(uint32_t lo, uint32_t hi, uint2* out, uint32_t cap, uint32_t* count, const ExpTable& et,
                           cudaStream_t st);

// Tensor-core decode attention (bf16 cache, head_dim 128, group <= 4), split
// over the context; partial holds flash_decode_mma_partial_floats floats.
bool flash_decode_mma_supported(const KvGeom& kv, int nh);
size_t flash_decode_mma_partial_floats(int T, int nh, int max_ctx);
int flash_decode_mma_prepare();  // outside graph capture; 0 on success
void launch_flash_decode_mma(const float* q, int T, int nh, const int32_t* tok_pos, const int32_t* tok_seq,
                             const int32_t* page_table, const KvGeom& kv, int layer, int max_ctx, float* out,
                             float* partial, cudaStream_t st);

// Fill positions [0, n) of sequence `seq` (all layers) with seeded N(0,1).
void launch_kv_fill_random(const KvGeom& kv, const int32_t* page_row, int n, uint64_t seed, uint32_t seq,
                           cudaStream_t st);
// Copy positions [0,n) between a host-layout staging buffer [layer][pos][kvh*hd] (f32) and the cache.
void launch_kv_copy(const KvGeom& kv, const int32_t* page_row, int n, float* k_stage, float* v_stage, bool to_cache,
                    cudaStream_t st);

// ---- one-row int8 lm_head + greedy argmax (kernels_lmhead.cu) ----
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();  // the driver's cuTensorMapEncodeTiled (or null)
bool lm_head_m1_supported(int H, int V);
size_t lm_head_m1_part_bytes(int V);  // scratch for the per-block argmax states
int lm_head_m1_prepare(int H);        // outside graph capture; 0 on success
int lm_head_m1_make_tmap(const int8_t* W, int V, int H, CUtensorMap* map);  // 0 on success
// logits[v] = dot_f32_i8w(W[v], h) * scales[v] for one row h, and *next = their greedy argmax.
void launch_lm_head_m1(const CUtensorMap& map, const float* h, const float* scales, int V, int H, float* out,
                       void* part, uint32_t* next, int32_t* status, cudaStream_t st);

// ---- whole-layer-stack decode of one token (kernels_decode1.cu) ----
// Per layer: the device weights of the four projections (qkv, o, gate/up,
// down), the four norm gains (attn_norm, attn_sub_norm, ffn_norm,
// ffn_sub_norm) and the seven per-tensor scales.
struct D1Layer {
  const uint32_t* w[4];
  const float* norm[4];
  float sq, sk, sv, so, sg, su, sd, pad;
};
struct D1Params {
  const D1Layer* layers = nullptr;  // device array [L]
  int L = 0, H = 0, nh = 0, nkv = 0, F = 0, V = 0;
  float eps = 0.0f;
  // shared-memory plan (decode1_plan): matmul CTAs' weight slots, norm row
  // and int8 row; attention CTAs' ring slots and score rows
  uint32_t slot_off[4] = {0, 0, 0, 0}, slot_bytes[4] = {0, 0, 0, 0};
  uint32_t row_off = 0, xq_off = 0, hown_off = 0, sc_off = 0;
  int hpc = 0;  // query heads per attention CTA (decode1_hpc)
  int ring_slots = 0, cap = 0;
  const uint16_t* embed = nullptr;  // [V][H] bf16
  const uint32_t* token = nullptr;  // the token (device)
  const int32_t *tok_pos = nullptr, *tok_seq = nullptr, *page_table = nullptr;
  KvGeom g;
  const float *rope_cos = nullptr, *rope_sin = nullptr;  // [max_pos][64]
  ExpTable et;
  float *h = nullptr, *qkv = nullptr, *attn = nullptr, *gu = nullptr;  // [H], [q+2kv], [q], [2F]
  const float* final_norm = nullptr;  // with hn: the final RMSNorm of h is written to hn [H]
  float* hn = nullptr;
  int32_t* status = nullptr;
  uint32_t* sync = nullptr;  // decode1_sync_bytes(), zeroed before every launch
};
// Query heads per attention CTA: the smallest divisor of the GQA group (1, 2,
// 4 or 8) that keeps the attention CTAs to 32; 0 when the group is unsupported.
int decode1_hpc(int nh, int nkv);
bool decode1_supported(int nh, int nkv, int H, int F, const KvGeom& g);
// Fills the shared-memory plan (and hpc) for `sms` CTAs and contexts of up to
// `cap` positions; the dynamic shared memory of the launch, 0 if over smem_limit.
size_t decode1_plan(D1Params* P, int sms, int cap, size_t smem_limit);
size_t decode1_smem_limit(int hpc);  // raises the kernel's limit; outside graph capture; 0 on failure
bool decode1_fits(int hpc, int grid, size_t smem);  // all `grid` CTAs co-resident
size_t decode1_sync_bytes();
// Cooperative launch of `grid` CTAs (grid - nh / hpc matmul CTAs); 0 on success.
int launch_decode1(const D1Params& P, const CUtensorMap& tmap, int grid, size_t smem, cudaStream_t st);

}  // namespace bitnet
