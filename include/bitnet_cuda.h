/*
 * bitnet_cuda.h — C ABI of the B200 (sm_100a) backend for bitnetrs.
 *
 * The library is a drop-in for the reference's operator boundary, the Rust
 * trait `bitnet_core::backend::Backend` (crates/bitnet-core/src/backend/mod.rs:128-517),
 * selected by `Device::Gpu { device_id }` in `create_backend`
 * (crates/bitnet-model/src/device.rs:79-121).  Every trait method has one
 * entry point below taking plain host pointers plus the length of every
 * slice, so the Rust shim can forward `&[T]` / `&mut [T]` without copies and
 * the library can reproduce the reference's shape validation.
 *
 * Beyond the trait, the library keeps weights and a paged KV cache resident
 * in HBM and exposes whole-forward entry points (BitNetModel::forward_into,
 * batched decode / prefill, greedy generate) — the reference's per-op host
 * slices cannot reach the device roofline.
 *
 * Conventions
 *  - Return value: BITNET_OK or one of the error codes, mirroring the
 *    BitNetError variants (crates/bitnet-core/src/error.rs:12-60).  The
 *    message of the last failure on the calling thread is returned by
 *    bitnet_cuda_last_error().  No entry point aborts the process and none
 *    falls back to the CPU.
 *  - Host pointers are only read/written during the call.  Outputs are
 *    caller-allocated and overwritten.
 *  - Entry points suffixed _device take device pointers and a cudaStream_t
 *    (passed as void*; NULL selects the context's stream) and return without
 *    synchronising.
 *  - A context is bound to one GPU.  Calls on one context are serialised by
 *    an internal mutex, so the handle is Send + Sync like the trait requires.
 */
#ifndef BITNET_CUDA_H
#define BITNET_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- error codes (BitNetError, crates/bitnet-core/src/error.rs:12-60) ---- */
#define BITNET_OK 0
#define BITNET_ERR_INVALID_SHAPE 1  /* BitNetError::InvalidShape { expected, got } */
#define BITNET_ERR_QUANTIZATION 2   /* BitNetError::QuantizationError(msg)          */
#define BITNET_ERR_BACKEND 3        /* BitNetError::BackendError { "CUDA", msg }     */
#define BITNET_ERR_INVALID_CONFIG 4 /* BitNetError::InvalidConfig(msg)              */

typedef struct bitnet_cuda_ctx bitnet_cuda_ctx;
typedef struct bitnet_cuda_model bitnet_cuda_model;
typedef struct bitnet_cuda_kv bitnet_cuda_kv;
typedef struct bitnet_cuda_weight bitnet_cuda_weight;

/* ===================================================================== */
/* Lifecycle                                                              */
/* ===================================================================== */

/* Replaces CudaBackend::new (crates/bitnet-gpu-cuda/src/lib.rs:94-104), which
 * is a stub in the reference; device_id is the CUDA ordinal. */
int bitnet_cuda_create(uint32_t device_id, bitnet_cuda_ctx** out);
void bitnet_cuda_destroy(bitnet_cuda_ctx* ctx);

/* Backend::device_name (mod.rs:516). */
const char* bitnet_cuda_device_name(const bitnet_cuda_ctx* ctx);

/* Message of the last failing call made by this thread ("" if none). */
const char* bitnet_cuda_last_error(void);

/* The two fields of BitNetError::InvalidShape { expected, got }
 * (crates/bitnet-core/src/error.rs:17-18) when the last failing call of this
 * thread returned BITNET_ERR_INVALID_SHAPE; "" after any other error.  The
 * message above is their Display form ("expected {expected}, got {got}"). */
const char* bitnet_cuda_last_error_expected(void);
const char* bitnet_cuda_last_error_got(void);

/* Library version string. */
const char* bitnet_cuda_version(void);

/* cudaFuncAttributes::binaryVersion of the library's kernels on the current
 * device: the SASS architecture the driver loaded them for (major * 10 +
 * minor; 100 for the sm_100a build).  No counterpart in the reference. */
int bitnet_cuda_kernel_binary_version(int32_t* out);

/* ===================================================================== */
/* Backend trait methods (host slices)                                    */
/* ===================================================================== */

/* Backend::ternary_gemv (mod.rs:152-160); CpuBackend: gemv.rs:108-165.
 * out[i] = ws * sum_j W[i,j] * x[j], f32 accumulation in the reference's order. */
int bitnet_cuda_ternary_gemv(bitnet_cuda_ctx* ctx, const uint8_t* weight_packed, size_t weight_len,
                             float weight_scale, const float* input, size_t input_len, float* output,
                             size_t output_len, size_t out_features, size_t in_features);

/* Backend::ternary_gemv_with_activation_quant (mod.rs:185-207); CpuBackend
 * override cpu/src/lib.rs:223-249 (absmax int8 quantisation + int32 GEMV). */
int bitnet_cuda_ternary_gemv_with_activation_quant(bitnet_cuda_ctx* ctx, const uint8_t* weight_packed,
                                                   size_t weight_len, float weight_scale, const float* input,
                                                   size_t input_len, float* output, size_t output_len,
                                                   size_t out_features, size_t in_features);

/* Backend::rms_norm (mod.rs:225); cpu/src/norm.rs:77-137. */
int bitnet_cuda_rms_norm(bitnet_cuda_ctx* ctx, const float* input, size_t input_len, const float* weight,
                         size_t weight_len, float eps, float* output, size_t output_len);

/* Backend::rope_embed (mod.rs:251-260); cpu/src/lib.rs:289-314 + rope.rs:312-355.
 * q and k are rotated in place (half-split convention). */
int bitnet_cuda_rope_embed(bitnet_cuda_ctx* ctx, float* q, size_t q_len, float* k, size_t k_len, size_t position,
                           size_t head_dim, size_t n_heads, size_t n_kv_heads, float theta);

/* Backend::masked_attention (mod.rs:301-311); cpu/src/attention.rs:97-209.
 * k_cache / v_cache are head-major [n_kv_heads][max_seq][head_dim]. */
int bitnet_cuda_masked_attention(bitnet_cuda_ctx* ctx, const float* q, size_t q_len, const float* k_cache,
                                 size_t k_len, const float* v_cache, size_t v_len, float* output, size_t output_len,
                                 size_t n_heads, size_t n_kv_heads, size_t head_dim, size_t cur_pos);

/* Backend::squared_relu (mod.rs:324); cpu/src/activation.rs:92. In place. */
int bitnet_cuda_squared_relu(bitnet_cuda_ctx* ctx, float* x, size_t len);

/* Backend::softmax (mod.rs:338); cpu/src/activation.rs:230. In place. */
int bitnet_cuda_softmax(bitnet_cuda_ctx* ctx, float* x, size_t len);

/* Backend::elementwise_mul (mod.rs:350); cpu/src/lib.rs:400-420. */
int bitnet_cuda_elementwise_mul(bitnet_cuda_ctx* ctx, const float* a, size_t a_len, const float* b, size_t b_len,
                                float* out, size_t out_len);

/* Backend::lm_head_matmul_into (mod.rs:372-383); cpu/src/lib.rs:426-447. */
int bitnet_cuda_lm_head_matmul_into(bitnet_cuda_ctx* ctx, const float* hidden, size_t hidden_len,
                                    const float* weights, size_t weights_len, float* output, size_t output_len,
                                    size_t vocab_size, size_t hidden_size);

/* Backend::lm_head_matmul_bf16_into (mod.rs:399-420); cpu/src/lib.rs:455-488.
 * weights are raw bf16 bit patterns. */
int bitnet_cuda_lm_head_matmul_bf16_into(bitnet_cuda_ctx* ctx, const float* hidden, size_t hidden_len,
                                         const uint16_t* weights_bf16, size_t weights_len, float* output,
                                         size_t output_len, size_t vocab_size, size_t hidden_size);

/* Backend::sqrelu_gate (mod.rs:432-444); cpu/src/lib.rs:494-509. */
int bitnet_cuda_sqrelu_gate(bitnet_cuda_ctx* ctx, const float* gate, size_t gate_len, const float* up, size_t up_len,
                            float* out, size_t out_len);

/* Backend::ternary_gemv_preq (mod.rs:459-468); cpu/src/lib.rs:519-538 -> gemv.rs:251-311.
 * out[i] = (sum_j W[i,j]*x_q[j]) as f32 * (weight_scale*act_absmax/127). */
int bitnet_cuda_ternary_gemv_preq(bitnet_cuda_ctx* ctx, const uint8_t* weight_packed, size_t weight_len,
                                  float weight_scale, const int8_t* activation_q, size_t activation_len,
                                  float act_absmax, float* output, size_t output_len, size_t out_features,
                                  size_t in_features);

/* Backend::lm_head_matmul_i8_into (mod.rs:486-509); cpu/src/lib.rs:544-575. */
int bitnet_cuda_lm_head_matmul_i8_into(bitnet_cuda_ctx* ctx, const float* hidden, size_t hidden_len,
                                       const int8_t* weights_i8, size_t weights_len, const float* scales,
                                       size_t scales_len, float* output, size_t output_len, size_t vocab_size,
                                       size_t hidden_size);

/* ---- hot-path helpers that the reference calls outside the trait ---- */

/* absmax_quantize_row_into (crates/bitnet-core/src/quant/absmax.rs:127-165):
 * the model quantises once per projection group (model/src/lib.rs:957-962). */
int bitnet_cuda_absmax_quantize_row(bitnet_cuda_ctx* ctx, const float* x, size_t len, int8_t* out, size_t out_len,
                                    float* scale);

/* ternary_gemv_preq that also returns the int32 accumulators
 * (gemv.rs:299-308 `acc`), for bit-exact parity checks. acc may be NULL. */
int bitnet_cuda_ternary_gemv_preq_acc(bitnet_cuda_ctx* ctx, const uint8_t* weight_packed, size_t weight_len,
                                      float weight_scale, const int8_t* activation_q, size_t activation_len,
                                      float act_absmax, float* output, size_t output_len, int32_t* acc,
                                      size_t out_features, size_t in_features);

/* Greedy sample_next_token (crates/bitnet-inference/src/lib.rs:263-274):
 * argmax with ties resolved to the last index, NaN comparing Equal. */
int bitnet_cuda_greedy_argmax(bitnet_cuda_ctx* ctx, const float* logits, size_t len, uint32_t* token);

/* SamplingConfig (crates/bitnet-inference/src/lib.rs:80-112); max_new_tokens
 * is the generate call's own argument. */
typedef struct {
  float temperature;
  float top_p;
  uint32_t top_k;
  float repetition_penalty;
  uint64_t seed;
} bitnet_cuda_sampling;

/* sample_next_token (crates/bitnet-inference/src/lib.rs:236-390) on the GPU:
 * repetition penalty over past[0..n_past), temperature, the top_k == 1 greedy
 * shortcut, top-k, top-p, softmax and one LCG step (seed + n_past) for the
 * inverse-CDF draw, in the reference's arithmetic order (equal
 * probabilities inside the top-p ordering go in ascending index order; the
 * reference's sort_unstable leaves that order unspecified).  logits (host,
 * len vocab) are modified in place as the reference modifies them.  With
 * top_p < 1, at most 4096 logits may remain finite after top-k, else
 * BackendError. */
int bitnet_cuda_sample_next_token(bitnet_cuda_ctx* ctx, float* logits, size_t vocab, const bitnet_cuda_sampling* cfg,
                                  const uint32_t* past, size_t n_past, uint32_t* token);

/* ===================================================================== */
/* Device-resident ternary matmul (op sweep, composition)                 */
/* ===================================================================== */

/* Upload one TernaryWeight (crates/bitnet-core/src/quant/ternary.rs:82-91):
 * rows*ceil(cols/4) bytes in the reference's 2-bit format; it is repacked once
 * into the device layout. */
int bitnet_cuda_weight_upload(bitnet_cuda_ctx* ctx, const uint8_t* packed, size_t packed_len, size_t rows,
                              size_t cols, float scale, bitnet_cuda_weight** out);
void bitnet_cuda_weight_destroy(bitnet_cuda_weight* w);

/* Per-token absmax quantisation of M rows (absmax.rs:127-165 per row):
 * x: device f32 [M][K] (row stride K) or bf16 when x_is_bf16 != 0.
 * xq: device int8 [M][ldq] (ldq >= K, multiple of 64; tail zero-filled),
 * act_absmax: device f32 [M] (the `scale*127` value the model passes on),
 * row_sum: device int32 [M] (sum of xq, used by the matmul),
 * status: device int32 (set non-zero if a row holds a non-finite value). */
int bitnet_cuda_quantize_rows_device(bitnet_cuda_ctx* ctx, const void* x, int x_is_bf16, size_t M, size_t K,
                                     int8_t* xq, size_t ldq, float* act_absmax, int32_t* row_sum, int32_t* status,
                                     void* stream);

/* out[m][n] = (sum_k W[n,k] xq[m][k]) * (scale * act_absmax[m] / 127), the
 * batched form of ternary_gemv_quantised (gemv.rs:251-311).  acc (optional)
 * receives the int32 accumulators [M][N]. */
int bitnet_cuda_ternary_matmul_device(bitnet_cuda_ctx* ctx, const bitnet_cuda_weight* w, const int8_t* xq,
                                      size_t ldq, const float* act_absmax, const int32_t* row_sum, size_t M,
                                      float* out, int32_t* acc, void* stream);

/* Decode GEMV with activation quantisation that allocates nothing (no
 * counterpart in the reference): out = ternary_gemv_with_activation_quant of
 * the uploaded weight `w` applied to x, with x (f32, x_len = in_features)
 * and out (f32, out_len = out_features) in device memory.  For callers that
 * must not allocate device memory on their serving path (a cudaMalloc
 * synchronises the device and is not allowed in some host frameworks after
 * warm-up): the activation scratch (int8 row, absmax, code sum, non-finite
 * flag) is a fixed 32 KiB + 256 B array inside this library, so
 * in_features is limited to 32768; longer rows return InvalidShape.  The
 * call resets the scratch's flag itself; nothing has to start at zero.
 *  - The first call on a device resolves the scratch's address; make it
 *    before any stream capture on that device.
 *  - The resolved address is kept for the life of the process: do not use
 *    this entry point across a cudaDeviceReset (or a reset of the primary
 *    context) of that device.
 *  - All calls on one device share the scratch: calls that overlap in time
 *    (other threads, or other streams still running) race; serialise them.
 *  - Runs on `stream` (NULL = the context's stream) and returns after the
 *    result is in `out`; a non-finite x returns QuantizationError, and `out`
 *    is then unspecified (the product has already run on the clamped codes),
 *    unlike the allocating path, which returns before touching `out`. */
int bitnet_cuda_ternary_gemv_quant_noalloc(bitnet_cuda_ctx* ctx, const bitnet_cuda_weight* w, const float* x,
                                           size_t x_len, float* out, size_t out_len, void* stream);

/* ===================================================================== */
/* Device-resident model, paged KV cache, forward / decode / generate     */
/* ===================================================================== */

/* ModelConfig (crates/bitnet-core/src/config.rs:26-62). */
typedef struct {
  uint32_t vocab_size;
  uint32_t hidden_size;
  uint32_t num_hidden_layers;
  uint32_t num_attention_heads;
  uint32_t num_key_value_heads;
  uint32_t intermediate_size;
  uint32_t max_position_embeddings;
  float rope_theta;
  float rms_norm_eps;
} bitnet_cuda_config;

/* LayerWeights (crates/bitnet-weights/src/loader.rs:121-203): packed ternary
 * projections in the reference format plus their per-tensor scales. */
typedef struct {
  const uint8_t *q_proj, *k_proj, *v_proj, *o_proj, *gate_proj, *up_proj, *down_proj;
  float q_scale, k_scale, v_scale, o_scale, gate_scale, up_scale, down_scale;
  const float *attention_norm, *attn_sub_norm, *ffn_norm, *ffn_sub_norm;
} bitnet_cuda_layer_weights;

/* ModelWeights (loader.rs:241-283): bf16 embedding (raw bits), the i8 lm_head
 * (loader.rs:297-340, weight-tied to the embedding) and its per-row scales. */
typedef struct {
  const uint16_t* embed_tokens;
  const int8_t* lm_head_i8;
  const float* lm_head_scales;
  const float* final_norm;
  const bitnet_cuda_layer_weights* layers; /* num_hidden_layers entries */
} bitnet_cuda_weights;

/* BitNetModel::new (crates/bitnet-model/src/lib.rs:462-500): validates the
 * config (config.rs:110-150) and uploads every tensor once. max_batch_tokens
 * bounds the tokens of one forward (decode batch or packed prefill). */
int bitnet_cuda_model_create(bitnet_cuda_ctx* ctx, const bitnet_cuda_config* config, const bitnet_cuda_weights* w,
                             uint32_t max_batch_tokens, bitnet_cuda_model** out);
void bitnet_cuda_model_destroy(bitnet_cuda_model* model);

/* Tensor parallelism for models too large for one device (no counterpart in
 * the reference, which runs on one device).  Rank `rank` of `world` keeps the
 * q/k/v rows of its num_attention_heads/world query heads and
 * num_key_value_heads/world KV heads, the gate/up rows of its
 * intermediate_size/world slice, and the matching input columns of o_proj and
 * down_proj; per-tensor scales stay those of the full tensors.  Every layer
 * all-gathers the attention output and the gated FFN activation, so that both
 * sub-norms and their int8 quantisation run over the full row in the
 * reference's order, and all-reduces the int32 accumulators of o_proj and
 * down_proj (exact), so every rank's hidden state is bit-identical to the
 * single-device model's.  Collectives run over NCCL, loaded at run time
 * (the process's libnccl.so.2, or BITNET_NCCL_LIBRARY).
 *
 * bitnet_cuda_tp_unique_id writes BITNET_TP_ID_BYTES bytes on one rank; every
 * rank then calls bitnet_cuda_model_create_tp with those bytes and the FULL
 * host weights (collective: all ranks call it together), and every later
 * forward, prefill and decode step on all ranks together with the same
 * batch.  Tensor-parallel decode steps run as CUDA graphs holding the NCCL
 * calls (prefill and forward launch eagerly).  A
 * rank's KV cache holds only its KV heads: bitnet_cuda_kv_seq_write / _read
 * take [layer][pos][local_kv_heads*head_dim] with local_kv_heads =
 * num_key_value_heads/world.
 * Requirements: num_attention_heads and num_key_value_heads divisible by
 * world, and
 * (hidden_size/num_attention_heads)*num_attention_heads/world and
 * intermediate_size/world multiples of 64 (InvalidConfig otherwise). */
#define BITNET_TP_ID_BYTES 128
int bitnet_cuda_tp_unique_id(uint8_t* id, size_t id_len);
int bitnet_cuda_model_create_tp(bitnet_cuda_ctx* ctx, const bitnet_cuda_config* config, const bitnet_cuda_weights* w,
                                uint32_t max_batch_tokens, uint32_t rank, uint32_t world, const uint8_t* nccl_id,
                                size_t id_len, bitnet_cuda_model** out);

/* ===================================================================== */
/* Checkpoint ingestion (host only; no context needed)                    */
/* ===================================================================== */

/* decode_packed_projection (crates/bitnet-convert/src/lib.rs:235-325): the
 * HuggingFace packed projection [packed_rows][cols] u8 -- byte (r, c) holds at
 * bits 2s..2s+1 the lane of logical row s*packed_rows + r, value lane - 1 --
 * into the reference runtime rows [4*packed_rows][ceil(cols/4)]
 * (ternary.rs:266-285) that bitnet_cuda_model_create takes.  weight_scale
 * (the checkpoint's *_scale) is only validated: it is the tensor's scale as
 * is.  Errors: zero sizes or short buffers (InvalidShape); a non-positive or
 * non-finite scale, or a lane 0b11 (QuantizationError, first position in the
 * reference's scan order). */
int bitnet_cuda_decode_hf_packed(const uint8_t* packed, size_t packed_len, size_t packed_rows, size_t cols,
                                 float weight_scale, uint8_t* out, size_t out_len);

/* quantise_weight (crates/bitnet-weights/src/loader.rs:1037-1070) for the bf16
 * checkpoint: absmean ternarisation (absmean.rs:71-102) of a dense f32
 * [rows][cols] tensor into reference runtime rows; *scale receives the
 * per-tensor scale.  Empty or non-finite input: QuantizationError. */
int bitnet_cuda_absmean_ternary(const float* w, size_t rows, size_t cols, uint8_t* out, size_t out_len,
                                float* scale);

/* quantize_bf16_rows_to_i8 (crates/bitnet-weights/src/loader.rs:297-340): the
 * i8 table and per-row scales of the lm_head, weight-tied to the bf16
 * embedding [rows][row_len] (raw bits). */
int bitnet_cuda_lm_head_i8_table(const uint16_t* embed_bf16, size_t rows, size_t row_len, int8_t* out,
                                 float* scales);

#define BITNET_KV_F32 0  /* the reference KVCache element type (model/src/lib.rs:118-169) */
#define BITNET_KV_BF16 1 /* paged bf16 cache */

/* Paged KV cache (replaces KVCache, model/src/lib.rs:118-315): num_pages pages
 * of 16 positions x all layers, shared by up to max_seqs sequences. */
int bitnet_cuda_kv_create(bitnet_cuda_model* model, uint32_t num_pages, uint32_t max_seqs, int kv_dtype,
                          bitnet_cuda_kv** out);
void bitnet_cuda_kv_destroy(bitnet_cuda_kv* kv);
/* KVCache::clear for one sequence (frees its pages). */
int bitnet_cuda_kv_seq_reset(bitnet_cuda_kv* kv, uint32_t seq);
/* KVCache::len for one sequence. */
int bitnet_cuda_kv_seq_len(bitnet_cuda_kv* kv, uint32_t seq, size_t* len);
/* Number of free pages. */
int bitnet_cuda_kv_free_pages(bitnet_cuda_kv* kv, size_t* n);
/* Seed positions [0, n) of sequence seq from host K/V laid out
 * [layer][pos][n_kv_heads*head_dim] (f32; rounded to bf16 for a bf16 cache). */
int bitnet_cuda_kv_seq_write(bitnet_cuda_kv* kv, uint32_t seq, size_t n, const float* k, const float* v);
/* Read positions [0, n) of sequence seq back in the same layout. */
int bitnet_cuda_kv_seq_read(bitnet_cuda_kv* kv, uint32_t seq, size_t n, float* k, float* v);
/* Seed positions [0, n) with seeded N(0,1) values, generated on the device
 * (continuous-batching benchmark contexts). */
int bitnet_cuda_kv_seq_fill_random(bitnet_cuda_kv* kv, uint32_t seq, size_t n, uint64_t seed);
/* Reserve pages so that sequence seq can grow to `len` positions without
 * further allocation (device-resident decode loops). */
int bitnet_cuda_kv_seq_reserve(bitnet_cuda_kv* kv, uint32_t seq, size_t len);

/* BitNetModel::forward_into (model/src/lib.rs:880-1170) for one sequence:
 * tokens are processed at positions start_pos.. (must equal the sequence's
 * current length); logits (host, vocab_size) receive the last token's logits. */
int bitnet_cuda_forward(bitnet_cuda_model* model, bitnet_cuda_kv* kv, uint32_t seq, const uint32_t* tokens,
                        size_t n_tokens, size_t start_pos, float* logits);

/* One decode step for `batch` sequences (one new token each, at each
 * sequence's current length).  logits (host [batch][vocab], may be NULL) and
 * next_tokens (host [batch], greedy argmax, may be NULL) are outputs. */
int bitnet_cuda_decode_step(bitnet_cuda_model* model, bitnet_cuda_kv* kv, size_t batch, const uint32_t* seq_ids,
                            const uint32_t* tokens, float* logits, uint32_t* next_tokens);

/* Device-resident decode step: seq_ids on the host (scheduler state),
 * tokens / next_tokens / logits in device memory.  next_tokens may alias
 * tokens.  Runs as one CUDA graph per batch size. */
int bitnet_cuda_decode_step_device(bitnet_cuda_model* model, bitnet_cuda_kv* kv, size_t batch,
                                   const uint32_t* seq_ids, const uint32_t* d_tokens, uint32_t* d_next_tokens,
                                   float* d_logits, void* stream);

/* Ragged prefill of n_seqs sequences packed back to back (tokens of sequence
 * i are tokens[cu_seqlens[i] .. cu_seqlens[i+1])), appended at each
 * sequence's current length.  logits (host [n_seqs][vocab], may be NULL) and
 * next_tokens (host [n_seqs], may be NULL) are for each sequence's last token. */
int bitnet_cuda_prefill(bitnet_cuda_model* model, bitnet_cuda_kv* kv, size_t n_seqs, const uint32_t* seq_ids,
                        const uint32_t* tokens, const uint32_t* cu_seqlens, float* logits, uint32_t* next_tokens);

/* generate_from_tokens_streaming (crates/bitnet-inference/src/lib.rs:701-777)
 * with greedy sampling: clear the sequence, prefill the prompt, then decode
 * until max_new tokens or eos0/eos1.  out_tokens holds up to max_new ids. */
int bitnet_cuda_generate(bitnet_cuda_model* model, bitnet_cuda_kv* kv, uint32_t seq, const uint32_t* prompt,
                         size_t n_prompt, size_t max_new, uint32_t eos0, uint32_t eos1, uint32_t* out_tokens,
                         size_t* n_out);

/* The same loop with sample_next_token on the device: the sampling config
 * is validated as SamplingConfig::validate (lib.rs:160-178) does, and every
 * step samples from the last logits with the prompt and the tokens generated
 * so far as the repetition history (lib.rs:721-733). */
int bitnet_cuda_generate_sampled(bitnet_cuda_model* model, bitnet_cuda_kv* kv, uint32_t seq, const uint32_t* prompt,
                                 size_t n_prompt, size_t max_new, const bitnet_cuda_sampling* cfg, uint32_t eos0,
                                 uint32_t eos1, uint32_t* out_tokens, size_t* n_out);

/* Numerics of the model's forward passes.  The ternary matmul, activation
 * quantisation, norms, RoPE and residual adds are bit-identical to the
 * reference CPU backend in every mode.
 *  AUTO  (default): attention in the reference's operation order (bit-
 *        identical except the exp, which is correctly rounded where glibc's
 *        expf may differ by one ulp); the lm_head of steps with more than 16
 *        output rows on tensor cores (every product exact, f32 accumulation
 *        in a different order: ~1e-7 relative), otherwise reference order.
 *  EXACT: reference operation order everywhere.
 *  FAST : tensor-core attention and lm_head at every size (f32-level
 *        accuracy; int8 re-quantisation then drifts from the reference over
 *        long sequences). */
#define BITNET_NUMERICS_AUTO 0
#define BITNET_NUMERICS_EXACT 1
#define BITNET_NUMERICS_FAST 2
int bitnet_cuda_model_set_numerics(bitnet_cuda_model* model, int mode);

/* One-token steps (decode at batch 1, a one-token forward) run every layer
 * as one persistent kernel when the model and cache fit it: not tensor-
 * parallel, a bf16 cache, head_dim 128, 1/2/4/8 query heads per kv head, and
 * the numerics mode is not FAST.  Same operations and order as the per-layer
 * kernels, so the same results bit for bit.  Enabled by default; 0 selects
 * the per-layer kernels (for comparison).  No counterpart in the reference. */
int bitnet_cuda_model_set_fused_decode(bitnet_cuda_model* model, int enable);

/* Per-kernel-class device timing of device-resident decode steps.  When
 * enabled, decode graphs captured afterwards record CUDA events around every
 * kernel launch; bitnet_cuda_model_kernel_times then returns, for the most
 * recent timed step, the summed device time (ms) and the launch count of each
 * class: [0] attention, [1] ternary matmul, [2] RMSNorm+quantise,
 * [3] RoPE + KV store, [4] lm_head, [5] other, [6] the fused layer stack of
 * a one-token step (decode1_kernel).  Arrays hold 7 entries. */
int bitnet_cuda_model_set_kernel_timing(bitnet_cuda_model* model, int enable);
int bitnet_cuda_model_kernel_times(bitnet_cuda_model* model, float* ms, int32_t* launches);

/* Synchronise the model's stream and report (then clear) a non-finite
 * activation (QuantizationError) or out-of-range token id (InvalidShape) seen
 * by device-resident steps since the last check, and a device-side wait that
 * gave up or a context beyond the attention kernel's capacity (BackendError). */
int bitnet_cuda_model_check(bitnet_cuda_model* model);

/* Diagnostics (no counterpart in the reference): writes into `name` (NUL
 * terminated, at most name_len bytes) the name of the attention kernel that a
 * step of `tokens` query tokens over `kv` launches under the current numerics
 * mode, for contexts up to the cache's capacity. */
int bitnet_cuda_model_attention_kernel(bitnet_cuda_model* model, bitnet_cuda_kv* kv, uint32_t tokens, char* name,
                                       size_t name_len);

/* Number of kernels this library launched on the context (all entry points,
 * graph-launched kernels included). */
uint64_t bitnet_cuda_kernel_launches(const bitnet_cuda_ctx* ctx);

#ifdef __cplusplus
}
#endif

#endif /* BITNET_CUDA_H */
