// internal.h — host-side structures shared by the C-ABI translation units.
#pragma once

#include <atomic>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "kernels.cuh"

namespace bitnet {

// Grow-only device buffer.
struct DevBuf {
  void* p = nullptr;
  size_t cap = 0;
  int ensure(size_t bytes);
  template <class T>
  T* as() const {
    return static_cast<T*>(p);
  }
  void release();
  ~DevBuf() { release(); }
};

// RoPE table with the reuse rule of CpuBackend::rope_embed (cpu/src/lib.rs:289-314):
// rebuilt when head_dim changes, theta moves by more than 1e-3, or pos >= max_seq.
struct RopeTable {
  bool valid = false;
  size_t head_dim = 0, max_seq = 0;
  float theta = 0.0f;
  std::vector<float> cos, sin;  // [max_seq][head_dim/2], glibc powf/cosf/sinf
  DevBuf d_cos, d_sin;
};

// Fill cos/sin for positions [0, max_seq) exactly as RopeCache::new (rope.rs:100-147).
int build_rope_host(size_t max_seq, size_t head_dim, float theta, std::vector<float>& cos, std::vector<float>& sin);

}  // namespace bitnet

// Handles are reference counted: models and uploaded weights keep their
// context alive and KV caches keep their model alive, so the public destroy
// functions may be called in any order.
struct bitnet_cuda_ctx {
  std::atomic<int> refs{1};
  int device = 0;
  cudaStream_t stream = nullptr;
  std::mutex mu;
  std::string name;
  bitnet::DevBuf b[8];  // scratch for the per-call trait methods
  bitnet::DevBuf status;
  bitnet::RopeTable rope;
  // host-libm expf exceptions (see ExpTable); built once per context
  bool exp_ready = false;
  bitnet::DevBuf exp_keys, exp_vals, exp_hash, exp_en, exp_fj;
  bitnet::ExpTable exp_table;
  // device sampler scratch: occurrence counts [vocab] (kept at zero between
  // calls), exp values [vocab], token + status words
  bitnet::DevBuf samp_counts, samp_e, samp_misc;
};

struct bitnet_cuda_weight {
  bitnet_cuda_ctx* ctx = nullptr;
  int rows = 0, cols = 0;
  float scale = 0.0f;
  uint32_t* words = nullptr;
};

namespace bitnet {
void ctx_retain(bitnet_cuda_ctx* c);
void ctx_release(bitnet_cuda_ctx* c);
// Builds ctx->exp_table on first use (caller holds ctx->mu, not capturing).
int ensure_exp_table(bitnet_cuda_ctx* c);
// sample_next_token on device logits [vocab] (modified in place) with the
// device history past[0..n_past); the token comes back to *token (host).
// Caller holds ctx->mu; synchronises st.
int sample_device(bitnet_cuda_ctx* c, float* d_logits, size_t vocab, const bitnet_cuda_sampling& cfg,
                  const uint32_t* d_past, size_t n_past, uint32_t* token, cudaStream_t st);
// SamplingConfig::validate (crates/bitnet-inference/src/lib.rs:160-178).
int validate_sampling(const bitnet_cuda_sampling& cfg, size_t max_new_tokens);
}  // namespace bitnet
