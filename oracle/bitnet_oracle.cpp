// bitnet_oracle.cpp — CPU restatement of the bitnetrs reference CPU backend.
//
// TEST INFRASTRUCTURE, NOT PRODUCT CODE.  This library is the parity checker
// for the CUDA backend and the timed CPU baseline.  Only tests/,
// __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm load it.
//
// What it restates (paths relative to the bitnetrs workspace root):
//   crates/bitnet-core/src/quant/ternary.rs   pack_ternary / unpack_ternary
//   crates/bitnet-core/src/quant/absmean.rs   absmean_quantize
//   crates/bitnet-core/src/quant/absmax.rs    absmax_quantize_row_into
//   crates/bitnet-cpu/src/simd.rs             AVX2/FMA kernels, same intrinsics in the same order
//   crates/bitnet-cpu/src/gemv.rs             ternary_gemv_f32 / ternary_gemv_quantised
//   crates/bitnet-cpu/src/norm.rs             rms_norm
//   crates/bitnet-cpu/src/rope.rs             RopeCache + half-split rotation
//   crates/bitnet-cpu/src/attention.rs        masked_attention
//   crates/bitnet-core/src/backend/ops.rs     softmax_f32
//   crates/bitnet-cpu/src/activation.rs       squared_relu / softmax
//   crates/bitnet-cpu/src/lib.rs              CpuBackend (validation order, RoPE cache reuse)
//   crates/bitnet-model/src/lib.rs            KVCache, BitNetModel::forward / forward_into
//   crates/bitnet-inference/src/lib.rs        sample_next_token (greedy and full), generate loop
//   crates/bitnet-convert/src/lib.rs          decode_packed_projection (HF packed layout)
//
// Floating point: compiled with -ffp-contract=off so scalar `a*b+c` stays two
// roundings, as in Rust; FMA appears only where the reference calls
// _mm256_fmadd_ps.  Threads split rows/heads exactly like Rayon does; results
// are independent of the thread count because every output element is
// computed by a single thread in a fixed order.
//
// Parity pinning: the known-answer vectors transcribed from the reference's
// own unit tests live in tests/golden/kats.json and are checked by
// tests/test_oracle_kats.py.

#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <functional>
#include <limits>
#include <mutex>
#include <thread>
#include <vector>

namespace {

// Error codes shared with include/bitnet_cuda.h (BitNetError variants).
enum : int {
  OK = 0,
  ERR_SHAPE = 1,   // BitNetError::InvalidShape
  ERR_QUANT = 2,   // BitNetError::QuantizationError
  ERR_BACKEND = 3, // BitNetError::BackendError
  ERR_CONFIG = 4,  // BitNetError::InvalidConfig
};

// ---------------------------------------------------------------------------
// Thread pool: a static-partition parallel_for standing in for Rayon.
// ---------------------------------------------------------------------------
class Pool {
 public:
  explicit Pool(int n) { resize(n); }
  ~Pool() { stop(); }

  void resize(int n) {
    stop();
    if (n <= 0) n = (int)std::max(1u, std::thread::hardware_concurrency());
    nthreads_ = n;
    quit_ = false;
    for (int i = 1; i < n; ++i) workers_.emplace_back([this, i] { loop(i); });
  }
  int size() const { return nthreads_; }

  // body(begin, end) over [0, n) split into contiguous chunks of >= min_len.
  void run(size_t n, size_t min_len, const std::function<void(size_t, size_t)>& body) {
    if (n == 0) return;
    size_t chunks = std::min<size_t>((size_t)nthreads_, (n + min_len - 1) / std::max<size_t>(min_len, 1));
    if (chunks <= 1) {
      body(0, n);
      return;
    }
    std::unique_lock<std::mutex> lk(m_);
    job_ = &body;
    job_n_ = n;
    job_chunks_ = chunks;
    pending_ = (int)chunks - 1;
    ++gen_;
    lk.unlock();
    cv_.notify_all();
    run_chunk(0);
    lk.lock();
    done_cv_.wait(lk, [this] { return pending_ == 0; });
    job_ = nullptr;
  }

 private:
  void run_chunk(size_t c) {
    size_t per = (job_n_ + job_chunks_ - 1) / job_chunks_;
    size_t b = c * per, e = std::min(job_n_, b + per);
    if (b < e) (*job_)(b, e);
  }
  void loop(int idx) {
    uint64_t seen = 0;
    for (;;) {
      std::unique_lock<std::mutex> lk(m_);
      cv_.wait(lk, [&] { return quit_ || gen_ != seen; });
      if (quit_) return;
      seen = gen_;
      if ((size_t)idx >= job_chunks_) continue;
      lk.unlock();
      run_chunk((size_t)idx);
      lk.lock();
      if (--pending_ == 0) done_cv_.notify_all();
    }
  }
  void stop() {
    {
      std::lock_guard<std::mutex> lk(m_);
      quit_ = true;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
    workers_.clear();
  }

  int nthreads_ = 1;
  std::vector<std::thread> workers_;
  std::mutex m_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(size_t, size_t)>* job_ = nullptr;
  size_t job_n_ = 0, job_chunks_ = 0;
  int pending_ = 0;
  uint64_t gen_ = 0;
  bool quit_ = false;
};

Pool& pool() {
  static Pool p(0);
  return p;
}

template <class F>
void par_for(size_t n, size_t min_len, F f) {
  std::function<void(size_t, size_t)> body = [&](size_t b, size_t e) {
    for (size_t i = b; i < e; ++i) f(i);
  };
  pool().run(n, min_len, body);
}

// ---------------------------------------------------------------------------
// Scalar helpers with Rust semantics.
// ---------------------------------------------------------------------------
inline float bf16_to_f32(uint16_t b) {  // half::bf16 -> f32: bits << 16
  uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
inline float rust_max(float a, float b) { return std::fmax(a, b); }  // f32::max (NaN-ignoring)
inline bool finite(float v) { return std::isfinite(v); }

// ---------------------------------------------------------------------------
// simd.rs restatements.
// ---------------------------------------------------------------------------

// hsum_f32_avx2 (simd.rs:292-307): lo+hi, movehdup add, movehl add_ss.
inline float hsum_f32(__m256 v) {
  __m128 hi128 = _mm256_extractf128_ps(v, 1);
  __m128 lo128 = _mm256_castps256_ps128(v);
  __m128 sum128 = _mm_add_ps(lo128, hi128);
  __m128 shuf = _mm_movehdup_ps(sum128);
  __m128 sum2 = _mm_add_ps(sum128, shuf);
  __m128 shuf2 = _mm_movehl_ps(sum2, sum2);
  __m128 sum1 = _mm_add_ss(sum2, shuf2);
  return _mm_cvtss_f32(sum1);
}

inline int32_t hsum_i32(__m256i v) {  // simd.rs:271-286
  __m128i hi128 = _mm256_extracti128_si256(v, 1);
  __m128i lo128 = _mm256_castsi256_si128(v);
  __m128i sum128 = _mm_add_epi32(lo128, hi128);
  __m128i hi64 = _mm_unpackhi_epi64(sum128, sum128);
  __m128i sum64 = _mm_add_epi32(sum128, hi64);
  __m128i hi32 = _mm_shuffle_epi32(sum64, 0x01);
  __m128i sum32 = _mm_add_epi32(sum64, hi32);
  return _mm_cvtsi128_si32(sum32);
}

// dot_ternary_i8_avx2 (simd.rs:118-171): VPMOVSXBW, VPSIGNW, VPMADDWD.
int32_t dot_ternary_i8(const int8_t* w, const int8_t* a, size_t len) {
  size_t chunks = len / 16, rem = len % 16;
  __m256i ones = _mm256_set1_epi16(1);
  __m256i acc = _mm256_setzero_si256();
  for (size_t i = 0; i < chunks; ++i) {
    __m128i w128 = _mm_loadu_si128((const __m128i*)(w + i * 16));
    __m128i a128 = _mm_loadu_si128((const __m128i*)(a + i * 16));
    __m256i wi = _mm256_cvtepi8_epi16(w128);
    __m256i ai = _mm256_cvtepi8_epi16(a128);
    __m256i prod = _mm256_sign_epi16(ai, wi);
    acc = _mm256_add_epi32(acc, _mm256_madd_epi16(prod, ones));
  }
  int32_t r = hsum_i32(acc);
  for (size_t i = 0; i < rem; ++i) r += (int32_t)w[chunks * 16 + i] * (int32_t)a[chunks * 16 + i];
  return r;
}

// DECODE_LUT (simd.rs:390-405): code -> {+1, 0, -1, 0}; code 3 decodes as 0.
struct Lut {
  int8_t t[256][4];
  Lut() {
    const int8_t dec[4] = {1, 0, -1, 0};
    for (int b = 0; b < 256; ++b)
      for (int j = 0; j < 4; ++j) t[b][j] = dec[(b >> (2 * j)) & 3];
  }
};
const Lut& lut() {
  static Lut l;
  return l;
}

// unpack_packed_to_i8 (simd.rs:415-445).
void unpack_packed_to_i8(const uint8_t* packed, int8_t* out, size_t n) {
  const Lut& L = lut();
  size_t full = n / 4, rem = n % 4;
  for (size_t i = 0; i < full; ++i) std::memcpy(out + 4 * i, L.t[packed[i]], 4);
  for (size_t j = 0; j < rem; ++j) out[full * 4 + j] = L.t[packed[full]][j];
}

// dot_packed_ternary_i8_avx2_chunked (simd.rs:461-499): 64-element chunks.
int32_t dot_packed_ternary_i8(const uint8_t* packed, const int8_t* act, size_t n) {
  const size_t CH = 64;
  size_t full = n / CH, rem = n % CH;
  int32_t total = 0;
  int8_t buf[CH];
  for (size_t c = 0; c < full; ++c) {
    unpack_packed_to_i8(packed + c * 16, buf, CH);
    total += dot_ternary_i8(buf, act + c * CH, CH);
  }
  if (rem) {
    unpack_packed_to_i8(packed + full * 16, buf, rem);
    for (size_t i = 0; i < rem; ++i) total += (int32_t)buf[i] * (int32_t)act[full * CH + i];
  }
  return total;
}

// dot_ternary_f32_avx2 (simd.rs:190-262): mul, mask w==0 lanes to +0, add.
float dot_ternary_f32(const int8_t* w, const float* x, size_t len) {
  size_t chunks = len / 8, rem = len % 8;
  __m256 acc = _mm256_setzero_ps();
  __m128i zero = _mm_setzero_si128();
  for (size_t i = 0; i < chunks; ++i) {
    __m128i w8 = _mm_loadl_epi64((const __m128i*)(w + i * 8));
    __m256i w32 = _mm256_cvtepi8_epi32(w8);
    __m128i cmp = _mm_cmpeq_epi8(w8, zero);
    __m256 mask = _mm256_castsi256_ps(_mm256_cvtepi8_epi32(cmp));
    __m256 wf = _mm256_cvtepi32_ps(w32);
    __m256 a = _mm256_loadu_ps(x + i * 8);
    __m256 prod = _mm256_mul_ps(wf, a);
    acc = _mm256_add_ps(acc, _mm256_andnot_ps(mask, prod));
  }
  float r = hsum_f32(acc);
  for (size_t i = 0; i < rem; ++i) r += (float)w[chunks * 8 + i] * x[chunks * 8 + i];
  return r;
}

// dot_packed_ternary_f32_avx2_chunked (simd.rs:572-610): 32-element chunks.
float dot_packed_ternary_f32(const uint8_t* packed, const float* x, size_t n) {
  const size_t CH = 32;
  size_t full = n / CH, rem = n % CH;
  float total = 0.0f;
  int8_t buf[CH];
  for (size_t c = 0; c < full; ++c) {
    unpack_packed_to_i8(packed + c * 8, buf, CH);
    total += dot_ternary_f32(buf, x + c * CH, CH);
  }
  if (rem) {
    unpack_packed_to_i8(packed + full * 8, buf, rem);
    for (size_t i = 0; i < rem; ++i) total += (float)buf[i] * x[full * CH + i];
  }
  return total;
}

// dot_f32_f32_avx2 (simd.rs:676-703).
float dot_f32_f32(const float* a, const float* b, size_t len) {
  size_t chunks = len / 8, rem = len % 8;
  __m256 acc = _mm256_setzero_ps();
  for (size_t i = 0; i < chunks; ++i)
    acc = _mm256_fmadd_ps(_mm256_loadu_ps(a + i * 8), _mm256_loadu_ps(b + i * 8), acc);
  float r = hsum_f32(acc);
  for (size_t i = 0; i < rem; ++i) r += a[chunks * 8 + i] * b[chunks * 8 + i];
  return r;
}

// axpy_f32_avx2 (simd.rs:743-770): out = fma(alpha, x, out); scalar tail out += alpha*x.
void axpy_f32(float alpha, const float* x, float* out, size_t len) {
  size_t chunks = len / 8, rem = len % 8;
  __m256 va = _mm256_set1_ps(alpha);
  for (size_t i = 0; i < chunks; ++i) {
    __m256 r = _mm256_fmadd_ps(va, _mm256_loadu_ps(x + i * 8), _mm256_loadu_ps(out + i * 8));
    _mm256_storeu_ps(out + i * 8, r);
  }
  for (size_t i = 0; i < rem; ++i) out[chunks * 8 + i] += alpha * x[chunks * 8 + i];
}

// sum_squares_f32_avx2 (simd.rs:802-826).
float sum_squares_f32(const float* x, size_t len) {
  size_t chunks = len / 8, rem = len % 8;
  __m256 acc = _mm256_setzero_ps();
  for (size_t i = 0; i < chunks; ++i) {
    __m256 v = _mm256_loadu_ps(x + i * 8);
    acc = _mm256_fmadd_ps(v, v, acc);
  }
  float r = hsum_f32(acc);
  for (size_t i = 0; i < rem; ++i) r += x[chunks * 8 + i] * x[chunks * 8 + i];
  return r;
}

// mul_scale_f32_avx2 (simd.rs:846-870): out = (x*scale)*w.
void mul_scale_f32(const float* x, float scale, const float* w, float* out, size_t len) {
  for (size_t i = 0; i < len; ++i) out[i] = (x[i] * scale) * w[i];
}

// dot_f32_bf16w_avx2 (simd.rs:972-1010).
float dot_f32_bf16w(const uint16_t* w, const float* h, size_t len) {
  size_t chunks = len / 8, rem = len % 8;
  __m256 acc = _mm256_setzero_ps();
  for (size_t i = 0; i < chunks; ++i) {
    __m128i wu16 = _mm_loadu_si128((const __m128i*)(w + i * 8));
    __m256i wu32 = _mm256_cvtepu16_epi32(wu16);
    __m256 wf = _mm256_castsi256_ps(_mm256_slli_epi32(wu32, 16));
    acc = _mm256_fmadd_ps(wf, _mm256_loadu_ps(h + i * 8), acc);
  }
  float r = hsum_f32(acc);
  for (size_t i = 0; i < rem; ++i) r += bf16_to_f32(w[chunks * 8 + i]) * h[chunks * 8 + i];
  return r;
}

// dot_f32_i8w_avx2 (simd.rs:1213-1250).
float dot_f32_i8w(const int8_t* w, const float* h, size_t len) {
  size_t chunks = len / 8, rem = len % 8;
  __m256 acc = _mm256_setzero_ps();
  for (size_t i = 0; i < chunks; ++i) {
    __m128i w8 = _mm_loadl_epi64((const __m128i*)(w + i * 8));
    __m256 wf = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(w8));
    acc = _mm256_fmadd_ps(wf, _mm256_loadu_ps(h + i * 8), acc);
  }
  float r = hsum_f32(acc);
  for (size_t i = 0; i < rem; ++i) r += (float)w[chunks * 8 + i] * h[chunks * 8 + i];
  return r;
}

// ---------------------------------------------------------------------------
// quant restatements.
// ---------------------------------------------------------------------------

// absmax_quantize_row_into (absmax.rs:127-165).
int absmax_quantize_row_into(const float* x, size_t n, int8_t* out, size_t out_len, float* scale_out) {
  if (n == 0) return ERR_QUANT;
  if (out_len != n) return ERR_QUANT;
  float max_abs = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    float v = x[i];
    if (!finite(v)) return ERR_QUANT;
    float a = std::fabs(v);
    if (a > max_abs) max_abs = a;
  }
  float mc = rust_max(max_abs, 1e-5f);
  float scale = mc / 127.0f;
  float inv = 127.0f / mc;
  for (size_t i = 0; i < n; ++i) {
    float s = std::round(x[i] * inv);
    s = std::min(std::max(s, -128.0f), 127.0f);
    out[i] = (int8_t)s;
  }
  *scale_out = scale;
  return OK;
}

// ---------------------------------------------------------------------------
// RoPE cache (rope.rs:100-147) with CpuBackend's reuse rule (cpu/lib.rs:289-314).
// ---------------------------------------------------------------------------
struct RopeCache {
  size_t max_seq = 0, head_dim = 0, half = 0;
  float theta = 0.0f;
  std::vector<float> cos, sin;
  bool valid = false;

  int build(size_t ms, size_t hd, float th) {
    if (hd == 0 || hd % 2 != 0) return ERR_CONFIG;
    if (!(th > 0.0f) || !finite(th)) return ERR_CONFIG;
    max_seq = ms;
    head_dim = hd;
    half = hd / 2;
    theta = th;
    cos.assign(ms * half, 0.0f);
    sin.assign(ms * half, 0.0f);
    for (size_t pos = 0; pos < ms; ++pos)
      for (size_t i = 0; i < half; ++i) {
        float exponent = -2.0f * (float)i / (float)hd;
        float freq = std::pow(th, exponent);  // powf
        float angle = (float)pos * freq;
        cos[pos * half + i] = std::cos(angle);
        sin[pos * half + i] = std::sin(angle);
      }
    valid = true;
    return OK;
  }
};

// apply_rope_to_head_slice (rope.rs:414-431).
inline void rope_head(float* x, const float* c, const float* s, size_t half) {
  for (size_t i = 0; i < half; ++i) {
    float lo = x[i], hi = x[i + half];
    x[i] = lo * c[i] - hi * s[i];
    x[i + half] = hi * c[i] + lo * s[i];
  }
}

struct Backend {
  std::mutex rope_mu;
  RopeCache rope;

  // CpuBackend::rope_embed (cpu/lib.rs:289-314).
  int rope_embed(float* q, size_t q_len, float* k, size_t k_len, size_t pos, size_t hd, size_t nh,
                 size_t nkv, float theta) {
    std::lock_guard<std::mutex> lk(rope_mu);
    bool reinit = !rope.valid || rope.head_dim != hd || std::fabs(rope.theta - theta) > 1e-3f ||
                  pos >= rope.max_seq;
    if (reinit) {
      size_t ms = std::max<size_t>(pos + 1, 4096);
      RopeCache fresh;
      int rc = fresh.build(ms, hd, theta);
      if (rc) return rc;
      rope = std::move(fresh);
    }
    // apply_rope_cached (rope.rs:312-355).
    size_t h = rope.head_dim, half = rope.half;
    if (q_len != nh * h) return ERR_SHAPE;
    if (k_len != nkv * h) return ERR_SHAPE;
    if (pos >= rope.max_seq) return ERR_SHAPE;
    const float* c = &rope.cos[pos * half];
    const float* s = &rope.sin[pos * half];
    for (size_t i = 0; i < nh; ++i) rope_head(q + i * h, c, s, half);
    for (size_t i = 0; i < nkv; ++i) rope_head(k + i * h, c, s, half);
    return OK;
  }
};

Backend& backend() {
  static Backend b;
  return b;
}

// softmax_f32 (ops.rs:206-227) == activation::softmax (activation.rs:230).
void softmax_f32(float* x, size_t n) {
  if (n == 0) return;
  float m = -INFINITY;
  for (size_t i = 0; i < n; ++i) m = rust_max(m, x[i]);
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    x[i] = std::exp(x[i] - m);  // expf
    sum += x[i];
  }
  float inv = 1.0f / sum;
  for (size_t i = 0; i < n; ++i) x[i] *= inv;
}

// ternary_gemv_quantised (gemv.rs:251-311); acc_out (optional) receives the i32 sums.
int gemv_quantised(const uint8_t* w, size_t w_len, float ws, const int8_t* xq, size_t xq_len, float act_scale,
                   float* out, size_t out_len, size_t N, size_t K, int32_t* acc_out) {
  size_t pc = (K + 3) / 4;
  if (w_len != N * pc) return ERR_SHAPE;
  if (xq_len != K) return ERR_SHAPE;
  if (out_len != N) return ERR_SHAPE;
  if (!(ws > 0.0f) || !finite(ws)) return ERR_QUANT;
  if (!(act_scale > 0.0f) || !finite(act_scale)) return ERR_QUANT;
  float combined = ws * act_scale / 127.0f;
  par_for(N, 32, [&](size_t r) {
    int32_t acc = dot_packed_ternary_i8(w + r * pc, xq, K);
    if (acc_out) acc_out[r] = acc;
    out[r] = (float)acc * combined;
  });
  return OK;
}

// attention.rs:97-209.
int masked_attention(const float* q, size_t q_len, const float* kc, size_t k_len, const float* vc, size_t v_len,
                     float* out, size_t out_len, size_t nh, size_t nkv, size_t hd, size_t cur_pos) {
  if (hd == 0) return ERR_SHAPE;
  if (nkv == 0) return ERR_CONFIG;
  if (nh == 0) return ERR_CONFIG;
  if (nh % nkv != 0) return ERR_CONFIG;
  size_t seq_len = cur_pos + 1;
  size_t stride = k_len / nkv;
  size_t required = nkv * stride;
  size_t qe = nh * hd;
  if (q_len != qe) return ERR_SHAPE;
  if (k_len < required) return ERR_SHAPE;
  if (v_len < required) return ERR_SHAPE;
  if (stride < seq_len * hd) return ERR_SHAPE;
  if (out_len != qe) return ERR_SHAPE;
  float scale = 1.0f / std::sqrt((float)hd);
  size_t group = nh / nkv;
  par_for(nh, 1, [&](size_t h) {
    size_t kvh = h / group;
    const float* qh = q + h * hd;
    std::vector<float> scores(seq_len);
    for (size_t t = 0; t < seq_len; ++t)
      scores[t] = dot_f32_f32(qh, kc + kvh * stride + t * hd, hd) * scale;
    softmax_f32(scores.data(), seq_len);
    float* o = out + h * hd;
    for (size_t d = 0; d < hd; ++d) o[d] = 0.0f;
    for (size_t t = 0; t < seq_len; ++t) axpy_f32(scores[t], vc + kvh * stride + t * hd, o, hd);
  });
  return OK;
}

// Greedy sample_next_token (inference/lib.rs:263-274): Iterator::max_by with
// partial_cmp, NaN compares Equal, ties resolve to the later index.
uint32_t greedy_argmax(const float* logits, size_t n) {
  if (n == 0) return 0;
  size_t best = 0;
  for (size_t j = 1; j < n; ++j) {
    float a = logits[best], b = logits[j];
    bool greater = !(std::isnan(a) || std::isnan(b)) && a > b;
    if (!greater) best = j;
  }
  return (uint32_t)best;
}

// ---------------------------------------------------------------------------
// Model (bitnet-model/src/lib.rs).
// ---------------------------------------------------------------------------
}  // namespace

extern "C" {

struct orc_config {
  uint32_t vocab_size, hidden_size, num_layers, num_heads, num_kv_heads, intermediate_size, max_position;
  float rope_theta, rms_norm_eps;
};

struct orc_layer {
  const uint8_t *q, *k, *v, *o, *gate, *up, *down;
  float sq, sk, sv, so, sg, su, sd;
  const float *attn_norm, *attn_sub_norm, *ffn_norm, *ffn_sub_norm;
};

struct orc_weights {
  const uint16_t* embed;     // bf16 [V, H]
  const int8_t* lm_head_i8;  // [V, H]
  const float* lm_head_scales;  // [V]
  const float* final_norm;   // [H]
  const orc_layer* layers;   // [L]
};

}  // extern "C"

namespace {

struct Model {
  orc_config c;
  orc_weights w;
  std::vector<orc_layer> layers;
  // ScratchBuffers (model/lib.rs:337-387).
  std::vector<float> h_norm, q, k, v, attn, attn_n, o, ffn_h, gate, up, inner, inner_n, ffn_out, final_n;
  std::vector<int8_t> qbuf, scratch;
};

struct KV {
  size_t n_layers, nkv, hd, max_seq, filled = 0;
  bool bf16;  // store K/V rounded to bf16 (the CUDA paged cache format)
  std::vector<std::vector<float>> k, v;
  std::vector<size_t> layer_len;
};

inline float round_bf16(float x) {  // bf16::from_f32 (round to nearest even, NaN kept)
  uint32_t u;
  std::memcpy(&u, &x, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) {
    u |= 0x00400000u;
  } else {
    u += 0x7fffu + ((u >> 16) & 1u);
  }
  u &= 0xffff0000u;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// KVCache::store_kv (model/lib.rs:185-236).
int kv_store(KV& kv, size_t layer, size_t pos, const float* kvec, const float* vvec) {
  if (pos >= kv.max_seq) return ERR_SHAPE;
  if (pos > kv.layer_len[layer]) return ERR_SHAPE;
  for (size_t h = 0; h < kv.nkv; ++h) {
    float* kd = &kv.k[layer][h * kv.max_seq * kv.hd + pos * kv.hd];
    float* vd = &kv.v[layer][h * kv.max_seq * kv.hd + pos * kv.hd];
    for (size_t d = 0; d < kv.hd; ++d) {
      float a = kvec[h * kv.hd + d], b = vvec[h * kv.hd + d];
      kd[d] = kv.bf16 ? round_bf16(a) : a;
      vd[d] = kv.bf16 ? round_bf16(b) : b;
    }
  }
  if (pos == kv.layer_len[layer]) kv.layer_len[layer] += 1;
  return OK;
}

int rms_norm_checked(const float* x, size_t xl, const float* w, size_t wl, float eps, float* out, size_t ol) {
  // norm.rs:77-107.
  if (xl != wl) return ERR_SHAPE;
  if (xl != ol) return ERR_SHAPE;
  if (!(eps > 0.0f) || !finite(eps)) return ERR_QUANT;
  if (xl == 0) return OK;
  float d = (float)xl;
  float ss = sum_squares_f32(x, xl);
  float rms = std::sqrt(ss / d + eps);
  float inv = 1.0f / rms;
  mul_scale_f32(x, inv, w, out, xl);
  return OK;
}

int gemv_act_quant(Model& m, const uint8_t* w, size_t w_len, float ws, const float* x, size_t x_len, float* out,
                   size_t out_len, size_t N, size_t K) {
  // CpuBackend::ternary_gemv_with_activation_quant (cpu/lib.rs:223-249).
  m.scratch.resize(K);
  float s = 0.0f;
  int rc = absmax_quantize_row_into(x, x_len, m.scratch.data(), K, &s);
  if (rc) return rc;
  float max_abs = s * 127.0f;
  return gemv_quantised(w, w_len, ws, m.scratch.data(), K, max_abs, out, out_len, N, K, nullptr);
}

int lm_head_i8(const float* h, const int8_t* w, const float* scales, float* out, size_t V, size_t H) {
  // CpuBackend::lm_head_matmul_i8_into (cpu/lib.rs:544-575): 256-row chunks.
  size_t chunks = (V + 255) / 256;
  par_for(chunks, 1, [&](size_t c) {
    size_t e = std::min(V, (c + 1) * 256);
    for (size_t v = c * 256; v < e; ++v) out[v] = dot_f32_i8w(w + v * H, h, H) * scales[v];
  });
  return OK;
}

// BitNetModel::forward (model/lib.rs:559-862); with n == 1 this is exactly the
// forward_into decode fast path (:931-1163).
int model_forward(Model& m, KV& kv, const uint32_t* tokens, size_t n, size_t start_pos, float* logits) {
  const orc_config& c = m.c;
  if (n == 0) return ERR_SHAPE;
  size_t end = start_pos + n;
  if (end > c.max_position) return ERR_SHAPE;
  if (end > kv.max_seq) return ERR_SHAPE;
  size_t H = c.hidden_size, hd = H / c.num_heads, nh = c.num_heads, nkv = c.num_kv_heads;
  size_t qd = nh * hd, kvd = nkv * hd, F = c.intermediate_size;
  float eps = c.rms_norm_eps, theta = c.rope_theta;
  std::vector<std::vector<float>> hs(n, std::vector<float>(H));
  for (size_t t = 0; t < n; ++t) {
    if (tokens[t] >= c.vocab_size) return ERR_SHAPE;
    for (size_t i = 0; i < H; ++i) hs[t][i] = bf16_to_f32(m.w.embed[(size_t)tokens[t] * H + i]);
  }
  size_t pcH = (H + 3) / 4, pcQ = (qd + 3) / 4, pcF = (F + 3) / 4;
  int rc;
  for (size_t l = 0; l < c.num_layers; ++l) {
    const orc_layer& L = m.layers[l];
    for (size_t t = 0; t < n; ++t) {
      size_t pos = start_pos + t;
      float* h = hs[t].data();
      if ((rc = rms_norm_checked(h, H, L.attn_norm, H, eps, m.h_norm.data(), H))) return rc;
      float qs = 0.0f;
      if ((rc = absmax_quantize_row_into(m.h_norm.data(), H, m.qbuf.data(), H, &qs))) return rc;
      float amax = qs * 127.0f;
      if ((rc = gemv_quantised(L.q, qd * pcH, L.sq, m.qbuf.data(), H, amax, m.q.data(), qd, qd, H, nullptr)))
        return rc;
      if ((rc = gemv_quantised(L.k, kvd * pcH, L.sk, m.qbuf.data(), H, amax, m.k.data(), kvd, kvd, H, nullptr)))
        return rc;
      if ((rc = gemv_quantised(L.v, kvd * pcH, L.sv, m.qbuf.data(), H, amax, m.v.data(), kvd, kvd, H, nullptr)))
        return rc;
      if ((rc = backend().rope_embed(m.q.data(), qd, m.k.data(), kvd, pos, hd, nh, nkv, theta))) return rc;
      if ((rc = kv_store(kv, l, pos, m.k.data(), m.v.data()))) return rc;
      size_t cap = kv.nkv * kv.max_seq * kv.hd;
      if ((rc = masked_attention(m.q.data(), qd, kv.k[l].data(), cap, kv.v[l].data(), cap, m.attn.data(), qd, nh,
                                 nkv, hd, pos)))
        return rc;
      if ((rc = rms_norm_checked(m.attn.data(), qd, L.attn_sub_norm, qd, eps, m.attn_n.data(), qd))) return rc;
      if ((rc = gemv_act_quant(m, L.o, H * pcQ, L.so, m.attn_n.data(), qd, m.o.data(), H, H, qd))) return rc;
      axpy_f32(1.0f, m.o.data(), h, H);
      if ((rc = rms_norm_checked(h, H, L.ffn_norm, H, eps, m.ffn_h.data(), H))) return rc;
      if ((rc = absmax_quantize_row_into(m.ffn_h.data(), H, m.qbuf.data(), H, &qs))) return rc;
      amax = qs * 127.0f;
      if ((rc = gemv_quantised(L.gate, F * pcH, L.sg, m.qbuf.data(), H, amax, m.gate.data(), F, F, H, nullptr)))
        return rc;
      if ((rc = gemv_quantised(L.up, F * pcH, L.su, m.qbuf.data(), H, amax, m.up.data(), F, F, H, nullptr)))
        return rc;
      for (size_t i = 0; i < F; ++i) {  // sqrelu_gate_f32_avx2: (r*r)*u
        float r = rust_max(m.gate[i], 0.0f);
        m.inner[i] = (r * r) * m.up[i];
      }
      if ((rc = rms_norm_checked(m.inner.data(), F, L.ffn_sub_norm, F, eps, m.inner_n.data(), F))) return rc;
      if ((rc = gemv_act_quant(m, L.down, H * pcF, L.sd, m.inner_n.data(), F, m.ffn_out.data(), H, H, F)))
        return rc;
      axpy_f32(1.0f, m.ffn_out.data(), h, H);
    }
  }
  for (size_t t = 0; t < n; ++t) {  // KVCache::advance
    if (kv.filled >= kv.max_seq) return ERR_SHAPE;
    kv.filled += 1;
  }
  if ((rc = rms_norm_checked(hs[n - 1].data(), H, m.w.final_norm, H, eps, m.final_n.data(), H))) return rc;
  return lm_head_i8(m.final_n.data(), m.w.lm_head_i8, m.w.lm_head_scales, logits, c.vocab_size, H);
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

int orc_set_threads(int n) {
  pool().resize(n);
  return pool().size();
}
int orc_threads(void) { return pool().size(); }

int orc_has_avx2_fma(void) { return __builtin_cpu_supports("avx2") && __builtin_cpu_supports("fma"); }

// ---- quant -----------------------------------------------------------------
void orc_pack_ternary(const int8_t* data, size_t n, uint8_t* packed) {
  // ternary.rs:266-285: +1->00, 0->01, -1->10, LSB first; padding bits stay 0.
  size_t pl = (n + 3) / 4;
  std::memset(packed, 0, pl);
  for (size_t i = 0; i < n; ++i) {
    uint8_t bits = data[i] == 1 ? 0 : (data[i] == 0 ? 1 : 2);
    packed[i / 4] |= (uint8_t)(bits << (2 * (i % 4)));
  }
}

int orc_unpack_ternary(const uint8_t* packed, size_t packed_len, size_t n, int8_t* out) {
  // ternary.rs:294-327: code 0b11 is an error.
  size_t req = (n + 3) / 4;
  if (packed_len < req) return ERR_SHAPE;
  for (size_t i = 0; i < n; ++i) {
    uint8_t bits = (packed[i / 4] >> (2 * (i % 4))) & 3;
    if (bits == 3) return ERR_QUANT;
    out[i] = bits == 0 ? 1 : (bits == 1 ? 0 : -1);
  }
  return OK;
}

int orc_decode_hf_packed(const uint8_t* packed, size_t packed_len, size_t packed_rows, size_t cols, float scale,
                         int8_t* logical) {
  // bitnet-convert decode_packed_projection (crates/bitnet-convert/src/lib.rs:235-325):
  // checks in its order, then for each packed row, column and shift 0,2,4,6
  // (shift index s) the lane of logical row s*packed_rows + r is value lane-1;
  // lane 0b11 is an error. Output: logical i8 [4*packed_rows][cols].
  if (packed_rows == 0 || cols == 0) return ERR_SHAPE;
  if (!(scale > 0.0f) || !finite(scale)) return ERR_QUANT;
  size_t logical_rows = packed_rows * 4, numel = logical_rows * cols;
  if (packed_len < (numel + 3) / 4) return ERR_SHAPE;
  for (size_t r = 0; r < packed_rows; ++r)
    for (size_t c = 0; c < cols; ++c) {
      uint8_t byte = packed[r * cols + c];
      for (int si = 0; si < 4; ++si) {
        int lane = (byte >> (2 * si)) & 3;
        if (lane == 3) return ERR_QUANT;
        logical[(si * packed_rows + r) * cols + c] = (int8_t)(lane - 1);
      }
    }
  return OK;
}

int orc_absmean_quantize(const float* w, size_t n, int8_t* q, float* scale) {
  // absmean.rs:71-102: sequential f32 sum of |w|, mean, clamp 1e-5, recip, round, clamp +-1.
  if (n == 0) return ERR_QUANT;
  for (size_t i = 0; i < n; ++i)
    if (!finite(w[i])) return ERR_QUANT;
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) sum += std::fabs(w[i]);
  float mean = sum / (float)n;
  float s = rust_max(mean, 1e-5f);
  float inv = 1.0f / s;
  for (size_t i = 0; i < n; ++i) {
    float r = std::round(w[i] * inv);
    r = std::min(std::max(r, -1.0f), 1.0f);
    q[i] = (int8_t)r;
  }
  *scale = s;
  return OK;
}

int orc_absmax_quantize_row_into(const float* x, size_t n, int8_t* out, size_t out_len, float* scale) {
  return absmax_quantize_row_into(x, n, out, out_len, scale);
}

void orc_quantize_bf16_rows_to_i8(const uint16_t* bf, size_t rows, size_t row_len, int8_t* out, float* scales) {
  // weights/src/loader.rs:297-340.
  par_for(rows, 64, [&](size_t r) {
    const uint16_t* row = bf + r * row_len;
    float m = 0.0f;
    for (size_t i = 0; i < row_len; ++i) {
      float a = std::fabs(bf16_to_f32(row[i]));
      if (a > m) m = a;
    }
    if (m < 1e-10f) m = 1e-10f;
    float inv = 127.0f / m;
    scales[r] = m / 127.0f;
    for (size_t i = 0; i < row_len; ++i) {
      float q = std::round(bf16_to_f32(row[i]) * inv);
      q = std::min(std::max(q, -128.0f), 127.0f);
      out[r * row_len + i] = (int8_t)q;
    }
  });
}

float orc_bf16_round(float x) { return round_bf16(x); }

// ---- Backend trait methods (CpuBackend) -----------------------------------
int orc_ternary_gemv(const uint8_t* w, size_t w_len, float ws, const float* x, size_t x_len, float* out,
                     size_t out_len, size_t N, size_t K) {
  // gemv.rs:108-165.
  size_t pc = (K + 3) / 4;
  if (w_len != N * pc) return ERR_SHAPE;
  if (x_len != K) return ERR_SHAPE;
  if (out_len != N) return ERR_SHAPE;
  if (!(ws > 0.0f) || !finite(ws)) return ERR_QUANT;
  par_for(N, 32, [&](size_t r) { out[r] = dot_packed_ternary_f32(w + r * pc, x, K) * ws; });
  return OK;
}

int orc_ternary_gemv_preq(const uint8_t* w, size_t w_len, float ws, const int8_t* xq, size_t xq_len, float amax,
                          float* out, size_t out_len, size_t N, size_t K, int32_t* acc_out) {
  return gemv_quantised(w, w_len, ws, xq, xq_len, amax, out, out_len, N, K, acc_out);
}

int orc_ternary_gemv_with_activation_quant(const uint8_t* w, size_t w_len, float ws, const float* x, size_t x_len,
                                           float* out, size_t out_len, size_t N, size_t K) {
  std::vector<int8_t> scratch(K);
  float s = 0.0f;
  int rc = absmax_quantize_row_into(x, x_len, scratch.data(), K, &s);
  if (rc) return rc;
  return gemv_quantised(w, w_len, ws, scratch.data(), K, s * 127.0f, out, out_len, N, K, nullptr);
}

int orc_rms_norm(const float* x, size_t xl, const float* w, size_t wl, float eps, float* out, size_t ol) {
  return rms_norm_checked(x, xl, w, wl, eps, out, ol);
}

int orc_rope_embed(float* q, size_t ql, float* k, size_t kl, size_t pos, size_t hd, size_t nh, size_t nkv,
                   float theta) {
  return backend().rope_embed(q, ql, k, kl, pos, hd, nh, nkv, theta);
}

int orc_masked_attention(const float* q, size_t ql, const float* k, size_t kl, const float* v, size_t vl, float* out,
                         size_t ol, size_t nh, size_t nkv, size_t hd, size_t cur_pos) {
  return masked_attention(q, ql, k, kl, v, vl, out, ol, nh, nkv, hd, cur_pos);
}

void orc_squared_relu(float* x, size_t n) {  // activation.rs:92
  for (size_t i = 0; i < n; ++i) {
    float r = rust_max(x[i], 0.0f);
    x[i] = r * r;
  }
}

void orc_softmax(float* x, size_t n) { softmax_f32(x, n); }

int orc_elementwise_mul(const float* a, size_t al, const float* b, size_t bl, float* out, size_t ol) {
  if (al != bl) return ERR_SHAPE;
  if (al != ol) return ERR_SHAPE;
  for (size_t i = 0; i < al; ++i) out[i] = a[i] * b[i];
  return OK;
}

int orc_sqrelu_gate(const float* g, size_t gl, const float* u, size_t ul, float* out, size_t ol) {
  if (gl != ul || gl != ol) return ERR_SHAPE;
  for (size_t i = 0; i < gl; ++i) {
    float r = rust_max(g[i], 0.0f);
    out[i] = (r * r) * u[i];
  }
  return OK;
}

int orc_lm_head_f32(const float* h, const float* w, float* out, size_t V, size_t H) {
  size_t chunks = (V + 255) / 256;
  par_for(chunks, 1, [&](size_t c) {
    size_t e = std::min(V, (c + 1) * 256);
    for (size_t v = c * 256; v < e; ++v) out[v] = dot_f32_f32(w + v * H, h, H);
  });
  return OK;
}

int orc_lm_head_bf16(const float* h, const uint16_t* w, float* out, size_t V, size_t H) {
  size_t chunks = (V + 255) / 256;
  par_for(chunks, 1, [&](size_t c) {
    size_t e = std::min(V, (c + 1) * 256);
    for (size_t v = c * 256; v < e; ++v) out[v] = dot_f32_bf16w(w + v * H, h, H);
  });
  return OK;
}

int orc_lm_head_i8(const float* h, const int8_t* w, const float* scales, float* out, size_t V, size_t H) {
  return lm_head_i8(h, w, scales, out, V, H);
}

uint32_t orc_greedy_argmax(const float* logits, size_t n) { return greedy_argmax(logits, n); }

// sample_next_token (crates/bitnet-inference/src/lib.rs:236-390), in place on
// logits like the reference: repetition penalty (divide), temperature
// (multiply by its reciprocal when |t - 1| > 1e-6), the top_k == 1 greedy
// shortcut, top-k (mask below the k-th largest), top-p (softmax over finite
// logits, descending order, smallest prefix with cumulative f32 probability
// >= p), a final softmax and one LCG step (seed + number of past tokens)
// mapped to [0, 1) for an inverse-CDF draw in index order, argmax fallback.
// The reference orders equal probabilities with sort_unstable (unspecified);
// here they go in ascending index order. Logits are assumed NaN-free (the
// forward pass rejects non-finite activations).
uint32_t orc_sample_next_token(float* logits, size_t vocab, float temperature, float top_p, size_t top_k,
                               float repetition_penalty, uint64_t seed, const uint32_t* past, size_t n_past) {
  if (vocab == 0) return 0;
  const float ninf = -std::numeric_limits<float>::infinity();
  if (repetition_penalty != 1.0f)
    for (size_t i = 0; i < n_past; ++i)
      if (past[i] < vocab) logits[past[i]] /= repetition_penalty;
  if (std::fabs(temperature - 1.0f) > 1e-6f) {
    const float inv = 1.0f / temperature;
    for (size_t i = 0; i < vocab; ++i) logits[i] *= inv;
  }
  if (top_k == 1) return greedy_argmax(logits, vocab);
  if (top_k > 0 && top_k < vocab) {
    std::vector<float> sorted(logits, logits + vocab);
    std::nth_element(sorted.begin(), sorted.begin() + (top_k - 1), sorted.end(), std::greater<float>());
    const float thr = sorted[top_k - 1];
    for (size_t i = 0; i < vocab; ++i)
      if (logits[i] < thr) logits[i] = ninf;
  }
  auto softmax_finite = [&](std::vector<float>& pr) {
    float mx = ninf;
    for (size_t i = 0; i < vocab; ++i)
      if (std::isfinite(logits[i])) mx = rust_max(mx, logits[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < vocab; ++i) {
      pr[i] = std::isfinite(logits[i]) ? std::exp(logits[i] - mx) : 0.0f;
      sum += pr[i];
    }
    const float inv = sum > 0.0f ? 1.0f / sum : 1.0f;
    for (size_t i = 0; i < vocab; ++i) pr[i] *= inv;
  };
  std::vector<float> pr(vocab);
  if (top_p < 1.0f) {
    softmax_finite(pr);
    std::vector<size_t> idx(vocab);
    for (size_t i = 0; i < vocab; ++i) idx[i] = i;
    std::stable_sort(idx.begin(), idx.end(), [&](size_t a, size_t b) { return pr[a] > pr[b]; });
    float cum = 0.0f;
    size_t cutoff = vocab;
    for (size_t r = 0; r < vocab; ++r) {
      cum += pr[idx[r]];
      if (cum >= top_p) {
        cutoff = r + 1;
        break;
      }
    }
    std::vector<char> keep(vocab, 0);
    for (size_t r = 0; r < cutoff; ++r) keep[idx[r]] = 1;
    for (size_t i = 0; i < vocab; ++i)
      if (!keep[i]) logits[i] = ninf;
  }
  softmax_finite(pr);
  uint64_t st = seed + (uint64_t)n_past;
  st = st * 6364136223846793005ULL + 1442695040888963407ULL;
  const float rf = (float)(st >> 11) / (float)(1ULL << 53);
  float cum = 0.0f;
  for (size_t i = 0; i < vocab; ++i) {
    cum += pr[i];
    if (rf <= cum) return (uint32_t)i;
  }
  return greedy_argmax(pr.data(), vocab);
}

// ---- model ------------------------------------------------------------------
void* orc_model_create(const orc_config* c, const orc_weights* w) {
  Model* m = new Model();
  m->c = *c;
  m->w = *w;
  m->layers.assign(w->layers, w->layers + c->num_layers);
  size_t H = c->hidden_size, hd = H / c->num_heads, qd = c->num_heads * hd, kvd = c->num_kv_heads * hd,
         F = c->intermediate_size;
  m->h_norm.resize(H);
  m->q.resize(qd);
  m->k.resize(kvd);
  m->v.resize(kvd);
  m->attn.resize(qd);
  m->attn_n.resize(qd);
  m->o.resize(H);
  m->ffn_h.resize(H);
  m->gate.resize(F);
  m->up.resize(F);
  m->inner.resize(F);
  m->inner_n.resize(F);
  m->ffn_out.resize(H);
  m->final_n.resize(H);
  m->qbuf.resize(std::max(H, F));
  return m;
}

void orc_model_destroy(void* m) { delete (Model*)m; }

void* orc_kv_create(const void* model, size_t max_seq, int kv_bf16) {
  const Model* m = (const Model*)model;
  KV* kv = new KV();
  kv->n_layers = m->c.num_layers;
  kv->nkv = m->c.num_kv_heads;
  kv->hd = m->c.hidden_size / m->c.num_heads;
  kv->max_seq = max_seq;
  kv->bf16 = kv_bf16 != 0;
  kv->k.assign(kv->n_layers, std::vector<float>(kv->nkv * max_seq * kv->hd, 0.0f));
  kv->v.assign(kv->n_layers, std::vector<float>(kv->nkv * max_seq * kv->hd, 0.0f));
  kv->layer_len.assign(kv->n_layers, 0);
  return kv;
}

void orc_kv_destroy(void* kv) { delete (KV*)kv; }

void orc_kv_clear(void* p) {  // KVCache::clear
  KV* kv = (KV*)p;
  for (size_t l = 0; l < kv->n_layers; ++l) {
    std::fill(kv->k[l].begin(), kv->k[l].end(), 0.0f);
    std::fill(kv->v[l].begin(), kv->v[l].end(), 0.0f);
    kv->layer_len[l] = 0;
  }
  kv->filled = 0;
}

size_t orc_kv_len(const void* p) { return ((const KV*)p)->filled; }

// Seed a context: positions [0, n) of every layer from k/v laid out
// [layer][pos][kv_head*hd] (values are rounded to bf16 when the cache is bf16).
int orc_kv_seed(void* p, size_t n, const float* k, const float* v) {
  KV* kv = (KV*)p;
  if (n > kv->max_seq) return ERR_SHAPE;
  size_t row = kv->nkv * kv->hd;
  for (size_t l = 0; l < kv->n_layers; ++l) {
    kv->layer_len[l] = 0;
    for (size_t t = 0; t < n; ++t) {
      int rc = kv_store(*kv, l, t, k + (l * n + t) * row, v + (l * n + t) * row);
      if (rc) return rc;
    }
  }
  kv->filled = n;
  return OK;
}

// Read positions [0, n) back in the [layer][pos][kv_head*hd] layout.
int orc_kv_read(const void* p, size_t n, float* k, float* v) {
  const KV* kv = (const KV*)p;
  if (n > kv->max_seq) return ERR_SHAPE;
  size_t row = kv->nkv * kv->hd;
  for (size_t l = 0; l < kv->n_layers; ++l)
    for (size_t t = 0; t < n; ++t)
      for (size_t h = 0; h < kv->nkv; ++h)
        for (size_t d = 0; d < kv->hd; ++d) {
          k[(l * n + t) * row + h * kv->hd + d] = kv->k[l][h * kv->max_seq * kv->hd + t * kv->hd + d];
          v[(l * n + t) * row + h * kv->hd + d] = kv->v[l][h * kv->max_seq * kv->hd + t * kv->hd + d];
        }
  return OK;
}

int orc_forward(void* model, void* kv, const uint32_t* tokens, size_t n, size_t start_pos, float* logits) {
  return model_forward(*(Model*)model, *(KV*)kv, tokens, n, start_pos, logits);
}

// generate_from_tokens_streaming (inference/lib.rs:701-777), greedy (top_k = 1).
// margins (optional, length max_new): top-1 minus top-2 logit before each pick.
int orc_generate(void* model, void* kvp, const uint32_t* prompt, size_t n_prompt, size_t max_new, uint32_t eos0,
                 uint32_t eos1, uint32_t* out_tokens, size_t* n_out, float* margins) {
  Model& m = *(Model*)model;
  KV& kv = *(KV*)kvp;
  *n_out = 0;
  if (n_prompt == 0) return OK;
  orc_kv_clear(&kv);
  std::vector<float> logits(m.c.vocab_size);
  int rc = model_forward(m, kv, prompt, n_prompt, 0, logits.data());
  if (rc) return rc;
  for (size_t step = 0; step < max_new; ++step) {
    uint32_t tok = greedy_argmax(logits.data(), logits.size());
    if (margins) {
      float b1 = -INFINITY, b2 = -INFINITY;
      for (float x : logits) {
        if (x > b1) {
          b2 = b1;
          b1 = x;
        } else if (x > b2) {
          b2 = x;
        }
      }
      margins[step] = b1 - b2;
    }
    if (tok == eos0 || tok == eos1) break;
    out_tokens[(*n_out)++] = tok;
    size_t pos = kv.filled;
    rc = model_forward(m, kv, &tok, 1, pos, logits.data());
    if (rc) return rc;
  }
  return OK;
}

}  // extern "C"
