// backend.cu — context lifecycle and the Backend-trait entry points.
//
// Each trait method validates its slices in the reference's order (so the
// same bad call yields the same BitNetError variant), copies the host slices
// into device scratch, runs the kernels, and copies the outputs back.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "internal.h"

using namespace bitnet;

// ---------------------------------------------------------------------------
// Errors.
// ---------------------------------------------------------------------------
namespace bitnet {

static thread_local std::string g_last_error;
// the fields of the last InvalidShape { expected, got } (empty after any other error)
static thread_local std::string g_last_expected, g_last_got;

void set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  const char* kind = code == BITNET_ERR_INVALID_SHAPE   ? "invalid tensor shape"
                     : code == BITNET_ERR_QUANTIZATION  ? "quantization error"
                     : code == BITNET_ERR_INVALID_CONFIG ? "invalid model configuration"
                                                         : "backend error (CUDA)";
  g_last_error = std::string(kind) + ": " + buf;
  g_last_expected.clear();
  g_last_got.clear();
}
int shape_error(const std::string& expected, const std::string& got) {
  set_error(BITNET_ERR_INVALID_SHAPE, "expected %s, got %s", expected.c_str(), got.c_str());
  g_last_expected = expected;
  g_last_got = got;
  return BITNET_ERR_INVALID_SHAPE;
}

int quant_error(const std::string& msg) {
  set_error(BITNET_ERR_QUANTIZATION, "%s", msg.c_str());
  return BITNET_ERR_QUANTIZATION;
}
int config_error(const std::string& msg) {
  set_error(BITNET_ERR_INVALID_CONFIG, "%s", msg.c_str());
  return BITNET_ERR_INVALID_CONFIG;
}
int backend_error(const std::string& msg) {
  set_error(BITNET_ERR_BACKEND, "%s", msg.c_str());
  return BITNET_ERR_BACKEND;
}
int cuda_error(cudaError_t e, const char* what) {
  set_error(BITNET_ERR_BACKEND, "%s failed: %s", what, cudaGetErrorString(e));
  return BITNET_ERR_BACKEND;
}

int DevBuf::ensure(size_t bytes) {
  if (bytes == 0) bytes = 16;
  if (bytes <= cap) return BITNET_OK;
  release();
  size_t want = round_up(bytes, 256);
  cudaError_t e = cudaMalloc(&p, want);
  if (e != cudaSuccess) {
    p = nullptr;
    return cuda_error(e, "cudaMalloc");
  }
  cap = want;
  return BITNET_OK;
}
void DevBuf::release() {
  if (p) cudaFree(p);
  p = nullptr;
  cap = 0;
}

int build_rope_host(size_t max_seq, size_t head_dim, float theta, std::vector<float>& cs, std::vector<float>& sn) {
  if (head_dim == 0 || head_dim % 2 != 0) return config_error("head_dim must be even and > 0, got " + std::to_string(head_dim));
  if (!(theta > 0.0f) || !std::isfinite(theta)) return config_error("theta must be finite and > 0");
  size_t half = head_dim / 2;
  cs.assign(max_seq * half, 0.0f);
  sn.assign(max_seq * half, 0.0f);
  std::vector<float> freq(half);
  for (size_t i = 0; i < half; ++i) {
    float exponent = -2.0f * (float)i / (float)head_dim;
    freq[i] = std::pow(theta, exponent);  // powf, as f32::powf
  }
  for (size_t pos = 0; pos < max_seq; ++pos)
    for (size_t i = 0; i < half; ++i) {
      float angle = (float)pos * freq[i];
      cs[pos * half + i] = std::cos(angle);  // cosf
      sn[pos * half + i] = std::sin(angle);  // sinf
    }
  return BITNET_OK;
}

// The host libm's expf on every x in [-112, -0] whose device exp
// (exp_candidate) lands within 0.003 ulp of a float rounding midpoint (the
// GPU enumerates them), kept where it differs from the device's value.  The
// pair tables of exp_pair are computed here first, in long double.
int ensure_exp_table(bitnet_cuda_ctx* c) {
  if (c->exp_ready) return BITNET_OK;
  {
    std::vector<float4> en(88);
    for (int k = 0; k < 88; ++k) {
      const long double v = expl(-(long double)k);
      const int S = (int)lrintl((long double)k * 1.442695040888963407359924681L);  // k / ln 2
      const long double w = ldexpl(v, S);
      const float h = (float)w;
      float sbits;
      std::memcpy(&sbits, &S, 4);
      en[k] = make_float4(h, (float)(w - (long double)h), sbits, 0.0f);
    }
    std::vector<float2> fj(128);
    for (int j = 0; j < 128; ++j) {
      const long double v = expl(-(long double)j / 128.0L);
      const float h = (float)v;
      fj[j] = make_float2(h, (float)(v - (long double)h));
    }
    BN_TRY(c->exp_en.ensure(en.size() * sizeof(float4)));
    BN_TRY(c->exp_fj.ensure(fj.size() * sizeof(float2)));
    BN_CUDA(cudaMemcpy(c->exp_en.p, en.data(), en.size() * sizeof(float4), cudaMemcpyHostToDevice));
    BN_CUDA(cudaMemcpy(c->exp_fj.p, fj.data(), fj.size() * sizeof(float2), cudaMemcpyHostToDevice));
    c->exp_table.en = c->exp_en.as<float4>();
    c->exp_table.fj = c->exp_fj.as<float2>();
  }
  const uint32_t lo = 0x80000000u, hi = 0xC2E00000u;  // -0 .. -112
  const uint32_t cap = 8u << 20;
  DevBuf cand, cnt;
  BN_TRY(cand.ensure((size_t)cap * sizeof(uint2)));
  BN_TRY(cnt.ensure(sizeof(uint32_t)));
  BN_CUDA(cudaMemsetAsync(cnt.p, 0, sizeof(uint32_t), c->stream));
  launch_exp_candidates(lo, hi, cand.as<uint2>(), cap, cnt.as<uint32_t>(), c->exp_table, c->stream);
  uint32_t n = 0;
  BN_CUDA(cudaMemcpyAsync(&n, cnt.p, sizeof(uint32_t), cudaMemcpyDeviceToHost, c->stream));
  BN_CUDA(cudaStreamSynchronize(c->stream));
  if (n > cap) return backend_error("exp exception candidates exceed the buffer");
  std::vector<uint2> h(n);
  BN_CUDA(cudaMemcpy(h.data(), cand.p, (size_t)n * sizeof(uint2), cudaMemcpyDeviceToHost));
  std::vector<std::pair<uint32_t, float>> ex;
  for (const uint2& e : h) {
    float x, f;
    std::memcpy(&x, &e.x, 4);
    std::memcpy(&f, &e.y, 4);
    float libm = std::exp(x);  // expf of the host libm, as f32::exp
    if (std::memcmp(&libm, &f, 4) != 0) ex.emplace_back(e.x, libm);
  }
  std::sort(ex.begin(), ex.end(), [](const auto& a, const auto& b) { return a.first < b.first; });
  std::vector<uint32_t> keys(ex.size());
  std::vector<float> vals(ex.size());
  for (size_t i = 0; i < ex.size(); ++i) {
    keys[i] = ex[i].first;
    vals[i] = ex[i].second;
  }
  BN_TRY(c->exp_keys.ensure(std::max<size_t>(keys.size(), 1) * 4));
  BN_TRY(c->exp_vals.ensure(std::max<size_t>(vals.size(), 1) * 4));
  if (!keys.empty()) {
    BN_CUDA(cudaMemcpy(c->exp_keys.p, keys.data(), keys.size() * 4, cudaMemcpyHostToDevice));
    BN_CUDA(cudaMemcpy(c->exp_vals.p, vals.data(), vals.size() * 4, cudaMemcpyHostToDevice));
  }
  // two-choice bucketed copy: start at ~2 keys per bucket of 8 and double
  // the bucket count until every key fits
  uint32_t bits = 4;
  while ((1u << bits) * 2 < keys.size()) ++bits;
  std::vector<uint2> slot;
  for (;; ++bits) {
    const uint32_t nb = 1u << bits;
    slot.assign((size_t)nb * kExpBucketSlots, make_uint2(0u, 0u));
    std::vector<int> fill(nb, 0);
    bool ok = true;
    for (size_t i = 0; i < keys.size() && ok; ++i) {
      const uint32_t b1 = (keys[i] * kExpHashMul) >> (32 - bits), b2 = (keys[i] * kExpHashMul2) >> (32 - bits);
      const uint32_t bk = fill[b2] < fill[b1] ? b2 : b1;
      if (fill[bk] == kExpBucketSlots) {
        ok = false;
        break;
      }
      uint32_t vb;
      std::memcpy(&vb, &vals[i], 4);
      slot[(size_t)bk * kExpBucketSlots + fill[bk]++] = make_uint2(keys[i], vb);
    }
    if (ok) break;
    if (bits >= 24) return backend_error("exp exception table does not fit its buckets");
  }
  BN_TRY(c->exp_hash.ensure(slot.size() * sizeof(uint2)));
  BN_CUDA(cudaMemcpy(c->exp_hash.p, slot.data(), slot.size() * sizeof(uint2), cudaMemcpyHostToDevice));
  c->exp_table.keys = c->exp_keys.as<uint32_t>();
  c->exp_table.vals = c->exp_vals.as<float>();
  c->exp_table.n = (int)keys.size();
  c->exp_table.buckets = c->exp_hash.as<uint4>();
  c->exp_table.bucket_shift = 32 - bits;
  c->exp_ready = true;
  return BITNET_OK;
}

void ctx_retain(bitnet_cuda_ctx* c) { c->refs.fetch_add(1); }

void ctx_release(bitnet_cuda_ctx* c) {
  if (c->refs.fetch_sub(1) != 1) return;
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  for (auto& b : c->b) b.release();
  c->status.release();
  c->rope.d_cos.release();
  c->rope.d_sin.release();
  c->exp_keys.release();
  c->exp_vals.release();
  c->exp_hash.release();
  c->samp_counts.release();
  c->samp_e.release();
  c->samp_misc.release();
  c->exp_en.release();
  c->exp_fj.release();
  cudaStreamDestroy(c->stream);
  delete c;
}

}  // namespace bitnet

// ---------------------------------------------------------------------------
// Helpers local to this file.
// ---------------------------------------------------------------------------
namespace {

std::string sz(size_t v) { return std::to_string(v); }

struct Guard {
  bitnet_cuda_ctx* c;
  std::lock_guard<std::mutex> lk;
  explicit Guard(bitnet_cuda_ctx* ctx) : c(ctx), lk(ctx->mu) { cudaSetDevice(ctx->device); }
};

int upload(DevBuf& b, const void* host, size_t bytes, cudaStream_t st) {
  BN_TRY(b.ensure(bytes));
  if (bytes) BN_CUDA(cudaMemcpyAsync(b.p, host, bytes, cudaMemcpyHostToDevice, st));
  return BITNET_OK;
}

int finish(bitnet_cuda_ctx* c) {
  BN_CUDA(cudaGetLastError());
  BN_CUDA(cudaStreamSynchronize(c->stream));
  return BITNET_OK;
}

int read_status(bitnet_cuda_ctx* c, int32_t* out) {
  BN_CUDA(cudaMemcpyAsync(out, c->status.p, sizeof(int32_t), cudaMemcpyDeviceToHost, c->stream));
  BN_CUDA(cudaStreamSynchronize(c->stream));
  return BITNET_OK;
}

int reset_status(bitnet_cuda_ctx* c) {
  BN_TRY(c->status.ensure(64));
  BN_CUDA(cudaMemsetAsync(c->status.p, 0, 64, c->stream));
  return BITNET_OK;
}

// Upload a reference-format ternary matrix and repack it into b[dst].
int stage_weight(bitnet_cuda_ctx* c, const uint8_t* w, size_t rows, size_t cols, DevBuf& raw, DevBuf& dst) {
  size_t pc = (cols + 3) / 4;
  BN_TRY(upload(raw, w, rows * pc, c->stream));
  BN_TRY(dst.ensure(rows * words_per_row(cols) * 4));
  launch_repack_ternary(raw.as<uint8_t>(), dst.as<uint32_t>(), (int)rows, (int)cols, c->stream);
  return BITNET_OK;
}

// gemv.rs:260-295 validation of ternary_gemv_quantised.
int validate_quantised(size_t w_len, float ws, size_t act_len, float act_scale, size_t out_len, size_t N, size_t K) {
  size_t pc = (K + 3) / 4;
  if (N != 0 && pc > SIZE_MAX / N) return shape_error("weight size fits usize", "overflow");
  size_t exp = N * pc;
  if (w_len != exp)
    return shape_error("weight_packed.len() == " + sz(N) + " * ceil(" + sz(K) + "/4) = " + sz(exp),
                       "weight_packed.len() == " + sz(w_len));
  if (act_len != K) return shape_error("activation.len() == " + sz(K), "activation.len() == " + sz(act_len));
  if (out_len != N) return shape_error("output.len() == " + sz(N), "output.len() == " + sz(out_len));
  if (!(ws > 0.0f) || !std::isfinite(ws)) return quant_error("weight_scale must be finite > 0");
  if (!(act_scale > 0.0f) || !std::isfinite(act_scale)) return quant_error("act_scale must be finite > 0");
  return BITNET_OK;
}

// Device int8 GEMV of one token (buffers: b0 raw W, b1 repacked W, b2 xq, b3 amax, b4 out, b5 acc).
int run_gemv_preq(bitnet_cuda_ctx* c, const uint8_t* w, float ws, size_t N, size_t K, float act_absmax, float* out,
                  int32_t* acc) {
  cudaStream_t st = c->stream;
  BN_TRY(stage_weight(c, w, N, K, c->b[0], c->b[1]));
  BN_TRY(c->b[3].ensure(sizeof(float)));
  BN_CUDA(cudaMemcpyAsync(c->b[3].p, &act_absmax, sizeof(float), cudaMemcpyHostToDevice, st));
  BN_TRY(c->b[4].ensure(N * sizeof(float)));
  if (acc) BN_TRY(c->b[5].ensure(N * sizeof(int32_t)));
  Segments seg;
  seg.n = 1;
  seg.end[0] = seg.end[1] = seg.end[2] = (int)N;
  seg.scale[0] = seg.scale[1] = seg.scale[2] = ws;
  launch_ternary_matmul(c->b[1].as<uint32_t>(), (int)N, (int)K, c->b[2].as<int8_t>(), (int)padded_cols(K),
                        c->b[3].as<float>(), nullptr, 1, seg, Epi::Store, c->b[4].as<float>(), (int)N,
                        acc ? c->b[5].as<int32_t>() : nullptr, st);
  BN_CUDA(cudaMemcpyAsync(out, c->b[4].p, N * sizeof(float), cudaMemcpyDeviceToHost, st));
  if (acc) BN_CUDA(cudaMemcpyAsync(acc, c->b[5].p, N * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
  return finish(c);
}

// Copy host int8 activations into b2, zero padded to a multiple of 64.
int stage_xq(bitnet_cuda_ctx* c, const int8_t* xq, size_t K) {
  size_t kp = padded_cols(K);
  BN_TRY(c->b[2].ensure(kp));
  BN_CUDA(cudaMemsetAsync(c->b[2].p, 0, kp, c->stream));
  if (K) BN_CUDA(cudaMemcpyAsync(c->b[2].p, xq, K, cudaMemcpyHostToDevice, c->stream));
  return BITNET_OK;
}

// Quantise host f32 x (length K) on the device into b2 (padded) and b3
// (act_absmax); returns QuantizationError on a non-finite input.
int device_quantize(bitnet_cuda_ctx* c, const float* x, size_t K, float* scale_out) {
  if (K > (size_t)kMaxRowFloats)
    return backend_error("activation rows longer than " + std::to_string(kMaxRowFloats) + " are not supported");
  cudaStream_t st = c->stream;
  BN_TRY(upload(c->b[6], x, K * sizeof(float), st));
  BN_TRY(c->b[2].ensure(padded_cols(K)));
  BN_TRY(c->b[3].ensure(2 * sizeof(float)));
  BN_TRY(reset_status(c));
  float* dev_amax = c->b[3].as<float>();
  launch_quantize_rows(c->b[6].p, false, (int)K, 1, (int)K, c->b[2].as<int8_t>(), (int)padded_cols(K), dev_amax,
                       dev_amax + 1, nullptr, c->status.as<int32_t>(), st);
  BN_CUDA(cudaGetLastError());
  int32_t status = 0;
  BN_TRY(read_status(c, &status));
  if (status) return quant_error("non-finite activation value");
  if (scale_out) BN_CUDA(cudaMemcpy(scale_out, dev_amax + 1, sizeof(float), cudaMemcpyDeviceToHost));
  return BITNET_OK;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

const char* bitnet_cuda_last_error(void) { return g_last_error.c_str(); }
const char* bitnet_cuda_last_error_expected(void) { return g_last_expected.c_str(); }
int bitnet_cuda_kernel_binary_version(int32_t* out) {
  if (!out) return shape_error("non-null out", "null");
  int v = 0;
  const int e = kernel_binary_version(&v);
  if (e) return cuda_error((cudaError_t)e, "cudaFuncGetAttributes");
  *out = v;
  return BITNET_OK;
}
const char* bitnet_cuda_last_error_got(void) { return g_last_got.c_str(); }
const char* bitnet_cuda_version(void) { return "bitnetrs-b200 0.1.0 (sm_100a)"; }

int bitnet_cuda_create(uint32_t device_id, bitnet_cuda_ctx** out) {
  if (!out) return shape_error("non-null out pointer", "null");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDeviceCount");
  if ((int)device_id >= n)
    return backend_error("CUDA device " + std::to_string(device_id) + " not present (" + std::to_string(n) + " devices)");
  BN_CUDA(cudaSetDevice((int)device_id));
  cudaDeviceProp prop;
  BN_CUDA(cudaGetDeviceProperties(&prop, (int)device_id));
  if (prop.major < 10)
    return backend_error(std::string("device ") + prop.name + " is not sm_100 (this build targets sm_100a)");
  auto* c = new bitnet_cuda_ctx();
  c->device = (int)device_id;
  c->name = std::string("CUDA ") + prop.name + " (sm_" + std::to_string(prop.major) + std::to_string(prop.minor) + ")";
  e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete c;
    return cuda_error(e, "cudaStreamCreate");
  }
  int rc = c->status.ensure(64);
  if (rc) {
    delete c;
    return rc;
  }
  if (row_kernels_prepare() != 0 || sampler_prepare() != 0) {
    delete c;
    return backend_error("raising the shared-memory limit of the row kernels failed");
  }
  {
    static std::mutex tc_mu;
    static bool tc_failed = false;
    std::lock_guard<std::mutex> lk(tc_mu);
    if (ternary_tc_prepare() != 0) tc_failed = true;
    set_ternary_tc_ready(!tc_failed);
  }
  *out = c;
  return BITNET_OK;
}

void bitnet_cuda_destroy(bitnet_cuda_ctx* c) {
  if (c) ctx_release(c);
}

const char* bitnet_cuda_device_name(const bitnet_cuda_ctx* c) { return c ? c->name.c_str() : ""; }

uint64_t bitnet_cuda_kernel_launches(const bitnet_cuda_ctx*) { return launches_total(); }

// ---- ternary_gemv (f32 input) -----------------------------------------------
int bitnet_cuda_ternary_gemv(bitnet_cuda_ctx* c, const uint8_t* w, size_t w_len, float ws, const float* x,
                             size_t x_len, float* out, size_t out_len, size_t N, size_t K) {
  size_t pc = (K + 3) / 4;
  if (N != 0 && pc > SIZE_MAX / N) return shape_error("weight size fits usize", "overflow");
  if (w_len != N * pc)
    return shape_error("weight_packed.len() == " + sz(N) + " * ceil(" + sz(K) + "/4) = " + sz(N * pc),
                       "weight_packed.len() == " + sz(w_len));
  if (x_len != K) return shape_error("input.len() == " + sz(K), "input.len() == " + sz(x_len));
  if (out_len != N) return shape_error("output.len() == " + sz(N), "output.len() == " + sz(out_len));
  if (!(ws > 0.0f) || !std::isfinite(ws)) return quant_error("weight_scale must be finite and > 0");
  if (N == 0) return BITNET_OK;
  Guard g(c);
  cudaStream_t st = c->stream;
  BN_TRY(upload(c->b[0], w, w_len, st));
  BN_TRY(upload(c->b[6], x, K * sizeof(float), st));
  BN_TRY(c->b[4].ensure(N * sizeof(float)));
  launch_ternary_gemv_f32(c->b[0].as<uint8_t>(), (int)N, (int)K, ws, c->b[6].as<float>(), c->b[4].as<float>(), st);
  BN_CUDA(cudaMemcpyAsync(out, c->b[4].p, N * sizeof(float), cudaMemcpyDeviceToHost, st));
  return finish(c);
}

// ---- ternary_gemv_preq ---------------------------------------------------------
int bitnet_cuda_ternary_gemv_preq_acc(bitnet_cuda_ctx* c, const uint8_t* w, size_t w_len, float ws,
                                      const int8_t* xq, size_t xq_len, float act_absmax, float* out, size_t out_len,
                                      int32_t* acc, size_t N, size_t K) {
  BN_TRY(validate_quantised(w_len, ws, xq_len, act_absmax, out_len, N, K));
  if (N == 0) return BITNET_OK;
  Guard g(c);
  BN_TRY(stage_xq(c, xq, K));
  return run_gemv_preq(c, w, ws, N, K, act_absmax, out, acc);
}

int bitnet_cuda_ternary_gemv_preq(bitnet_cuda_ctx* c, const uint8_t* w, size_t w_len, float ws, const int8_t* xq,
                                  size_t xq_len, float act_absmax, float* out, size_t out_len, size_t N, size_t K) {
  return bitnet_cuda_ternary_gemv_preq_acc(c, w, w_len, ws, xq, xq_len, act_absmax, out, out_len, nullptr, N, K);
}

// ---- ternary_gemv_with_activation_quant (cpu/src/lib.rs:223-249) ----------------
int bitnet_cuda_ternary_gemv_with_activation_quant(bitnet_cuda_ctx* c, const uint8_t* w, size_t w_len, float ws,
                                                   const float* x, size_t x_len, float* out, size_t out_len, size_t N,
                                                   size_t K) {
  // absmax_quantize_row_into(input, scratch[in_features]) runs first.
  if (x_len == 0) return quant_error("cannot quantise an empty activation vector");
  if (x_len != K) return quant_error("output buffer length " + sz(K) + " != input length " + sz(x_len));
  Guard g(c);
  float scale = 0.0f;
  BN_TRY(device_quantize(c, x, K, &scale));
  float max_abs = scale * 127.0f;
  BN_TRY(validate_quantised(w_len, ws, K, max_abs, out_len, N, K));
  if (N == 0) return BITNET_OK;
  return run_gemv_preq(c, w, ws, N, K, max_abs, out, nullptr);
}

int bitnet_cuda_absmax_quantize_row(bitnet_cuda_ctx* c, const float* x, size_t len, int8_t* out, size_t out_len,
                                    float* scale) {
  if (len == 0) return quant_error("cannot quantise an empty activation vector");
  if (out_len != len) return quant_error("output buffer length " + sz(out_len) + " != input length " + sz(len));
  Guard g(c);
  float s = 0.0f;
  BN_TRY(device_quantize(c, x, len, &s));
  BN_CUDA(cudaMemcpy(out, c->b[2].p, len, cudaMemcpyDeviceToHost));
  if (scale) *scale = s;
  return BITNET_OK;
}

// ---- rms_norm (norm.rs:77-107) -------------------------------------------------
int bitnet_cuda_rms_norm(bitnet_cuda_ctx* c, const float* x, size_t xl, const float* w, size_t wl, float eps,
                         float* out, size_t ol) {
  if (xl != wl) return shape_error("input.len() == weight.len() = " + sz(wl), "input.len() = " + sz(xl));
  if (xl != ol) return shape_error("input.len() == output.len() = " + sz(xl), "output.len() = " + sz(ol));
  if (!(eps > 0.0f) || !std::isfinite(eps)) return quant_error("eps must be finite and > 0");
  if (xl == 0) return BITNET_OK;
  if (xl > (size_t)kMaxRowFloats)
    return backend_error("rms_norm rows longer than " + sz(kMaxRowFloats) + " are not supported");
  Guard g(c);
  cudaStream_t st = c->stream;
  BN_TRY(upload(c->b[0], x, xl * 4, st));
  BN_TRY(upload(c->b[1], w, xl * 4, st));
  BN_TRY(c->b[4].ensure(xl * 4));
  launch_rms_norm(c->b[0].as<float>(), (int)xl, c->b[1].as<float>(), (int)xl, eps, c->b[4].as<float>(), (int)xl, 1, st);
  BN_CUDA(cudaMemcpyAsync(out, c->b[4].p, xl * 4, cudaMemcpyDeviceToHost, st));
  return finish(c);
}

// ---- rope_embed (cpu/src/lib.rs:289-314, rope.rs:312-355) ----------------------
int bitnet_cuda_rope_embed(bitnet_cuda_ctx* c, float* q, size_t ql, float* k, size_t kl, size_t pos, size_t hd,
                           size_t nh, size_t nkv, float theta) {
  Guard g(c);
  RopeTable& R = c->rope;
  bool reinit = !R.valid || R.head_dim != hd || std::fabs(R.theta - theta) > 1e-3f || pos >= R.max_seq;
  if (reinit) {
    size_t ms = std::max<size_t>(pos + 1, 4096);
    std::vector<float> cs, sn;
    BN_TRY(build_rope_host(ms, hd, theta, cs, sn));
    R.cos.swap(cs);
    R.sin.swap(sn);
    R.head_dim = hd;
    R.theta = theta;
    R.max_seq = ms;
    R.valid = true;
    BN_TRY(upload(R.d_cos, R.cos.data(), R.cos.size() * 4, c->stream));
    BN_TRY(upload(R.d_sin, R.sin.data(), R.sin.size() * 4, c->stream));
  }
  size_t h = R.head_dim;
  if (ql != nh * h) return shape_error("q.len() == " + sz(nh) + " * " + sz(h) + " = " + sz(nh * h), "q.len() = " + sz(ql));
  if (kl != nkv * h)
    return shape_error("k.len() == " + sz(nkv) + " * " + sz(h) + " = " + sz(nkv * h), "k.len() = " + sz(kl));
  if (ql == 0 && kl == 0) return BITNET_OK;
  cudaStream_t st = c->stream;
  // One row [q | k] rotated with the table row of `pos`.
  std::vector<float> row(ql + kl);
  std::memcpy(row.data(), q, ql * 4);
  std::memcpy(row.data() + ql, k, kl * 4);
  BN_TRY(upload(c->b[0], row.data(), row.size() * 4, st));
  BN_TRY(c->b[4].ensure((ql + kl + 1) * 4));
  launch_rope_apply(c->b[0].as<float>(), (int)nh, (int)nkv, (int)h, R.d_cos.as<float>(), R.d_sin.as<float>(), pos,
                    c->b[4].as<float>(), st);
  BN_CUDA(cudaMemcpyAsync(q, c->b[4].p, ql * 4, cudaMemcpyDeviceToHost, st));
  BN_CUDA(cudaMemcpyAsync(k, c->b[4].as<float>() + ql, kl * 4, cudaMemcpyDeviceToHost, st));
  return finish(c);
}

// ---- masked_attention (attention.rs:97-209) -------------------------------------
int bitnet_cuda_masked_attention(bitnet_cuda_ctx* c, const float* q, size_t ql, const float* kc, size_t kl,
                                 const float* vc, size_t vl, float* out, size_t ol, size_t nh, size_t nkv, size_t hd,
                                 size_t cur_pos) {
  if (hd == 0) return shape_error("head_dim > 0", "head_dim = 0");
  if (nkv == 0) return config_error("n_kv_heads must be > 0");
  if (nh == 0) return config_error("n_heads must be > 0");
  if (nh % nkv != 0) return config_error("n_heads (" + sz(nh) + ") must be divisible by n_kv_heads (" + sz(nkv) + ")");
  size_t seq_len = cur_pos + 1;
  size_t stride = kl / nkv;
  size_t required = nkv * stride;
  size_t qe = nh * hd;
  if (ql != qe) return shape_error("q.len() == n_heads * head_dim = " + sz(qe), "q.len() = " + sz(ql));
  if (kl < required) return shape_error("k_cache.len() >= " + sz(required), "k_cache.len() = " + sz(kl));
  if (vl < required) return shape_error("v_cache.len() >= " + sz(required), "v_cache.len() = " + sz(vl));
  if (stride < seq_len * hd)
    return shape_error("per-head cache stride >= " + sz(seq_len * hd), "per-head cache stride = " + sz(stride));
  if (ol != qe) return shape_error("output.len() == n_heads * head_dim = " + sz(qe), "output.len() = " + sz(ol));
  Guard g(c);
  cudaStream_t st = c->stream;
  size_t used = seq_len * hd;  // only positions 0..=cur_pos of each head are read
  BN_TRY(upload(c->b[0], q, ql * 4, st));
  BN_TRY(c->b[1].ensure(nkv * used * 4));
  BN_TRY(c->b[2].ensure(nkv * used * 4));
  BN_CUDA(cudaMemcpy2DAsync(c->b[1].p, used * 4, kc, stride * 4, used * 4, nkv, cudaMemcpyHostToDevice, st));
  BN_CUDA(cudaMemcpy2DAsync(c->b[2].p, used * 4, vc, stride * 4, used * 4, nkv, cudaMemcpyHostToDevice, st));
  BN_TRY(c->b[3].ensure(nh * seq_len * 4));
  BN_TRY(c->b[4].ensure(qe * 4));
  BN_TRY(ensure_exp_table(c));
  launch_masked_attention_headmajor(c->b[0].as<float>(), c->b[1].as<float>(), c->b[2].as<float>(), c->b[4].as<float>(),
                                    (int)nh, (int)nkv, (int)hd, (int)used, (int)seq_len, c->b[3].as<float>(),
                                    c->exp_table, st);
  BN_CUDA(cudaMemcpyAsync(out, c->b[4].p, qe * 4, cudaMemcpyDeviceToHost, st));
  return finish(c);
}

// ---- activations -------------------------------------------------------------
int bitnet_cuda_squared_relu(bitnet_cuda_ctx* c, float* x, size_t n) {
  if (n == 0) return BITNET_OK;
  Guard g(c);
  BN_TRY(upload(c->b[0], x, n * 4, c->stream));
  launch_squared_relu(c->b[0].as<float>(), n, c->stream);
  BN_CUDA(cudaMemcpyAsync(x, c->b[0].p, n * 4, cudaMemcpyDeviceToHost, c->stream));
  return finish(c);
}

int bitnet_cuda_softmax(bitnet_cuda_ctx* c, float* x, size_t n) {
  if (n == 0) return BITNET_OK;
  Guard g(c);
  BN_TRY(upload(c->b[0], x, n * 4, c->stream));
  BN_TRY(c->b[1].ensure(16));
  BN_TRY(ensure_exp_table(c));
  launch_softmax(c->b[0].as<float>(), n, c->b[1].as<float>(), c->exp_table, c->stream);
  BN_CUDA(cudaMemcpyAsync(x, c->b[0].p, n * 4, cudaMemcpyDeviceToHost, c->stream));
  return finish(c);
}

int bitnet_cuda_elementwise_mul(bitnet_cuda_ctx* c, const float* a, size_t al, const float* b, size_t bl, float* out,
                                size_t ol) {
  if (al != bl) return shape_error("a.len() == b.len() = " + sz(bl), "a.len() = " + sz(al));
  if (al != ol) return shape_error("a.len() == out.len() = " + sz(ol), "a.len() = " + sz(al));
  if (al == 0) return BITNET_OK;
  Guard g(c);
  BN_TRY(upload(c->b[0], a, al * 4, c->stream));
  BN_TRY(upload(c->b[1], b, al * 4, c->stream));
  BN_TRY(c->b[4].ensure(al * 4));
  launch_elementwise_mul(c->b[0].as<float>(), c->b[1].as<float>(), c->b[4].as<float>(), al, c->stream);
  BN_CUDA(cudaMemcpyAsync(out, c->b[4].p, al * 4, cudaMemcpyDeviceToHost, c->stream));
  return finish(c);
}

int bitnet_cuda_sqrelu_gate(bitnet_cuda_ctx* c, const float* gate, size_t gl, const float* up, size_t ul, float* out,
                            size_t ol) {
  if (gl != ul || gl != ol)
    return shape_error("gate.len() == up.len() == out.len() = " + sz(gl), "up.len()=" + sz(ul) + ", out.len()=" + sz(ol));
  if (gl == 0) return BITNET_OK;
  Guard g(c);
  BN_TRY(upload(c->b[0], gate, gl * 4, c->stream));
  BN_TRY(upload(c->b[1], up, gl * 4, c->stream));
  BN_TRY(c->b[4].ensure(gl * 4));
  launch_sqrelu_gate(c->b[0].as<float>(), c->b[1].as<float>(), c->b[4].as<float>(), gl, c->stream);
  BN_CUDA(cudaMemcpyAsync(out, c->b[4].p, gl * 4, cudaMemcpyDeviceToHost, c->stream));
  return finish(c);
}

// ---- lm_head ------------------------------------------------------------------
static int lm_head_common(bitnet_cuda_ctx* c, const float* h, size_t hl, const void* w, size_t wl, size_t wbytes,
                          const float* scales, size_t sl, bool need_scales, float* out, size_t ol, size_t V, size_t H,
                          LmW wt) {
  if (hl != H) return shape_error("hidden.len() == " + sz(H), "hidden.len() = " + sz(hl));
  if (V != 0 && H > SIZE_MAX / V) return shape_error("weights size fits usize", "overflow");
  if (wl != V * H) return shape_error("weights.len() == " + sz(V) + " * " + sz(H), "weights.len() = " + sz(wl));
  if (need_scales && sl != V) return shape_error("scales.len() == " + sz(V), "scales.len() = " + sz(sl));
  if (ol != V) return shape_error("output.len() == " + sz(V), "output.len() = " + sz(ol));
  if (V == 0) return BITNET_OK;
  Guard g(c);
  cudaStream_t st = c->stream;
  BN_TRY(upload(c->b[0], h, H * 4, st));
  BN_TRY(upload(c->b[1], w, wl * wbytes, st));
  if (need_scales) BN_TRY(upload(c->b[2], scales, V * 4, st));
  BN_TRY(c->b[4].ensure(V * 4));
  launch_lm_head(c->b[1].p, wt, need_scales ? c->b[2].as<float>() : nullptr, c->b[0].as<float>(), (int)H, 1, (int)V,
                 (int)H, c->b[4].as<float>(), (int)V, st);
  BN_CUDA(cudaMemcpyAsync(out, c->b[4].p, V * 4, cudaMemcpyDeviceToHost, st));
  return finish(c);
}

int bitnet_cuda_lm_head_matmul_into(bitnet_cuda_ctx* c, const float* h, size_t hl, const float* w, size_t wl,
                                    float* out, size_t ol, size_t V, size_t H) {
  return lm_head_common(c, h, hl, w, wl, 4, nullptr, 0, false, out, ol, V, H, LmW::F32);
}
int bitnet_cuda_lm_head_matmul_bf16_into(bitnet_cuda_ctx* c, const float* h, size_t hl, const uint16_t* w, size_t wl,
                                         float* out, size_t ol, size_t V, size_t H) {
  return lm_head_common(c, h, hl, w, wl, 2, nullptr, 0, false, out, ol, V, H, LmW::BF16);
}
int bitnet_cuda_lm_head_matmul_i8_into(bitnet_cuda_ctx* c, const float* h, size_t hl, const int8_t* w, size_t wl,
                                       const float* scales, size_t sl, float* out, size_t ol, size_t V, size_t H) {
  return lm_head_common(c, h, hl, w, wl, 1, scales, sl, true, out, ol, V, H, LmW::I8);
}

int bitnet_cuda_greedy_argmax(bitnet_cuda_ctx* c, const float* logits, size_t n, uint32_t* token) {
  if (!token) return shape_error("non-null token", "null");
  if (n == 0) {
    *token = 0;
    return BITNET_OK;
  }
  Guard g(c);
  BN_TRY(upload(c->b[0], logits, n * 4, c->stream));
  BN_TRY(c->b[1].ensure(4));
  launch_argmax(c->b[0].as<float>(), (int)n, 1, (int)n, c->b[1].as<uint32_t>(), c->stream);
  BN_CUDA(cudaMemcpyAsync(token, c->b[1].p, 4, cudaMemcpyDeviceToHost, c->stream));
  return finish(c);
}

// ---- sampling -----------------------------------------------------------------------
}  // extern "C"

namespace bitnet {
int validate_sampling(const bitnet_cuda_sampling& cfg, size_t max_new_tokens) {
  if (!(cfg.temperature > 0.0f))
    return config_error("temperature must be > 0, got " + std::to_string(cfg.temperature));
  if (!(cfg.top_p > 0.0f && cfg.top_p <= 1.0f))
    return config_error("top_p must be in (0, 1], got " + std::to_string(cfg.top_p));
  if (cfg.repetition_penalty < 1.0f)
    return config_error("repetition_penalty must be >= 1.0, got " + std::to_string(cfg.repetition_penalty));
  if (max_new_tokens == 0) return config_error("max_new_tokens must be > 0");
  return BITNET_OK;
}

int sample_device(bitnet_cuda_ctx* c, float* d_logits, size_t V, const bitnet_cuda_sampling& cfg,
                  const uint32_t* d_past, size_t n_past, uint32_t* token, cudaStream_t st) {
  if (V > 0x7fffffffu || n_past > 0xffffffffu) return shape_error("vocab < 2^31 and history < 2^32", sz(V));
  BN_TRY(ensure_exp_table(c));
  void* before = c->samp_counts.p;
  BN_TRY(c->samp_counts.ensure(V * 4));
  if (c->samp_counts.p != before) BN_CUDA(cudaMemsetAsync(c->samp_counts.p, 0, c->samp_counts.cap, st));
  BN_TRY(c->samp_e.ensure(V * 4));
  BN_TRY(c->samp_misc.ensure(16));
  BN_CUDA(cudaMemsetAsync(c->samp_misc.p, 0, 16, st));
  uint32_t* misc = c->samp_misc.as<uint32_t>();
  launch_sample(d_logits, (uint32_t)V, cfg, d_past, (uint32_t)n_past, c->samp_counts.as<int32_t>(),
                c->samp_e.as<float>(), misc, reinterpret_cast<int32_t*>(misc + 1), c->exp_table, st);
  BN_CUDA(cudaGetLastError());
  uint32_t h[2] = {0, 0};
  BN_CUDA(cudaMemcpyAsync(h, misc, 8, cudaMemcpyDeviceToHost, st));
  BN_CUDA(cudaStreamSynchronize(st));
  if (h[1]) return backend_error("top-p over more than 4096 finite logits is not supported by the device sampler");
  *token = h[0];
  return BITNET_OK;
}
}  // namespace bitnet

extern "C" {

int bitnet_cuda_sample_next_token(bitnet_cuda_ctx* c, float* logits, size_t vocab, const bitnet_cuda_sampling* cfg,
                                  const uint32_t* past, size_t n_past, uint32_t* token) {
  if (!c || !cfg || !token) return shape_error("non-null context, config and token", "null");
  if (vocab == 0) {
    *token = 0;
    return BITNET_OK;
  }
  if (!logits || (n_past && !past)) return shape_error("non-null logits and history", "null");
  Guard g(c);
  BN_TRY(upload(c->b[0], logits, vocab * 4, c->stream));
  if (n_past) BN_TRY(upload(c->b[1], past, n_past * 4, c->stream));
  BN_TRY(sample_device(c, c->b[0].as<float>(), vocab, *cfg, n_past ? c->b[1].as<uint32_t>() : nullptr, n_past, token,
                       c->stream));
  // the reference modifies the logits in place (penalty, temperature, masks)
  BN_CUDA(cudaMemcpyAsync(logits, c->b[0].p, vocab * 4, cudaMemcpyDeviceToHost, c->stream));
  return finish(c);
}

// ---- device-resident ternary matmul -------------------------------------------------
int bitnet_cuda_weight_upload(bitnet_cuda_ctx* c, const uint8_t* packed, size_t packed_len, size_t rows, size_t cols,
                              float scale, bitnet_cuda_weight** out) {
  if (!out) return shape_error("non-null out", "null");
  *out = nullptr;
  size_t pc = (cols + 3) / 4;
  if (packed_len != rows * pc)
    return shape_error("packed data: " + sz(rows) + " * ((" + sz(cols) + " + 3) / 4) = " + sz(rows * pc) + " bytes",
                       sz(packed_len) + " bytes");
  if (!(scale > 0.0f) || !std::isfinite(scale)) return quant_error("scale must be finite and > 0");
  Guard g(c);
  DevBuf raw;
  BN_TRY(upload(raw, packed, packed_len, c->stream));
  auto* w = new bitnet_cuda_weight();
  w->ctx = c;
  w->rows = (int)rows;
  w->cols = (int)cols;
  w->scale = scale;
  cudaError_t e = cudaMalloc(&w->words, std::max<size_t>(rows * words_per_row(cols) * 4, 16));
  if (e != cudaSuccess) {
    delete w;
    return cuda_error(e, "cudaMalloc");
  }
  launch_repack_ternary(raw.as<uint8_t>(), w->words, (int)rows, (int)cols, c->stream);
  int rc = finish(c);
  if (rc) {
    cudaFree(w->words);
    delete w;
    return rc;
  }
  ctx_retain(c);
  *out = w;
  return BITNET_OK;
}

void bitnet_cuda_weight_destroy(bitnet_cuda_weight* w) {
  if (!w) return;
  bitnet_cuda_ctx* c = w->ctx;
  cudaSetDevice(c->device);
  cudaFree(w->words);
  delete w;
  ctx_release(c);
}

int bitnet_cuda_quantize_rows_device(bitnet_cuda_ctx* c, const void* x, int x_is_bf16, size_t M, size_t K, int8_t* xq,
                                     size_t ldq, float* act_absmax, int32_t* row_sum, int32_t* status, void* stream) {
  if (K == 0) return quant_error("cannot quantise an empty activation vector");
  if (ldq < K || ldq % 64 != 0) return shape_error("ldq >= K and a multiple of 64", "ldq = " + sz(ldq));
  if (K > (size_t)kMaxRowFloats) return shape_error("K <= " + sz(kMaxRowFloats), "K = " + sz(K));
  cudaSetDevice(c->device);
  cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
  launch_quantize_rows(x, x_is_bf16 != 0, (int)K, (int)M, (int)K, xq, (int)ldq, act_absmax, nullptr, row_sum, status,
                       st);
  BN_CUDA(cudaGetLastError());
  return BITNET_OK;
}

int bitnet_cuda_ternary_matmul_device(bitnet_cuda_ctx* c, const bitnet_cuda_weight* w, const int8_t* xq, size_t ldq,
                                      const float* act_absmax, const int32_t* row_sum, size_t M, float* out,
                                      int32_t* acc, void* stream) {
  if (!w) return shape_error("weight handle", "null");
  if (ldq < padded_cols(w->cols)) return shape_error("ldq >= " + sz(padded_cols(w->cols)), "ldq = " + sz(ldq));
  cudaSetDevice(c->device);
  cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
  Segments seg;
  seg.end[0] = seg.end[1] = seg.end[2] = w->rows;
  seg.scale[0] = seg.scale[1] = seg.scale[2] = w->scale;
  launch_ternary_matmul(w->words, w->rows, w->cols, xq, (int)ldq, act_absmax, row_sum, (int)M, seg, Epi::Store, out,
                        w->rows, acc, st, c->status.as<int32_t>());
  BN_CUDA(cudaGetLastError());
  return BITNET_OK;
}

}  // extern "C"
