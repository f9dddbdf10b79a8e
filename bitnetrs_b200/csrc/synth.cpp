// synth.cpp — seeded synthetic inputs for benchmarks and parity tests.
//
// There is no checkpoint on the benchmark machines, so models are random-init
// with the reference's own quantisation pipeline:
//   * projections: W ~ N(0, std) f32, then absmean ternarisation
//     (crates/bitnet-core/src/quant/absmean.rs:71-102) and the 2-bit packing
//     (crates/bitnet-core/src/quant/ternary.rs:266-285);
//   * embedding: bf16 N(0, std); the weight-tied lm_head is its per-row absmax
//     i8 quantisation (crates/bitnet-weights/src/loader.rs:297-340).
// Random numbers are counter based (SplitMix64 finaliser over (seed, stream,
// index)) so any slice can be regenerated independently of thread count.
// Normal deviates: single-precision Box-Muller, both branches.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

constexpr uint64_t kGolden = 0x9e3779b97f4a7c15ULL;

inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}

inline uint64_t stream_key(uint64_t seed, uint64_t stream) { return mix64(seed ^ mix64(stream * kGolden + 0x77ULL)); }

// Box-Muller in single precision on one 64-bit draw: u1 from the top 24 bits
// (in (0, 1]), u2 from the low 24 bits; element 2j takes the cosine branch,
// element 2j+1 the sine branch of pair j.
inline float normal_at(uint64_t key, uint64_t i) {
  uint64_t a = mix64(key + (i >> 1) * kGolden);
  float u1 = (float)((a >> 40) + 1) * (1.0f / 16777216.0f);
  float u2 = (float)(a & 0xffffffu) * (1.0f / 16777216.0f);
  float r = std::sqrt(-2.0f * std::log(u1));
  float t = 6.28318530717958647692f * u2;
  return (i & 1) ? r * std::sin(t) : r * std::cos(t);
}

// Elements [b, e) of the same sequence as normal_at, scaled by stdev, with
// the radius of each pair computed once (same values, half the logarithms).
inline void normals_into(uint64_t key, uint64_t b, uint64_t e, float stdev, float* out) {
  uint64_t i = b;
  if (i < e && (i & 1)) *out++ = stdev * normal_at(key, i++);
  for (; i + 1 < e; i += 2) {
    uint64_t a = mix64(key + (i >> 1) * kGolden);
    float u1 = (float)((a >> 40) + 1) * (1.0f / 16777216.0f);
    float u2 = (float)(a & 0xffffffu) * (1.0f / 16777216.0f);
    float r = std::sqrt(-2.0f * std::log(u1));
    float t = 6.28318530717958647692f * u2;
    *out++ = stdev * (r * std::cos(t));
    *out++ = stdev * (r * std::sin(t));
  }
  if (i < e) *out = stdev * normal_at(key, i);
}

int g_threads = 0;

int nthreads() {
  int n = g_threads > 0 ? g_threads : (int)std::thread::hardware_concurrency();
  return std::max(1, n);
}

// Runs f(b, e) over [0, n) split across threads; `cost` is the work of one
// item in elements, so row loops spread over threads like element loops.
template <class F>
void par(size_t n, F f, size_t cost = 1) {
  int nt = (int)std::min<size_t>((size_t)nthreads(), std::max<size_t>(1, n * cost / 65536));
  if (nt <= 1) {
    f(0, n);
    return;
  }
  std::vector<std::thread> th;
  size_t per = (n + nt - 1) / nt;
  for (int t = 0; t < nt; ++t) {
    size_t b = t * per, e = std::min(n, b + per);
    if (b < e) th.emplace_back([=] { f(b, e); });
  }
  for (auto& x : th) x.join();
}

inline uint16_t f32_to_bf16(float x) {  // half::bf16::from_f32
  uint32_t u;
  std::memcpy(&u, &x, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u | 0x00400000u) >> 16);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
inline float bf16_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

}  // namespace

extern "C" {

int synth_set_threads(int n) {
  g_threads = n;
  return nthreads();
}

// out[i] = (float)(std * N(0,1)_{offset+i}) of stream (seed, stream).
void synth_normal_f32(uint64_t seed, uint64_t stream, uint64_t offset, size_t n, float stdev, float* out) {
  uint64_t key = stream_key(seed, stream);
  par(n, [&](size_t b, size_t e) { normals_into(key, offset + b, offset + e, stdev, out + b); });
}

void synth_bf16_normal(uint64_t seed, uint64_t stream, size_t n, float stdev, uint16_t* out) {
  uint64_t key = stream_key(seed, stream);
  par(n, [&](size_t b, size_t e) {
    for (size_t i = b; i < e; ++i) out[i] = f32_to_bf16(stdev * normal_at(key, i));
  });
}

// N(0, std) f32 [rows, cols] -> absmean ternary -> reference 2-bit rows.
// Returns 0, or 2 (QuantizationError) for an empty tensor.
int synth_ternary_absmean(uint64_t seed, uint64_t stream, size_t rows, size_t cols, float stdev, uint8_t* packed,
                          float* scale_out) {
  size_t n = rows * cols;
  if (n == 0) return 2;
  std::vector<float> w(n);
  synth_normal_f32(seed, stream, 0, n, stdev, w.data());
  // absmean.rs:90-93: sequential f32 sum of |w| in element order.
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) sum += std::fabs(w[i]);
  float mean = sum / (float)n;
  float scale = std::fmax(mean, 1e-5f);
  float inv = 1.0f / scale;
  size_t pc = (cols + 3) / 4;
  par(rows, [&](size_t b, size_t e) {
    for (size_t r = b; r < e; ++r) {
      uint8_t* dst = packed + r * pc;
      std::memset(dst, 0, pc);
      for (size_t c = 0; c < cols; ++c) {
        float q = std::round(w[r * cols + c] * inv);
        q = std::min(std::max(q, -1.0f), 1.0f);
        uint8_t bits = q > 0.5f ? 0 : (q < -0.5f ? 2 : 1);
        dst[c / 4] |= (uint8_t)(bits << (2 * (c % 4)));
      }
    }
  }, cols);
  *scale_out = scale;
  return 0;
}

// iid codes with P(-1) = p_neg, P(0) = p_zero, P(+1) = 1 - p_neg - p_zero.
void synth_ternary_codes(uint64_t seed, uint64_t stream, size_t rows, size_t cols, double p_neg, double p_zero,
                         uint8_t* packed) {
  uint64_t key = stream_key(seed, stream);
  size_t pc = (cols + 3) / 4;
  par(rows, [&](size_t b, size_t e) {
    for (size_t r = b; r < e; ++r) {
      uint8_t* dst = packed + r * pc;
      std::memset(dst, 0, pc);
      for (size_t c = 0; c < cols; ++c) {
        double u = (double)(mix64(key + (r * cols + c) * kGolden) >> 11) * (1.0 / 9007199254740992.0);
        uint8_t bits = u < p_neg ? 2 : (u < p_neg + p_zero ? 1 : 0);
        dst[c / 4] |= (uint8_t)(bits << (2 * (c % 4)));
      }
    }
  }, cols);
}

// loader.rs:297-340 (quantize_bf16_rows_to_i8).
void synth_quantize_bf16_rows_to_i8(const uint16_t* bf, size_t rows, size_t row_len, int8_t* out, float* scales) {
  par(rows, [&](size_t b, size_t e) {
    for (size_t r = b; r < e; ++r) {
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
    }
  }, row_len);
}

// Uniform integers in [lo, hi] (inclusive).
void synth_uniform_u32(uint64_t seed, uint64_t stream, size_t n, uint32_t lo, uint32_t hi, uint32_t* out) {
  uint64_t key = stream_key(seed, stream);
  uint64_t span = (uint64_t)hi - lo + 1;
  for (size_t i = 0; i < n; ++i) out[i] = lo + (uint32_t)(((mix64(key + i * kGolden) >> 32) * span) >> 32);
}

// The values bitnet_cuda_kv_seq_fill_random writes (before bf16 rounding),
// laid out [layer][pos][kv_head*hd] for positions [0, n).
void synth_kv_normal(uint64_t seed, uint32_t seq, uint32_t layers, uint32_t kv_heads, uint32_t hd, size_t n, float* k,
                     float* v) {
  par((size_t)layers * n, [&](size_t b, size_t e) {
    for (size_t lp = b; lp < e; ++lp) {
      uint32_t layer = (uint32_t)(lp / n);
      size_t pos = lp % n;
      for (uint32_t kind = 0; kind < 2; ++kind)
        for (uint32_t h = 0; h < kv_heads; ++h) {
          uint64_t key = mix64(seed ^ mix64(((uint64_t)seq << 40) ^ ((uint64_t)layer << 24) ^ ((uint64_t)kind << 20) ^
                                             ((uint64_t)h << 16) ^ 0x5eedULL));
          float* dst = (kind == 0 ? k : v) + (lp * kv_heads + h) * hd;
          normals_into(key, (uint64_t)pos * hd, (uint64_t)pos * hd + hd, 1.0f, dst);
        }
    }
  }, (size_t)2 * kv_heads * hd);
}

}  // extern "C"
