// ingest.cu — host-side conversion of checkpoint tensors into the formats
// bitnet_cuda_model_create uploads: the HuggingFace packed ternary layout, a
// dense f32 projection (absmean ternarisation) and the bf16 embedding (the
// weight-tied i8 lm_head table). Rows are independent, so each conversion
// runs over all host threads; results do not depend on the thread count.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "internal.h"

using namespace bitnet;

namespace {

template <class F>
void parallel_rows(size_t rows, F f) {
  const size_t hw = std::max(1u, std::thread::hardware_concurrency());
  const size_t nt = std::min(hw, std::max<size_t>(1, rows / 16));
  if (nt <= 1) {
    f(0, rows);
    return;
  }
  std::vector<std::thread> th;
  const size_t per = (rows + nt - 1) / nt;
  for (size_t t = 0; t < nt; ++t) {
    const size_t b = t * per, e = std::min(rows, b + per);
    if (b < e) th.emplace_back([=] { f(b, e); });
  }
  for (auto& x : th) x.join();
}

bool mul_overflows(size_t a, size_t b, size_t* out) { return __builtin_mul_overflow(a, b, out); }

// Reference 2-bit code of a ternary value (ternary.rs:266-285): +1 -> 00, 0 -> 01, -1 -> 10.
inline uint8_t code_of(int v) { return v > 0 ? 0 : (v == 0 ? 1 : 2); }

std::string fmt_float(float x) {
  char b[48];
  std::snprintf(b, sizeof b, "%g", (double)x);
  return b;
}

}  // namespace

extern "C" {

// decode_packed_projection (crates/bitnet-convert/src/lib.rs:235-325): byte
// (r, c) of the stored [packed_rows][cols] tensor holds, at bits 2s..2s+1, the
// lane of logical row s * packed_rows + r, column c; the value is lane - 1 and
// lane 0b11 is an error. The Q/K LLaMA permutation is not applied
// (requires_llama_permute is false: the RoPE is half-split). Output: the
// reference runtime rows [4 * packed_rows][ceil(cols / 4)].
int bitnet_cuda_decode_hf_packed(const uint8_t* packed, size_t packed_len, size_t packed_rows, size_t cols,
                                 float weight_scale, uint8_t* out, size_t out_len) {
  if (packed_rows == 0) return shape_error("packed_rows > 0", "0");
  if (cols == 0) return shape_error("cols > 0", "0");
  if (!(weight_scale > 0.0f) || !std::isfinite(weight_scale))
    return quant_error("weight_scale must be finite and > 0, got " + fmt_float(weight_scale));
  size_t rows = 0, numel = 0;
  if (mul_overflows(packed_rows, 4, &rows)) return shape_error("packed_rows * 4 without overflow", "overflow");
  if (mul_overflows(rows, cols, &numel)) return shape_error("rows * cols without overflow", "overflow");
  const size_t need = (numel + 3) / 4;
  if (!packed || packed_len < need)
    return shape_error("at least " + std::to_string(need) + " packed bytes for " + std::to_string(numel) +
                           " logical elements",
                       std::to_string(packed ? packed_len : 0) + " bytes");
  const size_t pc = (cols + 3) / 4;
  if (!out || out_len < rows * pc)
    return shape_error("output of " + std::to_string(rows * pc) + " bytes", std::to_string(out ? out_len : 0));
  // The first invalid lane in the reference's scan order (packed row, column,
  // shift) is reported; each thread finds the first one of its rows.
  const size_t none = (size_t)-1;
  size_t first_bad = none;
  std::mutex mu;
  parallel_rows(packed_rows, [&](size_t r0, size_t r1) {
    size_t bad = none;
    for (size_t r = r0; r < r1 && bad == none; ++r) {
      const uint8_t* src = packed + r * cols;
      for (size_t c = 0; c < cols; ++c)
        if (src[c] & (src[c] >> 1) & 0x55) {
          bad = r * cols + c;
          break;
        }
    }
    for (size_t r = r0; r < r1; ++r) {
      const uint8_t* src = packed + r * cols;
      for (int s = 0; s < 4; ++s) {
        uint8_t* dst = out + ((size_t)s * packed_rows + r) * pc;
        std::memset(dst, 0, pc);
        for (size_t c = 0; c < cols; ++c) {
          const int lane = (src[c] >> (2 * s)) & 3;
          dst[c / 4] |= (uint8_t)(code_of(lane - 1) << (2 * (c % 4)));
        }
      }
    }
    if (bad != none) {
      std::lock_guard<std::mutex> lk(mu);
      first_bad = std::min(first_bad, bad);
    }
  });
  if (first_bad != none) {
    const size_t r = first_bad / cols, c = first_bad % cols;
    const uint8_t b = packed[first_bad];
    int s = 0;
    while (((b >> (2 * s)) & 3) != 3) ++s;
    return quant_error("invalid packed lane value 0b11 at packed position (" + std::to_string(r) + ", " +
                       std::to_string(c) + "), shift " + std::to_string(2 * s));
  }
  return BITNET_OK;
}

// quantise_weight (crates/bitnet-weights/src/loader.rs:1037-1070): absmean
// ternarisation of a dense f32 [rows][cols] tensor (absmean.rs:71-102:
// s = max(sequential f32 sum of |w| / n, 1e-5), q = clamp(round(w * (1/s)),
// -1, 1)) packed into the reference runtime rows [rows][ceil(cols / 4)].
int bitnet_cuda_absmean_ternary(const float* w, size_t rows, size_t cols, uint8_t* out, size_t out_len,
                                float* scale_out) {
  size_t n = 0;
  if (mul_overflows(rows, cols, &n)) return shape_error("rows * cols without overflow", "overflow");
  if (n == 0) return quant_error("cannot quantise an empty weight slice");
  if (!w || !scale_out) return shape_error("non-null weights and scale", "null");
  const size_t pc = (cols + 3) / 4;
  if (!out || out_len < rows * pc)
    return shape_error("output of " + std::to_string(rows * pc) + " bytes", std::to_string(out ? out_len : 0));
  for (size_t i = 0; i < n; ++i)
    if (!std::isfinite(w[i]))
      return quant_error("non-finite weight value at index " + std::to_string(i) + ": " + fmt_float(w[i]));
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) sum += std::fabs(w[i]);
  const float mean = sum / (float)n;
  const float s = std::max(mean, 1e-5f);
  const float inv = 1.0f / s;
  parallel_rows(rows, [&](size_t r0, size_t r1) {
    for (size_t r = r0; r < r1; ++r) {
      uint8_t* dst = out + r * pc;
      std::memset(dst, 0, pc);
      for (size_t c = 0; c < cols; ++c) {
        const float q = std::min(std::max(std::round(w[r * cols + c] * inv), -1.0f), 1.0f);
        dst[c / 4] |= (uint8_t)(code_of((int)q) << (2 * (c % 4)));
      }
    }
  });
  *scale_out = s;
  return BITNET_OK;
}

// quantize_bf16_rows_to_i8 (crates/bitnet-weights/src/loader.rs:297-340): per
// row m = max|e| (NaN ignored, at least 1e-10), scale m / 127,
// q = clamp(round(e * (127 / m)), -128, 127) (NaN -> 0, Rust's saturating cast).
int bitnet_cuda_lm_head_i8_table(const uint16_t* embed_bf16, size_t rows, size_t row_len, int8_t* out,
                                 float* scales) {
  size_t n = 0;
  if (mul_overflows(rows, row_len, &n)) return shape_error("rows * row_len without overflow", "overflow");
  if ((n && (!embed_bf16 || !out)) || (rows && !scales))
    return shape_error("non-null embedding, table and scales", "null");
  parallel_rows(rows, [&](size_t r0, size_t r1) {
    for (size_t r = r0; r < r1; ++r) {
      const uint16_t* e = embed_bf16 + r * row_len;
      float m = 0.0f;
      for (size_t i = 0; i < row_len; ++i) {
        uint32_t u = (uint32_t)e[i] << 16;
        float v;
        std::memcpy(&v, &u, 4);
        const float a = std::fabs(v);
        if (a > m) m = a;
      }
      if (m < 1e-10f) m = 1e-10f;
      const float inv = 127.0f / m;
      scales[r] = m / 127.0f;
      for (size_t i = 0; i < row_len; ++i) {
        uint32_t u = (uint32_t)e[i] << 16;
        float v;
        std::memcpy(&v, &u, 4);
        const float y = std::round(v * inv);
        out[r * row_len + i] = std::isnan(y) ? (int8_t)0 : (int8_t)std::min(std::max(y, -128.0f), 127.0f);
      }
    }
  });
  return BITNET_OK;
}

}  // extern "C"
