/* trait_forward.c -- BitNetModel::forward_into's decode path driven through
 * the host-slice entry points of include/bitnet_cuda.h, one trait call per
 * reference call, in the reference's order
 * (crates/bitnet-model/src/lib.rs:931-1163).  This is what a Rust
 * CudaBackend shim does when the reference model calls it op by op; the
 * KV cache lives on the host in the reference's head-major layout
 * [layer][kv_head][max_seq][head_dim] (KVCache::store_kv, lib.rs:154-199).
 *
 *   trait_forward <model.bin> <logits.out>
 *
 * model.bin (little-endian): "BNTF", u32 version 1; u32 vocab, hidden,
 * layers, heads, kv_heads, intermediate, max_pos; f32 rope_theta, eps;
 * per layer the seven projections q k v o gate up down as (u64 nbytes,
 * packed bytes in the reference 2-bit format, f32 scale), then the four f32
 * norms (attention, attn_sub [q_dim], ffn, ffn_sub [intermediate]); the
 * bf16 embedding [vocab][hidden] (u16 bits), the i8 lm_head [vocab][hidden],
 * its f32 scales [vocab], the f32 final norm [hidden]; u32 n and n token
 * ids, decoded at positions 0..n-1.  logits.out: n rows of vocab f32.
 * Exit status 0 on success; a failing call prints the library's message. */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "bitnet_cuda.h"

typedef struct {
  uint8_t* w[7];
  size_t wlen[7];
  float s[7];
  float *attn_norm, *attn_sub_norm, *ffn_norm, *ffn_sub_norm;
} Layer;

static FILE* g_in;

static void* rd(size_t bytes) {
  void* p = malloc(bytes ? bytes : 1);
  if (!p || fread(p, 1, bytes, g_in) != bytes) {
    fprintf(stderr, "trait_forward: short read\n");
    exit(2);
  }
  return p;
}
static uint32_t rd_u32(void) {
  uint32_t v;
  if (fread(&v, 4, 1, g_in) != 1) exit(2);
  return v;
}
static float rd_f32(void) {
  float v;
  if (fread(&v, 4, 1, g_in) != 1) exit(2);
  return v;
}
static uint64_t rd_u64(void) {
  uint64_t v;
  if (fread(&v, 8, 1, g_in) != 1) exit(2);
  return v;
}

#define CALL(x)                                                                       \
  do {                                                                                \
    int rc_ = (x);                                                                    \
    if (rc_ != BITNET_OK) {                                                           \
      fprintf(stderr, "trait_forward: %s -> %d: %s\n", #x, rc_, bitnet_cuda_last_error()); \
      exit(1);                                                                        \
    }                                                                                 \
  } while (0)

int main(int argc, char** argv) {
  if (argc != 3) {
    fprintf(stderr, "usage: trait_forward <model.bin> <logits.out>\n");
    return 2;
  }
  g_in = fopen(argv[1], "rb");
  if (!g_in) return 2;
  char magic[4];
  if (fread(magic, 1, 4, g_in) != 4 || memcmp(magic, "BNTF", 4) != 0 || rd_u32() != 1) return 2;
  const size_t V = rd_u32(), H = rd_u32(), NL = rd_u32(), NH = rd_u32(), NKV = rd_u32(), F = rd_u32(),
               MAXP = rd_u32();
  const float theta = rd_f32(), eps = rd_f32();
  const size_t HD = H / NH, QD = NH * HD, KVD = NKV * HD;
  Layer* layers = calloc(NL, sizeof(Layer));
  for (size_t l = 0; l < NL; ++l) {
    for (int p = 0; p < 7; ++p) {
      layers[l].wlen[p] = (size_t)rd_u64();
      layers[l].w[p] = rd(layers[l].wlen[p]);
      layers[l].s[p] = rd_f32();
    }
    layers[l].attn_norm = rd(H * 4);
    layers[l].attn_sub_norm = rd(QD * 4);
    layers[l].ffn_norm = rd(H * 4);
    layers[l].ffn_sub_norm = rd(F * 4);
  }
  uint16_t* embed = rd(V * H * 2);
  int8_t* lm_i8 = rd(V * H);
  float* lm_scales = rd(V * 4);
  float* final_norm = rd(H * 4);
  const size_t n_tok = rd_u32();
  uint32_t* tokens = rd(n_tok * 4);
  fclose(g_in);
  if (n_tok > MAXP) return 2;

  bitnet_cuda_ctx* ctx = NULL;
  CALL(bitnet_cuda_create(0, &ctx));
  const size_t max_seq = n_tok;
  float** kc = calloc(NL, sizeof(float*));
  float** vc = calloc(NL, sizeof(float*));
  for (size_t l = 0; l < NL; ++l) {
    kc[l] = calloc(NKV * max_seq * HD, 4);
    vc[l] = calloc(NKV * max_seq * HD, 4);
  }
  float *h = malloc(H * 4), *h_norm = malloc(H * 4), *q = malloc(QD * 4), *k = malloc(KVD * 4),
        *v = malloc(KVD * 4), *attn = malloc(QD * 4), *attn_n = malloc(QD * 4), *o = malloc(H * 4),
        *gate = malloc(F * 4), *up = malloc(F * 4), *inner = malloc(F * 4), *inner_n = malloc(F * 4),
        *ffn_out = malloc(H * 4), *logits = malloc(V * 4);
  int8_t* xq = malloc(H);
  FILE* out = fopen(argv[2], "wb");
  if (!out) return 2;

  for (size_t t = 0; t < n_tok; ++t) {
    const size_t pos = t;
    /* embedding row, bf16 -> f32 (lib.rs:937-944) */
    for (size_t i = 0; i < H; ++i) {
      uint32_t b = (uint32_t)embed[(size_t)tokens[t] * H + i] << 16;
      memcpy(&h[i], &b, 4);
    }
    for (size_t l = 0; l < NL; ++l) {
      const Layer* L = &layers[l];
      float qs;
      CALL(bitnet_cuda_rms_norm(ctx, h, H, L->attn_norm, H, eps, h_norm, H));
      CALL(bitnet_cuda_absmax_quantize_row(ctx, h_norm, H, xq, H, &qs));
      const float amax_qkv = qs * 127.0f;
      CALL(bitnet_cuda_ternary_gemv_preq(ctx, L->w[0], L->wlen[0], L->s[0], xq, H, amax_qkv, q, QD, QD, H));
      CALL(bitnet_cuda_ternary_gemv_preq(ctx, L->w[1], L->wlen[1], L->s[1], xq, H, amax_qkv, k, KVD, KVD, H));
      CALL(bitnet_cuda_ternary_gemv_preq(ctx, L->w[2], L->wlen[2], L->s[2], xq, H, amax_qkv, v, KVD, KVD, H));
      CALL(bitnet_cuda_rope_embed(ctx, q, QD, k, KVD, pos, HD, NH, NKV, theta));
      /* KVCache::store_kv: head-major [kv_head][max_seq][head_dim] */
      for (size_t g = 0; g < NKV; ++g) {
        memcpy(kc[l] + (g * max_seq + pos) * HD, k + g * HD, HD * 4);
        memcpy(vc[l] + (g * max_seq + pos) * HD, v + g * HD, HD * 4);
      }
      CALL(bitnet_cuda_masked_attention(ctx, q, QD, kc[l], NKV * max_seq * HD, vc[l], NKV * max_seq * HD, attn, QD,
                                        NH, NKV, HD, pos));
      CALL(bitnet_cuda_rms_norm(ctx, attn, QD, L->attn_sub_norm, QD, eps, attn_n, QD));
      CALL(bitnet_cuda_ternary_gemv_with_activation_quant(ctx, L->w[3], L->wlen[3], L->s[3], attn_n, QD, o, H, H,
                                                          QD));
      for (size_t i = 0; i < H; ++i) h[i] = h[i] + o[i]; /* axpy_f32_fast(1.0, o, h) */
      CALL(bitnet_cuda_rms_norm(ctx, h, H, L->ffn_norm, H, eps, h_norm, H));
      CALL(bitnet_cuda_absmax_quantize_row(ctx, h_norm, H, xq, H, &qs));
      const float amax_ffn = qs * 127.0f;
      CALL(bitnet_cuda_ternary_gemv_preq(ctx, L->w[4], L->wlen[4], L->s[4], xq, H, amax_ffn, gate, F, F, H));
      CALL(bitnet_cuda_ternary_gemv_preq(ctx, L->w[5], L->wlen[5], L->s[5], xq, H, amax_ffn, up, F, F, H));
      CALL(bitnet_cuda_sqrelu_gate(ctx, gate, F, up, F, inner, F));
      CALL(bitnet_cuda_rms_norm(ctx, inner, F, L->ffn_sub_norm, F, eps, inner_n, F));
      CALL(bitnet_cuda_ternary_gemv_with_activation_quant(ctx, L->w[6], L->wlen[6], L->s[6], inner_n, F, ffn_out, H,
                                                          H, F));
      for (size_t i = 0; i < H; ++i) h[i] = h[i] + ffn_out[i];
    }
    CALL(bitnet_cuda_rms_norm(ctx, h, H, final_norm, H, eps, h_norm, H));
    CALL(bitnet_cuda_lm_head_matmul_i8_into(ctx, h_norm, H, lm_i8, V * H, lm_scales, V, logits, V, V, H));
    if (fwrite(logits, 4, V, out) != V) return 2;
  }
  fclose(out);
  bitnet_cuda_destroy(ctx);
  return 0;
}
