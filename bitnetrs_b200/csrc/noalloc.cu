// noalloc.cu — decode GEMV with activation quantisation that allocates
// nothing (bitnet_cuda_ternary_gemv_quant_noalloc).
//
// The activation scratch of ternary_gemv_with_activation_quant (the int8 row,
// its absmax, its code sum and the non-finite flag) normally lives in
// context buffers that are grown with cudaMalloc on demand.  This variant
// keeps it in one file-scope device array, g_scratch, sized for rows of up to
// kNoAllocMaxK elements; its address is resolved once per device with
// cudaGetSymbolAddress and passed to the kernels as a plain pointer.
#include <mutex>

#include "internal.h"

using namespace bitnet;

namespace {

constexpr size_t kNoAllocMaxK = 32768;  // longest activation row (int8 bytes)
// [0, kNoAllocMaxK) int8 row | +0 absmax f32 | +4 row sum i32 | +8 status i32
constexpr size_t kTail = kNoAllocMaxK;
static __device__ __align__(256) unsigned char g_scratch[kNoAllocMaxK + 256];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_addr[kMaxDevices] = {};

// Address of g_scratch on `device` (that device current); resolved on first use.
int scratch_address(int device, unsigned char** out) {
  if (device < 0 || device >= kMaxDevices) return backend_error("device ordinal out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(no-alloc scratch)");
    g_addr[device] = p;
  }
  *out = static_cast<unsigned char*>(g_addr[device]);
  return BITNET_OK;
}

}  // namespace

extern "C" {

int bitnet_cuda_ternary_gemv_quant_noalloc(bitnet_cuda_ctx* c, const bitnet_cuda_weight* w, const float* x,
                                           size_t x_len, float* out, size_t out_len, void* stream) {
  if (!c || !w) return shape_error("non-null context and weight", "null");
  if (x_len == 0) return quant_error("cannot quantise an empty activation vector");
  if (x_len != (size_t)w->cols) return shape_error("input length == in_features = " + std::to_string(w->cols),
                                                   "input length " + std::to_string(x_len));
  if (out_len != (size_t)w->rows)
    return shape_error("output length == out_features = " + std::to_string(w->rows),
                       "output length " + std::to_string(out_len));
  const size_t ldq = padded_cols(x_len);
  if (ldq > kNoAllocMaxK)
    return shape_error("in_features <= " + std::to_string(kNoAllocMaxK) + " (the no-alloc scratch)",
                       std::to_string(x_len));
  std::lock_guard<std::mutex> lk(c->mu);
  BN_CUDA(cudaSetDevice(c->device));
  unsigned char* s = nullptr;
  BN_TRY(scratch_address(c->device, &s));
  int8_t* xq = reinterpret_cast<int8_t*>(s);
  float* amax = reinterpret_cast<float*>(s + kTail);
  int32_t* row_sum = reinterpret_cast<int32_t*>(s + kTail + 4);
  int32_t* status = reinterpret_cast<int32_t*>(s + kTail + 8);
  cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
  // the quantiser only ever sets the flag, so it starts at zero every call
  BN_CUDA(cudaMemsetAsync(status, 0, sizeof(int32_t), st));
  launch_quantize_rows(x, false, (int)x_len, 1, (int)x_len, xq, (int)ldq, amax, nullptr, row_sum, status, st);
  Segments seg;
  seg.end[0] = seg.end[1] = seg.end[2] = w->rows;
  seg.scale[0] = seg.scale[1] = seg.scale[2] = w->scale;
  launch_ternary_matmul(w->words, w->rows, w->cols, xq, (int)ldq, amax, row_sum, 1, seg, Epi::Store, out, w->rows,
                        nullptr, st);
  BN_CUDA(cudaGetLastError());
  int32_t flag = 0;
  BN_CUDA(cudaMemcpyAsync(&flag, status, sizeof(int32_t), cudaMemcpyDeviceToHost, st));
  BN_CUDA(cudaStreamSynchronize(st));
  if (flag) return quant_error("non-finite activation value");
  return BITNET_OK;
}

}  // extern "C"
