// ffn.cu -- feed-forward block out = gelu_erf(h W1^T + b1) W2^T + b2.
//
// Two passes of the tcgen05 GEMM: the first applies bias and exact erf-GELU
// in its epilogue and writes the 16-bit hidden activations to the
// caller-provided scratch; the second applies bias and writes the output.
#include "common.cuh"

extern "C" int tjb_ffn(const void* h, const void* w1, const float* b1, const void* w2,
                       const float* b2, void* out, void* hidden, int T, int d, int F,
                       int in_dtype, int out_dtype, tjb_stream_t stream) {
  if (!h || !w1 || !w2 || !out || !hidden || T < 0 || d <= 0 || F <= 0)
    return TJB_ERR_INVALID_ARGUMENT;
  int st = tjb_gemm_bias(h, w1, b1, hidden, T, F, d, d, d, F, in_dtype, in_dtype, 1, stream);
  if (st != TJB_OK) return st;
  return tjb_gemm_bias(hidden, w2, b2, out, T, d, F, F, F, d, in_dtype, out_dtype, 0, stream);
}
