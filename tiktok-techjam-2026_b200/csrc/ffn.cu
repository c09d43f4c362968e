// ffn.cu -- feed-forward block out = gelu_erf(h W1^T + b1) W2^T + b2.
//
// Two passes of the tcgen05 GEMM: the first applies bias and exact erf-GELU
// in its epilogue and writes the 16-bit hidden activations to the
// caller-provided scratch; the second applies bias and writes the output.
#include <mutex>

#include "common.cuh"

extern "C" int tjb_ffn_tiles(const void* h, const void* w1, const float* b1, const void* w2,
                             const float* b2, void* out, void* hidden, int T, int d, int F,
                             int in_dtype, int out_dtype, const int32_t* m_tiles,
                             tjb_stream_t stream) {
  if (!h || !w1 || !w2 || !out || !hidden || T < 0 || d <= 0 || F <= 0)
    return TJB_ERR_INVALID_ARGUMENT;
  int st = tjb_gemm_bias_tiles(h, w1, b1, hidden, T, F, d, d, d, F, in_dtype, in_dtype, 1,
                               m_tiles, stream);
  if (st != TJB_OK) return st;
  return tjb_gemm_bias_tiles(hidden, w2, b2, out, T, d, F, F, F, d, in_dtype, out_dtype, 0,
                             m_tiles, stream);
}

extern "C" int tjb_ffn_tiles_ws(const void* h, const void* w1, const float* b1, const void* w2,
                                const float* b2, void* out, void* hidden, int T, int d, int F,
                                int in_dtype, int out_dtype, const int32_t* m_tiles,
                                void* workspace, size_t workspace_bytes, tjb_stream_t stream) {
  if (!h || !w1 || !w2 || !out || !hidden || !workspace || T < 0 || d <= 0 || F <= 0)
    return TJB_ERR_INVALID_ARGUMENT;
  int st = tjb_gemm_bias_tiles_ws(h, w1, b1, hidden, T, F, d, d, d, F, in_dtype, in_dtype, 1,
                                  m_tiles, workspace, workspace_bytes, stream);
  if (st != TJB_OK) return st;
  return tjb_gemm_bias_tiles_ws(hidden, w2, b2, out, T, d, F, F, F, d, in_dtype, out_dtype, 0,
                                m_tiles, workspace, workspace_bytes, stream);
}

extern "C" int tjb_ffn(const void* h, const void* w1, const float* b1, const void* w2,
                       const float* b2, void* out, void* hidden, int T, int d, int F,
                       int in_dtype, int out_dtype, tjb_stream_t stream) {
  return tjb_ffn_tiles(h, w1, b1, w2, b2, out, hidden, T, d, F, in_dtype, out_dtype, nullptr,
                       stream);
}

// ------------------------------------------------------------------------
// Allocation-free variant of tjb_ffn.
//
// Some callers cannot allocate device memory at the point they call into
// this library: a host runtime with its own fixed memory pool and no
// allocator hook, a plugin that must not touch the CUDA allocator while it
// runs, or code on a path where an allocation could block or fail.  For them
// tjb_ffn_noalloc keeps the [T, F] hidden activations in a buffer that lives
// inside the library itself: a file-scope device array of
// kNoAllocHiddenElems 16-bit values (16 MiB).  Every GPU that loads the
// library holds that array until the process exits.
//
// In host code the array's name is only a host-side stand-in, never a device
// address, so its device address is looked up once per device with
// cudaGetSymbolAddress (with that device current) and cached.  The first
// call on a device does that look-up, and with CUDA's lazy module loading it
// is also where the library's device code (the array included) gets loaded
// onto that device, which may itself take device memory: make the first call
// at set-up time, before any stream capture.  The cached address belongs to
// the device's current primary context; it does not survive a
// cudaDeviceReset, after which the library must be reloaded (a new process).
// All calls share the one array: the hidden tile is fully written by the
// first GEMM before the second reads it, so nothing needs clearing between
// calls, but calls that overlap on the GPU (different streams, or two
// threads) race on it and must be serialised by the caller.
namespace tjb {
namespace {

constexpr int64_t kNoAllocHiddenElems = int64_t(8) << 20;  // T * F limit
static __device__ __align__(256) uint16_t g_ffn_hidden[kNoAllocHiddenElems];

std::mutex g_hidden_mu;
void* g_hidden_addr[64] = {nullptr};

int hidden_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return TJB_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_hidden_mu);
  if (g_hidden_addr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_ffn_hidden);
    if (e != cudaSuccess) return cuda_status(e);  // recorded for tjb_last_cuda_error
    if (p == nullptr) return TJB_ERR_LAUNCH;
    g_hidden_addr[dev] = p;
  }
  *out = g_hidden_addr[dev];
  return TJB_OK;
}

}  // namespace
}  // namespace tjb

extern "C" int tjb_ffn_noalloc(const void* h, const void* w1, const float* b1, const void* w2,
                               const float* b2, void* out, int T, int d, int F, int in_dtype,
                               int out_dtype, tjb_stream_t stream) {
  if (!h || !w1 || !w2 || !out || T < 0 || d <= 0 || F <= 0) return TJB_ERR_INVALID_ARGUMENT;
  if (static_cast<int64_t>(T) * F > tjb::kNoAllocHiddenElems) return TJB_ERR_BAD_SHAPE;
  if (!tjb::device_ok()) return TJB_ERR_NO_DEVICE;
  void* hidden = nullptr;
  const int st = tjb::hidden_address(&hidden);
  if (st != TJB_OK) return st;
  return tjb_ffn(h, w1, b1, w2, b2, out, hidden, T, d, F, in_dtype, out_dtype, stream);
}
