// runtime.cu -- host-side runtime of libtjb200: status strings, the device
// status word, SM-count cache, tensor-map encoding through the driver entry
// point (no link-time dependency on libcuda), and two small device kernels:
// padding-mask classification and the bounded-wait self-test.
#include <cstdlib>
#include <mutex>

#include "common.cuh"

namespace tjb {

namespace {

constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};
int g_cc_major[kMaxDevices] = {0};
std::mutex g_dev_mu;

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
std::once_flag g_encode_once;

void load_encode() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
          cudaSuccess &&
      q == cudaDriverEntryPointSuccess) {
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  }
}

int current_device_cached() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
  std::lock_guard<std::mutex> lock(g_dev_mu);
  if (g_sm_count[dev] == 0) {
    int sms = 0, major = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    g_sm_count[dev] = sms > 0 ? sms : 1;
    g_cc_major[dev] = major;
  }
  return dev;
}

}  // namespace

int num_sms() {
  int dev = current_device_cached();
  return dev < 0 ? 1 : g_sm_count[dev];
}

bool device_ok() {
  int dev = current_device_cached();
  return dev >= 0 && g_cc_major[dev] == 10;
}

int make_tmap_16bit(CUtensorMap* map, int rank, const void* base, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box, bool bf16) {
  std::call_once(g_encode_once, load_encode);
  if (g_encode == nullptr) return TJB_ERR_TENSOR_MAP;
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
    if (i > 0) gstride[i - 1] = strides_bytes[i - 1];
  }
  CUresult r = g_encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        static_cast<cuuint32_t>(rank), const_cast<void*>(base), gdim, gstride,
                        bdim, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TJB_OK : TJB_ERR_TENSOR_MAP;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("TJB_NO_PDL");
    return !(e != nullptr && e[0] == '1');
  }();
  return on;
}

int make_tmap_2d(CUtensorMap* map, int dtype, const void* base, uint64_t cols, uint64_t rows,
                 uint64_t ld_bytes, uint32_t box_cols, uint32_t box_rows) {
  std::call_once(g_encode_once, load_encode);
  if (g_encode == nullptr) return TJB_ERR_TENSOR_MAP;
  const CUtensorMapDataType dt = dtype == TJB_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == TJB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t gdim[2] = {cols, rows};
  cuuint64_t gstride[1] = {ld_bytes};
  cuuint32_t bdim[2] = {box_cols, box_rows};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = g_encode(map, dt, 2, const_cast<void*>(base), gdim, gstride, bdim, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? TJB_OK : TJB_ERR_TENSOR_MAP;
}

// ------------------------------------------------------------ mask lengths
// One CTA walks every row: lengths[b] = popcount of row b; a row is a prefix
// mask iff it has no 0 -> 1 step.
__global__ void __launch_bounds__(1024) mask_lengths_kernel(const uint8_t* __restrict__ mask,
                                                            int B, int S,
                                                            int32_t* __restrict__ lengths,
                                                            int32_t* __restrict__ flags) {
  __shared__ int s_count[32];
  __shared__ int s_step[32];
  griddep_wait();
  griddep_launch_dependents();
  int any_step = 0;
  for (int b = 0; b < B; ++b) {
    const uint8_t* row = mask + static_cast<int64_t>(b) * S;
    int count = 0, step = 0;
    for (int j = threadIdx.x; j < S; j += blockDim.x) {
      const int v = row[j] != 0;
      count += v;
      if (j > 0 && v && row[j - 1] == 0) step = 1;
    }
    for (int o = 16; o > 0; o >>= 1) {
      count += __shfl_xor_sync(0xffffffffu, count, o);
      step |= __shfl_xor_sync(0xffffffffu, step, o);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
      s_count[warp] = count;
      s_step[warp] = step;
    }
    __syncthreads();
    if (warp == 0) {
      const int nw = (blockDim.x + 31) >> 5;
      count = lane < nw ? s_count[lane] : 0;
      step = lane < nw ? s_step[lane] : 0;
      for (int o = 16; o > 0; o >>= 1) {
        count += __shfl_xor_sync(0xffffffffu, count, o);
        step |= __shfl_xor_sync(0xffffffffu, step, o);
      }
      if (lane == 0) {
        lengths[b] = count;
        any_step |= step;
      }
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) *flags = any_step ? TJB_ERR_NON_PREFIX_MASK : 0;
}

// --------------------------------------------------------------- row tiles
// Live 128-row tiles of the flattened [B*S] token axis.  A tile is live when
// it holds a row (b, s) with s < round_up(lengths[b], 128): every valid row,
// plus the padded rows that share the valid rows' last 128-key attention
// tile (attention reads those keys, masked, so they must stay finite).  With
// a non-prefix mask (flags != 0) or no lengths every tile is live.
// tiles[0] = count, tiles[1..] = tile indices in increasing order.
__global__ void __launch_bounds__(1024) row_tiles_kernel(const int32_t* __restrict__ lengths,
                                                         const int32_t* __restrict__ flags,
                                                         int B, int S, int32_t* __restrict__ tiles) {
  __shared__ int s_warp[32];
  __shared__ int s_base;
  griddep_wait();
  griddep_launch_dependents();
  const int64_t T = static_cast<int64_t>(B) * S;
  const int n_tiles = static_cast<int>((T + 127) / 128);
  const bool all = lengths == nullptr || (flags != nullptr && __ldg(flags) != 0);
  if (threadIdx.x == 0) s_base = 0;
  __syncthreads();
  for (int t0 = 0; t0 < n_tiles; t0 += blockDim.x) {
    const int t = t0 + threadIdx.x;
    int live = 0;
    if (t < n_tiles) {
      if (all) {
        live = 1;
      } else {
        const int64_t r0 = static_cast<int64_t>(t) * 128;
        const int64_t r1 = min(r0 + 128, T);
        for (int64_t b = r0 / S; b * S < r1 && !live; ++b) {
          const int64_t first = max(r0, b * S) - b * S;  // first row of b inside the tile
          const int len = min(max(__ldg(lengths + b), 0), S);
          const int64_t reach = (static_cast<int64_t>(len) + 127) / 128 * 128;
          if (first < reach) live = 1;
        }
      }
    }
    // Block-wide exclusive scan of the live flags.
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned ballot = __ballot_sync(0xffffffffu, live);
    const int in_warp = __popc(ballot & ((1u << lane) - 1u));
    if (lane == 0) s_warp[warp] = __popc(ballot);
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < (blockDim.x >> 5); ++w) {
      if (w < warp) before += s_warp[w];
      total += s_warp[w];
    }
    if (live) tiles[1 + s_base + before + in_warp] = t;
    __syncthreads();
    if (threadIdx.x == 0) s_base += total;
    __syncthreads();
  }
  if (threadIdx.x == 0) tiles[0] = s_base;
}

// ------------------------------------------- mask lengths + tiles, one pass
// One CTA, one warp per row at a time (all rows in flight together, instead
// of one row after another): each lane reads 16 mask bytes per step, counts
// the non-zero ones and looks for a 0 -> 1 rise inside them and across the
// boundary with the previous lane's last byte; then, in the same launch,
// the live 128-row tiles are listed from the lengths just written (global
// writes of the CTA are visible to all its threads after __syncthreads).
__device__ __forceinline__ uint32_t nonzero_bytes(uint32_t w) {
  // 0x01 in each byte of w that is non-zero.
  return ((((w & 0x7F7F7F7Fu) + 0x7F7F7F7Fu) | w) >> 7) & 0x01010101u;
}

__global__ void __launch_bounds__(1024) mask_tiles_kernel(const uint8_t* __restrict__ mask,
                                                          int B, int S,
                                                          int32_t* lengths,
                                                          int32_t* __restrict__ flags,
                                                          int32_t* __restrict__ tiles) {
  __shared__ int s_step;
  __shared__ int s_warp[32];
  __shared__ int s_base;
  griddep_wait();
  griddep_launch_dependents();
  if (threadIdx.x == 0) {
    s_step = 0;
    s_base = 0;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = static_cast<int>(blockDim.x >> 5);
  const bool vec = (S % 16) == 0 && (reinterpret_cast<uintptr_t>(mask) & 15u) == 0;
  for (int b = warp; b < B; b += nwarps) {
    const uint8_t* row = mask + static_cast<int64_t>(b) * S;
    int count = 0, step = 0;
    if (vec) {
      uint32_t carry = 1;  // "the byte before is non-zero": no rise at column 0
      for (int j0 = 0; j0 < S; j0 += 32 * 16) {
        const int j = j0 + lane * 16;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (j < S) v = __ldg(reinterpret_cast<const uint4*>(row + j));
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t nz[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) nz[i] = nonzero_bytes(w[i]);
        // The byte before this lane's first byte: the previous lane's last.
        const uint32_t last = (nz[3] >> 24) & 1u;
        uint32_t prev = __shfl_up_sync(0xffffffffu, last, 1);
        if (lane == 0) prev = carry;
        carry = __shfl_sync(0xffffffffu, last, 31);
        if (j < S) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            count += __popc(nz[i]);
            // Byte k of the word rises when it is non-zero and byte k - 1 (or
            // the carried byte for k = 0) is zero.
            const uint32_t before = (nz[i] << 8) | prev;
            step |= (nz[i] & ~before) != 0u;
            prev = nz[i] >> 24;
          }
        }
      }
    } else {
      for (int j = lane; j < S; j += 32) {
        const int v = row[j] != 0;
        count += v;
        if (j > 0 && v && row[j - 1] == 0) step = 1;
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      count += __shfl_xor_sync(0xffffffffu, count, o);
      step |= __shfl_xor_sync(0xffffffffu, step, o);
    }
    if (lane == 0) {
      lengths[b] = count;
      if (step) s_step = 1;
    }
  }
  __syncthreads();
  const int any_step = s_step;
  if (threadIdx.x == 0) *flags = any_step ? TJB_ERR_NON_PREFIX_MASK : 0;
  if (tiles == nullptr) return;  // uniform
  // Live tiles, exactly as row_tiles_kernel lists them.
  const int64_t T = static_cast<int64_t>(B) * S;
  const int n_tiles = static_cast<int>((T + 127) / 128);
  for (int t0 = 0; t0 < n_tiles; t0 += blockDim.x) {
    const int t = t0 + threadIdx.x;
    int live = 0;
    if (t < n_tiles) {
      if (any_step) {
        live = 1;
      } else {
        const int64_t r0 = static_cast<int64_t>(t) * 128;
        const int64_t r1 = min(r0 + 128, T);
        for (int64_t bb = r0 / S; bb * S < r1 && !live; ++bb) {
          const int64_t first = max(r0, bb * S) - bb * S;
          const int len = min(max(lengths[bb], 0), S);
          const int64_t reach = (static_cast<int64_t>(len) + 127) / 128 * 128;
          if (first < reach) live = 1;
        }
      }
    }
    const unsigned ballot = __ballot_sync(0xffffffffu, live);
    const int in_warp = __popc(ballot & ((1u << lane) - 1u));
    if (lane == 0) s_warp[warp] = __popc(ballot);
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < nwarps; ++w) {
      if (w < warp) before += s_warp[w];
      total += s_warp[w];
    }
    if (live) tiles[1 + s_base + before + in_warp] = t;
    __syncthreads();
    if (threadIdx.x == 0) s_base += total;
    __syncthreads();
  }
  if (threadIdx.x == 0) tiles[0] = s_base;
}

// --------------------------------------------------------- bounded-wait test
__global__ void selftest_wait_kernel(const int32_t* flag, int64_t timeout_ns) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const volatile int32_t* f = flag;
  const uint64_t t0 = globaltimer();
  while (*f == 0) {
    if (globaltimer() - t0 > static_cast<uint64_t>(timeout_ns)) {
      record_status(TJB_ERR_DEVICE_TIMEOUT);
      return;
    }
    __nanosleep(1000);
  }
}

}  // namespace tjb

// ==================================================================== C ABI
extern "C" {

int tjb_version(void) { return 100; }

const char* tjb_status_string(int status) {
  switch (status) {
    case TJB_OK: return "ok";
    case TJB_ERR_INVALID_ARGUMENT: return "invalid argument";
    case TJB_ERR_BAD_SHAPE: return "shape outside the kernel contract";
    case TJB_ERR_BAD_ALIGNMENT: return "pointer or pitch not 16-byte aligned";
    case TJB_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype";
    case TJB_ERR_LAUNCH: return "CUDA launch error";
    case TJB_ERR_TENSOR_MAP: return "tensor map encoding failed";
    case TJB_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case TJB_ERR_NO_DEVICE: return "no sm_100 device is current";
    case TJB_ERR_NON_PREFIX_MASK: return "padding mask is not a prefix mask";
    default: return "unknown status";
  }
}

const char* tjb_last_cuda_error(void) {
  return cudaGetErrorString(tjb::last_cuda_error());
}

int tjb_device_status(int clear) {
  if (cudaDeviceSynchronize() != cudaSuccess) return TJB_ERR_LAUNCH;
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, tjb::g_device_status, sizeof(int)) != cudaSuccess)
    return TJB_ERR_LAUNCH;
  if (clear) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(tjb::g_device_status, &zero, sizeof(int)) != cudaSuccess)
      return TJB_ERR_LAUNCH;
  }
  return v;
}

int tjb_device_status_async(int32_t* host_dst, tjb_stream_t stream) {
  if (!host_dst || (reinterpret_cast<uintptr_t>(host_dst) & 3u) != 0)
    return TJB_ERR_INVALID_ARGUMENT;
  if (!tjb::device_ok()) return TJB_ERR_NO_DEVICE;
  // A copy-engine read of the word, ordered after every kernel already on
  // the stream; nothing is launched and nothing waits on the host.
  return tjb::cuda_status(cudaMemcpyFromSymbolAsync(host_dst, tjb::g_device_status,
                                                    sizeof(int32_t), 0,
                                                    cudaMemcpyDeviceToHost,
                                                    reinterpret_cast<cudaStream_t>(stream)));
}

int tjb_mask_lengths(const uint8_t* mask, int B, int S, int32_t* lengths, int32_t* flags,
                     tjb_stream_t stream) {
  if (!mask || !lengths || !flags || B <= 0 || S <= 0) return TJB_ERR_INVALID_ARGUMENT;
  if (!tjb::device_ok()) return TJB_ERR_NO_DEVICE;
  return tjb::launch_kernel(tjb::mask_lengths_kernel, dim3(1), dim3(1024), 0,
                         reinterpret_cast<cudaStream_t>(stream), mask, B, S, lengths, flags);
}

int tjb_mask_lengths_tiles(const uint8_t* mask, int B, int S, int32_t* lengths, int32_t* flags,
                           int32_t* tiles, tjb_stream_t stream) {
  if (!mask || !lengths || !flags || B <= 0 || S <= 0) return TJB_ERR_INVALID_ARGUMENT;
  if (!tjb::device_ok()) return TJB_ERR_NO_DEVICE;
  return tjb::launch_kernel(tjb::mask_tiles_kernel, dim3(1), dim3(1024), 0,
                            reinterpret_cast<cudaStream_t>(stream), mask, B, S, lengths, flags,
                            tiles);
}

int tjb_row_tiles(const int32_t* lengths, const int32_t* flags, int B, int S, int32_t* tiles,
                  tjb_stream_t stream) {
  if (!tiles || B <= 0 || S <= 0) return TJB_ERR_INVALID_ARGUMENT;
  if (!tjb::device_ok()) return TJB_ERR_NO_DEVICE;
  return tjb::launch_kernel(tjb::row_tiles_kernel, dim3(1), dim3(1024), 0,
                         reinterpret_cast<cudaStream_t>(stream), lengths, flags, B, S, tiles);
}

int tjb_selftest_wait(const int32_t* flag, int64_t timeout_ns, tjb_stream_t stream) {
  if (!flag || timeout_ns <= 0) return TJB_ERR_INVALID_ARGUMENT;
  if (!tjb::device_ok()) return TJB_ERR_NO_DEVICE;
  tjb::selftest_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(flag,
                                                                                  timeout_ns);
  return tjb::launch_status();
}

}  // extern "C"
