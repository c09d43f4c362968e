// layernorm.cu -- fused residual-add + LayerNorm (HBM-bound).
//
// One row is owned by TPR threads (a warp for d <= 1024, four warps for
// d <= 4096, eight for d <= 8192).  Each thread holds up to 8 float4 chunks
// of the row in registers (chunk i of thread t covers columns
// 4*(i*TPR + t) .. +3, so a warp's loads are 512 contiguous bytes), reduces
// sum and centred sum of squares with shuffles (plus shared memory across
// warps when TPR > 32), and writes the new residual and the normalised row
// with 16-byte (fp32) or 8-byte (16-bit) vector stores.
#include "common.cuh"

namespace tjb {

namespace {

__device__ __forceinline__ float4 load_delta4(const void* delta, int dtype, int64_t idx) {
  if (dtype == TJB_F32) {
    return __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(delta) + idx));
  }
  const uint2 raw = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(delta) + idx));
  float4 r;
  if (dtype == TJB_BF16) {
    const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
    const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
    const float2 a = __bfloat1622float2(lo), b = __bfloat1622float2(hi);
    r = make_float4(a.x, a.y, b.x, b.y);
  } else {
    const __half2 lo = *reinterpret_cast<const __half2*>(&raw.x);
    const __half2 hi = *reinterpret_cast<const __half2*>(&raw.y);
    const float2 a = __half22float2(lo), b = __half22float2(hi);
    r = make_float4(a.x, a.y, b.x, b.y);
  }
  return r;
}

__device__ __forceinline__ void store_out4(void* out, int dtype, int64_t idx, float4 y) {
  if (dtype == TJB_F32) {
    *reinterpret_cast<float4*>(static_cast<float*>(out) + idx) = y;
    return;
  }
  uint2 raw;
  if (dtype == TJB_BF16) {
    raw.x = Pack2<__nv_bfloat16>::pack(y.x, y.y);
    raw.y = Pack2<__nv_bfloat16>::pack(y.z, y.w);
  } else {
    raw.x = Pack2<__half>::pack(y.x, y.y);
    raw.y = Pack2<__half>::pack(y.z, y.w);
  }
  *reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + idx) = raw;
}

// Sum over the TPR threads that own one row.  Every thread of the block must
// call it (it may use __syncthreads).
template <int TPR>
__device__ __forceinline__ float row_sum(float v, float* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if constexpr (TPR <= 32) {
    return v;
  } else {
    constexpr int WPR = TPR / 32;  // warps per row
    const int warp = threadIdx.x >> 5;
    __syncthreads();  // scratch reuse across calls
    if ((threadIdx.x & 31) == 0) scratch[warp] = v;
    __syncthreads();
    const int first = (warp / WPR) * WPR;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < WPR; ++i) s += scratch[first + i];
    return s;
  }
}

constexpr int kBlock = 256;
constexpr int kMaxChunks = 8;
constexpr int kTileRows = 128;  // row-tile granularity of the live-tile list
constexpr int64_t kEarlyWMaxRows = 1024;

// kEarlyW: fetch the LayerNorm weights into registers before the wait for
// the previous kernel (small, latency-bound row counts; at large row counts
// the extra registers cost more occupancy than the latency saved).
template <int TPR, bool kEarlyW>
__global__ void __launch_bounds__(kBlock) add_layernorm_kernel(
    const float* res, const void* __restrict__ delta, float* res_out, void* out,
    const float* __restrict__ w, const float* __restrict__ b, int64_t rows, int d, float eps,
    int delta_dtype, int out_dtype, const uint8_t* __restrict__ row_mask,
    const int32_t* __restrict__ m_tiles) {
  static_assert(TPR == 32 || TPR == 128 || TPR == 256, "threads per row");
  constexpr int kRowsPerBlock = kBlock / TPR;
  __shared__ float scratch[kBlock / 32];
  const int t = threadIdx.x % TPR;
  // The LayerNorm weights are never written during a forward: with kEarlyW
  // this thread's columns are fetched before waiting for the kernel that
  // produces the rows, so their latency overlaps that kernel's tail.
  float4 wv[kEarlyW ? kMaxChunks : 1], bv[kEarlyW ? kMaxChunks : 1];
  if constexpr (kEarlyW) {
#pragma unroll
    for (int i = 0; i < kMaxChunks; ++i) {
      const int col = (i * TPR + t) * 4;
      wv[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      bv[i] = wv[i];
      if (col < d) {
        wv[i] = __ldg(reinterpret_cast<const float4*>(w + col));
        bv[i] = __ldg(reinterpret_cast<const float4*>(b + col));
      }
    }
  }
  griddep_wait();
  griddep_launch_dependents();

  int64_t row = static_cast<int64_t>(blockIdx.x) * kRowsPerBlock + threadIdx.x / TPR;
  if (m_tiles != nullptr) {
    // Blocks walk the listed 128-row tiles only (uniform per block).
    constexpr int kBlocksPerTile = kTileRows / kRowsPerBlock;
    const int li = blockIdx.x / kBlocksPerTile;
    if (li >= __ldg(m_tiles)) return;
    row = static_cast<int64_t>(__ldg(m_tiles + 1 + li)) * kTileRows +
          (blockIdx.x % kBlocksPerTile) * kRowsPerBlock + threadIdx.x / TPR;
  }
  const bool active = row < rows;
  const int64_t base = row * d;

  float4 v[kMaxChunks];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int col = (i * TPR + t) * 4;
    v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (active && col < d) {
      v[i] = __ldg(reinterpret_cast<const float4*>(res + base + col));
      if (delta != nullptr) {
        const float4 dl = load_delta4(delta, delta_dtype, base + col);
        v[i].x += dl.x;
        v[i].y += dl.y;
        v[i].z += dl.z;
        v[i].w += dl.w;
      }
      sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    }
  }
  const float inv_d = 1.0f / static_cast<float>(d);
  const float mean = row_sum<TPR>(sum, scratch) * inv_d;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int col = (i * TPR + t) * 4;
    if (active && col < d) {
      const float a = v[i].x - mean, bb = v[i].y - mean, c = v[i].z - mean, e = v[i].w - mean;
      sq += (a * a + bb * bb) + (c * c + e * e);
    }
  }
  const float var = row_sum<TPR>(sq, scratch) * inv_d;
  const float rstd = rsqrtf(var + eps);
  if (!active) return;
  const bool zero_row = row_mask != nullptr && row_mask[row] == 0;

#pragma unroll
  for (int i = 0; i < kMaxChunks; ++i) {
    const int col = (i * TPR + t) * 4;
    if (col < d) {
      if (res_out != nullptr) *reinterpret_cast<float4*>(res_out + base + col) = v[i];
      float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
      if (!zero_row) {
        float4 ww, bb;
        if constexpr (kEarlyW) {
          ww = wv[i];
          bb = bv[i];
        } else {
          ww = __ldg(reinterpret_cast<const float4*>(w + col));
          bb = __ldg(reinterpret_cast<const float4*>(b + col));
        }
        y.x = (v[i].x - mean) * rstd * ww.x + bb.x;
        y.y = (v[i].y - mean) * rstd * ww.y + bb.y;
        y.z = (v[i].z - mean) * rstd * ww.z + bb.z;
        y.w = (v[i].w - mean) * rstd * ww.w + bb.w;
      }
      store_out4(out, out_dtype, base + col, y);
    }
  }
}

// ------------------------------------------------------------------------
// d <= 1024 over many rows: one warp per row, persistent.  Each warp walks
// rows w, w + W, w + 2W, ... (W = warps in the grid) and issues the loads of
// its next row before it reduces and stores the current one, so DRAM keeps
// reading while the warp computes -- the one-row-per-warp kernel above puts
// every warp of a wave in the same phase (all loading, then all storing).
// kDelta: 0 no delta, 1 fp16, 2 bf16 (fp32 deltas would need 128 more
// bytes of registers per row in flight; they take the kernel above).
constexpr int kRowsMaxChunks = 8;  // 8 x 32 lanes x 4 columns = 1024

template <int kDelta>
struct RowLoad {
  float4 res[kRowsMaxChunks];
  // 16-bit deltas stay packed (8 bytes per chunk) until they are added.
  uint2 dl[kDelta == 0 ? 1 : kRowsMaxChunks];
};

template <int kDelta>
__device__ __forceinline__ void rows_load(RowLoad<kDelta>& L, const float* res, const void* delta,
                                          int64_t row, int64_t rows, int d, int lane) {
  const bool active = row < rows;
  const int64_t base = row * d;
#pragma unroll
  for (int i = 0; i < kRowsMaxChunks; ++i) {
    const int col = (i * 32 + lane) * 4;
    if (active && col < d) {
      L.res[i] = __ldcs(reinterpret_cast<const float4*>(res + base + col));
      if constexpr (kDelta != 0) {
        L.dl[i] = __ldcs(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(delta) + base + col));
      }
    }
  }
}

template <int kDelta>
__device__ __forceinline__ float4 rows_add(const RowLoad<kDelta>& L, int i) {
  float4 v = L.res[i];
  if constexpr (kDelta != 0) {
    float2 a, b;
    if constexpr (kDelta == 2) {
      a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&L.dl[i].x));
      b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&L.dl[i].y));
    } else {
      a = __half22float2(*reinterpret_cast<const __half2*>(&L.dl[i].x));
      b = __half22float2(*reinterpret_cast<const __half2*>(&L.dl[i].y));
    }
    v.x += a.x;
    v.y += a.y;
    v.z += b.x;
    v.w += b.y;
  }
  return v;
}

template <int kDelta>
__device__ __forceinline__ void rows_finish(RowLoad<kDelta>& L, float* res_out, void* out,
                                            const float4* sw, const float4* sb,
                                            const uint8_t* __restrict__ row_mask, int64_t row,
                                            int64_t rows, int d, float eps, int out_dtype,
                                            int lane) {
  if (row >= rows) return;  // warp-uniform
  const int64_t base = row * d;
  // Issued here so that its latency overlaps the reductions below.
  const bool keep = row_mask == nullptr || __ldg(row_mask + row) != 0;
  float4* v = L.res;  // the sum res + delta, in place
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kRowsMaxChunks; ++i) {
    const int col = (i * 32 + lane) * 4;
    if (col < d) {
      v[i] = rows_add(L, i);
      sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float inv_d = 1.0f / static_cast<float>(d);
  const float mean = sum * inv_d;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < kRowsMaxChunks; ++i) {
    const int col = (i * 32 + lane) * 4;
    if (col < d) {
      const float a = v[i].x - mean, bb = v[i].y - mean, c = v[i].z - mean, e = v[i].w - mean;
      sq += (a * a + bb * bb) + (c * c + e * e);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  const float rstd = rsqrtf(sq * inv_d + eps);
#pragma unroll
  for (int i = 0; i < kRowsMaxChunks; ++i) {
    const int col = (i * 32 + lane) * 4;
    if (col < d) {
      if (res_out != nullptr) *reinterpret_cast<float4*>(res_out + base + col) = v[i];
      float4 y = make_float4(0.f, 0.f, 0.f, 0.f);
      if (keep) {
        const float4 ww = sw[i * 32 + lane];
        const float4 bb = sb[i * 32 + lane];
        y.x = (v[i].x - mean) * rstd * ww.x + bb.x;
        y.y = (v[i].y - mean) * rstd * ww.y + bb.y;
        y.z = (v[i].z - mean) * rstd * ww.z + bb.z;
        y.w = (v[i].w - mean) * rstd * ww.w + bb.w;
      }
      store_out4(out, out_dtype, base + col, y);
    }
  }
}

constexpr int kRowsBlock = 256;  // 8 warps

template <int kDelta>
__global__ void __launch_bounds__(kRowsBlock, 2) add_layernorm_rows_kernel(
    const float* res, const void* __restrict__ delta, float* res_out, void* out,
    const float* __restrict__ w, const float* __restrict__ b, int64_t rows, int d, float eps,
    int out_dtype, const uint8_t* __restrict__ row_mask, const int32_t* __restrict__ m_tiles) {
  // The LayerNorm weights are never written during a forward: staged in
  // shared memory before the wait for the kernel that produces the rows.
  __shared__ float4 sw[kRowsMaxChunks * 32], sb[kRowsMaxChunks * 32];
  for (int c = threadIdx.x; c * 4 < d; c += kRowsBlock) {
    sw[c] = __ldg(reinterpret_cast<const float4*>(w) + c);
    sb[c] = __ldg(reinterpret_cast<const float4*>(b) + c);
  }
  __syncthreads();
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  // Row numbers fit 32 bits (the launcher checks rows < 2^31).
  const int stride = static_cast<int>(gridDim.x) * (kRowsBlock / 32);
  int i = static_cast<int>(blockIdx.x) * (kRowsBlock / 32) + (threadIdx.x >> 5);
  // Rows are numbered over the live tiles when there is a list.
  const int n = m_tiles != nullptr ? __ldg(m_tiles) * kTileRows : static_cast<int>(rows);
  auto phys = [&](int v) -> int {
    return m_tiles != nullptr ? __ldg(m_tiles + 1 + v / kTileRows) * kTileRows + v % kTileRows
                              : v;
  };
  RowLoad<kDelta> A, B;
  if (i >= n) return;
  int ra = phys(i);
  rows_load(A, res, delta, ra, rows, d, lane);
  for (;;) {
    int rb = 0;
    if (i + stride < n) {
      rb = phys(i + stride);
      rows_load(B, res, delta, rb, rows, d, lane);
    }
    rows_finish(A, res_out, out, sw, sb, row_mask, ra, rows, d, eps, out_dtype, lane);
    i += stride;
    if (i >= n) return;
    if (i + stride < n) {
      ra = phys(i + stride);
      rows_load(A, res, delta, ra, rows, d, lane);
    }
    rows_finish(B, res_out, out, sw, sb, row_mask, rb, rows, d, eps, out_dtype, lane);
    i += stride;
    if (i >= n) return;
  }
}

}  // namespace
}  // namespace tjb

extern "C" int tjb_add_layernorm_tiles(const float* res, const void* delta, float* res_out,
                                       void* out, const float* w, const float* b, int64_t rows,
                                       int d, float eps, int delta_dtype, int out_dtype,
                                       const uint8_t* row_mask, const int32_t* m_tiles,
                                       tjb_stream_t stream) {
  using namespace tjb;
  if (!res || !out || !w || !b || rows < 0 || d <= 0) return TJB_ERR_INVALID_ARGUMENT;
  if (d % 4 != 0 || d > 8192) return TJB_ERR_BAD_SHAPE;
  if (delta_dtype < TJB_F32 || delta_dtype > TJB_BF16 || out_dtype < TJB_F32 ||
      out_dtype > TJB_BF16)
    return TJB_ERR_UNSUPPORTED_DTYPE;
  if (!aligned16(res) || !aligned16(w) || !aligned16(b) || (res_out && !aligned16(res_out)) ||
      (delta && (reinterpret_cast<uintptr_t>(delta) & 7u)) ||
      (reinterpret_cast<uintptr_t>(out) & 7u))
    return TJB_ERR_BAD_ALIGNMENT;
  if (!device_ok()) return TJB_ERR_NO_DEVICE;
  if (rows == 0) return TJB_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // With a tile list the grid covers every 128-row tile; blocks past the
  // list's count exit at once.
  const int64_t tiles = (rows + kTileRows - 1) / kTileRows;
  // Early weight fetch below this many rows (measured: config 1's 64 rows
  // 3.5% faster forward; 5000-16000 rows 5% slower, from lost occupancy).
  const bool early = rows <= kEarlyWMaxRows;
  auto go = [&](auto kern, int64_t grid) {
    return launch_kernel(kern, dim3(static_cast<unsigned>(grid)), dim3(kBlock), 0, s, res, delta,
                         res_out, out, w, b, rows, d, eps, delta_dtype, out_dtype, row_mask,
                         m_tiles);
  };
  if (d <= 1024 && !early && (delta == nullptr || delta_dtype != TJB_F32) &&
      rows < (int64_t(1) << 31) - kTileRows) {
    // Persistent warp-per-row form: at most two CTAs of eight warps per SM,
    // and never more warps than rows.
    const int64_t max_rows = m_tiles ? tiles * kTileRows : rows;
    const int64_t blocks = (max_rows + kRowsBlock / 32 - 1) / (kRowsBlock / 32);
    const int64_t grid = blocks < 2 * num_sms() ? blocks : 2 * num_sms();
    auto run = [&](auto kern) {
      return launch_kernel(kern, dim3(static_cast<unsigned>(grid)), dim3(kRowsBlock), 0, s, res,
                           delta, res_out, out, w, b, rows, d, eps, out_dtype, row_mask, m_tiles);
    };
    if (delta == nullptr) return run(add_layernorm_rows_kernel<0>);
    if (delta_dtype == TJB_F16) return run(add_layernorm_rows_kernel<1>);
    if (delta_dtype == TJB_BF16) return run(add_layernorm_rows_kernel<2>);
  }
  if (d <= 1024) {
    const int64_t grid = m_tiles ? tiles * (kTileRows / 8) : (rows + 7) / 8;
    return early ? go(add_layernorm_kernel<32, true>, grid) : go(add_layernorm_kernel<32, false>, grid);
  } else if (d <= 4096) {
    const int64_t grid = m_tiles ? tiles * (kTileRows / 2) : (rows + 1) / 2;
    return early ? go(add_layernorm_kernel<128, true>, grid)
                 : go(add_layernorm_kernel<128, false>, grid);
  } else {
    const int64_t grid = m_tiles ? tiles * kTileRows : rows;
    return early ? go(add_layernorm_kernel<256, true>, grid)
                 : go(add_layernorm_kernel<256, false>, grid);
  }
}

extern "C" int tjb_add_layernorm(const float* res, const void* delta, float* res_out, void* out,
                                 const float* w, const float* b, int64_t rows, int d, float eps,
                                 int delta_dtype, int out_dtype, const uint8_t* row_mask,
                                 tjb_stream_t stream) {
  return tjb_add_layernorm_tiles(res, delta, res_out, out, w, b, rows, d, eps, delta_dtype,
                                 out_dtype, row_mask, nullptr, stream);
}
