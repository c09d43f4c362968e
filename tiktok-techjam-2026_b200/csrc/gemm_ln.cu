// gemm_ln.cu -- GEMM with the residual add and the following LayerNorm in
// its epilogue (the out-projection and FFN-out of a pre-LN block).
//
//   res_out[M, N] = res_in + A[M, K] * W[N, K]^T + bias
//   out[M, N]     = LayerNorm(res_out) * gamma + beta        (fp32 statistics)
//
// A persistent GEMM over 128 x 256 output tiles, numbered row block by row
// block (tile t = block * C + c, C = N / 256), so the C tiles of a row block
// run on neighbouring CTAs at about the same time.  The producer and MMA
// roles are the plain GEMM's (gemm_produce / gemm_mma), with a 3-stage ring
// to leave shared memory for the epilogue.  The eight epilogue warps (two per
// TMEM lane quarter, 128 columns each) work in 32-row x 32-column chunks of
// fp32: the residual chunk arrives by TMA in a 128-byte-swizzled staging
// buffer (two per warp, the next chunk loading while this one is used), is
// added to bias and accumulator, written back into the accumulator, and each
// row's 128 values are reduced to (mean, M2).  Each warp's 128 columns of
// bias, gamma and beta are staged in shared memory once per tile.  The 2C partials of a row meet
// in a global workspace: every warp publishes its 32 rows' partials and
// counts in on its row block's counter; once all 8C warps of the block have,
// each reads the 2C partials of its rows and combines them (Chan's formula
// for equal parts); the last reader returns the counters to zero.  A second
// pass normalises and sends the residual and the LayerNorm output out of the
// same staging buffers by TMA stores.  The GEMM's delta never reaches HBM and
// the LayerNorm needs no pass of its own.  Waits on partners only ever point
// to tiles of the same or a later round of the persistent loop, so with at
// least C CTAs, all resident, they cannot form a cycle; every wait is bounded.
#include "common.cuh"

namespace tjb {
namespace {

constexpr int kLnMaxC = 4;        // N = 256 .. 1024
constexpr int kLnStages = 3;      // operand ring depth (shared memory for staging)
constexpr uint32_t kLnChunk = 32 * 128;  // 32 rows x 32 fp32 columns, swizzled

struct GemmLnArgs {
  const float* bias;        // [N]
  const float* gamma;       // [N]
  const float* beta;        // [N]
  const uint8_t* row_mask;  // null, or per row: 0 -> output row is zero
  const int32_t* m_tiles;   // null, or the live 128-row tiles (see tjb_row_tiles)
  float2* part;             // [C][2][M] row partials (mean, M2) of each 128 columns
  int* count;               // [2][row blocks] arrivals / readers, zero between calls
  int M, N, K;
  int write_res;
  int out_dtype;
  float eps;
  uint32_t idesc;
};

struct GemmLnSmem {
  static constexpr size_t kRing = static_cast<size_t>(kLnStages) * GemmCfg<256>::kStageBytes;
  static constexpr size_t kStaging = 8 * 2 * kLnChunk;  // [warp][buffer]
  static constexpr size_t kParams = 8 * 3 * 128 * sizeof(float);  // [warp][bias|gamma|beta][128]
  static constexpr size_t kBytes = 1024 + kRing + kStaging + kParams + 512;
};

__device__ __forceinline__ void ld_chunk_row(const uint8_t* buf, int r, float (&v)[32]) {
  const uint4* row = reinterpret_cast<const uint4*>(buf + r * 128);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint4 q = row[k ^ (r & 7)];
    v[4 * k] = __uint_as_float(q.x);
    v[4 * k + 1] = __uint_as_float(q.y);
    v[4 * k + 2] = __uint_as_float(q.z);
    v[4 * k + 3] = __uint_as_float(q.w);
  }
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_ln_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmRin,
                   const __grid_constant__ CUtensorMap tmRout,
                   const __grid_constant__ CUtensorMap tmOut, const GemmLnArgs args) {
  using Cfg = GemmCfg<256>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kLnStages * Cfg::kABytes;
  uint8_t* staging = smem + GemmLnSmem::kRing;  // [warp 0..7][2][kLnChunk]
  float* params = reinterpret_cast<float*>(staging + GemmLnSmem::kStaging);
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(params) +
                                               GemmLnSmem::kParams);
  uint64_t* empty = full + kLnStages;
  uint64_t* tfull = empty + kLnStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* rbar = drain + 1;  // [warp][buffer]: residual chunk landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 16);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int C = args.N / 256;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kLnStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
    }
    for (int i = 0; i < 16; ++i) mbar_init(&rbar[i], 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmRin);
    prefetch_tmap(&tmRout);
    prefetch_tmap(&tmOut);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  // The first k-blocks of this CTA's first W tile into L2 before the wait
  // (weights are never written by the kernels this launch overlaps).
  if (warp == 0 && lane == 0)
    for (int kb = 0; kb < kLnStages && kb * kBK < args.K; ++kb)
      tma_prefetch_2d(&tmB, kb * kBK, (static_cast<int>(blockIdx.x) % C) * 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();
  griddep_launch_dependents();
  const int num_m = args.m_tiles != nullptr ? __ldg(args.m_tiles) : (args.M + kBM - 1) / kBM;
  const int num_tiles = num_m * C;
  const int num_k = (args.K + kBK - 1) / kBK;
  auto tiles = [&]() {
    int t = static_cast<int>(blockIdx.x);
    const int stride = static_cast<int>(gridDim.x);
    return [=](GemmPiece& un) mutable {
      if (t >= num_tiles) return false;
      un.tile = t;
      un.kb0 = 0;
      un.kb1 = num_k;
      t += stride;
      return true;
    };
  };
  auto m_block = [&](int blk) {
    return args.m_tiles != nullptr ? __ldg(args.m_tiles + 1 + blk) : blk;
  };

  if (warp == 0) {
    if (lane == 0)
      gemm_produce<256, kLnStages>(tiles(),
                                   [&](int tile, int& m_blk, int& n_blk) {
                                     m_blk = m_block(tile / C);
                                     n_blk = tile - (tile / C) * C;
                                   },
                                   &tmA, &tmB, sA, sB, full, empty, abort_flag);
  } else if (warp == 1) {
    gemm_mma<256, kLnStages>(tiles(), tmem_base, sA, sB, full, empty, tfull, tempty, drain,
                             args.idesc, abort_flag);
  } else {
    // -------------------------------------------------------------- epilogue
    const int ew = warp - 2;           // epilogue warp 0..7
    const int quad = warp & 3;         // TMEM lanes this warp may access
    const int half = (warp - 2) >> 2;  // which 128 of the tile's 256 columns
    uint8_t* const buf0 = staging + ew * 2 * kLnChunk;
    // This warp's 128 columns of bias, gamma and beta, staged once per tile
    // (every lane reads every column: shared-memory broadcasts).
    float* const prm = params + ew * 3 * 128;
    auto buf = [&](int b) { return buf0 + b * kLnChunk; };
    auto bar = [&](int b) { return &rbar[ew * 2 + b]; };
    uint32_t bar_phase = 0;  // bit b: parity of buffer b's next load
    uint32_t pending = 0;    // bit b: a load into buffer b not yet waited for
    const float inv_n = 1.0f / static_cast<float>(args.N);
    const int out_cols = args.out_dtype == TJB_F32 ? 32 : 64;  // one staged store's columns
    int acc = 0;
    uint32_t acc_phase = 0;
    auto next = tiles();
    GemmPiece un;
    // Loads the residual chunk c (32 columns) of this warp's rows into buffer b.
    auto load_res = [&](int b, int col, int row0) {
      pending |= 1u << b;
      if (lane == 0) {
        mbar_arrive_expect_tx(bar(b), kLnChunk);
        tma_load_2d(buf(b), &tmRin, bar(b), col, row0);
      }
    };
    auto wait_res = [&](int b) {
      const bool ok =
          __all_sync(0xffffffffu, mbar_wait(bar(b), (bar_phase >> b) & 1u, abort_flag));
      if (ok) {
        bar_phase ^= 1u << b;
        pending &= ~(1u << b);
      }
      return ok;
    };
    bool ok = true;
    while (ok && next(un)) {
      const int blk = un.tile / C;
      const int ncol = un.tile - blk * C;
      const int row0 = m_block(blk) * kBM + quad * 32;
      const int64_t row = static_cast<int64_t>(row0) + lane;
      const bool valid = row < args.M;
      const int col0 = ncol * 256 + half * 128;
      // Both staging buffers are free once their last TMA stores have read
      // them (the previous tile's pass 2).
      if (lane == 0) bulk_wait_read<0>();
      __syncwarp();
      load_res(0, col0, row0);
      // Column parameters and the row mask: loads issued before the wait
      // for the accumulator so that their latency hides behind it.
      float4 pv[3];
#pragma unroll
      for (int k = 0; k < 3; ++k) {
        const float* src = k == 0 ? args.bias : k == 1 ? args.gamma : args.beta;
        pv[k] = __ldg(reinterpret_cast<const float4*>(src + col0) + lane);
      }
      const bool zero_row = args.row_mask != nullptr && valid && args.row_mask[row] == 0;
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, abort_flag))) break;
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < 3; ++k) reinterpret_cast<float4*>(prm + k * 128)[lane] = pv[k];
      __syncwarp();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(acc * 256 + half * 128);
      // Pass 1: v = acc + bias + residual, back into the accumulator; this
      // row's mean and sum of squared deviations over its 128 columns.
      float mean = 0.f, m2 = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        if (c + 1 < 4) load_res((c + 1) & 1, col0 + (c + 1) * 32, row0);
        uint32_t r[32];
        tmem_ld32(taddr + c * 32, r);
        tmem_ld_wait(r);
        if (!wait_res(c & 1)) {
          ok = false;
          break;
        }
        float x[32];
        ld_chunk_row(buf(c & 1), lane, x);
        __syncwarp();  // every lane has read the buffer before it is refilled
        const float4* b4 = reinterpret_cast<const float4*>(prm + c * 32);
        float v[32];
        float sum = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 bb = b4[i];
          v[4 * i] = __uint_as_float(r[4 * i]) + bb.x + x[4 * i];
          v[4 * i + 1] = __uint_as_float(r[4 * i + 1]) + bb.y + x[4 * i + 1];
          v[4 * i + 2] = __uint_as_float(r[4 * i + 2]) + bb.z + x[4 * i + 2];
          v[4 * i + 3] = __uint_as_float(r[4 * i + 3]) + bb.w + x[4 * i + 3];
          sum += (v[4 * i] + v[4 * i + 1]) + (v[4 * i + 2] + v[4 * i + 3]);
        }
        const float cm = sum * (1.0f / 32.0f);
        float cm2 = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float e = v[i] - cm;
          cm2 = fmaf(e, e, cm2);
          r[i] = __float_as_uint(v[i]);
        }
        // Chan's combination of (32c values, mean, m2) with (32, cm, cm2).
        const float nw = 1.0f / static_cast<float>(c + 1);
        const float dlt = cm - mean;
        mean += dlt * nw;
        m2 += cm2 + dlt * dlt * (32.0f * static_cast<float>(c) * nw);
        tmem_st32(taddr + c * 32, r);
      }
      if (!ok) break;
      tmem_st_wait();
      // Publish this row's partial; count in; wait for the row block's 8C
      // warps; combine the block's 2C partials of this row.
      if (valid) args.part[(static_cast<int64_t>(ncol) * 2 + half) * args.M + row] =
          make_float2(mean, m2);
      __threadfence();
      __syncwarp();
      int* arrived = args.count + blk;
      int* readers = args.count + num_m + blk;
      if (lane == 0) atomicAdd(arrived, 1);
      if (lane == 0) ok = wait_count(arrived, 8 * C, abort_flag);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      float mu = 0.f, m2sum = 0.f;
      float pm[2 * kLnMaxC];
#pragma unroll
      for (int k = 0; k < 2 * kLnMaxC; ++k) {
        pm[k] = 0.f;
        if (k < 2 * C && valid) {
          const float2 p = __ldcg(args.part + static_cast<int64_t>(k) * args.M + row);
          pm[k] = p.x;
          mu += p.x;
          m2sum += p.y;
        }
      }
      mu *= 1.0f / static_cast<float>(2 * C);
#pragma unroll
      for (int k = 0; k < 2 * kLnMaxC; ++k) {
        if (k < 2 * C) {
          const float e = pm[k] - mu;
          m2sum = fmaf(128.0f * e, e, m2sum);
        }
      }
      const float rstd = rsqrtf(m2sum * inv_n + args.eps);
      __syncwarp();
      // The last of the block's 8C warps to have read returns both counters.
      if (lane == 0 && atomicAdd(readers, 1) == 8 * C - 1) {
        atomicExch(arrived, 0);
        atomicExch(readers, 0);
      }
      // Pass 2: normalise; stage and store the residual and the output.
      int sb = 0;  // staging buffer for the next store
#pragma unroll 1
      for (int c = 0; c < 4; c += out_cols / 32) {
        uint32_t w[32];
        for (int cc = 0; cc < out_cols / 32; ++cc) {
          uint32_t r[32];
          tmem_ld32(taddr + (c + cc) * 32, r);
          tmem_ld_wait(r);
          const int col = col0 + (c + cc) * 32;
          if (args.write_res) {
            if (lane == 0) bulk_wait_read<1>();  // this buffer's previous store has read it
            __syncwarp();
            stage_row(buf(sb), lane, r);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmRout, buf(sb), col, row0);
              bulk_commit();
            }
            sb ^= 1;
          }
          const float4* g4 = reinterpret_cast<const float4*>(prm + 128 + (c + cc) * 32);
          const float4* e4 = reinterpret_cast<const float4*>(prm + 256 + (c + cc) * 32);
          float y[32];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 gg = g4[i];
            const float4 bb = e4[i];
            y[4 * i] = (__uint_as_float(r[4 * i]) - mu) * rstd * gg.x + bb.x;
            y[4 * i + 1] = (__uint_as_float(r[4 * i + 1]) - mu) * rstd * gg.y + bb.y;
            y[4 * i + 2] = (__uint_as_float(r[4 * i + 2]) - mu) * rstd * gg.z + bb.z;
            y[4 * i + 3] = (__uint_as_float(r[4 * i + 3]) - mu) * rstd * gg.w + bb.w;
          }
          if (zero_row) {
#pragma unroll
            for (int i = 0; i < 32; ++i) y[i] = 0.f;
          }
          if (args.out_dtype == TJB_F32) {
#pragma unroll
            for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(y[i]);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              w[cc * 16 + i] = args.out_dtype == TJB_BF16
                                   ? Pack2<__nv_bfloat16>::pack(y[2 * i], y[2 * i + 1])
                                   : Pack2<__half>::pack(y[2 * i], y[2 * i + 1]);
          }
        }
        if (lane == 0) bulk_wait_read<1>();
        __syncwarp();
        stage_row(buf(sb), lane, w);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmOut, buf(sb), col0 + c * 32, row0);
          bulk_commit();
        }
        sb ^= 1;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    // Every bulk store has completed before the CTA exits.
    if (lane == 0) bulk_wait_all();
    __syncwarp();
    // Drain residual loads still in flight after an abort.
    for (int b = 0; b < 2; ++b)
      if (pending & (1u << b)) mbar_wait_drain(bar(b), (bar_phase >> b) & 1u);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

std::mutex g_ln_attr_mu;
bool g_ln_attr_done[64];

// Workspace layout: [2][row blocks] int counters (zero between calls), padded
// to 256 bytes, then the [C][2][M] float2 row partials.
size_t ln_count_bytes(int M) {
  const size_t blocks = static_cast<size_t>((M + kBM - 1) / kBM);
  return (2 * blocks * sizeof(int) + 255) / 256 * 256;
}

}  // namespace
}  // namespace tjb

extern "C" size_t tjb_gemm_add_layernorm_workspace_bytes(int M, int N) {
  using namespace tjb;
  if (M <= 0 || N <= 0) return 256;
  const size_t C = static_cast<size_t>((N + 255) / 256);
  return ln_count_bytes(M) + C * 2 * static_cast<size_t>(M) * sizeof(float2);
}

extern "C" int tjb_gemm_add_layernorm(const void* A, const void* W, const float* bias,
                                      const float* res_in, float* res_out, const float* gamma,
                                      const float* beta, void* out, int M, int N, int K,
                                      float eps, int in_dtype, int out_dtype,
                                      const uint8_t* row_mask, const int32_t* m_tiles,
                                      void* workspace, size_t workspace_bytes,
                                      tjb_stream_t stream) {
  using namespace tjb;
  if (!A || !W || !bias || !res_in || !gamma || !beta || !out || !workspace || M < 0 ||
      N <= 0 || K <= 0)
    return TJB_ERR_INVALID_ARGUMENT;
  if (in_dtype != TJB_F16 && in_dtype != TJB_BF16) return TJB_ERR_UNSUPPORTED_DTYPE;
  if (out_dtype != TJB_F32 && out_dtype != TJB_F16 && out_dtype != TJB_BF16)
    return TJB_ERR_UNSUPPORTED_DTYPE;
  const int C = N / 256;
  if (N % 256 != 0 || C > kLnMaxC || K % 8 != 0) return TJB_ERR_BAD_SHAPE;
  if (workspace_bytes < tjb_gemm_add_layernorm_workspace_bytes(M, N))
    return TJB_ERR_INVALID_ARGUMENT;
  if (!aligned16(A) || !aligned16(W) || !aligned16(bias) || !aligned16(res_in) ||
      (res_out && !aligned16(res_out)) || !aligned16(gamma) || !aligned16(beta) ||
      !aligned16(out) || !aligned16(workspace))
    return TJB_ERR_BAD_ALIGNMENT;
  if (!device_ok()) return TJB_ERR_NO_DEVICE;
  if (M == 0) return TJB_OK;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(g_ln_attr_mu);
    if (dev < 64 && !g_ln_attr_done[dev]) {
      if (const int fs = cuda_status(cudaFuncSetAttribute(
              gemm_ln_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
              static_cast<int>(GemmLnSmem::kBytes))))
        return fs;
      g_ln_attr_done[dev] = true;
    }
  }
  const bool bf16 = in_dtype == TJB_BF16;
  CUtensorMap tmA, tmB, tmRin, tmRout, tmOut;
  const uint64_t dimA[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
  const uint64_t strA[1] = {static_cast<uint64_t>(K) * 2};
  const uint32_t boxA[2] = {kBK, kBM};
  const uint64_t dimB[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
  const uint32_t boxB[2] = {kBK, 256};
  int st = make_tmap_16bit(&tmA, 2, A, dimA, strA, boxA, bf16);
  if (st != TJB_OK) return st;
  st = make_tmap_16bit(&tmB, 2, W, dimB, strA, boxB, bf16);
  if (st != TJB_OK) return st;
  const uint64_t n64 = static_cast<uint64_t>(N), m64 = static_cast<uint64_t>(M);
  st = make_tmap_2d(&tmRin, TJB_F32, res_in, n64, m64, n64 * 4, 32, 32);
  if (st != TJB_OK) return st;
  st = make_tmap_2d(&tmRout, TJB_F32, res_out ? res_out : res_in, n64, m64, n64 * 4, 32, 32);
  if (st != TJB_OK) return st;
  const uint64_t esz = out_dtype == TJB_F32 ? 4 : 2;
  st = make_tmap_2d(&tmOut, out_dtype, out, n64, m64, n64 * esz, static_cast<uint32_t>(128 / esz),
                    32);
  if (st != TJB_OK) return st;
  GemmLnArgs a;
  a.bias = bias;
  a.gamma = gamma;
  a.beta = beta;
  a.row_mask = row_mask;
  a.m_tiles = m_tiles;
  a.count = static_cast<int*>(workspace);
  a.part = reinterpret_cast<float2*>(static_cast<uint8_t*>(workspace) + ln_count_bytes(M));
  a.M = M;
  a.N = N;
  a.K = K;
  a.write_res = res_out != nullptr;
  a.eps = eps;
  a.out_dtype = out_dtype;
  a.idesc = idesc_f16(kBM, 256, bf16, false);
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = GemmLnSmem::kBytes;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  // Persistent: one CTA per SM (at least C of them, so that the C tiles of
  // any row block are always resident together), never more than the tiles.
  const int tiles = (M + kBM - 1) / kBM * C;
  cfg.gridDim = dim3(std::min(num_sms(), tiles));
  return cuda_status(cudaLaunchKernelEx(&cfg, gemm_ln_kernel, tmA, tmB, tmRin, tmRout, tmOut, a));
}
