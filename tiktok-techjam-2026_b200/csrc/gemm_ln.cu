// gemm_ln.cu -- GEMM with the residual add and the following LayerNorm in
// its epilogue (the out-projection and FFN-out of a pre-LN block).
//
//   res_out[M, N] = res_in + A[M, K] * W[N, K]^T + bias
//   out[M, N]     = LayerNorm(res_out) * gamma + beta        (fp32 statistics)
//
// N = d_model is covered by a cluster of C = N / 256 CTAs, CTA c owning the
// 128 x 256 output tile of columns [256c, 256c + 256) of one 128-row block;
// each cluster walks row blocks persistently.  The producer and MMA roles are
// the plain GEMM's (gemm_produce / gemm_mma).  The eight epilogue warps
// (two per TMEM lane quarter, 128 columns each) add bias and residual, write
// the sums back into the accumulator, and reduce their row's 128 values to a
// (mean, M2) pair; the pairs of all 2C warps that share a row meet in
// distributed shared memory (each CTA publishes its own, then every CTA
// reads the cluster's), combined with Chan's formula for equal-size parts;
// a second pass normalises and writes the residual and the LayerNorm output.
// The GEMM's delta never reaches HBM and the LayerNorm needs no pass of its
// own.  Publication uses a double-buffered statistics array with two
// cluster-scope mbarriers per buffer (ready: every warp of the cluster wrote;
// free: every warp read), all waits bounded.
#include "common.cuh"

namespace tjb {
namespace {

constexpr int kLnMaxCluster = 4;  // N = 256 .. 1024

struct GemmLnArgs {
  const float* bias;        // [N]
  const float* gamma;       // [N]
  const float* beta;        // [N]
  const float* res_in;      // [M, N] fp32
  float* res_out;           // [M, N] fp32 (may equal res_in), or null: not written
  void* out;                // [M, N] LayerNorm output, out_dtype
  const uint8_t* row_mask;  // null, or per row: 0 -> output row is zero
  const int32_t* m_tiles;   // null, or the live 128-row tiles (see tjb_row_tiles)
  int M, N, K;
  float eps;
  int out_dtype;
  uint32_t idesc;
};

struct GemmLnSmem {
  static constexpr int kStages = GemmCfg<256>::kStages;
  static constexpr size_t kRing = static_cast<size_t>(kStages) * GemmCfg<256>::kStageBytes;
  static constexpr size_t kStats = 2 * 2 * kBM * sizeof(float2);  // [buf][half][row]
  static constexpr size_t kBytes = 1024 + kRing + kStats + 512;
};

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_ln_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const GemmLnArgs args) {
  using Cfg = GemmCfg<256>;
  constexpr int kStages = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * Cfg::kABytes;
  float2* stats = reinterpret_cast<float2*>(smem + GemmLnSmem::kRing);  // [2][2][128]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + GemmLnSmem::kRing + GemmLnSmem::kStats);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* st_ready = drain + 1;  // [buf]
  uint64_t* st_free = st_ready + 2;  // [buf]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(st_free + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int C = args.N / 256;
  const uint32_t crank = cluster_ctarank();
  const int cid = static_cast<int>(blockIdx.x) / C;
  const int n_clusters = static_cast<int>(gridDim.x) / C;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
      mbar_init(&st_ready[b], 8 * C);  // every epilogue warp of the cluster
      mbar_init(&st_free[b], 8 * C);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // every CTA's barriers exist before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();
  griddep_launch_dependents();
  const int num_m = args.m_tiles != nullptr ? __ldg(args.m_tiles) : (args.M + kBM - 1) / kBM;
  const int num_k = (args.K + kBK - 1) / kBK;
  // This cluster's row blocks, one whole-K piece each; this CTA's column block.
  auto row_blocks = [&]() {
    int rb = cid;
    return [=](GemmPiece& un) mutable {
      if (rb >= num_m) return false;
      un.tile = rb;
      un.kb0 = 0;
      un.kb1 = num_k;
      rb += n_clusters;
      return true;
    };
  };
  auto m_block = [&](int tile) {
    return args.m_tiles != nullptr ? __ldg(args.m_tiles + 1 + tile) : tile;
  };

  if (warp == 0) {
    if (lane == 0)
      gemm_produce<256>(row_blocks(),
                        [&](int tile, int& m_blk, int& n_blk) {
                          m_blk = m_block(tile);
                          n_blk = static_cast<int>(crank);
                        },
                        &tmA, &tmB, sA, sB, full, empty, abort_flag);
  } else if (warp == 1) {
    gemm_mma<256>(row_blocks(), tmem_base, sA, sB, full, empty, tfull, tempty, drain, args.idesc,
                  abort_flag);
  } else {
    // -------------------------------------------------------------- epilogue
    const int quad = warp & 3;         // TMEM lanes this warp may access
    const int half = (warp - 2) >> 2;  // which 128 of the tile's 256 columns
    const int r_in = quad * 32 + lane;
    const int col0 = static_cast<int>(crank) * 256 + half * 128;
    const float inv_n = 1.0f / static_cast<float>(args.N);
    int acc = 0;
    uint32_t acc_phase = 0;
    auto next = row_blocks();
    GemmPiece un;
    for (int q = 0; next(un); ++q) {
      const int64_t row = static_cast<int64_t>(m_block(un.tile)) * kBM + r_in;
      const bool valid = row < args.M;
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], acc_phase, abort_flag))) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(acc * 256 + half * 128);
      // Pass 1: v = acc + bias + residual, back into the accumulator; this
      // row's mean and sum of squared deviations over the 128 columns.
      float mean = 0.f, m2 = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(taddr + c * 32, r);
        tmem_ld_wait(r);
        const int col = col0 + c * 32;
        const float4* b4 = reinterpret_cast<const float4*>(args.bias + col);
        const float4* x4 =
            reinterpret_cast<const float4*>(args.res_in + (valid ? row : 0) * args.N + col);
        float v[32];
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 bb = __ldg(b4 + i);
          const float4 xx = valid ? *(x4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
          v[4 * i] = __uint_as_float(r[4 * i]) + bb.x + xx.x;
          v[4 * i + 1] = __uint_as_float(r[4 * i + 1]) + bb.y + xx.y;
          v[4 * i + 2] = __uint_as_float(r[4 * i + 2]) + bb.z + xx.z;
          v[4 * i + 3] = __uint_as_float(r[4 * i + 3]) + bb.w + xx.w;
          s += (v[4 * i] + v[4 * i + 1]) + (v[4 * i + 2] + v[4 * i + 3]);
        }
        const float cm = s * (1.0f / 32.0f);
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
      tmem_st_wait();
      // Publish this warp's partials, wait for the cluster's, combine.
      const int buf = q & 1;
      const uint32_t use = static_cast<uint32_t>(q >> 1);
      bool ok = true;
      if (use >= 1)
        ok = __all_sync(0xffffffffu, mbar_wait_cluster(&st_free[buf], (use - 1) & 1, abort_flag));
      if (!ok) break;
      stats[(buf * 2 + half) * kBM + r_in] = make_float2(mean, m2);
      fence_acq_rel_cluster();
      __syncwarp();
      if (lane == 0)
        for (int dst = 0; dst < C; ++dst)
          mbar_arrive_cluster(map_to_rank(smem_u32(&st_ready[buf]), static_cast<uint32_t>(dst)));
      if (!__all_sync(0xffffffffu, mbar_wait_cluster(&st_ready[buf], use & 1, abort_flag))) break;
      float msum = 0.f, m2sum = 0.f;
      float pm[2 * kLnMaxCluster];
#pragma unroll
      for (int k = 0; k < 2 * kLnMaxCluster; ++k) {
        pm[k] = 0.f;
        if (k < 2 * C) {
          const uint32_t a = map_to_rank(
              smem_u32(&stats[(buf * 2 + (k & 1)) * kBM + r_in]), static_cast<uint32_t>(k >> 1));
          float2 p;
          asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];"
                       : "=f"(p.x), "=f"(p.y)
                       : "r"(a)
                       : "memory");
          pm[k] = p.x;
          msum += p.x;
          m2sum += p.y;
        }
      }
      const float mu = msum / static_cast<float>(2 * C);
#pragma unroll
      for (int k = 0; k < 2 * kLnMaxCluster; ++k) {
        if (k < 2 * C) {
          const float e = pm[k] - mu;
          m2sum = fmaf(128.0f * e, e, m2sum);
        }
      }
      const float rstd = rsqrtf(m2sum * inv_n + args.eps);
      fence_acq_rel_cluster();
      __syncwarp();
      if (lane == 0)
        for (int dst = 0; dst < C; ++dst)
          mbar_arrive_cluster(map_to_rank(smem_u32(&st_free[buf]), static_cast<uint32_t>(dst)));
      // Pass 2: normalise; write the residual and the LayerNorm output.
      const bool zero_row = args.row_mask != nullptr && valid && args.row_mask[row] == 0;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(taddr + c * 32, r);
        tmem_ld_wait(r);
        if (!valid) continue;
        const int col = col0 + c * 32;
        if (args.res_out != nullptr) {
          float4* d4 = reinterpret_cast<float4*>(args.res_out + row * args.N + col);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            d4[i] = make_float4(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1]),
                                __uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3]));
        }
        float y[32];
        const float4* g4 = reinterpret_cast<const float4*>(args.gamma + col);
        const float4* e4 = reinterpret_cast<const float4*>(args.beta + col);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 gg = __ldg(g4 + i);
          const float4 bb = __ldg(e4 + i);
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
          float4* o4 = reinterpret_cast<float4*>(static_cast<float*>(args.out) + row * args.N + col);
#pragma unroll
          for (int i = 0; i < 8; ++i) o4[i] = make_float4(y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
        } else {
          uint32_t p[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            p[i] = args.out_dtype == TJB_BF16 ? Pack2<__nv_bfloat16>::pack(y[2 * i], y[2 * i + 1])
                                              : Pack2<__half>::pack(y[2 * i], y[2 * i + 1]);
          uint4* o4 = reinterpret_cast<uint4*>(static_cast<uint16_t*>(args.out) + row * args.N + col);
#pragma unroll
          for (int i = 0; i < 4; ++i) o4[i] = make_uint4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while peers may still read its statistics
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

std::mutex g_ln_attr_mu;
bool g_ln_attr_done[64];

}  // namespace
}  // namespace tjb

extern "C" int tjb_gemm_add_layernorm(const void* A, const void* W, const float* bias,
                                      const float* res_in, float* res_out, const float* gamma,
                                      const float* beta, void* out, int M, int N, int K,
                                      float eps, int in_dtype, int out_dtype,
                                      const uint8_t* row_mask, const int32_t* m_tiles,
                                      tjb_stream_t stream) {
  using namespace tjb;
  if (!A || !W || !bias || !res_in || !gamma || !beta || !out || M < 0 || N <= 0 || K <= 0)
    return TJB_ERR_INVALID_ARGUMENT;
  if (in_dtype != TJB_F16 && in_dtype != TJB_BF16) return TJB_ERR_UNSUPPORTED_DTYPE;
  if (out_dtype != TJB_F32 && out_dtype != TJB_F16 && out_dtype != TJB_BF16)
    return TJB_ERR_UNSUPPORTED_DTYPE;
  const int C = N / 256;
  if (N % 256 != 0 || C > kLnMaxCluster || K % 8 != 0) return TJB_ERR_BAD_SHAPE;
  if (!aligned16(A) || !aligned16(W) || !aligned16(bias) || !aligned16(res_in) ||
      (res_out && !aligned16(res_out)) || !aligned16(gamma) || !aligned16(beta) ||
      !aligned16(out))
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
  CUtensorMap tmA, tmB;
  const uint64_t dimA[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
  const uint64_t strA[1] = {static_cast<uint64_t>(K) * 2};
  const uint32_t boxA[2] = {kBK, kBM};
  const uint64_t dimB[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
  const uint32_t boxB[2] = {kBK, 256};
  int st = make_tmap_16bit(&tmA, 2, A, dimA, strA, boxA, bf16);
  if (st != TJB_OK) return st;
  st = make_tmap_16bit(&tmB, 2, W, dimB, strA, boxB, bf16);
  if (st != TJB_OK) return st;
  GemmLnArgs a;
  a.bias = bias;
  a.gamma = gamma;
  a.beta = beta;
  a.res_in = res_in;
  a.res_out = res_out;
  a.out = out;
  a.row_mask = row_mask;
  a.m_tiles = m_tiles;
  a.M = M;
  a.N = N;
  a.K = K;
  a.eps = eps;
  a.out_dtype = out_dtype;
  a.idesc = idesc_f16(kBM, 256, bf16, false);
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = GemmLnSmem::kBytes;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  // As many clusters as can be resident at once, each walking row blocks.
  cfg.gridDim = dim3(num_sms() / C * C);
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, gemm_ln_kernel, &cfg) != cudaSuccess ||
      clusters <= 0)
    clusters = num_sms() / C;
  const int max_blocks = (M + kBM - 1) / kBM;
  if (clusters > max_blocks) clusters = max_blocks;
  cfg.gridDim = dim3(clusters * C);
  return cuda_status(cudaLaunchKernelEx(&cfg, gemm_ln_kernel, tmA, tmB, a));
}
