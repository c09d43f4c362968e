// ffn_fused.cu -- the feed-forward block in one kernel, hidden tile on chip:
//   out = gelu_erf(h W1^T + b1) W2^T + b2
//
// The fp32 output accumulator of a 128-token tile is 128 x d; tensor memory
// (512 columns) holds 256 of its columns next to the GEMM1 accumulators, so a
// cluster of C = d / 256 CTAs (one per SM) shares each token tile: CTA c owns
// output columns [256c, 256c + 256).  The hidden dimension F is walked in
// chunks of Fc = 128 C; for chunk j CTA c computes hidden columns
// [j Fc + 128c, +128):
//   GEMM1  G = h_tile [128 x d] * W1_slice^T   (tcgen05, 128 x 128, fp32 TMEM)
//   epilogue warps: + b1, exact erf-GELU, round to the input type, and store
//          the 128 x 128 slice into the hidden-chunk buffer of EVERY CTA of
//          the cluster (plain distributed-shared-memory stores), then arrive
//          on each CTA's h_ready barrier;
//   GEMM2  O += H_chunk [128 x Fc] * W2_slice^T  (A from this CTA's shared
//          memory, 128 x 256 into TMEM) once all C slices have landed.
// The hidden tile never leaves the SMs.  GEMM1 of chunk j+1 is issued before
// GEMM2 of chunk j (two GEMM1 accumulators), so the tensor core runs while the
// epilogue warps compute GELU and exchange slices.  A helper warp turns each
// local GEMM2 completion into an arrival on every CTA's h_free barrier: a
// CTA may overwrite the shared hidden chunk only when all C CTAs finished
// reading the previous one.
//
// Roles (256 threads): warp 0 TMA producer (one 32 KB-stage ring feeds both
// GEMMs in consumption order), warp 1 TMEM owner + MMA issuer, warp 2 cluster
// relay, warp 3 idle, warps 4-7 epilogue (one TMEM lane quadrant each).
// Persistent: each cluster walks 128-token tiles (optionally only the listed
// live tiles).  No TMA load is shared between CTAs.
#include <mutex>

#include "common.cuh"

namespace tjb {
namespace {

constexpr int kFfnThreads = 256;
constexpr uint32_t kFStage = 32768;  // one ring stage
constexpr uint32_t kFSub = 16384;    // 128 rows x 64 columns of 16-bit

struct FfnArgs {
  const float* b1;
  const float* b2;
  const int32_t* m_tiles;
  void* out;
  int T, d, F;
  int C;        // cluster size = d / 256
  int stages;   // ring depth
  int out_dtype;
  int bf16;
  uint32_t idesc1, idesc2;
};

__device__ __forceinline__ uint32_t swz(int row, int chunk16) {
  // 128-byte swizzle inside a 128-row x 64-column 16-bit sub-tile.
  return static_cast<uint32_t>(row * 128 + ((chunk16 ^ (row & 7)) << 4));
}

__global__ void __launch_bounds__(kFfnThreads, 1)
    ffn_fused_kernel(const __grid_constant__ CUtensorMap tmH, const __grid_constant__ CUtensorMap tmW1,
                     const __grid_constant__ CUtensorMap tmW2, const FfnArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int C = args.C;
  const int S = args.stages;
  uint8_t* ring = smem;                       // [S][32 KB]
  uint8_t* hbuf = ring + S * kFStage;         // [2C][16 KB]: the hidden chunk, 128 x Fc
  uint64_t* full = reinterpret_cast<uint64_t*>(hbuf + 2 * C * kFSub);
  uint64_t* empty = full + 8;
  uint64_t* g1_full = empty + 8;   // [2]
  uint64_t* g1_empty = g1_full + 2;
  uint64_t* h_ready = g1_empty + 2;
  uint64_t* h_free = h_ready + 1;
  uint64_t* g2_done = h_free + 1;
  uint64_t* o_full = g2_done + 1;
  uint64_t* o_empty = o_full + 1;
  uint64_t* drain = o_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const int cid = blockIdx.x / C;
  const int n_clusters = gridDim.x / C;
  const int Fc = 128 * C;
  const int NJ = args.F / Fc;
  const int nk1 = args.d / 64;  // GEMM1 k-blocks
  const int nk2 = 2 * C;        // GEMM2 k-blocks per chunk

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&g1_full[i], 1);
      mbar_init(&g1_empty[i], 4);
    }
    mbar_init(h_ready, 4 * C);
    mbar_init(h_free, C);
    mbar_init(g2_done, 1);
    mbar_init(o_full, 1);
    mbar_init(o_empty, 4);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmH);
    prefetch_tmap(&tmW1);
    prefetch_tmap(&tmW2);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  cluster_sync();  // every CTA's barriers exist before any remote arrive
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();
  griddep_launch_dependents();
  const uint32_t kOCol = 0, kG1Col = 256;
  const int num_m = args.m_tiles != nullptr ? __ldg(args.m_tiles) : (args.T + 127) / 128;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      int stage = 0;
      uint32_t phase = 0, issued = 0, issued_parity = 0;
      bool ok = true;
      auto next = [&](uint64_t*& bar, uint8_t*& dst) -> bool {
        if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) return false;
        bar = &full[stage];
        dst = ring + stage * kFStage;
        mbar_arrive_expect_tx(bar, kFStage);
        issued |= 1u << stage;
        issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
        if (++stage == S) {
          stage = 0;
          phase ^= 1;
        }
        return true;
      };
      for (int t = cid; t < num_m && ok; t += n_clusters) {
        const int m = args.m_tiles != nullptr ? __ldg(args.m_tiles + 1 + t) : t;
        for (int j = 0; j <= NJ && ok; ++j) {
          if (j < NJ) {
            for (int kb = 0; kb < nk1; ++kb) {
              uint64_t* bar;
              uint8_t* dst;
              if (!(ok = next(bar, dst))) break;
              tma_load_2d(dst, &tmH, bar, kb * 64, m * 128);
              tma_load_2d(dst + kFSub, &tmW1, bar, kb * 64, j * Fc + 128 * static_cast<int>(crank));
            }
          }
          if (j >= 1 && ok) {
            for (int kb = 0; kb < nk2; ++kb) {
              uint64_t* bar;
              uint8_t* dst;
              if (!(ok = next(bar, dst))) break;
              tma_load_2d(dst, &tmW2, bar, (j - 1) * Fc + kb * 64, 256 * static_cast<int>(crank));
            }
          }
        }
      }
      for (int s = 0; s < S; ++s)
        if ((issued >> s) & 1u) mbar_wait_drain(&full[s], (issued_parity >> s) & 1u);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    // The whole warp runs this loop, converged; one elected lane issues.
    const uint32_t hb = smem_u32(hbuf);
    int stage = 0;
    uint32_t phase = 0, g1c = 0, g2c = 0, tc = 0;
    bool ok = true;
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
    };
    for (int t = cid; t < num_m && ok; t += n_clusters) {
      for (int j = 0; j <= NJ && ok; ++j) {
        if (j < NJ) {
          const uint32_t buf = g1c & 1;
          if (!wait(&g1_empty[buf], ((g1c >> 1) & 1) ^ 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_g = tmem_base + kG1Col + buf * 128;
          for (int kb = 0; kb < nk1; ++kb) {
            if (!wait(&full[stage], phase)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a0 = smem_u32(ring + stage * kFStage);
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_ss_w(d_g, sdesc_sw128(a0 + k * 32, 16, 1024),
                        sdesc_sw128(a0 + kFSub + k * 32, 16, 1024), args.idesc1,
                        (kb | k) != 0 ? 1u : 0u);
            umma_commit_w(&empty[stage]);
            if (++stage == S) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (!ok) break;
          umma_commit_w(&g1_full[buf]);
          ++g1c;
        }
        if (j >= 1) {
          // All C slices of hidden chunk j-1 are in this CTA's buffer.
          if (!__all_sync(0xffffffffu, mbar_wait_cluster(h_ready, g2c & 1, abort_flag))) {
            ok = false;
            break;
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          tc_fence_after();
          if (j == 1 && !wait(o_empty, (tc & 1) ^ 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int kb = 0; kb < nk2; ++kb) {
            if (!wait(&full[stage], phase)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t b0 = smem_u32(ring + stage * kFStage);
            const uint32_t a0 = hb + kb * kFSub;
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_ss_w(tmem_base + kOCol, sdesc_sw128(a0 + k * 32, 16, 1024),
                        sdesc_sw128(b0 + k * 32, 16, 1024), args.idesc2,
                        (j > 1 || kb > 0 || k > 0) ? 1u : 0u);
            umma_commit_w(&empty[stage]);
            if (++stage == S) {
              stage = 0;
              phase ^= 1;
            }
          }
          if (!ok) break;
          umma_commit_w(g2_done);
          ++g2c;
        }
      }
      if (!ok) break;
      umma_commit_w(o_full);
      ++tc;
    }
    umma_commit_w(drain);
    mbar_wait_drain(drain, 0);
  } else if (warp == 2) {
    if (lane == 0) {
      // ------------------------------------------------ cluster relay of h_free
      // Each local GEMM2 completion means this CTA is done reading the shared
      // hidden chunk; tell every CTA of the cluster.
      const uint32_t hf = smem_u32(h_free);
      uint32_t n = 0;
      bool ok = true;
      for (int t = cid; t < num_m && ok; t += n_clusters) {
        for (int j = 0; j < NJ; ++j, ++n) {
          if (!mbar_wait(g2_done, n & 1, abort_flag)) {
            ok = false;
            break;
          }
          for (int r = 0; r < C; ++r) mbar_arrive_cluster(map_to_rank(hf, r));
        }
      }
    }
  } else if (warp >= 4) {
    // -------------------------------------------------------------- epilogue
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t hb = smem_u32(hbuf);
    const uint32_t hr = smem_u32(h_ready);
    uint32_t g1c = 0, hc = 0, tc = 0;
    bool ok = true;
    for (int t = cid; t < num_m && ok; t += n_clusters) {
      const int m = args.m_tiles != nullptr ? __ldg(args.m_tiles + 1 + t) : t;
      const int row = m * 128 + r;
      for (int j = 0; j < NJ; ++j) {
        const uint32_t buf = g1c & 1;
        bool w_ok = mbar_wait(&g1_full[buf], (g1c >> 1) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, w_ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t g[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32p(lane_base + kG1Col + buf * 128 + c * 32, g + c * 32);
        tmem_ld_wait_n<128>(g);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&g1_empty[buf]);
        ++g1c;
        const int hcol0 = j * Fc + 128 * static_cast<int>(crank);
        uint32_t hv[64];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float4 bb = __ldg(reinterpret_cast<const float4*>(args.b1 + hcol0) + c);
          const float x0 = gelu_erf(__uint_as_float(g[4 * c]) + bb.x);
          const float x1 = gelu_erf(__uint_as_float(g[4 * c + 1]) + bb.y);
          const float x2 = gelu_erf(__uint_as_float(g[4 * c + 2]) + bb.z);
          const float x3 = gelu_erf(__uint_as_float(g[4 * c + 3]) + bb.w);
          if (args.bf16) {
            hv[2 * c] = Pack2<__nv_bfloat16>::pack(x0, x1);
            hv[2 * c + 1] = Pack2<__nv_bfloat16>::pack(x2, x3);
          } else {
            hv[2 * c] = Pack2<__half>::pack(x0, x1);
            hv[2 * c + 1] = Pack2<__half>::pack(x2, x3);
          }
        }
        // Every CTA must have finished GEMM2 on the previous chunk.
        if (hc >= 1) {
          w_ok = mbar_wait_cluster(h_free, (hc - 1) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, w_ok)) {
            ok = false;
            break;
          }
        }
        // This CTA's 128 hidden columns are sub-tiles 2c and 2c+1 of the chunk.
        const uint32_t local = hb + 2 * crank * kFSub;
        for (int dst = 0; dst < C; ++dst) {
          const uint32_t base = map_to_rank(local, dst);
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const uint32_t off = (q >> 3) * kFSub + swz(r, q & 7);
            st_cluster_v4(base + off,
                          make_uint4(hv[4 * q], hv[4 * q + 1], hv[4 * q + 2], hv[4 * q + 3]));
          }
        }
        fence_proxy_async_smem_cluster();
        fence_acq_rel_cluster();
        __syncwarp();
        if (lane == 0)
          for (int dst = 0; dst < C; ++dst) mbar_arrive_cluster(map_to_rank(hr, dst));
        ++hc;
      }
      if (!ok) break;
      // Output tile: O + b2 -> out[:, 256c : 256c + 256).
      bool w_ok = mbar_wait(o_full, tc & 1, abort_flag);
      if (!__all_sync(0xffffffffu, w_ok)) break;
      tc_fence_after();
      const int col0 = 256 * static_cast<int>(crank);
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        uint32_t o[32];
        tmem_ld32(lane_base + kOCol + c * 32, o);
        tmem_ld_wait(o);
        if (row < args.T) {
          float v[32];
          const float4* b4 = reinterpret_cast<const float4*>(args.b2 + col0 + c * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 bb = __ldg(b4 + i);
            v[4 * i] = __uint_as_float(o[4 * i]) + bb.x;
            v[4 * i + 1] = __uint_as_float(o[4 * i + 1]) + bb.y;
            v[4 * i + 2] = __uint_as_float(o[4 * i + 2]) + bb.z;
            v[4 * i + 3] = __uint_as_float(o[4 * i + 3]) + bb.w;
          }
          const int64_t base = static_cast<int64_t>(row) * args.d + col0 + c * 32;
          if (args.out_dtype == TJB_F32) {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(args.out) + base);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              dst[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          } else {
            uint32_t p[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              p[i] = args.out_dtype == TJB_BF16 ? Pack2<__nv_bfloat16>::pack(v[2 * i], v[2 * i + 1])
                                                : Pack2<__half>::pack(v[2 * i], v[2 * i + 1]);
            uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(args.out) + base);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              dst[i] = make_uint4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_empty);
      ++tc;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while peers may still write into its shared memory
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

std::mutex g_ffn_attr_mu;
bool g_ffn_attr_done[64];

}  // namespace
}  // namespace tjb

// Fused FFN; see the file comment.  Needs d in {256, 512, 768, 1024},
// F % (128 * d / 256) == 0, f16/bf16 inputs; out fp32 or the input type.
extern "C" int tjb_ffn_fused(const void* h, const void* w1, const float* b1, const void* w2,
                             const float* b2, void* out, int T, int d, int F, int in_dtype,
                             int out_dtype, const int32_t* m_tiles, tjb_stream_t stream) {
  using namespace tjb;
  if (!h || !w1 || !w2 || !out || !b1 || !b2 || T < 0 || d <= 0 || F <= 0)
    return TJB_ERR_INVALID_ARGUMENT;
  if (in_dtype != TJB_F16 && in_dtype != TJB_BF16) return TJB_ERR_UNSUPPORTED_DTYPE;
  if (out_dtype != TJB_F32 && out_dtype != in_dtype) return TJB_ERR_UNSUPPORTED_DTYPE;
  const int C = d / 256;
  if (d % 256 != 0 || C < 1 || C > 4 || F % (128 * C) != 0) return TJB_ERR_BAD_SHAPE;
  if (!aligned16(h) || !aligned16(w1) || !aligned16(w2) || !aligned16(out) || !aligned16(b1) ||
      !aligned16(b2))
    return TJB_ERR_BAD_ALIGNMENT;
  if (!device_ok()) return TJB_ERR_NO_DEVICE;
  if (T == 0) return TJB_OK;
  const int stages = C == 4 ? 3 : (C == 3 ? 4 : (C == 2 ? 5 : 6));
  const size_t smem = 1024 + static_cast<size_t>(stages) * kFStage + 2 * C * kFSub + 512;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(g_ffn_attr_mu);
    if (dev < 64 && !g_ffn_attr_done[dev]) {
      if (const int fs = cuda_status(cudaFuncSetAttribute(
              ffn_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448)))
        return fs;
      g_ffn_attr_done[dev] = true;
    }
  }
  const bool bf16 = in_dtype == TJB_BF16;
  CUtensorMap tmH, tmW1, tmW2;
  const uint64_t dimH[2] = {static_cast<uint64_t>(d), static_cast<uint64_t>(T)};
  const uint64_t strH[1] = {static_cast<uint64_t>(d) * 2};
  const uint32_t box128[2] = {64, 128};
  const uint64_t dimW1[2] = {static_cast<uint64_t>(d), static_cast<uint64_t>(F)};
  const uint64_t dimW2[2] = {static_cast<uint64_t>(F), static_cast<uint64_t>(d)};
  const uint64_t strW2[1] = {static_cast<uint64_t>(F) * 2};
  const uint32_t box256[2] = {64, 256};
  int st = make_tmap_16bit(&tmH, 2, h, dimH, strH, box128, bf16);
  if (st == TJB_OK) st = make_tmap_16bit(&tmW1, 2, w1, dimW1, strH, box128, bf16);
  if (st == TJB_OK) st = make_tmap_16bit(&tmW2, 2, w2, dimW2, strW2, box256, bf16);
  if (st != TJB_OK) return st;
  FfnArgs a;
  a.b1 = b1;
  a.b2 = b2;
  a.m_tiles = m_tiles;
  a.out = out;
  a.T = T;
  a.d = d;
  a.F = F;
  a.C = C;
  a.stages = stages;
  a.out_dtype = out_dtype;
  a.bf16 = bf16;
  a.idesc1 = idesc_f16(128, 128, bf16, false);
  a.idesc2 = idesc_f16(128, 256, bf16, false);
  const int max_tiles = (T + 127) / 128;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kFfnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // As many clusters as can be resident at once (SMs are grouped, so this
  // can be fewer than SMs / C); each walks tiles persistently.
  cfg.gridDim = dim3(num_sms() / C * C);
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, ffn_fused_kernel, &cfg) != cudaSuccess ||
      clusters <= 0)
    clusters = num_sms() / C;
  if (clusters > max_tiles) clusters = max_tiles;
  cfg.gridDim = dim3(clusters * C);
  return cuda_status(cudaLaunchKernelEx(&cfg, ffn_fused_kernel, tmH, tmW1, tmW2, a));
}
