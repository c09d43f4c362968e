// forward_small.cu -- the whole encoder forward of a small batch (at most
// 256 tokens, head_dim 64) in one persistent cooperative kernel.
//
// At a few dozen tokens every GEMM of the block is a weight stream: each
// weight is used by at most 256 tokens, and a launch per op spends most of
// its time starting, filling its pipeline and draining.  Here one grid (one
// CTA per SM, co-resident by a cooperative launch) runs the forward as a
// sequence of phases separated by grid barriers (a counter and a generation
// word in global memory, every wait bounded):
//
//   per layer  LN1 (+ the previous FFN-out's split-K partials, bias, residual)
//              QKV GEMM -> qkv            attention -> ctx
//              out-projection GEMM, split over K -> fp32 partials
//              LN2 (+ those partials, bias, residual)
//              FFN-in GEMM + bias + erf-GELU -> hidden
//              FFN-out GEMM, split over K -> fp32 partials
//   then       final LayerNorm (+ the last partials), padded rows written as 0
//
// GEMMs are swapped so that the weights fill the MMA's M side: a work unit
// is 128 output features x up to 128 (padded) tokens x a range of k-blocks;
// warp 0 TMA-loads the weight tile (128 x 64) and the activation tile
// (tokens x 64, both K-major, 128-byte swizzle) into a 4-stage ring, warp 1
// issues tcgen05.mma (M=128, N=tokens, K=16) into one of two TMEM
// accumulators, and warps 2-9 read it back (one feature per TMEM lane, 32
// tokens per load) and store 32 consecutive features of a token per warp
// instruction.  The out-projection and FFN-out have few output features
// (d / 128 tiles), so their k-blocks are split over the grid and the next
// LayerNorm phase adds the partials in a fixed order.  While a phase runs,
// each CTA prefetches into L2 the weight boxes of its next GEMM phase.
// Attention (a sequence of at most 128 tokens) runs on the CUDA cores in
// fp32, a CTA per (sequence, head, 8 query rows).  Activations stay in L2
// between phases.
#include <algorithm>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace tjb {
namespace {

constexpr int kFsThreads = 320;   // producer warp, MMA warp, eight epilogue warps
constexpr int kFsMaxLayers = 12;
constexpr int kFsMaxTokens = 256;
constexpr int kFsUnitTokens = 128; // tokens of one GEMM unit (the MMA's N): a TMEM accumulator
constexpr int kFsMaxSeq = 128;    // attention keeps a sequence's K and V in shared memory
constexpr int kFsHead = 64;
constexpr int kFsStages = 4;
constexpr int kFsQRows = 16;      // most query rows per attention unit (two per warp)

struct FsLayer {
  const float* ln1_w;
  const float* ln1_b;
  const float* bqkv;
  const float* bo;
  const float* ln2_w;
  const float* ln2_b;
  const float* b1;
  const float* b2;
  float ln1_eps, ln2_eps;
};

struct FsArgs {
  // Weights (A operands, [out, in] K-major) and activations (B operands,
  // [tokens, K] K-major): 128-byte-swizzled 64-column boxes.
  CUtensorMap w_qkv[kFsMaxLayers], w_o[kFsMaxLayers], w_1[kFsMaxLayers], w_2[kFsMaxLayers];
  CUtensorMap x_h, x_ctx, x_h2, x_hidden;
  FsLayer layer[kFsMaxLayers];
  const float* lnf_w;
  const float* lnf_b;
  float lnf_eps;
  const float* x;           // [T, d] input
  float* out;               // [T, d] output
  const uint8_t* valid;     // [T]: 0 marks a padded token (masked key, zero output row), or null
  float* res;               // [T, d] residual stream
  uint16_t* h;              // [T, d] LN1 output
  uint16_t* qkv;            // [T, 3d]
  uint16_t* ctx;            // [T, d]
  uint16_t* h2;             // [T, d] LN2 output
  uint16_t* hidden;         // [T, F]
  float* part;              // [split][T][d] split-K partials
  unsigned* bar;            // [2]: arrivals, generation (the generation never resets)
  int B, S, T, Tpad, d, H, F, L;
  int Tsub, n_tsub;         // tokens per GEMM unit (<= 128) and sub-blocks of Tpad
  int causal;
  int qrows;                // query rows per attention unit: 8, or 16 when 8 would overfill the grid
  int ks_o, ks_2;           // k-splits of the out-projection and FFN-out
  uint32_t idesc;
  float scale_log2;         // softmax scale * log2(e)
};

struct FsSmem {
  static constexpr uint32_t kABytes = 128 * 64 * 2;
  static constexpr uint32_t kBBytes = kFsUnitTokens * 64 * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr size_t kRing = static_cast<size_t>(kFsStages) * kStageBytes;
  static constexpr size_t kBytes = 1024 + kRing + 1024;
};
// The attention phase keeps K, V and a query block in the (then idle) ring.
static_assert((2 * kFsHead * kFsMaxSeq + kFsQRows * kFsHead) * sizeof(float) <= FsSmem::kRing,
              "attention tiles must fit the operand ring");

__device__ __forceinline__ unsigned fs_ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Grid-wide barrier number `k` (1, 2, ...) of this launch; gen0 is the
// generation word read at entry.  Arrival is a release atomic on the
// counter (the CTA's writes, gathered by the __syncthreads before it); the
// last CTA in resets the counter and publishes the generation with a
// release store, which the others poll with acquire loads.  Bounded: false
// once the wait exceeds kWaitTimeoutNs (the status word records it).
__device__ __forceinline__ bool fs_grid_sync(unsigned* bar, unsigned gen0, unsigned k,
                                             volatile int* abort_flag) {
  // Generic-proxy writes of this phase (global activations, and the
  // attention tiles in the shared ring) are ordered before the next phase's
  // TMA (async-proxy) accesses.
  fence_proxy_async_global();
  fence_proxy_async_smem();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned target = gen0 + k;
    unsigned old;
    asm volatile("atom.add.release.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(bar) : "memory");
    if (old == gridDim.x - 1) {
      asm volatile("st.relaxed.gpu.global.u32 [%0], 0;" ::"l"(bar) : "memory");
      asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(bar + 1), "r"(target) : "memory");
    } else {
      const uint64_t t0 = globaltimer();
      for (uint32_t i = 1; static_cast<int>(fs_ld_acquire_u32(bar + 1) - target) < 0; ++i) {
        if ((i & 255) == 0 && globaltimer() - t0 > kWaitTimeoutNs) {
          record_status(TJB_ERR_DEVICE_TIMEOUT);
          *abort_flag = 1;
          break;
        }
      }
    }
  }
  __syncthreads();
  fence_proxy_async_global();
  return *abort_flag == 0;
}

// L2 prefetch of the weight boxes this CTA's units of a coming GEMM phase
// will load (one thread; the boxes are those fs_gemm's producer issues).
__device__ __forceinline__ void fs_prefetch_weights(const FsArgs& a, const CUtensorMap* tmW,
                                                    int N, int K, int ks) {
  const int kb_total = K / 64;
  const int kbu = (kb_total + ks - 1) / ks;
  const int units = (N / 128) * ks * a.n_tsub;
  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    if (u % a.n_tsub != 0) continue;  // the other token blocks read the same boxes
    const int rest = u / a.n_tsub;
    const int nt = rest / ks, kc = rest - (rest / ks) * ks;
    for (int kb = kc * kbu; kb < min(kb_total, kc * kbu + kbu); ++kb)
      asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                       reinterpret_cast<uint64_t>(tmW)),
                   "r"(kb * 64), "r"(nt * 128)
                   : "memory");
  }
}

// Ring and accumulator positions; every role keeps its own copy and moves
// only the fields it owns, across all GEMM phases of the launch.
struct FsRing {
  int stage = 0;
  uint32_t phase = 0;
  int acc = 0;
  uint32_t acc_phase = 0;
  uint32_t issued = 0, last_parity = 0;  // producer: stages with a load, its parity
};

struct FsShared {
  uint8_t* sA;
  uint8_t* sB;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* tfull;
  uint64_t* tempty;
  uint32_t tmem_base;
  volatile int* abort_flag;
};

// One GEMM phase: out[t][n] over N output features (weights [N, K]) and the
// padded tokens, K a multiple of 64, N of 128.  Units (feature tile nt,
// k-split kc) go to the CTAs in turn.  ks == 1: out16 = act(acc + bias) in
// 16-bit [T, N]; ks > 1: part[kc][T][N] = acc (fp32, no bias).
__device__ __forceinline__ void fs_gemm(const FsArgs& a, const CUtensorMap* tmW,
                                        const CUtensorMap* tmX, int N, int K, int ks,
                                        const float* bias, int act, uint16_t* out16, float* part,
                                        const FsShared& sh, FsRing& ring) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kb_total = K / 64;
  const int kbu = (kb_total + ks - 1) / ks;
  const int units = (N / 128) * ks * a.n_tsub;
  // Unit u: token sub-block u % n_tsub, then k-split, then feature tile.
  auto unit_range = [&](int u, int& nt, int& kc, int& kb0, int& kb1, int& ts) {
    ts = u % a.n_tsub;
    const int rest = u / a.n_tsub;
    nt = rest / ks;
    kc = rest - nt * ks;
    kb0 = kc * kbu;
    kb1 = min(kb_total, kb0 + kbu);
  };
  if (warp == 0) {
    if (lane == 0) {
      const uint32_t tx = FsSmem::kABytes + static_cast<uint32_t>(a.Tsub) * 128u;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
        int nt, kc, kb0, kb1, ts;
        unit_range(u, nt, kc, kb0, kb1, ts);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&sh.empty[ring.stage], ring.phase ^ 1, sh.abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&sh.full[ring.stage], tx);
          tma_load_2d(sh.sA + ring.stage * FsSmem::kABytes, tmW, &sh.full[ring.stage], kb * 64,
                      nt * 128);
          tma_load_2d(sh.sB + ring.stage * FsSmem::kBBytes, tmX, &sh.full[ring.stage], kb * 64,
                      ts * a.Tsub);
          ring.issued |= 1u << ring.stage;
          ring.last_parity = (ring.last_parity & ~(1u << ring.stage)) | (ring.phase << ring.stage);
          if (++ring.stage == kFsStages) {
            ring.stage = 0;
            ring.phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait(bar, parity, sh.abort_flag));
    };
    bool ok = true;
    for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
      int nt, kc, kb0, kb1, ts;
      unit_range(u, nt, kc, kb0, kb1, ts);
      if (kb0 >= kb1) continue;
      if (!wait(&sh.tempty[ring.acc], ring.acc_phase ^ 1)) break;
      tc_fence_after();
      const uint32_t d_tmem = sh.tmem_base + static_cast<uint32_t>(ring.acc * kFsUnitTokens);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!wait(&sh.full[ring.stage], ring.phase)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(sh.sA + ring.stage * FsSmem::kABytes);
        const uint32_t b0 = smem_u32(sh.sB + ring.stage * FsSmem::kBBytes);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_ss_w(d_tmem, sdesc_sw128(a0 + k * 32, 16, 1024), sdesc_sw128(b0 + k * 32, 16, 1024),
                    a.idesc, (kb > kb0 || k > 0) ? 1u : 0u);
        umma_commit_w(&sh.empty[ring.stage]);
        if (++ring.stage == kFsStages) {
          ring.stage = 0;
          ring.phase ^= 1;
        }
      }
      if (!ok) break;
      umma_commit_w(&sh.tfull[ring.acc]);
      if (++ring.acc == 2) {
        ring.acc = 0;
        ring.acc_phase ^= 1;
      }
    }
  } else {
    const int quad = warp & 3;         // TMEM lanes (features) this warp may read
    const int half = (warp - 2) >> 2;  // which token chunks
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      int nt, kc, kb0, kb1, ts;
      unit_range(u, nt, kc, kb0, kb1, ts);
      if (kb0 >= kb1) continue;
      if (!__all_sync(0xffffffffu, mbar_wait(&sh.tfull[ring.acc], ring.acc_phase, sh.abort_flag)))
        break;
      tc_fence_after();
      const int n = nt * 128 + quad * 32 + lane;  // this thread's output feature
      const uint32_t taddr = sh.tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(ring.acc * kFsUnitTokens);
      const float bn = ks == 1 && bias != nullptr ? __ldg(bias + n) : 0.f;
      const int t0 = ts * a.Tsub;
#pragma unroll 1
      for (int c = half; c * 32 < a.Tsub && t0 + c * 32 < a.T; c += 2) {
        uint32_t r[32];
        tmem_ld32(taddr + c * 32, r);
        tmem_ld_wait(r);
        if (ks == 1) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int t = t0 + c * 32 + i;
            float v = __uint_as_float(r[i]) + bn;
            if (act) v = gelu_erf(v);
            if (t < a.T) out16[static_cast<int64_t>(t) * N + n] = __half_as_ushort(__float2half_rn(v));
          }
        } else {
          float* dst = part + static_cast<int64_t>(kc) * a.T * N + n;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int t = t0 + c * 32 + i;
            if (t < a.T) __stcg(dst + static_cast<int64_t>(t) * N, __uint_as_float(r[i]));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.tempty[ring.acc]);
      if (++ring.acc == 2) {
        ring.acc = 0;
        ring.acc_phase ^= 1;
      }
    }
  }
}

// Two 16-bit values written earlier in this launch by another CTA: an L2
// (coherent) load, never the read-only path.
__device__ __forceinline__ __half2 fs_ld_half2(const uint16_t* p) {
  const unsigned u = __ldcg(reinterpret_cast<const unsigned*>(p));
  return *reinterpret_cast<const __half2*>(&u);
}

// Attention, fp32 on the CUDA cores: a unit is (sequence b, head hh,
// a.qrows query rows); 8-row units spread a small batch over more SMs,
// 16-row units keep a larger one within one unit per CTA.  K rows [0, keys) of the head go to shared memory dimension-major
// (sKT[e][j]) so that lane l reads keys 4l .. 4l + 3 of one dimension with
// a single 16-byte load; V stays row-major (lane l reads dimensions 2l,
// 2l + 1).  a.qrows / 2 warps take two query rows each and share every K
// and V load between them; all warps load the tiles.  Keys after a row
// (causal) and padded keys are left out; a row with no key left is written
// as zero.
__device__ __forceinline__ void fs_attention(const FsArgs& a, float* sm) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qb = (a.S + a.qrows - 1) / a.qrows;
  const int units = a.B * a.H * n_qb;
  const int ld = 3 * a.d;  // qkv row length
  float* sKT = sm;                           // [kFsHead][kFsMaxSeq]
  float* sV = sKT + kFsHead * kFsMaxSeq;     // [kFsMaxSeq][kFsHead]
  float* sQ = sV + kFsMaxSeq * kFsHead;      // [kFsQRows][kFsHead]
  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    const int qb = u % n_qb;
    const int bh = u / n_qb;
    const int b = bh / a.H, hh = bh - (bh / a.H) * a.H;
    const int q0 = qb * a.qrows, q1 = min(a.S, q0 + a.qrows);
    const int keys = a.causal ? q1 : a.S;
    const uint8_t* vk = a.valid != nullptr ? a.valid + static_cast<int64_t>(b) * a.S : nullptr;
    const uint16_t* base = a.qkv + static_cast<int64_t>(b) * a.S * ld + hh * kFsHead;
    __syncthreads();  // the previous unit is done with the shared tiles
    // Eight loads per thread in flight before their shared-memory stores.
    // K: consecutive threads take consecutive keys of one dimension pair
    // (dimension-major stores); V and Q: consecutive threads take
    // consecutive dimension pairs of a row.
    const int nk = keys * 32, nq = (q1 - q0) * 32;
    for (int i0 = 0; i0 < nk; i0 += 8 * kFsThreads) {
      __half2 kv[8], vv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int idx = i0 + i * kFsThreads + threadIdx.x;
        if (idx < nk) {
          const int r = idx % keys, c2 = (idx / keys) * 2;
          kv[i] = fs_ld_half2(base + static_cast<int64_t>(r) * ld + a.d + c2);
          const int rv = idx >> 5, cv = (idx & 31) * 2;
          vv[i] = fs_ld_half2(base + static_cast<int64_t>(rv) * ld + 2 * a.d + cv);
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int idx = i0 + i * kFsThreads + threadIdx.x;
        if (idx < nk) {
          const int r = idx % keys, c2 = (idx / keys) * 2;
          sKT[c2 * kFsMaxSeq + r] = __low2float(kv[i]);
          sKT[(c2 + 1) * kFsMaxSeq + r] = __high2float(kv[i]);
          const int rv = idx >> 5, cv = (idx & 31) * 2;
          *reinterpret_cast<float2*>(sV + rv * kFsHead + cv) = __half22float2(vv[i]);
        }
      }
    }
    for (int i0 = 0; i0 < nq; i0 += 2 * kFsThreads) {
      __half2 qv[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int idx = i0 + i * kFsThreads + threadIdx.x;
        if (idx < nq)
          qv[i] = fs_ld_half2(base + static_cast<int64_t>(q0 + (idx >> 5)) * ld + (idx & 31) * 2);
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int idx = i0 + i * kFsThreads + threadIdx.x;
        if (idx < nq)
          *reinterpret_cast<float2*>(sQ + (idx >> 5) * kFsHead + (idx & 31) * 2) =
              __half22float2(qv[i]);
      }
    }
    __syncthreads();
    if (warp >= a.qrows / 2) continue;
    const int iA = q0 + 2 * warp, iB = iA + 1;
    if (iA >= q1) continue;
    const bool hasB = iB < q1;
    const int limA = a.causal ? iA + 1 : a.S;
    const int limB = hasB ? (a.causal ? iB + 1 : a.S) : 0;
    const float* qA = sQ + (iA - q0) * kFsHead;
    const float* qB = sQ + (hasB ? iB - q0 : iA - q0) * kFsHead;
    float sA[4] = {0.f, 0.f, 0.f, 0.f}, sB[4] = {0.f, 0.f, 0.f, 0.f};
    if (4 * lane < keys) {
#pragma unroll 4
      for (int e4 = 0; e4 < kFsHead / 4; ++e4) {
        const float4 a4 = *reinterpret_cast<const float4*>(qA + 4 * e4);
        const float4 b4 = *reinterpret_cast<const float4*>(qB + 4 * e4);
        const float qa[4] = {a4.x, a4.y, a4.z, a4.w}, qbv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
        for (int ee = 0; ee < 4; ++ee) {
          const float4 k4 =
              *reinterpret_cast<const float4*>(sKT + (4 * e4 + ee) * kFsMaxSeq + 4 * lane);
          sA[0] = fmaf(qa[ee], k4.x, sA[0]);
          sA[1] = fmaf(qa[ee], k4.y, sA[1]);
          sA[2] = fmaf(qa[ee], k4.z, sA[2]);
          sA[3] = fmaf(qa[ee], k4.w, sA[3]);
          sB[0] = fmaf(qbv[ee], k4.x, sB[0]);
          sB[1] = fmaf(qbv[ee], k4.y, sB[1]);
          sB[2] = fmaf(qbv[ee], k4.z, sB[2]);
          sB[3] = fmaf(qbv[ee], k4.w, sB[3]);
        }
      }
    }
    float mA = -INFINITY, mB = -INFINITY;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int j = 4 * lane + m;
      const bool live = j < keys && (vk == nullptr || vk[j] != 0);
      sA[m] = live && j < limA ? sA[m] : -INFINITY;
      sB[m] = live && j < limB ? sB[m] : -INFINITY;
      mA = fmaxf(mA, sA[m]);
      mB = fmaxf(mB, sB[m]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      mA = fmaxf(mA, __shfl_xor_sync(0xffffffffu, mA, o));
      mB = fmaxf(mB, __shfl_xor_sync(0xffffffffu, mB, o));
    }
    float lA = 0.f, lB = 0.f;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      sA[m] = sA[m] != -INFINITY ? exp2f((sA[m] - mA) * a.scale_log2) : 0.f;
      sB[m] = sB[m] != -INFINITY ? exp2f((sB[m] - mB) * a.scale_log2) : 0.f;
      lA += sA[m];
      lB += sB[m];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      lA += __shfl_xor_sync(0xffffffffu, lA, o);
      lB += __shfl_xor_sync(0xffffffffu, lB, o);
    }
    float2 oA = make_float2(0.f, 0.f), oB = make_float2(0.f, 0.f);
    const int jmax = max(limA, limB) < keys ? max(limA, limB) : keys;
    for (int src = 0; 4 * src < jmax; ++src) {
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const float pa = __shfl_sync(0xffffffffu, sA[m], src);
        const float pb = __shfl_sync(0xffffffffu, sB[m], src);
        const int j = 4 * src + m;
        if (j < jmax) {
          const float2 v = *reinterpret_cast<const float2*>(sV + j * kFsHead + 2 * lane);
          oA.x = fmaf(pa, v.x, oA.x);
          oA.y = fmaf(pa, v.y, oA.y);
          oB.x = fmaf(pb, v.x, oB.x);
          oB.y = fmaf(pb, v.y, oB.y);
        }
      }
    }
    const float iaA = lA > 0.f ? 1.f / lA : 0.f;
    const __half2 rA = __floats2half2_rn(oA.x * iaA, oA.y * iaA);
    *reinterpret_cast<__half2*>(a.ctx + (static_cast<int64_t>(b) * a.S + iA) * a.d +
                                hh * kFsHead + 2 * lane) = rA;
    if (hasB) {
      const float iaB = lB > 0.f ? 1.f / lB : 0.f;
      const __half2 rB = __floats2half2_rn(oB.x * iaB, oB.y * iaB);
      *reinterpret_cast<__half2*>(a.ctx + (static_cast<int64_t>(b) * a.S + iB) * a.d +
                                  hh * kFsHead + 2 * lane) = rB;
    }
  }
}

// Block-wide sum over the CTA's 320 threads (red: 16 floats of shared
// memory, reused after the return).
__device__ __forceinline__ float fs_block_sum(float v, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();  // red is free (its last readers are past this point)
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kFsThreads / 32; ++w) t += red[w];
  return t;
}

// Rows t of v = in[t] (+ the ks split-K partials and bias, in order kc = 0,
// 1, ...): res_out[t] = v (if given); then LayerNorm(v) * w + bb in fp32
// statistics, to h16 (16-bit) or to out32 with rows past their sequence's
// length written as zero.  A CTA per row, thread i owning columns i, i +
// 320, ... (d <= 1280).
__device__ __forceinline__ void fs_layernorm(const FsArgs& a, const float* in, const float* part,
                                             int ks, const float* bias, float* res_out,
                                             uint16_t* h16, float* out32, const float* w,
                                             const float* bb, float eps, float* red) {
  const int d = a.d;
  const float inv_d = 1.f / static_cast<float>(d);
  for (int t = blockIdx.x; t < a.T; t += gridDim.x) {
    // v = in (+ partials in order, + bias) for this thread's columns; the
    // partials of all four columns are loaded in one sweep (two chains per
    // column), so their latencies overlap.
    float v[4], v2[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int j = threadIdx.x + kFsThreads * c;
      v[c] = j < d ? in[static_cast<int64_t>(t) * d + j] : 0.f;
      v2[c] = 0.f;
    }
    if (part != nullptr) {
      const int64_t stride = static_cast<int64_t>(a.T) * d;
      const float* pp = part + static_cast<int64_t>(t) * d + threadIdx.x;
      int kc = 0;
      for (; kc + 2 <= ks; kc += 2) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (threadIdx.x + kFsThreads * c < d) {
            v[c] += __ldcg(pp + kc * stride + kFsThreads * c);
            v2[c] += __ldcg(pp + (kc + 1) * stride + kFsThreads * c);
          }
        }
      }
      if (kc < ks) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (threadIdx.x + kFsThreads * c < d) v[c] += __ldcg(pp + kc * stride + kFsThreads * c);
      }
    }
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int j = threadIdx.x + kFsThreads * c;
      if (j < d) {
        v[c] += v2[c];
        if (part != nullptr) v[c] += __ldg(bias + j);
        s += v[c];
      }
    }
    const float mean = fs_block_sum(s, red) * inv_d;
    float sq = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int j = threadIdx.x + kFsThreads * c;
      if (j < d) sq += (v[c] - mean) * (v[c] - mean);
    }
    const float rstd = rsqrtf(fs_block_sum(sq, red) * inv_d + eps);
    const bool valid = a.valid == nullptr || a.valid[t] != 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int j = threadIdx.x + kFsThreads * c;
      if (j >= d) continue;
      const int64_t at = static_cast<int64_t>(t) * d + j;
      if (res_out != nullptr) res_out[at] = v[c];
      const float y = (v[c] - mean) * rstd * __ldg(w + j) + __ldg(bb + j);
      if (h16 != nullptr)
        h16[at] = __half_as_ushort(__float2half_rn(y));
      else
        out32[at] = valid ? y : 0.f;
    }
  }
}

__global__ void __launch_bounds__(kFsThreads, 1) forward_small_kernel(const __grid_constant__ FsArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  FsShared sh;
  sh.sA = smem;
  sh.sB = smem + kFsStages * FsSmem::kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + FsSmem::kRing);
  sh.full = bars;
  sh.empty = bars + kFsStages;
  sh.tfull = sh.empty + kFsStages;
  sh.tempty = sh.tfull + 2;
  uint64_t* drain = sh.tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  sh.abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile unsigned* gen_slot = reinterpret_cast<volatile unsigned*>(tmem_slot + 2);
  float* red = reinterpret_cast<float*>(tmem_slot + 4);  // [16]
  const int warp = threadIdx.x >> 5;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFsStages; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sh.tfull[b], 1);
      mbar_init(&sh.tempty[b], 8);
    }
    mbar_init(drain, 1);
    *sh.abort_flag = 0;
    // Every CTA reads the generation before it first arrives, so none can
    // see a barrier of this launch completed already.
    *gen_slot = fs_ld_acquire_u32(a.bar + 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * kFsUnitTokens);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  sh.tmem_base = *tmem_slot;
  const unsigned gen0 = *gen_slot;
  unsigned k = 0;
  FsRing ring;
  const int d = a.d;
  float* sm = reinterpret_cast<float*>(smem);  // attention tiles reuse the idle ring

  for (int l = 0; l < a.L; ++l) {
    const FsLayer& ly = a.layer[l];
    if (threadIdx.x == 0) fs_prefetch_weights(a, &a.w_qkv[l], 3 * d, d, 1);
    if (l == 0)
      fs_layernorm(a, a.x, nullptr, 0, nullptr, a.res, a.h, nullptr, ly.ln1_w, ly.ln1_b,
                   ly.ln1_eps, red);
    else
      fs_layernorm(a, a.res, a.part, a.ks_2, a.layer[l - 1].b2, a.res, a.h, nullptr, ly.ln1_w,
                   ly.ln1_b, ly.ln1_eps, red);
    if (!fs_grid_sync(a.bar, gen0, ++k, sh.abort_flag)) goto done;
    fs_gemm(a, &a.w_qkv[l], &a.x_h, 3 * d, d, 1, ly.bqkv, 0, a.qkv, nullptr, sh, ring);
    if (!fs_grid_sync(a.bar, gen0, ++k, sh.abort_flag)) goto done;
    if (threadIdx.x == 0) fs_prefetch_weights(a, &a.w_o[l], d, d, a.ks_o);
    fs_attention(a, sm);
    if (!fs_grid_sync(a.bar, gen0, ++k, sh.abort_flag)) goto done;
    fs_gemm(a, &a.w_o[l], &a.x_ctx, d, d, a.ks_o, nullptr, 0, nullptr, a.part, sh, ring);
    if (!fs_grid_sync(a.bar, gen0, ++k, sh.abort_flag)) goto done;
    if (threadIdx.x == 0) fs_prefetch_weights(a, &a.w_1[l], a.F, d, 1);
    fs_layernorm(a, a.res, a.part, a.ks_o, ly.bo, a.res, a.h2, nullptr, ly.ln2_w, ly.ln2_b,
                 ly.ln2_eps, red);
    if (!fs_grid_sync(a.bar, gen0, ++k, sh.abort_flag)) goto done;
    if (threadIdx.x == 0) fs_prefetch_weights(a, &a.w_2[l], d, a.F, a.ks_2);
    fs_gemm(a, &a.w_1[l], &a.x_h2, a.F, d, 1, ly.b1, 1, a.hidden, nullptr, sh, ring);
    if (!fs_grid_sync(a.bar, gen0, ++k, sh.abort_flag)) goto done;
    fs_gemm(a, &a.w_2[l], &a.x_hidden, d, a.F, a.ks_2, nullptr, 0, nullptr, a.part, sh, ring);
    if (!fs_grid_sync(a.bar, gen0, ++k, sh.abort_flag)) goto done;
  }
  fs_layernorm(a, a.res, a.part, a.ks_2, a.layer[a.L - 1].b2, nullptr, nullptr, a.out, a.lnf_w,
               a.lnf_b, a.lnf_eps, red);

done:
  // After an abort: the loads this CTA's producer issued land and its MMAs
  // retire before the shared and tensor memory are released.
  if (threadIdx.x == 0) {
    for (int s = 0; s < kFsStages; ++s)
      if ((ring.issued >> s) & 1u) mbar_wait_drain(&sh.full[s], (ring.last_parity >> s) & 1u);
  }
  if (warp == 1) {
    umma_commit_w(drain);
    mbar_wait_drain(drain, 0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(sh.tmem_base, 2 * kFsUnitTokens);
  }
}

std::mutex g_fs_mu;
bool g_fs_attr_done[64];


// Workspace layout (each part 256-byte aligned): barrier words, res, h,
// qkv, ctx, h2, hidden, split-K partials.
struct FsLayout {
  size_t bar, res, h, qkv, ctx, h2, hidden, part, total;
  int ks_o, ks_2;
};

size_t fs_align(size_t v) { return (v + 255) / 256 * 256; }

// k-split of a GEMM with N output features and K: as many units as CTAs at
// most, every split non-empty.
int fs_split(int N, int K, int grid) {
  const int nt = N / 128, kb = K / 64;
  const int want = std::max(1, std::min(kb, grid / std::max(nt, 1)));
  const int kbu = (kb + want - 1) / want;
  return (kb + kbu - 1) / kbu;
}

FsLayout fs_layout(int T, int d, int F, int grid) {
  FsLayout L;
  const int Tpad = (T + 15) / 16 * 16;
  const int n_tsub = (Tpad + 127) / 128;  // token sub-blocks of a GEMM phase
  L.ks_o = fs_split(d, d, std::max(1, grid / n_tsub));
  // FFN-out: half as many units as CTAs, so the next LayerNorm adds half as
  // many partials (its loads, not the GEMM's, were the longer chain: LN1
  // 8.5 -> 7.0 us, FFN-out 5.9 -> 6.7 us at config 1).
  L.ks_2 = fs_split(d, F, std::max(1, grid / (2 * n_tsub)));
  size_t at = 0;
  auto take = [&](size_t bytes) {
    const size_t here = at;
    at += fs_align(bytes);
    return here;
  };
  const size_t t = static_cast<size_t>(T);
  L.bar = take(256);
  L.res = take(t * d * 4);
  L.h = take(t * d * 2);
  L.qkv = take(t * 3 * d * 2);
  L.ctx = take(t * d * 2);
  L.h2 = take(t * d * 2);
  L.hidden = take(t * F * 2);
  L.part = take(static_cast<size_t>(std::max(L.ks_o, L.ks_2)) * t * d * 4);
  L.total = at;
  return L;
}

}  // namespace
}  // namespace tjb

extern "C" size_t tjb_forward_small_workspace_bytes(int B, int S, int d, int F) {
  using namespace tjb;
  if (B <= 0 || S <= 0 || d <= 0 || F <= 0) return 0;
  return fs_layout(B * S, d, F, num_sms()).total;
}

extern "C" int tjb_forward_small(const tjb_small_layer* layers, int L, const float* lnf_w,
                                 const float* lnf_b, float lnf_eps, const float* x, float* out,
                                 const uint8_t* valid, int B, int S, int d, int H, int F,
                                 int causal, int dtype, void* workspace, size_t workspace_bytes,
                                 tjb_stream_t stream) {
  using namespace tjb;
  if (!layers || !lnf_w || !lnf_b || !x || !out || !workspace || L <= 0 || B <= 0 || S <= 0)
    return TJB_ERR_INVALID_ARGUMENT;
  if (dtype != TJB_F16) return TJB_ERR_UNSUPPORTED_DTYPE;
  const int T = B * S;
  if (L > kFsMaxLayers || T > kFsMaxTokens || S > kFsMaxSeq || H <= 0 || H * kFsHead != d ||
      d % 128 != 0 || F % 128 != 0 || d > 4 * kFsThreads)
    return TJB_ERR_BAD_SHAPE;
  if (!device_ok()) return TJB_ERR_NO_DEVICE;
  const int grid = num_sms();
  const FsLayout lay = fs_layout(T, d, F, grid);
  if (workspace_bytes < lay.total || !aligned16(workspace)) return TJB_ERR_INVALID_ARGUMENT;
  if (!aligned16(x) || !aligned16(out)) return TJB_ERR_BAD_ALIGNMENT;
  for (int l = 0; l < L; ++l) {
    const tjb_small_layer& ly = layers[l];
    if (!ly.wqkv || !ly.wo || !ly.w1 || !ly.w2 || !ly.bqkv || !ly.bo || !ly.b1 || !ly.b2 ||
        !ly.ln1_w || !ly.ln1_b || !ly.ln2_w || !ly.ln2_b)
      return TJB_ERR_INVALID_ARGUMENT;
    if (!aligned16(ly.wqkv) || !aligned16(ly.wo) || !aligned16(ly.w1) || !aligned16(ly.w2))
      return TJB_ERR_BAD_ALIGNMENT;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(g_fs_mu);
    if (dev < 64 && !g_fs_attr_done[dev]) {
      if (const int fs = cuda_status(cudaFuncSetAttribute(
              forward_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
              static_cast<int>(FsSmem::kBytes))))
        return fs;
      g_fs_attr_done[dev] = true;
    }
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  FsArgs a;
  memset(&a, 0, sizeof(a));
  a.H = H;
  const int Tpad = (T + 15) / 16 * 16;
  const int Tsub = Tpad < kFsUnitTokens ? Tpad : kFsUnitTokens;  // tokens per GEMM unit
  auto wmap = [&](CUtensorMap* m, const void* w, int rows, int K) {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(rows)};
    const uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
    const uint32_t box[2] = {64, 128};
    return make_tmap_16bit(m, 2, w, dims, strides, box, false);
  };
  auto xmap = [&](CUtensorMap* m, const void* p, int K) {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(T)};
    const uint64_t strides[1] = {static_cast<uint64_t>(K) * 2};
    const uint32_t box[2] = {64, static_cast<uint32_t>(Tsub)};
    return make_tmap_16bit(m, 2, p, dims, strides, box, false);
  };
  for (int l = 0; l < L; ++l) {
    const tjb_small_layer& ly = layers[l];
    int st = wmap(&a.w_qkv[l], ly.wqkv, 3 * d, d);
    if (st == TJB_OK) st = wmap(&a.w_o[l], ly.wo, d, d);
    if (st == TJB_OK) st = wmap(&a.w_1[l], ly.w1, F, d);
    if (st == TJB_OK) st = wmap(&a.w_2[l], ly.w2, d, F);
    if (st != TJB_OK) return st;
    FsLayer& fl = a.layer[l];
    fl.ln1_w = ly.ln1_w;
    fl.ln1_b = ly.ln1_b;
    fl.bqkv = ly.bqkv;
    fl.bo = ly.bo;
    fl.ln2_w = ly.ln2_w;
    fl.ln2_b = ly.ln2_b;
    fl.b1 = ly.b1;
    fl.b2 = ly.b2;
    fl.ln1_eps = ly.ln1_eps;
    fl.ln2_eps = ly.ln2_eps;
  }
  a.h = reinterpret_cast<uint16_t*>(ws + lay.h);
  a.ctx = reinterpret_cast<uint16_t*>(ws + lay.ctx);
  a.h2 = reinterpret_cast<uint16_t*>(ws + lay.h2);
  a.hidden = reinterpret_cast<uint16_t*>(ws + lay.hidden);
  int st = xmap(&a.x_h, a.h, d);
  if (st == TJB_OK) st = xmap(&a.x_ctx, a.ctx, d);
  if (st == TJB_OK) st = xmap(&a.x_h2, a.h2, d);
  if (st == TJB_OK) st = xmap(&a.x_hidden, a.hidden, F);
  if (st != TJB_OK) return st;
  a.lnf_w = lnf_w;
  a.lnf_b = lnf_b;
  a.lnf_eps = lnf_eps;
  a.x = x;
  a.out = out;
  a.valid = valid;
  a.res = reinterpret_cast<float*>(ws + lay.res);
  a.qkv = reinterpret_cast<uint16_t*>(ws + lay.qkv);
  a.part = reinterpret_cast<float*>(ws + lay.part);
  a.bar = reinterpret_cast<unsigned*>(ws + lay.bar);
  a.B = B;
  a.S = S;
  a.T = T;
  a.d = d;
  a.Tpad = Tpad;
  a.Tsub = Tsub;
  a.n_tsub = (Tpad + Tsub - 1) / Tsub;
  a.F = F;
  a.L = L;
  a.causal = causal;
  // 8-row attention units unless that makes more units than CTAs (measured
  // at config 1, 48 -> 96 units on 148 SMs: 0.254 -> 0.249 ms a forward;
  // at 256 units, 2 x 8 heads x 16 blocks of 8 rows, 0.308 -> 0.318 ms).
  a.qrows = B * H * ((S + 7) / 8) <= grid ? 8 : kFsQRows;
  a.ks_o = lay.ks_o;
  a.ks_2 = lay.ks_2;
  a.idesc = idesc_f16(128, Tsub, false, false);
  a.scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(kFsHead));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kFsThreads);
  cfg.dynamicSmemBytes = FsSmem::kBytes;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, forward_small_kernel, a));
}
