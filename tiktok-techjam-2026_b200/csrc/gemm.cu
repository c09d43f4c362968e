// gemm.cu -- C = act(A * B^T + bias) on the 5th-generation tensor cores.
//
// Persistent, warp-specialised kernel, one CTA per SM (320 threads):
//   warp 0      TMA producer: streams 128x64 A tiles and BNx64 B tiles
//               (128-byte swizzle) into a kStages-deep shared-memory ring.
//   warp 1      allocates tensor memory; one lane issues tcgen05.mma
//               (M=128, N=BN, K=16) into a double-buffered fp32 accumulator
//               in TMEM and commits stage/accumulator completion to mbarriers.
//   warps 2..9  epilogue, two warps per TMEM lane quarter splitting the
//               columns: tcgen05.ld the accumulator (one TMEM lane = one
//               output row per thread), add bias, optional erf-GELU, convert,
//               write 128-byte row pieces into a swizzled shared-memory tile
//               (one per warp) that a TMA bulk store copies to C, so the
//               global writes are whole lines; then hand the accumulator
//               buffer back to the MMA warp.  Eight warps rather than four:
//               the GELU epilogue of the FFN's first GEMM is issue-bound.
// The epilogue of tile i overlaps the main loop of tile i+1.  With a list of
// live M tiles (padding-aware forward), only those row tiles are visited.
// Output tiles are visited in groups of 16 M-blocks so the CTAs resident at
// one time share both A rows and B columns in L2.  With a caller workspace,
// GEMMs whose tiles fill the SMs badly run stream-K (see kSkMinKBlocks): each
// CTA takes an equal run of the tile-major k-block space and split tiles meet
// in the workspace.
#include <cstdlib>
#include <mutex>

#include "common.cuh"

namespace tjb {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // 64 x 16-bit = one 128-byte swizzle row
constexpr int kGroupM = 16;
constexpr int kGemmThreads = 320;

template <int BN>
struct GemmCfg {
  static constexpr int kStages = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
  static constexpr uint32_t kABytes = kBM * kBK * 2;
  static constexpr uint32_t kBBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kTmemCols = 2 * BN;  // two accumulators; 128/256/512
  // Output staging: one 32-row x 128-byte tile per epilogue warp.
  static constexpr uint32_t kOutTile = 32 * 128;
  static constexpr uint32_t kOutBytes = 8 * kOutTile;
  static constexpr size_t kSmemBytes = 1024 + kStages * kStageBytes + kOutBytes + 256;
};

struct GemmArgs {
  const float* bias;
  // Optional list of live 128-row M tiles: m_tiles[0] = count, then the
  // tile indices.  Tiles not listed are neither computed nor written.
  const int32_t* m_tiles;
  void* C;
  int M, N, K, ldc;
  int out_dtype;
  int act;
  uint32_t idesc;
  // Split-K tail workspace (null: every tile is computed whole by one CTA).
  float* ws;      // [kSkMaxPartials][kBM][256] fp32 partial tiles
  // [2][kSkMaxPartials]: per contributor slot, the arrivals of its eight
  // epilogue warps, then the owner warps done reading it; zero between launches.
  int* ws_flags;
};

// Stream-K.  When the output tiles do not fill a whole number of waves over
// the grid (at least a quarter of the CTAs would idle in the last wave), the
// k-blocks of all tiles are laid end to end (tile-major) and every CTA takes
// one contiguous run of ceil(tiles * k_blocks / grid) of them.  A run covers
// whole tiles plus at most a tail piece of one tile at its start and a head
// piece of another at its end.  The CTA holding a tile's first k-block owns
// the tile; the CTAs holding the rest of it (its piece is the first of their
// runs, so they finish it early) write fp32 partials into their own
// workspace slot and count in; the owner (whose head piece is the last of its
// run) adds them before its epilogue and returns the counts to zero.
// Measured on a B200 (fp16, 128x256 tiles): a split tile costs its owner
// ~3 us (waiting for and adding the partial), so the rebalancing pays only
// for long tiles (K = 4096 with one tile in twelve left over: 48 -> 41 us)
// and loses for K = 1024 or a last wave more than a quarter full.
constexpr int kSkMinKBlocks = 48;
// Small-M form: at most one tile per kSkSmallTiles CTAs and K of at least
// kSkSmallMinKBlocks k-blocks; each tile's k-blocks go over up to
// kSkSmallRuns runs (its owner adds up to kSkSmallRuns - 1 partials).
// Measured: M=64 N=768 K=3072 13.6 -> 12.1 us, M=128 N=1024 K=4096 17.0 ->
// 12.9 us; with eight runs, or with K = 768 (three k-blocks a run), the
// owner's additions cost more than the spread saves.
constexpr int kSkSmallTiles = 4;
constexpr int kSkSmallRuns = 4;
constexpr int kSkSmallMinKBlocks = 32;
constexpr int kSkMaxPartials = 160;  // workspace slots: one per CTA, >= grid
constexpr size_t kSkPartialBytes = static_cast<size_t>(kSkMaxPartials) * kBM * 256 * 4;

struct GemmPiece {
  int tile, kb0, kb1;  // k-blocks [kb0, kb1) of output tile `tile`
};

// This CTA's work in order: whole tiles at a stride of the grid, or the
// pieces of its stream-K run [cursor, end) of the tile-major k-block space.
struct PieceIter {
  int cursor, end, num_k, num_tiles, stride;
  bool sk;
  __device__ __forceinline__ bool next(GemmPiece& p) {
    if (!sk) {
      if (cursor >= num_tiles) return false;
      p.tile = cursor;
      p.kb0 = 0;
      p.kb1 = num_k;
      cursor += stride;
      return true;
    }
    if (cursor >= end) return false;
    p.tile = cursor / num_k;
    p.kb0 = cursor - p.tile * num_k;
    p.kb1 = min(num_k, end - p.tile * num_k);
    cursor = p.tile * num_k + p.kb1;
    return true;
  }
};

// Bounded wait until *count reaches target (acquire).
__device__ __forceinline__ bool wait_count(const int* count, int target, volatile int* abort) {
  const uint64_t t0 = globaltimer();
  for (;;) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(count) : "memory");
    if (v >= target) return true;
    if (*abort) return false;
    if (globaltimer() - t0 > kWaitTimeoutNs) {
      *abort = 1;
      record_status(TJB_ERR_DEVICE_TIMEOUT);
      return false;
    }
    __nanosleep(100);
  }
}

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& m_blk, int& n_blk) {
  const int per_group = kGroupM * num_n;
  const int group = t / per_group;
  const int first_m = group * kGroupM;
  const int gsize = min(num_m - first_m, kGroupM);
  const int r = t - group * per_group;
  m_blk = first_m + r % gsize;
  n_blk = r / gsize;
}

// Bias and activation for one 32-column slice of one row.
__device__ __forceinline__ void bias_act(const GemmArgs& a, int col0, const uint32_t (&acc)[32],
                                         float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(acc[i]);
  if (a.bias != nullptr) {
    if (col0 + 32 <= a.N) {
      const float4* b4 = reinterpret_cast<const float4*>(a.bias + col0);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 bb = __ldg(b4 + i);
        v[4 * i] += bb.x;
        v[4 * i + 1] += bb.y;
        v[4 * i + 2] += bb.z;
        v[4 * i + 3] += bb.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (col0 + i < a.N) v[i] += __ldg(a.bias + col0 + i);
    }
  }
  if (a.act == 1) {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = gelu_erf(v[i]);
  }
}

// One 128-byte row piece (8 x 16 bytes) into a 128-byte-swizzled staging
// tile: 16-byte chunk k of row r lands at position k ^ (r & 7).
__device__ __forceinline__ void stage_row(uint8_t* tile, int r, const uint32_t (&w)[32]) {
  uint4* row = reinterpret_cast<uint4*>(tile + r * 128);
#pragma unroll
  for (int k = 0; k < 8; ++k)
    row[k ^ (r & 7)] = make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
}

// Producer role (one thread): TMA-loads the A and B k-blocks of every piece
// `next` yields into the stage ring; `coords(tile, m_blk, n_blk)` maps a
// piece's tile to its 128-row block of A and BN-row block of B.  Waits for
// every load it issued before returning (the CTA may then release memory).
template <int BN, int kStages = GemmCfg<BN>::kStages, class Next, class Coords>
__device__ __forceinline__ void gemm_produce(Next next, Coords coords, const CUtensorMap* tmA,
                                             const CUtensorMap* tmB, uint8_t* sA, uint8_t* sB,
                                             uint64_t* full, uint64_t* empty,
                                             volatile int* abort_flag) {
  using Cfg = GemmCfg<BN>;
  int stage = 0;
  uint32_t phase = 0, issued = 0, issued_parity = 0;
  bool ok = true;
  GemmPiece un;
  while (ok && next(un)) {
    int m_blk, n_blk;
    coords(un.tile, m_blk, n_blk);
    for (int kb = un.kb0; kb < un.kb1; ++kb) {
      if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
        ok = false;
        break;
      }
      mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
      tma_load_2d(sA + stage * Cfg::kABytes, tmA, &full[stage], kb * kBK, m_blk * kBM);
      tma_load_2d(sB + stage * Cfg::kBBytes, tmB, &full[stage], kb * kBK, n_blk * BN);
      issued |= 1u << stage;
      issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
      if (++stage == kStages) {
        stage = 0;
        phase ^= 1;
      }
    }
  }
  for (int s = 0; s < kStages; ++s)
    if ((issued >> s) & 1u) mbar_wait_drain(&full[s], (issued_parity >> s) & 1u);
}

// MMA role (one whole warp, converged; one elected lane issues): for every
// piece `next` yields, accumulate its k-blocks into one of the two TMEM
// accumulators (BN columns each) and signal tfull; waits for tempty before
// reusing an accumulator.  Retires every MMA before returning.
template <int BN, int kStages = GemmCfg<BN>::kStages, class Next>
__device__ __forceinline__ void gemm_mma(Next next, uint32_t tmem_base, uint8_t* sA, uint8_t* sB,
                                         uint64_t* full, uint64_t* empty, uint64_t* tfull,
                                         uint64_t* tempty, uint64_t* drain, uint32_t idesc,
                                         volatile int* abort_flag) {
  using Cfg = GemmCfg<BN>;
  int stage = 0, acc = 0;
  uint32_t phase = 0, acc_phase = 0;
  bool ok = true;
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
  };
  GemmPiece un;
  while (ok && next(un)) {
    if (!wait(&tempty[acc], acc_phase ^ 1)) break;
    tc_fence_after();
    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
    for (int kb = un.kb0; kb < un.kb1; ++kb) {
      if (!wait(&full[stage], phase)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t a0 = smem_u32(sA + stage * Cfg::kABytes);
      const uint32_t b0 = smem_u32(sB + stage * Cfg::kBBytes);
#pragma unroll
      for (int k = 0; k < kBK / 16; ++k) {
        umma_ss_w(d_tmem, sdesc_sw128(a0 + k * 32, 16, 1024), sdesc_sw128(b0 + k * 32, 16, 1024),
                  idesc, (kb > un.kb0 || k > 0) ? 1u : 0u);
      }
      umma_commit_w(&empty[stage]);
      if (++stage == kStages) {
        stage = 0;
        phase ^= 1;
      }
    }
    if (!ok) break;
    umma_commit_w(&tfull[acc]);
    if (++acc == 2) {
      acc = 0;
      acc_phase ^= 1;
    }
  }
  umma_commit_w(drain);
  mbar_wait_drain(drain, 0);
}

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, const GemmArgs args) {
  using Cfg = GemmCfg<BN>;
  constexpr int kStages = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * Cfg::kABytes;
  uint8_t* sOut = sB + kStages * Cfg::kBBytes;  // [epilogue warp][kOutTile]
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + Cfg::kOutBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 8);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmC);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  // The weights are never written by the kernels this launch overlaps:
  // pull the first k-blocks of this CTA's first B tile into L2 while the
  // previous kernel drains (its tile as the full M would place it).
  if (warp == 0 && lane == 0) {
    int m_blk, n_blk;
    tile_coords(static_cast<int>(blockIdx.x), (args.M + kBM - 1) / kBM, (args.N + BN - 1) / BN,
                m_blk, n_blk);
    for (int kb = 0; kb < Cfg::kStages && kb * kBK < args.K; ++kb)
      tma_prefetch_2d(&tmB, kb * kBK, n_blk * BN);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();
  griddep_launch_dependents();
  const int num_m = args.m_tiles != nullptr ? __ldg(args.m_tiles) : (args.M + kBM - 1) / kBM;
  const int num_n = (args.N + BN - 1) / BN;
  const int num_k = (args.K + kBK - 1) / kBK;
  const int num_tiles = num_m * num_n;
  const int grid = static_cast<int>(gridDim.x);
  bool sk = false;
  int sk_w = 0;  // k-blocks per CTA run
  if (args.ws != nullptr && grid <= kSkMaxPartials) {
    const int rem = num_tiles % grid;
    if (num_k >= kSkMinKBlocks && rem != 0 && 4 * (grid - rem) >= 3 * grid &&
        2 * num_tiles >= grid && num_tiles < 2 * grid) {
      // A last wave at most a quarter full, at most two waves (beyond that
      // the idle tail is a small share and every split costs; config 4's
      // 11-wave GEMMs ran 28% slower with it), and at least half a tile per
      // CTA (so a tile is split over at most three runs).
      sk = true;
      sk_w = (num_tiles * num_k + grid - 1) / grid;
    } else if (kSkSmallTiles * num_tiles <= grid && num_k >= kSkSmallMinKBlocks) {
      // Few tiles (small M): spread each tile's k-blocks over up to
      // kSkSmallRuns CTAs, so that many SMs stream the weights at once.
      sk = true;
      sk_w = max((num_tiles * num_k + grid - 1) / grid, (num_k + kSkSmallRuns - 1) / kSkSmallRuns);
    }
  }
  auto pieces = [&]() {
    PieceIter it;
    it.num_k = num_k;
    it.num_tiles = num_tiles;
    it.stride = grid;
    it.sk = sk;
    it.cursor = sk ? static_cast<int>(blockIdx.x) * sk_w : static_cast<int>(blockIdx.x);
    it.end = sk ? min((static_cast<int>(blockIdx.x) + 1) * sk_w, num_tiles * num_k) : 0;
    return it;
  };

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      PieceIter it = pieces();
      gemm_produce<BN>([&](GemmPiece& un) { return it.next(un); },
                       [&](int tile, int& m_blk, int& n_blk) {
                         tile_coords(tile, num_m, num_n, m_blk, n_blk);
                         if (args.m_tiles != nullptr) m_blk = __ldg(args.m_tiles + 1 + m_blk);
                       },
                       &tmA, &tmB, sA, sB, full, empty, abort_flag);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    PieceIter it = pieces();
    gemm_mma<BN>([&](GemmPiece& un) { return it.next(un); }, tmem_base, sA, sB, full, empty,
                 tfull, tempty, drain, args.idesc, abort_flag);
  } else {
    // -------------------------------------------------------------- epilogue
    const int quad = warp & 3;         // TMEM lanes this warp may access
    const int half = (warp - 2) >> 2;  // which of the quarter's two warps
    uint8_t* buf = sOut + (warp - 2) * Cfg::kOutTile;
    int acc = 0;
    uint32_t acc_phase = 0;
    PieceIter it = pieces();
    GemmPiece un;
    while (it.next(un)) {
      int m_blk, n_blk;
      tile_coords(un.tile, num_m, num_n, m_blk, n_blk);
      if (args.m_tiles != nullptr) m_blk = __ldg(args.m_tiles + 1 + m_blk);
      bool ok = mbar_wait(&tfull[acc], acc_phase, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const int row0 = m_blk * kBM + quad * 32;
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
      // Stream-K roles: a piece that starts past k-block 0 is a contributor
      // (it writes this CTA's partial slot); a piece that starts at 0 but
      // stops short of the end is the owner, and CTAs blockIdx.x + 1 ..
      // c_last hold the rest of its tile.
      const bool contributor = un.kb0 > 0;
      const bool owner = un.kb0 == 0 && un.kb1 < num_k;
      const int c_last = owner ? ((un.tile + 1) * num_k - 1) / sk_w : 0;
      // Partial slots are column-major ([slot][column][row], fp32), so one
      // warp-wide access of column j touches 32 consecutive rows = one
      // 128-byte line.  This thread's element of column j in slot p:
      auto partial_at = [&](int p, int j) {
        return args.ws + (static_cast<int64_t>(p) * 256 + j) * kBM + quad * 32 + lane;
      };
      if (contributor) {
        // ------------------------------------ stream-K contributor: fp32 partial
#pragma unroll 1
        for (int c = half; c < BN / 32; c += 2) {
          uint32_t r[32];
          tmem_ld32(taddr + c * 32, r);
          tmem_ld_wait(r);
#pragma unroll
          for (int i = 0; i < 32; ++i) __stcg(partial_at(blockIdx.x, c * 32 + i), __uint_as_float(r[i]));
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(args.ws_flags + blockIdx.x, 1);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
        continue;
      }
      if (owner) {
        // Each contributor's eight epilogue warps have counted in.
        if (lane == 0)
          for (int c = blockIdx.x + 1; c <= c_last; ++c) wait_count(args.ws_flags + c, 8, abort_flag);
        __syncwarp();
      }
      // Adds the contributors' partials for tile columns [c0, c0 + 32).
      auto add_partials = [&](uint32_t (&r)[32], int c0) {
        for (int p = blockIdx.x + 1; p <= c_last; ++p) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            r[i] = __float_as_uint(__uint_as_float(r[i]) + __ldcg(partial_at(p, c0 + i)));
        }
      };
      // One staged 32-row x 128-byte piece: wait until the store that last
      // read this buffer is done, write it, hand it to TMA.
      auto emit = [&](const uint32_t (&w)[32], int col) {
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
        stage_row(buf, lane, w);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmC, buf, col, row0);
          bulk_commit();
        }
      };
      if (args.out_dtype == TJB_F32) {
#pragma unroll 1
        for (int c = half; c < BN / 32; c += 2) {
          uint32_t r[32];
          tmem_ld32(taddr + c * 32, r);
          tmem_ld_wait(r);
          const int col0 = n_blk * BN + c * 32;
          if (col0 >= args.N) break;
          if (owner) add_partials(r, c * 32);
          float v[32];
          bias_act(args, col0, r, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(v[i]);
          emit(r, col0);
        }
      } else {
#pragma unroll 1
        for (int c = half; c < BN / 64; c += 2) {
          const int col0 = n_blk * BN + c * 64;
          uint32_t w[32];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            uint32_t r[32];
            tmem_ld32(taddr + c * 64 + hh * 32, r);
            tmem_ld_wait(r);
            if (owner) add_partials(r, c * 64 + hh * 32);
            float v[32];
            bias_act(args, col0 + hh * 32, r, v);
            if (args.out_dtype == TJB_BF16) {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                w[hh * 16 + i] = Pack2<__nv_bfloat16>::pack(v[2 * i], v[2 * i + 1]);
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                w[hh * 16 + i] = Pack2<__half>::pack(v[2 * i], v[2 * i + 1]);
            }
          }
          if (col0 >= args.N) break;
          emit(w, col0);
        }
      }
      if (owner) {
        // This warp has read its share of every partial.  The last of the
        // owner's eight warps to get here zeroes the slot's counters: every
        // owner warp has passed its wait by then, so none can miss the
        // arrivals (returning them one warp at a time could hide them from a
        // warp still waiting).
        __syncwarp();
        if (lane == 0)
          for (int c = blockIdx.x + 1; c <= c_last; ++c)
            if (atomicAdd(args.ws_flags + kSkMaxPartials + c, 1) == 7) {
              atomicExch(args.ws_flags + c, 0);
              atomicExch(args.ws_flags + kSkMaxPartials + c, 0);
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
    // Every bulk store has completed before the CTA exits.
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}

// ------------------------------------------------------------------------
// CTA-pair form (tcgen05 cta_group::2): a cluster of two CTAs computes one
// 256 x 256 output tile.  CTA r of the pair TMA-loads its own 128 rows of A
// (the pair's 128-row tile 2p + r) and its own 128 rows of B (output
// columns n*256 + 128r ..), each into its own shared memory, and both loads
// count on the leader's stage barrier; the leader (rank 0) issues M=256,
// N=256 MMAs that read both CTAs' tiles, and commits the stage release and
// the accumulator-ready signal to both CTAs' barriers at once.  Each CTA's
// tensor memory holds its own 128 rows x 256 columns, and its eight epilogue
// warps store them exactly as the single-CTA kernel does, then count in on
// the leader's accumulator-free barrier.  Per k-block a CTA loads 32 KB
// instead of 48 KB for the same tensor work, a third less L2 -> shared
// traffic, and its ring holds six stages.  No load is multicast.
constexpr int kPairStages = 6;

struct GemmPairCfg {
  static constexpr uint32_t kABytes = kBM * kBK * 2;   // 128 rows of A
  static constexpr uint32_t kBBytes = 128 * kBK * 2;   // this CTA's 128 rows of B
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kTmemCols = 512;           // two 256-column accumulators
  static constexpr uint32_t kOutTile = 32 * 128;
  static constexpr uint32_t kOutBytes = 8 * kOutTile;
  static constexpr size_t kSmemBytes = 1024 + kPairStages * kStageBytes + kOutBytes + 256;
};

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const GemmArgs args) {
  using Cfg = GemmPairCfg;
  constexpr int kStages = kPairStages;
  constexpr int BN = 256;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * Cfg::kABytes;
  uint8_t* sOut = sB + kStages * Cfg::kBBytes;  // [epilogue warp][kOutTile]
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + Cfg::kOutBytes);  // leader's are used
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;  // leader's are used
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: the leader, which issues the MMAs

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);   // the leader's expect-tx arrival + both CTAs' bytes
      mbar_init(&empty[s], 1);  // one multicast commit of the leader's MMAs
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 16);  // eight epilogue warps of each CTA
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmC);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  // This CTA's half of the first B tile, first k-blocks, into L2 before the
  // wait (weights are never written by the kernels this launch overlaps).
  if (warp == 0 && lane == 0) {
    int mp, n_blk;
    tile_coords(static_cast<int>(blockIdx.x >> 1), ((args.M + kBM - 1) / kBM + 1) / 2,
                (args.N + BN - 1) / BN, mp, n_blk);
    for (int kb = 0; kb < kStages && kb * kBK < args.K; ++kb)
      tma_prefetch_2d(&tmB, kb * kBK, n_blk * BN + static_cast<int>(rank) * 128);
  }
  // Both CTAs' barriers are initialised and their tensor memory allocated
  // before either signals the other.
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();
  griddep_launch_dependents();
  const int num_m = args.m_tiles != nullptr ? __ldg(args.m_tiles) : (args.M + kBM - 1) / kBM;
  const int num_mp = (num_m + 1) / 2;
  const int num_n = (args.N + BN - 1) / BN;
  const int num_k = (args.K + kBK - 1) / kBK;
  const int num_tiles = num_mp * num_n;
  const int pair_id = static_cast<int>(blockIdx.x >> 1);
  const int num_pairs = static_cast<int>(gridDim.x >> 1);
  // This CTA's 128-row tile of pair tile (mp, .): 2 mp + rank.  A pair whose
  // second tile does not exist loads the first one's rows again (the MMA
  // needs both halves) and the peer stores nothing.
  auto rows_of = [&](int mp, int& m_blk) {
    int mt = 2 * mp + static_cast<int>(rank);
    const bool has = mt < num_m;
    if (!has) mt = 2 * mp;
    m_blk = args.m_tiles != nullptr ? __ldg(args.m_tiles + 1 + mt) : mt;
    return has;
  };
  // Stream-K over pair tiles (see kSkMinKBlocks), with each CTA of a pair
  // writing its own 128 rows of a split tile's partial into its own slot.
  bool sk = false;
  int sk_w = 0;  // k-blocks per pair's run
  if (args.ws != nullptr && static_cast<int>(gridDim.x) <= kSkMaxPartials) {
    const int rem = num_tiles % num_pairs;
    if (num_k >= kSkMinKBlocks && rem != 0 && 4 * (num_pairs - rem) >= 3 * num_pairs &&
        2 * num_tiles >= num_pairs && num_tiles < 2 * num_pairs) {
      sk = true;
      sk_w = (num_tiles * num_k + num_pairs - 1) / num_pairs;
    }
  }
  auto pieces = [&]() {
    PieceIter it;
    it.num_k = num_k;
    it.num_tiles = num_tiles;
    it.stride = num_pairs;
    it.sk = sk;
    it.cursor = sk ? pair_id * sk_w : pair_id;
    it.end = sk ? min((pair_id + 1) * sk_w, num_tiles * num_k) : 0;
    return it;
  };

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ producer
      const uint32_t full_leader = map_to_rank(smem_u32(full), 0);
      int stage = 0;
      uint32_t phase = 0, issued = 0, last_parity = 0;
      bool ok = true;
      PieceIter pit = pieces();
      GemmPiece un;
      while (ok && pit.next(un)) {
        int mp, n_blk, m_blk;
        tile_coords(un.tile, num_mp, num_n, mp, n_blk);
        rows_of(mp, m_blk);
        for (int kb = un.kb0; kb < un.kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::kStageBytes);
          const uint32_t bar = full_leader + static_cast<uint32_t>(stage) * 8u;
          tma_load_2d_pair(sA + stage * Cfg::kABytes, &tmA, bar, kb * kBK, m_blk * kBM);
          tma_load_2d_pair(sB + stage * Cfg::kBBytes, &tmB, bar, kb * kBK,
                           n_blk * BN + static_cast<int>(rank) * 128);
          issued |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Every load this CTA issued has landed once the MMAs that read it
      // have released its stage (the loads count on the leader's barrier).
      for (int s = 0; s < kStages; ++s)
        if ((issued >> s) & 1u) mbar_wait_drain(&empty[s], (last_parity >> s) & 1u);
    }
  } else if (warp == 1) {
    if (rank == 0) {
      // ---------------------------------------------- MMA issuer (leader only)
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort_flag));
      };
      PieceIter pit = pieces();
      GemmPiece un;
      while (ok && pit.next(un)) {
        if (!wait(&tempty[acc], acc_phase ^ 1)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = un.kb0; kb < un.kb1; ++kb) {
          if (!wait(&full[stage], phase)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sA + stage * Cfg::kABytes);
          const uint32_t b0 = smem_u32(sB + stage * Cfg::kBBytes);
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_ss_pair_w(d_tmem, sdesc_sw128(a0 + k * 32, 16, 1024),
                           sdesc_sw128(b0 + k * 32, 16, 1024), args.idesc,
                           (kb > un.kb0 || k > 0) ? 1u : 0u);
          umma_commit_pair_w(&empty[stage], 0x3);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair_w(&tfull[acc], 0x3);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      umma_commit_pair_w(drain, 0x1);
      mbar_wait_drain(drain, 0);
    }
  } else {
    // -------------------------------------------------------------- epilogue
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    uint8_t* buf = sOut + (warp - 2) * Cfg::kOutTile;
    const uint32_t tempty_leader = map_to_rank(smem_u32(tempty), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    PieceIter pit = pieces();
    GemmPiece un;
    while (pit.next(un)) {
      int mp, n_blk, m_blk;
      tile_coords(un.tile, num_mp, num_n, mp, n_blk);
      const bool has_rows = rows_of(mp, m_blk);
      bool ok = mbar_wait(&tfull[acc], acc_phase, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const int row0 = m_blk * kBM + quad * 32;
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);
      // Stream-K roles as in the single-CTA kernel, per pair: a piece that
      // starts past k-block 0 is a contributor, one that starts at 0 and
      // stops short of the end the owner; pairs pair_id + 1 .. c_last hold
      // the rest of the owner's tile, and CTA r of the owner reads the slot
      // of CTA r of each of them (blockIdx 2p + r: the same 128 rows).
      const bool contributor = un.kb0 > 0;
      const bool owner = un.kb0 == 0 && un.kb1 < num_k;
      const int c_last = owner ? ((un.tile + 1) * num_k - 1) / sk_w : 0;
      auto partial_at = [&](int p, int j) {
        return args.ws + (static_cast<int64_t>(p) * 256 + j) * kBM + quad * 32 + lane;
      };
      if (contributor) {
#pragma unroll 1
        for (int c = half; c < BN / 32; c += 2) {
          uint32_t r[32];
          tmem_ld32(taddr + c * 32, r);
          tmem_ld_wait(r);
#pragma unroll
          for (int i = 0; i < 32; ++i)
            __stcg(partial_at(blockIdx.x, c * 32 + i), __uint_as_float(r[i]));
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(args.ws_flags + blockIdx.x, 1);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(tempty_leader + static_cast<uint32_t>(acc) * 8u);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
        continue;
      }
      if (owner) {
        // Each contributor CTA's eight epilogue warps have counted in.
        if (lane == 0)
          for (int p = pair_id + 1; p <= c_last; ++p)
            wait_count(args.ws_flags + 2 * p + static_cast<int>(rank), 8, abort_flag);
        __syncwarp();
      }
      auto add_partials = [&](uint32_t (&r)[32], int c0) {
        for (int p = pair_id + 1; p <= c_last; ++p) {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            r[i] = __float_as_uint(__uint_as_float(r[i]) +
                                   __ldcg(partial_at(2 * p + static_cast<int>(rank), c0 + i)));
        }
      };
      auto emit = [&](const uint32_t (&w)[32], int col) {
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
        stage_row(buf, lane, w);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmC, buf, col, row0);
          bulk_commit();
        }
      };
      if (has_rows && args.out_dtype == TJB_F32) {
#pragma unroll 1
        for (int c = half; c < BN / 32; c += 2) {
          uint32_t r[32];
          tmem_ld32(taddr + c * 32, r);
          tmem_ld_wait(r);
          const int col0 = n_blk * BN + c * 32;
          if (col0 >= args.N) break;
          if (owner) add_partials(r, c * 32);
          float v[32];
          bias_act(args, col0, r, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(v[i]);
          emit(r, col0);
        }
      } else if (has_rows) {
#pragma unroll 1
        for (int c = half; c < BN / 64; c += 2) {
          const int col0 = n_blk * BN + c * 64;
          if (col0 >= args.N) break;
          uint32_t w[32];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            uint32_t r[32];
            tmem_ld32(taddr + c * 64 + hh * 32, r);
            tmem_ld_wait(r);
            if (owner) add_partials(r, c * 64 + hh * 32);
            float v[32];
            bias_act(args, col0 + hh * 32, r, v);
            if (args.out_dtype == TJB_BF16) {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                w[hh * 16 + i] = Pack2<__nv_bfloat16>::pack(v[2 * i], v[2 * i + 1]);
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                w[hh * 16 + i] = Pack2<__half>::pack(v[2 * i], v[2 * i + 1]);
            }
          }
          emit(w, col0);
        }
      }
      if (owner) {
        // The last of this CTA's eight warps to have read every partial
        // returns the contributors' counters to zero (see gemm_kernel).
        __syncwarp();
        if (lane == 0)
          for (int p = pair_id + 1; p <= c_last; ++p) {
            const int slot = 2 * p + static_cast<int>(rank);
            if (atomicAdd(args.ws_flags + kSkMaxPartials + slot, 1) == 7) {
              atomicExch(args.ws_flags + slot, 0);
              atomicExch(args.ws_flags + kSkMaxPartials + slot, 0);
            }
          }
      }
      // This warp is done reading the accumulator: count in on the leader.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader + static_cast<uint32_t>(acc) * 8u);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  // Neither CTA releases its tensor memory (or exits) while the leader's
  // MMAs or the peer's epilogue may still touch the pair's resources.
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }
}

std::mutex g_pair_mu;
int g_pair_clusters[64] = {0};  // co-resident CTA pairs per device (0: not yet known)

int launch_gemm_pair(const void* A, const void* B, const GemmArgs& args, int lda, int ldb,
                     bool bf16, cudaStream_t stream) {
  using Cfg = GemmPairCfg;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return TJB_ERR_NO_DEVICE;
  int max_pairs = 0;
  {
    std::lock_guard<std::mutex> lock(g_pair_mu);
    if (g_pair_clusters[dev] == 0) {
      if (const int fs = cuda_status(cudaFuncSetAttribute(
              gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
              static_cast<int>(Cfg::kSmemBytes))))
        return fs;
      // How many pairs fit at once (an SM pairs only within its cluster
      // group, so this can be below half the SM count).
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * (num_sms() / 2));
      cfg.blockDim = dim3(kGemmThreads);
      cfg.dynamicSmemBytes = Cfg::kSmemBytes;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (const int qs = cuda_status(cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel, &cfg)))
        return qs;
      g_pair_clusters[dev] = n > 0 ? n : -1;
    }
    max_pairs = g_pair_clusters[dev];
  }
  if (max_pairs <= 0) return TJB_ERR_LAUNCH;
  CUtensorMap tmA, tmB;
  const uint64_t dimA[2] = {static_cast<uint64_t>(args.K), static_cast<uint64_t>(args.M)};
  const uint64_t strA[1] = {static_cast<uint64_t>(lda) * 2};
  const uint32_t boxA[2] = {kBK, kBM};
  const uint64_t dimB[2] = {static_cast<uint64_t>(args.K), static_cast<uint64_t>(args.N)};
  const uint64_t strB[1] = {static_cast<uint64_t>(ldb) * 2};
  const uint32_t boxB[2] = {kBK, 128};
  int st = make_tmap_16bit(&tmA, 2, A, dimA, strA, boxA, bf16);
  if (st != TJB_OK) return st;
  st = make_tmap_16bit(&tmB, 2, B, dimB, strB, boxB, bf16);
  if (st != TJB_OK) return st;
  const int esz = args.out_dtype == TJB_F32 ? 4 : 2;
  CUtensorMap tmC;
  st = make_tmap_2d(&tmC, args.out_dtype, args.C, static_cast<uint64_t>(args.N),
                    static_cast<uint64_t>(args.M), static_cast<uint64_t>(args.ldc) * esz,
                    static_cast<uint32_t>(128 / esz), 32);
  if (st != TJB_OK) return st;
  const int num_m = (args.M + kBM - 1) / kBM;
  const int pair_tiles = ((num_m + 1) / 2) * ((args.N + 255) / 256);
  const int pairs = pair_tiles < max_pairs ? pair_tiles : max_pairs;
  return launch_kernel_cluster(gemm_pair_kernel, dim3(2 * pairs), dim3(kGemmThreads),
                               Cfg::kSmemBytes, stream, 2u, tmA, tmB, tmC, args);
}

// CTA pairs: TJB_GEMM_PAIR=0 keeps every GEMM on single CTAs and =1 uses
// pairs wherever they apply (both for comparisons); unset, the tile choice
// below decides.
int pair_gemm_mode() {
  const char* v = std::getenv("TJB_GEMM_PAIR");
  if (v == nullptr || v[0] == '\0') return -1;
  return v[0] == '0' ? 0 : 1;
}

std::mutex g_attr_mu;
bool g_attr_done[64][3];

template <int BN>
int launch_gemm(const void* A, const void* B, const GemmArgs& args, int lda, int ldb, bool bf16,
                cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  int dev = 0;
  cudaGetDevice(&dev);
  const int slot = BN == 256 ? 0 : (BN == 128 ? 1 : 2);
  {
    std::lock_guard<std::mutex> lock(g_attr_mu);
    if (dev < 64 && !g_attr_done[dev][slot]) {
      if (const int fs = cuda_status(cudaFuncSetAttribute(gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(Cfg::kSmemBytes))))
        return fs;
      g_attr_done[dev][slot] = true;
    }
  }
  CUtensorMap tmA, tmB;
  const uint64_t dimA[2] = {static_cast<uint64_t>(args.K), static_cast<uint64_t>(args.M)};
  const uint64_t strA[1] = {static_cast<uint64_t>(lda) * 2};
  const uint32_t boxA[2] = {kBK, kBM};
  const uint64_t dimB[2] = {static_cast<uint64_t>(args.K), static_cast<uint64_t>(args.N)};
  const uint64_t strB[1] = {static_cast<uint64_t>(ldb) * 2};
  const uint32_t boxB[2] = {kBK, static_cast<uint32_t>(BN)};
  int st = make_tmap_16bit(&tmA, 2, A, dimA, strA, boxA, bf16);
  if (st != TJB_OK) return st;
  st = make_tmap_16bit(&tmB, 2, B, dimB, strB, boxB, bf16);
  if (st != TJB_OK) return st;
  // Output: 128-byte boxes of 32 rows (32 fp32 or 64 16-bit columns).
  const int esz = args.out_dtype == TJB_F32 ? 4 : 2;
  CUtensorMap tmC;
  st = make_tmap_2d(&tmC, args.out_dtype, args.C, static_cast<uint64_t>(args.N),
                    static_cast<uint64_t>(args.M), static_cast<uint64_t>(args.ldc) * esz,
                    static_cast<uint32_t>(128 / esz), 32);
  if (st != TJB_OK) return st;
  const int num_tiles = ((args.M + kBM - 1) / kBM) * ((args.N + BN - 1) / BN);
  int grid = num_tiles < num_sms() ? num_tiles : num_sms();
  // Few tiles with a stream-K workspace: launch a CTA per SM (up to the
  // workspace's slots) so the kernel can spread the k-blocks.
  if (args.ws != nullptr && kSkSmallTiles * num_tiles <= num_sms() &&
      (args.K + kBK - 1) / kBK >= kSkSmallMinKBlocks)
    grid = num_sms() < kSkMaxPartials ? num_sms() : kSkMaxPartials;
  return launch_kernel(gemm_kernel<BN>, dim3(grid), dim3(kGemmThreads), Cfg::kSmemBytes, stream,
                       tmA, tmB, tmC, args);
}

}  // namespace
}  // namespace tjb

namespace tjb {
namespace {
int gemm_impl(const void* A, const void* B, const float* bias, void* C, int M, int N, int K,
              int lda, int ldb, int ldc, int in_dtype, int out_dtype, int act,
              const int32_t* m_tiles, void* workspace, size_t workspace_bytes,
              tjb_stream_t stream) {
  if (!A || !B || !C || M < 0 || N <= 0 || K <= 0) return TJB_ERR_INVALID_ARGUMENT;
  if (workspace != nullptr &&
      (workspace_bytes < tjb_gemm_workspace_bytes() || !aligned16(workspace)))
    return TJB_ERR_INVALID_ARGUMENT;
  if (in_dtype != TJB_F16 && in_dtype != TJB_BF16) return TJB_ERR_UNSUPPORTED_DTYPE;
  if (out_dtype != TJB_F32 && out_dtype != in_dtype) return TJB_ERR_UNSUPPORTED_DTYPE;
  if (act != 0 && act != 1) return TJB_ERR_INVALID_ARGUMENT;
  if (K % 8 != 0 || N % 8 != 0 || lda < K || ldb < K || ldc < N) return TJB_ERR_BAD_SHAPE;
  if (lda % 8 != 0 || ldb % 8 != 0 || ldc % 8 != 0) return TJB_ERR_BAD_ALIGNMENT;
  if (!aligned16(A) || !aligned16(B) || !aligned16(C) || (bias && !aligned16(bias)))
    return TJB_ERR_BAD_ALIGNMENT;
  if (!device_ok()) return TJB_ERR_NO_DEVICE;
  if (M == 0) return TJB_OK;
  const bool bf16 = in_dtype == TJB_BF16;
  GemmArgs args;
  args.bias = bias;
  args.m_tiles = m_tiles;
  args.C = C;
  args.M = M;
  args.N = N;
  args.K = K;
  args.ldc = ldc;
  args.out_dtype = out_dtype;
  args.act = act;
  args.ws = static_cast<float*>(workspace);
  args.ws_flags = workspace == nullptr
                      ? nullptr
                      : reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + kSkPartialBytes);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int sms = num_sms();
  // Tile width: the fewest waves weighted by each width's time per tile
  // relative to a 256-wide one (fitted to a B200 sweep of M 4608-15104,
  // N 1024-4096, K 1024-4096: 0.65 for 128-wide, 0.5 for 64-wide).  With a
  // live-tile list the listed count is not known on the host, so M is taken
  // as given.
  // With a stream-K workspace a partial last wave costs only its share of the
  // k-blocks, so the widest (most efficient) tile wins whenever the kernel
  // can use stream-K (long K, at least half a 256-wide tile per SM; with a
  // live-tile list M is an upper bound and the kernel decides again).
  const long mt = (M + kBM - 1) / kBM;
  auto waves = [&](int bn) { return (mt * ((N + bn - 1) / bn) + sms - 1) / sms; };
  const int pair_mode = pair_gemm_mode();
  // Stream-K on CTA pairs where the pair tiles make one to two waves over
  // the pairs: the pair tile's lighter operand traffic and the balanced
  // k-block runs together (the kernel decides again from the live tiles).
  const long sk_pair_tiles = ((mt + 1) / 2) * ((N + 255) / 256);
  const long sk_pairs = sms / 2 > 0 ? sms / 2 : 1;
  if (workspace != nullptr && pair_mode != 0 && mt >= 2 && N >= 256 &&
      (K + kBK - 1) / kBK >= kSkMinKBlocks && 2 * sk_pair_tiles >= sk_pairs &&
      sk_pair_tiles < 2 * sk_pairs) {
    args.idesc = idesc_f16(2 * kBM, 256, bf16, false);
    return launch_gemm_pair(A, B, args, lda, ldb, bf16, s);
  }
  if (workspace != nullptr && N >= 256 && (K + kBK - 1) / kBK >= kSkMinKBlocks &&
      2 * mt * ((N + 255) / 256) >= sms && mt * ((N + 255) / 256) < 2 * sms) {
    args.idesc = idesc_f16(kBM, 256, bf16, false);
    return launch_gemm<256>(A, B, args, lda, ldb, bf16, s);
  }
  if (pair_mode == 1 && N >= 256 && mt >= 2) {
    args.idesc = idesc_f16(2 * kBM, 256, bf16, false);
    return launch_gemm_pair(A, B, args, lda, ldb, bf16, s);
  }
  // CTA pairs: waves of 256 x 256 pair tiles over half the SMs, each pair
  // tile costing 0.9 of a single-CTA 128 x 256 tile (measured on B200 at the
  // configs' shapes: M5504 N3072 K1024 36.9 vs 40.0 us, M5504 N1024 K1024
  // 25.6 vs 28.6 us against the 128-wide tile this model picked before).
  const bool pair_ok = mt >= 2 && N >= 256 && pair_mode != 0;
  const long pair_tiles = ((mt + 1) / 2) * ((N + 255) / 256);
  const long pair_slots = sms / 2 > 0 ? sms / 2 : 1;
  const double cpair = pair_ok ? ((pair_tiles + pair_slots - 1) / pair_slots) * 0.9 : 1e30;
  const double c256 = N >= 256 ? static_cast<double>(waves(256)) : 1e30;
  const double c128 = N >= 128 ? waves(128) * 0.65 : 1e30;
  const double c64 = waves(64) * 0.5;
  if (cpair <= c256 && cpair <= c128 && cpair <= c64) {
    args.idesc = idesc_f16(2 * kBM, 256, bf16, false);
    return launch_gemm_pair(A, B, args, lda, ldb, bf16, s);
  }
  if (c256 <= c128 && c256 <= c64) {
    args.idesc = idesc_f16(kBM, 256, bf16, false);
    return launch_gemm<256>(A, B, args, lda, ldb, bf16, s);
  }
  if (c128 <= c64) {
    args.idesc = idesc_f16(kBM, 128, bf16, false);
    return launch_gemm<128>(A, B, args, lda, ldb, bf16, s);
  }
  args.idesc = idesc_f16(kBM, 64, bf16, false);
  return launch_gemm<64>(A, B, args, lda, ldb, bf16, s);
}
}  // namespace
}  // namespace tjb

extern "C" size_t tjb_gemm_workspace_bytes(void) {
  return tjb::kSkPartialBytes + 2 * tjb::kSkMaxPartials * sizeof(int);
}

extern "C" int tjb_gemm_bias_tiles(const void* A, const void* B, const float* bias, void* C,
                                   int M, int N, int K, int lda, int ldb, int ldc, int in_dtype,
                                   int out_dtype, int act, const int32_t* m_tiles,
                                   tjb_stream_t stream) {
  return tjb::gemm_impl(A, B, bias, C, M, N, K, lda, ldb, ldc, in_dtype, out_dtype, act, m_tiles,
                        nullptr, 0, stream);
}

extern "C" int tjb_gemm_bias_tiles_ws(const void* A, const void* B, const float* bias, void* C,
                                      int M, int N, int K, int lda, int ldb, int ldc,
                                      int in_dtype, int out_dtype, int act,
                                      const int32_t* m_tiles, void* workspace,
                                      size_t workspace_bytes, tjb_stream_t stream) {
  if (workspace == nullptr) return TJB_ERR_INVALID_ARGUMENT;
  return tjb::gemm_impl(A, B, bias, C, M, N, K, lda, ldb, ldc, in_dtype, out_dtype, act, m_tiles,
                        workspace, workspace_bytes, stream);
}

extern "C" int tjb_gemm_bias(const void* A, const void* B, const float* bias, void* C, int M,
                             int N, int K, int lda, int ldb, int ldc, int in_dtype, int out_dtype,
                             int act, tjb_stream_t stream) {
  return tjb_gemm_bias_tiles(A, B, bias, C, M, N, K, lda, ldb, ldc, in_dtype, out_dtype, act,
                             nullptr, stream);
}
