// attention.cu -- causal / full multi-head attention forward on tcgen05.
//
// Reads Q, K and V straight from the packed QKV projection output
// [B, S, 3, H, hd] (TMA through a 3-D tensor map over [B][S][3*H*hd]; rows
// past S zero-fill) and writes context rows into out[B*S, H*hd] at column
// h*hd.  head_dim 64 or 128.
//
// One persistent kernel, one CTA per SM.  A CTA walks work items (batch*head,
// pair of consecutive 128-row query tiles), heaviest causal rows first.  The
// two query tiles are owned by two softmax warp groups that run against one
// MMA issuer, so while group 0 computes its softmax the tensor core works on
// group 1's products and vice versa; each K/V tile is loaded once for both.
//   warp 0        TMA producer: the item's Q pair (double-buffered at
//                 head_dim 64, so it lands while the previous item runs),
//                 then (K_j, V_j) 128-row tiles into a stage ring
//   warp 1        TMEM owner + MMA issuer (one lane):
//                   S_g = Q_g K_j^T  (M=N=128, K=hd) into TMEM
//                   O_g += P_g V_j   (M=128, N=hd, K=128; V read MN-major,
//                                     P read from TMEM as the A operand)
//   warps 2-5     softmax group 0 (query rows q0 .. q0+127)
//   warps 6-9     softmax group 1 (query rows q0+128 .. q0+255)
// Softmax thread r owns query row r: it reads its score row from TMEM,
// applies causal / length / key masks, keeps the running max and sum in fp32
// (exp2 with log2(e) folded into the scale), rescales O in TMEM when the max
// grows, writes P as 16-bit pairs back into TMEM and finally writes O / l.
// Key tiles above the diagonal are never loaded; only tiles that cross the
// diagonal or a length boundary are masked.  With a prefix padding mask,
// query tiles wholly past the sequence's valid length are skipped (their
// rows are written as zeros) and keys stop at the valid length.
#include <mutex>

#include "common.cuh"

namespace tjb {
namespace {

constexpr int kTileQ = 128;
constexpr int kTileK = 128;
constexpr uint32_t kSub = 128 * 64 * 2;  // one 128-row x 64-column 16-bit sub-tile

struct AttnArgs {
  void* out;
  int32_t* sched;  // [next item, CTAs done]: dynamic work queue, or null for a static one
  const int32_t* lengths;
  const uint8_t* key_mask;
  const int32_t* mask_flags;
  int B, S, H, ldo;
  float scale_log2;
  int causal;
  int bf16;
  int skip_dead;  // prefix mask: items with no key to attend are not queued (rows unwritten)
  uint32_t idesc_qk, idesc_pv;
};

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Ten warps put three on two of the SM's four sub-partitions, which caps a
// thread at 168 registers; the softmax (a 128-score row in registers) fits.
// Each group's exponentials are computed into registers before P is
// written, so the wait for the tensor core overlaps the math.
// O is rescaled lazily: only when a row's max grows by more than 2^8 (P stays
// below 256 in 16-bit, every sum stays in fp32 range); O / l is exact for any
// choice of the reference max.
constexpr int kPairThreads = 352;
constexpr int kMmaWarp1 = kPairThreads / 32 - 1;  // issues group 1's MMAs (warp 1: group 0's)
constexpr int kItemSlots = 4;  // work items queued from the producer to the other warps
constexpr float kRescaleLog2 = 8.0f;

template <int HD_>
struct PairCfg {
  static constexpr int HD = HD_;
  static constexpr int kSubs = HD / 64;
  // head_dim 64: S, O and a separate P per group fit the 512 TMEM columns, so
  // scores are released as soon as they are in registers.  head_dim 128: S
  // and O fill TMEM, so P is written over its own group's score columns and
  // the MMA issues PV of tile j-1 before QK of tile j (the tensor pipe runs
  // in order, so the next scores never overwrite an unread P).
  static constexpr bool kAlias = HD > 64;
  static constexpr int kQSlots = HD == 64 ? 2 : 1;
  // K and V tiles go through one ring of single-tile slots in the order
  // K0 V0 K1 V1 ...; a slot is released as soon as its last reader is done,
  // so K(j+1) loads while V(j) is still being read.
  static constexpr int kSlots = HD == 64 ? 10 : 5;
  static constexpr uint32_t kQBytes = kSubs * kSub;     // one 128 x HD tile per group
  static constexpr uint32_t kTileBytes = kSubs * kSub;  // one K or V tile
  static constexpr uint32_t kSmemBytes =
      1024 + 2 * kQSlots * kQBytes + kSlots * kTileBytes + 512;
  // TMEM columns, head_dim 64: S0 [0,128) S1 [128,256) O0 [256,320)
  // O1 [320,384) P0 [384,448) P1 [448,512); head_dim 128: S0/P0 [0,128)
  // S1/P1 [128,256) O0 [256,384) O1 [384,512).  P: 128 x 128 16-bit, two
  // values per column.
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kOCol = 256;
  static constexpr uint32_t kPCol = kAlias ? 0 : 384;
  static constexpr uint32_t kPStride = kAlias ? 128 : 64;
};

struct PairItem {
  int b, h, q0;
  int n_kv[2];
  int kv_len;
};

__device__ __forceinline__ PairItem decode_pair(int w, const AttnArgs& a, int num_pairs,
                                                bool prefix) {
  PairItem it;
  const int bh_count = a.B * a.H;
  const int pr = num_pairs - 1 - w / bh_count;
  const int bh = w - (w / bh_count) * bh_count;
  it.b = bh / a.H;
  it.h = bh - it.b * a.H;
  it.q0 = pr * 2 * kTileQ;
  int kv_len = a.S;
  if (prefix) kv_len = min(max(__ldg(a.lengths + it.b), 0), a.S);
  it.kv_len = kv_len;
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    const int qs = it.q0 + g * kTileQ;
    int n = 0;
    if (qs < kv_len || (!prefix && qs < a.S)) {
      n = (kv_len + kTileK - 1) / kTileK;
      if (a.causal) n = min(n, qs / kTileK + 1);
    }
    it.n_kv[g] = n;
  }
  return it;
}

// Warp-collective bounded wait: every lane agrees on the outcome.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, abort));
}

// S = Q K^T into TMEM columns d_s: HD/16 K-steps over 64-column sub-tiles.
template <int HD>
__device__ __forceinline__ void issue_qk(uint32_t d_s, uint32_t qa, uint32_t ka, uint32_t idesc) {
#pragma unroll
  for (int k = 0; k < HD / 16; ++k) {
    const uint32_t off = (k >> 2) * kSub + (k & 3) * 32;
    umma_ss_w(d_s, sdesc_sw128(qa + off, 16, 1024), sdesc_sw128(ka + off, 16, 1024), idesc,
              k > 0 ? 1u : 0u);
  }
}

// O (+)= P V: P read from TMEM columns pa, V (MN-major) from shared memory.
template <int HD>
__device__ __forceinline__ void issue_pv(uint32_t d_o, uint32_t pa, uint32_t va, uint32_t idesc,
                                         bool accumulate) {
#pragma unroll
  for (int k = 0; k < kTileK / 16; ++k)
    umma_ts_w(d_o, pa + k * 8, sdesc_sw128(va + k * 2048, kSub, 1024), idesc,
              (accumulate || k > 0) ? 1u : 0u);
}

// One group's S = Q K^T (the K tile has landed): with separate P columns,
// wait for the softmax to hold the previous scores (s_free); issue, commit.
template <int HD>
__device__ __forceinline__ bool qk_step(uint64_t* s_free, uint64_t* s_full, uint32_t& sc,
                                        volatile int* abort, uint32_t d_s, uint32_t q_addr,
                                        uint32_t k_addr, uint32_t idesc) {
  if (s_free != nullptr && sc > 0 && !warp_wait(s_free, (sc - 1) & 1, abort)) return false;
  tc_fence_after();
  issue_qk<HD>(d_s, q_addr, k_addr, idesc);
  umma_commit_w(s_full);
  ++sc;
  return true;
}

// One group's O += P V (the V tile has landed): wait for P, issue, commit.
template <int HD>
__device__ __forceinline__ bool pv_step(uint64_t* p_full, uint64_t* pv_done, uint32_t& pvc,
                                        volatile int* abort, uint32_t d_o, uint32_t pa,
                                        uint32_t v_addr, uint32_t idesc, bool accumulate) {
  if (!warp_wait(p_full, pvc & 1, abort)) return false;
  tc_fence_after();
  issue_pv<HD>(d_o, pa, v_addr, idesc, accumulate);
  umma_commit_w(pv_done);
  ++pvc;
  return true;
}

template <int HD, bool kBF16>
__global__ void __launch_bounds__(kPairThreads, 1)
    attn_pair_kernel(const __grid_constant__ CUtensorMap tm, const AttnArgs args) {
  using Cfg = PairCfg<HD>;
  constexpr uint32_t kSlots = Cfg::kSlots;
  constexpr int kSubs = Cfg::kSubs;
  constexpr uint32_t kQSlots = Cfg::kQSlots;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;                                 // [slot][group][kQBytes]
  uint8_t* sKV = sQ + 2 * kQSlots * Cfg::kQBytes;     // [kSlots][one K or V tile]
  uint64_t* q_full = reinterpret_cast<uint64_t*>(sKV + kSlots * Cfg::kTileBytes);  // [slot]
  uint64_t* q_empty = q_full + 2;                                           // [slot]
  uint64_t* kv_full = q_empty + 2;
  uint64_t* kv_empty = kv_full + kSlots;
  uint64_t* s_full = kv_empty + kSlots;  // [group]
  uint64_t* s_free = s_full + 2;          // [group]
  uint64_t* p_full = s_free + 2;          // [group]
  uint64_t* pv_done = p_full + 2;         // [group]
  uint64_t* drain = pv_done + 2;                   // [issuer]
  uint64_t* item_full = drain + 2;                 // [kItemSlots]
  uint64_t* item_empty = item_full + kItemSlots;   // [kItemSlots]
  volatile int* item_q = reinterpret_cast<volatile int*>(item_empty + kItemSlots);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(item_empty + kItemSlots) + kItemSlots;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_pairs = (args.S + 2 * kTileQ - 1) / (2 * kTileQ);
  const int total = args.B * args.H * num_pairs;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 2);  // one commit per MMA issuer
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&pv_done[i], 1);
    }
    for (uint32_t s = 0; s < kSlots; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 2);
    }
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    for (int i = 0; i < kItemSlots; ++i) {
      mbar_init(&item_full[i], 1);
      mbar_init(&item_empty[i], 2 + 8);  // the two MMA warps and the eight softmax warps
    }
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  griddep_wait();
  griddep_launch_dependents();
  const bool prefix = args.lengths != nullptr &&
                      (args.mask_flags == nullptr || __ldg(args.mask_flags) == 0);
  const bool use_key_mask = args.key_mask != nullptr && !prefix;

  if (warp == 0) {
    if (lane == 0) {
      // -------------------------------------------------------------- producer
      uint32_t seq = 0, n_items = 0;  // K/V tiles issued, items started
      uint32_t claims = 0;            // items claimed, queued or not
      bool ok = true;
      for (uint32_t qn = 0;; ++qn) {
        // Claim the next work item (from the shared counter, heaviest causal
        // rows first, or a fixed stride without one) and queue it for the
        // MMA and softmax warps; -1 ends their loops.
        int w = args.sched != nullptr ? atomicAdd(args.sched, 1)
                                      : static_cast<int>(blockIdx.x + (claims++) * gridDim.x);
        if (w >= total || !ok) w = -1;
        PairItem it;
        if (w >= 0) {
          it = decode_pair(w, args, num_pairs, prefix);
          // With skip_dead, an item with nothing to attend (both query tiles
          // wholly past a prefix length) is dropped here and its rows are
          // left unwritten; the same queue slot takes the next claim.
          if (args.skip_dead && prefix && max(it.n_kv[0], it.n_kv[1]) == 0) {
            --qn;
            continue;
          }
        }
        const uint32_t islot = qn % kItemSlots;
        if (qn >= kItemSlots &&
            !mbar_wait(&item_empty[islot], (qn / kItemSlots - 1) & 1, abort_flag))
          break;
        item_q[islot] = w;
        mbar_arrive(&item_full[islot]);
        if (w < 0) break;
        const int n = max(it.n_kv[0], it.n_kv[1]);
        if (n == 0) continue;
        const uint32_t slot = n_items % kQSlots;
        // The slot was last used by item n_items - kQSlots.
        if (n_items >= kQSlots &&
            !mbar_wait(&q_empty[slot], ((n_items - kQSlots) / kQSlots) & 1, abort_flag))
          break;
        const int colQ = it.h * HD;
        const int ntiles = (it.n_kv[0] > 0) + (it.n_kv[1] > 0);
        mbar_arrive_expect_tx(&q_full[slot], ntiles * Cfg::kQBytes);
        for (int g = 0; g < 2; ++g)
          if (it.n_kv[g] > 0)
            for (int sub = 0; sub < kSubs; ++sub)
              tma_load_3d(sQ + (slot * 2 + g) * Cfg::kQBytes + sub * kSub, &tm, &q_full[slot],
                          colQ + sub * 64, it.q0 + g * kTileQ, it.b);
        ++n_items;
        const int colK = (args.H + it.h) * HD;
        const int colV = (2 * args.H + it.h) * HD;
        for (int t = 0; t < 2 * n && ok; ++t, ++seq) {
          const uint32_t slot = seq % kSlots;
          if (!mbar_wait(&kv_empty[slot], ((seq / kSlots) & 1) ^ 1, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* dst = sKV + slot * Cfg::kTileBytes;
          const int col = (t & 1) ? colV : colK;
          mbar_arrive_expect_tx(&kv_full[slot], Cfg::kTileBytes);
          for (int sub = 0; sub < kSubs; ++sub)
            tma_load_3d(dst + sub * kSub, &tm, &kv_full[slot], col + sub * 64, (t >> 1) * kTileK,
                        it.b);
        }
      }
      // Let every load still in flight land before the CTA exits.
      for (uint32_t k = n_items >= kQSlots ? n_items - kQSlots : 0; k < n_items; ++k)
        mbar_wait_drain(&q_full[k % kQSlots], (k / kQSlots) & 1);
      for (uint32_t k = seq >= kSlots ? seq - kSlots : 0; k < seq; ++k)
        mbar_wait_drain(&kv_full[k % kSlots], (k / kSlots) & 1);
    }
  } else if (warp == 1 || warp == kMmaWarp1) {
    // ----------------------------------------------------------- MMA issuers
    // One warp per query-tile group (warp 1: group 0, the last warp: group
    // 1), on different SM sub-partitions: a lone issuer sharing its
    // sub-partition with two busy softmax warps measured ~100 clocks per MMA
    // against the tensor pipe's 64.  Each warp runs converged and one elected
    // lane issues; its commits track only its own group's MMAs, and every
    // shared slot (K/V tile, Q pair, work item) counts one release from each.
    const int g = warp == 1 ? 0 : 1;
    const uint32_t q_base = smem_u32(sQ);
    const uint32_t d_s = tmem_base + g * kTileK;
    const uint32_t d_o = tmem_base + Cfg::kOCol + g * HD;
    const uint32_t pa = tmem_base + Cfg::kPCol + g * Cfg::kPStride;
    uint32_t n_items = 0, base = 0;  // base: ring sequence number of the item's K(0)
    uint32_t sc = 0, pvc = 0;        // this group's QK / PV tiles issued
    bool ok = true;
    for (uint32_t qn = 0; ok; ++qn) {
      const uint32_t islot = qn % kItemSlots;
      if (!warp_wait(&item_full[islot], (qn / kItemSlots) & 1, abort_flag)) break;
      const int w = __shfl_sync(0xffffffffu, item_q[islot], 0);
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[islot]);
      if (w < 0) break;
      const PairItem it = decode_pair(w, args, num_pairs, prefix);
      const int n = max(it.n_kv[0], it.n_kv[1]);
      if (n == 0) continue;
      const int ng = it.n_kv[g];
      const uint32_t slot = n_items % kQSlots;
      if (!warp_wait(&q_full[slot], (n_items / kQSlots) & 1, abort_flag)) break;
      ++n_items;
      const uint32_t q_addr = q_base + (slot * 2 + g) * Cfg::kQBytes;
      for (int j = 0; j <= n; ++j) {
        const uint32_t kseq = base + 2 * j, vseq = kseq - 1;  // K(j), V(j-1)
        const uint32_t kslot = kseq % kSlots, vslot = vseq % kSlots;
        const bool do_pv = j >= 1 && j - 1 < ng;
        const bool do_qk = j < ng;
        const uint32_t k_addr = smem_u32(sKV + kslot * Cfg::kTileBytes);
        const uint32_t v_addr = smem_u32(sKV + vslot * Cfg::kTileBytes);
        // Each issuer waits for every K/V tile it releases, used by its
        // group or not, so that its release of a slot can never run ahead of
        // the fill it belongs to (the slot's barrier counts both issuers).
        const bool has_k = j < n, has_v = j >= 1;
        bool good = true;
        auto v_phase = [&]() {
          if (has_v) {
            good = warp_wait(&kv_full[vslot], (vseq / kSlots) & 1, abort_flag);
            if (good && do_pv)
              good = pv_step<HD>(&p_full[g], &pv_done[g], pvc, abort_flag, d_o, pa, v_addr,
                                 args.idesc_pv, j > 1);
            if (good) umma_commit_w(&kv_empty[vslot]);
          }
        };
        auto k_phase = [&]() {
          if (has_k && good) {
            good = warp_wait(&kv_full[kslot], (kseq / kSlots) & 1, abort_flag);
            if (good && do_qk)
              good = qk_step<HD>(Cfg::kAlias ? nullptr : &s_free[g], &s_full[g], sc, abort_flag,
                                 d_s, q_addr, k_addr, args.idesc_qk);
            if (good) umma_commit_w(&kv_empty[kslot]);
          }
        };
        if constexpr (Cfg::kAlias) {
          // PV of tile j-1 (reads P out of the score columns), then QK of
          // tile j into the same columns; the tensor pipe keeps this order.
          v_phase();
          k_phase();
        } else {
          // Scores first (S is released as soon as the softmax holds it in
          // registers), then PV of the previous tile from the P columns.
          k_phase();
          if (good) v_phase();
        }
        if (!good) {
          ok = false;
          break;
        }
        if (j == n - 1) umma_commit_w(&q_empty[slot]);
      }
      base += 2 * n;
    }
    umma_commit_w(&drain[g]);
    mbar_wait_drain(&drain[g], 0);
  } else {
    // -------------------------------------------------------------- softmax
    const int g = (warp - 2) >> 2;  // group 0: warps 2-5, group 1: warps 6-9
    const int quad = warp & 3;
    const int r = quad * 32 + lane;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t s_col = static_cast<uint32_t>(g * kTileK);
    const uint32_t o_col = Cfg::kOCol + g * HD;
    const float sl2 = args.scale_log2;
    const uint32_t p_col = Cfg::kPCol + g * Cfg::kPStride;
    uint32_t t = 0;  // tiles this group has processed (all items)
    bool ok = true;
    for (uint32_t qn = 0; ok; ++qn) {
      const uint32_t islot = qn % kItemSlots;
      if (!__all_sync(0xffffffffu, mbar_wait(&item_full[islot], (qn / kItemSlots) & 1, abort_flag)))
        break;
      const int w = item_q[islot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[islot]);
      if (w < 0) break;
      const PairItem it = decode_pair(w, args, num_pairs, prefix);
      const int qs = it.q0 + g * kTileQ;
      const int qi = qs + r;
      uint16_t* out_ptr = static_cast<uint16_t*>(args.out) +
                          (static_cast<int64_t>(it.b) * args.S + qi) * args.ldo + it.h * HD;
      const int nk = it.n_kv[g];
      if (nk == 0) {
        if (qi < args.S) {
#pragma unroll
          for (int c = 0; c < HD / 8; ++c)
            reinterpret_cast<uint4*>(out_ptr)[c] = make_uint4(0u, 0u, 0u, 0u);
        }
        continue;
      }
      const uint8_t* km =
          use_key_mask ? args.key_mask + static_cast<int64_t>(it.b) * args.S : nullptr;
      float m_ref = -INFINITY;  // reference max the exponentials are taken against
      float l_i = 0.f;
      for (int j = 0; j < nk; ++j) {
        bool w_ok = mbar_wait(&s_full[g], t & 1, abort_flag);
        if (!__all_sync(0xffffffffu, w_ok)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t sv[kTileK];
#pragma unroll
        for (int c = 0; c < kTileK / 32; ++c) tmem_ld32p(lane_base + s_col + c * 32, sv + c * 32);
        tmem_ld_wait_n<kTileK>(sv);
        if constexpr (!Cfg::kAlias) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s_free[g]);  // scores are in registers now
        }
        const int kv0 = j * kTileK;
        const bool need_mask = (args.causal && kv0 + kTileK - 1 > qs) ||
                               (kv0 + kTileK > it.kv_len) || use_key_mask;
        if (need_mask) {
          // Keys [kv0, kv0 + lim) of this row survive the causal and length
          // limits; c < lim compares against an immediate per column.
          const int lim = (args.causal ? min(it.kv_len, qi + 1) : it.kv_len) - kv0;
#pragma unroll
          for (int c = 0; c < kTileK; ++c)
            sv[c] = c < lim ? sv[c] : __float_as_uint(-INFINITY);
          if (km != nullptr) {
#pragma unroll
            for (int c = 0; c < kTileK; ++c) {
              const int kj = kv0 + c;
              if (kj < args.S && km[kj] == 0) sv[c] = __float_as_uint(-INFINITY);
            }
          }
        }
        // Row max: eight independent chains over 16-column steps, then combine.
        float pm[8];
#pragma unroll
        for (int a = 0; a < 8; ++a) pm[a] = fmaxf(__uint_as_float(sv[a]), __uint_as_float(sv[8 + a]));
#pragma unroll
        for (int c = 16; c < kTileK; c += 16) {
#pragma unroll
          for (int a = 0; a < 8; ++a)
            pm[a] = fmax3(pm[a], __uint_as_float(sv[c + a]), __uint_as_float(sv[c + 8 + a]));
        }
        const float mx = fmax3(fmax3(pm[0], pm[1], pm[2]), fmax3(pm[3], pm[4], pm[5]),
                               fmaxf(pm[6], pm[7]));
        const float m_new = fmaxf(m_ref, mx);
        const bool grow =
            m_new > m_ref && (m_ref == -INFINITY || (m_new - m_ref) * sl2 > kRescaleLog2);
        const float alpha = grow ? fast_exp2((m_ref - m_new) * sl2) : 1.f;
        if (grow) {
          l_i *= alpha;
          m_ref = m_new;
        }
        const float mb = m_ref == -INFINITY ? 0.f : m_ref * sl2;
        // Exponentials into registers (64 packed pairs) before P is touched.
        // One pair in four goes to a polynomial on the FMA pipe, the rest to
        // the MUFU unit (measured at B4 S4096: 1/4 -> 468 TFLOP/s, 1/2 -> 448,
        // 3/4 -> 380, none -> 460; the MUFU is no longer the limit once P
        // lives in tensor memory).  Row sums in fp32 (packed adds, two chains).
        uint32_t e[kTileK / 2];
        float sa0 = 0.f, sa1 = 0.f, sb0 = 0.f, sb1 = 0.f;
#pragma unroll
        for (int c = 0; c < kTileK / 2; ++c) {
          float x0, x1, p0, p1;
          ffma2(x0, x1, __uint_as_float(sv[2 * c]), __uint_as_float(sv[2 * c + 1]), sl2, -mb);
          if ((c & 3) == 0) {
            exp2_poly2(p0, p1, x0, x1);
            add2v(sb0, sb1, p0, p1);
          } else {
            p0 = fast_exp2(x0);
            p1 = fast_exp2(x1);
            add2v(sa0, sa1, p0, p1);
          }
          e[c] = kBF16 ? Pack2<__nv_bfloat16>::pack(p0, p1) : Pack2<__half>::pack(p0, p1);
        }
        const float rowsum = (sa0 + sa1) + (sb0 + sb1);
        l_i += rowsum;
        // The previous PV has read P and accumulated into O: P is free and O
        // current.  With P over the score columns this is already implied:
        // these scores were issued after that PV and commits complete in
        // order.
        if (!Cfg::kAlias && t >= 1) {
          w_ok = mbar_wait(&pv_done[g], (t - 1) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, w_ok)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        if (j > 0 && __any_sync(0xffffffffu, grow)) {
#pragma unroll
          for (int c = 0; c < HD / 32; ++c) {
            uint32_t o[32];
            const uint32_t ta = lane_base + o_col + c * 32;
            tmem_ld32(ta, o);
            tmem_ld_wait(o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(ta, o);
          }
          tmem_st_wait();
        }
        tmem_st32p(lane_base + p_col, e);
        tmem_st32p(lane_base + p_col + 32, e + 32);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[g]);
        ++t;
      }
      if (!ok) break;
      // Epilogue: O / l once the item's last PV has landed.
      const bool w_ok = mbar_wait(&pv_done[g], (t - 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, w_ok)) break;
      tc_fence_after();
      const float inv_l = l_i > 0.f ? 1.f / l_i : 0.f;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(lane_base + o_col + c * 32, o);
        tmem_ld_wait(o);
        if (qi < args.S) {
          uint32_t p[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float x0 = __uint_as_float(o[2 * i]) * inv_l;
            const float x1 = __uint_as_float(o[2 * i + 1]) * inv_l;
            p[i] = kBF16 ? Pack2<__nv_bfloat16>::pack(x0, x1) : Pack2<__half>::pack(x0, x1);
          }
          uint4* dst = reinterpret_cast<uint4*>(out_ptr + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[i] = make_uint4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]);
        }
      }
      tc_fence_before();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
  // The last CTA out returns the work counter to zero for the next launch
  // (every CTA has made its final claim before it counts itself done).
  if (threadIdx.x == 0 && args.sched != nullptr) {
    __threadfence();
    if (atomicAdd(args.sched + 1, 1) == static_cast<int>(gridDim.x) - 1) {
      atomicExch(args.sched, 0);
      atomicExch(args.sched + 1, 0);
      __threadfence();
    }
  }
}

std::mutex g_pair_attr_mu;
bool g_pair_attr_done[64][2];

template <int HD>
int launch_attn_pair(const void* qkv, const AttnArgs& args, cudaStream_t stream) {
  using Cfg = PairCfg<HD>;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(g_pair_attr_mu);
    const int slot = HD == 64 ? 0 : 1;
    if (dev < 64 && !g_pair_attr_done[dev][slot]) {
      for (auto fn : {attn_pair_kernel<HD, false>, attn_pair_kernel<HD, true>})
        if (const int fs = cuda_status(cudaFuncSetAttribute(
                fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                static_cast<int>(Cfg::kSmemBytes))))
          return fs;
      g_pair_attr_done[dev][slot] = true;
    }
  }
  CUtensorMap tm;
  const uint64_t row = 3ull * args.H * HD;
  const uint64_t dims[3] = {row, static_cast<uint64_t>(args.S), static_cast<uint64_t>(args.B)};
  const uint64_t strides[2] = {row * 2, row * 2 * static_cast<uint64_t>(args.S)};
  const uint32_t box[3] = {64, 128, 1};
  const int st = make_tmap_16bit(&tm, 3, qkv, dims, strides, box, args.bf16 != 0);
  if (st != TJB_OK) return st;
  const long total = static_cast<long>(args.B) * args.H * ((args.S + 2 * kTileQ - 1) / (2 * kTileQ));
  const int grid = static_cast<int>(total < num_sms() ? total : num_sms());
  return args.bf16 ? launch_kernel(attn_pair_kernel<HD, true>, dim3(grid), dim3(kPairThreads),
                                Cfg::kSmemBytes, stream, tm, args)
                   : launch_kernel(attn_pair_kernel<HD, false>, dim3(grid), dim3(kPairThreads),
                                Cfg::kSmemBytes, stream, tm, args);
}

}  // namespace
}  // namespace tjb

namespace tjb {
namespace {
int flash_fwd(const void* qkv, void* out, int B, int S, int H, int hd, float scale, int causal,
              const int32_t* lengths, const uint8_t* key_mask, const int32_t* mask_flags,
              int dtype, int32_t* sched, int skip_dead, tjb_stream_t stream) {
  if (!qkv || !out || B <= 0 || S <= 0 || H <= 0 || hd <= 0) return TJB_ERR_INVALID_ARGUMENT;
  if (dtype != TJB_F16 && dtype != TJB_BF16) return TJB_ERR_UNSUPPORTED_DTYPE;
  if (hd != 64 && hd != 128) return TJB_ERR_BAD_SHAPE;
  if (B * H > 2147483647 / 2 || (S + kTileQ - 1) / kTileQ > 65535) return TJB_ERR_BAD_SHAPE;
  if (!aligned16(qkv) || !aligned16(out)) return TJB_ERR_BAD_ALIGNMENT;
  if (sched != nullptr && (reinterpret_cast<uintptr_t>(sched) & 7u) != 0)
    return TJB_ERR_BAD_ALIGNMENT;
  if (!device_ok()) return TJB_ERR_NO_DEVICE;
  AttnArgs a;
  a.out = out;
  a.sched = sched;
  a.lengths = lengths;
  a.key_mask = key_mask;
  a.mask_flags = mask_flags;
  a.B = B;
  a.S = S;
  a.H = H;
  a.ldo = H * hd;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.causal = causal != 0;
  a.bf16 = dtype == TJB_BF16;
  a.skip_dead = skip_dead != 0;
  a.idesc_qk = idesc_f16(kTileQ, kTileK, a.bf16 != 0, false);
  a.idesc_pv = idesc_f16(kTileQ, hd, a.bf16 != 0, true);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return hd == 64 ? launch_attn_pair<64>(qkv, a, s) : launch_attn_pair<128>(qkv, a, s);
}
}  // namespace
}  // namespace tjb

extern "C" int tjb_flash_fwd(const void* qkv, void* out, int B, int S, int H, int hd, float scale,
                             int causal, const int32_t* lengths, const uint8_t* key_mask,
                             const int32_t* mask_flags, int dtype, tjb_stream_t stream) {
  return tjb::flash_fwd(qkv, out, B, S, H, hd, scale, causal, lengths, key_mask, mask_flags,
                        dtype, nullptr, 0, stream);
}

extern "C" int tjb_flash_fwd_sched(const void* qkv, void* out, int B, int S, int H, int hd,
                                   float scale, int causal, const int32_t* lengths,
                                   const uint8_t* key_mask, const int32_t* mask_flags, int dtype,
                                   int32_t* sched, int skip_dead_rows, tjb_stream_t stream) {
  if (sched == nullptr) return TJB_ERR_INVALID_ARGUMENT;
  return tjb::flash_fwd(qkv, out, B, S, H, hd, scale, causal, lengths, key_mask, mask_flags,
                        dtype, sched, skip_dead_rows, stream);
}
