/*
 * tjb200.h -- C ABI of libtjb200.so, the sm_100a (B200) kernels behind the
 * fused causal Transformer-encoder forward.
 *
 * The reference project (tjkernels, TechJam 2026) has no compiled code: its
 * kernel layer is a Python facade over Triton kernels.  Each entry point
 * below replaces one function of that facade; the facade signature it stands
 * in for is cited beside it (paths inside the reference project).
 *
 * Conventions (all entry points):
 *   - Plain device pointers and sizes; no framework types.  The caller owns
 *     and allocates every buffer (outputs included).  The library never
 *     allocates device memory, never synchronises the stream and launches
 *     only on the stream it is given, so every call may be captured in a CUDA
 *     graph.
 *   - Return 0 (TJB_OK) on success, otherwise a tjb_status code; no exception
 *     crosses the ABI.  tjb_status_string() names a code.
 *   - Dtype codes: TJB_F32 = 0, TJB_F16 = 1, TJB_BF16 = 2.
 *   - Row-major matrices; leading dimensions are in elements.  Tensor-memory
 *     (TMA) operands need 16-byte aligned base pointers and row pitches.
 *   - Device-side waits are bounded.  A wait that runs out records
 *     TJB_ERR_DEVICE_TIMEOUT in a device status word that
 *     tjb_device_status() reads back (that call synchronises the device).
 *   - Functions are thread-compatible: concurrent calls on different streams
 *     are safe; internal caches are mutex-guarded.
 */
#ifndef TJB200_H
#define TJB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* tjb_stream_t; /* == cudaStream_t */

enum tjb_status {
  TJB_OK = 0,
  TJB_ERR_INVALID_ARGUMENT = 1,  /* null pointer or negative size */
  TJB_ERR_BAD_SHAPE = 2,         /* shape outside the kernel's contract */
  TJB_ERR_BAD_ALIGNMENT = 3,     /* pointer or pitch not 16-byte aligned */
  TJB_ERR_UNSUPPORTED_DTYPE = 4,
  TJB_ERR_LAUNCH = 5,            /* CUDA reported a launch error */
  TJB_ERR_TENSOR_MAP = 6,        /* cuTensorMapEncodeTiled failed */
  TJB_ERR_DEVICE_TIMEOUT = 7,    /* a bounded device-side wait ran out */
  TJB_ERR_NO_DEVICE = 8,         /* no sm_100 device current */
  TJB_ERR_NON_PREFIX_MASK = 9    /* reported by tjb_mask_lengths' flag word */
};

enum tjb_dtype { TJB_F32 = 0, TJB_F16 = 1, TJB_BF16 = 2 };

/* Library version (major*10000 + minor*100 + patch). */
int tjb_version(void);

/* Human-readable name of a tjb_status code (static storage). */
const char* tjb_status_string(int status);

/*
 * Fused residual-add + LayerNorm over rows of length d.
 *   x        = res + delta            (delta may be NULL: x = res)
 *   res_out  = x                      (skipped when res_out is NULL)
 *   out      = (x - mean(x)) * rsqrt(var(x) + eps) * w + b   in out_dtype
 * Statistics in fp32.  When row_mask is non-NULL, rows with row_mask[r] == 0
 * get out = 0 exactly (the final padded-row zeroing of the forward).
 * res / res_out: fp32 [rows, d]; delta: delta_dtype [rows, d]; w, b: fp32 [d];
 * out: out_dtype [rows, d].  Needs d % 4 == 0 and d <= 8192; res_out may
 * alias res.
 * Replaces fused_add_layernorm(residual, delta, weight, bias, eps, out_dtype,
 * write_residual) -- tjkernels/kernels/__init__.py:48-70 and
 * tjkernels/kernels/layernorm.py:86-127; the row zeroing replaces
 * out.masked_fill(~mask[..., None], 0) at tjkernels/engine.py:267-268.
 */
int tjb_add_layernorm(const float* res, const void* delta, float* res_out, void* out,
                      const float* w, const float* b, int64_t rows, int d, float eps,
                      int delta_dtype, int out_dtype, const uint8_t* row_mask,
                      tjb_stream_t stream);

/*
 * tjb_add_layernorm restricted to the live 128-row tiles listed in m_tiles
 * (device int32: m_tiles[0] = count, then tile indices; see tjb_row_tiles).
 * Rows of unlisted tiles are neither read nor written.  m_tiles == NULL
 * processes every row.  Padding-aware form of the same facade function.
 */
int tjb_add_layernorm_tiles(const float* res, const void* delta, float* res_out, void* out,
                            const float* w, const float* b, int64_t rows, int d, float eps,
                            int delta_dtype, int out_dtype, const uint8_t* row_mask,
                            const int32_t* m_tiles, tjb_stream_t stream);

/*
 * GEMM with the residual add and the following LayerNorm in its epilogue:
 *   res_out[M, N] = res_in + A[M, K] * W[N, K]^T + bias      (fp32)
 *   out[M, N]     = LayerNorm(res_out) * gamma + beta         (eps, fp32 stats)
 * A, W: f16 or bf16 (same type), contiguous (row strides K); res_in,
 * res_out: fp32 contiguous [M, N] (res_out may equal res_in, or be NULL: not
 * written); out: f32/f16/bf16 contiguous.  N = 256, 512, 768 or 1024, K % 8
 * == 0.  The N/256 tiles of a 128-row block exchange per-row (mean, M2)
 * partials through `workspace` (tjb_gemm_add_layernorm_workspace_bytes(M, N)
 * bytes, 16-byte aligned, zero before the first call; every call that
 * completes leaves its counters zero again, but one whose bounded wait ran
 * out (TJB_ERR_DEVICE_TIMEOUT) may not: zero the workspace again before the
 * next call; calls that may overlap need separate workspaces).
 * row_mask (nullable): rows with 0 get a zero output row; m_tiles (nullable)
 * as in tjb_row_tiles.  Replaces the out-projection / FFN-out torch.addmm and
 * the fused_add_layernorm that follows it (tjkernels/engine.py:247-256;
 * tjkernels/kernels/__init__.py:48-70) with one launch in which the GEMM's
 * output never reaches HBM.
 */
int tjb_gemm_add_layernorm(const void* A, const void* W, const float* bias, const float* res_in,
                           float* res_out, const float* gamma, const float* beta, void* out,
                           int M, int N, int K, float eps, int in_dtype, int out_dtype,
                           const uint8_t* row_mask, const int32_t* m_tiles, void* workspace,
                           size_t workspace_bytes, tjb_stream_t stream);

/* Workspace bytes tjb_gemm_add_layernorm needs for M rows and N columns. */
size_t tjb_gemm_add_layernorm_workspace_bytes(int M, int N);

/*
 * C[M, N] = act(A[M, K] * B[N, K]^T + bias[N])   on tcgen05 tensor cores.
 * A, B: f16 or bf16 (same type), K-major (K contiguous; B is the nn.Linear
 * weight layout [out, in]).  bias: fp32 [N] or NULL.  act: 0 = none,
 * 1 = exact erf GELU.  C: out_dtype (f32, or the input type).
 * Accumulation in fp32.  Needs K % 8 == 0, N % 8 == 0, lda/ldb/ldc multiples
 * of 8 elements.
 * Replaces the packed-QKV and out-projection torch.addmm calls
 * (tjkernels/engine.py:245,247) and the unfused FFN fallback
 * addmm -> gelu -> addmm (tjkernels/kernels/__init__.py:88-89).
 */
int tjb_gemm_bias(const void* A, const void* B, const float* bias, void* C,
                  int M, int N, int K, int lda, int ldb, int ldc,
                  int in_dtype, int out_dtype, int act, tjb_stream_t stream);

/*
 * tjb_gemm_bias computing only the 128-row M tiles listed in m_tiles (device
 * int32: m_tiles[0] = count, then tile indices; see tjb_row_tiles); rows of
 * unlisted tiles of C are not written.  m_tiles == NULL computes all rows.
 * Padding-aware form of the engine.py:245,247 addmm calls.
 */
int tjb_gemm_bias_tiles(const void* A, const void* B, const float* bias, void* C,
                        int M, int N, int K, int lda, int ldb, int ldc,
                        int in_dtype, int out_dtype, int act, const int32_t* m_tiles,
                        tjb_stream_t stream);

/*
 * Bytes of device workspace tjb_gemm_bias_tiles_ws / tjb_ffn_tiles_ws need
 * (about 21 MB).
 */
size_t tjb_gemm_workspace_bytes(void);

/*
 * tjb_gemm_bias_tiles with stream-K: when K spans at least 48 k-blocks of 64
 * and the output tiles make at most two waves, the last of which would leave
 * at least three quarters of the SMs idle (or when there is at most one tile
 * per four SMs and K spans at least 32 k-blocks), the tiles' k-blocks are
 * divided into equal runs, one per CTA; a
 * tile whose k-blocks fall into two to four runs has its partial sums
 * (fp32) meet in the workspace, added by the CTA holding its first k-block.
 * Other shapes run as tjb_gemm_bias_tiles.  workspace: tjb_gemm_workspace_bytes()
 * bytes of device memory, 16-byte aligned, zero-filled before its first use;
 * each call leaves it ready for the next.  Calls that may run at the same
 * time need separate workspaces.  Same result layout as
 * tjb_gemm_bias_tiles; the summation order of the split tiles differs (fp32).
 * No counterpart in the reference (torch.addmm).
 */
int tjb_gemm_bias_tiles_ws(const void* A, const void* B, const float* bias, void* C,
                           int M, int N, int K, int lda, int ldb, int ldc,
                           int in_dtype, int out_dtype, int act, const int32_t* m_tiles,
                           void* workspace, size_t workspace_bytes, tjb_stream_t stream);

/*
 * Causal (or full) multi-head attention forward on tcgen05 tensor cores,
 * reading Q, K and V in place from the packed QKV projection output.
 *   qkv: [B, S, 3, H, hd] in dtype (f16 or bf16), row pitch 3*H*hd
 *   out: [B*S, H*hd] in dtype; out[b*S + i, h*hd + c]
 *   out = softmax(Q K^T * scale  (+ masking)) V   per (b, h)
 * Masking: causal (key j visible to query i iff j <= i) when causal != 0;
 * lengths (int32 [B], nullable) restricts keys to j < lengths[b];
 * key_mask (uint8 [B, S], nullable) hides keys with key_mask == 0.
 * mask_flags (int32, nullable, device) is the flag word written by
 * tjb_mask_lengths: when it reads 0 the mask is a prefix mask and query tiles
 * wholly at or past lengths[b] are skipped (their rows are written as 0).
 * Needs hd in {64, 128}.
 * Replaces flash_attention(qkv, heads, causal) --
 * tjkernels/kernels/attention.py:189-226 (kernel :34-125) -- and the
 * masked SDPA fallback at tjkernels/engine.py:184-203.
 */
int tjb_flash_fwd(const void* qkv, void* out, int B, int S, int H, int hd,
                  float scale, int causal, const int32_t* lengths,
                  const uint8_t* key_mask, const int32_t* mask_flags,
                  int dtype, tjb_stream_t stream);

/*
 * tjb_flash_fwd with work items handed out dynamically: CTAs claim
 * (batch*head, query-tile pair) items, heaviest causal rows first, from the
 * counter at sched[0], so ragged prefix lengths do not leave SMs idle.
 * sched: two int32 in device memory, 8-byte aligned, both zero before the
 * call; the kernel leaves them zero again when it completes, so one pair
 * serves any number of calls that run one after another (same stream, or a
 * CUDA graph).  Calls that may run at the same time need separate pairs.
 * skip_dead_rows: 0 writes the rows of query tiles wholly at or past
 * lengths[b] as 0, as tjb_flash_fwd does; non-zero (prefix masks only)
 * leaves those rows unspecified (work items with no live query tile are
 * dropped unwritten; others still write 0) -- for callers
 * that, like the forward with a live-tile list, never let a padded row reach
 * a valid one and zero padded rows at the end.
 * No counterpart in the reference (its Triton grid is static).
 */
int tjb_flash_fwd_sched(const void* qkv, void* out, int B, int S, int H, int hd,
                        float scale, int causal, const int32_t* lengths,
                        const uint8_t* key_mask, const int32_t* mask_flags,
                        int dtype, int32_t* sched, int skip_dead_rows, tjb_stream_t stream);

/*
 * Feed-forward block out = gelu_erf(h * w1^T + b1) * w2^T + b2.
 * h: [T, d]; w1: [F, d]; w2: [d, F] (nn.Linear layouts, f16/bf16);
 * b1: fp32 [F]; b2: fp32 [d]; out: out_dtype [T, d].
 * hidden: caller-provided scratch of T*F elements of the input dtype.
 * Replaces fused_ffn(h, w1, b1, w2, b2) -- tjkernels/kernels/__init__.py:80-89
 * and tjkernels/kernels/ffn.py:113-128.
 */
int tjb_ffn(const void* h, const void* w1, const float* b1, const void* w2,
            const float* b2, void* out, void* hidden, int T, int d, int F,
            int in_dtype, int out_dtype, tjb_stream_t stream);

/* tjb_ffn over the live 128-row tiles listed in m_tiles (see tjb_row_tiles). */
int tjb_ffn_tiles(const void* h, const void* w1, const float* b1, const void* w2,
                  const float* b2, void* out, void* hidden, int T, int d, int F,
                  int in_dtype, int out_dtype, const int32_t* m_tiles, tjb_stream_t stream);

/* tjb_ffn_tiles whose two GEMMs may use stream-K (see
 * tjb_gemm_bias_tiles_ws; one workspace serves both, they run in order). */
int tjb_ffn_tiles_ws(const void* h, const void* w1, const float* b1, const void* w2,
                     const float* b2, void* out, void* hidden, int T, int d, int F,
                     int in_dtype, int out_dtype, const int32_t* m_tiles, void* workspace,
                     size_t workspace_bytes, tjb_stream_t stream);

/*
 * The feed-forward block as ONE kernel whose [T, F] hidden activations never
 * leave the SMs: a cluster of d/256 CTAs shares each 128-token tile, each CTA
 * computing GEMM1 + bias + erf-GELU for a 128-column slice of every hidden
 * chunk, exchanging the slices through distributed shared memory, and
 * accumulating its 256 output columns of GEMM2 in tensor memory.
 * Needs d in {256, 512, 768, 1024} and F % (128 * d / 256) == 0 (else
 * TJB_ERR_BAD_SHAPE); m_tiles as in tjb_ffn_tiles (nullable).
 * Replaces the single-kernel fused_ffn of tjkernels/kernels/ffn.py:21-69,
 * which the reference could only use for d, F <= 256 (ffn.py:103-110).
 */
int tjb_ffn_fused(const void* h, const void* w1, const float* b1, const void* w2,
                  const float* b2, void* out, int T, int d, int F, int in_dtype,
                  int out_dtype, const int32_t* m_tiles, tjb_stream_t stream);

/*
 * tjb_ffn without any device allocation and without caller scratch: the
 * [T, F] hidden activations live in a 16 MiB device array inside the library
 * (T * F <= TJB_FFN_NOALLOC_MAX_HIDDEN, else TJB_ERR_BAD_SHAPE and nothing is
 * launched).  For callers that cannot allocate device memory when they run
 * (a fixed memory pool with no allocator hook, or a path where an allocation
 * may not block or fail).  Every GPU that loads the library holds the array
 * until exit.  The first call on a device looks up the array's device
 * address (and, with lazy module loading, loads the library's device code
 * there, which can take device memory): make it at set-up time, before any
 * stream capture.  The address is cached for the process and does not
 * survive cudaDeviceReset.  All calls share the array:
 * calls that overlap on the GPU race and must be serialised by the caller.
 * No counterpart in the reference.
 */
#define TJB_FFN_NOALLOC_MAX_HIDDEN (8ll << 20)
int tjb_ffn_noalloc(const void* h, const void* w1, const float* b1, const void* w2,
                    const float* b2, void* out, int T, int d, int F,
                    int in_dtype, int out_dtype, tjb_stream_t stream);

/*
 * Classify a padding mask on the device, with no host synchronisation.
 * mask: uint8/bool [B, S].  lengths[b] = number of valid positions in row b.
 * *flags = 0 when every row is a prefix (positions < lengths[b]) and
 * TJB_ERR_NON_PREFIX_MASK otherwise.
 * Replaces Engine._mask_mode (tjkernels/engine.py:131-158), which needed one
 * or two host synchronisations per distinct mask tensor.
 */
int tjb_mask_lengths(const uint8_t* mask, int B, int S, int32_t* lengths,
                     int32_t* flags, tjb_stream_t stream);

/*
 * tjb_mask_lengths and tjb_row_tiles in one launch: lengths, the flag word
 * and (tiles non-NULL) the live-tile list of tjb_row_tiles, all computed on
 * the device with one CTA that classifies the rows in parallel.  Same
 * outputs as the two calls in sequence.  Replaces Engine._mask_mode
 * (tjkernels/engine.py:131-158) together with the tile listing, which has
 * no counterpart in the reference.
 */
int tjb_mask_lengths_tiles(const uint8_t* mask, int B, int S, int32_t* lengths,
                           int32_t* flags, int32_t* tiles, tjb_stream_t stream);

/*
 * Live 128-row tiles of the flattened [B*S] token axis for a prefix padding
 * mask, on the device (no host synchronisation): a tile is live when it holds
 * a row (b, s) with s < round_up(lengths[b], 128) -- every valid row plus the
 * padded rows that share the last 128-key attention tile of a sequence.  With
 * flags pointing at a non-zero word (a non-prefix mask) or lengths == NULL,
 * every tile is live.  tiles: int32 [1 + ceil(B*S/128)]; tiles[0] = count.
 * Padded rows never influence valid rows (row-wise ops; attention masks or
 * never loads padded keys), so the forward may skip dead tiles and zero the
 * padded rows once at the end.  No counterpart in the reference (it computes
 * every row and zeroes padding after each block, engine.py:267-268).
 */
int tjb_row_tiles(const int32_t* lengths, const int32_t* flags, int B, int S, int32_t* tiles,
                  tjb_stream_t stream);

/*
 * Text of the last CUDA error this library saw on the calling thread (the
 * cause behind a TJB_ERR_LAUNCH).  No counterpart in the reference.
 */
const char* tjb_last_cuda_error(void);

/*
 * Device status word of the current device: TJB_OK, or the first error a
 * kernel recorded (TJB_ERR_DEVICE_TIMEOUT).  Synchronises the device.  When
 * clear != 0 the word is reset to TJB_OK afterwards.
 * No counterpart in the reference (its Triton kernels have no device-side
 * waits).
 */
int tjb_device_status(int clear);

/*
 * Stream-ordered snapshot of the device status word: copies it into
 * *host_dst (pinned host memory, 4-byte aligned) once every kernel enqueued
 * on `stream` before this call has finished.  Does not synchronise and
 * launches no kernel, so it may sit at the end of a captured CUDA graph; the
 * caller reads *host_dst later (after its next synchronisation, or at its
 * next call) and treats a non-zero value as TJB_ERR_DEVICE_TIMEOUT.
 * After a timeout the library's scratch state may be left mid-update:
 * every caller-owned workspace (tjb_gemm_add_layernorm's counters, the
 * stream-K workspace, the attention work counter) must be zero-filled again
 * before its next use, and the status cleared with tjb_device_status(1).
 * No counterpart in the reference (its Triton kernels have no device-side
 * waits).
 */
int tjb_device_status_async(int32_t* host_dst, tjb_stream_t stream);

/* One encoder block's parameters for tjb_forward_small (device pointers):
 * the nn.Linear weights [out, in] in the compute dtype, biases and
 * LayerNorm parameters fp32. */
typedef struct {
  const void* wqkv;  /* [3d, d]: Wq; Wk; Wv stacked */
  const void* wo;    /* [d, d] */
  const void* w1;    /* [F, d] */
  const void* w2;    /* [d, F] */
  const float* bqkv; /* [3d] */
  const float* bo;   /* [d] */
  const float* b1;   /* [F] */
  const float* b2;   /* [d] */
  const float* ln1_w;
  const float* ln1_b;
  const float* ln2_w;
  const float* ln2_b;
  float ln1_eps;
  float ln2_eps;
} tjb_small_layer;

/* Workspace bytes tjb_forward_small needs for B sequences of S tokens on
 * the current device (the split-K partials scale with its SM count). */
size_t tjb_forward_small_workspace_bytes(int B, int S, int d, int F);

/*
 * The whole encoder forward of a small batch in one launch:
 *   out = final_LN(blocks(x)), x and out fp32 [B*S, d]; valid (device
 *   uint8 [B*S], or NULL for all valid) marks padded tokens with 0: they
 *   are left out as keys and their output rows are written as zero (the
 *   reference's key-padding mask and masked_fill).
 * Pre-LN blocks as in tjb_add_layernorm / tjb_gemm_bias / tjb_flash_fwd
 * (residual stream fp32, LayerNorm statistics fp32, GEMM operands in the
 * compute dtype with fp32 accumulation, softmax in fp32), causal or not.
 * layers: host array of L (<= 12) blocks.  Needs B*S <= 256 tokens,
 * S <= 128, head_dim 64 (d = 64 H), d and F multiples of 128, d <= 1280,
 * dtype TJB_F16.  workspace: tjb_forward_small_workspace_bytes(B, S, d, F)
 * bytes, 16-byte aligned, zero before its first use and then left to this
 * function (its first 8 bytes hold the grid barrier: calls that may overlap
 * need separate workspaces; after TJB_ERR_DEVICE_TIMEOUT zero it again).
 * A cooperative launch of one CTA per SM runs the forward as phases
 * separated by bounded grid barriers.  Replaces, for small batches, the
 * per-layer launch sequence of the engine's forward (tjkernels/engine.py:
 * 205-269 in the reference), whose launches it fuses into one.
 */
int tjb_forward_small(const tjb_small_layer* layers, int L, const float* lnf_w,
                      const float* lnf_b, float lnf_eps, const float* x, float* out,
                      const uint8_t* valid, int B, int S, int d, int H, int F, int causal,
                      int dtype, void* workspace, size_t workspace_bytes, tjb_stream_t stream);

/*
 * Self-test of the bounded device-side wait: one thread spins on *flag
 * (device int32) until it becomes non-zero or timeout_ns elapses; on timeout
 * it records TJB_ERR_DEVICE_TIMEOUT in the device status word.
 * No counterpart in the reference; used to test failure detection without
 * faulting the GPU.
 */
int tjb_selftest_wait(const int32_t* flag, int64_t timeout_ns, tjb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* TJB200_H */
