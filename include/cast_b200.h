/*
 * cast_b200.h -- C ABI of the B200-native CAST RCSA/PAR hot path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream,
 * enqueues its kernels on that stream (no implicit synchronisation, no
 * allocation), and returns an int status (0 = CAST_OK).  The caller owns every
 * buffer, including the workspace whose size the *_workspace_bytes() queries
 * report.  Tensors are dense, contiguous, row-major in the shapes given.
 *
 * The reference interfaces each entry point replaces are cited beside it; all
 * paths are inside the CAST source tree (src/interaction_accel/methods/).
 */
#ifndef CAST_B200_H
#define CAST_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define CAST_API __attribute__((visibility("default")))
#else
#define CAST_API
#endif

/* cudaStream_t without pulling in the CUDA headers. */
typedef struct CUstream_st *cast_stream_t;

enum cast_status {
  CAST_OK = 0,
  CAST_ERR_INVALID_ARGUMENT = 1,  /* null pointer, negative size, bad enum */
  CAST_ERR_UNSUPPORTED = 2,       /* shape outside what the kernels implement */
  CAST_ERR_ALIGNMENT = 3,         /* pointer not 16-byte aligned */
  CAST_ERR_WORKSPACE = 4,         /* workspace too small */
  CAST_ERR_CUDA = 5,              /* a CUDA runtime/driver call failed */
  CAST_ERR_DEVICE_TIMEOUT = 6,    /* a bounded device-side wait gave up */
  CAST_ERR_NO_DEVICE = 7          /* no sm_100 device current */
};

/* Human-readable name of a status code. */
CAST_API const char *cast_status_string(int status);
/* Detail message of the last failing call on this host thread. */
CAST_API const char *cast_last_error_message(void);
/* Library version (major*10000 + minor*100 + patch). */
CAST_API int cast_version(void);
/* Test/debug helper: synchronises `stream`, then reads and clears the device
 * error word that bounded device-side waits set when they give up. */
CAST_API int cast_device_error(cast_stream_t stream);
/* Self-test of the bounded device-side wait (no counterpart in the reference):
 * one CTA waits on an mbarrier through the same bounded wait the kernels use,
 * with a limit of `limit_us` microseconds (1..1000000).  With `arrive` != 0 the
 * awaited arrival is made and the wait completes; with 0 nothing arrives, the
 * wait gives up, the kernel sets the device error word and returns normally,
 * and the next cast_device_error() reports CAST_ERR_DEVICE_TIMEOUT.  No trap,
 * no fault: the context stays usable. */
CAST_API int cast_selftest_bounded_wait(int arrive, int limit_us, cast_stream_t stream);

/* Selection rule for cast_rcsa_select_quant. */
enum cast_select_rule {
  /* Historical top-`budget` by pooled cosine (ties to the lower block index),
   * then current blocks 0..i for query block i (block-causal).  The last
   * n_query_blocks key blocks are the current chunk. */
  CAST_RULE_BUDGET_CAUSAL = 0
};

/* qk_mode values written by cast_rcsa_select_quant / read by the attention. */
enum cast_qk_mode { CAST_QK_BF16 = 0, CAST_QK_INT8 = 1 };
/* Precision policy for cast_rcsa_select_quant. */
enum cast_qk_policy {
  CAST_POLICY_BF16 = 0,   /* every (b,h,query block) uses bf16 QK^T */
  CAST_POLICY_INT8 = 1,   /* every (b,h,query block) uses int8 QK^T */
  CAST_POLICY_AUTO = 2    /* int8 where the predicted logit error is below
                             int8_tolerance, bf16 elsewhere */
};

/*
 * Pooled-QK block scoring + top-k historical block selection + per-block
 * symmetric int8 quantisation (fused), on packed [B,H,L,D] bf16 tensors whose
 * blocks of `block_size` tokens are contiguous.
 *
 * Replaces the pooled-Q/K top-k of
 *   proposed/qk_uncertainty_tangent_attention.py:1011-1042 (TABA select) and
 *   proposed/matrix_curvature_phase_frame_weave.py:5677-5831 (compact CWCA),
 * under the historical-budget + block-causal rule.  The int8 quantiser has no
 * reference counterpart (the reference attention is bf16,
 * proposed/matrix_jit_spatial_acceleration.py:676-678).
 *
 *   q        bf16 [B,H,Lq,D]   queries of the current chunk
 *   k        bf16 [B,H,Lk,D]   history blocks then the current chunk's blocks
 *   v        bf16 [B,H,Lk,D]   may be NULL (then v_codes/v_scales ignored)
 *   q_valid  uint8 [Lq], k_valid uint8 [Lk]: token validity of the compact
 *            packing (proposed/matrix_curvature_phase_frame_weave.py:5696-5699),
 *            the same for every (b,h); may be NULL (all valid).  Invalid
 *            tokens count as zero in a block's sums, amax and RMS, are left
 *            out of its pooled-mean denominator, and get code 0; k_valid also
 *            applies to v.
 *   sel_idx  int32 [B,H,nQb,maxdeg], maxdeg = min(budget,nKb-nQb)+nQb, -1 pad
 *   sel_cnt  int32 [B,H,nQb]
 *   q_codes  int8 [B,H,Lq,D], q_scales float [B,H,nQb]    (may be NULL)
 *   k_codes  int8 [B,H,Lk,D], k_scales float [B,H,nKb]    (may be NULL)
 *   v_codes  int8 [B,H,Lk,D], v_scales float [B,H,nKb]    (may be NULL)
 *   qk_mode  uint8 [B,H,nQb] (may be NULL), filled from `policy`
 *   pooled   double [B,H,nQb+nKb,D] normalised pooled means (may be NULL:
 *            then they live only in the workspace)
 * Quantiser: s = amax/127 (s = 1 if amax == 0),
 *            code = clamp(rint_half_even(x / s), -127, 127), IEEE division.
 * Scales are written for every block.  Codes: for every block, except under
 * CAST_POLICY_AUTO with qk_mode given and no v_codes, where only the blocks
 * an int8 query block reads get codes -- each int8 query block's own Q
 * block and the K blocks it selected -- and the other code bytes are left as
 * they were (the attention never reads them).
 */
CAST_API int cast_rcsa_select_quant(const void *q, const void *k, const void *v, const uint8_t *q_valid,
                           const uint8_t *k_valid, int B, int H, int Lq, int Lk, int D, int block_size, int budget, int rule,
                           int32_t *sel_idx, int32_t *sel_cnt, int8_t *q_codes, float *q_scales,
                           int8_t *k_codes, float *k_scales, int8_t *v_codes, float *v_scales,
                           uint8_t *qk_mode, int policy, float int8_tolerance, double *pooled,
                           void *workspace, size_t workspace_bytes, cast_stream_t stream);
CAST_API size_t cast_rcsa_select_quant_workspace_bytes(int B, int H, int Lq, int Lk, int D,
                                              int block_size);

/*
 * Allocation-free variant of cast_rcsa_select_quant (no counterpart in the
 * reference).  Same arguments, outputs and results, minus the workspace: the
 * scratch lives in one static device array of CAST_NOALLOC_SCRATCH_BYTES per
 * device, inside this library.  Loading the library reserves those 8 MiB on
 * every device where its module loads, for every process that loads it, even
 * one that never calls this entry point; they stay reserved until the process
 * exits.  The call makes no cudaMalloc / cudaFree or
 * other allocating call; its first call on a device looks up that array's
 * address (cudaGetSymbolAddress) with the device current.
 *
 * For callers that must not allocate device memory on the call path: hosts
 * with no caching allocator (a C, Go or Java process calling the C ABI), where
 * a cudaMalloc/cudaFree pair per call would synchronise the device and stall
 * every other stream, and serving processes that have reserved all free HBM up
 * front and have none left to hand out.
 *
 * Limit: cast_rcsa_select_quant_workspace_bytes(B,H,Lq,Lk,D,block_size) must
 * be <= CAST_NOALLOC_SCRATCH_BYTES, else CAST_ERR_WORKSPACE is returned before
 * anything is launched (for D=128 that is about 8,000 (b, h, block) triples,
 * counting query and key blocks).
 * Nothing in the scratch needs to start at zero: every element the selection
 * reads is written earlier in the same call.
 * Every call on a device shares the one array: calls whose kernels overlap on
 * the GPU (different streams without ordering between them) race and corrupt
 * each other's results.  Issue them on one stream, or order them with events.
 */
#define CAST_NOALLOC_SCRATCH_BYTES (8u << 20)
CAST_API int cast_rcsa_select_quant_noalloc(const void *q, const void *k, const void *v,
                                   const uint8_t *q_valid, const uint8_t *k_valid, int B, int H,
                                   int Lq, int Lk, int D, int block_size, int budget, int rule,
                                   int32_t *sel_idx, int32_t *sel_cnt, int8_t *q_codes,
                                   float *q_scales, int8_t *k_codes, float *k_scales,
                                   int8_t *v_codes, float *v_scales, uint8_t *qk_mode, int policy,
                                   float int8_tolerance, double *pooled, cast_stream_t stream);

/*
 * Compact-path selection: the pooled-Q/K ranking of
 * MatrixCurvaturePhaseFrameWeave._compact_cwca_attention (proposed/
 * matrix_curvature_phase_frame_weave.py:5687-5701 pooling, :5718-5725
 * stencil, :5828-5832 ranking and top-k) on the packed compact blocks, and
 * the per-block int8 quantisation the attention reads.
 *   q, k          bf16 [B,H,n_blocks*block_size,D], packed (padding rows may
 *                 hold anything: they are excluded by `valid`)
 *   valid         uint8 [n_blocks*block_size]: 1 for a real token
 *   nh, nw        the spatial block grid; blocks are (cell, nh, nw) row-major
 *   row_degrees   int32 [n_blocks] device: each row's degree (host-computed
 *                 budget, :5726-5817); max_degree = its maximum
 *   sel_idx       int32 [B,H,n_blocks,max_degree]: every block ranked by its
 *                 pooled (masked mean, L2-normalised) cosine + 1e6 on the
 *                 Manhattan-<=1 stencil, first max_degree in (rank desc,
 *                 index asc) order; sel_cnt int32 [B,H,n_blocks] = degrees
 *   q/k_codes, q/k_scales, qk_mode, policy, int8_tolerance: as
 *                 cast_rcsa_select_quant (auto: int8 QK^T only where the
 *                 predicted logit error over the row's counted blocks is below
 *                 the tolerance, codes written only for the blocks it reads)
 *   pooled        double [B,H,2*n_blocks,D] or NULL
 * Launches: 2 (3 under the auto policy).
 */
CAST_API int cast_compact_select(const void *q, const void *k, const uint8_t *valid, int B, int H,
                        int n_blocks, int block_size, int D, int nh, int nw,
                        const int32_t *row_degrees, int max_degree, int32_t *sel_idx,
                        int32_t *sel_cnt, int8_t *q_codes, float *q_scales, int8_t *k_codes,
                        float *k_scales, uint8_t *qk_mode, int policy, float int8_tolerance,
                        double *pooled, void *workspace, size_t workspace_bytes,
                        cast_stream_t stream);
CAST_API size_t cast_compact_select_workspace_bytes(int B, int H, int n_blocks, int block_size, int D);

/*
 * TABA full-layer selection: pooled-QK cosine on the (tt,th,tw) block grid of
 * a [T,Hl,Wl] latent, +1e6 Manhattan-<=1 stencil (added in float32 as the
 * reference does), stable descending order truncated to max(row_degrees).
 * Replaces MatrixTrajectoryAdaptiveBudgetAttentionCompiler.select
 * (proposed/qk_uncertainty_tangent_attention.py:988-1082) given its compiled
 * row degrees.  q, k: bf16 [B,H,T*Hl*Wl,D] in visual (t,h,w) order.
 *   row_degrees int32 [N] on the device, N = blocks of the grid;
 *   max_degree = max(row_degrees) (host int)
 *   sel_idx int32 [B,H,N,max_degree], sel_cnt int32 [B,H,N]
 *   scores  double [B,H,N,N] or NULL
 */
CAST_API int cast_taba_select(const void *q, const void *k, int B, int H, int T, int Hl, int Wl, int D,
                     int tt, int th, int tw, const int32_t *row_degrees, int max_degree,
                     int32_t *sel_idx, int32_t *sel_cnt, double *scores, void *workspace,
                     size_t workspace_bytes, cast_stream_t stream);
CAST_API size_t cast_taba_select_workspace_bytes(int B, int H, int T, int Hl, int Wl, int D, int tt,
                                        int th, int tw);

/*
 * Block-sparse flash attention (tcgen05 tensor cores, TMEM accumulators, TMA
 * tiles).  For every (b,h,query block i) the keys are the blocks
 * indices[b,h,i,0:counts[b,h,i]] of K, masked by key_valid.
 *   O = softmax(Q K^T * sm_scale) V, per row, over the allowed valid keys.
 * QK^T runs in int8 (codes x scales, int32 accumulate) where qk_mode==1 and
 * in bf16 where qk_mode==0; qk_mode NULL means int8 if q_codes/k_codes are
 * given, else bf16.  PV is bf16 with fp32 accumulation.  Rows with no valid
 * key produce zeros.
 *
 * Replaces MatrixJiTSpatialAcceleration._longcat_active
 * (proposed/matrix_jit_spatial_acceleration.py:663-729) and
 * MatrixCausalFrameLayerRelay._longcat_asymmetric
 * (proposed/matrix_curvature_phase_frame_weave.py:8847-8917), whose launch
 * of the external _attn_fwd_bsa_align takes the same operands.
 *
 *   q bf16 [B,H,Lq,D]; k, v bf16 [B,H,Lk,D]; out bf16 [B,H,Lq,D]
 *   indices int32 [B,H,nQb,max_degree]; counts int32 [B,H,nQb]
 *   key_valid uint8 [Lk] or NULL; lse float [B,H,Lq] (log2-domain row
 *   log-sum-exp of the scaled logits) or NULL.
 *   count_hint int32 [B,H,nQb] in HOST memory, or NULL: the counts the
 *   caller expects (NULL = max_degree everywhere).  Only the balance of the
 *   work over the SMs depends on it; the result follows `counts`.
 *   workspace: device memory of cast_rcsa_attention_workspace_bytes(...)
 *   bytes (same shape, max_degree and hint), 16-byte aligned, ZERO-FILLED
 *   before its first use; every completed call leaves it fit for the next.
 *   With a workspace the items that would run last are cut along their key
 *   tiles into parts whose partial results (fp32) are merged on the device;
 *   with NULL every item runs whole.  Calls that share a workspace must not
 *   overlap on the GPU.
 * Supported: D == 128, any q_block and k_block (compact blocks of 88 or 110
 * tokens included).
 */
CAST_API int cast_rcsa_attention(const void *q, const void *k, const void *v, const int8_t *q_codes,
                        const float *q_scales, const int8_t *k_codes, const float *k_scales,
                        const uint8_t *qk_mode, const int32_t *indices, const int32_t *counts,
                        int max_degree, const uint8_t *key_valid, int B, int H, int Lq, int Lk,
                        int D, int q_block, int k_block, float sm_scale, void *out, float *lse,
                        const int32_t *count_hint, void *workspace, size_t workspace_bytes,
                        cast_stream_t stream);
/* Workspace bytes for cast_rcsa_attention on the current device (0: no
 * item is cut, or the sizes are invalid / no sm_100 device). */
CAST_API size_t cast_rcsa_attention_workspace_bytes(int B, int H, int Lq, int Lk, int q_block,
                                                    int k_block, int max_degree,
                                                    const int32_t *count_hint);

/*
 * Head-sharded call with the all-gather of the head outputs fused into the
 * attention (no reference counterpart: the reference runs on one device; the
 * multi-GPU split is this library's, with the reference's per-head
 * arithmetic).  As cast_rcsa_attention, and every output row is also stored,
 * over NVLink, to the same offset of peer_out[r] (r < n_peers <= 7; host
 * arrays of device pointers, opened with cast_peer_open): this rank's slot of
 * each peer's gathered buffer (plain peer stores, no multicast).  Every CTA
 * fences its stores at system scope and counts itself in *done_ticket
 * (device memory, zero before the first call; the launch leaves it zero);
 * the launch's last CTA then stores the call's number, *calls + 1 (calls:
 * this rank's device call counter, which cast_peer_wait advances), to every
 * *peer_flag[r] (this rank's flag word in peer r, a release store at system
 * scope).  The counter lives on the device, so a CUDA graph of the call
 * replays correctly.  `out` is this rank's slot of its own gathered buffer.
 * A rank reads the gathered heads after cast_peer_wait on its stream.  Calls
 * that share done_ticket must not overlap on the GPU; every rank makes the
 * same number of calls; a peer must not write a gathered buffer its owner
 * still reads (alternate two buffers).
 */
CAST_API int cast_rcsa_attention_peers(
    const void *q, const void *k, const void *v, const int8_t *q_codes, const float *q_scales,
    const int8_t *k_codes, const float *k_scales, const uint8_t *qk_mode, const int32_t *indices,
    const int32_t *counts, int max_degree, const uint8_t *key_valid, int B, int H, int Lq, int Lk,
    int D, int q_block, int k_block, float sm_scale, void *out, float *lse,
    const int32_t *count_hint, void *workspace, size_t workspace_bytes, int n_peers,
    void *const *peer_out, uint32_t *const *peer_flag, uint32_t *done_ticket,
    const uint32_t *calls, cast_stream_t stream);

/*
 * The head outputs' gather as a launch of its own after the attention: one
 * CTA per SM streams `bytes` (a multiple of 16) of this rank's output slot
 * `src` into peer_dst[r] (r < n_peers <= 7; host array of device pointers to
 * this rank's slot in each peer's gathered buffer, from cast_peer_open) with
 * coalesced 16-byte peer stores; every CTA fences its stores at system scope
 * and counts itself in *done_ticket; the last one stores the call's number
 * (*calls + 1) to every *peer_flag[r] (release, system scope) and resets the
 * ticket.  Same contracts as cast_rcsa_attention_peers; follow it with
 * cast_peer_wait.
 */
CAST_API int cast_peer_push(const void *src, size_t bytes, int n_peers, void *const *peer_dst,
                            uint32_t *const *peer_flag, uint32_t *done_ticket, const uint32_t *calls,
                            cast_stream_t stream);

/*
 * One peer's share of the gather on a copy engine: on `stream`, one device-
 * to-device copy of `bytes` from this rank's slot `src` to `peer_dst` (this
 * rank's slot in the peer's gathered buffer, from cast_peer_open), then one
 * thread stores the call's number (*calls + 1) to *peer_flag (release,
 * system scope).  Issue one per peer on separate streams forked from the
 * caller's stream after the attention, join them back before
 * cast_peer_wait (which advances *calls).
 */
CAST_API int cast_peer_send(void *peer_dst, const void *src, size_t bytes, uint32_t *peer_flag,
                            const uint32_t *calls, cast_stream_t stream);

/*
 * Peer buffers for the fused gather (CUDA IPC, no multicast): cast_peer_alloc
 * makes a zero-filled device buffer of `bytes` on the current device and
 * writes its 64-byte IPC handle to ipc_handle; another process opens it with
 * cast_peer_open (peer access enabled) and releases it with cast_peer_close;
 * the owner frees it with cast_peer_free once no peer holds it open.
 */
CAST_API int cast_peer_alloc(size_t bytes, void **ptr, void *ipc_handle);
CAST_API int cast_peer_open(const void *ipc_handle, void **ptr);
CAST_API int cast_peer_close(void *ptr);
CAST_API int cast_peer_free(void *ptr);

/*
 * On `stream`: waits until flags[r] == *calls + 1 (acquire, system scope) for
 * every source rank r < n_src other than self_rank -- every peer's fused
 * gather of this call has landed in this rank's buffer -- then advances
 * *calls (device memory, this rank's call counter, zero at the start).
 * Bounded (1 s per rank); a wait that gives up sets the device error word
 * (CAST_ERR_DEVICE_TIMEOUT).  n_src <= 8.
 */
CAST_API int cast_peer_wait(const uint32_t *flags, int n_src, int self_rank, uint32_t *calls,
                            cast_stream_t stream);

/*
 * Compact-layout packing for the compact selection / attention path, with
 * the RoPE phase applied on the way.  Replaces, for one layer call, the
 * reference's RoPE rotation MatrixCurvaturePhaseFrameWeave.
 * _apply_compact_rope_phase (proposed/matrix_curvature_phase_frame_weave.py:
 * 5565-5574) of q and k, and the packing in _compact_cwca_attention
 * (:5677-5684: gather by block_indices, transpose, zero the padding) plus the
 * bf16 cast of the attention launch (proposed/matrix_jit_spatial_acceleration.py:679-681).
 *   q, k, v       [B,L,H,D] bf16 (in_dtype 0) or fp32 (in_dtype 1), token order
 *   phase         complex64 [L,phase_heads,D/2] as (re, im) float pairs, or
 *                 NULL (no rotation); phase_heads 1 or H
 *   block_indices int32 [P] packed slot -> token, -1 = padding
 *   q/k/v_out     bf16 [B,H,P,D]: rot(x)[b, block_indices[p], h, :] rounded
 *                 to bf16, zeros at padding.  The rotation multiplies the
 *                 (even, odd) pairs by the phase in fp32 with separately
 *                 rounded products and sums, as a complex64 multiply.
 * Supported: D == 128.  An index >= L is written as padding and reported by
 * cast_device_error().
 */
CAST_API int cast_compact_pack(const void *q, const void *k, const void *v, int in_dtype,
                      const float *phase, int phase_heads, const int32_t *block_indices, int B,
                      int L, int H, int D, int P, void *q_out, void *k_out, void *v_out,
                      cast_stream_t stream);
/*
 * The attention output back in token order (proposed/matrix_curvature_phase_
 * frame_weave.py:6095): out[b,t,h,:] = packed[b,h,token_to_packed[t],:].
 *   packed bf16 [B,H,P,D]; token_to_packed int32 [L]; out bf16 [B,L,H,D].
 * A position outside [0,P) gives zeros and is reported by cast_device_error().
 */
CAST_API int cast_compact_unpack(const void *packed, const int32_t *token_to_packed, int B, int L,
                        int H, int D, int P, void *out, cast_stream_t stream);

/*
 * Two-anchor residual writer of the control-barycentric reconstruction.
 * Replaces direct_control_barycentric_pair_write (proposed/matrix_control_
 * barycentric_pair_kernel.py:22-204), which the frame weave's control-
 * barycentric lift calls with arithmetic_mode "left_then_right_fma"
 * (proposed/matrix_curvature_phase_frame_weave.py:4278-4286).
 *   active_residual fp32 [A, spatial_channels]   (the reference's [1,A,S,C])
 *   weights         fp32 [N, 2]; source_pairs int32 [N, 2] (slots in [0,A));
 *   target_frames   int32 [N] (frames in [0,T)); output fp32 [T, spatial_channels]
 *   output[target[n]] = mix(active[pair[n][0]], w[n][0], active[pair[n][1]], w[n][1])
 * arithmetic_mode: 1 separate RN(RN(l*wl) + RN(r*wr)); 2 left_then_right_fma
 * FMA(r, wr, RN(l*wl)); 3 right_then_left_fma FMA(l, wl, RN(r*wr)); 0
 * "fused" (the reference leaves its rounding to the compiler) runs as 2.
 * Rows whose slots or frame are out of range are skipped and reported by
 * cast_device_error().
 */
CAST_API int cast_barycentric_pair_write(const float *active_residual, const float *weights,
                                const int32_t *source_pairs, const int32_t *target_frames,
                                float *output, int A, int T, int N, long long spatial_channels,
                                int arithmetic_mode, cast_stream_t stream);

/*
 * The control-barycentric lift's weights (MatrixCurvaturePhaseFrameWeave.
 * _control_barycentric_residual_lift, proposed/matrix_curvature_phase_frame_
 * weave.py:3903-3951 control state, :4094-4194 weights), one launch: for each
 * target n (targets[n] = target, left anchor, right anchor frame; prior[n] =
 * log1p(-alpha), log(alpha), alpha = (t - l) / (r - l)), weights[b, n, :] =
 * softmax(prior[n] - lambda_p * (1 - cos camera) - lambda_a * (1 - cos action))
 * over its two anchors, where the camera state of a frame is the L2-normalised
 * mean of its S rows of plucker ([B, rows >= T*S, P], fp32 or bf16) and the
 * action state the L2-normalised controls ([B, len, ch] fp32, frame rate)
 * area-pooled to the T - M current latent cells and concatenated along
 * channels, the "mouse" slot first, then the "keyboard" slot (the memory
 * frames use their own two slots, pooled to M cells and concatenated the same
 * way, their channels summing to the current ones; missing memory controls
 * count as zeros; no controls at all: equal action distances, which cancel).  A slot may be null; the host fills the
 * slots in the reference's order of the given sequences.  Cosines are
 * clamped to [-1, 1].  weights fp32 [B, n_targets, 2].  n_targets <= 64,
 * P <= 16, channels of the two slots <= 64.  With `slots` (HOST int32
 * [n_targets][2]: the rows of the active residual holding each target's left
 * and right anchor) the same launch also writes the pair writer's device
 * inputs: source_pairs int32 [n_targets][2] and target_frames int32
 * [n_targets] (all three given, or none), so a whole lift needs no copy.
 */
CAST_API int cast_barycentric_weights(const void *plucker, int plucker_bf16, int B, int rows, int P,
                             int S, int T, int M, const float *mouse, int mouse_len, int mouse_ch,
                             const float *keyboard, int keyboard_len, int keyboard_ch,
                             const float *mouse_memory, int mouse_memory_len, int mouse_memory_ch,
                             const float *keyboard_memory, int keyboard_memory_len,
                             int keyboard_memory_ch, int n_targets,
                             const int32_t *targets, const float *prior, float lambda_p,
                             float lambda_a, float *weights, const int32_t *slots,
                             int32_t *source_pairs, int32_t *target_frames, cast_stream_t stream);

/*
 * The swap router's objective and transport gates on the device: the
 * transport operators, coefficient vector and Hessian of
 * FCPASMLocalCoordinateSwapRouter._objective_terms (proposed/
 * fc_pasm_swap_routing.py:414-548, operators _transport_matrix :116-268) and
 * the gates of refine on the published sketch's mean affinities (:733-820).
 *   n              cells of the attention grid (nh*nw); R = cells * n rows
 *   u_re, u_im     fp32 [tiles][bins][n]: the operator's analysis of the grid's
 *                  basis maps (lift, reflect pad, windowed tiles, rfft2)
 *   v_re, v_im     fp32 [tiles][n][bins]: its synthesis of one tile's bin
 *                  (irfft2, windowed overlap-add, crop, pooling), for the real
 *                  and the imaginary unit -- both built once per geometry
 *   cell_anchor_count host fp32 [cells]: Exact anchors per temporal cell
 *   target_*       host tables of the skipped targets t (left anchor l, right
 *                  anchor r of one segment): the pair's theta and affinity
 *                  (device fp32 [tiles*bins], NULL: identity operator), alpha
 *                  = (t-l)/(r-l), and the (left, right) anchor cells
 *   pair_*         host tables of the same-segment anchor pairs with skipped
 *                  frames: the mean affinity (a device fp32 scalar, or NULL and
 *                  the host value), the first and last cell of the skipped
 *                  frames, whether the pair has a sketch
 * Writes coefficient [R] = lambda_anchor * anchors of the row's cell,
 * hessian [R,R] = lambda_reconstruction * sum_t [A_t B_t]^T [A_t B_t] on the
 * (left, right) cells with A_t = (1-a) M(a), B_t = a M(-(1-a)),
 * M(x) = I + sum_p V_p ((exp(i x g_p theta_p) - 1) U_p), operators [2T][n][n]
 * (scratch), the gate (0 ok, 1 the matching sketches' mean affinity is below
 * min_transport_affinity under require_fc_transport, 2 no cell passes the
 * pair gate) into gate[0] and stats[5], the matching affinity into stats[6],
 * the gated cells into stats[7], and, with min_pair_transport_affinity > 0,
 * row_gate [R].  Launches: 2.  No host synchronisation.
 */
CAST_API int cast_swap_objective(int n, int tiles, int bins, const float *u_re, const float *u_im,
                        const float *v_re, const float *v_im, int cells,
                        const float *cell_anchor_count, int n_targets,
                        const float *const *target_theta, const float *const *target_affinity,
                        const double *target_alpha, const int32_t *target_cells, int n_pairs,
                        const float *const *pair_mean, const float *pair_mean_value,
                        const int32_t *pair_cells, const int32_t *pair_matching,
                        int require_fc_transport, float min_transport_affinity,
                        float min_pair_transport_affinity, float lambda_anchor,
                        float lambda_reconstruction, float *coefficient, float *hessian,
                        uint8_t *row_gate, int32_t *gate, double *stats, float *operators,
                        cast_stream_t stream);

/*
 * FC-PASM fixed-budget swap router: the numeric body of
 * FCPASMLocalCoordinateSwapRouter.refine (proposed/fc_pasm_swap_routing.py:
 * 616-1077, called at proposed/matrix_curvature_phase_frame_weave.py:6040)
 * after its fallback gates.  Rows are pooled query blocks, memory blocks
 * first; the R = Q - memory_blocks current rows are searched.
 *   score        fp32 [B,H,Q,K] (as the call site passes it: local entries
 *                lowered by 1e6); pooled_value fp32 [B,H,K,D]
 *   selected     int64 [B,H,Q,S], rewritten IN PLACE by the accepted swaps;
 *                counts int64 [B,H,Q] (valid slots per row); local uint8 [Q,K]
 *   row_gate     uint8 [R] or NULL: rows a swap may touch (the per-pair
 *                transport-affinity gate, :785-820)
 *   gate         int32 [1] device or NULL: the transport gate written by
 *                cast_swap_objective; nonzero leaves the selection as it is
 *                (the kernels skip their work)
 *   coefficient  fp32 [R], hessian fp32 [R,R]: the objective
 *                J(e) = sum_r coefficient[r] |e_r|^2 + e^T hessian e over the
 *                current rows' sketched errors (anchor term and transport
 *                reconstruction terms, _objective_terms :414-548)
 *   stats        fp64 [14] device: [0] swaps made, [1] objective before,
 *                [2] objective after, [3] summed improvement, [4] the largest
 *                swappable count over all rows (0: nothing to swap, the
 *                selection is unchanged), [8] smallest, [9] largest and
 *                [10] summed row count, [11] historical slots before and
 *                [12] after, [13] 1 if a swap removed or added a current key;
 *                [5..7] belong to cast_swap_objective
 * Candidates are the top min(cand_blocks, multiplier*S) blocks of
 * score + 1e6*local (cand_blocks = memory_blocks if historical_only else K),
 * which holds every row's valid candidates of the reference's top-k; a
 * removed key's proxy is looked up only among the first
 * min(cand_blocks, multiplier*max swappable count) slots, the reference's
 * candidate width (:820-826), and is 0 beyond it.  Each
 * round accepts at most one swap over the whole call (the first minimum in
 * (b, h, row, slot, candidate) order) when it beats -swap_eps and the cap
 * allows.  A selected key outside [0,K) is skipped and reported by
 * cast_device_error().  Launches: a memset of the call state, then
 * 2 + num_swap_rounds kernels (3 when 0 rounds).
 */
CAST_API int cast_swap_route(const float *score, const float *pooled_value, long long *selected,
                    const long long *counts, const uint8_t *local, const uint8_t *row_gate,
                    const int32_t *gate, const float *coefficient, const float *hessian, int B, int H,
                    int Q, int K,
                    int D, int S, int memory_blocks, int candidate_multiplier, int num_swap_rounds,
                    float swap_eps, int sketch_groups, int max_swaps_per_call, int historical_only,
                    int same_bank_only, double *stats, void *workspace, size_t workspace_bytes,
                    cast_stream_t stream);
CAST_API size_t cast_swap_route_workspace_bytes(int B, int H, int Q, int K, int D, int S,
                                       int memory_blocks, int candidate_multiplier,
                                       int historical_only, int sketch_groups);

/*
 * Phase-Aware Reconstruction (FC-PASM reference numerics) on one model call.
 * Replaces WorldAlignedSpectralResidualCorrector.correct with the factory's
 * FC knobs (proposed/matrix_world_spectral_residual.py:5283-5394 ->
 * _correct_frequency_confidence_pasm_reference :2771-3662).
 *
 *   full_residual   bf16 [1,T,H*W,C], corrected IN PLACE: bracketed skipped
 *                   current frames replaced, active frames overwritten by
 *                   active_residual, memory frames untouched.
 *   active_residual bf16 [1,A,H*W,C] for active_frames (sorted, unique,
 *                   host int32 array of A global frame ids)
 *   tile_confidence float [n_pairs,P] or NULL: per-tile confidence replacing
 *                   base*ramp (the reference's precomputed_tile_confidence),
 *                   pairs in chronological order of the used anchor pairs.
 *   stats_out       float [16*(18*137) + 17] or NULL: for each of up to 16
 *                   used anchor pairs (chronological order of first use) a
 *                   block of 18*137 floats: theta [18,11,6], confidence [18],
 *                   affinity g [18,11,6], displacement [18,2], base confidence
 *                   [18], ramp confidence [18]; then, at offset 16*18*137, the
 *                   mean affinity of each pair [16] and the mean of every
 *                   target's pair affinity [1] -- the FC routing transport's
 *                   mean_affinity and the corrector's _fc_previous_mean_affinity
 *                   (:577-658, :3667-3669), reduced on the device in a fixed
 *                   order.  Written only when the call has targets.
 * Supported: H=22, W=40 (3x6 tiles of 11x10), C a multiple of 4.
 */
CAST_API int cast_par_fcpasm(void *full_residual, const void *active_residual, const int32_t *active_frames,
                    int n_active, int T, int memory_length, int H, int W, int C, float tau_low,
                    float tau_high, float freq_power, float temperature, int ramp_confidence,
                    int current_anchor_boundary, const float *tile_confidence, float *stats_out,
                    void *workspace, size_t workspace_bytes, cast_stream_t stream);
CAST_API size_t cast_par_fcpasm_workspace_bytes(int T, int H, int W, int C);

#ifdef __cplusplus
}
#endif

#endif /* CAST_B200_H */
