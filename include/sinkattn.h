/*
 * sinkattn.h — C ABI of libsinkattn.so, the sm_100a (B200) implementation of
 * SinkAttention's two hot paths:
 *
 *   1. block-sparse attention forward over kept 128x128 blocks
 *      (tcgen05 tensor cores, TMEM accumulators, TMA tile loads), and
 *   2. the calibration chain: 128-token mean pooling of Q/K, pooled-score
 *      softmax, batch mean / running accumulation, and the 0.85-coverage
 *      per-row block-mask build.
 *
 * Conventions shared by every entry point
 *   - All pointers are device pointers unless the parameter says "host".
 *   - Strides are in ELEMENTS, ordered (batch, head, seq, dim) for 4-D
 *     tensors; the innermost (dim) stride must be 1.
 *   - Every call is stream-ordered on `stream` and performs no host
 *     synchronisation and no device allocation; scratch memory, where a
 *     kernel needs any, is passed in by the caller (see *_workspace_size).
 *   - Return value: SA_OK (0) or a negative SA_E* code. The message of the
 *     last failure on the calling thread is returned by sa_last_error().
 *   - `status` arguments (nullable) point to one int32 that a kernel sets to
 *     a non-zero SA_DEV_* code when one of its bounded waits gives up; the
 *     kernel then returns early instead of spinning. Kernels write it only on
 *     failure and read it only while a wait is already slow, so it may live in
 *     mapped page-locked host memory (sa_status_create), where the host reads
 *     it at any time without synchronising (sa_check_status), or in device
 *     memory. It is never read inside these calls.
 */
#ifndef SINKATTN_H_
#define SINKATTN_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#if defined(__GNUC__)
#define SA_API __attribute__((visibility("default")))
#else
#define SA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define SA_OK 0
#define SA_EINVAL (-1)       /* bad argument (shape, stride, alignment, null) */
#define SA_EUNSUPPORTED (-2) /* valid request this build does not implement */
#define SA_ETIMEOUT (-3)     /* a device wait gave up (sa_check_status) */
#define SA_ECUDA (-4)        /* a CUDA runtime / driver call failed */

/* Device status codes written into `status` by kernels. */
#define SA_DEV_OK 0
#define SA_DEV_WAIT_TIMEOUT 1 /* an mbarrier wait exceeded its iteration limit */

/* Mask-builder modes (offline_text_video_coverage_mode). */
#define SA_COVERAGE_JOINT 0
#define SA_COVERAGE_VIDEO_RESIDUAL 1

/* Row flags written by sa_coverage_mask (bit set). */
#define SA_ROW_TIE_AT_CUT 1u      /* equal scores straddle the cut: order is a tie-break */
#define SA_ROW_NEAR_TARGET 2u     /* a cumulative sum is within 2 ulp of the target */
#define SA_ROW_EMPTY_FALLBACK 4u  /* the row was empty and kept its top-1 block */

SA_API const char* sa_last_error(void);
SA_API int sa_version(void);
/* Number of SMs of the current device (cached per device). */
SA_API int sa_device_sm_count(void);

/*
 * Block-sparse attention forward.
 * Replaces: block_sparse_attn_func(q_unpad, k_unpad, v_unpad, cu_seqlens_q,
 *   cu_seqlens_k, head_mask_type, streaming_info, base_blockmask, max_seqlen_q,
 *   max_seqlen_k, p_dropout=0.0, deterministic=True, softmax_scale=None,
 *   is_causal=False, exact_streaming=False, return_attn_probs=...)
 *   called at sinkattention/sparse_attention.py:735-771 (external package
 *   mit-han-lab/Block-Sparse-Attention, imported at sparse_attention.py:22-28).
 *
 * q [B,H,Sq,D], k/v [B,H,Sk,D], out [B,H,Sq,D]: bf16, any layout whose
 *   strides are multiples of 8 elements (16 bytes) with stride(dim)=1 and
 *   16-byte aligned base pointers. D must be 128.
 * block_mask: uint8 (torch.bool) [Bm, Hm, ceil(Sq/128), ceil(Sk/128)] with
 *   element strides m_strides (Bm is 1 or B; a batch stride of 0 broadcasts).
 * head_mask_type: nullable device int32 [H]. NULL => head h uses mask head h
 *   (requires Hm == H). Otherwise value t > 0 => head h uses mask head t-1
 *   and value 0 => head h is dense (all blocks). Negative values (streaming
 *   heads upstream) are not supported; the library never reads device
 *   memory on the host, so the Python layer rejects them before the call and
 *   the kernel treats them as dense.
 * softmax_scale: <= 0 selects 1/sqrt(D).
 * lse: nullable fp32 [B,H,Sq] contiguous, natural-log logsumexp per row. Rows
 *   whose mask row keeps no block produce out = 0 and lse = -inf.
 * status: nullable device int32, set to SA_DEV_WAIT_TIMEOUT if a bounded wait
 *   in the kernel gave up.
 * The launch is a persistent grid (one CTA per SM) that takes query tiles from
 *   a tile counter inside the library: 1024 counter slots per device, handed
 *   to launches round robin and reset by each launch's last CTA, so up to 1024
 *   launches may be in flight on one device.
 */
SA_API int sa_bsattn_fwd(const void* q, const void* k, const void* v,
                  const int64_t q_strides[4], const int64_t k_strides[4],
                  const int64_t v_strides[4], int B, int H, int Sq, int Sk,
                  int D, const uint8_t* block_mask, const int64_t m_strides[4],
                  int Hm, const int32_t* head_mask_type, float softmax_scale,
                  void* out, const int64_t o_strides[4], float* lse,
                  int32_t* status, cudaStream_t stream);

/*
 * Sink attention fused with the pooled-K/V dynamic branch.
 * Replaces, in one pass, the two _block_sparse_attn calls of
 * WanSinkSparseInnerAttention.forward (wanx/runtime/sink_sparse_wan.py:210-256)
 * and their adaptive mix _mix_attention_outputs (sinkattention/sparse_attention.py:
 * 898-919): with w_s = lse_s and w_d = lse_d + ln(gap), the mix equals one
 * softmax over the kept sink keys together with every pooled key, the pooled
 * keys' logits raised by ln(gap). That softmax is computed exactly (fp32
 * accumulation), without the mix's bf16-rounded LSEs.
 * Arguments are those of sa_bsattn_fwd plus the pooled keys/values k_pool,
 * v_pool [B,H,Sk_pool,D] (e.g. from sa_mean_pool_seq with pool = gap) and
 * log_gap = ln(gap). lse (nullable) is the natural-log LSE of the combined
 * softmax. Requires ceil(Sk/128) + ceil(Sk_pool/128) <= 1024.
 */
SA_API int sa_sink_dynamic_attn_fwd(
    const void* q, const void* k, const void* v, const int64_t q_strides[4],
    const int64_t k_strides[4], const int64_t v_strides[4], int B, int H, int Sq, int Sk,
    int D, const uint8_t* block_mask, const int64_t m_strides[4], int Hm,
    const int32_t* head_mask_type, const void* k_pool, const void* v_pool,
    const int64_t kp_strides[4], const int64_t vp_strides[4], int Sk_pool, float log_gap,
    float softmax_scale, void* out, const int64_t o_strides[4], float* lse, int32_t* status,
    cudaStream_t stream);

/*
 * Scratch bytes sa_pool_scores needs: the work counters and flags of the
 * fused kernel (128 * (H + 5) bytes rounded up to 256, then 8 bytes per
 * group of 16 block rows of every head, rounded up to 256), then pooled Q
 * and K in fp32 and the fp32 pooled logits, 4 * B * H * nb * (2 * D + nb)
 * bytes with nb = ceil(S/block).
 */
SA_API size_t sa_pool_scores_workspace_size(int B, int H, int S, int D, int block);

/*
 * Pooled block scores, `mean` mode.
 * Replaces: _compute_pooled_qk_block_scores (sinkattention/sparse_attention.py:118-142)
 *   with pooling_mode="mean": q_pool = _mean_pool_sequence(q.float(), block)
 *   (replicate-pads the last partial block with the final token,
 *   sparse_attention.py:79-94), scores = q_pool @ k_pool^T * scale,
 *   softmax over the key-block axis.
 * q, k: bf16 [B,H,S,D] strided (stride(dim) == 1). D <= 256, block >= 1.
 * scores: nullable fp32 [B,H,nb,nb] contiguous softmax rows.
 * batch_mean: nullable fp32 [H,nb,nb] contiguous = scores.mean(dim=0)
 *   (SinkMaskCalibrator.record, sparse_attention.py:580-581).
 * At least one of scores / batch_mean must be non-NULL.
 * workspace: device scratch of sa_pool_scores_workspace_size() bytes,
 *   256-byte aligned, with any contents (the fused kernel's work counters
 *   carry a per-launch tag, so nothing needs clearing). Calls sharing one
 *   workspace must not overlap on the GPU.
 * scale <= 0 selects 1/sqrt(D).
 * At D = 128, block = 128, nb <= 256, H <= 128 this runs the fused
 * calibration-layer kernel (as sa_calibration_layer), whose results agree
 * within one ulp with the pool / logits / softmax chain that other shapes
 * run. No status word: a
 * bounded wait that gives up (it does not in a working launch) leaves NaN
 * in the affected rows.
 */
SA_API int sa_pool_scores(const void* q, const void* k, const int64_t q_strides[4],
                   const int64_t k_strides[4], int B, int H, int S, int D,
                   int block, float scale, float* scores, float* batch_mean,
                   void* workspace, size_t ws_bytes, cudaStream_t stream);

/*
 * The two halves of sa_pool_scores, for callers that pipeline layers (the
 * HBM-bound pooling of one layer overlaps the small compute-bound score step
 * of the previous one on another stream).
 * sa_pool_means: block means of Q and K (sparse_attention.py:88-94 with the
 *   replicate padding of lines 79-85), qp/kp fp32 [B,H,nb,D] contiguous.
 * sa_pooled_softmax: softmax(qp kp^T * scale) per batch (sparse_attention.py:
 *   140-142) into scores [B,H,nb,nb] and/or its batch mean [H,nb,nb]
 *   (line 581); logits_ws is fp32 scratch of B*H*nb*nb elements.
 */
SA_API int sa_pool_means(const void* q, const void* k, const int64_t q_strides[4],
                         const int64_t k_strides[4], int B, int H, int S, int D,
                         int block, float* qp, float* kp, cudaStream_t stream);
SA_API int sa_pooled_softmax(const float* qp, const float* kp, int B, int H, int nb,
                             int D, float scale, float* scores, float* batch_mean,
                             float* logits_ws, cudaStream_t stream);

/*
 * sa_pooled_softmax over L stacked layers in two launches, for a calibration
 * pass over many layers: qp, kp fp32 [L,B,H,nb,D] (block means), batch_means
 * fp32 [L,H,nb,nb] (each layer's mean over its B), logits_ws fp32
 * [L*B*H*nb*nb]. scale <= 0 means 1/sqrt(D).
 * Replaces: the per-layer _compute_block_scores + batch mean of
 *   SinkMaskCalibrator.record (sparse_attention.py:138-142, 575-582).
 */
SA_API int sa_pooled_softmax_layers(const float* qp, const float* kp, int L, int B, int H, int nb,
                                    int D, float scale, float* batch_means, float* logits_ws,
                                    cudaStream_t stream);

/*
 * One calibration layer of the `mean` score mode in a single launch:
 * pooling of Q and K, pooled logits, per-batch softmax, batch mean, and
 * optionally the calibrator's running sums and the coverage mask.
 * Replaces: _compute_pooled_qk_block_scores with pooling_mode="mean"
 *   (sinkattention/sparse_attention.py:118-142), the batch mean of
 *   SinkMaskCalibrator.record (line 580), _accumulate_score (lines 537-549)
 *   and _build_direct_mean_coverage_mask (lines 241-376) on the batch mean.
 * The HBM-bound pooling overlaps the score work inside the launch: heads are
 * pooled in order and each head's rows are scored, and their mask rows
 * built, as soon as it is complete.
 * q, k: bf16 [B,H,S,128] strided (stride(dim) == 1, other strides multiples
 *   of 8 elements, 16-byte aligned); S <= 32768 (at most 256 blocks of 128).
 * scores: nullable fp32 [B,H,nb,nb]; batch_mean: nullable fp32 [H,nb,nb].
 * acc_sum / acc_sumsq: nullable pair fp32 [H,nb,nb]: sum += mean and
 *   sumsq += mean * mean with separate roundings, or set when acc_first != 0.
 * mask_out: nullable bool [H,nb,nb]: the coverage rule of sa_coverage_mask
 *   (mode, coverage, keep_diagonal, text_blocks, force_sink_col as there)
 *   on the batch mean, with row totals summed in fp64 and rounded;
 *   row_flags: nullable int32 [H,nb] SA_ROW_* bits (needs mask_out).
 * At least one output must be requested. The scores and batch mean equal
 * those of the three-kernel chain (pooling, pooled logits, softmax) to
 * within one ulp; the sums and the mask are exactly what
 * sa_score_accumulate and sa_coverage_mask (row_total NULL) give on this
 * launch's batch mean.
 * workspace: sa_calibration_layer_workspace_size() bytes, 256-byte aligned,
 *   with any contents: work counters and flags tagged with a per-launch
 *   number (so nothing needs clearing), the pooled Q and K, and a batch-mean
 *   scratch. Calls sharing one workspace must not overlap on the GPU. H is at
 *   most 128.
 * scale <= 0 selects 1/sqrt(128). status: as sa_bsattn_fwd; once a wait
 *   gives up, the launch's outputs are not valid.
 */
SA_API size_t sa_calibration_layer_workspace_size(int B, int H, int S);
SA_API int sa_calibration_layer(const void* q, const void* k, const int64_t q_strides[4],
                                const int64_t k_strides[4], int B, int H, int S, int D,
                                float scale, float* scores, float* batch_mean, float* acc_sum,
                                float* acc_sumsq, int acc_first, uint8_t* mask_out,
                                int32_t* row_flags, int mode, float coverage, int keep_diagonal,
                                int text_blocks, int force_sink_col, void* workspace,
                                size_t ws_bytes, int32_t* status, cudaStream_t stream);

/*
 * sa_pool_scores without a workspace argument. It has no counterpart in the
 * reference: it exists for callers that cannot allocate device memory when
 * they call in (a C/FFI host with no device allocator, or a server that
 * reserved all GPU memory at start-up and may not cudaMalloc while serving).
 * The scratch is a 16 MiB device array inside the library, held by every GPU
 * that loads it until the process exits; shapes needing more than 16 MiB
 * (see sa_pool_scores_workspace_size) return SA_EINVAL. The first call on a
 * device resolves the array's address with cudaGetSymbolAddress, so make it
 * before any stream capture; the address is kept until the process exits, so
 * no call may follow a cudaDeviceReset of that device. Nothing in the array
 * has to start at zero: the work counters at its start carry a per-launch
 * tag, and every other byte a call reads it writes first. All calls share
 * the array: calls that overlap on the GPU race and must be serialised by the
 * caller. Arguments and results are those of sa_pool_scores, which runs the
 * same kernels.
 */
SA_API int sa_pool_scores_noalloc(const void* q, const void* k,
                                  const int64_t q_strides[4],
                                  const int64_t k_strides[4], int B, int H,
                                  int S, int D, int block, float scale,
                                  float* scores, float* batch_mean,
                                  cudaStream_t stream);

/*
 * Block statistics of dense Q K^T for the two other calibration score modes.
 * mode SA_STATS_EXACT replaces _compute_exact_block_mass_scores
 *   (sinkattention/sparse_attention.py:145-227): scores[b,h,qb,kb] = mean over
 *   the valid rows of query block qb of the softmax mass of key block kb.
 * mode SA_STATS_MAX replaces the Triton kernel attn_with_pooling
 *   (sinkattention/pooling_kernel.py:194-248, selected by pooling_mode "triton"
 *   at sparse_attention.py:124-134): per row the bf16 maxima of the scaled
 *   logits of every key block, Po = bf16(max over the block's rows of
 *   exp2(R - row max)), then Po / sum(Po) rounded like bf16 tensors. For S not
 *   a multiple of 128, keys past S are masked and rows past S take no part in
 *   the column maxima (the Triton kernel reads past the head there).
 * q, k: bf16 [B,H,S,D] strided, D = 128. scores: fp32 [B,H,nb,nb] contiguous.
 * workspace: sa_block_stats_workspace_size() bytes, both modes (per-CTA
 * scratch of the persistent kernel). softmax_scale <= 0 selects 1/sqrt(D).
 * status: as sa_bsattn_fwd.
 */
#define SA_STATS_EXACT 0
#define SA_STATS_MAX 1
SA_API size_t sa_block_stats_workspace_size(int B, int H, int S, int mode);
SA_API int sa_block_stats(const void* q, const void* k, const int64_t q_strides[4],
                          const int64_t k_strides[4], int B, int H, int S, int D,
                          int mode, float softmax_scale, float* scores,
                          void* workspace, size_t ws_bytes, int32_t* status,
                          cudaStream_t stream);

/*
 * Running score statistics of one layer.
 * Replaces: SinkMaskCalibrator._accumulate_score (sparse_attention.py:537-549)
 *   on a device-resident accumulator: sum += x, sumsq += x*x, where x is an
 *   fp32 [n] tensor (typically the batch mean [H,nq,nk]). With `first` != 0
 *   the accumulators are overwritten (sum = x, sumsq = x*x).
 */
SA_API int sa_score_accumulate(const float* x, int64_t n, float* sum, float* sumsq,
                        int first, cudaStream_t stream);

/*
 * mean = sum / count; std = sqrt(clamp_min(sumsq / count - mean^2, 0)).
 * Replaces: SinkMaskCalibrator._build_mean_and_masks (sparse_attention.py:563-566).
 * `count` is a device fp32 tensor [n] of per-element counts, used as given,
 * or NULL with a scalar `scalar_count`. std is nullable. With emit_variance
 * != 0, std_out receives the clamped variance instead (no square root): the
 * reference takes that root with torch.sqrt on the CPU, which is not
 * correctly rounded in every case, so a host that wants its bits applies the
 * same operation itself.
 */
SA_API int sa_score_finalize(const float* sum, const float* sumsq, const float* count,
                      float scalar_count, int64_t n, float* mean, float* std_out,
                      int emit_variance, cudaStream_t stream);

/*
 * Z-Image calibration: one sample's block scores [H, n_blocks, n_blocks]
 * (n_blocks = image_blocks + text_blocks) placed into the fixed
 * [H, total_blocks, total_blocks] layout (image blocks first, the sample's
 * text blocks at the end) and accumulated: sum += s, sumsq += s*s,
 * presence += 1 where a score landed (0 elsewhere). `first` overwrites.
 * Replaces: _align_scores_image_text_suffix, _alignment_presence_mask and
 *   ZImageSinkMaskCalibrator._accumulate / record
 *   (zimg/runtime/sink_sparse_zimage.py:140-186, 262-278, 300-319).
 */
SA_API int sa_score_accumulate_aligned(const float* scores, int H, int n_blocks,
                                       int image_blocks, int text_blocks, int total_blocks,
                                       float* sum, float* sumsq, float* presence, int first,
                                       cudaStream_t stream);

/*
 * Presence-weighted mean and std: presence is raised to >= 1 in place, then
 * mean = sum / presence, std = sqrt(clamp_min(sumsq / presence - mean^2, 0)).
 * Replaces: ZImageSinkMaskCalibrator.build_package statistics
 *   (zimg/runtime/sink_sparse_zimage.py:330-334). std is nullable;
 *   emit_variance as for sa_score_finalize.
 */
SA_API int sa_score_finalize_presence(const float* sum, const float* sumsq, float* presence,
                                      int64_t n, float* mean, float* std_out,
                                      int emit_variance, cudaStream_t stream);

/*
 * Q/K producer of the sink attention: RMSNorm over the hidden dimension, then
 * the rotary embedding, for Q and K in one pass.
 *   y = bf16((x * rstd) * w), rstd = 1 / sqrt(sum(x^2) / hidden + eps);
 *   per head (D channels) and pair i at position s = row % S:
 *   out[2i] = bf16(y[2i] cos[s,i] - y[2i+1] sin[s,i]),
 *   out[2i+1] = bf16(y[2i] sin[s,i] + y[2i+1] cos[s,i]).
 * Rows are tokens (rows = B*S), `hidden` bf16 values each, row strides in
 * elements (multiples of 8); in place is allowed. w_q/w_k: [hidden] bf16
 * (w_is_bf16 != 0) or fp32, both NULL for no affine weight. cos/sin: fp32
 * [S, >= D/2] with the given row stride, both NULL for no rotation.
 * Replaces: apply_fast_qk_norm + apply_fast_rotary_qk in the Wan attention
 *   processor (wanx/runtime/sink_sparse_wan.py:300-315;
 *   wanx/runtime/fast_misc.py:834-864, 216-234).
 */
SA_API int sa_qk_norm_rope(const void* q_in, const void* k_in, int64_t q_in_row_stride,
                           int64_t k_in_row_stride, int rows, int S, int hidden, int D,
                           const void* w_q, const void* w_k, int w_is_bf16, float eps,
                           const float* cos_table, const float* sin_table,
                           int64_t freq_row_stride, void* q_out, void* k_out,
                           int64_t q_out_row_stride, int64_t k_out_row_stride,
                           cudaStream_t stream);

/*
 * Per-row minimal coverage block mask.
 * Replaces: _build_direct_mean_coverage_mask (sinkattention/sparse_attention.py:268-376)
 *   including _build_offline_required_mask (sparse_attention.py:241-265).
 * scores: fp32 [H,nq,nk] with element strides s_strides[3] (stride(-1) == 1).
 * mode: SA_COVERAGE_JOINT (lines 334-376) or SA_COVERAGE_VIDEO_RESIDUAL
 *   (lines 286-332; needs text_blocks > 0, else JOINT is used as upstream does).
 * coverage: offline_direct_coverage (clamped to [0,1] as line 276 does).
 * text_blocks: number of required leading query rows / key columns
 *   (ceil(text_length/block_size) when force_text_global_attention, else 0).
 * force_sink_col: non-zero adds key column 0 to the required set of every
 *   row before the coverage step (the "always keep key-block 0" rule; 0
 *   reproduces the unmodified reference).
 * row_total / row_selected: nullable fp32 [H,nq] contiguous. When given, they
 *   are used verbatim as sum_j s[j] and sum_j s[j]*req[j] (lines 334, 339);
 *   when NULL they are computed on the device in fp64 and rounded to fp32.
 * mask_out: uint8 [H,nq,nk] contiguous (0/1, torch.bool compatible).
 * row_flags: nullable int32 [H,nq], SA_ROW_* bits.
 * nk <= 4096.
 */
SA_API int sa_coverage_mask(const float* scores, const int64_t s_strides[3], int H,
                     int nq, int nk, int mode, float coverage,
                     int keep_diagonal, int text_blocks, int force_sink_col,
                     const float* row_total, const float* row_selected,
                     uint8_t* mask_out, int32_t* row_flags,
                     cudaStream_t stream);

/*
 * Sequence mean pooling with optional kept prefix.
 * Replaces: _mean_pool_sequence_preserve_prefix (sparse_attention.py:97-115),
 *   used for the pooled K/V of the dynamic branch
 *   (wanx/runtime/sink_sparse_wan.py:220-232). The tail is replicate-padded
 *   to a multiple of `pool` (sparse_attention.py:79-85). x, out: bf16,
 *   [B,H,S,D] -> [B,H,prefix + ceil((S-prefix)/pool),D]; fp32 accumulation,
 *   one rounding to bf16.
 */
SA_API int sa_mean_pool_seq(const void* x, const int64_t x_strides[4], int B, int H,
                     int S, int D, int pool, int prefix, void* out,
                     const int64_t o_strides[4], cudaStream_t stream);

/*
 * Adaptive LSE mix of the sink and dynamic branches.
 * Replaces: _mix_attention_outputs (sinkattention/sparse_attention.py:898-919)
 *   with mixing_mode="adaptive": w_s = lse_s, w_d = lse_d + ln(gap),
 *   alpha = e^{w_s}/(e^{w_s}+e^{w_d}), out = alpha*o_s + (1-alpha)*o_d.
 * o_s, o_d, out: bf16 [B,H,S,D] strided; lse_s, lse_d: fp32 [B,H,S]
 *   contiguous (natural log).
 */
SA_API int sa_mix_outputs(const void* o_s, const int64_t os_strides[4], const float* lse_s,
                   const void* o_d, const int64_t od_strides[4], const float* lse_d,
                   int B, int H, int S, int D, float log_gap, void* out,
                   const int64_t o_strides[4], cudaStream_t stream);

/*
 * Sequence-parallel (Ulysses) exchange over NVLink peer memory, and the CUDA
 * IPC helpers that map the peers' buffers. No counterpart in the reference,
 * which runs on one GPU (wanx/runtime/inference.py:65-69); they carry its
 * attention call across ranks in a sequence-parallel DiT
 * (sinkattn_b200/sharding.py). "Units" are the (batch, head) pairs u = b*H +
 * h; rank r owns units r*n_per .. r*n_per + n_per - 1 (n_per*P >= B*H).
 *
 * sa_ipc_alloc / sa_ipc_free: cudaMalloc / cudaFree of a buffer to share.
 * sa_ipc_get_handle: the 64-byte CUDA IPC handle of a buffer from
 *   sa_ipc_alloc. sa_ipc_open_handle: maps another process's buffer into this
 *   one (peer access enabled); sa_ipc_close unmaps it.
 *
 * sa_ulysses_dispatch: T (1..3) tensors, this rank's sequence shard
 *   [B, Sr, H, 128] bf16 each (element strides src_strides[4t..4t+3], last 1,
 *   others multiples of 8; 16-byte aligned), are written into the receive
 *   buffers dst[r] (r < P <= 8, device addresses, peers' included) of the
 *   units' owners: dst[owner] is [T][n_per][P*Sr][128] bf16, and the row of
 *   shard position s lands at sequence position rank*Sr + s of its unit.
 *   Rows of units past B*H are not written.
 * sa_ulysses_combine: this rank's units' attention output [n_per][P*Sr][128]
 *   bf16 (contiguous) and LSE [n_per][P*Sr] fp32 (nullable) are written into
 *   out_dst[p] ([B][Sr][H][128] bf16) and lse_dst[p] ([B][H][Sr] fp32) of the
 *   rank p owning each row's stretch of the sequence. All of them 16-byte
 *   aligned.
 * sa_ulysses_dispatch_units / sa_ulysses_combine_units: the same for the unit
 *   slots j0 <= j < j1 of every owner only (slot j of rank r is unit
 *   r*n_per + j), so that the exchange of one group of slots can run while
 *   attention works on another; the plain forms are [0, n_per).
 * Neither waits on another rank: the caller orders them against the peers'
 * use of the same buffers (stream-ordered collectives before and after).
 * Their kernels run 128-thread blocks at no more than 32 registers a thread,
 * so that a block fits on an SM beside an attention block.
 */
SA_API int sa_ipc_alloc(size_t bytes, void** ptr);
SA_API int sa_ipc_free(void* ptr);
SA_API int sa_ipc_get_handle(void* ptr, uint8_t handle[64]);
SA_API int sa_ipc_open_handle(const uint8_t handle[64], void** ptr);
SA_API int sa_ipc_close(void* ptr);
SA_API int sa_ulysses_dispatch(int T, const void* const* src, const int64_t* src_strides, int B,
                               int Sr, int H, int D, int P, int rank, int n_per,
                               void* const* dst, cudaStream_t stream);
SA_API int sa_ulysses_combine(const void* out_units, const float* lse_units, int B, int Sr, int H,
                              int D, int P, int rank, int n_per, void* const* out_dst,
                              float* const* lse_dst, cudaStream_t stream);
SA_API int sa_ulysses_dispatch_units(int T, const void* const* src, const int64_t* src_strides,
                                     int B, int Sr, int H, int D, int P, int rank, int n_per,
                                     int j0, int j1, void* const* dst, cudaStream_t stream);
SA_API int sa_ulysses_combine_units(const void* out_units, const float* lse_units, int B, int Sr,
                                    int H, int D, int P, int rank, int n_per, int j0, int j1,
                                    void* const* out_dst, float* const* lse_dst,
                                    cudaStream_t stream);

/*
 * The status word. No counterpart in the reference, whose kernels cannot
 * report a stalled wait.
 * sa_status_create: one int32 in mapped, portable page-locked host memory,
 *   set to SA_DEV_OK; returns its host address (NULL on failure, see
 *   sa_last_error). sa_status_device_pointer gives the address kernels use
 *   (the same address where the device uses unified addressing);
 *   sa_status_destroy frees it.
 * sa_check_status: reads a host-readable status word without synchronising:
 *   SA_OK if no kernel reported a failure, else SA_ETIMEOUT (with a message)
 *   and the word is reset to SA_DEV_OK. A launch's report becomes visible once
 *   the launch has run, so a caller that needs a verdict on a given launch
 *   synchronises its stream first.
 */
SA_API int32_t* sa_status_create(void);
SA_API int sa_status_device_pointer(int32_t* status, int32_t** device_ptr);
SA_API int sa_status_destroy(int32_t* status);
SA_API int sa_check_status(int32_t* status);

/*
 * Test support for failure detection: one warp waits on an mbarrier that
 * nobody arrives on, with a limit of limit_ns (1 us .. 1 s). The wait gives
 * up, the kernel writes SA_DEV_WAIT_TIMEOUT into *status (device-writable)
 * and returns; no copy or MMA is in flight, so the context stays usable. No
 * counterpart in the reference.
 */
SA_API int sa_selftest_wait_timeout(int32_t* status, uint64_t limit_ns, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* SINKATTN_H_ */
