/*
 * fftsparse_b200.h -- C ABI of the B200 (sm_100a) FFTSparse prefill hot path.
 *
 * The reference operator is `myattn_prefill` in attn_src/fft_attn/my_attn_v7.py
 * (lines 454-792): block mean pooling, FFT lag correlation, stripe/diffuse head
 * classification, four auxiliary block masks, and a call into the third-party
 * `block_sparse_attn_func` CUDA kernel (my_attn_v7.py:775-786).  ffts_pool +
 * ffts_block_mask + ffts_sparse_attn_fwd, in that order, replace the whole of
 * it; each cites the reference lines it replaces.  The other entry points serve
 * the operator's caller (ffts_rope_pool: its RoPE, layout and the pooling in one
 * pass) and the sharded prefill (query-row ranges, stores into peer GPUs'
 * buffers, CUDA IPC mapping, copy-engine row pushes, epoch flags).
 *
 * Conventions
 *   - All tensor arguments are DEVICE pointers with explicit element strides.
 *     The caller owns every buffer (inputs, outputs and the workspace); the
 *     library allocates nothing per call.
 *   - Work is enqueued on `stream` (a cudaStream_t passed as void*); no compute
 *     entry point synchronises the host with the device (the IPC mapping calls
 *     are one-time setup and may).
 *   - Every entry point returns FFTS_OK (0) or a negative FFTS_E* code; the
 *     message for the last failure on the calling thread is returned by
 *     ffts_last_error_string().  No C++ exception crosses this boundary.
 *   - dtype codes: FFTS_DTYPE_F32 = 0, FFTS_DTYPE_BF16 = 1.
 *   - q is [B, H, L, D]; k and v are [B, Hkv, L, D] with H % Hkv == 0 (the
 *     reference's callers pass Hkv == H, i.e. repeat_kv-expanded k/v,
 *     eval/LongBench/pred.py:204-205; Hkv < H is accepted as GQA).
 *   - Block masks are packed bits: word (b, h, i, w) bit t <=> key block
 *     j = 32*w + t is kept for query block i.  Row stride is W = ceil(N/32).
 *   - The first call on a device uploads the library's constant tables (FFT
 *     twiddles and log10 weights) to that device with a synchronous copy; make
 *     that first call (or ffts_init) before any stream capture.
 */
#ifndef FFTSPARSE_B200_H
#define FFTSPARSE_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define FFTS_API __attribute__((visibility("default")))
#else
#define FFTS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define FFTS_OK              0
#define FFTS_E_INVALID     (-1)  /* bad shape, stride, dtype or parameter  */
#define FFTS_E_UNSUPPORTED (-2)  /* valid but not implemented (e.g. D)     */
#define FFTS_E_CUDA        (-3)  /* a CUDA runtime call failed              */
#define FFTS_E_WORKSPACE   (-4)  /* workspace too small or misaligned       */
#define FFTS_E_DEVICE      (-5)  /* not an sm_100 device                    */

#define FFTS_DTYPE_F32  0
#define FFTS_DTYPE_BF16 1

#define FFTS_SEL_THRESHOLD 0   /* correlation_selection_mode="threshold" */
#define FFTS_SEL_TOPK      1   /* correlation_selection_mode="topk"      */

#define FFTS_MAX_DIAG_SAMPLES 64

/*
 * Derived integer/float parameters of one mask selection.  They are computed
 * on the host exactly as myattn_prefill derives them (my_attn_v7.py:532-540,
 * 583-594, 626-634); fftsparse_b200/params.py fills this struct.
 */
typedef struct ffts_mask_params {
  int32_t n_blocks;          /* N = ceil(L / block_size)                       */
  int32_t block_size;
  int32_t keep_sink;         /* :537                                           */
  int32_t keep_recent;       /* :538                                           */
  int32_t local_window;      /* :539-540                                       */
  int32_t corr_on;           /* enable_correlation_mask and N > corr top-k :579 */
  int32_t corr_mode;         /* FFTS_SEL_*                                      */
  float   corr_threshold;    /* fp32(corr_threshold)          (:206-208)        */
  float   corr_quantile;     /* fp32(1 - correlation_topk_ratio) (:199)         */
  int32_t exclude_tau;       /* local_window + 1              (:137)            */
  int32_t sink_tau_raw;      /* N - keep_sink - 5 (may be < 0) (:138)           */
  int32_t remote_start;      /* max(local_window, keep_recent-1)+1 (:183-184)   */
  int32_t n_diag_samples;    /* length of diag_taus                             */
  int32_t diag_taus[FFTS_MAX_DIAG_SAMPLES]; /* sampled lags (:325-334)          */
  int32_t stripe_all_diffuse;/* remote_start >= N-1 (:318-321)                  */
  float   stripe_threshold;  /* fp32(stripe_threshold)         (:363)           */
  float   qk_topk_ratio;     /* fp32(qk_topk_ratio)            (:271-272)       */
  int32_t col_on;            /* enable_column_mask and N > 1   (:622)           */
  int32_t col_start;         /* (:626-634, :429-430)                            */
  int32_t col_end;
  int32_t col_topk;          /* (:436-437)                                      */
  int32_t last_on;           /* enable_last_block_mask         (:558)           */
  int32_t last_topk;         /* min(128, N)                    (:65)            */
} ffts_mask_params;

/* Library version (major*10000 + minor*100 + patch). */
FFTS_API int32_t ffts_version(void);

/* Message for the last error returned on this thread ("" if none). */
FFTS_API const char *ffts_last_error_string(void);

/* Upload the constant tables to `device` (idempotent, synchronous). */
FFTS_API int32_t ffts_init(int32_t device);

/*
 * Block mean pooling.  Replaces block_mean_pool (my_attn_v7.py:105-114) as
 * called at :554-555: out[b, h, n, d] = mean over the block_size tokens of
 * block n (the partial last block is zero-padded and still divided by
 * block_size), rounded to the input dtype.  out is contiguous [B, H, N, D].
 */
FFTS_API int32_t ffts_pool(const void *x, int32_t dtype, int64_t B, int64_t H, int64_t L,
                  int64_t D, int64_t stride_b, int64_t stride_h, int64_t stride_l,
                  int32_t block_size, void *out, void *stream);

/*
 * The caller's rotary embedding, head-major layout and block pooling in one
 * pass, for one sequence.  Replaces, ahead of myattn_prefill, HF
 * apply_rotary_pos_emb on q and k as the caller applies it
 * (eval/LongBench/pred.py:191-194), the views of q/k/v as [1, H, L, D], and
 * the pooling of q and k (ffts_pool; my_attn_v7.py:105-114 at :554-555), so
 * that ffts_block_mask can take the pooled blocks directly.
 *   q_src [L, q_ld], k_src [L, k_ld], v_src [L, v_ld]: token-major bf16
 *     projections (head h in columns [h*D, h*D + D)); v_src may be NULL.
 *   cos, sin: bf16 [L, D] with row stride cs_ld.
 *   q_out [Hq, L, D], k_out / v_out [Hkv, L, D]: head-major, contiguous.
 *   q_pooled [Hq, N, D], k_pooled [Hkv, N, D], N = ceil(L / block_size).
 * out = bf16(bf16(x * cos) + bf16(rotate_half(x) * sin)), each operation in
 * fp32 (the torch bf16 expression op by op); pooled blocks are exactly those
 * ffts_pool computes from q_out / k_out.  D must be 128; bf16 only.
 */
FFTS_API int32_t ffts_rope_pool(const void *q_src, int64_t q_ld, const void *k_src, int64_t k_ld,
                  const void *v_src, int64_t v_ld, int64_t L, int64_t Hq, int64_t Hkv, int64_t D,
                  const void *cos, const void *sin, int64_t cs_ld, int32_t block_size,
                  void *q_out, void *k_out, void *v_out, void *q_pooled, void *k_pooled,
                  void *stream);

/*
 * The caller's QKV projection GEMM with the rotary embedding, head-major layout
 * and block pooling in its epilogue (tcgen05 tensor cores; the projection
 * itself never reaches memory unless proj_out is given).  Replaces, ahead of
 * myattn_prefill, the q_proj / k_proj / v_proj Linear calls of the HF attention
 * forward the caller runs (eval/LongBench/pred.py:177-194) and then everything
 * ffts_rope_pool replaces.
 *   x [B, L, hidden] bf16, row stride x_stride_l, sequence stride x_stride_b
 *     (ignored for B = 1); hidden, the strides, w_ld and cs_ld multiples of 8.
 *   w [(Hq + 2 Hkv) * D, hidden] bf16 (row stride w_ld): the q_proj, k_proj and
 *     v_proj weights stacked row-wise, torch Linear layout.
 *   bias [(Hq + 2 Hkv) * D] bf16 or NULL, added in fp32 before rounding.
 *   cos, sin: bf16 [L, D] (row stride cs_ld), the same positions for every sequence.
 *   q_out [B, Hq, L, D], k_out / v_out [B, Hkv, L, D]; q_pooled [B, Hq, N, D],
 *     k_pooled [B, Hkv, N, D], N = ceil(L / block_size), block_size 16..128.
 *   proj_out: NULL, or [B, L, proj_ld] receiving the bf16 projection before RoPE.
 *   workspace: device memory of ffts_qkv_workspace_bytes(L) bytes, 16-byte aligned
 *     (the cos / sin rows re-laid for coalesced loads); contents need not be kept.
 *   status: NULL or an int32 device word; a bounded wait that times out stores
 *     6 (copy producer), 7 (MMA issuer) or 8 (epilogue) and the outputs are
 *     invalid; 9 means the shared memory was misaligned and nothing ran.
 * proj = bf16(fp32 sum over hidden of x * w (+ bias)); q, k, v and the pooled
 * blocks are bit-identical to ffts_rope_pool applied to proj.  D must be 128.
 */
FFTS_API int32_t ffts_qkv_rope_pool(const void *x, int64_t B, int64_t L, int64_t hidden,
                  int64_t x_stride_l, int64_t x_stride_b, const void *w, int64_t w_ld,
                  const void *bias, int64_t Hq, int64_t Hkv, int64_t D, const void *cos,
                  const void *sin, int64_t cs_ld, int32_t block_size, void *q_out, void *k_out,
                  void *v_out, void *q_pooled, void *k_pooled, void *proj_out, int64_t proj_ld,
                  void *workspace, int64_t workspace_bytes, int32_t *status, void *stream);

/* Workspace bytes ffts_qkv_rope_pool needs for L tokens per sequence. */
FFTS_API int64_t ffts_qkv_workspace_bytes(int64_t L);

/*
 * Decode attention for one new token per sequence over the KV cache.  Replaces
 * the caller's eager decode branch (eval/LongBench/pred.py:306-322:
 * softmax(q k^T / sqrt(D)) v over the repeat_kv-expanded cache) after the
 * prefill, reading the cache un-expanded.
 *   q [B, H, D] bf16 (strides q_stride_b, q_stride_h; unit over D);
 *   k_cache, v_cache [B, Hkv, Lk, D] bf16 with strides (b, h, l), H % Hkv == 0,
 *     H / Hkv <= 16 (the layout ffts_rope_pool writes and an HF cache stores);
 *   out [B, H, D] bf16 (strides out_stride_b, out_stride_h);
 *   mask: NULL, or the caller's additive attention mask for this step, [B, Lk]
 *     (row stride mask_stride_b, unit over keys; dtype FFTS_DTYPE_F32 or
 *     FFTS_DTYPE_BF16), added to q k^T / sqrt(D) before the softmax as
 *     pred.py:311-313 adds attention_mask[:, :, :, :Lk] (0 keeps a key, a large
 *     negative value such as the dtype's minimum drops it; padding of a batch).
 * The keys are split over `splits` CTAs per KV head (fewer when Lk is short);
 * the workspace holds their partial results (ffts_decode_workspace_bytes).
 * fp32 scores, softmax and accumulation; D must be 128.
 */
FFTS_API int64_t ffts_decode_workspace_bytes(int64_t B, int64_t H, int64_t Hkv, int64_t splits);
FFTS_API int32_t ffts_decode_attn(const void *q, int64_t q_stride_b, int64_t q_stride_h,
                  const void *k_cache, const int64_t *k_strides /* b,h,l */,
                  const void *v_cache, const int64_t *v_strides /* b,h,l */,
                  int64_t B, int64_t H, int64_t Hkv, int64_t Lk, int64_t D, int64_t splits,
                  void *workspace, int64_t workspace_bytes, void *out,
                  int64_t out_stride_b, int64_t out_stride_h,
                  const void *mask, int32_t mask_dtype, int64_t mask_stride_b, void *stream);

/* Bytes of device workspace ffts_block_mask / ffts_prefill need. */
FFTS_API int64_t ffts_mask_workspace_bytes(int64_t B, int64_t H, int64_t N, int64_t D);

/*
 * Block-mask selection from pooled blocks.  Replaces my_attn_v7.py:546-641:
 * create_deterministic_block_mask (:74-98), create_last_block_query_mask
 * (:54-72), batch_fft_cross_correlation (:117-157),
 * create_correlation_block_mask (:160-227), compute_block_scores (:234-249),
 * compute_stripe_variance (:301-383), create_qk_topk_block_mask (:256-294),
 * create_column_block_mask (:390-447) and their union.
 *
 *   qb, kb      pooled blocks, contiguous [B, H, N, D] and [B, Hkv, N, D]
 *   mask_bits   out: uint32 [B, H, N, W]
 *   row_count   out: int32 [B, H, N] (number of kept blocks per row), or NULL
 *   corr        out: fp32 [B, H, N] final lag scores (corr_causal), or NULL
 *   corr_sum    out: fp32 [B, H, N] raw lag sums (corr_causal_sum), or NULL
 *   is_stripe   out: uint8 [B, H] (1 = stripe head), or NULL
 *   stripe_var  out: fp32 [B, H] mean normalised diff variance, or NULL
 *   workspace   >= ffts_mask_workspace_bytes(...) bytes, 256-byte aligned
 */
FFTS_API int32_t ffts_block_mask(const void *qb, const void *kb, int32_t dtype, int64_t B,
                        int64_t H, int64_t Hkv, int64_t D,
                        const ffts_mask_params *params, uint32_t *mask_bits,
                        int32_t *row_count, float *corr, float *corr_sum,
                        uint8_t *is_stripe, float *stripe_var, void *workspace,
                        int64_t workspace_bytes, void *stream);

/*
 * ffts_block_mask without a workspace argument.  No counterpart in the
 * reference.  It is for callers that may not allocate device memory when they
 * run the selection, such as an engine that reserves all GPU memory for its
 * own pool at start-up, or a plugin hook that must not call cudaMalloc because
 * it can synchronise the device.  It runs the same kernels on a scratch array
 * of 8 MiB compiled into the library (resident on every GPU that loads it) and
 * allocates nothing.  Shapes whose ffts_mask_workspace_bytes(...) exceeds 8 MiB
 * are rejected with FFTS_E_WORKSPACE (128K tokens x 32 heads needs about
 * 4.2 MB).  The first call on a device looks up the scratch address and may
 * upload the constant tables: make it before any stream capture.  All calls on
 * a device share the scratch, so calls whose kernels overlap on the GPU race;
 * serialise them.
 */
FFTS_API int32_t ffts_block_mask_noalloc(const void *qb, const void *kb, int32_t dtype,
                                         int64_t B, int64_t H, int64_t Hkv, int64_t D,
                                         const ffts_mask_params *params,
                                         uint32_t *mask_bits, int32_t *row_count,
                                         float *corr, float *corr_sum, uint8_t *is_stripe,
                                         float *stripe_var, void *stream);

/*
 * Expand packed bits to the reference's bool block mask [B, H, N, N] (uint8),
 * i.e. the `base_blockmask` argument at my_attn_v7.py:780.
 */
FFTS_API int32_t ffts_unpack_mask(const uint32_t *mask_bits, int64_t B, int64_t H, int64_t N,
                         uint8_t *out, void *stream);

/*
 * The selected blocks as a CSR index list, the block index list a block-sparse
 * kernel that takes indices consumes (the reference passes the bool form,
 * base_blockmask, my_attn_v7.py:780).  rows = B * H * N, in the [B, H, N]
 * order of the packed bits.
 *   ffts_mask_row_ptr: row_ptr[i] = sum of row_count[0..i) (int64, rows + 1
 *     entries; row_ptr[rows] = number of kept blocks), from the row_count that
 *     ffts_block_mask writes.
 *   ffts_mask_col_idx: col_idx[row_ptr[i] .. row_ptr[i+1]) = the kept key
 *     blocks of row i in ascending order (int32).  capacity = entries col_idx
 *     holds.  A row whose popcount differs from its row_ptr span, or that would
 *     end past capacity, is not written and *status (int32, device) is set to 1.
 */
FFTS_API int32_t ffts_mask_row_ptr(const int32_t *row_count, int64_t rows, int64_t *row_ptr, void *stream);
FFTS_API int32_t ffts_mask_col_idx(const uint32_t *mask_bits, int64_t rows, int64_t N,
                                   const int64_t *row_ptr, int32_t *col_idx, int64_t capacity,
                                   int32_t *status, void *stream);

/*
 * Block-sparse causal attention forward (bf16 in, fp32 accumulate, bf16 out).
 * Replaces block_sparse_attn_func (my_attn_v7.py:775-786; package
 * block_sparse_attn 0.0.2) with head_mask_type all 1 (:772), p_dropout 0,
 * scale 1/sqrt(D).  Query row t of block i attends to key s of block j iff
 * bit (i, j) is set and (not causal or s <= t).  Rows with no kept key
 * produce zeros.  out[b, t, h, :] is written at
 * out + b*out_stride_b + t*out_stride_l + h*out_stride_h (the reference's
 * [1, L, H*D] return layout, :789-790, when strides are (L*H*D, H*D, D)).
 * D must be 128; block_size 32, 64 or 128; q/k/v strides multiples of 8
 * elements with unit stride in D.
 */
FFTS_API int32_t ffts_sparse_attn_fwd(const void *q, const void *k, const void *v, int64_t B,
                             int64_t H, int64_t Hkv, int64_t L, int64_t D,
                             const int64_t *q_strides /* b,h,l */,
                             const int64_t *k_strides /* b,h,l */,
                             const int64_t *v_strides /* b,h,l */,
                             const uint32_t *mask_bits, int32_t block_size,
                             int32_t causal, void *out,
                             const int64_t *out_strides /* b,h,l */,
                             int32_t *status, void *stream);

/*
 * ffts_sparse_attn_fwd for the query rows [row_lo, row_hi) only (row_lo a
 * multiple of 128; row_hi a multiple of 128 or L).  The mask, q/k/v and all
 * other arguments are those of the whole call; query row t is written at
 * output row t - row_lo.  No counterpart in the reference: a sharded caller
 * computes the output in row chunks so that the all-gather of one chunk runs
 * while the next is computed.
 */
FFTS_API int32_t ffts_sparse_attn_fwd_rows(const void *q, const void *k, const void *v, int64_t B,
                             int64_t H, int64_t Hkv, int64_t L, int64_t D,
                             const int64_t *q_strides /* b,h,l */,
                             const int64_t *k_strides /* b,h,l */,
                             const int64_t *v_strides /* b,h,l */,
                             const uint32_t *mask_bits, int32_t block_size,
                             int32_t causal, int64_t row_lo, int64_t row_hi, void *out,
                             const int64_t *out_strides /* b,h,l */,
                             int32_t *status, void *stream);

/*
 * ffts_sparse_attn_fwd_rows that also stores every output row into each of
 * peer_out[0..n_peers), n_peers <= 15: other GPUs' buffers mapped into this
 * process (CUDA IPC; ffts_ipc_open) with the strides of out, 16-byte aligned.
 * The stores are made visible system-wide before the kernel completes, so a
 * flag stored after it on the same stream (ffts_signal) tells a peer that its
 * rows have arrived.  No counterpart in the reference: the sharded prefill's
 * output all-gather, fused into the attention epilogue over NVLink.
 */
FFTS_API int32_t ffts_sparse_attn_fwd_push(const void *q, const void *k, const void *v, int64_t B,
                             int64_t H, int64_t Hkv, int64_t L, int64_t D,
                             const int64_t *q_strides /* b,h,l */,
                             const int64_t *k_strides /* b,h,l */,
                             const int64_t *v_strides /* b,h,l */,
                             const uint32_t *mask_bits, int32_t block_size,
                             int32_t causal, int64_t row_lo, int64_t row_hi, void *out,
                             const int64_t *out_strides /* b,h,l */,
                             void *const *peer_out, int32_t n_peers,
                             int32_t *status, void *stream);

/*
 * One pitched copy (cudaMemcpy2DAsync, any direction): height rows of width
 * bytes from src (rows src_pitch bytes apart) to dst (rows dst_pitch apart) on
 * stream.  No counterpart in the reference, whose operator takes device tensors
 * only: fftsparse_b200.myattn_prefill_host uses it to read each head chunk's
 * output columns back into the caller's [B, L, H*D] host buffer while later
 * chunks are copied in and computed.
 */
FFTS_API int32_t ffts_copy_2d(void *dst, int64_t dst_pitch, const void *src, int64_t src_pitch, int64_t width,
                  int64_t height, void *stream);

/*
 * Copy-engine all-gather support for the sharded prefill (fftsparse_b200/dist.py,
 * PeerGather).  No counterpart in the reference, which runs on one GPU: a rank
 * maps its peers' output buffers (CUDA IPC), pushes each finished row chunk of
 * its heads into them with a strided copy on a copy stream while the next chunk
 * is computed, then stores an epoch number into each peer's flag; the consumer
 * waits until every flag reached the epoch.
 *
 * ffts_ipc_handle: a 64-byte IPC handle of the allocation holding ptr, and ptr's
 *   offset inside it.  ffts_ipc_open: the peer-side address of that buffer.
 * ffts_copy_rows: height rows of width bytes, pitch bytes apart on both sides,
 *   from src to dsts[i] on streams[i] (cudaStream_t), i < n; with a non-NULL
 *   `after` (cudaEvent_t) every stream first waits for that event.
 * ffts_signal: store value into *flags[i] (release, system scope) on streams[i],
 *   after that stream's earlier work, i < n <= 1024.  ffts_wait_flags: wait
 *   until flags[0..n) >= epoch (acquire), n <= 32; bounded at about 2 s, after
 *   which *status = 5 and the wait returns.
 */
FFTS_API int32_t ffts_ipc_handle(const void *ptr, void *handle, int64_t *offset);
FFTS_API int32_t ffts_ipc_open(const void *handle, int64_t offset, void **ptr);
FFTS_API int32_t ffts_ipc_close(void *ptr, int64_t offset);
FFTS_API int32_t ffts_copy_rows(void *const *dsts, void *const *streams, int32_t n, const void *src,
                               int64_t pitch, int64_t width, int64_t height, void *after);
FFTS_API int32_t ffts_signal(int32_t *const *flags, void *const *streams, int32_t n, int32_t value);
FFTS_API int32_t ffts_wait_flags(const int32_t *flags, int32_t n, int32_t epoch, int32_t *status,
                                 void *stream);

/*
 * Bounds-checked build.  No counterpart in the reference (its kernels are
 * library calls).  The library also builds as libfftsparse_b200_checked.so with
 * every data-dependent or ragged-edge index of its kernels tested against its
 * extent; a failed test skips the access and is recorded per source file on the
 * device, nothing traps.  ffts_bounds_check_enabled() is 1 in that build and 0
 * in the normal one.  ffts_bounds_report() reads the records of the current
 * device (zeroing them when clear != 0), fills up to max_records entries and
 * returns the number of source files with a failed check (0 in the normal build),
 * or a negative FFTS_E* code.
 */
typedef struct ffts_bounds_record {
  char file[48];   /* base name of the kernel's source file */
  int32_t line;    /* source line of the file's first failed check */
  uint32_t count;  /* failed checks in that file since the last clear */
  int64_t block;   /* linear block index of the first failure */
} ffts_bounds_record;

FFTS_API int32_t ffts_bounds_check_enabled(void);
FFTS_API int32_t ffts_bounds_report(ffts_bounds_record *records, int32_t max_records, int32_t clear);

#ifdef __cplusplus
}
#endif

#endif /* FFTSPARSE_B200_H */
