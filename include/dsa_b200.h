/*
 * dsa_b200.h — C ABI of the B200 DeepSeek Sparse Attention forward.
 *
 * Three sm_100a CUDA stages behind plain pointers and sizes:
 *   stage 1  Lightning Indexer scores   I[b,t,s] = sum_j w[b,t,j] * ReLU(<q[b,t,j,:], k[b,s,:]>)
 *            (tcgen05 tensor cores for bf16 / e4m3 inputs, CUDA cores otherwise)
 *   stage 2  per-row top-K threshold (k-th largest, ties kept) + the kept set, as an
 *            ascending index list or as a bitmap
 *   stage 3  attention over the kept keys: a masked flash attention on tcgen05 over the
 *            bitmap (bf16/fp16, head size 64 or 128), else a gather with an fp32 online softmax
 *
 * Conventions shared by every entry point
 *   - All pointers are device pointers on the current CUDA device, row-major
 *     and contiguous in the layouts given below, 16-byte aligned.  The _ex
 *     entry points take the input tensors with arbitrary element strides
 *     (struct dsa_layout) instead.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *     Every call only enqueues work: nothing synchronises, nothing allocates.
 *     The caller owns every buffer, outputs and workspaces included.
 *   - Returns DSA_OK (0) or a negative dsa_status.  On error,
 *     dsa_last_error_string() (per host thread) describes the failure.
 *   - Query rows: a call covers T_q query rows of each batch whose absolute
 *     positions are q_row0 .. q_row0+T_q-1 (so a GPU can own a block of
 *     rows of a longer sequence), against T_k key positions 0..T_k-1.  Key s
 *     is causal for query t iff s <= t.
 *   - dtype codes: DSA_F32, DSA_BF16, DSA_F16 (element type of the named
 *     tensors; everything else is fp32 / int32 as stated).
 *
 * Reference interfaces replaced (Infatoshi/dsa-cpu-topk, file:line):
 *   dsa_indexer_scores         lightning_indexer.py:100-125  indexer_scores_triton / _indexer_score_kernel
 *   dsa_topk_select            dsa_attention.py:343-344      scores.topk(k)[..., -1:] on the GPU, and
 *                              topk_avx512.cpp:226-257       topk_threshold / topk_threshold_batch_merge
 *   dsa_sparse_attn_threshold  dsa_attention.py:298-324      sparse_attention_with_threshold_triton
 *   dsa_sparse_attn            dsa_attention.py:72-87        (gather form of the selection, naive variant)
 *   dsa_kept_bitmap,           dsa_attention.py:230-324      _sparse_attn_threshold_kernel: its per-tile
 *   dsa_topk_select_bitmap,                                  mask (scores >= thr, s <= t) as a bitmap, and
 *   dsa_sparse_attn_bitmap
 *                                                            the masked flash attention on the tensor cores
 *   dsa_forward                dsa_attention.py:327-344      dsa_attention_split_triton (and the fused
 *                              dsa_attention.py:196-227      dsa_attention_triton, same result)
 */
#ifndef DSA_B200_H
#define DSA_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DSA_API __attribute__((visibility("default")))
#else
#define DSA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    DSA_OK = 0,
    DSA_ERR_INVALID = -1,      /* bad shape, pointer, alignment or argument */
    DSA_ERR_UNSUPPORTED = -2,  /* valid request this build cannot run (e.g. dtype) */
    DSA_ERR_CUDA = -3,         /* a CUDA runtime call failed (launch, attribute) */
    DSA_ERR_TIMEOUT = -4       /* a kernel gave up waiting on its own pipeline (see dsa_device_status) */
} dsa_status;

/* DSA_FP8_E4M3 is accepted for the indexer inputs (q, k) only. */
typedef enum { DSA_F32 = 0, DSA_BF16 = 1, DSA_F16 = 2, DSA_FP8_E4M3 = 3 } dsa_dtype;

/*
 * Strided inputs and row blocks (the _ex entry points).
 *
 * Element strides of each input tensor, outermost first; the innermost
 * dimension (DI, DQ or DV) is always contiguous:
 *   q_idx [B, T_q, HI, DI]  -> q[0..2]  = batch, row, head strides
 *   k_idx [B, T_k, DI]      -> k[0..1]  = batch, row
 *   w_idx [B, T_q, HI]      -> w[0..1]  = batch, row (heads contiguous)
 *   Q     [B, T_q, HQ, DQ]  -> Q[0..2]  = batch, row, head
 *   K, V  [B, T_k, HQ, D]   -> K[0..2], V[0..2]
 * A batch stride may be 0 (every batch reads the same tensor).  For example
 * K and V sliced out of a fused [B, T, 3, HQ, D] projection have row stride
 * 3*HQ*D and head stride D; no copy is needed.
 *
 * row_bstep: batch b's query rows sit at absolute positions
 * q_row0 + b*row_bstep + i (i < T_q); 0 in the plain contiguous case.  With
 * key-side batch strides of 0 this runs several row blocks of ONE sequence
 * in one launch, e.g. the two zig-zag blocks r and 2N-1-r that a GPU owns when
 * a sequence's query rows are split across N GPUs: B = 2, T_q = block rows,
 * q_row0 = r*T_q, row_bstep = (2N-1-2r)*T_q.
 *
 * The outputs (scores, O, thresholds, lists, bitmaps) stay contiguous.  Byte
 * strides that are not multiples of 16 run on the CUDA-core / gather kernels
 * instead of the tensor-core ones.  No counterpart in the reference, whose
 * Triton kernels take strides per tensor (lightning_indexer.py:116-124,
 * dsa_attention.py:313-323) but run one contiguous sequence per batch.
 */
typedef struct dsa_layout {
    int64_t q[3], k[2], w[2], Q[3], K[3], V[3];
    int64_t row_bstep;
} dsa_layout;

/* The contiguous layout of the shapes given (row_bstep 0). */
DSA_API void dsa_layout_contiguous(dsa_layout* out, int64_t T_q, int64_t T_k, int64_t HI,
                                   int64_t DI, int64_t HQ, int64_t DQ, int64_t DV);

/* Library version, (major << 16) | minor. */
DSA_API int dsa_version(void);

/* Message of the last failing call on this host thread ("" if none). */
DSA_API const char* dsa_last_error_string(void);

/*
 * Failure detection.  Every wait inside a kernel (the tensor-core indexer's
 * mbarrier pipeline) is bounded by 2 s of device time; a kernel that runs out
 * abandons its work, frees its tensor memory and sets a device flag instead of
 * hanging.  This call synchronises `stream`, then reads and clears that flag
 * for the current device: DSA_OK, or DSA_ERR_TIMEOUT if a launch since the
 * last call gave up (its outputs are incomplete).  No counterpart in the
 * reference (it has no device-side waits).
 */
DSA_API int dsa_device_status(void* stream);

/*
 * Checked build.  libdsa_b200_checked.so is this library compiled with
 * -DDSA_DEBUG_CHECKS (`python dsa-cpu-topk_b200/build.py --checked`): every
 * guarded access checks its index first, and a failing check sets a bit in a
 * device flag word instead of performing the access (no trap, no fault):
 *   1  a kept-index list entry outside 0 <= s <= t (dsa_sparse_attn): skipped
 *   2  a top-K candidate past the candidate buffer: not stored
 *   4  a decoded indexer tile or attention unit outside the launch's shape
 * dsa_debug_status synchronises `stream`, then returns the OR of the bits set
 * since the last call and clears them (always 0 in the normal build);
 * dsa_debug_checks_enabled says which build is loaded.  No counterpart in the
 * reference, which validates on the host only (topk_avx512.cpp:227-235).
 */
DSA_API int dsa_debug_checks_enabled(void);
DSA_API int dsa_debug_status(void* stream);

/*
 * Stage 1 — Lightning Indexer scores.
 *   q       [B, T_q, HI, DI]  dtype      indexer queries of rows q_row0..q_row0+T_q-1
 *   k       [B, T_k, DI]      dtype      shared indexer key
 *   w       [B, T_q, HI]      fp32       per-query head weights
 *   scores  [B, T_q, T_k]     fp32 out   score of causal entries; entries s > t are
 *                                        written -inf when fill_upper != 0, else left
 *                                        untouched or -inf (stages 2/3 never read them)
 * dtype DSA_BF16 with DI in {64, 128} and DSA_FP8_E4M3 with DI in {128, 256}
 * run on the tcgen05 tensor cores; other shapes and dtypes run the fp32
 * CUDA-core kernel (IEEE fp32 products and sums).
 * Replaces lightning_indexer.py:100-125 (which requires DI a power of two).
 */
DSA_API int dsa_indexer_scores(const void* q, const void* k, const float* w, float* scores,
                       int64_t B, int64_t T_q, int64_t T_k, int64_t q_row0,
                       int64_t HI, int64_t DI, int dtype, int fill_upper, void* stream);

/* dsa_indexer_scores over strided q/k/w and row blocks (layout may be NULL:
 * contiguous).  Only layout->q, k, w and row_bstep are read. */
DSA_API int dsa_indexer_scores_ex(const void* q, const void* k, const float* w, float* scores,
                                  int64_t B, int64_t T_q, int64_t T_k, int64_t q_row0,
                                  int64_t HI, int64_t DI, int dtype, int fill_upper,
                                  const dsa_layout* layout, void* stream);

/*
 * FP8 indexer with per-row scales.  No counterpart in the reference (its
 * Triton indexer is fp32 only, lightning_indexer.py:54-97); the DeepSeek-V3.2
 * indexer runs q/k in FP8 with scales this way.
 *   dsa_quantize_fp8_rows: rows of D values (fp32/bf16/fp16, row r at
 *     x + r*row_stride) -> out_e4m3 [rows, D] = e4m3(x / s) and scale_out[r] = s
 *     = max|x_r| / 448 (1 for an all-zero row).
 *   dsa_indexer_scores_fp8: I[b,t,s] = k_scale[b,s] * sum_j w[b,t,j] *
 *     ReLU(<q8[b,t,j,:], k8[b,s,:]>), s <= t.  q8 / k8 are e4m3 (layouts as in
 *     dsa_indexer_scores, strides through layout, may be NULL); k_scale is fp32
 *     [B, T_k] (or [1, T_k] when k's batch stride is 0).  Per-(query, head)
 *     scales of q are folded into w by the caller: w'[b,t,j] = w[b,t,j] *
 *     q_scale[b,t,j] (exact for positive scales, since ReLU(c x) = c ReLU(x)).
 */
DSA_API int dsa_quantize_fp8_rows(const void* x, int dtype, int64_t rows, int64_t D, int64_t row_stride,
                                  void* out_e4m3, float* scale_out, void* stream);
DSA_API int dsa_indexer_scores_fp8(const void* q8, const void* k8, const float* w, const float* k_scale,
                                   float* scores, int64_t B, int64_t T_q, int64_t T_k, int64_t q_row0,
                                   int64_t HI, int64_t DI, int fill_upper, const dsa_layout* layout,
                                   void* stream);

/*
 * Stage 2 — per-row top-K threshold and kept-index list (radix select).
 *   scores   n_rows rows of row_len fp32, row r at scores + r*row_stride
 *   thr_out  [n_rows] fp32 out: the k-th largest value of the row (as
 *            torch.topk(k).values[..., k-1]; -0.0 and +0.0 are one value)
 *   idx_out  [n_rows, idx_cap] int32 out (may be NULL): ascending positions s
 *            with scores[s] >= thr (and s <= t when causal); at most idx_cap written
 *   cnt_out  [n_rows] int32 out (may be NULL): number of kept positions, which
 *            can exceed k (ties are kept) and idx_cap (then the list is truncated)
 * causal != 0: row r is query t = q_row0 + r % rows_per_batch and entries
 * s > t count as -inf whatever is stored there (they are not read).
 * Requires 1 <= k <= row_len.
 */
DSA_API int dsa_topk_select(const float* scores, int64_t n_rows, int64_t row_len, int64_t row_stride,
                    int64_t rows_per_batch, int64_t q_row0, int causal, int64_t k,
                    float* thr_out, int32_t* idx_out, int32_t* cnt_out, int64_t idx_cap,
                    void* stream);

/* dsa_topk_select with row blocks and an optional bitmap: causal row r is
 * query t = q_row0 + (r / rows_per_batch)*row_bstep + r % rows_per_batch.
 * bits (may be NULL) receives the kept-set bitmap of dsa_kept_bitmap
 * (requires row_stride == row_len).  NaN scores rank above +inf, as in
 * torch.topk, and are never kept (score >= thr is false for NaN). */
DSA_API int dsa_topk_select_ex(const float* scores, int64_t n_rows, int64_t row_len,
                               int64_t row_stride, int64_t rows_per_batch, int64_t q_row0,
                               int64_t row_bstep, int causal, int64_t k, float* thr_out,
                               int32_t* idx_out, int32_t* cnt_out, int64_t idx_cap,
                               uint32_t* bits, int64_t words_per_row, void* stream);

/*
 * Stage 3 (threshold form) — attention of each query over the keys s <= t
 * with scores[s] >= thr[row].
 *   scores [B, T_q, T_k] fp32 (row stride T_k), thr [B*T_q] fp32
 *   Q [B, T_q, HQ, DQ], K [B, T_k, HQ, DQ], V [B, T_k, HQ, DV]   dtype
 *   O [B, T_q, HQ, DV] fp32 out
 * scale multiplies the logits (the reference uses 1/sqrt(DQ)).
 */
DSA_API int dsa_sparse_attn_threshold(const float* scores, const float* thr,
                              const void* Q, const void* K, const void* V, float* O,
                              int64_t B, int64_t T_q, int64_t T_k, int64_t q_row0,
                              int64_t HQ, int64_t DQ, int64_t DV, float scale,
                              int dtype, void* stream);

/*
 * Stage 3 (list form) — attention over the index lists of dsa_topk_select.
 *   idx [B*T_q, idx_cap] int32, cnt [B*T_q] int32
 * Rows whose cnt exceeds idx_cap fall back to the threshold form, so scores
 * and thr (as above) must be given whenever idx_cap < min(T_k, q_row0+T_q);
 * otherwise they may be NULL.
 */
DSA_API int dsa_sparse_attn(const int32_t* idx, const int32_t* cnt, int64_t idx_cap,
                    const float* scores, const float* thr,
                    const void* Q, const void* K, const void* V, float* O,
                    int64_t B, int64_t T_q, int64_t T_k, int64_t q_row0,
                    int64_t HQ, int64_t DQ, int64_t DV, float scale,
                    int dtype, void* stream);

/* dsa_sparse_attn (idx != NULL) or dsa_sparse_attn_threshold (idx == NULL)
 * over strided Q/K/V and row blocks (layout may be NULL: contiguous).  Only
 * layout->Q, K, V and row_bstep are read. */
DSA_API int dsa_sparse_attn_ex(const int32_t* idx, const int32_t* cnt, int64_t idx_cap,
                               const float* scores, const float* thr,
                               const void* Q, const void* K, const void* V, float* O,
                               int64_t B, int64_t T_q, int64_t T_k, int64_t q_row0,
                               int64_t HQ, int64_t DQ, int64_t DV, float scale,
                               int dtype, const dsa_layout* layout, void* stream);

/*
 * Stage 3 (bitmap form, tensor cores) — the kept set as one bit per
 * (query row, key), then a masked flash attention over it.
 *   dsa_bitmap_words(T_k): words per bitmap row, ceil(T_k/128)*4.
 *   dsa_kept_bitmap: bits [B*T_q, words_per_row] uint32 out; bit (s & 31) of
 *     word s/32 of row r is 1 iff s <= q_row0 + r % T_q and scores[r,s] >= thr[r]
 *     (scores, thr as in dsa_sparse_attn_threshold).  words_per_row must be a
 *     multiple of 4 and >= dsa_bitmap_words(T_k); words past T_k are zero.
 *   dsa_sparse_attn_bitmap: attention of each query over its set bits,
 *     O [B, T_q, HQ, DV] fp32 out; Q/K/V as in dsa_sparse_attn_threshold.
 *     bf16 or fp16 with DQ == DV in {64, 128}, else DSA_ERR_UNSUPPORTED.
 *     The softmax weights enter the P.V product rounded to the input dtype
 *     (this entry point has no workspace for an fp16 copy of V; the _ex form
 *     and dsa_forward use fp16 weights for bf16 inputs too).
 */
DSA_API int64_t dsa_bitmap_words(int64_t T_k);

DSA_API int dsa_kept_bitmap(const float* scores, const float* thr, uint32_t* bits,
                            int64_t B, int64_t T_q, int64_t T_k, int64_t q_row0,
                            int64_t words_per_row, void* stream);

/* Stage 2 writing the kept set as the bitmap of dsa_kept_bitmap instead of
 * index lists (rows with row_stride == row_len).  Same selection as
 * dsa_topk_select; cnt_out may be NULL.  Rows of 4K-32K entries get the bitmap
 * from the top-K kernel's last sweep, others from a dsa_kept_bitmap pass. */
DSA_API int dsa_topk_select_bitmap(const float* scores, int64_t n_rows, int64_t row_len,
                                   int64_t rows_per_batch, int64_t q_row0, int causal, int64_t k,
                                   float* thr_out, int32_t* cnt_out, uint32_t* bits,
                                   int64_t words_per_row, void* stream);

/* dsa_topk_select_bitmap with row blocks (row_bstep as in dsa_topk_select_ex)
 * and a workspace of
 * dsa_topk_select_bitmap_workspace_bytes(n_rows, words_per_row) bytes (256-byte
 * aligned).  Rows of 4K-32K entries then take two kernels: a sweep kernel that
 * writes the final bits of every score above the threshold's first-digit bin
 * and marks that bin's scores as candidates in the workspace, and a per-row
 * resolver that finds the exact threshold among the candidates.  Same outputs
 * as dsa_topk_select_bitmap, bit for bit.  Replaces the same reference
 * interface (dsa_attention.py:343-344 threshold + :230-324 mask). */
DSA_API size_t dsa_topk_select_bitmap_workspace_bytes(int64_t n_rows, int64_t words_per_row);
DSA_API int dsa_topk_select_bitmap_ws(const float* scores, int64_t n_rows, int64_t row_len,
                                      int64_t rows_per_batch, int64_t q_row0, int64_t row_bstep,
                                      int causal, int64_t k, float* thr_out, int32_t* cnt_out,
                                      uint32_t* bits, int64_t words_per_row, void* workspace,
                                      size_t workspace_bytes, void* stream);

DSA_API int dsa_sparse_attn_bitmap(const uint32_t* bits, int64_t words_per_row,
                                   const void* Q, const void* K, const void* V, float* O,
                                   int64_t B, int64_t T_q, int64_t T_k, int64_t q_row0,
                                   int64_t HQ, int64_t DQ, int64_t DV, float scale,
                                   int dtype, void* stream);

/* dsa_sparse_attn_bitmap over strided Q/K/V and row blocks (layout may be
 * NULL).  Only layout->Q, K, V and row_bstep are read.  With a workspace of
 * dsa_sparse_attn_bitmap_workspace_bytes(...) bytes (256-byte aligned):
 *   - a summary of the bitmap (one bit per 128-row query tile and 128-key
 *     block) lets the kernel skip key blocks no row of a tile keeps; the
 *     result is bit-identical to processing every causal block;
 *   - bf16 inputs: V is copied to fp16 (scaled by a power of two) and the
 *     softmax weights enter P.V in fp16, whose 11-bit significand keeps the
 *     output within 1e-3 + 2e-2|O| of the fp32 reference elementwise.
 * Without one (and in dsa_sparse_attn_bitmap) every causal block is
 * processed and the weights enter in the input type. */
DSA_API size_t dsa_sparse_attn_bitmap_workspace_bytes(int64_t B, int64_t T_q, int64_t T_k, int64_t HQ,
                                                      int64_t DV, int dtype);
DSA_API int dsa_sparse_attn_bitmap_ex(const uint32_t* bits, int64_t words_per_row,
                                      const void* Q, const void* K, const void* V, float* O,
                                      int64_t B, int64_t T_q, int64_t T_k, int64_t q_row0,
                                      int64_t HQ, int64_t DQ, int64_t DV, float scale,
                                      int dtype, const dsa_layout* layout, void* workspace,
                                      size_t workspace_bytes, void* stream);

/*
 * Whole forward (stage 1 -> 2 -> 3) in caller-provided workspace.
 * idx_dtype is the dtype of q_idx/k_idx, qkv_dtype that of Q/K/V; w_idx is fp32.
 * Layouts as above: q_idx [B,T_q,HI,DI], k_idx [B,T_k,DI], w_idx [B,T_q,HI],
 * Q [B,T_q,HQ,DQ], K [B,T_k,HQ,DQ], V [B,T_k,HQ,DV], O [B,T_q,HQ,DV] fp32.
 * top_k is clamped to T_k (k_eff = min(k, T), dsa_attention.py:41).
 * workspace must hold dsa_forward_workspace_bytes(...) bytes, 256-byte aligned.
 * Stage 3 runs on the tensor cores (threshold -> bitmap -> dsa_sparse_attn_bitmap)
 * when qkv_dtype is bf16/fp16 with DQ == DV in {64, 128}, else as the gather
 * over the kept lists (dsa_sparse_attn).
 */
DSA_API size_t dsa_forward_workspace_bytes(int64_t B, int64_t T_q, int64_t T_k, int64_t top_k);

/* Workspace for dsa_forward / dsa_forward_ex that also holds stage 3's
 * workspace on the tensor cores (dsa_sparse_attn_bitmap_ex: the block
 * summary, and for bf16 Q/K/V the fp16 copy of V).  Equal to
 * dsa_forward_workspace_bytes whenever that fits over the score region,
 * roughly T_q * (T_k + list capacity) * 4 >= T_k * HQ * DV * 2 (every full
 * sequence of the reference's configurations); with only
 * dsa_forward_workspace_bytes for shorter row blocks, stage 3 runs without
 * block skipping and with bf16 weights. */
DSA_API size_t dsa_forward_workspace_bytes_ex(int64_t B, int64_t T_q, int64_t T_k, int64_t top_k,
                                              int64_t HQ, int64_t DV, int qkv_dtype);

DSA_API int dsa_forward(const void* q_idx, const void* k_idx, const float* w_idx,
                const void* Q, const void* K, const void* V, float* O,
                int64_t B, int64_t T_q, int64_t T_k, int64_t q_row0,
                int64_t HI, int64_t DI, int64_t HQ, int64_t DQ, int64_t DV, int64_t top_k,
                int idx_dtype, int qkv_dtype, void* workspace, size_t workspace_bytes,
                void* stream);

/* dsa_forward over strided inputs and row blocks (layout may be NULL:
 * contiguous).  Same workspace size as dsa_forward.  The GPU that owns
 * zig-zag blocks r and 2N-1-r of one sequence runs both in one call per
 * stage: B = 2 with key-side batch strides 0 (see struct dsa_layout). */
DSA_API int dsa_forward_ex(const void* q_idx, const void* k_idx, const float* w_idx,
                           const void* Q, const void* K, const void* V, float* O,
                           int64_t B, int64_t T_q, int64_t T_k, int64_t q_row0,
                           int64_t HI, int64_t DI, int64_t HQ, int64_t DQ, int64_t DV,
                           int64_t top_k, int idx_dtype, int qkv_dtype,
                           const dsa_layout* layout, void* workspace, size_t workspace_bytes,
                           void* stream);

/*
 * Whole forward with no allocation and no caller workspace.  No counterpart
 * in the reference: it exists for callers that cannot allocate device memory
 * where they run the forward (a host framework that owns all GPU memory
 * through its own pool, a plugin that is only handed its input and output
 * buffers), so they cannot provide dsa_forward's workspace.
 *   Arguments as dsa_forward, minus workspace / workspace_bytes.
 *   Scratch: a 32 MiB device array inside the library, reserved on every GPU
 *   that loads the library until the process exits.  Shapes whose
 *   dsa_forward_workspace_bytes(...) exceeds 32 MiB are rejected with
 *   DSA_ERR_INVALID (e.g. B=16, T=512, top_k=32 fits; T=8192 does not).
 *   The first call on a device looks up the array's device address for that
 *   device (cudaGetSymbolAddress); make that first call before any stream
 *   capture.  The address is looked up again when the device's context has
 *   changed since (e.g. after cudaDeviceReset).  No cudaMalloc / cudaFree is
 *   ever called.  An empty call (B*T_q == 0) returns DSA_OK, as dsa_forward.
 *   All calls on a device share the one array and nothing in it needs
 *   clearing between calls; calls that overlap on the GPU (different streams,
 *   or host threads without ordering) race on it and must be serialised.
 */
DSA_API int dsa_forward_noalloc(const void* q_idx, const void* k_idx, const float* w_idx,
                                const void* Q, const void* K, const void* V, float* O,
                                int64_t B, int64_t T_q, int64_t T_k, int64_t q_row0,
                                int64_t HI, int64_t DI, int64_t HQ, int64_t DQ, int64_t DV,
                                int64_t top_k, int idx_dtype, int qkv_dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DSA_B200_H */
