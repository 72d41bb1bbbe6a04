// C ABI of libdsa_b200.so: argument checks, dispatch, per-thread error text,
// and the whole-forward pipeline (stage 1 -> 2 -> 3) over caller workspace.
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <string>

#include "common.cuh"

namespace dsa {

// defined in the stage files
int indexer_scores_simt(const void* q, const void* k, const float* w, float* scores, int64_t B,
                        int64_t T_q, int64_t T_k, int64_t q_row0, int64_t HI, int64_t DI,
                        int dtype, int fill_upper, const dsa_layout& L, const float* kscale,
                        cudaStream_t stream);
int indexer_scores_tc(const void* q, const void* k, const float* w, float* scores, int64_t B,
                      int64_t T_q, int64_t T_k, int64_t q_row0, int64_t HI, int64_t DI,
                      int fill_upper, int dtype, const dsa_layout& L, const float* kscale,
                      cudaStream_t stream);
bool indexer_tc_supported(int64_t HI, int64_t DI, int dtype);
int indexer_tc_take_timeout(cudaStream_t stream);
int topk_select(const float* scores, int64_t n_rows, int64_t row_len, int64_t row_stride,
                int64_t rows_per_batch, int64_t q_row0, int causal, int64_t k, float* thr,
                int32_t* idx, int32_t* cnt, int64_t idx_cap, uint32_t* bits, int64_t words,
                int64_t row_bstep, cudaStream_t stream, void* ws = nullptr, size_t ws_bytes = 0);
size_t topk_sweep_ws_bytes(int64_t n_rows, int64_t words);
int fused_small_forward(const void* q_idx, const void* k_idx, const float* w_idx, const void* Q,
                        const void* K, const void* V, float* O, int64_t B, int64_t T_q, int64_t T_k,
                        int64_t q_row0, int64_t HI, int64_t DI, int64_t HQ, int64_t DQ, int64_t DV,
                        int64_t k, int idx_dtype, int qkv_dtype, cudaStream_t stream);
int64_t bitmap_words(int64_t T_k);
int kept_bitmap(const float* scores, const float* thr, uint32_t* bits, int64_t B, int64_t T_q,
                int64_t T_k, int64_t q_row0, int64_t words, int64_t row_bstep, cudaStream_t stream);
bool attn_tc_supported(int64_t HQ, int64_t DQ, int64_t DV, int dtype);
int attn_tc(const uint32_t* bits, int64_t words, const void* Q, const void* K, const void* V,
            float* O, int64_t B, int64_t T_q, int64_t T_k, int64_t q_row0, int64_t HQ, int64_t D,
            float scale, int dtype, const dsa_layout& L, void* ws, size_t ws_bytes, cudaStream_t stream);
size_t attn_ws_bytes(int64_t B, int64_t T_q, int64_t T_k, int64_t HQ, int64_t D, int dtype);
int attn_tc_take_timeout(cudaStream_t stream);
int sparse_attn(const int32_t* idx, const int32_t* cnt, int64_t idx_cap, const float* scores,
                const float* thr, const void* Q, const void* K, const void* V, float* O, int64_t B,
                int64_t T_q, int64_t T_k, int64_t q_row0, int64_t HQ, int64_t DQ, int64_t DV,
                float scale, int dtype, const dsa_layout& L, cudaStream_t stream);

unsigned debug_flags_sparse_attn();
unsigned debug_flags_topk();
unsigned debug_flags_attn_tc();
unsigned debug_flags_indexer_tc();
unsigned debug_flags_indexer_simt();
unsigned debug_flags_fused_small();
unsigned debug_flags_fp8_quant();

namespace {
thread_local std::string g_last_error;
}

void set_error(const std::string& msg) { g_last_error = msg; }
void clear_error() { g_last_error.clear(); }
int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(DSA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
    return DSA_OK;
}

int num_sms() {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1)
        return 148;
    return n;
}

// kept-list capacity used by dsa_forward: k plus room for ties, multiple of 32
int64_t idx_cap_for(int64_t k, int64_t T_k) {
    int64_t cap = ((k + k / 4 + 32 + 31) / 32) * 32;
    return cap < T_k ? cap : T_k;
}

// DSA_FORCE_SIMT_INDEXER=1 routes every shape to the CUDA-core indexer
// (used to cross-check the two kernels against each other).
static bool force_simt() {
    const char* e = getenv("DSA_FORCE_SIMT_INDEXER");
    return e && e[0] == '1';
}

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// DSA_ATTN_GATHER=1 keeps bf16/fp16 attention on the gather kernel over the
// kept lists instead of the tensor-core kernel over the kept-set bitmap.
static bool force_gather() {
    const char* e = getenv("DSA_ATTN_GATHER");
    return e && e[0] == '1';
}

struct ForwardLayout {
    size_t scores, thr, cnt, idx, bits, total;
    int64_t idx_cap, words;
};

static ForwardLayout forward_layout(int64_t B, int64_t T_q, int64_t T_k, int64_t top_k) {
    ForwardLayout L;
    const int64_t rows = B * T_q;
    const int64_t k = top_k < T_k ? top_k : T_k;
    L.idx_cap = idx_cap_for(k, T_k);
    size_t off = 0;
    L.scores = off;
    off += align256((size_t)rows * (size_t)T_k * sizeof(float));
    L.thr = off;
    off += align256((size_t)rows * sizeof(float));
    L.cnt = off;
    off += align256((size_t)rows * sizeof(int32_t));
    L.idx = off;
    L.words = bitmap_words(T_k);
    // the index lists (gather path), or the bitmap top-K's candidate words (tensor-core path)
    const size_t list_bytes = (size_t)rows * (size_t)L.idx_cap * sizeof(int32_t);
    const size_t cand_bytes = topk_sweep_ws_bytes(rows, L.words);
    off += align256(list_bytes > cand_bytes ? list_bytes : cand_bytes);
    L.bits = off;
    off += align256((size_t)rows * (size_t)L.words * sizeof(uint32_t));
    L.total = off;
    return L;
}

static int check_indexer_args(const void* q, const void* k, const float* w, const float* scores,
                              int64_t B, int64_t T_q, int64_t T_k, int64_t q_row0, int64_t HI,
                              int64_t DI, int dtype) {
    if (B < 0 || T_q < 0 || T_k < 1 || q_row0 < 0 || HI < 1 || DI < 1)
        return fail(DSA_ERR_INVALID, "indexer_scores: bad sizes");
    if (HI > INT32_MAX || DI > INT32_MAX) return fail(DSA_ERR_INVALID, "indexer_scores: HI/DI too large");
    if (!dtype_ok(dtype)) return fail(DSA_ERR_INVALID, "indexer_scores: unknown dtype");
    // an empty call reads nothing, so its (possibly empty) tensors may be null
    if (B * T_q > 0 && (!q || !k || !w || !scores))
        return fail(DSA_ERR_INVALID, "indexer_scores: null pointer");
    return DSA_OK;
}

static int check_layout(const dsa_layout& L, const char* what) {
    const int64_t* all[] = {L.q, L.k, L.w, L.Q, L.K, L.V};
    const int n[] = {3, 2, 2, 3, 3, 3};
    for (int t = 0; t < 6; ++t)
        for (int i = 0; i < n[t]; ++i)
            if (all[t][i] < 0) return fail(DSA_ERR_INVALID, std::string(what) + ": negative stride in layout");
    if (L.row_bstep < 0) return fail(DSA_ERR_INVALID, std::string(what) + ": row_bstep must be >= 0");
    return DSA_OK;
}

static int run_indexer(const void* q, const void* k, const float* w, float* scores, int64_t B,
                       int64_t T_q, int64_t T_k, int64_t q_row0, int64_t HI, int64_t DI, int dtype,
                       int fill_upper, const dsa_layout& L, cudaStream_t st, const float* kscale = nullptr) {
    if (indexer_tc_supported(HI, DI, dtype) && aligned16(q) && aligned16(k) && aligned16(scores) &&
        aligned16(w) && !force_simt()) {
        const int rc = indexer_scores_tc(q, k, w, scores, B, T_q, T_k, q_row0, HI, DI, fill_upper,
                                         dtype, L, kscale, st);
        if (rc == -101) {
            // row blocks too many for one launch's tile table: one launch per batch
            const size_t e = dtype_size(dtype);
            dsa_layout Lb = L;
            Lb.row_bstep = 0;
            for (int64_t b = 0; b < B; ++b) {
                const int r = run_indexer(static_cast<const char*>(q) + b * L.q[0] * e,
                                          static_cast<const char*>(k) + b * L.k[0] * e, w + b * L.w[0],
                                          scores + b * T_q * T_k, 1, T_q, T_k, q_row0 + b * L.row_bstep,
                                          HI, DI, dtype, fill_upper, Lb, st,
                                          kscale ? kscale + (L.k[0] == 0 ? 0 : b * T_k) : nullptr);
                if (r) return r;
            }
            return DSA_OK;
        }
        if (rc != -100) return rc;  // -100: shape beyond the tensor-core kernel's limits
    }
    return indexer_scores_simt(q, k, w, scores, B, T_q, T_k, q_row0, HI, DI, dtype, fill_upper, L, kscale,
                               st);
}

}  // namespace dsa

using namespace dsa;

extern "C" {

int dsa_version(void) { return (0 << 16) | 2; }

const char* dsa_last_error_string(void) { return g_last_error.c_str(); }

void dsa_layout_contiguous(dsa_layout* out, int64_t T_q, int64_t T_k, int64_t HI, int64_t DI,
                           int64_t HQ, int64_t DQ, int64_t DV) {
    if (out) *out = layout_or_contiguous(nullptr, T_q, T_k, HI, DI, HQ, DQ, DV);
}

int dsa_indexer_scores_ex(const void* q, const void* k, const float* w, float* scores, int64_t B,
                          int64_t T_q, int64_t T_k, int64_t q_row0, int64_t HI, int64_t DI,
                          int dtype, int fill_upper, const dsa_layout* layout, void* stream) {
    clear_error();
    int rc = check_indexer_args(q, k, w, scores, B, T_q, T_k, q_row0, HI, DI, dtype);
    if (rc) return rc;
    const dsa_layout L = layout_or_contiguous(layout, T_q, T_k, HI, DI, 1, 1, 1);
    if ((rc = check_layout(L, "indexer_scores"))) return rc;
    if (B * T_q == 0) return DSA_OK;
    return run_indexer(q, k, w, scores, B, T_q, T_k, q_row0, HI, DI, dtype, fill_upper, L,
                       (cudaStream_t)stream);
}

int dsa_indexer_scores_fp8(const void* q8, const void* k8, const float* w, const float* k_scale,
                           float* scores, int64_t B, int64_t T_q, int64_t T_k, int64_t q_row0,
                           int64_t HI, int64_t DI, int fill_upper, const dsa_layout* layout, void* stream) {
    clear_error();
    int rc = check_indexer_args(q8, k8, w, scores, B, T_q, T_k, q_row0, HI, DI, DSA_FP8_E4M3);
    if (rc) return rc;
    const dsa_layout L = layout_or_contiguous(layout, T_q, T_k, HI, DI, 1, 1, 1);
    if ((rc = check_layout(L, "indexer_scores_fp8"))) return rc;
    if (B * T_q == 0) return DSA_OK;
    if (!k_scale) return fail(DSA_ERR_INVALID, "indexer_scores_fp8: k_scale is required");
    return run_indexer(q8, k8, w, scores, B, T_q, T_k, q_row0, HI, DI, DSA_FP8_E4M3, fill_upper, L,
                       (cudaStream_t)stream, k_scale);
}

int dsa_indexer_scores(const void* q, const void* k, const float* w, float* scores, int64_t B,
                       int64_t T_q, int64_t T_k, int64_t q_row0, int64_t HI, int64_t DI,
                       int dtype, int fill_upper, void* stream) {
    return dsa_indexer_scores_ex(q, k, w, scores, B, T_q, T_k, q_row0, HI, DI, dtype, fill_upper,
                                 nullptr, stream);
}

int dsa_topk_select_ex(const float* scores, int64_t n_rows, int64_t row_len, int64_t row_stride,
                       int64_t rows_per_batch, int64_t q_row0, int64_t row_bstep, int causal,
                       int64_t k, float* thr_out, int32_t* idx_out, int32_t* cnt_out,
                       int64_t idx_cap, uint32_t* bits, int64_t words_per_row, void* stream) {
    clear_error();
    if (row_bstep < 0) return fail(DSA_ERR_INVALID, "topk_select: row_bstep must be >= 0");
    return topk_select(scores, n_rows, row_len, row_stride, rows_per_batch, q_row0, causal, k,
                       thr_out, idx_out, cnt_out, idx_cap, bits, bits ? words_per_row : 0, row_bstep,
                       (cudaStream_t)stream);
}

int dsa_topk_select(const float* scores, int64_t n_rows, int64_t row_len, int64_t row_stride,
                    int64_t rows_per_batch, int64_t q_row0, int causal, int64_t k,
                    float* thr_out, int32_t* idx_out, int32_t* cnt_out, int64_t idx_cap,
                    void* stream) {
    return dsa_topk_select_ex(scores, n_rows, row_len, row_stride, rows_per_batch, q_row0, 0, causal,
                              k, thr_out, idx_out, cnt_out, idx_cap, nullptr, 0, stream);
}

int dsa_topk_select_bitmap(const float* scores, int64_t n_rows, int64_t row_len,
                           int64_t rows_per_batch, int64_t q_row0, int causal, int64_t k,
                           float* thr_out, int32_t* cnt_out, uint32_t* bits, int64_t words_per_row,
                           void* stream) {
    clear_error();
    if (!bits) return fail(DSA_ERR_INVALID, "topk_select_bitmap: bits is required");
    return dsa_topk_select_ex(scores, n_rows, row_len, row_len, rows_per_batch, q_row0, 0, causal, k,
                              thr_out, nullptr, cnt_out, 0, bits, words_per_row, stream);
}

size_t dsa_topk_select_bitmap_workspace_bytes(int64_t n_rows, int64_t words_per_row) {
    if (n_rows < 0 || words_per_row < 1) return 0;
    return topk_sweep_ws_bytes(n_rows, words_per_row);
}

int dsa_topk_select_bitmap_ws(const float* scores, int64_t n_rows, int64_t row_len,
                              int64_t rows_per_batch, int64_t q_row0, int64_t row_bstep, int causal,
                              int64_t k, float* thr_out, int32_t* cnt_out, uint32_t* bits,
                              int64_t words_per_row, void* workspace, size_t workspace_bytes,
                              void* stream) {
    clear_error();
    if (!bits) return fail(DSA_ERR_INVALID, "topk_select_bitmap: bits is required");
    if (row_bstep < 0) return fail(DSA_ERR_INVALID, "topk_select_bitmap: row_bstep must be >= 0");
    if (workspace && (reinterpret_cast<uintptr_t>(workspace) & 255u))
        return fail(DSA_ERR_INVALID, "topk_select_bitmap: workspace must be 256-byte aligned");
    if (n_rows > 0 && workspace_bytes < dsa_topk_select_bitmap_workspace_bytes(n_rows, words_per_row))
        return fail(DSA_ERR_INVALID, "topk_select_bitmap: workspace too small");
    return topk_select(scores, n_rows, row_len, row_len, rows_per_batch, q_row0, causal, k, thr_out,
                       nullptr, cnt_out, 0, bits, words_per_row, row_bstep, (cudaStream_t)stream,
                       workspace, workspace_bytes);
}

int dsa_sparse_attn_ex(const int32_t* idx, const int32_t* cnt, int64_t idx_cap, const float* scores,
                       const float* thr, const void* Q, const void* K, const void* V, float* O,
                       int64_t B, int64_t T_q, int64_t T_k, int64_t q_row0, int64_t HQ, int64_t DQ,
                       int64_t DV, float scale, int dtype, const dsa_layout* layout, void* stream) {
    clear_error();
    const dsa_layout L = layout_or_contiguous(layout, T_q, T_k, 1, 1, HQ, DQ, DV);
    const int rc = check_layout(L, "sparse_attn");
    if (rc) return rc;
    return sparse_attn(idx, cnt, idx_cap, scores, thr, Q, K, V, O, B, T_q, T_k, q_row0, HQ, DQ, DV,
                       scale, dtype, L, (cudaStream_t)stream);
}

int dsa_sparse_attn_threshold(const float* scores, const float* thr, const void* Q, const void* K,
                              const void* V, float* O, int64_t B, int64_t T_q, int64_t T_k,
                              int64_t q_row0, int64_t HQ, int64_t DQ, int64_t DV, float scale,
                              int dtype, void* stream) {
    return dsa_sparse_attn_ex(nullptr, nullptr, 0, scores, thr, Q, K, V, O, B, T_q, T_k, q_row0, HQ,
                              DQ, DV, scale, dtype, nullptr, stream);
}

int dsa_sparse_attn(const int32_t* idx, const int32_t* cnt, int64_t idx_cap, const float* scores,
                    const float* thr, const void* Q, const void* K, const void* V, float* O,
                    int64_t B, int64_t T_q, int64_t T_k, int64_t q_row0, int64_t HQ, int64_t DQ,
                    int64_t DV, float scale, int dtype, void* stream) {
    clear_error();
    if (!idx) return fail(DSA_ERR_INVALID, "sparse_attn: idx is required (use the threshold form)");
    return dsa_sparse_attn_ex(idx, cnt, idx_cap, scores, thr, Q, K, V, O, B, T_q, T_k, q_row0, HQ, DQ,
                              DV, scale, dtype, nullptr, stream);
}

int dsa_device_status(void* stream) {
    clear_error();
    const int r = indexer_tc_take_timeout((cudaStream_t)stream);
    const int a = attn_tc_take_timeout((cudaStream_t)stream);
    if (r < 0 || a < 0)
        return fail(DSA_ERR_CUDA, std::string("dsa_device_status: ") +
                                      cudaGetErrorString(cudaGetLastError()));
    if (r > 0)
        return fail(DSA_ERR_TIMEOUT, "a tensor-core indexer launch timed out waiting on its pipeline "
                                     "(its scores are incomplete)");
    if (a > 0)
        return fail(DSA_ERR_TIMEOUT, "a tensor-core attention launch timed out waiting on its "
                                     "pipeline (its output is incomplete)");
    return DSA_OK;
}

int dsa_debug_checks_enabled(void) {
#ifdef DSA_DEBUG_CHECKS
    return 1;
#else
    return 0;
#endif
}

int dsa_debug_status(void* stream) {
    clear_error();
    if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess)
        return fail(DSA_ERR_CUDA, "dsa_debug_status: stream synchronisation failed");
    return (int)(debug_flags_sparse_attn() | debug_flags_topk() | debug_flags_attn_tc() |
                 debug_flags_indexer_tc() | debug_flags_indexer_simt() | debug_flags_fused_small() |
                 debug_flags_fp8_quant());
}

int64_t dsa_bitmap_words(int64_t T_k) { return T_k < 1 ? 0 : bitmap_words(T_k); }

int dsa_kept_bitmap(const float* scores, const float* thr, uint32_t* bits, int64_t B, int64_t T_q,
                    int64_t T_k, int64_t q_row0, int64_t words_per_row, void* stream) {
    clear_error();
    return kept_bitmap(scores, thr, bits, B, T_q, T_k, q_row0, words_per_row, 0, (cudaStream_t)stream);
}

size_t dsa_sparse_attn_bitmap_workspace_bytes(int64_t B, int64_t T_q, int64_t T_k, int64_t HQ, int64_t DV,
                                              int dtype) {
    if (B < 0 || T_q < 0 || T_k < 1 || !attn_tc_supported(HQ, DV, DV, dtype)) return 0;
    return attn_ws_bytes(B, T_q, T_k, HQ, DV, dtype);
}

int dsa_sparse_attn_bitmap_ex(const uint32_t* bits, int64_t words_per_row, const void* Q,
                              const void* K, const void* V, float* O, int64_t B, int64_t T_q,
                              int64_t T_k, int64_t q_row0, int64_t HQ, int64_t DQ, int64_t DV,
                              float scale, int dtype, const dsa_layout* layout, void* workspace,
                              size_t workspace_bytes, void* stream) {
    clear_error();
    if (!bits || !Q || !K || !V || !O) return fail(DSA_ERR_INVALID, "sparse_attn_bitmap: null pointer");
    if (B < 0 || T_q < 0 || T_k < 1 || q_row0 < 0 || HQ < 1 || DQ < 1 || DV < 1)
        return fail(DSA_ERR_INVALID, "sparse_attn_bitmap: bad sizes");
    if (words_per_row < bitmap_words(T_k) || (words_per_row & 3))
        return fail(DSA_ERR_INVALID, "sparse_attn_bitmap: words_per_row must be a multiple of 4 and "
                                     ">= dsa_bitmap_words(T_k)");
    if (!attn_tc_supported(HQ, DQ, DV, dtype))
        return fail(DSA_ERR_UNSUPPORTED, "sparse_attn_bitmap: needs bf16/fp16 with DQ == DV in {64, 128}");
    const dsa_layout L = layout_or_contiguous(layout, T_q, T_k, 1, 1, HQ, DQ, DV);
    int rc = check_layout(L, "sparse_attn_bitmap");
    if (rc) return rc;
    rc = attn_tc(bits, words_per_row, Q, K, V, O, B, T_q, T_k, q_row0, HQ, DQ, scale, dtype, L, workspace,
                 workspace_bytes, (cudaStream_t)stream);
    if (rc == -100)
        return fail(DSA_ERR_UNSUPPORTED, "sparse_attn_bitmap: shape, stride or alignment outside the "
                                         "tensor-core kernel's limits");
    return rc;
}

int dsa_sparse_attn_bitmap(const uint32_t* bits, int64_t words_per_row, const void* Q, const void* K,
                           const void* V, float* O, int64_t B, int64_t T_q, int64_t T_k,
                           int64_t q_row0, int64_t HQ, int64_t DQ, int64_t DV, float scale,
                           int dtype, void* stream) {
    return dsa_sparse_attn_bitmap_ex(bits, words_per_row, Q, K, V, O, B, T_q, T_k, q_row0, HQ, DQ, DV,
                                     scale, dtype, nullptr, nullptr, 0, stream);
}

size_t dsa_forward_workspace_bytes(int64_t B, int64_t T_q, int64_t T_k, int64_t top_k) {
    if (B < 0 || T_q < 0 || T_k < 1 || top_k < 1) return 0;
    return forward_layout(B, T_q, T_k, top_k).total;
}

size_t dsa_forward_workspace_bytes_ex(int64_t B, int64_t T_q, int64_t T_k, int64_t top_k, int64_t HQ,
                                      int64_t DV, int qkv_dtype) {
    if (B < 0 || T_q < 0 || T_k < 1 || top_k < 1 || HQ < 1 || DV < 1) return 0;
    const ForwardLayout W = forward_layout(B, T_q, T_k, top_k);
    if (!attn_tc_supported(HQ, DV, DV, qkv_dtype)) return W.total;
    // stage 3's workspace (block summary; fp16 copy of V for bf16) overlays the
    // score and list region (dead once the bitmap is written), or follows the
    // workspace when that region is smaller
    const size_t a = attn_ws_bytes(B, T_q, T_k, HQ, DV, qkv_dtype);
    return a <= W.bits - W.scores ? W.total : W.total + a;
}

int dsa_forward_ex(const void* q_idx, const void* k_idx, const float* w_idx, const void* Q,
                   const void* K, const void* V, float* O, int64_t B, int64_t T_q, int64_t T_k,
                   int64_t q_row0, int64_t HI, int64_t DI, int64_t HQ, int64_t DQ, int64_t DV,
                   int64_t top_k, int idx_dtype, int qkv_dtype, const dsa_layout* layout,
                   void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    if (top_k < 1) return fail(DSA_ERR_INVALID, "dsa_forward: top_k must be >= 1");
    int rc = check_indexer_args(q_idx, k_idx, w_idx, O, B, T_q, T_k, q_row0, HI, DI, idx_dtype);
    if (rc) return rc;
    const dsa_layout L = layout_or_contiguous(layout, T_q, T_k, HI, DI, HQ, DQ, DV);
    if ((rc = check_layout(L, "dsa_forward"))) return rc;
    // an empty call has nothing to compute and needs no workspace
    if (B * T_q == 0) return DSA_OK;
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255u))
        return fail(DSA_ERR_INVALID, "dsa_forward: workspace must be non-null and 256-byte aligned");
    const ForwardLayout W = forward_layout(B, T_q, T_k, top_k);
    if (workspace_bytes < W.total)
        return fail(DSA_ERR_INVALID, "dsa_forward: workspace too small (need " +
                                         std::to_string(W.total) + " bytes)");
    cudaStream_t st = (cudaStream_t)stream;
    char* ws = static_cast<char*>(workspace);
    float* scores = reinterpret_cast<float*>(ws + W.scores);
    float* thr = reinterpret_cast<float*>(ws + W.thr);
    int32_t* cnt = reinterpret_cast<int32_t*>(ws + W.cnt);
    int32_t* idx = reinterpret_cast<int32_t*>(ws + W.idx);
    const int64_t k = top_k < T_k ? top_k : T_k;

    // Opt-in (DSA_FUSED_SMALL=1): short sequences (T_k <= 2048) in one fused
    // launch, contiguous inputs only.  Measured slower than the three stage
    // kernels on B200 (c1: 0.14 vs 0.117 ms), so the default stays the
    // three-stage pipeline.  DSA_FUSED_SMALL=require makes a shape outside the
    // fused kernel's limits an error instead of a fall-back (tests).
    const char* fs = getenv("DSA_FUSED_SMALL");
    if (fs && !layout) {
        rc = fused_small_forward(q_idx, k_idx, w_idx, Q, K, V, O, B, T_q, T_k, q_row0, HI, DI, HQ, DQ,
                                 DV, k, idx_dtype, qkv_dtype, st);
        if (rc != -100) return rc;
        if (!strcmp(fs, "require"))
            return fail(DSA_ERR_UNSUPPORTED, "dsa_forward: shape outside the fused small-T kernel's limits");
    }

    rc = run_indexer(q_idx, k_idx, w_idx, scores, B, T_q, T_k, q_row0, HI, DI, idx_dtype,
                     /*fill_upper=*/0, L, st);
    if (rc) return rc;
    const float scale = 1.0f / sqrtf((float)DQ);
    if (attn_tc_supported(HQ, DQ, DV, qkv_dtype) && !force_gather()) {
        // threshold and kept-set bitmap, then tensor-core attention
        uint32_t* bits = reinterpret_cast<uint32_t*>(ws + W.bits);
        rc = topk_select(scores, B * T_q, T_k, T_k, T_q, q_row0, /*causal=*/1, k, thr, nullptr,
                         nullptr, 0, bits, W.words, L.row_bstep, st, ws + W.idx, W.bits - W.idx);
        if (rc) return rc;
        // stage 3's workspace (block summary; fp16 copy of V for bf16 inputs):
        // over the dead score and list region, else after the workspace; with
        // neither, every causal block is processed and P.V runs in the input type
        void* aws = nullptr;
        size_t aws_bytes = 0;
        const size_t need = attn_ws_bytes(B, T_q, T_k, HQ, DV, qkv_dtype);
        if (need <= W.bits - W.scores) {
            aws = ws + W.scores;
            aws_bytes = W.bits - W.scores;
        } else if (workspace_bytes >= W.total + need) {
            aws = ws + W.total;
            aws_bytes = workspace_bytes - W.total;
        }
        rc = attn_tc(bits, W.words, Q, K, V, O, B, T_q, T_k, q_row0, HQ, DQ, scale, qkv_dtype, L, aws,
                     aws_bytes, st);
        if (rc != -100) return rc;
    }
    rc = topk_select(scores, B * T_q, T_k, T_k, T_q, q_row0, /*causal=*/1, k, thr, idx, cnt,
                     W.idx_cap, nullptr, 0, L.row_bstep, st);
    if (rc) return rc;
    return sparse_attn(idx, cnt, W.idx_cap, scores, thr, Q, K, V, O, B, T_q, T_k, q_row0, HQ, DQ,
                       DV, scale, qkv_dtype, L, st);
}

int dsa_forward(const void* q_idx, const void* k_idx, const float* w_idx, const void* Q,
                const void* K, const void* V, float* O, int64_t B, int64_t T_q, int64_t T_k,
                int64_t q_row0, int64_t HI, int64_t DI, int64_t HQ, int64_t DQ, int64_t DV,
                int64_t top_k, int idx_dtype, int qkv_dtype, void* workspace,
                size_t workspace_bytes, void* stream) {
    return dsa_forward_ex(q_idx, k_idx, w_idx, Q, K, V, O, B, T_q, T_k, q_row0, HI, DI, HQ, DQ, DV,
                          top_k, idx_dtype, qkv_dtype, nullptr, workspace, workspace_bytes, stream);
}

}  // extern "C"
