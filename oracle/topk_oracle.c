/*
 * TEST INFRASTRUCTURE ONLY — the CPU oracle for the top-K selection stage.
 *
 * Nothing in the shipped library links or calls this file.  Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg load the shared
 * object built from it, and only to check the CUDA path.
 *
 * What it restates (reference = Infatoshi/dsa-cpu-topk):
 *   - the per-row k-th-largest threshold:
 *       dsa_attention.py:41-44   topv, _ = scores.topk(k_eff); threshold = topv[..., -1:]
 *       dsa_attention.py:343-344 (split path, same rule)
 *       topk_avx512.cpp:226-249  topk_threshold_impl (CPU k-th largest, fp32)
 *   - the keep-ties selection rule:
 *       dsa_attention.py:46      sel = (scores >= threshold) & causal
 *       dsa_attention.py:256-258 keep = scores >= thr & s <= t
 *
 * The threshold is the k-th largest element of the row as a multiset
 * (k counted from 1, largest first), i.e. exactly the value torch.topk
 * returns at position k-1.  It is found by quickselect over an ordering key
 * that follows torch.topk's value order: -0.0 == +0.0, -inf last, and every
 * NaN above +inf (all NaNs equal).  The kept set then uses the float
 * comparison scores >= thr of the reference, so a NaN is never kept and a
 * NaN threshold keeps nothing.
 *
 * Causal rows: query row r of a batch of `rows_per_batch` rows sits at
 * position t = q_row0 + r % rows_per_batch; entries s > t count as -inf
 * whatever is stored there (the indexer writes -inf there,
 * lightning_indexer.py:32-33), and are never selected.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

static void swapf(float* a, float* b) { float t = *a; *a = *b; *b = t; }

/* torch.topk's order as a total order on floats: NaN (any sign or payload)
 * above +inf, -0.0 equal to +0.0, everything else by value. */
static int gt(float a, float b) {
    if (isnan(a)) return !isnan(b);
    if (isnan(b)) return 0;
    return a > b;
}
static int lt(float a, float b) { return gt(b, a); }

/* k-th largest (1-based) of buf[0..n), n >= k >= 1, in gt/lt order.  Reorders buf. */
static float kth_largest(float* buf, int64_t n, int64_t k) {
    int64_t lo = 0, hi = n - 1, want = k - 1; /* index in descending order */
    while (lo < hi) {
        /* median of three, pivot moved to hi */
        int64_t mid = lo + (hi - lo) / 2;
        if (gt(buf[mid], buf[lo])) swapf(&buf[mid], &buf[lo]);
        if (gt(buf[hi], buf[lo])) swapf(&buf[hi], &buf[lo]);
        if (gt(buf[mid], buf[hi])) swapf(&buf[mid], &buf[hi]);
        float p = buf[hi];
        /* three-way partition, descending: [> p | == p | < p] */
        int64_t g = lo, i = lo, l = hi;
        while (i <= l) {
            if (gt(buf[i], p)) { swapf(&buf[i], &buf[g]); g++; i++; }
            else if (lt(buf[i], p)) { swapf(&buf[i], &buf[l]); l--; }
            else i++;
        }
        if (want < g) hi = g - 1;
        else if (want > l) lo = l + 1;
        else return p;
    }
    return buf[lo];
}

/*
 * Per-row threshold and ascending index list of the kept entries.
 *   scores        row-major, row r starts at scores + r*row_stride
 *   thr_out[r]    k-th largest of the row (over all row_len entries)
 *   idx_out       may be NULL; else row r's kept indices go to
 *                 idx_out[r*idx_cap ...], at most idx_cap of them
 *   cnt_out[r]    number of kept entries (may exceed idx_cap)
 * Returns 0, or -1 on bad arguments.
 */
int oracle_topk_select(const float* scores, int64_t n_rows, int64_t row_len,
                       int64_t row_stride, int64_t rows_per_batch, int64_t q_row0,
                       int causal, int64_t k, float* thr_out, int32_t* idx_out,
                       int32_t* cnt_out, int64_t idx_cap) {
    if (k < 1 || k > row_len || n_rows < 0 || row_stride < row_len) return -1;
    if (causal && rows_per_batch < 1) return -1;
    float* buf = (float*)malloc(sizeof(float) * (size_t)(row_len > 0 ? row_len : 1));
    if (!buf) return -1;
    for (int64_t r = 0; r < n_rows; ++r) {
        const float* row = scores + r * row_stride;
        int64_t valid = row_len;
        if (causal) {
            int64_t t = q_row0 + r % rows_per_batch;
            valid = t + 1 < row_len ? t + 1 : row_len;
        }
        memcpy(buf, row, sizeof(float) * (size_t)valid);
        for (int64_t s = valid; s < row_len; ++s) buf[s] = -INFINITY;
        float thr = kth_largest(buf, row_len, k);
        thr_out[r] = thr;
        int32_t cnt = 0;
        for (int64_t s = 0; s < valid; ++s) {
            if (row[s] >= thr) {
                if (idx_out && cnt < idx_cap) idx_out[r * idx_cap + cnt] = (int32_t)s;
                cnt++;
            }
        }
        if (cnt_out) cnt_out[r] = cnt;
    }
    free(buf);
    return 0;
}

/* Threshold only: the topk_threshold(scores, k) contract of
 * topk_avx512.cpp:251-253 (rows of length N, output one value per row). */
int oracle_topk_threshold(const float* scores, int64_t n_rows, int64_t N, int64_t k,
                          float* thr_out) {
    return oracle_topk_select(scores, n_rows, N, N, 1, 0, 0, k, thr_out, NULL, NULL, 0);
}
