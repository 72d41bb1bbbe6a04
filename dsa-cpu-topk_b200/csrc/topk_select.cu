// Stage 2: per-row top-K threshold + kept-index list by shared-memory radix select.
//
// Replaces the GPU `scores.topk(k)` threshold of dsa_attention.py:343-344
// (which materialises k values and indices per row only to read one column)
// and the AVX-512 CPU k-th-largest of topk_avx512.cpp:226-249.
//
// One CTA owns one row at a time (grid-stride over rows).  The row is read
// from HBM once: its order-preserving 32-bit keys are cached in shared memory
// (up to cache_elems of them; a longer row re-reads the rest from L2).  Four
// 8-bit radix passes narrow the k-th largest key from the top: each pass
// histograms the digit of the keys that still match the selected prefix
// (4 histogram copies, one per warp group, spread same-bin atomics), and a
// 256-thread scan of the histogram picks the digit whose bin holds the k-th
// largest.  The kept list is then written in ascending position order by a
// warp-segmented ballot compaction, so the output is deterministic.
//
// Selection rule (dsa_attention.py:41-46): keep every position with
// score >= threshold (ties kept) and, for causal rows, s <= t.
#include "common.cuh"

namespace dsa {
namespace {

constexpr int NBINS = 256;
constexpr int NHIST = 4;

struct TopkArgs {
    const float* scores;
    int64_t n_rows, row_len, row_stride, rows_per_batch, q_row0;
    int causal;
    int k;
    float* thr;
    int32_t* idx;
    int32_t* cnt;
    int64_t idx_cap;
    int cache_elems;
    int vec_ok;
};

template <int BLOCK>
__device__ __forceinline__ uint32_t key_at(const uint32_t* cache, int ncache, const float* src,
                                           int64_t i) {
    return i < ncache ? cache[i] : f2key(__ldg(src + i));
}

template <int BLOCK>
__global__ void __launch_bounds__(BLOCK) topk_select_kernel(TopkArgs a) {
    static_assert(BLOCK >= NBINS && BLOCK % 32 == 0 && BLOCK <= 1024, "block size");
    constexpr int NW = BLOCK / 32;
    extern __shared__ uint32_t cache[];
    __shared__ uint32_t hist[NHIST * NBINS];
    __shared__ uint32_t warp_tot[NW];
    __shared__ uint32_t s_digit, s_krem;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint32_t* my_hist = hist + (warp % NHIST) * NBINS;

    for (int64_t row = blockIdx.x; row < a.n_rows; row += gridDim.x) {
        const float* src = a.scores + row * a.row_stride;
        int64_t valid = a.row_len;
        if (a.causal) {
            const int64_t t = a.q_row0 + row % a.rows_per_batch;
            valid = t + 1 < a.row_len ? t + 1 : a.row_len;
        }

        if ((int64_t)a.k > valid) {
            // Fewer causal entries than k: the k-th largest is one of the
            // masked -inf entries, so every causal position is kept.
            if (tid == 0) {
                a.thr[row] = __uint_as_float(0xff800000u);
                if (a.cnt) a.cnt[row] = (int32_t)valid;
            }
            if (a.idx) {
                const int64_t n = valid < a.idx_cap ? valid : a.idx_cap;
                for (int64_t i = tid; i < n; i += BLOCK) a.idx[row * a.idx_cap + i] = (int32_t)i;
            }
            continue;  // block-uniform branch; no shared memory touched
        }

        const int ncache = (int)(valid < a.cache_elems ? valid : a.cache_elems);

        // ---- pass 0: stream the row from HBM, cache keys, histogram the top digit
        for (int i = tid; i < NHIST * NBINS; i += BLOCK) hist[i] = 0;
        __syncthreads();
        if (a.vec_ok) {
            const int64_t n4 = valid >> 2;
            const float4* src4 = reinterpret_cast<const float4*>(src);
            for (int64_t i4 = tid; i4 < n4; i4 += BLOCK) {
                const float4 v = __ldg(src4 + i4);
                const float f[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const uint32_t key = f2key(f[e]);
                    const int64_t i = 4 * i4 + e;
                    if (i < ncache) cache[i] = key;
                    atomicAdd(&my_hist[key >> 24], 1u);
                }
            }
            for (int64_t i = 4 * n4 + tid; i < valid; i += BLOCK) {
                const uint32_t key = f2key(__ldg(src + i));
                if (i < ncache) cache[i] = key;
                atomicAdd(&my_hist[key >> 24], 1u);
            }
        } else {
            for (int64_t i = tid; i < valid; i += BLOCK) {
                const uint32_t key = f2key(__ldg(src + i));
                if (i < ncache) cache[i] = key;
                atomicAdd(&my_hist[key >> 24], 1u);
            }
        }
        __syncthreads();

        uint32_t prefix = 0, pmask = 0, krem = (uint32_t)a.k;
#pragma unroll 1
        for (int pass = 0; pass < 4; ++pass) {
            const int shift = 24 - 8 * pass;
            if (pass > 0) {
                for (int64_t i = tid; i < valid; i += BLOCK) {
                    const uint32_t key = key_at<BLOCK>(cache, ncache, src, i);
                    if ((key & pmask) == prefix) atomicAdd(&my_hist[(key >> shift) & 255u], 1u);
                }
                __syncthreads();
            }
            // scan bins from the largest digit down; find where the count reaches krem
            uint32_t h = 0, incl = 0;
            if (tid < NBINS) {
                const int d = NBINS - 1 - tid;
#pragma unroll
                for (int c = 0; c < NHIST; ++c) h += hist[c * NBINS + d];
                incl = h;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += y;
                }
                if (lane == 31) warp_tot[warp] = incl;
            }
            __syncthreads();
            if (tid < NBINS) {
                for (int w2 = 0; w2 < warp; ++w2) incl += warp_tot[w2];
                if (incl >= krem && incl - h < krem) {
                    s_digit = (uint32_t)(NBINS - 1 - tid);
                    s_krem = krem - (incl - h);
                }
            }
            __syncthreads();
            prefix |= s_digit << shift;
            pmask |= 255u << shift;
            krem = s_krem;
            // clear for the next pass (everyone has read the histogram above)
            for (int i = tid; i < NHIST * NBINS; i += BLOCK) hist[i] = 0;
            __syncthreads();
        }
        const uint32_t thr_key = prefix;
        if (tid == 0) a.thr[row] = key2f(thr_key);

        if (a.idx || a.cnt) {
            // warp w owns the contiguous segment [w*seg, (w+1)*seg) of the row
            const int64_t seg = ((valid + NW - 1) / NW + 31) & ~int64_t(31);
            const int64_t s0 = warp * seg;
            const int64_t s1 = s0 + seg < valid ? s0 + seg : valid;
            uint32_t c = 0;
            for (int64_t i = s0 + lane; i - lane < s1; i += 32) {
                const bool p = i < s1 && key_at<BLOCK>(cache, ncache, src, i) >= thr_key;
                c += __popc(__ballot_sync(0xffffffffu, p));
            }
            if (lane == 0) warp_tot[warp] = c;
            __syncthreads();
            uint32_t base = 0;
            for (int w2 = 0; w2 < warp; ++w2) base += warp_tot[w2];
            if (tid == 0 && a.cnt) {
                uint32_t tot = 0;
                for (int w2 = 0; w2 < NW; ++w2) tot += warp_tot[w2];
                a.cnt[row] = (int32_t)tot;
            }
            if (a.idx) {
                int32_t* out = a.idx + row * a.idx_cap;
                for (int64_t i = s0 + lane; i - lane < s1; i += 32) {
                    const bool p = i < s1 && key_at<BLOCK>(cache, ncache, src, i) >= thr_key;
                    const uint32_t m = __ballot_sync(0xffffffffu, p);
                    const uint32_t pos = base + __popc(m & ((1u << lane) - 1u));
                    if (p && pos < a.idx_cap) out[pos] = (int32_t)i;
                    base += __popc(m);
                }
            }
        }
        __syncthreads();  // shared memory is reused by the next row
    }
}

template <int BLOCK>
int launch_topk(const TopkArgs& a, cudaStream_t stream) {
    const size_t smem = (size_t)a.cache_elems * sizeof(uint32_t);
    auto kern = topk_select_kernel<BLOCK>;
    // static + dynamic shared memory may pass 48 KB, which needs the opt-in
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
        return fail(DSA_ERR_CUDA, "topk_select: cannot set dynamic shared memory size");
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, BLOCK, smem) != cudaSuccess ||
        per_sm < 1)
        per_sm = 1;
    int64_t grid = (int64_t)num_sms() * per_sm;
    if (grid > a.n_rows) grid = a.n_rows;
    kern<<<(unsigned)grid, BLOCK, smem, stream>>>(a);
    return check_launch("topk_select_kernel");
}

}  // namespace

int topk_select(const float* scores, int64_t n_rows, int64_t row_len, int64_t row_stride,
                int64_t rows_per_batch, int64_t q_row0, int causal, int64_t k, float* thr,
                int32_t* idx, int32_t* cnt, int64_t idx_cap, cudaStream_t stream) {
    if (n_rows < 0 || row_len < 1 || row_stride < row_len)
        return fail(DSA_ERR_INVALID, "topk_select: need n_rows >= 0, row_len >= 1, row_stride >= row_len");
    if (k < 1 || k > row_len)
        return fail(DSA_ERR_INVALID, "topk_select: need 1 <= k <= row_len (k=" + std::to_string(k) +
                                         ", row_len=" + std::to_string(row_len) + ")");
    if (row_len > INT32_MAX || k > INT32_MAX) return fail(DSA_ERR_INVALID, "topk_select: row too long");
    if (causal && rows_per_batch < 1) return fail(DSA_ERR_INVALID, "topk_select: rows_per_batch < 1");
    if (q_row0 < 0) return fail(DSA_ERR_INVALID, "topk_select: q_row0 < 0");
    if (!scores || !thr) return fail(DSA_ERR_INVALID, "topk_select: scores and thr_out are required");
    if (idx && idx_cap < 1) return fail(DSA_ERR_INVALID, "topk_select: idx_cap < 1 with idx_out");
    if (n_rows == 0) return DSA_OK;

    TopkArgs a;
    a.scores = scores;
    a.n_rows = n_rows;
    a.row_len = row_len;
    a.row_stride = row_stride;
    a.rows_per_batch = causal ? rows_per_batch : 1;
    a.q_row0 = q_row0;
    a.causal = causal ? 1 : 0;
    a.k = (int)k;
    a.thr = thr;
    a.idx = idx;
    a.cnt = cnt;
    a.idx_cap = idx ? idx_cap : 0;
    a.vec_ok = (aligned16(scores) && row_stride % 4 == 0) ? 1 : 0;
    // longest row any CTA will see
    int64_t longest = row_len;
    if (causal) {
        const int64_t tmax = q_row0 + (n_rows < rows_per_batch ? n_rows : rows_per_batch) - 1;
        longest = tmax + 1 < row_len ? tmax + 1 : row_len;
    }
    constexpr int64_t kCacheMax = 12288;  // 48 KB of keys per CTA
    a.cache_elems = (int)(longest < kCacheMax ? longest : kCacheMax);
    if (longest <= 4096) return launch_topk<256>(a, stream);
    if (longest <= 16384) return launch_topk<512>(a, stream);
    return launch_topk<1024>(a, stream);
}

}  // namespace dsa
