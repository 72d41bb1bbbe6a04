// Stage 2: per-row top-K threshold and kept set by radix select.
//
// Replaces the GPU `scores.topk(k)` threshold of dsa_attention.py:343-344
// (which materialises k values and indices per row only to read one column)
// and the AVX-512 CPU k-th-largest of topk_avx512.cpp:226-249.
//
// Scores become order-preserving 32-bit keys (f2key: -0 folded onto +0, every
// NaN one key above +inf, as torch.topk ranks it).  The k-th largest key is
// found digit by digit from the top; the kernel depends on the row length:
//   <= 512      topk_warp_kernel: one warp per row, the keys in registers,
//               four radix passes over a per-warp histogram, no block barriers
//   513..4096   topk_warp_l2_kernel: one warp per row re-reading the row from
//               L2 on each of its 9+8+8+7-bit passes
//   4K..32K     topk_cached_kernel: one CTA per row.  One HBM sweep builds an
//               11-bit first-digit histogram; a block scan finds the bin d0 of
//               the k-th largest; the keys of bin d0 become candidates (with
//               their positions) and two radix passes (11 + 10 bits) over the
//               candidates give the exact key.  Bitmap rows write every word
//               from the first digit in the candidate sweep and OR in the kept
//               candidates; list rows emit ascending positions by
//               warp-segmented ballots.  Rows up to 8K with lists cache the keys
//               in shared memory; the others re-read the row from L2.
//               Bitmap-only rows given a workspace (the forward's) take
//               topk_sweep_kernel + topk_resolve_kernel instead: a 12-bit
//               first digit, two sweeps with four block barriers per row,
//               and the bin-d0 candidates resolved one warp per row.
//   > 32K       topk_select_kernel: four 8-bit passes, each filtering the row
// Rows with fewer causal entries than k keep every causal entry (threshold
// -inf).  Output is deterministic: lists are in ascending position order.
//
// Selection rule (dsa_attention.py:41-46): keep every position with
// score >= threshold (ties kept, NaN never kept) and, for causal rows, s <= t.
#include <stdlib.h>

#include <type_traits>

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
    uint32_t* bits;     // kept-set bitmap [n_rows, words] (CTA-per-row kernel only), or null
    int64_t words;
    int cache_elems;
    int cand_max;
    int cand_words;     // words of the candidate bitmap (uncached bitmap rows), multiple of 4
    int vec_ok;
    int64_t row_bstep;  // causal rows of batch bq sit at q_row0 + bq*row_bstep + (row % rows_per_batch)
};

// Causal length of a row: positions s <= t of query t (all of the row when not causal).
__device__ __forceinline__ int64_t row_valid(const TopkArgs& a, int64_t row) {
    if (!a.causal) return a.row_len;
    const int64_t bq = row / a.rows_per_batch;
    const int64_t t = a.q_row0 + bq * a.row_bstep + (row - bq * a.rows_per_batch);
    return t + 1 < a.row_len ? t + 1 : a.row_len;
}

// A row with fewer causal entries than k (valid < k): the k-th largest is one
// of the masked -inf entries, so the threshold is -inf and every causal entry
// is kept except NaNs (NaN >= -inf is false).  One warp writes the threshold,
// the count, the ascending index list and the bitmap words (zero past valid).
__device__ __forceinline__ void short_row_warp(const TopkArgs& a, int64_t row, const float* src,
                                               int64_t valid) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = (valid + 31) >> 5;
    const int64_t words = a.bits ? a.words : 0;
    const int64_t end = nw > words ? nw : words;
    uint32_t n = 0;
    for (int64_t wd = 0; wd < end; ++wd) {
        const int64_t s = wd * 32 + lane;
        const bool p = s < valid && !isnan(__ldg(src + s));
        const uint32_t m = __ballot_sync(0xffffffffu, p);
        if (a.idx) {
            const uint32_t pos = n + __popc(m & ((1u << lane) - 1u));
            if (p && pos < (uint32_t)a.idx_cap) a.idx[row * a.idx_cap + pos] = (int32_t)s;
        }
        if (wd < words && lane == 0) a.bits[row * a.words + wd] = m;
        n += __popc(m);
    }
    if (lane == 0) {
        a.thr[row] = __uint_as_float(0xff800000u);
        if (a.cnt) a.cnt[row] = (int32_t)n;
    }
}

// short_row_warp for a whole CTA: warp w takes a contiguous run of words, so
// the row is read by every warp at once (four words in flight per lane).
// wtot holds BLOCK/32 words of shared memory; ends with a barrier.
template <int BLOCK>
__device__ __forceinline__ void short_row_block(const TopkArgs& a, int64_t row, const float* src,
                                                int64_t valid, uint32_t* wtot) {
    constexpr int NW = BLOCK / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t nw = (valid + 31) >> 5;
    const int64_t words = a.bits ? a.words : 0;
    const int64_t end = nw > words ? nw : words;
    const int64_t seg = (end + NW - 1) / NW;
    const int64_t w0 = warp * seg, w1 = w0 + seg < end ? w0 + seg : end;
    auto word = [&](int64_t wd) {
        const int64_t s = wd * 32 + lane;
        return __ballot_sync(0xffffffffu, s < valid && !isnan(__ldg(src + s)));
    };
    uint32_t n = 0;
    for (int64_t wd = w0; wd < w1; wd += 4) {
        uint32_t m[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) m[u] = wd + u < w1 ? word(wd + u) : 0u;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (wd + u < words && lane == 0) a.bits[row * a.words + wd + u] = m[u];
            n += __popc(m[u]);
        }
    }
    if (lane == 0) wtot[warp] = n;
    __syncthreads();
    uint32_t base = 0, tot = 0;
#pragma unroll
    for (int w2 = 0; w2 < NW; ++w2) {
        base += w2 < warp ? wtot[w2] : 0u;
        tot += wtot[w2];
    }
    if (a.idx) {
        for (int64_t wd = w0; wd < w1 && wd < nw; ++wd) {
            const uint32_t m = word(wd);
            const uint32_t pos = base + __popc(m & ((1u << lane) - 1u));
            if (((m >> lane) & 1u) && pos < (uint32_t)a.idx_cap) a.idx[row * a.idx_cap + pos] = (int32_t)(wd * 32 + lane);
            base += __popc(m);
        }
    }
    if (threadIdx.x == 0) {
        a.thr[row] = __uint_as_float(0xff800000u);
        if (a.cnt) a.cnt[row] = (int32_t)tot;
    }
    __syncthreads();
}

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
        const int64_t valid = row_valid(a, row);

        if ((int64_t)a.k > valid) {
            short_row_block<BLOCK>(a, row, src, valid, warp_tot);
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
                const bool p = i < s1 && kept_key(key_at<BLOCK>(cache, ncache, src, i), thr_key);
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
                    const bool p = i < s1 && kept_key(key_at<BLOCK>(cache, ncache, src, i), thr_key);
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

// ===========================================================================
// Rows that fit in shared memory (up to kRowCache entries, every row of the
// reference's configurations): the fast kernel.
//
//   sweep 1  HBM -> key cache (float4 loads, uint4 stores) + histogram of the
//            top 11 key bits; a block scan finds the bin d0 holding the k-th
//            largest key
//   sweep 2  over the cache: keys of bin d0 go with their positions to a
//            candidate list; each warp counts the keys above bin d0 in its
//            contiguous segment of the row
//   passes   two radix passes (11 + 10 bits) over the candidates alone give
//            the exact k-th largest key; kept candidates add to their
//            segment's count
//   sweep 3  ordered emission: a warp-wide scan of per-lane kept counts
//            places every kept position of the warp's segment
// A row whose bin d0 overflows the candidate buffer runs the two passes over
// the cached row instead.  All row indexing is 32-bit.
// ===========================================================================

constexpr int kRowCache = 32768;   // keys cached per CTA (128 KB)
constexpr int NB_TOP = 2048;       // 11-bit first digit

// Exclusive block-wide prefix sum of v; *total gets the sum.  Two barriers.
template <int BLOCK>
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t* wtot, uint32_t* total) {
    constexpr int NW = BLOCK / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) wtot[warp] = incl;
    __syncthreads();
    uint32_t before = 0, tot = 0;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        const uint32_t x = wtot[w];
        before += w < warp ? x : 0u;
        tot += x;
    }
    *total = tot;
    __syncthreads();
    return before + incl - v;
}

// Histograms of the fast kernel are stored in descending-digit order
// (slot nb-1-digit), so each thread's scan range is contiguous and is read as
// uint4s.  Finds the slot holding the krem-th largest key: res[0] = digit,
// res[1] = rank left inside the bin.  nbins is a power of two >= 4*32.
// Ends with a barrier.
template <int BLOCK>
__device__ __forceinline__ void block_find_desc(const uint32_t* hist, int nbins, uint32_t krem,
                                                uint32_t* wtot, uint32_t* res) {
    const int per4 = nbins >= 4 * BLOCK ? nbins / (4 * BLOCK) : 1;  // uint4s per thread
    const bool has = (int)threadIdx.x * per4 * 4 < nbins;
    const uint4* h4 = reinterpret_cast<const uint4*>(hist) + threadIdx.x * per4;
    uint32_t local = 0;
    for (int i = 0; has && i < per4; ++i) {
        const uint4 v = h4[i];
        local += v.x + v.y + v.z + v.w;
    }
    uint32_t tot;
    const uint32_t excl = block_excl_scan<BLOCK>(local, wtot, &tot);
    if (has && excl < krem && krem <= excl + local) {
        uint32_t c = excl;
        const int r0 = threadIdx.x * per4 * 4;
        for (int i = 0; i < per4 * 4; ++i) {
            const uint32_t h = hist[r0 + i];
            if (krem <= c + h) {
                res[0] = (uint32_t)(nbins - 1 - (r0 + i));
                res[1] = krem - c;
                break;
            }
            c += h;
        }
    }
    __syncthreads();
}

// Keys of group g (4 positions) of a row: from the shared cache, or (for rows
// kept out of shared memory) re-read from L2; positions >= valid give key 0.
template <bool CACHED>
__device__ __forceinline__ uint4 group_keys(const uint4* cache4, const float* src, int g, int valid,
                                            int vec_ok) {
    if constexpr (CACHED) {
        return cache4[g];
    } else {
        if (vec_ok && 4 * g + 3 < valid) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(src) + g);
            return make_uint4(f2key(v.x), f2key(v.y), f2key(v.z), f2key(v.w));
        }
        uint32_t e[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) e[j] = 4 * g + j < valid ? f2key(__ldg(src + 4 * g + j)) : 0u;
        return make_uint4(e[0], e[1], e[2], e[3]);
    }
}

// Kept-set bitmap of one row: bit s % 32 of word s / 32 is set iff s < valid
// and kept_key(key(s), thr_key).  Each thread turns one
// float4 group into a nibble and eight lanes OR theirs into a word; words is
// a multiple of 4, so every warp runs the same number of iterations.
template <int BLOCK, bool CACHED>
__device__ __forceinline__ void emit_bits(const TopkArgs& a, int64_t row, const float* src,
                                          const uint4* cache4, int valid, uint32_t thr_key) {
    uint32_t* out = a.bits + row * a.words;
    const int ng = (int)a.words * 8;
    const int g4 = (valid + 3) >> 2;
    const int lane = threadIdx.x & 31;
    for (int g = threadIdx.x; g < ng; g += BLOCK) {
        uint32_t nib = 0;
        if (g < g4) {
            // keys past `valid` are 0, below every real key
            const uint4 kk = group_keys<CACHED>(cache4, src, g, valid, a.vec_ok);
            nib = (uint32_t)kept_key(kk.x, thr_key) | (uint32_t)kept_key(kk.y, thr_key) << 1 |
                  (uint32_t)kept_key(kk.z, thr_key) << 2 | (uint32_t)kept_key(kk.w, thr_key) << 3;
        }
        uint32_t w = nib << (4 * (lane & 7));
        w |= __shfl_xor_sync(0xffffffffu, w, 1);
        w |= __shfl_xor_sync(0xffffffffu, w, 2);
        w |= __shfl_xor_sync(0xffffffffu, w, 4);
        if ((lane & 7) == 0) out[g >> 3] = w;
    }
}

// One row exactly, for rows holding NaN: four 8-bit radix passes over the
// canonical keys (every NaN one key above +inf), re-reading the row from L2
// each pass, then the count, the ascending list and the bitmap words.  Uses
// hist[0..255]; ends with a barrier.  Kept out of line so the hot kernel's
// register allocation does not carry it.
template <int BLOCK>
__device__ __noinline__ void exact_row_slow(const float* src, int valid, int k, float* thr_out,
                                            int32_t* cnt_out, int32_t* idx_out, int64_t idx_cap,
                                            uint32_t* bits_out, int64_t words, uint32_t* hist,
                                            uint32_t* wtot, uint32_t* res) {
    constexpr int NW = BLOCK / 32;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint32_t prefix = 0, pmask = 0, krem = (uint32_t)k;
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        for (int i = tid; i < 256; i += BLOCK) hist[i] = 0;
        __syncthreads();
        for (int i = tid; i < valid; i += BLOCK) {
            const uint32_t key = f2key(__ldg(src + i));
            if ((key & pmask) == prefix) atomicAdd(&hist[255 - ((key >> shift) & 255u)], 1u);
        }
        __syncthreads();
        block_find_desc<BLOCK>(hist, 256, krem, wtot, res);
        prefix |= res[0] << shift;
        pmask |= 255u << shift;
        krem = res[1];
    }
    const uint32_t thr_key = prefix;
    // warp w owns the contiguous segment [w*seg, (w+1)*seg) of the row
    const int seg = ((valid + NW - 1) / NW + 31) & ~31;
    const int s0 = warp * seg, s1 = s0 + seg < valid ? s0 + seg : valid;
    uint32_t c = 0;
    for (int i = s0 + lane; i - lane < s1; i += 32)
        c += __popc(__ballot_sync(0xffffffffu, i < s1 && kept_key(f2key(__ldg(src + i)), thr_key)));
    if (lane == 0) wtot[warp] = c;
    __syncthreads();
    uint32_t base = 0, tot = 0;
    for (int w2 = 0; w2 < NW; ++w2) {
        base += w2 < warp ? wtot[w2] : 0u;
        tot += wtot[w2];
    }
    if (tid == 0) {
        *thr_out = key2f(thr_key);
        if (cnt_out) *cnt_out = (int32_t)tot;
    }
    if (idx_out) {
        for (int i = s0 + lane; i - lane < s1; i += 32) {
            const bool p = i < s1 && kept_key(f2key(__ldg(src + i)), thr_key);
            const uint32_t m = __ballot_sync(0xffffffffu, p);
            const uint32_t pos = base + __popc(m & ((1u << lane) - 1u));
            if (p && pos < idx_cap) idx_out[pos] = i;
            base += __popc(m);
        }
    }
    if (bits_out) {
        for (int64_t wd = warp; wd < words; wd += NW) {
            const int64_t s = wd * 32 + lane;
            const bool p = s < valid && kept_key(f2key(__ldg(src + s)), thr_key);
            const uint32_t m = __ballot_sync(0xffffffffu, p);
            if (lane == 0) bits_out[wd] = m;
        }
    }
    __syncthreads();
}

template <int BLOCK, bool CACHED>
__global__ void __launch_bounds__(BLOCK, CACHED ? 1 : 1280 / BLOCK) topk_cached_kernel(TopkArgs a) {
    constexpr int NW = BLOCK / 32;
    constexpr int S0 = 21;  // shift of the first digit
    extern __shared__ uint4 dyn4[];
    uint32_t* cache = reinterpret_cast<uint32_t*>(dyn4);      // cache_elems keys (multiple of 4)
    uint32_t* cand_key = cache + a.cache_elems;               // cand_max
    int32_t* cand_pos = reinterpret_cast<int32_t*>(cand_key + a.cand_max);
    uint32_t* cbits = reinterpret_cast<uint32_t*>(cand_pos + a.cand_max);   // cand_words

    __shared__ __align__(16) uint32_t hist[NB_TOP];
    __shared__ uint32_t wtot[NW];
    __shared__ uint32_t seg_cnt[NW];
    __shared__ uint32_t seg_base[NW + 1];
    __shared__ uint32_t res[2];
    __shared__ uint32_t n_cand;
    __shared__ uint32_t n_keep;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    for (int64_t row = blockIdx.x; row < a.n_rows; row += gridDim.x) {
        const float* src = a.scores + row * a.row_stride;
        const int valid = (int)row_valid(a, row);
        if (a.k > valid) {
            short_row_block<BLOCK>(a, row, src, valid, wtot);
            continue;  // block-uniform branch
        }
        const int g4 = (valid + 3) >> 2;  // uint4 groups; padding keys are 0

        // ---- sweep 1 (raw keys: equal to f2key on rows without NaN, see below)
        for (int i = tid; i < NB_TOP; i += BLOCK) hist[i] = 0;
        if (tid == 0) n_cand = 0;
        __syncthreads();
        if (a.vec_ok) {
            // full groups, eight float4 loads in flight per thread
            const float4* src4 = reinterpret_cast<const float4*>(src);
            const int gfull = valid >> 2;
            constexpr int PIPE = 8;
            for (int g0 = tid; g0 < gfull; g0 += PIPE * BLOCK) {
                float4 v[PIPE];
#pragma unroll
                for (int u = 0; u < PIPE; ++u) {
                    const int g = g0 + u * BLOCK;
                    v[u] = g < gfull ? __ldg(src4 + g) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int u = 0; u < PIPE; ++u) {
                    const int g = g0 + u * BLOCK;
                    if (g < gfull) {
                        const uint4 kk = make_uint4(f2key_raw(v[u].x), f2key_raw(v[u].y), f2key_raw(v[u].z),
                                                    f2key_raw(v[u].w));
                        atomicAdd(&hist[(NB_TOP - 1) - (kk.x >> S0)], 1u);
                        atomicAdd(&hist[(NB_TOP - 1) - (kk.y >> S0)], 1u);
                        atomicAdd(&hist[(NB_TOP - 1) - (kk.z >> S0)], 1u);
                        atomicAdd(&hist[(NB_TOP - 1) - (kk.w >> S0)], 1u);
                        if (CACHED) dyn4[g] = kk;
                    }
                }
            }
            if (gfull < g4 && tid == BLOCK - 1) {  // the partial last group
                uint32_t e[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    e[j] = 4 * gfull + j < valid ? f2key_raw(__ldg(src + 4 * gfull + j)) : 0u;
                    if (4 * gfull + j < valid) atomicAdd(&hist[(NB_TOP - 1) - (e[j] >> S0)], 1u);
                }
                if (CACHED) dyn4[gfull] = make_uint4(e[0], e[1], e[2], e[3]);
            }
        } else {
            for (int g = tid; g < g4; g += BLOCK) {
                uint32_t e[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    e[j] = 4 * g + j < valid ? f2key_raw(__ldg(src + 4 * g + j)) : 0u;
                    if (4 * g + j < valid) atomicAdd(&hist[(NB_TOP - 1) - (e[j] >> S0)], 1u);
                }
                if (CACHED) dyn4[g] = make_uint4(e[0], e[1], e[2], e[3]);
            }
        }
        __syncthreads();
        // no key in bins 0-3 or 2044-2047 (NaNs, infinities and their
        // neighbours): float order is key order on this row
        const bool plain = (hist[0] | hist[1] | hist[2] | hist[3] | hist[NB_TOP - 4] | hist[NB_TOP - 3] |
                            hist[NB_TOP - 2] | hist[NB_TOP - 1]) == 0u;
        if (!plain) {
            // every NaN falls in those bins; a row that holds one takes the
            // exact slow path with NaN-canonical keys (rare rows)
            bool nan_here = false;
            for (int i = tid; i < valid && !nan_here; i += BLOCK) nan_here = isnan(__ldg(src + i));
            if (__syncthreads_or(nan_here)) {
                exact_row_slow<BLOCK>(src, valid, a.k, a.thr + row, a.cnt ? a.cnt + row : nullptr,
                                      a.idx ? a.idx + row * a.idx_cap : nullptr, a.idx_cap,
                                      a.bits ? a.bits + row * a.words : nullptr, a.words, hist, wtot, res);
                continue;   // block-uniform
            }
        }
        block_find_desc<BLOCK>(hist, NB_TOP, (uint32_t)a.k, wtot, res);
        const uint32_t d0 = res[0];
        uint32_t krem = res[1];
        const bool use_cand = hist[(NB_TOP - 1) - d0] <= (uint32_t)a.cand_max;
        __syncthreads();

        // warp w owns groups [w*gseg, min((w+1)*gseg, g4))
        const int gseg = (g4 + NW - 1) / NW;
        const int gs0 = warp * gseg;
        const int gs1 = gs0 + gseg < g4 ? gs0 + gseg : g4;
        uint32_t prefix = d0 << S0, pmask = ~0u << S0;

        if (a.bits && !a.idx && use_cand) {
            // Bitmap-only rows: one sweep writes every word from the first
            // digit alone (keys in bins above d0 are kept, below d0 dropped)
            // and collects bin d0's keys; the exact threshold inside d0 then
            // ORs the kept candidates in.  k - krem keys lie above bin d0.
            uint32_t* out = a.bits + row * a.words;
            // causal groups: keys at or above bin d0+1 set their bit; keys of
            // bin d0 become candidates (an unordered list: the selection does
            // not depend on their order).  Only the last group has positions
            // past `valid`; padding keys are 0, below every real bin above d0.
            // bin d0 = [lo, hi_key); for the top bin, hi_key = the largest key,
            // which is kept whatever the threshold in that bin is
            const uint32_t lo = d0 << S0;
            const uint32_t hi_key = d0 == NB_TOP - 1 ? 0xffffffffu : (d0 + 1) << S0;
            const int gw = ((g4 + 7) >> 3) << 3;   // groups of the words holding causal keys
            constexpr int PIPE = CACHED ? 1 : 4;
            // loop and break tests use the warp's first group (g0 - lane), so
            // whole warps run the shuffles; gw is a multiple of 8, so the 8
            // lanes of a word are all inside or all past it
            const bool float_path = !CACHED && plain && d0 >= 4 && d0 <= NB_TOP - 5;
            if (float_path) {
                // float compares against the bin edges (finite floats here);
                // positions past `valid` read as -inf, below bin d0
                const float hi_f = key2f(hi_key), lo_f = key2f(lo);
                // Warp w takes chunks of 32 words (1024 positions): lane L reads
                // position 32*i + L of word i, so one ballot per word gives the
                // kept bits (above bin d0) and one the candidates (bin d0); lane i
                // keeps word i and the chunk is stored as one coalesced line.
                // Words past `valid` (up to the row's word count) come out zero.
                const int nwords = (int)a.words;
                constexpr int SW2 = 16;   // loads in flight per lane
                for (int ch = warp; ch < ((nwords + 31) >> 5); ch += NW) {
                    const int s0c = ch * 1024;
                    uint32_t my_ab = 0, my_cb = 0;
                    if (s0c < valid) {
#pragma unroll 1
                        for (int i0 = 0; i0 < 32; i0 += SW2) {
                            float x[SW2];
#pragma unroll
                            for (int u = 0; u < SW2; ++u) {
                                const int sp = s0c + (i0 + u) * 32 + lane;
                                x[u] = sp < valid ? __ldg(src + sp) : __uint_as_float(0xff800000u);
                            }
#pragma unroll
                            for (int u = 0; u < SW2; ++u) {
                                const uint32_t ab = __ballot_sync(0xffffffffu, x[u] >= hi_f);
                                const uint32_t cb = __ballot_sync(0xffffffffu, x[u] >= lo_f && x[u] < hi_f);
                                if (lane == i0 + u) {
                                    my_ab = ab;
                                    my_cb = cb;
                                }
                            }
                        }
                    }
                    const int wd = ch * 32 + lane;
                    if (wd < nwords) out[wd] = my_ab;
                    if (wd < a.cand_words) cbits[wd] = my_cb;
                }
            } else
            for (int g0 = tid; g0 - lane < gw; g0 += PIPE * BLOCK) {
                uint4 kb[PIPE];
#pragma unroll
                for (int u = 0; u < PIPE; ++u) {
                    const int g = g0 + u * BLOCK;
                    kb[u] = g < g4 ? group_keys<CACHED>(dyn4, src, g, valid, a.vec_ok) : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int u = 0; u < PIPE; ++u) {
                    const int g = g0 + u * BLOCK;
                    if (g - lane >= gw) break;
                    const uint32_t e[4] = {kb[u].x, kb[u].y, kb[u].z, kb[u].w};
                    uint32_t nib = 0;
#pragma unroll
                    for (int j = 0; j < 4; ++j) nib |= (uint32_t)(e[j] >= hi_key) << j;
                    uint32_t wd = nib << (4 * (lane & 7));
                    wd |= __shfl_xor_sync(0xffffffffu, wd, 1);
                    wd |= __shfl_xor_sync(0xffffffffu, wd, 2);
                    wd |= __shfl_xor_sync(0xffffffffu, wd, 4);
                    if ((lane & 7) == 0 && g < gw) out[g >> 3] = wd;
                    if (g < g4) {
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            if (e[j] - lo < (1u << S0) && (g + 1 < g4 || 4 * g + j < valid)) {
                                const uint32_t at = atomicAdd(&n_cand, 1u);
                                if (DSA_CHECK(at < (uint32_t)a.cand_max, DBG_CAND_OVERFLOW)) {
                                    cand_key[at] = e[j];
                                    cand_pos[at] = 4 * g + j;
                                }
                            }
                    }
                }
            }
            // words past the causal end (the float path wrote them)
            if (!float_path)
                for (int wi = (gw >> 3) + tid; wi < (int)a.words; wi += BLOCK) out[wi] = 0u;
            if (tid == 0) n_keep = 0;
            __syncthreads();
            int nc = (int)n_cand;
            if (float_path) {
                // The candidate bitmap becomes the candidate list, in ascending
                // position: each thread takes a run of words, a block scan of
                // their popcounts places them, and each candidate's score is read
                // back (from L2) for its key.  No per-candidate atomics.
                const int nwc = gw >> 3;
                const int per = (nwc + BLOCK - 1) / BLOCK;
                const int w0 = tid * per, w1 = w0 + per < nwc ? w0 + per : nwc;
                uint32_t c = 0;
                for (int w = w0; w < w1; ++w) c += __popc(cbits[w]);
                uint32_t tot;
                uint32_t at = block_excl_scan<BLOCK>(c, wtot, &tot);
                for (int w = w0; w < w1; ++w) {
                    uint32_t m = cbits[w];
                    while (m) {
                        const int pos = w * 32 + __ffs(m) - 1;
                        m &= m - 1;
                        if (DSA_CHECK(at < (uint32_t)a.cand_max, DBG_CAND_OVERFLOW)) {
                            cand_key[at] = f2key_raw(__ldg(src + pos));   // no NaN on this path
                            cand_pos[at] = pos;
                        }
                        ++at;
                    }
                }
                nc = (int)tot;
                __syncthreads();
            }
            const uint32_t above = (uint32_t)a.k - krem;
#pragma unroll 1
            for (int pass = 1; pass <= 2; ++pass) {
                const int shift = pass == 1 ? 10 : 0;
                const int nb = pass == 1 ? 2048 : 1024;
                for (int i = tid; i < nb; i += BLOCK) hist[i] = 0;
                __syncthreads();
                for (int i = tid; i < nc; i += BLOCK) {
                    const uint32_t key = cand_key[i];
                    if ((key & pmask) == prefix)
                        atomicAdd(&hist[(nb - 1) - ((key >> shift) & (nb - 1))], 1u);
                }
                __syncthreads();
                block_find_desc<BLOCK>(hist, nb, krem, wtot, res);
                prefix |= res[0] << shift;
                pmask |= (uint32_t)(nb - 1) << shift;
                krem = res[1];
            }
            // the words are written (the barriers above order them before the ORs)
            uint32_t kc = 0;
            for (int i = tid; i < nc; i += BLOCK)
                if (kept_key(cand_key[i], prefix)) {
                    atomicOr(out + (cand_pos[i] >> 5), 1u << (cand_pos[i] & 31));
                    ++kc;
                }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) kc += __shfl_xor_sync(0xffffffffu, kc, o);
            if (lane == 0 && kc) atomicAdd(&n_keep, kc);
            __syncthreads();
            if (tid == 0) {
                a.thr[row] = key2f(prefix);
                if (a.cnt) a.cnt[row] = (int32_t)(above + n_keep);
            }
            __syncthreads();
            continue;
        }

        if (use_cand) {
            // ---- sweep 2: candidates + per-segment count of keys above bin d0
            uint32_t above = 0;
            for (int gb = gs0; gb < gs1; gb += 32) {
                const int g = gb + lane;
                uint4 kk = g < gs1 ? group_keys<CACHED>(dyn4, src, g, valid, a.vec_ok) : make_uint4(0, 0, 0, 0);
                const uint32_t e[4] = {kk.x, kk.y, kk.z, kk.w};
                uint32_t nin = 0;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    above += (e[j] >> S0) > d0;
                    nin += (e[j] >> S0) == d0;
                }
                // padding keys are 0: digit 0, never == d0 for finite data
                if (__any_sync(0xffffffffu, nin != 0)) {
                    uint32_t pre = nin;
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const uint32_t y = __shfl_up_sync(0xffffffffu, pre, o);
                        if (lane >= o) pre += y;
                    }
                    uint32_t base = 0;
                    if (lane == 31) base = atomicAdd(&n_cand, pre);
                    base = __shfl_sync(0xffffffffu, base, 31) + pre - nin;
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        if ((e[j] >> S0) == d0) {
                            if (DSA_CHECK(base < (uint32_t)a.cand_max, DBG_CAND_OVERFLOW)) {
                                cand_key[base] = e[j];
                                cand_pos[base] = 4 * g + j;
                            }
                            ++base;
                        }
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) above += __shfl_xor_sync(0xffffffffu, above, o);
            if (lane == 0) seg_cnt[warp] = above;
            __syncthreads();
            const int nc = (int)n_cand;
#pragma unroll 1
            for (int pass = 1; pass <= 2; ++pass) {
                const int shift = pass == 1 ? 10 : 0;
                const int nb = pass == 1 ? 2048 : 1024;
                for (int i = tid; i < nb; i += BLOCK) hist[i] = 0;
                __syncthreads();
                for (int i = tid; i < nc; i += BLOCK) {
                    const uint32_t key = cand_key[i];
                    if ((key & pmask) == prefix)
                        atomicAdd(&hist[(nb - 1) - ((key >> shift) & (nb - 1))], 1u);
                }
                __syncthreads();
                block_find_desc<BLOCK>(hist, nb, krem, wtot, res);
                prefix |= res[0] << shift;
                pmask |= (uint32_t)(nb - 1) << shift;
                krem = res[1];
            }
            for (int i = tid; i < nc; i += BLOCK)
                if (kept_key(cand_key[i], prefix)) atomicAdd(&seg_cnt[(cand_pos[i] >> 2) / gseg], 1u);
            __syncthreads();
        } else {
#pragma unroll 1
            for (int pass = 1; pass <= 2; ++pass) {
                const int shift = pass == 1 ? 10 : 0;
                const int nb = pass == 1 ? 2048 : 1024;
                for (int i = tid; i < nb; i += BLOCK) hist[i] = 0;
                __syncthreads();
                for (int g = tid; g < g4; g += BLOCK) {
                    const uint4 kk = group_keys<CACHED>(dyn4, src, g, valid, a.vec_ok);
                    const uint32_t e[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        if (4 * g + j < valid && (e[j] & pmask) == prefix)
                            atomicAdd(&hist[(nb - 1) - ((e[j] >> shift) & (nb - 1))], 1u);
                }
                __syncthreads();
                block_find_desc<BLOCK>(hist, nb, krem, wtot, res);
                prefix |= res[0] << shift;
                pmask |= (uint32_t)(nb - 1) << shift;
                krem = res[1];
            }
            uint32_t c = 0;
            for (int g = gs0 + lane; g < gs1; g += 32) {
                const uint4 kk = group_keys<CACHED>(dyn4, src, g, valid, a.vec_ok);
                c += kept_key(kk.x, prefix) + kept_key(kk.y, prefix) + kept_key(kk.z, prefix) +
                     kept_key(kk.w, prefix);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
            if (lane == 0) seg_cnt[warp] = c;
            __syncthreads();
        }
        const uint32_t thr_key = prefix;

        // ---- sweep 3: ordered emission (warp 0 turns segment counts into offsets)
        if (warp == 0) {
            const uint32_t c = lane < NW ? seg_cnt[lane] : 0u;
            uint32_t incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            if (lane < NW) seg_base[lane] = incl - c;
            if (lane == 31) seg_base[NW] = incl;
        }
        __syncthreads();
        uint32_t base = seg_base[warp];
        const uint32_t tot = seg_base[NW];
        if (tid == 0) {
            a.thr[row] = key2f(thr_key);
            if (a.cnt) a.cnt[row] = (int32_t)tot;
        }
        if (a.idx) {
            int32_t* out = a.idx + row * a.idx_cap;
            const uint32_t cap = (uint32_t)a.idx_cap;
            for (int gb = gs0; gb < gs1 && base < cap; gb += 32) {
                const int g = gb + lane;
                const uint4 kk = g < gs1 ? group_keys<CACHED>(dyn4, src, g, valid, a.vec_ok) : make_uint4(0, 0, 0, 0);
                const bool p0 = kept_key(kk.x, thr_key), p1 = kept_key(kk.y, thr_key),
                           p2 = kept_key(kk.z, thr_key), p3 = kept_key(kk.w, thr_key);
                const uint32_t n = p0 + p1 + p2 + p3;
                uint32_t pre = n;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t y = __shfl_up_sync(0xffffffffu, pre, o);
                    if (lane >= o) pre += y;
                }
                uint32_t pos = base + pre - n;
                if (p0 && pos < cap) out[pos] = 4 * g;
                pos += p0;
                if (p1 && pos < cap) out[pos] = 4 * g + 1;
                pos += p1;
                if (p2 && pos < cap) out[pos] = 4 * g + 2;
                pos += p2;
                if (p3 && pos < cap) out[pos] = 4 * g + 3;
                base += __shfl_sync(0xffffffffu, pre, 31);
            }
        }
        if (a.bits) emit_bits<BLOCK, CACHED>(a, row, src, dyn4, valid, thr_key);
        __syncthreads();
    }
}

// cand_div: the candidate buffer holds longest / cand_div keys (256..4096);
// a row whose threshold bin has more keys takes the exact path without it
template <int BLOCK, bool CACHED>
int launch_cached(TopkArgs a, int64_t longest, cudaStream_t stream, int cand_div = 4) {
    a.cache_elems = CACHED ? (int)((longest + 3) & ~int64_t(3)) : 0;
    const int64_t cm = longest / cand_div;
    a.cand_max = (int)(cm < 256 ? 256 : cm > 4096 ? 4096 : cm);
    // uncached rows: a candidate bitmap word per 32 positions (bitmap-only rows)
    a.cand_words = CACHED ? 0 : (int)(((longest + 127) / 128) * 4);
    const size_t smem = ((size_t)a.cache_elems + 2 * (size_t)a.cand_max + a.cand_words) * sizeof(uint32_t);
    auto kern = topk_cached_kernel<BLOCK, CACHED>;
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
    return check_launch("topk_cached_kernel");
}

// ===========================================================================
// Bitmap-only rows of 4K..32K entries (the forward's c4 and c5 rows) in two
// kernels, given a workspace.  The first streams the rows with four block
// barriers per row; the second resolves each row's threshold from its
// candidates, one warp per row.
//
// topk_sweep_kernel, one CTA per row:
//   sweep 1 (HBM)  histogram of the keys' top DBITS bits (12: sign, exponent
//                  and three mantissa bits, so the bin holding the k-th
//                  largest key of a c5 row keeps a few hundred keys)
//   find           the bin d0 holding the k-th largest key and the rank krem
//                  left inside it; each thread zeroes the bins it scanned, so
//                  the histogram is clear for the next row without a pass
//   sweep 2 (L2)   per 32 positions, one ballot gives the word of keys above
//                  bin d0 (final bits of the bitmap), one the word of keys in
//                  bin d0; after each 1024-position chunk the warp appends
//                  that chunk's bin-d0 keys and positions to the row's
//                  candidate list (one shared add per chunk; the keys are read
//                  back while the chunk is still in L2)
//   The row's (d0, krem, count) go to a meta word; the row ends without a
//   barrier, so warps run ahead into the next row's sweep 1.  Rows shorter
//   than k, rows holding NaN or an infinity (keys in the 16 edge bins at
//   either end) and rows whose bin d0 holds more keys than the list are
//   finished here (short_row_block / exact_row_slow) and marked done.
// topk_resolve_kernel, one warp per row:
//   three radix passes (8 + 8 + 4 bits) over the candidates' low 20 bits for
//   the exact krem-th largest, the kept candidates ORed into the bitmap, the
//   row's threshold and count.
// Output equals the one-kernel path's: threshold, count, bitmap words.
// ===========================================================================
constexpr uint32_t kRowDone = 0xffffffffu;   // meta.x of a row finished by the sweep kernel

template <int BLOCK, int DBITS>
__device__ __forceinline__ void fine_find(uint32_t* hist, uint32_t krem, uint32_t* wtot,
                                          uint32_t* res) {
    constexpr int NB = 1 << DBITS;
    constexpr int PER4 = NB / (4 * BLOCK);   // uint4 slots per thread
    static_assert(PER4 >= 1, "fine_find: at least 4 bins per thread");
    uint4* h4 = reinterpret_cast<uint4*>(hist) + threadIdx.x * PER4;
    uint32_t local = 0;
#pragma unroll
    for (int i = 0; i < PER4; ++i) {
        const uint4 v = h4[i];
        local += v.x + v.y + v.z + v.w;
    }
    // the edge bins (slots 0-15: NaN/+inf; slots NB-16..NB-1: -inf/-NaN)
    if (threadIdx.x == 0 || threadIdx.x == BLOCK - 1) {
        uint32_t e = 0;
        const int s0 = threadIdx.x == 0 ? 0 : NB - 16;
        for (int i = 0; i < 16; ++i) e |= hist[s0 + i];
        res[threadIdx.x == 0 ? 3 : 4] = e;
    }
    uint32_t tot;
    const uint32_t excl = block_excl_scan<BLOCK>(local, wtot, &tot);
    if (excl < krem && krem <= excl + local) {
        uint32_t c = excl;
        const int r0 = threadIdx.x * PER4 * 4;
        for (int i = 0; i < PER4 * 4; ++i) {
            const uint32_t h = hist[r0 + i];
            if (krem <= c + h) {
                res[0] = (uint32_t)(NB - 1 - (r0 + i));
                res[1] = krem - c;
                res[2] = h;
                break;
            }
            c += h;
        }
    }
    // every thread clears the slots it scanned (the crossing thread after its re-read)
#pragma unroll
    for (int i = 0; i < PER4; ++i) h4[i] = make_uint4(0, 0, 0, 0);
    __syncthreads();
}

// Candidate lists of the two-kernel bitmap path: per row, cap keys and cap
// 16-bit positions (rows of up to 32768 positions), and a meta word.
struct CandLists {
    uint32_t* key;   // [n_rows][cap]
    uint16_t* pos;   // [n_rows][cap]
    uint4* meta;     // [n_rows]: d0 (kRowDone: row finished by the sweep), krem, candidate count
    int cap;
};

// candidates a row may hold: 1/8 of its positions, 256..2048.  On the
// indexer's scores of a c5 sequence (t up to 32K, k = 2048) the threshold's
// 12-bit bin holds up to ~1,250 keys (about 3% of the row: those scores are
// wide relative to the threshold); with 1/16 (at most 1,024) about 5% of the
// long rows overflowed into the exact per-row path
__host__ __device__ inline int cand_cap_for(int64_t words) {
    const int64_t c = words * 4;
    return (int)(c < 256 ? 256 : c > 2048 ? 2048 : c);
}

inline size_t align256_sz(size_t x) { return (x + 255) / 256 * 256; }

size_t sweep_ws_bytes(int64_t n_rows, int64_t words) {
    const size_t cap = (size_t)cand_cap_for(words);
    return align256_sz((size_t)n_rows * cap * sizeof(uint32_t)) + align256_sz((size_t)n_rows * cap * sizeof(uint16_t)) +
           (size_t)n_rows * sizeof(uint4);
}

CandLists cand_lists(void* ws, int64_t n_rows, int64_t words) {
    CandLists c;
    c.cap = cand_cap_for(words);
    char* p = static_cast<char*>(ws);
    c.key = reinterpret_cast<uint32_t*>(p);
    p += align256_sz((size_t)n_rows * c.cap * sizeof(uint32_t));
    c.pos = reinterpret_cast<uint16_t*>(p);
    p += align256_sz((size_t)n_rows * c.cap * sizeof(uint16_t));
    c.meta = reinterpret_cast<uint4*>(p);
    return c;
}

// Sweep 2 over one chunk of 32 words (1024 positions) of a row: lane L reads
// position 32*i + L of word i, so one ballot gives word i's kept bits (keys
// above bin d0) and another its candidates (keys inside bin d0); lane 0
// stages both words in the warp's shared words.  CHECK: the chunk reaches
// past the row's causal end.
template <bool CHECK, int SW>
__device__ __forceinline__ void sweep2_chunk(const float* p, int left, float lo_f, float hi_f, int lane,
                                             uint32_t* st_ab, uint32_t* st_cb) {
#pragma unroll
    for (int i0 = 0; i0 < 32; i0 += SW) {
        float x[SW];
#pragma unroll
        for (int u = 0; u < SW; ++u) {
            const int o = (i0 + u) * 32;
            if (CHECK)
                x[u] = o + lane < left ? __ldg(p + o) : __uint_as_float(0xff800000u);
            else
                x[u] = __ldg(p + o);
        }
#pragma unroll
        for (int u = 0; u < SW; ++u) {
            const uint32_t ab = __ballot_sync(0xffffffffu, x[u] >= hi_f);
            const uint32_t ge = __ballot_sync(0xffffffffu, x[u] >= lo_f);
            if (lane == 0) {
                st_ab[i0 + u] = ab;
                st_cb[i0 + u] = ge & ~ab;
            }
        }
    }
}

// slot of a score in the descending first-digit histogram: (~key) >> S, where
// key is the order-preserving key of x (x + 0 turns -0 into +0)
template <int S>
__device__ __forceinline__ uint32_t desc_slot(float x) {
    const uint32_t b = __float_as_uint(x + 0.0f);
    const uint32_t s = (uint32_t)((int32_t)b >> 31);
    return (b ^ (~s & 0x7fffffffu)) >> S;
}

template <int BLOCK, int DBITS, int PIPE, int MINB, int SW2>
__global__ void __launch_bounds__(BLOCK, MINB) topk_sweep_kernel(TopkArgs a, CandLists cl) {
    constexpr int NW = BLOCK / 32;
    constexpr int NB = 1 << DBITS;
    constexpr int S = 32 - DBITS;   // shift of the first digit
    __shared__ __align__(16) uint32_t hist[NB];
    __shared__ uint32_t stage[NW][2][32];
    __shared__ uint32_t wtot[NW];
    __shared__ uint32_t res[5];
    __shared__ uint32_t s_cnt;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    for (int i = tid; i < NB; i += BLOCK) hist[i] = 0;
    __syncthreads();

    for (int64_t row = blockIdx.x; row < a.n_rows; row += gridDim.x) {
        const float* src = a.scores + row * a.row_stride;
        const int valid = (int)row_valid(a, row);
        uint32_t* out = a.bits + row * a.words;
        if (a.k > valid) {
            short_row_block<BLOCK>(a, row, src, valid, wtot);
            if (tid == 0) cl.meta[row] = make_uint4(kRowDone, 0u, 0u, 0u);
            continue;   // block-uniform
        }
        // ---- sweep 1: first-digit histogram
        const int gfull = a.vec_ok ? valid >> 2 : 0;   // whole float4 groups read as vectors
        {
            const float4* p4 = reinterpret_cast<const float4*>(src) + tid;
            int g = tid;
            for (; g + (PIPE - 1) * BLOCK < gfull; g += PIPE * BLOCK, p4 += PIPE * BLOCK) {
                float4 v[PIPE];
#pragma unroll
                for (int u = 0; u < PIPE; ++u) v[u] = __ldg(p4 + u * BLOCK);
#pragma unroll
                for (int u = 0; u < PIPE; ++u) {
                    atomicAdd(&hist[desc_slot<S>(v[u].x)], 1u);
                    atomicAdd(&hist[desc_slot<S>(v[u].y)], 1u);
                    atomicAdd(&hist[desc_slot<S>(v[u].z)], 1u);
                    atomicAdd(&hist[desc_slot<S>(v[u].w)], 1u);
                }
            }
            for (; g < gfull; g += BLOCK, p4 += BLOCK) {
                const float4 v = __ldg(p4);
                atomicAdd(&hist[desc_slot<S>(v.x)], 1u);
                atomicAdd(&hist[desc_slot<S>(v.y)], 1u);
                atomicAdd(&hist[desc_slot<S>(v.z)], 1u);
                atomicAdd(&hist[desc_slot<S>(v.w)], 1u);
            }
            for (int i = 4 * gfull + tid; i < valid; i += BLOCK) atomicAdd(&hist[desc_slot<S>(__ldg(src + i))], 1u);
        }
        __syncthreads();
        // every warp's appends of the previous row precede the barrier above,
        // and this row's follow the one that ends fine_find
        if (tid == 0) s_cnt = 0;
        fine_find<BLOCK, DBITS>(hist, (uint32_t)a.k, wtot, res);
        const uint32_t d0 = res[0], krem = res[1], n0 = res[2];
        const bool plain = (res[3] | res[4]) == 0u;
        if (!plain || n0 > (uint32_t)cl.cap) {   // block-uniform
            exact_row_slow<BLOCK>(src, valid, a.k, a.thr + row, a.cnt ? a.cnt + row : nullptr, nullptr, 0,
                                  out, a.words, hist, wtot, res);
            for (int i = tid; i < 256; i += BLOCK) hist[i] = 0;
            if (tid == 0) cl.meta[row] = make_uint4(kRowDone, 0u, 0u, 0u);
            __syncthreads();
            continue;
        }
        // ---- sweep 2: plain rows have every key in bins 16..NB-17, so both
        // edges of bin d0 are finite (hi may be +inf for the top finite bin);
        // exactly n0 keys lie in bin d0, so the appends fit the list
        const float hi_f = key2f((d0 + 1) << S), lo_f = key2f(d0 << S);
        uint32_t* ckey = cl.key + row * cl.cap;
        uint16_t* cpos = cl.pos + row * cl.cap;
        uint32_t* st_ab = stage[warp][0];
        uint32_t* st_cb = stage[warp][1];
        const int nwords = (int)a.words;
        for (int ch = warp; ch < ((nwords + 31) >> 5); ch += NW) {
            const int s0c = ch * 1024;
            const float* p = src + s0c + lane;
            const int wd = ch * 32 + lane;
            if (s0c >= valid) {   // words past the causal end
                if (wd < nwords) out[wd] = 0u;
                continue;
            }
            if (s0c + 1024 <= valid)
                sweep2_chunk<false, SW2>(p, valid - s0c, lo_f, hi_f, lane, st_ab, st_cb);
            else
                sweep2_chunk<true, SW2>(p, valid - s0c, lo_f, hi_f, lane, st_ab, st_cb);
            __syncwarp();
            if (wd < nwords) out[wd] = st_ab[lane];
            // the chunk's candidates: lane L takes word L's set bits, reserves
            // their slots with one shared add per chunk, and reads their keys
            // back (the chunk was just read, so from L2), four at a time
            uint32_t m = st_cb[lane];
            const uint32_t c = __popc(m);
            uint32_t incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const uint32_t tot = __shfl_sync(0xffffffffu, incl, 31);
            if (tot) {   // warp-uniform
                uint32_t base = 0;
                if (lane == 0) base = atomicAdd(&s_cnt, tot);
                uint32_t at = __shfl_sync(0xffffffffu, base, 0) + incl - c;
                const int pw = s0c + lane * 32;
                while (m) {
                    int ps[4];
                    float v[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        ps[j] = m ? pw + __ffs(m) - 1 : -1;
                        m &= m - 1;
                        v[j] = ps[j] >= 0 ? __ldg(src + ps[j]) : 0.f;
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        if (ps[j] >= 0) {
                            ckey[at] = f2key_raw(v[j]);
                            cpos[at] = (uint16_t)ps[j];
                            ++at;
                        }
                    }
                }
            }
            __syncwarp();
        }
        if (tid == 0) cl.meta[row] = make_uint4(d0, krem, n0, 0u);
    }
}

// One warp per row: the exact krem-th largest key among the row's bin-d0
// candidates (read from the row's list), their bits ORed into the bitmap,
// the threshold and the count.  Per warp in shared memory: cap keys and a
// 256-bin histogram.
template <int DBITS>
__global__ void __launch_bounds__(256, 4) topk_resolve_kernel(TopkArgs a, CandLists cl) {
    constexpr int S = 32 - DBITS;
    extern __shared__ uint4 dyn_r[];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    uint32_t* key = reinterpret_cast<uint32_t*>(dyn_r) + (size_t)wib * (cl.cap + 256);
    uint32_t* hist = key + cl.cap;
    const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + wib; row < a.n_rows; row += nwarps) {
        const uint4 m = cl.meta[row];
        if (m.x == kRowDone) continue;   // warp-uniform
        const uint32_t d0 = m.x;
        uint32_t krem = m.y;
        const uint32_t n = m.z <= (uint32_t)cl.cap ? m.z : (uint32_t)cl.cap;
        const uint32_t above = (uint32_t)a.k - krem;
        const uint32_t* ckey = cl.key + row * cl.cap;
        const uint16_t* cpos = cl.pos + row * cl.cap;
        uint32_t* out = a.bits + row * a.words;
        for (uint32_t i0 = 0; i0 < n; i0 += 256) {
            uint32_t x[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const uint32_t i = i0 + u * 32 + lane;
                x[u] = i < n ? ckey[i] : 0u;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const uint32_t i = i0 + u * 32 + lane;
                if (i < n) key[i] = x[u];
            }
        }
        // radix passes over the remaining S bits: 8, 8, then the rest
        uint32_t prefix = d0 << S, pmask = ~0u << S;
#pragma unroll 1
        for (int left = S; left > 0;) {
            const int nbits = left > 8 ? 8 : left;
            const int shift = left - nbits;
            const uint32_t nb = 1u << nbits;
#pragma unroll
            for (int j = 0; j < 8; ++j) hist[lane + 32 * j] = 0;
            __syncwarp();
            for (uint32_t i = lane; i < n; i += 32) {
                const uint32_t kk = key[i];
                if ((kk & pmask) == prefix) atomicAdd(&hist[(nb - 1) - ((kk >> shift) & (nb - 1))], 1u);
            }
            __syncwarp();
            // lane L scans slots [8L, 8L+8) (descending digits)
            uint32_t h[8], local = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                h[j] = hist[8 * lane + j];
                local += h[j];
            }
            uint32_t inc = local;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += y;
            }
            const uint32_t excl = inc - local;
            uint32_t dsel = 0, rsel = 0;
            const bool mine = excl < krem && krem <= inc;
            if (mine) {
                uint32_t cc = excl;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (rsel == 0 && krem <= cc + h[j]) {
                        dsel = (nb - 1) - (uint32_t)(8 * lane + j);
                        rsel = krem - cc;
                    }
                    cc += h[j];
                }
            }
            const int src_lane = __ffs(__ballot_sync(0xffffffffu, mine)) - 1;
            dsel = __shfl_sync(0xffffffffu, dsel, src_lane);
            rsel = __shfl_sync(0xffffffffu, rsel, src_lane);
            prefix |= dsel << shift;
            pmask |= (nb - 1) << shift;
            krem = rsel;
            left -= nbits;
            __syncwarp();
        }
        // kept candidates: their bits, and the count
        uint32_t kc = 0;
        for (uint32_t i = lane; i < n; i += 32) {
            if (key[i] >= prefix) {
                const uint32_t ps = cpos[i];
                atomicOr(out + (ps >> 5), 1u << (ps & 31));
                ++kc;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) kc += __shfl_xor_sync(0xffffffffu, kc, o);
        if (lane == 0) {
            a.thr[row] = key2f(prefix);
            if (a.cnt) a.cnt[row] = (int32_t)(above + kc);
        }
        __syncwarp();
    }
}


template <int DB>
int launch_sweep_resolve_t(const TopkArgs& a, void* ws, cudaStream_t stream) {
    const CandLists cl = cand_lists(ws, a.n_rows, a.words);
    {
        // 6 CTAs of 256 threads per SM (40 registers).  Measured on B200 at c5:
        // 512- or 1024-thread CTAs, 128-thread CTAs, more loads in flight in
        // sweep 2, chunks in reverse order, words kept in registers instead
        // of shared memory, and rows taken in a short/long interleaved order
        // (less L2 missing in sweep 2, but slower) were all slower or equal.
        auto kern = topk_sweep_kernel<256, DB, 4, 6, 4>;
        const int block = 256;
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, block, 0) != cudaSuccess || per_sm < 1)
            per_sm = 1;
        int64_t grid = (int64_t)num_sms() * per_sm;
        if (grid > a.n_rows) grid = a.n_rows;
        kern<<<(unsigned)grid, block, 0, stream>>>(a, cl);
        if (int rc = check_launch("topk_sweep_kernel")) return rc;
    }
    {
        auto kern = topk_resolve_kernel<DB>;
        const size_t smem = 8 * ((size_t)cl.cap + 256) * sizeof(uint32_t);
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return fail(DSA_ERR_CUDA, "topk_resolve: cannot set dynamic shared memory size");
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, smem) != cudaSuccess || per_sm < 1)
            per_sm = 1;
        int64_t grid = (int64_t)num_sms() * per_sm;
        const int64_t need = (a.n_rows + 7) / 8;
        if (grid > need) grid = need;
        kern<<<(unsigned)grid, 256, smem, stream>>>(a, cl);
        return check_launch("topk_resolve_kernel");
    }
}

// First-digit width by row length.  Rows of up to 8K entries (c4) take 11 bits:
// a 2048-bin histogram halves the per-row scan between the sweeps, which
// shorter rows pay on fewer bytes (c4 top-K 0.413 -> 0.357 ms); longer rows
// (c5) take 12, since 11 doubles their threshold bin's candidates and long
// rows of the indexer's scores then overflow the list (c5 1.05 -> 1.28 ms).
// 10 bits measured slower at c4 (0.425 ms).  DSA_TOPK_SWEEP_DBITS=11|12 forces one.
int launch_sweep_resolve(const TopkArgs& a, void* ws, cudaStream_t stream) {
    static const int forced = [] { const char* e = getenv("DSA_TOPK_SWEEP_DBITS"); return e ? atoi(e) : 0; }();
    const int db = forced ? forced : (a.words * 32 <= 8192 ? 11 : 12);
    return db == 11 ? launch_sweep_resolve_t<11>(a, ws, stream) : launch_sweep_resolve_t<12>(a, ws, stream);
}

// ===========================================================================
// Short rows (<= 512 entries: configs c1 and c3): one warp
// per row, the row's keys in registers (NG float4 groups per lane), no block
// barriers.  Four 8-bit radix passes over the register-resident keys use a
// 256-bin histogram per warp (descending slots, scanned by the warp);
// after the first pass only keys matching the selected prefix touch it.
// Emission orders the kept positions with ballots.
// ===========================================================================

// NB1: bins of the first pass (256 -> 8+8+8+8 bits; 2048 -> 11+8+8+5 bits).
template <int NG, int NB1>
__global__ void __launch_bounds__(256) topk_warp_kernel(TopkArgs a) {
    extern __shared__ uint4 wdyn[];  // 8 warps x NB1 bins
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t* hist = reinterpret_cast<uint32_t*>(wdyn) + warp * NB1;
    const uint32_t lt_mask = (1u << lane) - 1u;

    for (int64_t row = (int64_t)blockIdx.x * 8 + warp; row < a.n_rows; row += (int64_t)gridDim.x * 8) {
        const float* src = a.scores + row * a.row_stride;
        const int valid = (int)row_valid(a, row);
        if (a.k > valid) {
            short_row_warp(a, row, src, valid);
            continue;
        }
        // ---- load: group g = lane + 32j holds positions 4g..4g+3; padding keys are 0
        uint32_t key[NG][4];
#pragma unroll
        for (int j = 0; j < NG; ++j) {
            const int g = lane + 32 * j;
            if (a.vec_ok && 4 * g + 3 < valid) {
                const float4 v = __ldg(reinterpret_cast<const float4*>(src) + g);
                key[j][0] = f2key(v.x); key[j][1] = f2key(v.y); key[j][2] = f2key(v.z); key[j][3] = f2key(v.w);
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) key[j][e] = 4 * g + e < valid ? f2key(__ldg(src + 4 * g + e)) : 0u;
            }
        }
        // ---- radix passes, most significant first
        uint32_t prefix = 0, pmask = 0, krem = (uint32_t)a.k;
#pragma unroll 1
        for (int pass = 0; pass < 4; ++pass) {
            const int bits = pass == 0 ? (NB1 == 2048 ? 11 : 8) : (NB1 == 2048 && pass == 3 ? 5 : 8);
            const int shift = NB1 == 2048 ? (pass == 0 ? 21 : pass == 1 ? 13 : pass == 2 ? 5 : 0) : 24 - 8 * pass;
            const int nb = 1 << bits;
            const int nbs = nb < 256 ? 256 : nb;  // slots scanned (unused ones stay 0)
            const int per = nbs / 32;              // slots per lane: 8 or 64
            for (int i = lane * 4; i < nbs; i += 128) *reinterpret_cast<uint4*>(hist + i) = make_uint4(0, 0, 0, 0);
            __syncwarp();
#pragma unroll
            for (int j = 0; j < NG; ++j)
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    if (4 * (lane + 32 * j) + e < valid && (key[j][e] & pmask) == prefix)
                        atomicAdd(&hist[(nbs - 1) - ((key[j][e] >> shift) & (uint32_t)(nb - 1))], 1u);
            __syncwarp();
            // lane owns slots [per*lane, per*lane+per) (descending digits)
            uint32_t local = 0;
            for (int i = 0; i < per; i += 4) {
                const uint4 h = *reinterpret_cast<const uint4*>(hist + lane * per + i);
                local += h.x + h.y + h.z + h.w;
            }
            uint32_t incl = local;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const uint32_t excl = incl - local;
            const bool mine = excl < krem && krem <= incl;
            uint32_t dig = 0, kr = 0;
            if (mine) {
                uint32_t c = excl;
                for (int i = 0; i < per; ++i) {
                    const uint32_t h = hist[lane * per + i];
                    if (krem <= c + h) {
                        dig = (uint32_t)(nbs - 1 - (lane * per + i)) + 1u;  // +1: 0 marks "not found"
                        kr = krem - c;
                        break;
                    }
                    c += h;
                }
            }
            const uint32_t who = __ballot_sync(0xffffffffu, mine);
            const int src_lane = who ? __ffs(who) - 1 : 0;
            dig = __shfl_sync(0xffffffffu, dig, src_lane);
            kr = __shfl_sync(0xffffffffu, kr, src_lane);
            prefix |= (dig - 1u) << shift;
            pmask |= (uint32_t)(nb - 1) << shift;
            krem = kr;
            __syncwarp();
        }
        const uint32_t thr_key = prefix;

        // ---- count and ordered emission
        uint32_t base = 0;
        int32_t* out = a.idx ? a.idx + row * a.idx_cap : nullptr;
        const uint32_t cap = (uint32_t)a.idx_cap;
#pragma unroll
        for (int j = 0; j < NG; ++j) {
            const int g = lane + 32 * j;
            bool pk[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) pk[e] = 4 * g + e < valid && kept_key(key[j][e], thr_key);
            const uint32_t m0 = __ballot_sync(0xffffffffu, pk[0]), m1 = __ballot_sync(0xffffffffu, pk[1]),
                           m2 = __ballot_sync(0xffffffffu, pk[2]), m3 = __ballot_sync(0xffffffffu, pk[3]);
            if (out) {
                uint32_t pos = base + __popc(m0 & lt_mask) + __popc(m1 & lt_mask) + __popc(m2 & lt_mask) +
                               __popc(m3 & lt_mask);
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    if (pk[e]) {
                        if (pos < cap) out[pos] = 4 * g + e;
                        ++pos;
                    }
            }
            base += __popc(m0) + __popc(m1) + __popc(m2) + __popc(m3);
        }
        if (lane == 0) {
            a.thr[row] = key2f(thr_key);
            if (a.cnt) a.cnt[row] = (int32_t)base;
        }
    }
}

template <int NG, int NB1>
int launch_warp(const TopkArgs& a, cudaStream_t stream) {
    auto kern = topk_warp_kernel<NG, NB1>;
    const size_t smem = 8 * NB1 * sizeof(uint32_t);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return fail(DSA_ERR_CUDA, "topk_select: cannot set dynamic shared memory size");
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, smem) != cudaSuccess || per_sm < 1)
        per_sm = 1;
    int64_t grid = (int64_t)num_sms() * per_sm;
    const int64_t need = (a.n_rows + 7) / 8;
    if (grid > need) grid = need;
    kern<<<(unsigned)grid, 256, smem, stream>>>(a);
    return check_launch("topk_warp_kernel");
}

// ===========================================================================
// Rows of 513..4096 entries: one warp per row, no copy of the row on chip.
// Every pass re-reads the row (the first read comes from HBM, the rest from
// L2) so a warp needs only a 512-bin histogram (2 KB); with no block
// barriers, dozens of rows are in flight per SM, which hides each row's
// serial chain of sweeps.
//   passes   9 + 8 + 8 + 7 bits, most significant first; after the first,
//            only keys matching the selected prefix touch the histogram
//   emission one more sweep orders the kept positions with ballots
// ===========================================================================
constexpr int WL2_BINS = 512;

// Keys of group g: canonical (f2key) or raw (f2key_raw, equal on rows without NaN)
template <bool CANON>
__device__ __forceinline__ uint4 row_keys4(const float* src, int g, int valid, int vec_ok) {
    auto key = [](float x) { return CANON ? f2key(x) : f2key_raw(x); };
    if (vec_ok && 4 * g + 3 < valid) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(src) + g);
        return make_uint4(key(v.x), key(v.y), key(v.z), key(v.w));
    }
    uint32_t e[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) e[j] = 4 * g + j < valid ? key(__ldg(src + 4 * g + j)) : 0u;
    return make_uint4(e[0], e[1], e[2], e[3]);
}

// One row exactly, by one warp, for rows holding NaN: four 8-bit radix passes
// over the canonical keys (every NaN one key above +inf) re-reading the row,
// then the count and the ascending list.  hist: the warp's >= 256 slots.
// Kept out of line so the hot kernel's register allocation does not carry it.
__device__ __noinline__ void warp_exact_row_slow(const float* src, int valid, int k, float* thr_out,
                                                 int32_t* cnt_out, int32_t* idx_out, int64_t idx_cap,
                                                 uint32_t* hist) {
    const int lane = threadIdx.x & 31;
    uint32_t prefix = 0, pmask = 0, krem = (uint32_t)k;
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        for (int i = lane; i < 256; i += 32) hist[i] = 0;
        __syncwarp();
        for (int i = lane; i < valid; i += 32) {
            const uint32_t key = f2key(__ldg(src + i));
            if ((key & pmask) == prefix) atomicAdd(&hist[255 - ((key >> shift) & 255u)], 1u);
        }
        __syncwarp();
        // lane owns slots 8*lane .. 8*lane+7 (descending digits)
        uint32_t local = 0;
        for (int q = 0; q < 8; ++q) local += hist[lane * 8 + q];
        uint32_t incl = local;
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        const uint32_t excl = incl - local;
        const bool mine = excl < krem && krem <= incl;
        uint32_t dig = 0, kr = 0;
        if (mine) {
            uint32_t c = excl;
            for (int q = 0; q < 8; ++q) {
                const uint32_t h = hist[lane * 8 + q];
                if (krem <= c + h) {
                    dig = (uint32_t)(255 - (lane * 8 + q));
                    kr = krem - c;
                    break;
                }
                c += h;
            }
        }
        const uint32_t who = __ballot_sync(0xffffffffu, mine);
        const int srcl = who ? __ffs(who) - 1 : 0;
        prefix |= __shfl_sync(0xffffffffu, dig, srcl) << shift;
        pmask |= 255u << shift;
        krem = __shfl_sync(0xffffffffu, kr, srcl);
        __syncwarp();
    }
    uint32_t n = 0;
    for (int i0 = 0; i0 < valid; i0 += 32) {
        const int i = i0 + lane;
        const bool p = i < valid && kept_key(f2key(__ldg(src + i)), prefix);
        const uint32_t m = __ballot_sync(0xffffffffu, p);
        const uint32_t pos = n + __popc(m & ((1u << lane) - 1u));
        if (idx_out && p && pos < idx_cap) idx_out[pos] = i;
        n += __popc(m);
    }
    if (lane == 0) {
        *thr_out = key2f(prefix);
        if (cnt_out) *cnt_out = (int32_t)n;
    }
}

__global__ void __launch_bounds__(256, 5) topk_warp_l2_kernel(TopkArgs a) {
    extern __shared__ uint4 wl2_dyn[];  // 8 warps x WL2_BINS
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t* hist = reinterpret_cast<uint32_t*>(wl2_dyn) + warp * WL2_BINS;
    const uint32_t lt_mask = (1u << lane) - 1u;

    for (int64_t row = (int64_t)blockIdx.x * 8 + warp; row < a.n_rows; row += (int64_t)gridDim.x * 8) {
        const float* src = a.scores + row * a.row_stride;
        const int valid = (int)row_valid(a, row);
        if (a.k > valid) {
            short_row_warp(a, row, src, valid);
            continue;
        }
        const int g4 = (valid + 3) >> 2;
        uint32_t prefix = 0, pmask = 0, krem = (uint32_t)a.k, bin_n = 0;
        bool slow = false;
#pragma unroll 1
        for (int pass = 0; pass < 4; ++pass) {
            const int bits = pass == 0 ? 9 : pass == 3 ? 7 : 8;
            const int shift = pass == 0 ? 23 : pass == 1 ? 15 : pass == 2 ? 7 : 0;
            const uint32_t nb = 1u << bits;
            // clear this warp's slots
#pragma unroll
            for (int q = 0; q < WL2_BINS / 128; ++q) reinterpret_cast<uint4*>(hist)[lane + 32 * q] = make_uint4(0, 0, 0, 0);
            __syncwarp();
            // slot = WL2_BINS - 1 - digit (descending digits).  The first pass
            // uses canonical keys (every NaN in digit 511, beside +inf), the
            // later ones raw keys: they are equal on rows without NaN, and a
            // row with anything in digit 511 takes the exact slow path.
            auto accumulate = [&](auto canon_tag) {
                constexpr bool CANON = decltype(canon_tag)::value;
                for (int g0 = lane; g0 < g4; g0 += 32 * 4) {
                    uint4 kk[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int g = g0 + 32 * u;
                        kk[u] = g < g4 ? row_keys4<CANON>(src, g, valid, a.vec_ok) : make_uint4(0, 0, 0, 0);
                    }
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int g = g0 + 32 * u;
                        const uint32_t e[4] = {kk[u].x, kk[u].y, kk[u].z, kk[u].w};
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            if (4 * g + j < valid && (e[j] & pmask) == prefix)
                                atomicAdd(&hist[(WL2_BINS - 1) - ((e[j] >> shift) & (nb - 1))], 1u);
                    }
                }
            };
            if (pass == 0) accumulate(std::true_type{});
            else accumulate(std::false_type{});
            __syncwarp();
            if (pass == 0 && hist[0]) {   // +inf or NaN in the row (rare)
                slow = true;
                break;
            }
            // warp scan: lane owns slots [SPL*lane, SPL*lane+SPL)
            constexpr int SPL = WL2_BINS / 32;
            uint32_t local = 0;
#pragma unroll
            for (int q = 0; q < SPL / 4; ++q) {
                const uint4 h = reinterpret_cast<const uint4*>(hist)[lane * (SPL / 4) + q];
                local += h.x + h.y + h.z + h.w;
            }
            uint32_t incl = local;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const uint32_t excl = incl - local;
            const bool mine = excl < krem && krem <= incl;
            uint32_t dig = 0, kr = 0, bn = 0;
            if (mine) {
                uint32_t c = excl;
                for (int q = 0; q < SPL; ++q) {
                    const uint32_t h = hist[lane * SPL + q];
                    if (krem <= c + h) {
                        dig = (uint32_t)(WL2_BINS - (lane * SPL + q));  // digit + 1
                        kr = krem - c;
                        bn = h;
                        break;
                    }
                    c += h;
                }
            }
            const uint32_t who = __ballot_sync(0xffffffffu, mine);
            const int srcl = who ? __ffs(who) - 1 : 0;
            dig = __shfl_sync(0xffffffffu, dig, srcl);
            kr = __shfl_sync(0xffffffffu, kr, srcl);
            bin_n = __shfl_sync(0xffffffffu, bn, srcl);
            prefix |= (dig - 1u) << shift;
            pmask |= (nb - 1) << shift;
            krem = kr;
            __syncwarp();
        }
        if (slow) {
            warp_exact_row_slow(src, valid, a.k, a.thr + row, a.cnt ? a.cnt + row : nullptr,
                                a.idx ? a.idx + row * a.idx_cap : nullptr, a.idx_cap, hist);
            continue;
        }
        const uint32_t thr_key = prefix;
        // kept = keys above the k-th (k - krem of them) + keys equal to it (the final bin)
        const uint32_t total = (uint32_t)a.k - krem + bin_n;
        if (lane == 0) {
            a.thr[row] = key2f(thr_key);
            if (a.cnt) a.cnt[row] = (int32_t)total;
        }
        if (a.idx) {
            int32_t* out = a.idx + row * a.idx_cap;
            const uint32_t cap = (uint32_t)a.idx_cap;
            uint32_t base = 0;
            for (int gb = 0; gb < g4 && base < cap; gb += 32) {
                const int g = gb + lane;
                const uint4 kk = g < g4 ? row_keys4<false>(src, g, valid, a.vec_ok) : make_uint4(0, 0, 0, 0);
                const bool p0 = 4 * g < valid && kept_key(kk.x, thr_key),
                           p1 = 4 * g + 1 < valid && kept_key(kk.y, thr_key),
                           p2 = 4 * g + 2 < valid && kept_key(kk.z, thr_key),
                           p3 = 4 * g + 3 < valid && kept_key(kk.w, thr_key);
                const uint32_t m0 = __ballot_sync(0xffffffffu, p0), m1 = __ballot_sync(0xffffffffu, p1),
                               m2 = __ballot_sync(0xffffffffu, p2), m3 = __ballot_sync(0xffffffffu, p3);
                uint32_t pos = base + __popc(m0 & lt_mask) + __popc(m1 & lt_mask) + __popc(m2 & lt_mask) +
                               __popc(m3 & lt_mask);
                if (p0) { if (pos < cap) out[pos] = 4 * g; ++pos; }
                if (p1) { if (pos < cap) out[pos] = 4 * g + 1; ++pos; }
                if (p2) { if (pos < cap) out[pos] = 4 * g + 2; ++pos; }
                if (p3) { if (pos < cap) out[pos] = 4 * g + 3; ++pos; }
                base += __popc(m0) + __popc(m1) + __popc(m2) + __popc(m3);
            }
        }
    }
}

int launch_warp_l2(const TopkArgs& a, cudaStream_t stream) {
    const size_t smem = 8 * WL2_BINS * sizeof(uint32_t);
    if (cudaFuncSetAttribute(topk_warp_l2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
        return fail(DSA_ERR_CUDA, "topk_select: cannot set dynamic shared memory size");
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, topk_warp_l2_kernel, 256, smem) != cudaSuccess ||
        per_sm < 1)
        per_sm = 1;
    int64_t grid = (int64_t)num_sms() * per_sm;
    const int64_t need = (a.n_rows + 7) / 8;
    if (grid > need) grid = need;
    topk_warp_l2_kernel<<<(unsigned)grid, 256, smem, stream>>>(a);
    return check_launch("topk_warp_l2_kernel");
}

}  // namespace

// Workspace of the two-kernel bitmap path (candidate words, one meta word per row).
size_t topk_sweep_ws_bytes(int64_t n_rows, int64_t words) { return sweep_ws_bytes(n_rows, words); }

int kept_bitmap(const float* scores, const float* thr, uint32_t* bits, int64_t B, int64_t T_q,
                int64_t T_k, int64_t q_row0, int64_t words, int64_t row_bstep, cudaStream_t stream);
int64_t bitmap_words(int64_t T_k);

static int topk_launch(TopkArgs& a, int64_t longest, cudaStream_t stream);

int topk_select(const float* scores, int64_t n_rows, int64_t row_len, int64_t row_stride,
                int64_t rows_per_batch, int64_t q_row0, int causal, int64_t k, float* thr,
                int32_t* idx, int32_t* cnt, int64_t idx_cap, uint32_t* bits, int64_t words,
                int64_t row_bstep, cudaStream_t stream, void* ws, size_t ws_bytes) {
    if (n_rows < 0 || row_len < 1 || row_stride < row_len)
        return fail(DSA_ERR_INVALID, "topk_select: need n_rows >= 0, row_len >= 1, row_stride >= row_len");
    if (k < 1 || k > row_len)
        return fail(DSA_ERR_INVALID, "topk_select: need 1 <= k <= row_len (k=" + std::to_string(k) +
                                         ", row_len=" + std::to_string(row_len) + ")");
    if (row_len > INT32_MAX || k > INT32_MAX) return fail(DSA_ERR_INVALID, "topk_select: row too long");
    if (causal && rows_per_batch < 1) return fail(DSA_ERR_INVALID, "topk_select: rows_per_batch < 1");
    if (q_row0 < 0) return fail(DSA_ERR_INVALID, "topk_select: q_row0 < 0");
    if (causal && n_rows % rows_per_batch && row_bstep)
        return fail(DSA_ERR_INVALID, "topk_select: row_bstep needs n_rows a multiple of rows_per_batch");
    if (causal && q_row0 + (n_rows / rows_per_batch) * (row_bstep < 0 ? row_bstep : 0) < 0)
        return fail(DSA_ERR_INVALID, "topk_select: a row block starts before position 0");
    if (!scores || !thr) return fail(DSA_ERR_INVALID, "topk_select: scores and thr_out are required");
    if (idx && idx_cap < 1) return fail(DSA_ERR_INVALID, "topk_select: idx_cap < 1 with idx_out");
    if (bits && (words < bitmap_words(row_len) || (words & 3) || row_stride != row_len))
        return fail(DSA_ERR_INVALID, "topk_select: the bitmap needs words_per_row a multiple of 4, >= "
                                     "dsa_bitmap_words(row_len), and row_stride == row_len");
    if (n_rows == 0) return DSA_OK;

    TopkArgs a;
    a.scores = scores;
    a.n_rows = n_rows;
    a.row_len = row_len;
    a.row_stride = row_stride;
    a.rows_per_batch = causal ? rows_per_batch : 1;
    a.q_row0 = q_row0;
    a.row_bstep = causal ? row_bstep : 0;
    a.causal = causal ? 1 : 0;
    a.k = (int)k;
    a.thr = thr;
    a.idx = idx;
    a.cnt = cnt;
    a.idx_cap = idx ? idx_cap : 0;
    a.bits = nullptr;
    a.cand_words = 0;
    a.words = words;
    a.vec_ok = (aligned16(scores) && row_stride % 4 == 0) ? 1 : 0;
    // longest row any CTA will see
    int64_t longest = row_len;
    if (causal) {
        const int64_t nbat = (n_rows + rows_per_batch - 1) / rows_per_batch;
        const int64_t step = row_bstep > 0 ? row_bstep : 0;
        const int64_t tmax = q_row0 + (nbat - 1) * step + (n_rows < rows_per_batch ? n_rows : rows_per_batch) - 1;
        longest = tmax + 1 < row_len ? tmax + 1 : row_len;
    }
    constexpr int64_t kCacheMax = 12288;  // 48 KB of keys per CTA
    a.cache_elems = (int)(longest < kCacheMax ? longest : kCacheMax);
    // the CTA-per-row kernel writes the bitmap in its last sweep; rows the
    // other kernels take get it from kept_bitmap_kernel afterwards
    const bool cta_kernel = longest > 4096 && longest <= kRowCache && !getenv("DSA_TOPK_LONG_PATH");
    if (bits && cta_kernel) a.bits = bits;
    // bitmap-only rows with a workspace: the sweep kernel and the per-row resolver
    if (a.bits && !idx && longest > 4096 && ws && ws_bytes >= sweep_ws_bytes(n_rows, words) &&
        !getenv("DSA_TOPK_ONE_KERNEL"))
        return launch_sweep_resolve(a, ws, stream);
    int rc = topk_launch(a, longest, stream);
    if (rc || !bits || cta_kernel) return rc;
    // causal rows: key s kept only if s <= q_row0 + r % rows_per_batch;
    // otherwise a q_row0 past the row end makes every position causal
    return kept_bitmap(scores, thr, bits, n_rows / a.rows_per_batch, a.rows_per_batch, row_len,
                       causal ? q_row0 : row_len, words, a.row_bstep, stream);
}

static int topk_launch(TopkArgs& a, int64_t longest, cudaStream_t stream) {
    // rows <= 512: one warp per row (measured 2.6-2.9x faster than a CTA per
    // row there; slower than it on 1K-2K rows, where the CTA kernel is kept)
    if (longest <= 512 && !getenv("DSA_TOPK_LONG_PATH") && !getenv("DSA_TOPK_NO_WARP")) {
        if (longest <= 128) return launch_warp<1, 256>(a, stream);
        if (longest <= 256) return launch_warp<2, 256>(a, stream);
        return launch_warp<4, 256>(a, stream);
    }
    // rows of 513..4096: one warp per row re-reading the row from L2 (measured
    // faster than a CTA per row there; slower on the long rows of c4/c5)
    if (longest <= 4096 && !getenv("DSA_TOPK_LONG_PATH") && !getenv("DSA_TOPK_NO_WL2"))
        return launch_warp_l2(a, stream);
    if (longest <= kRowCache && !getenv("DSA_TOPK_LONG_PATH")) {
        // bitmap-only rows (the forward's): the fine-digit two-sweep kernel
        if (longest <= 2048) return launch_cached<128, true>(a, longest, stream);
        // bitmap-only rows of 4K-8K: 128-thread CTAs re-reading the row from L2,
        // with a candidate buffer of longest/8 keys, instead of 256 threads
        // caching the keys; far more rows are in flight (c4 top-K 0.61 -> 0.47 ms)
        if (longest <= 8192 && !(a.bits && !a.idx)) return launch_cached<256, true>(a, longest, stream);
        if (longest <= 8192) return launch_cached<128, false>(a, longest, stream, 8);
        // longer rows: the sweeps after the first re-read the row from L2, so
        // several CTAs fit on an SM (DSA_TOPK_SMEM_ROWS=1 caches them instead)
        if (getenv("DSA_TOPK_SMEM_ROWS")) return launch_cached<512, true>(a, longest, stream);
        return launch_cached<256, false>(a, longest, stream);
    }
    if (longest <= 4096) return launch_topk<256>(a, stream);
    if (longest <= 16384) return launch_topk<512>(a, stream);
    return launch_topk<1024>(a, stream);
}

DSA_DEBUG_FLAGS_READER(topk)

}  // namespace dsa
