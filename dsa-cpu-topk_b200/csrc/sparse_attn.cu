// Stage 3: sparse attention over the kept keys, gather + online softmax.
//
// Replaces _sparse_attn_kernel / sparse_attention_with_threshold_triton
// (dsa_attention.py:234-324), which loads all T key/value rows per query and
// masks, with a kernel that touches only the kept rows: O(k) bytes per query
// instead of O(T).
//
// One CTA per query row.  A "team" of L threads covers one key row (all
// heads): each thread owns up to two 16-byte chunks of one head (interleaved with
// the head's other lanes, so every load instruction is contiguous per head),
// and the G lanes that share a head reduce its dot product with log2(G)
// xor-shuffles.  Products and the p*V accumulation use packed fp32x2 FMAs.
// The CTA's BLOCK / L teams walk the key list with a stride, each keeping
// its own running max / sum / accumulator (online softmax over blocks of U
// keys in the exp2 domain, rescaled only when the max grows by more than
// 2^8), and merge through shared memory at the end.
//
// The key list comes either from dsa_topk_select's index list (list form) or
// from scanning the score row against the threshold (threshold form, and the
// fallback for a row whose kept count overflowed the list capacity).  Both
// visit kept keys in ascending position order.
#include <math.h>
#include <stdlib.h>

#include "common.cuh"

namespace dsa {
namespace {

template <typename T>
struct AttnArgs {
    const int32_t* idx;
    const int32_t* cnt;
    int64_t idx_cap;
    const float* scores;
    const float* thr;
    const T* Q;
    const T* K;
    const T* V;
    float* O;
    int64_t B, T_q, T_k, q_row0;
    int HQ, D;
    float scale_log2;  // logit scale * log2(e)
    // element strides (batch, row, head) of Q, K, V; batch b's rows start at
    // q_row0 + b*row_bstep.  O is contiguous [B, T_q, HQ, D].
    int64_t Qs[3], Ks[3], Vs[3];
    int64_t row_bstep;
};

constexpr float kNegInf = -INFINITY;
// Rescale the running output only when a new logit exceeds the running max by
// more than this many log2 units; until then exp2(x - m) <= 2^8 stays exact
// enough in fp32 and the final division by l cancels the stale max.
constexpr float kRescale = 8.f;

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(d)
        : "l"(*reinterpret_cast<unsigned long long*>(&a)),
          "l"(*reinterpret_cast<unsigned long long*>(&b)),
          "l"(*reinterpret_cast<unsigned long long*>(&c)));
    return *reinterpret_cast<float2*>(&d);
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;"
        : "=l"(d)
        : "l"(*reinterpret_cast<unsigned long long*>(&a)),
          "l"(*reinterpret_cast<unsigned long long*>(&b)));
    return *reinterpret_cast<float2*>(&d);
}

// one 32-bit word of T data -> the float pair it holds
template <typename T> __device__ __forceinline__ float2 word2(uint32_t w);
template <> __device__ __forceinline__ float2 word2<__nv_bfloat16>(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <> __device__ __forceinline__ float2 word2<__half>(uint32_t w) {
    return __half22float2(*reinterpret_cast<__half2*>(&w));
}
// fp32 data: two words make one pair
template <typename T> struct Pairs {  // 16-bit types: 4 words -> 4 pairs per 16 bytes
    static constexpr int PER16 = 4;
    static __device__ __forceinline__ float2 get(const uint4& v, int i) {
        const uint32_t w = i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
        return word2<T>(w);
    }
};
template <> struct Pairs<float> {
    static constexpr int PER16 = 2;
    static __device__ __forceinline__ float2 get(const uint4& v, int i) {
        return i == 0 ? make_float2(__uint_as_float(v.x), __uint_as_float(v.y))
                      : make_float2(__uint_as_float(v.z), __uint_as_float(v.w));
    }
};

// One CTA per query row.  A team of L = HQ*G threads covers a key row; each
// thread owns C contiguous 16-byte chunks (E elements) of one head, so the
// G lanes of a head reduce with log2(G) shuffles.  The P = BLOCK/L teams
// stride over the key list and merge at the end.
template <typename T, int C, int G, int BLOCK, int U, int MINB>
__global__ void __launch_bounds__(BLOCK, MINB) sparse_attn_kernel(AttnArgs<T> a) {
    constexpr int VEC = 16 / sizeof(T);
    constexpr int E = C * VEC;          // elements per thread
    constexpr int NP = E / 2;           // float pairs per thread
    constexpr int PP = Pairs<T>::PER16; // pairs per 16-byte chunk
    constexpr int NW = BLOCK / 32;
    constexpr int LIST = BLOCK;
    __shared__ int32_t keys_s[LIST];
    __shared__ uint32_t warp_tot[NW];
    __shared__ int s_n;
    extern __shared__ float merge_s[];  // [P*HQ] m, [P*HQ] l, [P*L*E] acc

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int L = a.HQ * G;
    const int P = BLOCK / L;
    const int team = tid / L;
    const int lt = tid - team * L;
    const bool active = team < P;

    const int64_t row = blockIdx.x;
    const int64_t b = row / a.T_q;
    const int64_t tq = row - b * a.T_q;
    const int64_t t = a.q_row0 + b * a.row_bstep + tq;
    const int64_t valid = t + 1 < a.T_k ? t + 1 : a.T_k;
    const int64_t rowlen = (int64_t)a.HQ * a.D;
    // lane g of head h owns chunks g, g+G, ..., g+(C-1)G of the head, so each
    // chunk-load instruction reads a contiguous span per head
    const int64_t hd = lt / G, lo = (lt % G) * VEC;
    const int64_t toff = hd * a.D + lo;   // in O
    const T* Kb = a.K + b * a.Ks[0] + hd * a.Ks[2] + lo;
    const T* Vb = a.V + b * a.Vs[0] + hd * a.Vs[2] + lo;
    const int64_t kr = a.Ks[1], vr = a.Vs[1];

    float2 q[NP], acc[NP];
    {
        const T* qp = a.Q + b * a.Qs[0] + tq * a.Qs[1] + hd * a.Qs[2] + lo;
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const uint4 v = active ? ldg16(qp + c * G * VEC) : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int i = 0; i < PP; ++i) {
                const float2 f = Pairs<T>::get(v, i);
                q[c * PP + i] = make_float2(f.x * a.scale_log2, f.y * a.scale_log2);
            }
        }
#pragma unroll
        for (int i = 0; i < NP; ++i) acc[i] = make_float2(0.f, 0.f);
    }
    float m = kNegInf, l = 0.f;

    int64_t n_total;
    bool list_mode = false;
    if (a.idx) {
        const int64_t c = a.cnt[row];
        if (c <= a.idx_cap) {
            list_mode = true;
            n_total = c;
        }
    }
    if (!list_mode) n_total = valid;
    const float thr = list_mode ? 0.f : a.thr[row];
    const float* srow = list_mode ? nullptr : a.scores + row * a.T_k;

    for (int64_t c0 = 0; c0 < n_total; c0 += LIST) {
        int n;
        if (list_mode) {
            n = (int)(n_total - c0 < LIST ? n_total - c0 : LIST);
            for (int i = tid; i < n; i += BLOCK) {
                const int32_t key = __ldg(a.idx + row * a.idx_cap + c0 + i);
                keys_s[i] = DSA_CHECK(key >= 0 && key < valid, DBG_LIST_KEY) ? key : -1;
            }
            __syncthreads();
        } else {
            const int64_t s = c0 + tid;
            const bool p = s < n_total && __ldg(srow + s) >= thr;
            const uint32_t bal = __ballot_sync(0xffffffffu, p);
            if (lane == 0) warp_tot[warp] = __popc(bal);
            __syncthreads();
            uint32_t base = 0, tot = 0;
            for (int w2 = 0; w2 < NW; ++w2) {
                const uint32_t x = warp_tot[w2];
                base += w2 < warp ? x : 0u;
                tot += x;
            }
            if (p) keys_s[base + __popc(bal & ((1u << lane) - 1u))] = (int32_t)s;
            if (tid == 0) s_n = (int)tot;
            __syncthreads();
            n = s_n;
        }

        for (int base = 0; base < n; base += P * U) {
            uint4 kreg[U][C], vreg[U][C];
            bool ok[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int j = base + team + u * P;
                ok[u] = active && j < n;
#ifdef DSA_DEBUG_CHECKS
                ok[u] = ok[u] && keys_s[j] >= 0;   // an entry the check dropped
#endif
                const int64_t key = ok[u] ? (int64_t)keys_s[j] : 0;
#pragma unroll
                for (int c = 0; c < C; ++c) {
                    kreg[u][c] = ok[u] ? ldg16(Kb + key * kr + c * G * VEC) : make_uint4(0, 0, 0, 0);
                    vreg[u][c] = ok[u] ? ldg16(Vb + key * vr + c * G * VEC) : make_uint4(0, 0, 0, 0);
                }
            }
            float x[U];
            float mx = kNegInf;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                float2 d2 = make_float2(0.f, 0.f);
#pragma unroll
                for (int c = 0; c < C; ++c)
#pragma unroll
                    for (int i = 0; i < PP; ++i) d2 = ffma2(q[c * PP + i], Pairs<T>::get(kreg[u][c], i), d2);
                float d = d2.x + d2.y;
#pragma unroll
                for (int o = G / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
                x[u] = ok[u] ? d : kNegInf;
                mx = fmaxf(mx, x[u]);
            }
            if (mx > m + kRescale) {  // also true on the first key (m = -inf)
                const float corr = exp2f(m - mx);
                const float2 c2 = make_float2(corr, corr);
                l *= corr;
#pragma unroll
                for (int i = 0; i < NP; ++i) acc[i] = fmul2(acc[i], c2);
                m = mx;
            }
            if (m == kNegInf) continue;  // no key of this team in the block yet
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const float p = exp2f(x[u] - m);  // 0 for skipped slots
                l += p;
                const float2 p2 = make_float2(p, p);
#pragma unroll
                for (int c = 0; c < C; ++c)
#pragma unroll
                    for (int i = 0; i < PP; ++i)
                        acc[c * PP + i] = ffma2(p2, Pairs<T>::get(vreg[u][c], i), acc[c * PP + i]);
            }
        }
        __syncthreads();
    }

    float* orow = a.O + row * rowlen + toff;
    if (P == 1) {
        if (active) {
            const float inv = 1.f / l;
#pragma unroll
            for (int c = 0; c < C; ++c)
#pragma unroll
                for (int i = 0; i < PP; i += 2) {
                    const float2 x0 = acc[c * PP + i], x1 = acc[c * PP + i + 1];
                    *reinterpret_cast<float4*>(orow + c * G * VEC + 2 * i) =
                        make_float4(x0.x * inv, x0.y * inv, x1.x * inv, x1.y * inv);
                }
        }
        return;
    }
    float* m_s = merge_s;
    float* l_s = m_s + P * a.HQ;
    float* acc_s = l_s + P * a.HQ;
    if (active) {
        if (lt % G == 0) {
            m_s[team * a.HQ + lt / G] = m;
            l_s[team * a.HQ + lt / G] = l;
        }
        // partial outputs in row layout: acc_s[team][element of the row]
#pragma unroll
        for (int c = 0; c < C; ++c)
#pragma unroll
            for (int i = 0; i < PP; ++i)
                *reinterpret_cast<float2*>(&acc_s[team * rowlen + toff + c * G * VEC + 2 * i]) =
                    acc[c * PP + i];
    }
    __syncthreads();
    // all threads share the output: element e of the row (e = lt*E + ...)
    for (int e = tid; e < L * E; e += BLOCK) {
        const int h = e / a.D;
        float mstar = kNegInf;
        for (int p = 0; p < P; ++p) mstar = fmaxf(mstar, m_s[p * a.HQ + h]);
        float lsum = 0.f, o = 0.f;
        for (int p = 0; p < P; ++p) {
            const float mp = m_s[p * a.HQ + h];
            const float f = mp == kNegInf ? 0.f : exp2f(mp - mstar);
            lsum += l_s[p * a.HQ + h] * f;
            o = fmaf(acc_s[p * rowlen + e], f, o);
        }
        a.O[row * rowlen + e] = o / lsum;
    }
}

// ---------------------------------------------------------------------------
// Small heads (a team of L = HQ*G <= 32 threads, L a power of two: configs
// c1-c3): one warp per query row, eight rows per CTA, no block barriers.  The
// warp's 32/L teams split the key list and merge with xor-shuffles.  Key
// indices arrive 32 at a time (one per lane) and are handed out by shuffle.
// ---------------------------------------------------------------------------
template <typename T, int C, int G, int U>
__global__ void __launch_bounds__(256) sparse_attn_warp_kernel(AttnArgs<T> a) {
    constexpr int VEC = 16 / sizeof(T);
    constexpr int NP = C * VEC / 2;
    constexpr int PP = Pairs<T>::PER16;
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (row >= a.B * a.T_q) return;  // warp-uniform
    const int L = a.HQ * G;
    const int P = 32 / L;
    const int team = lane / L;
    const int lt = lane - team * L;
    const int64_t b = row / a.T_q;
    const int64_t tq = row - b * a.T_q;
    const int64_t t = a.q_row0 + b * a.row_bstep + tq;
    const int64_t valid = t + 1 < a.T_k ? t + 1 : a.T_k;
    const int64_t rowlen = (int64_t)a.HQ * a.D;
    const int64_t hd = lt / G, lo = (lt % G) * VEC;
    const int64_t toff = hd * a.D + lo;   // in O
    const T* Kb = a.K + b * a.Ks[0] + hd * a.Ks[2] + lo;
    const T* Vb = a.V + b * a.Vs[0] + hd * a.Vs[2] + lo;
    const int64_t kr = a.Ks[1], vr = a.Vs[1];

    float2 q[NP], acc[NP];
    {
        const T* qp = a.Q + b * a.Qs[0] + tq * a.Qs[1] + hd * a.Qs[2] + lo;
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const uint4 v = ldg16(qp + c * G * VEC);
#pragma unroll
            for (int i = 0; i < PP; ++i) {
                const float2 f = Pairs<T>::get(v, i);
                q[c * PP + i] = make_float2(f.x * a.scale_log2, f.y * a.scale_log2);
            }
        }
#pragma unroll
        for (int i = 0; i < NP; ++i) acc[i] = make_float2(0.f, 0.f);
    }
    float m = kNegInf, l = 0.f;

    bool list_mode = false;
    int64_t n_total = valid;
    if (a.idx) {
        const int64_t c = a.cnt[row];
        if (c <= a.idx_cap) {
            list_mode = true;
            n_total = c;
        }
    }
    const float thr = list_mode ? 0.f : a.thr[row];
    const float* srow = list_mode ? nullptr : a.scores + row * a.T_k;

    for (int64_t c0 = 0; c0 < n_total; c0 += 32) {
        // this chunk's keys: lane r holds the r-th one
        int mykey = 0, n;
        if (list_mode) {
            n = (int)(n_total - c0 < 32 ? n_total - c0 : 32);
            if (lane < n) mykey = __ldg(a.idx + row * a.idx_cap + c0 + lane);
            if (lane < n && !DSA_CHECK(mykey >= 0 && mykey < valid, DBG_LIST_KEY)) mykey = -1;
        } else {
            const int64_t s = c0 + lane;
            const uint32_t bal = __ballot_sync(0xffffffffu, s < n_total && __ldg(srow + s) >= thr);
            n = __popc(bal);
            if (lane < n) mykey = (int)c0 + (int)__fns(bal, 0, lane + 1);
        }
        for (int base = 0; base < n; base += P * U) {
            uint4 kreg[U][C], vreg[U][C];
            bool ok[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int j = base + team + u * P;
                ok[u] = j < n;
                const int s = __shfl_sync(0xffffffffu, mykey, j & 31);
#ifdef DSA_DEBUG_CHECKS
                ok[u] = ok[u] && s >= 0;   // an entry the check dropped
#endif
                const int64_t key = ok[u] ? s : 0;
#pragma unroll
                for (int c = 0; c < C; ++c) {
                    kreg[u][c] = ok[u] ? ldg16(Kb + key * kr + c * G * VEC) : make_uint4(0, 0, 0, 0);
                    vreg[u][c] = ok[u] ? ldg16(Vb + key * vr + c * G * VEC) : make_uint4(0, 0, 0, 0);
                }
            }
            float x[U];
            float mx = kNegInf;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                float2 d2 = make_float2(0.f, 0.f);
#pragma unroll
                for (int c = 0; c < C; ++c)
#pragma unroll
                    for (int i = 0; i < PP; ++i) d2 = ffma2(q[c * PP + i], Pairs<T>::get(kreg[u][c], i), d2);
                float d = d2.x + d2.y;
#pragma unroll
                for (int o = G / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
                x[u] = ok[u] ? d : kNegInf;
                mx = fmaxf(mx, x[u]);
            }
            if (mx > m + kRescale) {
                const float corr = exp2f(m - mx);
                const float2 c2 = make_float2(corr, corr);
                l *= corr;
#pragma unroll
                for (int i = 0; i < NP; ++i) acc[i] = fmul2(acc[i], c2);
                m = mx;
            }
            if (m == kNegInf) continue;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const float p = exp2f(x[u] - m);
                l += p;
                const float2 p2 = make_float2(p, p);
#pragma unroll
                for (int c = 0; c < C; ++c)
#pragma unroll
                    for (int i = 0; i < PP; ++i)
                        acc[c * PP + i] = ffma2(p2, Pairs<T>::get(vreg[u][c], i), acc[c * PP + i]);
            }
        }
    }
    // merge the warp's teams
    for (int off = L; off < 32; off <<= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
        const float l2 = __shfl_xor_sync(0xffffffffu, l, off);
        const float mx = fmaxf(m, m2);
        const float f1 = m == kNegInf ? 0.f : exp2f(m - mx);
        const float f2 = m2 == kNegInf ? 0.f : exp2f(m2 - mx);
#pragma unroll
        for (int i = 0; i < NP; ++i) {
            const float ax = __shfl_xor_sync(0xffffffffu, acc[i].x, off);
            const float ay = __shfl_xor_sync(0xffffffffu, acc[i].y, off);
            acc[i] = make_float2(acc[i].x * f1 + ax * f2, acc[i].y * f1 + ay * f2);
        }
        l = l * f1 + l2 * f2;
        m = mx;
    }
    if (team == 0) {
        float* orow = a.O + row * rowlen + toff;
        const float inv = 1.f / l;
#pragma unroll
        for (int c = 0; c < C; ++c)
#pragma unroll
            for (int i = 0; i < PP; i += 2) {
                const float2 x0 = acc[c * PP + i], x1 = acc[c * PP + i + 1];
                *reinterpret_cast<float4*>(orow + c * G * VEC + 2 * i) =
                    make_float4(x0.x * inv, x0.y * inv, x1.x * inv, x1.y * inv);
            }
    }
}

template <typename T, int C, int G>
int launch_g(const AttnArgs<T>& a, cudaStream_t stream) {
    constexpr int VEC = 16 / sizeof(T);
    constexpr int E = C * VEC;
    const int L = a.HQ * G;
    const int64_t rows = a.B * a.T_q;
    if (rows > INT32_MAX) return fail(DSA_ERR_INVALID, "sparse_attn: too many query rows");
    int block;
    if (L <= 256) block = 256;
    else if (L <= 512) block = 512;
    else if (L <= 1024) block = 1024;
    else return fail(DSA_ERR_UNSUPPORTED, "sparse_attn: HQ*D too large for one CTA per key row");
    if (L <= 32 && (L & (L - 1)) == 0 && !getenv("DSA_ATTN_NO_WARP")) {
        sparse_attn_warp_kernel<T, C, G, 2><<<(unsigned)((rows + 7) / 8), 256, 0, stream>>>(a);
        return check_launch("sparse_attn_warp_kernel");
    }
    const int P = block / L;
    const size_t smem = P == 1 ? 0 : (size_t)(2 * P * a.HQ + P * L * E) * sizeof(float);
#define DSA_LAUNCH(BLK, UU, MB)                                                                   \
    {                                                                                                 \
        auto kern = sparse_attn_kernel<T, C, G, BLK, UU, MB>;                                     \
        if (smem > 48 * 1024 &&                                                                       \
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=     \
                cudaSuccess)                                                                          \
            return fail(DSA_ERR_CUDA, "sparse_attn: cannot set dynamic shared memory size");        \
        kern<<<(unsigned)rows, BLK, smem, stream>>>(a);                                               \
    }
    // 256 threads: two keys in flight per team, 4 CTAs per SM (80 -> 64
    // registers) measured best on B200 among U in {1, 2, 4} and 3 or 4 CTAs/SM
    if (block == 256) DSA_LAUNCH(256, 2, 4)
    else if (block == 512) DSA_LAUNCH(512, 2, 1)
    else DSA_LAUNCH(1024, 1, 1)
#undef DSA_LAUNCH
    return check_launch("sparse_attn_kernel");
}

template <typename T>
int launch_t(AttnArgs<T> a, cudaStream_t stream) {
    constexpr int VEC = 16 / sizeof(T);
    if (a.D % VEC != 0)
        return fail(DSA_ERR_UNSUPPORTED, "sparse_attn: head dim must be a multiple of " +
                                             std::to_string(VEC) + " for this dtype");
    const int chunks = a.D / VEC;  // 16-byte chunks per head
    switch (chunks) {
        case 1: return launch_g<T, 1, 1>(a, stream);
        case 2: return launch_g<T, 2, 1>(a, stream);
        case 4: return launch_g<T, 2, 2>(a, stream);
        case 8: return launch_g<T, 2, 4>(a, stream);
        case 16: return launch_g<T, 2, 8>(a, stream);
        case 32: return launch_g<T, 2, 16>(a, stream);
        case 64: return launch_g<T, 2, 32>(a, stream);
        default:
            return fail(DSA_ERR_UNSUPPORTED,
                        "sparse_attn: head dim / (16 bytes / element) must be a power of two <= 64");
    }
}

}  // namespace

int sparse_attn(const int32_t* idx, const int32_t* cnt, int64_t idx_cap, const float* scores,
                const float* thr, const void* Q, const void* K, const void* V, float* O, int64_t B,
                int64_t T_q, int64_t T_k, int64_t q_row0, int64_t HQ, int64_t DQ, int64_t DV,
                float scale, int dtype, const dsa_layout& L, cudaStream_t stream) {
    if (B < 0 || T_q < 0 || T_k < 1 || q_row0 < 0 || HQ < 1 || DQ < 1 || DV < 1)
        return fail(DSA_ERR_INVALID, "sparse_attn: bad sizes");
    {
        // every gathered 16-byte chunk must stay aligned
        const int64_t e = (int64_t)dtype_size(dtype);
        for (const int64_t* st : {L.Q, L.K, L.V})
            for (int i = 0; i < 3; ++i)
                if ((st[i] * e) & 15)
                    return fail(DSA_ERR_UNSUPPORTED, "sparse_attn: Q/K/V strides must be multiples of 16 bytes");
    }
    if (!dtype_ok(dtype)) return fail(DSA_ERR_INVALID, "sparse_attn: unknown dtype");
    if (dtype == DSA_FP8_E4M3)
        return fail(DSA_ERR_UNSUPPORTED, "sparse_attn: FP8 is supported for the indexer inputs only");
    if (DQ != DV)
        return fail(DSA_ERR_UNSUPPORTED, "sparse_attn: DQ != DV is not supported by this build");
    if (!Q || !K || !V || !O) return fail(DSA_ERR_INVALID, "sparse_attn: null Q/K/V/O");
    if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O))
        return fail(DSA_ERR_INVALID, "sparse_attn: Q/K/V/O must be 16-byte aligned");
    if (idx) {
        if (!cnt || idx_cap < 1) return fail(DSA_ERR_INVALID, "sparse_attn: idx needs cnt and idx_cap >= 1");
        const int64_t last = q_row0 + (B > 0 ? B - 1 : 0) * (L.row_bstep > 0 ? L.row_bstep : 0) + T_q;
        const int64_t longest = last < T_k ? last : T_k;
        if (idx_cap < longest && (!scores || !thr))
            return fail(DSA_ERR_INVALID,
                        "sparse_attn: idx_cap < longest row, so scores and thr are needed for overflow rows");
    } else if (!scores || !thr) {
        return fail(DSA_ERR_INVALID, "sparse_attn: threshold form needs scores and thr");
    }
    if (B * T_q == 0) return DSA_OK;
    const float scale_log2 = scale * 1.4426950408889634f;
#define DSA_ATTN_ARGS(TT)                                                                         \
    AttnArgs<TT> a{idx, cnt, idx_cap, scores, thr, (const TT*)Q, (const TT*)K, (const TT*)V, O, B, \
                   T_q, T_k, q_row0, (int)HQ, (int)DQ, scale_log2,                               \
                   {L.Q[0], L.Q[1], L.Q[2]}, {L.K[0], L.K[1], L.K[2]}, {L.V[0], L.V[1], L.V[2]},   \
                   L.row_bstep};
    if (dtype == DSA_F32) {
        DSA_ATTN_ARGS(float)
        return launch_t<float>(a, stream);
    } else if (dtype == DSA_BF16) {
        DSA_ATTN_ARGS(__nv_bfloat16)
        return launch_t<__nv_bfloat16>(a, stream);
    } else {
        DSA_ATTN_ARGS(__half)
        return launch_t<__half>(a, stream);
    }
#undef DSA_ATTN_ARGS
}

DSA_DEBUG_FLAGS_READER(sparse_attn)

}  // namespace dsa
