// Stage 3: sparse attention over the kept keys, gather + online softmax.
//
// Replaces _sparse_attn_kernel / sparse_attention_with_threshold_triton
// (dsa_attention.py:234-324), which loads all T key/value rows per query and
// masks, with a kernel that touches only the kept rows: O(k) bytes per query
// instead of O(T).
//
// One CTA per query row.  A "team" of L = HQ * D / VEC threads covers one
// key row (all heads) with one 16-byte load per thread, so every gathered K
// or V row is read as fully coalesced 16-byte vectors; G = D / VEC lanes of a
// team hold one head and reduce its dot product with xor-shuffles.  The CTA
// holds BLOCK / L teams which walk the key list with a stride, each keeping
// its own running max / sum / accumulator (online softmax over blocks of U
// keys, exp2 domain), merged through shared memory at the end.
//
// The key list comes either from dsa_topk_select's index list (list form) or
// from scanning the score row against the threshold (threshold form, and the
// fallback for a row whose kept count overflowed the list capacity).  Both
// visit kept keys in ascending position order.
#include <math.h>

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
};

constexpr float kNegInf = -INFINITY;

template <typename T, int G, int BLOCK, int U>
__global__ void __launch_bounds__(BLOCK) sparse_attn_kernel(AttnArgs<T> a) {
    constexpr int VEC = 16 / sizeof(T);
    constexpr int NW = BLOCK / 32;
    constexpr int LIST = BLOCK;  // keys staged per refill
    __shared__ int32_t keys_s[LIST];
    __shared__ uint32_t warp_tot[NW];
    __shared__ int s_n;
    __shared__ float m_s[BLOCK], l_s[BLOCK];        // per (team, head) — at most BLOCK entries
    __shared__ float acc_s[BLOCK * VEC];             // per (team, lane) partial outputs

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int L = a.HQ * G;          // threads per key row
    const int P = BLOCK / L;         // teams
    const int team = tid / L;
    const int lt = tid - team * L;   // lane within team: head h = lt / G
    const bool active = team < P;    // threads beyond P*L idle in the math

    const int64_t row = blockIdx.x;
    const int64_t b = row / a.T_q;
    const int64_t t = a.q_row0 + (row - b * a.T_q);
    const int64_t valid = t + 1 < a.T_k ? t + 1 : a.T_k;
    const int64_t rowlen = (int64_t)a.HQ * a.D;  // elements per K/V row
    const T* Kb = a.K + b * a.T_k * rowlen + (int64_t)lt * VEC;
    const T* Vb = a.V + b * a.T_k * rowlen + (int64_t)lt * VEC;

    float q[VEC], acc[VEC];
    {
        const uint4 qv = active ? ldg16(a.Q + row * rowlen + (int64_t)lt * VEC) : make_uint4(0, 0, 0, 0);
        unpack16<T>(qv, q);
#pragma unroll
        for (int v = 0; v < VEC; ++v) {
            q[v] *= a.scale_log2;
            acc[v] = 0.f;
        }
    }
    float m = kNegInf, l = 0.f;

    // list form unless the row's kept count overflowed the list
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
            for (int i = tid; i < n; i += BLOCK) keys_s[i] = __ldg(a.idx + row * a.idx_cap + c0 + i);
            __syncthreads();
        } else {
            // ordered compaction of positions c0 + tid with score >= thr
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

        // every thread runs the same trip count so shuffles stay warp-uniform
        for (int base = 0; base < n; base += P * U) {
            uint4 kr[U], vr[U];
            bool ok[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int j = base + team + u * P;
                ok[u] = active && j < n;
                const int64_t s = ok[u] ? keys_s[j] : 0;
                if (ok[u]) {
                    kr[u] = ldg16(Kb + s * rowlen);
                    vr[u] = ldg16(Vb + s * rowlen);
                } else {
                    kr[u] = make_uint4(0, 0, 0, 0);
                    vr[u] = make_uint4(0, 0, 0, 0);
                }
            }
            float x[U];
            float mx = m;
#pragma unroll
            for (int u = 0; u < U; ++u) {
                float kf[VEC];
                unpack16<T>(kr[u], kf);
                float d = 0.f;
#pragma unroll
                for (int v = 0; v < VEC; ++v) d = fmaf(q[v], kf[v], d);
#pragma unroll
                for (int o = G / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
                x[u] = ok[u] ? d : kNegInf;
                mx = fmaxf(mx, x[u]);
            }
            if (mx != kNegInf) {
                const float corr = exp2f(m - mx);
                l *= corr;
#pragma unroll
                for (int v = 0; v < VEC; ++v) acc[v] *= corr;
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const float p = exp2f(x[u] - mx);  // 0 for skipped slots
                    l += p;
                    float vf[VEC];
                    unpack16<T>(vr[u], vf);
#pragma unroll
                    for (int v = 0; v < VEC; ++v) acc[v] = fmaf(p, vf[v], acc[v]);
                }
                m = mx;
            }
        }
        __syncthreads();  // keys_s is refilled by the next chunk
    }

    // merge the teams and write O[row] (fp32, [HQ, DV])
    float* orow = a.O + row * rowlen + (int64_t)lt * VEC;
    if (P == 1) {
        if (active) {
            const float inv = 1.f / l;
#pragma unroll
            for (int v = 0; v < VEC; v += 4)
                *reinterpret_cast<float4*>(orow + v) =
                    make_float4(acc[v] * inv, acc[v + 1] * inv, acc[v + 2] * inv, acc[v + 3] * inv);
        }
        return;
    }
    if (active) {
        if (lt % G == 0) {
            m_s[team * a.HQ + lt / G] = m;
            l_s[team * a.HQ + lt / G] = l;
        }
#pragma unroll
        for (int v = 0; v < VEC; ++v) acc_s[(team * L + lt) * VEC + v] = acc[v];
    }
    __syncthreads();
    if (team == 0) {
        const int h = lt / G;
        float mstar = kNegInf;
        for (int p = 0; p < P; ++p) mstar = fmaxf(mstar, m_s[p * a.HQ + h]);
        float lsum = 0.f, o[VEC];
#pragma unroll
        for (int v = 0; v < VEC; ++v) o[v] = 0.f;
        for (int p = 0; p < P; ++p) {
            const float mp = m_s[p * a.HQ + h];
            const float f = mp == kNegInf ? 0.f : exp2f(mp - mstar);
            lsum += l_s[p * a.HQ + h] * f;
#pragma unroll
            for (int v = 0; v < VEC; ++v) o[v] = fmaf(acc_s[(p * L + lt) * VEC + v], f, o[v]);
        }
        const float inv = 1.f / lsum;
#pragma unroll
        for (int v = 0; v < VEC; v += 4)
            *reinterpret_cast<float4*>(orow + v) =
                make_float4(o[v] * inv, o[v + 1] * inv, o[v + 2] * inv, o[v + 3] * inv);
    }
}

template <typename T, int G>
int launch_g(const AttnArgs<T>& a, cudaStream_t stream) {
    const int L = a.HQ * G;
    const int64_t rows = a.B * a.T_q;
    if (rows > INT32_MAX) return fail(DSA_ERR_INVALID, "sparse_attn: too many query rows");
    if (L <= 256) {
        sparse_attn_kernel<T, G, 256, 4><<<(unsigned)rows, 256, 0, stream>>>(a);
    } else if (L <= 512) {
        sparse_attn_kernel<T, G, 512, 4><<<(unsigned)rows, 512, 0, stream>>>(a);
    } else if (L <= 1024) {
        sparse_attn_kernel<T, G, 1024, 2><<<(unsigned)rows, 1024, 0, stream>>>(a);
    } else {
        return fail(DSA_ERR_UNSUPPORTED, "sparse_attn: HQ*D too large for one CTA per key row");
    }
    return check_launch("sparse_attn_kernel");
}

template <typename T>
int launch_t(AttnArgs<T> a, cudaStream_t stream) {
    constexpr int VEC = 16 / sizeof(T);
    if (a.D % VEC != 0)
        return fail(DSA_ERR_UNSUPPORTED, "sparse_attn: head dim must be a multiple of " +
                                             std::to_string(VEC) + " for this dtype");
    const int G = a.D / VEC;
    switch (G) {
        case 1: return launch_g<T, 1>(a, stream);
        case 2: return launch_g<T, 2>(a, stream);
        case 4: return launch_g<T, 4>(a, stream);
        case 8: return launch_g<T, 8>(a, stream);
        case 16: return launch_g<T, 16>(a, stream);
        case 32: return launch_g<T, 32>(a, stream);
        default:
            return fail(DSA_ERR_UNSUPPORTED,
                        "sparse_attn: head dim / (16 bytes / element) must be a power of two <= 32");
    }
}

}  // namespace

int sparse_attn(const int32_t* idx, const int32_t* cnt, int64_t idx_cap, const float* scores,
                const float* thr, const void* Q, const void* K, const void* V, float* O, int64_t B,
                int64_t T_q, int64_t T_k, int64_t q_row0, int64_t HQ, int64_t DQ, int64_t DV,
                float scale, int dtype, cudaStream_t stream) {
    if (B < 0 || T_q < 0 || T_k < 1 || q_row0 < 0 || HQ < 1 || DQ < 1 || DV < 1)
        return fail(DSA_ERR_INVALID, "sparse_attn: bad sizes");
    if (!dtype_ok(dtype)) return fail(DSA_ERR_INVALID, "sparse_attn: unknown dtype");
    if (DQ != DV)
        return fail(DSA_ERR_UNSUPPORTED, "sparse_attn: DQ != DV is not supported by this build");
    if (!Q || !K || !V || !O) return fail(DSA_ERR_INVALID, "sparse_attn: null Q/K/V/O");
    if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O))
        return fail(DSA_ERR_INVALID, "sparse_attn: Q/K/V/O must be 16-byte aligned");
    if (idx) {
        if (!cnt || idx_cap < 1) return fail(DSA_ERR_INVALID, "sparse_attn: idx needs cnt and idx_cap >= 1");
        const int64_t longest = (q_row0 + T_q) < T_k ? (q_row0 + T_q) : T_k;
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
                   T_q, T_k, q_row0, (int)HQ, (int)DQ, scale_log2};
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

}  // namespace dsa
