// Whole DSA forward in one launch for short sequences (T_k <= 2048, small
// heads; rows of up to 512 keys take fused_short_kernel, the same steps with
// the score keys in registers): the B200 counterpart of the reference's fused Triton kernel
// _dsa_fused_kernel (dsa_attention.py:96-193), which does indexer -> tl.sort
// threshold -> dense masked attention per query.
//
// A CTA takes FS_ROWS consecutive query rows of one batch (one warp each).
//   1. Each warp's q_idx row and w row are staged in shared memory.
//   2. The causal indexer keys k_idx[b, 0..t_max] pass through shared memory
//      in chunks of up to 512 keys as fp32 (row stride DI+1, conflict-free);
//      each warp scores its query against the chunk's causal keys (lane l owns
//      keys c0 + l + 32 i), score = sum_j w_j * ReLU(<q_j, k_s>) in fp32, and
//      keeps the order-preserving keys of its row (up to 2048) in shared memory.
//   3. The k-th largest score is found by four 8-bit radix passes over the
//      row (256-bin histogram per warp), ties kept.
//   4. The kept positions are written to a per-warp 16-bit list in ascending order.
//   5. Attention over the list: the warp's 32/L teams gather K/V rows with
//      16-byte loads, online softmax in the exp2 domain, shuffle merge.
// No score matrix, threshold or index list ever reaches global memory.
// Opt-in (DSA_FUSED_SMALL=1): on B200 the three stage kernels are faster at
// these sizes (c1: 0.117 ms vs 0.14 ms for this kernel).
#include <math.h>

#include "common.cuh"

namespace dsa {
namespace {

constexpr int FS_ROWS = 8;      // query rows (warps) per CTA
constexpr int FS_MAXK = 2048;   // longest causal key range
constexpr int FS_KCMAX = 512;
constexpr int FS_SHORT = 512;   // rows of up to this many keys take fused_short_kernel
constexpr int FS_SNI = FS_SHORT / 32;   // keys staged per chunk (at most)
constexpr int FS_NI = FS_KCMAX / 32;
constexpr float kNegInfF = -INFINITY;
constexpr float kRescaleF = 8.f;

template <typename T>
struct FusedArgs {
    const T* q_idx;
    const T* k_idx;
    const float* w_idx;
    const T* Q;
    const T* K;
    const T* V;
    float* O;
    int64_t T_q, T_k, q_row0;
    int HI, DI, HQ, D, k;
    float scale_log2;
    int kc;   // keys staged per chunk (multiple of 32, <= FS_KCMAX)
    int rs;   // per-warp row stride of the score keys and lists: T_k rounded up to 32
};

__device__ __forceinline__ float2 f2fma(float2 a, float2 b, float2 c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(d)
        : "l"(*reinterpret_cast<unsigned long long*>(&a)),
          "l"(*reinterpret_cast<unsigned long long*>(&b)),
          "l"(*reinterpret_cast<unsigned long long*>(&c)));
    return *reinterpret_cast<float2*>(&d);
}
__device__ __forceinline__ float2 f2mul(float2 a, float2 b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;"
        : "=l"(d)
        : "l"(*reinterpret_cast<unsigned long long*>(&a)),
          "l"(*reinterpret_cast<unsigned long long*>(&b)));
    return *reinterpret_cast<float2*>(&d);
}

// float pair i of a 16-byte chunk of T data
template <typename T> __device__ __forceinline__ float2 pair_of(const uint4& v, int i);
template <> __device__ __forceinline__ float2 pair_of<float>(const uint4& v, int i) {
    return i == 0 ? make_float2(__uint_as_float(v.x), __uint_as_float(v.y))
                  : make_float2(__uint_as_float(v.z), __uint_as_float(v.w));
}
template <> __device__ __forceinline__ float2 pair_of<__nv_bfloat16>(const uint4& v, int i) {
    const uint32_t w = i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <> __device__ __forceinline__ float2 pair_of<__half>(const uint4& v, int i) {
    uint32_t w = i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
    return __half22float2(*reinterpret_cast<__half2*>(&w));
}

template <typename T, int C, int G>
__global__ void __launch_bounds__(32 * FS_ROWS) fused_small_kernel(FusedArgs<T> a) {
    constexpr int VEC = 16 / sizeof(T);
    constexpr int PP = VEC / 2;       // float pairs per 16-byte chunk
    constexpr int NP = C * PP;
    extern __shared__ __align__(16) float fsm[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t b = blockIdx.y;
    const int64_t tq0 = (int64_t)blockIdx.x * FS_ROWS;
    const int64_t tq_end = tq0 + FS_ROWS < a.T_q ? tq0 + FS_ROWS : a.T_q;
    const int64_t tmax = a.q_row0 + tq_end - 1;
    const int nk = (int)(tmax + 1 < a.T_k ? tmax + 1 : a.T_k);
    const int DI = a.DI, HI = a.HI, KS = a.DI + 1, KC = a.kc, RS = a.rs;

    // regions (in floats) start on 16-byte boundaries (the histograms are read as uint4)
    const size_t o_q = ((size_t)KC * KS + 3) & ~size_t(3);
    const size_t o_w = o_q + (((size_t)FS_ROWS * HI * DI + 3) & ~size_t(3));
    const size_t o_s = o_w + (((size_t)FS_ROWS * HI + 3) & ~size_t(3));
    const size_t o_h = o_s + (size_t)FS_ROWS * RS;
    float* ks = fsm;                                    // KC x (DI+1): one chunk of keys
    float* qs = fsm + o_q;                              // FS_ROWS x HI*DI
    float* ws = fsm + o_w;                              // FS_ROWS x HI
    uint32_t* srow = reinterpret_cast<uint32_t*>(fsm + o_s) + warp * RS;   // the row's score keys
    uint32_t* hist = reinterpret_cast<uint32_t*>(fsm + o_h) + warp * 256;
    uint16_t* list = reinterpret_cast<uint16_t*>(fsm + o_h + FS_ROWS * 256) + warp * RS;

    // ---- 1. the warp's q_idx and w rows
    const int64_t tq = tq0 + warp;
    const bool have = tq < a.T_q;
    if (have) {
        const T* qp = a.q_idx + (b * a.T_q + tq) * HI * DI;
        for (int e = lane; e < HI * DI; e += 32) qs[warp * HI * DI + e] = Elem<T>::to_f(qp[e]);
        const float* wp = a.w_idx + (b * a.T_q + tq) * HI;
        for (int e = lane; e < HI; e += 32) ws[warp * HI + e] = wp[e];
    }
    const int64_t t = a.q_row0 + tq;
    const int valid = have ? (int)(t + 1 < a.T_k ? t + 1 : a.T_k) : 0;   // causal keys 0..valid-1
    const float* qw = qs + warp * HI * DI;
    const float* ww = ws + warp * HI;

    // ---- 2. scores, one chunk of KC keys at a time staged in shared memory
    // as fp32 (row stride DI+1, conflict-free): lane l scores keys
    // c0 + l + 32 i; each dot sums d = 0..DI-1 in order and the heads j in
    // order, as the CUDA-core indexer does, so the scores are the same fp32
    // values.  The keys go to the warp's row in shared memory.
    const T* kb = a.k_idx + b * a.T_k * DI;
    for (int c0 = 0; c0 < nk; c0 += KC) {
        const int nc = nk - c0 < KC ? nk - c0 : KC;
        __syncthreads();   // the previous chunk is scored
        for (int e = threadIdx.x; e < nc * DI; e += 32 * FS_ROWS)
            ks[(e / DI) * KS + e % DI] = Elem<T>::to_f(kb[(int64_t)c0 * DI + e]);
        __syncthreads();
        const int nv = valid - c0 < nc ? valid - c0 : nc;   // this warp's causal keys in the chunk
        if (nv <= 0) continue;
        const int nli = (nv + 31) / 32;
        float sc[FS_NI];
#pragma unroll
        for (int i = 0; i < FS_NI; ++i) sc[i] = 0.f;
        for (int j = 0; j < HI; ++j) {
            const float* qj = qw + j * DI;
            float dot[FS_NI];
#pragma unroll
            for (int i = 0; i < FS_NI; ++i) dot[i] = 0.f;
            for (int d = 0; d < DI; ++d) {
                const float qv = qj[d];
#pragma unroll
                for (int i = 0; i < FS_NI; ++i)
                    if (i < nli) dot[i] = fmaf(qv, ks[(lane + 32 * i) * KS + d], dot[i]);
            }
            const float wj = ww[j];
#pragma unroll
            for (int i = 0; i < FS_NI; ++i) sc[i] = fmaf(wj, fmaxf(dot[i], 0.f), sc[i]);
        }
#pragma unroll
        for (int i = 0; i < FS_NI; ++i)
            if (lane + 32 * i < nv) srow[c0 + lane + 32 * i] = f2key(sc[i]);
    }
    if (!have) return;  // no barriers below
    __syncwarp();
    const int nslot = (valid + 31) / 32;   // 32-key slots of the row
    auto key_at = [&](int s) { return s < valid ? srow[s] : 0u; };

    // ---- 3. k-th largest (k_eff = min(k, T_k) counts the masked -inf entries)
    uint32_t thr_key;
    if (a.k > valid) {
        thr_key = 0u;  // threshold -inf: every causal key but NaN is kept (key 0 < any real key)
    } else {
        uint32_t prefix = 0, pmask = 0, krem = (uint32_t)a.k;
#pragma unroll 1
        for (int pass = 0; pass < 4; ++pass) {
            const int shift = 24 - 8 * pass;
            *reinterpret_cast<uint4*>(hist + lane * 8) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(hist + lane * 8 + 4) = make_uint4(0, 0, 0, 0);
            __syncwarp();
#pragma unroll 4
            for (int i = 0; i < nslot; ++i) {
                const int s = lane + 32 * i;
                const uint32_t kk = key_at(s);
                if (s < valid && (kk & pmask) == prefix) atomicAdd(&hist[255 - ((kk >> shift) & 255u)], 1u);
            }
            __syncwarp();
            const uint4 h0 = *reinterpret_cast<const uint4*>(hist + lane * 8);
            const uint4 h1 = *reinterpret_cast<const uint4*>(hist + lane * 8 + 4);
            const uint32_t hv[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
            uint32_t local = 0;
#pragma unroll
            for (int q = 0; q < 8; ++q) local += hv[q];
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
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    if (dig == 0 && krem <= c + hv[q]) {
                        dig = 256u - (uint32_t)(lane * 8 + q);  // digit + 1
                        kr = krem - c;
                    }
                    c += hv[q];
                }
            }
            const uint32_t who = __ballot_sync(0xffffffffu, mine);
            const int srcl = who ? __ffs(who) - 1 : 0;
            dig = __shfl_sync(0xffffffffu, dig, srcl);
            kr = __shfl_sync(0xffffffffu, kr, srcl);
            prefix |= (dig - 1u) << shift;
            pmask |= 255u << shift;
            krem = kr;
            __syncwarp();
        }
        thr_key = prefix;
    }

    // ---- 4. ascending kept list
    int n = 0;
    const uint32_t lt_mask = (1u << lane) - 1u;
#pragma unroll 4
    for (int i = 0; i < nslot; ++i) {
        const int s = lane + 32 * i;
        const bool p = s < valid && kept_key(key_at(s), thr_key);
        const uint32_t m = __ballot_sync(0xffffffffu, p);
        if (p) list[n + __popc(m & lt_mask)] = (uint16_t)s;
        n += __popc(m);
    }
    __syncwarp();

    // ---- 5. attention over the list (same scheme as the sparse-attention warp kernel)
    const int L = a.HQ * G;
    const int P = 32 / L;
    const int team = lane / L;
    const int lt = lane - team * L;
    const int64_t rowlen = (int64_t)a.HQ * a.D;
    const int64_t toff = (int64_t)(lt / G) * a.D + (lt % G) * VEC;
    const T* Kb = a.K + b * a.T_k * rowlen + toff;
    const T* Vb = a.V + b * a.T_k * rowlen + toff;
    const int64_t orow_i = b * a.T_q + tq;
    float2 q[NP], acc[NP];
    {
        const T* qp = a.Q + orow_i * rowlen + toff;
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const uint4 v = ldg16(qp + c * G * VEC);
#pragma unroll
            for (int i = 0; i < PP; ++i) {
                const float2 f = pair_of<T>(v, i);
                q[c * PP + i] = make_float2(f.x * a.scale_log2, f.y * a.scale_log2);
            }
        }
#pragma unroll
        for (int i = 0; i < NP; ++i) acc[i] = make_float2(0.f, 0.f);
    }
    float m = kNegInfF, l = 0.f;
    for (int base = 0; base < n; base += 2 * P) {
        uint4 kr[2][C], vr[2][C];
        bool ok[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int j = base + team + u * P;
            ok[u] = j < n;
            const int64_t off = (int64_t)(ok[u] ? list[j] : 0) * rowlen;
#pragma unroll
            for (int c = 0; c < C; ++c) {
                kr[u][c] = ok[u] ? ldg16(Kb + off + c * G * VEC) : make_uint4(0, 0, 0, 0);
                vr[u][c] = ok[u] ? ldg16(Vb + off + c * G * VEC) : make_uint4(0, 0, 0, 0);
            }
        }
        float x[2];
        float mx = kNegInfF;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            float2 d2 = make_float2(0.f, 0.f);
#pragma unroll
            for (int c = 0; c < C; ++c)
#pragma unroll
                for (int i = 0; i < PP; ++i) d2 = f2fma(q[c * PP + i], pair_of<T>(kr[u][c], i), d2);
            float d = d2.x + d2.y;
#pragma unroll
            for (int o = G / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
            x[u] = ok[u] ? d : kNegInfF;
            mx = fmaxf(mx, x[u]);
        }
        if (mx > m + kRescaleF) {
            const float corr = exp2f(m - mx);
            const float2 c2 = make_float2(corr, corr);
            l *= corr;
#pragma unroll
            for (int i = 0; i < NP; ++i) acc[i] = f2mul(acc[i], c2);
            m = mx;
        }
        if (m == kNegInfF) continue;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const float p = exp2f(x[u] - m);
            l += p;
            const float2 p2 = make_float2(p, p);
#pragma unroll
            for (int c = 0; c < C; ++c)
#pragma unroll
                for (int i = 0; i < PP; ++i) acc[c * PP + i] = f2fma(p2, pair_of<T>(vr[u][c], i), acc[c * PP + i]);
        }
    }
    for (int off = L; off < 32; off <<= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
        const float l2 = __shfl_xor_sync(0xffffffffu, l, off);
        const float mx = fmaxf(m, m2);
        const float f1 = m == kNegInfF ? 0.f : exp2f(m - mx);
        const float f2 = m2 == kNegInfF ? 0.f : exp2f(m2 - mx);
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
        float* orow = a.O + orow_i * rowlen + toff;
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

// Rows of T_k <= 512: the same steps with each lane's 16 score keys held in
// registers and the whole key range staged at once (faster at these sizes).
template <typename T, int C, int G>
__global__ void __launch_bounds__(32 * FS_ROWS) fused_short_kernel(FusedArgs<T> a) {
    constexpr int VEC = 16 / sizeof(T);
    constexpr int PP = VEC / 2;       // float pairs per 16-byte chunk
    constexpr int NP = C * PP;
    extern __shared__ __align__(16) float fsm[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t b = blockIdx.y;
    const int64_t tq0 = (int64_t)blockIdx.x * FS_ROWS;
    const int64_t tq_end = tq0 + FS_ROWS < a.T_q ? tq0 + FS_ROWS : a.T_q;
    const int64_t tmax = a.q_row0 + tq_end - 1;
    const int nk = (int)(tmax + 1 < a.T_k ? tmax + 1 : a.T_k);
    const int DI = a.DI, HI = a.HI, KS = a.DI + 1;

    // regions start on 16-byte boundaries (the histograms are read as uint4)
    const size_t o_q = ((size_t)a.T_k * KS + 3) & ~size_t(3);
    const size_t o_w = o_q + (((size_t)FS_ROWS * HI * DI + 3) & ~size_t(3));
    const size_t o_h = o_w + (((size_t)FS_ROWS * HI + 3) & ~size_t(3));
    float* ks = fsm;                                    // T_k x (DI+1), rows 0..nk-1 used
    float* qs = fsm + o_q;                              // FS_ROWS x HI*DI
    float* ws = fsm + o_w;                              // FS_ROWS x HI
    uint32_t* hist = reinterpret_cast<uint32_t*>(fsm + o_h) + warp * 256;
    uint16_t* list = reinterpret_cast<uint16_t*>(reinterpret_cast<uint32_t*>(fsm + o_h) + FS_ROWS * 256) + warp * FS_SHORT;

    // ---- 1. stage k_idx, q_idx, w
    const T* kb = a.k_idx + b * a.T_k * DI;
    for (int e = threadIdx.x; e < nk * DI; e += 32 * FS_ROWS) ks[(e / DI) * KS + e % DI] = Elem<T>::to_f(kb[e]);
    const int64_t tq = tq0 + warp;
    const bool have = tq < a.T_q;
    if (have) {
        const T* qp = a.q_idx + (b * a.T_q + tq) * HI * DI;
        for (int e = lane; e < HI * DI; e += 32) qs[warp * HI * DI + e] = Elem<T>::to_f(qp[e]);
        const float* wp = a.w_idx + (b * a.T_q + tq) * HI;
        for (int e = lane; e < HI; e += 32) ws[warp * HI + e] = wp[e];
    }
    __syncthreads();
    if (!have) return;  // no barriers below

    const int64_t t = a.q_row0 + tq;
    const int valid = (int)(t + 1 < a.T_k ? t + 1 : a.T_k);  // causal keys 0..valid-1
    const float* qw = qs + warp * HI * DI;
    const float* ww = ws + warp * HI;

    // ---- 2. scores of the lane's keys: 16 independent accumulation chains per
    // lane (key loop innermost); each dot sums d = 0..DI-1 in order, as the
    // CUDA-core indexer does, so the scores are the same fp32 values.
    float sc[FS_SNI];
#pragma unroll
    for (int i = 0; i < FS_SNI; ++i) sc[i] = 0.f;
    const int nli = (valid + 31) / 32;  // key slots any lane of this warp needs
    for (int j = 0; j < HI; ++j) {
        const float* qj = qw + j * DI;
        float dot[FS_SNI];
#pragma unroll
        for (int i = 0; i < FS_SNI; ++i) dot[i] = 0.f;
        for (int d = 0; d < DI; ++d) {
            const float qv = qj[d];
#pragma unroll
            for (int i = 0; i < FS_SNI; ++i)
                if (i < nli) dot[i] = fmaf(qv, ks[(lane + 32 * i) * KS + d], dot[i]);
        }
        const float wj = ww[j];
#pragma unroll
        for (int i = 0; i < FS_SNI; ++i) sc[i] = fmaf(wj, fmaxf(dot[i], 0.f), sc[i]);
    }
    uint32_t key[FS_SNI];
#pragma unroll
    for (int i = 0; i < FS_SNI; ++i) key[i] = lane + 32 * i < valid ? f2key(sc[i]) : 0u;

    // ---- 3. k-th largest (k_eff = min(k, T_k) counts the masked -inf entries)
    uint32_t thr_key;
    if (a.k > valid) {
        thr_key = 0u;  // threshold -inf: every causal key but NaN is kept (key 0 < any real key)
    } else {
        uint32_t prefix = 0, pmask = 0, krem = (uint32_t)a.k;
#pragma unroll 1
        for (int pass = 0; pass < 4; ++pass) {
            const int shift = 24 - 8 * pass;
            *reinterpret_cast<uint4*>(hist + lane * 8) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(hist + lane * 8 + 4) = make_uint4(0, 0, 0, 0);
            __syncwarp();
#pragma unroll
            for (int i = 0; i < FS_SNI; ++i)
                if (lane + 32 * i < valid && (key[i] & pmask) == prefix)
                    atomicAdd(&hist[255 - ((key[i] >> shift) & 255u)], 1u);
            __syncwarp();
            const uint4 h0 = *reinterpret_cast<const uint4*>(hist + lane * 8);
            const uint4 h1 = *reinterpret_cast<const uint4*>(hist + lane * 8 + 4);
            const uint32_t hv[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
            uint32_t local = 0;
#pragma unroll
            for (int q = 0; q < 8; ++q) local += hv[q];
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
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    if (dig == 0 && krem <= c + hv[q]) {
                        dig = 256u - (uint32_t)(lane * 8 + q);  // digit + 1
                        kr = krem - c;
                    }
                    c += hv[q];
                }
            }
            const uint32_t who = __ballot_sync(0xffffffffu, mine);
            const int srcl = who ? __ffs(who) - 1 : 0;
            dig = __shfl_sync(0xffffffffu, dig, srcl);
            kr = __shfl_sync(0xffffffffu, kr, srcl);
            prefix |= (dig - 1u) << shift;
            pmask |= 255u << shift;
            krem = kr;
            __syncwarp();
        }
        thr_key = prefix;
    }

    // ---- 4. ascending kept list
    int n = 0;
    const uint32_t lt_mask = (1u << lane) - 1u;
#pragma unroll
    for (int i = 0; i < FS_SNI; ++i) {
        const bool p = lane + 32 * i < valid && kept_key(key[i], thr_key);
        const uint32_t m = __ballot_sync(0xffffffffu, p);
        if (p) list[n + __popc(m & lt_mask)] = (uint16_t)(lane + 32 * i);
        n += __popc(m);
    }
    __syncwarp();

    // ---- 5. attention over the list (same scheme as the sparse-attention warp kernel)
    const int L = a.HQ * G;
    const int P = 32 / L;
    const int team = lane / L;
    const int lt = lane - team * L;
    const int64_t rowlen = (int64_t)a.HQ * a.D;
    const int64_t toff = (int64_t)(lt / G) * a.D + (lt % G) * VEC;
    const T* Kb = a.K + b * a.T_k * rowlen + toff;
    const T* Vb = a.V + b * a.T_k * rowlen + toff;
    const int64_t orow_i = b * a.T_q + tq;
    float2 q[NP], acc[NP];
    {
        const T* qp = a.Q + orow_i * rowlen + toff;
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const uint4 v = ldg16(qp + c * G * VEC);
#pragma unroll
            for (int i = 0; i < PP; ++i) {
                const float2 f = pair_of<T>(v, i);
                q[c * PP + i] = make_float2(f.x * a.scale_log2, f.y * a.scale_log2);
            }
        }
#pragma unroll
        for (int i = 0; i < NP; ++i) acc[i] = make_float2(0.f, 0.f);
    }
    float m = kNegInfF, l = 0.f;
    for (int base = 0; base < n; base += 2 * P) {
        uint4 kr[2][C], vr[2][C];
        bool ok[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int j = base + team + u * P;
            ok[u] = j < n;
            const int64_t off = (int64_t)(ok[u] ? list[j] : 0) * rowlen;
#pragma unroll
            for (int c = 0; c < C; ++c) {
                kr[u][c] = ok[u] ? ldg16(Kb + off + c * G * VEC) : make_uint4(0, 0, 0, 0);
                vr[u][c] = ok[u] ? ldg16(Vb + off + c * G * VEC) : make_uint4(0, 0, 0, 0);
            }
        }
        float x[2];
        float mx = kNegInfF;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            float2 d2 = make_float2(0.f, 0.f);
#pragma unroll
            for (int c = 0; c < C; ++c)
#pragma unroll
                for (int i = 0; i < PP; ++i) d2 = f2fma(q[c * PP + i], pair_of<T>(kr[u][c], i), d2);
            float d = d2.x + d2.y;
#pragma unroll
            for (int o = G / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
            x[u] = ok[u] ? d : kNegInfF;
            mx = fmaxf(mx, x[u]);
        }
        if (mx > m + kRescaleF) {
            const float corr = exp2f(m - mx);
            const float2 c2 = make_float2(corr, corr);
            l *= corr;
#pragma unroll
            for (int i = 0; i < NP; ++i) acc[i] = f2mul(acc[i], c2);
            m = mx;
        }
        if (m == kNegInfF) continue;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const float p = exp2f(x[u] - m);
            l += p;
            const float2 p2 = make_float2(p, p);
#pragma unroll
            for (int c = 0; c < C; ++c)
#pragma unroll
                for (int i = 0; i < PP; ++i) acc[c * PP + i] = f2fma(p2, pair_of<T>(vr[u][c], i), acc[c * PP + i]);
        }
    }
    for (int off = L; off < 32; off <<= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
        const float l2 = __shfl_xor_sync(0xffffffffu, l, off);
        const float mx = fmaxf(m, m2);
        const float f1 = m == kNegInfF ? 0.f : exp2f(m - mx);
        const float f2 = m2 == kNegInfF ? 0.f : exp2f(m2 - mx);
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
        float* orow = a.O + orow_i * rowlen + toff;
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
int launch_fs(FusedArgs<T> a, int64_t B, cudaStream_t stream) {
    if (a.T_k <= FS_SHORT) {   // all causal keys at once; score keys in registers
        const size_t smem = (((size_t)a.T_k * (a.DI + 1) + 3) / 4 * 4 + ((size_t)FS_ROWS * a.HI * a.DI + 3) / 4 * 4 +
                             ((size_t)FS_ROWS * a.HI + 3) / 4 * 4 + (size_t)FS_ROWS * 256) * 4 +
                            (size_t)FS_ROWS * FS_SHORT * 2;
        if (smem > 220 * 1024) return -100;
        auto kern = fused_short_kernel<T, C, G>;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return fail(DSA_ERR_CUDA, "fused_small: cannot set dynamic shared memory size");
        dim3 grid((unsigned)((a.T_q + FS_ROWS - 1) / FS_ROWS), (unsigned)B);
        kern<<<grid, 32 * FS_ROWS, smem, stream>>>(a);
        return check_launch("fused_short_kernel");
    }
    // shared memory: a key chunk, q/w rows, the rows' score keys, histograms, kept lists
    auto bytes = [&](int kc) {
        return (((size_t)kc * (a.DI + 1) + 3) / 4 * 4 + ((size_t)FS_ROWS * a.HI * a.DI + 3) / 4 * 4 +
                ((size_t)FS_ROWS * a.HI + 3) / 4 * 4 + (size_t)FS_ROWS * a.rs + (size_t)FS_ROWS * 256) * 4 +
               (size_t)FS_ROWS * a.rs * 2;
    };
    a.rs = (int)((a.T_k + 31) / 32 * 32);
    int kc = a.rs < FS_KCMAX ? a.rs : FS_KCMAX;
    while (kc > 32 && bytes(kc) > 220 * 1024) kc -= 32;
    if (bytes(kc) > 220 * 1024) return -100;
    a.kc = kc;
    const size_t smem = bytes(kc);
    auto kern = fused_small_kernel<T, C, G>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return fail(DSA_ERR_CUDA, "fused_small: cannot set dynamic shared memory size");
    dim3 grid((unsigned)((a.T_q + FS_ROWS - 1) / FS_ROWS), (unsigned)B);
    kern<<<grid, 32 * FS_ROWS, smem, stream>>>(a);
    return check_launch("fused_small_kernel");
}

template <typename T>
int dispatch_fs(const FusedArgs<T>& a, int64_t B, cudaStream_t stream) {
    constexpr int VEC = 16 / sizeof(T);
    const int chunks = a.D / VEC;
    // same lane mapping as the sparse-attention kernels: C chunks per thread, G lanes per head
    switch (chunks) {
        case 1: return a.HQ * 1 <= 32 ? launch_fs<T, 1, 1>(a, B, stream) : -100;
        case 2: return a.HQ * 1 <= 32 ? launch_fs<T, 2, 1>(a, B, stream) : -100;
        case 4: return a.HQ * 2 <= 32 ? launch_fs<T, 2, 2>(a, B, stream) : -100;
        case 8: return a.HQ * 4 <= 32 ? launch_fs<T, 2, 4>(a, B, stream) : -100;
        case 16: return a.HQ * 8 <= 32 ? launch_fs<T, 2, 8>(a, B, stream) : -100;
        default: return -100;
    }
}

}  // namespace

// Returns -100 when the shape is outside this kernel's limits (the caller then
// runs the three-stage pipeline).
int fused_small_forward(const void* q_idx, const void* k_idx, const float* w_idx, const void* Q,
                        const void* K, const void* V, float* O, int64_t B, int64_t T_q, int64_t T_k,
                        int64_t q_row0, int64_t HI, int64_t DI, int64_t HQ, int64_t DQ, int64_t DV,
                        int64_t k, int idx_dtype, int qkv_dtype, cudaStream_t stream) {
    if (idx_dtype != qkv_dtype || T_k > FS_MAXK || DQ != DV || HI * DI > 1024 || DI > 128 ||
        B > 65535 || T_q > 65535 * (int64_t)FS_ROWS)
        return -100;
    const int64_t hq = HQ;
    if ((hq & (hq - 1)) != 0) return -100;  // teams must tile the warp
    if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O)) return -100;
    const float scale_log2 = 1.4426950408889634f / sqrtf((float)DQ);
#define DSA_FS(TT)                                                                                   \
    {                                                                                                \
        FusedArgs<TT> a{(const TT*)q_idx, (const TT*)k_idx, w_idx, (const TT*)Q, (const TT*)K,       \
                        (const TT*)V, O, T_q, T_k, q_row0, (int)HI, (int)DI, (int)HQ, (int)DQ,       \
                        (int)k, scale_log2};                                                         \
        if (DQ % (16 / sizeof(TT)) != 0) return -100;                                               \
        return dispatch_fs<TT>(a, B, stream);                                                       \
    }
    if (idx_dtype == DSA_F32) DSA_FS(float)
    if (idx_dtype == DSA_BF16) DSA_FS(__nv_bfloat16)
    DSA_FS(__half)
#undef DSA_FS
}

DSA_DEBUG_FLAGS_READER(fused_small)

}  // namespace dsa
