// Stage 1 (CUDA-core path): Lightning Indexer scores in IEEE fp32.
//
//   I[b,t,s] = sum_j w[b,t,j] * ReLU(<q[b,t,j,:], k[b,s,:]>),  -inf for s > t
//
// Same arithmetic as _indexer_score_kernel (lightning_indexer.py:54-97), whose
// tl.dot runs with input_precision="ieee": fp32 products and sums, no TF32.
// This path serves fp32 inputs (configs c1-c3, where a 3xTF32 tensor-core
// split would buy nothing at these sizes) and any bf16/fp16 shape the
// tcgen05 kernel does not take.
//
// A 256-thread CTA owns a 64x64 (query x key) tile; each thread a 4x4
// register block (rows ty+16i, keys tx+16j).  Per head j the q and k slices
// go through shared memory in 32-wide chunks of the head dim (row-major,
// padded so the inner loop's float4 reads are conflict-free); the
// ReLU * w[t,j] epilogue accumulates in registers across heads.  Tiles
// entirely above the causal diagonal do no math (they are filled with -inf
// only when the caller asks for the full matrix).
#include <math.h>
#include <stdlib.h>

#include "common.cuh"

namespace dsa {
namespace {

constexpr int BT = 64, BS = 64, DC = 32;

// element strides of q (batch, row, head), k (batch, row), w (batch, row) and
// the per-batch step of the first query row
struct SimtLayout {
    int64_t qb, qr, qh, kb, kr, wb, wr, row_bstep;
    const float* kscale;   // per-key scales [B or 1, T_k] (batch stride ksb), or null
    int64_t ksb;
};

template <typename T>
__global__ void __launch_bounds__(256) indexer_simt_kernel(const T* __restrict__ q,
                                                          const T* __restrict__ k,
                                                          const float* __restrict__ w,
                                                          float* __restrict__ scores, int64_t T_q,
                                                          int64_t T_k, int64_t q_row0, int HI,
                                                          int DI, int fill_upper, SimtLayout ly) {
    // [row][dim] with a 4-float pad: the float4 reads of 16 consecutive rows
    // (stride 36 words) fall in distinct bank quads.
    __shared__ __align__(16) float qs[BT][DC + 4];
    __shared__ __align__(16) float ks[BS][DC + 4];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int64_t b = blockIdx.z;
    const int64_t tq0 = (int64_t)blockIdx.y * BT;  // first query row (relative)
    const int64_t s0 = (int64_t)blockIdx.x * BS;
    const int64_t tq_end = tq0 + BT < T_q ? tq0 + BT : T_q;
    q_row0 += b * ly.row_bstep;
    const int64_t t_max = q_row0 + tq_end - 1;
    float* srow0 = scores + (b * T_q) * T_k;
    const float NEG = -INFINITY;

    if (s0 > t_max) {  // whole tile above the diagonal
        if (fill_upper) {
            for (int e = tid; e < BT * BS; e += 256) {
                const int64_t tq = tq0 + e / BS, s = s0 + e % BS;
                if (tq < T_q && s < T_k) srow0[tq * T_k + s] = NEG;
            }
        }
        return;
    }

    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) acc[i][jj] = 0.f;

    const T* qb = q + b * ly.qb;
    const T* kb = k + b * ly.kb;
    const float* wrow[4];   // head weights of this thread's four query rows
#pragma unroll
    for (int i = 0; i < 4; ++i) wrow[i] = w + b * ly.wb + (tq0 + ty + 16 * i) * ly.wr;
    for (int j = 0; j < HI; ++j) {
        float dot[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) dot[i][jj] = 0.f;
        for (int dc = 0; dc < DI; dc += DC) {
            // each thread loads 8 q and 8 k elements (row = e / DC, dim = e % DC)
#pragma unroll
            for (int r = 0; r < (BT * DC) / 256; ++r) {
                const int e = tid + r * 256;
                const int rr = e / DC, d = e % DC;
                const int64_t tq = tq0 + rr, s = s0 + rr;
                float qv = 0.f, kv = 0.f;
                if (tq < T_q && dc + d < DI) qv = Elem<T>::to_f(qb[tq * ly.qr + j * ly.qh + dc + d]);
                if (s < T_k && dc + d < DI) kv = Elem<T>::to_f(kb[s * ly.kr + dc + d]);
                qs[rr][d] = qv;
                ks[rr][d] = kv;
            }
            __syncthreads();
#pragma unroll 2
            for (int d = 0; d < DC; d += 4) {
                float4 a4[4], b4[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    a4[i] = *reinterpret_cast<const float4*>(&qs[ty + 16 * i][d]);
                    b4[i] = *reinterpret_cast<const float4*>(&ks[tx + 16 * i][d]);
                }
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) {
                        // same summation order as a plain d = 0..DI-1 loop
                        float x = dot[i][jj];
                        x = fmaf(a4[i].x, b4[jj].x, x);
                        x = fmaf(a4[i].y, b4[jj].y, x);
                        x = fmaf(a4[i].z, b4[jj].z, x);
                        x = fmaf(a4[i].w, b4[jj].w, x);
                        dot[i][jj] = x;
                    }
            }
            __syncthreads();
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t tq = tq0 + ty + 16 * i;
            const float wv = tq < T_q ? wrow[i][j] : 0.f;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) acc[i][jj] = fmaf(wv, fmaxf(dot[i][jj], 0.f), acc[i][jj]);
        }
    }

#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t tq = tq0 + ty + 16 * i;
        if (tq >= T_q) continue;
        const int64_t t = q_row0 + tq;
        float* out = srow0 + tq * T_k;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const int64_t s = s0 + tx + 16 * jj;
            if (s < T_k)
                out[s] = s <= t ? (ly.kscale ? acc[i][jj] * __ldg(ly.kscale + b * ly.ksb + s) : acc[i][jj]) : NEG;
        }
    }
}

// Small heads (HI*DI <= 256): the tile's q rows of every head and its key
// rows are staged once (one barrier), then all heads are computed from
// shared memory.  Same per-(t,s) arithmetic and order as the kernel above.
template <typename T, bool V4>
__global__ void __launch_bounds__(256) indexer_simt_small_kernel(const T* __restrict__ q,
                                                                const T* __restrict__ k,
                                                                const float* __restrict__ w,
                                                                float* __restrict__ scores,
                                                                int64_t T_q, int64_t T_k,
                                                                int64_t q_row0, int HI, int DI,
                                                                int fill_upper, SimtLayout ly) {
    extern __shared__ __align__(16) float sm[];
    // row strides in floats: q rows are read as broadcasts, key rows by 16
    // lanes at once (stride DI+1 spreads them over distinct banks)
    // (V4: float4 reads along d, strides kept multiples of 4)
    const int QS = HI * DI + 4, KS = V4 ? DI + 4 : DI + 1;
    float* qs = sm;                            // [BT][QS]
    float* ks = sm + BT * QS;                  // [BS][KS]
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int64_t b = blockIdx.z;
    const int64_t tq0 = (int64_t)blockIdx.y * BT;
    const int64_t s0 = (int64_t)blockIdx.x * BS;
    const int64_t tq_end = tq0 + BT < T_q ? tq0 + BT : T_q;
    q_row0 += b * ly.row_bstep;
    const int64_t t_max = q_row0 + tq_end - 1;
    float* srow0 = scores + (b * T_q) * T_k;
    const float NEG = -INFINITY;
    if (s0 > t_max) {
        if (fill_upper) {
            for (int e = tid; e < BT * BS; e += 256) {
                const int64_t tq = tq0 + e / BS, s = s0 + e % BS;
                if (tq < T_q && s < T_k) srow0[tq * T_k + s] = NEG;
            }
        }
        return;
    }
    const int HD = HI * DI;
    const T* qb = q + b * ly.qb + tq0 * ly.qr;
    const T* kb = k + b * ly.kb + s0 * ly.kr;
    if (ly.qh == DI && ly.qr == HD) {   // contiguous rows: linear offsets
        for (int e = tid; e < BT * HD; e += 256)
            qs[(e / HD) * QS + e % HD] = tq0 + e / HD < T_q ? Elem<T>::to_f(qb[e]) : 0.f;
    } else if (ly.qh == DI) {   // heads contiguous within a row: one offset per row
        for (int e = tid; e < BT * HD; e += 256) {
            const int r = e / HD, c = e - r * HD;
            qs[r * QS + c] = tq0 + r < T_q ? Elem<T>::to_f(qb[r * ly.qr + c]) : 0.f;
        }
    } else {
        for (int e = tid; e < BT * HD; e += 256) {
            const int r = e / HD, c = e - r * HD;
            const int hh = c / DI, d = c - hh * DI;
            qs[r * QS + c] = tq0 + r < T_q ? Elem<T>::to_f(qb[r * ly.qr + hh * ly.qh + d]) : 0.f;
        }
    }
    for (int e = tid; e < BS * DI; e += 256) {
        const int r = e / DI, c = e - r * DI;
        ks[r * KS + c] = s0 + r < T_k ? Elem<T>::to_f(kb[ly.kr == DI ? (int64_t)e : r * ly.kr + c]) : 0.f;
    }
    __syncthreads();

    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) acc[i][jj] = 0.f;
    const float* wrow[4];   // head weights of this thread's four query rows
#pragma unroll
    for (int i = 0; i < 4; ++i) wrow[i] = w + b * ly.wb + (tq0 + ty + 16 * i) * ly.wr;
    for (int j = 0; j < HI; ++j) {
        float dot[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) dot[i][jj] = 0.f;
        if constexpr (V4) {
            for (int d = 0; d < DI; d += 4) {
                float4 a4[4], b4[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    a4[i] = *reinterpret_cast<const float4*>(&qs[(ty + 16 * i) * QS + j * DI + d]);
                    b4[i] = *reinterpret_cast<const float4*>(&ks[(tx + 16 * i) * KS + d]);
                }
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) {
                        float x = dot[i][jj];
                        x = fmaf(a4[i].x, b4[jj].x, x);
                        x = fmaf(a4[i].y, b4[jj].y, x);
                        x = fmaf(a4[i].z, b4[jj].z, x);
                        x = fmaf(a4[i].w, b4[jj].w, x);
                        dot[i][jj] = x;
                    }
            }
        } else {
            for (int d = 0; d < DI; ++d) {
                float av[4], bv[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    av[i] = qs[(ty + 16 * i) * QS + j * DI + d];
                    bv[i] = ks[(tx + 16 * i) * KS + d];
                }
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) dot[i][jj] = fmaf(av[i], bv[jj], dot[i][jj]);
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int64_t tq = tq0 + ty + 16 * i;
            const float wv = tq < T_q ? wrow[i][j] : 0.f;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) acc[i][jj] = fmaf(wv, fmaxf(dot[i][jj], 0.f), acc[i][jj]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t tq = tq0 + ty + 16 * i;
        if (tq >= T_q) continue;
        const int64_t t = q_row0 + tq;
        float* out = srow0 + tq * T_k;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const int64_t s = s0 + tx + 16 * jj;
            if (s < T_k)
                out[s] = s <= t ? (ly.kscale ? acc[i][jj] * __ldg(ly.kscale + b * ly.ksb + s) : acc[i][jj]) : NEG;
        }
    }
}

template <typename T>
int launch(const void* q, const void* k, const float* w, float* scores, int64_t B, int64_t T_q,
           int64_t T_k, int64_t q_row0, int64_t HI, int64_t DI, int fill_upper,
           const SimtLayout& ly, cudaStream_t stream) {
    const int64_t gx = (T_k + BS - 1) / BS, gy = (T_q + BT - 1) / BT;
    if (gx > INT32_MAX || gy > 65535 || B > 65535)
        return fail(DSA_ERR_INVALID, "indexer: grid too large (T_q/64 and B must be <= 65535)");
    dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)B);
    if (HI * DI <= 256 && !getenv("DSA_INDEXER_SIMT_GENERIC")) {
        const bool v4 = DI % 4 == 0;
        const size_t smem = ((size_t)BT * (HI * DI + 4) + (size_t)BS * (DI + (v4 ? 4 : 1))) * sizeof(float);
        auto kern = v4 ? indexer_simt_small_kernel<T, true> : indexer_simt_small_kernel<T, false>;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
            return fail(DSA_ERR_CUDA, "indexer: cannot set dynamic shared memory size");
        kern<<<grid, 256, smem, stream>>>((const T*)q, (const T*)k, w, scores, T_q, T_k, q_row0, (int)HI,
                                          (int)DI, fill_upper, ly);
        return check_launch("indexer_simt_small_kernel");
    }
    indexer_simt_kernel<T><<<grid, 256, 0, stream>>>((const T*)q, (const T*)k, w, scores, T_q, T_k,
                                                     q_row0, (int)HI, (int)DI, fill_upper, ly);
    return check_launch("indexer_simt_kernel");
}

}  // namespace

int indexer_scores_simt(const void* q, const void* k, const float* w, float* scores, int64_t B,
                        int64_t T_q, int64_t T_k, int64_t q_row0, int64_t HI, int64_t DI,
                        int dtype, int fill_upper, const dsa_layout& L, const float* kscale,
                        cudaStream_t stream) {
    const SimtLayout ly{L.q[0], L.q[1], L.q[2], L.k[0], L.k[1], L.w[0], L.w[1], L.row_bstep, kscale,
                        L.k[0] == 0 ? 0 : T_k};
    switch (dtype) {
        case DSA_F32:
            return launch<float>(q, k, w, scores, B, T_q, T_k, q_row0, HI, DI, fill_upper, ly, stream);
        case DSA_BF16:
            return launch<__nv_bfloat16>(q, k, w, scores, B, T_q, T_k, q_row0, HI, DI, fill_upper, ly,
                                         stream);
        case DSA_FP8_E4M3:
            return launch<__nv_fp8_e4m3>(q, k, w, scores, B, T_q, T_k, q_row0, HI, DI, fill_upper, ly,
                                         stream);
        default:
            return launch<__half>(q, k, w, scores, B, T_q, T_k, q_row0, HI, DI, fill_upper, ly, stream);
    }
}

DSA_DEBUG_FLAGS_READER(indexer_simt)

}  // namespace dsa
