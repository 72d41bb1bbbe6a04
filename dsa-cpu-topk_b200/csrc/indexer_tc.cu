// Stage 1 (tensor-core path): tcgen05 / TMEM Lightning Indexer for bf16 or
// FP8 (e4m3) inputs.
//
//   I[b,t,s] = sum_j w[b,t,j] * ReLU(<q[b,t,j,:], k[b,s,:]>),  s <= t
//
// The reference computes this with an IEEE-fp32 tl.dot per head on CUDA
// cores (lightning_indexer.py:83-90).  Here each head's dot products are one
// bf16 (kind::f16) or e4m3 (kind::f8f6f4, the FP8 indexer of the DeepSeek-V3.2
// paper) GEMM on the 5th-generation tensor cores with fp32 accumulation in
// tensor memory, and the ReLU * w[t,j] head reduction runs in the epilogue.
// Products of e4m3 (or bf16) values are exact in fp32, so both are faithful
// to the reference's fp32 arithmetic on the same inputs.
//
// Persistent, warp-specialised, one CTA per SM:
//   warp 0        TMA producer: per tile one key block k[s0:s0+256, :] (B operand),
//                 then per head j the query block q[t0:t0+128, j, :] (A operand),
//                 both 128-byte swizzled, through mbarrier rings
//   warp 1        MMA issuer (one thread): per head, DI/16 tcgen05.mma
//                 (M=128, N=256, K=16) into one of two TMEM accumulators
//                 (2 x 256 columns), committed to the epilogue's barrier
//   warps 2..9    epilogue: tcgen05.ld of the head's 128x256 fp32 tile (each
//                 thread one query row, 128 columns), acc += w[t,j]*max(x,0)
//                 in registers; after the last head the causal mask is applied
//                 and the tile is stored to the fp32 score matrix
// Tiles are the causal (query block, key block) pairs, dealt round-robin to
// the CTAs; all warps walk the same sequence.  Every mbarrier wait is
// bounded (2 s of device time): on timeout the CTA's warps leave their loops,
// TMEM is freed, and a device flag records it for dsa_device_status().
#include <cuda.h>
#include <math.h>
#include <stdlib.h>

#include "common.cuh"
#include "tc_ptx.cuh"

namespace dsa {

__device__ int g_indexer_tc_timeout = 0;

namespace {

using namespace tc;

constexpr int BM = 128;            // query rows per tile (TMEM lanes)
constexpr int BN = 256;            // keys per tile (MMA N, TMEM columns per accumulator)
constexpr int ROWB = 128;          // bytes per swizzle row (one K chunk): 64 bf16 or 128 e4m3
constexpr int EPI_WARPS = 8;
constexpr int NTHREADS = 64 + EPI_WARPS * 32;
constexpr int MAX_TBLK = 1024;     // query blocks per batch (T_q <= 131072)
constexpr uint32_t TMEM_COLS = 512;
constexpr int CHUNK = 16;                          // score columns per TMA store (64 bytes)
constexpr int STAGE_BYTES = 2 * 32 * CHUNK * 4;    // two 32-row chunk buffers per epilogue warp

struct TcParams {
    float* scores;
    const float* w;
    int64_t T_q, T_k, q_row0;
    int64_t row_bstep;          // batch b's rows start at q_row0 + b*row_bstep
    int64_t wb, wr;             // element strides of w (batch, row)
    int HI, DI, B;
    int flat;                   // tile prefix over (batch, query block) pairs (row blocks differ per batch)
    int kshared;                // k has batch stride 0: every batch reads batch 0's keys
    const float* kscale;        // per-key scales [B (1 if kshared), T_k] multiplying the scores, or null
    int n_tblk, nsb, tiles_per_batch, total_tiles;
    int nA, nB;
    uint32_t a_bytes, b_bytes;
    int vec_store;
    int vec8_store;             // rows 32-byte aligned: 256-bit score stores
    int tma_store;              // rows 16-byte aligned: staged TMA tensor stores of the scores
    int elt;                    // bytes per q/k element: 2 (bf16) or 1 (e4m3)
    int stall;                  // test hook: the producer issues no loads, so every wait times out
    unsigned long long timeout_ns;
};

// tile index -> (batch, query block, key block) through the prefix of key
// blocks per query block: per batch when every batch has the same rows,
// else over all (batch, query block) pairs
template <bool FLAT>
__device__ __forceinline__ void decode_tile(int lin, const int* pref, const TcParams& p, int& b,
                                            int& i, int& j) {
    if constexpr (FLAT) {
        int lo = 0, hi = p.B * p.n_tblk - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (pref[mid] <= lin) lo = mid;
            else hi = mid - 1;
        }
        j = lin - pref[lo];
        b = lo / p.n_tblk;
        i = lo - b * p.n_tblk;
    } else {
        b = lin / p.tiles_per_batch;
        const int r = lin - b * p.tiles_per_batch;
        int lo = 0, hi = p.n_tblk - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (pref[mid] <= r) lo = mid;
            else hi = mid - 1;
        }
        i = lo;
        j = r - pref[lo];
    }
    DSA_CHECK(b < p.B && i < p.n_tblk && j < p.nsb, DBG_TILE);   // flagged only: the walk stays as it is
}

template <bool FP8, bool FLAT>
__global__ void __launch_bounds__(NTHREADS, 1)
    indexer_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                      const __grid_constant__ CUtensorMap tms, const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ int pref[MAX_TBLK + 1];
    __shared__ uint32_t tmem_slot;
    __shared__ int s_abort;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = sA + (size_t)p.nA * p.a_bytes;
    uint8_t* sStage = sB + (size_t)p.nB * p.b_bytes;  // STAGE_BYTES per epilogue warp if tma_store
    uint64_t* fullA = reinterpret_cast<uint64_t*>(sStage + (p.tma_store ? EPI_WARPS * STAGE_BYTES : 0));
    uint64_t* emptyA = fullA + p.nA;
    uint64_t* fullB = emptyA + p.nA;
    uint64_t* emptyB = fullB + p.nB;
    uint64_t* tfull = emptyB + p.nB;
    uint64_t* tempty = tfull + 2;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nch = p.DI * p.elt / ROWB;   // 128-byte K chunks per row
    const int kch = ROWB / p.elt;          // elements per chunk (TMA x step)

    if (threadIdx.x == 0) {
        int acc = 0;
        const int nb = FLAT ? p.B : 1;
        for (int x = 0; x < nb * p.n_tblk; ++x) {
            const int bb = x / p.n_tblk, i = x - bb * p.n_tblk;
            pref[x] = acc;
            int64_t tq_end = (int64_t)(i + 1) * BM;
            if (tq_end > p.T_q) tq_end = p.T_q;
            const int64_t t_max = p.q_row0 + bb * p.row_bstep + tq_end - 1;
            int64_t c = t_max / BN + 1;
            if (c > p.nsb) c = p.nsb;
            acc += (int)c;
        }
        pref[nb * p.n_tblk] = acc;
    }
    if (threadIdx.x == 32) {
        s_abort = 0;
        for (int s = 0; s < p.nA; ++s) {
            mbar_init(&fullA[s], 1);
            mbar_init(&emptyA[s], 1);
        }
        for (int s = 0; s < p.nB; ++s) {
            mbar_init(&fullB[s], 1);
            mbar_init(&emptyB[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&tfull[s], 1);
            mbar_init(&tempty[s], EPI_WARPS);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&tmem_slot)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int as = 0, bs = 0;
            uint32_t aph = 0, bph = 0;
            bool ok = true;
            for (int lin = blockIdx.x; ok && lin < p.total_tiles; lin += gridDim.x) {
                int b, i, j;
                decode_tile<FLAT>(lin, pref, p, b, i, j);
                if (!(ok = mbar_wait(&emptyB[bs], bph ^ 1, &s_abort, p.timeout_ns, &g_indexer_tc_timeout))) break;
                if (!p.stall) mbar_expect_tx(&fullB[bs], p.b_bytes);
                for (int c = 0; c < nch && !p.stall; ++c)
                    tma_load_3d(sB + (size_t)bs * p.b_bytes + (size_t)c * BN * 128, &tmk, &fullB[bs],
                                c * kch, j * BN, p.kshared ? 0 : b);
                if (++bs == p.nB) { bs = 0; bph ^= 1; }
                for (int h = 0; h < p.HI; ++h) {
                    if (!(ok = mbar_wait(&emptyA[as], aph ^ 1, &s_abort, p.timeout_ns, &g_indexer_tc_timeout))) break;
                    if (!p.stall) mbar_expect_tx(&fullA[as], p.a_bytes);
                    for (int c = 0; c < nch && !p.stall; ++c)
                        tma_load_4d(sA + (size_t)as * p.a_bytes + (size_t)c * BM * 128, &tmq,
                                    &fullA[as], c * kch, h, i * BM, b);
                    if (++as == p.nA) { as = 0; aph ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            // D fp32 (bit 4); A/B formats at bits 7-9 / 10-12 (kind::f16: 1 = bf16;
            // kind::f8f6f4: 0 = e4m3); both K-major, N>>3 at bit 17, M>>4 at bit 24
            const uint32_t fmt = FP8 ? 0u : 1u;
            const uint32_t idesc = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(BN >> 3) << 17) |
                                   ((uint32_t)(BM >> 4) << 24);
            int as = 0, bs = 0, tb = 0;
            uint32_t aph = 0, bph = 0, tph = 0;
            bool ok = true;
            for (int lin = blockIdx.x; ok && lin < p.total_tiles; lin += gridDim.x) {
                if (!(ok = mbar_wait(&fullB[bs], bph, &s_abort, p.timeout_ns, &g_indexer_tc_timeout))) break;
                const uint32_t bbase = smem_u32(sB + (size_t)bs * p.b_bytes);
                for (int h = 0; h < p.HI; ++h) {
                    if (!(ok = mbar_wait(&fullA[as], aph, &s_abort, p.timeout_ns, &g_indexer_tc_timeout))) break;
                    if (!(ok = mbar_wait(&tempty[tb], tph ^ 1, &s_abort, p.timeout_ns, &g_indexer_tc_timeout))) break;
                    tc_fence_after();
                    const uint32_t abase = smem_u32(sA + (size_t)as * p.a_bytes);
                    const uint32_t d = tmem_base + (uint32_t)(tb * BN);
                    for (int c = 0; c < nch; ++c) {
#pragma unroll
                        for (int kk = 0; kk < ROWB / 32; ++kk) {
                            const uint64_t ad = sw128_desc(abase + c * BM * 128 + kk * 32);
                            const uint64_t bd = sw128_desc(bbase + c * BN * 128 + kk * 32);
                            umma<FP8>(d, ad, bd, idesc, (c | kk) != 0);
                        }
                    }
                    umma_commit(&emptyA[as]);
                    umma_commit(&tfull[tb]);
                    if (++as == p.nA) { as = 0; aph ^= 1; }
                    if (++tb == 2) { tb = 0; tph ^= 1; }
                }
                umma_commit(&emptyB[bs]);
                if (++bs == p.nB) { bs = 0; bph ^= 1; }
            }
        }
    } else {
        // ---------------- epilogue ----------------
        const int ew = warp - 2;
        const int quarter = warp & 3;       // TMEM lanes this warp may read
        const int half = ew >> 2;           // which 128 of the 256 columns
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        int tb = 0;
        uint32_t tph = 0;
        uint32_t nstore = 0;   // TMA stores issued by this warp (buffer = nstore & 1)
        uint8_t* stage = sStage + ew * STAGE_BYTES;
        bool ok = true;
        for (int lin = blockIdx.x; ok && lin < p.total_tiles; lin += gridDim.x) {
            int b, i, j;
            decode_tile<FLAT>(lin, pref, p, b, i, j);
            const int64_t tq = (int64_t)i * BM + row;
            const bool row_ok = tq < p.T_q;
            const float* wrow = p.w + (int64_t)b * p.wb + (row_ok ? tq : 0) * p.wr;
            float acc[128];
#pragma unroll
            for (int c = 0; c < 128; ++c) acc[c] = 0.f;
            // head weights prefetched two heads ahead (one global-load latency
            // is about one head's worth of work at DI=64)
            float wpre[2];
            wpre[0] = row_ok ? __ldg(wrow) : 0.f;
            wpre[1] = (row_ok && p.HI > 1) ? __ldg(wrow + 1) : 0.f;
            for (int h0 = 0; h0 < p.HI && ok; h0 += 2) {
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int h = h0 + u;
                    if (h >= p.HI) break;
                    const float wj = wpre[u];
                    wpre[u] = (row_ok && h + 2 < p.HI) ? __ldg(wrow + h + 2) : 0.f;
                    if (!(ok = mbar_wait(&tfull[tb], tph, &s_abort, p.timeout_ns, &g_indexer_tc_timeout))) break;
                    tc_fence_after();
                    const uint32_t taddr = tmem_base + lane_off + (uint32_t)(tb * BN + half * 128);
                    // 16-column chunks, the next chunk's load in flight while the
                    // current one is folded in
                    uint32_t rb[2][16];
                    tmem_ld16(taddr, rb[0]);
                    tmem_wait_ld(rb[0]);
#pragma unroll
                    for (int ch = 0; ch < 8; ++ch) {
                        if (ch + 1 < 8) tmem_ld16(taddr + (ch + 1) * 16, rb[(ch + 1) & 1]);
#pragma unroll
                        for (int e = 0; e < 16; ++e)
                            acc[ch * 16 + e] =
                                fmaf(wj, fmaxf(__uint_as_float(rb[ch & 1][e]), 0.f), acc[ch * 16 + e]);
                        if (ch + 1 < 8) tmem_wait_ld(rb[(ch + 1) & 1]);
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[tb]);
                    if (++tb == 2) { tb = 0; tph ^= 1; }
                }
            }
            const int64_t t = p.q_row0 + b * p.row_bstep + tq;
            const int64_t s0 = (int64_t)j * BN + half * 128;
            const float NEG = -INFINITY;
            if (FP8 && p.kscale) {   // compiled out of the bf16 kernel
                // FP8 keys quantised per row: I[t,s] = k_scale[s] * sum_j w_j ReLU(<q_j, k8_s>)
                const float* ks = p.kscale + (p.kshared ? 0 : (int64_t)b * p.T_k);
#pragma unroll
                for (int c = 0; c < 128; ++c)
                    acc[c] *= s0 + c < p.T_k ? __ldg(ks + s0 + c) : 0.f;
            }
            if (p.tma_store) {
                // Each 32-row x 16-column chunk is written to a shared buffer
                // (64-byte swizzle: 16-byte unit u of row r sits at unit
                // u ^ ((r >> 1) & 3), so a quarter-warp's 16-byte writes hit
                // distinct banks) and stored by one TMA tensor store; rows
                // past T_q and columns past T_k are clipped by the tensor map.
                if (!__all_sync(0xffffffffu, ok)) { ok = false; continue; }
#pragma unroll
                for (int ch = 0; ch < 128 / CHUNK; ++ch) {
                    uint8_t* buf = stage + (nstore & 1) * (32 * CHUNK * 4);
                    if (lane == 0) bulk_wait_read<1>();   // this buffer's previous store has read it
                    __syncwarp();
                    const int64_t c0 = s0 + ch * CHUNK;
#pragma unroll
                    for (int u = 0; u < CHUNK / 4; ++u) {
                        float4 v;
                        v.x = (c0 + u * 4 + 0 <= t) ? acc[ch * CHUNK + u * 4 + 0] : NEG;
                        v.y = (c0 + u * 4 + 1 <= t) ? acc[ch * CHUNK + u * 4 + 1] : NEG;
                        v.z = (c0 + u * 4 + 2 <= t) ? acc[ch * CHUNK + u * 4 + 2] : NEG;
                        v.w = (c0 + u * 4 + 3 <= t) ? acc[ch * CHUNK + u * 4 + 3] : NEG;
                        *reinterpret_cast<float4*>(buf + lane * 64 + ((u ^ ((lane >> 1) & 3)) << 4)) = v;
                    }
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_3d(&tms, buf, (int)c0, i * BM + quarter * 32, b);
                        bulk_commit();
                    }
                    ++nstore;
                }
                continue;
            }
            if (!ok || !row_ok) continue;
            float* out = p.scores + ((int64_t)b * p.T_q + tq) * p.T_k + s0;
            if (p.vec8_store && s0 + 128 <= p.T_k) {
                // 32-byte stores: each warp store writes whole sectors of its 32 rows
#pragma unroll
                for (int c = 0; c < 128; c += 8) {
                    float v[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[e] = (s0 + c + e <= t) ? acc[c + e] : NEG;
                    asm volatile("st.global.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(out + c),
                                 "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]),
                                 "f"(v[7])
                                 : "memory");
                }
            } else if (p.vec_store && s0 + 128 <= p.T_k) {
#pragma unroll
                for (int c = 0; c < 128; c += 4) {
                    float4 v;
                    v.x = (s0 + c + 0 <= t) ? acc[c + 0] : NEG;
                    v.y = (s0 + c + 1 <= t) ? acc[c + 1] : NEG;
                    v.z = (s0 + c + 2 <= t) ? acc[c + 2] : NEG;
                    v.w = (s0 + c + 3 <= t) ? acc[c + 3] : NEG;
                    *reinterpret_cast<float4*>(out + c) = v;
                }
            } else {
#pragma unroll
                for (int c = 0; c < 128; ++c)
                    if (s0 + c < p.T_k) out[c] = (s0 + c <= t) ? acc[c] : NEG;
            }
        }
        if (p.tma_store && lane == 0) bulk_wait_all();   // staging buffers stay live until stored
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                     "r"(TMEM_COLS)
                     : "memory");
    }
}

// -inf for every s > t (the full-matrix contract of the score output)
__global__ void fill_upper_kernel(float* scores, int64_t T_q, int64_t T_k, int64_t q_row0,
                                  int64_t row_bstep) {
    const int64_t row = blockIdx.x;  // b * T_q + tq
    const int64_t t = q_row0 + (row / T_q) * row_bstep + row % T_q;
    float* out = scores + row * T_k;
    for (int64_t s = t + 1 + threadIdx.x; s < T_k; s += blockDim.x) out[s] = -INFINITY;
}

}  // namespace

// Synchronises `stream`, reads and clears the timeout flag of this device.
// Returns 1 if a tensor-core indexer launch gave up on a wait, 0 if not,
// negative on a CUDA error.
int indexer_tc_take_timeout(cudaStream_t stream) {
    if (cudaStreamSynchronize(stream) != cudaSuccess) return -1;
    int flag = 0;
    if (cudaMemcpyFromSymbol(&flag, g_indexer_tc_timeout, sizeof(int)) != cudaSuccess) return -1;
    if (flag) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_indexer_tc_timeout, &zero, sizeof(int)) != cudaSuccess) return -1;
    }
    return flag ? 1 : 0;
}

bool indexer_tc_supported(int64_t HI, int64_t DI, int dtype) {
    if (HI < 1 || HI > 4096) return false;
    if (dtype == DSA_BF16) return DI == 64 || DI == 128;
    if (dtype == DSA_FP8_E4M3) return DI == 128 || DI == 256;
    return false;
}

static int encode_map(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims,
                      const cuuint64_t* strides, const cuuint32_t* box, const char* what, int elt) {
    return tc::encode_map(m, base, rank, dims, strides, box, std::string("indexer_tc: ") + what,
                          elt == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
}

int indexer_scores_tc(const void* q, const void* k, const float* w, float* scores, int64_t B,
                      int64_t T_q, int64_t T_k, int64_t q_row0, int64_t HI, int64_t DI,
                      int fill_upper, int dtype, const dsa_layout& L, const float* kscale,
                      cudaStream_t stream) {
    TcParams p;
    p.kscale = kscale;
    p.elt = dtype == DSA_FP8_E4M3 ? 1 : 2;
    // tensor-map strides: positive multiples of 16 bytes (a batch stride of 0
    // on k is read as one shared batch)
    if (!tma_stride_ok(L.q[2], p.elt) || !tma_stride_ok(L.q[1], p.elt) ||
        (B > 1 && !tma_stride_ok(L.q[0], p.elt)) || !tma_stride_ok(L.k[1], p.elt) ||
        (B > 1 && L.k[0] != 0 && !tma_stride_ok(L.k[0], p.elt)))
        return -100;
    p.kshared = (B > 1 && L.k[0] == 0) ? 1 : 0;
    p.row_bstep = L.row_bstep;
    p.wb = L.w[0];
    p.wr = L.w[1];
    const bool fp8 = p.elt == 1;
    const bool flat = L.row_bstep != 0;
    auto kern = fp8 ? (flat ? indexer_tc_kernel<true, true> : indexer_tc_kernel<true, false>)
                    : (flat ? indexer_tc_kernel<false, true> : indexer_tc_kernel<false, false>);
    p.scores = scores;
    p.w = w;
    p.T_q = T_q;
    p.T_k = T_k;
    p.q_row0 = q_row0;
    p.HI = (int)HI;
    p.DI = (int)DI;
    p.B = (int)B;
    p.n_tblk = (int)((T_q + BM - 1) / BM);
    p.nsb = (int)((T_k + BN - 1) / BN);
    if (p.n_tblk > MAX_TBLK) return -100;  // caller falls back to the CUDA-core kernel
    // batches whose rows start at different positions need the prefix over
    // every (batch, query block); the caller splits larger calls per batch
    p.flat = L.row_bstep != 0 ? 1 : 0;
    if (p.flat && B * p.n_tblk > MAX_TBLK) return -101;
    int64_t total = 0, per_batch = 0;
    for (int64_t bb = 0; bb < (p.flat ? B : 1); ++bb) {
        per_batch = 0;
        for (int i = 0; i < p.n_tblk; ++i) {
            int64_t tq_end = (int64_t)(i + 1) * BM;
            if (tq_end > T_q) tq_end = T_q;
            int64_t c = (q_row0 + bb * L.row_bstep + tq_end - 1) / BN + 1;
            if (c > p.nsb) c = p.nsb;
            per_batch += c;
        }
        total += per_batch;
    }
    if (!p.flat) total = per_batch * B;
    if (total > INT32_MAX) return -100;
    p.tiles_per_batch = (int)per_batch;
    p.total_tiles = (int)total;
    p.a_bytes = (uint32_t)(BM * DI * p.elt);
    p.b_bytes = (uint32_t)(BN * DI * p.elt);
    p.vec_store = (T_k % 4 == 0) ? 1 : 0;
    p.vec8_store = (T_k % 8 == 0 && (reinterpret_cast<uintptr_t>(scores) & 31u) == 0) ? 1 : 0;
    // DSA_INDEXER_DIRECT_STORE=1: per-thread global stores instead of TMA stores
    p.tma_store = (T_k % 4 == 0 && (reinterpret_cast<uintptr_t>(scores) & 15u) == 0 &&
                   !getenv("DSA_INDEXER_DIRECT_STORE"))
                      ? 1
                      : 0;
    // DSA_TEST_INDEXER_STALL=1: test hook for the timeout path (no loads are
    // issued, every wait runs out after 20 ms); never set in normal use
    p.stall = getenv("DSA_TEST_INDEXER_STALL") ? 1 : 0;
    p.timeout_ns = p.stall ? 20000000ull : 2000000000ull;  // 2 s of device time otherwise

    // shared memory: the device's opt-in limit minus the kernel's static
    // shared memory; 1 KB alignment slack + rings + barriers
    int dev = 0, optin = 0;
    cudaFuncAttributes fa;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
        cudaFuncGetAttributes(&fa, kern) != cudaSuccess)
        return fail(DSA_ERR_CUDA, "indexer_tc: cannot query shared memory limits");
    const size_t kMaxSmem = (size_t)optin - fa.sharedSizeBytes;
    const size_t fixed = 1024 + 256;
    const char* env_nb = getenv("DSA_TC_NB");  // ring depth of the key operand (1 or 2)
    p.nB = (env_nb && env_nb[0] == '1') ? 1 : 2;
    // the staging buffers take 32 KB; the A ring gives up a stage for them
    // (two A stages keep the tensor pipe as busy as three)
    size_t stage = p.tma_store ? (size_t)EPI_WARPS * STAGE_BYTES : 0;
    if (stage && kMaxSmem < fixed + stage + (size_t)p.nB * p.b_bytes + 2 * (size_t)p.a_bytes) {
        p.tma_store = 0;
        stage = 0;
    }
    if (kMaxSmem < fixed + stage + (size_t)p.nB * p.b_bytes + 2 * (size_t)p.a_bytes) p.nB = 1;
    p.nA = (int)((kMaxSmem - fixed - stage - (size_t)p.nB * p.b_bytes) / p.a_bytes);
    if (p.nA > 8) p.nA = 8;
    if (p.nA < 2) return -100;
    const size_t smem = fixed + stage + (size_t)p.nA * p.a_bytes + (size_t)p.nB * p.b_bytes;

    if (fill_upper) {
        fill_upper_kernel<<<(unsigned)(B * T_q), 256, 0, stream>>>(scores, T_q, T_k, q_row0, L.row_bstep);
        int rc = check_launch("fill_upper_kernel");
        if (rc) return rc;
    }
    if (p.total_tiles == 0) return DSA_OK;

    CUtensorMap tmq, tmk, tms;
    {
        const cuuint64_t dims[4] = {(cuuint64_t)DI, (cuuint64_t)HI, (cuuint64_t)T_q, (cuuint64_t)B};
        const cuuint64_t e = (cuuint64_t)p.elt;
        const cuuint64_t str[3] = {(cuuint64_t)L.q[2] * e, (cuuint64_t)L.q[1] * e,
                                   (cuuint64_t)(B > 1 ? L.q[0] : L.q[1] * T_q) * e};
        const cuuint32_t box[4] = {(cuuint32_t)(ROWB / p.elt), 1, BM, 1};
        int rc = encode_map(&tmq, q, 4, dims, str, box, "q", p.elt);
        if (rc) return rc;
    }
    {
        const cuuint64_t dims[3] = {(cuuint64_t)DI, (cuuint64_t)T_k, (cuuint64_t)(p.kshared ? 1 : B)};
        const cuuint64_t e = (cuuint64_t)p.elt;
        const cuuint64_t str[2] = {(cuuint64_t)L.k[1] * e,
                                   (cuuint64_t)(B > 1 && !p.kshared ? L.k[0] : L.k[1] * T_k) * e};
        const cuuint32_t box[3] = {(cuuint32_t)(ROWB / p.elt), BN, 1};
        int rc = encode_map(&tmk, k, 3, dims, str, box, "k", p.elt);
        if (rc) return rc;
    }
    if (p.tma_store) {
        // scores [B, T_q, T_k] fp32, box 16 columns x 32 rows, 64-byte swizzle
        const cuuint64_t dims[3] = {(cuuint64_t)T_k, (cuuint64_t)T_q, (cuuint64_t)B};
        const cuuint64_t str[2] = {(cuuint64_t)T_k * 4, (cuuint64_t)T_q * T_k * 4};
        const cuuint32_t box[3] = {(cuuint32_t)CHUNK, 32, 1};
        int rc = tc::encode_map(&tms, scores, 3, dims, str, box, "indexer_tc: scores",
                                CU_TENSOR_MAP_DATA_TYPE_FLOAT32, CU_TENSOR_MAP_SWIZZLE_64B);
        if (rc) return rc;
    } else {
        tms = tmk;  // unused
    }
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return fail(DSA_ERR_CUDA, "indexer_tc: cannot set dynamic shared memory size");
    int grid = num_sms();
    if (grid > p.total_tiles) grid = p.total_tiles;
    kern<<<grid, NTHREADS, smem, stream>>>(tmq, tmk, tms, p);
    return check_launch("indexer_tc_kernel");
}

DSA_DEBUG_FLAGS_READER(indexer_tc)

}  // namespace dsa
